"""Chakra execution-trace (.et) encoding and decoding, dependency-free.

A .et file is a stream of length-delimited protobuf messages: one GlobalMetadata, then one
Node per operator. Field numbers follow the public MLCommons Chakra schema (et_def.proto);
attribute names and kinds are the ones ASTRA-sim's feeder reads (is_cpu_op, num_ops,
tensor_size, comm_type, comm_size, pg_name, comm_src, comm_dst, comm_tag). Reference:
workload_export/chakra_writer.py.
"""
from __future__ import annotations

import struct

# Node.type (NodeType)
METADATA_NODE, MEM_LOAD_NODE, MEM_STORE_NODE, COMP_NODE, COMM_SEND_NODE, COMM_RECV_NODE, COMM_COLL_NODE = range(1, 8)
# CollectiveCommType
ALL_REDUCE, REDUCE, ALL_GATHER, GATHER, SCATTER, BROADCAST, ALL_TO_ALL, REDUCE_SCATTER = range(8)
COLL_NAMES = {ALL_REDUCE: "ALL_REDUCE", ALL_GATHER: "ALL_GATHER", REDUCE_SCATTER: "REDUCE_SCATTER"}
SCHEMA_VERSION = "0.0.4"

# Node fields
F_ID, F_NAME, F_TYPE, F_CTRL, F_DATA, F_START, F_DUR, F_IN, F_OUT, F_ATTR = range(1, 11)
# AttributeProto value fields: kind -> (field number, wire type)
ATTR_KINDS = {"double_val": (3, 1), "int32_val": (7, 0), "int64_val": (9, 0), "uint64_val": (13, 0),
              "bool_val": (27, 0), "string_val": (29, 2)}
_BY_FIELD = {v[0]: k for k, v in ATTR_KINDS.items()}


class _Buf:
    """Minimal protobuf wire writer."""

    def __init__(self):
        self.b = bytearray()

    @staticmethod
    def varint(n: int) -> bytes:
        if n < 0:
            n += 1 << 64
        out = bytearray()
        while True:
            lo = n & 0x7F
            n >>= 7
            out.append(lo | (0x80 if n else 0))
            if not n:
                return bytes(out)

    def tag(self, field, wire):
        self.b += self.varint((field << 3) | wire)
        return self

    def uint(self, field, v):
        self.tag(field, 0).b += self.varint(int(v))
        return self

    def blob(self, field, payload: bytes):
        self.tag(field, 2).b += self.varint(len(payload)) + payload
        return self

    def text(self, field, s: str):
        return self.blob(field, s.encode())

    def double(self, field, v):
        self.tag(field, 1).b += struct.pack("<d", float(v))
        return self


def _attr_bytes(name, kind, value) -> bytes:
    w = _Buf().text(1, name)
    field, wire = ATTR_KINDS[kind]
    if wire == 0:
        w.uint(field, (1 if value else 0) if kind == "bool_val" else int(value))
    elif wire == 1:
        w.double(field, value)
    else:
        w.text(field, str(value))
    return bytes(w.b)


def encode_node(n: dict) -> bytes:
    w = _Buf().uint(F_ID, n["id"]).text(F_NAME, n["name"]).uint(F_TYPE, n["type"])
    for field, deps in ((F_CTRL, n.get("ctrl_deps", ())), (F_DATA, n.get("data_deps", ()))):
        if deps:
            w.blob(field, b"".join(_Buf.varint(d) for d in deps))
    if n.get("duration_micros"):
        w.uint(F_DUR, n["duration_micros"])
    for field, key in ((F_IN, "inputs"), (F_OUT, "outputs")):
        io = n.get(key)
        if io:
            sub = _Buf()
            for i, k in ((1, "values"), (2, "shapes"), (3, "types")):
                if io.get(k):
                    sub.text(i, io[k])
            w.blob(field, bytes(sub.b))
    for name, kind, value in n.get("attrs", ()):
        w.blob(F_ATTR, _attr_bytes(name, kind, value))
    return bytes(w.b)


def encode_metadata(attrs=()) -> bytes:
    w = _Buf().text(1, SCHEMA_VERSION)
    for name, kind, value in attrs:
        w.blob(2, _attr_bytes(name, kind, value))
    return bytes(w.b)


def write_et(path, nodes, metadata_attrs=()):
    with open(path, "wb") as f:
        for msg in [encode_metadata(metadata_attrs)] + [encode_node(n) for n in nodes]:
            f.write(_Buf.varint(len(msg)))
            f.write(msg)


# ---------------------------------------------------------------- reader
def _uvarint(buf, i):
    shift = out = 0
    while True:
        c = buf[i]
        i += 1
        out |= (c & 0x7F) << shift
        if c < 0x80:
            return out, i
        shift += 7


def _fields(buf):
    i = 0
    while i < len(buf):
        key, i = _uvarint(buf, i)
        field, wire = key >> 3, key & 7
        if wire == 0:
            v, i = _uvarint(buf, i)
        elif wire == 1:
            v = struct.unpack_from("<d", buf, i)[0]
            i += 8
        elif wire == 2:
            ln, i = _uvarint(buf, i)
            v = bytes(buf[i:i + ln])
            i += ln
        elif wire == 5:
            v = struct.unpack_from("<f", buf, i)[0]
            i += 4
        else:
            raise ValueError(f"unsupported wire type {wire}")
        yield field, wire, v


def _signed(v):
    return v - (1 << 64) if v >= 1 << 63 else v


def _decode_attr(b):
    name, kind, value = None, None, None
    for field, wire, v in _fields(b):
        if field == 1:
            name = v.decode()
        elif field in _BY_FIELD:
            kind = _BY_FIELD[field]
            value = (bool(v) if kind == "bool_val" else v.decode() if kind == "string_val"
                     else _signed(v) if kind in ("int32_val", "int64_val") else v)
    return name, kind, value


def decode_node(b) -> dict:
    n = {"ctrl_deps": [], "data_deps": [], "attrs": [], "inputs": {}, "outputs": {}}
    for field, wire, v in _fields(b):
        if field == F_ID:
            n["id"] = v
        elif field == F_NAME:
            n["name"] = v.decode()
        elif field == F_TYPE:
            n["type"] = v
        elif field in (F_CTRL, F_DATA):
            key = "ctrl_deps" if field == F_CTRL else "data_deps"
            if wire == 2:
                j = 0
                while j < len(v):
                    d, j = _uvarint(v, j)
                    n[key].append(d)
            else:
                n[key].append(v)
        elif field == F_DUR:
            n["duration_micros"] = v
        elif field in (F_IN, F_OUT):
            io = {}
            for f2, _, v2 in _fields(v):
                io[{1: "values", 2: "shapes", 3: "types"}[f2]] = v2.decode()
            n["inputs" if field == F_IN else "outputs"] = io
        elif field == F_ATTR:
            n["attrs"].append(_decode_attr(v))
    return n


def read_et(path):
    """Returns (metadata dict, [node dict])."""
    data = open(path, "rb").read()
    msgs, i = [], 0
    while i < len(data):
        ln, i = _uvarint(data, i)
        msgs.append(data[i:i + ln])
        i += ln
    meta = {"attrs": []}
    for field, _, v in _fields(msgs[0]):
        if field == 1:
            meta["version"] = v.decode()
        elif field == 2:
            meta["attrs"].append(_decode_attr(v))
    return meta, [decode_node(m) for m in msgs[1:]]


def attr(node, name, default=None):
    for k, _, v in node.get("attrs", ()):
        if k == name:
            return v
    return default
