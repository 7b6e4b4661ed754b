"""Memory-safety checks of the memory-bound kernels (a stand-in for a memory sanitizer, which this
pool does not run).

Canaries: each op writes into a view inside a larger buffer whose surrounding elements hold a
known pattern (guard rows before and after, and columns past the row width where the op takes
a row pitch); on ragged shapes the pattern must be intact afterwards and the results must
match fp32 PyTorch. The same checks run twice: in this process on the release module, and in
a child process on the bounds-checked module (llmt._C_bounds, LLMT_BOUNDS=1), where every
guarded access also checks its index range and the module's record of violations must stay
empty. The child also runs the build's self-test: a store guarded at an index past the end is
recorded with its site and skipped (the buffer stays unchanged), which shows the checks are
live in that build.
"""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

GUARD = 3  # guard rows on each side


def _guarded(rows, cols, dtype, pitch=None, fill=-7.0):
    """(full buffer, view of rows x cols at row pitch `pitch` in its middle)."""
    pitch = pitch or cols
    buf = torch.full((rows + 2 * GUARD, pitch), fill, dtype=dtype, device="cuda")
    return buf, buf[GUARD:GUARD + rows, :cols]


def _outside_intact(buf, rows, cols, fill=-7.0):
    inside = torch.zeros_like(buf, dtype=torch.bool)
    inside[GUARD:GUARD + rows, :cols] = True
    return bool((buf[~inside].float() == fill).all())


def run_checks():
    """Every op on ragged shapes; returns {name: ok}."""
    from llmt.models.llama import rope_tables
    from llmt.ops import native as N
    g = torch.Generator(device="cuda").manual_seed(0)
    res = {}
    # SwiGLU forward and backward, strided outputs with padding columns
    rows, F = 37, 136
    gu = torch.randn(rows, 2 * F, device="cuda", generator=g).bfloat16()
    gg, uu = gu[:, :F], gu[:, F:]
    hb, h = _guarded(rows, F, torch.bfloat16, pitch=F + 24)
    N.swiglu_fwd(gg, uu, h)
    ref = torch.nn.functional.silu(gg.float()) * uu.float()
    res["swiglu_fwd"] = _outside_intact(hb, rows, F) and torch.allclose(h.float(), ref, rtol=2e-2, atol=2e-2)
    dh = torch.randn(rows, F, device="cuda", generator=g).bfloat16()
    dgb = torch.full((rows + 2 * GUARD, 2 * F + 16), -7.0, dtype=torch.bfloat16, device="cuda")
    dg, du = dgb[GUARD:GUARD + rows, :F], dgb[GUARD:GUARD + rows, F:2 * F]
    N.swiglu_bwd(dh, gg, uu, dg, du)
    res["swiglu_bwd"] = _outside_intact(dgb, rows, 2 * F)
    # RoPE forward in place on a packed qkv view (2 rotated heads + v) of 45 rows
    T, hd, nh = 45, 64, 3
    qb, qkv = _guarded(T, nh * hd, torch.bfloat16)
    x = torch.randn(T, nh * hd, device="cuda", generator=g).bfloat16()
    qkv.copy_(x)
    cos, sin = rope_tables(T, hd, 10000.0, "cuda")
    N.rope_inplace(qkv, cos, sin, T, 2, hd)
    from llmt.models.llama import apply_rope
    want = apply_rope(x.float().view(T, nh, hd)[:, :2].transpose(0, 1), cos, sin).transpose(0, 1).reshape(T, 2 * hd)
    res["rope"] = _outside_intact(qb, T, nh * hd) and torch.allclose(qkv[:, :2 * hd].float(), want, rtol=2e-2, atol=2e-2) \
        and torch.equal(qkv[:, 2 * hd:], x[:, 2 * hd:])
    # embedding gather into a guarded output, scatter-add into a guarded gradient
    V, d, n = 53, 40, 29
    W = torch.randn(V, d, device="cuda", generator=g)
    idx = torch.randint(0, V, (n,), device="cuda", generator=g)
    xb, xo = _guarded(n, d, torch.float32)
    N.embedding_fwd(idx, W, out=xo)
    res["embedding_fwd"] = _outside_intact(xb, n, d) and torch.equal(xo, W[idx])
    dWb, dW = _guarded(V, d, torch.float32, fill=0.0)
    dx = torch.randn(n, d, device="cuda", generator=g)
    N.embedding_bwd(idx, dx, dW)
    want = torch.zeros(V, d, device="cuda").index_add_(0, idx, dx)
    res["embedding_bwd"] = _outside_intact(dWb, V, d, fill=0.0) and torch.allclose(dW, want, rtol=1e-5, atol=1e-5)
    # cross entropy rows over logits with a pitch past the vocabulary
    R, Vc = 19, 200
    lb, logits = _guarded(R, Vc, torch.bfloat16, pitch=Vc + 40)
    lg = torch.randn(R, Vc, device="cuda", generator=g)
    logits.copy_(lg.bfloat16())
    tgt = torch.randint(0, Vc, (R,), device="cuda", generator=g)
    lse = torch.empty(R, device="cuda")
    loss = torch.empty(R, device="cuda")
    N.ce_fwd_rows(logits, tgt, lse, loss)
    want = torch.nn.functional.cross_entropy(logits.float(), tgt, reduction="none")
    ok_f = torch.allclose(loss, want, rtol=1e-3, atol=1e-3)
    N.ce_bwd_rows(logits, tgt, lse, None, 1.0 / R)
    res["ce_rows"] = ok_f and _outside_intact(lb, R, Vc)
    # fp32 -> bf16 cast into the middle of a guarded buffer
    src = torch.randn(1001, device="cuda", generator=g)
    cb = torch.full((1001 + 2 * GUARD,), -7.0, dtype=torch.bfloat16, device="cuda")
    N.cast_bf16(src, cb[GUARD:GUARD + 1001])
    res["cast_bf16"] = bool((cb[:GUARD].float() == -7).all() and (cb[-GUARD:].float() == -7).all()) and \
        torch.equal(cb[GUARD:GUARD + 1001], src.bfloat16())
    # add + RMSNorm forward and backward on a ragged width (outputs are allocated by the op)
    Nr, D = 37, 520
    r = torch.randn(Nr, D, device="cuda", generator=g)
    a = torch.randn(Nr, D, device="cuda", generator=g).bfloat16()
    w = 1 + 0.1 * torch.randn(D, device="cuda", generator=g)
    y, s, rstd = N.add_rmsnorm_fwd(a, r, w, 1e-5)
    sf = r + a.float()
    yref = sf * torch.rsqrt(sf.pow(2).mean(-1, keepdim=True) + 1e-5) * w
    dw = torch.zeros(D, device="cuda")
    dy = torch.randn(Nr, D, device="cuda", generator=g).bfloat16()
    ds, _ = N.rmsnorm_bwd(dy, s, w, rstd, None, dw, accumulate=False)
    res["rmsnorm"] = torch.allclose(y.float(), yref, rtol=2e-2, atol=2e-2) and bool(torch.isfinite(ds).all())
    torch.cuda.synchronize()
    return {k: bool(v) for k, v in res.items()}


def test_canaries_release_build():
    from llmt.ops import native as N
    res = run_checks()
    assert all(res.values()), res
    assert not N.ext().bounds_checking()


def test_bounds_checked_build_in_child():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, LLMT_BOUNDS="1", PYTHONPATH=root)
    out = subprocess.run([sys.executable, "-m", "tests.test_bounds_gpu"], cwd=root, env=env, capture_output=True,
                         text=True, timeout=600)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-2000:]
    res = json.loads(out.stdout.strip().splitlines()[-1])
    assert res["bounds_checking"] is True
    assert all(res["checks"].values()), res
    assert res["record_after_checks"] == 0, res
    # the self-test: index n of an n-float buffer, site 999, recorded and skipped
    probe = res["probe_record"]
    assert probe >> 63 == 1 and (probe >> 40) & 0x7FFFFF == 999 and probe & 0xFFFFFFFFFF == 64
    assert res["probe_buffer_unchanged"]


def _child():
    from llmt.ops import native as N
    C = N.ext()
    checks = run_checks()
    rec = C.bounds_error(True)
    buf = torch.zeros(64, device="cuda")
    C.bounds_probe(buf, 64)
    torch.cuda.synchronize()
    probe = C.bounds_error(True)
    print(json.dumps({"bounds_checking": C.bounds_checking(), "checks": checks, "record_after_checks": rec,
                      "probe_record": probe, "probe_buffer_unchanged": bool((buf == 0).all())}))


if __name__ == "__main__":
    _child()
