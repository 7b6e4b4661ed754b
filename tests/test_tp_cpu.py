"""Tensor + sequence parallel sharding math on CPU ranks (gloo): a TP=2 step of the sharded
model gives the single-process model's loss, and every rank's weight gradients are the
matching slices of the full model's gradients."""
import pytest
import torch

from tests.dist_helpers import run_ranks


def _tp_step(rank, world, overrides):
    import torch.distributed as dist
    from llmt.config import get_config
    from llmt.models.llama import build_model, make_batch
    from llmt.parallel.tp import TPTorchLlama, build_local_model, shard_state, sync_replicated_grads
    torch.manual_seed(0)
    cfg = get_config("tiny256", **overrides)
    B, T = 2, 64
    full = build_model(cfg, T, seed=0)
    idx, tgt = make_batch(B, T, cfg.vocab, "cpu")
    loss_full = full(idx, tgt)
    loss_full.backward()
    group = dist.new_group(list(range(world)))
    local = build_local_model(cfg, T, world, rank, seed=0, init="full")
    net = TPTorchLlama(local, group)
    loss = net(idx, tgt)
    loss.backward()
    sync_replicated_grads(local, group)
    assert abs(loss.item() - loss_full.item()) < 1e-4 * loss_full.item(), (loss.item(), loss_full.item())
    want = shard_state({k: p.grad for k, p in full.named_parameters()}, cfg, world, rank)
    for k, p in local.named_parameters():
        ref = want[k]
        err = (p.grad - ref).norm() / ref.norm().clamp_min(1e-12)
        assert err < 1e-4, (k, float(err))


@pytest.mark.parametrize("overrides", [{}, {"kv_heads": 2}])
def test_tp2_matches_single_process(overrides):
    run_ranks(_tp_step, 2, overrides)


def test_shard_unshard_roundtrip():
    from llmt.config import get_config
    from llmt.models.llama import build_model
    from llmt.parallel.tp import shard_state, unshard_state
    for overrides, tps in (({"kv_heads": 2}, (2,)), ({}, (2, 4))):
        cfg = get_config("tiny256", **overrides)
        sd = build_model(cfg, 32, seed=1).state_dict()
        for tp in tps:
            back = unshard_state([shard_state(sd, cfg, tp, r) for r in range(tp)], cfg)
            for k in sd:
                assert torch.equal(back[k], sd[k]), k


def test_rank_layout_matches_reference_order():
    from llmt.parallel.groups import Layout, coords_of, rank_of
    lay = Layout(dp=2, tp=2, pp=2)
    seen = set()
    for d in range(2):
        for p in range(2):
            for t in range(2):
                r = rank_of(d, p, t, lay.pp, lay.tp)
                assert coords_of(r, lay.pp, lay.tp) == (d, p, t)
                seen.add(r)
    assert seen == set(range(8))
    assert lay.tp_ranks(1, 0) == [4, 5] and lay.pp_ranks(0, 1) == [1, 3] and lay.dp_ranks(1, 1) == [3, 7]


def test_pending_gather_is_consumed_once():
    """A gather buffer that owes its all-gather hands it to the first GEMM that reads it with a
    K-major A, once; a consumer that reads it MN-major (a weight gradient) first runs it alone."""
    from llmt.ops import native as N
    from llmt.parallel.tp_p2p import AG_PIECES, PendingGather

    class Comm:
        tp, rank, nl = 2, 1, 128

        def __init__(self):
            self.ag_calls = [0, 0, 0]
            self.unfused = []

        def _gather(self, x_l, dst, code):
            self.unfused.append((x_l, dst, code))

    c = Comm()
    x_l, dst, flags = torch.zeros(128, 8), torch.zeros(2), torch.zeros(2)
    buf = torch.zeros(256, 8)
    a = buf.view_as(buf)
    a._llmt_pending_ag = PendingGather(c, x_l, 2, dst, flags)
    kw = N._take_ag(a)
    assert kw["ag_expect"] == AG_PIECES and kw["ag_tp"] == 2 and kw["tp_rank"] == 1 and kw["rows_per_rank"] == 128
    assert kw["ag_src"] is x_l and kw["ag_dst"] is dst and kw["ag_flags"] is flags
    assert N._take_ag(a) == {} and c.ag_calls == [0, 0, 1]
    a._llmt_pending_ag = PendingGather(c, x_l, 2, dst, flags)
    assert N._take_ag(a, ta=True) == {} and len(c.unfused) == 1 and c.ag_calls == [0, 0, 1]
    a._llmt_pending_ag = PendingGather(c, x_l, 2, dst, flags)
    assert N._take_ag(a)["ag_expect"] == 2 * AG_PIECES


def test_low_precision_tp_block_needs_nccl_collectives():
    """Low-precision block linears are not fused with the peer-memory collectives: asking for both
    is refused before any kernel runs."""
    from llmt.parallel.tp import native_tp_block
    with pytest.raises(ValueError, match="NCCL"):
        native_tp_block(None, None, None, None, None, 1, 128, None, None, comm=object(), i=0, linear="mxfp8")


class _FakeExt:
    """The parts of the extension TPPeerComm uses, over CPU memory: "pointers" are integers into
    per-allocation byte buffers, an opened peer handle maps to a distinct fake base."""

    def __init__(self, rank):
        self.bufs, self.next = {}, (rank + 1) << 40

    def _new(self, nbytes):
        base = self.next
        self.next += max(nbytes, 1 << 12) + (1 << 20)
        self.bufs[base] = torch.zeros(nbytes, dtype=torch.uint8)
        return base

    def ipc_alloc(self, nbytes):
        base = self._new(nbytes)
        return base, list(base.to_bytes(8, "little")) + [0] * 56

    def ipc_open(self, handle):
        return self._new(16) + (1 << 36)  # a peer's mapping: never dereferenced here

    def tensor_from_ptr(self, ptr, n, dtype, dev):
        base = max(b for b in self.bufs if b <= ptr)
        es = torch.empty((), dtype=dtype).element_size()
        return self.bufs[base][ptr - base: ptr - base + n * es].view(dtype)

    def ipc_close(self, p):
        pass

    def ipc_free(self, p):
        pass


def _peer_comm_layout(rank, world):
    import torch.distributed as dist
    from llmt.ops import native as N
    from llmt.parallel import tp_p2p
    fake = _FakeExt(rank)
    N.ext = lambda: fake
    tp_p2p.torch.cuda.synchronize = lambda *a, **k: None
    rows, d, sites, sets = 512, 64, 4, 2
    c = tp_p2p.TPPeerComm(dist.new_group([0, 1]), rows, d, sites, "cpu", sets=sets)
    blocks, mat = rows // 128, rows * d * 2
    assert c.fuse_gather and c.nl == 256 and len(c.site_local) == sites * sets
    x_l = torch.randn(c.nl, d).bfloat16()
    for k in range(sets):
        c.select_set(k + sets)  # micro-batch k + sets reuses set k
        out = c.all_gather_site(x_l, 3)
        pend = out._llmt_pending_ag
        idx = k * sites + 3
        assert pend.index == idx and out.data_ptr() == c.site_local[idx].data_ptr()
        # this rank's entry of the pointer arrays is its own buffer, the other rank's is the mapping
        assert int(pend.dst_ptrs[rank]) == c._own[0] + idx * mat
        assert int(pend.flag_ptrs[rank]) == c._own[2] + idx * blocks * 4
        assert int(pend.dst_ptrs[1 - rank]) != int(pend.dst_ptrs[rank])
        kw = pend.kwargs()
        assert kw["ag_expect"] == 8 and kw["rows_per_rank"] == 256 and kw["tp_rank"] == rank
    # distinct sets never share a buffer; the backward gathers come after every set's sites
    ptrs = {t.data_ptr() for t in c.site_local} | {t.data_ptr() for t in c.bwd_local}
    assert len(ptrs) == sites * sets + 2
    b = c.all_gather_bwd(x_l)._llmt_pending_ag
    assert b.index == sites * sets and int(b.flag_ptrs[rank]) == c._own[2] + sites * sets * blocks * 4
    assert len(c.ag_calls) == sites * sets + 2


def test_peer_comm_buffer_sets_and_flags():
    """Peer-memory tensor parallelism under pipeline parallelism: every in-flight micro-batch has
    its own forward gather buffers and flag counters, and the pointer arrays a fused gather hands
    the GEMM point at the right buffer of every rank (CPU stand-in for the extension)."""
    run_ranks(_peer_comm_layout, 2)


def test_mxfp8_shards_quantize_like_the_whole_tensor():
    """Under tensor parallelism each rank quantizes its own shards. For MXFP8 (one scale per 32
    elements along the contraction) that gives the same bytes and scales as quantizing the whole
    tensor, for row shards (qkv, w1||w3: output rows) and for column shards whose width is a
    multiple of 32 (wo, w2: the contraction itself), so the sharded model multiplies the same
    numbers as the single-GPU one."""
    from llmt.config import get_config
    from llmt.ops.lowp_ref import mxfp8_quant_ref
    from llmt.parallel.tp import shard_tensor
    cfg = get_config("tiny256", ffn=768)
    g = torch.Generator().manual_seed(0)
    tp = 2
    for name, shape in (("blocks.0.attn.qkv.weight", (3 * cfg.d, cfg.d)), ("blocks.0.mlp.w1.weight", (cfg.ffn, cfg.d)),
                        ("blocks.0.attn.wo.weight", (cfg.d, cfg.d)), ("blocks.0.mlp.w2.weight", (cfg.d, cfg.ffn))):
        w = torch.randn(*shape, generator=g) * 0.02
        q, s = mxfp8_quant_ref(w)
        for r in range(tp):
            qs, ss = mxfp8_quant_ref(shard_tensor(name, w, cfg, tp, r).contiguous())
            assert torch.equal(qs.view(torch.uint8), shard_tensor(name, q.view(torch.uint8), cfg, tp, r)), name
            if name.endswith(("wo.weight", "w2.weight")):  # column shard: the scales split by 32-blocks
                n = ss.shape[1]
                assert torch.equal(ss, s[:, r * n:(r + 1) * n]), name
            else:
                assert torch.equal(ss, shard_tensor(name, s, cfg, tp, r)), name
