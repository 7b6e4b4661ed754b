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
