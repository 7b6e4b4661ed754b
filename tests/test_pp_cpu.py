"""Pipeline (1F1B over point-to-point) and its composition with tensor parallelism on CPU
ranks (gloo): the sharded/staged step reproduces the single-process model's loss and every
rank's gradients are the matching slices of the full model's gradients."""
import pytest
import torch

from tests.dist_helpers import run_ranks


def _step(rank, world, dp, tp, pp, m):
    from llmt.config import get_config
    from llmt.models.llama import build_model, make_batch
    from llmt.parallel.engine import ParallelTrainer
    from llmt.parallel.groups import Layout
    from llmt.parallel.tp import shard_state
    torch.manual_seed(0)
    cfg = get_config("tiny256", kv_heads=2)
    B, T = 4, 32
    batches = [make_batch(B, T, cfg.vocab, "cpu", seed=d) for d in range(dp)]
    tr = ParallelTrainer(cfg, B, T, Layout(dp=dp, tp=tp, pp=pp), microbatches=m, device="cpu", impl="torch")
    g = tr.groups
    idx, tgt = batches[g.dp_rank]
    loss = tr.forward_backward(idx, tgt)
    # single-process reference on this data-parallel rank's batch, same micro-batching
    full = build_model(cfg, T, seed=0)
    ref_losses = []
    for i in range(m):
        sl = slice(i * B // m, (i + 1) * B // m)
        li = full(idx[sl], tgt[sl])
        (li / m).backward()
        ref_losses.append(li.item())
    if tr.is_last_stage:
        assert abs(loss.item() - sum(ref_losses) / m) < 1e-4 * abs(loss.item())
    grads = {k: p.grad for k, p in full.named_parameters()}
    if tp > 1:
        grads = shard_state(grads, cfg, tp, g.tp_rank)
    own = {}
    for k, p in tr.stage.named_parameters():
        if k.startswith("blocks."):
            i, rest = k[len("blocks."):].split(".", 1)
            k = f"blocks.{int(i) + tr.stage.l0}.{rest}"
        own[k] = p.grad
    assert own, "stage without parameters"
    for k, gr in own.items():
        ref = grads[k]
        err = (gr - ref).norm() / ref.norm().clamp_min(1e-12)
        assert err < 2e-4, (rank, k, float(err))


@pytest.mark.parametrize("dp,tp,pp,m", [(1, 1, 2, 4), (1, 2, 2, 4), (2, 1, 2, 2)])
def test_pipeline_matches_single_process(dp, tp, pp, m):
    run_ranks(_step, dp * tp * pp, dp, tp, pp, m)


def test_stage_layers_cover_model():
    from llmt.parallel.pp import stage_layers
    for L in (4, 5, 24, 32):
        for pp in (1, 2, 3, 4):
            spans = [stage_layers(L, pp, s) for s in range(pp)]
            assert spans[0][0] == 0 and spans[-1][1] == L
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
