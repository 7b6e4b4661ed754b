"""Native training path (every op on llmt._C) vs the plain PyTorch fp32 model on the same weights."""
import pytest
import torch

from tests.helpers import rel_err

pytestmark = pytest.mark.gpu


def _pair(cfg, T, seed=0):
    from llmt.models.llama import build_model
    from llmt.models.native import NativeLlama
    ref = build_model(cfg, T, seed=seed, device="cuda")
    ours = build_model(cfg, T, seed=seed, device="cuda")
    return ref, ours, NativeLlama(ours)


@pytest.mark.parametrize("overrides", [{}, {"kv_heads": 2}, {"H": 2}])
def test_native_loss_and_grads_match_fp32(overrides):
    from llmt.config import get_config
    from llmt.models.llama import make_batch
    from llmt.ops import native
    cfg = get_config("tiny256", **overrides)
    B, T = 2, 128
    ref, ours, net = _pair(cfg, T)
    idx, tgt = make_batch(B, T, cfg.vocab, "cuda")
    loss_ref = ref(idx, tgt)
    loss_ref.backward()
    loss = net(idx, tgt)
    loss.backward()
    torch.cuda.synchronize()
    assert native.gemm_error_code() == 0 and native.attn_error_code() == 0
    assert abs(loss.item() - loss_ref.item()) / loss_ref.item() < 1e-2
    for (name, p_ref), p in zip(ref.named_parameters(), ours.parameters()):
        assert p.grad is None
        assert rel_err(p.main_grad, p_ref.grad) < 5e-2, name


def test_native_training_decreases_loss_and_graph_matches_eager():
    from llmt.config import get_config
    from llmt.models.llama import make_batch
    from llmt.train import Trainer
    cfg = get_config("tiny256")
    idx, tgt = make_batch(2, 128, cfg.vocab, "cpu")
    eager = Trainer(cfg, 2, 128, cuda_graph=False)
    graph = Trainer(cfg, 2, 128, cuda_graph=True)
    le = [eager.train_step(idx, tgt) for _ in range(8)]
    lg = [graph.train_step(idx, tgt) for _ in range(8)]
    assert le[-1] < le[0] - 0.5
    # the capture's warm-up steps are undone: step i of the graph trainer is step i of the eager one
    assert max(abs(a - b) / b for a, b in zip(lg, le)) < 2e-2
    graph.release()


def test_native_step_matches_reference_adamw():
    """One full step (fwd + bwd + fused AdamW) vs torch.optim.AdamW on the fp32 model."""
    from llmt.config import get_config
    from llmt.models.llama import build_model, make_batch
    from llmt.train import Trainer
    cfg = get_config("tiny256")
    idx, tgt = make_batch(2, 128, cfg.vocab, "cpu")
    ref = build_model(cfg, 128, seed=0, device="cuda")
    opt = torch.optim.AdamW(ref.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1)
    ref(idx.cuda(), tgt.cuda()).backward()
    opt.step()
    tr = Trainer(cfg, 2, 128, cuda_graph=False)
    tr.train_step(idx, tgt)
    for (name, p_ref), p in zip(ref.named_parameters(), tr.model.parameters()):
        # one Adam step moves each weight by ~lr; compare the update directions
        assert rel_err(p.detach(), p_ref.detach()) < 5e-3, name


def _steps_vs_reference(graph, microbatches, steps=3):
    """Per step, the native trainer's weight gradients (left in the flat buffer: nothing clears
    it between steps, the first micro-batch's backward stores them) against PyTorch's fp32
    gradients of the same step; returns the worst relative error seen after the first step."""
    from llmt.config import get_config
    from llmt.models.llama import build_model, make_batch
    from llmt.train import Trainer
    cfg = get_config("tiny256")
    ref = build_model(cfg, 128, seed=0, device="cuda")
    opt = torch.optim.AdamW(ref.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1)
    tr = Trainer(cfg, 2, 128, cuda_graph=graph, microbatches=microbatches)
    assert tr.first_write
    worst = {}
    for step in range(steps):
        idx, tgt = make_batch(2, 128, cfg.vocab, "cpu", seed=step)
        opt.zero_grad(set_to_none=True)
        for m in range(microbatches):
            sl = slice(m * 2 // microbatches, (m + 1) * 2 // microbatches)
            (ref(idx[sl].cuda(), tgt[sl].cuda()) / microbatches).backward()
        tr.train_step(idx, tgt)
        torch.cuda.synchronize()
        for (name, p_ref), p in zip(ref.named_parameters(), tr.model.parameters()):
            worst[name] = max(worst.get(name, 0.0), rel_err(p.main_grad, p_ref.grad))
        opt.step()
    if graph:
        tr.release()
    return worst


@pytest.mark.parametrize("graph,microbatches", [(False, 1), (True, 1), (False, 2)])
def test_gradients_match_reference_every_step(graph, microbatches):
    """Three steps: every step's weight gradients match PyTorch's (a writer that added to the
    previous step's gradient instead of storing would be off by about 100%)."""
    worst = _steps_vs_reference(graph, microbatches)
    for name, e in worst.items():
        assert e < 5e-2, (name, e)


def test_stale_gradient_would_be_caught(monkeypatch):
    """Control for the test above: weight-gradient GEMMs that add on the first write (the
    buffer then still holds the previous step's gradient) must fail it."""
    from llmt.ops import functions
    from llmt.ops import native as N

    def always_add(dy, x, out):
        N.gemm(dy, x, ta=True, tb=False, out=out, accumulate=True)
    monkeypatch.setattr(functions, "wgrad_into", always_add)
    worst = _steps_vs_reference(False, 1)
    assert max(worst.values()) > 0.5, worst


@pytest.mark.parametrize("mode", [{"fwd": False, "bwd": False}, {"fwd": True, "bwd": False}, {"fwd": False, "bwd": True}])
def test_swiglu_unfused_paths_match_fp32(mode, monkeypatch):
    """The standalone-kernel SwiGLU paths give the same loss and gradients as the fp32 model."""
    from llmt.config import get_config
    from llmt.models.llama import make_batch
    from llmt.ops import functions
    monkeypatch.setattr(functions, "SWIGLU_EPILOGUE", dict(mode))
    cfg = get_config("tiny256")
    ref, ours, net = _pair(cfg, 128)
    idx, tgt = make_batch(2, 128, cfg.vocab, "cuda")
    loss_ref = ref(idx, tgt)
    loss_ref.backward()
    loss = net(idx, tgt)
    loss.backward()
    torch.cuda.synchronize()
    assert abs(loss.item() - loss_ref.item()) / loss_ref.item() < 1e-2
    for (name, p_ref), p in zip(ref.named_parameters(), ours.parameters()):
        assert rel_err(p.main_grad, p_ref.grad) < 5e-2, name


@pytest.mark.parametrize("fusion", [{"head_ce": True}, {"head_ce": False}, {"rope": False}])
def test_fusion_switches_match_fp32(fusion, monkeypatch):
    """Fused head CE (logits never written) and materialised-logit CE, and RoPE as a separate
    kernel, all give the fp32 model's loss and gradients."""
    from llmt.config import get_config
    from llmt.models.llama import make_batch
    from llmt.ops import functions
    monkeypatch.setattr(functions, "FUSION", {**functions.FUSION, **fusion})
    cfg = get_config("tiny256")
    ref, ours, net = _pair(cfg, 128)
    idx, tgt = make_batch(2, 128, cfg.vocab, "cuda")
    loss_ref = ref(idx, tgt)
    loss_ref.backward()
    loss = net(idx, tgt)
    loss.backward()
    torch.cuda.synchronize()
    assert abs(loss.item() - loss_ref.item()) / loss_ref.item() < 1e-2
    for (name, p_ref), p in zip(ref.named_parameters(), ours.parameters()):
        assert rel_err(p.main_grad, p_ref.grad) < 5e-2, name
