"""Two pipeline stages on one GPU, chained by hand (no NCCL) in the 1F1B order of stage 0
(F0, F1, B0, B1 with stage 1's F/B in between): stage 0's boundary activations are copied into
fresh tensors for stage 1 and stage 1's input gradients fed back into stage 0's backward,
which is what the 1F1B runner does across ranks. Loss and every gradient match the
single-stage native model on the same two micro-batches."""
import pytest
import torch

from tests.helpers import rel_err

pytestmark = pytest.mark.gpu


def test_two_native_stages_match_full_model():
    from llmt.config import get_config
    from llmt.models.llama import build_model, make_batch
    from llmt.models.native import NativeLlama
    from llmt.parallel.pp import NativeStage, build_stage
    cfg = get_config("tiny256", kv_heads=2)
    B, T, m = 1, 128, 2
    batches = [make_batch(B, T, cfg.vocab, "cuda", seed=i) for i in range(m)]
    full = build_model(cfg, T, seed=0, device="cuda")
    net = NativeLlama(full)
    loss_ref = 0.0
    for idx, tgt in batches:
        li = net(idx, tgt)
        (li / m).backward()
        loss_ref += li.item() / m
    s0 = NativeStage(build_stage(cfg, T, 2, 0, device="cuda"))
    s1 = NativeStage(build_stage(cfg, T, 2, 1, device="cuda"))
    outs, grads, losses = {}, {}, []

    def f0(i):
        outs[i] = s0.forward_blocks(s0.forward_first(batches[i][0]), B, T)

    def f1b1(i):
        recv = [t.detach().clone().requires_grad_(True) for t in outs[i]]
        li = s1.forward_last(s1.forward_blocks(tuple(recv), B, T), batches[i][1])
        (li / m).backward()
        losses.append(li.item())
        grads[i] = [t.grad.detach().clone() for t in recv]

    def b0(i):
        assert grads[i][0].dtype == torch.bfloat16 and grads[i][1].dtype == torch.float32
        torch.autograd.backward(list(outs[i]), grads[i])

    f0(0)
    f1b1(0)
    f0(1)
    b0(0)
    f1b1(1)
    b0(1)
    torch.cuda.synchronize()
    assert abs(sum(losses) / m - loss_ref) < 1e-3 * loss_ref
    ref = {k: p.main_grad for k, p in zip(net.flat.names, net.flat.params)}
    for st in (s0, s1):
        for k, p in zip(st.flat.names, st.flat.params):
            assert rel_err(p.main_grad, ref[k]) < 2e-2, k
