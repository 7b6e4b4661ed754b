"""All-gather fused into the GEMM's A loads (the tensor-parallel qkv, w1||w3 and dgrad GEMMs), on
one GPU with stand-ins for the other ranks.

This rank's gather buffer already holds the other ranks' rows and its flags say that their
pieces have landed, as if their kernels had stored them; the other ranks' buffers and flags are
local tensors. The GEMM must store this rank's rows into every buffer, count its 16-row pieces in
every rank's flags, and compute what a plain GEMM of the whole A computes (fp32 PyTorch reference).
The last test gives the wait a flag that nothing sets: the wait runs out after its limit, records
error code 8 and the kernel finishes, so the context stays usable."""
import pytest
import torch

from tests.helpers import rel_err

pytestmark = pytest.mark.gpu

PIECES = 8  # 16-row pieces per 128-row block (kAgPieces)


@pytest.fixture(scope="module")
def nat():
    from llmt.ops import native
    native.ext()
    native.gemm_error_code(reset=True)
    return native


class Ranks:
    """Every rank's gather buffer and flags (index `rank` is this rank's), with the other ranks'
    rows already in this rank's buffer."""

    def __init__(self, tp, rank, rows, K, seed=0):
        g = torch.Generator(device="cuda").manual_seed(seed)
        self.tp, self.rank, self.rows = tp, rank, rows
        self.full = torch.randn(tp * rows, K, device="cuda", generator=g).bfloat16()
        self.bufs = [torch.zeros(tp * rows, K, device="cuda", dtype=torch.bfloat16) for _ in range(tp)]
        for q in range(tp):
            if q != rank:
                self.bufs[rank][q * rows:(q + 1) * rows] = self.full[q * rows:(q + 1) * rows]
        self.flags = [torch.zeros(tp * rows // 128, device="cuda", dtype=torch.int32) for _ in range(tp)]
        self.dst = torch.tensor([b.data_ptr() for b in self.bufs], dtype=torch.int64, device="cuda")
        self.fl = torch.tensor([f.data_ptr() for f in self.flags], dtype=torch.int64, device="cuda")
        self.x_l = self.full[rank * rows:(rank + 1) * rows].clone()

    def own(self, p):
        return self.bufs[p][self.rank * self.rows:(self.rank + 1) * self.rows]

    def arrive(self, call):
        """The other ranks' pieces of call `call` have landed in this rank's flags."""
        bpr = self.rows // 128
        for q in range(self.tp):
            if q != self.rank:
                self.flags[self.rank][q * bpr:(q + 1) * bpr] = call * PIECES

    def kwargs(self, call):
        return dict(ag_src=self.x_l, ag_dst=self.dst, ag_flags=self.fl, ag_expect=call * PIECES, ag_tp=self.tp,
                    tp_rank=self.rank, rows_per_rank=self.rows)

    def check_stores(self, call):
        bpr = self.rows // 128
        lo, hi = self.rank * bpr, (self.rank + 1) * bpr
        for p in range(self.tp):
            assert torch.equal(self.own(p), self.x_l), f"rank {self.rank}'s rows not stored into buffer {p}"
            assert (self.flags[p][lo:hi] == call * PIECES).all(), self.flags[p]
            if p != self.rank:
                assert (self.flags[p][:lo] == 0).all() and (self.flags[p][hi:] == 0).all()
        assert torch.equal(self.bufs[self.rank], self.full)

    def reset_own(self):
        for p in range(self.tp):
            self.own(p).zero_()


@pytest.mark.parametrize("tp,rank,rows,bn", [(2, 0, 256, 0), (2, 1, 256, 256), (4, 2, 128, 128), (8, 5, 128, 0),
                                             (2, 1, 512, 128)])
def test_fused_allgather_gemm(nat, tp, rank, rows, bn):
    K, N = 1024, 768
    R = Ranks(tp, rank, rows, K, seed=tp * 16 + rank)
    w = torch.randn(N, K, device="cuda", generator=torch.Generator(device="cuda").manual_seed(7)).bfloat16()
    ref = R.full.float() @ w.float().t()
    for call in (1, 2):  # a second call: the flags keep counting, the rows are stored again
        R.reset_own()
        R.arrive(call)
        y = torch.empty(tp * rows, N, device="cuda", dtype=torch.bfloat16)
        nat.ext().gemm(R.bufs[rank], w, False, True, nat.EPI_BF16, y, bn=bn, **R.kwargs(call))
        torch.cuda.synchronize()
        assert nat.gemm_error_code() == 0
        assert rel_err(y, ref) < 1e-2
        R.check_stores(call)


class _Pending:
    def __init__(self, kw):
        self.kw, self.used = kw, 0

    def kwargs(self):
        self.used += 1
        return self.kw

    def run_unfused(self):
        raise AssertionError("the SwiGLU GEMM has a K-major A: the gather must be fused")


def test_fused_allgather_swiglu_through_wrapper(nat):
    """The wrapper consumes a pending gather once (merged w1||w3 GEMM with the SwiGLU epilogue)."""
    tp, rank, rows, K, ffn = 2, 1, 256, 512, 384
    R = Ranks(tp, rank, rows, K, seed=3)
    g = torch.Generator(device="cuda").manual_seed(4)
    w13 = (torch.randn(2 * ffn, K, device="cuda", generator=g) * 0.05).bfloat16()
    R.arrive(1)
    x = R.bufs[rank].view_as(R.bufs[rank])
    pend = _Pending(R.kwargs(1))
    x._llmt_pending_ag = pend
    h, gu = nat.gemm_swiglu(x, w13, ffn)
    torch.cuda.synchronize()
    assert pend.used == 1 and not hasattr(x, "_llmt_pending_ag")
    assert nat.gemm_error_code() == 0
    R.check_stores(1)
    gr = R.full.float() @ w13[:ffn].float().t()
    ur = R.full.float() @ w13[ffn:].float().t()
    assert rel_err(h, torch.nn.functional.silu(gr) * ur) < 2e-2


def test_fused_allgather_rope_epilogue(nat):
    """qkv GEMM with the RoPE epilogue and a fused gather against the same GEMM on the whole A."""
    tp, rank, rows, K, H, KV, hd, T = 4, 3, 128, 256, 4, 2, 64, 128
    R = Ranks(tp, rank, rows, K, seed=5)
    g = torch.Generator(device="cuda").manual_seed(6)
    w = (torch.randn((H + 2 * KV) * hd, K, device="cuda", generator=g) * 0.05).bfloat16()
    from llmt.models.llama import rope_tables
    cos, sin = rope_tables(T, hd, 10000.0, "cuda")
    ref = nat.gemm_rope(R.full, w, cos, sin, T, hd, (H + KV) * hd)
    R.arrive(1)
    out = torch.empty_like(ref)
    nat.ext().gemm(R.bufs[rank], w, False, True, nat.EPI_ROPE, out, cos_t=cos, sin_t=sin, T=T, hd=hd,
                   rot_cols=(H + KV) * hd, **R.kwargs(1))
    torch.cuda.synchronize()
    assert nat.gemm_error_code() == 0
    assert rel_err(out, ref.float()) < 1e-2
    R.check_stores(1)


def test_fused_allgather_wait_runs_out(nat):
    """The other rank's pieces never arrive: the producer's wait runs out (1 s), records code 8
    and the GEMM completes; a plain GEMM afterwards is still correct."""
    tp, rank, rows, K, N = 2, 0, 128, 256, 256
    R = Ranks(tp, rank, rows, K, seed=9)
    w = torch.randn(N, K, device="cuda").bfloat16()
    y = torch.empty(tp * rows, N, device="cuda", dtype=torch.bfloat16)
    nat.ext().gemm(R.bufs[rank], w, False, True, nat.EPI_BF16, y, **R.kwargs(1))  # no arrive()
    torch.cuda.synchronize()
    assert nat.gemm_error_code(reset=True) == 8
    assert nat.gemm_error_code() == 0
    R.check_stores(1)  # this rank's own pieces were stored and counted all the same
    x = torch.randn(256, K, device="cuda").bfloat16()
    assert rel_err(nat.gemm(x, w), x.float() @ w.float().t()) < 1e-2


@pytest.mark.parametrize("tp,rank,rows,N,bn", [(2, 1, 256, 512, 0), (4, 2, 128, 1024, 0), (2, 0, 200, 96, 0),
                                               (2, 1, 512, 1024, 256), (4, 3, 256, 768, 256)])
def test_peer_rs_epilogue_stand_in(nat, tp, rank, rows, N, bn):
    """GEMM -> reduce-scatter in one kernel (the wo / w2 GEMMs): output row r goes to slot `rank`
    of its owner r // rows; the owners' slot buffers are local stand-ins here. bn = 256 runs the
    256 x 256 tiles on CTA pairs."""
    from llmt.parallel.tp_p2p import EPI_PEER_RS
    K = 384
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(tp * rows, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    slots = [torch.full((tp * rows, N), 7.0, device="cuda", dtype=torch.bfloat16) for _ in range(tp)]
    ptrs = torch.tensor([s.data_ptr() for s in slots], dtype=torch.int64, device="cuda")
    nat.ext().gemm(x, w, False, True, EPI_PEER_RS, slots[rank], peer=ptrs, tp_rank=rank, rows_per_rank=rows, bn=bn)
    torch.cuda.synchronize()
    assert nat.gemm_error_code() == 0
    ref = x.float() @ w.float().t()
    for q in range(tp):
        mine = slots[q][rank * rows:(rank + 1) * rows]
        assert rel_err(mine, ref[q * rows:(q + 1) * rows]) < 1e-2
        other = torch.cat([slots[q][:rank * rows], slots[q][(rank + 1) * rows:]])
        assert (other == 7.0).all(), "rows written outside this rank's slot"
