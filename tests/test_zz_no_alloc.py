"""The allocation-free RMSNorm backward (C symbol llmt_rmsnorm_bwd_noalloc).

It exists for callers that cannot allocate device memory where they run the backward; its
scratch is a fixed static device array inside the library. This test calls it through the
exported C symbol (ctypes, no PyTorch binding in between) and checks its outputs against
the regular entry point, which allocates its scratch through PyTorch, on two calls in a row
(the second accumulating into dw, and reusing the shared scratch array). The file is named
to be collected last."""
import ctypes

import pytest
import torch

from tests.helpers import rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    from llmt.ops import native
    mod = native.ext()._mod
    so = ctypes.CDLL(mod.__file__)
    fn = so.llmt_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 8 + [ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    so.llmt_noalloc_last_error.restype = ctypes.c_char_p
    return so, native


def _call(so, dy, s, w, rstd, ds_in, ds, ds16, dw, accumulate):
    N, D = s.shape
    stream = torch.cuda.current_stream().cuda_stream
    return so.llmt_rmsnorm_bwd_noalloc(dy.data_ptr(), s.data_ptr(), w.data_ptr(), rstd.data_ptr(),
                                       ds_in.data_ptr() if ds_in is not None else None, ds.data_ptr(),
                                       ds16.data_ptr() if ds16 is not None else None, dw.data_ptr(), N, D,
                                       int(accumulate), stream)


# (4096, 4096) and (4096, 8192) want more partial rows than the fixed scratch holds, so the grid is
# cut to 256 and 128 CTAs and each CTA walks more rows.
@pytest.mark.parametrize("N,D", [(4096, 1024), (300, 768), (64, 8192), (4096, 4096), (4096, 8192)])
def test_noalloc_matches_regular_entry_point_twice(lib, N, D):
    so, native = lib
    g = torch.Generator(device="cuda").manual_seed(0)
    r = torch.randn(N, D, device="cuda", generator=g)
    a = torch.randn(N, D, device="cuda", generator=g).bfloat16()
    w = 1 + 0.1 * torch.randn(D, device="cuda", generator=g)
    _, s, rstd = native.add_rmsnorm_fwd(a, r, w, 1e-5)
    dw_ref = torch.zeros(D, device="cuda")
    dw = torch.zeros(D, device="cuda")
    for call in range(2):
        dy = torch.randn(N, D, device="cuda", generator=g).bfloat16()
        ds_in = torch.randn(N, D, device="cuda", generator=g)
        ds_ref, ds16_ref = native.rmsnorm_bwd(dy, s, w, rstd, ds_in, dw_ref, accumulate=call > 0)
        ds = torch.empty_like(s)
        ds16 = torch.empty(N, D, device="cuda", dtype=torch.bfloat16)
        rc = _call(so, dy, s, w, rstd, ds_in, ds, ds16, dw, accumulate=call > 0)
        torch.cuda.synchronize()
        assert rc == 0, so.llmt_noalloc_last_error()
        assert rel_err(ds, ds_ref) < 1e-5
        assert rel_err(ds16, ds16_ref) < 1e-2
        assert rel_err(dw, dw_ref) < 1e-4


def test_noalloc_without_optional_inputs(lib):
    """ds_in and ds16 are optional (NULL): no incoming residual gradient, no bf16 copy of ds."""
    so, native = lib
    N, D = 1000, 2048
    g = torch.Generator(device="cuda").manual_seed(1)
    r = torch.randn(N, D, device="cuda", generator=g)
    a = torch.randn(N, D, device="cuda", generator=g).bfloat16()
    w = 1 + 0.1 * torch.randn(D, device="cuda", generator=g)
    _, s, rstd = native.add_rmsnorm_fwd(a, r, w, 1e-5)
    dy = torch.randn(N, D, device="cuda", generator=g).bfloat16()
    dw_ref, dw = torch.zeros(D, device="cuda"), torch.zeros(D, device="cuda")
    ds_ref, _ = native.rmsnorm_bwd(dy, s, w, rstd, None, dw_ref, accumulate=False, write_ds16=False)
    ds = torch.empty_like(s)
    rc = _call(so, dy, s, w, rstd, None, ds, None, dw, accumulate=False)
    torch.cuda.synchronize()
    assert rc == 0, so.llmt_noalloc_last_error()
    assert rel_err(ds, ds_ref) < 1e-5
    assert rel_err(dw, dw_ref) < 1e-4


def test_noalloc_rejects_oversized_width(lib):
    so, _ = lib
    D = 8200  # beyond the 8192 maximum
    t = torch.zeros(8, D, device="cuda")
    b = torch.zeros(8, D, device="cuda", dtype=torch.bfloat16)
    v = torch.zeros(D, device="cuda")
    n = torch.zeros(8, device="cuda")
    rc = _call(so, b, t, v, n, None, t, None, v, accumulate=0)
    assert rc != 0
    assert b"8192" in so.llmt_noalloc_last_error()
