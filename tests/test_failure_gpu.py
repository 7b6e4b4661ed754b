"""A device-side wait that runs out, without a fault: the flag barrier kernel waits for a peer
slot that nothing ever sets, gives up after its bound (5 s), records an error code and
returns; the host reads the code and the context stays usable."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_flag_barrier_times_out_and_reports():
    from llmt.ops import native as N
    from llmt.parallel.health import DeviceWaitTimeout, check_device_errors
    C = N.ext()
    C.dp_error_code(True)
    mine = torch.zeros(64, dtype=torch.int32, device="cuda")   # this rank's signal pad
    other = torch.zeros(64, dtype=torch.int32, device="cuda")  # a "peer" pad: never written by a peer
    pads = torch.tensor([mine.data_ptr(), other.data_ptr()], dtype=torch.int64, device="cuda")
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.dp_barrier(pads, mine.data_ptr(), epoch, 0, 2, 900)  # rank 0 of 2: slot [1] of its pad stays 0
    torch.cuda.synchronize()
    assert C.dp_error_code(False) == 901  # code + the peer it waited for
    with pytest.raises(DeviceWaitTimeout):
        check_device_errors(reset=True)
    x = torch.randn(1024, device="cuda")
    y = torch.empty(1024, dtype=torch.bfloat16, device="cuda")
    N.cast_bf16(x, y)  # the context still runs kernels
    torch.cuda.synchronize()
    assert torch.allclose(y.float(), x, rtol=1e-2, atol=1e-2)
