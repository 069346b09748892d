"""Failure detection on the device without faulting the GPU: a cross-rank flag wait
whose peer never arrives runs out its bounded spin, records an error in the status
word and returns; the context stays usable."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_barrier_timeout_reports_status_and_context_survives():
    from drivedit_b200.ops._ext import check_device_status, device_status, ext, reset_device_status
    reset_device_status()
    world = 2
    buf = torch.zeros(2 * world, dtype=torch.int32, device="cuda")   # world u32 flags + world f32 payloads
    ptr = buf.data_ptr()
    # both "peers" are this buffer: our own arrival lands, the second flag is never set
    table = torch.tensor([ptr, ptr], dtype=torch.int64, device="cuda")
    ext().xrank_barrier(table, ptr, 0, world, 1, None)
    torch.cuda.synchronize()
    assert device_status() == 4  # peer timeout
    with pytest.raises(RuntimeError):
        check_device_status()
    assert device_status() == 0
    # the context is still healthy: a normal kernel runs and is correct
    x = torch.randn(256, 256, device="cuda")
    assert torch.allclose(x @ x.t(), (x.double() @ x.double().t()).float(), atol=1e-3)
