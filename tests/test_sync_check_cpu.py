"""Sync-check debug mode (``drivedit_b200.ops._ext.SyncChecked``) on a stand-in module:
every entry point is bracketed by a synchronize and a status read, faults are attributed
to the entry point during (or before) which they were raised, and queries pass through."""
import pytest
import torch

from drivedit_b200.ops._ext import KernelFault, SyncChecked


class FakeExt:
    def __init__(self):
        self.status = 0
        self.log = []

    def read_status(self):
        self.log.append("read_status")
        return self.status

    def reset_status(self):
        self.status = 0

    def launch_count(self):
        return 7

    def gemm(self, a, b):
        self.log.append("gemm")
        return a @ b

    def bad_kernel(self, x):
        self.status = 2  # a bounded wait ran out inside this launch
        return x


def test_calls_are_bracketed_and_recorded(tmp_path):
    syncs = []
    fake = FakeExt()
    log = tmp_path / "calls.log"
    m = SyncChecked(fake, str(log), sync=lambda: syncs.append(1))
    a = torch.ones(2, 3)
    out = m.gemm(a, torch.ones(3, 4))
    assert torch.equal(out, a @ torch.ones(3, 4))
    assert len(syncs) == 2 and fake.log == ["read_status", "gemm", "read_status"]
    assert m.launch_count() == 7 and len(syncs) == 2      # queries are not bracketed
    assert m.calls == 1 and "gemm((2, 3):float32, (3, 4):float32)" in m.recent[0]
    assert log.read_text().splitlines() == ["#1 gemm((2, 3):float32, (3, 4):float32)"]


def test_status_raised_by_an_entry_point_names_it():
    fake = FakeExt()
    m = SyncChecked(fake, sync=lambda: None)
    m.gemm(torch.ones(1, 1), torch.ones(1, 1))
    with pytest.raises(KernelFault, match=r"device status 2 in #2 bad_kernel.*#1 gemm"):
        m.bad_kernel(torch.zeros(3))
    assert fake.status == 0  # reset after the report


def test_error_from_earlier_work_is_reported_before_the_call():
    calls = {"n": 0}

    def sync():
        calls["n"] += 1
        if calls["n"] == 3:   # the first sync of the second call: raised by work before it
            raise RuntimeError("CUDA error: unspecified launch failure")

    m = SyncChecked(FakeExt(), sync=sync)
    m.gemm(torch.ones(1, 1), torch.ones(1, 1))
    with pytest.raises(KernelFault, match=r"CUDA error before #2 gemm"):
        m.gemm(torch.ones(1, 1), torch.ones(1, 1))
