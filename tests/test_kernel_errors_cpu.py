"""The error path of the GEMM and attention kernels' bounded waits, on the
host: the op wrappers check the device's kernel error record under
NAB_CHECK=1, and a non-zero record raises KernelError naming the kernel. The
native side is faked (no GPU here); the GPU tests check that the record stays
zero after good launches."""

import pytest

from numa_allreduce_b200.ops import errors, gemm as gemm_mod


class FakeOps:
    def __init__(self, code=0, stage=11):
        self.code = code
        self.stage = stage
        self.calls = []

    def kernel_error_code(self):
        return self.code

    def kernel_error_state(self):
        return [self.code, 0xFFFFFFFF, 0xFFFFFFFF, self.stage, 5, 0, 3, 2]

    def kernel_error_reset(self):
        self.code = 0

    def gemm(self, *args):
        self.calls.append(("gemm", args))


@pytest.fixture
def fake(monkeypatch):
    ops = FakeOps()
    monkeypatch.setattr(errors._ext, "load", lambda: ops)
    return ops


def test_nonzero_record_raises_with_the_kernel_named(fake):
    errors.check_kernels(sync=False)  # clean record: no error
    fake.code = 1
    with pytest.raises(errors.KernelError, match="GEMM kernel: a wait timed out.*CTA 5.*2 waits"):
        errors.check_kernels(sync=False)
    fake.stage = 12
    with pytest.raises(errors.KernelError, match="attention kernel"):
        errors.check_kernels(sync=False)
    errors.reset_kernels()
    errors.check_kernels(sync=False)


def test_gemm_wrapper_checks_after_launch_only_under_nab_check(fake, monkeypatch):
    import torch

    checked = []
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: False)
    monkeypatch.setattr(errors, "check_kernels", lambda sync=True: checked.append(sync))
    monkeypatch.setattr(gemm_mod._ext, "load", lambda: fake)
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    w = torch.zeros(128, 64, dtype=torch.bfloat16)
    out = torch.zeros(4, 128, dtype=torch.bfloat16)
    monkeypatch.delenv("NAB_CHECK", raising=False)
    gemm_mod.gemm(x, w, out=out)
    assert fake.calls and checked == []
    monkeypatch.setenv("NAB_CHECK", "1")
    gemm_mod.gemm(x, w, out=out)
    gemm_mod.gemm_swiglu(x, w, out=torch.zeros(4, 64, dtype=torch.bfloat16))
    assert checked == [True, True]
