"""The tcgen05 operand conventions the SSD kernels are built on, checked on the
GPU before anything depends on them: 128-byte-swizzled TMA tiles read as
K-major and MN-major MMA operands, a thread-written swizzled tile, fp32
accumulation in tensor memory.  Each mode is one 128-row bf16 GEMM compared
with a float64 product of the same bf16 inputs."""

import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

# test-only library built by ema-kernels_b200/build.py next to its source
_SELFTEST = os.path.join(os.path.dirname(os.path.abspath(__file__)), "native", "libema_selftest_b200.so")


def _selftest_lib():
    lib = ctypes.CDLL(_SELFTEST)
    lib.tc_selftest_gemm.restype = ctypes.c_int
    lib.tc_selftest_gemm.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 5
    lib.tc_selftest_last_error.restype = ctypes.c_char_p
    return lib


def _run(mode, a, b, n):
    from kernels import _lib
    st = _selftest_lib()
    d = torch.full((128, n), float("nan"), device="cuda", dtype=torch.float32)
    status = torch.zeros(1, device="cuda", dtype=torch.int32)
    rc = st.tc_selftest_gemm(mode, a.data_ptr(), b.data_ptr(), d.data_ptr(), status.data_ptr(),
                             _lib.stream_ptr(a.device))
    assert rc == 0, st.tc_selftest_last_error().decode()
    torch.cuda.synchronize()
    assert int(status.item()) == 0, "device-side wait timed out"
    return d


@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_tcgen05_gemm_modes(mode):
    g = torch.Generator(device="cuda").manual_seed(mode)
    a = torch.randn(128, 128, device="cuda", generator=g).bfloat16()
    n = 64 if mode == 1 else 128
    b = torch.randn(128, n, device="cuda", generator=g).bfloat16()
    if mode == 1:
        ref = a.double() @ b.double()
    elif mode == 2:
        ref = a.double().t() @ b.double()
    else:
        b = torch.randn(128, 128, device="cuda", generator=g).bfloat16()
        ref = a.double() @ b.double().t()
    d = _run(mode, a.contiguous(), b.contiguous(), n)
    torch.testing.assert_close(d.double(), ref, rtol=1e-5, atol=1e-4)


def test_tcgen05_m64_accumulator_lanes():
    """An M = 64 MMA (cta_group::1) writes row r of D to tensor-memory lane
    32 (r // 16) + r % 16: the first 16 lanes of each warp's lane quarter."""
    g = torch.Generator(device="cuda").manual_seed(9)
    a = torch.randn(64, 128, device="cuda", generator=g).bfloat16().contiguous()
    b = torch.randn(64, 128, device="cuda", generator=g).bfloat16().contiguous()
    d = _run(4, a, b, 64)  # all 128 lanes x 64 columns, zeroed before the MMA
    ref = a.double() @ b.double().t()
    lanes = torch.tensor([32 * (r // 16) + r % 16 for r in range(64)], device="cuda")
    torch.testing.assert_close(d[lanes].double(), ref, rtol=1e-5, atol=1e-4)
    others = torch.ones(128, dtype=torch.bool, device="cuda")
    others[lanes] = False
    assert float(d[others].abs().max()) == 0.0
