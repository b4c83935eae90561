"""ema_fwd_launch_noalloc: the EMA forward for callers that cannot allocate device memory.

Such callers (an FFI host with no device allocator, a runtime that forbids
allocation after start-up) get the look-back scratch from a static device
array inside the library instead of passing a workspace.  This test calls the
entry point through the C ABI twice in a row and checks each result against
the ordinary ema_fwd_launch (caller-provided workspace) within the tolerances
the other parity tests use.  Between and after those two calls it runs a
second shape (other tile count and headdim block, so the look-back records
move over bytes an earlier call left behind) and checks that too, and it
reads the array's status word through ema_noalloc_status after every call.
The file sorts last so a run that stops at the first failure has already run
every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

from _tol import assert_fp32_close, assert_lowp_close
from oracle import ema_oracle as eo

pytestmark = pytest.mark.gpu


def _args(_lib, x, dt, A, out, states, workspace=None):
    a = _lib.EmaFwdArgs()
    B, L, H, P = x.shape
    a.batch, a.seqlen, a.nheads, a.headdim, a.chunk_size = B, L, H, P, 256
    a.dtype = _lib.DTYPE_CODES[x.dtype]
    a.x, a.x_stride = x.data_ptr(), _lib.strides3(x)
    a.out, a.out_stride = out.data_ptr(), _lib.strides3(out)
    a.dt, a.A = dt.data_ptr(), A.data_ptr()
    s = states.stride()
    a.states, a.states_stride = states.data_ptr(), (_lib._i64 * 4)(s[0], s[1], s[2], s[3])
    if workspace is not None:
        a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel()
    return a


def _status(_lib, stream):
    word = ctypes.c_uint32(0xFFFFFFFF)
    rc = _lib.lib.ema_noalloc_status(ctypes.byref(word), 0, stream)
    assert rc == 0, _lib.lib.ema_last_error().decode()
    return word.value


class _Case:
    """One shape: inputs, and the ordinary entry point's results to compare with."""

    def __init__(self, _lib, dev, stream, B, L, H, P, seed):
        x, dt, A, _ = eo.make_dt_inputs(B, L, H, P, seed=seed)
        self.x = torch.from_numpy(x).to(dev, torch.bfloat16)
        self.dt = torch.from_numpy(dt).to(dev)
        self.A = torch.from_numpy(A).to(dev)
        self.shape = (B, L, H, P)
        self.nc = -(-L // 256)
        ws = torch.zeros(_lib.lib.ema_scan_workspace_size(B, L, H, P, 256), dtype=torch.uint8, device=dev)
        self.y_ref = torch.empty_like(self.x)
        self.st_ref = torch.empty(B, self.nc, H, P, dtype=torch.float32, device=dev)
        a = _args(_lib, self.x, self.dt, self.A, self.y_ref, self.st_ref, ws)
        _lib.check(_lib.lib.ema_fwd_launch(a, stream), "ema_fwd_launch")

    def run_noalloc(self, _lib, fn, dev, stream, what):
        B, L, H, P = self.shape
        y = torch.full_like(self.x, float("nan"))
        st = torch.full((B, self.nc, H, P), float("nan"), dtype=torch.float32, device=dev)
        rc = fn(_args(_lib, self.x, self.dt, self.A, y, st), stream)
        assert rc == 0, _lib.lib.ema_last_error().decode()
        torch.cuda.synchronize(dev)
        assert _status(_lib, stream) == 0, f"{what}: device status word set"
        assert_lowp_close(y, self.y_ref, f"{what}: y")
        assert_fp32_close(st, self.st_ref, f"{what}: chunk start states")
        return y


def test_noalloc_forward_matches_workspace_forward_twice():
    from kernels import _lib
    fn = _lib.lib.ema_fwd_launch_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(_lib.EmaFwdArgs), ctypes.c_void_p]
    _lib.lib.ema_noalloc_status.restype = ctypes.c_int
    _lib.lib.ema_noalloc_status.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int32, ctypes.c_void_p]

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    main = _Case(_lib, dev, stream, 2, 2048, 8, 64, seed=21)
    # fewer tiles, the 128-channel block and a ragged last chunk: its records
    # sit at other offsets of the same static array
    other = _Case(_lib, dev, stream, 1, 1000, 4, 128, seed=22)

    y = main.run_noalloc(_lib, fn, dev, stream, "call 0")
    other.run_noalloc(_lib, fn, dev, stream, "second shape, first call")
    y = main.run_noalloc(_lib, fn, dev, stream, "call 1")
    other.run_noalloc(_lib, fn, dev, stream, "second shape, second call")

    # both agree with the float64 recurrence as well
    r = eo.ema_dt_fwd(main.x.float().cpu().numpy(), main.dt.cpu().numpy(), main.A.cpu().numpy())
    assert_lowp_close(y, r["y"], "y vs oracle")

    # a shape whose scratch exceeds the static array is refused, with the limit in the message
    big = _args(_lib, main.x, main.dt, main.A, y, main.st_ref)
    big.seqlen = 1 << 22
    assert fn(big, stream) == 3
    msg = _lib.lib.ema_last_error().decode()
    assert "static array holds" in msg and str(4 << 20) in msg
    assert _status(_lib, stream) == 0
