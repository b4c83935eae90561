"""ema_fwd_launch_noalloc: the EMA forward for callers that cannot allocate device memory.

Such callers (an FFI host with no device allocator, a runtime that forbids
allocation after start-up) get the look-back scratch from a static device
array inside the library instead of passing a workspace.  This test calls the
entry point through the C ABI twice in a row and checks each result against
the ordinary ema_fwd_launch (caller-provided workspace) within the tolerances
the other parity tests use.  The file sorts last so a run that stops at the
first failure has already run every other test.
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


def test_noalloc_forward_matches_workspace_forward_twice():
    from kernels import _lib
    fn = _lib.lib.ema_fwd_launch_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(_lib.EmaFwdArgs), ctypes.c_void_p]

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, L, H, P = 2, 2048, 8, 64
    x, dt, A, _ = eo.make_dt_inputs(B, L, H, P, seed=21)
    x = torch.from_numpy(x).to(dev, torch.bfloat16)
    dt = torch.from_numpy(dt).to(dev)
    A = torch.from_numpy(A).to(dev)
    nc = L // 256
    stream = torch.cuda.current_stream(dev).cuda_stream

    # the ordinary entry point, with a caller-provided zeroed workspace
    ws = torch.zeros(_lib.lib.ema_scan_workspace_size(B, L, H, P, 256), dtype=torch.uint8, device=dev)
    y_ref = torch.empty_like(x)
    st_ref = torch.empty(B, nc, H, P, dtype=torch.float32, device=dev)
    _lib.check(_lib.lib.ema_fwd_launch(_args(_lib, x, dt, A, y_ref, st_ref, ws), stream), "ema_fwd_launch")

    for call in range(2):
        y = torch.full_like(x, float("nan"))
        st = torch.full((B, nc, H, P), float("nan"), dtype=torch.float32, device=dev)
        rc = fn(_args(_lib, x, dt, A, y, st), stream)
        assert rc == 0, _lib.lib.ema_last_error().decode()
        torch.cuda.synchronize(dev)
        assert_lowp_close(y, y_ref, f"call {call}: y")
        assert_fp32_close(st, st_ref, f"call {call}: chunk start states")

    # both agree with the float64 recurrence as well
    r = eo.ema_dt_fwd(x.float().cpu().numpy(), dt.cpu().numpy(), A.cpu().numpy())
    assert_lowp_close(y, r["y"], "y vs oracle")

    # a shape whose scratch exceeds the static array is refused, with the limit in the message
    big = _args(_lib, x, dt, A, y, st)
    big.seqlen = 1 << 22
    assert fn(big, stream) == 3
    msg = _lib.lib.ema_last_error().decode()
    assert "static array holds" in msg and str(4 << 20) in msg
