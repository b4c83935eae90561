"""GPU parity of the tensor-core (tcgen05) EMA forward -- dt form, bf16,
headdim 64, 128-token chunks -- against the float64 oracle and against the
CUDA-core forward on the same inputs.  y carries one bf16 rounding of the decay
matrix and of dt x, as the reference's forward rounds its decay matrix before
tl.dot (kernels/forward/ema_ssd_fwd.py:361-368); the chunk start states and
the final state are summed in fp32 and are held to the fp32 bound.  Steep
decays exercise the per-element (wide group) decay factors, ragged lengths the
clipped last tile, and the autograd pair the CUDA-core backward on the states
this forward saves."""

import math

import numpy as np
import pytest
import torch

from _tol import assert_fp32_close, assert_lowp_close, assert_reference_rule
from oracle import ema_oracle as eo

pytestmark = pytest.mark.gpu
DEV = "cuda"
FWD_TC = 2  # ema_set_tensor_core_path bit 1: the tensor-core forward


@pytest.fixture(autouse=True)
def _forward_path_and_status():
    from kernels import _lib
    prev = _lib.lib.ema_set_tensor_core_path(FWD_TC)
    yield
    _lib.lib.ema_set_tensor_core_path(prev)
    assert _lib.device_status(clear=True) == 0, "a device-side wait timed out"


def _path(bits):
    from kernels import _lib
    return _lib.lib.ema_set_tensor_core_path(bits)


def _case(B, L, H, seed, dt_range, a_log):
    x, dt, A, dy = eo.make_dt_inputs(B, L, H, 64, seed=seed, dt_range=dt_range, a_log_range=a_log)
    init = np.random.default_rng(seed + 100).standard_normal((B, H, 64)).astype(np.float32)
    return (torch.from_numpy(x).to(torch.bfloat16), torch.from_numpy(dt), torch.from_numpy(A),
            torch.from_numpy(dy).to(torch.bfloat16), init)


CASES = [
    (2, 1000, 3, 1, (1e-3, 1e-1), (0.0, math.log(16.0))),   # ragged last chunk
    (1, 4096, 4, 2, (1e-3, 1e-1), (0.0, math.log(16.0))),   # config 2 regime, 32 chunks per chain
    (2, 640, 2, 3, (1e-2, 1.0), (math.log(4.0), math.log(16.0))),  # steep: wide decay groups
    (1, 2048, 2, 4, (1e-4, 1e-3), (0.0, math.log(2.0))),    # slow decay: L ~ 1 everywhere
    (3, 128, 5, 5, (1e-3, 1e-1), (0.0, math.log(16.0))),    # one chunk per chain
    (1, 1, 2, 6, (1e-3, 1e-1), (0.0, math.log(16.0))),      # a single token
]


@pytest.mark.parametrize("B,L,H,seed,dtr,alog", CASES)
def test_forward_matches_oracle_and_cuda_core_kernel(B, L, H, seed, dtr, alog):
    from kernels.ema_chunk_scan import ema_chunk_scan_fwd
    tx, tdt, tA, _, init = _case(B, L, H, seed, dtr, alog)
    x, dt, A = (t.to(DEV) for t in (tx, tdt, tA))
    ti = torch.from_numpy(init).to(DEV)
    y, states, fin = ema_chunk_scan_fwd(x, dt, A, 128, initial_states=ti, return_final_states=True)
    torch.cuda.synchronize()
    _path(0)
    yc, statesc, finc = ema_chunk_scan_fwd(x, dt, A, 128, initial_states=ti, return_final_states=True)
    torch.cuda.synchronize()
    _path(FWD_TC)
    r = eo.ema_dt_fwd(tx.float().numpy(), tdt.numpy(), tA.numpy(), initial_state=init)
    assert_lowp_close(y, r["y"], "y")
    assert_reference_rule(y, r["y"], "y")
    assert_lowp_close(y, yc.float().cpu().numpy(), "y vs CUDA-core kernel")
    # the state entering chunk c is the oracle's state after token 128 c - 1
    ref_states = np.concatenate([init[:, None], r["y"][:, 127:L - 1:128]], axis=1) if L > 128 else init[:, None]
    assert_fp32_close(states, ref_states, "chunk states")
    assert_fp32_close(states, statesc.cpu().numpy(), "chunk states vs CUDA-core kernel")
    assert_fp32_close(fin, r["final_state"], "final state")
    if L >= 64:
        # the switch selected a different kernel: y differs in the low bits
        assert not torch.equal(y, yc), "tensor-core and CUDA-core forwards gave bitwise equal y"


def test_autograd_pair_on_tensor_core_forward_states():
    """ema_chunk_scan_combined at chunk 128 with the tensor-core forward: the
    CUDA-core backward runs on the fp32 states this forward saved; every
    gradient within the bf16 tolerance of the oracle (ddt is the precision-
    sensitive one: it multiplies the states by the arriving gradient)."""
    from kernels.ema_chunk_scan import ema_chunk_scan_combined
    tx, tdt, tA, tdy, init = _case(2, 3000, 4, 7, (1e-3, 1e-1), (0.0, math.log(16.0)))
    leaves = [t.to(DEV).requires_grad_() for t in (tx, tdt, tA)]
    y = ema_chunk_scan_combined(*leaves, 128)
    y.backward(tdy.to(DEV))
    torch.cuda.synchronize()
    xf = tx.float().numpy()
    r = eo.ema_dt_fwd(xf, tdt.numpy(), tA.numpy())
    g = eo.ema_dt_bwd(xf, tdt.numpy(), tA.numpy(), tdy.float().numpy())
    assert_lowp_close(y, r["y"], "y")
    for name, t in (("dx", leaves[0]), ("ddt", leaves[1])):
        assert_lowp_close(t.grad, g[name], name)
        assert_reference_rule(t.grad, g[name], name)
    e = float(np.abs(leaves[2].grad.double().cpu().numpy() - g["dA"]).max() / np.abs(g["dA"]).max())
    assert e <= 1e-3, f"dA: normwise relative error {e:.3e}"


def test_uncovered_shapes_fall_back_to_the_cuda_core_kernel():
    """Where the tensor-core forward does not apply (headdim 32, chunk 256,
    fp32 x) the switch leaves the CUDA-core forward in place: the call
    succeeds and agrees with the switch off."""
    from kernels.ema_chunk_scan import ema_chunk_scan_fwd
    for (P, Q, dtype) in ((32, 128, torch.bfloat16), (64, 256, torch.bfloat16), (64, 128, torch.float32)):
        x, dt, A, _ = eo.make_dt_inputs(1, 700, 2, P, seed=11)
        tx = torch.from_numpy(x).to(dtype).to(DEV)
        tdt, tA = torch.from_numpy(dt).to(DEV), torch.from_numpy(A).to(DEV)
        y_on, s_on, _ = ema_chunk_scan_fwd(tx, tdt, tA, Q)
        _path(0)
        y_off, s_off, _ = ema_chunk_scan_fwd(tx, tdt, tA, Q)
        _path(FWD_TC)
        torch.cuda.synchronize()
        # the forward combines predecessor records in whichever form lands first:
        # equal up to fp32 rounding, not bit for bit
        torch.testing.assert_close(y_on, y_off, rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(s_on, s_off, rtol=1e-5, atol=1e-5)
