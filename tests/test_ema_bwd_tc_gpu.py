"""GPU parity of the tensor-core (tcgen05) EMA backward -- bf16, headdim 64,
128-token chunks, the path the autograd op takes at chunk_size 256 -- against
the float64 oracle and against the CUDA-core backward on the same inputs.
Both decay forms: dt (benchmark configs 2 and 4) and the reference form
(compute_dpx).  Steep decays exercise the per-element (wide group) decay
factors; ragged lengths, initial / final state gradients and the last-token
gradient the boundary terms."""

import math

import numpy as np
import pytest
import torch

from _tol import assert_lowp_close, assert_reference_rule
from oracle import ema_oracle as eo

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _tensor_core_path_and_status():
    from kernels import _lib
    prev = _lib.lib.ema_set_tensor_core_path(1)
    yield
    _lib.lib.ema_set_tensor_core_path(prev)
    assert _lib.device_status(clear=True) == 0, "a device-side wait timed out"


def _tc(enable):
    from kernels import _lib
    return _lib.lib.ema_set_tensor_core_path(1 if enable else 0)


def _dt_case(B, L, H, seed, dt_range, a_log):
    x, dt, A, dy = eo.make_dt_inputs(B, L, H, 64, seed=seed, dt_range=dt_range, a_log_range=a_log)
    tx = torch.from_numpy(x).to(torch.bfloat16)
    tdy = torch.from_numpy(dy).to(torch.bfloat16)
    rng = np.random.default_rng(seed + 100)
    init = rng.standard_normal((B, H, 64)).astype(np.float32)
    dfin = rng.standard_normal((B, H, 64)).astype(np.float32)
    return tx, torch.from_numpy(dt), torch.from_numpy(A), tdy, init, dfin


DT_CASES = [
    (2, 1000, 3, 1, (1e-3, 1e-1), (0.0, math.log(16.0))),   # ragged last chunk
    (1, 4096, 4, 2, (1e-3, 1e-1), (0.0, math.log(16.0))),   # config 2 regime, 32 chunks per chain
    (2, 640, 2, 3, (1e-2, 1.0), (math.log(4.0), math.log(16.0))),  # steep: wide decay groups
    (1, 2048, 2, 4, (1e-4, 1e-3), (0.0, math.log(2.0))),    # slow decay: L ~ 1 everywhere
    (3, 128, 5, 5, (1e-3, 1e-1), (0.0, math.log(16.0))),    # one chunk per chain
    (1, 1, 2, 6, (1e-3, 1e-1), (0.0, math.log(16.0))),      # a single token
]


@pytest.mark.parametrize("B,L,H,seed,dtr,alog", DT_CASES)
def test_dt_form_matches_oracle_and_cuda_core_kernel(B, L, H, seed, dtr, alog):
    from kernels.ema_chunk_scan import ema_chunk_scan_bwd, ema_chunk_scan_fwd
    tx, tdt, tA, tdy, init, dfin = _dt_case(B, L, H, seed, dtr, alog)
    x, dt, A, dy = (t.to(DEV) for t in (tx, tdt, tA, tdy))
    ti, tf = torch.from_numpy(init).to(DEV), torch.from_numpy(dfin).to(DEV)
    _, states, _ = ema_chunk_scan_fwd(x, dt, A, 128, initial_states=ti, return_final_states=True)
    _tc(True)
    got = ema_chunk_scan_bwd(x, dt, A, states, dy, 128, d_final_states=tf, need_d_initial=True)
    torch.cuda.synchronize()
    _tc(False)
    core = ema_chunk_scan_bwd(x, dt, A, states, dy, 128, d_final_states=tf, need_d_initial=True)
    torch.cuda.synchronize()
    _tc(True)
    g = eo.ema_dt_bwd(tx.float().numpy(), tdt.numpy(), tA.numpy(), tdy.float().numpy(), initial_state=init,
                      d_final_state=dfin)
    for name, k, c in zip(("dx", "ddt", "dA", "d_init"), got, core):
        ref = g["d_initial_state"] if name == "d_init" else g[name]
        assert_lowp_close(k, ref, name)
        assert_reference_rule(k, ref, name)
        assert_lowp_close(k, c.float().cpu().numpy(), name + " vs CUDA-core kernel")
    if L >= 64:
        # the switch selected a different kernel: the results differ in the low bits
        assert not torch.equal(got[1], core[1]), "tensor-core and CUDA-core paths gave bitwise equal ddt"


def test_dt_form_through_autograd_at_chunk_256():
    """The autograd op at chunk 256 runs the backward on 128-token chunks
    (the tensor-core kernel here): gradients against the oracle."""
    from kernels.ema_chunk_scan import ema_chunk_scan_combined
    tx, tdt, tA, tdy, _, _ = _dt_case(2, 1500, 4, 11, (1e-3, 1e-1), (0.0, math.log(16.0)))
    x = tx.to(DEV).requires_grad_()
    dt = tdt.to(DEV).requires_grad_()
    A = tA.to(DEV).requires_grad_()
    y = ema_chunk_scan_combined(x, dt, A, chunk_size=256)
    y.backward(tdy.to(DEV))
    g = eo.ema_dt_bwd(tx.float().numpy(), tdt.numpy(), tA.numpy(), tdy.float().numpy())
    assert_lowp_close(x.grad, g["dx"], "dx")
    assert_lowp_close(dt.grad, g["ddt"], "ddt")
    assert_lowp_close(A.grad, g["dA"], "dA")


@pytest.mark.parametrize("L", [777, 2048, 128])
def test_reference_form_compute_dpx(L):
    """compute_dpx at chunk 128 with bf16 x: the reference-form tensor-core
    kernel, with the final-state and last-token gradients and the initial
    state gradient; dl (the reference's "dA") against the oracle."""
    from kernels.forward.ema_ssd_fwd import ema_fwd_triton
    from kernels.backward.ema_ssd_combined import compute_dpx
    rng = np.random.default_rng(L)
    B, H, P, Q = 2, 3, 64, 128
    x = torch.from_numpy(rng.standard_normal((B, L, H, P)).astype(np.float32)).to(torch.bfloat16)
    do = torch.from_numpy(rng.standard_normal((B, L, H, P)).astype(np.float32)).to(torch.bfloat16)
    dA = (-rng.random((B, H, L)) * 0.5).astype(np.float32)
    dfin = rng.standard_normal((B, H, P)).astype(np.float32)
    dlast = rng.standard_normal((B, H, P)).astype(np.float32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    _, st, cs, css = ema_fwd_triton(x.to(DEV), dA=t(dA), chunk_size=Q, store_states=True, store_da_cs=True,
                                    store_da_cs_sum=True)
    states = st.squeeze(3).permute(0, 2, 3, 1)
    dx, dl, dis = compute_dpx(x.to(DEV), cs, css, states, do.to(DEV), d_ossm_state=t(dfin),
                              d_ox_state=t(dlast), chunk_size=Q, has_input_state=True)
    f = eo.ema_fwd(x.float().numpy(), dA, Q)
    r = eo.ema_bwd(x.float().numpy(), f["da_cs"], f["da_cs_sum"], f["states"][:, :, :, 0, :].transpose(0, 2, 3, 1),
                   do.float().numpy(), d_ossm_state=dfin, d_ox_state=dlast, chunk_size=Q, has_input_state=True)
    assert_lowp_close(dx, r["dx"], "dx")
    assert_lowp_close(dl, r["dA"], "dl")
    assert_reference_rule(dl, r["dA"], "dl")
    assert_lowp_close(dis, r["d_issm_state"], "d_issm_state")


def test_strided_dx_and_inputs():
    """Non-contiguous x / dy (a head slice of a wider tensor): the tensor maps
    carry the strides."""
    from kernels.ema_chunk_scan import ema_chunk_scan_bwd, ema_chunk_scan_fwd
    tx, tdt, tA, tdy, init, dfin = _dt_case(2, 700, 6, 21, (1e-3, 1e-1), (0.0, math.log(16.0)))
    xw, dyw = tx.to(DEV), tdy.to(DEV)
    x, dy = xw[:, :, 1:4], dyw[:, :, 1:4]  # heads 1..3 of 6: strides of the wide tensors
    dt, A = tdt[:, :, 1:4].contiguous().to(DEV), tA[1:4].contiguous().to(DEV)
    _, states, _ = ema_chunk_scan_fwd(x, dt, A, 128, return_final_states=True)
    dx, ddt, dA, _ = ema_chunk_scan_bwd(x, dt, A, states, dy, 128)
    g = eo.ema_dt_bwd(tx[:, :, 1:4].float().numpy(), tdt[:, :, 1:4].numpy(), tA[1:4].numpy(),
                      tdy[:, :, 1:4].float().numpy())
    assert_lowp_close(dx, g["dx"], "dx")
    assert_lowp_close(ddt, g["ddt"], "ddt")
    assert_lowp_close(dA, g["dA"], "dA")
