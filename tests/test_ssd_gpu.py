"""GPU parity of the Mamba-2 SSD kernels (benchmark configs 3 and 5 form)
against the float64 oracle (oracle/ssd_oracle.py, unpinned: the reference has
no SSD implementation of its own).  bf16 inputs, fp32 accumulation: the
tolerance is 2e-2 relative / 1e-2 absolute elementwise, applied to the oracle
run on the same bf16-rounded inputs."""

import numpy as np
import pytest
import torch

from _tol import assert_lowp_close, assert_reference_rule
from oracle import ssd_oracle as so

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(B, L, H, P, N, G, seed):
    x, dt, A, Bm, Cm, D, dy = so.make_ssd_inputs(B, L, H, P, N, ngroups=G, seed=seed)
    bf = lambda a: torch.from_numpy(a).to(torch.bfloat16)  # noqa: E731
    return bf(x), torch.from_numpy(dt), torch.from_numpy(A), bf(Bm), bf(Cm), torch.from_numpy(D), bf(dy)


def _f64(t):
    return t.float().double().numpy()


def _device_status_clear():
    import ctypes

    from kernels import _lib
    v = ctypes.c_uint32(0)
    _lib.check(_lib.lib.ssd_device_status(ctypes.byref(v), 1, _lib.stream_ptr(torch.device(DEV))), "ssd_device_status")
    return v.value


# (H / G) even -> the tcgen05 forward (128-token chunks, head pairs); odd -> the mma.sync forward
@pytest.mark.parametrize("L,H,G,with_states", [(200, 4, 2, True), (128, 2, 1, False), (64, 2, 2, True),
                                               (320, 4, 1, True), (96, 6, 3, False), (130, 3, 3, True)])
def test_ssd_forward_backward_match_oracle(L, H, G, with_states):
    from kernels.ssd_combined import ssd_chunk_scan_bwd, ssd_chunk_scan_fwd
    B, P, N = 2, 64, 128
    tx, tdt, tA, tB, tC, tD, tdy = _inputs(B, L, H, P, N, G, seed=L + H)
    rng = np.random.default_rng(7)
    s0 = rng.standard_normal((B, H, P, N)).astype(np.float32) * 0.5 if with_states else None
    dfin = rng.standard_normal((B, H, P, N)).astype(np.float32) * 0.5 if with_states else None
    x, dt, A, Bm, Cm, D, dy = (t.to(DEV) for t in (tx, tdt, tA, tB, tC, tD, tdy))
    init = torch.from_numpy(s0).to(DEV) if s0 is not None else None
    y, cst, fin = ssd_chunk_scan_fwd(x, dt, A, Bm, Cm, D, init, return_final_states=True)
    dfin_t = torch.from_numpy(dfin).to(DEV) if dfin is not None else None
    dx, ddt, dA, dB, dC, dD, dinit = ssd_chunk_scan_bwd(x, dt, A, Bm, Cm, cst, dy, D, dfin_t, need_d_initial=True)
    torch.cuda.synchronize()
    assert _device_status_clear() == 0

    args = (_f64(tx), tdt.double().numpy(), tA.double().numpy(), _f64(tB), _f64(tC))
    r = so.ssd_fwd(*args, D=tD.double().numpy(), initial_state=s0)
    g = so.ssd_bwd(*args, _f64(tdy), D=tD.double().numpy(), initial_state=s0, d_final_state=dfin)
    assert_lowp_close(y, r["y"], "y")
    assert_lowp_close(fin, r["final_state"], "final_state")
    # the saved state entering every 64-token chunk (what the backward reads)
    nc = cst.shape[1]
    ref_states = np.concatenate([s0[:, None] if s0 is not None else np.zeros((B, 1, H, P, N)),
                                 r["states"][:, 63::64][:, :nc - 1]], axis=1)
    assert_lowp_close(cst, ref_states, "chunk_states")
    for name, k in (("dx", dx), ("ddt", ddt), ("dB", dB), ("dC", dC), ("d_initial_state", dinit)):
        assert_lowp_close(k, g[name], name)
        assert_reference_rule(k, g[name], name)
    # per-head reductions over every token: normwise
    for name, k in (("dA", dA), ("dD", dD)):
        ref = g[name]
        e = float(np.abs(k.cpu().double().numpy() - ref).max() / max(np.abs(ref).max(), 1e-30))
        assert e <= 2e-2, f"{name}: normwise relative error {e:.3e}"


def test_mamba_call_form_autograd():
    """mamba_chunk_scan_combined(x, dt, A, B, C, chunk_size, D, dt_bias, dt_softplus) through
    autograd equals the direct launchers plus the softplus chain rule."""
    from kernels.ssd_combined import mamba_chunk_scan_combined, ssd_chunk_scan_bwd, ssd_chunk_scan_fwd
    B, L, H, P, N, G = 1, 192, 4, 64, 128, 1
    tx, tdt, tA, tB, tC, tD, tdy = _inputs(B, L, H, P, N, G, seed=3)
    x, dt_raw, A, Bm, Cm, D, dy = (t.to(DEV) for t in (tx, tdt, tA, tB, tC, tD, tdy))
    bias = torch.full((H,), -1.0, device=DEV)
    leaves = [t.clone().requires_grad_() for t in (x, dt_raw, A, Bm, Cm, D)]
    y = mamba_chunk_scan_combined(*leaves[:5], 256, D=leaves[5], dt_bias=bias, dt_softplus=True)
    y.backward(dy)
    dt = torch.nn.functional.softplus(dt_raw + bias)
    y2, cst, _ = ssd_chunk_scan_fwd(x, dt, A, Bm, Cm, D)
    dx, ddt, dA, dB, dC, dD, _ = ssd_chunk_scan_bwd(x, dt, A, Bm, Cm, cst, dy, D)
    assert torch.equal(y, y2)
    torch.testing.assert_close(leaves[0].grad, dx, rtol=0, atol=0)
    torch.testing.assert_close(leaves[1].grad, ddt * torch.sigmoid(dt_raw + bias), rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(leaves[3].grad, dB.to(torch.bfloat16), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(leaves[2].grad, dA, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(leaves[5].grad, dD, rtol=1e-3, atol=1e-3)


def test_mamba_call_form_z_gating_and_dt_limit():
    """mamba_chunk_scan_combined with z gating and a dt_limit that clamps on both
    sides: equals the direct launchers on the clamped dt, gated by silu(z), with
    the chain rule through the clamp, the softplus and the gate."""
    from kernels.ssd_combined import mamba_chunk_scan_combined, ssd_chunk_scan_bwd, ssd_chunk_scan_fwd
    B, L, H, P, N, G = 1, 192, 4, 64, 128, 2
    tx, tdt, tA, tB, tC, tD, tdy = _inputs(B, L, H, P, N, G, seed=13)
    x, dt_raw, A, Bm, Cm, D, dy = (t.to(DEV) for t in (tx, tdt, tA, tB, tC, tD, tdy))
    z = torch.from_numpy(np.random.default_rng(14).standard_normal((B, L, H, P)).astype(np.float32))
    z = z.to(torch.bfloat16).to(DEV)
    bias = torch.full((H,), -1.0, device=DEV)
    limit = (0.32, 0.33)  # softplus(dt_raw - 1) spans ~0.313-0.341 here: both bounds bite
    leaves = [t.clone().requires_grad_() for t in (x, dt_raw, A, Bm, Cm, D, z)]
    y = mamba_chunk_scan_combined(*leaves[:5], 256, D=leaves[5], z=leaves[6], dt_bias=bias, dt_softplus=True,
                                  dt_limit=limit)
    y.backward(dy)
    pre = torch.nn.functional.softplus(dt_raw + bias)
    inside = (pre >= limit[0]) & (pre <= limit[1])
    assert 0 < int(inside.sum()) < inside.numel(), "the limit should clamp some but not all of dt"
    dt = pre.clamp(*limit)
    y2, cst, _ = ssd_chunk_scan_fwd(x, dt, A, Bm, Cm, D)
    gate = torch.nn.functional.silu(z.float())
    assert torch.equal(y, (y2.float() * gate).to(torch.bfloat16))
    dys = (dy.float() * gate).to(torch.bfloat16)
    dx, ddt, dA, dB, dC, dD, _ = ssd_chunk_scan_bwd(x, dt, A, Bm, Cm, cst, dys, D)
    torch.testing.assert_close(leaves[0].grad, dx, rtol=0, atol=0)
    torch.testing.assert_close(leaves[1].grad, ddt * inside * torch.sigmoid(dt_raw + bias), rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(leaves[2].grad, dA, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(leaves[5].grad, dD, rtol=1e-3, atol=1e-3)
    sg = torch.sigmoid(z.float())
    dz = (dy.float() * y2.float() * sg * (1 + z.float() * (1 - sg))).to(torch.bfloat16)
    torch.testing.assert_close(leaves[6].grad, dz, rtol=1e-2, atol=1e-2)


def test_ssd_forward_steep_decay_matches_oracle():
    """Large dt * A (cumsum spans over 60 within 16 tokens): the tcgen05 kernels'
    per-element decay path for such key groups, next to the factored one."""
    from kernels.ssd_combined import ssd_chunk_scan_fwd
    B, L, H, P, N, G = 1, 192, 2, 64, 128, 1
    x, dt, A, Bm, Cm, D, dy = so.make_ssd_inputs(B, L, H, P, N, ngroups=G, seed=5, dt_range=(0.05, 2.0))
    dt[:, :96] *= 0.05  # the first key groups stay narrow
    bf = lambda a: torch.from_numpy(a).to(torch.bfloat16)  # noqa: E731
    tx, tB, tC = bf(x), bf(Bm), bf(Cm)
    y, cst, fin = ssd_chunk_scan_fwd(tx.to(DEV), torch.from_numpy(dt).to(DEV), torch.from_numpy(A).to(DEV),
                                     tB.to(DEV), tC.to(DEV), torch.from_numpy(D).to(DEV), return_final_states=True)
    torch.cuda.synchronize()
    assert _device_status_clear() == 0
    r = so.ssd_fwd(_f64(tx), dt.astype(np.float64), A.astype(np.float64), _f64(tB), _f64(tC), D=D.astype(np.float64))
    assert_lowp_close(y, r["y"], "y")
    assert_lowp_close(fin, r["final_state"], "final_state")
    ref_states = np.concatenate([np.zeros((B, 1, H, P, N)), r["states"][:, 63::64][:, :cst.shape[1] - 1]], axis=1)
    assert_lowp_close(cst, ref_states, "chunk_states")
    # and the backward's per-element decay path for the same steep key groups
    from kernels.ssd_combined import ssd_chunk_scan_bwd
    tdy = bf(dy)
    dx, ddt, dA, dB, dC, dD, _ = ssd_chunk_scan_bwd(tx.to(DEV), torch.from_numpy(dt).to(DEV),
                                                    torch.from_numpy(A).to(DEV), tB.to(DEV), tC.to(DEV), cst,
                                                    tdy.to(DEV), torch.from_numpy(D).to(DEV))
    torch.cuda.synchronize()
    assert _device_status_clear() == 0
    g = so.ssd_bwd(_f64(tx), dt.astype(np.float64), A.astype(np.float64), _f64(tB), _f64(tC), _f64(tdy),
                   D=D.astype(np.float64))
    for name, k in (("dx", dx), ("ddt", ddt), ("dB", dB), ("dC", dC)):
        assert_lowp_close(k, g[name], name)


def test_ssd_backward_mma_sync_kernel_on_strided_dx():
    """A dx buffer whose strides the tensor-core backward cannot store into (not
    multiples of 8 elements) runs the mma.sync backward; both kernels match the
    oracle on the same inputs."""
    from kernels.ssd_combined import ssd_chunk_scan_bwd, ssd_chunk_scan_fwd
    B, L, H, P, N, G = 1, 160, 2, 64, 128, 1
    tx, tdt, tA, tB, tC, tD, tdy = _inputs(B, L, H, P, N, G, seed=21)
    x, dt, A, Bm, Cm, D, dy = (t.to(DEV) for t in (tx, tdt, tA, tB, tC, tD, tdy))
    y, cst, _ = ssd_chunk_scan_fwd(x, dt, A, Bm, Cm, D)
    pad = torch.zeros(B, L, H, P + 2, dtype=torch.bfloat16, device=DEV)  # head stride 66
    dx_view = pad[..., :P]
    outs_old = ssd_chunk_scan_bwd(x, dt, A, Bm, Cm, cst, dy, D, dx_out=dx_view)
    outs_new = ssd_chunk_scan_bwd(x, dt, A, Bm, Cm, cst, dy, D)
    torch.cuda.synchronize()
    assert _device_status_clear() == 0
    args = (_f64(tx), tdt.double().numpy(), tA.double().numpy(), _f64(tB), _f64(tC))
    g = so.ssd_bwd(*args, _f64(tdy), D=tD.double().numpy())
    for outs in (outs_old, outs_new):
        dx, ddt, dA, dB, dC, dD, _ = outs
        for name, k in (("dx", dx), ("ddt", ddt), ("dB", dB), ("dC", dC)):
            assert_lowp_close(k, g[name], name)
    assert float(pad[..., P:].abs().max()) == 0.0  # nothing written outside the view


def _reference_bench_call(batch, seqlen, nheads, headdim, seed, dtype):
    """The inputs kernels/benchmarks/bench_ema_total.py:62-76 builds for its SSD
    call: p = sigmoid(randn) per (batch, token); dt = -log(1 - p) repeated
    over heads; X_m = X / dt (fp32 by promotion); A_m = -1; B_m = p and
    C_m = ones of shape (batch, seqlen, 1, 1)."""
    g = torch.Generator().manual_seed(seed)
    X = torch.randn(batch, seqlen, nheads, headdim, generator=g).to(dtype)
    p = torch.sigmoid(torch.randn(batch, seqlen, 1, generator=g).to(dtype))
    dt1 = -torch.log(1 - p).to(torch.float32).squeeze(-1)
    Xm = (X.reshape(batch, seqlen, nheads * headdim) / dt1[..., None]).reshape(batch, seqlen, nheads, headdim)
    dt = dt1[:, :, None].expand(batch, seqlen, nheads).contiguous()
    A = -torch.ones(nheads)
    Bm = p.to(torch.float32)[..., None]
    Cm = torch.ones_like(Bm)
    dy = torch.randn(Xm.shape, generator=g)
    return Xm, dt, A, Bm, Cm, dy


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_reference_benchmark_call_form_dstate1(dtype):
    """mamba_chunk_scan_combined exactly as the reference's benchmark calls it
    (fp32 x, d_state 1, B = p, C = 1, A = -1, chunk 64) through autograd,
    against the float64 SSD oracle: y, dx, ddt, dA and dB."""
    from kernels.ssd_combined import mamba_chunk_scan_combined
    Xm, dt, A, Bm, Cm, dy = _reference_bench_call(2, 512, 4, 64, seed=5, dtype=dtype)
    assert Xm.dtype == torch.float32
    leaves = [t.to(DEV).requires_grad_() for t in (Xm, dt, A, Bm)]
    y = mamba_chunk_scan_combined(leaves[0], leaves[1], leaves[2], leaves[3], Cm.to(DEV), chunk_size=64,
                                  seq_idx=None)
    y.backward(dy.to(DEV))
    args = [t.double().numpy() for t in (Xm, dt, A, Bm, Cm)]
    r = so.ssd_fwd(*args)
    g = so.ssd_bwd(*args, dy.double().numpy())
    from _tol import assert_fp32_close
    assert_fp32_close(y, r["y"], "y")
    for name, t in (("dx", leaves[0]), ("ddt", leaves[1]), ("dA", leaves[2]), ("dB", leaves[3])):
        assert_fp32_close(t.grad, g[name], name)


def test_dstate1_groups_D_gates_and_states():
    """d_state 1 with two groups, bf16 x, D skip, non-trivial C, an initial state
    and the final state's gradient, z gating: every gradient against the oracle
    (z through torch autograd on the oracle's y)."""
    from kernels.ssd_combined import mamba_chunk_scan_combined
    rng = np.random.default_rng(9)
    b_, L, H, P, G = 2, 300, 4, 32, 2
    x = torch.from_numpy(rng.standard_normal((b_, L, H, P)).astype(np.float32)).to(torch.bfloat16)
    dt = torch.from_numpy(rng.uniform(0.01, 0.3, (b_, L, H)).astype(np.float32))
    A = torch.from_numpy(-rng.uniform(0.5, 4.0, H).astype(np.float32))
    Bm = torch.from_numpy(rng.standard_normal((b_, L, G, 1)).astype(np.float32))
    Cm = torch.from_numpy(rng.standard_normal((b_, L, G, 1)).astype(np.float32))
    D = torch.from_numpy(rng.standard_normal(H).astype(np.float32))
    s0 = torch.from_numpy(rng.standard_normal((b_, H, P, 1)).astype(np.float32))
    # y is bf16 like x, so the gradient reaching the scan is bf16: draw dy in bf16
    dy = torch.from_numpy(rng.standard_normal((b_, L, H, P)).astype(np.float32)).to(torch.bfloat16).float()
    dfin = torch.from_numpy(rng.standard_normal((b_, H, P, 1)).astype(np.float32))
    leaves = [t.to(DEV).requires_grad_() for t in (x, dt, A, Bm, Cm, D, s0)]
    y, fin = mamba_chunk_scan_combined(*leaves[:5], 128, D=leaves[5], initial_states=leaves[6],
                                       return_final_states=True)
    ((y.float() * dy.to(DEV)).sum() + (fin * dfin.to(DEV)).sum()).backward()
    args = [t.double().numpy() for t in (x.float(), dt, A, Bm, Cm)]
    r = so.ssd_fwd(*args, D=D.double().numpy(), initial_state=s0.double().numpy())
    g = so.ssd_bwd(*args, dy.double().numpy(), D=D.double().numpy(), initial_state=s0.double().numpy(),
                   d_final_state=dfin.double().numpy())
    assert_lowp_close(y, r["y"], "y")
    from _tol import assert_fp32_close
    assert_fp32_close(fin, r["final_state"], "final state")
    assert_lowp_close(leaves[0].grad, g["dx"], "dx")
    for name, i in (("ddt", 1), ("dA", 2), ("dB", 3), ("dC", 4), ("dD", 5), ("d_initial_state", 6)):
        assert_fp32_close(leaves[i].grad, g[name], name)
