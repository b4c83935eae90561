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


def _dt_map_np(raw, bias, softplus, lo, hi):
    """The kernels' dt map in float64: clamp(softplus(raw + bias), lo, hi) and its
    derivative (torch's softplus threshold 20; 0 where the clamp is active)."""
    v = raw + (bias[None, None, :] if bias is not None else 0.0)
    if softplus:
        sp = np.where(v <= 20.0, np.log1p(np.exp(np.minimum(v, 20.0))), v)
        d = np.where(v <= 20.0, 1.0 / (1.0 + np.exp(-v)), 1.0)
    else:
        sp, d = v, np.ones_like(v)
    inside = (sp >= lo) & (sp <= hi)
    return np.clip(sp, lo, hi), d * inside


def _limit_in_gaps(vals, q_lo, q_hi):
    """Clamp bounds near two quantiles of vals, each in the middle of the widest
    gap between neighbouring values there, so fp32 and float64 agree on which
    elements the clamp touches."""
    v = np.sort(vals.ravel())
    out = []
    for q in (q_lo, q_hi):
        k = int(q * (v.size - 1))
        w = slice(max(k - 20, 0), min(k + 20, v.size - 1))
        gaps = np.diff(v[w.start:w.stop + 1])
        j = w.start + int(np.argmax(gaps))
        out.append(0.5 * (v[j] + v[j + 1]))
    return tuple(out)


# (H, G): 2 heads per group -> tcgen05 forward; 1 head per group -> mma.sync forward;
# the backward is the tcgen05 kernel throughout (its mma.sync twin: the strided-dx test below)
@pytest.mark.parametrize("H,G,softplus,clamp,gate", [(4, 1, True, False, False), (4, 2, True, True, True),
                                                      (3, 3, False, True, True)])
def test_mamba_call_form_dt_map_and_gate_match_oracle(H, G, softplus, clamp, gate):
    """mamba_chunk_scan_combined with dt_bias / dt_softplus / dt_limit (mapped inside
    the SSD kernels) and z gating (the native gate kernels), through autograd,
    against the float64 oracle on the mapped dt: y, dx, ddt of the raw dt, the
    dt_bias gradient, dA, dB, dC, dD and dz."""
    from kernels.ssd_combined import mamba_chunk_scan_combined
    B, L, P, N = 2, 192, 64, 128
    tx, tdt, tA, tB, tC, tD, tdy = _inputs(B, L, H, P, N, G, seed=13 + H + G)
    rng = np.random.default_rng(14 + H)
    bias = rng.uniform(-2.0, 0.5, H).astype(np.float32)
    dt_target = tdt.double().numpy()
    raw = (np.log(np.expm1(dt_target)) if softplus else dt_target) - bias[None, None, :]
    raw = raw.astype(np.float32)
    pre, _ = _dt_map_np(raw.astype(np.float64), bias.astype(np.float64), softplus, -np.inf, np.inf)
    limit = _limit_in_gaps(pre, 0.1, 0.9) if clamp else (0.0, float("inf"))
    dt_eff, deriv = _dt_map_np(raw.astype(np.float64), bias.astype(np.float64), softplus, *limit)
    if clamp:
        assert 0 < int((deriv == 0).sum()) < deriv.size, "the limit should clamp some but not all of dt"
    z = rng.standard_normal((B, L, H, P)).astype(np.float32)
    tz = torch.from_numpy(z).to(torch.bfloat16)
    leaves = [t.to(DEV).requires_grad_() for t in (tx, torch.from_numpy(raw), tA, tB, tC, tD,
                                                    torch.from_numpy(bias), tz)]
    y = mamba_chunk_scan_combined(*leaves[:5], 256, D=leaves[5], z=leaves[7] if gate else None,
                                  dt_bias=leaves[6], dt_softplus=softplus, dt_limit=limit)
    y.backward(tdy.to(DEV))
    torch.cuda.synchronize()
    assert _device_status_clear() == 0

    args = (_f64(tx), dt_eff, tA.double().numpy(), _f64(tB), _f64(tC))
    r = so.ssd_fwd(*args, D=tD.double().numpy())
    zf = _f64(tz)
    sg = 1.0 / (1.0 + np.exp(-zf))
    dout = _f64(tdy)
    if gate:
        assert_lowp_close(y, r["y"] * zf * sg, "gated y")
        # the scan's incoming gradient, rounded to bf16 as the gate kernel stores it
        dys = torch.from_numpy(dout * zf * sg).to(torch.bfloat16).double().numpy()
        dz = dout * r["y"] * sg * (1.0 + zf * (1.0 - sg))
        assert_lowp_close(leaves[7].grad, dz, "dz")
    else:
        assert_lowp_close(y, r["y"], "y")
        dys = dout
    g = so.ssd_bwd(*args, dys, D=tD.double().numpy())
    ddt_raw = g["ddt"] * deriv
    for name, k, ref in (("dx", leaves[0].grad, g["dx"]), ("ddt", leaves[1].grad, ddt_raw),
                         ("dB", leaves[3].grad, g["dB"]), ("dC", leaves[4].grad, g["dC"])):
        assert_lowp_close(k, ref, name)
        assert_reference_rule(k, ref, name)
    for name, k, ref in (("dA", leaves[2].grad, g["dA"]), ("dD", leaves[5].grad, g["dD"]),
                         ("d dt_bias", leaves[6].grad, ddt_raw.sum(axis=(0, 1)))):
        e = float(np.abs(k.cpu().double().numpy() - ref).max() / max(np.abs(ref).max(), 1e-30))
        assert e <= 2e-2, f"{name}: normwise relative error {e:.3e}"


def test_dt_map_on_the_mma_sync_backward():
    """The dt map and the dt_bias gradient in the mma.sync backward (a dx buffer
    whose strides the tensor-core backward cannot store into), against the
    tensor-core backward and the oracle."""
    from kernels.ssd_combined import ssd_chunk_scan_bwd, ssd_chunk_scan_fwd
    B, L, H, P, N, G = 1, 160, 2, 64, 128, 1
    tx, tdt, tA, tB, tC, tD, tdy = _inputs(B, L, H, P, N, G, seed=23)
    x, A, Bm, Cm, D, dy = (t.to(DEV) for t in (tx, tA, tB, tC, tD, tdy))
    bias = np.array([-1.5, 0.25], dtype=np.float32)
    raw = (np.log(np.expm1(tdt.double().numpy())) - bias[None, None, :]).astype(np.float32)
    pre, _ = _dt_map_np(raw.astype(np.float64), bias.astype(np.float64), True, -np.inf, np.inf)
    limit = _limit_in_gaps(pre, 0.15, 0.85)
    dt_eff, deriv = _dt_map_np(raw.astype(np.float64), bias.astype(np.float64), True, *limit)
    traw, tbias = torch.from_numpy(raw).to(DEV), torch.from_numpy(bias).to(DEV)
    opts = dict(dt_bias=tbias, dt_softplus=True, dt_limit=limit)
    y, cst, _ = ssd_chunk_scan_fwd(x, traw, A, Bm, Cm, D, **opts)
    pad = torch.zeros(B, L, H, P + 2, dtype=torch.bfloat16, device=DEV)  # head stride 66: the mma.sync kernel
    db_old, db_new = (torch.empty(H, device=DEV) for _ in range(2))
    outs_old = ssd_chunk_scan_bwd(x, traw, A, Bm, Cm, cst, dy, D, dx_out=pad[..., :P], ddt_bias_out=db_old, **opts)
    outs_new = ssd_chunk_scan_bwd(x, traw, A, Bm, Cm, cst, dy, D, ddt_bias_out=db_new, **opts)
    torch.cuda.synchronize()
    assert _device_status_clear() == 0
    args = (_f64(tx), dt_eff, tA.double().numpy(), _f64(tB), _f64(tC))
    assert_lowp_close(y, so.ssd_fwd(*args, D=tD.double().numpy())["y"], "y")
    g = so.ssd_bwd(*args, _f64(tdy), D=tD.double().numpy())
    ddt_raw = g["ddt"] * deriv
    for outs, db in ((outs_old, db_old), (outs_new, db_new)):
        assert_lowp_close(outs[0], g["dx"], "dx")
        assert_lowp_close(outs[1], ddt_raw, "ddt")
        ref = ddt_raw.sum(axis=(0, 1))
        e = float(np.abs(db.cpu().double().numpy() - ref).max() / max(np.abs(ref).max(), 1e-30))
        assert e <= 2e-2, f"d dt_bias: normwise relative error {e:.3e}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("strided", [False, True])
def test_gate_kernels_match_float64(dtype, strided):
    """The native gate out = y silu(z) and its gradient (dy, dz) against float64,
    on contiguous tensors (16-byte vector path) and on views with a head stride
    of headdim + 2 (element path)."""
    from kernels.ssd_combined import ssd_gate
    rng = np.random.default_rng(31)
    B, L, H, P = 2, 70, 3, 64
    mk = lambda: torch.from_numpy(rng.standard_normal((B, L, H, P + 2)).astype(np.float32) * 2).to(dtype)  # noqa: E731
    yb, zb = (mk().to(DEV).requires_grad_() for _ in range(2))
    dout = mk().to(DEV)[..., :P]
    # views with head stride P + 2 (element path), or contiguous copies (vector path)
    y, z = (yb[..., :P], zb[..., :P]) if strided else (yb[..., :P].contiguous(), zb[..., :P].contiguous())
    if not strided:
        dout = dout.contiguous()
    out = ssd_gate(y, z)
    out.backward(dout)
    torch.cuda.synchronize()
    yl_grad, zl_grad = yb.grad[..., :P], zb.grad[..., :P]
    yd, zd, dd = (t.detach().double().cpu().numpy() for t in (y, z, dout))
    sg = 1.0 / (1.0 + np.exp(-zd))
    refs = (("out", out, yd * zd * sg), ("dy", yl_grad, dd * zd * sg),
            ("dz", zl_grad, dd * yd * sg * (1.0 + zd * (1.0 - sg))))
    for name, k, ref in refs:
        assert k.dtype == dtype, name
        if dtype == torch.float32:
            e = float(np.abs(k.detach().double().cpu().numpy() - ref).max() / np.abs(ref).max())
            assert e <= 1e-5, f"{name}: normwise relative error {e:.3e}"
        else:
            assert_lowp_close(k, ref, name)


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
