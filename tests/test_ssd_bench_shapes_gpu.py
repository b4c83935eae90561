"""SSD parity at the benchmark shapes (configs 3 and 5) on a seeded subset.

The whole batch runs on the GPU at full size; the float64 chunked oracle
(oracle/ssd_oracle.py: ssd_chunked_fwd / ssd_chunked_bwd, cross-checked
against the sequential recurrence and its adjoint on the CPU) runs on one
seeded batch row -- every head of it, so the group-summed dB and dC of that
(batch, group) are complete.  dA and dD sum over every batch row: they are
checked on a launch over that one row alone, whose other outputs must equal
the full-batch launch's row.  Parity is unpinned: the reference has no SSD of
its own (its benchmark calls the absent third-party mamba_ssm package).

Inputs are drawn on the GPU with a seeded torch generator (config 5 holds
1.3 G elements per activation tensor): x, dy ~ N(0,1) bf16; dt =
softplus(N(0,1) + b_h) clipped to [1e-3, 1e-1]; A = -exp(U(0, log 16));
B, C ~ N(0,1)/sqrt(dstate) bf16; D ~ N(0,1).
"""

import math

import numpy as np
import pytest
import torch

from _tol import assert_lowp_close, assert_reference_rule
from oracle import ssd_oracle as so

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(B, L, H, P, N, G, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    bf = torch.bfloat16
    x = torch.randn(B, L, H, P, generator=g, device=DEV).to(bf)
    dy = torch.randn(B, L, H, P, generator=g, device=DEV).to(bf)
    lo, hi = 1e-3, 1e-1
    u = torch.rand(H, generator=g, device=DEV) * (math.log(hi) - math.log(lo)) + math.log(lo)
    bias = torch.log(torch.expm1(torch.exp(u)))
    dt = torch.clamp(torch.nn.functional.softplus(torch.randn(B, L, H, generator=g, device=DEV) + bias), lo, hi)
    A = -torch.exp(torch.rand(H, generator=g, device=DEV) * math.log(16.0))
    Bm = (torch.randn(B, L, G, N, generator=g, device=DEV) / math.sqrt(N)).to(bf)
    Cm = (torch.randn(B, L, G, N, generator=g, device=DEV) / math.sqrt(N)).to(bf)
    D = torch.randn(H, generator=g, device=DEV)
    return x, dt, A, Bm, Cm, D, dy


def _status_clear():
    import ctypes

    from kernels import _lib
    v = ctypes.c_uint32(0)
    _lib.check(_lib.lib.ssd_device_status(ctypes.byref(v), 1, _lib.stream_ptr(torch.device(DEV))), "ssd_device_status")
    return v.value


def _f64(t):
    return t.detach().float().double().cpu().numpy()


@pytest.mark.parametrize("cfg", ["config3", "config5"])
def test_ssd_benchmark_shape_matches_oracle_on_a_batch_row(cfg):
    from kernels.ssd_combined import ssd_chunk_scan_bwd, ssd_chunk_scan_fwd
    shape = {"config3": (8, 4096, 64), "config5": (32, 8192, 80)}[cfg]
    B, L, H = shape
    P, N, G = 64, 128, 1
    seed = 3 if cfg == "config3" else 5
    x, dt, A, Bm, Cm, D, dy = _inputs(B, L, H, P, N, G, seed)
    row = int(np.random.default_rng(seed).integers(B))

    y, cst, _ = ssd_chunk_scan_fwd(x, dt, A, Bm, Cm, D)
    dx, ddt, dA, dB, dC, dD, _ = ssd_chunk_scan_bwd(x, dt, A, Bm, Cm, cst, dy, D)
    torch.cuda.synchronize()
    assert _status_clear() == 0
    got = {k: v[row:row + 1].detach().cpu() for k, v in (("y", y), ("dx", dx), ("ddt", ddt), ("dB", dB), ("dC", dC))}
    del y, cst, dx, ddt, dB, dC

    sl = slice(row, row + 1)
    xs, dts, Bs, Cs, dys = (t[sl].contiguous() for t in (x, dt, Bm, Cm, dy))
    del x, dy
    torch.cuda.empty_cache()
    # the same row alone: per-head reductions (dA, dD) of this row only
    y1, cst1, _ = ssd_chunk_scan_fwd(xs, dts, A, Bs, Cs, D)
    dx1, ddt1, dA1, dB1, dC1, dD1, _ = ssd_chunk_scan_bwd(xs, dts, A, Bs, Cs, cst1, dys, D)
    torch.cuda.synchronize()
    assert _status_clear() == 0
    torch.testing.assert_close(y1.cpu(), got["y"], rtol=0, atol=0)
    torch.testing.assert_close(dx1.cpu(), got["dx"], rtol=0, atol=0)
    torch.testing.assert_close(ddt1.cpu(), got["ddt"], rtol=1e-5, atol=1e-6)
    # dB / dC sum the heads with fp32 atomics: equal up to summation order
    torch.testing.assert_close(dB1.cpu(), got["dB"], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(dC1.cpu(), got["dC"], rtol=1e-4, atol=1e-5)

    args = [_f64(t) for t in (xs, dts, A, Bs, Cs)]
    Dd = _f64(D)
    r = so.ssd_chunked_fwd(*args, 128, D=Dd)
    gref = so.ssd_chunked_bwd(*args, _f64(dys), 128, D=Dd)
    assert_lowp_close(got["y"], r["y"], f"{cfg} y (row {row})")
    assert_reference_rule(got["y"], r["y"], f"{cfg} y")
    for name in ("dx", "ddt", "dB", "dC"):
        assert_lowp_close(got[name], gref[name], f"{cfg} {name} (row {row})")
        assert_reference_rule(got[name], gref[name], f"{cfg} {name}")
    for name, k in (("dA", dA1), ("dD", dD1)):
        ref = gref[name]
        e = float(np.abs(k.cpu().double().numpy() - ref).max() / max(np.abs(ref).max(), 1e-30))
        assert e <= 2e-2, f"{cfg} {name}: normwise relative error {e:.3e}"
