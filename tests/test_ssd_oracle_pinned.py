"""The SSD oracle pinned to the reference's own outputs (CPU only).

The reference has no SSD implementation, but with d_state 1 its recurrence
contains the reference EMA: with A_h = -1, dt_t = -ln(2) dA_t (so that
exp(dt_t A_h) = 2^dA_t, the reference's decay, kernels/forward/ema_ssd_fwd.py:
258-259), one group per head with B_t = 1 / dt_t (so that the input term
dt_t x_t B_t is x_t) and C = 1, the SSD state is the EMA state Z_t and y_t = Z_t.
So oracle/ssd_oracle.py -- the sequential recurrence and its chunked
restatement, forward and backward -- is checked here against the golden vectors
the reference's Triton kernels produced (tests/golden), at the fp32 bar of
1e-4 relative: y and the chunk start states against ema_fwd_triton, dx and
the per-token decay gradient against compute_dpx.  The decay gradient is read
off the SSD oracle's ddt: d ddt = A dl + sum_p dx_p x_p B (the decay and the
input term both carry dt), so dl = (ddt - sum_p dx_p x_p B) / A.
"""

import numpy as np
import pytest

from conftest import load_golden
from oracle import ssd_oracle as so

FP32_REL = 1e-4
LN2 = float(np.log(2.0))


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _ssd_args(x, dA):
    """SSD inputs whose recurrence is the reference EMA with log2 decay dA (B, H, L)."""
    dt = -LN2 * np.transpose(np.asarray(dA, np.float64), (0, 2, 1))  # (B, L, H) > 0
    A = -np.ones(x.shape[2])
    Bm = (1.0 / dt)[..., None]  # (B, L, G = H, 1)
    return np.asarray(x, np.float64), dt, A, Bm, np.ones_like(Bm)


@pytest.mark.parametrize("name", ["fwd_q64", "fwd_q64_shared", "fwd_q128_ragged", "fwd_q256", "fwd_q64_p48"])
def test_ssd_oracle_forward_is_the_reference_ema(name):
    g = load_golden(name)
    args = _ssd_args(g["x"], g["dA"])
    r = so.ssd_fwd(*args)
    assert rel_err(r["y"], g["out"]) < FP32_REL, rel_err(r["y"], g["out"])
    rc = so.ssd_chunked_fwd(*args, chunk_size=int(g["chunk_size"]))
    assert rel_err(rc["y"], g["out"]) < FP32_REL
    # the chunk start states, (B, nc, H, P, 1) against the reference's (B, nc, H, 1, P)
    assert rel_err(rc["chunk_states"][..., 0], g["states"][:, :, :, 0, :]) < FP32_REL


def _per_token_decay(da_cs, Q):
    """Per-token log2 decay from the reference's within-chunk cumsum."""
    dA = np.array(da_cs, np.float64)
    dA[..., 1:] -= da_cs[..., :-1]
    dA[..., ::Q] = da_cs[..., ::Q]
    return dA


@pytest.mark.parametrize("name", ["bwd_q64", "bwd_q64_opts", "bwd_q128", "bwd_q256_opts"])
@pytest.mark.parametrize("chunked", [False, True])
def test_ssd_oracle_backward_is_the_reference_ema(name, chunked):
    g = load_golden(name)
    Q = int(g["chunk_size"])
    x, dt, A, Bm, Cm = _ssd_args(g["x"], _per_token_decay(g["da_cs"], Q))
    init = np.asarray(g["ssm_states"][..., 0], np.float64)[..., None]  # the state entering chunk 0
    dfin = g["d_ossm_state"][..., None] if "d_ossm_state" in g else None
    if chunked:
        r = so.ssd_chunked_bwd(x, dt, A, Bm, Cm, g["do"], Q, initial_state=init, d_final_state=dfin)
    else:
        r = so.ssd_bwd(x, dt, A, Bm, Cm, g["do"], initial_state=init, d_final_state=dfin)
    dx = np.array(r["dx"])
    if "d_ox_state" in g:  # compute_dpx adds it to dX at the last token, outside the recurrence
        dx[:, -1] += g["d_ox_state"]
    assert rel_err(dx, g["dx"]) < FP32_REL, rel_err(dx, g["dx"])
    dl = (r["ddt"] - np.sum(r["dx"] * x, axis=-1) * Bm[..., 0]) / A  # (B, L, H)
    assert rel_err(np.transpose(dl, (0, 2, 1)), g["dA"]) < FP32_REL, rel_err(np.transpose(dl, (0, 2, 1)), g["dA"])
    if "d_issm_state" in g:
        assert rel_err(r["d_initial_state"][..., 0], g["d_issm_state"][..., 0]) < FP32_REL
