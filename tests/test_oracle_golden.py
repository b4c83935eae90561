"""Pin the float64 oracle to the reference's own outputs (CPU only).

The fixtures in ``tests/golden`` are the reference's Triton kernels run under
the Triton CPU interpreter in float32 (``tests/golden/make_golden.py``).  The
bar is the fp32 tolerance of the north-star spec: 1e-4 relative, measured as
``max|oracle - ref| / max|ref|`` per output.
"""

import numpy as np
import pytest

from conftest import load_golden
from oracle import ema_oracle as eo

FP32_REL = 1e-4


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


FWD_CASES = ["fwd_q64", "fwd_q64_shared", "fwd_q128_ragged", "fwd_q256", "fwd_q64_p48"]


@pytest.mark.parametrize("name", FWD_CASES)
def test_oracle_forward_matches_reference(name):
    g = load_golden(name)
    r = eo.ema_fwd(g["x"], g["dA"], int(g["chunk_size"]))
    for key in ("out", "states", "da_cs", "da_cs_sum"):
        assert r[key].shape == g[key].shape, key
        assert rel_err(r[key], g[key]) < FP32_REL, (key, rel_err(r[key], g[key]))


def test_oracle_forward_seq_idx_matches_reference():
    g = load_golden("fwd_seqidx_aligned")
    r = eo.ema_fwd(g["x"], g["dA"], int(g["chunk_size"]), seq_idx=g["seq_idx"])
    assert rel_err(r["out"], g["out"]) < FP32_REL
    assert rel_err(r["da_cs_sum"], g["da_cs_sum"]) < FP32_REL


@pytest.mark.parametrize("name", ["bwd_q64", "bwd_q64_opts", "bwd_q128", "bwd_q256_opts"])
def test_oracle_backward_matches_reference(name):
    g = load_golden(name)
    opts = "d_issm_state" in g
    r = eo.ema_bwd(g["x"], g["da_cs"], g["da_cs_sum"], g["ssm_states"], g["do"],
                   d_ossm_state=g.get("d_ossm_state"), d_ox_state=g.get("d_ox_state"),
                   chunk_size=int(g["chunk_size"]), has_input_state=opts)
    assert rel_err(r["dx"], g["dx"]) < FP32_REL, rel_err(r["dx"], g["dx"])
    assert rel_err(r["dA"], g["dA"]) < FP32_REL, rel_err(r["dA"], g["dA"])
    if opts:
        assert rel_err(r["d_issm_state"], g["d_issm_state"]) < FP32_REL


def test_oracle_combined_autograd_matches_reference():
    g = load_golden("combined_q64")
    r = eo.ema_combined_grads(g["x"], g["A"], g["dout"], int(g["chunk_size"]))
    for key in ("out", "dx", "dA"):
        assert rel_err(r[key], g[key]) < FP32_REL, (key, rel_err(r[key], g[key]))


@pytest.mark.parametrize("e2", [0, 1])
def test_oracle_chunk_cumsum_matches_reference(e2):
    g = load_golden(f"chunk_cumsum_exp2_{e2}")
    fwd, rev = eo.chunk_cumsum(g["dA"], int(g["chunk_size"]), exp2=bool(e2))
    assert rel_err(fwd, g["dA_cs"]) < FP32_REL
    assert rel_err(rev, g["dA_cs_rev"]) < FP32_REL


def test_oracle_start_state_invariant():
    """states[:, k] == out[:, k*Q - 1] for k >= 1 and states[:, 0] == 0
    (the reference's own check, test_ema_dpx.py:98-108)."""
    g = load_golden("fwd_q64")
    Q = int(g["chunk_size"])
    r = eo.ema_fwd(g["x"], g["dA"], Q)
    st = r["states"][:, :, :, 0, :]
    assert np.all(st[:, 0] == 0)
    for k in range(1, st.shape[1]):
        np.testing.assert_allclose(st[:, k], r["out"][:, k * Q - 1], rtol=0, atol=0)


def test_oracle_seq_idx_equals_independent_sequences():
    """seq_idx with K equal segments == K independent recurrences
    (the reference's ema_torch_ref_repeat comparison, ema_ssd_fwd.py:793-798)."""
    rng = np.random.default_rng(0)
    B, L, H, P, K = 2, 96, 2, 8, 3
    x = rng.standard_normal((B, L, H, P))
    dA = -rng.random((B, H, L))
    seq = np.repeat(np.arange(K), L // K)[None].repeat(B, 0)
    r = eo.ema_fwd(x, dA, 32, seq_idx=seq)["out"]
    n = L // K
    for k in range(K):
        part = eo.ema_fwd(x[:, k * n:(k + 1) * n], dA[:, :, k * n:(k + 1) * n], 32)["out"]
        np.testing.assert_allclose(r[:, k * n:(k + 1) * n], part, rtol=1e-12, atol=1e-12)


def test_dt_form_equals_reference_form():
    """The dt-parameterised EMA is the reference EMA with X = dt*x, dA = dt*A*log2(e)."""
    x, dt, A, dy = eo.make_dt_inputs(2, 64, 3, 8, seed=3)
    y = eo.ema_dt_fwd(x, dt, A)["y"]
    X = dt[..., None].astype(np.float64) * x
    dA = (dt.astype(np.float64) * A[None, None, :] * eo.LOG2E).transpose(0, 2, 1)
    y_ref = eo.ema_fwd(X, dA, 16)["out"]
    np.testing.assert_allclose(y, y_ref, rtol=1e-12, atol=1e-12)


def test_dt_form_gradients_match_torch_autograd():
    torch = pytest.importorskip("torch")
    x, dt, A, dy = eo.make_dt_inputs(2, 40, 2, 4, seed=4)
    h0 = np.random.default_rng(1).standard_normal((2, 2, 4))
    dfin = np.random.default_rng(2).standard_normal((2, 2, 4))
    tx, tdt, tA, th0 = (torch.tensor(v, dtype=torch.float64, requires_grad=True)
                        for v in (x, dt, A, h0))
    h = th0
    ys = []
    for t in range(x.shape[1]):
        a = torch.exp(tdt[:, t] * tA)[..., None]
        h = a * h + tdt[:, t, :, None] * tx[:, t]
        ys.append(h)
    y = torch.stack(ys, 1)
    loss = (y * torch.tensor(dy, dtype=torch.float64)).sum() + (h * torch.tensor(dfin)).sum()
    loss.backward()
    r = eo.ema_dt_bwd(x, dt, A, dy, initial_state=h0, d_final_state=dfin)
    np.testing.assert_allclose(r["dx"], tx.grad.numpy(), rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(r["ddt"], tdt.grad.numpy(), rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(r["dA"], tA.grad.numpy(), rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(r["d_initial_state"], th0.grad.numpy(), rtol=1e-10, atol=1e-10)
