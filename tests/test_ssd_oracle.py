"""The SSD oracle (oracle/ssd_oracle.py) is unpinned -- the reference has no SSD
implementation of its own (it calls the absent mamba_ssm package) -- so it is
cross-checked three ways: the chunked restatement against the sequential
recurrence, the hand-written adjoint against torch autograd of the same
recurrence in float64, and against central finite differences."""

import numpy as np
import pytest
import torch

from oracle import ssd_oracle as so


def _torch_recurrence(x, dt, A, B, C, D, s0):
    b_, L, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    hpg = H // G
    Bh = B.repeat_interleave(hpg, dim=2)
    Ch = C.repeat_interleave(hpg, dim=2)
    s = s0
    ys = []
    for t in range(L):
        a = torch.exp(dt[:, t] * A)[:, :, None, None]
        s = a * s + (dt[:, t, :, None, None] * x[:, t, :, :, None]) * Bh[:, t, :, None, :]
        ys.append(torch.einsum("bhpn,bhn->bhp", s, Ch[:, t]))
    y = torch.stack(ys, dim=1) + D[None, None, :, None] * x
    return y, s


@pytest.mark.parametrize("L,Q,G", [(50, 16, 1), (64, 32, 2)])
def test_chunked_restatement_matches_recurrence(L, Q, G):
    x, dt, A, B, C, D, _ = so.make_ssd_inputs(2, L, 4, 6, 5, ngroups=G, seed=L + Q)
    s0 = np.random.default_rng(1).standard_normal((2, 4, 6, 5))
    r = so.ssd_fwd(x, dt, A, B, C, D, initial_state=s0)
    c = so.ssd_chunked_fwd(x, dt, A, B, C, Q, D, initial_state=s0)
    np.testing.assert_allclose(c["y"], r["y"], rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(c["final_state"], r["final_state"], rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(c["chunk_states"][:, 1], r["states"][:, Q - 1], rtol=1e-10, atol=1e-10)


def test_adjoint_matches_torch_autograd():
    x, dt, A, B, C, D, dy = so.make_ssd_inputs(2, 24, 4, 5, 3, ngroups=2, seed=3, dt_range=(0.05, 0.5))
    rng = np.random.default_rng(2)
    s0 = rng.standard_normal((2, 4, 5, 3))
    dfin = rng.standard_normal((2, 4, 5, 3))
    ts = [torch.tensor(np.asarray(a, dtype=np.float64), requires_grad=True) for a in (x, dt, A, B, C, D, s0)]
    y, sf = _torch_recurrence(*ts)
    (y * torch.from_numpy(dy.astype(np.float64))).sum().backward(retain_graph=True)
    (sf * torch.from_numpy(dfin)).sum().backward()
    g = so.ssd_bwd(x, dt, A, B, C, dy, D, initial_state=s0, d_final_state=dfin)
    for name, t in zip(("dx", "ddt", "dA", "dB", "dC", "dD", "d_initial_state"), ts):
        np.testing.assert_allclose(g[name], t.grad.numpy(), rtol=1e-9, atol=1e-11, err_msg=name)
    f = so.ssd_fwd(x, dt, A, B, C, D, initial_state=s0)
    np.testing.assert_allclose(f["y"], y.detach().numpy(), rtol=1e-12, atol=1e-12)


def test_adjoint_matches_finite_differences():
    x, dt, A, B, C, D, dy = so.make_ssd_inputs(1, 9, 2, 3, 2, seed=4, dt_range=(0.05, 0.5))
    x, dt, A, B, C, D, dy = (np.asarray(a, dtype=np.float64) for a in (x, dt, A, B, C, D, dy))
    g = so.ssd_bwd(x, dt, A, B, C, dy, D)

    def loss(**kw):
        args = dict(x=x, dt=dt, A=A, B=B, C=C, D=D)
        args.update(kw)
        return float((so.ssd_fwd(**args)["y"] * dy).sum())

    eps = 1e-6
    for name, arr, idx, gname in (("dt", dt, (0, 4, 1), "ddt"), ("A", A, (1,), "dA"), ("B", B, (0, 3, 0, 1), "dB"),
                                  ("C", C, (0, 7, 0, 0), "dC"), ("x", x, (0, 2, 1, 2), "dx")):
        p, m = arr.copy(), arr.copy()
        p[idx] += eps
        m[idx] -= eps
        fd = (loss(**{name: p}) - loss(**{name: m})) / (2 * eps)
        np.testing.assert_allclose(g[gname][idx], fd, rtol=1e-6, atol=1e-8, err_msg=gname)


@pytest.mark.parametrize("L,Q,G", [(50, 16, 1), (64, 32, 2), (40, 64, 1)])
def test_chunked_adjoint_matches_sequential_adjoint(L, Q, G):
    x, dt, A, B, C, D, dy = so.make_ssd_inputs(2, L, 4, 6, 5, ngroups=G, seed=L * Q, dt_range=(0.05, 0.5))
    rng = np.random.default_rng(5)
    s0 = rng.standard_normal((2, 4, 6, 5))
    dfin = rng.standard_normal((2, 4, 6, 5))
    r = so.ssd_bwd(x, dt, A, B, C, dy, D, initial_state=s0, d_final_state=dfin)
    c = so.ssd_chunked_bwd(x, dt, A, B, C, dy, Q, D, initial_state=s0, d_final_state=dfin)
    for name in ("dx", "ddt", "dA", "dB", "dC", "dD", "d_initial_state"):
        np.testing.assert_allclose(c[name], r[name], rtol=1e-9, atol=1e-11, err_msg=name)
