"""GPU parity of the reference-facing EMA API (ema_fwd_triton, chunk_cumsum_triton,
compute_dpx, ema_combined) against the reference's own outputs (golden fixtures,
fp32) and the float64 oracle (fp32 and bf16 inputs)."""

import math

import numpy as np
import pytest
import torch

from _tol import assert_fp32_close, assert_lowp_close, assert_reference_rule
from conftest import load_golden
from oracle import ema_oracle as eo

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(autouse=True)
def _status_clean():
    from kernels import _lib
    yield
    assert _lib.device_status(clear=True) == 0, "a device-side wait timed out"


def _t(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


FWD_CASES = ["fwd_q64", "fwd_q64_shared", "fwd_q128_ragged", "fwd_q256", "fwd_q64_p48"]


@pytest.mark.parametrize("name", FWD_CASES)
def test_forward_matches_reference_outputs(name):
    from kernels.forward.ema_ssd_fwd import ema_fwd_triton
    g = load_golden(name)
    Q = int(g["chunk_size"])
    y, st, cs, css = ema_fwd_triton(_t(g["x"]), dA=_t(g["dA"]), chunk_size=Q, store_states=True,
                                    store_da_cs=True, store_da_cs_sum=True)
    assert y.shape == g["out"].shape and st.shape == g["states"].shape
    assert cs.shape == g["da_cs"].shape and css.shape == g["da_cs_sum"].shape
    for k, v in (("out", y), ("states", st), ("da_cs", cs), ("da_cs_sum", css)):
        assert_fp32_close(v, g[k], f"{name}.{k}")


def test_forward_seq_idx_matches_reference():
    from kernels.forward.ema_ssd_fwd import ema_fwd_triton
    g = load_golden("fwd_seqidx_aligned")
    y, css = ema_fwd_triton(_t(g["x"]), dA=_t(g["dA"]), seq_idx=torch.from_numpy(g["seq_idx"]).to(DEV),
                            chunk_size=int(g["chunk_size"]), store_da_cs_sum=True)
    assert_fp32_close(y, g["out"], "seq_idx out")
    assert_fp32_close(css, g["da_cs_sum"], "seq_idx da_cs_sum")


@pytest.mark.parametrize("Q", [64, 128, 256])
def test_forward_seq_idx_unaligned_segments(Q):
    """Segments starting inside chunks (reset rule of ema_torch_ref_seq_idx)."""
    from kernels.forward.ema_ssd_fwd import ema_fwd_triton
    rng = np.random.default_rng(5)
    B, L, H, P = 2, 700, 3, 64
    x = rng.standard_normal((B, L, H, P)).astype(np.float32)
    dA = (-rng.random((B, H, L)) * 0.3).astype(np.float32)
    seq = np.zeros((B, L), np.int32)
    for b, cuts in enumerate(([37, 300, 301, 555], [1, 129, 640])):
        for i, c in enumerate(cuts):
            seq[b, c:] = i + 1
    y, st = ema_fwd_triton(_t(x), dA=_t(dA), seq_idx=torch.from_numpy(seq).to(DEV), chunk_size=Q,
                           store_states=True)
    r = eo.ema_fwd(x, dA, Q, seq_idx=seq)
    assert_fp32_close(y, r["out"], "out")
    assert_fp32_close(st, r["states"], "states")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("Q", [64, 128, 256])
def test_forward_lowp_matches_oracle(dtype, Q):
    from kernels.forward.ema_ssd_fwd import ema_fwd_triton
    rng = np.random.default_rng(Q)
    B, L, H, P = 2, 1000, 4, 64
    x = torch.from_numpy(rng.standard_normal((B, L, H, P)).astype(np.float32)).to(dtype)
    dA = (-rng.random((B, H, L)) * math.log2(math.e)).astype(np.float32)
    y, st = ema_fwd_triton(x.to(DEV), dA=_t(dA), chunk_size=Q, store_states=True)
    assert y.dtype == dtype
    r = eo.ema_fwd(x.float().numpy(), dA, Q)
    assert_lowp_close(y, r["out"], "y")
    assert_fp32_close(st, r["states"], "states (fp32 accumulation)")


@pytest.mark.parametrize("P", [32, 48, 64, 96, 128])
def test_forward_headdims(P):
    from kernels.forward.ema_ssd_fwd import ema_fwd_triton
    rng = np.random.default_rng(P)
    B, L, H, Q = 1, 333, 2, 64
    x = rng.standard_normal((B, L, H, P)).astype(np.float32)
    dA = (-rng.random((B, H, L))).astype(np.float32)
    y, st, cs, css = ema_fwd_triton(_t(x), dA=_t(dA), chunk_size=Q, store_states=True, store_da_cs=True,
                                    store_da_cs_sum=True)
    r = eo.ema_fwd(x, dA, Q)
    for k, v in (("out", y), ("states", st), ("da_cs", cs), ("da_cs_sum", css)):
        assert_fp32_close(v, r[k], k)


def test_forward_out_argument_and_return_arity():
    from kernels.forward.ema_ssd_fwd import ema_fwd_triton
    x = torch.randn(1, 130, 2, 64, device=DEV)
    dA = -torch.rand(1, 2, 130, device=DEV)
    out = torch.empty_like(x)
    y = ema_fwd_triton(x, dA=dA, out=out)
    assert y is out
    assert isinstance(ema_fwd_triton(x, dA=dA), torch.Tensor)
    assert len(ema_fwd_triton(x, dA=dA, store_states=True)) == 2
    assert len(ema_fwd_triton(x, dA=dA, store_da_cs=True)) == 2
    assert len(ema_fwd_triton(x, dA=dA, store_da_cs_sum=True)) == 2
    assert len(ema_fwd_triton(x, dA=dA, store_states=True, store_da_cs=True)) == 3
    assert len(ema_fwd_triton(x, dA=dA, store_states=True, store_da_cs_sum=True)) == 3
    assert len(ema_fwd_triton(x, dA=dA, store_da_cs=True, store_da_cs_sum=True)) == 3
    # a non-contiguous out is honoured too
    big = torch.empty(1, 130, 2, 128, device=DEV)
    view = big[..., :64]
    ema_fwd_triton(x, dA=dA, out=view)
    assert_fp32_close(view, y, "strided out")


def test_forward_rejects_like_reference():
    from kernels.forward.ema_ssd_fwd import ema_fwd_triton
    x = torch.randn(1, 64, 1, 64, device=DEV)
    with pytest.raises(AssertionError):
        ema_fwd_triton(x, dA=None)
    with pytest.raises(AssertionError):
        ema_fwd_triton(x, dA=-torch.rand(1, 1, 64, device=DEV), chunk_size=100)
    with pytest.raises(AssertionError):
        ema_fwd_triton(x.cpu(), dA=-torch.rand(1, 1, 64))


@pytest.mark.parametrize("e2", [0, 1])
def test_chunk_cumsum_matches_reference(e2):
    from kernels.forward.ema_ssd_fwd import chunk_cumsum_triton
    g = load_golden(f"chunk_cumsum_exp2_{e2}")
    cs, rev = chunk_cumsum_triton(_t(g["dA"]), chunk_size=int(g["chunk_size"]), exp2=bool(e2))
    assert_fp32_close(cs, g["dA_cs"], "dA_cs")
    assert_fp32_close(rev, g["dA_cs_rev"], "dA_cs_rev")


def test_chunk_cumsum_strided_and_outputs_given():
    from kernels.forward.ema_ssd_fwd import chunk_cumsum_triton
    base = -torch.rand(2, 300, 3, device=DEV)
    dA = base.permute(0, 2, 1)  # (B, H, L), non-contiguous
    o1 = torch.empty(2, 3, 300, device=DEV)
    o2 = torch.empty(2, 3, 300, device=DEV)
    cs, rev = chunk_cumsum_triton(dA, chunk_size=128, dA_cs=o1, dA_cs_rev=o2)
    assert cs is o1 and rev is o2
    f, r = eo.chunk_cumsum(dA.cpu().numpy(), 128)
    assert_fp32_close(cs, f, "cs")
    assert_fp32_close(rev, r, "rev")


BWD_CASES = ["bwd_q64", "bwd_q64_opts", "bwd_q128", "bwd_q256_opts"]


@pytest.mark.parametrize("name", BWD_CASES)
def test_compute_dpx_matches_reference_outputs(name):
    from kernels.backward.ema_ssd_combined import compute_dpx
    g = load_golden(name)
    opts = "d_issm_state" in g
    dx, dA, d_issm = compute_dpx(_t(g["x"]), _t(g["da_cs"]), _t(g["da_cs_sum"]), _t(g["ssm_states"]),
                                 _t(g["do"]),
                                 d_ossm_state=_t(g["d_ossm_state"]) if opts else None,
                                 d_ox_state=_t(g["d_ox_state"]) if opts else None,
                                 chunk_size=int(g["chunk_size"]), has_input_state=opts)
    assert dx.shape == g["dx"].shape and dA.shape == g["dA"].shape
    assert_fp32_close(dx, g["dx"], "dx")
    assert_fp32_close(dA, g["dA"], "dA")
    if opts:
        assert d_issm.shape == g["d_issm_state"].shape
        assert_fp32_close(d_issm, g["d_issm_state"], "d_issm_state")
    else:
        assert d_issm is None


@pytest.mark.parametrize("L,Q", [(1000, 64), (777, 128), (513, 256), (64, 64), (1, 64)])
def test_compute_dpx_ragged_matches_oracle(L, Q):
    """Ragged last chunk (the reference backward reads/writes past seqlen here)."""
    from kernels.forward.ema_ssd_fwd import ema_fwd_triton
    from kernels.backward.ema_ssd_combined import compute_dpx
    rng = np.random.default_rng(L)
    B, H, P = 2, 3, 64
    x = rng.standard_normal((B, L, H, P)).astype(np.float32)
    dA = (-rng.random((B, H, L))).astype(np.float32)
    do = rng.standard_normal((B, L, H, P)).astype(np.float32)
    dfin = rng.standard_normal((B, H, P)).astype(np.float32)
    dlast = rng.standard_normal((B, H, P)).astype(np.float32)
    _, st, cs, css = ema_fwd_triton(_t(x), dA=_t(dA), chunk_size=Q, store_states=True, store_da_cs=True,
                                    store_da_cs_sum=True)
    states = st.squeeze(3).permute(0, 2, 3, 1)
    dx, dl, dis = compute_dpx(_t(x), cs, css, states, _t(do), d_ossm_state=_t(dfin), d_ox_state=_t(dlast),
                              chunk_size=Q, has_input_state=True)
    f = eo.ema_fwd(x, dA, Q)
    r = eo.ema_bwd(x, f["da_cs"], f["da_cs_sum"], f["states"][:, :, :, 0, :].transpose(0, 2, 3, 1), do,
                   d_ossm_state=dfin, d_ox_state=dlast, chunk_size=Q, has_input_state=True)
    assert_fp32_close(dx, r["dx"], "dx")
    assert_fp32_close(dl, r["dA"], "dA")
    assert_fp32_close(dis, r["d_issm_state"], "d_issm_state")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_compute_dpx_lowp_matches_oracle(dtype):
    from kernels.forward.ema_ssd_fwd import ema_fwd_triton
    from kernels.backward.ema_ssd_combined import compute_dpx
    rng = np.random.default_rng(3)
    B, L, H, P, Q = 2, 1024, 4, 64, 128
    x = torch.from_numpy(rng.standard_normal((B, L, H, P)).astype(np.float32)).to(dtype)
    do = torch.from_numpy(rng.standard_normal((B, L, H, P)).astype(np.float32)).to(dtype)
    dA = (-rng.random((B, H, L)) * 0.5).astype(np.float32)
    _, st, cs, css = ema_fwd_triton(x.to(DEV), dA=_t(dA), chunk_size=Q, store_states=True, store_da_cs=True,
                                    store_da_cs_sum=True)
    dx, dl, _ = compute_dpx(x.to(DEV), cs, css, st.squeeze(3).permute(0, 2, 3, 1), do.to(DEV), chunk_size=Q)
    assert dx.dtype == dtype
    f = eo.ema_fwd(x.float().numpy(), dA, Q)
    r = eo.ema_bwd(x.float().numpy(), f["da_cs"], f["da_cs_sum"],
                   f["states"][:, :, :, 0, :].transpose(0, 2, 3, 1), do.float().numpy(), chunk_size=Q)
    assert_lowp_close(dx, r["dx"], "dx")
    assert_lowp_close(dl, r["dA"], "dA")


def test_ema_combined_matches_reference_outputs():
    from kernels.backward.ema_ssd_combined import ema_combined
    g = load_golden("combined_q64")
    x = _t(g["x"]).requires_grad_()
    A = _t(g["A"]).requires_grad_()
    y = ema_combined(x, A, chunk_size=int(g["chunk_size"]))
    (y * _t(g["dout"])).sum().backward()
    assert_fp32_close(y, g["out"], "out")
    assert_fp32_close(x.grad, g["dx"], "dx")
    assert_fp32_close(A.grad, g["dA"], "dA")


def test_ema_combined_reference_test_shape():
    """The reference's own autograd test shape and inputs (B16 L2048 H32 P64, chunk 64,
    bf16 x, A = -U(0,1) shared by the heads; test_ema_combined_autograd.py:30-66),
    checked with its acceptance rule and with the bf16 tolerance, against the
    float64 recurrence."""
    from kernels.backward.ema_ssd_combined import ema_combined
    torch.manual_seed(0)
    B, L, H, P, Q = 16, 2048, 32, 64, 64
    A = torch.rand(B, L, device=DEV).neg_().requires_grad_()
    X = torch.randn(B, L, H, P, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    dout = torch.randn_like(X)
    out = ema_combined(X, A, chunk_size=Q)
    (out * dout).sum().backward()
    r = eo.ema_combined_grads(X.detach(), A.detach(), dout, Q)
    assert_reference_rule(X.grad, r["dx"], "dx")
    assert_reference_rule(A.grad, r["dA"], "dA")
    assert_lowp_close(out, r["out"], "out")
    assert_lowp_close(X.grad, r["dx"], "dx")
    assert_lowp_close(A.grad, r["dA"], "dA")


def test_value_errors_like_reference():
    from kernels.backward.ema_ssd_combined import ema_combined
    x = torch.randn(1, 64, 2, 64, device=DEV)
    with pytest.raises(ValueError):
        ema_combined(x[0], -torch.rand(1, 64, device=DEV))
    with pytest.raises(ValueError):
        ema_combined(x, -torch.rand(64, device=DEV))
    with pytest.raises(ValueError):
        ema_combined(x, -torch.rand(1, 63, device=DEV))


def test_start_state_invariant():
    """states[:, k] == y[:, k*Q - 1] (test_ema_dpx.py:98-108), to fp32 rounding."""
    from kernels.forward.ema_ssd_fwd import ema_fwd_triton
    x = torch.randn(3, 640, 2, 64, device=DEV)
    dA = -torch.rand(3, 2, 640, device=DEV)
    y, st = ema_fwd_triton(x, dA=dA, chunk_size=128, store_states=True)
    assert torch.all(st[:, 0] == 0)
    for k in range(1, st.shape[1]):
        assert_fp32_close(st[:, k, :, 0, :], y[:, k * 128 - 1], f"chunk {k}")
