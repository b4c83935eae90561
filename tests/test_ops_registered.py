"""The kernels as PyTorch dispatcher operators (namespace ema_b200), on CPU:
every operator is registered with its schema, its shape-only ("fake")
implementation gives the shapes, dtypes and strides the CUDA implementation
returns (fake CUDA tensors under FakeTensorMode), and autograd runs through the
registered formulas on meta tensors (the fake implementations serve the meta
device too).  No GPU and no kernel launch are needed."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

OPS = ["ema_scan_dt_fwd", "ema_scan_dt_bwd", "ema_fwd_ref", "ema_dpx", "ssd_fwd", "ssd_bwd", "ssd_gate_fwd",
       "ssd_gate_bwd"]


@pytest.fixture(scope="module", autouse=True)
def _load():
    import kernels.backward.ema_ssd_combined  # noqa: F401
    import kernels.ema_chunk_scan  # noqa: F401
    import kernels.ssd_combined  # noqa: F401


def test_every_operator_is_registered():
    for name in OPS:
        op = getattr(torch.ops.ema_b200, name)
        assert op.default._schema.name == f"ema_b200::{name}"


def test_dt_scan_fake_shapes_and_fake_autograd():
    from kernels.ema_chunk_scan import ema_chunk_scan_combined
    B, L, H, P = 2, 700, 4, 64
    with FakeTensorMode():
        x = torch.empty(B, L, H, P, dtype=torch.bfloat16, device="cuda", requires_grad=True)
        dt = torch.empty(B, L, H, device="cuda", requires_grad=True)
        A = torch.empty(H, device="cuda", requires_grad=True)
        y, st, fin, rows = torch.ops.ema_b200.ema_scan_dt_fwd(x, dt, A, 256, True, None)
        assert y.shape == x.shape and y.dtype == torch.bfloat16
        # the states entering every 128 tokens: a view of a (B, 2 nc, H, P) buffer
        assert st.shape == (B, 6, H, P) and st.stride() == (6 * H * P, H * P, P, 1)
        assert fin.shape == (B, H, P) and rows.shape == (B, H, L) and rows.dtype == torch.float32
    # autograd through the registered formula (meta tensors: the engine needs no device)
    x = torch.empty(B, L, H, P, dtype=torch.bfloat16, device="meta", requires_grad=True)
    dt = torch.empty(B, L, H, device="meta", requires_grad=True)
    A = torch.empty(H, device="meta", requires_grad=True)
    init = torch.empty(B, H, P, device="meta", requires_grad=True)
    y, _, final, _ = torch.ops.ema_b200.ema_scan_dt_fwd(x, dt, A, 256, True, init)
    (y.float().sum() + final.sum()).backward()
    for t in (x, dt, A, init):
        assert t.grad is not None and t.grad.shape == t.shape and t.grad.dtype == t.dtype


def test_reference_form_fake_autograd():
    from kernels.backward.ema_ssd_combined import ema_combined
    with FakeTensorMode():
        x = torch.empty(2, 300, 3, 64, device="cuda")
        out, st, cs, css = torch.ops.ema_b200.ema_fwd_ref(x, torch.empty(2, 3, 300, device="cuda"), 64)
        assert out.shape == x.shape
        assert st.shape == (2, 5, 3, 1, 64) and cs.shape == (2, 3, 300) and css.shape == (2, 3, 5)
    x = torch.empty(2, 300, 3, 64, device="meta", requires_grad=True)
    A = torch.empty(2, 300, device="meta", requires_grad=True)
    ema_combined(x, A, 64).sum().backward()
    assert x.grad.shape == x.shape and A.grad.shape == A.shape


@pytest.mark.parametrize("with_opts", [False, True])
def test_ssd_fake_autograd(with_opts):
    from kernels.ssd_combined import mamba_chunk_scan_combined
    B, L, H, P, G, N = 1, 200, 4, 64, 2, 128
    m = "meta"
    leaves = [torch.empty(B, L, H, P, dtype=torch.bfloat16, device=m), torch.empty(B, L, H, device=m),
              torch.empty(H, device=m), torch.empty(B, L, G, N, dtype=torch.bfloat16, device=m),
              torch.empty(B, L, G, N, dtype=torch.bfloat16, device=m), torch.empty(H, device=m),
              torch.empty(H, device=m), torch.empty(B, L, H, P, dtype=torch.bfloat16, device=m)]
    for t in leaves:
        t.requires_grad_()
    x, dt, A, Bm, Cm, D, bias, z = leaves
    kw = dict(z=z, dt_bias=bias, dt_softplus=True, dt_limit=(1e-3, 0.1)) if with_opts else {}
    y, fin = mamba_chunk_scan_combined(x, dt, A, Bm, Cm, 256, D=D, return_final_states=True, **kw)
    assert y.shape == x.shape and fin.shape == (B, H, P, N)
    (y.float().sum() + fin.sum()).backward()
    for t in (x, dt, A, Bm, Cm, D):
        assert t.grad is not None and t.grad.shape == t.shape and t.grad.dtype == t.dtype
    if with_opts:
        assert bias.grad.shape == (H,) and z.grad.shape == z.shape


def test_absent_outputs_are_distinct_tensors():
    """Outputs of a dispatcher operator may not alias one another: the optional
    gradients an SSD backward leaves empty are separate tensors."""
    m = "meta"
    B, L, H, P, G, N = 1, 100, 2, 64, 1, 128
    x = torch.empty(B, L, H, P, dtype=torch.bfloat16, device=m)
    args = (x, torch.empty(B, L, H, device=m), torch.empty(H, device=m),
            torch.empty(B, L, G, N, dtype=torch.bfloat16, device=m),
            torch.empty(B, L, G, N, dtype=torch.bfloat16, device=m),
            torch.empty(B, 2, H, P, N, device=m), torch.empty_like(x), None, None, False, None, False, 0.0,
            float("inf"))
    outs = torch.ops.ema_b200.ssd_bwd(*args)
    for i in range(len(outs)):
        for j in range(i + 1, len(outs)):
            assert outs[i] is not outs[j], (i, j)
    assert all(o.numel() == 0 for o in outs[5:])
