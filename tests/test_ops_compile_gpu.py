"""The dispatcher operators on the GPU: torch.compile traces each autograd path
in one graph (fullgraph=True, the aot_eager backend: no code generation, the
library's kernels run as the graph's operators) and matches eager execution,
and torch.library.opcheck accepts the forward operators (schema, fake
implementation, autograd registration, dispatch under AOT autograd)."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _close(a, b, what):
    tol = 2e-2 if a.dtype in (torch.bfloat16, torch.float16) else 1e-3
    torch.testing.assert_close(a.float(), b.float(), rtol=tol, atol=tol, msg=what)


def _run(fn, leaves, dy):
    leaves = [t.detach().clone().requires_grad_(t.is_floating_point()) for t in leaves]
    y = fn(*leaves)
    y.backward(dy)
    return [y.detach()] + [t.grad for t in leaves if t.requires_grad]


def _compare(fn, leaves, dy):
    torch._dynamo.reset()
    eager = _run(fn, leaves, dy)
    compiled = _run(torch.compile(fn, backend="aot_eager", fullgraph=True), leaves, dy)
    for k, (a, b) in enumerate(zip(compiled, eager)):
        _close(a, b, f"output {k}")


def test_dt_scan_compiles_in_one_graph():
    from kernels.ema_chunk_scan import ema_chunk_scan_combined
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 700, 4, 64, generator=g).to(DEV, torch.bfloat16)
    dt = (torch.rand(2, 700, 4, generator=g) * 0.1 + 1e-3).to(DEV)
    A = (-torch.rand(4, generator=g) * 4 - 0.5).to(DEV)
    dy = torch.randn(2, 700, 4, 64, generator=g).to(DEV, torch.bfloat16)
    _compare(lambda x, dt, A: ema_chunk_scan_combined(x, dt, A, 256), [x, dt, A], dy)


def test_reference_form_compiles_in_one_graph():
    from kernels.backward.ema_ssd_combined import ema_combined
    g = torch.Generator().manual_seed(2)
    x = torch.randn(1, 300, 2, 64, generator=g).to(DEV)
    A = (-torch.rand(1, 300, generator=g)).to(DEV)
    dy = torch.randn(1, 300, 2, 64, generator=g).to(DEV)
    _compare(lambda x, A: ema_combined(x, A, 64), [x, A], dy)


def test_ssd_with_gate_and_dt_map_compiles_in_one_graph():
    from oracle import ssd_oracle as so
    from kernels.ssd_combined import mamba_chunk_scan_combined
    x, dt, A, Bm, Cm, D, dy = so.make_ssd_inputs(1, 192, 4, 64, 128, ngroups=2, seed=4)
    bf = lambda a: torch.from_numpy(a).to(DEV, torch.bfloat16)  # noqa: E731
    z = bf(np.random.default_rng(5).standard_normal(x.shape).astype(np.float32))
    bias = torch.full((4,), -0.5, device=DEV)

    def fn(x, dt, A, Bm, Cm, D, z, bias):
        return mamba_chunk_scan_combined(x, dt, A, Bm, Cm, 256, D=D, z=z, dt_bias=bias, dt_softplus=True,
                                         dt_limit=(1e-3, 0.2))
    leaves = [bf(x), torch.from_numpy(dt).to(DEV), torch.from_numpy(A).to(DEV), bf(Bm), bf(Cm),
              torch.from_numpy(D).to(DEV), z, bias]
    _compare(fn, leaves, bf(dy))


def test_opcheck_forward_operators():
    import kernels.backward.ema_ssd_combined  # noqa: F401
    import kernels.ema_chunk_scan  # noqa: F401
    import kernels.ssd_combined  # noqa: F401
    from oracle import ssd_oracle as so
    g = torch.Generator().manual_seed(3)
    r = lambda *s: torch.randn(*s, generator=g).to(DEV)  # noqa: E731
    x = r(1, 300, 2, 64).to(torch.bfloat16).requires_grad_()
    dt = (torch.rand(1, 300, 2, generator=g) * 0.1 + 1e-3).to(DEV).requires_grad_()
    A = (-torch.rand(2, generator=g) - 0.5).to(DEV).requires_grad_()
    torch.library.opcheck(torch.ops.ema_b200.ema_scan_dt_fwd, (x, dt, A, 128, False, None))
    # (the reference form's autograd lives in _EmaFunction around this operator)
    torch.library.opcheck(torch.ops.ema_b200.ema_fwd_ref, (r(1, 300, 2, 64), -torch.rand(1, 2, 300, generator=g).to(DEV), 64))
    sx, sdt, sA, sB, sC, sD, _ = so.make_ssd_inputs(1, 130, 2, 64, 128, ngroups=1, seed=6)
    bf = lambda a: torch.from_numpy(a).to(DEV, torch.bfloat16).requires_grad_()  # noqa: E731
    f32 = lambda a: torch.from_numpy(a).to(DEV).requires_grad_()  # noqa: E731
    torch.library.opcheck(torch.ops.ema_b200.ssd_fwd,
                          (bf(sx), f32(sdt), f32(sA), bf(sB), bf(sC), f32(sD), None, None, False, 0.0, float("inf")))
    y = r(1, 50, 2, 64).to(torch.bfloat16).requires_grad_()
    z = r(1, 50, 2, 64).to(torch.bfloat16).requires_grad_()
    torch.library.opcheck(torch.ops.ema_b200.ssd_gate_fwd, (y, z))
