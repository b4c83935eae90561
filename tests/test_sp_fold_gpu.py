"""The sub-span fold kernels of the sequence-parallel EMA (ema_span_summary /
ema_span_expand, through kernels/ema_sp.py) against their float64 torch
restatement, both directions, from one to 64 sub-spans, with log decays from
mild to ones whose exponentials underflow."""

import pytest
import torch

from _sp_fold_ref import torch_fold

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("K", [1, 3, 8, 64])
@pytest.mark.parametrize("direction", [0, 1])
@pytest.mark.parametrize("scale", [0.05, 30.0, 2000.0])
def test_fold_kernels_match_float64(K, direction, scale):
    from kernels.ema_sp import _kernel_fold
    g = torch.Generator().manual_seed(K * 10 + direction)
    B, H, P = 2, 5, 48
    ld = (-torch.rand(B, K, H, generator=g, dtype=torch.float64) * scale).to(DEV)
    V = torch.randn(B * K, H, P, generator=g).to(DEV)
    bnd = torch.randn(B, H, P, generator=g).to(DEV)
    out, d = _kernel_fold(direction, False, ld, V)
    ref, dref = torch_fold(direction, False, ld, V)
    torch.testing.assert_close(out, ref, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(d, dref, rtol=1e-6, atol=1e-30)
    ex = _kernel_fold(direction, True, ld, V, bnd)
    torch.testing.assert_close(ex, torch_fold(direction, True, ld, V, bnd), rtol=1e-6, atol=1e-6)


def test_fold_refuses_more_than_64_subspans():
    from kernels import _lib
    from kernels.ema_sp import _kernel_fold
    ld = -torch.rand(1, 65, 2, dtype=torch.float64, device=DEV)
    V = torch.randn(65, 2, 8, device=DEV)
    with pytest.raises(_lib.EmaLaunchError, match="64 sub-spans"):
        _kernel_fold(0, False, ld, V)
