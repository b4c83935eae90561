"""The reference's PyTorch CPU path for the EMA, restated (TEST/BASELINE INFRASTRUCTURE ONLY).

The reference's CPU implementation of the EMA is a sequential PyTorch loop,
``ema_torch_ref`` (kernels/forward/ema_ssd_fwd.py:542-560):

    state = state * (1 - p_t) + x_t        for t = 0 .. L-1

over (batch, token, dim) tensors with a (batch, token, 1) "forget" weight p,
differentiated with torch autograd (the reference's tests backpropagate the
same loop, kernels/tests/ema_ssd_bwd/test_ema_dpx.py:20-30, :132-135).  The
dt-parameterised workload of the benchmark maps onto it with one row per
(batch, head): X = dt * x reshaped to (B*H, L, P) and p = 1 - exp(dt * A).

``bench.py`` times :func:`dt_form_fwd_bwd` on the GPU box's host cores as the
CPU baseline (``cpu_baseline``) and as the ``--impl reference`` arm.  It is
never part of the product path.
"""

from __future__ import annotations

import time

import torch


def ema_torch_ref(X: torch.Tensor, P: torch.Tensor) -> torch.Tensor:
    """Sequential EMA over dim 1: X (b, s, d), P (b, s, 1) -> (b, s, d)."""
    state = torch.zeros_like(X[:, 0, :])
    outs = []
    for t in range(X.shape[1]):
        state = state * (1 - P[:, t, :]) + X[:, t, :]
        outs.append(state)
    return torch.stack(outs, dim=1)


def dt_form_fwd_bwd(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, dy: torch.Tensor):
    """One forward + backward of the dt-form EMA through ``ema_torch_ref`` and autograd.

    x, dy (B, L, H, P); dt (B, L, H); A (H,).  Returns (y, dx, ddt, dA)."""
    B, L, H, Pd = x.shape
    x = x.detach().requires_grad_()
    dt = dt.detach().requires_grad_()
    A = A.detach().requires_grad_()
    X = (dt[..., None] * x).permute(0, 2, 1, 3).reshape(B * H, L, Pd)
    p = (1 - torch.exp(dt * A)).permute(0, 2, 1).reshape(B * H, L, 1)
    y = ema_torch_ref(X, p).reshape(B, H, L, Pd).permute(0, 2, 1, 3)
    (y * dy).sum().backward()
    return y.detach(), x.grad, dt.grad, A.grad


def time_sample(x, dt, A, dy, reps: int = 1):
    """Wall-clock seconds of ``reps`` forward+backward passes on the CPU."""
    t0 = time.perf_counter()
    for _ in range(reps):
        dt_form_fwd_bwd(x, dt, A, dy)
    return time.perf_counter() - t0
