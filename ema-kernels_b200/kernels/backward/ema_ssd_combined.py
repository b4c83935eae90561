"""EMA backward and autograd on B200 -- drop-in for ``kernels.backward.ema_ssd_combined``.

``compute_dpx``, ``_EmaFunction`` and ``ema_combined`` keep the reference's
signatures, shape checks and return conventions
(kernels/backward/ema_ssd_combined.py:48-229); the backward launches the
sm_100a kernel of libema_ssd_b200.so through its C ABI.

Semantics (as the reference): ``compute_dpx`` returns dX, the per-token
gradient with respect to the NATURAL-log decay (``dA``, shape (b, h, s) --
no ln2 factor, although the inputs are log2 cumsums), and optionally the
gradient of the chunk-0 start state.  ``d_ossm_state`` seeds the gradient of
the final state; ``d_ox_state`` is added to dX at the last token.

Differences, all deliberate:
* A ragged last chunk (seqlen % chunk_size != 0) is handled exactly; the
  reference backward reads and writes past seqlen there
  (ema_ssd_bwd.py:152-153, :277-278).
* ``SSM_States`` may have any strides (the forward's states are passed as a
  permuted view; the reference copies them with ``.contiguous()``,
  ema_ssd_combined.py:198).
* The ``d_ox_state`` addition is fused into the kernel's dX store.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from .. import _lib
from ..forward.ema_ssd_fwd import ema_fwd_triton

__all__ = ["compute_dpx", "ema_combined", "_EmaFunction"]


def compute_dpx(
    x: torch.Tensor,
    da_cs: torch.Tensor,
    da_cs_sum: torch.Tensor,
    SSM_States: torch.Tensor,
    do: torch.Tensor,
    d_ossm_state: Optional[torch.Tensor] = None,
    d_ox_state: Optional[torch.Tensor] = None,
    chunk_size: int = 64,
    has_input_state: bool = False,
) -> Tuple[torch.Tensor, torch.Tensor, Optional[torch.Tensor]]:
    """EMA backward for dX and the per-token decay gradient.

    Args:
        x: Input tensor (batch, seqlen, nheads, head_dim)
        da_cs: Per-token cumulative dA within each chunk (batch, nheads, seqlen)
        da_cs_sum: Per-chunk sum of dA (batch, nheads, nchunks)
        SSM_States: Per-chunk start states from forward (batch, nheads, head_dim, nchunks)
        do: Output gradient (batch, seqlen, nheads, head_dim)
        d_ossm_state: Optional gradient of output state (batch, nheads, head_dim)
        d_ox_state: Optional gradient added to last token (batch, nheads, head_dim)
        chunk_size: Chunk size (64, 128 or 256)
        has_input_state: Whether to return gradient for input states

    Returns:
        (dx, dA, d_issm_state) where d_issm_state is None if has_input_state=False.
    """
    batch, seqlen, nheads, head_dim = x.shape
    nchunks = (seqlen + chunk_size - 1) // chunk_size
    assert x.is_cuda and da_cs.is_cuda and da_cs_sum.is_cuda and do.is_cuda, "All tensors must be on CUDA"
    assert da_cs.shape == (batch, nheads, seqlen)
    assert da_cs_sum.shape == (batch, nheads, nchunks)
    assert SSM_States.shape == (batch, nheads, head_dim, nchunks)
    assert do.shape == (batch, seqlen, nheads, head_dim)
    assert d_ossm_state is None or d_ossm_state.shape == (batch, nheads, head_dim)
    assert d_ox_state is None or d_ox_state.shape == (batch, nheads, head_dim)
    assert chunk_size in (64, 128, 256), "chunk_size must be 64, 128 or 256"
    assert x.dtype in _lib.DTYPE_CODES, f"unsupported dtype {x.dtype}"
    dev = x.device

    x_k = _lib.tma_ready(x)
    do_k = _lib.tma_ready(do if do.dtype == x.dtype else do.to(x.dtype))
    cs_k = da_cs.to(torch.float32).contiguous()
    css_k = da_cs_sum.to(torch.float32).contiguous()
    st_k = SSM_States if SSM_States.dtype == torch.float32 else SSM_States.float()
    dfin = None if d_ossm_state is None else d_ossm_state.to(torch.float32).contiguous()
    dlast = None if d_ox_state is None else d_ox_state.to(torch.float32).contiguous()

    dx = torch.empty_like(x, memory_format=torch.contiguous_format)
    dA = torch.empty(batch, nheads, seqlen, dtype=torch.float32, device=dev)
    d_issm_state = (torch.empty((batch, nheads, head_dim, 1), dtype=torch.float32, device=dev)
                    if has_input_state else None)
    if x.numel() == 0:
        if d_issm_state is not None:
            d_issm_state.zero_()
        return dx, dA, d_issm_state

    ws = _lib.workspace(dev, _lib.lib.ema_scan_workspace_size(batch, seqlen, nheads, head_dim, chunk_size))
    a = _lib.EmaBwdArgs()
    a.batch, a.seqlen, a.nheads, a.headdim, a.chunk_size = batch, seqlen, nheads, head_dim, chunk_size
    a.dtype = _lib.DTYPE_CODES[x.dtype]
    a.x, a.x_stride = x_k.data_ptr(), _lib.strides3(x_k)
    a.dout, a.dout_stride = do_k.data_ptr(), _lib.strides3(do_k)
    a.dx, a.dx_stride = dx.data_ptr(), _lib.strides3(dx)
    a.da_cs, a.da_cs_sum = cs_k.data_ptr(), css_k.data_ptr()
    s = st_k.stride()  # (b, h, p, chunk) -> (b, chunk, h, p)
    a.states, a.states_stride = st_k.data_ptr(), (_lib._i64 * 4)(s[0], s[3], s[1], s[2])
    a.d_final_state = _lib.ptr(dfin)
    a.d_last_token = _lib.ptr(dlast)
    a.dl = dA.data_ptr()
    a.d_initial_state = _lib.ptr(d_issm_state)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    with torch.cuda.device(dev):
        _lib.check(_lib.lib.ema_bwd_launch(a, _lib.stream_ptr(dev)), "compute_dpx")
    return dx, dA, d_issm_state


# ---- dispatcher operators (namespace ema_b200) for the autograd pair below:
# torch.compile traces them (shape-only "fake" implementations) -------------
@torch.library.custom_op("ema_b200::ema_fwd_ref", mutates_args=(), device_types="cuda")
def _fwd_ref_op(x: torch.Tensor, dA: torch.Tensor, chunk_size: int) -> tuple[torch.Tensor, torch.Tensor,
                                                                             torch.Tensor, torch.Tensor]:
    """ema_fwd_triton with every store: (out, states (b, nc, h, 1, p), da_cs, da_cs_sum)."""
    out, states, da_cs, da_cs_sum = ema_fwd_triton(x, dA=dA, out=None, chunk_size=chunk_size, store_states=True,
                                                   store_da_cs=True, store_da_cs_sum=True)
    return out, states, da_cs, da_cs_sum


@_fwd_ref_op.register_fake
def _(x, dA, chunk_size):
    b, s, h, p = x.shape
    nc = -(-s // chunk_size)
    return (torch.empty_like(x, memory_format=torch.contiguous_format),
            x.new_empty((b, nc, h, 1, p), dtype=torch.float32), x.new_empty((b, h, s), dtype=torch.float32),
            x.new_empty((b, h, nc), dtype=torch.float32))


@torch.library.custom_op("ema_b200::ema_dpx", mutates_args=(), device_types="cuda")
def _dpx_op(x: torch.Tensor, da_cs: torch.Tensor, da_cs_sum: torch.Tensor, SSM_States: torch.Tensor,
            do: torch.Tensor, chunk_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    """compute_dpx without the optional state terms: (dX, per-token decay gradient)."""
    dx, dA, _ = compute_dpx(x, da_cs, da_cs_sum, SSM_States, do, chunk_size=chunk_size)
    return dx, dA


@_dpx_op.register_fake
def _(x, da_cs, da_cs_sum, SSM_States, do, chunk_size):
    b, s, h, _ = x.shape
    return (torch.empty_like(x, memory_format=torch.contiguous_format),
            x.new_empty((b, h, s), dtype=torch.float32))


class _EmaFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, A: torch.Tensor, chunk_size: int) -> torch.Tensor:
        # A is log(1 - P) in natural log space, shape (b, s), shared by all heads
        if x.ndim != 4:
            raise ValueError(f"x must be (batch, seqlen, nheads, head_dim), got {x.shape}")
        if A.ndim != 2:
            raise ValueError(f"A must be (batch, seqlen), got {A.shape}")
        batch, seqlen, nheads, _ = x.shape
        if A.shape != (batch, seqlen):
            raise ValueError(f"A must be (batch, seqlen), got {A.shape}")

        dA = (A * math.log2(math.e)).to(torch.float32)
        dA = dA[:, None, :].expand(batch, nheads, seqlen).contiguous()
        out, states, da_cs, da_cs_sum = torch.ops.ema_b200.ema_fwd_ref(x, dA, chunk_size)
        # (b, nchunks, h, 1, p) -> (b, h, p, nchunks) as a view; compute_dpx takes any strides
        ssm_states = states.squeeze(3).permute(0, 2, 3, 1)
        ctx.chunk_size = chunk_size
        ctx.save_for_backward(x, da_cs, da_cs_sum, ssm_states)
        return out

    @staticmethod
    def backward(ctx, grad_out: Optional[torch.Tensor] = None):
        if grad_out is None:
            return None, None, None
        x, da_cs, da_cs_sum, ssm_states = ctx.saved_tensors
        dx, dA = torch.ops.ema_b200.ema_dpx(x, da_cs, da_cs_sum, ssm_states, grad_out, ctx.chunk_size)
        # the decay is shared by all heads: its gradient is the head sum
        return dx, dA.sum(dim=1), None


def ema_combined(x: torch.Tensor, A: torch.Tensor, chunk_size: int = 64) -> torch.Tensor:
    return _EmaFunction.apply(x, A, chunk_size)
