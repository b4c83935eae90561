"""dt-parameterised EMA chunked scan (no counterpart in the reference's own code).

    h_t = exp(dt_t * A_h) * h_{t-1} + dt_t * x_t,     y_t = h_t

per (batch, head, channel).  This is the reference EMA with X = dt * x and
log2 decay dA = dt * A * log2(e), i.e. Mamba-2 SSD with d_state = 1 and
B = C = 1; the call form follows the SSD op the reference benchmarks against
(``mamba_chunk_scan_combined(x, dt, A, B, C, chunk_size, ...)``,
kernels/benchmarks/bench_ema_total.py:72-76) without B, C.

Shapes: x (batch, seqlen, nheads, headdim) bf16/fp16/fp32; dt (batch, seqlen,
nheads); A (nheads,); initial/final states (batch, nheads, headdim) fp32.
Gradients: dx = dt * G, ddt = sum_p G x + A * dl, dA = sum_{b,t} dt * dl with
G the state gradient and dl the per-token natural-log-decay gradient.

The forward stores only the chunk START states (batch, nchunks, nheads,
headdim) fp32 for the backward; everything else is recomputed on chip, so a
forward + backward moves the minimum HBM bytes: x twice, y, dy, dx once,
dt twice and ddt once.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib

__all__ = ["ema_chunk_scan_fwd", "ema_chunk_scan_bwd", "ema_chunk_scan_combined"]


def _check_inputs(x, dt, A, chunk_size):
    assert x.is_cuda and dt.is_cuda and A.is_cuda, "All tensors must be on CUDA"
    assert x.ndim == 4, "x must be (batch, seqlen, nheads, headdim)"
    B, L, H, P = x.shape
    assert dt.shape == (B, L, H), f"dt must be (batch, seqlen, nheads), got {tuple(dt.shape)}"
    assert A.shape == (H,), f"A must be (nheads,), got {tuple(A.shape)}"
    assert chunk_size in (64, 128, 256), "chunk_size must be 64, 128 or 256"
    assert x.dtype in _lib.DTYPE_CODES, f"unsupported dtype {x.dtype}"
    return B, L, H, P


def ema_chunk_scan_fwd(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, chunk_size: int = 256,
                       initial_states: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                       return_final_states: bool = False, state_only: bool = False,
                       half_chunk_states: bool = False, dt_rows: Optional[torch.Tensor] = None):
    """Forward.  Returns (y, chunk_start_states (B, nchunks, H, P) fp32, final_states or None).

    ``state_only``: compute only the final state (y and the chunk states are not
    written; returns (None, None, final)) -- the first pass of the sequence-
    parallel forward, which reads x once and writes nothing else.

    ``half_chunk_states``: the states returned are those entering every
    chunk_size / 2 tokens, (B, ceil(L / (chunk_size / 2)), H, P) -- what
    ``ema_chunk_scan_bwd`` takes with ``chunk_size // 2`` (chunk c's start
    state at index 2c)."""
    B, L, H, P = _check_inputs(x, dt, A, chunk_size)
    dev = x.device
    nc = -(-L // chunk_size)
    x_k = _lib.tma_ready(x)
    dt_k = dt.to(torch.float32).contiguous()
    A_k = A.to(torch.float32).contiguous()
    if state_only:
        assert out is None, "state_only writes no output"
        return_final_states = True
    elif out is None:
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
    if out is not None:
        assert out.shape == x.shape and out.dtype == x.dtype and _lib.tma_ok(out), "out must match x"
    states = None if state_only else torch.empty(B, nc, H, P, dtype=torch.float32, device=dev)
    mid = None
    if half_chunk_states and not state_only:
        fine = torch.empty(B, 2 * nc, H, P, dtype=torch.float32, device=dev)
        states, mid = fine[:, 0::2], fine[:, 1::2]
    final = torch.empty(B, H, P, dtype=torch.float32, device=dev) if return_final_states else None
    init = None
    if initial_states is not None:
        assert initial_states.shape == (B, H, P), "initial_states must be (batch, nheads, headdim)"
        init = initial_states.to(torch.float32).contiguous()
    if x.numel() == 0:
        if final is not None:
            final.copy_(init if init is not None else torch.zeros_like(final))
        return out, (fine[:, :-(-L // (chunk_size // 2))] if mid is not None else states), final
    ws = _lib.workspace(dev, _lib.lib.ema_scan_workspace_size(B, L, H, P, chunk_size))
    if dt_rows is None:
        dt_rows = torch.empty(B, H, L, dtype=torch.float32, device=dev)
    assert dt_rows.shape == (B, H, L) and dt_rows.dtype == torch.float32 and dt_rows.is_contiguous(), \
        "dt_rows must be a contiguous (batch, nheads, seqlen) float32 buffer"
    a = _lib.EmaFwdArgs()
    a.batch, a.seqlen, a.nheads, a.headdim, a.chunk_size = B, L, H, P, chunk_size
    a.dtype = _lib.DTYPE_CODES[x.dtype]
    a.x, a.x_stride = x_k.data_ptr(), _lib.strides3(x_k)
    if out is not None:
        a.out, a.out_stride = out.data_ptr(), _lib.strides3(out)
    a.dt, a.A = dt_k.data_ptr(), A_k.data_ptr()
    a.initial_state = _lib.ptr(init)
    if states is not None:
        s = states.stride()
        a.states, a.states_stride = states.data_ptr(), (_lib._i64 * 4)(s[0], s[1], s[2], s[3])
    if mid is not None:
        s = mid.stride()
        a.mid_states, a.mid_states_stride = mid.data_ptr(), (_lib._i64 * 4)(s[0], s[1], s[2], s[3])
    a.final_state = _lib.ptr(final)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    a.dt_rows = dt_rows.data_ptr()
    with torch.cuda.device(dev):
        _lib.check(_lib.lib.ema_fwd_launch(a, _lib.stream_ptr(dev)), "ema_chunk_scan_fwd")
    if mid is not None:  # the chunk-start states of chunk_size / 2 (a short last chunk has no mid)
        states = fine[:, :-(-L // (chunk_size // 2))]
    return out, states, final


def ema_chunk_scan_bwd(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, states: torch.Tensor,
                       dy: torch.Tensor, chunk_size: int = 256,
                       d_final_states: Optional[torch.Tensor] = None, need_d_initial: bool = False,
                       state_only: bool = False, dt_rows: Optional[torch.Tensor] = None):
    """Backward.  Returns (dx, ddt fp32 (B,L,H), dA fp32 (H,), d_initial_states or None).

    ``state_only``: compute only the gradient w.r.t. the initial state (returns
    (None, None, None, d_initial)) -- the first pass of the sequence-parallel
    backward; dx, ddt and dA are not written.

    ``dt_rows``: dt transposed to (B, H, L), as the forward leaves it in its
    ``dt_rows`` buffer; made here (one transpose launch) when not given."""
    B, L, H, P = _check_inputs(x, dt, A, chunk_size)
    dev = x.device
    nc = -(-L // chunk_size)
    assert states.shape == (B, nc, H, P), "states must be the forward's chunk start states"
    assert dy.shape == x.shape
    x_k = _lib.tma_ready(x)
    dy_k = _lib.tma_ready(dy if dy.dtype == x.dtype else dy.to(x.dtype))
    dt_k = dt.to(torch.float32).contiguous()
    A_k = A.to(torch.float32).contiguous()
    if state_only:
        need_d_initial = True
        dx = ddt = dA = None
    else:
        dx = torch.empty_like(x, memory_format=torch.contiguous_format)
        ddt = torch.empty(B, L, H, dtype=torch.float32, device=dev)
        dA = torch.empty(H, dtype=torch.float32, device=dev)
    d_init = torch.empty(B, H, P, dtype=torch.float32, device=dev) if need_d_initial else None
    dfin = None if d_final_states is None else d_final_states.to(torch.float32).contiguous()
    if x.numel() == 0:
        if dA is not None:
            dA.zero_()
        if d_init is not None:
            d_init.copy_(dfin if dfin is not None else torch.zeros_like(d_init))
        return dx, ddt, dA, d_init
    ws = _lib.workspace(dev, _lib.lib.ema_scan_workspace_size(B, L, H, P, chunk_size))
    if dt_rows is None:
        dt_rows = torch.empty(B, H, L, dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(_lib.lib.ema_dt_rows_launch(dt_k.data_ptr(), dt_rows.data_ptr(), B, L, H,
                                                   _lib.stream_ptr(dev)), "ema_dt_rows")
    assert dt_rows.shape == (B, H, L) and dt_rows.dtype == torch.float32 and dt_rows.is_contiguous(), \
        "dt_rows must be a contiguous (batch, nheads, seqlen) float32 buffer"
    a = _lib.EmaBwdArgs()
    a.batch, a.seqlen, a.nheads, a.headdim, a.chunk_size = B, L, H, P, chunk_size
    a.dtype = _lib.DTYPE_CODES[x.dtype]
    a.x, a.x_stride = x_k.data_ptr(), _lib.strides3(x_k)
    a.dout, a.dout_stride = dy_k.data_ptr(), _lib.strides3(dy_k)
    if dx is not None:
        a.dx, a.dx_stride = dx.data_ptr(), _lib.strides3(dx)
    a.dt, a.A = dt_k.data_ptr(), A_k.data_ptr()
    s = states.stride()
    a.states, a.states_stride = states.data_ptr(), (_lib._i64 * 4)(s[0], s[1], s[2], s[3])
    a.d_final_state = _lib.ptr(dfin)
    a.ddt, a.dA_out = _lib.ptr(ddt), _lib.ptr(dA)
    a.d_initial_state = _lib.ptr(d_init)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    a.dt_rows = dt_rows.data_ptr()
    with torch.cuda.device(dev):
        _lib.check(_lib.lib.ema_bwd_launch(a, _lib.stream_ptr(dev)), "ema_chunk_scan_bwd")
    return dx, ddt, dA, d_init


def backward_chunk(chunk_size: int) -> int:
    """Tile length the backward runs on for a forward of ``chunk_size``: 256-token
    forwards hand the backward 128-token chunk states (two backward CTAs per SM,
    measured faster on B200); otherwise the same length."""
    return 128 if chunk_size == 256 else chunk_size


# ---- dispatcher operators (namespace ema_b200): traceable by torch.compile,
# with shape-only ("fake") implementations and an autograd formula ----------
@torch.library.custom_op("ema_b200::ema_scan_dt_fwd", mutates_args=(), device_types="cuda")
def _scan_fwd_op(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, chunk_size: int, half_chunk_states: bool,
                 initial_states: Optional[torch.Tensor]) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor,
                                                                  torch.Tensor]:
    """(y, chunk start states, final state, dt as (B, H, L) rows for the backward)."""
    B, L, H, _ = x.shape
    dt_rows = torch.empty(B, H, L, dtype=torch.float32, device=x.device)
    y, states, final = ema_chunk_scan_fwd(x, dt, A, chunk_size, initial_states=initial_states,
                                          return_final_states=True, half_chunk_states=half_chunk_states,
                                          dt_rows=dt_rows)
    return y, states, final, dt_rows


@_scan_fwd_op.register_fake
def _(x, dt, A, chunk_size, half_chunk_states, initial_states):
    B, L, H, P = x.shape
    nc = -(-L // chunk_size)
    if half_chunk_states:
        states = x.new_empty((B, 2 * nc, H, P), dtype=torch.float32)[:, :-(-L // (chunk_size // 2))]
    else:
        states = x.new_empty((B, nc, H, P), dtype=torch.float32)
    return (torch.empty_like(x, memory_format=torch.contiguous_format), states,
            x.new_empty((B, H, P), dtype=torch.float32), x.new_empty((B, H, L), dtype=torch.float32))


@torch.library.custom_op("ema_b200::ema_scan_dt_bwd", mutates_args=(), device_types="cuda")
def _scan_bwd_op(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, states: torch.Tensor, dy: torch.Tensor,
                 chunk_size: int, d_final_states: Optional[torch.Tensor], need_d_initial: bool,
                 dt_rows: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """(dx, ddt, dA, d_initial_states -- empty unless ``need_d_initial``)."""
    dx, ddt, dA, d_init = ema_chunk_scan_bwd(x, dt, A, states, dy, chunk_size, d_final_states=d_final_states,
                                             need_d_initial=need_d_initial, dt_rows=dt_rows)
    return dx, ddt, dA, d_init if d_init is not None else x.new_empty((0,), dtype=torch.float32)


@_scan_bwd_op.register_fake
def _(x, dt, A, states, dy, chunk_size, d_final_states, need_d_initial, dt_rows):
    B, L, H, P = x.shape
    return (torch.empty_like(x, memory_format=torch.contiguous_format),
            x.new_empty((B, L, H), dtype=torch.float32), x.new_empty((H,), dtype=torch.float32),
            x.new_empty((B, H, P) if need_d_initial else (0,), dtype=torch.float32))


def _scan_setup(ctx, inputs, output):
    x, dt, A, chunk_size, half_chunk_states, initial_states = inputs
    ctx.save_for_backward(x, dt, A, output[1], output[3])
    ctx.chunk_size = chunk_size // 2 if half_chunk_states else chunk_size
    ctx.has_init = initial_states is not None


def _scan_backward(ctx, dy, _d_states, d_final, _d_rows):
    x, dt, A, states, dt_rows = ctx.saved_tensors
    if dy is None:
        dy = torch.zeros_like(x)
    dx, ddt, dA, d_init = torch.ops.ema_b200.ema_scan_dt_bwd(x, dt, A, states, dy, ctx.chunk_size, d_final,
                                                              ctx.has_init, dt_rows)
    return dx, ddt.to(dt.dtype), dA.to(A.dtype), None, None, d_init if ctx.has_init else None


torch.library.register_autograd("ema_b200::ema_scan_dt_fwd", _scan_backward, setup_context=_scan_setup)


def ema_chunk_scan_combined(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, chunk_size: int = 256,
                            initial_states: Optional[torch.Tensor] = None,
                            return_final_states: bool = False):
    """Autograd op: y (and the final state when ``return_final_states``).  Runs the
    registered operator ``torch.ops.ema_b200.ema_scan_dt_fwd`` (its backward:
    ``ema_scan_dt_bwd``), so ``torch.compile`` traces it without a graph break."""
    _check_inputs(x, dt, A, chunk_size)
    y, _, final, _ = torch.ops.ema_b200.ema_scan_dt_fwd(x, dt, A, chunk_size, backward_chunk(chunk_size) != chunk_size,
                                                         initial_states)
    return (y, final) if return_final_states else y
