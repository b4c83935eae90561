"""Mamba-2 SSD chunked scan (benchmark configs 3 and 5) on the B200 kernels.

Drop-in for the op the reference benchmarks its EMA against,
``mamba_ssm.ops.triton.ssd_combined.mamba_chunk_scan_combined(x, dt, A, B, C,
chunk_size, ...)`` (kernels/benchmarks/bench_ema_total.py:72-76; the package is
third-party and absent here).  Same argument names and layouts:

    x (batch, seqlen, nheads, headdim) bf16, dt (batch, seqlen, nheads),
    A (nheads,), B / C (batch, seqlen, ngroups, dstate) bf16, D (nheads,),
    initial_states / final states (batch, nheads, headdim, dstate) fp32

    s_t = exp(dt_t A_h) s_{t-1} + dt_t x_t B_t^T,   y_t = s_t C_t + D_h x_t

``dt_bias`` / ``dt_softplus`` / ``dt_limit`` map dt inside the SSD kernels
(dt <- clamp(softplus(dt + dt_bias), *dt_limit), the map's gradient folded into
the backward's ddt, plus the gradient of dt_bias), and ``z`` gates the output
(out <- y * silu(z), fp32 arithmetic, stored in y's dtype) on the native gate
kernels, one pass each way.  Not supported yet: ``seq_idx`` / ``cu_seqlens``
(packed sequences).

Two kernel families serve the call, by d_state:

* dstate 128, headdim 64, bf16 x (the Mamba-2 layer shapes of configs 3 and
  5): the SSD kernels (tcgen05 forward and backward).
* dstate 1 -- the reference's own benchmark call (bench_ema_total.py:62-76:
  x / dt in fp32, B = p and C = 1 of shape (batch, seqlen, 1, 1), A = -1): the
  state is a headdim vector, h_t = exp(dt_t A_h) h_{t-1} + dt_t B_t x_t,
  y_t = C_t h_t + D_h x_t, i.e. the dt-form EMA of B x scaled by C.  It runs
  on the EMA scan kernels (kernels.ema_chunk_scan) with the B and C scalings
  as autograd ops around them; any headdim <= 128, x in fp32 / bf16 / fp16.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F

from . import _lib

__all__ = ["ssd_chunk_scan_fwd", "ssd_chunk_scan_bwd", "mamba_chunk_scan_combined", "ssd_gate"]


def _s3(t):
    s = t.stride()
    return (_lib._i64 * 3)(s[0], s[1], s[2])


def _prep(x, dt, A, B, C, D):
    assert x.is_cuda and dt.is_cuda and A.is_cuda and B.is_cuda and C.is_cuda, "All tensors must be on CUDA"
    assert x.ndim == 4 and B.ndim == 4 and C.ndim == 4, "x (b,l,h,p); B, C (b,l,g,n)"
    b_, L, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    assert dt.shape == (b_, L, H), "dt must be (batch, seqlen, nheads)"
    assert A.shape == (H,), "A must be (nheads,)"
    assert B.shape == (b_, L, G, N) and C.shape == B.shape, "B and C must be (batch, seqlen, ngroups, dstate)"
    assert H % G == 0, "nheads must be a multiple of ngroups"
    assert D is None or D.shape == (H,), "D must be (nheads,)"
    assert x.dtype == torch.bfloat16, "the SSD kernels take bf16 x / B / C"

    def ok(t):
        return t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and all(s % 8 == 0 for s in t.stride()[:3])

    xk = x if ok(x) else x.contiguous()
    Bk = B.to(torch.bfloat16)
    Bk = Bk if ok(Bk) else Bk.contiguous()
    Ck = C.to(torch.bfloat16)
    Ck = Ck if ok(Ck) else Ck.contiguous()
    dtk = dt.to(torch.float32).contiguous()
    Ak = A.to(torch.float32).contiguous()
    Dk = None if D is None else D.to(torch.float32).contiguous()
    return b_, L, H, P, G, N, xk, dtk, Ak, Bk, Ck, Dk


def _set_dt_map(a, H, dev, dt_bias, dt_softplus, dt_limit):
    """The kernels' dt map in SsdFwdArgs / SsdBwdArgs: dt <- clamp(softplus(dt + dt_bias),
    *dt_limit), each step optional (the clamp only for a limit other than (0, inf), as
    the torch form of the map applies it).  Returns the bias tensor the launch reads."""
    bias = None
    if dt_bias is not None:
        assert dt_bias.shape == (H,), "dt_bias must be (nheads,)"
        bias = dt_bias.detach().to(device=dev, dtype=torch.float32).contiguous()
    lo, hi = float(dt_limit[0]), float(dt_limit[1])
    a.dt_bias = _lib.ptr(bias)
    a.dt_softplus = int(bool(dt_softplus))
    a.dt_clamp = int(lo > 0.0 or hi != float("inf"))
    a.dt_min, a.dt_max = lo, hi
    return bias


def ssd_chunk_scan_fwd(x, dt, A, B, C, D=None, initial_states=None, return_final_states=False,
                       save_states=True, dt_bias=None, dt_softplus=False, dt_limit=(0.0, float("inf"))):
    """Forward.  Returns (y, chunk_states or None, final_states or None).  ``dt`` is
    mapped inside the kernels: clamp(softplus(dt + dt_bias), *dt_limit), each step
    optional (mamba_chunk_scan_combined's dt options)."""
    b_, L, H, P, G, N, xk, dtk, Ak, Bk, Ck, Dk = _prep(x, dt, A, B, C, D)
    dev = x.device
    y = torch.empty(b_, L, H, P, dtype=x.dtype, device=dev)
    nci = int(_lib.lib.ssd_internal_chunks(L))
    cst = torch.empty(b_, nci, H, P, N, dtype=torch.float32, device=dev) if save_states else None
    fin = torch.empty(b_, H, P, N, dtype=torch.float32, device=dev) if return_final_states else None
    init = None
    if initial_states is not None:
        assert initial_states.shape == (b_, H, P, N), "initial_states must be (batch, nheads, headdim, dstate)"
        init = initial_states.to(torch.float32).contiguous()
    a = _lib.SsdFwdArgs()
    a.batch, a.seqlen, a.nheads, a.headdim, a.dstate, a.ngroups = b_, L, H, P, N, G
    a.dtype = _lib.DTYPE_CODES[torch.bfloat16]
    a.x, a.x_stride = xk.data_ptr(), _s3(xk)
    a.dt, a.A = dtk.data_ptr(), Ak.data_ptr()
    a.B, a.B_stride = Bk.data_ptr(), _s3(Bk)
    a.C, a.C_stride = Ck.data_ptr(), _s3(Ck)
    a.D = _lib.ptr(Dk)
    a.initial_state = _lib.ptr(init)
    a.out, a.out_stride = y.data_ptr(), _s3(y)
    a.chunk_states = _lib.ptr(cst)
    a.final_state = _lib.ptr(fin)
    bias = _set_dt_map(a, H, dev, dt_bias, dt_softplus, dt_limit)  # noqa: F841 (alive across the launch)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib.ssd_fwd_launch(a, _lib.stream_ptr(dev)), "ssd_chunk_scan_fwd")
    return y, cst, fin


def ssd_chunk_scan_bwd(x, dt, A, B, C, chunk_states, dy, D=None, d_final_states=None, need_d_initial=False,
                       dx_out=None, dt_bias=None, dt_softplus=False, dt_limit=(0.0, float("inf")),
                       ddt_bias_out=None):
    """Backward.  Returns (dx, ddt, dA, dB, dC, dD or None, d_initial_states or None);
    dB / dC are fp32 (batch, seqlen, ngroups, dstate), summed over each group's heads.
    With the forward's dt map (``dt_bias`` / ``dt_softplus`` / ``dt_limit``), ddt is
    the gradient of the dt given, and ``ddt_bias_out`` ((nheads,) fp32, optional)
    receives the gradient of dt_bias.
    ``dx_out``: a (batch, seqlen, nheads, headdim) bf16 buffer to write dx into
    (headdim stride 1, other strides even); the tensor-core kernel needs them to
    be multiples of 8 and 16-byte alignment, else the mma.sync kernel runs."""
    b_, L, H, P, G, N, xk, dtk, Ak, Bk, Ck, Dk = _prep(x, dt, A, B, C, D)
    dev = x.device
    assert dy.shape == x.shape
    dyk = dy.to(torch.bfloat16)
    dyk = dyk if (dyk.stride(-1) == 1 and dyk.data_ptr() % 16 == 0
                  and all(s % 8 == 0 for s in dyk.stride()[:3])) else dyk.contiguous()
    if dx_out is not None:
        assert dx_out.shape == x.shape and dx_out.dtype == x.dtype and dx_out.stride(-1) == 1, "dx_out"
        dx = dx_out
    else:
        dx = torch.empty(b_, L, H, P, dtype=x.dtype, device=dev)
    ddt = torch.empty(b_, L, H, dtype=torch.float32, device=dev)
    dA = torch.empty(H, dtype=torch.float32, device=dev)
    dB = torch.empty(b_, L, G, N, dtype=torch.float32, device=dev)
    dC = torch.empty(b_, L, G, N, dtype=torch.float32, device=dev)
    dD = torch.empty(H, dtype=torch.float32, device=dev) if D is not None else None
    d_init = torch.empty(b_, H, P, N, dtype=torch.float32, device=dev) if need_d_initial else None
    dfin = None if d_final_states is None else d_final_states.to(torch.float32).contiguous()
    a = _lib.SsdBwdArgs()
    a.batch, a.seqlen, a.nheads, a.headdim, a.dstate, a.ngroups = b_, L, H, P, N, G
    a.dtype = _lib.DTYPE_CODES[torch.bfloat16]
    a.x, a.x_stride = xk.data_ptr(), _s3(xk)
    a.dt, a.A = dtk.data_ptr(), Ak.data_ptr()
    a.B, a.B_stride = Bk.data_ptr(), _s3(Bk)
    a.C, a.C_stride = Ck.data_ptr(), _s3(Ck)
    a.D = _lib.ptr(Dk)
    a.chunk_states = chunk_states.data_ptr()
    a.dout, a.dout_stride = dyk.data_ptr(), _s3(dyk)
    a.d_final_state = _lib.ptr(dfin)
    a.dx, a.dx_stride = dx.data_ptr(), _s3(dx)
    a.ddt, a.dA, a.dB, a.dC = ddt.data_ptr(), dA.data_ptr(), dB.data_ptr(), dC.data_ptr()
    a.dD = _lib.ptr(dD)
    a.d_initial_state = _lib.ptr(d_init)
    bias = _set_dt_map(a, H, dev, dt_bias, dt_softplus, dt_limit)  # noqa: F841 (alive across the launch)
    if ddt_bias_out is not None:
        assert ddt_bias_out.shape == (H,) and ddt_bias_out.dtype == torch.float32 and ddt_bias_out.is_contiguous()
    a.ddt_bias = _lib.ptr(ddt_bias_out)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib.ssd_bwd_launch(a, _lib.stream_ptr(dev)), "ssd_chunk_scan_bwd")
    return dx, ddt, dA, dB, dC, dD, d_init


# ---- dispatcher operators (namespace ema_b200): torch.compile traces them
# (shape-only "fake" implementations), autograd through register_autograd ----
def _empty0(like):
    return like.new_empty((0,), dtype=torch.float32)


@torch.library.custom_op("ema_b200::ssd_fwd", mutates_args=(), device_types="cuda")
def _ssd_fwd_op(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, B: torch.Tensor, C: torch.Tensor,
                D: Optional[torch.Tensor], initial_states: Optional[torch.Tensor], dt_bias: Optional[torch.Tensor],
                dt_softplus: bool, dt_min: float, dt_max: float) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(y, the saved 64-token chunk states, the final state)."""
    return ssd_chunk_scan_fwd(x, dt, A, B, C, D, initial_states, True, dt_bias=dt_bias, dt_softplus=dt_softplus,
                              dt_limit=(dt_min, dt_max))


@_ssd_fwd_op.register_fake
def _(x, dt, A, B, C, D, initial_states, dt_bias, dt_softplus, dt_min, dt_max):
    b_, L, H, P = x.shape
    N = B.shape[3]
    nci = -(-L // 64)
    return (torch.empty(b_, L, H, P, dtype=x.dtype, device=x.device),
            x.new_empty((b_, nci, H, P, N), dtype=torch.float32), x.new_empty((b_, H, P, N), dtype=torch.float32))


@torch.library.custom_op("ema_b200::ssd_bwd", mutates_args=(), device_types="cuda")
def _ssd_bwd_op(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, B: torch.Tensor, C: torch.Tensor,
                chunk_states: torch.Tensor, dy: torch.Tensor, D: Optional[torch.Tensor],
                d_final_states: Optional[torch.Tensor], need_d_initial: bool, dt_bias: Optional[torch.Tensor],
                dt_softplus: bool, dt_min: float, dt_max: float) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor,
                                                                          torch.Tensor, torch.Tensor, torch.Tensor,
                                                                          torch.Tensor, torch.Tensor]:
    """(dx, ddt, dA, dB, dC, dD, d_initial_states, d dt_bias); the optional ones empty when absent."""
    dbias = None if dt_bias is None else torch.empty(dt_bias.shape, dtype=torch.float32, device=x.device)
    dx, ddt, dA, dB, dC, dD, d_init = ssd_chunk_scan_bwd(x, dt, A, B, C, chunk_states, dy, D, d_final_states,
                                                         need_d_initial, dt_bias=dt_bias, dt_softplus=dt_softplus,
                                                         dt_limit=(dt_min, dt_max), ddt_bias_out=dbias)
    # an absent output is its own empty tensor: outputs of an operator may not alias
    return (dx, ddt, dA, dB, dC, dD if dD is not None else _empty0(x), d_init if d_init is not None else _empty0(x),
            dbias if dbias is not None else _empty0(x))


@_ssd_bwd_op.register_fake
def _(x, dt, A, B, C, chunk_states, dy, D, d_final_states, need_d_initial, dt_bias, dt_softplus, dt_min, dt_max):
    b_, L, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    f32 = torch.float32
    return (torch.empty(b_, L, H, P, dtype=x.dtype, device=x.device), x.new_empty((b_, L, H), dtype=f32),
            x.new_empty((H,), dtype=f32), x.new_empty((b_, L, G, N), dtype=f32),
            x.new_empty((b_, L, G, N), dtype=f32), x.new_empty((H,), dtype=f32) if D is not None else _empty0(x),
            x.new_empty((b_, H, P, N), dtype=f32) if need_d_initial else _empty0(x),
            x.new_empty((H,), dtype=f32) if dt_bias is not None else _empty0(x))


def _ssd_setup(ctx, inputs, output):
    x, dt, A, B, C, D, initial_states, dt_bias, dt_softplus, dt_min, dt_max = inputs
    ctx.save_for_backward(x, dt, A, B, C, D, output[1], dt_bias)
    ctx.has_init = initial_states is not None
    ctx.opts = (dt_softplus, dt_min, dt_max)


def _ssd_backward(ctx, dy, _d_states, d_final):
    x, dt, A, B, C, D, cst, dt_bias = ctx.saved_tensors
    if dy is None:
        dy = torch.zeros_like(x)
    dx, ddt, dA, dB, dC, dD, d_init, dbias = torch.ops.ema_b200.ssd_bwd(x, dt, A, B, C, cst, dy, D, d_final,
                                                                        ctx.has_init, dt_bias, *ctx.opts)
    return (dx, ddt.to(dt.dtype), dA.to(A.dtype), dB.to(B.dtype), dC.to(C.dtype),
            None if D is None else dD.to(D.dtype), d_init if ctx.has_init else None,
            None if dt_bias is None else dbias.to(dt_bias.dtype), None, None, None)


torch.library.register_autograd("ema_b200::ssd_fwd", _ssd_backward, setup_context=_ssd_setup)


def _gate_args(y, z, out):
    a = _lib.SsdGateArgs()
    a.batch, a.seqlen, a.nheads, a.headdim = y.shape
    a.dtype = _lib.DTYPE_CODES[y.dtype]
    a.y, a.y_stride = y.data_ptr(), _s3(y)
    a.z, a.z_stride = z.data_ptr(), _s3(z)
    a.out, a.out_stride = out.data_ptr(), _s3(out)
    return a


def _last_dim_unit(t):
    return t if t.stride(-1) == 1 else t.contiguous()


@torch.library.custom_op("ema_b200::ssd_gate_fwd", mutates_args=(), device_types="cuda")
def _gate_fwd_op(y: torch.Tensor, z: torch.Tensor) -> torch.Tensor:
    """out = y * silu(z) on the native gate kernel (y, z of one dtype)."""
    assert y.ndim == 4 and z.shape == y.shape and z.dtype == y.dtype, "y and z: (batch, seqlen, nheads, headdim)"
    y, z = _last_dim_unit(y), _last_dim_unit(z)
    out = torch.empty_like(y, memory_format=torch.contiguous_format)
    a = _gate_args(y, z, out)
    with torch.cuda.device(y.device):
        _lib.check(_lib.lib.ssd_gate_fwd_launch(a, _lib.stream_ptr(y.device)), "ssd_gate_fwd")
    return out


@_gate_fwd_op.register_fake
def _(y, z):
    return torch.empty_like(y, memory_format=torch.contiguous_format)


@torch.library.custom_op("ema_b200::ssd_gate_bwd", mutates_args=(), device_types="cuda")
def _gate_bwd_op(y: torch.Tensor, z: torch.Tensor, dout: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(dy, dz) of out = y * silu(z), one pass."""
    y, z = _last_dim_unit(y), _last_dim_unit(z)
    dout = _last_dim_unit(dout.to(y.dtype))
    dy = torch.empty_like(y, memory_format=torch.contiguous_format)
    dz = torch.empty_like(z, memory_format=torch.contiguous_format)
    a = _gate_args(y, z, dy)
    a.dout, a.dout_stride = dout.data_ptr(), _s3(dout)
    a.dz, a.dz_stride = dz.data_ptr(), _s3(dz)
    with torch.cuda.device(y.device):
        _lib.check(_lib.lib.ssd_gate_bwd_launch(a, _lib.stream_ptr(y.device)), "ssd_gate_bwd")
    return dy, dz


@_gate_bwd_op.register_fake
def _(y, z, dout):
    return (torch.empty_like(y, memory_format=torch.contiguous_format),
            torch.empty_like(z, memory_format=torch.contiguous_format))


def _gate_setup(ctx, inputs, output):
    ctx.save_for_backward(*inputs)


def _gate_backward(ctx, dout):
    y, z = ctx.saved_tensors
    return torch.ops.ema_b200.ssd_gate_bwd(y, z, dout)


torch.library.register_autograd("ema_b200::ssd_gate_fwd", _gate_backward, setup_context=_gate_setup)


def ssd_gate(y: torch.Tensor, z: torch.Tensor) -> torch.Tensor:
    """out = y * silu(z) (mamba_chunk_scan_combined's ``z``), fp32 arithmetic rounded once
    to y's dtype; z is taken in y's dtype (its gradient returns in z's own)."""
    return torch.ops.ema_b200.ssd_gate_fwd(y, z.to(y.dtype))


def _ssd_state1(x, dt, A, B, C, D, initial_states, return_final_states, chunk_size):
    """d_state = 1: y = C * EMA_dt(B x) + D x on the EMA kernels (autograd throughout).

    B and C (batch, seqlen, ngroups, 1) are per-token scalars of each head's
    group; the products with them run in fp32 around the scan, which takes
    B x in fp32 whatever x's dtype, so no extra rounding enters."""
    from .ema_chunk_scan import ema_chunk_scan_combined
    b_, L, H, P = x.shape
    G = B.shape[2]
    assert B.shape == (b_, L, G, 1) and C.shape == B.shape, "B and C must be (batch, seqlen, ngroups, 1)"
    assert H % G == 0, "nheads must be a multiple of ngroups"
    assert dt.shape == (b_, L, H) and A.shape == (H,), "dt (batch, seqlen, nheads), A (nheads,)"
    grp = torch.arange(H, device=x.device) // (H // G)
    Bh = B[..., 0].float()[:, :, grp]  # (b, l, H)
    Ch = C[..., 0].float()[:, :, grp]
    xf = x.float()  # one conversion: both gradient paths into x sum in fp32 before its single rounding
    xb = xf * Bh[..., None]
    q = min(max(chunk_size, 64), 256)  # the scan's tile length; the result does not depend on it
    init = None if initial_states is None else initial_states[..., 0]
    out = ema_chunk_scan_combined(xb, dt, A, q, initial_states=init, return_final_states=return_final_states)
    z, fin = out if return_final_states else (out, None)
    y = z * Ch[..., None]
    if D is not None:
        y = y + D.float()[None, None, :, None] * xf
    y = y.to(x.dtype)
    return (y, fin[..., None]) if return_final_states else y


def mamba_chunk_scan_combined(x, dt, A, B, C, chunk_size, D=None, z=None, dt_bias=None, initial_states=None,
                              seq_idx=None, cu_seqlens=None, dt_softplus=False, dt_limit=(0.0, float("inf")),
                              return_final_states=False, return_varlen_states=False):
    """mamba_ssm's ``mamba_chunk_scan_combined`` on the B200 SSD kernels (autograd).

    Returns y, or (y, final_states) with ``return_final_states``; with ``z``
    (batch, seqlen, nheads, headdim) y is gated by silu(z).  ``chunk_size`` is
    accepted for signature compatibility; the result does not depend on it."""
    assert seq_idx is None and cu_seqlens is None and not return_varlen_states, \
        "packed sequences (seq_idx / cu_seqlens) are not supported yet"
    assert chunk_size > 0 and math.log2(chunk_size).is_integer(), "chunk_size must be a power of two"
    assert z is None or z.shape == x.shape, "z must have the shape of x"
    if B.shape[-1] == 1:
        # the EMA kernels take dt as given: the map runs as torch ops here
        if dt_bias is not None:
            dt = dt + dt_bias
        if dt_softplus:
            dt = F.softplus(dt)
        dt_min, dt_max = float(dt_limit[0]), float(dt_limit[1])
        if dt_min > 0.0 or dt_max != float("inf"):
            dt = dt.clamp(dt_min, dt_max)
        out = _ssd_state1(x, dt, A, B, C, D, initial_states, return_final_states, chunk_size)
    else:  # the SSD kernels apply the dt map themselves
        y, _, fin = torch.ops.ema_b200.ssd_fwd(x, dt, A, B, C, D, initial_states, dt_bias, bool(dt_softplus),
                                               float(dt_limit[0]), float(dt_limit[1]))
        out = (y, fin) if return_final_states else y
    if z is None:
        return out
    y, fin = out if return_final_states else (out, None)
    y = ssd_gate(y, z)
    return (y, fin) if return_final_states else y
