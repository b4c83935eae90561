"""EMA forward on B200 -- drop-in for ``kernels.forward.ema_ssd_fwd`` of the reference.

``ema_fwd_triton`` and ``chunk_cumsum_triton`` keep the reference's names,
argument names, defaults, output shapes/dtypes and return conventions
(kernels/forward/ema_ssd_fwd.py:160-212, :413-516), but launch the sm_100a
kernels of libema_ssd_b200.so through its C ABI instead of Triton kernels.

Differences, all deliberate:
* ``chunk_size`` may be 64, 128 or 256 (the reference asserts 64 or 128,
  ema_ssd_fwd.py:439); the result is mathematically chunk-size independent.
* The chunk decay matrix and the state-update weights are kept in fp32; the
  reference rounds both to the input dtype before its ``tl.dot``
  (ema_ssd_fwd.py:368, :385), so bf16 results here are closer to the exact
  recurrence.
* ``seq_idx`` restarts the state wherever the id changes from the previous
  token -- the rule of the reference's own oracle ``ema_torch_ref_seq_idx``
  (ema_ssd_fwd.py:562-594).  The reference kernel itself only handles
  segments that start on a chunk boundary with headdim == chunk_size
  (its mask at :389 is broadcast against the channel axis).
"""

from __future__ import annotations

from typing import Optional

import torch

from .. import _lib

__all__ = ["ema_fwd_triton", "chunk_cumsum_triton"]

_CHUNKS = (64, 128, 256)


def _seq_idx_arg(seq_idx: Optional[torch.Tensor]):
    if seq_idx is None:
        return None, 0
    if seq_idx.dtype not in _lib.IDX_CODES:
        seq_idx = seq_idx.to(torch.int32)
    seq_idx = seq_idx.contiguous()
    return seq_idx, _lib.IDX_CODES[seq_idx.dtype]


def ema_fwd_triton(
    x: torch.Tensor,  # (b, s, h, dx)
    dA: Optional[torch.Tensor] = None,  # (b, h, s)
    out: Optional[torch.Tensor] = None,  # (b, s, h, dx)
    seq_idx: Optional[torch.Tensor] = None,  # (b, s)
    chunk_size: int = 64,
    store_states: bool = False,
    store_da_cs: bool = False,
    store_da_cs_sum: bool = False,
):
    """EMA forward ``Z[t] = exp2(dA[t]) * Z[t-1] + X[t]`` per (batch, head).

    Args:
        x: (b, s, h, dx), float32 / bfloat16 / float16.
        dA: log2 decay (b, h, s); ``exp2(dA)`` is the per-token decay.
        out: optional output (b, s, h, dx) of x's dtype.
        seq_idx: optional (b, s) integer ids of packed sequences.
        chunk_size: 64, 128 or 256.
        store_states: also return per-chunk START states (b, nchunks, h, 1, dx), fp32.
        store_da_cs: also return the within-chunk cumsum of dA (b, h, s), fp32.
        store_da_cs_sum: also return per-chunk sums of dA (b, h, nchunks), fp32.

    Returns:
        out, or a tuple in the reference's order: (out, states, da_cs, da_cs_sum)
        restricted to the requested outputs.
    """
    assert chunk_size in _CHUNKS, f"chunk_size must be one of {_CHUNKS}"
    assert dA is not None
    assert x.is_cuda, "Tensors must be on CUDA"
    assert dA.is_cuda, "dA tensor must be on CUDA"
    assert x.ndim == 4, "x must be (batch, seqlen, nheads, headdim)"
    assert x.dtype in _lib.DTYPE_CODES, f"unsupported dtype {x.dtype}"

    batch, seqlen, nheads, headdim = x.shape
    assert dA.shape == (batch, nheads, seqlen), "dA must be (batch, nheads, seqlen)"
    num_chunks = -(-seqlen // chunk_size)
    dev = x.device

    x_k = _lib.tma_ready(x)
    dA_k = dA.to(torch.float32).contiguous()
    user_out = out
    if out is None:
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
    assert out.shape == x.shape and out.dtype == x.dtype, "out must match x"
    out_k = out if _lib.tma_ok(out) else torch.empty_like(x, memory_format=torch.contiguous_format)
    states = (torch.empty(batch, num_chunks, nheads, 1, headdim, dtype=torch.float32, device=dev)
              if store_states else None)
    da_cs = torch.empty(batch, nheads, seqlen, dtype=torch.float32, device=dev) if store_da_cs else None
    da_cs_sum = (torch.empty(batch, nheads, num_chunks, dtype=torch.float32, device=dev)
                 if store_da_cs_sum else None)
    seq_k, seq_code = _seq_idx_arg(seq_idx)

    if x.numel() > 0:
        ws = _lib.workspace(dev, _lib.lib.ema_scan_workspace_size(batch, seqlen, nheads, headdim, chunk_size))
        a = _lib.EmaFwdArgs()
        a.batch, a.seqlen, a.nheads, a.headdim, a.chunk_size = batch, seqlen, nheads, headdim, chunk_size
        a.dtype = _lib.DTYPE_CODES[x.dtype]
        a.seq_idx_type = seq_code
        a.x, a.x_stride = x_k.data_ptr(), _lib.strides3(x_k)
        a.out, a.out_stride = out_k.data_ptr(), _lib.strides3(out_k)
        a.dA = dA_k.data_ptr()
        a.seq_idx = _lib.ptr(seq_k)
        if states is not None:
            s = states.stride()
            a.states = states.data_ptr()
            a.states_stride = (_lib._i64 * 4)(s[0], s[1], s[2], s[4])
        a.da_cs = _lib.ptr(da_cs)
        a.da_cs_sum = _lib.ptr(da_cs_sum)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        with torch.cuda.device(dev):
            _lib.check(_lib.lib.ema_fwd_launch(a, _lib.stream_ptr(dev)), "ema_fwd_triton")
        if out_k is not out:
            out.copy_(out_k)
    out = user_out if user_out is not None else out

    if store_states and store_da_cs and store_da_cs_sum:
        return out, states, da_cs, da_cs_sum
    if store_states and store_da_cs:
        return out, states, da_cs
    if store_states and store_da_cs_sum:
        return out, states, da_cs_sum
    if store_da_cs and store_da_cs_sum:
        return out, da_cs, da_cs_sum
    if store_states:
        return out, states
    if store_da_cs:
        return out, da_cs
    if store_da_cs_sum:
        return out, da_cs_sum
    return out


def chunk_cumsum_triton(
    dA: torch.Tensor,  # (batch, nheads, seqlen)
    chunk_size: int = 64,
    dA_cs: Optional[torch.Tensor] = None,
    dA_cs_rev: Optional[torch.Tensor] = None,
    exp2: bool = False,
):
    """Within-chunk cumsums of dA (batch, nheads, seqlen).

    ``dA_cs[t]`` = sum of dA from the chunk start through t (inclusive);
    ``dA_cs_rev[t]`` = sum of dA over (t, chunk end] (exclusive, 0 at the
    chunk's last token).  With ``exp2`` both are exponentiated (base 2).

    Examples:
        Forward cumsum: [a, b, c, d] -> [a, a+b, a+b+c, a+b+c+d]
        Reverse (exclusive): [a, b, c, d] -> [b+c+d, c+d, d, 0]

    Returns:
        (dA_cs, dA_cs_rev)
    """
    batch, nheads, seqlen = dA.shape
    if dA_cs is None:
        dA_cs = torch.empty_like(dA)
    if dA_cs_rev is None:
        dA_cs_rev = torch.empty_like(dA)
    assert dA.is_cuda, "Input tensor must be on CUDA"
    assert dA_cs.shape == dA.shape, "Output tensor must have same shape as input"
    assert dA_cs_rev.shape == dA.shape, "Reverse cumsum output must have same shape as input"
    if dA.numel() == 0:
        return dA_cs, dA_cs_rev
    src = dA if dA.dtype == torch.float32 else dA.float()
    cs = dA_cs if dA_cs.dtype == torch.float32 else torch.empty(dA.shape, dtype=torch.float32, device=dA.device)
    rv = (dA_cs_rev if dA_cs_rev.dtype == torch.float32
          else torch.empty(dA.shape, dtype=torch.float32, device=dA.device))
    st = lambda t: (_lib._i64 * 3)(*t.stride())  # noqa: E731
    with torch.cuda.device(dA.device):
        _lib.check(_lib.lib.chunk_cumsum_launch(src.data_ptr(), st(src), cs.data_ptr(), st(cs), rv.data_ptr(),
                                                st(rv), batch, nheads, seqlen, chunk_size, int(bool(exp2)),
                                                _lib.stream_ptr(dA.device)), "chunk_cumsum_triton")
    if cs is not dA_cs:
        dA_cs.copy_(cs)
    if rv is not dA_cs_rev:
        dA_cs_rev.copy_(rv)
    return dA_cs, dA_cs_rev
