"""Sequence-parallel dt-form EMA over a torch.distributed process group.

For sequences too long for one GPU's time budget (benchmark config 4:
B1 L65536 H32 P64), rank r of a group of R owns tokens
[r L/R, (r+1) L/R) of every (batch, head) chain.  The recurrence

    h_t = exp(dt_t A_h) h_{t-1} + dt_t x_t

is affine in h, so a span acts on its incoming state as h -> D h + S with
D = exp(A_h sum_span dt) and S the span's end state from a zero start.

Forward:
  1. state-only pass over the local span (reads x once, writes nothing but
     S_r, (B, H, P) fp32; a weighted column sum, ``span_state``);
  2. chain the spans with NCCL send/recv, r -> r+1: rank r receives its
     incoming state Sin_r and sends D_r Sin_r + S_r on;
  3. the local pass from the true incoming state (y, chunk start states).
Backward, the mirror image:
  1. state-only pass: the gradient w.r.t. the span's incoming state from the
     local dy;
  2. chain r+1 -> r: rank r receives the gradient w.r.t. its span's end state
     Gin_r and sends D_r Gin_r + G_r back;
  3. the local backward with d_final_states = Gin_r (dx, ddt and this span's
     dA), then one all-reduce of the H per-head dA values.

Messages are (B, H, P) fp32 (8 KB at config 4); the only collective on the
data path is the per-head dA sum.  Every rank takes the same collective steps
in the same order.  The local passes are injectable so the host logic can be
tested on CPU ranks (gloo) against the float64 oracle.

``exchange="allgather"`` replaces each direction's chain of R - 1 dependent
send/recv hops by one all_gather of every rank's span summary (its end state,
or start gradient, from a zero boundary, and its decay D); each rank then
folds the summaries before its span itself -- the same fp32 arithmetic the
chain performs, without R - 1 message latencies in series.  The default is
the send/recv chain.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _lib
from .ema_chunk_scan import backward_chunk, ema_chunk_scan_bwd, ema_chunk_scan_fwd

__all__ = ["span_decay", "span_state", "subspan_count", "sp_forward", "sp_backward", "ema_chunk_scan_sp",
           "p2p_exchange_status"]


def span_decay(dt: torch.Tensor, A: torch.Tensor) -> torch.Tensor:
    """D = exp(A_h * sum_t dt[b, t, h]) over the local span, (B, H) fp32."""
    return torch.exp(dt.to(torch.float32).sum(dim=1) * A.to(torch.float32))


def _gather(v: torch.Tensor, D: torch.Tensor, group):
    """Every rank's (B, H, P) vector and (B, H) decay, stacked by rank: one
    all_gather into a flat buffer."""
    world = dist.get_world_size(group)
    msg = torch.cat([v.reshape(-1), D.reshape(-1)]).to(torch.float32).contiguous()
    out = torch.empty(world * msg.numel(), dtype=torch.float32, device=msg.device)
    dist.all_gather_into_tensor(out, msg, group=group)
    out = out.view(world, -1)
    n = v.numel()
    return out[:, :n].view(world, *v.shape), out[:, n:].view(world, *D.shape)


def _fold(V: torch.Tensor, D: torch.Tensor) -> torch.Tensor:
    """sum_q (prod_{j > q} D_j) V_q over the stacked summaries V (n, B, H, P) and
    decays D (n, B, H): the chain's recurrence s <- D_q s + V_q from s = 0
    (without the last decay), in a fixed number of launches."""
    n = V.shape[0]
    if n == 1:
        return V[0].clone()
    # w_q = D_{q+1} ... D_{n-1}, w_{n-1} = 1
    w = torch.cat([torch.cumprod(D[1:].flip(0), dim=0).flip(0), torch.ones_like(D[:1])], dim=0)
    return (w[..., None] * V).sum(dim=0)


class _P2PExchange:
    """Exchange buffers of one process group for the "p2p" span exchange
    (ema_span_exchange): this rank's buffer (ema_p2p_alloc, zeroed) and every
    peer's, mapped through CUDA IPC.  Built on the first exchange of a
    (group, device, batch x heads, headdim) -- outside CUDA graph capture --
    and kept for the life of the process.  The ranks must sit on different
    GPUs: the kernel of every rank waits for the others' flags, which two
    launches on one GPU cannot be relied on to satisfy."""
    _cache = {}

    @classmethod
    def get(cls, group, device, bh: int, P: int):
        key = (id(group), device.index, bh, P)
        ex = cls._cache.get(key)
        if ex is None:
            assert not torch.cuda.is_current_stream_capturing(), \
                "the p2p span exchange sets up its buffers on its first call, outside CUDA graph capture"
            ex = cls._cache[key] = cls(group, device, bh, P)
        return ex

    def __init__(self, group, device, bh: int, P: int):
        import ctypes
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if self.world > _lib.SPAN_EXCHANGE_MAX_RANKS:
            raise ValueError(f"the p2p span exchange takes at most {_lib.SPAN_EXCHANGE_MAX_RANKS} ranks")
        uuids = [None] * self.world
        dist.all_gather_object(uuids, str(torch.cuda.get_device_properties(device).uuid), group=group)
        if len(set(uuids)) != self.world:
            raise ValueError("the p2p span exchange needs every rank on its own GPU")
        self.nbytes = int(_lib.lib.ema_span_exchange_bytes(self.world, bh, P))
        own = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * _lib.P2P_HANDLE_BYTES)()
        with torch.cuda.device(device):
            _lib.check(_lib.lib.ema_p2p_alloc(self.nbytes, ctypes.byref(own)), "ema_p2p_alloc")
            _lib.check(_lib.lib.ema_p2p_handle(own, handle), "ema_p2p_handle")
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            self.ptrs = []
            for q, hb in enumerate(handles):
                if q == self.rank:
                    self.ptrs.append(own.value)
                    continue
                peer = ctypes.c_void_p()
                hq = (ctypes.c_ubyte * _lib.P2P_HANDLE_BYTES).from_buffer_copy(hb)
                _lib.check(_lib.lib.ema_p2p_open(hq, ctypes.byref(peer)), "ema_p2p_open")
                self.ptrs.append(peer.value)
        dist.barrier(group=group)  # every buffer zeroed and mapped everywhere before the first exchange

    def status(self, clear: bool = False) -> int:
        """The own buffer's status word (bit 1: a wait for a peer's flag passed 1 s)."""
        import ctypes
        word = ctypes.c_uint32()
        _lib.check(_lib.lib.ema_span_exchange_status(ctypes.c_void_p(self.ptrs[self.rank]), ctypes.byref(word),
                                                     int(clear)), "ema_span_exchange_status")
        return int(word.value)


def _p2p_exchange(direction: int, ld: torch.Tensor, V: torch.Tensor, boundary: Optional[torch.Tensor], group):
    """The span exchange in one kernel over NVLink peer memory (ema_span_exchange):
    the summary of this rank's sub-spans, the exchange, the fold of the spans
    before (direction 0) / after (direction 1) this one and its expansion over
    the sub-spans.  ld (B, K, H) float64, V (B K, H, P) fp32, ``boundary`` the
    sequence's initial state (direction 0) / final-state gradient (direction 1)
    or None.  Returns (span boundary value (B, H, P), per sub-span (B K, H, P))."""
    B, K, H = ld.shape
    P = V.shape[-1]
    ex = _P2PExchange.get(group, V.device, B * H, P)
    ld, V = ld.contiguous(), V.to(torch.float32).contiguous()
    bnd = None if boundary is None else boundary.to(torch.float32).contiguous()
    span_in = torch.empty(B, H, P, dtype=torch.float32, device=V.device)
    out = torch.empty(B * K, H, P, dtype=torch.float32, device=V.device)
    a = _lib.EmaSpanExchangeArgs()
    a.batch, a.subspans, a.nheads, a.headdim = B, K, H, P
    a.direction, a.rank, a.world = direction, ex.rank, ex.world
    a.log_decay, a.values = ld.data_ptr(), V.data_ptr()
    a.boundary = None if bnd is None else bnd.data_ptr()
    a.span_in, a.out = span_in.data_ptr(), out.data_ptr()
    a.buffer_bytes = ex.nbytes
    for q, ptr in enumerate(ex.ptrs):
        a.buffers[q] = ptr
    with torch.cuda.device(V.device):
        _lib.check(_lib.lib.ema_span_exchange(a, _lib.stream_ptr(V.device)), "ema_span_exchange")
    return span_in, out


def p2p_exchange_status(group=None, device=None, clear: bool = False) -> int:
    """OR of the status words of this process's p2p exchange buffers for
    ``group`` (0: every wait saw its peers' flags in time)."""
    st = 0
    for (gid, dev, _, _), ex in _P2PExchange._cache.items():
        if gid == id(group) and (device is None or dev == torch.device(device).index):
            st |= ex.status(clear)
    return st


def _peer(group, r):
    """Global rank of group rank ``r`` (send/recv address global ranks)."""
    return r if group is None else dist.get_global_rank(group, r)


def span_state(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, direction: int, log_decay: bool = False):
    """Per (row, head) of x (rows, L, H, P): direction 0, the row's end state from
    a zero start; direction 1 (x = dy), the gradient w.r.t. the row's start state
    from its own dy -- as weighted column sums (ema_span_state_launch), (rows, H, P)
    fp32.  headdim 32, 64 or 128.  With ``log_decay`` also the rows' log decays
    A_h sum dt, (rows, H) float64, from the same launch: returns (out, ld)."""
    rows, L, H, P = x.shape
    xk = _lib.tma_ready(x)
    dtk = dt.to(torch.float32).contiguous()
    Ak = A.to(torch.float32).contiguous()
    out = torch.empty(rows, H, P, dtype=torch.float32, device=x.device)
    ld = torch.empty(rows, H, dtype=torch.float64, device=x.device) if log_decay else None
    a = _lib.EmaSpanStateArgs()
    a.rows, a.seqlen, a.nheads, a.headdim = rows, L, H, P
    a.dtype, a.direction = _lib.DTYPE_CODES[x.dtype], direction
    a.x, a.x_stride = xk.data_ptr(), _lib.strides3(xk)
    a.dt, a.A, a.out = dtk.data_ptr(), Ak.data_ptr(), out.data_ptr()
    a.log_decay = ld.data_ptr() if ld is not None else None
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib.ema_span_state_launch(a, _lib.stream_ptr(x.device)), "ema_span_state")
    return (out, ld) if log_decay else out


_SPAN_STATE_P = (32, 64, 128)
_EXCHANGES = ("chain", "allgather", "p2p")


# The state callables of sp_forward / sp_backward return the sub-span rows'
# boundary values (B K, H, P), or (values, log decays (B K, H) float64) when the
# same launch gives the log decays.
def _kernel_state_fwd(x, dt, A, chunk_size):
    if x.shape[-1] in _SPAN_STATE_P:  # a reduction: no scan, no look-back
        return span_state(x, dt, A, 0, log_decay=True)
    return ema_chunk_scan_fwd(x, dt, A, chunk_size, state_only=True)[2]


def _kernel_fwd(x, dt, A, chunk_size, initial_states):
    # the autograd op's pair: 256-token forward tiles hand the backward 128-token chunk states
    return ema_chunk_scan_fwd(x, dt, A, chunk_size, initial_states=initial_states, return_final_states=True,
                              half_chunk_states=backward_chunk(chunk_size) != chunk_size)


def _kernel_state_bwd(x, dt, A, states, dy, chunk_size):
    if dy.shape[-1] in _SPAN_STATE_P:
        return span_state(dy if dy.dtype == x.dtype else dy.to(x.dtype), dt, A, 1, log_decay=True)
    return ema_chunk_scan_bwd(x, dt, A, states, dy, backward_chunk(chunk_size), state_only=True)[3]


def _kernel_bwd(x, dt, A, states, dy, chunk_size, d_final_states, need_d_initial):
    return ema_chunk_scan_bwd(x, dt, A, states, dy, backward_chunk(chunk_size), d_final_states=d_final_states,
                              need_d_initial=need_d_initial)


def _values_and_logs(r, dt_rows: torch.Tensor, A: torch.Tensor, B: int, K: int):
    """A state callable's result -> (values, log decays (B, K, H) float64)."""
    if isinstance(r, tuple):
        V, ld = r
        return V, ld.view(B, K, -1)
    return r, _log_decays(dt_rows, A, B, K)


def _kernel_fold(direction: int, expand: bool, ld: torch.Tensor, V: torch.Tensor,
                 boundary: Optional[torch.Tensor] = None):
    """The sub-span folds on the GPU (ema_span_summary / ema_span_expand).
    ld (B, K, H) float64, V (B K, H, P) float32.  Summary: (span value (B, H, P),
    span decay (B, H)); expansion (``boundary`` (B, H, P)): (B K, H, P)."""
    B, K, H = ld.shape
    P = V.shape[-1]
    ld, V = ld.contiguous(), V.to(torch.float32).contiguous()
    a = _lib.EmaSpanFoldArgs()
    a.batch, a.subspans, a.nheads, a.headdim, a.direction = B, K, H, P, direction
    a.log_decay, a.values = ld.data_ptr(), V.data_ptr()
    with torch.cuda.device(V.device):
        if expand:
            bnd = boundary.to(torch.float32).contiguous()
            out = torch.empty(B * K, H, P, dtype=torch.float32, device=V.device)
            a.boundary, a.out = bnd.data_ptr(), out.data_ptr()
            _lib.check(_lib.lib.ema_span_expand(a, _lib.stream_ptr(V.device)), "ema_span_expand")
            return out
        out = torch.empty(B, H, P, dtype=torch.float32, device=V.device)
        dspan = torch.empty(B, H, dtype=torch.float32, device=V.device)
        a.out, a.span_decay = out.data_ptr(), dspan.data_ptr()
        _lib.check(_lib.lib.ema_span_summary(a, _lib.stream_ptr(V.device)), "ema_span_summary")
        return out, dspan


def subspan_count(batch: int, nheads: int, span: int, chunk_size: int, ranks: int = 2) -> int:
    """Sub-spans a rank cuts its span into: the largest power of two K <= 64
    with span % K == 0 and, over several ranks, at least four chunks per
    sub-span and at most 2048 chains (batch * nheads * K) -- measured fastest at
    config 4: K = 32 / 16 / 8 over 2 / 4 / 8 ranks; on one GPU (``ranks`` 1,
    where the sub-spans only add parallelism) at least sixteen chunks per
    sub-span and at most 512 chains -- K = 16 at config 4 (383.6 against 462.7
    us for the whole sequence as 32 chains; 402 / 388 / 400 us at K = 8 / 32 /
    64).  K = 1 means the span runs whole."""
    min_chunks, max_chains = (16, 512) if ranks == 1 else (4, 2048)
    K = 1
    while (2 * K <= 64 and span % (2 * K) == 0 and span // (2 * K) >= min_chunks * chunk_size
           and batch * nheads * 2 * K <= max_chains):
        K *= 2
    return K


def _rows(t: torch.Tensor, K: int) -> torch.Tensor:
    """(B, L, ...) -> (B K, L / K, ...): sub-span k of batch row b becomes row b K + k."""
    B, L = t.shape[:2]
    return t.reshape(B * K, L // K, *t.shape[2:])


def _log_decays(dt_rows: torch.Tensor, A: torch.Tensor, B: int, K: int) -> torch.Tensor:
    """A_h * (sum of dt over each sub-span), (B, K, H) float64: the log of its
    decay.  The folds over sub-spans run in float64 on these few (B, K, H, P)
    values, so exponentials of long cumulative sums add no fp32 rounding."""
    return (dt_rows.sum(dim=1, dtype=torch.float64) * A.to(torch.float64)).view(B, K, -1)


def sp_forward(x, dt, A, chunk_size: int = 256, group=None, initial_states: Optional[torch.Tensor] = None,
               state_fwd: Callable = _kernel_state_fwd, local_fwd: Callable = _kernel_fwd,
               exchange: str = "chain", subspans: Optional[int] = None, fold: Callable = _kernel_fold):
    """Sequence-parallel forward of this rank's span.

    The span is cut into K sub-spans run as extra batch rows (``subspans``;
    default :func:`subspan_count`), so both passes -- the state-only pass and
    the full pass -- run on K times more, K times shorter chains.  The
    sub-spans' end states from zero and decays fold (in log space, float64,
    ``fold``: the ema_span_summary / ema_span_expand kernels) into the span's
    summary for the exchange, and the state entering the span into each
    sub-span's incoming state for the full pass.

    Returns (y, chunk_start_states, Sin, final): y in x's layout;
    ``chunk_start_states`` of the sub-span rows (B K, nchunks, H, P), what
    :func:`sp_backward` takes; ``Sin`` the state entering this span; ``final``
    this span's end state (the sequence's final state on the last rank).
    ``exchange``: "chain" (NCCL send/recv r -> r+1), "allgather" (one
    all_gather of the span summaries) or "p2p" (summary, exchange, fold and
    expansion in one kernel over NVLink peer memory, ema_span_exchange; every
    rank on its own GPU, headdim <= 128)."""
    assert exchange in _EXCHANGES, "exchange must be 'chain', 'allgather' or 'p2p'"
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    B, Ls, H, P = x.shape
    K = subspans if subspans is not None else subspan_count(B, H, Ls, chunk_size, world)
    if world == 1 and K == 1:  # one span, whole: no state-only pass
        init = None if initial_states is None else initial_states.to(torch.float32)
        Sin = init if init is not None else torch.zeros(B, H, P, dtype=torch.float32, device=x.device)
        y, states, final = local_fwd(x, dt, A, chunk_size, Sin)
        return y, states, Sin, final
    assert Ls % K == 0, "the span length must be a multiple of the sub-span count"
    xr, dtr = _rows(x, K), _rows(dt, K)
    # sub-span summaries (end states from zero, log decays) -> the span's end state from zero, its decay
    S, ld = _values_and_logs(state_fwd(xr, dtr, A, chunk_size), dtr, A, B, K)
    init = None
    if world == 1:  # one span cut into sub-spans: nothing to exchange
        Sin = (initial_states.to(torch.float32).clone() if initial_states is not None
               else torch.zeros(B, H, P, dtype=torch.float32, device=x.device))
    elif exchange == "p2p":  # summary, exchange, fold and expansion in one kernel
        Sin, init = _p2p_exchange(0, ld, S, initial_states if rank == 0 else None, group)
    elif exchange == "allgather":
        S_loc, D = fold(0, False, ld, S)
        if rank == 0 and initial_states is not None:  # rank 0's summary includes the initial state
            S_loc = D[..., None] * initial_states.to(torch.float32) + S_loc
        Ss, Ds = _gather(S_loc, D, group)
        if rank == 0:
            Sin = (initial_states.to(torch.float32).clone() if initial_states is not None
                   else torch.zeros(B, H, P, dtype=torch.float32, device=x.device))
        else:  # the spans before this one, folded in order
            Sin = _fold(Ss[:rank], Ds[:rank])
    else:
        S_loc, D = fold(0, False, ld, S)
        if rank == 0:
            Sin = (initial_states.to(torch.float32).clone() if initial_states is not None
                   else torch.zeros(B, H, P, dtype=torch.float32, device=x.device))
        else:
            Sin = torch.empty(B, H, P, dtype=torch.float32, device=x.device)
            dist.recv(Sin, src=_peer(group, rank - 1), group=group)
        if rank + 1 < world:
            Sout = D[..., None] * Sin + S_loc
            dist.send(Sout.to(torch.float32).contiguous(), dst=_peer(group, rank + 1), group=group)
    # the state entering every sub-span, from the state entering the span
    if init is None:
        init = fold(0, True, ld, S, Sin)
    y, states, final = local_fwd(xr, dtr, A, chunk_size, init)
    return y.reshape(B, Ls, H, P), states, Sin, final.reshape(B, K, H, P)[:, -1]


def sp_backward(x, dt, A, states, dy, chunk_size: int = 256, group=None,
                d_final_states: Optional[torch.Tensor] = None, need_d_initial: bool = False,
                state_bwd: Callable = _kernel_state_bwd, local_bwd: Callable = _kernel_bwd,
                exchange: str = "chain", fold: Callable = _kernel_fold):
    """Sequence-parallel backward of this rank's span.

    ``states`` are the sub-span rows' chunk start states from
    :func:`sp_forward` (which started every sub-span from its true incoming
    state); the sub-span count is read off their shape.  Returns (dx, ddt, dA,
    d_initial): dx and ddt in x's and dt's layouts; dA summed over the group;
    d_initial (rank 0, when asked) the gradient w.r.t. the sequence's initial
    state.  ``exchange`` as in :func:`sp_forward`, running r+1 -> r."""
    assert exchange in _EXCHANGES, "exchange must be 'chain', 'allgather' or 'p2p'"
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    B, Ls, H, P = x.shape
    if world == 1 and states.shape[0] == B:  # one span, whole
        Gin = (d_final_states.to(torch.float32).clone() if d_final_states is not None
               else torch.zeros(B, H, P, dtype=torch.float32, device=x.device))
        dx, ddt, dA, d_init = local_bwd(x, dt, A, states, dy, chunk_size, Gin, need_d_initial)
        return dx, ddt, dA.to(torch.float32).contiguous(), d_init
    K = states.shape[0] // B
    xr, dtr, dyr = _rows(x, K), _rows(dt, K), _rows(dy, K)
    # sub-span summaries (start gradients from their own dy, nothing arriving) -> the span's
    G, ld = _values_and_logs(state_bwd(xr, dtr, A, states, dyr, chunk_size), dtr, A, B, K)
    dfin = None
    if world == 1:  # one span cut into sub-spans: nothing to exchange
        Gin = (d_final_states.to(torch.float32).clone() if d_final_states is not None
               else torch.zeros(B, H, P, dtype=torch.float32, device=x.device))
    elif exchange == "p2p":  # summary, exchange, fold and expansion in one kernel
        Gin, dfin = _p2p_exchange(1, ld, G, d_final_states if rank == world - 1 else None, group)
    elif exchange == "allgather":
        G_loc, D = fold(1, False, ld, G)
        if rank == world - 1 and d_final_states is not None:  # the last summary includes the final gradient
            G_loc = D[..., None] * d_final_states.to(torch.float32) + G_loc
        Gs, Ds = _gather(G_loc, D, group)
        if rank == world - 1:
            Gin = (d_final_states.to(torch.float32).clone() if d_final_states is not None
                   else torch.zeros(B, H, P, dtype=torch.float32, device=x.device))
        else:  # the spans after this one, folded from the last backwards
            Gin = _fold(Gs[rank + 1:].flip(0), Ds[rank + 1:].flip(0))
    else:
        G_loc, D = fold(1, False, ld, G)
        if rank == world - 1:
            Gin = (d_final_states.to(torch.float32).clone() if d_final_states is not None
                   else torch.zeros(B, H, P, dtype=torch.float32, device=x.device))
        else:
            Gin = torch.empty(B, H, P, dtype=torch.float32, device=x.device)
            dist.recv(Gin, src=_peer(group, rank + 1), group=group)
        if rank > 0:
            Gout = D[..., None] * Gin + G_loc
            dist.send(Gout.to(torch.float32).contiguous(), dst=_peer(group, rank - 1), group=group)
    # the gradient arriving at every sub-span's end, from the one arriving at the span's end
    if dfin is None:
        dfin = fold(1, True, ld, G, Gin)
    dx, ddt, dA, d_init = local_bwd(xr, dtr, A, states, dyr, chunk_size, dfin, need_d_initial and rank == 0)
    dA = dA.to(torch.float32).contiguous()
    if world > 1:
        dist.all_reduce(dA, group=group)
    if d_init is not None:
        d_init = d_init.reshape(B, K, H, P)[:, 0]
    return dx.reshape(B, Ls, H, P), ddt.reshape(B, Ls, H), dA, d_init


class _EmaChunkScanSPFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dt, A, chunk_size, group, exchange):
        y, states, _, _ = sp_forward(x, dt, A, chunk_size, group, exchange=exchange)
        ctx.save_for_backward(x, dt, A, states)
        ctx.chunk_size, ctx.group, ctx.exchange = chunk_size, group, exchange
        ctx.dt_dtype, ctx.A_dtype = dt.dtype, A.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        x, dt, A, states = ctx.saved_tensors
        dx, ddt, dA, _ = sp_backward(x, dt, A, states, dy.contiguous(), ctx.chunk_size, ctx.group,
                                     exchange=ctx.exchange)
        return dx, ddt.to(ctx.dt_dtype), dA.to(ctx.A_dtype), None, None, None


def ema_chunk_scan_sp(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, chunk_size: int = 256, group=None,
                      exchange: str = "chain"):
    """Autograd op over this rank's span of a sequence split across ``group``;
    ``exchange``: "chain" (NCCL send/recv between neighbours), "allgather" or
    "p2p" (one kernel over NVLink peer memory)."""
    return _EmaChunkScanSPFn.apply(x, dt, A, chunk_size, group, exchange)
