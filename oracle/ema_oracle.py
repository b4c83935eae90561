"""float64 numpy oracle for the EMA chunked scan (TEST INFRASTRUCTURE ONLY).

Restates, from the equations, what the reference's EMA path computes:

* ``ema_fwd``        -- ``ema_fwd_triton`` / ``ema_fwd_kernel``
                        (kernels/forward/ema_ssd_fwd.py:236-398, 413-516):
                        ``Z[t] = exp2(dA[t]) * Z[t-1] + X[t]`` per (batch, head),
                        plus the per-chunk START states (stored before the chunk
                        update, ema_ssd_fwd.py:378-382), the within-chunk
                        inclusive cumsum of dA (:328-333) and the per-chunk dA
                        totals (:329, :397-398).  ``seq_idx`` resets the state
                        where the id changes from the previous token, the rule of
                        the reference's own oracle ``ema_torch_ref_seq_idx``
                        (ema_ssd_fwd.py:562-594).
* ``ema_bwd``        -- ``compute_dpx`` / ``ema_ssd_bwd_kernel_dpx``
                        (kernels/backward/ema_ssd_combined.py:48-169,
                        kernels/backward/ema_ssd_bwd.py:38-295).  Returns dX,
                        the per-token gradient with respect to the NATURAL-log
                        decay (the kernel applies no ln2 factor, and
                        ``_EmaFunction.backward`` returns its head-sum as dL/dA
                        for ``A = ln(decay)``, ema_ssd_combined.py:205-225), and
                        optionally the initial-state gradient.  ``d_ossm_state``
                        seeds the reverse state gradient (ema_ssd_bwd.py:111-117);
                        ``d_ox_state`` is added to dX at the last token
                        (ema_ssd_combined.py:165-167).
* ``chunk_cumsum``   -- ``chunk_cumsum_triton`` (ema_ssd_fwd.py:109-212): the
                        inclusive within-chunk cumsum and the EXCLUSIVE reverse
                        within-chunk cumsum (``rev[t] = sum_{k>t in chunk} dA[k]``,
                        0 at the chunk's last token), optionally exponentiated.
* ``ema_dt_fwd`` / ``ema_dt_bwd`` -- the dt-parameterised EMA of the benchmark
                        configs: ``h_t = exp(dt_t*A_h) h_{t-1} + dt_t x_t``,
                        ``y_t = h_t``; i.e. the reference EMA with
                        ``X = dt*x`` and ``dA = dt*A*log2(e)``.

All arithmetic is float64; inputs of any float dtype are promoted.
"""

from __future__ import annotations

import math

import numpy as np

LOG2E = 1.0 / math.log(2.0)


def _f64(a):
    if a is None:
        return None
    if hasattr(a, "detach"):  # torch tensor without importing torch here
        a = a.detach().cpu().double().numpy()
    return np.asarray(a, dtype=np.float64)


def _resets(seq_idx, batch, seqlen):
    """Boolean (B, L): True where the state restarts (id differs from the previous token)."""
    if seq_idx is None:
        return None
    s = np.asarray(seq_idx.detach().cpu().numpy() if hasattr(seq_idx, "detach") else seq_idx)
    r = np.zeros((batch, seqlen), dtype=bool)
    r[:, 1:] = s[:, 1:] != s[:, :-1]
    return r


def scan_forward(u, a, z0=None, resets=None):
    """Sequential ``z_t = a_t z_{t-1} + u_t``.

    u: (B, L, H, P); a: (B, L, H); z0: (B, H, P) or None; resets: (B, L) bool.
    Returns (z (B,L,H,P), zprev (B,L,H,P), final (B,H,P)); zprev[:, t] is the
    carried state z_{t-1} before any restart at t (a restart acts as a_t = 0).
    """
    B, L, H, P = u.shape
    z = np.zeros((B, H, P)) if z0 is None else z0.copy()
    out = np.empty_like(u)
    prev = np.empty_like(u)
    for t in range(L):
        prev[:, t] = z
        at = a[:, t, :, None]
        if resets is not None and t > 0:
            at = at * (~resets[:, t])[:, None, None]
        z = at * z + u[:, t]
        out[:, t] = z
    return out, prev, z


def scan_reverse(dz, a, gseed=None, resets=None):
    """Adjoint of :func:`scan_forward`.

    Returns (G (B,L,H,P) = dLoss/dz_t including all later paths,
             d_z0 (B,H,P) = dLoss/dz0).
    """
    B, L, H, P = dz.shape
    g = np.zeros((B, H, P)) if gseed is None else gseed.copy()  # grad wrt z_t from t+1..
    G = np.empty_like(dz)
    for t in range(L - 1, -1, -1):
        g = dz[:, t] + g
        G[:, t] = g
        g = a[:, t, :, None] * g  # grad wrt z_{t-1}
        if resets is not None and t > 0:
            g = g * (~resets[:, t])[:, None, None]
    return G, g


# --------------------------------------------------------------------------
# Reference-form EMA (log2 decay dA of shape (B, H, L))
# --------------------------------------------------------------------------

def ema_fwd(x, dA, chunk_size=64, seq_idx=None, initial_state=None):
    """Forward of the reference EMA.

    x: (B, L, H, P); dA: (B, H, L) log2 decay.
    Returns dict with ``out`` (B,L,H,P), ``states`` (B,nc,H,1,P) chunk START
    states, ``da_cs`` (B,H,L), ``da_cs_sum`` (B,H,nc), ``final_state`` (B,H,P).
    """
    x = _f64(x)
    dA = _f64(dA)
    B, L, H, P = x.shape
    Q = int(chunk_size)
    nc = -(-L // Q)
    a = np.exp2(dA).transpose(0, 2, 1)  # (B, L, H)
    z0 = _f64(initial_state)
    resets = _resets(seq_idx, B, L)
    y, prev, final = scan_forward(x, a, z0, resets)
    states = np.zeros((B, nc, H, 1, P))
    for c in range(nc):
        states[:, c, :, 0, :] = prev[:, c * Q]  # state before the chunk's first token
    # with seq_idx the stored start state is the carried state before any
    # restart at the chunk's first token (what the reference kernel stores,
    # ema_ssd_fwd.py:379-382, for chunk-aligned segments)
    da_cs = np.empty((B, H, L))
    da_cs_sum = np.empty((B, H, nc))
    for c in range(nc):
        s, e = c * Q, min(L, (c + 1) * Q)
        da_cs[:, :, s:e] = np.cumsum(dA[:, :, s:e], axis=-1)
        da_cs_sum[:, :, c] = dA[:, :, s:e].sum(-1)
    return {"out": y, "states": states, "da_cs": da_cs, "da_cs_sum": da_cs_sum,
            "final_state": final}


def ema_bwd(x, da_cs, da_cs_sum, ssm_states, do, d_ossm_state=None, d_ox_state=None,
            chunk_size=64, has_input_state=False):
    """Backward of the reference EMA, with ``compute_dpx``'s inputs.

    ssm_states: (B, H, P, nc) chunk START states (the forward's ``states``
    permuted, ema_ssd_combined.py:198).  Within chunk c the decay of token t is
    ``exp2(da_cs[t] - da_cs[t-1])`` (``exp2(da_cs[t0])`` at the chunk's first
    token); the decay across the whole chunk is ``exp2(da_cs_sum[c])``.  The
    forward states inside a chunk are recomputed from ``ssm_states[..., c]``.

    Returns dict ``dx`` (B,L,H,P), ``dA`` (B,H,L) = dLoss/d(ln decay),
    ``d_issm_state`` (B,H,P,1) or None.
    """
    x = _f64(x)
    cs = _f64(da_cs)
    tot = _f64(da_cs_sum)
    S = _f64(ssm_states)
    do = _f64(do)
    B, L, H, P = x.shape
    Q = int(chunk_size)
    nc = -(-L // Q)
    dx = np.empty_like(x)
    dl = np.empty((B, H, L))
    dS = np.zeros((B, H, P)) if d_ossm_state is None else _f64(d_ossm_state).copy()
    for c in range(nc - 1, -1, -1):
        s, e = c * Q, min(L, (c + 1) * Q)
        csc = cs[:, :, s:e].transpose(0, 2, 1)  # (B, n, H)
        a = np.exp2(np.diff(np.concatenate([np.zeros((B, 1, H)), csc], axis=1), axis=1))
        # forward recompute inside the chunk from its start state
        _, prev, _ = scan_forward(x[:, s:e], a, S[..., c])
        # reverse: gradient wrt the chunk-end state is dS; chunk decay uses da_cs_sum
        G = np.empty((B, e - s, H, P))
        g = dS * np.exp2(tot[:, :, c] - csc[:, -1, :])[:, :, None]
        for t in range(e - s - 1, -1, -1):
            g = do[:, s + t] + g
            G[:, t] = g
            g = a[:, t, :, None] * g
        dx[:, s:e] = G
        dl[:, :, s:e] = np.einsum("bthp,bthp->bht", G, a[..., None] * prev)
        # gradient wrt the previous chunk's end state (ema_ssd_bwd.py:283-289 form)
        dS = np.exp2(tot[:, :, c])[:, :, None] * dS + np.einsum(
            "bth,bthp->bhp", np.exp2(csc), do[:, s:e])
    if d_ox_state is not None:
        dx[:, -1] += _f64(d_ox_state)
    d_issm = dS[..., None] if has_input_state else None
    return {"dx": dx, "dA": dl, "d_issm_state": d_issm}


def ema_combined_grads(x, A, dout, chunk_size=64):
    """``ema_combined`` forward + autograd backward (ema_ssd_combined.py:172-229).

    A: (B, L) natural-log decay shared by all heads.  Returns dict ``out``,
    ``dx`` (B,L,H,P), ``dA`` (B,L) (per-head gradients summed over heads).
    """
    x = _f64(x)
    A = _f64(A)
    B, L, H, P = x.shape
    dA = np.repeat((A * LOG2E)[:, None, :], H, axis=1)
    f = ema_fwd(x, dA, chunk_size)
    states = f["states"][:, :, :, 0, :].transpose(0, 2, 3, 1)
    b = ema_bwd(x, f["da_cs"], f["da_cs_sum"], states, dout, chunk_size=chunk_size)
    return {"out": f["out"], "dx": b["dx"], "dA": b["dA"].sum(1)}


def chunk_cumsum(dA, chunk_size=64, exp2=False):
    """``chunk_cumsum_triton``: (inclusive cumsum, exclusive reverse cumsum) per chunk."""
    dA = _f64(dA)
    B, H, L = dA.shape
    Q = int(chunk_size)
    fwd = np.empty_like(dA)
    rev = np.empty_like(dA)
    for s in range(0, L, Q):
        e = min(L, s + Q)
        blk = dA[..., s:e]
        fwd[..., s:e] = np.cumsum(blk, -1)
        inc_rev = np.cumsum(blk[..., ::-1], -1)[..., ::-1]
        rev[..., s:e - 1] = inc_rev[..., 1:]
        rev[..., e - 1] = 0.0
    if exp2:
        fwd = np.exp2(fwd)
        rev = np.exp2(rev)
    return fwd, rev


# --------------------------------------------------------------------------
# dt-parameterised EMA (benchmark configs 1, 2, 4)
# --------------------------------------------------------------------------

def ema_dt_fwd(x, dt, A, initial_state=None):
    """x (B,L,H,P), dt (B,L,H), A (H,).  Returns dict ``y``, ``final_state``."""
    x, dt, A = _f64(x), _f64(dt), _f64(A)
    a = np.exp(dt * A[None, None, :])
    u = dt[..., None] * x
    y, _, final = scan_forward(u, a, _f64(initial_state))
    return {"y": y, "final_state": final}


def ema_dt_bwd(x, dt, A, dy, initial_state=None, d_final_state=None):
    """Gradients of the dt-form EMA.

    Returns dict ``dx``, ``ddt`` (B,L,H), ``dA`` (H,), ``d_initial_state`` (B,H,P),
    and ``dl`` (B,L,H) = dLoss/d(ln decay) per token.
    """
    x, dt, A, dy = _f64(x), _f64(dt), _f64(A), _f64(dy)
    a = np.exp(dt * A[None, None, :])
    u = dt[..., None] * x
    _, prev, _ = scan_forward(u, a, _f64(initial_state))
    G, dz0 = scan_reverse(dy, a, _f64(d_final_state))
    dl = np.einsum("blhp,blhp->blh", G, a[..., None] * prev)
    ddt = np.einsum("blhp,blhp->blh", G, x) + A[None, None, :] * dl
    dA = np.einsum("blh,blh->h", dt, dl)
    return {"dx": dt[..., None] * G, "ddt": ddt, "dA": dA, "d_initial_state": dz0, "dl": dl}


# --------------------------------------------------------------------------
# Seeded synthetic inputs for the benchmark configs
# --------------------------------------------------------------------------

def make_dt_inputs(batch, seqlen, nheads, headdim, seed=0, dt_range=(1e-3, 1e-1),
                   a_log_range=(0.0, math.log(16.0))):
    """Config-2 style inputs: x ~ N(0,1); dt = softplus(N(0,1) + b_h) clamped to
    ``dt_range`` with per-head bias b_h placing dt inside it; A = -exp(U(a_log_range)).
    Returns float32 numpy arrays (x, dt, A, dy)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((batch, seqlen, nheads, headdim), dtype=np.float32)
    lo, hi = dt_range
    target = np.exp(rng.uniform(math.log(lo), math.log(hi), size=nheads))
    bias = np.log(np.expm1(target))  # softplus^-1(target)
    pre = rng.standard_normal((batch, seqlen, nheads)).astype(np.float64) + bias
    dt = np.clip(np.logaddexp(0.0, pre), lo, hi).astype(np.float32)
    A = (-np.exp(rng.uniform(a_log_range[0], a_log_range[1], size=nheads))).astype(np.float32)
    dy = rng.standard_normal((batch, seqlen, nheads, headdim), dtype=np.float32)
    return x, dt, A, dy
