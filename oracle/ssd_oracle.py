"""Float64 CPU oracle for the Mamba-2 SSD scan (benchmark configs 3 and 5).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU legs of bench.py, never by the product path.

Parity status: pinned through the d_state-1 reduction, otherwise unpinned.
The reference does not implement SSD itself; its benchmark calls the
third-party ``mamba_ssm`` package
(``mamba_ssm.ops.triton.ssd_combined.mamba_chunk_scan_combined``, imported at
kernels/benchmarks/bench_ema_total.py:18 and called at :72-76 as
``(x, dt, A, B, C, chunk_size, seq_idx=None)``), which has no pinned version
and is not present here.  This file restates the published Mamba-2 SSD
recurrence (state-space duality; per head h of group g = h // (H / G)):

    s_t = exp(dt_t A_h) s_{t-1} + dt_t x_t B_t^T        (headdim x d_state)
    y_t = s_t C_t + D_h x_t

with x (batch, seqlen, nheads, headdim), dt (batch, seqlen, nheads) already
positive (no bias / softplus), A (nheads,), B and C (batch, seqlen, ngroups,
d_state), D (nheads,) and states (batch, nheads, headdim, d_state) -- the
layouts of ``mamba_chunk_scan_combined``.  The backward is the exact adjoint
of the recurrence (back-propagation through the sequence), cross-checked in
tests/test_ssd_oracle.py against torch autograd of the same recurrence and
against finite differences.  With d_state 1, A = -1, dt = -ln(2) dA, B = 1 / dt
(one group per head) and C = 1 the recurrence is the reference's own EMA
(kernels/forward/ema_ssd_fwd.py:258-259), so tests/test_ssd_oracle_pinned.py
checks this file, forward and backward, sequential and chunked, against the
golden vectors of the reference's kernels; the d_state > 1 contractions and
dB / dC are beyond that reduction.
"""

from __future__ import annotations

import numpy as np


def _f64(a):
    return np.asarray(a, dtype=np.float64)


def ssd_fwd(x, dt, A, B, C, D=None, initial_state=None):
    """Sequential recurrence.  Returns {"y", "final_state", "states"} where
    ``states[:, t]`` is the state after token t (batch, seqlen, nheads, P, N)."""
    x, dt, A, B, C = (_f64(a) for a in (x, dt, A, B, C))
    b_, L, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    hpg = H // G
    Bh = np.repeat(B, hpg, axis=2)  # (b, L, H, N)
    Ch = np.repeat(C, hpg, axis=2)
    s = np.zeros((b_, H, P, N)) if initial_state is None else _f64(initial_state).copy()
    y = np.empty((b_, L, H, P))
    states = np.empty((b_, L, H, P, N))
    for t in range(L):
        a = np.exp(dt[:, t] * A)[:, :, None, None]  # (b, H, 1, 1)
        s = a * s + (dt[:, t, :, None, None] * x[:, t, :, :, None]) * Bh[:, t, :, None, :]
        states[:, t] = s
        y[:, t] = np.einsum("bhpn,bhn->bhp", s, Ch[:, t])
    if D is not None:
        y = y + _f64(D)[None, None, :, None] * x
    return {"y": y, "final_state": s, "states": states}


def ssd_bwd(x, dt, A, B, C, dy, D=None, initial_state=None, d_final_state=None):
    """Adjoint of ssd_fwd.  Returns {"dx", "ddt", "dA", "dB", "dC", "dD",
    "d_initial_state"}; dB / dC are summed over the heads of each group."""
    x, dt, A, B, C, dy = (_f64(a) for a in (x, dt, A, B, C, dy))
    b_, L, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    hpg = H // G
    Bh = np.repeat(B, hpg, axis=2)
    Ch = np.repeat(C, hpg, axis=2)
    f = ssd_fwd(x, dt, A, B, C, None, initial_state)
    S = f["states"]
    s0 = np.zeros((b_, H, P, N)) if initial_state is None else _f64(initial_state)
    g = np.zeros((b_, H, P, N)) if d_final_state is None else _f64(d_final_state).copy()
    dx = np.empty_like(x)
    ddt = np.empty_like(dt)
    dA = np.zeros(H)
    dBh = np.empty((b_, L, H, N))
    dCh = np.empty((b_, L, H, N))
    for t in range(L - 1, -1, -1):
        s_prev = S[:, t - 1] if t > 0 else s0
        # y_t = s_t C_t: gradient into s_t and C_t
        g = g + dy[:, t, :, :, None] * Ch[:, t, :, None, :]
        dCh[:, t] = np.einsum("bhpn,bhp->bhn", S[:, t], dy[:, t])
        a = np.exp(dt[:, t] * A)  # (b, H)
        # s_t = a s_{t-1} + dt x B^T
        gs = np.einsum("bhpn,bhpn->bh", g, s_prev)  # d/da . s_prev
        gxb = np.einsum("bhpn,bhp,bhn->bh", g, x[:, t], Bh[:, t])
        ddt[:, t] = gs * a * A + gxb
        dA += np.einsum("bh,bh->h", gs * a, dt[:, t])
        dx[:, t] = dt[:, t, :, None] * np.einsum("bhpn,bhn->bhp", g, Bh[:, t])
        dBh[:, t] = dt[:, t, :, None] * np.einsum("bhpn,bhp->bhn", g, x[:, t])
        g = a[:, :, None, None] * g
    dD = None
    if D is not None:
        dx = dx + _f64(D)[None, None, :, None] * dy
        dD = np.einsum("blhp,blhp->h", dy, x)
    dB = dBh.reshape(b_, L, G, hpg, N).sum(3)
    dC = dCh.reshape(b_, L, G, hpg, N).sum(3)
    return {"dx": dx, "ddt": ddt, "dA": dA, "dB": dB, "dC": dC, "dD": dD, "d_initial_state": g}


def ssd_chunked_fwd(x, dt, A, B, C, chunk_size, D=None, initial_state=None):
    """Chunked restatement (chunk_cumsum -> chunk_state -> state_passing ->
    chunk_scan) of ssd_fwd, for shapes where the sequential loop is slow;
    cross-checked against ssd_fwd in tests.  Returns {"y", "final_state",
    "chunk_states"} with chunk_states[:, c] the state entering chunk c."""
    x, dt, A, B, C = (_f64(a) for a in (x, dt, A, B, C))
    b_, L, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    hpg = H // G
    Q = chunk_size
    nc = -(-L // Q)
    s = np.zeros((b_, H, P, N)) if initial_state is None else _f64(initial_state).copy()
    y = np.empty((b_, L, H, P))
    chunk_states = np.empty((b_, nc, H, P, N))
    grp = np.arange(H) // hpg
    for c in range(nc):
        t0, t1 = c * Q, min(L, (c + 1) * Q)
        q = t1 - t0
        xc = np.ascontiguousarray(x[:, t0:t1].transpose(0, 2, 1, 3))   # (b, H, q, P)
        w = np.ascontiguousarray(dt[:, t0:t1].transpose(0, 2, 1))       # (b, H, q)
        Bg = np.ascontiguousarray(B[:, t0:t1].transpose(0, 2, 1, 3))    # (b, G, q, N)
        Cg = np.ascontiguousarray(C[:, t0:t1].transpose(0, 2, 1, 3))
        Bc, Cc = Bg[:, grp], Cg[:, grp]
        cs = np.cumsum(w * A[None, :, None], axis=2)  # natural-log decay from the chunk start
        chunk_states[:, c] = s
        # intra-chunk: y_i += sum_{j<=i} (C_i . B_j) exp(cs_i - cs_j) dt_j x_j
        CB = (Cg @ Bg.transpose(0, 1, 3, 2))[:, grp]                     # (b, H, i, j)
        mask = np.tril(np.ones((q, q), dtype=bool))
        E = np.where(mask, np.exp(np.where(mask, cs[:, :, :, None] - cs[:, :, None, :], 0.0)), 0.0)
        yc = (CB * E) @ (w[..., None] * xc)
        # inter-chunk: y_i += exp(cs_i) s C_i
        yc += np.exp(cs)[..., None] * (Cc @ s.transpose(0, 1, 3, 2))
        y[:, t0:t1] = yc.transpose(0, 2, 1, 3)
        # state passing
        wt = np.exp(cs[:, :, -1:] - cs) * w                              # (b, H, q)
        s = np.exp(cs[:, :, -1])[:, :, None, None] * s + (wt[..., None] * xc).transpose(0, 1, 3, 2) @ Bc
    if D is not None:
        y = y + _f64(D)[None, None, :, None] * x
    return {"y": y, "final_state": s, "chunk_states": chunk_states}


def ssd_chunked_bwd(x, dt, A, B, C, dy, chunk_size, D=None, initial_state=None, d_final_state=None):
    """Chunked restatement of ssd_bwd (the adjoint of ssd_chunked_fwd, chunk by
    chunk in reverse): memory grows with one chunk, not with the sequence, so a
    whole batch row of the benchmark shapes (config 3: L4096 H64; config 5:
    L8192 H80) fits.  Cross-checked against ssd_bwd in tests.  Same outputs as
    ssd_bwd.

    Per chunk with ``cs`` the within-chunk cumsum of ``dt A`` (natural log),
    ``E_ij = exp(cs_i - cs_j)`` for ``j <= i``, ``Xw_j = dt_j x_j`` and ``g`` the
    gradient of the state leaving the chunk:

        dXw_j = sum_i (C_i.B_j) E_ij dy_i + exp(cs_e - cs_j) g B_j
        dC_i  = sum_j (dy_i.Xw_j) E_ij B_j + exp(cs_i) s_in^T dy_i
        dB_j  = sum_i (dy_i.Xw_j) E_ij C_i + exp(cs_e - cs_j) g^T Xw_j
        g_in  = sum_i exp(cs_i) dy_i C_i^T + exp(cs_e) g

    and the gradient of every ``cs_k`` collected from each exponential it sits
    in, reverse-cumsummed into the per-token log-decay gradient ``dl``;
    ``ddt = x.dXw + A dl`` and ``dA = sum dt dl``."""
    x, dt, A, B, C, dy = (_f64(a) for a in (x, dt, A, B, C, dy))
    b_, L, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    hpg = H // G
    Q = chunk_size
    nc = -(-L // Q)
    f = ssd_chunked_fwd(x, dt, A, B, C, Q, None, initial_state)
    S = f["chunk_states"]  # (b, nc, H, P, N): state entering each chunk
    g = np.zeros((b_, H, P, N)) if d_final_state is None else _f64(d_final_state).copy()
    dx = np.empty_like(x)
    ddt = np.empty_like(dt)
    dA = np.zeros(H)
    dB = np.empty((b_, L, G, N))
    dC = np.empty((b_, L, G, N))
    grp = np.arange(H) // hpg
    for c in range(nc - 1, -1, -1):
        t0, t1 = c * Q, min(L, (c + 1) * Q)
        q = t1 - t0
        # per (b, h) matrices, tokens in the last-but-one axis; B and C per group
        # (shared by the group's heads: their products are formed once)
        xc = np.ascontiguousarray(x[:, t0:t1].transpose(0, 2, 1, 3))     # (b, H, q, P)
        dyc = np.ascontiguousarray(dy[:, t0:t1].transpose(0, 2, 1, 3))
        w = np.ascontiguousarray(dt[:, t0:t1].transpose(0, 2, 1))         # (b, H, q)
        Bg = np.ascontiguousarray(B[:, t0:t1].transpose(0, 2, 1, 3))      # (b, G, q, N)
        Cg = np.ascontiguousarray(C[:, t0:t1].transpose(0, 2, 1, 3))
        Bc, Cc = Bg[:, grp], Cg[:, grp]                                    # (b, H, q, N)
        s_in = S[:, c]                                                     # (b, H, P, N)
        cs = np.cumsum(w * A[None, :, None], axis=2)                       # (b, H, q)
        cse = cs[:, :, -1:]                                                # (b, H, 1)
        mask = np.tril(np.ones((q, q), dtype=bool))
        E = np.where(mask, np.exp(np.where(mask, cs[:, :, :, None] - cs[:, :, None, :], 0.0)), 0.0)
        Xw = w[..., None] * xc
        CB = (Cg @ Bg.transpose(0, 1, 3, 2))[:, grp]                       # (b, H, i, j)
        GX = dyc @ Xw.transpose(0, 1, 3, 2)                                # dy_i . Xw_j
        M = CB * E
        dcb = GX * E                                                       # gradient of (C_i . B_j)
        tail = np.exp(cse - cs)                                            # exp(cs_e - cs_j)
        gB = Bc @ g.transpose(0, 1, 3, 2)                                  # (g B_j)[p] as (b, H, q, P)
        dXw = M.transpose(0, 1, 3, 2) @ dyc + tail[..., None] * gB
        dxc = w[..., None] * dXw
        dw = (xc * dXw).sum(-1)
        # dC_i = sum over the group's heads of (dcb B)_i + exp(cs_i) s_in^T dy_i; dB likewise
        dcb_g = dcb.reshape(b_, G, hpg, q, q).sum(2)
        dCc = dcb_g @ Bg + (np.exp(cs)[..., None] * (dyc @ s_in)).reshape(b_, G, hpg, q, N).sum(2)
        dBc = dcb_g.transpose(0, 1, 3, 2) @ Cg + (tail[..., None] * (Xw @ g)).reshape(b_, G, hpg, q, N).sum(2)
        # gradient of each within-chunk cumsum entry
        T = GX * M                                                         # d/dE_ij * E_ij
        dcs = T.sum(3) - T.sum(2)
        yin = Cc @ s_in.transpose(0, 1, 3, 2)                              # (s_in C_i)[p] as (b, H, q, P)
        dcs += np.exp(cs) * (dyc * yin).sum(-1)
        U = tail * (Xw * gB).sum(-1)                                       # exp(cs_e - cs_j) <g, Xw_j B_j^T>
        dcs -= U
        dcs[:, :, -1] += U.sum(-1) + np.exp(cse[:, :, 0]) * (g * s_in).sum((-1, -2))
        dl = np.cumsum(dcs[:, :, ::-1], axis=2)[:, :, ::-1]
        dx[:, t0:t1] = dxc.transpose(0, 2, 1, 3)
        ddt[:, t0:t1] = (dw + A[None, :, None] * dl).transpose(0, 2, 1)
        dA += (w * dl).sum((0, 2))
        dB[:, t0:t1] = dBc.transpose(0, 2, 1, 3)
        dC[:, t0:t1] = dCc.transpose(0, 2, 1, 3)
        g = (np.exp(cs)[..., None] * dyc).transpose(0, 1, 3, 2) @ Cc + np.exp(cse)[..., None] * g
    dD = None
    if D is not None:
        dx = dx + _f64(D)[None, None, :, None] * dy
        dD = np.einsum("blhp,blhp->h", dy, x)
    return {"dx": dx, "ddt": ddt, "dA": dA, "dB": dB, "dC": dC, "dD": dD, "d_initial_state": g}


def make_ssd_inputs(batch, seqlen, nheads, headdim, dstate, ngroups=1, seed=0, dt_range=(1e-3, 1e-1),
                    a_log_range=(0.0, float(np.log(16.0)))):
    """Seeded synthetic inputs of the benchmark's SSD configs: x, dy ~ N(0,1);
    dt = softplus(N(0,1) + b_h) clipped to dt_range; A = -exp(U(a_log_range));
    B, C ~ N(0,1) / sqrt(dstate); D ~ N(0,1).  float32 arrays."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((batch, seqlen, nheads, headdim)).astype(np.float32)
    dy = rng.standard_normal((batch, seqlen, nheads, headdim)).astype(np.float32)
    lo, hi = dt_range
    bias = np.log(np.expm1(np.exp(rng.uniform(np.log(lo), np.log(hi), size=nheads))))
    raw = rng.standard_normal((batch, seqlen, nheads)) + bias
    dt = np.clip(np.log1p(np.exp(raw)), lo, hi).astype(np.float32)
    A = (-np.exp(rng.uniform(a_log_range[0], a_log_range[1], size=nheads))).astype(np.float32)
    B = (rng.standard_normal((batch, seqlen, ngroups, dstate)) / np.sqrt(dstate)).astype(np.float32)
    C = (rng.standard_normal((batch, seqlen, ngroups, dstate)) / np.sqrt(dstate)).astype(np.float32)
    D = rng.standard_normal(nheads).astype(np.float32)
    return x, dt, A, B, C, D, dy
