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
@pytest.mark.parametrize("P", [48, 7])
def test_fold_kernels_match_float64(K, direction, scale, P):
    """P = 7: an expansion CTA's 256 outputs span many sub-spans (rows of
    weights); P = 48: a sub-span's channels straddle two CTAs."""
    from kernels.ema_sp import _kernel_fold
    g = torch.Generator().manual_seed(K * 10 + direction)
    B, H = 2, 5
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


@pytest.mark.parametrize("P,dtype", [(64, torch.bfloat16), (32, torch.float32), (128, torch.float16)])
@pytest.mark.parametrize("L,dt_range", [(1000, (1e-3, 1e-1)), (4096, (1e-2, 1.0)), (300, (1e-4, 1e-3))])
def test_span_state_matches_scan_state_only_passes_and_oracle(P, dtype, L, dt_range):
    """The state-only passes as weighted column sums (ema_span_state_launch)
    against the scan kernels' state-only modes and the float64 oracle: the end
    state from zero (direction 0) and the start-state gradient from dy
    (direction 1), ragged lengths, steep and slow decays."""
    import numpy as np
    from kernels.ema_chunk_scan import ema_chunk_scan_bwd, ema_chunk_scan_fwd
    from kernels.ema_sp import span_state
    from oracle import ema_oracle as eo
    x, dt, A, dy = eo.make_dt_inputs(3, L, 4, P, seed=L + P, dt_range=dt_range)
    tx, tdy = (torch.from_numpy(a).to(dtype).to(DEV) for a in (x, dy))
    tdt, tA = torch.from_numpy(dt).to(DEV), torch.from_numpy(A).to(DEV)
    s_end, ld0 = span_state(tx, tdt, tA, 0, log_decay=True)
    g_start, ld1 = span_state(tdy, tdt, tA, 1, log_decay=True)
    ld_ref = tdt.double().sum(dim=1) * tA.double()  # the rows' log decays, float64
    for ld in (ld0, ld1):
        assert ld.dtype == torch.float64
        torch.testing.assert_close(ld, ld_ref, rtol=1e-12, atol=0.0)
    torch.testing.assert_close(span_state(tx, tdt, tA, 0), s_end, rtol=0, atol=0)
    s_scan = ema_chunk_scan_fwd(tx, tdt, tA, 128, state_only=True)[2]
    _, states, _ = ema_chunk_scan_fwd(tx, tdt, tA, 128)
    g_scan = ema_chunk_scan_bwd(tx, tdt, tA, states, tdy, 128, state_only=True)[3]
    xf, dyf = tx.float().cpu().numpy(), tdy.float().cpu().numpy()
    r = eo.ema_dt_fwd(xf, dt, A)
    g = eo.ema_dt_bwd(xf, dt, A, dyf)
    for got, scan, ref, what in ((s_end, s_scan, r["final_state"], "end state"),
                                 (g_start, g_scan, g["d_initial_state"], "start gradient")):
        ref = np.asarray(ref)
        e = float(np.abs(got.double().cpu().numpy() - ref).max() / max(np.abs(ref).max(), 1e-30))
        assert e <= 1e-4, f"{what}: normwise relative error {e:.3e} against the oracle"
        torch.testing.assert_close(got, scan, rtol=1e-4, atol=1e-5 * float(scan.abs().max()), msg=what)


@pytest.mark.parametrize("K", [4, 8])
def test_one_gpu_subspans_match_oracle(K):
    """One GPU, one long sequence cut into K sub-spans run as batch rows (what
    kernels/ema_sp.py does at world size 1 for long sequences: column-sum state
    pass, expansion fold, full passes on the rows) against the float64 oracle
    on the same bf16 inputs."""
    import torch.distributed as dist
    from _tol import assert_lowp_close
    from kernels import ema_sp
    from oracle import ema_oracle as eo
    own = not dist.is_initialized()
    if own:  # a one-rank group, as bench.py's config-4 leg uses on one GPU
        dist.init_process_group("gloo", store=dist.HashStore(), rank=0, world_size=1)
    try:
        B, L, H, P, Q = 1, 8192, 4, 64, 256
        x, dt, A, dy = eo.make_dt_inputs(B, L, H, P, seed=31)
        tx, tdy = (torch.from_numpy(a).to(torch.bfloat16).to(DEV) for a in (x, dy))
        tdt, tA = torch.from_numpy(dt).to(DEV), torch.from_numpy(A).to(DEV)
        y, states, _, _ = ema_sp.sp_forward(tx, tdt, tA, Q, subspans=K)
        assert states.shape[0] == B * K
        dx, ddt, dA, _ = ema_sp.sp_backward(tx, tdt, tA, states, tdy, Q)
        xf, dyf = tx.float().cpu().numpy(), tdy.float().cpu().numpy()
        r = eo.ema_dt_fwd(xf, dt, A)
        g = eo.ema_dt_bwd(xf, dt, A, dyf)
        assert_lowp_close(y, r["y"], "y")
        assert_lowp_close(dx, g["dx"], "dx")
        assert_lowp_close(ddt, g["ddt"], "ddt")
        assert_lowp_close(dA, g["dA"], "dA")
    finally:
        if own:
            dist.destroy_process_group()


def _exchange_args(_lib, B, K, H, P, direction, rank, world, ld, V, bnd, span_in, out, bufs, nbytes):
    a = _lib.EmaSpanExchangeArgs()
    a.batch, a.subspans, a.nheads, a.headdim = B, K, H, P
    a.direction, a.rank, a.world = direction, rank, world
    a.log_decay, a.values = ld.data_ptr(), V.data_ptr()
    a.boundary = None if bnd is None else bnd.data_ptr()
    a.span_in, a.out = span_in.data_ptr(), out.data_ptr()
    a.buffer_bytes = nbytes
    for q, b in enumerate(bufs):
        a.buffers[q] = b.value
    return a


@pytest.mark.parametrize("direction", [0, 1])
def test_exchange_kernel_one_rank_expands_like_the_fold(direction):
    """The peer-memory exchange kernel (ema_span_exchange) as a one-rank group
    on one GPU: no peer to wait for, the span's boundary value is the given
    one, and its expansion over the sub-spans (a float64 recurrence) matches
    the float64 pairwise fold; three calls in a row on the same buffer."""
    import ctypes
    from kernels import _lib
    L = _lib.lib
    B, K, H, P = 2, 8, 5, 48
    g = torch.Generator().manual_seed(40 + direction)
    dev = torch.device("cuda", torch.cuda.current_device())
    nbytes = L.ema_span_exchange_bytes(1, B * H, P)
    buf = ctypes.c_void_p()
    _lib.check(L.ema_p2p_alloc(nbytes, ctypes.byref(buf)), "ema_p2p_alloc")
    try:
        for call in range(3):
            ld = (-torch.rand(B, K, H, generator=g, dtype=torch.float64) * (0.05, 30.0, 2.0)[call]).to(dev)
            V = torch.randn(B * K, H, P, generator=g).to(dev)
            bnd = torch.randn(B, H, P, generator=g).to(dev)
            span_in = torch.empty(B, H, P, device=dev)
            out = torch.empty(B * K, H, P, device=dev)
            a = _exchange_args(_lib, B, K, H, P, direction, 0, 1, ld, V, bnd, span_in, out, [buf], nbytes)
            _lib.check(L.ema_span_exchange(ctypes.byref(a), _lib.stream_ptr(dev)), "ema_span_exchange")
            torch.testing.assert_close(span_in, bnd, rtol=0, atol=0)
            torch.testing.assert_close(out, torch_fold(direction, True, ld, V, bnd), rtol=1e-6, atol=1e-6)
        word = ctypes.c_uint32()
        _lib.check(L.ema_span_exchange_status(buf, ctypes.byref(word), 0), "ema_span_exchange_status")
        assert word.value == 0
    finally:
        L.ema_p2p_free(buf)


def test_exchange_wait_for_a_missing_rank_runs_out_and_reports():
    """Failure detection of the exchange kernel without a second GPU: rank 0 of
    a two-rank group whose rank 1 never calls (its flags are never set; both
    buffers are local).  The bounded wait gives up after about 1 s, sets bit 1
    of the buffer's status word and the launch finishes; clearing the word
    leaves it at zero."""
    import ctypes
    import time
    from kernels import _lib
    L = _lib.lib
    B, K, H, P = 1, 4, 2, 64
    dev = torch.device("cuda", torch.cuda.current_device())
    nbytes = L.ema_span_exchange_bytes(2, B * H, P)
    bufs = [ctypes.c_void_p(), ctypes.c_void_p()]
    for b in bufs:
        _lib.check(L.ema_p2p_alloc(nbytes, ctypes.byref(b)), "ema_p2p_alloc")
    try:
        ld = -torch.rand(B, K, H, dtype=torch.float64, device=dev)
        V = torch.randn(B * K, H, P, device=dev)
        span_in = torch.empty(B, H, P, device=dev)
        out = torch.empty(B * K, H, P, device=dev)
        a = _exchange_args(_lib, B, K, H, P, 0, 0, 2, ld, V, None, span_in, out, bufs, nbytes)
        torch.cuda.synchronize(dev)
        t0 = time.monotonic()
        _lib.check(L.ema_span_exchange(ctypes.byref(a), _lib.stream_ptr(dev)), "ema_span_exchange")
        torch.cuda.synchronize(dev)
        waited = time.monotonic() - t0
        word = ctypes.c_uint32()
        _lib.check(L.ema_span_exchange_status(bufs[0], ctypes.byref(word), 1), "ema_span_exchange_status")
        assert word.value == 1, f"status word {word.value}"
        assert 0.9 <= waited < 20.0, f"the wait ended after {waited:.2f} s"
        _lib.check(L.ema_span_exchange_status(bufs[0], ctypes.byref(word), 0), "ema_span_exchange_status")
        assert word.value == 0
    finally:
        for b in bufs:
            L.ema_p2p_free(b)
