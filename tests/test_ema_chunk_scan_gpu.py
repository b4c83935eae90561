"""GPU parity of the dt-parameterised EMA (benchmark configs 1, 2, 4 form)
against the float64 oracle, plus launch-protocol checks (many launches in a
row, CUDA-graph replay, concurrent streams)."""

import numpy as np
import pytest
import torch

from _tol import assert_fp32_close, assert_lowp_close
from oracle import ema_oracle as eo

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _status_clean():
    from kernels import _lib
    yield
    assert _lib.device_status(clear=True) == 0, "a device-side wait timed out"


def _inputs(B, L, H, P, seed, dtype, dt_range=(1e-3, 1e-1), a_log=(0.0, np.log(16.0))):
    x, dt, A, dy = eo.make_dt_inputs(B, L, H, P, seed=seed, dt_range=dt_range, a_log_range=a_log)
    tx = torch.from_numpy(x).to(dtype)
    tdy = torch.from_numpy(dy).to(dtype)
    return tx, torch.from_numpy(dt), torch.from_numpy(A), tdy


def _run(tx, tdt, tA, tdy, Q, init=None, dfin=None):
    from kernels.ema_chunk_scan import ema_chunk_scan_bwd, ema_chunk_scan_fwd
    x, dt, A, dy = (t.to(DEV) for t in (tx, tdt, tA, tdy))
    y, states, fin = ema_chunk_scan_fwd(x, dt, A, Q, initial_states=init, return_final_states=True)
    dx, ddt, dA, dinit = ema_chunk_scan_bwd(x, dt, A, states, dy, Q, d_final_states=dfin,
                                            need_d_initial=True)
    return y, fin, dx, ddt, dA, dinit, states


def test_config1_fp32_forward():
    """B2 L512 H4 P64 chunk 64, fp32, dt = softplus(N(0,1) - 4),
    A = -exp(U(log 1, log 16)); y against the sequential recurrence."""
    rng = np.random.default_rng(0)
    B, L, H, P, Q = 2, 512, 4, 64, 64
    x = rng.standard_normal((B, L, H, P)).astype(np.float32)
    dt = np.logaddexp(0.0, rng.standard_normal((B, L, H)) - 4.0).astype(np.float32)
    A = (-np.exp(rng.uniform(0.0, np.log(16.0), H))).astype(np.float32)
    dy = rng.standard_normal((B, L, H, P)).astype(np.float32)
    y, fin, dx, ddt, dA, dinit, _ = _run(*(torch.from_numpy(v) for v in (x, dt, A, dy)), Q)
    r = eo.ema_dt_fwd(x, dt, A)
    g = eo.ema_dt_bwd(x, dt, A, dy)
    assert_fp32_close(y, r["y"], "y")
    assert_fp32_close(fin, r["final_state"], "final")
    assert_fp32_close(dx, g["dx"], "dx")
    assert_fp32_close(ddt, g["ddt"], "ddt")
    assert_fp32_close(dA, g["dA"], "dA")


_ORACLE_CACHE = {}


def _full_size_case(B, L, seed):
    """Seeded bf16 inputs of a benchmark shape (H32 P64) and the float64 oracle's
    outputs on the same bf16-rounded values, computed once per module."""
    key = (B, L, seed)
    if key not in _ORACLE_CACHE:
        H, P = 32, 64
        tx, tdt, tA, tdy = _inputs(B, L, H, P, seed, torch.bfloat16)
        xf, dyf = tx.float().numpy(), tdy.float().numpy()
        r = eo.ema_dt_fwd(xf, tdt.numpy(), tA.numpy())
        g = eo.ema_dt_bwd(xf, tdt.numpy(), tA.numpy(), dyf)
        _ORACLE_CACHE[key] = (tx, tdt, tA, tdy, r["y"], g)
    return _ORACLE_CACHE[key]


def _autograd_step(tx, tdt, tA, tdy, Q):
    from kernels.ema_chunk_scan import ema_chunk_scan_combined
    x, dt, A = (t.to(DEV).requires_grad_() for t in (tx, tdt, tA))
    y = ema_chunk_scan_combined(x, dt, A, Q)
    y.backward(tdy.to(DEV))
    return y.detach(), x.grad, dt.grad, A.grad


def test_config2_bf16_full_size():
    """BASELINE config 2 at full size: B8 L4096 H32 P64 chunk 256, bf16 I/O,
    fp32 accumulation, through the autograd op the benchmark times (256-token
    forward saving the state entering every 128 tokens, 128-token backward,
    dt transposed once and shared); y, dx, ddt and dA within 2e-2 rel / 1e-2 abs."""
    tx, tdt, tA, tdy, y_ref, g = _full_size_case(8, 4096, 7)
    y, dx, ddt, dA = _autograd_step(tx, tdt, tA, tdy, 256)
    assert_lowp_close(y, y_ref, "y")
    assert_lowp_close(dx, g["dx"], "dx")
    assert_lowp_close(ddt, g["ddt"], "ddt")
    assert_lowp_close(dA, g["dA"], "dA")
    assert_fp32_close(ddt, g["ddt"], "ddt (fp32 accumulation)")


def test_config2_bf16_full_size_direct_launchers():
    """The same inputs through the direct launchers at 256-token tiles in both
    directions (the pair a caller without the autograd op gets)."""
    tx, tdt, tA, tdy, y_ref, g = _full_size_case(8, 4096, 7)
    y, fin, dx, ddt, dA, _, _ = _run(tx, tdt, tA, tdy, 256)
    assert_lowp_close(y, y_ref, "y")
    assert_lowp_close(dx, g["dx"], "dx")
    assert_lowp_close(ddt, g["ddt"], "ddt")
    assert_lowp_close(dA, g["dA"], "dA")


def test_config4_bf16_full_size_one_gpu():
    """BASELINE config 4's sequence on one GPU: B1 L65536 H32 P64 chunk 256, bf16,
    through the autograd op (32 chains of 256 tiles: the longest look-back
    chains of the benchmark shapes)."""
    tx, tdt, tA, tdy, y_ref, g = _full_size_case(1, 65536, 21)
    y, dx, ddt, dA = _autograd_step(tx, tdt, tA, tdy, 256)
    assert_lowp_close(y, y_ref, "y")
    assert_lowp_close(dx, g["dx"], "dx")
    assert_lowp_close(ddt, g["ddt"], "ddt")
    assert_lowp_close(dA, g["dA"], "dA")


def _abi_fwd(x, dt, A, Q, ws, y, states):
    """ema_fwd_launch through the C ABI (strided dt, no dt_rows) on a caller workspace."""
    import ctypes

    from kernels import _lib
    B, L, H, P = x.shape
    a = _lib.EmaFwdArgs()
    a.batch, a.seqlen, a.nheads, a.headdim, a.chunk_size = B, L, H, P, Q
    a.dtype = _lib.DTYPE_CODES[x.dtype]
    a.x, a.x_stride = x.data_ptr(), _lib.strides3(x)
    a.out, a.out_stride = y.data_ptr(), _lib.strides3(y)
    a.dt, a.A = dt.data_ptr(), A.data_ptr()
    a.states, a.states_stride = states.data_ptr(), (_lib._i64 * 4)(*states.stride())
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(_lib.lib.ema_fwd_launch(ctypes.byref(a), _lib.stream_ptr(x.device)), "ema_fwd_launch")


def _abi_bwd(x, dt, A, states, dy, Q, ws, dx, ddt, dA):
    import ctypes

    from kernels import _lib
    B, L, H, P = x.shape
    b = _lib.EmaBwdArgs()
    b.batch, b.seqlen, b.nheads, b.headdim, b.chunk_size = B, L, H, P, Q
    b.dtype = _lib.DTYPE_CODES[x.dtype]
    b.x, b.x_stride = x.data_ptr(), _lib.strides3(x)
    b.dout, b.dout_stride = dy.data_ptr(), _lib.strides3(dy)
    b.dx, b.dx_stride = dx.data_ptr(), _lib.strides3(dx)
    b.dt, b.A = dt.data_ptr(), A.data_ptr()
    b.states, b.states_stride = states.data_ptr(), (_lib._i64 * 4)(*states.stride())
    b.ddt, b.dA_out = ddt.data_ptr(), dA.data_ptr()
    b.workspace, b.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(_lib.lib.ema_bwd_launch(ctypes.byref(b), _lib.stream_ptr(x.device)), "ema_bwd_launch")


def test_epoch_wrap_clears_stale_records():
    """Look-back records are tagged with the launch epoch + 1, and the epoch wraps
    to 0 after 2^30 launches.  A workspace is set up as it could be found then:
    epoch 2^30 - 1 and every record word holding a stale value under tag 1, the
    tag of the first launch after the wrap.  A small launch (which wraps the
    epoch) and then a larger one, which reads slots the small one never wrote,
    must both match the same launches on a fresh workspace, forward and
    backward; the status word stays clear."""
    from kernels import _lib
    Q = 256
    small = _inputs(1, 512, 2, 64, 31, torch.bfloat16)
    big = _inputs(2, 2048, 8, 64, 32, torch.bfloat16)
    need = _lib.lib.ema_scan_workspace_size(2, 2048, 8, 64, Q)

    def stale_workspace():
        ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
        words = ws[256:].view(torch.int64)
        stale = (1 << 32) | int(np.array(1e30, dtype=np.float32).view(np.uint32))
        words.fill_(stale)
        ws[:4].view(torch.int32).fill_(0x3FFFFFFF)
        return ws

    def run(case, ws):
        x, dt, A, dy = (t.to(DEV) for t in case)
        B, L, H, P = x.shape
        nc = -(-L // Q)
        y = torch.empty_like(x)
        st = torch.empty(B, nc, H, P, dtype=torch.float32, device=DEV)
        _abi_fwd(x, dt, A, Q, ws, y, st)
        dx = torch.empty_like(x)
        ddt = torch.empty(B, L, H, dtype=torch.float32, device=DEV)
        dA = torch.empty(H, dtype=torch.float32, device=DEV)
        return y, st, dx, ddt, dA, (x, dt, A, dy)

    def run_bwd(out, ws):
        y, st, dx, ddt, dA, (x, dt, A, dy) = out
        _abi_bwd(x, dt, A, st, dy, Q, ws, dx, ddt, dA)
        return y, dx, ddt, dA

    fresh = torch.zeros(need, dtype=torch.uint8, device=DEV)
    ref = run_bwd(run(big, fresh), fresh)
    # forward: the small launch wraps the epoch, the big one runs at tag 1
    ws = stale_workspace()
    fs = run(small, ws)
    fb = run(big, ws)
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32).item()) == 1, "two launches after 2^30 - 1 leave epoch 1"
    # backward, the same way
    ws2 = stale_workspace()
    run_bwd(fs, ws2)
    got = run_bwd(fb, ws2)
    torch.cuda.synchronize()
    for w in (ws, ws2):
        assert int(w[12:16].view(torch.int32).item()) == 0, "device status word set"
    close = dict(rtol=1e-2, atol=1e-3)
    torch.testing.assert_close(got[0], ref[0], **close)
    torch.testing.assert_close(got[1], ref[1], **close)
    torch.testing.assert_close(got[2], ref[2], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(got[3], ref[3], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("L", [1000, 999])
def test_dt_rows_and_strided_dt_agree(L):
    """The launchers read each tile's dt either as one row of the (B, H, L) copy
    the forward makes (the Python API's path) or as a column of dt (B, L, H)
    strided by nheads (a C caller that passes no dt_rows buffer).  Both agree
    with each other and with the oracle; L = 999 leaves the rows unaligned for
    bulk copies (element-wise fallback)."""
    import ctypes

    from kernels import _lib
    from kernels.ema_chunk_scan import ema_chunk_scan_bwd, ema_chunk_scan_fwd
    B, H, P, Q = 2, 3, 64, 256
    tx, tdt, tA, tdy = _inputs(B, L, H, P, L, torch.bfloat16)
    x, dt, A, dy = (t.to(DEV) for t in (tx, tdt, tA, tdy))
    y, st, _ = ema_chunk_scan_fwd(x, dt, A, Q)
    dx, ddt, dA, _ = ema_chunk_scan_bwd(x, dt, A, st, dy, Q)

    nc = -(-L // Q)
    stream = _lib.stream_ptr(torch.device(DEV))
    ws = torch.zeros(_lib.lib.ema_scan_workspace_size(B, L, H, P, Q), dtype=torch.uint8, device=DEV)
    y2 = torch.empty_like(x)
    st2 = torch.empty(B, nc, H, P, dtype=torch.float32, device=DEV)
    a = _lib.EmaFwdArgs()
    a.batch, a.seqlen, a.nheads, a.headdim, a.chunk_size = B, L, H, P, Q
    a.dtype = _lib.DTYPE_CODES[x.dtype]
    a.x, a.x_stride = x.data_ptr(), _lib.strides3(x)
    a.out, a.out_stride = y2.data_ptr(), _lib.strides3(y2)
    a.dt, a.A = dt.data_ptr(), A.data_ptr()
    s = st2.stride()
    a.states, a.states_stride = st2.data_ptr(), (_lib._i64 * 4)(*s)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(_lib.lib.ema_fwd_launch(ctypes.byref(a), stream), "forward, strided dt")
    dx2 = torch.empty_like(x)
    ddt2 = torch.empty(B, L, H, dtype=torch.float32, device=DEV)
    dA2 = torch.empty(H, dtype=torch.float32, device=DEV)
    b = _lib.EmaBwdArgs()
    b.batch, b.seqlen, b.nheads, b.headdim, b.chunk_size = B, L, H, P, Q
    b.dtype = a.dtype
    b.x, b.x_stride = x.data_ptr(), _lib.strides3(x)
    b.dout, b.dout_stride = dy.data_ptr(), _lib.strides3(dy)
    b.dx, b.dx_stride = dx2.data_ptr(), _lib.strides3(dx2)
    b.dt, b.A = dt.data_ptr(), A.data_ptr()
    b.states, b.states_stride = st2.data_ptr(), (_lib._i64 * 4)(*s)
    b.ddt, b.dA_out = ddt2.data_ptr(), dA2.data_ptr()
    b.workspace, b.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(_lib.lib.ema_bwd_launch(ctypes.byref(b), stream), "backward, strided dt")
    torch.cuda.synchronize()
    close = dict(rtol=1e-2, atol=1e-3)  # one bf16 ulp: tiles may combine aggregate or inclusive records
    torch.testing.assert_close(y2, y, **close)
    torch.testing.assert_close(st2, st, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(dx2, dx, **close)
    torch.testing.assert_close(ddt2, ddt, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(dA2, dA, rtol=1e-4, atol=1e-4)
    g = eo.ema_dt_bwd(tx.float().numpy(), tdt.numpy(), tA.numpy(), tdy.float().numpy())
    assert_lowp_close(dx2, g["dx"], "dx (strided dt)")
    assert_lowp_close(ddt2, g["ddt"], "ddt (strided dt)")


@pytest.mark.parametrize("Q", [64, 128, 256])
@pytest.mark.parametrize("P", [32, 64, 128])
def test_fp32_states_and_boundaries(Q, P):
    B, L, H = 2, 777, 3
    tx, tdt, tA, tdy = _inputs(B, L, H, P, Q + P, torch.float32, dt_range=(1e-3, 0.5))
    rng = np.random.default_rng(1)
    init = rng.standard_normal((B, H, P)).astype(np.float32)
    dfin = rng.standard_normal((B, H, P)).astype(np.float32)
    if P == 128 and Q == 256:
        # fp32 x and dy tiles of 256 x 128 need 256 KB of shared memory: the
        # backward rejects the combination with a clear error (chunk <= 128 works)
        from kernels._lib import EmaLaunchError
        with pytest.raises(EmaLaunchError, match="shared memory"):
            _run(tx, tdt, tA, tdy, Q)
        return
    y, fin, dx, ddt, dA, dinit, states = _run(tx, tdt, tA, tdy, Q, init=torch.from_numpy(init).to(DEV),
                                              dfin=torch.from_numpy(dfin).to(DEV))
    r = eo.ema_dt_fwd(tx.numpy(), tdt.numpy(), tA.numpy(), initial_state=init)
    g = eo.ema_dt_bwd(tx.numpy(), tdt.numpy(), tA.numpy(), tdy.numpy(), initial_state=init,
                      d_final_state=dfin)
    assert_fp32_close(y, r["y"], "y")
    assert_fp32_close(fin, r["final_state"], "final")
    assert_fp32_close(dx, g["dx"], "dx")
    assert_fp32_close(ddt, g["ddt"], "ddt")
    assert_fp32_close(dA, g["dA"], "dA")
    assert_fp32_close(dinit, g["d_initial_state"], "d_initial")
    # chunk start states: chunk 0 is the initial state, chunk k the state after token k*Q-1
    st = states.cpu().numpy()
    np.testing.assert_allclose(st[:, 0].transpose(0, 1, 2), init, rtol=0, atol=0)
    for k in range(1, st.shape[1]):
        assert_fp32_close(st[:, k], r["y"][:, k * Q - 1], f"state {k}")


@pytest.mark.parametrize("L", [1, 63, 256, 257])
def test_short_and_ragged_sequences(L):
    tx, tdt, tA, tdy = _inputs(3, L, 2, 64, L, torch.float32)
    y, fin, dx, ddt, dA, _, _ = _run(tx, tdt, tA, tdy, 256)
    r = eo.ema_dt_fwd(tx.numpy(), tdt.numpy(), tA.numpy())
    g = eo.ema_dt_bwd(tx.numpy(), tdt.numpy(), tA.numpy(), tdy.numpy())
    assert_fp32_close(y, r["y"], "y")
    assert_fp32_close(dx, g["dx"], "dx")
    assert_fp32_close(ddt, g["ddt"], "ddt")
    assert_fp32_close(dA, g["dA"], "dA")


def test_autograd_matches_oracle_and_reuses_workspace():
    from kernels.ema_chunk_scan import ema_chunk_scan_combined
    tx, tdt, tA, tdy = _inputs(2, 600, 4, 64, 11, torch.bfloat16)
    x = tx.to(DEV).requires_grad_()
    dt = tdt.to(DEV).requires_grad_()
    A = tA.to(DEV).requires_grad_()
    for _ in range(3):  # repeated launches on one workspace
        x.grad = dt.grad = A.grad = None
        y = ema_chunk_scan_combined(x, dt, A, chunk_size=128)
        (y * tdy.to(DEV)).sum().backward()
    g = eo.ema_dt_bwd(tx.float().numpy(), tdt.numpy(), tA.numpy(), tdy.float().numpy())
    assert_lowp_close(x.grad, g["dx"], "dx")
    assert_lowp_close(dt.grad, g["ddt"], "ddt")
    assert_lowp_close(A.grad, g["dA"], "dA")


def test_final_state_gradient_through_autograd():
    from kernels.ema_chunk_scan import ema_chunk_scan_combined
    tx, tdt, tA, tdy = _inputs(1, 300, 2, 32, 12, torch.float32)
    rng = np.random.default_rng(3)
    init = torch.from_numpy(rng.standard_normal((1, 2, 32)).astype(np.float32)).to(DEV).requires_grad_()
    dfin = rng.standard_normal((1, 2, 32)).astype(np.float32)
    x, dt, A = (t.to(DEV).requires_grad_() for t in (tx, tdt, tA))
    y, fin = ema_chunk_scan_combined(x, dt, A, 64, initial_states=init, return_final_states=True)
    ((y * tdy.to(DEV)).sum() + (fin * torch.from_numpy(dfin).to(DEV)).sum()).backward()
    g = eo.ema_dt_bwd(tx.numpy(), tdt.numpy(), tA.numpy(), tdy.numpy(),
                      initial_state=init.detach().cpu().numpy(), d_final_state=dfin)
    assert_fp32_close(x.grad, g["dx"], "dx")
    assert_fp32_close(dt.grad, g["ddt"], "ddt")
    assert_fp32_close(A.grad, g["dA"], "dA")
    assert_fp32_close(init.grad, g["d_initial_state"], "d_init")


def test_many_launches_and_cuda_graph_replay():
    """The self-resetting workspace protocol: 200 back-to-back launches, then a
    captured graph replayed 50 times, all equal to the first result up to the
    rounding of the look-back path (a tile may combine its predecessor's
    aggregate or its inclusive prefix, whichever is published first)."""
    from kernels.ema_chunk_scan import ema_chunk_scan_bwd, ema_chunk_scan_fwd
    tx, tdt, tA, tdy = _inputs(2, 1024, 8, 64, 13, torch.bfloat16)
    x, dt, A, dy = (t.to(DEV) for t in (tx, tdt, tA, tdy))
    y0, st0, _ = ema_chunk_scan_fwd(x, dt, A, 256)
    dx0, ddt0, dA0, _ = ema_chunk_scan_bwd(x, dt, A, st0, dy, 256)
    for _ in range(200):
        y, st, _ = ema_chunk_scan_fwd(x, dt, A, 256)
    dx, ddt, dA, _ = ema_chunk_scan_bwd(x, dt, A, st, dy, 256)
    close = dict(rtol=1e-2, atol=1e-3)  # one bf16 ulp
    torch.testing.assert_close(y, y0, **close)
    torch.testing.assert_close(dx, dx0, **close)
    torch.testing.assert_close(ddt, ddt0, rtol=1e-4, atol=1e-4)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ema_chunk_scan_fwd(x, dt, A, 256)  # warm the side stream's workspace
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        yg, stg, _ = ema_chunk_scan_fwd(x, dt, A, 256)
        dxg, ddtg, dAg, _ = ema_chunk_scan_bwd(x, dt, A, stg, dy, 256)
    for _ in range(50):
        g.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(yg, y0, **close)
    torch.testing.assert_close(dxg, dx0, **close)
    torch.testing.assert_close(dAg, dA0, rtol=1e-4, atol=1e-4)


def test_concurrent_streams_use_separate_workspaces():
    from kernels.ema_chunk_scan import ema_chunk_scan_fwd
    tx, tdt, tA, _ = _inputs(4, 2048, 16, 64, 14, torch.bfloat16)
    x, dt, A = (t.to(DEV) for t in (tx, tdt, tA))
    ref, _, _ = ema_chunk_scan_fwd(x, dt, A, 256)
    streams = [torch.cuda.Stream() for _ in range(3)]
    outs = []
    for s in streams:
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            outs.append(ema_chunk_scan_fwd(x, dt, A, 256)[0])
    for s in streams:
        torch.cuda.current_stream().wait_stream(s)
    for o in outs:
        torch.testing.assert_close(o, ref, rtol=1e-2, atol=1e-3)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_state_only_passes_and_span_chaining(dtype):
    """The sequence-parallel building blocks on one GPU: state-only passes give
    the same final state / initial-state gradient as the full passes, and a
    sequence split into spans, chained on the host as kernels/ema_sp.py chains
    them over NCCL, reproduces the whole-sequence results."""
    from kernels.ema_chunk_scan import ema_chunk_scan_bwd, ema_chunk_scan_fwd
    from kernels.ema_sp import span_decay
    B, L, H, P, Q, R = 2, 1024, 3, 64, 128, 4
    tx, tdt, tA, tdy = _inputs(B, L, H, P, 31, dtype)
    x, dt, A, dy = (t.to(DEV) for t in (tx, tdt, tA, tdy))
    y_full, st_full, fin_full = ema_chunk_scan_fwd(x, dt, A, Q, return_final_states=True)
    dx_full, ddt_full, dA_full, _ = ema_chunk_scan_bwd(x, dt, A, st_full, dy, Q)

    none_y, none_st, fin_so = ema_chunk_scan_fwd(x, dt, A, Q, state_only=True)
    assert none_y is None and none_st is None
    assert_fp32_close(fin_so, fin_full.cpu().numpy(), "state-only final state")
    dinit_full = ema_chunk_scan_bwd(x, dt, A, st_full, dy, Q, need_d_initial=True)[3]
    dx_so, ddt_so, dA_so, dinit_so = ema_chunk_scan_bwd(x, dt, A, st_full, dy, Q, state_only=True)
    assert dx_so is None and ddt_so is None and dA_so is None
    assert_fp32_close(dinit_so, dinit_full.cpu().numpy(), "state-only initial-state gradient")

    span = L // R
    sl = [slice(r * span, (r + 1) * span) for r in range(R)]
    xs = [x[:, s].contiguous() for s in sl]
    dts = [dt[:, s].contiguous() for s in sl]
    dys = [dy[:, s].contiguous() for s in sl]
    # forward chain r -> r+1
    Sin, sins = torch.zeros(B, H, P, device=DEV), []
    for r in range(R):
        sins.append(Sin)
        S_loc = ema_chunk_scan_fwd(xs[r], dts[r], A, Q, state_only=True)[2]
        Sin = span_decay(dts[r], A)[..., None] * Sin + S_loc
    outs = [ema_chunk_scan_fwd(xs[r], dts[r], A, Q, initial_states=sins[r]) for r in range(R)]
    y_sp = torch.cat([o[0] for o in outs], dim=1)
    # backward chain r+1 -> r
    Gin, gins = torch.zeros(B, H, P, device=DEV), [None] * R
    for r in reversed(range(R)):
        gins[r] = Gin
        G_loc = ema_chunk_scan_bwd(xs[r], dts[r], A, outs[r][1], dys[r], Q, state_only=True)[3]
        Gin = span_decay(dts[r], A)[..., None] * Gin + G_loc
    grads = [ema_chunk_scan_bwd(xs[r], dts[r], A, outs[r][1], dys[r], Q, d_final_states=gins[r])
             for r in range(R)]
    dx_sp = torch.cat([g[0] for g in grads], dim=1)
    ddt_sp = torch.cat([g[1] for g in grads], dim=1)
    dA_sp = sum(g[2] for g in grads)
    check = assert_fp32_close if dtype == torch.float32 else assert_lowp_close
    check(y_sp, y_full.float().cpu().numpy(), "span-chained y")
    check(dx_sp, dx_full.float().cpu().numpy(), "span-chained dx")
    check(ddt_sp, ddt_full.cpu().numpy(), "span-chained ddt")
    check(dA_sp, dA_full.cpu().numpy(), "span-chained dA")


@pytest.mark.parametrize("P,L", [(64, 1000), (128, 700), (64, 256), (64, 600)])
def test_half_chunk_states_feed_the_half_chunk_backward(P, L):
    """A 256-token forward with half_chunk_states returns the state entering
    every 128 tokens (chunk c's start at 2c, matching the 128-token forward's
    states); the backward on those 128-token chunks matches the oracle.  This
    is the pair the autograd op runs at chunk_size 256."""
    from kernels.ema_chunk_scan import (backward_chunk, ema_chunk_scan_bwd, ema_chunk_scan_combined,
                                        ema_chunk_scan_fwd)
    assert backward_chunk(256) == 128
    tx, tdt, tA, tdy = _inputs(2, L, 3, P, 31 + L, torch.float32)
    x, dt, A, dy = (t.to(DEV) for t in (tx, tdt, tA, tdy))
    rng = np.random.default_rng(3)
    init = torch.from_numpy(rng.standard_normal((2, 3, P)).astype(np.float32)).to(DEV)
    y, fine, fin = ema_chunk_scan_fwd(x, dt, A, 256, initial_states=init, return_final_states=True,
                                      half_chunk_states=True)
    y128, st128, fin128 = ema_chunk_scan_fwd(x, dt, A, 128, initial_states=init, return_final_states=True)
    nc128 = -(-L // 128)
    assert fine.shape == (2, nc128, 3, P)
    assert_fp32_close(fine, st128, "half-chunk states")
    assert_fp32_close(y, y128, "y")
    dfin = torch.from_numpy(rng.standard_normal((2, 3, P)).astype(np.float32)).to(DEV)
    g128 = ema_chunk_scan_bwd(x, dt, A, fine, dy, 128, d_final_states=dfin, need_d_initial=True)
    # the same backward on the 128-token forward's states (headdim 128 has no
    # 256-token backward: its tiles do not fit in shared memory)
    gref = ema_chunk_scan_bwd(x, dt, A, st128, dy, 128, d_final_states=dfin, need_d_initial=True)
    for name, a, b in zip(("dx", "ddt", "dA", "d_init"), g128, gref):
        assert_fp32_close(a, b, name)
    g = eo.ema_dt_bwd(tx.numpy(), tdt.numpy(), tA.numpy(), tdy.numpy(), initial_state=init.cpu().numpy(),
                      d_final_state=dfin.cpu().numpy())
    assert_fp32_close(g128[0], g["dx"], "dx vs oracle")
    assert_fp32_close(g128[1], g["ddt"], "ddt vs oracle")
    # the autograd op at chunk 256 (which takes this path) agrees too
    xg = x.clone().requires_grad_()
    yy = ema_chunk_scan_combined(xg, dt, A, chunk_size=256)
    (yy * dy).sum().backward()
    g0 = eo.ema_dt_bwd(tx.numpy(), tdt.numpy(), tA.numpy(), tdy.numpy())
    assert_fp32_close(xg.grad, g0["dx"], "autograd dx")


@pytest.mark.parametrize("Q", [128, 256])
def test_few_long_chains_match_oracle(Q):
    """Two (batch, head) sequences of 16-32 tiles each (every tile's look-back
    walks a chain with many tiles in flight): forward with an initial state,
    backward with a final-state gradient, both state-only passes (the backward
    one reads no x) and the autograd pair, all in fp32 against the float64
    oracle."""
    from kernels.ema_chunk_scan import ema_chunk_scan_bwd, ema_chunk_scan_fwd
    B, L, H, P = 1, 4096, 2, 64
    tx, tdt, tA, tdy = _inputs(B, L, H, P, 40 + Q, torch.float32, dt_range=(1e-3, 0.2))
    rng = np.random.default_rng(5)
    init = rng.standard_normal((B, H, P)).astype(np.float32)
    dfin = rng.standard_normal((B, H, P)).astype(np.float32)
    x, dt, A, dy = (t.to(DEV) for t in (tx, tdt, tA, tdy))
    ti, tf = torch.from_numpy(init).to(DEV), torch.from_numpy(dfin).to(DEV)
    y, st, fin = ema_chunk_scan_fwd(x, dt, A, Q, initial_states=ti, return_final_states=True)
    _, _, fin_only = ema_chunk_scan_fwd(x, dt, A, Q, initial_states=ti, state_only=True)
    dx, ddt, dA, dinit = ema_chunk_scan_bwd(x, dt, A, st, dy, Q, d_final_states=tf, need_d_initial=True)
    _, _, _, dinit_only = ema_chunk_scan_bwd(x, dt, A, st, dy, Q, d_final_states=tf, state_only=True)
    r = eo.ema_dt_fwd(tx.numpy(), tdt.numpy(), tA.numpy(), initial_state=init)
    g = eo.ema_dt_bwd(tx.numpy(), tdt.numpy(), tA.numpy(), tdy.numpy(), initial_state=init, d_final_state=dfin)
    assert_fp32_close(y, r["y"], "y")
    assert_fp32_close(fin, r["final_state"], "final")
    assert_fp32_close(fin_only, r["final_state"], "final (state-only)")
    assert_fp32_close(st[:, 1:], r["y"][:, Q - 1::Q][:, :st.shape[1] - 1], "chunk start states")
    assert_fp32_close(dx, g["dx"], "dx")
    assert_fp32_close(ddt, g["ddt"], "ddt")
    assert_fp32_close(dA, g["dA"], "dA")
    assert_fp32_close(dinit, g["d_initial_state"], "d_initial")
    assert_fp32_close(dinit_only, g["d_initial_state"], "d_initial (state-only)")
    # the autograd pair: a 256-token forward with half-chunk states and the 128-token backward
    if Q == 256:
        from kernels.ema_chunk_scan import ema_chunk_scan_combined
        xg, dtg, Ag = (t.clone().requires_grad_() for t in (x, dt, A))
        yg = ema_chunk_scan_combined(xg, dtg, Ag, 256)
        yg.backward(dy)
        g0 = eo.ema_dt_bwd(tx.numpy(), tdt.numpy(), tA.numpy(), tdy.numpy())
        assert_fp32_close(xg.grad, g0["dx"], "autograd dx")
        assert_fp32_close(dtg.grad, g0["ddt"], "autograd ddt")
        assert_fp32_close(Ag.grad, g0["dA"], "autograd dA")
