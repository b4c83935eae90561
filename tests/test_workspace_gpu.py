"""The per-stream look-back workspace (kernels/_lib.py): sizes grow by powers
of two, a replaced buffer is dropped unless a CUDA graph capture used it, and a
captured graph keeps running on its buffer after the stream's workspace grew."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_growth_and_retirement():
    from kernels import _lib
    s = torch.cuda.Stream(DEV)
    with torch.cuda.stream(s):
        a = _lib.workspace(DEV, 1000)
        n0 = a.numel()  # (a recycled stream handle may already own a larger buffer)
        assert n0 >= 1 << 20 and n0 & (n0 - 1) == 0
        was_captured = (DEV.index, s.cuda_stream) in _lib._ws_captured
        n_retired = len(_lib._ws_retired)
        want = 3 * n0 + 1
        b = _lib.workspace(DEV, want)
        assert b.numel() == 1 << (want - 1).bit_length()
        assert len(_lib._ws_retired) == n_retired + int(was_captured)  # never captured: dropped
        assert _lib.workspace(DEV, want) is b


def test_captured_graph_survives_growth():
    from kernels.ema_chunk_scan import ema_chunk_scan_fwd
    from kernels import _lib
    g = torch.Generator(device="cpu").manual_seed(3)
    x = torch.randn(1, 512, 2, 64, generator=g).to(DEV, torch.bfloat16)
    dt = (torch.rand(1, 512, 2, generator=g) * 0.1 + 1e-3).to(DEV)
    A = -torch.rand(2, generator=g).to(DEV) - 0.5
    s = torch.cuda.Stream(DEV)
    s.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(s):
        y_ref, _, _ = ema_chunk_scan_fwd(x, dt, A, 128)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            y_g, _, _ = ema_chunk_scan_fwd(x, dt, A, 128)
        n_retired = len(_lib._ws_retired)
        big = _lib.workspace(DEV, 64 << 20)  # the stream's workspace grows past the captured one
        assert len(_lib._ws_retired) == n_retired + 1
        graph.replay()
        s.synchronize()
    torch.testing.assert_close(y_g, y_ref, rtol=1e-2, atol=1e-2)
    assert big.numel() >= 64 << 20
    assert _lib.device_status(clear=True) == 0
