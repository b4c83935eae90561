"""Sequence-parallel EMA (kernels/ema_sp.py) on two GPUs over NCCL: each rank
runs the CUDA kernels on its span of the sequence, the span states (forward)
and span-end gradients (backward) cross between the GPUs by NCCL send/recv or
by the one-kernel exchange over NVLink peer memory, dA is all-reduced, and the result equals the single-GPU op on the whole sequence
within the bf16 tolerance.  Skipped where fewer than two GPUs are visible
(the host logic is also covered on CPU ranks by test_sp_gloo.py)."""

import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from _tol import assert_lowp_close
from oracle import ema_oracle as eo

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(600)]

B, L, H, P, Q = 2, 4096, 4, 64, 256


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, exchange, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                        "ema-kernels_b200"))
        from kernels.ema_chunk_scan import ema_chunk_scan_combined
        from kernels import ema_sp
        from kernels.ema_sp import ema_chunk_scan_sp

        x, dt, A, dy = eo.make_dt_inputs(B, L, H, P, seed=9)
        tx = torch.from_numpy(x).to(torch.bfloat16)
        tdy = torch.from_numpy(dy).to(torch.bfloat16)
        span = L // world
        sl = slice(rank * span, (rank + 1) * span)
        xs = tx[:, sl].contiguous().to(dev).requires_grad_()
        dts = torch.from_numpy(np.ascontiguousarray(dt[:, sl])).to(dev).requires_grad_()
        As = torch.from_numpy(A).to(dev).requires_grad_()
        ys = ema_chunk_scan_sp(xs, dts, As, Q, exchange=exchange)
        ys.backward(tdy[:, sl].contiguous().to(dev))
        torch.cuda.synchronize(dev)
        dist.barrier()

        # the whole sequence on this rank's GPU through the single-GPU op
        xf = tx.to(dev).requires_grad_()
        dtf = torch.from_numpy(dt).to(dev).requires_grad_()
        Af = torch.from_numpy(A).to(dev).requires_grad_()
        yf = ema_chunk_scan_combined(xf, dtf, Af, chunk_size=Q)
        yf.backward(tdy.to(dev))
        torch.cuda.synchronize(dev)
        assert_lowp_close(ys, yf[:, sl], f"rank {rank} y")
        assert_lowp_close(xs.grad, xf.grad[:, sl], f"rank {rank} dx")
        assert_lowp_close(dts.grad, dtf.grad[:, sl], f"rank {rank} ddt")
        assert_lowp_close(As.grad, Af.grad, f"rank {rank} dA")
        if exchange == "p2p":
            # the sequence's boundary values (rank 0's initial state, the last rank's
            # final-state gradient) through the one-kernel exchange against the chain
            g = torch.Generator().manual_seed(7)
            init = torch.randn(B, H, P, generator=g).to(dev)
            dfin = torch.randn(B, H, P, generator=g).to(dev)
            x0, dt0, A0 = xs.detach(), dts.detach(), As.detach()
            dy0 = tdy[:, sl].contiguous().to(dev)
            got = {}
            for ex in ("chain", "p2p"):
                y, st, Sin, fin = ema_sp.sp_forward(x0, dt0, A0, Q, initial_states=init, exchange=ex)
                dx, ddt, dA, d_init = ema_sp.sp_backward(x0, dt0, A0, st, dy0, Q, d_final_states=dfin,
                                                         need_d_initial=True, exchange=ex)
                got[ex] = (y, Sin, fin, dx, ddt, dA, d_init)
            torch.cuda.synchronize(dev)
            for name, a, b in zip(("y", "Sin", "final", "dx", "ddt", "dA", "d_init"), got["p2p"], got["chain"]):
                if b is None:
                    assert a is None, name
                    continue
                assert_lowp_close(a, b, f"rank {rank} p2p against chain: {name}")
            assert ema_sp.p2p_exchange_status() == 0, "a p2p exchange wait ran out"
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported through the queue; the exit code marks the failure too
        errq.put(f"rank {rank}: {e!r}")
        raise


@pytest.mark.parametrize("exchange", ["chain", "p2p"])
def test_sequence_parallel_two_gpus_matches_single_gpu(exchange):
    """exchange "p2p": the summary, exchange, fold and expansion as one kernel
    over NVLink peer memory (ema_span_exchange), also against the NCCL chain
    with the sequence's boundary values, and its wait status clear."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, exchange, errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not alive, "a rank did not finish"
    assert not errs, "\n".join(errs)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
