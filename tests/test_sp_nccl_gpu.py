"""Sequence-parallel EMA (kernels/ema_sp.py) on two GPUs over NCCL: each rank
runs the CUDA kernels on its span of the sequence, the span states (forward)
and span-end gradients (backward) cross between the GPUs by send/recv, dA is
all-reduced, and the result equals the single-GPU op on the whole sequence
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


def _worker(rank, world, port, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                        "ema-kernels_b200"))
        from kernels.ema_chunk_scan import ema_chunk_scan_combined
        from kernels.ema_sp import ema_chunk_scan_sp

        x, dt, A, dy = eo.make_dt_inputs(B, L, H, P, seed=9)
        tx = torch.from_numpy(x).to(torch.bfloat16)
        tdy = torch.from_numpy(dy).to(torch.bfloat16)
        span = L // world
        sl = slice(rank * span, (rank + 1) * span)
        xs = tx[:, sl].contiguous().to(dev).requires_grad_()
        dts = torch.from_numpy(np.ascontiguousarray(dt[:, sl])).to(dev).requires_grad_()
        As = torch.from_numpy(A).to(dev).requires_grad_()
        ys = ema_chunk_scan_sp(xs, dts, As, Q)
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
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported through the queue; the exit code marks the failure too
        errq.put(f"rank {rank}: {e!r}")
        raise


def test_sequence_parallel_two_gpus_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, errq)) for r in range(2)]
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
