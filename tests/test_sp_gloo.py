"""Sequence-parallel host logic (kernels/ema_sp.py) on CPU ranks over gloo.

Each rank owns one span of the sequence, cut into sub-spans run as batch rows;
the local passes are the float64 oracle and the sub-span folds the float64
torch restatement (tests/_sp_fold_ref.py) instead of the CUDA kernels, so what
is tested is the sub-span bookkeeping, the span chaining
(send/recv order, the span decay, the incoming state and the gradient at the
span end -- through the send/recv chain and through one all_gather of the span
summaries) and the dA all-reduce.  The spans' results must equal the oracle on
the whole sequence up to the fp32 rounding of the exchanged (B, H, P) states.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ema_oracle as eo

pytestmark = pytest.mark.timeout(300)

B, L, H, P, Q = 2, 384, 3, 8, 64


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _np(t):
    return t.detach().to(torch.float64).numpy()


# oracle-backed local passes with the signatures kernels/ema_sp.py injects
def _state_fwd(x, dt, A, chunk_size):
    return torch.from_numpy(eo.ema_dt_fwd(_np(x), _np(dt), _np(A))["final_state"])


def _local_fwd(x, dt, A, chunk_size, initial_states):
    r = eo.ema_dt_fwd(_np(x), _np(dt), _np(A), initial_state=_np(initial_states))
    # the oracle's backward restarts from the span's incoming state, which
    # stands in for the chunk start states the kernels save
    return torch.from_numpy(r["y"]), initial_states.clone(), torch.from_numpy(r["final_state"])


def _state_bwd(x, dt, A, states, dy, chunk_size):
    r = eo.ema_dt_bwd(_np(x), _np(dt), _np(A), _np(dy), initial_state=_np(states))
    return torch.from_numpy(r["d_initial_state"])


def _local_bwd(x, dt, A, states, dy, chunk_size, d_final_states, need_d_initial):
    r = eo.ema_dt_bwd(_np(x), _np(dt), _np(A), _np(dy), initial_state=_np(states),
                      d_final_state=_np(d_final_states))
    d_init = torch.from_numpy(r["d_initial_state"]) if need_d_initial else None
    return torch.from_numpy(r["dx"]), torch.from_numpy(r["ddt"]), torch.from_numpy(r["dA"]), d_init


def _worker(rank, world, port, with_init, exchange, subspans, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import sys
        sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                        "ema-kernels_b200"))
        from kernels import ema_sp

        x, dt, A, dy = eo.make_dt_inputs(B, L, H, P, seed=5)
        rng = np.random.default_rng(6)
        init = rng.standard_normal((B, H, P)) if with_init else None
        dfin = rng.standard_normal((B, H, P)) if with_init else None
        full_f = eo.ema_dt_fwd(x, dt, A, initial_state=init)
        full_b = eo.ema_dt_bwd(x, dt, A, dy, initial_state=init, d_final_state=dfin)

        span = L // world
        sl = slice(rank * span, (rank + 1) * span)
        tx, tdt, tdy = (torch.from_numpy(np.ascontiguousarray(a[:, sl])) for a in (x, dt, dy))
        tA = torch.from_numpy(A)
        tinit = torch.from_numpy(init) if init is not None else None
        from _sp_fold_ref import torch_fold
        y, states, Sin, final = ema_sp.sp_forward(tx, tdt, tA, Q, initial_states=tinit,
                                                  state_fwd=_state_fwd, local_fwd=_local_fwd, exchange=exchange,
                                                  subspans=subspans, fold=torch_fold)
        np.testing.assert_allclose(_np(y), full_f["y"][:, sl], rtol=1e-5, atol=1e-6)
        if rank == world - 1:
            np.testing.assert_allclose(_np(final), full_f["final_state"], rtol=1e-5, atol=1e-6)

        tdfin = torch.from_numpy(dfin) if dfin is not None else None
        dx, ddt, dA, d_init = ema_sp.sp_backward(tx, tdt, tA, states, tdy, Q, d_final_states=tdfin,
                                                 need_d_initial=True, state_bwd=_state_bwd,
                                                 local_bwd=_local_bwd, exchange=exchange, fold=torch_fold)
        np.testing.assert_allclose(_np(dx), full_b["dx"][:, sl], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(_np(ddt), full_b["ddt"][:, sl], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(_np(dA), full_b["dA"], rtol=1e-5, atol=1e-6)
        if rank == 0:
            np.testing.assert_allclose(_np(d_init), full_b["d_initial_state"], rtol=1e-5, atol=1e-6)
        else:
            assert d_init is None
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent, which fails the test
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


# subspans: None = the automatic choice (here 2 or 1 sub-spans per rank's span);
# world 1 with sub-spans: one GPU's sequence cut into sub-spans, nothing exchanged
@pytest.mark.parametrize("world,with_init,exchange,subspans", [
    (2, False, "chain", None), (3, True, "chain", None), (3, True, "allgather", None), (4, False, "allgather", None),
    (2, True, "chain", 4), (3, True, "allgather", 2), (2, True, "allgather", 3),
    (1, True, "chain", 4), (1, False, "allgather", 3)])
def test_sequence_parallel_matches_whole_sequence(world, with_init, exchange, subspans):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(world, _free_port(), with_init, exchange, subspans, errq), nprocs=world,
                       join=True,
                       start_method="spawn")
    assert errq.empty(), errq.get()


def test_span_decay_composes():
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "ema-kernels_b200"))
    from kernels.ema_sp import span_decay

    x, dt, A, _ = eo.make_dt_inputs(1, 128, 2, 4, seed=3)
    D = span_decay(torch.from_numpy(dt), torch.from_numpy(A)).double().numpy()
    np.testing.assert_allclose(D, np.exp(dt.sum(1) * A), rtol=1e-6)


def test_subspan_counts_at_config_4():
    """The sub-span rule at config 4 (B1 L65536 H32, chunk 256): 16 on one GPU,
    32 / 16 / 8 per rank over 2 / 4 / 8 ranks; config 2 (B8 L4096) on one GPU
    runs whole."""
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "ema-kernels_b200"))
    from kernels.ema_sp import subspan_count

    assert subspan_count(1, 32, 65536, 256, 1) == 16
    assert [subspan_count(1, 32, 65536 // r, 256, r) for r in (2, 4, 8)] == [32, 16, 8]
    assert subspan_count(8, 32, 4096, 256, 1) == 1
