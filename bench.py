"""Benchmark: EMA fwd+bwd Mtokens/s at B8 L4096 H32 P64 bf16 (chunk 256), one B200 per rank.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (config 2 of the benchmark spec): the dt-parameterised EMA
``h_t = exp(dt_t A_h) h_{t-1} + dt_t x_t`` forward + backward (dx, ddt, dA) on
seeded synthetic inputs -- x, dy ~ N(0,1) bf16; dt = softplus(N(0,1) + b_h) in
[1e-3, 1e-1]; A = -exp(U(0, log 16)).  A "step" is one forward and one
backward through the public API (kernels.ema_chunk_scan).

Multi-GPU: one process per GPU (torchrun), each rank processes its own
B8 L4096 H32 P64 batch (weak scaling: batch x heads shard with no data-path
collective; the per-head dA partials would join the model's gradient
all-reduce, which this op does not own).

Timing: ``value`` replays the step as two CUDA graphs (forward, backward) with
inputs resident in HBM; before every step, outside the timed intervals, the L2
is flushed by a 256 MiB write followed by a 256 MiB read of another buffer (so
the timed step neither hits its own data in L2 nor pays for writing back the
flush's dirty lines); CUDA events on the launching stream, summed over exactly
K steps; max over ranks.  Each step launches exactly two kernels of this
library (ema_fwd_kernel, ema_bwd_kernel).  ``e2e`` calls the public
API eagerly: every step copies its inputs from pinned host memory (the next
step's copy overlapped with this step's compute) and reads back the loss and
dA, all inside the timed region.  ``cpu_baseline`` times the reference's PyTorch CPU path
(oracle/ema_torch_path.py) on a bounded sample on rank 0 at N=1.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import re
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ema-kernels_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

B, L, H, P, Q = 8, 4096, 32, 64, 256
TOKENS = B * L
# minimum HBM bytes per token of one forward + backward (x read twice, y, dy, dx
# once in bf16; dt read twice and ddt written once in fp32)
BYTES_PER_TOKEN = 10 * H * P + 12 * H
FWD_BYTES_PER_TOKEN = 4 * H * P + 4 * H       # x, dt read; y written
BWD_BYTES_PER_TOKEN = 6 * H * P + 8 * H       # x, dy, dt read; dx, ddt written
METRIC = "EMA-SSD fwd+bwd Mtokens/s (B8 L4096 H32 P64 bf16) and % of HBM roofline"
WORKLOAD = "EMA dt-form fwd+bwd, B8 L4096 H32 P64, chunk 256, bf16 I/O, fp32 accumulation"
FALLBACK_HBM_GBS = 6650.0


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def _profile_traffic():
    """DRAM bytes per backward launch from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "ema_bwd_kernel_cfg2.md")
    try:
        txt = open(path).read()
    except OSError:
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", txt)
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.samples = []
        self._proc = None
        self._thr = None
        self.window = None

    def start(self):
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self._proc = None
            return
        self._thr = threading.Thread(target=self._read, daemon=True)
        self._thr.start()

    def _read(self):
        for line in self._proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append((time.time(), parts))

    def stop(self):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sel = self.samples
        if self.window is not None:
            w = [s for s in self.samples if self.window[0] <= s[0] <= self.window[1]]
            if w:
                sel = w

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None

        sm = [num(p[1]) for _, p in sel if num(p[1]) is not None]
        mx = [num(p[2]) for _, p in sel if num(p[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, p in sel for i in range(4) if p[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sel)}


def _inputs(rank, device, dtype=torch.bfloat16):
    from oracle.ema_oracle import make_dt_inputs
    x, dt, A, dy = make_dt_inputs(B, L, H, P, seed=1234 + rank)
    return (torch.from_numpy(x).to(dtype), torch.from_numpy(dt), torch.from_numpy(A),
            torch.from_numpy(dy).to(dtype))


def _cpu_baseline():
    """The reference's CPU path (ema_torch_ref + autograd) on one batch row of the
    workload at full length: L4096 H32 P64 bf16 = 4096 tokens."""
    from oracle import ema_torch_path as tp
    from oracle.ema_oracle import make_dt_inputs
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    x, dt, A, dy = make_dt_inputs(1, L, H, P, seed=99)
    tx = torch.from_numpy(x).to(torch.bfloat16)
    tdy = torch.from_numpy(dy).to(torch.bfloat16)
    secs = tp.time_sample(tx, torch.from_numpy(dt), torch.from_numpy(A), tdy)
    return {"value": L / secs / 1e6, "unit": "Mtokens/s", "cores": cores, "kind": "port",
            "sample": f"1 of the {B} batch rows at full length (L{L} H{H} P{P} bf16 = {L} tokens), "
                      f"fwd + autograd bwd of ema_torch_ref in torch on {cores} threads, {secs:.1f} s"}


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    steps = max(1, args.steps)
    warm = 3  # the contract's minimum; each step is a bounded sample
    from oracle import ema_torch_path as tp
    from oracle.ema_oracle import make_dt_inputs
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    # each step: fwd+bwd of a bounded sample of the workload -- one batch row
    # (all heads) over Ls tokens, Ls sized so warm-up + K steps take ~2 minutes
    def sample(n):
        x, dt, A, dy = make_dt_inputs(1, n, H, P, seed=7)
        return (torch.from_numpy(x).to(torch.bfloat16), torch.from_numpy(dt), torch.from_numpy(A),
                torch.from_numpy(dy).to(torch.bfloat16))

    t_probe = tp.time_sample(*sample(256))
    budget = 120.0 / (steps + warm)
    Ls = int(min(L, max(64, 256 * budget / max(t_probe, 1e-6))) // 64 * 64)
    tx, tdt, tA, tdy = sample(Ls)
    for _ in range(warm):
        tp.dt_form_fwd_bwd(tx, tdt, tA, tdy)
    secs = tp.time_sample(tx, tdt, tA, tdy, reps=steps)
    value = steps * Ls / secs / 1e6
    sample = (f"per step 1 batch row x L{Ls} (H{H} P{P} bf16, {Ls} tokens) of the workload: fwd + "
              f"autograd bwd of ema_torch_ref in torch on {cores} threads")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "Mtokens/s", "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": secs / steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample_tokens_per_step": Ls},
        "cpu_baseline": {"value": value, "unit": "Mtokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "Mtokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def _event_ms(fn, K, warmup, stream, flush=None):
    """K timed calls of fn() on `stream` (CUDA events around each), after warm-up."""
    for _ in range(warmup):
        if flush is not None:
            flush()
        fn()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    for k in range(K):
        if flush is not None:
            flush()
        ev[k][0].record(stream)
        fn()
        ev[k][1].record(stream)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in ev)


SSD_CFG = dict(B=8, L=4096, H=64, P=64, N=128, G=1)
# minimum HBM bytes per token of SSD fwd+bwd (bf16 x, y, dy, dx: 10 H P; B, C read twice and dB, dC
# written, fp32 gradients: 12 G N; dt read twice, ddt written: 12 H) -- 43,264 B at config 3
SSD_BYTES_PER_TOKEN = 10 * 64 * 64 + 12 * 1 * 128 + 12 * 64
# tensor-core flops per token of the chunked algorithm at 64-token chunks (fwd: C B^T, M x, C s^T,
# x^T B; bwd: the nine contractions of ssd_bwd_kernel, state operands counted twice for the split)
SSD_FLOPS_PER_TOKEN = 2 * 64 * (64 * 128 + 64 * 64 + 128 * 64 + 64 * 128) + \
    2 * 64 * (64 * 128 + 64 * 64 + 64 * 64 + 2 * 128 * 64 + 64 * 128 + 64 * 64 + 64 * 128 + 2 * 64 * 128 + 2 * 64 * 128)


def run_ssd(args, rank, world, local_rank):
    """Config 3 (Mamba-2 SSD) fwd+bwd per rank; batch x heads shard with no collective."""
    from oracle import ssd_oracle as so
    from kernels.ssd_combined import ssd_chunk_scan_bwd, ssd_chunk_scan_fwd
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    c = dict(SSD_CFG)
    if args.mode == "profile" and args.profile_batch:
        c["B"] = args.profile_batch  # a smaller capture of the same per-head work
    x, dt, A, Bm, Cm, D, dy = so.make_ssd_inputs(c["B"], c["L"], c["H"], c["P"], c["N"], c["G"], seed=11 + rank)
    bf = lambda a: torch.from_numpy(a).to(torch.bfloat16).to(dev)  # noqa: E731
    x, Bm, Cm, dy = bf(x), bf(Bm), bf(Cm), bf(dy)
    dt, A, D = (torch.from_numpy(a).to(dev) for a in (dt, A, D))
    if args.mode == "profile":
        for _ in range(max(1, args.steps)):
            y, cst, _ = ssd_chunk_scan_fwd(x, dt, A, Bm, Cm, D)
            ssd_chunk_scan_bwd(x, dt, A, Bm, Cm, cst, dy, D)
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.destroy_process_group()
        return
    side = torch.cuda.Stream(dev)
    with torch.cuda.stream(side):
        y, cst, _ = ssd_chunk_scan_fwd(x, dt, A, Bm, Cm, D)
        ssd_chunk_scan_bwd(x, dt, A, Bm, Cm, cst, dy, D)
        side.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            y, cst, _ = ssd_chunk_scan_fwd(x, dt, A, Bm, Cm, D)
            ssd_chunk_scan_bwd(x, dt, A, Bm, Cm, cst, dy, D)
        K = max(1, min(args.steps, 50))
        clocks = ClockSampler(local_rank)
        clocks.start()
        if dist is not None:
            dist.barrier()
        t0 = time.time()
        ms = _event_ms(g.replay, K, args.warmup, side)
        t1 = time.time()
    clocks.window = (t0, t1)
    clocks.stop()
    tm = torch.tensor([ms], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
    ms = float(tm.item()) / K
    if rank == 0:
        peak, kind = _peaks()
        tflops_peak = _tc_peak()
        tokens = c["B"] * c["L"]
        gbs = SSD_BYTES_PER_TOKEN * tokens / (ms * 1e-3) / 1e9
        tfl = SSD_FLOPS_PER_TOKEN * tokens / (ms * 1e-3) / 1e12
        print(json.dumps({
            "metric": "SSD fwd+bwd Mtokens/s (config 3: B8 L4096 H64 P64 N128 G1 bf16)",
            "value": world * tokens / (ms * 1e-3) / 1e6, "unit": "Mtokens/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "Mamba-2 SSD fwd+bwd (config 3)", **c,
                       "kernels": "forward: tcgen05/TMEM, 128-token chunks, 2 heads per CTA; "
                                  "backward: tcgen05/TMEM, 64-token chunks, 1 head per CTA",
                       "l2": "step inputs 1.4 GB > 126 MB L2, no flush", "timing": "one CUDA graph per step"},
            "roofline": {"bound": "ridge", "hbm": {"achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak},
                         "tensor": {"achieved": tfl, "peak": tflops_peak, "unit": "TFLOP/s",
                                    "frac": tfl / tflops_peak, "flops_per_token": SSD_FLOPS_PER_TOKEN}},
            "gpu_launches": 2 * K, "clocks": clocks.summary(),
            "cpu_baseline": {"value": None, "unit": "Mtokens/s", "cores": 0, "kind": "port",
                             "sample": "none in the reference (SSD is the absent mamba_ssm package)"},
        }), flush=True)
    del g
    if dist is not None:
        dist.destroy_process_group()


SP_CFG = dict(B=1, L=65536, H=32, P=64, Q=256)


def run_sp(args, rank, world, local_rank):
    """Config 4: one B1 L65536 H32 P64 sequence split over the ranks (strong scaling);
    fwd+bwd through kernels.ema_sp (state-only pass, NCCL send/recv chain, local pass)."""
    from oracle.ema_oracle import make_dt_inputs
    from kernels import ema_sp
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    import torch.distributed as dist
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    else:
        dist.init_process_group("gloo", store=dist.HashStore(), rank=0, world_size=1)
    c = SP_CFG
    span = c["L"] // world
    x, dt, A, dy = make_dt_inputs(c["B"], c["L"], c["H"], c["P"], seed=21)
    sl = slice(rank * span, (rank + 1) * span)
    x = torch.from_numpy(np.ascontiguousarray(x[:, sl])).to(torch.bfloat16).to(dev)
    dy = torch.from_numpy(np.ascontiguousarray(dy[:, sl])).to(torch.bfloat16).to(dev)
    dt = torch.from_numpy(np.ascontiguousarray(dt[:, sl])).to(dev)
    A = torch.from_numpy(A).to(dev)
    def step():
        y, states, Sin, _ = ema_sp.sp_forward(x, dt, A, c["Q"])
        ema_sp.sp_backward(x, dt, A, states, dy, c["Q"])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    K = max(1, min(args.steps, 200))
    dist.barrier()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / K], dtype=torch.float64, device=dev if world > 1 else "cpu")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    if rank == 0:
        peak, _ = _peaks()
        tokens = c["B"] * c["L"]
        gbs = BYTES_PER_TOKEN * tokens / (ms * 1e-3) / 1e9
        print(json.dumps({
            "metric": "EMA fwd+bwd Mtokens/s, sequence parallel (config 4: B1 L65536 H32 P64 bf16)",
            "value": tokens / (ms * 1e-3) / 1e6, "unit": "Mtokens/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "EMA dt-form fwd+bwd, one sequence split over the ranks", **c,
                       "span_per_rank": span, "parallelism": f"sequence parallel over {world} GPU(s), "
                       "NCCL send/recv state chain + dA all-reduce",
                       "timing": "eager calls, CUDA events around K steps, max over ranks"},
            "roofline": {"bound": "hbm", "achieved": gbs / world, "peak": peak, "unit": "GB/s",
                         "frac": gbs / world / peak,
                         "note": "per-GPU algorithmic bytes of one fwd+bwd (the state-only passes "
                                 "re-read x and dy)"},
            "gpu_launches": K * (4 if world > 1 else 2),  # state-only passes only when split
        }), flush=True)
    dist.destroy_process_group()


def _tc_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return 1590.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--mode", choices=["bench", "profile"], default="bench",
                    help="profile: run --steps eager fwd+bwd steps and exit (for ncu captures)")
    ap.add_argument("--profile-batch", type=int, default=0,
                    help="with --mode profile --workload ssd: batch of the capture (default: the config's)")
    ap.add_argument("--workload", choices=["ema", "ssd", "sp"], default="ema",
                    help="ema: config 2 (the headline); ssd: config 3 (Mamba-2 SSD B8 L4096 H64 P64 N128 G1); "
                         "sp: config 4 (EMA B1 L65536 H32 P64, the sequence split over the ranks)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference":
        if args.workload != "ema":
            if rank == 0:
                print(json.dumps({"impl": "reference", "workload": args.workload,
                                  "unavailable": "the reference has no CPU path for this workload "
                                                 "(SSD is the absent mamba_ssm package; SP is not in the reference)"}))
            return
        run_reference_arm(args, rank, world)
        return
    if args.workload == "ssd":
        run_ssd(args, rank, world, local_rank)
        return
    if args.workload == "sp":
        run_sp(args, rank, world, local_rank)
        return

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    from kernels import _lib
    from kernels.ema_chunk_scan import backward_chunk, ema_chunk_scan_bwd, ema_chunk_scan_fwd
    QB = backward_chunk(Q)  # what the autograd op runs: 128-token backward tiles on half-chunk states

    hx, hdt, hA, hdy = _inputs(rank, dev)
    x, dt, A, dy = (t.to(dev) for t in (hx, hdt, hA, hdy))
    # dt transposed to (B, H, L) by the forward launch and read by the backward,
    # as the autograd op does (ctx saves it)
    dtr = torch.empty(x.shape[0], H, L, dtype=torch.float32, device=dev)
    if args.mode == "profile":
        for _ in range(max(1, args.steps)):
            y, states, _ = ema_chunk_scan_fwd(x, dt, A, Q, half_chunk_states=QB != Q, dt_rows=dtr)
            ema_chunk_scan_bwd(x, dt, A, states, dy, QB, dt_rows=dtr)
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.destroy_process_group()
        return

    # eager warm-up (allocates the workspace of this stream), then two graphs
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        y, states, _ = ema_chunk_scan_fwd(x, dt, A, Q, half_chunk_states=QB != Q, dt_rows=dtr)
        ema_chunk_scan_bwd(x, dt, A, states, dy, QB, dt_rows=dtr)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    g_fwd, g_bwd = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_fwd, stream=side):
        y, states, _ = ema_chunk_scan_fwd(x, dt, A, Q, half_chunk_states=QB != Q, dt_rows=dtr)
    with torch.cuda.graph(g_bwd, pool=g_fwd.pool(), stream=side):
        dx, ddt, dA, _ = ema_chunk_scan_bwd(x, dt, A, states, dy, QB, dt_rows=dtr)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_rd = torch.ones(64 << 20, dtype=torch.float32, device=dev)  # 256 MiB, read to clean the L2

    def flush_l2():
        flush.zero_()
        flush_rd.sum()

    clocks = ClockSampler(local_rank)
    clocks.start()
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        flush_l2()
        g_fwd.replay()
        g_bwd.replay()
    K = args.steps
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t_wall0 = time.time()
    for k in range(K):
        flush_l2()
        ev[k][0].record(stream)
        g_fwd.replay()
        ev[k][1].record(stream)
        g_bwd.replay()
        ev[k][2].record(stream)
    torch.cuda.synchronize(dev)
    t_wall1 = time.time()
    if dist is not None:
        dist.barrier()
    clocks.window = (t_wall0, t_wall1)
    fwd_ms = sum(e[0].elapsed_time(e[1]) for e in ev)
    bwd_ms = sum(e[1].elapsed_time(e[2]) for e in ev)
    step_ms = sum(e[0].elapsed_time(e[2]) for e in ev)
    tm = torch.tensor([step_ms, fwd_ms, bwd_ms], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
    step_ms, fwd_ms, bwd_ms = (float(v) for v in tm.tolist())
    clocks.stop()
    status = _lib.device_status()

    # ---- end to end through the public API with host buffers --------------
    # Every step copies its inputs (x, dt, A, dy: 272 MB) from pinned host memory,
    # runs forward + backward through the autograd op, and reads back the step's
    # result: the loss sum(y * dy) and the parameter gradient dA.  The copy of
    # step k+1's inputs runs on a copy stream while step k computes (two device
    # input buffers), as a training loop's data loader would.
    from kernels.ema_chunk_scan import ema_chunk_scan_combined
    px, pdt, pA, pdy = (t.pin_memory() for t in (hx, hdt, hA, hdy))
    out_loss = torch.empty(1, dtype=torch.float32).pin_memory()
    out_dA = torch.empty(hA.shape, dtype=torch.float32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in (px, pdt, pA, pdy))
    d2h = sum(t.numel() * t.element_size() for t in (out_loss, out_dA))
    copy_stream = torch.cuda.Stream(dev)
    bufs = [[torch.empty_like(t, device=dev) for t in (px, pdt, pA, pdy)] for _ in range(2)]
    loaded = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]

    def h2d_copy(k):
        i = k % 2
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(consumed[i])
            for dst, src in zip(bufs[i], (px, pdt, pA, pdy)):
                dst.copy_(src, non_blocking=True)
            loaded[i].record(copy_stream)

    def e2e_step(k):
        i = k % 2
        stream.wait_event(loaded[i])
        xd, dtd, Ad, dyd = bufs[i]
        xd = xd.detach().requires_grad_()
        dtd = dtd.detach().requires_grad_()
        Ad = Ad.detach().requires_grad_()
        yd = ema_chunk_scan_combined(xd, dtd, Ad, Q)
        yd.backward(dyd)
        loss = (yd.detach().float() * dyd.float()).sum()
        consumed[i].record(stream)
        out_loss.copy_(loss.reshape(1), non_blocking=True)
        out_dA.copy_(Ad.grad, non_blocking=True)

    for i in range(2):
        consumed[i].record(stream)
    h2d_copy(0)
    for k in range(2):
        h2d_copy(k + 1)
        e2e_step(k)
    torch.cuda.synchronize(dev)
    E = max(1, args.e2e_steps)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0.record(stream)
    copy_stream.wait_stream(stream)
    h2d_copy(0)
    for k in range(E):
        if k + 1 < E:
            h2d_copy(k + 1)
        e2e_step(k)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / E], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
        dist.barrier()
    e2e_ms = float(e2e_ms.item())

    if rank == 0:
        peak, peak_kind = _peaks()
        ms = step_ms / K
        value = world * TOKENS / (ms * 1e-3) / 1e6
        bwd_launch_s = bwd_ms / K * 1e-3
        fwd_launch_s = fwd_ms / K * 1e-3
        bwd_gbs = BWD_BYTES_PER_TOKEN * TOKENS / bwd_launch_s / 1e9
        fwd_gbs = FWD_BYTES_PER_TOKEN * TOKENS / fwd_launch_s / 1e9
        step_gbs = BYTES_PER_TOKEN * TOKENS / (ms * 1e-3) / 1e9
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = _cpu_baseline()
        line = {
            "metric": METRIC, "value": value, "unit": "Mtokens/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "batch_per_gpu": B, "global_batch": B * world, "seq_len": L,
                       "nheads": H, "headdim": P, "chunk_size": Q, "backward_chunk": QB,
                       "parallelism": f"batch x heads sharded over {world} GPU(s), no collective",
                       "l2": "flushed before every step outside the timed intervals: 256 MiB write, then "
                             "256 MiB read of another buffer; step inputs 272 MB > 126 MB L2",
                       "timing": "two CUDA graphs per step (fwd, bwd), events on the launching stream"},
            "roofline": {"bound": "hbm", "kernel": "ema_bwd_kernel", "achieved": bwd_gbs, "peak": peak,
                         "unit": "GB/s", "frac": bwd_gbs / peak, "traffic": _profile_traffic(),
                         "algorithmic_bytes_per_launch": BWD_BYTES_PER_TOKEN * TOKENS,
                         "launch_ms": bwd_launch_s * 1e3, "peak_source": f"{peak_kind} (hbm_gbs)"},
            "kernels": {"ema_fwd_kernel": {"ms": fwd_launch_s * 1e3, "gbs": fwd_gbs, "frac": fwd_gbs / peak},
                        "ema_bwd_kernel": {"ms": bwd_launch_s * 1e3, "gbs": bwd_gbs, "frac": bwd_gbs / peak}},
            "step_roofline": {"algorithmic_bytes_per_step": BYTES_PER_TOKEN * TOKENS, "achieved_gbs": step_gbs,
                              "frac": step_gbs / peak, "peak_source": peak_kind},
            "e2e": {"value": world * TOKENS / (e2e_ms * 1e-3) / 1e6, "unit": "Mtokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": E,
                    "api": "kernels.ema_chunk_scan.ema_chunk_scan_combined (autograd); inputs copied from "
                           "pinned host memory every step (next step's copy overlapped with this step's "
                           "compute), the loss and dA read back"},
            "gpu_launches": 3 * K,  # dt_rows_kernel + ema_fwd_kernel + ema_bwd_kernel per step
            "clocks": clocks.summary(),
            "device_status": status,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    del g_fwd, g_bwd
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
