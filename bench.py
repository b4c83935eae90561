"""Benchmark: EMA fwd+bwd Mtokens/s at B8 L4096 H32 P64 bf16 (chunk 256).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (config 2 of the benchmark spec): the dt-parameterised EMA
``h_t = exp(dt_t A_h) h_{t-1} + dt_t x_t`` forward + backward (dx, ddt, dA) on
seeded synthetic inputs -- x, dy ~ N(0,1) bf16; dt = softplus(N(0,1) + b_h) in
[1e-3, 1e-1]; A = -exp(U(0, log 16)).  A "step" is one forward and one
backward of the whole B8 L4096 batch through kernels.ema_chunk_scan.

Multi-GPU (one process per GPU under torchrun): ``value`` is STRONG scaling --
the global B8 batch is split by batch rows over the ranks (by heads where the
rows do not divide), no collective on the data path (the per-head dA partials
would join the model's gradient all-reduce, which this op does not own).
Extra keys on the same line: ``weak`` (every rank a whole B8 batch),
``sp_config4`` (config 4, one B1 L65536 sequence split over the ranks with
the NCCL state chain, and its error against the single-GPU op; at N > 1 also
``sp_config4_allgather``, the same with one all_gather per direction, and
``sp_config4_p2p``, the same with the exchange and both sub-span folds as one
kernel over NVLink peer memory) and
``ssd_config5`` (config 5, the Mamba-2 SSD at B32 L8192 H80 split by batch
rows); rank 0 adds ``bench_ema_total``, the reference's own benchmark
(ema_combined against its d_state-1 mamba_chunk_scan_combined call) on the
drop-ins at that benchmark's default shape.

Timing: ``value`` replays the step as ONE CUDA graph (dt transpose, forward,
backward) with inputs resident in HBM; before every step, outside the timed
interval, the L2 is flushed by a 256 MiB write followed by a 256 MiB read of
another buffer; CUDA events around each replay on the launching stream, summed
over exactly K steps; max over ranks.  The kernels of a step are launched with
programmatic dependent launch, so each one's launch overlaps the previous one's
tail; a second graph of the same step, with events captured between forward
and backward, splits it into the forward (transpose + ema_fwd_kernel) and the
backward (ema_bwd_kernel) for the per-kernel roofline.  ``e2e`` calls the public
autograd API eagerly: every step copies its inputs from pinned host memory
(the next step's copy overlapped with this step's compute) and reads back the
loss and dA, all inside the timed region.  ``cpu_baseline`` times the
reference's PyTorch CPU path (oracle/ema_torch_path.py) on one fixed sample
(one batch row at full length) on rank 0 at N=1; ``--impl reference`` times
the same sample per step.
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


def _profile_traffic(tokens=None):
    """DRAM bytes per backward launch from the committed ncu summary (captured on
    the whole config-2 batch), scaled to a launch over ``tokens`` tokens -- the
    traffic grows with the rows processed -- or None."""
    path = os.path.join(ROOT, "profiles", "ema_bwd_kernel_cfg2.md")
    try:
        txt = open(path).read()
    except OSError:
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", txt)
    if not m:
        return None
    return float(m.group(1)) * (1.0 if tokens is None else tokens / TOKENS)


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


CPU_SAMPLE = f"1 of the {B} batch rows at full length (L{L} H{H} P{P} bf16 = {L} tokens)"


def _ema_config(world, shard=None):
    """The workload description both arms print (the reference arm's is identical)."""
    return {"workload": WORKLOAD, "global_batch": B, "seq_len": L, "nheads": H, "headdim": P, "chunk_size": Q,
            "parallelism": f"batch x heads split over {world} GPU(s) (strong scaling), no collective",
            "l2": "flushed before every step outside the timed interval: 256 MiB write, then 256 MiB read "
                  "of another buffer; step inputs 272 MB > 126 MB L2"}


def _cpu_sample_seconds(reps, warm):
    """Seconds per fwd + autograd bwd of the reference's CPU path on the fixed sample:
    one batch row of the workload at full length, on all host threads."""
    from oracle import ema_torch_path as tp
    from oracle.ema_oracle import make_dt_inputs
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    x, dt, A, dy = make_dt_inputs(1, L, H, P, seed=99)
    tx = torch.from_numpy(x).to(torch.bfloat16)
    tdy = torch.from_numpy(dy).to(torch.bfloat16)
    tdt, tA = torch.from_numpy(dt), torch.from_numpy(A)
    for _ in range(warm):
        tp.dt_form_fwd_bwd(tx, tdt, tA, tdy)
    return tp.time_sample(tx, tdt, tA, tdy, reps=reps) / reps, cores


def _cpu_baseline():
    secs, cores = _cpu_sample_seconds(reps=3, warm=1)
    return {"value": L / secs / 1e6, "unit": "Mtokens/s", "cores": cores, "kind": "port",
            "sample": f"{CPU_SAMPLE}, fwd + autograd bwd of ema_torch_ref in torch on {cores} threads, "
                      f"1 warm-up + 3 timed passes, {secs:.2f} s per pass"}


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    steps = max(1, args.steps)
    warm = max(3, args.warmup)
    secs, cores = _cpu_sample_seconds(reps=steps, warm=warm)
    value = L / secs / 1e6
    sample = (f"per step {CPU_SAMPLE}: fwd + autograd bwd of ema_torch_ref in torch on {cores} threads "
              f"({warm} warm-up passes)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "Mtokens/s", "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": secs * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": _ema_config(world),
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
    """Config 4: one B1 L65536 H32 P64 sequence split over the ranks (strong
    scaling), fwd+bwd through kernels.ema_sp -- the same graph-timed step as the
    ``sp_config4`` leg of the default run (``--exchange`` picks the span exchange)."""
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    leg = _sp_leg(args, rank, world, dev, dist, exchange=args.exchange)
    if rank == 0:
        c = SP_CFG
        print(json.dumps({
            "metric": leg["metric"], "value": leg["value"], "unit": "Mtokens/s", "n_gpus": world,
            "steps": leg["steps"], "warmup": args.warmup, "ms_per_step": leg["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": "EMA dt-form fwd+bwd, one sequence split over the ranks", **c,
                       "span_per_rank": leg["span_per_rank"], "parallelism": leg["parallelism"],
                       "timing": leg["timing"]},
            "roofline": leg["roofline"], "max_rel_err_vs_single_gpu": leg["max_rel_err_vs_single_gpu"],
            # per step and direction: the column-sum state pass, the span summary fold (ranks > 1),
            # the expansion fold and the full pass (dt transpose + scan), or with "p2p" the
            # column sums, the exchange kernel and the full pass; the whole sequence as 32 chains
            # (no sub-spans): dt transpose + scan per direction
            "gpu_launches": leg["steps"] * _sp_launches_per_step(world, args.exchange),
        }), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def _tc_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return 1590.0



def _shard(world, rank):
    """Rows (or, where the rows do not divide, heads) of the global batch for this rank."""
    if B % world == 0:
        n = B // world
        return slice(rank * n, (rank + 1) * n), slice(0, H)
    if H % world == 0:
        n = H // world
        return slice(0, B), slice(rank * n, (rank + 1) * n)
    raise SystemExit(f"--gpus {world} divides neither the batch ({B}) nor the heads ({H})")


class StepGraph:
    """One step (dt transpose + forward, then the backward) captured twice.
    The timed graph holds only the kernels, so each kernel's launch and prologue
    overlap the previous kernel's tail (programmatic dependent launch).  The
    split graph has events captured between forward and backward -- an event
    there makes the backward wait for the forward in full -- and gives the
    per-kernel times of the same step."""

    def __init__(self, x, dt, A, dy, dev, fq=Q):
        from kernels.ema_chunk_scan import backward_chunk, ema_chunk_scan_bwd, ema_chunk_scan_fwd
        b_, l_, h_, _ = x.shape
        self.qb = backward_chunk(fq)  # what the autograd op runs: 128-token backward tiles on half-chunk states
        self.dtr = torch.empty(b_, h_, l_, dtype=torch.float32, device=dev)

        def fwd():
            return ema_chunk_scan_fwd(x, dt, A, fq, half_chunk_states=self.qb != fq, dt_rows=self.dtr)

        def bwd(states):
            return ema_chunk_scan_bwd(x, dt, A, states, dy, self.qb, dt_rows=self.dtr)

        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):  # eager warm-up: allocates this stream's workspace
            _, st, _ = fwd()
            bwd(st)
        side.synchronize()
        self.ev = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(3)]
        self.g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.g, stream=side):
            self.y, st, _ = fwd()
            self.grads = bwd(st)
        self.gs = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.gs, stream=side):
            self.ev[0].record()
            _, st, _ = fwd()
            self.ev[1].record()
            bwd(st)
            self.ev[2].record()
        torch.cuda.current_stream(dev).wait_stream(side)

    def run(self, K, W, flush, stream):
        """W untimed replays of each graph, K timed replays of the step graph,
        then K replays of the split graph; each replay after an L2 flush.
        Returns summed (step, forward, backward) milliseconds."""
        for _ in range(W):
            flush()
            self.g.replay()
            flush()
            self.gs.replay()
        torch.cuda.synchronize()
        tot = [0.0, 0.0, 0.0]
        for _ in range(K):
            flush()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            self.g.replay()
            e1.record(stream)
            e1.synchronize()
            tot[0] += e0.elapsed_time(e1)
        for _ in range(K):
            flush()
            self.gs.replay()
            self.ev[2].synchronize()
            tot[1] += self.ev[0].elapsed_time(self.ev[1])
            tot[2] += self.ev[1].elapsed_time(self.ev[2])
        return tot


def _max_over_ranks(vals, dev, dist):
    t = torch.tensor(vals, dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def _sp_launches_per_step(world, exchange="chain"):
    """This library's kernels per config-4 SP step (see run_sp)."""
    from kernels import ema_sp
    c = SP_CFG
    if world == 1 and ema_sp.subspan_count(c["B"], c["H"], c["L"], c["Q"], 1) == 1:
        return 4
    if world > 1 and exchange == "p2p":  # column sums, the exchange kernel, dt transpose, scan
        return 8
    return 2 * (4 + (world > 1))


def _sp_leg(args, rank, world, dev, dist, exchange="chain"):
    """Config 4: one B1 L65536 H32 P64 sequence split over the ranks (strong
    scaling) through kernels.ema_sp -- each rank's span cut into sub-spans run
    as batch rows: state-only pass, sub-span fold, span exchange (NCCL send/recv
    state chain, or one all_gather of the span summaries), local pass, dA
    all-reduce -- and its largest error against the single-GPU op on the whole
    sequence (normwise, max over ranks)."""
    import torch.distributed as tdist
    from kernels import ema_sp
    from kernels.ema_chunk_scan import ema_chunk_scan_bwd, ema_chunk_scan_fwd
    from oracle.ema_oracle import make_dt_inputs
    c = SP_CFG
    own_group = not tdist.is_initialized()
    if own_group:  # one rank: a local group so the span code runs unchanged
        tdist.init_process_group("gloo", store=tdist.HashStore(), rank=0, world_size=1)
    span = c["L"] // world
    x, dt, A, dy = make_dt_inputs(c["B"], c["L"], c["H"], c["P"], seed=21)
    fx = torch.from_numpy(x).to(torch.bfloat16).to(dev)
    fdy = torch.from_numpy(dy).to(torch.bfloat16).to(dev)
    fdt = torch.from_numpy(dt).to(dev)
    A = torch.from_numpy(A).to(dev)
    sl = slice(rank * span, (rank + 1) * span)
    xs, dys, dts = (t[:, sl].contiguous() for t in (fx, fdy, fdt))

    def step():
        y, states, _, _ = ema_sp.sp_forward(xs, dts, A, c["Q"], exchange=exchange)
        return (y,) + tuple(ema_sp.sp_backward(xs, dts, A, states, dys, c["Q"], exchange=exchange)[:3])

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    K = max(1, min(args.steps, 50))
    ms = 0.0
    with torch.cuda.stream(side):
        for _ in range(args.warmup):  # eager warm-up: communicators, workspaces
            out = step()
        side.synchronize()
        if world > 1:
            dist.barrier()
        g = torch.cuda.CUDAGraph()  # the step's kernels, sub-span folds and NCCL calls, replayed as one graph
        with torch.cuda.graph(g, stream=side):
            out = step()
        for _ in range(3):
            g.replay()
        side.synchronize()
        if world > 1:
            dist.barrier()
        for _ in range(K):
            flush.zero_()  # the L2, outside the timed interval
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(side)
            g.replay()
            e1.record(side)
            e1.synchronize()
            ms += e0.elapsed_time(e1)
        ms /= K
    torch.cuda.current_stream(dev).wait_stream(side)
    del g  # (a graph holding NCCL calls is released before the process group)
    # the single-GPU op on the whole sequence, this rank's span compared
    yr, st, _ = ema_chunk_scan_fwd(fx, fdt, A, c["Q"])
    dxr, ddtr, dAr, _ = ema_chunk_scan_bwd(fx, fdt, A, st, fdy, c["Q"])
    refs = (yr[:, sl], dxr[:, sl], ddtr[:, sl], dAr)
    errs = [float((o.float() - r.float()).abs().max() / r.float().abs().max().clamp_min(1e-30))
            for o, r in zip(out, refs)]
    ms, *errs = _max_over_ranks([ms] + errs, dev, dist if world > 1 else None)
    if own_group:
        tdist.destroy_process_group()
    tokens = c["B"] * c["L"]
    peak, _ = _peaks()
    gbs = BYTES_PER_TOKEN * tokens / (ms * 1e-3) / 1e9 / world
    return {"metric": "EMA fwd+bwd Mtokens/s, sequence parallel (config 4: B1 L65536 H32 P64 bf16)",
            "value": tokens / (ms * 1e-3) / 1e6, "unit": "Mtokens/s", "ms_per_step": ms, "steps": K,
            "scaling": "strong", "span_per_rank": span,
            "parallelism": (f"sequence parallel over {world} GPU(s): "
                            + {"chain": "NCCL send/recv state chain",
                               "allgather": "one NCCL all_gather of the span summaries per direction",
                               "p2p": "summary, exchange and expansion in one kernel over NVLink peer memory "
                                      "(ema_span_exchange) per direction"}[exchange] + " + dA all-reduce")
                           if world > 1 else (f"one GPU: the sequence cut into {ema_sp.subspan_count(c['B'], c['H'], c['L'], c['Q'], 1)} "
                                              "sub-spans run as batch rows, no exchange"),
            "roofline": {"bound": "hbm", "achieved_per_gpu": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak},
            "max_rel_err_vs_single_gpu": dict(zip(("y", "dx", "ddt", "dA"), errs)),
            "timing": "one CUDA graph per step (kernels, sub-span folds, NCCL calls), L2 flushed before each replay "
                      "outside the timed interval, CUDA events around each replay, max over ranks"}


SSD5_CFG = dict(B=32, L=8192, H=80, P=64, N=128, G=1)
SSD5_BYTES_PER_TOKEN = 10 * 80 * 64 + 12 * 1 * 128 + 12 * 80  # 53,696 B


def _ssd5_leg(args, rank, world, dev, dist):
    """Config 5: the Mamba-2 SSD fwd+bwd at B32 L8192 H80 P64 N128 (Mamba-2-2.7B
    layer shape), the global batch split by rows over the ranks (strong
    scaling), one CUDA graph per step, inputs larger than L2."""
    import math
    from kernels.ssd_combined import ssd_chunk_scan_bwd, ssd_chunk_scan_fwd
    c = SSD5_CFG
    if c["B"] % world:
        return {"unavailable": f"{world} ranks do not divide the batch of {c['B']}"}
    nb = c["B"] // world
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(500 + rank)
    shp = (nb, c["L"], c["H"])
    x = torch.randn(*shp, c["P"], generator=g, device=dev).to(bf)
    dy = torch.randn(*shp, c["P"], generator=g, device=dev).to(bf)
    bias = torch.log(torch.expm1(torch.exp(torch.rand(c["H"], generator=g, device=dev)
                                           * math.log(100.0) + math.log(1e-3))))
    dt = torch.clamp(torch.nn.functional.softplus(torch.randn(*shp, generator=g, device=dev) + bias), 1e-3, 1e-1)
    A = -torch.exp(torch.rand(c["H"], generator=g, device=dev) * math.log(16.0))
    Bm = (torch.randn(nb, c["L"], c["G"], c["N"], generator=g, device=dev) / math.sqrt(c["N"])).to(bf)
    Cm = (torch.randn(nb, c["L"], c["G"], c["N"], generator=g, device=dev) / math.sqrt(c["N"])).to(bf)
    D = torch.randn(c["H"], generator=g, device=dev)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        y, cst, _ = ssd_chunk_scan_fwd(x, dt, A, Bm, Cm, D)
        ssd_chunk_scan_bwd(x, dt, A, Bm, Cm, cst, dy, D)
        side.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=side):
            y, cst, _ = ssd_chunk_scan_fwd(x, dt, A, Bm, Cm, D)
            ssd_chunk_scan_bwd(x, dt, A, Bm, Cm, cst, dy, D)
        K = max(1, min(args.steps, 10))
        if dist is not None:
            dist.barrier()
        ms = _event_ms(gr.replay, K, 3, side)
    (ms,) = _max_over_ranks([ms / K], dev, dist)
    del gr
    tokens = c["B"] * c["L"]
    peak, _ = _peaks()
    gbs = SSD5_BYTES_PER_TOKEN * tokens / (ms * 1e-3) / 1e9 / world
    return {"metric": "SSD fwd+bwd Mtokens/s (config 5: B32 L8192 H80 P64 N128 G1 bf16)",
            "value": tokens / (ms * 1e-3) / 1e6, "unit": "Mtokens/s", "ms_per_step": ms, "steps": K,
            "scaling": "strong", "batch_per_gpu": nb,
            "parallelism": f"batch rows split over {world} GPU(s), no collective",
            "roofline": {"bound": "ridge (HBM figure)", "achieved_per_gpu": gbs, "peak": peak, "unit": "GB/s",
                         "frac": gbs / peak},
            "timing": "one CUDA graph per step (forward + backward), CUDA events, inputs > L2, max over ranks"}


TOTAL_CFG = dict(B=16, L=2048, H=32, P=64, Q=64)  # bench_ema_total.py's argparse defaults (:94-103)


def _ema_total_leg(dev, reps=20, warm=3):
    """The reference's own benchmark (kernels/benchmarks/bench_ema_total.py:38-91)
    on this repository's drop-ins, at its default shape (B16 L2048 H32 P64,
    chunk 64, bf16): ``run_combined`` = ema_combined fwd + bwd with A (B, L)
    shared over heads; ``run_mamba`` = mamba_chunk_scan_combined fwd + bwd
    called as it calls it (x / dt fp32, B = p, C = 1 of shape (B, L, 1, 1),
    A = -1: d_state 1).  Each rep is the eager call sequence the reference
    times (input clones, forward, loss, backward), CUDA events, median of reps."""
    from kernels.backward.ema_ssd_combined import ema_combined
    from kernels.ssd_combined import mamba_chunk_scan_combined
    c = TOTAL_CFG
    g = torch.Generator(device=dev).manual_seed(0)
    A = -torch.rand(c["B"], c["L"], generator=g, device=dev, dtype=torch.bfloat16)
    X = torch.randn(c["B"], c["L"], c["H"], c["P"], generator=g, device=dev, dtype=torch.bfloat16)
    dout = torch.randn(X.shape, generator=g, device=dev, dtype=torch.bfloat16)

    def run_combined():
        A_c = A.detach().clone().requires_grad_()
        X_c = X.detach().clone().requires_grad_()
        out = ema_combined(X_c, A_c, chunk_size=c["Q"])
        (out * dout).sum().backward()

    def run_mamba():
        p = torch.sigmoid(torch.randn((c["B"], c["L"], 1), generator=g, dtype=torch.bfloat16, device=dev))
        dt = -torch.log(1 - p).to(torch.float32).squeeze(-1).requires_grad_()
        X_beta = (X.reshape(c["B"], c["L"], c["H"] * c["P"]) / dt[..., None]).requires_grad_()
        X_m = X_beta.reshape(c["B"], c["L"], c["H"], c["P"])
        dt_m = dt[:, :, None].expand(c["B"], c["L"], c["H"])
        A_m = -1 * torch.ones(c["H"], dtype=torch.float32, device=dev, requires_grad=True)
        B_m = p.to(torch.float32)[..., None]
        C_m = torch.ones_like(B_m)
        out_m = mamba_chunk_scan_combined(X_m, dt_m, A_m, B_m, C_m, chunk_size=c["Q"], seq_idx=None)
        dout_m = torch.randn(out_m.shape, generator=g, dtype=out_m.dtype, device=dev)
        (out_m * dout_m).sum().backward()

    res = {}
    for name, fn in (("ema_combined_fwd_bwd_ms", run_combined), ("mamba_chunk_scan_combined_fwd_bwd_ms", run_mamba)):
        for _ in range(warm):
            fn()
        ts = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        res[name] = float(np.median(ts))
    tokens = c["B"] * c["L"]
    return {"config": {**c, "dtype": "bf16", "source": "kernels/benchmarks/bench_ema_total.py defaults"},
            **res, "ema_combined_mtok_s": tokens / res["ema_combined_fwd_bwd_ms"] / 1e3,
            "mamba_chunk_scan_combined_mtok_s": tokens / res["mamba_chunk_scan_combined_fwd_bwd_ms"] / 1e3,
            "timing": "eager calls as the reference times them (clones, forward, loss, backward), CUDA events, "
                      f"median of {reps} after {warm} warm-up; L2 not flushed (inputs 268 MB)"}


def run_ema(args, rank, world, local_rank):
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    from kernels import _lib
    from kernels.ema_chunk_scan import backward_chunk, ema_chunk_scan_bwd, ema_chunk_scan_fwd
    # tensor-core variants, for comparison (ema_set_tensor_core_path bits 0 / 1):
    # the tcgen05 backward on 128-token tiles; the tcgen05 forward on 128-token
    # tiles (it then runs at chunk 128, and the backward with it)
    FQ = 128 if args.ema_forward == "tc" else Q
    QB = backward_chunk(FQ)
    bwd_kernel = "ema_bwd_tc_kernel" if args.ema_backward == "tc" else "ema_bwd_kernel"
    fwd_kernel = "ema_fwd_tc_kernel" if args.ema_forward == "tc" else "ema_fwd_kernel"
    tc_bits = (1 if args.ema_backward == "tc" else 0) | (2 if args.ema_forward == "tc" else 0)
    if tc_bits:
        _lib.lib.ema_set_tensor_core_path(tc_bits)
    rows, heads = _shard(world, rank)
    hx, hdt, hA, hdy = _inputs(0, dev)  # the global batch (same seed on every rank), then this rank's part
    hx, hdy = hx[rows, :, heads].contiguous(), hdy[rows, :, heads].contiguous()
    hdt, hA = hdt[rows, :, heads].contiguous(), hA[heads].contiguous()
    x, dt, A, dy = (t.to(dev) for t in (hx, hdt, hA, hdy))
    tokens_rank = x.shape[0] * L * x.shape[2] / H  # token rows of this rank, in whole-head units
    if args.mode == "profile":
        dtr = torch.empty(x.shape[0], x.shape[2], L, dtype=torch.float32, device=dev)
        for _ in range(max(1, args.steps)):
            y, states, _ = ema_chunk_scan_fwd(x, dt, A, FQ, half_chunk_states=QB != FQ, dt_rows=dtr)
            ema_chunk_scan_bwd(x, dt, A, states, dy, QB, dt_rows=dtr)
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.destroy_process_group()
        return

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_rd = torch.ones(64 << 20, dtype=torch.float32, device=dev)  # 256 MiB, read to clean the L2

    def flush_l2():
        flush.zero_()
        flush_rd.sum()

    stream = torch.cuda.current_stream(dev)
    sg = StepGraph(x, dt, A, dy, dev, FQ)
    clocks = ClockSampler(local_rank)
    clocks.start()
    K = args.steps
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t_wall0 = time.time()
    step_ms, fwd_ms, bwd_ms = sg.run(K, args.warmup, flush_l2, stream)
    t_wall1 = time.time()
    clocks.window = (t_wall0, t_wall1)
    step_ms, fwd_ms, bwd_ms = _max_over_ranks([step_ms, fwd_ms, bwd_ms], dev, dist)
    clocks.stop()
    status = _lib.device_status()
    del sg

    weak = None
    if world > 1:  # every rank a whole B8 batch of its own
        wx, wdt, wA, wdy = (t.to(dev) for t in _inputs(rank, dev))
        wg = StepGraph(wx, wdt, wA, wdy, dev, FQ)
        if dist is not None:
            dist.barrier()
        (wms, _, _) = _max_over_ranks(wg.run(K, args.warmup, flush_l2, stream), dev, dist)
        weak = {"value": world * TOKENS / (wms / K * 1e-3) / 1e6, "unit": "Mtokens/s",
                "ms_per_step": wms / K, "batch_per_gpu": B, "scaling": "weak"}
        del wg, wx, wdt, wA, wdy

    # ---- end to end through the public API with host buffers --------------
    # Every step copies this rank's inputs (x, dt, A, dy) from pinned host
    # memory, runs forward + backward through the autograd op, and reads back
    # the step's result: the loss sum(y * dy) and the parameter gradient dA.
    # The copy of step k+1's inputs runs on a copy stream while step k computes
    # (two device input buffers), as a training loop's data loader would.
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
        yd = ema_chunk_scan_combined(xd, dtd, Ad, FQ)
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
    (e2e_ms,) = _max_over_ranks([e0.elapsed_time(e1) / E], dev, dist)
    del bufs

    sp = sp_ag = sp_p2p = ssd5 = total = None
    if not args.no_extra_legs:
        try:
            sp = _sp_leg(args, rank, world, dev, dist)
        except Exception as e:  # a leg's failure is reported, the headline line still prints
            sp = {"unavailable": f"{type(e).__name__}: {e}"}
        if world > 1:
            try:
                sp_ag = _sp_leg(args, rank, world, dev, dist, exchange="allgather")
            except Exception as e:
                sp_ag = {"unavailable": f"{type(e).__name__}: {e}"}
            try:
                sp_p2p = _sp_leg(args, rank, world, dev, dist, exchange="p2p")
            except Exception as e:
                sp_p2p = {"unavailable": f"{type(e).__name__}: {e}"}
        torch.cuda.empty_cache()
        try:
            ssd5 = _ssd5_leg(args, rank, world, dev, dist)
        except Exception as e:
            ssd5 = {"unavailable": f"{type(e).__name__}: {e}"}
        torch.cuda.empty_cache()
        if rank == 0:
            try:
                total = _ema_total_leg(dev)
            except Exception as e:
                total = {"unavailable": f"{type(e).__name__}: {e}"}

    if rank == 0:
        peak, peak_kind = _peaks()
        ms = step_ms / K
        value = TOKENS / (ms * 1e-3) / 1e6  # the whole global batch per step
        toks = tokens_rank  # algorithmic bytes of one launch on one rank
        bwd_launch_s = bwd_ms / K * 1e-3
        fwd_launch_s = fwd_ms / K * 1e-3
        bwd_gbs = BWD_BYTES_PER_TOKEN * toks / bwd_launch_s / 1e9
        fwd_gbs = FWD_BYTES_PER_TOKEN * toks / fwd_launch_s / 1e9
        step_gbs = BYTES_PER_TOKEN * toks / (ms * 1e-3) / 1e9
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = _cpu_baseline()
        cfg = _ema_config(world)
        cfg.update({"rows_per_gpu": hx.shape[0], "heads_per_gpu": hx.shape[2], "forward_chunk": FQ,
                    "backward_chunk": QB, "forward_kernel": fwd_kernel, "backward_kernel": bwd_kernel,
                    "timing": "one CUDA graph per step (dt transpose, forward, backward; programmatic "
                              "dependent launch between them); events around each replay on the launching "
                              "stream; the per-kernel split from a second graph of the same step with events "
                              "captured between forward and backward"})
        line = {
            "metric": METRIC, "value": value, "unit": "Mtokens/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": cfg,
            "roofline": {"bound": "hbm", "kernel": bwd_kernel, "achieved": bwd_gbs, "peak": peak,
                         "unit": "GB/s", "frac": bwd_gbs / peak,
                         "traffic": _profile_traffic(toks) if bwd_kernel == "ema_bwd_kernel" else None,
                         "algorithmic_bytes_per_launch": BWD_BYTES_PER_TOKEN * toks,
                         "launch_ms": bwd_launch_s * 1e3, "peak_source": f"{peak_kind} (hbm_gbs)"},
            "kernels": {f"forward (dt_rows_kernel + {fwd_kernel})": {"ms": fwd_launch_s * 1e3, "gbs": fwd_gbs,
                                                                     "frac": fwd_gbs / peak},
                        bwd_kernel: {"ms": bwd_launch_s * 1e3, "gbs": bwd_gbs, "frac": bwd_gbs / peak}},
            "step_roofline": {"algorithmic_bytes_per_step_per_gpu": BYTES_PER_TOKEN * toks, "achieved_gbs": step_gbs,
                              "frac": step_gbs / peak, "peak_source": peak_kind},
            "e2e": {"value": TOKENS / (e2e_ms * 1e-3) / 1e6, "unit": "Mtokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": E,
                    "api": "kernels.ema_chunk_scan.ema_chunk_scan_combined (autograd); each rank's inputs copied "
                           "from pinned host memory every step (next step's copy overlapped with this step's "
                           "compute), the loss and dA read back"},
            "gpu_launches": 3 * K,  # dt_rows_kernel + ema_fwd_kernel + ema_bwd_kernel per step
            "clocks": clocks.summary(),
            "device_status": status,
        }
        if weak is not None:
            line["weak"] = weak
        if sp is not None:
            line["sp_config4"] = sp
        if sp_ag is not None:
            line["sp_config4_allgather"] = sp_ag
        if sp_p2p is not None:
            line["sp_config4_p2p"] = sp_p2p
        if ssd5 is not None:
            line["ssd_config5"] = ssd5
        if total is not None:
            line["bench_ema_total"] = total
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra-legs", action="store_true",
                    help="skip the sequence-parallel config-4 and SSD config-5 legs of the line")
    ap.add_argument("--mode", choices=["bench", "profile"], default="bench",
                    help="profile: run --steps eager fwd+bwd steps and exit (for ncu captures)")
    ap.add_argument("--profile-batch", type=int, default=0,
                    help="with --mode profile --workload ssd: batch of the capture (default: the config's)")
    ap.add_argument("--ema-backward", choices=["scan", "tc"], default="scan",
                    help="EMA backward kernel: scan (CUDA-core scan, the default the autograd op runs) or tc "
                         "(the tcgen05 backward, ema_bwd_tc_kernel; for comparison)")
    ap.add_argument("--ema-forward", choices=["scan", "tc"], default="scan",
                    help="EMA forward kernel: scan (CUDA-core scan at chunk 256, the default) or tc (the tcgen05 "
                         "forward, ema_fwd_tc_kernel, at chunk 128; for comparison)")
    ap.add_argument("--exchange", choices=["chain", "allgather", "p2p"], default="chain",
                    help="with --workload sp: the span exchange (NCCL send/recv chain, one all_gather, or one "
                         "kernel over NVLink peer memory)")
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

    run_ema(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
