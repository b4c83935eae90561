"""Generate golden fixtures from the reference's own EMA kernels (run by hand, on CPU).

The reference (kartiksrinivas007/ema-kernels) is Python/Triton.  Its kernels run
on the CPU under the Triton interpreter (``TRITON_INTERPRET=1``) in float32
after three mechanical edits to a throw-away copy, none of which touches the
arithmetic:

1. the ``x.is_cuda`` / ``dA.is_cuda`` asserts become ``pass``
   (kernels/forward/ema_ssd_fwd.py:441-442, :188; ema_ssd_combined.py:82);
2. the TMA scratch allocator allocates on ``cpu`` instead of ``cuda``
   (ema_ssd_fwd.py:404, ema_ssd_bwd.py:19, ema_ssd_combined.py:23);
3. the ``chunk_size in [64, 128]`` assert becomes ``pass`` so chunk 256 runs
   (ema_ssd_fwd.py:439).

The copy lives in a temporary directory and is deleted afterwards; nothing of
the reference is written into this repository except the numeric outputs in
``tests/golden/*.npz``.  bf16 is not generated: the interpreter's bf16 ``dot``
is not meaningful, so fixtures are float32 and bf16 parity is checked against
the float64 oracle instead.

Usage:  python tests/golden/make_golden.py [--reference PATH]
"""

from __future__ import annotations

import argparse
import math
import os
import shutil
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

PATCHES = {
    "kernels/forward/ema_ssd_fwd.py": [
        ('device="cuda", dtype=torch.int8', 'device="cpu", dtype=torch.int8'),
        ("assert chunk_size in [64, 128]", "pass"),
        ('assert x.is_cuda, "Tensors must be on CUDA"', "pass"),
        ('assert dA.is_cuda, "dA tensor must be on CUDA"', "pass"),
        ('assert dA.is_cuda, "Input tensor must be on CUDA"', "pass"),
    ],
    "kernels/backward/ema_ssd_bwd.py": [
        ('device="cuda", dtype=torch.int8', 'device="cpu", dtype=torch.int8'),
    ],
    "kernels/backward/ema_ssd_combined.py": [
        ('device="cuda", dtype=torch.int8', 'device="cpu", dtype=torch.int8'),
        ('assert x.is_cuda and da_cs.is_cuda and da_cs_sum.is_cuda and do.is_cuda, '
         '"All tensors must be on CUDA"', "pass"),
    ],
}


def _stage_reference(ref_root: str) -> str:
    tmp = tempfile.mkdtemp(prefix="ema_ref_")
    shutil.copytree(os.path.join(ref_root, "kernels"), os.path.join(tmp, "kernels"),
                    ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    for rel, subs in PATCHES.items():
        path = os.path.join(tmp, rel)
        with open(path) as f:
            src = f.read()
        for old, new in subs:
            if old not in src:
                raise RuntimeError(f"patch target not found in {rel}: {old!r}")
            src = src.replace(old, new)
        with open(path, "w") as f:
            f.write(src)
    return tmp


def _np(t):
    return t.detach().cpu().float().numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("EMA_REFERENCE_DIR"),
                    help="root of a checkout of the reference repository (or set EMA_REFERENCE_DIR)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or EMA_REFERENCE_DIR: the reference checkout to generate fixtures from")
    os.environ["TRITON_INTERPRET"] = "1"
    tmp = _stage_reference(args.reference)
    sys.path.insert(0, tmp)
    try:
        import torch
        from kernels.forward.ema_ssd_fwd import chunk_cumsum_triton, ema_fwd_triton
        from kernels.backward.ema_ssd_combined import compute_dpx, ema_combined

        LOG2E = math.log2(math.e)
        out = {}

        def fwd_case(name, B, L, H, P, Q, seed, shared_heads=False, seq_idx=None):
            torch.manual_seed(seed)
            x = torch.randn(B, L, H, P)
            if shared_heads:
                A = -torch.rand(B, L)
                dA = (A * LOG2E)[:, None, :].repeat(1, H, 1).contiguous()
            else:
                dA = (-torch.rand(B, H, L) * LOG2E).contiguous()
            if seq_idx is None:
                y, st, cs, css = ema_fwd_triton(x, dA=dA, chunk_size=Q, store_states=True,
                                                store_da_cs=True, store_da_cs_sum=True)
                out[name] = dict(x=_np(x), dA=_np(dA), chunk_size=Q, out=_np(y), states=_np(st),
                                 da_cs=_np(cs), da_cs_sum=_np(css))
            else:
                y, css = ema_fwd_triton(x, dA=dA, seq_idx=seq_idx, chunk_size=Q,
                                        store_states=False, store_da_cs_sum=True)
                out[name] = dict(x=_np(x), dA=_np(dA), chunk_size=Q, seq_idx=seq_idx.numpy(),
                                 out=_np(y), da_cs_sum=_np(css))
            return x, dA

        def bwd_case(name, B, L, H, P, Q, seed, with_opts):
            x, dA = fwd_case(name + "_fwdin", B, L, H, P, Q, seed)
            f = out.pop(name + "_fwdin")
            torch.manual_seed(seed + 1000)
            do = torch.randn(B, L, H, P)
            d_ossm = torch.randn(B, H, P) if with_opts else None
            d_ox = torch.randn(B, H, P) if with_opts else None
            da_cs = torch.from_numpy(f["da_cs"])
            da_cs_sum = torch.from_numpy(f["da_cs_sum"])
            states = torch.from_numpy(f["states"]).squeeze(3).permute(0, 2, 3, 1).contiguous()
            if with_opts:  # a non-zero chunk-0 start state exercises the input-state path
                states[..., 0] = torch.randn(B, H, P)
            dx, dAk, d_issm = compute_dpx(x, da_cs, da_cs_sum, states, do, d_ossm_state=d_ossm,
                                          d_ox_state=d_ox, chunk_size=Q,
                                          has_input_state=with_opts)
            case = dict(x=_np(x), da_cs=f["da_cs"], da_cs_sum=f["da_cs_sum"], ssm_states=_np(states),
                        do=_np(do), chunk_size=Q, dx=_np(dx), dA=_np(dAk))
            if with_opts:
                case.update(d_ossm_state=_np(d_ossm), d_ox_state=_np(d_ox),
                            d_issm_state=_np(d_issm))
            out[name] = case

        fwd_case("fwd_q64", 2, 192, 2, 32, 64, seed=1)
        fwd_case("fwd_q64_shared", 2, 128, 3, 64, 64, seed=2, shared_heads=True)
        fwd_case("fwd_q128_ragged", 1, 200, 2, 64, 128, seed=3)
        fwd_case("fwd_q256", 1, 512, 1, 64, 256, seed=4)
        fwd_case("fwd_q64_p48", 1, 128, 1, 48, 64, seed=5)
        # seq_idx: the reference kernel broadcasts its per-token "same id as the
        # previous chunk" mask against the (1, headdim) carried state
        # (ema_ssd_fwd.py:389), which only type-checks when headdim == chunk_size
        # and is only right when every segment starts on a chunk boundary.  The
        # fixture therefore uses headdim == chunk_size with chunk-aligned segments
        # (the layout of the reference's own test_ema_seqidx, ema_ssd_fwd.py:765-768).
        K = 4
        aligned = torch.arange(K, dtype=torch.int8).repeat_interleave(256 // K)[None].repeat(2, 1)
        fwd_case("fwd_seqidx_aligned", 2, 256, 2, 64, 64, seed=6, seq_idx=aligned.contiguous())

        bwd_case("bwd_q64", 2, 192, 2, 32, 64, seed=11, with_opts=False)
        bwd_case("bwd_q64_opts", 1, 128, 2, 64, 64, seed=12, with_opts=True)
        bwd_case("bwd_q128", 1, 256, 2, 64, 128, seed=13, with_opts=False)
        bwd_case("bwd_q256_opts", 1, 512, 1, 64, 256, seed=14, with_opts=True)

        torch.manual_seed(21)
        B, L, H, P, Q = 1, 128, 2, 32, 64
        A = (-torch.rand(B, L)).requires_grad_()
        x = torch.randn(B, L, H, P).requires_grad_()
        dout = torch.randn(B, L, H, P)
        y = ema_combined(x, A, chunk_size=Q)
        (y * dout).sum().backward()
        out["combined_q64"] = dict(x=_np(x), A=_np(A), dout=_np(dout), chunk_size=Q, out=_np(y),
                                   dx=_np(x.grad), dA=_np(A.grad))

        torch.manual_seed(31)
        dA = -torch.rand(2, 2, 200) * LOG2E
        for e2 in (False, True):
            cs, rev = chunk_cumsum_triton(dA.contiguous(), chunk_size=64, exp2=e2)
            out[f"chunk_cumsum_exp2_{int(e2)}"] = dict(dA=_np(dA), chunk_size=64, exp2=int(e2),
                                                       dA_cs=_np(cs), dA_cs_rev=_np(rev))

        for name, case in out.items():
            path = os.path.join(HERE, f"{name}.npz")
            np.savez_compressed(path, **{k: np.asarray(v) for k, v in case.items()})
            print("wrote", path, {k: np.asarray(v).shape for k, v in case.items()})
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


if __name__ == "__main__":
    main()
