"""Per-kernel timing of the tcgen05 contractions (CUDA events, warm).

    python -m rustnn_b200.kernel_bench conv --cin 64 --cout 64 --hw 32 --batch 256 [--k 3 --stride 1]
    python -m rustnn_b200.kernel_bench gemm            # the six gemm.rs bench shapes (bench.rs:17-24)

Prints one line per kernel: time per launch, algorithmic TFLOP/s (2*M*N*K),
and the minimum HBM bytes / achieved GB/s.  Also the target of the ncu
captures summarised under profiles/.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import ops


def _time(fn, reps):
    fn()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(reps):
        fn()
    e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps / 1e3


def conv(args):
    n, ci, co, h, k, st = args.batch, args.cin, args.cout, args.hw, args.k, args.stride
    pad = 1 if k == 3 else 0
    oh = (h + 2 * pad - k) // st + 1
    dev = "cuda"
    x = torch.randn(n * ci * h * h, device=dev)
    w = torch.randn(co * ci * k * k, device=dev) * 0.05
    dy = torch.randn(n * co * oh * oh, device=dev)
    y = torch.empty_like(dy)
    dx = torch.empty_like(x)
    dw = torch.zeros_like(w)
    flops = 2.0 * n * oh * oh * co * ci * k * k
    out = []
    cases = {
        "fwd": (lambda: ops.conv2d_forward(x, w, n, ci, h, h, co, k, st, pad, y=y), x.numel() + y.numel()),
        "dgrad": (lambda: ops.conv2d_dgrad(dy, w, n, ci, h, h, co, k, st, pad, dx=dx), dy.numel() + dx.numel()),
        "wgrad": (lambda: ops.conv2d_wgrad(x, dy, n, ci, h, h, co, k, st, pad, dw=dw), x.numel() + dy.numel()),
    }
    for name in args.which.split(","):
        fn, elems = cases[name]
        t = _time(fn, args.reps)
        out.append({"kernel": f"conv_{name}", "shape": f"n{n} {ci}->{co} {h}x{h} k{k} s{st}", "ms": round(t * 1e3, 4),
                    "tflops": round(flops / t / 1e12, 2), "min_bytes": int(elems * 4),
                    "gbs": round(elems * 4 / t / 1e9, 1)})
    return out


BENCH = [  # bench.rs:17-24
    (16384, 768, 256, False, True, "S3 qkv fwd"),
    (16384, 704, 256, False, True, "S3 swiglu wg"),
    (16384, 256, 768, False, False, "S3 qkv dX"),
    (768, 256, 16384, True, False, "S3 qkv dW"),
    (16384, 256, 352, False, True, "S3 swiglu wd fwd"),
    (4096, 384, 1024, False, True, "merge fwd"),
]


def gemm(args):
    out = []
    for m, n, k, at, bt, tag in BENCH:
        a = torch.randn(m * k, device="cuda")
        b = torch.randn(k * n, device="cuda")
        c = torch.empty(m * n, device="cuda")
        t = _time(lambda: ops.matmul(m, n, k, a, at, b, bt, c), args.reps)
        out.append({"kernel": "gemm", "shape": f"{tag} {m}x{n}x{k}", "ms": round(t * 1e3, 4),
                    "tflops": round(2.0 * m * n * k / t / 1e12, 2),
                    "gbs": round((m * k + k * n + m * n) * 4 / t / 1e9, 1)})
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["conv", "gemm"])
    ap.add_argument("--cin", type=int, default=64)
    ap.add_argument("--cout", type=int, default=64)
    ap.add_argument("--hw", type=int, default=32)
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--k", type=int, default=3)
    ap.add_argument("--stride", type=int, default=1)
    ap.add_argument("--which", default="fwd,dgrad,wgrad")
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args()
    rows = conv(args) if args.what == "conv" else gemm(args)
    for r in rows:
        print(json.dumps(r))


if __name__ == "__main__":
    main()
