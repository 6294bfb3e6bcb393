"""Per-kernel timing of the tcgen05 contractions (CUDA events, warm).

    python -m rustnn_b200.kernel_bench conv --cin 64 --cout 64 --hw 32 --batch 256 [--k 3 --stride 1]
    python -m rustnn_b200.kernel_bench gemm            # the six gemm.rs bench shapes (bench.rs:17-24)
    python -m rustnn_b200.kernel_bench attn [--dh 64]  # Core fwd/bwd at the attention config (B=128, h=4, dh=32)
    python -m rustnn_b200.kernel_bench ln              # LayerNorm fwd/bwd at the rustvit row counts
    python -m rustnn_b200.kernel_bench muon            # Muon (Newton-Schulz) over the 39 rustvit weight matrices
    python -m rustnn_b200.kernel_bench vitstep         # one rustvit Trainer::step (batch 128) after 3 warm-ups,
                                                       # alone between cudaProfilerStart/Stop (ncu
                                                       # --profile-from-start off lists exactly its launches)
    python -m rustnn_b200.kernel_bench resnetstep --batch 128   # one ResNet-56 W=64 graph step, same way
    python -m rustnn_b200.kernel_bench data --batch 1024        # batch builder and mixes per call

--graph times a CUDA-graph replay of the calls instead of back-to-back
Python calls (device time without the host's per-call cost).

Prints one line per kernel: time per launch, algorithmic TFLOP/s (2*M*N*K),
and the minimum HBM bytes / achieved GB/s.  Also the target of the ncu
captures summarised under profiles/.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import ops


GRAPH = False  # set by --graph


def _time(fn, reps):
    """Seconds per call of fn.  Back-to-back calls from Python by default
    (what a caller of the Python API sees: small calls are bounded by the
    host); with --graph the reps calls are captured once into a CUDA graph
    and the replay is timed (device time, no host launch cost)."""
    if GRAPH:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()  # binds the context to s, sizes workspaces, sets attributes
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(reps):
                fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            g.replay()
            e0.record(s)
            g.replay()
            e1.record(s)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps / 1e3
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


def attn(args):
    """Core::forward/backward (attn.rs:148-343) at B=128, h=4, dh=32: self
    attention over 8x8 tokens (diagonal masked) and cross attention from 8x8
    queries into a 16x16 memory.  Bytes count every tensor the kernels must
    read or write once, P included (the backward reads it)."""
    n, h, dh = args.batch if args.batch != 256 else 128, 4, args.dh
    c = h * dh
    out = []
    for tag, (th, mh, self_) in (("self 64x64", (8, 8, True)), ("cross 64x256", (8, 16, False))):
        tq, tk = th * th, mh * mh
        _, nrel = ops.rel_index(th, th, mh, mh)
        g = torch.Generator(device="cuda").manual_seed(0)
        if self_:
            q = torch.randn(n * tq * 3 * c, device="cuda", generator=g) / 32 ** 0.5
            kv, qs, qo, kvs, ko, vo = q, 3 * c, 0, 3 * c, c, 2 * c
        else:
            q = torch.randn(n * tq * c, device="cuda", generator=g) / 32 ** 0.5
            kv = torch.randn(n * tk * 2 * c, device="cuda", generator=g) / 32 ** 0.5
            qs, qo, kvs, ko, vo = c, 0, 2 * c, 0, c
        tau = torch.full((h,), 1 / dh ** 0.5, device="cuda")
        rel = torch.randn(h * nrel, device="cuda", generator=g)
        p, o = ops.attn_forward(n, h, dh, th, th, mh, mh, self_, q, qs, qo, kv, kvs, ko, vo, tau, rel)
        dout = torch.randn_like(o)
        dq, dkv = torch.zeros_like(q), torch.zeros_like(kv)
        dtau, drel = torch.zeros_like(tau), torch.zeros_like(rel)
        fl_f = 2.0 * 2 * n * h * tq * tk * dh
        fl_b = 2.0 * 5 * n * h * tq * tk * dh  # dV, dP, QK^T recompute (dtau), dQ, dK
        pb = n * h * tq * tk * 4
        qkvo = (n * tq * c * 2 + n * tk * c * 2) * 4
        tf = _time(lambda: ops.attn_forward(n, h, dh, th, th, mh, mh, self_, q, qs, qo, kv, kvs, ko, vo, tau, rel),
                   args.reps)
        tb = _time(lambda: ops.attn_backward(n, h, dh, th, th, mh, mh, q, qs, qo, kv, kvs, ko, vo, tau, p, dout, dq,
                                             dkv, dtau, drel), args.reps)
        fb, bb = qkvo + pb, qkvo + pb + n * tq * c * 4 + (n * tq * c + n * tk * 2 * c) * 4 * 2
        for kind, t, fl, by in (("fwd", tf, fl_f, fb), ("bwd", tb, fl_b, bb)):
            out.append({"kernel": f"attn_{kind}", "shape": f"{tag} n{n} h{h} dh{dh}", "ms": round(t * 1e3, 4),
                        "tflops": round(fl / t / 1e12, 2), "min_bytes": int(by), "gbs": round(by / t / 1e9, 1)})
    return out


def ln(args):
    """LayerNorm (norm.rs:38-137) fwd/bwd at the rustvit row counts (B=128)."""
    out = []
    for rows, c in ((8192, 256), (2048, 384), (32768, 512), (2048, 1024)):
        x = torch.randn(rows * c, device="cuda")
        gm, bt = torch.randn(c, device="cuda"), torch.randn(c, device="cuda")
        y, xh, inv = ops.layernorm_forward(x, rows, c, gm, bt)
        dy = torch.randn_like(x)
        dg, db = torch.zeros(c, device="cuda"), torch.zeros(c, device="cuda")
        tf = _time(lambda: ops.layernorm_forward(x, rows, c, gm, bt), args.reps)
        tb = _time(lambda: ops.layernorm_backward(dy, xh, inv, rows, c, gm, dg, db), args.reps)
        fb, bb = rows * c * 4 * 3 + rows * 4, rows * c * 4 * 3 + rows * 4
        out.append({"kernel": "layernorm_fwd", "shape": f"{rows}x{c}", "ms": round(tf * 1e3, 4), "min_bytes": fb,
                    "gbs": round(fb / tf / 1e9, 1)})
        out.append({"kernel": "layernorm_bwd", "shape": f"{rows}x{c}", "ms": round(tb * 1e3, 4), "min_bytes": bb,
                    "gbs": round(bb / tb / 1e9, 1)})
    return out


RUSTVIT_2D = ([(768, 256), (256, 256), (704, 256), (256, 352)] * 5 + [(256, 256), (256, 256)] * 2
              + [(1152, 384), (384, 384), (1024, 384), (384, 512)] * 2 + [(384, 1024), (20, 384), (100, 384),
                                                                          (100, 96), (384, 96), (100, 256), (384, 256)])


def muon(args):
    """Muon over the 39 rustvit Linear weights (optim.rs:177-203): 3 quintic
    Newton-Schulz iterations each.  Flops per matrix with s = min dim, l = max:
    per iteration 2*s*s*l (X X^T) + 2*s*s*s (A A) + 2*s*s*l (B X)."""
    mats = []
    fl = 0.0
    for r, c in RUSTVIT_2D:
        v = torch.randn(r * c, device="cuda") * 0.02
        g = torch.randn(r * c, device="cuda")
        m = torch.zeros(r * c, device="cuda")
        mats.append((v, g, m, r, c))
        s, l = min(r, c), max(r, c)
        fl += 3 * (4.0 * s * s * l + 2.0 * s * s * s)

    def step():
        for v, g, m, r, c in mats:
            ops.muon_step_(v, g, m, r, c, 3, 0.02)

    t = _time(step, args.reps)
    return [{"kernel": "muon_step", "shape": f"{len(mats)} matrices (rustvit)", "ms": round(t * 1e3, 4),
             "tflops": round(fl / t / 1e12, 2), "gflop": round(fl / 1e9, 2)}]


def databatch(args):
    """data::make_batch_train (data.rs:384-412) and mix_batch (data.rs:467-491)
    per batch of args.batch images from a resident 50,000-image u8 split:
    time per call as a caller sees it (the host's draws included)."""
    import numpy as np

    from . import data

    n, bs = 50_000, args.batch
    rng = np.random.default_rng(0)
    images = torch.from_numpy(rng.integers(0, 256, size=n * 3072, dtype=np.uint8)).cuda()
    labels = torch.from_numpy(rng.integers(0, 100, size=n, dtype=np.uint8)).cuda()
    idx = torch.from_numpy(rng.permutation(n)[:bs].astype(np.int32)).cuda()
    out = torch.empty(bs * 3072, device="cuda")
    lab = torch.empty(bs, dtype=torch.int32, device="cuda")
    rows = []
    for tag, aug in (("resnet aug (pad 4, erase 1.0 side 8)", data.Aug(pad=4, erase=1.0, erase_side=8)),
                     ("randaugment x2 m0.6, erase 0.25", data.Aug(pad=4, ra_mag=0.6, ra_n=2, erase=0.25))):
        t = _time(lambda: data.make_batch_train(images, labels, None, idx, aug, 7, out=out, labels_out=lab),
                  args.reps)
        rows.append({"kernel": "make_batch_train", "shape": f"batch {bs}, {tag}", "ms": round(t * 1e3, 4)})
    st = np.array([1, 2, 3, 4], dtype=np.uint64)
    for tag, m, c in (("mixup 0.8", 0.8, 0.0), ("cutmix 1.0", 0.0, 1.0)):
        t = _time(lambda: data.mix_batch(out, bs, m, c, 0.5, st), args.reps)
        rows.append({"kernel": "mix_batch", "shape": f"batch {bs}, {tag}", "ms": round(t * 1e3, 4)})
    return rows


def vitstep(args):
    """Trainer::step of the default rustvit (train.rs:346-387) at batch
    args.batch, synthetic data; the timed step runs alone inside the
    profiler range."""
    import numpy as np

    from . import vit

    n = args.batch
    net = vit.RustViT(vit.VitCfg(), vit.cifar_parent(), 20, 0)
    rng = np.random.default_rng(100)
    x = torch.from_numpy(rng.standard_normal(n * 3 * 32 * 32).astype(np.float32)).cuda()
    hard = rng.integers(0, 100, size=n).astype(np.uint32)
    tf, tc, coarse = vit.targets(hard, vit.cifar_parent(), 20)
    tfd, tcd = torch.from_numpy(tf).cuda(), torch.from_numpy(tc).cuda()
    hd = torch.from_numpy(hard.astype(np.int32)).cuda()
    cd = torch.from_numpy(coarse.astype(np.int32)).cuda()
    for i in range(3):
        net.train_step(x, tfd, tcd, hd, cd, drop_seed=i, stats=False)
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = ops.lib().rnn_launch_count()
    torch.cuda.cudart().cudaProfilerStart()
    e0.record(s)
    net.train_step(x, tfd, tcd, hd, cd, drop_seed=9, stats=False)
    e1.record(s)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    launches = ops.lib().rnn_launch_count() - l0
    net.close()
    return [{"kernel": "rustvit_step", "shape": f"batch {n}", "ms": round(e0.elapsed_time(e1), 3),
             "launches": int(launches)}]


def resnetstep(args):
    """The ResNet-56 W=64 training step (BASELINE config 5's network) at batch
    args.batch, replayed from a CUDA graph: ten steps timed with CUDA events
    after four warm-ups, then one step alone inside the profiler range."""
    import numpy as np

    from . import model

    n = args.batch
    net = model.ResNet(9, 64, 100, 0)
    net.use_graph(True)
    rng = np.random.default_rng(100)
    u = rng.integers(0, 256, size=n * 3 * 32 * 32).astype(np.float32)
    x = torch.from_numpy(((u - 127.5) / 73.9).astype(np.float32)).cuda()
    lab = torch.from_numpy(rng.integers(0, 100, size=n).astype(np.int32)).cuda()
    for _ in range(4):
        net.train_step(x, lab)
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(10):
        net.train_step(x, lab)
    e1.record(s)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStart()
    net.train_step(x, lab)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    net.close()
    return [{"kernel": "resnet56_step", "shape": f"batch {n}", "ms": round(e0.elapsed_time(e1) / 10, 3)}]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["conv", "gemm", "attn", "ln", "muon", "vitstep", "resnetstep", "data"])
    ap.add_argument("--cin", type=int, default=64)
    ap.add_argument("--cout", type=int, default=64)
    ap.add_argument("--hw", type=int, default=32)
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--k", type=int, default=3)
    ap.add_argument("--stride", type=int, default=1)
    ap.add_argument("--which", default="fwd,dgrad,wgrad")
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--dh", type=int, default=32, help="attention head dim (32: BASELINE config 3; 64: rustvit)")
    ap.add_argument("--graph", action="store_true", help="time a CUDA-graph replay of the calls (device time)")
    args = ap.parse_args()
    global GRAPH
    GRAPH = args.graph
    rows = {"conv": conv, "gemm": gemm, "attn": attn, "ln": ln, "muon": muon, "vitstep": vitstep,
            "resnetstep": resnetstep, "data": databatch}[args.what](args)
    for r in rows:
        print(json.dumps(r))


if __name__ == "__main__":
    main()
