"""Run one grouped GEMV of a model shape repeatedly: a small, self-contained case for profilers (ncu) and timing.

usage: python -m pingala8_llm_b200.profile [--group gate_up|qkv|o|down] [--iters N] [--copies C] [--graph]
                                            [--ncols N] [--encode ROWS]

Weights are seeded synthetic class-3 slots of the Llama-3.1-8B shapes. With --copies > 1 the calls rotate over
distinct weight copies so repeated calls read DRAM rather than L2. Prints the mean time per call (CUDA events).
--ncols N (N >= 4) runs the batched product (tcgen05 GEMM) of each tensor of the group on N tokens instead of the
grouped batch-1 GEMV. --encode ROWS runs the offline trellis encoder (k_vit) on a ROWS x 4096 class-3 tensor with a
random Hessian instead, --iters times, and prints the time per weight.
"""
import argparse

import torch

from . import synth
from .ops import P8Tensor, group_workspace_size, mul_mat_vec_group

GROUPS = {  # Llama-3.1-8B: (rows, K) per tensor of a group that reads one x
    "qkv": [(4096, 4096), (1024, 4096), (1024, 4096)],
    "o": [(4096, 4096)],
    "gate_up": [(14336, 4096), (14336, 4096)],
    "down": [(4096, 14336)],
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--group", default="gate_up", choices=sorted(GROUPS))
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--copies", type=int, default=1)
    ap.add_argument("--graph", action="store_true", help="capture the calls in a CUDA graph (no host launch overhead)")
    ap.add_argument("--ncols", type=int, default=1, help="tokens per call; > 1 runs the batched product per tensor")
    ap.add_argument("--grouped", action="store_true",
                    help="with --ncols > 1: the group as one grouped product (mul_mat_group: one activation prep, "
                         "tensors of one shape in one launch where that fills the waves better)")
    ap.add_argument("--encode", type=int, default=0, help="run the trellis encoder on ROWS x 4096 instead")
    a = ap.parse_args()
    if a.encode:
        return run_encoder(a)
    shapes = GROUPS[a.group]
    if a.ncols > 1:
        return run_batched(a, shapes)
    copies = []
    for c in range(a.copies):
        copies.append([P8Tensor(synth.make_slot_device(r, k, seed=100 * c + i), k, r) for i, (r, k) in enumerate(shapes)])
    K = shapes[0][1]
    x = torch.randn(K, device="cuda")
    outs = [torch.empty(r, device="cuda") for r, _ in shapes]
    ws = torch.empty(max(group_workspace_size(ts) for ts in copies), dtype=torch.uint8, device="cuda")
    for ts in copies:  # warm-up
        mul_mat_vec_group(ts, x, outs=outs, workspace=ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if a.graph:
        s = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for i in range(a.iters):
                    mul_mat_vec_group(copies[i % len(copies)], x, outs=outs, workspace=ws, stream=s)
        g.replay()
        torch.cuda.synchronize()
        e0.record()
        g.replay()
        e1.record()
    else:
        e0.record()
        for i in range(a.iters):
            mul_mat_vec_group(copies[i % len(copies)], x, outs=outs, workspace=ws)
        e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / a.iters
    nbytes = sum((r // 32) * (k // 256) * (68 + 2048) for r, k in shapes)
    print(f"group {a.group}: {us:.2f} us/call, {nbytes / us / 1e3:.1f} GB/s (algorithmic, class 3)")


def run_batched(a, shapes):
    ts = [P8Tensor(synth.make_slot_device(r, k, seed=i), k, r) for i, (r, k) in enumerate(shapes)]
    X = torch.randn(a.ncols, shapes[0][1], device="cuda")
    outs = [torch.empty(a.ncols, r, device="cuda") for r, _ in shapes]
    if a.grouped:
        from .ops import mul_mat_group

        gws = torch.empty(max(group_workspace_size(ts, a.ncols), 256), dtype=torch.uint8, device="cuda")

        def once():
            mul_mat_group(ts, X, outs=outs, workspace=gws)
    else:
        ws = [t.workspace(a.ncols) for t in ts]

        def once():
            for t, y, w in zip(ts, outs, ws):
                t.mul_mat(X, out=y, workspace=w)
    once()  # warm-up
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        once()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / a.iters
    flop = sum(2.0 * r * k * a.ncols for r, k in shapes)
    print(f"group {a.group} x {a.ncols} tokens: {us:.2f} us/call, {flop / us / 1e6:.1f} TFLOP/s")




def run_encoder(a):
    from .encoder import encode

    n, rows = 4096, a.encode
    g = torch.Generator(device="cuda").manual_seed(0)
    X = torch.randn(2 * n, n, device="cuda", generator=g, dtype=torch.float64)
    H = X.T @ X / (2 * n)
    H += 0.1 * H.diagonal().mean() * torch.eye(n, device="cuda", dtype=torch.float64)
    Uc = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(H)), upper=True).float()
    Y = torch.randn(rows, n, device="cuda", generator=g)
    cls = torch.full((rows, n // 256), 3, dtype=torch.int64)
    Sb = torch.full((rows, n // 256), 1 / 16.0)
    encode(Y[:16], Uc, cls[:16], Sb[:16])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        encode(Y, Uc, cls, Sb)
    e1.record()
    torch.cuda.synchronize()
    dt = e0.elapsed_time(e1) / 1e3 / a.iters
    print(f"encode {rows} x {n} class 3: {dt * 1e3:.3f} ms per tensor, {dt / (rows * n) * 1e9:.3f} ns per weight")


if __name__ == "__main__":
    main()
