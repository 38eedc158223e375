#!/usr/bin/env python
"""Pingala-8 batch-1 decode throughput on B200 (and the reference CPU path on the same host).

Headline workload (the metric "decode tok/s bs1 (Llama-3.1-8B shape, 2-bit)"): one decode token through
every Pingala-8 projection of a Llama-3.1-8B-architecture model -- 32 layers x {q, k, v, o, gate, up, down}
(224 GEMVs, 1.80 GB of class-3 slots: seeded random valid codes, shapes of the real model). The projections are
chained on the device (x -> q,k,v; q-out -> o; o-out -> gate,up; gate-out -> down; down-out -> next layer), launched
as 4 grouped GEMV calls per layer (tensors that read the same x share one prepared activation), captured once as a
CUDA graph and replayed per step. Attention, norms and the LM head are not part of this path.

  value     tokens/s with inputs resident in HBM (device-timed with CUDA events, max over ranks)
  e2e       the same through the public op API with a pinned-host input vector copied in and the final output copied
            out every step, the host waiting for each step's output before it starts the next
  roofline  the dominant call type (p8_mul_mat_vec_group = k_gemv + k_gemv_reduce): algorithmic bytes / per-call
            duration, timed with CUDA events around a graph of that call type's 32 per-layer calls, against
            MEASURED_PEAKS.json hbm_gbs; traffic = DRAM bytes of the same call from an ncu capture
  cpu_baseline  the reference's own CPU core (oracle/_ref, x16 vrc_tg) on one layer's 7 GEMVs, all host threads
  prefill   (1 GPU) the batched product: 512 tokens through all 224 projections (tcgen05 GEMM), the projections on
            one input as grouped products (p8_mul_mat_group), TFLOP/s against MEASURED_PEAKS.json bf16_tflops; the
            same pass as separate p8_mul_mat calls beside it; c3_per_gemm: each of the 7 projections alone at 512 and
            2,048 tokens
  batched_decode  (1 GPU) bs = 2, 3, 4, 8, 32, 64 sequences stepping together through the same chain, every group call the
            grouped batched product (bs 2-5: the two-column batch-1 GEMV in pairs, weights decoded once per two
            sequences; from bs 6 the split-K tcgen05 GEMM): tok/s per bs
  layer_prologues (1 GPU) the chain with each layer's input ops (RMSNorm x weight, SwiGLU) fused into the GEMV's
            activation prep, against the same ops as separate torch kernels

usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

LLAMA8B = dict(name="llama3.1-8b", layers=32, hidden=4096, ffn=14336, q=4096, kv=1024)
QWEN14B = dict(name="qwen3-14b", layers=40, hidden=5120, ffn=17408, q=5120, kv=1024)  # benchmark config C5
# a small layer whose o split at 2 ranks is not whole 256-column blocks (5 query heads = 640 columns per rank): the
# shared-boundary-block path that Qwen3-14B takes at 8 ranks, checked at 2
UNALIGNED2 = dict(name="10-head-2-kv (o split 640 | 640)", layers=1, hidden=1280, ffn=2560, q=1280, kv=256)
METRIC = "decode tok/s bs1 (Llama-3.1-8B shape, 2-bit); dequant-GEMV HBM GB/s % of peak"


def layer_shapes(m):
    h, f, q, kv = m["hidden"], m["ffn"], m["q"], m["kv"]
    # (name, rows, K): ggml [K, rows]
    return [("q", q, h), ("k", kv, h), ("v", kv, h), ("o", h, q), ("gate", f, h), ("up", f, h), ("down", h, f)]


def kernel_bytes_of(rows, K, cls=3):
    nt = (rows // 32) * (K // 256)
    nw = [0, 4, 6, 8, 10, 12, 16, 24][cls]
    return ((2064 + 68 * nt + 15) & ~15) + 4 * nt * 64 * nw


def algo_bytes_gemv(rows, K, cls=3):
    """bytes one GEMV must move: M + S + payload of the slot (the rest of the header and side data are cached), x, y"""
    nt = (rows // 32) * (K // 256)
    nw = [0, 4, 6, 8, 10, 12, 16, 24][cls]
    return 4 * nt + 64 * nt + 4 * nt * 64 * nw + 4 * K + 4 * rows


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled every 2 ms through NVML while the timed region runs
    (read-only queries); falls back to nvidia-smi -lms 200 when NVML is unavailable."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap",
               0x80: "hw_power_brake_slowdown"}
    Q = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown," \
        "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, index):
        self.index = index
        self.sm, self.mx, self.reasons = [], None, set()
        self.stop = threading.Event()
        self.proc = None
        self.t = None

    def __enter__(self):
        try:
            import pynvml as N
            N.nvmlInit()
            h = N.nvmlDeviceGetHandleByIndex(self.index)
            self.mx = float(N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM))
            get_reasons = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or N.nvmlDeviceGetCurrentClocksThrottleReasons

            def poll():
                while not self.stop.is_set():
                    self._nvml_sample(N, h, get_reasons)
                    time.sleep(0.002)
                self._nvml_sample(N, h, get_reasons)

            self.t = threading.Thread(target=poll, daemon=True)
            self.t.start()
        except Exception:
            try:
                self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "200",
                                              "-i", str(self.index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self.t = threading.Thread(target=self._smi_read, daemon=True)
                self.t.start()
            except (OSError, FileNotFoundError):
                self.proc = None
        return self

    def _nvml_sample(self, N, h, get_reasons):
        try:
            self.sm.append(float(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)))
            r = int(get_reasons(h))
            for bit, name in self.REASONS.items():
                if r & bit:
                    self.reasons.add(name)
        except Exception:
            pass

    def _smi_read(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.proc.stdout:
            p = [x.strip() for x in ln.strip().split(",")]
            if len(p) < 9:
                continue
            try:
                self.sm.append(float(p[1]))
                self.mx = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    self.reasons.add(n)

    def __exit__(self, *a):
        self.stop.set()
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.t:
            self.t.join(timeout=5)

    def summary(self):
        if not self.sm:
            return {"sm_mhz": None, "sm_max_mhz": self.mx, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": self.mx, "reasons": sorted(self.reasons),
                "samples": len(self.sm)}


# DRAM bytes (read + write) of one call (k_gemv + k_gemv_reduce), from ncu captures of the same call at 1 GPU
# (profiles/k_gemv_llama8b_gate_up.md); reported only for the configuration the capture measured
TRAFFIC_BYTES = {"gate+up": 30377728 + 3584 + 2026240}


def measured_bf16_tflops():
    """(peak, source): MEASURED_PEAKS.json bf16_tflops, else the pool's earlier measurement 1,590 TFLOP/s"""
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        v = json.load(open(p)).get("bf16_tflops")
        if v:
            return float(v), "measured: MEASURED_PEAKS.json bf16_tflops (cuBLAS bf16 burst)"
    return 1590.0, "fallback: 1,590 TFLOP/s, an earlier cuBLAS bf16 burst measurement on this pool (MEASURED_PEAKS.json absent)"


def measured_peaks():
    """(peak, source): MEASURED_PEAKS.json hbm_gbs, else the pool's earlier measurement 6,650 GB/s"""
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        v = json.load(open(p)).get("hbm_gbs")
        if v:
            return float(v), "measured: MEASURED_PEAKS.json hbm_gbs (burst copy)"
    return 6650.0, "fallback: 6,650 GB/s, an earlier copy measurement on this pool (MEASURED_PEAKS.json absent)"


# ------------------------------------------------------------------------------------------------ CPU reference leg
_REF_CACHE = {}


def ref_slots(model, seed=0):
    """The reference legs' decode token: 32 x 7 distinct class-3 slots built with numpy (oracle/synth_np.py), each
    held by a RefOracle (the reference CPU core's view of it), and one seeded x per input width."""
    from oracle import synth_np
    from oracle.oracle import RefOracle

    key = (model["name"], seed)
    if key not in _REF_CACHE:
        mats = []
        for L in range(model["layers"]):
            for i, (nm, rows, K) in enumerate(layer_shapes(model)):
                mats.append(RefOracle(synth_np.make_slot(rows, K, seed=seed + 1000 * L + 17 * i), rows, K))
        xs = {K: np.random.default_rng(K).normal(0, 1, K).astype(np.float32) for _, _, K in layer_shapes(model)}
        _REF_CACHE[key] = (mats, xs)
    return _REF_CACHE[key]


def cpu_reference_token(model, reps, warmup, seed=0):
    """The reference's own CPU core (oracle/_ref: vr-native-cpu-core.h with the vrc_tg glue, x16 activations) over one
    decode token: every projection of every layer, 32 x 7 distinct class-3 slots (1.80 GB, far larger than any host
    cache, so weights stream from DRAM as on the GPU). Slots are built with numpy (oracle/synth_np.py): this leg never
    loads the product library. OpenMP threads = all host cores, set explicitly (torchrun exports OMP_NUM_THREADS=1).
    Returns (median seconds per token, threads, ISA)."""
    from oracle.oracle import RefOracle

    ncores = os.cpu_count() or 1
    RefOracle.set_threads(ncores)
    mats, xs = ref_slots(model, seed)

    def token():
        for r in mats:
            r.gemv(xs[r.K])

    for _ in range(warmup):
        token()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        token()
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts), RefOracle.threads(), RefOracle.isa()


def gpu_reference_token(model, steps, warmup, seed=0):
    """The reference's own CUDA GEMV (oracle/_ref/libp8ref_gpu.so: k_vr_qx_real + cudaMemset + k_vr<1, V, 8, 108>, cut
    from its patch) over the same decode token as cpu_reference_token: the same 224 numpy-built slots, uploaded once,
    one call per projection (the reference has no grouped call), captured as one CUDA graph per variant (llama.cpp
    replays its decode graph the same way) and replayed per step, timed with CUDA events on the capture stream. V 5 is
    the shipped instance (GGML_VRC_V=5), V 7 the code default. Per projection type: the 32 per-layer calls in a graph
    of their own, per-call duration against the call's algorithmic bytes, as the b200 arm's roofline does.
    Weights (1.80 GB) exceed L2, so replays stream from HBM. Slots, x and y live on cuda:0; nothing of the product
    library is loaded."""
    import torch
    from oracle.oracle import RefGpu

    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    if not RefGpu.available():
        return {"unavailable": "oracle/_ref/libp8ref_gpu.so not built (needs the reference patch at build time)"}
    mats, xs = ref_slots(model, seed)
    dev = torch.device("cuda", 0)
    RefGpu.set_tables(mats[0].slot)
    shapes = layer_shapes(model)
    slots = [torch.from_numpy(r.slot).to(dev) for r in mats]
    xd = {K: torch.from_numpy(v).to(dev) for K, v in xs.items()}
    ys = [torch.empty(r.rows, device=dev) for r in mats]
    kmax = max(xs)
    xq = torch.empty(kmax, dtype=torch.int8, device=dev)
    xsc = torch.empty(kmax // 128, device=dev)
    st = torch.cuda.Stream(dev)

    def call(i, V):
        r = mats[i]
        RefGpu.gemv(slots[i].data_ptr(), r.slot.size, r.rows, r.K, 0, xd[r.K].data_ptr(), ys[i].data_ptr(),
                    xq.data_ptr(), xsc.data_ptr(), V=V, RL=1, stream=st.cuda_stream)

    def graph_of(idx, V):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(st):
            for i in idx:  # one eager pass first (module load, first-launch set-up)
                call(i, V)
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=st):
                for i in idx:
                    call(i, V)
        return g

    def timed(g, n):
        ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(st):
            for _ in range(warmup):
                g.replay()
            torch.cuda.synchronize()
            ea.record(st)
            for _ in range(n):
                g.replay()
            eb.record(st)
        torch.cuda.synchronize()
        return ea.elapsed_time(eb) / 1e3 / n

    out = {"kernels": "k_vr_qx_real + k_vr<1, V, 8, 108> (reference CU:3003-3018, CU:2662-2727), one call per projection",
           "graph": True, "l2": "weights 1.80 GB > L2", "variants": {}}
    allidx = list(range(len(mats)))
    per_tok_bytes = sum(algo_bytes_gemv(r.rows, r.K) for r in mats)
    peak, peak_kind = measured_peaks()
    for V in (5, 7):
        g = graph_of(allidx, V)
        t = timed(g, max(3, steps))
        del g
        out["variants"][f"V{V}"] = {"tok_s": round(1.0 / t, 2), "ms_per_token": round(1e3 * t, 4),
                                    "weight_gbs": round(per_tok_bytes / t / 1e9, 1)}
        if V == 5:
            calls = {}
            for j, (nm, rows, K) in enumerate(shapes):
                idx = [L * len(shapes) + j for L in range(model["layers"])]
                gj = graph_of(idx, V)
                tc = timed(gj, max(3, steps // 4)) / len(idx)
                del gj
                gbs = algo_bytes_gemv(rows, K) / tc / 1e9
                calls[nm] = {"us_per_call": round(1e6 * tc, 2), "gbs": round(gbs, 1), "frac": round(gbs / peak, 3)}
            out["per_call_V5"] = calls
    # one sanity figure: the reference kernels' y against the CPU reference core on the same slot and x (int8 x' in
    # the kernel vs x16 in the core: relative L2 near 1e-2 is expected)
    torch.cuda.synchronize()
    r0 = mats[0]
    yc = r0.gemv(xs[r0.K])
    yg = ys[0].cpu().numpy()
    out["rel_l2_vs_cpu_core"] = float(np.linalg.norm(yg - yc) / np.linalg.norm(yc))
    out["tok_s"] = out["variants"]["V5"]["tok_s"]
    out["hbm_peak_gbs"] = peak
    out["peak_kind"] = peak_kind
    del slots
    torch.cuda.empty_cache()
    return out


def run_reference(args, rank, world):
    model = LLAMA8B
    if rank != 0:
        return 0
    tok_s_time, cores, isa = cpu_reference_token(model, reps=max(1, args.steps), warmup=max(1, args.warmup))
    tok_s = 1.0 / tok_s_time
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tok_s, 4), "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1e3 * tok_s_time, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int32+fp32 (x16 activations)", "data": "synthetic",
        "config": {"workload": "llama3.1-8b-bs1-decode-projections", "layers": model["layers"], "projections_per_layer": 7,
                   "batch": 1, "classes": "3"},
        "cpu_baseline": {"value": round(tok_s, 4), "unit": "tok/s", "cores": cores, "kind": "reference",
                         "sample": f"every step one token: all {model['layers'] * 7} projections, distinct slots (1.80 GB); "
                                   f"median of {max(1, args.steps)}; {isa} vr-native-cpu-core.h, {cores} OpenMP threads"},
        "e2e": {"value": round(tok_s, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_ref_gpu:
        try:
            line["reference_gpu"] = gpu_reference_token(model, steps=max(3, args.steps), warmup=max(1, args.warmup))
        except Exception as e:  # reported, never fatal: the CPU line above is the reference arm's measurement
            line["reference_gpu"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------------------------ tensor parallel
def tp_dims(model):
    from pingala8_llm_b200 import tp

    return tp.LayerDims(hidden=model["hidden"], ffn=model["ffn"], heads=model["q"] // 128, kv_heads=model["kv"] // 128,
                        head_dim=128)


def tp_parity(model, world, rank, dev, comm):
    """One layer's q and gate (column-parallel) and o and down (row-parallel) of `model`, as full slots with the same
    bytes on every rank, sharded by tp.layer_plan with the host shard transforms and run through the TP path (the
    row-parallel sum inside the GEMV over peer memory when comm is given, else an NCCL all-reduce), against the
    unsharded tensor's GEMV on the same GPU. Returns (relative L2 error per tensor, the bar): 1e-5 when every
    row-parallel split is whole 256-column blocks (the same integer sums, float order only), 1e-3 when a boundary
    block is shared (each rank quantises its own masked half of the block, x16)."""
    import torch

    from pingala8_llm_b200 import synth, tp
    from pingala8_llm_b200.ops import P8Tensor

    plan = tp.layer_plan(tp_dims(model), world, rank)
    shapes = {n: (r, k) for n, r, k in layer_shapes(model)}
    errs = {}
    aligned = True
    for i, nm in enumerate(("q", "o", "gate", "down")):
        rows, K = shapes[nm]
        slot = synth.make_slot(rows, K, seed=4242 + i, nd=5)  # the same bytes on every rank
        g = torch.Generator(device=dev)
        g.manual_seed(77 + i)
        x = torch.randn(K, device=dev, generator=g)
        y_full = P8Tensor(slot, K, rows).mul_mat_vec(x)
        e = plan[nm]
        if e.kind == "col":
            sh = tp.shard_for(e, slot, world, rank)
            y = P8Tensor(sh.slot, K, sh.rows).mul_mat_vec(x) if sh.rows else torch.empty(0, device=dev)
            ref = y_full[e.lo:e.hi]
        else:
            aligned = aligned and e.lo % 256 == 0 and e.hi % 256 == 0
            rp = tp.RowParallel(slot, K, rows, world, rank, comm=comm, cols=(e.lo, e.hi))
            y = rp(x[e.lo:e.hi].contiguous())
            ref = y_full
        torch.cuda.synchronize()
        errs[nm] = float((y.double() - ref.double()).norm() / ref.double().norm()) if ref.numel() else 0.0
    return errs, (1e-5 if aligned else 1e-3)


def tp_model_decode(model, args, rank, world, dev, comm, stream):
    """Benchmark config C5 on this model: every projection split over the ranks by tp.layer_plan (q/k/v/gate/up
    column-parallel, o/down row-parallel; an o split that is not whole 256-column blocks shares its boundary block,
    the rank's input zero-padded), each rank's shards synthesised directly (seeded random codes). bs 1: the grouped
    GEMV chain as a CUDA graph, row-parallel sums inside the GEMV over peer memory (comm) or NCCL; bs 16: the batched
    product, row-parallel partials summed by an NCCL all-reduce, launched eagerly. Device-timed; max over ranks."""
    import torch
    import torch.distributed as dist

    from pingala8_llm_b200 import synth, tp
    from pingala8_llm_b200.ops import P8Tensor, group_workspace_size, mul_mat_group, mul_mat_vec_group

    plan = tp.layer_plan(tp_dims(model), world, rank)
    shapes = layer_shapes(model)
    local = {nm: (plan[nm].shard_rows, plan[nm].shard_K) for nm, _, _ in shapes}
    layers = []
    for L in range(model["layers"]):
        ts = {}
        for i, (nm, _, _) in enumerate(shapes):
            rows, K = local[nm]
            perm_seed = 5000 * L + 17 * i + 31 if plan[nm].kind == "row" else None
            ts[nm] = P8Tensor(synth.make_slot_device(rows, K, seed=5000 * L + 17 * i + 7919 * rank, device=dev, perm_seed=perm_seed), K, rows)
        layers.append(ts)
    h = model["hidden"]
    eo = plan["o"]
    off, qn, oK = eo.lo - 256 * eo.b0, plan["q"].shard_rows, eo.shard_K
    groups = [("q", "k", "v"), ("o",), ("gate", "up"), ("down",)]
    ws = torch.empty(max(group_workspace_size([ts[n] for n in g]) for ts in layers for g in groups), dtype=torch.uint8, device=dev)
    buf = {nm: torch.empty(local[nm][0], device=dev) for nm, _, _ in shapes}
    buf["x"] = torch.randn(h, device=dev)
    oin = torch.zeros(oK, device=dev)

    def o_input(q):  # the rank's q rows placed into its o shard's blocks (zero elsewhere)
        if off == 0 and oK == qn:
            return q
        oin[off:off + qn].copy_(q)
        return oin

    def row(t, x, out, st):
        if comm is not None and world > 1:
            t.mul_mat_vec_allreduce(x, comm, out=out, workspace=ws, stream=st)
        else:
            t.mul_mat_vec(x, out=out, workspace=ws, stream=st)
            if world > 1:
                tp.reduce_partials(out)

    def step1(st):
        x = buf["x"]
        for ts in layers:
            mul_mat_vec_group([ts["q"], ts["k"], ts["v"]], x, outs=[buf["q"], buf["k"], buf["v"]], workspace=ws, stream=st)
            row(ts["o"], o_input(buf["q"]), buf["o"], st)
            mul_mat_vec_group([ts["gate"], ts["up"]], buf["o"], outs=[buf["gate"], buf["up"]], workspace=ws, stream=st)
            row(ts["down"], buf["gate"], buf["down"], st)
            x = buf["down"]

    with torch.cuda.stream(stream):
        step1(stream)
    torch.cuda.synchronize()
    g1 = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g1, stream=stream):
            step1(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    n1 = max(10, args.steps)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        for _ in range(3):
            g1.replay()
        e0.record(stream)
        for _ in range(n1):
            g1.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    t1 = e0.elapsed_time(e1) / 1e3 / n1
    del g1
    torch.cuda.synchronize()
    # bs 16: the batched product per projection, NCCL for the row-parallel partials, eager
    B = 16
    X = torch.randn(B, h, device=dev)
    Y = {nm: torch.empty(B, local[nm][0], device=dev) for nm, _, _ in shapes}
    Xo = torch.zeros(B, oK, device=dev)
    bws = torch.empty(max(group_workspace_size([ts[n] for n in g], B) for ts in layers for g in groups), dtype=torch.uint8, device=dev)

    def step16():
        x = X
        for ts in layers:
            mul_mat_group([ts["q"], ts["k"], ts["v"]], x, outs=[Y["q"], Y["k"], Y["v"]], workspace=bws)
            xo = Y["q"] if (off == 0 and oK == qn) else Xo
            if xo is Xo:
                Xo[:, off:off + qn].copy_(Y["q"])
            ts["o"].mul_mat(xo, out=Y["o"], workspace=bws)
            if world > 1:
                tp.reduce_partials(Y["o"])
            mul_mat_group([ts["gate"], ts["up"]], Y["o"], outs=[Y["gate"], Y["up"]], workspace=bws)
            ts["down"].mul_mat(Y["gate"], out=Y["down"], workspace=bws)
            if world > 1:
                tp.reduce_partials(Y["down"])
            x = Y["down"]

    step16()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n16 = 3
    e2.record()
    for _ in range(n16):
        step16()
    e3.record()
    torch.cuda.synchronize()
    t16 = e2.elapsed_time(e3) / 1e3 / n16
    tt = torch.tensor([t1, t16], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t1, t16 = tt[0].item(), tt[1].item()
    nbytes = sum(algo_bytes_gemv(r, k) for _, r, k in shapes) * model["layers"]
    return {"model": model["name"], "layers": model["layers"], "parallelism": f"tp{world}",
            "bs1": {"tok_s": round(1.0 / t1, 1), "ms_per_token": round(t1 * 1e3, 4),
                    "hbm_gbs_step_all_ranks": round(nbytes / t1 / 1e9, 1),
                    "row_parallel_sum": "inside the GEMV over peer memory" if comm is not None and world > 1 else
                                        ("NCCL all-reduce" if world > 1 else "none (1 GPU)")},
            "bs16": {"tok_s": round(B / t16, 1), "ms_per_step": round(t16 * 1e3, 3), "launch": "eager (host launches)",
                     "row_parallel_sum": "NCCL all-reduce" if world > 1 else "none (1 GPU)"},
            "o_split": {"cols": [eo.lo, eo.hi], "blocks": [eo.b0, eo.b1]},
            "weights": "seeded random class-3 codes per rank shard; the prompt phase is not part of this number"}


# ------------------------------------------------------------------------------------------------ GPU leg
def run_b200(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from pingala8_llm_b200 import synth, tp
    from pingala8_llm_b200.ops import P8Tensor, device_error, group_workspace_size, mul_mat_group, mul_mat_vec_group

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    model = LLAMA8B
    shapes = layer_shapes(model)
    # ---- tensor-parallel plan (world 1: every projection whole). Column-parallel q/k/v/gate/up keep the rank's output
    # rows, row-parallel o/down the rank's input columns (their partial outputs are summed by an NCCL all-reduce).
    dims = tp.LayerDims(hidden=model["hidden"], ffn=model["ffn"], heads=model["q"] // 128, kv_heads=model["kv"] // 128,
                        head_dim=128)
    plan = tp.layer_plan(dims, world, rank)
    local = {}  # name -> (rows, K) of this rank's shard
    for nm, rows, K in shapes:
        local[nm] = (plan[nm].shard_rows, plan[nm].shard_K)
    # ---- weights: 32 x 7 distinct slots (1.80 GB in total over the ranks), seeded per rank and layer. Each rank
    # synthesises slots of its shard's shape directly (random valid codes; the shard transforms themselves are
    # checked bit-exact in the tests)
    layers = []
    for L in range(model["layers"]):
        ts = {}
        for i, (nm, _, _) in enumerate(shapes):
            rows, K = local[nm]
            # a row-parallel shard keeps its tensor's row order on every rank (as p8_tp_shard_cols shards do)
            perm_seed = 1000 * L + 17 * i + 31 if plan[nm].kind == "row" else None
            slot = synth.make_slot_device(rows, K, seed=1000 * L + 17 * i + 7919 * rank, device=dev, perm_seed=perm_seed)
            ts[nm] = P8Tensor(slot, K, rows)
        layers.append(ts)
    groups = [("q", "k", "v"), ("o",), ("gate", "up"), ("down",)]  # tensors of a group read the same x
    reduce_after = {("o",): world > 1, ("down",): world > 1}
    ws_bytes = max(group_workspace_size([ts[n] for n in grp]) for ts in layers for grp in groups)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    h = model["hidden"]
    x0 = torch.randn(h, device=dev)
    buf = {"x": torch.empty(h, device=dev)}
    for nm in ("q", "k", "v", "o", "gate", "up", "down"):
        buf[nm] = torch.empty(local[nm][0], device=dev)

    def inputs(x):
        return {("q", "k", "v"): x, ("o",): buf["q"], ("gate", "up"): buf["o"], ("down",): buf["gate"]}

    # row-parallel sums: inside the GEMV (fused exchange over peer memory) or an NCCL all-reduce after it
    comm = (tp.TpComm.connect(max_rows=max(h, QWEN14B["hidden"]), timeout_ms=5000)
            if world > 1 and args.tp_exchange == "fused" else None)

    def call(ts, grp, src, stream):
        if comm is not None and reduce_after.get(grp):
            ts[grp[0]].mul_mat_vec_allreduce(src, comm, out=buf[grp[0]], workspace=ws, stream=stream)
            return
        mul_mat_vec_group([ts[n] for n in grp], src, outs=[buf[n] for n in grp], workspace=ws, stream=stream)
        if reduce_after.get(grp):
            tp.reduce_partials(buf[grp[0]])

    def step(stream):
        x = buf["x"]
        for ts in layers:
            src = inputs(x)
            for grp in groups:
                call(ts, grp, src[grp], stream)
            x = buf["down"]
        return x

    launches_ops = 2 * len(groups) * model["layers"]  # k_gemv + k_gemv_reduce per group
    # ---- (1 GPU) the same chain as chained launches (p8_chain: each projection one k_gemv_chain launch that reads
    # the previous one's partials). Chains split where attention sits in a real decoder layer (between q/k/v and o):
    # [q/k/v 0], [o L-1, gate/up L-1, down L-1, q/k/v L] for L = 1..31, [o 31, gate/up 31, down 31]
    chains = None
    if world == 1 and (args.decode == "chain" or not args.no_chain):
        from pingala8_llm_b200.ops import Chain

        def cstep(L, grp):
            x = {("q", "k", "v"): buf["x"] if L == 0 else buf["down"], ("o",): buf["q"], ("gate", "up"): buf["o"],
                 ("down",): buf["gate"]}[grp]
            return dict(tensors=[layers[L][n] for n in grp], x=x, outs=[buf[n] for n in grp])

        nL = model["layers"]
        plan_c = [[cstep(0, groups[0])]] + [[cstep(L - 1, g) for g in groups[1:]] + [cstep(L, groups[0])] for L in range(1, nL)]
        plan_c.append([cstep(nL - 1, g) for g in groups[1:]])
        chains = [Chain(c) for c in plan_c]
        cws = torch.empty(max(c.workspace_size() for c in chains), dtype=torch.uint8, device=dev)
    launches_per_step = len(chains) if args.decode == "chain" and chains is not None else launches_ops

    def step_chain(stream):
        for c in chains:
            c.run(workspace=cws, stream=stream)

    stream = torch.cuda.Stream(device=dev)
    buf["x"].copy_(x0)
    torch.cuda.synchronize()
    graphs = {}
    for name, fn in (("ops", step), ("chain", step_chain)):
        if name == "chain" and chains is None:
            continue
        with torch.cuda.stream(stream):
            fn(stream)  # warm-up outside capture (kernel attributes, lazy module loading)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                fn(stream)
        torch.cuda.synchronize()
        graphs[name] = g
    graph = graphs[args.decode] if args.decode in graphs else graphs["ops"]
    other = ("ops" if args.decode == "chain" else "chain") if len(graphs) > 1 else None

    def barrier():
        # the device is idle before the collective: a collective kernel that waits for other ranks must never share
        # the GPU with the persistent GEMV (its CTAs could keep a GEMV CTA from becoming resident while that GEMV's
        # peers wait for it in the fused exchange)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- device-timed steps, inputs resident
    for _ in range(args.warmup):
        graph.replay()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        # the sampler thread is polling before the timed launches start, so its start-up (NVML calls under the GIL)
        # cannot delay the enqueueing of the first replays
        time.sleep(0.05)
        e0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(args.steps):
                graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    t_dev = e0.elapsed_time(e1) / 1e3
    # ---- end to end through the op API: pinned host input in, final output out, every step
    x_host = torch.randn(h, pin_memory=True)
    y_host = torch.empty(h, pin_memory=True)
    for _ in range(args.warmup):
        with torch.cuda.stream(stream):
            buf["x"].copy_(x_host, non_blocking=True)
            graph.replay()
            y_host.copy_(buf["down"], non_blocking=True)
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(args.steps):  # the host waits for each step's output, as a decode loop reading it would
            buf["x"].copy_(x_host, non_blocking=True)
            graph.replay()
            y_host.copy_(buf["down"], non_blocking=True)
            stream.synchronize()
    e3.record(stream)
    torch.cuda.synchronize()
    barrier()
    t_e2e = e2.elapsed_time(e3) / 1e3
    # ---- the other decode path at 1 GPU (per-op calls when the headline is the chain), device-timed
    t_other = None
    if other is not None:
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                graphs[other].replay()
        torch.cuda.synchronize()
        eo0, eo1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        eo0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(args.steps):
                graphs[other].replay()
        eo1.record(stream)
        torch.cuda.synchronize()
        t_other = eo0.elapsed_time(eo1) / 1e3
    # ---- (N > 1) the step time of every rank over 200 replays (min / median / max), and the tensor-parallel path
    # against the unsharded GEMV (one layer of the headline model and of C5's Qwen3-14B; exit status 1 above the bar)
    tp_par, spread, par_fail = None, None, False
    if world > 1:
        barrier()
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(201)]
        with torch.cuda.stream(stream):
            evs[0].record(stream)
            for i in range(200):
                graph.replay()
                evs[i + 1].record(stream)
        torch.cuda.synchronize()
        per = [evs[i].elapsed_time(evs[i + 1]) for i in range(200)]
        st_ = torch.tensor([min(per), statistics.median(per), max(per)], dtype=torch.float64, device=dev)
        gathered = [torch.zeros_like(st_) for _ in range(world)]
        barrier()
        dist.all_gather(gathered, st_)
        spread = [{"rank": r, "min": round(g[0].item(), 4), "median": round(g[1].item(), 4), "max": round(g[2].item(), 4)}
                  for r, g in enumerate(gathered)]
        tp_par = {}
        for mdl in (LLAMA8B, QWEN14B) + ((UNALIGNED2,) if world == 2 else ()):
            barrier()
            errs, bar = tp_parity(mdl, world, rank, dev, comm)
            et = torch.tensor([errs[n] for n in sorted(errs)], dtype=torch.float64, device=dev)
            barrier()
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
            per_t = {n: float(f"{v:.3e}") for n, v in zip(sorted(errs), et.tolist())}
            tp_par[mdl["name"]] = {"max_rel": max(per_t.values()), "bar": bar, "per_tensor": per_t}
            par_fail = par_fail or max(per_t.values()) > bar
    c5 = None
    if not args.no_c5:
        barrier()
        c5 = tp_model_decode(QWEN14B, args, rank, world, dev, comm, stream)
        barrier()
    # ---- roofline per call type: the 32 calls of one group type (one per layer, distinct weights) captured as a
    # graph and replayed; per-call duration = replay time / 32, against the call's algorithmic bytes
    dims = dict(local)
    reps = max(3, args.steps // 4)
    per_group = {}
    for gi, grp in enumerate(groups):
        gg = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(gg, stream=stream):
                for L, ts in enumerate(layers):
                    src = inputs(buf["x"] if L == 0 else buf["down"])
                    mul_mat_vec_group([ts[n] for n in grp], src[grp], outs=[buf[n] for n in grp], workspace=ws, stream=stream)
            gg.replay()
        torch.cuda.synchronize()
        ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ea.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(reps):
                gg.replay()
        eb.record(stream)
        torch.cuda.synchronize()
        call_s = ea.elapsed_time(eb) / 1e3 / (reps * model["layers"])
        nbytes = sum(algo_bytes_gemv(*dims[n]) for n in grp) - 4 * dims[grp[0]][1] * (len(grp) - 1)
        per_group["+".join(grp)] = (call_s, nbytes)
        del gg
    # ---- (1 GPU) the projections with the elementwise ops that produce their inputs in a llama layer: RMSNorm x
    # weight -> q/k/v, o, RMSNorm x weight -> gate/up, SwiGLU -> down; fused into the GEMV's activation prep
    # (p8_mul_mat_vec_group_ex) vs the same ops as separate torch kernels before the plain GEMV. One graph per variant.
    layer = None
    if world == 1 and not args.no_layer:
        eps = 1e-5
        nw = [torch.rand(h, device=dev) + 0.5 for _ in range(2)]

        def layer_fused(stream):
            x = buf["x"]
            for ts in layers:
                mul_mat_vec_group([ts[n] for n in ("q", "k", "v")], x, outs=[buf[n] for n in ("q", "k", "v")], workspace=ws,
                                  stream=stream, norm_weight=nw[0], eps=eps)
                mul_mat_vec_group([ts["o"]], buf["q"], outs=[buf["o"]], workspace=ws, stream=stream)
                mul_mat_vec_group([ts["gate"], ts["up"]], buf["o"], outs=[buf["gate"], buf["up"]], workspace=ws,
                                  stream=stream, norm_weight=nw[1], eps=eps)
                mul_mat_vec_group([ts["down"]], buf["gate"], outs=[buf["down"]], workspace=ws, stream=stream, up=buf["up"])
                x = buf["down"]

        def layer_torch(stream):
            x = buf["x"]
            for ts in layers:
                xn = (x * torch.rsqrt(torch.mean(x * x) + eps)) * nw[0]
                mul_mat_vec_group([ts[n] for n in ("q", "k", "v")], xn, outs=[buf[n] for n in ("q", "k", "v")], workspace=ws,
                                  stream=stream)
                mul_mat_vec_group([ts["o"]], buf["q"], outs=[buf["o"]], workspace=ws, stream=stream)
                on = (buf["o"] * torch.rsqrt(torch.mean(buf["o"] * buf["o"]) + eps)) * nw[1]
                mul_mat_vec_group([ts["gate"], ts["up"]], on, outs=[buf["gate"], buf["up"]], workspace=ws, stream=stream)
                mul_mat_vec_group([ts["down"]], torch.nn.functional.silu(buf["gate"]) * buf["up"], outs=[buf["down"]],
                                  workspace=ws, stream=stream)
                x = buf["down"]

        layer = {}
        for name, fn in (("fused", layer_fused), ("torch_ops", layer_torch)):
            gl = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                fn(stream)
                torch.cuda.synchronize()
                with torch.cuda.graph(gl, stream=stream):
                    fn(stream)
            for _ in range(3):
                gl.replay()
            torch.cuda.synchronize()
            el0, el1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            nrep = max(10, args.steps // 2)
            el0.record(stream)
            with torch.cuda.stream(stream):
                for _ in range(nrep):
                    gl.replay()
            el1.record(stream)
            torch.cuda.synchronize()
            layer[name] = el0.elapsed_time(el1) / 1e3 / nrep
            del gl
    # ---- (1 GPU) batched decode: bs sequences step together through the same projection chain, each group of
    # projections on one input (q/k/v, o, gate/up, down) one grouped batched product (p8_mul_mat_group: bs 2-5 the
    # two-column batch-1 GEMV in pairs, from bs 6 one activation prep, then the split-K tcgen05 GEMM per tensor); one
    # graph per bs, device-timed
    groups = (("q", "k", "v"), ("o",), ("gate", "up"), ("down",))
    batched = None
    if world == 1 and not args.no_batched:
        batched = {}
        for bs in (2, 3, 4, 8, 32, 64):
            bws = torch.empty(max(group_workspace_size([ts[n] for n in g], bs) for ts in layers for g in groups),
                              dtype=torch.uint8, device=dev)
            bx = {"x": torch.randn(bs, h, device=dev)}
            for nm in ("q", "k", "v", "o", "gate", "up", "down"):
                bx[nm] = torch.empty(bs, local[nm][0], device=dev)
            bsrc = {"q": "x", "k": "x", "v": "x", "o": "q", "gate": "o", "up": "o", "down": "gate"}

            def bstep():
                for L, ts in enumerate(layers):
                    for g in groups:
                        src = bx[bsrc[g[0]]] if not (g[0] == "q" and L > 0) else bx["down"]
                        mul_mat_group([ts[n] for n in g], src, outs=[bx[n] for n in g], workspace=bws, stream=stream)

            gb = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                bstep()
                torch.cuda.synchronize()
                with torch.cuda.graph(gb, stream=stream):
                    bstep()
            for _ in range(3):
                gb.replay()
            torch.cuda.synchronize()
            b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            nb_ = max(5, args.steps // 5)
            b0.record(stream)
            with torch.cuda.stream(stream):
                for _ in range(nb_):
                    gb.replay()
            b1.record(stream)
            torch.cuda.synchronize()
            t_b = b0.elapsed_time(b1) / 1e3 / nb_
            batched[bs] = (t_b, bs / t_b)
            del gb, bws, bx
    # ---- prefill (batched product, tcgen05 GEMM) at 1 GPU: 512 tokens through every projection of all 32 layers
    # (1.80 GB of weights per pass, larger than L2), one CUDA graph per pass, device-timed; the projections on one
    # input as grouped products (p8_mul_mat_group, one activation prep per group), and as separate p8_mul_mat calls
    prefill = None
    if world == 1 and not args.no_prefill:
        ntok = 512
        pws = torch.empty(max(group_workspace_size([ts[n] for n in g], ntok) for ts in layers for g in groups),
                          dtype=torch.uint8, device=dev)
        Xp = {K: torch.randn(ntok, K, device=dev) for K in {k for _, _, k in shapes}}
        Yp = {n: torch.empty(ntok, r, device=dev) for n, (r, k) in local.items()}

        def pass_grouped(lys):
            for ts in lys:
                for g in groups:
                    mul_mat_group([ts[n] for n in g], Xp[ts[g[0]].K], outs=[Yp[n] for n in g], workspace=pws, stream=stream)

        def pass_separate(lys):
            for ts in lys:
                for n, tt in ts.items():
                    tt.mul_mat(Xp[tt.K], out=Yp[n], workspace=pws, stream=stream)

        t_pf = {}
        for name, fn in (("grouped", pass_grouped), ("separate", pass_separate)):
            gp = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                fn(layers[:1])
                torch.cuda.synchronize()
                with torch.cuda.graph(gp, stream=stream):
                    fn(layers)
            gp.replay()
            torch.cuda.synchronize()
            ep0, ep1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            npass = 3
            ep0.record(stream)
            with torch.cuda.stream(stream):
                for _ in range(npass):
                    gp.replay()
            ep1.record(stream)
            torch.cuda.synchronize()
            t_pf[name] = ep0.elapsed_time(ep1) / 1e3 / npass
            del gp
        flop = sum(2.0 * r * k * ntok for _, r, k in shapes) * model["layers"]
        # config C3 as stated: each projection of layer 0 alone (p8_mul_mat) at 512 and 2,048 tokens, a graph of 5
        # calls replayed twice, device-timed (one tensor's weights, so they may stay in L2: this is the GEMM alone)
        c3 = {}
        for n3 in (512, 2048):
            X3 = {K: torch.randn(n3, K, device=dev) for K in {tt.K for tt in layers[0].values()}}
            ws3 = torch.empty(max(group_workspace_size([tt], n3) for tt in layers[0].values()), dtype=torch.uint8, device=dev)
            per = {}
            for nm, tt in layers[0].items():
                Y3 = torch.empty(n3, tt.rows, device=dev)
                with torch.cuda.stream(stream):
                    tt.mul_mat(X3[tt.K], out=Y3, workspace=ws3, stream=stream)
                torch.cuda.synchronize()
                g3 = torch.cuda.CUDAGraph()
                with torch.cuda.stream(stream):
                    with torch.cuda.graph(g3, stream=stream):
                        for _ in range(5):
                            tt.mul_mat(X3[tt.K], out=Y3, workspace=ws3, stream=stream)
                    g3.replay()
                torch.cuda.synchronize()
                e30, e31 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e30.record(stream)
                with torch.cuda.stream(stream):
                    for _ in range(2):
                        g3.replay()
                e31.record(stream)
                torch.cuda.synchronize()
                t3 = e30.elapsed_time(e31) / 1e3 / 10
                per[nm] = {"us": round(t3 * 1e6, 1), "tflops": round(2.0 * tt.rows * tt.K * n3 / t3 / 1e12, 1)}
                del g3, Y3
            c3[str(n3)] = per
            del X3, ws3
        prefill = (ntok, t_pf["grouped"], flop, t_pf["separate"], c3)
    # ---- (1 GPU) model-level decode: a random-init model of the named architecture with every projection Pingala-8
    # (pingala8_llm_b200.decode: fused input ops, torch SDPA attention on a static KV cache, Q8_0 embeddings and head),
    # a seeded prompt through the batched product, then greedy tokens as graph replays; device-timed
    model_dec = None
    if world == 1 and not args.no_model:
        model_dec = {}
        from pingala8_llm_b200 import decode

        for mc, T, n_new in ((decode.QWEN3_4B, 512, 128), (decode.LLAMA31_8B, 1024, 64)):
            m = decode.Model(mc, seed=3)
            g = torch.Generator(device=dev)
            g.manual_seed(11)
            prompt = torch.randint(0, mc.vocab, (T,), device=dev, generator=g)
            m.generate(prompt[:16], 4)  # capture the step graph, warm every path
            m.alloc(T + n_new)
            m.capture()
            m.kv.zero_()
            ep0, ep1, ep2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            torch.cuda.synchronize()
            with torch.cuda.stream(m.stream):
                ep0.record(m.stream)
                lg = m.prefill(prompt)
                ep1.record(m.stream)
                m.tok.copy_(torch.argmax(lg).view(1))
                m.pos.fill_(T)
                for _ in range(n_new):
                    m.graph.replay()
                    m.pos += 1
                ep2.record(m.stream)
            torch.cuda.synchronize()
            t_pf, t_dec = ep0.elapsed_time(ep1) / 1e3, ep1.elapsed_time(ep2) / 1e3
            pbytes = sum(algo_bytes_gemv(r, k) for _, r, k in decode.proj_shapes(mc)) * mc.layers
            model_dec[mc.name] = {
                "layers": mc.layers, "prompt_tokens": T, "new_tokens": n_new, "prefill_ms": round(t_pf * 1e3, 2),
                "prefill_tok_s": round(T / t_pf, 1), "decode_tok_s": round(n_new / t_dec, 1),
                "decode_ms_per_token": round(1e3 * t_dec / n_new, 3),
                "pingala8_bytes_per_token": pbytes, "head_bytes_per_token": mc.vocab * mc.hidden * 2}
            del m
            torch.cuda.empty_cache()
    # ---- max over ranks
    gnames = list(per_group)
    times = torch.tensor([t_dev, t_e2e] + [per_group[g][0] for g in gnames], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    t_dev, t_e2e = times[0].item(), times[1].item()
    del graph
    graphs.clear()
    torch.cuda.synchronize()
    derr = device_error()
    if derr:
        raise RuntimeError(f"a kernel gave up on a bounded wait (device error bits {derr:#x}): results invalid")
    if comm is not None:  # no kernel of any rank uses the exchange buffers past this barrier
        dist.barrier()
        comm.close()
    for i, g in enumerate(gnames):
        per_group[g] = (times[2 + i].item(), per_group[g][1])
    bytes_token = sum(algo_bytes_gemv(r, k) for _, r, k in shapes) * model["layers"]
    if rank != 0:
        return 1 if par_fail else 0
    peak, peak_kind = measured_peaks()
    # dominant call type by device time per step
    dom = max(gnames, key=lambda g: per_group[g][0])
    dom_s, dom_bytes = per_group[dom]
    achieved = dom_bytes / dom_s / 1e9
    per_call = {g: {"us": round(per_group[g][0] * 1e6, 3), "gbs": round(per_group[g][1] / per_group[g][0] / 1e9, 1)}
                for g in gnames}
    if args.decode == "chain" and chains is not None:  # the step is nothing but chain launches: the kernel's bytes and time are the step's
        dom_s = t_dev / args.steps / len(chains)
        dom_bytes = bytes_token / len(chains)
        roof = {"kernel": f"p8_chain_run ({len(chains)} chains per token, 4 projections per chain in layers 1-31; "
                          f"k_gemv_chain per projection, k_gemv_reduce per chain)", "bound": "hbm", "achieved": round(dom_bytes / dom_s / 1e9, 1), "peak": peak,
                "unit": "GB/s", "frac": round(dom_bytes / dom_s / 1e9 / peak, 4),
                "traffic": TRAFFIC_BYTES.get("chain"), "algorithmic_bytes": round(dom_bytes), "call_us": round(dom_s * 1e6, 3),
                "peak_source": peak_kind,
                "timing": "CUDA events around graph replays of the whole step; every kernel of the step is a chain launch"}
    else:
        roof = {"kernel": f"p8_mul_mat_vec_group {dom} (k_gemv + k_gemv_reduce)", "bound": "hbm", "achieved": round(achieved, 1),
                "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "traffic": TRAFFIC_BYTES.get(dom) if world == 1 else None, "algorithmic_bytes": dom_bytes,
                "call_us": round(dom_s * 1e6, 3), "peak_source": peak_kind,
                "per_call_type": per_call}
    tok_s = args.steps / t_dev  # one token stream; with N GPUs every token is split over the ranks (strong scaling)
    line = {
        "metric": METRIC, "value": round(tok_s, 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * t_dev / args.steps, 4), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "int32+fp32 (x16 activations)", "data": "synthetic (seeded random valid Pingala-8 codes, class 3)",
        "config": {"workload": "llama3.1-8b-bs1-decode-projections", "layers": model["layers"], "projections_per_layer": 7,
                   "batch": 1, "classes": "3", "parallelism": f"tp{world}" if world > 1 else "single",
                   "tp": (("column-parallel q/k/v/gate/up, row-parallel o/down summed inside the GEMV "
                           "(p8_tp_gemv_allreduce: peer stores over NVLink, rank-order sum)") if comm is not None else
                          "column-parallel q/k/v/gate/up, row-parallel o/down + NCCL all-reduce (fp32, 16 KB) after each")
                         if world > 1 else None,
                   "weight_bytes_per_token": bytes_token, "l2": "inputs larger than L2 (1.80 GB of weights streamed per step)",
                   "hbm_gbs_step": round(bytes_token / (t_dev / args.steps) / 1e9, 1)},
        "roofline": roof,
        "e2e": {"value": round(args.steps / t_e2e, 3), "unit": "tok/s", "h2d_bytes_per_step": 4 * h, "d2h_bytes_per_step": 4 * h},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    if t_other is not None and other == "ops":
        line["per_op_decode"] = {"tok_s": round(args.steps / t_other, 3), "ms_per_step": round(1e3 * t_other / args.steps, 4),
                                 "kernels": "p8_mul_mat_vec_group per group call (k_gemv + k_gemv_reduce), 256 launches per token",
                                 "per_call_type": per_call}
    if t_other is not None and other == "chain":
        line["chain_decode"] = {"tok_s": round(args.steps / t_other, 3), "ms_per_step": round(1e3 * t_other / args.steps, 4),
                                "kernels": f"p8_chain_run: {len(chains)} chains per token (the projections between two attention "
                                           "points), each projection one k_gemv_chain launch that reads its input from the "
                                           "previous one's partials, one k_gemv_reduce after a chain's last projection",
                                "hbm_gbs_step": round(bytes_token / (t_other / args.steps) / 1e9, 1)}
    if tp_par is not None:
        line["tp_parity"] = {"what": "one layer's q, gate (column-parallel) and o, down (row-parallel) sharded by the plan "
                                     "and run through the TP path, against the unsharded GEMV on the same GPU; relative "
                                     "L2, max over ranks", **tp_par}
    if spread is not None:
        line["per_rank_step_ms"] = {"steps": 200, "ranks": spread}
    if c5 is not None:
        line["c5_tp_decode"] = c5
    if model_dec is not None:
        line["model_decode"] = {
            "what": "random-init model, every projection Pingala-8 class 3 (p8_mul_mat_vec_group with fused RMSNorm / "
                    "SwiGLU; the prompt via p8_mul_mat_group), torch SDPA attention on a static KV cache, Q8_0 "
                    "embeddings and head (fp16 head GEMV), greedy; one decode step = one CUDA graph replay",
            "parity": "tests/test_gpu_decode.py: logits within 5e-3 of an fp32 torch forward on the oracle's dequantised "
                      "weights", **model_dec}
    if batched is not None:
        line["batched_decode"] = {
            "kernel": "p8_mul_mat_group per input: bs 2-5 k_gemv2 + k_gemv_reduce2 (two columns per launch, an odd column "
                      "through k_gemv); from bs 6 k_gx_max + k_gx_prep once, then k_gemm + k_splitk_reduce per projection",
            "per_bs": {str(bs): {"ms_per_step": round(t * 1e3, 3), "tok_s": round(v, 1),
                                 "weight_gbs": round(bytes_token / t / 1e9, 1)} for bs, (t, v) in batched.items()}}
    if layer is not None:
        line["layer_prologues"] = {
            "ops": "RMSNorm*w -> q,k,v; o; RMSNorm*w -> gate,up; SwiGLU -> down (x 32 layers, graph-replayed, device-timed)",
            "fused_tok_s": round(1.0 / layer["fused"], 1), "torch_ops_tok_s": round(1.0 / layer["torch_ops"], 1),
            "fused": "p8_mul_mat_vec_group_ex (input op in k_gemv's table build)",
            "torch_ops": "separate torch elementwise/reduction kernels, then p8_mul_mat_vec_group"}
    if prefill is not None:
        ntok, t_pass, flop, t_sep, c3 = prefill
        bf16_peak, bf16_kind = measured_bf16_tflops()
        line["prefill"] = {"tokens": ntok, "ms": round(t_pass * 1e3, 3), "tok_s": round(ntok / t_pass, 1),
                           "kernel": "p8_mul_mat_group per input (k_gx_max + k_gx_prep once; k_gemm, tcgen05 kind::f16, "
                                     "fp32 accumulate, + k_unpermute per projection)",
                           "separate_calls": {"ms": round(t_sep * 1e3, 3), "tflops": round(flop / t_sep / 1e12, 1),
                                              "kernel": "p8_mul_mat per projection"},
                           "tflops": round(flop / t_pass / 1e12, 1), "bound": "tensor", "peak_tflops": bf16_peak,
                           "frac": round(flop / t_pass / 1e12 / bf16_peak, 4),
                           "peak_source": bf16_kind + "; the GEMM runs fp16 operands at the bf16 rate",
                           "config": "512 tokens x 224 projections (32 layers), distinct weights, inputs resident",
                           "c3_per_gemm": {"what": "config C3: each projection alone (p8_mul_mat), per call; tflops of "
                                                   "2 x rows x K x tokens", "tokens": c3}}
    if world == 1 and not args.no_cpu:
        tok_time, cores, isa = cpu_reference_token(model, reps=5, warmup=1)
        line["cpu_baseline"] = {"value": round(1.0 / tok_time, 4), "unit": "tok/s", "cores": cores, "kind": "reference",
                                "sample": f"5 tokens, each all {model['layers'] * 7} projections (distinct slots, 1.80 GB), median; "
                                          f"{isa} vr-native-cpu-core.h, {cores} OpenMP threads"}
    print(json.dumps(line), flush=True)
    return 1 if par_fail else 0


# ------------------------------------------------------------------------------------------------ profiling cases
# One kernel family on one shape, repeated: small self-contained cases for ncu captures and quick timings
# (python bench.py --case ...). Weights are seeded synthetic class-3 slots of the Llama-3.1-8B shapes.
CASE_GROUPS = {  # Llama-3.1-8B: (rows, K) per tensor of a group that reads one x
    "qkv": [(4096, 4096), (1024, 4096), (1024, 4096)],
    "o": [(4096, 4096)],
    "gate_up": [(14336, 4096), (14336, 4096)],
    "down": [(4096, 14336)],
}


def run_case(args):
    """--case gemv:GROUP          the grouped batch-1 GEMV (k_gemv + k_gemv_reduce), --iters calls rotating over --copies
                                  distinct weight copies (copies > 1 read DRAM rather than L2), optionally --graph
       --case gemv2:GROUP         the grouped product of two columns (two sequences: k_gemv2 + k_gemv_reduce2)
       --case gemm:GROUP:NCOLS    the batched product per tensor (tcgen05 GEMM), or :grouped for p8_mul_mat_group
       --case get_rows:GROUP:N    p8_get_rows of N random rows of each tensor of the group
       --case dequant:GROUP       p8_dequant_f32 of each tensor of the group
       --case encode:ROWS         the offline trellis encoder (k_vit) on ROWS x 4096 class 3 with a random Hessian
    Prints the mean time per call (CUDA events)."""
    import torch

    from pingala8_llm_b200 import synth
    from pingala8_llm_b200.ops import P8Tensor, group_workspace_size, mul_mat_group, mul_mat_vec_group

    kind, *rest = args.case.split(":")
    if kind == "encode":
        return _case_encode(int(rest[0]), args.iters)
    if kind == "chain":
        return _case_chain(int(rest[0]) if rest else 8, args)
    if kind == "chain_tiny":
        return _case_chain_tiny(int(rest[0]), int(rest[1]), int(rest[2]), args)
    shapes = CASE_GROUPS[rest[0]]
    copies = [[P8Tensor(synth.make_slot_device(r, k, seed=100 * c + i), k, r) for i, (r, k) in enumerate(shapes)]
              for c in range(max(1, args.copies))]
    K = shapes[0][1]
    if kind == "gemv":
        x = torch.randn(K, device="cuda")
        outs = [torch.empty(r, device="cuda") for r, _ in shapes]
        ws = torch.empty(max(group_workspace_size(ts) for ts in copies), dtype=torch.uint8, device="cuda")

        def once(i, stream=None):
            mul_mat_vec_group(copies[i % len(copies)], x, outs=outs, workspace=ws, stream=stream)
        nbytes = sum((r // 32) * (k // 256) * (68 + 2048) for r, k in shapes)
        unit = lambda us: f"{nbytes / us / 1e3:.1f} GB/s (algorithmic, class 3)"  # noqa: E731
    elif kind == "gemv2":
        X = torch.randn(2, K, device="cuda")
        outs = [torch.empty(2, r, device="cuda") for r, _ in shapes]
        ws = torch.empty(max(group_workspace_size(ts, 2) for ts in copies), dtype=torch.uint8, device="cuda")

        def once(i, stream=None):
            mul_mat_group(copies[i % len(copies)], X, outs=outs, workspace=ws, stream=stream)
        nbytes = sum((r // 32) * (k // 256) * (68 + 2048) for r, k in shapes)
        unit = lambda us: f"{nbytes / us / 1e3:.1f} GB/s of weights (algorithmic, class 3, read once for both columns)"  # noqa: E731
    elif kind == "gemm":
        ncols = int(rest[1])
        grouped = len(rest) > 2 and rest[2] == "grouped"
        X = torch.randn(ncols, K, device="cuda")
        outs = [torch.empty(ncols, r, device="cuda") for r, _ in shapes]
        gws = torch.empty(max(max(group_workspace_size(ts, ncols) for ts in copies), 256), dtype=torch.uint8, device="cuda")

        def once(i, stream=None):
            ts = copies[i % len(copies)]
            if grouped:
                mul_mat_group(ts, X, outs=outs, workspace=gws, stream=stream)
            else:
                for t, y in zip(ts, outs):
                    t.mul_mat(X, out=y, workspace=gws, stream=stream)
        flop = sum(2.0 * r * k * ncols for r, k in shapes)
        unit = lambda us: f"{flop / us / 1e6:.1f} TFLOP/s"  # noqa: E731
    elif kind == "get_rows":
        n = int(rest[1])
        ids = [torch.randint(0, r, (n,), dtype=torch.int32, device="cuda") for r, _ in shapes]
        outs = [torch.empty(n, K, device="cuda") for _ in shapes]

        def once(i, stream=None):
            for t, d, o in zip(copies[i % len(copies)], ids, outs):
                t.get_rows(d, out=o, stream=stream)
        nbytes = sum(n * (K // 256) * (2048 + 2 + 4 + K // (K // 256) * 4) for _ in shapes)
        unit = lambda us: f"{nbytes / us / 1e3:.1f} GB/s (rows' tiles + f32 out)"  # noqa: E731
    elif kind == "dequant":
        outs = [torch.empty(r, k, device="cuda") for r, k in shapes]

        def once(i, stream=None):
            for t, o in zip(copies[i % len(copies)], outs):
                t.dequant(out=o, stream=stream)
        nbytes = sum((r // 32) * (k // 256) * (68 + 2048) + 4 * r * k for r, k in shapes)
        unit = lambda us: f"{nbytes / us / 1e3:.1f} GB/s (slot + f32 out)"  # noqa: E731
    else:
        raise SystemExit(f"unknown case {args.case}")
    for i in range(len(copies)):  # warm-up
        once(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.graph:
        st = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                for i in range(args.iters):
                    once(i, stream=st)
        g.replay()
        torch.cuda.synchronize()
        e0.record(st)
        g.replay()
        e1.record(st)
    else:
        e0.record()
        for i in range(args.iters):
            once(i)
        e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.iters
    print(f"case {args.case}: {us:.2f} us/call, {unit(us)}", flush=True)
    return 0


def _case_chain(nlayers, args):
    """--case chain:L  the decode chain of L Llama-3.1-8B layers as per-layer p8_chain launches (split at the attention
    boundary, as the bench's headline step), timed; with --trace, the per-step phase stamps of one mid-layer launch
    (globaltimer, per CTA) summarised as median / max over CTAs"""
    import torch

    from pingala8_llm_b200 import synth
    from pingala8_llm_b200.ops import Chain, P8Tensor

    shapes = layer_shapes(LLAMA8B)
    layers = [{n: P8Tensor(synth.make_slot_device(r, k, seed=1000 * L + 17 * i), k, r) for i, (n, r, k) in enumerate(shapes)}
              for L in range(nlayers)]
    buf = {n: torch.empty(r, device="cuda") for n, r, _ in shapes}
    buf["x"] = torch.randn(4096, device="cuda")
    groups = [("q", "k", "v"), ("o",), ("gate", "up"), ("down",)]

    def cstep(L, grp):
        x = {("q", "k", "v"): buf["x"] if L == 0 else buf["down"], ("o",): buf["q"], ("gate", "up"): buf["o"],
             ("down",): buf["gate"]}[grp]
        return dict(tensors=[layers[L][n] for n in grp], x=x, outs=[buf[n] for n in grp])

    plan = [[cstep(0, groups[0])]] + [[cstep(L - 1, g) for g in groups[1:]] + [cstep(L, groups[0])] for L in range(1, nlayers)]
    plan.append([cstep(nlayers - 1, g) for g in groups[1:]])
    chains = [Chain(c) for c in plan]
    ws = torch.empty(max(c.workspace_size() for c in chains), dtype=torch.uint8, device="cuda")
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        for c in chains:
            c.run(workspace=ws, stream=st)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            for c in chains:
                c.run(workspace=ws, stream=st)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):  # replays run on the current stream
        e0.record(st)
        for _ in range(args.iters):
            g.replay()
        e1.record(st)
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / args.iters
    nbytes = sum(algo_bytes_gemv(r, k) for _, r, k in shapes) * nlayers
    out = {"case": args.case, "us_per_token": round(t * 1e6, 2), "launches": len(chains),
           "us_per_mid_launch": round(t * 1e6 / len(chains), 2), "gbs": round(nbytes / t / 1e9, 1)}
    if args.trace:
        mid = chains[len(chains) // 2]
        nsm = torch.cuda.get_device_properties(0).multi_processor_count
        tb = torch.zeros(4 * nsm * 8, dtype=torch.int64, device="cuda")
        mid.trace(tb)
        g2 = torch.cuda.CUDAGraph()  # the traced run inside the same sequence of launches (same cache state)
        with torch.cuda.stream(st):
            with torch.cuda.graph(g2, stream=st):
                for c in chains:
                    c.run(workspace=ws, stream=st)
        with torch.cuda.stream(st):
            g2.replay()
        torch.cuda.synchronize()
        mid.trace(None)
        T = tb.view(4, nsm, 8).cpu().numpy().astype(np.float64)
        # stamps of the chained steps (1..3; the first step reads memory and is not stamped): [0] past the wait,
        # [2] inputs ready, [3] tables built, [4] units done, [5] the previous step's unread rows reduced
        live = T[1:, :, 0] > 0
        t0 = T[1:, :, 0][live].min()
        phases = {}
        spans = [("inputs", 0, 2), ("tables", 2, 3), ("units", 3, 4), ("unread_rows", 4, 5)]
        if (T[1:, :, 6] > 0).any():  # a build that also stamps inside the table build: [6] x16 ints ready, [7] coset ready
            spans += [("fwht_q", 2, 6), ("coset", 6, 7), ("table_fill", 7, 3)]
        for sidx in range(1, 4):
            ok = T[sidx, :, 0] > 0
            d = {nm: [round(float(np.median(T[sidx, ok, b] - T[sidx, ok, a])) / 1e3, 3),
                      round(float(np.max(T[sidx, ok, b] - T[sidx, ok, a])) / 1e3, 3)] for nm, a, b in spans}
            d["start_us"] = [round(float(T[sidx, ok, 0].min() - t0) / 1e3, 3), round(float(T[sidx, ok, 0].max() - t0) / 1e3, 3)]
            d["end_us"] = round(float(T[sidx, ok, 5].max() - t0) / 1e3, 3)
            phases[f"step{sidx}"] = d
        out["trace_median_max_us"] = phases
    print(json.dumps(out), flush=True)
    return 0


def _case_chain_tiny(nsteps, rows, K, args):
    """--case chain_tiny:S:R:K  one launch of S chained square-ish steps (R x K, R == K) whose units are few: the
    per-step fixed cost of the chain (barrier, prep, tables) with the trace's phase medians"""
    import torch

    from pingala8_llm_b200 import synth
    from pingala8_llm_b200.ops import Chain, P8Tensor

    assert rows == K
    ts = [P8Tensor(synth.make_slot_device(rows, K, seed=i), K, rows) for i in range(nsteps)]
    bufs = [torch.randn(K, device="cuda")] + [torch.empty(rows, device="cuda") for _ in range(nsteps)]
    ch = Chain([dict(tensors=[ts[i]], x=bufs[i], outs=[bufs[i + 1]]) for i in range(nsteps)])
    ws = torch.empty(ch.workspace_size(), dtype=torch.uint8, device="cuda")
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        ch.run(workspace=ws, stream=st)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):
        e0.record(st)
        for _ in range(args.iters):
            ch.run(workspace=ws, stream=st)
        e1.record(st)
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / args.iters
    out = {"case": args.case, "us_per_launch": round(t * 1e6, 2), "us_per_step": round(t * 1e6 / nsteps, 3)}
    if args.trace:
        nsm = torch.cuda.get_device_properties(0).multi_processor_count
        tb = torch.zeros(nsteps * nsm * 8, dtype=torch.int64, device="cuda")
        ch.trace(tb)
        with torch.cuda.stream(st):
            ch.run(workspace=ws, stream=st)
        torch.cuda.synchronize()
        T = tb.view(nsteps, nsm, 8).cpu().numpy().astype(np.float64)
        mid = T[1:-1]
        med = lambda a: round(float(np.median(a)) / 1e3, 3)  # noqa: E731
        has = mid[:, :, 3] > 0
        out["phase_median_us"] = {"inputs": med((mid[:, :, 2] - mid[:, :, 0])[has]),
                                  "tables": med((mid[:, :, 3] - mid[:, :, 2])[has]),
                                  "units": med((mid[:, :, 4] - mid[:, :, 3])[has]),
                                  "unread_rows": med(mid[:, :, 5] - mid[:, :, 4]),
                                  "step_to_step": med(T[2:, :, 0].min(1) - T[1:-1, :, 0].min(1))}
    print(json.dumps(out), flush=True)
    return 0


def _case_encode(rows, iters):
    import torch

    from pingala8_llm_b200.encoder import encode

    n = 4096
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
    for _ in range(iters):
        encode(Y, Uc, cls, Sb)
    e1.record()
    torch.cuda.synchronize()
    dt = e0.elapsed_time(e1) / 1e3 / iters
    print(f"case encode:{rows}: {dt * 1e3:.3f} ms per {rows} x {n} tensor, {dt / (rows * n) * 1e9:.3f} ns per weight")
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-prefill", action="store_true", help="skip the batched-product (prefill) measurement")
    ap.add_argument("--no-layer", action="store_true", help="skip the fused-prologue layer measurement")
    ap.add_argument("--no-batched", action="store_true", help="skip the batched-decode (bs 8/32/64) measurement")
    ap.add_argument("--no-chain", action="store_true", help="skip the chained-launch decode measurement")
    ap.add_argument("--no-model", action="store_true", help="skip the model-level decode (C2 Qwen3-4B, Llama-3.1-8B)")
    ap.add_argument("--no-c5", action="store_true", help="skip the C5 Qwen3-14B tensor-parallel decode block")
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="--impl reference: skip the reference's own CUDA GEMV timed on this GPU beside its CPU core")
    ap.add_argument("--decode", default="ops", choices=["chain", "ops"],
                    help="1 GPU decode path timed as the headline: chained launches (p8_chain) or per-op group calls")
    ap.add_argument("--tp-exchange", default="fused", choices=["fused", "nccl"],
                    help="row-parallel sum for N > 1: inside the GEMV over peer memory, or an NCCL all-reduce after it")
    ap.add_argument("--case", default="", help="run one profiling case instead of the bench (see run_case)")
    ap.add_argument("--iters", type=int, default=20, help="--case: calls timed")
    ap.add_argument("--copies", type=int, default=1, help="--case: distinct weight copies the calls rotate over")
    ap.add_argument("--graph", action="store_true", help="--case: capture the calls in a CUDA graph")
    ap.add_argument("--trace", action="store_true", help="--case chain: per-step phase stamps of one launch")
    args = ap.parse_args()
    if args.case:
        return run_case(args)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
    try:
        return run_b200(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
