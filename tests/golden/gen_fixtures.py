"""Generate the golden fixtures in tests/golden/ with the REFERENCE's own Python encoder and CPU core.

Run in the build container only (it imports research/detail/*.py from the reference checkout and needs the
reference CPU core built by oracle/build_ref.py). The outputs are committed; nothing at test time reads the
reference checkout.

Pipeline per fixture (the reference's own steps):
  weights  W = N(0, 0.02^2) from numpy default_rng(seed); entries with rand < 1e-3 replaced by standard_t(3) * 0.1
  encode   r48k.k_tensor (research/detail/r48k.py:213) with R48K_NS=8, R48K_SHIFTS=0,0,0,0,2,3,2,4/0,0,0,0,0,0,0,2,
           c = 1 (uniform importance matrix), H = I, damp 0.1, alpha 1.05, tables research/work/r48k3/tables_vrc.pt
  blob     r48k.pack_blob -> r48k.relayout (VRK2) -> r51_transcode.transcode (kernel bytes, r51_transcode.py:33)
  delta    r51_delta.py: entries of W' = ifw(Yq)/c with |W'| > wmax, value clamp(W') - W'
  slot     assembled as the reference loader does (llama-model-loader.cpp vr_native_load, CU:3527-3580):
           kernel bytes | ... | E delta | C c16 | P prm | Q pinv | SG signs | trailer, offsets top-down (CU:30-37),
           slot size = smallest of IQ2_XXS, Q2_K..Q6_K rows with nbytes >= vrn_need (CU:3493-3497)
Golden values stored: the slot bytes, seeded activations, the reference CPU core's x16 GEMV / batch outputs
(oracle/_ref), and SHA-256 digests of the reference Python decoders' outputs (r51_transcode.cpu_vr_port over the
kernel bytes = v*S in sorted rows; r48k.unpack_blob + ifw/c = original-domain weights).

usage: python tests/golden/gen_fixtures.py [--reference REFERENCE_CHECKOUT]
"""
import argparse
import hashlib
import json
import os
import struct
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))

SLOTS = [("IQ2_XXS", 66), ("Q2_K", 84), ("Q3_K", 110), ("Q4_K", 144), ("Q5_K", 176), ("Q6_K", 210)]
RATES = [0, 1, 1.5, 2, 2.5, 3, 4, 6]


def a16(n):
    return (n + 15) & ~15


def need(kbytes, rows, K, nd):  # CU:27-29
    return a16(kbytes) + a16(8 * nd) + a16(2 * K) + 2 * a16(2 * rows) + 256 + 32 + 64


def offsets(n, rows, K, nd):  # CU:30-37
    offT = n - 32
    offSG = offT - 256
    offQ = (offSG - 2 * rows) & ~15
    offP = (offQ - 2 * rows) & ~15
    offC = (offP - 2 * K) & ~15
    offE = (offC - 8 * nd) & ~15
    return offE, offC, offP, offQ, offSG, offT


def assemble_slot(kb, rows, K, c16, prm, drow, dcol, dval, signs):
    """llama-model-loader.cpp vr_native_load (CU:3527-3580) restated in numpy."""
    nd = len(dval)
    nd_need = need(len(kb), rows, K, nd)
    for name, bpb in SLOTS:
        n = rows * (K // 256) * bpb
        if n >= nd_need:
            break
    else:
        raise ValueError("no slot type fits")
    buf = np.zeros(n, np.uint8)
    buf[: len(kb)] = np.frombuffer(kb, np.uint8)
    offE, offC, offP, offQ, offSG, offT = offsets(n, rows, K, nd)
    assert len(kb) <= offE
    buf[offC : offC + 2 * K] = np.asarray(c16, np.float16).view(np.uint8)
    prm16 = np.asarray(prm, np.int16)
    buf[offP : offP + 2 * rows] = prm16.view(np.uint8)
    pinv = np.empty(rows, np.int16)
    pinv[prm16.astype(np.int64)] = np.arange(rows, dtype=np.int16)
    buf[offQ : offQ + 2 * rows] = pinv.view(np.uint8)
    if nd:
        buf[offE : offE + 2 * nd] = np.asarray(drow, np.uint16).view(np.uint8)
        buf[offE + 2 * nd : offE + 4 * nd] = np.asarray(dcol, np.uint16).view(np.uint8)
        buf[offE + 4 * nd : offE + 8 * nd] = np.asarray(dval, np.float32).view(np.uint8)
    buf[offSG : offSG + 256] = np.asarray(signs, np.int8).view(np.uint8)
    tr = struct.pack("<8I", 0x4E525656, 0x31354952, len(kb), nd, rows, K, 108, 1)
    buf[offT : offT + 32] = np.frombuffer(tr, np.uint8)
    return buf, name


def sha(a):
    """digest of a float array by VALUE: -0.0 and +0.0 hash alike (the reference decoders disagree on zero signs)"""
    a = np.ascontiguousarray(a)
    if a.dtype.kind == "f":
        a = a + a.dtype.type(0)
    return hashlib.sha256(a.tobytes()).hexdigest()


def weights(rows, n, seed, flat_outliers=False):
    rng = np.random.default_rng(seed)
    W = rng.normal(0, 0.02, (rows, n))
    m = rng.random((rows, n)) < 1e-3
    W[m] = rng.standard_t(3, int(m.sum())) * 0.1
    if flat_outliers:  # every outlier at the same magnitude: many of them decode past the clamp bound max|W|
        W[m] = np.sign(W[m]) * 0.3
    return W.astype(np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    os.environ["R48K_NS"] = "8"
    os.environ["R48K_SHIFTS"] = "0,0,0,0,2,3,2,4/0,0,0,0,0,0,0,2"
    sys.path.insert(0, os.path.join(a.reference, "research", "detail"))
    sys.path.insert(0, REPO)
    import torch
    import r48k as K_
    import r52a_k as RK
    import r51_transcode as TC
    import r48_a1gpu as A1
    from oracle.oracle import RefOracle

    torch.set_num_threads(os.cpu_count())
    RK.set_ns(8)
    tab_dir = os.path.join(a.reference, "research", "work", "r48k3")
    T = torch.load(os.path.join(tab_dir, "tables_vrc.pt"))
    J = json.load(open(os.path.join(tab_dir, "tables_vrc.json")))
    G = {int(x): y for x, y in J["G"].items()}
    CD = torch.tensor([J["D"][str(i)] for i in range(8)], dtype=torch.float64)
    tab = RK.tables_blob(T, True)
    fw, ifw = A1.make_fw("cpu")
    g0 = torch.Generator().manual_seed(0)
    signs = (torch.randint(0, 2, (256,), generator=g0) * 2 - 1).numpy().astype(np.int8)  # r48_a1gpu.make_fw seed 0

    specs = [
        # name, rows, K, weight seed, rate (b/w) or None for rate-on allocation, nsal
        ("c1_1024x2560_c3", 1024, 2560, 0, 2.0, 0),
        ("mix_256x1024_sal", 256, 1024, 5, None, 4),
    ] + [(f"cls{k}_64x512", 64, 512, 10 + k, RATES[k], 0) for k in range(1, 7)] + [
        # class 7 (6 b/w) needs a larger tensor to fit a Q6_K slot together with its side data
        ("cls7_256x1024", 256, 1024, 17, RATES[7], 0),
        # config C1 at its stated size (Qwen3-4B ffn_up 9728 x 2560, seed 0): pure class 3, and class 3 with four
        # salient class-6 tiles per row group
        ("c1_9728x2560_c3", 9728, 2560, 0, 2.0, 0),
        ("c1_9728x2560_sal", 9728, 2560, 0, None, 4),
    ]
    # clamp-delta coverage: the C1 recipe leaves no decoded weight past the clamp bound (nd = 0 at both sizes), so this
    # case sets every outlier to the same magnitude 0.3: decoded outliers then overshoot the fp16 bound max|W| * 1.001
    # about half the time, and the slot carries the reference pipeline's own delta entries (r51_delta.py semantics)
    specs_alpha = {}
    flat = {"dl_2048x2560_c3"}
    specs += [("dl_2048x2560_c3", 2048, 2560, 3, 2.0, 0)]
    if a.only:
        specs = [s for s in specs if s[0] in a.only.split(",")]
    index = {}
    for name, rows, n, seed, rate, nsal in specs:
        t0 = time.time()
        W = torch.tensor(weights(rows, n, seed, flat_outliers=name in flat))
        c = torch.ones(n)
        Hf = torch.eye(n)
        sw = torch.ones(n)
        RK.RATEOFF[0] = rate is not None
        r = rate if rate is not None else 2.0

        def bud(r_, n_, r=r):
            return r * r_ * n_

        R = K_.k_tensor(W, c, Hf, sw, bud, T, CD, G, True, alpha=specs_alpha.get(name, 1.05), dev="cpu", damp=0.1, nsal=nsal)
        blob = K_.pack_blob(c.half().numpy(), R["prm"], R["S16"].numpy(), R["cs"], R["IDX"].cpu().numpy(), R["wmax"], True)
        hdr, Yd = K_.unpack_blob(blob, T)
        assert torch.equal(Yd, R["Yq"].cpu())
        b2 = K_.relayout(blob)
        kb, side = TC.transcode(b2, tab)
        # reference decoders: numpy port of the CUDA bit-level decoder (sorted rows, v*S) and r48k's own unpack
        port = TC.cpu_vr_port(kb, rows, n)
        h2, Yq = K_.unpack_blob(b2, T)
        assert np.array_equal(port, Yq[h2["prm"]].numpy()), "reference decoders disagree"  # == (signed zeros differ)
        Wp = ifw(Yq) / h2["c"]  # original-domain weights before the clamp (r51_delta.py)
        wm = h2["wmax"]
        rr, cc = torch.nonzero(Wp.abs() > wm, as_tuple=True)
        w = Wp[rr, cc]
        dval = (w.clamp(-wm, wm) - w).numpy().astype(np.float32)
        Wq = Wp.clamp(-wm, wm).numpy().astype(np.float32)  # the encoder's clamped weights (k_tensor Wq)
        slot, slot_type = assemble_slot(kb, rows, n, side["c16"], side["prm"], rr.numpy(), cc.numpy(), dval, signs)
        # activations
        x = np.random.default_rng(1).normal(0, 1, n).astype(np.float32)
        X = np.random.default_rng(2).normal(0, 1, (8, n)).astype(np.float32)
        ref = RefOracle(slot, rows, n)
        y_ref = ref.gemv(x)
        Y_ref = ref.mul_mat(X)
        W_ref = ref.dequant()
        hist = np.bincount((np.frombuffer(kb, "<u4", (rows // 32) * (n // 256), 2064) >> 29).astype(np.int64), minlength=8).tolist()
        slot.tofile(os.path.join(HERE, f"{name}.slot"))
        np.save(os.path.join(HERE, f"{name}.x.npy"), x)
        np.save(os.path.join(HERE, f"{name}.X.npy"), X)
        np.save(os.path.join(HERE, f"{name}.y_ref.npy"), y_ref)
        np.save(os.path.join(HERE, f"{name}.Y_ref.npy"), Y_ref)
        meta = dict(
            name=name, rows=rows, K=n, seed=seed, rate=rate, nsal=nsal, alpha=specs_alpha.get(name, 1.05), flat_outliers=name in flat,
            nd=int(len(dval)),
            kbytes=len(kb),
            slot_type=slot_type, slot_nbytes=int(slot.size), class_hist=hist, wmax=float(wm),
            sha_port_vs=sha(port),              # r51_transcode.cpu_vr_port: v*S fp32, sorted rows
            sha_wq_clamped=sha(Wq),             # encoder: clamp(ifw(Yq)/c), original rows
            sha_ref_dequant=sha(W_ref),         # reference CPU core vrc_dequant_f32
            ref_dequant_eq_wq=bool(np.array_equal(W_ref, Wq)),
            ref_dequant_maxdiff_wq=float(np.abs(W_ref - Wq).max()),
            ref_isa=RefOracle.isa(),
            encode_seconds=round(time.time() - t0, 1),
        )
        with open(os.path.join(HERE, f"{name}.json"), "w") as f:
            json.dump(meta, f, indent=1)
        index[name] = meta
        print(f"{name}: rows {rows} K {n} kbytes {len(kb)} slot {slot_type} {slot.size} nd {len(dval)} hist {hist} "
              f"ref_dequant==Wq {meta['ref_dequant_eq_wq']} ({meta['ref_dequant_maxdiff_wq']:.3e}) t {time.time() - t0:.1f}s", flush=True)
    if not a.only:
        with open(os.path.join(HERE, "signs.json"), "w") as f:
            json.dump([int(s) for s in signs], f)


if __name__ == "__main__":
    main()
