"""Seeded synthetic Pingala-8 slots built with numpy alone. TEST INFRASTRUCTURE ONLY.

bench.py's reference arm and CPU-baseline leg time the reference's own CPU core (oracle/_ref) and must not load the
product library (pingala8_llm_b200/libpingala8_b200.so), so they build their slots here instead of through
pingala8_llm_b200.synth (which assembles slots through the C ABI). Same recipe as that module: random payload words
(every bit pattern of a tile payload is a valid code; the reference times on random codes the same way, vr49.cuh
CU:2936), scales S = 1.05 * sigma * U(0.8, 1.25) / G[class] (r48k.py:231), the reference's shipped codebook, coset
and Hadamard signs (pingala8_llm_b200/tables_pingala8.bin, read as a data file), and the slot assembled as the
reference loader does (vr_native_load, CU:3527-3580; offsets CU:25-51; slot type = the smallest of IQ2_XXS,
Q2_K..Q6_K that holds vrn_need bytes, CU:3493-3497).
"""
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_TAB = os.path.join(os.path.dirname(HERE), "pingala8_llm_b200", "tables_pingala8.bin")
SLOT_BYTES_PER_BLOCK = [66, 84, 110, 144, 176, 210]  # IQ2_XXS, Q2_K .. Q6_K bytes per 256 weights
NW = [0, 4, 6, 8, 10, 12, 16, 24]
GAIN = {1: 24.5999, 2: 23.557, 3: 23.557, 4: 90.233, 5: 172.815, 6: 79.236, 7: 255.218}


def _a16(n):
    return (n + 15) & ~15


def _tables():
    t = np.fromfile(_TAB, np.uint8)
    return t[:2064].copy(), t[2064:2320].view(np.int8).copy()


def make_slot(rows, K, seed=0, cls=3, sigma=0.02):
    """A valid single-class slot (numpy uint8) of shape [K, rows] with a random row permutation and no clamp delta."""
    header, signs = _tables()
    rng = np.random.default_rng(seed)
    ng, nb = rows // 32, K // 256
    nt = ng * nb
    words = 64 * NW[cls]
    M = ((np.arange(nt, dtype=np.uint64) * words) | (np.uint64(cls) << np.uint64(29))).astype(np.uint32)
    S = (1.05 * sigma * rng.uniform(0.8, 1.25, (nb, rows)) / GAIN[cls]).astype(np.float16)
    offD = (2064 + 68 * nt + 15) & ~15
    kbytes = offD + 4 * words * nt
    need = _a16(kbytes) + _a16(2 * K) + 2 * _a16(2 * rows) + 256 + 32 + 64  # vrn_need with nd = 0
    n = next((rows * nb * b for b in SLOT_BYTES_PER_BLOCK if rows * nb * b >= need), 0)
    if not n:
        raise ValueError("no slot type fits")
    buf = np.zeros(n, np.uint8)
    buf[:2064] = header
    buf[2064 : 2064 + 4 * nt] = M.view(np.uint8)
    buf[2064 + 4 * nt : 2064 + 68 * nt] = S.ravel().view(np.uint8)
    buf[offD:kbytes] = np.frombuffer(rng.bytes(4 * words * nt), np.uint8)
    offT = n - 32
    offSG = offT - 256
    offQ = (offSG - 2 * rows) & ~15
    offP = (offQ - 2 * rows) & ~15
    offC = (offP - 2 * K) & ~15
    prm = rng.permutation(rows).astype(np.int16)
    pinv = np.empty(rows, np.int16)
    pinv[prm.astype(np.int64)] = np.arange(rows, dtype=np.int16)
    buf[offC : offC + 2 * K] = np.ones(K, np.float16).view(np.uint8)
    buf[offP : offP + 2 * rows] = prm.view(np.uint8)
    buf[offQ : offQ + 2 * rows] = pinv.view(np.uint8)
    buf[offSG : offSG + 256] = signs.view(np.uint8)
    buf[offT:] = np.frombuffer(struct.pack("<8I", 0x4E525656, 0x31354952, kbytes, 0, rows, K, 108, 1), np.uint8)
    return buf
