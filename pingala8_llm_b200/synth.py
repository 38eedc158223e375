"""Seeded synthetic Pingala-8 slots of any shape (valid codes, realistic scales) for large-size tests and the bench.

Every bit pattern of a tile payload is a valid code, so random payload words give a valid tensor of the requested
classes; the reference makes the same point for its timing arms ("timing does not depend on values", vr49.cuh,
CU:2936, k_fill_rand CU:582-587). The codebook A, coset c and Hadamard signs are the reference's shipped tables
(research/work/r48k3/tables_vrc.pt; signs of r48_a1gpu.make_fw seed 0), kept in tables_pingala8.bin.
Scales follow the encoder's rule S = 1.05 * rms / G[class] (r48k.py:231) for weights of sigma 0.02.
"""
import os

import numpy as np

from . import fmt

HERE = os.path.dirname(os.path.abspath(__file__))
_TAB = np.fromfile(os.path.join(HERE, "tables_pingala8.bin"), np.uint8)
HEADER = _TAB[:2064].copy()          # A | B | c, NS = 108, TRL = 2, word 515 = 0
SIGNS = _TAB[2064:2320].view(np.int8).copy()
GAIN = {1: 24.5999, 2: 23.557, 3: 23.557, 4: 90.233, 5: 172.815, 6: 79.236, 7: 255.218}  # tables_vrc.json G
NW = [0, 4, 6, 8, 10, 12, 16, 24]


def kernel_bytes(rows, K, classes, rng, sigma=0.02):
    """Kernel bytes (header | M | S | pad | D) with random payload. classes: int or (ng, nb) int array."""
    ng, nb = rows // 32, K // 256
    cls = np.broadcast_to(np.asarray(classes, np.int64), (ng, nb)).copy()
    words = 64 * np.asarray(NW)[cls]
    off = np.concatenate([[0], np.cumsum(words.ravel())[:-1]]).reshape(ng, nb)
    M = (off.astype(np.uint64) | (cls.astype(np.uint64) << np.uint64(29))).astype(np.uint32)
    g = np.array([0.0] + [GAIN[k] for k in range(1, 8)])
    gain_rows = np.repeat(g[cls], 32, axis=0)  # (rows, nb)
    S = (1.05 * sigma * rng.uniform(0.8, 1.25, (rows, nb)) / np.where(gain_rows > 0, gain_rows, 1.0))
    S = np.where(gain_rows > 0, S, 0.0).astype(np.float16).T.copy()  # [b][r]
    nt = ng * nb
    D = rng.integers(0, 2**32, int(words.sum()), dtype=np.uint64).astype(np.uint32)
    od = fmt.off_d(rows, K)
    kb = np.zeros(od + 4 * D.size, np.uint8)
    kb[:2064] = HEADER
    kb[2064 : 2064 + 4 * nt] = M.ravel().view(np.uint8)
    kb[fmt.off_s(rows, K) : fmt.off_s(rows, K) + 2 * nt * 32] = S.ravel().view(np.uint8)
    kb[od:] = D.view(np.uint8)
    return kb


def make_slot(rows, K, classes=3, seed=0, nd=0, permute=True, c16=None, sigma=0.02):
    """A complete, validated host slot (numpy uint8)."""
    rng = np.random.default_rng(seed)
    kb = kernel_bytes(rows, K, classes, rng, sigma)
    prm = rng.permutation(rows).astype(np.int16) if permute else None
    if c16 is None:
        c16 = np.ones(K, np.float16)
    elif isinstance(c16, str) and c16 == "random":
        c16 = rng.uniform(0.5, 2.0, K).astype(np.float16)
    if nd:
        flat = rng.choice(rows * K, size=nd, replace=False)
        flat.sort()
        drow, dcol = (flat // K).astype(np.uint16), (flat % K).astype(np.uint16)
        dval = rng.normal(0, 0.01, nd).astype(np.float32)
    else:
        drow = dcol = dval = None
    return fmt.assemble_slot(kb, rows, K, c16, prm, drow, dcol, dval, SIGNS)


def make_slot_device(rows, K, classes=3, seed=0, device="cuda", nd=0, permute=True, perm_seed=None):
    """Like make_slot, but the random payload is drawn on the GPU (fast for model-size tensors).

    The header, M, S and side data are built on the host from a payload-free copy and the payload words are filled
    on the device, so a 15 MB tensor costs ~1 ms of host work. perm_seed (optional) draws the row permutation from its
    own seed, so slots made with different seeds can share a row order (the column shards of one tensor do).
    """
    import torch

    rng = np.random.default_rng(seed)
    ng, nb = rows // 32, K // 256
    cls = np.broadcast_to(np.asarray(classes, np.int64), (ng, nb))
    nwords = int((64 * np.asarray(NW)[cls]).sum())
    # host slot with an all-zero payload (same layout and size as the real one)
    kb = kernel_bytes(rows, K, classes, np.random.default_rng(seed + 1_000_003))
    od = fmt.off_d(rows, K)
    kb[od:] = 0
    prm = rng.permutation(rows).astype(np.int16) if permute else None
    if permute and perm_seed is not None:
        prm = np.random.default_rng(perm_seed).permutation(rows).astype(np.int16)
    if nd:
        flat = np.sort(rng.choice(rows * K, size=nd, replace=False))
        drow, dcol = (flat // K).astype(np.uint16), (flat % K).astype(np.uint16)
        dval = rng.normal(0, 0.01, nd).astype(np.float32)
    else:
        drow = dcol = dval = None
    host = fmt.assemble_slot(kb, rows, K, np.ones(K, np.float16), prm, drow, dcol, dval, SIGNS)
    dev = torch.from_numpy(host).to(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    payload = torch.randint(-(2**31), 2**31 - 1, (nwords,), dtype=torch.int32, device=device, generator=gen)
    dev[od : od + 4 * nwords].copy_(payload.view(torch.uint8))
    return dev
