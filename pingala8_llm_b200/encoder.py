"""Offline trellis encoder on the GPU: the reference's encode(Y, Uc, cls, Sb, T, tr=True) (research/detail/r48k.py:105)
with its per-slice Viterbi (vit_k / best_cw / zero_ldlq) in CUDA (p8_encode_slice) and the feedback between slices as
a plain fp32 GEMM (cuBLAS through torch, TF32 off as in the reference).

    Q, IDX = encode(Y, Uc, cls, Sb)      # Y [rows, n] FWHT-domain weights (CUDA f32), Uc [n, n] upper Cholesky factor
                                         # of the inverse Hessian, cls / Sb [rows, n / 256] classes and scales

Q [rows, n] are the quantised values (codeword x scale), IDX [rows, n / 4, 3] the (f1, f2, f3) code fields, in the
reference's layout (natural rows; packing them into a slot sorts rows and tiles as the reference's pack_blob does).
The 4 x 4 block inverses A4 are computed on the host CPU with torch.linalg.inv, as the reference computes them.
"""
import ctypes as C

import numpy as np
import torch

from ._lib import check, lib
from .synth import HEADER


def default_tables(device="cuda"):
    """the shipped codebook A [256, 4] (device int8) and coset vector c [4] (host int8)"""
    A = torch.from_numpy(HEADER[:1024].view(np.int8).reshape(256, 4).copy()).to(device)
    c = HEADER[2048:2052].view(np.int8).copy()
    return A, c


def encode(Y, Uc, cls, Sb, codebook=None, coset=None, stream=None):
    if not (Y.is_cuda and Y.dtype == torch.float32 and Y.dim() == 2):
        raise ValueError("Y must be a 2-D float32 CUDA tensor")
    rows, n = Y.shape
    if n % 256 or Uc.shape != (n, n) or cls.shape != (rows, n // 256) or Sb.shape != (rows, n // 256):
        raise ValueError("shapes: Y [rows, n] (n % 256 == 0), Uc [n, n], cls and Sb [rows, n / 256]")
    dev = Y.device
    if codebook is None:
        codebook, coset = default_tables(dev)
    coset = np.ascontiguousarray(np.asarray(coset, np.int8))
    Ucd = Uc.to(dev, torch.float32).contiguous()
    Uch = Ucd.cpu()
    W = Y.clone().contiguous()
    Q = torch.zeros_like(W)
    IDX = torch.zeros(rows, n // 4, 3, dtype=torch.uint8, device=dev)
    E = torch.empty(rows, 128, dtype=torch.float32, device=dev)
    clsd = cls.to(dev, torch.uint8).contiguous()
    Sbd = Sb.to(dev, torch.float32).contiguous()
    ws = torch.empty(int(lib().p8_encode_workspace()), dtype=torch.uint8, device=dev)
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    vp = lambda t, off=0: C.c_void_p(t.data_ptr() + off * t.element_size())
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        with torch.cuda.stream(s):
            for i0 in range(0, n, 128):
                i1, b = i0 + 128, i0 // 256
                Hb = Uch[i0:i1, i0:i1]
                A4 = torch.linalg.inv(torch.stack([Hb[j:j + 4, j:j + 4] for j in range(0, 128, 4)])).contiguous().to(dev)
                check(lib().p8_encode_slice(vp(W, i0), n, vp(Ucd, i0 * n + i0), n, vp(A4), vp(codebook),
                                            coset.ctypes.data_as(C.c_void_p), vp(clsd, b), n // 256, vp(Sbd, b), n // 256, rows,
                                            vp(Q, i0), n, vp(E), 128, vp(IDX, 3 * (i0 // 4)), 3 * (n // 4), vp(ws), ws.numel(),
                                            C.c_void_p(s.cuda_stream)), "p8_encode_slice")
                if i1 < n:
                    W[:, i1:] -= E @ Ucd[i0:i1, i1:]
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    return Q, IDX
