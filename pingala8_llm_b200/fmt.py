"""Host-side Pingala-8 slot format helpers over the C ABI (numpy in, numpy out).

These mirror the reference's loader-side code (ggml-vr-native.h CU:1-51, llama-vr3.h CU:3621-3661,
llama-model-loader.cpp vr_native_load CU:3527-3580) and add the tensor-parallel shard transforms.
"""
import ctypes as C

import numpy as np

from ._lib import check, lib

SLOT_TYPES = ["IQ2_XXS", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"]
HDR = 2064


def _p(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


def nt_of(rows, K):
    return (rows // 32) * (K // 256)


def off_s(rows, K):
    return HDR + 4 * nt_of(rows, K)


def off_d(rows, K):
    return (HDR + 68 * nt_of(rows, K) + 15) & ~15


def slot_need(kbytes, rows, K, nd):
    return lib().p8_slot_need(kbytes, rows, K, nd)


def slot_offsets(n, rows, K, nd):
    o = (C.c_size_t * 6)()
    lib().p8_slot_offsets(n, rows, K, nd, o)
    return dict(zip(("E", "C", "P", "Q", "SG", "T"), tuple(o)))


def slot_nbytes(rows, K, need):
    idx = C.c_int(-1)
    n = lib().p8_slot_nbytes(rows, K, need, C.byref(idx))
    return n, (SLOT_TYPES[idx.value] if idx.value >= 0 else None)


def kbytes_from_m(rows, K, M):
    M = np.ascontiguousarray(M, np.uint32)
    return lib().p8_kbytes_from_m(rows, K, _p(M))


def check_slot(slot, K, rows):
    """Raise P8Error if the host slot fails any loader / prepare check."""
    slot = np.ascontiguousarray(slot, np.uint8)
    check(lib().p8_slot_check(_p(slot), slot.size, K, rows), "p8_slot_check")


def slot_status(slot, K, rows):
    slot = np.ascontiguousarray(slot, np.uint8)
    return lib().p8_slot_check(_p(slot), slot.size, K, rows)


def assemble_slot(kbytes, rows, K, c16, prm, drow, dcol, dval, signs):
    """Kernel bytes + side tensors -> slot bytes (vr_native_load). prm None = identity (VR3)."""
    kb = np.ascontiguousarray(np.frombuffer(kbytes, np.uint8) if isinstance(kbytes, (bytes, bytearray)) else kbytes, np.uint8)
    c16 = np.ascontiguousarray(c16, np.float16).view(np.uint16)
    prm = None if prm is None else np.ascontiguousarray(prm, np.int16)
    nd = 0 if dval is None else len(dval)
    drow = np.ascontiguousarray(drow if nd else np.zeros(1), np.uint16)
    dcol = np.ascontiguousarray(dcol if nd else np.zeros(1), np.uint16)
    dval = np.ascontiguousarray(dval if nd else np.zeros(1), np.float32)
    signs = np.ascontiguousarray(signs, np.int8)
    n, _ = slot_nbytes(rows, K, slot_need(kb.size, rows, K, nd))
    if n == 0:
        from ._lib import P8Error
        raise P8Error(-15, "p8_slot_assemble")
    out = np.empty(n, np.uint8)
    on = C.c_size_t(0)
    check(lib().p8_slot_assemble(_p(kb), kb.size, rows, K, _p(c16), _p(prm), _p(drow), _p(dcol), _p(dval), nd, _p(signs),
                                 _p(out), out.size, C.byref(on)), "p8_slot_assemble")
    return out[: on.value]


def vr3_rows(fbytes, K, w515):
    kb = C.c_size_t(0)
    r = lib().p8_vr3_rows(fbytes, K, w515, C.byref(kb))
    return r, kb.value


def vr3_expand(f, K):
    f = np.ascontiguousarray(f, np.uint8)
    w515 = int(f[2060:2064].view(np.uint32)[0])
    rows, kb = vr3_rows(f.size, K, w515)
    if rows == 0:
        from ._lib import P8Error
        raise P8Error(-1, "p8_vr3_rows: not a VR3 tensor")
    out = np.empty(kb, np.uint8)
    check(lib().p8_vr3_expand(_p(f), f.size, rows, K, _p(out), out.size), "p8_vr3_expand")
    return out, rows


def _shard_cap(slot):
    return slot.size + (1 << 20)


def shard_rows(slot, K, rows, r0, r1):
    """Column-parallel shard: ORIGINAL output rows [r0, r1). Returns (slot bytes, original row of each shard row)."""
    slot = np.ascontiguousarray(slot, np.uint8)
    out = np.empty(_shard_cap(slot), np.uint8)
    on = C.c_size_t(0)
    orig = np.empty(r1 - r0, np.int32)
    check(lib().p8_tp_shard_rows(_p(slot), slot.size, K, rows, r0, r1, _p(out), out.size, C.byref(on), _p(orig)),
          "p8_tp_shard_rows")
    return out[: on.value].copy(), orig


def shard_cols(slot, K, rows, b0, b1):
    """Row-parallel shard: 256-column blocks [b0, b1)."""
    slot = np.ascontiguousarray(slot, np.uint8)
    out = np.empty(_shard_cap(slot), np.uint8)
    on = C.c_size_t(0)
    check(lib().p8_tp_shard_cols(_p(slot), slot.size, K, rows, b0, b1, _p(out), out.size, C.byref(on)), "p8_tp_shard_cols")
    return out[: on.value].copy()


def split_kernel_bytes(slot, K, rows):
    """(kernel bytes, c16, prm, (drow, dcol, dval), signs) of a slot: the loader's inputs, read back."""
    slot = np.ascontiguousarray(slot, np.uint8)
    tr = slot[-32:].view(np.uint32)
    kb, nd = int(tr[2]), int(tr[3])
    o = slot_offsets(slot.size, rows, K, nd)
    c16 = slot[o["C"] : o["C"] + 2 * K].view(np.float16)
    prm = slot[o["P"] : o["P"] + 2 * rows].view(np.int16)
    drow = slot[o["E"] : o["E"] + 2 * nd].view(np.uint16)
    dcol = slot[o["E"] + 2 * nd : o["E"] + 4 * nd].view(np.uint16)
    dval = slot[o["E"] + 4 * nd : o["E"] + 8 * nd].view(np.float32)
    signs = slot[o["SG"] : o["SG"] + 256].view(np.int8)
    return slot[:kb], c16, prm, (drow, dcol, dval), signs
