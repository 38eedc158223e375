"""ctypes binding of libpingala8_b200.so (the C ABI in include/pingala8.h).

The library is built in-tree by `python -m pingala8_llm_b200.build` (or __graft_entry__.build()). There is no
fallback: importing the compute API without the library raises.
"""
import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpingala8_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "pingala8.h")

P8_STATUS = {
    0: "P8_OK", -1: "P8_ERR_ARG", -2: "P8_ERR_TRAILER", -3: "P8_ERR_HEADER", -4: "P8_ERR_PAYLOAD", -5: "P8_ERR_PERM",
    -6: "P8_ERR_DELTA", -7: "P8_ERR_SIGNS", -8: "P8_ERR_TABLES", -9: "P8_ERR_SHAPE", -10: "P8_ERR_CUDA",
    -11: "P8_ERR_WORKSPACE", -12: "P8_ERR_NOT_PREPARED", -13: "P8_ERR_UNSUPPORTED", -14: "P8_ERR_TIMEOUT", -15: "P8_ERR_SLOT",
    -16: "P8_ERR_FILE", -17: "P8_ERR_MODEL", -18: "P8_ERR_NOALLOC_SCRATCH",
}


class P8Error(RuntimeError):
    """A C-ABI call returned a non-zero p8_status (the reference aborts / throws in these places)."""

    def __init__(self, status, what=""):
        self.status = int(status)
        self.name = P8_STATUS.get(self.status, str(status))
        msg = _lib().p8_status_str(self.status).decode() if _LIB is not None else self.name
        super().__init__(f"{what}: {self.name} ({msg})" if what else f"{self.name} ({msg})")


_LIB = None

_vp, _sz, _i64, _u32 = C.c_void_p, C.c_size_t, C.c_int64, C.c_uint32


class Prologue(C.Structure):
    """p8_prologue: activation prologue of p8_mul_mat_vec_group_ex (kind 0 none, 1 RMSNorm with w and eps, 2 SwiGLU
    with x2 = up)"""
    _fields_ = [("kind", C.c_int), ("w", C.c_void_p), ("x2", C.c_void_p), ("eps", C.c_float)]


class ChainStepC(C.Structure):
    """p8_chain_step: one step of a chained batch-1 GEMV run (p8_chain_create)"""
    _fields_ = [("n", C.c_int), ("t", C.c_void_p * 4), ("x", C.c_void_p), ("pro", Prologue), ("y", C.c_void_p * 4),
                ("res", C.c_void_p * 4)]


_SIGS = {
    "p8_prepare": (C.c_int, [_vp, _sz, _i64, _i64, _vp, C.POINTER(_vp)]),
    "p8_release": (C.c_int, [_vp]),
    "p8_active": (C.c_int, [_vp]),
    "p8_tensor_info": (C.c_int, [_vp, C.POINTER(_i64), C.POINTER(_i64), C.POINTER(_i64), C.POINTER(C.c_uint64)]),
    "p8_workspace_size": (_sz, [_vp, _i64]),
    "p8_mul_mat_vec": (C.c_int, [_vp, _vp, _vp, _vp, _sz, _vp]),
    "p8_workspace_size_group": (_sz, [_vp, C.c_int, _i64]),
    "p8_mul_mat_vec_group": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp, _sz, _vp]),
    "p8_mul_mat_vec_group_ex": (C.c_int, [_vp, C.c_int, _vp, C.POINTER(Prologue), _vp, _vp, _sz, _vp]),
    "p8_workspace_size_ex": (_sz, [_vp, _i64, C.c_int]),
    "p8_mul_mat_ex": (C.c_int, [_vp, _vp, _i64, _i64, C.POINTER(Prologue), _vp, _i64, _vp, _sz, _vp]),
    "p8_workspace_size_group_ex": (_sz, [_vp, C.c_int, _i64, C.c_int]),
    "p8_mul_mat_group": (C.c_int, [_vp, C.c_int, _vp, _i64, _i64, C.POINTER(Prologue), _vp, _vp, _vp, _sz, _vp]),
    "p8_noalloc_scratch_bytes": (_sz, []),
    "p8_mul_mat_vec_noalloc": (C.c_int, [_vp, _vp, _vp, _vp]),
    "p8_mul_mat": (C.c_int, [_vp, _vp, _i64, _i64, _vp, _i64, _vp, _sz, _vp]),
    "p8_get_rows": (C.c_int, [_vp, _vp, _i64, _vp, _i64, _vp]),
    "p8_dequant_f32": (C.c_int, [_vp, _vp, _vp]),
    "p8_decode_int": (C.c_int, [_vp, _vp, _vp]),
    "p8_slot_need": (_sz, [_sz, _sz, _sz, _sz]),
    "p8_slot_offsets": (None, [_sz, _sz, _sz, _sz, C.POINTER(_sz)]),
    "p8_kbytes_from_m": (_sz, [_sz, _sz, _vp]),
    "p8_slot_nbytes": (_sz, [_sz, _sz, _sz, C.POINTER(C.c_int)]),
    "p8_slot_assemble": (C.c_int, [_vp, _sz, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _sz, C.POINTER(_sz)]),
    "p8_slot_check": (C.c_int, [_vp, _sz, _i64, _i64]),
    "p8_vr3_rows": (_sz, [_sz, _sz, _u32, C.POINTER(_sz)]),
    "p8_vr3_expand": (C.c_int, [_vp, _sz, _sz, _sz, _vp, _sz]),
    "p8_tp_shard_rows": (C.c_int, [_vp, _sz, _i64, _i64, _i64, _i64, _vp, _sz, C.POINTER(_sz), _vp]),
    "p8_tp_shard_cols": (C.c_int, [_vp, _sz, _i64, _i64, _i64, _i64, _vp, _sz, C.POINTER(_sz)]),
    "p8_gguf_open": (C.c_int, [C.c_char_p, C.POINTER(_vp)]),
    "p8_gguf_close": (None, [_vp]),
    "p8_gguf_n_linear": (_i64, [_vp]),
    "p8_gguf_linear_info": (C.c_int, [_vp, _i64, C.POINTER(C.c_char_p), C.POINTER(_i64), C.POINTER(_i64), C.POINTER(_i64),
                                      C.POINTER(_sz), C.POINTER(C.c_int)]),
    "p8_gguf_load_linear": (C.c_int, [_vp, _i64, _vp, _sz, C.POINTER(_sz)]),
    "p8_tp_comm_create": (C.c_int, [C.c_int, C.c_int, _i64, _u32, C.POINTER(_vp)]),
    "p8_tp_comm_destroy": (C.c_int, [_vp]),
    "p8_tp_comm_ipc_handle": (C.c_int, [_vp, _vp, _sz]),
    "p8_tp_comm_open_peer": (C.c_int, [_vp, C.c_int, _vp, _sz]),
    "p8_tp_comm_set_peer": (C.c_int, [_vp, C.c_int, _vp]),
    "p8_tp_comm_buffer": (C.c_int, [_vp, C.POINTER(_vp), C.POINTER(_sz)]),
    "p8_tp_comm_epoch": (C.c_int, [_vp, C.POINTER(_u32)]),
    "p8_tp_comm_reset": (C.c_int, [_vp, _vp]),
    "p8_tp_gemv_allreduce": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "p8_encode_workspace": (_sz, []),
    "p8_encode_slice": (C.c_int, [_vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _i64, _vp,
                                  _i64, _vp, _sz, _vp]),
    "p8_chain_create": (C.c_int, [C.POINTER(ChainStepC), C.c_int, C.POINTER(_vp)]),
    "p8_chain_workspace_size": (_sz, [_vp]),
    "p8_chain_run": (C.c_int, [_vp, _vp, _sz, _vp]),
    "p8_chain_destroy": (C.c_int, [_vp]),
    "p8_chain_trace": (C.c_int, [_vp, _vp, _sz]),
    "p8_device_error": (C.c_int, []),
    "p8_status_str": (C.c_char_p, [C.c_int]),
    "p8_build_info": (C.c_char_p, []),
}


def _lib():
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m pingala8_llm_b200.build` (no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


lib = _lib


def check(status, what=""):
    if status != 0:
        raise P8Error(status, what)


def header_functions():
    """Names of every function declared in include/pingala8.h."""
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(p8_[a-z0-9_]+)\s*\(", txt)))
