"""ctypes access to the two CPU oracles and the reference's GPU kernels. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg and reference arm import this module. The product package
(pingala8_llm_b200) never imports it and has no CPU fallback.

  Oracle    -- our plain-C restatement of the reference CPU path (oracle/p8_oracle.c -> oracle/libp8oracle.so)
  RefOracle -- the reference's own CPU core compiled from its patch (oracle/_ref/libp8ref_{vnni,avx2}.so)
  RefGpu    -- the reference's own CUDA GEMV kernels compiled from its patch (oracle/_ref/libp8ref_gpu.so)
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_fp = C.POINTER(C.c_float)
_dp = C.POINTER(C.c_double)
_i16p = C.POINTER(C.c_int16)
_i32p = C.POINTER(C.c_int32)
_u8p = C.POINTER(C.c_uint8)


def _ptr(a, t):
    return a.ctypes.data_as(t)


def _cpu_has(flag):
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("flags"):
                    return flag in ln.split()
    except OSError:
        pass
    return False


class Oracle:
    """Our restatement (p8_oracle.c). `slot` is the full slot byte array (numpy uint8)."""

    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            path = os.path.join(HERE, "libp8oracle.so")
            if not os.path.exists(path):
                raise FileNotFoundError(f"{path} missing: run python oracle/build_ref.py")
            L = C.CDLL(path)
            L.p8o_sizeof.restype = C.c_size_t
            L.p8o_init.argtypes = [C.c_void_p, _u8p, C.c_size_t, C.c_int, C.c_int]
            L.p8o_free.argtypes = [C.c_void_p]
            L.p8o_nd.argtypes = [C.c_void_p]
            L.p8o_kbytes.argtypes = [C.c_void_p]
            L.p8o_kbytes.restype = C.c_size_t
            L.p8o_decode_tile_int.argtypes = [C.c_void_p, C.c_int, C.c_int, _i16p]
            L.p8o_decode_int_all.argtypes = [C.c_void_p, _i16p]
            L.p8o_dequant_f32.argtypes = [C.c_void_p, _fp]
            L.p8o_get_rows.argtypes = [C.c_void_p, _i32p, C.c_int, _fp, C.c_int]
            L.p8o_prep_x16.argtypes = [C.c_void_p, _fp, _i32p, _fp]
            L.p8o_mul_mat_x16.argtypes = [C.c_void_p, _fp, C.c_int, C.c_int, _fp, C.c_int]
            L.p8o_mul_mat_f64.argtypes = [C.c_void_p, _fp, C.c_int, C.c_int, _dp, C.c_int]
            L.p8o_need.argtypes = [C.c_size_t] * 4
            L.p8o_need.restype = C.c_size_t
            L.p8o_threads.restype = C.c_int
            cls._lib = L
        return cls._lib

    def __init__(self, slot, rows, K):
        L = self.lib()
        self.slot = np.ascontiguousarray(slot, dtype=np.uint8)
        self.rows, self.K = int(rows), int(K)
        self._m = C.create_string_buffer(L.p8o_sizeof())
        rc = L.p8o_init(self._m, _ptr(self.slot, _u8p), self.slot.size, self.rows, self.K)
        if rc:
            raise ValueError(f"oracle: not a valid Pingala-8 slot (rc {rc})")
        self.nd = L.p8o_nd(self._m)
        self.kbytes = L.p8o_kbytes(self._m)

    def __del__(self):
        if getattr(self, "_m", None) is not None and self._lib is not None:
            self._lib.p8o_free(self._m)
            self._m = None

    def decode_tile_int(self, g, b):
        out = np.empty((32, 256), np.int16)
        self.lib().p8o_decode_tile_int(self._m, g, b, _ptr(out, _i16p))
        return out

    def decode_int(self):
        """exact integer weights, sorted rows x K"""
        out = np.empty((self.rows, self.K), np.int16)
        self.lib().p8o_decode_int_all(self._m, _ptr(out, _i16p))
        return out

    def dequant(self):
        out = np.empty((self.rows, self.K), np.float32)
        self.lib().p8o_dequant_f32(self._m, _ptr(out, _fp))
        return out

    def get_rows(self, ids):
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty((ids.size, self.K), np.float32)
        self.lib().p8o_get_rows(self._m, _ptr(ids, _i32p), ids.size, _ptr(out, _fp), self.K)
        return out

    def prep_x16(self, x):
        x = np.ascontiguousarray(x, np.float32)
        q = np.empty(self.K, np.int32)
        d = np.empty(self.K // 128, np.float32)
        self.lib().p8o_prep_x16(self._m, _ptr(x, _fp), _ptr(q, _i32p), _ptr(d, _fp))
        return q, d

    def mul_mat(self, X):
        """X: (ncols, K) float32 -> Y (ncols, rows) float32, x16 activations (reference default)"""
        X = np.ascontiguousarray(np.atleast_2d(X), np.float32)
        Y = np.empty((X.shape[0], self.rows), np.float32)
        self.lib().p8o_mul_mat_x16(self._m, _ptr(X, _fp), X.shape[0], self.K, _ptr(Y, _fp), self.rows)
        return Y

    def mul_mat_f64(self, X):
        X = np.ascontiguousarray(np.atleast_2d(X), np.float32)
        Y = np.empty((X.shape[0], self.rows), np.float64)
        self.lib().p8o_mul_mat_f64(self._m, _ptr(X, _fp), X.shape[0], self.K, _ptr(Y, _dp), self.rows)
        return Y

    @classmethod
    def threads(cls):
        return cls.lib().p8o_threads()


class RefOracle:
    """The reference's own CPU core (vr-native-cpu-core.h) built by oracle/build_ref.py."""

    _lib = None
    _path = None

    @classmethod
    def available(cls):
        try:
            cls.lib()
            return True
        except (OSError, FileNotFoundError):
            return False

    @classmethod
    def lib(cls):
        if cls._lib is None:
            name = "libp8ref_vnni.so" if _cpu_has("avx_vnni") else "libp8ref_avx2.so"
            path = os.path.join(HERE, "_ref", name)
            if not os.path.exists(path):
                raise FileNotFoundError(f"{path} missing (built from the reference patch by oracle/build_ref.py)")
            L = C.CDLL(path)
            L.ref_meta_size.restype = C.c_size_t
            L.ref_init.argtypes = [C.c_void_p, _u8p, C.c_size_t, C.c_int, C.c_int]
            L.ref_free.argtypes = [C.c_void_p]
            L.ref_decode_tile_int.argtypes = [C.c_void_p, C.c_int, C.c_int, _i16p]
            L.ref_dequant_f32.argtypes = [C.c_void_p, _fp]
            L.ref_gemv_x16.argtypes = [C.c_void_p, _fp, _fp]
            L.ref_mul_mat_x16.argtypes = [C.c_void_p, _fp, C.c_int, C.c_int, _fp, C.c_int]
            L.ref_threads.restype = C.c_int
            L.ref_set_threads.argtypes = [C.c_int]
            L.ref_has_v4.restype = C.c_int
            L.ref_isa.restype = C.c_char_p
            L.ref_need.argtypes = [C.c_size_t] * 4
            L.ref_need.restype = C.c_size_t
            L.ref_offsets.argtypes = [C.c_size_t] * 4 + [C.POINTER(C.c_size_t)]
            L.ref_vr3_rows.argtypes = [C.c_size_t, C.c_size_t, C.c_uint32, C.POINTER(C.c_size_t)]
            L.ref_vr3_rows.restype = C.c_size_t
            L.ref_vr3_expand.argtypes = [_u8p, C.c_size_t, C.c_size_t, C.c_size_t, _u8p]
            cls._lib = L
            cls._path = path
        return cls._lib

    def __init__(self, slot, rows, K):
        L = self.lib()
        self.slot = np.ascontiguousarray(slot, dtype=np.uint8)
        self.rows, self.K = int(rows), int(K)
        self._m = C.create_string_buffer(L.ref_meta_size())
        rc = L.ref_init(self._m, _ptr(self.slot, _u8p), self.slot.size, self.rows, self.K)
        if rc:
            raise ValueError(f"reference vrc_init rejected the slot (rc {rc})")

    def __del__(self):
        if getattr(self, "_m", None) is not None and self._lib is not None:
            self._lib.ref_free(self._m)
            self._m = None

    def decode_tile_int(self, g, b):
        out = np.empty((32, 256), np.int16)
        self.lib().ref_decode_tile_int(self._m, g, b, _ptr(out, _i16p))
        return out

    def dequant(self):
        out = np.empty((self.rows, self.K), np.float32)
        self.lib().ref_dequant_f32(self._m, _ptr(out, _fp))
        return out

    def gemv(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(self.rows, np.float32)
        self.lib().ref_gemv_x16(self._m, _ptr(x, _fp), _ptr(y, _fp))
        return y

    def mul_mat(self, X):
        X = np.ascontiguousarray(np.atleast_2d(X), np.float32)
        Y = np.empty((X.shape[0], self.rows), np.float32)
        self.lib().ref_mul_mat_x16(self._m, _ptr(X, _fp), X.shape[0], self.K, _ptr(Y, _fp), self.rows)
        return Y

    @classmethod
    def threads(cls):
        return cls.lib().ref_threads()

    @classmethod
    def set_threads(cls, n):
        """OpenMP threads of the reference core's parallel loops (overrides OMP_NUM_THREADS)."""
        cls.lib().ref_set_threads(int(n))

    @classmethod
    def isa(cls):
        return cls.lib().ref_isa().decode()

    @classmethod
    def need(cls, kbytes, rows, K, nd):
        return cls.lib().ref_need(kbytes, rows, K, nd)

    @classmethod
    def offsets(cls, n, rows, K, nd):
        o = (C.c_size_t * 6)()
        cls.lib().ref_offsets(n, rows, K, nd, o)
        return tuple(o)

    @classmethod
    def vr3_rows(cls, fbytes, K, w515):
        kb = C.c_size_t(0)
        r = cls.lib().ref_vr3_rows(fbytes, K, w515, C.byref(kb))
        return r, kb.value

    @classmethod
    def vr3_expand(cls, f, rows, K, kbytes):
        f = np.ascontiguousarray(f, np.uint8)
        out = np.full(kbytes, 0xA5, np.uint8)
        cls.lib().ref_vr3_expand(_ptr(f, _u8p), f.size, rows, K, _ptr(out, _u8p))
        return out


class RefGpu:
    """The reference's own batch-1 GEMV kernels (k_vr_qx_real + k_vr, cut from its patch) on the GPU, built by
    oracle/build_ref.py into oracle/_ref/libp8ref_gpu.so. A comparison arm for timing and a sanity check, never the
    product path. Arguments are raw device pointers (the caller owns the memory and the stream)."""

    _lib = None

    @classmethod
    def available(cls):
        try:
            cls.lib()
            return True
        except (OSError, FileNotFoundError):
            return False

    @classmethod
    def lib(cls):
        if cls._lib is None:
            path = os.path.join(HERE, "_ref", "libp8ref_gpu.so")
            if not os.path.exists(path):
                raise FileNotFoundError(f"{path} missing (built from the reference patch by oracle/build_ref.py)")
            L = C.CDLL(path)
            L.refgpu_set_tables.argtypes = [C.POINTER(C.c_uint32), C.POINTER(C.c_int8)]
            L.refgpu_set_tables.restype = C.c_int
            L.refgpu_gemv.argtypes = [C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
            L.refgpu_gemv.restype = C.c_int
            L.refgpu_error_string.argtypes = [C.c_int]
            L.refgpu_error_string.restype = C.c_char_p
            cls._lib = L
        return cls._lib

    @classmethod
    def _check(cls, rc, what):
        if rc:
            raise RuntimeError(f"{what}: {cls.lib().refgpu_error_string(rc).decode()} ({rc})")

    @classmethod
    def set_tables(cls, slot):
        """Codebook A/B, coset c (slot words 0-512) and the slot's Hadamard signs (32 + 256 bytes before its end) into
        the kernels' symbols, as the reference's native prepare does once per model."""
        slot = np.ascontiguousarray(slot, np.uint8)
        hdr = np.ascontiguousarray(slot[:513 * 4].view(np.uint32))
        signs = np.ascontiguousarray(slot[slot.size - 288 : slot.size - 32].view(np.int8))
        cls._check(cls.lib().refgpu_set_tables(_ptr(hdr, C.POINTER(C.c_uint32)), _ptr(signs, C.POINTER(C.c_int8))),
                   "refgpu_set_tables")

    @classmethod
    def gemv(cls, slot_ptr, nbytes, rows, K, nd, x_ptr, y_ptr, xq_ptr, xs_ptr, V=5, RL=1, stream=0):
        """y[rows] = W x through k_vr_qx_real and k_vr<RL, V, 8, 108>, enqueued on `stream` (a cudaStream_t)."""
        cls._check(cls.lib().refgpu_gemv(slot_ptr, nbytes, rows, K, nd, x_ptr, y_ptr, xq_ptr, xs_ptr, V, RL, stream),
                   "refgpu_gemv")
