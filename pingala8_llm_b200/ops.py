"""Operator layer: a prepared Pingala-8 weight and the ggml MUL_MAT / GET_ROWS / to_fp32 ops on it.

Mirrors the reference's op hooks (ggml_cuda_f44_active / _prepare_graph / _mul_mat_vec / _mul_mat_q8, CU:1293-1302)
with torch tensors as the device-memory carrier. Every call goes through the C ABI of libpingala8_b200.so on the
current torch CUDA stream; there is no CPU path.
"""
import ctypes as C

import numpy as np
import torch

from ._lib import P8Error, check, lib


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _ptr(t):
    return C.c_void_p(t.data_ptr())


class P8Tensor:
    """A Pingala-8 slot on the GPU, prepared once (validation + side structures), like ggml_cuda_f44_prepare_graph.

    slot: torch.uint8 CUDA tensor or numpy uint8 array (copied to the current device). Shape [K, rows] in ggml terms.
    """

    def __init__(self, slot, K, rows, stream=None):
        if isinstance(slot, np.ndarray):
            slot = torch.from_numpy(np.ascontiguousarray(slot, np.uint8)).cuda()
        if not (isinstance(slot, torch.Tensor) and slot.is_cuda and slot.dtype == torch.uint8 and slot.is_contiguous()):
            raise ValueError("slot must be a contiguous torch.uint8 CUDA tensor")
        self.slot, self.K, self.rows = slot, int(K), int(rows)
        h = C.c_void_p()
        check(lib().p8_prepare(_ptr(slot), slot.numel(), self.K, self.rows, _stream(stream), C.byref(h)), "p8_prepare")
        self._h = h
        self._ws = {}

    @property
    def handle(self):
        if self._h is None:
            raise P8Error(-12, "tensor released")
        return self._h

    def info(self):
        r, k, nd = C.c_int64(), C.c_int64(), C.c_int64()
        hist = (C.c_uint64 * 8)()
        check(lib().p8_tensor_info(self.handle, C.byref(r), C.byref(k), C.byref(nd), hist), "p8_tensor_info")
        return dict(rows=r.value, K=k.value, nd=nd.value, class_hist=list(hist))

    def workspace_size(self, ncols=1):
        return int(lib().p8_workspace_size(self.handle, ncols))

    def workspace(self, ncols=1):
        n = self.workspace_size(ncols)
        w = self._ws.get("buf")
        if w is None or w.numel() < n:
            w = torch.empty(max(n, 256), dtype=torch.uint8, device=self.slot.device)
            self._ws["buf"] = w
        return w

    def mul_mat_vec(self, x, out=None, workspace=None, stream=None):
        """y = W x, x float32 [K] on the GPU -> float32 [rows]."""
        x = x.contiguous()
        if x.dtype != torch.float32 or x.numel() != self.K or not x.is_cuda:
            raise ValueError("x must be float32 CUDA with K elements")
        y = out if out is not None else torch.empty(self.rows, dtype=torch.float32, device=x.device)
        ws = workspace if workspace is not None else self.workspace(1)
        check(lib().p8_mul_mat_vec(self.handle, _ptr(x), _ptr(y), _ptr(ws), ws.numel(), _stream(stream)), "p8_mul_mat_vec")
        return y

    def mul_mat_vec_allreduce(self, x, comm, out=None, workspace=None, stream=None):
        """y = sum over the ranks of comm of (rank's shard) x (rank's x): this tensor is the rank's row-parallel shard
        (p8_tp_shard_cols), x its input slice; the partial rows are exchanged inside the GEMV (p8_tp_gemv_allreduce).
        Every rank gets the same y (sum in rank order)."""
        x = x.contiguous()
        if x.dtype != torch.float32 or x.numel() != self.K or not x.is_cuda:
            raise ValueError("x must be float32 CUDA with K elements")
        y = out if out is not None else torch.empty(self.rows, dtype=torch.float32, device=x.device)
        ws = workspace if workspace is not None else self.workspace(1)
        check(lib().p8_tp_gemv_allreduce(self.handle, _ptr(x), _ptr(y), comm.handle, _ptr(ws), ws.numel(), _stream(stream)),
              "p8_tp_gemv_allreduce")
        return y

    def mul_mat(self, X, out=None, workspace=None, stream=None, norm_weight=None, eps=1e-5, up=None):
        """Y = X W^T: X float32 [ncols, K] -> Y float32 [ncols, rows] (ggml dst [rows, ncols]).

        X and out may be row-strided views (unit column stride; X's row stride a multiple of 4 floats), as ggml's
        src1 / dst with nb[1] > ne[0] * 4. norm_weight / up: each token's input op fused into the activation prep
        (p8_mul_mat_ex): RMSNorm(X[n]) * norm_weight, or silu(X[n]) * up[n]."""
        if X.dim() == 2 and (X.stride(1) != 1 or X.stride(0) % 4 or X.data_ptr() % 16):
            X = X.contiguous()
        if X.dtype != torch.float32 or X.dim() != 2 or X.shape[1] != self.K or not X.is_cuda:
            raise ValueError("X must be float32 CUDA [ncols, K]")
        n = X.shape[0]
        Y = out if out is not None else torch.empty(n, self.rows, dtype=torch.float32, device=X.device)
        if Y.dim() != 2 or Y.shape[0] != n or Y.shape[1] != self.rows or Y.stride(1) != 1 or Y.dtype != torch.float32:
            raise ValueError("out must be float32 [ncols, rows] with unit column stride")
        if norm_weight is None and up is None:
            ws = workspace if workspace is not None else self.workspace(n)
            check(lib().p8_mul_mat(self.handle, _ptr(X), n, X.stride(0), _ptr(Y), Y.stride(0), _ptr(ws), ws.numel(),
                                   _stream(stream)), "p8_mul_mat")
            return Y
        from ._lib import Prologue

        if norm_weight is not None and up is not None:
            raise ValueError("one prologue per call: norm_weight or up")
        if norm_weight is not None:
            if norm_weight.dtype != torch.float32 or not norm_weight.is_cuda or norm_weight.numel() != self.K:
                raise ValueError("norm_weight must be float32 CUDA with K elements")
            norm_weight = norm_weight.contiguous()
            pro, kind = Prologue(1, norm_weight.data_ptr(), None, float(eps)), 1
        else:
            if up.shape != X.shape or up.stride() != X.stride() or up.dtype != torch.float32 or not up.is_cuda:
                raise ValueError("up must be float32 CUDA with X's shape and strides")
            pro, kind = Prologue(2, None, up.data_ptr(), 0.0), 2
        need = int(lib().p8_workspace_size_ex(self.handle, n, kind))
        ws = workspace if workspace is not None else torch.empty(max(need, 256), dtype=torch.uint8, device=X.device)
        check(lib().p8_mul_mat_ex(self.handle, _ptr(X), n, X.stride(0), C.byref(pro), _ptr(Y), Y.stride(0), _ptr(ws),
                                  ws.numel(), _stream(stream)), "p8_mul_mat_ex")
        return Y

    def get_rows(self, ids, out=None, stream=None):
        """rows ids (ORIGINAL row indices, int32 CUDA) -> float32 [n, K]"""
        ids = ids.to(torch.int32).contiguous()
        if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= self.rows):
            raise P8Error(-1, "p8_get_rows: row id out of range")
        out = out if out is not None else torch.empty(ids.numel(), self.K, dtype=torch.float32, device=self.slot.device)
        check(lib().p8_get_rows(self.handle, _ptr(ids), ids.numel(), _ptr(out), out.stride(0), _stream(stream)), "p8_get_rows")
        return out

    def dequant(self, out=None, stream=None):
        out = out if out is not None else torch.empty(self.rows, self.K, dtype=torch.float32, device=self.slot.device)
        check(lib().p8_dequant_f32(self.handle, _ptr(out), _stream(stream)), "p8_dequant_f32")
        return out

    def decode_int(self, out=None, stream=None):
        out = out if out is not None else torch.empty(self.rows, self.K, dtype=torch.int16, device=self.slot.device)
        check(lib().p8_decode_int(self.handle, _ptr(out), _stream(stream)), "p8_decode_int")
        return out

    def release(self):
        if self._h is not None:
            check(lib().p8_release(self._h), "p8_release")
            self._h = None

    def __del__(self):
        try:
            if getattr(self, "_h", None) is not None:
                lib().p8_release(self._h)
                self._h = None
        except Exception:
            pass


def group_workspace_size(tensors, ncols=1, kind=0):
    """workspace bytes of mul_mat_vec_group (ncols 1) and mul_mat_group over ncols tokens (prologue kind 0/1/2)"""
    arr = (C.c_void_p * len(tensors))(*[t.handle.value for t in tensors])
    return int(lib().p8_workspace_size_group_ex(arr, len(tensors), ncols, kind))


def mul_mat_vec_group(tensors, x, outs=None, workspace=None, stream=None, norm_weight=None, eps=1e-5, up=None):
    """y_i = W_i x for tensors sharing x (q/k/v, gate/up): one prepared activation, one launch (<= 4 tensors).

    Fused activation prologue (p8_mul_mat_vec_group_ex): norm_weight -> the tensors multiply RMSNorm(x) * norm_weight
    (eps as ggml's rms_norm); up -> they multiply silu(x) * up (x = the gate output)."""
    x = x.contiguous()
    if x.dtype != torch.float32 or not x.is_cuda or x.numel() != tensors[0].K:
        raise ValueError("x must be float32 CUDA with K elements")
    if norm_weight is not None and up is not None:
        raise ValueError("one prologue per call: norm_weight or up")
    outs = outs if outs is not None else [torch.empty(t.rows, dtype=torch.float32, device=x.device) for t in tensors]
    n = len(tensors)
    arr = (C.c_void_p * n)(*[t.handle.value for t in tensors])
    ys = (C.c_void_p * n)(*[o.data_ptr() for o in outs])
    if workspace is None:
        workspace = torch.empty(max(group_workspace_size(tensors), 256), dtype=torch.uint8, device=x.device)
    if norm_weight is None and up is None:
        check(lib().p8_mul_mat_vec_group(arr, n, _ptr(x), ys, _ptr(workspace), workspace.numel(), _stream(stream)),
              "p8_mul_mat_vec_group")
        return outs
    from ._lib import Prologue

    extra = norm_weight if norm_weight is not None else up
    if extra.dtype != torch.float32 or not extra.is_cuda or not extra.is_contiguous() or extra.numel() != tensors[0].K:
        raise ValueError("norm_weight / up must be contiguous float32 CUDA with K elements")
    pro = Prologue(1, extra.data_ptr(), None, float(eps)) if norm_weight is not None else Prologue(2, None, extra.data_ptr(), 0.0)
    check(lib().p8_mul_mat_vec_group_ex(arr, n, _ptr(x), C.byref(pro), ys, _ptr(workspace), workspace.numel(),
                                        _stream(stream)), "p8_mul_mat_vec_group_ex")
    return outs


def mul_mat_group(tensors, X, outs=None, workspace=None, stream=None, norm_weight=None, eps=1e-5, up=None):
    """Y_i = X W_i^T for tensors sharing X [ncols, K] (q/k/v, gate/up; <= 4): the activation prep, prologue included,
    runs once (p8_mul_mat_group); bit-identical to separate P8Tensor.mul_mat calls except the K-split tail rows of
    two tensors that share one launch (fp32 summation order). outs: float32 [ncols, rows_i]
    with unit column stride; norm_weight / up as P8Tensor.mul_mat."""
    if X.dim() == 2 and (X.stride(1) != 1 or X.stride(0) % 4 or X.data_ptr() % 16):
        X = X.contiguous()
    if X.dtype != torch.float32 or X.dim() != 2 or X.shape[1] != tensors[0].K or not X.is_cuda:
        raise ValueError("X must be float32 CUDA [ncols, K]")
    if norm_weight is not None and up is not None:
        raise ValueError("one prologue per call: norm_weight or up")
    n, nt = X.shape[0], len(tensors)
    outs = outs if outs is not None else [torch.empty(n, t.rows, dtype=torch.float32, device=X.device) for t in tensors]
    for t, o in zip(tensors, outs):
        if o.dim() != 2 or o.shape[0] != n or o.shape[1] != t.rows or o.stride(1) != 1 or o.dtype != torch.float32:
            raise ValueError("outs must be float32 [ncols, rows] with unit column stride")
    from ._lib import Prologue

    kind = 0
    pro = None
    if norm_weight is not None:
        if norm_weight.dtype != torch.float32 or not norm_weight.is_cuda or norm_weight.numel() != X.shape[1]:
            raise ValueError("norm_weight must be float32 CUDA with K elements")
        norm_weight = norm_weight.contiguous()
        pro, kind = Prologue(1, norm_weight.data_ptr(), None, float(eps)), 1
    elif up is not None:
        if up.shape != X.shape or up.stride() != X.stride() or up.dtype != torch.float32 or not up.is_cuda:
            raise ValueError("up must be float32 CUDA with X's shape and strides")
        pro, kind = Prologue(2, None, up.data_ptr(), 0.0), 2
    arr = (C.c_void_p * nt)(*[t.handle.value for t in tensors])
    ys = (C.c_void_p * nt)(*[o.data_ptr() for o in outs])
    lds = (C.c_int64 * nt)(*[o.stride(0) for o in outs])
    if workspace is None:
        need = int(lib().p8_workspace_size_group_ex(arr, nt, n, kind))
        workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=X.device)
    check(lib().p8_mul_mat_group(arr, nt, _ptr(X), n, X.stride(0), C.byref(pro) if pro is not None else None, ys, lds,
                                 _ptr(workspace), workspace.numel(), _stream(stream)), "p8_mul_mat_group")
    return outs


class Chain:
    """A run of batch-1 projections as chained launches (p8_chain_*): each step one GEMV launch that reads its input
    straight from the previous step's partial sums, one row reduce after the last step. Each step is a dict
        tensors      list of P8Tensor reading the same input (1..4; q/k/v, gate/up)
        x            float32 CUDA [K]: any buffer, or exactly an output of the previous step (read from its partials)
        outs         float32 CUDA [rows_i] per tensor
        norm_weight  RMSNorm weight [K] (with eps), or up: SwiGLU's up [K] (may be the previous step's other output)
        res          optional list of residuals [rows_i] (or None entries) added to the outputs
    Buffers are fixed at creation (like a captured graph); run() enqueues the chain's launches and is capturable. Results equal
    the separate mul_mat_vec_group calls up to float rounding."""

    def __init__(self, steps):
        from ._lib import ChainStepC, Prologue

        self._keep = []
        arr = (ChainStepC * len(steps))()
        for i, st in enumerate(steps):
            ts, x, outs = st["tensors"], st["x"], st["outs"]
            if not 1 <= len(ts) <= 4 or len(outs) != len(ts):
                raise ValueError("a chain step has 1..4 tensors and one output per tensor")
            for o, t in zip(outs, ts):
                if o.dtype != torch.float32 or not o.is_cuda or not o.is_contiguous() or o.numel() != t.rows:
                    raise ValueError("outs must be contiguous float32 CUDA [rows]")
            if x.dtype != torch.float32 or not x.is_cuda or not x.is_contiguous() or x.numel() != ts[0].K:
                raise ValueError("x must be contiguous float32 CUDA [K]")
            c = arr[i]
            c.n = len(ts)
            for j, t in enumerate(ts):
                c.t[j] = t.handle.value
                c.y[j] = outs[j].data_ptr()
                r = (st.get("res") or [None] * len(ts))[j]
                c.res[j] = r.data_ptr() if r is not None else None
            c.x = x.data_ptr()
            nw, up = st.get("norm_weight"), st.get("up")
            if nw is not None and up is not None:
                raise ValueError("one prologue per step: norm_weight or up")
            if nw is not None:
                c.pro = Prologue(1, nw.data_ptr(), None, float(st.get("eps", 1e-5)))
            elif up is not None:
                c.pro = Prologue(2, None, up.data_ptr(), 0.0)
            self._keep.append((ts, x, outs, nw, up, st.get("res")))
        h = C.c_void_p()
        check(lib().p8_chain_create(arr, len(steps), C.byref(h)), "p8_chain_create")
        self._h = h
        self._ws = None
        self.device = steps[0]["x"].device

    def workspace_size(self):
        return int(lib().p8_chain_workspace_size(self._h))

    def run(self, workspace=None, stream=None):
        if workspace is None:
            if self._ws is None:
                self._ws = torch.empty(max(self.workspace_size(), 256), dtype=torch.uint8, device=self.device)
            workspace = self._ws
        check(lib().p8_chain_run(self._h, _ptr(workspace), workspace.numel(), _stream(stream)), "p8_chain_run")

    def trace(self, buf):
        """record per-step, per-CTA phase stamps of later runs into buf (int64 CUDA, nsteps x SMs x 8; None: off)"""
        if buf is None:
            check(lib().p8_chain_trace(self._h, None, 0), "p8_chain_trace")
        else:
            check(lib().p8_chain_trace(self._h, _ptr(buf), buf.numel()), "p8_chain_trace")

    def close(self):
        if getattr(self, "_h", None) is not None:
            lib().p8_chain_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def active(slot):
    """ggml_cuda_f44_active: is this device slot a prepared Pingala-8 tensor?"""
    return bool(lib().p8_active(_ptr(slot)))


def device_error():
    """1 if a kernel gave up on a bounded device wait since the last call (synchronises)."""
    return int(lib().p8_device_error())
