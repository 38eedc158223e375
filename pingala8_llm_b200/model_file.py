"""Pingala-8 model files (GGUF, "VR native" layout 2 or 3): list the linears, assemble their slots, prepare them.

Thin binding of the C ABI's p8_gguf_* entry points (a native GGUF reader and the reference loader's checks,
llama_model_loader::vr_native_init / vr_native_load). The slot bytes are the ones the reference builds in device
memory; upload them and prepare them with P8Tensor.

    with ModelFile("model.gguf") as mf:
        for info in mf.linears:
            t = mf.tensor(info.name)          # P8Tensor on cuda:0
"""
import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import check, lib


@dataclass
class LinearInfo:
    index: int
    name: str      # <base>.weight
    K: int
    rows: int
    nd: int        # clamp-delta entries
    nbytes: int    # slot bytes (smallest IQ2_XXS .. Q6_K tensor that holds the slot)
    layout: int    # 2 or 3 (VR3 file tensors)


class ModelFile:
    def __init__(self, path):
        h = C.c_void_p()
        check(lib().p8_gguf_open(str(path).encode(), C.byref(h)), f"p8_gguf_open({path})")
        self._h = h
        self.linears = []
        for i in range(int(lib().p8_gguf_n_linear(h))):
            name = C.c_char_p()
            K, rows, nd = C.c_int64(), C.c_int64(), C.c_int64()
            nb, lay = C.c_size_t(), C.c_int()
            check(lib().p8_gguf_linear_info(h, i, C.byref(name), C.byref(K), C.byref(rows), C.byref(nd), C.byref(nb),
                                            C.byref(lay)), "p8_gguf_linear_info")
            self.linears.append(LinearInfo(i, name.value.decode(), K.value, rows.value, nd.value, nb.value, lay.value))
        self._by_name = {li.name: li for li in self.linears}

    def info(self, key):
        return self.linears[key] if isinstance(key, int) else self._by_name[key]

    def slot(self, key):
        """host slot bytes (numpy uint8) of linear `key` (index or <base>.weight name)"""
        li = self.info(key)
        out = np.empty(li.nbytes, np.uint8)
        n = C.c_size_t(0)
        check(lib().p8_gguf_load_linear(self._h, li.index, out.ctypes.data_as(C.c_void_p), out.size, C.byref(n)),
              f"p8_gguf_load_linear({li.name})")
        return out[: n.value]

    def tensor(self, key, device="cuda", stream=None):
        """linear `key` uploaded and prepared (P8Tensor)"""
        import torch

        from .ops import P8Tensor

        li = self.info(key)
        return P8Tensor(torch.from_numpy(self.slot(li.index)).to(device), li.K, li.rows, stream=stream)

    def close(self):
        if self._h:
            lib().p8_gguf_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
