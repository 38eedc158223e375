"""pingala8_llm_b200 -- B200-native (sm_100a) Pingala-8 quantized-weight matmul path.

Drop-in for the reference's ggml Pingala-8 hooks (Genrius-AI/pingala8-llm): batch-1 table GEMV, batched product,
get_rows / f32 dequant, and a tensor-parallel split. The compute lives in libpingala8_b200.so (C ABI:
include/pingala8.h); this package is the thin host mirror over it.
"""
from ._lib import LIB_PATH, P8Error, P8_STATUS, header_functions, lib  # noqa: F401
from . import fmt, synth  # noqa: F401

__all__ = ["P8Error", "P8Tensor", "fmt", "synth", "lib", "active", "device_error"]


def __getattr__(name):
    # the torch-facing operator layer is imported lazily so the host format helpers work without CUDA
    if name in ("P8Tensor", "active", "device_error", "mul_mat_vec_group", "group_workspace_size", "mul_mat_group"):
        import importlib

        return getattr(importlib.import_module(".ops", __name__), name)
    raise AttributeError(name)
