"""The allocation-free GEMV entry point p8_mul_mat_vec_noalloc, called through the C ABI.

It serves callers that cannot allocate device memory when the op runs and have no scratch buffer to lend: its scratch
is a fixed device array inside the library. This file is collected last (tests/test_zz_*) so that a run stopping at
the first failure has already run every other test; it also passes on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

import pingala8_llm_b200 as p8  # noqa: E402
from pingala8_llm_b200 import synth  # noqa: E402
from pingala8_llm_b200.ops import P8Tensor  # noqa: E402

def noalloc(t, x):
    y = torch.empty(t.rows, dtype=torch.float32, device=x.device)
    st = p8.lib().p8_mul_mat_vec_noalloc(t.handle, C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()),
                                         C.c_void_p(torch.cuda.current_stream().cuda_stream))
    if st != 0:
        raise p8.P8Error(st, "p8_mul_mat_vec_noalloc")
    return y


@pytest.mark.parametrize("rows,K", [(4096, 4096), (14336, 4096), (4096, 14336), (1024, 2560)])
def test_noalloc_matches_workspace_entry_point_two_calls_in_a_row(rows, K):
    t = P8Tensor(synth.make_slot(rows, K, seed=rows + 3 * K, nd=13), K, rows)
    assert t.workspace_size(1) <= p8.lib().p8_noalloc_scratch_bytes()
    g = torch.Generator(device="cuda")
    g.manual_seed(rows)
    x1 = torch.randn(K, device="cuda", generator=g)
    x2 = torch.randn(K, device="cuda", generator=g)
    ref1, ref2 = t.mul_mat_vec(x1), t.mul_mat_vec(x2)
    y1 = noalloc(t, x1)  # two calls in a row share the scratch array
    y2 = noalloc(t, x2)
    torch.cuda.synchronize()
    # the same deterministic kernels on the same inputs: the same bits, not merely within tolerance
    assert torch.equal(y1, ref1) and torch.equal(y2, ref2)
    assert p8.device_error() == 0


def test_noalloc_rejects_tensors_beyond_its_scratch():
    rows, K = 32736, 12544  # row partials per 256-column block: 49 blocks x 32736 rows x 4 B = 6.4 MB > the 6 MiB array
    t = P8Tensor(synth.make_slot_device(rows, K, seed=5), K, rows)
    assert t.workspace_size(1) > p8.lib().p8_noalloc_scratch_bytes()
    with pytest.raises(p8.P8Error) as e:
        noalloc(t, torch.randn(K, device="cuda"))
    assert e.value.status == -11  # P8_ERR_WORKSPACE
