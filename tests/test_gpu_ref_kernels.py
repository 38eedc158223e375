"""The reference's own batch-1 GEMV kernels (k_vr_qx_real + k_vr<1, V, 8, 108>, compiled from its patch into
oracle/_ref/libp8ref_gpu.so) on the golden fixtures: the same-box GPU comparison arm must compute the product it is
timed on. Its activations are int8 per 128 columns (not the CPU core's x16), so it is held to 3e-2 relative L2 against
the reference CPU core's y (measured q8 error is a few 1e-3), not to the 1e-3 bar this library meets.

Test infrastructure for the comparison arm only: nothing of the product library is loaded here.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from oracle.oracle import RefGpu  # noqa: E402

from conftest import fixture_names, load_fixture  # noqa: E402

if not RefGpu.available():
    pytest.skip("oracle/_ref/libp8ref_gpu.so not built (needs the reference patch at build time)", allow_module_level=True)

Q8_BAR = 3e-2


@pytest.mark.parametrize("V", [5, 7])
@pytest.mark.parametrize("name", [n for n in fixture_names() if n.startswith(("c1_1024", "cls3", "cls7", "mix", "dl_"))])
def test_reference_kernels_compute_the_product(name, V):
    f = load_fixture(name)
    dev = torch.device("cuda", 0)
    RefGpu.set_tables(f.slot)
    slot = torch.from_numpy(f.slot).to(dev)
    x = torch.from_numpy(np.ascontiguousarray(f.x, np.float32)).to(dev)
    y = torch.empty(f.rows, device=dev)
    xq = torch.empty(f.K, dtype=torch.int8, device=dev)
    xs = torch.empty(f.K // 128, device=dev)
    nd = int(f.meta.get("nd", 0))
    RefGpu.gemv(slot.data_ptr(), f.slot.size, f.rows, f.K, nd, x.data_ptr(), y.data_ptr(), xq.data_ptr(), xs.data_ptr(),
                V=V, RL=1, stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    yg = y.cpu().numpy().astype(np.float64)
    yr = f.y_ref.astype(np.float64)
    err = float(np.linalg.norm(yg - yr) / np.linalg.norm(yr))
    assert err < Q8_BAR, f"{name} V{V}: relative L2 {err:.3e}"
