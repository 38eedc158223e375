"""The two-column batch-1 GEMV (k_gemv2 + k_gemv_reduce2: batched decode of 2 or 3 sequences, the weights decoded
once for two columns) through the C ABI: every column must equal the one-column call on that column bit for bit (the
same exact-integer tables, the same lane-sum and row-reduce order), for every input op, a group of tensors, clamp
deltas and a row permutation; and the CPU oracle on the inputs within the path's bar.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from pingala8_llm_b200 import synth  # noqa: E402
from pingala8_llm_b200.ops import P8Tensor, device_error, mul_mat_group, mul_mat_vec_group  # noqa: E402
from oracle.oracle import Oracle  # noqa: E402

K = 2048


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def inputs(ncols, prologue, seed):
    rng = np.random.default_rng(seed)
    X = torch.from_numpy((rng.normal(0, 1, (ncols, K)) * rng.uniform(0.2, 20, (ncols, 1))).astype(np.float32)).cuda()
    if prologue == "rmsnorm":
        return X, dict(norm_weight=torch.from_numpy(rng.normal(1, 0.3, K).astype(np.float32)).cuda(), eps=1e-5)
    if prologue == "swiglu":
        return X, dict(up=torch.from_numpy(rng.normal(0, 1, (ncols, K)).astype(np.float32)).cuda())
    return X, {}


def column_kw(kw, n):
    return {k: (v[n] if k == "up" else v) for k, v in kw.items()}


@pytest.mark.parametrize("prologue", ["none", "rmsnorm", "swiglu"])
@pytest.mark.parametrize("ncols", [2, 3])
def test_two_columns_equal_one_column_calls(ncols, prologue):
    t = P8Tensor(synth.make_slot(1536, K, classes=3, seed=41, nd=9), K, 1536)
    X, kw = inputs(ncols, prologue, ncols)
    Y = t.mul_mat(X, **kw)
    torch.cuda.synchronize()
    assert device_error() == 0
    for n in range(ncols):
        y = mul_mat_vec_group([t], X[n], **column_kw(kw, n))[0]
        assert torch.equal(Y[n], y), (n, prologue)
    if prologue == "none":  # and the reference restatement on the same inputs
        o = Oracle(t.slot.cpu().numpy(), t.rows, t.K).mul_mat(X.cpu().numpy())
        assert rel(Y.cpu().numpy(), o) < 1e-5


@pytest.mark.parametrize("prologue", ["none", "rmsnorm", "swiglu"])
def test_two_column_group_equals_one_column_calls(prologue):
    ts = [P8Tensor(synth.make_slot(r, K, classes=3, seed=50 + i, nd=4), K, r) for i, r in enumerate((1024, 512, 512))]
    X, kw = inputs(2, prologue, 7)
    Ys = mul_mat_group(ts, X, **kw)
    torch.cuda.synchronize()
    for n in range(2):
        ys = mul_mat_vec_group(ts, X[n], **column_kw(kw, n))
        for Y, y in zip(Ys, ys):
            assert torch.equal(Y[n], y), (n, prologue)


def test_two_columns_with_strided_input_and_output():
    t = P8Tensor(synth.make_slot(1024, K, classes=3, seed=61, nd=3), K, 1024)
    big = torch.randn(2, K + 64, device="cuda")
    X = big[:, :K]  # row stride K + 64 (a multiple of 4 floats)
    out = torch.full((2, 1024 + 32), float("nan"), device="cuda")[:, :1024]
    t.mul_mat(X, out=out)
    torch.cuda.synchronize()
    for n in range(2):
        assert torch.equal(out[n], t.mul_mat_vec(X[n].contiguous()))
