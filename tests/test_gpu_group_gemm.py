"""Grouped batched product (p8_mul_mat_group): tensors that read the same X share one activation prep.

The bar is bit-identity with separate p8_mul_mat / p8_mul_mat_ex calls, whose parity with the oracle the GEMM and
prologue tests hold; where two tensors of one shape share a launch ending in a K-split tail, those tail rows are
held to fp32 summation order instead. The row counts are chosen so that the tensors' plans pad the tokens differently (q: 4096 rows ->
128-token tiles, k/v: 1024 rows -> 64-token tiles at 300 tokens), so the shared prep is laid out for the larger
padding and the smaller tensors read a prefix of it. Token counts cover the per-column GEMV (2), split-K (32),
direct epilogue (48) and the staged epilogue (100, 300, 512).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

import pingala8_llm_b200 as p8  # noqa: E402
from pingala8_llm_b200 import synth  # noqa: E402
from pingala8_llm_b200.ops import P8Tensor, device_error, mul_mat_group  # noqa: E402
from oracle.oracle import Oracle  # noqa: E402

K = 2048


@pytest.fixture(scope="module")
def qkv():
    return [P8Tensor(synth.make_slot(rows, K, seed=70 + i, nd=60), K, rows) for i, rows in enumerate((4096, 1024, 1024))]


@pytest.mark.parametrize("ncols", [2, 32, 48, 100, 300, 512])
@pytest.mark.parametrize("prologue", ["none", "rmsnorm", "swiglu"])
def test_group_equals_separate_calls(qkv, ncols, prologue):
    rng = np.random.default_rng(ncols)
    X = torch.from_numpy((rng.normal(0, 1, (ncols, K)) * rng.uniform(0.2, 20, (ncols, 1))).astype(np.float32)).cuda()
    kw = {}
    if prologue == "rmsnorm":
        kw = dict(norm_weight=torch.from_numpy(rng.normal(1, 0.3, K).astype(np.float32)).cuda(), eps=1e-5)
    elif prologue == "swiglu":
        kw = dict(up=torch.from_numpy(rng.normal(0, 1, (ncols, K)).astype(np.float32)).cuda())
    ys = mul_mat_group(qkv, X, **kw)
    torch.cuda.synchronize()
    assert device_error() == 0
    for t, y in zip(qkv, ys):
        assert torch.equal(y, t.mul_mat(X, **kw)), (t.rows, ncols, prologue)
    assert device_error() == 0


def test_group_strided_outputs_and_oracle(qkv):
    """outputs written into column slices of one fused [ncols, q+k+v] buffer (ggml's views of a fused qkv dst)"""
    ncols = 200
    X = torch.randn(ncols, K, device="cuda")
    total = sum(t.rows for t in qkv)
    out = torch.full((ncols, total), float("nan"), device="cuda")
    views, o = [], 0
    for t in qkv:
        views.append(out[:, o:o + t.rows])
        o += t.rows
    mul_mat_group(qkv, X, outs=views)
    torch.cuda.synchronize()
    assert not torch.isnan(out).any()
    for t, v in zip(qkv, views):
        assert torch.equal(v, t.mul_mat(X))
    ref = Oracle(qkv[1].slot.cpu().numpy(), qkv[1].rows, K).mul_mat(X[:8].cpu().numpy())
    got = views[1][:8].cpu().numpy().astype(np.float64)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-3


def test_group_rejects_tensors_with_other_activation_tables(qkv):
    other = P8Tensor(synth.make_slot(1024, K, seed=1, c16="random"), K, 1024)
    X = torch.randn(64, K, device="cuda")
    with pytest.raises(p8.P8Error):
        mul_mat_group([qkv[0], other], X)


@pytest.mark.parametrize("rows,K,ncols", [(6144, 1024, 512), (9728, 2560, 32)])
def test_pair_sharing_one_launch(rows, K, ncols):
    """Two tensors of one shape (gate/up) whose row tiles fill the waves better together run as one k_gemm launch;
    here the joint launch ends in a tail split (the last row tiles of the second tensor summed over K splits). The
    first tensor and the second's other rows equal separate calls bit for bit, the tail rows within fp32 summation
    order; both against the dequantized weight at the 1e-3 bar."""
    ts = [P8Tensor(synth.make_slot(rows, K, seed=90 + i, nd=40), K, rows) for i in range(2)]
    X = torch.from_numpy(np.random.default_rng(ncols).normal(0, 1, (ncols, K)).astype(np.float32)).cuda()
    ys = mul_mat_group(ts, X)
    torch.cuda.synchronize()
    assert device_error() == 0
    sep = [t.mul_mat(X) for t in ts]
    assert torch.equal(ys[0], sep[0])
    same = (ys[1] == sep[1]).all(dim=0)
    assert int(same.sum()) >= rows // 3, int(same.sum())  # the rows outside the tail
    assert float(torch.linalg.norm(ys[1] - sep[1]) / torch.linalg.norm(sep[1])) < 1e-5
    for t, y in zip(ts, ys):
        ref = X.double() @ t.dequant().double().T
        assert float(torch.linalg.norm(y.double() - ref) / torch.linalg.norm(ref)) < 1e-3
    assert all(torch.equal(a, b) for a, b in zip(mul_mat_group(ts, X), ys))  # deterministic
