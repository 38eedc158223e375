"""GPU parity of the batched product (tcgen05 GEMM: p8_mul_mat with ncols >= 4) through the C ABI.

Bar (the path's stated target): within 1e-3 relative L2 of the reference's CPU result (fp32 accumulate). The GEMM's
operands are fp16 (weights int * S, activations H256(x sgn/c) / 16, each with a power-of-two range scale), so its
error against the exact product is fp16 rounding, about 3e-4; the tests assert the 1e-3 bar.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from pingala8_llm_b200 import synth  # noqa: E402
from pingala8_llm_b200.ops import P8Tensor, device_error  # noqa: E402
from oracle.oracle import Oracle, RefOracle  # noqa: E402

from conftest import fixture_names, load_fixture  # noqa: E402

BAR = 1e-3


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def gemm(t, X, **kw):
    Y = t.mul_mat(X, **kw)
    torch.cuda.synchronize()
    assert device_error() == 0
    return Y


@pytest.mark.parametrize("name", fixture_names())
def test_gemm_vs_reference_cpu(name):
    """Golden fixtures (reference encoder + transcoder, Y_ref from the reference CPU core)."""
    f = load_fixture(name)
    t = P8Tensor(f.slot, f.K, f.rows)
    Y = gemm(t, torch.from_numpy(f.X).cuda()).cpu().numpy()
    assert rel(Y, f.Y_ref) < BAR


@pytest.mark.parametrize("rows,K,ncols", [(1024, 2560, 64), (4096, 4096, 200), (1024, 4096, 37), (96, 512, 8),
                                          (2560, 9728, 24), (4096, 4096, 4), (4096, 14336, 16)])
def test_gemm_vs_oracle_shapes(rows, K, ncols):
    """Model shapes plus ragged cases: rows not a multiple of 128, token counts not a multiple of the tile width; small
    token counts run split-K (CTAs share an output tile along K, the tile's last CTA sums the partials in order)."""
    s = synth.make_slot(rows, K, seed=rows + 7 * ncols, nd=23)
    t = P8Tensor(s, K, rows)
    o = Oracle(s, rows, K)
    X = np.random.default_rng(ncols).normal(0, 1, (ncols, K)).astype(np.float32)
    Y = gemm(t, torch.from_numpy(X).cuda()).cpu().numpy()
    assert rel(Y, o.mul_mat(X)) < BAR
    assert rel(Y, o.mul_mat_f64(X)) < BAR


@pytest.mark.parametrize("rows,K,ncols", [(20000, 1024, 40), (20000, 1024, 300), (9696, 2560, 512)])
def test_gemm_tail_split(rows, K, ncols):
    """Tile counts that fill some waves and leave a partial one: the row tiles of the full waves run single-split,
    the rest as a second launch split along K (direct stores at 40 tokens, staged outputs at 300 and 512; ragged last
    row tile at both row counts). The two smaller cases against the oracle, the 512-token one against the product
    with the dequantized weight in fp64 (the dequant is bit-exact to the oracle's)."""
    s = synth.make_slot(rows, K, seed=rows + ncols, nd=31)
    t = P8Tensor(s, K, rows)
    X = np.random.default_rng(ncols).normal(0, 1, (ncols, K)).astype(np.float32)
    Xd = torch.from_numpy(X).cuda()
    Y = gemm(t, Xd)
    if ncols <= 300:
        assert rel(Y.cpu().numpy(), Oracle(s, rows, K).mul_mat(X)) < BAR
    else:
        ref = (Xd.double() @ t.dequant().double().T)
        assert float(torch.linalg.norm(Y.double() - ref) / torch.linalg.norm(ref)) < BAR
    assert torch.equal(gemm(t, Xd), Y)  # deterministic (the tail's partials are summed in split order)


@pytest.mark.parametrize("cls", [1, 2, 3, 4, 5, 6, 7])
def test_gemm_each_class(cls):
    rows, K = 256, 1024
    s = synth.make_slot(rows, K, classes=cls, seed=10 + cls, nd=9, c16="random")
    t = P8Tensor(s, K, rows)
    o = Oracle(s, rows, K)
    X = np.random.default_rng(cls).normal(0, 1, (16, K)).astype(np.float32)
    assert rel(gemm(t, torch.from_numpy(X).cuda()).cpu().numpy(), o.mul_mat_f64(X)) < BAR


def test_gemm_mixed_classes_and_zero_tiles():
    rows, K = 512, 2048
    cls = np.random.default_rng(5).integers(0, 8, (rows // 32, K // 256))
    s = synth.make_slot(rows, K, classes=cls, seed=9, nd=21)
    t = P8Tensor(s, K, rows)
    o = Oracle(s, rows, K)
    X = np.random.default_rng(3).normal(0, 1, (48, K)).astype(np.float32)
    assert rel(gemm(t, torch.from_numpy(X).cuda()).cpu().numpy(), o.mul_mat_f64(X)) < BAR


def test_gemm_strides_and_extreme_token_scales():
    """ldx > K, ldy > rows; tokens spanning 1e-30 .. 1e30 (per-token power-of-two scale keeps each one accurate);
    an all-zero token gives zeros."""
    rows, K, n = 512, 1024, 12
    s = synth.make_slot(rows, K, seed=4, nd=0, c16="random")
    t = P8Tensor(s, K, rows)
    o = Oracle(s, rows, K)
    X = np.random.default_rng(4).normal(0, 1, (n, K))
    scales = np.array([1e-30, 1e-12, 1e-3, 1, 1, 10, 1e3, 1e12, 1e30, 1, 1, 0.0])
    X = (X * scales[:, None]).astype(np.float32)
    Xs = torch.zeros(n, K + 12, dtype=torch.float32, device="cuda")
    Xs[:, :K] = torch.from_numpy(X).cuda()
    Ys = torch.full((n, rows + 20), 7.0, dtype=torch.float32, device="cuda")
    Y = t.mul_mat(Xs[:, :K], out=Ys[:, :rows])
    torch.cuda.synchronize()
    assert device_error() == 0
    Y = Ys[:, :rows].cpu().numpy()
    ref = o.mul_mat_f64(X.astype(np.float64))
    for i in range(n - 1):
        assert rel(Y[i], ref[i]) < BAR, (i, scales[i])
    assert np.all(Y[n - 1] == 0)
    assert torch.all(Ys[:, rows:] == 7.0)  # nothing written outside the output rows


@pytest.mark.parametrize("label,rows,K,ncols", [("llama_gate", 14336, 4096, 512), ("llama_down", 4096, 14336, 256)])
def test_full_size_gemm_unit_vectors(label, rows, K, ncols):
    """Size-independent property at the benchmark shapes: a batch of unit vectors e_k gives the columns W[:, k] of the
    bit-exact dequantized weight (up to the operands' fp16 rounding)."""
    s = synth.make_slot_device(rows, K, seed=rows ^ K)
    t = P8Tensor(s, K, rows)
    W = t.dequant()
    ks = torch.from_numpy(np.random.default_rng(7).choice(K, ncols, replace=False)).cuda()
    X = torch.zeros(ncols, K, dtype=torch.float32, device="cuda")
    X[torch.arange(ncols, device="cuda"), ks] = 1.0
    Y = gemm(t, X)
    ref = W[:, ks].T.contiguous()
    err = torch.linalg.norm((Y - ref).double()) / torch.linalg.norm(ref.double())
    assert float(err) < BAR


@pytest.mark.parametrize("label,rows,K,ncols", [("llama_gate", 14336, 4096, 2048), ("llama_gate", 14336, 4096, 512),
                                                ("llama_down", 4096, 14336, 2048), ("llama_down", 4096, 14336, 512)])
def test_full_size_gemm_dense_tokens(label, rows, K, ncols):
    """Benchmark config C3 at its token counts with dense N(0, 1) activations (every token accumulates over all of K):
    against the product with the bit-exact dequantized weight in fp64 on a subset of 1024 rows, and the first 8
    tokens against the reference's own CPU core (oracle/_ref, x16 batch path) on every row"""
    s = synth.make_slot_device(rows, K, seed=rows + K + ncols, nd=0)
    t = P8Tensor(s, K, rows)
    g = torch.Generator(device="cuda")
    g.manual_seed(ncols)
    X = torch.randn(ncols, K, device="cuda", generator=g)
    Y = gemm(t, X)
    sub = torch.from_numpy(np.random.default_rng(ncols).choice(rows, 1024, replace=False)).cuda()
    W = t.dequant()[sub]
    ref = X.double() @ W.double().T
    err = float(torch.linalg.norm(Y[:, sub].double() - ref) / torch.linalg.norm(ref))
    assert err < BAR, err
    if RefOracle.available():
        r = RefOracle(s.cpu().numpy(), rows, K)
        Yr = r.mul_mat(X[:8].cpu().numpy())
        assert rel(Y[:8].cpu().numpy(), Yr) < BAR


def test_gemm_deterministic_and_graph_capturable():
    rows, K, n = 1024, 2048, 64
    s = synth.make_slot(rows, K, seed=21, nd=5)
    t = P8Tensor(s, K, rows)
    X = torch.randn(n, K, device="cuda")
    y1 = gemm(t, X).clone()
    y2 = gemm(t, X).clone()
    assert torch.equal(y1, y2)
    ws = t.workspace(n)
    out = torch.empty_like(y1)
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        t.mul_mat(X, out=out, workspace=ws, stream=st)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=st):
            t.mul_mat(X, out=out, workspace=ws, stream=st)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, y1)


def test_gemm_staged_outputs_with_strides():
    """From 64 tokens (single split) the outputs are written in sorted-row order first and un-permuted into Y: with
    ldx > K and ldy > rows, nothing outside the output rows is touched and every value matches the oracle"""
    rows, K, n = 768, 2048, 80
    s = synth.make_slot(rows, K, seed=12, nd=17, c16="random")
    t = P8Tensor(s, K, rows)
    o = Oracle(s, rows, K)
    X = np.random.default_rng(12).normal(0, 1, (n, K)).astype(np.float32)
    Xs = torch.zeros(n, K + 8, dtype=torch.float32, device="cuda")
    Xs[:, :K] = torch.from_numpy(X).cuda()
    Ys = torch.full((n, rows + 36), 7.0, dtype=torch.float32, device="cuda")
    t.mul_mat(Xs[:, :K], out=Ys[:, :rows])
    torch.cuda.synchronize()
    assert device_error() == 0
    assert rel(Ys[:, :rows].cpu().numpy(), o.mul_mat_f64(X.astype(np.float64))) < BAR
    assert torch.all(Ys[:, rows:] == 7.0)
