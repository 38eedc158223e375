"""GPU parity: every CUDA entry point against the CPU oracle / the reference's stored outputs, through the C ABI.

Bars (the path's stated targets): integer decode and f32 dequant BIT-EXACT vs the reference CPU path; GEMV / batched
product within 1e-3 relative L2 of the reference's x16 CPU vec_dot (the GEMV's integer sums are exact, so the
measured gap is float rounding, ~1e-7; the tests assert 1e-5 and the 1e-3 bar).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # the gpu marker is deselected on CPU runs; guard direct invocations too
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

import pingala8_llm_b200 as p8  # noqa: E402
from pingala8_llm_b200 import synth  # noqa: E402
from pingala8_llm_b200.ops import P8Tensor, active  # noqa: E402
from oracle.oracle import Oracle, RefOracle  # noqa: E402

from conftest import fixture_names, load_fixture  # noqa: E402

BAR = 1e-3    # north_star tolerance (relative L2, fp32 accumulate)
TIGHT = 1e-5  # what the exact-integer GEMV actually achieves


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.fixture(scope="module")
def prepared():
    cache = {}

    def get(name):
        if name not in cache:
            f = load_fixture(name)
            cache[name] = (f, P8Tensor(f.slot, f.K, f.rows), Oracle(f.slot, f.rows, f.K))
        return cache[name]

    return get


@pytest.mark.parametrize("name", fixture_names())
def test_decode_int_bit_exact(prepared, name):
    f, t, o = prepared(name)
    assert np.array_equal(t.decode_int().cpu().numpy(), o.decode_int())


@pytest.mark.parametrize("name", fixture_names())
def test_dequant_bit_exact(prepared, name):
    f, t, o = prepared(name)
    W = t.dequant().cpu().numpy()
    assert np.array_equal(W.view(np.uint32), o.dequant().view(np.uint32))


@pytest.mark.parametrize("name", fixture_names())
def test_get_rows_bit_exact(prepared, name):
    f, t, o = prepared(name)
    rng = np.random.default_rng(7)
    ids = np.unique(np.concatenate([[0, f.rows - 1], rng.integers(0, f.rows, 13)])).astype(np.int32)
    out = t.get_rows(torch.from_numpy(ids).cuda()).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), o.get_rows(ids).view(np.uint32))


@pytest.mark.parametrize("name", fixture_names())
def test_gemv_vs_reference_cpu(prepared, name):
    f, t, o = prepared(name)
    y = t.mul_mat_vec(torch.from_numpy(f.x).cuda()).cpu().numpy()
    r = rel(y, f.y_ref)
    assert r < TIGHT and r < BAR, r


@pytest.mark.parametrize("name", fixture_names())
@pytest.mark.parametrize("ncols", [2, 8])
def test_mul_mat_vs_reference_cpu(prepared, name, ncols):
    f, t, o = prepared(name)
    X = torch.from_numpy(f.X[:ncols]).cuda()
    Y = t.mul_mat(X).cpu().numpy()
    assert rel(Y, f.Y_ref[:ncols]) < BAR


def test_gemv_deterministic_and_graph_capturable(prepared):
    f, t, o = prepared("c1_1024x2560_c3")
    x = torch.from_numpy(f.x).cuda()
    y1 = t.mul_mat_vec(x).clone()
    y2 = t.mul_mat_vec(x).clone()
    assert torch.equal(y1, y2)
    ws = t.workspace(1)
    out = torch.empty_like(y1)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        t.mul_mat_vec(x, out=out, workspace=ws, stream=s)  # warm-up on the capture stream
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            t.mul_mat_vec(x, out=out, workspace=ws, stream=s)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, y1)


# --------------------------------------------------------------------------- benchmark shapes (synthetic, full size)
SHAPES = [
    ("c1_ffn_up", 9728, 2560),          # config C1 (Qwen3-4B ffn_up)
    ("llama_q", 4096, 4096),
    ("llama_kv", 1024, 4096),
    ("llama_gate", 14336, 4096),
    ("llama_down", 4096, 14336),
    ("qwen4b_down", 2560, 9728),
]


@pytest.mark.parametrize("label,rows,K", SHAPES)
def test_full_size_gemv_vs_oracle(label, rows, K):
    """Benchmark shapes at full size against the restated oracle AND the reference's own CPU core (oracle/_ref,
    vrc_tg with x16 activations) on the same slot and input"""
    s = synth.make_slot(rows, K, seed=rows + K, nd=37)
    t = P8Tensor(s, K, rows)
    o = Oracle(s, rows, K)
    x = np.random.default_rng(1).normal(0, 1, K).astype(np.float32)
    y = t.mul_mat_vec(torch.from_numpy(x).cuda()).cpu().numpy()
    r = rel(y, o.mul_mat(x)[0])
    assert r < TIGHT, r
    if RefOracle.available():
        r_ref = rel(y, RefOracle(s, rows, K).gemv(x))
        assert r_ref < TIGHT, r_ref


@pytest.mark.parametrize("rows,K", [(256, 49152), (256, 65280)])
def test_gemv_table_refills_long_rows(rows, K):
    """Few rows and long K: a CTA's units span three 256-column blocks, so a table buffer is refilled (by the last warp
    done with it) while other warps still work on the previous block. K = 65280 is the largest K a slot can hold."""
    s = synth.make_slot(rows, K, seed=rows + K, nd=7)
    t = P8Tensor(s, K, rows)
    o = Oracle(s, rows, K)
    x = np.random.default_rng(rows).normal(0, 1, K).astype(np.float32)
    y1 = t.mul_mat_vec(torch.from_numpy(x).cuda()).cpu().numpy()
    y2 = t.mul_mat_vec(torch.from_numpy(x).cuda()).cpu().numpy()
    assert rel(y1, o.mul_mat(x)[0]) < TIGHT
    assert np.array_equal(y1, y2)


@pytest.mark.parametrize("label,rows,K", SHAPES[:3])
def test_full_size_unit_vector_property(label, rows, K):
    """Size-independent property: W e_k is column k of W. x16 quantises a Hadamard-rotated unit vector exactly, so
    the GEMV of e_k equals the (bit-exact) dequant column up to float rounding."""
    s = synth.make_slot(rows, K, seed=3 * rows + K, nd=11)
    t = P8Tensor(s, K, rows)
    W = t.dequant()
    for k in (0, K // 3, K - 1):
        x = torch.zeros(K, dtype=torch.float32, device="cuda")
        x[k] = 1.0
        y = t.mul_mat_vec(x)
        assert rel(y.cpu().numpy(), W[:, k].cpu().numpy()) < 1e-5


@pytest.mark.parametrize("cls", [1, 2, 4, 5, 6, 7])
def test_all_classes_full_tiles_vs_oracle(cls):
    rows, K = (512, 2048) if cls < 7 else (512, 2048)
    s = synth.make_slot(rows, K, classes=cls, seed=cls, nd=9, c16="random")
    t = P8Tensor(s, K, rows)
    o = Oracle(s, rows, K)
    assert np.array_equal(t.dequant().cpu().numpy().view(np.uint32), o.dequant().view(np.uint32))
    x = np.random.default_rng(cls).normal(0, 1, K).astype(np.float32)
    assert rel(t.mul_mat_vec(torch.from_numpy(x).cuda()).cpu().numpy(), o.mul_mat(x)[0]) < TIGHT


def test_mixed_class_tiles_vs_oracle():
    rows, K = 1024, 2048
    cls = np.random.default_rng(5).integers(0, 8, (rows // 32, K // 256))
    s = synth.make_slot(rows, K, classes=cls, seed=9, nd=21)
    t = P8Tensor(s, K, rows)
    o = Oracle(s, rows, K)
    assert np.array_equal(t.decode_int().cpu().numpy(), o.decode_int())
    x = np.random.default_rng(2).normal(0, 1, K).astype(np.float32)
    assert rel(t.mul_mat_vec(torch.from_numpy(x).cuda()).cpu().numpy(), o.mul_mat(x)[0]) < TIGHT


def test_group_gemv_equals_single_calls():
    """q/k/v (and gate/up) as one grouped launch == three single calls, bit for bit (exact fixed-point accumulation)."""
    from pingala8_llm_b200.ops import mul_mat_vec_group

    shapes = [(1024, 2048), (256, 2048), (256, 2048)]
    ts = [P8Tensor(synth.make_slot(r, k, seed=40 + i, nd=3 * i), k, r) for i, (r, k) in enumerate(shapes)]
    x = torch.randn(2048, device="cuda")
    ys = mul_mat_vec_group(ts, x)
    for t, y in zip(ts, ys):
        assert torch.equal(y, t.mul_mat_vec(x))
    o = Oracle(ts[0].slot.cpu().numpy(), 1024, 2048)
    assert rel(ys[0].cpu().numpy(), o.mul_mat(x.cpu().numpy())[0]) < TIGHT
    other = P8Tensor(synth.make_slot(256, 2048, seed=1, c16="random"), 2048, 256)
    with pytest.raises(p8.P8Error):  # different column scales: cannot share the prepared activation
        mul_mat_vec_group([ts[0], other], x)


# --------------------------------------------------------------------------- error behaviour through the C ABI
def test_prepare_rejects_corrupted_device_slot():
    f = load_fixture("cls3_64x512")
    bad = f.slot.copy()
    bad[-32] ^= 1  # trailer magic
    with pytest.raises(p8.P8Error) as e:
        P8Tensor(bad, f.K, f.rows)
    assert e.value.status == -2
    bad = f.slot.copy()
    bad[2052] = 104  # header NS
    with pytest.raises(p8.P8Error) as e:
        P8Tensor(bad, f.K, f.rows)
    assert e.value.status == -3


def test_workspace_and_handle_errors():
    f = load_fixture("cls3_64x512")
    t = P8Tensor(f.slot, f.K, f.rows)
    assert active(t.slot)
    x = torch.from_numpy(f.x).cuda()
    small = torch.empty(16, dtype=torch.uint8, device="cuda")
    with pytest.raises(p8.P8Error) as e:
        t.mul_mat_vec(x, workspace=small)
    assert e.value.status == -11
    t.release()
    assert not active(t.slot)
    with pytest.raises(p8.P8Error):
        t.mul_mat_vec(x)
    with pytest.raises(p8.P8Error):
        P8Tensor(f.slot, f.K + 256, f.rows)
    assert p8.device_error() == 0
