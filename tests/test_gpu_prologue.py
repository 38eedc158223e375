"""Fused activation prologues of the decode GEMV (p8_mul_mat_vec_group_ex) against the oracle.

The reference runs RMSNorm, the norm-weight multiply and SwiGLU as separate ggml ops before the projection; here they
are computed in the GEMV's activation prep. The oracle's GEMV (the reference CPU core's x16 path restated) is applied
to the prologue's output computed in numpy fp32, and the bar is 1e-4 relative L2: the prologue itself is fp32 (its
sum of squares runs in a different order, and expf vs numpy's exp differ by an ulp), so one x16 activation can land
on the other side of a rounding step. Each case also checks that it would see clamp deltas applied to the raw input
instead of the prologue output (the GEMV's delta term must use x').
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from pingala8_llm_b200 import fmt, synth  # noqa: E402
from pingala8_llm_b200.ops import P8Tensor, device_error, mul_mat_vec_group  # noqa: E402
from oracle.oracle import Oracle  # noqa: E402

BAR = 1e-4


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def rmsnorm_np(x, w, eps):
    x = x.astype(np.float32)
    mean = np.float32(np.sum(x.astype(np.float64) ** 2) / x.size)
    scale = np.float32(1.0) / np.sqrt(np.float32(mean + np.float32(eps)))
    return ((x * scale).astype(np.float32) * w).astype(np.float32)


def swiglu_np(g, u):
    g = g.astype(np.float32)
    return ((g / (np.float32(1) + np.exp(-g))).astype(np.float32) * u).astype(np.float32)


def _tensors(specs, K, seed, nd=40):
    """tensors sharing K (and, from one seed family, the codebook/coset/signs of the shipped tables)"""
    out = []
    for i, rows in enumerate(specs):
        s = synth.make_slot(rows, K, seed=seed + i, nd=nd)
        out.append((s, rows, P8Tensor(s, K, rows)))
    return out


def _delta_shift(slot, rows, K, x_raw, x_pro):
    """y difference if the delta term used x_raw instead of x_pro"""
    _, _, _, (drow, dcol, dval), _ = fmt.split_kernel_bytes(slot, K, rows)
    d = np.zeros(rows)
    for r, c, v in zip(drow, dcol, dval):
        d[int(r)] += float(v) * (float(x_raw[int(c)]) - float(x_pro[int(c)]))
    return d


@pytest.mark.parametrize("K,rows,xscale", [(4096, (1024, 256, 256), 30.0), (2048, (512,), 0.01), (14336, (128,), 3.0)])
def test_rmsnorm_prologue(K, rows, xscale):
    ts = _tensors(rows, K, seed=11 + K)
    rng = np.random.default_rng(K)
    x = (rng.normal(0, 1, K) * xscale).astype(np.float32)
    w = rng.normal(1, 0.3, K).astype(np.float32)
    eps = 1e-5
    xp = rmsnorm_np(x, w, eps)
    ys = mul_mat_vec_group([t for _, _, t in ts], torch.from_numpy(x).cuda(), norm_weight=torch.from_numpy(w).cuda(), eps=eps)
    torch.cuda.synchronize()
    assert device_error() == 0
    for (s, r, _), y in zip(ts, ys):
        ref = Oracle(s, r, K).mul_mat(xp[None])[0]
        assert rel(y.cpu().numpy(), ref) < BAR
        wrong = ref + _delta_shift(s, r, K, x, xp)
        assert rel(wrong, ref) > 10 * BAR  # the case would see deltas applied to the raw x


@pytest.mark.parametrize("K,rows,nd", [(14336, 4096, 300), (2560, 512, 60)])
def test_swiglu_prologue(K, rows, nd):
    (s, r, t), = _tensors((rows,), K, seed=5 + K, nd=nd)
    rng = np.random.default_rng(rows)
    g = rng.normal(0, 2, K).astype(np.float32)
    u = rng.normal(0, 1, K).astype(np.float32)
    xp = swiglu_np(g, u)
    y = mul_mat_vec_group([t], torch.from_numpy(g).cuda(), up=torch.from_numpy(u).cuda())[0]
    torch.cuda.synchronize()
    assert device_error() == 0
    ref = Oracle(s, r, K).mul_mat(xp[None])[0]
    assert rel(y.cpu().numpy(), ref) < BAR
    assert rel(ref + _delta_shift(s, r, K, g, xp), ref) > 10 * BAR


def test_prologue_equals_plain_call_on_torch_prologue_and_is_deterministic():
    """fused vs the plain GEMV on x' computed by torch: the same x16 path, so only the prologue's own rounding differs;
    repeated and graph-replayed fused calls give identical bits"""
    K, rows = 4096, 2048
    (s, r, t), = _tensors((rows,), K, seed=77)
    x = torch.randn(K, device="cuda") * 4
    w = torch.rand(K, device="cuda") + 0.5
    up = torch.randn(K, device="cuda")
    y_n = mul_mat_vec_group([t], x, norm_weight=w, eps=1e-6)[0].clone()
    xp = (x * (1.0 / torch.sqrt(torch.mean(x * x) + 1e-6))) * w
    y_p = t.mul_mat_vec(xp)
    assert rel(y_n.cpu().numpy(), y_p.cpu().numpy()) < 1e-5
    y_s = mul_mat_vec_group([t], x, up=up)[0].clone()
    y_sp = t.mul_mat_vec(torch.nn.functional.silu(x) * up)
    assert rel(y_s.cpu().numpy(), y_sp.cpu().numpy()) < 1e-5
    ws = t.workspace(1)
    out = torch.empty(rows, device="cuda")
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        mul_mat_vec_group([t], x, outs=[out], workspace=ws, stream=st, norm_weight=w, eps=1e-6)
        st.synchronize()
        with torch.cuda.graph(g, stream=st):
            mul_mat_vec_group([t], x, outs=[out], workspace=ws, stream=st, norm_weight=w, eps=1e-6)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert device_error() == 0
    assert torch.equal(out, y_n)


def test_prologue_arguments_are_checked():
    import ctypes as C

    from pingala8_llm_b200._lib import Prologue, lib

    (s, r, t), = _tensors((256,), 1024, seed=3, nd=0)
    x = torch.randn(1024, device="cuda")
    y = torch.empty(256, device="cuda")
    ws = t.workspace(1)
    arr = (C.c_void_p * 1)(t.handle.value)
    ys = (C.c_void_p * 1)(y.data_ptr())
    w = torch.ones(1025, device="cuda")

    def call(pro):
        return lib().p8_mul_mat_vec_group_ex(arr, 1, C.c_void_p(x.data_ptr()), C.byref(pro), ys, C.c_void_p(ws.data_ptr()),
                                             ws.numel(), C.c_void_p(torch.cuda.current_stream().cuda_stream))

    assert call(Prologue(1, w.data_ptr() + 4, None, 1e-5)) == -1   # weight not 16-byte aligned
    assert call(Prologue(1, None, None, 1e-5)) == -1                # no weight
    assert call(Prologue(1, w.data_ptr(), None, -1.0)) == -1        # negative eps
    assert call(Prologue(2, None, None, 0.0)) == -1                 # SwiGLU without up
    assert call(Prologue(7, w.data_ptr(), None, 0.0)) == -1         # unknown kind
    assert call(Prologue(0, None, None, 0.0)) == 0                  # none: the plain call
    torch.cuda.synchronize()
    assert torch.equal(y, t.mul_mat_vec(x))


@pytest.mark.parametrize("ncols", [2, 16, 256])
def test_batched_rmsnorm_prologue(ncols):
    """p8_mul_mat_ex: RMSNorm per token (its own scale) with a shared weight; 2 tokens run the batch-1 GEMV per column
    (1e-4), 16 and 256 the tcgen05 GEMM (fp16 operands: the 1e-3 bar)"""
    K, rows = 4096, 512
    (s, r, t), = _tensors((rows,), K, seed=31, nd=120)
    rng = np.random.default_rng(ncols)
    X = (rng.normal(0, 1, (ncols, K)) * rng.uniform(0.1, 30, (ncols, 1))).astype(np.float32)
    w = rng.normal(1, 0.3, K).astype(np.float32)
    Xp = np.stack([rmsnorm_np(X[n], w, 1e-5) for n in range(ncols)])
    Y = t.mul_mat(torch.from_numpy(X).cuda(), norm_weight=torch.from_numpy(w).cuda(), eps=1e-5)
    torch.cuda.synchronize()
    assert device_error() == 0
    ref = Oracle(s, r, K).mul_mat(Xp)
    bar = BAR if ncols < 4 else 1e-3
    assert rel(Y.cpu().numpy(), ref) < bar
    wrong = ref + np.stack([_delta_shift(s, r, K, X[n], Xp[n]) for n in range(ncols)])
    assert rel(wrong, ref) > 10 * bar


@pytest.mark.parametrize("ncols", [3, 64])
def test_batched_swiglu_prologue(ncols):
    K, rows = 14336, 256
    (s, r, t), = _tensors((rows,), K, seed=41, nd=1000)
    rng = np.random.default_rng(ncols)
    G = rng.normal(0, 2, (ncols, K)).astype(np.float32)
    U = rng.normal(0, 1, (ncols, K)).astype(np.float32)
    Xp = swiglu_np(G, U)
    Y = t.mul_mat(torch.from_numpy(G).cuda(), up=torch.from_numpy(U).cuda())
    torch.cuda.synchronize()
    assert device_error() == 0
    ref = Oracle(s, r, K).mul_mat(Xp)
    bar = BAR if ncols < 4 else 1e-3
    assert rel(Y.cpu().numpy(), ref) < bar
    wrong = ref + np.stack([_delta_shift(s, r, K, G[n], Xp[n]) for n in range(ncols)])
    assert rel(wrong, ref) > 10 * bar
