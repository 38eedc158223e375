"""GPU parity of the chained batch-1 GEMV (p8_chain_*: a run of projections in one persistent launch), through the C ABI.

Each chain output is compared with the separate per-op calls (p8_mul_mat_vec_group_ex) on the SAME inputs (the chain's
own previous outputs, so errors do not compound) and with the CPU oracle on those inputs. The chain applies the
RMSNorm scale to the product instead of to its input, which moves the x16 quantisation by float rounding only; the
bar is 1e-4 relative L2 (the prologue tests' bar), against 1e-3 for the path.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

import pingala8_llm_b200 as p8  # noqa: E402
from pingala8_llm_b200 import synth  # noqa: E402
from pingala8_llm_b200.ops import Chain, P8Tensor, device_error, mul_mat_vec_group  # noqa: E402
from oracle.oracle import Oracle  # noqa: E402

BAR = 1e-4


def rel(a, b):
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / b.norm())


def rmsnorm(x, w, eps):
    return (x * torch.rsqrt(torch.mean(x * x) + eps)) * w


def layer(hidden, q, kv, ffn, seed, nd=5, classes=3):
    mk = lambda r, k, i: P8Tensor(synth.make_slot(r, k, classes=classes, seed=seed + i, nd=nd), k, r)  # noqa: E731
    return dict(q=mk(q, hidden, 0), k=mk(kv, hidden, 1), v=mk(kv, hidden, 2), o=mk(hidden, q, 3), gate=mk(ffn, hidden, 4),
                up=mk(ffn, hidden, 5), down=mk(hidden, ffn, 6))


def buffers(L, dev="cuda"):
    return {n: torch.empty(t.rows, device=dev) for n, t in L.items()}


def llama_chain(L, L2, x0, y, y2, w, eps):
    """o (+ x0) -> gate/up (RMSNorm) -> down (SwiGLU, + h) -> next layer's q/k/v (RMSNorm), with the layer's own
    q/k/v (RMSNorm on x0) first: five steps covering every prologue, residuals, a 3-tensor and a 2-tensor step, and
    outputs the next step does not read (k, v)"""
    return [
        dict(tensors=[L["q"], L["k"], L["v"]], x=x0, outs=[y["q"], y["k"], y["v"]], norm_weight=w[0], eps=eps),
        dict(tensors=[L["o"]], x=y["q"], outs=[y["o"]], res=[x0]),
        dict(tensors=[L["gate"], L["up"]], x=y["o"], outs=[y["gate"], y["up"]], norm_weight=w[1], eps=eps),
        dict(tensors=[L["down"]], x=y["gate"], up=y["up"], outs=[y["down"]], res=[y["o"]]),
        dict(tensors=[L2["q"], L2["k"], L2["v"]], x=y["down"], outs=[y2["q"], y2["k"], y2["v"]], norm_weight=w[2], eps=eps),
    ]


def check_against_separate_calls(L, L2, x0, y, y2, w, eps, oracle=True):
    # step by step on the chain's own inputs
    ref = {}
    ref["q"], ref["k"], ref["v"] = mul_mat_vec_group([L["q"], L["k"], L["v"]], x0, norm_weight=w[0], eps=eps)
    ref["o"] = L["o"].mul_mat_vec(y["q"]) + x0
    ref["gate"], ref["up"] = mul_mat_vec_group([L["gate"], L["up"]], y["o"], norm_weight=w[1], eps=eps)
    ref["down"] = mul_mat_vec_group([L["down"]], y["gate"], up=y["up"])[0] + y["o"]
    r2 = mul_mat_vec_group([L2["q"], L2["k"], L2["v"]], y["down"], norm_weight=w[2], eps=eps)
    for n in ref:
        assert rel(y[n], ref[n]) < BAR, (n, rel(y[n], ref[n]))
    for n, r in zip(("q", "k", "v"), r2):
        assert rel(y2[n], r) < BAR, ("next " + n, rel(y2[n], r))
    if not oracle:
        return
    # the CPU oracle (x16 GEMV) on numpy's prologue of the chain's inputs, for the o and down steps
    xo = y["q"].cpu().numpy()
    yo = Oracle(L["o"].slot.cpu().numpy(), L["o"].rows, L["o"].K).mul_mat(xo)[0] + x0.cpu().numpy()
    assert rel(y["o"], yo) < BAR
    g, u = y["gate"].cpu().numpy().astype(np.float64), y["up"].cpu().numpy().astype(np.float64)
    xd = (g / (1 + np.exp(-g)) * u).astype(np.float32)
    yd = Oracle(L["down"].slot.cpu().numpy(), L["down"].rows, L["down"].K).mul_mat(xd)[0] + y["o"].cpu().numpy()
    assert rel(y["down"], yd) < BAR


@pytest.mark.parametrize("dims", [(1024, 1024, 256, 2048), (4096, 4096, 1024, 14336)])
def test_chain_layer_matches_separate_calls(dims):
    hidden, q, kv, ffn = dims
    L, L2 = layer(hidden, q, kv, ffn, seed=11), layer(hidden, q, kv, ffn, seed=71)
    y, y2 = buffers(L), buffers(L2)
    x0 = torch.randn(hidden, device="cuda")
    w = [torch.rand(hidden, device="cuda") + 0.5 for _ in range(3)]
    ch = Chain(llama_chain(L, L2, x0, y, y2, w, 1e-5))
    ch.run()
    torch.cuda.synchronize()
    assert device_error() == 0
    check_against_separate_calls(L, L2, x0, y, y2, w, 1e-5, oracle=hidden <= 1024)


def test_chain_mixed_classes_and_deltas():
    """every class 0..7 in random tiles (the table loop's general path), clamp deltas in every tensor"""
    hidden, q, kv, ffn = 1024, 1024, 256, 2048
    cls = lambda r, k, s: np.random.default_rng(s).integers(0, 8, (r // 32, k // 256))  # noqa: E731
    L = {}
    shapes = dict(q=(q, hidden), k=(kv, hidden), v=(kv, hidden), o=(hidden, q), gate=(ffn, hidden), up=(ffn, hidden),
                  down=(hidden, ffn))
    for i, (n, (r, k)) in enumerate(shapes.items()):
        L[n] = P8Tensor(synth.make_slot(r, k, classes=cls(r, k, i), seed=300 + i, nd=17), k, r)
    L2 = layer(hidden, q, kv, ffn, seed=91)
    y, y2 = buffers(L), buffers(L2)
    x0 = torch.randn(hidden, device="cuda")
    w = [torch.rand(hidden, device="cuda") + 0.5 for _ in range(3)]
    Chain(llama_chain(L, L2, x0, y, y2, w, 1e-6)).run()
    torch.cuda.synchronize()
    assert device_error() == 0
    check_against_separate_calls(L, L2, x0, y, y2, w, 1e-6)


def test_chain_single_step_equals_gemv():
    t = P8Tensor(synth.make_slot(9728, 2560, seed=5, nd=29), 2560, 9728)
    x = torch.randn(2560, device="cuda")
    y = torch.empty(9728, device="cuda")
    Chain([dict(tensors=[t], x=x, outs=[y])]).run()
    ref = t.mul_mat_vec(x)
    torch.cuda.synchronize()
    assert rel(y, ref) < 1e-6


def test_chain_long_rows_two_blocks_per_cta():
    """64 rows x 65280 columns: 2 tiles per block, so most CTAs' units span two 256-column blocks (two tables)"""
    rows, K = 64, 65280
    t = P8Tensor(synth.make_slot(rows, K, seed=6, nd=7), K, rows)
    x = torch.randn(K, device="cuda")
    y = torch.empty(rows, device="cuda")
    Chain([dict(tensors=[t], x=x, outs=[y])]).run()
    o = Oracle(t.slot.cpu().numpy(), rows, K)
    torch.cuda.synchronize()
    assert rel(y, o.mul_mat(x.cpu().numpy())[0]) < 1e-5


def test_chain_graph_replay_and_determinism():
    hidden, q, kv, ffn = 1024, 1024, 256, 2048
    L, L2 = layer(hidden, q, kv, ffn, seed=21), layer(hidden, q, kv, ffn, seed=23)
    y, y2 = buffers(L), buffers(L2)
    x0 = torch.randn(hidden, device="cuda")
    w = [torch.rand(hidden, device="cuda") + 0.5 for _ in range(3)]
    ch = Chain(llama_chain(L, L2, x0, y, y2, w, 1e-5))
    ch.run()
    torch.cuda.synchronize()
    written = {**y, **{"n" + k: y2[k] for k in ("q", "k", "v")}}  # the chain writes every y and the next q, k, v
    first = {n: v.clone() for n, v in written.items()}
    ws = torch.empty(ch.workspace_size(), dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        ch.run(workspace=ws, stream=s)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            ch.run(workspace=ws, stream=s)
    for v in list(y.values()) + list(y2.values()):
        v.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert device_error() == 0
    now = written
    for n in first:
        assert torch.equal(first[n], now[n]), n


def test_chain_rejects_overlaps_and_bad_shapes():
    t = P8Tensor(synth.make_slot(512, 1024, seed=1), 1024, 512)
    t2 = P8Tensor(synth.make_slot(1024, 512, seed=2), 512, 1024)
    x = torch.randn(1024, device="cuda")
    y = torch.empty(512, device="cuda")
    big = torch.empty(2048, device="cuda")
    with pytest.raises(p8.P8Error):  # the next step reads part of the previous output (not exactly it)
        Chain([dict(tensors=[t], x=x, outs=[big[:512]]), dict(tensors=[t2], x=big[4:516], outs=[torch.empty(1024, device="cuda")])])
    with pytest.raises(p8.P8Error):  # the residual is the output itself
        Chain([dict(tensors=[t], x=x, outs=[y], res=[y])])
    with pytest.raises(p8.P8Error):  # the previous output (512 rows) read as x of a step with K = 1024
        Chain([dict(tensors=[t], x=x, outs=[big[:512]]), dict(tensors=[t], x=big[:1024], outs=[y])])
