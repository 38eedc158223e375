"""Model-level decode (a llama-style model with every projection Pingala-8, through the C ABI) against a plain fp32
torch forward of the same architecture on the CPU oracle's dequantised weights.

The model is the Qwen3-4B architecture of benchmark config C2 (hidden 2560, FFN 9728, 32 query / 8 KV heads, head_dim
128, q/k RMSNorm, RoPE theta 1e6) with 2 of its 36 layers and an 8192-token vocabulary, so that the oracle's CPU dequant
and the fp32 reference stay small. The reference llama.cpp runtime is not available; the fp32 forward is its restatement.
Teacher forcing: the reference runs on the decoder's own token sequence, and the comparison is per position. Bars: the
final normed hidden state within 2e-3 relative L2 (x16 activations in the GEMV, fp16 operands in the prompt's GEMM,
compounded over the layers), the logits within 5e-3 (the head multiplies fp16 copies of its Q8_0 values).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from pingala8_llm_b200 import decode, synth  # noqa: E402
from pingala8_llm_b200.ops import device_error  # noqa: E402
from oracle.oracle import Oracle  # noqa: E402

CFG = decode.ModelConfig("qwen3-4b-2l", 2, 2560, 9728, 32, 8, 128, 8192, 1e6, True)


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


@pytest.fixture(scope="module")
def model_and_ref():
    slots = [{n: synth.make_slot(r, k, seed=100 * L + i, nd=3) for i, (n, r, k) in enumerate(decode.proj_shapes(CFG))}
             for L in range(CFG.layers)]
    m = decode.Model(CFG, seed=1, slots=slots)
    W = [{n: torch.from_numpy(Oracle(slots[L][n], r, k).dequant()).cuda() for n, r, k in decode.proj_shapes(CFG)}
         for L in range(CFG.layers)]
    norms = [(ly["attn_norm"], ly["ffn_norm"], ly["qk_norm"]) for ly in m.layers]
    return m, W, norms


@pytest.mark.parametrize("graph", [True, False])
def test_decode_logits_vs_fp32_reference(model_and_ref, graph):
    m, W, norms = model_and_ref
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    T, n_new = 12, 6
    prompt = torch.randint(0, CFG.vocab, (T,), device="cuda", generator=g)
    toks, logits, hid = m.generate(prompt, n_new, graph=graph)
    torch.cuda.synchronize()
    assert device_error() == 0
    seq = torch.cat([prompt, toks[:-1]])
    ref_logits, ref_xl = decode.reference_forward(CFG, W, norms, m.embed, m.head, m.final_norm, seq)
    for i in range(n_new):
        eh, el = rel(hid[i], ref_xl[T - 1 + i]), rel(logits[i], ref_logits[T - 1 + i])
        assert eh < 2e-3 and el < 5e-3, (i, eh, el)
    # greedy tokens follow the decoder's own logits
    assert all(int(toks[i]) == int(torch.argmax(logits[i])) for i in range(n_new))


def test_graph_and_eager_decode_agree(model_and_ref):
    m, _, _ = model_and_ref
    prompt = torch.arange(5, 17, device="cuda") * 97 % CFG.vocab
    t1, l1, _ = m.generate(prompt, 5, graph=True)
    t2, l2, _ = m.generate(prompt, 5, graph=False)
    assert torch.equal(t1, t2)
    for a, b in zip(l1, l2):
        assert torch.equal(a, b)
