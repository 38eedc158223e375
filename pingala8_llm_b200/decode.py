"""Batch-1 decode of a llama-style model whose linear layers are Pingala-8 tensors: the workload the path serves.

Every projection runs through the C ABI: the prompt through the batched product (p8_mul_mat_group, tcgen05 GEMM) and
each decode token through the batch-1 GEMV (p8_mul_mat_vec_group), both with the layer's input ops fused (RMSNorm x
norm weight before q/k/v and gate/up, SwiGLU before down). The rest is ordinary torch: embeddings and the output head
in Q8_0 (blocks of 32 int8 with one fp16 scale, as the reference's model files keep them; the head multiplies the
Q8_0 values as fp16), RoPE, the optional per-head q/k RMSNorm of Qwen3, attention with torch SDPA over a static KV
cache, residual adds, greedy sampling. A decode step reads its position from the device and writes into fixed
buffers, so it is captured once as a CUDA graph and replayed per token.

The reference runs this model in llama.cpp (MUL_MAT nodes dispatched to ggml_cuda_f44_mul_mat_vec / _mul_mat_q8,
CU:1330-1342); its runtime is not available here, so this module restates the same architecture as a plain
fp32 torch forward (`reference_forward`) on weights given by the caller (the tests pass the CPU oracle's dequantised
weights) and the decoder's logits are compared against it.
"""
import math
from dataclasses import dataclass

import torch

from . import synth
from .ops import P8Tensor, group_workspace_size, mul_mat_group, mul_mat_vec_group


@dataclass(frozen=True)
class ModelConfig:
    name: str
    layers: int
    hidden: int
    ffn: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    rope_theta: float
    qk_norm: bool
    eps: float = 1e-6


QWEN3_4B = ModelConfig("qwen3-4b", 36, 2560, 9728, 32, 8, 128, 151936, 1e6, True)
LLAMA31_8B = ModelConfig("llama3.1-8b", 32, 4096, 14336, 32, 8, 128, 128256, 5e5, False, 1e-5)


def proj_shapes(c):
    """(name, rows, K) of a layer's Pingala-8 projections (ggml [K, rows])"""
    q, kv = c.heads * c.head_dim, c.kv_heads * c.head_dim
    return [("q", q, c.hidden), ("k", kv, c.hidden), ("v", kv, c.hidden), ("o", c.hidden, q), ("gate", c.ffn, c.hidden),
            ("up", c.ffn, c.hidden), ("down", c.hidden, c.ffn)]


class Q8_0:
    """A [rows, K] weight in Q8_0: per 32 consecutive values one fp16 scale d = max|w| / 127 and int8 q = round(w / d)."""

    def __init__(self, w):
        rows, K = w.shape
        wb = w.float().reshape(rows, K // 32, 32)
        d = (wb.abs().amax(-1) / 127.0).half()
        q = torch.where(d[..., None] > 0, torch.round(wb / d.float()[..., None]), torch.zeros_like(wb)).clamp(-127, 127)
        self.q, self.d, self.rows, self.K = q.to(torch.int8).reshape(rows, K), d, rows, K

    def dequant(self, rows=None):
        q = self.q if rows is None else self.q[rows]
        d = self.d if rows is None else self.d[rows]
        return (q.reshape(q.shape[0], -1, 32).float() * d.float()[..., None]).reshape(q.shape[0], self.K)


def rope_tables(c, max_len, device):
    inv = 1.0 / (c.rope_theta ** (torch.arange(0, c.head_dim, 2, dtype=torch.float64, device=device) / c.head_dim))
    ang = torch.arange(max_len, dtype=torch.float64, device=device)[:, None] * inv[None, :]
    return torch.cos(ang).float(), torch.sin(ang).float()  # [max_len, head_dim / 2]


def apply_rope(x, cos, sin):
    """x [..., T, head_dim] with cos / sin [T, head_dim / 2] (rotate-half form)"""
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def rms(x, w, eps):
    return (x * torch.rsqrt(torch.mean(x * x, dim=-1, keepdim=True) + eps)) * w


class Model:
    """Random-init weights of architecture c on one GPU. Projections: seeded random valid Pingala-8 codes (class 3,
    scales for sigma 0.02 weights); norms 1 + U(-0.1, 0.1); embeddings and head N(0, 0.02) in Q8_0."""

    def __init__(self, c, seed=0, device="cuda", layers=None, slots=None):
        self.c = c
        self.nl = layers or c.layers
        self.device = torch.device(device)
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        self.layers = []
        for L in range(self.nl):
            ts = {}
            for i, (n, r, k) in enumerate(proj_shapes(c)):
                s = slots[L][n] if slots is not None else synth.make_slot_device(r, k, seed=seed + 1000 * L + 17 * i, device=self.device)
                ts[n] = P8Tensor(s, k, r)
            norms = [1 + 0.2 * (torch.rand(c.hidden, device=self.device, generator=g) - 0.5) for _ in range(2)]
            qk = [1 + 0.2 * (torch.rand(c.head_dim, device=self.device, generator=g) - 0.5) for _ in range(2)] if c.qk_norm else None
            self.layers.append(dict(t=ts, attn_norm=norms[0], ffn_norm=norms[1], qk_norm=qk))
        self.final_norm = 1 + 0.2 * (torch.rand(c.hidden, device=self.device, generator=g) - 0.5)
        self.embed = Q8_0(0.02 * torch.randn(c.vocab, c.hidden, device=self.device, generator=g))
        self.head = Q8_0(0.02 * torch.randn(c.vocab, c.hidden, device=self.device, generator=g))
        self.head_w = self.head.dequant().half()  # the Q8_0 values exactly, as fp16 operands of the head GEMV

    # ------------------------------------------------------------------ state
    def alloc(self, max_len):
        c, dev = self.c, self.device
        self.max_len = max_len
        self.kv = torch.zeros(self.nl, 2, c.kv_heads, max_len, c.head_dim, device=dev)
        self.cos, self.sin = rope_tables(c, max_len, dev)
        shapes = {n: r for n, r, _ in proj_shapes(c)}
        self.buf = {n: torch.empty(r, device=dev) for n, r in shapes.items()}
        self.x = torch.empty(c.hidden, device=dev)
        self.h = torch.empty(c.hidden, device=dev)
        self.logits = torch.empty(c.vocab, device=dev)
        self.xl = torch.empty(c.hidden, device=dev)  # the final normed hidden state (the head's input)
        self.pos = torch.zeros(1, dtype=torch.int64, device=dev)
        self.tok = torch.zeros(1, dtype=torch.int64, device=dev)
        self.ws = torch.empty(max(group_workspace_size([L["t"][n] for n in g], 1, 1)
                                  for L in self.layers for g in (("q", "k", "v"), ("gate", "up"))), dtype=torch.uint8, device=dev)
        self.ws2 = torch.empty(max(group_workspace_size([L["t"][n]], 1, 2) for L in self.layers for n in ("o", "down")),
                               dtype=torch.uint8, device=dev)

    # ------------------------------------------------------------------ attention (torch)
    def _attend(self, L, layer, q, k, v, start, T):
        """q [T, heads * hd], k, v [T, kv * hd] of positions start .. start + T - 1 (start a python int or a device
        scalar for T = 1); writes k / v into the cache, returns [T, heads * hd]"""
        c = self.c
        q = q.view(T, c.heads, c.head_dim).transpose(0, 1)
        k = k.view(T, c.kv_heads, c.head_dim).transpose(0, 1)
        v = v.view(T, c.kv_heads, c.head_dim).transpose(0, 1)
        if c.qk_norm:
            q = rms(q, layer["qk_norm"][0], c.eps)
            k = rms(k, layer["qk_norm"][1], c.eps)
        if T == 1:
            cos, sin = self.cos.index_select(0, start), self.sin.index_select(0, start)
        else:
            cos, sin = self.cos[start:start + T], self.sin[start:start + T]
        q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
        if T == 1:
            self.kv[L, 0].index_copy_(1, start, k)
            self.kv[L, 1].index_copy_(1, start, v)
            valid = torch.arange(self.max_len, device=self.device) <= start
            mask = valid[None, None, :]
            o = torch.nn.functional.scaled_dot_product_attention(q[None], self.kv[L, 0][None], self.kv[L, 1][None],
                                                                 attn_mask=mask, enable_gqa=True)
        else:
            self.kv[L, 0, :, start:start + T] = k
            self.kv[L, 1, :, start:start + T] = v
            kk, vv = self.kv[L, 0, :, :start + T], self.kv[L, 1, :, :start + T]
            mask = torch.ones(T, start + T, dtype=torch.bool, device=self.device).tril(start)
            o = torch.nn.functional.scaled_dot_product_attention(q[None], kk[None], vv[None], attn_mask=mask[None, None],
                                                                 enable_gqa=True)
        return o[0].transpose(0, 1).reshape(T, c.heads * c.head_dim)

    # ------------------------------------------------------------------ prompt (batched product)
    def prefill(self, tokens):
        """tokens: int64 CUDA [T] at positions 0 .. T-1; returns the last position's logits"""
        c = self.c
        T = tokens.numel()
        x = self.embed.dequant(tokens)
        for L, layer in enumerate(self.layers):
            t = layer["t"]
            q, k, v = mul_mat_group([t["q"], t["k"], t["v"]], x, norm_weight=layer["attn_norm"], eps=c.eps)
            a = self._attend(L, layer, q, k, v, 0, T)
            h = x + t["o"].mul_mat(a.contiguous())
            g, u = mul_mat_group([t["gate"], t["up"]], h, norm_weight=layer["ffn_norm"], eps=c.eps)
            x = h + t["down"].mul_mat(g, up=u)
        self.xl.copy_(rms(x[-1], self.final_norm, c.eps))  # the fixed buffer the decode graph also writes
        return torch.mv(self.head_w, self.xl.half()).float()

    # ------------------------------------------------------------------ one decode token (graph-capturable)
    def step(self, stream=None):
        """self.tok at position self.pos -> self.logits; advances nothing on the host (the caller bumps pos / tok)"""
        c, b = self.c, self.buf
        self.x.copy_(self.embed.dequant(self.tok)[0])
        x = self.x
        for L, layer in enumerate(self.layers):
            t = layer["t"]
            mul_mat_vec_group([t["q"], t["k"], t["v"]], x, outs=[b["q"], b["k"], b["v"]], workspace=self.ws, stream=stream,
                              norm_weight=layer["attn_norm"], eps=c.eps)
            a = self._attend(L, layer, b["q"][None], b["k"][None], b["v"][None], self.pos, 1)[0]
            t["o"].mul_mat_vec(a.contiguous(), out=b["o"], workspace=self.ws2, stream=stream)
            torch.add(x, b["o"], out=self.h)
            mul_mat_vec_group([t["gate"], t["up"]], self.h, outs=[b["gate"], b["up"]], workspace=self.ws, stream=stream,
                              norm_weight=layer["ffn_norm"], eps=c.eps)
            mul_mat_vec_group([t["down"]], b["gate"], outs=[b["down"]], workspace=self.ws2, stream=stream, up=b["up"])
            torch.add(self.h, b["down"], out=self.x)
        self.xl.copy_(rms(self.x, self.final_norm, c.eps))
        self.logits.copy_(torch.mv(self.head_w, self.xl.half()).float())
        self.tok.copy_(torch.argmax(self.logits).view(1))

    def capture(self):
        """the decode step as a CUDA graph (buffers, KV cache, pos and tok are fixed device tensors)"""
        st = torch.cuda.Stream(device=self.device)
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            self.step(st)  # warm-up outside capture
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                self.step(st)
        torch.cuda.synchronize()
        self.graph, self.stream = g, st
        return g

    def generate(self, prompt, n_new, graph=True):
        """greedy: prompt tokens (int64 CUDA [T]) then n_new tokens; returns (tokens [n_new], logits of each step,
        final normed hidden state of each step)"""
        T = prompt.numel()
        if not hasattr(self, "kv") or self.max_len < T + n_new:
            self.alloc(T + n_new)
        self.kv.zero_()
        lg = self.prefill(prompt)
        self.tok.copy_(torch.argmax(lg).view(1))
        self.pos.fill_(T)
        out, logits, hid = [], [lg], [self.xl.clone()]
        if graph and not hasattr(self, "graph"):
            self.capture()
            self.kv.zero_()  # the capture's warm-up step wrote position T: redo the prompt
            lg = self.prefill(prompt)
            self.tok.copy_(torch.argmax(lg).view(1))
            self.pos.fill_(T)
            logits, hid = [lg], [self.xl.clone()]
        for i in range(n_new):
            out.append(self.tok.clone())
            if i == n_new - 1:
                break
            if graph:
                with torch.cuda.stream(self.stream):
                    self.graph.replay()
                torch.cuda.current_stream().wait_stream(self.stream)
            else:
                self.step()
            logits.append(self.logits.clone())
            hid.append(self.xl.clone())
            self.pos += 1
        return torch.cat(out), logits, hid


def reference_forward(c, weights, norms, embed, head, final_norm, seq):
    """The same architecture as a plain fp32 torch forward over the whole sequence seq (int64 [T], causal), on the
    given fp32 projection weights weights[L][name] [rows, K] (ORIGINAL row order), norms[L] = (attn_norm, ffn_norm,
    qk_norms or None), embed / head Q8_0 objects; returns (logits [T, vocab], final normed hidden states [T, hidden])
    of every position."""
    dev = seq.device
    T = seq.numel()
    cos, sin = rope_tables(c, T, dev)
    x = embed.dequant(seq)
    for L in range(len(weights)):
        W = weights[L]
        an, fn, qk = norms[L]
        xn = rms(x, an, c.eps)
        q = (xn @ W["q"].T).view(T, c.heads, c.head_dim).transpose(0, 1)
        k = (xn @ W["k"].T).view(T, c.kv_heads, c.head_dim).transpose(0, 1)
        v = (xn @ W["v"].T).view(T, c.kv_heads, c.head_dim).transpose(0, 1)
        if qk is not None:
            q, k = rms(q, qk[0], c.eps), rms(k, qk[1], c.eps)
        q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
        rep = c.heads // c.kv_heads
        k, v = k.repeat_interleave(rep, 0), v.repeat_interleave(rep, 0)
        s = (q @ k.transpose(-1, -2)) / math.sqrt(c.head_dim)
        s = s.masked_fill(~torch.ones(T, T, dtype=torch.bool, device=dev).tril(), float("-inf"))
        a = (torch.softmax(s, -1) @ v).transpose(0, 1).reshape(T, -1)
        h = x + a @ W["o"].T
        hn = rms(h, fn, c.eps)
        g, u = hn @ W["gate"].T, hn @ W["up"].T
        x = h + (torch.nn.functional.silu(g) * u) @ W["down"].T
    xl = rms(x, final_norm, c.eps)
    return xl @ head.dequant().T, xl
