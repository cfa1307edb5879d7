"""Whole-model decode-step oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/ and bench.py's baseline legs may import this module, as the
checker; the product package never does.

Restates in numpy float32, rounding to fp16 wherever the reference writes a
half buffer, the single-token decode step of kandiga/metal/full_forward_lg.m
(bakan_full_forward, 1078-1354 for an attention layer) with the kernels of
kandiga/metal/attention.metal it dispatches:

  embed_lookup           190-224   q * scale + bias (fma) -> half
  rmsnorm_forward        235-274   x / sqrt(mean(x^2) + eps) * w -> half
  rmsnorm_matvec_4bit    530-675   normed x (half) . dequantised rows -> half
  rope_kernel            697-734   pairs (i, i + rope_dim/2), theta^(-2i/rope_dim)
  gqa_attention_decode   752-849   softmax(q k / sqrt(hd)) v, q head h on kv head h / (nq / nkv)
  kv_cache_append        861-886
  rmsnorm_per_head       898-949   per-head RMSNorm with weight -> half
  sigmoid_gate_mul       1005-1017 attn * sigmoid(gate) -> half
  residual_add           1027-1037 half(a + b)
  split_q_gate           1350-1370 q_proj rows [head][q | gate]

The reference's step has a MoE block after attention; a dense decoder has a
SwiGLU MLP there instead: half(silu(gate x) * (up x)) then down, the expert
arithmetic of kandiga/metal/kandiga_cpu_expert.m:355-401 on one dense
matrix pair.

Parity unpinned: the reference's engine is Metal code and cannot run here.
The GPU engine and this oracle consume the same quantized weights, so the
comparison tests the arithmetic, within a floating-point tolerance.
"""
from __future__ import annotations

import numpy as np

from .oracle import dequantize_affine

F16 = np.float16
F32 = np.float32


def h(x):
    """round to fp16 and back (a half buffer between two kernels)"""
    return np.asarray(x, F32).astype(F16).astype(F32)


def rms(x, w, eps):
    x = np.asarray(x, F32)
    ss = F32((x * x).sum(dtype=F32))
    sc = F32(1.0) / np.sqrt(F32(ss / F32(x.shape[-1])) + F32(eps))
    return (x * sc) * np.asarray(w, F32)


def packed_rows(packed, bits, rows):
    """packed codes as the oracle's unpacker wants them: uint32 words (4-bit) or bytes (3-bit)"""
    b = np.ascontiguousarray(packed).view(np.uint8)
    return (b.view(np.uint32) if bits == 4 else b).reshape(rows, -1)


class QLinear:
    """MLX-affine quantized [rows, cols] (packed bytes, 16-bit scales/biases)."""

    def __init__(self, packed, scales, biases, bits, cols, sb="bf16", gs=64):
        self.w = dequantize_affine(packed_rows(packed, bits, scales.shape[0]), scales, biases, bits, cols, gs,
                                   sb).astype(F32)

    def __call__(self, x):
        return self.w @ np.asarray(x, F32)


class FullStepRef:
    """Decode step of a dense GQA decoder (config keys as the engine reads them).

    weights: name -> array, names without the model prefix:
      embed_tokens.{weight,scales,biases} (quantized) or embed_tokens.weight (fp16),
      layers.i.input_layernorm.weight, layers.i.post_attention_layernorm.weight,
      layers.i.self_attn.{q,k,v,o}_proj.{weight,scales,biases},
      layers.i.self_attn.{q,k}_norm.weight (optional),
      layers.i.mlp.{gate,up,down}_proj.{weight,scales,biases}, norm.weight,
      lm_head.{weight,scales,biases} (optional: tied to the embedding).
    Quantized weights: packed bytes (any integer view), scales/biases uint16
    bit patterns in `sb` ("bf16" or "f16"); norm weights fp32 values."""

    def __init__(self, cfg: dict, weights: dict, bits: int, sb: str = "bf16"):
        self.c = dict(cfg)
        c = self.c
        self.H, self.I, self.L = c["hidden_size"], c["intermediate_size"], c["num_hidden_layers"]
        self.nq, self.nkv = c["num_attention_heads"], c["num_key_value_heads"]
        self.hd = c.get("head_dim", self.H // self.nq)
        self.vocab = c["vocab_size"]
        self.eps = F32(c.get("rms_norm_eps", 1e-6))
        self.theta = F32(c.get("rope_theta", 10000.0))
        rd = int(self.hd * c.get("partial_rotary_factor", 1.0))
        self.rd = rd - rd % 2
        self.max_seq = c.get("max_cache_len", 4096)
        self.bits, self.sb, self.gs = bits, sb, c.get("group_size", 64)
        W = weights

        def ql(name, cols):
            return QLinear(W[name + ".weight"], W[name + ".scales"], W[name + ".biases"], bits, cols, sb, self.gs)

        if W["embed_tokens.weight"].dtype == np.float16:
            self.emb = W["embed_tokens.weight"].astype(F32)
            self.emb_q = None
        else:
            self.emb = None
            self.emb_q = (W["embed_tokens.weight"], W["embed_tokens.scales"], W["embed_tokens.biases"])
        self.lm = ql("lm_head", self.H) if "lm_head.weight" in W else ql("embed_tokens", self.H)
        self.norm = np.asarray(W["norm.weight"], F32)
        self.layers = []
        for l in range(self.L):
            p = f"layers.{l}."
            self.layers.append(dict(
                in_norm=np.asarray(W[p + "input_layernorm.weight"], F32),
                post_norm=np.asarray(W[p + "post_attention_layernorm.weight"], F32),
                q_norm=np.asarray(W[p + "self_attn.q_norm.weight"], F32) if p + "self_attn.q_norm.weight" in W else None,
                k_norm=np.asarray(W[p + "self_attn.k_norm.weight"], F32) if p + "self_attn.k_norm.weight" in W else None,
                q=ql(p + "self_attn.q_proj", self.H), k=ql(p + "self_attn.k_proj", self.H),
                v=ql(p + "self_attn.v_proj", self.H), o=ql(p + "self_attn.o_proj", self.nq * self.hd),
                gate=ql(p + "mlp.gate_proj", self.H), up=ql(p + "mlp.up_proj", self.H),
                down=ql(p + "mlp.down_proj", self.I)))
        self.reset()

    def reset(self):
        self.kc = np.zeros((self.L, self.nkv, self.max_seq, self.hd), F16)
        self.vc = np.zeros_like(self.kc)

    def embed(self, tok):
        if self.emb is not None:
            return h(self.emb[tok])
        w, s, b = self.emb_q
        row = dequantize_affine(packed_rows(w, self.bits, self.vocab)[tok:tok + 1],
                                s[tok:tok + 1], b[tok:tok + 1], self.bits, self.H, self.gs, self.sb)[0]
        return h(row)

    def rope(self, v, pos):
        hr = self.rd // 2
        i = np.arange(hr, dtype=F32)
        freq = F32(1.0) / np.power(self.theta, (F32(2.0) * i) / F32(self.rd), dtype=F32)
        ang = F32(pos) * freq
        c, s = np.cos(ang).astype(F32), np.sin(ang).astype(F32)
        out = v.copy()
        x0, x1 = v[..., :hr], v[..., hr:self.rd]
        out[..., :hr] = h(x0 * c - x1 * s)
        out[..., hr:self.rd] = h(x0 * s + x1 * c)
        return out

    def attention(self, l, q, pos):
        """gqa_attention_decode over positions [0, pos]."""
        G = self.nq // self.nkv
        out = np.zeros((self.nq, self.hd), F32)
        for hq in range(self.nq):
            kv = hq // G
            k = self.kc[l, kv, :pos + 1].astype(F32)
            v = self.vc[l, kv, :pos + 1].astype(F32)
            s = (k @ q[hq]) * (F32(1.0) / np.sqrt(F32(self.hd)))
            p = np.exp(s - s.max())
            out[hq] = h((p @ v) * (F32(1.0) / p.sum(dtype=F32)))
        return out

    def step(self, tok: int, pos: int) -> np.ndarray:
        x = self.embed(tok)
        for l, P in enumerate(self.layers):
            xn = h(rms(x, P["in_norm"], self.eps))
            qp = h(P["q"](xn))
            k = h(P["k"](xn)).reshape(self.nkv, self.hd)
            v = h(P["v"](xn)).reshape(self.nkv, self.hd)
            gate = None
            if qp.size == 2 * self.nq * self.hd:  # split_q_gate
                qg = qp.reshape(self.nq, 2, self.hd)
                q, gate = qg[:, 0].copy(), qg[:, 1].copy()
            else:
                q = qp.reshape(self.nq, self.hd)
            if P["q_norm"] is not None:
                q = np.stack([h(rms(q[i], P["q_norm"], self.eps)) for i in range(self.nq)])
            if P["k_norm"] is not None:
                k = np.stack([h(rms(k[i], P["k_norm"], self.eps)) for i in range(self.nkv)])
            q, k = self.rope(q, pos), self.rope(k, pos)
            self.kc[l, :, pos] = k.astype(F16)
            self.vc[l, :, pos] = v.astype(F16)
            a = self.attention(l, q, pos)
            if gate is not None:
                a = h(a * (F32(1.0) / (F32(1.0) + np.exp(-gate))))
            x = h(x + h(P["o"](a.reshape(-1))))
            xn = h(rms(x, P["post_norm"], self.eps))
            g, u = P["gate"](xn), P["up"](xn)
            act = h((g / (F32(1.0) + np.exp(-g))) * u)
            x = h(x + h(P["down"](act)))
        return self.lm(h(rms(x, self.norm, self.eps))).astype(F32)


def random_model(cfg: dict, bits: int = 4, sb: str = "bf16", seed: int = 0, std: float = 0.05, q_norm=True,
                 gate=False, tied=False, quant_embed=True):
    """Seeded random weights for a dense decoder, as name -> array.  Linears
    ~N(0, std) quantized MLX-affine (packed as uint32 rows); norms
    1 + N(0, 0.1) rounded to bf16 values (held as fp32), so they are exact
    in bf16 and fp16 alike."""
    from .oracle import bf16_bits_to_f32, f32_to_bf16_bits, quantize_affine
    rng = np.random.RandomState(seed)
    H, I, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    nq, nkv = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    hd = cfg.get("head_dim", H // nq)
    V = cfg["vocab_size"]
    W = {}

    def lin(name, rows, cols, scale=std):
        p, s, b = quantize_affine(rng.randn(rows, cols).astype(F32) * F32(scale), bits, 64, sb)
        W[name + ".weight"] = np.ascontiguousarray(p).view(np.uint8).reshape(rows, -1).view(np.uint32)
        W[name + ".scales"], W[name + ".biases"] = s, b

    def norm(name, n):
        W[name] = bf16_bits_to_f32(f32_to_bf16_bits((1.0 + 0.1 * rng.randn(n)).astype(F32)))

    if quant_embed:
        lin("embed_tokens", V, H, 1.0)
    else:
        W["embed_tokens.weight"] = rng.randn(V, H).astype(F16)
    for l in range(L):
        p = f"layers.{l}."
        norm(p + "input_layernorm.weight", H)
        norm(p + "post_attention_layernorm.weight", H)
        lin(p + "self_attn.q_proj", nq * hd * (2 if gate else 1), H)
        lin(p + "self_attn.k_proj", nkv * hd, H)
        lin(p + "self_attn.v_proj", nkv * hd, H)
        lin(p + "self_attn.o_proj", H, nq * hd)
        if q_norm:
            norm(p + "self_attn.q_norm.weight", hd)
            norm(p + "self_attn.k_norm.weight", hd)
        lin(p + "mlp.gate_proj", I, H)
        lin(p + "mlp.up_proj", I, H)
        lin(p + "mlp.down_proj", H, I)
    norm("norm.weight", H)
    if not tied:
        lin("lm_head", V, H)
    return W
