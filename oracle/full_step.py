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

GatedDeltaNet layers (full_forward_lg.m:1361-1508): conv1d_buffer_update
1282-1305 and depthwise_conv1d_silu 1055-1078, split_qkv 1314-1340,
rmsnorm_per_head_no_weight 951-1003 on q and k, scale_vector 1262-1272
(q * 1/kd, k * 1/sqrt(kd)), gated_delta_state_update 1108-1178,
rmsnorm_gated_kernel 1197-1260, out_proj.

MLP: the MoE block of kandiga/metal/moe_block.metal:134-584 (RMSNorm,
quantized router, softmax top-K, routed experts, shared expert with a sigmoid
gate, blend with the residual) through the C oracle; or, for a dense decoder,
half(silu(gate x) * (up x)) then down, the expert arithmetic of
kandiga/metal/kandiga_cpu_expert.m:355-401 on one dense matrix pair.

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


def layer_kinds(cfg: dict):
    """per layer: True for GatedDeltaNet (config "layer_types", else every
    layer but each full_attention_interval-th when linear heads are set)"""
    L = cfg["num_hidden_layers"]
    if "layer_types" in cfg:
        return [t == "linear_attention" for t in cfg["layer_types"]][:L]
    if cfg.get("linear_num_value_heads", 0) > 0:
        every = cfg.get("full_attention_interval", 4)
        return [every > 1 and (l + 1) % every != 0 for l in range(L)]
    return [False] * L


class FullStepRef:
    """Decode step of a GQA decoder, optionally with GatedDeltaNet layers and
    MoE blocks (config keys as the engine reads them).

    weights: name -> array, names without the model prefix:
      embed_tokens.{weight,scales,biases} (quantized) or embed_tokens.weight (fp16),
      layers.i.input_layernorm.weight, layers.i.post_attention_layernorm.weight,
      layers.i.self_attn.{q,k,v,o}_proj.{weight,scales,biases},
      layers.i.self_attn.{q,k}_norm.weight (optional),
      layers.i.mlp.{gate,up,down}_proj.{weight,scales,biases}, norm.weight,
      lm_head.{weight,scales,biases} (optional: tied to the embedding).
    Quantized weights: packed bytes (any integer view), scales/biases uint16
    bit patterns in `sb` ("bf16" or "f16"); norm weights fp32 values."""

    def __init__(self, cfg: dict, weights: dict, bits: int, sb: str = "bf16", moe=None):
        self.c = dict(cfg)
        c = self.c
        self.H, self.I, self.L = c["hidden_size"], c.get("intermediate_size", 0), c["num_hidden_layers"]
        self.nq, self.nkv = c["num_attention_heads"], c["num_key_value_heads"]
        self.hd = c.get("head_dim", self.H // self.nq)
        self.vocab = c["vocab_size"]
        self.eps = F32(c.get("rms_norm_eps", 1e-6))
        self.theta = F32(c.get("rope_theta", 10000.0))
        rd = int(self.hd * c.get("partial_rotary_factor", 1.0))
        self.rd = rd - rd % 2
        self.max_seq = c.get("max_cache_len", 4096)
        self.bits, self.sb, self.gs = bits, sb, c.get("group_size", 64)
        self.kinds = layer_kinds(c)
        self.nk, self.nv = c.get("linear_num_key_heads", 0), c.get("linear_num_value_heads", 0)
        self.kd, self.vd = c.get("linear_key_head_dim", 0), c.get("linear_value_head_dim", 0)
        self.ck = c.get("linear_conv_kernel_dim", 4)
        self.cdim = 2 * self.nk * self.kd + self.nv * self.vd
        self.moe = moe  # None or per layer dict(experts=ExpertLayer, router, sgate, shared, norm, top_k)
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
            P = dict(in_norm=np.asarray(W[p + "input_layernorm.weight"], F32), linear=self.kinds[l])
            if moe is None:
                P.update(post_norm=np.asarray(W[p + "post_attention_layernorm.weight"], F32),
                         gate=ql(p + "mlp.gate_proj", self.H), up=ql(p + "mlp.up_proj", self.H),
                         down=ql(p + "mlp.down_proj", self.I))
            if self.kinds[l]:
                a = p + "linear_attn."
                P.update(proj=[ql(a + n, self.H) for n in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a")],
                         out=ql(a + "out_proj", self.nv * self.vd),
                         conv_w=np.asarray(W[a + "conv1d.weight"], F32).reshape(self.cdim, self.ck),
                         a_log=np.asarray(W[a + "A_log"], F32), dt_bias=np.asarray(W[a + "dt_bias"], F32),
                         gnorm=np.asarray(W[a + "norm.weight"], F32))
            else:
                P.update(q_norm=np.asarray(W[p + "self_attn.q_norm.weight"], F32) if p + "self_attn.q_norm.weight" in W
                         else None,
                         k_norm=np.asarray(W[p + "self_attn.k_norm.weight"], F32) if p + "self_attn.k_norm.weight" in W
                         else None,
                         q=ql(p + "self_attn.q_proj", self.H), k=ql(p + "self_attn.k_proj", self.H),
                         v=ql(p + "self_attn.v_proj", self.H), o=ql(p + "self_attn.o_proj", self.nq * self.hd))
            self.layers.append(P)
        self.reset()

    def reset(self):
        self.kc = np.zeros((self.L, self.nkv, self.max_seq, self.hd), F16)
        self.vc = np.zeros_like(self.kc)
        self.conv = np.zeros((self.L, max(self.cdim, 1), self.ck), F16)
        self.state = np.zeros((self.L, max(self.nv, 1), max(self.vd, 1), max(self.kd, 1)), F32)

    def linear_attention(self, l, P, x):
        """GatedDeltaNet token mixer; returns the new hidden state."""
        xn = h(rms(x, P["in_norm"], self.eps))
        proj = np.concatenate([h(m(xn)) for m in P["proj"]])
        cd, vt, nv = self.cdim, self.nv * self.vd, self.nv
        qkv, z, b, a = proj[:cd], proj[cd:cd + vt], proj[cd + vt:cd + vt + nv], proj[cd + vt + nv:cd + vt + 2 * nv]
        st = self.conv[l]
        st[:, :-1] = st[:, 1:]
        st[:, -1] = qkv.astype(F16)
        acc = np.zeros(cd, F32)
        for k in range(self.ck):
            acc = acc + st[:, k].astype(F32) * P["conv_w"][:, k]
        conv = h(acc / (F32(1.0) + np.exp(-acc)))
        nk, kd, vd = self.nk, self.kd, self.vd
        q = conv[:nk * kd].reshape(nk, kd)
        k = conv[nk * kd:2 * nk * kd].reshape(nk, kd)
        v = conv[2 * nk * kd:].reshape(nv, vd)
        inv = F32(1.0) / np.sqrt(F32(kd))
        ones = np.ones(kd, F32)
        q = np.stack([h(h(rms(q[i], ones, self.eps)) * (inv * inv)) for i in range(nk)])
        k = np.stack([h(h(rms(k[i], ones, self.eps)) * inv) for i in range(nk)])
        o = np.zeros((nv, vd), F32)
        for hv in range(nv):
            hk = hv // (nv // nk)
            sp = np.log(F32(1.0) + np.exp(a[hv] + P["dt_bias"][hv]))
            g = np.exp(-np.exp(P["a_log"][hv]) * sp).astype(F32)
            beta = F32(1.0) / (F32(1.0) + np.exp(-b[hv]))
            S = self.state[l, hv] * g
            kvm = S @ k[hk]
            delta = (v[hv] - kvm) * beta
            S = S + np.outer(delta, k[hk]).astype(F32)
            self.state[l, hv] = S
            o[hv] = h(S @ q[hk])
        out = np.zeros((nv, vd), F32)
        for hv in range(nv):
            normed = rms(o[hv], P["gnorm"], self.eps)
            zz = z[hv * vd:(hv + 1) * vd]
            out[hv] = h((zz / (F32(1.0) + np.exp(-zz))) * normed)
        return h(x + h(P["out"](out.reshape(-1))))

    def moe_block(self, l, x):
        """out = x + MoE(rmsnorm(x)) (moe_block.metal:134-584), via the C oracle"""
        from . import oracle as O
        m = self.moe[l]
        xn = O.rms_norm(x, m["norm"], self.eps).astype(F32)
        rpk, rs, rb = m["router"]
        logits = O.matvec(4, rpk, rs, rb, xn, "bf16")
        idx, w = O.router_topk(logits[None], m["top_k"])
        y = m["experts"].moe(xn[None], idx)
        gpk, gs, gb = m["sgate"]
        gate = O.shared_gate(xn[None], gpk, gs, gb, 4, "bf16")
        shared = m["shared"].moe(xn[None], np.zeros((1, 1), np.int32))[0, 0].astype(F16).astype(F32)
        return h(O.combine(y, w, x[None].astype(F32), shared[None], gate)[0])

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

    def attention_layer(self, l, P, x, pos):
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
        return h(x + h(P["o"](a.reshape(-1))))

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
            if P["linear"]:
                x = self.linear_attention(l, P, x)
            else:
                x = self.attention_layer(l, P, x, pos)
            if self.moe is not None:
                x = self.moe_block(l, x)
            else:
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
    H, I, L = cfg["hidden_size"], cfg.get("intermediate_size", 0), cfg["num_hidden_layers"]
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

    def bf(x):
        return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x, F32)))

    kinds = layer_kinds(cfg)
    nk, nv = cfg.get("linear_num_key_heads", 0), cfg.get("linear_num_value_heads", 0)
    kd, vd = cfg.get("linear_key_head_dim", 0), cfg.get("linear_value_head_dim", 0)
    ck = cfg.get("linear_conv_kernel_dim", 4)
    cdim = 2 * nk * kd + nv * vd
    dense_mlp = cfg.get("num_experts", 0) == 0
    if quant_embed:
        lin("embed_tokens", V, H, 1.0)
    else:
        W["embed_tokens.weight"] = rng.randn(V, H).astype(F16)
    for l in range(L):
        p = f"layers.{l}."
        norm(p + "input_layernorm.weight", H)
        if dense_mlp:
            norm(p + "post_attention_layernorm.weight", H)
        if kinds[l]:
            a = p + "linear_attn."
            lin(a + "in_proj_qkv", cdim, H)
            lin(a + "in_proj_z", nv * vd, H)
            lin(a + "in_proj_b", nv, H, 0.5)
            lin(a + "in_proj_a", nv, H, 0.5)
            lin(a + "out_proj", H, nv * vd)
            W[a + "conv1d.weight"] = bf(rng.randn(cdim, ck, 1) * 0.4)
            W[a + "A_log"] = bf(np.log(rng.uniform(1.0, 16.0, nv)))
            W[a + "dt_bias"] = bf(rng.randn(nv) * 0.5)
            norm(a + "norm.weight", vd)
        else:
            lin(p + "self_attn.q_proj", nq * hd * (2 if gate else 1), H)
            lin(p + "self_attn.k_proj", nkv * hd, H)
            lin(p + "self_attn.v_proj", nkv * hd, H)
            lin(p + "self_attn.o_proj", H, nq * hd)
            if q_norm:
                norm(p + "self_attn.q_norm.weight", hd)
                norm(p + "self_attn.k_norm.weight", hd)
        if dense_mlp:
            lin(p + "mlp.gate_proj", I, H)
            lin(p + "mlp.up_proj", I, H)
            lin(p + "mlp.down_proj", H, I)
    norm("norm.weight", H)
    if not tied:
        lin("lm_head", V, H)
    return W


def random_moe(cfg: dict, seed: int = 0, expert_bits: int = 3):
    """Seeded MoE blocks for every layer: routed experts (ExpertLayer, written
    to BKEX files by the caller), a 4-bit router, a 4-bit shared-expert gate row,
    a 4-bit shared expert and the post-attention norm.  Returns (moe list for
    FullStepRef, name -> array of the block tensors for the engine)."""
    from .oracle import ExpertLayer, bf16_bits_to_f32, f32_to_bf16_bits, quantize_affine
    rng = np.random.RandomState(seed + 1000)
    H, L, E = cfg["hidden_size"], cfg["num_hidden_layers"], cfg["num_experts"]
    I, IS, K = cfg["moe_intermediate_size"], cfg["shared_expert_intermediate_size"], cfg["num_experts_per_tok"]
    moe, W = [], {}

    def u32(packed, rows):
        return np.ascontiguousarray(packed).view(np.uint8).reshape(rows, -1).view(np.uint32)

    for l in range(L):
        p = f"layers.{l}."
        normv = bf16_bits_to_f32(f32_to_bf16_bits((1.0 + 0.1 * rng.randn(H)).astype(F32)))
        router = quantize_affine((rng.randn(E, H) * 0.05).astype(F32), 4, 64, "bf16")
        sgate = quantize_affine((rng.randn(1, H) * 0.05).astype(F32), 4, 64, "bf16")
        shared = ExpertLayer.random(4, H, IS, 1, seed=seed + 200 + l, sb_dtype="bf16")
        experts = ExpertLayer.random(expert_bits, H, I, E, seed=seed + 300 + l, sb_dtype="bf16")
        moe.append(dict(norm=normv, router=router, sgate=sgate, shared=shared, experts=experts, top_k=K))
        W[p + "post_attention_layernorm.weight"] = normv
        for name, (pk, sc, bi), rows in (("mlp.gate", router, E), ("mlp.shared_expert_gate", sgate, 1)):
            W[p + name + ".weight"], W[p + name + ".scales"], W[p + name + ".biases"] = u32(pk, rows), sc, bi
        for name, m, rows in (("gate_proj", 0, IS), ("up_proj", 1, IS), ("down_proj", 2, H)):
            q = p + "mlp.shared_expert." + name
            W[q + ".weight"] = u32(shared.w[m][0], rows)
            W[q + ".scales"], W[q + ".biases"] = shared.s[m][0], shared.b[m][0]
    return moe, W
