"""Whole-model decode step (bakan_full_*) against the numpy restatement of
the reference's step (oracle/full_step.py).

Tolerance: logits within 5e-3 relative L2 of the oracle at every step, and
the same arg-max.  Both sides round every inter-kernel buffer to fp16 as the
reference does; the remaining differences are fp32 summation order and the
fp16 rounding of the projections' inputs inside the GEMV.  Replays of the
same graphs are bit-identical (prefill vs forward, reset_cache)."""
import numpy as np
import pytest

from oracle.full_step import FullStepRef, random_model

pytestmark = pytest.mark.gpu
TOL = 5e-3

BASE = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
            num_key_value_heads=2, head_dim=64, vocab_size=512, rms_norm_eps=1e-6, rope_theta=10000.0,
            partial_rotary_factor=0.5, max_cache_len=96)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def load(e, W, sb):
    """norm weights go in as bf16 bit patterns (their values are bf16-exact),
    scales/biases as `sb` bit patterns, packed codes and fp16 as they are"""
    from oracle.oracle import f32_to_bf16_bits
    for k, v in W.items():
        if v.dtype == np.float32 and v.ndim == 1:
            assert e.set_weight(k, f32_to_bf16_bits(v), sb="bf16") == 0
        else:
            assert e.set_weight(k, v, sb=sb) == 0


def engine(cfg, W, sb="bf16"):
    from kandiga_b200 import _native as N
    from kandiga_b200.full import FullForwardEngine
    e = FullForwardEngine("", cfg["num_hidden_layers"], config=cfg)
    load(e, W, sb)
    assert N.load().bakan_full_build(e._engine) == 0
    return e


CASES = {
    "4bit_bf16_qknorm": dict(bits=4, sb="bf16", q_norm=True, gate=False, tied=False),
    "3bit_f16_gate_tied": dict(bits=3, sb="f16", q_norm=False, gate=True, tied=True),
    "4bit_hd128_g4_fp16emb": dict(bits=4, sb="bf16", q_norm=True, gate=True, tied=False, quant_embed=False,
                                  cfg=dict(head_dim=128, num_attention_heads=8, num_key_value_heads=2,
                                           partial_rotary_factor=0.25)),
    "3bit_hd256_g8": dict(bits=3, sb="bf16", q_norm=True, gate=True, tied=False,
                          cfg=dict(hidden_size=512, head_dim=256, num_attention_heads=8, num_key_value_heads=1,
                                   partial_rotary_factor=1.0, rope_theta=1e6)),
}


@pytest.mark.parametrize("case", list(CASES))
def test_decode_steps_match_oracle(gpu, case):
    spec = dict(CASES[case])
    cfg = dict(BASE, **spec.pop("cfg", {}))
    bits, sb = spec.pop("bits"), spec.pop("sb")
    W = random_model(cfg, bits=bits, sb=sb, seed=3, **spec)
    ref = FullStepRef(cfg, W, bits, sb)
    e = engine(cfg, W, sb)
    rng = np.random.RandomState(5)
    toks = rng.randint(0, cfg["vocab_size"], 40)  # crosses one 32-token attention chunk
    worst = 0.0
    for pos, t in enumerate(toks):
        got = e.forward(int(t), pos)
        want = ref.step(int(t), pos)
        err = rel_l2(got, want)
        worst = max(worst, err)
        assert err < TOL, (case, pos, err)
        assert int(np.argmax(got)) == int(np.argmax(want)), (case, pos)
    assert e.position == len(toks)
    print(case, "worst rel L2", worst)


def test_prefill_reset_and_replay_bit_identical(gpu):
    cfg = dict(BASE)
    W = random_model(cfg, bits=4, seed=7)
    e = engine(cfg, W)
    ids = [5, 17, 300, 2, 99, 411]
    seq = [e.forward(t, p) for p, t in enumerate(ids)]
    e.reset_cache()
    pre = e.prefill(ids)
    assert np.array_equal(pre, seq[-1])
    e.reset_cache()
    assert np.array_equal(e.forward(ids[0], 0), seq[0])


def test_set_kv_cache_then_decode(gpu):
    """a cache handed over from another prefill (bakan_full_set_kv_cache), then decode"""
    cfg = dict(BASE)
    W = random_model(cfg, bits=4, seed=11)
    ref = FullStepRef(cfg, W, 4, "bf16")
    e = engine(cfg, W)
    rng = np.random.RandomState(2)
    S = 50
    for l in range(cfg["num_hidden_layers"]):
        k = rng.randn(cfg["num_key_value_heads"], S, cfg["head_dim"]).astype(np.float16)
        v = rng.randn(cfg["num_key_value_heads"], S, cfg["head_dim"]).astype(np.float16)
        assert e.set_kv_cache(l, k, v) == 0
        ref.kc[l, :, :S] = k
        ref.vc[l, :, :S] = v
    assert e.set_position(S) == 0
    for i in range(3):
        got = e.forward(10 + i, S + i)
        want = ref.step(10 + i, S + i)
        assert rel_l2(got, want) < TOL


def test_configs2_layer_shape_at_kv_2048(gpu):
    """The benched dense decoder's per-layer shape: H 2560, 16 q / 4 kv heads x
    256 with q/k norms, SwiGLU 9216, 3-bit with fp16 scales, rope_theta 1e6,
    the KV cache pre-filled to 2048 tokens ~N(0,1) through set_kv_cache.  Two
    layers and a 4096-token vocabulary keep the numpy oracle small; the
    attention runs the same context split (one chunk per SM) and merge as the
    36-layer bench (kandiga/metal/full_forward_lg.m:1078-1354,
    kandiga/metal/attention.metal:752-849)."""
    cfg = dict(hidden_size=2560, intermediate_size=9216, num_hidden_layers=2, num_attention_heads=16,
               num_key_value_heads=4, head_dim=256, vocab_size=4096, rms_norm_eps=1e-6, rope_theta=1e6,
               max_cache_len=2048 + 8)
    W = random_model(cfg, bits=3, sb="f16", seed=21, std=0.02)
    ref = FullStepRef(cfg, W, 3, "f16")
    e = engine(cfg, W, "f16")
    rng = np.random.RandomState(4)
    S = 2048
    for l in range(cfg["num_hidden_layers"]):
        k = rng.randn(4, S, 256).astype(np.float16)
        v = rng.randn(4, S, 256).astype(np.float16)
        assert e.set_kv_cache(l, k, v) == 0
        ref.kc[l, :, :S], ref.vc[l, :, :S] = k, v
    assert e.set_position(S) == 0
    worst = 0.0
    for i in range(4):
        got, want = e.forward(7 + i, S + i), ref.step(7 + i, S + i)
        err = rel_l2(got, want)
        worst = max(worst, err)
        assert err < TOL, (i, err)
        assert int(np.argmax(got)) == int(np.argmax(want))
    print("configs[2] layer shape worst rel L2", worst)


def test_errors_are_reported(gpu):
    from kandiga_b200 import _native as N
    from kandiga_b200.full import FullForwardEngine
    cfg = dict(BASE)
    W = random_model(cfg, bits=4, seed=1)
    e = engine(cfg, W)
    with pytest.raises(RuntimeError):
        e.forward(cfg["vocab_size"], 0)          # token outside the vocabulary
    with pytest.raises(RuntimeError):
        e.forward(1, cfg["max_cache_len"])        # position past the cache
    assert e.set_weight("norm.weight", np.ones(cfg["hidden_size"], np.float32)) == -1  # after build
    assert np.all(np.isfinite(e.forward(1, 0)))   # the engine still works
    # a missing tensor fails the build
    e2 = FullForwardEngine("", cfg["num_hidden_layers"], config=cfg)
    load(e2, {k: v for k, v in W.items() if "layers.1.mlp.down_proj" not in k}, "bf16")
    assert N.load().bakan_full_build(e2._engine) == -1
    # unsupported shapes are refused at init
    with pytest.raises(RuntimeError):
        FullForwardEngine("", 2, config=dict(cfg, head_dim=96))


HYBRID_TOL_STEP = 1e-2     # any single step
HYBRID_TOL_MEDIAN = 2e-3   # median over the 24 steps
HYBRID = dict(hidden_size=256, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
              vocab_size=512, rms_norm_eps=1e-6, rope_theta=10000.0, partial_rotary_factor=0.25, max_cache_len=64,
              linear_num_key_heads=2, linear_num_value_heads=8, linear_key_head_dim=64, linear_value_head_dim=64,
              linear_conv_kernel_dim=4, full_attention_interval=4, num_experts=16, num_experts_per_tok=4,
              moe_intermediate_size=256, shared_expert_intermediate_size=256)


@pytest.fixture(scope="module", params=[3, 4])
def hybrid(tmp_path_factory, gpu, request):
    """the hybrid shape in miniature: 3 GatedDeltaNet layers and 1 attention
    layer (with output gate), MoE blocks with a shared expert; BKEX expert
    files and config.json in a directory, as bakan_full_init reads them.
    Routed experts 3-bit: the 4-bit shared expert keeps its own table; 4-bit:
    it joins the routed table (the merged MoE block)."""
    import json
    from oracle.full_step import random_moe
    from tests.test_bakan_gpu import write_bkex
    d = tmp_path_factory.mktemp("hybrid")
    W = random_model(HYBRID, bits=4, seed=21, gate=True)
    moe, WM = random_moe(HYBRID, seed=21, expert_bits=request.param)
    write_bkex(str(d), [m["experts"] for m in moe])
    (d / "config.json").write_text(json.dumps(HYBRID))
    return str(d), W, moe, WM


def hybrid_engine(d, W, WM):
    from kandiga_b200 import _native as N
    from kandiga_b200.full import FullForwardEngine
    e = FullForwardEngine(d, HYBRID["num_hidden_layers"])   # config.json from the directory
    load(e, W, "bf16")
    load(e, WM, "bf16")
    assert N.load().bakan_full_build(e._engine) == 0
    return e


def test_hybrid_gated_delta_net_and_moe_match_oracle(hybrid):
    d, W, moe, WM = hybrid
    ref = FullStepRef(HYBRID, W, 4, "bf16", moe=moe)
    e = hybrid_engine(d, W, WM)
    rng = np.random.RandomState(8)
    errs = []
    for pos, t in enumerate(rng.randint(0, HYBRID["vocab_size"], 24)):
        got = e.forward(int(t), pos)
        want = ref.step(int(t), pos)
        err = rel_l2(got, want)
        errs.append(err)
        assert err < HYBRID_TOL_STEP, (pos, err)
    # A random recurrent model amplifies rounding differences at single steps
    # (isolated spikes of 3.6e-3 to 7.2e-3 between steps at ~1e-3, with no
    # routing tie and no carry-over into later steps); drift would raise the
    # median.
    assert np.median(errs) < HYBRID_TOL_MEDIAN, errs
    print("hybrid worst rel L2", max(errs), "median", np.median(errs))


def test_hybrid_state_handover(hybrid):
    """bakan_full_set_linear_state / set_conv_state / set_kv_cache / set_position:
    a state handed over from elsewhere, then decode continues from it"""
    d, W, moe, WM = hybrid
    ref = FullStepRef(HYBRID, W, 4, "bf16", moe=moe)
    e = hybrid_engine(d, W, WM)
    rng = np.random.RandomState(3)
    S = 20
    lin = [l for l in range(HYBRID["num_hidden_layers"]) if ref.kinds[l]]
    att = [l for l in range(HYBRID["num_hidden_layers"]) if not ref.kinds[l]]
    for i, l in enumerate(lin):
        st = (rng.randn(*ref.state[l].shape) * 0.1).astype(np.float32)
        cv = (rng.randn(*ref.conv[l].shape) * 0.5).astype(np.float16)
        assert e.set_linear_state(i, st) == 0 and e.set_conv_state(i, cv) == 0
        ref.state[l], ref.conv[l] = st, cv
    for i, l in enumerate(att):
        k = rng.randn(HYBRID["num_key_value_heads"], S, HYBRID["head_dim"]).astype(np.float16)
        v = rng.randn(HYBRID["num_key_value_heads"], S, HYBRID["head_dim"]).astype(np.float16)
        assert e.set_kv_cache(i, k, v) == 0
        ref.kc[l, :, :S], ref.vc[l, :, :S] = k, v
    assert e.set_position(S) == 0
    for i in range(3):
        assert rel_l2(e.forward(7 + i, S + i), ref.step(7 + i, S + i)) < TOL
    assert e.set_linear_state(len(lin), np.zeros_like(ref.state[0])) == -1   # no such linear layer
    assert e.set_conv_state(0, np.zeros((3, 3), np.float16)) == -1           # wrong size
