"""CPU checks of the whole-decode-step oracle (oracle/full_step.py): the layer
layout rule the reference uses (kandiga/metal/full_forward_lg.m:1137: every
fourth layer is full attention), the generated weights' shapes, the oracle's
attention against softmax attention in float64, its linear-attention state
bookkeeping, and determinism."""
import numpy as np

from oracle.full_step import FullStepRef, layer_kinds, random_model, random_moe

HYB = dict(hidden_size=128, num_hidden_layers=4, num_attention_heads=2, num_key_value_heads=1, head_dim=64,
           vocab_size=64, rms_norm_eps=1e-6, rope_theta=10000.0, partial_rotary_factor=0.5, max_cache_len=16,
           linear_num_key_heads=1, linear_num_value_heads=2, linear_key_head_dim=64, linear_value_head_dim=64,
           linear_conv_kernel_dim=4, full_attention_interval=4, intermediate_size=128)


def test_layer_layout_rule():
    assert layer_kinds(dict(num_hidden_layers=8, linear_num_value_heads=4)) == [True, True, True, False] * 2
    assert layer_kinds(dict(num_hidden_layers=3)) == [False] * 3
    kinds = ["linear_attention", "full_attention", "linear_attention"]
    assert layer_kinds(dict(num_hidden_layers=3, layer_types=kinds)) == [True, False, True]


def test_generated_shapes():
    W = random_model(HYB, bits=4, seed=1, gate=True)
    cdim = 2 * 1 * 64 + 2 * 64
    assert W["layers.0.linear_attn.in_proj_qkv.scales"].shape == (cdim, 2)
    assert W["layers.0.linear_attn.conv1d.weight"].shape == (cdim, 4, 1)
    assert W["layers.3.self_attn.q_proj.scales"].shape == (2 * 2 * 64, 2)   # q and gate per head
    assert "layers.3.linear_attn.A_log" not in W and "layers.0.self_attn.q_proj.weight" not in W
    cfg = dict(HYB, num_experts=16, num_experts_per_tok=2, moe_intermediate_size=128,
               shared_expert_intermediate_size=128)
    moe, WM = random_moe(cfg, seed=1)
    assert len(moe) == 4 and WM["layers.0.mlp.gate.scales"].shape == (16, 2)
    assert "layers.0.mlp.gate_proj.weight" not in random_model(cfg, bits=4, seed=1)


def test_oracle_linear_attention_updates_state_and_ring():
    """one GatedDeltaNet step from a random state: the fp32 state moves and stays
    finite, and the conv window shifts the new projection in at its last tap"""
    W = random_model(HYB, bits=4, seed=2)
    ref = FullStepRef(HYB, W, 4, "bf16")
    rng = np.random.RandomState(0)
    ref.state[0] = (rng.randn(*ref.state[0].shape) * 0.1).astype(np.float32)
    S0 = ref.state[0].copy()
    x = np.asarray(rng.randn(HYB["hidden_size"]).astype(np.float16), np.float32)
    ref.linear_attention(0, ref.layers[0], x)
    assert np.all(np.isfinite(ref.state[0])) and not np.allclose(ref.state[0], S0)
    assert np.all(ref.conv[0][:, :-1] == 0) and np.any(ref.conv[0][:, -1] != 0)  # ring buffer shifted in


def test_oracle_attention_is_softmax_attention():
    W = random_model(dict(HYB, linear_num_value_heads=0), bits=4, seed=3)
    cfg = dict(HYB, linear_num_value_heads=0)
    ref = FullStepRef(cfg, W, 4, "bf16")
    rng = np.random.RandomState(1)
    pos = 9
    ref.kc[0, :, :pos + 1] = rng.randn(1, pos + 1, 64).astype(np.float16)
    ref.vc[0, :, :pos + 1] = rng.randn(1, pos + 1, 64).astype(np.float16)
    q = rng.randn(2, 64).astype(np.float16).astype(np.float32)
    out = ref.attention(0, q, pos)
    k = ref.kc[0, 0, :pos + 1].astype(np.float64)
    v = ref.vc[0, 0, :pos + 1].astype(np.float64)
    for h in range(2):
        s = k @ q[h] / np.sqrt(64.0)
        p = np.exp(s - s.max())
        want = (p / p.sum()) @ v
        np.testing.assert_allclose(out[h], want, rtol=2e-3, atol=2e-3)


def test_oracle_steps_are_deterministic():
    W = random_model(HYB, bits=4, seed=4, gate=True)
    a, b = FullStepRef(HYB, W, 4, "bf16"), FullStepRef(HYB, W, 4, "bf16")
    for pos, t in enumerate([3, 9, 1]):
        assert np.array_equal(a.step(t, pos), b.step(t, pos))
