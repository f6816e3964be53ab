"""Pin the CPU oracle (oracle/gncx_oracle.c) to the reference.

1. Against the committed golden vectors (generated from the reference's own
   compiled kernels by tests/golden/make_golden.py): bit-exact.
2. Where the reference library is built here (oracle/_ref): bit-exact against
   the strict-IEEE build on fresh seeded inputs of the configuration shapes,
   and within 1e-6 relative of the as-shipped (FMA) build.
"""
import numpy as np
import pytest

from conftest import golden
from gncx_b200 import synth
from gncx_b200.core import BF16, Q4_0, Q4_K, Q6_K, Q8_0

TYPES = [Q4_0, Q8_0, Q4_K, Q6_K, BF16]


@pytest.mark.parametrize("t", TYPES)
def test_gemv_golden(oracle, t):
    g = golden(f"gemv_{t}.npz")
    rows = g["y_strict"].size
    assert np.array_equal(oracle.matvec(g["w"], t, g["x"], rows), g["y_strict"])
    assert np.array_equal(oracle.matbatch(g["w"], t, g["xb"], rows), g["yb_strict"])
    y = oracle.matvec(g["w"], t, g["x"], rows)
    assert np.max(np.abs(y - g["y_native"])) <= 1e-6 * np.max(np.abs(g["y_native"]))


def test_lm_head_golden(oracle):
    g = golden("lm_head.npz")
    assert np.array_equal(oracle.lm_head(g["w"], Q6_K, g["h"], 100, 30.0), g["y_strict"])
    assert np.array_equal(oracle.lm_head(g["w"], Q6_K, g["h"], 100, 0.0), g["y_nocap"])


def test_norm_golden(oracle):
    g = golden("norm.npz")
    assert np.array_equal(oracle.rmsnorm(g["x"], g["w"], float(g["eps"])), g["y_strict"])
    assert np.array_equal(oracle.rmsnorm_heads(g["v"], g["wh"], 8, 64, 1e-6), g["heads_strict"])
    assert np.array_equal(oracle.rmsnorm_heads(g["v"], None, 8, 64, 1e-6), g["heads_nw_strict"])


def test_rope_golden(oracle):
    g = golden("rope.npz")
    for i, p in enumerate(g["pos"]):
        q, k = oracle.rope(g["q"], g["k"], 8, 2, 64, int(p), 1e6)
        assert np.array_equal(q, g["q_strict"][i]) and np.array_equal(k, g["k_strict"][i])
        qf, _ = oracle.rope(g["q"], None, 8, 2, 64, int(p), 1e4, g["ff"])
        assert np.array_equal(qf, g["qff_strict"][i])


def test_attention_golden(oracle):
    g = golden("attention.npz")
    out, kc, vc = oracle.attention(g["q"], g["k"], g["v"], g["kc"], g["vc"], 36, 8, 2, 64, 0.125, 0, 1)
    assert np.array_equal(out, g["out_strict"])
    assert np.array_equal(kc, g["kc_after"]) and np.array_equal(vc, g["vc_after"])
    out16, _, _ = oracle.attention(g["q"], g["k"], g["v"], g["kc"], g["vc"], 36, 8, 2, 64, 0.125, 16, 1)
    assert np.array_equal(out16, g["out_window16_strict"])
    assert np.max(np.abs(out - g["out_native"])) <= 1e-6 * np.max(np.abs(g["out_native"]))


def test_glu_golden(oracle):
    g = golden("glu.npz")
    assert np.array_equal(oracle.glu(g["g"], g["u"]), g["swiglu_strict"])
    assert np.array_equal(oracle.glu(g["g"], g["u"], gelu=True), g["geglu_strict"])


def test_embed_golden(oracle):
    g = golden("embed.npz")
    for t in (Q8_0, Q6_K, BF16):
        got = np.stack([oracle.embed(g[f"w_{t}"], t, r, 512, s) for r in (0, 3, 9) for s in (1.0, 22.627417)])
        assert np.array_equal(got, g[f"rows_{t}"])


def test_dequant_matches_embedding_fetch(oracle):
    """Q8_0/Q6_K/BF16 dequant == the reference's row fetch at scale 1 (:693-780)."""
    g = golden("embed.npz")
    for t in (Q8_0, Q6_K, BF16):
        w = g[f"w_{t}"]
        for i, r in enumerate((0, 3, 9)):
            assert np.array_equal(oracle.dequant_row(w[r], t, 512), g[f"rows_{t}"][2 * i])


def test_dequant_q4_consistent_with_matvec(oracle):
    """Q4_0/Q4_K have no reference dequant routine; a one-hot activation
    (act scale exactly 1/127*amax) recovers each weight through the matvec
    to fp32 rounding (a few ulps of the row's largest weight)."""
    for t in (Q4_0, Q4_K):
        w = synth.random_weights(t, 8, 256, seed=5)
        deq = np.stack([oracle.dequant_row(w[r], t, 256) for r in range(8)])
        for col in (0, 17, 31, 32, 200, 255):
            x = np.zeros(256, np.float32)
            x[col] = 127.0
            y = oracle.matvec(w, t, x, 8)
            ref = deq[:, col] * 127.0
            assert np.max(np.abs(y - ref)) <= 1e-6 * np.max(np.abs(deq)) * 127.0


def test_sample_greedy_semantics(oracle):
    """lua/gncx_streamer.lua:1229-1273: doubles, strict >, lowest index on ties,
    penalty on the last 65 tokens, v/p for positive, v*p otherwise."""
    logits = np.array([1.0, 3.0, 3.0, -1.0, 2.9], np.float32)
    assert oracle.sample_greedy(logits, [], 1.15) == 1                 # tie -> lowest index
    assert oracle.sample_greedy(logits, [1], 1.15) == 2                # 3/1.15 < 3
    assert oracle.sample_greedy(logits, [1, 2], 1.15) == 4             # 2.9 wins
    assert oracle.sample_greedy(np.full(4, -2e30, np.float32), [], 1.15) == 0  # nothing beats -1e30
    neg = np.array([-5.0, -1.0, -1.05], np.float32)
    assert oracle.sample_greedy(neg, [1], 1.10) == 2                   # -1*1.1 < -1.05
    # only the last 65 recent tokens are penalized
    lg = np.zeros(100, np.float32)
    lg[7] = 1.0
    lg[8] = 0.95
    recent = [7] + [50] * 65
    assert oracle.sample_greedy(lg, recent, 1.15) == 7
    assert oracle.sample_greedy(lg, recent[1:] + [7], 1.15) == 8


@pytest.mark.parametrize("t", [Q4_0, Q8_0, Q4_K, Q6_K])
@pytest.mark.parametrize("shape", [(256, 4096), (64, 12288)])
def test_oracle_vs_reference_configs(oracle, ref_strict, ref_native, t, shape):
    out_dim, in_dim = shape
    w = synth.random_weights(t, out_dim, in_dim, seed=11)
    x = synth.random_activations(in_dim, seed=12)
    a = oracle.matvec(w, t, x, out_dim)
    assert np.array_equal(a, ref_strict.matvec(w, t, x, out_dim))
    n = ref_native.matvec(w, t, x, out_dim)
    assert np.max(np.abs(a - n)) <= 1e-6 * np.max(np.abs(n))
    xb = synth.random_activations(in_dim, seed=13, rows=4)
    assert np.array_equal(oracle.matbatch(w, t, xb, out_dim), ref_strict.matbatch(w, t, xb, out_dim))


def test_oracle_vs_reference_attention_ctx(oracle, ref_strict):
    L = 700
    kc = synth.random_activations(L * 8 * 128, seed=31)
    vc = synth.random_activations(L * 8 * 128, seed=32)
    q = synth.random_activations(32 * 128, seed=33)
    for win in (0, 128):
        a = oracle.attention(q, None, None, kc, vc, L - 1, 32, 8, 128, 1 / np.sqrt(128), win, 0)
        b = ref_strict.attention(q, None, None, kc, vc, L - 1, 32, 8, 128, 1 / np.sqrt(128), win, 0)
        assert np.array_equal(a[0], b[0])
