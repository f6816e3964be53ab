"""Whole-model parity of the B200 engine against the reference.

The oracle is oracle/gncx_oracle_model.c (the reference orchestrator's
forward_token / prefill / sample / generate, restated because LuaJIT is not
available) driving the reference's own compiled kernels (oracle/_ref) when
present, else the C restatement pinned to them.  Checks:
  * greedy token streams identical (north star: >= 64 steps);
  * prefill and decode logits within 1e-3 relative of the reference
    (they agree far closer: only exp() and the softmax sum order differ);
  * logits finite and the top-1/top-2 gap not degenerate.
Random-init Q4_K weights (the benchmark distribution) carry a positive row
mean that drives greedy decoding to a repeated token after a few steps, so
the small symmetric-format models (Q6_K, Q8_0) are there to make the token
stream check a strong one.
"""
import numpy as np
import pytest

from gncx_b200 import gguf
from gncx_b200.core import Q4_K, Q6_K, Q8_0

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TINY = dict(n_layers=4, dim=256, n_heads=4, n_kv=2, head_dim=64, ffn=512, vocab=4000, eps=1e-6, rope_base=1e6)
LOGIT_TOL = 1e-3


def rel(a, b):
    return float(np.max(np.abs(a - b)) / max(1e-30, np.max(np.abs(b))))


@pytest.fixture(scope="module")
def oracle_model_cls():
    from oracle.oracle import OracleModel
    return OracleModel


def _check_logits(lg):
    assert np.all(np.isfinite(lg))
    s = np.sort(lg)
    assert s[-1] - s[-2] > 1e-4 * np.abs(s[-1])  # not a degenerate tie


@pytest.mark.parametrize("wtype", [Q4_K, Q6_K, Q8_0])
def test_tiny_model_stream(tmp_path, oracle_model_cls, wtype):
    """Exact-softmax mode: the token stream is identical to the reference's."""
    from gncx_b200.streamer import GNCXStreamer
    path = gguf.write_random_model(tmp_path / "tiny.gguf", TINY, seed=3, wtype=wtype)
    rng = np.random.default_rng(wtype)
    prompt = rng.integers(0, TINY["vocab"], 37).tolist()
    ref = oracle_model_cls(path, 160)
    with GNCXStreamer(path, max_seq_len=160, exact_attention=True) as eng:
        lg = eng.prefill(prompt)
        lr = ref.prefill(prompt)
        _check_logits(lr)
        assert rel(lg, lr) <= LOGIT_TOL
        # decode logits, step by step, through forward_token
        toks_ref, toks = [], []
        all_ids = list(prompt)
        for step in range(8):
            t_ref = ref_sample(lr, all_ids)
            t = eng.sample(all_ids, 1.15)
            assert t == t_ref, step
            all_ids.append(t)
            lr = ref.forward_token(t, len(all_ids) - 1)
            lg = eng.forward_token(t, len(all_ids) - 1)
            assert rel(lg, lr) <= LOGIT_TOL, step
        # the device-driven loop
        got = eng.generate_ids(prompt, 96, 1.15, eos_id=-1)
    want = ref.generate(prompt, 96, 1.15, -1)
    ref.close()
    assert len(want) == 96
    assert got == want
    if wtype != Q4_K:
        assert len(set(want)) > 20  # a diverse stream


@pytest.mark.parametrize("wtype", [Q4_K, Q6_K])
def test_tiny_model_fast_attention(tmp_path, oracle_model_cls, wtype):
    """Split-KV softmax mode: logits within tolerance at every step."""
    from gncx_b200.streamer import GNCXStreamer
    path = gguf.write_random_model(tmp_path / "tiny.gguf", TINY, seed=6, wtype=wtype)
    prompt = np.random.default_rng(7).integers(0, TINY["vocab"], 50).tolist()
    ref = oracle_model_cls(path, 128)
    with GNCXStreamer(path, max_seq_len=128) as eng:
        lg, lr = eng.prefill(prompt), ref.prefill(prompt)
        errs = [rel(lg, lr)]
        ids = list(prompt)
        for step in range(24):
            t = ref_sample(lr, ids)
            ids.append(t)
            lr = ref.forward_token(t, len(ids) - 1)
            lg = eng.forward_token(t, len(ids) - 1)
            errs.append(rel(lg, lr))
    ref.close()
    # A softmax sum formed in another order moves an attention output by ~1e-6;
    # when that output sits at an int8 rounding boundary of the next GEMV's
    # activation quantization it flips one quant step (~1e-2 of the logits).
    # Most steps agree to ~1e-6.
    print("fast-mode logit errors:", ["%.1e" % x for x in errs])
    assert max(errs) <= 3e-2
    assert np.median(errs) <= 1e-4


def ref_sample(logits, recent, penalty=1.15):
    from oracle.oracle import Oracle
    return Oracle().sample_greedy(logits, recent, penalty)


def test_qwen3_0p6b_config(tmp_path, oracle_model_cls):
    """Benchmark configuration 4: random-init Qwen3-0.6B shape, Q4_K weights,
    Q6_K tied head, 128-token seeded prompt, 256 greedy tokens."""
    from gncx_b200.streamer import GNCXStreamer
    path = gguf.write_random_model(tmp_path / "q06b.gguf", "qwen3-0.6b", seed=4)
    prompt = np.random.default_rng(4).integers(0, 151936, 128).tolist()
    ref = oracle_model_cls(path, 128 + 256)
    want = ref.generate(prompt, 256, 1.15, -1)
    lr = ref.prefill(prompt)
    ref.close()
    _check_logits(lr)
    with GNCXStreamer(path, max_seq_len=128 + 256, exact_attention=True) as eng:
        lg = eng.prefill(prompt)
        assert rel(lg, lr) <= LOGIT_TOL
        got = eng.generate_ids(prompt, 256, 1.15, eos_id=-1)
        t = eng.timing()
        eng.set_exact_attention(False)
        fast = eng.generate_ids(prompt, 256, 1.15, eos_id=-1)
    assert got == want
    assert t["decode_steps"] == 255 and t["decode_ms"] > 0
    # split-KV mode: report how far it agrees (a near-tie may flip late)
    agree = next((i for i, (a, b) in enumerate(zip(fast, want)) if a != b), len(want))
    print(f"split-KV softmax stream agrees for {agree} of {len(want)} tokens")
    assert agree >= 64


def test_engine_rejects_bad_input(tmp_path):
    from gncx_b200 import core
    from gncx_b200.streamer import GNCXStreamer
    with pytest.raises(core.GncxError):
        GNCXStreamer(tmp_path / "missing.gguf")
    path = gguf.write_random_model(tmp_path / "t.gguf", TINY, seed=5)
    with GNCXStreamer(path, max_seq_len=64) as eng:
        with pytest.raises(core.GncxError):
            eng.forward_token(TINY["vocab"] + 5, 0)
        with pytest.raises(core.GncxError):
            eng.forward_token(1, 64)
        # generation stops at the context limit (lua/gncx_streamer.lua:1288)
        assert len(eng.generate_ids(list(range(60)), 50, eos_id=-1)) == 4
