"""The persistent decode step (gncx_b200/csrc/decode_step.cu): one kernel per
token for the whole layer stack on one GPU.

For every weight format the kernel dispatches (Q4_0, Q8_0, Q4_K, Q6_K), the
head geometries of the benchmark configurations (G = 2 with head_dim 64 and
128, G = 4 with the 8B layer shape) and contexts spanning many attention
chunks:
  * exact attention mode: every logit vector (prefill, then each
    forward_token) is bit-identical to this library's per-kernel decode
    (GNCX_DECODE_PERSISTENT=0), which is pinned to the reference elsewhere --
    the same GEMV, norm, GLU and attention arithmetic in the same order;
  * split-KV mode: each forward_token's logits, teacher-forced on the
    reference's tokens, against the reference orchestration over the
    reference's own kernels (lua/gncx_streamer.lua:759-965) within the
    split-KV bounds, and against the per-kernel split-KV decode;
  * the device-driven greedy loop (one CUDA graph per token) against the same
    engine stepped token by token on the host: identical.
"""
import os

import numpy as np
import pytest

from gncx_b200 import gguf
from gncx_b200.core import Q4_0, Q4_K, Q6_K, Q8_0

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TINY = dict(n_layers=4, dim=256, n_heads=4, n_kv=2, head_dim=64, ffn=512, vocab=4000, eps=1e-6, rope_base=1e6)
W1024 = dict(n_layers=3, dim=1024, n_heads=16, n_kv=8, head_dim=128, ffn=3072, vocab=3000, eps=1e-6, rope_base=1e6)
W8B = dict(n_layers=2, dim=4096, n_heads=32, n_kv=8, head_dim=128, ffn=12288, vocab=3000, eps=1e-6, rope_base=1e6)


def rel(a, b):
    return float(np.max(np.abs(a - b)) / max(1e-30, np.max(np.abs(b))))


def _engine(path, max_seq, persistent=True, exact=False):
    from gncx_b200.streamer import GNCXStreamer
    old = os.environ.get("GNCX_DECODE_PERSISTENT")
    os.environ["GNCX_DECODE_PERSISTENT"] = "1" if persistent else "0"
    try:
        eng = GNCXStreamer(path, max_seq_len=max_seq, exact_attention=exact)
    finally:
        if old is None:
            os.environ.pop("GNCX_DECODE_PERSISTENT", None)
        else:
            os.environ["GNCX_DECODE_PERSISTENT"] = old
    assert eng.persistent_decode() == persistent
    return eng


def _ref_tokens(path, prompt, n_steps, max_seq):
    from oracle.oracle import Oracle, OracleModel
    orc = Oracle()
    ref = OracleModel(path, max_seq)
    lr = ref.prefill(prompt)
    ids, toks, logits = list(prompt), [], [lr]
    for _ in range(n_steps):
        t = orc.sample_greedy(lr, ids, 1.15)
        toks.append(t)
        ids.append(t)
        lr = ref.forward_token(t, len(ids) - 1)
        logits.append(lr)
    ref.close()
    return toks, logits


def _teacher_forced(eng, prompt, toks):
    out = [eng.prefill(prompt)]
    for i, t in enumerate(toks):
        out.append(eng.forward_token(t, len(prompt) + i))
    return out


CASES = [
    ("q4_0-tiny", TINY, Q4_0, 50, 20),
    ("q8_0-tiny", TINY, Q8_0, 50, 20),
    ("q4_k-tiny", TINY, Q4_K, 300, 20),   # 300 positions: three 128-position chunks per KV head
    ("q6_k-tiny", TINY, Q6_K, 50, 20),
    ("q4_k-1024", W1024, Q4_K, 200, 12),  # configuration 4's layer shape
    ("q4_k-8b", W8B, Q4_K, 700, 10),      # configuration 5's layer shape: 11 chunks x 8 KV heads
]


@pytest.mark.parametrize("name,hp,wtype,n_prompt,n_steps", CASES, ids=[c[0] for c in CASES])
def test_persistent_step_exact_bit_identical(tmp_path, name, hp, wtype, n_prompt, n_steps):
    path = gguf.write_random_model(tmp_path / f"{name}.gguf", hp, seed=11, wtype=wtype)
    rng = np.random.default_rng(13)
    prompt = rng.integers(0, hp["vocab"], n_prompt).tolist()
    toks = rng.integers(0, hp["vocab"], n_steps).tolist()
    max_seq = n_prompt + n_steps + 8
    with _engine(path, max_seq, persistent=True, exact=True) as eng:
        got = _teacher_forced(eng, prompt, toks)
    with _engine(path, max_seq, persistent=False, exact=True) as eng:
        want = _teacher_forced(eng, prompt, toks)
    same = [bool(np.array_equal(a, b)) for a, b in zip(got, want)]
    print(f"{name} exact: {sum(same)}/{len(same)} logit vectors bit-identical; "
          f"max rel diff {max(rel(a, b) for a, b in zip(got, want)):.2e}")
    assert all(same)


@pytest.mark.parametrize("name,hp,wtype,n_prompt,n_steps", CASES, ids=[c[0] for c in CASES])
def test_persistent_step_split_kv(tmp_path, name, hp, wtype, n_prompt, n_steps):
    path = gguf.write_random_model(tmp_path / f"{name}.gguf", hp, seed=11, wtype=wtype)
    prompt = np.random.default_rng(12).integers(0, hp["vocab"], n_prompt).tolist()
    max_seq = n_prompt + n_steps + 8
    toks, ref_logits = _ref_tokens(path, prompt, n_steps, max_seq)
    with _engine(path, max_seq, persistent=True) as eng:
        got = _teacher_forced(eng, prompt, toks)
    with _engine(path, max_seq, persistent=False) as eng:
        per_kernel = _teacher_forced(eng, prompt, toks)
    errs = np.array([rel(g, r) for g, r in zip(got[1:], ref_logits[1:])])
    diffs = np.array([rel(g, k) for g, k in zip(got[1:], per_kernel[1:])])
    print(f"{name} split-KV: vs reference max {errs.max():.2e} median {np.median(errs):.2e}; "
          f"vs per-kernel max {diffs.max():.2e} median {np.median(diffs):.2e}")
    for g in got:
        assert np.all(np.isfinite(g))
    # split-KV bounds (as for the per-kernel split-KV decode): an attention
    # output moved by ~1e-6 can flip one int8 quant of the next GEMV's input
    assert errs.max() <= 3e-2 and np.median(errs) <= 1e-4
    assert diffs.max() <= 3e-2 and np.median(diffs) <= 1e-4


@pytest.mark.parametrize("exact", [False, True], ids=["split_kv", "exact"])
def test_persistent_step_graph_loop(tmp_path, exact):
    """generate_ids (graph replays, state on the device) equals the same engine
    stepped on the host: prefill, then sample + forward_token per token."""
    path = gguf.write_random_model(tmp_path / "g.gguf", TINY, seed=21, wtype=Q6_K)
    prompt = np.random.default_rng(22).integers(0, TINY["vocab"], 40).tolist()
    n_new = 48
    with _engine(path, 128, persistent=True, exact=exact) as eng:
        got = eng.generate_ids(prompt, n_new, 1.15, eos_id=-1)
        ids = list(prompt)
        eng.prefill(prompt)
        want = []
        for _ in range(n_new):
            t = eng.sample(ids, 1.15)
            want.append(t)
            ids.append(t)
            eng.forward_token(t, len(ids) - 1)
    assert got == want
    assert len(set(got)) > 10  # a diverse stream
