"""GPU parity of every hot-path kernel, called through the C ABI, against the
CPU oracle (itself pinned to the reference by test_oracle.py) and against the
golden vectors generated from the reference.

Bars: integer/byte work and the GEMV/GEMM/RMSNorm/RoPE/embedding paths are
bit-exact; attention and the GLU activations use exp/tanh, where the
reference's libm differs from a correctly rounded result on ~1e-4 of inputs,
so they are held to max |err| <= 1e-5 * max |ref| (north star allows 1e-3).
"""
import ctypes

import numpy as np
import pytest

from conftest import golden
from gncx_b200 import core, synth
from gncx_b200.core import BF16, Q4_0, Q4_K, Q6_K, Q8_0

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

ATTN_TOL = 1e-5


# Every device buffer made here stays referenced until the test ends: a
# temporary whose address went to the C ABI must not be freed (and its memory
# handed to the next upload) before the kernel has read it.
_KEEP: list = []


@pytest.fixture(autouse=True)
def _keep_buffers():
    _KEEP.clear()
    yield
    torch.cuda.synchronize()
    _KEEP.clear()


def dev(a: np.ndarray):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _KEEP.append(t)
    return t


def out(n, dtype=torch.float32):
    t = torch.full((n,), float("nan"), dtype=dtype, device="cuda")
    _KEEP.append(t)
    return t


def P(t):
    return ctypes.c_void_p(t.data_ptr())


def host(t) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()


def matvec(lib, w_d, t, x, out_dim, off=0):
    y = out(out_dim)
    lib.gncx_xfold_universal_matvec(P(w_d), off, t, P(dev(x)), None, x.size, out_dim, P(y), None)
    core.check(lib)
    return host(y)


# ---------------------------------------------------------------- GEMV
@pytest.mark.parametrize("t", [Q4_0, Q8_0, Q4_K, Q6_K, BF16])
def test_gemv_golden(gpu, t):
    g = golden(f"gemv_{t}.npz")
    rows = g["y_strict"].size
    assert np.array_equal(matvec(gpu, dev(g["w"]), t, g["x"], rows), g["y_strict"])


SHAPES = [(4096, 4096), (4096, 12288), (12288, 4096), (1000, 1024), (37, 2048), (5, 256)]


@pytest.mark.parametrize("t", [Q4_0, Q8_0, Q4_K, Q6_K])
@pytest.mark.parametrize("shape", SHAPES)
def test_gemv_bit_exact(gpu, oracle, t, shape):
    out_dim, in_dim = shape
    w = synth.random_weights(t, out_dim, in_dim, seed=out_dim + in_dim + t)
    x = synth.random_activations(in_dim, seed=in_dim)
    x[256:288] = 0.0  # an all-zero act block
    got = matvec(gpu, dev(w), t, x, out_dim)
    assert np.array_equal(got, oracle.matvec(w, t, x, out_dim))


@pytest.mark.parametrize("t", [Q4_0, Q8_0, Q4_K, Q6_K])
def test_gemv_unaligned_base(gpu, oracle, t):
    """Any base alignment works (rows are copied as 16-byte-aligned supersets)."""
    out_dim, in_dim = 70, 1024
    w = synth.random_weights(t, out_dim, in_dim, seed=3)
    x = synth.random_activations(in_dim, seed=4)
    buf = np.zeros(w.size + 64, np.uint8)
    for shift in (2, 6, 8, 14):
        buf[:] = 0
        buf[shift:shift + w.size] = w.reshape(-1)
        got = matvec(gpu, dev(buf), t, x, out_dim, off=shift)
        assert np.array_equal(got, oracle.matvec(w, t, x, out_dim)), shift


def test_gemv_lm_head_config(gpu, oracle):
    """The 151936x4096 LM-head shape (Q6_K) and the 0.6B head (151936x1024)."""
    for in_dim in (4096, 1024):
        w = synth.random_weights_fast(Q6_K, 151936, in_dim, seed=in_dim)
        x = synth.random_activations(in_dim, seed=1)
        got = matvec(gpu, dev(w), Q6_K, x, 151936)
        assert np.array_equal(got, oracle.matvec(w, Q6_K, x, 151936))


def test_lm_head_softcap(gpu):
    g = golden("lm_head.npz")
    y = out(100)
    gpu.gncx_universal_lm_head_logits(P(dev(g["w"])), 0, Q6_K, P(dev(g["h"])), 256, 100, 30.0, P(y))
    core.check(gpu)
    got = host(y)
    assert np.max(np.abs(got - g["y_strict"])) <= 2e-7 * 30.0  # tanh rounding only
    y2 = out(100)
    gpu.gncx_universal_lm_head_logits(P(dev(g["w"])), 0, Q6_K, P(dev(g["h"])), 256, 100, 0.0, P(y2))
    assert np.array_equal(host(y2), g["y_nocap"])


def test_act_quantize_bit_exact(gpu, oracle):
    x = synth.random_activations(12288, seed=5) * 7.0
    x[64:96] = 0.0
    a = torch.zeros(12288 // 32 * 48, dtype=torch.uint8, device="cuda")
    assert gpu.gncx_act_quantize(P(dev(x)), 1, 12288, P(a)) == 0
    blk = host(a).view(np.int32).reshape(-1, 12)
    ref = oracle.act_quantize(x)
    assert np.array_equal(blk[:, 0].view(np.float32), ref["d"])
    assert np.array_equal(blk[:, 1], ref["sum_lo"]) and np.array_equal(blk[:, 2], ref["sum_hi"])
    assert np.array_equal(blk[:, 4:].copy().view(np.int8), ref["qs"])


@pytest.mark.parametrize("t", [Q4_0, Q4_K, Q6_K])
def test_matvec_preq_matches(gpu, oracle, t):
    w = synth.random_weights(t, 512, 4096, seed=9)
    x = synth.random_activations(4096, seed=10)
    a = torch.zeros(4096 // 32 * 48, dtype=torch.uint8, device="cuda")
    assert gpu.gncx_act_quantize(P(dev(x)), 1, 4096, P(a)) == 0
    y = out(512)
    assert gpu.gncx_matvec_preq(P(dev(w)), 0, t, P(a), 4096, 512, P(y)) == 0
    assert np.array_equal(host(y), oracle.matvec(w, t, x, 512))


def test_gemv_rejects_bad_args(gpu):
    w = dev(synth.random_weights(Q4_K, 4, 256))
    y = out(4)
    gpu.gncx_xfold_universal_matvec(P(w), 0, 99, P(dev(np.zeros(256, np.float32))), None, 256, 4, P(y), None)
    assert gpu.gncx_last_error() == 1
    gpu.gncx_clear_error()
    gpu.gncx_xfold_universal_matvec(P(w), 0, Q4_K, P(dev(np.zeros(200, np.float32))), None, 200, 4, P(y), None)
    assert gpu.gncx_last_error() == 1
    gpu.gncx_clear_error()
    host_buf = (ctypes.c_float * 256)()
    gpu.gncx_xfold_universal_matvec(P(w), 0, Q4_K, host_buf, None, 256, 4, P(y), None)
    assert gpu.gncx_last_error() == 6  # not device-accessible
    gpu.gncx_clear_error()


def test_telemetry_counters(gpu):
    w = dev(synth.random_weights(Q4_K, 64, 512))
    tel = core.GNCXTelemetryStats()
    y = out(64)
    gpu.gncx_xfold_universal_matvec(P(w), 0, Q4_K, P(dev(np.ones(512, np.float32))), None, 512, 64, P(y),
                                    ctypes.byref(tel))
    core.check(gpu)
    assert tel.total_macs_equivalent == 512 * 64
    assert tel.zero_weight_skips == 512 * 64 // 15
    assert tel.xfold_bucket_merges == 16 * 64


# ---------------------------------------------------------------- prefill GEMM
@pytest.mark.parametrize("t", [Q4_0, Q8_0, Q4_K, Q6_K, BF16])
def test_matbatch_golden(gpu, t):
    g = golden(f"gemv_{t}.npz")
    rows = g["y_strict"].size
    xb = g["xb"]
    y = out(xb.shape[0] * rows)
    gpu.gncx_xfold_universal_matbatch(P(dev(g["w"])), 0, t, P(dev(xb)), xb.shape[0], xb.shape[1], rows, P(y), None)
    core.check(gpu)
    assert np.array_equal(host(y).reshape(xb.shape[0], rows), g["yb_strict"])


@pytest.mark.parametrize("t", [Q4_0, Q8_0, Q4_K, Q6_K])
def test_matbatch_bit_exact(gpu, oracle, t):
    out_dim, in_dim, B = 300, 2048, 70
    w = synth.random_weights(t, out_dim, in_dim, seed=21 + t)
    xb = synth.random_activations(in_dim, seed=22, rows=B)
    xb[3, :32] = 0.0
    y = out(B * out_dim)
    gpu.gncx_xfold_universal_matbatch(P(dev(w)), 0, t, P(dev(xb)), B, in_dim, out_dim, P(y), None)
    core.check(gpu)
    assert np.array_equal(host(y).reshape(B, out_dim), oracle.matbatch(w, t, xb, out_dim))


# ---------------------------------------------------------------- norms, rope, glu, embed
def test_rmsnorm(gpu, oracle):
    g = golden("norm.npz")
    y = out(1024)
    gpu.gncx_rmsnorm_and_encode_4phase(P(dev(g["x"])), P(dev(g["w"])), 0, 1024, 1e-6, 3, P(y), None, None)
    core.check(gpu)
    assert np.array_equal(host(y), g["y_strict"])
    for dim in (4096, 1024, 4100):
        x = synth.random_activations(dim, seed=dim) * 5
        w = synth.random_activations(dim, seed=dim + 1)
        y = out(dim)
        scale = ctypes.c_float(0.0)
        gpu.gncx_rmsnorm_and_encode_4phase(P(dev(x)), P(dev(w)), 0, dim, 1e-6, 3, P(y), None, ctypes.byref(scale))
        core.check(gpu)
        assert np.array_equal(host(y), oracle.rmsnorm(x, w, 1e-6))
        assert scale.value == 1.0


def test_rmsnorm_heads(gpu):
    g = golden("norm.npz")
    v = dev(g["v"])
    gpu.gncx_rmsnorm_inplace_heads(P(v), P(dev(g["wh"])), 0, 1, 8, 64, 1e-6)
    core.check(gpu)
    assert np.array_equal(host(v), g["heads_strict"])
    v2 = dev(g["v"])
    gpu.gncx_rmsnorm_inplace_heads(P(v2), None, 0, 0, 8, 64, 1e-6)
    core.check(gpu)
    assert np.array_equal(host(v2), g["heads_nw_strict"])


def test_rope(gpu):
    g = golden("rope.npz")
    for i, p in enumerate(g["pos"]):
        q, k = dev(g["q"]), dev(g["k"])
        gpu.gncx_apply_rope_xor11_ext(P(q), P(k), None, None, 0, 0, 8, 2, 64, int(p), 1e6)
        core.check(gpu)
        assert np.array_equal(host(q), g["q_strict"][i]) and np.array_equal(host(k), g["k_strict"][i])
        qf = dev(g["q"])
        gpu.gncx_apply_rope_xor11_ext(P(qf), None, None, P(dev(g["ff"])), 0, 1, 8, 2, 64, int(p), 1e4)
        core.check(gpu)
        assert np.array_equal(host(qf), g["qff_strict"][i])


def test_glu(gpu):
    g = golden("glu.npz")
    for gelu, key in ((False, "swiglu_strict"), (True, "geglu_strict")):
        y = out(1000)
        fn = gpu.gncx_geglu_activation if gelu else gpu.gncx_swiglu_activation
        fn(P(dev(g["g"])), P(dev(g["u"])), 1000, P(y))
        core.check(gpu)
        r = g[key]
        assert np.max(np.abs(host(y) - r)) <= 4e-7 * np.max(np.abs(r))


def test_embedding_and_dequant(gpu, oracle):
    g = golden("embed.npz")
    for t, fn in ((Q8_0, gpu.gncx_fetch_token_embedding_q8_0), (Q6_K, gpu.gncx_fetch_token_embedding_q6_k),
                  (BF16, gpu.gncx_fetch_token_embedding_bf16)):
        w = dev(g[f"w_{t}"])
        got = []
        for r in (0, 3, 9):
            for s in (1.0, 22.627417):
                y = out(512)
                fn(P(w), 0, r, 512, s, P(y))
                core.check(gpu)
                got.append(host(y))
        assert np.array_equal(np.stack(got), g[f"rows_{t}"])
    for t in (Q4_0, Q8_0, Q4_K, Q6_K, BF16):
        w = synth.random_weights(t, 6, 512, seed=40 + t)
        y = out(6 * 512)
        assert gpu.gncx_dequantize_rows(P(dev(w)), 0, t, 6, 512, P(y)) == 0
        ref = np.stack([oracle.dequant_row(w[r], t, 512) for r in range(6)])
        assert np.array_equal(host(y).reshape(6, 512), ref)


# ---------------------------------------------------------------- attention
def test_attention_golden(gpu):
    g = golden("attention.npz")
    kc, vc = dev(g["kc"]), dev(g["vc"])
    y = out(8 * 64)
    gpu.gncx_mqa_attention_step_ext(P(dev(g["q"])), P(dev(g["k"])), P(dev(g["v"])), P(kc), P(vc), 36, 8, 2, 64,
                                    0.125, 0, 1, P(y))
    core.check(gpu)
    assert np.array_equal(host(kc), g["kc_after"]) and np.array_equal(host(vc), g["vc_after"])
    r = g["out_strict"]
    assert np.max(np.abs(host(y) - r)) <= ATTN_TOL * np.max(np.abs(r))
    y16 = out(8 * 64)
    gpu.gncx_mqa_attention_step_ext(P(dev(g["q"])), None, None, P(kc), P(vc), 36, 8, 2, 64, 0.125, 16, 0, P(y16))
    core.check(gpu)
    r16 = g["out_window16_strict"]
    assert np.max(np.abs(host(y16) - r16)) <= ATTN_TOL * np.max(np.abs(r16))


@pytest.mark.parametrize("ctx,window", [(1, 0), (512, 0), (4096, 0), (5000, 4096), (32768, 0)])
def test_attention_config(gpu, oracle, ctx, window):
    nh, nkv, hd = 32, 8, 128
    kc_np = synth.random_activations(ctx * nkv * hd, seed=ctx)
    vc_np = synth.random_activations(ctx * nkv * hd, seed=ctx + 1)
    q = synth.random_activations(nh * hd, seed=2)
    k = synth.random_activations(nkv * hd, seed=3)
    v = synth.random_activations(nkv * hd, seed=4)
    scale = float(np.float32(1.0 / np.sqrt(128.0)))
    ref, kc_ref, _ = oracle.attention(q, k, v, kc_np, vc_np, ctx - 1, nh, nkv, hd, scale, window, 1)
    kc, vc = dev(kc_np), dev(vc_np)
    y = out(nh * hd)
    gpu.gncx_mqa_attention_step_ext(P(dev(q)), P(dev(k)), P(dev(v)), P(kc), P(vc), ctx - 1, nh, nkv, hd, scale,
                                    window, 1, P(y))
    core.check(gpu)
    got = host(y)
    assert np.max(np.abs(got - ref)) <= ATTN_TOL * np.max(np.abs(ref))
    assert np.array_equal(host(kc)[(ctx - 1) * nkv * hd:], kc_ref[(ctx - 1) * nkv * hd:])


@pytest.mark.parametrize("nh,nkv,hd", [(4, 2, 64), (8, 1, 128), (32, 8, 128), (8, 8, 128)])
@pytest.mark.parametrize("exact", [0, 1])
def test_attention_write_kv(gpu, oracle, nh, nkv, hd, exact):
    """write_kv = 1 (:1903-1907): the new K/V rows land in the cache at `pos`
    and the step attends to them, whether the kernel reads them in place or
    they are copied first; k/v from device memory and from host memory."""
    scale = float(np.float32(1.0 / np.sqrt(hd)))
    gpu.gncx_set_exact_attention(exact)
    try:
        for ctx in (1, 2, 17, 63, 64, 65, 129, 1025, 4097):
            kc_np = synth.random_activations(ctx * nkv * hd, seed=ctx + 11)
            vc_np = synth.random_activations(ctx * nkv * hd, seed=ctx + 12)
            q = synth.random_activations(nh * hd, seed=ctx + 13)
            k = synth.random_activations(nkv * hd, seed=ctx + 14)
            v = synth.random_activations(nkv * hd, seed=ctx + 15)
            for window in (0, 17):
                ref, kc_ref, vc_ref = oracle.attention(q, k, v, kc_np, vc_np, ctx - 1, nh, nkv, hd, scale, window, 1)
                for on_host in (False, True):
                    kc, vc = dev(kc_np), dev(vc_np)
                    kp = k.ctypes.data_as(ctypes.c_void_p) if on_host else P(dev(k))
                    vp = v.ctypes.data_as(ctypes.c_void_p) if on_host else P(dev(v))
                    y = out(nh * hd)
                    gpu.gncx_mqa_attention_step_ext(P(dev(q)), kp, vp, P(kc), P(vc), ctx - 1, nh, nkv, hd, scale,
                                                    window, 1, P(y))
                    core.check(gpu)
                    err = np.max(np.abs(host(y) - ref)) / np.max(np.abs(ref))
                    assert err <= ATTN_TOL, (ctx, window, on_host, err)
                    assert np.array_equal(host(kc), kc_ref) and np.array_equal(host(vc), vc_ref), (ctx, on_host)
    finally:
        gpu.gncx_set_exact_attention(0)


@pytest.mark.parametrize("nh,nkv,hd", [(4, 2, 64), (8, 1, 128), (16, 8, 64), (32, 8, 128), (8, 8, 128), (8, 2, 64)])
@pytest.mark.parametrize("exact", [0, 1])
def test_attention_lengths(gpu, oracle, nh, nkv, hd, exact):
    """Every context length up to 70 and the chunk edges around 128 / 1024,
    with and without a sliding window, in both softmax modes."""
    scale = float(np.float32(1.0 / np.sqrt(hd)))
    gpu.gncx_set_exact_attention(exact)
    try:
        for ctx in list(range(1, 71)) + [127, 128, 129, 1023, 1024, 1025]:
            kc_np = synth.random_activations(ctx * nkv * hd, seed=ctx)
            vc_np = synth.random_activations(ctx * nkv * hd, seed=ctx + 7)
            q = synth.random_activations(nh * hd, seed=ctx + 3)
            kc, vc = dev(kc_np), dev(vc_np)
            for window in (0, 17):
                ref, _, _ = oracle.attention(q, None, None, kc_np, vc_np, ctx - 1, nh, nkv, hd, scale, window, 0)
                y = out(nh * hd)
                gpu.gncx_mqa_attention_step_ext(P(dev(q)), None, None, P(kc), P(vc), ctx - 1, nh, nkv, hd, scale,
                                                window, 0, P(y))
                core.check(gpu)
                err = np.max(np.abs(host(y) - ref)) / np.max(np.abs(ref))
                assert err <= ATTN_TOL, (ctx, window, err)
    finally:
        gpu.gncx_set_exact_attention(0)


# ---------------------------------------------------------------- sampling
def test_sample_greedy(gpu, oracle):
    rng = np.random.default_rng(0)
    for trial in range(5):
        logits = rng.normal(0, 3, size=151936).astype(np.float32)
        logits[rng.integers(0, 151936, 4)] = logits.max()  # ties
        recent = rng.integers(0, 151936, size=rng.integers(0, 200)).astype(np.int32)
        recent[-3:] = np.argsort(logits)[-3:]
        rc = (ctypes.c_int32 * max(1, recent.size))(*recent.tolist())
        got = gpu.gncx_sample_greedy(P(dev(logits)), 151936, rc, recent.size, 1.15)
        core.check(gpu)
        assert got == oracle.sample_greedy(logits, recent, 1.15)


# ---------------------------------------------------------------- headline GEMV instantiations
@pytest.mark.parametrize("t", [Q4_K, Q4_0, Q8_0])
def test_gemv_headline_shape(gpu, oracle, t):
    """151936 x 4096, the shape whose launch carries the bench's roofline:
    at >= 16 eight-warp tiles per SM the launcher takes the 4-warp, two
    CTAs per SM instantiation (aligned rows, fp32 x re-quantized in the
    kernel), csrc/gncx_llm_kernels.cpp:1362-1431."""
    w = synth.random_weights_fast(t, 151936, 4096, seed=100 + t)
    x = synth.random_activations(4096, seed=101)
    x[1024:1056] = 0.0  # an all-zero act block
    assert np.array_equal(matvec(gpu, dev(w), t, x, 151936), oracle.matvec(w, t, x, 151936))


@pytest.mark.parametrize("t", [Q4_K, Q6_K])
def test_gemv_headline_shape_staged_act(gpu, oracle, t):
    """The same shape fed a pre-quantized (staged) activation vector, as the
    engine's LM head and decode GEMVs are."""
    w = synth.random_weights_fast(t, 151936, 4096, seed=200 + t)
    x = synth.random_activations(4096, seed=201)
    a = torch.zeros(4096 // 32 * 48, dtype=torch.uint8, device="cuda")
    _KEEP.append(a)
    assert gpu.gncx_act_quantize(P(dev(x)), 1, 4096, P(a)) == 0
    y = out(151936)
    assert gpu.gncx_matvec_preq(P(dev(w)), 0, t, P(a), 4096, 151936, P(y)) == 0
    assert np.array_equal(host(y), oracle.matvec(w, t, x, 151936))


# ---------------------------------------------------------------- causal prefill attention
def _prefill_rows(n_tok):
    """Rows to check against the oracle: the first 70, every chunk and group
    edge, a stride through the middle, the last."""
    rows = set(range(min(70, n_tok)))
    for e in (63, 64, 65, 127, 128, 129, 255, 256, 257, 511, 512, 513, 1023, 1024, 1025, 1535, 2047):
        if e < n_tok:
            rows.add(e)
    rows.update(range(0, n_tok, 29))
    rows.add(n_tok - 1)
    return sorted(rows)


@pytest.mark.parametrize("nh,nkv,hd,pos0,n_tok", [(32, 8, 128, 0, 2048), (32, 8, 128, 300, 333), (16, 8, 64, 0, 600),
                                                  (6, 2, 96, 5, 300)])
@pytest.mark.parametrize("exact", [0, 1])
def test_attention_prefill(gpu, oracle, nh, nkv, hd, pos0, n_tok, exact):
    """The causal prefill kernel (query-tiled, split records merged per query)
    row by row against the reference's decode step at that row's position
    (csrc/gncx_llm_kernels.cpp:1887-1994 called per prompt position,
    lua/gncx_streamer.lua:1079-1109).  32/8 x 128 and 16/8 x 64 take the
    query-tiled kernel; 6/2 x 96 the general split kernel; exact mode the
    serial-order kernels."""
    if exact and n_tok > 1000:
        pytest.skip("exact mode: the shorter prompts cover it")
    total = pos0 + n_tok
    kvd = nkv * hd
    kc_np = synth.random_activations(total * kvd, seed=total)
    vc_np = synth.random_activations(total * kvd, seed=total + 1)
    q = synth.random_activations(nh * hd, seed=nh + hd, rows=n_tok)
    scale = float(np.float32(1.0 / np.sqrt(hd)))
    y = out(n_tok * nh * hd)
    gpu.gncx_set_exact_attention(exact)
    try:
        st = gpu.gncx_attention_prefill(P(dev(q)), P(dev(kc_np)), P(dev(vc_np)), pos0, n_tok, nh, nkv, hd, scale, P(y))
        assert st == 0, (gpu.gncx_last_error_message() or b"").decode()
    finally:
        gpu.gncx_set_exact_attention(0)
    got = host(y).reshape(n_tok, nh * hd)
    worst = 0.0
    for z in _prefill_rows(n_tok):
        pos = pos0 + z
        ref, _, _ = oracle.attention(q[z], None, None, kc_np[:(pos + 1) * kvd], vc_np[:(pos + 1) * kvd], pos, nh, nkv,
                                     hd, scale, 0, 0)
        err = np.max(np.abs(got[z] - ref)) / np.max(np.abs(ref))
        worst = max(worst, err)
        assert err <= ATTN_TOL, (z, err)
    assert np.all(np.isfinite(got))
    print(f"prefill attention {nh}/{nkv}x{hd} pos0={pos0} n={n_tok} exact={exact}: worst rel err {worst:.2e}")
