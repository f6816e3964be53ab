"""Generate the golden vectors in this directory from the REFERENCE itself.

Run in a checkout where the reference sources are present (they are compiled by
oracle/Makefile into oracle/_ref/):

    python tests/golden/make_golden.py

Every output array comes from calling the reference's compiled kernels through
its C ABI on seeded inputs: ``*_strict`` from the -ffp-contract=off build (the
bit-exact pin of the oracle and of the CUDA kernels), ``*_native`` from the
as-shipped flags (FMA contraction allowed; a tolerance pin).  The reference's
own tests hold no golden values for this path, so these fixtures are the pin.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from gncx_b200 import synth  # noqa: E402
from gncx_b200.core import BF16, Q4_0, Q4_K, Q6_K, Q8_0  # noqa: E402
from oracle.oracle import REF_NATIVE_SO, REF_STRICT_SO, RefLib, build  # noqa: E402

OUT = Path(__file__).resolve().parent


def main() -> None:
    build(with_reference=True)
    S, N = RefLib(REF_STRICT_SO), RefLib(REF_NATIVE_SO)
    # GEMV + prefill GEMM, every format
    for t, (rows, n) in {Q4_0: (40, 512), Q8_0: (40, 512), Q4_K: (40, 512), Q6_K: (40, 512), BF16: (24, 256)}.items():
        w = synth.random_weights(t, rows, n, seed=100 + t)
        x = synth.random_activations(n, seed=200 + t)
        x[32:64] = 0.0  # an all-zero activation block (d == 0 is skipped by the reference)
        xb = synth.random_activations(n, seed=300 + t, rows=3)
        xb[1, 64:96] = 0.0
        np.savez_compressed(OUT / f"gemv_{t}.npz", w=w, x=x, xb=xb, y_strict=S.matvec(w, t, x, rows),
                            y_native=N.matvec(w, t, x, rows), yb_strict=S.matbatch(w, t, xb, rows),
                            yb_native=N.matbatch(w, t, xb, rows))
    # LM head with softcap
    w = synth.random_weights(Q6_K, 100, 256, seed=7)
    h = synth.random_activations(256, seed=8) * 40.0
    np.savez_compressed(OUT / "lm_head.npz", w=w, h=h, y_strict=S.lm_head(w, Q6_K, h, 100, 30.0),
                        y_nocap=S.lm_head(w, Q6_K, h, 100, 0.0))
    # norms
    x = synth.random_activations(1024, seed=9) * 3.0
    wn = synth.random_activations(1024, seed=10)
    v = synth.random_activations(8 * 64, seed=11)
    wh = synth.random_activations(64, seed=12)
    np.savez_compressed(OUT / "norm.npz", x=x, w=wn, eps=np.float32(1e-6), y_strict=S.rmsnorm(x, wn, 1e-6),
                        v=v, wh=wh, heads_strict=S.rmsnorm_heads(v, wh, 8, 64, 1e-6),
                        heads_nw_strict=S.rmsnorm_heads(v, None, 8, 64, 1e-6))
    # RoPE at a few positions, with and without frequency factors
    q = synth.random_activations(8 * 64, seed=13)
    k = synth.random_activations(2 * 64, seed=14)
    ff = (1.0 + np.abs(synth.random_activations(32, seed=15))).astype(np.float32)
    pos = np.array([0, 1, 100, 4095, 32767], np.int32)
    rq, rk, fq = [], [], []
    for p in pos:
        a, b = S.rope(q, k, 8, 2, 64, int(p), 1e6)
        rq.append(a)
        rk.append(b)
        fq.append(S.rope(q, None, 8, 2, 64, int(p), 1e4, ff)[0])
    np.savez_compressed(OUT / "rope.npz", q=q, k=k, ff=ff, pos=pos, q_strict=np.stack(rq), k_strict=np.stack(rk),
                        qff_strict=np.stack(fq))
    # decode attention (GQA 8/2, head_dim 64), full and sliding window
    L = 37
    kc = synth.random_activations(L * 2 * 64, seed=16)
    vc = synth.random_activations(L * 2 * 64, seed=17)
    qa = synth.random_activations(8 * 64, seed=18)
    ka = synth.random_activations(2 * 64, seed=19)
    va = synth.random_activations(2 * 64, seed=20)
    o0, kc0, vc0 = S.attention(qa, ka, va, kc, vc, L - 1, 8, 2, 64, 0.125, 0, 1)
    o1, _, _ = S.attention(qa, ka, va, kc, vc, L - 1, 8, 2, 64, 0.125, 16, 1)
    o2, _, _ = N.attention(qa, ka, va, kc, vc, L - 1, 8, 2, 64, 0.125, 0, 1)
    np.savez_compressed(OUT / "attention.npz", q=qa, k=ka, v=va, kc=kc, vc=vc, out_strict=o0, out_window16_strict=o1,
                        out_native=o2, kc_after=kc0, vc_after=vc0)
    # GLU
    g = synth.random_activations(1000, seed=21) * 4.0
    u = synth.random_activations(1000, seed=22)
    np.savez_compressed(OUT / "glu.npz", g=g, u=u, swiglu_strict=S.glu(g, u), geglu_strict=S.glu(g, u, True))
    # embedding rows
    emb = {}
    for t in (Q8_0, Q6_K, BF16):
        e = synth.random_weights(t, 10, 512, seed=23 + t)
        emb[f"w_{t}"] = e
        emb[f"rows_{t}"] = np.stack([S.embed(e, t, r, 512, s) for r in (0, 3, 9) for s in (1.0, 22.627417)])
    np.savez_compressed(OUT / "embed.npz", **emb)
    print("golden vectors written to", OUT)


if __name__ == "__main__":
    main()
