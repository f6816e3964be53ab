"""The drop-in boundary driven the way the reference's Lua streamer drives it.

The reference orchestration (forward_token / prefill / generate of
lua/gncx_streamer.lua, restated in oracle/gncx_oracle_model.c) is bound to
this library's exported entry points instead of the reference's: the model
file is mapped with gncx_gla_map_readonly, the vectors and KV caches come
from gncx_ram_alloc, every call is synchronous and the residual adds run on
the host in between -- exactly what the unchanged Lua code would do through
LuaJIT.  Its logits and greedy token stream must match the same
orchestration over the reference's own kernels.
"""
import numpy as np
import pytest

from gncx_b200 import core, gguf
from gncx_b200.core import Q6_K, Q8_0

pytestmark = pytest.mark.gpu
pytest.importorskip("torch")

TINY = dict(n_layers=3, dim=256, n_heads=4, n_kv=2, head_dim=64, ffn=512, vocab=3000, eps=1e-6, rope_base=1e6)


def rel(a, b):
    return float(np.max(np.abs(a - b)) / max(1e-30, np.max(np.abs(b))))


@pytest.mark.parametrize("wtype", [Q8_0, Q6_K])
def test_reference_orchestration_over_the_dropin_library(tmp_path, wtype):
    from oracle.oracle import REF_STRICT_SO, OracleModel
    lib = core.load()
    lib.gncx_set_synchronous(1)
    lib.gncx_set_exact_attention(1)  # the reference's softmax order
    path = gguf.write_random_model(tmp_path / "tiny.gguf", TINY, seed=9, wtype=wtype)
    prompt = np.random.default_rng(wtype).integers(0, TINY["vocab"], 29).tolist()
    ref = OracleModel(path, 96, REF_STRICT_SO)
    dut = OracleModel(path, 96, core.LIB_PATH, drive_lib=lib)
    try:
        assert dut.kind == "drop-in"
        lr, lg = ref.prefill(prompt), dut.prefill(prompt)
        core.check(lib)
        assert np.all(np.isfinite(lg)) and rel(lg, lr) <= 1e-3
        ids = list(prompt)
        for _ in range(6):
            ids.append(int(np.argmax(lr)))
            lr, lg = ref.forward_token(ids[-1], len(ids) - 1), dut.forward_token(ids[-1], len(ids) - 1)
            assert rel(lg, lr) <= 1e-3
        want = ref.generate(prompt, 48, 1.15, -1)
        got = dut.generate(prompt, 48, 1.15, -1)
        core.check(lib)
        assert len(want) == 48 and got == want
        assert len(set(want)) > 8
    finally:
        ref.close()
        dut.close()
        lib.gncx_set_exact_attention(0)
