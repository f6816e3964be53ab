"""CPU tests of the model-level pieces: GGUF writing/reading and the
whole-model oracle (its orchestration restated from lua/gncx_streamer.lua is
checked against itself when driven by the reference's compiled kernels vs by
the C restatement)."""
import numpy as np
import pytest

from gncx_b200 import gguf
from gncx_b200.core import F32, Q4_K, Q6_K, Q8_0, row_bytes

TINY = dict(n_layers=2, dim=256, n_heads=4, n_kv=2, head_dim=64, ffn=512, vocab=1000, eps=1e-6, rope_base=1e6)


def test_gguf_roundtrip(tmp_path):
    path = gguf.write_random_model(tmp_path / "m.gguf", TINY, seed=1)
    g = gguf.read(path)
    hp = gguf.model_desc(g)
    assert hp["n_layers"] == 2 and hp["dim"] == 256 and hp["vocab"] == 1000 and hp["head_dim"] == 64
    assert hp["n_heads"] == 4 and hp["n_kv"] == 2 and hp["ffn"] == 512
    assert np.float32(hp["eps"]) == np.float32(1e-6) and hp["rope_base"] == 1e6
    assert g.data_offset % 32 == 0
    t = g.tensors["blk.1.attn_k.weight"]
    assert t.ggml_type == Q4_K and t.dims == [256, 128] and t.nbytes == 128 * row_bytes(Q4_K, 256)
    assert t.abs_offset % 32 == 0
    raw = np.fromfile(path, dtype=np.uint8)
    e = g.tensors["token_embd.weight"]
    assert e.ggml_type == Q6_K and e.abs_offset + e.nbytes <= raw.size
    n = g.tensors["output_norm.weight"]
    assert n.ggml_type == F32
    assert np.all(raw[n.abs_offset:n.abs_offset + 1024].view(np.float32) == 1.0)


def test_gguf_metadata_types(tmp_path):
    meta = {"general.architecture": "qwen3", "a.int": 7, "a.float": 0.5, "a.str": "x", "a.list": [1, 2, 3],
            "a.strs": ["p", "q"], "a.bool": True}
    w = np.zeros(2 * row_bytes(Q8_0, 32), np.uint8)
    gguf.write(tmp_path / "k.gguf", meta, [("w", [32, 2], Q8_0, w)])
    g = gguf.read(tmp_path / "k.gguf")
    for k, v in meta.items():
        assert g.metadata[k] == v
    assert g.tensors["w"].nbytes == w.size


@pytest.mark.parametrize("wtype", [Q4_K, Q8_0])
def test_oracle_model_matches_reference_kernels(tmp_path, wtype):
    from oracle.oracle import REF_STRICT_SO, OracleModel
    if not REF_STRICT_SO.exists():
        pytest.skip("reference library not built here")
    path = gguf.write_random_model(tmp_path / "m.gguf", TINY, seed=2, wtype=wtype)
    prompt = np.random.default_rng(3).integers(0, 1000, 24).tolist()
    a = OracleModel(path, 96, None)
    b = OracleModel(path, 96, REF_STRICT_SO)
    assert a.kind == "port" and b.kind == "reference"
    assert np.array_equal(a.prefill(prompt), b.prefill(prompt))
    assert np.array_equal(a.forward_token(5, 24), b.forward_token(5, 24))
    assert a.generate(prompt, 40, 1.15, -1) == b.generate(prompt, 40, 1.15, -1)
    a.close()
    b.close()


def test_oracle_model_single_token_prefill_is_forward(tmp_path):
    """prefill of one token is forward_token(id, 0) (lua/gncx_streamer.lua:971-973)."""
    from oracle.oracle import OracleModel
    path = gguf.write_random_model(tmp_path / "m.gguf", TINY, seed=4)
    m = OracleModel(path, 16, None)
    a = m.prefill([17])
    b = m.forward_token(17, 0)
    assert np.array_equal(a, b)
    m.close()


def test_orchestration_over_a_librarys_own_memory(tmp_path):
    """The drop-in harness of tests/test_dropin_orchestration_gpu.py, checked
    on CPU with the reference library itself as the driven library: the model
    file mapped by its gncx_gla_map_readonly, every vector and KV cache from
    its gncx_ram_alloc arena -- the same logits and stream as the plain run."""
    import ctypes
    from oracle.oracle import REF_STRICT_SO, OracleModel
    if not REF_STRICT_SO.exists():
        pytest.skip("reference library not built here (oracle/_ref)")
    ref = ctypes.CDLL(str(REF_STRICT_SO))
    ref.gncx_gla_map_readonly.restype = ctypes.c_void_p
    ref.gncx_gla_map_readonly.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_size_t)]
    ref.gncx_gla_get_base_ptr.restype = ctypes.c_void_p
    ref.gncx_gla_get_base_ptr.argtypes = [ctypes.c_void_p]
    cfg = dict(n_layers=2, dim=256, n_heads=4, n_kv=2, head_dim=64, ffn=512, vocab=1500, eps=1e-6, rope_base=1e6)
    path = gguf.write_random_model(tmp_path / "m.gguf", cfg, seed=4, wtype=Q8_0)
    prompt = np.random.default_rng(2).integers(0, cfg["vocab"], 13).tolist()
    a = OracleModel(path, 48, REF_STRICT_SO)
    b = OracleModel(path, 48, REF_STRICT_SO, drive_lib=ref)
    try:
        assert b.kind == "drop-in"
        assert np.array_equal(a.prefill(prompt), b.prefill(prompt))
        assert np.array_equal(a.forward_token(prompt[-1], 13), b.forward_token(prompt[-1], 13))
        assert a.generate(prompt, 12, 1.15, -1) == b.generate(prompt, 12, 1.15, -1)
    finally:
        a.close()
        b.close()
