"""The C-ABI library loads, exports every entry point include/*.h declares,
and refuses to run without a GPU (there is no CPU fallback)."""
import ctypes
import re
from pathlib import Path

import pytest

from gncx_b200 import core

ROOT = Path(__file__).resolve().parents[1]


def declared_functions() -> list[str]:
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"\b(gncx_\w+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_reference_entry_points():
    names = set(declared_functions())
    # the reference symbols the hot path binds (lua/gncx_streamer.lua:16-252)
    for n in ["gncx_xfold_universal_matvec", "gncx_xfold_universal_matbatch", "gncx_xfold_q4_0_matvec",
              "gncx_xfold_q4_0_matbatch", "gncx_universal_lm_head_logits", "gncx_q8_0_lm_head_logits",
              "gncx_mqa_attention_step_ext", "gncx_mqa_attention_step", "gncx_apply_rope_xor11_ext",
              "gncx_apply_rope_xor11", "gncx_rmsnorm_and_encode_4phase", "gncx_rmsnorm_inplace_heads",
              "gncx_swiglu_activation", "gncx_geglu_activation", "gncx_fetch_token_embedding_q8_0",
              "gncx_fetch_token_embedding_q6_k", "gncx_fetch_token_embedding_bf16", "gncx_gla_map_readonly",
              "gncx_gla_get_base_ptr", "gncx_gla_unmap", "gncx_ram_alloc", "gncx_ram_copy_chunk", "gncx_ram_free"]:
        assert n in names, n


def test_library_exports_every_declared_symbol():
    lib = core.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_ctypes_signatures_cover_header():
    assert set(declared_functions()) <= set(core._SIGS), set(declared_functions()) - set(core._SIGS)


def test_reference_signature_arity_matches_reference_source():
    from oracle.oracle import reference_source
    root = reference_source()
    if root is None:
        pytest.skip("reference sources not present (set GNCX_REFERENCE)")
    src = root / "csrc" / "gncx_llm_kernels.cpp"
    text = src.read_text(errors="replace")
    for name in declared_functions():
        m = re.search(r"GNCX_LLM_API\s+[\w\s\*]+?\b" + name + r"\s*\((.*?)\)\s*\{", text, flags=re.S)
        if not m:
            continue  # added entry point, no reference counterpart
        params = re.sub(r"//[^\n]*", "", m.group(1))
        ref_args = [a for a in params.split(",") if a.strip()]
        assert len(core._SIGS[name][1]) == len(ref_args), name


def test_fails_loudly_without_gpu():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = core.load()
    lib.gncx_clear_error()
    x = (ctypes.c_float * 256)()
    y = (ctypes.c_float * 4)()
    w = (ctypes.c_uint8 * 4096)()
    lib.gncx_xfold_universal_matvec(w, 0, core.Q4_K, x, None, 256, 4, y, None)
    assert lib.gncx_last_error() == 4  # GNCX_ERR_NO_DEVICE
    with pytest.raises(core.GncxError):
        core.check(lib)
    assert lib.gncx_device_alloc(16) is None


def test_bench_reference_arm_prints_the_contract_line():
    """`bench.py --impl reference` (the reference's CPU matvec over the same
    Q4_K sweep) prints one JSON line with the keys the driver reads."""
    import json
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    r = subprocess.run([sys.executable, str(root / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       cwd=root, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [x for x in r.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] >= 3
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
