"""Python handle on the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use
this module, and only as the checker / baseline, never as the product path.

Two oracles are exposed with the same numpy-level API:
  * :class:`Oracle` -- the plain-C restatement in gncx_oracle.c
    (``oracle/_build/liboracle.so``);
  * :class:`RefLib` -- the reference's own sources compiled here
    (``oracle/_ref/libgncx_ref_strict.so`` is the strict-IEEE pin,
    ``oracle/_ref/libgncx_ref.so`` the as-shipped flags), called through its
    exported C ABI exactly as its own ctypes harness does
    (verify_gncx_fixes.py:25-117).
"""
from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
from ctypes import POINTER, c_char_p, c_double, c_float, c_int32, c_size_t, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "liboracle.so"
REF_STRICT_SO = HERE / "_ref" / "libgncx_ref_strict.so"
REF_NATIVE_SO = HERE / "_ref" / "libgncx_ref.so"
REF_SPR_SO = HERE / "_ref" / "libgncx_ref_spr.so"
# CPU flags a -march=sapphirerapids build may use in compiler-generated code
_SPR_FLAGS = {"avx512f", "avx512dq", "avx512cd", "avx512bw", "avx512vl", "avx512ifma", "avx512vbmi", "avx512_vbmi2",
              "avx512_vnni", "avx512_bitalg", "avx512_vpopcntdq", "avx512_bf16", "avx512_fp16", "amx_tile",
              "amx_int8", "amx_bf16", "avx_vnni", "gfni", "vaes", "vpclmulqdq", "bmi2", "fma", "f16c", "movbe"}


def _host_flags() -> set:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("flags"):
                return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def timing_reference_so() -> Path:
    """The reference build for timing on this host: the -march=sapphirerapids
    one (what the shipped -march=native gives there) when the host has every
    extension it may use, else the portable AVX2 one."""
    if REF_SPR_SO.exists() and _SPR_FLAGS <= _host_flags():
        return REF_SPR_SO
    return REF_NATIVE_SO


def reference_source() -> Path | None:
    """Where the reference's sources lie, if anywhere: ``$GNCX_REFERENCE``, else
    the ``reference_path`` that BASELINE.json at the repository root names.
    None when neither exists (the GPU box carries only the prebuilt _ref/)."""
    cand = os.environ.get("GNCX_REFERENCE")
    if not cand:
        try:
            import json
            cand = json.loads((HERE.parent / "BASELINE.json").read_text()).get("reference_path")
        except (OSError, ValueError):
            cand = None
    if not cand:
        return None
    p = Path(cand)
    return p if (p / "csrc" / "gncx_llm_kernels.cpp").exists() else None


ACT_DTYPE = np.dtype([("d", "<f4"), ("sum_q", "<i4"), ("sum_lo", "<i4"), ("sum_hi", "<i4"), ("qs", "i1", (32,))])


def build(with_reference: bool = True) -> None:
    """Build liboracle.so and, when the reference sources exist, oracle/_ref."""
    if shutil.which("make") is None:
        return
    subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)
    src = reference_source() if with_reference else None
    if src is not None:
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={src}"], check=True)


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


class Oracle:
    """The C restatement."""

    def __init__(self, path: Path = ORACLE_SO):
        if not Path(path).exists():
            build(with_reference=False)
        L = ctypes.CDLL(str(path))
        self.lib = L
        L.orc_matvec.argtypes = [c_void_p, c_int32, c_void_p, c_int32, c_int32, c_void_p]
        L.orc_matbatch.argtypes = [c_void_p, c_int32, c_void_p, c_int32, c_int32, c_int32, c_void_p]
        L.orc_lm_head.argtypes = [c_void_p, c_int32, c_void_p, c_int32, c_int32, c_float, c_void_p]
        L.orc_act_quantize.argtypes = [c_void_p, c_int32, c_void_p]
        L.orc_dequant_row.argtypes = [c_void_p, c_int32, c_int32, c_void_p]
        L.orc_rmsnorm.argtypes = [c_void_p, c_void_p, c_int32, c_float, c_void_p]
        L.orc_rmsnorm_heads.argtypes = [c_void_p, c_void_p, c_int32, c_int32, c_float]
        L.orc_rope_table.argtypes = [c_int32, c_int32, c_float, c_void_p, c_void_p, c_void_p]
        L.orc_rope.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32, c_float]
        L.orc_attention_step.argtypes = [c_void_p] * 5 + [c_int32] * 4 + [c_float, c_int32, c_int32, c_void_p]
        L.orc_swiglu.argtypes = [c_void_p, c_void_p, c_int32, c_void_p]
        L.orc_geglu.argtypes = [c_void_p, c_void_p, c_int32, c_void_p]
        L.orc_embed_row.argtypes = [c_void_p, c_int32, c_int32, c_int32, c_float, c_void_p]
        L.orc_sample_greedy.argtypes = [c_void_p, c_int32, c_void_p, c_int32, c_double]
        L.orc_sample_greedy.restype = c_int32
        L.orc_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.orc_fp16_to_fp32.restype = c_float

    def matvec(self, w: np.ndarray, t: int, x, out_dim: int) -> np.ndarray:
        x = _f32(x)
        y = np.zeros(out_dim, np.float32)
        self.lib.orc_matvec(_ptr(np.ascontiguousarray(w)), t, _ptr(x), x.size, out_dim, _ptr(y))
        return y

    def matbatch(self, w: np.ndarray, t: int, xb, out_dim: int) -> np.ndarray:
        xb = _f32(xb)
        B, n = xb.shape
        y = np.zeros((B, out_dim), np.float32)
        self.lib.orc_matbatch(_ptr(np.ascontiguousarray(w)), t, _ptr(xb), B, n, out_dim, _ptr(y))
        return y

    def lm_head(self, w, t, h, vocab, softcap=0.0):
        h = _f32(h)
        y = np.zeros(vocab, np.float32)
        self.lib.orc_lm_head(_ptr(np.ascontiguousarray(w)), t, _ptr(h), h.size, vocab, softcap, _ptr(y))
        return y

    def act_quantize(self, x) -> np.ndarray:
        x = _f32(x)
        out = np.zeros(x.size // 32, ACT_DTYPE)
        self.lib.orc_act_quantize(_ptr(x), x.size, _ptr(out))
        return out

    def dequant_row(self, row: np.ndarray, t: int, n: int) -> np.ndarray:
        out = np.zeros(n, np.float32)
        self.lib.orc_dequant_row(_ptr(np.ascontiguousarray(row)), t, n, _ptr(out))
        return out

    def rmsnorm(self, x, w, eps) -> np.ndarray:
        x, w = _f32(x), _f32(w)
        out = np.zeros_like(x)
        self.lib.orc_rmsnorm(_ptr(x), _ptr(w), x.size, eps, _ptr(out))
        return out

    def rmsnorm_heads(self, v, w, n_heads, head_dim, eps) -> np.ndarray:
        v = _f32(v).copy()
        self.lib.orc_rmsnorm_heads(_ptr(v), _ptr(None if w is None else _f32(w)), n_heads, head_dim, eps)
        return v

    def rope_table(self, pos, hd, base, ff=None):
        c = np.zeros(hd // 2, np.float32)
        s = np.zeros(hd // 2, np.float32)
        self.lib.orc_rope_table(pos, hd, base, _ptr(None if ff is None else _f32(ff)), _ptr(c), _ptr(s))
        return c, s

    def rope(self, q, k, n_heads, n_kv, hd, pos, base, ff=None):
        q = None if q is None else _f32(q).copy()
        k = None if k is None else _f32(k).copy()
        self.lib.orc_rope(_ptr(q), _ptr(k), _ptr(None if ff is None else _f32(ff)), n_heads, n_kv, hd, pos, base)
        return q, k

    def attention(self, q, k, v, kc, vc, pos, n_heads, n_kv, hd, scale, window=0, write_kv=1):
        kc, vc = _f32(kc).copy(), _f32(vc).copy()
        out = np.zeros(n_heads * hd, np.float32)
        self.lib.orc_attention_step(_ptr(_f32(q)), _ptr(None if k is None else _f32(k)),
                                    _ptr(None if v is None else _f32(v)), _ptr(kc), _ptr(vc), pos, n_heads, n_kv,
                                    hd, scale, window, write_kv, _ptr(out))
        return out, kc, vc

    def glu(self, g, u, gelu=False):
        g, u = _f32(g), _f32(u)
        out = np.zeros_like(g)
        (self.lib.orc_geglu if gelu else self.lib.orc_swiglu)(_ptr(g), _ptr(u), g.size, _ptr(out))
        return out

    def embed(self, tensor, t, token, dim, scale=1.0):
        out = np.zeros(dim, np.float32)
        self.lib.orc_embed_row(_ptr(np.ascontiguousarray(tensor)), t, token, dim, scale, _ptr(out))
        return out

    def sample_greedy(self, logits, recent, penalty=1.15) -> int:
        logits = _f32(logits)
        r = np.ascontiguousarray(recent, dtype=np.int32)
        return int(self.lib.orc_sample_greedy(_ptr(logits), logits.size, _ptr(r), r.size, penalty))


class RefLib:
    """The reference library built from its sources, called through its C ABI."""

    def __init__(self, path: Path = REF_STRICT_SO):
        L = ctypes.CDLL(str(path))
        self.lib = L
        L.gncx_gla_map_readonly.restype = c_void_p
        L.gncx_gla_map_readonly.argtypes = [c_char_p, POINTER(c_size_t)]
        # fills the fp16 table and starts the pool (csrc/gncx_llm_kernels.cpp:327-329);
        # never unmapped (gncx_gla_unmap stops the pool, :392)
        self._h = L.gncx_gla_map_readonly(str(path).encode(), None)
        V = c_void_p
        L.gncx_xfold_universal_matvec.argtypes = [V, c_size_t, c_int32, V, V, c_int32, c_int32, V, V]
        L.gncx_xfold_universal_matbatch.argtypes = [V, c_size_t, c_int32, V, c_int32, c_int32, c_int32, V, V]
        L.gncx_universal_lm_head_logits.argtypes = [V, c_size_t, c_int32, V, c_int32, c_int32, c_float, V]
        L.gncx_rmsnorm_and_encode_4phase.argtypes = [V, V, c_size_t, c_int32, c_float, c_int32, V, V, V]
        L.gncx_rmsnorm_inplace_heads.argtypes = [V, V, c_size_t, c_int32, c_int32, c_int32, c_float]
        L.gncx_apply_rope_xor11_ext.argtypes = [V, V, V, V, c_size_t, c_int32, c_int32, c_int32, c_int32, c_int32,
                                                c_float]
        L.gncx_mqa_attention_step_ext.argtypes = [V] * 5 + [c_int32] * 4 + [c_float, c_int32, c_int32, V]
        L.gncx_swiglu_activation.argtypes = [V, V, c_int32, V]
        L.gncx_geglu_activation.argtypes = [V, V, c_int32, V]
        for n in ("q8_0", "q6_k", "bf16"):
            getattr(L, f"gncx_fetch_token_embedding_{n}").argtypes = [V, c_size_t, c_int32, c_int32, c_float, V]

    def matvec(self, w, t, x, out_dim):
        x = _f32(x)
        y = np.zeros(out_dim, np.float32)
        self.lib.gncx_xfold_universal_matvec(_ptr(np.ascontiguousarray(w)), 0, t, _ptr(x), None, x.size, out_dim,
                                             _ptr(y), None)
        return y

    def matbatch(self, w, t, xb, out_dim):
        xb = _f32(xb)
        B, n = xb.shape
        y = np.zeros((B, out_dim), np.float32)
        self.lib.gncx_xfold_universal_matbatch(_ptr(np.ascontiguousarray(w)), 0, t, _ptr(xb), B, n, out_dim, _ptr(y),
                                               None)
        return y

    def lm_head(self, w, t, h, vocab, softcap=0.0):
        h = _f32(h)
        y = np.zeros(vocab, np.float32)
        self.lib.gncx_universal_lm_head_logits(_ptr(np.ascontiguousarray(w)), 0, t, _ptr(h), h.size, vocab, softcap,
                                               _ptr(y))
        return y

    def rmsnorm(self, x, w, eps):
        x, w = _f32(x), _f32(w)
        out = np.zeros_like(x)
        self.lib.gncx_rmsnorm_and_encode_4phase(_ptr(x), _ptr(w), 0, x.size, eps, 0, _ptr(out), None, None)
        return out

    def rmsnorm_heads(self, v, w, n_heads, head_dim, eps):
        v = _f32(v).copy()
        wp = None if w is None else _f32(w)
        self.lib.gncx_rmsnorm_inplace_heads(_ptr(v), _ptr(wp), 0, 0 if w is None else 1, n_heads, head_dim, eps)
        return v

    def rope(self, q, k, n_heads, n_kv, hd, pos, base, ff=None):
        q = None if q is None else _f32(q).copy()
        k = None if k is None else _f32(k).copy()
        ffa = None if ff is None else _f32(ff)
        self.lib.gncx_apply_rope_xor11_ext(_ptr(q), _ptr(k), None, _ptr(ffa), 0, 0 if ff is None else 1, n_heads,
                                           n_kv, hd, pos, base)
        return q, k

    def attention(self, q, k, v, kc, vc, pos, n_heads, n_kv, hd, scale, window=0, write_kv=1):
        kc, vc = _f32(kc).copy(), _f32(vc).copy()
        out = np.zeros(n_heads * hd, np.float32)
        self.lib.gncx_mqa_attention_step_ext(_ptr(_f32(q)), _ptr(None if k is None else _f32(k)),
                                             _ptr(None if v is None else _f32(v)), _ptr(kc), _ptr(vc), pos, n_heads,
                                             n_kv, hd, scale, window, write_kv, _ptr(out))
        return out, kc, vc

    def glu(self, g, u, gelu=False):
        g, u = _f32(g), _f32(u)
        out = np.zeros_like(g)
        fn = self.lib.gncx_geglu_activation if gelu else self.lib.gncx_swiglu_activation
        fn(_ptr(g), _ptr(u), g.size, _ptr(out))
        return out

    def embed(self, tensor, t, token, dim, scale=1.0):
        out = np.zeros(dim, np.float32)
        name = {8: "q8_0", 14: "q6_k", 30: "bf16"}[t]
        getattr(self.lib, f"gncx_fetch_token_embedding_{name}")(_ptr(np.ascontiguousarray(tensor)), 0, token, dim,
                                                                  scale, _ptr(out))
        return out


def ref_build_flags(so: Path) -> str:
    """The compiler and flags a reference library under _ref/ was built with."""
    f = Path(str(so) + ".flags")
    return f.read_text().strip() if f.exists() else "unknown"


def reference_available(strict: bool = True) -> bool:
    return (REF_STRICT_SO if strict else REF_NATIVE_SO).exists()


class OracleModel:
    """Whole-model CPU oracle (oracle/gncx_oracle_model.c) over a GGUF file:
    the reference orchestrator's forward_token / prefill / generate, with the
    kernels of the reference library itself (``ref_lib``) or of the C
    restatement (``ref_lib=None``)."""

    NT = 11  # tensors per layer in the descriptor

    class _Desc(ctypes.Structure):
        _fields_ = [("n_layers", c_int32), ("dim", c_int32), ("n_heads", c_int32), ("n_kv", c_int32),
                    ("head_dim", c_int32), ("ffn_dim", c_int32), ("vocab", c_int32), ("max_seq", c_int32),
                    ("eps", c_float), ("rope_base", c_float), ("softcap", c_float), ("arch", c_int32),
                    ("base", c_void_p), ("tok_embd_off", ctypes.c_uint64), ("tok_embd_type", c_int32),
                    ("out_norm_off", ctypes.c_uint64), ("off", c_void_p), ("typ", c_void_p)]

    def __init__(self, gguf_path, max_seq: int, ref_lib: Path | None = REF_STRICT_SO, drive_lib=None):
        """drive_lib: a loaded library with the reference's entry points whose
        kernels need memory they can reach (the B200 library): the orchestration
        then runs its kernels, with the model file mapped through the library's
        gncx_gla_map_readonly and the vectors from its gncx_ram_alloc, as the
        Lua streamer sets them up (lua/gncx_streamer.lua:462-464, :539-662)."""
        from gncx_b200 import gguf as _gguf
        o = Oracle()
        L = o.lib
        L.orc_model_create.restype = c_void_p
        L.orc_model_create.argtypes = [c_void_p, c_char_p]
        L.orc_model_create_ex.restype = c_void_p
        L.orc_model_create_ex.argtypes = [c_void_p, c_char_p, c_int32]
        L.orc_model_destroy.argtypes = [c_void_p]
        L.orc_model_forward.restype = c_void_p
        L.orc_model_forward.argtypes = [c_void_p, c_int32, c_int32]
        L.orc_model_prefill.restype = c_void_p
        L.orc_model_prefill.argtypes = [c_void_p, c_void_p, c_int32]
        L.orc_model_generate.restype = c_int32
        L.orc_model_generate.argtypes = [c_void_p, c_void_p, c_int32, c_int32, c_double, c_int32, c_void_p]
        self.lib = L
        g = _gguf.read(gguf_path)
        hp = _gguf.model_desc(g)
        self.hp = hp
        if drive_lib is not None:
            size = ctypes.c_size_t()
            handle = drive_lib.gncx_gla_map_readonly(str(gguf_path).encode(), ctypes.byref(size))
            base = drive_lib.gncx_gla_get_base_ptr(handle) if handle else None
            if not base:
                raise RuntimeError("gncx_gla_map_readonly failed")
            self.mm = None
            base_ptr = c_void_p(base)
        else:
            self.mm = np.memmap(gguf_path, dtype=np.uint8, mode="r")
            base_ptr = self.mm.ctypes.data_as(c_void_p)
        names = ["attn_norm", "attn_q", "attn_k", "attn_v", "attn_q_norm", "attn_k_norm", "attn_output", "ffn_norm",
                 "ffn_gate", "ffn_up", "ffn_down"]
        off = np.full((hp["n_layers"], self.NT), np.iinfo(np.uint64).max, dtype=np.uint64)
        typ = np.zeros((hp["n_layers"], self.NT), dtype=np.int32)
        for l in range(hp["n_layers"]):
            for i, n in enumerate(names):
                t = g.tensors.get(f"blk.{l}.{n}.weight")
                if t is not None:
                    off[l, i] = t.abs_offset
                    typ[l, i] = t.ggml_type
        self._off, self._typ = off, typ
        emb = g.tensors["token_embd.weight"]
        arch = {"qwen": 0, "llam": 1, "gemm": 2}.get(hp["arch"][:4], 0)
        d = self._Desc(hp["n_layers"], hp["dim"], hp["n_heads"], hp["n_kv"], hp["head_dim"], hp["ffn"], hp["vocab"],
                       int(max_seq), hp["eps"], hp["rope_base"], hp["softcap"], arch,
                       base_ptr, emb.abs_offset, emb.ggml_type,
                       g.tensors["output_norm.weight"].abs_offset, off.ctypes.data_as(c_void_p),
                       typ.ctypes.data_as(c_void_p))
        if drive_lib is not None:
            lib_path = str(ref_lib).encode()
            self.kind = "drop-in"
            self.h = L.orc_model_create_ex(ctypes.byref(d), lib_path, 1)
        else:
            lib_path = str(ref_lib).encode() if ref_lib is not None and Path(ref_lib).exists() else None
            self.kind = "reference" if lib_path else "port"
            self.h = L.orc_model_create(ctypes.byref(d), lib_path)
        if not self.h:
            raise RuntimeError("oracle model creation failed")

    def forward_token(self, tok: int, pos: int) -> np.ndarray:
        p = self.lib.orc_model_forward(self.h, tok, pos)
        return np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(c_float)), (self.hp["vocab"],)).copy()

    def prefill(self, ids) -> np.ndarray:
        a = np.ascontiguousarray(ids, dtype=np.int32)
        p = self.lib.orc_model_prefill(self.h, a.ctypes.data_as(c_void_p), a.size)
        return np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(c_float)), (self.hp["vocab"],)).copy()

    def generate(self, prompt, max_new: int, penalty: float = 1.15, eos: int = -1) -> list[int]:
        a = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(1, max_new), np.int32)
        n = self.lib.orc_model_generate(self.h, a.ctypes.data_as(c_void_p), a.size, max_new, penalty, eos,
                                        out.ctypes.data_as(c_void_p))
        return out[:n].tolist()

    def close(self):
        if self.h:
            self.lib.orc_model_destroy(self.h)
            self.h = None
