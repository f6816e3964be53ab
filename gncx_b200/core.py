"""ctypes binding of the C ABI in ``include/gncx_llm_core.h``.

This mirrors how the reference's own harness binds its library
(verify_gncx_fixes.py:66-117 of omega-Core-Dev/gnc-x) and what
lua/gncx_streamer.lua:16-252 declares with ffi.cdef: the reference-named entry
points keep their names and argument order; the pointers they take are device
pointers (``torch.Tensor.data_ptr()`` of CUDA tensors) instead of host RAM.

There is no CPU path: loading works anywhere, but every compute call on a
machine without a GPU records GNCX_ERR_NO_DEVICE and :func:`check` raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_double, c_float, c_int32, c_size_t, c_uint8, c_uint64, c_void_p
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libgncx_llm_core.so"

# ggml type ids (lua/gncx_gguf.lua:31-47)
F32, F16, Q4_0, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 2, 8, 12, 14, 30
TYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K", BF16: "BF16"}
# (elements per block, bytes per block) -- lua/gncx_gguf.lua:50-66
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}
ACT_BLOCK_BYTES = 48

STATUS = {
    0: "OK", 1: "INVALID_ARG", 2: "UNALIGNED", 3: "CUDA", 4: "NO_DEVICE", 5: "TIMEOUT",
    6: "NOT_DEVICE_ACCESSIBLE", 7: "OUT_OF_MEMORY", 8: "CAPACITY",
}


def row_bytes(ggml_type: int, n: int) -> int:
    be, bb = BLOCK[ggml_type]
    return (n // be) * bb


class GncxError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"gncx error {code} ({STATUS.get(code, '?')}): {message}")
        self.code = code


class GNCXCompactToken(ctypes.Structure):
    _pack_ = 1
    _fields_ = [("phase_2bit", c_uint8), ("diag_d", c_uint8), ("abs_delta", ctypes.c_uint16)]


class GNCXTelemetryStats(ctypes.Structure):
    _pack_ = 1
    _fields_ = [("total_macs_equivalent", c_uint64), ("zero_origin_cancellations", c_uint64),
                ("zero_weight_skips", c_uint64), ("xfold_bucket_merges", c_uint64)]


P = c_void_p  # every buffer argument travels as a raw address
_SIGS = {
    # reference-named (csrc/gncx_llm_kernels.cpp line of each in include/gncx_llm_core.h)
    "gncx_gla_map_readonly": (c_void_p, [c_char_p, POINTER(c_size_t)]),
    "gncx_gla_get_base_ptr": (c_void_p, [c_void_p]),
    "gncx_gla_unmap": (None, [c_void_p]),
    "gncx_gla_prefetch_range": (None, [P, c_size_t, c_size_t]),
    "gncx_ram_alloc_colored": (c_void_p, [c_size_t, c_uint8, c_uint8, c_uint8]),
    "gncx_ram_alloc": (c_void_p, [c_size_t]),
    "gncx_ram_get_ptr": (c_void_p, [c_void_p]),
    "gncx_ram_get_ddr3_bank": (c_uint8, [c_void_p]),
    "gncx_ram_get_l1_set": (c_uint8, [c_void_p]),
    "gncx_ram_free": (None, [c_void_p]),
    "gncx_ram_copy_chunk": (None, [c_void_p, c_size_t, P, c_size_t, c_size_t]),
    "gncx_fetch_token_embedding_q8_0": (None, [P, c_size_t, c_int32, c_int32, c_float, P]),
    "gncx_fetch_token_embedding_q6_k": (None, [P, c_size_t, c_int32, c_int32, c_float, P]),
    "gncx_fetch_token_embedding_bf16": (None, [P, c_size_t, c_int32, c_int32, c_float, P]),
    "gncx_rmsnorm_and_encode_4phase": (None, [P, P, c_size_t, c_int32, c_float, c_int32, P, P, P]),
    "gncx_rmsnorm_inplace_heads": (None, [P, P, c_size_t, c_int32, c_int32, c_int32, c_float]),
    "gncx_xfold_universal_matvec": (None, [P, c_size_t, c_int32, P, P, c_int32, c_int32, P, P]),
    "gncx_xfold_q4_0_matvec": (None, [P, c_size_t, P, P, c_int32, c_int32, P, P]),
    "gncx_xfold_universal_matbatch": (None, [P, c_size_t, c_int32, P, c_int32, c_int32, c_int32, P, P]),
    "gncx_xfold_q4_0_matbatch": (None, [P, c_size_t, P, c_int32, c_int32, c_int32, P, P]),
    "gncx_universal_lm_head_logits": (None, [P, c_size_t, c_int32, P, c_int32, c_int32, c_float, P]),
    "gncx_q8_0_lm_head_logits": (None, [P, c_size_t, P, c_int32, c_int32, P]),
    "gncx_apply_rope_xor11_ext": (None, [P, P, P, P, c_size_t, c_int32, c_int32, c_int32, c_int32, c_int32, c_float]),
    "gncx_apply_rope_xor11": (None, [P, P, P, c_int32, c_int32, c_int32, c_int32, c_float]),
    "gncx_mqa_attention_step_ext": (None, [P, P, P, P, P, c_int32, c_int32, c_int32, c_int32, c_float, c_int32,
                                           c_int32, P]),
    "gncx_mqa_attention_step": (None, [P, P, P, P, P, c_int32, c_int32, c_int32, c_int32, P]),
    "gncx_geglu_activation": (None, [P, P, c_int32, P]),
    "gncx_swiglu_activation": (None, [P, P, c_int32, P]),
    # added entry points
    "gncx_last_error": (c_int32, []),
    "gncx_last_error_message": (c_char_p, []),
    "gncx_clear_error": (None, []),
    "gncx_sync": (c_int32, []),
    "gncx_set_stream": (None, [c_void_p]),
    "gncx_get_stream": (c_void_p, []),
    "gncx_set_synchronous": (None, [c_int32]),
    "gncx_set_weight_prefetch": (None, [c_int32]),
    "gncx_set_exact_attention": (None, [c_int32]),
    "gncx_engine_set_exact": (c_int32, [c_void_p, c_int32]),
    "gncx_device_count": (c_int32, []),
    "gncx_set_device": (c_int32, [c_int32]),
    "gncx_device_alloc": (c_void_p, [c_size_t]),
    "gncx_device_free": (None, [c_void_p]),
    "gncx_memcpy": (c_int32, [P, P, c_size_t]),
    "gncx_act_quantize": (c_int32, [P, c_int32, c_int32, P]),
    "gncx_matvec_preq": (c_int32, [P, c_size_t, c_int32, P, c_int32, c_int32, P]),
    "gncx_dequantize_rows": (c_int32, [P, c_size_t, c_int32, c_int32, c_int32, P]),
    "gncx_sample_greedy": (c_int32, [P, c_int32, POINTER(c_int32), c_int32, c_double]),
    "gncx_trace_enable": (c_int32, [P, P, ctypes.c_uint32]),
    "gncx_attention_prefill": (c_int32, [P, P, P, c_int32, c_int32, c_int32, c_int32, c_int32, c_float, P]),
    "gncx_mqa_attention_step_noalloc": (c_int32, [P, P, P, P, P, c_int32, c_int32, c_int32, c_int32, c_float,
                                                  c_int32, c_int32, P, P]),
    # model engine
    "gncx_engine_create": (c_void_p, [c_char_p, c_int32]),
    "gncx_engine_create_tp": (c_void_p, [c_char_p, c_int32, c_int32, c_int32]),
    "gncx_engine_tp_handle": (c_int32, [c_void_p, c_void_p]),
    "gncx_engine_tp_connect": (c_int32, [c_void_p, c_void_p]),
    "gncx_engine_tp_share": (c_int32, [POINTER(c_int32), c_int32, c_int32, POINTER(c_int32)]),
    "gncx_engine_destroy": (None, [c_void_p]),
    "gncx_engine_hparams": (c_int32, [c_void_p, POINTER(c_int32)]),
    "gncx_engine_error": (c_char_p, [c_void_p]),
    "gncx_engine_stream": (c_void_p, [c_void_p]),
    "gncx_engine_forward_token": (c_int32, [c_void_p, c_int32, c_int32, P]),
    "gncx_engine_prefill": (c_int32, [c_void_p, POINTER(c_int32), c_int32, P]),
    "gncx_engine_logits": (c_void_p, [c_void_p]),
    "gncx_engine_generate": (c_int32, [c_void_p, POINTER(c_int32), c_int32, c_int32, c_double, c_int32,
                                       POINTER(c_int32)]),
    "gncx_engine_timing": (c_int32, [c_void_p, POINTER(c_double), POINTER(c_double), POINTER(c_int32)]),
    "gncx_engine_decode_path": (c_int32, [c_void_p]),
}

_lib = None


def load(path: str | Path | None = None) -> ctypes.CDLL:
    """Load the in-tree CUDA library (raises if it has not been built)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    # GNCX_LIB names another build of the library (e.g. the tracing one)
    p = Path(path) if path else Path(os.environ.get("GNCX_LIB") or LIB_PATH)
    if not p.exists():
        raise FileNotFoundError(f"{p} is missing: build it with `python -m gncx_b200.build` "
                                "(this package has no CPU fallback)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def check(lib: ctypes.CDLL | None = None) -> None:
    """Raise GncxError if the library recorded an error; clears it."""
    lib = lib or load()
    code = lib.gncx_last_error()
    if code:
        msg = (lib.gncx_last_error_message() or b"").decode(errors="replace")
        lib.gncx_clear_error()
        raise GncxError(code, msg)


def bind_torch_stream(lib: ctypes.CDLL | None = None, device: int | None = None):
    """Make torch and the library enqueue on one stream.

    torch's default stream has handle 0, which the library reads as "use my
    own stream"; so a dedicated stream is created, made torch's current
    stream and handed to the library.  Returns the torch stream.
    """
    import torch

    lib = lib or load()
    if device is not None:
        torch.cuda.set_device(device)
    s = torch.cuda.Stream()
    torch.cuda.set_stream(s)
    lib.gncx_set_stream(ctypes.c_void_p(s.cuda_stream))
    check(lib)
    return s


def exported_symbols(lib: ctypes.CDLL | None = None) -> list[str]:
    lib = lib or load()
    return [n for n in _SIGS if getattr(lib, n, None) is not None]
