"""GNCXStreamer: the reference orchestrator's interface over the B200 engine.

Mirrors lua/gncx_streamer.lua (``GNCXStreamer.new``, ``forward_token``,
``prefill``, ``sample``, ``generate``) with token ids in place of the
tokenizer, which is out of scope here.  All compute runs in the CUDA engine of
libgncx_llm_core.so; this class only marshals arguments.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from . import core


TP_HANDLE_BYTES = 64


def torch_exchange(blob: bytes) -> list:
    """All ranks' `blob`s in rank order over the default torch.distributed group."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, blob)
    return out


class GNCXStreamer:
    """tp_size > 1: this process is rank tp_rank of a tensor-parallel engine on
    the current (or `device`) GPU; `exchange(bytes) -> [bytes per rank]` passes
    the exchange-region handles between the ranks (default: torch.distributed)."""

    def __init__(self, model_path: str | Path, max_seq_len: int = 4096, device: int | None = None,
                 exact_attention: bool = False, tp_rank: int = 0, tp_size: int = 1, exchange=None):
        self.lib = core.load()
        if device is not None:
            if self.lib.gncx_set_device(int(device)) != 0:
                core.check(self.lib)
        self.tp_rank, self.tp_size = int(tp_rank), int(tp_size)
        self.handle = self.lib.gncx_engine_create_tp(str(model_path).encode(), int(max_seq_len), self.tp_rank,
                                                     self.tp_size)
        if not self.handle:
            raise core.GncxError(1, f"could not load {model_path} on the GPU (see stderr)")
        if self.tp_size > 1:
            mine = (ctypes.c_uint8 * TP_HANDLE_BYTES)()
            self._check(self.lib.gncx_engine_tp_handle(self.handle, mine))
            blobs = (exchange or torch_exchange)(bytes(mine))
            if len(blobs) != self.tp_size or any(len(b) != TP_HANDLE_BYTES for b in blobs):
                raise core.GncxError(1, "tensor-parallel handle exchange returned the wrong number of handles")
            allh = (ctypes.c_uint8 * (TP_HANDLE_BYTES * self.tp_size)).from_buffer_copy(b"".join(blobs))
            st = self.lib.gncx_engine_tp_connect(self.handle, allh)
            # all ranks connect or none does: no rank may write into a peer that gave up
            oks = (exchange or torch_exchange)(bytes([st == 0]))
            if st or not all(b == b"\x01" for b in oks):
                msg = (self.lib.gncx_engine_error(self.handle) or b"").decode()
                self.close()
                raise core.GncxError(st or 1, "tensor-parallel connect failed on " +
                                     ("this rank: " + msg if st else "another rank"))
        hp = (ctypes.c_int32 * 12)()
        self.lib.gncx_engine_hparams(self.handle, hp)
        (self.n_layers, self.embed_dim, self.n_heads, self.n_kv_heads, self.head_dim, self.ffn_dim, self.vocab_size,
         self.max_seq_len, self.eos_id, self.arch, self.embd_type, self.qk_norm) = list(hp)
        self.set_exact_attention(exact_attention)

    def set_exact_attention(self, on: bool) -> None:
        """Exact serial softmax (the reference's summation order; bit-exact up to
        expf rounding) or the split-KV softmax (default, ~1e-6 relative)."""
        self.lib.gncx_engine_set_exact(self.handle, 1 if on else 0)

    # -- lifecycle --------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.gncx_engine_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, st: int) -> None:
        if st:
            raise core.GncxError(st, (self.lib.gncx_engine_error(self.handle) or b"").decode())

    # -- lua/gncx_streamer.lua:759-965 -----------------------------------------
    def forward_token(self, token_id: int, pos: int) -> np.ndarray:
        out = np.empty(self.vocab_size, np.float32)
        self._check(self.lib.gncx_engine_forward_token(self.handle, int(token_id), int(pos),
                                                       out.ctypes.data_as(ctypes.c_void_p)))
        return out

    # -- lua/gncx_streamer.lua:968-1208 ----------------------------------------
    def prefill(self, token_ids) -> np.ndarray:
        ids = np.ascontiguousarray(token_ids, dtype=np.int32)
        out = np.empty(self.vocab_size, np.float32)
        self._check(self.lib.gncx_engine_prefill(self.handle, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                                 ids.size, out.ctypes.data_as(ctypes.c_void_p)))
        return out

    # -- lua/gncx_streamer.lua:1229-1273 ---------------------------------------
    def sample(self, recent_tokens=(), repeat_penalty: float = 1.15) -> int:
        """Penalized greedy argmax over the logits of the last forward/prefill
        (computed on the device; both of the reference's branches are greedy)."""
        rec = np.ascontiguousarray(recent_tokens, dtype=np.int32)
        buf = (ctypes.c_int32 * max(1, rec.size))(*rec.tolist())
        tok = self.lib.gncx_sample_greedy(ctypes.c_void_p(self.lib.gncx_engine_logits(self.handle)),
                                          self.vocab_size, buf, rec.size, float(repeat_penalty))
        if tok < 0:
            core.check(self.lib)
        return int(tok)

    # -- lua/gncx_streamer.lua:1276-1311 ---------------------------------------
    def generate_ids(self, prompt_ids, max_new_tokens: int = 256, repeat_penalty: float = 1.15,
                     eos_id: int | None = None) -> list[int]:
        ids = np.ascontiguousarray(prompt_ids, dtype=np.int32)
        out = (ctypes.c_int32 * max(1, max_new_tokens))()
        eos = self.eos_id if eos_id is None else eos_id
        n = self.lib.gncx_engine_generate(self.handle, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), ids.size,
                                          int(max_new_tokens), float(repeat_penalty), int(eos), out)
        if n < 0:
            self._check(-n)
        return list(out[:n])

    def persistent_decode(self) -> bool:
        """True when decode steps run as one persistent kernel per token."""
        return self.lib.gncx_engine_decode_path(self.handle) == 1

    def timing(self) -> dict:
        p, d, n = ctypes.c_double(), ctypes.c_double(), ctypes.c_int32()
        self.lib.gncx_engine_timing(self.handle, ctypes.byref(p), ctypes.byref(d), ctypes.byref(n))
        return {"prefill_ms": p.value, "decode_ms": d.value, "decode_steps": n.value}


GNCXEngine = GNCXStreamer  # lua/gncx_streamer.lua:1226
