"""GGUF v3 reading and writing, plus random-init decoder models.

The reader follows the reference loader (lua/gncx_gguf.lua:223-306): metadata
KV pairs, tensor records {name, dims, ggml_type, relative offset}, data section
aligned to ``general.alignment`` (default 32); a tensor's absolute offset is
data_offset + relative offset and its byte size comes from the block table
(:50-66).  The writer produces files that loader accepts, in native block
layout, used to build the random-init models of the benchmark configurations.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from .core import BLOCK, F32, Q4_K, Q6_K, row_bytes

# GGUF value types (lua/gncx_gguf.lua:15-29)
U8, I8, U16, I16, U32, I32, F32V, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32V: "<f", BOOL: "<?", U64: "<Q",
           I64: "<q", F64: "<d"}


@dataclass
class TensorInfo:
    name: str
    dims: list
    ggml_type: int
    rel_offset: int
    abs_offset: int = 0
    n_elements: int = 0
    nbytes: int = 0


@dataclass
class GGUF:
    path: Path
    version: int
    metadata: dict = field(default_factory=dict)
    tensors: dict = field(default_factory=dict)
    data_offset: int = 0

    def meta(self, key, default=None):
        return self.metadata.get(key, default)


class _Reader:
    def __init__(self, buf):
        self.b = buf
        self.p = 0

    def take(self, fmt):
        v = struct.unpack_from(fmt, self.b, self.p)[0]
        self.p += struct.calcsize(fmt)
        return v

    def string(self):
        n = self.take("<Q")
        s = bytes(self.b[self.p:self.p + n]).decode("utf-8", errors="replace")
        self.p += n
        return s

    def value(self, t):
        if t in _SCALAR:
            return self.take(_SCALAR[t])
        if t == STRING:
            return self.string()
        if t == ARRAY:
            et = self.take("<I")
            n = self.take("<Q")
            if et == STRING:
                return [self.string() for _ in range(n)]
            if et in _SCALAR:
                fmt = _SCALAR[et]
                sz = struct.calcsize(fmt)
                arr = np.frombuffer(self.b, dtype=np.dtype(fmt), count=n, offset=self.p).tolist()
                self.p += sz * n
                return arr
            return [self.value(et) for _ in range(n)]
        raise ValueError(f"unknown GGUF value type {t}")


def read(path: str | Path) -> GGUF:
    path = Path(path)
    with open(path, "rb") as f:
        head = f.read(64 << 20)  # metadata (incl. a 151936-entry vocab) fits well below this
    r = _Reader(head)
    if bytes(head[:4]) != b"GGUF":
        raise ValueError(f"{path}: not a GGUF file")
    r.p = 4
    g = GGUF(path=path, version=r.take("<I"))
    n_tensors = r.take("<Q")
    n_kv = r.take("<Q")
    for _ in range(n_kv):
        key = r.string()
        t = r.take("<I")
        g.metadata[key] = r.value(t)
    for _ in range(n_tensors):
        name = r.string()
        nd = r.take("<I")
        dims = [r.take("<Q") for _ in range(nd)]
        t = r.take("<I")
        off = r.take("<Q")
        g.tensors[name] = TensorInfo(name, dims, t, off)
    align = g.metadata.get("general.alignment", 32)
    align = align if isinstance(align, int) and align > 0 else 32
    g.data_offset = (r.p + align - 1) // align * align
    for ti in g.tensors.values():
        n = int(np.prod(ti.dims)) if ti.dims else 1
        ti.n_elements = n
        be, bb = BLOCK.get(ti.ggml_type, (1, 0))
        ti.nbytes = (n // be) * bb
        ti.abs_offset = g.data_offset + ti.rel_offset
    return g


# ---------------------------------------------------------------- writer
def _w_str(f, s: str):
    b = s.encode()
    f.write(struct.pack("<Q", len(b)))
    f.write(b)


def _w_value(f, v):
    if isinstance(v, bool):
        f.write(struct.pack("<I", BOOL)); f.write(struct.pack("<?", v))
    elif isinstance(v, int):
        f.write(struct.pack("<I", U32 if 0 <= v < 2**32 else I64))
        f.write(struct.pack("<I" if 0 <= v < 2**32 else "<q", v))
    elif isinstance(v, float):
        f.write(struct.pack("<I", F32V)); f.write(struct.pack("<f", v))
    elif isinstance(v, str):
        f.write(struct.pack("<I", STRING)); _w_str(f, v)
    elif isinstance(v, (list, tuple)):
        f.write(struct.pack("<I", ARRAY))
        if v and isinstance(v[0], str):
            f.write(struct.pack("<I", STRING)); f.write(struct.pack("<Q", len(v)))
            for s in v:
                _w_str(f, s)
        else:
            f.write(struct.pack("<I", I32)); f.write(struct.pack("<Q", len(v)))
            f.write(np.asarray(v, dtype="<i4").tobytes())
    else:
        raise TypeError(type(v))


def write(path: str | Path, metadata: dict, tensors: list, alignment: int = 32) -> None:
    """tensors: list of (name, dims[ne0, ne1...], ggml_type, payload: np.uint8 array or callable->array)."""
    path = Path(path)
    metadata = dict(metadata)
    metadata.setdefault("general.alignment", alignment)
    infos = []
    off = 0
    for name, dims, t, payload in tensors:
        n = int(np.prod(dims))
        be, bb = BLOCK[t]
        nbytes = (n // be) * bb
        infos.append((name, dims, t, off, nbytes, payload))
        off = (off + nbytes + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(b"GGUF")
        f.write(struct.pack("<IQQ", 3, len(infos), len(metadata)))
        for k, v in metadata.items():
            _w_str(f, k)
            _w_value(f, v)
        for name, dims, t, o, _, _ in infos:
            _w_str(f, name)
            f.write(struct.pack("<I", len(dims)))
            for d in dims:
                f.write(struct.pack("<Q", d))
            f.write(struct.pack("<IQ", t, o))
        pos = f.tell()
        f.write(b"\0" * ((pos + alignment - 1) // alignment * alignment - pos))
        base = f.tell()
        for name, dims, t, o, nbytes, payload in infos:
            here = f.tell() - base
            f.write(b"\0" * (o - here))
            data = payload() if callable(payload) else payload
            data = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
            if data.size != nbytes:
                raise ValueError(f"{name}: {data.size} bytes, expected {nbytes}")
            f.write(data.tobytes())


# ---------------------------------------------------------------- random-init decoders
CONFIGS = {
    # Qwen3-0.6B shape (benchmark configuration 4)
    "qwen3-0.6b": dict(n_layers=28, dim=1024, n_heads=16, n_kv=8, head_dim=128, ffn=3072, vocab=151936,
                       eps=1e-6, rope_base=1e6),
    # 8B shape (benchmark configuration 5)
    "qwen3-8b": dict(n_layers=36, dim=4096, n_heads=32, n_kv=8, head_dim=128, ffn=12288, vocab=151936,
                     eps=1e-6, rope_base=1e6),
    # the 8B layer shape with two layers: profiling captures of single decode
    # kernels (a few hundred MB on the device instead of ~5 GB)
    "qwen3-8b-2l": dict(n_layers=2, dim=4096, n_heads=32, n_kv=8, head_dim=128, ffn=12288, vocab=151936,
                        eps=1e-6, rope_base=1e6),
}


def write_random_model(path: str | Path, cfg: dict | str, seed: int = 0, wtype: int = Q4_K,
                       embd_type: int = Q6_K, vocab: int | None = None, n_layers: int | None = None) -> Path:
    """A random-init Qwen3-architecture GGUF (all linear layers `wtype`, tied
    `embd_type` embedding / LM head, F32 norm gains of 1.0)."""
    from .synth import random_weights_fast
    c = dict(CONFIGS[cfg]) if isinstance(cfg, str) else dict(cfg)
    if vocab is not None:
        c["vocab"] = vocab
    if n_layers is not None:
        c["n_layers"] = n_layers
    L, D, H, KV, HD, F, V = (c[k] for k in ("n_layers", "dim", "n_heads", "n_kv", "head_dim", "ffn", "vocab"))
    arch = "qwen3"
    meta = {
        "general.architecture": arch,
        f"{arch}.block_count": L,
        f"{arch}.embedding_length": D,
        f"{arch}.attention.head_count": H,
        f"{arch}.attention.head_count_kv": KV,
        f"{arch}.attention.key_length": HD,
        f"{arch}.attention.layer_norm_rms_epsilon": float(c["eps"]),
        f"{arch}.rope.freq_base": float(c["rope_base"]),
        f"{arch}.feed_forward_length": F,
        f"{arch}.context_length": 40960,
        "tokenizer.ggml.tokens": [f"<t{i}>" for i in range(V)],
        "tokenizer.ggml.eos_token_id": 151645 if V > 151645 else V - 1,
    }
    ones = lambda n: np.ones(n, np.float32)  # noqa: E731
    k = [0]

    def rnd(t, out_dim, in_dim):
        k[0] += 1
        s = seed * 1000 + k[0]
        return lambda: random_weights_fast(t, out_dim, in_dim, seed=s)

    tensors = [("token_embd.weight", [D, V], embd_type, rnd(embd_type, V, D)),
               ("output_norm.weight", [D], F32, ones(D))]
    for layer in range(L):
        p = f"blk.{layer}."
        tensors += [
            (p + "attn_norm.weight", [D], F32, ones(D)),
            (p + "attn_q.weight", [D, H * HD], wtype, rnd(wtype, H * HD, D)),
            (p + "attn_k.weight", [D, KV * HD], wtype, rnd(wtype, KV * HD, D)),
            (p + "attn_v.weight", [D, KV * HD], wtype, rnd(wtype, KV * HD, D)),
            (p + "attn_q_norm.weight", [HD], F32, ones(HD)),
            (p + "attn_k_norm.weight", [HD], F32, ones(HD)),
            (p + "attn_output.weight", [H * HD, D], wtype, rnd(wtype, D, H * HD)),
            (p + "ffn_norm.weight", [D], F32, ones(D)),
            (p + "ffn_gate.weight", [D, F], wtype, rnd(wtype, F, D)),
            (p + "ffn_up.weight", [D, F], wtype, rnd(wtype, F, D)),
            (p + "ffn_down.weight", [F, D], wtype, rnd(wtype, D, F)),
        ]
    write(path, meta, tensors)
    return Path(path)


def model_desc(g: GGUF) -> dict:
    """Hyper-parameters the orchestrator reads (lua/gncx_streamer.lua:344-441)."""
    arch = str(g.meta("general.architecture", "qwen3"))
    H = int(g.meta(f"{arch}.attention.head_count", 0))
    D = int(g.meta(f"{arch}.embedding_length", 0))
    return dict(
        arch=arch,
        n_layers=int(g.meta(f"{arch}.block_count", 0)),
        dim=D,
        n_heads=H,
        n_kv=int(g.meta(f"{arch}.attention.head_count_kv", H)),
        head_dim=int(g.meta(f"{arch}.attention.key_length", D // H if H else 0)),
        ffn=int(g.meta(f"{arch}.feed_forward_length", 0)),
        vocab=len(g.meta("tokenizer.ggml.tokens", [])),
        eps=float(g.meta(f"{arch}.attention.layer_norm_rms_epsilon", 1e-6)),
        rope_base=float(g.meta(f"{arch}.rope.freq_base", 10000.0)),
        softcap=float(g.meta(f"{arch}.final_logit_softcapping", 0.0)),
        eos=int(g.meta("tokenizer.ggml.eos_token_id", 151645)),
    )
