"""gncx_b200 -- B200-native (sm_100a) build of GNC-X's decode/prefill hot path.

The product is the CUDA library ``libgncx_llm_core.so`` behind the C ABI in
``include/gncx_llm_core.h`` (drop-in names of csrc/gncx_llm_kernels.cpp).  This
package holds its sources (``csrc/``), the build step (:mod:`gncx_b200.build`),
the ctypes binding (:mod:`gncx_b200.core`), GGUF reading/writing
(:mod:`gncx_b200.gguf`), the model engine front end (:mod:`gncx_b200.streamer`)
and seeded synthetic inputs (:mod:`gncx_b200.synth`).
"""
from .core import BF16, F16, F32, Q4_0, Q4_K, Q6_K, Q8_0, GncxError, check, load, row_bytes  # noqa: F401

__all__ = ["load", "check", "row_bytes", "GncxError", "F32", "F16", "Q4_0", "Q8_0", "Q4_K", "Q6_K", "BF16"]
