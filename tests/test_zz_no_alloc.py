"""gncx_mqa_attention_step_noalloc (decode attention whose scratch is a fixed
array in the library) against the regular entry point
gncx_mqa_attention_step_ext on the same inputs, two calls in a row.

Collected last on purpose: it must pass both alone in a fresh process and
after every other test has used the library.
"""
import ctypes

import numpy as np
import pytest

from gncx_b200 import core

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

NH, NKV, HD = 32, 8, 128
GNCX_ERR_CAPACITY = 8


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _run_case(ctx, window, device=0):
    lib = core.load()
    dev = torch.device("cuda", device)
    torch.cuda.set_device(dev)
    g = torch.Generator(device="cpu").manual_seed(ctx + window)
    kc = torch.randn(ctx * NKV * HD, generator=g).to(dev)
    vc = torch.randn(ctx * NKV * HD, generator=g).to(dev)
    q = torch.randn(NH * HD, generator=g).to(dev)
    k = torch.randn(NKV * HD, generator=g).to(dev)
    v = torch.randn(NKV * HD, generator=g).to(dev)
    scale = float(np.float32(1.0 / np.sqrt(HD)))
    pos = ctx - 1
    torch.cuda.synchronize()

    # the regular entry point on its own copy of the caches
    kc_a, vc_a = kc.clone(), vc.clone()
    y_ref = torch.zeros(NH * HD, device=dev)
    torch.cuda.synchronize()
    lib.gncx_set_exact_attention(0)
    lib.gncx_mqa_attention_step_ext(_p(q), _p(k), _p(v), _p(kc_a), _p(vc_a), pos, NH, NKV, HD, scale, window, 1,
                                    _p(y_ref))
    assert lib.gncx_sync() == 0
    core.check(lib)

    # the allocation-free one, twice in a row, on a stream of the caller's
    kc_b, vc_b = kc.clone(), vc.clone()
    outs = [torch.zeros(NH * HD, device=dev) for _ in range(2)]
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()
    # The first call on a device is its one-time set-up: it looks up the fixed
    # array, which (with lazy module loading) is when the 4 MiB array itself
    # is placed on the device.  The calls after it must not change free memory.
    setup = torch.zeros(NH * HD, device=dev)
    torch.cuda.synchronize()
    st = lib.gncx_mqa_attention_step_noalloc(_p(q), _p(k), _p(v), _p(kc_b), _p(vc_b), pos, NH, NKV, HD, scale, window,
                                             1, _p(setup), ctypes.c_void_p(stream.cuda_stream))
    assert st == 0, (lib.gncx_last_error_message() or b"").decode()
    stream.synchronize()
    free_before = torch.cuda.mem_get_info(dev)[0]
    for y in outs:
        st = lib.gncx_mqa_attention_step_noalloc(_p(q), _p(k), _p(v), _p(kc_b), _p(vc_b), pos, NH, NKV, HD, scale,
                                                 window, 1, _p(y), ctypes.c_void_p(stream.cuda_stream))
        assert st == 0, (lib.gncx_last_error_message() or b"").decode()
    stream.synchronize()
    free_after = torch.cuda.mem_get_info(dev)[0]
    assert free_after == free_before  # no device memory was allocated by the calls

    # Both entry points launch the same kernels with the same split geometry
    # on the same inputs, so the outputs agree bit for bit.
    for y in outs:
        assert torch.all(torch.isfinite(y))
        assert torch.equal(y, y_ref)
    row = slice(pos * NKV * HD, ctx * NKV * HD)
    assert torch.equal(kc_b[row], k) and torch.equal(vc_b[row], v)
    assert torch.equal(kc_b, kc_a) and torch.equal(vc_b, vc_a)


@pytest.mark.parametrize("ctx,window", [(3001, 0), (3001, 1000), (1, 0)])
def test_noalloc_attention_matches_regular(ctx, window):
    _run_case(ctx, window)


def test_noalloc_attention_second_device():
    """A second GPU in the same process gets its own set-up (array address and
    kernel shared-memory limits are per device)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    try:
        _run_case(3001, 0, device=0)
        _run_case(3001, 0, device=1)
    finally:
        torch.cuda.set_device(0)
        core.load().gncx_set_device(0)


def test_noalloc_attention_rejects_oversized_window():
    lib = core.load()
    dev = torch.device("cuda", 0)
    small = torch.zeros(NKV * HD, device=dev)
    y = torch.zeros(NH * HD, device=dev)
    lib.gncx_clear_error()
    # a 40,000-position window needs ~5 MB of records: refused before any GPU work
    st = lib.gncx_mqa_attention_step_noalloc(_p(small), None, None, _p(small), _p(small), 39999, NH, NKV, HD, 0.088,
                                             0, 0, _p(y), None)
    assert st == GNCX_ERR_CAPACITY
    msg = (lib.gncx_last_error_message() or b"").decode()
    assert "scratch" in msg and "4194304" in msg
    lib.gncx_clear_error()
