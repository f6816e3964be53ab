"""Host side of the tensor-parallel engine, on CPU: the exchange-region
handles travel between the ranks in rank order (gloo, world size 2), and the
header declares the tensor-parallel entry points the library exports."""
import datetime
import os
import socket

import pytest

torch = pytest.importorskip("torch")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    import torch.distributed as dist
    from gncx_b200.streamer import torch_exchange
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        blob = bytes([rank]) * 64
        q.put((rank, torch_exchange(blob)))
    finally:
        dist.destroy_process_group()


def test_handle_exchange_in_rank_order():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        assert got[r] == [bytes([0]) * 64, bytes([1]) * 64]


def _share(lib, hp, tp, rank):
    import ctypes
    out = (ctypes.c_int32 * 6)()
    st = lib.gncx_engine_tp_share((ctypes.c_int32 * 6)(*hp), tp, rank, out)
    return st, list(out)


@pytest.mark.parametrize("hp", [(32, 8, 128, 4096, 12288, 151936), (16, 8, 128, 1024, 3072, 151936),
                                (4, 2, 64, 256, 512, 4000)])
def test_tp_shares_cover_the_model(hp):
    """Every q/KV head, ffn row, model row and vocabulary row belongs to exactly
    one rank, in rank order; vocabulary slices start on 4-row boundaries."""
    from gncx_b200 import core
    lib = core.load()
    nh, nkv, hd, dim, ffn, vocab = hp
    for tp in (1, 2, 4, 8):
        if nkv % tp or dim % (4 * tp) or ffn % (32 * tp):
            assert _share(lib, hp, tp, 0)[0] == 1  # GNCX_ERR_INVALID_ARG
            continue
        shares = [_share(lib, hp, tp, r) for r in range(tp)]
        assert all(st == 0 for st, _ in shares)
        s = [o for _, o in shares]
        assert sum(o[0] for o in s) == nh and sum(o[1] for o in s) == nkv
        assert sum(o[2] for o in s) == ffn and sum(o[3] for o in s) == dim
        assert s[0][4] == 0 and all(s[r][4] + s[r][5] == s[r + 1][4] for r in range(tp - 1))
        assert s[-1][4] + s[-1][5] == vocab and all(o[4] % 4 == 0 and o[5] > 0 for o in s)
        assert all(o[0] % o[1] == 0 and o[0] // o[1] == nh // nkv for o in s)  # whole GQA groups per rank


def test_tp_share_rejects_bad_sizes():
    from gncx_b200 import core
    lib = core.load()
    hp = (32, 8, 128, 4096, 12288, 151936)
    assert _share(lib, hp, 3, 0)[0] == 1   # 8 KV heads over 3 ranks
    assert _share(lib, hp, 16, 0)[0] == 1  # more ranks than the exchange supports
    assert _share(lib, hp, 2, 2)[0] == 1   # rank out of range


def test_tp_entry_points_declared_and_exported():
    from pathlib import Path
    from gncx_b200 import core
    hdr = (Path(__file__).resolve().parents[1] / "include" / "gncx_llm_core.h").read_text()
    for name in ("gncx_engine_create_tp", "gncx_engine_tp_handle", "gncx_engine_tp_connect", "gncx_engine_tp_share"):
        assert name + "(" in hdr
        assert name in core._SIGS
    assert "#define GNCX_TP_HANDLE_BYTES 64" in hdr
