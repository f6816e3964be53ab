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


def test_tp_entry_points_declared_and_exported():
    from pathlib import Path
    from gncx_b200 import core
    hdr = (Path(__file__).resolve().parents[1] / "include" / "gncx_llm_core.h").read_text()
    for name in ("gncx_engine_create_tp", "gncx_engine_tp_handle", "gncx_engine_tp_connect"):
        assert name + "(" in hdr
        assert name in core._SIGS
    assert "#define GNCX_TP_HANDLE_BYTES 64" in hdr
