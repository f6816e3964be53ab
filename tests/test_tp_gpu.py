"""Tensor-parallel engine on 2 GPUs (one process per GPU, launched with
torch.distributed.run): the same prompt, forward_token steps and greedy
generate give logits and token ids identical, bit for bit, to the 1-GPU
engine, in both attention modes.  A rank that stops taking part makes the
other rank's call fail with GNCX_ERR_TIMEOUT instead of hanging.
Skipped on a box with fewer than 2 GPUs."""
import json
import os
import signal
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from gncx_b200 import gguf
from gncx_b200.core import Q4_K, Q8_0

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

ROOT = Path(__file__).resolve().parents[1]
TINY = dict(n_layers=3, dim=256, n_heads=4, n_kv=2, head_dim=64, ffn=512, vocab=4000, eps=1e-6, rope_base=1e6)


def _need_gpus(n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _launch(n, args, timeout=300, extra_env=None):
    """Run under torch.distributed.run in a session of its own, so that on a
    timeout the launcher and all its ranks end together."""
    env = dict(os.environ, PYTHONPATH=str(ROOT), NCCL_NVLS_ENABLE="0", **(extra_env or {}))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}", "--master-addr",
           "127.0.0.1", "--master-port", str(_port()), *args]
    p = subprocess.Popen(cmd, cwd=ROOT, env=env, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                         start_new_session=True)
    try:
        out, err = p.communicate(timeout=timeout)
    except subprocess.TimeoutExpired:
        os.killpg(p.pid, signal.SIGKILL)  # the process group this test started
        out, err = p.communicate()
    return subprocess.CompletedProcess(cmd, p.returncode, out, err)


def _tp_run(tmp_path, model, n, exact, outsplit=False):
    out = tmp_path / f"tp{n}_{int(exact)}_{int(outsplit)}.npz"
    args = ["-m", "gncx_b200.tp_run", str(model), "--prompt-len", "37", "--steps", "5", "--new", "24", "--seed", "3",
            "--out", str(out)] + (["--exact"] if exact else [])
    r = _launch(n, args, extra_env={"GNCX_TP_OUTSPLIT": "1"} if outsplit else None)
    assert r.returncode == 0, (r.stdout[-4000:], r.stderr[-4000:])
    z = np.load(out)
    info = json.loads(str(z["info"]))
    assert info["ranks_agree"] and info["tp"] == n
    return z["logits"], z["ids"]


@pytest.mark.parametrize("wtype,exact,outsplit", [(Q4_K, True, False), (Q8_0, False, False), (Q4_K, True, True)])
def test_tp2_matches_one_gpu(tmp_path, wtype, exact, outsplit):
    """Logits of the prefill and of every forward step, and the greedy stream
    (each rank's penalized maximum over its vocabulary slice, swapped as
    (value, id) pairs), equal the 1-GPU engine's; also with attn_output and
    ffn_down split by rows in decode (GNCX_TP_OUTSPLIT=1)."""
    _need_gpus(2)
    model = gguf.write_random_model(tmp_path / "tiny.gguf", TINY, seed=5, wtype=wtype)
    l1, i1 = _tp_run(tmp_path, model, 1, exact)
    l2, i2 = _tp_run(tmp_path, model, 2, exact, outsplit)
    assert np.all(np.isfinite(l1)) and len(i1) == 24
    assert np.array_equal(l1, l2)
    assert np.array_equal(i1, i2)


def test_tp_stalled_rank_times_out(tmp_path):
    _need_gpus(2)
    model = gguf.write_random_model(tmp_path / "tiny.gguf", TINY, seed=5, wtype=Q8_0)
    r = _launch(2, [str(ROOT / "tests" / "tp_stall_rank.py"), str(model)])
    assert r.returncode == 0, (r.stdout[-4000:], r.stderr[-4000:])
    assert "rank0 status 5" in r.stdout  # GNCX_ERR_TIMEOUT
