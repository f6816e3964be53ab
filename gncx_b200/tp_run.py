"""Tensor-parallel prefill + greedy decode, one process per GPU.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m gncx_b200.tp_run MODEL.gguf --prompt-len 128 --new 64 --out result.npz

Every rank loads its share of MODEL (GNCXStreamer with tp_rank/tp_size), the
ranks swap their exchange-region handles over torch.distributed (gloo: the
data path is the library's own NVLink all-gather, not a torch collective),
then all ranks run the same calls.  Rank 0 checks that every rank produced
the same logits and ids and writes them, with the device timings, to --out.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import numpy as np


def run(model: str, prompt_len: int, new: int, steps: int, exact: bool, seed: int, max_seq: int,
        penalty: float = 1.15):
    import torch.distributed as dist

    from .streamer import GNCXStreamer

    rank, world = dist.get_rank(), dist.get_world_size()
    local = int(os.environ.get("LOCAL_RANK", rank))
    eng = GNCXStreamer(model, max_seq_len=max_seq, device=local, exact_attention=exact, tp_rank=rank, tp_size=world)
    try:
        prompt = np.random.default_rng(seed).integers(0, eng.vocab_size, prompt_len).tolist()
        logits = [eng.prefill(prompt)]
        ids = list(prompt)
        for _ in range(steps):  # forward_token with plain argmax feeding the next step
            ids.append(int(np.argmax(logits[-1])))
            logits.append(eng.forward_token(ids[-1], len(ids) - 1))
        gen = eng.generate_ids(prompt, new, penalty, eos_id=-1) if new > 0 else []
        timing = eng.timing()
    finally:
        # No rank unmaps its exchange region while another may still write into
        # it: a rank that failed waits here for the others' (bounded) calls.
        dist.barrier()
        eng.close()
    mine = {"logits": np.stack(logits), "ids": np.asarray(gen, np.int32)}
    allr = [None] * world
    dist.all_gather_object(allr, mine)
    same = all(np.array_equal(r["logits"], mine["logits"]) and np.array_equal(r["ids"], mine["ids"]) for r in allr)
    return mine, timing, same


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("model")
    ap.add_argument("--prompt-len", type=int, default=128)
    ap.add_argument("--new", type=int, default=64, help="tokens of the greedy generate loop")
    ap.add_argument("--steps", type=int, default=0, help="forward_token calls after the prefill")
    ap.add_argument("--exact", action="store_true", help="exact serial softmax in attention")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--max-seq", type=int, default=0)
    ap.add_argument("--out", default="")
    a = ap.parse_args(argv)
    import torch.distributed as dist
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    try:
        max_seq = a.max_seq or (a.prompt_len + max(a.new, a.steps) + 8)
        res, timing, same = run(a.model, a.prompt_len, a.new, a.steps, a.exact, a.seed, max_seq)
        if dist.get_rank() == 0:
            info = {"tp": dist.get_world_size(), "ranks_agree": bool(same), **timing}
            if a.out:
                np.savez(a.out, logits=res["logits"], ids=res["ids"], info=json.dumps(info))
            print(json.dumps(info), flush=True)
        dist.barrier()
        return 0 if same else 1
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    raise SystemExit(main())
