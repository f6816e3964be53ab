"""Helper of tests/test_tp_gpu.py (run under torch.distributed.run, 2 ranks):
rank 1 connects and then takes no part (it keeps its memory mapped and waits
on the host); rank 0's prefill must come back with GNCX_ERR_TIMEOUT from the
library's bounded wait.  No kernel or collective of rank 1 is in flight."""
import datetime
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch.distributed as dist  # noqa: E402

from gncx_b200 import core  # noqa: E402
from gncx_b200.streamer import GNCXStreamer  # noqa: E402


def main():
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    rank = dist.get_rank()
    eng = GNCXStreamer(sys.argv[1], max_seq_len=64, device=int(os.environ["LOCAL_RANK"]), tp_rank=rank, tp_size=2)
    if rank == 0:
        try:
            eng.prefill([1, 2, 3, 4])
            status = 0
        except core.GncxError as e:
            status = e.code
        print(f"rank0 status {status}", flush=True)
    dist.barrier()  # rank 1 unmaps its region only after rank 0's call returned
    eng.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
