"""Host-side failure detection for the multi-rank path (gloo, CPU): a rank that
leaves before a collective makes the survivor's next collective fail within the
process group's short timeout instead of hanging."""

import os
import socket
import sys
import time
from datetime import timedelta

import torch


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=5))
    dist.barrier()
    if rank == 1:
        os._exit(0)  # leaves between steps, without joining the next exchange
    time.sleep(0.5)
    out = torch.empty(4)
    start = time.time()
    try:
        dist.all_to_all_single(out, torch.arange(4.0), output_split_sizes=[2, 2],
                               input_split_sizes=[2, 2])
        q.put(("no error", time.time() - start))
    except Exception as exc:  # noqa: BLE001 - any backend error is the detection
        q.put((type(exc).__name__, time.time() - start))
    sys.exit(0)


def test_peer_exit_is_detected_not_hung():
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
        assert p.exitcode is not None, "a rank hung"
    kind, seconds = q.get(timeout=10)
    assert kind != "no error"
    assert seconds < 60
