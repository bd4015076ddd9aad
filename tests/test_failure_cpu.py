"""A rank that leaves between steps (world size 2, gloo, on the CPU).

Both ranks run one sharded step (the all-gather of their per-shard lists
that the multi-GPU search makes, xvec_b200.sharded.exchange); then rank 1
exits, with nothing of its own in flight.  Rank 0's next step must end with
an error within the process group's short timeout instead of waiting for
ever (the reference ends a search on ctx.Err(), internal/core/topk.go:130).
The failure is made on the host; no GPU is involved."""
import multiprocessing as mp
import os
import socket
import time

import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, q):
    import datetime

    import torch
    import torch.distributed as dist

    from xvec_b200.sharded import exchange

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=5))
    keys = torch.arange(6, dtype=torch.int64).view(2, 3) + 10 * rank
    scores = torch.zeros((2, 3), dtype=torch.float32)
    counts = torch.full((2,), 3, dtype=torch.int32)
    all_k, _, _ = exchange(keys, scores, counts)
    q.put(("step1", rank, all_k.shape[0]))
    if rank == 1:
        # Leaves between steps: nothing in flight, the process ends.
        q.close()
        q.join_thread()
        os._exit(0)
    time.sleep(0.5)
    t0 = time.time()
    try:
        exchange(keys, scores, counts)
        q.put(("step2", rank, "completed", time.time() - t0))
    except Exception as e:  # noqa: BLE001 — any error ends the step, which is the point
        q.put(("step2", rank, type(e).__name__, time.time() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


def test_rank_leaving_between_steps_ends_the_next_step_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank waited for ever"
    msgs = [q.get(timeout=10) for _ in range(3)]
    assert sorted(m[1] for m in msgs if m[0] == "step1") == [0, 1]
    step2 = [m for m in msgs if m[0] == "step2"]
    assert len(step2) == 1
    _, rank, outcome, secs = step2[0]
    assert rank == 0
    assert outcome != "completed"
    assert secs < 60
