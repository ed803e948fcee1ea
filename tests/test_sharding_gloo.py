"""Multi-process host work queue (no GPU): two ranks over gloo / TCPStore on
127.0.0.1 claim independent leaf tasks, journal completion, re-run the tasks of
a rank that fails, and assemble results on rank 0."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from shear_b200 import sharding as S


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_plan_lpt_is_balanced_and_deterministic():
    costs = [S.leaf_cost(n) for n in (2048, 10, 700, 1500, 300, 300, 64, 900)]
    a = S.plan_lpt(costs, 3)
    assert a == S.plan_lpt(costs, 3)
    assert sorted(sum(a, [])) == list(range(len(costs)))
    loads = [sum(costs[i] for i in r) for r in a]
    assert max(loads) <= costs[0] + min(loads)


def _leaf_task(t):
    # Tiny deterministic leaf per task, solved with the CPU checker (this test
    # exercises the host queue, not the kernel).
    from oracle import oracle as O
    rng = np.random.default_rng(t)
    n = 20 + 7 * t
    x = rng.standard_normal((n, 24)).astype(np.float32)
    c, s, nr = O.quantize_sq8(x)
    ids, d = O.leaf_topk_sq8(c, s, nr, np.arange(n, dtype=np.uint32), np.arange(n, dtype=np.uint32), [0], [n], 3)
    return int(ids.astype(np.int64).sum())


def _worker(rank, world, port, ntasks, fail_rank, out_dir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=__import__("datetime").timedelta(seconds=60))
    costs = [S.leaf_cost(20 + 7 * t) for t in range(ntasks)]
    out = open(os.path.join(out_dir, f"res{rank}"), "w")

    def emit(t, v):  # the host reducer's side: results persist as they arrive
        out.write(f"{t} {v}\n")
        out.flush()

    try:
        q, res = S.run_sharded(store, rank, world, costs, _leaf_task, name="t",
                               fail_after=1 if rank == fail_rank else None, emit=emit)
    except RuntimeError:
        open(os.path.join(out_dir, f"failed{rank}"), "w").write("1")
        return
    if rank == 0:
        # the rank that created the store keeps it alive until everyone is done
        q.wait_exited(world)


def _run(tmp_path, fail_rank):
    world, ntasks = 2, 9
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, ntasks, fail_rank, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    got = {}
    for r in range(world):
        p = tmp_path / f"res{r}"
        if p.exists():
            for line in p.read_text().split("\n"):
                if line:
                    t, v = line.split()
                    assert int(t) not in got, "task ran twice"
                    got[int(t)] = int(v)
    return got, ntasks


def test_two_ranks_claim_every_task_once(tmp_path):
    got, n = _run(tmp_path, fail_rank=None)
    assert sorted(got) == list(range(n))
    assert got == {t: _leaf_task(t) for t in range(n)}


def test_failed_rank_tasks_are_rerun_by_survivor(tmp_path):
    got, n = _run(tmp_path, fail_rank=1)
    assert (tmp_path / "failed1").exists()
    assert sorted(got) == list(range(n))
    assert got == {t: _leaf_task(t) for t in range(n)}
