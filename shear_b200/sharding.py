"""Host work queue that spreads independent leaf / subtree tasks over the GPUs of one box.

Leaves and D1+ subtree tasks are independent (reference:
shear-core/src/algorithm/pipnn/rbc_partition.rs:15558-15600 processes each child
task alone), so the path shards with no collective on the data path: one
process per GPU, each claiming tasks from a shared queue and running them on its
own device; results go to the host reducer.  The queue lives in the
``torch.distributed`` store (TCPStore / FileStore): ``store.add`` is an atomic
fetch-and-add, so ranks claim tasks without a collective.

* ``plan_lpt`` -- static longest-processing-time assignment (cost = pairs),
  used when ranks must know their shard up front;
* ``StoreWorkQueue`` -- dynamic claiming in longest-first order, a completion
  journal (``done/<task>`` keys), and ``requeue_missing`` so that tasks claimed
  by a rank that failed are run again by the survivors (the journal also makes
  a multi-GPU run resumable at task granularity);
* ``run_sharded`` -- the per-rank driver loop: claim, run, journal, re-run the
  tasks of failed ranks; the rank that owns the store keeps it alive with
  ``wait_exited`` until every rank is done with it.
"""
from __future__ import annotations

import heapq
import time
from dataclasses import dataclass, field


def leaf_cost(rows: int) -> int:
    """Work of one leaf in candidate pairs (P/tessa_replay.rs:1087-1097)."""
    return rows * max(rows - 1, 0)


def plan_lpt(costs, world: int):
    """Greedy longest-processing-time assignment of tasks to `world` ranks.

    Returns a list of task-index lists, one per rank, each in descending cost
    order.  Deterministic: ties break by task index, then by rank.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0, r) for r in range(world)]
    heapq.heapify(heap)
    shards = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    return shards


@dataclass
class StoreWorkQueue:
    """Longest-first task queue shared by all ranks through a c10d store."""

    store: object
    costs: list
    name: str = "tessa"
    order: list = field(init=False)

    def __post_init__(self):
        self.order = sorted(range(len(self.costs)), key=lambda i: (-self.costs[i], i))

    def _k(self, suffix: str) -> str:
        return f"{self.name}/{suffix}"

    def claim(self):
        """Next task index, or None when the queue is drained."""
        slot = self.store.add(self._k("next"), 1) - 1
        return self.order[slot] if slot < len(self.order) else None

    def mark_done(self, task: int) -> None:
        self.store.set(self._k(f"done/{task}"), b"1")

    def is_done(self, task: int) -> bool:
        return self.store.check([self._k(f"done/{task}")])

    def missing(self):
        return [t for t in self.order if not self.is_done(t)]

    def requeue_missing(self, rank: int, world: int, run_task):
        """Run the tasks nobody finished (their rank failed), split by rank.

        Every surviving rank calls this after the main loop; each takes the
        missing tasks congruent to its position among the survivors.  Returns
        the tasks this rank ran.
        """
        alive = self.alive_ranks(world)
        if rank not in alive:
            return []
        me = alive.index(rank)
        ran = []
        for n, t in enumerate(self.missing()):
            if n % len(alive) == me:
                run_task(t)
                self.mark_done(t)
                ran.append(t)
        return ran

    def heartbeat(self, rank: int) -> None:
        self.store.set(self._k(f"alive/{rank}"), str(time.time()).encode())

    def mark_failed(self, rank: int) -> None:
        self.store.set(self._k(f"failed/{rank}"), b"1")

    def alive_ranks(self, world: int):
        return [r for r in range(world) if not self.store.check([self._k(f"failed/{r}")])]

    def mark_finished(self, rank: int) -> None:
        self.store.set(self._k(f"finished/{rank}"), b"1")

    def mark_exited(self, rank: int) -> None:
        self.store.set(self._k(f"exited/{rank}"), b"1")

    def wait_exited(self, world: int, timeout_s: float = 60.0) -> None:
        """The store's owner calls this last: every rank is done with the store."""
        deadline = time.time() + timeout_s
        while any(not self.store.check([self._k(f"exited/{r}")]) and
                  not self.store.check([self._k(f"failed/{r}")]) for r in range(world)):
            if time.time() > deadline:
                raise TimeoutError("ranks still using the work-queue store")
            time.sleep(0.01)

    def wait_settled(self, world: int, timeout_s: float = 60.0) -> None:
        """Wait until every rank has either finished its main loop or failed.

        Uses store polling with a deadline, never a collective, so a rank that
        died cannot hang the survivors.
        """
        deadline = time.time() + timeout_s
        while True:
            pending = [r for r in range(world)
                       if not self.store.check([self._k(f"finished/{r}")])
                       and not self.store.check([self._k(f"failed/{r}")])]
            if not pending:
                return
            if time.time() > deadline:
                raise TimeoutError(f"ranks {pending} neither finished nor failed within {timeout_s} s")
            time.sleep(0.01)


def run_sharded(store, rank: int, world: int, costs, run_task, name: str = "tessa", fail_after=None,
                emit=None):
    """Per-rank driver: claim tasks until the queue drains, journal each.

    ``run_task(task) -> result`` runs one task on this rank's GPU; ``emit(task,
    result)`` hands the result to the host reducer before the task is marked
    done, so a journaled task's output survives a later failure of its rank
    (the candidate records stream to the reducer as they are produced).
    Returns ``{task: result}`` for the tasks this rank ran (including re-queued
    ones).
    ``fail_after`` (tests only) makes the rank raise after that many tasks, as
    a crashed host process would; the rank marks itself failed first so the
    survivors re-run its unfinished tasks.
    """
    q = StoreWorkQueue(store, list(costs), name)
    q.heartbeat(rank)
    results = {}
    try:
        while True:
            t = q.claim()
            if t is None:
                break
            if fail_after is not None and len(results) >= fail_after:
                raise RuntimeError(f"rank {rank}: injected host failure after {fail_after} tasks")
            results[t] = run_task(t)
            if emit is not None:
                emit(t, results[t])
            q.mark_done(t)
    except Exception:
        q.mark_failed(rank)
        raise
    q.mark_finished(rank)
    q.wait_settled(world)
    def rerun(t):
        results[t] = run_task(t)
        if emit is not None:
            emit(t, results[t])

    q.requeue_missing(rank, world, rerun)
    q.mark_exited(rank)
    return q, results
