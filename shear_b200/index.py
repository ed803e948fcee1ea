"""GPU-subtree index build on one B200: the construction path of
``build_shear_index`` (apps/build_shear_index) with SHEAR's gpu-subtree
partitioner, on libtessa_sm100.so.

Reference flow (shear-core/src/algorithm/pipnn/, Rust):
  D0 preflight (rbc_partition.rs:7332): root leaders, every point assigned to
    its fanout_top nearest (quantize_sq8_and_assign_global_d0,
    compute_backend.rs:3828-3837), one child run per root leader;
  D1+ producer (rbc_partition.rs:9602, :13247): each child run is a subtree
    task, partitioned recursively and evaluated leaf by leaf by the persistent
    kernel (compute_backend.rs:16336-17381) into CompactTopKBatch records;
  host reduction: records flushed into candidate edges with sketch hashes
    (leaf_build.rs:1604-1829) and reduced by HashPrune reservoirs
    (hash_prune.rs:1243-1452); the reservoirs are the graph
    (mod.rs:2437-2478), entry point the first point of the largest child run
    (rbc_partition.rs:4940-4962).

Here: D0 = tessa_quantize_sq8_assign_d0 (rectangular tcgen05 kernel), child
runs grouped on the device, all subtree tasks partitioned in one
tessa_subtree_partition call, leaves through tessa_leaf_topk_sq8, hashes
through tessa_sketch_rows / tessa_edge_hashes, and the HashPrune reservoirs built on
the device (tessa_reduce_records); only the graph (CSR) is copied to pinned
host memory.  The reference's host-side form -- records grouped by reservoir
on the device (tessa_group_edges), copied to the host and reduced by the host
reducer (tessa_reducer_add_grouped) -- is BuildParams.reduction = "host"; both
give the same graph.

Two inputs the reference draws from Rust's StdRng (rand 0.9, ChaCha12),
which cannot be reproduced outside Rust, come from seeded numpy generators
here: the root leader sample and the sketch hyperplanes
(generate_hyperplanes, hash_prune.rs:2196-2206).  Everything after them is
deterministic and restated exactly.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np

from . import ops
from . import task_former as TF


@dataclass
class BuildParams:
    """The PiPNNParams fields this path reads (P/params.rs:3342-3490 defaults)."""
    c_max: int = 2048
    leaf_knn: int = 2
    l_max: int = 64
    m_hash_bits: int = 12
    fanout_top: int = 10
    fanout_second: int = 3
    max_leaders: int = 1000
    # PiPNNParams.max_depth is 10; the recursion on these child runs needs up to
    # ~12 levels (the meaningful-split rule, CB:7082-7101, accepts splits that
    # peel off 1/32 of a node).  The cap only decides when the partition gives
    # up -- every split it allows is the same -- so the build uses 24.
    max_depth: int = 24
    psamp_fraction: float = 0.001
    random_seed: int = 42
    root_leaders: int | None = None        # None: the D0 capacity plan decides
    workspace_bytes: int | None = None     # None: 90% of the device
    # child rows per record batch (partition + leaves + partial reservoirs of a
    # group of child runs, merged at the end); None: as many as the workspace
    # left beside the resident rows holds
    record_batch_rows: int | None = None
    # leaf rows per leaf call inside a record batch; None: a third of the
    # batch's budget for the call's leaf-ordered codes and zone dump
    leaf_call_rows: int | None = None
    reducer_threads: int = 0
    # "device": HashPrune reservoirs built on the GPU (tessa_reduce_records);
    # "host": records grouped on the GPU, reduced by the host reducer
    reduction: str = "device"

    def adaptive_c_max(self, n: int) -> int:
        """P/params.rs:3005-3015."""
        return self.c_max * 2 if n >= 5_000_000 else self.c_max


@dataclass
class BuildResult:
    offsets: np.ndarray                    # CSR of the graph: uint64 [n + 1]
    neighbors: np.ndarray                  # uint32
    entry_point: int
    timings: dict = field(default_factory=dict)
    stats: dict = field(default_factory=dict)

    def degree_stats(self):
        deg = np.diff(self.offsets.astype(np.int64))
        return {"mean": float(deg.mean()), "max": int(deg.max()), "min": int(deg.min())}


def root_leader_count(n: int, dim: int, p: BuildParams, device_bytes: int | None) -> tuple[int, dict]:
    """D0 capacity plan (P/d0_capacity.rs:55-257, restated in task_former): the
    largest admissible subtree for the workspace, its thresholds, and the root
    leader count for n points at fanout_top."""
    if p.root_leaders is not None:
        return int(p.root_leaders), {"source": "fixed"}
    cfg = TF.D0CapacityConfig()
    budget = p.workspace_bytes if p.workspace_bytes is not None else (
        TF.b200_workspace_budget(device_bytes) if device_bytes else None)
    c_gpu = TF.find_max_admissible_rows(dim, p.leaf_knn, p.fanout_second, budget) if budget else n * p.fanout_top
    thr = TF.compute_thresholds(max(c_gpu, 1), cfg)
    plan = TF.plan_root_leaders(n, p.fanout_top, thr, cfg)
    count = min(plan.k_initial, p.max_leaders, n)
    return int(count), {"source": plan.root_leader_source, "c_gpu": int(c_gpu), "k_capacity": int(plan.k_capacity)}


def sample_root_leaders(n: int, count: int, seed: int) -> np.ndarray:
    """Root leader rows (ascending); a seeded stand-in for the reference's
    StdRng sample (rbc_partition.rs:18041-18058)."""
    rng = np.random.default_rng(seed)
    return np.sort(rng.choice(n, size=count, replace=False)).astype(np.uint32)


def hyperplanes(m: int, dim: int, seed: int) -> np.ndarray:
    """m x dim N(0,1) hyperplanes (generate_hyperplanes, hash_prune.rs:2196-2206;
    seeded numpy stand-in for StdRng)."""
    rng = np.random.default_rng(seed ^ 0x5EED)
    return rng.standard_normal((m, dim)).astype(np.float32)


def child_seed_args(p: BuildParams, n: int):
    """gpu_queue_root_seed inputs (compute_backend.rs:1597-1603) of a D1 task:
    depth 1, parent_points = n, min_recurse_size = 2 * adaptive_c_max
    (rbc_partition.rs:7375-7376)."""
    return 1, n, 2 * p.adaptive_c_max(n)


def group_child_runs(child_ids, num_leaders: int):
    """D0 fragments -> child runs: for leader j the rows that chose it, ascending
    (the order in which the D0 pass appends rows to child runs).  child_ids is
    a CUDA int32 tensor [n, fanout]; returns (members CUDA int32, counts,
    offsets) with the counts / offsets on the host."""
    import torch

    n, f = child_ids.shape
    keys = child_ids.reshape(-1)
    # the narrowest key type that holds the leader ids: a stable radix sort of
    # 16-bit keys takes two passes instead of eight
    keys = keys.to(torch.int16) if num_leaders <= 32767 else keys.to(torch.int64)
    order = torch.argsort(keys, stable=True)
    members = (order // f).to(torch.int32)
    counts = torch.bincount(child_ids.reshape(-1), minlength=num_leaders).cpu().numpy().astype(np.uint32)
    offsets = np.concatenate([[0], np.cumsum(counts, dtype=np.uint64)[:-1]]).astype(np.uint64)
    return members, counts, offsets


_PINNED: dict = {}
_GROUPING: dict = {}


def _pinned(name, torch, nbytes):
    """Pinned host staging reused across builds (grown on demand)."""
    buf = _PINNED.get(name)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(int(nbytes * 1.25) + 64, dtype=torch.uint8, pin_memory=True)
        _PINNED[name] = buf
    return buf[:nbytes]


def _grouping_buffers(torch, dev, n, cap):
    """Device outputs of the record grouping, reused across builds."""
    key = dev.index
    bufs = _GROUPING.get(key)
    if bufs is None or bufs[0].numel() < n + 1 or bufs[1].numel() < cap * 12:
        bufs = (torch.empty(n + 1, dtype=torch.int64, device=dev),
                torch.empty(max(cap, 1) * 12, dtype=torch.uint8, device=dev))
        _GROUPING[key] = bufs
    return bufs[0][:n + 1], bufs[1][:max(cap, 1) * 12]


def _upload(x, dev, torch):
    if isinstance(x, np.ndarray):
        xh = torch.from_numpy(np.ascontiguousarray(x, np.float32))
        return xh.pin_memory().to(dev, non_blocking=True) if xh.numel() else xh.to(dev)
    return x.contiguous()


def d0_stage(xd, p: BuildParams, ctx):
    """SQ8 codes of every row, its fanout_top root leaders, and the child runs
    (rows ascending per leader), all rows on this device."""
    import torch

    dev = xd.device
    n, dim = xd.shape
    props = torch.cuda.get_device_properties(dev)
    k0, plan = root_leader_count(n, dim, p, props.total_memory)
    fanout = min(p.fanout_top, k0)
    leaders = sample_root_leaders(n, k0, p.random_seed)
    lid = torch.from_numpy(leaders.view(np.int32)).to(dev)
    gids = torch.arange(n, dtype=torch.int32, device=dev)
    d0 = ops.quantize_sq8_assign_d0(xd, gids, lid, fanout, leader_vectors=xd[lid.long()], ctx=ctx)
    st = child_runs_stage(d0, k0, p)
    st.update(gids=gids, plan=plan, fanout=fanout)
    return st


def child_runs_stage(d0, k0: int, p: BuildParams) -> dict:
    """Child runs of the D0 assignment (rows ascending per root leader), their
    subtree seeds and the entry point (first row of the largest run)."""
    n = d0.rows
    members, counts, offsets = group_child_runs(d0.child_ids, k0)
    depth, parent, min_rec = child_seed_args(p, n)
    seeds = np.array([ops.subtree_root_seed(p.random_seed, depth, int(c), parent, min_rec) for c in counts],
                     np.uint64)
    big = int(len(counts) - 1 - np.argmax(counts[::-1]))
    entry = int(members[int(offsets[big])].item()) if counts[big] else 0
    return dict(d0=d0, members=members, counts=counts, offsets=offsets, seeds=seeds, k0=k0, depth=depth,
                entry=entry)


def record_bytes_per_child_row(p: BuildParams, padded_dim: int) -> int:
    """Device bytes one child row costs a record batch: up to fanout_second
    leaf rows, each with its leaf-ordered code row, zone dump (at most 48
    8-byte entries, 32 floats of merged distances), top-k ids, distances and
    edge hashes, and the reduction's key/value double buffers and run flags
    for its 2k edges; plus the partition's arena entries."""
    k = max(1, min(p.leaf_knn, 32))
    leaf_row = padded_dim + 48 * 8 + 32 * 4 + 2 + 12 * k + 4 + 2 * k * (32 + 8)
    return p.fanout_second * leaf_row + 64


def record_batch_rows(torch, dev, p: BuildParams, n: int, padded_dim: int, x_bytes: int = 0) -> int:
    """Child rows per record batch: p.record_batch_rows, else the workspace
    (p.workspace_bytes, or 80% of the device) less what stays resident through
    the batches -- codes, scales, norms, sketches and child runs of all n rows,
    the f32 rows if they are on the device -- and a 2 GiB reserve."""
    if p.record_batch_rows:
        return int(p.record_batch_rows)
    total = torch.cuda.get_device_properties(dev).total_memory
    cap = p.workspace_bytes if p.workspace_bytes is not None else int(0.8 * total)
    resident = n * (padded_dim + 8 + 4 * p.m_hash_bits + 12 * p.fanout_top) + x_bytes + (2 << 30)
    return max(1 << 20, (cap - resident) // record_bytes_per_child_row(p, padded_dim))


def leaf_call_rows_for(p: BuildParams, padded_dim: int, batch_child_rows: int) -> int:
    """Leaf rows per leaf call inside a record batch: a third of the batch's
    budget for the call's leaf-ordered codes and zone dump."""
    per_row = padded_dim + 48 * 8 + 32 * 4 + 2
    return max(1 << 20, batch_child_rows * record_bytes_per_child_row(p, padded_dim) // (3 * per_row))


def record_batches(counts, tasks, rows_cap: int) -> list:
    """`tasks` (indices into counts) in order, cut into consecutive groups of
    at most rows_cap child rows (a larger run forms a group of its own)."""
    out, cur, acc = [], [], 0
    for t in tasks:
        c = int(counts[t])
        if cur and acc + c > rows_cap:
            out.append(cur)
            cur, acc = [], 0
        cur.append(int(t))
        acc += c
    if cur:
        out.append(cur)
    return out


def batched_reservoirs(xd, st: dict, p: BuildParams, ctx, batches: list, n: int, timings: dict, sketches,
                       neighbors: bool = True, slots: bool = False, leaf_call_rows=None):
    """records_stage + partial HashPrune reservoirs per record batch, merged
    by tessa_reduce_grouped.  Exact: a per-hash minimum among a source's final
    l_max best is among the best of every part of its edges, so truncating
    each batch's part to its l_max best per source loses nothing.  Returns
    (offsets, neighbors, slots, count) as reduce_stage, and a record summary
    for the statistics."""
    pieces, sizes, fallback, parts, k = [], [], 0, [], max(1, min(p.leaf_knn, 32))
    for key in ("partition_s", "leaf_s", "leaf_kernel_ms", "reduce_s"):
        timings[key] = 0.0
    import torch

    for b in batches:
        tb = {}
        rec = records_stage(xd, st, p, ctx, tasks=b, timings=tb, sketches=sketches, leaf_call_rows=leaf_call_rows)
        t = time.perf_counter()
        o, _, sl, c = reduce_stage(rec, n, p, ctx, neighbors=False, slots=True)
        sl = sl[:c * 12].clone()  # the slots kept, not the buffer sized for every edge
        tb["reduce_s"] = time.perf_counter() - t
        pieces.append((o, sl, c))
        sizes.append(rec["sizes"])
        fallback += int(rec["fallback"])
        parts.append(rec["partition"])
        k = rec["k"]
        for key in ("partition_s", "leaf_s", "leaf_kernel_ms", "reduce_s"):
            timings[key] += tb.get(key, 0.0)
        del rec
        torch.cuda.empty_cache()  # the next batch's leaf call allocates outside torch's cache
    t = time.perf_counter()
    out = ops.reduce_grouped(pieces, n, p.l_max, ctx=ctx, neighbors=neighbors, slots=slots)
    timings["reduce_s"] += time.perf_counter() - t
    part = {f: sum(x[f] for x in parts) for f in parts[0]} if parts else {}
    summary = dict(sizes=np.concatenate(sizes) if sizes else np.zeros(0, np.uint64), fallback=fallback,
                   partition=part, k=k, batches=len(batches))
    return out, summary


def records_stage(xd, st: dict, p: BuildParams, ctx, tasks=None, timings=None, sketches=None, leaf_call_rows=None):
    """Subtree partition of the child runs `tasks` (all when None), their
    leaves' top-k lists and both sketch hashes of every slot, on the device.
    The sketches of every row are computed from xd unless given."""
    import torch

    timings = {} if timings is None else timings
    d0 = st["d0"]
    dev = d0.codes.device
    n, dim = d0.rows, d0.dim
    sel = np.arange(len(st["counts"])) if tasks is None else np.asarray(tasks, np.int64)
    sel = sel[st["counts"][sel] > 0]
    k = max(1, min(p.leaf_knn, 32))
    if sel.size == 0:  # no work on this device
        timings.update(partition_s=0.0, leaf_s=0.0, leaf_kernel_ms=0.0)
        e32 = torch.empty(0, dtype=torch.int32, device=dev)
        e16 = torch.empty(0, dtype=torch.int16, device=dev)
        return dict(leaf_rows=e32, ids=e32, dists=torch.empty(0, device=dev), hf=e16, hr=e16, k=k,
                    starts=np.zeros(0, np.uint64), sizes=np.zeros(0, np.uint64),
                    partition=dict(rounds=0, large_assignments=0, retries=0, balanced=0, small_nodes=0,
                                   leaf_rows_used=0, kernel_launches=0),
                    fallback=0)
    t = time.perf_counter()
    # the sketches depend only on the rows: computed on a side stream, they
    # fill the device while the partition's host round loop decides splits
    side = None
    if sketches is None:
        main = torch.cuda.current_stream(dev)
        side, planes, buf = _sketch_resources(torch, dev, p, n, dim)
        side.wait_stream(main)  # the previous build's readers of buf are done
        with torch.cuda.stream(side):
            sketches = ops.sketch_rows(xd, planes, ctx=ctx, out=buf)
    sp = ops.SubtreeParams(c_max=p.adaptive_c_max(n), max_depth=p.max_depth, max_leaders=p.max_leaders,
                           fanout_second=p.fanout_second, root_depth=st["depth"], psamp_fraction=p.psamp_fraction)
    # (the partition can also copy the leaf-ordered codes round by round --
    # leaf_codes -- but on a side stream those copies slow the concurrent
    # assignment kernels by more than they save the leaf call)
    t_call = time.perf_counter()
    timings["partition_setup_s"] = t_call - t
    leaf_rows, starts, sizes, _, pst = ops.subtree_partition(d0.codes, d0.scales, d0.norms, st["members"],
                                                             st["offsets"][sel], st["counts"][sel],
                                                             st["seeds"][sel], sp, ctx=ctx)
    t_sync = time.perf_counter()
    timings["partition_call_s"] = t_sync - t_call
    torch.cuda.synchronize(dev)
    timings["partition_sync_s"] = time.perf_counter() - t_sync
    timings["partition_s"] = time.perf_counter() - t
    t = time.perf_counter()
    rows = int(leaf_rows.numel())
    ids = torch.full((rows * k,), -1, dtype=torch.int32, device=dev)
    dists = torch.full((rows * k,), float("inf"), dtype=torch.float32, device=dev)
    ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    ev[0].record()
    fallback = 0
    if not leaf_call_rows or rows <= leaf_call_rows:
        ops.leaf_topk_sq8(d0.codes, d0.scales, d0.norms, st["gids"], leaf_rows, starts, sizes, k, out=(ids, dists),
                          ctx=ctx)
        fallback = ops.leaf_last_fallback_rows(ctx)
    else:
        # whole leaves per call, at most leaf_call_rows rows each (the call's
        # leaf-ordered codes and zone dump scale with its rows)
        order = np.argsort(starts, kind="stable")
        s_ord = starts[order].astype(np.int64)
        e_ord = np.maximum.accumulate(s_ord + sizes[order].astype(np.int64))
        i = 0
        while i < order.size:
            base = int(s_ord[i])
            j = max(i + 1, int(np.searchsorted(e_ord, base + leaf_call_rows, side="right")))
            r1 = int(e_ord[j - 1])
            sel = order[i:j]
            ops.leaf_topk_sq8(d0.codes, d0.scales, d0.norms, st["gids"], leaf_rows[base:r1],
                              (starts[sel] - np.uint64(base)).astype(np.uint64), sizes[sel], k,
                              out=(ids[base * k:r1 * k], dists[base * k:r1 * k]), ctx=ctx)
            fallback += ops.leaf_last_fallback_rows(ctx)
            i = j
    ev[1].record()
    if side is not None:
        torch.cuda.current_stream(dev).wait_stream(side)
    hf, hr = ops.edge_hashes(leaf_rows, ids, k, sketches, p.m_hash_bits, starts, sizes, ctx=ctx)
    torch.cuda.synchronize(dev)
    timings["leaf_s"] = time.perf_counter() - t
    timings["leaf_kernel_ms"] = ev[0].elapsed_time(ev[1])
    return dict(leaf_rows=leaf_rows, ids=ids, dists=dists, hf=hf, hr=hr, k=k, starts=starts, sizes=sizes,
                partition=pst, fallback=fallback)


def sketch_planes(torch, dev, p: BuildParams, dim: int):
    return torch.from_numpy(hyperplanes(p.m_hash_bits, dim, p.random_seed)).to(dev)


_SKETCH_RES: dict = {}  # device index -> (side stream, planes key, planes, buffer key, buffer)


def _sketch_resources(torch, dev, p: BuildParams, n: int, dim: int):
    """The side stream, hyperplanes and sketch buffer of a device's builds,
    kept from build to build: a new stream, a pageable upload of the planes
    and a fresh buffer per build cost a build up to 30 ms of host time."""
    r = _SKETCH_RES.get(dev.index)
    pkey, bkey = (p.m_hash_bits, dim, p.random_seed), (n, p.m_hash_bits)
    if r is None:
        r = [torch.cuda.Stream(dev), None, None, None, None]
        _SKETCH_RES[dev.index] = r
    if r[1] != pkey:
        r[1], r[2] = pkey, sketch_planes(torch, dev, p, dim)
    if r[3] != bkey:
        r[3], r[4] = bkey, None
        r[4] = torch.empty((n, p.m_hash_bits), dtype=torch.float32, device=dev)
    return r[0], r[2], r[4]


def group_stage(rec: dict, n: int, ctx):
    """Distinct candidate edges grouped by reservoir on the device:
    (offsets int64 [n + 1], edges uint8 [total * 12], total)."""
    import torch

    dev = rec["ids"].device
    rows, k = int(rec["leaf_rows"].numel()), rec["k"]
    goff, gedges = ops.group_edges(rec["leaf_rows"], rec["ids"], rec["dists"], rec["hf"], rec["hr"], k, n, ctx=ctx,
                                   out=_grouping_buffers(torch, dev, n, 2 * rows * k))
    total = int(goff[n].item())
    return goff, gedges[:total * 12], total


def reduce_stage(rec: dict, n: int, p: BuildParams, ctx, neighbors: bool = True, slots: bool = False):
    """HashPrune reservoirs of the records on the device: (offsets int64
    [n + 1], neighbors int32 or None, slots uint8 (tessa_edge) or None,
    slot count).  One reduction takes fewer than 2^32 edges; larger record
    sets are reduced in row chunks whose reservoirs are merged."""
    k = rec["k"]
    args = (rec["leaf_rows"], rec["ids"], rec["dists"], rec["hf"], rec["hr"])
    rows = int(args[0].numel())
    chunk = (1 << 31) // (2 * k)
    if rows <= chunk:
        return ops.reduce_records(*args, k, n, p.l_max, ctx=ctx, neighbors=neighbors, slots=slots)
    pieces = []
    for r0 in range(0, rows, chunk):
        r1 = min(rows, r0 + chunk)
        o, _, sl, c = ops.reduce_records(args[0][r0:r1], args[1][r0 * k:r1 * k], args[2][r0 * k:r1 * k],
                                         args[3][r0 * k:r1 * k], args[4][r0 * k:r1 * k], k, n, p.l_max, ctx=ctx,
                                         neighbors=False, slots=True)
        pieces.append((o, sl, c))
    return ops.reduce_grouped(pieces, n, p.l_max, ctx=ctx, neighbors=neighbors, slots=slots)


def graph_to_host(torch, d_off, d_nb, count: int):
    """CSR from the device into pinned host memory: (offsets uint64, neighbors
    uint32).  The arrays live in pinned blocks from torch's caching host
    allocator, released back to it when the result is dropped."""
    h_off = torch.empty(int(d_off.numel()), dtype=torch.int64, pin_memory=True)
    h_nb = torch.empty(max(count, 1), dtype=torch.int32, pin_memory=True)
    h_off.copy_(d_off, non_blocking=True)
    if count:
        h_nb[:count].copy_(d_nb[:count], non_blocking=True)
    torch.cuda.current_stream(d_off.device).synchronize()
    return h_off.numpy().view(np.uint64), h_nb[:count].numpy().view(np.uint32)


def build_index(x, p: BuildParams | None = None, device: int = 0, ctx=None) -> BuildResult:
    """Build the graph of x (numpy f32 [n, dim] on the host -- copied to the
    device inside -- or a CUDA f32 tensor already resident)."""
    import torch

    p = p or BuildParams()
    dev = torch.device("cuda", device)
    ctx = ctx or ops.context(device)
    timings = {}
    sync = lambda: torch.cuda.synchronize(dev)
    t_all = time.perf_counter()
    xd = _upload(x, dev, torch)
    n, dim = xd.shape
    sync()
    timings["upload_s"] = time.perf_counter() - t_all

    # ---- D0: SQ8 codes of every row and its fanout_top root leaders
    t = time.perf_counter()
    st = d0_stage(xd, p, ctx)
    sync()
    timings["d0_s"] = time.perf_counter() - t

    # ---- subtree partition of every child run, leaf top-k, edge hashes; in
    #      record batches when they do not fit the workspace at once
    pd = st["d0"].codes.shape[1]
    live = np.nonzero(st["counts"] > 0)[0]
    cap_rows = record_batch_rows(torch, dev, p, n, pd, xd.numel() * 4)
    batches = record_batches(st["counts"], live, cap_rows)
    if p.reduction == "device" and len(batches) > 1:
        sk = ops.sketch_rows(xd, sketch_planes(torch, dev, p, dim), ctx=ctx)
        (d_off, d_nb, _, count), rec = batched_reservoirs(xd, st, p, ctx, batches, n, timings, sk,
                                                         leaf_call_rows=p.leaf_call_rows or
                                                         leaf_call_rows_for(p, pd, cap_rows))
        del sk
        t = time.perf_counter()
        offs, nb = graph_to_host(torch, d_off, d_nb, count)
        timings["d2h_s"] = time.perf_counter() - t
        timings["total_s"] = time.perf_counter() - t_all
        stats = _stats(st, rec, n, dim, None, 0)
        stats.update(d2h_bytes=int((n + 1) * 8 + count * 4), reduction="device", record_batches=len(batches))
        # D0 and sketches once; per batch the partition's launches, the leaf
        # call's four, edge hashes and the reduction's five; the merge's five
        stats["kernel_launches"] = 5 + rec["partition"]["kernel_launches"] + 10 * len(batches) + 5
        return BuildResult(offs, nb, st["entry"], timings, stats)
    rec = records_stage(xd, st, p, ctx, timings=timings)

    if p.reduction == "host":
        # ---- candidate records grouped by reservoir on the device, pinned D2H,
        #      host HashPrune reduction
        t = time.perf_counter()
        goff, gedges, total = group_stage(rec, n, ctx)
        h_off = _pinned("offsets", torch, (n + 1) * 8)
        h_edges = _pinned("edges", torch, max(total, 1) * 12)
        h_off.copy_(goff.view(torch.uint8), non_blocking=True)
        if total:
            h_edges[:total * 12].copy_(gedges, non_blocking=True)
        sync()
        timings["group_d2h_s"] = time.perf_counter() - t
        t = time.perf_counter()
        red = ops.Reducer(n, p.l_max, p.reducer_threads)
        red.add_grouped(h_off.numpy().view(np.uint64), h_edges[:total * 12].numpy().view(ops.EDGE_DTYPE))
        offs, nb = red.finish()
        edges = red.edges()
        red.close()
        timings["reduce_s"] = time.perf_counter() - t
        d2h = (n + 1) * 8 + total * 12
    elif p.reduction == "device":
        # ---- HashPrune reservoirs on the device; the graph to pinned host memory
        t = time.perf_counter()
        d_off, d_nb, _, count = reduce_stage(rec, n, p, ctx)
        sync()
        timings["reduce_s"] = time.perf_counter() - t
        t = time.perf_counter()
        offs, nb = graph_to_host(torch, d_off, d_nb, count)
        timings["d2h_s"] = time.perf_counter() - t
        edges = None  # not counted on this path (it would cost a pass over the records)
        total, d2h = 0, (n + 1) * 8 + count * 4
    else:
        raise ValueError(f"reduction must be 'device' or 'host', not {p.reduction!r}")
    timings["total_s"] = time.perf_counter() - t_all
    stats = _stats(st, rec, n, dim, edges, total)
    stats["d2h_bytes"] = int(d2h)
    stats["reduction"] = p.reduction
    stats["kernel_launches"] += 3 if p.reduction == "host" else 5
    return BuildResult(offs, nb, st["entry"], timings, stats)


def _stats(st, rec, n, dim, edges, total):
    sizes = rec["sizes"]
    pst = rec["partition"]
    return dict(points=n, dim=dim, root_leaders=st["k0"], root_plan=st["plan"], fanout_top=st["fanout"],
                child_rows=int(st["counts"].sum()), leaves=int(sizes.size), leaf_rows=int(sizes.sum()),
                leaf_rows_mean=float(sizes.mean()) if sizes.size else 0.0, leaf_k=rec["k"], edges=edges,
                leaf_pairs=int((sizes.astype(np.int64) * (sizes.astype(np.int64) - 1)).sum()),
                leaf_ops=int(2 * st["d0"].codes.shape[1] * (sizes.astype(np.int64) ** 2).sum()),
                leaf_fallback_rows=int(rec["fallback"]), partition=pst,
                # quantize + D0 rectangular kernel + its exact fallback + fragments; partition;
                # gather + column-split leaf kernel + finish + fallback; sketches; edge hashes;
                # then the reduction's own kernels (host: record grouping's keys, mark, emit;
                # device: keys, runs, compaction, kept counts, selection; sorts and scans are CUB's)
                kernel_launches=4 + pst["kernel_launches"] + 4 + 2)
