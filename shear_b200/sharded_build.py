"""One index build split over the GPUs of one box (strong scaling).

The reference's GPU build fans its D1+ subtree tasks out over the devices of a
box (independent child tasks, shear-core/src/algorithm/pipnn/rbc_partition.rs:
15558-15600) and funnels every leaf record into one host-side HashPrune
reducer.  Here each rank runs the same stages as the one-GPU build
(shear_b200.index) on its share, and the reduction stays on the GPUs:

  rows      rank r holds rows [r*R, min(n, (r+1)*R)), R = ceil(n / world),
            uploaded from the host by that rank alone;
  D0        every rank quantizes and assigns its own rows against the same root
            leaders (the leader rows travel as exact bit patterns through one
            all-reduce); codes, scales, norms, D0 children and sketches of all
            rows are then all-gathered over NVLink (about 0.9 KB a row), so
            every rank sees the one-GPU build's D0 result bit for bit;
  subtrees  the child runs (one per root leader) are dealt out by
            longest-processing-time on their row counts (sharding.plan_lpt);
            each rank partitions its runs, evaluates their leaves and hashes
            the candidate edges;
  reduce    each rank builds partial HashPrune reservoirs of its own records on
            the device -- per source the l_max best per-hash minima, which the
            final reservoir keeps or drops exactly as if it saw every record
            (the same order-independence that lets the reference merge
            batches) -- then ONE all-to-all sends each source's partial slots
            to the rank that owns it (owner ranges = row ranges) and the owner
            merges the pieces into the final reservoirs;
  graph     the owners' CSR pieces are gathered on rank 0 and copied to its
            pinned host memory.

The result equals build_index on the same rows: the same leaders, child runs,
seeds, leaves and records, and a reduction whose result does not depend on how
the records are split.  Collectives: one all-reduce (leader rows, k0 x dim
words), five all-gathers (row data), three all-to-alls (counts, slots,
offsets), two gathers (graph); every rank takes all of them in the same order.
"""
from __future__ import annotations

import time

import numpy as np

from . import index as IX
from . import ops
from .sharding import plan_lpt


def row_range(n: int, world: int, rank: int):
    """Rows (and owned reservoirs) of `rank`: [lo, hi) with R = ceil(n / world)
    rows per rank, so that the ranks' padded blocks concatenate to rows 0..n-1."""
    per = -(-n // world)
    lo = min(n, rank * per)
    return lo, min(n, lo + per), per


def _dist():
    import torch.distributed as dist
    return dist


def exchange_reservoirs(offsets, slots, n: int, group=None):
    """All-to-all of partial reservoirs by owner range.

    offsets: int64 tensor [n + 1] (slot offsets of every source), slots: uint8
    tensor of 12-byte tessa_edge slots.  Returns this rank's pieces, one per
    sender in rank order: (offsets int64 [range + 1] -- absolute in the
    sender's numbering --, slots uint8, slot count)."""
    import torch

    dist = _dist()
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    dev = offsets.device
    bounds = [row_range(n, world, o)[0] for o in range(world)] + [n]
    at = offsets[torch.tensor(bounds, device=dev)].cpu().tolist()
    send_counts = torch.tensor([at[o + 1] - at[o] for o in range(world)], dtype=torch.int64, device=dev)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    rc = recv_counts.cpu().tolist()
    sc = send_counts.cpu().tolist()
    send = slots[at[0] * 12:at[world] * 12]
    recv = torch.empty(max(sum(rc), 1) * 12, dtype=torch.uint8, device=dev)
    dist.all_to_all_single(recv[:sum(rc) * 12], send, output_split_sizes=[c * 12 for c in rc],
                           input_split_sizes=[c * 12 for c in sc], group=group)
    lo, hi, _ = row_range(n, world, rank)
    span = hi - lo + 1
    send_off = torch.cat([offsets[bounds[o]:bounds[o + 1] + 1] for o in range(world)])
    recv_off = torch.empty(world * span, dtype=torch.int64, device=dev)
    dist.all_to_all_single(recv_off, send_off, output_split_sizes=[span] * world,
                           input_split_sizes=[bounds[o + 1] - bounds[o] + 1 for o in range(world)], group=group)
    pieces, base = [], 0
    for s in range(world):
        pieces.append((recv_off[s * span:(s + 1) * span], recv[base * 12:], rc[s]))
        base += rc[s]
    return pieces


def gather_graph(offsets, neighbors, count: int, n: int, group=None, dst: int = 0):
    """The owners' CSR pieces (offsets int64 [range + 1] from 0, neighbors
    int32 [>= count]) gathered on rank `dst` into one CSR over all n points:
    (offsets int64 [n + 1], neighbors int32 [total]) there, None elsewhere."""
    import torch

    dist = _dist()
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    dev = offsets.device
    counts = [torch.zeros(1, dtype=torch.int64, device=dev) for _ in range(world)]
    dist.all_gather(counts, torch.tensor([count], dtype=torch.int64, device=dev), group=group)
    counts = [int(c.item()) for c in counts]
    width = max(max(counts), 1)
    per = row_range(n, world, 0)[2]
    nb = torch.zeros(width, dtype=torch.int32, device=dev)
    nb[:count] = neighbors[:count]
    off = torch.zeros(per + 1, dtype=torch.int64, device=dev)
    off[:offsets.numel()] = offsets
    nb_list = [torch.empty(width, dtype=torch.int32, device=dev) for _ in range(world)] if rank == dst else None
    off_list = [torch.empty(per + 1, dtype=torch.int64, device=dev) for _ in range(world)] if rank == dst else None
    dist.gather(nb, nb_list, dst=dst, group=group)
    dist.gather(off, off_list, dst=dst, group=group)
    if rank != dst:
        return None
    all_off = torch.empty(n + 1, dtype=torch.int64, device=dev)
    parts, base = [], 0
    for s in range(world):
        lo, hi, _ = row_range(n, world, s)
        all_off[lo:hi] = off_list[s][:hi - lo] + base
        parts.append(nb_list[s][:counts[s]])
        base += counts[s]
    all_off[n] = base
    return all_off, torch.cat(parts) if parts else torch.empty(0, dtype=torch.int32, device=dev)


def build_index_sharded(x_local, n: int, p: IX.BuildParams | None = None, device: int = 0, ctx=None, group=None):
    """Build the graph of n rows split over the ranks of `group` (NCCL, one
    rank per GPU).  x_local holds this rank's rows row_range(n, world, rank)
    (host numpy f32, copied to the device inside, or a CUDA tensor).  Every
    rank must call it; rank 0 returns the BuildResult (graph in host memory),
    the others a BuildResult without a graph (offsets and neighbors None)."""
    import torch

    dist = _dist()
    p = p or IX.BuildParams()
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    dev = torch.device("cuda", device)
    ctx = ctx or ops.context(device)
    lo, hi, per = row_range(n, world, rank)
    rows = hi - lo
    timings = {}
    sync = lambda: torch.cuda.synchronize(dev)
    t_all = time.perf_counter()
    xs = IX._upload(x_local, dev, torch) if rows else torch.empty((0, 1), device=dev)
    if rows and (xs.shape[0] != rows):
        raise ValueError(f"rank {rank}: x_local has {xs.shape[0]} rows, its range [{lo}, {hi}) has {rows}")
    dim_t = torch.tensor([xs.shape[1] if rows else 0], dtype=torch.int64, device=dev)
    dist.all_reduce(dim_t, op=dist.ReduceOp.MAX, group=group)
    dim = int(dim_t.item())
    sync()
    timings["upload_s"] = time.perf_counter() - t_all

    # ---- D0 on this rank's rows against the common root leaders
    t = time.perf_counter()
    props = torch.cuda.get_device_properties(dev)
    k0, plan = IX.root_leader_count(n, dim, p, props.total_memory)
    chk = torch.tensor([k0, -k0], dtype=torch.int64, device=dev)
    dist.all_reduce(chk, op=dist.ReduceOp.MAX, group=group)
    if int(chk[0]) != k0 or int(chk[1]) != -k0:
        raise RuntimeError("ranks disagree on the root leader count (devices of different memory sizes)")
    fanout = min(p.fanout_top, k0)
    leaders = IX.sample_root_leaders(n, k0, p.random_seed)
    lid = torch.from_numpy(leaders.view(np.int32)).to(dev)
    # leader rows as int32 bit patterns: one owner, zeros elsewhere, so the sum is exact
    lv = torch.zeros((k0, dim), dtype=torch.int32, device=dev)
    mine = np.nonzero((leaders >= lo) & (leaders < hi))[0]
    if mine.size:
        idx = torch.from_numpy(mine).to(dev)
        src = torch.from_numpy((leaders[mine] - lo).astype(np.int64)).to(dev)
        lv[idx] = xs[src].view(torch.int32)
    dist.all_reduce(lv, group=group)
    pd = ops.padded_dim(dim)
    codes = torch.empty((world * per, pd), dtype=torch.int8, device=dev)
    scales = torch.empty(world * per, dtype=torch.float32, device=dev)
    norms = torch.empty(world * per, dtype=torch.float32, device=dev)
    child = torch.empty(world * per * fanout, dtype=torch.int32, device=dev)
    width = p.m_hash_bits
    sk = torch.empty((world * per, width), dtype=torch.float32, device=dev)
    b0, b1 = rank * per, rank * per + per
    if rows:
        gids = torch.arange(lo, hi, dtype=torch.int32, device=dev)
        point = torch.empty(rows * fanout, dtype=torch.int32, device=dev)
        d0d = torch.empty(rows * fanout, dtype=torch.float32, device=dev)
        ops.quantize_sq8_assign_d0(xs, gids, lid, fanout, leader_vectors=lv.view(torch.float32), ctx=ctx,
                                   out=(codes[b0:b0 + rows], scales[b0:b0 + rows], norms[b0:b0 + rows],
                                        child[b0 * fanout:(b0 + rows) * fanout], point, d0d))
        ops.sketch_rows(xs, IX.sketch_planes(torch, dev, p, dim), ctx=ctx, out=sk[b0:b0 + rows])
    for t_ in (codes, scales, norms, sk):
        dist.all_gather_into_tensor(t_, t_[b0:b1].contiguous(), group=group)
    dist.all_gather_into_tensor(child, child[b0 * fanout:b1 * fanout].contiguous(), group=group)
    d0 = ops.D0Result(codes[:n], scales[:n], norms[:n], child[:n * fanout].view(n, fanout), None, None, dim)
    st = IX.child_runs_stage(d0, k0, p)
    st.update(gids=torch.arange(n, dtype=torch.int32, device=dev), plan=plan, fanout=fanout)
    sync()
    timings["d0_s"] = time.perf_counter() - t

    # ---- this rank's child runs: partition, leaves, hashes, partial reservoirs
    shards = plan_lpt([int(c) for c in st["counts"]], world)
    tasks = sorted(shards[rank])
    live = [t_ for t_ in tasks if st["counts"][t_] > 0]
    cap_rows = IX.record_batch_rows(torch, dev, p, n, pd, xs.numel() * 4)
    batches = IX.record_batches(st["counts"], live, cap_rows)
    if len(batches) > 1:  # the rank's records do not fit the workspace at once
        (off, _, slots, cnt), rec = IX.batched_reservoirs(None, st, p, ctx, batches, n, timings, sk[:n],
                                                         neighbors=False, slots=True,
                                                         leaf_call_rows=p.leaf_call_rows or
                                                         IX.leaf_call_rows_for(p, pd, cap_rows))
        sync()
    else:
        rec = IX.records_stage(None, st, p, ctx, tasks=tasks, timings=timings, sketches=sk[:n])
        t = time.perf_counter()
        off, _, slots, cnt = IX.reduce_stage(rec, n, p, ctx, neighbors=False, slots=True)
        sync()
        timings["reduce_s"] = time.perf_counter() - t

    # ---- exchange by owner range, merge, gather the graph on rank 0
    t = time.perf_counter()
    pieces = exchange_reservoirs(off, slots, n, group)
    if rows:
        o_off, o_nb, _, o_cnt = ops.reduce_grouped(pieces, rows, p.l_max, ctx=ctx)
    else:
        o_off, o_nb, o_cnt = torch.zeros(1, dtype=torch.int64, device=dev), None, 0
    g = gather_graph(o_off, o_nb if o_nb is not None else torch.empty(0, dtype=torch.int32, device=dev), o_cnt, n,
                     group)
    sync()
    timings["exchange_s"] = time.perf_counter() - t
    offs = nb = None
    if g is not None:
        t = time.perf_counter()
        offs, nb = IX.graph_to_host(torch, g[0], g[1], int(g[1].numel()))
        timings["d2h_s"] = time.perf_counter() - t
    timings["total_s"] = time.perf_counter() - t_all
    stats = IX._stats(st, rec, n, dim, None, 0)
    stats.update(tasks=len(tasks), task_rows=int(st["counts"][tasks].sum()) if tasks else 0, record_batches=len(batches),
                 partial_slots=int(cnt), owned_slots=int(o_cnt), reduction="device",
                 d2h_bytes=int((n + 1) * 8 + nb.size * 4) if nb is not None else 0,
                 # D0 + partition + leaf + hashes of this rank, the local reduction, the owners' merge
                 kernel_launches=(IX._stats(st, rec, n, dim, None, 0)["kernel_launches"] + 10))
    return IX.BuildResult(offs, nb, st["entry"], timings, stats)
