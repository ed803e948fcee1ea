"""The sharded build's exchange and gather steps on two CPU ranks (gloo).

shear_b200.sharded_build splits one build over the GPUs of a box; its only
data-path collectives are the all-to-all of partial reservoirs by owner range
and the gather of the owners' graph pieces.  Here two gloo ranks on 127.0.0.1
each hold candidate edges for every point (grouped by source, as a rank's
partial reservoirs are), exchange them with exchange_reservoirs, merge what
they own with the host reducer, and gather the graph on rank 0 with
gather_graph; rank 0 checks it against one reducer fed every rank's edges.
The device reduction is checked against the host reducer on the GPU."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from shear_b200.sharded_build import row_range


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_row_ranges_cover_rows_in_padded_blocks():
    for n, world in ((10, 3), (7, 8), (1_000_000, 8), (5, 1), (9, 4)):
        ranges = [row_range(n, world, r) for r in range(world)]
        per = ranges[0][2]
        assert per == -(-n // world)
        assert ranges[0][0] == 0 and ranges[-1][1] == n
        for r, (lo, hi, _) in enumerate(ranges):
            assert lo <= hi and hi - lo <= per
            if hi > lo:
                assert lo == r * per  # block r of the padded all-gather holds these rows
        assert sum(hi - lo for lo, hi, _ in ranges) == n


def _edges(rank, n, m):
    from shear_b200 import ops
    rng = np.random.default_rng(100 + rank)
    src = rng.integers(0, n, m)
    e = np.zeros(m, ops.EDGE_DTYPE)
    e["target"] = rng.integers(0, n, m)
    e["dist"] = np.round(rng.random(m) * 16).astype(np.float32) / np.float32(16)
    e["hash"] = rng.integers(0, 64, m)
    order = np.argsort(src, kind="stable")
    counts = np.bincount(src, minlength=n)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    return offsets, e[order]


def _worker(rank, world, port, n, m, l_max, out_dir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import datetime

    import torch
    import torch.distributed as dist

    from shear_b200 import ops
    from shear_b200.sharded_build import exchange_reservoirs, gather_graph
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        offsets, e = _edges(rank, n, m)
        pieces = exchange_reservoirs(torch.from_numpy(offsets), torch.from_numpy(e.view(np.uint8).copy()), n)
        lo, hi, _ = row_range(n, world, rank)
        # the host reducer spans all n points (targets are global ids); only
        # the owned range receives edges
        red = ops.Reducer(n, l_max, 2)
        for off, sl, cnt in pieces:
            o = off.numpy().astype(np.uint64)
            full = np.zeros(n + 1, np.uint64)
            full[lo:hi + 1] = o - o[0]
            full[hi + 1:] = o[-1] - o[0]
            red.add_grouped(full, sl.numpy()[:cnt * 12].view(ops.EDGE_DTYPE))
        f_off, f_nb = red.finish()
        red.close()
        o_off = f_off[lo:hi + 1] - f_off[lo]
        o_nb = f_nb[int(f_off[lo]):int(f_off[hi])]
        g = gather_graph(torch.from_numpy(o_off.astype(np.int64)), torch.from_numpy(o_nb.view(np.int32)),
                         int(o_nb.size), n)
        if rank == 0:
            np.save(os.path.join(out_dir, "off.npy"), g[0].numpy())
            np.save(os.path.join(out_dir, "nb.npy"), g[1].numpy())
        else:
            assert g is None
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n", [(2, 3001), (3, 500)])
def test_exchange_and_gather_equal_one_reducer(tmp_path, world, n):
    from shear_b200 import ops
    m, l_max = 20000, 8
    mp.start_processes(_worker, args=(world, _free_port(), n, m, l_max, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    red = ops.Reducer(n, l_max, 2)
    for r in range(world):
        off, e = _edges(r, n, m)
        red.add_grouped(off.astype(np.uint64), e)
    want_off, want_nb = red.finish()
    red.close()
    got_off = np.load(tmp_path / "off.npy")
    got_nb = np.load(tmp_path / "nb.npy")
    assert np.array_equal(got_off, want_off.astype(np.int64))
    assert np.array_equal(got_nb.view(np.uint32), want_nb)
