"""shear_b200.sharded_build on B200s: one build split over the GPUs of a box
must give the one-GPU build's graph bit for bit (same leaders, child runs,
leaves and records; a reduction that does not depend on how the records are
split).  World size 1 runs on any box; world size 2 needs two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rows(n, dim, seed):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from subtreecases import clustered_rows
    return clustered_rows(n, dim, 48, seed=seed, unit=dim >= 256)


def _worker(rank, world, port, n, dim, c_max, out_dir, batch_rows=None):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import datetime

    import torch
    import torch.distributed as dist

    from shear_b200.index import BuildParams
    from shear_b200.sharded_build import build_index_sharded, row_range
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    try:
        x = _rows(n, dim, seed=n + dim)
        lo, hi, _ = row_range(n, world, rank)
        p = BuildParams(c_max=c_max, record_batch_rows=batch_rows)
        r = build_index_sharded(np.ascontiguousarray(x[lo:hi]), n, p, device=rank)
        if batch_rows:
            assert r.stats["record_batches"] > 1
        if rank == 0:
            np.save(os.path.join(out_dir, "off.npy"), r.offsets)
            np.save(os.path.join(out_dir, "nb.npy"), r.neighbors)
            np.save(os.path.join(out_dir, "entry.npy"), np.array([r.entry_point]))
        else:
            assert r.offsets is None
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run(tmp_path, world, n, dim, c_max, batch_rows=None):
    from shear_b200.index import BuildParams, build_index
    mp.start_processes(_worker, args=(world, _free_port(), n, dim, c_max, str(tmp_path), batch_rows), nprocs=world,
                       start_method="spawn", join=True)
    want = build_index(_rows(n, dim, seed=n + dim), BuildParams(c_max=c_max))
    assert np.array_equal(np.load(tmp_path / "off.npy"), want.offsets)
    assert np.array_equal(np.load(tmp_path / "nb.npy"), want.neighbors)
    assert int(np.load(tmp_path / "entry.npy")[0]) == want.entry_point


def test_sharded_build_one_rank_equals_build_index(tmp_path):
    _run(tmp_path, 1, 20000, 128, 1024)


def test_sharded_build_one_rank_in_record_batches_equals_build_index(tmp_path):
    # the rank's child runs in record batches (partial reservoirs merged
    # before the owner exchange) give the one-pass graph
    _run(tmp_path, 1, 20000, 128, 1024, batch_rows=40000)


@pytest.mark.parametrize("n,dim,c_max", [(30001, 128, 1024), (12000, 768, 2048)])
def test_sharded_build_two_ranks_equals_build_index(tmp_path, n, dim, c_max):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run(tmp_path, 2, n, dim, c_max)
