"""bench.py's multi-GPU host logic as 2 gloo ranks on CPU: image sharding covers the batch exactly once,
the device times reduce to the max over ranks, per-rank results gather in rank order, and a rank's shard
computed on its own equals the same images taken from the single-process run."""
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def test_shard_images_partition():
    for total in (1, 7, 32, 33, 256):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                s, n = bench.shard_images(total, r, world)
                seen.extend(range(s, s + n))
            assert seen == list(range(total))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        dev = torch.device("cpu")
        t = bench.max_over_ranks(10.0 + rank, dist, dev)
        rows = bench.gather_floats([float(rank), 2.0 * rank, 7.0], dist, dev)
        # each rank "processes" its shard of a seeded batch; the gathered checksums must equal the
        # single-process checksums of the same images
        start, n = bench.shard_images(6, rank, world)
        batch = np.random.default_rng(5).standard_normal((6, 4)).astype(np.float64)
        sums = bench.gather_floats([float(batch[start:start + n].sum())], dist, dev)
        if rank == 0:
            np.save(os.path.join(outdir, "out.npy"), np.array([t] + [v for r in rows for v in r] + [s[0] for s in sums]))
    finally:
        dist.destroy_process_group()


def test_two_rank_gather_and_max(tmp_path):
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    out = np.load(tmp_path / "out.npy")
    assert out[0] == 11.0                                   # max over ranks
    assert out[1:7].tolist() == [0.0, 0.0, 7.0, 1.0, 2.0, 7.0]  # rank-ordered gather
    batch = np.random.default_rng(5).standard_normal((6, 4)).astype(np.float64)
    assert out[7:].sum() == pytest.approx(batch.sum())
    assert out[7] == pytest.approx(batch[:3].sum()) and out[8] == pytest.approx(batch[3:].sum())


def _failing_worker(rank, world, port, outdir, mode):
    """Rank 1 fails on the host; rank 0 must see an error (not hang) within the process group's timeout."""
    import datetime
    import json
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if mode == "before_init" and rank == 1:
        return  # never joins the rendezvous
    t0 = time.time()
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    except Exception as e:  # rank 0 in "before_init": the store times out waiting for rank 1
        if rank == 0:
            json.dump({"error": type(e).__name__, "where": "init", "s": time.time() - t0},
                      open(os.path.join(outdir, "r0.json"), "w"))
        return
    if mode == "after_init" and rank == 1:
        os._exit(0)  # leaves between steps, with no collective in flight
    try:
        bench.gather_floats([1.0, 2.0], dist, torch.device("cpu"))
        res = {"error": None}
    except Exception as e:
        res = {"error": type(e).__name__, "where": "gather", "s": time.time() - t0}
    if rank == 0:
        json.dump(res, open(os.path.join(outdir, "r0.json"), "w"))
    os._exit(0)


@pytest.mark.parametrize("mode", ["before_init", "after_init"])
def test_rank_failure_surfaces_as_an_error(tmp_path, mode):
    """A rank that never joins, or exits after init, ends the other rank's next step with an error inside the
    process group's timeout (the host side of the multi-GPU path; no GPU is involved)."""
    import json
    port = _free_port()
    ctx = mp.start_processes(_failing_worker, args=(2, port, str(tmp_path), mode), nprocs=2, start_method="spawn",
                             join=False)
    deadline = time.time() + 60
    while not ctx.join(timeout=1):
        assert time.time() < deadline, "a rank hung"
    r0 = json.load(open(tmp_path / "r0.json"))
    assert r0["error"] is not None
    assert r0["where"] == ("init" if mode == "before_init" else "gather")
    assert r0["s"] < 30
