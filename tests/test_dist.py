"""Multi-process logic of the batch-sharded job, as gloo ranks on the CPU.

Each rank owns a contiguous shard of the batch (tdc_workloads.shard_range),
draws exactly the images the full batch would hold there (make_inputs with
n_offset), convolves them (here with the CPU oracle standing in for the
device kernel), and the job's time is the max over ranks.  Checked:

* the shards tile the batch, and the gathered shard outputs equal the
  single-process output bit for bit;
* max/sum over ranks;
* a rank that leaves early makes the other rank's next collective fail with an
  error within the process-group timeout instead of waiting for ever.
"""
import os
import socket
import sys
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "tma-depthwise-conv_b200")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _env(rank, world, port):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    for p in (PKG, os.path.join(REPO, "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _shard_worker(rank, world, port, out_dir):
    _env(rank, world, port)
    import oracle
    import tdc_dist
    from tdc_workloads import Workload, make_inputs, shard_range
    r, wsz, _ = tdc_dist.init("gloo", timeout_s=30)
    assert (r, wsz) == (rank, world)
    wl = Workload("t", 5, 12, 20, 64, 1, "normal")
    n0, n1 = shard_range(wl.N, world, rank)
    x, w = make_inputs(wl, "cpu", seed=3, n=n1 - n0, n_offset=n0)
    y = oracle.dwconv_f16(x.numpy(), w.numpy(), wl.pad)
    t0 = time.perf_counter()
    tdc_dist.barrier()
    mx = tdc_dist.max_over_ranks(float(rank + 1))
    sm = tdc_dist.sum_over_ranks(float(n1 - n0))
    gathered = [None] * world
    dist.all_gather_object(gathered, (n0, n1, y))
    if rank == 0:
        full_x, full_w = make_inputs(wl, "cpu", seed=3)
        full = oracle.dwconv_f16(full_x.numpy(), full_w.numpy(), wl.pad)
        pieces = sorted(gathered, key=lambda g: g[0])
        assert [g[0] for g in pieces][0] == 0 and pieces[-1][1] == wl.N
        assert all(a[1] == b[0] for a, b in zip(pieces, pieces[1:]))
        cat = np.concatenate([g[2] for g in pieces if g[1] > g[0]])
        ok = np.array_equal(cat.view(np.uint16), full.view(np.uint16))
        np.save(os.path.join(out_dir, "result.npy"),
                np.array([ok, mx, sm, time.perf_counter() - t0], dtype=np.float64))
    tdc_dist.finalize()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_batch_matches_single_process(tmp_path, world):
    mp.start_processes(_shard_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn")
    ok, mx, sm, _ = np.load(tmp_path / "result.npy")
    assert ok == 1.0 and mx == float(world) and sm == 5.0


def _leaver_worker(rank, world, port, out_dir):
    _env(rank, world, port)
    import tdc_dist
    tdc_dist.init("gloo", timeout_s=5)
    if rank == 1:
        os._exit(0)  # leaves between steps, no collective in flight
    t0 = time.perf_counter()
    err = ""
    try:
        tdc_dist.barrier()
        tdc_dist.max_over_ranks(1.0)
    except Exception as e:  # the expected outcome
        err = type(e).__name__ + ": " + str(e)[:200]
    with open(os.path.join(out_dir, "leaver.txt"), "w") as f:
        f.write(f"{time.perf_counter() - t0:.3f}\n{err}\n")
    os._exit(0)


def test_rank_leaving_is_detected_not_hung(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_leaver_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive(), "a rank is still waiting"
    elapsed, err = open(tmp_path / "leaver.txt").read().split("\n", 1)
    assert err.strip(), "the surviving rank's collective did not report the missing peer"
    assert float(elapsed) < 60


def test_shard_range_tiles_any_batch():
    sys.path.insert(0, PKG)
    from tdc_workloads import shard_range
    for n in range(0, 70):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_make_inputs_shards_are_slices_of_the_batch():
    sys.path.insert(0, PKG)
    from tdc_workloads import Workload, make_inputs
    wl = Workload("t", 6, 5, 7, 64, 1, "uniform")
    x, w = make_inputs(wl, "cpu", seed=1)
    xs, ws = make_inputs(wl, "cpu", seed=1, n=2, n_offset=3)
    assert torch.equal(x[3:5], xs) and torch.equal(w, ws)
    assert x.abs().max() <= 1 and w.abs().max() <= 1 / 3 + 1e-3
