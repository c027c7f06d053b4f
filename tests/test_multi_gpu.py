"""The batch-sharded path on several GPUs (skipped with fewer than two).

* one process, several devices: the C ABI keeps per-device state (SM count,
  occupancy, kernel attributes) and launches on the device that is current;
  each device convolves its own shard and the shards equal the oracle;
* one process per GPU (torch.multiprocessing, gloo for the host-side
  rendezvous only — the data path has no collective): every rank convolves
  its shard of a seeded batch on its own GPU and rank 0 checks the gathered
  result against the single-device output bit for bit.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "tma-depthwise-conv_b200")

needs_two = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")


@needs_two
def test_one_process_two_devices():
    import tma_dwconv as T
    from tdc_workloads import Workload, make_inputs, shard_range
    wl = Workload("t", 6, 40, 70, 128, 1, "normal")
    x, w = make_inputs(wl, "cpu", seed=5)
    ref = oracle.dwconv_f16(x.numpy(), w.numpy(), wl.pad)
    outs = []
    for d in range(2):
        a, b = shard_range(wl.N, 2, d)
        xd, wd = x[a:b].to(f"cuda:{d}"), w.to(f"cuda:{d}")
        y = T.dwconv_ws(xd, wd, wl.pad, 2 + d)
        assert y.device == torch.device(f"cuda:{d}")
        outs.append(y)
    got = torch.cat([o.cpu() for o in outs]).numpy()
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
    for d in range(2):
        assert T.device_status(d)[0] == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path[:0] = [PKG, os.path.join(REPO, "oracle")]
    import torch.distributed as dist
    import tdc_dist
    import tma_dwconv as T
    from tdc_workloads import Workload, make_inputs, shard_range
    tdc_dist.init("gloo", timeout_s=60)
    torch.cuda.set_device(rank)
    wl = Workload("t", 7, 56, 96, 256, 1, "uniform")
    a, b = shard_range(wl.N, world, rank)
    x, w = make_inputs(wl, f"cuda:{rank}", seed=2, n=b - a, n_offset=a)
    y = T.dwconv_ws(x, w, wl.pad, 2).cpu()
    parts = [None] * world
    dist.all_gather_object(parts, (a, y.numpy()))
    if rank == 0:
        xf, wf = make_inputs(wl, "cuda:0", seed=2)
        full = T.dwconv_ws(xf, wf, wl.pad, 2).cpu().numpy()
        cat = np.concatenate([p[1] for p in sorted(parts, key=lambda p: p[0])])
        np.save(os.path.join(out_dir, "ok.npy"), np.array([np.array_equal(cat.view(np.uint16),
                                                                          full.view(np.uint16))]))
    tdc_dist.finalize()


@needs_two
def test_process_per_gpu_shards(tmp_path):
    world = min(torch.cuda.device_count(), 4)
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn")
    assert bool(np.load(tmp_path / "ok.npy")[0])
