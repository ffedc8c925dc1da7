"""The sharded design on CPU with two gloo ranks: the contiguous shards cover
the rows, and exact int64 histograms summed over ranks equal the one-GPU
histogram (the property that makes results independent of the GPU count)."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import checkers as C


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(5)
    n, c = 5000, 6
    X = rng.normal(size=(n, c)).astype(np.float32)
    X[rng.random(X.shape) < 0.1] = np.nan
    o = C.oracle()
    cuts, counts, minima = o.sketch_cuts(X, 32)
    bins = o.quantize(X, cuts, counts)
    pairs = np.stack([rng.normal(size=n), rng.random(n)], 1).astype(np.float32)[:, None, :]
    scale = o.gradient_scales(pairs)[0]
    q = np.ascontiguousarray(o.quantize_gradients(pairs, scale[None])[:, 0, :])
    lo, hi = n * rank // world, n * (rank + 1) // world
    stride = cuts.shape[1]
    local = np.zeros((c, stride + 1, 2), np.int64)
    rows = np.arange(lo, hi, dtype=np.uint32)
    o._l.lib.orc_histogram(C._ptr(bins), C._U32(c), C._U32(stride), C._ptr(q), C._ptr(rows),
                           C._U32(len(rows)), C._ptr(local))
    t = torch.from_numpy(local.copy())
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    full = np.zeros_like(local)
    allrows = np.arange(n, dtype=np.uint32)
    o._l.lib.orc_histogram(C._ptr(bins), C._U32(c), C._U32(stride), C._ptr(q), C._ptr(allrows),
                           C._U32(n), C._ptr(full))
    out[rank] = int(np.array_equal(t.numpy(), full)) + 2 * int(hi - lo > 0)
    dist.destroy_process_group()


def test_two_gloo_ranks_sum_to_the_full_histogram():
    world = 2
    out = mp.Manager().dict()
    mp.spawn(_rank, args=(world, _free_port(), out), nprocs=world, join=True)
    assert dict(out) == {0: 3, 1: 3}
