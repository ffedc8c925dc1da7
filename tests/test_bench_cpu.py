"""Host-side parts of the bench line, checked on the CPU with bench.py's own
functions.

The data digest: a hash of the SHA-256 of each block of rows (X bytes, then
labels), blocks in row order, that every GPU count must give alike for the
same rows. The block size tiles the shards of 1, 2, 4 and 8 ranks at every
workload's row count, the digest of a whole matrix equals the one gathered
from its shards over two and four gloo ranks (the bench's own Dist class),
and one changed value changes it.

The kernel launch count (`gpu_launches`) against the committed launch list
of the c4 bench, and the CPU record that goes beside the CPU timings."""
import hashlib
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _matrix(rows, cols=6, seed=11):
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(rows, cols)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    return X, rng.normal(size=rows).astype(np.float32)


class _OneRank:
    rank, world = 0, 1

    def gather_bytes(self, data):
        return [data]


@pytest.mark.parametrize("wl", sorted(bench.WORKLOADS))
def test_blocks_tile_every_shard(wl):
    rows = bench.WORKLOADS[wl]["rows"]
    block = bench.digest_block_rows(rows)
    assert 0 < block <= bench.DIGEST_BLOCK_ROWS
    for world in (1, 2, 4, 8):
        for rank in range(world):
            lo, hi = bench.shard(rows, rank, world)
            assert lo % block == 0 and (hi - lo) % block == 0, (wl, world, rank)


def test_one_rank_digest_is_a_hash_of_block_hashes():
    X, y = _matrix(4000)
    block = bench.digest_block_rows(4000)
    assert block == 500
    want = b"".join(hashlib.sha256(X[b:b + block].tobytes() + y[b:b + block].tobytes()).digest()
                    for b in range(0, 4000, block))
    got = bench.data_digest(X, y, 4000, _OneRank())
    assert got["input_sha256"] == hashlib.sha256(want).hexdigest()
    assert got["blocks"] == 8 and got["block_rows"] == 500
    X2 = X.copy()
    X2[3999, 5] = np.float32(1.5)
    assert bench.data_digest(X2, y, 4000, _OneRank())["input_sha256"] != got["input_sha256"]


def test_rows_that_eight_does_not_divide_hash_as_one_block():
    X, y = _matrix(1001)
    assert bench.digest_block_rows(1001) == 1001
    got = bench.data_digest(X, y, 1001, _OneRank())
    assert got["blocks"] == 1
    assert got["input_sha256"] == hashlib.sha256(
        hashlib.sha256(X.tobytes() + y.tobytes()).digest()).hexdigest()


def _rank(rank, world, port, rows, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    d = bench.Dist()
    X, y = _matrix(rows)
    lo, hi = bench.shard(rows, rank, world)
    got = bench.data_digest(np.ascontiguousarray(X[lo:hi]), np.ascontiguousarray(y[lo:hi]), rows, d)
    if rank == 0:
        out["digest"] = got["input_sha256"]
        out["blocks"] = got["blocks"]
    else:
        out["other"] = got
    d.close()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_give_the_one_rank_digest(world):
    rows = 8 * 700
    X, y = _matrix(rows)
    want = bench.data_digest(X, y, rows, _OneRank())
    out = mp.Manager().dict()
    mp.spawn(_rank, args=(world, _free_port(), rows, out), nprocs=world, join=True)
    assert out["digest"] == want["input_sha256"]
    assert out["blocks"] == want["blocks"] == 8
    assert out["other"] is None


def test_cpu_record_names_the_host():
    got = bench.cpu_model()
    assert isinstance(got["model"], str) and got["model"]
    assert got["logical_cpus"] >= got["usable_cpus"] == bench.cpu_cores() >= 1


def test_launch_count_matches_the_committed_c4_launch_list():
    """profiles/launches_c4_bench.md lists 1,131 launches of this library's
    kernels over 15 c4 rounds on one GPU, 3 of them base_chunk_kernel and 3
    fill_margins_kernel (one each per booster's first round): 75 per round,
    the last level's margins in two passes over 50M rows."""
    W = bench.WORKLOADS
    assert bench.launches_per_round(W["c4"], 1, 50_000_000) == (1131 - 3 - 3) // 15 == 75
    # Sharded: two mass-limb conversions per round, pack and merge per level,
    # and one margin pass once a rank's margins fit in 96 MiB.
    assert bench.launches_per_round(W["c4"], 2, 25_000_000) == 75 + 2 + 20 - 1
    assert bench.launches_per_round(W["c4"], 8, 6_250_000) == 96
    # uint8 codes with real hessians add the staged three-limb launch per level.
    c3 = bench.launches_per_round(W["c3"], 1, 1_000_000)
    assert c3 == 5 + 10 * (1 + 6 * 5 + 3 * 5 + 1)


@pytest.mark.skipif(not __import__("checkers").have_reference(), reason="reference harness not built")
def test_tree_comparison_of_the_reference_parity_checks():
    """compare_trees, which the bench's c2 and c4 CPU legs use to hold this
    library's trees to the reference path's: equal tables give None, across the two
    record layouts (the library's 48-byte records, the reference harness's
    40-byte ones); a changed threshold, leaf bit or node count is named."""
    import checkers as C
    import product as P
    o, r = C.oracle(), C.reference()
    rng = np.random.default_rng(21)
    X = rng.normal(size=(3000, 5)).astype(np.float32)
    y = (X[:, 0] - X[:, 1] ** 2).astype(np.float32)
    cuts, counts, minima = r.sketch_cuts(X, 64)
    bins = r.quantize(X, cuts, counts)
    pairs = C.oracle_gradients("reg:squarederror", np.zeros((3000, 1), np.float32), y)
    s = r.gradient_scales(pairs)
    q = r.quantize_gradients(pairs, s)
    tp = dict(max_depth=5, eta=0.3, reg_lambda=1.0, reg_alpha=0.0, min_child_weight=1.0, max_delta_step=0.0,
              min_split_loss=0.0)
    want = [r.grow_tree(bins, q[:, 0, :], s[0], cuts, counts, minima, tp)[0]]
    dev = np.zeros(len(want[0]), P.DEVNODE_DTYPE)
    for f in C.NODE_DTYPE.names:
        dev[f] = want[0][f]
    assert bench.compare_trees([dev], want) is None
    assert bench.compare_trees([o.grow_tree(bins, q[:, 0, :], s[0], cuts, counts, minima, tp)[0]], want) is None
    changed = dev.copy()
    split = np.nonzero(changed["left"] >= 0)[0][1]
    changed["threshold"][split] = np.nextafter(changed["threshold"][split], np.float32(np.inf))
    assert bench.compare_trees([changed], want) == "tree 0: threshold"
    changed = dev.copy()
    leaf = np.nonzero(changed["left"] < 0)[0][0]
    changed["leaf"][leaf] = -changed["leaf"][leaf]
    assert bench.compare_trees([changed], want) == "tree 0: leaf"
    assert bench.compare_trees([dev[:-1]], want).startswith("tree 0: ")
    assert bench.compare_trees([], want) == "0 trees against 1"


@pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="needs a machine without a GPU")
def test_reference_parity_failure_is_recorded_not_raised():
    """Without a GPU the library refuses to train; the check records that in
    the bench line instead of raising."""
    class _Ref:
        trees = []
    X = np.zeros((10, 3), np.float32)
    got = bench.reference_parity(_Ref(), X, np.zeros(10, np.float32), bench.params_for("c2"), 4, 0.0)
    assert got["identical"] is None and "error" in got
