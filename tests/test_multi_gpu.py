"""Row-sharded training over NCCL, one process per GPU: every rank's model
equals the single-GPU model (checked against the oracle on all rows, bit for
bit). Needs two or more GPUs; skipped otherwise."""
import os
import subprocess
import sys

import numpy as np
import pytest

import checkers as C

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:  # pragma: no cover
        return 0


@pytest.mark.skipif(gpu_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("objective,cols,mode,port", [("reg:squarederror", 12, "train", 29533),
                                                      ("binary:logistic", 13, "train", 29541),
                                                      ("binary:logistic", 12, "lazy", 29543)])
def test_two_ranks_match_the_oracle(tmp_path, objective, cols, mode, port):
    """Each rank holds and quantises only its rows; the cuts of all ranks'
    rows are computed on every GPU, so the model equals the single-GPU model.
    13 features over 2 ranks: the padded feature of the reduce-scatter
    layout and an uneven split of the split search. "lazy": a plain DMatrix
    quantised at the first round, also over all ranks' rows."""
    sys.path.insert(0, HERE)
    import mgpu_worker
    # One node: NCCL's bootstrap sockets on loopback, no NVLink multicast.
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", NCCL_NVLS_ENABLE="0", NCCL_SOCKET_IFNAME="lo")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=%d" % port,
           os.path.join(HERE, "mgpu_worker.py"), str(tmp_path), objective, str(cols), mode]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=420)
    assert proc.returncode == 0, proc.stderr[-3000:]
    X, y = mgpu_worker.data(objective, cols)
    params = C.train_params(dict(objective=objective, max_depth=6, eta=0.3, max_bin=64))
    _, margins, _ = C.oracle_train(X, y, params, 6)
    for r in range(2):
        got = np.load(os.path.join(tmp_path, "margins_%d.npy" % r))
        np.testing.assert_array_equal(got.view(np.uint32), margins[:, 0].view(np.uint32))


@pytest.mark.skipif(gpu_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("objective,port", [("reg:squarederror", 29537), ("binary:logistic", 29539)])
def test_two_ranks_host_driven_trees_and_global_metrics(tmp_path, objective, port):
    """Loss-guided trees with a leaf budget over 2 ranks (node histograms
    summed over ranks) equal the oracle's on all rows, and every rank reports
    the evaluation scores of all rows."""
    sys.path.insert(0, HERE)
    import json

    import mgpu_worker
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", NCCL_NVLS_ENABLE="0", NCCL_SOCKET_IFNAME="lo")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=%d" % port,
           os.path.join(HERE, "mgpu_worker.py"), str(tmp_path), objective, "12", "hostdriven"]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=420)
    assert proc.returncode == 0, proc.stderr[-3000:]
    X, y = mgpu_worker.data(objective, 12)
    params = C.train_params(dict(objective=objective, eta=0.3, max_bin=64, **mgpu_worker.HOST_DRIVEN))
    _, margins, _ = C.oracle_train(X, y, params, 6)
    for r in range(2):
        got = np.load(os.path.join(tmp_path, "margins_%d.npy" % r))
        np.testing.assert_array_equal(got.view(np.uint32), margins[:, 0].view(np.uint32))
    evals = [json.load(open(os.path.join(tmp_path, "evals_%d.json" % r))) for r in range(2)]
    assert evals[0] == evals[1]
    last = {k: v[-1] for k, v in evals[0]["train"].items()}
    m = margins[:, 0].astype(np.float64)
    if objective == "reg:squarederror":
        assert last["rmse"] == pytest.approx(np.sqrt(np.mean((m - y) ** 2)), rel=1e-5)
    else:
        p = 1 / (1 + np.exp(-m))
        assert last["error"] == pytest.approx(np.mean((p > 0.5) != (y > 0.5)), abs=1e-9)


@pytest.mark.skipif(gpu_count() < 2, reason="needs two GPUs")
def test_rank_that_leaves_ends_the_others_with_an_error(tmp_path):
    """Failure detection without a GPU fault: rank 1 leaves between rounds
    with nothing in flight. Rank 0's next round cannot complete its
    collectives; after the communicator's 15 s limit the communicator is
    aborted and the round raises XGBoostError (rank 0 then exits with 3)."""
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", NCCL_NVLS_ENABLE="0", NCCL_SOCKET_IFNAME="lo")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29535",
           os.path.join(HERE, "mgpu_worker.py"), str(tmp_path), "reg:squarederror", "12", "leave"]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    out = proc.stdout + proc.stderr
    assert "rank 1 leaves after 2 rounds" in out, out[-3000:]
    assert "rank 0 raised:" in out, out[-3000:]
    assert "did not complete within" in out or "NCCL error" in out, out[-3000:]
    assert proc.returncode != 0
