"""One rank of the row-sharded training check (launched by test_multi_gpu.py
under torch.distributed.run, one process per GPU): quantises and trains on its
contiguous row shard only (the cuts cover every rank's rows) and writes the
full-matrix margins."""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "xgboost-metal_b200"))

import torch  # noqa: E402  (first, so its NCCL is the process's NCCL)
import torch.distributed as dist  # noqa: E402

import xgboost as xgb  # noqa: E402
from xgboost import core  # noqa: E402


def data(objective, c=12):
    rng = np.random.default_rng(2026)
    n = 30000
    X = rng.normal(size=(n, c)).astype(np.float32)
    X[rng.random(X.shape) < 0.08] = np.nan
    z = np.nan_to_num(X) @ rng.normal(size=c)
    if objective == "binary:logistic":
        y = (rng.random(n) < 1 / (1 + np.exp(-z))).astype(np.float32)
    else:
        y = (z + rng.normal(size=n)).astype(np.float32)
    return X, y


def leave_after_two_rounds(params, shard, rank, world):
    """The last rank leaves between rounds, its work finished and nothing in
    flight; the others must end a later round with an error (after the
    communicator's 15 s limit) instead of waiting for it forever."""
    bst = xgb.Booster(params, [shard])
    for i in range(2):
        bst.update(shard, i)
    core.synchronize()
    if rank == world - 1:
        print("rank %d leaves after 2 rounds" % rank, flush=True)
        os._exit(0)
    try:
        for i in range(2, 8):
            bst.update(shard, i)
        core.synchronize()
    except xgb.core.XGBoostError as e:
        # After an aborted communicator the process exits at once.
        print("rank %d raised: %s" % (rank, e), flush=True)
        os._exit(3)
    print("rank %d: no error" % rank, flush=True)
    os._exit(1)


HOST_DRIVEN = {"grow_policy": "lossguide", "max_depth": 0, "max_leaves": 24}


def main():
    import faulthandler
    faulthandler.dump_traceback_later(int(os.environ.get("XGBB_WORKER_TIMEOUT", "240")), exit=True)
    out_dir, objective = sys.argv[1], sys.argv[2]
    cols = int(sys.argv[3]) if len(sys.argv) > 3 else 12
    mode = sys.argv[4] if len(sys.argv) > 4 else "train"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo")
    core.set_device(local)
    box = [xgb.collective.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    xgb.collective.init(rank=rank, world_size=world, nccl_unique_id=box[0], device=local,
                        timeout=15.0 if mode == "leave" else None)
    X, y = data(objective, cols)
    lo, hi = len(y) * rank // world, len(y) * (rank + 1) // world
    # Every rank quantises only its own rows: the cuts come from the rows of
    # all ranks (assembled over NCCL), so they equal the single-GPU cuts.
    if mode == "lazy":
        shard = xgb.DMatrix(X[lo:hi], label=y[lo:hi])
    else:
        shard = xgb.QuantileDMatrix(X[lo:hi], label=y[lo:hi], max_bin=64)
    params = {"objective": objective, "max_depth": 6, "eta": 0.3, "max_bin": 64,
              "device": "cuda", "tree_method": "hist",
              "cuda_graph": int(os.environ.get("XGBB_WORKER_GRAPH", "1"))}
    if mode == "leave":
        leave_after_two_rounds(params, shard, rank, world)
        return
    evals_result = {}
    if mode == "hostdriven":
        # Loss-guided trees under a leaf budget, evaluated on every rank's
        # shard: the scores cover all ranks' rows.
        params.update(HOST_DRIVEN)
        metrics = ["rmse", "mae"] if objective == "reg:squarederror" else ["logloss", "error", "auc"]
        params["eval_metric"] = metrics
        bst = xgb.train(params, shard, 6, evals=[(shard, "train")], evals_result=evals_result)
    else:
        bst = xgb.train(params, shard, 6)
    margins = bst.predict(xgb.DMatrix(X), output_margin=True)
    np.save(os.path.join(out_dir, "margins_%d.npy" % rank), margins)
    with open(os.path.join(out_dir, "evals_%d.json" % rank), "w") as f:
        json.dump(evals_result, f)
    xgb.collective.finalize()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
