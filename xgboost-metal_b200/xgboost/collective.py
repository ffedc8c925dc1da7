"""Row-sharded multi-GPU training (one process per GPU over NCCL).

Upstream XGBoost's collective module (python-package/xgboost/collective.py in
the reference) wraps a tracker; the reference's C ABI stubs it out
(src/c_api.cpp:600-614). Here XGCommunicatorInit builds an NCCL communicator
from a unique id that rank 0 creates and the ranks share out of band (for
example through torch.distributed or any key-value store):

    uid = xgboost.collective.nccl_unique_id()          # on rank 0, then share
    with xgboost.collective.CommunicatorContext(rank=r, world_size=n,
                                                nccl_unique_id=uid, device=r):
        xgboost.train(params, dtrain_shard, rounds)
"""
import ctypes
import json

from .core import _LIB, _c_str, _check_call

__all__ = ["init", "finalize", "get_rank", "get_world_size", "nccl_unique_id",
           "CommunicatorContext"]


def nccl_unique_id():
    out = ctypes.c_char_p()
    _check_call(_LIB.XGBBNcclUniqueId(ctypes.byref(out)))
    return out.value.decode()


def init(**args):
    cfg = {"rank": int(args.get("rank", 0)), "world_size": int(args.get("world_size", 1)),
           "device": int(args.get("device", 0)),
           "nccl_unique_id": args.get("nccl_unique_id", "")}
    # Seconds a collective may wait for the other ranks before the
    # communicator is aborted and the waiting call raises XGBoostError.
    if args.get("timeout") is not None:
        cfg["timeout"] = float(args["timeout"])
    _check_call(_LIB.XGCommunicatorInit(_c_str(json.dumps(cfg))))


def finalize():
    _check_call(_LIB.XGCommunicatorFinalize())


def get_rank():
    return int(_LIB.XGCommunicatorGetRank())


def get_world_size():
    return int(_LIB.XGCommunicatorGetWorldSize())


class CommunicatorContext:
    def __init__(self, **args):
        self.args = args

    def __enter__(self):
        init(**self.args)
        return self

    def __exit__(self, *exc):
        finalize()
