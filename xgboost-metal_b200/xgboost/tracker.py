"""RabitTracker (python-package/xgboost/tracker.py in the reference). Ranks of
this library bootstrap NCCL from a unique id shared out of band
(xgboost.collective.nccl_unique_id / init), so there is no tracker to run."""
from .core import XGBoostError

__all__ = ["RabitTracker"]


class RabitTracker:
    def __init__(self, n_workers, host_ip=None, port=0, *, sortby="host", timeout=0):
        raise XGBoostError("Trackers are not used by the CUDA backend: share "
                           "xgboost.collective.nccl_unique_id() with every rank and call "
                           "xgboost.collective.init(rank=..., world_size=..., nccl_unique_id=...).")
