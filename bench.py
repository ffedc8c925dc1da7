#!/usr/bin/env python
"""Benchmark: train ms per 100 rounds (and histogram-build HBM GB/s) of the
CUDA trainer on the BASELINE.json workload, at 1..8 GPUs of one node.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c4|c2|c1|c0]
    torchrun --nproc-per-node N bench.py --gpus N ...        (one rank per GPU)
    python bench.py --impl reference ...                     (CPU reference arm)

A step is one boosting round. Data are synthetic and seeded per 1M-row chunk,
generated on the GPU, so every GPU count trains on the same rows (strong
scaling: the total row count is fixed and rows are sharded contiguously).
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "xgboost-metal_b200"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

METRIC = "train ms per 100 rounds (histogram build in roofline GB/s)"
UNIT = "ms/100 rounds"

WORKLOADS = {
    # the 1/2/4/8-GPU workload.
    "c4": dict(rows=50_000_000, cols=128, nan=0.05, objective="binary:logistic", max_depth=10,
               eta=0.1, labels="logistic"),
    # the 10x-vs-CPU workload.
    "c2": dict(rows=262_144, cols=64, nan=0.0, objective="reg:squarederror", max_depth=8,
               eta=0.3, labels="linear"),
    "c1": dict(rows=100_000, cols=32, nan=0.15, objective="reg:squarederror", max_depth=6,
               eta=0.3, labels="linear"),
    "c0": dict(rows=100_000, cols=32, nan=0.0, objective="reg:squarederror", max_depth=6,
               eta=0.3, labels="linear"),
    # 10-class softprob on integer-valued images (<= 256 distinct
    # values per feature, ~80 % zeros, no missing), a synthetic stand-in.
    "c3": dict(rows=1_000_000, cols=784, nan=0.0, objective="multi:softprob", max_depth=6,
               eta=0.3, labels="classes", num_class=10),
}
CHUNK = 1_000_000


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ---------------------------------------------------------------------------
# Synthetic data (GPU, seeded per chunk)
# ---------------------------------------------------------------------------
def gen_classes_chunk(spec, begin, n, device):
    """Rows of the class-pattern workload: class patterns P[k] ~ U(0, 255) per
    pixel (seed 7), cells below the 80th percentile of P[k] are 0, the rest
    clip(Poisson(P[k]), 0, 255); row i has class (i mod K) under a fixed
    shuffle (seed 8)."""
    import torch
    K, cols, rows = spec["num_class"], spec["cols"], spec["rows"]
    P = np.random.default_rng(7).uniform(0, 255, size=(K, cols)).astype(np.float32)
    thr = np.quantile(P, 0.8, axis=1, keepdims=True).astype(np.float32)
    labels = (np.arange(rows) % K)[np.random.default_rng(8).permutation(rows)][begin:begin + n]
    Pd = torch.from_numpy(P).to(device)
    keep = torch.from_numpy(P >= thr).to(device)
    lab = torch.from_numpy(labels.astype(np.int64)).to(device)
    g = torch.Generator(device=device)
    g.manual_seed(1341 * 1000003 + begin // CHUNK)
    X = torch.poisson(Pd[lab], generator=g).clamp_(0, 255)
    X = torch.where(keep[lab], X, torch.zeros_like(X))
    return X, lab.float()


def gen_chunk(wl, c, device):
    """Rows [c*CHUNK, min((c+1)*CHUNK, rows)) of workload `wl`, on the GPU."""
    import torch
    spec = WORKLOADS[wl]
    begin = c * CHUNK
    n = min(CHUNK, spec["rows"] - begin)
    cols = spec["cols"]
    if spec["labels"] == "classes":
        return gen_classes_chunk(spec, begin, n, device)
    g = torch.Generator(device=device)
    g.manual_seed(1337 * 1000003 + c)
    X = torch.randn(n, cols, generator=g, device=device, dtype=torch.float32)
    mask = torch.rand(n, cols, generator=g, device=device) < spec["nan"] if spec["nan"] else None
    g2 = torch.Generator(device=device)
    g2.manual_seed(1340 * 1000003 + c)
    if spec["labels"] == "logistic":
        w = torch.from_numpy(np.random.default_rng(1339).normal(0, 0.1, cols).astype(np.float32)).to(device)
        Xz = X if mask is None else X.masked_fill(mask, 0.0)
        logits = Xz @ w + 0.5 * Xz[:, 0] * Xz[:, 1]
        y = (torch.rand(n, generator=g2, device=device) < torch.sigmoid(logits)).float()
    else:
        w = torch.from_numpy(np.random.default_rng(1338).normal(size=cols).astype(np.float32)).to(device)
        y = X @ w + 0.1 * torch.randn(n, generator=g2, device=device)
    if mask is not None:
        X = X.masked_fill(mask, float("nan"))
    return X, y


def gen_rows(wl, begin, end, device, pin=True):
    """Host (pinned) copies of global rows [begin, end)."""
    import torch
    cols = WORKLOADS[wl]["cols"]
    n = end - begin
    Xh = torch.empty((n, cols), dtype=torch.float32, pin_memory=pin)
    yh = torch.empty((n,), dtype=torch.float32, pin_memory=pin)
    c = begin // CHUNK
    while c * CHUNK < end:
        X, y = gen_chunk(wl, c, device)
        lo, hi = max(begin, c * CHUNK), min(end, c * CHUNK + X.shape[0])
        Xh[lo - begin:hi - begin].copy_(X[lo - c * CHUNK:hi - c * CHUNK])
        yh[lo - begin:hi - begin].copy_(y[lo - c * CHUNK:hi - c * CHUNK])
        del X, y
        c += 1
    torch.cuda.synchronize(device)
    return Xh.numpy(), yh.numpy()


def params_for(wl):
    s = WORKLOADS[wl]
    p = {"objective": s["objective"], "max_depth": s["max_depth"], "eta": s["eta"],
         "max_bin": 256, "tree_method": "hist", "device": "cuda", "seed": 42,
         "reg_lambda": 1.0}
    if "num_class" in s:
        p["num_class"] = s["num_class"]
    return p


def groups_of(wl):
    return int(WORKLOADS[wl].get("num_class", 1))


# ---------------------------------------------------------------------------
# Clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(mx)),
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# Distributed plumbing (one process per GPU)
# ---------------------------------------------------------------------------
class Dist:
    def __init__(self):
        self.rank = int(os.environ.get("RANK", 0))
        self.world = int(os.environ.get("WORLD_SIZE", 1))
        self.local = int(os.environ.get("LOCAL_RANK", 0))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist
            dist.init_process_group("gloo", timeout=datetime.timedelta(minutes=15))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v):
        if not self.pg:
            return v
        import torch
        t = torch.tensor([float(v)], dtype=torch.float64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def gather_bytes(self, data):
        """Every rank's bytes on rank 0, in rank order (None elsewhere)."""
        if not self.pg:
            return [data]
        box = [None] * self.world if self.rank == 0 else None
        self.pg.gather_object(data, box, dst=0)
        return box

    def bcast(self, obj):
        if not self.pg:
            return obj
        box = [obj]
        self.pg.broadcast_object_list(box, src=0)
        return box[0]

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


def shard(rows, rank, world):
    return rows * rank // world, rows * (rank + 1) // world


# The reference's benchmark records the SHA-256 of its input rows and labels
# with every run (benchmarks/controlled_comparison.py:107-108). A 25.6 GB
# matrix takes too long to hash serially, and a shard's hash depends on the
# GPU count, so the digest here is a hash of block hashes: SHA-256 of each
# block of rows (X bytes then y bytes), then SHA-256 over the block digests
# in row order. Blocks divide every shard of 1, 2, 4 and 8 ranks, so every
# GPU count gives the same digest for the same rows.
DIGEST_BLOCK_ROWS = 250_000


def digest_block_rows(rows):
    """Rows per digest block: the largest divisor of rows/8 that is at most
    DIGEST_BLOCK_ROWS when 8 divides the rows (so blocks tile the shards of
    1, 2, 4 and 8 ranks), else the whole matrix."""
    if rows % 8:
        return rows
    eighth = rows // 8
    for d in range(min(eighth, DIGEST_BLOCK_ROWS), 0, -1):
        if eighth % d == 0:
            return d
    return eighth


def block_digests(Xh, yh, block, threads):
    """SHA-256 of each `block` rows of (Xh, yh), in row order, hashed on
    `threads` host threads (hashlib releases the GIL on large buffers)."""
    import hashlib
    from concurrent.futures import ThreadPoolExecutor
    assert Xh.shape[0] == yh.shape[0] and Xh.shape[0] % block == 0, "blocks must tile the rows"
    X2 = np.ascontiguousarray(Xh)
    y2 = np.ascontiguousarray(yh)

    def one(b):
        h = hashlib.sha256(memoryview(X2[b * block:(b + 1) * block]).cast("B"))
        h.update(memoryview(y2[b * block:(b + 1) * block]).cast("B"))
        return h.digest()

    with ThreadPoolExecutor(max_workers=max(1, threads)) as pool:
        return list(pool.map(one, range(Xh.shape[0] // block)))


def data_digest(Xh, yh, rows, dist):
    """{input_sha256, blocks, block_rows} over all ranks' rows, on rank 0
    (None elsewhere); outside every timed region."""
    import hashlib
    block = digest_block_rows(rows)
    if Xh.shape[0] % block:
        block = Xh.shape[0] if dist.world == 1 else 0
    mine = b"".join(block_digests(Xh, yh, block, cpu_cores() // dist.world)) if block else b"?"
    parts = dist.gather_bytes(mine)
    if parts is None:
        return None
    if any(p == b"?" for p in parts):
        return {"input_sha256": None, "note": "the shards do not divide into equal digest blocks"}
    joined = b"".join(parts)
    return {"input_sha256": hashlib.sha256(joined).hexdigest(), "blocks": len(joined) // 32,
            "block_rows": block,
            "note": "SHA-256 over the SHA-256 of each block of rows (float32 X bytes, then float32 "
                    "labels), blocks in row order; the same at every GPU count"}


def parity_digest(bst, dtrain, dist, next_round):
    """SHA-256 of every tree of the booster (node arrays of the model JSON)
    and of the root level's int64 (g, h) histogram words of one more round,
    the feature ranges of all ranks joined in rank order. Both are the same
    at every GPU count when training is bit-exact."""
    import hashlib

    import product as P
    trees = json.loads(bst.save_raw("json"))["learner"]["gradient_booster"]["model"]["trees"]
    model = hashlib.sha256(json.dumps(trees, sort_keys=True).encode()).hexdigest()
    P.capture_level_histograms(bst, 0)
    bst.update(dtrain, next_round)
    meta, hist, _ = P.level_histograms(bst)
    parts = dist.gather_bytes(np.ascontiguousarray(hist).tobytes())
    return {"model_sha256": model, "trees": len(trees),
            "root_hist_sha256": hashlib.sha256(b"".join(parts)).hexdigest() if parts else None,
            "root_hist_words": int(hist.size) * dist.world if parts else None,
            "note": "trees after warm-up + timed rounds; root histogram of the round after them"}


def launches_per_round(spec, world, rows_local):
    """This library's kernel launches in one device-driven round of
    workload `spec` on `world` ranks holding `rows_local` rows each.

    Per round: gradients, mass window, scales, exact mass, exact scales, and
    with several ranks the mass limbs' two conversions around their sum.
    Per tree: init; per level the histogram launches (the unstaged
    three-limb kernel and the staged two-limb one, one of which exits at
    once, plus the staged three-limb one for uint8 codes with real
    hessians), evaluation and control, and with several ranks the best-split
    pack and merge; per level but the last, partition, child counts and the
    next level's plan; at the last level one margin pass per 96 MiB of the
    rank's margins (tree.cu, tree_level_partition)."""
    depth = spec["max_depth"]
    groups = int(spec.get("num_class", 1))
    codes8 = spec["nan"] == 0  # 256 bins: uint8 codes only without missing values
    unit_h = spec["objective"] == "reg:squarederror"
    hist = 2 + (1 if codes8 and not unit_h else 0)
    margin_bytes = rows_local * 4 * min(groups, 8)
    passes = max(1, -(-margin_bytes // (96 << 20)))
    sharded = world > 1
    per_tree = 1 + depth * (hist + 2 + 2 * sharded) + 3 * (depth - 1) + passes
    return 5 + 2 * sharded + groups * per_tree


# ---------------------------------------------------------------------------
# CPU baselines: the reference's own functions on the host (oracle/_ref)
# ---------------------------------------------------------------------------
def cpu_sample_rows(wl):
    """Rows the CPU legs time: the whole matrix when it is small (c0-c2), a
    leading 2M-row sample of c4 (c3: 200k rows of 784 features x 10
    classes), so that a timed round takes seconds."""
    spec = WORKLOADS[wl]
    if spec["rows"] <= 300_000:
        return spec["rows"]
    return 200_000 if spec["cols"] * spec.get("num_class", 1) > 1000 else 2_000_000


class ReferencePath:
    """One boosting round of the reference's own CPU path on a fixed sample:
    its gradients kernel, gradient scales and quantisation, then its split
    evaluation, selection, tree driver and predict functions over its
    feature-major uint16 bins, building the smaller child of each node pair
    and subtracting the sibling as its level loop does, on every host thread
    (oracle/_ref/libxgbref.so, compiled from the reference's sources). The
    cuts and bins come from the reference's own sketch and quantize kernel
    (the DMatrix step, not timed)."""

    def __init__(self, wl, rows, device, keep_trees=False):
        import checkers as C
        self.C = C
        self.r = C.reference()
        self.trees = [] if keep_trees else None
        spec = WORKLOADS[wl]
        self.spec, self.rows = spec, rows
        X, self.y = gen_rows(wl, 0, rows, device, pin=False)
        self.cuts, self.counts, self.minima = self.r.sketch_cuts(X, 256)
        self.fm = C.reference_quantize_fm(X, self.cuts, self.counts)
        del X
        self.groups = groups_of(wl)
        self.margins = np.zeros((rows, self.groups), np.float32)
        self.tp = dict(max_depth=spec["max_depth"], eta=spec["eta"], reg_lambda=1.0, reg_alpha=0.0,
                       min_child_weight=1.0, max_delta_step=0.0, min_split_loss=0.0)

    def round(self):
        """Seconds of one boosting round (wall clock)."""
        C = self.C
        t = time.perf_counter()
        pairs = C.reference_gradients(self.spec["objective"], self.margins, self.y)
        scale = self.r.gradient_scales(pairs)
        q = self.r.quantize_gradients(pairs, scale)
        for g in range(self.groups):   # one tree per class
            nodes, leaf = C.reference_grow_tree_fm(self.fm, q[:, g, :], scale[g], self.cuts, self.counts,
                                                   self.minima, self.tp)
            self.margins[:, g] += leaf
            if self.trees is not None:
                self.trees.append(nodes)
        return time.perf_counter() - t


def compare_trees(got, want):
    """The first difference between two lists of node tables (this
    library's 48-byte records or the reference path's 40-byte ones, by field
    name), or None: structure, features, leaf values and covers bit for bit,
    and at split nodes the thresholds, gains, default directions and split
    bins."""
    def bits(a):
        return np.ascontiguousarray(a).view(np.uint32)
    if len(got) != len(want):
        return "%d trees against %d" % (len(got), len(want))
    for t, (g, w) in enumerate(zip(got, want)):
        if len(g) != len(w):
            return "tree %d: %d nodes against %d" % (t, len(g), len(w))
        for f in ("left", "right", "parent", "feature"):
            if not np.array_equal(g[f], w[f]):
                return "tree %d: %s" % (t, f)
        for f in ("leaf", "cover"):
            if not np.array_equal(bits(g[f]), bits(w[f])):
                return "tree %d: %s" % (t, f)
        split = w["left"] >= 0
        for f in ("threshold", "gain"):
            if not np.array_equal(bits(g[f][split]), bits(w[f][split])):
                return "tree %d: %s" % (t, f)
        for f in ("default_left", "split_bin"):
            if not np.array_equal(g[f][split].astype(np.int64), w[f][split].astype(np.int64)):
                return "tree %d: %s" % (t, f)
    return None


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count()


def cpu_model():
    """The host CPU's model name and logical CPU count, recorded beside the
    CPU timings (the reference's benchmark records the platform with each
    run)."""
    name = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    name = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    import platform
    return {"model": name or platform.processor() or platform.machine(), "logical_cpus": os.cpu_count(),
            "usable_cpus": cpu_cores()}


def _full_rows_model(wl, device, measured):
    """A labelled estimate of the reference path at the workload's full row
    count: per-round seconds t = a + b * rows fitted through a second,
    half-size sample (the per-node split search is the constant part, the
    histograms and partitions grow with rows), evaluated at the full rows."""
    import checkers as C
    spec = WORKLOADS[wl]
    rows2, t2 = measured
    if rows2 >= spec["rows"] or not C.have_reference():
        return None
    half = ReferencePath(wl, rows2 // 2, device)
    half.round()
    t1 = min(half.round(), half.round())
    b = (t2 - t1) / (rows2 - rows2 // 2)
    a = t1 - b * (rows2 // 2)
    return {"ms_per_100_rounds": round((a + b * spec["rows"]) * 1e5, 1), "rows": spec["rows"],
            "model": "t = a + b*rows through %d rows (%.3f s) and %d rows (%.3f s) per round"
                     % (rows2 // 2, t1, rows2, t2), "kind": "extrapolated"}


def cpu_baseline_leg(wl, device):
    """cpu_baseline: the reference path on the sample, warm-up round then the
    best of three timed rounds (about 10-30 s of CPU work)."""
    import checkers as C
    if not C.have_reference():
        return None
    rows = cpu_sample_rows(wl)
    spec = WORKLOADS[wl]
    check = spec["objective"] == "binary:logistic"
    ref = ReferencePath(wl, rows, device, keep_trees=check)
    ref.round()
    per_round = min(ref.round() for _ in range(3))
    out = {"value": round(per_round * 1e5, 1), "unit": UNIT, "cores": cpu_cores(), "kind": "reference",
           "cpu": cpu_model(),
           "rows": rows,
           "sample": "the reference's CPU path (oracle/_ref: its gradients, scales, split evaluation, "
                     "selection, tree driver and predict functions over its feature-major uint16 bins, "
                     "smaller child built, sibling subtracted) on the first %d rows of %s, best of 3 "
                     "rounds after 1 warm-up, x100 rounds; measured, not scaled to %d rows"
                     % (rows, wl, WORKLOADS[wl]["rows"])}
    if check:
        # The first round only: from margin 0 both sides take sigmoid(0) = 0.5
        # exactly; later rounds go through the reference harness's libm exp,
        # which can differ by an ulp from this library's deterministic one.
        Xs, ys = gen_rows(wl, 0, rows, device, pin=False)
        out["reference_parity"] = reference_parity(ref, Xs, ys, params_for(wl), 1, 0.5)
        del Xs, ys
    del ref
    model = _full_rows_model(wl, device, (rows, per_round))
    if model:
        out["full_rows_estimate"] = model
    return out


def reference_arm(args, wl, device):
    """--impl reference: every step one boosting round of the reference's CPU
    path (ReferencePath) on the sample, all host threads; value and
    ms_per_step are what the steps measured."""
    import checkers as C
    spec = WORKLOADS[wl]
    if not C.have_reference():
        return {"impl": "reference", "unavailable": "oracle/_ref/libxgbref.so (the reference's functions "
                "compiled for the host) was not built"}
    rows = cpu_sample_rows(wl)
    ref = ReferencePath(wl, rows, device)
    for _ in range(args.warmup):
        ref.round()
    times = [ref.round() for _ in range(args.steps)]
    per_round = float(np.mean(times))
    value = per_round * 1e5
    sample = ("the reference's CPU path (oracle/_ref) on the first %d of %s's %d rows, one round per "
              "step, %d timed steps after %d warm-up, %d host threads; measured on the sample"
              % (rows, wl, spec["rows"], args.steps, args.warmup, cpu_cores()))
    return {"impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(per_round * 1000, 3), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "int64", "data": "synthetic",
            "config": {"workload": wl, "rows": rows, "sample_of_rows": spec["rows"], "cols": spec["cols"],
                       "max_depth": spec["max_depth"], "objective": spec["objective"]},
            "cpu_baseline": {"value": round(value, 1), "unit": UNIT, "cores": cpu_cores(), "kind": "reference",
                             "cpu": cpu_model(),
                             "sample": sample},
            "e2e": {"value": round(value, 1), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def c2_comparison(xgb, core, device, rounds=100, ref_rounds=3):
    """BASELINE's c2 workload (262,144 x 64, depth 8, 100 rounds), where
    north_star asks for 10x over the host CPU, measured in full on both
    sides: this library end to end (DMatrix from pinned host arrays, lazy
    quantisation inside train, as the reference's protocol times it) and on
    the device, and the reference's CPU path on every host thread over all
    262,144 rows."""
    wl = "c2"
    spec = WORKLOADS[wl]
    Xh, yh = gen_rows(wl, 0, spec["rows"], device)
    params = params_for(wl)
    core.synchronize()
    t0 = time.perf_counter()
    bst = xgb.train(params, xgb.DMatrix(Xh, label=yh), rounds)
    core.synchronize()
    e2e_ms = (time.perf_counter() - t0) * 1000 * 100.0 / rounds
    del bst
    d = xgb.DMatrix(Xh, label=yh)
    bst = xgb.Booster(params, [d])
    for i in range(3):
        bst.update(d, i)
    core.synchronize()
    bst.record_event(0)
    for i in range(rounds):
        bst.update(d, 3 + i)
    bst.record_event(1)
    dev_ms = bst.event_elapsed(0, 1) * 100.0 / rounds
    core.synchronize()
    out = {"workload": "c2", "rows": spec["rows"], "cols": spec["cols"], "max_depth": spec["max_depth"],
           "rounds": rounds, "e2e_ms_per_100_rounds": round(e2e_ms, 2),
           "device_ms_per_100_rounds": round(dev_ms, 2)}
    import checkers as C
    if C.have_reference():
        ref = ReferencePath(wl, spec["rows"], device, keep_trees=True)
        ref.round()
        t = float(np.mean([ref.round() for _ in range(ref_rounds)]))
        out["reference_parity"] = reference_parity(ref, Xh, yh, params, ref_rounds + 1, 0.0)
        out.update({"reference_cpu_ms_per_100_rounds": round(t * 1e5, 1), "reference_cpu_cores": cpu_cores(),
                    "reference_cpu_rounds_timed": ref_rounds,
                    "speedup_e2e": round(t * 1e5 / e2e_ms, 1), "speedup_device": round(t * 1e5 / dev_ms, 1),
                    "reference": "the reference's CPU path (oracle/_ref) on all rows; stock XGBoost CPU hist "
                                 "is not installable here"})
    return out


def reference_parity(ref, Xh, yh, params, rounds, base_score):
    """This library's trees against the first `rounds` rounds the reference
    path `ref` has grown from margin 0 with the reference's own functions
    over the same rows (Xh, yh): the same rounds through the library's
    training entry point, with the base_score whose margin is 0, compared
    node for node. A failure here is recorded, never raised: the bench line
    still prints."""
    try:
        import product as P
        p = {k: v for k, v in params.items() if k not in ("device", "tree_method", "seed")}
        trees, _ = P.train(Xh, yh, dict(p, base_score=base_score), rounds)
        want = ref.trees[:len(trees)]
        diff = compare_trees(trees, want)
        return {"rounds": rounds, "rows": int(Xh.shape[0]), "trees": len(trees),
                "nodes": int(sum(len(t) for t in trees)), "identical": diff is None, "first_difference": diff,
                "note": "this library's trees (XGBBTrainHost, margin 0 at the start) against the "
                        "reference's own CPU path on the same rows, node for node"}
    except Exception as e:  # noqa: BLE001 -- recorded in the line instead
        return {"rounds": rounds, "identical": None, "error": "%s: %s" % (type(e).__name__, e)}


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def phase_breakdown(xgb, core, params, dtrain, dist, rounds=3):
    """Milliseconds per round of each phase of the tree levels (histogram,
    reduce-scatter over ranks, split search, best-split gather, partition,
    child counts), from CUDA events around each launch group
    (cuda_profile=2), max over ranks; measured after the timed region on a
    fresh booster, so the extra events do not touch `value`."""
    bst = xgb.Booster(dict(params, cuda_profile=2), [dtrain])
    for i in range(2):
        bst.update(dtrain, i)
    core.synchronize()
    bst.reset_cuda_profile()
    for i in range(rounds):
        bst.update(dtrain, 2 + i)
    prof = bst.cuda_profile()
    out = {k: round(dist.max(v) / rounds, 3) for k, v in prof["phases"].items()}
    levels = [[round(dist.max(v) / rounds, 3) for v in row] for row in prof["level_phases"]]
    del bst
    return {"ms_per_round": out, "per_level_ms": [r for r in levels if any(r)],
            "columns": list(prof["phases"].keys()), "rounds": rounds,
            "note": "CUDA events around each phase on the booster's stream (cuda_profile=2) on a "
                    "fresh booster after the timed region; max over ranks"}


def ncu_traffic(wl):
    """Per-launch DRAM bytes of the histogram kernel from the committed ncu
    summary, scaled to one average launch of this workload, or None."""
    path = os.path.join(ROOT, "profiles", "hist_traffic_%s.json" % wl)
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


# ---------------------------------------------------------------------------
def probe_shared_pipe():
    """SM cycles per warp-level shared instruction for each probe variant, at
    16 and 32 warps per SM: the throughput figures behind the histogram
    kernels' limb scheme."""
    import ctypes
    import xgboost as xgb  # noqa: F401
    from xgboost import core
    names = {0: "red.shared.add.s32 x4", 1: "red.shared.add.s32 x1", 2: "st.shared.b32 x4",
             3: "atom.shared.add.u64 x2"}
    out = {"probe": "shared_pipe", "unit": "SM cycles per warp instruction", "variants": {}}
    for v, name in names.items():
        for warps in (16, 32):
            c = ctypes.c_double()
            core._check_call(core._LIB.XGBBProbeSharedPipe(ctypes.c_int(v), ctypes.c_uint32(warps),
                                                           ctypes.c_uint32(2000), ctypes.byref(c)))
            out["variants"]["%s, %d warps" % (name, warps)] = round(c.value, 3)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c4", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--rows", type=int, default=0,
                    help="override the row count (small profiling cases only; not a bench line)")
    ap.add_argument("--probe", action="store_true",
                    help="measure the shared-memory pipe (XGBBProbeSharedPipe) instead of training")
    args = ap.parse_args()
    if args.probe:
        print(json.dumps(probe_shared_pipe()), flush=True)
        return
    assert args.warmup >= 3, "at least 3 warm-up rounds"
    dist = Dist()
    wl = args.workload
    if args.rows:
        WORKLOADS[wl] = dict(WORKLOADS[wl], rows=args.rows)
    spec = WORKLOADS[wl]
    import torch
    device = torch.device("cuda", dist.local)
    torch.cuda.set_device(device)

    if args.impl == "reference":
        if dist.rank == 0:
            print(json.dumps(reference_arm(args, wl, device)), flush=True)
        dist.close()
        return

    import xgboost as xgb
    from xgboost import core
    core.set_device(dist.local)
    if dist.world > 1:
        # One node: NCCL bootstrap on loopback; data moves over NVLink.
        os.environ.setdefault("NCCL_SOCKET_IFNAME", "lo")
        uid = dist.bcast(xgb.collective.nccl_unique_id() if dist.rank == 0 else None)
        xgb.collective.init(rank=dist.rank, world_size=dist.world, nccl_unique_id=uid,
                            device=dist.local)

    begin, end = shard(spec["rows"], dist.rank, dist.world)
    t = time.perf_counter()
    Xh, yh = gen_rows(wl, begin, end, device)
    log("rank %d: rows [%d, %d) generated in %.1fs" % (dist.rank, begin, end, time.perf_counter() - t))
    t = time.perf_counter()
    digest = data_digest(Xh, yh, spec["rows"], dist)
    log("rank %d: data digest in %.1fs" % (dist.rank, time.perf_counter() - t))
    params = params_for(wl)
    K, W = args.steps, args.warmup
    groups = groups_of(wl)

    # End to end through the public API from pinned host arrays: ingest (the
    # H2D copy, the quantile sketch of every row -- over all ranks' rows, on
    # every GPU, when sharded -- and binning; a plain DMatrix does this lazily
    # in the first round), then K rounds, each reading its trees back.
    dist.barrier()
    core.synchronize()
    t0 = time.perf_counter()
    if wl in ("c4", "c3"):
        dtrain = xgb.QuantileDMatrix(Xh, label=yh, max_bin=256)
    else:
        dtrain = xgb.DMatrix(Xh, label=yh)
    core.synchronize()
    t1 = time.perf_counter()
    stamps = []

    class _Stamp(xgb.callback.TrainingCallback):
        # Wall clock at the end of each round (rounds are enqueued
        # asynchronously, so this is when the host was done with a round).
        def after_iteration(self, model, epoch, evals_log):
            stamps.append(time.perf_counter())
            return False

    bst = xgb.train(params, dtrain, K, callbacks=[_Stamp()])
    core.synchronize()
    t2 = time.perf_counter()
    e2e_ms = dist.max((t2 - t0) * 1000)
    ingest_ms = dist.max((t1 - t0) * 1000)
    rounds_ms = dist.max((t2 - t1) * 1000)
    # The first round also allocates the training state and captures the
    # CUDA graphs; the rest replay them.
    first_round_ms = dist.max((stamps[0] - t1) * 1000) if stamps else 0.0
    later_round_ms = dist.max((t2 - stamps[0]) * 1000 / max(K - 1, 1)) if len(stamps) > 1 else 0.0
    del bst

    # Device-resident: a fresh booster on the quantised matrix, W warm-up
    # rounds, then K rounds between CUDA events on the booster's stream.
    bst = xgb.Booster(dict(params, cuda_profile=1), [dtrain])
    for i in range(W):
        bst.update(dtrain, i)
    dist.barrier()
    core.synchronize()
    bst.reset_cuda_profile()
    with ClockSampler(dist.local) as clocks:
        bst.record_event(0)
        for i in range(K):
            bst.update(dtrain, W + i)
        bst.record_event(1)
        dev_ms = bst.event_elapsed(0, 1)
        core.synchronize()
    dev_ms = dist.max(dev_ms)
    prof = bst.cuda_profile()
    parity = parity_digest(bst, dtrain, dist, W + K)
    value = dev_ms * 100.0 / K
    del bst
    phases = phase_breakdown(xgb, core, params, dtrain, dist)

    peak, peak_kind = measured_peak()
    hist_gbs = prof["hist_bytes"] / prof["hist_ms"] / 1e6 if prof["hist_ms"] > 0 else 0.0
    traffic = ncu_traffic(wl)
    roofline = {"bound": "hbm", "achieved": round(hist_gbs, 1), "peak": peak, "unit": "GB/s",
                "frac": round(hist_gbs / peak, 4), "peak_kind": peak_kind,
                "traffic": traffic["dram_bytes_per_launch"] if traffic else None,
                "kernel": "hist2_kernel",
                "algorithmic_bytes_per_launch": prof["hist_bytes"] / max(prof["hist_launches"], 1),
                "avg_launch_ms": prof["hist_ms"] / max(prof["hist_launches"], 1),
                "launches": prof["hist_launches"],
                "hist_ms_per_round": prof["hist_ms"] / K,
                "per_level_ms_mrows": [[round(ms / K, 3), round(rows / K / 1e6, 3)]
                                       for ms, rows, _ in prof.get("levels", []) if rows]}

    cpu, c2 = None, None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        # c2 runs before the CPU legs, with c4's matrix released, so that
        # neither c4's memory nor the CPU legs' load reaches its timings.
        del dtrain
        if wl == "c4" and not args.rows:
            c2 = c2_comparison(xgb, core, device)
        cpu = cpu_baseline_leg(wl, device)

    bytes_per_code = 2 if (spec["nan"] > 0) else 1
    x_bytes = Xh.nbytes + yh.nbytes
    node_table = groups * ((2 << spec["max_depth"]) - 1) * 48 + 32 + 2 * 10 * 12
    out = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": dist.world,
        "steps": K, "warmup": W, "ms_per_step": round(dev_ms / K, 4), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "int64",
        "data": "synthetic (seeded per 1M-row chunk, generated on the GPU)",
        "config": {"workload": wl + ("-rows%d" % args.rows if args.rows else ""),
                   "rows": spec["rows"], "cols": spec["cols"],
                   "objective": spec["objective"], "max_depth": spec["max_depth"],
                   "max_bin": 256, "eta": spec["eta"], "nan_fraction": spec["nan"],
                   "bins": "uint%d ELLPACK" % (8 * bytes_per_code),
                   "parallelism": "row-shard dp%d" % dist.world,
                   "cuts": "sketch of every row (GPU sketch; over all ranks' rows when sharded)",
                   "l2": "inputs larger than L2 (quantised matrix %.1f GB)"
                         % (spec["rows"] * spec["cols"] * bytes_per_code / 1e9)},
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_ms * 100.0 / K, 3), "unit": UNIT,
                "h2d_bytes_per_step": int(x_bytes / K), "d2h_bytes_per_step": node_table,
                "ingest_ms": round(ingest_ms, 1), "per_round_ms": round(rounds_ms / K, 3), "rounds": K,
                "first_round_ms": round(first_round_ms, 1), "later_round_ms": round(later_round_ms, 3),
                "note": "QuantileDMatrix (c3, c4) or DMatrix from pinned host arrays, then xgb.train for "
                        "K rounds; wall clock, max over ranks. ingest = H2D + sketch of all rows + "
                        "binning; the ingest is amortised over K rounds in value"},
        "parity": parity,
        "data_digest": digest,
        "phases": phases,
        "c2": c2,
        "gpu_launches": launches_per_round(spec, dist.world, end - begin) * K,
        "clocks": clocks.summary(),
    }
    if dist.rank == 0:
        print(json.dumps(out), flush=True)
    if dist.world > 1:
        xgb.collective.finalize()
    dist.close()


if __name__ == "__main__":
    main()
