"""Benchmark: boosting rounds/s of the reference's binary-logloss path on B200.

Workload (BASELINE.json metric "boosting rounds/sec at 1M x 100 depth 6"):
config 4's data -- 1,000,000 x 100 float32, 30 % NaN, 60 N(0,1) / 30 Exp(1) /
10 integer-level columns, 99/1 sparse-logistic label (seeded synthetic
stand-in) -- binned with the reference's rules (255 bins + NaN bin), trained
with max_depth 6, 63 leaves, lr 0.08, subsample 0.75, colsample 0.7,
min_child_weight 3, lambda 1, class_weight balanced_sqrt (power 0.35).

A step is one boosting round: the reference's row/feature sampler, the tree
(gradients, histograms, splits, partitions), the F update and the train
logloss.  `value` times K rounds on the binned matrix already resident in
HBM, queued back to back through gbm_fit_rounds (device CUDA events on the
engine stream; every round starts with a 256 MB L2-evicting write whose
device time is measured and excluded);
`e2e` times the public estimator API (`fit_binned`) from host arrays,
including the upload of the binned matrix and every round's mask/tree
copies.  Rows are sharded over N GPUs (one process per GPU, NCCL allreduce
of the exact histogram words), so the total work is fixed: strong scaling.

--impl reference times the reference's algorithm on the host cores instead:
the CPU oracle (a C restatement of the reference's Numba path, OpenMP over
features like its prange), the same config and metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "bsscl-gbm_b200"), os.path.join(ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

CONFIGS = {
    # the headline: BASELINE's metric (1M x 100 at depth 6) on configs[3]'s data
    "4": dict(n=1_000_000, p=100, max_depth=6, max_leaves=63, lr=0.08, subsample=0.75, colsample=0.7,
              mcw=3.0, lam=1.0, msl=5, class_weight="balanced_sqrt", seed=0,
              metric="boosting rounds/sec at 1M x 100 depth 6",
              workload="config4 1M x 100 f32 30% NaN, depth 6, 63 leaves",
              data="synthetic (config 4 stand-in, seed 3)", cpu_rows=None),
    # the box-scale case (training part) for the scaling study
    "5": dict(n=10_000_000, p=200, max_depth=10, max_leaves=63, lr=0.08, subsample=0.5, colsample=0.7,
              mcw=3.0, lam=5.0, msl=5, class_weight="balanced_sqrt", seed=0,
              metric="boosting rounds/sec at 10M x 200 depth 10",
              workload="config5 10M x 200 pre-binned uint8 U{1..254} + 10% NaN bin, depth 10, 63 leaves",
              data="synthetic (config 5 stand-in, seed 5)", cpu_rows=1_000_000),
}
CFG = CONFIGS["4"]
METRIC = CFG["metric"]


def workload(cfg, rows=None):
    """(X_bin, y, counts): config 4's data binned exactly as the reference bins
    it (all rows), or config 5's pre-binned rows `rows` (default all)."""
    from bsscl_gbm_b200 import binning, datasets
    if cfg is CONFIGS["5"]:
        Xb, y = datasets.config5_bins(n=cfg["n"], p=cfg["p"], rows=rows)
        return Xb, y, np.full(cfg["p"], 256, np.int32)
    X, y = datasets.config4(n=cfg["n"])
    edges, counts, nanb = binning.build_bin_edges(X, 255)
    Xb = binning.bin_features(X, edges, counts, nanb)
    return Xb, y, counts


def bin_on_gpu(eng, X, lo, hi):
    """Config 4's edges and bins made on the GPU: gbm_bin_edges over all rows,
    gbm_upload_binned_rows for this rank's rows (the training matrix), and
    gbm_bin_features for the host copy of the ids that the estimator arm and
    the CPU baseline use.  Host wall times of each step (edges include the
    host -> device copy of X); the edges run twice and the second is kept."""
    t0 = time.perf_counter()
    eng.bin_edges(X, 255)
    t1 = time.perf_counter()
    edges, counts, nanb = eng.bin_edges(X, 255)
    t2 = time.perf_counter()
    eng.upload_binned_rows(lo, hi, edges, counts, nanb)
    eng.sync()
    t3 = time.perf_counter()
    Xb = eng.bin_features(X, edges, counts, nanb)
    t4 = time.perf_counter()
    stats = {"edges_ms": (t2 - t1) * 1e3, "edges_first_call_ms": (t1 - t0) * 1e3,
             "bin_into_engine_ms": (t3 - t2) * 1e3, "raw_ids_to_host_ms": (t4 - t3) * 1e3,
             "x_bytes": int(X.nbytes), "rows": int(X.shape[0]), "features": int(X.shape[1]),
             "note": "host wall times of gbm_bin_edges (sample_weight=None, n_bins 255), "
                     "gbm_upload_binned_rows and gbm_bin_features (uint16 ids to host)"}
    return Xb, counts, stats


class Clocks:
    """SM clock and throttle reasons sampled DURING the timed region: NVML
    (read only) polled every 2 ms from a thread; nvidia-smi as a fallback."""
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.thread = None
        self.samples = []
        self.stop_flag = False
        self.nv = None

    def _poll(self, h):
        nv = self.nv
        while not self.stop_flag:
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((sm, mx, rs))
            except Exception:
                pass
            time.sleep(0.002)

    def start(self):
        try:
            import pynvml as nv
            import threading
            nv.nvmlInit()
            self.nv = nv
            uuid = None
            try:
                import torch
                uuid = str(torch.cuda.get_device_properties(self.index).uuid)
            except Exception:
                pass
            h = None
            if uuid:
                try:
                    h = nv.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
                except Exception:
                    h = None
            if h is None:
                h = nv.nvmlDeviceGetHandleByIndex(self.index)
            self.thread = threading.Thread(target=self._poll, args=(h,), daemon=True)
            self.thread.start()
            return
        except Exception:
            self.nv = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self.stop_flag = True
            self.thread.join()
            if not self.samples:
                return None
            reasons = set()
            for _, _, rs in self.samples:
                for name, attr in self.REASONS:
                    bit = getattr(self.nv, attr, None)
                    if bit is not None and rs & bit:
                        reasons.add(name)
            return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                    "sm_max_mhz": max(s[1] for s in self.samples), "reasons": sorted(reasons),
                    "samples": len(self.samples), "source": "NVML, every 2 ms during the timed region"}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for k, nm in enumerate(names):
                if f[5 + k].lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi -lms 100"}


def parity_check(res, first_round, record):
    """The timed rounds against the reference's own fit of the same workload,
    recorded at full size (tests/golden/fit_full_<record>.npz, made by
    tests/golden/make_golden_full.py): round first_round + i of this run is
    round first_round + i of that fit.  Topology (features, thresholds,
    children, node count) must be identical, leaf values within 1e-6 and
    train losses within 1e-9.  Rounds past the record are not checked."""
    path = os.path.join(ROOT, "tests", "golden", f"fit_full_{record}.npz")
    if not os.path.exists(path):
        return {"checked_rounds": 0, "ok": None, "note": f"no record {os.path.basename(path)}"}
    d = np.load(path)
    T = int(d["n_trees"])
    topo_ok, max_dv, max_dl, k = True, 0.0, 0.0, 0
    for i, (tree, loss) in enumerate(res):
        t = first_round + i
        if t >= T:
            break
        k += 1
        nc = int(d["nc"][t])
        if tree[5] != nc or any(not np.array_equal(np.asarray(tree[j])[:nc], d[key][t][:nc])
                                for j, key in ((0, "tf"), (1, "tt"), (3, "tl"), (4, "tr"))):
            topo_ok = False
        max_dv = max(max_dv, float(np.abs(np.asarray(tree[2])[:nc] - d["tv"][t][:nc]).max()))
        max_dl = max(max_dl, abs(loss - float(d["train_loss"][t])))
    return {"checked_rounds": k, "first_round": first_round, "topology_identical": topo_ok,
            "max_leaf_value_diff": max_dv, "max_train_loss_diff": max_dl,
            "ok": bool(k > 0 and topo_ok and max_dv <= 1e-6 and max_dl <= 1e-9),
            "record": f"the reference's fit recorded in tests/golden/fit_full_{record}.npz ({T} rounds)"}


# The shared-memory atomic ceiling of the histogram's update pattern, measured
# on this pool's B200s with a microbenchmark (2 CTAs x 512 threads per SM,
# 148 SMs, 32-bit atomicAdd on shared memory): 2.97 T lane-atomics/s with
# k_hist's layout (6 digit arrays x 16 features x 256 bins, uniform random
# bins) and 9.05 T/s conflict-free (one warp instruction per SM clock).
SMEM_ATOMIC_PEAK = {"random_bins_g_per_s": 2968, "conflict_free_g_per_s": 9054}

# The CPU port (oracle.c, REF mode) against the reference's own Numba fit,
# measured in the build container with oracle/calibrate_port.py: config 4's
# data at 1,000,000 x 100, bench parameters, 10 trees, 8 threads each, the
# same tree topology.  The port is the faster of the two, so ratios against
# the reference arm (the port) understate the speed-up over the reference.
PORT_CALIBRATION = {"rows": 1_000_000, "trees": 10, "threads": 8, "reference_rounds_per_s": 0.942,
                    "port_rounds_per_s": 1.359, "port_over_reference": 1.442, "same_topology": True,
                    "how": "oracle/calibrate_port.py"}

# DRAM traffic of the histogram kernel per launch on this workload, from one
# ncu capture (dram__bytes_read.sum + dram__bytes_write.sum over the six
# histogram launches of one round, averaged).  A constant here, since a
# capture cannot run inside the timed run; the capture is named in `source`.
HIST_TRAFFIC = {"dram_bytes_per_launch": 88251989,
                "source": "ncu capture (dram__bytes_read.sum + dram__bytes_write.sum, cold cache) of the six "
                          "k_hist3 launches of one timed config-4 round of this build, averaged per launch"}


def measured_peak_hbm():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def cpu_rounds(Xb, y, counts, rounds, warmup=1, budget_s=None):
    """The reference's loop on the CPU oracle (REF mode): rounds/s of the
    given rows."""
    import oracle as O
    c = CFG
    kw = dict(learning_rate=c["lr"], max_leaves=c["max_leaves"], max_depth=c["max_depth"],
              min_samples_leaf=c["msl"], min_child_weight=c["mcw"], reg_lambda=c["lam"],
              gamma=0.0, subsample=c["subsample"], colsample=c["colsample"],
              class_weight=c["class_weight"], random_state=c["seed"], mode=O.MODE_REF)
    O.fit_binary(Xb, y, counts, n_estimators=warmup, **kw)
    t0 = time.perf_counter()
    done = 0
    while True:
        O.fit_binary(Xb, y, counts, n_estimators=1, **kw)
        done += 1
        el = time.perf_counter() - t0
        if done >= rounds or (budget_s is not None and el > budget_s):
            break
    # each call also pays one base-score/gradient pass; that is part of a round anyway
    return done / el, done, O.num_threads()


def run_reference(args):
    """--impl reference: the reference's algorithm (CPU oracle) on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle as O
    c = CFG
    m = c["cpu_rows"] or c["n"]
    Xb, y, counts = workload(c, rows=(0, m))
    y = y[:m]
    kw = dict(learning_rate=c["lr"], max_leaves=c["max_leaves"], max_depth=c["max_depth"],
              min_samples_leaf=c["msl"], min_child_weight=c["mcw"], reg_lambda=c["lam"],
              gamma=0.0, subsample=c["subsample"], colsample=c["colsample"],
              class_weight=c["class_weight"], random_state=c["seed"], mode=O.MODE_REF)
    O.fit_binary(Xb, y, counts, n_estimators=max(1, args.warmup), **kw)
    t0 = time.perf_counter()
    O.fit_binary(Xb, y, counts, n_estimators=args.steps, **kw)
    el = time.perf_counter() - t0
    # a row sample's rounds/s scaled to the full row count (a round's work is linear in rows)
    v = args.steps / el * (m / c["n"])
    sample = (f"{args.steps} rounds of the full workload" if m == c["n"] else
              f"{args.steps} rounds on the first {m:,} of {c['n']:,} rows, rounds/s scaled by {m / c['n']:g}")
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "rounds/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 / v, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f64", "data": c["data"],
        "config": {"workload": c["workload"], "n_rows": c["n"], "n_features": c["p"],
                   "max_depth": c["max_depth"], "max_leaves": c["max_leaves"], "subsample": c["subsample"],
                   "colsample": c["colsample"]},
        "cpu_baseline": {"value": v, "unit": "rounds/s", "cores": O.num_threads(), "kind": "port",
                         "sample": sample, "calibration": PORT_CALIBRATION},
        "e2e": {"value": v, "unit": "rounds/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config5_subrecord(eng, args, world, rank, local, dist):
    """configs[4]'s training at this run's GPU count: 10,000,000 x 200
    pre-binned rows sharded over the ranks (each rank makes only its own
    rows), max_depth 10, 63 leaves, subsample 0.5, colsample 0.7, lambda 5,
    rounds queued back to back (gbm_fit_rounds), device-timed, max over
    ranks.  Rows are drawn by the throughput-mode device sampler
    (gbm_sampler_create_device): the reference's cumulative shuffle of 10M
    rows costs ~7 ms of host time per round on every rank, which would cap
    every GPU count at ~140 rounds/s.  Throughput only: no parity claim."""
    import torch
    from bsscl_gbm_b200 import GbmParams, Sampler
    import oracle as O
    c = CONFIGS["5"]
    n = c["n"]
    lo, hi = (n * rank) // world, (n * (rank + 1)) // world
    Xb, y, counts = workload(c, rows=(lo, hi))
    p = Xb.shape[1]
    w2 = O.class_weights(y, c["class_weight"])
    base = O.base_score(y, w2)
    eng.upload_bins(Xb, counts)
    del Xb
    eng.upload_labels(y[lo:hi].astype(np.uint8), w2, base, n_global=n)
    prm = GbmParams(c["lam"], 0.0, c["mcw"], c["lr"], c["msl"], c["max_depth"], c["max_leaves"], 0, None)
    cap = 2 * c["max_leaves"] + 2
    smp = Sampler.device(c["seed"], n, p, c["subsample"], int(p * c["colsample"]), True, look_ahead=3)
    eng.set_l2_flush(256 << 20)
    eng.set_profiling(True)
    eng.fit_rounds(smp, lo, prm, cap, args.warmup)
    eng.reset_stats()
    k = args.config5_steps
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    eng.event(8)
    res = eng.fit_rounds(smp, lo, prm, cap, k)
    eng.event(9)
    eng.sync()
    st = eng.stats()
    eng.set_profiling(False)
    eng.set_l2_flush(0)
    ms = eng.elapsed_ms(8, 9) - st["flush_ms"]
    if dist is not None:
        t = torch.tensor([ms], device=f"cuda:{local}", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    smp.close()
    return {"value": k / (ms / 1000.0), "unit": "rounds/s", "ms_per_step": ms / k, "steps": k,
            "scaling": "strong", "n_gpus": world, "hist_ms_per_round": st["hist_ms"] / k,
            "collectives_device_ms_per_round": st["comm_ms"] / k,
            "collective_mb_per_round": st["comm_bytes"] / k / 1e6,
            "train_loss_last": res[-1][1] if res else None,
            "sampler": "throughput-mode device sampler (each row in-bag with probability 0.5 by a "
                       "counter-based hash; gbm_sampler_create_device), not the reference's shuffle",
            "config": {"workload": c["workload"], "n_rows": n, "n_features": p, "max_depth": c["max_depth"],
                       "max_leaves": c["max_leaves"], "subsample": c["subsample"], "colsample": c["colsample"]}}


def other_objectives(eng, local, X, y, c, rounds=20):
    """The estimator's other device objectives on config 4's rows, `rounds`
    rounds each: multi-class softmax over 3 classes (3 trees a round,
    gbm_round_mc) and mse regression (gbm_round_reg), config 4's tree
    parameters.  Both run one round per engine call, with no pipelining across
    rounds; the figure is the host wall time of the rounds (the estimator's
    times['rounds']).  The labels are synthetic functions of the rows."""
    from bsscl_gbm_b200 import HybridHistGBMNumbaV1_0_1
    f0 = np.nan_to_num(X[:, 0].astype(np.float64), nan=0.0)
    f1 = np.nan_to_num(X[:, 1].astype(np.float64), nan=0.0)
    y3 = y.astype(np.int64) + (f0 > np.median(f0)).astype(np.int64)
    yr = f0 + 0.5 * f1 + 0.1 * y.astype(np.float64)
    common = dict(n_estimators=rounds, max_depth=c["max_depth"], learning_rate=c["lr"],
                  min_child_weight=c["mcw"], subsample=c["subsample"], colsample_bytree=c["colsample"],
                  reg_lambda=c["lam"], n_bins=255, random_state=c["seed"], verbose=False)
    out = {}
    for name, kw, target in [("multiclass_3", {}, y3),
                             ("regression_mse", {"objective": "regression", "loss": "mse"}, yr)]:
        m = HybridHistGBMNumbaV1_0_1(**common, **kw)
        m._engine, m._engine_dev = eng, local
        m.fit(X, target)
        ms = m.times["rounds"]
        out[name] = {"value": rounds / (ms / 1000.0), "unit": "rounds/s", "rounds": rounds,
                     "ms_per_round": ms / rounds}
    out["note"] = ("HybridHistGBMNumbaV1_0_1.fit on config 4's 1M x 100 rows (3 synthetic classes; a "
                   "synthetic float target), one round per engine call; host wall time of the rounds")
    return out


def run_engine(args):
    import torch
    from bsscl_gbm_b200 import Engine, GbmParams, HybridHistGBMNumbaV1_0_1, Sampler, binning
    import oracle as O

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    c = CFG
    n = c["n"]
    lo, hi = (n * rank) // world, (n * (rank + 1)) // world
    five = c is CONFIGS["5"]
    eng = Engine(local)
    if world > 1:
        uid = [Engine.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        eng.init_comm(uid[0], world, rank, timeout_ms=120000)
    bin_stats = None
    X = None
    if five:
        # each rank makes only its rows (2 GB per 10M x 200)
        Xb, y, counts = workload(c, rows=(lo, hi))
        Xl = Xb
        eng.upload_bins(Xl, counts)
    else:
        # config 4: raw float32 rows, binned on the GPU
        from bsscl_gbm_b200 import datasets
        X, y = datasets.config4(n=n)
        Xb, counts, bin_stats = bin_on_gpu(eng, X, lo, hi)
        Xl = Xb[lo:hi]
    p = Xb.shape[1]
    w2 = O.class_weights(y, c["class_weight"])
    base = O.base_score(y, w2)
    Xd = binning.device_bins(Xl, counts)
    eng.upload_labels(y[lo:hi].astype(np.uint8), w2, base, n_global=n)
    prm = GbmParams(c["lam"], 0.0, c["mcw"], c["lr"], c["msl"], c["max_depth"], c["max_leaves"], 0,
                    None)
    cap = 2 * c["max_leaves"] + 2
    n_sub, n_feat = int(n * c["subsample"]), int(p * c["colsample"])
    sampler = Sampler(c["seed"], n, p, n_sub, n_feat, True, True, look_ahead=3)
    # L2 eviction at the start of every round: a 256 MB write on the engine
    # stream (B200 L2 is 126 MB), timed separately and taken out of the total
    eng.set_l2_flush(256 << 20)
    eng.set_profiling(True)     # before the warm-up: the timed rounds reuse its captured graphs
    eng.fit_rounds(sampler, lo, prm, cap, args.warmup)
    eng.reset_stats()
    clocks = Clocks(local)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    # the K rounds are queued back to back (gbm_fit_rounds: the host waits
    # only for the round four places back); CUDA events on the engine stream
    eng.event(0)
    # an NVTX range around the timed rounds: ncu --nvtx --nvtx-include "bench_timed_rounds/"
    # captures only their launches
    torch.cuda.nvtx.range_push("bench_timed_rounds")
    res = eng.fit_rounds(sampler, lo, prm, cap, args.steps)
    torch.cuda.nvtx.range_pop()
    eng.event(1)
    eng.sync()
    torch.cuda.synchronize()
    clk = clocks.stop()
    losses = [r[1] for r in res]
    if args.part == "rounds":   # profiling aid: the timed rounds alone
        st = eng.stats()
        ms = eng.elapsed_ms(0, 1) - st["flush_ms"]
        if rank == 0:
            print(json.dumps({"part": "rounds", "workload": c["workload"], "rounds": args.steps,
                              "ms_per_round": ms / args.steps, "rounds_per_s": args.steps / (ms / 1000.0),
                              "hist_launches": st["hist_launches"], "hist_ms": st["hist_ms"],
                              "hist_alg_bytes": st["hist_alg_bytes"], "kernel_launches": st["kernel_launches"],
                              "sampler_ms": st["sampler_ms"] / args.steps,
                              "engine_wait_for_sampler_ms": st["sampler_stall_ms"] / args.steps}),
                  flush=True)
        sampler.close()
        eng.close()
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return
    # the timed rounds are rounds W .. W+K-1 of one fit: compare them with the
    # reference's own fit of this workload (config 4 at depth 6)
    parity = parity_check(res, args.warmup, "cfg4_d6") if not five else {
        "checked_rounds": 0, "ok": None, "note": "config 5 computes f32-quantised inputs: throughput only"}
    if dist is not None:
        dist.barrier()
    st = eng.stats()
    eng.set_profiling(False)
    wall_ms = eng.elapsed_ms(0, 1)
    total_ms = wall_ms - st["flush_ms"]
    if dist is not None:
        t = torch.tensor([total_ms], device=f"cuda:{local}", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    value = args.steps / (total_ms / 1000.0)

    # ---- configs[3] literally: the same data at max_depth 8 (config 4 only) -------
    d8_ms = None
    if not five:
        prm8 = GbmParams(c["lam"], 0.0, c["mcw"], c["lr"], c["msl"], 8, c["max_leaves"], 0, None)
        s8 = Sampler(c["seed"], n, p, n_sub, n_feat, True, True, look_ahead=3)
        eng.upload_labels(y[lo:hi].astype(np.uint8), w2, base, n_global=n)
        eng.set_profiling(True)
        eng.fit_rounds(s8, lo, prm8, cap, args.warmup)
        if dist is not None:
            dist.barrier()
        eng.reset_stats()
        eng.event(6)
        eng.fit_rounds(s8, lo, prm8, cap, args.steps)
        eng.event(7)
        eng.sync()
        st8 = eng.stats()
        eng.set_profiling(False)
        d8_ms = eng.elapsed_ms(6, 7) - st8["flush_ms"]
        if dist is not None:
            t = torch.tensor([d8_ms], device=f"cuda:{local}", dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            d8_ms = float(t.item())
        s8.close()
    eng.set_l2_flush(0)

    # ---- e2e: the public estimator API from host arrays ----------------------
    m = HybridHistGBMNumbaV1_0_1(n_estimators=args.steps, max_depth=c["max_depth"],
                                 learning_rate=c["lr"], min_child_weight=c["mcw"],
                                 subsample=c["subsample"], colsample_bytree=c["colsample"],
                                 reg_lambda=c["lam"], class_weight=c["class_weight"],
                                 random_state=c["seed"], verbose=False)
    m.max_leaves = c["max_leaves"]
    m._engine, m._engine_dev = eng, local
    e2e = None
    e2e_parts = None
    if not (five and world > 1):   # the estimator takes every row on every rank
        if dist is not None:
            dist.barrier()
        eng.event(2)
        m.fit_binned(Xb, y, counts)
        eng.event(3)
        e2e_ms = eng.elapsed_ms(2, 3)
        if dist is not None:
            t = torch.tensor([e2e_ms], device=f"cuda:{local}", dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = float(t.item())
        e2e = args.steps / (e2e_ms / 1000.0)
        e2e_parts = {"total_ms": e2e_ms, "upload_ms": m.times["upload"], "rounds_ms": m.times["rounds"],
                     "training_ms": m.times["training"]}
    # ---- the whole public fit from raw float32 rows (binning on the GPU) -------
    fit_raw = None
    if X is not None:
        m2 = HybridHistGBMNumbaV1_0_1(n_estimators=args.steps, max_depth=c["max_depth"],
                                      learning_rate=c["lr"], min_child_weight=c["mcw"],
                                      subsample=c["subsample"], colsample_bytree=c["colsample"],
                                      reg_lambda=c["lam"], class_weight=c["class_weight"], n_bins=255,
                                      random_state=c["seed"], verbose=False)
        m2._engine, m2._engine_dev = eng, local
        if dist is not None:
            dist.barrier()
        t0 = time.perf_counter()
        m2.fit(X, y)
        fit_s = time.perf_counter() - t0
        fit_raw = {"seconds": fit_s, "rounds": args.steps, "binning_ms": m2.times["binning"],
                   "training_ms": m2.times["training"],
                   "note": "HybridHistGBMNumbaV1_0_1.fit(X float32 [n, p], y) wall time on this rank: "
                           "adaptive hyper-parameters, GPU edges and bins, labels, the rounds"}
    other = other_objectives(eng, local, X, y, c) if X is not None and world == 1 else None
    rows = hi - lo
    nblk = (p + 15) // 16
    # once per fit: bins (1 byte per id: uint16 ids are narrowed on the host
    # as they stream through the pinned buffers), labels, bin counts; every
    # round: the global row sample's swap targets and the feature tables
    once = rows * p + rows + 4 * p
    per_round = 4 * (n - 1) + 4 * n_feat + 2 * 16 * nblk + 4 * nblk
    h2d = once / args.steps + per_round
    d2h = 9240 + 8                          # the tree record and the loss

    # ---- predict rows/s (device-resident rows and ensemble) ----------------------
    from bsscl_gbm_b200 import datasets
    ens = datasets.config5_ensemble(n_trees=1000, depth=8, p=p, seed=5)
    eng.predict_set_model(ens, 1000, p)
    eng.predict_upload(Xd)
    eng.predict_run(c["lr"], base)
    eng.sync()
    eng.event(4)
    reps = 3
    for _ in range(reps):
        eng.predict_run(c["lr"], base)
    eng.event(5)
    pred_ms = eng.elapsed_ms(4, 5) / reps
    if dist is not None:
        t = torch.tensor([pred_ms], device=f"cuda:{local}", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pred_ms = float(t.item())
    pred_rows_s = n / (pred_ms / 1000.0)

    # ---- configs[4] at this GPU count (a sub-record of every config-4 line) --------
    c5 = None
    if not five and not args.no_config5:
        c5 = config5_subrecord(eng, args, world, rank, local, dist)

    peak, peak_kind = measured_peak_hbm()
    achieved = (st["hist_alg_bytes"] / (st["hist_ms"] / 1000.0)) / 1e9 if st["hist_ms"] > 0 else 0.0
    atomics = None
    if st["hist_ms"] > 0:
        g = 6 * st["hist_updates"] / (st["hist_ms"] / 1000.0) / 1e9
        atomics = {"achieved_g_per_s": g, "unit": "G shared-memory atomic adds/s",
                   "peak_random_bins_g_per_s": SMEM_ATOMIC_PEAK["random_bins_g_per_s"],
                   "peak_conflict_free_g_per_s": SMEM_ATOMIC_PEAK["conflict_free_g_per_s"],
                   "frac_of_conflict_free_peak": g / SMEM_ATOMIC_PEAK["conflict_free_g_per_s"],
                   "source": "microbenchmark of 32-bit shared-memory atomicAdd on this pool's B200s"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        mr = c["cpu_rows"] or n
        v_cpu, done, cores = cpu_rounds(Xb[:mr], y[:mr], counts, rounds=50, warmup=1, budget_s=20.0)
        v_cpu *= mr / n
        cpu = {"value": v_cpu, "unit": "rounds/s", "cores": cores, "kind": "port",
               "sample": (f"{done} rounds of the full workload on the CPU oracle (REF mode)" if mr == n else
                          f"{done} rounds on the first {mr:,} of {n:,} rows on the CPU oracle (REF mode), "
                          f"rounds/s scaled by {mr / n:g}")}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "rounds/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
            "data": c["data"],
            "config": {"workload": c["workload"],
                       "n_rows": n, "n_features": p, "max_depth": c["max_depth"],
                       "max_leaves": c["max_leaves"], "subsample": c["subsample"],
                       "colsample": c["colsample"]},
            "run": {"parallelism": f"rows sharded x{world}",
                    "l2": "flushed at the start of every timed round (256 MB write on the "
                          "engine stream; its device time is excluded)"},
            "parity": parity,
            "roofline": {"bound": "hbm", "kernel": "k_hist3 (every histogram launch of the round, on the "
                                                   "round's selected features packed into 16-feature blocks)",
                         "achieved": achieved, "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": achieved / peak if peak else None,
                         "traffic": None if five else HIST_TRAFFIC["dram_bytes_per_launch"],
                         "traffic_source": None if five else HIST_TRAFFIC["source"],
                         "alg_bytes_per_launch": st["hist_alg_bytes"] / max(1, st["hist_launches"]),
                         "hist_launches": st["hist_launches"], "hist_ms": st["hist_ms"],
                         "alg_bytes": st["hist_alg_bytes"],
                         "smem_atomics": atomics},
            "breakdown_ms_per_round": {
                "hist_kernel": st["hist_ms"] / args.steps,
                "host_wait_sampler": st["host_sample_ms"] / args.steps,
                "host_wait_device": st["host_sync_ms"] / args.steps,
                "host_replay": st["host_replay_ms"] / args.steps,
                "host_collective_calls": st["host_comm_ms"] / args.steps,
                "collectives_device": st["comm_ms"] / args.steps,
                "collective_mb": st["comm_bytes"] / args.steps / 1e6,
                "peer_wait": st["peer_wait_ms"] / args.steps,
                "l2_flush_excluded": st["flush_ms"] / args.steps,
                "sampler_stream_device": st["sampler_ms"] / args.steps,
                "engine_wait_for_sampler_device": st["sampler_stall_ms"] / args.steps,
                "waves": st["waves"] / args.steps},
            "e2e": ({"value": e2e, "unit": "rounds/s", "h2d_bytes_per_step": int(h2d),
                     "d2h_bytes_per_step": int(d2h), "parts_ms": e2e_parts} if e2e is not None else
                    {"value": None, "note": "the estimator takes every row on every rank; config 5 ranks "
                                            "hold only their own rows"}),
            "gpu_launches": st["kernel_launches"],
            "predict": {"rows_per_s": pred_rows_s, "node_visits_per_s": pred_rows_s * 1000 * 8,
                        "ensemble": f"1000 full depth-8 random trees (config 5 ensemble, p={p})"},
            "train_loss_last": losses[-1] if losses else None,
            "config4_depth8": ({"value": args.steps / (d8_ms / 1000.0), "unit": "rounds/s",
                                "ms_per_step": d8_ms / args.steps,
                                "config": "BASELINE configs[3] literally: same data, max_depth 8, 63 leaves"}
                               if d8_ms else None),
            "config5": c5,
            "clocks": clk,
            "binning": bin_stats,
            "fit_from_raw": fit_raw,
            "other_objectives": other,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    sampler.close()
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_predict_only(args):
    """--part predict: only the predict leg (for profiling k_predict): 1000
    full depth-8 random trees (config 5's ensemble) over --predict-rows rows
    of uint8 bins with the workload's feature count, rows and ensemble
    resident on the device; prints one JSON line with rows/s."""
    import torch
    from bsscl_gbm_b200 import Engine, datasets
    c = CFG
    p = c["p"]
    n = args.predict_rows
    Xb = np.random.default_rng(5).integers(0, 256, size=(n, p)).astype(np.uint8)
    eng = Engine(0)
    ens = datasets.config5_ensemble(n_trees=1000, depth=8, p=p, seed=5)
    eng.predict_set_model(ens, 1000, p)
    eng.predict_upload(Xb)
    for _ in range(max(1, args.warmup)):
        eng.predict_run(c["lr"], 0.0)
    eng.sync()
    torch.cuda.nvtx.range_push("bench_predict")
    eng.event(4)
    for _ in range(args.steps):
        eng.predict_run(c["lr"], 0.0)
    eng.event(5)
    torch.cuda.nvtx.range_pop()
    ms = eng.elapsed_ms(4, 5) / args.steps
    print(json.dumps({"part": "predict", "rows": n, "features": p, "trees": 1000, "depth": 8,
                      "ms_per_launch": ms, "rows_per_s": n / (ms / 1000.0),
                      "node_visits_per_s": n * 8000 / (ms / 1000.0)}), flush=True)
    eng.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    # 200 rounds (~0.2 s on one B200): the steady state of the pipelined rounds
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="engine", choices=["engine", "reference"])
    ap.add_argument("--config", default="4", choices=sorted(CONFIGS),
                    help="4 (default): the headline, 1M x 100 depth 6; 5: 10M x 200 depth 10")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--part", default="all", choices=["all", "predict", "rounds"],
                    help="predict: time only the ensemble predict (k_predict); rounds: only the "
                         "upload and the timed rounds (both for profiling)")
    ap.add_argument("--predict-rows", type=int, default=1_000_000)
    ap.add_argument("--config5-steps", type=int, default=20,
                    help="timed rounds of the configs[4] (10M x 200) sub-record")
    ap.add_argument("--no-config5", action="store_true", help="skip the configs[4] sub-record")
    args = ap.parse_args()
    global CFG, METRIC
    CFG = CONFIGS[args.config]
    METRIC = CFG["metric"]
    if args.part == "predict":
        run_predict_only(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_engine(args)


if __name__ == "__main__":
    main()
