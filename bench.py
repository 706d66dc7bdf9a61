"""Benchmark of the GBDT training hot path: boosting rounds/s and histogram GB/s.

Default workload (`--config c2`): binary logistic
with quantized gradients, 10,000,000 rows x 100 float32 features ~ N(0,1),
label ~ Bernoulli(sigmoid(w.x[0:20] + 0.5 x20 x21)), w ~ N(0, 0.3), seed 1;
max_bin 255, num_leaves 255, int8 gradients with seeded stochastic rounding
into integer histograms.  `--config c1|c4|c5` run configs[0], [3] and [4]
(c5: 200M x 128 pre-binned rows split evenly over the GPUs, strong scaling).
Synthetic data of each configuration's recipe (the reference names no
dataset).

A step is one boosting round.  `value` = timed rounds / device time of those
rounds (CUDA events recorded on the trainer's stream at every round boundary
of one fit, after W warm-up rounds of the same fit); inputs are resident in
HBM (binning and upload precede the first round).  The row-major bin matrix
exceeds L2 (126 MB), so no flush is needed between rounds.  `e2e` is the same
metric through the public C ABI (mojotrees_train_dense with a host float64
matrix, or the pre-binned uint8 entry point for c5): bin fitting (host), the
copies and binning on the device, and the tree read-back are inside the timed
wall-clock region.  The histogram roofline comes from the same timed rounds:
CUDA events around every histogram launch on the trainer's stream.

Multi-GPU (torchrun, one process per GPU): for c1, c2 and c4 every GPU holds
its own shard of the configuration's size (weak scaling, `value` counts
rounds x shards / s); c5 splits its 200M rows.  The ranks grow one shared
model through NCCL histogram exchanges (mojotrees_b200_train_binned_u8_dp).

`--impl reference` and the `cpu_baseline` leg time the reference algorithm's
CPU path (the C++ restatement in oracle/, Float64 histograms, all host
threads) on the configuration's own rows, one fit, per-round wall clock; the
CPU arm bins through the oracle's restatement of the reference binner and
never loads this library.
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
sys.path.insert(0, ROOT)

N_ROWS = 10_000_000
N_FEAT = 100
MAX_BIN = 255
LEAVES = 255
# DRAM bytes (read + write) per row built, from the ncu capture of the root
# histogram launch of the 2M-row case (k_hist, 16-bit packed cells):
# 236.4 MB read + 4.1 MB written for 2,000,000 rows
HIST_DRAM_BYTES_PER_ROW = (237.680384e6 + 9.167616e6) / 2_000_000
UNIT = "rounds/s"

# The benchmark configurations: rows (per GPU for the
# weak-scaled c2, global for the strong-scaled c5), features, objective,
# classes, bins, leaves, gradient mode.
CONFIGS = {
    "c1": dict(index=0, rows=1_000_000, feats=28, objective="regression", K=1, max_bin=255, leaves=255, quant=False,
               scaling="weak", desc="configs[0]: L2 regression, 1M x 28 (half N(0,1), half U(0,1)), max_bin 255, "
                                    "num_leaves 255, fixed-point gradients"),
    "c2": dict(index=1, rows=10_000_000, feats=100, objective="binary", K=1, max_bin=255, leaves=255, quant=True,
               scaling="weak", desc="configs[1]: binary logistic, quantized int8 gradients, 10M x 100 per GPU, "
                                    "max_bin 255, num_leaves 255"),
    "c3": dict(index=2, rows=5_000_000, feats=408, objective="regression", K=1, max_bin=63, leaves=127,
               quant=False, scaling="weak",
               desc="configs[2]: regression, 5M x (400 numeric at 90% zeros + 8 categorical of cardinality 1000), "
                    "max_bin 63, num_leaves 127, fixed-point gradients; sparse histograms (per row the bins outside "
                    "each feature's default bin), unbundled (no bundle forms under max_conflict_rate 0)"),
    "c4": dict(index=3, rows=4_000_000, feats=64, objective="multiclass", K=10, max_bin=255, leaves=63, quant=False,
               scaling="weak", desc="configs[3]: softmax K=10, 4M x 64, max_bin 255, num_leaves 63, fixed-point "
                                    "gradients (ten trees per round)"),
    "c5": dict(index=4, rows=200_000_000, feats=128, objective="binary", K=1, max_bin=255, leaves=255, quant=True,
               scaling="strong", desc="configs[4]: binary logistic, quantized int8 gradients, 200M x 128 pre-binned "
                                      "uint8 split evenly over the GPUs, num_leaves 255"),
}


def metric_of(cfg):
    c = CONFIGS[cfg]
    per = " per GPU" if c["scaling"] == "weak" and cfg == "c2" else ""
    return (f"boosting rounds/sec ({c['objective']}{', quantized gradients' if c['quant'] else ''}, "
            f"{c['rows'] / 1e6:g}M x {c['feats']}{per}, {c['leaves']} leaves)")


METRIC = metric_of("c2")


def make_data(n_rows, seed=1, row_offset=0):
    """rows [row_offset, row_offset + n_rows) of the seeded
    synthetic dataset; X is feature-major float32."""
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.3, size=20)
    rng = np.random.default_rng([seed, row_offset])
    X = rng.standard_normal(size=(N_FEAT, n_rows), dtype=np.float32)  # feature-major
    s = (w.astype(np.float32) @ X[:20]).astype(np.float64) + 0.5 * X[20].astype(np.float64) * X[21]
    p = 1.0 / (1.0 + np.exp(-s))
    y = (rng.random(n_rows) < p).astype(np.float64)
    return X, y


def make_c1(n_rows, seed=0, row_offset=0):
    """28 features, half ~N(0,1), half ~U(0,1); y = sin(3 x0) +
    x1 x2 - 0.5 x3^2 + 0.1 N(0,1).  X is feature-major float64."""
    rng = np.random.default_rng([seed, row_offset])
    X = np.empty((28, n_rows))
    X[:14] = rng.standard_normal((14, n_rows))
    X[14:] = rng.random((14, n_rows))
    y = np.sin(3 * X[0]) + X[1] * X[2] - 0.5 * X[3] ** 2 + 0.1 * rng.standard_normal(n_rows)
    return X, y


def make_c4(n_rows, seed=3, row_offset=0):
    """64 features ~N(0,1); class = argmax of 10 random linear
    projections plus Gumbel noise.  X is feature-major float64."""
    W = np.random.default_rng(seed).standard_normal((64, 10))
    rng = np.random.default_rng([seed, row_offset])
    X = rng.standard_normal((64, n_rows))
    y = np.argmax(X.T @ W + rng.gumbel(size=(n_rows, 10)), axis=1).astype(np.float64)
    return X, y


def make_c3(n_rows, seed=2, row_offset=0):
    """400 numeric features at 90% zeros (nonzeros ~ LogNormal(0, 1))
    then 8 categorical features of cardinality 1000 drawn Zipf(1.1) (codes
    above 1000 folded back); y = sum of per-category random effects ~ N(0, 1)
    + 0.2 x the sum of the first 10 numeric features.  X is feature-major
    float64."""
    effects = np.random.default_rng(seed).standard_normal((8, 1000))
    rng = np.random.default_rng([seed, row_offset])
    X = np.zeros((408, n_rows))
    for f in range(400):
        nz = np.flatnonzero(rng.random(n_rows) < 0.1)
        X[f, nz] = rng.lognormal(0.0, 1.0, size=nz.size)
    y = 0.2 * X[:10].sum(axis=0)
    for c in range(8):
        codes = (rng.zipf(1.1, size=n_rows) - 1) % 1000
        X[400 + c] = codes
        y += effects[c][codes]
    return X, y


C5_BLOCK = 1_000_000


def make_c5(row_begin, row_end, seed=4):
    """pre-binned uint8 [128, rows] uniform over 255 bins; label ~
    Bernoulli(sigmoid(sum over 16 features of a per-bin effect ~ N(0, 0.2))).
    Generated in blocks of 1M rows, each seeded by its index, so any split
    of the rows over GPUs sees the same dataset."""
    eff = np.random.default_rng(seed).normal(0.0, 0.2, size=(16, 255))
    n = row_end - row_begin
    bins = np.empty((128, n), np.uint8)
    y = np.empty(n)
    for b0 in range(row_begin - row_begin % C5_BLOCK, row_end, C5_BLOCK):
        rng = np.random.default_rng([seed, b0 // C5_BLOCK])
        blk = rng.integers(0, 255, size=(128, C5_BLOCK), dtype=np.uint8)
        u = rng.random(C5_BLOCK)
        lo, hi = max(b0, row_begin), min(b0 + C5_BLOCK, row_end)
        sl = slice(lo - b0, hi - b0)
        s = np.zeros(hi - lo)
        for j in range(16):
            s += eff[j][blk[j, sl]]
        bins[:, lo - row_begin:hi - row_begin] = blk[:, sl]
        y[lo - row_begin:hi - row_begin] = (u[sl] < 1.0 / (1.0 + np.exp(-s))).astype(np.float64)
    return bins, y


def binning_params(cfg):
    p = {"max_bin": CONFIGS[cfg]["max_bin"]}
    if cfg == "c3":
        p["categorical_feature"] = ",".join(str(f) for f in range(400, 408))
    return p


def params(rounds, quant=True, extra=None, cfg="c2"):
    c = CONFIGS[cfg]
    p = {"objective": c["objective"], "num_iterations": rounds, "num_leaves": c["leaves"], "min_data_in_leaf": 20,
         "learning_rate": 0.1, "use_quantized_grad": c["quant"] and quant, **binning_params(cfg)}
    if c["K"] > 1:
        p["num_class"] = c["K"]
    if extra:
        p.update(extra)
    return p


class ClockSampler:
    """SM clock and throttle reasons, read through NVML every ~10 ms with host
    timestamps (reads only), so the summary can cover just the timed rounds.
    Falls back to nvidia-smi queries when NVML is not importable."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, gpu_index, period=0.01):
        self.gpu = gpu_index
        self.period = period
        self.samples = []  # (monotonic time, sm MHz, max sm MHz, reason names)
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            mx = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))

            def read():
                sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                return sm, mx, {n for n, b in self.REASONS if bits & b}
        except Exception:
            q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap")

            def read():
                out = subprocess.run(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                v = [x.strip() for x in out.split(",")]
                return float(v[0]), float(v[1]), {n for (n, _), x in zip(self.REASONS, v[2:6])
                                                  if x.lower() == "active"}
        while not self._stop.is_set():
            try:
                t = time.monotonic()
                sm, mx_, rs = read()
                self.samples.append(((t + time.monotonic()) / 2, sm, mx_, rs))
            except Exception:
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self, window=None):
        """Median SM clock and the reasons seen, over the samples inside
        window = (t0, t1) (monotonic seconds) when given."""
        sel = [s for s in self.samples if window is None or window[0] <= s[0] <= window[1]]
        sm = [s[1] for s in sel]
        reasons = set()
        for s in sel:
            reasons |= s[3]
        mx = self.samples[-1][2] if self.samples else None
        out = {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
               "samples": len(sm)}
        if window is not None:
            out["window"] = "timed rounds (host window ending when the fit returned, their device time long)"
        return out


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def config_data(cfg, rank=0, world=1, rows=None):
    """This rank's share of the configuration's dataset: (feature-major uint8
    bins or None, feature-major float matrix or None, labels, global row
    offset, global rows).  Weak-scaled configurations give every rank `rows`
    rows of its own; c5 splits its fixed row count."""
    c = CONFIGS[cfg]
    n = rows or c["rows"]
    if c["scaling"] == "strong":
        lo, hi = n * rank // world, n * (rank + 1) // world
        bins, y = make_c5(lo, hi)
        return bins, None, y, lo, n
    off = rank * n
    if cfg == "c1":
        X, y = make_c1(n, row_offset=off)
    elif cfg == "c4":
        X, y = make_c4(n, row_offset=off)
    elif cfg == "c3":
        X, y = make_c3(n, row_offset=off)
    else:
        X, y = make_data(n, seed=1, row_offset=off)
    return None, X, y, off, n * world


def oracle_bins(X, max_bin, categorical=()):
    """Bins of the feature-major matrix X through the oracle's restatement of
    the reference binner (the CPU arms never load this library)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_api
    return oracle_api.bin_dense(np.asarray(X, dtype=np.float64).T, max_bin=max_bin, categorical=categorical)


def cpu_fit_timed(cfg, bins, nb, y, mbin, ncat, warmup, steps):
    """The oracle's CPU trainer (restatement of the reference device=cpu path,
    Float64 histograms, all host threads) over warmup + steps rounds of one
    fit; returns seconds of the `steps` rounds after the warm-up ones."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_api
    c = CONFIGS[cfg]
    obj = {"regression": oracle_api.OBJ_L2, "binary": oracle_api.OBJ_LOGISTIC,
           "multiclass": oracle_api.OBJ_SOFTMAX}[c["objective"]]
    m = oracle_api.train(bins, nb, y, missing_bin=mbin, n_cats=ncat, objective=obj, n_classes=c["K"],
                         num_rounds=warmup + steps, num_leaves=c["leaves"], min_data_in_leaf=20, learning_rate=0.1,
                         mode=oracle_api.MODE_CPU, n_threads=os.cpu_count() or 1)
    rs = m.round_seconds
    t0 = rs[warmup - 1] if warmup > 0 else 0.0
    return float(rs[warmup + steps - 1] - t0), float(rs[warmup + steps - 1])


CPU_DESC = ("C++ restatement of the reference device=cpu trainer (Float64 histograms), OpenMP over features and "
            "row blocks")


CPU_SAMPLE_ROWS = 20_000_000


def cpu_baseline(cfg, bins, nb, y, mbin, ncat, n_rows, warmup=1, steps=2):
    """Reference CPU path on the configuration's own rows, a few rounds (the
    bounded sample is the round count).  Above 20M rows the
    first 20M rows are fitted and the per-round time is scaled by the row
    ratio, which the sample text states."""
    threads = os.cpu_count() or 1
    n_fit = min(n_rows, CPU_SAMPLE_ROWS)
    if n_fit < n_rows:
        bins = np.ascontiguousarray(bins[:, :n_fit])
        y = y[:n_fit]
        warmup, steps = 1, 1
    dt, total = cpu_fit_timed(cfg, bins, nb, y, mbin, ncat, warmup, steps)
    scale = n_rows / n_fit
    where = (f"all {n_rows:,} rows of the workload" if n_fit == n_rows else
             f"the first {n_fit:,} of the workload's {n_rows:,} rows, per-round time scaled by {scale:g}")
    return {"value": steps / (dt * scale), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"rounds {warmup + 1}..{warmup + steps} of one fit on {where} "
                      f"({dt:.1f} s of the fit's {total:.1f} s, per-round wall clock); " + CPU_DESC}


def run_reference(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return
    cfg = args.config
    c = CONFIGS[cfg]
    bins, X, y, _, n = config_data(cfg, rows=args.rows)
    if bins is None:
        bins, mbin, ncat, nb = oracle_bins(X, c["max_bin"], list(range(400, 408)) if cfg == "c3" else ())
        del X
    else:
        mbin, ncat, nb = None, None, c["max_bin"]
    threads = os.cpu_count() or 1
    dt, total = cpu_fit_timed(cfg, bins, nb, y, mbin, ncat, args.warmup, args.steps)
    value = args.steps / dt
    b = {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
         "sample": f"rounds {args.warmup + 1}..{args.warmup + args.steps} of one fit on all {n:,} rows of the "
                   f"workload ({dt:.1f} s of the fit's {total:.1f} s, per-round wall clock); " + CPU_DESC}
    line = {"impl": "reference", "metric": metric_of(cfg), "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 / value,
            "higher_is_better": True, "scaling": c["scaling"], "vs_baseline": None, "dtype": "f64",
            "data": "synthetic", "config": {"workload": c["desc"] + " (reference CPU path: Float64 histograms)",
                                            "rows": n, "features": c["feats"]},
            "cpu_baseline": b, "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def run_gpu(args):
    import mojoboost_b200 as mb
    cfg = args.config
    c = CONFIGS[cfg]
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    dist = None
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("gloo")
    bins, X, y, row_off, n_global = config_data(cfg, rank, world, args.rows)
    X64 = None
    if bins is None:
        X64 = np.asfortranarray(X.T.astype(np.float64))  # column-major float64 for the C ABI
        del X
        # one bin mapper for all shards: each rank fits it on its own rows
        # (weak scaling: the shards are statistically identical)
        bins, mbin, ncat, nb = mb.bin_dense(X64, binning_params(cfg))
    else:
        mbin, ncat, nb = None, None, c["max_bin"]
    n_local = bins.shape[1]
    F = c["feats"]
    pair_bytes = 2 if c["quant"] else 8
    rounds = args.warmup + args.steps
    def fit(profile):
        p = params(rounds, cfg=cfg, extra={"gpu_device_id": local, "profile_histogram": profile})
        if world > 1:
            import torch
            nid = torch.from_numpy(mb.nccl_unique_id() if rank == 0 else np.zeros(128, np.uint8))
            dist.broadcast(nid, 0)
            return mb.train_binned_dp(bins, nb, y, nid.numpy(), rank, world, row_off, n_global, p,
                                      missing_bin=mbin, n_categories=ncat)
        return mb.train_binned(bins, nb, y, p, missing_bin=mbin, n_categories=ncat)

    # the timed fit runs as a user's fit does, without profiling events
    with ClockSampler(local) as clocks:
        model = fit(False)
        t_fit_end = time.monotonic()
    rs = model.round_stats()[args.warmup:args.warmup + args.steps]
    dev_ms = float(np.sum(rs[:, 0]))
    if world > 1:
        import torch
        t = torch.tensor([dev_ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_ms = float(t.item())
    # a second fit of the same workload carries CUDA events around every
    # histogram launch: the kernel's time inside the timed rounds (the events
    # cost ~2.5% of the round, so they stay out of the timed fit)
    if not args.no_phase_events:
        pmodel = fit(True)
        prs = pmodel.round_stats()[args.warmup:args.warmup + args.steps]
        st = pmodel.stats()
    else:
        prs = rs
        st = model.stats()
    # weak scaling: every rank's rounds are a full workload's rounds
    value = (world if c["scaling"] == "weak" else 1) * len(rs) / (dev_ms / 1000.0)
    # histogram roofline over the timed rounds (this rank)
    hist_ms = float(np.sum(prs[:, 1]))
    hist_launches = float(np.sum(prs[:, 2]))
    hist_rows = float(np.sum(prs[:, 3]))
    # the tree's counts are global: with several ranks this rank's histogram
    # launches read about its share of them (the shards are equal in size)
    hist_rows_local = hist_rows * n_local / n_global if world > 1 else hist_rows
    sparse_entries = st.get("hist_sparse_entries", 0.0)
    # sparse histograms read, per built row, its listed entries (4 B each),
    # its row id (4 B), its two row offsets (16 B) and its gradient pair
    row_bytes = (4.0 * sparse_entries / n_local + 20 + pair_bytes) if sparse_entries else (F + pair_bytes)
    hist_bytes = hist_rows_local * row_bytes
    hist_gbs = hist_bytes / (hist_ms / 1000.0) / 1e9 if hist_ms > 0 else None
    per_round = 1.0 / max(1, st["rounds"])
    phases = {"hist_ms": st["hist_ms"] * per_round}
    phases.update({"iterations_per_tree": st["iterations"] * per_round / c["K"],
                   "pick_steps_per_tree": st.get("pick_steps", 0.0) * per_round / c["K"],
                   "expansions_per_tree": st["expansions"] * per_round / c["K"],
                   "hist_launches_timed": hist_launches, "hist_rows_timed": hist_rows})
    smem_peak = mb.shared_atomic_peak() if hist_ms > 0 else None
    # useful shared atomics of the histogram: (g+count word, h word) per row and feature
    # (sparse histograms: two atomics per listed entry for a constant hessian, three otherwise)
    atomics_per_row = (sparse_entries / n_local * (2 if c["objective"] == "regression" else 3)
                       if sparse_entries else F * 2)
    smem_achieved = hist_rows_local * atomics_per_row / (hist_ms / 1000.0) if hist_ms > 0 else None
    peak, peak_kind = measured_peak()
    e2e = None
    if world == 1 and not args.no_e2e:
        pe = params(args.steps, cfg=cfg, extra={"gpu_device_id": local})
        t0 = time.perf_counter()
        if X64 is not None:
            m2 = mb.train_dense(X64, y, pe)
            h2d = 8 * n_local * F + 8 * n_local + 8 * n_local * c["K"]
            api = "mojotrees_train_dense (host float64 matrix; includes host bin fitting)"
        else:
            m2 = mb.train_binned(bins, nb, y, pe)
            h2d = n_local * F + 8 * n_local + 8 * n_local
            api = "mojotrees_b200_train_binned_u8 (host pre-binned uint8 matrix)"
        e2e_s = time.perf_counter() - t0
        s2 = m2.stats()
        # copied to the device per fit: the input matrix, labels, initial
        # scores; read back per round: the trees' node tables
        e2e = {"value": args.steps / e2e_s, "unit": UNIT,
               "h2d_bytes_per_step": h2d / max(1, args.steps),
               "d2h_bytes_per_step": 88 * (2 * c["leaves"] - 1) * c["K"], "seconds": e2e_s,
               "rounds": args.steps, "host_binning_s": s2["binning_seconds"], "upload_s": s2["upload_seconds"],
               "device_loop_s": s2["fit_seconds"], "api": api}
    cpu = None
    if not args.no_cpu_baseline and world == 1 and rank == 0:
        try:
            cpu = cpu_baseline(cfg, bins, nb, y, mbin, ncat, n_local)
        except Exception as e:  # the baseline is reported, not required
            cpu = {"error": str(e)}
    if rank != 0:
        return
    line = {
        "metric": metric_of(cfg), "value": value, "unit": UNIT, "n_gpus": world, "steps": len(rs),
        "warmup": args.warmup, "ms_per_step": dev_ms / max(1, len(rs)), "higher_is_better": True,
        "scaling": c["scaling"], "vs_baseline": None,
        "dtype": "int8-grad/int32-hist" if c["quant"] else "int32-fixed-point-grad/int32-hist",
        "data": "synthetic",
        "config": {"workload": c["desc"], "rows_per_gpu": n_local, "rows_total": n_global, "features": F,
                   "l2": "inputs (row-major bins, > 126 MB) larger than L2; no flush", "parallelism": f"dp{world}",
                   **({"dp_exchange": os.environ.get("MOJOTREES_DP_EXCHANGE", "allreduce")} if world > 1 else {})},
        "roofline": {"bound": "hbm", "achieved": hist_gbs, "peak": peak, "unit": "GB/s",
                     "frac": (hist_gbs / peak) if hist_gbs else None,
                     "traffic": (HIST_DRAM_BYTES_PER_ROW * hist_rows_local / hist_launches)
                     if hist_launches and cfg == "c2" else None,
                     "peak_source": peak_kind, "kernel": "k_hist",
                     "algorithmic_bytes": ("with several ranks: this rank's share of the built rows (global / "
                                           "ranks); " if world > 1 else "") +
                                          (f"per launch: rows of the built children x {row_bytes:.1f} B (sparse "
                                           f"histograms: {sparse_entries / n_local:.1f} listed entries x 4 B + "
                                           f"row id, row offsets and {pair_bytes} gradient bytes)"
                                           if sparse_entries else
                                           f"per launch: rows of the built children x ({F} bin bytes + "
                                           f"{pair_bytes} gradient bytes)") +
                                          "; achieved = their sum over the timed "
                                          "rounds / the summed CUDA-event time of the histogram launches "
                                          "(a second fit of the same workload with those events on)",
                     "traffic_source": "ncu dram read+write bytes per row of the k_hist capture "
                                       "(profiles/k_hist_quant16_root_2M.txt) x rows per launch",
                     "shared_atomics": {"achieved": smem_achieved, "peak": smem_peak, "unit": "lane atomics/s",
                                        "frac": (smem_achieved / smem_peak) if smem_achieved and smem_peak
                                        else None,
                                        "peak_source": "mojotrees_b200_shared_atomic_peak on this GPU"}},
        "phase_ms_per_round": phases,
        "e2e": e2e,
        "gpu_launches": int(np.sum(rs[:, 4])),
        "clocks": clocks.summary((t_fit_end - dev_ms / 1000.0 - 0.005, t_fit_end)),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end fit through the dense entry point")
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS),
                    help="benchmark configuration (default c2 = configs[1], the headline workload)")
    ap.add_argument("--rows", type=int, default=None,
                    help="rows (default: the configuration's; smaller only for profiling captures and tests)")
    ap.add_argument("--no-phase-events", action="store_true",
                    help="no CUDA events around the histogram launches (no roofline)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
