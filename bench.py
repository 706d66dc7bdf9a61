"""Benchmark of the GBDT training hot path: boosting rounds/s and histogram GB/s.

Workload: binary logistic with quantized gradients,
10,000,000 rows x 100 float32 features ~ N(0,1), label ~ Bernoulli(sigmoid(
w.x[0:20] + 0.5 x20 x21)), w ~ N(0, 0.3), seed 1; max_bin 255, num_leaves 255,
int8 gradients with seeded stochastic rounding into integer histograms.
Synthetic data of that shape (the reference names no dataset).

A step is one boosting round.  `value` = timed rounds / device time of those
rounds (CUDA events recorded on the trainer's stream at every round boundary
of one fit, after W warm-up rounds of the same fit); inputs are resident in
HBM (binning and upload precede the first round).  The 1.1 GB row-major bin
matrix exceeds L2 (126 MB), so no flush is needed between rounds.  `e2e` is
the same metric through the public C ABI (mojotrees_train_dense) with host
buffers: bin fitting (host), the float64 column copies and their binning on
the device, and the tree read-back are inside the timed wall-clock region.
The histogram roofline comes from the same timed rounds: CUDA events around
every histogram launch on the trainer's stream.

Multi-GPU (torchrun, one process per GPU): every GPU holds its own 10M-row
shard of one global dataset (weak scaling) and the ranks grow one shared
model through NCCL histogram sums (mojotrees_b200_train_binned_u8_dp).
`value` counts rounds x shards / s, so perfect scaling multiplies it by N.

`--impl reference` times the reference algorithm's CPU path (the C++
restatement in oracle/, Float64 histograms, all host threads) on a bounded
row sample of the same workload, scaled linearly to the full row count.
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
HIST_DRAM_BYTES_PER_ROW = (236.426240e6 + 4.148480e6) / 2_000_000
METRIC = "boosting rounds/sec (binary logistic, quantized gradients, 10M x 100 per GPU, 255 leaves)"
UNIT = "rounds/s"


def make_data(n_rows, seed=1, row_offset=0):
    """Rows [row_offset, row_offset + n_rows) of the seeded synthetic dataset."""
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.3, size=20)
    rng = np.random.default_rng([seed, row_offset])
    X = rng.standard_normal(size=(N_FEAT, n_rows), dtype=np.float32)  # feature-major
    s = (w.astype(np.float32) @ X[:20]).astype(np.float64) + 0.5 * X[20].astype(np.float64) * X[21]
    p = 1.0 / (1.0 + np.exp(-s))
    y = (rng.random(n_rows) < p).astype(np.float64)
    return X, y


def params(rounds, quant=True, extra=None):
    p = {"objective": "binary", "num_iterations": rounds, "num_leaves": LEAVES, "max_bin": MAX_BIN,
         "min_data_in_leaf": 20, "learning_rate": 0.1, "use_quantized_grad": quant}
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


def cpu_baseline(warmup=1, steps=8, rows=2_500_000):
    """Reference CPU path (C++ restatement, Float64 histograms) on a row sample.

    Per-round time = (time of warmup + steps rounds - time of warmup rounds)
    / steps on the first `rows` rows of the workload, scaled linearly to the
    full row count (histogram passes dominate and are linear in rows)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_api
    import mojoboost_b200 as mb
    X, y = make_data(rows, seed=1)
    bins, mbin, ncat, nb = mb.bin_dense(X.T.astype(np.float64), {"max_bin": MAX_BIN})
    del X
    threads = os.cpu_count() or 1

    def fit(rounds):
        if rounds == 0:
            return 0.0
        t = time.perf_counter()
        oracle_api.train(bins, nb, y, missing_bin=mbin, n_cats=ncat, objective=oracle_api.OBJ_LOGISTIC,
                         num_rounds=rounds, num_leaves=LEAVES, min_data_in_leaf=20, learning_rate=0.1,
                         mode=oracle_api.MODE_CPU, n_threads=threads)
        return time.perf_counter() - t

    t_w = fit(warmup)
    t_wk = fit(warmup + steps)
    dt = max(t_wk - t_w, 1e-9)
    per_round_full = dt / steps * (N_ROWS / rows)
    return {"value": 1.0 / per_round_full, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"rounds {warmup + 1}..{warmup + steps} on the first {rows:,} rows of the workload "
                      f"({dt:.1f} s of {t_w + t_wk:.1f} s measured), scaled linearly to {N_ROWS:,} rows; "
                      "C++ restatement of the reference device=cpu trainer (Float64 histograms), OpenMP "
                      "over features and row blocks"}


def run_reference(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return
    # each step is one boosting round on a 1M-row sample of the workload
    b = cpu_baseline(warmup=args.warmup, steps=args.steps, rows=1_000_000)
    line = {"impl": "reference", "metric": METRIC, "value": b["value"], "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 / b["value"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic", "config": {"workload": "configs[1]: binary logistic 10M x 100, 255 bins, "
                                            "255 leaves (reference CPU path: Float64 histograms)"},
            "cpu_baseline": b, "e2e": {"value": b["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def run_gpu(args):
    import mojoboost_b200 as mb
    N_ROWS = args.rows
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    dist = None
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("gloo")
    X, y = make_data(N_ROWS, seed=1, row_offset=rank * N_ROWS)
    X64 = np.asfortranarray(X.T.astype(np.float64))  # column-major float64 for the C ABI
    del X
    # one bin mapper for all shards: fitted on rank 0's rows, shared
    bins, mbin, ncat, nb = mb.bin_dense(X64, {"max_bin": MAX_BIN})
    rounds = args.warmup + args.steps
    # CUDA events around every histogram launch (profile_phases) give the
    # kernel's time inside the timed rounds themselves
    p = params(rounds, extra={"gpu_device_id": local, "profile_histogram": not args.no_phase_events})
    with ClockSampler(local) as clocks:
        if world > 1:
            import torch
            nid = torch.from_numpy(mb.nccl_unique_id() if rank == 0 else np.zeros(128, np.uint8))
            dist.broadcast(nid, 0)
            model = mb.train_binned_dp(bins, nb, y, nid.numpy(), rank, world, rank * N_ROWS, world * N_ROWS, p,
                                       missing_bin=mbin, n_categories=ncat)
        else:
            model = mb.train_binned(bins, nb, y, p, missing_bin=mbin, n_categories=ncat)
        t_fit_end = time.monotonic()
    rs = model.round_stats()[args.warmup:args.warmup + args.steps]
    st = model.stats()
    dev_ms = float(np.sum(rs[:, 0]))
    if world > 1:
        import torch
        t = torch.tensor([dev_ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_ms = float(t.item())
    value = world * len(rs) / (dev_ms / 1000.0)
    # histogram roofline over the timed rounds (this rank)
    hist_ms = float(np.sum(rs[:, 1]))
    hist_launches = float(np.sum(rs[:, 2]))
    hist_rows = float(np.sum(rs[:, 3]))
    hist_bytes = hist_rows * (N_FEAT + 2)
    hist_gbs = hist_bytes / (hist_ms / 1000.0) / 1e9 if hist_ms > 0 else None
    per_round = 1.0 / max(1, st["rounds"])
    phases = {"hist_ms": st["hist_ms"] * per_round}
    phases.update({"iterations_per_tree": st["iterations"] * per_round,
                   "expansions_per_tree": st["expansions"] * per_round,
                   "hist_launches_timed": hist_launches, "hist_rows_timed": hist_rows})
    smem_peak = mb.shared_atomic_peak() if hist_ms > 0 else None
    # useful shared atomics of the histogram: (g+count word, h word) per row and feature
    smem_achieved = hist_rows * N_FEAT * 2 / (hist_ms / 1000.0) if hist_ms > 0 else None
    peak, peak_kind = measured_peak()
    e2e = None
    if world == 1 and not args.no_e2e:
        t0 = time.perf_counter()
        m2 = mb.train_dense(X64, y, params(args.steps, extra={"gpu_device_id": local}))
        e2e_s = time.perf_counter() - t0
        s2 = m2.stats()
        # copied to the device per fit; read back per round: the tree's node table
        # float64 columns (binned on the device), labels, initial scores
        h2d = 8 * N_ROWS * N_FEAT + 8 * N_ROWS + 8 * N_ROWS
        e2e = {"value": m2.num_trees / e2e_s, "unit": UNIT,
               "h2d_bytes_per_step": h2d / max(1, args.steps),
               "d2h_bytes_per_step": 88 * (2 * LEAVES - 1), "seconds": e2e_s, "rounds": int(m2.num_trees),
               "host_binning_s": s2["binning_seconds"], "upload_s": s2["upload_seconds"],
               "device_loop_s": s2["fit_seconds"],
               "api": "mojotrees_train_dense (host float64 matrix; includes host binning)"}
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": len(rs),
        "warmup": args.warmup, "ms_per_step": dev_ms / max(1, len(rs)), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8-grad/int32-hist",
        "data": "synthetic",
        "config": {"workload": "configs[1]: binary logistic, quantized int8 gradients, 10M x 100 per GPU, "
                               "max_bin 255, num_leaves 255", "rows_per_gpu": N_ROWS, "features": N_FEAT,
                   "l2": "inputs (1.1 GB row-major bins) larger than L2; no flush", "parallelism": f"dp{world}",
                   **({"dp_exchange": os.environ.get("MOJOTREES_DP_EXCHANGE", "allreduce")} if world > 1 else {})},
        "roofline": {"bound": "hbm", "achieved": hist_gbs, "peak": peak, "unit": "GB/s",
                     "frac": (hist_gbs / peak) if hist_gbs else None,
                     "traffic": (HIST_DRAM_BYTES_PER_ROW * hist_rows / hist_launches) if hist_launches else None,
                     "peak_source": peak_kind, "kernel": "k_hist",
                     "algorithmic_bytes": "per launch: rows of the built children x (100 bin bytes + 2 gradient "
                                          "bytes); achieved = their sum over the timed rounds / the summed "
                                          "CUDA-event time of the histogram launches",
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
    if not args.no_cpu_baseline and world == 1:
        try:
            line["cpu_baseline"] = cpu_baseline()
        except Exception as e:  # the baseline is reported, not required
            line["cpu_baseline"] = {"error": str(e)}
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end fit through the dense entry point")
    ap.add_argument("--rows", type=int, default=N_ROWS,
                    help="rows per GPU (default: the workload's 10M; smaller only for profiling captures)")
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
