"""The reference's seven golden fixtures, regenerated from closed-form inputs.

Inputs follow tests/test_golden_bits.mojo:7920-8120 of the reference: every
feature value is `_uniform(k + seed)` (SplitMix64 over the column-major index,
tests/support.mojo:25-36) and targets are closed-form.  Nothing here is data
from the reference; the literal expected bits live in golden_bits.json.
"""
import json
import math
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
M64 = (1 << 64) - 1


def splitmix64(x):
    x = np.asarray(x, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = x + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def uniform(counter):
    return (splitmix64(counter) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def features(n_rows, n_features, seed):
    k = np.arange(n_rows * n_features, dtype=np.uint64) + np.uint64(seed)
    return uniform(k).reshape(n_features, n_rows)  # feature-major


# The reference's fixture arithmetic was compiled with floating-point
# contraction, so `a*b + c` patterns in its closed-form targets became fused
# multiply-adds (LLVM's fadd/fsub(fmul) -> fma folds).  These helpers spell
# the fused forms out; math via libm fma keeps them correctly rounded.
def regression_target(x):
    """3*x0 - 2*x1 + x2*x3 + 0.5*(x2 - 0.5)^2 as the reference evaluated it."""
    out = np.empty(x.shape[1])
    for r in range(x.shape[1]):
        x0, x1, x2, x3 = (float(x[i, r]) for i in range(4))
        t = x2 - 0.5
        v = fma(3.0, x0, -(2.0 * x1))
        v = fma(x2, x3, v)
        out[r] = fma(0.5 * t, t, v)
    return out


def bin_equal_width(x, n_bins):
    F, N = x.shape
    out = np.zeros((F, N), np.uint8)
    for f in range(F):
        col = x[f]
        lo = col[0]
        hi = col[0]
        for v in col[1:]:
            if v < lo:
                lo = v
            if v > hi:
                hi = v
        width = (hi - lo) / float(n_bins)
        for r in range(N):
            v = col[r]
            if width <= 0.0 or math.isnan(v):
                b = 0
            else:
                b = int((v - lo) / width)
                b = min(max(b, 0), n_bins - 1)
            out[f, r] = b
    return out


def load_golden():
    with open(os.path.join(HERE, "golden", "golden_bits.json")) as f:
        return json.load(f)["fixtures"]


# Fixture definitions: name -> dict(x, y, bins spec, trainer params).
def fixture(name):
    if name == "l2":
        x = features(200, 8, 0)
        return dict(x=x, y=regression_target(x), binning=("equal", 32), objective=0,
                    rounds=8, lr=0.3, leaves=8, min_data=5)
    if name == "logit":
        x = features(200, 8, 10_000)
        s = np.array([fma(float(x[2, r]), float(x[3, r]), fma(2.0, float(x[0, r]), -float(x[1, r])))
                      for r in range(x.shape[1])])
        return dict(x=x, y=(s > 1.0).astype(np.float64), binning=("equal", 32), objective=1,
                    rounds=8, lr=0.3, leaves=8, min_data=5)
    if name == "multi":
        x = features(150, 6, 20_000)
        s = np.array([fma(0.2, float(x[2, r]), fma(0.5, float(x[0, r]), 0.3 * float(x[1, r])))
                      for r in range(x.shape[1])])
        k = (s * 3.0).astype(np.int64)
        k = np.where(k >= 3, 2, k)
        return dict(x=x, y=k.astype(np.float64), binning=("equal", 32), objective=2, n_classes=3,
                    rounds=4, lr=0.3, leaves=6, min_data=5)
    if name == "bag":
        x = features(200, 8, 0)
        return dict(x=x, y=regression_target(x), binning=("equal", 32), objective=0,
                    rounds=8, lr=0.3, leaves=8, min_data=5,
                    extra=dict(bagging_fraction=0.6, bagging_freq=1, bagging_seed=7))
    if name == "ffrac":
        x = features(200, 12, 30_000)
        return dict(x=x, y=regression_target(x), binning=("equal", 32), objective=0,
                    rounds=8, lr=0.3, leaves=8, min_data=5, extra=dict(feature_fraction=0.5))
    if name == "large":
        n = 12_000
        x = features(n, 6, 90_000)
        r = np.arange(n)
        x[4] = (r % 16).astype(np.float64)
        x[5] = np.where(r % 97 == 0, 8 + (r // 97) % 32, r % 8).astype(np.float64)
        return dict(x=x, y=regression_target(x), binning=("fit", 255, []), objective=0,
                    rounds=8, lr=0.3, leaves=31, min_data=20)
    if name == "misscat":
        n, F, seed = 200, 5, 40_000
        u = features(n, F, seed)
        x = u.copy()
        r = np.arange(n)
        x[1] = np.where(r % 7 == 0, np.nan, u[1])
        x[2] = np.floor(u[2] * 6.0)
        table = np.array([0.0, 1.5, -1.0, 0.7, -2.0, 2.5])
        y = 2.0 * x[0] + np.where(np.isnan(x[1]), 0.5, x[1]) + table[x[2].astype(int)]
        return dict(x=x, y=y, binning=("fit", 32, [2]), objective=0, rounds=8, lr=0.3,
                    leaves=8, min_data=5,
                    extra=dict(max_cat_to_onehot=4, max_cat_threshold=32, cat_smooth=2.0,
                               cat_l2=10.0, min_data_per_group=5))
    raise KeyError(name)


def predict_tree(model, t, bins_fm, r):
    node = 0
    feat = model.feature[t]
    while feat[node] >= 0:
        b = int(bins_fm[feat[node], r])
        if model.cat_bits[t, node].any() or model.threshold_bin[t, node] < 0:
            bits = model.cat_bits[t, node]
            left = 0 < b < 256 and (int(bits[b >> 6]) >> (b & 63)) & 1
        elif b == model.missing_bin[t, node]:
            left = bool(model.default_left[t, node])
        else:
            left = b <= model.threshold_bin[t, node]
        node = model.left[t, node] if left else model.right[t, node]
    return model.value[t, node]


_libm = None


def fma(a, b, c):
    """Correctly rounded a*b+c (libm fma; math.fma needs Python 3.13)."""
    global _libm
    if _libm is None:
        import ctypes
        _libm = ctypes.CDLL("libm.so.6")
        _libm.fma.restype = ctypes.c_double
        _libm.fma.argtypes = [ctypes.c_double] * 3
    return _libm.fma(a, b, c)


def record(model, bins_fm, lr, n_classes=1, objective=0, pred_fma=False):
    """Flat ints, value bits, raw bits and prediction bits in the reference's order."""
    ints = [model.n_trees]
    vals = []
    for t in range(model.n_trees):
        nn = int(model.n_nodes[t])
        ints.append(nn)
        for i in range(nn):
            ints += [int(model.feature[t, i]), int(model.threshold_bin[t, i]),
                     int(model.left[t, i]), int(model.right[t, i])]
            vals.append(float(model.value[t, i]))
    N = bins_fm.shape[1]
    raw, pred = [], []
    K = n_classes
    for r in range(N):
        if K == 1:
            s = float(model.base_scores[0])
            for t in range(model.n_trees):
                v = predict_tree(model, t, bins_fm, r)
                s = fma(lr, v, s) if pred_fma else s + lr * v
            raw.append(s)
            if objective == 1:
                pred.append(1.0 / (1.0 + math.exp(-s)) if s >= 0 else math.exp(s) / (1.0 + math.exp(s)))
            else:
                pred.append(s)
        else:
            row = [float(b) for b in model.base_scores]
            for i in range(model.n_trees // K):
                for k in range(K):
                    v = predict_tree(model, i * K + k, bins_fm, r)
                    row[k] = fma(lr, v, row[k]) if pred_fma else row[k] + lr * v
            m = max(row)
            e = [math.exp(v - m) for v in row]
            tot = 0.0
            for v in e:
                tot += v
            raw += row
            pred += [v / tot for v in e]
    return ints, vals, raw, pred
