"""The reference's golden fits, carried through the product's model-file
loader and host predictor.

For each fixture of tests/test_golden_bits.mojo the oracle's trees (pinned
bit for bit to the reference there) are written as a format-v4 model file by
the restatement of serialize.mojo below.  The file is loaded through
mojotrees_load_model, and prediction on the fixture's bins must reproduce the
reference's golden raw-score bits.  The C ABI's writer must then write the
loaded model back as exactly the same bytes.
"""
import hashlib
import struct

import numpy as np
import pytest

from golden_fixtures import fixture, load_golden
from test_golden import REFERENCE_BASE, _bins, bits

GOLDEN = load_golden()


def _u64(x):
    return str(struct.unpack("<Q", struct.pack("<d", float(x)))[0])


def _row(vals):
    return "".join(f"{v} " for v in vals) + "\n"


def v4_text(m, K, lr, objective, n_features, n_bins, mbin, ncat):
    """A format-v4 model file (serialize.mojo:999-1119, 431-572) for oracle
    trees over pre-binned columns: an edge-free mapper carrying the bin
    width, the missing bins and categorical bins 1..n (codes 0..n-1)."""
    s = "mojotrees v4\n"
    if K > 1:
        s += f"multiclass {K}\nlearning_rate {_u64(lr)}\nbase_scores"
        s += "".join(" " + _u64(b) for b in m.base_scores) + "\n"
    else:
        s += f"objective {objective}\nlearning_rate {_u64(lr)}\nbase_score {_u64(m.base_scores[0])}\n"
    s += f"mapper {n_features} {n_bins} 0\n\n" + _row([0] * (n_features + 1)) + _row([int(v) for v in mbin])
    cats = [int(c) for c in ncat]
    if any(c >= 0 for c in cats):
        codes, offs = [], [0]
        for c in cats:
            codes += list(range(max(c, 0)))
            offs.append(len(codes))
        s += f"categorical {n_features} {len(codes)}\n" + _row([1 if c >= 0 else 0 for c in cats])
        s += _row(codes) + _row(offs)
    s += f"trees {m.n_trees}\n"
    for t in range(m.n_trees):
        nn = int(m.n_nodes[t])
        feat = [int(v) for v in m.feature[t, :nn]]
        leaf = [f < 0 for f in feat]
        is_cat = [not leaf[i] and (m.cat_bits[t, i].any() or m.threshold_bin[t, i] < 0) for i in range(nn)]
        pool, off = [], []
        for i in range(nn):
            if is_cat[i]:
                off.append(len(pool))
                pool += [int(w) for w in m.cat_bits[t, i]]
            else:
                off.append(-1)
        s += f"tree {nn} {sum(leaf)}\n" + _row([-1 if leaf[i] else feat[i] for i in range(nn)])
        s += _row([-1 if leaf[i] or is_cat[i] else int(m.threshold_bin[t, i]) for i in range(nn)])
        s += _row([-1 if leaf[i] else int(m.left[t, i]) for i in range(nn)])
        s += _row([-1 if leaf[i] else int(m.right[t, i]) for i in range(nn)])
        s += _row([_u64(v) for v in m.value[t, :nn]])
        s += _row([0 if leaf[i] or is_cat[i] else int(m.default_left[t, i] != 0) for i in range(nn)])
        s += _row([-1 if leaf[i] or is_cat[i] else int(m.missing_bin[t, i]) for i in range(nn)])
        counts = [float(c) for c in m.count[t, :nn]]
        covers = all(c > 0 for c in counts)
        s += f"counts {1 if covers else 0}\n" + (_row([_u64(c) for c in counts]) if covers else "")
        gains = [0.0 if leaf[i] else float(m.gain[t, i]) for i in range(nn)]
        has_g = any(g > 0 for g in gains)
        s += f"gains {1 if has_g else 0}\n" + (_row([_u64(g) for g in gains]) if has_g else "")
        if pool:
            s += f"cat {len(pool)}\n" + _row(off) + _row(pool)
    return s


@pytest.mark.parametrize("name", ["l2", "bag", "ffrac", "misscat", "large", "logit", "multi"])
def test_golden_fit_through_model_file(name, oracle, mtlib, tmp_path):
    fx = fixture(name)
    bins, nb, mbin, ncat = _bins(fx, oracle)
    K = fx.get("n_classes", 1)
    kw = dict(objective=fx["objective"], n_classes=K, num_rounds=fx["rounds"], learning_rate=fx["lr"],
              num_leaves=fx["leaves"], min_data_in_leaf=fx["min_data"], base_override=REFERENCE_BASE.get(name))
    kw.update(fx.get("extra", {}))
    m = oracle.train(bins, nb, fx["y"], missing_bin=mbin, n_cats=ncat, **kw)
    objective = 1 if fx["objective"] == 1 else 0
    text = v4_text(m, K, fx["lr"], objective, bins.shape[0], nb, mbin, ncat)
    path = tmp_path / f"{name}.mbst"
    path.write_text(text)
    model = mtlib.Model.load(str(path))
    raw = model.predict_binned(bins).reshape(-1)
    g = GOLDEN[name]
    if "raw" in g:
        assert [bits(v) for v in raw] == g["raw"], "raw scores differ from the reference's golden bits"
    else:
        digest = hashlib.sha256(b"".join(struct.pack("<d", v) for v in raw)).hexdigest()
        assert digest == g["raw_sha256"], "raw scores differ from the reference's golden digest"
    out = tmp_path / f"{name}_again.mbst"
    model.save(str(out))
    assert out.read_text() == text
