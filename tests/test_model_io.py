"""Model files in the reference's text format (src/mojotrees/serialize.mojo).

CPU tests load hand-written files of format v1, v3 and v4 (the token layout
of serialize.mojo:999-1119 and :1121-1370, floats as decimal IEEE-754 bit
patterns), predict through the C ABI and check the values worked out by hand
from the trees, and check that a v4 file is written back byte for byte.  GPU
tests round-trip trained models.
"""
import struct

import numpy as np
import pytest


def b(x):
    """A float as the format writes it: the decimal value of its bit pattern."""
    return str(struct.unpack("<Q", struct.pack("<d", float(x)))[0])


def row(vals):
    return "".join(f"{v} " for v in vals) + "\n"


def frow(vals):
    return row([b(v) for v in vals])


# Regression model, two features.  f0 edges (0.5, 1.5) and a missing bin 3;
# f1 edge 0.0 and no missing bin.  Node 0 splits f0 at bin 1 (missing goes
# left), node 1 splits f1 at bin 0; leaves 2, 3, 4 hold 3.0, -1.0, 2.0.
TREE_A = dict(feature=[0, 1, -1, -1, -1], thr=[1, 0, -1, -1, -1], left=[1, 3, -1, -1, -1],
              right=[2, 4, -1, -1, -1], value=[0.25, 0.5, 3.0, -1.0, 2.0], dleft=[1, 0, 0, 0, 0],
              mbin=[3, -1, -1, -1, -1], counts=[100.0, 60.0, 40.0, 30.0, 30.0], gains=[5.0, 2.0, 0.0, 0.0, 0.0])
X_A = np.array([[0.0, -1.0], [1.0, 0.5], [2.0, 0.0], [np.nan, 0.0], [1.0, np.nan], [0.5, 0.0], [1.5, 1e300]])
# base 0.25 + 0.5 * leaf value; NaN in f1 (no missing bin) is binned as 0.0
RAW_A = np.array([-0.25, 1.25, 1.75, -0.25, -0.25, -0.25, 1.25])


def model_a(version=4, names=False, monotone=False):
    t = TREE_A
    s = f"mojotrees v{version}\n"
    if names:
        s += "feature_names 2\nalpha beta \n"
    s += f"objective 0\nlearning_rate {b(0.5)}\nbase_score {b(0.25)}\n"
    s += "mapper 2 255 3\n" + frow([0.5, 1.5, 0.0]) + row([0, 2, 3])
    if version >= 2:
        s += row([3, -1])
    if monotone:
        s += "monotone 2 1 0\n"
    s += "trees 1\ntree 5 3\n"
    s += row(t["feature"]) + row(t["thr"]) + row(t["left"]) + row(t["right"]) + frow(t["value"])
    if version >= 2:
        s += row(t["dleft"]) + row(t["mbin"])
    if version == 3:
        s += frow(t["counts"])
    if version >= 4:
        s += "counts 1\n" + frow(t["counts"]) + "gains 1\n" + frow(t["gains"])
    return s


def write(tmp_path, name, text):
    p = tmp_path / name
    p.write_text(text)
    return str(p)


def test_v4_file_loads_predicts_and_writes_back_identically(mtlib, tmp_path):
    text = model_a(4)
    m = mtlib.Model.load(write(tmp_path, "a.mbst", text))
    assert (m.num_features, m.num_classes, m.num_trees) == (2, 1, 1)
    np.testing.assert_array_equal(m.predict(X_A, raw_score=True), RAW_A)
    out = str(tmp_path / "a2.mbst")
    m.save(out)
    assert open(out).read() == text
    t = m.tree(0)
    np.testing.assert_array_equal(t["value"], TREE_A["value"])


def test_optional_sections_are_read(mtlib, tmp_path):
    m = mtlib.Model.load(write(tmp_path, "n.mbst", model_a(4, names=True, monotone=True)))
    np.testing.assert_array_equal(m.predict(X_A, raw_score=True), RAW_A)


def test_v1_and_v3_files_load(mtlib, tmp_path):
    m3 = mtlib.Model.load(write(tmp_path, "v3.mbst", model_a(3)))
    np.testing.assert_array_equal(m3.predict(X_A, raw_score=True), RAW_A)
    # v1: no missing routing anywhere (NaN is binned as 0.0), no covers, no gains
    m1 = mtlib.Model.load(write(tmp_path, "v1.mbst", model_a(1)))
    X = X_A[~np.isnan(X_A).any(axis=1)]
    np.testing.assert_array_equal(m1.predict(X, raw_score=True), RAW_A[~np.isnan(X_A).any(axis=1)])
    out = str(tmp_path / "v1_as_v4.mbst")
    m1.save(out)
    text = open(out).read()
    assert text.startswith("mojotrees v4\n") and "gains 0\n" in text
    np.testing.assert_array_equal(mtlib.Model.load(out).predict(X, raw_score=True),
                                  m1.predict(X, raw_score=True))


def test_multiclass_file(mtlib, tmp_path):
    s = "mojotrees v4\nmulticlass 3\n" + f"learning_rate {b(1.0)}\nbase_scores {b(0.0)} {b(0.5)} {b(-1.0)}\n"
    s += "mapper 1 255 1\n" + frow([0.0]) + row([0, 1]) + row([-1]) + "trees 3\n"
    for v in (1.0, 2.0, 3.0):
        s += "tree 1 1\n" + row([-1]) * 4 + frow([v]) + row([0]) + row([-1])
        s += "counts 1\n" + frow([10.0]) + "gains 0\n"
    m = mtlib.Model.load(write(tmp_path, "mc.mbst", s))
    assert (m.num_classes, m.num_trees, m.num_iterations) == (3, 3, 1)
    raw = m.predict(np.zeros((2, 1)), raw_score=True).reshape(2, 3)
    np.testing.assert_array_equal(raw, [[1.0, 2.5, 2.0]] * 2)
    out = str(tmp_path / "mc2.mbst")
    m.save(out)
    assert open(out).read() == s


def test_categorical_file(mtlib, tmp_path):
    # codes 3, 7, 9 -> bins 1, 2, 3 (unseen, negative and NaN -> bin 0);
    # the root sends the set {bin 2} = {code 7} left
    s = "mojotrees v4\nobjective 0\n" + f"learning_rate {b(1.0)}\nbase_score {b(0.0)}\n"
    s += "mapper 1 255 0\n\n" + row([0, 0]) + row([-1])
    s += "categorical 1 3\n" + row([1]) + row([3, 7, 9]) + row([0, 3])
    s += "trees 1\ntree 3 2\n" + row([0, -1, -1]) + row([-1, -1, -1]) + row([1, -1, -1]) + row([2, -1, -1])
    s += frow([0.0, 1.0, 2.0]) + row([0, 0, 0]) + row([-1, -1, -1])
    s += "counts 1\n" + frow([9.0, 4.0, 5.0]) + "gains 1\n" + frow([1.5, 0.0, 0.0])
    s += "cat 4\n" + row([0, -1, -1]) + row([4, 0, 0, 0])
    m = mtlib.Model.load(write(tmp_path, "cat.mbst", s))
    X = np.array([[7.0], [3.0], [9.0], [100.0], [-1.0], [np.nan]])
    np.testing.assert_array_equal(m.predict(X, raw_score=True), [1.0, 2.0, 2.0, 2.0, 2.0, 2.0])
    out = str(tmp_path / "cat2.mbst")
    m.save(out)
    assert open(out).read() == s


@pytest.mark.parametrize("mutate, code", [
    (lambda s: s.replace("mojotrees v4", "mojotrees v5"), -4),
    (lambda s: s.replace("mojotrees v4", "mojotrees v9"), -3),
    (lambda s: s.replace("mojotrees v4", "lightgbm v4"), -3),
    (lambda s: s.replace(row([1, 3, -1, -1, -1]), row([1, 0, -1, -1, -1])), -3),   # child before its parent
    (lambda s: s.replace("objective 0", "objective 7"), -4),
    (lambda s: s.replace("tree 5 3", "tree 5 2"), -3),                          # leaf count
    (lambda s: s.replace("mapper 2 255 3", "mapper 2 999 3"), -3),              # bins beyond a byte
    (lambda s: s[: len(s) // 2], -3),                                           # truncated
    (lambda s: s.replace(b(0.25), "18446744073709551616", 1), -3),              # 2^64 does not fit
])
def test_bad_files_are_refused(mtlib, tmp_path, mutate, code):
    p = write(tmp_path, "bad.mbst", mutate(model_a(4)))
    with pytest.raises(mtlib.MojoTreesError) as ei:
        mtlib.Model.load(p)
    assert ei.value.code == code


@pytest.mark.gpu
@pytest.mark.parametrize("kind, quant", [("regression", False), ("binary", True), ("multiclass", False)])
def test_gpu_trained_model_round_trip(mtlib, tmp_path, kind, quant):
    """A fitted model written and read back predicts bit for bit the same and
    writes back the same bytes; missing values and categoricals included."""
    from parity_util import make_data, params_for
    nc = 3 if kind == "multiclass" else 1
    X, y = make_data(31, 20_000, 8, kind=kind, n_classes=nc, nan_frac=0.05, cat_cols=(3,), n_cat=10)
    p = params_for(kind, 3, 15, quant=quant, n_classes=nc, extra={"categorical_feature": "3"})
    m = mtlib.train_dense(X, y, p)
    a = str(tmp_path / "m.mbst")
    m.save(a)
    m2 = mtlib.Model.load(a)
    np.testing.assert_array_equal(m2.predict(X, raw_score=True), m.predict(X, raw_score=True))
    c = str(tmp_path / "m2.mbst")
    m2.save(c)
    assert open(c).read() == open(a).read()


@pytest.mark.gpu
def test_gpu_prebinned_model_round_trip(mtlib, tmp_path):
    """A model fitted on pre-binned columns is written with an edge-free
    mapper; read back it predicts the same on bins and refuses raw values."""
    from parity_util import make_data, params_for
    X, y = make_data(32, 20_000, 6, kind="binary")
    bins, mbin, ncat, nb = mtlib.bin_dense(X, {})
    m = mtlib.train_binned(bins, nb, y, params_for("binary", 3, 15), missing_bin=mbin, n_categories=ncat)
    a = str(tmp_path / "b.mbst")
    m.save(a)
    m2 = mtlib.Model.load(a)
    np.testing.assert_array_equal(m2.predict_binned(bins), m.predict_binned(bins))
    with pytest.raises(mtlib.MojoTreesError):
        m2.predict(X, raw_score=True)


def test_corrupted_files_never_crash(mtlib, tmp_path):
    """Seeded token-level corruption of valid files (replaced, dropped and
    repeated tokens, truncation): every load either fails with a status or
    yields a model whose host prediction runs."""
    rng = np.random.default_rng(7)
    base = model_a(4).split()
    repl = ["-1", "0", "1", "2", "3", "7", "255", "256", "-2", "4294967299", "9223372036854775807",
            "18446744073709551615", "99999999999999999999", "x", "tree", "cat", "counts", "gains", "mapper"]
    p = str(tmp_path / "fuzz.mbst")
    loaded = 0
    for _ in range(600):
        tok = list(base)
        for _ in range(rng.integers(1, 4)):
            i = int(rng.integers(0, len(tok)))
            op = rng.integers(0, 4)
            if op == 0:
                tok[i] = repl[int(rng.integers(0, len(repl)))]
            elif op == 1:
                del tok[i]
            elif op == 2:
                tok.insert(i, tok[i])
            else:
                tok = tok[:i]
            if not tok:
                tok = ["mojotrees"]
        open(p, "w").write(" ".join(tok))
        try:
            m = mtlib.Model.load(p)
        except mtlib.MojoTreesError:
            continue
        loaded += 1
        try:
            m.predict(X_A, raw_score=True)
        except mtlib.MojoTreesError:
            pass
    assert loaded > 0


def test_dump_json_inspection_schema(mtlib, tmp_path):
    """mojotrees_model_dump_json writes the reference's inspection schema
    (model_dump.mojo, inspection.mojo): thresholds as the split bins' upper
    edges, category sets as codes, leaf ordinals, depths."""
    import json
    d = json.loads(mtlib.Model.load(write(tmp_path, "a.mbst", model_a(4))).dump_json())
    assert (d["dump_format_version"], d["producer"], d["model_format_version"]) == (1, "mojotrees", 4)
    assert (d["objective_code"], d["num_class"], d["num_iteration"], d["num_feature"]) == (0, 1, 1, 2)
    assert d["learning_rate"] == 0.5 and d["base_score"] == [0.25]
    f0, f1 = d["feature_infos"]
    assert f0["bin_upper_bounds"] == [0.5, 1.5] and f0["missing_type"] == "NaN" and f0["num_bin"] == 4
    assert f1["bin_upper_bounds"] == [0.0] and f1["missing_type"] == "None" and f1["num_bin"] == 2
    assert d["has_split_gain"] and d["has_node_count"]
    t = d["tree_info"][0]
    assert (t["num_leaves"], t["num_nodes"], t["max_depth"], t["num_cat"]) == (3, 5, 2, 0)
    root = t["tree_structure"]
    assert (root["split_feature"], root["threshold"], root["threshold_bin"], root["default_left"]) == (0, 1.5, 1, True)
    assert root["split_gain"] == 5.0 and root["missing_bin"] == 3 and root["decision_type"] == "<="
    node1 = root["left_child"]
    assert (node1["split_feature"], node1["threshold"], node1["depth"]) == (1, 0.0, 1)
    assert root["right_child"] == {"node_index": 2, "leaf_index": 0, "leaf_value": 3.0, "leaf_count": 40.0, "depth": 1}
    assert node1["left_child"]["leaf_index"] == 1 and node1["right_child"]["leaf_value"] == 2.0


def test_dump_json_categorical_and_multiclass(mtlib, tmp_path):
    import json
    s = "mojotrees v4\nobjective 0\n" + f"learning_rate {b(1.0)}\nbase_score {b(0.0)}\n"
    s += "mapper 1 255 0\n\n" + row([0, 0]) + row([-1])
    s += "categorical 1 3\n" + row([1]) + row([3, 7, 9]) + row([0, 3])
    s += "trees 1\ntree 3 2\n" + row([0, -1, -1]) + row([-1, -1, -1]) + row([1, -1, -1]) + row([2, -1, -1])
    s += frow([0.0, 1.0, 2.0]) + row([0, 0, 0]) + row([-1, -1, -1])
    s += "counts 1\n" + frow([9.0, 4.0, 5.0]) + "gains 1\n" + frow([1.5, 0.0, 0.0])
    s += "cat 4\n" + row([0, -1, -1]) + row([4, 0, 0, 0])
    d = json.loads(mtlib.Model.load(write(tmp_path, "cat.mbst", s)).dump_json())
    assert d["feature_infos"][0]["type"] == "categorical" and d["feature_infos"][0]["categories"] == [3, 7, 9]
    root = d["tree_info"][0]["tree_structure"]
    assert (root["decision_type"], root["categories"], root["category_bins"], root["threshold"]) == ("==", [7], [2], None)
    assert d["tree_info"][0]["num_cat"] == 1
    s = "mojotrees v4\nmulticlass 2\n" + f"learning_rate {b(1.0)}\nbase_scores {b(0.0)} {b(0.5)}\n"
    s += "mapper 1 255 1\n" + frow([0.0]) + row([0, 1]) + row([-1]) + "trees 2\n"
    for v in (1.0, 2.0):
        s += "tree 1 1\n" + row([-1]) * 4 + frow([v]) + row([0]) + row([-1]) + "counts 1\n" + frow([3.0]) + "gains 0\n"
    d = json.loads(mtlib.Model.load(write(tmp_path, "mc.mbst", s)).dump_json())
    assert d["objective_code"] is None and d["num_tree_per_iteration"] == 2 and d["base_score"] == [0.0, 0.5]
    assert [(t["iteration"], t["class_id"]) for t in d["tree_info"]] == [(0, 0), (0, 1)]
    assert d["has_split_gain"] is False and d["tree_info"][1]["tree_structure"]["leaf_value"] == 2.0
