"""The objective and metric registry the reference's Python package reads from
its extension at import (python/mojotrees/_eval.py:110-276), restated as
data from src/mojotrees/objective_registry.mojo and metrics.mojo.

The records have the layout of bindings/objective_bindings.mojo:
  metrics:    [code, canonical_name, task, higher_is_better, needs, transform]
  objectives: [code, canonical_name, task, link, param_name, default_param,
               renews_leaves, multi_output, needs_groups,
               gradients_on_device, backends, builtin, default_metric_code]
Codes, names and aliases are the reference's own numbers and spellings: they
cross the Python boundary and live in model files, so they must be alike.
The table describes the reference's objectives; which of them this library
trains is decided at fit time (`_mojotrees.param_string`), not here.
"""

# tasks (objective_registry.mojo:406-409, task_name :565-575)
_TASK = {0: "regression", 1: "binary", 2: "multiclass", 3: "ranking"}
# needs / transform flags (objective_registry.mojo:437-450)
NEEDS_NOTHING, NEEDS_PARAM, NEEDS_N_CLASSES, NEEDS_GROUPS, NEEDS_CUTOFF = 0, 1, 2, 4, 8
TRANSFORM_OBJECTIVE_LINK, TRANSFORM_SOFTMAX, TRANSFORM_RAW = 0, 1, 2
LINK_IDENTITY, LINK_SIGMOID, LINK_EXP, LINK_SOFTMAX = 0, 1, 2, 3
SUPPORTS_CPU, SUPPORTS_GPU = 1, 2

# metric codes (metrics.mojo:60-89) with canonical name and task
# (objective_registry.mojo:1671-1816)
_METRICS = [
    (0, "l2", 0), (1, "rmse", 0), (2, "l1", 0), (3, "quantile", 0), (4, "huber", 0),
    (5, "binary_logloss", 1), (6, "binary_error", 1), (7, "auc", 1), (8, "multi_logloss", 2),
    (9, "multi_error", 2), (10, "ndcg", 3), (11, "mape", 0), (12, "fair", 0), (13, "poisson", 0),
    (14, "gamma", 0), (15, "gamma_deviance", 0), (16, "tweedie", 0), (17, "cross_entropy", 0),
    (18, "kullback_leibler", 0), (19, "average_precision", 1), (20, "map", 3),
]
_HIGHER_IS_BETTER = {7, 19, 10, 20}              # auc, average_precision, ndcg, map
_NEEDS_PARAM = {3, 4, 12, 16}                    # quantile, huber, fair, tweedie
_MULTICLASS_METRICS = {8, 9}
_RANKING_METRICS = {10, 20}

# metric spellings in METRIC_ALIAS_NAMES order (objective_registry.mojo:2160)
# with the code metric_code_from_name gives each (:1718-1793)
_METRIC_ALIASES = [
    ("l2", 0), ("mean_squared_error", 0), ("mse", 0), ("regression_l2", 0), ("regression", 0),
    ("rmse", 1), ("root_mean_squared_error", 1), ("l2_root", 1),
    ("l1", 2), ("mean_absolute_error", 2), ("mae", 2), ("regression_l1", 2),
    ("quantile", 3), ("huber", 4), ("mape", 11), ("mean_absolute_percentage_error", 11), ("fair", 12),
    ("poisson", 13), ("gamma", 14), ("gamma_deviance", 15), ("gamma_dev", 15), ("tweedie", 16),
    ("cross_entropy", 17), ("xentropy", 17), ("kullback_leibler", 18), ("kldiv", 18),
    ("binary_logloss", 5), ("binary", 5), ("binary_error", 6), ("auc", 7), ("average_precision", 19),
    ("multi_logloss", 8), ("multiclass", 8), ("softmax", 8), ("multi_error", 9),
    ("ndcg", 10), ("lambdarank", 10), ("map", 20), ("mean_average_precision", 20),
]

# objective codes (objective_registry.mojo:273-332), in all_objective_codes
# order (:2202-2230)
SQUARED_ERROR, BINARY_LOGISTIC, POISSON, HUBER, QUANTILE, L1 = 0, 1, 2, 3, 4, 5
CUSTOM, LAMBDARANK, GAMMA, TWEEDIE, MAPE, FAIR, CROSS_ENTROPY = 6, 7, 8, 9, 10, 11, 12
MULTICLASS = -1
_OBJECTIVE_ORDER = [SQUARED_ERROR, BINARY_LOGISTIC, POISSON, HUBER, QUANTILE, L1, GAMMA, TWEEDIE, MAPE, FAIR,
                    CROSS_ENTROPY, MULTICLASS, LAMBDARANK, CUSTOM]
_OBJECTIVE_NAME = {SQUARED_ERROR: "regression", BINARY_LOGISTIC: "binary", POISSON: "poisson", HUBER: "huber",
                   QUANTILE: "quantile", L1: "mae", GAMMA: "gamma", TWEEDIE: "tweedie", MAPE: "mape", FAIR: "fair",
                   CROSS_ENTROPY: "cross_entropy", MULTICLASS: "multiclass", LAMBDARANK: "lambdarank",
                   CUSTOM: "custom"}
_BUILTIN = {SQUARED_ERROR, BINARY_LOGISTIC, POISSON, HUBER, QUANTILE, L1, GAMMA, TWEEDIE, MAPE, FAIR, CROSS_ENTROPY}
_DEFAULT_METRIC = {SQUARED_ERROR: 0, L1: 2, HUBER: 4, QUANTILE: 3, POISSON: 13, GAMMA: 14, TWEEDIE: 16, MAPE: 11,
                   FAIR: 12, CROSS_ENTROPY: 17, BINARY_LOGISTIC: 5, MULTICLASS: 8, LAMBDARANK: 10, CUSTOM: -1}

# objective spellings in OBJECTIVE_ALIAS_NAMES order (:2122-2127) with the
# code objective_code_from_name gives each (:943-990)
_OBJECTIVE_ALIASES = [
    ("regression", 0), ("regression_l2", 0), ("l2", 0), ("mean_squared_error", 0), ("mse", 0),
    ("binary", 1), ("poisson", 2), ("huber", 3), ("quantile", 4),
    ("mae", 5), ("regression_l1", 5), ("l1", 5), ("mean_absolute_error", 5),
    ("gamma", 8), ("tweedie", 9), ("mape", 10), ("mean_absolute_percentage_error", 10), ("fair", 11),
    ("cross_entropy", 12), ("xentropy", 12), ("multiclass", -1), ("softmax", -1), ("lambdarank", 7),
    ("custom", 6),
]

# name-status vocabulary (objective_registry.mojo:453-455)
NAME_SUPPORTED, NAME_UNIMPLEMENTED, NAME_UNKNOWN = 0, 1, 2


def _objective_task(code):
    return {BINARY_LOGISTIC: 1, MULTICLASS: 2, LAMBDARANK: 3}.get(code, 0)


def _objective_link(code):
    if code in (BINARY_LOGISTIC, CROSS_ENTROPY):
        return LINK_SIGMOID
    if code in (POISSON, GAMMA, TWEEDIE):
        return LINK_EXP
    return LINK_SOFTMAX if code == MULTICLASS else LINK_IDENTITY


def _objective_param_name(code):
    return {HUBER: "alpha", QUANTILE: "alpha", FAIR: "fair_c", TWEEDIE: "tweedie_variance_power"}.get(code, "")


def registry_metrics():
    out = []
    for code, name, task in _METRICS:
        needs = (NEEDS_PARAM if code in _NEEDS_PARAM else NEEDS_N_CLASSES if code in _MULTICLASS_METRICS
                 else NEEDS_GROUPS | NEEDS_CUTOFF if code in _RANKING_METRICS else NEEDS_NOTHING)
        transform = (TRANSFORM_SOFTMAX if code in _MULTICLASS_METRICS else TRANSFORM_RAW if code in _RANKING_METRICS
                     else TRANSFORM_OBJECTIVE_LINK)
        out.append([code, name, _TASK[task], code in _HIGHER_IS_BETTER, needs, transform])
    return out


def registry_metric_aliases():
    return [[a, c] for a, c in _METRIC_ALIASES]


def registry_objectives():
    out = []
    for code in _OBJECTIVE_ORDER:
        default_param = 1.0 if code == FAIR else 1.5 if code == TWEEDIE else 0.9
        needs_groups = code == LAMBDARANK
        out.append([code, _OBJECTIVE_NAME[code], _TASK[_objective_task(code)], _objective_link(code),
                    _objective_param_name(code), default_param, code in (QUANTILE, L1, MAPE), code == MULTICLASS,
                    needs_groups, code in _BUILTIN, SUPPORTS_CPU if needs_groups else SUPPORTS_CPU | SUPPORTS_GPU,
                    code in _BUILTIN, _DEFAULT_METRIC[code]])
    return out


def registry_objective_aliases():
    return [[a, c] for a, c in _OBJECTIVE_ALIASES]


def registry_vocabulary():
    return {"n_builtin_metrics": len(_METRICS), "name_supported": NAME_SUPPORTED,
            "name_unimplemented": NAME_UNIMPLEMENTED, "name_unknown": NAME_UNKNOWN}


def metric_code_of_name(name):
    for alias, code in _METRIC_ALIASES:
        if alias == name:
            return code
    raise ValueError(f"unknown metric '{name}'")


def objective_code_of_name(name):
    for alias, code in _OBJECTIVE_ALIASES:
        if alias == name:
            return code
    known = ", ".join(a for a, _ in _OBJECTIVE_ALIASES)
    raise ValueError(f"unknown objective '{name}'; expected one of {known}")


def objective_name_status_of(name):
    return NAME_SUPPORTED if any(a == name for a, _ in _OBJECTIVE_ALIASES) else NAME_UNKNOWN


def registry_objective_unimplemented():
    # The reference lists LightGBM objectives it has not implemented, with a
    # reason each; none of them reaches this library's trainer either, and
    # they resolve as unknown names here.
    return []
