"""Data-parallel fit over 2 GPUs (one process per GPU, NCCL) against the
single-GPU fit of the same rows: every tree bit-identical (integer histogram
sums are exact in any order; the scale, the rounding streams and the pick
replay are global).  Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]

N_SHARD = 40_960  # a multiple of 1024 rows per shard (fixed-point mode needs it)
N_SHARD_RAGGED = 30_001  # quantized mode takes any shard size


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data(quant, n_shard=N_SHARD):
    rng = np.random.default_rng(5)
    n = 2 * n_shard
    bins = rng.integers(0, 63, size=(12, n), dtype=np.uint8)
    s = bins[0].astype(np.float64) / 63 - bins[3].astype(np.float64) / 90 + 0.3 * rng.standard_normal(n)
    y = (s > 0.1).astype(np.float64)
    params = {"objective": "binary", "num_iterations": 4, "num_leaves": 31, "max_bin": 63,
              "use_quantized_grad": quant}
    return bins, y, params


def _rank_main(rank, world, port, quant, n_shard, out_q, exchange="allreduce", extra=None):
    import torch.distributed as dist

    if exchange == "feature":
        os.environ["MOJOTREES_DP_EXCHANGE"] = "feature"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import mojoboost_b200 as mb

        bins, y, params = _data(quant, n_shard)
        params = dict(params, gpu_device_id=rank, **(extra or {}))
        nid = torch.from_numpy(mb.nccl_unique_id() if rank == 0 else np.zeros(128, np.uint8))
        dist.broadcast(nid, 0)
        lo, hi = rank * n_shard, (rank + 1) * n_shard
        m = mb.train_binned_dp(np.ascontiguousarray(bins[:, lo:hi]), 63, y[lo:hi], nid.numpy(), rank, world, lo,
                               world * n_shard, params)
        out_q.put((rank, [m.tree(t) for t in range(m.num_trees)]))
    finally:
        dist.destroy_process_group()


# exchange "allreduce" (the default) sums every work slot on every rank;
# "feature" reduce-scatters them by feature block and merges per-child bests
# (MOJOTREES_DP_EXCHANGE=feature).  feature_fraction 0.25 leaves some trees
# with no active feature in one rank's block.
@pytest.mark.parametrize("quant,n_shard,exchange,extra", [
    (True, N_SHARD, "allreduce", None), (False, N_SHARD, "allreduce", None), (True, N_SHARD_RAGGED, "allreduce", None),
    (True, N_SHARD, "feature", None), (False, N_SHARD, "feature", None), (True, N_SHARD_RAGGED, "feature", None),
    (True, N_SHARD, "feature", {"feature_fraction": 0.25}),
    (False, N_SHARD, "allreduce", {"gpu_histogram_precision": "int64"}),
    (False, N_SHARD, "feature", {"gpu_histogram_precision": "int64"}),
])
def test_two_gpu_fit_equals_single_gpu(mtlib, quant, n_shard, exchange, extra):
    import torch.multiprocessing as mp

    bins, y, params = _data(quant, n_shard)
    single = mtlib.train_binned(bins, 63, y, dict(params, gpu_device_id=0, **(extra or {})))
    ref = [single.tree(t) for t in range(single.num_trees)]
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, quant, n_shard, q, exchange, extra))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank in range(world):
        trees = results[rank]
        assert len(trees) == len(ref), f"rank {rank}: {len(trees)} trees vs {len(ref)}"
        for t, (a, b) in enumerate(zip(trees, ref)):
            for k in b:
                np.testing.assert_array_equal(np.asarray(a[k]), np.asarray(b[k]), err_msg=f"rank {rank} tree {t} {k}")
