"""Host side of the data-parallel path on CPU ranks (gloo, world size 2).

What needs no GPU: rank 0 makes the NCCL unique id through the library,
torch.distributed (gloo) broadcasts it, every rank holds the same bytes, and a
data-parallel fit that the ranks cannot run (no CUDA device here) is refused
the same way on every rank, before any collective, so no rank waits on
another.  Also the argument checks every rank applies before joining.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.skipif(torch.cuda.is_available(), reason="host-only test (a GPU box runs the real path)")


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import mojoboost_b200 as mb

        nid = torch.from_numpy(mb.nccl_unique_id() if rank == 0 else np.zeros(128, np.uint8))
        dist.broadcast(nid, 0)
        ids = [torch.zeros(128, dtype=torch.uint8) for _ in range(world)]
        dist.all_gather(ids, nid)
        same = all(torch.equal(ids[0], x) for x in ids)
        nonzero = bool(ids[0].any())
        n_local = 2048
        rng = np.random.default_rng(rank)
        bins = rng.integers(0, 16, size=(4, n_local), dtype=np.uint8)
        y = (rng.random(n_local) < 0.5).astype(np.float64)
        params = {"objective": "binary", "num_iterations": 2, "num_leaves": 7, "use_quantized_grad": True}
        try:
            mb.train_binned_dp(bins, 16, y, nid.numpy(), rank, world, rank * n_local, world * n_local, params)
            outcome = "trained"
        except mb.UnsupportedError as e:
            outcome = "unsupported: " + str(e)
        # bad arguments are refused locally, also before any collective
        try:
            mb.train_binned_dp(bins, 16, y, nid.numpy(), rank, world, world * n_local, world * n_local, params)
            bad = "accepted"
        except mb.MojoTreesError as e:
            bad = type(e).__name__ + ": " + str(e)
        dist.barrier()
        out_q.put((rank, same, nonzero, outcome, bad))
    finally:
        dist.destroy_process_group()


def test_two_cpu_ranks_share_the_id_and_refuse_together():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    assert [r[0] for r in results] == [0, 1]
    for rank, same, nonzero, outcome, bad in results:
        assert same and nonzero, f"rank {rank}: NCCL id not shared"
        assert outcome.startswith("unsupported") and "CUDA device" in outcome, f"rank {rank}: {outcome}"
        assert "row_offset" in bad, f"rank {rank}: {bad}"
