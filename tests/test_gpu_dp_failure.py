"""Failure handling of the data-parallel fit on 2 GPUs: no rank blocks
forever on another.

The failures are made on the host, never on the GPU: (1) one rank stops
participating after a completed round (a test hook: it sleeps with nothing in
flight, its communicator and memory intact, then fails); (2) one rank never
joins the communicator.  The surviving rank must return an error within its
`dp_timeout_seconds` (plus slack) instead of blocking: its bounded host wait
aborts the NCCL communicator, which ends the collective waiting for the peer.
NVLS is off in both processes (NCCL_NVLS_ENABLE=0), as a rank leaving while
its memory is bound to an NVLink multicast object faults the other GPUs.
"""
import os
import socket
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]

TIMEOUT_S = 5.0
STALL_S = 20.0


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, scenario, out_q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    if scenario == "stall":
        os.environ["MOJOTREES_DP_TEST_STALL_RANK"] = "1"
        os.environ["MOJOTREES_DP_TEST_STALL_AFTER_ROUNDS"] = "1"
        os.environ["MOJOTREES_DP_TEST_STALL_S"] = str(STALL_S)
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import mojoboost_b200 as mb

    n = 20_480
    rng = np.random.default_rng(rank)
    bins = rng.integers(0, 63, size=(8, n), dtype=np.uint8)
    y = (rng.random(n) < 0.5).astype(np.float64)
    params = {"objective": "binary", "num_iterations": 6, "num_leaves": 15, "max_bin": 63,
              "use_quantized_grad": True, "gpu_device_id": rank, "dp_timeout_seconds": TIMEOUT_S}
    nid = torch.from_numpy(mb.nccl_unique_id() if rank == 0 else np.zeros(128, np.uint8))
    dist.broadcast(nid, 0)
    t0 = time.monotonic()
    if scenario == "absent" and rank == 1:
        outcome = "absent"
    else:
        try:
            mb.train_binned_dp(bins, 63, y, nid.numpy(), rank, world, rank * n, world * n, params)
            outcome = "trained"
        except mb.MojoTreesError as e:
            outcome = "error: " + str(e)
    elapsed = time.monotonic() - t0
    out_q.put((rank, outcome, elapsed))
    # the survivor's result is in before any process leaves (gloo only)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("scenario", ["stall", "absent"])
def test_surviving_rank_errors_within_the_timeout(scenario):
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict((r, (o, t)) for r, o, t in (q.get(timeout=180) for _ in range(world)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    outcome0, t0 = results[0]
    assert outcome0.startswith("error") and "timed out" in outcome0, outcome0
    assert t0 < TIMEOUT_S + 15.0, f"rank 0 took {t0:.1f} s"
    if scenario == "stall":
        assert "injected failure" in results[1][0], results[1][0]
