"""A rank leaves between steps on 2 GPUs (NCCL ranks, NVLS off, no symmetric
memory, short process-group timeout): the surviving rank must stop at the
start of its next step with an error that names the departed rank, within
the configured host wait, and its GPU must still run kernels afterwards.
No GPU is faulted: the departing rank has no kernel or collective in flight
when it leaves, and the survivor learns of it on the host (the step-entry
heartbeat in shared host memory) before it launches anything of the step."""
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from tests._fault_worker import run

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("leave", ["close", "exit"])
def test_rank_leaves_between_steps_two_gpus(tmp_path, leave):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = str(tmp_path / "res")
    ctx = mp.get_context("spawn")
    port = _port()
    ps = [ctx.Process(target=run, args=(r, 2, port, out, "gpu_reduce", leave, True)) for r in range(2)]
    t0 = time.time()
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=300)
    assert all(p.exitcode is not None for p in ps), "a rank hung"
    r0 = torch.load(out + ".0")
    assert torch.load(out + ".1").get("left")
    assert r0["steps"] == 1, r0
    err = r0["error"] or ""
    if leave == "close":
        assert err.startswith("RankLeftError") and "rank 1 left the run after step 1" in err, err
    else:
        assert err.startswith("TimeoutError") and "rank 1 did not start step 2" in err, err
    assert r0["gpu_ok"], r0.get("gpu_error")
    assert time.time() - t0 < 300
