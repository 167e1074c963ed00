"""Failure detection without any GPU fault: a rank leaves between steps and
the surviving rank stops with a bounded, named error instead of hanging."""
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from tests._fault_worker import run, run_mismatch, run_multinode


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("grad_mode", ["gpu_reduce", "cpu_reduce"])
def test_dead_rank_detected_by_survivor(tmp_path, grad_mode):
    out = str(tmp_path / "res")
    ctx = mp.get_context("spawn")
    port = _port()
    ps = [ctx.Process(target=run, args=(r, 2, port, out, grad_mode)) for r in range(2)]
    t0 = time.time()
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=240)
    assert time.time() - t0 < 240, "survivor hung"
    r0 = torch.load(out + ".0")
    r1 = torch.load(out + ".1")
    assert r1.get("left")
    assert r0["error"] is not None, "rank 0 should have failed"
    msg = r0["error"].lower()
    assert ("timed out" in msg or "timeout" in msg or "connection" in msg or "closed" in msg
            or "peer" in msg or "gloo" in msg), r0["error"]


def test_closed_rank_reported_at_next_step(tmp_path):
    """A rank that closes its engine between steps is named at once by the
    others' next step (no timeout needed)."""
    out = str(tmp_path / "res")
    ctx = mp.get_context("spawn")
    port = _port()
    ps = [ctx.Process(target=run, args=(r, 2, port, out, "gpu_reduce", "close")) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=240)
    r0 = torch.load(out + ".0")
    assert torch.load(out + ".1").get("left")
    assert r0["error"] is not None and r0["error"].startswith("RankLeftError"), r0["error"]
    assert "rank 1 left the run after step 1" in r0["error"], r0["error"]
    assert r0["steps"] == 1


def test_update_wait_timeout_names_layer():
    from test1_b200.runtime.host_memory import HostRegion
    from test1_b200.runtime.update import UpdateScheduler

    region = HostRegion(4096)
    ctr = region.view(torch.uint8, 0, 64)
    sch = UpdateScheduler(ctr, timeout_s=0.3)
    t0 = time.time()
    with pytest.raises(TimeoutError, match="layer 3 parameter update timed out"):
        sch.wait_counter(3, 5)
    assert time.time() - t0 < 5
    sch.close()
    region.close()


def test_rank_with_another_layout_refuses_the_shared_region(tmp_path):
    out = str(tmp_path / "res")
    ctx = mp.get_context("spawn")
    port = _port()
    ps = [ctx.Process(target=run_mismatch, args=(r, 2, port, out)) for r in range(2)]
    t0 = time.time()
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=240)
    assert time.time() - t0 < 240, "a rank hung"
    r1 = torch.load(out + ".1")
    assert r1["error"] is not None and "every local rank must run the same model" in r1["error"], r1
    assert torch.load(out + ".0")["error"] is not None  # the creator's next collective fails, bounded


def test_region_header_detects_overwrite_and_corruption(tmp_path):
    from test1_b200.runtime.host_memory import (REGION_HEADER_BYTES, HostRegion, check_region_header,
                                                write_region_header)

    path = f"/dev/shm/t1b200_test_{os.getpid()}.bin"
    fields = {"region_bytes": 8192, "world_size": 2, "num_layers": 6, "total_params": 12345,
              "layout_code": 77}
    owner = HostRegion(8192, shm_path=path, create=True)
    try:
        write_region_header(owner, 0, fields)
        peer = HostRegion(8192, shm_path=path, create=False)
        check_region_header(peer, 0, fields, rank=1)
        with pytest.raises(RuntimeError, match="num_layers = 6, this rank expects 5"):
            check_region_header(peer, 0, dict(fields, num_layers=5), rank=1)
        words = owner.view(torch.int64, 0, REGION_HEADER_BYTES // 8)
        words[4] += 1  # one flipped field: the checksum no longer matches
        with pytest.raises(RuntimeError, match="corrupt"):
            check_region_header(peer, 0, fields, rank=1)
        words[0] = 0  # overwritten by something else
        with pytest.raises(RuntimeError, match="no test1_b200 header"):
            check_region_header(peer, 0, fields, rank=1)
        peer.close()
    finally:
        owner.close()


def test_ranks_on_several_nodes_are_refused(tmp_path):
    out = str(tmp_path / "res")
    ctx = mp.get_context("spawn")
    port = _port()
    ps = [ctx.Process(target=run_multinode, args=(r, 2, port, out)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
    for r in range(2):
        err = torch.load(out + f".{r}")["error"]
        assert err is not None and "runs on one node" in err, err
