"""Failure detection and recovery, exercised on the host (CPU Gloo ranks, files).

A rank that dies between steps is noticed through the store heartbeat before the
next collective; a collective with a dead peer ends with an error within the
process-group timeout; a hung loop trips the watchdog; a partially written
checkpoint is never picked by resume; a non-finite gradient aborts the step; a
failing dataset item is replaced.
"""
import os
import socket
import tempfile
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from osp_next_b200.utils.watchdog import RankHeartbeat, StepWatchdog


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _hb_worker(rank, port, out):
    store = dist.TCPStore("127.0.0.1", port, 2, rank == 0, timeout=timedelta(seconds=20))
    hb = RankHeartbeat(store, rank, 2, timeout_s=0.5)
    hb.beat(0)
    if rank == 1:
        return                       # rank 1 "dies" after step 0, between steps
    time.sleep(1.5)
    hb.beat(1)
    with open(out, "w") as f:
        f.write(",".join(map(str, hb.dead_ranks())))
    store.set("done", "1")


def test_dead_rank_detected_by_heartbeat():
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "dead.txt")
        mp.start_processes(_hb_worker, args=(_port(), out), nprocs=2, join=True, start_method="spawn")
        assert open(out).read() == "1"


def _pg_worker(rank, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=3))
    if rank == 1:
        os._exit(0)                  # leaves without joining the next collective
    t0 = time.time()
    try:
        dist.all_reduce(torch.ones(4))
        res = "no-error"
    except Exception as e:          # the survivor gets an error instead of waiting forever
        res = f"error:{type(e).__name__}"
    with open(out, "w") as f:
        f.write(f"{res},{time.time() - t0:.1f}")


def test_collective_with_dead_peer_errors_within_timeout():
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "pg.txt")
        ctx = mp.start_processes(_pg_worker, args=(_port(), out), nprocs=2, join=False, start_method="spawn")
        deadline = time.time() + 90
        while not ctx.join(timeout=2) and time.time() < deadline:
            pass
        res, dt = open(out).read().split(",")
        assert res.startswith("error") and float(dt) < 30


def test_watchdog_fires_on_stall():
    fired = []
    wd = StepWatchdog(0.3, on_timeout=fired.append, poll_s=0.05)
    for _ in range(5):
        wd.heartbeat()
        time.sleep(0.05)
    assert not fired
    time.sleep(0.6)
    wd.stop()
    assert fired and fired[0] > 0.3


def test_partial_checkpoint_is_ignored(tmp_path):
    from osp_next_b200.parallel.checkpoint import Checkpointer, get_latest_checkpoint_folder
    m = torch.nn.Linear(4, 4)
    ck = Checkpointer(str(tmp_path))
    ck.save(10, m)
    os.makedirs(tmp_path / "iter_000000020.tmp")            # crash mid-save
    os.makedirs(tmp_path / "iter_000000030")                # directory without weights
    assert get_latest_checkpoint_folder(str(tmp_path)) == 10
    m2 = torch.nn.Linear(4, 4)
    Checkpointer(str(tmp_path)).load_model(m2)
    assert torch.equal(m.weight, m2.weight)


def test_nonfinite_grad_aborts_step():
    from osp_next_b200.utils.clip_grads import AdaptiveGradClipper
    p = torch.nn.Parameter(torch.ones(3))
    p.grad = torch.tensor([1.0, float("nan"), 0.0])
    with pytest.raises(RuntimeError):
        AdaptiveGradClipper().adaptive_clip([p])


def test_failing_dataset_item_is_replaced(tmp_path):
    from osp_next_b200.data.datasets.t2v_dataset import WanT2VDataset
    meta = tmp_path / "meta.jsonl"
    meta.write_text('{"path": "/nonexistent.mp4", "cap": "x", "num_frames": 10, "fps": 16}\n' * 3)
    ds = WanT2VDataset(str(meta), None, sample_height=32, sample_width=32, sample_num_frames=5, train_fps=16,
                       timeout=5)
    with pytest.raises(RuntimeError):       # every item fails → bounded retries then a clear error
        ds[0]
