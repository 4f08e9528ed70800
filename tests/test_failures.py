"""Failure detection without GPU faults: a corrupt checkpoint is refused and resume falls back to the newest intact
one; a rank that dies makes the surviving rank's next collective fail within the process-group timeout; a message
the SSD drafter never sends ends the target's wait with an error; on the GPU a bounded device wait that nothing
satisfies reports its status instead of hanging."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import economize_b200 as eco
from economize_b200.train.checkpoint import RunCheckpointer, verify


def _save(ck: RunCheckpointer, step: int) -> None:
    ck.save(step, {"w": torch.full((4,), float(step))}, None, None, {})


def test_corrupt_checkpoint_is_refused_and_skipped(tmp_path):
    ck = RunCheckpointer(tmp_path, keep=3)
    _save(ck, 1)
    _save(ck, 2)
    newest = ck.latest()
    assert newest.name == "checkpoint-2" and verify(newest)
    data = bytearray((newest / "weights.pt").read_bytes())
    data[len(data) // 2] ^= 0xFF  # a flipped byte in the newest shard
    (newest / "weights.pt").write_bytes(bytes(data))
    assert not verify(newest)
    with pytest.raises(eco.CheckpointFormatError):
        RunCheckpointer.load(newest)
    assert ck.latest().name == "checkpoint-1"
    w, state = RunCheckpointer.load(ck.latest())
    assert float(w["w"][0]) == 1.0 and state["step"] == 1


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dying_worker(rank, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import time

    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=5))
    t = torch.ones(4)
    dist.all_reduce(t)  # both ranks alive
    if rank == 1:
        os._exit(0)  # the rank dies between steps, without a word
    start = time.monotonic()
    try:
        dist.all_reduce(t)
        queue.put(("no error", time.monotonic() - start))
    except Exception as err:  # the surviving rank learns of it from its collective
        queue.put((type(err).__name__, time.monotonic() - start))


def test_dead_rank_fails_the_next_collective():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_dying_worker, args=(r, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        kind, waited = queue.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert kind != "no error" and waited < 60, (kind, waited)


def _ssd_drop_worker(rank, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    from economize_b200.parallel.ssd import AsyncSpeculativeDecoder, SSDConfig

    from .helpers import prompts, tiny_model

    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=5))
    if rank == 1:  # the drafter receives the root and then drops out without sending its spine
        first = torch.zeros(2, dtype=torch.long)
        dist.recv(first, 0)
        os._exit(0)
    try:
        AsyncSpeculativeDecoder(tiny_model(), SSDConfig(draft_length=2, fanout=1)).generate(prompts((9,))[0], 8)
        queue.put("no error")
    except Exception as err:
        queue.put(type(err).__name__)


def test_dropped_ssd_message_ends_the_wait():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_ssd_drop_worker, args=(r, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        kind = queue.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert kind != "no error", kind


@pytest.mark.gpu
def test_bounded_device_wait_reports_a_timeout(cuda):
    """An expert-parallel segments kernel waits for dispatch arrivals that nothing sends: after its bounded wait it
    sets the wait-peer status bit and returns; the host turns that into CommTimeoutError."""
    from economize_b200.ops._ext import require
    from economize_b200.parallel.moe import FusedExpertParallel

    C = require()
    C.status(cuda.index or 0)  # clear
    own, _ = C.symm_alloc(C.ep_buffer_bytes(1, 2, 8, 64, 8))
    try:
        status = C.ep_wait_probe(own, 2, 8, 64, 8)
        assert status & 8, status
        ep = FusedExpertParallel(0, 1)
        ep._ext = C
        with pytest.raises(eco.CommTimeoutError):
            # the probe left the status bit set once more for check() to read
            C.ep_wait_probe(own, 2, 8, 64, 8, keep_status=True)
            ep.check()
    finally:
        torch.cuda.synchronize()
        C.symm_free(own)
