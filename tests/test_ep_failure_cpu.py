"""Failure detection of the expert-parallel exchange (nemotron-super-8gb_b200/ep.py) on CPU ranks over gloo, world
size 2, with no GPU involved: a rank leaves between two ExpertParallelMoE steps, with none of its collectives in
flight, and the remaining rank's next step must end with an error from the process group instead of hanging.

Two ways of leaving: the rank stops taking collective steps while staying alive (the surviving rank's next
all_to_all runs into the process group's timeout, given at init_process_group), or the rank's process exits (the
surviving rank's next all_to_all fails on the closed connection). The device steps are the oracle's CPU
restatements (test_ep_cpu.OracleOps), so only the host protocol runs. The reference engine has no counterpart:
its only guard is an assert on the expert cache (nem_super.py:131)."""
import datetime
import os
import queue
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from test_ep_cpu import NE, OracleOps, _bank, _free_port, _inputs

PG_TIMEOUT_S = 5


def _worker(rank, world, port, mode, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    for p in (os.path.join(here, "..", "nemotron-super-8gb_b200"), os.path.join(here, ".."), os.path.join(here, "golden"),
              here):
        sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
        import ep
        blocks, s2 = _bank()
        lo, hi = ep.shard_bounds(NE, world, rank)
        store = torch.zeros(hi - lo, 8, dtype=torch.uint8)   # shape check only; OracleOps reads the blocks
        layer = ep.ExpertParallelMoE(store, torch.from_numpy(s2[lo:hi]), n_experts=NE, ops=OracleOps(blocks[lo:hi]))
        X, ids, w = (torch.from_numpy(a) for a in _inputs(rank))
        layer(X, ids, w)                                     # step 1: every rank
        q.put((rank, "step1"))
        if rank == 1:                                        # leaves between the steps
            if mode == "exit":
                q.close()
                q.join_thread()
                os._exit(0)
            time.sleep(6 * PG_TIMEOUT_S)                     # alive, but takes no further collective step
            q.put((rank, "left"))
            return
        t0 = time.time()
        try:
            layer(X, ids, w)                                 # step 2: the peer is gone
            q.put((rank, "returned", time.time() - t0, ""))
        except Exception as exc:                             # the failure surfaces here
            q.put((rank, "error", time.time() - t0, f"{type(exc).__name__}: {str(exc)[:200]}"))
    except Exception as exc:
        q.put((rank, "setup error", 0.0, repr(exc)))
    finally:
        q.close()
        q.join_thread()
        os._exit(0)   # no process-group teardown with a peer missing


@pytest.mark.parametrize("mode", ["stall", "exit"])
def test_ep_rank_leaving_between_steps_is_detected(mode):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        msgs = {}
        deadline = time.time() + 240
        while time.time() < deadline and not any(m[0] == 0 and m[1] != "step1" for m in msgs.values()):
            try:
                m = q.get(timeout=5)
            except queue.Empty:
                continue
            msgs[(m[0], m[1])] = m
        assert (0, "step1") in msgs and (1, "step1") in msgs, msgs
        res = [m for m in msgs.values() if m[0] == 0 and m[1] != "step1"]
        assert res, f"rank 0 neither failed nor returned: {msgs}"
        _, kind, dt, text = res[0]
        assert kind == "error", f"rank 0's step 2 {kind} after the peer left ({text})"
        # bounded: the process-group timeout (stall) or the closed connection (exit), not a hang
        assert dt < 6 * PG_TIMEOUT_S, dt
        if mode == "stall":
            assert dt >= 0.5 * PG_TIMEOUT_S, dt   # it waited for the peer up to the timeout
    finally:
        for p in procs:
            p.join(timeout=10 * PG_TIMEOUT_S)
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
