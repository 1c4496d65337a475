"""Multi-rank host logic on the CPU (gloo, world size 2): sequence sharding,
the verification gather, max/OR over ranks, and detection of a rank that dies
before a collective. The per-rank compute stand-in is the oracle."""
from __future__ import annotations

import os
import socket
import sys
import traceback

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank: int, world: int, port: int, timeout_s: float = 60.0):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    from littlellm_b200 import dist as kd
    kd.init("gloo", timeout_s=timeout_s)
    return kd


def _worker_gather(rank, world, port, out_dir):
    try:
        import torch
        import torch.distributed as dist
        kd = _setup(rank, world, port)
        from oracle.oracle import Oracle
        o = Oracle()
        n_seqs, seq_len, H = 6, 5, 16
        rng = np.random.default_rng(123)  # same global batch on every rank
        x = rng.standard_normal((n_seqs * seq_len, H)).astype(np.float32)
        s0, s1 = kd.shard_range(n_seqs, rank, world)
        local_x = x[s0 * seq_len:s1 * seq_len]
        local_last, rc = o.select_last_rows(local_x, seq_len=seq_len, n_seqs=s1 - s0)
        assert rc == 0
        gathered = kd.gather_rows(torch.from_numpy(local_last))
        t_max = kd.max_over_ranks(float(rank + 1))
        flags = kd.or_over_ranks(1 << rank)
        if rank == 0:
            full, _ = o.select_last_rows(x, seq_len=seq_len, n_seqs=n_seqs)
            ok = (np.array_equal(gathered.numpy(), full) and t_max == float(world)
                  and flags == (1 << world) - 1)
            with open(os.path.join(out_dir, "result"), "w") as f:
                f.write("ok" if ok else f"mismatch t_max={t_max} flags={flags}")
        else:
            assert gathered is None
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(out_dir, f"error{rank}"), "w") as f:
            f.write(traceback.format_exc())
        raise


def _worker_dead_peer(rank, world, port, out_dir):
    import time

    import torch
    kd = _setup(rank, world, port, timeout_s=5.0)
    if rank == 1:
        os._exit(3)  # leaves between steps, before the gather
    t0 = time.time()
    try:
        kd.gather_rows(torch.zeros(2, 4))
        outcome = "no error"
    except Exception as e:  # noqa: BLE001 - any collective failure is the detection
        outcome = f"detected after {time.time() - t0:.1f}s: {type(e).__name__}"
    with open(os.path.join(out_dir, "result"), "w") as f:
        f.write(outcome)
    os._exit(0)


def _spawn(fn, tmp_path, world=2):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish in 120 s")
    return procs


def test_shard_range():
    sys.path.insert(0, ROOT)
    from littlellm_b200.dist import shard_range
    assert [shard_range(8, r, 4) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    assert shard_range(2048, 7, 8) == (1792, 2048)
    with pytest.raises(ValueError):
        shard_range(10, 0, 4)
    with pytest.raises(ValueError):
        shard_range(8, 4, 4)


def test_sharded_gather_matches_unsharded(tmp_path):
    procs = _spawn(_worker_gather, tmp_path)
    errors = [p.name for p in procs if p.exitcode != 0]
    msg = "".join(open(os.path.join(tmp_path, f)).read() for f in os.listdir(tmp_path) if f.startswith("error"))
    assert not errors, msg
    assert open(os.path.join(tmp_path, "result")).read() == "ok"


def test_dead_rank_is_detected_not_hung(tmp_path):
    _spawn(_worker_dead_peer, tmp_path)
    result = open(os.path.join(tmp_path, "result")).read()
    assert result.startswith("detected"), result
