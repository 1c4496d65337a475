"""Sequence-sharded chain on 2 GPUs (one process each, NCCL only for the
verification gather) reproduces the single-GPU chain bit for bit, with and
without attention in the chain. The whole forward step (GEMMs and lm_head
included) is bit-identical for prefill and agrees within the fp16
tolerance of the parity tests for decode: a decode
GEMM splits its k range over a cluster by a factor that depends on the rows
of the call (their fp32 partial sums must fit the leader's shared memory),
so 8 rows per GPU and 16 rows on one GPU add their partial sums in different
groupings. Skipped when fewer than 2 GPUs are visible."""
from __future__ import annotations

import os
import socket
import sys
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir, decode, attention, gemm=False):
    try:
        sys.path.insert(0, ROOT)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                          WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        from littlellm_b200 import dist as kd
        from littlellm_b200.chain import ChainRunner, ModelShape, Workload
        kd.init("nccl", dev, timeout_s=120)
        shape = ModelShape("qwen-2l", 896, 14, 2, 64, 4864, 4096, 2, 1e-6, 1e6)
        w = (Workload("d", shape, n_seqs=16, seq_len=1, max_seq=256, decode=True) if decode
             else Workload("p", shape, n_seqs=4, seq_len=64, max_seq=128, decode=False))
        part = ChainRunner(w, device=dev, seed=77, use_pdl=True, shard=(rank, world), attention=attention,
                           gemm=gemm)
        part.run()
        torch.cuda.synchronize(dev)
        last = kd.gather_rows(part.last_rows)
        normed = kd.gather_rows(part.final_norm_out)
        swiglu = kd.gather_rows(part.layers[-1]["swiglu_out"])
        ctx = kd.gather_rows(part.layers[-1]["attn_ctx"]) if attention else None
        logits = kd.gather_rows(part.logits) if gemm else None
        flags = kd.or_over_ranks(int(part.err_flags.item()), dev)
        if rank == 0:
            full = ChainRunner(w, device=dev, seed=77, use_pdl=True, attention=attention, gemm=gemm)
            full.run()
            torch.cuda.synchronize(dev)
            if gemm and decode:  # 8 vs 16 decode rows take different split-K factors
                def same(a, b):  # |a - b| <= 1e-2 + 1e-2 |b|, the parity tolerance
                    a, b = a.float(), b.float()
                    return bool(((a - b).abs() <= 1e-2 + 1e-2 * b.abs()).all())
            else:
                same = torch.equal
            ok = (same(last, full.last_rows) and same(normed, full.final_norm_out)
                  and same(swiglu, full.layers[-1]["swiglu_out"]) and flags == 0)
            if attention:
                ok = ok and same(ctx, full.layers[-1]["attn_ctx"])
            if gemm:
                ok = ok and same(logits, full.logits)
            with open(os.path.join(out_dir, "result"), "w") as f:
                f.write("ok" if ok else "mismatch")
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    except Exception:
        with open(os.path.join(out_dir, f"error{rank}"), "w") as f:
            f.write(traceback.format_exc())
        raise


@pytest.mark.parametrize("attention,gemm", [(False, False), (True, False), (True, True)])
@pytest.mark.parametrize("decode", [False, True])
def test_two_gpu_shards_equal_single_gpu(tmp_path, decode, attention, gemm):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path), decode, attention, gemm))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish in 300 s")
    errs = "".join(open(os.path.join(tmp_path, f)).read() for f in os.listdir(tmp_path) if f.startswith("error"))
    assert all(p.exitcode == 0 for p in procs), errs
    assert open(os.path.join(tmp_path, "result")).read() == "ok"
