#!/usr/bin/env python
"""Layer-op chain benchmark: tokens/s and achieved HBM GB/s on B200.

One step = the whole non-GEMM op chain of one decoder forward step
(embedding; per layer add+RMSNorm, fused bias+RoPE+KV append, add+RMSNorm,
SwiGLU; final add+RMSNorm; select_last_rows) over one batch of seeded
synthetic inputs, launched by the native chain executor and replayed as a CUDA
graph. Default workload: Qwen2.5-0.5B shapes, 8 sequences x 512 tokens = 4096
tokens per GPU, 24 layers, KV cache [24, 2, 8, 2, 4096, 64] fp16.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)
    python bench.py --impl reference ...   (the reference CPU implementation)

Rank 0 prints one JSON line. `value` is whole-job tokens/s from CUDA-event
device time, max over ranks; `e2e` is the same metric through the C ABI with
the step's inputs copied from pinned host memory and the result copied back
inside the timed region; `roofline` is the dominant kernel (SwiGLU) timed
alone over its per-layer buffers; `cpu_baseline` times the reference's own
CPU operators (compiled from its sources, oracle/_ref) on a bounded sample.
"""
from __future__ import annotations

import argparse
from dataclasses import replace
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "layer-op tokens/s"
UNIT = "tokens/s"


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="qwen_prefill")
    ap.add_argument("--no-pdl", action="store_true", help="launch without programmatic dependent launch")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-other-configs", action="store_true",
                    help="time only the headline workload (skip the other survey configs and the reference "
                         "CUDA kernels)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample length")
    ap.add_argument("--layers", type=int, default=None,
                    help="run only this many decoder layers (small profiling cases; not a bench line)")
    ap.add_argument("--forward", action="store_true",
                    help="time the whole forward step (chain + attention + tcgen05 GEMMs + lm_head)")
    ap.add_argument("--attention", action="store_true",
                    help="chain workloads: run attention over the cache in every layer as part of the chain")
    ap.add_argument("--sequences", type=int, default=None,
                    help="attention workloads: run this many sequences (small profiling cases; not a bench line)")
    ap.add_argument("--settle-seconds", type=float, default=1.5,
                    help="untimed graph replays before timing so clocks settle under load")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# environment / distributed plumbing
# ---------------------------------------------------------------------------


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def load_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def ncu_traffic(kernel: str, workload: str):
    """dram bytes per launch of `kernel` from the committed ncu summary
    (profiles/<kernel>_<workload>.txt, a line `traffic_bytes_per_launch: N`),
    or None when no capture has been summarised."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_{workload}.txt")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        for line in f:
            if line.startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1]))
    return None


class ClockSampler:
    """Samples SM clock, power and throttle reasons of one GPU with nvidia-smi
    every 200 ms while running."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, torch_device):
        import torch
        p = torch.cuda.get_device_properties(torch_device)
        self.bus = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.bus, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._t.join(timeout=5)
        sm, mx, power, reasons = [], [], [], set()
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
                power.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(self.REASONS, parts[4:8]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own CPU operators (oracle/_ref), or the oracle port
# ---------------------------------------------------------------------------


def time_reference_cpu(model, tokens: int, threads: int, seconds: float, steps: int | None = None,
                       warmup: int = 0):
    """Runs the reference's non-GEMM chain (all layers of `model`) on one
    sequence of `tokens` tokens per thread, `threads` threads in parallel,
    through the reference's public kllm::op API on fp32 CPU tensors.
    Returns (tokens/s, per-step seconds list, kind)."""
    import ctypes
    from concurrent.futures import ThreadPoolExecutor

    from oracle.oracle import Reference, reference_available
    if not reference_available():
        return time_oracle_port(model, tokens, seconds)
    ref = Reference()
    lib = ref.lib
    table = lib.kref_table_create(model.vocab, model.hidden, 0x4B4C4C4D)
    if not table:
        raise RuntimeError(lib.kref_last_error().decode())
    chains = []
    for i in range(threads):
        c = lib.kref_chain_create(table, tokens, model.n_heads, model.n_kv_heads, model.head_dim,
                                  model.intermediate, max(tokens, 512), ctypes.c_float(model.eps),
                                  ctypes.c_float(model.theta), 1000 + i)
        if not c:
            raise RuntimeError(lib.kref_last_error().decode())
        chains.append(c)

    def one(c):
        rc = lib.kref_chain_run(c, model.n_layers)
        if rc != 0:
            raise RuntimeError(lib.kref_last_error().decode())

    step_times = []
    with ThreadPoolExecutor(threads) as ex:
        for _ in range(warmup):
            list(ex.map(one, chains))
        t_start = time.perf_counter()
        while True:
            t0 = time.perf_counter()
            list(ex.map(one, chains))
            step_times.append(time.perf_counter() - t0)
            if steps is not None and len(step_times) >= steps:
                break
            if steps is None and time.perf_counter() - t_start >= seconds:
                break
    for c in chains:
        lib.kref_chain_destroy(c)
    lib.kref_table_destroy(table)
    total = sum(step_times)
    return threads * tokens * len(step_times) / total, step_times, "reference"


def time_oracle_port(model, tokens: int, seconds: float):
    """Fallback when oracle/_ref is absent: the oracle restatement of the same
    chain, single-threaded."""
    import numpy as np

    from oracle.oracle import Oracle
    o = Oracle()
    rng = np.random.default_rng(0)
    H, D = model.hidden, model.head_dim
    table = rng.normal(0, 0.02, (model.vocab, H)).astype(np.float32)
    ids = rng.integers(0, model.vocab, tokens).astype(np.int32)
    q = rng.standard_normal((tokens, model.n_heads, D)).astype(np.float32)
    k = rng.standard_normal((tokens, model.n_kv_heads, D)).astype(np.float32)
    x = rng.standard_normal((tokens, H)).astype(np.float32)
    g = rng.standard_normal((tokens, model.intermediate)).astype(np.float32)
    w = np.ones(H, np.float32)
    steps = []
    t_start = time.perf_counter()
    while time.perf_counter() - t_start < seconds or not steps:
        t0 = time.perf_counter()
        res = o.embedding(table, ids)
        for _ in range(model.n_layers):
            o.rms_norm(res, w, model.eps)
            o.rope(q, 0, model.theta)
            o.rope(k, 0, model.theta)
            res = o.add(res, x)
            o.rms_norm(res, w, model.eps)
            o.silu_mul(g, g)
            res = o.add(res, x)
        o.rms_norm(res, w, model.eps)
        steps.append(time.perf_counter() - t0)
    return tokens * len(steps) / sum(steps), steps, "port"


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------


def run_reference_dequant(args):
    """The reference weight loader's host INT8 -> fp16 loop body
    (src/model/weights.cpp:139-148: float(q) * scale, float_to_half) on the
    host cores, one slice of a 64 M-value sample per thread; metric as our
    arm's (1 B read + 2 B written per value)."""
    import ctypes
    from concurrent.futures import ThreadPoolExecutor

    import numpy as np

    from oracle.oracle import Oracle, Reference, reference_available
    kind = "reference" if reference_available() else "port"
    fn = Reference().lib.kref_dequantize_int8_f16 if kind == "reference" else \
        Oracle().lib.kllm_oracle_dequantize_int8_f16
    threads = host_threads()
    n = 1 << 26
    q = np.random.default_rng(5).integers(-127, 128, n, dtype=np.int8)
    out16 = np.empty(n, np.uint16)
    bounds = np.linspace(0, n, threads + 1).astype(np.int64)

    def one(i):
        lo, hi = int(bounds[i]), int(bounds[i + 1])
        fn(ctypes.c_void_p(q.ctypes.data + lo), hi - lo, ctypes.c_float(0.0047),
           ctypes.c_void_p(out16.ctypes.data + 2 * lo))

    steps = []
    with ThreadPoolExecutor(threads) as ex:
        for _ in range(args.warmup):
            list(ex.map(one, range(threads)))
        for _ in range(args.steps):
            t0 = time.perf_counter()
            list(ex.map(one, range(threads)))
            steps.append(time.perf_counter() - t0)
    value = 3 * n * len(steps) / sum(steps) / 1e9
    emit({"metric": "int8->fp16 dequant throughput", "value": value, "unit": "GB/s", "impl": "reference",
          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
          "ms_per_step": 1000.0 * statistics.mean(steps), "higher_is_better": True, "scaling": "none",
          "vs_baseline": None, "dtype": "i8->f16", "data": "synthetic",
          "config": {"workload": "llama_int8_dequant", "params_per_step": n,
                     "impl_detail": "reference weight-loader dequant loop (src/model/weights.cpp)"},
          "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": kind,
                           "sample": f"{n} int8 values per step split over {threads} threads"},
          "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})


def run_reference_load(args):
    """The reference's own ModelWeights::load (CUDA device, host dequant,
    src/model/weights.cpp:81-160) on the same partial Llama-2-7B INT8 file as
    our arm; each step is one whole load, at most 3 steps (about 7 s each)."""
    import subprocess
    import tempfile
    exe = os.path.join(ROOT, "oracle", "_ref", "refcuda", "ref_load")
    if not os.path.exists(exe):
        emit({"impl": "reference", "unavailable": "oracle/_ref/refcuda/ref_load was not built"})
        return
    layers = args.layers or 4
    times = []
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "llama_int8.kllm")
        names = _write_llama_int8(path, layers)
        file_bytes = os.path.getsize(path)
        names_path = os.path.join(tmp, "names.txt")
        with open(names_path, "w") as f:
            f.write("\n".join(names) + "\n")
        for _ in range(min(max(args.steps, 1), 3)):
            r = subprocess.run([exe, path, names_path], capture_output=True, text=True, timeout=1200)
            if r.returncode != 0:
                emit({"impl": "reference", "unavailable": "ref_load failed: " + r.stderr.strip()[-200:]})
                return
            times.append(float(r.stdout.splitlines()[0].split()[1]))
    value = file_bytes / min(times) / 1e9
    emit({"metric": "int8 .kllm checkpoint load", "value": value, "unit": "GB/s", "impl": "reference",
          "n_gpus": args.gpus, "steps": len(times), "warmup": 0, "ms_per_step": 1000.0 * min(times),
          "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "i8->f16",
          "data": "synthetic",
          "config": {"workload": "llama_int8_load", "layers": layers, "file_bytes": file_bytes,
                     "tensors": len(names), "impl_detail": "reference ModelWeights::load(path, CUDA)"},
          "cpu_baseline": {"value": value, "unit": "GB/s", "cores": 1, "kind": "reference",
                           "sample": f"{len(times)} whole loads of a {file_bytes} B file"},
          "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})


def run_reference(args):
    # the shapes only: this arm must not map libkllm_b200.so
    from littlellm_b200.workloads import WORKLOADS
    world, rank, _ = dist_env()
    if rank != 0:
        return
    if args.workload == "llama_int8_dequant":
        return run_reference_dequant(args)
    if args.workload in ATTENTION_WORKLOADS:
        return run_reference_attention(args)
    if args.workload in GEMM_WORKLOADS:
        return run_reference_gemm(args)
    if args.workload in GENERATE_WORKLOADS:
        emit({"impl": "reference", "metric": GENERATE_METRIC,
              "unavailable": "the reference's generation loop runs only from a .kllm checkpoint; "
                             "not timed for this synthetic workload"})
        return None
    if args.workload == "llama_int8_load":
        return run_reference_load(args)
    w = WORKLOADS[args.workload]
    threads = host_threads()
    tokens = 128
    value, steps, kind = time_reference_cpu(w.model, tokens, threads, 0.0, steps=args.steps,
                                            warmup=args.warmup)
    ms = 1000.0 * statistics.mean(steps)
    sample = (f"{threads} threads x one {tokens}-token sequence each through all {w.model.n_layers} layers "
              f"of the {w.model.name} non-GEMM chain per step (fp32 CPU tensors, kllm::op API)")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak" if args.workload == "qwen_prefill" else "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": w.name, "shapes": w.model.name, "layers": w.model.n_layers,
                   "tokens_per_step": threads * tokens, "impl_detail": "reference CPU operators (src/op/cpu)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------


def time_graph(g, stream, reps: int) -> float:
    """ms per replay of a CUDA graph, CUDA events on its stream."""
    import torch
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(reps):
            g.replay()
        end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / reps


def capture(fn, stream):
    import torch
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    return g


def per_op_timing(runner, stream, reps: int, pdl: bool = False) -> dict:
    """Each op kind timed alone: one graph of that op's C-ABI entry over all
    layers' buffers (several GB, larger than L2), replayed `reps` times. With
    `pdl` the entries launch with programmatic dependent launch
    (kllm_b200_set_pdl), as a runner calling them one by one can ask for."""
    import torch

    from littlellm_b200 import ops
    prev = ops.set_pdl(pdl)
    try:
        return _per_op_timing(runner, stream, reps)
    finally:
        ops.set_pdl(prev)


def _per_op_timing(runner, stream, reps: int) -> dict:
    import torch

    from littlellm_b200 import ops
    w, m = runner.w, runner.w.model
    T, H, D = w.n_tokens, m.hidden, m.head_dim
    L = runner.layers
    eps, theta = m.eps, m.theta

    # distinct ids per launch so table rows are not re-read from L2
    gen = torch.Generator(device=runner.device)
    gen.manual_seed(7)
    ids = [torch.randint(0, m.vocab, (T,), generator=gen, device=runner.device, dtype=torch.int32) for _ in L]

    def embed():
        for layer, idx in zip(L, ids):
            ops.embedding(runner.table, idx, out=layer["attn_norm_out"])

    def norm():
        # per-layer residual buffers (attn_norm_out stands in), so no launch
        # re-reads another's data from L2
        for layer in L:
            ops.add_rms_norm(layer["attn_norm_out"], layer["attn_out"], layer["post_norm_w"], eps,
                             out=layer["ffn_norm_out"])

    def qkv():
        for layer in L:
            ops.qkv_bias_rope_kv_append(layer["q"].view(T, m.n_heads, D), layer["k"].view(T, m.n_kv_heads, D),
                                        layer["v"].view(T, m.n_kv_heads, D), layer["q_bias"], layer["k_bias"],
                                        layer["v_bias"], runner.positions, runner.slots, theta,
                                        layer["k_cache"], layer["v_cache"], runner.err_flags)

    def silu():
        for layer in L:
            ops.silu_mul(layer["gate"], layer["up"], out=layer["swiglu_out"])

    def select():
        # the last row of every sequence, from each layer's own T x H buffer
        for layer in L:
            ops.select_last_rows(layer["ffn_norm_out"], seq_len=w.seq_len, n_seqs=w.n_seqs,
                                 out=layer["attn_norm_out"][:w.n_seqs])

    qkv_bytes = 2 * T * (m.n_heads + 2 * m.n_kv_heads) * D * 2 + 8 * T
    table = {
        "embedding": (embed, 2 * T * H * 2 + 4 * T),
        "add_rms_norm": (norm, 4 * T * H * 2),
        "qkv_bias_rope_kv_append": (qkv, qkv_bytes),
        "silu_mul": (silu, 3 * T * m.intermediate * 2),
        "select_last_rows": (select, 2 * w.n_seqs * H * 2),
    }
    out = {}
    with torch.cuda.stream(stream):
        for name, (fn, nbytes) in table.items():
            fn()  # warm (occupancy caches, clocks)
            g = capture(fn, stream)
            g.replay()
            ms = time_graph(g, stream, reps) / len(L)
            out[name] = {"us_per_launch": ms * 1000.0, "bytes_per_launch": nbytes,
                         "gbs": nbytes / (ms * 1e-3) / 1e9}
            del g
    return out


def measure_dequant(device, steps: int, warmup: int, peaks: dict) -> dict:
    """INT8 -> fp16 dequant of every Llama-2-7B linear/embedding tensor
    (6.74 B parameters, int8 ~U[-127,127], fp32 scale ~U(1e-3,1e-2) per
    tensor) with the reference weight loader's rounding; one step = the whole
    checkpoint, one CUDA graph. Also times the fp32-output form on four
    11008 x 4096 tensors, the form the reference's own GPU op has
    (src/op/cuda/quantize.cu:110-121). Returns the variants and the device
    tensors of the first one (for the CPU sample)."""
    import torch

    from littlellm_b200 import ops
    from littlellm_b200.workloads import LLAMA2_7B_INT8_TENSORS
    gen = torch.Generator(device=device)
    gen.manual_seed(5)
    data, scales, outs = [], [], []
    for rows, cols, count in LLAMA2_7B_INT8_TENSORS:
        for _ in range(count):
            data.append(torch.randint(-127, 128, (rows, cols), generator=gen, device=device, dtype=torch.int8))
            scales.append(torch.rand((1,), generator=gen, device=device) * 9e-3 + 1e-3)
            outs.append(torch.empty((rows, cols), dtype=torch.float16, device=device))
    n_params = sum(d.numel() for d in data)
    nbytes = 3 * n_params + 4 * len(data)
    log(f"dequant: {len(data)} tensors, {n_params} params allocated")
    stream = torch.cuda.Stream(device)
    results = {}
    f32_in = [data[128 + i] for i in range(4)]  # four gate/up tensors, 11008 x 4096
    f32_out = [torch.empty(d.shape, dtype=torch.float32, device=device) for d in f32_in]
    f32_bytes = sum(5 * d.numel() for d in f32_in)
    variants = (
        ("batched", nbytes, 1, lambda: ops.dequantize_int8_batched(data, scales, outs)),
        ("per_tensor", nbytes, len(data),
         lambda: [ops.dequantize_int8(d, sc, out=o) for d, sc, o in zip(data, scales, outs)]),
        ("f32_out_4x11008x4096", f32_bytes, 4,
         lambda: [ops.dequantize_int8(d, scales[0], out=o) for d, o in zip(f32_in, f32_out)]),
    )
    with torch.cuda.stream(stream):
        for name, vbytes, launches, fn in variants:
            fn()
            stream.synchronize()
            g = capture(fn, stream)
            for _ in range(max(warmup, 3)):
                g.replay()
            stream.synchronize()
            ms = time_graph(g, stream, steps)
            gbs = vbytes / (ms * 1e-3) / 1e9
            results[name] = {"ms_per_step": ms, "gbs": gbs, "frac_of_measured": gbs / peaks["hbm_gbs"],
                             "bytes_per_step": vbytes, "launches_per_step": launches}
            del g
    results["_tensors"] = (data, scales)
    results["_meta"] = {"tensors": len(data), "params": n_params, "bytes_per_step": nbytes}
    return results


def run_dequant(args):
    """INT8 -> fp16 dequant of every Llama-2-7B linear/embedding tensor; one
    step = the whole checkpoint. Metric: algorithmic GB/s (1 B read + 2 B
    written per value)."""
    import torch

    from littlellm_b200 import build as kbuild
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA GPU")
    world, rank, local = dist_env()
    if world > 1:
        raise SystemExit("the dequant workload runs on one GPU")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    kbuild.build()
    peaks = load_peaks()
    results = measure_dequant(device, args.steps, args.warmup, peaks)
    data, scales = results.pop("_tensors")
    meta = results.pop("_meta")
    import numpy as np
    cpu = None
    if not args.no_cpu_baseline:
        from oracle.oracle import Oracle, Reference, reference_available
        o = Oracle()
        q = np.ascontiguousarray(data[0].flatten()[: 1 << 26].cpu().numpy())
        sample = q.size
        out16 = np.empty(sample, np.uint16)
        fn = (Reference().lib.kref_dequantize_int8_f16 if reference_available()
              else o.lib.kllm_oracle_dequantize_int8_f16)
        import ctypes
        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < args.cpu_seconds / 2 or reps == 0:
            fn(ctypes.c_void_p(q.ctypes.data), sample, ctypes.c_float(float(scales[0].item())),
               ctypes.c_void_p(out16.ctypes.data))
            reps += 1
        dt = time.perf_counter() - t0
        cpu = {"value": 3 * sample * reps / dt / 1e9, "unit": "GB/s", "cores": 1,
               "kind": "reference" if reference_available() else "port",
               "sample": f"{sample} values x {reps} through the weight loader's loop body "
                         "(float(q) * scale, float_to_half), single thread"}
    del data, scales
    b = results["batched"]
    emit({"metric": "int8->fp16 dequant throughput", "value": b["gbs"], "unit": "GB/s", "n_gpus": 1,
          "steps": args.steps, "warmup": args.warmup, "ms_per_step": b["ms_per_step"], "higher_is_better": True,
          "scaling": "none", "vs_baseline": None, "dtype": "i8->f16", "data": "synthetic",
          "config": {"workload": "llama_int8_dequant", **meta,
                     "l2": "no flush: 20.2 GB per step >> 126 MB L2"},
          "roofline": {"bound": "hbm", "kernel": "dequant_batched_kernel", "achieved": b["gbs"],
                       "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": b["frac_of_measured"],
                       "traffic": None, "peak_source": peaks["source"]},
          "variants": results, "gpu_launches": args.steps,
          "cpu_baseline": cpu})


def per_op_chain_timing(runner, stream, reps: int) -> dict:
    """The per-layer ops timed the way the chain runs them: the chain
    executor launches only one op kind (op_mask) over all layers, with PDL,
    as one CUDA graph replayed `reps` times; us/launch = replay time /
    launches. Layer buffers are distinct, so one replay streams several GB
    (> L2); the add+RMSNorm launches share the running residual as in the
    chain."""
    import torch

    from littlellm_b200 import _capi
    w, m = runner.w, runner.w.model
    T, H, L = w.n_tokens, m.hidden, runner.n_layers
    qkv_bytes = 2 * T * (m.n_heads + 2 * m.n_kv_heads) * m.head_dim * 2 + 8 * T
    kinds = {
        "add_rms_norm": (_capi.OP_INPUT_NORM | _capi.OP_POST_NORM,
                         (2 * T * H * 2 + (L - 1) * 4 * T * H * 2 + L * 4 * T * H * 2) / (2 * L)),
        "qkv_bias_rope_kv_append": (_capi.OP_QKV_ROPE, qkv_bytes),
        "silu_mul": (_capi.OP_SWIGLU, 3 * T * m.intermediate * 2),
    }
    if runner.attention:
        # per layer (a decode layer launches the attention kernel and the split
        # combine); bytes as chain_bytes counts them
        from littlellm_b200.chain import chain_bytes
        att = chain_bytes(w, L, positions=runner.positions.cpu().numpy())["attention"] / L
        kinds["attention"] = (_capi.OP_ATTENTION, att)
    out = {}
    with torch.cuda.stream(stream):
        for name, (mask, nbytes) in kinds.items():
            runner.desc.op_mask = mask
            n = runner.run(stream)
            g = capture(lambda: runner.run(stream), stream)
            g.replay()
            per = L if name == "attention" else n
            ms = time_graph(g, stream, reps) / per
            out[name] = {"us_per_launch": ms * 1000.0, "bytes_per_launch": int(nbytes),
                         "gbs": nbytes / (ms * 1e-3) / 1e9, "launches_per_replay": per}
            if name == "attention":
                out[name]["kernel_launches_per_replay"] = n
                out[name]["note"] = "per layer, not per kernel launch"
            del g
        # ablation: the whole step with this op kind removed; the difference
        # is the op's marginal cost where it really sits in the chain (after
        # the neighbours it has in a forward step, not after itself)
        full = runner.full_mask or _capi.OP_CHAIN  # op_mask 0 means the seven chain ops
        runner.desc.op_mask = full
        n_full = runner.run(stream)
        g = capture(lambda: runner.run(stream), stream)
        g.replay()
        t_full = time_graph(g, stream, reps)
        del g
        for name, (mask, nbytes) in kinds.items():
            if name == "attention":
                continue
            runner.desc.op_mask = full & ~mask
            n_without = runner.run(stream)
            g = capture(lambda: runner.run(stream), stream)
            g.replay()
            t_without = time_graph(g, stream, reps)
            del g
            removed = n_full - n_without
            if removed > 0:
                us = (t_full - t_without) * 1000.0 / removed
                out[name]["marginal_us_per_launch"] = us
                out[name]["marginal_gbs"] = nbytes / (us * 1e-6) / 1e9 if us > 0 else None
        runner.desc.op_mask = runner.full_mask
    return out


def _write_llama_int8(path: str, layers: int, seed: int = 11) -> list[str]:
    """A Llama-2-7B-shaped .kllm file with INT8 linear/embedding records
    (int8 ~U[-127,127] + fp32 scale ~U(1e-3,1e-2)) and fp16 norm weights;
    returns the tensor names."""
    import struct

    import numpy as np
    rng = np.random.default_rng(seed)
    H, I, V = 4096, 11008, 32000
    recs = [("model.embed_tokens.weight", (V, H), "i8")]
    for i in range(layers):
        p = f"model.layers.{i}."
        recs += [(p + "input_layernorm.weight", (H,), "f16")]
        recs += [(p + f"self_attn.{m}_proj.weight", (H, H), "i8") for m in "qkvo"]
        recs += [(p + "post_attention_layernorm.weight", (H,), "f16"),
                 (p + "mlp.gate_proj.weight", (I, H), "i8"), (p + "mlp.up_proj.weight", (I, H), "i8"),
                 (p + "mlp.down_proj.weight", (H, I), "i8")]
    recs += [("model.norm.weight", (H,), "f16"), ("lm_head.weight", (V, H), "i8")]
    with open(path, "wb") as f:
        f.write(b"KLLM0001" + struct.pack("<II", 1, 0))
        f.write(struct.pack("<8i", V, H, I, layers, 32, 32, 128, 4096))
        f.write(struct.pack("<ffBBBBI", 1e-5, 1e4, 0, 0, 0, 0, len(recs)))
        for name, shape, dt in recs:
            n = int(np.prod(shape))
            enc = name.encode()
            f.write(struct.pack("<I", len(enc)) + enc)
            f.write(struct.pack("<II", 3 if dt == "i8" else 1, len(shape)))
            f.write(b"".join(struct.pack("<q", d) for d in shape))
            if dt == "i8":
                f.write(struct.pack("<Q", n + 4))
                f.write(rng.integers(-127, 128, n, dtype=np.int8).tobytes())
                f.write(np.array([rng.uniform(1e-3, 1e-2)], np.float32).tobytes())
            else:
                f.write(struct.pack("<Q", 2 * n))
                f.write(rng.uniform(0.5, 1.5, n).astype(np.float16).tobytes())
    return [r[0] for r in recs]


def _checksums(t) -> tuple[int, int]:
    import numpy as np
    b = t.contiguous().view(-1).cpu().numpy().view(np.uint8)
    pad = (-b.size) % 8
    if pad:
        b = np.concatenate([b, np.zeros(pad, np.uint8)])
    w = b.view(np.uint64)
    return int(w.sum(dtype=np.uint64)), int(np.bitwise_xor.reduce(w))


def run_load(args):
    """.kllm checkpoint load onto the GPU: a partial Llama-2-7B INT8 file
    (embedding, 4 decoder layers, lm_head: 1.07 B parameters) loaded by the
    streaming loader (device-side dequant) and by the reference's own
    ModelWeights::load (host dequant). Metric: file GB/s, wall clock (both
    loads end synchronised, the file is in the page cache for both)."""
    import subprocess
    import tempfile

    import torch

    from littlellm_b200 import build as kbuild
    from littlellm_b200 import loader
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA GPU")
    device = torch.device("cuda", dist_env()[2])
    torch.cuda.set_device(device)
    kbuild.build()
    layers = args.layers or 4
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "llama_int8.kllm")
        names = _write_llama_int8(path, layers)
        file_bytes = os.path.getsize(path)
        log(f"load: wrote {file_bytes / 1e9:.2f} GB")
        idx = loader.read_index(path)
        times = []
        for _ in range(max(args.steps, 1)):
            t0 = time.perf_counter()
            _, tensors = loader.load(path, device, index=idx)
            torch.cuda.synchronize(device)
            times.append(time.perf_counter() - t0)
            if len(times) < max(args.steps, 1):
                del tensors
        ours = min(times)
        ref = None
        exe = os.path.join(ROOT, "oracle", "_ref", "refcuda", "ref_load")
        match = None
        if os.path.exists(exe):
            names_path = os.path.join(tmp, "names.txt")
            with open(names_path, "w") as f:
                f.write("\n".join(names) + "\n")
            r = subprocess.run([exe, path, names_path], capture_output=True, text=True, timeout=1200)
            if r.returncode == 0:
                lines = r.stdout.splitlines()
                ref = float(lines[0].split()[1])
                want = {ln.split()[0]: (int(ln.split()[1]), int(ln.split()[2])) for ln in lines[1:]}
                match = all(_checksums(tensors[n]) == want[n] for n in names)
            else:
                log(f"reference loader failed: {r.stderr.strip()[-300:]}")
    emit({"metric": "int8 .kllm checkpoint load", "value": file_bytes / ours / 1e9, "unit": "GB/s",
          "n_gpus": 1, "steps": len(times), "warmup": 0, "ms_per_step": ours * 1e3, "higher_is_better": True,
          "scaling": "none", "vs_baseline": None, "dtype": "i8->f16", "data": "synthetic",
          "config": {"workload": "llama_int8_load", "layers": layers, "file_bytes": file_bytes,
                     "tensors": len(names), "staging": "2 x 32 MB pinned host, 2 x 32 MB device"},
          "reference_loader_seconds": ref, "speedup_vs_reference_loader": (ref / ours) if ref else None,
          "bit_exact_vs_reference_loader": match, "all_load_seconds": times})


# ---------------------------------------------------------------------------
# attention over the head-major cache (scope row f1)
# ---------------------------------------------------------------------------

ATTENTION_WORKLOADS = {
    # 2048 sequences x 1 token at positions U[0, 4095) over the Qwen2.5-0.5B cache [24, 2, 2048, 2, 4096, 64]
    "qwen_decode_attention": "qwen_decode",
    # 8 x 512-token Qwen2.5-0.5B prefill, cache [24, 2, 8, 2, 4096, 64]
    "qwen_prefill_attention": "qwen_prefill",
    # 32 x 512-token Llama-2-7B prefill, cache [32, 2, 32, 32, 512, 128]
    "llama_prefill_attention": "llama_prefill",
}
ATTN_METRIC = "attention tokens/s"


def attention_work(w, positions, n_layers: int) -> dict:
    """Algorithmic bytes and FLOPs of one step (attention in every layer).
    Bytes: each sequence's cached K and V rows 0..position read once (decode:
    once per token; prefill: once per sequence), q read and out written, in
    fp16. FLOPs: 4 * D per (token, query head, attended position)."""
    import numpy as np
    m = w.model
    pos = np.asarray(positions, dtype=np.int64)
    if w.decode:
        kv_rows = int((pos + 1).sum())
    else:
        kv_rows = w.n_seqs * w.seq_len
    per_layer_bytes = kv_rows * m.n_kv_heads * m.head_dim * 2 * 2 + w.n_tokens * m.n_heads * m.head_dim * 2 * 2
    per_layer_flops = int((pos + 1).sum()) * m.n_heads * m.head_dim * 4
    return {"bytes": per_layer_bytes * n_layers, "flops": per_layer_flops * n_layers}


def time_reference_attention(w, n_layers: int, threads: int, seconds: float, steps: int | None = None,
                             warmup: int = 0):
    """The reference's kllm::op::attention (CPU, fp32 tensors, cache
    [max_seq, Hkv, D] per sequence) on `threads` threads, each running one
    sequence's tokens of this workload (decode: one token at position
    max_seq / 2; prefill: a seq_len-token prefill) through every layer.
    Returns (tokens/s, per-step seconds, kind)."""
    from concurrent.futures import ThreadPoolExecutor

    import numpy as np

    from oracle.oracle import Reference, reference_available
    if not reference_available():
        raise RuntimeError("compiled reference (oracle/_ref) not available")
    ref = Reference()
    m = w.model
    tokens = 1 if w.decode else w.seq_len
    past = w.max_seq // 2 if w.decode else 0
    rng = np.random.default_rng(0)
    kc = rng.standard_normal((past + tokens, m.n_kv_heads, m.head_dim)).astype(np.float32)
    vc = rng.standard_normal((past + tokens, m.n_kv_heads, m.head_dim)).astype(np.float32)
    qs = [rng.standard_normal((tokens, m.n_heads, m.head_dim)).astype(np.float32) for _ in range(threads)]

    def one(i):
        for _ in range(n_layers):
            ref.attention(qs[i], kc, vc, past, m.n_kv_heads)

    step_times = []
    with ThreadPoolExecutor(threads) as ex:
        for _ in range(warmup):
            list(ex.map(one, range(threads)))
        t_start = time.perf_counter()
        while True:
            t0 = time.perf_counter()
            list(ex.map(one, range(threads)))
            step_times.append(time.perf_counter() - t0)
            if steps is not None and len(step_times) >= steps:
                break
            if steps is None and time.perf_counter() - t_start >= seconds:
                break
    return threads * tokens * len(step_times) / sum(step_times), step_times, "reference"


def run_attention(args):
    """One step = attention over the head-major cache in every layer for the
    workload's tokens (one launch per layer, plus the split combine), replayed
    as one CUDA graph; the cache stays resident, q differs per layer."""
    import torch

    from littlellm_b200 import build as kbuild
    from littlellm_b200 import ops
    from littlellm_b200.chain import WORKLOADS, shard

    world, rank, local = dist_env()
    if world == 1 and args.gpus > 1:
        raise SystemExit("--gpus N > 1 must be launched with torchrun (one rank per GPU)")
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA GPU")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    kbuild.build()
    from littlellm_b200 import dist as kd
    dist = None
    if world > 1:
        import torch.distributed as dist
        kd.init("nccl", device, timeout_s=300)

    base = WORKLOADS[ATTENTION_WORKLOADS[args.workload]]
    if args.sequences:
        base = replace(base, n_seqs=args.sequences)
    weak = base.name == "qwen_prefill"
    w = base if weak else shard(base, rank, world)
    m = w.model
    L = args.layers or m.n_layers
    T, B, S = w.n_tokens, w.n_seqs, w.max_seq
    gen = torch.Generator(device=device)
    gen.manual_seed(3000 + rank)
    cache = torch.empty((L, 2, B, m.n_kv_heads, S, m.head_dim), dtype=torch.float16, device=device)
    cache.normal_(generator=gen)
    q = torch.empty((L, T, m.n_heads, m.head_dim), dtype=torch.float16, device=device).normal_(generator=gen)
    out = torch.empty_like(q)
    if w.decode:
        positions = torch.randint(0, S - 1, (T,), generator=gen, device=device, dtype=torch.int32)
        slots = torch.arange(T, device=device, dtype=torch.int32)
    else:
        t = torch.arange(T, device=device, dtype=torch.int32)
        positions, slots = t % w.seq_len, t // w.seq_len
    ws_bytes = ops.attention_workspace_bytes(T, m.n_heads, m.n_kv_heads, m.head_dim, S)
    ws = torch.zeros(max(ws_bytes, 16), dtype=torch.uint8, device=device)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    work = attention_work(w, positions.cpu().numpy(), L)
    log(f"attention: {args.workload}, {L} layers, cache {cache.numel() * 2 / 1e9:.1f} GB, "
        f"workspace {ws_bytes / 1e6:.1f} MB, {work['bytes'] / 1e9:.2f} GB / {work['flops'] / 1e12:.3f} TFLOP per step")

    def step():
        for layer in range(L):
            ops.attention_head_major(q[layer], cache[layer, 0], cache[layer, 1], positions, slots,
                                     seq_len=w.seq_len, out=out[layer], workspace=ws, err_flags=err)

    launches = L * (2 if ws_bytes > 0 else 1)  # decode + split combine per layer
    stream = torch.cuda.Stream(device)
    torch.cuda.synchronize(device)
    with torch.cuda.stream(stream):
        step()
        stream.synchronize()
        graph = capture(step, stream)
        for _ in range(max(args.warmup, 3)):
            graph.replay()
        stream.synchronize()
        sampler = ClockSampler(device)
        sampler.start()
        t_end = time.perf_counter() + args.settle_seconds
        while time.perf_counter() < t_end:
            graph.replay()
            stream.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        end.record(stream)
        end.synchronize()
        torch.cuda.synchronize(device)
    if dist is not None:
        dist.barrier()
    tt = torch.tensor([start.elapsed_time(end)], dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    max_ms = float(tt.item())
    clocks = sampler.stop()
    flags = kd.or_over_ranks(int(err.item()), device)
    finite = bool(torch.isfinite(out).all().item())

    ms = max_ms / args.steps
    value = T * world / (ms * 1e-3)
    peaks = load_peaks()
    gbs = work["bytes"] / (ms * 1e-3) / 1e9
    tflops = work["flops"] / (ms * 1e-3) / 1e12
    if w.decode:
        roofline = {"bound": "hbm", "kernel": "attn_decode_kernel", "achieved": gbs, "peak": peaks["hbm_gbs"],
                    "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"], "traffic": None, "peak_source": peaks["source"],
                    "timing": f"{L} layers per CUDA graph replay (decode + split combine per layer), CUDA events"}
    else:
        tc_peak = load_tc_peak()
        kernel = "attn_prefill_tc_kernel (tcgen05)" if m.head_dim == 128 else "attn_prefill_kernel (mma.sync)"
        roofline = {"bound": "tensor", "kernel": kernel, "achieved": tflops, "peak": tc_peak["tflops"],
                    "unit": "TFLOP/s", "frac": tflops / tc_peak["tflops"], "traffic": None,
                    "peak_source": tc_peak["source"],
                    "timing": f"{L} layers per CUDA graph replay, CUDA events"}

    e2e = None
    if not args.no_e2e:
        qh = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
        qh.copy_(q.cpu())
        ph = torch.empty(positions.shape, dtype=torch.int32, pin_memory=True)
        ph.copy_(positions.cpu())
        sh = torch.empty(slots.shape, dtype=torch.int32, pin_memory=True)
        sh.copy_(slots.cpu())
        oh = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)

        def e2e_step():
            q.copy_(qh, non_blocking=True)
            positions.copy_(ph, non_blocking=True)
            slots.copy_(sh, non_blocking=True)
            step()
            oh.copy_(out, non_blocking=True)

        with torch.cuda.stream(stream):
            for _ in range(2):
                e2e_step()
            stream.synchronize()
            if dist is not None:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                e2e_step()
            e1.record(stream)
            e1.synchronize()
        et = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
        if dist is not None:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e_ms = float(et.item()) / args.steps
        e2e = {"value": T * world / (e_ms * 1e-3), "unit": "tokens/s",
               "h2d_bytes_per_step": q.numel() * 2 + positions.numel() * 4 + slots.numel() * 4,
               "d2h_bytes_per_step": out.numel() * 2, "ms_per_step": e_ms,
               "path": "ops.attention_head_major (C ABI) per layer, eager launches; q, positions and slots "
                       "copied from pinned host memory and every layer's output copied back each step"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            v, st, kind = time_reference_attention(w, L, 1, args.cpu_seconds)
            cpu = {"value": v, "unit": "tokens/s", "cores": 1, "kind": kind,
                   "sample": f"{'one token at position %d' % (S // 2) if w.decode else 'one %d-token prefill' % w.seq_len}"
                             f" through the attention of all {L} layers, repeated {len(st)}x ({sum(st):.1f} s), "
                             "fp32, single thread"}
        except RuntimeError as e:
            log(f"cpu baseline skipped: {e}")

    del graph
    if rank == 0:
        emit({
            "metric": ATTN_METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak" if weak else "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": args.workload, "shapes": m.name, "layers": L, "tokens_per_gpu": T,
                       "sequences_per_gpu": B, "seq_len": w.seq_len,
                       "kv_cache": [L, 2, B, m.n_kv_heads, S, m.head_dim],
                       "positions": "U[0, %d)" % (S - 1) if w.decode else "0..%d per sequence" % (w.seq_len - 1),
                       "parallelism": f"dp{world} (sequences split, no collective on the path)",
                       "math": "fp16 operands, fp32 accumulate, fp32 online softmax",
                       "l2": "no flush: each step reads %.2f GB of distinct per-layer K/V (>> 126 MB L2)"
                             % (work["bytes"] / 1e9) if w.decode else
                             "per-sequence K/V is L2-resident within a layer; layers use distinct caches",
                       "workspace_bytes": ws_bytes, "cuda_graph": True},
            "hbm_gbs": gbs, "tflops": tflops, "bytes_per_step": work["bytes"], "flops_per_step": work["flops"],
            "roofline": roofline, "clocks": clocks, "gpu_launches": launches * args.steps,
            "launches_per_step": launches, "e2e": e2e, "cpu_baseline": cpu,
            "verification": {"ranks": world, "finite": finite, "err_flags": flags},
        })
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_reference_attention(args):
    from littlellm_b200.workloads import WORKLOADS
    w = WORKLOADS[ATTENTION_WORKLOADS[args.workload]]
    L = args.layers or w.model.n_layers
    threads = host_threads()
    value, st, kind = time_reference_attention(w, L, threads, 0.0, steps=args.steps, warmup=args.warmup)
    tokens = 1 if w.decode else w.seq_len
    emit({"metric": ATTN_METRIC, "value": value, "unit": "tokens/s", "impl": "reference", "n_gpus": args.gpus,
          "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * statistics.mean(st),
          "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
          "config": {"workload": args.workload, "shapes": w.model.name, "layers": L,
                     "tokens_per_step": threads * tokens,
                     "impl_detail": "reference kllm::op::attention on CPU tensors (src/op/cpu/attention.cpp)"},
          "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": kind,
                           "sample": f"{threads} threads x {tokens} token(s) each through {L} layers per step"},
          "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})


def load_tc_peak(sustained: bool = False) -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        if sustained and "bf16_tflops_sustained" in p:
            return {"tflops": float(p["bf16_tflops_sustained"]), "source": "measured (cuBLAS bf16 sustained)"}
        return {"tflops": float(p["bf16_tflops"]), "source": "measured (cuBLAS bf16 burst)"}
    return {"tflops": 1400.0 if sustained else 1590.0, "source": "fallback"}


# ---------------------------------------------------------------------------
# scope row f4: the MLP's gate/up GEMM with the SwiGLU epilogue fused
# ---------------------------------------------------------------------------

GEMM_WORKLOADS = {
    # Qwen2.5-0.5B, 8 x 512 tokens: x [4096, 896] @ [w_gate; w_up] [2 x 4864, 896]^T -> silu_mul, 24 layers
    "qwen_mlp_gemm": "qwen_prefill",
    # Llama-2-7B, 32 x 512 tokens: x [16384, 4096] @ [2 x 11008, 4096]^T -> silu_mul, 32 layers
    "llama_mlp_gemm": "llama_prefill",
}
GEMM_METRIC = "MLP gate/up+SwiGLU tokens/s"


def time_reference_mlp(m, n_layers: int, threads: int, seconds: float, rows: int, steps: int | None = None,
                       warmup: int = 0):
    """The reference's linear() + silu_mul on the CPU (kllm::op::matmul, CPU
    F32 tensors; no MLP bias in either model) for `rows` token rows per
    thread through every layer, one layer's weights reused for all layers (at
    these sizes the weights stream from DRAM either way). Returns (tokens/s,
    per-step seconds, kind)."""
    from concurrent.futures import ThreadPoolExecutor

    import numpy as np

    from oracle.oracle import Reference, reference_available
    if not reference_available():
        raise RuntimeError("compiled reference (oracle/_ref) not available")
    ref = Reference()
    rng = np.random.default_rng(0)
    wg = (rng.standard_normal((m.intermediate, m.hidden)) / np.sqrt(m.hidden)).astype(np.float32)
    wu = (rng.standard_normal((m.intermediate, m.hidden)) / np.sqrt(m.hidden)).astype(np.float32)
    xs = [rng.standard_normal((rows, m.hidden)).astype(np.float32) for _ in range(threads)]

    def one(i):
        for _ in range(n_layers):
            ref.silu_mul(ref.matmul(xs[i], wg), ref.matmul(xs[i], wu))

    step_times = []
    with ThreadPoolExecutor(threads) as ex:
        for _ in range(warmup):
            list(ex.map(one, range(threads)))
        t_start = time.perf_counter()
        while True:
            t0 = time.perf_counter()
            list(ex.map(one, range(threads)))
            step_times.append(time.perf_counter() - t0)
            if steps is not None and len(step_times) >= steps:
                break
            if steps is None and time.perf_counter() - t_start >= seconds:
                break
    return threads * rows * len(step_times) / sum(step_times), step_times, "reference"


def run_gemm(args):
    """One step = kllm_b200_linear_swiglu of every layer (x [T, H] of the layer
    times its own w_gate and w_up [I, H], SwiGLU in the epilogue), replayed as
    one CUDA graph; every layer has distinct x, weights and output (several
    GB, far beyond L2). The same step with cuBLAS (torch.matmul over the
    stacked [w_gate; w_up]) plus this library's silu_mul is timed beside it
    as the unfused baseline."""
    import torch

    from littlellm_b200 import build as kbuild
    from littlellm_b200 import ops
    from littlellm_b200.chain import WORKLOADS, shard

    world, rank, local = dist_env()
    if world == 1 and args.gpus > 1:
        raise SystemExit("--gpus N > 1 must be launched with torchrun (one rank per GPU)")
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA GPU")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    kbuild.build()
    from littlellm_b200 import dist as kd
    dist = None
    if world > 1:
        import torch.distributed as dist
        kd.init("nccl", device, timeout_s=300)

    base = WORKLOADS[GEMM_WORKLOADS[args.workload]]
    if args.sequences:
        base = replace(base, n_seqs=args.sequences)
    weak = base.name == "qwen_prefill"
    w = base if weak else shard(base, rank, world)
    m = w.model
    L = args.layers or m.n_layers
    T, H, I = w.n_tokens, m.hidden, m.intermediate
    gen = torch.Generator(device=device)
    gen.manual_seed(5000 + rank)
    x = torch.empty((L, T, H), dtype=torch.float16, device=device).normal_(generator=gen)
    # [w_gate; w_up] stacked per layer: the fused kernel reads the two halves,
    # cuBLAS the whole
    wgu = torch.empty((L, 2 * I, H), dtype=torch.float16, device=device).normal_(std=H ** -0.5, generator=gen)
    out = torch.empty((L, T, I), dtype=torch.float16, device=device)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    flops_per_layer = 2 * T * H * 2 * I
    flops = flops_per_layer * L
    log(f"gemm: {args.workload}, {L} layers, x {x.numel() * 2 / 1e9:.2f} GB, weights {wgu.numel() * 2 / 1e9:.2f} GB,"
        f" out {out.numel() * 2 / 1e9:.2f} GB, {flops / 1e12:.2f} TFLOP per step")

    def step():
        for layer in range(L):
            ops.linear_swiglu(x[layer], wgu[layer, :I], wgu[layer, I:], out=out[layer], err_flags=err)

    gu = torch.empty((T, 2 * I), dtype=torch.float16, device=device)
    g_buf = torch.empty((T, I), dtype=torch.float16, device=device)
    u_buf = torch.empty((T, I), dtype=torch.float16, device=device)

    def step_unfused():
        # the reference's structure: linear(gate), linear(up), silu_mul
        for layer in range(L):
            torch.matmul(x[layer], wgu[layer, :I].T, out=g_buf)
            torch.matmul(x[layer], wgu[layer, I:].T, out=u_buf)
            ops.silu_mul(g_buf, u_buf, out=out[layer])

    def step_gemm_only():
        for layer in range(L):
            torch.matmul(x[layer], wgu[layer].T, out=gu)

    stream = torch.cuda.Stream(device)
    torch.cuda.synchronize(device)

    def timed(graph, reps):
        for _ in range(max(args.warmup, 3)):
            graph.replay()
        stream.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(reps):
            graph.replay()
        e.record(stream)
        e.synchronize()
        return s.elapsed_time(e) / reps

    with torch.cuda.stream(stream):
        step()
        stream.synchronize()
        graph = capture(step, stream)
        for _ in range(max(args.warmup, 3)):
            graph.replay()
        stream.synchronize()
        sampler = ClockSampler(device)
        sampler.start()
        t_end = time.perf_counter() + args.settle_seconds
        while time.perf_counter() < t_end:
            graph.replay()
            stream.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        end.record(stream)
        end.synchronize()
        torch.cuda.synchronize(device)
    if dist is not None:
        dist.barrier()
    tt = torch.tensor([start.elapsed_time(end)], dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    max_ms = float(tt.item())
    clocks = sampler.stop()
    flags = kd.or_over_ranks(int(err.item()), device)
    finite = bool(torch.isfinite(out[-1]).all().item())
    # spot check against a torch fp32 reference on a few rows of the last layer
    rows = torch.arange(0, T, max(1, T // 16), device=device)
    xs = x[-1, rows].float()
    gref = xs @ wgu[-1, :I].float().T
    uref = xs @ wgu[-1, I:].float().T
    yref = gref * torch.sigmoid(gref) * uref
    spot_ok = bool(((out[-1, rows].float() - yref).abs() <= 1e-2 + 1e-2 * yref.abs()).all().item())

    comparison = None
    if rank == 0:
        with torch.cuda.stream(stream):
            g_unf = capture(step_unfused, stream)
            unf_ms = timed(g_unf, args.steps)
            g_cb = capture(step_gemm_only, stream)
            cb_ms = timed(g_cb, args.steps)
        del g_unf, g_cb
        comparison = {"unfused_ms_per_step": unf_ms, "cublas_gemm_only_ms_per_step": cb_ms,
                      "fused_speedup_vs_unfused": unf_ms / (max_ms / args.steps),
                      "unfused": "per layer torch.matmul (cuBLAS, fp16, fp32 accumulate) for gate and for up, "
                                 "then kllm_b200_silu_mul; CUDA graph",
                      "cublas_gemm_only": "one torch.matmul per layer over the stacked [w_gate; w_up] (N = 2I), "
                                          "no SwiGLU: the GEMM work alone"}

    ms = max_ms / args.steps
    value = T * world / (ms * 1e-3)
    tflops = flops / (ms * 1e-3) / 1e12
    # the clocks are settled under this load before timing (power-capped steady
    # state), so the sustained GEMM peak is the denominator; burst beside it
    tc = load_tc_peak(sustained=True)
    burst = load_tc_peak(sustained=False)
    roofline = {"bound": "tensor", "kernel": "gemm_tc_kernel<SwiGLU> (tcgen05)", "achieved": tflops,
                "peak": tc["tflops"], "unit": "TFLOP/s", "frac": tflops / tc["tflops"],
                "frac_of_burst_peak": tflops / burst["tflops"],
                "traffic": ncu_traffic("gemm_tc_swiglu", args.workload), "peak_source": tc["source"],
                "flops_per_launch": flops_per_layer,
                "timing": f"{L} launches per CUDA graph replay, {args.steps} replays, CUDA events"}

    e2e = None
    if not args.no_e2e:
        xh = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        xh.copy_(x.cpu())
        last = torch.arange(w.seq_len - 1, T, w.seq_len, device=device)
        oh = torch.empty((last.numel(), I), dtype=out.dtype, pin_memory=True)

        def e2e_step():
            x.copy_(xh, non_blocking=True)
            step()
            oh.copy_(out[-1].index_select(0, last), non_blocking=True)

        with torch.cuda.stream(stream):
            for _ in range(2):
                e2e_step()
            stream.synchronize()
            if dist is not None:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                e2e_step()
            e1.record(stream)
            e1.synchronize()
        et = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
        if dist is not None:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e_ms = float(et.item()) / args.steps
        e2e = {"value": T * world / (e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e_ms,
               "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": oh.numel() * 2,
               "path": "every layer's x copied from pinned host memory, kllm_b200_linear_swiglu per layer "
                       "(eager), the last layer's last-token rows copied back"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            sample_rows = 8 if m.hidden <= 1024 else 1
            v, st, kind = time_reference_mlp(m, L, 1, args.cpu_seconds, sample_rows)
            cpu = {"value": v, "unit": "tokens/s", "cores": 1, "kind": kind,
                   "sample": f"{sample_rows} token row(s) through the gate/up linears + silu_mul of all {L} layers "
                             f"(reference CPU matmul, fp32), repeated {len(st)}x ({sum(st):.1f} s), single thread"}
        except RuntimeError as e:
            log(f"cpu baseline skipped: {e}")

    del graph
    if rank == 0:
        emit({
            "metric": GEMM_METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak" if weak else "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": args.workload, "shapes": m.name, "layers": L, "tokens_per_gpu": T,
                       "gemm": [T, 2 * I, H], "parallelism": f"dp{world} (token rows split, no collective)",
                       "math": "fp16 operands, fp32 accumulate (tcgen05 TMEM), fp16 gate/up rounding then SwiGLU "
                               "in fp32, fp16 out",
                       "l2": "no flush: each step reads %.2f GB of distinct per-layer x and weights and writes "
                             "%.2f GB (>> 126 MB L2)" % ((x.numel() + wgu.numel()) * 2 / 1e9, out.numel() * 2 / 1e9),
                       "cuda_graph": True},
            "tflops": tflops, "flops_per_step": flops, "roofline": roofline, "clocks": clocks,
            "gpu_launches": L * args.steps, "launches_per_step": L, "comparison": comparison, "e2e": e2e,
            "cpu_baseline": cpu,
            "verification": {"ranks": world, "finite": finite, "err_flags": flags,
                             "torch_fp32_spot_check": spot_ok},
        })
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_reference_gemm(args):
    from littlellm_b200.workloads import WORKLOADS
    m = WORKLOADS[GEMM_WORKLOADS[args.workload]].model
    L = args.layers or m.n_layers
    threads = host_threads()
    rows = 4 if m.hidden <= 1024 else 1
    value, st, kind = time_reference_mlp(m, L, threads, 0.0, rows, steps=args.steps, warmup=args.warmup)
    emit({"metric": GEMM_METRIC, "value": value, "unit": "tokens/s", "impl": "reference", "n_gpus": args.gpus,
          "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * statistics.mean(st),
          "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
          "config": {"workload": args.workload, "shapes": m.name, "layers": L, "tokens_per_step": threads * rows,
                     "impl_detail": "reference linear() (kllm::op::matmul, CPU) x2 + silu_mul on CPU F32 tensors"},
          "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": kind,
                           "sample": f"{threads} threads x {rows} token row(s) each through {L} layers per step"},
          "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})


def ref_cuda_ops(w, n_layers: int, dequant_shape=None, timeout: float = 900.0) -> dict:
    """The reference's own CUDA operators (its src/op/cuda/*.cu built for
    sm_100a by oracle/Makefile into oracle/_ref/refcuda/ref_cuda_ops), timed
    on this GPU at the workload's shapes in a child process: eager launches
    on the legacy stream as the reference issues them, over distinct buffer
    sets larger than L2, CUDA events. A baseline only, run after our timing.
    Returns {op: {"us": per call group, "launches": kernels per group}}."""
    exe = os.path.join(ROOT, "oracle", "_ref", "refcuda", "ref_cuda_ops")
    if not os.path.exists(exe):
        return {"unavailable": "oracle/_ref/refcuda/ref_cuda_ops was not built (needs the reference sources)"}
    m = w.model
    sets = 8 if m.hidden <= 1024 else 4
    dq = dequant_shape or (0, 0)
    argv = [exe, w.n_tokens, m.hidden, m.n_heads, m.n_kv_heads, m.head_dim, m.intermediate, m.vocab, n_layers,
            sets, 3, m.eps, m.theta, w.n_seqs, dq[0], dq[1]]
    try:
        r = subprocess.run([str(a) for a in argv], capture_output=True, text=True, timeout=timeout)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"ref_cuda_ops timed out after {timeout:.0f} s"}
    if r.returncode != 0:
        return {"unavailable": "ref_cuda_ops failed: " + (r.stderr.strip() or r.stdout.strip())[-300:]}
    out = {}
    for line in r.stdout.splitlines():
        parts = line.split()
        if len(parts) == 3:
            out[parts[0]] = {"us": float(parts[1]), "launches": int(parts[2])}
    out["method"] = (f"reference src/op/cuda ops, eager launches on the legacy stream, {n_layers} calls per pass "
                     f"over {sets} distinct buffer sets, CUDA events; select_last_rows = one call per sequence")
    return out


def merge_ref_cuda(ops_table: dict, ref: dict, field: str = "ref_cuda_us") -> None:
    """Adds the reference CUDA time of each op and our speed-up over it. The
    fused embedding + input norm compares with the reference's embedding
    followed by its plain rms_norm."""
    ref = dict(ref)
    if "embedding" in ref and "rms_norm" in ref:
        ref["embedding_input_norm"] = {"us": ref["embedding"]["us"] + ref["rms_norm"]["us"],
                                       "launches": ref["embedding"]["launches"] + ref["rms_norm"]["launches"]}
    for name, v in ops_table.items():
        r = ref.get(name)
        if isinstance(r, dict) and "us" in r and v.get("us_per_launch"):
            v[field] = r["us"]
            v["ref_cuda_launches"] = r["launches"]
            v["speedup_vs_ref_cuda"] = r["us"] / v["us_per_launch"]


def embedding_chain_timing(runner, stream, reps: int) -> dict:
    """Embedding + layer 0's input RMSNorm as the chain executor launches them
    (op mask EMBEDDING | INPUT_NORM over one layer, PDL), one chain call per
    layer's buffers captured into one graph: distinct ids, residual and
    normed-output buffers per call, so no call re-reads another's rows from
    L2. Algorithmic bytes per call: the table rows read once, the residual and
    the normed rows written once, the ids read (3*T*H*2 + 4*T)."""
    import torch

    from littlellm_b200 import _capi
    w, m = runner.w, runner.w.model
    T, H = w.n_tokens, m.hidden
    L = runner.layers
    gen = torch.Generator(device=runner.device)
    gen.manual_seed(7)
    ids = [torch.randint(0, m.vocab, (T,), generator=gen, device=runner.device, dtype=torch.int32) for _ in L]
    d = runner.desc
    # integer fields and addresses (a pointer field read from a ctypes
    # structure is a view of the structure, not a copy)
    saved = (d.op_mask, d.n_layers, d.ids, d.residual)
    arrs = []
    for i, layer in enumerate(L):
        a = (_capi.LayerBuffers * 1)()
        a[0] = runner._layer_arr[i]
        arrs.append(a)

    def calls():
        n = 0
        for i, layer in enumerate(L):
            d.op_mask = _capi.OP_EMBEDDING | _capi.OP_INPUT_NORM
            d.n_layers = 1
            d.ids = ids[i].data_ptr()
            d.residual = layer["ffn_norm_out"].data_ptr()  # a T x H buffer of this layer's own
            d.layers = ctypes_cast_layers(arrs[i])
            n += runner.run(stream)
        return n

    try:
        with torch.cuda.stream(stream):
            n = calls()
            g = capture(calls, stream)
            g.replay()
            ms = time_graph(g, stream, reps) / len(L)
            del g
    finally:
        d.op_mask, d.n_layers, d.ids, d.residual = saved
        d.layers = ctypes_cast_layers(runner._layer_arr)
    nbytes = 3 * T * H * 2 + 4 * T
    return {"us_per_launch": ms * 1000.0, "bytes_per_launch": nbytes, "gbs": nbytes / (ms * 1e-3) / 1e9,
            "launches_per_replay": n, "kernels_per_call": n // len(L),
            "note": "each call's launch is a chain's first: it reads its ids and table rows only after "
                    "its dependency wait (the launch before a chain may have written them)"}


def ctypes_cast_layers(arr):
    import ctypes

    from littlellm_b200 import _capi
    return ctypes.cast(arr, ctypes.POINTER(_capi.LayerBuffers))


def measure_chain(w, args, device, dist, *, seed: int, steps: int, warmup: int, attention: bool = False,
                  per_op: bool = True, standalone: bool = True):
    """One chain step of workload `w` (this rank's share) as a CUDA graph:
    capture, `warmup` replays, clock settling, then `steps` replays between a
    barrier and device syncs on both sides, CUDA events on the launch stream,
    the time as the max over ranks. Returns (runner, stream, stats)."""
    import torch

    from littlellm_b200.chain import ChainRunner, chain_bytes
    runner = ChainRunner(w, device=device, seed=seed, use_pdl=not args.no_pdl, n_layers=args.layers,
                         attention=attention)
    stream = torch.cuda.Stream(device)
    torch.cuda.synchronize(device)
    with torch.cuda.stream(stream):
        launches = runner.run(stream)
        stream.synchronize()
        graph = capture(lambda: runner.run(stream), stream)
        for _ in range(max(warmup, 3)):
            graph.replay()
        stream.synchronize()
        sampler = ClockSampler(device)
        sampler.start()
        t_end = time.perf_counter() + args.settle_seconds
        while time.perf_counter() < t_end:
            for _ in range(20):
                graph.replay()
            stream.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(steps):
            graph.replay()
        end.record(stream)
        end.synchronize()
        torch.cuda.synchronize(device)
    if dist is not None:
        dist.barrier()
    t = torch.tensor([start.elapsed_time(end)], dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    clocks = sampler.stop()
    del graph
    ms = float(t.item()) / steps
    peaks = load_peaks()
    bytes_step = chain_bytes(w, runner.n_layers, positions=runner.positions.cpu().numpy() if attention else None,
                             fused_embedding=runner.fused_embedding, fused_select=runner.fused_select)
    gbs = bytes_step["total"] / (ms * 1e-3) / 1e9
    stats = {"ms_per_step": ms, "launches_per_step": launches, "clocks": clocks,
             "chain_bytes_per_step": bytes_step["total"], "hbm_gbs_chain": gbs,
             "hbm_frac_chain": gbs / peaks["hbm_gbs"], "peak_gbs": peaks["hbm_gbs"],
             "peak_source": peaks["source"]}
    if per_op:
        op_chain = per_op_chain_timing(runner, stream, max(steps, 5))
        op_chain["embedding_input_norm"] = embedding_chain_timing(runner, stream, max(steps, 5))
        tables = [op_chain]
        stats["ops"] = op_chain
        if standalone:
            op_alone = per_op_timing(runner, stream, max(steps, 5))
            op_alone_pdl = per_op_timing(runner, stream, max(steps, 5), pdl=True)
            tables += [op_alone, op_alone_pdl]
            stats["ops_standalone"] = op_alone
            stats["ops_standalone_pdl"] = op_alone_pdl
        for table in tables:
            for v in table.values():
                v["frac_of_measured"] = v["gbs"] / peaks["hbm_gbs"]
                if v.get("marginal_gbs"):
                    v["marginal_frac_of_measured"] = v["marginal_gbs"] / peaks["hbm_gbs"]
    return runner, stream, stats


def release_device_memory() -> None:
    """Returns the memory of tensors no longer referenced to the device (call
    after dropping the last reference to a runner)."""
    import gc

    import torch
    gc.collect()
    torch.cuda.empty_cache()


OTHER_CONFIGS_N1 = ("llama_prefill", "qwen_decode")


def run_ours(args):
    import torch

    from littlellm_b200 import build as kbuild
    from littlellm_b200.chain import WORKLOADS, shard

    world, rank, local = dist_env()
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            raise SystemExit("--gpus N > 1 must be launched with torchrun (one rank per GPU)")
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA GPU")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    kbuild.build()

    from littlellm_b200 import dist as kd
    dist = None
    if world > 1:
        import torch.distributed as dist
        kd.init("nccl", device, timeout_s=300)

    base = WORKLOADS[args.workload]
    weak = args.workload == "qwen_prefill"
    w = base if weak else shard(base, rank, world)
    single = world == 1
    runner, stream, st = measure_chain(w, args, device, dist, seed=1000 + rank, steps=args.steps,
                                       warmup=args.warmup, attention=args.attention, standalone=single)
    peaks = load_peaks()
    ms_per_step = st["ms_per_step"]
    value = w.n_tokens * world / (ms_per_step * 1e-3)
    op_chain = st["ops"]

    # verification: every rank's last rows gathered to rank 0 (NCCL all_gather,
    # off the timed path) and the device error flags OR-ed over ranks
    flags = kd.or_over_ranks(int(runner.err_flags.item()), device)
    last = kd.gather_rows(runner.last_rows)
    verification = None
    if rank == 0:
        verification = {"ranks": world, "rows_gathered": int(last.shape[0]),
                        "finite": bool(torch.isfinite(last).all().item()), "err_flags": flags}

    silu = op_chain["silu_mul"]
    roofline = {
        "bound": "hbm", "kernel": "silu_mul_f16_kernel", "achieved": silu["gbs"], "peak": peaks["hbm_gbs"],
        "unit": "GB/s", "frac": silu["gbs"] / peaks["hbm_gbs"],
        "traffic": ncu_traffic("silu_mul", w.name), "peak_source": peaks["source"],
        "bytes_per_launch": silu["bytes_per_launch"], "us_per_launch": silu["us_per_launch"],
        "timing": f"{runner.n_layers} PDL launches per CUDA graph (chain executor, op mask), CUDA events on the "
                  "launch stream",
    }
    if args.attention and w.decode:  # the attention dominates a decode step: HBM-bound K/V reads
        att = op_chain["attention"]
        roofline = {
            "bound": "hbm", "kernel": "attn_decode_kernel + attn_combine_kernel", "achieved": att["gbs"],
            "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": att["gbs"] / peaks["hbm_gbs"], "traffic": None,
            "peak_source": peaks["source"], "bytes_per_layer": att["bytes_per_launch"],
            "us_per_layer": att["us_per_launch"],
            "timing": f"attention of {runner.n_layers} layers per CUDA graph (chain executor, op mask, PDL)"}

    # end to end through the C ABI with host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(runner, stream, args.steps, device, dist, world)

    cpu = None
    if rank == 0 and single and not args.no_cpu_baseline and not args.attention:
        threads = 1
        tokens = 128
        v, steps, kind = time_reference_cpu(w.model, tokens, threads, args.cpu_seconds)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": kind,
               "sample": f"one {tokens}-token sequence through all {w.model.n_layers} layers of the "
                         f"{w.model.name} non-GEMM chain, repeated {len(steps)}x "
                         f"({sum(steps):.1f} s), fp32, single thread (the reference CPU path is single-threaded)"}
    n_layers = runner.n_layers
    launches = st["launches_per_step"]
    fused, fused_sel = runner.fused_embedding, runner.fused_select
    del runner
    release_device_memory()

    # the reference's own CUDA kernels at this workload's shapes (1 GPU only)
    run_extra = args.layers is None and not args.attention and not args.no_other_configs
    if rank == 0 and single and run_extra:
        ref = ref_cuda_ops(w, n_layers)
        merge_ref_cuda(op_chain, ref)
        merge_ref_cuda(st.get("ops_standalone", {}), ref)
        merge_ref_cuda(st.get("ops_standalone_pdl", {}), ref)
        st["ref_cuda"] = ref

    # the survey's other configurations, each its own graph and clock record:
    # 1 GPU: Llama-2-7B prefill (config 3), Qwen decode 2048 x 1 (config 4),
    # the Llama-2-7B INT8 dequant (config 5a); N GPUs: config 3 and config 4
    # split N ways (strong scaling) and, from 4 GPUs, the 64K-token Llama
    # prefill (config 5b)
    other = {}
    if run_extra:
        names = list(OTHER_CONFIGS_N1)
        if world >= 4:
            names.append("llama_prefill_64k")
        for name in names:
            wk = WORKLOADS[name]
            if wk.n_seqs % world != 0:
                continue
            ws = shard(wk, rank, world)
            log(f"other config {name}: {ws.n_seqs} sequences on this rank")
            r2, _, s2 = measure_chain(ws, args, device, dist, seed=2000 + rank, steps=args.steps,
                                      warmup=args.warmup, standalone=single)
            s2["value"] = wk.n_tokens / (s2["ms_per_step"] * 1e-3)
            s2["unit"] = UNIT
            s2["scaling"] = "strong"
            s2["tokens_per_step_all_gpus"] = wk.n_tokens
            s2["sequences_per_gpu"] = ws.n_seqs
            s2["kv_cache"] = [r2.n_layers, 2, ws.n_seqs, ws.model.n_kv_heads, ws.max_seq, ws.model.head_dim]
            s2["err_flags"] = kd.or_over_ranks(int(r2.err_flags.item()), device)
            nl = r2.n_layers
            del r2
            release_device_memory()
            if rank == 0 and single:
                ref = ref_cuda_ops(ws, nl, dequant_shape=(11008, 4096) if name == "llama_prefill" else None)
                merge_ref_cuda(s2["ops"], ref)
                merge_ref_cuda(s2.get("ops_standalone", {}), ref)
                merge_ref_cuda(s2.get("ops_standalone_pdl", {}), ref)
                s2["ref_cuda"] = ref
            other[name] = s2
        if single:
            log("other config llama_int8_dequant")
            sampler = ClockSampler(device)
            sampler.start()
            dq = measure_dequant(device, args.steps, args.warmup, peaks)
            dq.pop("_tensors")
            meta = dq.pop("_meta")
            dq_clocks = sampler.stop()
            torch.cuda.empty_cache()
            b = dq["batched"]
            entry = {"ms_per_step": b["ms_per_step"], "value": b["gbs"], "unit": "GB/s",
                     "hbm_frac_chain": b["frac_of_measured"], "variants": dq, "clocks": dq_clocks, **meta}
            if "llama_prefill" in other and "dequant_f32" in other["llama_prefill"].get("ref_cuda", {}):
                r = other["llama_prefill"]["ref_cuda"]["dequant_f32"]["us"]
                ours = dq["f32_out_4x11008x4096"]["ms_per_step"] * 1000.0 / 4
                entry["f32_vs_ref_cuda"] = {"ref_cuda_us_per_tensor": r, "ours_us_per_tensor": ours,
                                            "speedup": r / ours}
            other["llama_int8_dequant"] = entry

    if rank == 0:
        line = {
            "metric": METRIC + (" (chain with attention)" if args.attention else ""), "value": value, "unit": UNIT,
            "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak" if weak else "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic",
            "config": {
                "workload": w.name, "shapes": w.model.name, "layers": n_layers,
                "tokens_per_gpu": w.n_tokens, "sequences_per_gpu": w.n_seqs, "seq_len": w.seq_len,
                "kv_cache": [n_layers, 2, w.n_seqs, w.model.n_kv_heads, w.max_seq, w.model.head_dim],
                "parallelism": f"dp{world} (sequences split, no collective on the path)",
                "math": "fp16 storage, fp32 arithmetic",
                "l2": "no flush: each step streams %.2f GB of distinct per-layer buffers (>> 126 MB L2)"
                      % (st["chain_bytes_per_step"] / 1e9),
                "pdl": not args.no_pdl, "cuda_graph": True, "attention": bool(args.attention),
                "embedding_fused_with_input_norm": fused,
                "select_fused_with_final_norm": fused_sel,
            },
            "hbm_gbs_chain": st["hbm_gbs_chain"],
            "hbm_frac_chain": st["hbm_frac_chain"],
            "chain_bytes_per_step": st["chain_bytes_per_step"],
            "roofline": roofline,
            "ops": op_chain,
            "ops_standalone": st.get("ops_standalone"),
            "ops_standalone_pdl": st.get("ops_standalone_pdl"),
            "ref_cuda": st.get("ref_cuda"),
            "clocks": st["clocks"],
            "gpu_launches": launches * args.steps,
            "launches_per_step": launches,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "verification": verification,
            "other_configs": other,
        }
        emit(line)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()



FORWARD_METRIC = "forward tokens/s"


def forward_flops(w, n_layers: int, positions) -> dict:
    """Tensor work of one forward step: the GEMMs (q/k/v, o, gate/up, down per
    layer; lm_head on the last rows) and attention (4 * D FLOPs per token,
    query head and attended position)."""
    import numpy as np
    m = w.model
    T, H, I = w.n_tokens, m.hidden, m.intermediate
    qd, kvd = m.n_heads * m.head_dim, m.n_kv_heads * m.head_dim
    per_layer = 2 * T * (H * (qd + 2 * kvd) + qd * H + H * 2 * I + I * H)
    gemm = per_layer * n_layers + 2 * w.n_seqs * H * m.vocab
    attn = int((np.asarray(positions, dtype=np.int64) + 1).sum()) * m.n_heads * m.head_dim * 4 * n_layers
    return {"gemm": gemm, "gemm_per_layer": per_layer, "attention": attn, "total": gemm + attn}


def run_forward(args):
    """One step = the whole forward of a decoder step (KLLM_B200_OP_GEMM: the
    chain with its GEMMs; LlamaRunner::forward, src/model/llama.cpp:78-184)
    for the workload's tokens, one CUDA graph replay. Random weights of the
    model's shapes; the roofline is the GEMM work, timed alone on the same
    buffers (tcgen05, tensor-bound)."""
    import torch

    from littlellm_b200 import build as kbuild
    from littlellm_b200 import ops
    from littlellm_b200.chain import WORKLOADS, ChainRunner, shard

    world, rank, local = dist_env()
    if world == 1 and args.gpus > 1:
        raise SystemExit("--gpus N > 1 must be launched with torchrun (one rank per GPU)")
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA GPU")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    kbuild.build()
    from littlellm_b200 import dist as kd
    dist = None
    if world > 1:
        import torch.distributed as dist
        kd.init("nccl", device, timeout_s=300)

    base = WORKLOADS[args.workload]
    weak = args.workload == "qwen_prefill"
    w = base if weak else shard(base, rank, world)
    r = ChainRunner(w, device=device, seed=1000 + rank, use_pdl=not args.no_pdl, n_layers=args.layers,
                    attention=True, gemm=True)
    m, L = w.model, r.n_layers
    work = forward_flops(w, L, r.positions.cpu().numpy())
    stream = torch.cuda.Stream(device)
    torch.cuda.synchronize(device)

    def timed(graph, reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(reps):
            graph.replay()
        e.record(stream)
        e.synchronize()
        return s.elapsed_time(e) / reps

    with torch.cuda.stream(stream):
        launches = r.run(stream)
        stream.synchronize()
        graph = capture(lambda: r.run(stream), stream)
        for _ in range(max(args.warmup, 3)):
            graph.replay()
        stream.synchronize()
        sampler = ClockSampler(device)
        sampler.start()
        t_end = time.perf_counter() + args.settle_seconds
        while time.perf_counter() < t_end:
            graph.replay()
            stream.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        end.record(stream)
        end.synchronize()
        torch.cuda.synchronize(device)
    if dist is not None:
        dist.barrier()
    tt = torch.tensor([start.elapsed_time(end)], dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    max_ms = float(tt.item())
    clocks = sampler.stop()
    flags = kd.or_over_ranks(int(r.err_flags.item()), device)
    logits_ok = bool(torch.isfinite(r.logits.float()).all().item())

    # the GEMMs of the step alone (same kernels, shapes and buffers), for the roofline
    T, H, I = w.n_tokens, m.hidden, m.intermediate

    def gemms():
        for Lb, W in zip(r.layers, r.weights):
            ops.qkv_linear_rope_kv_append(Lb["attn_norm_out"], W["wq"], W["wk"], W["wv"], Lb["q_bias"],
                                          Lb["k_bias"], Lb["v_bias"], r.positions, r.slots, m.theta,
                                          Lb["k_cache"], Lb["v_cache"], q_out=Lb["q"])
            ops.linear(Lb["attn_ctx"], W["wo"], out=Lb["attn_out"])
            ops.linear_swiglu(Lb["ffn_norm_out"], W["w_gate"], W["w_up"], out=Lb["swiglu_out"])
            ops.linear(Lb["swiglu_out"], W["w_down"], out=Lb["ffn_out"])
        ops.linear(r.last_rows, r.lm_head, out=r.logits)

    with torch.cuda.stream(stream):
        g2 = capture(gemms, stream)
        for _ in range(2):
            g2.replay()
        gemm_ms = timed(g2, max(args.steps, 5))
    del g2

    ms = max_ms / args.steps
    value = T * world / (ms * 1e-3)
    gemm_tflops = work["gemm"] / (gemm_ms * 1e-3) / 1e12
    tc = load_tc_peak(sustained=True)
    roofline = {"bound": "tensor",
                "kernel": "gemm_tc_kernel (q/k/v with RoPE/KV append, o, gate/up+SwiGLU, down, lm_head)",
                "achieved": gemm_tflops, "peak": tc["tflops"], "unit": "TFLOP/s", "frac": gemm_tflops / tc["tflops"],
                "traffic": None, "peak_source": tc["source"], "flops_per_step": work["gemm"],
                "ms_per_step": gemm_ms, "share_of_step": gemm_ms / ms,
                "timing": f"the step's {4 * L + 1} GEMM launches alone in one CUDA graph, CUDA events"}

    e2e = None
    if not args.no_e2e:
        ins = [r.ids, r.positions, r.slots]
        hosts = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in ins]
        for h, t in zip(hosts, ins):
            h.copy_(t.cpu())
        lh = torch.empty(r.logits.shape, dtype=r.logits.dtype, pin_memory=True)

        def e2e_step():
            for h, t in zip(hosts, ins):
                t.copy_(h, non_blocking=True)
            r.run(stream)
            lh.copy_(r.logits, non_blocking=True)

        with torch.cuda.stream(stream):
            for _ in range(2):
                e2e_step()
            stream.synchronize()
            if dist is not None:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                e2e_step()
            e1.record(stream)
            e1.synchronize()
        et = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
        if dist is not None:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e_ms = float(et.item()) / args.steps
        e2e = {"value": T * world / (e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e_ms,
               "h2d_bytes_per_step": sum(t.numel() * 4 for t in ins), "d2h_bytes_per_step": r.logits.numel() * 2,
               "path": "ids, positions, slots from pinned host memory; kllm_b200_chain_run (whole forward, eager "
                       "launches); logits of the last tokens to pinned host memory"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        if m.hidden <= 1024:
            cpu = time_oracle_forward(r, args.cpu_seconds)
        else:  # a 7B model's weights as fp32 numpy (27 GB) and ~1 minute per token on one core
            log("cpu baseline skipped for the forward of a model this size")

    del graph
    if rank == 0:
        emit({
            "metric": FORWARD_METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak" if weak else "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": w.name, "shapes": m.name, "layers": L, "tokens_per_gpu": T,
                       "sequences_per_gpu": w.n_seqs, "seq_len": w.seq_len,
                       "kv_cache": [L, 2, w.n_seqs, m.n_kv_heads, w.max_seq, m.head_dim],
                       "weights": "random, N(0, 1/fan_in), fp16", "parallelism": f"dp{world} (sequences split)",
                       "math": "fp16 storage, fp32 accumulation (tcgen05 GEMMs, attention), fp32 elementwise",
                       "pdl": not args.no_pdl, "cuda_graph": True},
            "tflops_step": work["total"] / (ms * 1e-3) / 1e12, "flops_per_step": work["total"],
            "roofline": roofline, "clocks": clocks, "gpu_launches": launches * args.steps,
            "launches_per_step": launches, "e2e": e2e, "cpu_baseline": cpu,
            "verification": {"ranks": world, "logits_finite": logits_ok, "err_flags": flags},
        })
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


GENERATE_WORKLOADS = {
    # Qwen2.5-0.5B: an 8 x 512 prefill, then decode steps of the 8 sequences (one token each per step)
    "qwen_generate": "qwen_prefill",
}
GENERATE_METRIC = "decode tokens/s"


def run_generate(args):
    """Serving loop: one prefill of the workload's sequences through the whole
    forward step (KLLM_B200_OP_GEMM), then decode steps: every step runs the
    whole forward for one new token per sequence at the next position over
    the caches the earlier steps filled (ChainRunner.decode_runner), one CUDA
    graph replay that also advances the positions. Token ids are seeded random
    (sampling is outside the library). Each decode step streams all the
    weights (lm_head included) and the cache rows attended: the HBM roofline."""
    import torch

    from littlellm_b200 import build as kbuild
    from littlellm_b200.chain import WORKLOADS, ChainRunner

    world, rank, local = dist_env()
    if world > 1:
        raise SystemExit("qwen_generate runs on one GPU (a replica per GPU would be independent)")
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA GPU")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    kbuild.build()
    w = WORKLOADS[GENERATE_WORKLOADS[args.workload]]
    m = w.model
    r = ChainRunner(w, device=device, seed=1000, attention=True, gemm=True, n_layers=args.layers)
    L, B = r.n_layers, w.n_seqs
    stream = torch.cuda.Stream(device)
    total_steps = max(args.warmup, 3) + args.steps + 2
    if w.seq_len + total_steps > w.max_seq:
        raise SystemExit("too many decode steps for the cache")
    gen = torch.Generator(device=device)
    gen.manual_seed(77)
    ids_all = torch.randint(0, m.vocab, (total_steps, B), generator=gen, device=device, dtype=torch.int32)
    step_idx = torch.zeros((), dtype=torch.int64, device=device)
    with torch.cuda.stream(stream):
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        r.run(stream)
        p1.record(stream)
        p1.synchronize()
        prefill_ms = p0.elapsed_time(p1)
        d = r.decode_runner(ids_all[0], torch.full((B,), w.seq_len, dtype=torch.int32, device=device))
        launches = d.run(stream)  # the first decode step (position seq_len)

        def step():
            # next token: ids of this step, one position further
            step_idx.add_(1)
            d.ids.copy_(ids_all.index_select(0, step_idx.view(1)).view(-1))
            d.positions.add_(1)
            d.run(stream)

        stream.synchronize()
        graph = capture(step, stream)
        for _ in range(max(args.warmup, 3)):
            graph.replay()
        stream.synchronize()
        sampler = ClockSampler(device)
        sampler.start()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        end.record(stream)
        end.synchronize()
    clocks = sampler.stop()
    ms = start.elapsed_time(end) / args.steps
    last_pos = int(d.positions[0].item())
    flags = int(d.err_flags.item()) | int(r.err_flags.item())
    finite = bool(torch.isfinite(d.logits.float()).all().item())
    weight_bytes = sum(t.numel() * 2 for W in r.weights for t in W.values()) + r.lm_head.numel() * 2
    mean_pos = last_pos - args.steps / 2.0
    kv_bytes = L * B * (mean_pos + 1) * m.n_kv_heads * m.head_dim * 2 * 2
    bytes_step = weight_bytes + kv_bytes
    gbs = bytes_step / (ms * 1e-3) / 1e9
    peaks = load_peaks()
    roofline = {"bound": "hbm", "kernel": "the decode step (GEMMs streaming the weights, attention)",
                "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"],
                "traffic": None, "peak_source": peaks["source"], "bytes_per_step": int(bytes_step),
                "timing": "one CUDA graph replay per decode step, CUDA events"}
    del graph
    emit({
        "metric": GENERATE_METRIC, "value": B / (ms * 1e-3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": args.workload, "shapes": m.name, "layers": L, "sequences": B,
                   "prompt_tokens": w.seq_len, "decode_positions": [w.seq_len + 1, last_pos],
                   "weights": "random, N(0, 1/fan_in), fp16", "cuda_graph": True, "pdl": True,
                   "ids": "seeded random per step (no sampler)"},
        "prefill_ms": prefill_ms, "prefill_tokens_per_s": w.n_tokens / (prefill_ms * 1e-3),
        "roofline": roofline, "clocks": clocks, "gpu_launches": launches * args.steps,
        "launches_per_step": launches, "e2e": None, "cpu_baseline": None,
        "verification": {"logits_finite": finite, "err_flags": flags},
    })


def time_oracle_forward(r, seconds: float) -> dict:
    """The oracle forward (the reference forward restated on the C oracle's
    operators, single thread, fp32) on a bounded sample: one 8-token sequence
    of the runner's model and weights through every layer and the lm_head."""
    import numpy as np

    from oracle.oracle import Oracle
    o = Oracle()
    m = r.w.model
    tokens = 8

    def npf(t):
        return t.detach().float().cpu().numpy()

    shape = (1, m.n_kv_heads, tokens, m.head_dim)
    layers = []
    for Lb, W in zip(r.layers, r.weights):
        d = {k: npf(Lb[k]) for k in ("input_norm_w", "post_norm_w", "q_bias", "k_bias", "v_bias")}
        d.update({k: npf(t) for k, t in W.items()})
        d["k_cache"], d["v_cache"] = np.zeros(shape, np.float32), np.zeros(shape, np.float32)
        layers.append(d)
    p = {"table": npf(r.table), "ids": npf(r.ids)[:tokens].astype(np.int32),
         "positions": np.arange(tokens, dtype=np.int32), "slots": np.zeros(tokens, np.int32),
         "final_norm_w": npf(r.final_norm_w), "lm_head": npf(r.lm_head), "layers": layers,
         "n_heads": m.n_heads, "n_kv_heads": m.n_kv_heads, "head_dim": m.head_dim, "eps": m.eps, "theta": m.theta,
         "seq_len": tokens, "n_seqs": 1}
    times = []
    t_start = time.perf_counter()
    while not times or time.perf_counter() - t_start < seconds:
        t0 = time.perf_counter()
        o.forward(p, fp16_storage=False)
        times.append(time.perf_counter() - t0)
    return {"value": tokens * len(times) / sum(times), "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": f"one {tokens}-token sequence through all {len(layers)} layers and the lm_head "
                      f"(oracle forward pinned to the reference LlamaRunner), repeated {len(times)}x "
                      f"({sum(times):.1f} s), fp32, single thread"}


def run_e2e(runner, stream, steps: int, device, dist, world: int) -> dict:
    """tokens/s through the C ABI with host buffers: every step copies its
    inputs (ids, positions, slots, each layer's GEMM outputs) from pinned host
    memory, runs the chain and copies the result (last rows) back. (Spreading
    the copies over four streams measured no faster: the host link is the
    bound.)"""
    import torch
    inputs = runner.step_inputs()
    hosts = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in inputs]
    for h, t in zip(hosts, inputs):
        h.copy_(t.cpu())
    result_host = torch.empty(runner.last_rows.shape, dtype=runner.last_rows.dtype, pin_memory=True)
    h2d = sum(t.numel() * t.element_size() for t in inputs)
    d2h = runner.last_rows.numel() * runner.last_rows.element_size()

    def step():
        for h, t in zip(hosts, inputs):
            t.copy_(h, non_blocking=True)
        runner.run(stream)
        result_host.copy_(runner.last_rows, non_blocking=True)

    with torch.cuda.stream(stream):
        for _ in range(2):
            step()
        stream.synchronize()
        if dist is not None:
            dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(steps):
            step()
        end.record(stream)
        end.synchronize()
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item()) / steps
    return {"value": runner.w.n_tokens * world / (ms_step * 1e-3), "unit": UNIT, "ms_per_step": ms_step,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            # the step's bytes over the host link per second of the whole step: the e2e bound when it
            # nears the link's rate (about 55 GB/s host to device on PCIe 5.0 x16)
            "host_link_gbs": (h2d + d2h) / (ms_step * 1e-3) / 1e9,
            "path": "pinned host -> cudaMemcpyAsync -> kllm_b200_chain_run -> last rows -> pinned host"}


_JSON_OUT = None


def log(msg: str) -> None:
    """Progress markers on stderr (stdout carries only the JSON line)."""
    sys.stderr.write(f"[bench] {msg}\n")
    sys.stderr.flush()


def emit(line: dict) -> None:
    """Writes the result line to the process's real stdout (libraries such as
    NCCL may print banners; those go to stderr, see main())."""
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    global _JSON_OUT
    import faulthandler
    faulthandler.enable()
    args = parse_args()
    # keep stdout for the one JSON line: everything else written to fd 1
    # (library banners, warnings) is redirected to stderr
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "llama_int8_dequant":
        run_dequant(args)
    elif args.workload == "llama_int8_load":
        run_load(args)
    elif args.workload in ATTENTION_WORKLOADS:
        run_attention(args)
    elif args.workload in GEMM_WORKLOADS:
        run_gemm(args)
    elif args.workload in GENERATE_WORKLOADS:
        run_generate(args)
    elif args.forward:
        run_forward(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
