"""The layer-op chain of a decoder forward step on one GPU.

``ChainRunner`` owns the device buffers of one step of LlamaRunner::forward's
non-GEMM work (src/model/llama.cpp:78-178) for a model shape and a batch, fills
them with seeded synthetic data (GEMM outputs ~N(0,1), norm weights
~U(0.5,1.5), biases and the embedding table ~N(0,0.02)) and launches the whole
chain through ``kllm_b200_chain_run``. Every layer has its own input and output
buffers, so one step streams its whole working set (several GB) and nothing is
served from the 126 MB L2 across layers or steps. With ``attention=True,
gemm=True`` the step is the whole forward (attention, the tcgen05 GEMMs with
random N(0, 1/fan_in) weights, the lm_head), and ``decode_runner`` continues
it with decode steps over the same weights and KV caches.

Model shapes and workloads are the ones the benchmark is quoted on:
Qwen2.5-0.5B (hidden 896, 14/2 heads x 64, intermediate 4864, vocab 151936,
24 layers, eps 1e-6, theta 1e6) and Llama-2-7B (4096, 32/32 x 128, 11008,
32000, 32 layers, eps 1e-5, theta 1e4).
"""
from __future__ import annotations

import ctypes
from dataclasses import replace

import torch

from . import _capi
# shapes and workloads live in a module that maps no library (re-exported here)
from .workloads import (LLAMA2_7B, QWEN2_5_0_5B, WORKLOADS, ModelShape, Workload,  # noqa: F401
                        chain_bytes, shard, silu_bytes_per_launch)


class ChainRunner:
    """Device buffers + launch descriptor of one chain step.

    With ``shard=(rank, world)`` the workload is the global batch: data is
    generated for all of it (same seed on every rank, so identical to an
    unsharded run) and the runner keeps only this rank's sequences. That is
    for exact sharded-vs-unsharded checks on small cases; the benchmark gives
    each rank its own workload and seed instead.
    """

    TOKEN_TENSORS = ("q", "k", "v", "attn_out", "ffn_out", "gate", "up")

    def __init__(self, workload: Workload, device: torch.device | str = "cuda:0", seed: int = 0,
                 use_pdl: bool = True, n_layers: int | None = None,
                 weight_dtype: torch.dtype = torch.float16, shard: tuple[int, int] | None = None,
                 attention: bool = False, gemm: bool = False):
        m = workload.model
        self.device = torch.device(device)
        self.n_layers = n_layers or m.n_layers
        if shard is not None:
            from .dist import shard_range
            s0, s1 = shard_range(workload.n_seqs, *shard)
            self.w = replace(workload, n_seqs=s1 - s0)
        else:
            s0, s1 = 0, workload.n_seqs
            self.w = workload
        T, H, I = workload.n_tokens, m.hidden, m.intermediate
        t0, t1 = s0 * workload.seq_len, s1 * workload.seq_len
        qd, kvd = m.n_heads * m.head_dim, m.n_kv_heads * m.head_dim
        dev = self.device
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        f16 = torch.float16

        def normal(shape, std=1.0, dtype=f16):
            return (torch.randn(shape, generator=gen, device=dev, dtype=torch.float32) * std).to(dtype)

        def uniform(shape, lo, hi, dtype):
            return (torch.rand(shape, generator=gen, device=dev, dtype=torch.float32) * (hi - lo) + lo).to(dtype)

        def rows(t):
            return t if (t0, t1) == (0, T) else t[t0:t1].contiguous()

        Tl = t1 - t0
        if gemm and not attention:
            raise ValueError("the GEMM ops need attention (o_proj reads the attention output)")
        with torch.cuda.device(dev):
            self.table = normal((m.vocab, H), 0.02)
            self.ids = rows(torch.randint(0, m.vocab, (T,), generator=gen, device=dev, dtype=torch.int32))
            if workload.decode:
                self.positions = rows(torch.randint(0, workload.max_seq - 1, (T,), generator=gen, device=dev,
                                                    dtype=torch.int32))
                self.slots = torch.arange(Tl, device=dev, dtype=torch.int32)
            else:
                t = torch.arange(Tl, device=dev, dtype=torch.int32)
                self.positions = t % workload.seq_len
                self.slots = t // workload.seq_len
            self.residual = torch.empty((Tl, H), dtype=f16, device=dev)
            self.final_norm_w = uniform((H,), 0.5, 1.5, weight_dtype)
            self.final_norm_out = torch.empty((Tl, H), dtype=f16, device=dev)
            self.last_rows = torch.empty((s1 - s0, H), dtype=f16, device=dev)
            self.err_flags = torch.zeros((1,), dtype=torch.int32, device=dev)
            self.layers = []
            for _ in range(self.n_layers):
                if gemm:  # GEMM outputs are produced in the step; weights scaled by 1/sqrt(fan_in)
                    out = {"q": torch.empty((Tl, qd), dtype=f16, device=dev),
                           "k": torch.empty((Tl, kvd), dtype=f16, device=dev),
                           "v": torch.empty((Tl, kvd), dtype=f16, device=dev),
                           "attn_out": torch.empty((Tl, H), dtype=f16, device=dev),
                           "ffn_out": torch.empty((Tl, H), dtype=f16, device=dev)}
                else:
                    out = {"q": rows(normal((T, qd))), "k": rows(normal((T, kvd))), "v": rows(normal((T, kvd))),
                           "attn_out": rows(normal((T, H))), "ffn_out": rows(normal((T, H))),
                           "gate": rows(normal((T, I))), "up": rows(normal((T, I)))}
                L = {
                    **out,
                    "q_bias": normal((qd,), 0.02, weight_dtype), "k_bias": normal((kvd,), 0.02, weight_dtype),
                    "v_bias": normal((kvd,), 0.02, weight_dtype),
                    "input_norm_w": uniform((H,), 0.5, 1.5, weight_dtype),
                    "post_norm_w": uniform((H,), 0.5, 1.5, weight_dtype),
                    "attn_norm_out": torch.empty((Tl, H), dtype=f16, device=dev),
                    "ffn_norm_out": torch.empty((Tl, H), dtype=f16, device=dev),
                    "swiglu_out": torch.empty((Tl, I), dtype=f16, device=dev),
                    "k_cache": torch.empty((s1 - s0, m.n_kv_heads, workload.max_seq, m.head_dim),
                                           dtype=f16, device=dev),
                    "v_cache": torch.empty((s1 - s0, m.n_kv_heads, workload.max_seq, m.head_dim),
                                           dtype=f16, device=dev),
                }
                if attention:
                    # the step attends to the whole cache up to each position:
                    # earlier positions hold values from previous steps (the
                    # whole batch's values drawn, this shard's slots kept, so a
                    # sharded run sees the same cache rows as an unsharded one)
                    for name in ("k_cache", "v_cache"):
                        full = normal((workload.n_seqs, m.n_kv_heads, workload.max_seq, m.head_dim))
                        L[name].copy_(full[s0:s1] if (s0, s1) != (0, workload.n_seqs) else full)
                        del full
                    L["attn_ctx"] = torch.empty((Tl, qd), dtype=f16, device=dev)
                self.layers.append(L)
            self.attention = attention
            self.gemm = gemm
            self.weights = []
            if gemm:
                for _ in range(self.n_layers):
                    self.weights.append({
                        "wq": normal((qd, H), H ** -0.5), "wk": normal((kvd, H), H ** -0.5),
                        "wv": normal((kvd, H), H ** -0.5), "wo": normal((H, qd), qd ** -0.5),
                        "w_gate": normal((I, H), H ** -0.5), "w_up": normal((I, H), H ** -0.5),
                        "w_down": normal((H, I), I ** -0.5)})
                self.lm_head = normal((m.vocab, H), H ** -0.5)
                self.logits = torch.empty((s1 - s0, m.vocab), dtype=f16, device=dev)
            if attention:
                from . import ops
                nbytes = ops.attention_workspace_bytes(Tl, m.n_heads, m.n_kv_heads, m.head_dim, workload.max_seq)
                self.attn_workspace = torch.zeros(max(nbytes, 16), dtype=torch.uint8, device=dev)
        self.weight_dtype = weight_dtype
        self._build_desc(use_pdl)

    # tensors of a layer that a decode runner shares with the runner it follows
    _SHARED = ("q_bias", "k_bias", "v_bias", "input_norm_w", "post_norm_w", "k_cache", "v_cache")

    def decode_runner(self, ids: torch.Tensor, positions: torch.Tensor,
                      use_pdl: bool = True) -> "ChainRunner":
        """A runner for one new token per sequence (slot b for sequence b) that
        shares this runner's weights, norms, biases, embedding table, lm_head
        and KV caches, so a prefill step followed by decode steps runs as
        LlamaRunner::forward does across calls (src/model/llama.cpp:68-184):
        each decode step appends its k/v at positions[b] and attends to the
        cache rows the earlier steps wrote. Needs the whole forward
        (attention=True, gemm=True)."""
        if not (self.attention and self.gemm):
            raise ValueError("a decode runner needs the whole forward step (attention and GEMMs)")
        m = self.w.model
        B = self.w.n_seqs
        if ids.numel() != B or positions.numel() != B:
            raise ValueError("one id and one position per sequence")
        dev, f16 = self.device, torch.float16
        qd, kvd, H, I = m.n_heads * m.head_dim, m.n_kv_heads * m.head_dim, m.hidden, m.intermediate
        r = ChainRunner.__new__(ChainRunner)
        r.device, r.n_layers, r.weight_dtype = dev, self.n_layers, self.weight_dtype
        r.w = replace(self.w, seq_len=1, decode=True)
        r.attention, r.gemm = True, True
        r.table, r.final_norm_w, r.weights = self.table, self.final_norm_w, self.weights
        with torch.cuda.device(dev):
            r.ids = ids.to(device=dev, dtype=torch.int32).contiguous()
            r.positions = positions.to(device=dev, dtype=torch.int32).contiguous()
            r.slots = torch.arange(B, device=dev, dtype=torch.int32)
            r.residual = torch.empty((B, H), dtype=f16, device=dev)
            r.final_norm_out = torch.empty((B, H), dtype=f16, device=dev)
            r.last_rows = torch.empty((B, H), dtype=f16, device=dev)
            r.err_flags = torch.zeros((1,), dtype=torch.int32, device=dev)
            r.layers = []
            for L in self.layers:
                D = {k: L[k] for k in self._SHARED}
                D.update({"q": torch.empty((B, qd), dtype=f16, device=dev),
                          "k": torch.empty((B, kvd), dtype=f16, device=dev),
                          "v": torch.empty((B, kvd), dtype=f16, device=dev),
                          "attn_out": torch.empty((B, H), dtype=f16, device=dev),
                          "ffn_out": torch.empty((B, H), dtype=f16, device=dev),
                          "attn_norm_out": torch.empty((B, H), dtype=f16, device=dev),
                          "ffn_norm_out": torch.empty((B, H), dtype=f16, device=dev),
                          "swiglu_out": torch.empty((B, I), dtype=f16, device=dev),
                          "attn_ctx": torch.empty((B, qd), dtype=f16, device=dev)})
                r.layers.append(D)
            r.lm_head = self.lm_head
            r.logits = torch.empty((B, m.vocab), dtype=f16, device=dev)
            from . import ops
            nbytes = ops.attention_workspace_bytes(B, m.n_heads, m.n_kv_heads, m.head_dim, r.w.max_seq)
            r.attn_workspace = torch.zeros(max(nbytes, 16), dtype=torch.uint8, device=dev)
        r._build_desc(use_pdl)
        return r

    def _build_desc(self, use_pdl: bool) -> None:
        w, m = self.w, self.w.model
        arr = (_capi.LayerBuffers * self.n_layers)()
        for i, L in enumerate(self.layers):
            for name, t in L.items():
                setattr(arr[i], name, t.data_ptr())
        self._layer_arr = arr
        c = _capi.Chain()
        c.n_tokens, c.hidden, c.n_heads, c.n_kv_heads = w.n_tokens, m.hidden, m.n_heads, m.n_kv_heads
        c.head_dim, c.intermediate, c.vocab, c.n_layers = m.head_dim, m.intermediate, m.vocab, self.n_layers
        c.n_slots, c.max_seq, c.n_seqs, c.seq_len = w.n_seqs, w.max_seq, w.n_seqs, w.seq_len
        c.eps, c.theta = m.eps, m.theta
        c.weight_dtype = _capi.F16 if self.weight_dtype == torch.float16 else _capi.F32
        c.use_pdl = int(use_pdl)
        c.embed_table, c.ids = self.table.data_ptr(), self.ids.data_ptr()
        c.positions, c.slots, c.seq_ends = self.positions.data_ptr(), self.slots.data_ptr(), None
        c.residual, c.final_norm_w = self.residual.data_ptr(), self.final_norm_w.data_ptr()
        c.final_norm_out, c.last_rows = self.final_norm_out.data_ptr(), self.last_rows.data_ptr()
        c.layers = ctypes.cast(arr, ctypes.POINTER(_capi.LayerBuffers))
        c.err_flags = self.err_flags.data_ptr()
        if self.attention:
            c.op_mask = _capi.OP_CHAIN | _capi.OP_ATTENTION
            c.attn_workspace = self.attn_workspace.data_ptr()
            c.attn_workspace_bytes = self.attn_workspace.numel()
        if self.gemm:
            warr = (_capi.LayerWeights * self.n_layers)()
            for i, W in enumerate(self.weights):
                for name, t in W.items():
                    setattr(warr[i], name, t.data_ptr())
            self._weight_arr = warr
            c.weights = ctypes.cast(warr, ctypes.POINTER(_capi.LayerWeights))
            c.lm_head, c.logits = self.lm_head.data_ptr(), self.logits.data_ptr()
            c.op_mask = _capi.OP_FORWARD
        self.desc = c
        self.full_mask = c.op_mask

    @property
    def fused_embedding(self) -> bool:
        """Whether the step runs the embedding and layer 0's input norm as
        one kernel (the chain executor fuses them when both ops are on)."""
        mask = self.desc.op_mask or _capi.OP_CHAIN
        both = _capi.OP_EMBEDDING | _capi.OP_INPUT_NORM
        return (mask & both) == both

    @property
    def fused_select(self) -> bool:
        """Whether the final norm's kernel also writes the last rows (the
        chain executor fuses them when both ops are on and every sequence has
        seq_len rows)."""
        mask = self.desc.op_mask or _capi.OP_CHAIN
        both = _capi.OP_FINAL_NORM | _capi.OP_SELECT
        return (mask & both) == both and not self.desc.seq_ends

    def set_pdl(self, use_pdl: bool) -> None:
        self.desc.use_pdl = int(use_pdl)

    def run(self, stream: torch.cuda.Stream | None = None) -> int:
        """Enqueues one chain step; returns the number of kernels launched."""
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        n = ctypes.c_int(0)
        with torch.cuda.device(self.device):
            _capi.check(_capi.lib.kllm_b200_chain_run(ctypes.byref(self.desc), ctypes.byref(n), s.cuda_stream))
        return n.value

    def step_inputs(self) -> list[torch.Tensor]:
        """Tensors a step consumes that a real forward would produce afresh
        each step (ids, positions, slots and the GEMM outputs)."""
        out = [self.ids, self.positions, self.slots]
        if self.gemm:  # the whole forward: every other tensor is produced in the step
            return out
        for L in self.layers:
            out += [L[k] for k in ("q", "k", "v", "attn_out", "ffn_out", "gate", "up")]
        return out
