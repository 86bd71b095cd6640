"""Registers the B200 kernels as kernel_backend="b200" in an importable reference nano-vllm, without editing it.

The reference selects its kernels with the module-global string `nanovllm.kernels.backend`, which
`ModelRunner.__init__` sets from `Config.kernel_backend` before building the model
(nanovllm/engine/model_runner.py:83) and the layers read once in `__init__`. install():

1. lets `Config.__post_init__` accept "b200" (it asserts the backend is compile/triton/triton_fused,
   nanovllm/config.py:39);
2. makes the kernel names the layers bound at import (nanovllm/layers/layernorm.py:5, layers/activation.py:6,
   layers/attention.py:7) and the `nanovllm.kernels.*` module attributes resolve to the b200 functions whenever
   `nanovllm.kernels.backend == "b200"`; every other backend keeps the reference's own kernels;
3. makes `Qwen3Attention` (nanovllm/models/qwen3.py:73-75) take the fused path for "b200" as for "triton_fused",
   so q/k norm, RoPE and the KV write run as one kernel inside Attention.forward (layers/attention.py:64-76);
4. makes the tensor-parallel worker processes (spawned, nanovllm/engine/llm_engine.py:24-30) run install() too;
5. under tensor parallelism, makes RowParallelLinear (o_proj, down_proj; nanovllm/layers/linear.py:131-156) run
   decode-sized batches (at most 64 rows, bf16, no bias) as one fused GEMM + NVLink all-reduce kernel per rank
   (nanovllm_b200.parallel.RowParallelAllReduce) instead of F.linear and an NCCL all-reduce. Its exchange buffers
   are set up collectively on the first call, which is the warm-up prefill (never a CUDA-graph capture), so the
   decode graphs capture only the kernel;
6. makes the attention layer's plain KV-cache write (store_kvcache, nanovllm/layers/attention.py:34-41, the route of
   models whose q/k are normalised before the layer) and its decode attention (the flash_attn_with_kvcache call of
   Attention.forward, :84-91) run the b200 kernels while the backend is "b200". Decode calls outside what the b200
   kernel takes (`nanovllm_b200.kernels.attention.supports`: bf16, head_dim 128, at most 16 query rows per KV head)
   keep flash-attn's; prefill attention (flash_attn_varlen_func, :79-83) stays flash-attn's;
7. makes Qwen3MLP (nanovllm/models/qwen3.py:133-137) run its gate_up projection and SiLU x Mul as one kernel
   (nanovllm_b200.kernels.matmul.linear_decode with swiglu) for the batches `fused_gate_up_applies` admits;
8. makes ColumnParallelLinear (nanovllm/layers/linear.py:72-73) and, on one GPU, RowParallelLinear (:152-156) run
   the projections `decode_gemm_applies` admits (decode-sized bf16 batches, no bias, N <= K: o_proj and down_proj)
   through nanovllm_b200.kernels.matmul.linear_decode instead of F.linear (cuBLAS): a weight-streaming kernel whose
   weight loads start while the preceding kernel finishes. The thresholds of both steps are the measured
   crossovers against cuBLAS (nanovllm_b200/kernels/matmul.py).
9. makes the decode steps of Qwen3Attention (nanovllm/models/qwen3.py:77-84) on one GPU run the qkv projection with
   the fused q/k op as its epilogue (nanovllm_b200.kernels.qk_norm_rope_kv.linear_qkv_norm_rope_kv: one kernel, the
   qkv intermediate never written) and then the decode attention (step 6), for the batches that kernel takes. (Under
   tensor parallelism each rank's few heads leave the kernel with too little work per CTA: the TP 2 step measured
   slower with it, 1628 us against 1469 us without it on another box.)

Call it once, before constructing `LLM(..., kernel_backend="b200")`.
"""
import functools

BACKEND = "b200"
_installed = False
# Depth of Qwen3Attention.__init__ calls of a b200 model in progress: step 3 runs them with the backend string set to
# "triton_fused", so the layers built inside (qkv_proj, o_proj) ask this rather than the string.
_attention_init_depth = 0


def _by_backend(kernels_mod, ours, theirs):
    @functools.wraps(theirs)
    def fn(*args, **kwargs):
        return (ours if kernels_mod.backend == BACKEND else theirs)(*args, **kwargs)
    fn.__b200__ = ours
    return fn


def _building_b200(kernels_mod) -> bool:
    """Whether a layer being constructed belongs to a kernel_backend="b200" model."""
    return kernels_mod.backend == BACKEND or _attention_init_depth > 0


def _model_runner(config, rank, event):
    """Spawned TP worker entry: register the backend in this fresh process, then run the reference's ModelRunner."""
    install()
    from nanovllm.engine.model_runner import ModelRunner
    return ModelRunner(config, rank, event)


def install() -> None:
    global _installed
    if _installed:
        return
    import nanovllm.config as config_mod
    import nanovllm.engine.llm_engine as engine_mod
    import nanovllm.kernels as kernels_mod
    import nanovllm.kernels.matmul as ref_matmul
    import nanovllm.kernels.qk_norm_rope_kv as ref_fused
    import nanovllm.kernels.rms_norm as ref_norm
    import nanovllm.kernels.swiglu as ref_swiglu
    import nanovllm.layers.activation as activation_mod
    import nanovllm.layers.attention as attention_mod
    import nanovllm.layers.layernorm as layernorm_mod
    import nanovllm.models.qwen3 as qwen3_mod

    from nanovllm_b200.kernels import attention as b200_attention
    from nanovllm_b200.kernels import matmul as b200_matmul
    from nanovllm_b200.kernels import qk_norm_rope_kv as b200_fused
    from nanovllm_b200.kernels import rms_norm as b200_norm
    from nanovllm_b200.kernels import swiglu as b200_swiglu

    # 1. Config accepts "b200".
    post_init = config_mod.Config.__post_init__

    def __post_init__(self):
        if self.kernel_backend != BACKEND:
            return post_init(self)
        self.kernel_backend = "triton_fused"
        try:
            post_init(self)
        finally:
            self.kernel_backend = BACKEND
    config_mod.Config.__post_init__ = __post_init__

    # 2. Kernel names resolve by backend.
    pairs = [
        (ref_norm, "rms_norm", b200_norm.rms_norm), (ref_norm, "fused_add_rms_norm", b200_norm.fused_add_rms_norm),
        (ref_swiglu, "silu_and_mul", b200_swiglu.silu_and_mul),
        (ref_fused, "qk_norm_rope_kv", b200_fused.qk_norm_rope_kv), (ref_matmul, "matmul", b200_matmul.matmul),
        (layernorm_mod, "rms_norm", b200_norm.rms_norm),
        (layernorm_mod, "fused_add_rms_norm", b200_norm.fused_add_rms_norm),
        (activation_mod, "silu_and_mul", b200_swiglu.silu_and_mul),
        (attention_mod, "qk_norm_rope_kv", b200_fused.qk_norm_rope_kv),
        (attention_mod, "store_kvcache", b200_attention.store_kvcache),
    ]
    for mod, name, ours in pairs:
        setattr(mod, name, _by_backend(kernels_mod, ours, getattr(mod, name)))

    # Decode attention: the b200 kernel for the calls it takes, flash-attn's for the rest.
    flash_decode = attention_mod.flash_attn_with_kvcache

    @functools.wraps(flash_decode)
    def flash_attn_with_kvcache(*args, **kwargs):
        if kernels_mod.backend == BACKEND and b200_attention.supports(*args, **kwargs):
            return b200_attention.flash_attn_with_kvcache(*args, **kwargs)
        return flash_decode(*args, **kwargs)
    flash_attn_with_kvcache.__b200__ = b200_attention.flash_attn_with_kvcache
    attention_mod.flash_attn_with_kvcache = flash_attn_with_kvcache

    # 3. Qwen3Attention treats "b200" as a fused backend.
    attn_init = qwen3_mod.Qwen3Attention.__init__

    @functools.wraps(attn_init)
    def __init__(self, *args, **kwargs):
        global _attention_init_depth
        if kernels_mod.backend != BACKEND:
            return attn_init(self, *args, **kwargs)
        kernels_mod.backend = "triton_fused"
        _attention_init_depth += 1
        try:
            attn_init(self, *args, **kwargs)
        finally:
            _attention_init_depth -= 1
            kernels_mod.backend = BACKEND
        self._b200_qkv = self.fused_norm_rope
    qwen3_mod.Qwen3Attention.__init__ = __init__

    # 9. Decode steps of a b200 Qwen3Attention: the qkv projection with the fused q/k op as its epilogue (one kernel,
    # nvb200_linear_qkv_norm_rope_kv), then the decode attention on the cache it wrote; other calls (prefill, more
    # rows than the kernel takes) run the forward above.
    attn_forward = qwen3_mod.Qwen3Attention.forward
    import nanovllm.utils.context as context_mod

    @functools.wraps(attn_forward)
    def qwen3_attention_forward(self, positions, hidden_states):
        ctx = context_mod.get_context()
        if (getattr(self, "_b200_qkv", False) and not ctx.is_prefill and hidden_states.dim() == 2
                and self.qkv_proj.tp_size == 1 and getattr(self.qkv_proj, "bias", None) is None
                and self.attn.k_cache.numel() > 0):
            attn = self.attn
            q_norm, k_norm, rotary = attn.norm_rope
            q = b200_fused.linear_qkv_norm_rope_kv(
                hidden_states, self.qkv_proj.weight, self.num_heads, self.num_kv_heads, positions, q_norm.weight,
                k_norm.weight, q_norm.eps, rotary.cos_sin_cache, attn.k_cache, attn.v_cache, ctx.slot_mapping)
            if q is not None:
                num_seqs = ctx.context_lens.size(0)
                o = attention_mod.flash_attn_with_kvcache(
                    q.reshape(num_seqs, -1, attn.num_heads, attn.head_dim), attn.k_cache, attn.v_cache,
                    cache_seqlens=ctx.context_lens, block_table=ctx.block_tables, softmax_scale=attn.scale,
                    causal=True)
                return self.post_attn(o.view(-1, attn.num_heads, attn.head_dim))
        return attn_forward(self, positions, hidden_states)
    qwen3_mod.Qwen3Attention.forward = qwen3_attention_forward

    # 4. Spawned tensor-parallel workers register the backend before building their ModelRunner.
    engine_mod.ModelRunner = _model_runner

    # 5. Row-parallel layers of a b200 model: fused GEMM + all-reduce for decode-sized batches.
    import nanovllm.layers.linear as linear_mod
    row_init, row_forward = linear_mod.RowParallelLinear.__init__, linear_mod.RowParallelLinear.forward

    @functools.wraps(row_init)
    def row_parallel_init(self, *args, **kwargs):
        row_init(self, *args, **kwargs)
        self._b200_fused = _building_b200(kernels_mod) and self.tp_size > 1
        self._b200_matmul = _building_b200(kernels_mod)

    @functools.wraps(row_forward)
    def row_parallel_forward(self, x):
        if not getattr(self, "_b200_fused", False):
            return row_forward(self, x)
        op = _row_parallel_op(self.weight.shape[0], x.device)
        if (op is None or self.bias is not None or x.dim() != 2 or x.shape[0] > 64 or x.dtype != self.weight.dtype
                or self.weight.shape[0] > op.max_n):
            return row_forward(self, x)
        return op(x, self.weight.t())
    linear_mod.RowParallelLinear.__init__ = row_parallel_init
    linear_mod.RowParallelLinear.forward = row_parallel_forward

    # 7. Qwen3MLP (models/qwen3.py:133-137) of a b200 model: the gate_up projection and SiLU x Mul as one kernel
    # (nvb200_linear_decode with swiglu) for the batches where it was measured faster than the projection followed by
    # the SiLU x Mul kernel; the down projection goes through its own layer (steps 5 and 8).
    mlp_init, mlp_forward = qwen3_mod.Qwen3MLP.__init__, qwen3_mod.Qwen3MLP.forward

    @functools.wraps(mlp_init)
    def qwen3_mlp_init(self, *args, **kwargs):
        mlp_init(self, *args, **kwargs)
        self._b200_fused = _building_b200(kernels_mod)

    @functools.wraps(mlp_forward)
    def qwen3_mlp_forward(self, x):
        w = self.gate_up_proj.weight
        if (not getattr(self, "_b200_fused", False) or getattr(self.gate_up_proj, "bias", None) is not None
                or not b200_matmul.fused_gate_up_applies(x, w)):
            return mlp_forward(self, x)
        y = b200_matmul.linear_decode(x, w, swiglu=True)
        return mlp_forward(self, x) if y is None else self.down_proj(y)
    qwen3_mod.Qwen3MLP.__init__ = qwen3_mlp_init
    qwen3_mod.Qwen3MLP.forward = qwen3_mlp_forward

    # 8. Decode-sized projections of a b200 model: column-parallel layers, and row-parallel ones without tensor
    # parallelism (step 5 takes them under it), through b200 `matmul`.
    col_init, col_forward = linear_mod.ColumnParallelLinear.__init__, linear_mod.ColumnParallelLinear.forward

    @functools.wraps(col_init)
    def column_parallel_init(self, *args, **kwargs):
        col_init(self, *args, **kwargs)
        self._b200_matmul = _building_b200(kernels_mod)

    @functools.wraps(col_forward)
    def column_parallel_forward(self, x):
        if (not getattr(self, "_b200_matmul", False) or self.bias is not None
                or not b200_matmul.decode_gemm_applies(x, self.weight)):
            return col_forward(self, x)
        y = b200_matmul.linear_decode(x, self.weight)
        return col_forward(self, x) if y is None else y
    linear_mod.ColumnParallelLinear.__init__ = column_parallel_init
    linear_mod.ColumnParallelLinear.forward = column_parallel_forward

    row_fused_forward = linear_mod.RowParallelLinear.forward

    @functools.wraps(row_fused_forward)
    def row_parallel_single_forward(self, x):
        if (self.tp_size == 1 and getattr(self, "_b200_matmul", False) and self.bias is None
                and b200_matmul.decode_gemm_applies(x, self.weight)):
            y = b200_matmul.linear_decode(x, self.weight)
            if y is not None:
                return y
        return row_fused_forward(self, x)
    linear_mod.RowParallelLinear.forward = row_parallel_single_forward
    _installed = True


_row_op = None


def _row_parallel_op(n_out, device):
    """The process's RowParallelAllReduce, created (collectively: every rank runs the same layers) by the first
    row-parallel call outside a CUDA-graph capture; None while it does not exist and a capture is running."""
    global _row_op
    if _row_op is None:
        import torch
        if torch.cuda.is_current_stream_capturing():
            return None
        from nanovllm_b200.parallel import RowParallelAllReduce
        _row_op = RowParallelAllReduce(max_n=n_out, device=device)
        # One call at once (every rank reaches this point together), so that the kernel's one-time set-up (its
        # shared-memory attribute) is done before any graph capture.
        x = torch.zeros(1, 64, dtype=torch.bfloat16, device=device)
        _row_op(x, torch.zeros(n_out, 64, dtype=torch.bfloat16, device=device).t())
    return _row_op
