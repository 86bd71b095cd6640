"""nanovllm_b200.install() against the reference package, on CPU (no kernels run).

Needs an importable reference nano-vllm, looked for in this order: the offline install under baseline/_ref
(`pip install --no-deps --target baseline/_ref <reference checkout>`), the path in $NANOVLLM_REFERENCE, and a
checkout named `reference` beside this repository. Checks that kernel_backend="b200" is accepted by Config, that the
layers' kernel names resolve to the b200 functions only while the backend is "b200", and that Qwen3Attention takes
the fused path for it.
"""
import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CANDIDATES = [os.path.join(ROOT, "baseline", "_ref"), os.environ.get("NANOVLLM_REFERENCE", ""),
              os.path.join(os.path.dirname(ROOT), "reference")]
REF = next((p for p in CANDIDATES if p and os.path.isdir(os.path.join(p, "nanovllm"))), None)
pytestmark = pytest.mark.skipif(REF is None, reason="no importable reference nano-vllm")

QWEN3_06B = {"architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "hidden_size": 1024,
             "intermediate_size": 3072, "num_hidden_layers": 28, "num_attention_heads": 16,
             "num_key_value_heads": 8, "head_dim": 128, "vocab_size": 151936, "max_position_embeddings": 40960,
             "rms_norm_eps": 1e-6, "rope_theta": 1000000, "tie_word_embeddings": True, "torch_dtype": "bfloat16",
             "hidden_act": "silu", "attention_bias": False}


@pytest.fixture(scope="module")
def ref():
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import nanovllm_b200
    nanovllm_b200.install()
    import nanovllm.kernels as kernels
    return kernels


def test_config_accepts_b200(ref, tmp_path):
    (tmp_path / "config.json").write_text(json.dumps(QWEN3_06B))
    from nanovllm.config import Config
    cfg = Config(str(tmp_path), kernel_backend="b200")
    assert cfg.kernel_backend == "b200"
    with pytest.raises(AssertionError):
        Config(str(tmp_path), kernel_backend="nonsense")


def test_kernel_names_follow_the_backend(ref):
    import nanovllm.layers.activation as act
    import nanovllm.layers.attention as att
    import nanovllm.layers.layernorm as ln
    from nanovllm_b200.kernels import qk_norm_rope_kv, rms_norm, swiglu
    assert ln.rms_norm.__b200__ is rms_norm.rms_norm
    assert ln.fused_add_rms_norm.__b200__ is rms_norm.fused_add_rms_norm
    assert act.silu_and_mul.__b200__ is swiglu.silu_and_mul
    assert att.qk_norm_rope_kv.__b200__ is qk_norm_rope_kv.qk_norm_rope_kv


def test_attention_layer_routes(ref):
    """The plain KV-cache write and decode attention of layers/attention.py resolve to the b200 kernels for "b200";
    decode calls the b200 kernel does not take keep flash-attn's function."""
    import torch
    import nanovllm.layers.attention as att
    from nanovllm_b200.kernels import attention
    assert att.store_kvcache.__b200__ is attention.store_kvcache
    assert att.flash_attn_with_kvcache.__b200__ is attention.flash_attn_with_kvcache
    q = torch.zeros(2, 1, 16, 128, dtype=torch.bfloat16)
    cache = torch.zeros(4, 256, 8, 128, dtype=torch.bfloat16)
    table = torch.zeros(2, 2, dtype=torch.int32)
    lens = torch.ones(2, dtype=torch.int32)
    kw = dict(cache_seqlens=lens, block_table=table, softmax_scale=0.1, causal=True)
    assert attention.supports(q, cache, cache, **kw)                      # the decode branch's call
    assert not attention.supports(q.float(), cache.float(), cache.float(), **kw)
    assert not attention.supports(q[..., :64], cache[..., :64], cache[..., :64], **kw)
    assert not attention.supports(torch.zeros(2, 9, 16, 128, dtype=torch.bfloat16), cache, cache, **kw)  # 18 rows
    assert not attention.supports(q, cache, cache, window_size=(8, 0), **kw)
    with pytest.raises(NotImplementedError):
        attention.flash_attn_with_kvcache(q, cache, cache, return_softmax_lse=True, **kw)


def test_qwen3_attention_is_fused_for_b200(ref):
    import torch
    import torch.distributed as dist
    from nanovllm.models.qwen3 import Qwen3Attention
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29617")
        dist.init_process_group("gloo", rank=0, world_size=1)
    old = ref.backend
    try:
        ref.backend = "b200"
        with torch.device("meta"):
            a = Qwen3Attention(1024, 16, 8, max_position=4096, head_dim=128, rope_theta=1e6)
        assert a.fused_norm_rope and a.attn.norm_rope is not None
        assert ref.backend == "b200"
        ref.backend = "compile"
        with torch.device("meta"):
            b = Qwen3Attention(1024, 16, 8, max_position=4096, head_dim=128, rope_theta=1e6)
        assert not b.fused_norm_rope
    finally:
        ref.backend = old


def test_projections_of_a_b200_model_take_the_b200_routes(ref):
    """Every projection of a b200 Qwen3 layer is marked for the b200 GEMM routes (steps 5, 7 and 8), including the
    qkv and o projections that Qwen3Attention builds while its constructor runs with the backend string set to
    "triton_fused"; the layers of other backends are not."""
    import torch
    import torch.distributed as dist
    from nanovllm.models.qwen3 import Qwen3Attention, Qwen3MLP
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29617")
        dist.init_process_group("gloo", rank=0, world_size=1)
    old = ref.backend
    try:
        for backend, expected in (("b200", True), ("compile", False)):
            ref.backend = backend
            with torch.device("meta"):
                a = Qwen3Attention(1024, 16, 8, max_position=4096, head_dim=128, rope_theta=1e6)
                m = Qwen3MLP(1024, 3072, "silu")
            assert getattr(a.qkv_proj, "_b200_matmul", False) is expected
            assert getattr(a, "_b200_qkv", False) is expected  # step 9: qkv projection + fused q/k epilogue
            assert getattr(a.o_proj, "_b200_matmul", False) is expected
            assert getattr(m.down_proj, "_b200_matmul", False) is expected
            assert getattr(m, "_b200_fused", False) is expected
            assert not getattr(a.o_proj, "_b200_fused", False)  # one rank: no all-reduce to fuse
            assert ref.backend == backend
    finally:
        ref.backend = old
