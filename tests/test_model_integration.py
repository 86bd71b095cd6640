"""The reference's own Qwen3 model (nanovllm/models/qwen3.py) with kernel_backend="b200", end to end on the GPU.

Three copies of a 2-layer Qwen3-0.6B-architecture model (hidden 1024, 16 q / 8 kv heads of 128, intermediate 3072,
vocab 151936, tied embeddings) get the same random bf16 weights and the same randomly filled paged KV cache:
  * "compile" run eagerly (torch.compiler.set_stance("force_eager")): the reference's torch code, layer by layer
    (layers/layernorm.py, rotary_embedding.py, activation.py, the Triton store_kvcache of attention.py:11-41 and
    flash-attn) - the semantics the oracle restates;
  * "triton_fused": the reference's own Triton kernels (kernels/*.py), the same-box bar;
  * "b200": nanovllm_b200.install() routing (RMSNorm / Add+RMSNorm, the fused q/k norm + RoPE + KV write inside
    Attention.forward, SiLU x Mul, and this library's decode attention).
Each runs one prefill of three sequences (no prefix cache: Attention.forward's write_k path, attention.py:69-76)
and then one decode step (the flash_attn_with_kvcache branch, :84-91), with contexts set as ModelRunner sets them.

The referee is the same model in fp32 (every weight widened, no rounding between ops, softmax attention in fp32 over
each sequence's own keys), the reference's own way of judging its backends end to end. Checks: b200's logits after
the prefill and after the decode step, and the k and v rows it wrote into every layer's cache, deviate from the fp32
referee by no more than the reference's own backends do (largest and mean deviation at most 1.5x the worse of
"compile" and "triton_fused", plus one bf16 ulp at the values' scale for rounding-boundary noise); the logits stay
within 2 % of their largest magnitude of the fp32 referee; every cache row that was not written is bitwise
untouched.

Needs an importable reference nano-vllm: baseline/_ref (the offline install the benchmark uses), $NANOVLLM_REFERENCE
or a checkout named `reference` beside this repository.
"""
import json
import os
import socket
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CANDIDATES = [os.path.join(ROOT, "baseline", "_ref"), os.environ.get("NANOVLLM_REFERENCE", ""),
              os.path.join(os.path.dirname(ROOT), "reference")]
REF = next((p for p in CANDIDATES if p and os.path.isdir(os.path.join(p, "nanovllm"))), None)

CONFIG = {"architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "hidden_size": 1024,
          "intermediate_size": 3072, "num_hidden_layers": 2, "num_attention_heads": 16, "num_key_value_heads": 8,
          "head_dim": 128, "vocab_size": 151936, "max_position_embeddings": 40960, "rms_norm_eps": 1e-6,
          "rope_theta": 1000000, "tie_word_embeddings": True, "torch_dtype": "bfloat16", "dtype": "bfloat16",
          "hidden_act": "silu", "attention_bias": False}
BLOCK, NUM_BLOCKS = 256, 16
LENS = [100, 37, 300]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def models(cuda, tmp_path_factory):
    if REF is None:
        pytest.skip("no importable reference nano-vllm")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import torch.distributed as dist
    import nanovllm_b200
    nanovllm_b200.install()
    import nanovllm.kernels as kernels
    from nanovllm.models.qwen3 import Qwen3ForCausalLM
    from transformers import AutoConfig
    if not dist.is_initialized():  # Qwen3Attention reads the tensor-parallel size from the process group
        dist.init_process_group("gloo", f"tcp://127.0.0.1:{_free_port()}", world_size=1, rank=0)
    d = tmp_path_factory.mktemp("qwen3")
    (d / "config.json").write_text(json.dumps(CONFIG))
    hf = AutoConfig.from_pretrained(str(d))

    built = {}
    old_backend, old_dtype = kernels.backend, torch.get_default_dtype()
    try:
        for backend in ("compile", "triton_fused", "b200"):
            kernels.backend = backend  # the layers read it in __init__ (ModelRunner sets it the same way)
            torch.set_default_dtype(torch.bfloat16)
            with torch.device(cuda):
                built[backend] = Qwen3ForCausalLM(hf)
    finally:
        kernels.backend = old_backend
        torch.set_default_dtype(old_dtype)
    g = torch.Generator(device=cuda).manual_seed(0)
    with torch.no_grad():
        for name, p in built["compile"].named_parameters():
            if name.endswith("norm.weight"):
                p.copy_(1 + 0.1 * torch.randn(p.shape, generator=g, device=cuda))
            else:
                p.copy_(0.02 * torch.randn(p.shape, generator=g, device=cuda))
        state = built["compile"].state_dict()
        for backend in ("triton_fused", "b200"):
            built[backend].load_state_dict(state)
    cache0 = torch.randn(2, CONFIG["num_hidden_layers"], NUM_BLOCKS, BLOCK, 8, 128, generator=g,
                         device=cuda).to(torch.bfloat16)
    caches = {}
    for backend, model in built.items():
        kv = cache0.clone()
        layer = 0
        for m in model.modules():
            if hasattr(m, "k_cache") and hasattr(m, "v_cache"):
                m.k_cache, m.v_cache = kv[0, layer], kv[1, layer]
                layer += 1
        assert layer == CONFIG["num_hidden_layers"]
        caches[backend] = kv
    return dict(models=built, caches=caches, cache0=cache0, kernels=kernels)


def _block_tables(cuda):
    g = torch.Generator().manual_seed(1)
    perm = torch.randperm(NUM_BLOCKS, generator=g).tolist()
    tables, i = [], 0
    for L in LENS:
        n = (L + 1 + BLOCK - 1) // BLOCK  # room for the decode token
        tables.append(perm[i:i + n])
        i += n
    return tables


def _slot(table, pos):
    return table[pos // BLOCK] * BLOCK + pos % BLOCK


def _run(state, backend, cuda):
    """One prefill of LENS tokens, then one decode step; returns (prefill logits, decode logits, written slots)."""
    from nanovllm.utils.context import reset_context, set_context
    kernels, model = state["kernels"], state["models"][backend]
    tables = _block_tables(cuda)
    g = torch.Generator().manual_seed(2)
    ids = [torch.randint(0, CONFIG["vocab_size"], (L,), generator=g) for L in LENS]
    next_ids = torch.randint(0, CONFIG["vocab_size"], (len(LENS),), generator=g)
    positions = torch.cat([torch.arange(L) for L in LENS])
    slots = [_slot(t, p) for t, L in zip(tables, LENS) for p in range(L)]
    cu = torch.tensor([0] + list(torch.tensor(LENS).cumsum(0)), dtype=torch.int32)
    old = kernels.backend
    kernels.backend = backend  # the kernel names the layers bound resolve by it at call time
    try:
        with torch.inference_mode(), torch.compiler.set_stance("force_eager"):
            set_context(True, cu.to(cuda), cu.to(cuda), max(LENS), max(LENS),
                        torch.tensor(slots, dtype=torch.int32, device=cuda), None, None)
            h = model(torch.cat(ids).to(cuda), positions.to(cuda))
            prefill = model.compute_logits(h).float()
            width = max(len(t) for t in tables)
            bt = torch.tensor([t + [-1] * (width - len(t)) for t in tables], dtype=torch.int32, device=cuda)
            dslots = [_slot(t, L) for t, L in zip(tables, LENS)]
            set_context(False, slot_mapping=torch.tensor(dslots, dtype=torch.int32, device=cuda),
                        context_lens=torch.tensor([L + 1 for L in LENS], dtype=torch.int32, device=cuda),
                        block_tables=bt)
            h = model(next_ids.to(cuda), torch.tensor(LENS, device=cuda))
            decode = model.compute_logits(h).float()
            torch.cuda.synchronize()
    finally:
        kernels.backend = old
        reset_context()
    return prefill, decode, slots + dslots


@pytest.fixture(scope="module")
def runs(models, cuda):
    return {b: _run(models, b, cuda) for b in ("compile", "triton_fused", "b200")}




def _rms(x, w, eps=1e-6):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _rope(x, pos, d=128, theta=1e6):
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32, device=x.device) / d))
    f = pos.float()[:, None] * inv[None]
    cos, sin = f.cos()[:, None], f.sin()[:, None]
    x1, x2 = x[..., :d // 2], x[..., d // 2:]
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), -1)


def _referee(models, cuda):
    """fp32 forward of each sequence's L prompt tokens and its decode token (causal attention over its own L + 1
    tokens): logits at the last prompt position and at the decode position, and every layer's k (normed and
    rotated) and v rows for the L + 1 positions."""
    sd = {k: v.float() for k, v in models["models"]["compile"].state_dict().items()}
    hq, hkv, d, H = 16, 8, 128, CONFIG["hidden_size"]
    g = torch.Generator().manual_seed(2)
    ids = [torch.randint(0, CONFIG["vocab_size"], (L,), generator=g) for L in LENS]
    next_ids = torch.randint(0, CONFIG["vocab_size"], (len(LENS),), generator=g)
    prefill, decode, kv_rows = [], [], []
    for b, L in enumerate(LENS):
        tok = torch.cat([ids[b], next_ids[b:b + 1]]).to(cuda)
        pos = torch.arange(L + 1, device=cuda)
        h = sd["model.embed_tokens.weight"][tok]
        res, rows = None, []
        for i in range(CONFIG["num_hidden_layers"]):
            pre = f"model.layers.{i}."
            res = h if res is None else h + res
            x = _rms(res, sd[pre + "input_layernorm.weight"])
            qkv = x @ sd[pre + "self_attn.qkv_proj.weight"].t()
            q, k, v = qkv.split([hq * d, hkv * d, hkv * d], -1)
            q = _rope(_rms(q.view(-1, hq, d), sd[pre + "self_attn.q_norm.weight"]), pos)
            k = _rope(_rms(k.view(-1, hkv, d), sd[pre + "self_attn.k_norm.weight"]), pos)
            v = v.view(-1, hkv, d)
            rows.append((k, v))
            kk, vv = k.repeat_interleave(hq // hkv, 1), v.repeat_interleave(hq // hkv, 1)
            att = torch.einsum("qhd,khd->hqk", q, kk) * d ** -0.5
            att = att.masked_fill(torch.ones(L + 1, L + 1, dtype=torch.bool, device=cuda).triu(1), float("-inf"))
            o = torch.einsum("hqk,khd->qhd", att.softmax(-1), vv).reshape(L + 1, hq * d)
            h = o @ sd[pre + "self_attn.o_proj.weight"].t()
            res = h + res
            x = _rms(res, sd[pre + "post_attention_layernorm.weight"])
            gu = x @ sd[pre + "mlp.gate_up_proj.weight"].t()
            gate, up = gu.chunk(2, -1)
            h = (torch.nn.functional.silu(gate) * up) @ sd[pre + "mlp.down_proj.weight"].t()
        out = _rms(h + res, sd["model.norm.weight"]) @ sd["lm_head.weight"].t()
        prefill.append(out[L - 1])
        decode.append(out[L])
        kv_rows.append(rows)
    return torch.stack(prefill), torch.stack(decode), kv_rows


@pytest.fixture(scope="module")
def referee(models, cuda):
    with torch.no_grad():
        return _referee(models, cuda)


def _no_worse(devs, ref, what):
    """b200's largest and mean deviation from the fp32 referee at most 1.5x the worse of the reference's two
    backends, plus one bf16 ulp at ref's magnitude."""
    ulp = 2.0 ** (torch.log2(ref.abs().max()).floor().item() - 7)
    stats = {b: ((x - ref).abs().max().item(), (x - ref).abs().mean().item()) for b, x in devs.items()}
    print(what, {b: (f"max {m:.4g}", f"mean {a:.3g}") for b, (m, a) in stats.items()})
    worst_max = max(stats["compile"][0], stats["triton_fused"][0])
    worst_mean = max(stats["compile"][1], stats["triton_fused"][1])
    assert stats["b200"][0] <= 1.5 * worst_max + ulp, (what, stats)
    assert stats["b200"][1] <= 1.5 * worst_mean + ulp / 64, (what, stats)


@pytest.mark.parametrize("phase", ["prefill", "decode"])
def test_logits_against_fp32_referee(runs, referee, phase):
    i = 0 if phase == "prefill" else 1
    ref = referee[i]
    got = {b: runs[b][i] for b in ("compile", "triton_fused", "b200")}
    assert got["b200"].shape == ref.shape and torch.isfinite(got["b200"]).all()
    _no_worse(got, ref, f"{phase} logits")
    # Sanity bound: the reference's own backends stay within about 1.2 % of the logits' largest magnitude of the
    # fp32 referee after two bf16 layers; b200 within 2 %.
    scale = ref.abs().max().item()
    torch.testing.assert_close(got["b200"], ref, rtol=0, atol=2e-2 * scale)


def test_kv_cache_rows(runs, models, referee):
    """Rows written at the prefill and decode slots against the referee's k and v; every other row untouched."""
    written = torch.tensor(runs["b200"][2])
    assert written.unique().numel() == written.numel()
    untouched = torch.ones(NUM_BLOCKS * BLOCK, dtype=torch.bool)
    untouched[written] = False
    cache0 = models["cache0"].flatten(2, 3).cpu()
    for backend in ("compile", "triton_fused", "b200"):
        kv = models["caches"][backend].flatten(2, 3).cpu()
        assert torch.equal(kv[:, :, untouched], cache0[:, :, untouched]), backend
    # Slot order of `written`: each sequence's prefill positions in order, then every sequence's decode position.
    order = []
    n_prefill = sum(LENS)
    offset = 0
    for b, L in enumerate(LENS):
        order += [(b, p, offset + p) for p in range(L)]
        offset += L
    order += [(b, L, n_prefill + b) for b, L in enumerate(LENS)]
    for layer in range(CONFIG["num_hidden_layers"]):
        for j, name in enumerate(("k", "v")):
            ref = torch.stack([referee[2][b][layer][j][p] for b, p, _ in order])
            idx = torch.tensor([written[i] for _, _, i in order], device=ref.device)
            got = {bk: models["caches"][bk][j, layer].flatten(0, 1)[idx].float()
                   for bk in ("compile", "triton_fused", "b200")}
            _no_worse(got, ref, f"layer {layer} {name} rows")
