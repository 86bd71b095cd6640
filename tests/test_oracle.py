"""The oracle (oracle/reference_math.py) against the reference's own outputs (tests/golden/golden.pt), bit for bit.

golden.pt was written by tests/golden/make_golden.py from the reference's layer modules run eagerly on CPU; this
test needs neither the reference nor a GPU.
"""
import os

import pytest
import torch

from oracle import reference_math as om

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.pt")


@pytest.fixture(scope="module")
def golden():
    return torch.load(GOLDEN)


def test_golden_file_is_small(golden):
    assert os.path.getsize(GOLDEN) < 1_000_000


@pytest.mark.parametrize("case", ["rms_7x128", "rms_5x1024", "rms_3x200"])
def test_rms_norm(golden, case):
    c = golden[case]
    assert torch.equal(om.rms_forward(c["x"], c["w"], golden["eps"]), c["y"])


def test_rms_norm_strided_q_view(golden):
    c = golden["rms_qview"]
    q = c["qkv"].split([16 * 128, 8 * 128, 8 * 128], dim=-1)[0].view(-1, 16, 128)
    assert q.stride(0) == 32 * 128  # really a strided view
    assert torch.equal(om.rms_forward(q, c["w"], golden["eps"]), c["y"])


@pytest.mark.parametrize("case", ["add_rms_7x1024", "add_rms_4x128"])
def test_add_rms_norm(golden, case):
    c = golden[case]
    y, s = om.add_rms_forward(c["x"], c["r"], c["w"], golden["eps"])
    assert torch.equal(y, c["y"]) and torch.equal(s, c["s"])


@pytest.mark.parametrize("max_pos", [4096, 40960])
def test_rope_table(golden, max_pos):
    c = golden[f"rope_table_{max_pos}"]
    table = om.rope_cos_sin_cache(128, max_pos, 1e6)
    assert table.shape == (max_pos, 1, 128) and table.dtype == torch.float32
    assert torch.equal(table[c["positions"]], c["rows"])


@pytest.mark.parametrize("case", ["fused_06b", "fused_8b"])
def test_fused_composition(golden, case):
    c = golden[case]
    hq, hkv = c["hq"], c["hkv"]
    q, k, v = c["qkv"].split([hq * 128, hkv * 128, hkv * 128], dim=-1)
    q, k, v = q.view(-1, hq, 128), k.view(-1, hkv, 128), v.view(-1, hkv, 128)
    T = q.shape[0]
    table = om.rope_cos_sin_cache(128, 4096, 1e6)
    kc = torch.randn(4, 256, hkv, 128).to(torch.bfloat16)
    vc = torch.randn(4, 256, hkv, 128).to(torch.bfloat16)
    before_k, before_v = kc.clone(), vc.clone()
    slots = torch.arange(T, dtype=torch.int32) * 3
    slots[1] = -1
    q_out, k_out = om.qk_norm_rope_kv(q, k, v, c["positions"], c["q_w"], c["k_w"], golden["eps"], table, kc, vc,
                                      slots, True)
    assert torch.equal(q_out, c["q_out"]) and torch.equal(k_out, c["k_out"])
    # KV write as store_kvcache_kernel: rows at kept slots, nothing else touched.
    flat_k, flat_v = kc.view(-1, hkv, 128), vc.view(-1, hkv, 128)
    keep = slots >= 0
    assert torch.equal(flat_k[slots[keep].long()], c["k_out"][keep])
    assert torch.equal(flat_v[slots[keep].long()], v[keep])
    untouched = torch.ones(flat_k.shape[0], dtype=torch.bool)
    untouched[slots[keep].long()] = False
    assert torch.equal(flat_k[untouched], before_k.view(-1, hkv, 128)[untouched])
    assert torch.equal(flat_v[untouched], before_v.view(-1, hkv, 128)[untouched])


def test_silu_and_mul(golden):
    c = golden["silu_3x3072"]
    assert torch.equal(om.silu_and_mul(c["x"]), c["y"])


def test_ulp_metric():
    a = torch.tensor([1.0, -1.0, 0.0, 2.0]).to(torch.bfloat16)
    b = torch.tensor([1.0078125, -1.0078125, -0.0, 2.0]).to(torch.bfloat16)  # one bf16 step at 1.0
    assert om.bf16_ulp_diff(a, b).tolist() == [1, 1, 0, 0]


def test_byte_formulas():
    # scripts/bench_qk_rope_kv.py:10-12: Qwen3-0.6B moves 16,908 B per token plus the two weight rows.
    assert om.qk_norm_rope_kv_bytes(1, 16, 8, 128) == 16908 + 512
    assert om.qk_norm_rope_kv_bytes(2048, 16, 8, 128) == 34_628_096
    assert om.qk_norm_rope_kv_bytes(8192, 32, 8, 128) == 8192 * 25_100 + 512
    assert om.matmul_flops(4096, 4096, 4096) == 137_438_953_472
