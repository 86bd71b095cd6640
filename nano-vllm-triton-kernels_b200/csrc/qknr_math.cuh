// Per-head math of the fused q/k RMSNorm + neox RoPE, shared by the fused op's kernels (qk_norm_rope_kv.cu) and the
// decode qkv projection with that op as its epilogue (matmul_tc.cu), so that both compute the same bits.
//
// Numerics (nanovllm/layers/layernorm.py:20-30, layers/rotary_embedding.py:6-14): x * rsqrt(mean(x^2) + eps) in
// fp32, rounded to bf16, times the bf16 weight (the exact product rounded once); then y1 = x1 cos - x2 sin,
// y2 = x2 cos + x1 sin with separately rounded fp32 products (no FMA contraction).
#pragma once

#include "common.cuh"

namespace nvb200 {
namespace {

// x1/x2: the 8 + 8 elements a lane holds of the two halves of a head (fp32 values of bf16 inputs). rstd: 1/rms of
// the head. w1/w2: the matching weights as bf16x2 words. c/s: cos/sin of the lane's 8 RoPE pairs. y1/y2: the rotated
// outputs in fp32 (rounded to bf16 by the caller's pack).
NVB200_DEVICE void norm_rope8(const float (&x1)[8], const float (&x2)[8], float rstd, const uint32_t (&w1)[4],
                              const uint32_t (&w2)[4], const float (&c)[8], const float (&s)[8], float (&y1)[8],
                              float (&y2)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // torch: x.mul_(rsqrt(var + eps)) in fp32, .to(bf16), .mul_(weight) in bf16 (exact product, one rounding).
    const uint32_t n1 = bf16x2_mul(pack_bf16x2(__fmul_rn(x1[2 * i], rstd), __fmul_rn(x1[2 * i + 1], rstd)), w1[i]);
    const uint32_t n2 = bf16x2_mul(pack_bf16x2(__fmul_rn(x2[2 * i], rstd), __fmul_rn(x2[2 * i + 1], rstd)), w2[i]);
    const float a0 = bf16_lo(n1), a1 = bf16_hi(n1), b0 = bf16_lo(n2), b1 = bf16_hi(n2);
    // apply_rotary_emb: y1 = x1*cos - x2*sin, y2 = x2*cos + x1*sin, each product rounded separately.
    y1[2 * i] = __fsub_rn(__fmul_rn(a0, c[2 * i]), __fmul_rn(b0, s[2 * i]));
    y1[2 * i + 1] = __fsub_rn(__fmul_rn(a1, c[2 * i + 1]), __fmul_rn(b1, s[2 * i + 1]));
    y2[2 * i] = __fadd_rn(__fmul_rn(b0, c[2 * i]), __fmul_rn(a0, s[2 * i]));
    y2[2 * i + 1] = __fadd_rn(__fmul_rn(b1, c[2 * i + 1]), __fmul_rn(a1, s[2 * i + 1]));
  }
}

NVB200_DEVICE void load_w8(const __nv_bfloat16 *p, uint32_t (&w)[4]) {
  const uint4 v = __ldg(reinterpret_cast<const uint4 *>(p));
  w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
}

// One head of 128 elements in the direct kernel's lane layout: lane j (0..7) of an 8-lane group holds xa = elements
// [8 j, 8 j + 8) and xb = [64 + 8 j, 64 + 8 j + 8). The group's sum of squares (fma over xa, then xb, then xor
// shuffles 4, 2, 1 within group_mask), RMSNorm with the bf16 weights w, RoPE with the fp32 cos | sin row cs; returns
// the lane's outputs for the same elements. The same operations in the same order as qknr_direct_kernel<128>.
// w and cs may point to global or shared memory (plain loads).
NVB200_DEVICE void head128_norm_rope(const uint4 &xa, const uint4 &xb, const __nv_bfloat16 *w, const float *cs,
                                     int j, float eps, unsigned group_mask, uint4 &ya, uint4 &yb) {
  uint32_t w1[4], w2[4];
  {
    const uint4 a = *reinterpret_cast<const uint4 *>(w + 8 * j), b = *reinterpret_cast<const uint4 *>(w + 64 + 8 * j);
    w1[0] = a.x, w1[1] = a.y, w1[2] = a.z, w1[3] = a.w, w2[0] = b.x, w2[1] = b.y, w2[2] = b.z, w2[3] = b.w;
  }
  float c[8], sn[8];
  {
    const float4 c0 = *reinterpret_cast<const float4 *>(cs + 8 * j);
    const float4 c1 = *reinterpret_cast<const float4 *>(cs + 8 * j + 4);
    const float4 s0 = *reinterpret_cast<const float4 *>(cs + 64 + 8 * j);
    const float4 s1 = *reinterpret_cast<const float4 *>(cs + 64 + 8 * j + 4);
    c[0] = c0.x, c[1] = c0.y, c[2] = c0.z, c[3] = c0.w, c[4] = c1.x, c[5] = c1.y, c[6] = c1.z, c[7] = c1.w;
    sn[0] = s0.x, sn[1] = s0.y, sn[2] = s0.z, sn[3] = s0.w, sn[4] = s1.x, sn[5] = s1.y, sn[6] = s1.z, sn[7] = s1.w;
  }
  float x1[8], x2[8];
  unpack8(xa, x1);
  unpack8(xb, x2);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = fmaf(x1[i], x1[i], ss);
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = fmaf(x2[i], x2[i], ss);
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) ss += __shfl_xor_sync(group_mask, ss, o);
  const float rstd = rsqrtf(ss / 128.f + eps);
  float y1[8], y2[8];
  norm_rope8(x1, x2, rstd, w1, w2, c, sn, y1, y2);
  ya = pack8(y1);
  yb = pack8(y2);
}

}  // namespace
}  // namespace nvb200
