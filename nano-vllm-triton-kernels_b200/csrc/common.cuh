// Shared device helpers for the sm_100a kernels: bf16 rounding, packed 16-byte vectors, mbarriers with bounded
// waits, and the 1-D bulk-copy (cp.async.bulk) engine that moves token tiles between HBM and shared memory.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "nvb200.h"

#define NVB200_DEVICE __device__ __forceinline__

namespace nvb200 {

// ---------------------------------------------------------------------------------------------------------------
// Numeric helpers. All rounding is round-to-nearest-even, as torch's .to(bfloat16) / .to(float16).

template <typename T> struct Elem;
template <> struct Elem<__nv_bfloat16> {
  static NVB200_DEVICE float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static NVB200_DEVICE __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Elem<__half> {
  static NVB200_DEVICE float to_f(__half x) { return __half2float(x); }
  static NVB200_DEVICE __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct Elem<float> {
  static NVB200_DEVICE float to_f(float x) { return x; }
  static NVB200_DEVICE float from_f(float x) { return x; }
};

// Round an fp32 value to T and back (the value torch holds after .to(T)).
template <typename T> NVB200_DEVICE float round_to(float x) { return Elem<T>::to_f(Elem<T>::from_f(x)); }

// 16 bytes as 8 bf16, for vectorised global and shared-memory access. Element 2i is the low half of word i.
union Pack8 {
  uint4 u;
  __nv_bfloat162 h2[4];
  __nv_bfloat16 h[8];
};

// Two bf16 in one 32-bit word -> fp32 (exact: a bf16 is the top half of an fp32).
NVB200_DEVICE float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
NVB200_DEVICE float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Rounds lo and hi to bf16 (round to nearest even) and packs them, lo in the low half.
NVB200_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

NVB200_DEVICE void unpack8(const uint4 &u, float (&f)[8]) {
  f[0] = bf16_lo(u.x), f[1] = bf16_hi(u.x), f[2] = bf16_lo(u.y), f[3] = bf16_hi(u.y);
  f[4] = bf16_lo(u.z), f[5] = bf16_hi(u.z), f[6] = bf16_lo(u.w), f[7] = bf16_hi(u.w);
}

NVB200_DEVICE uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

// Product of two bf16x2 words, each lane rounded once to bf16 (the exact product of two bf16 fits fp32, so this
// equals torch's bf16 multiply: fp32 product rounded to bf16).
NVB200_DEVICE uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// SiLU x Mul on bf16, shared by the SiLU x Mul kernel and the gate_up GEMM epilogue.
// Fast path: silu(g) rounded to bf16 depends only on the 16-bit g, so an estimate that lies close enough to
// the exact fp32 value rounds the same way. The estimate g * rcp(1 + 2^(-g log2 e)) (the operations of __expf and
// __fdividef, documented bounds 2 + floor(1.173 |x|) ulps and 2 ulps) lies within a few tens of fp32 ulps of the
// exact value for |g| <= 16; wherever the estimate's low
// 16 bits lie within kSiluMargin of the bf16 rounding midpoint 0x8000, or |g| > 16 (or g is not finite), the exact
// expression is evaluated instead. Away from the midpoint the estimate and the exact value round to the same bf16.
// The exact path costs about twice the instructions (accurate expf, IEEE division) and kept the kernel issue-bound
// below the memory roofline; the tests compare all 65,536 bf16 gate values with torch bit for bit.
constexpr float kSiluFastRange = 16.0f;
constexpr uint32_t kSiluMargin = 64;

// 2^x and 1/x by the hardware approximations, flushing denormal inputs and results (never met by the fast path's
// arguments: 2^(-g log2 e) and 1 + that lie in [1e-7, 1e7] for |g| <= 16). These are the operations __expf and
// __fdividef are built on, minus their denormal handling.
NVB200_DEVICE float ex2_approx_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
NVB200_DEVICE float rcp_approx_ftz(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two fp32 values in one 64-bit register pair, for sm_100's packed fp32 arithmetic (add / mul .f32x2: one
// instruction for both lanes, each rounded as its scalar form is).
NVB200_DEVICE uint64_t f32x2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
NVB200_DEVICE float2 f32x2_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
NVB200_DEVICE uint64_t f32x2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
NVB200_DEVICE uint64_t f32x2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// silu(g) rounded to bf16, as an fp32 value, by the exact expression (the fallback of the fast path).
NVB200_DEVICE float silu_bf16_exact(float g) {
  return bf16_lo(__bfloat16_as_ushort(__float2bfloat16_rn(g / (1.0f + expf(-g)))));
}

// Eight gate and eight up values (bf16) -> eight outputs: silu rounded to bf16, times up, rounded once
// (mul.rn.bf16x2: the product of two bf16 values is exact in fp32, so this is torch's fp32 multiply then round).
// The eight fast estimates are checked together: an estimate whose low 16 bits lie within kSiluMargin of 0x8000
// (test: (b - (0x8000 - margin)) mod 2^16 <= 2 margin) sends the thread through the exact expression for the flagged
// elements, and a gate outside the fast range for all eight. Elsewhere the estimate rounds to the same bf16 as the
// exact value under round-to-nearest-even (cvt.rn.bf16x2), since no exact tie lies outside the margin.
NVB200_DEVICE uint4 silu_mul8_bf16(const uint4 &g, const uint4 &u) {
  const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, uw[4] = {u.x, u.y, u.z, u.w};
  // A gate outside the fast range (|g| > 16, or not finite) sends all eight through the check below: for each bf16
  // half h of a word, (h & 0x7fff) > 0x4180 (16.0) exactly when (h & 0x7fff) + 0x3e7f sets bit 15 (no carry crosses
  // into the other half: both terms are below 0x8000).
  uint32_t wide = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) wide |= ((gw[i] & 0x7FFF7FFFu) + 0x3E7F3E7Fu) & 0x80008000u;
  float gf[8], est[8];
  uint32_t flags = wide ? 0xFFu : 0u;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // Pairs in packed fp32 (f32x2) arithmetic: est = g * rcp(1 + 2^(-g log2 e)), two elements per instruction.
    gf[2 * i] = bf16_lo(gw[i]), gf[2 * i + 1] = bf16_hi(gw[i]);
    const uint64_t x = f32x2_pack(gf[2 * i], gf[2 * i + 1]);
    const float2 t = f32x2_unpack(f32x2_mul(x, f32x2_pack(-1.4426950408889634f, -1.4426950408889634f)));
    const uint64_t d = f32x2_add(f32x2_pack(ex2_approx_ftz(t.x), ex2_approx_ftz(t.y)), f32x2_pack(1.0f, 1.0f));
    const float2 dd = f32x2_unpack(d);
    const float2 e = f32x2_unpack(f32x2_mul(x, f32x2_pack(rcp_approx_ftz(dd.x), rcp_approx_ftz(dd.y))));
    est[2 * i] = e.x, est[2 * i + 1] = e.y;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t b = __float_as_uint(est[i]);
    flags |= static_cast<uint32_t>(((b - (0x8000u - kSiluMargin)) & 0xFFFFu) <= 2 * kSiluMargin) << i;
  }
  if (flags != 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (flags & (1u << i)) est[i] = silu_bf16_exact(gf[i]);
  }
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = bf16x2_mul(pack_bf16x2(est[2 * i], est[2 * i + 1]), uw[i]);
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// ---------------------------------------------------------------------------------------------------------------
// Shared-memory addresses and vector access.

NVB200_DEVICE uint32_t smem_addr(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

NVB200_DEVICE uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

NVB200_DEVICE float4 ld_shared_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

NVB200_DEVICE void st_shared_v4(uint32_t addr, const uint4 &v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// Warp-level bf16 MMA (m16n8k16, fp32 accumulation) and its ldmatrix fragment loads, for the small per-warp tiles of
// the decode kernels. Fragment layout (lane = 4 g + t): A (16 x 16) a0 = (g, 2t..2t+1), a1 = (g + 8, 2t..),
// a2 = (g, 2t + 8..), a3 = (g + 8, 2t + 8..); B (16 x 8) b0 = (2t..2t+1, g), b1 = (2t + 8.., g); C (16 x 8)
// c0, c1 = (g, 2t..2t+1), c2, c3 = (g + 8, 2t..2t+1).

NVB200_DEVICE void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
NVB200_DEVICE void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
NVB200_DEVICE void ldsm_x2(uint32_t addr, uint32_t (&r)[2]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}
NVB200_DEVICE void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// ---------------------------------------------------------------------------------------------------------------
// mbarrier (shared-memory transaction barrier).

NVB200_DEVICE void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes the initialised barriers visible to the async proxy (the bulk-copy engine) before first use.
NVB200_DEVICE void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

NVB200_DEVICE void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}

NVB200_DEVICE void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

NVB200_DEVICE bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

NVB200_DEVICE uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Upper bound of any single wait in these kernels. A healthy wait lasts microseconds; one second means the
// awaited copy or arrival will never come, and the kernel gives up instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 1000000000ull;

// Waits for the phase of `bar` with the given parity to complete. Returns false if it has not after
// kWaitLimitNs: the caller then records NVB200_STATUS_WAIT_TIMEOUT and winds its CTA down. The global timer is only
// read after 1024 unsuccessful polls (each poll may suspend the thread for a while), so a wait that ends normally
// never pays for a timer read.
NVB200_DEVICE bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  uint64_t start = 0;
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 1023u) == 0) {
      const uint64_t now = global_timer_ns();
      if (start == 0) start = now;
      else if (now - start > kWaitLimitNs) return false;
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// 1-D bulk copies (cp.async.bulk). Both addresses 16-byte aligned, size a multiple of 16 bytes.

// Global -> shared, completion counted on `bar` as transaction bytes.
NVB200_DEVICE void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Shared -> global, tracked in the issuing thread's bulk group.
NVB200_DEVICE void bulk_s2g(void *dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes)
               : "memory");
}

NVB200_DEVICE void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Waits until all but the N most recent bulk groups of this thread have finished READING shared memory.
template <int N> NVB200_DEVICE void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Waits until all but the N most recent bulk groups of this thread are complete (writes visible).
template <int N> NVB200_DEVICE void bulk_wait() { asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory"); }

// Orders this thread's generic-proxy shared-memory writes before later async-proxy (bulk copy) reads.
NVB200_DEVICE void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Programmatic dependent launch. launch_dependents(): the next kernel in the stream, if it was launched with
// programmatic stream serialization, may start once every CTA of this grid has executed this (or exited); a kernel
// launched in plain stream order is unaffected. grid_dependency_wait(): blocks the calling thread until the grids this
// one depends on programmatically have completed and their writes are visible (at once when there are none).
NVB200_DEVICE void launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
NVB200_DEVICE void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

NVB200_DEVICE void set_status(int32_t *status, int32_t bits) {
  if (status != nullptr) atomicOr(status, bits);
}

}  // namespace nvb200

// ---------------------------------------------------------------------------------------------------------------
// Host helpers shared by the entry points.

namespace nvb200 {

// Streaming multiprocessors of the current device (cached per device; 148 on B200).
int sm_count();

// Returns NVB200_OK if the current device is sm_100 (B200/GB200), else NVB200_ERR_NO_DEVICE.
int check_device();

// Programmatic stream serialization for the decode-path kernels that launch through launch_ex, per kernel class: 1
// lets their CTAs be scheduled while the preceding kernel finishes (when it lets its dependents start early; they
// wait for it with grid_dependency_wait() before touching memory), 0 keeps plain stream order. Measured on B200, the
// Qwen3-0.6B decode step (batch 32, context 1024, CUDA graph; the weight-streaming GEMM, which has its own switch,
// launched so in every case): all plain 1548.7 us; the norms so 1481.6 us; the fused q/k op and decode attention
// so 1645.5 us. Hence norms on, the others off.
#ifndef NVB200_PDL
#define NVB200_PDL 0
#endif
#ifndef NVB200_PDL_NORM
#define NVB200_PDL_NORM 1
#endif
#ifndef NVB200_PDL_QKNR
#define NVB200_PDL_QKNR NVB200_PDL
#endif
#ifndef NVB200_PDL_ATTN
#define NVB200_PDL_ATTN NVB200_PDL
#endif

// Launches `kernel` with cudaLaunchKernelEx: a thread-block cluster of cluster_x CTAs (1: none) and, if pdl,
// programmatic stream serialization. The kernel must call grid_dependency_wait() before its first global access.
template <typename... KArgs, typename... Args>
int launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, int cluster_x,
              bool pdl, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x, attr[n].val.clusterDim.y = 1, attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...) == cudaSuccess ? NVB200_OK : NVB200_ERR_CUDA;
}

inline int launch_status() { return cudaGetLastError() == cudaSuccess ? NVB200_OK : NVB200_ERR_CUDA; }

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace nvb200
