// Fused per-head q/k RMSNorm + neox RoPE + paged KV-cache write for sm_100a.
//
// Behaviour follows nanovllm/kernels/qk_norm_rope_kv.py:45-82 (the Triton kernel) and the torch code it replaces:
// layers/layernorm.py:20-30 (RMSNorm.rms_forward), layers/rotary_embedding.py:6-14,37-48 (apply_rotary_emb,
// RotaryEmbedding.forward) and layers/attention.py:11-31 (store_kvcache_kernel: slot -1 is skipped).
//
// Design (bulk path, used whenever every row is 16-byte aligned, i.e. always for qkv_proj views):
//   * Work unit = one token x a group of G kv heads and the G*R q heads that share them (GQA, R = Hq/Hkv).
//     Large batches use G = Hkv (one unit per token); small batches split heads so that every SM gets work.
//   * Two or three persistent CTAs per SM (by unit size) each own a contiguous range of units (one CTA per SM
//     measured 30 % slower: a single producer cannot keep enough copies in flight). Warp 0 is the producer: it
//     prefetches 32
//     positions/slots at a time with one coalesced load and moves each unit's q rows, k rows, v rows (only when
//     the slot is kept) and cos/sin row from HBM into a shared-memory stage with 1-D bulk copies
//     (cp.async.bulk, completion counted on an mbarrier). Up to 8 stages are in flight per CTA.
//   * Consumer warps (8 or 6) each own a fixed set of stages and take the units that land in them. A warp normalises and rotates 32/LPH heads per step in place in
//     shared memory, each lane holding 8 elements of the first half and the matching 8 of the second half
//     (LPH = D/16 lanes per head), so RoPE pairs are lane-local and the sum of squares needs log2(LPH) shuffles.
//   * The finished q rows go to q_out, the k rows to k_out and/or k_cache[slot], and the v rows straight from the
//     stage to v_cache[slot] with bulk stores (cp.async.bulk shared->global): v never enters registers.
// Numerics: torch's two roundings (bf16 after the normalisation, bf16 product with the weight, which equals the
// exact product rounded once) and RoPE with separately rounded fp32 products (no FMA contraction).
#include <algorithm>

#include "common.cuh"
#include "qknr_math.cuh"

namespace nvb200 {
namespace {

// Launch shapes, chosen per call by the size of a work unit (one shared-memory stage). Measured on B200 (bench.py,
// T = 8192): units of >= 11 KB (a Qwen3-8B token, 12.8 KB) run best as 2 CTAs per SM with 8 consumer warps and
// 8 stages; smaller units (a Qwen3-0.6B token, 8.7 KB) as 3 CTAs per SM with 6 consumer warps. A build may
// override the constants with -D for tuning sweeps.
#ifndef NVB200_QKNR_LARGE_CONSUMERS
#define NVB200_QKNR_LARGE_CONSUMERS 8
#endif
#ifndef NVB200_QKNR_LARGE_CTAS
#define NVB200_QKNR_LARGE_CTAS 2
#endif
#ifndef NVB200_QKNR_LARGE_STAGES
#define NVB200_QKNR_LARGE_STAGES 8
#endif
#ifndef NVB200_QKNR_SMALL_CONSUMERS
#define NVB200_QKNR_SMALL_CONSUMERS 6
#endif
#ifndef NVB200_QKNR_SMALL_CTAS
#define NVB200_QKNR_SMALL_CTAS 3
#endif
#ifndef NVB200_QKNR_SMALL_STAGES
#define NVB200_QKNR_SMALL_STAGES 8
#endif
#ifndef NVB200_QKNR_SMALL_UNIT_BYTES
#define NVB200_QKNR_SMALL_UNIT_BYTES (11 * 1024)
#endif

constexpr int kHeaderBytes = 512;  // mbarriers and per-stage slot numbers
constexpr int kMaxStagesAny = 16;
static_assert(2 * 8 * kMaxStagesAny + 4 * kMaxStagesAny <= kHeaderBytes, "header too small");
static_assert(NVB200_QKNR_LARGE_STAGES <= kMaxStagesAny && NVB200_QKNR_SMALL_STAGES <= kMaxStagesAny, "stages");

// Shared memory of a CTA when `ctas` share an SM (228 KB per SM, 1 KB reserved per CTA).
constexpr int stage_budget(int ctas) { return (228 * 1024) / ctas - 1024 - kHeaderBytes; }

struct QknrParams {
  __nv_bfloat16 *q_out;
  __nv_bfloat16 *k_out;
  const __nv_bfloat16 *q;
  const __nv_bfloat16 *k;
  const __nv_bfloat16 *v;
  int64_t q_stride, k_stride, v_stride;
  const int64_t *positions;
  const int32_t *slots;
  const __nv_bfloat16 *q_w;
  const __nv_bfloat16 *k_w;
  const float *cos_sin;
  int64_t cs_stride, num_positions;
  __nv_bfloat16 *k_cache;
  __nv_bfloat16 *v_cache;
  int64_t num_slots;
  int64_t num_tokens;
  int hq, hkv;
  int splits;       // units per token (S)
  int g;            // kv heads per unit (G = Hkv / S)
  int r;            // q heads per kv head (R)
  int64_t units;    // T * S
  int64_t chunk;    // units per CTA
  int stages;       // pipeline depth
  int consumers;    // consumer warps in use (<= the launch shape's W); each owns stages w, w + consumers, ...
  int qkv_row;      // 1: q, k, v are consecutive in memory (one qkv_proj row per token) and a unit is a whole
                    // token, so one bulk copy moves the unit's q | k | v (v is then read for skipped slots too,
                    // as the reference's byte count assumes)
  int stage_bytes;  // bytes per stage (multiple of 128)
  int tpu;          // tokens per unit of the multi-token kernel (1 for the others)
  float eps;
  int32_t *status;
};

// Token of work unit `unit` and the head group `s` it covers; splits == 1 (large batches) needs no division, and
// otherwise the units fit 31 bits (checked on the host), so the division is a cheap 32-bit one.
NVB200_DEVICE int64_t unit_token(int64_t unit, int splits, int &s) {
  if (splits == 1) {
    s = 0;
    return unit;
  }
  const uint32_t u = static_cast<uint32_t>(unit), d = static_cast<uint32_t>(splits);
  const uint32_t t = u / d;
  s = static_cast<int>(u - t * d);
  return t;
}

// Next unit after `it` whose stage (unit % NS) belongs to the same consumer warp (stages w, w + W, w + 2W, ...).
NVB200_DEVICE int next_unit(int it, int NS, int W) {
  const int st = it % NS;
  return st + W < NS ? it + W : it - st + NS + st % W;
}

// ---------------------------------------------------------------------------------------------------------------
// Bulk-copy pipeline kernel. D in {64, 128, 256}.

template <int D, int W, int CTAS>
__global__ void __launch_bounds__(32 * (1 + W), CTAS) qknr_bulk_kernel(const __grid_constant__ QknrParams p) {
  launch_dependents();     // a dependent launched early waits for this grid before reading its output
  grid_dependency_wait();  // this grid may itself have been launched early
  constexpr int HALF = D / 2;
  constexpr int LPH = D / 16;    // lanes per head: each lane holds 8 + 8 elements
  constexpr int HPI = 32 / LPH;  // heads per warp step
  extern __shared__ __align__(128) uint8_t smem[];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NS = p.stages;
  const uint32_t bar_base = smem_addr(smem);  // full[0..NS), empty[0..NS)
  int32_t *meta = reinterpret_cast<int32_t *>(smem + 2 * 8 * kMaxStagesAny);
  const uint32_t stage_base = smem_addr(smem + kHeaderBytes);

  const int64_t first = static_cast<int64_t>(blockIdx.x) * p.chunk;
  if (first >= p.units) return;
  const int n_units = static_cast<int>(p.chunk < p.units - first ? p.chunk : p.units - first);

  const int nq = p.g * p.r;  // q heads per unit
  const uint32_t qb = nq * D * 2, kb = p.g * D * 2, csb = D * 4;
  const bool store = p.k_cache != nullptr;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(bar_base + 8 * i, 1);         // full: producer's arrive + transaction bytes
      mbar_init(bar_base + 8 * (NS + i), 1);  // empty: the consuming warp's arrive
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    // Units go in batches of 32, one position and slot per lane, loaded one batch ahead so their latency is hidden
    // after the first batch. Per unit, lane 0 waits for the stage, issues the q/k/v copies (they do not depend on
    // the position), then the cos/sin copy and the arrive that sets the stage's byte count (copies may complete
    // before it: the count may go negative in between).
    const uint32_t v_bytes = store ? kb : 0;  // v is only read when the cache is written
    bool abort = false;
    int64_t pos_next = 0;
    int32_t slot_next = -1;
    if (lane < n_units) {
      int s_;
      const int64_t t = unit_token(first + lane, p.splits, s_);
      pos_next = __ldg(p.positions + t);
      if (store) slot_next = __ldg(p.slots + t);
    }
    for (int base = 0; base < n_units && !abort; base += 32) {
      const int64_t pos = pos_next;
      const int32_t slot = slot_next;
      if (base + 32 + lane < n_units) {
        int s_;
        const int64_t t = unit_token(first + base + 32 + lane, p.splits, s_);
        pos_next = __ldg(p.positions + t);
        if (store) slot_next = __ldg(p.slots + t);
      }
      const int cnt = min(32, n_units - base);
      for (int j = 0; j < cnt; ++j) {
        const int it = base + j;
        const int st = it % NS;
        const uint32_t full = bar_base + 8 * st, empty = bar_base + 8 * (NS + st);
        const uint32_t sb = stage_base + st * p.stage_bytes;
        if (lane == 0) {
          if (!mbar_wait_bounded(empty, ((it / NS) & 1) ^ 1)) {
            set_status(p.status, NVB200_STATUS_WAIT_TIMEOUT);
            abort = true;
          } else {
            const int64_t unit = first + it;
            int s;
            const int64_t t = unit_token(unit, p.splits, s);
            if (p.qkv_row) {
              bulk_g2s(sb, p.q + t * p.q_stride, qb + 2 * kb, full);
            } else {
              bulk_g2s(sb, p.q + t * p.q_stride + static_cast<int64_t>(s) * nq * D, qb, full);
              bulk_g2s(sb + qb, p.k + t * p.k_stride + static_cast<int64_t>(s) * p.g * D, kb, full);
              if (v_bytes) bulk_g2s(sb + qb + kb, p.v + t * p.v_stride + static_cast<int64_t>(s) * p.g * D, kb, full);
            }
          }
        }
        abort = __shfl_sync(0xffffffffu, abort, 0);
        if (abort) break;
        int64_t pj = __shfl_sync(0xffffffffu, pos, j);
        int32_t sj = __shfl_sync(0xffffffffu, slot, j);
        if (lane == 0) {
          if (pj < 0 || pj >= p.num_positions) {
            set_status(p.status, NVB200_STATUS_BAD_POSITION);
            pj = 0;
          }
          if (sj < -1 || sj >= p.num_slots) {
            set_status(p.status, NVB200_STATUS_BAD_SLOT);
            sj = -1;
          }
          meta[st] = sj;
          mbar_arrive_expect_tx(full, qb + kb + v_bytes + csb);
          bulk_g2s(sb + qb + 2 * kb, p.cos_sin + pj * p.cs_stride, csb, full);
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------------- consumers
  const int cw = warp - 1;
  const int j = lane % LPH;   // 8-element column block inside each half
  const int hl = lane / LPH;  // head within the warp step
  uint32_t wq1[4], wq2[4], wk1[4], wk2[4];
  load_w8(p.q_w + 8 * j, wq1);
  load_w8(p.q_w + HALF + 8 * j, wq2);
  load_w8(p.k_w + 8 * j, wk1);
  load_w8(p.k_w + HALF + 8 * j, wk2);
  const int total = nq + p.g;

  // Warp cw owns stages cw, cw + W, ... and consumes exactly the units that land in them, in order. Every waiter
  // of a stage's full barrier thus sees each of its phases, which the parity wait requires (a warp that could run
  // two phases ahead of a stage would read a parity that aliases an older phase).
  const int nw = p.consumers;
  if (cw >= nw) return;
  for (int it = cw; it < n_units; it = next_unit(it, NS, nw)) {
    const int st = it % NS;
    const uint32_t ph = (it / NS) & 1;
    const uint32_t full = bar_base + 8 * st, empty = bar_base + 8 * (NS + st);
    if (!mbar_wait_bounded(full, ph)) {
      if (lane == 0) set_status(p.status, NVB200_STATUS_WAIT_TIMEOUT);
      break;
    }
    const int32_t slot = meta[st];
    const uint32_t sb = stage_base + st * p.stage_bytes;
    const uint32_t sq = sb, sk = sb + qb, sv = sb + qb + kb, scs = sb + qb + 2 * kb;

    float c[8], s[8];
    {
      const float4 c0 = ld_shared_f4(scs + 32 * j), c1 = ld_shared_f4(scs + 32 * j + 16);
      const float4 s0 = ld_shared_f4(scs + 4 * HALF + 32 * j), s1 = ld_shared_f4(scs + 4 * HALF + 32 * j + 16);
      c[0] = c0.x, c[1] = c0.y, c[2] = c0.z, c[3] = c0.w, c[4] = c1.x, c[5] = c1.y, c[6] = c1.z, c[7] = c1.w;
      s[0] = s0.x, s[1] = s0.y, s[2] = s0.z, s[3] = s0.w, s[4] = s1.x, s[5] = s1.y, s[6] = s1.z, s[7] = s1.w;
    }

    for (int h0 = 0; h0 < total; h0 += HPI) {
      const int h = h0 + hl;
      const bool active = h < total;
      const bool isq = h < nq;
      const uint32_t row = active ? (isq ? sq + h * D * 2 : sk + (h - nq) * D * 2) : sq;
      const uint4 a = ld_shared_v4(row + 16 * j);
      const uint4 b = ld_shared_v4(row + 2 * HALF + 16 * j);
      float x1[8], x2[8];
      unpack8(a, x1);
      unpack8(b, x2);
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(x1[i], x1[i], ss);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(x2[i], x2[i], ss);
#pragma unroll
      for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rstd = rsqrtf(ss / static_cast<float>(D) + p.eps);
      uint32_t w1[4], w2[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        w1[i] = isq ? wq1[i] : wk1[i];
        w2[i] = isq ? wq2[i] : wk2[i];
      }
      float y1[8], y2[8];
      norm_rope8(x1, x2, rstd, w1, w2, c, s, y1, y2);
      if (active) {
        st_shared_v4(row + 16 * j, pack8(y1));
        st_shared_v4(row + 2 * HALF + 16 * j, pack8(y2));
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      const int64_t unit = first + it;
      // The 64-bit division here is deliberate: this form, and equally a non-inlined call in its place, measured
      // 5.8 TB/s on the Qwen3-8B shape at T = 8192 against 4.6 TB/s for the inlined division-free mapping that
      // the producer uses (B200, same launch shape); the call boundary changes how the compiler schedules the
      // consumer loop, and explicit delays of 32-512 cycles at this point did not reproduce the gain.
      const int64_t t = unit / p.splits;
      const int sp = static_cast<int>(unit % p.splits);
      bulk_s2g(p.q_out + (t * p.hq + static_cast<int64_t>(sp) * nq) * D, sq, qb);
      if (p.k_out) bulk_s2g(p.k_out + (t * p.hkv + static_cast<int64_t>(sp) * p.g) * D, sk, kb);
      if (slot >= 0) {
        const int64_t off = (static_cast<int64_t>(slot) * p.hkv + static_cast<int64_t>(sp) * p.g) * D;
        bulk_s2g(p.k_cache + off, sk, kb);
        bulk_s2g(p.v_cache + off, sv, kb);
      }
      bulk_commit();
      bulk_wait_read<0>();  // the stores have read the stage: hand it back to the producer
      mbar_arrive(empty);
    }
    __syncwarp();
  }
  // Stores still in flight may finish after the CTA exits; their shared-memory reads are done (waited above).
}

// ---------------------------------------------------------------------------------------------------------------
// Multi-token bulk kernel: the same pipeline with a unit of B consecutive tokens, for shards whose tokens are small
// (a tensor-parallel rank's 1-4 kv heads: 2-6.5 KB per token), where one token per unit would spend as much time
// on per-unit barrier and issue work as on moving bytes. It needs q | k | v consecutive in one qkv_proj row per
// token and consecutive rows (the layout of a rank's qkv_proj output), so the producer moves a unit's B rows with
// one bulk copy (q | k per token when the cache is not written). Stage layout: B rows of qb + 2 kb bytes (the v
// slot unused without a cache), then B cos/sin rows. Positions and slots are loaded 32 tokens at a time, one
// batch ahead; lane i of the producer issues the cos/sin copy of the unit's token i.

constexpr int kMultiMaxTpu = 16;                    // tokens per unit (a power of two)
#ifndef NVB200_QKNR_MULTI_UNIT_BYTES
#define NVB200_QKNR_MULTI_UNIT_BYTES (18 * 1024)
#endif
constexpr int64_t kMultiUnitBytes = NVB200_QKNR_MULTI_UNIT_BYTES;  // largest multi-token unit
constexpr int kMultiHeader = 256 + 4 * kMaxStagesAny * kMultiMaxTpu;  // barriers + per-stage slot numbers
constexpr int multi_stage_budget(int ctas) { return (228 * 1024) / ctas - 1024 - kMultiHeader; }

template <int D, int W, int CTAS>
__global__ void __launch_bounds__(32 * (1 + W), CTAS) qknr_multi_kernel(const __grid_constant__ QknrParams p) {
  launch_dependents();     // a dependent launched early waits for this grid before reading its output
  grid_dependency_wait();  // this grid may itself have been launched early
  constexpr int HALF = D / 2;
  constexpr int LPH = D / 16;    // lanes per head: each lane holds 8 + 8 elements
  constexpr int HPI = 32 / LPH;  // heads per warp step
  extern __shared__ __align__(128) uint8_t smem[];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NS = p.stages;
  const int B = p.tpu;
  const uint32_t bar_base = smem_addr(smem);  // full[0..NS), empty[0..NS)
  int32_t *meta = reinterpret_cast<int32_t *>(smem + 256);  // slot of token i of stage st at st * kMultiMaxTpu + i
  const uint32_t stage_base = smem_addr(smem + kMultiHeader);

  const int64_t first = static_cast<int64_t>(blockIdx.x) * p.chunk;  // first unit of this CTA
  if (first >= p.units) return;
  const int n_units = static_cast<int>(p.chunk < p.units - first ? p.chunk : p.units - first);
  const int64_t t_first = first * B;
  const int64_t t_end = (first + n_units) * B < p.num_tokens ? (first + n_units) * B : p.num_tokens;

  const int nq = p.hq;  // a unit holds every head of its tokens
  const uint32_t qb = nq * D * 2, kb = p.hkv * D * 2, csb = D * 4;
  const uint32_t row_stage = qb + 2 * kb;
  const bool store = p.k_cache != nullptr;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(bar_base + 8 * i, 1);
      mbar_init(bar_base + 8 * (NS + i), 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    const int upb = 32 / B;  // units per batch of 32 tokens
    bool abort = false;
    int64_t pos_next = 0;
    int32_t slot_next = -1;
    if (t_first + lane < t_end) {
      pos_next = __ldg(p.positions + t_first + lane);
      if (store) slot_next = __ldg(p.slots + t_first + lane);
    }
    for (int base = 0; base < n_units && !abort; base += upb) {
      const int64_t pos = pos_next;
      const int32_t slot = slot_next;
      const int64_t tn = t_first + static_cast<int64_t>(base + upb) * B + lane;
      if (tn < t_end) {
        pos_next = __ldg(p.positions + tn);
        if (store) slot_next = __ldg(p.slots + tn);
      }
      const int cnt = min(upb, n_units - base);
      for (int jj = 0; jj < cnt; ++jj) {
        const int it = base + jj;
        const int st = it % NS;
        const uint32_t full = bar_base + 8 * st, empty = bar_base + 8 * (NS + st);
        const uint32_t sb = stage_base + st * p.stage_bytes;
        const int64_t t0 = t_first + static_cast<int64_t>(it) * B;
        const int nt = static_cast<int>(B < t_end - t0 ? B : t_end - t0);
        if (lane == 0) {
          if (!mbar_wait_bounded(empty, ((it / NS) & 1) ^ 1)) {
            set_status(p.status, NVB200_STATUS_WAIT_TIMEOUT);
            abort = true;
          } else if (store) {
            bulk_g2s(sb, p.q + t0 * p.q_stride, nt * row_stage, full);
          } else {
            for (int i = 0; i < nt; ++i) bulk_g2s(sb + i * row_stage, p.q + (t0 + i) * p.q_stride, qb + kb, full);
          }
        }
        abort = __shfl_sync(0xffffffffu, abort, 0);
        if (abort) break;
        const int src = jj * B + (lane < B ? lane : 0);
        int64_t pj = __shfl_sync(0xffffffffu, pos, src);
        int32_t sj = __shfl_sync(0xffffffffu, slot, src);
        if (lane < nt) {
          if (pj < 0 || pj >= p.num_positions) {
            set_status(p.status, NVB200_STATUS_BAD_POSITION);
            pj = 0;
          }
          if (sj < -1 || sj >= p.num_slots) {
            set_status(p.status, NVB200_STATUS_BAD_SLOT);
            sj = -1;
          }
          meta[st * kMultiMaxTpu + lane] = sj;
        }
        __syncwarp();  // the slot numbers are written before lane 0's arrive releases the stage
        if (lane == 0) mbar_arrive_expect_tx(full, nt * ((store ? row_stage : qb + kb) + csb));
        if (lane < nt) bulk_g2s(sb + B * row_stage + lane * csb, p.cos_sin + pj * p.cs_stride, csb, full);
      }
    }
    return;
  }

  // -------------------------------------------------------------------- consumers
  const int cw = warp - 1;
  const int j = lane % LPH;   // 8-element column block inside each half
  const int hl = lane / LPH;  // head within the warp step
  uint32_t wq1[4], wq2[4], wk1[4], wk2[4];
  load_w8(p.q_w + 8 * j, wq1);
  load_w8(p.q_w + HALF + 8 * j, wq2);
  load_w8(p.k_w + 8 * j, wk1);
  load_w8(p.k_w + HALF + 8 * j, wk2);
  const int total = nq + p.hkv;

  // Warp cw owns stages cw, cw + W, ... (every waiter of a stage's full barrier sees each of its phases).
  const int nw = p.consumers;
  if (cw >= nw) return;
  for (int it = cw; it < n_units; it = next_unit(it, NS, nw)) {
    const int st = it % NS;
    const uint32_t full = bar_base + 8 * st, empty = bar_base + 8 * (NS + st);
    if (!mbar_wait_bounded(full, (it / NS) & 1)) {
      if (lane == 0) set_status(p.status, NVB200_STATUS_WAIT_TIMEOUT);
      break;
    }
    const uint32_t sb = stage_base + st * p.stage_bytes;
    const int64_t t0 = t_first + static_cast<int64_t>(it) * B;
    const int nt = static_cast<int>(B < t_end - t0 ? B : t_end - t0);
    // The unit's (token, head) pairs in order, HPI per warp step: a token's heads need not fill a step (a rank with
    // one kv head has 5 per token), so steps run across token boundaries. (ti, hi): this lane group's pair.
    const int nflat = nt * total;
    int ti = 0, hi = hl;
    while (hi >= total) hi -= total, ++ti;
    for (int f0 = 0; f0 < nflat; f0 += HPI) {
      const bool active = f0 + hl < nflat;
      const int i = active ? ti : 0;
      const bool isq = hi < nq;
      const uint32_t sq = sb + i * row_stage;
      const uint32_t row = active ? (isq ? sq + hi * D * 2 : sq + qb + (hi - nq) * D * 2) : sq;
      const uint32_t scs = sb + B * row_stage + i * csb;
      float c[8], s[8];
      {
        const float4 c0 = ld_shared_f4(scs + 32 * j), c1 = ld_shared_f4(scs + 32 * j + 16);
        const float4 s0 = ld_shared_f4(scs + 4 * HALF + 32 * j), s1 = ld_shared_f4(scs + 4 * HALF + 32 * j + 16);
        c[0] = c0.x, c[1] = c0.y, c[2] = c0.z, c[3] = c0.w, c[4] = c1.x, c[5] = c1.y, c[6] = c1.z, c[7] = c1.w;
        s[0] = s0.x, s[1] = s0.y, s[2] = s0.z, s[3] = s0.w, s[4] = s1.x, s[5] = s1.y, s[6] = s1.z, s[7] = s1.w;
      }
      const uint4 a = ld_shared_v4(row + 16 * j);
      const uint4 b = ld_shared_v4(row + 2 * HALF + 16 * j);
      float x1[8], x2[8];
      unpack8(a, x1);
      unpack8(b, x2);
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(x1[e], x1[e], ss);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(x2[e], x2[e], ss);
#pragma unroll
      for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rstd = rsqrtf(ss / static_cast<float>(D) + p.eps);
      uint32_t w1[4], w2[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        w1[e] = isq ? wq1[e] : wk1[e];
        w2[e] = isq ? wq2[e] : wk2[e];
      }
      float y1[8], y2[8];
      norm_rope8(x1, x2, rstd, w1, w2, c, s, y1, y2);
      if (active) {
        st_shared_v4(row + 16 * j, pack8(y1));
        st_shared_v4(row + 2 * HALF + 16 * j, pack8(y2));
      }
      hi += HPI;
      while (hi >= total) hi -= total, ++ti;
    }
    fence_proxy_async_smem();
    __syncwarp();
    // Lane i issues token i's stores (q_out, k_out, the k and v cache rows), so the unit's bulk stores go out in
    // parallel rather than one after another from one lane; each lane then waits until its stores have read the
    // stage, and lane 0 hands the stage back once every lane has.
    if (lane < nt) {
      const int64_t t = t0 + lane;
      const uint32_t sq = sb + lane * row_stage;
      bulk_s2g(p.q_out + t * p.hq * D, sq, qb);
      if (p.k_out) bulk_s2g(p.k_out + t * p.hkv * D, sq + qb, kb);
      const int32_t slot = meta[st * kMultiMaxTpu + lane];
      if (slot >= 0) {
        const int64_t off = static_cast<int64_t>(slot) * p.hkv * D;
        bulk_s2g(p.k_cache + off, sq + qb, kb);
        bulk_s2g(p.v_cache + off, sq + qb + kb, kb);
      }
      bulk_commit();
      bulk_wait_read<0>();
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty);  // every lane's stores have read the stage: hand it back to the producer
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Direct kernel for small batches (decode): no staging, so the latency is one position load and the cos/sin row
// behind it, in parallel with the q/k/v loads. One warp handles 32/LPH heads of one token with the bulk consumer's
// lane layout (8 + 8 elements per lane, 16-byte loads and stores); the warps of a CTA cover a token's q heads,
// then its k heads, each k-head lane group also copying its v row to the cache. Same 16-byte alignment
// requirements as the bulk kernel.

constexpr int kDirectWarps = 4;
#ifndef NVB200_QKNR_DIRECT_MAX_TOKENS
#define NVB200_QKNR_DIRECT_MAX_TOKENS 512
#endif
constexpr int64_t kDirectMaxTokens = NVB200_QKNR_DIRECT_MAX_TOKENS;
// Batches whose q/k/v rows total at most this many bytes also take the direct kernel when the multi-token kernel does
// not apply. Measured on B200 (L2 flushed): Qwen3-8B shape T = 1024 / 2048: 11.9 / 15.3 us direct vs 13.6 / 16.2 us
// bulk; T = 4096 (50 MB): 23.7 vs 22.5 us; Qwen3-0.6B shape T = 4096 (34 MB): 17.5 vs 18.3 us, T = 8192: 28.9 vs
// 26.0 us. Beyond a few tens of MB the persistent bulk pipeline keeps more bytes in flight than one-shot CTAs do.
#ifndef NVB200_QKNR_DIRECT_MAX_BYTES
#define NVB200_QKNR_DIRECT_MAX_BYTES (40LL << 20)
#endif
constexpr int64_t kDirectMaxBytes = NVB200_QKNR_DIRECT_MAX_BYTES;

template <int D>
__global__ void __launch_bounds__(32 * kDirectWarps) qknr_direct_kernel(const __grid_constant__ QknrParams p) {
  launch_dependents();     // a dependent launched early waits for this grid before reading its output
  grid_dependency_wait();  // this grid may itself have been launched early
  constexpr int HALF = D / 2;
  constexpr int LPH = D / 16;
  constexpr int HPI = 32 / LPH;
  const int lane = threadIdx.x & 31;
  const int j = lane % LPH;
  const int64_t t = blockIdx.x;
  const int h = (blockIdx.y * kDirectWarps + (threadIdx.x >> 5)) * HPI + lane / LPH;
  const int total = p.hq + p.hkv;
  if (h >= total) return;  // whole head groups drop out; the row reduction below stays within a head's lanes
  const bool isq = h < p.hq;
  const int hk = h - p.hq;
  int64_t pos = __ldg(p.positions + t);
  int32_t slot = -1;
  if (!isq && p.k_cache != nullptr) slot = __ldg(p.slots + t);
  const __nv_bfloat16 *x = isq ? p.q + t * p.q_stride + static_cast<int64_t>(h) * D
                               : p.k + t * p.k_stride + static_cast<int64_t>(hk) * D;
  const uint4 xa = __ldg(reinterpret_cast<const uint4 *>(x + 8 * j));
  const uint4 xb = __ldg(reinterpret_cast<const uint4 *>(x + HALF + 8 * j));
  uint32_t w1[4], w2[4];
  load_w8((isq ? p.q_w : p.k_w) + 8 * j, w1);
  load_w8((isq ? p.q_w : p.k_w) + HALF + 8 * j, w2);
  uint4 va = make_uint4(0, 0, 0, 0), vb = va;
  const bool kv_store = !isq && p.k_cache != nullptr;
  if (kv_store) {
    const __nv_bfloat16 *vr = p.v + t * p.v_stride + static_cast<int64_t>(hk) * D;
    va = __ldg(reinterpret_cast<const uint4 *>(vr + 8 * j));
    vb = __ldg(reinterpret_cast<const uint4 *>(vr + HALF + 8 * j));
  }
  if (pos < 0 || pos >= p.num_positions) {
    if (j == 0) set_status(p.status, NVB200_STATUS_BAD_POSITION);
    pos = 0;
  }
  const float *cs = p.cos_sin + pos * p.cs_stride;
  float c[8], sn[8];
  {
    const float4 c0 = __ldg(reinterpret_cast<const float4 *>(cs + 8 * j));
    const float4 c1 = __ldg(reinterpret_cast<const float4 *>(cs + 8 * j + 4));
    const float4 s0 = __ldg(reinterpret_cast<const float4 *>(cs + HALF + 8 * j));
    const float4 s1 = __ldg(reinterpret_cast<const float4 *>(cs + HALF + 8 * j + 4));
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
  // The lanes of one head are LPH consecutive lanes; heads past `total` left whole groups, so the xor partners of
  // every live lane are live.
  const unsigned group_mask = LPH == 32 ? 0xffffffffu : (((1u << LPH) - 1u) << (lane / LPH * LPH));
#pragma unroll
  for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(group_mask, ss, o);
  const float rstd = rsqrtf(ss / static_cast<float>(D) + p.eps);
  float y1[8], y2[8];
  norm_rope8(x1, x2, rstd, w1, w2, c, sn, y1, y2);
  const uint4 ya = pack8(y1), yb = pack8(y2);
  if (isq) {
    __nv_bfloat16 *o = p.q_out + (t * p.hq + h) * D;
    *reinterpret_cast<uint4 *>(o + 8 * j) = ya;
    *reinterpret_cast<uint4 *>(o + HALF + 8 * j) = yb;
    return;
  }
  if (p.k_out) {
    __nv_bfloat16 *o = p.k_out + (t * p.hkv + hk) * D;
    *reinterpret_cast<uint4 *>(o + 8 * j) = ya;
    *reinterpret_cast<uint4 *>(o + HALF + 8 * j) = yb;
  }
  if (kv_store) {
    if (slot < -1 || slot >= p.num_slots) {
      if (j == 0) set_status(p.status, NVB200_STATUS_BAD_SLOT);
      slot = -1;
    }
    if (slot >= 0) {
      const int64_t off = (static_cast<int64_t>(slot) * p.hkv + hk) * D;
      *reinterpret_cast<uint4 *>(p.k_cache + off + 8 * j) = ya;
      *reinterpret_cast<uint4 *>(p.k_cache + off + HALF + 8 * j) = yb;
      *reinterpret_cast<uint4 *>(p.v_cache + off + 8 * j) = va;
      *reinterpret_cast<uint4 *>(p.v_cache + off + HALF + 8 * j) = vb;
    }
  }
}

template <int D> int launch_direct(QknrParams &p, cudaStream_t stream) {
  constexpr int heads_per_cta = kDirectWarps * (32 / (D / 16));
  const dim3 grid(static_cast<unsigned>(p.num_tokens), (p.hq + p.hkv + heads_per_cta - 1) / heads_per_cta);
  return launch_ex(qknr_direct_kernel<D>, grid, dim3(32 * kDirectWarps), 0, stream, 1, NVB200_PDL_QKNR, p);
}

// ---------------------------------------------------------------------------------------------------------------
// Generic kernel for layouts the bulk engine cannot move (a row not 16-byte aligned, or D outside {64,128,256}).
// One warp per (token, head); lane i holds the RoPE pairs (i, i + D/2), (i + 32, i + 32 + D/2), ...

constexpr int kGenericWarps = 4;
constexpr int kGenericMaxPairs = 8;  // D <= 512

__global__ void __launch_bounds__(32 * kGenericWarps) qknr_generic_kernel(const __grid_constant__ QknrParams p,
                                                                          int D) {
  launch_dependents();     // a dependent launched early waits for this grid before reading its output
  grid_dependency_wait();  // this grid may itself have been launched early
  const int lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x;
  const int h = blockIdx.y * kGenericWarps + (threadIdx.x >> 5);
  if (h >= p.hq + p.hkv) return;
  const int HALF = D / 2;
  const bool isq = h < p.hq;
  const int hk = h - p.hq;
  const __nv_bfloat16 *x = isq ? p.q + t * p.q_stride + static_cast<int64_t>(h) * D
                               : p.k + t * p.k_stride + static_cast<int64_t>(hk) * D;
  const __nv_bfloat16 *w = isq ? p.q_w : p.k_w;

  int64_t pos = p.positions[t];
  if (pos < 0 || pos >= p.num_positions) {
    if (lane == 0) set_status(p.status, NVB200_STATUS_BAD_POSITION);
    pos = 0;
  }
  const float *cs = p.cos_sin + pos * p.cs_stride;

  float x1[kGenericMaxPairs], x2[kGenericMaxPairs];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kGenericMaxPairs; ++k) {
    const int i = lane + 32 * k;
    x1[k] = x2[k] = 0.f;
    if (i < HALF) {
      x1[k] = __bfloat162float(x[i]);
      x2[k] = __bfloat162float(x[i + HALF]);
      ss = fmaf(x1[k], x1[k], ss);
      ss = fmaf(x2[k], x2[k], ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rstd = rsqrtf(ss / static_cast<float>(D) + p.eps);

  int32_t slot = -1;
  if (!isq && p.k_cache != nullptr) {
    slot = p.slots[t];
    if (slot < -1 || slot >= p.num_slots) {
      if (lane == 0) set_status(p.status, NVB200_STATUS_BAD_SLOT);
      slot = -1;
    }
  }
#pragma unroll
  for (int k = 0; k < kGenericMaxPairs; ++k) {
    const int i = lane + 32 * k;
    if (i >= HALF) break;
    const float n1 = __bfloat162float(__hmul(__float2bfloat16_rn(__fmul_rn(x1[k], rstd)), w[i]));
    const float n2 = __bfloat162float(__hmul(__float2bfloat16_rn(__fmul_rn(x2[k], rstd)), w[i + HALF]));
    const float c = cs[i], s = cs[i + HALF];
    const __nv_bfloat16 y1 = __float2bfloat16_rn(__fsub_rn(__fmul_rn(n1, c), __fmul_rn(n2, s)));
    const __nv_bfloat16 y2 = __float2bfloat16_rn(__fadd_rn(__fmul_rn(n2, c), __fmul_rn(n1, s)));
    if (isq) {
      __nv_bfloat16 *o = p.q_out + (t * p.hq + h) * D;
      o[i] = y1;
      o[i + HALF] = y2;
    } else {
      if (p.k_out) {
        __nv_bfloat16 *o = p.k_out + (t * p.hkv + hk) * D;
        o[i] = y1;
        o[i + HALF] = y2;
      }
      if (slot >= 0) {
        const int64_t off = (static_cast<int64_t>(slot) * p.hkv + hk) * D;
        p.k_cache[off + i] = y1;
        p.k_cache[off + i + HALF] = y2;
      }
    }
  }
  if (slot >= 0) {
    const __nv_bfloat16 *vr = p.v + t * p.v_stride + static_cast<int64_t>(hk) * D;
    __nv_bfloat16 *vo = p.v_cache + (static_cast<int64_t>(slot) * p.hkv + hk) * D;
    for (int i = lane; i < D; i += 32) vo[i] = vr[i];
  }
}

template <int D, int W, int CTAS, int MAX_STAGES>
int launch_bulk(QknrParams &p, int sms, cudaStream_t stream) {
  constexpr int budget = stage_budget(CTAS);
  p.stages = std::min(MAX_STAGES, budget / p.stage_bytes);
  if (p.stages < 2) return NVB200_ERR_UNSUPPORTED;  // a unit larger than half the budget: too many heads
  p.consumers = std::min(W, p.stages);
  p.stages -= p.stages % p.consumers;  // every consumer warp owns the same number of stages
  const int smem = kHeaderBytes + p.stages * p.stage_bytes;
  static int configured[64] = {0};  // per device: max dynamic shared memory raised once
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(qknr_bulk_kernel<D, W, CTAS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kHeaderBytes + budget) != cudaSuccess)
      return NVB200_ERR_CUDA;
    configured[dev] = 1;
  }
  const int64_t grid = std::min<int64_t>(p.units, static_cast<int64_t>(sms) * CTAS);
  p.chunk = (p.units + grid - 1) / grid;
  const int64_t blocks = (p.units + p.chunk - 1) / p.chunk;
  return launch_ex(qknr_bulk_kernel<D, W, CTAS>, dim3(static_cast<unsigned>(blocks)), dim3(32 * (1 + W)), smem,
                   stream, 1, NVB200_PDL_QKNR, p);
}

template <int D, int W, int CTAS, int MAX_STAGES>
int launch_multi(QknrParams &p, int sms, cudaStream_t stream) {
  constexpr int budget = multi_stage_budget(CTAS);
  p.stages = std::min(MAX_STAGES, budget / p.stage_bytes);
  if (p.stages < 2) return NVB200_ERR_UNSUPPORTED;
  p.consumers = std::min(W, p.stages);
  p.stages -= p.stages % p.consumers;
  const int smem = kMultiHeader + p.stages * p.stage_bytes;
  static int configured[64] = {0};  // per device: max dynamic shared memory raised once
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(qknr_multi_kernel<D, W, CTAS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kMultiHeader + budget) != cudaSuccess)
      return NVB200_ERR_CUDA;
    configured[dev] = 1;
  }
  const int64_t grid = std::min<int64_t>(p.units, static_cast<int64_t>(sms) * CTAS);
  p.chunk = (p.units + grid - 1) / grid;
  const int64_t blocks = (p.units + p.chunk - 1) / p.chunk;
  return launch_ex(qknr_multi_kernel<D, W, CTAS>, dim3(static_cast<unsigned>(blocks)), dim3(32 * (1 + W)), smem,
                   stream, 1, NVB200_PDL_QKNR, p);
}

template <int D> int launch_multi_shaped(QknrParams &p, int sms, cudaStream_t stream) {
  if (p.stage_bytes >= NVB200_QKNR_SMALL_UNIT_BYTES)
    return launch_multi<D, NVB200_QKNR_LARGE_CONSUMERS, NVB200_QKNR_LARGE_CTAS, NVB200_QKNR_LARGE_STAGES>(p, sms, stream);
  return launch_multi<D, NVB200_QKNR_SMALL_CONSUMERS, NVB200_QKNR_SMALL_CTAS, NVB200_QKNR_SMALL_STAGES>(p, sms, stream);
}

template <int D> int launch_bulk_shaped(QknrParams &p, int sms, cudaStream_t stream) {
  if (p.stage_bytes >= NVB200_QKNR_SMALL_UNIT_BYTES)
    return launch_bulk<D, NVB200_QKNR_LARGE_CONSUMERS, NVB200_QKNR_LARGE_CTAS, NVB200_QKNR_LARGE_STAGES>(p, sms, stream);
  return launch_bulk<D, NVB200_QKNR_SMALL_CONSUMERS, NVB200_QKNR_SMALL_CTAS, NVB200_QKNR_SMALL_STAGES>(p, sms, stream);
}

}  // namespace

// Checks the arguments and launches the kernel the sizes and layout call for. With `plan` non-null nothing is
// launched: the kernel that would run is written to plan[0] (an NVB200_QKNR_KERNEL_* code) and its tokens per work
// unit to plan[1].
int qk_norm_rope_kv_launch(const nvb200_qk_norm_rope_kv_args *a, cudaStream_t stream, int32_t *plan) {
  if (a == nullptr) return NVB200_ERR_ARG;
  const int64_t T = a->num_tokens;
  const int hq = a->num_q_heads, hkv = a->num_kv_heads, D = a->head_dim;
  if (T < 0 || hq <= 0 || hkv <= 0 || D <= 0 || hq % hkv != 0 || D % 2 != 0) return NVB200_ERR_ARG;
  if (D > 2 * 32 * kGenericMaxPairs) return NVB200_ERR_UNSUPPORTED;
  if (plan) plan[0] = NVB200_QKNR_KERNEL_NONE, plan[1] = 0;
  if (T == 0) return NVB200_OK;
  const bool store = a->k_cache != nullptr || a->v_cache != nullptr;
  if (!a->q_out || !a->q || !a->k || !a->positions || !a->q_weight || !a->k_weight || !a->cos_sin) return NVB200_ERR_ARG;
  if (store && (!a->k_cache || !a->v_cache || !a->slot_mapping || !a->v || a->num_slots <= 0)) return NVB200_ERR_ARG;
  if (a->num_positions <= 0 || a->cos_sin_stride < D) return NVB200_ERR_ARG;
  if (int rc = check_device()) return rc;

  QknrParams p{};
  p.q_out = static_cast<__nv_bfloat16 *>(a->q_out);
  p.k_out = static_cast<__nv_bfloat16 *>(a->k_out);
  p.q = static_cast<const __nv_bfloat16 *>(a->q);
  p.k = static_cast<const __nv_bfloat16 *>(a->k);
  p.v = static_cast<const __nv_bfloat16 *>(a->v);
  p.q_stride = a->q_token_stride;
  p.k_stride = a->k_token_stride;
  p.v_stride = a->v_token_stride;
  p.positions = a->positions;
  p.slots = store ? a->slot_mapping : nullptr;
  p.q_w = static_cast<const __nv_bfloat16 *>(a->q_weight);
  p.k_w = static_cast<const __nv_bfloat16 *>(a->k_weight);
  p.cos_sin = a->cos_sin;
  p.cs_stride = a->cos_sin_stride;
  p.num_positions = a->num_positions;
  p.k_cache = store ? static_cast<__nv_bfloat16 *>(a->k_cache) : nullptr;
  p.v_cache = store ? static_cast<__nv_bfloat16 *>(a->v_cache) : nullptr;
  p.num_slots = store ? a->num_slots : 0;
  p.num_tokens = T;
  p.hq = hq;
  p.hkv = hkv;
  p.r = hq / hkv;
  p.eps = a->eps;
  p.status = a->status;

  const bool rows16 = (a->q_token_stride * 2) % 16 == 0 && (a->k_token_stride * 2) % 16 == 0 &&
                      (!store || (a->v_token_stride * 2) % 16 == 0) && (a->cos_sin_stride * 4) % 16 == 0;
  const bool ptrs16 = aligned16(a->q_out) && aligned16(a->k_out) && aligned16(a->q) && aligned16(a->k) &&
                      aligned16(a->v) && aligned16(a->cos_sin) && aligned16(a->q_weight) &&
                      aligned16(a->k_weight) && aligned16(a->k_cache) && aligned16(a->v_cache);
  const bool bulk = (D == 64 || D == 128 || D == 256) && rows16 && ptrs16;

  if (!bulk) {
    p.splits = 1;
    p.g = hkv;
    dim3 grid(static_cast<unsigned>(T), (hq + hkv + kGenericWarps - 1) / kGenericWarps);
    if (T > 0x7fffffffLL) return NVB200_ERR_UNSUPPORTED;
    if (plan) {
      plan[0] = NVB200_QKNR_KERNEL_GENERIC, plan[1] = 1;
      return NVB200_OK;
    }
    qknr_generic_kernel<<<grid, 32 * kGenericWarps, 0, stream>>>(p, D);
    return launch_status();
  }

  if (T <= kDirectMaxTokens) {
    if (plan) {
      plan[0] = NVB200_QKNR_KERNEL_DIRECT, plan[1] = 1;
      return NVB200_OK;
    }
    switch (D) {
      case 64: return launch_direct<64>(p, stream);
      case 128: return launch_direct<128>(p, stream);
      default: return launch_direct<256>(p, stream);
    }
  }

  const int sms = sm_count();
  // Small tokens in a rank's qkv_proj layout: units of B consecutive tokens (B a power of two, the unit at most
  // kMultiUnitBytes), when that still gives every SM's CTAs work.
  {
    const int64_t row_stage = static_cast<int64_t>(hq + 2 * hkv) * D * 2;
    const int64_t unit1 = row_stage + D * 4;
    const bool rows_consecutive = a->k == p.q + static_cast<int64_t>(hq) * D &&
                                  a->v == p.k + static_cast<int64_t>(hkv) * D &&
                                  a->q_token_stride == static_cast<int64_t>(hq + 2 * hkv) * D &&
                                  a->k_token_stride == a->q_token_stride && a->v_token_stride == a->q_token_stride;
    int B = 1;
    while (B < kMultiMaxTpu && 2 * B * unit1 <= kMultiUnitBytes) B *= 2;
    // Measured on B200: 2 tokens per unit ran slower than 1 (6.5 KB tokens: 4.7 vs 5.4 TB/s), 4 and 8 faster.
    if (B >= 4 && rows_consecutive && (T + B - 1) / B >= 2 * sms) {
      p.tpu = B;
      p.splits = 1;
      p.g = hkv;
      p.units = (T + B - 1) / B;
      p.stage_bytes = static_cast<int>((B * unit1 + 127) / 128 * 128);
      if (plan) {
        plan[0] = NVB200_QKNR_KERNEL_MULTI, plan[1] = B;
        return NVB200_OK;
      }
      switch (D) {
        case 64: return launch_multi_shaped<64>(p, sms, stream);
        case 128: return launch_multi_shaped<128>(p, sms, stream);
        default: return launch_multi_shaped<256>(p, sms, stream);
      }
    }
  }
  p.tpu = 1;
  if (T * static_cast<int64_t>(hq + 2 * hkv) * D * 2 <= kDirectMaxBytes && T <= 0x7fffffffLL) {
    if (plan) {
      plan[0] = NVB200_QKNR_KERNEL_DIRECT, plan[1] = 1;
      return NVB200_OK;
    }
    switch (D) {
      case 64: return launch_direct<64>(p, stream);
      case 128: return launch_direct<128>(p, stream);
      default: return launch_direct<256>(p, stream);
    }
  }

  // Heads per unit: as many as possible while the units still cover every SM once.
  int splits = hkv;
  for (int d = 1; d <= hkv; ++d) {
    if (hkv % d == 0 && T * d >= sms) {
      splits = d;
      break;
    }
  }
  p.splits = splits;
  p.g = hkv / splits;
  p.units = T * splits;
  if (splits > 1 && p.units > 0x7fffffffLL) return NVB200_ERR_UNSUPPORTED;
  p.qkv_row = splits == 1 && store && a->k == p.q + static_cast<int64_t>(hq) * D &&
              a->v == p.k + static_cast<int64_t>(hkv) * D && a->q_token_stride == a->k_token_stride &&
              a->k_token_stride == a->v_token_stride;
  const int unit_bytes = (p.g * p.r + 2 * p.g) * D * 2 + D * 4;
  p.stage_bytes = (unit_bytes + 127) / 128 * 128;
  if (plan) {
    plan[0] = NVB200_QKNR_KERNEL_BULK, plan[1] = 1;
    return NVB200_OK;
  }
  switch (D) {
    case 64: return launch_bulk_shaped<64>(p, sms, stream);
    case 128: return launch_bulk_shaped<128>(p, sms, stream);
    default: return launch_bulk_shaped<256>(p, sms, stream);
  }
}

}  // namespace nvb200

extern "C" int nvb200_qk_norm_rope_kv(const nvb200_qk_norm_rope_kv_args *args, nvb200_stream_t stream) {
  return nvb200::qk_norm_rope_kv_launch(args, reinterpret_cast<cudaStream_t>(stream), nullptr);
}

extern "C" int nvb200_qk_norm_rope_kv_plan(const nvb200_qk_norm_rope_kv_args *args, int32_t *kernel,
                                           int32_t *tokens_per_unit) {
  int32_t plan[2] = {NVB200_QKNR_KERNEL_NONE, 0};
  const int rc = nvb200::qk_norm_rope_kv_launch(args, nullptr, plan);
  if (kernel) *kernel = plan[0];
  if (tokens_per_unit) *tokens_per_unit = plan[1];
  return rc;
}
