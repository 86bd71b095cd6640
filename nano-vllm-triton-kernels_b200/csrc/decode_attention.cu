// Paged decode attention on B200: o = softmax(q k^T * scale) v over each sequence's keys in the paged KV cache,
// with bottom-right causal alignment (query i of n sees keys [0, L - n + i]) and grouped-query heads. It replaces
// the flash_attn_with_kvcache call of the reference's decode branch (nanovllm/layers/attention.py:84-91), reading
// the [blocks, block_size, Hkv, D] cache that the fused norm/RoPE/KV-write kernel and store_kvcache fill.
//
// Decode attention streams the cache once and is HBM-bound (1 to 16 query rows per KV head against every key), so
// the kernel is organised around the stream:
//   * grid (splits, Hkv, batch); a thread-block cluster of `splits` CTAs shares one (sequence, KV head) and each
//     CTA takes a contiguous share of its keys, in 16-token tiles;
//   * each of a CTA's 4 warps streams every 4th tile through its own cp.async ring (2 stages: one tile in flight while
//     one is consumed; 16-byte copies of whole 256-byte K and V rows, looked up token by token through the block
//     table; rows past the share are zero-filled), so no CTA-wide barrier sits in the loop. At 2 query rows a CTA
//     holds 66 KB of shared memory and three share an SM (a 3-stage ring measured the same or up to 4 % slower at
//     two CTAs per SM, a 4-stage ring 25-30 % slower at one);
//   * q k^T: two lanes per token, each dotting half of the K row (read from a swizzled layout, conflict-free) with
//     the fp32 query rows held in shared memory (pre-scaled by scale * log2(e), broadcast reads); p v: each lane
//     owns 4 of the 128 output columns and reads V rows and the tile's probabilities from shared memory;
//   * online softmax in base 2 per warp (running max and sum per query row), merged across the CTA's warps in
//     shared memory and across the cluster's CTAs through distributed shared memory (each CTA stores its partial
//     into rank 0's shared memory with st.shared::cluster; one cluster barrier; rank 0 writes the output). No global
//     scratch and one launch per call.
// Keys whose block-table entry lies outside [0, num_blocks), and sequence lengths beyond what the block-table row
// addresses, are never read: they are skipped (zero rows, clamped length) and reported in the status word.
#include <algorithm>
#include <atomic>
#include <cmath>

#include "common.cuh"

namespace nvb200 {
namespace {

// Warps per CTA and cp.async ring depth per warp (build-time: -DNVB200_ATTN_WARPS=..., -DNVB200_ATTN_STAGES=...).
#ifndef NVB200_ATTN_WARPS
#define NVB200_ATTN_WARPS 4
#endif
#ifndef NVB200_ATTN_STAGES
#define NVB200_ATTN_STAGES 2
#endif
constexpr int kAttnWarps = NVB200_ATTN_WARPS;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kHeadDim = 128;
// The merges give thread d output column d (and the partial pushes address records by thread index).
static_assert(kAttnThreads == kHeadDim, "one thread per output column: 4 warps at head_dim 128");
constexpr int kRowBytes = kHeadDim * 2;                          // one bf16 K or V row
constexpr int kTileTokens = 16;                                  // keys per warp tile
constexpr int kTileBytes = kTileTokens * kRowBytes;              // 4 KB of K (or of V)
constexpr int kStages = NVB200_ATTN_STAGES;                      // cp.async ring depth per warp
constexpr int kStageBytes = 2 * kTileBytes;                      // the K tile, then the V tile
constexpr int kRingBytes = kAttnWarps * kStages * kStageBytes;   // 64 KB at 4 warps x 2 stages
constexpr int kMaxRows = 16;                                     // query rows per KV head (queries x group)
constexpr int kMaxSplits = 8;                                    // portable cluster size
constexpr int kStateStride = 132;  // floats per partial-state record: o[128], running max, running sum, 2 pad

struct AttnParams {
  const __nv_bfloat16 *q;
  int64_t q_batch_stride, q_token_stride, q_head_stride;
  const __nv_bfloat16 *k_cache;
  const __nv_bfloat16 *v_cache;
  int64_t blk_stride, tok_stride, head_stride;
  int64_t num_blocks;
  const int32_t *block_table;  // NULL: sequence b is block b
  int64_t bt_stride;
  const int32_t *seqlens;
  __nv_bfloat16 *out;          // [batch, sq, hq, 128] contiguous
  int sq, hq, group, block_size, max_pages, rows, causal, splits;
  float scale_log2;
  int32_t *status;
};

NVB200_DEVICE void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
NVB200_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> NVB200_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

NVB200_DEVICE uint2 ld_shared_v2(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
NVB200_DEVICE float2 ld_shared_f2(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
  return v;
}
NVB200_DEVICE float ld_shared_f1(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

NVB200_DEVICE uint32_t cta_rank_in_cluster() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory location in CTA `rank` of this cluster.
NVB200_DEVICE uint32_t map_shared_to(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
NVB200_DEVICE void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
NVB200_DEVICE void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Physical 16-byte chunk of logical chunk c (0..15) of K row t in a tile. The q k^T loop has lane 2t + h read chunk
// 8h + c of row t; within each group of 8 lanes (4 rows x 2 halves) the physical chunks then differ in their low 3
// bits, i.e. fall in distinct shared-memory bank groups.
NVB200_DEVICE int k_chunk(int t, int c) { return c ^ (t & 7) ^ ((c >> 3) << 2); }

// Index in the fp32 query block of element d of query row r: rows of 8 chunks x (2 halves x 8), so that the lanes
// reading half 0 and half 1 of a chunk hit different banks.
NVB200_DEVICE int q_index(int r, int d) { return (r * 8 + ((d >> 3) & 7)) * 16 + (d >> 6) * 8 + (d & 7); }

constexpr int smem_bytes(int R) { return kRingBytes + R * kHeadDim * 4 + kAttnWarps * kTileTokens * R * 4; }
// CTAs per SM at the largest row count (228 KB of shared memory per SM, 1 KB reserved per CTA).
constexpr int kSmemPerSm = 228 * 1024;
constexpr int kFitBlocks = kSmemPerSm / (smem_bytes(kMaxRows) + 1024);
constexpr int kMinBlocks = kFitBlocks > 0 ? kFitBlocks : 1;

template <int R>
__global__ void __launch_bounds__(kAttnThreads, kMinBlocks) paged_decode_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = p.splits > 1 ? cta_rank_in_cluster() : 0u;  // == blockIdx.x: one cluster spans the x axis
  float *q_s = reinterpret_cast<float *>(smem + kRingBytes);
  float *p_w = q_s + R * kHeadDim + warp * kTileTokens * R;  // this warp's probabilities [kTileTokens][R]
  const uint32_t q_addr = smem_addr(q_s), p_addr = smem_addr(p_w);
  const uint32_t wring = smem_addr(smem) + warp * (kStages * kStageBytes);

  // Keys of this sequence: [0, L), clamped to what its block-table row addresses.
  int64_t L = p.seqlens[b];
  const int64_t cap = static_cast<int64_t>(p.max_pages) * p.block_size;
  if (L < 0 || L > cap) {
    if (tid == 0 && rank == 0) set_status(p.status, NVB200_STATUS_BAD_SLOT);
    L = L < 0 ? 0 : cap;
  }
  // This CTA's share [js, je), a whole number of tiles.
  const int64_t per = ((L + p.splits - 1) / p.splits + kTileTokens - 1) / kTileTokens * kTileTokens;
  const int64_t js = min(L, static_cast<int64_t>(rank) * per), je = min(L, js + per);
  const int ntiles = static_cast<int>((je - js + kTileTokens - 1) / kTileTokens);
  const int my_tiles = warp < ntiles ? (ntiles - warp + kAttnWarps - 1) / kAttnWarps : 0;
  const int64_t bt_row = static_cast<int64_t>(b) * p.bt_stride;

  // Copies this warp's i-th tile (keys js + (warp + 4 i) * 16 + [0, 16)) into ring stage `stage`.
  auto issue = [&](int i, int stage) {
    const int64_t j = js + static_cast<int64_t>(warp + i * kAttnWarps) * kTileTokens + (lane & 15);
    int64_t off = -1;  // element offset of key j's row for head h; -1 = not read (zero-filled)
    if (j < je) {
      const int64_t page = j / p.block_size;
      const int64_t blk = p.block_table ? static_cast<int64_t>(__ldg(p.block_table + bt_row + page)) : b;
      if (blk >= 0 && blk < p.num_blocks)
        off = blk * p.blk_stride + (j - page * p.block_size) * p.tok_stride + static_cast<int64_t>(h) * p.head_stride;
      else if (lane < 16)
        set_status(p.status, NVB200_STATUS_BAD_SLOT);
    }
    const uint32_t dst = wring + stage * kStageBytes;
#pragma unroll
    for (int r2 = 0; r2 < kTileTokens / 2; ++r2) {
      const int row = r2 * 2 + (lane >> 4), c = lane & 15;
      const long long o = __shfl_sync(0xffffffffu, static_cast<long long>(off), row);
      const bool ok = o >= 0;
      cp_async16(dst + row * kRowBytes + k_chunk(row, c) * 16, p.k_cache + (ok ? o + c * 8 : 0), ok ? 16u : 0u);
      cp_async16(dst + kTileBytes + row * kRowBytes + c * 16, p.v_cache + (ok ? o + c * 8 : 0), ok ? 16u : 0u);
    }
  };
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < my_tiles) issue(s, s);
    cp_async_commit();
  }

  // Query rows r = i * group + g (query i, q head h * group + g), fp32, scaled; rows past `rows` are zero.
  for (int i = tid; i < R * kHeadDim; i += kAttnThreads) {
    const int r = i / kHeadDim, d = i % kHeadDim;
    float x = 0.f;
    if (r < p.rows) {
      const int qi = r / p.group, g = r - qi * p.group;
      const int64_t at = static_cast<int64_t>(b) * p.q_batch_stride + static_cast<int64_t>(qi) * p.q_token_stride +
                         (static_cast<int64_t>(h) * p.group + g) * p.q_head_stride + d;
      x = __bfloat162float(p.q[at]) * p.scale_log2;
    }
    q_s[q_index(r, d)] = x;
  }
  __syncthreads();

  // Last key each row may see (inclusive).
  int64_t lim[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int qi = r < p.rows ? r / p.group : p.sq - 1;
    lim[r] = p.causal ? L - p.sq + qi : L - 1;
  }

  float m[R], l[R], o[R][4];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    m[r] = -INFINITY, l[r] = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) o[r][e] = 0.f;
  }
  const int t = lane >> 1, half = lane & 1;

  for (int i = 0; i < my_tiles; ++i) {
    if (i + kStages - 1 < my_tiles) issue(i + kStages - 1, (i + kStages - 1) % kStages);
    cp_async_commit();
    cp_async_wait<kStages - 1>();  // this lane's copies of tile i have landed
    __syncwarp();                  // ... and every other lane's
    const uint32_t kt = wring + (i % kStages) * kStageBytes;

    // Scores of key t against every query row, half of the row per lane.
    float s[R];
#pragma unroll
    for (int r = 0; r < R; ++r) s[r] = 0.f;
    const uint32_t krow = kt + t * kRowBytes;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float kf[8];
      unpack8(ld_shared_v4(krow + k_chunk(t, half * 8 + c) * 16), kf);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint32_t qa = q_addr + ((r * 8 + c) * 16 + half * 8) * 4;
        const float4 x = ld_shared_f4(qa), y = ld_shared_f4(qa + 16);
        float acc = s[r];
        acc = fmaf(kf[0], x.x, acc), acc = fmaf(kf[1], x.y, acc), acc = fmaf(kf[2], x.z, acc);
        acc = fmaf(kf[3], x.w, acc), acc = fmaf(kf[4], y.x, acc), acc = fmaf(kf[5], y.y, acc);
        acc = fmaf(kf[6], y.z, acc), acc = fmaf(kf[7], y.w, acc);
        s[r] = acc;
      }
    }
    const int64_t j = js + static_cast<int64_t>(warp + i * kAttnWarps) * kTileTokens + t;
    float alpha[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float sc = s[r] + __shfl_xor_sync(0xffffffffu, s[r], 1);
      if (j >= je || j > lim[r]) sc = -INFINITY;
      float mt = sc;
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
      const float mn = fmaxf(m[r], mt);
      const float mu = mn == -INFINITY ? 0.f : mn;  // no key seen yet: any finite reference keeps exp2 at 0
      alpha[r] = exp2f(m[r] - mu);
      m[r] = mn;
      const float pr = exp2f(sc - mu);
      l[r] = fmaf(l[r], alpha[r], half ? 0.f : pr);  // one lane of the pair counts the key
      if (half == (r & 1)) p_w[t * R + r] = pr;
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
#pragma unroll
      for (int e = 0; e < 4; ++e) o[r][e] *= alpha[r];
    }
    __syncwarp();  // the tile's probabilities are in p_w

    const uint32_t vt = kt + kTileBytes + lane * 8;
#pragma unroll 4
    for (int tt = 0; tt < kTileTokens; ++tt) {
      const uint2 vv = ld_shared_v2(vt + tt * kRowBytes);
      const float v0 = bf16_lo(vv.x), v1 = bf16_hi(vv.x), v2 = bf16_lo(vv.y), v3 = bf16_hi(vv.y);
      float pr[R];
      const uint32_t pa = p_addr + tt * R * 4;
      if constexpr (R >= 4) {
#pragma unroll
        for (int r = 0; r < R; r += 4) {
          const float4 x = ld_shared_f4(pa + r * 4);
          pr[r] = x.x, pr[r + 1] = x.y, pr[r + 2] = x.z, pr[r + 3] = x.w;
        }
      } else if constexpr (R == 2) {
        const float2 x = ld_shared_f2(pa);
        pr[0] = x.x, pr[1] = x.y;
      } else {
        pr[0] = ld_shared_f1(pa);
      }
#pragma unroll
      for (int r = 0; r < R; ++r) {
        o[r][0] = fmaf(pr[r], v0, o[r][0]), o[r][1] = fmaf(pr[r], v1, o[r][1]);
        o[r][2] = fmaf(pr[r], v2, o[r][2]), o[r][3] = fmaf(pr[r], v3, o[r][3]);
      }
    }
    __syncwarp();  // every lane is done with this stage and p_w before they are refilled
  }
  cp_async_wait<0>();

#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) l[r] += __shfl_xor_sync(0xffffffffu, l[r], off);
  }
  __syncthreads();  // every warp is done with its ring, queries and probabilities: the records below reuse them

  // Merge the warps: record (o, m, l) per warp and row, then thread d combines column d.
  float *rec = reinterpret_cast<float *>(smem);  // [kAttnWarps][R][kStateStride]
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float *w = rec + (warp * R + r) * kStateStride;
    *reinterpret_cast<float4 *>(w + 4 * lane) = make_float4(o[r][0], o[r][1], o[r][2], o[r][3]);
    if (lane == 0) w[kHeadDim] = m[r], w[kHeadDim + 1] = l[r];
  }
  __syncthreads();
  float oc[R], mc[R], lc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, rec[(w * R + r) * kStateStride + kHeadDim]);
    const float mu = mx == -INFINITY ? 0.f : mx;
    float acc = 0.f, sum = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float *x = rec + (w * R + r) * kStateStride;
      const float sc = exp2f(x[kHeadDim] - mu);
      acc = fmaf(sc, x[tid], acc);
      sum = fmaf(sc, x[kHeadDim + 1], sum);
    }
    oc[r] = acc, mc[r] = mx, lc[r] = sum;
  }

  auto write_row = [&](int r, float acc, float sum) {
    if (r >= p.rows) return;
    const int qi = r / p.group, g = r - qi * p.group;
    const int64_t idx = ((static_cast<int64_t>(b) * p.sq + qi) * p.hq + static_cast<int64_t>(h) * p.group + g) *
                        kHeadDim + tid;
    p.out[idx] = __float2bfloat16_rn(sum > 0.f ? acc / sum : 0.f);
  };
  if (p.splits == 1) {
#pragma unroll
    for (int r = 0; r < R; ++r) write_row(r, oc[r], lc[r]);
    return;
  }

  // Merge the cluster's CTAs in rank 0. The first barrier: every CTA has read its own records, so rank 0's ring
  // may take the partials; the second: every partial has landed.
  cluster_barrier();
  float *part = reinterpret_cast<float *>(smem);  // in rank 0: [splits][R][kStateStride]
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const uint32_t base = smem_addr(part + (rank * R + r) * kStateStride);
    st_cluster_f32(map_shared_to(base + tid * 4, 0), oc[r]);
    if (tid == 0) {
      st_cluster_f32(map_shared_to(base + kHeadDim * 4, 0), mc[r]);
      st_cluster_f32(map_shared_to(base + (kHeadDim + 1) * 4, 0), lc[r]);
    }
  }
  cluster_barrier();
  if (rank != 0) return;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float mx = -INFINITY;
    for (int s = 0; s < p.splits; ++s) mx = fmaxf(mx, part[(s * R + r) * kStateStride + kHeadDim]);
    const float mu = mx == -INFINITY ? 0.f : mx;
    float acc = 0.f, sum = 0.f;
    for (int s = 0; s < p.splits; ++s) {
      const float *x = part + (s * R + r) * kStateStride;
      const float sc = exp2f(x[kHeadDim] - mu);
      acc = fmaf(sc, x[tid], acc);
      sum = fmaf(sc, x[kHeadDim + 1], sum);
    }
    write_row(r, acc, sum);
  }
}

// The merge records (per warp, then per cluster CTA) reuse the whole dynamic shared memory; both grow linearly in R,
// as the shared memory does, so fitting at the largest R means fitting at every R.
static_assert(kAttnWarps * kMaxRows * kStateStride * 4 <= smem_bytes(kMaxRows), "warp records must fit");
static_assert(kMaxSplits * kMaxRows * kStateStride * 4 <= smem_bytes(kMaxRows), "cluster partials must fit");
static_assert(kAttnWarps * kStateStride * 4 <= kRingBytes && kMaxSplits * kStateStride * 4 <= kRingBytes,
              "records of one row fit in the ring (so they fit at every R once they fit at the largest)");
static_assert(smem_bytes(kMaxRows) <= 227 * 1024, "a CTA's shared memory");

template <int R> int launch_rows(const AttnParams &p, int batch, int hkv, cudaStream_t stream) {
  static std::atomic<int> configured[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NVB200_ERR_CUDA;
  const int smem = smem_bytes(R);
  if (dev >= 64 || configured[dev].load(std::memory_order_acquire) == 0) {
    if (cudaFuncSetAttribute(paged_decode_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return NVB200_ERR_CUDA;
    if (dev < 64) configured[dev].store(1, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(p.splits), static_cast<unsigned>(hkv), static_cast<unsigned>(batch));
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(p.splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, paged_decode_kernel<R>, p) == cudaSuccess ? NVB200_OK : NVB200_ERR_CUDA;
}

}  // namespace
}  // namespace nvb200

using namespace nvb200;

extern "C" int nvb200_paged_decode_splits(int32_t batch, int32_t num_kv_heads, int32_t max_blocks_per_seq,
                                          int32_t block_size, int32_t num_splits) {
  if (batch <= 0 || num_kv_heads <= 0 || max_blocks_per_seq <= 0 || block_size <= 0) return 1;
  // Enough CTAs for one wave at two per SM, each with at least one tile per warp of the longest sequence.
  const int64_t pairs = static_cast<int64_t>(batch) * num_kv_heads;
  int64_t splits = num_splits > 0 ? num_splits : std::max<int64_t>(1, 2 * static_cast<int64_t>(sm_count()) / pairs);
  const int64_t max_len = static_cast<int64_t>(max_blocks_per_seq) * block_size;
  const int64_t useful = std::max<int64_t>(1, (max_len + kAttnWarps * kTileTokens - 1) / (kAttnWarps * kTileTokens));
  splits = std::min<int64_t>({splits, useful, kMaxSplits});
  return static_cast<int>(std::max<int64_t>(1, splits));
}

extern "C" int nvb200_paged_decode_attention(const nvb200_paged_decode_args *a, nvb200_stream_t stream) {
  if (!a) return NVB200_ERR_ARG;
  if (a->batch < 0 || a->queries_per_seq <= 0 || a->num_q_heads <= 0 || a->num_kv_heads <= 0 || a->head_dim <= 0 ||
      a->block_size <= 0 || a->max_blocks_per_seq <= 0 || a->num_blocks < 0 || a->num_splits < 0 ||
      a->num_q_heads % a->num_kv_heads != 0)
    return NVB200_ERR_ARG;
  if (a->dtype != NVB200_BF16 && a->dtype != NVB200_F16 && a->dtype != NVB200_F32) return NVB200_ERR_ARG;
  if (!a->block_table && a->max_blocks_per_seq != 1) return NVB200_ERR_ARG;
  if (a->batch == 0) return NVB200_OK;
  if (!a->out || !a->q || !a->k_cache || !a->v_cache || !a->seqlens) return NVB200_ERR_ARG;
  const int group = a->num_q_heads / a->num_kv_heads;
  const int64_t rows = static_cast<int64_t>(a->queries_per_seq) * group;
  if (a->dtype != NVB200_BF16 || a->head_dim != kHeadDim || rows > kMaxRows) return NVB200_ERR_UNSUPPORTED;
  if (!aligned16(a->k_cache) || !aligned16(a->v_cache) || a->cache_block_stride % 8 != 0 ||
      a->cache_token_stride % 8 != 0 || a->cache_head_stride % 8 != 0)
    return NVB200_ERR_UNSUPPORTED;
  if (a->batch > 65535 || a->num_kv_heads > 65535) return NVB200_ERR_UNSUPPORTED;
  if (int rc = check_device()) return rc;

  AttnParams p{};
  p.q = static_cast<const __nv_bfloat16 *>(a->q);
  p.q_batch_stride = a->q_batch_stride, p.q_token_stride = a->q_token_stride, p.q_head_stride = a->q_head_stride;
  p.k_cache = static_cast<const __nv_bfloat16 *>(a->k_cache);
  p.v_cache = static_cast<const __nv_bfloat16 *>(a->v_cache);
  p.blk_stride = a->cache_block_stride, p.tok_stride = a->cache_token_stride, p.head_stride = a->cache_head_stride;
  p.num_blocks = a->num_blocks;
  p.block_table = a->block_table, p.bt_stride = a->block_table_stride;
  p.seqlens = a->seqlens;
  p.out = static_cast<__nv_bfloat16 *>(a->out);
  p.sq = a->queries_per_seq, p.hq = a->num_q_heads, p.group = group;
  p.block_size = a->block_size, p.max_pages = a->max_blocks_per_seq, p.rows = static_cast<int>(rows);
  p.causal = a->causal != 0;
  p.splits = nvb200_paged_decode_splits(a->batch, a->num_kv_heads, a->max_blocks_per_seq, a->block_size,
                                        a->num_splits);
  p.scale_log2 = static_cast<float>(static_cast<double>(a->softmax_scale) * 1.4426950408889634);
  p.status = a->status;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (rows <= 1) return launch_rows<1>(p, a->batch, a->num_kv_heads, s);
  if (rows <= 2) return launch_rows<2>(p, a->batch, a->num_kv_heads, s);
  if (rows <= 4) return launch_rows<4>(p, a->batch, a->num_kv_heads, s);
  if (rows <= 8) return launch_rows<8>(p, a->batch, a->num_kv_heads, s);
  return launch_rows<16>(p, a->batch, a->num_kv_heads, s);
}
