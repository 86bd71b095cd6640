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
// A second kernel below (stream-K) runs the same per-tile code on a persistent grid that divides all of a batch's
// tiles evenly between the SMs and merges split sequences through a workspace; it pays off when the batch has more
// (sequence, head) pairs than one wave of the first kernel holds.
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
// CTAs per SM the cluster kernel's launch bounds ask for at R rows: as many as its shared memory allows, at most 3
// (three at 1-8 rows, two at 16); the register budget per thread follows from it.
constexpr int cluster_min_blocks(int R) {
  return kSmemPerSm / (smem_bytes(R) + 1024) >= 3 ? 3 : (kSmemPerSm / (smem_bytes(R) + 1024) > 0 ? 2 : 1);
}

// Online-softmax state of one warp over R query rows (base 2, scores pre-scaled by scale * log2 e). Lane 2t + half
// scores key t of a tile against half `half` of each query row; o[r][e] is output column 4 * lane + e of row r;
// l[r] is the lane's share of row r's sum (lanes with half = 0 count their key), summed over the warp at the end.
template <int R> struct WarpSoftmax {
  float m[R], l[R], o[R][4];
  NVB200_DEVICE void reset() {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      m[r] = -INFINITY, l[r] = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) o[r][e] = 0.f;
    }
  }
  // Sums the lanes' shares of the row sums (every lane ends with the warp's total).
  NVB200_DEVICE void reduce_sums() {
#pragma unroll
    for (int r = 0; r < R; ++r) {
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) l[r] += __shfl_xor_sync(0xffffffffu, l[r], off);
    }
  }
};

// Last key (inclusive) each query row may see in a sequence of L keys: row r is query r / group of sq.
template <int R>
NVB200_DEVICE void row_limits(int64_t (&lim)[R], int64_t L, int rows, int group, int sq, int causal) {
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int qi = r < rows ? r / group : sq - 1;
    lim[r] = causal ? L - sq + qi : L - 1;
  }
}

// Folds one 16-key tile into the warp's state: kt is the ring stage (K tile, then V tile, both landed and visible to
// the whole warp), q_addr the fp32 query block, p_w / p_addr the warp's [kTileTokens][R] probability scratch. j0 is
// the index of the tile's first key; keys at or past je, or past a row's limit, get probability zero. Ends with a
// __syncwarp, after which the stage and p_w may be refilled.
template <int R>
NVB200_DEVICE void fold_tile(WarpSoftmax<R> &st, uint32_t kt, uint32_t q_addr, float *p_w, uint32_t p_addr, int lane,
                             int64_t j0, int64_t je, const int64_t (&lim)[R]) {
  const int t = lane >> 1, half = lane & 1;
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
  const int64_t j = j0 + t;
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
    const float mn = fmaxf(st.m[r], mt);
    const float mu = mn == -INFINITY ? 0.f : mn;  // no key seen yet: any finite reference keeps exp2 at 0
    alpha[r] = exp2f(st.m[r] - mu);
    st.m[r] = mn;
    const float pr = exp2f(sc - mu);
    st.l[r] = fmaf(st.l[r], alpha[r], half ? 0.f : pr);  // one lane of the pair counts the key
    if (half == (r & 1)) p_w[t * R + r] = pr;
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int e = 0; e < 4; ++e) st.o[r][e] *= alpha[r];
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
      st.o[r][0] = fmaf(pr[r], v0, st.o[r][0]), st.o[r][1] = fmaf(pr[r], v1, st.o[r][1]);
      st.o[r][2] = fmaf(pr[r], v2, st.o[r][2]), st.o[r][3] = fmaf(pr[r], v3, st.o[r][3]);
    }
  }
  __syncwarp();  // every lane is done with this stage and p_w before they are refilled
}

// Writes the warp's (o, m, l) per row into records rec[warp][R][kStateStride] (after reduce_sums).
template <int R> NVB200_DEVICE void store_warp_record(const WarpSoftmax<R> &st, float *rec, int warp, int lane) {
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float *w = rec + (warp * R + r) * kStateStride;
    *reinterpret_cast<float4 *>(w + 4 * lane) = make_float4(st.o[r][0], st.o[r][1], st.o[r][2], st.o[r][3]);
    if (lane == 0) w[kHeadDim] = st.m[r], w[kHeadDim + 1] = st.l[r];
  }
}

// Thread d merges column d of the CTA's warp records: unnormalised output oc, max mc and sum lc per row.
template <int R>
NVB200_DEVICE void merge_warp_records(const float *rec, int tid, float (&oc)[R], float (&mc)[R], float (&lc)[R]) {
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
}

// ---------------------------------------------------------------------------------------------------------------
// Tile fold on the tensor cores (the cluster kernel). Per 16-key tile a warp runs S = Q K^T and O += P V as warp-level
// bf16 MMAs (m16n8k16, fp32 accumulation) with the query rows as the MMA's 16 rows (rows past R are zero), instead of
// one FMA per key, dimension and row on the CUDA cores: about 130 instructions per tile instead of about 500, which is
// what bounded the CUDA-core fold at the decode shape (few warps per SM, each issue-bound). The tiles are 16 x 16 and
// 16 x 128, far below the 128-row tiles tcgen05.mma works on, and a warp owns its tile stream end to end, so the
// warp-synchronous MMA fits here where a CTA-wide tcgen05 pipeline would not. K and V rows sit in shared memory with
// the k_chunk swizzle, so the ldmatrix row addresses of each 8 x 8 matrix fall in distinct bank groups. (The MMA
// and ldmatrix wrappers and the fragment layout are in common.cuh.)

// One warp's online-softmax state for the MMA fold: lane 4 g + t holds rows g and g + 8 (index 0 and 1): running max
// m (base 2, scaled scores), its share l of the row sums (the keys of its columns; summed over t at the end), and
// o[n] = the C fragment of output columns 8 n .. 8 n + 7.
struct MmaSoftmax {
  float m[2], l[2], o[16][4];
  NVB200_DEVICE void reset() {
    m[0] = m[1] = -INFINITY, l[0] = l[1] = 0.f;
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  }
  NVB200_DEVICE void reduce_sums() {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      l[i] += __shfl_xor_sync(0xffffffffu, l[i], 1);
      l[i] += __shfl_xor_sync(0xffffffffu, l[i], 2);
    }
  }
};

// A fragments of the query block (rows r = i * group + gq, bf16 as stored, unscaled) for the 8 k-steps of head_dim
// 128; rows at or past `rows` are zero.
NVB200_DEVICE void load_q_frags(const AttnParams &p, int b, int h, int lane, uint32_t (&qa)[8][4]) {
  const int g = lane >> 2, t = lane & 3;
  const uint32_t *rowp[2] = {nullptr, nullptr};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = g + 8 * i;
    if (r < p.rows) {
      const int qi = r / p.group, gq = r - qi * p.group;
      rowp[i] = reinterpret_cast<const uint32_t *>(
          p.q + static_cast<int64_t>(b) * p.q_batch_stride + static_cast<int64_t>(qi) * p.q_token_stride +
          (static_cast<int64_t>(h) * p.group + gq) * p.q_head_stride);
    }
  }
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    qa[ks][0] = rowp[0] ? __ldg(rowp[0] + 8 * ks + t) : 0u;
    qa[ks][1] = rowp[1] ? __ldg(rowp[1] + 8 * ks + t) : 0u;
    qa[ks][2] = rowp[0] ? __ldg(rowp[0] + 8 * ks + 4 + t) : 0u;
    qa[ks][3] = rowp[1] ? __ldg(rowp[1] + 8 * ks + 4 + t) : 0u;
  }
}

// Folds one 16-key tile (K tile at kt, V tile at kt + kTileBytes, both k_chunk-swizzled, landed and visible to the
// warp) into the state. j0: index of the tile's first key; keys at or past je, or past a row's limit (lim0: row g,
// lim1: row g + 8), get probability zero. scale: softmax_scale * log2(e). Ends with a __syncwarp, after which the
// stage may be refilled.
NVB200_DEVICE void fold_tile_mma(MmaSoftmax &st, uint32_t kt, const uint32_t (&qa)[8][4], int lane, int64_t j0,
                                 int64_t je, int64_t lim0, int64_t lim1, float scale) {
  const int t = lane & 3, mq = lane >> 3, rr = lane & 7;
  // S = Q K^T: n-tile 0 holds keys 0-7, n-tile 1 keys 8-15. ldmatrix matrix mq: keys (mq >> 1) * 8 + rr, 16-byte
  // chunk 2 ks + (mq & 1) of head_dim.
  float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
  const int kkey = (mq >> 1) * 8 + rr;
  const uint32_t krow = kt + kkey * kRowBytes;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    uint32_t bk[4];
    ldsm_x4(krow + k_chunk(kkey, 2 * ks + (mq & 1)) * 16, bk);
    mma_16816(s0, qa[ks], bk[0], bk[1]);
    mma_16816(s1, qa[ks], bk[2], bk[3]);
  }
  // sc[0..3]: row g at keys 2t, 2t + 1, 8 + 2t, 9 + 2t; sc[4..7]: row g + 8 at the same keys.
  float sc[8] = {s0[0], s0[1], s1[0], s1[1], s0[2], s0[3], s1[2], s1[3]};
  const int kj[4] = {2 * t, 2 * t + 1, 8 + 2 * t, 9 + 2 * t};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t j = j0 + kj[i];
    sc[i] = (j >= je || j > lim0) ? -INFINITY : sc[i] * scale;
    sc[4 + i] = (j >= je || j > lim1) ? -INFINITY : sc[4 + i] * scale;
  }
  float alpha[2], pr[8];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    float mt = fmaxf(fmaxf(sc[4 * i], sc[4 * i + 1]), fmaxf(sc[4 * i + 2], sc[4 * i + 3]));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
    const float mn = fmaxf(st.m[i], mt);
    const float mu = mn == -INFINITY ? 0.f : mn;  // no key seen yet: any finite reference keeps exp2 at 0
    alpha[i] = exp2f(st.m[i] - mu);
    st.m[i] = mn;
    float sum = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      pr[4 * i + e] = exp2f(sc[4 * i + e] - mu);
      sum += pr[4 * i + e];
    }
    st.l[i] = fmaf(st.l[i], alpha[i], sum);
  }
  if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      st.o[n][0] *= alpha[0], st.o[n][1] *= alpha[0];
      st.o[n][2] *= alpha[1], st.o[n][3] *= alpha[1];
    }
  }
  // P as the A operand of O += P V (k = the tile's 16 keys): the C fragments of the two key n-tiles, in bf16.
  const uint32_t pa[4] = {pack_bf16x2(pr[0], pr[1]), pack_bf16x2(pr[4], pr[5]), pack_bf16x2(pr[2], pr[3]),
                          pack_bf16x2(pr[6], pr[7])};
  // V as the B operand, transposed by ldmatrix: matrix mq holds keys (mq & 1) * 8 + rr, chunk 2 np + (mq >> 1).
  const int vkey = (mq & 1) * 8 + rr;
  const uint32_t vrow = kt + kTileBytes + vkey * kRowBytes;
#pragma unroll
  for (int np = 0; np < 8; ++np) {
    uint32_t bv[4];
    ldsm_x4_trans(vrow + k_chunk(vkey, 2 * np + (mq >> 1)) * 16, bv);
    mma_16816(st.o[2 * np], pa, bv[0], bv[1]);
    mma_16816(st.o[2 * np + 1], pa, bv[2], bv[3]);
  }
  __syncwarp();  // every lane is done with this stage before it is refilled
}

// Writes the warp's (o, m, l) for rows below R into records rec[warp][R][kStateStride] (after reduce_sums).
template <int R> NVB200_DEVICE void store_warp_record_mma(const MmaSoftmax &st, float *rec, int warp, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = g + 8 * i;
    if (r >= R) continue;
    float *w = rec + (warp * R + r) * kStateStride;
#pragma unroll
    for (int n = 0; n < 16; ++n)
      *reinterpret_cast<float2 *>(w + 8 * n + 2 * t) = make_float2(st.o[n][2 * i], st.o[n][2 * i + 1]);
    if (t == 0) w[kHeadDim] = st.m[i], w[kHeadDim + 1] = st.l[i];
  }
}

template <int R>
__global__ void __launch_bounds__(kAttnThreads, cluster_min_blocks(R))
    paged_decode_kernel(const __grid_constant__ AttnParams p) {
  launch_dependents();  // a dependent launched early waits for this grid before reading its output
  grid_dependency_wait();  // this grid may itself have been launched early
  extern __shared__ __align__(128) uint8_t smem[];
  const int h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = p.splits > 1 ? cta_rank_in_cluster() : 0u;  // == blockIdx.x: one cluster spans the x axis
  const uint32_t wring = smem_addr(smem) + warp * (kStages * kStageBytes);

  const int64_t bt_row = static_cast<int64_t>(b) * p.bt_stride;
  int32_t bt_lane = 0;
  if (p.splits == 1 && p.block_table && lane < p.max_pages) bt_lane = __ldg(p.block_table + bt_row + lane);
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
  // The block-table entries of the share's first 32 pages, one per lane, loaded once: a tile's copy then needs no
  // table read of its own (which would put a round trip to L2 in front of every tile's copies). Without a split the
  // share starts at key 0, so they were loaded above, together with the length.
  const int64_t page0 = js / p.block_size;
  if (p.splits > 1 && p.block_table && page0 + lane < p.max_pages)
    bt_lane = __ldg(p.block_table + bt_row + page0 + lane);

  // Copies this warp's i-th tile (keys js + (warp + 4 i) * 16 + [0, 16)) into ring stage `stage`.
  auto issue = [&](int i, int stage) {
    const int64_t j = js + static_cast<int64_t>(warp + i * kAttnWarps) * kTileTokens + (lane & 15);
    int64_t off = -1;  // element offset of key j's row for head h; -1 = not read (zero-filled)
    const int64_t page = j / p.block_size;
    const int64_t rel = page - page0;
    const int32_t cached = __shfl_sync(0xffffffffu, bt_lane, static_cast<int>(rel < 31 ? rel : 31));
    if (j < je) {
      const int64_t blk = !p.block_table ? b
                          : rel < 32     ? static_cast<int64_t>(cached)
                                         : static_cast<int64_t>(__ldg(p.block_table + bt_row + page));
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
      cp_async16(dst + kTileBytes + row * kRowBytes + k_chunk(row, c) * 16, p.v_cache + (ok ? o + c * 8 : 0),
                 ok ? 16u : 0u);
    }
  };
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < my_tiles) issue(s, s);
    cp_async_commit();
  }

  // Query rows r = i * group + g (query i, q head h * group + g) as MMA A fragments; rows past `rows` are zero.
  uint32_t qa[8][4];
  load_q_frags(p, b, h, lane, qa);
  // Key limits of this lane's two rows (g and g + 8).
  int64_t lim[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = (lane >> 2) + 8 * i;
    const int qi = r < p.rows ? r / p.group : p.sq - 1;
    lim[i] = p.causal ? L - p.sq + qi : L - 1;
  }
  MmaSoftmax st;
  st.reset();

  for (int i = 0; i < my_tiles; ++i) {
    if (i + kStages - 1 < my_tiles) issue(i + kStages - 1, (i + kStages - 1) % kStages);
    cp_async_commit();
    cp_async_wait<kStages - 1>();  // this lane's copies of tile i have landed
    __syncwarp();                  // ... and every other lane's
    fold_tile_mma(st, wring + (i % kStages) * kStageBytes, qa, lane,
                  js + static_cast<int64_t>(warp + i * kAttnWarps) * kTileTokens, je, lim[0], lim[1], p.scale_log2);
  }
  cp_async_wait<0>();
  st.reduce_sums();
  __syncthreads();  // every warp is done with its ring: the records below reuse it

  // Merge the warps: record (o, m, l) per warp and row, then thread d combines column d.
  float *rec = reinterpret_cast<float *>(smem);  // [kAttnWarps][R][kStateStride]
  store_warp_record_mma<R>(st, rec, warp, lane);
  __syncthreads();
  float oc[R], mc[R], lc[R];
  merge_warp_records<R>(rec, tid, oc, mc, lc);

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

// ---------------------------------------------------------------------------------------------------------------
// Stream-K form. The work of one call is a sequence of units (sequence b, KV head h, 16-key tile), ordered by b, then
// h, then tile; sequence b has T_b = ceil(L_b / 16) tiles per head, so U = Hkv * sum_b T_b units in all. A persistent
// grid of G CTAs (as many as are resident at once) gives CTA c the units [c U / G, (c + 1) U / G): every SM gets the
// same number of tiles whatever the batch shape, where one CTA per (sequence, head) leaves some SMs with one CTA
// and others with two. A CTA walks its range one segment (the units of one (b, h)) at a time; its warps split each
// segment's tiles (warp w takes every 4th) and keep their cp.async rings running across segment ends, so a new
// segment's first tiles are in flight while the last one is merged. A segment that is a whole (b, h) writes its
// output rows directly. A (b, h) split between CTAs (only the first and last segment of a range can be) leaves one
// partial record (o, m, l per row) per CTA in the workspace; each such CTA then takes a ticket from the (b, h)'s
// arrival counter and the last to arrive merges the records in CTA order (so results do not depend on timing) and
// resets the counter to zero. No CTA waits for another.
//
// Workspace: the partial records fp32 [2 * grid][R][kStateStride] at offset 0 (CTA c writes slots 2c and 2c + 1), in a
// region of one fixed size per device (the largest any row count needs), then the counters int32 [batch * Hkv] (zero
// before the first call; every call leaves them zero). The fixed split keeps every call's counters off every other
// call's records, whatever their batch sizes and row counts.
constexpr int64_t kCounterAlign = 256;
// Fewest tiles a CTA takes (4 per warp) when the batch has too few for every resident CTA: shorter ranges spend more
// time starting and merging than streaming.
constexpr int64_t kMinTilesPerCta = 16;

struct StreamKParams {
  int32_t *counters;
  float *partials;
  int batch, hkv;
};

constexpr int streamk_smem_bytes(int R) { return smem_bytes(R) + kAttnWarps * R * kStateStride * 4 + 16; }
static_assert(streamk_smem_bytes(kMaxRows) <= 227 * 1024, "a stream-K CTA's shared memory");
// CTAs per SM that the shared memory of R rows allows (the register budget follows it through the launch bounds).
constexpr int streamk_min_blocks(int R) {
  return kSmemPerSm / (streamk_smem_bytes(R) + 1024) > 0 ? kSmemPerSm / (streamk_smem_bytes(R) + 1024) : 1;
}

// Keys of sequence b, clamped to [0, what its block-table row addresses].
NVB200_DEVICE int64_t seq_keys(const AttnParams &p, int b) {
  const int64_t L = p.seqlens[b];
  const int64_t cap = static_cast<int64_t>(p.max_pages) * p.block_size;
  return L < 0 ? 0 : (L > cap ? cap : L);
}
NVB200_DEVICE int64_t tiles_of(int64_t keys) { return (keys + kTileTokens - 1) / kTileTokens; }

// The units of one (b, h) inside one CTA's range. CTA-uniform: every thread of the CTA holds the same values. Unit
// indices fit in 32 bits (the host checks batch * Hkv * the longest sequence's tiles < 2^31).
struct Segment {
  int32_t u;       // global index of the segment's first unit
  int32_t pair_u;  // global index of unit 0 of (b, h)
  int32_t pre;     // tiles of the sequences before b (units before b = hkv * pre)
  int32_t tiles;   // T_b
  int32_t t0;      // first tile of the segment within (b, h)
  int32_t n;       // tiles in the segment; 0 = the range is exhausted
  int32_t b, h;
  int64_t L;       // keys of sequence b

  // Moves to the next (b, h) of the range [., u1).
  NVB200_DEVICE void next(const AttnParams &p, int batch, int hkv, int32_t u1) {
    u += n;
    if (u >= u1) {
      n = 0;
      return;
    }
    if (h + 1 < hkv) {
      ++h;
    } else {
      pre += tiles;
      h = 0;
      do {
        ++b;
        L = seq_keys(p, b);
        tiles = static_cast<int32_t>(tiles_of(L));
      } while (tiles == 0 && b + 1 < batch);
    }
    pair_u = hkv * pre + h * tiles;
    t0 = 0;
    n = min(tiles, u1 - u);
  }
  NVB200_DEVICE bool whole() const { return t0 == 0 && n == tiles; }
};

// First unit of CTA c's range, and the CTA whose range holds unit u (G <= U, so no range is empty).
NVB200_DEVICE int64_t range_start(int64_t c, int64_t U, int64_t G) { return c * U / G; }
NVB200_DEVICE int64_t range_owner(int64_t u, int64_t U, int64_t G) { return ((u + 1) * G - 1) / U; }
// Partial-record slot of CTA c for the (b, h) whose unit 0 is pair_u: 2c if (b, h) holds c's first unit, else 2c + 1
// (then it is c's last segment).
NVB200_DEVICE int64_t partial_slot(int64_t c, int64_t pair_u, int64_t U, int64_t G) {
  return 2 * c + (pair_u <= range_start(c, U, G) ? 0 : 1);
}

NVB200_DEVICE long long warp_sum_i64(long long x) {
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}
NVB200_DEVICE long long warp_inclusive_scan_i64(long long x, int lane) {
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const long long y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  return x;
}

template <int R>
__global__ void __launch_bounds__(kAttnThreads, streamk_min_blocks(R))
    paged_decode_streamk_kernel(const __grid_constant__ AttnParams p, const __grid_constant__ StreamKParams sk) {
  launch_dependents();  // a dependent launched early waits for this grid before reading its output
  grid_dependency_wait();  // this grid may itself have been launched early
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float *q_s = reinterpret_cast<float *>(smem + kRingBytes);
  float *p_w = q_s + R * kHeadDim + warp * kTileTokens * R;
  float *rec = q_s + R * kHeadDim + kAttnWarps * kTileTokens * R;  // [kAttnWarps][R][kStateStride]
  long long *meta = reinterpret_cast<long long *>(rec + kAttnWarps * R * kStateStride);  // [2]: U, then a flag
  const uint32_t q_addr = smem_addr(q_s), p_addr = smem_addr(p_w);
  const uint32_t wring = smem_addr(smem) + warp * (kStages * kStageBytes);
  const int hkv = sk.hkv, batch = sk.batch;

  auto write_row = [&](int b, int h, int r, float acc, float sum) {
    if (r >= p.rows) return;
    const int qi = r / p.group, g = r - qi * p.group;
    const int64_t idx = ((static_cast<int64_t>(b) * p.sq + qi) * p.hq + static_cast<int64_t>(h) * p.group + g) *
                        kHeadDim + tid;
    p.out[idx] = __float2bfloat16_rn(sum > 0.f ? acc / sum : 0.f);
  };

  // Sequences without keys own no units: their rows are zeros, written by CTA (b * hkv + h) mod grid.
  for (int64_t pr = blockIdx.x; pr < static_cast<int64_t>(batch) * hkv; pr += gridDim.x) {
    const int b = static_cast<int>(pr / hkv), h = static_cast<int>(pr - static_cast<int64_t>(b) * hkv);
    if (seq_keys(p, b) == 0) {
      for (int r = 0; r < p.rows; ++r) write_row(b, h, r, 0.f, 0.f);
    }
  }

  // U, by warp 0 (CTA 0 also flags lengths outside [0, what the block table addresses]).
  if (warp == 0) {
    long long tot = 0;
    bool bad = false;
    const int64_t cap = static_cast<int64_t>(p.max_pages) * p.block_size;
    for (int b0 = 0; b0 < batch; b0 += 32) {
      const int b = b0 + lane;
      long long t = 0;
      if (b < batch) {
        const int64_t raw = p.seqlens[b];
        bad |= raw < 0 || raw > cap;
        t = tiles_of(seq_keys(p, b));
      }
      tot += warp_sum_i64(t);
    }
    if (blockIdx.x == 0 && __any_sync(0xffffffffu, bad) && lane == 0) set_status(p.status, NVB200_STATUS_BAD_SLOT);
    if (lane == 0) meta[0] = tot * hkv;
  }
  __syncthreads();
  const int64_t U = meta[0];
  const int64_t G = min(static_cast<int64_t>(gridDim.x), max(int64_t{1}, U / kMinTilesPerCta));
  const int64_t c = blockIdx.x;
  if (U == 0 || c >= G) return;
  const int32_t u0 = static_cast<int32_t>(range_start(c, U, G)), u1 = static_cast<int32_t>(range_start(c + 1, U, G));

  // The segment holding u0: sequence b with hkv * P(b) <= u0 < hkv * P(b + 1), P the tile prefix (every warp scans,
  // so the result is in every thread's registers without another barrier).
  Segment seg{};
  {
    long long base = 0;
    for (int b0 = 0; b0 < batch; b0 += 32) {
      const int b = b0 + lane;
      const long long t = b < batch ? tiles_of(seq_keys(p, b)) : 0;
      const long long incl = warp_inclusive_scan_i64(t, lane);
      const unsigned hit = __ballot_sync(0xffffffffu, b < batch && (base + incl) * hkv > u0);
      if (hit) {
        const int first = __ffs(hit) - 1;
        seg.b = b0 + first;
        seg.tiles = static_cast<int32_t>(__shfl_sync(0xffffffffu, t, first));
        seg.pre = static_cast<int32_t>(base + __shfl_sync(0xffffffffu, incl, first)) - seg.tiles;
        break;
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    seg.L = seq_keys(p, seg.b);
    const int32_t within = u0 - hkv * seg.pre;
    seg.h = within / seg.tiles;
    seg.t0 = within - seg.h * seg.tiles;
    seg.pair_u = hkv * seg.pre + seg.h * seg.tiles;
    seg.u = u0;
    seg.n = min(seg.tiles - seg.t0, u1 - u0);
  }

  // This warp's issue cursor: item i of segment `is` is tile is.t0 + warp + 4 i of (is.b, is.h).
  Segment is = seg;
  int ii = 0;
  auto skip_empty = [&]() {
    while (is.n > 0 && warp + ii * kAttnWarps >= is.n) {
      is.next(p, batch, hkv, u1);
      ii = 0;
    }
  };
  skip_empty();
  auto issue_next = [&](int stage) {
    const int64_t j = (is.t0 + warp + static_cast<int64_t>(ii) * kAttnWarps) * kTileTokens + (lane & 15);
    int64_t off = -1;  // element offset of key j's row for head is.h; -1 = not read (zero-filled)
    if (j < is.L) {
      const int64_t page = j / p.block_size;
      const int64_t blk =
          p.block_table ? static_cast<int64_t>(__ldg(p.block_table + static_cast<int64_t>(is.b) * p.bt_stride + page))
                        : is.b;
      if (blk >= 0 && blk < p.num_blocks)
        off = blk * p.blk_stride + (j - page * p.block_size) * p.tok_stride +
              static_cast<int64_t>(is.h) * p.head_stride;
      else if (lane < 16)
        set_status(p.status, NVB200_STATUS_BAD_SLOT);
    }
    const uint32_t dst = wring + stage * kStageBytes;
#pragma unroll
    for (int r2 = 0; r2 < kTileTokens / 2; ++r2) {
      const int row = r2 * 2 + (lane >> 4), cc = lane & 15;
      const long long o = __shfl_sync(0xffffffffu, static_cast<long long>(off), row);
      const bool ok = o >= 0;
      cp_async16(dst + row * kRowBytes + k_chunk(row, cc) * 16, p.k_cache + (ok ? o + cc * 8 : 0), ok ? 16u : 0u);
      cp_async16(dst + kTileBytes + row * kRowBytes + cc * 16, p.v_cache + (ok ? o + cc * 8 : 0), ok ? 16u : 0u);
    }
    ++ii;
    skip_empty();
  };
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (is.n > 0) issue_next(s);
    cp_async_commit();
  }

  auto load_q = [&](int b, int h) {
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
  };
  load_q(seg.b, seg.h);
  __syncthreads();

  // Query element (row k, column tid) of (b, h), scaled; rows past `rows` are zero.
  auto fetch_q = [&](int b, int h, int k) {
    if (k >= p.rows) return 0.f;
    const int qi = k / p.group, gg = k - qi * p.group;
    const int64_t at = static_cast<int64_t>(b) * p.q_batch_stride + static_cast<int64_t>(qi) * p.q_token_stride +
                       (static_cast<int64_t>(h) * p.group + gg) * p.q_head_stride + tid;
    return __bfloat162float(p.q[at]) * p.scale_log2;
  };
  // Up to 8 rows, the next segment's queries are fetched into registers when a segment starts, so that their loads
  // are in flight while it streams rather than after it.
  constexpr bool kPrefetchQ = R <= 8;
  float qn[kPrefetchQ ? R : 1];

  int g = 0;  // this warp's items consumed so far (ring stage g % kStages)
  while (seg.n > 0) {
    Segment nx = seg;
    nx.next(p, batch, hkv, u1);
    if constexpr (kPrefetchQ) {
      if (nx.n > 0) {
#pragma unroll
        for (int k = 0; k < R; ++k) qn[k] = fetch_q(nx.b, nx.h, k);
      }
    }
    const int my = seg.n > warp ? static_cast<int>((seg.n - warp + kAttnWarps - 1) / kAttnWarps) : 0;
    int64_t lim[R];
    row_limits<R>(lim, seg.L, p.rows, p.group, p.sq, p.causal);
    WarpSoftmax<R> st;
    st.reset();
    for (int i = 0; i < my; ++i, ++g) {
      if (is.n > 0) issue_next((g + kStages - 1) % kStages);
      cp_async_commit();
      cp_async_wait<kStages - 1>();  // this lane's copies of item g have landed
      __syncwarp();                  // ... and every other lane's
      fold_tile<R>(st, wring + (g % kStages) * kStageBytes, q_addr, p_w, p_addr, lane,
                   (seg.t0 + warp + static_cast<int64_t>(i) * kAttnWarps) * kTileTokens, seg.L, lim);
    }
    st.reduce_sums();
    store_warp_record<R>(st, rec, warp, lane);
    __syncthreads();  // records complete; every warp is done with the segment's queries
    float oc[R], mc[R], lc[R];
    merge_warp_records<R>(rec, tid, oc, mc, lc);

    if (seg.whole()) {
#pragma unroll
      for (int r = 0; r < R; ++r) write_row(seg.b, seg.h, r, oc[r], lc[r]);
    } else {
      // Publish this CTA's partial, then take a ticket; the last of the (b, h)'s CTAs merges.
      float *mine = sk.partials + partial_slot(c, seg.pair_u, U, G) * (R * kStateStride);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        mine[r * kStateStride + tid] = oc[r];
        if (tid == 0) mine[r * kStateStride + kHeadDim] = mc[r], mine[r * kStateStride + kHeadDim + 1] = lc[r];
      }
      __threadfence();
      __syncthreads();
      const int64_t pair = static_cast<int64_t>(seg.b) * hkv + seg.h;
      const int64_t first = range_owner(seg.pair_u, U, G), last = range_owner(seg.pair_u + seg.tiles - 1, U, G);
      if (tid == 0) {
        const int ticket = atomicAdd(sk.counters + pair, 1);
        const bool closing = ticket == static_cast<int>(last - first);
        if (closing) {
          sk.counters[pair] = 0;  // every other contributor has taken its ticket
          __threadfence();
        }
        meta[1] = closing ? 1 : 0;
      }
      __syncthreads();
      if (meta[1]) {
        // One pass over the contributors in CTA order with a running maximum; the loads of consecutive contributors
        // do not depend on one another, so the unrolled loop keeps several in flight.
        float mx[R], acc[R], sum[R];
#pragma unroll
        for (int r = 0; r < R; ++r) mx[r] = -INFINITY, acc[r] = 0.f, sum[r] = 0.f;
#pragma unroll 4
        for (int64_t cc = first; cc <= last; ++cc) {
          const float *x = sk.partials + partial_slot(cc, seg.pair_u, U, G) * (R * kStateStride);
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const float m_c = __ldcg(x + r * kStateStride + kHeadDim);
            const float l_c = __ldcg(x + r * kStateStride + kHeadDim + 1);
            const float o_c = __ldcg(x + r * kStateStride + tid);
            const float mn = fmaxf(mx[r], m_c);
            const float mu = mn == -INFINITY ? 0.f : mn;
            const float a_old = exp2f(mx[r] - mu), a_new = exp2f(m_c - mu);
            acc[r] = fmaf(a_new, o_c, acc[r] * a_old);
            sum[r] = fmaf(a_new, l_c, sum[r] * a_old);
            mx[r] = mn;
          }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) write_row(seg.b, seg.h, r, acc[r], sum[r]);
      }
    }
    seg = nx;
    if (seg.n > 0) {
      if constexpr (kPrefetchQ) {
#pragma unroll
        for (int k = 0; k < R; ++k) q_s[q_index(k, tid)] = qn[k];
      } else {
        load_q(seg.b, seg.h);
      }
    }
    __syncthreads();  // the next segment's queries are in place; records and the flag may be rewritten
  }
  cp_async_wait<0>();
}

// Rounds v up to a multiple of a.
constexpr int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// Resident CTAs of the stream-K kernel for R rows on the current device (cached per device), times the SM count.
template <int R> int streamk_grid() {
  static std::atomic<int> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 0;
  int per_sm = dev < 64 ? cached[dev].load(std::memory_order_acquire) : 0;
  if (per_sm == 0) {
    const int smem = streamk_smem_bytes(R);
    if (cudaFuncSetAttribute(paged_decode_streamk_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, paged_decode_streamk_kernel<R>, kAttnThreads, smem) !=
            cudaSuccess ||
        per_sm <= 0)
      return 0;
    if (dev < 64) cached[dev].store(per_sm, std::memory_order_release);
  }
  return per_sm * sm_count();
}

// Bytes of the partial records for `grid` CTAs at R rows.
constexpr int64_t streamk_partial_bytes(int64_t grid, int R) { return 2 * grid * R * kStateStride * 4; }

template <int R>
int launch_streamk(const AttnParams &p, int batch, int hkv, int grid, int32_t *counters, float *partials,
                   cudaStream_t stream) {
  StreamKParams sk{};
  sk.counters = counters, sk.partials = partials, sk.batch = batch, sk.hkv = hkv;
  paged_decode_streamk_kernel<R><<<grid, kAttnThreads, streamk_smem_bytes(R), stream>>>(p, sk);
  return launch_status();
}

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
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(p.splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = NVB200_PDL_ATTN ? 2 : 1;
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

namespace nvb200 {
namespace {

// Checks a call's arguments and fills the kernel parameters (splits not set). Returns NVB200_OK with *launch = false
// for an empty batch (nothing to do), NVB200_OK with *launch = true, or the error code.
int prepare_decode(const nvb200_paged_decode_args *a, AttnParams &p, bool *launch) {
  *launch = false;
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

  p = AttnParams{};
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
  p.scale_log2 = static_cast<float>(static_cast<double>(a->softmax_scale) * 1.4426950408889634);
  p.status = a->status;
  *launch = true;
  return NVB200_OK;
}

// Query-row bucket (the kernels' template R) of a call with `rows` rows.
int row_bucket(int rows) { return rows <= 1 ? 1 : rows <= 2 ? 2 : rows <= 4 ? 4 : rows <= 8 ? 8 : 16; }

int streamk_grid_for(int R) {
  switch (R) {
    case 1: return streamk_grid<1>();
    case 2: return streamk_grid<2>();
    case 4: return streamk_grid<4>();
    case 8: return streamk_grid<8>();
    default: return streamk_grid<16>();
  }
}

// Whether the stream-K kernel's unit indices fit: batch * Hkv * tiles of the longest addressable sequence < 2^31.
bool streamk_fits(const nvb200_paged_decode_args *a) {
  const int64_t cap_tiles = (static_cast<int64_t>(a->max_blocks_per_seq) * a->block_size + kTileTokens - 1) /
                            kTileTokens;
  return static_cast<int64_t>(a->batch) * a->num_kv_heads * cap_tiles < (int64_t{1} << 31);
}

// Bytes of the workspace's record region on the current device: the most that any row count's grid writes (cached
// per device; 0 if a launch shape could not be determined).
int64_t streamk_record_region() {
  static std::atomic<int64_t> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 0;
  int64_t v = dev < 64 ? cached[dev].load(std::memory_order_acquire) : 0;
  if (v == 0) {
    for (int R : {1, 2, 4, 8, 16}) {
      const int grid = streamk_grid_for(R);
      if (grid <= 0) return 0;
      v = std::max(v, round_up(streamk_partial_bytes(grid, R), kCounterAlign));
    }
    if (dev < 64) cached[dev].store(v, std::memory_order_release);
  }
  return v;
}

// Workspace bytes of a stream-K call: the record region, then the counters.
int64_t streamk_workspace_bytes(int64_t batch, int64_t hkv) {
  const int64_t region = streamk_record_region();
  return region > 0 ? region + round_up(batch * hkv * 4, kCounterAlign) : -1;
}

int launch_streamk_rows(int R, const AttnParams &p, int batch, int hkv, int grid, int32_t *counters, float *partials,
                        cudaStream_t s) {
  switch (R) {
    case 1: return launch_streamk<1>(p, batch, hkv, grid, counters, partials, s);
    case 2: return launch_streamk<2>(p, batch, hkv, grid, counters, partials, s);
    case 4: return launch_streamk<4>(p, batch, hkv, grid, counters, partials, s);
    case 8: return launch_streamk<8>(p, batch, hkv, grid, counters, partials, s);
    default: return launch_streamk<16>(p, batch, hkv, grid, counters, partials, s);
  }
}

}  // namespace
}  // namespace nvb200

extern "C" int nvb200_paged_decode_attention(const nvb200_paged_decode_args *a, nvb200_stream_t stream) {
  AttnParams p;
  bool launch = false;
  if (int rc = prepare_decode(a, p, &launch)) return rc;
  if (!launch) return NVB200_OK;
  const int64_t rows = p.rows;
  p.splits = nvb200_paged_decode_splits(a->batch, a->num_kv_heads, a->max_blocks_per_seq, a->block_size,
                                        a->num_splits);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (rows <= 1) return launch_rows<1>(p, a->batch, a->num_kv_heads, s);
  if (rows <= 2) return launch_rows<2>(p, a->batch, a->num_kv_heads, s);
  if (rows <= 4) return launch_rows<4>(p, a->batch, a->num_kv_heads, s);
  if (rows <= 8) return launch_rows<8>(p, a->batch, a->num_kv_heads, s);
  return launch_rows<16>(p, a->batch, a->num_kv_heads, s);
}

extern "C" int64_t nvb200_paged_decode_workspace_size(const nvb200_paged_decode_args *a) {
  if (!a || a->batch < 0 || a->num_kv_heads <= 0 || a->num_q_heads <= 0 || a->queries_per_seq <= 0 ||
      a->num_q_heads % a->num_kv_heads != 0)
    return -1;
  const int64_t rows = static_cast<int64_t>(a->queries_per_seq) * (a->num_q_heads / a->num_kv_heads);
  if (rows > kMaxRows) return -1;
  return streamk_workspace_bytes(a->batch, a->num_kv_heads);
}

extern "C" int nvb200_paged_decode_attention_streamk(const nvb200_paged_decode_args *a, void *workspace,
                                                     int64_t workspace_bytes, nvb200_stream_t stream) {
  AttnParams p;
  bool launch = false;
  if (int rc = prepare_decode(a, p, &launch)) return rc;
  if (!launch) return NVB200_OK;
  if (!streamk_fits(a)) return NVB200_ERR_UNSUPPORTED;
  const int R = row_bucket(p.rows);
  const int grid = streamk_grid_for(R);
  if (grid <= 0) return NVB200_ERR_CUDA;
  const int64_t need = streamk_workspace_bytes(a->batch, a->num_kv_heads);
  if (need <= 0) return NVB200_ERR_CUDA;
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & (kCounterAlign - 1)) != 0 || workspace_bytes < need)
    return NVB200_ERR_ARG;
  p.splits = 1;
  auto *base = static_cast<uint8_t *>(workspace);
  return launch_streamk_rows(R, p, a->batch, a->num_kv_heads, grid,
                             reinterpret_cast<int32_t *>(base + streamk_record_region()),
                             reinterpret_cast<float *>(base), reinterpret_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------------------------------------------
// Allocation-free decode attention: the stream-K kernel with its workspace in a fixed array of the library's own
// device memory, for callers that cannot allocate device memory at call time. nano-vllm-style engines reserve nearly
// all free HBM for the KV cache at start-up (gpu_memory_utilization), so a later allocation can fail; cudaMalloc and
// cudaFree may synchronise the device in the middle of a decode loop; and some host plugin interfaces hand a kernel
// only its input and output pointers, with no allocator to draw a workspace from.
//
// The array (NVB200_DECODE_NOALLOC_SCRATCH_BYTES, 4 MiB) is part of the library's device image, so every GPU that
// loads the library holds it until the process exits. It holds the arrival counters of at most
// NVB200_DECODE_NOALLOC_MAX_PAIRS (sequence, KV head) pairs, then the partial records; calls with 16 query rows per KV
// head get fewer CTAs than the SMs could hold (244 instead of 296) so that their records fit.
namespace nvb200 {
namespace {

constexpr int64_t kNoAllocBytes = NVB200_DECODE_NOALLOC_SCRATCH_BYTES;
constexpr int64_t kNoAllocPairs = NVB200_DECODE_NOALLOC_MAX_PAIRS;
constexpr int64_t kNoAllocCounterBytes = round_up(kNoAllocPairs * 4, kCounterAlign);
static_assert(kNoAllocCounterBytes < kNoAllocBytes, "the counters leave room for partial records");
static_assert(streamk_partial_bytes(1, kMaxRows) <= kNoAllocBytes - kNoAllocCounterBytes, "one CTA's records fit");

static __device__ __align__(256) uint8_t g_decode_scratch[kNoAllocBytes];

// Device address of g_decode_scratch on each device (0 = not looked up yet). The host-side name of the array is a
// stand-in, not a device address, so the address is taken once per device with that device current.
std::atomic<uintptr_t> g_decode_scratch_addr[64];

int decode_scratch(uint8_t **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NVB200_ERR_CUDA;
  uintptr_t a = g_decode_scratch_addr[dev].load(std::memory_order_acquire);
  if (a == 0) {
    void *ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_decode_scratch) != cudaSuccess || ptr == nullptr) return NVB200_ERR_CUDA;
    a = reinterpret_cast<uintptr_t>(ptr);
    g_decode_scratch_addr[dev].store(a, std::memory_order_release);
  }
  *out = reinterpret_cast<uint8_t *>(a);
  return NVB200_OK;
}

}  // namespace
}  // namespace nvb200

extern "C" int nvb200_paged_decode_attention_noalloc(const nvb200_paged_decode_args *a, nvb200_stream_t stream) {
  AttnParams p;
  bool launch = false;
  if (int rc = prepare_decode(a, p, &launch)) return rc;
  if (!launch) return NVB200_OK;
  if (!streamk_fits(a)) return NVB200_ERR_UNSUPPORTED;
  const int64_t pairs = static_cast<int64_t>(a->batch) * a->num_kv_heads;
  if (pairs > kNoAllocPairs) return NVB200_ERR_UNSUPPORTED;  // beyond the fixed array's counters
  const int R = row_bucket(p.rows);
  int grid = streamk_grid_for(R);
  if (grid <= 0) return NVB200_ERR_CUDA;
  const int64_t fit = (kNoAllocBytes - kNoAllocCounterBytes) / streamk_partial_bytes(1, R);
  grid = static_cast<int>(std::min<int64_t>(grid, fit));
  uint8_t *scratch = nullptr;
  if (int rc = decode_scratch(&scratch)) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // The kernel leaves every counter it used at zero, so after a completed call this memset finds zeros; it is kept
  // so that each call starts from zeroed counters even when a previous call on the array was aborted, faulted or
  // used more pairs in a way that left them non-zero (the array keeps whatever the last call left).
  if (cudaMemsetAsync(scratch, 0, static_cast<size_t>(pairs) * 4, s) != cudaSuccess) return NVB200_ERR_CUDA;
  p.splits = 1;
  return launch_streamk_rows(R, p, a->batch, a->num_kv_heads, grid, reinterpret_cast<int32_t *>(scratch),
                             reinterpret_cast<float *>(scratch + kNoAllocCounterBytes), s);
}
