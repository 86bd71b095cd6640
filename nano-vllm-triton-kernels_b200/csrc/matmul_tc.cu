// tcgen05 (5th-generation tensor core) matmul for sm_100a: C[M, N] = A[M, K] @ B[K, N], fp32 accumulation in TMEM.
//
// Behaviour follows nanovllm/kernels/matmul.py:33-81 (tiles in GROUP_M-swizzled order, K tail zero-filled, masked
// M/N edges); the machinery is Blackwell's:
//   * Persistent kernels with 128 x BN output tiles on one CTA (BN = 256, or 128 when that gives more tiles per SM)
//     or 256 x 256 tiles on a CTA pair (cta_group::2, below), and a skinny kernel for M <= 64 (further below).
//   * Warp 0 (one elected lane) moves A and B tiles HBM -> shared memory with TMA (cp.async.bulk.tensor, 128-byte
//     swizzle) into a ring of stages of two 64-wide K sub-tiles; completion is counted on mbarriers.
//   * Warp 1 (one elected lane) issues tcgen05.mma (kind::f16 for bf16, kind::tf32 for fp32) from the shared-memory
//     descriptors into a TMEM accumulator, and tcgen05.commit releases each stage when its MMAs are done. Two TMEM
//     accumulators (2 x BN columns) let the epilogue of one tile overlap the MMAs of the next.
//   * Warps 2-9 (the epilogue; two per 32-lane TMEM quarter, each draining half of the columns) read the
//     accumulator with tcgen05.ld, round to C's dtype, stage 32 x 32 chunks in swizzled shared memory and write
//     them with TMA stores (a thread holds one row, so direct stores would scatter every warp instruction over
//     32 rows). The gate_up variant pairs gate and up columns in one tile and applies SiLU x Mul there instead.
// Operand layouts: A and B may each be K-major (the contiguous dim is K: A row-major, B = weight.t()) or MN-major
// (B row-major [K, N], A column-major); the instruction descriptor's major bits select it, so no transpose pass.
// Any layout TMA cannot describe (a non-unit inner stride, or a row pitch that is not a multiple of 16 bytes) is
// reported as unsupported and the caller runs the SIMT kernel instead.
// No TMA multicast is used anywhere (this code may run in multi-GPU jobs).
#include <algorithm>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "qknr_math.cuh"

namespace nvb200 {
namespace {

constexpr int BM = 128;
// Epilogue warps: two per TMEM lane quarter (a warp may only read the quarter warp_id % 4), each draining half of a
// tile's columns. Four warps kept up with the MMAs of the plain GEMM but not with the SiLU x Mul epilogue at short K.
constexpr int kEpilogueWarps = 8;
constexpr int kThreads = 32 * (2 + kEpilogueWarps);
constexpr int kGroupM = 8;
constexpr int kTileBytesA = BM * 128;  // one 128-byte swizzle row per M row (BK * elem = 128 B)
constexpr int kMaxStages2 = 8;         // stage ring capacity (barriers reserved in the header)
#ifndef NVB200_MM_KSUB
#define NVB200_MM_KSUB 2
#endif

struct TcParams {
  void *c;
  int64_t scm, scn;
  int M, N, K;
  int bn;          // tile N (256 or 128)
  int tiles_m, tiles_n;
  int k_blocks;    // pipeline stages per tile: ceil(K / (BK * ksub))
  int k_subs;      // 64-element (128-byte) K sub-tiles per tile: ceil(K / BK)
  int ksub;        // 64-element (128-byte) K sub-tiles per stage: one commit releases 4 * ksub MMAs' operands
  int stages;      // pipeline depth
  uint32_t idesc;  // tcgen05 instruction descriptor
  int a_mn_major, b_mn_major;
  uint32_t a_sbo, b_sbo;    // descriptor stride byte offsets (MN-major: bytes between groups of k rows)
  uint32_t a_swz, b_swz;    // descriptor layout types (2 = 128-byte swizzle, 1 = 128-byte swizzle of 32-byte atoms)
  int elem_bytes;  // 2 (bf16) or 4 (fp32/tf32)
  int c_is_f32;
  int c_tma;          // 1: C is written by TMA stores from shared-memory staging (row-major C, 16-byte pitch)
  int swiglu;         // 1: gate_up GEMM with the SiLU x Mul epilogue (B holds 2 * N columns: gate | up)
  uint32_t epi_off;   // byte offset of the epilogue staging buffers in shared memory
  int epi_bufs;       // staging tiles per epilogue warp: 2 for bf16 C (double-buffered), 1 for fp32 C
  uint32_t hdr_off;   // byte offset of the barriers / TMEM slot
  int32_t *status;
};

// ---------------------------------------------------------------------------------------------------------------
// PTX wrappers for TMA tensor loads, tcgen05 and TMEM.

NVB200_DEVICE void tma_load_2d(uint32_t dst, const CUtensorMap *map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(map), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

NVB200_DEVICE void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

NVB200_DEVICE void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

NVB200_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

NVB200_DEVICE void tmem_alloc2(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

NVB200_DEVICE void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

NVB200_DEVICE uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in CTA `rank` of this cluster.
NVB200_DEVICE uint32_t map_to_cta(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

NVB200_DEVICE void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

NVB200_DEVICE void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// TMA load whose completion is counted on the pair leader's mbarrier (cta_group::2; no multicast).
NVB200_DEVICE void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, int c0, int c1, uint32_t leader_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst), "l"(map), "r"(c0), "r"(c1), "r"(leader_bar)
      : "memory");
}

template <bool TF32>
NVB200_DEVICE void tc_mma2(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  if (TF32) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// Arrives on `bar` (same offset) in both CTAs of the pair once this thread's tcgen05.mma ops have completed.
NVB200_DEVICE void tc_commit_pair(uint32_t bar) {
  const uint16_t mask = 3;
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
               ::"r"(bar), "h"(mask)
               : "memory");
}

NVB200_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
NVB200_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

template <bool TF32>
NVB200_DEVICE void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  if (TF32) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// Arrives on `bar` once every tcgen05.mma this thread issued so far has completed.
NVB200_DEVICE void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
NVB200_DEVICE void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor (sm100 version bits = 1). layout: 2 = 128-byte swizzle of 16-byte chunks (what
// TMA's SWIZZLE_128B writes), 1 = 128-byte swizzle of 32-byte chunks (TMA's SWIZZLE_128B_ATOM_32B), the form
// 32-bit (tf32) MN-major operands need.
NVB200_DEVICE uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;
  d |= static_cast<uint64_t>(layout) << 61;
  return d;
}

// K sub-tiles of stage kb that hold any of K (the last stage may end early); the rest are neither loaded nor used.
NVB200_DEVICE int stage_subtiles(const TcParams &p, int kb) {
  const int left = p.k_subs - kb * p.ksub;
  return left < p.ksub ? left : p.ksub;
}

// One K sub-tile (BK = 128 bytes of K) is 4 MMAs of UK = 32 bytes of K, for bf16 and tf32 alike.
constexpr int kMmaPerSub = 4;

// Shared-memory descriptors of stage 0's first A and B sub-tiles and the increments of their address field (16-byte
// units) per MMA K step, per sub-tile and per stage. The MMA loop only adds these: shared-memory addresses stay
// below 2^18 bytes, so the 14-bit address field never carries into the next field. Keeping the issue loop down to
// a few integer adds matters: the issuing thread's work between two tcgen05.mma instructions shows up as tensor-pipe
// idle time.
struct OperandDescs {
  uint64_t a0, b0;
  uint32_t a_k, b_k;      // one MMA's K step
  uint32_t a_sub, b_sub;  // one K sub-tile
  uint32_t stage;         // one stage
};

NVB200_DEVICE OperandDescs operand_descs(const TcParams &p, uint32_t stage0, int sub_b, int stage_bytes) {
  const int BK = 128 / p.elem_bytes, UK = 32 / p.elem_bytes;
  const uint32_t b_base = stage0 + p.ksub * kTileBytesA;
  // K-major: the K step moves 32 B inside the swizzle row; SBO = 8 rows * 128 B.
  // MN-major: the K step moves UK rows of 128 B; LBO = next 128-byte MN block (BK rows), SBO = one swizzle atom of
  // k rows (8 rows, or 4 rows for the 32-byte-atom swizzle).
  OperandDescs d;
  d.a0 = p.a_mn_major ? smem_desc(stage0, BK * 128, p.a_sbo, p.a_swz) : smem_desc(stage0, 16, 1024, 2);
  d.b0 = p.b_mn_major ? smem_desc(b_base, BK * 128, p.b_sbo, p.b_swz) : smem_desc(b_base, 16, 1024, 2);
  d.a_k = (p.a_mn_major ? UK * 128 : 32) >> 4;
  d.b_k = (p.b_mn_major ? UK * 128 : 32) >> 4;
  d.a_sub = kTileBytesA >> 4;
  d.b_sub = static_cast<uint32_t>(sub_b) >> 4;
  d.stage = static_cast<uint32_t>(stage_bytes) >> 4;
  return d;
}

// Column of B that tile column c (0..BN) of output tile pn reads. Plain GEMM: pn * BN + c. Gate_up GEMM with the
// SiLU x Mul epilogue: a 256-column tile pairs the 128 gate columns [pn * 128, +128) with the matching up columns
// [N + pn * 128, +128), N being the output width (B holds gate | up, 2 N columns).
NVB200_DEVICE int b_col(const TcParams &p, int pn, int c) {
  if (!p.swiglu) return pn * p.bn + c;
  return c < 128 ? pn * 128 + c : p.N + pn * 128 + (c - 128);
}

// GROUP_M-swizzled tile order (nanovllm/kernels/matmul.py:50-57).
NVB200_DEVICE void tile_coords(int tile, int tiles_m, int tiles_n, int &pm, int &pn) {
  const int in_group = kGroupM * tiles_n;
  const int first_m = (tile / in_group) * kGroupM;
  const int group_m = min(tiles_m - first_m, kGroupM);
  pm = first_m + (tile % in_group) % group_m;
  pn = (tile % in_group) / group_m;
}

// Epilogue: this thread's accumulator row (one TMEM lane) -> C[row, col0 .. col0 + ncols), 32 columns per
// tcgen05.ld, rounded to C's dtype. Every lane of the warp must call it (tcgen05.ld is warp-wide).
NVB200_DEVICE void store_tile_rows(const TcParams &p, uint32_t taddr, int row, int col_base, int ncols) {
  for (int c0 = 0; c0 < ncols; c0 += 32) {
    float v[32];
    tmem_ld32(taddr + c0, v);
    const int col0 = col_base + c0;
    if (row >= p.M || col0 >= p.N) continue;
    if (p.c_is_f32) {
      float *c = static_cast<float *>(p.c) + row * p.scm;
      if (p.scn == 1 && col0 + 32 <= p.N && ((reinterpret_cast<uintptr_t>(c + col0) & 15) == 0)) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4 *>(c + col0 + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (col0 + i < p.N) c[(col0 + i) * p.scn] = v[i];
      }
    } else {
      __nv_bfloat16 *c = static_cast<__nv_bfloat16 *>(p.c) + row * p.scm;
      if (p.scn == 1 && col0 + 32 <= p.N && ((reinterpret_cast<uintptr_t>(c + col0) & 15) == 0)) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          const float f[8] = {v[i], v[i + 1], v[i + 2], v[i + 3], v[i + 4], v[i + 5], v[i + 6], v[i + 7]};
          *reinterpret_cast<uint4 *>(c + col0 + i) = pack8(f);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (col0 + i < p.N) c[(col0 + i) * p.scn] = __float2bfloat16_rn(v[i]);
      }
    }
  }
}

NVB200_DEVICE void tma_store_2d(const CUtensorMap *map, int c0, int c1, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(c0),
               "r"(c1), "r"(src)
               : "memory");
}

// Epilogue through shared memory: per 32-column chunk, each lane converts its row (one TMEM lane) and writes it
// into a 32 x 32 staging tile (rows of 64 B for bf16 / 128 B for fp32, 16-byte chunks XOR-swizzled as TMA's
// SWIZZLE_64B / SWIZZLE_128B expect, so the 32 lanes' writes hit distinct banks); lane 0 then TMA-stores the tile,
// which clips rows >= M and columns >= N. Two staging tiles per warp alternate; a tile is rewritten only after the
// store issued from it two chunks earlier has read it. `stage` = the warp's two tiles, `chunks` counts its stores.
NVB200_DEVICE void store_tile_tma(const TcParams &p, const CUtensorMap *map_c, uint32_t taddr, int row0, int col_base,
                                  int ncols, uint32_t stage, int &chunks) {
  const int lane = threadIdx.x & 31;
  const int row_bytes = p.c_is_f32 ? 128 : 64;
  for (int c0 = 0; c0 < ncols; c0 += 32) {
    float v[32];
    tmem_ld32(taddr + c0, v);
    if (row0 >= p.M || col_base + c0 >= p.N) continue;
    const uint32_t buf = stage + (p.epi_bufs == 2 ? (chunks & 1) * 32 * row_bytes : 0);
    if (lane == 0) {
      if (p.epi_bufs == 2 && chunks >= 2) bulk_wait_read<1>();
      if (p.epi_bufs == 1 && chunks >= 1) bulk_wait_read<0>();
    }
    __syncwarp();
    const uint32_t row_addr = buf + lane * row_bytes;
    if (p.c_is_f32) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint4 w = make_uint4(__float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]),
                                   __float_as_uint(v[4 * j + 2]), __float_as_uint(v[4 * j + 3]));
        st_shared_v4(row_addr + ((j ^ (lane & 7)) << 4), w);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float f[8] = {v[8 * j], v[8 * j + 1], v[8 * j + 2], v[8 * j + 3],
                            v[8 * j + 4], v[8 * j + 5], v[8 * j + 6], v[8 * j + 7]};
        st_shared_v4(row_addr + ((j ^ ((lane >> 1) & 3)) << 4), pack8(f));
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(map_c, col_base + c0, row0, buf);
      bulk_commit();
    }
    ++chunks;
  }
}

// Epilogue of the gate_up GEMM: per 32 output columns, the gate accumulators (TMEM columns c0..) and the up
// accumulators (columns 128 + c0..) are rounded to bf16 (what the plain GEMM would write) and combined by the
// SiLU x Mul kernel's own routine, so the result equals silu_and_mul(matmul(a, b)) bit for bit; staging and TMA
// stores as store_tile_tma (bf16 C).
NVB200_DEVICE void store_tile_tma_swiglu(const TcParams &p, const CUtensorMap *map_c, uint32_t taddr, int row0,
                                         int col_base, int c_begin, int c_end, uint32_t stage, int &chunks) {
  const int lane = threadIdx.x & 31;
  for (int c0 = c_begin; c0 < c_end; c0 += 32) {
    float g[32], u[32];
    tmem_ld32(taddr + c0, g);
    tmem_ld32(taddr + 128 + c0, u);
    if (row0 >= p.M || col_base + c0 >= p.N) continue;
    const uint32_t buf = stage + (chunks & 1) * 32 * 64;
    if (chunks >= 2 && lane == 0) bulk_wait_read<1>();
    __syncwarp();
    const uint32_t row_addr = buf + lane * 64;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gf[8] = {g[8 * j], g[8 * j + 1], g[8 * j + 2], g[8 * j + 3],
                           g[8 * j + 4], g[8 * j + 5], g[8 * j + 6], g[8 * j + 7]};
      const float uf[8] = {u[8 * j], u[8 * j + 1], u[8 * j + 2], u[8 * j + 3],
                           u[8 * j + 4], u[8 * j + 5], u[8 * j + 6], u[8 * j + 7]};
      st_shared_v4(row_addr + ((j ^ ((lane >> 1) & 3)) << 4), silu_mul8_bf16(pack8(gf), pack8(uf)));
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(map_c, col_base + c0, row0, buf);
      bulk_commit();
    }
    ++chunks;
  }
}

// Stage layout (each operand tile 1024-byte aligned, as the 128-byte swizzle requires):
//   A: BM x BK, K-major: row m at m * 128 B.            MN-major: BK rows of 128 B per 128-byte MN block.
//   B: BN x BK, K-major: row n at n * 128 B.            MN-major: BK rows of 128 B per 128-byte MN block.
// BK = 128 / elem_bytes (64 bf16, 32 tf32). One MMA consumes UK = 32 / elem_bytes of K (16 bf16, 8 tf32).
template <bool TF32>
__global__ void __launch_bounds__(kThreads, 1)
    matmul_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_c, const __grid_constant__ TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int sub_b = p.bn * 128;                          // one 64-wide K sub-tile of B
  const int stage_bytes = p.ksub * (kTileBytesA + sub_b);  // [A sub-tiles | B sub-tiles]
  const int stages = p.stages;
  uint8_t *hdr = smem + p.hdr_off;
  const uint32_t bar_full = smem_addr(hdr);                    // stages x 8
  const uint32_t bar_empty = bar_full + 8 * kMaxStages2;       // stages x 8
  const uint32_t bar_acc_full = bar_empty + 8 * kMaxStages2;   // 2 x 8
  const uint32_t bar_acc_empty = bar_acc_full + 16;            // 2 x 8
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(hdr + 16 * kMaxStages2 + 32);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(hdr + 16 * kMaxStages2 + 36);
  const uint32_t stage0 = smem_addr(smem);
  const int BK = 128 / p.elem_bytes;
  const int num_tiles = p.tiles_m * p.tiles_n;

  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(bar_full + 8 * i, 1);
      mbar_init(bar_empty + 8 * i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_acc_full + 8 * i, 1);
      mbar_init(bar_acc_empty + 8 * i, kEpilogueWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&map_a);
    prefetch_tmap(&map_b);
  }
  if (warp == 1) tmem_alloc(smem_addr(tmem_slot), 2 * p.bn <= 256 ? 256 : 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int st = 0;
      uint32_t ph = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        int pm, pn;
        tile_coords(tile, p.tiles_m, p.tiles_n, pm, pn);
        const int m0 = pm * BM, n0 = pn * p.bn;
        for (int kb = 0; kb < p.k_blocks; ++kb, st = st + 1 == stages ? 0 : st + 1, ph ^= st == 0) {
          if (!mbar_wait_bounded(bar_empty + 8 * st, ph ^ 1)) {
            set_status(p.status, NVB200_STATUS_WAIT_TIMEOUT);
            *abort_flag = 1;
            break;
          }
          const uint32_t full = bar_full + 8 * st;
          const int nsub = stage_subtiles(p, kb);
          mbar_arrive_expect_tx(full, nsub * (kTileBytesA + sub_b));
          for (int u = 0; u < nsub; ++u) {
            const uint32_t sa = stage0 + st * stage_bytes + u * kTileBytesA;
            const uint32_t sb = stage0 + st * stage_bytes + p.ksub * kTileBytesA + u * sub_b;
            const int k0 = (kb * p.ksub + u) * BK;
            if (p.a_mn_major) {  // A^T stored [K][M]: boxes of 128 B along M, BK rows
              for (int j = 0; j < BM / BK; ++j) tma_load_2d(sa + j * BK * 128, &map_a, m0 + j * BK, k0, full);
            } else {
              tma_load_2d(sa, &map_a, k0, m0, full);
            }
            if (p.b_mn_major) {  // B stored [K][N]: boxes of 128 B along N, BK rows
              for (int j = 0; j < p.bn / BK; ++j) tma_load_2d(sb + j * BK * 128, &map_b, b_col(p, pn, j * BK), k0, full);
            } else if (p.swiglu) {  // two boxes of 128 rows: gate, then up
              tma_load_2d(sb, &map_b, k0, b_col(p, pn, 0), full);
              tma_load_2d(sb + 128 * 128, &map_b, k0, b_col(p, pn, 128), full);
            } else {
              tma_load_2d(sb, &map_b, k0, n0, full);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    const OperandDescs od = operand_descs(p, stage0, sub_b, stage_bytes);
    int st = 0, local = 0;
    uint32_t ph = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int buf = local & 1;
      const uint32_t acc_ph = (local >> 1) & 1;
      bool ok = mbar_wait_bounded(bar_acc_empty + 8 * buf, acc_ph ^ 1);
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * p.bn;
      for (int kb = 0; kb < p.k_blocks && ok; ++kb, st = st + 1 == stages ? 0 : st + 1, ph ^= st == 0) {
        if (!mbar_wait_bounded(bar_full + 8 * st, ph)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const int nsub = stage_subtiles(p, kb);
          const uint64_t a_st = od.a0 + st * od.stage, b_st = od.b0 + st * od.stage;
          for (int u = 0; u < nsub; ++u) {
#pragma unroll
            for (int k = 0; k < kMmaPerSub; ++k)
              tc_mma<TF32>(d_tmem, a_st + u * od.a_sub + k * od.a_k, b_st + u * od.b_sub + k * od.b_k, p.idesc,
                           (kb > 0 || u > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(bar_empty + 8 * st);
        }
        __syncwarp();
      }
      if (!ok) {
        if (lane == 0) set_status(p.status, NVB200_STATUS_WAIT_TIMEOUT);
        *abort_flag = 1;
        break;
      }
      if (lane == 0) tc_commit(bar_acc_full + 8 * buf);
      __syncwarp();
    }
  } else {
    // ---------------------------------------------------------------- epilogue: TMEM -> registers -> C
    const int q = warp & 3;         // TMEM lane quarter this warp may read
    const int half = (warp - 2) >> 2;  // which half of the tile's columns it drains
    const uint32_t epi_stage = smem_addr(smem) + p.epi_off + (warp - 2) * p.epi_bufs * 32 * (p.c_is_f32 ? 128 : 64);
    int chunks = 0;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      int pm, pn;
      tile_coords(tile, p.tiles_m, p.tiles_n, pm, pn);
      const int buf = local & 1;
      if (!mbar_wait_bounded(bar_acc_full + 8 * buf, (local >> 1) & 1)) {
        if (lane == 0) set_status(p.status, NVB200_STATUS_WAIT_TIMEOUT);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * p.bn;
      const int hc = p.bn / 2;  // accumulator columns per half
      if (p.swiglu)
        store_tile_tma_swiglu(p, &map_c, taddr, pm * BM + q * 32, pn * 128, half * 64, half * 64 + 64, epi_stage,
                              chunks);
      else if (p.c_tma)
        store_tile_tma(p, &map_c, taddr + half * hc, pm * BM + q * 32, pn * p.bn + half * hc, hc, epi_stage, chunks);
      else
        store_tile_rows(p, taddr + half * hc, pm * BM + q * 32 + lane, pn * p.bn + half * hc, hc);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_acc_empty + 8 * buf);
    }
  }

  if (warp >= 2 && lane == 0) bulk_wait<0>();  // epilogue TMA stores complete
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * p.bn <= 256 ? 256 : 512);
  }
}


// ---------------------------------------------------------------------------------------------------------------
// CTA-pair kernel (cluster of 2 on neighbouring SMs, tcgen05.mma.cta_group::2): the pair computes a 256 x BN tile.
// CTA r holds rows [128 r, 128 r + 128) of the A tile and columns [r BN/2, (r + 1) BN/2) of the B tile, so each
// SM loads a third less operand data per FLOP than a lone 128 x BN tile. The leader (rank 0) issues the MMAs;
// both CTAs' TMA loads count on the leader's full barrier; tcgen05.commit multicasts stage releases and
// accumulator-ready signals to both CTAs; each CTA's epilogue drains its own 128 TMEM lanes and tells the leader
// through a cluster-scope arrive when its accumulator buffer is free. No TMA load uses multicast.
template <bool TF32>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    matmul_tc2_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                      const __grid_constant__ CUtensorMap map_c, const __grid_constant__ TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int half_bn = p.bn / 2;
  const int sub_b = half_bn * 128;                         // one 64-wide K sub-tile of this CTA's half of B
  const int stage_bytes = p.ksub * (kTileBytesA + sub_b);  // [A sub-tiles | B sub-tiles]
  const int stages = p.stages;
  uint8_t *hdr = smem + p.hdr_off;
  const uint32_t bar_full = smem_addr(hdr);                 // stages x 8 (used in the leader)
  const uint32_t bar_empty = bar_full + 8 * kMaxStages2;    // stages x 8 (both CTAs)
  const uint32_t bar_acc_full = bar_empty + 8 * kMaxStages2;  // 2 x 8 (both CTAs)
  const uint32_t bar_acc_empty = bar_acc_full + 16;           // 2 x 8 (used in the leader)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(hdr + 16 * kMaxStages2 + 32);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(hdr + 16 * kMaxStages2 + 36);
  const uint32_t stage0 = smem_addr(smem);
  const int BK = 128 / p.elem_bytes;
  const int num_tiles = p.tiles_m * p.tiles_n;  // 256-row tiles
  const int cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(bar_full + 8 * i, 1);
      mbar_init(bar_empty + 8 * i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_acc_full + 8 * i, 1);
      mbar_init(bar_acc_empty + 8 * i, 2 * kEpilogueWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&map_a);
    prefetch_tmap(&map_b);
  }
  if (warp == 1) tmem_alloc2(smem_addr(tmem_slot), 2 * p.bn <= 256 ? 256 : 512);
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any cross-CTA traffic
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (both CTAs)
    if (lane == 0) {
      int st = 0;
      uint32_t ph = 0;
      for (int tile = cluster; tile < num_tiles && !*abort_flag; tile += clusters) {
        int pm, pn;
        tile_coords(tile, p.tiles_m, p.tiles_n, pm, pn);
        const int m0 = pm * 2 * BM + static_cast<int>(rank) * BM;
        const int n0 = b_col(p, pn, static_cast<int>(rank) * half_bn);  // this CTA's half of the B tile
        for (int kb = 0; kb < p.k_blocks; ++kb, st = st + 1 == stages ? 0 : st + 1, ph ^= st == 0) {
          if (!mbar_wait_bounded(bar_empty + 8 * st, ph ^ 1)) {
            set_status(p.status, NVB200_STATUS_WAIT_TIMEOUT);
            *abort_flag = 1;
            break;
          }
          const uint32_t full = map_to_cta(bar_full + 8 * st, 0);
          const int nsub = stage_subtiles(p, kb);
          if (leader) mbar_arrive_expect_tx(bar_full + 8 * st, 2 * nsub * (kTileBytesA + sub_b));
          for (int u = 0; u < nsub; ++u) {
            const uint32_t sa = stage0 + st * stage_bytes + u * kTileBytesA;
            const uint32_t sb = stage0 + st * stage_bytes + p.ksub * kTileBytesA + u * sub_b;
            const int k0 = (kb * p.ksub + u) * BK;
            if (p.a_mn_major) {
              for (int j = 0; j < BM / BK; ++j) tma_load_2d_pair(sa + j * BK * 128, &map_a, m0 + j * BK, k0, full);
            } else {
              tma_load_2d_pair(sa, &map_a, k0, m0, full);
            }
            if (p.b_mn_major) {
              for (int j = 0; j < half_bn / BK; ++j)
                tma_load_2d_pair(sb + j * BK * 128, &map_b, n0 + j * BK, k0, full);
            } else {
              tma_load_2d_pair(sb, &map_b, k0, n0, full);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (leader only)
    if (leader) {
      const OperandDescs od = operand_descs(p, stage0, sub_b, stage_bytes);
      int st = 0, local = 0;
      uint32_t ph = 0;
      for (int tile = cluster; tile < num_tiles; tile += clusters, ++local) {
        const int buf = local & 1;
        bool ok = mbar_wait_bounded(bar_acc_empty + 8 * buf, ((local >> 1) & 1) ^ 1);
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * p.bn;
        for (int kb = 0; kb < p.k_blocks && ok; ++kb, st = st + 1 == stages ? 0 : st + 1, ph ^= st == 0) {
          if (!mbar_wait_bounded(bar_full + 8 * st, ph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const int nsub = stage_subtiles(p, kb);
            const uint64_t a_st = od.a0 + st * od.stage, b_st = od.b0 + st * od.stage;
            for (int u = 0; u < nsub; ++u) {
#pragma unroll
              for (int k = 0; k < kMmaPerSub; ++k)
                tc_mma2<TF32>(d_tmem, a_st + u * od.a_sub + k * od.a_k, b_st + u * od.b_sub + k * od.b_k, p.idesc,
                              (kb > 0 || u > 0 || k > 0) ? 1u : 0u);
            }
            tc_commit_pair(bar_empty + 8 * st);
          }
          __syncwarp();
        }
        if (!ok) {
          if (lane == 0) set_status(p.status, NVB200_STATUS_WAIT_TIMEOUT);
          *abort_flag = 1;
          break;
        }
        if (lane == 0) tc_commit_pair(bar_acc_full + 8 * buf);
        __syncwarp();
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (both CTAs, own TMEM lanes)
    const int q = warp & 3;            // TMEM lane quarter this warp may read
    const int half = (warp - 2) >> 2;  // which half of the tile's columns it drains
    const uint32_t leader_acc_empty = map_to_cta(bar_acc_empty, 0);
    const uint32_t epi_stage = smem_addr(smem) + p.epi_off + (warp - 2) * p.epi_bufs * 32 * (p.c_is_f32 ? 128 : 64);
    int chunks = 0;
    int local = 0;
    for (int tile = cluster; tile < num_tiles; tile += clusters, ++local) {
      int pm, pn;
      tile_coords(tile, p.tiles_m, p.tiles_n, pm, pn);
      const int buf = local & 1;
      if (!mbar_wait_bounded(bar_acc_full + 8 * buf, (local >> 1) & 1)) {
        if (lane == 0) set_status(p.status, NVB200_STATUS_WAIT_TIMEOUT);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * p.bn;
      const int row0 = pm * 2 * BM + static_cast<int>(rank) * BM + q * 32;
      const int hc = p.bn / 2;  // accumulator columns per half
      if (p.swiglu)
        store_tile_tma_swiglu(p, &map_c, taddr, row0, pn * 128, half * 64, half * 64 + 64, epi_stage, chunks);
      else if (p.c_tma)
        store_tile_tma(p, &map_c, taddr + half * hc, row0, pn * p.bn + half * hc, hc, epi_stage, chunks);
      else
        store_tile_rows(p, taddr + half * hc, row0 + lane, pn * p.bn + half * hc, hc);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(leader_acc_empty + 8 * buf);
    }
  }

  if (warp >= 2 && lane == 0) bulk_wait<0>();  // epilogue TMA stores complete
  tc_fence_before();
  cluster_sync();  // the peer's MMAs and remote arrivals are done before TMEM and shared memory go away
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem_base, 2 * p.bn <= 256 ? 256 : 512);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Host side: tensor maps (cuTensorMapEncodeTiled through the runtime's driver entry point, so the library has no
// link-time dependency on libcuda) and the launch.

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 2-D map of a row-pitched matrix: inner dim `inner` contiguous elements, `outer` rows `pitch` elements apart,
// box of `box_inner` x `box_outer`, 128-byte swizzle (of 16-byte chunks, or of 32-byte chunks when atom32),
// out-of-range elements read as zero.
bool make_map(CUtensorMap *map, const void *base, bool f32, int64_t inner, int64_t outer, int64_t pitch,
              int box_inner, int box_outer, bool atom32 = false) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const int es = f32 ? 4 : 2;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch * es)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                        const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Map of C for the epilogue's TMA stores: [M, N] row-major with pitch `pitch`, boxes of 32 x 32 elements, the
// swizzle matching the staging tiles (64-byte rows for bf16, 128-byte rows for fp32).
bool make_map_c(CUtensorMap *map, void *base, bool f32, int64_t M, int64_t N, int64_t pitch) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const int es = f32 ? 4 : 2;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch * es)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

constexpr int kMaxDynamicSmem = 227 * 1024;

// Raises `kernel`'s dynamic shared-memory limit to at least smem bytes, once per device and size; `slot` identifies
// the kernel (each kernel instantiation has its own slot: the limit is an attribute of the function).
constexpr int kConfigureSlots = 8;
template <typename Kernel> int configure_once(Kernel kernel, int smem, int slot) {
  static int configured[kConfigureSlots][64] = {{0}};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && configured[slot][dev] >= smem) return NVB200_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return NVB200_ERR_CUDA;
  if (dev < 64) configured[slot][dev] = smem;
  return NVB200_OK;
}

// ---------------------------------------------------------------------------------------------------------------
// Skinny GEMM (M <= 64 rows, the decode-sized case): C^T = B^T A^T on the tensor cores, so the weight's N
// dimension fills the MMA's 128 rows and M is the MMA's N (16..64), split over K across a thread-block cluster of S
// CTAs whose fp32 partials are summed through distributed shared memory (no global scratch).
//   * CTA (tile t, rank r) of a cluster multiplies the 128 x K-slice r of B^T (K-major: B = weight.t()) with the
//     M_pad x K-slice of A, 64-element (128-byte) K blocks through a TMA ring; one elected thread issues
//     tcgen05.mma (M = 128, N = M_pad) into TMEM. The producer starts loading as soon as its barriers exist.
//   * S = 1: each thread holds row n of C^T (one TMEM lane) and writes C[:, n] (consecutive n per warp).
//   * S > 1: CTA r owns rows [r 128/S, (r+1) 128/S) of C^T. Every CTA pushes each row of its partial into the
//     owner's shared memory (st.shared::cluster, slot [source rank][m][row]); after one cluster barrier each owner
//     sums its S slots locally and writes C. Nothing reads a peer's memory, so no second barrier is needed.
// Every wait is bounded; on a timeout a CTA sets the status bit and still takes the cluster barrier, so its peers
// never wait on it forever.

constexpr int kSkinnyThreads = 128;  // 4 warps: warp 0 lane 0 loads, warp 1 lane 0 issues MMAs, all 4 drain TMEM
constexpr int kSkinnyMaxStages = 8;
constexpr int kSkinnyMaxM = 64;
constexpr int kArMaxRanks = 8;
constexpr int kArMaxGrid = 256;  // CTAs of a fused all-reduce call at most (all resident)
#ifndef NVB200_SKINNY_KPB
#define NVB200_SKINNY_KPB 2
#endif

struct SkinnyParams {
  void *c;
  int64_t scm, scn;
  int M, N, K;
  int m_pad;        // M rounded up to 16 (the MMA's N)
  int split;        // CTAs per cluster (K split)
  int k_blocks;     // 128-byte K blocks in total
  int kpb;          // K blocks per stage (1 or 2): one tcgen05.commit releases 4 kpb MMAs' operands
  int stages;
  uint32_t idesc;
  int elem_bytes;
  int c_is_f32;
  int swiglu;       // 1: gate_up GEMM with the SiLU x Mul epilogue (B holds 2 N columns, gate | up; a tile is the 64
                    // gate columns n0 .. n0 + 63 and the matching 64 up columns; C = silu(gate) * up, [M, N] bf16)
  int red_off;      // shared-memory offset of the partial slots [S][m_pad][128 / S] fp32 (S > 1, or all-reduce)
  int hdr_off;      // barriers and the TMEM slot
  int32_t *status;
  // Row-parallel all-reduce across GPUs (ar_world > 1): every rank's exchange buffer, mapped in this process.
  int ar_world, ar_rank;
  int64_t ar_max_n;
  uint8_t *ar_base[kArMaxRanks];
};

// Exchange buffer of one rank: a 256-byte header (the number of calls completed on this rank, and the count of
// CTAs of the current call that are done), then two parities of [source rank][kSkinnyMaxM][max_n] 8-byte words,
// each an fp32 partial in the low half and the epoch (call number) of the call that wrote it in the high half
// (written with one 8-byte store, so a reader that sees the epoch sees the value: no fences or separate flags).
// Calls alternate parities, so a rank that runs ahead never overwrites a word a peer may still be waiting for.
// The epoch lives in device memory and the kernel advances it, so a call captured in a CUDA graph gets a new epoch
// on every replay; every rank makes the same calls, so the counters of all ranks advance together.
constexpr int kArHeaderBytes = 256;
struct ArHeader {
  uint32_t completed;  // calls completed on this rank: this call's epoch is completed + 1
  uint32_t arrived;    // CTAs of the current call that are done
};
NVB200_DEVICE ArHeader *ar_header_at(uint8_t *const *bases, int owner) {
  return reinterpret_cast<ArHeader *>(bases[owner]);
}
NVB200_DEVICE uint64_t *ar_slot_at(uint8_t *const *bases, int64_t max_n, uint32_t epoch, int owner, int source) {
  const int64_t parity = epoch & 1;
  return reinterpret_cast<uint64_t *>(bases[owner] + kArHeaderBytes) +
         ((parity * kArMaxRanks + source) * kSkinnyMaxM) * max_n;
}
NVB200_DEVICE ArHeader *ar_header(const SkinnyParams &p, int owner) { return ar_header_at(p.ar_base, owner); }
NVB200_DEVICE uint64_t *ar_slot(const SkinnyParams &p, uint32_t epoch, int owner, int source) {
  return ar_slot_at(p.ar_base, p.ar_max_n, epoch, owner, source);
}

// Waits until the 8-byte exchange word at w carries `epoch` (bounded: after kWaitLimitNs the status bit is set and
// *expired stops every later wait of the thread) and returns its fp32 value.
NVB200_DEVICE float ar_take(const uint64_t *w, uint32_t epoch, bool *expired, uint64_t *start, int32_t *status) {
  uint64_t a;
  for (uint32_t spin = 1;; ++spin) {
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(a) : "l"(w) : "memory");
    if ((a >> 32) == epoch || *expired) break;
    if ((spin & 1023u) == 0) {
      const uint64_t now = global_timer_ns();
      if (*start == 0) *start = now;
      else if (now - *start > kWaitLimitNs) {
        set_status(status, NVB200_STATUS_WAIT_TIMEOUT);
        *expired = true;
      }
    }
  }
  return __uint_as_float(static_cast<uint32_t>(a));
}

NVB200_DEVICE void store_c(const SkinnyParams &p, int m, int n, float v) {
  const int64_t idx = m * p.scm + static_cast<int64_t>(n) * p.scn;
  if (p.c_is_f32)
    static_cast<float *>(p.c)[idx] = v;
  else
    static_cast<__nv_bfloat16 *>(p.c)[idx] = __float2bfloat16_rn(v);
}

// One stage of the skinny kernel: nsub consecutive K blocks from kb, each [B^T tile | A tile]. With up0 >= 0 (the
// gate_up form) the B^T tile is two 64-row boxes: the gate rows from n0 and the up rows from up0.
NVB200_DEVICE void skinny_load_stage(const CUtensorMap &map_w, const CUtensorMap &map_x, uint32_t full, uint32_t sw,
                                     int kb, int nsub, uint32_t sub_bytes, uint32_t tile_w, int BK, int n0, int up0) {
  mbar_arrive_expect_tx(full, nsub * sub_bytes);
  for (int u = 0; u < nsub; ++u) {
    tma_load_2d(sw + u * sub_bytes, &map_w, (kb + u) * BK, n0, full);
    if (up0 >= 0) tma_load_2d(sw + u * sub_bytes + tile_w / 2, &map_w, (kb + u) * BK, up0, full);
    tma_load_2d(sw + u * sub_bytes + tile_w, &map_x, (kb + u) * BK, 0, full);
  }
}

// out[m, n] for the 4 consecutive columns n .. n + 3 of row m from gate and up sums in fp32: each rounded to bf16,
// then the SiLU x Mul routine of the two-step form (so the result is bitwise that of the GEMM into bf16 followed by
// nvb200_silu_and_mul). Columns at or past N are not stored.
NVB200_DEVICE void store_swiglu4(const SkinnyParams &p, int m, int n, const float (&g)[4], const float (&u)[4]) {
  const uint4 gv = make_uint4(pack_bf16x2(g[0], g[1]), pack_bf16x2(g[2], g[3]), 0u, 0u);
  const uint4 uv = make_uint4(pack_bf16x2(u[0], u[1]), pack_bf16x2(u[2], u[3]), 0u, 0u);
  const uint4 o = silu_mul8_bf16(gv, uv);
  __nv_bfloat16 *c = static_cast<__nv_bfloat16 *>(p.c) + m * p.scm + n;
  const uint32_t w[2] = {o.x, o.y};
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (n + i < p.N) c[i] = __ushort_as_bfloat16(static_cast<unsigned short>(i & 1 ? w[i >> 1] >> 16 : w[i >> 1] & 0xFFFFu));
}

template <bool TF32>
__global__ void __launch_bounds__(kSkinnyThreads)
    matmul_skinny_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                         const __grid_constant__ SkinnyParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int S = p.split;
  // First row of B^T (column of C) of this tile; the gate_up form's tiles are 64 gate rows and the 64 matching up
  // rows, which start at up0.
  const int n0 = (blockIdx.x / S) * (p.swiglu ? BM / 2 : BM);
  const int up0 = p.swiglu ? p.N + n0 : -1;
  const int BK = 128 / p.elem_bytes;
  const uint32_t tile_w = BM * 128, tile_x = static_cast<uint32_t>(p.m_pad) * 128;
  const uint32_t sub_bytes = tile_w + tile_x;  // one K block: [B^T tile | A tile]
  const int kpb = p.kpb;
  const uint32_t stage_bytes = kpb * sub_bytes;
  const int stages = p.stages;
  uint8_t *hdr = smem + p.hdr_off;
  const uint32_t bar_full = smem_addr(hdr);
  const uint32_t bar_empty = bar_full + 8 * kSkinnyMaxStages;
  const uint32_t bar_acc = bar_empty + 8 * kSkinnyMaxStages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(hdr + 16 * kSkinnyMaxStages + 8);
  const uint32_t stage0 = smem_addr(smem);
  const uint32_t tmem_cols = p.m_pad <= 32 ? 32 : 64;
  // This CTA's K blocks: an even share of the tile's blocks.
  const int kb_begin = static_cast<int>((static_cast<int64_t>(p.k_blocks) * rank) / S);
  const int kb_end = static_cast<int>((static_cast<int64_t>(p.k_blocks) * (rank + 1)) / S);

  // Thread 0 creates the barriers and, as the producer, fills the ring at once; the rest of the set-up (TMEM) runs
  // while those loads are in flight.
  int pst = 0, pkb = kb_begin;  // producer: next stage slot, first K block of the next stage
  uint32_t pph = 0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(bar_full + 8 * i, 1);
      mbar_init(bar_empty + 8 * i, 1);
    }
    mbar_init(bar_acc, 1);
    fence_mbar_init();
    for (int i = 0; pkb < kb_end && i < stages; ++i, pkb += kpb, pst = pst + 1 == stages ? 0 : pst + 1, pph ^= pst == 0)
      skinny_load_stage(map_w, map_x, bar_full + 8 * pst, stage0 + pst * stage_bytes, pkb, min(kpb, kb_end - pkb),
                        sub_bytes, tile_w, BK, n0, up0);
  }
  if (warp == 1) tmem_alloc(smem_addr(tmem_slot), tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  bool ok = true;

  if (warp == 0 && lane == 0) {
    // ---------------------------------------------------------------- TMA producer (the rest of the K blocks)
    for (; pkb < kb_end; pkb += kpb, pst = pst + 1 == stages ? 0 : pst + 1, pph ^= pst == 0) {
      if (!mbar_wait_bounded(bar_empty + 8 * pst, pph ^ 1)) {
        set_status(p.status, NVB200_STATUS_WAIT_TIMEOUT);
        break;
      }
      skinny_load_stage(map_w, map_x, bar_full + 8 * pst, stage0 + pst * stage_bytes, pkb, min(kpb, kb_end - pkb),
                        sub_bytes, tile_w, BK, n0, up0);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    const uint64_t w0 = smem_desc(stage0, 16, 1024, 2), x0 = smem_desc(stage0 + tile_w, 16, 1024, 2);
    const uint32_t step = stage_bytes >> 4, sub = sub_bytes >> 4;
    int st = 0;
    uint32_t ph = 0;
    for (int kb = kb_begin; kb < kb_end; kb += kpb, st = st + 1 == stages ? 0 : st + 1, ph ^= st == 0) {
      if (!mbar_wait_bounded(bar_full + 8 * st, ph)) {
        if (lane == 0) set_status(p.status, NVB200_STATUS_WAIT_TIMEOUT);
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const int nsub = min(kpb, kb_end - kb);
        for (int u = 0; u < nsub; ++u) {
          const uint64_t wd = w0 + st * step + u * sub, xd = x0 + st * step + u * sub;
#pragma unroll
          for (int k = 0; k < kMmaPerSub; ++k)
            tc_mma<TF32>(tmem_base, wd + k * 2, xd + k * 2, p.idesc, (kb > kb_begin || u > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(bar_empty + 8 * st);
      }
      __syncwarp();
    }
    if (lane == 0) tc_commit(bar_acc);  // arrives once every MMA above has completed
    __syncwarp();
  }

  // -------------------------------------------------------------------- epilogue
  __syncwarp();
  ok = mbar_wait_bounded(bar_acc, 0) && ok;
  if (!ok && lane == 0) set_status(p.status, NVB200_STATUS_WAIT_TIMEOUT);
  tc_fence_after();
  const int nt = warp * 32 + lane;  // this thread's TMEM lane: row n0 + nt of C^T
  const uint32_t taddr = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
  const int rows = BM / S;                          // rows of C^T this CTA finishes (its cluster slice)
  const int o0 = static_cast<int>(rank) * rows;      // first of them
  float *part = reinterpret_cast<float *>(smem + p.red_off);  // all-reduce: this CTA's partial, [m][rows]
  if (S == 1 && p.swiglu) {
    // Lanes 64-127 (the up columns) hand their sums to lanes 0-63 (the gate columns) through shared memory, 32 rows
    // at a time ([32][64] fp32); thread nt < 64 then finishes column n0 + nt of those rows, 4 rows per step.
    float *xch = reinterpret_cast<float *>(smem + p.red_off);
    const int n = n0 + nt;
    for (int c0 = 0; c0 < p.m_pad; c0 += 32) {
      float v[32];
      tmem_ld32(taddr + c0, v);
      if (nt >= BM / 2) {
#pragma unroll
        for (int i = 0; i < 32; ++i) xch[i * (BM / 2) + nt - BM / 2] = v[i];
      }
      __syncthreads();
      if (nt < BM / 2 && n < p.N) {
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          if (c0 + i >= p.M) break;
          const uint4 gv = make_uint4(pack_bf16x2(v[i], v[i + 1]), pack_bf16x2(v[i + 2], v[i + 3]), 0u, 0u);
          const uint4 uv = make_uint4(pack_bf16x2(xch[i * (BM / 2) + nt], xch[(i + 1) * (BM / 2) + nt]),
                                      pack_bf16x2(xch[(i + 2) * (BM / 2) + nt], xch[(i + 3) * (BM / 2) + nt]), 0u, 0u);
          const uint4 o = silu_mul8_bf16(gv, uv);
          const uint32_t w[2] = {o.x, o.y};
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (c0 + i + e < p.M)
              static_cast<__nv_bfloat16 *>(p.c)[(c0 + i + e) * p.scm + n] =
                  __ushort_as_bfloat16(static_cast<unsigned short>(e & 1 ? w[e >> 1] >> 16 : w[e >> 1] & 0xFFFFu));
        }
      }
      __syncthreads();  // the gate lanes are done with xch before the next 32 rows overwrite it
    }
    tc_fence_before();
    __syncthreads();  // every TMEM read done before the columns are freed
  } else if (S == 1) {
    const int n = n0 + nt;
    for (int c0 = 0; c0 < p.m_pad; c0 += 32) {
      float v[32];
      tmem_ld32(taddr + c0, v);
      if (p.ar_world > 1) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (c0 + i < p.m_pad) part[(c0 + i) * BM + nt] = v[i];
      } else if (n < p.N) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (c0 + i < p.M) store_c(p, c0 + i, n, v[i]);
      }
    }
    tc_fence_before();
    __syncthreads();  // every TMEM read done before the columns are freed (and the partial complete)
  } else {
    // Push this CTA's partial of row nt to its owner: slot [rank][m][nt - owner * rows] of the owner's buffer. In
    // the gate_up form, owner r takes the gate rows r * (64 / S) ... and the matching up rows: its slot row i is gate
    // row r * (64 / S) + i for i < 64 / S, then up row 64 + r * (64 / S) + (i - 64 / S).
    const int half = rows / 2;  // gate_up form: gate (and up) rows per owner
    const int owner = p.swiglu ? (nt & (BM / 2 - 1)) / half : nt / rows;
    const int local = p.swiglu ? (nt < BM / 2 ? nt - owner * half : half + (nt - BM / 2) - owner * half)
                               : nt - owner * rows;
    const uint32_t dst = map_to_cta(smem_addr(smem + p.red_off), owner) +
                         static_cast<uint32_t>((static_cast<int>(rank) * p.m_pad * rows + local) * 4);
    for (int c0 = 0; c0 < p.m_pad; c0 += 32) {
      float v[32];
      tmem_ld32(taddr + c0, v);
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (c0 + i < p.m_pad)
          asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dst + (c0 + i) * rows * 4), "f"(v[i]) : "memory");
    }
    tc_fence_before();
    cluster_sync();  // every partial is in its owner's memory (and every TMEM read done)
    // Sum the S slots of this CTA's rows, 4 consecutive rows (columns n of C) per step. With an all-reduce to
    // follow, the sum goes back into slot 0 (the same thread read it) as this GPU's partial.
    float *red = reinterpret_cast<float *>(smem + p.red_off);
    if (p.swiglu) {
      // Owner: gate and up sums of its 64 / S columns n0 + rank * (64 / S) + [0, 64 / S), 4 columns per step.
      const int qpg = half / 4;
      for (int gi = threadIdx.x; gi < p.M * qpg; gi += kSkinnyThreads) {
        const int m = gi / qpg, q = gi - m * qpg;
        float g4[4] = {0.f, 0.f, 0.f, 0.f}, u4[4] = {0.f, 0.f, 0.f, 0.f};
        for (int r = 0; r < S; ++r) {
          const float *row = red + (r * p.m_pad + m) * rows;
          const float4 x = *reinterpret_cast<const float4 *>(row + 4 * q);
          const float4 y = *reinterpret_cast<const float4 *>(row + half + 4 * q);
          g4[0] += x.x, g4[1] += x.y, g4[2] += x.z, g4[3] += x.w;
          u4[0] += y.x, u4[1] += y.y, u4[2] += y.z, u4[3] += y.w;
        }
        store_swiglu4(p, m, n0 + static_cast<int>(rank) * half + 4 * q, g4, u4);
      }
    }
    const int qpr = p.swiglu ? 0 : rows / 4;
    for (int gi = threadIdx.x; gi < p.M * qpr; gi += kSkinnyThreads) {
      const int m = gi / qpr, q = gi - m * qpr;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int r = 0; r < S; ++r) {
        const float4 x = *reinterpret_cast<const float4 *>(red + (r * p.m_pad + m) * rows + 4 * q);
        acc[0] += x.x, acc[1] += x.y, acc[2] += x.z, acc[3] += x.w;
      }
      const int n = n0 + o0 + 4 * q;
      if (p.ar_world > 1) {
        *reinterpret_cast<float4 *>(red + m * rows + 4 * q) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (n + i < p.N) store_c(p, m, n + i, acc[i]);
      }
    }
    if (p.ar_world > 1) __syncthreads();
  }

  if (p.ar_world > 1) {
    // ------------------------------------------------------------------ all-reduce over the GPUs (NVLink)
    // 1. This GPU's partial of the CTA's slice goes to every other rank's exchange buffer, tagged with the epoch.
    const int W = p.ar_world, me = p.ar_rank;
    const int qpr = rows / 4;
    // This call's epoch. The header's count only advances once every CTA of the call is done (below), and every CTA
    // reads it before it is done, so all CTAs read the same value.
    uint32_t epoch;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(epoch) : "l"(&ar_header(p, me)->completed) : "memory");
    epoch += 1;
    const uint64_t tag = static_cast<uint64_t>(epoch) << 32;
    for (int dst_rank = 0; dst_rank < W; ++dst_rank) {
      if (dst_rank == me) continue;
      uint64_t *slot = ar_slot(p, epoch, dst_rank, me);
      for (int gi = threadIdx.x; gi < p.M * qpr; gi += kSkinnyThreads) {
        const int m = gi / qpr, q = gi - m * qpr;
        const int n = n0 + o0 + 4 * q;
        if (n >= p.N) continue;
        const float4 v = *reinterpret_cast<const float4 *>(part + m * rows + 4 * q);
        uint64_t *dst = slot + m * p.ar_max_n + n;
        asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(tag | __float_as_uint(v.x)),
                     "l"(tag | __float_as_uint(v.y))
                     : "memory");
        asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(dst + 2), "l"(tag | __float_as_uint(v.z)),
                     "l"(tag | __float_as_uint(v.w))
                     : "memory");
      }
    }
    // 2. Sum the W partials in rank order (the same order, hence the same bits, on every GPU): this GPU's from shared
    // memory, the others' from its exchange buffer once their words carry this call's epoch (bounded wait: after
    // 1 s without a peer the status bit is set and the thread stops waiting).
    bool expired = false;
    uint64_t start = 0;
    for (int gi = threadIdx.x; gi < p.M * qpr; gi += kSkinnyThreads) {
      const int m = gi / qpr, q = gi - m * qpr;
      const int n = n0 + o0 + 4 * q;
      if (n >= p.N) continue;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int src = 0; src < W; ++src) {
        float x[4];
        if (src == me) {
          const float4 v = *reinterpret_cast<const float4 *>(part + m * rows + 4 * q);
          x[0] = v.x, x[1] = v.y, x[2] = v.z, x[3] = v.w;
        } else {
          const uint64_t *w = ar_slot(p, epoch, me, src) + m * p.ar_max_n + n;
          uint64_t a0, a1, a2, a3;
          for (uint32_t spin = 1;; ++spin) {
            asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a0), "=l"(a1) : "l"(w) : "memory");
            asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a2), "=l"(a3) : "l"(w + 2) : "memory");
            if (((a0 & a1 & a2 & a3) >> 32) == epoch && ((a0 | a1 | a2 | a3) >> 32) == epoch) break;
            if (expired) break;
            if ((spin & 1023u) == 0) {
              const uint64_t now = global_timer_ns();
              if (start == 0) start = now;
              else if (now - start > kWaitLimitNs) {
                set_status(p.status, NVB200_STATUS_WAIT_TIMEOUT);
                expired = true;
              }
            }
          }
          x[0] = __uint_as_float(static_cast<uint32_t>(a0)), x[1] = __uint_as_float(static_cast<uint32_t>(a1));
          x[2] = __uint_as_float(static_cast<uint32_t>(a2)), x[3] = __uint_as_float(static_cast<uint32_t>(a3));
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] += x[i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) store_c(p, m, n + i, acc[i]);
    }
    // 3. The last CTA of the call to finish advances this rank's epoch (and resets the count for the next call).
    __syncthreads();
    if (threadIdx.x == 0) {
      ArHeader *h = ar_header(p, me);
      if (atomicAdd(&h->arrived, 1u) == gridDim.x - 1) {
        h->arrived = 0;
        __threadfence();
        h->completed = epoch;
      }
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Weight-streaming GEMM for decode-sized rows (bf16, M <= 64, A row-major, B = weight.t(): both K-major). A decode
// step's linear layers stream each layer's weights from HBM once (tens of MB per layer, gone from L2 by the next
// step) against 1-64 activation rows: the time is the weight stream, the fixed cost of a launch and the wait for
// the preceding kernel, not arithmetic. So:
//   * a CTA owns a slice of NS = 8 NT weight rows (output columns) and a share of K; a thread-block cluster of S CTAs
//     splits K, their fp32 partials are summed through distributed shared memory. NT and S are chosen so that the
//     grid covers the SMs with the least data per SM (weights from HBM plus the A rows each CTA re-reads from L2);
//   * the weights do not depend on the preceding kernel, the A rows do. The kernel is launched with programmatic
//     stream serialization: its producer issues the weight loads of the first ring stages, then waits for the
//     preceding grid (griddepcontrol.wait), then loads A. When the preceding kernel lets its dependents start early
//     (griddepcontrol.launch_dependents, as this library's norm, SiLU x Mul and decode-attention kernels do), the
//     weight stream overlaps it;
//   * TMA moves 128-element K chunks (two 64-element boxes per operand, 128-byte swizzle) through a ring; 8 consumer
//     warps each take one 16-element k-step of every chunk on warp-level bf16 MMAs (the slice is 32-128 rows wide,
//     below the 64/128-row tiles of tcgen05.mma at 1-32 activation rows) and one pass through shared memory sums the
//     warps' shares.
// Epilogues: bf16 stores; the gate_up form (NS / 2 gate rows and the matching NS / 2 up rows, finished with the SiLU x
// Mul routine of the two-step form); the row-parallel form (the sums exchanged with the other GPUs over NVLink, as
// the skinny kernel's all-reduce does); the qkv form (each slice one head, finished with the fused q/k op's per-head
// math and stored to q_out and the KV cache).

constexpr int kStreamKc = 128;  // K elements per stage: two 64-element (128-byte) TMA boxes per operand
constexpr int kStreamConsumers = 8;
constexpr int kStreamThreads = 32 * (kStreamConsumers + 1);  // the consumer warps, then the producer warp
constexpr int kStreamMaxStages = 8;
// Ring bytes per CTA (one CTA per SM; it still fits beside the CTAs of this library's norm and SiLU x Mul kernels,
// which use no shared memory). Measured on the Qwen3-0.6B decode step (batch 32, context 1024; it changes only the
// gate_up + SiLU x Mul kernel's ring there, 8 -> 6 of its 8 chunks, so that a CTA of the down_proj kernel after it
// fits beside it and starts its weight loads): 96 KB 1522 us, 128 KB 1494.8 us, 192 KB 1499.0 us.
#ifndef NVB200_STREAM_RING_KB
#define NVB200_STREAM_RING_KB 128
#endif
constexpr uint32_t kStreamRingBytes = NVB200_STREAM_RING_KB * 1024;

struct StreamParams {
  __nv_bfloat16 *c;
  int64_t scm;
  int M, N, K;
  int chunks;         // ceil(K / kStreamKc)
  int split;          // S: CTAs of a cluster (consecutive blockIdx.x) sharing one slice, each a range of the chunks
  int stages;
  int swiglu;         // 1: rows n0 .. n0 + ns/2 - 1 are gate rows, their up rows start at N + n0; C = silu(g) * u
  uint32_t a_bytes;   // one stage's A tile: 2 boxes of m_pad rows x 128 bytes
  uint32_t w_bytes;   // one stage's weight tile: 2 boxes of ns rows x 128 bytes (each box two half-boxes for swiglu)
  uint32_t slot_off;  // the partials other CTAs of the cluster send (after the ring, which the sums reuse)
  uint32_t hdr_off;   // barriers
  int32_t *status;
  // Fused all-reduce over ar_world GPUs (1: none): the exchange buffers of every rank, as for the skinny kernel.
  int ar_world, ar_rank;
  int64_t ar_max_n;
  uint8_t *ar_base[kArMaxRanks];
  // epi = 1: the qkv projection with the fused q/k op as its epilogue. Slice t of 128 columns is head t of
  // [Hq q heads | Hkv k heads | Hkv v heads]; q heads get RMSNorm (q_w) + RoPE into q_out [M, Hq, 128], k heads
  // RMSNorm (k_w) + RoPE into k_cache[slot], v heads go to v_cache[slot] (slot -1: not stored; no cache: nothing).
  int epi;
  __nv_bfloat16 *q_out, *k_cache, *v_cache;
  const int64_t *positions;
  const int32_t *slots;
  const float *cos_sin;
  int64_t cs_stride, num_positions, num_slots;
  const __nv_bfloat16 *q_w, *k_w;
  int hq, hkv;
  float eps;
  uint32_t head_off;  // shared-memory offset of the [16 MT][128] bf16 staging tile of the slice's rows
  uint32_t side_off;  // shared-memory offset of the epilogue's inputs: 32 slots and 32 positions (int32), the rows'
                      // cos | sin ([16 MT][128] fp32), the 128 bf16 norm weights of the slice's head
};

// Address of the 16-byte chunk `ch` (0..7) of row `row` in a 128-byte-swizzled TMA tile at `tile` (rows of 128 bytes;
// TMA's SWIZZLE_128B stores chunk ch of row r at position ch ^ (r & 7), the tile 1024-byte aligned).
NVB200_DEVICE uint32_t sw128(uint32_t tile, int row, int ch) {
  return tile + row * 128 + ((ch ^ (row & 7)) << 4);
}

// 16-byte asynchronous global -> shared copy (cp.async), its commit and the wait for all of a thread's copies.
NVB200_DEVICE void cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
NVB200_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
NVB200_DEVICE void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// WN: the consumer warps split the slice's NT tiles into WN parts; warp w takes the WN k-steps w mod KW, + KW, ...
// (KW = 8 / WN) of every chunk for the NT / WN tiles of part w / KW (WN = 1: one k-step, every tile).
template <int MT, int NT, int WN = 1>
__global__ void __launch_bounds__(kStreamThreads, 1)
    matmul_stream_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                         const __grid_constant__ StreamParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int NS = 8 * NT;
  constexpr int G = MT * NT * 32;  // fragment groups: (m tile, n tile, lane), four fp32 values each
  constexpr int NTW = NT / WN, KW = kStreamConsumers / WN;
  static_assert(NT % WN == 0 && kStreamConsumers % WN == 0, "tiles and warps must split evenly");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.split, stages = p.stages;
  const int rank = static_cast<int>(blockIdx.x) % S, tile = static_cast<int>(blockIdx.x) / S;
  // This CTA's chunks: an even share of the K chunks (S <= chunks, so every share holds at least one).
  const int c_begin = rank * p.chunks / S, nch = (rank + 1) * p.chunks / S - c_begin;
  const uint32_t base = smem_addr(smem);
  const uint32_t stage_bytes = p.a_bytes + p.w_bytes;
  const uint32_t bar_full = base + p.hdr_off, bar_empty = bar_full + 8 * kStreamMaxStages;
  const int n0 = tile * (p.swiglu ? NS / 2 : NS);  // first weight row (gate row) of the slice
  launch_dependents();
  // Distributed shared memory may be written only once every CTA of the cluster runs: arrive now, wait before the
  // first remote store.
  if (S > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

  // The producer lane sets up the barriers and starts the weight loads of the first stages (they do not depend on
  // the preceding kernel) before the CTA's first barrier, so the loads start as early as possible.
  const bool producer = warp == kStreamConsumers && lane == 0;
  const int pre = min(nch, stages);
  auto load_w = [&](int i) {
    const uint32_t sw = base + (i % stages) * stage_bytes + p.a_bytes, full = bar_full + 8 * (i % stages);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int k = (c_begin + i) * kStreamKc + h * 64;
      tma_load_2d(sw + h * (p.w_bytes / 2), &map_w, k, n0, full);
      if (p.swiglu) tma_load_2d(sw + h * (p.w_bytes / 2) + p.w_bytes / 4, &map_w, k, p.N + n0, full);
    }
  };
  auto load_a = [&](int i) {
    const uint32_t sa = base + (i % stages) * stage_bytes, full = bar_full + 8 * (i % stages);
#pragma unroll
    for (int h = 0; h < 2; ++h)
      tma_load_2d(sa + h * (p.a_bytes / 2), &map_a, (c_begin + i) * kStreamKc + h * 64, 0, full);
  };
  if (producer) {
    prefetch_tmap(&map_w);
    prefetch_tmap(&map_a);
    for (int i = 0; i < stages; ++i) {
      mbar_init(bar_full + 8 * i, 1);
      mbar_init(bar_empty + 8 * i, kStreamConsumers);
    }
    fence_mbar_init();
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(bar_full + 8 * i, stage_bytes);
      load_w(i);
    }
  }
  __syncthreads();

  float acc[MT][NTW][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NTW; ++nt) acc[mt][nt][0] = acc[mt][nt][1] = acc[mt][nt][2] = acc[mt][nt][3] = 0.f;

  if (warp == kStreamConsumers) {
    // ------------------------------------------------------------------ producer (one lane): A, then the rest
    if (lane == 0) {
      grid_dependency_wait();
      for (int i = 0; i < pre; ++i) load_a(i);
      for (int i = pre; i < nch; ++i) {
        const int st = i % stages;
        if (!mbar_wait_bounded(bar_empty + 8 * st, ((i / stages) & 1) ^ 1)) {
          set_status(p.status, NVB200_STATUS_WAIT_TIMEOUT);
          break;
        }
        mbar_arrive_expect_tx(bar_full + 8 * st, stage_bytes);
        load_w(i);
        load_a(i);
      }
    }
  } else {
    // ------------------------------------------------------------------ consumers
    if (p.epi == 1) {
      // qkv epilogue inputs, fetched while the first chunks are on their way: for each row this CTA finishes, its
      // slot and position (out-of-range values flagged as the fused op flags them), then asynchronous copies of its
      // cos | sin row and of the head's norm weights into shared memory (waited for before the epilogue).
      grid_dependency_wait();
      const int head = static_cast<int>(blockIdx.x) / S;
      const bool isq = head < p.hq, isv = head >= p.hq + p.hkv;
      int32_t *slot_s = reinterpret_cast<int32_t *>(smem + p.side_off);
      int32_t *pos_s = slot_s + 32;
      const uint32_t cs_s = base + p.side_off + 64 * 4, w_s = cs_s + 16 * MT * 128 * 4;
      const int own = p.M > rank ? (p.M - rank + S - 1) / S : 0;  // rows rank, rank + S, ...
      const int t = threadIdx.x;                                 // 0..255 (the consumer warps)
      if (t < own) {
        const int m = rank + S * t;
        int32_t slot = -1;
        if (!isq && p.k_cache != nullptr) {
          slot = __ldg(p.slots + m);
          if (slot < -1 || slot >= p.num_slots) {
            set_status(p.status, NVB200_STATUS_BAD_SLOT);
            slot = -1;
          }
        }
        int64_t pos = -1;
        if (!isv && (isq || slot >= 0)) {
          pos = __ldg(p.positions + m);
          if (pos < 0 || pos >= p.num_positions) {
            set_status(p.status, NVB200_STATUS_BAD_POSITION);
            pos = 0;
          }
        }
        slot_s[m] = slot;
        pos_s[t] = static_cast<int32_t>(pos);
      }
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kStreamConsumers) : "memory");  // the consumer warps only
      for (int idx = t; idx < own * 32; idx += 32 * kStreamConsumers) {
        const int u = idx >> 5, i = idx & 31;
        const int32_t pos = pos_s[u];
        if (pos >= 0) cp_async16(cs_s + ((rank + S * u) * 128 + 4 * i) * 4, p.cos_sin + pos * p.cs_stride + 4 * i);
      }
      if (!isv && t < 16) cp_async16(w_s + 16 * t, (isq ? p.q_w : p.k_w) + 8 * t);
      cp_async_commit();
    }
    const int kw = warp % KW, npart = warp / KW;
    const int arow = (lane & 7) + ((lane >> 3) & 1) * 8;
    const int wrow = ((lane >> 4) << 3) + (lane & 7);
    for (int i = 0; i < nch; ++i) {
      const int st = i % stages;
      if (!mbar_wait_bounded(bar_full + 8 * st, (i / stages) & 1)) {
        if (lane == 0) set_status(p.status, NVB200_STATUS_WAIT_TIMEOUT);
        break;
      }
#pragma unroll
      for (int ks = 0; ks < WN; ++ks) {
        const int kstep = kw + KW * ks;      // 0..7: 16-element step of the chunk
        const int h = kstep >> 2;            // which 64-element box of the chunk
        const int ch0 = (kstep & 3) * 2;     // first 16-byte chunk of the k-step in the box's 128-byte rows
        const int ach = ch0 + (lane >> 4), wch = ch0 + ((lane >> 3) & 1);
        const uint32_t abox = base + st * stage_bytes + h * (p.a_bytes / 2);
        // This warp's part of the slice starts NTW * 8 rows into the box (a multiple of 8 rows: same swizzle).
        const uint32_t wbox = base + st * stage_bytes + p.a_bytes + h * (p.w_bytes / 2) + npart * NTW * 8 * 128;
        uint32_t af[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) ldsm_x4(sw128(abox, mt * 16 + arow, ach), af[mt]);
#pragma unroll
        for (int np = 0; np < NTW / 2; ++np) {
          uint32_t bw[4];
          ldsm_x4(sw128(wbox, np * 16 + wrow, wch), bw);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            mma_16816(acc[mt][2 * np], af[mt], bw[0], bw[1]);
            mma_16816(acc[mt][2 * np + 1], af[mt], bw[2], bw[3]);
          }
        }
        if constexpr (NTW % 2 == 1) {
          uint32_t bw[2];
          ldsm_x2(sw128(wbox, (NTW - 1) * 8 + (lane & 7), ch0 + ((lane >> 3) & 1)), bw);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) mma_16816(acc[mt][NTW - 1], af[mt], bw[0], bw[1]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_empty + 8 * st);  // this warp is done with the stage
    }
  }

  if (p.epi == 1) cp_async_wait_all();  // the epilogue's inputs (a no-op for threads that copied nothing)
  // -------------------------------------------------------------------- sums
  // Every chunk was consumed, so no copy is in flight and the ring is free: the warps' shares go there in fragment
  // order (group j = (mt NT + nt) 32 + lane, a float4 per group and warp: conflict-free), each thread then sums the
  // eight shares of its groups. With a split, the sum of group j goes to the shared memory of the CTA that finishes
  // it (rank j % S, slot [this rank][j / S]); one cluster barrier later each CTA adds the S partials of its groups.
  __syncthreads();
  float4 *red = reinterpret_cast<float4 *>(smem);  // [k part][G]
  if (warp < kStreamConsumers) {
    const int kw = warp % KW, npart = warp / KW;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NTW; ++nt)
        red[kw * G + (mt * NT + npart * NTW + nt) * 32 + lane] =
            make_float4(acc[mt][nt][0], acc[mt][nt][1], acc[mt][nt][2], acc[mt][nt][3]);
  }
  __syncthreads();
  // Owner of group j and its slot there. Plain and gate_up forms: rank j mod S, slot j / S. The qkv epilogue keeps
  // rows together: rank g mod S, g = (j mod 32) / 4 the group's row in its m tile (rows g and g + 8 share it, S | 8),
  // slot (j / 32) (32 / S) + (g / S) 4 + j mod 4.
  auto owner = [&](int j) { return p.epi ? ((j & 31) >> 2) % S : j % S; };
  auto slot_of = [&](int j) { return p.epi ? (j >> 5) * (32 / S) + (((j & 31) >> 2) / S) * 4 + (j & 3) : j / S; };
  const int per_owner = (G + S - 1) / S;
  const uint32_t slots = base + p.slot_off;  // [S][per_owner] float4
  if (S > 1) asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  for (int j = threadIdx.x; j < G; j += kStreamThreads) {
    float4 v = red[j];
#pragma unroll
    for (int w = 1; w < KW; ++w) {
      const float4 x = red[w * G + j];
      v.x += x.x, v.y += x.y, v.z += x.z, v.w += x.w;
    }
    if (S == 1) {
      red[j] = v;  // this thread's element alone
    } else {
      const uint32_t dst = map_to_cta(slots + (rank * per_owner + slot_of(j)) * 16, owner(j));
      asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "f"(v.x), "f"(v.y), "f"(v.z),
                   "f"(v.w)
                   : "memory");
    }
  }
  if (S > 1) cluster_sync();
  else __syncthreads();
  // Group j's finished values: c0, c1 at (row mt 16 + g, columns nt 8 + 2t, + 1), c2, c3 eight rows below.
  auto group_sum = [&](int j) {
    if (S == 1) return red[j];
    const float4 *sl = reinterpret_cast<const float4 *>(smem + p.slot_off);
    const int li = slot_of(j);
    float4 v = sl[li];
    for (int q = 1; q < S; ++q) {
      const float4 x = sl[q * per_owner + li];
      v.x += x.x, v.y += x.y, v.z += x.z, v.w += x.w;
    }
    return v;
  };
  auto store = [&](int row, int col, uint32_t packed) {
    if (row >= p.M) return;
    __nv_bfloat16 *dst = p.c + row * p.scm + col;
    if (col < p.N) dst[0] = __ushort_as_bfloat16(static_cast<unsigned short>(packed & 0xFFFFu));
    if (col + 1 < p.N) dst[1] = __ushort_as_bfloat16(static_cast<unsigned short>(packed >> 16));
  };
  // Groups finished here: j = rank + S li (all of them when S == 1); for swiglu only the gate tiles (nt < NT / 2),
  // whose up partner j + 16 NT has the same owner (16 NT is a multiple of S).
  if (p.epi == 1) {
    // ------------------------------------------------------------------ qkv epilogue: the fused q/k op per row
    // This CTA's rows (m mod S == rank) of the slice, rounded to bf16 as the projection's output, go to a staging
    // tile; then 8 lanes per row run the fused op's per-head math on them (the direct kernel's lane layout and
    // operations, so the same bits as qk_norm_rope_kv on that output).
    __nv_bfloat16 *hs = reinterpret_cast<__nv_bfloat16 *>(smem + p.head_off);  // [16 MT][128]
    for (int j = threadIdx.x; j < G; j += kStreamThreads) {
      if (owner(j) != rank) continue;
      const int ln = j & 31, t = j >> 5, mt = t / NT, nt = t % NT;
      const int row = mt * 16 + (ln >> 2), col = nt * 8 + 2 * (ln & 3);
      const float4 v = group_sum(j);
      *reinterpret_cast<uint32_t *>(hs + row * 128 + col) = pack_bf16x2(v.x, v.y);
      *reinterpret_cast<uint32_t *>(hs + (row + 8) * 128 + col) = pack_bf16x2(v.z, v.w);
    }
    __syncthreads();
    const int head = tile;  // slice = head of the qkv output
    const int32_t *slot_s = reinterpret_cast<const int32_t *>(smem + p.side_off);
    const float *cs_s = reinterpret_cast<const float *>(smem + p.side_off + 64 * 4);
    const __nv_bfloat16 *w_s = reinterpret_cast<const __nv_bfloat16 *>(smem + p.side_off + 64 * 4 + 16 * MT * 128 * 4);
    const int nrows = p.M > rank ? (p.M - rank + S - 1) / S : 0;
    const int j8 = lane & 7;
    const unsigned gmask = 0xffu << (lane & 24);
    for (int u = threadIdx.x >> 3; u < nrows; u += kStreamThreads / 8) {
      const int m = rank + S * u;
      const uint4 xa = *reinterpret_cast<const uint4 *>(hs + m * 128 + 8 * j8);
      const uint4 xb = *reinterpret_cast<const uint4 *>(hs + m * 128 + 64 + 8 * j8);
      const bool isq = head < p.hq, isv = head >= p.hq + p.hkv;
      const int32_t slot = slot_s[m];
      if (isv) {
        if (slot >= 0) {
          __nv_bfloat16 *o = p.v_cache + (static_cast<int64_t>(slot) * p.hkv + (head - p.hq - p.hkv)) * 128;
          *reinterpret_cast<uint4 *>(o + 8 * j8) = xa;
          *reinterpret_cast<uint4 *>(o + 64 + 8 * j8) = xb;
        }
        continue;
      }
      if (!isq && slot < 0) continue;  // a k head with nowhere to go
      uint4 ya, yb;
      head128_norm_rope(xa, xb, w_s, cs_s + m * 128, j8, p.eps, gmask, ya, yb);
      __nv_bfloat16 *o = isq ? p.q_out + (static_cast<int64_t>(m) * p.hq + head) * 128
                             : p.k_cache + (static_cast<int64_t>(slot) * p.hkv + (head - p.hq)) * 128;
      *reinterpret_cast<uint4 *>(o + 8 * j8) = ya;
      *reinterpret_cast<uint4 *>(o + 64 + 8 * j8) = yb;
    }
    return;
  }

  const int tiles_done = p.swiglu ? MT * (NT / 2) : MT * NT;
  if (p.ar_world <= 1) {
    for (int e = threadIdx.x; e < tiles_done * 32; e += kStreamThreads) {
      const int ln = e & 31, t = e >> 5;
      const int mt = p.swiglu ? t / (NT / 2) : t / NT, nt = p.swiglu ? t % (NT / 2) : t % NT;
      const int j = (mt * NT + nt) * 32 + ln;
      if (owner(j) != rank) continue;
      const int row = mt * 16 + (ln >> 2), col = nt * 8 + 2 * (ln & 3);
      const float4 v = group_sum(j);
      if (!p.swiglu) {
        store(row, n0 + col, pack_bf16x2(v.x, v.y));
        store(row + 8, n0 + col, pack_bf16x2(v.z, v.w));
      } else {
        const float4 u = group_sum(j + 16 * NT);
        const uint4 o = silu_mul8_bf16(make_uint4(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w), 0u, 0u),
                                       make_uint4(pack_bf16x2(u.x, u.y), pack_bf16x2(u.z, u.w), 0u, 0u));
        store(row, n0 + col, o.x);
        store(row + 8, n0 + col, o.y);
      }
    }
    return;
  }

  // -------------------------------------------------------------------- all-reduce over the GPUs (NVLink)
  // The protocol of the skinny kernel's all-reduce (exchange buffers of epoch-tagged 8-byte words, two parities):
  // 1. this GPU's sums of the CTA's groups go to every other rank's exchange buffer; 2. each group is summed over
  // the ranks in rank order (the same bits on every GPU), the others' words taken once they carry this call's
  // epoch; 3. the last CTA of the call advances this rank's epoch. Plain layout only (the host checks), N % 8 == 0
  // so a group's column pair lies within N, and every CTA of the grid resident at once (the host checks).
  const int W = p.ar_world, me = p.ar_rank;
  uint32_t epoch;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];"
               : "=r"(epoch)
               : "l"(&ar_header_at(p.ar_base, me)->completed)
               : "memory");
  epoch += 1;
  const uint64_t tag = static_cast<uint64_t>(epoch) << 32;
  for (int e = threadIdx.x; e < tiles_done * 32; e += kStreamThreads) {
    const int ln = e & 31, t = e >> 5, mt = t / NT, nt = t % NT;
    const int j = (mt * NT + nt) * 32 + ln;
    if (owner(j) != rank) continue;
    const int row = mt * 16 + (ln >> 2), n = n0 + nt * 8 + 2 * (ln & 3);
    if (n >= p.N) continue;
    const float4 v = group_sum(j);
    for (int dst = 0; dst < W; ++dst) {
      if (dst == me) continue;
      uint64_t *slot = ar_slot_at(p.ar_base, p.ar_max_n, epoch, dst, me) + n;
      if (row < p.M)
        asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(slot + row * p.ar_max_n),
                     "l"(tag | __float_as_uint(v.x)), "l"(tag | __float_as_uint(v.y))
                     : "memory");
      if (row + 8 < p.M)
        asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(slot + (row + 8) * p.ar_max_n),
                     "l"(tag | __float_as_uint(v.z)), "l"(tag | __float_as_uint(v.w))
                     : "memory");
    }
  }
  bool expired = false;
  uint64_t start = 0;
  for (int e = threadIdx.x; e < tiles_done * 32; e += kStreamThreads) {
    const int ln = e & 31, t = e >> 5, mt = t / NT, nt = t % NT;
    const int j = (mt * NT + nt) * 32 + ln;
    if (owner(j) != rank) continue;
    const int row = mt * 16 + (ln >> 2), n = n0 + nt * 8 + 2 * (ln & 3);
    if (n >= p.N) continue;
    const float4 mine = group_sum(j);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int src = 0; src < W; ++src) {
      float x[4] = {mine.x, mine.y, mine.z, mine.w};
      if (src != me) {
        const uint64_t *w = ar_slot_at(p.ar_base, p.ar_max_n, epoch, me, src) + n;
        if (row < p.M) {
          x[0] = ar_take(w + row * p.ar_max_n, epoch, &expired, &start, p.status);
          x[1] = ar_take(w + row * p.ar_max_n + 1, epoch, &expired, &start, p.status);
        }
        if (row + 8 < p.M) {
          x[2] = ar_take(w + (row + 8) * p.ar_max_n, epoch, &expired, &start, p.status);
          x[3] = ar_take(w + (row + 8) * p.ar_max_n + 1, epoch, &expired, &start, p.status);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] += x[i];
    }
    store(row, n, pack_bf16x2(acc[0], acc[1]));
    store(row + 8, n, pack_bf16x2(acc[2], acc[3]));
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    ArHeader *h = ar_header_at(p.ar_base, me);
    if (atomicAdd(&h->arrived, 1u) == gridDim.x - 1) {
      h->arrived = 0;
      __threadfence();
      h->completed = epoch;
    }
  }
}

#ifndef NVB200_MM_STREAM
#define NVB200_MM_STREAM 1
#endif
// 1: launch with programmatic stream serialization (the weight loads of the first stages overlap the preceding
// kernel); 0: plain stream order. Measured on B200, the Qwen3-0.6B decode step (batch 32, context 1024): 1549 us
// with it, 1595 us without.
#ifndef NVB200_MM_STREAM_PDL
#define NVB200_MM_STREAM_PDL 1
#endif

template <int MT, int NT, int WN = 1>
int launch_stream_mt_nt(const CUtensorMap &map_a, const CUtensorMap &map_w, const StreamParams &p, int grid, int smem,
                        bool early_weights, cudaStream_t stream) {
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || configured[dev] < smem) {
    if (cudaFuncSetAttribute(matmul_stream_kernel<MT, NT, WN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem) != cudaSuccess)
      return NVB200_ERR_CUDA;
    if (dev < 64) configured[dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kStreamThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (p.split > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = p.split, attr[n].val.clusterDim.y = 1, attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (NVB200_MM_STREAM_PDL && early_weights) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, matmul_stream_kernel<MT, NT, WN>, map_a, map_w, p) == cudaSuccess
             ? NVB200_OK
             : NVB200_ERR_CUDA;
}

template <int MT> int launch_stream_mt(int nt, const CUtensorMap &map_a, const CUtensorMap &map_w,
                                       const StreamParams &p, int grid, int smem, bool early_weights,
                                       cudaStream_t stream) {
  // MT x NT <= 16 (accumulator registers); the selection never asks for more.
  switch (nt) {
    case 1: return launch_stream_mt_nt<MT, 1>(map_a, map_w, p, grid, smem, early_weights, stream);
    case 2: return launch_stream_mt_nt<MT, 2>(map_a, map_w, p, grid, smem, early_weights, stream);
    case 3: return launch_stream_mt_nt<MT, 3>(map_a, map_w, p, grid, smem, early_weights, stream);
    case 4: return launch_stream_mt_nt<MT, 4>(map_a, map_w, p, grid, smem, early_weights, stream);
    case 5: return launch_stream_mt_nt<MT, (MT <= 2 ? 5 : 4)>(map_a, map_w, p, grid, smem, early_weights, stream);
    case 6: return launch_stream_mt_nt<MT, (MT <= 2 ? 6 : 4)>(map_a, map_w, p, grid, smem, early_weights, stream);
    case 7: return launch_stream_mt_nt<MT, (MT <= 2 ? 7 : 4)>(map_a, map_w, p, grid, smem, early_weights, stream);
    default: return launch_stream_mt_nt<MT, (MT <= 2 ? 8 : 4)>(map_a, map_w, p, grid, smem, early_weights, stream);
  }
}

// Slice width (NT 8-column tiles) and K split S for a decode-sized GEMM. A CTA's time is about the bytes it moves
// (its weight rows and the A rows it re-reads, over its share of K) plus a fixed start-up cost, and with a split the
// cluster reduction; the kernel's time is a CTA's times the waves of CTAs. So: the pair with the least
//   waves x (bytes per CTA + 40 KB) + (S > 1: 40 KB + 8 KB x S),
// at least 4 tiles per slice (narrower slices re-read A for too few weight rows); ties go to more CTAs. On B200 this
// picks, at the Qwen3-0.6B and -8B decode projections with 1, 32 and 64 rows, the (NT, S) that a sweep of every pair
// measured fastest or within a few percent of it (32 rows: o_proj and down_proj 4 x 4, gate_up with SiLU x Mul 6 x 1,
// 8B o_proj and down_proj 7 x 2).
struct StreamPlan {
  int nt, split;
};

#ifndef NVB200_STREAM_FORCE_NT
#define NVB200_STREAM_FORCE_NT 0
#endif
#ifndef NVB200_STREAM_FORCE_SPLIT
#define NVB200_STREAM_FORCE_SPLIT 0
#endif

StreamPlan stream_plan(int64_t M, int64_t N, int64_t K, bool swiglu, int sms) {
  const int MT = M <= 16 ? 1 : (M <= 32 ? 2 : 4);
  const int64_t chunks = (K + kStreamKc - 1) / kStreamKc;
  StreamPlan best{0, 0};
  int64_t best_cost = 0, best_ctas = 0;
  for (int nt = 4; nt <= 8; ++nt) {
    if (MT * nt > 16 || (swiglu && nt % 2)) continue;
    if (NVB200_STREAM_FORCE_NT && nt != NVB200_STREAM_FORCE_NT) continue;
    const int64_t cols = swiglu ? 4 * nt : 8 * nt;
    const int64_t tiles = (N + cols - 1) / cols;
    for (int s = 1; s <= 8; s *= 2) {
      if (s > chunks || (NVB200_STREAM_FORCE_SPLIT && s != NVB200_STREAM_FORCE_SPLIT)) continue;
      const int64_t ctas = tiles * s, cpc = (chunks + s - 1) / s, waves = (ctas + sms - 1) / sms;
      const int64_t cost = waves * (cpc * (4096LL * MT + 2048LL * nt) + 40960) + (s > 1 ? 40960 + 8192LL * s : 0);
      if (best.nt == 0 || cost < best_cost || (cost == best_cost && ctas > best_ctas))
        best = {nt, s}, best_cost = cost, best_ctas = ctas;
    }
  }
  return best;
}

// Launches the weight-streaming kernel for bf16, M <= 64, K-major A and B (16-byte aligned rows), C row-major
// (scn == 1); returns NVB200_ERR_UNSUPPORTED otherwise. early_weights: the caller guarantees that no kernel in
// flight writes B (model weights), so the launch may let the weight loads overlap the preceding kernel.
int launch_stream(void *c, const void *a, const void *b, int64_t M, int64_t N, int64_t K, int64_t sam, int64_t sbn,
                  int64_t scm, int64_t scn, bool swiglu, bool early_weights, int32_t *status, cudaStream_t stream,
                  const nvb200_allreduce_group *ar = nullptr) {
  if (!NVB200_MM_STREAM || M <= 0 || M > 64 || N <= 0 || scn != 1 || K <= 0 || (sam * 2) % 16 != 0 ||
      (sbn * 2) % 16 != 0 || N > 0x3fffffffLL || K > 0x3fffffffLL)
    return NVB200_ERR_UNSUPPORTED;
  const int MT = M <= 16 ? 1 : (M <= 32 ? 2 : 4);
  const StreamPlan plan = stream_plan(M, N, K, swiglu, sm_count());
  if (plan.nt == 0) return NVB200_ERR_UNSUPPORTED;
  const int nt = plan.nt, NS = 8 * nt;
  const int64_t cols = swiglu ? NS / 2 : NS;  // output columns per slice
  const int64_t grid = (N + cols - 1) / cols * plan.split;
  if (grid > 0x7fffffffLL) return NVB200_ERR_UNSUPPORTED;
  StreamParams p{};
  p.c = static_cast<__nv_bfloat16 *>(c), p.scm = scm;
  p.M = static_cast<int>(M), p.N = static_cast<int>(N), p.K = static_cast<int>(K);
  p.chunks = static_cast<int>((K + kStreamKc - 1) / kStreamKc);
  p.split = plan.split;
  p.swiglu = swiglu ? 1 : 0;
  p.a_bytes = 2u * (16u * MT) * 128u;
  p.w_bytes = 2u * static_cast<uint32_t>(NS) * 128u;
  const uint32_t stage_bytes = p.a_bytes + p.w_bytes;
  const int cpc = (p.chunks + p.split - 1) / p.split;
  p.stages = std::max(1, std::min({kStreamMaxStages, cpc, static_cast<int>(kStreamRingBytes / stage_bytes)}));
  const uint32_t groups = 32u * MT * nt;
  const uint32_t red_bytes = kStreamConsumers * groups * 16u;
  p.slot_off = (std::max(p.stages * stage_bytes, red_bytes) + 255u) / 256u * 256u;
  p.hdr_off = p.slot_off + (p.split > 1 ? (groups + p.split - 1) / p.split * p.split * 16u : 0u);
  p.status = status;
  p.ar_world = 1;
  if (ar != nullptr) {
    // Every CTA waits for its counterparts on the other GPUs, so the whole grid must be resident (one CTA per SM).
    // (16-byte word pairs: the row pitch max_n must be even.)
    if (swiglu || ar->world < 2 || ar->world > kArMaxRanks || ar->rank < 0 || ar->rank >= ar->world || N % 8 != 0 ||
        N > ar->max_n || ar->max_n % 2 != 0 || M > kSkinnyMaxM || grid > std::min(sm_count(), kArMaxGrid))
      return NVB200_ERR_UNSUPPORTED;
    p.ar_world = ar->world, p.ar_rank = ar->rank, p.ar_max_n = ar->max_n;
    for (int r = 0; r < ar->world; ++r) {
      if (ar->buffers[r] == nullptr) return NVB200_ERR_ARG;
      p.ar_base[r] = static_cast<uint8_t *>(ar->buffers[r]);
    }
  }
  const int smem = static_cast<int>(1024 + p.hdr_off + 2 * 8 * kStreamMaxStages);
  CUtensorMap map_a, map_w;
  if (!make_map(&map_a, a, false, K, M, sam, 64, 16 * MT) ||
      !make_map(&map_w, b, false, K, swiglu ? 2 * N : N, sbn, 64, static_cast<int>(cols)))
    return NVB200_ERR_UNSUPPORTED;
  switch (MT) {
    case 1: return launch_stream_mt<1>(nt, map_a, map_w, p, static_cast<int>(grid), smem, early_weights, stream);
    case 2: return launch_stream_mt<2>(nt, map_a, map_w, p, static_cast<int>(grid), smem, early_weights, stream);
    default: return launch_stream_mt<4>(nt, map_a, map_w, p, static_cast<int>(grid), smem, early_weights, stream);
  }
}

// Launches the skinny kernel for M <= kSkinnyMaxM with K-major A and B (A row-major, B = weight.t()); returns
// NVB200_ERR_UNSUPPORTED otherwise.
int launch_skinny(void *c, const void *a, const void *b, int64_t M, int64_t N, int64_t K, int64_t sam, int64_t sbn,
                  int64_t scm, int64_t scn, bool f32, int32_t *status, cudaStream_t stream,
                  const nvb200_allreduce_group *ar = nullptr, bool swiglu = false) {
  if (M > kSkinnyMaxM || M <= 0) return NVB200_ERR_UNSUPPORTED;
  if (swiglu && (f32 || ar != nullptr || scn != 1)) return NVB200_ERR_UNSUPPORTED;
  const int es = f32 ? 4 : 2;
  const int BK = 128 / es;
  SkinnyParams p{};
  p.c = c, p.scm = scm, p.scn = scn;
  p.M = static_cast<int>(M), p.N = static_cast<int>(N), p.K = static_cast<int>(K);
  p.m_pad = static_cast<int>((M + 15) / 16 * 16);
  p.k_blocks = static_cast<int>((K + BK - 1) / BK);
  p.elem_bytes = es, p.c_is_f32 = f32, p.status = status;
  p.swiglu = swiglu ? 1 : 0;
  const int tile_cols = swiglu ? BM / 2 : BM;  // output columns per tile
  const int tiles = static_cast<int>((N + tile_cols - 1) / tile_cols);
  const int sms = sm_count();
  int split = 1;
  while (split < 8 && static_cast<int64_t>(tiles) * split * 2 <= sms && split * 2 <= p.k_blocks) split *= 2;
  p.split = split;
  if (ar != nullptr) {
    // Every CTA waits for its peers' CTAs of the same slice, so all of them must be resident at once.
    if (ar->world < 2 || ar->world > kArMaxRanks || ar->rank < 0 || ar->rank >= ar->world || N % 4 != 0 ||
        N > ar->max_n || ar->max_n % 2 != 0 || static_cast<int64_t>(tiles) * split > std::min(sms, kArMaxGrid))
      return NVB200_ERR_UNSUPPORTED;
    p.ar_world = ar->world, p.ar_rank = ar->rank, p.ar_max_n = ar->max_n;
    for (int r = 0; r < ar->world; ++r) {
      if (ar->buffers[r] == nullptr) return NVB200_ERR_ARG;
      p.ar_base[r] = static_cast<uint8_t *>(ar->buffers[r]);
    }
  }
  CUtensorMap map_w, map_x;
  if (!make_map(&map_w, b, f32, K, swiglu ? 2 * N : N, sbn, BK, swiglu ? BM / 2 : BM) ||
      !make_map(&map_x, a, f32, K, M, sam, BK, p.m_pad))
    return NVB200_ERR_UNSUPPORTED;
  const uint32_t fmt = f32 ? 2u : 1u;
  p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (static_cast<uint32_t>(p.m_pad >> 3) << 17) |
            (static_cast<uint32_t>(BM >> 4) << 24);
  const int blocks_per_cta = (p.k_blocks + split - 1) / split;
  // Two K blocks per stage (8 MMAs per commit) for a K split with at least 4 blocks per CTA; without a split the
  // smaller ring of three CTAs per SM keeps one block per stage.
  p.kpb = split > 1 && blocks_per_cta >= 4 ? NVB200_SKINNY_KPB : 1;
  const int stage_bytes = p.kpb * (BM * 128 + p.m_pad * 128);
  // One CTA per SM with a K split (the grid is at most one wave); without one, the grid has many waves and three
  // CTAs per SM overlap one's epilogue with the others' loads.
  const int ring_budget = split > 1 ? 160 * 1024 : 72 * 1024;
  p.stages = std::max(1, std::min({kSkinnyMaxStages, (blocks_per_cta + p.kpb - 1) / p.kpb, ring_budget / stage_bytes}));
  p.red_off = p.stages * stage_bytes;
  // Partial slots (K split, all-reduce) or the gate_up form's exchange of 32 rows of up sums.
  p.hdr_off = p.red_off + (split > 1 || p.ar_world > 1 ? p.m_pad * BM * 4 : (swiglu ? 32 * (BM / 2) * 4 : 0));
  const int smem = 1024 + p.hdr_off + 256;
  const int rc = f32 ? configure_once(matmul_skinny_kernel<true>, smem, 4) : configure_once(matmul_skinny_kernel<false>, smem, 5);
  if (rc) return rc;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(tiles * split), 1, 1);
  cfg.blockDim = dim3(kSkinnyThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(split);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = f32 ? cudaLaunchKernelEx(&cfg, matmul_skinny_kernel<true>, map_w, map_x, p)
                            : cudaLaunchKernelEx(&cfg, matmul_skinny_kernel<false>, map_w, map_x, p);
  return e == cudaSuccess ? NVB200_OK : NVB200_ERR_CUDA;
}

}  // namespace

namespace {

// Shared launcher. swiglu: N is the output width, B holds 2 N columns (gate | up) and the epilogue is SiLU x Mul
// (bf16 only, C row-major with a 16-byte row pitch).
int tc_launch(void *c, const void *a, const void *b, int64_t M, int64_t N, int64_t K, int64_t sam, int64_t sak,
              int64_t sbk, int64_t sbn, int64_t scm, int64_t scn, int dtype, bool swiglu, int32_t *status,
              cudaStream_t stream) {
  if (K <= 0 || M > 0x7fffffffLL || N > 0x3fffffffLL || K > 0x7fffffffLL) return NVB200_ERR_UNSUPPORTED;
  if (swiglu && dtype != NVB200_BF16) return NVB200_ERR_UNSUPPORTED;
  const bool f32 = dtype == NVB200_F32;
  const int es = f32 ? 4 : 2;
  const int BK = 128 / es;
  // Operand layouts TMA can read: one unit stride, the other a multiple of 16 bytes, base 16-byte aligned.
  bool a_mn;
  if (sak == 1 && (sam * es) % 16 == 0) a_mn = false;
  else if (sam == 1 && (sak * es) % 16 == 0) a_mn = true;
  else return NVB200_ERR_UNSUPPORTED;
  bool b_mn;
  if (sbk == 1 && (sbn * es) % 16 == 0) b_mn = false;
  else if (sbn == 1 && (sbk * es) % 16 == 0) b_mn = true;
  else return NVB200_ERR_UNSUPPORTED;
  if (!aligned16(a) || !aligned16(b)) return NVB200_ERR_UNSUPPORTED;
  if (M <= kSkinnyMaxM && !a_mn && !b_mn) {
    if (!f32) {
      const int rc = launch_stream(c, a, b, M, N, K, sam, sbn, scm, scn, swiglu, false, status, stream);
      if (rc != NVB200_ERR_UNSUPPORTED) return rc;
    }
    const int rc = launch_skinny(c, a, b, M, N, K, sam, sbn, scm, scn, f32, status, stream, nullptr, swiglu);
    if (rc != NVB200_ERR_UNSUPPORTED) return rc;
  }

  const int sms = sm_count();
  // CTA pairs (256-row tiles) when M fills at least two 128-row tiles and the pairs' tiles occupy at least half the
  // SMs; single CTAs (128-row tiles) otherwise. Measured on B200: 4096 x 1024 x 3072 (64 pair tiles on 128 SMs)
  // runs at 1168 TF/s as pairs against 1034 as 128 single-CTA tiles of 128 x 256.
  const int64_t tm1 = (M + BM - 1) / BM;
  const int64_t tm2 = (M + 2 * BM - 1) / (2 * BM);
  const int64_t out_cols = swiglu ? 128 : 256;  // output columns of a 256-column tile
  const bool pair = tm1 >= 2 && tm2 * ((N + out_cols - 1) / out_cols) * 4 >= sms;
  int bn = 256;
  // 128-column tiles only where 256-column ones would leave SMs idle (an N = 128 MMA takes nearly as long as an
  // N = 256 one, so they halve the rate per SM).
  if (!swiglu && !pair && tm1 * ((N + 255) / 256) < sms && tm1 * ((N + 127) / 128) > tm1 * ((N + 255) / 256)) bn = 128;
  // B rows (K-major) or columns (MN-major) one TMA box holds: half a tile per CTA of a pair, and the gate / up
  // halves of a gate_up tile are separate boxes.
  const int box_n = pair || swiglu ? bn / 2 : bn;
  const int64_t b_cols = swiglu ? 2 * N : N;

  // 32-bit MN-major operands use the 32-byte-atom swizzle (4-row atoms); everything else the 16-byte one.
  CUtensorMap map_a, map_b;
  const bool ok_a = a_mn ? make_map(&map_a, a, f32, M, K, sak, BK, BK, f32) : make_map(&map_a, a, f32, K, M, sam, BK, BM);
  const bool ok_b = b_mn ? make_map(&map_b, b, f32, b_cols, K, sbk, BK, BK, f32)
                         : make_map(&map_b, b, f32, K, b_cols, sbn, BK, box_n);
  if (!ok_a || !ok_b) return NVB200_ERR_UNSUPPORTED;

  TcParams p{};
  p.c = c;
  p.scm = scm;
  p.scn = scn;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.bn = bn;
  p.tiles_m = static_cast<int>(pair ? tm2 : tm1);
  p.tiles_n = static_cast<int>(swiglu ? (N + 127) / 128 : (N + bn - 1) / bn);  // output columns per tile: 128 or bn
  p.swiglu = swiglu;
  // Two 64-wide K sub-tiles per stage: one tcgen05.commit then releases 8 MMAs' operands. (Each commit and
  // stage handoff idles the tensor pipe for some hundreds of cycles; measured on B200, 4 MMAs per commit ran at
  // 58 % of the back-to-back MMA rate, 8 at 92 %, 16 at 98 %.)
  p.ksub = NVB200_MM_KSUB;
  p.k_blocks = static_cast<int>((K + BK * p.ksub - 1) / (BK * p.ksub));
  p.k_subs = static_cast<int>((K + BK - 1) / BK);
  p.a_mn_major = a_mn;
  p.b_mn_major = b_mn;
  p.a_swz = p.b_swz = f32 ? 1u : 2u;
  p.a_sbo = p.b_sbo = f32 ? 512u : 1024u;
  p.elem_bytes = es;
  p.c_is_f32 = f32;
  p.status = status;
  // C through shared memory and TMA stores when C is row-major with a 16-byte pitch; direct stores otherwise.
  CUtensorMap map_c;
  p.c_tma = scn == 1 && (scm * es) % 16 == 0 && aligned16(c) && make_map_c(&map_c, c, f32, M, N, scm);
  if (swiglu && !p.c_tma) return NVB200_ERR_UNSUPPORTED;
  if (!p.c_tma) map_c = map_a;  // unused
  p.epi_bufs = f32 ? 1 : 2;
  const int epi_bytes = p.c_tma ? kEpilogueWarps * p.epi_bufs * 32 * 32 * es : 0;
  // Instruction descriptor: D fp32 (bits 4-5 = 1), A/B format (bits 7-9, 10-12: 1 = bf16, 2 = tf32), major bits
  // 15/16 (1 = MN-major), N >> 3 at bit 17, M >> 4 at bit 24 (M = 256 for a CTA pair).
  const uint32_t fmt = f32 ? 2u : 1u;
  const int mma_m = pair ? 2 * BM : BM;
  p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (static_cast<uint32_t>(a_mn) << 15) |
            (static_cast<uint32_t>(b_mn) << 16) | (static_cast<uint32_t>(bn >> 3) << 17) |
            (static_cast<uint32_t>(mma_m >> 4) << 24);
  if (static_cast<int64_t>(p.tiles_m) * p.tiles_n > 0x7fffffffLL) return NVB200_ERR_UNSUPPORTED;
  const int tiles = p.tiles_m * p.tiles_n;

  // Shared memory: 1 KB alignment slack | stages | epilogue staging | 256 B of barriers and the TMEM slot.
  if (pair) {
    const int stage_bytes = p.ksub * (kTileBytesA + (bn / 2) * 128);
    p.stages = std::min(kMaxStages2, (kMaxDynamicSmem - 1024 - 256 - epi_bytes) / stage_bytes);
    if (p.stages < 2) return NVB200_ERR_UNSUPPORTED;
    p.epi_off = p.stages * stage_bytes;
    p.hdr_off = p.epi_off + epi_bytes;
    const int smem = 1024 + p.hdr_off + 256;
    const int rc = f32 ? configure_once(matmul_tc2_kernel<true>, smem, 2) : configure_once(matmul_tc2_kernel<false>, smem, 3);
    if (rc) return rc;
    const unsigned grid = 2u * static_cast<unsigned>(std::min(tiles, sms / 2));
    if (f32)
      matmul_tc2_kernel<true><<<grid, kThreads, smem, stream>>>(map_a, map_b, map_c, p);
    else
      matmul_tc2_kernel<false><<<grid, kThreads, smem, stream>>>(map_a, map_b, map_c, p);
    return launch_status();
  }
  const int stage_bytes = p.ksub * (kTileBytesA + bn * 128);
  p.stages = std::min(kMaxStages2, (kMaxDynamicSmem - 1024 - 256 - epi_bytes) / stage_bytes);
  if (p.stages < 2) return NVB200_ERR_UNSUPPORTED;
  p.epi_off = p.stages * stage_bytes;
  p.hdr_off = p.epi_off + epi_bytes;
  const int smem = 1024 + p.hdr_off + 256;
  const int rc = f32 ? configure_once(matmul_tc_kernel<true>, smem, 0) : configure_once(matmul_tc_kernel<false>, smem, 1);
  if (rc) return rc;
  const unsigned grid = static_cast<unsigned>(std::min(tiles, sms));
  if (f32)
    matmul_tc_kernel<true><<<grid, kThreads, smem, stream>>>(map_a, map_b, map_c, p);
  else
    matmul_tc_kernel<false><<<grid, kThreads, smem, stream>>>(map_a, map_b, map_c, p);
  return launch_status();
}

}  // namespace

int matmul_tc_launch(void *c, const void *a, const void *b, int64_t M, int64_t N, int64_t K, int64_t sam,
                     int64_t sak, int64_t sbk, int64_t sbn, int64_t scm, int64_t scn, int dtype, int32_t *status,
                     cudaStream_t stream) {
  return tc_launch(c, a, b, M, N, K, sam, sak, sbk, sbn, scm, scn, dtype, false, status, stream);
}

int matmul_swiglu_launch(void *c, const void *a, const void *b, int64_t M, int64_t N, int64_t K, int64_t sam,
                         int64_t sak, int64_t sbk, int64_t sbn, int64_t scm, int32_t *status, cudaStream_t stream) {
  return tc_launch(c, a, b, M, N, K, sam, sak, sbk, sbn, scm, 1, NVB200_BF16, true, status, stream);
}

int linear_decode_plan(int64_t M, int64_t N, int64_t K, bool swiglu, int32_t *nt, int32_t *split) {
  if (M <= 0 || M > 64 || N <= 0 || K <= 0 || N > 0x3fffffffLL || K > 0x3fffffffLL) return NVB200_ERR_UNSUPPORTED;
  const StreamPlan plan = stream_plan(M, N, K, swiglu, sm_count());
  if (plan.nt == 0) return NVB200_ERR_UNSUPPORTED;
  if (nt) *nt = plan.nt;
  if (split) *split = plan.split;
  return NVB200_OK;
}

int linear_decode_launch(void *y, const void *x, const void *w, int64_t M, int64_t N, int64_t K, int64_t sx,
                         int64_t sw, int64_t sy, bool swiglu, int32_t *status, cudaStream_t stream) {
  if (!aligned16(x) || !aligned16(w)) return NVB200_ERR_UNSUPPORTED;
  return launch_stream(y, x, w, M, N, K, sx, sw, sy, 1, swiglu, true, status, stream);
}

// The decode qkv projection with the fused q/k op as its epilogue (StreamParams::epi = 1): slices of one 128-column
// head (NT = 16, the consumer warps split into two 64-column parts), K split over a cluster so that the grid covers
// about the SMs, weight loads overlapping the preceding kernel. M <= 32 rows, head_dim 128, x and W K-major with
// 16-byte row pitches, no k_out; NVB200_ERR_UNSUPPORTED otherwise.
int linear_qkv_launch(const void *x, int64_t sx, const void *w, int64_t sw, int64_t K,
                      const nvb200_qk_norm_rope_kv_args &a, cudaStream_t stream) {
  const int64_t M = a.num_tokens;
  if (!NVB200_MM_STREAM || M < 1 || M > 32 || a.head_dim != 128 || a.k_out != nullptr || K <= 0 ||
      K > 0x3fffffffLL || (sx * 2) % 16 != 0 || (sw * 2) % 16 != 0 || !aligned16(x) || !aligned16(w) ||
      !aligned16(a.q_out) || a.cos_sin_stride % 4 != 0 || !aligned16(a.cos_sin) ||
      reinterpret_cast<uintptr_t>(a.q_weight) % 16 != 0 || reinterpret_cast<uintptr_t>(a.k_weight) % 16 != 0)
    return NVB200_ERR_UNSUPPORTED;
  if (a.k_cache != nullptr && (!aligned16(a.k_cache) || !aligned16(a.v_cache))) return NVB200_ERR_UNSUPPORTED;
  const int MT = M <= 16 ? 1 : 2;
  constexpr int NT = 16, WN = 2;
  const int heads = a.num_q_heads + 2 * a.num_kv_heads;
  const int64_t chunks = (K + kStreamKc - 1) / kStreamKc;
  const int sms = sm_count();
  // K split: the largest power of two up to 4 that keeps heads x split within the SMs (clusters of 8 CTAs measured
  // slower than 4 in every sweep of the weight-streaming kernel).
  int split = 1;
  while (split < 4 && split * 2 <= chunks && static_cast<int64_t>(heads) * split * 2 <= sms) split *= 2;
#ifdef NVB200_QKV_SPLIT
  split = std::min<int64_t>(NVB200_QKV_SPLIT, chunks);
#endif
  StreamParams p{};
  p.M = static_cast<int>(M), p.N = heads * 128, p.K = static_cast<int>(K);
  p.chunks = static_cast<int>(chunks);
  p.split = split;
  p.a_bytes = 2u * (16u * MT) * 128u;
  p.w_bytes = 2u * (8u * NT) * 128u;
  const uint32_t stage_bytes = p.a_bytes + p.w_bytes;
  const int cpc = (p.chunks + split - 1) / split;
  p.stages = std::max(1, std::min({kStreamMaxStages, cpc, static_cast<int>(kStreamRingBytes / stage_bytes)}));
  const uint32_t groups = 32u * MT * NT;
  const uint32_t red_bytes = (kStreamConsumers / WN) * groups * 16u;
  p.slot_off = (std::max(p.stages * stage_bytes, red_bytes) + 255u) / 256u * 256u;
  p.head_off = p.slot_off + (split > 1 ? groups * 16u : 0u);
  p.side_off = p.head_off + 16u * MT * 128u * 2u;
  p.hdr_off = p.side_off + 64u * 4u + 16u * MT * 128u * 4u + 128u * 2u;
  p.status = a.status;
  p.ar_world = 1;
  p.epi = 1;
  p.q_out = static_cast<__nv_bfloat16 *>(a.q_out);
  p.k_cache = static_cast<__nv_bfloat16 *>(a.k_cache);
  p.v_cache = static_cast<__nv_bfloat16 *>(a.v_cache);
  p.positions = a.positions;
  p.slots = a.slot_mapping;
  p.cos_sin = a.cos_sin;
  p.cs_stride = a.cos_sin_stride, p.num_positions = a.num_positions, p.num_slots = a.num_slots;
  p.q_w = static_cast<const __nv_bfloat16 *>(a.q_weight);
  p.k_w = static_cast<const __nv_bfloat16 *>(a.k_weight);
  p.hq = a.num_q_heads, p.hkv = a.num_kv_heads;
  p.eps = a.eps;
  const int smem = static_cast<int>(1024 + p.hdr_off + 2 * 8 * kStreamMaxStages);
  CUtensorMap map_a, map_w;
  if (!make_map(&map_a, x, false, K, M, sx, 64, 16 * MT) || !make_map(&map_w, w, false, K, p.N, sw, 64, 8 * NT))
    return NVB200_ERR_UNSUPPORTED;
  const int grid = heads * split;
  return MT == 1 ? launch_stream_mt_nt<1, NT, WN>(map_a, map_w, p, grid, smem, true, stream)
                 : launch_stream_mt_nt<2, NT, WN>(map_a, map_w, p, grid, smem, true, stream);
}

int64_t allreduce_buffer_bytes(int64_t max_n) {
  return kArHeaderBytes + 2LL * kArMaxRanks * kSkinnyMaxM * max_n * 8;
}

int matmul_allreduce_launch(void *c, const void *a, const void *b, int64_t M, int64_t N, int64_t K, int64_t sam,
                            int64_t sak, int64_t sbk, int64_t sbn, int64_t scm, const nvb200_allreduce_group *g,
                            int32_t *status, cudaStream_t stream) {
  if (K <= 0 || M > kSkinnyMaxM || N > 0x3fffffffLL || K > 0x7fffffffLL) return NVB200_ERR_UNSUPPORTED;
  if (sak != 1 || sbk != 1 || (sam * 2) % 16 != 0 || (sbn * 2) % 16 != 0 || !aligned16(a) || !aligned16(b))
    return NVB200_ERR_UNSUPPORTED;
  // The weight-streaming kernel with the all-reduce epilogue (plain stream order: B is not promised to be a weight
  // that no kernel in flight writes) for shards of at most 16 MB of B, else the skinny kernel's. Measured on two
  // B200s: the Qwen3-0.6B decode step at TP 2 (o_proj / down_proj shards of 2-3 MB) 1608 -> 1469 us with the former;
  // the Qwen3-8B down_proj shard (50 MB, bench.py --workload rowpar) 26.5 us with the skinny kernel, 31.3 with it.
  if (N * K * 2 <= (16LL << 20)) {
    const int rc = launch_stream(c, a, b, M, N, K, sam, sbn, scm, 1, false, false, status, stream, g);
    if (rc != NVB200_ERR_UNSUPPORTED) return rc;
  }
  return launch_skinny(c, a, b, M, N, K, sam, sbn, scm, 1, false, status, stream, g);
}

}  // namespace nvb200
