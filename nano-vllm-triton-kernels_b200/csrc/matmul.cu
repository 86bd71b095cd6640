// Tiled matmul C = A @ B with fp32 accumulation: the C ABI entry point and the CUDA-core (SIMT) kernel.
//
// Behaviour follows nanovllm/kernels/matmul.py:33-99: A [M, K] and B [K, N] with ANY strides (B is usually an
// nn.Linear weight.t()), fp32 accumulation, C in the inputs' dtype, tiles walked in GROUP_M-swizzled order
// (:50-57) so that concurrently running CTAs share A rows and B columns in L2, and a masked K tail (:68-75).
//
// Routing (nvb200_matmul):
//   bf16, or fp32 with tf32 = 1, and operands TMA can read  -> tcgen05 kernel (matmul_tc.cu): tensor cores,
//                                                              TMA-fed shared-memory stages, TMEM accumulators
//   fp32 with tf32 = 0 ("ieee"), or any other layout        -> this file's SIMT kernel: exact fp32 FMA for ieee;
//                                                              for tf32 it rounds the operands to tf32 first
#include <algorithm>
#include <cstring>

#include "common.cuh"

namespace nvb200 {

// Implemented in matmul_tc.cu. Return NVB200_ERR_UNSUPPORTED when the layout is not TMA-readable.
int matmul_swiglu_launch(void *c, const void *a, const void *b, int64_t M, int64_t N, int64_t K, int64_t sam,
                         int64_t sak, int64_t sbk, int64_t sbn, int64_t scm, int32_t *status, cudaStream_t stream);
int linear_decode_launch(void *y, const void *x, const void *w, int64_t M, int64_t N, int64_t K, int64_t sx,
                         int64_t sw, int64_t sy, bool swiglu, int32_t *status, cudaStream_t stream);
int linear_decode_plan(int64_t M, int64_t N, int64_t K, bool swiglu, int32_t *nt, int32_t *split);
int linear_qkv_launch(const void *x, int64_t sx, const void *w, int64_t sw, int64_t K,
                      const nvb200_qk_norm_rope_kv_args &a, cudaStream_t stream);
int64_t allreduce_buffer_bytes(int64_t max_n);
int matmul_allreduce_launch(void *c, const void *a, const void *b, int64_t M, int64_t N, int64_t K, int64_t sam,
                            int64_t sak, int64_t sbk, int64_t sbn, int64_t scm, const nvb200_allreduce_group *g,
                            int32_t *status, cudaStream_t stream);
int matmul_tc_launch(void *c, const void *a, const void *b, int64_t M, int64_t N, int64_t K, int64_t sam,
                     int64_t sak, int64_t sbk, int64_t sbn, int64_t scm, int64_t scn, int dtype, int32_t *status,
                     cudaStream_t stream);

namespace {

constexpr int BM = 128, BN = 128, BK = 16, kSimtThreads = 256, kGroupM = 8;

template <typename T> NVB200_DEVICE float load_operand(const T *p, bool tf32) {
  float v = Elem<T>::to_f(*p);
  if (tf32) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
    v = __uint_as_float(r);
  }
  return v;
}

// One CTA computes a BM x BN tile of C; 256 threads each own an 8 x 8 sub-tile split in two 4-row and two
// 4-column strips (rows tm*4.. and 64 + tm*4.., likewise columns) so shared-memory reads are conflict-free float4s.
// The next K tile is fetched into registers while the current one is multiplied from shared memory.
template <typename T>
__global__ void __launch_bounds__(kSimtThreads) matmul_simt_kernel(T *c, const T *a, const T *b, int M, int N, int K,
                                                                   int64_t sam, int64_t sak, int64_t sbk,
                                                                   int64_t sbn, int64_t scm, int64_t scn,
                                                                   bool tf32) {
  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];

  // GROUP_M swizzle of the linear CTA index (matmul.py:50-57).
  const int tiles_m = (M + BM - 1) / BM, tiles_n = (N + BN - 1) / BN;
  const int pid = blockIdx.x;
  const int in_group = kGroupM * tiles_n;
  const int first_m = (pid / in_group) * kGroupM;
  const int group_m = min(tiles_m - first_m, kGroupM);
  const int pm = first_m + (pid % in_group) % group_m;
  const int pn = (pid % in_group) / group_m;
  const int m0 = pm * BM, n0 = pn * BN;

  const int t = threadIdx.x;
  const int tm = t / 16, tn = t % 16;
  const bool a_kfast = sak == 1;  // A row-major: consecutive threads walk K
  const bool b_nfast = sbn == 1;  // B row-major [K, N]: consecutive threads walk N

  float ra[8], rb[8];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = t + kSimtThreads * i;
      int m, k;
      if (a_kfast) m = e / BK, k = e % BK; else m = e % BM, k = e / BM;
      const int gm = m0 + m, gk = k0 + k;
      ra[i] = (gm < M && gk < K) ? load_operand(a + gm * sam + gk * sak, tf32) : 0.f;
      int n, kb;
      if (b_nfast) n = e % BN, kb = e / BN; else n = e / BK, kb = e % BK;
      const int gn = n0 + n, gkb = k0 + kb;
      rb[i] = (gn < N && gkb < K) ? load_operand(b + gkb * sbk + gn * sbn, tf32) : 0.f;
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = t + kSimtThreads * i;
      int m, k;
      if (a_kfast) m = e / BK, k = e % BK; else m = e % BM, k = e / BM;
      As[buf][k][m] = ra[i];
      int n, kb;
      if (b_nfast) n = e % BN, kb = e / BN; else n = e / BK, kb = e % BK;
      Bs[buf][kb][n] = rb[i];
    }
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int ktiles = (K + BK - 1) / BK;
  fetch(0);
  stash(0);
  __syncthreads();
  for (int kt = 0; kt < ktiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ktiles) fetch((kt + 1) * BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][kk][tm * 4]);
      const float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][kk][64 + tm * 4]);
      const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][tn * 4]);
      const float4 b1 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][64 + tn * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (kt + 1 < ktiles) {
      stash(buf ^ 1);
      __syncthreads();
    }
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int gm = m0 + (i < 4 ? tm * 4 + i : 64 + tm * 4 + i - 4);
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + (j < 4 ? tn * 4 + j : 64 + tn * 4 + j - 4);
      if (gn < N) c[gm * scm + gn * scn] = Elem<T>::from_f(acc[i][j]);
    }
  }
}

int matmul_simt_launch(void *c, const void *a, const void *b, int64_t M, int64_t N, int64_t K, int64_t sam,
                       int64_t sak, int64_t sbk, int64_t sbn, int64_t scm, int64_t scn, int dtype, bool tf32,
                       cudaStream_t stream) {
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  if (tiles > 0x7fffffffLL || M > 0x7fffffffLL || N > 0x7fffffffLL || K > 0x7fffffffLL)
    return NVB200_ERR_UNSUPPORTED;
  const unsigned grid = static_cast<unsigned>(tiles);
  if (dtype == NVB200_BF16) {
    matmul_simt_kernel<__nv_bfloat16><<<grid, kSimtThreads, 0, stream>>>(
        static_cast<__nv_bfloat16 *>(c), static_cast<const __nv_bfloat16 *>(a), static_cast<const __nv_bfloat16 *>(b),
        static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), sam, sak, sbk, sbn, scm, scn, false);
  } else {
    matmul_simt_kernel<float><<<grid, kSimtThreads, 0, stream>>>(
        static_cast<float *>(c), static_cast<const float *>(a), static_cast<const float *>(b), static_cast<int>(M),
        static_cast<int>(N), static_cast<int>(K), sam, sak, sbk, sbn, scm, scn, tf32);
  }
  return launch_status();
}

}  // namespace
}  // namespace nvb200

using namespace nvb200;

extern "C" int64_t nvb200_matmul_workspace_size(int64_t M, int64_t N, int64_t K, int64_t sam, int64_t sak,
                                                int64_t sbk, int64_t sbn, int dtype) {
  (void)M, (void)N, (void)K, (void)sam, (void)sak, (void)sbk, (void)sbn, (void)dtype;
  return 0;
}

extern "C" int nvb200_matmul(void *c, const void *a, const void *b, int64_t M, int64_t N, int64_t K, int64_t sam,
                             int64_t sak, int64_t sbk, int64_t sbn, int64_t scm, int64_t scn, int dtype, int tf32,
                             void *workspace, int64_t workspace_bytes, int32_t *status, nvb200_stream_t stream) {
  (void)workspace, (void)workspace_bytes;
  if (M < 0 || N < 0 || K < 0) return NVB200_ERR_ARG;
  if (dtype != NVB200_BF16 && dtype != NVB200_F32) return NVB200_ERR_ARG;
  if (M == 0 || N == 0) return NVB200_OK;
  if (!c || (K > 0 && (!a || !b))) return NVB200_ERR_ARG;
  if (int rc = check_device()) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == NVB200_BF16 || tf32) {
    const int rc = matmul_tc_launch(c, a, b, M, N, K, sam, sak, sbk, sbn, scm, scn, dtype, status, s);
    if (rc != NVB200_ERR_UNSUPPORTED) return rc;
  }
  return matmul_simt_launch(c, a, b, M, N, K, sam, sak, sbk, sbn, scm, scn, dtype, tf32 != 0, s);
}

extern "C" int nvb200_matmul_silu_and_mul(void *c, const void *a, const void *b, int64_t M, int64_t N, int64_t K,
                                          int64_t sam, int64_t sak, int64_t sbk, int64_t sbn, int64_t scm,
                                          int32_t *status, nvb200_stream_t stream) {
  if (M < 0 || N < 0 || K < 0) return NVB200_ERR_ARG;
  if (M == 0 || N == 0) return NVB200_OK;
  if (K == 0) return NVB200_ERR_UNSUPPORTED;  // silu(0) * 0: left to the caller's unfused path
  if (!c || !a || !b) return NVB200_ERR_ARG;
  if (int rc = check_device()) return rc;
  return matmul_swiglu_launch(c, a, b, M, N, K, sam, sak, sbk, sbn, scm, status, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int nvb200_linear_decode(void *y, const void *x, const void *weight, int64_t M, int64_t N, int64_t K,
                                    int64_t sx, int64_t sw, int64_t sy, int swiglu, int32_t *status,
                                    nvb200_stream_t stream) {
  if (M < 0 || N < 0 || K < 0 || (swiglu != 0 && swiglu != 1)) return NVB200_ERR_ARG;
  if (M == 0 || N == 0) return NVB200_OK;
  if (K == 0) return NVB200_ERR_UNSUPPORTED;
  if (!y || !x || !weight) return NVB200_ERR_ARG;
  if (int rc = check_device()) return rc;
  return linear_decode_launch(y, x, weight, M, N, K, sx, sw, sy, swiglu != 0, status,
                              reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int nvb200_linear_decode_plan(int64_t M, int64_t N, int64_t K, int swiglu, int32_t *tiles,
                                         int32_t *split) {
  if (M < 0 || N < 0 || K < 0 || (swiglu != 0 && swiglu != 1)) return NVB200_ERR_ARG;
  return linear_decode_plan(M, N, K, swiglu != 0, tiles, split);
}

extern "C" int nvb200_linear_qkv_norm_rope_kv(const nvb200_linear_qkv_args *args, nvb200_stream_t stream) {
  if (args == nullptr) return NVB200_ERR_ARG;
  const nvb200_qk_norm_rope_kv_args &a = args->qknr;
  if (a.num_tokens < 0 || a.num_q_heads <= 0 || a.num_kv_heads <= 0 || a.num_q_heads % a.num_kv_heads != 0 ||
      a.head_dim <= 0 || args->K < 0 || a.num_positions <= 0 || a.cos_sin_stride < 0)
    return NVB200_ERR_ARG;
  if (a.k_cache != nullptr && (a.v_cache == nullptr || a.slot_mapping == nullptr || a.num_slots <= 0))
    return NVB200_ERR_ARG;
  if (a.num_tokens == 0) return NVB200_OK;
  if (args->K == 0) return NVB200_ERR_UNSUPPORTED;
  if (!args->x || !args->qkv_weight || !a.q_out || !a.positions || !a.q_weight || !a.k_weight || !a.cos_sin)
    return NVB200_ERR_ARG;
  if (int rc = check_device()) return rc;
  return linear_qkv_launch(args->x, args->x_row_stride, args->qkv_weight, args->weight_row_stride, args->K, a,
                           reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int64_t nvb200_allreduce_buffer_bytes(int64_t max_n) {
  return max_n > 0 ? allreduce_buffer_bytes(max_n) : 0;
}

extern "C" int nvb200_allreduce_buffer_create(int64_t max_n, void **buffer, void *ipc_handle) {
  if (max_n <= 0 || max_n > 0x3fffffffLL || buffer == nullptr || ipc_handle == nullptr) return NVB200_ERR_ARG;
  if (int rc = check_device()) return rc;
  const int64_t bytes = allreduce_buffer_bytes(max_n);
  void *p = nullptr;
  if (cudaMalloc(&p, static_cast<size_t>(bytes)) != cudaSuccess) return NVB200_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, static_cast<size_t>(bytes)) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return NVB200_ERR_CUDA;
  }
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  memcpy(ipc_handle, &h, sizeof(h));
  *buffer = p;
  return NVB200_OK;
}

extern "C" int nvb200_allreduce_buffer_open(const void *ipc_handle, void **buffer) {
  if (ipc_handle == nullptr || buffer == nullptr) return NVB200_ERR_ARG;
  if (int rc = check_device()) return rc;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cudaIpcOpenMemHandle(buffer, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? NVB200_OK : NVB200_ERR_CUDA;
}

extern "C" int nvb200_allreduce_buffer_close(void *buffer, int owned) {
  if (buffer == nullptr) return NVB200_OK;
  const cudaError_t e = owned ? cudaFree(buffer) : cudaIpcCloseMemHandle(buffer);
  return e == cudaSuccess ? NVB200_OK : NVB200_ERR_CUDA;
}

extern "C" int nvb200_matmul_allreduce(void *out, const void *a, const void *b, int64_t M, int64_t N, int64_t K,
                                       int64_t sam, int64_t sak, int64_t sbk, int64_t sbn, int64_t scm,
                                       const nvb200_allreduce_group *group, int32_t *status, nvb200_stream_t stream) {
  if (M < 0 || N < 0 || K < 0 || group == nullptr) return NVB200_ERR_ARG;
  if (M == 0 || N == 0) return NVB200_OK;
  if (!out || !a || !b) return NVB200_ERR_ARG;
  if (int rc = check_device()) return rc;
  return matmul_allreduce_launch(out, a, b, M, N, K, sam, sak, sbk, sbn, scm, group, status,
                                 reinterpret_cast<cudaStream_t>(stream));
}
