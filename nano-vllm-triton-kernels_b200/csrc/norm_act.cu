// RMSNorm, Add+RMSNorm and SiLU x Mul on strided row views, for sm_100a.
//
// Behaviour follows nanovllm/kernels/rms_norm.py:34-80 and nanovllm/kernels/swiglu.py:19-31, whose numerics are the
// torch code of nanovllm/layers/layernorm.py:20-44 and nanovllm/layers/activation.py:15-18:
//   rms_norm      y = T(T(x.float() * rsqrt(mean(x.float()^2) + eps)) * w)
//   add_rms_norm  s = x.float() + r.float(); residual_out = T(s); y = rms_norm of the unrounded s
//   silu_and_mul  out = T(T(silu(gate.float())) * up)
// where T(.) rounds to the tensor dtype (bf16, fp16 or fp32) and the product of two bf16/fp16 values is exact in
// fp32, so T(a * b) equals torch's dtype multiply.
//
// These ops are HBM-bound (bytes per row: rms 2n, add_rms 4n, silu 3n elements). Every row lives in registers, up
// to 4 16-byte vectors per thread: rows of up to 1024 bf16 elements (512 fp32) take a group of L lanes (L a power of
// two <= 32, sum of squares by log2(L) shuffles), rows up to 32768 bf16 elements one CTA each (block reduction).
// Longer rows take a CTA and a second pass over the row (served from L2).
#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace nvb200 {
namespace {

constexpr int kRowThreads = 256;
constexpr int kVecPerThread = 4;        // 16-byte vectors a thread holds of its row
constexpr int kMaxBlockThreads = 1024;  // block-per-row kernel: threads per row

// VEC consecutive elements of type T: raw 16-byte (or scalar) loads and stores, and conversion to/from fp32.
template <typename T, int VEC> struct VecIO;
template <> struct VecIO<__nv_bfloat16, 8> {
  using Raw = uint4;
  static NVB200_DEVICE Raw load_raw(const __nv_bfloat16 *p) { return *reinterpret_cast<const uint4 *>(p); }
  static NVB200_DEVICE void unpack(const Raw &r, float (&f)[8]) { unpack8(r, f); }
  static NVB200_DEVICE void load(const __nv_bfloat16 *p, float (&f)[8]) { unpack8(load_raw(p), f); }
  static NVB200_DEVICE void store(__nv_bfloat16 *p, const float (&f)[8]) { *reinterpret_cast<uint4 *>(p) = pack8(f); }
};
template <> struct VecIO<__half, 8> {
  using Raw = uint4;
  static NVB200_DEVICE Raw load_raw(const __half *p) { return *reinterpret_cast<const uint4 *>(p); }
  static NVB200_DEVICE void unpack(const Raw &r, float (&f)[8]) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  static NVB200_DEVICE void load(const __half *p, float (&f)[8]) { unpack(load_raw(p), f); }
  static NVB200_DEVICE void store(__half *p, const float (&f)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t *>(&h);
    }
    *reinterpret_cast<uint4 *>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  }
};
template <> struct VecIO<float, 4> {
  using Raw = float4;
  static NVB200_DEVICE Raw load_raw(const float *p) { return *reinterpret_cast<const float4 *>(p); }
  static NVB200_DEVICE void unpack(const Raw &v, float (&f)[4]) { f[0] = v.x, f[1] = v.y, f[2] = v.z, f[3] = v.w; }
  static NVB200_DEVICE void load(const float *p, float (&f)[4]) { unpack(load_raw(p), f); }
  static NVB200_DEVICE void store(float *p, const float (&f)[4]) {
    *reinterpret_cast<float4 *>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
};
template <typename T> struct VecIO<T, 1> {
  using Raw = T;
  static NVB200_DEVICE Raw load_raw(const T *p) { return *p; }
  static NVB200_DEVICE void unpack(const Raw &r, float (&f)[1]) { f[0] = Elem<T>::to_f(r); }
  static NVB200_DEVICE void load(const T *p, float (&f)[1]) { f[0] = Elem<T>::to_f(*p); }
  static NVB200_DEVICE void store(T *p, const float (&f)[1]) { *p = Elem<T>::from_f(f[0]); }
};

struct RowArgs {
  void *y;
  void *res_out;
  const void *x;
  const void *r;
  const void *w;
  int64_t rows;
  int64_t rows_per_group;  // rms_norm 3-D views; 1 otherwise
  int64_t x_group_stride, x_row_stride, r_row_stride;
  int n;
  int lanes;  // L: lanes per row (register kernel)
  float eps;
};

// y = T(T(v * rstd) * w): v * rstd rounded to fp32 then to T, times w in fp32 (exact for 16-bit T), rounded.
// Element offset of row `row` of x: 2-D views (rows_per_group == 1) need no division; 3-D [T, H, n] views divide in
// 32 bits (the host guarantees rows < 2^31), avoiding the slow 64-bit division routine on the load path.
NVB200_DEVICE int64_t row_offset(const RowArgs &a, int64_t row) {
  if (a.rows_per_group == 1) return row * a.x_group_stride;
  const uint32_t r = static_cast<uint32_t>(row), h = static_cast<uint32_t>(a.rows_per_group);
  const uint32_t g = r / h;
  return static_cast<int64_t>(g) * a.x_group_stride + static_cast<int64_t>(r - g * h) * a.x_row_stride;
}

template <typename T> NVB200_DEVICE float norm_out(float v, float rstd, float w) {
  return __fmul_rn(round_to<T>(__fmul_rn(v, rstd)), w);
}

template <typename T, int VEC> using RawVec = typename VecIO<T, VEC>::Raw;

// Loads this thread's vectors of one row (x, plus the residual for ADD, summed in fp32) and the matching weight
// vectors (raw, issued with the row's loads so the store pass does not wait for them); returns the thread's
// partial sum of squares.
template <typename T, int VEC, bool ADD>
NVB200_DEVICE float load_row(const T *x, const T *r, const T *w, int n, int first, int step,
                             float (&v)[kVecPerThread][VEC], RawVec<T, VEC> (&wr)[kVecPerThread]) {
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kVecPerThread; ++k) {
    const int col = (first + k * step) * VEC;
    if (col < n) {
      VecIO<T, VEC>::load(x + col, v[k]);
      wr[k] = VecIO<T, VEC>::load_raw(w + col);
      if (ADD) {
        float rv[VEC];
        VecIO<T, VEC>::load(r + col, rv);
#pragma unroll
        for (int e = 0; e < VEC; ++e) v[k][e] = __fadd_rn(v[k][e], rv[e]);
      }
#pragma unroll
      for (int e = 0; e < VEC; ++e) ss = fmaf(v[k][e], v[k][e], ss);
    }
  }
  return ss;
}

template <typename T, int VEC, bool ADD>
NVB200_DEVICE void store_row(T *y, T *so, int n, int first, int step, float rstd, const float (&v)[kVecPerThread][VEC],
                             const RawVec<T, VEC> (&wr)[kVecPerThread]) {
#pragma unroll
  for (int k = 0; k < kVecPerThread; ++k) {
    const int col = (first + k * step) * VEC;
    if (col < n) {
      float wv[VEC], out[VEC];
      VecIO<T, VEC>::unpack(wr[k], wv);
      if (ADD) VecIO<T, VEC>::store(so + col, v[k]);
#pragma unroll
      for (int e = 0; e < VEC; ++e) out[e] = norm_out<T>(v[k][e], rstd, wv[e]);
      VecIO<T, VEC>::store(y + col, out);
    }
  }
}

// A group of L lanes (a power of two <= 32) per row; a CTA holds 256 / L rows.
template <typename T, int VEC, bool ADD>
__global__ void __launch_bounds__(kRowThreads) row_norm_kernel(const __grid_constant__ RowArgs a) {
  const int L = a.lanes;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kRowThreads / L) + threadIdx.x / L;
  const int li = threadIdx.x % L;
  const bool live = row < a.rows;
  const T *x = static_cast<const T *>(a.x);
  const T *r = static_cast<const T *>(a.r);
  float v[kVecPerThread][VEC];
  RawVec<T, VEC> wr[kVecPerThread];
  float ss = 0.f;
  if (live) {
    const int64_t xoff = row_offset(a, row);
    ss = load_row<T, VEC, ADD>(x + xoff, ADD ? r + row * a.r_row_stride : nullptr, static_cast<const T *>(a.w), a.n,
                               li, L, v, wr);
  }
  for (int o = L / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (!live) return;
  const float rstd = rsqrtf(ss / static_cast<float>(a.n) + a.eps);
  store_row<T, VEC, ADD>(static_cast<T *>(a.y) + row * a.n, ADD ? static_cast<T *>(a.res_out) + row * a.n : nullptr,
                         a.n, li, L, rstd, v, wr);
}

// One CTA (blockDim.x threads, a multiple of 32) per row, the row in registers, a block-wide sum of squares.
template <typename T, int VEC, bool ADD>
__global__ void __launch_bounds__(kMaxBlockThreads) block_row_norm_kernel(const __grid_constant__ RowArgs a) {
  __shared__ float partial[kMaxBlockThreads / 32];
  const int64_t row = blockIdx.x;
  const T *x = static_cast<const T *>(a.x) + row_offset(a, row);
  const T *r = ADD ? static_cast<const T *>(a.r) + row * a.r_row_stride : nullptr;
  float v[kVecPerThread][VEC];
  RawVec<T, VEC> wr[kVecPerThread];
  float ss = load_row<T, VEC, ADD>(x, r, static_cast<const T *>(a.w), a.n, threadIdx.x, blockDim.x, v, wr);
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) tot += partial[i];
  const float rstd = rsqrtf(tot / static_cast<float>(a.n) + a.eps);
  store_row<T, VEC, ADD>(static_cast<T *>(a.y) + row * a.n, ADD ? static_cast<T *>(a.res_out) + row * a.n : nullptr,
                         a.n, threadIdx.x, blockDim.x, rstd, v, wr);
}

// Rows longer than a CTA holds in registers: one CTA per row, sum of squares first, then a second pass.
template <typename T, bool ADD>
__global__ void __launch_bounds__(kRowThreads) long_row_norm_kernel(const __grid_constant__ RowArgs a) {
  __shared__ float partial[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const T *x = static_cast<const T *>(a.x) + row_offset(a, row);
  const T *r = ADD ? static_cast<const T *>(a.r) + row * a.r_row_stride : nullptr;
  const T *w = static_cast<const T *>(a.w);
  T *y = static_cast<T *>(a.y) + row * a.n;
  T *so = ADD ? static_cast<T *>(a.res_out) + row * a.n : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x; i < a.n; i += kRowThreads) {
    float s = Elem<T>::to_f(x[i]);
    if (ADD) {
      s = __fadd_rn(s, Elem<T>::to_f(r[i]));
      so[i] = Elem<T>::from_f(s);
    }
    ss = fmaf(s, s, ss);
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kRowThreads / 32; ++i) tot += partial[i];
  const float rstd = rsqrtf(tot / static_cast<float>(a.n) + a.eps);
  for (int i = threadIdx.x; i < a.n; i += kRowThreads) {
    float s = Elem<T>::to_f(x[i]);
    if (ADD) s = __fadd_rn(s, Elem<T>::to_f(r[i]));
    y[i] = Elem<T>::from_f(norm_out<T>(s, rstd, Elem<T>::to_f(w[i])));
  }
}

// Up to this many rows, rows of 64..128 vectors (e.g. the 1024-element hidden of Qwen3-0.6B) take one CTA each with
// one vector per thread (shorter serial chain per thread at decode sizes); measured on B200: better up to ~1024
// rows, worse beyond, and worse for longer rows, which keep 4 vectors per thread.
constexpr int kFewRows = 1024;

template <typename T, int VEC, bool ADD> int launch_norm_vec(RowArgs &a, cudaStream_t stream) {
  const int nvec = (a.n + VEC - 1) / VEC;
  if (a.rows <= kFewRows && nvec >= 64 && nvec <= 32 * kVecPerThread) {
    // Decode-sized batches: spread each row over a CTA so every thread does one vector (short serial chain).
    const int threads = (nvec + 31) / 32 * 32;
    block_row_norm_kernel<T, VEC, ADD><<<static_cast<unsigned>(a.rows), threads, 0, stream>>>(a);
    return launch_status();
  }
  if (nvec <= 32 * kVecPerThread) {
    int L = 1;
    while (L < 32 && L * kVecPerThread < nvec) L *= 2;
    a.lanes = L;
    const int64_t rows_per_block = kRowThreads / L;
    const int64_t blocks = (a.rows + rows_per_block - 1) / rows_per_block;
    if (blocks > 0x7fffffffLL) return NVB200_ERR_UNSUPPORTED;
    row_norm_kernel<T, VEC, ADD><<<static_cast<unsigned>(blocks), kRowThreads, 0, stream>>>(a);
    return launch_status();
  }
  if (a.rows > 0x7fffffffLL) return NVB200_ERR_UNSUPPORTED;
  if (nvec <= kMaxBlockThreads * kVecPerThread) {
    int threads = 64;
    while (threads * kVecPerThread < nvec) threads *= 2;
    block_row_norm_kernel<T, VEC, ADD><<<static_cast<unsigned>(a.rows), threads, 0, stream>>>(a);
    return launch_status();
  }
  long_row_norm_kernel<T, ADD><<<static_cast<unsigned>(a.rows), kRowThreads, 0, stream>>>(a);
  return launch_status();
}

template <typename T, bool ADD> int launch_norm(RowArgs &a, bool vec_ok, cudaStream_t stream) {
  constexpr int VEC = sizeof(T) == 4 ? 4 : 8;
  if (vec_ok && a.n % VEC == 0) return launch_norm_vec<T, VEC, ADD>(a, stream);
  return launch_norm_vec<T, 1, ADD>(a, stream);
}

template <bool ADD> int dispatch_norm(RowArgs &a, bool vec_ok, int dtype, cudaStream_t stream) {
  switch (dtype) {
    case NVB200_BF16: return launch_norm<__nv_bfloat16, ADD>(a, vec_ok, stream);
    case NVB200_F16: return launch_norm<__half, ADD>(a, vec_ok, stream);
    case NVB200_F32: return launch_norm<float, ADD>(a, vec_ok, stream);
    default: return NVB200_ERR_ARG;
  }
}

int elem_size(int dtype) { return dtype == NVB200_F32 ? 4 : 2; }

// ---------------------------------------------------------------------------------------------------------------
// SiLU x Mul: thread (x, y) owns vector column x of rows y, y + gridDim.y, ...: two 16-byte loads and one store per
// step, no division on the index path. (Taking 4 rows per step, or prefetching the next row into registers,
// measured no faster at 8192 rows.)

template <typename T> NVB200_DEVICE float silu_mul(float g, float u) {
  // torch's silu: x / (1 + exp(-x)) in fp32, rounded to T; then T(silu * up) (exact product for 16-bit T).
  const float sl = g / (1.0f + expf(-g));
  return __fmul_rn(round_to<T>(sl), u);
}

// bf16 fast path. silu(g) rounded to bf16 depends only on the 16-bit g, so an estimate that lies close enough to
// the exact fp32 value rounds the same way. __expf and __fdividef estimate g / (1 + exp(-g)) within a few tens of
// fp32 ulps for |g| <= 16 (documented bounds: 2 + floor(1.173 |x|) ulps and 2 ulps); wherever the estimate's low
// 16 bits lie within kSiluMargin of the bf16 rounding midpoint 0x8000, or |g| > 16 (or g is not finite), the exact
// expression is evaluated instead. Away from the midpoint, round-to-nearest-even is round-half-up on the bit
// pattern. The exact path costs about twice the instructions (accurate expf, IEEE division) and kept the kernel
// issue-bound below the memory roofline; the tests compare all 65,536 bf16 gate values with torch bit for bit.
constexpr float kSiluFastRange = 16.0f;
constexpr uint32_t kSiluMargin = 64;

NVB200_DEVICE uint32_t silu_bf16_bits(float g) {
  const uint32_t b = __float_as_uint(__fdividef(g, 1.0f + __expf(-g)));
  const uint32_t low = b & 0xFFFFu;
  const uint32_t dist = low >= 0x8000u ? low - 0x8000u : 0x8000u - low;
  if (fabsf(g) <= kSiluFastRange && dist > kSiluMargin) return (b + 0x8000u) >> 16;
  return __bfloat16_as_ushort(__float2bfloat16_rn(g / (1.0f + expf(-g))));
}

// Eight gate and eight up values (bf16) -> eight outputs: silu rounded to bf16, times up, rounded once
// (mul.rn.bf16x2: the product of two bf16 values is exact in fp32, so this is torch's fp32 multiply then round).
NVB200_DEVICE uint4 silu_mul8_bf16(const uint4 &g, const uint4 &u) {
  const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, uw[4] = {u.x, u.y, u.z, u.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo = silu_bf16_bits(__uint_as_float(gw[i] << 16));
    const uint32_t hi = silu_bf16_bits(__uint_as_float(gw[i] & 0xFFFF0000u));
    o[i] = bf16x2_mul(lo | (hi << 16), uw[i]);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

constexpr int kSiluThreads = 128;

template <typename T, int VEC>
__global__ void __launch_bounds__(kSiluThreads) silu_and_mul_kernel(T *out, const T *x, int64_t rows, int n,
                                                                     int64_t x_row_stride) {
  const int nv = n / VEC;
  const int cv = blockIdx.x * kSiluThreads + threadIdx.x;
  if (cv >= nv) return;
  const int col = cv * VEC;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const T *src = x + r * x_row_stride + col;
    if constexpr (std::is_same<T, __nv_bfloat16>::value && VEC == 8) {
      const uint4 g = *reinterpret_cast<const uint4 *>(src), u = *reinterpret_cast<const uint4 *>(src + n);
      *reinterpret_cast<uint4 *>(out + r * n + col) = silu_mul8_bf16(g, u);
    } else {
      float g[VEC], u[VEC], o[VEC];
      VecIO<T, VEC>::load(src, g);
      VecIO<T, VEC>::load(src + n, u);
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] = silu_mul<T>(g[e], u[e]);
      VecIO<T, VEC>::store(out + r * n + col, o);
    }
  }
}

template <typename T> int launch_silu(void *out, const void *x, int64_t rows, int64_t n, int64_t stride,
                                      bool vec_ok, cudaStream_t stream) {
  constexpr int VEC = sizeof(T) == 4 ? 4 : 8;
  const bool vec = vec_ok && n % VEC == 0;
  const int64_t nv = vec ? n / VEC : n;
  const int64_t gx = (nv + kSiluThreads - 1) / kSiluThreads;
  if (gx > 0x7fffffffLL) return NVB200_ERR_UNSUPPORTED;
  const int64_t cap_y = std::max<int64_t>(1, static_cast<int64_t>(sm_count()) * 16 / gx);  // ~16 CTAs per SM
  const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(std::min<int64_t>(std::min(rows, cap_y), 65535)));
  T *o = static_cast<T *>(out);
  const T *i = static_cast<const T *>(x);
  const int ni = static_cast<int>(n);
  if (vec)
    silu_and_mul_kernel<T, VEC><<<grid, kSiluThreads, 0, stream>>>(o, i, rows, ni, stride);
  else
    silu_and_mul_kernel<T, 1><<<grid, kSiluThreads, 0, stream>>>(o, i, rows, ni, stride);
  return launch_status();
}

}  // namespace
}  // namespace nvb200

using namespace nvb200;

extern "C" int nvb200_rms_norm(void *y, const void *x, const void *w, int64_t groups, int64_t rows_per_group,
                               int64_t group_stride, int64_t row_stride, int64_t n, float eps, int dtype,
                               nvb200_stream_t stream) {
  if (groups < 0 || rows_per_group <= 0 || n <= 0 || n > 0x7fffffffLL) return NVB200_ERR_ARG;
  if (dtype != NVB200_BF16 && dtype != NVB200_F16 && dtype != NVB200_F32) return NVB200_ERR_ARG;
  const int64_t rows = groups * rows_per_group;
  if (rows == 0) return NVB200_OK;
  if (rows_per_group > 1 && rows > 0x7fffffffLL) return NVB200_ERR_UNSUPPORTED;
  if (!y || !x || !w) return NVB200_ERR_ARG;
  if (int rc = check_device()) return rc;
  const int es = elem_size(dtype);
  RowArgs a{};
  a.y = y, a.x = x, a.w = w, a.rows = rows, a.rows_per_group = rows_per_group;
  a.x_group_stride = group_stride, a.x_row_stride = row_stride, a.n = static_cast<int>(n), a.eps = eps;
  const bool vec_ok = aligned16(y) && aligned16(x) && aligned16(w) && (group_stride * es) % 16 == 0 &&
                      (row_stride * es) % 16 == 0;
  return dispatch_norm<false>(a, vec_ok, dtype, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int nvb200_fused_add_rms_norm(void *y, void *residual_out, const void *x, const void *residual,
                                         const void *w, int64_t rows, int64_t n, int64_t x_row_stride,
                                         int64_t residual_row_stride, float eps, int dtype, nvb200_stream_t stream) {
  if (rows < 0 || n <= 0 || n > 0x7fffffffLL) return NVB200_ERR_ARG;
  if (dtype != NVB200_BF16 && dtype != NVB200_F16 && dtype != NVB200_F32) return NVB200_ERR_ARG;
  if (rows == 0) return NVB200_OK;
  if (!y || !residual_out || !x || !residual || !w) return NVB200_ERR_ARG;
  if (int rc = check_device()) return rc;
  const int es = elem_size(dtype);
  RowArgs a{};
  a.y = y, a.res_out = residual_out, a.x = x, a.r = residual, a.w = w, a.rows = rows, a.rows_per_group = 1;
  a.x_group_stride = x_row_stride, a.x_row_stride = 0, a.r_row_stride = residual_row_stride;
  a.n = static_cast<int>(n), a.eps = eps;
  const bool vec_ok = aligned16(y) && aligned16(residual_out) && aligned16(x) && aligned16(residual) &&
                      aligned16(w) && (x_row_stride * es) % 16 == 0 && (residual_row_stride * es) % 16 == 0;
  return dispatch_norm<true>(a, vec_ok, dtype, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int nvb200_silu_and_mul(void *out, const void *x, int64_t rows, int64_t n, int64_t x_row_stride,
                                   int dtype, nvb200_stream_t stream) {
  if (rows < 0 || n <= 0 || n > 0x3fffffffLL) return NVB200_ERR_ARG;
  if (rows == 0) return NVB200_OK;
  if (!out || !x) return NVB200_ERR_ARG;
  if (int rc = check_device()) return rc;
  const int es = elem_size(dtype);
  const bool vec_ok = aligned16(out) && aligned16(x) && (x_row_stride * es) % 16 == 0 && (n * es) % 16 == 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case NVB200_BF16: return launch_silu<__nv_bfloat16>(out, x, rows, n, x_row_stride, vec_ok, s);
    case NVB200_F16: return launch_silu<__half>(out, x, rows, n, x_row_stride, vec_ok, s);
    case NVB200_F32: return launch_silu<float>(out, x, rows, n, x_row_stride, vec_ok, s);
    default: return NVB200_ERR_ARG;
  }
}
