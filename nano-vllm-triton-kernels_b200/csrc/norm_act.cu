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

// Eight normalised bf16 outputs from fp32 values v, 1/rms and the raw bf16 weights: T(T(v * rstd) * w) as two
// packed conversions and a bf16x2 multiply per pair (the bf16 x bf16 product is exact in fp32, so mul.rn.bf16x2
// rounds it once, as torch's bf16 multiply does).
NVB200_DEVICE uint4 norm8_bf16(const float (&v)[8], float rstd, const uint4 &w) {
  return make_uint4(bf16x2_mul(pack_bf16x2(__fmul_rn(v[0], rstd), __fmul_rn(v[1], rstd)), w.x),
                    bf16x2_mul(pack_bf16x2(__fmul_rn(v[2], rstd), __fmul_rn(v[3], rstd)), w.y),
                    bf16x2_mul(pack_bf16x2(__fmul_rn(v[4], rstd), __fmul_rn(v[5], rstd)), w.z),
                    bf16x2_mul(pack_bf16x2(__fmul_rn(v[6], rstd), __fmul_rn(v[7], rstd)), w.w));
}

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
      if (ADD) VecIO<T, VEC>::store(so + col, v[k]);
      if constexpr (std::is_same<T, __nv_bfloat16>::value && VEC == 8) {
        *reinterpret_cast<uint4 *>(y + col) = norm8_bf16(v[k], rstd, wr[k]);
      } else {
        float wv[VEC], out[VEC];
        VecIO<T, VEC>::unpack(wr[k], wv);
#pragma unroll
        for (int e = 0; e < VEC; ++e) out[e] = norm_out<T>(v[k][e], rstd, wv[e]);
        VecIO<T, VEC>::store(y + col, out);
      }
    }
  }
}

// A group of L lanes (a power of two <= 32) per row; a CTA holds 256 / L rows.
template <typename T, int VEC, bool ADD>
__global__ void __launch_bounds__(kRowThreads) row_norm_kernel(const __grid_constant__ RowArgs a) {
  launch_dependents();  // a dependent launched early waits for this grid before reading its output
  grid_dependency_wait();  // this grid may itself have been launched early
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
  launch_dependents();  // a dependent launched early waits for this grid before reading its output
  grid_dependency_wait();  // this grid may itself have been launched early
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

// Large batches of short rows (up to 32 x kVecPerThread vectors, e.g. the 1024-element hidden of Qwen3-0.6B):
// a persistent grid of as many CTAs as are resident at once, each warp taking rows (32 / L of them per step, L lanes
// each) at a stride of the whole grid. A lane keeps its raw 16-byte vectors (x, and the residual for ADD) in
// registers and issues the loads of its next row before it reduces and stores the current one, so every warp has
// two rows in flight and no second wave waits for the first to drain (the one-row-per-warp kernel above ran 1.7
// waves at 8192 rows). fp32 values are recomputed from the raw vectors in each pass instead of being held.
template <typename T, int VEC, bool ADD>
__global__ void __launch_bounds__(kRowThreads) row_norm_pipe_kernel(const __grid_constant__ RowArgs a) {
  launch_dependents();  // a dependent launched early waits for this grid before reading its output
  grid_dependency_wait();  // this grid may itself have been launched early
  using Raw = RawVec<T, VEC>;
  const int L = a.lanes;
  const int lane = threadIdx.x & 31;
  const int li = lane % L;
  const int64_t step_rows = static_cast<int64_t>(gridDim.x) * (kRowThreads / L);
  const int64_t warp_first = (static_cast<int64_t>(blockIdx.x) * (kRowThreads / 32) + (threadIdx.x >> 5)) * (32 / L);
  const T *x = static_cast<const T *>(a.x);
  const T *r = static_cast<const T *>(a.r);
  const T *w = static_cast<const T *>(a.w);
  Raw xc[kVecPerThread], rc[kVecPerThread], xn[kVecPerThread], rn[kVecPerThread];

  auto load = [&](int64_t row, Raw (&xv)[kVecPerThread], Raw (&rv)[kVecPerThread]) {
    if (row >= a.rows) return;
    const T *xr = x + row_offset(a, row);
    const T *rr = ADD ? r + row * a.r_row_stride : nullptr;
#pragma unroll
    for (int k = 0; k < kVecPerThread; ++k) {
      const int col = (li + k * L) * VEC;
      if (col < a.n) {
        xv[k] = VecIO<T, VEC>::load_raw(xr + col);
        if (ADD) rv[k] = VecIO<T, VEC>::load_raw(rr + col);
      }
    }
  };
  // Sum of x (+ residual) in fp32, as the unrounded value torch normalises.
  auto value = [&](const Raw &xv, const Raw &rv, float (&v)[VEC]) {
    VecIO<T, VEC>::unpack(xv, v);
    if (ADD) {
      float t[VEC];
      VecIO<T, VEC>::unpack(rv, t);
#pragma unroll
      for (int e = 0; e < VEC; ++e) v[e] = __fadd_rn(v[e], t[e]);
    }
  };

  int64_t row = warp_first + lane / L;
  load(row, xc, rc);
  for (int64_t base = warp_first; base < a.rows; base += step_rows, row += step_rows) {
    load(row + step_rows, xn, rn);
    float ss = 0.f;
    if (row < a.rows) {
#pragma unroll
      for (int k = 0; k < kVecPerThread; ++k) {
        const int col = (li + k * L) * VEC;
        if (col < a.n) {
          float v[VEC];
          value(xc[k], rc[k], v);
          if (ADD) VecIO<T, VEC>::store(static_cast<T *>(a.res_out) + row * a.n + col, v);
#pragma unroll
          for (int e = 0; e < VEC; ++e) ss = fmaf(v[e], v[e], ss);
        }
      }
    }
    for (int o = L / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (row < a.rows) {
      const float rstd = rsqrtf(ss / static_cast<float>(a.n) + a.eps);
      T *y = static_cast<T *>(a.y) + row * a.n;
#pragma unroll
      for (int k = 0; k < kVecPerThread; ++k) {
        const int col = (li + k * L) * VEC;
        if (col < a.n) {
          float v[VEC];
          value(xc[k], rc[k], v);
          if constexpr (std::is_same<T, __nv_bfloat16>::value && VEC == 8) {
            *reinterpret_cast<uint4 *>(y + col) = norm8_bf16(v, rstd, __ldg(reinterpret_cast<const uint4 *>(w + col)));
          } else {
            float wv[VEC], out[VEC];
            VecIO<T, VEC>::load(w + col, wv);
#pragma unroll
            for (int e = 0; e < VEC; ++e) out[e] = norm_out<T>(v[e], rstd, wv[e]);
            VecIO<T, VEC>::store(y + col, out);
          }
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kVecPerThread; ++k) {
      xc[k] = xn[k];
      if (ADD) rc[k] = rn[k];
    }
  }
}

// Resident CTAs per SM of a kernel with `threads` threads and no dynamic shared memory (cached per device).
template <typename K> int resident_blocks(K kernel, int *cache, int threads = kRowThreads) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  if (cache[dev] == 0) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0) != cudaSuccess || per_sm < 1)
      per_sm = 1;
    cache[dev] = per_sm;
  }
  return cache[dev];
}

// Rows longer than a CTA holds in registers: one CTA per row, sum of squares first, then a second pass.
template <typename T, bool ADD>
__global__ void __launch_bounds__(kRowThreads) long_row_norm_kernel(const __grid_constant__ RowArgs a) {
  launch_dependents();  // a dependent launched early waits for this grid before reading its output
  grid_dependency_wait();  // this grid may itself have been launched early
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
    return launch_ex(block_row_norm_kernel<T, VEC, ADD>, dim3(static_cast<unsigned>(a.rows)), dim3(threads), 0,
                     stream, 1, NVB200_PDL_NORM, a);
  }
  if (nvec <= 32 * kVecPerThread) {
    int L = 1;
    while (L < 32 && L * kVecPerThread < nvec) L *= 2;
    a.lanes = L;
    const int64_t rows_per_block = kRowThreads / L;
    const int64_t blocks = (a.rows + rows_per_block - 1) / rows_per_block;
    if (blocks > 0x7fffffffLL) return NVB200_ERR_UNSUPPORTED;
    static int resident[64] = {0};
    const int64_t slots = static_cast<int64_t>(sm_count()) *
                          resident_blocks(row_norm_pipe_kernel<T, VEC, ADD>, resident);
    if (blocks > slots) {
      // More rows than one wave holds: the persistent two-rows-in-flight kernel.
      return launch_ex(row_norm_pipe_kernel<T, VEC, ADD>, dim3(static_cast<unsigned>(slots)), dim3(kRowThreads), 0,
                       stream, 1, NVB200_PDL_NORM, a);
    }
    return launch_ex(row_norm_kernel<T, VEC, ADD>, dim3(static_cast<unsigned>(blocks)), dim3(kRowThreads), 0,
                     stream, 1, NVB200_PDL_NORM, a);
  }
  if (a.rows > 0x7fffffffLL) return NVB200_ERR_UNSUPPORTED;
  if (nvec <= kMaxBlockThreads * kVecPerThread) {
    int threads = 64;
    while (threads * kVecPerThread < nvec) threads *= 2;
    return launch_ex(block_row_norm_kernel<T, VEC, ADD>, dim3(static_cast<unsigned>(a.rows)), dim3(threads), 0,
                     stream, 1, NVB200_PDL_NORM, a);
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
// row (bf16: two rows per step), no division on the index path.

template <typename T> NVB200_DEVICE float silu_mul(float g, float u) {
  // torch's silu: x / (1 + exp(-x)) in fp32, rounded to T; then T(silu * up) (exact product for 16-bit T).
  const float sl = g / (1.0f + expf(-g));
  return __fmul_rn(round_to<T>(sl), u);
}

constexpr int kSiluThreads = 128;
#ifndef NVB200_SILU_PIPE
#define NVB200_SILU_PIPE 1
#endif

template <typename T, int VEC>
__global__ void __launch_bounds__(kSiluThreads) silu_and_mul_kernel(T *out, const T *x, int64_t rows, int n,
                                                                     int64_t x_row_stride) {
  launch_dependents();  // a dependent launched early waits for this grid before reading its output
  grid_dependency_wait();  // this grid may itself have been launched early
  const int nv = n / VEC;
  const int cv = blockIdx.x * kSiluThreads + threadIdx.x;
  if (cv >= nv) return;
  const int col = cv * VEC;
  int64_t r = blockIdx.y;
  if constexpr (std::is_same<T, __nv_bfloat16>::value && VEC == 8) {
#if NVB200_SILU_PIPE
    // Two rows per step, and the next step's four 16-byte loads issued before this step's arithmetic, so the loads
    // of one step overlap the SiLU arithmetic of the previous one.
    const int64_t step = gridDim.y;
    auto ld = [&](int64_t row, uint4 &g, uint4 &u) {
      if (row < rows) {
        const T *s0 = x + row * x_row_stride + col;
        g = *reinterpret_cast<const uint4 *>(s0), u = *reinterpret_cast<const uint4 *>(s0 + n);
      }
    };
    uint4 g0{}, u0{}, g1{}, u1{}, h0{}, v0{}, h1{}, v1{};
    ld(r, g0, u0);
    ld(r + step, g1, u1);
    for (; r < rows; r += 2 * step) {
      ld(r + 2 * step, h0, v0);
      ld(r + 3 * step, h1, v1);
      *reinterpret_cast<uint4 *>(out + r * n + col) = silu_mul8_bf16(g0, u0);
      if (r + step < rows) *reinterpret_cast<uint4 *>(out + (r + step) * n + col) = silu_mul8_bf16(g1, u1);
      g0 = h0, u0 = v0, g1 = h1, u1 = v1;
    }
    r = rows;  // every row done: the loop below has nothing left
#else
    // Two rows per step: four 16-byte loads in flight per thread before the arithmetic.
    const int64_t step = gridDim.y;
    for (; r + step < rows; r += 2 * step) {
      const T *s0 = x + r * x_row_stride + col, *s1 = s0 + step * x_row_stride;
      const uint4 g0 = *reinterpret_cast<const uint4 *>(s0), u0 = *reinterpret_cast<const uint4 *>(s0 + n);
      const uint4 g1 = *reinterpret_cast<const uint4 *>(s1), u1 = *reinterpret_cast<const uint4 *>(s1 + n);
      *reinterpret_cast<uint4 *>(out + r * n + col) = silu_mul8_bf16(g0, u0);
      *reinterpret_cast<uint4 *>(out + (r + step) * n + col) = silu_mul8_bf16(g1, u1);
    }
#endif
  }
  for (; r < rows; r += gridDim.y) {
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
  // As many CTAs as are resident at once (one wave), each column of CTAs striding over the rows.
  static int resident[2][64] = {{0}};
  const int per_sm = vec ? resident_blocks(silu_and_mul_kernel<T, VEC>, resident[0], kSiluThreads)
                         : resident_blocks(silu_and_mul_kernel<T, 1>, resident[1], kSiluThreads);
  const int64_t cap_y = std::max<int64_t>(1, static_cast<int64_t>(sm_count()) * per_sm / gx);
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

// ---------------------------------------------------------------------------------------------------------------
// Bulk-copy RMSNorm for long bf16 rows in large batches (the producer / consumer pipeline of the fused q/k kernel).
// A unit is R consecutive rows. Warp 0 (one lane) copies each unit's rows HBM -> shared memory with cp.async.bulk
// into a ring of stages (completion counted in mbarrier transaction bytes); consumer warp w owns stages w, w + W, ...
// (so it observes every phase of their barriers), normalises the rows in place and writes them with cp.async.bulk
// stores, then frees the stage once the stores have read it. The copies keep tens of KB per SM in flight without
// registers, which the register kernels cannot for 8 KB rows (one 128-thread CTA per row, 64 B in flight per
// thread). Measured on B200 at 8192 rows: 4096-element rows 28.7 us against 32.8 us for the register kernel;
// 1024-element rows no faster, and Add+RMSNorm and SiLU x Mul slower (their register kernels keep more loads in
// flight per thread, and SiLU's arithmetic wants more warps than a producer / consumer CTA has), so only RMSNorm
// with rows of at least kStreamMinRowBytes takes this path.

constexpr int kStreamWarps = 8;      // consumer warps per CTA
constexpr int kStreamCtas = 2;       // CTAs per SM
constexpr int kStreamMaxStages = 8;  // multiple of kStreamWarps
constexpr int kStreamHeader = 256;   // full[kStreamMaxStages], empty[kStreamMaxStages]
constexpr int kStreamUnitTarget = 12 * 1024;
constexpr int kStreamBudget = (228 * 1024) / kStreamCtas - 1024 - kStreamHeader;
constexpr int kStreamMinRowBytes = 8 * 1024;
#ifndef NVB200_STREAM_MIN_ROWS
#define NVB200_STREAM_MIN_ROWS 2048
#endif
constexpr int64_t kStreamMinRows = NVB200_STREAM_MIN_ROWS;  // below this the register kernels are as fast

struct StreamArgs {
  const __nv_bfloat16 *x, *w;
  __nv_bfloat16 *y;
  int64_t rows;
  int64_t x_stride;  // elements between consecutive rows of x
  int n;             // elements per row
  int rows_per_unit;
  int64_t units, chunk;  // units in total, units per CTA
  int stages, consumers, stage_bytes;
  float eps;
  int32_t *status;
};

NVB200_DEVICE int stream_next_unit(int it, int NS, int W) {
  const int st = it % NS;
  return st + W < NS ? it + W : it - st + NS + st % W;
}

__global__ void __launch_bounds__(32 * (1 + kStreamWarps), kStreamCtas)
    rms_stream_kernel(const __grid_constant__ StreamArgs a) {
  launch_dependents();  // a dependent launched early waits for this grid before reading its output
  grid_dependency_wait();  // this grid may itself have been launched early
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NS = a.stages;
  const uint32_t bar_base = smem_addr(smem);  // full[0..NS), empty[0..NS)
  const uint32_t stage_base = smem_addr(smem + kStreamHeader);
  const int64_t first = static_cast<int64_t>(blockIdx.x) * a.chunk;
  if (first >= a.units) return;
  const int n_units = static_cast<int>(a.chunk < a.units - first ? a.chunk : a.units - first);
  const int R = a.rows_per_unit;
  const uint32_t rb = 2u * static_cast<uint32_t>(a.n);  // bytes of one row
  const int64_t x_pitch = a.x_stride * 2;               // bytes between rows of x

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(bar_base + 8 * i, 1);
      mbar_init(bar_base + 8 * (NS + i), 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------------------------ producer (lane 0)
    if (lane != 0) return;
    const uint8_t *xb = reinterpret_cast<const uint8_t *>(a.x);
    const bool dense = x_pitch == static_cast<int64_t>(rb);
    for (int it = 0; it < n_units; ++it) {
      const int st = it % NS;
      const uint32_t full = bar_base + 8 * st, empty = bar_base + 8 * (NS + st);
      if (!mbar_wait_bounded(empty, ((it / NS) & 1) ^ 1)) {
        set_status(a.status, NVB200_STATUS_WAIT_TIMEOUT);
        return;
      }
      const int64_t r0 = (first + it) * R;
      const int nr = static_cast<int>(R < a.rows - r0 ? R : a.rows - r0);
      const uint32_t sb = stage_base + st * a.stage_bytes;
      mbar_arrive_expect_tx(full, nr * rb);
      if (dense) {
        bulk_g2s(sb, xb + r0 * x_pitch, nr * rb, full);
      } else {
        for (int i = 0; i < nr; ++i) bulk_g2s(sb + i * rb, xb + (r0 + i) * x_pitch, rb, full);
      }
    }
    return;
  }

  // -------------------------------------------------------------------- consumers
  const int cw = warp - 1;
  const int nw = a.consumers;
  if (cw >= nw) return;
  const int nv = a.n / 8;
  for (int it = cw; it < n_units; it = stream_next_unit(it, NS, nw)) {
    const int st = it % NS;
    const uint32_t full = bar_base + 8 * st, empty = bar_base + 8 * (NS + st);
    if (!mbar_wait_bounded(full, (it / NS) & 1)) {
      if (lane == 0) set_status(a.status, NVB200_STATUS_WAIT_TIMEOUT);
      break;
    }
    const int64_t r0 = (first + it) * R;
    const int nr = static_cast<int>(R < a.rows - r0 ? R : a.rows - r0);
    const uint32_t sb = stage_base + st * a.stage_bytes;
    for (int i = 0; i < nr; ++i) {
      const uint32_t xr = sb + i * rb;
      float ss = 0.f;
      for (int v = lane; v < nv; v += 32) {
        float f[8];
        unpack8(ld_shared_v4(xr + 16 * v), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rstd = rsqrtf(ss / static_cast<float>(a.n) + a.eps);
      // y = T(T(x * rstd) * w): the bf16 x bf16 product is exact in fp32, so mul.rn.bf16x2 rounds it once.
      for (int v = lane; v < nv; v += 32) {
        float f[8];
        unpack8(ld_shared_v4(xr + 16 * v), f);
        const uint4 wv = __ldg(reinterpret_cast<const uint4 *>(a.w) + v);
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          o[k] = bf16x2_mul(pack_bf16x2(__fmul_rn(f[2 * k], rstd), __fmul_rn(f[2 * k + 1], rstd)), ww[k]);
        st_shared_v4(xr + 16 * v, make_uint4(o[0], o[1], o[2], o[3]));
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      bulk_s2g(a.y + r0 * a.n, sb, nr * rb);
      bulk_commit();
      bulk_wait_read<0>();  // the stores have read the stage: hand it back to the producer
      mbar_arrive(empty);
    }
    __syncwarp();
  }
  // Stores still in flight may finish after the CTA exits; their shared-memory reads are done (waited above).
}

// Launches the bulk-copy RMSNorm when it applies (bf16, long rows of whole 16-byte vectors, 16-byte aligned rows,
// a large batch); returns NVB200_ERR_UNSUPPORTED otherwise so the caller runs the register kernels.
int launch_rms_stream(StreamArgs &a, cudaStream_t stream) {
  const int rb = 2 * a.n;
  if (a.rows < kStreamMinRows || a.n % 8 != 0 || rb < kStreamMinRowBytes || rb > kStreamBudget / 2)
    return NVB200_ERR_UNSUPPORTED;
  a.rows_per_unit = std::max(1, kStreamUnitTarget / rb);
  a.stage_bytes = a.rows_per_unit * rb;
  a.stages = std::min(kStreamMaxStages, kStreamBudget / a.stage_bytes);
  a.consumers = std::min(kStreamWarps, a.stages);
  a.stages -= a.stages % a.consumers;
  a.units = (a.rows + a.rows_per_unit - 1) / a.rows_per_unit;
  if (a.units > 0x7fffffffLL) return NVB200_ERR_UNSUPPORTED;
  const int smem = kStreamHeader + a.stages * a.stage_bytes;
  static int configured[64] = {0};  // per device: max dynamic shared memory raised once
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(rms_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kStreamHeader + kStreamBudget) != cudaSuccess)
      return NVB200_ERR_CUDA;
    configured[dev] = 1;
  }
  const int64_t grid = std::min<int64_t>(a.units, static_cast<int64_t>(sm_count()) * kStreamCtas);
  a.chunk = (a.units + grid - 1) / grid;
  const int64_t blocks = (a.units + a.chunk - 1) / a.chunk;
  rms_stream_kernel<<<static_cast<unsigned>(blocks), 32 * (1 + kStreamWarps), smem, stream>>>(a);
  return launch_status();
}

}  // namespace
}  // namespace nvb200

using namespace nvb200;

extern "C" int nvb200_rms_norm(void *y, const void *x, const void *w, int64_t groups, int64_t rows_per_group,
                               int64_t group_stride, int64_t row_stride, int64_t n, float eps, int dtype,
                               int32_t *status, nvb200_stream_t stream) {
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
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == NVB200_BF16 && vec_ok && rows_per_group == 1) {
    StreamArgs sa{};
    sa.x = static_cast<const __nv_bfloat16 *>(x), sa.w = static_cast<const __nv_bfloat16 *>(w);
    sa.y = static_cast<__nv_bfloat16 *>(y), sa.rows = rows, sa.x_stride = group_stride, sa.n = static_cast<int>(n);
    sa.eps = eps, sa.status = status;
    const int rc = launch_rms_stream(sa, s);
    if (rc != NVB200_ERR_UNSUPPORTED) return rc;
  }
  return dispatch_norm<false>(a, vec_ok, dtype, s);
}

extern "C" int nvb200_fused_add_rms_norm(void *y, void *residual_out, const void *x, const void *residual,
                                         const void *w, int64_t rows, int64_t n, int64_t x_row_stride,
                                         int64_t residual_row_stride, float eps, int dtype, int32_t *status,
                                         nvb200_stream_t stream) {
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
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return dispatch_norm<true>(a, vec_ok, dtype, s);
}

extern "C" int nvb200_silu_and_mul(void *out, const void *x, int64_t rows, int64_t n, int64_t x_row_stride,
                                   int dtype, int32_t *status, nvb200_stream_t stream) {
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
