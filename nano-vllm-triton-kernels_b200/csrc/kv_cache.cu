// Plain paged KV-cache write: row t of key and value ([Hkv * D] elements) is copied to row slot_mapping[t] of the
// k and v caches, and tokens whose slot is -1 are skipped. This is the non-fused route of the reference's attention
// layer (nanovllm/layers/attention.py:11-41, store_kvcache and store_kvcache_kernel), taken by models whose q/k are
// normalised and rotated before the attention layer (qkv_bias models, models/qwen3.py:68-73,99-103).
//
// HBM-bound copy: a warp moves a token's two rows with the widest access that every address and stride allows
// (16, 8, 4 or 2 bytes), issuing all of a lane's loads before its stores so that several are in flight; rows of up
// to 128 accesses (2 KB at 16 bytes) take a persistent kernel that keeps two tokens per warp in flight.
// Slots outside [-1, num_slots) are not stored and are reported in the status word (the reference leaves them
// undefined).
#include <algorithm>

#include "common.cuh"

namespace nvb200 {
namespace {

constexpr int kStoreWarps = 8;                // tokens per CTA at a time
constexpr int kStoreThreads = kStoreWarps * 32;
constexpr int kStoreUnroll = 4;               // accesses per lane in flight, per row

template <int VEC> struct VecType;
template <> struct VecType<16> { using T = uint4; };
template <> struct VecType<8> { using T = uint2; };
template <> struct VecType<4> { using T = uint32_t; };
template <> struct VecType<2> { using T = uint16_t; };

struct StoreArgs {
  const char *key;
  const char *value;
  int64_t key_stride;    // bytes between tokens
  int64_t value_stride;  // bytes between tokens
  char *k_cache;
  char *v_cache;
  const void *slots;
  int64_t tokens;
  int64_t row_bytes;
  int64_t num_slots;
  int slot64;            // slot_mapping holds int64 (else int32)
  int32_t *status;
};

template <int VEC>
__global__ void __launch_bounds__(kStoreThreads) store_kvcache_kernel(const __grid_constant__ StoreArgs a) {
  using V = typename VecType<VEC>::T;
  const int lane = threadIdx.x & 31;
  const int64_t chunks = a.row_bytes / VEC;
  const int64_t step = static_cast<int64_t>(gridDim.x) * kStoreWarps;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kStoreWarps + (threadIdx.x >> 5); t < a.tokens; t += step) {
    const int64_t slot = a.slot64 ? static_cast<int64_t>(__ldg(static_cast<const long long *>(a.slots) + t))
                                  : static_cast<int64_t>(__ldg(static_cast<const int *>(a.slots) + t));
    if (slot == -1) continue;
    if (slot < 0 || slot >= a.num_slots) {
      if (lane == 0) set_status(a.status, NVB200_STATUS_BAD_SLOT);
      continue;
    }
    const V *__restrict__ ks = reinterpret_cast<const V *>(a.key + t * a.key_stride);
    const V *__restrict__ vs = reinterpret_cast<const V *>(a.value + t * a.value_stride);
    V *__restrict__ kd = reinterpret_cast<V *>(a.k_cache + slot * a.row_bytes);
    V *__restrict__ vd = reinterpret_cast<V *>(a.v_cache + slot * a.row_bytes);
    for (int64_t c0 = lane; c0 < chunks; c0 += 32 * kStoreUnroll) {
      V kr[kStoreUnroll], vr[kStoreUnroll];
#pragma unroll
      for (int u = 0; u < kStoreUnroll; ++u) {
        const int64_t c = c0 + 32 * u;
        if (c < chunks) kr[u] = __ldg(ks + c), vr[u] = __ldg(vs + c);
      }
#pragma unroll
      for (int u = 0; u < kStoreUnroll; ++u) {
        const int64_t c = c0 + 32 * u;
        if (c < chunks) kd[c] = kr[u], vd[c] = vr[u];
      }
    }
  }
}

// Rows of at most 32 x kStoreUnroll accesses (a 2 KB row of 16-byte accesses: 8 kv heads of 128 bf16) on a
// persistent grid. Warp w takes tokens w, w + W, w + 2W, ... (W warps in the grid) in batches of 32: one load per
// lane fetches the batch's 32 slot numbers at once, and the rows of a batch's next kept token are loaded before the
// current token's are stored, so each warp keeps two tokens' rows in flight and no row load waits behind its slot.
template <int VEC>
__global__ void __launch_bounds__(kStoreThreads) store_kvcache_pipe_kernel(const __grid_constant__ StoreArgs a) {
  using V = typename VecType<VEC>::T;
  const int lane = threadIdx.x & 31;
  const int chunks = static_cast<int>(a.row_bytes / VEC);
  const int64_t W = static_cast<int64_t>(gridDim.x) * kStoreWarps;
  const int64_t w = static_cast<int64_t>(blockIdx.x) * kStoreWarps + (threadIdx.x >> 5);
  V k0[kStoreUnroll], v0[kStoreUnroll], k1[kStoreUnroll], v1[kStoreUnroll];
  auto load_rows = [&](int64_t t, V (&kr)[kStoreUnroll], V (&vr)[kStoreUnroll]) {
    const V *__restrict__ ks = reinterpret_cast<const V *>(a.key + t * a.key_stride);
    const V *__restrict__ vs = reinterpret_cast<const V *>(a.value + t * a.value_stride);
#pragma unroll
    for (int u = 0; u < kStoreUnroll; ++u) {
      const int c = lane + 32 * u;
      if (c < chunks) kr[u] = __ldg(ks + c), vr[u] = __ldg(vs + c);
    }
  };
  auto store_rows = [&](int64_t slot, const V (&kr)[kStoreUnroll], const V (&vr)[kStoreUnroll]) {
    V *__restrict__ kd = reinterpret_cast<V *>(a.k_cache + slot * a.row_bytes);
    V *__restrict__ vd = reinterpret_cast<V *>(a.v_cache + slot * a.row_bytes);
#pragma unroll
    for (int u = 0; u < kStoreUnroll; ++u) {
      const int c = lane + 32 * u;
      if (c < chunks) kd[c] = kr[u], vd[c] = vr[u];
    }
  };
  for (int64_t base = w; base < a.tokens; base += 32 * W) {
    // Slot of this lane's token of the batch; -1 for tokens past the end, and out-of-range slots flagged and
    // skipped here so the loop below only sees -1 or valid slots.
    const int64_t tl = base + lane * W;
    int64_t slot = -1;
    if (tl < a.tokens) {
      slot = a.slot64 ? static_cast<int64_t>(__ldg(static_cast<const long long *>(a.slots) + tl))
                      : static_cast<int64_t>(__ldg(static_cast<const int *>(a.slots) + tl));
      if (slot < -1 || slot >= a.num_slots) {
        set_status(a.status, NVB200_STATUS_BAD_SLOT);
        slot = -1;
      }
    }
    // The batch's kept tokens in order, two at a time through the two register buffers: the next token's rows are
    // loaded before the current token's are stored.
    uint32_t kept = __ballot_sync(0xffffffffu, slot >= 0);
    if (kept == 0) continue;
    int j = __ffs(kept) - 1;
    kept &= kept - 1;
    load_rows(base + j * W, k0, v0);
    while (true) {
      int64_t sj = __shfl_sync(0xffffffffu, slot, j);
      int next = kept ? __ffs(kept) - 1 : -1;
      if (next >= 0) {
        kept &= kept - 1;
        load_rows(base + next * W, k1, v1);
      }
      store_rows(sj, k0, v0);
      if (next < 0) break;
      j = next;
      sj = __shfl_sync(0xffffffffu, slot, j);
      next = kept ? __ffs(kept) - 1 : -1;
      if (next >= 0) {
        kept &= kept - 1;
        load_rows(base + next * W, k0, v0);
      }
      store_rows(sj, k1, v1);
      if (next < 0) break;
      j = next;
    }
  }
}

bool divides(int v, uintptr_t x) { return x % static_cast<uintptr_t>(v) == 0; }

template <int VEC> int resident_store_blocks() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  if (cached[dev] == 0) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, store_kvcache_pipe_kernel<VEC>, kStoreThreads, 0) !=
            cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    cached[dev] = per_sm;
  }
  return cached[dev];
}

template <int VEC> int launch_store(const StoreArgs &a, cudaStream_t stream) {
  const int64_t need = (a.tokens + kStoreWarps - 1) / kStoreWarps;
  if (a.row_bytes / VEC <= 32 * kStoreUnroll) {
    const int64_t slots = static_cast<int64_t>(sm_count()) * resident_store_blocks<VEC>();
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(need, slots));
    store_kvcache_pipe_kernel<VEC><<<static_cast<unsigned>(grid), kStoreThreads, 0, stream>>>(a);
    return launch_status();
  }
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(need, static_cast<int64_t>(sm_count()) * 16));
  store_kvcache_kernel<VEC><<<static_cast<unsigned>(grid), kStoreThreads, 0, stream>>>(a);
  return launch_status();
}

}  // namespace
}  // namespace nvb200

using namespace nvb200;

extern "C" int nvb200_store_kvcache(const void *key, int64_t key_token_stride, const void *value,
                                    int64_t value_token_stride, void *k_cache, void *v_cache,
                                    const void *slot_mapping, int slot_bytes, int64_t num_tokens, int64_t row_elems,
                                    int64_t num_slots, int dtype, int32_t *status, nvb200_stream_t stream) {
  if (num_tokens < 0 || row_elems <= 0 || num_slots < 0) return NVB200_ERR_ARG;
  if (dtype != NVB200_BF16 && dtype != NVB200_F16 && dtype != NVB200_F32) return NVB200_ERR_ARG;
  if (slot_bytes != 4 && slot_bytes != 8) return NVB200_ERR_ARG;
  if (num_tokens == 0) return NVB200_OK;
  if (!key || !value || !k_cache || !v_cache || !slot_mapping) return NVB200_ERR_ARG;
  const int64_t es = dtype == NVB200_F32 ? 4 : 2;
  if (row_elems > INT64_MAX / es / 2) return NVB200_ERR_ARG;
  if (int rc = check_device()) return rc;
  StoreArgs a{};
  a.key = static_cast<const char *>(key), a.value = static_cast<const char *>(value);
  a.key_stride = key_token_stride * es, a.value_stride = value_token_stride * es;
  a.k_cache = static_cast<char *>(k_cache), a.v_cache = static_cast<char *>(v_cache);
  a.slots = slot_mapping, a.tokens = num_tokens, a.row_bytes = row_elems * es, a.num_slots = num_slots;
  a.slot64 = slot_bytes == 8, a.status = status;
  // The widest access that divides every base address, token stride and the row size.
  const uintptr_t bits = reinterpret_cast<uintptr_t>(key) | reinterpret_cast<uintptr_t>(value) |
                         reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
                         static_cast<uintptr_t>(a.key_stride) | static_cast<uintptr_t>(a.value_stride) |
                         static_cast<uintptr_t>(a.row_bytes);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (divides(16, bits)) return launch_store<16>(a, s);
  if (divides(8, bits)) return launch_store<8>(a, s);
  if (divides(4, bits)) return launch_store<4>(a, s);
  if (divides(2, bits)) return launch_store<2>(a, s);
  return NVB200_ERR_ARG;  // an element pointer that is not even 2-byte aligned
}
