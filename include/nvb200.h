/* nvb200.h — C ABI of the B200 (sm_100a) kernels behind nanovllm_b200.
 *
 * Every entry point takes plain device pointers, element strides and sizes, launches on the given CUDA
 * stream, never synchronises, never allocates and never reads device data on the host, so each call can be
 * captured in a CUDA graph (nvb200_paged_decode_attention_noalloc aside: nothing is stated about capturing it).
 * The return value is NVB200_OK or an NVB200_ERR_* code; no C++ exception crosses this boundary. Strides are in
 * ELEMENTS (as torch's Tensor.stride()), sizes in elements.
 *
 * The Python functions that mirror the reference's nanovllm/kernels API (nanovllm_b200.kernels.*) validate
 * their torch arguments exactly as the reference's wrappers do, allocate the outputs with torch, and then call
 * these functions through ctypes. A C, C++ or Python/ctypes caller can call them directly.
 */
#ifndef NVB200_H
#define NVB200_H

#include <stdint.h>

#if defined(__GNUC__)
#define NVB200_API __attribute__((visibility("default")))
#else
#define NVB200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t; NULL is the legacy default stream. */
typedef struct CUstream_st *nvb200_stream_t;

enum {
  NVB200_OK = 0,
  NVB200_ERR_ARG = 1,         /* a size, stride, pointer or dtype that the op does not accept */
  NVB200_ERR_UNSUPPORTED = 2, /* a valid request that this build has no kernel for (e.g. head_dim > 512) */
  NVB200_ERR_CUDA = 3,        /* a CUDA runtime call or the launch itself failed (cudaGetLastError) */
  NVB200_ERR_NO_DEVICE = 4    /* the current device is not sm_100 */
};

/* Element types. */
enum { NVB200_BF16 = 0, NVB200_F16 = 1, NVB200_F32 = 2 };

/* Bits an entry point may OR into its optional device status word (int32, zero it to clear). The kernels
 * never trap: an index they cannot honour is skipped and reported here. */
enum {
  NVB200_STATUS_BAD_POSITION = 1, /* positions[t] outside [0, num_positions): cos/sin row 0 used instead  */
  NVB200_STATUS_BAD_SLOT = 2,     /* slot_mapping[t] outside [-1, num_slots): the k/v rows are not stored */
  NVB200_STATUS_WAIT_TIMEOUT = 4  /* an mbarrier wait ran past its bound; the CTA stopped early            */
};

/* Human-readable name of an NVB200_* return code. */
NVB200_API const char *nvb200_status_string(int code);

/* Fused per-head q/k RMSNorm + neox RoPE + paged KV-cache write.
 * Replaces: nanovllm/kernels/qk_norm_rope_kv.py:92-125 (qk_norm_rope_kv) and its Triton kernel :45-82.
 *
 *   q [T, Hq, D], k, v [T, Hkv, D] bf16, each head contiguous (stride(2) == 1, stride(1) == D), any token stride.
 *   positions [T] int64; cos_sin fp32 rows of D (cos | sin), row r at cos_sin + r * cos_sin_stride.
 *   q_weight, k_weight [D] bf16.
 *   k_cache, v_cache: contiguous [num_slots, Hkv, D] bf16 (a [blocks, block_size, Hkv, D] cache), or both NULL:
 *     then nothing is stored and slot_mapping may be NULL. slot_mapping [T] int32, -1 = do not store.
 *   q_out [T, Hq, D] contiguous bf16 (written), k_out [T, Hkv, D] contiguous bf16 or NULL (normed+rotated k).
 *   status: optional int32 device word for NVB200_STATUS_* bits, may be NULL.
 * Numerics: n = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w) per head in fp32; y1 = n1*cos - n2*sin,
 * y2 = n2*cos + n1*sin with separately rounded fp32 products (no FMA), rounded to bf16. v is stored raw. */
typedef struct nvb200_qk_norm_rope_kv_args {
  void *q_out;
  void *k_out;
  const void *q;
  const void *k;
  const void *v;
  int64_t q_token_stride;
  int64_t k_token_stride;
  int64_t v_token_stride;
  const int64_t *positions;
  const int32_t *slot_mapping;
  const void *q_weight;
  const void *k_weight;
  const float *cos_sin;
  int64_t cos_sin_stride;
  int64_t num_positions;
  void *k_cache;
  void *v_cache;
  int64_t num_slots;
  int64_t num_tokens;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  float eps;
  int32_t *status;
} nvb200_qk_norm_rope_kv_args;

NVB200_API int nvb200_qk_norm_rope_kv(const nvb200_qk_norm_rope_kv_args *args, nvb200_stream_t stream);

/* Which kernel nvb200_qk_norm_rope_kv would launch for these arguments on the current device, without launching
 * anything: *kernel gets an NVB200_QKNR_KERNEL_* code and *tokens_per_unit the tokens one work unit covers (either
 * pointer may be NULL). Returns what nvb200_qk_norm_rope_kv would return for an argument error; T = 0 gives
 * NVB200_QKNR_KERNEL_NONE. Host-only (reads the SM count), for tests and tools that check a shape's route.
 * Replaces: nothing in the reference (its wrapper always launches one Triton kernel, qk_norm_rope_kv.py:117-124). */
enum {
  NVB200_QKNR_KERNEL_NONE = 0,    /* T = 0: no launch                                                        */
  NVB200_QKNR_KERNEL_GENERIC = 1, /* rows not 16-byte aligned or D outside {64, 128, 256}: one warp per head  */
  NVB200_QKNR_KERNEL_DIRECT = 2,  /* T <= 512, or q/k/v rows of at most 40 MB: direct loads and stores       */
  NVB200_QKNR_KERNEL_MULTI = 3,   /* small tokens in a rank's qkv_proj layout: units of 4-16 tokens, bulk copies */
  NVB200_QKNR_KERNEL_BULK = 4     /* one token (or a head group of one) per unit, bulk-copy pipeline          */
};
NVB200_API int nvb200_qk_norm_rope_kv_plan(const nvb200_qk_norm_rope_kv_args *args, int32_t *kernel,
                                           int32_t *tokens_per_unit);

/* RMSNorm over the last dim, y contiguous [groups * rows_per_group, n].
 * Replaces: nanovllm/kernels/rms_norm.py:83-98 (rms_norm) and _rms_norm_kernel :34-54.
 * Row g * rows_per_group + r of x starts at x + g * group_stride + r * row_stride (a 2-D [rows, n] view is
 * groups = rows, rows_per_group = 1; a 3-D [T, H, n] view is groups = T, rows_per_group = H). Unit last stride.
 * y = (x.float() * rsqrt(mean(x.float()^2) + eps)).to(dtype) * w, the product in dtype.
 * status (nullable, device int32): NVB200_STATUS_WAIT_TIMEOUT is OR-ed in if a pipeline wait gave up (long bf16
 * rows in large batches run a bulk-copy pipeline whose waits are bounded). The two functions below take the same
 * argument for the same purpose; their current kernels have no waits and never set it. */
NVB200_API int nvb200_rms_norm(void *y, const void *x, const void *w, int64_t groups, int64_t rows_per_group,
                    int64_t group_stride, int64_t row_stride, int64_t n, float eps, int dtype,
                    int32_t *status, nvb200_stream_t stream);

/* s = x + residual in fp32; residual_out = s.to(dtype); y = RMSNorm of the unrounded s. y, residual_out
 * contiguous [rows, n]; x and residual have unit last stride and any row stride.
 * Replaces: nanovllm/kernels/rms_norm.py:101-111 (fused_add_rms_norm) and _fused_add_rms_norm_kernel :57-80. */
NVB200_API int nvb200_fused_add_rms_norm(void *y, void *residual_out, const void *x, const void *residual, const void *w,
                              int64_t rows, int64_t n, int64_t x_row_stride, int64_t residual_row_stride,
                              float eps, int dtype, int32_t *status, nvb200_stream_t stream);

/* out[r, :] = silu(x[r, :n].float()).to(dtype) * x[r, n:2n]; out contiguous [rows, n]; x unit last stride.
 * Replaces: nanovllm/kernels/swiglu.py:34-43 (silu_and_mul) and _silu_and_mul_kernel :19-31. */
NVB200_API int nvb200_silu_and_mul(void *out, const void *x, int64_t rows, int64_t n, int64_t x_row_stride, int dtype,
                        int32_t *status, nvb200_stream_t stream);

/* C[M, N] = A[M, K] @ B[K, N] with fp32 accumulation, C in the inputs' dtype (bf16 or fp32).
 * Replaces: nanovllm/kernels/matmul.py:84-99 (matmul) and _matmul_kernel :33-81.
 * Any strides for A and B (B is typically weight.t(), strides (1, K)); C any strides.
 * dtype: NVB200_BF16 (tcgen05 kind::f16) or NVB200_F32 with tf32 = 1 (tcgen05 kind::tf32, inputs rounded to
 * tf32) or tf32 = 0 ("ieee": fp32 FMA on the CUDA cores).
 * workspace, workspace_bytes: reserved for kernels that need device scratch; nvb200_matmul_workspace_size()
 * tells how much a call needs, and every current path needs none (it returns 0, and both may be 0 / NULL). */
NVB200_API int64_t nvb200_matmul_workspace_size(int64_t M, int64_t N, int64_t K, int64_t sam, int64_t sak, int64_t sbk,
                                     int64_t sbn, int dtype);
NVB200_API int nvb200_matmul(void *c, const void *a, const void *b, int64_t M, int64_t N, int64_t K, int64_t sam,
                  int64_t sak, int64_t sbk, int64_t sbn, int64_t scm, int64_t scn, int dtype, int tf32,
                  void *workspace, int64_t workspace_bytes, int32_t *status, nvb200_stream_t stream);

/* out[M, N] = silu(G).to(bf16) * U, where [G | U] = A[M, K] @ B[K, 2N] in bf16 (G the first N columns): the gate_up
 * projection and SiLU x Mul of a SwiGLU MLP in one kernel, without writing the [M, 2N] intermediate. Bitwise equal
 * to nvb200_matmul into a bf16 [M, 2N] followed by nvb200_silu_and_mul.
 * Replaces: nanovllm/kernels/matmul.py:84-99 (matmul, whose module notes plan this SiLU*up epilogue at :3-4)
 * followed by nanovllm/kernels/swiglu.py:34-43 (silu_and_mul), as layers/activation.py:15-22 applies it to
 * MergedColumnParallelLinear's output (models/qwen3.py:133-137).
 * bf16 only; A and B each with one unit stride (TMA-readable, 16-byte aligned), out row-major with a 16-byte row
 * pitch scm. Returns NVB200_ERR_UNSUPPORTED for layouts it does not take (K = 0 included), in which case the
 * caller runs the two steps separately. */
NVB200_API int nvb200_matmul_silu_and_mul(void *out, const void *a, const void *b, int64_t M, int64_t N, int64_t K,
                               int64_t sam, int64_t sak, int64_t sbk, int64_t sbn, int64_t scm, int32_t *status,
                               nvb200_stream_t stream);

/* y[M, N] = x[M, K] @ weight[N, K]^T for decode-sized batches (bf16, 1 <= M <= 64): a linear layer's projection
 * with the layer's weight read as it is stored (nn.Linear layout, K-major rows). The caller guarantees that no
 * kernel still in flight on the stream writes `weight` (model parameters), which lets the launch start the weight
 * loads while the preceding kernel finishes (programmatic dependent launch; x is read only after it completes).
 * swiglu = 1: weight holds 2N rows, the N gate rows then the N up rows (MergedColumnParallelLinear's gate_up
 * layout), and y = silu(x gate^T).to(bf16) * (x up^T).to(bf16), the SiLU x Mul of the two-step form.
 * Replaces: F.linear in ColumnParallelLinear.forward / RowParallelLinear.forward (nanovllm/layers/linear.py:72-73,
 * :152-153; the projections of models/qwen3.py) at decode-sized batches, and for swiglu = 1 the gate_up projection
 * with SiluAndMul (models/qwen3.py:133-137, kernels/swiglu.py:34-43).
 * x and weight with unit last strides (row pitches sx, sw, 16-byte multiples, bases 16-byte aligned), y row-major with
 * row pitch sy. Returns NVB200_ERR_UNSUPPORTED for shapes or layouts it does not take (M > 64, K = 0 included): the
 * caller then runs F.linear / nvb200_matmul. */
NVB200_API int nvb200_linear_decode(void *y, const void *x, const void *weight, int64_t M, int64_t N, int64_t K,
                                    int64_t sx, int64_t sw, int64_t sy, int swiglu, int32_t *status,
                                    nvb200_stream_t stream);

/* The launch shape nvb200_linear_decode picks for an M x N x K call on the current device (148 SMs when no GPU
 * answers), without launching: *tiles = 8-column tiles per CTA (the CTA's weight rows / 8; with swiglu half of them
 * gate rows), *split = CTAs of a thread-block cluster that split K. NVB200_ERR_UNSUPPORTED for shapes the kernel does
 * not take. Host-only, for tests and tools. Replaces: nothing in the reference. */
NVB200_API int nvb200_linear_decode_plan(int64_t M, int64_t N, int64_t K, int swiglu, int32_t *tiles, int32_t *split);

/* The decode qkv projection with the fused q/k op as its epilogue: qkv = x[M, K] @ qkv_weight^T rounded to bf16
 * ([Hq q heads | Hkv k heads | Hkv v heads] of 128 columns, QKVParallelLinear's layout), then exactly what
 * nvb200_qk_norm_rope_kv does with q, k, v = the three parts of qkv: q heads RMSNorm + RoPE into q_out, k heads
 * RMSNorm + RoPE into k_cache[slot], v heads into v_cache[slot] (slot -1 skipped; k_cache NULL: nothing stored).
 * The qkv intermediate is never written. As for nvb200_linear_decode, qkv_weight is a model parameter that no kernel
 * in flight writes (its loads may start while the preceding kernel finishes).
 * Replaces: the qkv_proj F.linear (nanovllm/layers/linear.py:72-73 via models/qwen3.py:91-94) followed by
 * qk_norm_rope_kv (nanovllm/kernels/qk_norm_rope_kv.py:92-125, called at layers/attention.py:71-72) in the decode
 * branch of kernel_backend "triton_fused".
 * qknr: the fused op's arguments with num_tokens = M; q, k, v and their strides are ignored; k_out must be NULL.
 * Takes bf16, 1 <= M <= 32, head_dim 128, x and qkv_weight with unit last strides and 16-byte row pitches (x_row_stride,
 * weight_row_stride in elements); NVB200_ERR_UNSUPPORTED otherwise (the caller runs the two steps). */
typedef struct nvb200_linear_qkv_args {
  const void *x;
  int64_t x_row_stride;
  const void *qkv_weight;
  int64_t weight_row_stride;
  int64_t K;
  nvb200_qk_norm_rope_kv_args qknr;
} nvb200_linear_qkv_args;

NVB200_API int nvb200_linear_qkv_norm_rope_kv(const nvb200_linear_qkv_args *args, nvb200_stream_t stream);

/* Row-parallel GEMM fused with its all-reduce over NVLink (decode-sized rows), for tensor parallelism: rank r
 * holds A_r [M, K_r] and B_r [K_r, N] (its K shard); every rank receives out[M, N] = sum over ranks of A_r @ B_r in
 * bf16, summed in fp32 in rank order (so every rank gets the same bits). One kernel per rank computes its partial
 * with the tensor cores, pushes it into every rank's exchange buffer over NVLink and sums the ranks' partials in
 * rank order as they arrive (each partial travels as 8-byte words tagged with the call's epoch: no flags or fences).
 * Replaces: nanovllm/layers/linear.py:131-156 (RowParallelLinear.forward: F.linear, then dist.all_reduce).
 * Exchange buffers: one per rank, nvb200_allreduce_buffer_bytes(max_n) bytes, created by
 * nvb200_allreduce_buffer_create (cudaMalloc'd and zeroed: a set-up call, not a per-step one) and shared through
 * its CUDA IPC handle (64 bytes); each rank opens its peers' handles with nvb200_allreduce_buffer_open. The group
 * lists every rank's buffer as mapped in the calling process (buffers[rank] = its own). The call number (epoch) is
 * kept in each rank's buffer and advanced by the kernel, so calls may be captured in a CUDA graph and replayed.
 * All ranks must make the same sequence of calls with the same shapes on one set of buffers; the kernels of one
 * call must run concurrently on all ranks (one process per GPU).
 * Takes bf16, M <= 64, N a multiple of 4 and <= max_n, A row-major and B K-major (an nn.Linear weight.t()), and a
 * grid that fits on the GPU at once; returns NVB200_ERR_UNSUPPORTED otherwise (the caller then runs a GEMM and an
 * all-reduce). A peer that does not arrive within 1 s sets NVB200_STATUS_WAIT_TIMEOUT in *status. */
typedef struct {
  int world;            /* ranks, 2..8 */
  int rank;             /* this rank */
  int64_t max_n;        /* the max_n the buffers were created with */
  void *buffers[8];     /* every rank's exchange buffer, as mapped in this process */
} nvb200_allreduce_group;

NVB200_API int64_t nvb200_allreduce_buffer_bytes(int64_t max_n);
NVB200_API int nvb200_allreduce_buffer_create(int64_t max_n, void **buffer, void *ipc_handle);
NVB200_API int nvb200_allreduce_buffer_open(const void *ipc_handle, void **buffer);
NVB200_API int nvb200_allreduce_buffer_close(void *buffer, int owned);
NVB200_API int nvb200_matmul_allreduce(void *out, const void *a, const void *b, int64_t M, int64_t N, int64_t K,
                            int64_t sam, int64_t sak, int64_t sbk, int64_t sbn, int64_t scm,
                            const nvb200_allreduce_group *group, int32_t *status, nvb200_stream_t stream);

/* Paged KV-cache write without norm or RoPE: row t of key and value (row_elems = Hkv * D elements, contiguous) is
 * copied to row slot_mapping[t] of k_cache and v_cache (row s at element s * row_elems); slot -1 is skipped.
 * Replaces: nanovllm/layers/attention.py:34-41 (store_kvcache) and store_kvcache_kernel :11-31, the attention
 * layer's non-fused route (:75-76).
 * key, value: token t's row at key + t * key_token_stride (elements). slot_mapping: int32 (slot_bytes 4) or int64
 * (slot_bytes 8). num_slots: rows the caches hold; a slot outside [-1, num_slots) is not stored and sets
 * NVB200_STATUS_BAD_SLOT in *status (nullable). dtype: NVB200_BF16, NVB200_F16 or NVB200_F32 (a byte copy). */
NVB200_API int nvb200_store_kvcache(const void *key, int64_t key_token_stride, const void *value,
                                    int64_t value_token_stride, void *k_cache, void *v_cache,
                                    const void *slot_mapping, int slot_bytes, int64_t num_tokens, int64_t row_elems,
                                    int64_t num_slots, int dtype, int32_t *status, nvb200_stream_t stream);

/* Paged decode attention: out[b, i, hq] = softmax(q[b, i, hq] . K^T * softmax_scale) V over the keys of sequence b
 * in the paged cache, K and V of KV head hq / (num_q_heads / num_kv_heads). With causal != 0 query i of n =
 * queries_per_seq sees keys [0, seqlens[b] - n + i] (bottom-right alignment); otherwise keys [0, seqlens[b]). A query
 * that sees no key gets zeros.
 * Replaces: the flash_attn_with_kvcache call of nanovllm/layers/attention.py:84-91 (the decode branch of
 * Attention.forward: q [num_seqs, n, Hq, D], cache_seqlens = context_lens, block_table = block_tables, causal).
 *   q: [batch, queries_per_seq, num_q_heads, head_dim] with the given element strides and a unit last stride.
 *   k_cache, v_cache: [num_blocks, block_size, num_kv_heads, head_dim], both with the given strides, unit last stride.
 *   block_table: [batch, max_blocks_per_seq] int32, row stride block_table_stride; key j of sequence b is token
 *     j % block_size of block block_table[b, j / block_size]. NULL: sequence b is block b (max_blocks_per_seq 1).
 *   seqlens: [batch] int32, the keys in the cache per sequence (the new tokens included).
 *   out: [batch, queries_per_seq, num_q_heads, head_dim] contiguous, written.
 *   num_splits: CTAs (a thread-block cluster) sharing one sequence's keys, 1..8; 0 = chosen from the sizes
 *     (nvb200_paged_decode_splits tells which).
 * Takes bf16, head_dim 128, queries_per_seq * (num_q_heads / num_kv_heads) <= 16 and 16-byte aligned cache rows;
 * returns NVB200_ERR_UNSUPPORTED otherwise. Block-table entries outside [0, num_blocks) and seqlens beyond
 * max_blocks_per_seq * block_size are not followed: NVB200_STATUS_BAD_SLOT is set in *status (nullable). */
typedef struct nvb200_paged_decode_args {
  void *out;
  const void *q;
  int64_t q_batch_stride;
  int64_t q_token_stride;
  int64_t q_head_stride;
  const void *k_cache;
  const void *v_cache;
  int64_t cache_block_stride;
  int64_t cache_token_stride;
  int64_t cache_head_stride;
  int64_t num_blocks;
  const int32_t *block_table;
  int64_t block_table_stride;
  const int32_t *seqlens;
  int32_t batch;
  int32_t queries_per_seq;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t block_size;
  int32_t max_blocks_per_seq;
  int32_t causal;
  int32_t num_splits;
  int32_t dtype;
  float softmax_scale;
  int32_t *status;
} nvb200_paged_decode_args;

NVB200_API int nvb200_paged_decode_attention(const nvb200_paged_decode_args *args, nvb200_stream_t stream);

/* The split count nvb200_paged_decode_attention uses for these sizes (num_splits 0 = its automatic choice). */
NVB200_API int nvb200_paged_decode_splits(int32_t batch, int32_t num_kv_heads, int32_t max_blocks_per_seq,
                                          int32_t block_size, int32_t num_splits);

/* The same attention (same arguments, same results within rounding) with the work split evenly over every SM: a
 * persistent grid of as many CTAs as are resident at once, each taking an equal share of all (sequence, KV head,
 * 16-key tile) units of the batch, so that SMs stay equally loaded whatever the number of (sequence, head) pairs.
 * A pair split between CTAs is merged by the last of them to finish, through the workspace. num_splits is ignored.
 * Replaces: the same flash_attn_with_kvcache call of nanovllm/layers/attention.py:84-91.
 *   workspace: device memory of at least nvb200_paged_decode_workspace_size(args) bytes, 256-byte aligned, zero-filled
 *     before its first use; each call leaves its counters at zero again, so it is zeroed once, not per call. Calls
 *     that may run at the same time (different streams) need separate workspaces.
 * Returns NVB200_ERR_ARG for a missing or short workspace, NVB200_ERR_UNSUPPORTED where the plain entry point does
 * and when batch * num_kv_heads * (max_blocks_per_seq * block_size / 16) reaches 2^31. */
NVB200_API int64_t nvb200_paged_decode_workspace_size(const nvb200_paged_decode_args *args);
NVB200_API int nvb200_paged_decode_attention_streamk(const nvb200_paged_decode_args *args, void *workspace,
                                                     int64_t workspace_bytes, nvb200_stream_t stream);

/* The stream-K attention above for callers that cannot allocate device memory when they call: an engine that has
 * already handed nearly all free HBM to its KV cache (as nano-vllm does at start-up), a decode loop that must not
 * risk cudaMalloc/cudaFree synchronising the device, or a host plugin interface that passes a kernel only its input
 * and output pointers. It allocates nothing and takes no workspace: its scratch is a fixed array of
 * NVB200_DECODE_NOALLOC_SCRATCH_BYTES (4 MiB) in the library's own device memory, which every GPU that loads the
 * library holds until the process exits.
 * No counterpart in the reference: an addition of this library.
 *   - The first call on a device looks up the array's device address (cudaGetSymbolAddress, with that device
 *     current); make that first call before any stream capture.
 *   - Each call clears the array's counters on `stream` (cudaMemsetAsync) before its kernel, since the array keeps
 *     what the previous call left.
 *   - Every call on a device shares the one array: calls that may overlap on the GPU (different streams without
 *     ordering between them) race and give wrong results. Order them on one stream.
 *   - Returns NVB200_ERR_UNSUPPORTED when batch * num_kv_heads exceeds NVB200_DECODE_NOALLOC_MAX_PAIRS (16384), and
 *     otherwise where nvb200_paged_decode_attention_streamk does. With 16 query rows per KV head it runs 244 CTAs
 *     (the array's limit) rather than one per resident slot. */
#define NVB200_DECODE_NOALLOC_SCRATCH_BYTES (4 << 20)
#define NVB200_DECODE_NOALLOC_MAX_PAIRS 16384
NVB200_API int nvb200_paged_decode_attention_noalloc(const nvb200_paged_decode_args *args, nvb200_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* NVB200_H */
