/*
 * attn_b200.h - C ABI of the B200 (sm_100a) attention kernels.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as void*, NULL = legacy default stream) and enqueues work on that
 * stream without synchronising the host. Tensors are dense and row-major:
 *
 *   prefill q, k, v, o : fp16 [batch, heads, seq, head_dim]
 *   decode  q, out     : fp16 [batch, num_heads, head_dim]
 *   k_cache, v_cache   : fp16 [num_blocks, num_kv_heads, block_size, head_dim]
 *   block_tables       : int32 [batch, max_blocks_per_seq]
 *   context_lens       : int32 [batch]
 *
 * The caller owns every buffer, outputs included. Kernels that need scratch
 * memory take a `workspace` pointer whose minimum size a *_workspace_bytes()
 * query returns; no entry point allocates device memory. The library does
 * hold two fixed device arrays of its own: the 8-byte status word, and the
 * 32 MiB scratch array of attn_paged_decode_noalloc. Both are module globals,
 * so every GPU on which the library's kernels are loaded (the CUDA runtime
 * loads them on the first call that uses that device) holds them until the
 * process exits, whether or not the no-alloc entry point is ever called.
 *
 * Return value: ATTN_OK (0) or an attn_status_t error code; the message of
 * the last error on the calling thread is in attn_last_error(). Argument
 * errors are reported before anything is enqueued.
 *
 * The kernels run on the device that is current on the calling thread.
 */
#ifndef ATTN_B200_H_
#define ATTN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ATTN_ABI_VERSION 1

typedef enum {
  ATTN_OK = 0,
  ATTN_ERR_INVALID = 1,     /* bad argument (shape, pointer, alignment) */
  ATTN_ERR_UNSUPPORTED = 2, /* valid but not implemented (head_dim, group size) */
  ATTN_ERR_CUDA = 3,        /* a CUDA runtime call failed */
  ATTN_ERR_WORKSPACE = 4    /* workspace pointer missing or too small */
} attn_status_t;

/* Device-side status codes, read back with attn_device_status(). */
#define ATTN_DEVICE_OK 0u
#define ATTN_DEVICE_WAIT_TIMEOUT 1u /* an mbarrier wait exceeded its time limit */
#define ATTN_DEVICE_BAD_BLOCK 2u    /* a block-table entry outside [0, num_blocks); block 0 was read */

/* ABI version of the loaded library (ATTN_ABI_VERSION). */
int attn_abi_version(void);

/* Message of the last error returned on this thread ("" if none). */
const char* attn_last_error(void);

/* ------------------------------------------------------------------ prefill */

/*
 * FlashAttention forward on the 5th-generation tensor cores (tcgen05 MMAs with
 * TMEM accumulators, TMA-staged tiles, online softmax, causal tile skipping).
 * o = softmax(scale * q k^T [+ top-left causal mask]) v, fp32 accumulation,
 * P rounded to fp16 for the second product, fp16 output.
 * head_dim must be 64 or 128; q, k, v, o 16-byte aligned.
 *
 * Replaces the reference binding `flash_wmma(q, k, v, causal, scale, block_n)`
 * (attnkernels/csrc/ext.cpp:7-8, implemented at attnkernels/csrc/flash_wmma.cu:241-257).
 * block_n must be 32 or 64 as in the reference; both select the same kernel,
 * whose key tile is 128 rows.
 */
int attn_flash_fwd(const void* q, const void* k, const void* v, void* o, int64_t batch,
                   int64_t heads, int64_t seq, int64_t head_dim, int causal, float scale,
                   int64_t block_n, void* stream);

/*
 * Tiled online-softmax attention on the CUDA cores (fp32 arithmetic).
 * Replaces the reference binding `flash_simt(q, k, v, causal, scale)`
 * (attnkernels/csrc/ext.cpp:5-6, implemented at attnkernels/csrc/flash_simt.cu:209-221).
 */
int attn_flash_simt_fwd(const void* q, const void* k, const void* v, void* o, int64_t batch,
                        int64_t heads, int64_t seq, int64_t head_dim, int causal, float scale,
                        void* stream);

/* Bytes of workspace attn_naive_fwd needs: the fp32 [batch, heads, seq, seq] scores. */
size_t attn_naive_workspace_bytes(int64_t batch, int64_t heads, int64_t seq);

/*
 * Textbook attention: S = scale q k^T to DRAM, row softmax in place, O = P v.
 * Replaces the reference binding `naive_attention(q, k, v, causal, scale)`
 * (attnkernels/csrc/ext.cpp:3-4, implemented at attnkernels/csrc/naive_attn.cu:65-86).
 */
int attn_naive_fwd(const void* q, const void* k, const void* v, void* o, int64_t batch,
                   int64_t heads, int64_t seq, int64_t head_dim, int causal, float scale,
                   void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------- decode */

/*
 * Bytes of workspace attn_paged_decode / attn_paged_decode_partials need for
 * split-K partials (fp32 o, m, l per (sequence, query head, part)) and the
 * work counters: parts = k * ceil(max_context_len / partition), where k = 4 or 2
 * while batch * num_heads * parts stays within 8192 rows (and partition / k >= 64
 * tokens), else 1. Calls with that few partial rows may cut each partition into
 * k sub-partitions so that more warps share a short decode; the output differs
 * only by rounding.
 */
size_t attn_paged_decode_workspace_bytes(int64_t batch, int64_t num_heads, int64_t head_dim,
                                         int64_t max_context_len, int64_t partition);

/*
 * Decode attention of one query token per sequence over a paged KV cache,
 * split-K over context partitions of `partition` tokens (a positive multiple
 * of 256), merged by a log-sum-exp reduce kernel. Grouped-query attention:
 * num_heads / num_kv_heads in {1, 2, 4, 8}; head_dim 64 or 128.
 * Tokens past ceil(max_context_len / partition) * partition are not read, so
 * max_context_len must be >= max(context_lens). A sequence with context length 0
 * gets a zero output row.
 *
 * Replaces the reference binding `paged_decode(q, kc, vc, bt, ctx, max_ctx, scale,
 * partition)` (attnkernels/csrc/ext.cpp:9-10, implemented at
 * attnkernels/csrc/paged_decode.cu:256-277).
 */
int attn_paged_decode(const void* q, const void* k_cache, const void* v_cache,
                      const int32_t* block_tables, const int32_t* context_lens, void* out,
                      int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                      int64_t block_size, int64_t num_blocks, int64_t max_blocks_per_seq,
                      int64_t max_context_len, float scale, int64_t partition, void* workspace,
                      size_t workspace_bytes, void* stream);

/*
 * Same computation as attn_paged_decode, but instead of the fp16 output it
 * writes the un-merged softmax state of each (sequence, query head) row over
 * the context this cache holds: o_part fp32 [batch, num_heads, head_dim]
 * (normalised by l), m_part and l_part fp32 [batch, num_heads] (running max in
 * log2 units of scale * q.k, and the sum of 2^(s - m)). Rows with no context
 * get m = -inf, l = 0, o = 0. Used when a sequence's context is split across
 * GPUs; attn_merge_partials combines the pieces.
 *
 * No counterpart in the reference binding (the reference is single-GPU); it
 * exposes the split state that paged_decode_kernel writes at
 * attnkernels/csrc/paged_decode.cu:182-192.
 */
int attn_paged_decode_partials(const void* q, const void* k_cache, const void* v_cache,
                               const int32_t* block_tables, const int32_t* context_lens,
                               float* o_part, float* m_part, float* l_part, int64_t batch,
                               int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                               int64_t block_size, int64_t num_blocks,
                               int64_t max_blocks_per_seq, int64_t max_context_len, float scale,
                               int64_t partition, void* workspace, size_t workspace_bytes,
                               void* stream);

/*
 * Merge num_parts softmax partials per row into fp16 rows:
 *   M = max_p m_p,  w_p = l_p 2^(m_p - M),  out = sum_p w_p o_p / sum_p w_p.
 * Part p of row r is at o_parts[p * o_part_stride + r * head_dim + d] and
 * m_parts/l_parts[p * ml_part_stride + r]. Rows whose parts all have l = 0
 * get zeros. The same merge as the reference's paged_reduce_kernel
 * (attnkernels/csrc/paged_decode.cu:196-216), applied across GPUs.
 * The kernel is launched as a programmatic dependent of the previous kernel on
 * `stream`: it may start while that kernel runs, and reads no partial before it
 * has completed (the same holds for the merge inside attn_paged_decode and for
 * attn_exchange_merge_partials).
 */
int attn_merge_partials(const float* o_parts, const float* m_parts, const float* l_parts,
                        int64_t num_parts, int64_t rows, int64_t head_dim, int64_t o_part_stride,
                        int64_t ml_part_stride, void* out, void* stream);

/*
 * Context-parallel decode across GPUs, the exchange and the merge in one
 * kernel: pushes this rank's softmax partials to every peer over peer memory
 * (NVLink stores), signals each peer, waits (time-limited) for every peer's
 * partials, and merges them into fp16 rows (the merge of attn_merge_partials).
 *
 *   slots[q]   rank q's receive area for this call, a device pointer valid on
 *              the current device (peer memory, e.g. torch symmetric memory):
 *              `world` slots, `slot_stride` floats apart, each holding
 *              o [rows][head_dim], m [rows], l [rows] fp32. Before the call,
 *              this rank's own partials must be in slot `rank` of its own area
 *              (attn_paged_decode_partials writing there).
 *   flags[q]   rank q's flag words, uint32 [world][ceil(rows / 8)], zeroed once
 *              before the first call.
 *   epoch      1 on the first call, +1 on every call (the same on all ranks);
 *              consecutive calls must alternate between two receive areas.
 *   out        fp16 [rows][head_dim] on this rank.
 * world <= 16; every rank calls with the same world, rows, head_dim, slot_stride
 * and epoch. A peer that does not arrive within the wait limit leaves blocks of
 * `out` unwritten and attn_device_status() reports ATTN_DEVICE_WAIT_TIMEOUT.
 *
 * No counterpart in the reference (single-GPU); it replaces the NCCL
 * all-gather + attn_merge_partials pair of the context-parallel decode.
 */
int attn_exchange_merge_partials(float* const* slots, uint32_t* const* flags, int world, int rank,
                                 uint32_t epoch, int64_t rows, int64_t head_dim,
                                 int64_t slot_stride, void* out, void* stream);

/*
 * attn_paged_decode without a workspace argument, for callers that cannot
 * allocate device memory where they run decode: a plugin inside a serving
 * framework that owns the whole device-memory pool and gives its plugins no
 * allocator, or a latency-critical loop in which cudaMalloc / cudaFree (which
 * can synchronise the device) are not allowed. It calls no allocating routine.
 * Its split-K scratch is a fixed 32 MiB (33554432-byte) array inside the
 * library, which every GPU that loads the library holds until the process
 * exits. Problems whose scratch, attn_paged_decode_workspace_bytes(batch,
 * num_heads, head_dim, max_context_len, partition), exceeds 32 MiB are rejected
 * with ATTN_ERR_WORKSPACE and a message; a larger partition shrinks the need.
 * The first call on a device looks up the array's device address, so make it
 * before any stream capture. All calls on a device share the array: calls that
 * overlap on the GPU (two streams at once) race on it. Same arguments,
 * checks and result as attn_paged_decode otherwise.
 *
 * No counterpart in the reference, whose paged_decode always allocates its
 * scratch from the caching allocator.
 */
int attn_paged_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                              const int32_t* block_tables, const int32_t* context_lens, void* out,
                              int64_t batch, int64_t num_heads, int64_t num_kv_heads,
                              int64_t head_dim, int64_t block_size, int64_t num_blocks,
                              int64_t max_blocks_per_seq, int64_t max_context_len, float scale,
                              int64_t partition, void* stream);

/* ------------------------------------------------------------ device status */

/*
 * Read and clear the device status word of the current device (synchronises
 * the device). *code is ATTN_DEVICE_OK, ATTN_DEVICE_WAIT_TIMEOUT or
 * ATTN_DEVICE_BAD_BLOCK (first failure wins); *site
 * names the wait that gave up (kernel-specific number). A kernel whose wait
 * times out stops early, releases its tensor memory and leaves its output
 * incomplete; the CUDA context stays usable.
 */
int attn_device_status(uint32_t* code, uint32_t* site);

/*
 * Launch one CTA that waits on an mbarrier nothing ever arrives on, with the
 * same bounded wait the production kernels use and the given limit in
 * nanoseconds. It exercises the timeout path: afterwards attn_device_status()
 * reports ATTN_DEVICE_WAIT_TIMEOUT. No counterpart in the reference.
 */
int attn_selftest_wait_timeout(uint64_t timeout_ns, void* stream);

/*
 * Evaluate the exponentials of the prefill kernel's softmax on n fp32 inputs
 * (device arrays of n elements): y_poly = the FMA-pipe 2^x (range reduction plus
 * a degree-3 minimax polynomial, relative error <= 7.5e-5 for x in
 * [-125.99, 127); inputs below -126 and -inf give a value below 2^-125),
 * y_mufu = ex2.approx.ftz.f32, y_lib = exp2f. For the tests; no counterpart in
 * the reference, whose kernels call exp2f.
 */
int attn_selftest_exp2(const float* x, float* y_poly, float* y_mufu, float* y_lib, int64_t n,
                       void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ATTN_B200_H_ */
