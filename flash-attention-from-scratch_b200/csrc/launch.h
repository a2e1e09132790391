// Host-side launchers of the kernels, called by the C ABI in api.cu. Each
// returns cudaSuccess or the launch error; argument checking is done by the
// caller.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

#include <cuda_runtime.h>

#include "common.cuh"

namespace fab {

struct LaunchCtx {
  cudaStream_t stream;
  DeviceStatus* status;          // device status word of the current device
  unsigned long long timeout_ns; // limit of every bounded wait
  int sm_count;                  // SMs of the current device
};

// tcgen05 FlashAttention forward; q, k, v, o fp16 [bh, n, d], d in {64, 128}.
cudaError_t launch_flash_tc(const void* q, const void* k, const void* v, void* o, int64_t bh,
                            int64_t n, int d, bool causal, float scale, const LaunchCtx& ctx,
                            std::string* err);

// CUDA-core tiled online-softmax attention, same layout.
cudaError_t launch_flash_simt(const void* q, const void* k, const void* v, void* o, int64_t bh,
                              int64_t n, int d, bool causal, float scale, const LaunchCtx& ctx);

// Three-kernel attention with fp32 scores in `scores` ([bh, n, n]).
cudaError_t launch_naive(const void* q, const void* k, const void* v, void* o, float* scores,
                         int64_t bh, int64_t n, int d, bool causal, float scale,
                         const LaunchCtx& ctx);

struct DecodeArgs {
  const void* q;          // fp16 [batch, hq, d]
  const void* k_cache;    // fp16 [num_blocks, hkv, bs, d]
  const void* v_cache;
  const int32_t* block_tables;  // [batch, max_blocks]
  const int32_t* context_lens;  // [batch]
  void* out;              // fp16 [batch, hq, d]           (final mode)
  float* o_final;         // fp32 [batch, hq, d] partials   (partials mode)
  float* m_final;         // fp32 [batch, hq]
  float* l_final;
  int64_t batch, hq, hkv, d, bs, num_blocks, max_blocks, max_ctx, partition;
  float scale;
  void* workspace;
  size_t workspace_bytes;
};

// Workspace layout of the decode path.
size_t decode_workspace_bytes(int64_t batch, int64_t hq, int64_t d, int64_t max_ctx,
                              int64_t partition);

cudaError_t launch_paged_decode(const DecodeArgs& a, bool partials_mode, const LaunchCtx& ctx);

cudaError_t launch_merge(const float* o_parts, const float* m_parts, const float* l_parts,
                         int64_t num_parts, int64_t rows, int64_t d, int64_t o_part_stride,
                         int64_t ml_part_stride, void* out, const LaunchCtx& ctx);

cudaError_t launch_selftest_wait(unsigned long long timeout_ns, const LaunchCtx& ctx);

// The prefill softmax's exponentials on n inputs: FMA-pipe polynomial, MUFU
// ex2.approx and exp2f (fp32 device arrays of n elements each).
cudaError_t launch_selftest_exp2(const float* x, float* y_poly, float* y_mufu, float* y_lib,
                                int64_t n, const LaunchCtx& ctx);

// Most ranks attn_exchange_merge_partials takes.
constexpr int kMaxPeers = 16;

// Context-parallel partials pushed to every peer over peer memory, then merged
// (csrc/exchange.cu). slots[q] / flags[q]: rank q's receive area for this call
// and its flag words, as device pointers valid on the current device.
cudaError_t launch_exchange_merge(float* const* slots, unsigned int* const* flags, int world,
                                  int rank, unsigned int epoch, int64_t rows, int d,
                                  int64_t slot_stride, void* out, const LaunchCtx& ctx);

// Size of the fixed device array that attn_paged_decode_noalloc uses as its
// split-K scratch (32 MiB per device that loads the library).
constexpr size_t kDecodeStaticScratchBytes = size_t(32) << 20;

// paged_decode (final fp16 output) with the scratch in that fixed array; the
// first call on a device looks up the array's device address. Fails with *err
// set when the problem needs more scratch than the array holds.
cudaError_t paged_decode_static_scratch(DecodeArgs a, const LaunchCtx& ctx, std::string* err);

}  // namespace fab
