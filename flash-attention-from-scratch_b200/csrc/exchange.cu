// Exchange of context-parallel decode partials over NVLink peer memory, fused
// with their merge: one kernel per rank replaces the all-gather collective and
// the merge launch of the context-parallel decode.
//
// Every rank holds a receive area in memory all ranks can address (peer
// pointers, e.g. from torch symmetric memory): `world` slots of the softmax
// state (o [rows][D], m [rows], l [rows], fp32; `slot_stride` floats apart),
// and a flag word per (source rank, block of rows). A rank's decode writes its
// own partials into its own slot. This kernel then, for each block of 8 rows:
//   1. pushes the block's rows of its own slot into the same slot of every
//      other rank (plain stores to peer memory over NVLink),
//   2. fences at system scope and stores `epoch` into each peer's flag of
//      (this rank, this block) with release semantics,
//   3. waits, with a time limit, until every peer's flag for this block in its
//      own memory has reached `epoch` (acquire), and
//   4. merges the `world` states of each row (M = max m, w = l 2^(m - M),
//      out = sum w o / sum w, the merge of the reference's paged_reduce_kernel,
//      attnkernels/csrc/paged_decode.cu:196-216) into fp16.
// Flags only grow (the host passes a new epoch per call), so nothing is reset.
// A rank can be at most one call ahead of another: it cannot finish call t
// without every peer's data of call t, which each peer pushes only after its
// merge of call t - 1. Callers therefore alternate two receive areas by call
// parity, and a wait accepts any flag value >= epoch.
//
// All blocks of the grid must be resident at once on every rank (a block waits
// for the same block on the other ranks); the grid is one block per 8 rows,
// capped at the SM count, blocks looping over row blocks in the same order on
// every rank.
#include <algorithm>

#include "common.cuh"
#include "launch.h"

namespace fab {
namespace {

enum : unsigned int { kSiteExchangeWait = 401 };

struct XParams {
  float* slots[kMaxPeers];         // rank q's receive area for this call (world slots)
  unsigned int* flags[kMaxPeers];  // rank q's flags: [world][num_blocks]
  __half* out;                     // fp16 [rows, D]
  DeviceStatus* status;
  unsigned long long timeout_ns;
  long long slot_stride;  // floats between slots
  int rows, world, rank, num_blocks;
  unsigned int epoch;
};

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One warp per row, lane owns D / 32 columns; 8 rows per block.
template <int D>
__global__ void __launch_bounds__(256) exchange_merge_kernel(const XParams p) {
  constexpr int DV = D / 32;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  __shared__ int failed;
  // Launched as a programmatic dependent of the kernel that writes this rank's
  // partials: nothing is read or written before that kernel has completed.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const long long o_floats = static_cast<long long>(p.rows) * D;
  const float* mine = p.slots[p.rank] + p.rank * p.slot_stride;  // own slot in own area
  for (int blk = blockIdx.x; blk < p.num_blocks; blk += gridDim.x) {
    const int row = blk * 8 + warp;
    const bool live = row < p.rows;
    // 1. Push this rank's rows of the block to every peer.
    if (live) {
      const float* src = mine + static_cast<long long>(row) * D + lane * DV;
      float v[DV];
#pragma unroll
      for (int j = 0; j < DV; ++j) v[j] = src[j];
      const float m = mine[o_floats + row];
      const float l = mine[o_floats + p.rows + row];
      for (int q = 0; q < p.world; ++q) {
        if (q == p.rank) continue;
        float* dst = p.slots[q] + p.rank * p.slot_stride;
        float* drow = dst + static_cast<long long>(row) * D + lane * DV;
        if constexpr (DV == 4) {
          *reinterpret_cast<float4*>(drow) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
          *reinterpret_cast<float2*>(drow) = make_float2(v[0], v[1]);
        }
        if (lane == 0) {
          dst[o_floats + row] = m;
          dst[o_floats + p.rows + row] = l;
        }
      }
      __threadfence_system();  // this thread's peer stores before the flags below
    }
    // 2. Publish the block to every peer.
    __syncthreads();
    if (threadIdx.x == 0) {
      failed = 0;
      __threadfence_system();
      for (int q = 0; q < p.world; ++q)
        if (q != p.rank) st_release_sys(p.flags[q] + p.rank * p.num_blocks + blk, p.epoch);
    }
    // 3. Wait for every peer's rows of the block (lane q of warp 0 polls rank q).
    if (warp == 0 && lane < p.world && lane != p.rank) {
      const unsigned int* f = p.flags[p.rank] + lane * p.num_blocks + blk;
      if (static_cast<int>(ld_acquire_sys(f) - p.epoch) < 0) {
        const uint64_t t0 = globaltimer_ns();
        for (uint32_t n = 1;; ++n) {
          if (static_cast<int>(ld_acquire_sys(f) - p.epoch) >= 0) break;
          if ((n & 63u) == 0u && globaltimer_ns() - t0 > p.timeout_ns) {
            report_status(p.status, 1u /* ATTN_DEVICE_WAIT_TIMEOUT */, kSiteExchangeWait);
            failed = 1;
            break;
          }
        }
      }
    }
    __syncthreads();
    if (failed) return;  // the output block stays unwritten; the status word says why
    // 4. Merge the world states of each row.
    if (live) {
      const float* area = p.slots[p.rank];
      float mx = -INFINITY;
      for (int q = 0; q < p.world; ++q) mx = fmaxf(mx, area[q * p.slot_stride + o_floats + row]);
      float num[DV];
#pragma unroll
      for (int j = 0; j < DV; ++j) num[j] = 0.f;
      float den = 0.f;
      if (mx != -INFINITY) {
        for (int q = 0; q < p.world; ++q) {
          const float* s = area + q * p.slot_stride;
          const float w = s[o_floats + p.rows + row] * fast_exp2(s[o_floats + row] - mx);
          den += w;
          const float* o = s + static_cast<long long>(row) * D + lane * DV;
#pragma unroll
          for (int j = 0; j < DV; ++j) num[j] = fmaf(w, o[j], num[j]);
        }
      }
      const float inv = den > 0.f ? 1.f / den : 0.f;
      __half* dst = p.out + static_cast<long long>(row) * D + lane * DV;
      if constexpr (DV == 4) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(pack_half2(num[0] * inv, num[1] * inv),
                                                    pack_half2(num[2] * inv, num[3] * inv));
      } else {
        *reinterpret_cast<uint32_t*>(dst) = pack_half2(num[0] * inv, num[1] * inv);
      }
    }
    __syncthreads();  // `failed` is rewritten by the next block's publisher
  }
}

}  // namespace

cudaError_t launch_exchange_merge(float* const* slots, unsigned int* const* flags, int world,
                                  int rank, unsigned int epoch, int64_t rows, int d,
                                  int64_t slot_stride, void* out, const LaunchCtx& ctx) {
  XParams p{};
  for (int q = 0; q < world; ++q) {
    p.slots[q] = slots[q];
    p.flags[q] = flags[q];
  }
  p.out = static_cast<__half*>(out);
  p.status = ctx.status;
  p.timeout_ns = ctx.timeout_ns;
  p.slot_stride = slot_stride;
  p.rows = static_cast<int>(rows);
  p.world = world;
  p.rank = rank;
  p.num_blocks = static_cast<int>((rows + 7) / 8);
  p.epoch = epoch;
  const int grid = std::max(1, std::min(p.num_blocks, ctx.sm_count));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = ctx.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return d == 64 ? cudaLaunchKernelEx(&cfg, exchange_merge_kernel<64>, p)
                 : cudaLaunchKernelEx(&cfg, exchange_merge_kernel<128>, p);
}

}  // namespace fab
