// Attention on the CUDA cores: the two non-tensor-core prefill entry points
// the reference exposes next to its tensor-core kernel.
//
//  * flash_simt: tiled online-softmax attention in fp32 (the reference's
//    flash_simt_kernel, attnkernels/csrc/flash_simt.cu:46-187, computes the same
//    thing). A CTA of 4 warps owns 16 query rows; each warp owns 4 rows. Key and
//    value tiles of 32 rows are staged in shared memory as fp32; lane j scores
//    key j of the tile, the row max / sum are warp shuffles, and for P V each
//    lane owns D / 32 output columns.
//  * naive: the textbook three kernels of attnkernels/csrc/naive_attn.cu:18-61,
//    S = scale q k^T (fp32, to DRAM), a row softmax in place, O = P V.
//
// Both work in base 2 (scores pre-multiplied by scale * log2 e) and use the
// top-left causal mask (key > query masked).
#include "common.cuh"
#include "launch.h"

namespace fab {
namespace {

template <int D>
__global__ void __launch_bounds__(128)
    flash_simt_kernel(const __half* __restrict__ q, const __half* __restrict__ k,
                      const __half* __restrict__ v, __half* __restrict__ o, int n,
                      float scale_log2, int causal) {
  constexpr int BR = 16, BC = 32, RPW = 4, DL = D / 32;
  __shared__ float qs[BR][D];
  __shared__ float ks[BC][D + 1];  // +1: lane j reads row j without bank conflicts
  __shared__ float vs[BC][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t base = static_cast<size_t>(blockIdx.y) * n * D;
  const int q0 = blockIdx.x * BR;
  for (int i = threadIdx.x; i < BR * D; i += 128) {
    const int r = i / D, c = i % D;
    qs[r][c] = (q0 + r < n) ? __half2float(q[base + static_cast<size_t>(q0 + r) * D + c]) * scale_log2
                            : 0.f;
  }
  float m[RPW], l[RPW], acc[RPW][DL];
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int e = 0; e < DL; ++e) acc[i][e] = 0.f;
  }
  const int kend = causal ? min(n, q0 + BR) : n;
  for (int k0 = 0; k0 < kend; k0 += BC) {
    __syncthreads();
    for (int i = threadIdx.x; i < BC * D; i += 128) {
      const int r = i / D, c = i % D;
      const bool in = k0 + r < n;
      ks[r][c] = in ? __half2float(k[base + static_cast<size_t>(k0 + r) * D + c]) : 0.f;
      vs[r][c] = in ? __half2float(v[base + static_cast<size_t>(k0 + r) * D + c]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const int r = warp * RPW + i;
      const int qr = q0 + r;
      const int key = k0 + lane;
      float s = 0.f;
#pragma unroll 8
      for (int c = 0; c < D; ++c) s = fmaf(qs[r][c], ks[lane][c], s);
      const bool valid = key < n && (!causal || key <= qr);
      s = valid ? s : -INFINITY;
      const float mn = fmaxf(m[i], warp_max(s));
      const float m_use = (mn == -INFINITY) ? 0.f : mn;
      const float alpha = fast_exp2(m[i] - m_use);
      const float p = fast_exp2(s - m_use);
      l[i] = l[i] * alpha + warp_sum(p);
      m[i] = mn;
#pragma unroll
      for (int e = 0; e < DL; ++e) acc[i][e] *= alpha;
#pragma unroll 4
      for (int j = 0; j < BC; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
#pragma unroll
        for (int e = 0; e < DL; ++e) acc[i][e] = fmaf(pj, vs[j][lane + 32 * e], acc[i][e]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int qr = q0 + warp * RPW + i;
    if (qr >= n) continue;
    const float inv = l[i] > 0.f ? 1.f / l[i] : 0.f;
#pragma unroll
    for (int e = 0; e < DL; ++e)
      o[base + static_cast<size_t>(qr) * D + lane + 32 * e] = __float2half(acc[i][e] * inv);
  }
}

// S[bh][i][j] = scale_log2 * q_i . k_j (-inf where masked). CTA: 8 queries x 32 keys.
template <int D>
__global__ void __launch_bounds__(256)
    naive_scores_kernel(const __half* __restrict__ q, const __half* __restrict__ k,
                        float* __restrict__ s, int n, float scale_log2, int causal) {
  __shared__ float qs[8][D];
  __shared__ float ks[32][D + 1];
  const size_t base = static_cast<size_t>(blockIdx.z) * n * D;
  const int j0 = blockIdx.x * 32, i0 = blockIdx.y * 8;
  const int tid = threadIdx.y * 32 + threadIdx.x;
  for (int t = tid; t < 8 * D; t += 256) {
    const int r = t / D, c = t % D;
    qs[r][c] = (i0 + r < n) ? __half2float(q[base + static_cast<size_t>(i0 + r) * D + c]) : 0.f;
  }
  for (int t = tid; t < 32 * D; t += 256) {
    const int r = t / D, c = t % D;
    ks[r][c] = (j0 + r < n) ? __half2float(k[base + static_cast<size_t>(j0 + r) * D + c]) : 0.f;
  }
  __syncthreads();
  const int i = i0 + threadIdx.y, j = j0 + threadIdx.x;
  if (i >= n || j >= n) return;
  float acc = 0.f;
#pragma unroll 8
  for (int c = 0; c < D; ++c) acc = fmaf(qs[threadIdx.y][c], ks[threadIdx.x][c], acc);
  s[(static_cast<size_t>(blockIdx.z) * n + i) * n + j] =
      (causal && j > i) ? -INFINITY : acc * scale_log2;
}

// In-place row softmax (base 2), one warp per row.
__global__ void __launch_bounds__(256) naive_softmax_kernel(float* __restrict__ s, long long rows,
                                                            int n) {
  const long long row = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float* r = s + row * n;
  float mx = -INFINITY;
  for (int j = lane; j < n; j += 32) mx = fmaxf(mx, r[j]);
  mx = warp_max(mx);
  float sum = 0.f;
  for (int j = lane; j < n; j += 32) sum += fast_exp2(r[j] - mx);
  const float inv = 1.f / warp_sum(sum);
  for (int j = lane; j < n; j += 32) r[j] = fast_exp2(r[j] - mx) * inv;
}

// O[bh][i][:] = P[bh][i][:] V[bh]; one CTA per (i, bh), one thread per column.
__global__ void naive_pv_kernel(const float* __restrict__ p, const __half* __restrict__ v,
                                __half* __restrict__ o, int n, int d, int causal) {
  const int i = blockIdx.x, col = threadIdx.x;
  const size_t bh = blockIdx.y;
  const float* prow = p + (bh * n + i) * n;
  const __half* vb = v + bh * n * d;
  const int jend = causal ? i + 1 : n;
  float acc = 0.f;
  for (int j = 0; j < jend; ++j) acc = fmaf(prow[j], __half2float(vb[static_cast<size_t>(j) * d + col]), acc);
  o[(bh * n + i) * d + col] = __float2half(acc);
}

}  // namespace

cudaError_t launch_flash_simt(const void* q, const void* k, const void* v, void* o, int64_t bh,
                              int64_t n, int d, bool causal, float scale, const LaunchCtx& ctx) {
  dim3 grid(static_cast<unsigned>((n + 15) / 16), static_cast<unsigned>(bh));
  const float sl2 = scale * kLog2e;
  auto qh = static_cast<const __half*>(q);
  auto kh = static_cast<const __half*>(k);
  auto vh = static_cast<const __half*>(v);
  auto oh = static_cast<__half*>(o);
  if (d == 64)
    flash_simt_kernel<64><<<grid, 128, 0, ctx.stream>>>(qh, kh, vh, oh, static_cast<int>(n), sl2, causal);
  else
    flash_simt_kernel<128><<<grid, 128, 0, ctx.stream>>>(qh, kh, vh, oh, static_cast<int>(n), sl2, causal);
  return cudaGetLastError();
}

cudaError_t launch_naive(const void* q, const void* k, const void* v, void* o, float* scores,
                         int64_t bh, int64_t n, int d, bool causal, float scale,
                         const LaunchCtx& ctx) {
  const float sl2 = scale * kLog2e;
  const int ni = static_cast<int>(n);
  auto qh = static_cast<const __half*>(q);
  auto kh = static_cast<const __half*>(k);
  dim3 sg(static_cast<unsigned>((n + 31) / 32), static_cast<unsigned>((n + 7) / 8),
          static_cast<unsigned>(bh));
  dim3 sb(32, 8);
  if (d == 64)
    naive_scores_kernel<64><<<sg, sb, 0, ctx.stream>>>(qh, kh, scores, ni, sl2, causal);
  else
    naive_scores_kernel<128><<<sg, sb, 0, ctx.stream>>>(qh, kh, scores, ni, sl2, causal);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const long long rows = bh * n;
  naive_softmax_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, ctx.stream>>>(scores, rows, ni);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  naive_pv_kernel<<<dim3(static_cast<unsigned>(n), static_cast<unsigned>(bh)), d, 0, ctx.stream>>>(
      scores, static_cast<const __half*>(v), static_cast<__half*>(o), ni, d, causal);
  return cudaGetLastError();
}

}  // namespace fab
