// Paged-KV decode attention with split-K ("flash-decoding") and the merge of
// the split partials.
//
// Semantics follow the reference's paged_decode_kernel / paged_reduce_kernel
// (attnkernels/csrc/paged_decode.cu:39-216): sequence b has context_lens[b]
// tokens; token t lives in physical block block_tables[b][t / bs] at row
// t % bs of cache [num_blocks, H_kv, bs, D]; query head h reads kv head
// h / G; the context is cut into partitions of `partition` tokens; each
// partition yields (o = acc / l, m, l) with scores in log2 units
// (q pre-multiplied by scale * log2 e); the merge is
//     M = max_s m_s,  w_s = l_s 2^(m_s - M),  O = sum_s w_s o_s / sum_s w_s.
//
// The B200 design is different from the reference's one-CTA-per-split grid:
//   * A persistent grid of one CTA per SM, 8 warps per CTA (16 at head_dim
//     64). Each warp is an
//     independent pipeline that owns whole work units (sequence, kv head,
//     split) and fetches the next unit from an atomic counter, so no CTA-wide
//     barrier is ever taken inside the main loop and the short final splits of
//     ragged sequences balance across warps.
//   * K, V and q move by 1-D bulk copies (cp.async.bulk, the TMA engine) of
//     whole page runs into a per-warp ring of 16-token stages signalled by
//     mbarriers: a page of one head is bs * D * 2 contiguous bytes (4 KB at
//     bs = 16, D = 128), so every copy is a long contiguous DRAM burst and
//     128 KB of K and V per SM is in flight at D = 128. The producer runs
//     `STAGES` stages ahead of the consumer, across unit boundaries.
//   * G = 1 (one query row per kv head) needs no tensor cores: scores with 8
//     lanes per token and 16-byte shared-memory loads, an online softmax per
//     16-token stage, and P V with each lane owning D / 32 output columns.
//   * G > 1 (G = H / H_kv query heads share every K/V byte) does G times the
//     arithmetic per byte, which the CUDA cores cannot hide under the stream:
//     the G heads become the rows of a 16-row mma.sync tile (m16n8k16, rows
//     past G zero), K and V fragments come from shared memory by ldmatrix
//     (transposed for V), and each lane runs the softmax of its head's row on
//     the accumulator fragment it holds. K and V arrive one token row per
//     bulk copy, each row 16 bytes past a multiple of 128, so the 8 rows an
//     ldmatrix reads hit 8 different bank groups.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "launch.h"

namespace fab {
namespace {

constexpr int kTok = 16;           // tokens per pipeline stage
constexpr int kMinLaunchBatch = 2048;  // sequences any configuration takes per launch

enum : unsigned int { kSiteDecodeWait = 201, kSiteDecodeDrain = 202, kSiteBadBlock = 203 };

// Token rows per bulk copy in the G > 1 ring. Measured on B200 at 64 sequences
// x 8192 tokens, 32 query over 8 kv heads, d 128 (us per launch): 1 row 467,
// 2 rows 375, 4 rows 352, 8 rows 422, 16 rows 700. Fewer, larger copies issue
// faster; more rows per group put more of an ldmatrix's 8 rows in one bank group.
// Warps per CTA at head_dim 64. A 16-token stage there is 4 KB of K and V, and a
// warp's stage is latency-bound (about 0.2 instructions per cycle per warp), so
// twice the warps of head_dim 128 keep HBM busy: 64 sequences x 8192 tokens, 8
// kv heads, B200, 8 -> 16 warps: G = 1 276 -> 202 us, G = 4 297 -> 213 us.
#ifndef FAB_DEC_W64
#define FAB_DEC_W64 16
#endif
#ifndef FAB_DEC_CP
#define FAB_DEC_CP 4
#endif

// Eight warps per CTA at head_dim 128, 16 at 64. G = 1 streams K and V with
// CUDA-core arithmetic. G > 1 (query heads sharing a kv head) puts the scores and P V on
// the tensor cores (mma.sync m16n8k16, fp16 in, fp32 accumulate, one 16-row
// tile with the G heads as rows). Its ring stores a stage's 16 token rows in
// groups of CP consecutive rows (one bulk copy each), the groups GS = CP ROW + 16
// bytes apart: token t sits at (t / CP) GS + (t % CP) ROW, so rows of tokens in
// different groups start in different 16-byte bank groups.
template <int D, int G>
struct DecCfg {
  static constexpr bool MMA = G > 1;
  static constexpr int W = D == 64 ? FAB_DEC_W64 : 8;
  static constexpr int THREADS = W * 32;
  static constexpr int MAXB = 2048;                        // sequences per launch
  static constexpr int ROW = D * 2;                        // bytes of one token of one head
  static constexpr int CP = MMA ? FAB_DEC_CP : kTok;       // token rows per copy group
  static constexpr int NGRP = kTok / CP;                   // copy groups per stage and tensor
  static constexpr int GS = CP * ROW + (MMA ? 16 : 0);     // ring bytes per copy group
  static constexpr int KV = NGRP * GS;                     // K (or V) bytes of one stage
  static constexpr int QB = (G * D * 2 + 15) / 16 * 16;    // q bytes of one unit
  static constexpr int STAGE = 2 * KV + QB;
  static constexpr int BUDGET = 196 * 1024 / W;            // ring bytes per warp
  static constexpr int STAGES = std::max(2, std::min(6, BUDGET / STAGE));
  static constexpr int RING = STAGES * STAGE;
  static constexpr int BAR_OFF = W * RING;
  // The int4 stage descriptors need 16-byte alignment (an odd W * STAGES would
  // leave the barriers' end 8 bytes past it).
  static constexpr int META_OFF = (BAR_OFF + W * STAGES * 8 + 15) / 16 * 16;
  static constexpr int PREFIX_OFF = META_OFF + W * STAGES * 16;
  static constexpr int CTX_OFF = PREFIX_OFF + (MAXB + 1) * 4;
  static constexpr int SMEM = (CTX_OFF + MAXB * 4 + 15) / 16 * 16 + 16;  // + the abort flag
  static constexpr int E = D / 8;    // K elements per lane in the score phase (G = 1)
  static constexpr int DV = D / 32;  // output columns per lane (G = 1)
  static_assert(STAGES >= 2, "ring needs two stages");
  static_assert(STAGE % 16 == 0 && BAR_OFF % 16 == 0 && META_OFF % 16 == 0,
                "bulk copy, ldmatrix and int4 alignment of the shared-memory layout");
  static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
  static_assert(!MMA || G <= 8, "one 16-row MMA tile holds the heads");
};

struct DecParams {
  const __half* q;
  const __half* kc;
  const __half* vc;
  const int* bt;
  const int* ctx;
  __half* out;     // fp16 [batch, hq, D]: rows of sequences with one split (direct_out)
  float* o_part;   // fp32 [batch * hq, num_splits, D]
  float* m_part;   // fp32 [batch * hq, num_splits]
  float* l_part;
  unsigned int* counter;  // work counter, zero at launch
  DeviceStatus* status;
  unsigned long long timeout_ns;
  long long block_stride;  // elements between physical blocks (hkv * bs * D)
  int batch, hq, hkv, bs, max_blocks, partition, num_splits;
  int num_blocks;  // physical blocks in the cache: block ids outside [0, num_blocks) are rejected
  int direct_out;  // 1: a sequence with a single split writes its fp16 row directly
  float scale_log2;
};


// ldmatrix of four 8x8 fp16 matrices; lanes 8 i .. 8 i + 7 give the row
// addresses of matrix i (16 bytes each, 16-byte aligned).
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// D[0:8, 0:8] += A[0:8, 0:16] B[0:16, 0:8] with mma.sync m16n8k16 (fp16 in,
// fp32 accumulate) whose rows 8..15 are zero: the lane passes its row-g
// fragments a0 (columns 2 t + {0, 1}) and a2 (columns 8 + 2 t + {0, 1}) and its
// row-g accumulators d0, d1; the instruction's rows 8..15 get zeros in and are
// dropped.
__device__ __forceinline__ void mma_16816_rows8(float& d0, float& d1, uint32_t a0, uint32_t a2,
                                                uint32_t b0, uint32_t b1) {
  asm volatile(
      "{\n\t.reg .f32 u0, u1;\n\t"
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, u0, u1}, "
      "{%2, %3, %4, %3}, {%5, %6}, {%0, %1, %7, %7};\n\t}"
      : "+f"(d0), "+f"(d1)
      : "r"(a0), "r"(0u), "r"(a2), "r"(b0), "r"(b1), "f"(0.f));
}

template <int D, int G>
__global__ void __launch_bounds__(DecCfg<D, G>::THREADS, 1) paged_decode_kernel(const DecParams p) {
  using C = DecCfg<D, G>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int grp = lane >> 3;  // token of a 4-token step in the score phase
  const int l8 = lane & 7;    // 16-byte column chunk of that token
  uint8_t* ring = smem + warp * C::RING;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF) + warp * C::STAGES;
  int4* meta = reinterpret_cast<int4*>(smem + C::META_OFF) + warp * C::STAGES;
  int* prefix = reinterpret_cast<int*>(smem + C::PREFIX_OFF);
  int* ctx_s = reinterpret_cast<int*>(smem + C::CTX_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::SMEM - 16);
  // The merge launch that follows may be scheduled now; it waits for this
  // launch's completion before it reads the partials.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // Context lengths and the prefix sums of the splits per sequence: active
  // (sequence, split) pairs are numbered densely, v in [0, prefix[batch]).
  for (int b = threadIdx.x; b < p.batch; b += C::THREADS) ctx_s[b] = max(p.ctx[b], 0);
  if (threadIdx.x < C::W * C::STAGES)
    mbar_init(reinterpret_cast<uint64_t*>(smem + C::BAR_OFF) + threadIdx.x, 1);
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {
    const int per = (p.batch + 31) / 32;
    const int b0 = lane * per;
    int sum = 0;
    for (int i = 0; i < per; ++i) {
      const int b = b0 + i;
      if (b < p.batch) sum += min((ctx_s[b] + p.partition - 1) / p.partition, p.num_splits);
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    int run = incl - sum;
    for (int i = 0; i < per; ++i) {
      const int b = b0 + i;
      if (b < p.batch) {
        prefix[b] = run;
        run += min((ctx_s[b] + p.partition - 1) / p.partition, p.num_splits);
      }
    }
    if (lane == 31) prefix[p.batch] = incl;
  }
  __syncthreads();
  // Without a merge pass, rows of empty sequences are written here (zeros).
  if (p.direct_out && p.num_splits == 1 && blockIdx.x == 0) {
    for (int b = warp; b < p.batch; b += C::W) {
      if (ctx_s[b] != 0) continue;
      for (int i = lane; i < p.hq * D / 2; i += 32)
        reinterpret_cast<uint32_t*>(p.out + static_cast<size_t>(b) * p.hq * D)[i] = 0u;
    }
  }
  const int total_units = prefix[p.batch] * p.hkv;

  // ---------------------------------------------------------- producer state
  int pu = -1, pb = 0, pkvh = 0, psplit = 0, pstart = 0, pend = 0, pst = 0, pnst = 0;
  int bt_base = 0, bt_reg = 0;
  unsigned int nxt = 0;  // next unit id (valid in lane 0), fetched one unit ahead
  unsigned int p_item = 0, c_item = 0;

  auto advance = [&]() {
    const int u = static_cast<int>(__shfl_sync(0xffffffffu, nxt, 0));
    if (u >= total_units) {
      pu = -1;
      return;
    }
    pu = u;
    const int v = u / p.hkv;
    pkvh = u - v * p.hkv;
    int lo = 0, hi = p.batch - 1;  // last sequence whose first pair is <= v
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (prefix[mid] <= v) lo = mid; else hi = mid - 1;
    }
    pb = lo;
    psplit = v - prefix[lo];
    pstart = psplit * p.partition;
    pend = min(ctx_s[pb], pstart + p.partition);
    pst = 0;
    pnst = (pend - pstart + kTok - 1) / kTok;
    bt_base = -(1 << 30);
    if (lane == 0) nxt = C::W * gridDim.x + atomicAdd(p.counter, 1u);
  };

  // Issue the copies of the producer's next stage into its ring slot.
  auto produce = [&]() {
    if (pu < 0) return;
    const unsigned int slot = p_item % C::STAGES;
    uint8_t* st = ring + slot * C::STAGE;
    uint64_t* bar = full + slot;
    const int t0 = pstart + pst * kTok;
    const int nt = min(kTok, pend - t0);
    const int rows_copied = C::MMA ? kTok : nt;
    if (lane == 0)
      mbar_arrive_expect_tx(bar, 2 * rows_copied * C::ROW + (pst == 0 ? G * D * 2 : 0));
    const int* btrow = p.bt + static_cast<size_t>(pb) * p.max_blocks;
    if constexpr (C::MMA) {
      // Lane r (and r + 16) looks up token row r of the stage (rows past a
      // partial stage's last token repeat it: the tensor-core P V reads all 16
      // rows, with P = 0 there, so a stage never holds another unit's data).
      // Lanes [0, NGRP) then copy the K groups, lanes [16, 16 + NGRP) the V
      // groups: one bulk copy when the group's rows are consecutive in one page,
      // else one per row. The stage spans at most 16 pages, inside one 32-entry
      // window of the block table.
      const int pg_first = t0 / p.bs, pg_last = (t0 + nt - 1) / p.bs;
      if (pg_last - bt_base >= 32 || pg_first < bt_base) {
        bt_base = pg_first;
        bt_reg = (pg_first + lane < p.max_blocks) ? btrow[pg_first + lane] : 0;
      }
      const int r = lane & 15;
      const int t = t0 + min(r, nt - 1);
      const int pg = t / p.bs;
      int page = __shfl_sync(0xffffffffu, bt_reg, pg - bt_base);
      if (page < 0 || page >= p.num_blocks) {  // never read outside the cache
        if (r < nt) report_status(p.status, 2u /* ATTN_DEVICE_BAD_BLOCK */, kSiteBadBlock);
        page = 0;
      }
      const long long eoff = static_cast<long long>(page) * p.block_stride +
                             (static_cast<long long>(pkvh) * p.bs + (t - pg * p.bs)) * D;
      const int gi = r < C::NGRP ? r : 0;
      long long eo[C::CP];
      bool whole = true;
#pragma unroll
      for (int i = 0; i < C::CP; ++i) {
        eo[i] = __shfl_sync(0xffffffffu, eoff, gi * C::CP + i);
        whole = whole && eo[i] == eo[0] + i * D;
      }
      __syncwarp();  // the expected bytes are set before any copy completes
      if (r < C::NGRP) {
        const __half* base = lane < 16 ? p.kc : p.vc;
        uint8_t* dst = st + (lane < 16 ? 0 : C::KV) + r * C::GS;
        if (whole) {
          bulk_g2s(dst, base + eo[0], C::CP * C::ROW, bar);
        } else {
#pragma unroll
          for (int i = 0; i < C::CP; ++i) bulk_g2s(dst + i * C::ROW, base + eo[i], C::ROW, bar);
        }
      }
    } else {
    for (int t = t0; t < t0 + nt;) {
      const int pg = t / p.bs;
      const int off = t - pg * p.bs;
      const int rows = min(p.bs - off, t0 + nt - t);
      if (pg - bt_base >= 32 || pg < bt_base) {  // next 32 block-table entries, one per lane
        bt_base = pg;
        bt_reg = (pg + lane < p.max_blocks) ? btrow[pg + lane] : 0;
      }
      int page = __shfl_sync(0xffffffffu, bt_reg, pg - bt_base);
      if (page < 0 || page >= p.num_blocks) {  // never read outside the cache
        if (lane == 0) report_status(p.status, 2u /* ATTN_DEVICE_BAD_BLOCK */, kSiteBadBlock);
        page = 0;
      }
      if (lane == 0) {
        const size_t eoff = static_cast<size_t>(page) * p.block_stride +
                            (static_cast<size_t>(pkvh) * p.bs + off) * D;
        const uint32_t dst = static_cast<uint32_t>(t - t0) * C::ROW;
        bulk_g2s(st + dst, p.kc + eoff, rows * C::ROW, bar);
        bulk_g2s(st + C::KV + dst, p.vc + eoff, rows * C::ROW, bar);
      }
      t += rows;
    }
    }
    if (lane == 0) {
      if (pst == 0)
        bulk_g2s(st + 2 * C::KV, p.q + (static_cast<size_t>(pb) * p.hq + pkvh * G) * D,
                 G * D * 2, bar);
      meta[slot] = make_int4(pb, pkvh, psplit,
                             nt | ((pst == 0) ? 32 : 0) | ((pst == pnst - 1) ? 64 : 0));
    }
    ++p_item;
    if (++pst == pnst) advance();
  };

  // ---------------------------------------------------------- consumer state
  // G = 1: q * scale * log2(e) as packed fp32 pairs, the 16 (or 8) elements this
  // lane multiplies in the score phase; running max and sum; output columns
  // [lane * DV, lane * DV + DV) as DV / 2 packed pairs, in two accumulator sets
  // (even / odd tokens) to halve the FMA chains.
  uint64_t qf[C::MMA ? 1 : G][C::E / 2];
  float m[G], l[G];
  constexpr int NACC = 2;
  uint64_t acc[C::MMA ? 1 : NACC][G][C::DV / 2];

  auto half2_pair = [](uint32_t h2) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h2));
    return f2_pack(f.x, f.y);
  };

  // G > 1: mma.sync m16n8k16 with the G query heads as the rows of one 16-row
  // tile (rows G..15 zero). Lane = (group g = lane / 4, t4 = lane % 4) holds, in
  // the fragment layouts of that instruction, row g: q as A fragments (a0, a2
  // per 16-element k-step; a1 = a3 = 0), the scores of tokens 2 t4, 2 t4 + 1
  // (+ 8) and the output columns 8 n + 2 t4, 8 n + 2 t4 + 1 of every 8-column
  // n-tile. Rows g >= G compute zeros and are not written.
  constexpr int KS = D / 16, NT = D / 8;
  const int g4 = lane >> 2, t4 = lane & 3;
  uint32_t qa[C::MMA ? KS : 1][2];
  float oc[C::MMA ? NT : 1][2];
  float m_r = -INFINITY, l_r = 0.f;  // row g's running max (log2 units) and sum

  // One stage of a unit with G > 1 query heads per kv head (st: the stage's
  // ring slot, nt: its tokens, md: its unit and flags).
  auto consume_mma = [&](const uint8_t* st, int nt, const int4 md) {
   if constexpr (C::MMA) {
    // Token columns: n-tile 0 holds the stage's even tokens, n-tile 1 the odd
    // ones (column j of tile n is token 2 j + n), so the 8 rows of every
    // ldmatrix spread over all 16 / CP copy groups (with CP = 4: two rows in
    // each, a 2-way bank conflict).
    // Scores S [heads x 16 tokens]: B = K rows read by ldmatrix, two k-steps per
    // x4 load.
    const uint32_t kst = smem_u32(st), vst = smem_u32(st + C::KV);
    auto row_off = [](int tok) { return (tok / C::CP) * C::GS + (tok % C::CP) * C::ROW; };
    float s[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < KS; ks += 2) {
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        uint32_t b[4];
        ldmatrix_x4(b, kst + row_off(2 * (lane & 7) + n) + (16 * ks + 8 * (lane >> 3)) * 2);
        mma_16816_rows8(s[n][0], s[n][1], qa[ks][0], qa[ks][1], b[0], b[1]);
        mma_16816_rows8(s[n][0], s[n][1], qa[ks + 1][0], qa[ks + 1][1], b[2], b[3]);
      }
    }
    // Online softmax of row g over the stage's tokens (the 4 lanes of a group
    // hold its 16 scores), in log2 units.
    float mx = -INFINITY;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int tok = 2 * (2 * t4 + c) + n;
        s[n][c] = tok < nt ? s[n][c] * p.scale_log2 : -INFINITY;
        mx = fmaxf(mx, s[n][c]);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(m_r, mx);
    const float alpha = fast_exp2(m_r - mn);
    float ps = 0.f;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        s[n][c] = fast_exp2(s[n][c] - mn);
        ps += s[n][c];
      }
    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    l_r = l_r * alpha + ps;
    m_r = mn;
    if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        oc[n][0] *= alpha;
        oc[n][1] *= alpha;
      }
    }
    // O += P V: A = P (fp16, from the score fragments: k slots 0-7 the even
    // tokens, 8-15 the odd ones), B = V with the same k order, n = columns, read
    // by transposing ldmatrix, two n-tiles per load.
    const uint32_t pa0 = pack_half2(s[0][0], s[0][1]);
    const uint32_t pa2 = pack_half2(s[1][0], s[1][1]);
#pragma unroll
    for (int n = 0; n < NT; n += 2) {
      uint32_t b[4];
      ldmatrix_x4_trans(b, vst + row_off(2 * (lane & 7) + ((lane >> 3) & 1)) +
                               (8 * n + 8 * (lane >> 4)) * 2);
      mma_16816_rows8(oc[n][0], oc[n][1], pa0, pa2, b[0], b[1]);
      mma_16816_rows8(oc[n + 1][0], oc[n + 1][1], pa0, pa2, b[2], b[3]);
    }
    if ((md.w & 64) && g4 < G) {
      const int b = md.x, kvh = md.y, split = md.z;
      const int ns = min((ctx_s[b] + p.partition - 1) / p.partition, p.num_splits);
      const float inv = 1.f / l_r;
      const size_t row = static_cast<size_t>(b) * p.hq + kvh * G + g4;
      if (p.direct_out && ns == 1) {
        uint32_t* dst = reinterpret_cast<uint32_t*>(p.out + row * D + 2 * t4);
#pragma unroll
        for (int n = 0; n < NT; ++n) dst[4 * n] = pack_half2(oc[n][0] * inv, oc[n][1] * inv);
      } else {
        const size_t pr = row * p.num_splits + split;
        float2* dst = reinterpret_cast<float2*>(p.o_part + pr * D + 2 * t4);
#pragma unroll
        for (int n = 0; n < NT; ++n) dst[4 * n] = make_float2(oc[n][0] * inv, oc[n][1] * inv);
        if (t4 == 0) {
          p.m_part[pr] = m_r;
          p.l_part[pr] = l_r;
        }
      }
    }
    __syncwarp();
   }
  };

  auto consume = [&]() -> bool {
    const unsigned int slot = c_item % C::STAGES;
    const uint32_t parity = (c_item / C::STAGES) & 1u;
    const bool ok = mbar_wait(full + slot, parity, abort_flag, p.status, kSiteDecodeWait,
                              p.timeout_ns);
    if (!__all_sync(0xffffffffu, ok)) return false;
    const int4 md = meta[slot];
    const uint8_t* st = ring + slot * C::STAGE;
    const int nt = md.w & 31;
    if constexpr (C::MMA) {
      if (md.w & 32) {
        // q of the unit as A fragments (rows = heads; rows >= G zero), fp16 as
        // stored; the scale is applied to the fp32 scores.
        const __half* qs = reinterpret_cast<const __half*>(st + 2 * C::KV);
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          const bool real = g4 < G;
          qa[ks][0] = real ? *reinterpret_cast<const uint32_t*>(qs + g4 * D + 16 * ks + 2 * t4) : 0u;
          qa[ks][1] =
              real ? *reinterpret_cast<const uint32_t*>(qs + g4 * D + 16 * ks + 8 + 2 * t4) : 0u;
        }
        m_r = -INFINITY;
        l_r = 0.f;
#pragma unroll
        for (int n = 0; n < NT; ++n) oc[n][0] = oc[n][1] = 0.f;
      }
      consume_mma(st, nt, md);
    } else {
    if (md.w & 32) {
      const __half* qs = reinterpret_cast<const __half*>(st + 2 * C::KV);
      const uint64_t sc = f2_pack(p.scale_log2, p.scale_log2);
#pragma unroll
      for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int e8 = 0; e8 < C::E / 8; ++e8) {
          const uint4 raw = *reinterpret_cast<const uint4*>(qs + g * D + e8 * 64 + l8 * 8);
          qf[g][e8 * 4 + 0] = f2_mul(half2_pair(raw.x), sc);
          qf[g][e8 * 4 + 1] = f2_mul(half2_pair(raw.y), sc);
          qf[g][e8 * 4 + 2] = f2_mul(half2_pair(raw.z), sc);
          qf[g][e8 * 4 + 3] = f2_mul(half2_pair(raw.w), sc);
        }
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int a = 0; a < NACC; ++a)
#pragma unroll
          for (int j = 0; j < C::DV / 2; ++j) acc[a][g][j] = f2_pack(0.f, 0.f);
      }
    }
    // Scores: token 4 * step + grp, 8 lanes per token, two FMA chains per head.
    float s[kTok / 4][G];
    const __half* kst = reinterpret_cast<const __half*>(st);
#pragma unroll
    for (int step = 0; step < kTok / 4; ++step) {
      const int t = step * 4 + grp;
      uint64_t kf[C::E / 2];
#pragma unroll
      for (int e8 = 0; e8 < C::E / 8; ++e8) {
        const uint4 raw = *reinterpret_cast<const uint4*>(kst + t * D + e8 * 64 + l8 * 8);
        kf[e8 * 4 + 0] = half2_pair(raw.x);
        kf[e8 * 4 + 1] = half2_pair(raw.y);
        kf[e8 * 4 + 2] = half2_pair(raw.z);
        kf[e8 * 4 + 3] = half2_pair(raw.w);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        uint64_t d0 = f2_mul(qf[g][0], kf[0]);
        uint64_t d1 = f2_mul(qf[g][1], kf[1]);
#pragma unroll
        for (int e = 2; e < C::E / 2; e += 2) {
          d0 = f2_fma(qf[g][e], kf[e], d0);
          d1 = f2_fma(qf[g][e + 1], kf[e + 1], d1);
        }
        float a0, a1, b0, b1;
        f2_unpack(d0, a0, a1);
        f2_unpack(d1, b0, b1);
        float dot = (a0 + a1) + (b0 + b1);
        dot += __shfl_xor_sync(0xffffffffu, dot, 4);
        dot += __shfl_xor_sync(0xffffffffu, dot, 2);
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        s[step][g] = (t < nt) ? dot : -INFINITY;
      }
    }
    // Online softmax over the stage's tokens (the 4 lane groups hold 4 tokens each).
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = fmaxf(fmaxf(s[0][g], s[1][g]), fmaxf(s[2][g], s[3][g]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float mn = fmaxf(m[g], mx);
      const float alpha = fast_exp2(m[g] - mn);
      float ps = 0.f;
#pragma unroll
      for (int step = 0; step < kTok / 4; ++step) {
        s[step][g] = fast_exp2(s[step][g] - mn);
        ps += s[step][g];
      }
      ps += __shfl_xor_sync(0xffffffffu, ps, 8);
      ps += __shfl_xor_sync(0xffffffffu, ps, 16);
      l[g] = l[g] * alpha + ps;
      m[g] = mn;
      const uint64_t al2 = f2_pack(alpha, alpha);
#pragma unroll
      for (int a = 0; a < NACC; ++a)
#pragma unroll
        for (int j = 0; j < C::DV / 2; ++j) acc[a][g][j] = f2_mul(acc[a][g][j], al2);
    }
    // P V: lane owns output columns [lane * DV, lane * DV + DV). A full stage
    // runs branch-free; a partial one (the last of a unit) skips the missing
    // tokens, whose shared-memory rows hold stale data.
    const __half* vst = reinterpret_cast<const __half*>(st + C::KV) + lane * C::DV;
    auto pv = [&](int t) {
      uint64_t vf[C::DV / 2];
      if constexpr (C::DV == 4) {
        const uint2 raw = *reinterpret_cast<const uint2*>(vst + t * D);
        vf[0] = half2_pair(raw.x);
        vf[1] = half2_pair(raw.y);
      } else {
        vf[0] = half2_pair(*reinterpret_cast<const uint32_t*>(vst + t * D));
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pt = __shfl_sync(0xffffffffu, s[t >> 2][g], (t & 3) * 8);
        const uint64_t pt2 = f2_pack(pt, pt);
#pragma unroll
        for (int j = 0; j < C::DV / 2; ++j)
          acc[t % NACC][g][j] = f2_fma(pt2, vf[j], acc[t % NACC][g][j]);
      }
    };
    if (nt == kTok) {
#pragma unroll
      for (int t = 0; t < kTok; ++t) pv(t);
    } else {
#pragma unroll
      for (int t = 0; t < kTok; ++t)
        if (t < nt) pv(t);
    }
    __syncwarp();
    if (md.w & 64) {
      const int b = md.x, kvh = md.y, split = md.z;
      const int ns = min((ctx_s[b] + p.partition - 1) / p.partition, p.num_splits);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float inv = 1.f / l[g];
        float o[C::DV];
#pragma unroll
        for (int j = 0; j < C::DV / 2; ++j) {
          uint64_t v = acc[0][g][j];
          if constexpr (NACC == 2) v = f2_add(v, acc[1][g][j]);
          f2_unpack(v, o[2 * j], o[2 * j + 1]);
          o[2 * j] *= inv;
          o[2 * j + 1] *= inv;
        }
        const size_t row = static_cast<size_t>(b) * p.hq + kvh * G + g;
        if (p.direct_out && ns == 1) {
          __half* dst = p.out + row * D + lane * C::DV;
          if constexpr (C::DV == 4) {
            *reinterpret_cast<uint2*>(dst) =
                make_uint2(pack_half2(o[0], o[1]), pack_half2(o[2], o[3]));
          } else {
            *reinterpret_cast<uint32_t*>(dst) = pack_half2(o[0], o[1]);
          }
        } else {
          const size_t pr = row * p.num_splits + split;
          float* dst = p.o_part + pr * D + lane * C::DV;
          if constexpr (C::DV == 4) {
            *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
          } else {
            *reinterpret_cast<float2*>(dst) = make_float2(o[0], o[1]);
          }
          if (lane == 0) {
            p.m_part[pr] = m[g];
            p.l_part[pr] = l[g];
          }
        }
      }
    }
    }  // G == 1
    ++c_item;
    return true;
  };

  // First unit: warp w of CTA c takes unit w * grid + c, so a launch with fewer
  // units than warps spreads them over all SMs; later units come from the counter.
  nxt = warp * gridDim.x + blockIdx.x;
  advance();
  for (int i = 0; i < C::STAGES; ++i) produce();
  while (c_item < p_item) {
    if (!consume()) break;
    // The slot just read is refilled by the async proxy.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    produce();
  }
  // Never exit with a copy in flight (only reached with copies pending after a timeout).
  while (c_item < p_item) {
    const unsigned int slot = c_item % C::STAGES;
    mbar_wait(full + slot, (c_item / C::STAGES) & 1u, nullptr, p.status, kSiteDecodeDrain,
              p.timeout_ns);
    ++c_item;
  }
}


struct MergeParams {
  const float* o;
  const float* m;
  const float* l;
  const int* ctx;  // non-null: row r has min(ceil(ctx[r / hq] / partition), num_parts) parts
  long long rows;
  long long o_row_stride, o_part_stride, ml_row_stride, ml_part_stride;
  int hq, partition, num_parts;
  int skip_single;  // rows with exactly one part were written by the decode kernel
  __half* out16;    // fp16 [rows, D], or else the merged partial state:
  float* out_o;     // fp32 [rows, D]
  float* out_m;     // fp32 [rows]
  float* out_l;
};

// WPR warps per row (1 or 8): a CTA of 8 warps merges 8 / WPR rows, and the
// warps of one row take contiguous ranges of its parts. Lane owns D / 32
// consecutive columns. A warp walks its parts in chunks of 8, loading the
// chunk's m, l and o rows at once and folding them into a running
// (max, sum, numerator) like the online softmax, so the loads of a warp's parts
// are one round trip per chunk; the warps of a row then combine their states in
// shared memory, each rescaled to the row's max. With many parts per row (a long
// context cut into many splits, few rows) eight warps keep eight times as many
// part rows in flight.
//
// The kernel is launched as a programmatic dependent of the decode launch before
// it: it may start while that launch runs and waits (griddepcontrol.wait) for
// its completion before reading the partials. context_lens, an input of the
// decode launch, is read before the wait.
template <int D, int WPR>
__global__ void __launch_bounds__(256) merge_partials_kernel(const MergeParams p) {
  constexpr int DV = D / 32;
  constexpr int ROWS = 8 / WPR;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int sub = warp % WPR;
  const long long row = static_cast<long long>(blockIdx.x) * ROWS + warp / WPR;
  bool live = row < p.rows;
  int ns = p.num_parts;
  if (live && p.ctx != nullptr) {
    const int c = max(p.ctx[row / p.hq], 0);
    ns = min((c + p.partition - 1) / p.partition, p.num_parts);
  }
  if (live && p.skip_single && ns == 1) live = false;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // A programmatic dependent launched after this kernel (the exchange of
  // context-parallel decode) may be scheduled now; it waits for this kernel's
  // completion before it reads the merged partials.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if constexpr (WPR == 1) {
    if (!live) return;
  }
  float mw = -INFINITY;  // running max of this warp's parts
  float den = 0.f;       // sum of l_s 2^(m_s - mw)
  float num[DV];         // sum of l_s 2^(m_s - mw) o_s, this lane's columns
#pragma unroll
  for (int j = 0; j < DV; ++j) num[j] = 0.f;
  if (live) {
    const float* mrow = p.m + row * p.ml_row_stride;
    const float* lrow = p.l + row * p.ml_row_stride;
    const float* orow = p.o + row * p.o_row_stride + lane * DV;
    const int per = (ns + WPR - 1) / WPR;
    const int s_begin = min(ns, sub * per);
    const int s_end = min(ns, s_begin + per);
    for (int s0 = s_begin; s0 < s_end; s0 += 8) {
      const int cnt = min(8, s_end - s0);
      // Lane u holds m and l of part s0 + u % 8 (the four octets alike).
      const bool have = (lane & 7) < cnt;
      const long long su = static_cast<long long>(s0 + (lane & 7)) * p.ml_part_stride;
      const float mu = have ? mrow[su] : -INFINITY;
      const float lu = have ? lrow[su] : 0.f;
      float v[8][DV];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float* src = orow + static_cast<long long>(s0 + u) * p.o_part_stride;
        if (u < cnt) {
          if constexpr (DV == 4) {
            const float4 x = *reinterpret_cast<const float4*>(src);
            v[u][0] = x.x; v[u][1] = x.y; v[u][2] = x.z; v[u][3] = x.w;
          } else {
            const float2 x = *reinterpret_cast<const float2*>(src);
            v[u][0] = x.x; v[u][1] = x.y;
          }
        } else {
#pragma unroll
          for (int j = 0; j < DV; ++j) v[u][j] = 0.f;
        }
      }
      float cm = mu;
      cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 1));
      cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 2));
      cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 4));
      const float mn = fmaxf(mw, cm);
      if (mn == -INFINITY) continue;  // no context in these parts, nor before
      const float alpha = fast_exp2(mw - mn);
      const float wu = lu * fast_exp2(mu - mn);
      float ws = wu;
      ws += __shfl_xor_sync(0xffffffffu, ws, 1);
      ws += __shfl_xor_sync(0xffffffffu, ws, 2);
      ws += __shfl_xor_sync(0xffffffffu, ws, 4);
      den = den * alpha + ws;
#pragma unroll
      for (int j = 0; j < DV; ++j) num[j] *= alpha;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float w = __shfl_sync(0xffffffffu, wu, u);
#pragma unroll
        for (int j = 0; j < DV; ++j) num[j] = fmaf(w, v[u][j], num[j]);
      }
      mw = mn;
    }
  }
  if constexpr (WPR > 1) {
    // The row's warps combine their states in shared memory; the first one writes.
    __shared__ float red[8][D + 2];
#pragma unroll
    for (int j = 0; j < DV; ++j) red[warp][lane * DV + j] = num[j];
    if (lane == 0) {
      red[warp][D] = den;
      red[warp][D + 1] = mw;
    }
    __syncthreads();
    if (!live || sub != 0) return;
    float mrow_max = mw;
    for (int w = 1; w < WPR; ++w) mrow_max = fmaxf(mrow_max, red[warp + w][D + 1]);
    if (mrow_max == -INFINITY) {
      den = 0.f;
    } else {
      const float a0 = fast_exp2(mw - mrow_max);
      den *= a0;
#pragma unroll
      for (int j = 0; j < DV; ++j) num[j] *= a0;
      for (int w = 1; w < WPR; ++w) {
        const float a = fast_exp2(red[warp + w][D + 1] - mrow_max);
        den = fmaf(a, red[warp + w][D], den);
#pragma unroll
        for (int j = 0; j < DV; ++j) num[j] = fmaf(a, red[warp + w][lane * DV + j], num[j]);
      }
    }
    mw = mrow_max;
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  if (p.out16 != nullptr) {
    __half* dst = p.out16 + row * D + lane * DV;
    if constexpr (DV == 4) {
      *reinterpret_cast<uint2*>(dst) =
          make_uint2(pack_half2(num[0] * inv, num[1] * inv), pack_half2(num[2] * inv, num[3] * inv));
    } else {
      *reinterpret_cast<uint32_t*>(dst) = pack_half2(num[0] * inv, num[1] * inv);
    }
  } else {
    float* dst = p.out_o + row * D + lane * DV;
#pragma unroll
    for (int j = 0; j < DV; ++j) dst[j] = num[j] * inv;
    if (lane == 0) {
      p.out_m[row] = mw;
      p.out_l[row] = den;
    }
  }
}

// Waits on an mbarrier that nothing arrives on: the bounded wait must give up,
// record ATTN_DEVICE_WAIT_TIMEOUT and let the kernel finish.
__global__ void wait_selftest_kernel(DeviceStatus* status, unsigned long long timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  mbar_wait(&bar, 0, &abort_flag, status, 301u, timeout_ns);
  __syncthreads();
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

struct DecodeWorkspace {
  unsigned int* counters;
  float* o_part;
  float* m_part;
  float* l_part;
  size_t bytes;
};

DecodeWorkspace carve_workspace(void* base, int64_t batch, int64_t hq, int64_t d,
                                int64_t num_splits) {
  DecodeWorkspace w;
  const int64_t chunks = (batch + kMinLaunchBatch - 1) / kMinLaunchBatch;
  const size_t rows = static_cast<size_t>(batch) * hq;
  const size_t c_bytes = align256(static_cast<size_t>(chunks) * 4);
  const size_t o_bytes = align256(rows * num_splits * d * 4);
  const size_t ml_bytes = align256(rows * num_splits * 4);
  uint8_t* b = static_cast<uint8_t*>(base);
  w.counters = reinterpret_cast<unsigned int*>(b);
  w.o_part = reinterpret_cast<float*>(b + c_bytes);
  w.m_part = reinterpret_cast<float*>(b + c_bytes + o_bytes);
  w.l_part = reinterpret_cast<float*>(b + c_bytes + o_bytes + ml_bytes);
  w.bytes = c_bytes + o_bytes + 2 * ml_bytes;
  return w;
}

int64_t splits_of(int64_t max_ctx, int64_t partition) {
  return max_ctx > 0 ? (max_ctx + partition - 1) / partition : 0;
}

template <int D, int G>
cudaError_t launch_decode_kernel(const DecParams& prm, int64_t upper_units, const LaunchCtx& ctx) {
  using C = DecCfg<D, G>;
  auto kern = paged_decode_kernel<D, G>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  });
  if (attr_err != cudaSuccess) return attr_err;
  // One CTA per SM, or one per unit when there are fewer units than SMs.
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ctx.sm_count, upper_units)));
  kern<<<grid, C::THREADS, C::SMEM, ctx.stream>>>(prm);
  return cudaGetLastError();
}

// Sequences one launch of the (d, g) configuration takes.
int64_t launch_batch(int64_t d, int64_t g) {
  if (d == 64) {
    switch (g) {
      case 1: return DecCfg<64, 1>::MAXB;
      case 2: return DecCfg<64, 2>::MAXB;
      case 4: return DecCfg<64, 4>::MAXB;
      default: return DecCfg<64, 8>::MAXB;
    }
  }
  switch (g) {
    case 1: return DecCfg<128, 1>::MAXB;
    case 2: return DecCfg<128, 2>::MAXB;
    case 4: return DecCfg<128, 4>::MAXB;
    default: return DecCfg<128, 8>::MAXB;
  }
}

template <int D>
cudaError_t dispatch_group(int g, const DecParams& prm, int64_t upper, const LaunchCtx& ctx) {
  switch (g) {
    case 1: return launch_decode_kernel<D, 1>(prm, upper, ctx);
    case 2: return launch_decode_kernel<D, 2>(prm, upper, ctx);
    case 4: return launch_decode_kernel<D, 4>(prm, upper, ctx);
    case 8: return launch_decode_kernel<D, 8>(prm, upper, ctx);
    default: return cudaErrorInvalidValue;
  }
}

// Launched as a programmatic dependent of the stream's previous kernel (the
// kernel waits for it before reading any partial).
template <int D, int WPR>
cudaError_t launch_merge_kernel(const MergeParams& mp, unsigned grid, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, merge_partials_kernel<D, WPR>, mp);
}

cudaError_t launch_merge_impl(const MergeParams& mp, int d, cudaStream_t stream) {
  if (mp.rows == 0) return cudaSuccess;
  // Eight warps per row from 32 parts up (at least four parts per warp).
  if (mp.num_parts >= 32) {
    const unsigned grid = static_cast<unsigned>(mp.rows);
    return d == 64 ? launch_merge_kernel<64, 8>(mp, grid, stream)
                   : launch_merge_kernel<128, 8>(mp, grid, stream);
  }
  const unsigned grid = static_cast<unsigned>((mp.rows + 7) / 8);
  return d == 64 ? launch_merge_kernel<64, 1>(mp, grid, stream)
                 : launch_merge_kernel<128, 1>(mp, grid, stream);
}

}  // namespace

// Sub-splits. A call with few (sequence, kv head, split) units leaves most of the
// resident warps idle while each busy warp walks its split one 16-token stage at
// a time, so the launch takes about (tokens per split / 16) stage latencies. Such
// calls cut every partition into k = 2 or 4 sub-partitions (at least 64 tokens)
// that are merged like splits; the result differs from k = 1 only by rounding.
// The workspace is sized for the largest k the sizes allow (a bound on the
// partial rows that keeps it small), so sizing needs no device query; the launch
// picks k from the units and the resident warps of the device.
constexpr int64_t kSubRowBudget = 8192;  // (sequence, query head, part) rows at most

int64_t sub_split_cap(int64_t batch, int64_t hq, int64_t max_ctx, int64_t partition) {
  const int64_t rows = batch * hq * splits_of(max_ctx, partition);
  for (int64_t k = 4; k > 1; k /= 2)
    if (partition / k >= 64 && rows * k <= kSubRowBudget) return k;
  return 1;
}

int64_t resident_warps(int64_t d, int64_t g, int64_t sm_count) {
  const int64_t w = d == 64 ? (g == 1 ? DecCfg<64, 1>::W : g == 2 ? DecCfg<64, 2>::W
                                       : g == 4 ? DecCfg<64, 4>::W : DecCfg<64, 8>::W)
                            : (g == 1 ? DecCfg<128, 1>::W : g == 2 ? DecCfg<128, 2>::W
                                       : g == 4 ? DecCfg<128, 4>::W : DecCfg<128, 8>::W);
  return w * sm_count;
}

size_t decode_workspace_bytes(int64_t batch, int64_t hq, int64_t d, int64_t max_ctx,
                              int64_t partition) {
  const int64_t cap = sub_split_cap(batch, hq, max_ctx, partition);
  return carve_workspace(nullptr, batch, hq, d, splits_of(max_ctx, partition) * cap).bytes;
}

cudaError_t launch_paged_decode(const DecodeArgs& a, bool partials_mode, const LaunchCtx& ctx) {
  // Sub-split only while the units stay within one per resident warp.
  int64_t k = sub_split_cap(a.batch, a.hq, a.max_ctx, a.partition);
  const int64_t units = a.batch * a.hkv * splits_of(a.max_ctx, a.partition);
  while (k > 1 && units * k > resident_warps(a.d, a.hq / a.hkv, ctx.sm_count)) k /= 2;
  const int64_t part = a.partition / k;
  const int64_t num_splits = splits_of(a.max_ctx, part);
  const int64_t rows = a.batch * a.hq;
  DecodeWorkspace w = carve_workspace(a.workspace, a.batch, a.hq, a.d, num_splits);
  if (num_splits == 0 && !partials_mode) {
    return cudaMemsetAsync(a.out, 0, static_cast<size_t>(rows) * a.d * 2, ctx.stream);
  }
  if (num_splits > 0) {
    const int g = static_cast<int>(a.hq / a.hkv);
    const int64_t per_launch = launch_batch(a.d, g);  // >= kMinLaunchBatch: one counter each
    const int64_t chunks = (a.batch + per_launch - 1) / per_launch;
    cudaError_t e = cudaMemsetAsync(w.counters, 0, static_cast<size_t>(chunks) * 4, ctx.stream);
    if (e != cudaSuccess) return e;
    for (int64_t c = 0; c < chunks; ++c) {
      const int64_t b0 = c * per_launch;
      const int64_t nb = std::min<int64_t>(per_launch, a.batch - b0);
      DecParams prm;
      prm.q = static_cast<const __half*>(a.q) + b0 * a.hq * a.d;
      prm.kc = static_cast<const __half*>(a.k_cache);
      prm.vc = static_cast<const __half*>(a.v_cache);
      prm.bt = a.block_tables + b0 * a.max_blocks;
      prm.ctx = a.context_lens + b0;
      prm.out = partials_mode ? nullptr : static_cast<__half*>(a.out) + b0 * a.hq * a.d;
      prm.o_part = w.o_part + b0 * a.hq * num_splits * a.d;
      prm.m_part = w.m_part + b0 * a.hq * num_splits;
      prm.l_part = w.l_part + b0 * a.hq * num_splits;
      prm.counter = w.counters + c;
      prm.status = ctx.status;
      prm.timeout_ns = ctx.timeout_ns;
      prm.block_stride = a.hkv * a.bs * a.d;
      prm.batch = static_cast<int>(nb);
      prm.hq = static_cast<int>(a.hq);
      prm.hkv = static_cast<int>(a.hkv);
      prm.bs = static_cast<int>(a.bs);
      prm.max_blocks = static_cast<int>(a.max_blocks);
      prm.partition = static_cast<int>(part);
      prm.num_blocks = static_cast<int>(a.num_blocks);
      prm.num_splits = static_cast<int>(num_splits);
      prm.direct_out = partials_mode ? 0 : 1;
      prm.scale_log2 = a.scale * kLog2e;
      const int64_t upper = nb * a.hkv * num_splits;
      e = (a.d == 64) ? dispatch_group<64>(g, prm, upper, ctx)
                      : dispatch_group<128>(g, prm, upper, ctx);
      if (e != cudaSuccess) return e;
    }
  }
  if (!partials_mode && num_splits <= 1) return cudaSuccess;
  MergeParams mp;
  mp.o = w.o_part;
  mp.m = w.m_part;
  mp.l = w.l_part;
  mp.ctx = a.context_lens;
  mp.rows = rows;
  mp.o_row_stride = num_splits * a.d;
  mp.o_part_stride = a.d;
  mp.ml_row_stride = num_splits;
  mp.ml_part_stride = 1;
  mp.hq = static_cast<int>(a.hq);
  mp.partition = static_cast<int>(part);
  mp.num_parts = static_cast<int>(num_splits);
  mp.skip_single = partials_mode ? 0 : 1;
  mp.out16 = partials_mode ? nullptr : static_cast<__half*>(a.out);
  mp.out_o = a.o_final;
  mp.out_m = a.m_final;
  mp.out_l = a.l_final;
  return launch_merge_impl(mp, static_cast<int>(a.d), ctx.stream);
}

cudaError_t launch_merge(const float* o_parts, const float* m_parts, const float* l_parts,
                         int64_t num_parts, int64_t rows, int64_t d, int64_t o_part_stride,
                         int64_t ml_part_stride, void* out, const LaunchCtx& ctx) {
  MergeParams mp;
  mp.o = o_parts;
  mp.m = m_parts;
  mp.l = l_parts;
  mp.ctx = nullptr;
  mp.rows = rows;
  mp.o_row_stride = d;
  mp.o_part_stride = o_part_stride;
  mp.ml_row_stride = 1;
  mp.ml_part_stride = ml_part_stride;
  mp.hq = 1;
  mp.partition = 1;
  mp.num_parts = static_cast<int>(num_parts);
  mp.skip_single = 0;
  mp.out16 = static_cast<__half*>(out);
  mp.out_o = nullptr;
  mp.out_m = nullptr;
  mp.out_l = nullptr;
  return launch_merge_impl(mp, static_cast<int>(d), ctx.stream);
}

cudaError_t launch_selftest_wait(unsigned long long timeout_ns, const LaunchCtx& ctx) {
  wait_selftest_kernel<<<1, 32, 0, ctx.stream>>>(ctx.status, timeout_ns);
  return cudaGetLastError();
}


// ------------------------------------------------ allocation-free decode entry
//
// Some callers cannot allocate device memory at the point where they run decode:
// a plugin inside a serving framework that owns the whole device-memory pool and
// hands its plugins no allocator, or a latency-critical serving loop where a
// cudaMalloc / cudaFree (which can synchronise the device) is not allowed. For
// them the split-K scratch of the decode path (work counters and the fp32
// (o, m, l) partials) can live in this fixed array instead of a caller
// workspace. Every GPU that loads the library holds these bytes until the
// process exits. All calls on a device share the array: calls that overlap on
// the GPU (for example on two streams at once) race on it and must not be made.
// The counters are cleared by every call; the partials are fully rewritten
// before they are read.
static __device__ __align__(256) uint8_t g_decode_scratch[kDecodeStaticScratchBytes];

namespace {

std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {};

}  // namespace

cudaError_t paged_decode_static_scratch(DecodeArgs a, const LaunchCtx& ctx, std::string* err) {
  const size_t need = decode_workspace_bytes(a.batch, a.hq, a.d, a.max_ctx, a.partition);
  if (need > kDecodeStaticScratchBytes) {
    *err = "paged_decode_noalloc: this problem needs " + std::to_string(need) +
           " bytes of split-K scratch, above the fixed " +
           std::to_string(kDecodeStaticScratchBytes) +
           " bytes; use attn_paged_decode with a caller workspace, or a larger partition";
    return cudaErrorInvalidValue;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  void* base = nullptr;
  {
    // Set-up once per device, with that device current: the array's name is a
    // host-side stand-in, so the kernels get its device address instead.
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_ptr[dev] == nullptr) {
      void* ptr = nullptr;
      e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
      if (e != cudaSuccess) {
        *err = std::string("paged_decode_noalloc: cudaGetSymbolAddress failed: ") +
               cudaGetErrorString(e);
        return e;
      }
      g_scratch_ptr[dev] = ptr;
    }
    base = g_scratch_ptr[dev];
  }
  a.workspace = base;
  a.workspace_bytes = kDecodeStaticScratchBytes;
  return launch_paged_decode(a, false, ctx);
}

}  // namespace fab
