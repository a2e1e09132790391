// FlashAttention forward on the sm_100a tensor cores.
//
// Same mathematics as the reference's flash_wmma_kernel
// (attnkernels/csrc/flash_wmma.cu:53-219): per query row an online softmax in
// base 2 (m_new = max(m, rowmax), alpha = 2^(m - m_new), l = l alpha + sum p,
// O = O alpha + P V, O / l at the end), fp32 scores, P rounded to fp16 for the
// second product, top-left causal mask (key > query masked) and masking of keys
// past the sequence end. The execution model is Blackwell's:
//
//   * A CTA owns NQ = 2 query tiles of 128 rows of one (batch, head) and walks
//     the key/value tiles of 128 rows. Warp roles:
//       warps 0-3, 4-7  softmax warpgroups, one per query tile, one thread per row
//       warp  8         MMA issuer (the warp runs the loop, one elected lane
//                       issues) + tensor-memory allocator
//       warp  9         TMA producer (one thread)
//       warp 10         step signaller: one barrier per key step once V_j and
//                       K_{j+1} have both arrived, so the MMA warp waits once
//       warp 11         idle (it completes the control warpgroup)
//     setmaxnreg moves registers from the control warpgroup to the softmax
//     warpgroups, so a whole 128-column score row stays in registers.
//   * Q, K, V tiles arrive by TMA (128-byte swizzle, zero fill past the end of
//     the sequence) into one ring of K and V tiles (5 slots at D = 128).
//   * S_i = Q_i K^T is a tcgen05.mma with both operands in shared memory and the
//     fp32 result in tensor memory (TMEM). The softmax thread of row r reads row
//     r of S_i from TMEM lane r, writes P as packed fp16 back over the first 64
//     columns of S_i, and O_i += P_i V is a tcgen05.mma with A = P read from
//     TMEM and B = V from shared memory (MN-major), accumulating in TMEM.
//   * The two query tiles ping-pong: while one warpgroup does its softmax the
//     tensor core runs the other tile's products.
//   * O is rescaled only when a row's running max grows by more than 2^8
//     (P then stays <= 256, well inside fp16); the final O / l uses the same
//     stale max for numerator and denominator, so the result is unchanged.
//   * Causal: key tiles after a query tile's diagonal are never loaded or
//     multiplied; only the diagonal tile is masked element-wise. CTAs run
//     longest first inside groups of (batch, head) pairs, so the K/V tiles
//     of the CTAs in flight stay in L2.
//
// TMEM columns (512 allocated): S_0 [0,128), S_1 [128,256), O_0 and O_1 after.
// Every mbarrier wait is bounded; on timeout the CTA records the failure in
// the device status word, drains its copies and MMAs, frees TMEM and exits.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "launch.h"

namespace fab {
namespace {

constexpr int kBM = 128;                   // query rows per tile (MMA M)
constexpr int kBN = 128;                   // key rows per tile
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O when m grows by > 2^8
// Of the 128 exponentials per row, how many run on the FMA pipe (a compile-time
// tuning constant, a multiple of 4 up to 128; the rest use the MUFU).
#ifndef FAB_POLY_COLS
#define FAB_POLY_COLS 16
#endif
constexpr int kPolyCols = FAB_POLY_COLS;
static_assert(kPolyCols % 4 == 0 && kPolyCols <= kBN, "pairs of columns in each half");
// Register split of setmaxnreg (tuning constants; see TcCfg).
#ifndef FAB_CONTROL_REGS
#define FAB_CONTROL_REGS 64
#endif
#ifndef FAB_SOFTMAX_REGS
#define FAB_SOFTMAX_REGS 216
#endif

// Sites reported in the status word when a wait times out.
enum : unsigned int {
  kSiteLoadK = 101,
  kSiteLoadV,
  kSiteDrainLoads,
  kSiteMmaQ,
  kSiteMmaK,
  kSiteMmaV,
  kSiteMmaP,
  kSiteDrainMma,
  kSiteSoftS,
  kSiteSoftO,  // (unused: the rescale needs no wait; kept so site numbers stay stable)
  kSiteEpilogue
};

constexpr int pow2_ceil(int x) {
  int p = 32;
  while (p < x) p *= 2;
  return p;
}

template <int D, int NQ>
struct TcCfg {
  static constexpr int NHALF = D / 64;                // 64-column swizzle blocks per row
  static constexpr int BLK_BYTES = kBM * 64 * 2;      // one [128 rows][64 cols] block: 16 KB
  static constexpr int TILE_BYTES = NHALF * BLK_BYTES;
  static constexpr int Q_OFF = 0;
  // One ring of K and V tiles in load order K_0 V_0 K_1 V_1 ...: as many
  // slots as fit (5 at D = 128), so loads run about 1.5 key tiles ahead.
  static constexpr int RING_OFF = Q_OFF + NQ * TILE_BYTES;
  static constexpr int SLOTS_FIT = (227 * 1024 - 1024 - RING_OFF - 512) / TILE_BYTES;
  static constexpr int SLOTS = SLOTS_FIT < 8 ? SLOTS_FIT : 8;
  static constexpr int BAR_OFF = RING_OFF + SLOTS * TILE_BYTES;
  static constexpr int PAIRS = 4;  // key steps whose V_j + K_{j+1} arrival is signalled ahead
  static constexpr int NUM_BARS = 1 + 2 * SLOTS + 4 * NQ + 1 + PAIRS;
  static_assert(SLOTS >= 3, "K/V ring");
  static constexpr int MISC_OFF = BAR_OFF + NUM_BARS * 8;
  static constexpr int SMEM_ALLOC = MISC_OFF + 16 + 1024;  // + slack to align the base to 1 KB
  static constexpr int SOFT_WARPS = 4 * NQ;
  static constexpr int MMA_WARP = SOFT_WARPS;       // first warp of the control warpgroup
  static constexpr int LOAD_WARP = SOFT_WARPS + 1;
  static constexpr int THREADS = 32 * (SOFT_WARPS + 4);
  // Register split (setmaxnreg): launched at 168 per thread (65536 / 384,
  // rounded down to 8); the control warpgroup drops to 64 and the softmax
  // warpgroups rise to 216: 128 * 64 + 256 * 216 <= 384 * 168.
  static constexpr int LAUNCH_REGS = 168;
  static constexpr int CONTROL_REGS = FAB_CONTROL_REGS;
  static constexpr int SOFTMAX_REGS = FAB_SOFTMAX_REGS;
  static_assert(NQ == 2, "the register split assumes two softmax warpgroups");
  static_assert(128 * CONTROL_REGS + 256 * SOFTMAX_REGS <= THREADS * LAUNCH_REGS, "register split");
  static constexpr int O_COL = NQ * kBN;  // first O column; S_i at i * kBN
  static constexpr int TMEM_COLS = pow2_ceil(NQ * (kBN + D));
  static_assert(TMEM_COLS <= 512, "tensor memory holds 512 columns");
  static_assert(SMEM_ALLOC <= 227 * 1024, "shared memory per CTA");
};

struct TcParams {
  CUtensorMap tq, tk, tv;  // [bh][n][d] fp16, box 64 x 128 x 1, 128-byte swizzle
  __half* o;
  DeviceStatus* status;
  unsigned long long timeout_ns;
  int n;            // sequence length
  int n_tiles;      // ceil(n / 128): query tiles = key tiles
  int n_cta_tiles;  // ceil(n_tiles / NQ)
  int bh;           // batch * heads
  int group;        // (batch, head) pairs per scheduling group
  int first_group;  // pairs in the first group (1 .. group; the remainder)
  int causal;
  float scale_log2;
};

__device__ __forceinline__ int kv_tiles_of(const TcParams& p, int qt) {
  if (qt >= p.n_tiles) return 0;
  return p.causal ? min(qt + 1, p.n_tiles) : p.n_tiles;
}

template <int D, int NQ>
__global__ void __launch_bounds__(TcCfg<D, NQ>::THREADS, 1)
    flash_tc_kernel(const __grid_constant__ TcParams p) {
  using C = TcCfg<D, NQ>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars;
  uint64_t* full = q_full + 1;           // ring slot loaded (TMA transaction count)
  uint64_t* empty = full + C::SLOTS;     // ring slot released by the MMAs that read it
  uint64_t* s_full = empty + C::SLOTS;   // MMA -> softmax: S_i ready
  uint64_t* p_full = s_full + NQ;       // softmax -> MMA: half h of P_i written (2 i + h)
  uint64_t* o_full = p_full + 2 * NQ;   // MMA -> softmax: the last P_i V done
  uint64_t* drain = o_full + NQ;
  uint64_t* step_full = drain + 1;  // key step j: V_j and K_{j+1} both loaded (j % PAIRS)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::MISC_OFF + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // CTA order: the (batch, head) pairs in groups (the remainder group first,
  // then groups of p.group); inside a group the CTA rows run longest first
  // (row y = 0 holds the tiles nearest the end of the sequence), the pairs of
  // one row next to each other. The CTAs in flight then read the K/V of about
  // one group of pairs, which stays in L2, and the grid still ends on short
  // tiles, as a plain longest-first order does.
  int bh, qt0;
  {
    int r = static_cast<int>(blockIdx.x), g0 = 0, g_n = p.first_group;
    const int first_items = p.first_group * p.n_cta_tiles;
    if (r >= first_items) {
      r -= first_items;
      const int grp = r / (p.group * p.n_cta_tiles);
      r -= grp * p.group * p.n_cta_tiles;
      g0 = p.first_group + grp * p.group;
      g_n = p.group;
    }
    const int y = r / g_n;
    bh = g0 + (r - y * g_n);
    qt0 = (p.n_cta_tiles - 1 - y) * NQ;
  }
  const int nkv_max = kv_tiles_of(p, min(qt0 + NQ - 1, p.n_tiles - 1));

  // The TMA producer thread initialises the barriers and issues Q and the first
  // ring loads before the CTA-wide barrier, so those copies overlap the tensor
  // memory allocation and the barrier itself. A ring slot's first use needs no
  // wait; `issued` carries the count into the producer loop.
  const bool producer = warp == C::LOAD_WARP && lane == 0;
  int issued = 0;
  if (producer) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::SLOTS; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int i = 0; i < NQ; ++i) {
      mbar_init(s_full + i, 1);
      mbar_init(p_full + 2 * i, 4);  // one arrival per softmax warp
      mbar_init(p_full + 2 * i + 1, 4);
      mbar_init(o_full + i, 1);
    }
    mbar_init(drain, 1);
    for (int s = 0; s < C::PAIRS; ++s) mbar_init(step_full + s, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tensormap(&p.tq);
    prefetch_tensormap(&p.tk);
    prefetch_tensormap(&p.tv);
    int nq = 0;
    for (int i = 0; i < NQ; ++i) nq += (qt0 + i < p.n_tiles) ? 1 : 0;
    mbar_arrive_expect_tx(q_full, nq * C::TILE_BYTES);
    for (int i = 0; i < nq; ++i)
      for (int h = 0; h < C::NHALF; ++h)
        tma_load_3d(smem + C::Q_OFF + i * C::TILE_BYTES + h * C::BLK_BYTES, &p.tq, q_full,
                    h * 64, (qt0 + i) * kBM, bh);
    // Item 2 j is K_j and item 2 j + 1 is V_j; item `it` goes to slot
    // it % SLOTS on its (it / SLOTS)-th use of that slot.
    for (; issued < 2 * nkv_max && issued < C::SLOTS; ++issued) {
      mbar_arrive_expect_tx(full + issued, C::TILE_BYTES);
      const CUtensorMap* map = (issued & 1) ? &p.tv : &p.tk;
      for (int h = 0; h < C::NHALF; ++h)
        tma_load_3d(smem + C::RING_OFF + issued * C::TILE_BYTES + h * C::BLK_BYTES, map,
                    full + issued, h * 64, (issued >> 1) * kBN, bh);
    }
  }
  if (warp == C::MMA_WARP) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Each role sets its register budget and ends at its own copy of the final
  // barrier, so ptxas allocates every role's code at that role's budget.
  if (warp >= C::SOFT_WARPS) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::CONTROL_REGS));
    if (warp == C::LOAD_WARP) {
    // ------------------------------------------------------------ TMA producer
    if (producer) {
      // Q and the first SLOTS ring items were issued before the CTA barrier.
      for (int it = issued; it < 2 * nkv_max; ++it) {
        const int slot = it % C::SLOTS;
        if (!mbar_wait(empty + slot, ((it / C::SLOTS) & 1) ^ 1, abort_flag, p.status,
                       (it & 1) ? kSiteLoadV : kSiteLoadK, p.timeout_ns))
          break;
        mbar_arrive_expect_tx(full + slot, C::TILE_BYTES);
        const CUtensorMap* map = (it & 1) ? &p.tv : &p.tk;
        for (int h = 0; h < C::NHALF; ++h)
          tma_load_3d(smem + C::RING_OFF + slot * C::TILE_BYTES + h * C::BLK_BYTES, map,
                      full + slot, h * 64, (it >> 1) * kBN, bh);
        ++issued;
      }
      // Never leave with a copy in flight: wait (bounded, regardless of the
      // abort flag) for the last phase issued on every full barrier.
      mbar_wait(q_full, 0, nullptr, p.status, kSiteDrainLoads, p.timeout_ns);
      for (int sl = 0; sl < C::SLOTS; ++sl) {
        const int cnt = issued > sl ? (issued - 1 - sl) / C::SLOTS + 1 : 0;
        if (cnt > 0)
          mbar_wait(full + sl, (cnt - 1) & 1, nullptr, p.status, kSiteDrainLoads, p.timeout_ns);
      }
    }
  } else if (warp == C::MMA_WARP + 2) {
    // -------------------------------------------------------- step signaller
    // Folds the two ring waits of a key step into one for the MMA warp: waits
    // for V_j and then K_{j+1} and arrives on step_full[j % PAIRS]. It runs at
    // most the ring's depth ahead of the MMAs, fewer key steps than PAIRS.
    if (lane == 0) {
      int slot = 1 % C::SLOTS;  // ring item 1: V_0
      uint32_t phase = 1 / C::SLOTS;
      auto advance = [&]() {
        if (++slot == C::SLOTS) {
          slot = 0;
          phase ^= 1u;
        }
      };
      for (int j = 0; j < nkv_max; ++j) {
        if (!mbar_wait(full + slot, phase & 1, abort_flag, p.status, kSiteMmaV, p.timeout_ns))
          break;
        advance();
        if (j + 1 < nkv_max) {
          if (!mbar_wait(full + slot, phase & 1, abort_flag, p.status, kSiteMmaK, p.timeout_ns))
            break;
          advance();
        }
        mbar_arrive(step_full + j % C::PAIRS);
      }
    }
    __syncwarp();
  } else if (warp == C::MMA_WARP) {
    // ------------------------------------------------------------- MMA issuer
    // The whole warp runs the loop and its waits (voted, so every lane takes
    // the same path) and computes the operands as warp-uniform values; each
    // group of MMAs and commits is then issued by one elected lane.
    {
      constexpr uint32_t kIdescS = idesc_f16_f32(kBM, kBN, false, false);
      constexpr uint32_t kIdescO = idesc_f16_f32(kBM, D, false, true);
      // Descriptors are built once; a K step or a ring slot moves the start
      // address field (address / 16, bits 0-13), which never carries out
      // because shared memory ends below 256 KB.
      const uint64_t q_desc = sdesc_sw128(smem_u32(smem + C::Q_OFF), 16, 1024);
      const uint64_t k_desc0 = sdesc_sw128(smem_u32(smem + C::RING_OFF), 16, 1024);
      const uint64_t v_desc0 = sdesc_sw128(smem_u32(smem + C::RING_OFF), C::BLK_BYTES, 1024);
      constexpr uint32_t kTileStep = C::TILE_BYTES >> 4;
      auto wait_slot = [&](int slot, uint32_t phase, unsigned int site) {
        const bool r = mbar_wait(full + slot, phase, abort_flag, p.status, site, p.timeout_ns);
        return __all_sync(0xffffffffu, r);
      };
      int nkv[NQ];
#pragma unroll
      for (int i = 0; i < NQ; ++i) nkv[i] = kv_tiles_of(p, qt0 + i);

      // S_i = Q_i K^T: K = D in steps of 16 (32 bytes inside a 128-byte swizzle row).
      auto issue_s = [&](int i, int slot) {
        const uint64_t a0 = q_desc + i * kTileStep;
        const uint64_t b0 = k_desc0 + static_cast<uint32_t>(slot) * kTileStep;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          constexpr uint32_t kBlk = C::BLK_BYTES >> 4;
          const uint32_t off = (kk >> 2) * kBlk + (kk & 3) * 2;
          mma_f16_ss(tmem + i * kBN, a0 + off, b0 + off, kIdescS, kk > 0 ? 1u : 0u);
        }
      };
      // O_i (+)= P_i V: K = 128 keys in steps of 16 rows (2 KB of V); V is
      // MN-major, the 64-column blocks 16 KB apart (LBO), 8-row groups 1 KB (SBO).
      // Half h covers keys [64 h, 64 h + 64): P columns [32 h, 32 h + 32).
      auto issue_pv = [&](int i, int slot, int h, bool accumulate) {
        const uint64_t b0 = v_desc0 + static_cast<uint32_t>(slot) * kTileStep;
#pragma unroll
        for (int kk = 4 * h; kk < 4 * h + 4; ++kk) {
          mma_f16_ts(tmem + C::O_COL + i * D, tmem + i * kBN + kk * 8, b0 + kk * (2048 >> 4),
                     kIdescO, (accumulate || kk > 0) ? 1u : 0u);
        }
      };

      // Ring position of the next item: slot and the parity of its use.
      int slot = 0;
      uint32_t phase = 0;
      auto advance = [&]() {
        if (++slot == C::SLOTS) {
          slot = 0;
          phase ^= 1u;
        }
      };
      bool ok = __all_sync(0xffffffffu,
                           mbar_wait(q_full, 0, abort_flag, p.status, kSiteMmaQ, p.timeout_ns));
      ok = ok && wait_slot(0, 0, kSiteMmaK);
      if (ok) {
        tc_fence_after();
        if (elect_one()) {
#pragma unroll
          for (int i = 0; i < NQ; ++i) {
            if (nkv[i] > 0) {
              issue_s(i, 0);
              tc_commit(s_full + i);
            }
          }
          tc_commit(empty + 0);
        }
        __syncwarp();
      }
      advance();  // item 1: V_0
      for (int j = 0; ok && j < nkv_max; ++j) {
        const int v_slot = slot;  // V_j
        const uint32_t v_phase = phase;
        advance();
        const int k_slot = slot;  // K_{j+1}
        const uint32_t k_phase = phase;
        advance();
        (void)v_phase;
        (void)k_phase;
        // V_j and K_{j+1} are loaded (one wait; the fence follows the P wait).
        ok = __all_sync(0xffffffffu, mbar_wait(step_full + j % C::PAIRS, (j / C::PAIRS) & 1,
                                               abort_flag, p.status, kSiteMmaV, p.timeout_ns));
        if (!ok) break;
        const bool next = j + 1 < nkv_max;
        bool k_ready = false;
#pragma unroll
        for (int i = 0; i < NQ; ++i) {
          if (j < nkv[i]) {
            ok = __all_sync(0xffffffffu, mbar_wait(p_full + 2 * i, j & 1, abort_flag, p.status,
                                                   kSiteMmaP, p.timeout_ns));
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) issue_pv(i, v_slot, 0, j > 0);
            __syncwarp();
            ok = __all_sync(0xffffffffu, mbar_wait(p_full + 2 * i + 1, j & 1, abort_flag, p.status,
                                                   kSiteMmaP, p.timeout_ns));
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
              issue_pv(i, v_slot, 1, true);
              if (j + 1 == nkv[i]) tc_commit(o_full + i);  // O_i final
            }
            __syncwarp();
            if (next && j + 1 < nkv[i]) {
              k_ready = true;  // K_{j+1} came with the step signal
              if (elect_one()) {
                issue_s(i, k_slot);
                tc_commit(s_full + i);
              }
              __syncwarp();
            }
          }
        }
        if (!ok) break;
        if (elect_one()) {
          tc_commit(empty + v_slot);
          if (next && k_ready) tc_commit(empty + k_slot);
        }
        __syncwarp();
      }
      // Every MMA issued completes before tensor memory is released.
      if (elect_one()) tc_commit(drain);
      __syncwarp();
      mbar_wait(drain, 0, nullptr, p.status, kSiteDrainMma, p.timeout_ns);
    }
    __syncwarp();
    }
    tc_fence_before();
    named_barrier_sync(1, C::THREADS);
    if (warp == C::MMA_WARP) {
      tc_fence_after();
      tmem_dealloc(tmem, C::TMEM_COLS);
    }
  } else {
    // ------------------------------------------------------- softmax warpgroups
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(C::SOFTMAX_REGS));
    const int wg = warp >> 2;   // query tile of this warpgroup
    const int quarter = warp & 3;  // TMEM lanes [32 quarter, 32 quarter + 32)
    const int row = quarter * 32 + lane;
    const int qt = qt0 + wg;
    const int n_i = kv_tiles_of(p, qt);
    if (n_i > 0) {
      const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
      const uint32_t t_s = tmem + lane_off + wg * kBN;
      const uint32_t t_o = tmem + lane_off + C::O_COL + wg * D;
      const int q_row = qt * kBM + row;
      float m = -INFINITY;  // running max, log2 units
      float l = 0.f;        // running sum of 2^(x - m)
      bool ok = true;
      for (int j = 0; j < n_i; ++j) {
        ok = mbar_wait(s_full + wg, j & 1, abort_flag, p.status, kSiteSoftS, p.timeout_ns);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        // One register array for the row: fp32 scores in, packed fp16 P out
        // (P pair c overwrites slot c, whose scores were consumed at pair c).
        // With a positive scale the max is taken on the raw scores and the
        // scale is folded into the exponent's FMA; otherwise the row is
        // scaled first.
        uint32_t sr[kBN];
        const float cs = p.scale_log2 > 0.f ? p.scale_log2 : 1.f;
        const int k0 = j * kBN;
        const bool masked = (p.causal && j == qt) || k0 + kBN > p.n;
        // Columns [lo, hi) of the scores just loaded: scaled when the scale is
        // not positive, keys past the causal diagonal or the sequence end -inf.
        auto fix_cols = [&](int lo, int hi) {
          if (p.scale_log2 <= 0.f) {
            const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2);
#pragma unroll
            for (int c = lo; c < hi; c += 2) {
              float a, b;
              f2_unpack(f2_mul(f2_pack(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), sc2),
                        a, b);
              sr[c] = __float_as_uint(a);
              sr[c + 1] = __float_as_uint(b);
            }
          }
          if (masked) {
            const int lim = p.causal ? min(q_row + 1, p.n) : p.n;  // keys [0, lim) are visible
#pragma unroll
            for (int c = lo; c < hi; ++c)
              if (k0 + c >= lim) sr[c] = __float_as_uint(-INFINITY);
          }
        };
        // P = 2^(cs * s - m) in two halves of 64 keys; each half is stored and
        // handed to the MMA warp at once, so P V on the first half overlaps the
        // exponentials of the second. In each half the last kPolyCols / 2
        // columns go to the FMA pipe (f2_exp2_poly), the rest to the MUFU.
        uint64_t cs2, nm2, rs0, rs1;
        auto start_exps = [&]() {
          const float m_use = (m == -INFINITY) ? 0.f : m;
          cs2 = f2_pack(cs, cs);
          nm2 = f2_pack(-m_use, -m_use);
          rs0 = f2_pack(0.f, 0.f);
          rs1 = rs0;
        };
        auto exp_pair = [&](int c) {  // pair c: scores 2c, 2c+1 -> packed fp16 in sr[c]
          const uint64_t x =
              f2_fma(f2_pack(__uint_as_float(sr[2 * c]), __uint_as_float(sr[2 * c + 1])), cs2, nm2);
          uint64_t pr;
          if ((2 * c) % (kBN / 2) < kBN / 2 - kPolyCols / 2) {
            float a, b;
            f2_unpack(x, a, b);
            pr = f2_pack(fast_exp2(a), fast_exp2(b));
          } else {
            pr = f2_exp2_poly(x);
          }
          if (c & 1) rs1 = f2_add(rs1, pr); else rs0 = f2_add(rs0, pr);
          float a, b;
          f2_unpack(pr, a, b);
          sr[c] = pack_half2(a, b);
        };
        // O and l to a new running max. O_i already holds P_{j-1} V: the MMAs
        // of one thread complete in order, and S_i(j), whose completion this
        // thread waited for, was issued after P_{j-1} V.
        auto rescale = [&](float m_new) {
          const float alpha = fast_exp2(m - m_new);
#pragma unroll
          for (int c0 = 0; c0 < D; c0 += 32) {
            uint32_t o[32];
            tmem_ld32_wait(t_o + c0, o);
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              float a, b;
              f2_unpack(f2_mul(f2_pack(__uint_as_float(o[e]), __uint_as_float(o[e + 1])),
                               f2_pack(alpha, alpha)), a, b);
              o[e] = __float_as_uint(a);
              o[e + 1] = __float_as_uint(b);
            }
            tmem_st32<0>(t_o + c0, o);
          }
          tmem_st_wait();
          l *= alpha;
          m = m_new;
        };
        tmem_ld128_wait(t_s, sr);
        fix_cols(0, kBN);
        {
          // The row max (eight 3-input max chains), then O and l rescaled if it
          // grew by more than kRescaleThreshold.
          float mt[8];
#pragma unroll
          for (int a = 0; a < 8; ++a)
            mt[a] = fmax3(__uint_as_float(sr[3 * a]), __uint_as_float(sr[3 * a + 1]),
                          __uint_as_float(sr[3 * a + 2]));
#pragma unroll
          for (int c = 24; c < kBN; c += 2)
            mt[(c / 2) & 7] = fmax3(mt[(c / 2) & 7], __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
          const float m_new = fmaxf(
              m, fmax3(fmax3(mt[0], mt[1], mt[2]), fmax3(mt[3], mt[4], mt[5]), fmaxf(mt[6], mt[7])) * cs);
          if (j == 0)
            m = m_new;
          else if (__any_sync(0xffffffffu, m_new > m + kRescaleThreshold))
            rescale(m_new);
          start_exps();
#pragma unroll
          for (int c = 0; c < kBN / 4; ++c) exp_pair(c);
        }
        tmem_st32<0>(t_s, sr);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full + 2 * wg);
#pragma unroll
        for (int c = kBN / 4; c < kBN / 2; ++c) exp_pair(c);
        tmem_st32<32>(t_s + 32, sr);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full + 2 * wg + 1);
        {
          float a, b, c2, d2;
          f2_unpack(rs0, a, b);
          f2_unpack(rs1, c2, d2);
          l += (a + b) + (c2 + d2);
        }
      }
      if (ok) {
        ok = mbar_wait(o_full + wg, 0, abort_flag, p.status, kSiteEpilogue,
                       p.timeout_ns);
        ok = __all_sync(0xffffffffu, ok);
      }
      if (ok) {
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        __half* orow = p.o + (static_cast<size_t>(bh) * p.n + q_row) * D;
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          tmem_ld32_wait(t_o + c0, o);
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            w[e] = pack_half2(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
          if (q_row < p.n) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c0);
#pragma unroll
            for (int e = 0; e < 4; ++e)
              dst[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
          }
        }
      }
    }
    tc_fence_before();
    named_barrier_sync(1, C::THREADS);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// [bh][n][d] fp16 tensor, boxes of 64 columns x 128 rows, 128-byte swizzle.
bool make_qkv_map(CUtensorMap* map, const void* base, int64_t bh, int64_t n, int d,
                  std::string* err) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) {
    *err = "cuTensorMapEncodeTiled is not available from the driver";
    return false;
  }
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(n),
                        static_cast<cuuint64_t>(bh)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(d) * 2, static_cast<cuuint64_t>(n * d) * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims,
                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(r));
    return false;
  }
  return true;
}

template <int D, int NQ>
cudaError_t launch_tc(const TcParams& prm, int64_t bh, const LaunchCtx& ctx) {
  using C = TcCfg<D, NQ>;
  auto kern = flash_tc_kernel<D, NQ>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    C::SMEM_ALLOC);
  });
  if (attr_err != cudaSuccess) return attr_err;
  const unsigned grid = static_cast<unsigned>(bh * prm.n_cta_tiles);
  kern<<<grid, C::THREADS, C::SMEM_ALLOC, ctx.stream>>>(prm);
  return cudaGetLastError();
}

// Evaluates the exponentials the softmax uses, for the tests: y_poly[i] =
// f2_exp2_poly (FMA pipe), y_mufu[i] = ex2.approx.ftz, y_lib[i] = exp2f, each
// of x[i]. One thread per pair of inputs, as the kernel evaluates them.
__global__ void exp2_selftest_kernel(const float* __restrict__ x, float* __restrict__ y_poly,
                                     float* __restrict__ y_mufu, float* __restrict__ y_lib,
                                     int64_t n) {
  const int64_t i = 2 * (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const bool pair = i + 1 < n;
  const float a = x[i], b = pair ? x[i + 1] : x[i];
  float pa, pb;
  f2_unpack(f2_exp2_poly(f2_pack(a, b)), pa, pb);
  y_poly[i] = pa;
  y_mufu[i] = fast_exp2(a);
  y_lib[i] = exp2f(a);
  if (pair) {
    y_poly[i + 1] = pb;
    y_mufu[i + 1] = fast_exp2(b);
    y_lib[i + 1] = exp2f(b);
  }
}

}  // namespace

cudaError_t launch_flash_tc(const void* q, const void* k, const void* v, void* o, int64_t bh,
                            int64_t n, int d, bool causal, float scale, const LaunchCtx& ctx,
                            std::string* err) {
  constexpr int kNQ = 2;
  TcParams prm;
  if (!make_qkv_map(&prm.tq, q, bh, n, d, err) || !make_qkv_map(&prm.tk, k, bh, n, d, err) ||
      !make_qkv_map(&prm.tv, v, bh, n, d, err))
    return cudaErrorInvalidValue;
  prm.o = static_cast<__half*>(o);
  prm.status = ctx.status;
  prm.timeout_ns = ctx.timeout_ns;
  prm.n = static_cast<int>(n);
  prm.n_tiles = static_cast<int>((n + kBM - 1) / kBM);
  prm.n_cta_tiles = (prm.n_tiles + kNQ - 1) / kNQ;
  prm.bh = static_cast<int>(bh);
  // Pairs per group: enough for about four CTAs per SM, which keeps the
  // finishing times as even as one longest-first wave (checked by simulating
  // the greedy block dispatch over batch, head and length mixes).
  const int64_t want = (4 * static_cast<int64_t>(ctx.sm_count) + prm.n_cta_tiles - 1) /
                       prm.n_cta_tiles;
  prm.group = static_cast<int>(std::min<int64_t>(bh, std::max<int64_t>(1, want)));
  const int64_t n_groups = (bh + prm.group - 1) / prm.group;
  prm.first_group = static_cast<int>(bh - (n_groups - 1) * prm.group);
  prm.causal = causal ? 1 : 0;
  prm.scale_log2 = scale * kLog2e;
  if (d == 64) return launch_tc<64, kNQ>(prm, bh, ctx);
  return launch_tc<128, kNQ>(prm, bh, ctx);
}

cudaError_t launch_selftest_exp2(const float* x, float* y_poly, float* y_mufu, float* y_lib,
                                int64_t n, const LaunchCtx& ctx) {
  const int64_t pairs = (n + 1) / 2;
  const unsigned grid = static_cast<unsigned>((pairs + 255) / 256);
  exp2_selftest_kernel<<<grid, 256, 0, ctx.stream>>>(x, y_poly, y_mufu, y_lib, n);
  return cudaGetLastError();
}

}  // namespace fab
