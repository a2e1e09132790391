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
//       warps 10-11     idle (they complete the control warpgroup)
//     setmaxnreg moves registers from the control warpgroup to the softmax
//     warpgroups, so a whole 128-column score row stays in registers.
//   * Q, K, V tiles arrive by TMA (128-byte swizzle, zero fill past the end of
//     the sequence). K and V move in stages: the stage of key step j holds V_j
//     and K_{j+1}, loaded onto one mbarrier and released by one commit (2
//     stages at D = 128), so the MMA warp waits once and commits once per step.
//   * S_i = Q_i K^T is a tcgen05.mma with both operands in shared memory and the
//     fp32 result in tensor memory (TMEM). The softmax thread of row r reads row
//     r of S_i from TMEM lane r, writes P as packed fp16 back over 64 of the
//     128 columns of S_i, and O_i += P_i V is a tcgen05.mma with A = P read from
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
#include <functional>
#include <map>
#include <mutex>
#include <queue>
#include <tuple>
#include <vector>

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
  kSiteEpilogue,
  kSiteLoadQ,   // producer: the previous item's S MMAs to release Q
  kSiteMmaO     // MMA warp: the previous item's O_i to be read out
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
  // K/V stages: stage use g of an item holds K_g and V_{g-1} (use 0: K_0
  // alone), the two tiles key step g - 1 needs (V_{g-1} for P V, K_g for the
  // next S), loaded onto one barrier and released by one commit. Uses are
  // numbered over all of a CTA's items. As many stages as fit, at most 4
  // (2 at D = 128, 4 at D = 64).
  static constexpr int STAGE_OFF = Q_OFF + NQ * TILE_BYTES;
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;  // K tile, then V tile
  static constexpr int STAGES_FIT = (227 * 1024 - 1024 - STAGE_OFF - 512) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT < 4 ? STAGES_FIT : 4;
  static constexpr int BAR_OFF = STAGE_OFF + STAGES * STAGE_BYTES;
  static constexpr int NUM_BARS = 2 + 2 * STAGES + 5 * NQ + 1;
  static_assert(STAGES >= 2, "K/V stages");
  static_assert(NUM_BARS * 8 + 16 <= 512, "barriers fit the reserved bytes");
  static constexpr int MISC_OFF = BAR_OFF + NUM_BARS * 8;
  static constexpr int SMEM_ALLOC = MISC_OFF + 16 + 1024;  // + slack to align the base to 1 KB
  static constexpr int SOFT_WARPS = 4 * NQ;
  static constexpr int MMA_WARP = SOFT_WARPS;       // first warp of the control warpgroup
  static constexpr int LOAD_WARP = SOFT_WARPS + 1;
  static constexpr int THREADS = 32 * (SOFT_WARPS + 4);
  // Register split (setmaxnreg): launched at 168 per thread (65536 / 384,
  // rounded down to 8); the control warpgroup drops to CONTROL_REGS and the
  // softmax warpgroups rise to SOFTMAX_REGS, so a whole 128-column score row
  // stays in registers.
  static constexpr int LAUNCH_REGS = 168;
  static constexpr int CONTROL_REGS = FAB_CONTROL_REGS;
  static constexpr int SOFTMAX_REGS = FAB_SOFTMAX_REGS;
  static_assert(NQ == 2, "the register split assumes two softmax warpgroups");
  static_assert(128 * CONTROL_REGS + 256 * SOFTMAX_REGS <= THREADS * LAUNCH_REGS, "register split");
  static constexpr int O_COL = NQ * kBN;  // first O column; S_i at i * kBN
  // At D = 64 the next S_i is computed in two N = 64 halves and P_i (packed
  // fp16, 64 columns) is written over the second half of S_i, so the first
  // half of the next S_i (keys 0-63) runs while P_i V still reads P_i.
  // Measured on B200: config 2 at d 64 +2.5 %; at D = 128 the N = 64 S MMAs
  // are shared-memory bound (an SS 128x64x16 MMA reads 6 KB) and the split
  // costs 12 %, so there the whole S_i follows P_i V and P_i sits in the first
  // half.
  static constexpr bool SPLIT_S = D == 64;
  static constexpr int P_COL = SPLIT_S ? kBN / 2 : 0;
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

// Kernel arguments: the problem and this launch's schedule. An item is NQ
// query tiles of one (batch, head), numbered in the order of item_coords.
// With sched_ctas == 0, CTA b runs item b alone. Otherwise the grid has
// sched_ctas CTAs and CTA c runs, in order, the items
// sched[sched_ctas + 1 + sched[c]] .. sched[sched_ctas + 1 + sched[c + 1] - 1],
// a list schedule computed on the host. It travels by value in the kernel
// parameters: a launch needs no device memory and no counter, and launches on
// several streams or in CUDA graphs share no state.
template <int CAP>
struct TcArgs {
  TcParams p;
  int sched_ctas;
  uint16_t sched[CAP];
};
// Schedule capacities (entries): kernel parameters are limited to 32764 bytes.
constexpr int kSchedSmall = 2048;
constexpr int kSchedLarge = 15872;

__host__ __device__ __forceinline__ int kv_tiles_of(const TcParams& p, int qt) {
  if (qt >= p.n_tiles) return 0;
  return p.causal ? (qt + 1 < p.n_tiles ? qt + 1 : p.n_tiles) : p.n_tiles;
}

// Item r -> (batch * head index, first query tile). The (batch, head) pairs
// are cut into groups (the remainder group first, then groups of p.group);
// inside a group the rows of items run longest first (row y = 0 holds the
// tiles nearest the end of the sequence), the pairs of one row next to each
// other. The items in flight then read the K/V of about one group of pairs,
// which stays in L2, and the schedule still ends on short tiles.
template <int NQ>
__host__ __device__ __forceinline__ void item_coords(const TcParams& p, int r, int& bh, int& qt0) {
  int g0 = 0, g_n = p.first_group;
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

template <int NQ>
__host__ __device__ __forceinline__ int item_kv_steps(const TcParams& p, int qt0) {
  return kv_tiles_of(p, (qt0 + NQ - 1 < p.n_tiles - 1) ? qt0 + NQ - 1 : p.n_tiles - 1);
}

template <int D, int NQ, int CAP>
__global__ void __launch_bounds__(TcCfg<D, NQ>::THREADS, 1)
    flash_tc_kernel(const __grid_constant__ TcArgs<CAP> args) {
  using C = TcCfg<D, NQ>;
  const TcParams& p = args.p;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars;                // producer -> MMA: the item's Q loaded
  uint64_t* q_empty = q_full + 1;         // MMA -> producer: the item's last S read Q
  uint64_t* stage_full = q_empty + 1;     // stage loaded (TMA transaction count)
  uint64_t* stage_free = stage_full + C::STAGES;  // stage released by the MMAs that read it
  uint64_t* s_full = stage_free + C::STAGES;  // MMA -> softmax: S_i ready
  uint64_t* p_full = s_full + NQ;       // softmax -> MMA: half h of P_i written (2 i + h)
  uint64_t* o_full = p_full + 2 * NQ;   // MMA -> softmax: the item's last P_i V done
  uint64_t* o_empty = o_full + NQ;      // softmax -> MMA: O_i read out of tensor memory
  uint64_t* drain = o_empty + NQ;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::MISC_OFF + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // This CTA's items (read from the kernel parameters where needed, so they
  // hold no registers across the loops).
  const int n_items = args.sched_ctas == 0
                          ? 1
                          : static_cast<int>(args.sched[blockIdx.x + 1]) - args.sched[blockIdx.x];
  auto item_of = [&](int t) -> int {
    return args.sched_ctas == 0
               ? static_cast<int>(blockIdx.x)
               : args.sched[args.sched_ctas + 1 + args.sched[blockIdx.x] + t];
  };

  // Stage use u (over all items) of an item at its use g: K_g (if g < nkv) and
  // V_{g-1} (if g > 0) of pair bh into stage u % STAGES.
  auto issue_stage = [&](int u, int g, int nkv, int bh) {
    const int st = u % C::STAGES;
    const bool has_k = g < nkv, has_v = g > 0;
    uint8_t* buf = smem + C::STAGE_OFF + st * C::STAGE_BYTES;
    mbar_arrive_expect_tx(stage_full + st, ((has_k ? 1 : 0) + (has_v ? 1 : 0)) * C::TILE_BYTES);
    for (int h = 0; h < C::NHALF; ++h) {
      if (has_k)
        tma_load_3d(buf + h * C::BLK_BYTES, &p.tk, stage_full + st, h * 64, g * kBN, bh);
      if (has_v)
        tma_load_3d(buf + C::TILE_BYTES + h * C::BLK_BYTES, &p.tv, stage_full + st, h * 64,
                    (g - 1) * kBN, bh);
    }
  };
  auto issue_q = [&](int qt0, int bh) {
    int nq = 0;
    for (int i = 0; i < NQ; ++i) nq += (qt0 + i < p.n_tiles) ? 1 : 0;
    mbar_arrive_expect_tx(q_full, nq * C::TILE_BYTES);
    for (int i = 0; i < nq; ++i)
      for (int h = 0; h < C::NHALF; ++h)
        tma_load_3d(smem + C::Q_OFF + i * C::TILE_BYTES + h * C::BLK_BYTES, &p.tq, q_full,
                    h * 64, (qt0 + i) * kBM, bh);
  };

  // The TMA producer thread initialises the barriers and issues the first
  // item's Q and first stages before the CTA-wide barrier, so those copies
  // overlap the tensor memory allocation and the barrier itself. A stage's
  // first use needs no wait; `issued` carries the count into the producer loop.
  const bool producer = warp == C::LOAD_WARP && lane == 0;
  int issued = 0;
  if (producer) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int st = 0; st < C::STAGES; ++st) {
      mbar_init(stage_full + st, 1);
      mbar_init(stage_free + st, 1);
    }
    for (int i = 0; i < NQ; ++i) {
      mbar_init(s_full + i, 1);
      mbar_init(p_full + 2 * i, 4);  // one arrival per softmax warp
      mbar_init(p_full + 2 * i + 1, 4);
      mbar_init(o_full + i, 1);
      mbar_init(o_empty + i, 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tensormap(&p.tq);
    prefetch_tensormap(&p.tk);
    prefetch_tensormap(&p.tv);
    if (n_items > 0) {
      int bh, qt0;
      item_coords<NQ>(p, item_of(0), bh, qt0);
      const int nkv = item_kv_steps<NQ>(p, qt0);
      issue_q(qt0, bh);
      for (; issued <= nkv && issued < C::STAGES; ++issued) issue_stage(issued, issued, nkv, bh);
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
      // Item 0's Q and first stage uses were issued before the CTA barrier.
      // Use u reuses the stage of use u - STAGES once the MMAs released it;
      // an item's Q is loaded once the previous item's last S MMAs read theirs.
      int u = issued;
      int q_loads = n_items > 0 ? 1 : 0;
      bool ok = true;
      for (int t = 0; ok && t < n_items; ++t) {
        int bh, qt0;
        item_coords<NQ>(p, item_of(t), bh, qt0);
        const int nkv = item_kv_steps<NQ>(p, qt0);
        int g = 0;
        if (t == 0) {
          g = issued;
        } else {
          if (!mbar_wait(q_empty, (t - 1) & 1, abort_flag, p.status, kSiteLoadQ, p.timeout_ns)) {
            ok = false;
            break;
          }
          issue_q(qt0, bh);
          ++q_loads;
        }
        for (; g <= nkv; ++g, ++u) {
          if (u >= C::STAGES &&
              !mbar_wait(stage_free + u % C::STAGES, (u / C::STAGES - 1) & 1, abort_flag,
                         p.status, kSiteLoadK, p.timeout_ns)) {
            ok = false;
            break;
          }
          issue_stage(u, g, nkv, bh);
        }
      }
      // Never leave with a copy in flight: wait (bounded, regardless of the
      // abort flag) for the last phase issued on every barrier a copy signals.
      if (q_loads > 0)
        mbar_wait(q_full, (q_loads - 1) & 1, nullptr, p.status, kSiteDrainLoads, p.timeout_ns);
      for (int st = 0; st < C::STAGES; ++st) {
        const int cnt = u > st ? (u - 1 - st) / C::STAGES + 1 : 0;
        if (cnt > 0)
          mbar_wait(stage_full + st, (cnt - 1) & 1, nullptr, p.status, kSiteDrainLoads,
                    p.timeout_ns);
      }
    }
  } else if (warp == C::MMA_WARP) {
    // ------------------------------------------------------------- MMA issuer
    // The whole warp runs the loop and its waits (voted, so every lane takes
    // the same path) and computes the operands as warp-uniform values; each
    // group of MMAs and commits is then issued by one elected lane.
    {
      constexpr uint32_t kIdescS = idesc_f16_f32(kBM, kBN, false, false);
      constexpr uint32_t kIdescS64 = idesc_f16_f32(kBM, kBN / 2, false, false);
      constexpr uint32_t kIdescO = idesc_f16_f32(kBM, D, false, true);
      // Descriptors are built once; a K step or a stage moves the start
      // address field (address / 16, bits 0-13), which never carries out
      // because shared memory ends below 256 KB.
      const uint64_t q_desc = sdesc_sw128(smem_u32(smem + C::Q_OFF), 16, 1024);
      const uint64_t k_desc0 = sdesc_sw128(smem_u32(smem + C::STAGE_OFF), 16, 1024);
      const uint64_t v_desc0 =
          sdesc_sw128(smem_u32(smem + C::STAGE_OFF + C::TILE_BYTES), C::BLK_BYTES, 1024);
      constexpr uint32_t kTileStep = C::TILE_BYTES >> 4;
      constexpr uint32_t kStageStep = C::STAGE_BYTES >> 4;
      auto vote_wait = [&](uint64_t* bar, uint32_t phase, unsigned int site) {
        const bool r = mbar_wait(bar, phase, abort_flag, p.status, site, p.timeout_ns);
        return __all_sync(0xffffffffu, r);
      };
      // S_i = Q_i K^T: K = D in steps of 16 (32 bytes inside a 128-byte swizzle row).
      auto issue_s = [&](int i, int st) {
        const uint64_t a0 = q_desc + i * kTileStep;
        const uint64_t b0 = k_desc0 + static_cast<uint32_t>(st) * kStageStep;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          constexpr uint32_t kBlk = C::BLK_BYTES >> 4;
          const uint32_t off = (kk >> 2) * kBlk + (kk & 3) * 2;
          mma_f16_ss(tmem + i * kBN, a0 + off, b0 + off, kIdescS, kk > 0 ? 1u : 0u);
        }
      };
      // Keys [64 h, 64 h + 64) of S_i into TMEM columns [64 h, 64 h + 64) of S_i
      // (N = 64; the K rows start 64 rows = 8 KB into each 64-column block).
      auto issue_s_half = [&](int i, int st, int h) {
        const uint64_t a0 = q_desc + i * kTileStep;
        const uint64_t b0 = k_desc0 + static_cast<uint32_t>(st) * kStageStep + h * (8192 >> 4);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          constexpr uint32_t kBlk = C::BLK_BYTES >> 4;
          const uint32_t off = (kk >> 2) * kBlk + (kk & 3) * 2;
          mma_f16_ss(tmem + i * kBN + h * (kBN / 2), a0 + off, b0 + off, kIdescS64,
                     kk > 0 ? 1u : 0u);
        }
      };
      // O_i (+)= P_i V: K = 128 keys in steps of 16 rows (2 KB of V); V is
      // MN-major, the 64-column blocks 16 KB apart (LBO), 8-row groups 1 KB (SBO).
      // Half h covers keys [64 h, 64 h + 64): P columns [32 h, 32 h + 32).
      auto issue_pv = [&](int i, int st, int h, bool accumulate) {
        const uint64_t b0 = v_desc0 + static_cast<uint32_t>(st) * kStageStep;
#pragma unroll
        for (int kk = 4 * h; kk < 4 * h + 4; ++kk) {
          mma_f16_ts(tmem + C::O_COL + i * D, tmem + i * kBN + C::P_COL + kk * 8, b0 + kk * (2048 >> 4),
                     kIdescO, (accumulate || kk > 0) ? 1u : 0u);
        }
      };

      // Stage of the current use and the parity of its phase (uses counted
      // over all items); key steps of tile i so far (s_full / p_full phases)
      // and items in which tile i had work (o_full / o_empty phases). A stage
      // is released by one commit placed with the next P V (or, at an item's
      // start, with its first S), when the MMA queue has room again: its last
      // readers were issued before.
      int st = C::STAGES - 1;
      uint32_t ph = 1;
      auto next_use = [&]() {
        if (++st == C::STAGES) {
          st = 0;
          ph ^= 1u;
        }
      };
      int pending = -1;  // stage whose release is due
      // Bit i: parity of tile i's key steps so far (s_full / p_full phases);
      // bit 4 + i: parity of the items in which tile i had work (o_full /
      // o_empty phases); bit 8 + i: tile i had work in an earlier item.
      uint32_t par = 0;
      bool ok = true;
      for (int t = 0; ok && t < n_items; ++t) {
        int bh, qt0;
        item_coords<NQ>(p, item_of(t), bh, qt0);
        (void)bh;
        int nkv[NQ];
#pragma unroll
        for (int i = 0; i < NQ; ++i) nkv[i] = kv_tiles_of(p, qt0 + i);
        const int nkv_max = item_kv_steps<NQ>(p, qt0);
        // Use 0 of the item (K_0): the first S of both tiles.
        next_use();
        ok = vote_wait(q_full, t & 1, kSiteMmaQ) && vote_wait(stage_full + st, ph, kSiteMmaK);
        if (!ok) break;
        tc_fence_after();
        if (elect_one()) {
#pragma unroll
          for (int i = 0; i < NQ; ++i) {
            if (nkv[i] > 0) {
              issue_s(i, st);
              tc_commit(s_full + i);
            }
          }
          if (pending >= 0) tc_commit(stage_free + pending);
          if (nkv_max == 1) tc_commit(q_empty);  // the item's only S MMAs read Q
        }
        __syncwarp();
        pending = st;
        for (int j = 0; j < nkv_max; ++j) {
          next_use();  // V_j and K_{j+1}
          ok = vote_wait(stage_full + st, ph, kSiteMmaV);
          if (!ok) break;
          const bool next = j + 1 < nkv_max;
#pragma unroll
          for (int i = 0; i < NQ; ++i) {
            if (j < nkv[i]) {
              // The first P_i V of an item overwrites O_i: the previous item's
              // O_i must have been read out of tensor memory.
              if (j == 0 && (par >> (8 + i)) & 1u) {
                ok = vote_wait(o_empty + i, ((par >> (4 + i)) & 1u) ^ 1u, kSiteMmaO);
                if (!ok) break;
              }
              ok = vote_wait(p_full + 2 * i, (par >> i) & 1u, kSiteMmaP);
              if (!ok) break;
              tc_fence_after();
              if (elect_one()) {
                issue_pv(i, st, 0, j > 0);
                if (pending >= 0) tc_commit(stage_free + pending);
                // Keys 0-63 of the next S go to columns P_i does not occupy.
                if (C::SPLIT_S && next && j + 1 < nkv[i]) issue_s_half(i, st, 0);
              }
              __syncwarp();
              pending = -1;
              ok = vote_wait(p_full + 2 * i + 1, (par >> i) & 1u, kSiteMmaP);
              if (!ok) break;
              tc_fence_after();
              if (elect_one()) {
                issue_pv(i, st, 1, true);
                if (j + 1 == nkv[i]) tc_commit(o_full + i);  // O_i final
                if (next && j + 1 < nkv[i]) {
                  if (C::SPLIT_S)
                    issue_s_half(i, st, 1);  // keys 64-127 of S_i(j + 1), over P_i
                  else
                    issue_s(i, st);  // K_{j+1}
                  tc_commit(s_full + i);
                }
              }
              __syncwarp();
              par ^= 1u << i;
            }
          }
          if (!ok) break;
          if (j + 2 == nkv_max) {  // the item's last S MMAs were issued in this step
            if (elect_one()) tc_commit(q_empty);
            __syncwarp();
          }
          pending = st;
        }
#pragma unroll
        for (int i = 0; i < NQ; ++i)
          if (nkv[i] > 0) par = (par ^ (1u << (4 + i))) | (1u << (8 + i));
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
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_s = tmem + lane_off + wg * kBN;
    const uint32_t t_o = tmem + lane_off + C::O_COL + wg * D;
    int sc = 0, oc = 0;  // key steps and items of this tile so far (barrier phases)
    bool ok = true;
    for (int t = 0; ok && t < n_items; ++t) {
      int bh, qt0;
      item_coords<NQ>(p, item_of(t), bh, qt0);
      const int qt = qt0 + wg;
      const int n_i = kv_tiles_of(p, qt);
      if (n_i == 0) continue;
      const int q_row = qt * kBM + row;
      float m = -INFINITY;  // running max, log2 units
      float l = 0.f;        // running sum of 2^(x - m)
      for (int j = 0; j < n_i; ++j, ++sc) {
            ok = mbar_wait(s_full + wg, sc & 1, abort_flag, p.status, kSiteSoftS, p.timeout_ns);
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
            tmem_st32<0>(t_s + C::P_COL, sr);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full + 2 * wg);
#pragma unroll
            for (int c = kBN / 4; c < kBN / 2; ++c) exp_pair(c);
            tmem_st32<32>(t_s + C::P_COL + 32, sr);
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
      if (!ok) break;
      ok = mbar_wait(o_full + wg, oc & 1, abort_flag, p.status, kSiteEpilogue, p.timeout_ns);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      item_coords<NQ>(p, item_of(t), bh, qt0);
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
      // O_i is read out: the MMA warp may start the next item's P_i V.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_empty + wg);
      ++oc;
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

// Cost of an item in the list schedule: its tile-key steps (each query tile's
// key tiles) plus one for the per-item work around them.
int item_cost(const TcParams& p, int qt0, int nq) {
  int c = 1;
  for (int i = 0; i < nq; ++i) {
    const int qt = qt0 + i;
    c += kv_tiles_of(p, qt);
  }
  return c;
}

// List schedule of the items, in item order, over `ctas` persistent CTAs:
// each item goes to the CTA that becomes free first by the cost model (ties
// to the lowest index), which is the order in which the hardware would start
// one CTA per item, without the per-CTA start-up and wind-down. Returns the
// packed table of TcArgs::sched (ctas + 1 offsets, then the item lists), or
// an empty vector if it does not fit `cap` entries. Cached per shape.
template <int NQ>
std::vector<uint16_t> list_schedule(const TcParams& p, int ctas, int cap) {
  const int items = p.bh * p.n_cta_tiles;
  if (items + ctas + 1 > cap || items > 65535) return {};
  using Key = std::tuple<int, int, int, int, int, int>;
  static std::mutex mu;
  static std::map<Key, std::vector<uint16_t>> cache;
  const Key key{p.bh, p.n, p.causal, ctas, NQ, cap};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  using Slot = std::pair<long long, int>;  // (time the CTA becomes free, CTA)
  std::priority_queue<Slot, std::vector<Slot>, std::greater<Slot>> free_at;
  for (int c = 0; c < ctas; ++c) free_at.push({0, c});
  std::vector<std::vector<uint16_t>> lists(ctas);
  for (int r = 0; r < items; ++r) {
    int bh, qt0;
    item_coords<NQ>(p, r, bh, qt0);
    Slot s = free_at.top();
    free_at.pop();
    lists[s.second].push_back(static_cast<uint16_t>(r));
    s.first += item_cost(p, qt0, NQ);
    free_at.push(s);
  }
  std::vector<uint16_t> table(ctas + 1 + items);
  int off = 0;
  for (int c = 0; c < ctas; ++c) {
    table[c] = static_cast<uint16_t>(off);
    for (uint16_t r : lists[c]) table[ctas + 1 + off++] = r;
  }
  table[ctas] = static_cast<uint16_t>(off);
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() >= 64) cache.clear();
  cache.emplace(key, table);
  return table;
}

template <int D, int NQ, int CAP>
cudaError_t launch_tc_sched(const TcParams& prm, const std::vector<uint16_t>& table, int ctas,
                            const LaunchCtx& ctx) {
  using C = TcCfg<D, NQ>;
  static_assert(sizeof(TcArgs<CAP>) <= 32764, "kernel parameters are limited to 32764 bytes");
  auto kern = flash_tc_kernel<D, NQ, CAP>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    C::SMEM_ALLOC);
  });
  if (attr_err != cudaSuccess) return attr_err;
  TcArgs<CAP> args;
  args.p = prm;
  args.sched_ctas = table.empty() ? 0 : ctas;
  std::copy(table.begin(), table.end(), args.sched);
  const unsigned grid =
      table.empty() ? static_cast<unsigned>(prm.bh * prm.n_cta_tiles) : static_cast<unsigned>(ctas);
  kern<<<grid, C::THREADS, C::SMEM_ALLOC, ctx.stream>>>(args);
  return cudaGetLastError();
}

// Sequences up to this many CTA rows of query tiles (8192 tokens) run
// persistent: their items are short, so the start-up and wind-down of a CTA
// per item weigh (measured on B200: +4 % at 4096 tokens, +8-15 % at 512-1024);
// longer items keep one CTA per item (config 3's 32768 tokens: 2 % faster so).
constexpr int kPersistentMaxRows = 32;

// Persistent launch: one CTA per SM walking its items of the list schedule
// (kernel parameters of 4 KB or 32 KB); one CTA per item when the schedule
// does not fit, the sequence is long, or there are no more items than SMs.
template <int D, int NQ>
cudaError_t launch_tc(const TcParams& prm, const LaunchCtx& ctx) {
  const int items = prm.bh * prm.n_cta_tiles;
  const int ctas = std::min(items, ctx.sm_count);
  if (items > ctas && prm.n_cta_tiles <= kPersistentMaxRows) {
    std::vector<uint16_t> t = list_schedule<NQ>(prm, ctas, kSchedSmall);
    if (!t.empty()) return launch_tc_sched<D, NQ, kSchedSmall>(prm, t, ctas, ctx);
    t = list_schedule<NQ>(prm, ctas, kSchedLarge);
    if (!t.empty()) return launch_tc_sched<D, NQ, kSchedLarge>(prm, t, ctas, ctx);
  }
  return launch_tc_sched<D, NQ, kSchedSmall>(prm, {}, ctas, ctx);
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
  if (d == 64) return launch_tc<64, kNQ>(prm, ctx);
  return launch_tc<128, kNQ>(prm, ctx);
}

cudaError_t launch_selftest_exp2(const float* x, float* y_poly, float* y_mufu, float* y_lib,
                                int64_t n, const LaunchCtx& ctx) {
  const int64_t pairs = (n + 1) / 2;
  const unsigned grid = static_cast<unsigned>((pairs + 255) / 256);
  exp2_selftest_kernel<<<grid, 256, 0, ctx.stream>>>(x, y_poly, y_mufu, y_lib, n);
  return cudaGetLastError();
}

}  // namespace fab
