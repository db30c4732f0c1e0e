// Tree-masked GQA verify attention on tcgen05 tensor cores (sm_100a).
//
// Replaces the verify-forward attention of the reference: transformers'
// sdpa_attention_forward (integrations/sdpa_attention.py:40-103) calling
// scaled_dot_product_attention with the dense additive mask built by
// compile_ddtree_tree (ddtree.py:262-264).  Instead of an [N, P+N] mask the kernel
// reads per-node ancestor bitmasks: every prefix key is visible, tree key j is visible
// to node i iff bit j of anc_bits[i] is set.
//
// Work unit (one CTA): one KV head, two tiles of 128 query rows (256 rows), one key
// split.  Query rows are (node, q head of the GQA group) pairs, node-major, so the whole
// group shares every K/V tile.  Warp roles (12 warps, 3 warpgroups):
//   warp 0      TMA producer: both Q tiles once, then K and V tiles (128 keys x 128 dims,
//               128-byte swizzle) into a 2-stage ring; never multicast.
//   warp 1      allocates all 512 TMEM columns; one thread issues tcgen05.mma:
//               S_q = Q_q K^T (SMEM x SMEM) and O_q += P_q V with P_q read from TMEM.
//   warps 2-3   idle (they complete warpgroup 0, which gives its registers away)
//   warps 4-7   softmax of query tile 0, warps 8-11 of query tile 1: thread t of a warp
//               owns row 32 * (warp % 4) + t (the TMEM lane quarter of the warp).  Pass 1 loads the S row and takes the masked max; pass 2
//               reloads it, computes P = exp2(S * scale - m) and writes P back as packed
//               bf16 into the first 64 columns of the tile's S region, where the P V MMA
//               reads it.  O is rescaled in TMEM only when the row max grew by > 2^8.
// The two softmax warpgroups work on different query tiles, so while one computes
// exponentials the tensor pipe runs the other's MMAs.
// TMEM columns: S0/P0 [0,128) O0 [128,256) S1/P1 [256,384) O1 [384,512).
// Splits of the key range write fp32 partials (O, m, l) that ddt_attn_merge combines;
// the same partial format is exchanged between GPUs for sequence-sharded prefixes.
// Every mbarrier wait is bounded; a timeout sets *status and unwinds the CTA.  Every
// tcgen05.ld / st / wait is executed by whole warps.
#include <cuda.h>
#include <cuda_bf16.h>

#include "common.cuh"
#include "peer.cuh"
#include "tc.cuh"

namespace ddt {
namespace attn {

constexpr int kBlockM = 128;
constexpr int kBlockN = 128;
constexpr int kHeadDim = 128;
constexpr int kStages = 2;
constexpr int kThreads = 384;
// Register split (setmaxnreg): the launch gives every thread 168 registers (3 warps per SM
// sub-partition share its 16K-entry file); warpgroup 0 (TMA, MMA, 2 idle warps) gives
// back down to 64 and the two softmax warpgroups take 216:
// 128 * 64 + 256 * 216 = 63488 <= 384 * 168.  (Measured against 56 / 224: the same
// schedule ran 52.0 against 52.5 us at the Qwen3-8B verify shape.)
constexpr int kRegsLaunch = 168;
constexpr int kRegsControl = 64;
constexpr int kRegsSoftmax = 216;
static_assert(128 * kRegsControl + 256 * kRegsSoftmax <= kThreads * kRegsLaunch,
              "register split exceeds the launch's registers");
constexpr int kRowsPerCta = 2 * kBlockM;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.0f;
constexpr uint64_t kTimeoutNs = 2000000000ull;
constexpr uint32_t kHalfBytes = kBlockM * 64 * 2;   // one 64-dim half of a 128-row tile
constexpr uint32_t kTileBytes = 2 * kHalfBytes;     // 32 KB
constexpr uint32_t kSmemQ = 0;                      // Q0, Q1
constexpr uint32_t kSmemK = kSmemQ + 2 * kTileBytes;
constexpr uint32_t kSmemV = kSmemK + kStages * kTileBytes;
constexpr uint32_t kSmemBytes = kSmemV + kStages * kTileBytes;  // 192 KB
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;               // + alignment slack
constexpr uint32_t kIdescS = tc::idesc_bf16_f32(kBlockM, kBlockN, false, false);
constexpr uint32_t kIdescPV = tc::idesc_bf16_f32(kBlockM, kHeadDim, false, true);
constexpr int kStatusTimeout = 1;
// a launch with a device-side prefix length found it outside [0, planned prefix]: it ran with
// the planned length instead (every access stays in bounds; the output is not meaningful)
constexpr int kStatusPastRange = 4;
// Pairs (of the 16 in each 32-column chunk of an S row) whose exponentials are computed by
// the FMA-pipe polynomial instead of MUFU: pairs 0, 3, 6, 9 and 12, 10 of every 32
// exponentials.  Measured per-CTA cycles against MUFU alone: -10% (prefix 8192, 257 rows),
// -14% (prefix 131072); 3, 4, 6 and 8 pairs were slower than 5.  (With the MMAs issued from a
// lone lane this offload did not pay: the FMA-bound softmax warps starved that lane.)
#ifndef DDT_POLY_PAIRS
#define DDT_POLY_PAIRS 0x1249u
#endif
constexpr uint32_t kPolyPairs = DDT_POLY_PAIRS;
// TMEM column of query tile q's S/P region and O accumulator
__device__ __forceinline__ uint32_t col_s(int q) { return q ? 256u : 0u; }
__device__ __forceinline__ uint32_t col_o(int q) { return q ? 384u : 128u; }

struct Params {
  int n_nodes, past_len, group, q_heads, n_pairs, n_splits;
  int balanced;        // 1: work items from the Sched table, partials in per-part slots
  int key_base;        // global key index of local key 0
  int key_lo, key_hi;  // global key range covered by this launch
  const uint32_t* anc;
  int anc_words, mask_mode;
  float scale_log2;
  __nv_bfloat16* out;
  long long o_node_stride, o_head_stride;
  float* o_part;  // uniform splits: [n_splits][n_nodes * q_heads][128]
  // balanced parts: O / l of each part in bf16, [slot][dim / 8][unit row][8]
  __nv_bfloat16* o_slot;
  float* m_part;  // [n_splits][n_nodes * q_heads] or [slot][unit row]
  float* l_part;
  int partial;
  int* status;
  // limit of every bounded wait of the kernel (2 s in the product entry points)
  unsigned long long timeout_ns;
  // diagnostic launches only (ddt_tree_attn_wait_check): the producer issues no load, so the
  // first wait of every consumer runs out after timeout_ns and the kernel unwinds
  int withhold_loads;
  // ddt_tree_attn_device_past: the live prefix length, read by the kernel (past_len is then
  // the planned maximum: the schedule, the tile counts and the tensor maps cover past_len +
  // n_nodes keys, and keys at or beyond live + node + 1 are masked); null otherwise
  const int64_t* past_dev;
};

// Balanced schedule ("stream-K" over the key tiles): the flattened (work unit, key tile)
// space is cut into equal contiguous ranges, one per CTA, so every SM runs the same number of
// tiles whatever the number of work units.  A CTA's range may cover the end of one unit and
// the start of the next: each such piece is one item, whose partial (O / l in bf16, m and l
// in fp32) goes to its own slot; the parts of a unit have consecutive slots, starting at
// unit_slot[unit].  Built on the host and passed by value (kernel parameter space).
constexpr int kMaxCtas = 148;
constexpr int kMaxItems = 320;
constexpr int kMaxUnits = 256;
constexpr int kMaxPartsPerUnit = 32;  // merge_slots_kernel keeps one weight per part
// The balanced cut staggers the key positions that the row pairs of a head read at a time.
// That costs nothing while the launch's K / V stay in L2, but K / V much larger than L2 are
// then read from HBM once per row pair; uniform splits keep the pairs in step (each K / V
// tile read once and shared through L2).  Balanced only below this many K / V bytes.
constexpr int64_t kBalancedMaxKvBytes = 64ll << 20;
inline bool kv_fits_l2(int64_t keys, int64_t kv_heads) {
  return 2 * kv_heads * keys * kHeadDim * 2 <= kBalancedMaxKvBytes;
}
struct SchedItem {
  uint16_t unit, t0, nt, slot;  // work unit, first key tile of the unit, tiles, partial slot
};
struct Sched {
  uint16_t cta_first[kMaxCtas + 1];  // items of CTA c: [cta_first[c], cta_first[c + 1])
  SchedItem items[kMaxItems];
};
struct SlotTable {
  uint16_t unit_slot[kMaxUnits + 1];  // parts of unit u: slots [unit_slot[u], unit_slot[u + 1])
};

// Rows, key range and tile count of work unit u (one KV head, 256 query rows); shared by
// the host schedule and the kernel.
struct UnitGeo {
  int h, row0, g_end, ntot;
};
// `past` is the prefix length the mask uses: p.past_len, or the live length of a device-past
// launch (its tile count ntot then still covers the planned p.past_len).
__host__ __device__ inline UnitGeo unit_geo(const Params& p, int u, int past) {
  UnitGeo g;
  g.h = u / p.n_pairs;
  g.row0 = (u % p.n_pairs) * kRowsPerCta;
  int node_hi = (g.row0 + kRowsPerCta - 1) / p.group;
  if (node_hi > p.n_nodes - 1) node_hi = p.n_nodes - 1;
  // keys beyond past + node_hi are invisible to every row of the unit (tree and causal
  // masks); without a mask every row sees every key
  const int plan_end = p.mask_mode == DDT_MASK_NONE ? p.key_hi : p.past_len + node_hi + 1;
  g.g_end = p.mask_mode == DDT_MASK_NONE ? p.key_hi : past + node_hi + 1;
  if (g.g_end > p.key_hi) g.g_end = p.key_hi;
  g.ntot = plan_end > p.key_lo
               ? ((plan_end < p.key_hi ? plan_end : p.key_hi) - p.key_lo + kBlockN - 1) / kBlockN
               : 0;
  return g;
}
__host__ __device__ inline UnitGeo unit_geo(const Params& p, int u) {
  return unit_geo(p, u, p.past_len);
}

struct Bars {
  // K and V stages are released separately: K_j once both S_q(j) MMAs completed, V_j once
  // both P V MMAs of tile j completed, so the next K load starts a full tile earlier.
  // q_empty: both S MMAs of an item's last tile are done, Q may be replaced.
  uint64_t q_full, q_empty, k_full[kStages], v_full[kStages], k_empty[kStages],
      v_empty[kStages], s_full[2], p_half[2], p_full[2], o_ready[2], mma_done[2];
  // MMA blocks issued per query tile (S_q(0), then P V(j) + S(j + 1) per tile): the two
  // issuers take turns, tile 0 then tile 1, so the two softmax warpgroups stay half a
  // period apart instead of competing for the same SM sub-partitions
  uint32_t issued[2];
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void raise_abort(Bars& b, int* status) {
  *reinterpret_cast<volatile int*>(&b.abort) = 1;
  if (status) atomicOr(status, kStatusTimeout);
}

// Visibility mask of 32 consecutive keys starting at global key g0 for one node.
__device__ __forceinline__ uint32_t visible32(const Params& p, int node, int g0, int g_end,
                                              int past) {
  uint32_t m = 0xffffffffu;
  // keys at or beyond g_end (other shard / past the window) are invisible
  const int n_ok = g_end - g0;
  if (n_ok <= 0) return 0u;
  if (n_ok < 32) m = (1u << n_ok) - 1u;
  if (p.mask_mode == DDT_MASK_NONE) return m;
  if (p.mask_mode == DDT_MASK_CAUSAL) {
    const int lim = past + node + 1 - g0;  // keys < lim visible
    if (lim <= 0) return 0u;
    if (lim < 32) m &= (1u << lim) - 1u;
    return m;
  }
  const int o0 = g0 - past;  // tree offset of the first key
  if (o0 + 32 <= 0) return m;      // all prefix
  uint32_t tree;
  const uint32_t* row = p.anc + static_cast<long long>(node) * p.anc_words;
  if (o0 >= 0) {
    const int w = o0 >> 5, b = o0 & 31;
    const uint32_t lo = (w < p.anc_words) ? __ldg(row + w) : 0u;
    const uint32_t hi = (b && w + 1 < p.anc_words) ? __ldg(row + w + 1) : 0u;
    tree = b ? __funnelshift_r(lo, hi, b) : lo;
  } else {
    // keys [g0, past) are prefix (visible); tree bits start at bit -o0
    const int sh = -o0;
    const uint32_t w0 = p.anc_words > 0 ? __ldg(row) : 0u;
    tree = (w0 << sh) | ((1u << sh) - 1u);
  }
  return m & tree;
}

template <bool kLivePast>
__global__ void __launch_bounds__(kThreads, 1)
tree_attn_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ Params p,
                 const __grid_constant__ Sched sched) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ Bars bars;
  const uint32_t raw = tc::smem_u32(smem_raw);
  unsigned char* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rows = p.n_nodes * p.group;

  // ---- work items of this CTA ----------------------------------------------------------
  // uniform splits: one item, (unit, split) from blockIdx.x; balanced: the Sched table.
  // Barrier phases run on the CTA-wide tile count, across items.
  const int item_lo = p.balanced ? sched.cta_first[blockIdx.x] : 0;
  const int n_items = p.balanced ? sched.cta_first[blockIdx.x + 1] - item_lo : 1;
  auto item = [&](int i, int& u, int& t0, int& nt, int& slot) {
    if (p.balanced) {
      const SchedItem it = sched.items[item_lo + i];
      u = it.unit;
      t0 = it.t0;
      nt = it.nt;
      slot = it.slot;
    } else {
      const int split = blockIdx.x % p.n_splits;
      u = blockIdx.x / p.n_splits;
      slot = split;
      const int ntot = unit_geo(p, u).ntot;
      const int tps = (ntot + p.n_splits - 1) / p.n_splits;
      t0 = split * tps < ntot ? split * tps : ntot;
      nt = (t0 + tps < ntot ? t0 + tps : ntot) - t0;
    }
  };
  int total = 0;
  for (int i = 0; i < n_items; ++i) {
    int u, t0, nt, sl;
    item(i, u, t0, nt, sl);
    total += nt;
  }

  if (tid == 0) {
    tc::mbar_init(&bars.q_full, 1);
    tc::mbar_init(&bars.q_empty, 2);  // one commit per MMA issuer
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&bars.k_full[s], 1);
      tc::mbar_init(&bars.v_full[s], 1);
      tc::mbar_init(&bars.k_empty[s], 2);
      tc::mbar_init(&bars.v_empty[s], 2);
    }
    for (int q = 0; q < 2; ++q) {
      tc::mbar_init(&bars.s_full[q], 1);
      tc::mbar_init(&bars.p_half[q], 4);  // one arrive per softmax warp
      tc::mbar_init(&bars.p_full[q], 4);
      bars.issued[q] = 0;
      tc::mbar_init(&bars.o_ready[q], 1);
      tc::mbar_init(&bars.mma_done[q], 1);
    }
    bars.abort = 0;
    tc::fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(&bars.tmem_base, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = bars.tmem_base;
  volatile int* abort_flag = &bars.abort;

  unsigned char* sQ = smem + kSmemQ;
  unsigned char* sK = smem + kSmemK;
  unsigned char* sV = smem + kSmemV;

  if (warp < 4) {
    tc::reg_dealloc<kRegsControl>();
    if (warp == 0) {
      // ---------------------------- TMA producer -------------------------------------
      if (lane == 0 && total > 0 && !p.withhold_loads) {
        tc::tma_prefetch_desc(&tm_q);
        tc::tma_prefetch_desc(&tm_k);
        tc::tma_prefetch_desc(&tm_v);
        // both query tiles of a unit; the second one of a unit's last row pair may lie
        // past the last node, where the load reads zeros and its rows are not stored
        int q_loads = 0;
        auto load_q = [&](const UnitGeo& g) {
          tc::mbar_expect_tx(&bars.q_full, 2 * kTileBytes);
          for (int q = 0; q < 2; ++q) {
            const int node0 = (g.row0 + q * kBlockM) / p.group;
            tc::tma_load_3d(sQ + q * kTileBytes, &tm_q, &bars.q_full, 0, g.h * p.group, node0);
            tc::tma_load_3d(sQ + q * kTileBytes + kHalfBytes, &tm_q, &bars.q_full, 64,
                            g.h * p.group, node0);
          }
          ++q_loads;
        };
        int issued_k = 0, issued_v = 0, J = 0;
        bool ok = true;
        for (int i = 0; ok && i < n_items; ++i) {
          int u, t0, nt, sl;
          item(i, u, t0, nt, sl);
          const UnitGeo g = unit_geo(p, u);
          const int lk0 = p.key_lo - p.key_base + t0 * kBlockN;  // local key of the first tile
          if (i == 0) load_q(g);
          for (int j = 0; j < nt; ++j) {
            const int jg = J + j;
            const int st = jg % kStages;
            const uint32_t ph = ((jg / kStages) - 1) & 1;  // release phase of tile jg - kStages
            const int key = lk0 + j * kBlockN;
            if (jg >= kStages && !(ok = tc::mbar_wait(&bars.k_empty[st], ph, abort_flag, p.timeout_ns)))
              break;
            unsigned char* kd = sK + st * kTileBytes;
            tc::mbar_expect_tx(&bars.k_full[st], kTileBytes);
            tc::tma_load_3d(kd, &tm_k, &bars.k_full[st], 0, key, g.h);
            tc::tma_load_3d(kd + kHalfBytes, &tm_k, &bars.k_full[st], 64, key, g.h);
            issued_k = jg + 1;
            if (jg >= kStages && !(ok = tc::mbar_wait(&bars.v_empty[st], ph, abort_flag, p.timeout_ns)))
              break;
            unsigned char* vd = sV + st * kTileBytes;
            tc::mbar_expect_tx(&bars.v_full[st], kTileBytes);
            tc::tma_load_3d(vd, &tm_v, &bars.v_full[st], 0, key, g.h);
            tc::tma_load_3d(vd + kHalfBytes, &tm_v, &bars.v_full[st], 64, key, g.h);
            issued_v = jg + 1;
            if (j == 0 && i > 0) {
              // the item's Q replaces the previous item's once both its S MMAs are done;
              // the first K / V tile of the item is already on its way
              if (!(ok = tc::mbar_wait(&bars.q_empty, (i - 1) & 1, abort_flag, p.timeout_ns))) break;
              load_q(g);
            }
          }
          J += nt;
        }
        if (!ok) raise_abort(bars, p.status);
        if (*abort_flag) {
          // let the loads already in flight land before the CTA releases its smem
          if (q_loads > 0) tc::mbar_wait_drain(&bars.q_full, (q_loads - 1) & 1, kTimeoutNs);
          for (int j = issued_k > kStages ? issued_k - kStages : 0; j < issued_k; ++j)
            tc::mbar_wait_drain(&bars.k_full[j % kStages], (j / kStages) & 1, kTimeoutNs);
          for (int j = issued_v > kStages ? issued_v - kStages : 0; j < issued_v; ++j)
            tc::mbar_wait_drain(&bars.v_full[j % kStages], (j / kStages) & 1, kTimeoutNs);
        }
      }
    } else if (warp == 1 || warp == 3) {
      // ---------------------------- MMA issuers, one per query tile ------------------
      // Query tile 0's MMAs come from warp 1, tile 1's from warp 3.  An mbarrier wait (or
      // any acquire) holds the waiting thread until its own MMAs in flight have drained
      // (measured ~180 cycles of idle tensor pipe per wait with a single issuer).  With one
      // issuer per tile every wait falls where that tile's previous MMAs are complete anyway
      // (P_q(j) ready implies S_q(j) done), while the other tile's MMAs keep the pipe busy.
      // The whole warp runs the loop (uniform control flow, warp-collective waits) and one
      // elected lane issues: a lone lane in a divergent branch issued one MMA per ~130
      // cycles next to FMA-bound softmax warps on its sub-partition (measured), against
      // the pipe's 64.
      const int q = warp == 1 ? 0 : 1;
      if (total > 0) {
        // descriptor low words of the Q, K and V tiles; every MMA adds a constant to them
        constexpr uint32_t kDescHi = tc::desc_sw128_hi(1024);
        const uint32_t a_q = tc::desc_sw128_lo(tc::smem_u32(sQ), 16) + q * (kTileBytes >> 4);
        const uint32_t k_lo = tc::desc_sw128_lo(tc::smem_u32(sK), 16);
        const uint32_t v_lo = tc::desc_sw128_lo(tc::smem_u32(sV), kHalfBytes);
        const uint32_t d_s = tmem + col_s(q), d_o = tmem + col_o(q);
        volatile uint32_t* my_turns = &bars.issued[q];
        const volatile uint32_t* other_turns = &bars.issued[q ^ 1];
        // S_q = Q_q K^T of CTA tile jg into the S region of query tile q; the block's turn
        // count `turn` is published right after its last MMA.  (Publishing it after half of
        // the S MMAs, so the other issuer's block would queue behind this one, measured
        // 5% slower: the two softmax warpgroups drift into each other.)
        auto issue_s = [&](int jg, uint32_t turn) {
          const uint32_t b = k_lo + (jg % kStages) * (kTileBytes >> 4);
          tc::mma_bf16_ss_w<0>(d_s, a_q, b, kDescHi, kIdescS);
#pragma unroll
          for (int kk = 1; kk < kHeadDim / 16; ++kk) {
            const uint32_t off = ((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4;
            tc::mma_bf16_ss_w<1>(d_s, a_q + off, b + off, kDescHi, kIdescS);
            if (kk == kHeadDim / 16 - 1) *my_turns = turn;
          }
          tc::mma_commit(&bars.s_full[q]);
        };
        // O_q += P_q V of tile jg (item tile j; j == 0 starts the item's O), P_q in TMEM
        // (first 64 columns of the S region, 8 per K step), in two halves of 64 keys: the
        // first runs while the softmax computes the second
        auto issue_pv = [&](int jg, int j, int half) {
          const uint32_t b = v_lo + (jg % kStages) * (kTileBytes >> 4);
#pragma unroll
          for (int k4 = 0; k4 < kBlockN / 32; ++k4) {
            const int kk = half * (kBlockN / 32) + k4;
            tc::mma_bf16_ts_w(d_o, d_s + kk * 8, b + ((kk * 2048) >> 4), kDescHi, kIdescPV,
                              (j > 0 || kk > 0) ? 1u : 0u);
          }
          if (half) tc::mma_commit(&bars.o_ready[q]);
        };
        // Turn-taking on plain (volatile) loads and stores: an acquire or release here
        // would wait for this thread's MMAs in flight, and the turns order only the issue
        // of the two tiles' MMAs, no data.  Blocks per item: S of its first tile, then one
        // per tile (P V(j) + S(j + 1)); `base` counts the blocks of earlier items.
        auto wait_turn = [&](uint32_t target) {
          uint64_t t0 = 0;
          for (uint32_t it = 0;; ++it) {
            if (__all_sync(DDT_FULL_MASK, *other_turns >= target)) return true;
            if ((it & 255u) == 255u) {
              const uint64_t now = global_timer_ns();
              if (t0 == 0) t0 = now;
              if (__any_sync(DDT_FULL_MASK, *abort_flag != 0 || now - t0 > p.timeout_ns))
                return false;
            }
          }
        };
        // stage releases (k_empty / v_empty count one commit per issuer) are committed
        // only where the producer will wait for them
        bool ok = true;
        uint32_t base = 0;
        int J = 0;
        for (int i = 0; ok && i < n_items; ++i) {
          int u, t0, nt, sl;
          item(i, u, t0, nt, sl);
          if (!(ok = tc::mbar_wait_warp(&bars.q_full, i & 1, abort_flag, p.timeout_ns))) break;
          if (!(ok = tc::mbar_wait_warp(&bars.k_full[J % kStages], (J / kStages) & 1, abort_flag,
                                        p.timeout_ns)))
            break;
          if (!(ok = wait_turn(q == 0 ? base : base + 1))) break;
          tc::tc_fence_after();
          if (tc::elect_one()) {
            issue_s(J, base + 1);
            if (J + kStages < total) tc::mma_commit(&bars.k_empty[J % kStages]);
          }
          __syncwarp();
          for (int j = 0; j < nt; ++j) {
            const int jg = J + j;
            const int st = jg % kStages;
            const int sn = (jg + 1) % kStages;
            const bool more = j + 1 < nt;
            // K / V of the tile landed long before P_q(j): waited first, while the softmax runs
            if (!(ok = tc::mbar_wait_warp(&bars.v_full[st], (jg / kStages) & 1, abort_flag,
                                          p.timeout_ns)))
              break;
            if (more && !(ok = tc::mbar_wait_warp(&bars.k_full[sn], ((jg + 1) / kStages) & 1,
                                                  abort_flag, p.timeout_ns)))
              break;
            if (!(ok = tc::mbar_wait_warp(&bars.p_half[q], jg & 1, abort_flag, p.timeout_ns))) break;
            if (!(ok = wait_turn(q == 0 ? base + j + 1 : base + j + 2))) break;
            tc::tc_fence_after();
            if (tc::elect_one()) issue_pv(jg, j, 0);
            __syncwarp();
            if (!(ok = tc::mbar_wait_warp(&bars.p_full[q], jg & 1, abort_flag, p.timeout_ns))) break;
            tc::tc_fence_after();
            if (tc::elect_one()) {
              issue_pv(jg, j, 1);
              if (jg + kStages < total) tc::mma_commit(&bars.v_empty[st]);
              if (more) {
                issue_s(jg + 1, base + j + 2);  // reuses S_q / P_q: runs after the P V above
                if (jg + 1 + kStages < total) tc::mma_commit(&bars.k_empty[sn]);
              } else {
                *my_turns = base + j + 2;
              }
            }
            __syncwarp();
          }
          // the item's S MMAs are all issued: Q may be replaced once they are done
          if (ok && i + 1 < n_items && tc::elect_one()) tc::mma_commit(&bars.q_empty);
          __syncwarp();
          base += nt + 1;
          J += nt;
        }
        if (!ok) {
          if (lane == 0) raise_abort(bars, p.status);
          // wait for every MMA this warp issued before TMEM is released
          if (tc::elect_one()) tc::mma_commit(&bars.mma_done[q]);
          __syncwarp();
          tc::mbar_wait_drain(&bars.mma_done[q], 0, kTimeoutNs);
        }
      }
    }
  } else {
    tc::reg_alloc<kRegsSoftmax>();
    // ---------------------------- softmax warpgroups -------------------------------
    const int q = (warp - 4) >> 2;  // query tile of this warpgroup (warps 4-7 / 8-11)
    const int wq = warp & 3;        // TMEM lane quarter a warp may access: warp id % 4
    const int r = wq * 32 + lane;
    const uint32_t tl = tmem + (static_cast<uint32_t>(wq * 32) << 16);
    const uint32_t tS = tl + col_s(q);
    const uint32_t tO = tl + col_o(q);
    const float sl2 = p.scale_log2;
    const tc::Exp2Poly exp2_poly;
    // the prefix length of the mask: the launch's, or the one in device memory (a value
    // outside [0, planned] is reported and replaced by the planned length)
    int past = p.past_len;
    if (kLivePast) {
      const int64_t live = *p.past_dev;
      if (live >= 0 && live <= p.past_len) past = static_cast<int>(live);
      else if (warp == 4 && lane == 0 && p.status) atomicOr(p.status, kStatusPastRange);
    }
    bool ok = true;
    int J = 0;
    for (int i = 0; i < n_items; ++i) {
      int u, t0, nt, slot;
      item(i, u, t0, nt, slot);
      const UnitGeo g = unit_geo(p, u, past);
      const int R = g.row0 + q * kBlockM + r;
      const int node = R / p.group;
      const int qh = g.h * p.group + (R % p.group);
      const bool valid = R < rows;
      const int vnode = valid ? node : p.n_nodes - 1;
      const int g_end = g.g_end;
      // the whole key range of the tile is visible to this row (no mask needed) when it
      // ends before the tree window / the launch's last key
      const int full_end = p.mask_mode == DDT_MASK_NONE ? g_end
                           : p.mask_mode == DDT_MASK_CAUSAL
                               ? (g_end < past + vnode + 1 ? g_end : past + vnode + 1)
                               : (g_end < past ? g_end : past);
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; ok && j < nt; ++j) {
        const int jg = J + j;
        if (!tc::mbar_wait_warp(&bars.s_full[q], jg & 1, abort_flag, p.timeout_ns)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const int gk = p.key_lo + (t0 + j) * kBlockN;  // global key of column 0
        const bool masked = __any_sync(DDT_FULL_MASK, gk + kBlockN > full_end);
        uint32_t vis[4] = {~0u, ~0u, ~0u, ~0u};
        if (masked) {
#pragma unroll
          for (int c = 0; c < 4; ++c) vis[c] = visible32(p, vnode, gk + c * 32, g_end, past);
        }
        // the whole S row (128 fp32) comes out of TMEM in one round trip
        uint32_t sv[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tc::tmem_ld32(tS + c * 32, sv[c]);
        tc::tmem_wait_ld();
        if (masked) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (!((vis[c] >> e) & 1u)) sv[c][e] = __float_as_uint(-INFINITY);
        }
        // masked row max of the raw scores: three-input maxima in 8 independent chains
        float mx8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mx8[k] = -INFINITY;
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; e += 2)
            mx8[(e >> 1) & 7] = tc::fmax3(mx8[(e >> 1) & 7], __uint_as_float(sv[c][e]),
                                          __uint_as_float(sv[c][e + 1]));
        const float mx = tc::fmax3(tc::fmax3(mx8[0], mx8[1], mx8[2]),
                                   tc::fmax3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
        bool rescale = false;
        float alpha = 1.f;
        if (mx > -INFINITY) {
          const float ms = mx * sl2;
          if (m_used == -INFINITY) {
            m_used = ms;  // nothing accumulated yet: O and l are zero
          } else if (ms > m_used + kRescaleLog2) {
            alpha = tc::ex2_approx(m_used - ms);
            m_used = ms;
            rescale = true;
          }
        }
        if (__any_sync(DDT_FULL_MASK, rescale)) {
          // O_q is stable once the previous P V MMA of this item completed
          if (j > 0 && !tc::mbar_wait_warp(&bars.o_ready[q], (jg - 1) & 1, abort_flag, p.timeout_ns)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tc::tmem_ld32(tO + c * 32, o);
            tc::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tc::tmem_st32(tO + c * 32, o);
          }
          l *= alpha;
        }
        const float nm = (m_used == -INFINITY) ? 0.f : -m_used;
        // P = exp2(S * scale - m), packed bf16 into columns [0, 64) of S_q (masked keys hold
        // -inf and give 0, or 2^-126 on the polynomial lanes).  Scale and row sum run on
        // packed fp32 pairs; the pairs selected by kPolyPairs take the polynomial
        // exponential, the rest the MUFU one.
        const uint64_t sl2x2 = tc::f2_pack(sl2, sl2), nmx2 = tc::f2_pack(nm, nm);
        uint64_t ls2[4] = {0ull, 0ull, 0ull, 0ull};
        // keys [0, 64) first: their P columns are stored and signalled (p_half) while the
        // second half is computed, so the first four P V MMAs overlap it
        uint32_t pk[2][32];
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const uint64_t x = tc::f2_fma(tc::f2_pack(__uint_as_float(sv[hf * 2 + c][e]),
                                                        __uint_as_float(sv[hf * 2 + c][e + 1])),
                                            sl2x2, nmx2);
              float a, b;
              if ((kPolyPairs >> (e >> 1)) & 1u) {
                exp2_poly(x, a, b);
              } else {
                float x0, x1;
                tc::f2_unpack(x, x0, x1);
                a = tc::ex2_approx(x0);
                b = tc::ex2_approx(x1);
              }
              ls2[(e >> 1) & 3] = tc::f2_add(ls2[(e >> 1) & 3], tc::f2_pack(a, b));
              pk[hf][c * 16 + e / 2] = tc::pack_bf16x2(a, b);
            }
          }
          if (hf == 0) tc::tmem_st32(tS, pk[0]);
        }
        tc::tmem_wait_st();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars.p_half[q]);
        tc::tmem_st32(tS + 32, pk[1]);
        float l0, l1, l2, l3;
        tc::f2_unpack(tc::f2_add(ls2[0], ls2[1]), l0, l1);
        tc::f2_unpack(tc::f2_add(ls2[2], ls2[3]), l2, l3);
        l += (l0 + l1) + (l2 + l3);
        tc::tmem_wait_st();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars.p_full[q]);
      }
      if (ok && nt > 0 &&
          !tc::mbar_wait_warp(&bars.o_ready[q], (J + nt - 1) & 1, abort_flag, p.timeout_ns))
        ok = false;
      const bool have = ok && nt > 0;  // warp-uniform
      if (have) tc::tc_fence_after();
      // ---- epilogue of the item ----------------------------------------------------------
      if (p.partial && p.balanced) {
        // the part's own slot: O / l in bf16 (a convex combination of V rows, so in V's
        // range), laid out [dim / 8][unit row][8]: the 32 lanes of a warp (consecutive rows)
        // store 512 contiguous bytes per instruction.  Half the bytes of fp32 O for the
        // merge to read; the merge weights each part by 2^(m - M) l.
        const int lr = q * kBlockM + r;
        const float inv = (have && l > 0.f) ? 1.f / l : 0.f;
        __nv_bfloat16* op =
            p.o_slot + static_cast<long long>(slot) * kRowsPerCta * kHeadDim + lr * 8;
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          if (have) {
            tc::tmem_ld32(tO + c * 32, o);
            tc::tmem_wait_ld();
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = 0u;
          }
          if (valid) {
#pragma unroll
            for (int e = 0; e < 32; e += 8) {
              uint4 v;
              v.x = tc::pack_bf16x2(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv);
              v.y = tc::pack_bf16x2(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
              v.z = tc::pack_bf16x2(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv);
              v.w = tc::pack_bf16x2(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv);
              *reinterpret_cast<uint4*>(op + ((c * 32 + e) / 8) * kRowsPerCta * 8) = v;
            }
          }
        }
        if (valid) {
          const long long mi = static_cast<long long>(slot) * kRowsPerCta + lr;
          p.m_part[mi] = have ? m_used : -INFINITY;
          p.l_part[mi] = have ? l : 0.f;
        }
      } else if (p.partial) {
        // uniform splits: split-major rows in (node, q head) order, the layout the
        // cross-GPU merge exchanges
        const long long orow_idx = static_cast<long long>(node) * p.q_heads + qh;
        const long long pi = static_cast<long long>(slot) * p.n_nodes * p.q_heads + orow_idx;
        float* op = p.o_part + pi * kHeadDim;
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          if (have) {
            tc::tmem_ld32(tO + c * 32, o);
            tc::tmem_wait_ld();
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = 0u;
          }
          if (valid) {
#pragma unroll
            for (int e = 0; e < 32; e += 4)
              *reinterpret_cast<float4*>(op + c * 32 + e) =
                  make_float4(__uint_as_float(o[e]), __uint_as_float(o[e + 1]),
                              __uint_as_float(o[e + 2]), __uint_as_float(o[e + 3]));
          }
        }
        if (valid) {
          p.m_part[pi] = have ? m_used : -INFINITY;
          p.l_part[pi] = have ? l : 0.f;
        }
      } else {
        const float inv = (have && l > 0.f) ? 1.f / l : 0.f;
        __nv_bfloat16* orow = p.out + static_cast<long long>(vnode) * p.o_node_stride +
                              static_cast<long long>(qh) * p.o_head_stride;
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          if (have) {
            tc::tmem_ld32(tO + c * 32, o);
            tc::tmem_wait_ld();
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = 0u;
          }
          if (valid) {
#pragma unroll
            for (int e = 0; e < 32; e += 8) {
              uint4 v;
              v.x = tc::pack_bf16x2(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv);
              v.y = tc::pack_bf16x2(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
              v.z = tc::pack_bf16x2(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv);
              v.w = tc::pack_bf16x2(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv);
              *reinterpret_cast<uint4*>(orow + c * 32 + e) = v;
            }
          }
        }
      }
      // the O columns are read: the next item's first P V MMA may overwrite them (it waits
      // for this warpgroup's p_half of that item, which comes after this point)
      tc::tc_fence_before();
      J += nt;
      if (!ok) break;
    }
    if (!ok && lane == 0) raise_abort(bars, p.status);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- split merge ---------------------------------------------------------------------
// One warp per (node, q head) row.  Lane i < parts loads part i's (m, l); the row max M
// and the weights exp2(m_i - M) come from warp shuffles, then every lane accumulates 4 of the
// 128 dims with all parts' loads in flight (a serial walk over the parts made the merge
// latency-bound).  Up to 32 parts per pass.
template <typename PartIndex>
__device__ __forceinline__ void merge_row(const float* __restrict__ o_parts,
                                          const float* __restrict__ m_parts,
                                          const float* __restrict__ l_parts, int n_parts,
                                          PartIndex part_index, int lane, float4& acc, float& M,
                                          float& L) {
  M = -INFINITY;
  L = 0.f;
  acc = make_float4(0.f, 0.f, 0.f, 0.f);
  constexpr int kFast = 8;
  if (n_parts <= kFast) {
    // one round trip: every part's (m, l) and O issued before any is used
    const long long pi = lane < n_parts ? part_index(lane) : 0;
    float4 ov[kFast];
#pragma unroll
    for (int k = 0; k < kFast; ++k) {
      const long long pk = __shfl_sync(DDT_FULL_MASK, pi, k);
      ov[k] = k < n_parts ? *reinterpret_cast<const float4*>(o_parts + pk * kHeadDim + lane * 4)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float mi = lane < n_parts ? m_parts[pi] : -INFINITY;
    const float li = lane < n_parts ? l_parts[pi] : 0.f;
    float mx = mi;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(DDT_FULL_MASK, mx, o));
    M = mx;
    if (M == -INFINITY) return;
    const float wi = mi == -INFINITY ? 0.f : exp2f(mi - M);
    float lw = wi * li;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lw += __shfl_xor_sync(DDT_FULL_MASK, lw, o);
    L = lw;
#pragma unroll
    for (int k = 0; k < kFast; ++k) {
      const float w = __shfl_sync(DDT_FULL_MASK, wi, k);  // 0 for k >= n_parts
      acc.x += w * ov[k].x;
      acc.y += w * ov[k].y;
      acc.z += w * ov[k].z;
      acc.w += w * ov[k].w;
    }
    return;
  }
  for (int base = 0; base < n_parts; base += 32) {
    const int cnt = n_parts - base < 32 ? n_parts - base : 32;
    const long long pi = lane < cnt ? part_index(base + lane) : 0;
    const float mi = lane < cnt ? m_parts[pi] : -INFINITY;
    const float li = lane < cnt ? l_parts[pi] : 0.f;
    float mx = mi;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(DDT_FULL_MASK, mx, o));
    const float Mn = fmaxf(M, mx);
    if (Mn == -INFINITY) continue;  // warp-uniform: nothing visible yet
    const float cs = M == -INFINITY ? 0.f : exp2f(M - Mn);  // rescale of the earlier passes
    acc.x *= cs;
    acc.y *= cs;
    acc.z *= cs;
    acc.w *= cs;
    L *= cs;
    M = Mn;
    const float wi = mi == -INFINITY ? 0.f : exp2f(mi - M);
    float lw = wi * li;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lw += __shfl_xor_sync(DDT_FULL_MASK, lw, o);
    L += lw;
    constexpr int kBatch = 8;
    for (int k0 = 0; k0 < cnt; k0 += kBatch) {
      float4 ov[kBatch];
      float wv[kBatch];
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const int kk = k0 + k < cnt ? k0 + k : cnt - 1;
        wv[k] = __shfl_sync(DDT_FULL_MASK, wi, kk);
        const long long pk = __shfl_sync(DDT_FULL_MASK, pi, kk);
        ov[k] = *reinterpret_cast<const float4*>(o_parts + pk * kHeadDim + lane * 4);
        if (k0 + k >= cnt) wv[k] = 0.f;
      }
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        acc.x += wv[k] * ov[k].x;
        acc.y += wv[k] * ov[k].y;
        acc.z += wv[k] * ov[k].z;
        acc.w += wv[k] * ov[k].w;
      }
    }
  }
}

// push.world > 0 (split-KV over NVLink peer memory): the merged partial goes to slot
// push.rank of every rank's receive buffer instead of o_merged / m_merged / l_merged, and the
// grid's last CTA (ticket), after a system-scope fence, bumps counter push.rank in each.
__global__ void merge_kernel(const float* __restrict__ o_parts, const float* __restrict__ m_parts,
                             const float* __restrict__ l_parts, int n_parts, long long rows,
                             int q_heads, __nv_bfloat16* __restrict__ out, long long o_node_stride,
                             long long o_head_stride, float* __restrict__ o_merged,
                             float* __restrict__ m_merged, float* __restrict__ l_merged,
                             const __grid_constant__ peer::Push push) {
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row < rows) {  // warp-uniform
    float4 acc;
    float M, L;
    merge_row(o_parts, m_parts, l_parts, n_parts,
              [&](int i) { return static_cast<long long>(i) * rows + row; }, lane, acc, M, L);
    if (out) {
      const float inv = L > 0.f ? 1.f / L : 0.f;
      const long long node = row / q_heads, qh = row % q_heads;
      __nv_bfloat16* orow = out + node * o_node_stride + qh * o_head_stride + lane * 4;
      uint2 v;
      v.x = tc::pack_bf16x2(acc.x * inv, acc.y * inv);
      v.y = tc::pack_bf16x2(acc.z * inv, acc.w * inv);
      *reinterpret_cast<uint2*>(orow) = v;
    } else if (push.world > 0) {
      const long long slot = static_cast<long long>(push.rank) * rows + row;
      for (int w = 0; w < push.world; ++w) {
        reinterpret_cast<float4*>(push.base[w] + push.o_off)[slot * (kHeadDim / 4) + lane] = acc;
        if (lane == 0) {
          reinterpret_cast<float*>(push.base[w] + push.m_off)[slot] = M;
          reinterpret_cast<float*>(push.base[w] + push.l_off)[slot] = L;
        }
      }
    } else {
      *reinterpret_cast<float4*>(o_merged + row * kHeadDim + lane * 4) = acc;
      if (lane == 0) {
        m_merged[row] = M;
        l_merged[row] = L;
      }
    }
  }
  if (push.world > 0) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned int t = atomicAdd(push.ticket, 1u);
      if (t == gridDim.x - 1) {
        __threadfence_system();
        for (int w = 0; w < push.world; ++w)
          atomicAdd_system(reinterpret_cast<unsigned int*>(push.base[w]) + push.rank, 1u);
        atomicExch(push.ticket, 0u);
      }
    }
  }
}

// ---- merge of balanced parts -------------------------------------------------------------
// One warp per (work unit, 32 consecutive unit rows, 16 of the 128 dims), one lane per row;
// the unit's parts are slots [unit_slot[u], unit_slot[u + 1]), each holding that part's
// O / l in bf16 laid out [dim / 8][unit row][8] and its m, l per unit row, so a warp's loads
// are 512 (O) or 128 (m, l) contiguous bytes.  Part i has weight 2^(m_i - M) l_i, computed
// once for the lane's 16 dims.  Batches of 6 parts with every load in flight and an online
// maximum (earlier batches rescaled when it grows): one L2 round trip for the ~5 parts of a
// unit at the Qwen3-8B verify shape.  96 registers and 2-warp blocks keep the grid one wave.
// (One warp per 8 dims with full-precision exp2f issued 2.8 M instructions at that shape and
// was instruction-bound: 7.7 us, measured; 32 dims per warp in batches of 4 took 5.2 us.)
// kFp32: write the merged partial (O un-normalised, m, l) in (node, q head) row order, the
// cross-GPU exchange format, instead of the bf16 output.
constexpr int kMergeBatch = 6;
constexpr int kMergeDims = 16;
constexpr int kMergeVecs = kMergeDims / 8;  // 16-byte loads per part and lane
constexpr int kMergeWarps = 2;              // warps per block
template <bool kFp32>
__global__ void __launch_bounds__(kMergeWarps * 32, 9)
merge_slots_kernel(const __nv_bfloat16* __restrict__ o_parts, const float* __restrict__ m_parts,
                   const float* __restrict__ l_parts, const __grid_constant__ SlotTable tab,
                   const Params p, __nv_bfloat16* __restrict__ out, long long o_node_stride,
                   long long o_head_stride, float* __restrict__ o_merged,
                   float* __restrict__ m_merged, float* __restrict__ l_merged) {
  constexpr int kRowGroups = kRowsPerCta / 32, kDimGroups = kHeadDim / kMergeDims;
  const int gw = blockIdx.x * kMergeWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int u = gw / (kRowGroups * kDimGroups);
  if (u >= p.n_pairs * (p.q_heads / p.group)) return;
  const int rg = (gw / kDimGroups) % kRowGroups, dq = gw % kDimGroups;
  const int lr = rg * 32 + lane;
  const int R = (u % p.n_pairs) * kRowsPerCta + lr;
  const int rows = p.n_nodes * p.group;
  if (R >= rows) return;
  const int s0 = tab.unit_slot[u], n = tab.unit_slot[u + 1] - s0;
  // the lane's dims of part slot sl: loads of 8 dims, kRowsPerCta * 8 elements apart
  const __nv_bfloat16* obase =
      o_parts + static_cast<long long>(dq) * kMergeVecs * kRowsPerCta * 8 + lr * 8;
  constexpr long long kSlotElems = static_cast<long long>(kRowsPerCta) * kHeadDim;
  float M = -INFINITY, L = 0.f;
  float a[kMergeDims];
#pragma unroll
  for (int d = 0; d < kMergeDims; ++d) a[d] = 0.f;
  for (int k0 = 0; k0 < n; k0 += kMergeBatch) {
    float mv[kMergeBatch], lv[kMergeBatch];
    uint4 ov[kMergeBatch][kMergeVecs];
#pragma unroll
    for (int k = 0; k < kMergeBatch; ++k) {
      const bool in = k0 + k < n;
      const int sl = s0 + k0 + (in ? k : 0);
      const int pi = sl * kRowsPerCta + lr;
      const __nv_bfloat16* op = obase + sl * kSlotElems;
      mv[k] = in ? m_parts[pi] : -INFINITY;
      lv[k] = in ? l_parts[pi] : 0.f;
#pragma unroll
      for (int d = 0; d < kMergeVecs; ++d)
        ov[k][d] = in ? *reinterpret_cast<const uint4*>(op + d * kRowsPerCta * 8)
                      : make_uint4(0u, 0u, 0u, 0u);
    }
    float Mb = M;
#pragma unroll
    for (int k = 0; k < kMergeBatch; ++k) Mb = fmaxf(Mb, mv[k]);
    if (Mb == -INFINITY) continue;
    if (Mb > M) {
      const float cs = M == -INFINITY ? 0.f : tc::ex2_approx(M - Mb);
      M = Mb;
      L *= cs;
#pragma unroll
      for (int d = 0; d < kMergeDims; ++d) a[d] *= cs;
    }
#pragma unroll
    for (int k = 0; k < kMergeBatch; ++k) {
      const float w = mv[k] == -INFINITY ? 0.f : tc::ex2_approx(mv[k] - M) * lv[k];
      L += w;
#pragma unroll
      for (int d = 0; d < kMergeVecs; ++d) {
        const uint32_t wd[4] = {ov[k][d].x, ov[k][d].y, ov[k][d].z, ov[k][d].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          a[d * 8 + 2 * e] = fmaf(w, __uint_as_float(wd[e] << 16), a[d * 8 + 2 * e]);
          a[d * 8 + 2 * e + 1] = fmaf(w, __uint_as_float(wd[e] & 0xffff0000u), a[d * 8 + 2 * e + 1]);
        }
      }
    }
  }
  const int h = u / p.n_pairs;
  const long long node = R / p.group, qh = h * p.group + R % p.group;
  if constexpr (kFp32) {
    const long long row = node * p.q_heads + qh;
    float* o = o_merged + row * kHeadDim + dq * kMergeDims;
#pragma unroll
    for (int d = 0; d < kMergeDims; d += 4)
      *reinterpret_cast<float4*>(o + d) = make_float4(a[d], a[d + 1], a[d + 2], a[d + 3]);
    if (dq == 0) {
      m_merged[row] = M;
      l_merged[row] = L;
    }
  } else {
    const float inv = L > 0.f ? 1.f / L : 0.f;
    __nv_bfloat16* o = out + node * o_node_stride + qh * o_head_stride + dq * kMergeDims;
#pragma unroll
    for (int d = 0; d < kMergeDims; d += 8) {
      uint4 v;
      v.x = tc::pack_bf16x2(a[d] * inv, a[d + 1] * inv);
      v.y = tc::pack_bf16x2(a[d + 2] * inv, a[d + 3] * inv);
      v.z = tc::pack_bf16x2(a[d + 4] * inv, a[d + 5] * inv);
      v.w = tc::pack_bf16x2(a[d + 6] * inv, a[d + 7] * inv);
      *reinterpret_cast<uint4*>(o + d) = v;
    }
  }
}

// ---- mask -> bitmask -------------------------------------------------------------------
template <typename T>
__global__ void mask_to_bits_kernel(const T* __restrict__ mask, int n, long long row_stride,
                                    uint32_t* __restrict__ bits, int words) {
  const int i = blockIdx.x;
  for (int w = threadIdx.x; w < words; w += blockDim.x) {
    uint32_t v = 0;
    for (int b = 0; b < 32; ++b) {
      const int j = w * 32 + b;
      if (j < n && static_cast<float>(mask[i * row_stride + j]) == 0.f) v |= 1u << b;
    }
    bits[static_cast<long long>(i) * words + w] = v;
  }
}

// ---- host side ----------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 3-D bf16 tensor map: dims {d0 (contiguous), d1, d2}, byte strides {s1, s2}, box
// {b0, b1, b2}, 128-byte swizzle, zero fill out of bounds.
inline int make_map(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                    uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return DDT_ERR_CUDA;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {s1, s2};
  const cuuint32_t box[3] = {b0, b1, b2};
  const cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DDT_OK : DDT_ERR_ALIGN;
}

struct Launch {
  CUtensorMap q, k, v;
  Params p;
  Sched sched;
  SlotTable slots;
  int grid;
  int n_parts;
};

// Size checks and the size-dependent Params fields of a launch over the global key range
// [key_lo, key_hi) (no pointers, no device work): shared by the launching entry points and the
// host-only plan query.
inline int prepare_sizes(Params& p, int64_t n_nodes, int64_t past_length, int64_t q_heads,
                         int64_t kv_heads, int64_t key_lo, int64_t key_hi) {
  if (n_nodes <= 0 || past_length < 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads)
    return DDT_ERR_INVALID;
  const int64_t group = q_heads / kv_heads;
  if (group > kBlockM || kBlockM % group) return DDT_ERR_CAPACITY;
  if (past_length + n_nodes >= (int64_t(1) << 31)) return DDT_ERR_CAPACITY;
  if (key_lo < 0 || key_hi < key_lo || key_hi > past_length + n_nodes) return DDT_ERR_INVALID;
  p.n_nodes = static_cast<int>(n_nodes);
  p.past_len = static_cast<int>(past_length);
  p.group = static_cast<int>(group);
  p.q_heads = static_cast<int>(q_heads);
  p.n_pairs = static_cast<int>((n_nodes * group + kRowsPerCta - 1) / kRowsPerCta);
  p.key_base = p.key_lo = static_cast<int>(key_lo);
  p.key_hi = static_cast<int>(key_hi);
  p.anc = nullptr;
  p.anc_words = 0;
  p.mask_mode = DDT_MASK_TREE;
  p.scale_log2 = 0.f;
  p.out = nullptr;
  p.o_part = p.m_part = p.l_part = nullptr;
  p.o_slot = nullptr;
  p.partial = 0;
  p.balanced = 0;
  p.n_splits = 1;
  p.status = nullptr;
  p.timeout_ns = kTimeoutNs;
  p.withhold_loads = 0;
  p.past_dev = nullptr;
  return DDT_OK;
}

// prepare_sizes plus the pointer, mask and stride checks and the TMA tensor maps; the K / V
// pointers address global key key_lo (the first key of the launch's range).
inline int prepare(Launch& L, const void* q, int64_t q_node_stride, int64_t q_head_stride,
                   const void* k, const void* v, int64_t kv_head_stride, int64_t kv_seq_stride,
                   int64_t key_lo, int64_t key_hi, int64_t n_nodes, int64_t past_length,
                   int64_t q_heads, int64_t kv_heads, int64_t head_dim, const uint32_t* anc_bits,
                   int64_t anc_words, int mask_mode, float scale) {
  if (!q || !k || !v) return DDT_ERR_INVALID;
  if (head_dim != kHeadDim) return DDT_ERR_CAPACITY;
  int rc = prepare_sizes(L.p, n_nodes, past_length, q_heads, kv_heads, key_lo, key_hi);
  if (rc) return rc;
  if (mask_mode != DDT_MASK_TREE && mask_mode != DDT_MASK_CAUSAL && mask_mode != DDT_MASK_NONE)
    return DDT_ERR_INVALID;
  if (mask_mode == DDT_MASK_TREE && (!anc_bits || anc_words * 32 < n_nodes)) return DDT_ERR_INVALID;
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16)) return DDT_ERR_ALIGN;
  if ((q_node_stride * 2) % 16 || (q_head_stride * 2) % 16 || (kv_head_stride * 2) % 16 ||
      (kv_seq_stride * 2) % 16)
    return DDT_ERR_ALIGN;
  const int64_t group = q_heads / kv_heads;
  const int64_t kv_len_local = key_hi > key_lo ? key_hi - key_lo : 1;
  rc = make_map(&L.q, q, kHeadDim, q_heads, n_nodes, q_head_stride * 2, q_node_stride * 2, 64,
                static_cast<uint32_t>(group), static_cast<uint32_t>(kBlockM / group));
  if (rc) return rc;
  rc = make_map(&L.k, k, kHeadDim, kv_len_local, kv_heads, kv_seq_stride * 2, kv_head_stride * 2,
                64, kBlockN, 1);
  if (rc) return rc;
  rc = make_map(&L.v, v, kHeadDim, kv_len_local, kv_heads, kv_seq_stride * 2, kv_head_stride * 2,
                64, kBlockN, 1);
  if (rc) return rc;
  Params& p = L.p;
  p.anc = anc_bits;
  p.anc_words = static_cast<int>(anc_words);
  p.mask_mode = mask_mode;
  p.scale_log2 = scale * 1.4426950408889634f;
  return DDT_OK;
}

// Balanced schedule: the flattened (unit, key tile) cost range cut into G equal pieces (CTA
// c: [c W / G, (c + 1) W / G)).  Costs are in eighths of a key tile and follow per-CTA cycle
// counts measured at the Qwen3-8B verify shape, fitted as cycles = 2494 per key tile + 1527
// per tile that ends past the prefix (the tree window: masked, for some rows, in the
// softmax) + 4918 per item (Q load, pipeline refill, the partial's epilogue):
//   kCostTile = 8, kCostMasked = 13 (1.6 tiles), kCostItem = 16 (2 tiles, paid at the start
//   of each unit's range, so a CTA whose range reaches into a second unit gets
//   correspondingly fewer tiles).
// A CTA's cost range maps to whole tiles of a unit by the unit's cumulative cost (a tile goes
// to the CTA whose range holds the tile's start); a CTA may get no tile of a unit it touches,
// and then has no item for it.  Returns false (and leaves the launch on uniform splits) when
// a limit of the tables is exceeded or a unit has no key tile.
constexpr int kCostTile = 8;
constexpr int kCostMasked = 13;
constexpr int kCostItem = 16;

inline bool build_balanced(Launch& L, int64_t units) {
  Params& p = L.p;
  if (units <= 0 || units > kMaxUnits) return false;
  int64_t W = 0, real = 0;
  int ntot[kMaxUnits], nfull[kMaxUnits];
  int64_t cost[kMaxUnits];
  // tiles of a unit that end at or before the prefix end (unmasked in the tree window sense)
  int64_t before = (static_cast<int64_t>(p.past_len) - p.key_lo) / kBlockN;
  if (p.past_len < p.key_lo) before = 0;
  for (int u = 0; u < units; ++u) {
    ntot[u] = unit_geo(p, u).ntot;
    if (ntot[u] <= 0 || ntot[u] > 0xffff) return false;
    nfull[u] = static_cast<int>(before < ntot[u] ? before : ntot[u]);
    cost[u] = static_cast<int64_t>(nfull[u]) * kCostTile +
              static_cast<int64_t>(ntot[u] - nfull[u]) * kCostMasked;
    W += kCostItem + cost[u];
    real += ntot[u];
  }
  const int64_t G = real < kMaxCtas ? real : kMaxCtas;
  auto cta_of = [&](int64_t x) { return ((x + 1) * G - 1) / W; };  // CTA holding position x
  // items in unit order (slots of a unit consecutive); CTA lists follow since units and
  // CTAs both advance monotonically along the flattened range
  int n = 0;
  int64_t T = 0;  // cost position of unit u's first tile
  int cur_cta = -1;
  for (int u = 0; u < units; ++u) {
    T += kCostItem;
    L.slots.unit_slot[u] = static_cast<uint16_t>(n);
    // tile boundary at cost offset x of this unit (the first tile not started before x)
    const int64_t fcost = static_cast<int64_t>(nfull[u]) * kCostTile;
    auto tile_at = [&](int64_t x) -> int64_t {
      if (x >= cost[u]) return ntot[u];
      if (x <= fcost) return (x + kCostTile - 1) / kCostTile;
      const int64_t t = nfull[u] + (x - fcost + kCostMasked - 1) / kCostMasked;
      return t < ntot[u] ? t : ntot[u];
    };
    const int64_t cf = cta_of(T), cl = cta_of(T + cost[u] - 1);
    if (cl - cf + 1 > kMaxPartsPerUnit) return false;
    for (int64_t c = cf; c <= cl; ++c) {
      const int64_t b = c * W / G, e = (c + 1) * W / G;
      const int64_t lo = b > T ? b : T, hi = e < T + cost[u] ? e : T + cost[u];
      const int64_t tlo = tile_at(lo - T), thi = tile_at(hi - T);
      if (thi <= tlo) continue;
      if (n >= kMaxItems) return false;
      while (cur_cta < c) L.sched.cta_first[++cur_cta] = static_cast<uint16_t>(n);
      L.sched.items[n] = SchedItem{static_cast<uint16_t>(u), static_cast<uint16_t>(tlo),
                                   static_cast<uint16_t>(thi - tlo), static_cast<uint16_t>(n)};
      ++n;
    }
    T += cost[u];
  }
  while (cur_cta < G) L.sched.cta_first[++cur_cta] = static_cast<uint16_t>(n);
  L.slots.unit_slot[units] = static_cast<uint16_t>(n);
  L.grid = static_cast<int>(G);
  L.n_parts = n;
  p.balanced = 1;
  return true;
}

inline int pick_splits(int64_t units, int64_t kv_tiles) {
  // One CTA per SM (192 KB of shared memory each): split the key range so the grid
  // fills at most one wave of 148 SMs, keeping at least 4 key tiles per split.
  int64_t s = units >= 148 ? 1 : 148 / units;
  const int64_t cap = kv_tiles / 4 > 1 ? kv_tiles / 4 : 1;
  if (s > cap) s = cap;
  if (s < 1) s = 1;
  if (s > 64) s = 64;
  return static_cast<int>(s);
}

inline size_t part_bytes(int64_t rows, int64_t splits) {
  return static_cast<size_t>(splits) * rows * (kHeadDim + 2) * sizeof(float) + 256;
}

// bytes of `parts` balanced partials of 256 rows each (O / l in bf16, m and l in fp32)
inline size_t slot_bytes(int64_t parts) {
  return static_cast<size_t>(parts) * kRowsPerCta *
             (kHeadDim * sizeof(__nv_bfloat16) + 2 * sizeof(float)) +
         256;
}
// workspace carve-up of balanced parts: O slots, then m, then l (16-byte aligned)
struct SlotPtrs {
  __nv_bfloat16* o;
  float* m;
  float* l;
};
inline SlotPtrs slot_ptrs(void* ws, int64_t parts) {
  SlotPtrs sp;
  sp.o = static_cast<__nv_bfloat16*>(ws);
  sp.m = reinterpret_cast<float*>(sp.o + static_cast<size_t>(parts) * kRowsPerCta * kHeadDim);
  sp.l = sp.m + static_cast<size_t>(parts) * kRowsPerCta;
  return sp;
}

inline int launch(const Launch& L, int64_t kv_heads, cudaStream_t st) {
  // the attribute belongs to the current device: set on every launch (it costs a host call),
  // so a process that uses several GPUs, from several threads, needs no per-device state
  auto kern = L.p.past_dev ? tree_attn_kernel<true> : tree_attn_kernel<false>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc) !=
      cudaSuccess)
    return DDT_ERR_CUDA;
  const int64_t grid = L.p.balanced ? L.grid : kv_heads * L.p.n_pairs * L.p.n_splits;
  kern<<<static_cast<unsigned>(grid), kThreads, kSmemAlloc, st>>>(L.q, L.k, L.v, L.p, L.sched);
  return launch_status();
}

// How a launch covers its work.
//   kPlanSingle    one launch, every CTA one work unit over all its keys, bf16 out directly
//   kPlanUniform   every unit's key tiles cut into p.n_splits equal splits, fp32 partials,
//                  merge_kernel
//   kPlanBalanced  the (unit, key tile) space cut over the SMs by the cost model
//                  (build_balanced), bf16 parts in slots, merge_slots_kernel
enum PlanKind { kPlanSingle = 0, kPlanUniform = 1, kPlanBalanced = 2 };

// The one place that picks the plan, used by ddt_tree_attn (shard = false), by
// ddt_tree_attn_partial_merged (shard = true) and by the host-only ddt_tree_attn_plan, so the
// plan the query reports (and the CPU tests sweep) is the plan that is launched.  L.p must
// come from prepare_sizes.  Full range: balanced when the split count is automatic, there
// are fewer units than SMs, more than one split pays and the K / V fit in L2; otherwise
// uniform splits (merged) or one launch.  A shard: balanced whenever its K / V fit in L2,
// otherwise uniform splits, always merged to one partial per row (even with one split).
inline int choose_plan(Launch& L, int64_t kv_heads, int64_t kv_splits, bool shard, int& kind) {
  Params& p = L.p;
  const int64_t units = kv_heads * p.n_pairs;
  const int64_t local = static_cast<int64_t>(p.key_hi) - p.key_lo;
  const int64_t kv_tiles = local > 0 ? (local + kBlockN - 1) / kBlockN : 1;
  const int64_t splits = (!shard && kv_splits > 0) ? kv_splits : pick_splits(units, kv_tiles);
  if (splits > 64) return DDT_ERR_CAPACITY;
  p.n_splits = static_cast<int>(splits);
  p.balanced = 0;
  const bool try_balanced =
      kv_fits_l2(local, kv_heads) &&
      (shard || (kv_splits <= 0 && units < kMaxCtas && splits > 1));
  if (try_balanced && build_balanced(L, units)) {
    kind = kPlanBalanced;
    return DDT_OK;
  }
  p.balanced = 0;
  L.grid = static_cast<int>(units * splits);
  L.n_parts = static_cast<int>(splits);
  kind = (shard || splits > 1) ? kPlanUniform : kPlanSingle;
  return DDT_OK;
}

// Workspace bytes a plan needs (0 for kPlanSingle).
inline size_t plan_workspace(const Launch& L, int kind) {
  if (kind == kPlanBalanced) return slot_bytes(L.n_parts);
  if (kind == kPlanUniform)
    return part_bytes(static_cast<int64_t>(L.p.n_nodes) * L.p.q_heads, L.p.n_splits);
  return 0;
}

// Runs a chosen plan: the attention launch and, for split plans, its merge.  The result is
// bf16 `out` (strides o_node_stride, o_head_stride) or, when out is null, one fp32 partial per
// row in (node, q head) order: o_merged [rows, 128], m_merged / l_merged [rows].
inline int run(Launch& L, int kind, int64_t kv_heads, void* workspace, size_t workspace_bytes,
               __nv_bfloat16* out, int64_t o_node_stride, int64_t o_head_stride, float* o_merged,
               float* m_merged, float* l_merged, cudaStream_t st,
               const peer::Push& push = peer::Push{}) {
  Params& p = L.p;
  const int64_t rows = static_cast<int64_t>(p.n_nodes) * p.q_heads;
  if (kind == kPlanSingle) {
    if (!out) return DDT_ERR_INVALID;
    p.out = out;
    p.o_node_stride = o_node_stride;
    p.o_head_stride = o_head_stride;
    return launch(L, kv_heads, st);
  }
  if (!workspace || workspace_bytes < plan_workspace(L, kind)) return DDT_ERR_WORKSPACE;
  if (!aligned(workspace, 16)) return DDT_ERR_ALIGN;
  p.partial = 1;
  if (kind == kPlanBalanced) {
    const SlotPtrs sp = slot_ptrs(workspace, L.n_parts);
    p.o_slot = sp.o;
    p.m_part = sp.m;
    p.l_part = sp.l;
    int rc = launch(L, kv_heads, st);
    if (rc) return rc;
    const int64_t units = kv_heads * p.n_pairs;
    const int64_t warps = units * (kRowsPerCta / 32) * (kHeadDim / kMergeDims);
    const unsigned blocks = static_cast<unsigned>((warps + kMergeWarps - 1) / kMergeWarps);
    if (out)
      merge_slots_kernel<false><<<blocks, kMergeWarps * 32, 0, st>>>(
          sp.o, sp.m, sp.l, L.slots, p, out, o_node_stride, o_head_stride, nullptr, nullptr,
          nullptr);
    else
      merge_slots_kernel<true><<<blocks, kMergeWarps * 32, 0, st>>>(
          sp.o, sp.m, sp.l, L.slots, p, nullptr, 0, 0, o_merged, m_merged, l_merged);
    return launch_status();
  }
  float* op = static_cast<float*>(workspace);
  float* mp = op + static_cast<size_t>(p.n_splits) * rows * kHeadDim;
  float* lp = mp + static_cast<size_t>(p.n_splits) * rows;
  p.o_part = op;
  p.m_part = mp;
  p.l_part = lp;
  int rc = launch(L, kv_heads, st);
  if (rc) return rc;
  const int wpb = 8;
  merge_kernel<<<static_cast<unsigned>((rows + wpb - 1) / wpb), wpb * 32, 0, st>>>(
      op, mp, lp, p.n_splits, rows, p.q_heads, out, o_node_stride, o_head_stride, o_merged,
      m_merged, l_merged, push);
  return launch_status();
}

}  // namespace attn
}  // namespace ddt

using namespace ddt;

extern "C" size_t ddt_tree_attn_workspace_bytes(int64_t n_nodes, int64_t q_heads, int64_t head_dim,
                                                int64_t kv_splits) {
  (void)head_dim;
  const int64_t rows = n_nodes * q_heads;
  if (kv_splits > 0) return attn::part_bytes(rows, kv_splits);
  // automatic: balanced parts (at most one per CTA plus one per work unit; units <=
  // rows / 256 + q_heads), or, when the schedule tables do not fit, uniform splits, whose
  // splits * rows stay below 148 * 256 (splits <= 148 / units, rows <= 256 units)
  const int64_t parts = attn::kMaxCtas + (rows + attn::kRowsPerCta - 1) / attn::kRowsPerCta + q_heads;
  const size_t a = attn::slot_bytes(parts);
  const size_t b = attn::part_bytes(attn::kMaxCtas * attn::kRowsPerCta, 1);
  return a > b ? a : b;
}

extern "C" int ddt_tree_attn(const void* q, int64_t q_node_stride, int64_t q_head_stride,
                             const void* k, const void* v, int64_t kv_head_stride,
                             int64_t kv_seq_stride, void* out, int64_t o_node_stride,
                             int64_t o_head_stride, int64_t n_nodes, int64_t past_length,
                             int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                             const uint32_t* anc_bits, int64_t anc_words, int mask_mode,
                             float scale, int64_t kv_splits, void* workspace,
                             size_t workspace_bytes, int32_t* status, void* stream) {
  if (!out) return DDT_ERR_INVALID;
  if (!aligned(out, 16) || (o_node_stride * 2) % 16 || (o_head_stride * 2) % 16) return DDT_ERR_ALIGN;
  attn::Launch L;
  int rc = attn::prepare(L, q, q_node_stride, q_head_stride, k, v, kv_head_stride, kv_seq_stride, 0,
                         past_length + n_nodes, n_nodes, past_length, q_heads, kv_heads, head_dim,
                         anc_bits, anc_words, mask_mode, scale);
  if (rc) return rc;
  int kind = 0;
  rc = attn::choose_plan(L, kv_heads, kv_splits, false, kind);
  if (rc) return rc;
  L.p.status = status;
  return attn::run(L, kind, kv_heads, workspace, workspace_bytes, static_cast<__nv_bfloat16*>(out),
                   o_node_stride, o_head_stride, nullptr, nullptr, nullptr,
                   static_cast<cudaStream_t>(stream));
}

// ddt_tree_attn with the prefix length in device memory, so that one launch (one CUDA graph
// node) serves every prefix length up to max_past_length.  The plan, the schedule and the
// tensor maps are made for max_past_length: K / V hold max_past_length + n_nodes rows, the
// tree's rows sit at [live, live + n_nodes) and the keys after them are masked, so the launch
// costs what a launch at max_past_length costs.
extern "C" int ddt_tree_attn_device_past(const void* q, int64_t q_node_stride,
                                         int64_t q_head_stride, const void* k, const void* v,
                                         int64_t kv_head_stride, int64_t kv_seq_stride, void* out,
                                         int64_t o_node_stride, int64_t o_head_stride,
                                         int64_t n_nodes, int64_t max_past_length,
                                         const int64_t* past_length_dev, int64_t q_heads,
                                         int64_t kv_heads, int64_t head_dim,
                                         const uint32_t* anc_bits, int64_t anc_words,
                                         int mask_mode, float scale, int64_t kv_splits,
                                         void* workspace, size_t workspace_bytes, int32_t* status,
                                         void* stream) {
  if (!out || !past_length_dev || !status) return DDT_ERR_INVALID;
  // every row sees every key without a mask, including the rows after the live window
  if (mask_mode == DDT_MASK_NONE) return DDT_ERR_INVALID;
  if (!aligned(past_length_dev, 8)) return DDT_ERR_ALIGN;
  if (!aligned(out, 16) || (o_node_stride * 2) % 16 || (o_head_stride * 2) % 16) return DDT_ERR_ALIGN;
  attn::Launch L;
  int rc = attn::prepare(L, q, q_node_stride, q_head_stride, k, v, kv_head_stride, kv_seq_stride, 0,
                         max_past_length + n_nodes, n_nodes, max_past_length, q_heads, kv_heads,
                         head_dim, anc_bits, anc_words, mask_mode, scale);
  if (rc) return rc;
  int kind = 0;
  rc = attn::choose_plan(L, kv_heads, kv_splits, false, kind);
  if (rc) return rc;
  L.p.status = status;
  L.p.past_dev = past_length_dev;
  return attn::run(L, kind, kv_heads, workspace, workspace_bytes, static_cast<__nv_bfloat16*>(out),
                   o_node_stride, o_head_stride, nullptr, nullptr, nullptr,
                   static_cast<cudaStream_t>(stream));
}

extern "C" int64_t ddt_tree_attn_partial_splits(int64_t n_nodes, int64_t key_count,
                                                int64_t q_heads, int64_t kv_heads) {
  if (n_nodes <= 0 || key_count <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads)
    return 1;
  const int64_t pairs = (n_nodes * (q_heads / kv_heads) + attn::kRowsPerCta - 1) / attn::kRowsPerCta;
  return attn::pick_splits(kv_heads * pairs, (key_count + attn::kBlockN - 1) / attn::kBlockN);
}

// The launch plan of ddt_tree_attn (key_end < 0) or of ddt_tree_attn_partial_merged over the
// shard [key_begin, key_end), from attn::choose_plan (the function both of them launch
// through), plus a check of a balanced table: every key tile of every work unit in exactly
// one item, the items of a unit in key order with consecutive slots, every item in one CTA's
// list.
extern "C" int ddt_tree_attn_plan(int64_t n_nodes, int64_t past_length, int64_t q_heads,
                                  int64_t kv_heads, int64_t kv_splits, int64_t key_begin,
                                  int64_t key_end, int64_t* plan) {
  if (!plan || kv_splits < 0) return DDT_ERR_INVALID;
  const bool shard = key_end >= 0;
  attn::Launch L;
  int rc = attn::prepare_sizes(L.p, n_nodes, past_length, q_heads, kv_heads,
                               shard ? key_begin : 0, shard ? key_end : past_length + n_nodes);
  if (rc) return rc;
  int kind = 0;
  rc = attn::choose_plan(L, kv_heads, kv_splits, shard, kind);
  if (rc) return rc;
  const attn::Params& p = L.p;
  const int64_t units = kv_heads * p.n_pairs;
  if (kind == attn::kPlanBalanced) {
    int64_t max_items = 0;
    for (int c = 0; c < L.grid; ++c) {
      const int64_t k = L.sched.cta_first[c + 1] - L.sched.cta_first[c];
      if (k < 0) return 1;
      if (k > max_items) max_items = k;
    }
    if (L.sched.cta_first[0] != 0 || L.sched.cta_first[L.grid] != L.n_parts) return 1;
    for (int64_t u = 0; u < units; ++u) {
      const int s0 = L.slots.unit_slot[u], s1 = L.slots.unit_slot[u + 1];
      if (s1 <= s0 || s1 - s0 > attn::kMaxPartsPerUnit) return 1;
      int next = 0;
      for (int sl = s0; sl < s1; ++sl) {
        const attn::SchedItem& it = L.sched.items[sl];
        if (it.unit != u || it.slot != sl || it.t0 != next || it.nt == 0) return 1;
        next += it.nt;
      }
      if (next != attn::unit_geo(p, static_cast<int>(u)).ntot) return 1;
    }
    plan[0] = 1;
    plan[1] = L.grid;
    plan[2] = L.n_parts;
    plan[3] = max_items;
    return DDT_OK;
  }
  plan[0] = 0;
  plan[1] = L.grid;
  plan[2] = kind == attn::kPlanUniform ? p.n_splits : 0;
  plan[3] = 1;
  return DDT_OK;
}

extern "C" int ddt_tree_attn_partial(const void* q, int64_t q_node_stride, int64_t q_head_stride,
                                     const void* k, const void* v, int64_t kv_head_stride,
                                     int64_t kv_seq_stride, int64_t key_begin, int64_t key_end,
                                     float* o_part, float* m_part, float* l_part, int64_t n_nodes,
                                     int64_t past_length, int64_t q_heads, int64_t kv_heads,
                                     int64_t head_dim, const uint32_t* anc_bits,
                                     int64_t anc_words, int mask_mode, float scale,
                                     int64_t kv_splits, int32_t* status, void* stream) {
  if (!o_part || !m_part || !l_part) return DDT_ERR_INVALID;
  if (!aligned(o_part, 16)) return DDT_ERR_ALIGN;
  attn::Launch L;
  int rc = attn::prepare(L, q, q_node_stride, q_head_stride, k, v, kv_head_stride, kv_seq_stride,
                         key_begin, key_end, n_nodes, past_length, q_heads, kv_heads, head_dim,
                         anc_bits, anc_words, mask_mode, scale);
  if (rc) return rc;
  const int64_t local = key_end - key_begin;
  if (kv_splits <= 0) {
    const int64_t kv_tiles = local > 0 ? (local + attn::kBlockN - 1) / attn::kBlockN : 1;
    kv_splits = attn::pick_splits(kv_heads * L.p.n_pairs, kv_tiles);
  }
  if (kv_splits > 64) return DDT_ERR_CAPACITY;
  L.p.n_splits = static_cast<int>(kv_splits);
  L.p.status = status;
  L.p.o_part = o_part;
  L.p.m_part = m_part;
  L.p.l_part = l_part;
  L.p.partial = 1;
  return attn::launch(L, kv_heads, static_cast<cudaStream_t>(stream));
}

extern "C" size_t ddt_tree_attn_partial_merged_workspace_bytes(int64_t n_nodes, int64_t q_heads,
                                                               int64_t head_dim) {
  return ddt_tree_attn_workspace_bytes(n_nodes, q_heads, head_dim, 0);
}

extern "C" int ddt_tree_attn_partial_merged(
    const void* q, int64_t q_node_stride, int64_t q_head_stride, const void* k, const void* v,
    int64_t kv_head_stride, int64_t kv_seq_stride, int64_t key_begin, int64_t key_end,
    float* o_part, float* m_part, float* l_part, int64_t n_nodes, int64_t past_length,
    int64_t q_heads, int64_t kv_heads, int64_t head_dim, const uint32_t* anc_bits,
    int64_t anc_words, int mask_mode, float scale, void* workspace, size_t workspace_bytes,
    int32_t* status, void* stream) {
  if (!o_part || !m_part || !l_part) return DDT_ERR_INVALID;
  if (!aligned(o_part, 16)) return DDT_ERR_ALIGN;
  attn::Launch L;
  int rc = attn::prepare(L, q, q_node_stride, q_head_stride, k, v, kv_head_stride, kv_seq_stride,
                         key_begin, key_end, n_nodes, past_length, q_heads, kv_heads, head_dim,
                         anc_bits, anc_words, mask_mode, scale);
  if (rc) return rc;
  int kind = 0;
  rc = attn::choose_plan(L, kv_heads, 0, true, kind);
  if (rc) return rc;
  L.p.status = status;
  return attn::run(L, kind, kv_heads, workspace, workspace_bytes, nullptr, 0, 0, o_part, m_part,
                   l_part, static_cast<cudaStream_t>(stream));
}

extern "C" int ddt_peer_push(const float* o, const float* m, const float* l, int64_t n_nodes,
                             int64_t q_heads, int64_t head_dim, void* const* peer_bases,
                             int64_t world, int64_t rank, uint32_t epoch, uint32_t* ticket,
                             void* stream);

// rows x (128 + 2) fp32 after the partials, for plans whose merge is not the uniform one
extern "C" size_t ddt_tree_attn_partial_push_workspace_bytes(int64_t n_nodes, int64_t q_heads,
                                                             int64_t head_dim) {
  const size_t rows = static_cast<size_t>(n_nodes > 0 ? n_nodes : 0) *
                      static_cast<size_t>(q_heads > 0 ? q_heads : 0);
  return peer::align256(ddt_tree_attn_workspace_bytes(n_nodes, q_heads, head_dim, 0)) +
         peer::align256(rows * (attn::kHeadDim + 2) * sizeof(float));
}

extern "C" int ddt_tree_attn_partial_push(
    const void* q, int64_t q_node_stride, int64_t q_head_stride, const void* k, const void* v,
    int64_t kv_head_stride, int64_t kv_seq_stride, int64_t key_begin, int64_t key_end,
    int64_t n_nodes, int64_t past_length, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
    const uint32_t* anc_bits, int64_t anc_words, int mask_mode, float scale,
    void* const* peer_bases, int64_t world, int64_t rank, uint32_t epoch, uint32_t* ticket,
    void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  if (!peer_bases || !ticket || epoch == 0 || !workspace) return DDT_ERR_INVALID;
  if (world <= 0 || world > peer::kMaxWorld) return DDT_ERR_CAPACITY;
  if (rank < 0 || rank >= world) return DDT_ERR_INVALID;
  for (int w = 0; w < world; ++w)
    if (!peer_bases[w] || !aligned(peer_bases[w], 256)) return DDT_ERR_INVALID;
  attn::Launch L;
  int rc = attn::prepare(L, q, q_node_stride, q_head_stride, k, v, kv_head_stride, kv_seq_stride,
                         key_begin, key_end, n_nodes, past_length, q_heads, kv_heads, head_dim,
                         anc_bits, anc_words, mask_mode, scale);
  if (rc) return rc;
  int kind = 0;
  rc = attn::choose_plan(L, kv_heads, 0, true, kind);
  if (rc) return rc;
  L.p.status = status;
  const int64_t rows = n_nodes * q_heads;
  const size_t part = peer::align256(attn::plan_workspace(L, kind));
  const size_t local = peer::align256(static_cast<size_t>(rows) * (attn::kHeadDim + 2) * sizeof(float));
  if (workspace_bytes < part + local) return DDT_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (kind == attn::kPlanUniform) {
    // the merge of the shard's key splits stores straight into every rank's buffer
    const peer::Layout lay = peer::layout(world, rows);
    const int par = static_cast<int>(epoch & 1u);
    peer::Push push{};
    for (int w = 0; w < world; ++w) push.base[w] = static_cast<unsigned char*>(peer_bases[w]);
    push.world = static_cast<int>(world);
    push.rank = static_cast<int>(rank);
    push.o_off = lay.o[par];
    push.m_off = lay.m[par];
    push.l_off = lay.l[par];
    push.ticket = ticket;
    return attn::run(L, kind, kv_heads, workspace, workspace_bytes, nullptr, 0, 0, nullptr,
                     nullptr, nullptr, st, push);
  }
  // balanced shards (K / V within L2): merged locally, then pushed by a copy kernel
  float* o = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + part);
  float* m = o + static_cast<size_t>(rows) * attn::kHeadDim;
  float* l = m + rows;
  rc = attn::run(L, kind, kv_heads, workspace, part, nullptr, 0, 0, o, m, l, st);
  if (rc) return rc;
  return ddt_peer_push(o, m, l, n_nodes, q_heads, head_dim, peer_bases, world, rank, epoch,
                       ticket, stream);
}

extern "C" int ddt_attn_merge(const float* o_parts, const float* m_parts, const float* l_parts,
                              int64_t n_parts, int64_t n_nodes, int64_t q_heads, int64_t head_dim,
                              void* out, int64_t o_node_stride, int64_t o_head_stride,
                              void* stream) {
  if (!o_parts || !m_parts || !l_parts || !out || n_parts <= 0 || n_nodes <= 0 || q_heads <= 0)
    return DDT_ERR_INVALID;
  if (head_dim != attn::kHeadDim) return DDT_ERR_CAPACITY;
  if (!aligned(o_parts, 16) || !aligned(out, 8) || (o_node_stride * 2) % 8 || (o_head_stride * 2) % 8)
    return DDT_ERR_ALIGN;
  const int64_t rows = n_nodes * q_heads;
  const int wpb = 8;
  attn::merge_kernel<<<static_cast<unsigned>((rows + wpb - 1) / wpb), wpb * 32, 0,
                       static_cast<cudaStream_t>(stream)>>>(
      o_parts, m_parts, l_parts, static_cast<int>(n_parts), rows, static_cast<int>(q_heads),
      static_cast<__nv_bfloat16*>(out), o_node_stride, o_head_stride, nullptr, nullptr, nullptr,
      peer::Push{});
  return launch_status();
}

extern "C" int ddt_mask_to_bits(const void* mask, int dtype, int64_t n_nodes, int64_t row_stride,
                                uint32_t* anc_bits, int64_t anc_words, void* stream) {
  if (!mask || !anc_bits || n_nodes <= 0 || anc_words * 32 < n_nodes || row_stride < n_nodes)
    return DDT_ERR_INVALID;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == DDT_BF16)
    attn::mask_to_bits_kernel<__nv_bfloat16><<<static_cast<unsigned>(n_nodes), 64, 0, st>>>(
        static_cast<const __nv_bfloat16*>(mask), static_cast<int>(n_nodes), row_stride, anc_bits,
        static_cast<int>(anc_words));
  else if (dtype == DDT_F32)
    attn::mask_to_bits_kernel<float><<<static_cast<unsigned>(n_nodes), 64, 0, st>>>(
        static_cast<const float*>(mask), static_cast<int>(n_nodes), row_stride, anc_bits,
        static_cast<int>(anc_words));
  else
    return DDT_ERR_DTYPE;
  return launch_status();
}

extern "C" int ddt_tree_attn_wait_check(const void* q, const void* k, const void* v, void* out,
                                        int64_t n_nodes, int64_t past_length, int64_t q_heads,
                                        int64_t kv_heads, const uint32_t* anc_bits,
                                        int64_t anc_words, uint64_t timeout_ns, int32_t* status,
                                        void* stream) {
  if (!out || !status) return DDT_ERR_INVALID;
  if (timeout_ns < 100000ull || timeout_ns > attn::kTimeoutNs) return DDT_ERR_INVALID;
  if (!aligned(out, 16)) return DDT_ERR_ALIGN;
  attn::Launch L;
  const int64_t S = past_length + n_nodes;
  int rc = attn::prepare(L, q, q_heads * attn::kHeadDim, attn::kHeadDim, k, v, S * attn::kHeadDim,
                         attn::kHeadDim, 0, S, n_nodes, past_length, q_heads, kv_heads,
                         attn::kHeadDim, anc_bits, anc_words, DDT_MASK_TREE,
                         1.0f / sqrtf(static_cast<float>(attn::kHeadDim)));
  if (rc) return rc;
  // one CTA per work unit over all of its keys, output written directly (no workspace)
  L.p.n_splits = 1;
  L.p.balanced = 0;
  L.p.status = status;
  L.p.timeout_ns = timeout_ns;
  L.p.withhold_loads = 1;
  L.p.out = static_cast<__nv_bfloat16*>(out);
  L.p.o_node_stride = q_heads * attn::kHeadDim;
  L.p.o_head_stride = attn::kHeadDim;
  return attn::launch(L, kv_heads, static_cast<cudaStream_t>(stream));
}
