// Draft-tree construction: per-depth log Z + top-k over the vocabulary, best-first
// expansion and ancestor bitmasks, in ONE launch.
//
// Replaces build_ddtree_tree (ddtree.py:84-166) and the id / position part of
// compile_ddtree_tree (ddtree.py:248-257).  The reference sorts on the device, copies
// the top-k to the host and runs a Python heapq loop plus an O(N^2) numpy visibility
// loop; here everything stays on the device.
//
// Grid: depths x chunks CTAs of 512 threads.
//   phase 1 (every CTA): one chunk of one depth row is read once from HBM (16-byte
//     vector loads), giving the chunk max, sum exp(x - max) in double, and the exact
//     top-k of the chunk under the canonical order (value desc, index asc) by a
//     radix select on the 64-bit composite (order key << 32 | ~index).
//   phase 2 (last CTA of a row, by atomic counter): merges the chunks' candidates,
//     log Z = max + log(sum) in double rounded once to float, top log-probs
//     lp = value - logZ in float (ddtree.py:109), sorted by the canonical order.
//   phase 3 (last row to finish): one warp replays the reference heap exactly
//     (ddtree.py:116-147: keys (-logw, rank tuple) with logw accumulated in double in
//     the reference's operation order), then all threads emit node ids, depths,
//     parents, verify ids / positions and the ancestor bitmasks.
// No CTA waits on another (last-arriver pattern only), so nothing can hang.
#include <float.h>

#include "common.cuh"

namespace ddt {
namespace topk {

constexpr int kThreads = 512;
constexpr int kEPT = 40;                    // elements per thread held in registers
constexpr int kChunk = kThreads * kEPT;     // max elements per chunk (20480): 8 chunks of
                                            // a 151936 vocabulary, 120 CTAs for 15 depths
constexpr int kMaxCand = kThreads * kEPT;   // max candidates merged per row
constexpr int kEPTMerge = 16;               // candidates per thread when at most 8192
constexpr int kRankBits = 12;               // bits per level in the packed rank tuple
constexpr int kLevelsPerWord = 5;

struct RadixShared {
  uint32_t hist[256];
  uint32_t warp_tot[8];
  unsigned long long prefix;
  unsigned long long mask;
  uint32_t remaining;
  int done;
  uint32_t out_count;
  int is_last;
  float fred[32];
  double dred[32];
};

struct WsLayout {
  size_t counters, chunk_max, chunk_sum, cand, cand_count, top_lp, top_ids, total;
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

__host__ __device__ inline int num_chunks(int64_t vocab) {
  return static_cast<int>((vocab + kChunk - 1) / kChunk);
}
__host__ __device__ inline int64_t chunk_len(int64_t vocab, int chunks) {
  int64_t c = (vocab + chunks - 1) / chunks;
  return (c + 7) / 8 * 8;
}

__host__ __device__ inline WsLayout ws_layout(int64_t L, int64_t V, int64_t k) {
  const int C = num_chunks(V);
  WsLayout w;
  size_t o = 0;
  w.counters = o;   o = align_up(o + sizeof(uint32_t) * (L + 1), 256);
  w.chunk_max = o;  o = align_up(o + sizeof(float) * L * C, 256);
  w.chunk_sum = o;  o = align_up(o + sizeof(double) * L * C, 256);
  w.cand = o;       o = align_up(o + sizeof(unsigned long long) * L * C * k, 256);
  w.cand_count = o; o = align_up(o + sizeof(uint32_t) * L * C, 256);
  w.top_lp = o;     o = align_up(o + sizeof(float) * L * k, 256);
  w.top_ids = o;    o = align_up(o + sizeof(uint32_t) * L * k, 256);
  w.total = o;
  return w;
}

// dynamic shared memory: max over the merge phase and the heap phase
__host__ inline size_t smem_bytes(int64_t L, int64_t k, int64_t budget) {
  int64_t kpad = 1;
  while (kpad < k) kpad <<= 1;
  size_t merge = sizeof(unsigned long long) * kpad;
  const int64_t fcap = budget + 1;
  size_t heap = align_up(sizeof(float) * L * k, 16) + sizeof(unsigned long long) * fcap +
                sizeof(double) * fcap + sizeof(double) * budget +
                4 * sizeof(unsigned long long) * fcap + sizeof(uint32_t) * fcap +
                sizeof(uint32_t) * budget;
  return align_up(merge > heap ? merge : heap, 16);
}

// ---- exp in double for the log-partition sum ------------------------------------------
// exp(d) for d <= 0 to ~1e-15 relative: Cody-Waite argument reduction d = n ln2 + r with
// ln2 split into a 32-bit-exact head and a tail (Cody & Waite, Software Manual for the
// Elementary Functions, 1980), then the Taylor series of e^r on |r| <= ln2 / 2 to degree
// 13 (truncation < 3e-16), scaled by 2^n through the exponent field.
__device__ __forceinline__ double exp_neg_d(double d) {
  if (d < -708.0) return 0.0;
  const double kLn2Hi = 6.93147180369123816490e-01;  // ln 2 to 32 significant bits
  const double kLn2Lo = 1.90821492927058770002e-10;  // ln 2 - kLn2Hi
  const double n = rint(d * 1.44269504088896340736);  // d / ln 2, nearest integer
  const double r = fma(-n, kLn2Lo, fma(-n, kLn2Hi, d));
  double p = 1.0 / 6227020800.0;  // 1/13!
  p = fma(p, r, 1.0 / 479001600.0);
  p = fma(p, r, 1.0 / 39916800.0);
  p = fma(p, r, 1.0 / 3628800.0);
  p = fma(p, r, 1.0 / 362880.0);
  p = fma(p, r, 1.0 / 40320.0);
  p = fma(p, r, 1.0 / 5040.0);
  p = fma(p, r, 1.0 / 720.0);
  p = fma(p, r, 1.0 / 120.0);
  p = fma(p, r, 1.0 / 24.0);
  p = fma(p, r, 1.0 / 6.0);
  p = fma(p, r, 0.5);
  p = fma(p, r, 1.0);
  p = fma(p, r, 1.0);
  // 2^n for n in [-1022, 0]
  return p * __longlong_as_double(static_cast<long long>(1023 + static_cast<int>(n)) << 52);
}

template <bool kBF16>
__device__ __forceinline__ float composite_value(unsigned long long c) {
  const uint32_t key = static_cast<uint32_t>(c >> 32);
  return kBF16 ? key_bf16(key >> 16) : key_f32(key);
}

// ---- block radix select over register-resident 64-bit composites ----------------
// Finds (prefix, mask) such that exactly `k` valid composites satisfy
// (c & mask) >= prefix.  Composites are unique; 0 marks an invalid slot.
// Radix passes run over the value key first, then over the index bits.  bf16 keys
// occupy bits 63..48 only (bits 47..32 are zero), so their passes skip that byte pair.
template <bool kBF16>
__device__ __forceinline__ int pass_shift(int p) {
  if (kBF16) return p < 2 ? 56 - 8 * p : 24 - 8 * (p - 2);
  return 56 - 8 * p;
}
template <bool kBF16>
__device__ __forceinline__ int num_passes() { return kBF16 ? 6 : 8; }

// small_index: every index is below 2^24, so the top byte of ~index is 0xff for every element
// and the pass over it (the first index pass) would choose bin 0xff with all active elements;
// it is applied without counting.
template <int EPT, bool kBF16>
__device__ void radix_select(const unsigned long long (&comp)[EPT], uint32_t k, RadixShared& s,
                             bool small_index) {
  const int npass = num_passes<kBF16>();
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  if (tid == 0) {
    s.prefix = 0ull;
    s.mask = 0ull;
    s.remaining = k;
    s.done = 0;
  }
  __syncthreads();
  for (int p = 0; p < npass; ++p) {
    if (s.done) break;
    const int sh = pass_shift<kBF16>(p);
    if (small_index && sh == 24) {
      if (tid == 0) {
        s.prefix |= 0xffull << 24;
        s.mask |= 0xffull << 24;
      }
      __syncthreads();
      continue;
    }
    if (tid < 256) s.hist[tid] = 0;
    __syncthreads();
    // read the pass state before the barrier that precedes its update
    const unsigned long long prefix = s.prefix, mask = s.mask;
    const uint32_t rem = s.remaining;
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
      const bool act = comp[j] != 0ull && (comp[j] & mask) == prefix;
      const uint32_t digit = static_cast<uint32_t>(comp[j] >> sh) & 255u;
      const unsigned am = __ballot_sync(DDT_FULL_MASK, act);
      if (act) {
        const unsigned peers = __match_any_sync(am, digit);
        if (lane == __ffs(peers) - 1) atomicAdd(&s.hist[digit], static_cast<uint32_t>(__popc(peers)));
      }
    }
    __syncthreads();
    uint32_t v = 0, x = 0;
    if (tid < 256) {
      v = s.hist[255 - tid];
      x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        uint32_t y = __shfl_up_sync(DDT_FULL_MASK, x, o);
        if (lane >= o) x += y;
      }
      if (lane == 31) s.warp_tot[tid >> 5] = x;
    }
    __syncthreads();
    if (tid < 256) {
      uint32_t base = 0;
      for (int w = 0; w < (tid >> 5); ++w) base += s.warp_tot[w];
      const uint32_t cum = base + x;
      const uint32_t prev = cum - v;
      if (prev < rem && cum >= rem) {
        const uint32_t b = 255u - tid;
        const uint32_t nrem = rem - prev;
        s.prefix = prefix | (static_cast<unsigned long long>(b) << sh);
        s.mask = mask | (255ull << sh);
        s.remaining = nrem;
        if (v == nrem) s.done = 1;
      }
    }
    __syncthreads();
  }
}

__device__ __forceinline__ bool selected(unsigned long long c, const RadixShared& s) {
  return c != 0ull && (c & s.mask) >= s.prefix;
}

// Appends the selected composites of this thread to out[0, cap) in arbitrary order with
// one shared atomic per warp and element slot (ballot + prefix count), instead of one
// atomic per element on a single counter.
template <int EPT>
__device__ __forceinline__ void append_selected(const unsigned long long (&comp)[EPT],
                                                RadixShared& s, unsigned long long* out,
                                                uint32_t cap) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const bool sel = selected(comp[j], s);
    const unsigned m = __ballot_sync(DDT_FULL_MASK, sel);
    if (m == 0u) continue;
    uint32_t base = 0;
    if (lane == __ffs(m) - 1) base = atomicAdd(&s.out_count, static_cast<uint32_t>(__popc(m)));
    base = __shfl_sync(DDT_FULL_MASK, base, __ffs(m) - 1);
    if (sel) {
      const uint32_t pos = base + __popc(m & ((1u << lane) - 1u));
      if (pos < cap) out[pos] = comp[j];
    }
  }
}

__device__ __forceinline__ float block_max_f(float v, RadixShared& s) {
  v = warp_max_f(v);
  if ((threadIdx.x & 31) == 0) s.fred[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float w = threadIdx.x < (blockDim.x >> 5) ? s.fred[threadIdx.x] : -INFINITY;
    w = warp_max_f(w);
    if (threadIdx.x == 0) s.fred[0] = w;
  }
  __syncthreads();
  float r = s.fred[0];
  __syncthreads();
  return r;
}

__device__ __forceinline__ double block_sum_d(double v, RadixShared& s) {
  v = warp_sum_d(v);
  if ((threadIdx.x & 31) == 0) s.dred[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    double w = threadIdx.x < (blockDim.x >> 5) ? s.dred[threadIdx.x] : 0.0;
    w = warp_sum_d(w);
    if (threadIdx.x == 0) s.dred[0] = w;
  }
  __syncthreads();
  double r = s.dred[0];
  __syncthreads();
  return r;
}

// ---- packed rank tuples -------------------------------------------------------------
// Level j (0-based) holds rank + 1 in 12 bits of word j / 5, most significant level
// first, so comparing the 4 words as unsigned integers equals Python's tuple order
// (element-wise, a shorter prefix first).
__device__ __forceinline__ int rank_shift(int level) {
  return (kLevelsPerWord - 1 - level % kLevelsPerWord) * kRankBits + 4;
}

// Adds v to level `lv` of a packed rank tuple.  The word is chosen with predicated,
// fully unrolled updates so the tuple stays in registers (a runtime array index would
// move it to local memory).
__device__ __forceinline__ void add_level(unsigned long long (&r)[4], int lv, unsigned long long v) {
  const int word = lv / kLevelsPerWord;
  const unsigned long long inc = v << rank_shift(lv);
#pragma unroll
  for (int w = 0; w < 4; ++w) r[w] += (w == word) ? inc : 0ull;
}

// Order-preserving unsigned key of a double (larger logw -> larger key); +0 and -0 map to
// the same key, so key equality is exactly double equality for the finite values here.
__device__ __forceinline__ unsigned long long dkey(double x) {
  const unsigned long long u = static_cast<unsigned long long>(__double_as_longlong(x == 0.0 ? 0.0 : x));
  return (u >> 63) ? ~u : (u | 0x8000000000000000ull);
}

// Frontier slot layout in shared memory (struct of arrays, fcap slots):
//   key u64 (order key of logw), logw f64, r[4] u64 (packed rank tuple), meta u32
struct Frontier {
  unsigned long long* key;
  double* logw;
  unsigned long long* r;  // [4][fcap]
  uint32_t* meta;         // parent | depth << 12 | rank << 17
  int fcap;
  __device__ unsigned long long& rw(int w, int s) { return r[w * fcap + s]; }
};

__device__ __forceinline__ uint32_t pack_meta(int parent, int depth, int rank) {
  return static_cast<uint32_t>(parent) | (static_cast<uint32_t>(depth) << 12) |
         (static_cast<uint32_t>(rank) << 17);
}

__device__ __forceinline__ bool ranks_less(const unsigned long long (&a)[4],
                                           const unsigned long long (&b)[4]) {
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    if (a[w] != b[w]) return a[w] < b[w];
  }
  return false;
}

// slot a pops before slot b: larger logw, then the smaller rank tuple
__device__ __forceinline__ bool slot_before(Frontier& f, int a, unsigned long long ka, int b,
                                            unsigned long long kb) {
  if (ka != kb) return ka > kb;
  unsigned long long ra[4], rb[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    ra[w] = f.rw(w, a);
    rb[w] = f.rw(w, b);
  }
  return ranks_less(ra, rb);
}

// Warp-wide best of the slots the lanes offer (-1 = none); integer keys only, rank tuples
// are read only when two keys are equal.
__device__ __forceinline__ int warp_best_slot(Frontier& f, int slot, unsigned long long key) {
  const int lane = threadIdx.x & 31;
  const bool has = slot >= 0;
  unsigned long long m = has ? key : 0ull;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long y = __shfl_xor_sync(DDT_FULL_MASK, m, o);
    m = y > m ? y : m;
  }
  const unsigned tied = __ballot_sync(DDT_FULL_MASK, has && key == m);
  if (tied == 0u) return -1;
  if (__popc(tied) == 1) return __shfl_sync(DDT_FULL_MASK, slot, __ffs(tied) - 1);
  const bool mine = (tied >> lane) & 1u;
  unsigned long long r[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) r[w] = mine ? f.rw(w, slot) : ~0ull;
  int cand = mine ? slot : 0x7fffffff;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long q[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) q[w] = __shfl_xor_sync(DDT_FULL_MASK, r[w], o);
    const int qc = __shfl_xor_sync(DDT_FULL_MASK, cand, o);
    const bool qless = ranks_less(q, r) || (!ranks_less(r, q) && qc < cand);
    if (qless) {
#pragma unroll
      for (int w = 0; w < 4; ++w) r[w] = q[w];
      cand = qc;
    }
  }
  return cand;
}

// One warp replays ddtree.py:116-147 exactly.  The frontier holds one entry per sibling
// chain (the next unpopped child of some popped node).  Each round:
//   1. the warp finds the best entry W and the best entry S2 of all the others;
//   2. lane 0 walks W's chain: the popped node's child key (logw + lp[d, 0]) joins the
//      "best of the rest" k2 if it beats it, and the chain's next sibling
//      ((logw - lp[d-1, r]) + lp[d-1, r+1], the reference's operation order) is popped
//      next iff it still pops before k2 -- the heap would pop exactly these nodes, in
//      this order.  Only the keys of the run are kept (run_keys);
//   3. the whole warp emits the run's nodes and writes their child entries.
// A frontier scan is paid once per run instead of once per node.
__device__ int heap_build(const float* lp, int L, int k, int budget, Frontier f,
                          uint32_t* node_meta, double* run_keys) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) {
    const double l0 = static_cast<double>(lp[0]);
    f.key[0] = dkey(l0);
    f.logw[0] = l0;
    f.rw(0, 0) = 1ull << rank_shift(0);
    f.rw(1, 0) = 0ull;
    f.rw(2, 0) = 0ull;
    f.rw(3, 0) = 0ull;
    f.meta[0] = pack_meta(0, 1, 0);
  }
  __syncwarp();
  int count = 0, fcount = 1;
  while (count < budget && fcount > 0) {
    // lane-local best and second best among slots lane, lane + 32, ...
    int b1 = -1, b2 = -1;
    unsigned long long k1 = 0ull, k2v = 0ull;
    for (int s = lane; s < fcount; s += 32) {
      const unsigned long long ks = f.key[s];
      if (b1 < 0 || slot_before(f, s, ks, b1, k1)) {
        b2 = b1;
        k2v = k1;
        b1 = s;
        k1 = ks;
      } else if (b2 < 0 || slot_before(f, s, ks, b2, k2v)) {
        b2 = s;
        k2v = ks;
      }
    }
    const int W = warp_best_slot(f, b1, k1);
    const bool w_mine = (b1 == W);
    const int S2 = warp_best_slot(f, w_mine ? b2 : b1, w_mine ? k2v : k1);
    // ---- 2. serial walk along W's chain (lane 0) ----
    int run = 0;
    if (lane == 0) {
      const uint32_t meta = f.meta[W];
      const int depth = (meta >> 12) & 31;
      const int rank = static_cast<int>(meta >> 17);
      bool have2 = S2 >= 0;
      unsigned long long k2key = have2 ? f.key[S2] : 0ull;
      unsigned long long k2r[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) k2r[w] = have2 ? f.rw(w, S2) : 0ull;
      unsigned long long wr[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) wr[w] = f.rw(w, W);
      const double c0 = depth < L ? static_cast<double>(lp[depth * k]) : 0.0;
      const float* row = lp + (depth - 1) * k;
      double logw = f.logw[W];
      int j = 0;
      for (;;) {
        // pop node (rank + j) with key logw
        run_keys[j] = logw;
        ++j;
        if (depth < L) {
          const double ch = logw + c0;
          const unsigned long long chk = dkey(ch);
          // child ranks: W's tuple with level depth-1 = rank + j (stored + 1) and level depth = 1
          bool better = !have2 || chk > k2key;
          if (have2 && chk == k2key) {
            unsigned long long cr[4];
#pragma unroll
            for (int w = 0; w < 4; ++w) cr[w] = wr[w];
            add_level(cr, depth - 1, static_cast<unsigned long long>(j - 1));
            add_level(cr, depth, 1ull);
            better = ranks_less(cr, k2r);
          }
          if (better) {
            have2 = true;
            k2key = chk;
#pragma unroll
            for (int w = 0; w < 4; ++w) k2r[w] = wr[w];
            add_level(k2r, depth - 1, static_cast<unsigned long long>(j - 1));
            add_level(k2r, depth, 1ull);
          }
        }
        const int r = rank + j - 1;  // rank just popped
        if (r + 1 >= k || count + j >= budget) break;
        const double sib = (logw - static_cast<double>(row[r])) + static_cast<double>(row[r + 1]);
        const unsigned long long sk = dkey(sib);
        bool next = !have2 || sk > k2key;
        if (have2 && sk == k2key) {
          unsigned long long sr[4];
#pragma unroll
          for (int w = 0; w < 4; ++w) sr[w] = wr[w];
          add_level(sr, depth - 1, static_cast<unsigned long long>(j));
          next = ranks_less(sr, k2r);
        }
        if (!next) break;
        logw = sib;
      }
      run = j;
    }
    run = __shfl_sync(DDT_FULL_MASK, run, 0);
    __syncwarp();
    // ---- 3. the warp emits the run and its child entries ----
    const uint32_t meta = f.meta[W];
    const int depth = (meta >> 12) & 31;
    const int rank = static_cast<int>(meta >> 17);
    const int parent = static_cast<int>(meta & 0xfffu);
    unsigned long long wr[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) wr[w] = f.rw(w, W);
    const double logw_w = f.logw[W];
    const bool kids = depth < L;
    const double c0 = kids ? static_cast<double>(lp[depth * k]) : 0.0;
    for (int j = lane; j < run; j += 32) {
      node_meta[count + j] = pack_meta(parent, depth, rank + j);
      if (kids) {
        const int s = fcount + j;
        const double ch = run_keys[j] + c0;
        f.logw[s] = ch;
        f.key[s] = dkey(ch);
        unsigned long long cr[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) cr[w] = wr[w];
        add_level(cr, depth - 1, static_cast<unsigned long long>(j));
        add_level(cr, depth, 1ull);
#pragma unroll
        for (int w = 0; w < 4; ++w) f.rw(w, s) = cr[w];
        f.meta[s] = pack_meta(count + j + 1, depth + 1, 0);
      }
    }
    __syncwarp();
    int fc = fcount + (kids ? run : 0);
    const int last_rank = rank + run - 1;
    if (lane == 0) {
      if (last_rank + 1 < k) {  // W now holds the chain's next sibling
        const double lw = run_keys[run - 1];
        const float* row = lp + (depth - 1) * k;
        const double sib = (lw - static_cast<double>(row[last_rank])) +
                           static_cast<double>(row[last_rank + 1]);
        f.logw[W] = sib;
        f.key[W] = dkey(sib);
        unsigned long long sr[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) sr[w] = wr[w];
        add_level(sr, depth - 1, static_cast<unsigned long long>(run));
#pragma unroll
        for (int w = 0; w < 4; ++w) f.rw(w, W) = sr[w];
        f.meta[W] = pack_meta(parent, depth, last_rank + 1);
      } else {  // chain exhausted: move the last entry into W
        const int last = fc - 1;
        if (W != last) {
          f.logw[W] = f.logw[last];
          f.key[W] = f.key[last];
#pragma unroll
          for (int w = 0; w < 4; ++w) f.rw(w, W) = f.rw(w, last);
          f.meta[W] = f.meta[last];
        }
      }
    }
    if (last_rank + 1 >= k) fc -= 1;
    (void)logw_w;
    count += run;
    fcount = fc;
    __syncwarp();
  }
  return count;
}

// Per-request strides of a batched launch (all zero / null for a single tree): request r
// reads logits + r * logits, writes its nodes at r * nodes (node_token_ids, node_depths) and
// r * (nodes + 1) (parents, verify ids / positions, rows of anc_bits), its count at
// node_count + r, and uses workspace slice r of ws_bytes.  budgets / starts / root tokens
// are per-request device arrays when given.
// The atomic tickets of all requests sit together at the start of the workspace
// (counters + r * (depths + 1)); the entry point zero-fills them before every launch, so a
// workspace can be reused whatever the shape of the previous launch.
struct Batch {
  int64_t logits;
  int64_t nodes;
  size_t ws_bytes;
  int kmax;
  const int32_t* budgets;
  const int64_t* starts;
  uint32_t* counters;
};

// Top k of a row's merged candidates (ncand composites at row_cand, EPT per thread) into
// sel[0, kpad) in arbitrary order.
template <int EPT, bool kBF16>
__device__ __forceinline__ void merge_select(const unsigned long long* row_cand, int ncand, int k,
                                             RadixShared& rs, unsigned long long* sel, int kpad,
                                             bool small_index) {
  unsigned long long c[EPT];
#pragma unroll
  for (int j = 0; j < EPT; ++j) {
    const int i = j * kThreads + threadIdx.x;
    c[j] = i < ncand ? __ldcg(&row_cand[i]) : 0ull;
  }
  radix_select<EPT, kBF16>(c, static_cast<uint32_t>(k), rs, small_index);
  if (threadIdx.x == 0) rs.out_count = 0;
  __syncthreads();
  append_selected<EPT>(c, rs, sel, static_cast<uint32_t>(kpad));
}

template <bool kBF16>
__global__ void __launch_bounds__(kThreads, 1)
topk_tree_kernel(const void* __restrict__ logits, int L, int64_t V, int64_t row_stride, int k,
                 int budget, float* __restrict__ out_top_lp, int64_t* __restrict__ out_top_ids,
                 int64_t* __restrict__ node_token_ids, int64_t* __restrict__ node_depths,
                 int32_t* __restrict__ parents, int32_t* __restrict__ node_count,
                 uint32_t* __restrict__ anc_bits, int anc_words,
                 const int64_t* __restrict__ root_token, int64_t start,
                 int64_t* __restrict__ verify_ids, int64_t* __restrict__ verify_pos,
                 unsigned char* __restrict__ ws, int vec_ok, const Batch batch) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ RadixShared rs;
  const int tid = threadIdx.x;
  const int C = num_chunks(V);
  const int r = blockIdx.x / (L * C);
  const int d = (blockIdx.x / C) % L;
  const int c = blockIdx.x % C;
  int kmax = k;
  if (batch.budgets) {  // request r of a batched launch
    budget = batch.budgets[r];
    if (budget > batch.nodes) budget = static_cast<int>(batch.nodes);  // stays in its slice
    k = budget < V ? budget : static_cast<int>(V);
    kmax = batch.kmax;
    const int64_t nodes1 = batch.nodes + 1;
    if (kBF16) logits = static_cast<const uint16_t*>(logits) + r * batch.logits;
    else logits = static_cast<const float*>(logits) + r * batch.logits;
    node_token_ids += r * batch.nodes;
    node_depths += r * batch.nodes;
    parents += r * nodes1;
    node_count += r;
    anc_bits += r * nodes1 * anc_words;
    if (root_token) root_token += r;
    if (batch.starts) start = batch.starts[r];
    if (verify_ids) verify_ids += r * nodes1;
    if (verify_pos) verify_pos += r * nodes1;
    ws += r * batch.ws_bytes;
    if (budget <= 0) {  // the empty tree (root only), written by the request's first CTA
      if (d == 0 && c == 0 && tid == 0) {
        parents[0] = -1;
        *node_count = 0;
        for (int w = 0; w < anc_words; ++w) anc_bits[w] = (w == 0) ? 1u : 0u;
        if (verify_ids) verify_ids[0] = root_token ? *root_token : 0;
        if (verify_pos) verify_pos[0] = start;
      }
      return;
    }
  }
  const WsLayout wl = ws_layout(L, V, kmax);
  uint32_t* counters = batch.budgets ? batch.counters + r * (L + 1)
                                     : reinterpret_cast<uint32_t*>(ws + wl.counters);
  float* chunk_max = reinterpret_cast<float*>(ws + wl.chunk_max);
  double* chunk_sum = reinterpret_cast<double*>(ws + wl.chunk_sum);
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(ws + wl.cand);
  uint32_t* cand_count = reinterpret_cast<uint32_t*>(ws + wl.cand_count);
  float* top_lp = reinterpret_cast<float*>(ws + wl.top_lp);
  uint32_t* top_ids = reinterpret_cast<uint32_t*>(ws + wl.top_ids);

  // ------------------------------ phase 1 ----------------------------------------
  const int64_t CH = chunk_len(V, C);
  const int64_t c0 = static_cast<int64_t>(c) * CH;
  const int64_t c1 = (c0 + CH < V) ? c0 + CH : V;
  const int64_t n = c1 > c0 ? c1 - c0 : 0;
  unsigned long long comp[kEPT];
  if constexpr (kBF16) {
    const uint16_t* row = static_cast<const uint16_t*>(logits) + d * row_stride + c0;
    if (vec_ok) {
#pragma unroll
      for (int j = 0; j < kEPT / 8; ++j) {
        const int64_t e0 = (static_cast<int64_t>(j) * kThreads + tid) * 8;
        uint4 q = make_uint4(0, 0, 0, 0);
        if (e0 < n) q = __ldcs(reinterpret_cast<const uint4*>(row + e0));  // streamed once
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int64_t idx = e0 + e;
          const uint16_t b = static_cast<uint16_t>(w[e >> 1] >> ((e & 1) * 16));
          const bool ok = idx < n;
          comp[j * 8 + e] = ok ? ((static_cast<unsigned long long>(bf16_key(b)) << 48) |
                                  static_cast<uint32_t>(~static_cast<uint32_t>(c0 + idx)))
                               : 0ull;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < kEPT; ++j) {
        const int64_t idx = static_cast<int64_t>(j) * kThreads + tid;
        const bool ok = idx < n;
        const uint16_t b = ok ? row[idx] : 0;
        comp[j] = ok ? ((static_cast<unsigned long long>(bf16_key(b)) << 48) |
                        static_cast<uint32_t>(~static_cast<uint32_t>(c0 + idx)))
                     : 0ull;
      }
    }
  } else {
    const float* row = static_cast<const float*>(logits) + d * row_stride + c0;
    if (vec_ok) {
#pragma unroll
      for (int j = 0; j < kEPT / 4; ++j) {
        const int64_t e0 = (static_cast<int64_t>(j) * kThreads + tid) * 4;
        float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
        if (e0 < n) q = __ldcs(reinterpret_cast<const float4*>(row + e0));
        const float w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int64_t idx = e0 + e;
          const bool ok = idx < n;
          comp[j * 4 + e] = ok ? ((static_cast<unsigned long long>(f32_key(w[e])) << 32) |
                                  static_cast<uint32_t>(~static_cast<uint32_t>(c0 + idx)))
                               : 0ull;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < kEPT; ++j) {
        const int64_t idx = static_cast<int64_t>(j) * kThreads + tid;
        const bool ok = idx < n;
        const float x = ok ? row[idx] : -INFINITY;
        comp[j] = ok ? ((static_cast<unsigned long long>(f32_key(x)) << 32) |
                        static_cast<uint32_t>(~static_cast<uint32_t>(c0 + idx)))
                     : 0ull;
      }
    }
  }
  // chunk max and sum exp(x - max), both exact-order independent up to double rounding
  // values are decoded from the composites (keeps the register footprint to one array)
  unsigned long long top = 0ull;
#pragma unroll
  for (int j = 0; j < kEPT; ++j) top = comp[j] > top ? comp[j] : top;
  const float lm = top ? composite_value<kBF16>(top) : -INFINITY;
  const float cm = block_max_f(lm, rs);
  double ls = 0.0;
#pragma unroll
  for (int j = 0; j < kEPT; ++j)
    if (comp[j] != 0ull)
      ls += exp_neg_d(static_cast<double>(composite_value<kBF16>(comp[j])) - static_cast<double>(cm));
  const double csum = block_sum_d(ls, rs);

  // exact top-k of the chunk
  const int kk = static_cast<int>(n < k ? n : k);
  if (kk < n) {
    radix_select<kEPT, kBF16>(comp, static_cast<uint32_t>(kk), rs, V <= (int64_t(1) << 24));
  } else if (tid == 0) {
    rs.prefix = 0ull;
    rs.mask = 0ull;
  }
  if (tid == 0) rs.out_count = 0;
  __syncthreads();
  unsigned long long* my_cand = cand + (static_cast<int64_t>(d) * C + c) * k;
  append_selected<kEPT>(comp, rs, my_cand, static_cast<uint32_t>(k));
  __syncthreads();
  const uint32_t n_out = rs.out_count < static_cast<uint32_t>(k) ? rs.out_count : k;
  for (int i = static_cast<int>(n_out) + tid; i < k; i += kThreads) my_cand[i] = 0ull;
  if (tid == 0) {
    chunk_max[d * C + c] = cm;
    chunk_sum[d * C + c] = csum;
    cand_count[d * C + c] = n_out;
  }
  // every writer fences its own stores to GPU scope before the CTA signals completion
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const uint32_t prev = atomicAdd(&counters[d], 1u);
    rs.is_last = (prev == static_cast<uint32_t>(C - 1));
  }
  __syncthreads();
  if (!rs.is_last) return;
  __threadfence();

  // ------------------------------ phase 2 ----------------------------------------
  if (tid == 0) counters[d] = 0;  // self-reset for the next launch
  // log Z from the chunk statistics
  __shared__ float s_logz;
  if (tid == 0) {
    float M = -INFINITY;
    for (int i = 0; i < C; ++i) M = fmaxf(M, __ldcg(&chunk_max[d * C + i]));
    double S = 0.0;
    for (int i = 0; i < C; ++i)
      S += __ldcg(&chunk_sum[d * C + i]) *
           exp_neg_d(static_cast<double>(__ldcg(&chunk_max[d * C + i])) - static_cast<double>(M));
    s_logz = static_cast<float>(static_cast<double>(M) + log(S));
  }
  // candidates of the row: C * k composites, 0 = empty; up to 8192 of them (budgets to 1024
  // at 8 chunks) are held 16 per thread, so the radix passes visit 16 slots, not 40
  const unsigned long long* row_cand = cand + static_cast<int64_t>(d) * C * k;
  const int ncand = C * k;
  unsigned long long* sel = reinterpret_cast<unsigned long long*>(smem);
  int kpad = 1;
  while (kpad < k) kpad <<= 1;
  const bool small_index = V <= (int64_t(1) << 24);
  if (ncand <= kThreads * kEPTMerge)
    merge_select<kEPTMerge, kBF16>(row_cand, ncand, k, rs, sel, kpad, small_index);
  else
    merge_select<kEPT, kBF16>(row_cand, ncand, k, rs, sel, kpad, small_index);
  __syncthreads();
  for (int i = k + tid; i < kpad; i += kThreads) sel[i] = 0ull;
  __syncthreads();
  // bitonic sort, descending
  for (int size = 2; size <= kpad; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < kpad; i += kThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const unsigned long long a = sel[i], b = sel[j];
          const bool desc = (i & size) == 0;
          if (desc ? (a < b) : (a > b)) {
            sel[i] = b;
            sel[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  const float lz = s_logz;
  for (int i = tid; i < k; i += kThreads) {
    const unsigned long long cv = sel[i];
    const uint32_t key = static_cast<uint32_t>(cv >> 32);
    const float value = kBF16 ? key_bf16(key >> 16) : key_f32(key);
    const uint32_t idx = ~static_cast<uint32_t>(cv);
    const float lpv = value - lz;  // ddtree.py:109, float subtraction
    top_lp[d * k + i] = lpv;
    top_ids[d * k + i] = idx;
    if (out_top_lp) out_top_lp[static_cast<int64_t>(d) * k + i] = lpv;
    if (out_top_ids) out_top_ids[static_cast<int64_t>(d) * k + i] = idx;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const uint32_t prev = atomicAdd(&counters[L], 1u);
    rs.is_last = (prev == static_cast<uint32_t>(L - 1));
  }
  __syncthreads();
  if (!rs.is_last) return;
  __threadfence();

  // ------------------------------ phase 3 ----------------------------------------
  if (tid == 0) counters[L] = 0;
  float* lp_s = reinterpret_cast<float*>(smem);
  const int fcap = budget + 1;
  unsigned long long* f_key = reinterpret_cast<unsigned long long*>(
      smem + align_up(sizeof(float) * static_cast<size_t>(L) * k, 16));
  double* f_logw = reinterpret_cast<double*>(f_key + fcap);
  double* run_keys = f_logw + fcap;
  unsigned long long* f_r = reinterpret_cast<unsigned long long*>(run_keys + budget);
  uint32_t* f_meta = reinterpret_cast<uint32_t*>(f_r + 4 * fcap);
  uint32_t* node_meta = f_meta + fcap;
  for (int i = tid; i < L * k; i += kThreads) lp_s[i] = __ldcg(&top_lp[i]);
  __syncthreads();
  __shared__ int s_count;
  if (tid < 32) {
    Frontier fr{f_key, f_logw, f_r, f_meta, fcap};
    const int cnt = heap_build(lp_s, L, k, budget, fr, node_meta, run_keys);
    if (tid == 0) s_count = cnt;
  }
  __syncthreads();
  const int count = s_count;
  const int nn = count + 1;
  for (int i = tid; i < count; i += kThreads) {
    const uint32_t meta = node_meta[i];
    const int depth = (meta >> 12) & 31;
    const int rank = static_cast<int>(meta >> 17);
    const int64_t tok = static_cast<int64_t>(__ldcg(&top_ids[(depth - 1) * k + rank]));
    node_token_ids[i] = tok;
    node_depths[i] = depth;
    parents[i + 1] = static_cast<int32_t>(meta & 0xfffu);
    if (verify_ids) verify_ids[i + 1] = tok;
    if (verify_pos) verify_pos[i + 1] = start + depth;
  }
  if (tid == 0) {
    parents[0] = -1;
    *node_count = count;
    if (verify_ids) verify_ids[0] = root_token ? *root_token : 0;
    if (verify_pos) verify_pos[0] = start;
  }
  // ancestor bitmasks, one row per thread, written from the highest word down
  for (int i = tid; i < nn; i += kThreads) {
    uint32_t* row = anc_bits + static_cast<int64_t>(i) * anc_words;
    int wcur = anc_words - 1;
    uint32_t acc = 0;
    int j = i;
    for (;;) {
      const int wj = j >= 0 ? (j >> 5) : -1;
      while (wcur > wj) {
        row[wcur] = acc;
        acc = 0;
        --wcur;
      }
      if (j < 0) break;
      acc |= 1u << (j & 31);
      j = (j == 0) ? -1 : static_cast<int>(node_meta[j - 1] & 0xfffu);
    }
  }
}

__global__ void empty_tree_kernel(int32_t* parents, int32_t* node_count, uint32_t* anc_bits,
                                  int anc_words, const int64_t* root_token, int64_t start,
                                  int64_t* verify_ids, int64_t* verify_pos) {
  if (threadIdx.x == 0) {
    parents[0] = -1;
    *node_count = 0;
    for (int w = 0; w < anc_words; ++w) anc_bits[w] = (w == 0) ? 1u : 0u;
    if (verify_ids) verify_ids[0] = root_token ? *root_token : 0;
    if (verify_pos) verify_pos[0] = start;
  }
}

}  // namespace topk
}  // namespace ddt

using namespace ddt;

extern "C" size_t ddt_topk_tree_workspace_bytes(int64_t depths, int64_t vocab, int64_t budget) {
  if (depths <= 0 || vocab <= 0 || budget <= 0) return 256;
  const int64_t k = budget < vocab ? budget : vocab;
  return topk::ws_layout(depths, vocab, k).total;
}

extern "C" int ddt_topk_tree(const void* draft_logits, int dtype, int64_t depths, int64_t vocab,
                             int64_t row_stride, int64_t budget, float* top_log_probs,
                             int64_t* top_token_ids, int64_t* node_token_ids,
                             int64_t* node_depths, int32_t* parents, int32_t* node_count,
                             uint32_t* anc_bits, int64_t anc_words, const int64_t* root_token,
                             int64_t start, int64_t* verify_ids, int64_t* verify_pos,
                             void* workspace, size_t workspace_bytes, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype != DDT_F32 && dtype != DDT_BF16) return DDT_ERR_DTYPE;
  if (!parents || !node_count || !anc_bits || depths < 0 || vocab <= 0) return DDT_ERR_INVALID;
  if (budget > DDT_MAX_BUDGET || depths > DDT_MAX_DEPTH) return DDT_ERR_CAPACITY;
  const int64_t nmax = (budget > 0 ? budget : 0) + 1;
  if (anc_words * 32 < nmax) return DDT_ERR_INVALID;
  if (budget <= 0 || depths == 0) {
    topk::empty_tree_kernel<<<1, 32, 0, st>>>(parents, node_count, anc_bits,
                                              static_cast<int>(anc_words), root_token, start,
                                              verify_ids, verify_pos);
    return launch_status();
  }
  if (!draft_logits || !node_token_ids || !node_depths || !workspace) return DDT_ERR_INVALID;
  if (row_stride < vocab || vocab >= (int64_t(1) << 31)) return DDT_ERR_INVALID;
  const int64_t k = budget < vocab ? budget : vocab;
  const int C = topk::num_chunks(vocab);
  if (static_cast<int64_t>(C) * k > topk::kMaxCand) return DDT_ERR_CAPACITY;
  const topk::WsLayout wl = topk::ws_layout(depths, vocab, k);
  if (workspace_bytes < wl.total) return DDT_ERR_WORKSPACE;
  const size_t esz = dtype == DDT_BF16 ? 2 : 4;
  // 16-byte vectors never cross the end of a row: chunk starts are multiples of 8
  // elements, and the vocabulary must be a whole number of vectors
  const int vec_ok = aligned(draft_logits, 16) && ((row_stride * esz) % 16 == 0) &&
                     ((vocab * esz) % 16 == 0);
  const size_t smem = topk::smem_bytes(depths, k, budget);
  const dim3 grid(static_cast<unsigned>(depths * C));
  if (dtype == DDT_BF16) {
    auto kern = topk::topk_tree_kernel<true>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return DDT_ERR_CUDA;
    kern<<<grid, topk::kThreads, smem, st>>>(
        draft_logits, static_cast<int>(depths), vocab, row_stride, static_cast<int>(k),
        static_cast<int>(budget), top_log_probs, top_token_ids, node_token_ids, node_depths,
        parents, node_count, anc_bits, static_cast<int>(anc_words), root_token, start,
        verify_ids, verify_pos, static_cast<unsigned char*>(workspace), vec_ok, topk::Batch{});
  } else {
    auto kern = topk::topk_tree_kernel<false>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return DDT_ERR_CUDA;
    kern<<<grid, topk::kThreads, smem, st>>>(
        draft_logits, static_cast<int>(depths), vocab, row_stride, static_cast<int>(k),
        static_cast<int>(budget), top_log_probs, top_token_ids, node_token_ids, node_depths,
        parents, node_count, anc_bits, static_cast<int>(anc_words), root_token, start,
        verify_ids, verify_pos, static_cast<unsigned char*>(workspace), vec_ok, topk::Batch{});
  }
  return launch_status();
}

// ---- batched: one launch builds the trees of many requests -----------------------------
namespace {
size_t batched_ws_slice(int64_t depths, int64_t vocab, int64_t max_budget) {
  const int64_t k = max_budget < vocab ? max_budget : vocab;
  return topk::align_up(topk::ws_layout(depths, vocab, k).total, 256);
}
size_t batched_counter_bytes(int64_t n_requests, int64_t depths) {
  return topk::align_up(sizeof(uint32_t) * static_cast<size_t>(n_requests * (depths + 1)), 256);
}
}  // namespace

extern "C" size_t ddt_topk_tree_batched_workspace_bytes(int64_t n_requests, int64_t depths,
                                                        int64_t vocab, int64_t max_budget) {
  if (n_requests <= 0 || depths <= 0 || vocab <= 0 || max_budget <= 0) return 256;
  return batched_counter_bytes(n_requests, depths) +
         static_cast<size_t>(n_requests) * batched_ws_slice(depths, vocab, max_budget);
}

extern "C" int ddt_topk_tree_batched(const void* draft_logits, int dtype, int64_t n_requests,
                                     int64_t depths, int64_t vocab, int64_t row_stride,
                                     int64_t request_stride, const int32_t* budgets,
                                     int64_t max_budget, int64_t* node_token_ids,
                                     int64_t* node_depths, int32_t* parents, int32_t* node_count,
                                     uint32_t* anc_bits, int64_t anc_words,
                                     const int64_t* root_tokens, const int64_t* starts,
                                     int64_t* verify_ids, int64_t* verify_pos, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype != DDT_F32 && dtype != DDT_BF16) return DDT_ERR_DTYPE;
  if (!draft_logits || !budgets || !node_token_ids || !node_depths || !parents || !node_count ||
      !anc_bits || !workspace || n_requests < 0 || depths <= 0 || vocab <= 0 || max_budget <= 0)
    return DDT_ERR_INVALID;
  if (max_budget > DDT_MAX_BUDGET || depths > DDT_MAX_DEPTH) return DDT_ERR_CAPACITY;
  if (anc_words * 32 < max_budget + 1) return DDT_ERR_INVALID;
  if (row_stride < vocab || request_stride < depths * row_stride ||
      vocab >= (int64_t(1) << 31))
    return DDT_ERR_INVALID;
  const int64_t kmax = max_budget < vocab ? max_budget : vocab;
  const int C = topk::num_chunks(vocab);
  if (static_cast<int64_t>(C) * kmax > topk::kMaxCand) return DDT_ERR_CAPACITY;
  const size_t slice = batched_ws_slice(depths, vocab, max_budget);
  const size_t cbytes = batched_counter_bytes(n_requests, depths);
  if (n_requests == 0) return DDT_OK;
  if (workspace_bytes < cbytes + slice * static_cast<size_t>(n_requests)) return DDT_ERR_WORKSPACE;
  if (static_cast<int64_t>(n_requests) * depths * C > 0x7fffffffLL) return DDT_ERR_CAPACITY;
  const size_t esz = dtype == DDT_BF16 ? 2 : 4;
  const int vec_ok = aligned(draft_logits, 16) && ((row_stride * esz) % 16 == 0) &&
                     ((request_stride * esz) % 16 == 0) && ((vocab * esz) % 16 == 0);
  const size_t smem = topk::smem_bytes(depths, kmax, max_budget);
  const dim3 grid(static_cast<unsigned>(n_requests * depths * C));
  unsigned char* wsb = static_cast<unsigned char*>(workspace);
  const topk::Batch batch{request_stride, max_budget, slice, static_cast<int>(kmax), budgets,
                          starts, reinterpret_cast<uint32_t*>(wsb)};
  auto kern = dtype == DDT_BF16 ? topk::topk_tree_kernel<true> : topk::topk_tree_kernel<false>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return DDT_ERR_CUDA;
  if (cudaMemsetAsync(wsb, 0, cbytes, st) != cudaSuccess) return DDT_ERR_CUDA;
  kern<<<grid, topk::kThreads, smem, st>>>(
      draft_logits, static_cast<int>(depths), vocab, row_stride, static_cast<int>(kmax),
      static_cast<int>(max_budget), nullptr, nullptr, node_token_ids, node_depths, parents,
      node_count, anc_bits, static_cast<int>(anc_words), root_tokens, 0, verify_ids, verify_pos,
      wsb + cbytes, vec_ok, batch);
  return launch_status();
}

// ---------------------------------------------------------------------------------------
// Tree build without a caller-provided workspace.
//
// Some callers of this library cannot allocate device memory at call time: serving stacks
// that reserve all device memory in their own pool at start-up and forbid any allocation
// afterwards, and plugin hosts whose interface only carries inputs and outputs, so there is
// no way to hand a workspace through.  For them the tree build keeps its scratch (chunk
// statistics, top-k candidates, the merged log-prob table and the atomic tickets) in a
// fixed array of this library's device image instead.  The array is
// DDT_NOALLOC_SCRATCH_BYTES long and every GPU that loads the library keeps it until the
// process exits.  Its device address is looked up once per device, on that device's first
// call, with cudaGetSymbolAddress (so the first call on a device should happen before any
// stream capture), and again on the first call in a new context of that device (after a
// cudaDeviceReset the module is loaded anew).  All calls share the one array: calls whose work overlaps on the GPU
// (different streams, or several host threads) race and must be serialised by the caller.
// ---------------------------------------------------------------------------------------
#include <cuda.h>

#include <mutex>

namespace ddt {
namespace topk {

static __device__ __align__(256) unsigned char g_noalloc_scratch[DDT_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
static void* g_noalloc_addr[kMaxDevices] = {};
// unique id of the CUDA context the cached address belongs to: after cudaDeviceReset (or any
// teardown of the primary context) the module is loaded anew, possibly elsewhere, so a call in
// a new context looks the address up again instead of writing through a stale one
static unsigned long long g_noalloc_ctx[kMaxDevices] = {};
static std::mutex g_noalloc_mu;

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current context (0 if it cannot be read).
static unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(fn);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current && get_id && get_current(&ctx) == CUDA_SUCCESS && ctx &&
      get_id(ctx, &id) == CUDA_SUCCESS)
    return id;
  return 0;
}

// Device address of this device's copy of the scratch array, looked up with
// cudaGetSymbolAddress once per device and context (set-up work of the first call).
static int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return DDT_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return DDT_ERR_CAPACITY;
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev] || ctx == 0 || g_noalloc_ctx[dev] != ctx) {
    // also makes the device's primary context current when no context is yet
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return DDT_ERR_CUDA;
    g_noalloc_addr[dev] = p;
    g_noalloc_ctx[dev] = current_context_id();
  }
  *out = g_noalloc_addr[dev];
  return DDT_OK;
}

}  // namespace topk
}  // namespace ddt

extern "C" int ddt_topk_tree_noalloc(const void* draft_logits, int dtype, int64_t depths,
                                     int64_t vocab, int64_t row_stride, int64_t budget,
                                     float* top_log_probs, int64_t* top_token_ids,
                                     int64_t* node_token_ids, int64_t* node_depths,
                                     int32_t* parents, int32_t* node_count, uint32_t* anc_bits,
                                     int64_t anc_words, const int64_t* root_token, int64_t start,
                                     int64_t* verify_ids, int64_t* verify_pos, void* stream) {
  if (depths > 0 && vocab > 0 && budget > 0 &&
      ddt_topk_tree_workspace_bytes(depths, vocab, budget) > DDT_NOALLOC_SCRATCH_BYTES)
    return DDT_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  int rc = topk::noalloc_scratch(&scratch);
  if (rc != DDT_OK) return rc;
  if (depths > 0 && vocab > 0 && budget > 0 && depths <= DDT_MAX_DEPTH) {
    // the array keeps the previous call's contents; the atomic tickets must start at zero
    const size_t tickets = sizeof(uint32_t) * static_cast<size_t>(depths + 1);
    if (cudaMemsetAsync(static_cast<unsigned char*>(scratch) +
                            topk::ws_layout(depths, vocab, budget < vocab ? budget : vocab).counters,
                        0, tickets, static_cast<cudaStream_t>(stream)) != cudaSuccess)
      return DDT_ERR_CUDA;
  }
  return ddt_topk_tree(draft_logits, dtype, depths, vocab, row_stride, budget, top_log_probs,
                       top_token_ids, node_token_ids, node_depths, parents, node_count, anc_bits,
                       anc_words, root_token, start, verify_ids, verify_pos, scratch,
                       DDT_NOALLOC_SCRATCH_BYTES, stream);
}
