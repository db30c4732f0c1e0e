// Sampled candidate chains and their trie: the draft tree of the MDFlash / P-Express
// variants, which sample chains from the drafter instead of expanding a best-first tree.
//
// ddt_sample_chains replaces sample_candidate_chains (mdflash.py:19-40): per drafted depth,
// num_samples tokens drawn with replacement from softmax(logits / T) (inverse CDF over the
// vocabulary with counter-based uniforms), or, for T < 1e-5, the depth's argmax (ties to the
// lowest index) repeated.  Chains are the per-depth samples stacked: chain s takes sample s
// of every depth.
//
// ddt_chain_tree replaces build_sampled_candidate_tree (ddtree.py:169-224): the chains are
// merged into a trie in chain order, a node per distinct prefix, until the budget is full.
// The reference inserts chain by chain and stops at the first new node past the budget;
// the nodes it keeps are therefore exactly the first `budget` "new" positions (chain c,
// depth d) in (c, d) order, where (c, d) is new when no earlier chain shares the prefix
// chain[c][0..d].  The kernel computes, depth by depth, the first chain holding each
// prefix, ranks the new positions with one scan, and emits node tokens, depths, parents,
// ancestor bitmasks and verify ids / positions in the layout of ddt_topk_tree.
#include <cuda_bf16.h>

#include "common.cuh"

namespace ddt {
namespace sampled {

constexpr int kThreads = 1024;
constexpr int kMaxChains = DDT_MAX_BUDGET;

// SplitMix64 (Steele, Lea and Flood, "Fast splittable pseudorandom number generators",
// OOPSLA 2014): additive constant, then two xor-shift-multiply rounds.
__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Uniform in [0, 1) with 53 random bits for (seed, offset, depth, sample).
__device__ __forceinline__ double uniform01(uint64_t seed, uint64_t offset, int depth, int s) {
  const uint64_t counter = (offset << 32) ^ (static_cast<uint64_t>(depth) << 20) ^
                           static_cast<uint64_t>(s);
  const uint64_t z = splitmix64(seed ^ splitmix64(counter));
  return static_cast<double>(z >> 11) * (1.0 / 9007199254740992.0);
}

template <bool kBF16>
__device__ __forceinline__ float load_logit(const void* row, int64_t i) {
  if constexpr (kBF16)
    return bf16_bits_to_f32(static_cast<const uint16_t*>(row)[i]);
  else
    return static_cast<const float*>(row)[i];
}

__device__ __forceinline__ unsigned long long argmax_comp(float x, uint32_t idx) {
  const uint32_t key = isnan(x) ? 0xffffffffu : f32_key(x);
  return (static_cast<unsigned long long>(key) << 32) | static_cast<uint32_t>(~idx);
}

// One CTA per depth.  chains [n_samples, depths] (row stride `depths`).
template <bool kBF16>
__global__ void __launch_bounds__(kThreads)
sample_chains_kernel(const void* __restrict__ logits, int64_t vocab, int64_t row_stride,
                     int depths, int n_samples, float inv_temp, int greedy, uint64_t seed,
                     uint64_t offset, int64_t* __restrict__ chains) {
  const int d = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const char* row = static_cast<const char*>(logits) + d * row_stride * (kBF16 ? 2 : 4);
  __shared__ unsigned long long s_best[kThreads / 32];
  __shared__ double s_chunk[kThreads + 1];
  __shared__ float s_max;
  __shared__ int64_t s_argmax;
  // pass 1: argmax composite (ties to the lowest index, NaN largest) and the row maximum
  unsigned long long best = 0ull;
  for (int64_t i = tid; i < vocab; i += kThreads) {
    const unsigned long long c = argmax_comp(load_logit<kBF16>(row, i), static_cast<uint32_t>(i));
    best = c > best ? c : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long y = __shfl_xor_sync(DDT_FULL_MASK, best, o);
    best = y > best ? y : best;
  }
  if (lane == 0) s_best[warp] = best;
  __syncthreads();
  if (warp == 0) {
    unsigned long long b = s_best[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long y = __shfl_xor_sync(DDT_FULL_MASK, b, o);
      b = y > b ? y : b;
    }
    if (lane == 0) {
      s_argmax = static_cast<int64_t>(~static_cast<uint32_t>(b));
      s_max = key_f32(static_cast<uint32_t>(b >> 32));
    }
  }
  __syncthreads();
  if (greedy) {
    for (int s = tid; s < n_samples; s += kThreads) chains[static_cast<int64_t>(s) * depths + d] = s_argmax;
    return;
  }
  // pass 2: weights w_i = exp((x_i - max) / T); chunk sums (contiguous chunks, one per
  // thread) in double, then their exclusive prefix
  const float m = s_max;
  const int64_t chunk = (vocab + kThreads - 1) / kThreads;
  const int64_t c0 = tid * chunk < vocab ? tid * chunk : vocab;
  const int64_t c1 = c0 + chunk < vocab ? c0 + chunk : vocab;
  double sum = 0.0;
  for (int64_t i = c0; i < c1; ++i) sum += expf((load_logit<kBF16>(row, i) - m) * inv_temp);
  // block-wide exclusive scan of the chunk sums
  double incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(DDT_FULL_MASK, incl, o);
    if (lane >= o) incl += y;
  }
  __shared__ double s_warp[kThreads / 32];
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    double w = s_warp[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(DDT_FULL_MASK, w, o);
      if (lane >= o) w += y;
    }
    s_warp[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  const double before_warp = warp > 0 ? s_warp[warp - 1] : 0.0;
  s_chunk[tid] = before_warp + incl - sum;  // exclusive prefix of chunk tid
  if (tid == kThreads - 1) s_chunk[kThreads] = before_warp + incl;  // total
  __syncthreads();
  const double total = s_chunk[kThreads];
  // pass 3: one uniform per sample; the chunk holding u * total by binary search, then the
  // element inside the chunk by a running sum of the same weights
  for (int s = tid; s < n_samples; s += kThreads) {
    const double target = uniform01(seed, offset, d, s) * total;
    int lo = 0, hi = kThreads - 1;  // largest t with prefix[t] <= target
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_chunk[mid] <= target) lo = mid; else hi = mid - 1;
    }
    const int64_t b0 = lo * chunk < vocab ? lo * chunk : vocab;
    const int64_t b1 = b0 + chunk < vocab ? b0 + chunk : vocab;
    double acc = s_chunk[lo];
    int64_t pick = -1, last_pos = -1;
    for (int64_t i = b0; i < b1; ++i) {
      const float w = expf((load_logit<kBF16>(row, i) - m) * inv_temp);
      if (w > 0.f) last_pos = i;
      acc += w;
      if (acc > target) {
        pick = i;
        break;
      }
    }
    if (pick < 0) pick = last_pos >= 0 ? last_pos : s_argmax;  // rounding at a chunk end
    chains[static_cast<int64_t>(s) * depths + d] = pick;
  }
}

// Single CTA.  Shared memory: first[d][c] (int32, depths x n), rank[c * depths + d] (int32),
// the current depth's tokens (int64, n), parents of the kept nodes (int32, budget + 1).
__global__ void __launch_bounds__(kThreads)
chain_tree_kernel(const int64_t* __restrict__ chains, int n, int depths, int64_t chain_stride,
                  int budget, int64_t* __restrict__ node_token_ids,
                  int64_t* __restrict__ node_depths, int32_t* __restrict__ parents,
                  int32_t* __restrict__ node_count, uint32_t* __restrict__ anc_bits,
                  int anc_words, const int64_t* __restrict__ root_token, int64_t start,
                  int64_t* __restrict__ verify_ids, int64_t* __restrict__ verify_pos) {
  extern __shared__ __align__(16) unsigned char smem[];
  int64_t* s_tok = reinterpret_cast<int64_t*>(smem);                 // [n]
  int32_t* s_first = reinterpret_cast<int32_t*>(s_tok + n);          // [depths][n]
  int32_t* s_rank = s_first + static_cast<int64_t>(depths) * n;      // [n * depths]
  int32_t* s_par = s_rank + static_cast<int64_t>(depths) * n;        // [budget + 1]
  __shared__ int s_warp[kThreads / 32];
  __shared__ int s_total;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // first[d][c]: the first chain holding chain c's prefix of length d + 1
  for (int d = 0; d < depths; ++d) {
    for (int c = tid; c < n; c += kThreads) s_tok[c] = chains[c * chain_stride + d];
    __syncthreads();
    const int32_t* prev = d > 0 ? s_first + static_cast<int64_t>(d - 1) * n : nullptr;
    int32_t* cur = s_first + static_cast<int64_t>(d) * n;
    for (int c = tid; c < n; c += kThreads) {
      const int pc = prev ? prev[c] : 0;
      const int64_t t = s_tok[c];
      int f = c;
      for (int c2 = prev ? pc : 0; c2 < c; ++c2) {  // chains before pc differ in the prefix
        if ((!prev || prev[c2] == pc) && s_tok[c2] == t) {
          f = c2;
          break;
        }
      }
      cur[c] = f;
    }
    __syncthreads();
  }
  // ranks of the new positions in (chain, depth) order: every thread scans a contiguous
  // piece of the flattened n x depths grid
  const int total_pos = n * depths;
  const int per = (total_pos + kThreads - 1) / kThreads;
  const int p0 = tid * per < total_pos ? tid * per : total_pos;
  const int p1 = p0 + per < total_pos ? p0 + per : total_pos;
  int cnt = 0;
  for (int pos = p0; pos < p1; ++pos) {
    const int c = pos / depths, d = pos % depths;
    cnt += s_first[static_cast<int64_t>(d) * n + c] == c;
  }
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(DDT_FULL_MASK, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = s_warp[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(DDT_FULL_MASK, w, o);
      if (lane >= o) w += y;
    }
    s_warp[lane] = w;
    if (lane == 31) s_total = w;
  }
  __syncthreads();
  int r = (warp > 0 ? s_warp[warp - 1] : 0) + incl - cnt;
  for (int pos = p0; pos < p1; ++pos) {
    const int c = pos / depths, d = pos % depths;
    const bool is_new = s_first[static_cast<int64_t>(d) * n + c] == c;
    s_rank[pos] = is_new ? r : -1;
    r += is_new;
  }
  __syncthreads();
  const int count = s_total < budget ? s_total : budget;
  // the kept nodes: rank < budget; node index = rank + 1
  for (int pos = tid; pos < total_pos; pos += kThreads) {
    const int rk = s_rank[pos];
    if (rk < 0 || rk >= budget) continue;
    const int c = pos / depths, d = pos % depths;
    int parent = 0;
    if (d > 0) {
      const int fc = s_first[static_cast<int64_t>(d - 1) * n + c];
      parent = s_rank[fc * depths + d - 1] + 1;
    }
    const int64_t tok = chains[c * chain_stride + d];
    node_token_ids[rk] = tok;
    node_depths[rk] = d + 1;
    parents[rk + 1] = parent;
    s_par[rk + 1] = parent;
    if (verify_ids) verify_ids[rk + 1] = tok;
    if (verify_pos) verify_pos[rk + 1] = start + d + 1;
  }
  if (tid == 0) {
    parents[0] = -1;
    s_par[0] = -1;
    *node_count = count;
    if (verify_ids) verify_ids[0] = root_token ? *root_token : 0;
    if (verify_pos) verify_pos[0] = start;
  }
  __syncthreads();
  // ancestor bitmasks (ancestor-or-self, the root included), rows of unused nodes zeroed
  for (int w = tid; w < (budget + 1) * anc_words; w += kThreads) anc_bits[w] = 0u;
  __syncthreads();
  for (int i = tid; i <= count; i += kThreads) {
    uint32_t* rowp = anc_bits + static_cast<int64_t>(i) * anc_words;
    for (int j = i; j >= 0; j = j > 0 ? s_par[j] : -1) rowp[j >> 5] |= 1u << (j & 31);
  }
}

}  // namespace sampled
}  // namespace ddt

using namespace ddt;

extern "C" int ddt_sample_chains(const void* draft_logits, int dtype, int64_t depths,
                                 int64_t vocab, int64_t row_stride, int64_t num_samples,
                                 float temperature, uint64_t seed, uint64_t offset,
                                 int64_t* chains, void* stream) {
  if (depths < 0 || vocab < 0 || num_samples < 0 || row_stride < vocab) return DDT_ERR_INVALID;
  if (depths == 0 || num_samples == 0) return DDT_OK;
  if (!draft_logits || !chains || vocab == 0) return DDT_ERR_INVALID;
  if (depths > DDT_MAX_DEPTH || vocab >= (int64_t(1) << 32) || num_samples > (int64_t(1) << 20))
    return DDT_ERR_CAPACITY;
  if (!(temperature >= 0.f)) return DDT_ERR_INVALID;
  const int greedy = temperature < 1e-5f;
  const float inv_temp = greedy ? 0.f : 1.0f / temperature;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == DDT_BF16)
    sampled::sample_chains_kernel<true><<<static_cast<unsigned>(depths), sampled::kThreads, 0, st>>>(
        draft_logits, vocab, row_stride, static_cast<int>(depths), static_cast<int>(num_samples),
        inv_temp, greedy, seed, offset, chains);
  else if (dtype == DDT_F32)
    sampled::sample_chains_kernel<false><<<static_cast<unsigned>(depths), sampled::kThreads, 0, st>>>(
        draft_logits, vocab, row_stride, static_cast<int>(depths), static_cast<int>(num_samples),
        inv_temp, greedy, seed, offset, chains);
  else
    return DDT_ERR_DTYPE;
  return launch_status();
}

extern "C" int ddt_chain_tree(const int64_t* chains, int64_t num_chains, int64_t depths,
                              int64_t chain_stride, int64_t budget, int64_t* node_token_ids,
                              int64_t* node_depths, int32_t* parents, int32_t* node_count,
                              uint32_t* anc_bits, int64_t anc_words, const int64_t* root_token,
                              int64_t start, int64_t* verify_ids, int64_t* verify_pos,
                              void* stream) {
  if (num_chains < 0 || depths < 0 || budget < 0) return DDT_ERR_INVALID;
  if (!parents || !node_count || !anc_bits) return DDT_ERR_INVALID;
  if (num_chains > sampled::kMaxChains || depths > DDT_MAX_DEPTH || budget > DDT_MAX_BUDGET)
    return DDT_ERR_CAPACITY;
  if (anc_words * 32 < budget + 1) return DDT_ERR_INVALID;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool empty = num_chains == 0 || depths == 0 || budget == 0;
  if (!empty && (!chains || chain_stride < depths || !node_token_ids || !node_depths))
    return DDT_ERR_INVALID;
  const int n = empty ? 0 : static_cast<int>(num_chains);
  const int L = empty ? 0 : static_cast<int>(depths);
  const size_t smem = sizeof(int64_t) * n + sizeof(int32_t) * (2 * static_cast<size_t>(n) * L +
                                                               static_cast<size_t>(budget) + 1);
  if (cudaFuncSetAttribute(sampled::chain_tree_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return DDT_ERR_CUDA;
  sampled::chain_tree_kernel<<<1, sampled::kThreads, smem, st>>>(
      chains, n, L, chain_stride, static_cast<int>(budget), node_token_ids, node_depths, parents,
      node_count, anc_bits, static_cast<int>(anc_words), root_token, start, verify_ids,
      verify_pos);
  return launch_status();
}
