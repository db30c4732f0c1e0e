// Greedy posterior (row argmax), accept walk and KV-cache compaction.
//
// ddt_argmax replaces sample() at temperature 0 (model/utils.py:28-30), i.e.
// torch.argmax over the verify logits (ddtree.py:478): a cluster of 4 CTAs per row
// streams the row with 16-byte loads and reduces (order key, ~index) composites, so ties
// resolve to the lowest index and NaN (canonicalised to the largest key) wins like in
// torch.
//
// ddt_accept_compact fuses follow_verified_tree (ddtree.py:270-281) with
// compact_dynamic_cache (ddtree.py:284-335): every CTA replays the short walk from
// shared memory (at most depth + 1 steps), then each warp moves the accepted rows of
// one (tensor, head) slice.  The reference's index_select + copy_ reads all source rows
// before writing; rows may overlap (row past+j is the source of an earlier row when
// accepted[j'] == j), so a warp loads every row of its slice into registers before it
// stores any.  Rows already in place (accepted[j] == j) are skipped.
#include <cooperative_groups.h>

#include "common.cuh"

namespace ddt {
namespace accept {

constexpr int kArgmaxThreads = 256;
constexpr int kArgmaxCluster = 4;  // CTAs per row (rows * 4 CTAs fit in one wave at N = 257)
constexpr int kCompactWarps = 8;
constexpr int kMaxRows = DDT_MAX_DEPTH + 1;  // accepted rows: root + one per depth
constexpr int kMaxVecPerLane = 24;           // rows * (row bytes / 16) / 32

// Order keys of the two bf16 in a 32-bit word, per 16-bit half: 0x8000 + |b| for positive
// values and 0x8000 - |b| for negative ones, so -0 and +0 share 0x8000 and the order is that
// of argmax_comp on the fp32 value for all numbers; NaNs land above +inf's key (0xff80) when
// positive and below -inf's (0x0080) when negative, which the caller checks for.
// prmt replicates each half's sign bit over the half (0xffff in negative halves); the add
// (x ^ neg) + 0x8000 - neg stays within each half, so one 32-bit add serves both.
__device__ __forceinline__ uint32_t bf16x2_order_keys(uint32_t w) {
  uint32_t neg;
  asm("prmt.b32 %0, %1, 0, 0xbb99;" : "=r"(neg) : "r"(w));
  return ((w & 0x7fff7fffu) ^ neg) + 0x80008000u - neg;
}

__device__ __forceinline__ unsigned long long argmax_comp(float x, uint32_t idx) {
  const uint32_t key = isnan(x) ? 0xffffffffu : f32_key(x);
  return (static_cast<unsigned long long>(key) << 32) | static_cast<uint32_t>(~idx);
}

// One thread-block cluster of kArgmaxCluster CTAs per row: CTA c streams the c-th
// contiguous chunk of the row (four 16-byte loads in flight per thread), reduces it to one
// composite, and cluster rank 0 combines the cluster's composites through distributed
// shared memory.  Rows are spread over rows * 8 CTAs instead of one CTA per row, which
// left SMs idle and each thread with a single load in flight.
template <bool kBF16>
__global__ void __cluster_dims__(kArgmaxCluster, 1, 1) __launch_bounds__(kArgmaxThreads)
argmax_kernel(const void* __restrict__ logits, int64_t cols, int64_t row_stride,
              int64_t* __restrict__ out, int vec_ok) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int part = static_cast<int>(cluster.block_rank());
  const int64_t r = blockIdx.x / kArgmaxCluster;
  const int tid = threadIdx.x;
  constexpr int kPer = kBF16 ? 8 : 4;  // elements per 16-byte vector
  constexpr int kUnroll = 8;  // 16-byte loads in flight per thread
  unsigned long long best = 0ull;
  auto take = [&](float x, int64_t i) {
    const unsigned long long c = argmax_comp(x, static_cast<uint32_t>(i));
    best = c > best ? c : best;
  };
  auto elem = [&](int64_t i) -> float {
    if constexpr (kBF16)
      return bf16_bits_to_f32(static_cast<const uint16_t*>(logits)[r * row_stride + i]);
    else
      return static_cast<const float*>(logits)[r * row_stride + i];
  };
  // element range [e0, e1) of this CTA; with 16-byte loads the split is in whole vectors
  // and the last CTA also takes the ragged tail
  const int64_t unit = vec_ok ? kPer : 1;
  const int64_t units = cols / unit;
  const int64_t per = (units + kArgmaxCluster - 1) / kArgmaxCluster;
  const int64_t u0 = part * per < units ? part * per : units;
  const int64_t u1 = (part + 1) * per < units ? (part + 1) * per : units;
  if (vec_ok) {
    const uint4* rv = reinterpret_cast<const uint4*>(static_cast<const char*>(logits) +
                                                     r * row_stride * (kBF16 ? 2 : 4));
    // bf16: order keys on packed 16-bit halves (bf16x2_order_keys: three instructions per
    // pair) and packed 16-bit max / min trees per 16-byte vector; a thread keeps
    // (best vector key << 16 | 0xffff - vector ordinal) and only re-reads its winning vector
    // to find the first element holding that key.  NaNs (positive: keys above +inf's, negative:
    // keys below -inf's) send the thread to the exact per-element path.  About three
    // instructions per element; a 64-bit composite per element made the kernel issue-bound.
    if (kBF16 && per <= static_cast<int64_t>(kArgmaxThreads) * 0xfff0) {
      uint32_t bestc = 0u, kmin = 0xffffffffu, m = 0u;
      for (int64_t v = u0 + tid; v < u1; v += kUnroll * kArgmaxThreads) {
        uint4 q[kUnroll];
#pragma unroll
        for (int k = 0; k < kUnroll; ++k) {
          const int64_t vi = v + k * kArgmaxThreads;
          q[k] = vi < u1 ? __ldcs(rv + vi) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int k = 0; k < kUnroll; ++k) {
          if (v + k * kArgmaxThreads >= u1) break;
          const uint32_t k0 = bf16x2_order_keys(q[k].x), k1 = bf16x2_order_keys(q[k].y);
          const uint32_t k2 = bf16x2_order_keys(q[k].z), k3 = bf16x2_order_keys(q[k].w);
          const uint32_t kx = __vmaxu2(__vmaxu2(k0, k1), __vmaxu2(k2, k3));
          kmin = __vminu2(kmin, __vminu2(__vminu2(k0, k1), __vminu2(k2, k3)));
          const uint32_t vk = max(kx >> 16, kx & 0xffffu);
          bestc = max(bestc, (vk << 16) | (0xffffu - m));
          ++m;
        }
      }
      const bool has_nan = (bestc >> 16) > 0xff80u || (kmin & 0xffffu) < 0x0080u ||
                           (kmin >> 16) < 0x0080u;
      if (has_nan) {
        for (int64_t vi = u0 + tid; vi < u1; vi += kArgmaxThreads) {
          const uint4 q = rv[vi];
          const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int e = 0; e < 8; ++e)
            take(bf16_bits_to_f32(static_cast<uint16_t>(w[e >> 1] >> ((e & 1) * 16))), vi * 8 + e);
        }
      } else if (bestc) {
        const uint32_t kbest = bestc >> 16;
        const int64_t vi = u0 + tid + static_cast<int64_t>(0xffffu - (bestc & 0xffffu)) * kArgmaxThreads;
        const uint4 q = rv[vi];
        const uint32_t kw[4] = {bf16x2_order_keys(q.x), bf16x2_order_keys(q.y),
                                bf16x2_order_keys(q.z), bf16x2_order_keys(q.w)};
        int e = 7;
#pragma unroll
        for (int x = 7; x >= 0; --x)
          if (((kw[x >> 1] >> ((x & 1) * 16)) & 0xffffu) == kbest) e = x;
        // the 32-bit key of the same value as argmax_comp builds it from the fp32 value
        const uint32_t key32 = kbest >= 0x8000u ? kbest << 16 : ((kbest - 1u) << 16) | 0xffffu;
        best = (static_cast<unsigned long long>(key32) << 32) |
               static_cast<uint32_t>(~static_cast<uint32_t>(vi * 8 + e));
      }
    } else {
      // fp32 (and very long bf16 rows): a 64-bit composite per element
      for (int64_t v = u0 + tid; v < u1; v += kUnroll * kArgmaxThreads) {
        uint4 q[kUnroll];
#pragma unroll
        for (int k = 0; k < kUnroll; ++k) {
          const int64_t vi = v + k * kArgmaxThreads;
          q[k] = vi < u1 ? __ldcs(rv + vi) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int k = 0; k < kUnroll; ++k) {
          const int64_t vi = v + k * kArgmaxThreads;
          if (vi >= u1) break;
          const uint32_t w[4] = {q[k].x, q[k].y, q[k].z, q[k].w};
          if constexpr (kBF16) {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              take(bf16_bits_to_f32(static_cast<uint16_t>(w[e >> 1] >> ((e & 1) * 16))),
                   vi * 8 + e);
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) take(__uint_as_float(w[e]), vi * 4 + e);
          }
        }
      }
    }
    if (part == kArgmaxCluster - 1)
      for (int64_t i = units * kPer + tid; i < cols; i += kArgmaxThreads) take(elem(i), i);
  } else {
    for (int64_t i = u0 + tid; i < u1; i += kArgmaxThreads) take(elem(i), i);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long y = __shfl_xor_sync(DDT_FULL_MASK, best, o);
    best = y > best ? y : best;
  }
  __shared__ unsigned long long wbest[kArgmaxThreads / 32];
  __shared__ unsigned long long cta_best;
  if ((tid & 31) == 0) wbest[tid >> 5] = best;
  __syncthreads();
  if (tid < 32) {
    unsigned long long b = tid < kArgmaxThreads / 32 ? wbest[tid] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long y = __shfl_xor_sync(DDT_FULL_MASK, b, o);
      b = y > b ? y : b;
    }
    if (tid == 0) cta_best = b;
  }
  cluster.sync();
  if (part == 0 && tid < 32) {
    unsigned long long b = tid < kArgmaxCluster ? *cluster.map_shared_rank(&cta_best, tid) : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long y = __shfl_xor_sync(DDT_FULL_MASK, b, o);
      b = y > b ? y : b;
    }
    if (tid == 0) out[r] = static_cast<int64_t>(~static_cast<uint32_t>(b));
  }
  cluster.sync();  // every CTA's shared memory stays live until rank 0 has read it
}

struct KvDesc {
  void* const* ptrs;
  int64_t n_tensors, heads, head_stride, seq_stride;  // strides in elements
  int elem_bytes, vec_per_row;                         // 16-byte vectors per row
  int64_t past_length;
};

// Moves rows past + keep[j] -> past + j (j < cnt) for one (tensor, head) slice.  The
// whole slice is staged in registers before any store.
__device__ __forceinline__ void move_slice(const KvDesc& kv, int64_t slice, const int64_t* keep,
                                           int cnt, int lane) {
  const int64_t t = slice / kv.heads;
  const int64_t h = slice % kv.heads;
  unsigned char* base = static_cast<unsigned char*>(kv.ptrs[t]) +
                        (h * kv.head_stride + kv.past_length * kv.seq_stride) * kv.elem_bytes;
  const int64_t row_bytes = kv.seq_stride * kv.elem_bytes;
  const int total = cnt * kv.vec_per_row;
  uint4 buf[kMaxVecPerLane];
#pragma unroll
  for (int i = 0; i < kMaxVecPerLane; ++i) {
    const int v = i * 32 + lane;
    if (v < total) {
      const int j = v / kv.vec_per_row, c = v % kv.vec_per_row;
      if (keep[j] != j)
        buf[i] = *reinterpret_cast<const uint4*>(base + keep[j] * row_bytes + c * 16);
    }
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < kMaxVecPerLane; ++i) {
    const int v = i * 32 + lane;
    if (v < total) {
      const int j = v / kv.vec_per_row, c = v % kv.vec_per_row;
      if (keep[j] != j) *reinterpret_cast<uint4*>(base + j * row_bytes + c * 16) = buf[i];
    }
  }
}

// follow_verified_tree (ddtree.py:270-281) by one warp over a tree staged in shared memory
// (s_par: parents, s_tok: node tokens with -1 for the root, s_post: posterior): from the root,
// repeatedly the child whose token is the posterior of the current node (the last such child
// in node order, as a dict built in node order keeps), at most kMaxRows nodes.  Lane 0 writes
// the accepted node indices to acc; returns their count and sets next (the posterior of the
// last accepted node) on every lane.
__device__ __forceinline__ int walk_tree(const int32_t* s_par, const int64_t* s_tok,
                                         const int64_t* s_post, int n_nodes, int64_t* acc,
                                         int64_t& next) {
  const int lane = threadIdx.x & 31;
  int cur = 0, cnt = 1;
  if (lane == 0) acc[0] = 0;
  int64_t tok = s_post[0];
  for (;;) {
    int found = -1;
    for (int i = 1 + lane; i < n_nodes; i += 32)
      if (s_par[i] == cur && s_tok[i] == tok) found = i;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) found = max(found, __shfl_xor_sync(DDT_FULL_MASK, found, o));
    if (found < 0 || cnt >= kMaxRows) break;
    cur = found;
    if (lane == 0) acc[cnt] = cur;
    ++cnt;
    tok = s_post[cur];
  }
  next = tok;
  return cnt;
}

// walk + compaction; every CTA replays the walk (it is a few shared-memory steps).
__global__ void __launch_bounds__(kCompactWarps * 32)
accept_compact_kernel(const int64_t* __restrict__ posterior, const int32_t* __restrict__ parents,
                      const int64_t* __restrict__ node_ids, int n_nodes, KvDesc kv,
                      int64_t* __restrict__ accepted, int32_t* __restrict__ n_accepted,
                      int64_t* __restrict__ next_token) {
  extern __shared__ __align__(16) unsigned char smem[];
  int32_t* s_par = reinterpret_cast<int32_t*>(smem);
  int64_t* s_tok = reinterpret_cast<int64_t*>(smem + ((sizeof(int32_t) * n_nodes + 15) / 16) * 16);
  int64_t* s_post = s_tok + n_nodes;
  __shared__ int64_t s_acc[kMaxRows];
  __shared__ int s_cnt;
  __shared__ int64_t s_next;
  const int tid = threadIdx.x;
  for (int i = tid; i < n_nodes; i += blockDim.x) {
    s_par[i] = parents[i];
    s_tok[i] = i > 0 ? node_ids[i - 1] : -1;
    s_post[i] = posterior[i];
  }
  __syncthreads();
  if (tid < 32) {
    int64_t tok;
    const int cnt = walk_tree(s_par, s_tok, s_post, n_nodes, s_acc, tok);
    if (tid == 0) {
      s_cnt = cnt;
      s_next = tok;
    }
  }
  __syncthreads();
  const int cnt = s_cnt;
  if (blockIdx.x == 0) {
    for (int i = tid; i < cnt; i += blockDim.x) accepted[i] = s_acc[i];
    if (tid == 0) {
      *n_accepted = cnt;
      *next_token = s_next;
    }
  }
  const int lane = tid & 31;
  const int64_t nslices = kv.n_tensors * kv.heads;
  for (int64_t sl = static_cast<int64_t>(blockIdx.x) * kCompactWarps + (tid >> 5); sl < nslices;
       sl += static_cast<int64_t>(gridDim.x) * kCompactWarps)
    move_slice(kv, sl, s_acc, cnt, lane);
}

__global__ void __launch_bounds__(kCompactWarps * 32)
compact_kernel(const int64_t* __restrict__ keep, int cnt, KvDesc kv) {
  __shared__ int64_t s_keep[kMaxRows];
  if (threadIdx.x < cnt) s_keep[threadIdx.x] = keep[threadIdx.x];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t nslices = kv.n_tensors * kv.heads;
  for (int64_t sl = static_cast<int64_t>(blockIdx.x) * kCompactWarps + (threadIdx.x >> 5);
       sl < nslices; sl += static_cast<int64_t>(gridDim.x) * kCompactWarps)
    move_slice(kv, sl, s_keep, cnt, lane);
}

// ---- batched: the walks of all requests, then all their compactions (two launches) ----

// move_slice with the slice staged in shared memory (stage: this warp's kMaxRows x
// vec_per_row vectors) instead of registers, so a CTA needs few registers and many warps
// per SM keep loads in flight.
__device__ __forceinline__ void move_slice_smem(const KvDesc& kv, int64_t slice,
                                                const int64_t* keep, int cnt, int lane,
                                                uint4* stage) {
  const int64_t t = slice / kv.heads;
  const int64_t h = slice % kv.heads;
  unsigned char* base = static_cast<unsigned char*>(kv.ptrs[t]) +
                        (h * kv.head_stride + kv.past_length * kv.seq_stride) * kv.elem_bytes;
  const int64_t row_bytes = kv.seq_stride * kv.elem_bytes;
  const int total = cnt * kv.vec_per_row;
  for (int v = lane; v < total; v += 32) {
    const int j = v / kv.vec_per_row, c = v % kv.vec_per_row;
    if (keep[j] != j) stage[v] = *reinterpret_cast<const uint4*>(base + keep[j] * row_bytes + c * 16);
  }
  __syncwarp();
  for (int v = lane; v < total; v += 32) {
    const int j = v / kv.vec_per_row, c = v % kv.vec_per_row;
    if (keep[j] != j) *reinterpret_cast<uint4*>(base + j * row_bytes + c * 16) = stage[v];
  }
  __syncwarp();  // the stage is reused for the warp's next slice
}
// Walk of request blockIdx.x (one warp): its tree is staged in shared memory, then walked
// as in accept_compact_kernel; writes accepted[r], n_accepted[r], next_token[r].
__global__ void __launch_bounds__(32)
accept_walk_batched_kernel(const int64_t* __restrict__ posterior, int64_t post_stride,
                           const int32_t* __restrict__ parents, int64_t par_stride,
                           const int64_t* __restrict__ node_ids, int64_t ids_stride,
                           const int32_t* __restrict__ node_counts, int max_nodes,
                           int64_t* __restrict__ accepted, int64_t acc_stride,
                           int32_t* __restrict__ n_accepted, int64_t* __restrict__ next_token) {
  extern __shared__ __align__(16) unsigned char smem[];
  int32_t* s_par = reinterpret_cast<int32_t*>(smem);
  int64_t* s_tok = reinterpret_cast<int64_t*>(smem + ((sizeof(int32_t) * max_nodes + 15) / 16) * 16);
  int64_t* s_post = s_tok + max_nodes;
  const int lane = threadIdx.x;
  const int r = blockIdx.x;
  int n_nodes = node_counts[r] + 1;
  if (n_nodes > max_nodes) n_nodes = max_nodes;
  if (n_nodes < 1) n_nodes = 1;
  const int32_t* par = parents + r * par_stride;
  const int64_t* ids = node_ids + r * ids_stride;
  const int64_t* post = posterior + r * post_stride;
  for (int i = lane; i < n_nodes; i += 32) {
    s_par[i] = par[i];
    s_tok[i] = i > 0 ? ids[i - 1] : -1;
    s_post[i] = post[i];
  }
  __syncwarp();
  int64_t tok;
  const int cnt = walk_tree(s_par, s_tok, s_post, n_nodes, accepted + r * acc_stride, tok);
  if (lane == 0) {
    n_accepted[r] = cnt;
    next_token[r] = tok;
  }
}

// Compaction of every request's cache after accept_walk_batched_kernel: G CTAs per request;
// request r's tensors are kv_ptrs[r * n_tensors + t], with head_strides[r] elements per head
// and prefix past[r].  A request whose head stride is not a whole number of 16-byte vectors
// (checked here, since the strides live on the device) moves nothing and sets *status.
struct KvBatch {
  void* const* ptrs;
  const int64_t* head_strides;
  const int64_t* past;
  int64_t n_tensors, heads, seq_stride;
  int elem_bytes, vec_per_row;
};

__global__ void __launch_bounds__(kCompactWarps * 32)
compact_batched_kernel(const int64_t* __restrict__ accepted, int64_t acc_stride,
                       const int32_t* __restrict__ n_accepted, KvBatch kb, int G, int* status) {
  extern __shared__ __align__(16) unsigned char stage_raw[];
  __shared__ int64_t s_acc[kMaxRows];
  const int tid = threadIdx.x;
  const int r = blockIdx.x / G, g = blockIdx.x % G;
  int cnt = n_accepted[r];
  cnt = cnt < 0 ? 0 : (cnt > kMaxRows ? kMaxRows : cnt);
  if (tid < cnt) s_acc[tid] = accepted[r * acc_stride + tid];
  __syncthreads();
  const int64_t hs = kb.head_strides[r];
  if ((hs * kb.elem_bytes) % 16 != 0) {
    if (g == 0 && tid == 0 && status) atomicOr(status, 2);
    return;
  }
  KvDesc kv;
  kv.ptrs = kb.ptrs + r * kb.n_tensors;
  kv.n_tensors = kb.n_tensors;
  kv.heads = kb.heads;
  kv.head_stride = hs;
  kv.seq_stride = kb.seq_stride;
  kv.elem_bytes = kb.elem_bytes;
  kv.vec_per_row = kb.vec_per_row;
  kv.past_length = kb.past[r];
  const int lane = tid & 31;
  uint4* stage = reinterpret_cast<uint4*>(stage_raw) + (tid >> 5) * kMaxRows * kb.vec_per_row;
  const int64_t nslices = kv.n_tensors * kv.heads;
  for (int64_t sl = static_cast<int64_t>(g) * kCompactWarps + (tid >> 5); sl < nslices;
       sl += static_cast<int64_t>(G) * kCompactWarps)
    move_slice_smem(kv, sl, s_acc, cnt, lane, stage);
}

inline int make_desc(void* const* kv_ptrs, int64_t n_tensors, int64_t heads, int64_t head_dim,
                     int64_t head_stride, int64_t seq_stride, int64_t elem_bytes,
                     int64_t past_length, KvDesc* d) {
  if (!kv_ptrs || n_tensors < 0 || heads <= 0 || head_dim <= 0 || past_length < 0)
    return DDT_ERR_INVALID;
  if (elem_bytes != 2 && elem_bytes != 4) return DDT_ERR_DTYPE;
  const int64_t row_bytes = head_dim * elem_bytes;
  if (row_bytes % 16 || (seq_stride * elem_bytes) % 16 || (head_stride * elem_bytes) % 16)
    return DDT_ERR_ALIGN;
  if (seq_stride < head_dim) return DDT_ERR_INVALID;
  d->ptrs = kv_ptrs;
  d->n_tensors = n_tensors;
  d->heads = heads;
  d->head_stride = head_stride;
  d->seq_stride = seq_stride;
  d->elem_bytes = static_cast<int>(elem_bytes);
  d->vec_per_row = static_cast<int>(row_bytes / 16);
  d->past_length = past_length;
  if (static_cast<int64_t>(kMaxRows) * d->vec_per_row > 32 * kMaxVecPerLane) return DDT_ERR_CAPACITY;
  return DDT_OK;
}

inline unsigned compact_grid(int64_t n_tensors, int64_t heads) {
  const int64_t slices = n_tensors * heads;
  int64_t g = (slices + kCompactWarps - 1) / kCompactWarps;
  if (g < 1) g = 1;
  if (g > 4 * 148) g = 4 * 148;
  return static_cast<unsigned>(g);
}

// One decode-loop round's bookkeeping on the device, after the walk (ddtree.py:488-498): the
// accepted tokens and the next token go to the output row at the round's start, the next
// token becomes the next round's root, the acceptance length is logged and the start
// advances.  One warp per request; writes beyond a buffer's capacity are dropped and set
// status bit 8.
constexpr int kStatusLogFull = 8;

__global__ void advance_round_kernel(int64_t* __restrict__ starts, int32_t* __restrict__ rounds,
                                     const int32_t* __restrict__ n_accepted,
                                     const int64_t* __restrict__ accepted, int64_t acc_stride,
                                     const int64_t* __restrict__ verify_ids, int64_t ids_stride,
                                     const int64_t* __restrict__ next_token,
                                     int64_t* __restrict__ root_tokens,
                                     int64_t* __restrict__ output_ids, int64_t out_stride,
                                     int64_t out_capacity, int32_t* __restrict__ acceptance,
                                     int64_t len_stride, int64_t len_capacity, int max_nodes,
                                     int* status) {
  const int r = blockIdx.x;
  const int lane = threadIdx.x;
  const int64_t start = starts[r];
  int k = n_accepted[r];
  k = k < 0 ? 0 : (k > max_nodes ? max_nodes : k);
  const int64_t tok = next_token[r];
  bool dropped = false;
  for (int i = lane; i <= k; i += 32) {
    const int64_t pos = start + i;
    if (pos < 0 || pos >= out_capacity) {
      dropped = true;
      continue;
    }
    int64_t t = tok;
    if (i < k) {
      const int64_t node = accepted[r * acc_stride + i];
      t = (node >= 0 && node < max_nodes) ? verify_ids[r * ids_stride + node] : -1;
    }
    output_ids[r * out_stride + pos] = t;
  }
  dropped = __any_sync(DDT_FULL_MASK, dropped);
  if (lane == 0) {
    const int32_t round = rounds[r];
    if (round >= 0 && round < len_capacity) acceptance[r * len_stride + round] = k;
    else dropped = true;
    rounds[r] = round + 1;
    starts[r] = start + k;
    root_tokens[r] = tok;
    if (dropped && status) atomicOr(status, kStatusLogFull);
  }
}

// out[i] = src[idx[i]] for i < *count (count read on the device, clamped to max_rows), rows of
// row_vecs 16-byte vectors at the given strides; one warp per output row.  An index outside
// [0, src_rows) writes zeros.
__global__ void gather_rows_kernel(const uint4* __restrict__ src, int64_t src_stride_vec,
                                   int64_t src_rows, const int64_t* __restrict__ idx,
                                   const int32_t* __restrict__ count, int max_rows,
                                   uint4* __restrict__ out, int64_t out_stride_vec,
                                   int64_t row_vecs) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  int n = count ? *count : max_rows;
  n = n < 0 ? 0 : (n > max_rows ? max_rows : n);
  if (row >= n) return;
  const int64_t s = idx[row];
  const bool ok = s >= 0 && s < src_rows;
  const uint4* sp = src + (ok ? s : 0) * src_stride_vec;
  uint4* op = out + static_cast<int64_t>(row) * out_stride_vec;
  for (int64_t v = lane; v < row_vecs; v += 32) op[v] = ok ? __ldg(sp + v) : make_uint4(0, 0, 0, 0);
}

}  // namespace accept
}  // namespace ddt

using namespace ddt;

extern "C" int ddt_argmax(const void* logits, int dtype, int64_t rows, int64_t cols,
                          int64_t row_stride, int64_t* out, void* stream) {
  if (dtype != DDT_F32 && dtype != DDT_BF16) return DDT_ERR_DTYPE;
  if (rows < 0 || cols <= 0 || row_stride < cols || (rows > 0 && (!logits || !out)))
    return DDT_ERR_INVALID;
  if (cols >= (int64_t(1) << 32) - 1 || rows > 0x7fffffff / accept::kArgmaxCluster)
    return DDT_ERR_CAPACITY;
  if (rows == 0) return DDT_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t esz = dtype == DDT_BF16 ? 2 : 4;
  const int vec_ok = aligned(logits, 16) && (row_stride * esz) % 16 == 0;
  if (dtype == DDT_BF16)
    accept::argmax_kernel<true><<<static_cast<unsigned>(rows * accept::kArgmaxCluster),
                                  accept::kArgmaxThreads, 0, st>>>(
        logits, cols, row_stride, out, vec_ok);
  else
    accept::argmax_kernel<false><<<static_cast<unsigned>(rows * accept::kArgmaxCluster),
                                   accept::kArgmaxThreads, 0, st>>>(
        logits, cols, row_stride, out, vec_ok);
  return launch_status();
}

extern "C" int ddt_accept_compact(const int64_t* posterior, const int32_t* parents,
                                  const int64_t* node_token_ids, int64_t n_nodes,
                                  void* const* kv_ptrs, int64_t n_tensors, int64_t heads,
                                  int64_t head_dim, int64_t head_stride, int64_t seq_stride,
                                  int64_t elem_bytes, int64_t past_length, int64_t* accepted,
                                  int32_t* n_accepted, int64_t* next_token, void* stream) {
  if (!posterior || !parents || !accepted || !n_accepted || !next_token) return DDT_ERR_INVALID;
  if (n_nodes < 1) return DDT_ERR_INVALID;
  if (n_nodes > DDT_MAX_NODES) return DDT_ERR_CAPACITY;
  if (n_nodes > 1 && !node_token_ids) return DDT_ERR_INVALID;
  accept::KvDesc kv;
  int rc = accept::make_desc(kv_ptrs, n_tensors, heads, head_dim, head_stride, seq_stride,
                             elem_bytes, past_length, &kv);
  if (rc != DDT_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t smem = ((sizeof(int32_t) * n_nodes + 15) / 16) * 16 + 2 * sizeof(int64_t) * n_nodes;
  accept::accept_compact_kernel<<<accept::compact_grid(n_tensors, heads), accept::kCompactWarps * 32,
                                  smem, st>>>(posterior, parents, node_token_ids,
                                              static_cast<int>(n_nodes), kv, accepted, n_accepted,
                                              next_token);
  return launch_status();
}

extern "C" int ddt_compact_kv(const int64_t* keep, int64_t keep_count, void* const* kv_ptrs,
                              int64_t n_tensors, int64_t heads, int64_t head_dim,
                              int64_t head_stride, int64_t seq_stride, int64_t elem_bytes,
                              int64_t past_length, void* stream) {
  if (keep_count < 0 || (keep_count > 0 && !keep)) return DDT_ERR_INVALID;
  if (keep_count > accept::kMaxRows) return DDT_ERR_CAPACITY;
  accept::KvDesc kv;
  int rc = accept::make_desc(kv_ptrs, n_tensors, heads, head_dim, head_stride, seq_stride,
                             elem_bytes, past_length, &kv);
  if (rc != DDT_OK) return rc;
  if (keep_count == 0 || n_tensors == 0) return DDT_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  accept::compact_kernel<<<accept::compact_grid(n_tensors, heads), accept::kCompactWarps * 32, 0,
                           st>>>(keep, static_cast<int>(keep_count), kv);
  return launch_status();
}

extern "C" int ddt_accept_compact_batched(
    int64_t n_requests, const int64_t* posterior, int64_t post_stride, const int32_t* parents,
    int64_t par_stride, const int64_t* node_token_ids, int64_t ids_stride,
    const int32_t* node_counts, int64_t max_nodes, void* const* kv_ptrs, int64_t n_tensors,
    int64_t heads, int64_t head_dim, const int64_t* head_strides, int64_t seq_stride,
    int64_t elem_bytes, const int64_t* past_lengths, int64_t* accepted, int64_t acc_stride,
    int32_t* n_accepted, int64_t* next_token, int32_t* status, void* stream) {
  if (n_requests < 0 || !posterior || !parents || !node_token_ids || !node_counts ||
      !head_strides || !past_lengths || !accepted || !n_accepted || !next_token)
    return DDT_ERR_INVALID;
  if (max_nodes < 1 || post_stride < max_nodes || par_stride < max_nodes ||
      ids_stride < max_nodes - 1 || acc_stride < 1)
    return DDT_ERR_INVALID;
  if (max_nodes > DDT_MAX_NODES) return DDT_ERR_CAPACITY;
  accept::KvDesc d;
  int rc = accept::make_desc(kv_ptrs, n_tensors, heads, head_dim, 0, seq_stride, elem_bytes, 0, &d);
  if (rc != DDT_OK) return rc;
  if (acc_stride < accept::kMaxRows && acc_stride < max_nodes) return DDT_ERR_INVALID;
  if (n_requests == 0) return DDT_OK;
  const unsigned per = accept::compact_grid(n_tensors, heads) / 4 > 0
                           ? (accept::compact_grid(n_tensors, heads) + 3) / 4 : 1u;
  if (static_cast<int64_t>(per) * n_requests > 0x7fffffffLL) return DDT_ERR_CAPACITY;
  accept::KvBatch kb{kv_ptrs, head_strides, past_lengths, n_tensors, heads, seq_stride,
                     d.elem_bytes, d.vec_per_row};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t smem = ((sizeof(int32_t) * max_nodes + 15) / 16) * 16 + 2 * sizeof(int64_t) * max_nodes;
  accept::accept_walk_batched_kernel<<<static_cast<unsigned>(n_requests), 32, smem, st>>>(
      posterior, post_stride, parents, par_stride, node_token_ids, ids_stride, node_counts,
      static_cast<int>(max_nodes), accepted, acc_stride, n_accepted, next_token);
  rc = launch_status();
  if (rc != DDT_OK || n_tensors == 0) return rc;
  const size_t stage = static_cast<size_t>(accept::kCompactWarps) * accept::kMaxRows *
                       d.vec_per_row * 16;
  if (cudaFuncSetAttribute(accept::compact_batched_kernel,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(stage)) != cudaSuccess)
    return DDT_ERR_CUDA;
  accept::compact_batched_kernel<<<static_cast<unsigned>(per * n_requests),
                                   accept::kCompactWarps * 32, stage, st>>>(
      accepted, acc_stride, n_accepted, kb, static_cast<int>(per), status);
  return launch_status();
}

extern "C" int ddt_advance_round(int64_t n_requests, int64_t* starts, int32_t* rounds,
                                 const int32_t* n_accepted, const int64_t* accepted,
                                 int64_t acc_stride, const int64_t* verify_ids,
                                 int64_t ids_stride, int64_t max_nodes,
                                 const int64_t* next_token, int64_t* root_tokens,
                                 int64_t* output_ids, int64_t out_stride, int64_t out_capacity,
                                 int32_t* acceptance, int64_t len_stride, int64_t len_capacity,
                                 int32_t* status, void* stream) {
  if (n_requests < 0 || !starts || !rounds || !n_accepted || !accepted || !verify_ids ||
      !next_token || !root_tokens || !output_ids || !acceptance)
    return DDT_ERR_INVALID;
  if (max_nodes < 1 || max_nodes > DDT_MAX_NODES || acc_stride < 1 || ids_stride < max_nodes ||
      out_capacity < 1 || out_stride < out_capacity || len_capacity < 1 ||
      len_stride < len_capacity)
    return DDT_ERR_INVALID;
  if (n_requests == 0) return DDT_OK;
  if (n_requests > 0x7fffffffLL) return DDT_ERR_CAPACITY;
  accept::advance_round_kernel<<<static_cast<unsigned>(n_requests), 32, 0,
                                 static_cast<cudaStream_t>(stream)>>>(
      starts, rounds, n_accepted, accepted, acc_stride, verify_ids, ids_stride, next_token,
      root_tokens, output_ids, out_stride, out_capacity, acceptance, len_stride, len_capacity,
      static_cast<int>(max_nodes), status);
  return launch_status();
}

extern "C" int ddt_gather_rows(const void* src, int64_t src_rows, int64_t src_row_stride,
                               const int64_t* idx, const int32_t* count, int64_t max_rows,
                               void* out, int64_t out_row_stride, int64_t row_bytes,
                               void* stream) {
  if (!src || !idx || !out || src_rows < 0 || max_rows < 0 || row_bytes < 0) return DDT_ERR_INVALID;
  if (row_bytes % 16 || src_row_stride % 16 || out_row_stride % 16 || !aligned(src, 16) ||
      !aligned(out, 16))
    return DDT_ERR_ALIGN;
  if (src_row_stride < row_bytes || out_row_stride < row_bytes) return DDT_ERR_INVALID;
  if (max_rows == 0 || row_bytes == 0) return DDT_OK;
  if (max_rows > 0x7fffffffLL) return DDT_ERR_CAPACITY;
  constexpr int kWarps = 4;
  accept::gather_rows_kernel<<<static_cast<unsigned>((max_rows + kWarps - 1) / kWarps),
                               kWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), src_row_stride / 16, src_rows, idx, count,
      static_cast<int>(max_rows), static_cast<uint4*>(out), out_row_stride / 16, row_bytes / 16);
  return launch_status();
}
