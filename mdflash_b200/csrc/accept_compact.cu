// Greedy posterior (row argmax), accept walk and KV-cache compaction.
//
// ddt_argmax replaces sample() at temperature 0 (model/utils.py:28-30), i.e.
// torch.argmax over the verify logits (ddtree.py:478): one CTA per row streams the row
// with 16-byte loads and reduces (order key, ~index) composites, so ties resolve to
// the lowest index and NaN (canonicalised to the largest key) wins like in torch.
//
// ddt_accept_compact fuses follow_verified_tree (ddtree.py:270-281) with
// compact_dynamic_cache (ddtree.py:284-335): every CTA replays the short walk from
// shared memory (at most depth + 1 steps), then each warp moves the accepted rows of
// one (tensor, head) slice.  The reference's index_select + copy_ reads all source rows
// before writing; rows may overlap (row past+j is the source of an earlier row when
// accepted[j'] == j), so a warp loads every row of its slice into registers before it
// stores any.  Rows already in place (accepted[j] == j) are skipped.
#include "common.cuh"

namespace ddt {
namespace accept {

constexpr int kArgmaxThreads = 512;
constexpr int kCompactWarps = 8;
constexpr int kMaxRows = DDT_MAX_DEPTH + 1;  // accepted rows: root + one per depth
constexpr int kMaxVecPerLane = 24;           // rows * (row bytes / 16) / 32

__device__ __forceinline__ unsigned long long argmax_comp(float x, uint32_t idx) {
  const uint32_t key = isnan(x) ? 0xffffffffu : f32_key(x);
  return (static_cast<unsigned long long>(key) << 32) | static_cast<uint32_t>(~idx);
}

template <bool kBF16>
__global__ void __launch_bounds__(kArgmaxThreads)
argmax_kernel(const void* __restrict__ logits, int64_t cols, int64_t row_stride,
              int64_t* __restrict__ out, int vec_ok) {
  const int64_t r = blockIdx.x;
  const int tid = threadIdx.x;
  unsigned long long best = 0ull;
  if constexpr (kBF16) {
    const uint16_t* row = static_cast<const uint16_t*>(logits) + r * row_stride;
    if (vec_ok) {
      const int64_t nvec = cols / 8;
      const uint4* rv = reinterpret_cast<const uint4*>(row);
      for (int64_t v = tid; v < nvec; v += kArgmaxThreads) {
        const uint4 q = __ldcs(rv + v);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const uint16_t b = static_cast<uint16_t>(w[e >> 1] >> ((e & 1) * 16));
          const unsigned long long c = argmax_comp(bf16_bits_to_f32(b), static_cast<uint32_t>(v * 8 + e));
          best = c > best ? c : best;
        }
      }
      for (int64_t i = nvec * 8 + tid; i < cols; i += kArgmaxThreads) {
        const unsigned long long c = argmax_comp(bf16_bits_to_f32(row[i]), static_cast<uint32_t>(i));
        best = c > best ? c : best;
      }
    } else {
      for (int64_t i = tid; i < cols; i += kArgmaxThreads) {
        const unsigned long long c = argmax_comp(bf16_bits_to_f32(row[i]), static_cast<uint32_t>(i));
        best = c > best ? c : best;
      }
    }
  } else {
    const float* row = static_cast<const float*>(logits) + r * row_stride;
    if (vec_ok) {
      const int64_t nvec = cols / 4;
      const float4* rv = reinterpret_cast<const float4*>(row);
      for (int64_t v = tid; v < nvec; v += kArgmaxThreads) {
        const float4 q = __ldcs(rv + v);
        const float w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const unsigned long long c = argmax_comp(w[e], static_cast<uint32_t>(v * 4 + e));
          best = c > best ? c : best;
        }
      }
      for (int64_t i = nvec * 4 + tid; i < cols; i += kArgmaxThreads) {
        const unsigned long long c = argmax_comp(row[i], static_cast<uint32_t>(i));
        best = c > best ? c : best;
      }
    } else {
      for (int64_t i = tid; i < cols; i += kArgmaxThreads) {
        const unsigned long long c = argmax_comp(row[i], static_cast<uint32_t>(i));
        best = c > best ? c : best;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long y = __shfl_xor_sync(DDT_FULL_MASK, best, o);
    best = y > best ? y : best;
  }
  __shared__ unsigned long long wbest[kArgmaxThreads / 32];
  if ((tid & 31) == 0) wbest[tid >> 5] = best;
  __syncthreads();
  if (tid < 32) {
    unsigned long long b = tid < kArgmaxThreads / 32 ? wbest[tid] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long y = __shfl_xor_sync(DDT_FULL_MASK, b, o);
      b = y > b ? y : b;
    }
    if (tid == 0) out[r] = static_cast<int64_t>(~static_cast<uint32_t>(b));
  }
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
    const int lane = tid;
    int cur = 0, cnt = 1;
    if (lane == 0) s_acc[0] = 0;
    int64_t tok = s_post[0];
    for (;;) {
      int found = -1;
      for (int i = 1 + lane; i < n_nodes; i += 32)
        if (s_par[i] == cur && s_tok[i] == tok) found = i;  // last match, like a dict overwrite
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) found = max(found, __shfl_xor_sync(DDT_FULL_MASK, found, o));
      if (found < 0 || cnt >= kMaxRows) break;
      cur = found;
      if (lane == 0) s_acc[cnt] = cur;
      ++cnt;
      tok = s_post[cur];
    }
    if (lane == 0) {
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

}  // namespace accept
}  // namespace ddt

using namespace ddt;

extern "C" int ddt_argmax(const void* logits, int dtype, int64_t rows, int64_t cols,
                          int64_t row_stride, int64_t* out, void* stream) {
  if (dtype != DDT_F32 && dtype != DDT_BF16) return DDT_ERR_DTYPE;
  if (rows < 0 || cols <= 0 || row_stride < cols || (rows > 0 && (!logits || !out)))
    return DDT_ERR_INVALID;
  if (cols >= (int64_t(1) << 32) - 1 || rows > 0x7fffffff) return DDT_ERR_CAPACITY;
  if (rows == 0) return DDT_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t esz = dtype == DDT_BF16 ? 2 : 4;
  const int vec_ok = aligned(logits, 16) && (row_stride * esz) % 16 == 0;
  if (dtype == DDT_BF16)
    accept::argmax_kernel<true><<<static_cast<unsigned>(rows), accept::kArgmaxThreads, 0, st>>>(
        logits, cols, row_stride, out, vec_ok);
  else
    accept::argmax_kernel<false><<<static_cast<unsigned>(rows), accept::kArgmaxThreads, 0, st>>>(
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
