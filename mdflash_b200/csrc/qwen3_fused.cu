// Fused elementwise stages of the Qwen3 verify forward.
//
// transformers runs each of these as a chain of small kernels (about 55 launches per
// decoder layer at verify size); here each is one launch that reads and writes the
// activations once.  The bf16 rounding points of the transformers code are kept:
//   ddt_add_rmsnorm          residual + hidden (bf16 add), Qwen3RMSNorm
//                            (modeling_qwen3.py:59-64: fp32 x * rsqrt(mean(x^2) + eps),
//                            cast to bf16, then weight * x in bf16)
//   ddt_qk_norm_rope_cache   q_norm / k_norm (the same RMSNorm over head_dim,
//                            modeling_qwen3.py:263-264), rotary embedding
//                            (Qwen3RotaryEmbedding.forward :137-147 builds cos / sin in
//                            fp32 and casts them to bf16; apply_rotary_pos_emb :151-181
//                            rounds q*cos, rotate_half(q)*sin and their sum to bf16),
//                            and the KV-cache write that DynamicLayer.update does with
//                            torch.cat (cache_utils.py:119-120), in place at rows past + i;
//                            the _table form reads cos / sin from ddt_rope_table's table,
//                            built once per forward (the same values)
//   ddt_silu_mul             Qwen3MLP.forward (:81-83): bf16(silu(gate)) * up in bf16
#include <cuda_bf16.h>

#include "common.cuh"

namespace ddt {
namespace fused {

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(DDT_FULL_MASK, v, o);
  return v;
}

// One CTA per row: hidden / 8 vectors of 8 elements, spread over at most 512 threads in
// kPasses <= 4 passes.  The weight vectors are loaded together with the row, before the
// reduction, so that their latency overlaps it.
constexpr int kNormThreads = 512;
constexpr int kNormMaxPasses = 4;

__device__ __forceinline__ uint4 ld16(const __nv_bfloat16* p) { return *reinterpret_cast<const uint4*>(p); }

template <int kPasses>
__global__ void __launch_bounds__(kNormThreads)
add_rmsnorm_kernel(const __nv_bfloat16* x, const __nv_bfloat16* __restrict__ delta,
                   const __nv_bfloat16* __restrict__ w, int hidden, float eps,
                   __nv_bfloat16* residual_out, __nv_bfloat16* __restrict__ norm_out) {
  // residual_out may alias x: each thread reads its elements before it writes them
  const long long row = blockIdx.x;
  const int tid = threadIdx.x;
  const int nthr = blockDim.x;
  const int vecs = hidden >> 3;
  const __nv_bfloat16* xr = x + row * hidden;
  const __nv_bfloat16* dr = delta ? delta + row * hidden : nullptr;
  uint4 xv[kPasses], dv[kPasses], wv[kPasses];
#pragma unroll
  for (int c = 0; c < kPasses; ++c) {
    const int vi = c * nthr + tid;
    xv[c] = dv[c] = wv[c] = make_uint4(0, 0, 0, 0);
    if (vi < vecs) {
      xv[c] = ld16(xr + vi * 8);
      if (dr) dv[c] = ld16(dr + vi * 8);
      wv[c] = ld16(w + vi * 8);
    }
  }
  float v[kPasses * 8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kPasses; ++c) {
    const int vi = c * nthr + tid;
    const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv[c]);
    const __nv_bfloat16* de = reinterpret_cast<const __nv_bfloat16*>(&dv[c]);
    uint4 rv;
    __nv_bfloat16* re = reinterpret_cast<__nv_bfloat16*>(&rv);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float r = dr ? bf(__bfloat162float(xe[e]) + __bfloat162float(de[e]))
                         : __bfloat162float(xe[e]);
      re[e] = __float2bfloat16_rn(r);
      v[c * 8 + e] = r;
      ss += r * r;  // padding vectors hold zeros
    }
    if (residual_out && vi < vecs)
      *reinterpret_cast<uint4*>(residual_out + row * hidden + vi * 8) = rv;
  }
  __shared__ float red[kNormThreads / 32];
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (nthr >> 5); ++i) tot += red[i];
  const float inv = rsqrtf(tot / static_cast<float>(hidden) + eps);
#pragma unroll
  for (int c = 0; c < kPasses; ++c) {
    const int vi = c * nthr + tid;
    if (vi >= vecs) break;
    const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv[c]);
    uint4 ov;
    __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
    for (int e = 0; e < 8; ++e) oe[e] = __float2bfloat16_rn(__bfloat162float(we[e]) * bf(v[c * 8 + e] * inv));
    *reinterpret_cast<uint4*>(norm_out + row * hidden + vi * 8) = ov;
  }
}

// cos / sin of the rotary embedding for every (token, frequency): the bf16 values that
// Qwen3RotaryEmbedding.forward produces (fp32 inv_freq * position, cos / sin in fp32, times
// attention_scaling, cast to bf16), packed as (cos | sin << 16) in one 32-bit word.  Built
// once per forward and read by every layer's q/k rotary embedding.
__global__ void rope_table_kernel(const int64_t* __restrict__ positions, int n_tokens,
                                  const float* __restrict__ inv_freq, int half, float rope_scale,
                                  uint32_t* __restrict__ table) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_tokens * half) return;
  const int tok = i / half, fi = i - tok * half;
  const float f = inv_freq[fi] * static_cast<float>(positions[tok]);
  const __nv_bfloat16 c = __float2bfloat16_rn(cosf(f) * rope_scale);
  const __nv_bfloat16 s = __float2bfloat16_rn(sinf(f) * rope_scale);
  table[i] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&c)) |
             (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&s)) << 16);
}

// One warp per (token, head) of the fused qkv projection; head_dim 128, lane owns
// elements [4 lane, 4 lane + 4), the rotate_half partner lives in lane ^ 16.  kTable: cos /
// sin come from the rope table (16 bytes per lane), else they are computed here.
constexpr int kHeadDim = 128;

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

template <bool kTable>
__global__ void __launch_bounds__(256)
qk_norm_rope_cache_kernel(const __nv_bfloat16* __restrict__ qkv, int n_tokens, int q_heads,
                          int kv_heads, const __nv_bfloat16* __restrict__ qw,
                          const __nv_bfloat16* __restrict__ kw, float eps,
                          const int64_t* __restrict__ positions, const float* __restrict__ inv_freq,
                          float rope_scale, const uint32_t* __restrict__ table,
                          __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_cache,
                          __nv_bfloat16* __restrict__ v_cache, long long head_stride,
                          long long seq_stride, long long past,
                          const int64_t* __restrict__ past_dev) {
  if (past_dev) {
    // device-side prefix length, at most `past` (the rows the caller sized the cache for);
    // outside [0, past] nothing is written (the attention launch of the step reports it)
    const long long live = *past_dev;
    if (live < 0 || live > past) return;
    past = live;
  }
  const int warps = blockDim.x >> 5;
  const long long gw = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int heads = q_heads + 2 * kv_heads;
  if (gw >= static_cast<long long>(n_tokens) * heads) return;
  const int tok = static_cast<int>(gw / heads);
  const int hh = static_cast<int>(gw % heads);
  const __nv_bfloat16* src = qkv + (static_cast<long long>(tok) * heads + hh) * kHeadDim + lane * 4;
  const uint2 raw = *reinterpret_cast<const uint2*>(src);
  const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&raw);
  if (hh >= q_heads + kv_heads) {  // value head: copy into the cache row
    const int h = hh - q_heads - kv_heads;
    *reinterpret_cast<uint2*>(v_cache + h * head_stride + (past + tok) * seq_stride + lane * 4) = raw;
    return;
  }
  const bool is_q = hh < q_heads;
  const __nv_bfloat16* nw = is_q ? qw : kw;
  const uint2 wraw = *reinterpret_cast<const uint2*>(nw + lane * 4);
  const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wraw);
  uint4 cs = make_uint4(0, 0, 0, 0);
  if (kTable)  // emb = cat(freqs, freqs): lanes l and l ^ 16 share frequencies 4 (l & 15) ..
    cs = *reinterpret_cast<const uint4*>(table + static_cast<long long>(tok) * (kHeadDim / 2) +
                                         (lane & 15) * 4);
  const uint32_t* csw = reinterpret_cast<const uint32_t*>(&cs);
  float x[4];
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    x[e] = __bfloat162float(xe[e]);
    ss += x[e] * x[e];
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / static_cast<float>(kHeadDim) + eps);
  float n[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) n[e] = bf(__bfloat162float(we[e]) * bf(x[e] * inv));
  // rotate_half: first half takes -x[d + 64], second half x[d - 64] (lane ^ 16)
  float partner[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) partner[e] = __shfl_xor_sync(DDT_FULL_MASK, n[e], 16);
  uint2 outv;
  __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&outv);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int d = lane * 4 + e;
    float c, s;
    if (kTable) {
      c = bf_lo(csw[e]);
      s = bf_hi(csw[e]);
    } else {
      const float f = inv_freq[d & 63] * static_cast<float>(positions[tok]);
      c = bf(cosf(f) * rope_scale);
      s = bf(sinf(f) * rope_scale);
    }
    const float rot = d < 64 ? -partner[e] : partner[e];
    oe[e] = __float2bfloat16_rn(bf(n[e] * c) + bf(rot * s));
  }
  if (is_q) {
    *reinterpret_cast<uint2*>(q_out + (static_cast<long long>(tok) * q_heads + hh) * kHeadDim + lane * 4) = outv;
  } else {
    const int h = hh - q_heads;
    *reinterpret_cast<uint2*>(k_cache + h * head_stride + (past + tok) * seq_stride + lane * 4) = outv;
  }
}

// One 8-element vector of gate and of up per thread.  (Two vectors per thread, both loaded
// before either is computed, measured slower at the verify size: 8.3 against 7.3 us.)
__device__ __forceinline__ uint4 silu_mul8(uint4 gv, uint4 uv) {
  const __nv_bfloat16* ge = reinterpret_cast<const __nv_bfloat16*>(&gv);
  const __nv_bfloat16* ue = reinterpret_cast<const __nv_bfloat16*>(&uv);
  uint4 ov;
  __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float g = __bfloat162float(ge[e]);
    const float s = bf(g / (1.f + expf(-g)));
    oe[e] = __float2bfloat16_rn(s * __bfloat162float(ue[e]));
  }
  return ov;
}

__global__ void __launch_bounds__(256)
silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, long long rows, int inter,
                __nv_bfloat16* __restrict__ out) {
  const long long v = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int per_row = inter >> 3;
  if (v >= rows * per_row) return;
  const long long r = v / per_row;
  const int c = static_cast<int>(v - r * per_row) * 8;
  const uint4 g = ld16(gu + r * 2 * inter + c);
  const uint4 u = ld16(gu + r * 2 * inter + inter + c);
  *reinterpret_cast<uint4*>(out + r * inter + c) = silu_mul8(g, u);
}

}  // namespace fused
}  // namespace ddt

using namespace ddt;

namespace {

// hidden / 8 vectors in at most kNormMaxPasses passes of at most kNormThreads threads.
bool norm_shape(int64_t hidden, int& nthr) {
  if (hidden <= 0 || hidden % 8) return false;
  const int64_t vecs = hidden / 8;
  const int64_t passes = (vecs + fused::kNormThreads - 1) / fused::kNormThreads;
  if (passes > fused::kNormMaxPasses) return false;
  const int64_t per = (vecs + passes - 1) / passes;
  nthr = static_cast<int>((per + 31) / 32 * 32);
  return true;
}

int qk_norm_rope_launch(const void* qkv, int64_t n_tokens, int64_t q_heads, int64_t kv_heads,
                        int64_t head_dim, const void* q_norm_w, const void* k_norm_w, float eps,
                        const int64_t* positions, const float* inv_freq, float rope_scale,
                        const void* table, void* q_out, void* k_cache, void* v_cache,
                        int64_t head_stride, int64_t seq_stride, int64_t past_length,
                        const int64_t* past_dev, void* stream) {
  if (!qkv || !q_norm_w || !k_norm_w || !q_out || !k_cache || !v_cache) return DDT_ERR_INVALID;
  if (!table && (!positions || !inv_freq)) return DDT_ERR_INVALID;
  if (head_dim != fused::kHeadDim) return DDT_ERR_CAPACITY;
  if (n_tokens < 0 || q_heads <= 0 || kv_heads <= 0 || past_length < 0) return DDT_ERR_INVALID;
  if (past_dev && !aligned(past_dev, 8)) return DDT_ERR_ALIGN;
  if (!aligned(qkv, 8) || !aligned(q_out, 8) || !aligned(k_cache, 8) || !aligned(v_cache, 8) ||
      !aligned(q_norm_w, 8) || !aligned(k_norm_w, 8) || (table && !aligned(table, 16)) ||
      (head_stride * 2) % 8 || (seq_stride * 2) % 8)
    return DDT_ERR_ALIGN;
  if (n_tokens == 0) return DDT_OK;
  const long long warps = n_tokens * (q_heads + 2 * kv_heads);
  const dim3 grid(static_cast<unsigned>((warps + 7) / 8));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const auto* in = static_cast<const __nv_bfloat16*>(qkv);
  const auto* qw = static_cast<const __nv_bfloat16*>(q_norm_w);
  const auto* kw = static_cast<const __nv_bfloat16*>(k_norm_w);
  auto* qo = static_cast<__nv_bfloat16*>(q_out);
  auto* kc = static_cast<__nv_bfloat16*>(k_cache);
  auto* vc = static_cast<__nv_bfloat16*>(v_cache);
  if (table)
    fused::qk_norm_rope_cache_kernel<true><<<grid, 256, 0, st>>>(
        in, static_cast<int>(n_tokens), static_cast<int>(q_heads), static_cast<int>(kv_heads), qw,
        kw, eps, nullptr, nullptr, 1.f, static_cast<const uint32_t*>(table), qo, kc, vc,
        head_stride, seq_stride, past_length, past_dev);
  else
    fused::qk_norm_rope_cache_kernel<false><<<grid, 256, 0, st>>>(
        in, static_cast<int>(n_tokens), static_cast<int>(q_heads), static_cast<int>(kv_heads), qw,
        kw, eps, positions, inv_freq, rope_scale, nullptr, qo, kc, vc, head_stride, seq_stride,
        past_length, past_dev);
  return launch_status();
}

}  // namespace

extern "C" int ddt_add_rmsnorm(const void* x, const void* delta, const void* weight, int64_t rows,
                               int64_t hidden, float eps, void* residual_out, void* norm_out,
                               void* stream) {
  if (!x || !weight || !norm_out || rows < 0) return DDT_ERR_INVALID;
  int nthr = 0;
  if (!norm_shape(hidden, nthr)) return DDT_ERR_CAPACITY;
  if (!aligned(x, 16) || !aligned(weight, 16) || !aligned(norm_out, 16) ||
      (delta && !aligned(delta, 16)) || (residual_out && !aligned(residual_out, 16)))
    return DDT_ERR_ALIGN;
  if (rows == 0) return DDT_OK;
  const auto* xp = static_cast<const __nv_bfloat16*>(x);
  const auto* dp = static_cast<const __nv_bfloat16*>(delta);
  const auto* wp = static_cast<const __nv_bfloat16*>(weight);
  auto* rp = static_cast<__nv_bfloat16*>(residual_out);
  auto* np = static_cast<__nv_bfloat16*>(norm_out);
  const int h = static_cast<int>(hidden);
  const dim3 grid(static_cast<unsigned>(rows));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch ((hidden / 8 + nthr - 1) / nthr) {
    case 1: fused::add_rmsnorm_kernel<1><<<grid, nthr, 0, st>>>(xp, dp, wp, h, eps, rp, np); break;
    case 2: fused::add_rmsnorm_kernel<2><<<grid, nthr, 0, st>>>(xp, dp, wp, h, eps, rp, np); break;
    case 3: fused::add_rmsnorm_kernel<3><<<grid, nthr, 0, st>>>(xp, dp, wp, h, eps, rp, np); break;
    default: fused::add_rmsnorm_kernel<4><<<grid, nthr, 0, st>>>(xp, dp, wp, h, eps, rp, np); break;
  }
  return launch_status();
}

extern "C" int ddt_rope_table(const int64_t* positions, int64_t n_tokens, const float* inv_freq,
                              int64_t head_dim, float rope_scale, void* table, void* stream) {
  if (!positions || !inv_freq || !table || n_tokens < 0) return DDT_ERR_INVALID;
  if (head_dim != fused::kHeadDim) return DDT_ERR_CAPACITY;
  if (!aligned(table, 16)) return DDT_ERR_ALIGN;
  if (n_tokens == 0) return DDT_OK;
  const long long n = n_tokens * (head_dim / 2);
  fused::rope_table_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0,
                             static_cast<cudaStream_t>(stream)>>>(
      positions, static_cast<int>(n_tokens), inv_freq, static_cast<int>(head_dim / 2), rope_scale,
      static_cast<uint32_t*>(table));
  return launch_status();
}

extern "C" int ddt_qk_norm_rope_cache(const void* qkv, int64_t n_tokens, int64_t q_heads,
                                      int64_t kv_heads, int64_t head_dim, const void* q_norm_w,
                                      const void* k_norm_w, float eps, const int64_t* positions,
                                      const float* inv_freq, float rope_scale, void* q_out,
                                      void* k_cache, void* v_cache, int64_t head_stride,
                                      int64_t seq_stride, int64_t past_length, void* stream) {
  if (!positions || !inv_freq) return DDT_ERR_INVALID;
  return qk_norm_rope_launch(qkv, n_tokens, q_heads, kv_heads, head_dim, q_norm_w, k_norm_w, eps,
                             positions, inv_freq, rope_scale, nullptr, q_out, k_cache, v_cache,
                             head_stride, seq_stride, past_length, nullptr, stream);
}

extern "C" int ddt_qk_norm_rope_cache_table(const void* qkv, int64_t n_tokens, int64_t q_heads,
                                            int64_t kv_heads, int64_t head_dim,
                                            const void* q_norm_w, const void* k_norm_w, float eps,
                                            const void* rope_table, void* q_out, void* k_cache,
                                            void* v_cache, int64_t head_stride, int64_t seq_stride,
                                            int64_t past_length, void* stream) {
  if (!rope_table) return DDT_ERR_INVALID;
  return qk_norm_rope_launch(qkv, n_tokens, q_heads, kv_heads, head_dim, q_norm_w, k_norm_w, eps,
                             nullptr, nullptr, 1.f, rope_table, q_out, k_cache, v_cache,
                             head_stride, seq_stride, past_length, nullptr, stream);
}

// The table form with the prefix length in device memory (*past_length_dev, at most
// max_past_length: the cache must hold max_past_length + n_tokens rows), for a verify step
// recorded once and replayed at every prefix length.
extern "C" int ddt_qk_norm_rope_cache_table_device_past(
    const void* qkv, int64_t n_tokens, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
    const void* q_norm_w, const void* k_norm_w, float eps, const void* rope_table, void* q_out,
    void* k_cache, void* v_cache, int64_t head_stride, int64_t seq_stride,
    int64_t max_past_length, const int64_t* past_length_dev, void* stream) {
  if (!rope_table || !past_length_dev) return DDT_ERR_INVALID;
  return qk_norm_rope_launch(qkv, n_tokens, q_heads, kv_heads, head_dim, q_norm_w, k_norm_w, eps,
                             nullptr, nullptr, 1.f, rope_table, q_out, k_cache, v_cache,
                             head_stride, seq_stride, max_past_length, past_length_dev, stream);
}

extern "C" int ddt_silu_mul(const void* gate_up, int64_t rows, int64_t inter, void* out,
                            void* stream) {
  if (!gate_up || !out || rows < 0 || inter <= 0) return DDT_ERR_INVALID;
  if (inter % 8 || !aligned(gate_up, 16) || !aligned(out, 16)) return DDT_ERR_ALIGN;
  if (rows == 0) return DDT_OK;
  const long long vecs = rows * inter / 8;
  fused::silu_mul_kernel<<<static_cast<unsigned>((vecs + 255) / 256), 256, 0,
                           static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(gate_up), rows, static_cast<int>(inter),
      static_cast<__nv_bfloat16*>(out));
  return launch_status();
}
