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
//                            torch.cat (cache_utils.py:119-120), in place at rows past + i
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

// One CTA per row (up to 256 threads); each thread owns 8 consecutive elements per pass,
// at most 4 passes.
constexpr int kNormThreads = 256;
constexpr int kNormMaxPasses = 4;

__global__ void __launch_bounds__(kNormThreads)
add_rmsnorm_kernel(const __nv_bfloat16* x, const __nv_bfloat16* __restrict__ delta,
                   const __nv_bfloat16* __restrict__ w, int hidden, float eps,
                   __nv_bfloat16* residual_out, __nv_bfloat16* __restrict__ norm_out) {
  // residual_out may alias x: each thread reads its elements before it writes them
  const long long row = blockIdx.x;
  const int tid = threadIdx.x;
  const __nv_bfloat16* xr = x + row * hidden;
  const __nv_bfloat16* dr = delta ? delta + row * hidden : nullptr;
  const int nthr = blockDim.x;
  const int passes = hidden / (nthr * 8);
  float v[kNormMaxPasses * 8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kNormMaxPasses; ++c) {
    if (c >= passes) break;
    const int base = (c * nthr + tid) * 8;
    const uint4 xv = *reinterpret_cast<const uint4*>(xr + base);
    const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xv);
    uint4 dv = make_uint4(0, 0, 0, 0);
    if (dr) dv = *reinterpret_cast<const uint4*>(dr + base);
    const __nv_bfloat16* de = reinterpret_cast<const __nv_bfloat16*>(&dv);
    uint4 rv;
    __nv_bfloat16* re = reinterpret_cast<__nv_bfloat16*>(&rv);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float r = dr ? bf(__bfloat162float(xe[e]) + __bfloat162float(de[e]))
                         : __bfloat162float(xe[e]);
      re[e] = __float2bfloat16_rn(r);
      v[c * 8 + e] = r;
      ss += r * r;
    }
    if (residual_out) *reinterpret_cast<uint4*>(residual_out + row * hidden + base) = rv;
  }
  __shared__ float red[kNormThreads / 32];
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (nthr >> 5); ++i) tot += red[i];
  const float inv = rsqrtf(tot / static_cast<float>(hidden) + eps);
#pragma unroll
  for (int c = 0; c < kNormMaxPasses; ++c) {
    if (c >= passes) break;
    const int base = (c * nthr + tid) * 8;
    const uint4 wv = *reinterpret_cast<const uint4*>(w + base);
    const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
    uint4 ov;
    __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
    for (int e = 0; e < 8; ++e) oe[e] = __float2bfloat16_rn(__bfloat162float(we[e]) * bf(v[c * 8 + e] * inv));
    *reinterpret_cast<uint4*>(norm_out + row * hidden + base) = ov;
  }
}

// One warp per (token, head) of the fused qkv projection; head_dim 128, lane owns
// elements [4 lane, 4 lane + 4), the rotate_half partner lives in lane ^ 16.
constexpr int kHeadDim = 128;

__global__ void __launch_bounds__(256)
qk_norm_rope_cache_kernel(const __nv_bfloat16* __restrict__ qkv, int n_tokens, int q_heads,
                          int kv_heads, const __nv_bfloat16* __restrict__ qw,
                          const __nv_bfloat16* __restrict__ kw, float eps,
                          const int64_t* __restrict__ positions, const float* __restrict__ inv_freq,
                          float rope_scale, __nv_bfloat16* __restrict__ q_out,
                          __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
                          long long head_stride, long long seq_stride, long long past) {
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
  for (int e = 0; e < 4; ++e) n[e] = bf(__bfloat162float(nw[lane * 4 + e]) * bf(x[e] * inv));
  // rotate_half: first half takes -x[d + 64], second half x[d - 64] (lane ^ 16)
  float partner[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) partner[e] = __shfl_xor_sync(DDT_FULL_MASK, n[e], 16);
  const float pos = static_cast<float>(positions[tok]);
  uint2 outv;
  __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&outv);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int d = lane * 4 + e;
    const int fi = d & 63;  // emb = cat(freqs, freqs)
    const float f = inv_freq[fi] * pos;
    const float c = bf(cosf(f) * rope_scale);
    const float s = bf(sinf(f) * rope_scale);
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

__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, long long rows, int inter,
                                __nv_bfloat16* __restrict__ out) {
  const long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  const long long total = rows * inter;
  if (i >= total) return;
  const long long r = i / inter;
  const int c = static_cast<int>(i % inter);
  const uint4 gv = *reinterpret_cast<const uint4*>(gu + r * 2 * inter + c);
  const uint4 uv = *reinterpret_cast<const uint4*>(gu + r * 2 * inter + inter + c);
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
  *reinterpret_cast<uint4*>(out + i) = ov;
}

}  // namespace fused
}  // namespace ddt

using namespace ddt;

extern "C" int ddt_add_rmsnorm(const void* x, const void* delta, const void* weight, int64_t rows,
                               int64_t hidden, float eps, void* residual_out, void* norm_out,
                               void* stream) {
  if (!x || !weight || !norm_out || rows < 0) return DDT_ERR_INVALID;
  int nthr = static_cast<int>(hidden / 8);
  if (nthr > fused::kNormThreads) nthr = fused::kNormThreads;
  nthr &= ~31;
  if (nthr < 32 || hidden % (nthr * 8) || hidden / (nthr * 8) > fused::kNormMaxPasses)
    return DDT_ERR_CAPACITY;
  if (!aligned(x, 16) || !aligned(weight, 16) || !aligned(norm_out, 16) ||
      (delta && !aligned(delta, 16)) || (residual_out && !aligned(residual_out, 16)))
    return DDT_ERR_ALIGN;
  if (rows == 0) return DDT_OK;
  fused::add_rmsnorm_kernel<<<static_cast<unsigned>(rows), nthr, 0,
                              static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(delta),
      static_cast<const __nv_bfloat16*>(weight), static_cast<int>(hidden), eps,
      static_cast<__nv_bfloat16*>(residual_out), static_cast<__nv_bfloat16*>(norm_out));
  return launch_status();
}

extern "C" int ddt_qk_norm_rope_cache(const void* qkv, int64_t n_tokens, int64_t q_heads,
                                      int64_t kv_heads, int64_t head_dim, const void* q_norm_w,
                                      const void* k_norm_w, float eps, const int64_t* positions,
                                      const float* inv_freq, float rope_scale, void* q_out,
                                      void* k_cache, void* v_cache, int64_t head_stride,
                                      int64_t seq_stride, int64_t past_length, void* stream) {
  if (!qkv || !q_norm_w || !k_norm_w || !positions || !inv_freq || !q_out || !k_cache || !v_cache)
    return DDT_ERR_INVALID;
  if (head_dim != fused::kHeadDim) return DDT_ERR_CAPACITY;
  if (n_tokens < 0 || q_heads <= 0 || kv_heads <= 0 || past_length < 0) return DDT_ERR_INVALID;
  if (!aligned(qkv, 8) || !aligned(q_out, 8) || !aligned(k_cache, 8) || !aligned(v_cache, 8) ||
      (head_stride * 2) % 8 || (seq_stride * 2) % 8)
    return DDT_ERR_ALIGN;
  if (n_tokens == 0) return DDT_OK;
  const long long warps = n_tokens * (q_heads + 2 * kv_heads);
  fused::qk_norm_rope_cache_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0,
                                     static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(qkv), static_cast<int>(n_tokens), static_cast<int>(q_heads),
      static_cast<int>(kv_heads), static_cast<const __nv_bfloat16*>(q_norm_w),
      static_cast<const __nv_bfloat16*>(k_norm_w), eps, positions, inv_freq, rope_scale,
      static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_cache),
      static_cast<__nv_bfloat16*>(v_cache), head_stride, seq_stride, past_length);
  return launch_status();
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
