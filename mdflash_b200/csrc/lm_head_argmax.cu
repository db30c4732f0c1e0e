// Fused lm_head -> greedy posterior: for every verify row n, argmax_v bf16(h[n] . W[v]) with
// ties to the lowest index and NaN largest, without writing the [N, V] logits.
//
// Replaces, in the verify step, the lm_head projection of the target (a plain
// Linear(hidden, vocab) on the final normed hidden states, whose bf16 logits the reference
// materialises at ddtree.py:467-478) followed by sample() at temperature 0
// (model/utils.py:28-30, torch.argmax over the logits).  The logits are the bf16 rounding
// (round to nearest even) of fp32 dot products, as a bf16 GEMM with fp32 accumulation
// produces them; the argmax is taken over those bf16 values.
//
// tcgen05 GEMM with the vocabulary as M: D[v, n] = W[v, :] . h[n, :] for a tile of 128
// vocabulary rows (A, K-major) against a group of up to 272 verify rows (B, K-major), both
// staged by TMA in 64-element K chunks with the 128-byte swizzle.  The group is split in two
// parts (rows [0, 144) and [144, 272)) with one MMA-issuing warp each, so that while one
// issuer waits for a stage (a wait holds the thread until its own MMAs drain) the other's
// MMAs keep the tensor pipe busy.  D of part 0 lives in TMEM columns [0, 144), of part 1 in
// [256, 384).  Eight epilogue warps (two per TMEM lane quarter, one pair per part) read D
// into registers, hand the columns back to the issuers, and reduce: per verify row the
// largest 16-bit order key of the bf16 logit across the tile's 128 lanes (warp redux, then
// four lane quarters through shared memory), kept per CTA as a 64-bit (key, ~index)
// composite.  At the end every CTA folds its composites into the workspace with atomicMax,
// and the last CTA (atomic ticket) writes the indices and clears the workspace.
#include <cuda.h>
#include <cuda_bf16.h>

#include "common.cuh"
#include "tc.cuh"

namespace ddt {
namespace lmhead {

constexpr int kM = 128;            // vocabulary rows per tile
constexpr int kK = 64;             // K elements per stage (128 bytes of a row)
constexpr int kStages = 4;
constexpr int kThreads = 384;
constexpr int kGroup = 272;  // verify rows per group: part 0 = 144 rows, part 1 = 128
__host__ __device__ constexpr int part_rows(int q) { return q ? 128 : 144; }
__host__ __device__ constexpr uint32_t col_base(int q) { return q ? 256u : 0u; }  // TMEM column
__host__ __device__ constexpr int part_chunks(int q) { return q ? 4 : 5; }  // 32-column chunks
constexpr uint32_t kABytes = kM * kK * 2;                 // 16 KB
constexpr uint32_t kB0Bytes = 144 * kK * 2;               // 18 KB
constexpr uint32_t kB1Bytes = 128 * kK * 2;               // 16 KB
constexpr uint32_t kStageBytes = kABytes + kB0Bytes + kB1Bytes;  // 50 KB, 1 KB multiple
constexpr uint32_t kSmemTiles = kStages * kStageBytes;
constexpr uint32_t kSmemAlloc = kSmemTiles + 1024;
constexpr int kRegsControl = 56;
constexpr int kRegsEpilogue = 224;
static_assert(128 * kRegsControl + 256 * kRegsEpilogue <= kThreads * 168, "register split");
constexpr uint64_t kTimeoutNs = 2000000000ull;

struct Params {
  int n_rows;       // verify rows
  int vocab;
  int k_chunks;     // hidden / 64
  int tiles;        // vocabulary tiles
  int groups;       // verify-row groups of 272
  unsigned long long* best;  // workspace: per verify row, 64-bit composite (zero on entry)
  unsigned int* ticket;      // workspace: CTAs done (zero on entry)
  int64_t* out;
  __nv_bfloat16* logits;     // optional bf16 logits [n_rows, logits_ld] (testing aid)
  long long logits_ld;
  int* status;
};

struct Bars {
  uint64_t full[kStages], empty[kStages], d_full[2], d_empty[2], mma_done[2];
  uint32_t tmem_base;
  int abort;
  int last;
};

// 16-bit order key of the bf16 rounding of x: larger value, larger key; -0 and +0 equal;
// every NaN above +inf (torch.argmax's rule).
__device__ __forceinline__ uint32_t logit_key(float x) {
  if (isnan(x)) return 0xffffu;
  const __nv_bfloat16 b = __float2bfloat16_rn(x);
  return bf16_key(*reinterpret_cast<const uint16_t*>(&b));
}

__global__ void __launch_bounds__(kThreads, 1)
lm_head_argmax_kernel(const __grid_constant__ CUtensorMap tm_w,
                      const __grid_constant__ CUtensorMap tm_h0,
                      const __grid_constant__ CUtensorMap tm_h1, const __grid_constant__ Params p) {
  extern __shared__ unsigned char smem_raw[];
  __shared__ Bars bars;
  __shared__ uint32_t s_red[2][4][kGroup];      // per lane quarter, per column
  __shared__ unsigned long long s_best[kGroup];  // this CTA's best composite per column
  const uint32_t raw = tc::smem_u32(smem_raw);
  unsigned char* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_items = p.tiles * p.groups;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&bars.full[s], 1);
      tc::mbar_init(&bars.empty[s], 2);  // one commit per issuer
    }
    for (int q = 0; q < 2; ++q) {
      tc::mbar_init(&bars.d_full[q], 1);
      tc::mbar_init(&bars.d_empty[q], 4);  // the 4 epilogue warps of the part
      tc::mbar_init(&bars.mma_done[q], 1);
    }
    bars.abort = 0;
    bars.last = 0;
    tc::fence_mbar_init();
  }
  for (int c = tid; c < kGroup; c += kThreads) s_best[c] = 0ull;
  if (warp == 1) {
    tc::tmem_alloc(&bars.tmem_base, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = bars.tmem_base;
  volatile int* abort_flag = &bars.abort;

  if (warp < 4) {
    tc::reg_dealloc<kRegsControl>();
    if (warp == 0) {
      // ---------------- TMA producer: W tile + both parts of the verify-row group ----------
      if (lane == 0) {
        tc::tma_prefetch_desc(&tm_w);
        tc::tma_prefetch_desc(&tm_h0);
        tc::tma_prefetch_desc(&tm_h1);
        bool ok = true;
        int issued = 0;
        for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x) {
          const int g = w / p.tiles, t = w % p.tiles;
          for (int kc = 0; kc < p.k_chunks; ++kc, ++issued) {
            const int s = issued % kStages;
            if (issued >= kStages &&
                !(ok = tc::mbar_wait(&bars.empty[s], ((issued / kStages) - 1) & 1, abort_flag,
                                     kTimeoutNs)))
              break;
            unsigned char* st = smem + s * kStageBytes;
            tc::mbar_expect_tx(&bars.full[s], kStageBytes);
            tc::tma_load_2d(st, &tm_w, &bars.full[s], kc * kK, t * kM);
            tc::tma_load_2d(st + kABytes, &tm_h0, &bars.full[s], kc * kK, g * kGroup);
            tc::tma_load_2d(st + kABytes + kB0Bytes, &tm_h1, &bars.full[s], kc * kK,
                            g * kGroup + part_rows(0));
          }
        }
        if (!ok) {
          *reinterpret_cast<volatile int*>(&bars.abort) = 1;
          if (p.status) atomicOr(p.status, 1);
        }
        if (*abort_flag) {
          // let the loads in flight land before the CTA releases its shared memory
          for (int j = issued > kStages ? issued - kStages : 0; j < issued; ++j)
            tc::mbar_wait_drain(&bars.full[j % kStages], (j / kStages) & 1, kTimeoutNs);
        }
      }
    } else if (warp == 1 || warp == 3) {
      // ---------------- MMA issuers: part 0 from warp 1, part 1 from warp 3 ------------------
      const int q = warp == 1 ? 0 : 1;
      constexpr uint32_t kDescHi = tc::desc_sw128_hi(1024);
      const uint32_t a_lo = tc::desc_sw128_lo(tc::smem_u32(smem), 16);
      const uint32_t b_lo = tc::desc_sw128_lo(
          tc::smem_u32(smem + kABytes + (q ? kB0Bytes : 0u)), 16);
      const uint32_t d = tmem + col_base(q);
      bool ok = true;
      int it = 0, gi = 0;
      for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x, ++it) {
        const int g = w / p.tiles;
        int rows = p.n_rows - g * kGroup - (q ? part_rows(0) : 0);
        rows = rows < 0 ? 0 : (rows > part_rows(q) ? part_rows(q) : rows);
        const int n_mma = (rows + 15) & ~15;  // MMA N: a multiple of 16
        const uint32_t idesc = tc::idesc_bf16_f32(kM, n_mma > 0 ? n_mma : 16, false, false);
        // the epilogue has read this part's previous D
        if (it > 0 && !(ok = tc::mbar_wait_warp(&bars.d_empty[q], (it - 1) & 1, abort_flag,
                                                kTimeoutNs)))
          break;
        // stages are consumed two at a time: both waits come first (the second one finds no
        // MMA of this warp in flight), then 8 MMAs, so a wait that drains this warp's MMAs
        // comes once per 8 MMAs instead of once per 4
        for (int kc = 0; kc < p.k_chunks; kc += 2) {
          const int nk = kc + 1 < p.k_chunks ? 2 : 1;
          for (int x = 0; x < nk; ++x) {
            const int s = (gi + x) % kStages;
            if (!(ok = tc::mbar_wait_warp(&bars.full[s], ((gi + x) / kStages) & 1, abort_flag,
                                          kTimeoutNs)))
              break;
          }
          if (!ok) break;
          tc::tc_fence_after();
          if (tc::elect_one()) {
            for (int x = 0; x < nk; ++x) {
              const int s = (gi + x) % kStages;
              if (n_mma > 0) {
                const uint32_t so = (s * kStageBytes) >> 4;
#pragma unroll
                for (int k = 0; k < kK / 16; ++k) {
                  const uint32_t off = so + ((k * 32) >> 4);
                  if (kc + x == 0 && k == 0)
                    tc::mma_bf16_ss_w<0>(d, a_lo + off, b_lo + off, kDescHi, idesc);
                  else
                    tc::mma_bf16_ss_w<1>(d, a_lo + off, b_lo + off, kDescHi, idesc);
                }
              }
              tc::mma_commit(&bars.empty[s]);
            }
            if (kc + nk == p.k_chunks) tc::mma_commit(&bars.d_full[q]);
          }
          __syncwarp();
          gi += nk;
        }
      }
      if (!ok) {
        if (lane == 0) {
          *reinterpret_cast<volatile int*>(&bars.abort) = 1;
          if (p.status) atomicOr(p.status, 1);
        }
        if (tc::elect_one()) tc::mma_commit(&bars.mma_done[q]);
        __syncwarp();
        tc::mbar_wait_drain(&bars.mma_done[q], 0, kTimeoutNs);
      }
    }
  } else {
    tc::reg_alloc<kRegsEpilogue>();
    // ---------------- epilogue: warps 4-7 read part 0, warps 8-11 part 1 ----------------------
    const int q = (warp - 4) >> 2;
    const int wq = warp & 3;  // TMEM lane quarter
    const int r = wq * 32 + lane;  // vocabulary row of the tile
    const int et = tid - 128;      // 0..255 over the epilogue warps
    const uint32_t tq = tmem + (static_cast<uint32_t>(wq * 32) << 16) + col_base(q);
    const int col0 = q ? part_rows(0) : 0;  // first group column of this part
    bool ok = true;
    int it = 0, buf = 0, cur_group = -1;
    auto flush = [&](int g) {
      // this thread's columns of the group: et and et + 256
      for (int c = et; c < kGroup; c += 256) {
        const int row = g * kGroup + c;
        const unsigned long long b = s_best[c];
        if (row < p.n_rows && b != 0ull) atomicMax(p.best + row, b);
        s_best[c] = 0ull;
      }
    };
    for (int w = blockIdx.x; w < n_items; w += gridDim.x, ++it) {
      const int g = w / p.tiles, t = w % p.tiles;
      if (g != cur_group) {
        if (cur_group >= 0) flush(cur_group);
        cur_group = g;
      }
      const bool got = tc::mbar_wait_warp(&bars.d_full[q], it & 1, abort_flag, kTimeoutNs);
      if (got) {
        tc::tc_fence_after();
        uint32_t v[5][32];
#pragma unroll
        for (int i = 0; i < 5; ++i)
          if (i < part_chunks(q)) tc::tmem_ld32(tq + i * 32, v[i]);
        tc::tmem_wait_ld();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars.d_empty[q]);  // the issuer may overwrite D
        const int vrow = t * kM + r;
        const bool vok = vrow < p.vocab;
        const int prows = part_rows(q);
#pragma unroll
        for (int i = 0; i < 5; ++i) {
          if (i >= part_chunks(q)) break;
          uint32_t mine = 0u;
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int c = i * 32 + e;  // column within the part
            const int row = g * kGroup + col0 + c;
            const float x = __uint_as_float(v[i][e]);
            const bool ok_c = vok && c < prows && row < p.n_rows;
            if (ok_c && p.logits) p.logits[row * p.logits_ld + vrow] = __float2bfloat16_rn(x);
            const uint32_t comp =
                ok_c ? ((logit_key(x) << 8) | static_cast<uint32_t>(127 - r)) : 0u;
            const uint32_t m = __reduce_max_sync(DDT_FULL_MASK, comp);
            if (lane == e) mine = m;
          }
          const int c = i * 32 + lane;
          if (c < prows) s_red[buf][wq][col0 + c] = mine;
        }
      }
      // one barrier per tile for all 8 epilogue warps, which also tells every warp whether all
      // of them got their D: on a timeout they all leave the loop at the same tile, so the
      // (unbounded) named barriers below stay paired
      if (!tc::named_sync_and(1, 256, got)) {
        ok = false;
        break;
      }
      for (int c = et; c < kGroup; c += 256) {
        uint32_t b = s_red[buf][0][c];
        b = max(b, s_red[buf][1][c]);
        b = max(b, s_red[buf][2][c]);
        b = max(b, s_red[buf][3][c]);
        if (b != 0u) {
          const uint32_t idx = static_cast<uint32_t>(t * kM + 127 - static_cast<int>(b & 0xffu));
          const unsigned long long comp =
              (static_cast<unsigned long long>(b >> 8) << 32) | static_cast<uint32_t>(~idx);
          if (comp > s_best[c]) s_best[c] = comp;
        }
      }
      buf ^= 1;
    }
    if (ok && cur_group >= 0) flush(cur_group);
    if (!ok && lane == 0) {
      *reinterpret_cast<volatile int*>(&bars.abort) = 1;
      if (p.status) atomicOr(p.status, 1);
    }
    // the last CTA to finish writes the indices and clears the workspace
    tc::named_sync(1, 256);
    if (et == 0) {
      __threadfence();
      const unsigned int done = atomicAdd(p.ticket, 1u);
      bars.last = done == gridDim.x - 1;
    }
    tc::named_sync(1, 256);
    if (bars.last) {
      __threadfence();
      for (int row = et; row < p.n_rows; row += 256) {
        const unsigned long long b = atomicExch(p.best + row, 0ull);
        p.out[row] = b ? static_cast<int64_t>(~static_cast<uint32_t>(b)) : 0;
      }
      if (et == 0) atomicExch(p.ticket, 0u);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

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

// 2-D bf16 map of a row-major [rows, cols] array (row stride ld elements), box
// {64 columns, box_rows rows}, 128-byte swizzle, zero fill out of bounds.
inline int make_map_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows,
                       uint64_t ld, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return DDT_ERR_CUDA;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kK), box_rows};
  const cuuint32_t es[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DDT_OK : DDT_ERR_ALIGN;
}

}  // namespace lmhead
}  // namespace ddt

using namespace ddt;

extern "C" size_t ddt_lm_head_argmax_workspace_bytes(int64_t n_rows) {
  return static_cast<size_t>(n_rows > 0 ? n_rows : 0) * sizeof(unsigned long long) + 256;
}

extern "C" int ddt_lm_head_argmax(const void* hidden, int64_t hidden_ld, const void* weight,
                                  int64_t weight_ld, int64_t n_rows, int64_t hidden_size,
                                  int64_t vocab, int64_t* out, void* logits_out,
                                  int64_t logits_ld, void* workspace, size_t workspace_bytes,
                                  int32_t* status, void* stream) {
  if (!hidden || !weight || !out || n_rows <= 0 || hidden_size <= 0 || vocab <= 0)
    return DDT_ERR_INVALID;
  if (hidden_size % lmhead::kK) return DDT_ERR_CAPACITY;
  if (vocab >= (int64_t(1) << 31) || n_rows > (int64_t(1) << 20)) return DDT_ERR_CAPACITY;
  if (hidden_ld < hidden_size || weight_ld < hidden_size) return DDT_ERR_INVALID;
  if (logits_out && logits_ld < vocab) return DDT_ERR_INVALID;
  if (!aligned(hidden, 16) || !aligned(weight, 16) || (hidden_ld * 2) % 16 || (weight_ld * 2) % 16)
    return DDT_ERR_ALIGN;
  if (!workspace || workspace_bytes < ddt_lm_head_argmax_workspace_bytes(n_rows))
    return DDT_ERR_WORKSPACE;
  if (!aligned(workspace, 16)) return DDT_ERR_ALIGN;
  CUtensorMap tm_w, tm_h0, tm_h1;
  int rc = lmhead::make_map_2d(&tm_w, weight, hidden_size, vocab, weight_ld, lmhead::kM);
  if (rc) return rc;
  rc = lmhead::make_map_2d(&tm_h0, hidden, hidden_size, n_rows, hidden_ld, lmhead::part_rows(0));
  if (rc) return rc;
  rc = lmhead::make_map_2d(&tm_h1, hidden, hidden_size, n_rows, hidden_ld, lmhead::part_rows(1));
  if (rc) return rc;
  lmhead::Params p;
  p.n_rows = static_cast<int>(n_rows);
  p.vocab = static_cast<int>(vocab);
  p.k_chunks = static_cast<int>(hidden_size / lmhead::kK);
  p.tiles = static_cast<int>((vocab + lmhead::kM - 1) / lmhead::kM);
  p.groups = static_cast<int>((n_rows + lmhead::kGroup - 1) / lmhead::kGroup);
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  p.best = reinterpret_cast<unsigned long long*>(ws);
  p.ticket = reinterpret_cast<unsigned int*>(ws + static_cast<size_t>(n_rows) * 8);
  p.out = out;
  p.logits = static_cast<__nv_bfloat16*>(logits_out);
  p.logits_ld = logits_ld;
  p.status = status;
  const int64_t items = static_cast<int64_t>(p.tiles) * p.groups;
  const unsigned grid = static_cast<unsigned>(items < 148 ? items : 148);
  if (cudaFuncSetAttribute(lmhead::lm_head_argmax_kernel,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           lmhead::kSmemAlloc) != cudaSuccess)
    return DDT_ERR_CUDA;
  lmhead::lm_head_argmax_kernel<<<grid, lmhead::kThreads, lmhead::kSmemAlloc,
                                  static_cast<cudaStream_t>(stream)>>>(tm_w, tm_h0, tm_h1, p);
  return launch_status();
}
