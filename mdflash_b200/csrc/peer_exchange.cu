// Exchange of split-KV attention partials over NVLink peer memory, replacing the NCCL
// all-gather of (O, m, l) between the ranks that each attend over one shard of a long prefix.
//
// No counterpart in the reference (its verify attention runs on one device, ddtree.py:467).
// Every rank owns one receive buffer, allocated here with cudaMalloc and shared with the
// other ranks of the node through CUDA IPC handles (the handles travel over the process
// group).  ddt_peer_push writes this rank's merged partial (one per query row: O un-normalised
// fp32 [rows, 128], m, l) straight into slot `rank` of every rank's receive buffer with
// 16-byte stores over NVLink (plain stores: no multicast object, no TMA), then the push's
// last CTA (atomic ticket) increments counter `rank` of every receive buffer once, after a
// system-scope fence.  ddt_peer_merge waits (bounded) until every counter has reached the
// call's epoch, then merges the world partials of its own buffer into the bf16 output.
//
// Receive buffer: [counters: kMaxWorld u32][parity 0: O, m, l][parity 1: O, m, l], with
// O [world][rows][128] f32 and m, l [world][rows] f32.  Call e (epochs start at 1) uses parity
// e & 1.  A rank pushes call e + 2 into parity e & 1 only after its own merge of call e + 1
// saw every rank's push of e + 1, which each rank issued after its merge of call e: so no rank
// is still reading a parity that a peer overwrites.
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "peer.cuh"

namespace ddt {
namespace peer {

constexpr int kStatusTimeout = 1;

struct Dests {
  unsigned char* base[kMaxWorld];
};

// Grid-stride copy of this rank's partial into slot `rank` of every destination buffer, then
// one counter increment per destination from the last CTA.
__global__ void __launch_bounds__(256)
push_kernel(const float4* __restrict__ o, const float* __restrict__ m,
            const float* __restrict__ l, long long rows, const __grid_constant__ Dests dst,
            int world, int rank, unsigned long long o_off, unsigned long long m_off,
            unsigned long long l_off, unsigned int* ticket) {
  const long long n4 = rows * (kHeadDim / 4);
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long t0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long slot4 = static_cast<long long>(rank) * n4;
  for (long long i = t0; i < n4; i += stride) {
    const float4 v = o[i];
    for (int w = 0; w < world; ++w)
      reinterpret_cast<float4*>(dst.base[w] + o_off)[slot4 + i] = v;
  }
  const long long slot = static_cast<long long>(rank) * rows;
  for (long long i = t0; i < rows; i += stride) {
    const float mv = m[i], lv = l[i];
    for (int w = 0; w < world; ++w) {
      reinterpret_cast<float*>(dst.base[w] + m_off)[slot + i] = mv;
      reinterpret_cast<float*>(dst.base[w] + l_off)[slot + i] = lv;
    }
  }
  // every thread's peer stores are ordered before its CTA's ticket; the last CTA then
  // publishes the whole push with one counter increment per destination
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int t = atomicAdd(ticket, 1u);
    if (t == gridDim.x - 1) {
      __threadfence_system();
      for (int w = 0; w < world; ++w)
        atomicAdd_system(reinterpret_cast<unsigned int*>(dst.base[w]) + rank, 1u);
      atomicExch(ticket, 0u);
    }
  }
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Lane w waits until counter w has reached the epoch; bounded by timeout_ns.
__global__ void wait_kernel(const unsigned int* __restrict__ counters, int world,
                            unsigned int epoch, int* status, unsigned long long timeout_ns) {
  const int w = threadIdx.x;
  bool ok = true;
  if (w < world) {
    const unsigned long long t0 = global_timer_ns();
    unsigned int it = 0;
    // counters are monotonic: (int)(c - epoch) >= 0 once the push of this epoch has landed
    while (static_cast<int>(ld_acquire_sys(counters + w) - epoch) < 0) {
      if ((++it & 63u) == 0 && global_timer_ns() - t0 > timeout_ns) {
        ok = false;
        break;
      }
    }
  }
  if (!ok && status) atomicOr(status, kStatusTimeout);
  __threadfence_system();
}

}  // namespace peer
}  // namespace ddt

using namespace ddt;

extern "C" int ddt_attn_merge(const float* o_parts, const float* m_parts, const float* l_parts,
                              int64_t n_parts, int64_t n_nodes, int64_t q_heads, int64_t head_dim,
                              void* out, int64_t o_node_stride, int64_t o_head_stride,
                              void* stream);

extern "C" size_t ddt_peer_buffer_bytes(int64_t world, int64_t n_nodes, int64_t q_heads,
                                        int64_t head_dim) {
  if (world <= 0 || world > peer::kMaxWorld || n_nodes <= 0 || q_heads <= 0 ||
      head_dim != peer::kHeadDim)
    return 0;
  return peer::layout(world, n_nodes * q_heads).total;
}

extern "C" int ddt_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes == 0) return DDT_ERR_INVALID;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return DDT_ERR_CUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess ||
      cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p) != cudaSuccess) {
    cudaFree(p);
    return DDT_ERR_CUDA;
  }
  *ptr = p;
  return DDT_OK;
}

extern "C" int ddt_peer_open(const void* ipc_handle, void** ptr) {
  if (!ptr || !ipc_handle) return DDT_ERR_INVALID;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return DDT_ERR_CUDA;
  return DDT_OK;
}

extern "C" int ddt_peer_close(void* ptr) {
  if (!ptr) return DDT_ERR_INVALID;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? DDT_OK : DDT_ERR_CUDA;
}

extern "C" int ddt_peer_free(void* ptr) {
  if (!ptr) return DDT_ERR_INVALID;
  return cudaFree(ptr) == cudaSuccess ? DDT_OK : DDT_ERR_CUDA;
}

extern "C" int ddt_peer_push(const float* o, const float* m, const float* l, int64_t n_nodes,
                             int64_t q_heads, int64_t head_dim, void* const* peer_bases,
                             int64_t world, int64_t rank, uint32_t epoch, uint32_t* ticket,
                             void* stream) {
  if (!o || !m || !l || !peer_bases || !ticket || n_nodes <= 0 || q_heads <= 0 || epoch == 0)
    return DDT_ERR_INVALID;
  if (head_dim != peer::kHeadDim || world <= 0 || world > peer::kMaxWorld) return DDT_ERR_CAPACITY;
  if (rank < 0 || rank >= world) return DDT_ERR_INVALID;
  if (!aligned(o, 16)) return DDT_ERR_ALIGN;
  peer::Dests d{};
  for (int w = 0; w < world; ++w) {
    if (!peer_bases[w] || !aligned(peer_bases[w], 256)) return DDT_ERR_INVALID;
    d.base[w] = static_cast<unsigned char*>(peer_bases[w]);
  }
  const int64_t rows = n_nodes * q_heads;
  const peer::Layout L = peer::layout(world, rows);
  const int par = static_cast<int>(epoch & 1u);
  peer::push_kernel<<<296, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float4*>(o), m, l, rows, d, static_cast<int>(world),
      static_cast<int>(rank), L.o[par], L.m[par], L.l[par], ticket);
  return launch_status();
}

extern "C" int ddt_peer_merge(const void* local_base, int64_t world, int64_t n_nodes,
                              int64_t q_heads, int64_t head_dim, uint32_t epoch, void* out,
                              int64_t o_node_stride, int64_t o_head_stride, int32_t* status,
                              uint64_t timeout_ns, void* stream) {
  if (!local_base || !out || !status || n_nodes <= 0 || q_heads <= 0 || epoch == 0)
    return DDT_ERR_INVALID;
  if (head_dim != peer::kHeadDim || world <= 0 || world > peer::kMaxWorld) return DDT_ERR_CAPACITY;
  if (timeout_ns < 100000ull || timeout_ns > 2000000000ull) return DDT_ERR_INVALID;
  const int64_t rows = n_nodes * q_heads;
  const peer::Layout L = peer::layout(world, rows);
  const int par = static_cast<int>(epoch & 1u);
  const unsigned char* b = static_cast<const unsigned char*>(local_base);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  peer::wait_kernel<<<1, 32, 0, st>>>(reinterpret_cast<const unsigned int*>(b),
                                      static_cast<int>(world), epoch, status, timeout_ns);
  const int rc = launch_status();
  if (rc) return rc;
  return ddt_attn_merge(reinterpret_cast<const float*>(b + L.o[par]),
                        reinterpret_cast<const float*>(b + L.m[par]),
                        reinterpret_cast<const float*>(b + L.l[par]), world, n_nodes, q_heads,
                        head_dim, out, o_node_stride, o_head_stride, stream);
}
