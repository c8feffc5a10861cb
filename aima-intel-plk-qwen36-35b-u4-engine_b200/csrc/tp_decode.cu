// tp_decode.cu — the peer exchange of tensor-parallel batch-1 decode.
//
// No counterpart in the reference (one Intel iGPU, no collectives). The
// north star shards the decode GEMVs across 2/4/8 GPUs and completes each
// row-parallel sub-block (attention / DeltaNet output projection, MoE
// experts) with an allreduce over NVLink. A batch-1 sub-block exchanges one
// [hidden] fp32 vector per rank (8 KB), so the exchange is latency-bound;
// this is a one-shot allreduce in one small kernel:
//
//   1. each rank stores its partial sum into slot [rank] of every rank's
//      receive buffer (plain peer stores over NVLink into memory mapped
//      with CUDA IPC; no multicast, no bulk-copy engine, no library kernel
//      on peer memory);
//   2. after a __syncthreads and a system-scope fence, thread 0 raises this
//      rank's flag at every rank (st.release.sys of the call's sequence
//      number);
//   3. threads 0..P-1 poll the P flags of their own buffer (ld.acquire.sys,
//      bounded by kWaitLimitNs: on expiry the kernel counts a timeout,
//      readable through iq36_wait_timeouts, and leaves the residual
//      untouched);
//   4. every thread sums the P slots of its elements in rank order and
//      updates the fp32 residual with the fp16-rounded sum, the rounding
//      point of the single-GPU decode step.
//
// Buffers are double-buffered by the parity of the call's sequence number:
// a rank can be at most one call ahead of any peer (to finish call n + 1 it
// needs every peer's flag for n + 1, raised only after that peer finished
// call n), so the slots of call n are never overwritten while being read.
// The sequence number is a per-rank device counter the kernel itself
// advances, so a captured CUDA graph replays it correctly; all ranks issue
// the same sequence of exchanges.

#include <string.h>

#include "common.cuh"
#include "launch.cuh"
#include "sync_sm100.cuh"

namespace iq36 {

constexpr int kTpMaxRanks = 8;
constexpr int kTpThreads = 512;

__device__ int g_tp_wait_timeouts;

struct TpPeers {
  float* recv[kTpMaxRanks];            // each rank's receive buffer [2][P][H] fp32
  unsigned* flags[kTpMaxRanks];        // each rank's flag words [P]
  unsigned long long* keys[kTpMaxRanks];  // each rank's key slots [2][P] (argmax merge)
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Threads 0..P-1 wait for peer tid's flag to reach seq; the result is shared
// through `ok` after a __syncthreads.
__device__ __forceinline__ bool tp_wait_peers(const unsigned* my_flags, int P, unsigned seq,
                                              int* ok) {
  if (threadIdx.x == 0) *ok = 1;
  __syncthreads();
  if ((int)threadIdx.x < P) {
    bool got = false;
    uint64_t t0 = 0;
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
      if ((int)(ld_acquire_sys(my_flags + threadIdx.x) - seq) >= 0) {
        got = true;
        break;
      }
      if (i == 0) t0 = globaltimer_ns();
      else if ((i & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
    if (!got) {
      atomicAdd(&g_tp_wait_timeouts, 1);
      *ok = 0;
    }
  }
  __syncthreads();
  return *ok != 0;
}

__global__ void __launch_bounds__(kTpThreads) tp_allreduce_kernel(TpPeers pr, float* residual,
                                                                   const float* partial,
                                                                   const float* my_recv,
                                                                   const unsigned* my_flags,
                                                                   unsigned* counter, int rank,
                                                                   int P, int H) {
  __shared__ int ok;
  pdl_wait();
  const unsigned seq = *counter + 1u;
  const int par = seq & 1u;
  const int tid = threadIdx.x;
  const float4* src = reinterpret_cast<const float4*>(partial);
  for (int i = tid; i < H / 4; i += kTpThreads) {
    const float4 v = src[i];
    for (int q = 0; q < P; ++q)
      reinterpret_cast<float4*>(pr.recv[q] + ((size_t)par * P + rank) * H)[i] = v;
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    for (int q = 0; q < P; ++q) st_release_sys(pr.flags[q] + rank, seq);
  }
  const bool got = tp_wait_peers(my_flags, P, seq, &ok);
  if (got) {
    for (int i = tid; i < H; i += kTpThreads) {
      float y = 0.f;
      for (int q = 0; q < P; ++q) y += __ldcg(my_recv + ((size_t)par * P + q) * H + i);
      residual[i] = residual[i] + __half2float(__float2half_rn(y));
    }
  }
  __syncthreads();
  if (tid == 0) *counter = seq;
  pdl_launch_dependents();
}

constexpr int kTpKeyBlocks = 148;

// Greedy top-1 key (order-preserving fp32 bits, inverted global id): the
// largest key is the largest logit, lowest id on ties (iq36_greedy_top1.cl:
// 8-13; the same key as the single-GPU argmax).
__device__ __forceinline__ unsigned long long key_of(float v, uint32_t id) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b ^ 0x80000000u);
  return ((unsigned long long)ord << 32) | (unsigned long long)(~id);
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long k) {
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
    k = other > k ? other : k;
  }
  return k;
}

// Per-block best keys of logits[0, n) with global ids id0 + i.
__global__ void __launch_bounds__(256) tp_local_key_kernel(const float* logits, int n, int id0,
                                                           unsigned long long* partial) {
  __shared__ unsigned long long red[8];
  pdl_wait();
  unsigned long long best = 0ull;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const unsigned long long k = key_of(logits[i], (uint32_t)(id0 + i));
    best = k > best ? k : best;
  }
  best = warp_max_u64(best);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  pdl_launch_dependents();
  if (threadIdx.x < 32) {
    best = warp_max_u64(threadIdx.x < 8 ? red[threadIdx.x] : 0ull);
    if (threadIdx.x == 0) partial[blockIdx.x] = best;
  }
}

// This rank's best key (max of the block partials) to every rank's key slot,
// then the largest key over the ranks is the token.
__global__ void __launch_bounds__(256) tp_argmax_merge_kernel(TpPeers pr,
                                                              const unsigned long long* partial,
                                                              int np,
                                                              const unsigned long long* my_keys,
                                                              const unsigned* my_flags,
                                                              unsigned* counter, int rank, int P,
                                                              int32_t* token) {
  __shared__ unsigned long long red[8];
  __shared__ int ok;
  pdl_wait();
  const unsigned seq = *counter + 1u;
  const int par = seq & 1u;
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < np; i += blockDim.x) best = partial[i] > best ? partial[i] : best;
  best = warp_max_u64(best);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x < 32) {
    best = warp_max_u64(threadIdx.x < 8 ? red[threadIdx.x] : 0ull);
    if ((int)threadIdx.x < P) pr.keys[threadIdx.x][par * P + rank] = best;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int q = 0; q < P; ++q) st_release_sys(pr.flags[q] + rank, seq);
  }
  const bool got = tp_wait_peers(my_flags, P, seq, &ok);
  if (threadIdx.x == 0) {
    if (got) {
      unsigned long long m = 0ull;
      for (int q = 0; q < P; ++q) {
        const unsigned long long k = __ldcg(my_keys + par * P + q);
        m = k > m ? k : m;
      }
      *token = (int32_t)(~(uint32_t)(m & 0xFFFFFFFFull));
    }
    *counter = seq;
  }
  pdl_launch_dependents();
}

int tp_wait_timeouts(int* count, int reset) {
  if (cudaMemcpyFromSymbol(count, g_tp_wait_timeouts, sizeof(int)) != cudaSuccess)
    return IQ36_ERR_CUDA;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_tp_wait_timeouts, &zero, sizeof(int)) != cudaSuccess)
      return IQ36_ERR_CUDA;
  }
  return IQ36_OK;
}

static int tp_peers(const iq36_tp_comm* c, TpPeers* pr) {
  if (!c || c->world < 1 || c->world > kTpMaxRanks || c->rank < 0 || c->rank >= c->world ||
      c->hidden < 4 || c->hidden % 4)
    return IQ36_ERR_SHAPE;
  *pr = TpPeers{};
  for (int q = 0; q < c->world; ++q) {
    if (!c->peer_recv[q] || !c->peer_flags[q] || !c->peer_keys[q]) return IQ36_ERR_ARG;
    if (!aligned(c->peer_recv[q], 16)) return IQ36_ERR_ALIGN;
    pr->recv[q] = c->peer_recv[q];
    pr->flags[q] = c->peer_flags[q];
    pr->keys[q] = c->peer_keys[q];
  }
  if (!c->counter) return IQ36_ERR_ARG;
  return IQ36_OK;
}

}  // namespace iq36

extern "C" size_t iq36_tp_argmax_workspace_bytes(void) { return iq36::kTpKeyBlocks * 8; }

extern "C" size_t iq36_tp_comm_bytes(int32_t world, int32_t hidden) {
  // [recv 2 x P x H fp32][flags P u32, padded][keys 2 x P u64][counter]
  return (size_t)2 * world * hidden * 4 + 256 + (size_t)2 * world * 8 + 256;
}

// The exchange buffer is a whole cudaMalloc allocation of its own: a CUDA IPC
// handle names an allocation from its base, and the peers map that base.
extern "C" int iq36_tp_comm_alloc(size_t bytes, void** dev_ptr) {
  if (!dev_ptr || bytes == 0) return IQ36_ERR_ARG;
  if (cudaMalloc(dev_ptr, bytes) != cudaSuccess) return IQ36_ERR_CUDA;
  if (cudaMemset(*dev_ptr, 0, bytes) != cudaSuccess) return IQ36_ERR_CUDA;
  return cudaDeviceSynchronize() == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

extern "C" int iq36_tp_comm_free(void* dev_ptr) {
  if (!dev_ptr) return IQ36_ERR_ARG;
  return cudaFree(dev_ptr) == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

extern "C" int iq36_ipc_get_handle(const void* dev_ptr, void* handle) {
  if (!dev_ptr || !handle) return IQ36_ERR_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)) != cudaSuccess) return IQ36_ERR_CUDA;
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  memcpy(handle, &h, sizeof(h));
  return IQ36_OK;
}

extern "C" int iq36_ipc_open_handle(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return IQ36_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  if (cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return IQ36_ERR_CUDA;
  return IQ36_OK;
}

extern "C" int iq36_ipc_close_handle(void* dev_ptr) {
  if (!dev_ptr) return IQ36_ERR_ARG;
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

extern "C" int iq36_tp_allreduce_residual(const iq36_tp_comm* comm, float* residual,
                                          const float* partial, iq36_stream_t stream) {
  using namespace iq36;
  TpPeers pr;
  const int st = tp_peers(comm, &pr);
  if (st != IQ36_OK) return st;
  if (!residual || !partial) return IQ36_ERR_ARG;
  if (!aligned(partial, 16)) return IQ36_ERR_ALIGN;
  const float* my_recv = comm->local_recv;
  const unsigned* my_flags = comm->local_flags;
  if (!my_recv || !my_flags) return IQ36_ERR_ARG;
  const cudaError_t e =
      launch(tp_allreduce_kernel, dim3(1), dim3(kTpThreads), 0, as_stream(stream), pr, residual,
             partial, my_recv, my_flags, comm->counter, comm->rank, comm->world, comm->hidden);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

extern "C" int iq36_tp_argmax(const iq36_tp_comm* comm, const float* logits_local, int32_t n_local,
                              int32_t id0, int32_t* token_out, void* key_ws,
                              iq36_stream_t stream) {
  using namespace iq36;
  TpPeers pr;
  const int st = tp_peers(comm, &pr);
  if (st != IQ36_OK) return st;
  if (!logits_local || !token_out || !key_ws || n_local < 1 || id0 < 0) return IQ36_ERR_ARG;
  if (!comm->local_keys || !comm->local_flags) return IQ36_ERR_ARG;
  unsigned long long* part = reinterpret_cast<unsigned long long*>(key_ws);
  cudaError_t e = launch(tp_local_key_kernel, dim3(kTpKeyBlocks), dim3(256), 0, as_stream(stream),
                         logits_local, n_local, id0, part);
  if (e != cudaSuccess) return IQ36_ERR_CUDA;
  e = launch(tp_argmax_merge_kernel, dim3(1), dim3(256), 0, as_stream(stream), pr,
             (const unsigned long long*)part, kTpKeyBlocks,
             (const unsigned long long*)comm->local_keys, (const unsigned*)comm->local_flags,
             comm->counter, comm->rank, comm->world, token_out);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}
