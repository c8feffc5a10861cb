// u4_stream.cu — streaming (cp.async.bulk ring) version of the decode
// multi-output projections (fixed-FC family, LM head). Semantics are those of
// u4_gemv.cu (same quantisation arithmetic and rounding points); the
// difference is how weights reach the SM and the zero-point handling (see
// u4_stream.cuh). MoE experts stay on the register kernels of moe_decode.cu:
// routed weights cannot be fetched before the router has run, and right after
// the wait those kernels' many independent loads beat one producer thread.
//
// Work split: chunk = 16 rows x full K. Every consumer warp of a CTA works
// on every chunk, a slice of the quant groups each, so a ring stage is
// released a slice-time after it lands and the whole ring stays in flight. The per-warp partial
// sums go to shared memory and are summed in fixed warp order every
// kRedChunks chunks (double-buffered, one named barrier per batch).

#include <algorithm>
#include <atomic>

#include "launch.cuh"
#include "u4_stream.cuh"

namespace iq36 {

constexpr int kStreamCtas = 148;
constexpr int kRedChunks = 8;  // chunks per deferred cross-warp reduction

// Count of bounded waits that gave up, per device (read by iq36_wait_timeouts).
__device__ int g_stream_wait_timeouts;

__device__ __forceinline__ void stream_note_timeout(int* err) {
  if (threadIdx.x % 32 == 0) atomicAdd(&g_stream_wait_timeouts, 1);
  if (err) atomicExch(err, 1);
}

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;\n" ::"r"(kStreamConsumers * 32) : "memory");
}

// Stage the activation for the consumer threads only (named barrier 1):
// xs[c] = permuted fp16 chunk c (see u4_core.cuh), and per quant group
// xc[g] = {1024*E + 64*O, E + O} over the fp16 values actually staged.
template <int G>
__device__ __forceinline__ void stream_stage_x(uint4* xs, float2* xc, const __half* x16,
                                               const float* x32, const float* nw, float eps,
                                               int K, float* red) {
  const int tid = threadIdx.x, nt = kStreamConsumers * 32;
  float scale = 1.0f;
  if (x32 != nullptr) {
    float ss = 0.0f;
    for (int i = tid; i < K; i += nt) ss = fmaf(x32[i], x32[i], ss);
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    consumer_sync();
    float v = 0.f;
    for (int i = 0; i < kStreamConsumers; ++i) v += red[i];
    scale = rsqrtf(v / (float)K + eps);
  }
  const __half2 sixteenth = __float2half2_rn(0.0625f);
  constexpr int kPerGroup = G / 8;  // chunks per quant group (a power of two <= 16)
  for (int base = 0; base < K / 8; base += nt) {
    const int c = base + tid;
    float e = 0.f, o = 0.f;
    if (c < K / 8) {
      __half h[8];
      if (x32 != nullptr) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          h[j] = __float2half_rn(x32[c * 8 + j] * scale * nw[c * 8 + j]);
      } else {
        const uint4 raw = *reinterpret_cast<const uint4*>(x16 + c * 8);
        const __half* hp = reinterpret_cast<const __half*>(&raw);
#pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = hp[j];
      }
      __half2 p0 = __halves2half2(h[0], h[4]);
      __half2 p1 = __hmul2(__halves2half2(h[1], h[5]), sixteenth);
      __half2 p2 = __halves2half2(h[2], h[6]);
      __half2 p3 = __hmul2(__halves2half2(h[3], h[7]), sixteenth);
      uint4 q;
      q.x = *reinterpret_cast<uint32_t*>(&p0);
      q.y = *reinterpret_cast<uint32_t*>(&p1);
      q.z = *reinterpret_cast<uint32_t*>(&p2);
      q.w = *reinterpret_cast<uint32_t*>(&p3);
      xs[c] = q;
      e = (__half2float(h[0]) + __half2float(h[2])) + (__half2float(h[4]) + __half2float(h[6]));
      o = (__half2float(h[1]) + __half2float(h[3])) + (__half2float(h[5]) + __half2float(h[7]));
    }
#pragma unroll
    for (int m = kPerGroup / 2; m > 0; m >>= 1) {
      e += __shfl_xor_sync(0xffffffffu, e, m);
      o += __shfl_xor_sync(0xffffffffu, o, m);
    }
    if (c < K / 8 && (c % kPerGroup) == 0) xc[c / kPerGroup] = make_float2(1024.f * e + 64.f * o, e + o);
  }
  consumer_sync();
}

// Shared-memory layout of every streaming kernel:
//   [ring: stages x stage_bytes][xs: K/8 x 16 B][xc: K/G x 8 B]
//   [red: 2 x kRedChunks x consumer warps x 16 floats][misc: 16 floats]
//   [barriers: full[kStreamMaxStages], empty[kStreamMaxStages]]
//   [seq: chunk armed per stage [kStreamMaxStages], abort flag]
struct StreamSmem {
  uint32_t ring, xs, xc, red, misc, full, empty, seq;
  int total;
};

__host__ __device__ inline StreamSmem stream_smem(const StreamGeom& g, int xs_k, int G) {
  StreamSmem s;
  s.ring = 0;
  s.xs = g.stages * g.stage_bytes;
  s.xc = s.xs + xs_k / 8 * 16;
  s.red = s.xc + (xs_k / G) * 8;
  s.misc = s.red + 2 * kRedChunks * kStreamConsumers * 16 * 4;
  s.full = s.misc + 64;
  s.empty = s.full + 8 * kStreamMaxStages;
  s.seq = s.empty + 8 * kStreamMaxStages;
  s.total = s.seq + 4 * (kStreamMaxStages + 1);
  return s;
}

// ---------------------------------------------------------------------------
// Multi-output projections

struct StreamProj {
  const uint8_t* w[4];
  const __half* s[4];
  const uint8_t* z[4];
  void* out[4];
  int dtype[4];
  int acc[4];
  int chunk_start[5];
  int n_proj;
  // Chunk-list mode (the certified LM head): only the chunks chunk_list[0 ..
  // *chunk_count) are computed, each exactly as in a full launch; a count above
  // chunk_capacity means every chunk. Both words come from the previous
  // launch, so this mode waits before it streams.
  const int* chunk_list;
  const int* chunk_count;
  int chunk_capacity;
};

__device__ __forceinline__ void store_row(void* out, int dtype, int acc, int row, float v) {
  if (dtype == IQ36_F16) {
    reinterpret_cast<__half*>(out)[row] = __float2half_rn(v);
  } else if (acc) {
    float* o = reinterpret_cast<float*>(out);
    o[row] = o[row] + __half2float(__float2half_rn(v));
  } else {
    reinterpret_cast<float*>(out)[row] = v;
  }
}

__device__ __forceinline__ ChunkSrc proj_chunk(const StreamProj& ps, const int* list, int q, int K,
                                               int ng, int& p, int& r0) {
  if (list != nullptr) q = list[q];
  p = 0;
  while (p + 1 < ps.n_proj && q >= ps.chunk_start[p + 1]) ++p;
  r0 = (q - ps.chunk_start[p]) * 16;
  ChunkSrc c;
  for (int h = 0; h < 2; ++h) {
    const int r = r0 + 8 * h;
    c.w[h] = ps.w[p] + (size_t)r * (K / 2);
    c.s[h] = ps.s[p] + (size_t)r * ng;
    c.z[h] = ps.z[p] + (size_t)r * ng / 2;
    c.rows[h] = 8;
  }
  return c;
}

// kList: chunk-list mode, compiled as its own instantiation so that the
// list handling adds no registers to the decode projections (sharing one
// instantiation spilled and cost ~0.7 us per launch).
template <int G, bool kList>
__global__ void __launch_bounds__(kStreamThreads, 1)
    u4_stream_proj_kernel(StreamProj ps, const __half* x16, const float* x32, const float* nw,
                          float eps, int K, int* err) {
  extern __shared__ __align__(128) uint8_t smem[];
  const StreamGeom geo = stream_geom(K, G);
  const StreamSmem L = stream_smem(geo, K, G);
  const uint32_t sbase = smem_u32(smem);
  volatile int* seq = reinterpret_cast<volatile int*>(smem + L.seq);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int total = ps.chunk_start[ps.n_proj];
  const int* list = nullptr;
  if constexpr (kList) {
    pdl_wait();
    const int n = *ps.chunk_count;
    if (n <= ps.chunk_capacity) {
      total = n;
      list = ps.chunk_list;
    }
  }
  const int per = (total + gridDim.x - 1) / gridDim.x;
  const int c0 = blockIdx.x * per, nloc = max(min(c0 + per, total) - c0, 0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < geo.stages; ++s) {
      mbar_init(sbase + L.full + 8 * s, 1);
      mbar_init(sbase + L.empty + 8 * s, kStreamConsumers);
    }
    for (int s = 0; s < kStreamMaxStages; ++s) seq[s] = -1;  // no chunk armed yet
    seq[kStreamMaxStages] = 0;                                // abort flag
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  bool ok = true;
  if (warp == kStreamConsumers) {
    // producer: weights only, no dependency on the previous kernel
    pdl_launch_dependents();
    if (lane == 0) {
      for (int c = 0; c < nloc && ok; ++c) {
        const int s = c % geo.stages;
        const uint32_t ph = (uint32_t)((c / geo.stages) & 1);
        ok = mbar_wait(sbase + L.empty + 8 * s, ph ^ 1u);
        if (!ok) break;
        int p, r0;
        const ChunkSrc src = proj_chunk(ps, list, c0 + c, K, geo.ng, p, r0);
        mbar_arrive_tx(sbase + L.full + 8 * s, chunk_bytes(geo, src));
        ring_publish(seq, s, c);
        issue_chunk(geo, src, sbase + L.ring + s * geo.stage_bytes, sbase + L.full + 8 * s);
      }
    }
  } else {
    pdl_wait();
    float* red = reinterpret_cast<float*>(smem + L.red);
    uint4* xs = reinterpret_cast<uint4*>(smem + L.xs);
    float2* xc = reinterpret_cast<float2*>(smem + L.xc);
    stream_stage_x<G>(xs, xc, x16, x32, nw, eps, K, reinterpret_cast<float*>(smem + L.misc));
    pdl_launch_dependents();
    const int g = lane >> 2, t = lane & 3;
    const int gb = warp * geo.ng / kStreamConsumers, ge = (warp + 1) * geo.ng / kStreamConsumers;
    XSlice xr;
    load_xslice(xr, xs, xc, t, gb, ge);
    // With four or more ring stages the warps take chunks in pairs (two
    // independent mma chains per group); the sums per chunk are unchanged.
    const bool pair = geo.stages >= 4;
    int c = 0;
    while (c < nloc && ok) {
      const int n = (pair && c + 1 < nloc) ? 2 : 1;
      const int s0 = c % geo.stages, s1 = (c + 1) % geo.stages;
      float a0 = 0.f, b0 = 0.f, a1 = 0.f, b1 = 0.f;
      bool got = __all_sync(0xffffffffu, ring_wait(seq, sbase + L.full + 8 * s0, s0, c, geo.stages));
      if (got && n == 2)
        got = __all_sync(0xffffffffu,
                         ring_wait(seq, sbase + L.full + 8 * s1, s1, c + 1, geo.stages));
      if (got) {
        if (n == 2)
          chunk_dot_pair_x(geo, smem + L.ring + s0 * geo.stage_bytes,
                           smem + L.ring + s1 * geo.stage_bytes, xr, lane, gb, ge, a0, b0, a1, b1);
        else
          chunk_dot_range_x(geo, smem + L.ring + s0 * geo.stage_bytes, xr, lane, gb, ge, a0, b0);
        // generic reads of the stages before the producer's next bulk copies
        // (async proxy) into them
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(sbase + L.empty + 8 * s0);
          if (n == 2) mbar_arrive(sbase + L.empty + 8 * s1);
        }
      } else if (lane == 0) {
        seq[kStreamMaxStages] = 1;  // shared so every consumer warp leaves at the barrier below
      }
      for (int u = 0; u < n && ok; ++u) {
        const int cc = c + u, j = cc % kRedChunks;
        float* rbuf = red + ((cc / kRedChunks) & 1) * kRedChunks * kStreamConsumers * 16;
        if (t == 0) {
          rbuf[(j * kStreamConsumers + warp) * 16 + g] = u ? a1 : a0;
          rbuf[(j * kStreamConsumers + warp) * 16 + g + 8] = u ? b1 : b0;
        }
        if (j == kRedChunks - 1 || cc == nloc - 1) {
          consumer_sync();
          if (seq[kStreamMaxStages] != 0) {
            ok = false;
            break;
          }
          for (int i = threadIdx.x; i < (j + 1) * 16; i += kStreamConsumers * 32) {
            const int jj = i >> 4, r = i & 15;
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kStreamConsumers; ++w)
              v += rbuf[(jj * kStreamConsumers + w) * 16 + r];
            int p, r0;
            proj_chunk(ps, list, c0 + cc - j + jj, K, geo.ng, p, r0);
            store_row(ps.out[p], ps.dtype[p], ps.acc[p], r0 + r, v);
          }
        }
      }
      c += n;
    }
  }
  if (!ok) stream_note_timeout(err);
}

// ---------------------------------------------------------------------------
// Host launchers

// The dynamic shared-memory opt-in is a per-device function attribute: set it
// once per device to the largest layout any K (<= 4096) needs.
template <bool kList>
static int stream_attr() {
  const void* fn = (const void*)u4_stream_proj_kernel<128, kList>;
  static std::atomic<bool> attr_set[64];  // per instantiation
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return IQ36_ERR_CUDA;
  if (attr_set[dev].load(std::memory_order_acquire)) return IQ36_OK;
  int bytes = 0;
  for (int K = 512; K <= 4096; K += 512)
    bytes = std::max(bytes, stream_smem(stream_geom(K, 128), K, 128).total);
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return IQ36_ERR_CUDA;
  attr_set[dev].store(true, std::memory_order_release);
  return IQ36_OK;
}

bool stream_proj_ok(int K, int G, int n_proj, const iq36_u4_projection* proj) {
  if (G != 128 || K % 512 || K > 4096) return false;
  for (int i = 0; i < n_proj; ++i) {
    const iq36_u4_projection& p = proj[i];
    if (p.m.rows % 16 || !aligned(p.m.weight, 16) || !aligned(p.m.scale, 16) ||
        !aligned(p.m.zp, 16))
      return false;
  }
  return true;
}

int stream_proj_launch(const void* x_f16, const float* x_f32, const float* nw, float eps, int K,
                       int G, int n_proj, const iq36_u4_projection* proj, cudaStream_t stream) {
  StreamProj ps = {};
  ps.n_proj = n_proj;
  int ch = 0;
  for (int i = 0; i < n_proj; ++i) {
    ps.w[i] = proj[i].m.weight;
    ps.s[i] = reinterpret_cast<const __half*>(proj[i].m.scale);
    ps.z[i] = proj[i].m.zp;
    ps.out[i] = proj[i].out;
    ps.dtype[i] = proj[i].out_dtype;
    ps.acc[i] = proj[i].accumulate;
    ps.chunk_start[i] = ch;
    ch += proj[i].m.rows / 16;
  }
  ps.chunk_start[n_proj] = ch;
  const StreamGeom geo = stream_geom(K, G);
  const StreamSmem L = stream_smem(geo, K, G);
  const int grid = std::min(kStreamCtas, ch);
  if (stream_attr<false>() != IQ36_OK)
    return IQ36_ERR_CUDA;
  const cudaError_t e =
      launch(u4_stream_proj_kernel<128, false>, dim3(grid), dim3(kStreamThreads), (size_t)L.total, stream,
             ps, reinterpret_cast<const __half*>(x_f16), x_f32, nw, eps, K, (int*)nullptr);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

int stream_wait_timeouts(int* count, int reset) {
  if (cudaMemcpyFromSymbol(count, g_stream_wait_timeouts, sizeof(int)) != cudaSuccess)
    return IQ36_ERR_CUDA;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_stream_wait_timeouts, &zero, sizeof(int)) != cudaSuccess)
      return IQ36_ERR_CUDA;
  }
  return IQ36_OK;
}

}  // namespace iq36


// ---------------------------------------------------------------------------
// LM-head certified greedy top-1
//
// Greedy decode needs only the argmax of the head. Each row's logit is bounded
// by Cauchy-Schwarz per quant group, sum_g |s_rg| ||q_rg - zp_rg||_2 ||x_g||_2,
// plus max_g |s_rg| * sum_g guard_g for the fp32 rounding of the group sums.
// A lower bound on the logit of some row (the best row of the seed token's
// 16-row chunk, computed here in fp32 minus twice its rounding guard) sets the
// bar; chunks holding a row whose bound reaches it are computed by the
// streaming kernel above in chunk-list mode, i.e. with the full head's own
// arithmetic, so their argmax (lowest id on ties) is the full head's argmax
// bit for bit. More chunks than the capacity: every chunk.

namespace iq36 {

constexpr float kCertGuardRel = 1.0f / 4096.0f;  // > 16 fp32 ulps of the group sums' terms
// An odd activation below 2^-10 loses bits when staged as x/16 (fp16
// subnormal); each such element moves the group sum by at most (64 + 15) * 2^-21.
constexpr float kCertGuardAbs = 64.0f * 80.0f / 2097152.0f;
constexpr int kCertArgmaxBlocks = 148;

// table[r * ng + g] = |s_rg| * ||q_rg - zp_rg||_2 rounded up, then
// table[rows * ng + r] = max_g |s_rg| (one thread per row; built once).
__global__ void __launch_bounds__(256) cert_table_kernel(const uint8_t* w, const __half* s,
                                                         const uint8_t* z, int rows, int K,
                                                         __half* table) {
  const int ng = K / 128;
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float smax = 0.f;
  for (int g = 0; g < ng; ++g) {
    const int64_t idx = (int64_t)r * ng + g;
    const uint4* row = reinterpret_cast<const uint4*>(w + (int64_t)r * (K / 2) + g * 64);
    const int zp = (z[idx >> 1] >> ((idx & 1) * 4)) & 15;
    int ss = 0;  // exact: at most 128 * 225
    for (int i = 0; i < 4; ++i) {
      const uint4 v = row[i];
      const uint32_t words[4] = {v.x, v.y, v.z, v.w};
      for (int j = 0; j < 4; ++j)
        for (int b = 0; b < 8; ++b) {
          const int d = (int)((words[j] >> (4 * b)) & 15u) - zp;
          ss += d * d;
        }
    }
    const float a = fabsf(__half2float(s[idx]));
    smax = fmaxf(smax, a);
    table[idx] = __float2half_ru(sqrtf((float)ss) * a * (1.0f + 1.0f / 1048576.0f));
  }
  table[(int64_t)rows * ng + r] = __float2half_ru(smax);
}

struct CertMisc {
  float guard_sum;  // sum_g guard_g
  float bar;        // lower bound on the best logit of the seed chunk
  int count;        // chunks appended by the scan
  int done;         // argmax blocks finished
};

// One CTA of the streaming kernel's 16 consumer warps: the same staged
// activation (stream_stage_x); per quant group ||x_g|| (rounded up) and the
// rounding guard; the seed chunk's 16 logits in fp32 (one warp per row) and
// the bar; the counters cleared.
__global__ void __launch_bounds__(kStreamConsumers * 32) cert_prep_kernel(
    const __half* x16, const float* x32, const float* nw, float eps, int K, int rows,
    const __half* s, const uint8_t* z, const uint8_t* w, const __half* table,
    const int32_t* seed_token, float* xnorm, CertMisc* misc) {
  extern __shared__ __align__(16) uint8_t sm[];
  uint4* xs = reinterpret_cast<uint4*>(sm);
  float2* xc = reinterpret_cast<float2*>(sm + K / 8 * 16);
  float* red = reinterpret_cast<float*>(sm + K / 8 * 16 + K / 128 * 8);  // 16 floats
  float* gsm = red + 16;                                                 // 32 guards
  float* lbs = gsm + 32;                                                 // 16 row bars
  pdl_wait();
  stream_stage_x<128>(xs, xc, x16, x32, nw, eps, K, red);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ng = K / 128;
  for (int g = warp; g < ng; g += kStreamConsumers) {
    // 16 staged uint4 per group, one per lane l < 16. A staged uint4 holds the
    // pairs (x0,x4), (x1,x5)/16, (x2,x6), (x3,x7)/16: words 0 and 2 carry even
    // k, words 1 and 3 odd k divided by 16 (multiplied back here).
    float sq = 0.f, ae = 0.f, ao = 0.f;
    if (lane < 16) {
      const uint4 v = xs[g * 16 + lane];
      const __half2* hp = reinterpret_cast<const __half2*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(hp[j]);
        const float m = (j & 1) ? 16.f : 1.f;
        const float a = f.x * m, b = f.y * m;
        sq += a * a + b * b;
        if (j & 1) ao += fabsf(a) + fabsf(b);
        else ae += fabsf(a) + fabsf(b);
      }
    }
    sq = warp_sum(sq);
    ae = warp_sum(ae);
    ao = warp_sum(ao);
    if (lane == 0) {
      xnorm[g] = sqrtf(sq * (1.0f + 1.0f / 65536.0f)) * (1.0f + 1.0f / 1048576.0f);
      gsm[g] = kCertGuardRel * (1024.f * ae + 64.f * ao + 16.f * (ae + ao)) + kCertGuardAbs;
    }
  }
  consumer_sync();
  float gsum = 0.f;
  for (int g = 0; g < ng; ++g) gsum += gsm[g];
  gsum *= 1.0f + 1.0f / 65536.0f;
  // the seed chunk: warp = row within the chunk
  const int r = min(max(*seed_token, 0), rows - 1) / 16 * 16 + warp;
  float acc = 0.f;
  for (int c = lane; c < K / 8; c += 32) {
    const int g = c / 16;
    const int64_t gi = (int64_t)r * ng + g;
    const int zp = (z[gi >> 1] >> ((gi & 1) * 4)) & 15;
    const uint32_t wb = *reinterpret_cast<const uint32_t*>(w + (int64_t)r * (K / 2) + c * 4);
    const uint4 v = xs[c];
    const __half2* hp = reinterpret_cast<const __half2*>(&v);
    // staged order: k = 0,4 | 1,5 (/16) | 2,6 | 3,7 (/16)
    const float2 p0 = __half22float2(hp[0]), p1 = __half22float2(hp[1]);
    const float2 p2 = __half22float2(hp[2]), p3 = __half22float2(hp[3]);
    const float xv[8] = {p0.x, 16.f * p1.x, p2.x, 16.f * p3.x, p0.y, 16.f * p1.y, p2.y, 16.f * p3.y};
    float d = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) d = fmaf((float)((int)((wb >> (4 * j)) & 15u) - zp), xv[j], d);
    acc = fmaf(__half2float(s[gi]), d, acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) {
    const float guard = __half2float(table[(int64_t)rows * ng + r]) * gsum;
    lbs[warp] = acc - 2.0f * guard * (1.0f + 1.0f / 1024.0f);
  }
  consumer_sync();
  if (threadIdx.x == 0) {
    float bar = lbs[0];
    for (int i = 1; i < 16; ++i) bar = fmaxf(bar, lbs[i]);
    misc->guard_sum = gsum;
    misc->bar = bar;
    misc->count = 0;
    misc->done = 0;
  }
  pdl_launch_dependents();
}

// One thread per row: the bound against the bar; flagged chunks appended to
// the list, one atomic per CTA (16 chunks). The table is constant per head and
// read before the wait.
__global__ void __launch_bounds__(256) cert_scan_kernel(const __half* table, int rows, int K,
                                                        const float* xnorm, CertMisc* misc,
                                                        int* list) {
  __shared__ float xn[32];
  __shared__ int fl[16];
  const int ng = K / 128;
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  float t[32];
  float smax = 0.f;
  if (r < rows) {
    const uint2* tr = reinterpret_cast<const uint2*>(table + (int64_t)r * ng);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < ng / 4) {
        const uint2 v = tr[i];
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
        t[4 * i] = a.x;
        t[4 * i + 1] = a.y;
        t[4 * i + 2] = b.x;
        t[4 * i + 3] = b.y;
      }
    smax = __half2float(table[(int64_t)rows * ng + r]);
  }
  pdl_wait();
  if (threadIdx.x < ng) xn[threadIdx.x] = xnorm[threadIdx.x];
  __syncthreads();
  bool f = false;
  if (r < rows) {
    float up = 0.f;
#pragma unroll
    for (int g = 0; g < 32; ++g)
      if (g < ng) up = fmaf(t[g], xn[g], up);
    up = fmaf(smax, misc->guard_sum, up) * (1.0f + 1.0f / 65536.0f);
    f = up >= misc->bar;
  }
  const unsigned m = __ballot_sync(0xffffffffu, f);
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    fl[2 * warp] = (m & 0xFFFFu) != 0u;
    fl[2 * warp + 1] = (m >> 16) != 0u;
  }
  __syncthreads();
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    int n = 0;
    for (int i = 0; i < 16; ++i) n += fl[i];
    if (n > 0) {
      int slot = atomicAdd(&misc->count, n);
      const int nchunks = rows / 16;
      for (int i = 0; i < 16; ++i)
        if (fl[i] && slot < nchunks) list[slot++] = blockIdx.x * 16 + i;
    }
  }
}

// Order-preserving key: larger logit first, then the lower row id.
__device__ __forceinline__ uint64_t cert_key(float v, uint32_t id) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b ^ 0x80000000u);
  return ((uint64_t)ord << 32) | (uint64_t)(~id);
}

__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t other = __shfl_xor_sync(0xffffffffu, v, o);
    v = other > v ? other : v;
  }
  return v;
}

// Argmax over the evaluated chunks; the last CTA to finish merges the
// per-CTA keys (no waiting: the others have published theirs before counting).
__global__ void __launch_bounds__(256) cert_argmax_kernel(const float* logits, int rows,
                                                          const int* list, int capacity,
                                                          CertMisc* misc, uint64_t* partial,
                                                          int32_t* token, int32_t* evaluated) {
  __shared__ uint64_t red[8];
  __shared__ bool last;
  pdl_wait();
  const int count = misc->count;
  const bool all = count > capacity;
  const int n = all ? rows : count * 16;
  uint64_t best = 0ull;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int row = all ? i : list[i >> 4] * 16 + (i & 15);
    const uint64_t k = cert_key(logits[row], (uint32_t)row);
    best = k > best ? k : best;
  }
  best = warp_max_u64(best);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 0; w < 8; ++w) best = red[w] > best ? red[w] : best;
    partial[blockIdx.x] = best;
    __threadfence();
    last = atomicAdd(&misc->done, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x < 32) {
    __threadfence();
    uint64_t b = 0ull;
    for (int i = threadIdx.x; i < (int)gridDim.x; i += 32) {
      const uint64_t v = __ldcg(reinterpret_cast<const unsigned long long*>(partial) + i);
      b = v > b ? v : b;
    }
    b = warp_max_u64(b);
    if (threadIdx.x == 0) {
      *token = (int32_t)(~(uint32_t)(b & 0xFFFFFFFFull));
      if (evaluated) *evaluated = all ? rows / 16 : count;
      misc->done = 0;
    }
  }
}

struct CertWs {
  float* xnorm;
  CertMisc* misc;
  int* list;
  uint64_t* partial;
  size_t bytes;
};

static CertWs cert_ws(void* base, int rows) {
  CertWs w;
  char* p = reinterpret_cast<char*>(base);
  auto take = [&](size_t n) {
    char* q = p;
    p += (n + 255) / 256 * 256;
    return q;
  };
  w.xnorm = reinterpret_cast<float*>(take(32 * 4));
  w.misc = reinterpret_cast<CertMisc*>(take(sizeof(CertMisc)));
  w.list = reinterpret_cast<int*>(take((size_t)(rows / 16) * 4));
  w.partial = reinterpret_cast<uint64_t*>(take(kCertArgmaxBlocks * 8));
  w.bytes = (size_t)(p - reinterpret_cast<char*>(base));
  return w;
}

}  // namespace iq36

extern "C" size_t iq36_lm_head_cert_table_bytes(int32_t rows, int32_t K, int32_t G) {
  if (rows < 16 || rows % 16 || G != 128 || K % 512 || K > 4096) return 0;
  return (size_t)rows * (K / 128 + 1) * 2;
}

extern "C" int iq36_lm_head_cert_table(const iq36_u4_matrix* w, int32_t K, int32_t G,
                                       void* table_f16, iq36_stream_t stream) {
  using namespace iq36;
  if (!w || !w->weight || !w->scale || !w->zp || !table_f16) return IQ36_ERR_ARG;
  if (iq36_lm_head_cert_table_bytes(w->rows, K, G) == 0) return IQ36_ERR_SHAPE;
  if (!aligned(w->weight, 16) || !aligned(table_f16, 16)) return IQ36_ERR_ALIGN;
  cert_table_kernel<<<(unsigned)((w->rows + 255) / 256), 256, 0, as_stream(stream)>>>(
      w->weight, reinterpret_cast<const __half*>(w->scale), w->zp, w->rows, K,
      reinterpret_cast<__half*>(table_f16));
  return cudaGetLastError() == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

extern "C" size_t iq36_lm_head_top1_certified_workspace_bytes(int32_t rows, int32_t K) {
  if (rows < 16 || rows % 16 || K < 512) return 0;
  return iq36::cert_ws(nullptr, rows).bytes;
}

extern "C" int iq36_lm_head_top1_certified(const void* x_f16, const float* x_f32,
                                           const float* norm_weight, float norm_eps, int32_t K,
                                           int32_t G, const iq36_u4_matrix* w,
                                           const void* table_f16, const int32_t* seed_token,
                                           int32_t capacity_chunks, float* logits,
                                           int32_t* token_out, int32_t* evaluated_chunks,
                                           void* workspace, size_t workspace_bytes,
                                           iq36_stream_t stream) {
  using namespace iq36;
  if (!w || !w->weight || !w->scale || !w->zp || !table_f16 || !seed_token || !logits ||
      !token_out || !workspace)
    return IQ36_ERR_ARG;
  if (x_f32) {
    if (x_f16 || !norm_weight) return IQ36_ERR_ARG;
  } else if (!x_f16) {
    return IQ36_ERR_ARG;
  }
  iq36_u4_projection proj{*w, logits, IQ36_F32, 0};
  if (iq36_lm_head_cert_table_bytes(w->rows, K, G) == 0 || !stream_proj_ok(K, G, 1, &proj))
    return IQ36_ERR_SHAPE;
  if (capacity_chunks < 1) return IQ36_ERR_SHAPE;
  const CertWs ws = cert_ws(workspace, w->rows);
  if (workspace_bytes < ws.bytes) return IQ36_ERR_WORKSPACE;
  if (!aligned(workspace, 256) || !aligned(table_f16, 16)) return IQ36_ERR_ALIGN;
  if (x_f16 && !aligned(x_f16, 16)) return IQ36_ERR_ALIGN;
  const cudaStream_t s = as_stream(stream);
  const int nchunks = w->rows / 16;
  const __half* sc = reinterpret_cast<const __half*>(w->scale);
  const __half* tb = reinterpret_cast<const __half*>(table_f16);
  const size_t prep_smem = (size_t)K / 8 * 16 + K / 128 * 8 + 64 * 4;
  cudaError_t e = launch(cert_prep_kernel, dim3(1), dim3(kStreamConsumers * 32), prep_smem, s,
                         reinterpret_cast<const __half*>(x_f16), x_f32, norm_weight, norm_eps, K,
                         w->rows, sc, w->zp, w->weight, tb, seed_token, ws.xnorm, ws.misc);
  if (e != cudaSuccess) return IQ36_ERR_CUDA;
  e = launch(cert_scan_kernel, dim3((w->rows + 255) / 256), dim3(256), 0, s, tb, w->rows, K,
             (const float*)ws.xnorm, ws.misc, ws.list);
  if (e != cudaSuccess) return IQ36_ERR_CUDA;
  StreamProj ps = {};
  ps.n_proj = 1;
  ps.w[0] = w->weight;
  ps.s[0] = sc;
  ps.z[0] = w->zp;
  ps.out[0] = logits;
  ps.dtype[0] = IQ36_F32;
  ps.acc[0] = 0;
  ps.chunk_start[0] = 0;
  ps.chunk_start[1] = nchunks;
  ps.chunk_list = ws.list;
  ps.chunk_count = &ws.misc->count;
  ps.chunk_capacity = capacity_chunks;
  const StreamGeom geo = stream_geom(K, G);
  const StreamSmem L = stream_smem(geo, K, G);
  if (stream_attr<true>() != IQ36_OK) return IQ36_ERR_CUDA;
  e = launch(u4_stream_proj_kernel<128, true>, dim3(std::min(kStreamCtas, nchunks)),
             dim3(kStreamThreads), (size_t)L.total, s, ps,
             reinterpret_cast<const __half*>(x_f16), x_f32, norm_weight, norm_eps, K,
             (int*)nullptr);
  if (e != cudaSuccess) return IQ36_ERR_CUDA;
  e = launch(cert_argmax_kernel, dim3(kCertArgmaxBlocks), dim3(256), 0, s, (const float*)logits,
             w->rows, (const int*)ws.list, (int)capacity_chunks, ws.misc, ws.partial, token_out,
             evaluated_chunks);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}
