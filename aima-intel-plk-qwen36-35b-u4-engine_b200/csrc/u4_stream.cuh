// u4_stream.cuh — bulk-copy streaming version of the u4 dot engine.
//
// One CTA per SM walks a contiguous list of "chunks" (16 weight rows x full
// K). A single producer thread streams every chunk's codes, scales and zero
// points with cp.async.bulk (TMA engine, contiguous 16-byte-multiple pieces,
// no multicast) into a ring of shared-memory stages, each guarded by an
// mbarrier pair (full: transaction bytes; empty: the consuming warp). Because
// weights never depend on the previous kernel, the producer starts before
// griddepcontrol.wait, so up to a full ring of weights per SM is in flight
// while the previous kernel drains. Eight consumer warps run the mma dot
// engine of u4_core.cuh on operands read from shared memory.
//
// Copy granularity sets the stream rate: the bulk-copy engine is bound by
// copies issued, not bytes, for small pieces (measured on B200: 1 KB copies
// cap a 148-SM stream near 3.1 TB/s, 8-16 KB copies reach ~6.2 TB/s). So a
// chunk's codes, scales and zero points each move as one contiguous copy
// (two when the chunk's halves are separate runs, as gate/up rows are), and
// code rows are stored unpadded: the 2-way bank conflict of the consumers'
// 16-byte reads (rows 1 KB apart) costs less shared-memory time than the
// stream delivers per chunk.
#pragma once

#include "sync_sm100.cuh"
#include "u4_core.cuh"

namespace iq36 {

constexpr int kStreamConsumers = 16;                      // consumer warps
constexpr int kStreamThreads = (kStreamConsumers + 1) * 32;
constexpr int kStreamRingBytes = 128 * 1024;
constexpr int kStreamMaxStages = 8;  // mbarrier pairs and stage sequence words reserved
// Rings whose chunks are taken by several independent consumer warps: a fast
// warp can reach chunk c while the stage still holds chunk c - stages (its
// consumer has not released it yet), and an mbarrier's parity cannot tell
// that older phase from chunk c's. So the producer publishes, per stage, the
// index of the chunk it has armed (after arrive.expect_tx); a consumer first
// waits until the stage holds its chunk — from then on the stage cannot move
// past chunk c before this consumer releases it — and then waits on the
// parity of chunk c's phase, which is now exact.
__device__ __forceinline__ void ring_publish(volatile int* seq, int s, int c) {
  __threadfence_block();
  seq[s] = c;
}
__device__ __forceinline__ bool ring_wait(volatile int* seq, uint32_t full_bar, int s, int c,
                                          int stages) {
  if (seq[s] != c) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t i = 0;
    while (seq[s] != c) {
      if ((++i & 255u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
  }
  __threadfence_block();
  return mbar_wait(full_bar, (uint32_t)((c / stages) & 1));
}

bool stream_proj_ok(int K, int G, int n_proj, const iq36_u4_projection* proj);
int stream_proj_launch(const void* x_f16, const float* x_f32, const float* nw, float eps, int K,
                       int G, int n_proj, const iq36_u4_projection* proj, cudaStream_t stream);
int stream_wait_timeouts(int* count, int reset);

// ---- chunk geometry -------------------------------------------------------
// A chunk is two 8-row halves (A = rows 0..7 of the chunk, B = rows 8..15),
// each a run of consecutive rows of one weight matrix with K columns.
struct ChunkSrc {
  const uint8_t* w[2];   // first code row of each half
  const __half* s[2];    // first scale row of each half
  const uint8_t* z[2];   // first zero-point byte of each half (row*ng/2)
  int rows[2];           // valid rows in each half (0..8)
};

struct StreamGeom {
  int K, ng;             // reduction length and groups per row
  int row_pitch;         // shared-memory bytes per code row (K/2)
  int off_scale, off_zp; // offsets inside a stage
  int stage_bytes;
  int stages;
};

__host__ __device__ inline StreamGeom stream_geom(int K, int G) {
  StreamGeom g;
  g.K = K;
  g.ng = K / G;
  g.row_pitch = K / 2;
  g.off_scale = 16 * g.row_pitch;
  g.off_zp = g.off_scale + 16 * g.ng * 2;
  g.stage_bytes = ((g.off_zp + 16 * g.ng / 2) + 127) / 128 * 128;
  g.stages = kStreamRingBytes / g.stage_bytes;
  if (g.stages > kStreamMaxStages) g.stages = kStreamMaxStages;
  return g;
}

// Producer side: copy one chunk into `stage` (shared address), completing on
// `bar`. Returns the number of bytes expected (arrive_tx must precede).
__device__ __forceinline__ uint32_t chunk_bytes(const StreamGeom& g, const ChunkSrc& c) {
  uint32_t b = 0;
  for (int h = 0; h < 2; ++h)
    b += c.rows[h] * (uint32_t)(g.K / 2) + c.rows[h] * g.ng * 2 + c.rows[h] * g.ng / 2;
  return b;
}

// Copies: codes, scales and zero points of the chunk as one run each when
// half B continues half A in global memory, else one run of each per half.
__device__ __forceinline__ void issue_chunk(const StreamGeom& g, const ChunkSrc& c, uint32_t stage,
                                            uint32_t bar) {
  const uint32_t rb = g.K / 2, sb = g.ng * 2, zb = g.ng / 2;  // bytes per row
  if (c.rows[0] == 8 && c.rows[1] == 8 && c.w[1] == c.w[0] + 8 * rb &&
      c.s[1] == c.s[0] + 8 * g.ng && c.z[1] == c.z[0] + 8 * zb) {
    bulk_load(stage, c.w[0], 16 * rb, bar);
    bulk_load(stage + g.off_scale, c.s[0], 16 * sb, bar);
    bulk_load(stage + g.off_zp, c.z[0], 16 * zb, bar);
    return;
  }
  for (int h = 0; h < 2; ++h) {
    const int n = c.rows[h];
    if (n == 0) continue;
    bulk_load(stage + h * 8 * g.row_pitch, c.w[h], n * rb, bar);
    bulk_load(stage + g.off_scale + h * 8 * sb, c.s[h], n * sb, bar);
    bulk_load(stage + g.off_zp + h * 8 * zb, c.z[h], n * zb, bar);
  }
}

// Consumer side: the dot products of the chunk's row g (half A) and row g+8
// (half B) with the staged activation over groups [g_begin, g_end). Lanes of
// a lane group end with identical sums.
//
// The codes enter the mma as fp16 1024+q (even nibbles) and 1024+16q (odd
// nibbles, against x/16) with no per-element zero-point subtraction, so
//   C = sum_k A_k x'_k = 1024*E + 64*O + sum_k q_k x_k,
// with E / O the group's sums of x over even / odd k. The exact group dot is
//   sum_k (q_k - zp) x_k = C - (1024*E + 64*O) - zp*(E + O),
// where xc[group] = {1024*E + 64*O, E + O} comes from the activation staging.
// Products are exact in fp32; C carries the 1024*E offset (|C| ~ 1e4 for unit
// activations), which costs ~1e-4 relative accuracy per group against the
// ~1e-7 of subtracting first, and saves 8 of ~13 instructions per 8 codes.
template <int G>
__device__ __forceinline__ void chunk_dot_range(const StreamGeom& geo, const uint8_t* stage,
                                                const uint4* __restrict__ xs,
                                                const float2* __restrict__ xc, int lane,
                                                int g_begin, int g_end, float& accA,
                                                float& accB) {
  constexpr int W = G / 32;
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* rowA = stage + g * geo.row_pitch + t * (G / 8);
  const uint8_t* rowB = stage + (g + 8) * geo.row_pitch + t * (G / 8);
  const __half* sA = reinterpret_cast<const __half*>(stage + geo.off_scale) + g * geo.ng;
  const __half* sB = reinterpret_cast<const __half*>(stage + geo.off_scale) + (g + 8) * geo.ng;
  const uint8_t* zb = stage + geo.off_zp;
  const int eA = g * geo.ng, eB = (g + 8) * geo.ng;
#pragma unroll 2
  for (int gi = g_begin; gi < g_end; ++gi) {
    uint32_t ra[W], rb[W];
    if constexpr (W == 4) {
      const uint4 va = *reinterpret_cast<const uint4*>(rowA + gi * (G / 2));
      const uint4 vb = *reinterpret_cast<const uint4*>(rowB + gi * (G / 2));
      ra[0] = va.x; ra[1] = va.y; ra[2] = va.z; ra[3] = va.w;
      rb[0] = vb.x; rb[1] = vb.y; rb[2] = vb.z; rb[3] = vb.w;
    } else {
      const uint2 va = *reinterpret_cast<const uint2*>(rowA + gi * (G / 2));
      const uint2 vb = *reinterpret_cast<const uint2*>(rowB + gi * (G / 2));
      ra[0] = va.x; ra[1] = va.y;
      rb[0] = vb.x; rb[1] = vb.y;
    }
    float c0 = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
#pragma unroll
    for (int i = 0; i < W; ++i) {
      const uint4 xv = xs[gi * (G / 8) + t * W + i];
      uint32_t a = ra[i], b = rb[i];
      mma_16816(c0, c1, c2, c3, lop3_and_or(a, 0x000F000Fu, kMagic),
                lop3_and_or(b, 0x000F000Fu, kMagic), lop3_and_or(a, 0x00F000F0u, kMagic),
                lop3_and_or(b, 0x00F000F0u, kMagic), xv.x, xv.y);
      a >>= 8;
      b >>= 8;
      mma_16816(c0, c1, c2, c3, lop3_and_or(a, 0x000F000Fu, kMagic),
                lop3_and_or(b, 0x000F000Fu, kMagic), lop3_and_or(a, 0x00F000F0u, kMagic),
                lop3_and_or(b, 0x00F000F0u, kMagic), xv.z, xv.w);
    }
    const float2 cr = xc[gi];
    const float za = (float)((zb[(eA + gi) >> 1] >> (((eA + gi) & 1) * 4)) & 15u);
    const float zz = (float)((zb[(eB + gi) >> 1] >> (((eB + gi) & 1) * 4)) & 15u);
    accA = fmaf(__half2float(sA[gi]), fmaf(-za, cr.y, c0 - cr.x), accA);
    accB = fmaf(__half2float(sB[gi]), fmaf(-zz, cr.y, c2 - cr.x), accB);
  }
}

// Two chunks at once (stages st0, st1; same group range): two independent
// mma chains per group, each with chunk_dot_range's arithmetic.
template <int G>
__device__ __forceinline__ void chunk_dot_pair(const StreamGeom& geo, const uint8_t* st0,
                                               const uint8_t* st1, const uint4* __restrict__ xs,
                                               const float2* __restrict__ xc, int lane,
                                               int g_begin, int g_end, float& accA0,
                                               float& accB0, float& accA1, float& accB1) {
  static_assert(G == 128, "pair consumption is built for group 128");
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* st[2] = {st0, st1};
  const int eA = g * geo.ng, eB = (g + 8) * geo.ng;
  for (int gi = g_begin; gi < g_end; ++gi) {
    uint4 va[2], vb[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      va[u] = *reinterpret_cast<const uint4*>(st[u] + g * geo.row_pitch + t * (G / 8) + gi * (G / 2));
      vb[u] = *reinterpret_cast<const uint4*>(st[u] + (g + 8) * geo.row_pitch + t * (G / 8) +
                                              gi * (G / 2));
    }
    float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 xv = xs[gi * (G / 8) + t * 4 + i];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        uint32_t a = (&va[u].x)[i], b = (&vb[u].x)[i];
        mma_16816(c[u][0], c[u][1], c[u][2], c[u][3], lop3_and_or(a, 0x000F000Fu, kMagic),
                  lop3_and_or(b, 0x000F000Fu, kMagic), lop3_and_or(a, 0x00F000F0u, kMagic),
                  lop3_and_or(b, 0x00F000F0u, kMagic), xv.x, xv.y);
        a >>= 8;
        b >>= 8;
        mma_16816(c[u][0], c[u][1], c[u][2], c[u][3], lop3_and_or(a, 0x000F000Fu, kMagic),
                  lop3_and_or(b, 0x000F000Fu, kMagic), lop3_and_or(a, 0x00F000F0u, kMagic),
                  lop3_and_or(b, 0x00F000F0u, kMagic), xv.z, xv.w);
      }
    }
    const float2 cr = xc[gi];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const __half* sc = reinterpret_cast<const __half*>(st[u] + geo.off_scale);
      const uint8_t* zb = st[u] + geo.off_zp;
      const float za = (float)((zb[(eA + gi) >> 1] >> (((eA + gi) & 1) * 4)) & 15u);
      const float zz = (float)((zb[(eB + gi) >> 1] >> (((eB + gi) & 1) * 4)) & 15u);
      float& aA = u ? accA1 : accA0;
      float& aB = u ? accB1 : accB0;
      aA = fmaf(__half2float(sc[g * geo.ng + gi]), fmaf(-za, cr.y, c[u][0] - cr.x), aA);
      aB = fmaf(__half2float(sc[(g + 8) * geo.ng + gi]), fmaf(-zz, cr.y, c[u][2] - cr.x), aB);
    }
  }
}

// A consumer warp's activation slice: its quant groups [gb, gb + 2) (16
// consumer warps cover K <= 4096 with at most two groups each) held in
// registers for every chunk, instead of re-read from shared memory per chunk.
struct XSlice {
  uint4 x[2][4];
  float2 c[2];
};

__device__ __forceinline__ void load_xslice(XSlice& xr, const uint4* __restrict__ xs,
                                            const float2* __restrict__ xc, int t, int gb,
                                            int ge) {
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int gi = min(gb + j, ge - 1);
    if (gi < gb) continue;  // empty slice
#pragma unroll
    for (int i = 0; i < 4; ++i) xr.x[j][i] = xs[gi * 16 + t * 4 + i];
    xr.c[j] = xc[gi];
  }
}

// chunk_dot_pair / chunk_dot_range with the activation slice in registers
// (G = 128, ge - gb <= 2): the same arithmetic in the same order.
__device__ __forceinline__ void chunk_dot_pair_x(const StreamGeom& geo, const uint8_t* st0,
                                                 const uint8_t* st1, const XSlice& xr, int lane,
                                                 int gb, int ge, float& accA0, float& accB0,
                                                 float& accA1, float& accB1) {
  constexpr int G = 128;
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* st[2] = {st0, st1};
  const int eA = g * geo.ng, eB = (g + 8) * geo.ng;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int gi = gb + j;
    if (gi >= ge) break;
    uint4 va[2], vb[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      va[u] = *reinterpret_cast<const uint4*>(st[u] + g * geo.row_pitch + t * (G / 8) + gi * (G / 2));
      vb[u] = *reinterpret_cast<const uint4*>(st[u] + (g + 8) * geo.row_pitch + t * (G / 8) +
                                              gi * (G / 2));
    }
    float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 xv = xr.x[j][i];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        uint32_t a = (&va[u].x)[i], b = (&vb[u].x)[i];
        mma_16816(c[u][0], c[u][1], c[u][2], c[u][3], lop3_and_or(a, 0x000F000Fu, kMagic),
                  lop3_and_or(b, 0x000F000Fu, kMagic), lop3_and_or(a, 0x00F000F0u, kMagic),
                  lop3_and_or(b, 0x00F000F0u, kMagic), xv.x, xv.y);
        a >>= 8;
        b >>= 8;
        mma_16816(c[u][0], c[u][1], c[u][2], c[u][3], lop3_and_or(a, 0x000F000Fu, kMagic),
                  lop3_and_or(b, 0x000F000Fu, kMagic), lop3_and_or(a, 0x00F000F0u, kMagic),
                  lop3_and_or(b, 0x00F000F0u, kMagic), xv.z, xv.w);
      }
    }
    const float2 cr = xr.c[j];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const __half* sc = reinterpret_cast<const __half*>(st[u] + geo.off_scale);
      const uint8_t* zb = st[u] + geo.off_zp;
      const float za = (float)((zb[(eA + gi) >> 1] >> (((eA + gi) & 1) * 4)) & 15u);
      const float zz = (float)((zb[(eB + gi) >> 1] >> (((eB + gi) & 1) * 4)) & 15u);
      float& aA = u ? accA1 : accA0;
      float& aB = u ? accB1 : accB0;
      aA = fmaf(__half2float(sc[g * geo.ng + gi]), fmaf(-za, cr.y, c[u][0] - cr.x), aA);
      aB = fmaf(__half2float(sc[(g + 8) * geo.ng + gi]), fmaf(-zz, cr.y, c[u][2] - cr.x), aB);
    }
  }
}

__device__ __forceinline__ void chunk_dot_range_x(const StreamGeom& geo, const uint8_t* stage,
                                                  const XSlice& xr, int lane, int gb, int ge,
                                                  float& accA, float& accB) {
  constexpr int G = 128;
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* rowA = stage + g * geo.row_pitch + t * (G / 8);
  const uint8_t* rowB = stage + (g + 8) * geo.row_pitch + t * (G / 8);
  const __half* sA = reinterpret_cast<const __half*>(stage + geo.off_scale) + g * geo.ng;
  const __half* sB = reinterpret_cast<const __half*>(stage + geo.off_scale) + (g + 8) * geo.ng;
  const uint8_t* zb = stage + geo.off_zp;
  const int eA = g * geo.ng, eB = (g + 8) * geo.ng;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int gi = gb + j;
    if (gi >= ge) break;
    const uint4 va = *reinterpret_cast<const uint4*>(rowA + gi * (G / 2));
    const uint4 vb = *reinterpret_cast<const uint4*>(rowB + gi * (G / 2));
    const uint32_t ra[4] = {va.x, va.y, va.z, va.w}, rb[4] = {vb.x, vb.y, vb.z, vb.w};
    float c0 = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 xv = xr.x[j][i];
      uint32_t a = ra[i], b = rb[i];
      mma_16816(c0, c1, c2, c3, lop3_and_or(a, 0x000F000Fu, kMagic),
                lop3_and_or(b, 0x000F000Fu, kMagic), lop3_and_or(a, 0x00F000F0u, kMagic),
                lop3_and_or(b, 0x00F000F0u, kMagic), xv.x, xv.y);
      a >>= 8;
      b >>= 8;
      mma_16816(c0, c1, c2, c3, lop3_and_or(a, 0x000F000Fu, kMagic),
                lop3_and_or(b, 0x000F000Fu, kMagic), lop3_and_or(a, 0x00F000F0u, kMagic),
                lop3_and_or(b, 0x00F000F0u, kMagic), xv.z, xv.w);
    }
    const float2 cr = xr.c[j];
    const float za = (float)((zb[(eA + gi) >> 1] >> (((eA + gi) & 1) * 4)) & 15u);
    const float zz = (float)((zb[(eB + gi) >> 1] >> (((eB + gi) & 1) * 4)) & 15u);
    accA = fmaf(__half2float(sA[gi]), fmaf(-za, cr.y, c0 - cr.x), accA);
    accB = fmaf(__half2float(sB[gi]), fmaf(-zz, cr.y, c2 - cr.x), accB);
  }
}

template <int G>
__device__ __forceinline__ void chunk_dot(const StreamGeom& geo, const uint8_t* stage,
                                          const uint4* __restrict__ xs,
                                          const float2* __restrict__ xc, int lane, float& accA,
                                          float& accB) {
  chunk_dot_range<G>(geo, stage, xs, xc, lane, 0, geo.ng, accA, accB);
}

}  // namespace iq36
