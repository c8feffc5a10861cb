// u4_core.cuh — the u4 group-wise dequant dot engine shared by every GEMV-shaped
// kernel (plain projections, MoE gate_up + SwiGLU, MoE down + combine, LM head).
//
// Semantics (reference engine/openvino/custom/iq36_fixed_fc_multi_output.cl:
// 112-167): y[n] = sum_k x[k] * (q[n,k] - zp[n,g]) * s[n,g], g = k / G.
//
// Work decomposition. One warp owns 16 weight rows, split as "row A" (lane
// group g = lane/4 -> row g) and "row B" (row g+8), and walks K one quant group
// per step. Lane t = lane%4 streams G/8 contiguous bytes of each of its two
// rows per group, so a warp moves 16 rows x G/2 bytes per step in 32-byte
// sectors that are fully used.
//
// Unpack. Each 32-bit word holds 8 codes (low nibble = even k). Two LOP3s per
// half2 build fp16 values 1024+q (mask 0x000F000F) and 1024+16q (mask
// 0x00F000F0) by OR-ing the magic exponent 0x6400; one HSUB2 against the
// per-group constant 1024+zp (or 1024+16zp) leaves the exact integer q-zp (or
// 16(q-zp)) in fp16. The words shifted right by 8 give the other four codes.
//
// Dot. The dequantised codes are the A operand of mma.m16n8k16 (rows = the
// warp's 16 weight rows, k = 16 codes); B is the activation, staged once per
// CTA in shared memory in the matching permuted order with the odd codes'
// activations pre-divided by 16 (exact: a power of two). Every B column holds
// the same activation, so each lane's c0 (row A) and c2 (row B) carry the full
// group dot product, exact products accumulated in fp32. The group result is
// scaled by s[n,g] in fp32 FMA. The tensor pipe here is only a cheap exact
// dot engine: the kernel is bound by HBM, and the mma keeps the unpack at
// ~1.3 issued instructions per weight so the ALUs never limit the stream.
#pragma once

#include "common.cuh"

namespace iq36 {

constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024.0 in both halves

// Stage an fp16 activation vector into the permuted layout consumed by
// u4_dot2: chunk c (k = 8c..8c+7) -> {(x0,x4), (x1,x5)/16, (x2,x6), (x3,x7)/16}.
// When x32 != nullptr the activation is first RMS-normalised (fp32 input,
// per-element weight, eps) and rounded to fp16 (reference
// engine/src/gguf_loader.cpp:3368-3391 then the fp16 Convert in front of every
// fixed-FC, tools/intel_qwen36_openvino_fixed_fc.py:292-296).
// Block-wide; ends with __syncthreads().
__device__ __forceinline__ void stage_x_perm(uint4* xs, const __half* x16, const float* x32,
                                             const float* norm_w, float eps, int K,
                                             float* red /* >= 33 floats */) {
  const int tid = threadIdx.x, nt = blockDim.x;
  float scale = 1.0f;
  if (x32 != nullptr) {
    float ss = 0.0f;
    for (int i = tid; i < K; i += nt) ss = fmaf(x32[i], x32[i], ss);
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    if (tid < 32) {
      float v = tid < (nt >> 5) ? red[tid] : 0.0f;
      v = warp_sum(v);
      if (tid == 0) red[32] = rsqrtf(v / (float)K + eps);
    }
    __syncthreads();
    scale = red[32];
  }
  const __half2 sixteenth = __float2half2_rn(0.0625f);
  for (int c = tid; c < K / 8; c += nt) {
    __half h[8];
    if (x32 != nullptr) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int k = c * 8 + j;
        h[j] = __float2half_rn(x32[k] * scale * norm_w[k]);
      }
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
    uint4 o;
    o.x = *reinterpret_cast<uint32_t*>(&p0);
    o.y = *reinterpret_cast<uint32_t*>(&p1);
    o.z = *reinterpret_cast<uint32_t*>(&p2);
    o.w = *reinterpret_cast<uint32_t*>(&p3);
    xs[c] = o;
  }
  __syncthreads();
}

__device__ __forceinline__ uint32_t zp_nibble(const uint8_t* zp, int64_t e) {
  return (uint32_t)(__ldg(zp + (e >> 1)) >> ((e & 1) * 4)) & 15u;
}

// One prefetched chunk: U quant groups of the lane's two rows (codes, scales,
// zero points) held in registers.
template <int G, int U>
struct U4Chunk {
  uint32_t ra[U][G / 32], rb[U][G / 32];
  uint32_t za[U], zb[U];
  float sa[U], sb[U];
};

// Row pair of one warp task: row starts, scale row starts, zp element index of
// (row, group 0).
struct U4Rows {
  const uint8_t* wA;
  const uint8_t* wB;
  const __half* sA;
  const __half* sB;
  const uint8_t* zp;
  int64_t zeA, zeB;
};

template <int G, int U>
__device__ __forceinline__ void u4_load_chunk(U4Chunk<G, U>& c, const U4Rows& r, int g0, int g_end,
                                              int t) {
  constexpr int W = G / 32;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int gi = min(g0 + u, g_end - 1);
    const int off = gi * (G / 2) + t * (G / 8);
    if constexpr (W == 4) {
      const uint4 va = ld_stream_v4(r.wA + off);
      const uint4 vb = ld_stream_v4(r.wB + off);
      c.ra[u][0] = va.x; c.ra[u][1] = va.y; c.ra[u][2] = va.z; c.ra[u][3] = va.w;
      c.rb[u][0] = vb.x; c.rb[u][1] = vb.y; c.rb[u][2] = vb.z; c.rb[u][3] = vb.w;
    } else {
      const uint2 va = ld_stream_v2(r.wA + off);
      const uint2 vb = ld_stream_v2(r.wB + off);
      c.ra[u][0] = va.x; c.ra[u][1] = va.y;
      c.rb[u][0] = vb.x; c.rb[u][1] = vb.y;
    }
    c.sa[u] = __half2float(r.sA[gi]);
    c.sb[u] = __half2float(r.sB[gi]);
    c.za[u] = zp_nibble(r.zp, r.zeA + gi);
    c.zb[u] = zp_nibble(r.zp, r.zeB + gi);
  }
}

template <int G, int U>
__device__ __forceinline__ void u4_compute_chunk(const U4Chunk<G, U>& c,
                                                 const uint4* __restrict__ xs, int g0, int g_end,
                                                 int t, float& accA, float& accB) {
  constexpr int W = G / 32;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (g0 + u < g_end) {
      const int gi = g0 + u;
      const uint32_t zloA = kMagic | c.za[u] | (c.za[u] << 16);
      const uint32_t zhiA = kMagic | (c.za[u] << 4) | (c.za[u] << 20);
      const uint32_t zloB = kMagic | c.zb[u] | (c.zb[u] << 16);
      const uint32_t zhiB = kMagic | (c.zb[u] << 4) | (c.zb[u] << 20);
      float c0 = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
#pragma unroll
      for (int i = 0; i < W; ++i) {
        const uint4 xv = xs[gi * (G / 8) + t * W + i];
        uint32_t a = c.ra[u][i], b = c.rb[u][i];
        mma_16816(c0, c1, c2, c3, hsub2_u32(lop3_and_or(a, 0x000F000Fu, kMagic), zloA),
                  hsub2_u32(lop3_and_or(b, 0x000F000Fu, kMagic), zloB),
                  hsub2_u32(lop3_and_or(a, 0x00F000F0u, kMagic), zhiA),
                  hsub2_u32(lop3_and_or(b, 0x00F000F0u, kMagic), zhiB), xv.x, xv.y);
        a >>= 8;
        b >>= 8;
        mma_16816(c0, c1, c2, c3, hsub2_u32(lop3_and_or(a, 0x000F000Fu, kMagic), zloA),
                  hsub2_u32(lop3_and_or(b, 0x000F000Fu, kMagic), zloB),
                  hsub2_u32(lop3_and_or(a, 0x00F000F0u, kMagic), zhiA),
                  hsub2_u32(lop3_and_or(b, 0x00F000F0u, kMagic), zhiB), xv.z, xv.w);
      }
      accA = fmaf(c.sa[u], c0, accA);
      accB = fmaf(c.sb[u], c2, accB);
    }
  }
}

// Software-pipelined walk over [g_begin, g_end): the caller has already loaded
// the first chunk into `first` (typically before griddepcontrol.wait, since
// weights never depend on the previous kernel); each step loads the next
// chunk before computing the current one.
template <int G, int U>
__device__ __forceinline__ void u4_dot2_pipelined(U4Chunk<G, U>& first, const U4Rows& r,
                                                  const uint4* __restrict__ xs, int g_begin,
                                                  int g_end, int t, float& accA, float& accB) {
  U4Chunk<G, U> next;
  int g0 = g_begin;
  while (g0 < g_end) {
    const int g1 = g0 + U;
    if (g1 < g_end) u4_load_chunk<G, U>(next, r, g1, g_end, t);
    u4_compute_chunk<G, U>(first, xs, g0, g_end, t, accA, accB);
    if (g1 >= g_end) break;
    g0 = g1;
    if (g0 + U < g_end) {
      u4_load_chunk<G, U>(first, r, g0 + U, g_end, t);
    }
    u4_compute_chunk<G, U>(next, xs, g0, g_end, t, accA, accB);
    g0 += U;
  }
}

// Dot products of two weight rows (A, B) with the staged activation over
// quant groups [g_begin, g_end). wA/wB: row starts (K/2 bytes each); sA/sB:
// row scale starts; zeA/zeB: zp element index of (row, group 0). Results are
// added into accA/accB (identical in the four lanes of a lane group).
template <int G, int U>
__device__ __forceinline__ void u4_dot2(const uint8_t* __restrict__ wA,
                                        const uint8_t* __restrict__ wB,
                                        const __half* __restrict__ sA,
                                        const __half* __restrict__ sB,
                                        const uint8_t* __restrict__ zp, int64_t zeA, int64_t zeB,
                                        const uint4* __restrict__ xs, int g_begin, int g_end,
                                        int t, float& accA, float& accB) {
  constexpr int W = G / 32;  // 32-bit words per lane per row per group
  static_assert(W == 2 || W == 4, "G must be 64 or 128");
  for (int g0 = g_begin; g0 < g_end; g0 += U) {
    uint32_t ra[U][W], rb[U][W];
    uint32_t za[U], zb[U];
    float sa[U], sb[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int gi = min(g0 + u, g_end - 1);
      const int off = gi * (G / 2) + t * (G / 8);
      if constexpr (W == 4) {
        const uint4 va = ld_stream_v4(wA + off);
        const uint4 vb = ld_stream_v4(wB + off);
        ra[u][0] = va.x; ra[u][1] = va.y; ra[u][2] = va.z; ra[u][3] = va.w;
        rb[u][0] = vb.x; rb[u][1] = vb.y; rb[u][2] = vb.z; rb[u][3] = vb.w;
      } else {
        const uint2 va = ld_stream_v2(wA + off);
        const uint2 vb = ld_stream_v2(wB + off);
        ra[u][0] = va.x; ra[u][1] = va.y;
        rb[u][0] = vb.x; rb[u][1] = vb.y;
      }
      sa[u] = __half2float(sA[gi]);
      sb[u] = __half2float(sB[gi]);
      za[u] = zp_nibble(zp, zeA + gi);
      zb[u] = zp_nibble(zp, zeB + gi);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (g0 + u < g_end) {
        const int gi = g0 + u;
        const uint32_t zloA = kMagic | za[u] | (za[u] << 16);
        const uint32_t zhiA = kMagic | (za[u] << 4) | (za[u] << 20);
        const uint32_t zloB = kMagic | zb[u] | (zb[u] << 16);
        const uint32_t zhiB = kMagic | (zb[u] << 4) | (zb[u] << 20);
        float c0 = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
#pragma unroll
        for (int i = 0; i < W; ++i) {
          const uint4 xv = xs[gi * (G / 8) + t * W + i];
          uint32_t a = ra[u][i], b = rb[u][i];
          mma_16816(c0, c1, c2, c3,
                    hsub2_u32(lop3_and_or(a, 0x000F000Fu, kMagic), zloA),
                    hsub2_u32(lop3_and_or(b, 0x000F000Fu, kMagic), zloB),
                    hsub2_u32(lop3_and_or(a, 0x00F000F0u, kMagic), zhiA),
                    hsub2_u32(lop3_and_or(b, 0x00F000F0u, kMagic), zhiB), xv.x, xv.y);
          a >>= 8;
          b >>= 8;
          mma_16816(c0, c1, c2, c3,
                    hsub2_u32(lop3_and_or(a, 0x000F000Fu, kMagic), zloA),
                    hsub2_u32(lop3_and_or(b, 0x000F000Fu, kMagic), zloB),
                    hsub2_u32(lop3_and_or(a, 0x00F000F0u, kMagic), zhiA),
                    hsub2_u32(lop3_and_or(b, 0x00F000F0u, kMagic), zhiB), xv.z, xv.w);
        }
        accA = fmaf(sa[u], c0, accA);
        accB = fmaf(sb[u], c2, accB);
      }
    }
  }
}

}  // namespace iq36
