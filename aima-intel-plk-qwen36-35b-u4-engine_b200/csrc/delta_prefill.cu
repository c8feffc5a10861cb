// delta_prefill.cu — the Gated DeltaNet block over T prompt tokens at once.
//
// The per-token decode path (delta_prep_kernel + delta_step_kernel) runs the
// causal conv and the recurrence for one token per launch. Prefill runs the
// same arithmetic over a whole prompt in five launches per layer:
//   1. delta_conv_batch_kernel: causal depthwise conv(4) + SiLU for every
//      (token, channel) — the conv is a 4-tap FIR over the previous three
//      inputs (or the carried state before token 0) — then the per-head L2
//      normalisation of q and k, and the gates g (log decay) and
//      beta = sigmoid(b) per (token, value head).
//   2. delta_conv_state_kernel: carried conv state := the last four inputs.
//   3. delta_chunk_prep_kernel: the chunked (WY) form of the recurrence,
//      parallel over 32-token chunks x value heads: cumulative log decay G,
//      A = beta_r e^(G_r - G_s) k_r.k_s (s < r), the triangular solve
//      (I + A) [W | U] = [beta e^G k | beta v], and the chunk's output and
//      state-update operands e^G q, e^(G_last - G) k, e^(G_r - G_s) q_r.k_s.
//   4. delta_chunk_scan_kernel: the only sequential part, over chunks: per
//      chunk Delta = U - W S, O = (e^G q) S + P Delta, S = e^G_last S + K~^T Delta,
//      as 3xTF32 tensor-core products (fp32-accurate: hi/lo split of every
//      operand), the state held in registers.
//   5. delta_gated_norm_kernel: gated RMSNorm of every (token, value head).
//
// Semantics (same as the decode path): OpenVINO gated delta net
// (iq36_gated_delta_net.cl:36-150) — key head = value head / (nv/nk), q and k
// L2-normalised with rsqrt(sum + 1e-6), q additionally * 1/sqrt(D); per token
// S = exp(g) S; sk = S^T k; delta = (v - sk) beta; S += k delta^T; o = S^T q.
// Unrolling that step over a chunk gives exactly the chunked products above
// (delta_r + sum_{s<r} A_rs delta_s = beta_r v_r - beta_r e^(G_r) S0^T k_r).
// Conv with fp16 rounding points of iq36_linear_conv_swish.cl:25-63; gates of
// gguf_loader.cpp:4875-4912; gated RMSNorm of gguf_loader.cpp:4770-4786.

#include <atomic>

#include "launch.cuh"
#include "common.cuh"

namespace iq36 {

constexpr int kDhd = 128;       // DeltaNet head dim (key and value)
constexpr int kConvTok = 32;    // tokens per CTA of the conv kernel

// ---------------------------------------------------------------------------
// 1. conv + SiLU + q/k normalisation + gates. Grid (ceil(T/32), ceil(segments/8)),
// 8 warps; warp = one 128-channel segment (a q head, a k head or a v head)
// over 32 consecutive tokens, lane = 4 channels; the last three inputs ride
// along in registers, so every input row is read once.
__global__ void __launch_bounds__(256) delta_conv_batch_kernel(
    const __half* qkv, int T, int nk, int nv, const float* conv_state, const float* conv_w,
    const __half* a, const __half* b, int gate_stride, const float* a_log, const float* dtb,
    float* qk_out, __half* v_out, float* lg_out, float* beta_out) {
  pdl_wait();
  const int t0 = blockIdx.x * kConvTok, t1 = min(T, t0 + kConvTok);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (blockIdx.y == 0) {
    for (int i = threadIdx.x; i < (t1 - t0) * nv; i += blockDim.x) {
      const int t = t0 + i / nv, h = i % nv;
      const float xa = __half2float(a[(size_t)t * gate_stride + h]) + dtb[h];
      const float sp = xa > 20.f ? xa : log1pf(expf(xa));
      lg_out[(size_t)t * nv + h] = -expf(a_log[h]) * sp;  // g = log of the decay
      beta_out[(size_t)t * nv + h] = sigmoidf_acc(__half2float(b[(size_t)t * gate_stride + h]));
    }
  }
  const int nseg = 2 * nk + nv;
  const int seg = blockIdx.y * 8 + warp;
  if (seg >= nseg) return;
  const int C = nseg * kDhd;
  const int c0 = seg * kDhd + 4 * lane;
  auto load_row = [&](int tt, float* x) {
    if (tt >= 0) {
      const uint2 raw = *reinterpret_cast<const uint2*>(qkv + (size_t)tt * C + c0);
      const __half2 lo = *reinterpret_cast<const __half2*>(&raw.x);
      const __half2 hi = *reinterpret_cast<const __half2*>(&raw.y);
      x[0] = __low2float(lo);
      x[1] = __high2float(lo);
      x[2] = __low2float(hi);
      x[3] = __high2float(hi);
    } else {
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) x[ch] = conv_state[(size_t)(c0 + ch) * 4 + 4 + tt];
    }
  };
  float4 w[4];
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) w[ch] = reinterpret_cast<const float4*>(conv_w)[c0 + ch];
  // x3 = input t-3, x2 = t-2, x1 = t-1
  float x3[4], x2[4], x1[4];
  load_row(t0 - 3, x3);
  load_row(t0 - 2, x2);
  load_row(t0 - 1, x1);
  const float qscale = rsqrtf((float)kDhd);
  for (int t = t0; t < t1; ++t) {
    float x0[4];
    load_row(t, x0);
    float act[4];
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      float s = w[ch].x * x3[ch];
      s = fmaf(w[ch].y, x2[ch], s);
      s = fmaf(w[ch].z, x1[ch], s);
      s = fmaf(w[ch].w, x0[ch], s);
      const float conv = __half2float(__float2half_rn(s));
      act[ch] = __half2float(__float2half_rn(conv / (1.0f + expf(-conv))));
      x3[ch] = x2[ch];
      x2[ch] = x1[ch];
      x1[ch] = x0[ch];
    }
    if (seg >= 2 * nk) {
      const __half2 lo = __floats2half2_rn(act[0], act[1]);
      const __half2 hi = __floats2half2_rn(act[2], act[3]);
      uint2 raw;
      raw.x = *reinterpret_cast<const uint32_t*>(&lo);
      raw.y = *reinterpret_cast<const uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(v_out + (size_t)t * nv * kDhd + (seg - 2 * nk) * kDhd +
                                4 * lane) = raw;
    } else {
      const float ss = warp_sum(act[0] * act[0] + act[1] * act[1] + act[2] * act[2] +
                                act[3] * act[3]);
      const float r = rsqrtf(ss + 1e-6f);
      float4 y;
      if (seg < nk) {
        y = make_float4(act[0] * r * qscale, act[1] * r * qscale, act[2] * r * qscale,
                        act[3] * r * qscale);
      } else {
        y = make_float4(act[0] * r, act[1] * r, act[2] * r, act[3] * r);
      }
      *reinterpret_cast<float4*>(qk_out + ((size_t)t * 2 * nk + seg) * kDhd + 4 * lane) = y;
    }
  }
  pdl_launch_dependents();
}

// 2. conv state [C, 4] := inputs T-4 .. T-1 (older ones from the old state).
__global__ void __launch_bounds__(256) delta_conv_state_kernel(const __half* qkv, int T, int C,
                                                               float* conv_state) {
  pdl_wait();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c < C) {
    const float4 old = reinterpret_cast<const float4*>(conv_state)[c];
    const float o[4] = {old.x, old.y, old.z, old.w};
    float n[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int tt = T - 4 + j;
      n[j] = tt >= 0 ? __half2float(qkv[(size_t)tt * C + c]) : o[T + j];
    }
    reinterpret_cast<float4*>(conv_state)[c] = make_float4(n[0], n[1], n[2], n[3]);
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// 3./4. the recurrence in chunked form.

// m16n8k8 TF32 tensor-core product with fp32 accumulate; A row-major 16x8
// (a0 (g,t), a1 (g+8,t), a2 (g,t+4), a3 (g+8,t+4)), B 8x8 (b0 (k=t,n=g),
// b1 (k=t+4,n=g)), C (c0,c1 (g,2t..), c2,c3 (g+8,2t..)).
__device__ __forceinline__ void mma_tf32(float (&c)[4], const uint32_t (&a)[4],
                                         const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(hi) : "f"(x));
  const float r = x - __uint_as_float(hi);
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(lo) : "f"(r));
}
constexpr int kCk = 32;  // tokens per chunk
// Per (chunk, value head) operand block (floats): W [32][128], U [32][128],
// Qg = e^G q [32][128], Kt = e^(G_last - G) k key-major [128][32], P [32][32],
// gC = e^G_last.
constexpr int kOffW = 0, kOffU = 4096, kOffQ = 8192, kOffKt = 12288, kOffPm = 16384,
              kOffGc = 17408, kCkBlk = 17412;
constexpr int kPrepSmem = (2 * kCk * 132 + kCk * 128 + kCk * 36 + 4 * kCk) * 4;

__global__ void __launch_bounds__(256) delta_chunk_prep_kernel(const float* __restrict__ qk,
                                                               const __half* __restrict__ v,
                                                               const float* __restrict__ lg,
                                                               const float* __restrict__ beta,
                                                               int T, int nk, int nv,
                                                               float* __restrict__ blocks) {
  extern __shared__ __align__(16) float sm[];
  float* sk = sm;                  // k rows [32][132]
  float* sq = sk + kCk * 132;      // q rows [32][132]
  float* sv = sq + kCk * 132;      // v rows [32][128]
  float* sA = sv + kCk * 128;      // A [32][36]
  float* sB = sA + kCk * 36;       // beta [32]
  float* sE = sB + kCk;            // e^G_r
  float* sL = sE + kCk;            // e^(G_last - G_r)
  float* sG = sL + kCk;            // G_r
  const int c = blockIdx.x, h = blockIdx.y, kh = h / (nv / nk);
  const int t0 = c * kCk, n = min(kCk, T - t0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();
  for (int i = tid; i < kCk * 32; i += blockDim.x) {
    const int r = i >> 5, p = i & 31;
    float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f), qv4 = kv4, vv4 = kv4;
    if (r < n) {
      const size_t row = (size_t)(t0 + r) * 2 * nk;
      kv4 = *reinterpret_cast<const float4*>(qk + (row + nk + kh) * kDhd + 4 * p);
      qv4 = *reinterpret_cast<const float4*>(qk + (row + kh) * kDhd + 4 * p);
      const uint2 raw =
          *reinterpret_cast<const uint2*>(v + (size_t)(t0 + r) * nv * kDhd + h * kDhd + 4 * p);
      const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
      const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
      vv4 = make_float4(lo.x, lo.y, hi.x, hi.y);
    }
    *reinterpret_cast<float4*>(sk + r * 132 + 4 * p) = kv4;
    *reinterpret_cast<float4*>(sq + r * 132 + 4 * p) = qv4;
    *reinterpret_cast<float4*>(sv + r * 128 + 4 * p) = vv4;
  }
  if (warp == 0) {
    float x = lane < n ? lg[(size_t)(t0 + lane) * nv + h] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    const float gl = __shfl_sync(0xffffffffu, x, n - 1);
    sG[lane] = x;
    sE[lane] = lane < n ? expf(x) : 0.f;
    sL[lane] = lane < n ? expf(gl - x) : 0.f;
    sB[lane] = lane < n ? beta[(size_t)(t0 + lane) * nv + h] : 0.f;
  }
  __syncthreads();
  float* blk = blocks + ((size_t)c * nv + h) * kCkBlk;
  // K K^T and Q K^T (32 x 32, K = 128) on tensor cores, 3xTF32 (operands split
  // on the fly); warp w: rows 16(w>>2).., columns 8(w&3)..
  {
    const int mt = warp >> 2, nt = warp & 3, g = lane >> 2, t = lane & 3;
    float ck[4] = {0.f, 0.f, 0.f, 0.f}, cq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int ks = 0; ks < kDhd / 8; ++ks) {
      uint32_t bh[2], bl[2], kh4[4], kl4[4], qh4[4], ql4[4];
      const float* kb = sk + (8 * nt + g) * 132 + 8 * ks + t;  // B[k=d][n=s] = k_s[d]
      split_tf32(kb[0], bh[0], bl[0]);
      split_tf32(kb[4], bh[1], bl[1]);
      const int o0 = (16 * mt + g) * 132 + 8 * ks + t, o1 = o0 + 8 * 132;
      split_tf32(sk[o0], kh4[0], kl4[0]);
      split_tf32(sk[o1], kh4[1], kl4[1]);
      split_tf32(sk[o0 + 4], kh4[2], kl4[2]);
      split_tf32(sk[o1 + 4], kh4[3], kl4[3]);
      split_tf32(sq[o0], qh4[0], ql4[0]);
      split_tf32(sq[o1], qh4[1], ql4[1]);
      split_tf32(sq[o0 + 4], qh4[2], ql4[2]);
      split_tf32(sq[o1 + 4], qh4[3], ql4[3]);
      mma_tf32(ck, kl4, bh);
      mma_tf32(ck, kh4, bl);
      mma_tf32(ck, kh4, bh);
      mma_tf32(cq, ql4, bh);
      mma_tf32(cq, qh4, bl);
      mma_tf32(cq, qh4, bh);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = 16 * mt + g + (e >> 1) * 8, s2 = 8 * nt + 2 * t + (e & 1);
      const bool lower = s2 <= r && r < n;
      const float dec = lower ? expf(sG[r] - sG[s2]) : 0.f;
      sA[r * 36 + s2] = s2 < r && r < n ? sB[r] * dec * ck[e] : 0.f;
      blk[kOffPm + r * kCk + s2] = dec * cq[e];
    }
  }
  __syncthreads();
  // (I + A) X = [beta e^G k | beta v]: thread j owns column j, forward substitution
  {
    const int j = tid;
    float x[kCk];
#pragma unroll
    for (int r = 0; r < kCk; ++r) {
      float acc = j < kDhd ? sB[r] * sE[r] * sk[r * 132 + j] : sB[r] * sv[r * 128 + j - kDhd];
#pragma unroll
      for (int q = 0; q < (r + 3) / 4; ++q) {
        const float4 a4 = *reinterpret_cast<const float4*>(sA + r * 36 + 4 * q);
        if (4 * q + 0 < r) acc = fmaf(-a4.x, x[4 * q + 0], acc);
        if (4 * q + 1 < r) acc = fmaf(-a4.y, x[4 * q + 1], acc);
        if (4 * q + 2 < r) acc = fmaf(-a4.z, x[4 * q + 2], acc);
        if (4 * q + 3 < r) acc = fmaf(-a4.w, x[4 * q + 3], acc);
      }
      x[r] = acc;
    }
    float* dst = blk + (j < kDhd ? kOffW + j : kOffU + j - kDhd);
#pragma unroll
    for (int r = 0; r < kCk; ++r) dst[r * kDhd] = x[r];
  }
  for (int i = tid; i < kCk * kDhd; i += blockDim.x) {
    const int r = i >> 7, d = i & 127;
    blk[kOffQ + i] = sE[r] * sq[r * 132 + d];
    const int dk = i >> 5, rk = i & 31;  // Kt[dk][rk]
    blk[kOffKt + i] = sL[rk] * sk[rk * 132 + dk];
  }
  if (tid == 0) blk[kOffGc] = expf(sG[n - 1]);
  pdl_launch_dependents();
}

struct Tf32Frag4 {
  uint32_t hi[4], lo[4];
};
struct Tf32Frag2 {
  uint32_t hi[2], lo[2];
};
__device__ __forceinline__ Tf32Frag4 frag_a(const float* p, int ld, int g, int t) {
  Tf32Frag4 f;
  split_tf32(p[g * ld + t], f.hi[0], f.lo[0]);
  split_tf32(p[(g + 8) * ld + t], f.hi[1], f.lo[1]);
  split_tf32(p[g * ld + t + 4], f.hi[2], f.lo[2]);
  split_tf32(p[(g + 8) * ld + t + 4], f.hi[3], f.lo[3]);
  return f;
}
__device__ __forceinline__ Tf32Frag2 frag_b(const float* p, int ld, int g, int t) {
  Tf32Frag2 f;
  split_tf32(p[t * ld + g], f.hi[0], f.lo[0]);
  split_tf32(p[(t + 4) * ld + g], f.hi[1], f.lo[1]);
  return f;
}
// c += a b with fp32-level accuracy: a_lo b_hi + a_hi b_lo + a_hi b_hi
__device__ __forceinline__ void mma3(float (&c)[4], const Tf32Frag4& a, const Tf32Frag2& b) {
  mma_tf32(c, a.lo, b.hi);
  mma_tf32(c, a.hi, b.lo);
  mma_tf32(c, a.hi, b.hi);
}

// fragments from operands already split (hi bits and lo bits in two arrays of one layout)
__device__ __forceinline__ Tf32Frag2 frag_b_pre(const float* hi, const float* lo, int ld, int g,
                                                int t) {
  Tf32Frag2 f;
  f.hi[0] = __float_as_uint(hi[t * ld + g]);
  f.hi[1] = __float_as_uint(hi[(t + 4) * ld + g]);
  f.lo[0] = __float_as_uint(lo[t * ld + g]);
  f.lo[1] = __float_as_uint(lo[(t + 4) * ld + g]);
  return f;
}
__device__ __forceinline__ void put_split(float* hi, float* lo, int i, float x) {
  uint32_t h, l;
  split_tf32(x, h, l);
  hi[i] = __uint_as_float(h);
  lo[i] = __uint_as_float(l);
}

constexpr int kScCols = 32;  // value columns per CTA
// one chunk's operands in shared memory (floats), padded for conflict-free fragments
constexpr int kStW = 0, kStQ = kCk * 132, kStU = 2 * kCk * 132, kStPm = kStU + kCk * 36,
              kStKt = kStPm + kCk * 36, kStGc = kStKt + kDhd * 36, kStFloats = kStGc + 4;
constexpr int kPartLd = 40;                             // partial-sum row stride
constexpr int kPartFloats = 8 * 2 * 16 * kPartLd;       // [warp][product][16][40]
constexpr int kScanSmem =
    (2 * kStFloats + 2 * kDhd * 40 + 2 * kCk * 40 + kCk * 40 + kPartFloats) * 4;

// Grid (128/32 column blocks, nv), 8 warps. Warp w keeps state rows
// 16w..16w+15 (key) x the CTA's 32 value columns as mma accumulators. Per chunk:
//  b. Delta = U - W S and Oa = Qg S: warp w multiplies rows 16(w&1).. over the
//     key quarter 32(w>>1).. for all 32 columns (its W / Qg fragments split
//     once), then the four key-quarter partials are summed in shared memory;
//  c. O = Oa + P Delta on a 16 x 8 tile per warp;
//  d. S = gC S + Kt^T Delta on the warp's own state rows.
// S and Delta are stored split (tf32 hi / lo) by the threads that produce them.
__global__ void __launch_bounds__(256, 1)
    delta_chunk_scan_kernel(const float* __restrict__ blocks, float* __restrict__ state,
                            float* __restrict__ o_out, int T, int nv) {
  extern __shared__ __align__(16) float sm[];
  float* sSh = sm + 2 * kStFloats;  // state hi [128][40] (B operand)
  float* sSl = sSh + kDhd * 40;     // state lo
  float* sDh = sSl + kDhd * 40;     // Delta hi [32][40] (B operand)
  float* sDl = sDh + kCk * 40;      // Delta lo
  float* sOa = sDl + kCk * 40;      // Oa [32][40]
  float* sPart = sOa + kCk * 40;    // step-b partials
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int h = blockIdx.y, j0 = blockIdx.x * kScCols;
  const int nchunks = (T + kCk - 1) / kCk;
  auto stage = [&](int buf) { return sm + buf * kStFloats; };
  auto load_stage = [&](int c, int buf) {
    const float* blk = blocks + ((size_t)c * nv + h) * kCkBlk;
    const uint32_t st = smem_u32(stage(buf));
    for (int i = threadIdx.x; i < kCk * 32; i += blockDim.x) {
      const int r = i >> 5, p = i & 31;
      cp_async_16(st + (kStW + r * 132 + 4 * p) * 4, blk + kOffW + r * kDhd + 4 * p, 16);
      cp_async_16(st + (kStQ + r * 132 + 4 * p) * 4, blk + kOffQ + r * kDhd + 4 * p, 16);
    }
    for (int i = threadIdx.x; i < kCk * 8; i += blockDim.x) {
      const int r = i >> 3, p = i & 7;
      cp_async_16(st + (kStU + r * 36 + 4 * p) * 4, blk + kOffU + r * kDhd + j0 + 4 * p, 16);
      cp_async_16(st + (kStPm + r * 36 + 4 * p) * 4, blk + kOffPm + r * kCk + 4 * p, 16);
    }
    for (int i = threadIdx.x; i < kDhd * 8; i += blockDim.x) {
      const int d = i >> 3, p = i & 7;
      cp_async_16(st + (kStKt + d * 36 + 4 * p) * 4, blk + kOffKt + d * kCk + 4 * p, 16);
    }
    if (threadIdx.x == 0) cp_async_16(st + kStGc * 4, blk + kOffGc, 16);
  };
  pdl_wait();
  // state slice: rows 16w + g (+8), columns 8nt + 2t (+1)
  float accS[4][4];
  const size_t sbase = (size_t)h * kDhd * kDhd;
  const int ra = 16 * warp + g, rb = ra + 8;
  auto put_state = [&]() {
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int cc = 8 * nt + 2 * t;
      put_split(sSh, sSl, ra * 40 + cc, accS[nt][0]);
      put_split(sSh, sSl, ra * 40 + cc + 1, accS[nt][1]);
      put_split(sSh, sSl, rb * 40 + cc, accS[nt][2]);
      put_split(sSh, sSl, rb * 40 + cc + 1, accS[nt][3]);
    }
  };
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int cc = j0 + 8 * nt + 2 * t;
    accS[nt][0] = state[sbase + (size_t)ra * kDhd + cc];
    accS[nt][1] = state[sbase + (size_t)ra * kDhd + cc + 1];
    accS[nt][2] = state[sbase + (size_t)rb * kDhd + cc];
    accS[nt][3] = state[sbase + (size_t)rb * kDhd + cc + 1];
  }
  put_state();
  load_stage(0, 0);
  cp_async_commit();
  const int mt = warp & 1, kq = warp >> 1;  // step b: row tile, key quarter
  const int mw = warp >> 2, nw = warp & 3;  // step c: O tile
  for (int c = 0; c < nchunks; ++c) {
    const int buf = c & 1;
    if (c + 1 < nchunks) {
      load_stage(c + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float* st = stage(buf);
    // b: partial W S and Qg S over this warp's key quarter
    {
      float pd[4][4] = {}, po[4][4] = {};
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int k0 = 32 * kq + 8 * ks;
        const Tf32Frag4 aW = frag_a(st + kStW + 16 * mt * 132 + k0, 132, g, t);
        const Tf32Frag4 aQ = frag_a(st + kStQ + 16 * mt * 132 + k0, 132, g, t);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const Tf32Frag2 bS = frag_b_pre(sSh + k0 * 40 + 8 * nt, sSl + k0 * 40 + 8 * nt, 40, g, t);
          mma3(pd[nt], aW, bS);
          mma3(po[nt], aQ, bS);
        }
      }
      float* pw = sPart + warp * 2 * 16 * kPartLd;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int cc = 8 * nt + 2 * t;
        *reinterpret_cast<float2*>(pw + g * kPartLd + cc) = make_float2(pd[nt][0], pd[nt][1]);
        *reinterpret_cast<float2*>(pw + (g + 8) * kPartLd + cc) = make_float2(pd[nt][2], pd[nt][3]);
        *reinterpret_cast<float2*>(pw + 16 * kPartLd + g * kPartLd + cc) =
            make_float2(po[nt][0], po[nt][1]);
        *reinterpret_cast<float2*>(pw + 16 * kPartLd + (g + 8) * kPartLd + cc) =
            make_float2(po[nt][2], po[nt][3]);
      }
    }
    __syncthreads();
    // sum the key quarters: thread -> row r (0..31), columns 4c4..4c4+3
    {
      const int r = threadIdx.x >> 3, c4 = threadIdx.x & 7;
      const int m = r >> 4, rr = r & 15;
      float4 d = make_float4(0.f, 0.f, 0.f, 0.f), o = d;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float* pw = sPart + (2 * q + m) * 2 * 16 * kPartLd;
        const float4 a = *reinterpret_cast<const float4*>(pw + rr * kPartLd + 4 * c4);
        const float4 b = *reinterpret_cast<const float4*>(pw + 16 * kPartLd + rr * kPartLd + 4 * c4);
        d.x += a.x; d.y += a.y; d.z += a.z; d.w += a.w;
        o.x += b.x; o.y += b.y; o.z += b.z; o.w += b.w;
      }
      const float4 u = *reinterpret_cast<const float4*>(st + kStU + r * 36 + 4 * c4);
      const float dv[4] = {u.x - d.x, u.y - d.y, u.z - d.z, u.w - d.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) put_split(sDh, sDl, r * 40 + 4 * c4 + e, dv[e]);
      *reinterpret_cast<float4*>(sOa + r * 40 + 4 * c4) = o;
    }
    __syncthreads();
    // c: O = Oa + P Delta
    const int r0 = 16 * mw + g, r1 = r0 + 8, cc = 8 * nw + 2 * t;
    float o[4] = {sOa[r0 * 40 + cc], sOa[r0 * 40 + cc + 1], sOa[r1 * 40 + cc],
                  sOa[r1 * 40 + cc + 1]};
#pragma unroll
    for (int ks = 0; ks < kCk / 8; ++ks) {
      const Tf32Frag4 aP = frag_a(st + kStPm + 16 * mw * 36 + 8 * ks, 36, g, t);
      const Tf32Frag2 bD = frag_b_pre(sDh + 8 * ks * 40 + 8 * nw, sDl + 8 * ks * 40 + 8 * nw, 40, g, t);
      mma3(o, aP, bD);
    }
    const int t0 = c * kCk, n = min(kCk, T - t0);
    if (r0 < n)
      *reinterpret_cast<float2*>(o_out + ((size_t)(t0 + r0) * nv + h) * kDhd + j0 + cc) =
          make_float2(o[0], o[1]);
    if (r1 < n)
      *reinterpret_cast<float2*>(o_out + ((size_t)(t0 + r1) * nv + h) * kDhd + j0 + cc) =
          make_float2(o[2], o[3]);
    // d: S = gC S + Kt^T Delta on this warp's key rows
    const float gc = st[kStGc];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) accS[nt][e] *= gc;
#pragma unroll
    for (int ks = 0; ks < kCk / 8; ++ks) {
      const Tf32Frag4 aK = frag_a(st + kStKt + 16 * warp * 36 + 8 * ks, 36, g, t);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const Tf32Frag2 bD =
            frag_b_pre(sDh + 8 * ks * 40 + 8 * nt, sDl + 8 * ks * 40 + 8 * nt, 40, g, t);
        mma3(accS[nt], aK, bD);
      }
    }
    __syncthreads();  // every warp is done reading S (step b) and Delta before they change
    put_state();
    // the next iteration's first barrier publishes S; this stage is refilled after it
  }
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int cc2 = j0 + 8 * nt + 2 * t;
    state[sbase + (size_t)ra * kDhd + cc2] = accS[nt][0];
    state[sbase + (size_t)ra * kDhd + cc2 + 1] = accS[nt][1];
    state[sbase + (size_t)rb * kDhd + cc2] = accS[nt][2];
    state[sbase + (size_t)rb * kDhd + cc2 + 1] = accS[nt][3];
  }
  pdl_launch_dependents();
}

// 4. gated RMSNorm: one warp per (token, value head), lane = 4 columns.
__global__ void __launch_bounds__(256) delta_gated_norm_kernel(const float* o, const __half* z,
                                                               const float* norm_w, float eps,
                                                               int rows, __half* out) {
  pdl_wait();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row < rows) {
    const float4 v = *reinterpret_cast<const float4*>(o + (size_t)row * kDhd + 4 * lane);
    const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
    const float nsc = rsqrtf(ss / (float)kDhd + eps);
    const uint2 zr = *reinterpret_cast<const uint2*>(z + (size_t)row * kDhd + 4 * lane);
    const __half2 zlo = *reinterpret_cast<const __half2*>(&zr.x);
    const __half2 zhi = *reinterpret_cast<const __half2*>(&zr.y);
    const float zv[4] = {__low2float(zlo), __high2float(zlo), __low2float(zhi), __high2float(zhi)};
    const float ov[4] = {v.x, v.y, v.z, v.w};
    float y[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      y[i] = ov[i] * nsc * norm_w[4 * lane + i] * (zv[i] * sigmoidf_acc(zv[i]));
    const __half2 lo = __floats2half2_rn(y[0], y[1]);
    const __half2 hi = __floats2half2_rn(y[2], y[3]);
    uint2 raw;
    raw.x = *reinterpret_cast<const uint32_t*>(&lo);
    raw.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(out + (size_t)row * kDhd + 4 * lane) = raw;
  }
  pdl_launch_dependents();
}

// workspace: qk fp32 [T, 2nk, D] | v fp16 [T, nv*D] | g, beta fp32 [T, nv] | o fp32 [T, nv, D]
// | chunk operand blocks [ceil(T/32), nv, kCkBlk] fp32
struct DeltaWs {
  size_t qk, v, decay, beta, o, blocks, total;
};
static DeltaWs delta_ws(int T, int nk, int nv) {
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  DeltaWs w;
  w.qk = 0;
  w.v = up(w.qk + (size_t)T * 2 * nk * kDhd * 4);
  w.decay = up(w.v + (size_t)T * nv * kDhd * 2);
  w.beta = up(w.decay + (size_t)T * nv * 4);
  w.o = up(w.beta + (size_t)T * nv * 4);
  w.blocks = up(w.o + (size_t)T * nv * kDhd * 4);
  w.total = up(w.blocks + (size_t)((T + kCk - 1) / kCk) * nv * kCkBlk * 4);
  return w;
}

}  // namespace iq36

using namespace iq36;

extern "C" size_t iq36_delta_prefill_workspace_bytes(int32_t tokens, int32_t n_k_heads,
                                                     int32_t n_v_heads) {
  if (tokens < 1 || n_k_heads < 1 || n_v_heads < 1) return 0;
  return delta_ws(tokens, n_k_heads, n_v_heads).total;
}

extern "C" int iq36_delta_prefill(const void* qkv_f16, int32_t tokens, int32_t n_k_heads,
                                  int32_t n_v_heads, int32_t head_dim, float* conv_state,
                                  const float* conv_w, const void* a_f16, const void* b_f16,
                                  int32_t gate_stride, const float* a_log, const float* dt_bias,
                                  float* state, const void* z_f16, const float* norm_w,
                                  float eps, void* out_f16, void* workspace,
                                  size_t workspace_bytes, iq36_stream_t stream) {
  if (!qkv_f16 || !conv_state || !conv_w || !a_f16 || !b_f16 || !a_log || !dt_bias || !state ||
      !z_f16 || !norm_w || !out_f16 || !workspace)
    return IQ36_ERR_ARG;
  const int T = tokens, nk = n_k_heads, nv = n_v_heads;
  if (head_dim != kDhd || T < 1 || nk < 1 || nv < 1 || nv % nk || nv > 256 || gate_stride < nv)
    return IQ36_ERR_SHAPE;
  const DeltaWs w = delta_ws(T, nk, nv);
  if (workspace_bytes < w.total) return IQ36_ERR_WORKSPACE;
  if (!aligned(qkv_f16, 16) || !aligned(conv_state, 16) || !aligned(conv_w, 16) ||
      !aligned(state, 16) || !aligned(z_f16, 16) || !aligned(out_f16, 16) ||
      !aligned(workspace, 256))
    return IQ36_ERR_ALIGN;
  static std::atomic<bool> attr_set[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return IQ36_ERR_CUDA;
  if (!attr_set[dev].load()) {
    if (cudaFuncSetAttribute(delta_chunk_scan_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kScanSmem) !=
            cudaSuccess ||
        cudaFuncSetAttribute(delta_chunk_prep_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kPrepSmem) !=
            cudaSuccess)
      return IQ36_ERR_CUDA;
    attr_set[dev].store(true);
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* qk = reinterpret_cast<float*>(ws + w.qk);
  __half* v = reinterpret_cast<__half*>(ws + w.v);
  float* dec = reinterpret_cast<float*>(ws + w.decay);
  float* bet = reinterpret_cast<float*>(ws + w.beta);
  float* o = reinterpret_cast<float*>(ws + w.o);
  float* blocks = reinterpret_cast<float*>(ws + w.blocks);
  const cudaStream_t s = as_stream(stream);
  const int nseg = 2 * nk + nv, C = nseg * kDhd;
  cudaError_t e = launch(delta_conv_batch_kernel, dim3(ceil_div(T, kConvTok), ceil_div(nseg, 8)),
                         dim3(256), 0, s,
                         reinterpret_cast<const __half*>(qkv_f16), T, nk, nv,
                         (const float*)conv_state, conv_w, reinterpret_cast<const __half*>(a_f16),
                         reinterpret_cast<const __half*>(b_f16), gate_stride, a_log, dt_bias, qk,
                         v, dec, bet);
  if (e == cudaSuccess)
    e = launch(delta_conv_state_kernel, dim3(ceil_div(C, 256)), dim3(256), 0, s,
               reinterpret_cast<const __half*>(qkv_f16), T, C, conv_state);
  if (e == cudaSuccess)
    e = launch(delta_chunk_prep_kernel, dim3(ceil_div(T, kCk), nv), dim3(256), (size_t)kPrepSmem,
               s, (const float*)qk, (const __half*)v, (const float*)dec, (const float*)bet, T, nk,
               nv, blocks);
  if (e == cudaSuccess)
    e = launch(delta_chunk_scan_kernel, dim3(kDhd / kScCols, nv), dim3(256), (size_t)kScanSmem,
               s, (const float*)blocks, state, o, T, nv);
  if (e == cudaSuccess)
    e = launch(delta_gated_norm_kernel, dim3(ceil_div(T * nv, 8)), dim3(256), 0, s,
               (const float*)o, reinterpret_cast<const __half*>(z_f16), norm_w, eps, T * nv,
               reinterpret_cast<__half*>(out_f16));
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}
