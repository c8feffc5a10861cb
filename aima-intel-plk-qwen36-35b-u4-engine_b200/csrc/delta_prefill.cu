// delta_prefill.cu — the Gated DeltaNet block over T prompt tokens at once.
//
// The per-token decode path (delta_prep_kernel + delta_step_kernel) runs the
// causal conv and the recurrence for one token per launch. Prefill runs the
// same arithmetic over a whole prompt in five launches per layer (six when the
// chunk scan is split):
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
//      operand), the state held in TMEM. From 16 chunks on, the prompt is cut
//      in two segments scanned at the same time, and delta_scan_join_kernel
//      applies the state at the cut to the second one.
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

#include <algorithm>
#include <atomic>

#include "launch.cuh"
#include "common.cuh"
#include "tc_sm100.cuh"

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
// Per (chunk, value head) operand block (floats), laid out as the scan's
// shared-memory images so that one bulk copy places each:
//   B1 [4 slabs][64 rows][32]: rows 0..31 W_t, rows 32..63 Qg_t = e^G q_t,
//      slab j = keys 32j..32j+31 (SWIZZLE_128B K-major, 8 KB per slab)
//   Kt [128 rows (key)][32 (t)]: e^(G_last - G_t) k_t, SWIZZLE_128B
//   P  [32 rows (t)][32 (s)]: e^(G_t - G_s) q_t.k_s (s <= t), SWIZZLE_128B
//   U  [32][128] plain
// and gC = e^G_last per (chunk, head) in a separate array.
constexpr int kBlkB1 = 0, kBlkKt = 8192, kBlkP = 12288, kBlkU = 13312, kCkBlk = 17408;
constexpr int kPrepSmem = (2 * kCk * 132 + kCk * 128 + kCk * 36 + 4 * kCk) * 4;

// float index of (row, col) in a SWIZZLE_128B K-major tile of 32-float rows:
// the 16-byte chunk col/4 of row `row` sits at chunk position (col/4) ^ (row % 8)
__host__ __device__ __forceinline__ int sw128_f(int row, int col) {
  return row * 32 + ((((col >> 2) ^ (row & 7))) << 2) + (col & 3);
}
__host__ __device__ __forceinline__ int blk_b1(int r, int k) {
  return kBlkB1 + (k >> 5) * 2048 + sw128_f(r, k & 31);
}

__global__ void __launch_bounds__(256) delta_chunk_prep_kernel(const float* __restrict__ qk,
                                                               const __half* __restrict__ v,
                                                               const float* __restrict__ lg,
                                                               const float* __restrict__ beta,
                                                               int T, int nk, int nv,
                                                               float* __restrict__ blocks,
                                                               float* __restrict__ gcs) {
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
  // Every global load of this thread is issued before any shared-memory
  // store (one DRAM round trip for the phase instead of one per row group).
  float lgv = 0.f, btv = 0.f;
  if (warp == 0 && lane < n) {
    lgv = lg[(size_t)(t0 + lane) * nv + h];
    btv = beta[(size_t)(t0 + lane) * nv + h];
  }
  constexpr int kLd = kCk * 32 / 256;  // float4 columns per thread (blockDim 256)
  float4 kv4[kLd], qv4[kLd];
  uint2 vraw[kLd];
#pragma unroll
  for (int u = 0; u < kLd; ++u) {
    const int i = tid + 256 * u, r = i >> 5, p = i & 31;
    kv4[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    qv4[u] = kv4[u];
    vraw[u] = make_uint2(0u, 0u);
    if (r < n) {
      const size_t row = (size_t)(t0 + r) * 2 * nk;
      kv4[u] = *reinterpret_cast<const float4*>(qk + (row + nk + kh) * kDhd + 4 * p);
      qv4[u] = *reinterpret_cast<const float4*>(qk + (row + kh) * kDhd + 4 * p);
      vraw[u] =
          *reinterpret_cast<const uint2*>(v + (size_t)(t0 + r) * nv * kDhd + h * kDhd + 4 * p);
    }
  }
#pragma unroll
  for (int u = 0; u < kLd; ++u) {
    const int i = tid + 256 * u, r = i >> 5, p = i & 31;
    const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&vraw[u].x));
    const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&vraw[u].y));
    *reinterpret_cast<float4*>(sk + r * 132 + 4 * p) = kv4[u];
    *reinterpret_cast<float4*>(sq + r * 132 + 4 * p) = qv4[u];
    *reinterpret_cast<float4*>(sv + r * 128 + 4 * p) = make_float4(lo.x, lo.y, hi.x, hi.y);
  }
  if (warp == 0) {
    float x = lgv;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    const float gl = __shfl_sync(0xffffffffu, x, n - 1);
    sG[lane] = x;
    sE[lane] = lane < n ? expf(x) : 0.f;
    sL[lane] = lane < n ? expf(gl - x) : 0.f;
    sB[lane] = btv;
  }
  __syncthreads();
  float* blk = blocks + ((size_t)c * nv + h) * kCkBlk;
  // Warps 0-3: K K^T and Q K^T (32 x 32, K = 128) on tensor cores, 3xTF32
  // (operands split on the fly); warp w: product w >> 1 (K, then Q rows as
  // A), rows 16 (w & 1).. against all four 8-column tiles, so each A fragment
  // is split once per k-step. Warps 4-7 meanwhile write the e^G q and
  // e^(G_last - G) k operand images.
  if (warp < 4) {
    const int pr = warp >> 1, mt = warp & 1, g = lane >> 2, t = lane & 3;
    const float* sa = pr ? sq : sk;
    float cc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e2 = 0; e2 < 4; ++e2) cc[nt][e2] = 0.f;
#pragma unroll 2
    for (int ks = 0; ks < kDhd / 8; ++ks) {
      uint32_t ah[4], al[4];
      const int o0 = (16 * mt + g) * 132 + 8 * ks + t, o1 = o0 + 8 * 132;
      split_tf32(sa[o0], ah[0], al[0]);
      split_tf32(sa[o1], ah[1], al[1]);
      split_tf32(sa[o0 + 4], ah[2], al[2]);
      split_tf32(sa[o1 + 4], ah[3], al[3]);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        uint32_t bh[2], bl[2];
        const float* kb = sk + (8 * nt + g) * 132 + 8 * ks + t;  // B[k=d][n=s] = k_s[d]
        split_tf32(kb[0], bh[0], bl[0]);
        split_tf32(kb[4], bh[1], bl[1]);
        mma_tf32(cc[nt], al, bh);
        mma_tf32(cc[nt], ah, bl);
        mma_tf32(cc[nt], ah, bh);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e2 = 0; e2 < 4; ++e2) {
        const int r = 16 * mt + g + (e2 >> 1) * 8, s2 = 8 * nt + 2 * t + (e2 & 1);
        const bool lower = s2 <= r && r < n;
        const float dec = lower ? expf(sG[r] - sG[s2]) : 0.f;
        if (pr == 0) sA[r * 36 + s2] = s2 < r && r < n ? sB[r] * dec * cc[nt][e2] : 0.f;
        else blk[kBlkP + sw128_f(r, s2)] = dec * cc[nt][e2];
      }
  } else {
    // four consecutive columns of a row are one 16-byte chunk of the swizzled image
    for (int i = tid - 128; i < kCk * kDhd / 4; i += 128) {
      const int r = i >> 5, d = 4 * (i & 31);
      const float e = sE[r];
      const float4 x = *reinterpret_cast<const float4*>(sq + r * 132 + d);
      *reinterpret_cast<float4*>(blk + blk_b1(kCk + r, d)) =
          make_float4(e * x.x, e * x.y, e * x.z, e * x.w);
      const int dk = i >> 3, rk = 4 * (i & 7);  // Kt[dk][rk .. rk + 3]
      const float4 l = *reinterpret_cast<const float4*>(sL + rk);
      *reinterpret_cast<float4*>(blk + kBlkKt + sw128_f(dk, rk)) =
          make_float4(l.x * sk[rk * 132 + dk], l.y * sk[(rk + 1) * 132 + dk],
                      l.z * sk[(rk + 2) * 132 + dk], l.w * sk[(rk + 3) * 132 + dk]);
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
    if (j < kDhd) {
#pragma unroll
      for (int r = 0; r < kCk; ++r) blk[blk_b1(r, j)] = x[r];
    } else {
#pragma unroll
      for (int r = 0; r < kCk; ++r) blk[kBlkU + r * kDhd + j - kDhd] = x[r];
    }
  }
  if (tid == 0) gcs[(size_t)c * nv + h] = expf(sG[n - 1]);
  pdl_launch_dependents();
}

// 4. the chunk scan on tcgen05 tensor cores: one CTA per value head.
//
// The state is kept transposed, S^T [128 value rows x 128 keys], as an fp32
// TMEM accumulator (lanes = value rows), so every product has M = 128:
//   (1) X = S^T [W | Qg]^T          M 128, N 64, K 128, A = S^T from TMEM
//   (2) Delta^T = U^T - X[:, 0:32]  epilogue warps, into shared memory
//   (4) S^T = gC S^T + Delta^T Kt^T M 128, N 128, K 32
//   (3) X[:, 32:64] += Delta^T P^T  M 128, N 32,  K 32  -> O^T
// Every product is 3xTF32: the tensor cores truncate fp32 operands to tf32, so
// an fp32 value x is its own hi operand and lo = rna(x - trunc(x)) the second
// (a_hi b_hi + a_hi b_lo + a_lo b_hi; the dropped a_lo b_lo is below 2^-20
// relative). After each update the epilogue writes the A copies of the new
// state (x and its lo part) and the gC-scaled accumulator, key quarter by key
// quarter, and (1) of the next chunk starts on each quarter as it is released;
// the splitters write the lo parts of the B operands one chunk ahead and copy
// each chunk's output rows out of TMEM once its (3) has completed.
//
// Warps: 0 bulk-copy loader, 1 TMEM owner + MMA issuer, 2-5 splitters, 6-13
// epilogue in two groups of four (warp w reads TMEM lanes 32 (w % 4) ..; group
// g takes tokens 16 g .. 16 g + 15 of Delta and keys 32 q + 16 g .. + 15 of each
// key quarter q). TMEM columns: 0 S^T accumulator, 128 the A copy of S^T, 256
// its lo part, 384 and 448 X of even and odd chunks.
//
// Segments. Per chunk the update is affine in the incoming state:
// S^T' = S^T (gC I - W^T Kt^T) + U^T Kt^T and O^T = S^T (Qg^T - W^T P^T) + U^T P^T.
// So a long prompt is cut at chunk m into two segments scanned at the same time
// (grid.y): segment 0 from the real state; segment 1 twice, from a zero state
// (outputs O_R, final state R) and as the transition scan (start I, U = 0:
// outputs O_M, final state M). With Z the state at chunk m, the real outputs
// of segment 1 are O_R + Z O_M and its final state Z M + R
// (delta_scan_join_kernel), which halves the sequential chain.
struct ScanSeg {
  const float* s_in;  // incoming state per head [128 keys][128 values] (start 0)
  float* s_out;       // final state, same layout
  float* o;           // output (t, h, v) at (t - t_off) o_ts + h o_hs + v
  int c0, c1;         // chunks [c0, c1)
  int t_off, o_ts, o_hs;
  int start;          // 0: s_in, 1: zero state, 2: identity state and U = 0
};
struct ScanSegs {
  ScanSeg s[3];
};
constexpr int kScSplitMin = 16;  // chunks: shorter prompts run one segment
__host__ __device__ constexpr int scan_split(int T) {
  return (T + kCk - 1) / kCk >= kScSplitMin ? ((T + kCk - 1) / kCk + 1) / 2 : 0;
}
constexpr int kScThreads = 448;
constexpr int kScEpiWarps = 8;
constexpr uint32_t kScB1Raw = 0, kScB1Lo = 65536, kScKtRaw = 131072, kScKtLo = 147456,
                   kScPRaw = 163840, kScPLo = 167936, kScDHi = 172032, kScDLo = 188416,
                   kScStg = 204800, kScBar = 225280;
constexpr int kScanSmem = (int)kScBar + 256 + 1024;
constexpr uint32_t kTmAcc = 0, kTmHi = 128, kTmLo = 256, kTmX = 384;  // X: 2 x 64 columns
// instruction descriptors: D fp32, A and B tf32, both K-major, M 128
__host__ __device__ constexpr uint32_t tf32_idesc(int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ int g_delta_wait_timeouts;

// second tf32 operand of x: the part below tf32 precision, itself rounded to tf32
__device__ __forceinline__ uint32_t tf32_lo(float x) {
  const float hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x - hi));
  return r;
}
// D (TMEM) (+)= A (TMEM) * B (shared-memory descriptor)
__device__ __forceinline__ void umma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z));
}
// D (TMEM) (+)= A (shared-memory descriptor) * B (shared-memory descriptor)
__device__ __forceinline__ void umma_tf32_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z));
}
// lo parts of `n4` float4s into a buffer of the same layout (128 threads)
__device__ __forceinline__ void split_lo(const float* src, float* lo, int n4, int t) {
  for (int i = t; i < n4; i += 128) {
    const float4 v = reinterpret_cast<const float4*>(src)[i];
    reinterpret_cast<uint4*>(lo)[i] = make_uint4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
  }
}
// raw copy and lo parts
__device__ __forceinline__ void split_copy(const float* src, float* raw, float* lo, int n4, int t) {
  for (int i = t; i < n4; i += 128) {
    const float4 v = reinterpret_cast<const float4*>(src)[i];
    reinterpret_cast<float4*>(raw)[i] = v;
    reinterpret_cast<uint4*>(lo)[i] = make_uint4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
  }
}

__global__ void __launch_bounds__(kScThreads, 1)
    delta_chunk_scan_kernel(const float* __restrict__ blocks, const float* __restrict__ gcs,
                            const ScanSegs segs, int T, int nv) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_raw = smem_u32(smem_raw);
  const uint32_t base = (base_raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - base_raw);
  const uint32_t bar = base + kScBar;
  const uint32_t b1_full = bar, b1_ready = bar + 16, b1_empty = bar + 32;  // [2] each
  const uint32_t stg_full = bar + 48, stg_empty = bar + 56, kp_ready = bar + 64,
                 kp_empty = bar + 72, x_done = bar + 88, d_ready = bar + 96, u_done = bar + 104,
                 done = bar + 112;
  const uint32_t a_ready = bar + 128;  // [4]: key quarters of the state copies
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kScBar + 192);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  const ScanSeg sg = blockIdx.y == 0 ? segs.s[0] : (blockIdx.y == 1 ? segs.s[1] : segs.s[2]);
  const int c0 = sg.c0;
  const int nchunks = sg.c1 - sg.c0;  // local chunk c is chunk c0 + c
  if (threadIdx.x == 0) {
    // commits and the loader count 1; thread groups arrive once per warp
    for (int b = 0; b < 2; ++b) {
      mbar_init(b1_full + 8 * b, 1);
      mbar_init(b1_ready + 8 * b, 4);
      mbar_init(b1_empty + 8 * b, 1);
    }
    mbar_init(stg_full, 1);
    mbar_init(stg_empty, 4);
    mbar_init(kp_ready, 4);
    mbar_init(kp_empty, 1);
    for (int q = 0; q < 4; ++q) mbar_init(a_ready + 8 * q, kScEpiWarps);
    mbar_init(x_done, 1);
    mbar_init(d_ready, kScEpiWarps);
    mbar_init(u_done, 1);
    mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // operand blocks, gC values and the state come from earlier launches
  bool ok = true;

  if (warp == 0) {
    // ---- loader: B1 images (double-buffered) and the raw Kt / P staging ----
    if (lane == 0) {
      for (int c = 0; c < nchunks && ok; ++c) {
        const float* blk = blocks + ((size_t)(c0 + c) * nv + h) * kCkBlk;
        const int b = c & 1;
        ok = mbar_wait(b1_empty + 8 * b, ((c >> 1) & 1) ^ 1u);
        if (!ok) break;
        mbar_arrive_tx(b1_full + 8 * b, 32768u);
        bulk_load(base + kScB1Raw + b * 32768u, blk + kBlkB1, 32768u, b1_full + 8 * b);
        ok = mbar_wait(stg_empty, (c & 1) ^ 1u);
        if (!ok) break;
        mbar_arrive_tx(stg_full, 20480u);
        bulk_load(base + kScStg, blk + kBlkKt, 20480u, stg_full);  // Kt then P (contiguous)
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      const uint32_t acc = tmem + kTmAcc, ahi = tmem + kTmHi, alo = tmem + kTmLo;
      // descriptors differ only in the start-address field (16-byte units)
      const uint64_t ddh = sw128_desc(base + kScDHi), ddl = sw128_desc(base + kScDLo);
      const uint64_t dkh = sw128_desc(base + kScKtRaw), dkl = sw128_desc(base + kScKtLo);
      const uint64_t dph = sw128_desc(base + kScPRaw), dpl = sw128_desc(base + kScPLo);
      for (int c = 0; c < nchunks && ok; ++c) {
        const int b = c & 1;
        const uint32_t xd = tmem + kTmX + 64u * (uint32_t)b;
        ok = mbar_wait(b1_ready + 8 * b, (c >> 1) & 1);
        if (!ok) break;
        // (1) X = S^T [W | Qg]^T, one key quarter (32 keys = one B1 slab) at a
        // time as the epilogue releases the state copies
        const uint64_t dbh = sw128_desc(base + kScB1Raw + b * 32768u);
        const uint64_t dbl = sw128_desc(base + kScB1Lo + b * 32768u);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          ok = mbar_wait(a_ready + 8 * q, c & 1);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int j = 4 * q + jj;
            const uint64_t off = (uint64_t)(q * 8192 + jj * 32) >> 4;
            umma_tf32_ts(xd, ahi + 8 * j, dbh + off, tf32_idesc(64), j > 0 ? 1u : 0u);
            umma_tf32_ts(xd, ahi + 8 * j, dbl + off, tf32_idesc(64), 1u);
            umma_tf32_ts(xd, alo + 8 * j, dbh + off, tf32_idesc(64), 1u);
          }
        }
        if (!ok) break;
        umma_commit(x_done);
        umma_commit(b1_empty + 8 * b);
        ok = mbar_wait(d_ready, c & 1) && mbar_wait(kp_ready, c & 1);
        if (!ok) break;
        tc_fence_after();
        // (4) S^T = gC S^T + Delta^T Kt^T first (the next chunk waits on it),
        // then (3) O^T = Oa^T + Delta^T P^T
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint64_t o = (uint64_t)(32 * j) >> 4;
          umma_tf32_ss(acc, ddh + o, dkh + o, tf32_idesc(128), 1u);
          umma_tf32_ss(acc, ddh + o, dkl + o, tf32_idesc(128), 1u);
          umma_tf32_ss(acc, ddl + o, dkh + o, tf32_idesc(128), 1u);
        }
        umma_commit(u_done);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint64_t o = (uint64_t)(32 * j) >> 4;
          umma_tf32_ss(xd + 32, ddh + o, dph + o, tf32_idesc(32), 1u);
          umma_tf32_ss(xd + 32, ddh + o, dpl + o, tf32_idesc(32), 1u);
          umma_tf32_ss(xd + 32, ddl + o, dph + o, tf32_idesc(32), 1u);
        }
        umma_commit(kp_empty);
      }
      // every MMA issued above has completed before the teardown
      umma_commit(done);
      if (!mbar_wait(done, 0)) ok = false;
    }
  } else if (warp < 6) {
    // ---- splitters: lo parts of every B operand, one chunk ahead; then the
    // previous chunk's output rows (warp w reads TMEM lanes 32 (w % 4)..,
    // all 32 tokens) ----
    const int t = threadIdx.x - 64;
    const int v = (warp & 3) * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const float* stg = reinterpret_cast<const float*>(smem + kScStg);
    auto store_o = [&](int cc) {
      const int t0 = (c0 + cc) * kCk, n = min(kCk, T - t0);
      float* orow = sg.o + (size_t)(t0 - sg.t_off) * sg.o_ts + (size_t)h * sg.o_hs + v;
      uint32_t oa[32];
      tmem_ld32(tmem + kTmX + 64u * (uint32_t)(cc & 1) + lane_off + 32, oa);
      tmem_ld_wait();
#pragma unroll
      for (int tt = 0; tt < kCk; ++tt)
        if (tt < n) orow[(size_t)tt * sg.o_ts] = __uint_as_float(oa[tt]);
    };
    for (int c = 0; c < nchunks && ok; ++c) {
      const int b = c & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(b1_full + 8 * b, (c >> 1) & 1));
      if (!ok) break;
      split_lo(reinterpret_cast<const float*>(smem + kScB1Raw + b * 32768u),
               reinterpret_cast<float*>(smem + kScB1Lo + b * 32768u), 2048, t);
      fence_proxy_async_smem();  // generic writes before the MMAs read them
      __syncwarp();
      if (lane == 0) mbar_arrive(b1_ready + 8 * b);
      // Kt / P: the staged raw copy, once the previous chunk's products are done
      ok = __all_sync(0xffffffffu, mbar_wait(stg_full, c & 1) && mbar_wait(kp_empty, (c & 1) ^ 1u));
      if (!ok) break;
      split_copy(stg, reinterpret_cast<float*>(smem + kScKtRaw),
                 reinterpret_cast<float*>(smem + kScKtLo), 1024, t);
      split_copy(stg + 4096, reinterpret_cast<float*>(smem + kScPRaw),
                 reinterpret_cast<float*>(smem + kScPLo), 256, t);
      fence_proxy_async_smem();  // the staging reads before the next bulk copy into it
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(stg_empty);
        mbar_arrive(kp_ready);
      }
      // chunk c - 1's (3) has completed (kp_empty above): its O^T leaves TMEM;
      // its X buffer is rewritten only by chunk c + 1's (1), which waits for
      // this warp's next b1_ready
      if (c > 0) store_o(c - 1);
    }
    if (ok && nchunks > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(kp_empty, (nchunks - 1) & 1));
      if (ok) store_o(nchunks - 1);
    }
  } else {
    // ---- epilogue: thread = value row v (TMEM lane) ----
    const int sp = warp & 3;
    const int eg = (warp - 6) >> 2;
    const int v = sp * 32 + lane;
    const uint32_t lane_off = (uint32_t)(sp * 32) << 16;
    const uint32_t kofs = 16u * (uint32_t)eg;
    const int tofs = 16 * eg;
    const uint32_t tacc = tmem + kTmAcc + lane_off + kofs, thi = tmem + kTmHi + lane_off + kofs,
                   tlo = tmem + kTmLo + lane_off + kofs;
    float* sdh = reinterpret_cast<float*>(smem + kScDHi);
    float* sdl = reinterpret_cast<float*>(smem + kScDLo);
    const float* sin = sg.start == 0 ? sg.s_in + (size_t)h * kDhd * kDhd : nullptr;
    float* sth = sg.s_out + (size_t)h * kDhd * kDhd;
    // key quarter q of the state: A copy (x, its lo part) and g x as the
    // accumulator, then the quarter is released to (1)
    auto put_quarter = [&](int q, const uint32_t (&src)[16], float g) {
      uint32_t vh[16], vl[16], vs[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float x = __uint_as_float(src[e]);
        vh[e] = src[e];
        vl[e] = tf32_lo(x);
        vs[e] = __float_as_uint(g * x);
      }
      tmem_st16(thi + 32 * q, vh);
      tmem_st16(tlo + 32 * q, vl);
      tmem_st16(tacc + 32 * q, vs);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(a_ready + 8 * q);
    };
    {
      const float g0 = gcs[(size_t)c0 * nv + h];
#pragma unroll 1
      for (int q = 0; q < 4; ++q) {
        uint32_t x0[16];
        const int k0 = (int)kofs + 32 * q;
        if (sin) {
#pragma unroll
          for (int e = 0; e < 16; ++e) x0[e] = __float_as_uint(sin[(size_t)(k0 + e) * kDhd + v]);
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            x0[e] = __float_as_uint(sg.start == 2 && k0 + e == v ? 1.f : 0.f);
        }
        put_quarter(q, x0, g0);
      }
    }
    for (int c = 0; c < nchunks && ok; ++c) {
      const float* blk = blocks + ((size_t)(c0 + c) * nv + h) * kCkBlk;
      const uint32_t tx = tmem + kTmX + 64u * (uint32_t)(c & 1) + lane_off;
      float u[16];
      if (sg.start != 2) {
#pragma unroll
        for (int tt = 0; tt < 16; ++tt) u[tt] = blk[kBlkU + (tofs + tt) * kDhd + v];
      } else {
#pragma unroll
        for (int tt = 0; tt < 16; ++tt) u[tt] = 0.f;
      }
      const float gnext = c + 1 < nchunks ? gcs[(size_t)(c0 + c + 1) * nv + h] : 0.f;
      ok = __all_sync(0xffffffffu, mbar_wait(x_done, c & 1));
      if (!ok) break;
      tc_fence_after();
      // (2) Delta^T row v, this group's 16 tokens = U^T - (W S)^T: the raw value
      // and its lo part as the A operand of (3) and (4)
      {
        uint32_t xa[16];
        tmem_ld16(tx + tofs, xa);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t hh[4], ll[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float d = u[4 * q + e] - __uint_as_float(xa[4 * q + e]);
            hh[e] = __float_as_uint(d);
            ll[e] = tf32_lo(d);
          }
          const int qq = (tofs >> 2) + q;  // 16-byte chunk of the 128-byte row
          const int pos = v * 32 + ((qq ^ (v & 7)) << 2);
          *reinterpret_cast<uint4*>(sdh + pos) = make_uint4(hh[0], hh[1], hh[2], hh[3]);
          *reinterpret_cast<uint4*>(sdl + pos) = make_uint4(ll[0], ll[1], ll[2], ll[3]);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(d_ready);
      ok = __all_sync(0xffffffffu, mbar_wait(u_done, c & 1));
      if (!ok) break;
      tc_fence_after();
      // S_{c+1}: all four quarters' loads in flight at once, then each quarter
      // is written and released before the next; the last chunk stores the
      // final state
      uint32_t va[16], vb[16], vc[16], vd[16];
      tmem_ld16(tacc, va);
      tmem_ld16(tacc + 32, vb);
      tmem_ld16(tacc + 64, vc);
      tmem_ld16(tacc + 96, vd);
      tmem_ld_wait();
      if (c + 1 == nchunks) {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          sth[(size_t)(kofs + e) * kDhd + v] = __uint_as_float(va[e]);
          sth[(size_t)(kofs + 32 + e) * kDhd + v] = __uint_as_float(vb[e]);
          sth[(size_t)(kofs + 64 + e) * kDhd + v] = __uint_as_float(vc[e]);
          sth[(size_t)(kofs + 96 + e) * kDhd + v] = __uint_as_float(vd[e]);
        }
      } else {
        put_quarter(0, va, gnext);
        put_quarter(1, vb, gnext);
        put_quarter(2, vc, gnext);
        put_quarter(3, vd, gnext);
      }
    }
  }
  if (!ok && lane == 0) atomicAdd(&g_delta_wait_timeouts, 1);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// 4b. joins segment 1 of a split scan to segment 0. Per value head, row r:
// dst[r][v] = add[r][v] + sum_k' src[r][k'] Z[k'][v], Z = the state at the cut
// ([128 k'][128 v], segment 0's final state). Token rows: src = O_M, add = dst
// = the zero-start outputs; state rows (the last 128-row tile of each head):
// src = M, add = R, dst = the real state.
//
// On tcgen05, 3xTF32 like the scan, in the scan's own shape: D^T [128 v x 128
// rows] = Z^T X^T with A = Z^T from TMEM (lane = v, column = k'; the raw value
// and its lo part, written once per CTA) and B = the tile's rows [128 x 128 k']
// K-major SWIZZLE_128B in shared memory, placed by TMA (double-buffered) with
// their lo parts written beside them; 16 k-steps x 3 MMAs of N = 128. O_M
// ([nv][T1][128]) and M ([nv][128][128]) are one row-major block, so a tile is
// four 32-column boxes of one tensor map. A CTA takes every gridDim.x-th tile
// of one head. 8 warps: warp w moves lanes 32 (w % 4).. and columns
// 64 (w / 4).. of TMEM; the epilogue's reads and writes run along v, so each
// warp touches 128 contiguous bytes per row.
constexpr int kJnRows = 128;
constexpr uint32_t kJnX = 0, kJnXLo = 131072, kJnBar = 196608;  // X: 2 x 64 KB
constexpr int kJoinSmem = (int)kJnBar + 64 + 1024;
constexpr uint32_t kJnTmD = 0, kJnTmHi = 128, kJnTmLo = 256;
__global__ void __launch_bounds__(256, 1) delta_scan_join_kernel(
    const __grid_constant__ CUtensorMap tmX, const float* __restrict__ zst,
    float* __restrict__ o, const float* __restrict__ rs, float* __restrict__ state, int T1,
    int nv) {
  extern __shared__ uint8_t jsm_raw[];
  const uint32_t base_raw = smem_u32(jsm_raw);
  const uint32_t base = (base_raw + 1023u) & ~1023u;
  uint8_t* smem = jsm_raw + (base - base_raw);
  const uint32_t full = base + kJnBar, mma_bar = base + kJnBar + 16;  // full[2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kJnBar + 32);
  const int h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ntt = (T1 + kJnRows - 1) / kJnRows, ntiles = ntt + 1;
  if (tid == 0) {
    mbar_init(full, 1);
    mbar_init(full + 8, 1);
    mbar_init(mma_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // Z, O_M, O_R, M and R come from the scan
  // tile (in this CTA's order `it`) into X buffer it % 2 (thread 0)
  auto load_tile = [&](int it) {
    const int tile = blockIdx.x + it * gridDim.x;
    const int row = tile < ntt ? h * T1 + tile * kJnRows : nv * T1 + h * kDhd;
    const uint32_t b = (uint32_t)(it & 1);
    mbar_arrive_tx(full + 8 * b, 65536u);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      tma_load_2d(base + kJnX + b * 65536u + q * 16384u, &tmX, 32 * q, row, full + 8 * b);
  };
  const int nmine = ((int)blockIdx.x < ntiles) ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  if (tid == 0) {
    if (nmine > 0) load_tile(0);
    if (nmine > 1) load_tile(1);
  }
  const int sp = warp & 3, hf = warp >> 2;
  const int v = 32 * sp + lane;  // this thread's TMEM lane = value column
  const uint32_t lane_off = (uint32_t)(32 * sp) << 16;
  {
    // A = Z^T: lane v, columns k' = 64 hf .. 64 hf + 63 (all loads in flight at once)
    const float* z = zst + (size_t)h * kDhd * kDhd + (size_t)(64 * hf) * kDhd + v;
    float zv[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) zv[i] = z[(size_t)i * kDhd];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      uint32_t vh[16], vl[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        vh[e] = __float_as_uint(zv[16 * g + e]);
        vl[e] = tf32_lo(zv[16 * g + e]);
      }
      tmem_st16(tmem + kJnTmHi + lane_off + 64 * hf + 16 * g, vh);
      tmem_st16(tmem + kJnTmLo + lane_off + 64 * hf + 16 * g, vl);
    }
    tmem_st_wait();
  }
  bool ok = true;
  for (int it = 0; it < nmine; ++it) {
    const int tile = blockIdx.x + it * gridDim.x;
    const int b = it & 1;
    const int r0 = tile < ntt ? tile * kJnRows : 0;
    const int nrows = tile < ntt ? min(kJnRows, T1 - r0) : kJnRows;
    ok = __syncthreads_and(mbar_wait(full + 8 * b, (it >> 1) & 1));
    if (!ok) break;
    // lo parts of the tile, same (swizzled) positions
    {
      const uint4* xs = reinterpret_cast<const uint4*>(smem + kJnX + b * 65536);
      uint4* xl = reinterpret_cast<uint4*>(smem + kJnXLo);
#pragma unroll 4
      for (int i = tid; i < 4096; i += 256) {
        const uint4 x = xs[i];
        xl[i] = make_uint4(tf32_lo(__uint_as_float(x.x)), tf32_lo(__uint_as_float(x.y)),
                           tf32_lo(__uint_as_float(x.z)), tf32_lo(__uint_as_float(x.w)));
      }
    }
    fence_proxy_async_smem();  // generic writes before the MMAs read them
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint64_t dxh = sw128_desc(base + kJnX + b * 65536u), dxl = sw128_desc(base + kJnXLo);
      const uint32_t d = tmem + kJnTmD, zhi = tmem + kJnTmHi, zlo = tmem + kJnTmLo;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint64_t off = (uint64_t)((j >> 2) * 16384 + (j & 3) * 32) >> 4;
        umma_tf32_ts(d, zhi + 8 * j, dxh + off, tf32_idesc(128), j > 0 ? 1u : 0u);
        umma_tf32_ts(d, zhi + 8 * j, dxl + off, tf32_idesc(128), 1u);
        umma_tf32_ts(d, zlo + 8 * j, dxh + off, tf32_idesc(128), 1u);
      }
      umma_commit(mma_bar);
    }
    // the values this thread adds to (column v of rows 64 hf ..), read while the MMAs run
    float* dst = tile < ntt ? o + ((size_t)r0 * nv + h) * kDhd + v : state + (size_t)h * kDhd * kDhd + v;
    const float* add = tile < ntt ? (const float*)o + ((size_t)r0 * nv + h) * kDhd + v
                                  : rs + (size_t)h * kDhd * kDhd + v;
    const size_t rstride = tile < ntt ? (size_t)nv * kDhd : (size_t)kDhd;
    float av[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const int r = 64 * hf + i;
      av[i] = r < nrows ? add[(size_t)r * rstride] : 0.f;
    }
    ok = __syncthreads_and(mbar_wait(mma_bar, it & 1));
    if (!ok) break;
    tc_fence_after();
    // X buffer b is free again: the tile after next goes into it
    if (tid == 0 && it + 2 < nmine) load_tile(it + 2);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      uint32_t dv[16];
      tmem_ld16(tmem + kJnTmD + lane_off + 64 * hf + 16 * g, dv);
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int r = 64 * hf + 16 * g + e;
        if (r < nrows) dst[(size_t)r * rstride] = av[16 * g + e] + __uint_as_float(dv[e]);
      }
    }
    tc_fence_before();
    __syncthreads();  // D and the lo buffer are rewritten by the next tile
  }
  if (!ok && tid == 0) atomicAdd(&g_delta_wait_timeouts, 1);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// 2-D fp32 row-major tensor map [rows][128], box 32 columns x 128 rows,
// SWIZZLE_128B (each box lands as one SW128 K-major slab).
static bool make_join_map(CUtensorMap* m, const float* ptr, uint64_t rows) {
  auto enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)kDhd, rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kDhd * 4};
  const cuuint32_t box[2] = {32u, (cuuint32_t)kJnRows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int delta_wait_timeouts(int* count, int reset) {
  if (cudaMemcpyFromSymbol(count, g_delta_wait_timeouts, sizeof(int)) != cudaSuccess)
    return IQ36_ERR_CUDA;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_delta_wait_timeouts, &zero, sizeof(int)) != cudaSuccess)
      return IQ36_ERR_CUDA;
  }
  return IQ36_OK;
}

// 4. gated RMSNorm: one warp per (token, value head), lane = 4 columns.
__global__ void __launch_bounds__(256) delta_gated_norm_kernel(const float* o, const __half* z,
                                                               const float* norm_w, float eps,
                                                               int rows, __half* out) {
  pdl_wait();
  // Each warp normalises kRows rows (one 128-wide head row of one token
  // each); the rows' loads are all issued before the first is used.
  constexpr int kRows = 4;
  const int row0 = (blockIdx.x * 8 + (threadIdx.x >> 5)) * kRows, lane = threadIdx.x & 31;
  float4 ov4[kRows];
  uint2 zr[kRows];
#pragma unroll
  for (int i = 0; i < kRows; ++i) {
    if (row0 + i < rows) {
      ov4[i] = *reinterpret_cast<const float4*>(o + (size_t)(row0 + i) * kDhd + 4 * lane);
      zr[i] = *reinterpret_cast<const uint2*>(z + (size_t)(row0 + i) * kDhd + 4 * lane);
    }
  }
  const float nwv[4] = {norm_w[4 * lane], norm_w[4 * lane + 1], norm_w[4 * lane + 2],
                        norm_w[4 * lane + 3]};
#pragma unroll
  for (int i = 0; i < kRows; ++i) {
    if (row0 + i >= rows) break;  // warp-uniform
    const float4 v = ov4[i];
    const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
    const float nsc = rsqrtf(ss / (float)kDhd + eps);
    const __half2 zlo = *reinterpret_cast<const __half2*>(&zr[i].x);
    const __half2 zhi = *reinterpret_cast<const __half2*>(&zr[i].y);
    const float zv[4] = {__low2float(zlo), __high2float(zlo), __low2float(zhi), __high2float(zhi)};
    const float ovv[4] = {v.x, v.y, v.z, v.w};
    float y[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) y[j] = ovv[j] * nsc * nwv[j] * (zv[j] * sigmoidf_acc(zv[j]));
    const __half2 lo = __floats2half2_rn(y[0], y[1]);
    const __half2 hi = __floats2half2_rn(y[2], y[3]);
    uint2 raw;
    raw.x = *reinterpret_cast<const uint32_t*>(&lo);
    raw.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(out + (size_t)(row0 + i) * kDhd + 4 * lane) = raw;
  }
  pdl_launch_dependents();
}

// workspace: qk fp32 [T, 2nk, D] | v fp16 [T, nv*D] | g, beta fp32 [T, nv] | o fp32 [T, nv, D]
// | chunk operand blocks [ceil(T/32), nv, kCkBlk] fp32 | gC [ceil(T/32), nv]; a split
// scan adds the states Z, R [nv, D, D], O_M [nv, T - 32 m, D] and M [nv, D, D]
struct DeltaWs {
  size_t qk, v, decay, beta, o, blocks, gcs, zst, rst, mst, om, total;
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
  w.gcs = up(w.blocks + (size_t)((T + kCk - 1) / kCk) * nv * kCkBlk * 4);
  w.zst = up(w.gcs + (size_t)((T + kCk - 1) / kCk) * nv * 4);
  const int m = scan_split(T);
  const size_t st = m ? (size_t)nv * kDhd * kDhd * 4 : 0;
  w.rst = w.zst + st;
  w.om = w.rst + st;  // O_M, then M right behind it (one row-major block)
  w.mst = w.om + (m ? (size_t)(T - m * kCk) * nv * kDhd * 4 : 0);
  w.total = up(w.mst + st);
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
        cudaFuncSetAttribute(delta_scan_join_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kJoinSmem) !=
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
  float* gcs = reinterpret_cast<float*>(ws + w.gcs);
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
               nv, blocks, gcs);
  const int nchunks = ceil_div(T, kCk), m = scan_split(T);
  ScanSegs sgs = {};
  if (!m) {
    sgs.s[0] = ScanSeg{state, state, o, 0, nchunks, 0, nv * kDhd, kDhd, 0};
  } else {
    float* zst = reinterpret_cast<float*>(ws + w.zst);
    sgs.s[0] = ScanSeg{state, zst, o, 0, m, 0, nv * kDhd, kDhd, 0};
    sgs.s[1] = ScanSeg{nullptr, reinterpret_cast<float*>(ws + w.rst), o, m, nchunks, 0,
                       nv * kDhd, kDhd, 1};
    // O_M head-major: the join copies a tile's rows as one block
    sgs.s[2] = ScanSeg{nullptr, reinterpret_cast<float*>(ws + w.mst),
                       reinterpret_cast<float*>(ws + w.om), m, nchunks, m * kCk, kDhd,
                       (T - m * kCk) * kDhd, 2};
  }
  if (e == cudaSuccess)
    e = launch(delta_chunk_scan_kernel, dim3(nv, m ? 3 : 1), dim3(kScThreads), (size_t)kScanSmem,
               s, (const float*)blocks, (const float*)gcs, sgs, T, nv);
  if (e == cudaSuccess && m) {
    const int T1 = T - m * kCk;
    // CTAs per head: the tiles of one head share its Z^T; one wave of CTAs
    const int tiles = ceil_div(T1, kJnRows) + 1;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return IQ36_ERR_CUDA;
    const int cph = std::max(1, std::min(tiles, sms / nv));
    CUtensorMap tmx;
    if (!make_join_map(&tmx, reinterpret_cast<const float*>(ws + w.om),
                       (uint64_t)nv * (T1 + kDhd)))
      return IQ36_ERR_CUDA;
    e = launch(delta_scan_join_kernel, dim3(cph, nv), dim3(256), (size_t)kJoinSmem, s, tmx,
               (const float*)(ws + w.zst), o + (size_t)m * kCk * nv * kDhd,
               (const float*)(ws + w.rst), state, T1, nv);
  }
  if (e == cudaSuccess)
    e = launch(delta_gated_norm_kernel, dim3(ceil_div(T * nv, 32)), dim3(256), 0, s,
               (const float*)o, reinterpret_cast<const __half*>(z_f16), norm_w, eps, T * nv,
               reinterpret_cast<__half*>(out_f16));
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}
