// delta_prefill.cu — the Gated DeltaNet block over T prompt tokens at once.
//
// The per-token decode path (delta_prep_kernel + delta_step_kernel) runs the
// causal conv and the recurrence for one token per launch. Prefill runs the
// same arithmetic over a whole prompt in four launches per layer:
//   1. delta_conv_batch_kernel: causal depthwise conv(4) + SiLU for every
//      (token, channel) — fully parallel, the conv is a 4-tap FIR over the
//      previous three inputs (or the carried state before token 0) — then the
//      per-head L2 normalisation of q and k, and the gates decay = exp(g),
//      beta = sigmoid(b) per (token, value head).
//   2. delta_conv_state_kernel: carried conv state := the last four inputs.
//   3. delta_scan_kernel: the recurrence, sequential over tokens. A warp owns
//      eight value columns of one head and keeps their 128 x 8 state slice in
//      registers for the whole prompt; the inputs of 32 tokens at a time are
//      staged in shared memory with cp.async, double-buffered.
//   4. delta_gated_norm_kernel: gated RMSNorm of every (token, value head).
//
// Semantics (same as the decode path): OpenVINO gated delta net
// (iq36_gated_delta_net.cl:36-150) — key head = value head / (nv/nk), q and k
// L2-normalised with rsqrt(sum + 1e-6), q additionally * 1/sqrt(D); per token
// S = exp(g) S; sk = S^T k; delta = (v - sk) beta; S += k delta^T; o = S^T q;
// conv with fp16 rounding points of iq36_linear_conv_swish.cl:25-63; gates of
// gguf_loader.cpp:4875-4912; gated RMSNorm of gguf_loader.cpp:4770-4786.

#include <atomic>

#include "launch.cuh"
#include "common.cuh"

namespace iq36 {

constexpr int kDhd = 128;       // DeltaNet head dim (key and value)
constexpr int kScanTC = 32;     // tokens per shared-memory chunk
constexpr int kScanWarps = 4;   // warps per CTA; 8 value columns per warp
constexpr int kScanCols = 8 * kScanWarps;
constexpr int kScanStage = 2 * kScanTC * kDhd * 4 + kScanTC * kScanCols * 2 + 2 * kScanTC * 4;
constexpr int kScanSmem = 2 * kScanStage;
constexpr int kConvTok = 32;    // tokens per CTA of the conv kernel

// Packed fp32 pairs (two independent round-to-nearest operations, the same
// results as two scalar fmaf / multiplies).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;\n"
      : "=l"(d)
      : "l"(*reinterpret_cast<const uint64_t*>(&a)), "l"(*reinterpret_cast<const uint64_t*>(&b)),
        "l"(*reinterpret_cast<const uint64_t*>(&c)));
  return *reinterpret_cast<const float2*>(&d);
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;\n"
      : "=l"(d)
      : "l"(*reinterpret_cast<const uint64_t*>(&a)), "l"(*reinterpret_cast<const uint64_t*>(&b)));
  return *reinterpret_cast<const float2*>(&d);
}

// ---------------------------------------------------------------------------
// 1. conv + SiLU + q/k normalisation + gates. Grid (ceil(T/32), ceil(segments/8)),
// 8 warps; warp = one 128-channel segment (a q head, a k head or a v head)
// over 32 consecutive tokens, lane = 4 channels; the last three inputs ride
// along in registers, so every input row is read once.
__global__ void __launch_bounds__(256) delta_conv_batch_kernel(
    const __half* qkv, int T, int nk, int nv, const float* conv_state, const float* conv_w,
    const __half* a, const __half* b, int gate_stride, const float* a_log, const float* dtb,
    float* qk_out, __half* v_out, float* decay_out, float* beta_out) {
  pdl_wait();
  const int t0 = blockIdx.x * kConvTok, t1 = min(T, t0 + kConvTok);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (blockIdx.y == 0) {
    for (int i = threadIdx.x; i < (t1 - t0) * nv; i += blockDim.x) {
      const int t = t0 + i / nv, h = i % nv;
      const float xa = __half2float(a[(size_t)t * gate_stride + h]) + dtb[h];
      const float sp = xa > 20.f ? xa : log1pf(expf(xa));
      const float g = -expf(a_log[h]) * sp;
      decay_out[(size_t)t * nv + h] = expf(g);
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
// 3. the recurrence. Grid (128/32, nv), 4 warps. Warp w owns value columns
// j = j0 + 8w + cl (cl = lane & 7); lane group rg = lane >> 3 owns the 32 key
// rows r = 16m + 4rg + e (m in 0..7, e in 0..3), so each q/k row load is a
// 16-byte vector and the four lane groups read one contiguous 64-byte piece.
// Sums over key rows are a per-lane 32-term partial (packed fp32 pairs) plus
// two xor-shuffles (lane bits 3, 4). Per token, both sums are taken on the
// state before the update,
//   pk = S^T k, pq = S^T q  (reduced together),
//   delta = beta (v - a pk),  o = a pq + delta (k . q),  S = a S + k delta^T,
// which is the step above rearranged (S^T q after the update equals
// a S^T q + delta (k . q)), so only pk -> delta -> S is on the token-to-token
// chain. k . q per token is computed once per chunk; outputs are staged in
// shared memory and written per chunk.
__global__ void __launch_bounds__(32 * kScanWarps, 1)
    delta_scan_kernel(const float* __restrict__ qk, const __half* __restrict__ v,
                      const float* __restrict__ decay, const float* __restrict__ beta,
                      float* __restrict__ state, float* __restrict__ o_out, int T, int nk,
                      int nv) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float kq_s[kScanTC];
  __shared__ __align__(16) float o_s[kScanTC][kScanCols];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rg = lane >> 3, cl = lane & 7;
  const int vh = blockIdx.y, j0 = blockIdx.x * kScanCols;
  const int kh = vh / (nv / nk);
  const int col = j0 + 8 * warp + cl;

  auto sq = [&](int buf) { return reinterpret_cast<float*>(smem + buf * kScanStage); };
  auto sk = [&](int buf) { return sq(buf) + kScanTC * kDhd; };
  auto sv = [&](int buf) { return reinterpret_cast<__half*>(sk(buf) + kScanTC * kDhd); };
  auto sd = [&](int buf) { return reinterpret_cast<float*>(sv(buf) + kScanTC * kScanCols); };
  auto sb = [&](int buf) { return sd(buf) + kScanTC; };

  pdl_wait();
  // stage the inputs of tokens [t0, t0 + kScanTC) into buffer buf
  auto load_chunk = [&](int t0, int buf) {
    const int n = min(kScanTC, T - t0);
    const uint32_t q_s = smem_u32(sq(buf)), k_s = smem_u32(sk(buf)), v_s = smem_u32(sv(buf));
    // q and k: n tokens x 32 pieces of 16 bytes each
    for (int i = threadIdx.x; i < 2 * kScanTC * 32; i += blockDim.x) {
      const int which = i / (kScanTC * 32), rem = i % (kScanTC * 32);
      const int u = rem >> 5, p = rem & 31;
      if (u < n) {
        const float* src =
            qk + ((size_t)(t0 + u) * 2 * nk + (which ? nk + kh : kh)) * kDhd + 4 * p;
        cp_async_16((which ? k_s : q_s) + (u * kDhd + 4 * p) * 4, src, 16);
      }
    }
    // v: n tokens x 4 pieces (32 halves)
    for (int i = threadIdx.x; i < kScanTC * 4; i += blockDim.x) {
      const int u = i >> 2, p = i & 3;
      if (u < n)
        cp_async_16(v_s + (u * kScanCols + 8 * p) * 2,
                    v + (size_t)(t0 + u) * nv * kDhd + vh * kDhd + j0 + 8 * p, 16);
    }
    if (threadIdx.x < kScanTC && (int)threadIdx.x < n) {
      sd(buf)[threadIdx.x] = decay[(size_t)(t0 + threadIdx.x) * nv + vh];
      sb(buf)[threadIdx.x] = beta[(size_t)(t0 + threadIdx.x) * nv + vh];
    }
  };

  // S2[2m + h] = rows (16m + 4rg + 2h, +1) of column col
  float2 S2[16];
  const size_t sbase = (size_t)vh * kDhd * kDhd;
#pragma unroll
  for (int m = 0; m < 8; ++m)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const size_t r = 16 * m + 4 * rg + 2 * h;
      S2[2 * m + h] = make_float2(state[sbase + r * kDhd + col], state[sbase + (r + 1) * kDhd + col]);
    }

  const int nchunks = (T + kScanTC - 1) / kScanTC;
  load_chunk(0, 0);
  cp_async_commit();
  for (int c = 0; c < nchunks; ++c) {
    const int buf = c & 1;
    if (c + 1 < nchunks) {
      load_chunk((c + 1) * kScanTC, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int t0 = c * kScanTC, n = min(kScanTC, T - t0);
    const float* qs = sq(buf);
    const float* ks = sk(buf);
    const __half* vs = sv(buf);
    const float* ds = sd(buf);
    const float* bs = sb(buf);
    // k . q of the chunk's tokens
    for (int u = warp; u < n; u += kScanWarps) {
      const float4 x = *reinterpret_cast<const float4*>(qs + u * kDhd + 4 * lane);
      const float4 y = *reinterpret_cast<const float4*>(ks + u * kDhd + 4 * lane);
      const float d = warp_sum(x.x * y.x + x.y * y.y + x.z * y.z + x.w * y.w);
      if (lane == 0) kq_s[u] = d;
    }
    __syncthreads();
#pragma unroll 2
    for (int u = 0; u < n; ++u) {
      float2 k2[16], q2[16];
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const float4 k4 = *reinterpret_cast<const float4*>(ks + u * kDhd + 16 * m + 4 * rg);
        const float4 q4 = *reinterpret_cast<const float4*>(qs + u * kDhd + 16 * m + 4 * rg);
        k2[2 * m] = make_float2(k4.x, k4.y);
        k2[2 * m + 1] = make_float2(k4.z, k4.w);
        q2[2 * m] = make_float2(q4.x, q4.y);
        q2[2 * m + 1] = make_float2(q4.z, q4.w);
      }
      const float a = ds[u], bt = bs[u], kq = kq_s[u];
      const float vv = __half2float(vs[u * kScanCols + 8 * warp + cl]);
      float2 pk[4], pq[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        pk[i] = fmul2(S2[i], k2[i]);
        pq[i] = fmul2(S2[i], q2[i]);
      }
#pragma unroll
      for (int i = 4; i < 16; ++i) {
        pk[i & 3] = ffma2(S2[i], k2[i], pk[i & 3]);
        pq[i & 3] = ffma2(S2[i], q2[i], pq[i & 3]);
      }
      float sk = ((pk[0].x + pk[0].y) + (pk[1].x + pk[1].y)) +
                 ((pk[2].x + pk[2].y) + (pk[3].x + pk[3].y));
      float sq_ = ((pq[0].x + pq[0].y) + (pq[1].x + pq[1].y)) +
                  ((pq[2].x + pq[2].y) + (pq[3].x + pq[3].y));
      sk += __shfl_xor_sync(0xffffffffu, sk, 8);
      sq_ += __shfl_xor_sync(0xffffffffu, sq_, 8);
      sk += __shfl_xor_sync(0xffffffffu, sk, 16);
      sq_ += __shfl_xor_sync(0xffffffffu, sq_, 16);
      const float delta = (vv - a * sk) * bt;
      const float2 a2 = make_float2(a, a), d2 = make_float2(delta, delta);
#pragma unroll
      for (int i = 0; i < 16; ++i) S2[i] = ffma2(k2[i], d2, fmul2(S2[i], a2));
      if (rg == 0) o_s[u][8 * warp + cl] = fmaf(delta, kq, a * sq_);
    }
    __syncthreads();  // o_s complete; buffer buf is refilled by the next iteration's load
    for (int i = threadIdx.x; i < n * (kScanCols / 4); i += blockDim.x) {
      const int u = i / (kScanCols / 4), p = i % (kScanCols / 4);
      *reinterpret_cast<float4*>(o_out + ((size_t)(t0 + u) * nv + vh) * kDhd + j0 + 4 * p) =
          *reinterpret_cast<const float4*>(&o_s[u][4 * p]);
    }
  }
#pragma unroll
  for (int m = 0; m < 8; ++m)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const size_t r = 16 * m + 4 * rg + 2 * h;
      state[sbase + r * kDhd + col] = S2[2 * m + h].x;
      state[sbase + (r + 1) * kDhd + col] = S2[2 * m + h].y;
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

// workspace: qk fp32 [T, 2nk, D] | v fp16 [T, nv*D] | decay, beta fp32 [T, nv] | o fp32 [T, nv, D]
struct DeltaWs {
  size_t qk, v, decay, beta, o, total;
};
static DeltaWs delta_ws(int T, int nk, int nv) {
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  DeltaWs w;
  w.qk = 0;
  w.v = up(w.qk + (size_t)T * 2 * nk * kDhd * 4);
  w.decay = up(w.v + (size_t)T * nv * kDhd * 2);
  w.beta = up(w.decay + (size_t)T * nv * 4);
  w.o = up(w.beta + (size_t)T * nv * 4);
  w.total = up(w.o + (size_t)T * nv * kDhd * 4);
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
    if (cudaFuncSetAttribute(delta_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kScanSmem) != cudaSuccess)
      return IQ36_ERR_CUDA;
    attr_set[dev].store(true);
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* qk = reinterpret_cast<float*>(ws + w.qk);
  __half* v = reinterpret_cast<__half*>(ws + w.v);
  float* dec = reinterpret_cast<float*>(ws + w.decay);
  float* bet = reinterpret_cast<float*>(ws + w.beta);
  float* o = reinterpret_cast<float*>(ws + w.o);
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
    e = launch(delta_scan_kernel, dim3(kDhd / kScanCols, nv), dim3(32 * kScanWarps),
               (size_t)kScanSmem, s, (const float*)qk, (const __half*)v, (const float*)dec,
               (const float*)bet, state, o, T, nk, nv);
  if (e == cudaSuccess)
    e = launch(delta_gated_norm_kernel, dim3(ceil_div(T * nv, 8)), dim3(256), 0, s,
               (const float*)o, reinterpret_cast<const __half*>(z_f16), norm_w, eps, T * nv,
               reinterpret_cast<__half*>(out_f16));
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}
