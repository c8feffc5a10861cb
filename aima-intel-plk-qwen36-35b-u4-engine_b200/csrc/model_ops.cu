// model_ops.cu — the small per-token ops around the four hot operators that a
// full batch-1 decode step of the Qwen3.6-35B-A3B-shaped model needs.

#include <cooperative_groups.h>

#include "../../include/iq36_synth.h"
#include "launch.cuh"
#include "common.cuh"

namespace cg = cooperative_groups;

namespace iq36 {

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < nw; ++i) r += red[i];
  return r;
}

// ---------------------------------------------------------------------------
// RMSNorm: one CTA per (row, segment of wlen). gguf_loader.cpp:3368-3391,
// repeated form :3410-3439.
__global__ void __launch_bounds__(256) rms_norm_kernel(const float* in, int dim, const float* w,
                                                       int wlen, float eps, void* out,
                                                       int out_dtype) {
  __shared__ float red[32];
  pdl_wait();
  const size_t base = (size_t)blockIdx.x * dim + (size_t)blockIdx.y * wlen;
  float ss = 0.f;
  for (int i = threadIdx.x; i < wlen; i += blockDim.x) ss = fmaf(in[base + i], in[base + i], ss);
  ss = block_sum(ss, red);
  const float sc = rsqrtf(ss / (float)wlen + eps);
  pdl_launch_dependents();
  for (int i = threadIdx.x; i < wlen; i += blockDim.x) {
    const float y = in[base + i] * sc * w[i];
    if (out_dtype == IQ36_F16) reinterpret_cast<__half*>(out)[base + i] = __float2half_rn(y);
    else reinterpret_cast<float*>(out)[base + i] = y;
  }
}

// ---------------------------------------------------------------------------
// Full-attention pre-step. One warp per head vector (n_q query heads, then n_kv
// key heads); lane owns dims [8*lane, 8*lane+8) of a 256-dim head.
// Split q/gate (gguf_loader.cpp:5928-5950), per-head RMSNorm, rotate-half RoPE
// on the first rope_dim dims (iq36_qk_rope_layout.cl:37-60) with angles
// evaluated in fp64 once per token (shared memory), fp16 store; K/V appended
// at *pos_dev through the block table (iq36_hot_ring_update.cl:7-28). Block x handles token x of a batch
// (position *pos_dev + x; rows of q_full, k, v, q_out, gate_out per token);
// the decode step launches one block.
__global__ void attn_prep_kernel(const __half* q_full, const __half* k, const __half* v,
                                 const float* qn_w, const float* kn_w, float eps,
                                 const int32_t* pos_dev, int n_q, int n_kv, int rope_dim,
                                 float rope_base, const int32_t* bt, int bs, __half* kc,
                                 __half* vc, __half* q_out, __half* gate_out) {
  __shared__ float rope_c[128], rope_s[128];
  // the attention split kernel may launch now: before its wait it only
  // prefetches cache pages that precede the token appended here
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = 256;
  // The positions are written before the step (never by the projection this
  // kernel waits on), so the angles are computed before the wait. Frequency
  // i's angle is computed once per token, in fp64, by thread i mod blockDim;
  // element d takes frequency d % half.
  const int pos = *pos_dev + blockIdx.x;
  const int half = rope_dim / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const double inv = pow((double)rope_base, -2.0 * (double)i / (double)rope_dim);
    double sn, cs;
    sincos((double)pos * inv, &sn, &cs);
    rope_c[i] = (float)cs;
    rope_s[i] = (float)sn;
  }
  pdl_wait();
  // Each warp loads and RMS-normalises its row before the barrier that
  // publishes the angles, so the fp64 angle latency overlaps the loads.
  const bool active = warp < n_q + n_kv;  // warp-uniform
  q_full += (size_t)blockIdx.x * 2 * n_q * D;
  k += (size_t)blockIdx.x * n_kv * D;
  v += (size_t)blockIdx.x * n_kv * D;
  q_out += (size_t)blockIdx.x * n_q * D;
  gate_out += (size_t)blockIdx.x * n_q * D;
  const bool is_q = warp < n_q;
  const int h = is_q ? warp : warp - n_q;
  const __half* src = is_q ? q_full + (size_t)(2 * h) * D : k + (size_t)h * D;
  const float* nw = is_q ? qn_w : kn_w;
  float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (active) {
    const uint4 raw = *reinterpret_cast<const uint4*>(src + 8 * lane);
    const __half* hp = reinterpret_cast<const __half*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = __half2float(hp[j]);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(x[j], x[j], ss);
    ss = warp_sum(ss);
    const float sc = rsqrtf(ss / (float)D + eps);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = x[j] * sc * nw[8 * lane + j];
  }
  __syncthreads();  // rope_c / rope_s written
  if (!active) return;
  const int xo = half / 8;  // partner lane offset
  float y[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float partner = __shfl_xor_sync(0xffffffffu, x[j], xo);
    const int d = 8 * lane + j;
    y[j] = x[j];
    if (d < rope_dim) {
      const float c = rope_c[d % half], sn = rope_s[d % half];
      y[j] = d < half ? x[j] * c - partner * sn : x[j] * c + partner * sn;
    }
  }
  uint4 packed;
  __half* ph = reinterpret_cast<__half*>(&packed);
#pragma unroll
  for (int j = 0; j < 8; ++j) ph[j] = __float2half_rn(y[j]);
  if (is_q) {
    *reinterpret_cast<uint4*>(q_out + (size_t)h * D + 8 * lane) = packed;
    *reinterpret_cast<uint4*>(gate_out + (size_t)h * D + 8 * lane) =
        *reinterpret_cast<const uint4*>(q_full + (size_t)(2 * h + 1) * D + 8 * lane);
  } else {
    const int blk = bt[pos / bs];
    const size_t slot = (((size_t)blk * bs + pos % bs) * n_kv + h) * D + 8 * lane;
    *reinterpret_cast<uint4*>(kc + slot) = packed;
    *reinterpret_cast<uint4*>(vc + slot) =
        *reinterpret_cast<const uint4*>(v + (size_t)h * D + 8 * lane);
  }
}

// ---------------------------------------------------------------------------
// DeltaNet pre-step: causal conv(4) + SiLU for one token with fp16 rounding of
// the convolution and of the activation (iq36_linear_conv_swish.cl:25-63),
// state [C, 4] fp32 (fp16-exact values); gate/beta (gguf_loader.cpp:4875-4912).
__global__ void __launch_bounds__(256) delta_prep_kernel(const __half* qkv, int C,
                                                         float* conv_state, const float* conv_w,
                                                         const __half* a, const __half* b,
                                                         const float* a_log, const float* dtb,
                                                         int nv, __half* act, float* g_out,
                                                         float* beta_out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  // the conv state and weights do not depend on the projection: load them first
  float4 st = make_float4(0.f, 0.f, 0.f, 0.f), w = st;
  if (c < C) {
    st = reinterpret_cast<const float4*>(conv_state)[c];
    w = reinterpret_cast<const float4*>(conv_w)[c];
  }
  pdl_wait();
  // the recurrence kernel may launch now (the projection has completed): it
  // loads its state slice before its own wait while this kernel runs
  pdl_launch_dependents();
  if (c < C) {
    const float xv = __half2float(qkv[c]);
    float s = w.x * st.y;
    s = fmaf(w.y, st.z, s);
    s = fmaf(w.z, st.w, s);
    s = fmaf(w.w, xv, s);
    const float conv = __half2float(__float2half_rn(s));
    act[c] = __float2half_rn(conv / (1.0f + expf(-conv)));
    reinterpret_cast<float4*>(conv_state)[c] = make_float4(st.y, st.z, st.w, xv);
  }
  if (blockIdx.x == 0 && threadIdx.x < nv) {
    const int h = threadIdx.x;
    const float xa = __half2float(a[h]) + dtb[h];
    const float sp = xa > 20.f ? xa : log1pf(expf(xa));
    g_out[h] = -expf(a_log[h]) * sp;
    beta_out[h] = sigmoidf_acc(__half2float(b[h]));
  }
}

// ---------------------------------------------------------------------------
// Gated DeltaNet recurrent step (OpenVINO semantics,
// iq36_gated_delta_net.cl:36-150) fused with the gated RMSNorm
// (gguf_loader.cpp:4770-4786). Grid (nv, D/16) with clusters of D/16 CTAs
// along y: one cluster per value head; CTA = 128 threads, thread i owns key
// row i of the 16-column state slice. The head's RMS is summed across the
// cluster through distributed shared memory.

// Reduce 16 per-thread column values over the warp: returns the full sum of
// column col(lane) = bits 4..1 of lane (pairs of lanes hold the same column).
__device__ __forceinline__ float reduce_scatter16(float v[16]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const bool up = lane & 16;
    const float send = up ? v[j] : v[j + 8];
    const float keep = up ? v[j + 8] : v[j];
    v[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const bool up = lane & 8;
    const float send = up ? v[j] : v[j + 4];
    const float keep = up ? v[j + 4] : v[j];
    v[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const bool up = lane & 4;
    const float send = up ? v[j] : v[j + 2];
    const float keep = up ? v[j + 2] : v[j];
    v[j] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  {
    const bool up = lane & 2;
    const float send = up ? v[0] : v[1];
    const float keep = up ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

__device__ __forceinline__ int scatter16_col(int lane) {
  return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}

__global__ void __cluster_dims__(1, 8, 1) __launch_bounds__(128)
    delta_step_kernel(const __half* act, const float* g, const float* beta, float* state,
                      const __half* z, const float* norm_w, float eps, int nk, int nv,
                      __half* out) {
  constexpr int D = 128, NC = 16;
  __shared__ float red[4][NC];
  __shared__ float vals[3][NC];  // delta, o, scratch
  __shared__ float qk_red[2][4];
  __shared__ float part;
  cg::cluster_group cluster = cg::this_cluster();
  const int vh = blockIdx.x, j0 = blockIdx.y * NC;
  const int i = threadIdx.x, lane = i & 31, warp = i >> 5;
  const int kh = vh / (nv / nk);
  // the state slice is written only by this kernel's previous token
  float s[NC];
  float* srow = state + ((size_t)vh * D + i) * D + j0;
#pragma unroll
  for (int j = 0; j < NC; j += 4) {
    const float4 v4 = *reinterpret_cast<const float4*>(srow + j);
    s[j] = v4.x;
    s[j + 1] = v4.y;
    s[j + 2] = v4.z;
    s[j + 3] = v4.w;
  }
  pdl_wait();
  float q = __half2float(act[(size_t)kh * D + i]);
  float kk = __half2float(act[(size_t)(nk + kh) * D + i]);
  {
    const float qs = warp_sum(q * q), ks = warp_sum(kk * kk);
    if (lane == 0) {
      qk_red[0][warp] = qs;
      qk_red[1][warp] = ks;
    }
  }
  __syncthreads();
  const float qs = qk_red[0][0] + qk_red[0][1] + qk_red[0][2] + qk_red[0][3];
  const float ks = qk_red[1][0] + qk_red[1][1] + qk_red[1][2] + qk_red[1][3];
  q = q * rsqrtf(qs + 1e-6f) * rsqrtf((float)D);
  kk = kk * rsqrtf(ks + 1e-6f);
  const float decay = expf(g[vh]);
  const float b = beta[vh];
  float tmp[NC];
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    s[j] *= decay;
    tmp[j] = s[j] * kk;
  }
  {
    const float r = reduce_scatter16(tmp);
    if ((lane & 1) == 0) red[warp][scatter16_col(lane)] = r;
  }
  __syncthreads();
  if (i < NC) {
    const float sk = red[0][i] + red[1][i] + red[2][i] + red[3][i];
    const float vv = __half2float(act[(size_t)(2 * nk + vh) * D + j0 + i]);
    vals[0][i] = (vv - sk) * b;
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    s[j] = fmaf(kk, vals[0][j], s[j]);
    tmp[j] = s[j] * q;
  }
#pragma unroll
  for (int j = 0; j < NC; j += 4)
    *reinterpret_cast<float4*>(srow + j) = make_float4(s[j], s[j + 1], s[j + 2], s[j + 3]);
  {
    const float r = reduce_scatter16(tmp);
    __syncthreads();
    if ((lane & 1) == 0) red[warp][scatter16_col(lane)] = r;
  }
  __syncthreads();
  if (i < NC) vals[1][i] = red[0][i] + red[1][i] + red[2][i] + red[3][i];
  __syncthreads();
  if (i == 0) {
    float p = 0.f;
    for (int j = 0; j < NC; ++j) p = fmaf(vals[1][j], vals[1][j], p);
    part = p;
  }
  cluster.sync();
  if (i < NC) {
    float tot = 0.f;
    for (unsigned r = 0; r < cluster.num_blocks(); ++r) tot += *cluster.map_shared_rank(&part, r);
    const float nsc = rsqrtf(tot / (float)D + eps);
    const float zv = __half2float(z[(size_t)vh * D + j0 + i]);
    const float y = vals[1][i] * nsc * norm_w[j0 + i] * (zv * sigmoidf_acc(zv));
    out[(size_t)vh * D + j0 + i] = __float2half_rn(y);
  }
  pdl_launch_dependents();
  cluster.sync();
}

// ---------------------------------------------------------------------------
// Row y of h [T, hidden] = float(table[tok[y]]) (grid y = token; decode: T = 1).
__global__ void embed_kernel(const __half* table, int hidden, const int32_t* tok, float* h) {
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < hidden)
    h[(size_t)blockIdx.y * hidden + i] = __half2float(table[(size_t)tok[blockIdx.y] * hidden + i]);
}

// Greedy top-1 keys: (order-preserving fp32 bits, inverted id); the larger key
// is the larger logit, then the lower id (iq36_greedy_top1.cl:8-13).
__device__ __forceinline__ uint64_t top1_key(float v, uint32_t id) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b ^ 0x80000000u);
  return ((uint64_t)ord << 32) | (uint64_t)(~id);
}

__device__ __forceinline__ uint64_t block_max_u64(uint64_t k, uint64_t* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t other = __shfl_xor_sync(0xffffffffu, k, o);
    k = other > k ? other : k;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = k;
  __syncthreads();
  uint64_t r = 0;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) r = red[i] > r ? red[i] : r;
  return r;
}

__global__ void __launch_bounds__(256) argmax_partial_kernel(const float* logits, int n,
                                                             uint64_t* partial) {
  __shared__ uint64_t red[8];
  pdl_wait();
  uint64_t best = 0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const uint64_t k = top1_key(logits[i], (uint32_t)i);
    best = k > best ? k : best;
  }
  best = block_max_u64(best, red);
  pdl_launch_dependents();
  if (threadIdx.x == 0) partial[blockIdx.x] = best;
}

__global__ void __launch_bounds__(256) argmax_final_kernel(const uint64_t* partial, int np,
                                                           int32_t* token) {
  __shared__ uint64_t red[8];
  pdl_wait();
  uint64_t best = 0;
  for (int i = threadIdx.x; i < np; i += blockDim.x) best = partial[i] > best ? partial[i] : best;
  best = block_max_u64(best, red);
  if (threadIdx.x == 0) *token = (int32_t)(~(uint32_t)(best & 0xFFFFFFFFu));
}

constexpr int kArgmaxBlocks = 296;

// ---------------------------------------------------------------------------
__global__ void synth_fill_kernel(void* dst, int64_t count, int kind, uint64_t seed,
                                  uint64_t tensor, float lo, float hi) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    switch (kind) {
      case 0: reinterpret_cast<uint8_t*>(dst)[i] = iq36_synth_u8(seed, tensor, (uint64_t)i); break;
      case 1:
        reinterpret_cast<__half*>(dst)[i] =
            __float2half_rn(iq36_synth_uniform(seed, tensor, (uint64_t)i, lo, hi));
        break;
      case 2:
        reinterpret_cast<__half*>(dst)[i] =
            __float2half_rn(iq36_synth_normal(seed, tensor, (uint64_t)i, lo));
        break;
      case 3:
        reinterpret_cast<float*>(dst)[i] = iq36_synth_uniform(seed, tensor, (uint64_t)i, lo, hi);
        break;
      case 4: reinterpret_cast<float*>(dst)[i] = iq36_synth_normal(seed, tensor, (uint64_t)i, lo); break;
      default: break;
    }
  }
}

}  // namespace iq36

using namespace iq36;

extern "C" int iq36_rms_norm(const float* in, int32_t rows, int32_t dim, const float* weight,
                             int32_t weight_len, float eps, void* out, int32_t out_dtype,
                             iq36_stream_t stream) {
  if (!in || !weight || !out) return IQ36_ERR_ARG;
  if (rows < 1 || dim < 1 || weight_len < 1 || dim % weight_len) return IQ36_ERR_SHAPE;
  if (out_dtype != IQ36_F32 && out_dtype != IQ36_F16) return IQ36_ERR_ARG;
  const cudaError_t e = launch(rms_norm_kernel, dim3(rows, dim / weight_len), dim3(256), 0,
                               as_stream(stream), in, dim, weight, weight_len, eps, out,
                               out_dtype);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

static int attn_prep_launch(const void* q_full_f16, const void* k_f16, const void* v_f16,
                            const float* q_norm_w, const float* k_norm_w, float eps,
                            const int32_t* pos_dev, int32_t tokens, int32_t n_q_heads,
                            int32_t n_kv_heads, int32_t head_dim, int32_t rope_dim,
                            float rope_base, const int32_t* block_table, int32_t block_size,
                            void* k_cache, void* v_cache, void* q_out_f16, void* gate_out_f16,
                            iq36_stream_t stream) {
  if (!q_full_f16 || !k_f16 || !v_f16 || !q_norm_w || !k_norm_w || !pos_dev || !block_table ||
      !k_cache || !v_cache || !q_out_f16 || !gate_out_f16)
    return IQ36_ERR_ARG;
  if (head_dim != 256 || n_q_heads < 1 || n_kv_heads < 1 || n_q_heads + n_kv_heads > 32 ||
      block_size < 1 || tokens < 1)
    return IQ36_ERR_SHAPE;
  if (rope_dim != 16 && rope_dim != 32 && rope_dim != 64 && rope_dim != 128 && rope_dim != 256)
    return IQ36_ERR_SHAPE;
  if (!aligned(q_full_f16, 16) || !aligned(k_f16, 16) || !aligned(v_f16, 16) ||
      !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(q_out_f16, 16) ||
      !aligned(gate_out_f16, 16))
    return IQ36_ERR_ALIGN;
  const cudaError_t e = launch(
      attn_prep_kernel, dim3(tokens), dim3(32 * (n_q_heads + n_kv_heads)), 0, as_stream(stream),
      reinterpret_cast<const __half*>(q_full_f16), reinterpret_cast<const __half*>(k_f16),
      reinterpret_cast<const __half*>(v_f16), q_norm_w, k_norm_w, eps, pos_dev, n_q_heads,
      n_kv_heads, rope_dim, rope_base, block_table, block_size,
      reinterpret_cast<__half*>(k_cache), reinterpret_cast<__half*>(v_cache),
      reinterpret_cast<__half*>(q_out_f16), reinterpret_cast<__half*>(gate_out_f16));
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

extern "C" int iq36_attn_prep(const void* q_full_f16, const void* k_f16, const void* v_f16,
                              const float* q_norm_w, const float* k_norm_w, float eps,
                              const int32_t* pos_dev, int32_t n_q_heads, int32_t n_kv_heads,
                              int32_t head_dim, int32_t rope_dim, float rope_base,
                              const int32_t* block_table, int32_t block_size, void* k_cache,
                              void* v_cache, void* q_out_f16, void* gate_out_f16,
                              iq36_stream_t stream) {
  return attn_prep_launch(q_full_f16, k_f16, v_f16, q_norm_w, k_norm_w, eps, pos_dev, 1,
                          n_q_heads, n_kv_heads, head_dim, rope_dim, rope_base, block_table,
                          block_size, k_cache, v_cache, q_out_f16, gate_out_f16, stream);
}

extern "C" int iq36_attn_prep_batch(const void* q_full_f16, const void* k_f16,
                                    const void* v_f16, const float* q_norm_w,
                                    const float* k_norm_w, float eps, const int32_t* pos_dev,
                                    int32_t tokens, int32_t n_q_heads, int32_t n_kv_heads,
                                    int32_t head_dim, int32_t rope_dim, float rope_base,
                                    const int32_t* block_table, int32_t block_size,
                                    void* k_cache, void* v_cache, void* q_out_f16,
                                    void* gate_out_f16, iq36_stream_t stream) {
  return attn_prep_launch(q_full_f16, k_f16, v_f16, q_norm_w, k_norm_w, eps, pos_dev, tokens,
                          n_q_heads, n_kv_heads, head_dim, rope_dim, rope_base, block_table,
                          block_size, k_cache, v_cache, q_out_f16, gate_out_f16, stream);
}

extern "C" int iq36_delta_prep(const void* qkv_f16, int32_t channels, float* conv_state,
                               const float* conv_w, const void* a_f16, const void* b_f16,
                               const float* a_log, const float* dt_bias, int32_t n_v_heads,
                               void* qkv_act_f16, float* g_out, float* beta_out,
                               iq36_stream_t stream) {
  if (!qkv_f16 || !conv_state || !conv_w || !a_f16 || !b_f16 || !a_log || !dt_bias ||
      !qkv_act_f16 || !g_out || !beta_out)
    return IQ36_ERR_ARG;
  if (channels < 1 || n_v_heads < 1 || n_v_heads > 256) return IQ36_ERR_SHAPE;
  if (!aligned(conv_state, 16) || !aligned(conv_w, 16)) return IQ36_ERR_ALIGN;
  const cudaError_t e =
      launch(delta_prep_kernel, dim3(ceil_div(channels, 256)), dim3(256), 0, as_stream(stream),
             reinterpret_cast<const __half*>(qkv_f16), channels, conv_state, conv_w,
             reinterpret_cast<const __half*>(a_f16), reinterpret_cast<const __half*>(b_f16),
             a_log, dt_bias, n_v_heads, reinterpret_cast<__half*>(qkv_act_f16), g_out, beta_out);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

extern "C" int iq36_delta_step(const void* qkv_act_f16, const float* g, const float* beta,
                               float* state, const void* z_f16, const float* norm_w, float eps,
                               int32_t n_k_heads, int32_t n_v_heads, int32_t head_dim,
                               void* out_f16, iq36_stream_t stream) {
  if (!qkv_act_f16 || !g || !beta || !state || !z_f16 || !norm_w || !out_f16) return IQ36_ERR_ARG;
  if (head_dim != 128 || n_k_heads < 1 || n_v_heads < 1 || n_v_heads % n_k_heads)
    return IQ36_ERR_SHAPE;
  if (!aligned(state, 16)) return IQ36_ERR_ALIGN;
  const cudaError_t e = launch(delta_step_kernel, dim3(n_v_heads, head_dim / 16), dim3(128), 0,
                               as_stream(stream), reinterpret_cast<const __half*>(qkv_act_f16),
                               g, beta, state, reinterpret_cast<const __half*>(z_f16), norm_w,
                               eps, n_k_heads, n_v_heads, reinterpret_cast<__half*>(out_f16));
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

extern "C" int iq36_embed(const void* table_f16, int32_t vocab, int32_t hidden,
                          const int32_t* token_dev, float* h, iq36_stream_t stream) {
  if (!table_f16 || !token_dev || !h) return IQ36_ERR_ARG;
  if (vocab < 1 || hidden < 1) return IQ36_ERR_SHAPE;
  const cudaError_t e = launch(embed_kernel, dim3(ceil_div(hidden, 256)), dim3(256), 0,
                               as_stream(stream), reinterpret_cast<const __half*>(table_f16),
                               hidden, token_dev, h);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

extern "C" int iq36_embed_batch(const void* table_f16, int32_t vocab, int32_t hidden,
                                const int32_t* tokens_dev, int32_t T, float* h,
                                iq36_stream_t stream) {
  if (!table_f16 || !tokens_dev || !h) return IQ36_ERR_ARG;
  if (vocab < 1 || hidden < 1 || T < 1 || T > 65535) return IQ36_ERR_SHAPE;
  const cudaError_t e = launch(embed_kernel, dim3(ceil_div(hidden, 256), T), dim3(256), 0,
                               as_stream(stream), reinterpret_cast<const __half*>(table_f16),
                               hidden, tokens_dev, h);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

extern "C" size_t iq36_argmax_workspace_bytes(void) { return kArgmaxBlocks * sizeof(uint64_t); }

extern "C" int iq36_argmax(const float* logits, int32_t n, int32_t* token_out, void* workspace,
                           size_t workspace_bytes, iq36_stream_t stream) {
  if (!logits || !token_out) return IQ36_ERR_ARG;
  if (n < 1) return IQ36_ERR_SHAPE;
  if (!workspace || workspace_bytes < iq36_argmax_workspace_bytes()) return IQ36_ERR_WORKSPACE;
  if (!aligned(workspace, 8)) return IQ36_ERR_ALIGN;
  uint64_t* part = reinterpret_cast<uint64_t*>(workspace);
  const int nb = std::min(kArgmaxBlocks, ceil_div(n, 256));
  cudaError_t e = launch(argmax_partial_kernel, dim3(nb), dim3(256), 0, as_stream(stream), logits,
                         n, part);
  if (e != cudaSuccess) return IQ36_ERR_CUDA;
  e = launch(argmax_final_kernel, dim3(1), dim3(256), 0, as_stream(stream),
             (const uint64_t*)part, nb, token_out);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

extern "C" int iq36_synth_fill(void* dst, int64_t count, int32_t kind, uint64_t seed,
                               uint64_t tensor, float lo, float hi, iq36_stream_t stream) {
  if (!dst || kind < 0 || kind > 4) return IQ36_ERR_ARG;
  if (count < 0) return IQ36_ERR_SHAPE;
  if (count == 0) return IQ36_OK;
  const int64_t blocks = std::min<int64_t>((count + 255) / 256, 148 * 16);
  synth_fill_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(dst, count, kind, seed,
                                                                      tensor, lo, hi);
  return cudaGetLastError() == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

extern "C" uint64_t iq36_synth_tensor_id(int32_t layer, int32_t slot, int32_t sub) {
  return iq36_tensor_id(layer, slot, sub);
}

extern "C" void iq36_synth_tensor_spec(int32_t slot, int32_t sub, int32_t* kind, float* lo,
                                       float* hi) {
  int k;
  iq36_synth_spec(slot, sub, &k, lo, hi);
  *kind = k;
}

namespace iq36 {
__global__ void decode_positions_kernel(int32_t* pos, int32_t* ctx, int advance) {
  pdl_wait();
  if (threadIdx.x == 0) {
    const int p = *pos + advance;
    *pos = p;
    *ctx = p + 1;
  }
}
}  // namespace iq36

extern "C" int iq36_decode_positions(int32_t* pos_dev, int32_t* ctx_dev, int32_t advance,
                                     iq36_stream_t stream) {
  if (!pos_dev || !ctx_dev) return IQ36_ERR_ARG;
  if (advance < 0) return IQ36_ERR_SHAPE;
  const cudaError_t e = launch(decode_positions_kernel, dim3(1), dim3(32), 0, as_stream(stream),
                               pos_dev, ctx_dev, (int)advance);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// u4 layout adapter: the reference's fixed-FC custom op takes each projection's
// scales and zero points transposed to group-major order
// (tools/intel_qwen36_openvino_fixed_fc.py:218-258: scale [groups, M] fp16,
// zero points [groups, M] u4 packed low nibble first; the weight bytes
// unchanged). These kernels map that form to and from the row-major
// (OpenVINO compressed-constant) layout the kernels here read.
namespace iq36 {
// scale transpose through a 32 x 33 tile: out[c][r] = in[r][c], in [R, C]
__global__ void __launch_bounds__(256) transpose_f16_kernel(const __half* in, int R, int C,
                                                            __half* out) {
  __shared__ __half tile[32][34];
  pdl_wait();
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int y = ty; y < 32; y += 8) {
    const int r = r0 + y, c = c0 + tx;
    if (r < R && c < C) tile[y][tx] = in[(size_t)r * C + c];
  }
  __syncthreads();
  for (int y = ty; y < 32; y += 8) {
    const int c = c0 + y, r = r0 + tx;
    if (c < C && r < R) out[(size_t)c * R + r] = tile[tx][y];
  }
  pdl_launch_dependents();
}
// nibble transpose: logical out[c * R + r] = in[r * C + c] (in [R, C], u4
// packed two per byte, low nibble = even element); thread per output byte
__global__ void __launch_bounds__(256) transpose_u4_kernel(const uint8_t* in, int R, int C,
                                                           uint8_t* out) {
  pdl_wait();
  const size_t j = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t n = (size_t)R * C;
  if (2 * j < n) {
    uint32_t b = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const size_t e = 2 * j + h;  // output element (c, r)
      if (e < n) {
        const size_t c = e / R, r = e % R;
        const size_t s = r * C + c;  // input element
        b |= (uint32_t)((in[s >> 1] >> ((s & 1) * 4)) & 15u) << (4 * h);
      }
    }
    out[j] = (uint8_t)b;
  }
  pdl_launch_dependents();
}
static int u4_layout_transpose(const void* scale_in, const uint8_t* zp_in, int R, int C,
                               void* scale_out, uint8_t* zp_out, iq36_stream_t stream) {
  if (!scale_in || !zp_in || !scale_out || !zp_out) return IQ36_ERR_ARG;
  if (R < 1 || C < 1 || ((int64_t)R * C) % 2 || (int64_t)R * C > (1ll << 31)) return IQ36_ERR_SHAPE;
  const cudaStream_t s = as_stream(stream);
  cudaError_t e = launch(transpose_f16_kernel, dim3(ceil_div(C, 32), ceil_div(R, 32)), dim3(256),
                         0, s, reinterpret_cast<const __half*>(scale_in), R, C,
                         reinterpret_cast<__half*>(scale_out));
  const int64_t nb = (int64_t)R * C / 2;
  if (e == cudaSuccess)
    e = launch(transpose_u4_kernel, dim3((unsigned)((nb + 255) / 256)), dim3(256), 0, s, zp_in, R,
               C, zp_out);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}
}  // namespace iq36

extern "C" int iq36_u4_layout_from_group_major(const void* scale_gm_f16, const uint8_t* zp_gm,
                                               int32_t rows, int32_t groups, void* scale_f16,
                                               uint8_t* zp, iq36_stream_t stream) {
  // group-major [groups, rows] -> row-major [rows, groups]
  return iq36::u4_layout_transpose(scale_gm_f16, zp_gm, groups, rows, scale_f16, zp, stream);
}

extern "C" int iq36_u4_layout_to_group_major(const void* scale_f16, const uint8_t* zp,
                                             int32_t rows, int32_t groups, void* scale_gm_f16,
                                             uint8_t* zp_gm, iq36_stream_t stream) {
  return iq36::u4_layout_transpose(scale_f16, zp, rows, groups, scale_gm_f16, zp_gm, stream);
}
