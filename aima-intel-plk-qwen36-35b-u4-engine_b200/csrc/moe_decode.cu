// moe_decode.cu — batch-1 router and routed/shared expert FFN.
//
// Reference semantics: run_qwen36_moe_ffn_layer (engine/src/gguf_loader.cpp:
// 5654-5782) = select_router_topk (:3733-3743) -> gate_up matvec per selected
// expert (:4316) -> apply_swiglu_from_gate_up (:4640-4668) -> down matvec
// (:4467) -> apply_expert_weights (:3773-3797) -> aggregate_experts in rank
// order (:3799-3819) -> + sigmoid(shared gate) * shared expert (:5767-5779).
// The product runs the routed part in OpenVINO moe_3gemm_swiglu_opt
// (engine/openvino/iq36-pr35924-grouped-postops.patch:86-124) and the router /
// shared projections as the router_shared_input FC4 group
// (tools/intel_qwen36_openvino_fixed_fc.py:166-177).
//
// Kernels (all launched with programmatic dependent launch):
//   router_logits  — fp16 [E(+1), H] GEMV, warp per row, fp32 FMA, fixed order;
//   router_select  — warp per token: fp64 softmax, top-k by (prob, -id) 64-bit
//                    keys, fp32 renormalisation in rank order;
//   moe_gate_up    — u4 dot engine; each warp's row A = gate row j, row B =
//                    up row I+j of the same expert, so SwiGLU fuses into the
//                    epilogue; writes act [slots, I] fp16 to the workspace;
//   moe_down       — one CTA per 16 output rows, one warp per expert slot;
//                    the weighted sum over slots runs in rank order in shared
//                    memory (deterministic), shared expert added last.

#include <atomic>

#include "launch.cuh"
#include "sync_sm100.cuh"
#include "u4_core.cuh"

namespace iq36 {

// ---------------------------------------------------------------------------
// Router

// Stage x (fp16, optionally RMS-normalised from fp32) in plain order.
__device__ __forceinline__ void stage_x_plain(__half* xs, const __half* x16, const float* x32,
                                              const float* nw, float eps, int H, float* red) {
  const int tid = threadIdx.x, nt = blockDim.x;
  float scale = 1.0f;
  if (x32 != nullptr) {
    float ss = 0.0f;
    for (int i = tid; i < H; i += nt) ss = fmaf(x32[i], x32[i], ss);
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    if (tid < 32) {
      float v = tid < (nt >> 5) ? red[tid] : 0.0f;
      v = warp_sum(v);
      if (tid == 0) red[32] = rsqrtf(v / (float)H + eps);
    }
    __syncthreads();
    scale = red[32];
    for (int i = tid; i < H; i += nt) xs[i] = __float2half_rn(x32[i] * scale * nw[i]);
  } else {
    for (int i = tid; i < H; i += nt) xs[i] = x16[i];
  }
  __syncthreads();
}

__global__ void __launch_bounds__(256) router_logits_kernel(const __half* x16, const float* x32,
                                                            const float* nw, float eps, int H,
                                                            const __half* W, int E,
                                                            const __half* wsg, float* logits,
                                                            float* slogit) {
  extern __shared__ __align__(16) __half xsh[];
  __shared__ float nred[33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  const __half* wr = nullptr;
  if (row < E) wr = W + (size_t)row * H;
  else if (row == E && wsg != nullptr) wr = wsg;
  // Router weights do not depend on the previous kernel: fetch the first
  // 8 x 16 bytes of this lane's row before waiting on it.
  constexpr int kPre = 8;
  uint4 pre[kPre];
  if (wr != nullptr) {
#pragma unroll
    for (int j = 0; j < kPre; ++j) {
      const int c = lane + 32 * j;
      if (c < H / 8) pre[j] = ld_stream_v4(wr + c * 8);
    }
  }
  pdl_wait();
  const int tok = blockIdx.y;
  stage_x_plain(xsh, x16 ? x16 + (size_t)tok * H : nullptr, x32 ? x32 + (size_t)tok * H : nullptr,
                nw, eps, H, nred);
  pdl_launch_dependents();
  float acc = 0.f;
  const uint4* xv4 = reinterpret_cast<const uint4*>(xsh);
  auto dot8 = [&](const uint4& wv, const uint4& xv) {
    const __half2* wh = reinterpret_cast<const __half2*>(&wv);
    const __half2* xh = reinterpret_cast<const __half2*>(&xv);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 wf = __half22float2(wh[j]);
      const float2 xf = __half22float2(xh[j]);
      acc = fmaf(wf.x, xf.x, acc);
      acc = fmaf(wf.y, xf.y, acc);
    }
  };
  if (wr != nullptr) {
#pragma unroll
    for (int j = 0; j < kPre; ++j) {
      const int c = lane + 32 * j;
      if (c < H / 8) dot8(pre[j], xv4[c]);
    }
    for (int c = lane + 32 * kPre; c < H / 8; c += 32) dot8(ld_stream_v4(wr + c * 8), xv4[c]);
    acc = warp_sum(acc);
    if (lane == 0) {
      if (row < E) logits[(size_t)tok * E + row] = acc;
      else slogit[tok] = acc;
    }
  }
}

// ---------------------------------------------------------------------------
// The prompt path's router input: the decode router's normalised fp16 input,
// bit for bit, for T tokens at once.

// xn[t] = fp16(x[t] * rsqrt(mean(x[t]^2) + eps) * nw), one 256-thread CTA per
// token with stage_x_plain's own reduction (thread j sums x[j + 256m]^2 in
// order, warp butterflies, then the 8 warp sums butterflied by one warp), so
// the result equals the decode router's normalised input bit for bit. Each
// load and store instruction covers 1 KB / 512 B of one row (the former
// warp-per-token form, 64 scalar loads per lane, cost 23 us more per layer
// at 4096 tokens).
__global__ void __launch_bounds__(256) x_norm_plain_kernel(const float* x32, const float* nw,
                                                           float eps, int T, int H,
                                                           __half* xn) {
  __shared__ float red[33];
  pdl_wait();
  const int t = blockIdx.x, tid = threadIdx.x;
  const float* x = x32 + (size_t)t * H;
  constexpr int kM = 8;  // H <= 2048: x[tid + 256 m]
  float xv[kM];
#pragma unroll
  for (int m = 0; m < kM; ++m) xv[m] = tid + 256 * m < H ? x[tid + 256 * m] : 0.f;
  float ss = 0.0f;
#pragma unroll
  for (int m = 0; m < kM; ++m)
    if (tid + 256 * m < H) ss = fmaf(xv[m], xv[m], ss);
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  if (tid < 32) {
    float v = tid < 8 ? red[tid] : 0.0f;
    v = warp_sum(v);
    if (tid == 0) red[32] = rsqrtf(v / (float)H + eps);
  }
  __syncthreads();
  const float scale = red[32];
  __half* o = xn + (size_t)t * H;
#pragma unroll
  for (int m = 0; m < kM; ++m)
    if (tid + 256 * m < H) o[tid + 256 * m] = __float2half_rn(xv[m] * scale * nw[tid + 256 * m]);
  pdl_launch_dependents();
}

// Top-k of one token's E router logits by one warp (E <= 256: 8 logits per
// lane; k <= 16). Every lane ends with the same sel_id / sel_w (rank order).
__device__ __forceinline__ void router_topk_warp(const float* l, int E, int k, uint32_t* sel_id,
                                                 float* sel_w) {
  const int lane = threadIdx.x & 31;
  const int per = (E + 31) / 32;
  float lv[8];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int idx = lane + 32 * i;
    lv[i] = (i < per && idx < E) ? l[idx] : -INFINITY;
    mx = fmaxf(mx, lv[i]);
  }
  mx = warp_max(mx);
  // softmax (gguf_loader.cpp:3646-3670): fp64 exp(l - max), fp64 sum,
  // probabilities rounded to fp32.
  double ev[8];
  double s = 0.0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int idx = lane + 32 * i;
    ev[i] = (i < per && idx < E) ? exp((double)lv[i] - (double)mx) : 0.0;
    s += ev[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  uint64_t key[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int idx = lane + 32 * i;
    const float p = (float)(ev[i] / s);
    key[i] = (i < per && idx < E)
                 ? (((uint64_t)__float_as_uint(p) << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)idx))
                 : 0ull;
  }
  // top_k_indices (:3672-3697): descending probability, lower id on ties —
  // the larger 64-bit key (prob bits, inverted id) wins.
  // ranks unrolled to the maximum k (16) and predicated, so that sel_id /
  // sel_w stay in registers (a runtime-bounded loop put them in local memory)
  float sum = 0.0f;
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    if (r >= k) break;  // warp-uniform
    uint64_t best = 0ull;
#pragma unroll
    for (int i = 0; i < 8; ++i) best = key[i] > best ? key[i] : best;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (key[i] == best) key[i] = 0ull;
    sel_id[r] = 0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFu);
    sel_w[r] = __uint_as_float((uint32_t)(best >> 32));
    sum = __fadd_rn(sum, sel_w[r]);
  }
  // normalize_weights (:3712-3731), min sum 6.103515625e-5 (:5665).
  const float den = fmaxf(sum, 6.103515625e-5f);
#pragma unroll
  for (int r = 0; r < 16; ++r)
    if (r < k) sel_w[r] = __fdiv_rn(sel_w[r], den);
}

// Warp per token. E <= 256, k <= 16.
__global__ void __launch_bounds__(256) router_select_kernel(const float* logits, int T, int E,
                                                            int k, int32_t* ids, float* weights) {
  // the expert kernel that follows may launch now: before its wait it only
  // prefetches the shared expert's weights
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int tok = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (tok >= T) return;
  uint32_t sel_id[16];
  float sel_w[16];
  router_topk_warp(logits + (size_t)tok * E, E, k, sel_id, sel_w);
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      if (r < k) {
        ids[(size_t)tok * k + r] = (int32_t)sel_id[r];
        weights[(size_t)tok * k + r] = sel_w[r];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Experts

struct ExpertArgs {
  const uint8_t* gu_w;
  const __half* gu_s;
  const uint8_t* gu_z;
  const uint8_t* d_w;
  const __half* d_s;
  const uint8_t* d_z;
  const uint8_t* sgu_w;
  const __half* sgu_s;
  const uint8_t* sgu_z;
  const uint8_t* sd_w;
  const __half* sd_s;
  const uint8_t* sd_z;
  int H, I, k, n_slots, num_experts;
  int e_lo;  // global id of the bank's expert 0 (expert-sharded decode)
};

// Local index of the expert routed to `slot`, or -1 when the bank does not
// hold it (another rank owns it, or the id is out of range): such slots read
// no weights and contribute zero.
__device__ __forceinline__ int owned_expert(const ExpertArgs& a, const int32_t* ids, int slot) {
  const int e = ids[slot] - a.e_lo;
  return (e >= 0 && e < a.num_experts) ? e : -1;
}

// Row pair (gate row j, up row I+j) of one gate_up warp task.
template <int G>
__device__ __forceinline__ U4Rows gate_up_rows(const ExpertArgs& a, const int32_t* ids, int slot,
                                               int j, int g) {
  const int H = a.H, I = a.I, ng = H / G;
  const uint8_t* w;
  const __half* s;
  const uint8_t* z;
  int64_t zbase;
  if (slot < a.k) {
    const int64_t e = max(owned_expert(a, ids, slot), 0);
    w = a.gu_w + e * (int64_t)(2 * I) * (H / 2);
    s = a.gu_s + e * (int64_t)(2 * I) * ng;
    z = a.gu_z;
    zbase = e * (int64_t)(2 * I) * ng;
  } else {
    w = a.sgu_w;
    s = a.sgu_s;
    z = a.sgu_z;
    zbase = 0;
  }
  const int rowA = j + g, rowB = I + j + g;
  return U4Rows{w + (size_t)rowA * (H / 2), w + (size_t)rowB * (H / 2), s + (size_t)rowA * ng,
                s + (size_t)rowB * ng, z, zbase + (int64_t)rowA * ng, zbase + (int64_t)rowB * ng};
}

// ONE: every warp's group range fits one 4-group chunk, loaded at once (one
// memory round trip); otherwise 2-group chunks, software-pipelined. Both
// accumulate the groups in the same order.
template <int G, bool ONE>
__global__ void __launch_bounds__(256) moe_gate_up_kernel(ExpertArgs a, const int32_t* ids,
                                                          const __half* x16, const float* x32,
                                                          const float* nw, float eps,
                                                          __half* act, int ks_log2) {
  extern __shared__ uint4 xs[];
  __shared__ float red[8][16];
  __shared__ float nred[33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int KS = 1 << ks_log2;
  const int rb = blockIdx.x * (8 >> ks_log2) + (warp >> ks_log2);
  const int ks = warp & (KS - 1);
  const int rb_per_exp = a.I / 8;
  const int I = a.I, ng = a.H / G, per = ng >> ks_log2;
  const bool valid = rb < a.n_slots * rb_per_exp;
  const int slot = valid ? rb / rb_per_exp : 0;
  const int j0 = (rb - slot * rb_per_exp) * 8;
  float accA = 0.f, accB = 0.f;
  U4Rows rows{};
  constexpr int U = ONE ? 4 : 2;
  U4Chunk<G, U> first;
  // The shared expert's weights are known up front: stream them before the
  // wait. Routed experts depend on the router output of the previous kernel.
  if (valid && slot >= a.k) {
    rows = gate_up_rows<G>(a, ids, slot, j0, g);
    u4_load_chunk<G, U>(first, rows, ks * per, (ks + 1) * per, t);
  }
  pdl_wait();
  const bool work = valid && (slot >= a.k || owned_expert(a, ids, slot) >= 0);
  if (work && slot < a.k) {
    rows = gate_up_rows<G>(a, ids, slot, j0, g);
    u4_load_chunk<G, U>(first, rows, ks * per, (ks + 1) * per, t);
  }
  stage_x_perm(xs, x16, x32, nw, eps, a.H, nred);
  pdl_launch_dependents();
  if (work) {
    if constexpr (ONE)
      u4_compute_chunk<G, U>(first, xs, ks * per, (ks + 1) * per, t, accA, accB);
    else
      u4_dot2_pipelined<G, U>(first, rows, xs, ks * per, (ks + 1) * per, t, accA, accB);
  }
  if (KS > 1) {
    if (t == 0) {
      red[warp][g] = accA;
      red[warp][g + 8] = accB;
    }
    __syncthreads();
    if (ks == 0) {
      accA = 0.f;
      accB = 0.f;
      for (int j = 0; j < KS; ++j) {
        accA += red[warp + j][g];
        accB += red[warp + j][g + 8];
      }
    }
  }
  if (valid && ks == 0 && t == 0) {
    // SwiGLU: gate * sigmoid(gate) * up, rounded to fp16 (input of the down GEMV).
    const float gate = accA, up = accB;
    act[(size_t)slot * I + j0 + g] = __float2half_rn(gate * sigmoidf_acc(gate) * up);
  }
}

template <int G, bool ONE>
__global__ void moe_down_kernel(ExpertArgs a, const int32_t* ids, const float* wts,
                                const float* slogit, const __half* act, void* out, int out_dtype,
                                int accumulate) {
  extern __shared__ uint4 xs[];
  __shared__ float red[16][16];
  __shared__ float nred[33];
  const int H = a.H, I = a.I, ngi = I / G;
  const int slot = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int h0 = blockIdx.x * 16;
  const int rowA = min(h0 + g, H - 1), rowB = min(h0 + g + 8, H - 1);
  // The expert ids were written by the router two launches back (every kernel
  // waits on its predecessor before releasing its dependents), so they, and
  // the expert weights they select, can be read before this kernel's wait.
  const uint8_t* w;
  const __half* s;
  const uint8_t* z;
  int64_t zbase;
  const int owned = slot < a.k ? owned_expert(a, ids, slot) : 0;
  if (slot < a.k) {
    const int64_t e = max(owned, 0);
    w = a.d_w + e * (int64_t)H * (I / 2);
    s = a.d_s + e * (int64_t)H * ngi;
    z = a.d_z;
    zbase = e * (int64_t)H * ngi;
  } else {
    w = a.sd_w;
    s = a.sd_s;
    z = a.sd_z;
    zbase = 0;
  }
  const U4Rows rows{w + (size_t)rowA * (I / 2), w + (size_t)rowB * (I / 2),
                    s + (size_t)rowA * ngi, s + (size_t)rowB * ngi, z,
                    zbase + (int64_t)rowA * ngi, zbase + (int64_t)rowB * ngi};
  constexpr int U = ONE ? 4 : 2;
  U4Chunk<G, U> first;
  if (owned >= 0) u4_load_chunk<G, U>(first, rows, 0, ngi, t);
  pdl_wait();
  stage_x_perm(xs, act, nullptr, nullptr, 0.f, a.n_slots * I, nred);
  pdl_launch_dependents();
  float accA = 0.f, accB = 0.f;
  if (owned >= 0) {
    if constexpr (ONE)
      u4_compute_chunk<G, U>(first, xs + (size_t)slot * (I / 8), 0, ngi, t, accA, accB);
    else
      u4_dot2_pipelined<G, U>(first, rows, xs + (size_t)slot * (I / 8), 0, ngi, t, accA, accB);
  }
  if (t == 0) {
    red[slot][g] = accA;
    red[slot][g + 8] = accB;
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    const int r = threadIdx.x, row = h0 + r;
    if (row < H) {
      float y = 0.0f;
      for (int j = 0; j < a.k; ++j) y = __fadd_rn(y, __fmul_rn(red[j][r], wts[j]));
      if (a.n_slots > a.k) y = __fadd_rn(y, __fmul_rn(red[a.k][r], sigmoidf_acc(slogit[0])));
      if (out_dtype == IQ36_F16) {
        reinterpret_cast<__half*>(out)[row] = __float2half_rn(y);
      } else if (accumulate) {
        float* o = reinterpret_cast<float*>(out);
        o[row] = o[row] + __half2float(__float2half_rn(y));
      } else {
        reinterpret_cast<float*>(out)[row] = y;
      }
    }
  }
}

int u4_ks_log2(int total_rb, int ng);

static int check_bank(const iq36_expert_bank* b) {
  if (!b || !b->gate_up_weight || !b->gate_up_scale || !b->gate_up_zp || !b->down_weight ||
      !b->down_scale || !b->down_zp)
    return IQ36_ERR_ARG;
  const int G = b->group, H = b->hidden, I = b->intermediate;
  if (G != 64 && G != 128) return IQ36_ERR_SHAPE;
  if (b->num_experts < 1 || H < G || I < G || H % G || I % G || H % 16 || I % 8 || H > 16384)
    return IQ36_ERR_SHAPE;
  if (!aligned(b->gate_up_weight, 16) || !aligned(b->down_weight, 16)) return IQ36_ERR_ALIGN;
  return IQ36_OK;
}

size_t moe_decode_ws(int k, int hidden, int intermediate) {
  (void)hidden;
  return (((size_t)(k + 1) * intermediate * 2) + 255) / 256 * 256;
}

// Layer workspace: the SwiGLU activations [k+1, I] fp16, then 256 bytes
// holding the one-launch form's grid-barrier counter (zero before first use).
size_t moe_layer_ws(int k, int hidden, int intermediate) {
  return moe_decode_ws(k, hidden, intermediate) + 256;
}

int moe_decode_launch(const void* x_f16, const float* x_f32, const float* nw, float eps,
                      const int32_t* ids, const float* weights, int k,
                      const iq36_expert_bank* routed, const iq36_expert_bank* shared,
                      const float* shared_logit, void* out, int out_dtype, int accumulate,
                      void* ws, size_t ws_bytes, cudaStream_t stream, int e_lo = 0) {
  int st = check_bank(routed);
  if (st != IQ36_OK) return st;
  if (!ids || !weights || !out) return IQ36_ERR_ARG;
  if (x_f32) {
    if (x_f16 || !nw) return IQ36_ERR_ARG;
  } else {
    if (!x_f16) return IQ36_ERR_ARG;
    if (!aligned(x_f16, 16)) return IQ36_ERR_ALIGN;
  }
  if (k < 1 || k > 15 || e_lo < 0 || (e_lo == 0 && k > routed->num_experts))
    return IQ36_ERR_SHAPE;
  if (out_dtype != IQ36_F32 && out_dtype != IQ36_F16) return IQ36_ERR_ARG;
  if (accumulate && out_dtype != IQ36_F32) return IQ36_ERR_ARG;
  ExpertArgs a = {};
  a.e_lo = e_lo;
  a.gu_w = routed->gate_up_weight;
  a.gu_s = reinterpret_cast<const __half*>(routed->gate_up_scale);
  a.gu_z = routed->gate_up_zp;
  a.d_w = routed->down_weight;
  a.d_s = reinterpret_cast<const __half*>(routed->down_scale);
  a.d_z = routed->down_zp;
  a.H = routed->hidden;
  a.I = routed->intermediate;
  a.k = k;
  a.n_slots = k;
  a.num_experts = routed->num_experts;
  if (shared) {
    st = check_bank(shared);
    if (st != IQ36_OK) return st;
    if (shared->hidden != a.H || shared->intermediate != a.I || shared->group != routed->group)
      return IQ36_ERR_SHAPE;
    if (!shared_logit) return IQ36_ERR_ARG;
    a.sgu_w = shared->gate_up_weight;
    a.sgu_s = reinterpret_cast<const __half*>(shared->gate_up_scale);
    a.sgu_z = shared->gate_up_zp;
    a.sd_w = shared->down_weight;
    a.sd_s = reinterpret_cast<const __half*>(shared->down_scale);
    a.sd_z = shared->down_zp;
    a.n_slots = k + 1;
  }
  if (!ws || ws_bytes < moe_decode_ws(k, a.H, a.I)) return IQ36_ERR_WORKSPACE;
  if (!aligned(ws, 16)) return IQ36_ERR_ALIGN;
  __half* act = reinterpret_cast<__half*>(ws);
  const int G = routed->group;
  const int ng = a.H / G;
  const int total_rb = a.n_slots * (a.I / 8);
  const int ks_log2 = u4_ks_log2(total_rb, ng);
  const dim3 grid1(ceil_div(total_rb, 8 >> ks_log2));
  const size_t smem1 = (size_t)a.H / 8 * sizeof(uint4);
  const __half* xh = reinterpret_cast<const __half*>(x_f16);
  cudaError_t e;
  const bool one1 = (ng >> ks_log2) <= 4;
  if (G == 128)
    e = one1 ? launch(moe_gate_up_kernel<128, true>, grid1, dim3(256), smem1, stream, a, ids, xh,
                      x_f32, nw, eps, act, ks_log2)
             : launch(moe_gate_up_kernel<128, false>, grid1, dim3(256), smem1, stream, a, ids, xh,
                      x_f32, nw, eps, act, ks_log2);
  else
    e = one1 ? launch(moe_gate_up_kernel<64, true>, grid1, dim3(256), smem1, stream, a, ids, xh,
                      x_f32, nw, eps, act, ks_log2)
             : launch(moe_gate_up_kernel<64, false>, grid1, dim3(256), smem1, stream, a, ids, xh,
                      x_f32, nw, eps, act, ks_log2);
  if (e != cudaSuccess) return IQ36_ERR_CUDA;
  const dim3 grid2(ceil_div(a.H, 16));
  const size_t smem2 = (size_t)a.n_slots * a.I / 8 * sizeof(uint4);
  const __half* acth = act;
  const bool one2 = a.I / G <= 4;
  if (G == 128)
    e = one2 ? launch(moe_down_kernel<128, true>, grid2, dim3(32 * a.n_slots), smem2, stream, a,
                      ids, weights, shared_logit, acth, out, out_dtype, accumulate)
             : launch(moe_down_kernel<128, false>, grid2, dim3(32 * a.n_slots), smem2, stream, a,
                      ids, weights, shared_logit, acth, out, out_dtype, accumulate);
  else
    e = one2 ? launch(moe_down_kernel<64, true>, grid2, dim3(32 * a.n_slots), smem2, stream, a,
                      ids, weights, shared_logit, acth, out, out_dtype, accumulate)
             : launch(moe_down_kernel<64, false>, grid2, dim3(32 * a.n_slots), smem2, stream, a,
                      ids, weights, shared_logit, acth, out, out_dtype, accumulate);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// The decode MoE FFN layer as ONE persistent launch (iq36_moe_layer_decode).
//
// One CTA of 16 warps per SM runs the layer's four dependent steps as three
// phases separated by two grid barriers:
//   A  x = f16(RMSNorm(residual)); the router logits, one warp per row, rows
//      spread over the CTAs; the shared expert's gate_up + SwiGLU, whose
//      weights (and its down rows) were fetched before griddepcontrol.wait;
//   -- barrier 1: every logit written --
//   B  every CTA selects the top-k from the logits itself (no broadcast step),
//      starts the bulk copies of its 16 down-projection rows of the k selected
//      experts into shared memory, then runs its gate_up units of those
//      experts (unit = 8 gate rows + the matching 8 up rows, K split over the
//      4 warps of a quad);
//   -- barrier 2: every SwiGLU activation written --
//   C  CTAs with a down row block: the k+1 slots' dot products from the copies
//      already in shared memory, rank-order combine, residual update.
// CTAs without a row block arrive at barrier 2 and exit, so the next kernel
// (released once every CTA is past barrier 2) starts streaming its weights on
// their SMs while phase C runs.
//
// Reduction orders, dot engine and rounding points are those of the
// four-launch form (router_logits_kernel, router_topk_warp,
// moe_gate_up_kernel<128, true> with a 4-way K split, moe_down_kernel<128,
// true>), so both forms produce the same bits.
//
// Grid barrier: one 64-bit arrival counter in the caller's workspace (zero
// before first use). It only grows: every launch adds exactly 2 x gridDim
// arrivals, so after its griddepcontrol.wait (the previous launch sharing the
// workspace has completed) a CTA reads the counter and rounds it down to a
// multiple of gridDim — fewer than gridDim arrivals of this launch can
// precede that read — to get the launch's base; barrier j is passed when the
// counter reaches base + j * gridDim. An arrival is one fire-and-forget
// red.release after the CTA's bar.sync (release is cumulative over the
// writes that bar.sync ordered before it); waiters poll with ld.acquire.
// Waits are bounded (kWaitLimitNs): on expiry the CTA counts a timeout
// (iq36_wait_timeouts) and skips the rest of its work.

constexpr int kLayerThreads = 512;  // 16 warps = 4 gate_up quads
constexpr int kLayerQuads = kLayerThreads / 128;

__device__ int g_moe_wait_timeouts;

struct LayerArgs {
  ExpertArgs e;
  float* residual;
  const float* nw;
  float eps;
  const __half* w_router;
  const __half* w_sg;  // shared-expert gate row (nullptr without a shared expert)
  int E;
  float* logits;
  float* slogit;
  int32_t* ids_out;
  float* wts_out;
  __half* act;               // [n_slots, I] SwiGLU activations (workspace)
  unsigned long long* bar;   // grid-barrier arrival counter (workspace)
  float* partial_out;        // tensor-parallel rank: fp32 share of the output, residual read-only
};

struct LayerSmem {
  int xplain, xperm, act, logit, stage, slot_bytes, total;
};

__host__ __device__ inline LayerSmem layer_smem(int H, int I, int n_slots) {
  LayerSmem s;
  const int ngi = I / 128;
  s.xplain = 0;
  s.xperm = s.xplain + H * 2;
  s.act = s.xperm + H * 2;
  s.logit = s.act + n_slots * I * 2;
  s.stage = (s.logit + 256 * 4 + 127) / 128 * 128;
  // 16 rows per slot: codes [16][I/2] (one bulk copy), scales [16][ngi],
  // zero points [16*ngi/2]
  s.slot_bytes = 8 * I + 40 * ngi;
  s.total = s.stage + n_slots * s.slot_bytes;
  return s;
}

__host__ __device__ inline int down_pitch(int I) { return I / 2; }

__device__ __forceinline__ uint64_t ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void layer_bar_arrive(unsigned long long* bar) {
  asm volatile("red.release.gpu.global.add.u64 [%0], 1;\n" ::"l"(bar) : "memory");
}

__device__ __forceinline__ bool layer_bar_wait(const unsigned long long* bar,
                                               unsigned long long target) {
  uint64_t t0 = 0;
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (ld_acquire_u64(bar) >= target) return true;
    if (i == 0) t0 = globaltimer_ns();
    else if ((i & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
  return false;
}

// Top-k of the E <= 256 router logits in shared memory by the whole CTA, with
// exactly the arithmetic of router_topk_warp: max, fp64 exp(l - max), the fp64
// sum in that function's order (lane l adds elements l + 32i for i = 0..7,
// then a butterfly over the lanes), probabilities rounded to fp32, the k
// largest (probability bits, inverted id) keys in order, fp32 renormalisation
// in rank order. The exponentials and divisions run one element per thread;
// for k <= 8 the selection ranks a small candidate set in parallel, otherwise
// warp 0 selects with two redux.sync rounds per rank. Ends with sel_id /
// sel_w in shared memory and a __syncthreads.
__device__ __forceinline__ void router_topk_cta(const float* l, int E, int k, double* ev,
                                                uint64_t* key, float* red /* >= 80 floats */,
                                                int32_t* sel_id, float* sel_w) {
  uint64_t* ev_scratch = reinterpret_cast<uint64_t*>(ev);  // reused once the keys exist
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < 256) {
    const float v = tid < E ? l[tid] : -INFINITY;
    const float m = warp_max(v);
    if (lane == 0) red[warp] = m;
  }
  __syncthreads();
  float mx = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
  if (tid < 256) ev[tid] = tid < E ? exp((double)l[tid] - (double)mx) : 0.0;
  __syncthreads();
  // lane l's butterfly result divides the elements l + 32i, as in
  // router_topk_warp (the lanes' sums may differ in the last bit)
  double* lane_sum = reinterpret_cast<double*>(red) + 8;
  if (warp == 0) {
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += ev[lane + 32 * i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    lane_sum[lane] = s;
  }
  __syncthreads();
  if (tid < 256) {
    const double s = lane_sum[tid & 31];
    const float p = (float)(ev[tid] / s);
    key[tid] = tid < E ? (((uint64_t)__float_as_uint(p) << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)tid))
                       : 0ull;
  }
  __syncthreads();
  if (k <= 8) {
    // Candidates: the smallest of the 8 per-warp maximum keys bounds the k-th
    // largest key from below (8 distinct keys reach it), so the top k are
    // among the keys at or above it — usually a few more than k. Each
    // candidate counts the candidates above it: that count is its rank.
    uint64_t* wmax = reinterpret_cast<uint64_t*>(red) + 24;  // [8]
    int* ncand = reinterpret_cast<int*>(red) + 64;
    uint64_t* cand = ev_scratch;
    if (tid < 256) {
      const uint64_t my = key[tid];
      const uint32_t hi = __reduce_max_sync(0xffffffffu, (uint32_t)(my >> 32));
      const uint32_t lo =
          __reduce_max_sync(0xffffffffu, (uint32_t)(my >> 32) == hi ? (uint32_t)my : 0u);
      if (lane == 0) wmax[warp] = ((uint64_t)hi << 32) | lo;
    }
    if (tid == 0) *ncand = 0;
    __syncthreads();
    if (tid < 256) {
      uint64_t th = wmax[0];
#pragma unroll
      for (int w = 1; w < 8; ++w) th = wmax[w] < th ? wmax[w] : th;
      const uint64_t my = key[tid];
      if (my >= th && my != 0ull) cand[atomicAdd(ncand, 1)] = my;
    }
    __syncthreads();
    const int n = *ncand;
    if (tid < n) {
      const uint64_t my = cand[tid];
      int r = 0;
      for (int j = 0; j < n; ++j) r += cand[j] > my;
      if (r < k) {
        sel_id[r] = (int32_t)(0xFFFFFFFFu - (uint32_t)my);
        sel_w[r] = __uint_as_float((uint32_t)(my >> 32));
      }
    }
    __syncthreads();
    if (warp == 0) {
      float sum = 0.0f;
      for (int r = 0; r < k; ++r) sum = __fadd_rn(sum, sel_w[r]);
      const float den = fmaxf(sum, 6.103515625e-5f);
      const float w = lane < k ? __fdiv_rn(sel_w[lane], den) : 0.f;
      __syncwarp();
      if (lane < k) sel_w[lane] = w;
    }
  } else if (warp == 0) {
    uint64_t kk[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) kk[i] = key[lane + 32 * i];
    float sum = 0.0f;
    for (int r = 0; r < k; ++r) {
      uint64_t best = 0ull;
#pragma unroll
      for (int i = 0; i < 8; ++i) best = kk[i] > best ? kk[i] : best;
      const uint32_t hi = __reduce_max_sync(0xffffffffu, (uint32_t)(best >> 32));
      const uint32_t lo =
          __reduce_max_sync(0xffffffffu, (uint32_t)(best >> 32) == hi ? (uint32_t)best : 0u);
      const uint64_t win = ((uint64_t)hi << 32) | lo;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (kk[i] == win) kk[i] = 0ull;
      const float p = __uint_as_float(hi);
      if (lane == 0) {
        sel_id[r] = (int32_t)(0xFFFFFFFFu - lo);
        sel_w[r] = p;
      }
      sum = __fadd_rn(sum, p);
    }
    const float den = fmaxf(sum, 6.103515625e-5f);
    __syncwarp();
    if (lane < k) sel_w[lane] = __fdiv_rn(sel_w[lane], den);
  }
  __syncthreads();
}

// Eight fp16 values into the permuted operand order of u4_core.cuh (odd
// positions pre-divided by 16), as stage_x_perm writes them.
__device__ __forceinline__ uint4 perm8(const __half h[8]) {
  const __half2 sixteenth = __float2half2_rn(0.0625f);
  __half2 p0 = __halves2half2(h[0], h[4]);
  __half2 p1 = __hmul2(__halves2half2(h[1], h[5]), sixteenth);
  __half2 p2 = __halves2half2(h[2], h[6]);
  __half2 p3 = __hmul2(__halves2half2(h[3], h[7]), sixteenth);
  uint4 o;
  o.x = *reinterpret_cast<uint32_t*>(&p0);
  o.y = *reinterpret_cast<uint32_t*>(&p1);
  o.z = *reinterpret_cast<uint32_t*>(&p2);
  o.w = *reinterpret_cast<uint32_t*>(&p3);
  return o;
}

// Rows g and g+8 of a 16-row down block held in shared memory (codes
// [16][I/2], scales [16][ngi], zero points [16*ngi/2]) into a register chunk,
// as u4_load_chunk<128, 4> loads them from global memory.
__device__ __forceinline__ void load_chunk_smem(U4Chunk<128, 4>& c, const uint8_t* st, int I,
                                                int ngi, int g, int t) {
  const int pitch = down_pitch(I);
  const __half* sc = reinterpret_cast<const __half*>(st + 16 * pitch);
  const uint8_t* zp = st + 16 * pitch + 32 * ngi;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int gi = min(u, ngi - 1);
    const uint4 va = *reinterpret_cast<const uint4*>(st + g * pitch + gi * 64 + t * 16);
    const uint4 vb = *reinterpret_cast<const uint4*>(st + (g + 8) * pitch + gi * 64 + t * 16);
    c.ra[u][0] = va.x; c.ra[u][1] = va.y; c.ra[u][2] = va.z; c.ra[u][3] = va.w;
    c.rb[u][0] = vb.x; c.rb[u][1] = vb.y; c.rb[u][2] = vb.z; c.rb[u][3] = vb.w;
    const int ea = g * ngi + gi, eb = (g + 8) * ngi + gi;
    c.sa[u] = __half2float(sc[ea]);
    c.sb[u] = __half2float(sc[eb]);
    c.za[u] = (uint32_t)(zp[ea >> 1] >> ((ea & 1) * 4)) & 15u;
    c.zb[u] = (uint32_t)(zp[eb >> 1] >> ((eb & 1) * 4)) & 15u;
  }
}

// Rows h0..h0+15 of one expert's down matrix into a slot stage: the codes
// (16 x I/2 contiguous bytes) as one bulk copy completing on `bar` (issued by
// the calling lane), the scales and zero points (2*ngi + ngi/2 16-byte
// pieces) as cp.async pieces spread over the calling warp's lanes. Bulk
// copies take no load/store-unit requests, which the gate_up loads saturate.
__device__ __forceinline__ void down_codes_bulk(const uint8_t* w, int64_t e, int H, int I, int h0,
                                                uint32_t dst, uint32_t bar) {
  bulk_load(dst, w + (e * H + h0) * (I / 2), 8 * I, bar);
}
__device__ __forceinline__ void down_meta_async(const __half* s, const uint8_t* z, int64_t e,
                                                int H, int I, int h0, uint8_t* dst, int piece) {
  const int ngi = I / 128;
  const int64_t row = e * H + h0;
  if (piece < 2 * ngi)
    cp_async_16(smem_u32(dst + 8 * I + piece * 16),
                reinterpret_cast<const uint8_t*>(s + row * ngi) + piece * 16, 16);
  else if (piece < 2 * ngi + ngi / 2)
    cp_async_16(smem_u32(dst + 8 * I + 32 * ngi + (piece - 2 * ngi) * 16),
                z + row * ngi / 2 + (piece - 2 * ngi) * 16, 16);
}

// One gate_up quarter-unit into registers, values as u4_load_chunk<128, 4>
// loads them: the lane's codes of gate row rowA0 + g and up row rowB0 + g
// over groups gb..gb+3 directly, while the 16 rows' scales (one 8-byte load
// per row) and zero points (one 2-byte load per row) are fetched by lanes
// 0..15 and handed to the lane groups by shuffles: 10 load requests per lane
// instead of 24. quarter_issue only issues the loads (nothing waits on
// them); quarter_finish does the shuffles, so it is called where the values
// are about to be used.
struct QuarterRaw {
  uint2 sc;
  uint32_t zz;
};

__device__ __forceinline__ void quarter_issue(U4Chunk<128, 4>& c, QuarterRaw& q, const uint8_t* w,
                                              const __half* s, const uint8_t* z, int64_t zbase,
                                              int rowA0, int rowB0, int H, int gb, int lane) {
  const int g = lane >> 2, t = lane & 3, ng = H / 128;
  const uint8_t* wA = w + (size_t)(rowA0 + g) * (H / 2) + t * 16;
  const uint8_t* wB = w + (size_t)(rowB0 + g) * (H / 2) + t * 16;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const uint4 va = ld_stream_v4(wA + (gb + u) * 64);
    const uint4 vb = ld_stream_v4(wB + (gb + u) * 64);
    c.ra[u][0] = va.x; c.ra[u][1] = va.y; c.ra[u][2] = va.z; c.ra[u][3] = va.w;
    c.rb[u][0] = vb.x; c.rb[u][1] = vb.y; c.rb[u][2] = vb.z; c.rb[u][3] = vb.w;
  }
  q.sc = make_uint2(0u, 0u);
  q.zz = 0u;
  if (lane < 16) {
    const int row = lane < 8 ? rowA0 + lane : rowB0 + lane - 8;
    q.sc = ld_stream_v2(s + (size_t)row * ng + gb);
    const int64_t e0 = zbase + (int64_t)row * ng + gb;  // multiple of 4: 4 nibbles in 2 bytes
    q.zz = (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(z + (e0 >> 1)));
  }
}

__device__ __forceinline__ void quarter_finish(U4Chunk<128, 4>& c, const QuarterRaw& q, int lane) {
  const int g = lane >> 2;
  const uint32_t sAx = __shfl_sync(0xffffffffu, q.sc.x, g), sAy = __shfl_sync(0xffffffffu, q.sc.y, g);
  const uint32_t sBx = __shfl_sync(0xffffffffu, q.sc.x, g + 8),
                 sBy = __shfl_sync(0xffffffffu, q.sc.y, g + 8);
  const uint32_t zA = __shfl_sync(0xffffffffu, q.zz, g), zB = __shfl_sync(0xffffffffu, q.zz, g + 8);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const uint32_t wa = u < 2 ? sAx : sAy, wb = u < 2 ? sBx : sBy;
    c.sa[u] = __half2float(__ushort_as_half((unsigned short)(wa >> (16 * (u & 1)))));
    c.sb[u] = __half2float(__ushort_as_half((unsigned short)(wb >> (16 * (u & 1)))));
    c.za[u] = (zA >> (4 * u)) & 15u;
    c.zb[u] = (zB >> (4 * u)) & 15u;
  }
}

__global__ void __launch_bounds__(kLayerThreads, 1) moe_layer_kernel(LayerArgs a) {
  extern __shared__ __align__(128) uint8_t lsm[];
  __shared__ float red[16][16];
  __shared__ __align__(8) float nred[80];
  __shared__ double s_ev[256];
  __shared__ uint64_t s_key[256];
  __shared__ int32_t s_ids[16];
  __shared__ float s_wts[16];
  __shared__ __align__(8) uint64_t mbar[2];  // down codes: 0 shared slot, 1 routed slots
  __shared__ int s_ok;
  __shared__ unsigned long long s_base;
  __shared__ float s_res[16];  // this CTA's residual rows h0..h0+15 (phase C)
  const ExpertArgs& e = a.e;
  const int H = e.H, I = e.I, ngi = I / 128, k = e.k, n_slots = e.n_slots;
  const int ng = H / 128;
  const LayerSmem L = layer_smem(H, I, n_slots);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int cta = blockIdx.x, nb = gridDim.x;
  const int quad = warp >> 2, ks = warp & 3;
  const int ups = I / 8;  // gate_up units per slot
  const int n_routed_units = k * ups, n_units = n_slots * ups;
  const int unit = cta + quad * nb;  // host: kLayerQuads * nb >= n_units
  const bool has_unit = unit < n_units;
  const bool shared_unit = has_unit && unit >= n_routed_units;
  const int uslot = has_unit ? unit / ups : 0;
  const int j0 = (unit % ups) * 8;
  const int drb = nb - 1 - cta;  // down row block (the last H/16 CTAs)
  const bool has_down = drb < H / 16;
  const bool shared_down = has_down && n_slots > k;
  const int h0 = drb * 16;
  const int n_rows = a.E + (a.w_sg != nullptr ? 1 : 0);
  const int rrow = cta + warp * nb;  // router row of this warp
  const bool has_row = rrow < n_rows;
  const int meta = 2 * ngi + ngi / 2;  // 16-byte scale / zero-point pieces per slot
  const uint32_t bar_s = smem_u32(&mbar[0]), bar_r = smem_u32(&mbar[1]);
  uint8_t* stage = lsm + L.stage;
  constexpr int kRes = 8;  // residual values per thread (threads < 256; H <= 2048)

  // ---- prologue: weights only (nothing here depends on earlier launches)
  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_r, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  if (warp == k && shared_down) {
    if (lane == 0) {
      mbar_arrive_tx(bar_s, 8 * I);
      down_codes_bulk(e.sd_w, 0, H, I, h0, smem_u32(stage + k * L.slot_bytes), bar_s);
    }
    down_meta_async(e.sd_s, e.sd_z, 0, H, I, h0, stage + k * L.slot_bytes, lane);
    cp_async_commit();
  }
  float nwv[kRes];
  if (tid < 256) {
#pragma unroll
    for (int m = 0; m < kRes; ++m) nwv[m] = tid + 256 * m < H ? a.nw[tid + 256 * m] : 0.f;
  }
  const __half* wr = nullptr;
  if (has_row) wr = rrow < a.E ? a.w_router + (size_t)rrow * H : a.w_sg;
  constexpr int kPre = 8;
  uint4 pre[kPre];
  if (has_row) {
#pragma unroll
    for (int j = 0; j < kPre; ++j) {
      const int c = lane + 32 * j;
      if (c < H / 8) pre[j] = ld_stream_v4(wr + c * 8);
    }
  }
  U4Chunk<128, 4> ch;
  QuarterRaw qr;
  if (shared_unit)
    quarter_issue(ch, qr, e.sgu_w, e.sgu_s, e.sgu_z, 0, j0, I + j0, H, ks * 4, lane);
  pdl_wait();

  // ---- phase A: x, router logits, shared expert gate_up
  if (tid == kLayerThreads - 32) {
    // the barrier base, by a thread with no residual loads to delay
    unsigned long long c0;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];\n" : "=l"(c0) : "l"(a.bar) : "memory");
    s_base = c0 / (unsigned long long)nb * nb;
  }
  float resv[kRes];
  {
    // the 256-thread reduction order of stage_x_plain / stage_x_perm
    if (tid < 256) {
      float ss = 0.f;
#pragma unroll
      for (int m = 0; m < kRes; ++m) {
        resv[m] = tid + 256 * m < H ? a.residual[tid + 256 * m] : 0.f;
        if (tid + 256 * m < H) ss = fmaf(resv[m], resv[m], ss);
      }
      ss = warp_sum(ss);
      if (lane == 0) nred[warp] = ss;
      if (has_down) {
#pragma unroll
        for (int m = 0; m < kRes; ++m) {
          const int i = tid + 256 * m;
          if (i >= h0 && i < h0 + 16) s_res[i - h0] = resv[m];
        }
      }
    }
    __syncthreads();
    // every warp sums the 8 warp totals as warp 0 of the 256-thread kernels
    // did, and takes lane 0's butterfly result (the value those kernels used)
    float v = lane < 8 ? nred[lane] : 0.f;
    v = __shfl_sync(0xffffffffu, warp_sum(v), 0);
    const float scale = rsqrtf(v / (float)H + a.eps);
    // each value straight into both layouts: plain, and the permuted operand
    // order of perm8 (element j of chunk c at half 2(j%4) + j/4, odd j / 16)
    __half* xp = reinterpret_cast<__half*>(lsm + L.xplain);
    __half* xq = reinterpret_cast<__half*>(lsm + L.xperm);
    const __half sixteenth = __float2half_rn(0.0625f);
    if (tid < 256) {
#pragma unroll
      for (int m = 0; m < kRes; ++m) {
        const int i = tid + 256 * m;
        if (i < H) {
          const __half hv = __float2half_rn(resv[m] * scale * nwv[m]);
          const int j = i & 7;
          xp[i] = hv;
          xq[(i & ~7) + 2 * (j & 3) + (j >> 2)] = (j & 1) ? __hmul(hv, sixteenth) : hv;
        }
      }
    }
    __syncthreads();
  }
  if (has_row) {
    const uint4* xv4 = reinterpret_cast<const uint4*>(lsm + L.xplain);
    float acc = 0.f;
    auto dot8 = [&](const uint4& wv, const uint4& xv) {
      const __half2* wh = reinterpret_cast<const __half2*>(&wv);
      const __half2* xh = reinterpret_cast<const __half2*>(&xv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 wf = __half22float2(wh[j]);
        const float2 xf = __half22float2(xh[j]);
        acc = fmaf(wf.x, xf.x, acc);
        acc = fmaf(wf.y, xf.y, acc);
      }
    };
#pragma unroll
    for (int j = 0; j < kPre; ++j) {
      const int c = lane + 32 * j;
      if (c < H / 8) dot8(pre[j], xv4[c]);
    }
    for (int c = lane + 32 * kPre; c < H / 8; c += 32) dot8(ld_stream_v4(wr + c * 8), xv4[c]);
    acc = warp_sum(acc);
    if (lane == 0) {
      if (rrow < a.E) a.logits[rrow] = acc;
      else a.slogit[0] = acc;
    }
  }
  __syncthreads();  // logits stored
  if (tid == 0) layer_bar_arrive(a.bar);
  const uint4* xs = reinterpret_cast<const uint4*>(lsm + L.xperm);
  float accA = 0.f, accB = 0.f;
  if (shared_unit) {
    quarter_finish(ch, qr, lane);
    u4_compute_chunk<128, 4>(ch, xs, ks * 4, ks * 4 + 4, t, accA, accB);
  }
  if (shared_unit && t == 0) {
    red[warp][g] = accA;
    red[warp][g + 8] = accB;
  }
  if (tid == 0) s_ok = layer_bar_wait(a.bar, s_base + (unsigned long long)nb) ? 1 : 0;
  __syncthreads();
  if (shared_unit && ks == 0 && t == 0) {
    float ga = 0.f, ub = 0.f;
    for (int j = 0; j < 4; ++j) {
      ga += red[warp + j][g];
      ub += red[warp + j][g + 8];
    }
    a.act[(size_t)uslot * I + j0 + g] = __float2half_rn(ga * sigmoidf_acc(ga) * ub);
  }
  if (!s_ok) {
    // leave no copy in flight into this CTA's shared memory
    cp_async_wait<0>();
    if (tid == 0) {
      atomicAdd(&g_moe_wait_timeouts, 1);
      if (shared_down) (void)mbar_wait(bar_s, 0);
    }
    return;
  }

  // ---- phase B: top-k, routed down copies, routed gate_up
  float* sl = reinterpret_cast<float*>(lsm + L.logit);
  if (tid < a.E) sl[tid] = __ldcg(a.logits + tid);
  const float slogit = (n_slots > k && tid == 0) ? __ldcg(a.slogit) : 0.f;
  router_topk_cta(sl, a.E, k, s_ev, s_key, nred, s_ids, s_wts);
  const bool routed_unit = has_unit && !shared_unit;
  if (routed_unit) {
    const int64_t ex = s_ids[uslot];
    quarter_issue(ch, qr, e.gu_w + ex * (2 * I) * (H / 2), e.gu_s + ex * (2 * I) * ng, e.gu_z,
                  ex * (2 * I) * ng, j0, I + j0, H, ks * 4, lane);
  }
  // the down rows are needed only after barrier 2: issued after this warp's
  // own gate_up loads
  if (warp == 0) {
    if (cta == 0 && lane < k) {
      a.ids_out[lane] = s_ids[lane];
      a.wts_out[lane] = s_wts[lane];
    }
    if (has_down) {
      if (lane == 0) mbar_arrive_tx(bar_r, (uint32_t)k * 8 * I);
      __syncwarp();
      if (lane < k)
        down_codes_bulk(e.d_w, (int64_t)s_ids[lane], H, I, h0,
                        smem_u32(stage + lane * L.slot_bytes), bar_r);
      for (int p = lane; p < k * meta; p += 32)
        down_meta_async(e.d_s, e.d_z, (int64_t)s_ids[p / meta], H, I, h0,
                        stage + (p / meta) * L.slot_bytes, p % meta);
      cp_async_commit();
    }
  }
  accA = 0.f;
  accB = 0.f;
  if (routed_unit) {
    quarter_finish(ch, qr, lane);
    u4_compute_chunk<128, 4>(ch, xs, ks * 4, ks * 4 + 4, t, accA, accB);
    if (t == 0) {
      red[warp][g] = accA;
      red[warp][g + 8] = accB;
    }
  }
  __syncthreads();
  if (routed_unit && ks == 0 && t == 0) {
    float ga = 0.f, ub = 0.f;
    for (int j = 0; j < 4; ++j) {
      ga += red[warp + j][g];
      ub += red[warp + j][g + 8];
    }
    a.act[(size_t)uslot * I + j0 + g] = __float2half_rn(ga * sigmoidf_acc(ga) * ub);
  }
  __syncthreads();
  if (tid == 0) layer_bar_arrive(a.bar);
  if (!has_down) return;
  if (tid == 0) s_ok = layer_bar_wait(a.bar, s_base + 2ull * nb) ? 1 : 0;
  __syncthreads();
  if (!s_ok) {
    cp_async_wait<0>();
    if (tid == 0) {
      atomicAdd(&g_moe_wait_timeouts, 1);
      if (shared_down) (void)mbar_wait(bar_s, 0);
      (void)mbar_wait(bar_r, 0);
    }
    return;
  }
  // every CTA is past barrier 2, hence resident: the next kernel may launch
  pdl_launch_dependents();

  // ---- phase C: down projections of this CTA's 16 rows, combine, residual
  uint4* xa = reinterpret_cast<uint4*>(lsm + L.act);
  for (int c = tid; c < n_slots * I / 8; c += kLayerThreads) {
    const uint4 raw = __ldcg(reinterpret_cast<const uint4*>(a.act) + c);
    xa[c] = perm8(reinterpret_cast<const __half*>(&raw));
  }
  cp_async_wait<0>();  // scale / zero-point pieces (warps 0 and k issued them)
  if (tid == 0) nred[33] = slogit;
  __syncthreads();
  if (warp < n_slots) {
    const bool got = mbar_wait(warp < k ? bar_r : bar_s, 0);
    accA = 0.f;
    accB = 0.f;
    if (got) {
      load_chunk_smem(ch, stage + warp * L.slot_bytes, I, ngi, g, t);
      u4_compute_chunk<128, 4>(ch, xa + (size_t)warp * (I / 8), 0, ngi, t, accA, accB);
    } else if (lane == 0) {
      atomicAdd(&g_moe_wait_timeouts, 1);
    }
    if (t == 0) {
      red[warp][g] = accA;
      red[warp][g + 8] = accB;
    }
  }
  __syncthreads();
  if (tid < 16) {
    const int row = h0 + tid;
    float y = 0.0f;
    for (int j = 0; j < k; ++j) y = __fadd_rn(y, __fmul_rn(red[j][tid], s_wts[j]));
    if (n_slots > k) y = __fadd_rn(y, __fmul_rn(red[k][tid], sigmoidf_acc(nred[33])));
    // s_res: this CTA's rows as read in phase A (no CTA writes the residual
    // before barrier 2)
    if (a.partial_out != nullptr) a.partial_out[row] = y;
    else a.residual[row] = s_res[tid] + __half2float(__float2half_rn(y));
  }
}

// Whether the one-launch form covers this layer on `sms` SMs (otherwise the
// four-launch form runs).
static bool layer_fused_ok(const iq36_expert_bank* r, const iq36_expert_bank* s, int k, int E,
                           int sms) {
  const int H = r->hidden, I = r->intermediate;
  const int n_slots = k + (s ? 1 : 0);
  if (r->group != 128 || H % 512 || H > 2048 || I % 256 || I > 512 || E > 256 || k > 15)
    return false;
  if (n_slots * (I / 8) > kLayerQuads * sms || H / 16 > sms || E + 1 > 16 * sms) return false;
  if (!aligned(r->down_scale, 16) || !aligned(r->down_zp, 16) || !aligned(r->gate_up_scale, 8) ||
      !aligned(r->gate_up_zp, 2))
    return false;
  if (s && (!aligned(s->down_weight, 16) || !aligned(s->down_scale, 16) ||
            !aligned(s->down_zp, 16) || !aligned(s->gate_up_scale, 8) ||
            !aligned(s->gate_up_zp, 2)))
    return false;
  return layer_smem(H, I, n_slots).total <= 200 * 1024;
}

static int device_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
  int v = cache[dev].load(std::memory_order_acquire);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    if (cudaFuncSetAttribute(moe_layer_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             200 * 1024) != cudaSuccess)
      return -1;
    cache[dev].store(v, std::memory_order_release);
  }
  return v;
}

int moe_wait_timeouts(int* count, int reset) {
  if (cudaMemcpyFromSymbol(count, g_moe_wait_timeouts, sizeof(int)) != cudaSuccess)
    return IQ36_ERR_CUDA;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_moe_wait_timeouts, &zero, sizeof(int)) != cudaSuccess)
      return IQ36_ERR_CUDA;
  }
  return IQ36_OK;
}

int router_logits_launch(const void* x_f16, const float* x_f32, const float* nw, float eps, int T,
                         int H, const void* w_router, int E, const void* w_sg, float* logits,
                         float* slogit, cudaStream_t stream) {
  if (!w_router || !logits || T < 1 || E < 1 || H < 8 || H % 8) return IQ36_ERR_ARG;
  if (w_sg && !slogit) return IQ36_ERR_ARG;
  if (x_f32) {
    if (x_f16 || !nw) return IQ36_ERR_ARG;
  } else if (!x_f16) {
    return IQ36_ERR_ARG;
  }
  if (!aligned(w_router, 16) || (w_sg && !aligned(w_sg, 16)) || (x_f16 && !aligned(x_f16, 16)))
    return IQ36_ERR_ALIGN;
  const int rows = E + (w_sg ? 1 : 0);
  const dim3 grid(ceil_div(rows, 8), T);
  const cudaError_t e = launch(router_logits_kernel, grid, dim3(256), (size_t)H * 2, stream,
                               reinterpret_cast<const __half*>(x_f16), x_f32, nw, eps, H,
                               reinterpret_cast<const __half*>(w_router), E,
                               reinterpret_cast<const __half*>(w_sg), logits, slogit);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

// xn [T, H] fp16 = the decode router's normalised input (stage_x_plain), bit
// for bit. Requires H % 32 == 0, H <= 2048.
int x_norm_launch(const float* x32, const float* nw, float eps, int T, int H, __half* xn,
                  cudaStream_t stream) {
  if (!x32 || !nw || !xn || T < 1) return IQ36_ERR_ARG;
  if (H < 256 || H % 256 || H > 2048) return IQ36_ERR_SHAPE;
  if (!aligned(xn, 16)) return IQ36_ERR_ALIGN;
  const cudaError_t e = launch(x_norm_plain_kernel, dim3(T), dim3(256), 0, stream,
                               x32, nw, eps, T, H, xn);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

int router_select_launch(const float* logits, int T, int E, int k, int32_t* ids, float* weights,
                         cudaStream_t stream) {
  if (!logits || !ids || !weights) return IQ36_ERR_ARG;
  if (T < 1 || E < 1 || E > 256 || k < 1 || k > 16 || k > E) return IQ36_ERR_SHAPE;
  const cudaError_t e = launch(router_select_kernel, dim3(ceil_div(T, 8)), dim3(256), 0, stream,
                               logits, T, E, k, ids, weights);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

}  // namespace iq36

extern "C" int iq36_router_logits(const void* x_f16, const float* x_f32, const float* norm_weight,
                                  float norm_eps, int32_t T, int32_t H, const void* w_router_f16,
                                  int32_t E, const void* w_shared_gate_f16, float* logits,
                                  float* shared_logit, iq36_stream_t stream) {
  return iq36::router_logits_launch(x_f16, x_f32, norm_weight, norm_eps, T, H, w_router_f16, E,
                                    w_shared_gate_f16, logits, shared_logit,
                                    iq36::as_stream(stream));
}

extern "C" int iq36_router_select(const float* logits, int32_t T, int32_t E, int32_t k,
                                  int32_t* ids, float* weights, iq36_stream_t stream) {
  return iq36::router_select_launch(logits, T, E, k, ids, weights, iq36::as_stream(stream));
}

extern "C" size_t iq36_moe_decode_workspace_bytes(int32_t k, int32_t hidden, int32_t intermediate) {
  return iq36::moe_decode_ws(k, hidden, intermediate);
}

extern "C" int iq36_moe_decode(const void* x_f16, const float* x_f32, const float* norm_weight,
                               float norm_eps, const int32_t* ids, const float* weights,
                               int32_t k, const iq36_expert_bank* routed,
                               const iq36_expert_bank* shared, const float* shared_logit,
                               void* out, int32_t out_dtype, int32_t accumulate, void* workspace,
                               size_t workspace_bytes, iq36_stream_t stream) {
  return iq36::moe_decode_launch(x_f16, x_f32, norm_weight, norm_eps, ids, weights, k, routed,
                                 shared, shared_logit, out, out_dtype, accumulate, workspace,
                                 workspace_bytes, iq36::as_stream(stream));
}

extern "C" int iq36_moe_decode_sharded(const void* x_f16, const float* x_f32,
                                       const float* norm_weight, float norm_eps,
                                       const int32_t* ids, const float* weights, int32_t k,
                                       const iq36_expert_bank* local_bank, int32_t expert_lo,
                                       const iq36_expert_bank* shared, const float* shared_logit,
                                       void* out, int32_t out_dtype, int32_t accumulate,
                                       void* workspace, size_t workspace_bytes,
                                       iq36_stream_t stream) {
  return iq36::moe_decode_launch(x_f16, x_f32, norm_weight, norm_eps, ids, weights, k, local_bank,
                                 shared, shared_logit, out, out_dtype, accumulate, workspace,
                                 workspace_bytes, iq36::as_stream(stream), expert_lo);
}

extern "C" size_t iq36_moe_block_decode_workspace_bytes(int32_t k, int32_t hidden,
                                                        int32_t intermediate) {
  return iq36::moe_decode_ws(k, hidden, intermediate) + 256;
}

extern "C" int iq36_moe_block_decode(const void* x_f16, const void* w_router_f16,
                                     const void* w_shared_gate_f16, int32_t k,
                                     const iq36_expert_bank* routed,
                                     const iq36_expert_bank* shared, int32_t* ids, float* weights,
                                     float* logits, void* out, int32_t out_dtype, void* workspace,
                                     size_t workspace_bytes, iq36_stream_t stream) {
  using namespace iq36;
  if (!routed || !workspace || !x_f16 || !w_router_f16 || !ids || !weights || !logits || !out)
    return IQ36_ERR_ARG;
  if (shared && !w_shared_gate_f16) return IQ36_ERR_ARG;
  // Validate everything before the first launch so a failed call enqueues nothing.
  int st0 = check_bank(routed);
  if (st0 == IQ36_OK && shared) st0 = check_bank(shared);
  if (st0 != IQ36_OK) return st0;
  if (shared && (shared->hidden != routed->hidden || shared->intermediate != routed->intermediate ||
                 shared->group != routed->group))
    return IQ36_ERR_SHAPE;
  if (k < 1 || k > 15 || k > routed->num_experts || routed->num_experts > 256)
    return IQ36_ERR_SHAPE;
  if (out_dtype != IQ36_F32 && out_dtype != IQ36_F16) return IQ36_ERR_ARG;
  if (!aligned(x_f16, 16) || !aligned(w_router_f16, 16) ||
      (shared && !aligned(w_shared_gate_f16, 16)) || !aligned(workspace, 256))
    return IQ36_ERR_ALIGN;
  const size_t need = iq36_moe_block_decode_workspace_bytes(k, routed->hidden, routed->intermediate);
  if (workspace_bytes < need) return IQ36_ERR_WORKSPACE;
  float* slogit = reinterpret_cast<float*>(workspace);
  void* ws2 = reinterpret_cast<char*>(workspace) + 256;
  const cudaStream_t s = as_stream(stream);
  int st = router_logits_launch(x_f16, nullptr, nullptr, 0.f, 1, routed->hidden, w_router_f16,
                                routed->num_experts, shared ? w_shared_gate_f16 : nullptr, logits,
                                slogit, s);
  if (st != IQ36_OK) return st;
  st = router_select_launch(logits, 1, routed->num_experts, k, ids, weights, s);
  if (st != IQ36_OK) return st;
  return moe_decode_launch(x_f16, nullptr, nullptr, 0.f, ids, weights, k, routed, shared,
                           shared ? slogit : nullptr, out, out_dtype, 0, ws2, workspace_bytes - 256,
                           s);
}

namespace iq36 {
// The decode MoE layer: residual += f16(layer output), or, with partial_out,
// partial_out = the fp32 layer output over this bank's rows (residual read).
static int moe_layer_impl(float* residual, int32_t hidden, const float* norm_weight,
                          float norm_eps, const void* w_router_f16, const void* w_shared_gate_f16,
                          int32_t k, const iq36_expert_bank* routed,
                          const iq36_expert_bank* shared, int32_t* ids, float* weights,
                          float* logits, float* shared_logit, float* partial_out, void* workspace,
                          size_t workspace_bytes, iq36_stream_t stream) {
  if (!residual || !norm_weight || !w_router_f16 || !routed || !ids || !weights || !logits ||
      !workspace)
    return IQ36_ERR_ARG;
  if (shared && (!w_shared_gate_f16 || !shared_logit)) return IQ36_ERR_ARG;
  int st0 = check_bank(routed);
  if (st0 == IQ36_OK && shared) st0 = check_bank(shared);
  if (st0 != IQ36_OK) return st0;
  if (hidden != routed->hidden || hidden % 8) return IQ36_ERR_SHAPE;
  if (shared && (shared->hidden != routed->hidden || shared->intermediate != routed->intermediate ||
                 shared->group != routed->group))
    return IQ36_ERR_SHAPE;
  if (k < 1 || k > 15 || k > routed->num_experts || routed->num_experts > 256)
    return IQ36_ERR_SHAPE;
  if (!aligned(w_router_f16, 16) || (shared && !aligned(w_shared_gate_f16, 16)) ||
      !aligned(workspace, 16))
    return IQ36_ERR_ALIGN;
  if (workspace_bytes < moe_layer_ws(k, routed->hidden, routed->intermediate))
    return IQ36_ERR_WORKSPACE;
  const cudaStream_t s = as_stream(stream);
  const int sms = device_sms();
  if (sms < 1) return IQ36_ERR_CUDA;
  if (layer_fused_ok(routed, shared, k, routed->num_experts, sms)) {
    LayerArgs la = {};
    ExpertArgs& a = la.e;
    a.gu_w = routed->gate_up_weight;
    a.gu_s = reinterpret_cast<const __half*>(routed->gate_up_scale);
    a.gu_z = routed->gate_up_zp;
    a.d_w = routed->down_weight;
    a.d_s = reinterpret_cast<const __half*>(routed->down_scale);
    a.d_z = routed->down_zp;
    a.H = hidden;
    a.I = routed->intermediate;
    a.k = k;
    a.n_slots = k;
    a.num_experts = routed->num_experts;
    a.e_lo = 0;
    if (shared) {
      a.sgu_w = shared->gate_up_weight;
      a.sgu_s = reinterpret_cast<const __half*>(shared->gate_up_scale);
      a.sgu_z = shared->gate_up_zp;
      a.sd_w = shared->down_weight;
      a.sd_s = reinterpret_cast<const __half*>(shared->down_scale);
      a.sd_z = shared->down_zp;
      a.n_slots = k + 1;
      la.w_sg = reinterpret_cast<const __half*>(w_shared_gate_f16);
      la.slogit = shared_logit;
    }
    la.residual = residual;
    la.nw = norm_weight;
    la.eps = norm_eps;
    la.w_router = reinterpret_cast<const __half*>(w_router_f16);
    la.E = routed->num_experts;
    la.logits = logits;
    la.ids_out = ids;
    la.wts_out = weights;
    la.act = reinterpret_cast<__half*>(workspace);
    la.partial_out = partial_out;
    la.bar = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(workspace) +
                                                   moe_decode_ws(k, hidden, routed->intermediate));
    const LayerSmem L = layer_smem(hidden, routed->intermediate, a.n_slots);
    const cudaError_t e =
        launch(moe_layer_kernel, dim3(sms), dim3(kLayerThreads), (size_t)L.total, s, la);
    return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
  }
  int st = router_logits_launch(nullptr, residual, norm_weight, norm_eps, 1, hidden, w_router_f16,
                                routed->num_experts, shared ? w_shared_gate_f16 : nullptr, logits,
                                shared_logit, s);
  if (st != IQ36_OK) return st;
  // A separate selection launch measured faster than running the top-k in
  // the router's last CTA or inside the expert kernels.
  st = router_select_launch(logits, 1, routed->num_experts, k, ids, weights, s);
  if (st != IQ36_OK) return st;
  if (partial_out)
    return moe_decode_launch(nullptr, residual, norm_weight, norm_eps, ids, weights, k, routed,
                             shared, shared ? shared_logit : nullptr, partial_out, IQ36_F32, 0,
                             workspace, workspace_bytes, s);
  return moe_decode_launch(nullptr, residual, norm_weight, norm_eps, ids, weights, k, routed,
                           shared, shared ? shared_logit : nullptr, residual, IQ36_F32, 1,
                           workspace, workspace_bytes, s);
}
}  // namespace iq36

extern "C" int iq36_moe_layer_decode(float* residual, int32_t hidden, const float* norm_weight,
                                     float norm_eps, const void* w_router_f16,
                                     const void* w_shared_gate_f16, int32_t k,
                                     const iq36_expert_bank* routed,
                                     const iq36_expert_bank* shared, int32_t* ids, float* weights,
                                     float* logits, float* shared_logit, void* workspace,
                                     size_t workspace_bytes, iq36_stream_t stream) {
  return iq36::moe_layer_impl(residual, hidden, norm_weight, norm_eps, w_router_f16,
                              w_shared_gate_f16, k, routed, shared, ids, weights, logits,
                              shared_logit, nullptr, workspace, workspace_bytes, stream);
}

extern "C" int iq36_moe_layer_decode_partial(const float* residual, int32_t hidden,
                                             const float* norm_weight, float norm_eps,
                                             const void* w_router_f16,
                                             const void* w_shared_gate_f16, int32_t k,
                                             const iq36_expert_bank* routed,
                                             const iq36_expert_bank* shared, int32_t* ids,
                                             float* weights, float* logits, float* shared_logit,
                                             float* partial_out, void* workspace,
                                             size_t workspace_bytes, iq36_stream_t stream) {
  if (!partial_out) return IQ36_ERR_ARG;
  return iq36::moe_layer_impl(const_cast<float*>(residual), hidden, norm_weight, norm_eps,
                              w_router_f16, w_shared_gate_f16, k, routed, shared, ids, weights,
                              logits, shared_logit, partial_out, workspace, workspace_bytes,
                              stream);
}

extern "C" size_t iq36_moe_layer_decode_workspace_bytes(int32_t k, int32_t hidden,
                                                        int32_t intermediate) {
  return iq36::moe_layer_ws(k, hidden, intermediate);
}
