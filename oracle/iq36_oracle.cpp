// iq36_oracle.cpp — CPU restatement of the reference's batch-1 hot path.
//
// TEST INFRASTRUCTURE ONLY. This file is the checker for the CUDA library:
// only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
// arm may load it. The product path (the CUDA library and engine/) never links,
// imports or calls anything here.
//
// Every function cites the reference file:line it restates (paths relative to
// the reference checkout). Where the reference keeps a float accumulation the
// "precise" variants accumulate in fp64 to give an error-bound reference; the
// fp16/bf16 rounding points are semantic and are kept exactly.
//
// Parity pinning: the functions shared with the reference's own CPU model
// (router selection, SwiGLU, expert weighting/aggregation, RMSNorm, attention
// core and gate, DeltaNet delta core) are checked against the reference code
// itself compiled from engine/src/gguf_loader.cpp (oracle/Makefile -> _ref/),
// and against golden vectors generated from it (tests/golden/).

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

#include "../include/iq36_synth.h"

namespace {

inline float h2f(uint16_t h) {
  _Float16 v;
  std::memcpy(&v, &h, 2);
  return (float)v;
}
inline uint16_t f2h(float f) {
  _Float16 v = (_Float16)f;  // IEEE round-to-nearest-even
  uint16_t h;
  std::memcpy(&h, &v, 2);
  return h;
}
inline float round_f16(float f) { return h2f(f2h(f)); }
inline float bf2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
inline uint16_t f2bf(float f) {  // round-to-nearest-even (finite inputs)
  uint32_t u;
  std::memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
inline float round_bf16(float f) { return bf2f(f2bf(f)); }

inline int nib(const uint8_t* p, int64_t e) {
  const uint8_t b = p[e >> 1];
  return (e & 1) ? (b >> 4) : (b & 15);
}

// gguf_loader.cpp:3638-3644
inline float sigmoid_scalar(float value) {
  const double x = value;
  const double r = x >= 0.0 ? 1.0 / (1.0 + std::exp(-x)) : std::exp(x) / (1.0 + std::exp(x));
  return (float)r;
}

inline double sigmoid_d(double x) {
  return x >= 0.0 ? 1.0 / (1.0 + std::exp(-x)) : std::exp(x) / (1.0 + std::exp(x));
}

void set_threads(int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
}

// One u4 row dot product, precise: fp64 sum of the exact fp32 products
// x[k] * ((float)(q - zp) * scale) of iq36_fixed_fc_multi_output.cl:112-167.
double u4_row_dot_precise(const float* x, int K, int G, const uint8_t* w, const uint16_t* scale,
                          const uint8_t* zp, int64_t row) {
  const int ng = K / G;
  const uint8_t* wr = w + row * (int64_t)(K / 2);
  double acc = 0.0;
  for (int g = 0; g < ng; ++g) {
    const float s = h2f(scale[row * ng + g]);
    const int z = nib(zp, row * ng + g);
    for (int k = g * G; k < (g + 1) * G; ++k) {
      const int q = (k & 1) ? (wr[k >> 1] >> 4) : (wr[k >> 1] & 15);
      const float deq = (float)(q - z) * s;
      acc += (double)x[k] * (double)deq;
    }
  }
  return acc;
}

// Same row, fp32 (the timed CPU baseline): per-group integer-weight dot, then
// scale * (dot - zp * sum(x_group)). Vectorises with -O3.
float u4_row_dot_fast(const float* x, const float* xg_sum, int K, int G, const uint8_t* w,
                      const uint16_t* scale, const uint8_t* zp, int64_t row) {
  const int ng = K / G;
  const uint8_t* wr = w + row * (int64_t)(K / 2);
  float acc = 0.0f;
  for (int g = 0; g < ng; ++g) {
    const uint8_t* wb = wr + g * (G / 2);
    const float* xb = x + g * G;
    float d0 = 0.0f, d1 = 0.0f;
    for (int j = 0; j < G / 2; ++j) {
      d0 += xb[2 * j] * (float)(wb[j] & 15);
      d1 += xb[2 * j + 1] * (float)(wb[j] >> 4);
    }
    const float s = h2f(scale[row * ng + g]);
    const int z = nib(zp, row * ng + g);
    acc += s * ((d0 + d1) - (float)z * xg_sum[g]);
  }
  return acc;
}

void u4_gemv_f32in(const float* x, int K, int G, const uint8_t* w, const uint16_t* scale,
                   const uint8_t* zp, int64_t N, float* out, int precise) {
  if (precise) {
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) out[n] = (float)u4_row_dot_precise(x, K, G, w, scale, zp, n);
  } else {
    std::vector<float> xg(K / G, 0.0f);
    for (int g = 0; g < K / G; ++g)
      for (int k = g * G; k < (g + 1) * G; ++k) xg[g] += x[k];
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) out[n] = u4_row_dot_fast(x, xg.data(), K, G, w, scale, zp, n);
  }
}

// softmax of gguf_loader.cpp:3646-3670 (fp64 exp and sum, fp32 result).
std::vector<float> softmax_ref(const float* logits, int n) {
  const float mx = *std::max_element(logits, logits + n);
  std::vector<double> e(n);
  double sum = 0.0;
  for (int i = 0; i < n; ++i) {
    e[i] = std::exp((double)logits[i] - (double)mx);
    sum += e[i];
  }
  std::vector<float> p(n);
  for (int i = 0; i < n; ++i) p[i] = (float)(e[i] / sum);
  return p;
}

// top_k_indices (:3672-3697): descending value, lower id first on ties.
std::vector<int32_t> top_k_ref(const std::vector<float>& v, int k) {
  std::vector<int32_t> idx(v.size());
  std::iota(idx.begin(), idx.end(), 0);
  std::partial_sort(idx.begin(), idx.begin() + k, idx.end(), [&](int32_t a, int32_t b) {
    if (v[a] == v[b]) return a < b;
    return v[a] > v[b];
  });
  idx.resize(k);
  return idx;
}

}  // namespace

extern "C" {

int orc_version(void) { return 1; }

void orc_f16_to_f32(const uint16_t* in, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = h2f(in[i]);
}
void orc_f32_to_f16(const float* in, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = f2h(in[i]);
}

// Host twin of the device generator (include/iq36_synth.h); same kinds as
// iq36_synth_fill.
// Elements [offset, offset + count) of one synthetic tensor into dst[0..count).
void orc_synth_fill_at(void* dst, int64_t offset, int64_t count, int kind, uint64_t seed,
                       uint64_t tensor, float lo, float hi) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < count; ++i) {
    const uint64_t j = (uint64_t)(offset + i);
    switch (kind) {
      case 0: ((uint8_t*)dst)[i] = iq36_synth_u8(seed, tensor, j); break;
      case 1: ((uint16_t*)dst)[i] = f2h(iq36_synth_uniform(seed, tensor, j, lo, hi)); break;
      case 2: ((uint16_t*)dst)[i] = f2h(iq36_synth_normal(seed, tensor, j, lo)); break;
      case 3: ((float*)dst)[i] = iq36_synth_uniform(seed, tensor, j, lo, hi); break;
      case 4: ((float*)dst)[i] = iq36_synth_normal(seed, tensor, j, lo); break;
      default: break;
    }
  }
}

void orc_synth_fill(void* dst, int64_t count, int kind, uint64_t seed, uint64_t tensor, float lo,
                    float hi) {
  orc_synth_fill_at(dst, 0, count, kind, seed, tensor, lo, hi);
}

// u4 GEMV, fp16 activation. Restates iq36_fixed_fc_multi_output.cl:112-167
// (op order: (int)(q - zp) -> float -> * scale -> fma with x, fp32 sum) and
// the stock pattern fixed_fc.py:107-144. precise=1: fp64 accumulation.
void orc_u4_gemv(const uint16_t* x_f16, int K, int G, const uint8_t* w, const uint16_t* scale,
                 const uint8_t* zp, int64_t N, float* out, int precise, int threads) {
  set_threads(threads);
  std::vector<float> x(K);
  for (int k = 0; k < K; ++k) x[k] = h2f(x_f16[k]);
  u4_gemv_f32in(x.data(), K, G, w, scale, zp, N, out, precise);
}

// fp16-weight linear (router 2048->256, shared gate 2048->1): fp64 dot
// rounded to fp32, as the reference CPU matvec reports f32 logits.
void orc_f16_linear(const uint16_t* x_f16, int H, const uint16_t* W, int E, float* out) {
  for (int e = 0; e < E; ++e) {
    double acc = 0.0;
    for (int h = 0; h < H; ++h) acc += (double)h2f(x_f16[h]) * (double)h2f(W[(int64_t)e * H + h]);
    out[e] = (float)acc;
  }
}

// select_router_topk (gguf_loader.cpp:3733-3743) = softmax (:3646-3670),
// top_k_indices (:3672-3697), gather_values, normalize_weights (:3712-3731)
// with min_weight_sum 6.103515625e-5 (:5665).
void orc_router_select(const float* logits, int T, int E, int k, int32_t* ids, float* weights) {
  for (int t = 0; t < T; ++t) {
    const auto p = softmax_ref(logits + (int64_t)t * E, E);
    const auto top = top_k_ref(p, k);
    float sum = 0.0f;
    for (int r = 0; r < k; ++r) sum += p[top[r]];
    const float den = std::max(sum, 6.103515625e-5f);
    for (int r = 0; r < k; ++r) {
      ids[(int64_t)t * k + r] = top[r];
      weights[(int64_t)t * k + r] = p[top[r]] / den;
    }
  }
}

// apply_swiglu_from_gate_up (gguf_loader.cpp:4640-4668): fp64 g*sigmoid(g)*u.
void orc_swiglu(const float* gate, const float* up, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) {
    const double g = gate[i], u = up[i];
    out[i] = (float)(g * sigmoid_d(g) * u);
  }
}

// MoE decode block, run_qwen36_moe_ffn_layer (gguf_loader.cpp:5654-5782):
// per routed expert gate_up u4 GEMV -> SwiGLU (rounded to fp16 as the input of
// the down GEMV) -> down u4 GEMV -> * router weight (apply_expert_weights
// :3773-3797) -> fp32 sum in rank order (aggregate_experts :3799-3819); shared
// expert likewise times sigmoid_scalar(shared_logit) (:5767-5778), added last
// (:5779). out fp32 (the CUDA op rounds its output to fp16 or accumulates).
void orc_moe_decode(const uint16_t* x_f16, const int32_t* ids, const float* weights, int k,
                    const uint8_t* gu_w, const uint16_t* gu_s, const uint8_t* gu_z,
                    const uint8_t* d_w, const uint16_t* d_s, const uint8_t* d_z,
                    const uint8_t* sgu_w, const uint16_t* sgu_s, const uint8_t* sgu_z,
                    const uint8_t* sd_w, const uint16_t* sd_s, const uint8_t* sd_z,
                    const float* shared_logit, int H, int I, int G, float* out, int precise,
                    int threads) {
  set_threads(threads);
  const int64_t gu_wb = (int64_t)2 * I * H / 2, gu_sn = (int64_t)2 * I * H / G,
                gu_zb = (int64_t)2 * I * H / G / 2;
  const int64_t d_wb = (int64_t)H * I / 2, d_sn = (int64_t)H * I / G, d_zb = (int64_t)H * I / G / 2;
  std::vector<float> x(H), gu(2 * I), act(I), dn(H), acc(H, 0.0f);
  for (int h = 0; h < H; ++h) x[h] = h2f(x_f16[h]);
  const int n_exp = k + (sgu_w ? 1 : 0);
  for (int r = 0; r < n_exp; ++r) {
    const bool shared = r == k;
    const int64_t e = shared ? 0 : ids[r];
    const uint8_t* w1 = shared ? sgu_w : gu_w + e * gu_wb;
    const uint16_t* s1 = shared ? sgu_s : gu_s + e * gu_sn;
    const uint8_t* z1 = shared ? sgu_z : gu_z + e * gu_zb;
    const uint8_t* w2 = shared ? sd_w : d_w + e * d_wb;
    const uint16_t* s2 = shared ? sd_s : d_s + e * d_sn;
    const uint8_t* z2 = shared ? sd_z : d_z + e * d_zb;
    u4_gemv_f32in(x.data(), H, G, w1, s1, z1, 2 * I, gu.data(), precise);
    orc_swiglu(gu.data(), gu.data() + I, I, act.data());
    for (int i = 0; i < I; ++i) act[i] = round_f16(act[i]);
    u4_gemv_f32in(act.data(), I, G, w2, s2, z2, H, dn.data(), precise);
    const float wr = shared ? sigmoid_scalar(*shared_logit) : weights[r];
    for (int h = 0; h < H; ++h) acc[h] += dn[h] * wr;
  }
  for (int h = 0; h < H; ++h) out[h] = acc[h];
}

// Paged GQA decode. run_qwen36_full_attention_core (gguf_loader.cpp:6071-6137)
// over the K/V rows gathered through the block table, then the output gate of
// run_qwen36_full_attention_gate (:6034-6069). Scores: fp64 dot * scale
// rounded to fp32; softmax as :3646-3670; weighted V sum in fp64 (precise).
void orc_paged_gqa(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* bt,
                   int ctx, int nq, int nkv, int D, int bs, float scale, const uint16_t* gate,
                   float* out, int threads) {
  set_threads(threads);
  const int grp = nq / nkv;
#pragma omp parallel for schedule(dynamic)
  for (int h = 0; h < nq; ++h) {
    const int kvh = h / grp;
    std::vector<float> sc(ctx);
    std::vector<double> qd(D);
    for (int d = 0; d < D; ++d) qd[d] = h2f(q[h * D + d]);
    for (int t = 0; t < ctx; ++t) {
      const int64_t base = (((int64_t)bt[t / bs] * bs + (t % bs)) * nkv + kvh) * D;
      double dot = 0.0;
      for (int d = 0; d < D; ++d) dot += qd[d] * (double)h2f(kc[base + d]);
      sc[t] = (float)(dot * (double)scale);
    }
    const auto w = softmax_ref(sc.data(), ctx);
    std::vector<double> o(D, 0.0);
    for (int t = 0; t < ctx; ++t) {
      const int64_t base = (((int64_t)bt[t / bs] * bs + (t % bs)) * nkv + kvh) * D;
      for (int d = 0; d < D; ++d) o[d] += (double)w[t] * (double)h2f(vc[base + d]);
    }
    for (int d = 0; d < D; ++d) {
      float v = (float)o[d];
      if (gate) v = v * sigmoid_scalar(h2f(gate[h * D + d]));
      out[h * D + d] = v;
    }
  }
}

// RMSNorm, apply_rms_norm / apply_repeated_rms_norm (gguf_loader.cpp:3368-3391,
// 3410-3439), fp64 sum of squares.
void orc_rms_norm(const float* in, int rows, int dim, const float* w, int wlen, float eps,
                  float* out) {
  for (int r = 0; r < rows; ++r) {
    for (int base = 0; base < dim; base += wlen) {
      const float* x = in + (int64_t)r * dim + base;
      double ss = 0.0;
      for (int i = 0; i < wlen; ++i) ss += (double)x[i] * x[i];
      const float sc = (float)(1.0 / std::sqrt(ss / wlen + (double)eps));
      for (int i = 0; i < wlen; ++i) out[(int64_t)r * dim + base + i] = x[i] * sc * w[i];
    }
  }
}

// Partial rotate-half RoPE of iq36_qk_rope_layout.cl:37-60 for one head vector
// in place: dims < rope_dim rotated with theta_d = pos * base^(-2(d mod
// rope_dim/2)/rope_dim); the tail copied.
void orc_rope(float* x, int D, int rope_dim, int pos, float base) {
  const int half = rope_dim / 2;
  std::vector<double> y(rope_dim);
  for (int d = 0; d < rope_dim; ++d) {
    const int i = d % half;
    const double inv = std::pow((double)base, -2.0 * i / rope_dim);
    const double th = (double)pos * inv;
    const double c = std::cos(th), s = std::sin(th);
    y[d] = d < half ? x[d] * c - x[d + half] * s : x[d] * c + x[d - half] * s;
  }
  for (int d = 0; d < rope_dim; ++d) x[d] = (float)y[d];
  (void)D;
}

// Full-attention pre-step (see iq36_attn_prep in include/iq36_b200.h).
// Outputs fp32 holding fp16-rounded values: q_out [nq*D], gate_out [nq*D],
// k_new [nkv*D] (the cache row), v_new [nkv*D].
void orc_attn_prep(const uint16_t* q_full, const uint16_t* k, const uint16_t* v,
                   const float* qn_w, const float* kn_w, float eps, int pos, int nq, int nkv,
                   int D, int rope_dim, float base, float* q_out, float* gate_out, float* k_new,
                   float* v_new) {
  std::vector<float> tmp(D);
  for (int h = 0; h < nq; ++h) {
    for (int d = 0; d < D; ++d) tmp[d] = h2f(q_full[(h * 2) * D + d]);
    orc_rms_norm(tmp.data(), 1, D, qn_w, D, eps, tmp.data());
    orc_rope(tmp.data(), D, rope_dim, pos, base);
    for (int d = 0; d < D; ++d) {
      q_out[h * D + d] = round_f16(tmp[d]);
      gate_out[h * D + d] = h2f(q_full[(h * 2 + 1) * D + d]);
    }
  }
  for (int h = 0; h < nkv; ++h) {
    for (int d = 0; d < D; ++d) tmp[d] = h2f(k[h * D + d]);
    orc_rms_norm(tmp.data(), 1, D, kn_w, D, eps, tmp.data());
    orc_rope(tmp.data(), D, rope_dim, pos, base);
    for (int d = 0; d < D; ++d) {
      k_new[h * D + d] = round_f16(tmp[d]);
      v_new[h * D + d] = h2f(v[h * D + d]);
    }
  }
}

// DeltaNet pre-step: conv of iq36_linear_conv_swish.cl:25-63 for one token
// (combined = [state0..3, x]; out = sum_tap w[tap] * combined[1+tap]; fp16
// rounding of the convolution and of the SiLU output; next state = last four
// of combined), and the gate/beta transform of gguf_loader.cpp:4875-4912.
void orc_delta_prep(const uint16_t* qkv, int C, float* conv_state, const float* conv_w,
                    const uint16_t* a, const uint16_t* b, const float* a_log,
                    const float* dt_bias, int nv, float* act_out, float* g_out,
                    float* beta_out) {
  for (int c = 0; c < C; ++c) {
    const float xv = h2f(qkv[c]);
    const float comb[5] = {conv_state[c * 4 + 0], conv_state[c * 4 + 1], conv_state[c * 4 + 2],
                           conv_state[c * 4 + 3], xv};
    double s = 0.0;
    for (int tap = 0; tap < 4; ++tap) s += (double)conv_w[c * 4 + tap] * comb[1 + tap];
    const float conv = round_f16((float)s);
    const double act = (double)conv / (1.0 + std::exp(-(double)conv));
    act_out[c] = round_f16((float)act);
    for (int j = 0; j < 4; ++j) conv_state[c * 4 + j] = comb[1 + j];
  }
  for (int h = 0; h < nv; ++h) {
    const double xa = (double)h2f(a[h]) + dt_bias[h];
    const double sp = xa > 20.0 ? xa : std::log1p(std::exp(xa));
    g_out[h] = (float)(-std::exp((double)a_log[h]) * sp);
    beta_out[h] = (float)sigmoid_d(h2f(b[h]));
  }
}

// Gated DeltaNet step, OpenVINO semantics (iq36_gated_delta_net.cl:36-150):
// key head = value head / (nv/nk); q,k L2-normalised with rsqrt(sum + 1e-6),
// q additionally * 1/sqrt(D); S = exp(g) S; sk = S^T k; delta = (v - sk) beta;
// S += k delta^T; o = S^T q. State [nv, D(key), D(value)]. Then the gated
// RMSNorm of gguf_loader.cpp:4770-4786: o * rsqrt(mean(o^2)+eps) * w * silu(z).
void orc_delta_step(const float* act, const float* g, const float* beta, float* state,
                    const uint16_t* z, const float* norm_w, float eps, int nk, int nv, int D,
                    float* out) {
  const int ratio = nv / nk;
  for (int vh = 0; vh < nv; ++vh) {
    const int kh = vh / ratio;
    const float* q = act + kh * D;
    const float* kk = act + (nk + kh) * D;
    const float* vv = act + (2 * nk + vh) * D;
    double qs = 0.0, ks = 0.0;
    for (int i = 0; i < D; ++i) {
      qs += (double)q[i] * q[i];
      ks += (double)kk[i] * kk[i];
    }
    const double qsc = 1.0 / std::sqrt(qs + 1e-6) / std::sqrt((double)D);
    const double ksc = 1.0 / std::sqrt(ks + 1e-6);
    std::vector<double> qn(D), kn(D), sk(D, 0.0), o(D, 0.0);
    for (int i = 0; i < D; ++i) {
      qn[i] = q[i] * qsc;
      kn[i] = kk[i] * ksc;
    }
    float* S = state + (int64_t)vh * D * D;
    const double decay = std::exp((double)g[vh]);
    for (int i = 0; i < D; ++i)
      for (int j = 0; j < D; ++j) {
        S[i * D + j] = (float)(S[i * D + j] * decay);
        sk[j] += (double)S[i * D + j] * kn[i];
      }
    for (int j = 0; j < D; ++j) {
      const double delta = ((double)vv[j] - sk[j]) * beta[vh];
      for (int i = 0; i < D; ++i) S[i * D + j] = (float)(S[i * D + j] + kn[i] * delta);
    }
    for (int i = 0; i < D; ++i)
      for (int j = 0; j < D; ++j) o[j] += (double)S[i * D + j] * qn[i];
    double ss = 0.0;
    for (int j = 0; j < D; ++j) ss += o[j] * o[j];
    const double nsc = 1.0 / std::sqrt(ss / D + eps);
    for (int j = 0; j < D; ++j) {
      const double zv = h2f(z[vh * D + j]);
      out[vh * D + j] = (float)(o[j] * nsc * norm_w[j] * (zv * sigmoid_d(zv)));
    }
  }
}

// Grouped MoE prefill for a subset of tokens (each token's output depends only
// on its own routing, so parity at full T is checked on a sample). Gen-1
// dataflow grouped_s8_u4_f16_contribution_moe.cl:13-222 (schedule) and
// :847-861 (scatter, fixed rank order), stock gather/GEMM/scatter
// iq36-pr35924-grouped-postops.patch:15-124. Rounding points of the tensor-core
// path: gate_up and down accumulate in fp32 (fp64 here), SwiGLU output rounded
// to fp16 (the second GEMM's operand type), contribution = down * weight in
// fp32, out = sum over ranks in rank order. Weights are dequantised exactly
// (the tensor-core path rounds each dequantised weight to fp16; the tolerance
// covers that).
void orc_moe_prefill(const uint16_t* x_bf16, const int32_t* tokens, int n_tokens, int H,
                     const int32_t* ids, const float* weights, int k, const uint8_t* gu_w,
                     const uint16_t* gu_s, const uint8_t* gu_z, const uint8_t* d_w,
                     const uint16_t* d_s, const uint8_t* d_z, int I, int G, float* out,
                     int threads) {
  set_threads(threads);
  const int64_t gu_wb = (int64_t)2 * I * H / 2, gu_sn = (int64_t)2 * I * H / G,
                gu_zb = (int64_t)2 * I * H / G / 2;
  const int64_t d_wb = (int64_t)H * I / 2, d_sn = (int64_t)H * I / G, d_zb = (int64_t)H * I / G / 2;
#pragma omp parallel for schedule(dynamic)
  for (int i = 0; i < n_tokens; ++i) {
    const int64_t t = tokens[i];
    std::vector<float> x(H), act(I), acc(H, 0.0f);
    std::vector<float> gu(2 * I), dn(H);
    for (int h = 0; h < H; ++h) x[h] = bf2f(x_bf16[t * H + h]);
    for (int r = 0; r < k; ++r) {
      const int64_t e = ids[t * k + r];
      for (int n = 0; n < 2 * I; ++n)
        gu[n] = (float)u4_row_dot_precise(x.data(), H, G, gu_w + e * gu_wb, gu_s + e * gu_sn,
                                          gu_z + e * gu_zb, n);
      for (int j = 0; j < I; ++j) {
        const double gg = gu[j], uu = gu[I + j];
        act[j] = round_f16((float)(gg * sigmoid_d(gg) * uu));
      }
      for (int n = 0; n < H; ++n)
        dn[n] = (float)u4_row_dot_precise(act.data(), I, G, d_w + e * d_wb, d_s + e * d_sn,
                                          d_z + e * d_zb, n);
      const float w = weights[t * k + r];
      for (int h = 0; h < H; ++h) acc[h] += dn[h] * w;
    }
    for (int h = 0; h < H; ++h) out[(int64_t)i * H + h] = acc[h];
  }
}

// Greedy top-1, lowest id on ties (iq36_greedy_top1.cl:8-46, np.argmax).
int orc_argmax(const float* logits, int64_t n) {
  int64_t best = 0;
  for (int64_t i = 1; i < n; ++i)
    if (logits[i] > logits[best]) best = i;
  return (int)best;
}

}  // extern "C"
