// iq36_oracle_model.cpp — CPU restatement of the batch-1 decode step of the
// synthetic Qwen3.6-35B-A3B-shaped model.
//
// TEST INFRASTRUCTURE ONLY (see iq36_oracle.cpp). Composes the per-op
// restatements in the order of the reference graph (its call stack; per
// layer: RMSNorm -> attention or DeltaNet -> residual -> RMSNorm -> router +
// routed/shared experts -> residual; then final RMSNorm -> LM head -> greedy),
// following gguf_loader.cpp run_qwen36_layer_with_external_attention_state
// (:6207-6242), run_qwen36_stateful_full_attention_layer (:6140-6205) and
// run_qwen36_moe_ffn_layer (:5654-5782), with the OpenVINO fp16 rounding points
// (every fixed-FC output rounded to fp16: iq36_fixed_fc_multi_output.cl:198).
// Weights come from the shared synthetic generator (include/iq36_synth.h).

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "../include/iq36_synth.h"

extern "C" {
void orc_synth_fill(void* dst, int64_t count, int kind, uint64_t seed, uint64_t tensor, float lo,
                    float hi);
void orc_synth_fill_at(void* dst, int64_t offset, int64_t count, int kind, uint64_t seed,
                       uint64_t tensor, float lo, float hi);
void orc_u4_gemv(const uint16_t* x_f16, int K, int G, const uint8_t* w, const uint16_t* scale,
                 const uint8_t* zp, int64_t N, float* out, int precise, int threads);
void orc_f16_linear(const uint16_t* x_f16, int H, const uint16_t* W, int E, float* out);
void orc_router_select(const float* logits, int T, int E, int k, int32_t* ids, float* weights);
void orc_moe_decode(const uint16_t* x_f16, const int32_t* ids, const float* weights, int k,
                    const uint8_t* gu_w, const uint16_t* gu_s, const uint8_t* gu_z,
                    const uint8_t* d_w, const uint16_t* d_s, const uint8_t* d_z,
                    const uint8_t* sgu_w, const uint16_t* sgu_s, const uint8_t* sgu_z,
                    const uint8_t* sd_w, const uint16_t* sd_s, const uint8_t* sd_z,
                    const float* shared_logit, int H, int I, int G, float* out, int precise,
                    int threads);
void orc_paged_gqa(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* bt,
                   int ctx, int nq, int nkv, int D, int bs, float scale, const uint16_t* gate,
                   float* out, int threads);
void orc_rms_norm(const float* in, int rows, int dim, const float* w, int wlen, float eps,
                  float* out);
void orc_attn_prep(const uint16_t* q_full, const uint16_t* k, const uint16_t* v,
                   const float* qn_w, const float* kn_w, float eps, int pos, int nq, int nkv,
                   int D, int rope_dim, float base, float* q_out, float* gate_out, float* k_new,
                   float* v_new);
void orc_delta_prep(const uint16_t* qkv, int C, float* conv_state, const float* conv_w,
                    const uint16_t* a, const uint16_t* b, const float* a_log,
                    const float* dt_bias, int nv, float* act_out, float* g_out, float* beta_out);
void orc_delta_step(const float* act, const float* g, const float* beta, float* state,
                    const uint16_t* z, const float* norm_w, float eps, int nk, int nv, int D,
                    float* out);
int orc_argmax(const float* logits, int64_t n);
}

namespace {

inline uint16_t f2h(float f) {
  _Float16 v = (_Float16)f;
  uint16_t h;
  std::memcpy(&h, &v, 2);
  return h;
}
inline float h2f(uint16_t h) {
  _Float16 v;
  std::memcpy(&v, &h, 2);
  return (float)v;
}

}  // namespace

// Model dimensions; the field order is part of the C ABI of this file.
struct OrcModelConfig {
  int32_t hidden, layers, attn_interval, nq, nkv, head_dim, rope_dim, nk, nv, dk, conv, experts,
      topk, inter, shared_inter, vocab, group;
  float rope_base, eps;
  int32_t fc_group;  // attention and DeltaNet projections (0: group)
};

namespace {

struct U4 {
  std::vector<uint8_t> w, z;
  std::vector<uint16_t> s;
  int64_t rows = 0;
  int K = 0;
};

struct Layer {
  bool attn = false;
  std::vector<float> in_norm, post_norm;
  U4 q, k, v, o;                                  // attention
  std::vector<float> qn, kn;
  U4 qkv, z, a, b, out;                           // DeltaNet
  std::vector<float> conv_w, a_log, dt_bias, dnorm;
  std::vector<uint16_t> router, sgate;            // MoE
  U4 gu, down, sgu, sdown;  // gu/down hold all experts, or (lazy) the k selected ones
  // state
  std::vector<float> conv_state, rec_state;
  std::vector<uint16_t> kc, vc;
};

struct Model {
  OrcModelConfig c;
  uint64_t seed;
  int max_ctx;
  // Lazy expert banks: above kLazyBankBytes per layer the routed experts are
  // not materialised; each step regenerates only the k selected experts'
  // rows from the counter-based generator (same values, element for element),
  // so the full 256-expert model needs ~1 GB of host memory instead of ~17 GB.
  bool lazy = false;
  // GEMV and expert accumulation in fp64 instead of the fp32 mirror
  // (IQ36_ORACLE_PRECISE=1): a second checker that differs from the first only
  // in summation rounding, used to measure how far the deep random-init model
  // amplifies rounding differences.
  int precise = 0;
  std::vector<Layer> layers;
  std::vector<float> final_norm;
  U4 lm_head;
  std::vector<int32_t> bt;
};

void fill_f32(std::vector<float>& v, int64_t n, uint64_t seed, int layer, int slot) {
  int kind;
  float lo, hi;
  iq36_synth_spec(slot, 0, &kind, &lo, &hi);
  v.resize(n);
  orc_synth_fill(v.data(), n, kind, seed, iq36_tensor_id(layer, slot, 0), lo, hi);
}

void fill_f16(std::vector<uint16_t>& v, int64_t n, uint64_t seed, int layer, int slot) {
  int kind;
  float lo, hi;
  iq36_synth_spec(slot, 0, &kind, &lo, &hi);
  v.resize(n);
  orc_synth_fill(v.data(), n, kind, seed, iq36_tensor_id(layer, slot, 0), lo, hi);
}

void fill_u4(U4& m, int64_t rows, int K, int G, uint64_t seed, int layer, int slot) {
  m.rows = rows;
  m.K = K;
  const int64_t nw = rows * K / 2, ns = rows * K / G, nz = rows * K / G / 2;
  m.w.resize(nw);
  m.s.resize(ns);
  m.z.resize(nz);
  int kind;
  float lo, hi;
  iq36_synth_spec(slot, 0, &kind, &lo, &hi);
  orc_synth_fill(m.w.data(), nw, kind, seed, iq36_tensor_id(layer, slot, 0), lo, hi);
  iq36_synth_spec(slot, 1, &kind, &lo, &hi);
  orc_synth_fill(m.s.data(), ns, kind, seed, iq36_tensor_id(layer, slot, 1), lo, hi);
  iq36_synth_spec(slot, 2, &kind, &lo, &hi);
  orc_synth_fill(m.z.data(), nz, kind, seed, iq36_tensor_id(layer, slot, 2), lo, hi);
}

constexpr int64_t kLazyBankBytes = 256ll << 20;

// Rows [row0, row0 + rows) of a u4 matrix tensor (codes, scales, zero
// points) into slot `dst_row0` of m (m already sized).
void fill_u4_rows(U4& m, int64_t dst_row0, int64_t row0, int64_t rows, int K, int G,
                  uint64_t seed, int layer, int slot) {
  const int ng = K / G;
  int kind;
  float lo, hi;
  iq36_synth_spec(slot, 0, &kind, &lo, &hi);
  orc_synth_fill_at(m.w.data() + dst_row0 * (K / 2), row0 * (K / 2), rows * (K / 2), kind, seed,
                    iq36_tensor_id(layer, slot, 0), lo, hi);
  iq36_synth_spec(slot, 1, &kind, &lo, &hi);
  orc_synth_fill_at(m.s.data() + dst_row0 * ng, row0 * ng, rows * ng, kind, seed,
                    iq36_tensor_id(layer, slot, 1), lo, hi);
  iq36_synth_spec(slot, 2, &kind, &lo, &hi);
  orc_synth_fill_at(m.z.data() + dst_row0 * ng / 2, row0 * ng / 2, rows * ng / 2, kind, seed,
                    iq36_tensor_id(layer, slot, 2), lo, hi);
}

// Copies rows [0, per) of m (codes, scales, zero points) to the n - 1 blocks
// of `per` rows that follow.
void replicate_rows(U4& m, int64_t per, int n) {
  const int64_t bw = per * m.K / 2, bs = (int64_t)m.s.size() / n, bz = (int64_t)m.z.size() / n;
#pragma omp parallel for schedule(static)
  for (int e = 1; e < n; ++e) {
    std::memcpy(m.w.data() + e * bw, m.w.data(), bw);
    std::memcpy(m.s.data() + e * bs, m.s.data(), bs * sizeof(uint16_t));
    std::memcpy(m.z.data() + e * bz, m.z.data(), bz);
  }
}

void size_u4(U4& m, int64_t rows, int K, int G) {
  m.rows = rows;
  m.K = K;
  m.w.resize(rows * K / 2);
  m.s.resize(rows * K / G);
  m.z.resize(rows * K / G / 2);
}

void gemv16(const U4& m, const uint16_t* x, int G, std::vector<float>& y, int threads,
            int precise) {
  y.resize(m.rows);
  orc_u4_gemv(x, m.K, G, m.w.data(), m.s.data(), m.z.data(), m.rows, y.data(), precise, threads);
}

std::vector<uint16_t> to_f16(const std::vector<float>& v) {
  std::vector<uint16_t> r(v.size());
  for (size_t i = 0; i < v.size(); ++i) r[i] = f2h(v[i]);
  return r;
}

}  // namespace

extern "C" {

void* orc_model_create(const OrcModelConfig* cfg, uint64_t seed, int max_ctx) {
  auto* M = new Model();
  M->c = *cfg;
  M->seed = seed;
  M->max_ctx = max_ctx;
  const OrcModelConfig& c = *cfg;
  const int H = c.hidden, G = c.group, FG = c.fc_group > 0 ? c.fc_group : c.group;
  M->layers.resize(c.layers);
  for (int l = 0; l < c.layers; ++l) {
    Layer& L = M->layers[l];
    L.attn = (l % c.attn_interval) == (c.attn_interval - 1);
    fill_f32(L.in_norm, H, seed, l, IQ36_T_IN_NORM);
    fill_f32(L.post_norm, H, seed, l, IQ36_T_POST_NORM);
    if (L.attn) {
      fill_u4(L.q, (int64_t)2 * c.nq * c.head_dim, H, FG, seed, l, IQ36_T_Q);
      fill_u4(L.k, (int64_t)c.nkv * c.head_dim, H, FG, seed, l, IQ36_T_K);
      fill_u4(L.v, (int64_t)c.nkv * c.head_dim, H, FG, seed, l, IQ36_T_V);
      fill_u4(L.o, H, c.nq * c.head_dim, FG, seed, l, IQ36_T_O);
      fill_f32(L.qn, c.head_dim, seed, l, IQ36_T_QNORM);
      fill_f32(L.kn, c.head_dim, seed, l, IQ36_T_KNORM);
      const int64_t blocks = (max_ctx + 15) / 16;
      L.kc.assign(blocks * 16 * c.nkv * c.head_dim, 0);
      L.vc.assign(blocks * 16 * c.nkv * c.head_dim, 0);
    } else {
      const int64_t C = (int64_t)(2 * c.nk + c.nv) * c.dk;
      fill_u4(L.qkv, C, H, FG, seed, l, IQ36_T_QKV);
      fill_u4(L.z, (int64_t)c.nv * c.dk, H, FG, seed, l, IQ36_T_Z);
      fill_u4(L.a, c.nv, H, FG, seed, l, IQ36_T_A);
      fill_u4(L.b, c.nv, H, FG, seed, l, IQ36_T_B);
      fill_u4(L.out, H, c.nv * c.dk, FG, seed, l, IQ36_T_OUT);
      fill_f32(L.conv_w, C * c.conv, seed, l, IQ36_T_CONV);
      fill_f32(L.a_log, c.nv, seed, l, IQ36_T_ALOG);
      fill_f32(L.dt_bias, c.nv, seed, l, IQ36_T_DTB);
      fill_f32(L.dnorm, c.dk, seed, l, IQ36_T_DNORM);
      L.conv_state.assign(C * c.conv, 0.0f);
      L.rec_state.assign((int64_t)c.nv * c.dk * c.dk, 0.0f);
    }
    fill_f16(L.router, (int64_t)c.experts * H, seed, l, IQ36_T_ROUTER);
    fill_f16(L.sgate, H, seed, l, IQ36_T_SGATE);
    M->lazy = (int64_t)c.experts * 3 * c.inter * H / 2 > kLazyBankBytes;
    if (const char* f = std::getenv("IQ36_ORACLE_LAZY")) M->lazy = f[0] == '1';
    if (const char* f = std::getenv("IQ36_ORACLE_PRECISE")) M->precise = f[0] == '1';
    // Timing-only banks (IQ36_ORACLE_REPLICATED=1): expert 0 generated, then
    // copied to every other expert. The router still spreads tokens over all
    // experts, so each step reads the same bytes and does the same arithmetic
    // as with distinct experts; only the values differ. Used by the timed CPU
    // baseline, whose model would otherwise take minutes to generate.
    const char* rep = std::getenv("IQ36_ORACLE_REPLICATED");
    if (M->lazy) {
      size_u4(L.gu, (int64_t)c.topk * 2 * c.inter, H, G);
      size_u4(L.down, (int64_t)c.topk * H, c.inter, G);
    } else if (rep && rep[0] == '1') {
      size_u4(L.gu, (int64_t)c.experts * 2 * c.inter, H, G);
      size_u4(L.down, (int64_t)c.experts * H, c.inter, G);
      fill_u4_rows(L.gu, 0, 0, 2 * c.inter, H, G, seed, l, IQ36_T_GU);
      fill_u4_rows(L.down, 0, 0, H, c.inter, G, seed, l, IQ36_T_DOWN);
      replicate_rows(L.gu, 2 * c.inter, c.experts);
      replicate_rows(L.down, H, c.experts);
    } else {
      fill_u4(L.gu, (int64_t)c.experts * 2 * c.inter, H, G, seed, l, IQ36_T_GU);
      fill_u4(L.down, (int64_t)c.experts * H, c.inter, G, seed, l, IQ36_T_DOWN);
    }
    fill_u4(L.sgu, (int64_t)2 * c.shared_inter, H, G, seed, l, IQ36_T_SGU);
    fill_u4(L.sdown, H, c.shared_inter, G, seed, l, IQ36_T_SDOWN);
  }
  fill_f32(M->final_norm, H, seed, -1, IQ36_T_FINAL_NORM);
  fill_u4(M->lm_head, c.vocab, H, G, seed, -1, IQ36_T_LM_HEAD);
  M->bt.resize((max_ctx + 15) / 16);
  for (size_t i = 0; i < M->bt.size(); ++i) M->bt[i] = (int32_t)i;
  return M;
}

void orc_model_destroy(void* m) { delete static_cast<Model*>(m); }

// One decode step at position pos (the KV cache and recurrent states hold
// positions < pos). Writes fp32 logits [vocab] when logits != NULL and returns
// the greedy token.
int orc_model_step_opt(void* mp, int token, int pos, float* logits, int threads, int lm_head,
                       float* hidden, int32_t* ids_out, float* router_out);

int orc_model_step(void* mp, int token, int pos, float* logits, int threads) {
  return orc_model_step_opt(mp, token, pos, logits, threads, 1, nullptr, nullptr, nullptr);
}

// The step without the final norm and LM head (returns -1): feeds a prompt
// token whose next-token distribution is not needed.
int orc_model_feed(void* mp, int token, int pos, int threads) {
  return orc_model_step_opt(mp, token, pos, nullptr, threads, 0, nullptr, nullptr, nullptr);
}

// The step with its trace: hidden [(layers + 1) * hidden] receives the fp32
// residual stream entering each layer and, last, leaving the final layer;
// ids_out [layers * topk] the routed expert ids of every layer (rank order);
// router_out [layers * experts] every layer's router logits.
int orc_model_step_trace(void* mp, int token, int pos, float* logits, int threads, float* hidden,
                         int32_t* ids_out, float* router_out) {
  return orc_model_step_opt(mp, token, pos, logits, threads, 1, hidden, ids_out, router_out);
}

int orc_model_step_opt(void* mp, int token, int pos, float* logits, int threads, int lm_head,
                       float* hidden, int32_t* ids_out, float* router_out) {
  Model& M = *static_cast<Model*>(mp);
  const OrcModelConfig& c = M.c;
  const int H = c.hidden, G = c.group, FG = c.fc_group > 0 ? c.fc_group : c.group;
  std::vector<float> h(H), xn(H), y, y2, y3, y4;
  {
    int kind;
    float lo, hi;
    iq36_synth_spec(IQ36_T_EMBED, 0, &kind, &lo, &hi);
    std::vector<uint16_t> row(H);
    // Row `token` of the fp16 [vocab, H] embedding table: elements
    // token*H .. token*H+H-1 of that tensor.
    for (int i = 0; i < H; ++i)
      row[i] = f2h(iq36_synth_normal(M.seed, iq36_tensor_id(-1, IQ36_T_EMBED, 0),
                                     (uint64_t)token * H + i, lo));
    for (int i = 0; i < H; ++i) h[i] = h2f(row[i]);
  }
  for (int l = 0; l < c.layers; ++l) {
    Layer& L = M.layers[l];
    if (hidden) std::memcpy(hidden + (int64_t)l * H, h.data(), sizeof(float) * H);
    orc_rms_norm(h.data(), 1, H, L.in_norm.data(), H, c.eps, xn.data());
    const auto x16 = to_f16(xn);
    if (L.attn) {
      const int D = c.head_dim;
      gemv16(L.q, x16.data(), FG, y, threads, M.precise);
      gemv16(L.k, x16.data(), FG, y2, threads, M.precise);
      gemv16(L.v, x16.data(), FG, y3, threads, M.precise);
      const auto qf = to_f16(y), kf = to_f16(y2), vf = to_f16(y3);
      std::vector<float> qo(c.nq * D), go(c.nq * D), kn(c.nkv * D), vn(c.nkv * D);
      orc_attn_prep(qf.data(), kf.data(), vf.data(), L.qn.data(), L.kn.data(), c.eps, pos, c.nq,
                    c.nkv, D, c.rope_dim, c.rope_base, qo.data(), go.data(), kn.data(),
                    vn.data());
      const int64_t slot = ((int64_t)M.bt[pos / 16] * 16 + pos % 16) * c.nkv * D;
      for (int i = 0; i < c.nkv * D; ++i) {
        L.kc[slot + i] = f2h(kn[i]);
        L.vc[slot + i] = f2h(vn[i]);
      }
      const auto q16 = to_f16(qo), g16 = to_f16(go);
      std::vector<float> att(c.nq * D);
      orc_paged_gqa(q16.data(), L.kc.data(), L.vc.data(), M.bt.data(), pos + 1, c.nq, c.nkv, D,
                    16, 1.0f / std::sqrt((float)D), g16.data(), att.data(), threads);
      const auto a16 = to_f16(att);
      gemv16(L.o, a16.data(), FG, y4, threads, M.precise);
    } else {
      const int C = (2 * c.nk + c.nv) * c.dk;
      gemv16(L.qkv, x16.data(), FG, y, threads, M.precise);
      gemv16(L.z, x16.data(), FG, y2, threads, M.precise);
      std::vector<float> ya, yb;
      gemv16(L.a, x16.data(), FG, ya, threads, M.precise);
      gemv16(L.b, x16.data(), FG, yb, threads, M.precise);
      const auto qkv16 = to_f16(y), z16 = to_f16(y2), a16 = to_f16(ya), b16 = to_f16(yb);
      std::vector<float> act(C), g(c.nv), beta(c.nv), o(c.nv * c.dk);
      orc_delta_prep(qkv16.data(), C, L.conv_state.data(), L.conv_w.data(), a16.data(),
                     b16.data(), L.a_log.data(), L.dt_bias.data(), c.nv, act.data(), g.data(),
                     beta.data());
      orc_delta_step(act.data(), g.data(), beta.data(), L.rec_state.data(), z16.data(),
                     L.dnorm.data(), c.eps, c.nk, c.nv, c.dk, o.data());
      const auto o16 = to_f16(o);
      gemv16(L.out, o16.data(), FG, y4, threads, M.precise);
    }
    for (int i = 0; i < H; ++i) h[i] += h2f(f2h(y4[i]));
    orc_rms_norm(h.data(), 1, H, L.post_norm.data(), H, c.eps, xn.data());
    const auto x2 = to_f16(xn);
    std::vector<float> lg(c.experts), w(c.topk), mo(H);
    std::vector<int32_t> ids(c.topk);
    float sl = 0.0f;
    orc_f16_linear(x2.data(), H, L.router.data(), c.experts, lg.data());
    orc_f16_linear(x2.data(), H, L.sgate.data(), 1, &sl);
    orc_router_select(lg.data(), 1, c.experts, c.topk, ids.data(), w.data());
    if (ids_out) std::memcpy(ids_out + (int64_t)l * c.topk, ids.data(), sizeof(int32_t) * c.topk);
    if (router_out)
      std::memcpy(router_out + (int64_t)l * c.experts, lg.data(), sizeof(float) * c.experts);
    if (M.lazy) {
      // the selected experts' rows into slots 0..k-1, then index by slot
      for (int r = 0; r < c.topk; ++r) {
        fill_u4_rows(L.gu, (int64_t)r * 2 * c.inter, (int64_t)ids[r] * 2 * c.inter, 2 * c.inter, H,
                     G, M.seed, l, IQ36_T_GU);
        fill_u4_rows(L.down, (int64_t)r * H, (int64_t)ids[r] * H, H, c.inter, G, M.seed, l,
                     IQ36_T_DOWN);
        ids[r] = r;
      }
    }
    orc_moe_decode(x2.data(), ids.data(), w.data(), c.topk, L.gu.w.data(), L.gu.s.data(),
                   L.gu.z.data(), L.down.w.data(), L.down.s.data(), L.down.z.data(),
                   L.sgu.w.data(), L.sgu.s.data(), L.sgu.z.data(), L.sdown.w.data(),
                   L.sdown.s.data(), L.sdown.z.data(), &sl, H, c.inter, G, mo.data(), M.precise,
                   threads);
    for (int i = 0; i < H; ++i) h[i] += h2f(f2h(mo[i]));
  }
  if (hidden) std::memcpy(hidden + (int64_t)c.layers * H, h.data(), sizeof(float) * H);
  if (!lm_head) return -1;
  orc_rms_norm(h.data(), 1, H, M.final_norm.data(), H, c.eps, xn.data());
  const auto xf = to_f16(xn);
  std::vector<float> lo;
  gemv16(M.lm_head, xf.data(), G, lo, threads, M.precise);
  if (logits) std::memcpy(logits, lo.data(), sizeof(float) * c.vocab);
  return orc_argmax(lo.data(), c.vocab);
}

}  // extern "C"
