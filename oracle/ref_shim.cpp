// ref_shim.cpp — extern "C" wrappers around the reference's own CPU model
// functions (engine/src/gguf_loader.cpp, compiled unchanged from the reference
// checkout by oracle/Makefile into oracle/_ref/libiq36_ref.so).
//
// TEST INFRASTRUCTURE ONLY: used to pin the CPU restatement
// (oracle/iq36_oracle.cpp) and to generate tests/golden/ fixtures. Nothing in
// the product path loads it.

#include <cstdint>
#include <cstring>
#include <vector>

#include "intel_qwen36/gguf_loader.hpp"

using iq36::RouterTopKSelection;

namespace iq36 {
// Defined with external linkage in gguf_loader.cpp:3410 but not declared in
// its header.
std::vector<float> apply_repeated_rms_norm(const std::vector<float>& input,
                                           const std::vector<float>& weight, float epsilon);
}  // namespace iq36

extern "C" {

float ref_sigmoid_scalar(float x) { return iq36::sigmoid_scalar(x); }

void ref_softmax(const float* logits, int n, float* out) {
  const auto p = iq36::softmax(std::vector<float>(logits, logits + n));
  std::memcpy(out, p.data(), sizeof(float) * n);
}

// select_router_topk, gguf_loader.cpp:3733-3743.
void ref_router_select(const float* logits, int E, int k, float min_weight_sum, int32_t* ids,
                       float* weights, float* normalized) {
  const RouterTopKSelection s =
      iq36::select_router_topk(std::vector<float>(logits, logits + E), k, min_weight_sum);
  for (int r = 0; r < k; ++r) {
    ids[r] = s.expert_ids[r];
    weights[r] = s.weights[r];
    normalized[r] = s.normalized_weights[r];
  }
}

// apply_swiglu_from_gate_up, :4640-4668.
void ref_swiglu_from_gate_up(const float* gate_up, int I, int n_exp, float* out) {
  const auto o = iq36::apply_swiglu_from_gate_up(
      std::vector<float>(gate_up, gate_up + (size_t)2 * I * n_exp), I, n_exp);
  std::memcpy(out, o.data(), sizeof(float) * o.size());
}

// apply_expert_weights (:3773-3797) then aggregate_experts (:3799-3819).
void ref_weight_aggregate(const float* down, const float* weights, int n_exp, int H, float* out) {
  const auto wd = iq36::apply_expert_weights(
      std::vector<float>(down, down + (size_t)n_exp * H),
      std::vector<float>(weights, weights + n_exp), H);
  const auto agg = iq36::aggregate_experts(wd, n_exp, H);
  std::memcpy(out, agg.data(), sizeof(float) * H);
}

// apply_rms_norm (:3368-3391) or apply_repeated_rms_norm (:3410-3439).
void ref_rms_norm(const float* in, int n, const float* w, int wlen, float eps, float* out) {
  std::vector<float> x(in, in + n), ww(w, w + wlen);
  const auto o = (wlen == n) ? iq36::apply_rms_norm(x, ww, eps)
                             : iq36::apply_repeated_rms_norm(x, ww, eps);
  std::memcpy(out, o.data(), sizeof(float) * n);
}

// run_qwen36_full_attention_core (:6071-6137) over a contiguous history
// k_hist/v_hist [T, nkv*D].
void ref_attention_core(const float* q, const float* k_hist, const float* v_hist, int T, int D,
                        int nq, int nkv, float scale, float* pregate) {
  std::vector<std::vector<float>> kh(T), vh(T);
  for (int t = 0; t < T; ++t) {
    kh[t].assign(k_hist + (size_t)t * nkv * D, k_hist + (size_t)(t + 1) * nkv * D);
    vh[t].assign(v_hist + (size_t)t * nkv * D, v_hist + (size_t)(t + 1) * nkv * D);
  }
  const auto r = iq36::run_qwen36_full_attention_core(std::vector<float>(q, q + (size_t)nq * D),
                                                      kh, vh, D, nq, nkv, scale);
  std::memcpy(pregate, r.attn_pregate.data(), sizeof(float) * nq * D);
}

// run_qwen36_full_attention_gate (:6034-6069); q_full [nq, 2, D].
void ref_attention_gate(const float* q_full, const float* pregate, int nq, int D, float* out) {
  const auto r = iq36::run_qwen36_full_attention_gate(
      std::vector<float>(q_full, q_full + (size_t)2 * nq * D),
      std::vector<float>(pregate, pregate + (size_t)nq * D), D);
  std::memcpy(out, r.attn_gated.data(), sizeof(float) * nq * D);
}

// run_qwen36_linear_attention_delta_core (:4670-4788) for nq query heads and
// nv value heads (value head v uses query head v % nq); state
// [nv, D(value row), D(key col)].
void ref_delta_core(const float* q, const float* k, const float* v, const float* gate,
                    const float* beta, const float* state, const float* z, const float* norm_w,
                    int nq, int nv, int D, float eps, float* attn_out, float* state_out,
                    float* final_out) {
  const auto r = iq36::run_qwen36_linear_attention_delta_core(
      std::vector<float>(q, q + (size_t)nq * D), std::vector<float>(k, k + (size_t)nq * D),
      std::vector<float>(v, v + (size_t)nv * D), std::vector<float>(gate, gate + nv),
      std::vector<float>(beta, beta + nv),
      std::vector<float>(state, state + (size_t)nv * D * D),
      std::vector<float>(z, z + (size_t)nv * D), std::vector<float>(norm_w, norm_w + D), eps);
  std::memcpy(attn_out, r.attention_output.data(), sizeof(float) * nv * D);
  std::memcpy(state_out, r.recurrent_state.data(), sizeof(float) * nv * D * D);
  std::memcpy(final_out, r.final_output.data(), sizeof(float) * nv * D);
}

}  // extern "C"
