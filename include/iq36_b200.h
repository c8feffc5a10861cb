/*
 * iq36_b200.h — C ABI of the B200 (sm_100a) batch-1 hot path of a
 * Qwen3.6-35B-A3B-shaped hybrid MoE.
 *
 * Conventions shared by every entry point:
 *   - all tensor pointers are caller-owned DEVICE memory;
 *   - work is enqueued on the caller's stream (cudaStream_t passed as void*;
 *     NULL = legacy default stream); no entry point synchronises or allocates;
 *   - the return value is 0 (IQ36_OK) or a negative iq36_status; shape and
 *     pointer checks happen on the host before any launch, so a failed call has
 *     enqueued nothing;
 *   - fp16 tensors are IEEE binary16 passed as uint16_t / void*;
 *   - kernels are launched with programmatic dependent launch (PDL). A kernel
 *     reads what earlier launches produce only after griddepcontrol.wait,
 *     except for its EARLY inputs, which it reads before that wait: weights
 *     (every entry point), and for the decode entries the position words
 *     (iq36_attn_prep), the conv state (iq36_delta_prep), the recurrent state
 *     (iq36_delta_step), the cache pages before the appended token
 *     (iq36_paged_gqa_decode) and the expert ids (the down-projection kernel
 *     of iq36_moe_decode).
 *     Rule for early inputs: let W be the most recent earlier launch on the
 *     stream that WAITS BEFORE IT RELEASES its dependents. An early input must
 *     not be written by W or by any launch after W. Everything launched before
 *     W has completed when the early read runs: W released only after its
 *     wait, i.e. after its predecessor completed, and every kernel of this
 *     library waits on its predecessor before it exits, so completion carries
 *     back through the whole stream (the early read relies on that completion
 *     having made the writes visible, as it does through L2; PTX promises
 *     visibility only after griddepcontrol.wait, and only for the prerequisite
 *     grid).
 *     Launches that RELEASE BEFORE THEY WAIT: the weight-streaming kernel of
 *     iq36_u4_gemv / iq36_u4_gemv_multi (G = 128, rows % 16 == 0, K % 512 ==
 *     0), iq36_attn_prep, and iq36_router_select (also the selection launch
 *     inside iq36_moe_block_decode and the four-launch form of
 *     iq36_moe_layer_decode). Every other launch waits first.
 *     Example: iq36_delta_prep reads the conv state early, so the sequence
 *     iq36_delta_prep, iq36_u4_gemv_multi, iq36_delta_prep on one stream needs
 *     a waiting launch between the two pre-steps (a decode step has several
 *     per layer: the recurrence, the embedding, the MoE layer's router).
 *
 * u4 matrix layout (the OpenVINO compressed-constant layout before the
 * reference's group-major repack; reference
 * tools/intel_qwen36_openvino_fixed_fc.py:107-144, shapes [M, K/G, G]):
 *   weight [rows, K/2] u8, two codes per byte, LOW nibble = even k
 *          (engine/openvino/custom/iq36_fixed_fc_multi_output.cl:122-124);
 *   scale  [rows, K/G] fp16;
 *   zp     [rows*K/G/2] u8, code (row, g) at element row*(K/G)+g, low nibble =
 *          even element (fixed_fc.py:240-248 unpacks the same way).
 *   w[row, k] = (q[row, k] - zp[row, k/G]) * scale[row, k/G].
 */
#ifndef IQ36_B200_H
#define IQ36_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* iq36_stream_t; /* cudaStream_t */

enum iq36_status {
  IQ36_OK = 0,
  IQ36_ERR_ARG = -1,       /* null pointer or bad enum value */
  IQ36_ERR_SHAPE = -2,     /* unsupported or inconsistent shape */
  IQ36_ERR_ALIGN = -3,     /* pointer alignment requirement violated */
  IQ36_ERR_WORKSPACE = -4, /* workspace missing or too small */
  IQ36_ERR_CUDA = -5,      /* CUDA runtime error at launch */
  IQ36_ERR_TIMEOUT = -6,   /* a bounded device-side wait expired */
  IQ36_ERR_DEVICE = -7     /* a device-side check wrote an error word */
};

enum iq36_dtype { IQ36_F32 = 0, IQ36_F16 = 1, IQ36_BF16 = 2 };

typedef struct {
  const uint8_t* weight;
  const uint16_t* scale;
  const uint8_t* zp;
  int32_t rows;
} iq36_u4_matrix;

/* One output of a multi-output u4 GEMV launch. accumulate=1 adds into an fp32
 * output (residual update) instead of overwriting it. */
typedef struct {
  iq36_u4_matrix m;
  void* out;
  int32_t out_dtype;
  int32_t accumulate;
} iq36_u4_projection;

/* A bank of E experts, each gate_up [2I, H] (rows 0..I-1 = gate, I..2I-1 = up)
 * and down [H, I], all u4 group-G, expert-major contiguous. */
typedef struct {
  const uint8_t* gate_up_weight;  /* [E, 2I, H/2]      */
  const uint16_t* gate_up_scale;  /* [E, 2I, H/G]      */
  const uint8_t* gate_up_zp;      /* [E, 2I*H/G/2]     */
  const uint8_t* down_weight;     /* [E, H, I/2]       */
  const uint16_t* down_scale;     /* [E, H, I/G]       */
  const uint8_t* down_zp;         /* [E, H*I/G/2]      */
  int32_t num_experts;
  int32_t hidden;
  int32_t intermediate;
  int32_t group;
} iq36_expert_bank;

const char* iq36_version(void);
const char* iq36_status_string(int status);

/* ---- (1) u4 group-wise asymmetric GEMV -------------------------------------
 * out[n] = sum_k x[k] * (q[n,k] - zp[n,k/G]) * scale[n,k/G]; fp32 accumulate,
 * out fp32 or fp16 (RTE).
 * Replaces the custom op IQ36FixedFC1 (engine/openvino/custom/
 * iq36_fixed_fc_multi_output.cl:36-44, scalar semantics :112-167; op class
 * tools/intel_qwen36_openvino_fixed_fc.py:31-92).
 * Requirements: G in {64,128}; K % G == 0; 16 <= K <= 16384; rows >= 1;
 * weight 16-byte aligned and K/2 % 16 == 0; x 16-byte aligned. */
int iq36_u4_gemv(const void* x_f16, int32_t K, int32_t G, const iq36_u4_matrix* w,
                 void* out, int32_t out_dtype, iq36_stream_t stream);

/* Arity-1..4 multi-output launch sharing one activation: replaces
 * IQ36FixedFC{1,3,4} (iq36_fixed_fc_multi_output.cl:6-29,45-85; grouping
 * fixed_fc.py:180-215). The optional fused prologue applies RMSNorm to an fp32
 * input before the GEMV (norm_weight != NULL): x = f16(in * rsqrt(mean(in^2) +
 * eps) * norm_weight), as gguf_loader.cpp:3368-3391 then the f16 Convert of
 * fixed_fc.py:292-296. x_f16 must be NULL in that case, and x_f32 set. */
int iq36_u4_gemv_multi(const void* x_f16, const float* x_f32, const float* norm_weight,
                       float norm_eps, int32_t K, int32_t G, int32_t n_proj,
                       const iq36_u4_projection* proj, iq36_stream_t stream);

/* ---- (4) router -------------------------------------------------------------
 * logits[t, e] = sum_h x[t,h] * W[e,h] (fp16 weights, fp32 accumulate); the
 * optional extra fp16 row (shared-expert gate, 2048->1) writes
 * shared_logit[t]. Replaces the router/shared-gate outputs of the
 * router_shared_input FC4 group (fixed_fc.py:166-177). */
int iq36_router_logits(const void* x_f16, const float* x_f32, const float* norm_weight,
                       float norm_eps, int32_t T, int32_t H, const void* w_router_f16,
                       int32_t E, const void* w_shared_gate_f16, float* logits,
                       float* shared_logit, iq36_stream_t stream);

/* Selection on fp32 logits, per token: probs = softmax (fp64 exp and sum,
 * rounded to fp32), ids = top-k by (prob desc, id asc), weights = probs[ids] /
 * max(sum_fp32(probs[ids]), 6.103515625e-5). Bit-exact restatement of
 * select_router_topk (engine/src/gguf_loader.cpp:3646-3743).
 * Requirements: 1 <= k <= 16, k <= E <= 256. */
int iq36_router_select(const float* logits, int32_t T, int32_t E, int32_t k,
                       int32_t* ids, float* weights, iq36_stream_t stream);

/* ---- (2a) MoE decode (batch 1) ---------------------------------------------
 * out = sum_{r<k} weights[r] * Down_{ids[r]}(SwiGLU(GateUp_{ids[r]}(x)))
 *       [+ sigmoid(shared_logit) * Down_s(SwiGLU(GateUp_s(x)))]
 * SwiGLU(g,u) = g*sigmoid(g)*u, rounded to fp16 as the down GEMV input; expert
 * sum in fp32 in rank order, shared expert added last.
 * Follows run_qwen36_moe_ffn_layer (engine/src/gguf_loader.cpp:5654-5782) and
 * the routed part of OpenVINO moe_3gemm_swiglu_opt (patch
 * engine/openvino/iq36-pr35924-grouped-postops.patch:86-124).
 * accumulate=1: out must be fp32 and receives out += result (residual).
 * The activation is x_f16, or (x_f16 NULL) the fp32 residual x_f32 normalised
 * in the kernel prologue with norm_weight/norm_eps as in iq36_u4_gemv_multi. */
int iq36_moe_decode(const void* x_f16, const float* x_f32, const float* norm_weight,
                    float norm_eps, const int32_t* ids, const float* weights, int32_t k,
                    const iq36_expert_bank* routed, const iq36_expert_bank* shared,
                    const float* shared_logit, void* out, int32_t out_dtype,
                    int32_t accumulate, void* workspace, size_t workspace_bytes,
                    iq36_stream_t stream);
size_t iq36_moe_decode_workspace_bytes(int32_t k, int32_t hidden, int32_t intermediate);

/* Expert-sharded form of iq36_moe_decode for expert-parallel decode (no
 * counterpart in the reference, which runs on one device): local_bank holds
 * the experts with global ids [expert_lo, expert_lo + local_bank->num_experts);
 * routed slots whose expert lies outside that range read no weights and
 * contribute zero, so summing the outputs of all ranks (one allreduce) gives
 * the full block. Pass the shared expert on exactly one rank. */
int iq36_moe_decode_sharded(const void* x_f16, const float* x_f32, const float* norm_weight,
                            float norm_eps, const int32_t* ids, const float* weights, int32_t k,
                            const iq36_expert_bank* local_bank, int32_t expert_lo,
                            const iq36_expert_bank* shared, const float* shared_logit, void* out,
                            int32_t out_dtype, int32_t accumulate, void* workspace,
                            size_t workspace_bytes, iq36_stream_t stream);

/* Config-1 block: router logits -> select -> routed + shared experts.
 * ids/weights/logits are outputs (device). */
int iq36_moe_block_decode(const void* x_f16, const void* w_router_f16, const void* w_shared_gate_f16,
                          int32_t k, const iq36_expert_bank* routed,
                          const iq36_expert_bank* shared, int32_t* ids, float* weights,
                          float* logits, void* out, int32_t out_dtype, void* workspace,
                          size_t workspace_bytes, iq36_stream_t stream);
size_t iq36_moe_block_decode_workspace_bytes(int32_t k, int32_t hidden, int32_t intermediate);

/* One decode MoE FFN layer on the fp32 residual stream, as
 * run_qwen36_moe_ffn_layer (engine/src/gguf_loader.cpp:5654-5782) with the
 * post-attention RMSNorm in front (:3368-3391):
 *   x = rms_norm(residual) * norm_weight, rounded to fp16;
 *   logits = W_router x (fp32, [E]); shared_logit = w_shared_gate . x;
 *   ids, weights = top-k of softmax(logits) (as iq36_router_select);
 *   residual += f16(sum_r weights[r] * Expert_{ids[r]}(x)
 *                   + sigmoid(shared_logit) * Shared(x)).
 * ids / weights / logits / shared_logit are device outputs.
 * At the config-4 shapes (group 128, hidden <= 2048 and a multiple of 512,
 * intermediate 256 or 512, E <= 256, k <= 15, 16-byte aligned down scales and
 * zero points) this is ONE persistent launch, one CTA per SM, whose phases
 * (router | top-k + routed gate_up | down + combine) are separated by two grid
 * barriers kept in the workspace; other shapes run four launches (router,
 * top-k, gate_up + SwiGLU, down + combine). Both forms give the same bits.
 * workspace: 16-byte aligned, iq36_moe_layer_decode_workspace_bytes long,
 * ZERO-FILLED before its first use; it stays valid across calls (the barrier
 * words return to rest after each call). Calls sharing one workspace must be
 * ordered on one stream. If iq36_wait_timeouts reports a timeout, zero the
 * workspace again before the next call. */
int iq36_moe_layer_decode(float* residual, int32_t hidden, const float* norm_weight,
                          float norm_eps, const void* w_router_f16, const void* w_shared_gate_f16,
                          int32_t k, const iq36_expert_bank* routed,
                          const iq36_expert_bank* shared, int32_t* ids, float* weights,
                          float* logits, float* shared_logit, void* workspace,
                          size_t workspace_bytes, iq36_stream_t stream);
size_t iq36_moe_layer_decode_workspace_bytes(int32_t k, int32_t hidden, int32_t intermediate);

/* iq36_moe_layer_decode for a rank of tensor-parallel decode (no counterpart
 * in the single-device reference): the banks hold this rank's slice of every
 * expert's intermediate rows (gate and up rows, the matching K slice of down),
 * and instead of updating the residual the call writes this rank's fp32 share
 * of the layer output, partial_out[hidden] = sum_r w_r Down_r(SwiGLU(..)) +
 * sigmoid(g) Shared(..) over its rows; the residual is only read. The ranks'
 * partials summed (iq36_tp_allreduce_residual) give the layer output. Same
 * workspace rules as iq36_moe_layer_decode. */
int iq36_moe_layer_decode_partial(const float* residual, int32_t hidden, const float* norm_weight,
                                  float norm_eps, const void* w_router_f16,
                                  const void* w_shared_gate_f16, int32_t k,
                                  const iq36_expert_bank* routed, const iq36_expert_bank* shared,
                                  int32_t* ids, float* weights, float* logits,
                                  float* shared_logit, float* partial_out, void* workspace,
                                  size_t workspace_bytes, iq36_stream_t stream);

/* ---- (2b) grouped MoE prefill ----------------------------------------------
 * For T tokens with top-k routing (ids, weights [T,k]): permute token rows by
 * expert (stable: by expert, then token, then rank), per expert
 * Y = fp16(weights * SwiGLU(X W_gu^T) W_d^T) on tcgen05 tensor cores (x as fp16,
 * u4 dequantised to fp16 in shared memory, fp32 accumulate), then
 * out[t] = sum_{r<k} Y[row(t,r)] in rank order in fp32. Follows the Gen-1
 * schedule grouped_s8_u4_f16_contribution_moe.cl:13-222 with its fp16
 * contribution scatter :831-845, and the stock gather/GEMM/scatter of
 * iq36-pr35924-grouped-postops.patch:15-124. x bf16 [T, H]; out fp32, bf16 or
 * fp16 (with k = 1 the fp16 output is the contribution itself, exactly).
 * Requirements: H % 256 == 0, I % 128 == 0, H, I <= 2048, G == 128 or 64. */
int iq36_moe_prefill(const void* x_bf16, int32_t T, const int32_t* ids, const float* weights,
                     int32_t k, const iq36_expert_bank* routed, void* out, int32_t out_dtype,
                     void* workspace, size_t workspace_bytes, iq36_stream_t stream);
/* The MoE block of one decoder layer over T prompt tokens, fp32 residual
 * [T, hidden] updated in place: router logits on RMSNorm(residual) (the
 * decode router's fp16 input bit for bit; the logits on tensor cores, equal
 * to the decode router's up to fp32 summation order, within the reference's
 * 1e-4 router gate), top-k
 * selection (ids, weights [T, k]; logits [T, E] kept for inspection), the
 * routed experts as in iq36_moe_prefill (x = fp16 RMSNorm(residual); fp16
 * contributions summed in rank order, added to the residual), and the shared
 * expert (when `shared` is set) as dense tcgen05 GEMMs: SwiGLU(x Wgu^T), then
 * residual += fp16(sigmoid(x . w_shared_gate) * (act Wd^T)).
 * run_qwen36_moe_ffn_layer (gguf_loader.cpp:5654-5782) over a prompt, grouped
 * schedule of grouped_s8_u4_f16_contribution_moe.cl:13-222.
 * Requirements: those of iq36_moe_prefill; the shared bank has the routed
 * bank's hidden, intermediate and group. workspace:
 * iq36_moe_layer_prefill_workspace_bytes. */
int iq36_moe_layer_prefill(float* residual, int32_t T, int32_t hidden, const float* norm_weight,
                           float norm_eps, const void* w_router_f16,
                           const void* w_shared_gate_f16, int32_t k,
                           const iq36_expert_bank* routed, const iq36_expert_bank* shared,
                           int32_t* ids, float* weights, float* logits, void* workspace,
                           size_t workspace_bytes, iq36_stream_t stream);
size_t iq36_moe_layer_prefill_workspace_bytes(int32_t T, int32_t k, int32_t num_experts,
                                              int32_t hidden, int32_t intermediate);

/* Dense u4 GEMM for batched (prefill) projections: out[T, N] = x W^T with
 * W = (q - zp) * s (group 128 or 64 along K: the reference's fixed FCs are
 * group 64, fixed_fc.py:26), fp16 operands on tcgen05 tensor cores,
 * fp32 accumulate. x is fp16 [T, K], or fp32 [T, K] optionally RMS-normalised
 * in the prologue with norm_weight / norm_eps and rounded to fp16 (as the
 * decode projections do). out: fp16 [T, N] store, or fp32 [T, N] store
 * (accumulate = 0) or residual update out += f16(x W^T) (accumulate = 1).
 * The batched form of the fixed-FC projections (IQ36FixedFC over [T, K],
 * tools/intel_qwen36_openvino_fixed_fc.py:31-92; the prefill buckets of the
 * OpenVINO graph run the same FCs with M = T). Requirements: group 128 or 64,
 * K % 256 == 0, K <= 4096, N % 256 == 0; x and norm_weight 16-byte aligned. */
int iq36_u4_gemm(const void* x, int32_t x_dtype, const float* norm_weight, float norm_eps,
                 int32_t T, int32_t K, int32_t group, const iq36_u4_matrix* w, void* out,
                 int32_t out_dtype, int32_t accumulate, void* workspace, size_t workspace_bytes,
                 iq36_stream_t stream);
size_t iq36_u4_gemm_workspace_bytes(int32_t T, int32_t K);

/* iq36_u4_gemm for 1..4 projections that share the input x (same K), in one
 * input preparation and one persistent GEMM launch whose units span all of
 * them: proj[p].out [T, proj[p].m.rows] (fp16, or fp32 with accumulate).
 * Each m.rows a multiple of 256. The batched form of the reference's
 * multi-output fixed-FC groups (iq36_fixed_fc_multi_output.cl:6-29,45-85;
 * grouping fixed_fc.py:180-215) over a prompt chunk. Workspace as
 * iq36_u4_gemm_workspace_bytes(T, K). */
int iq36_u4_gemm_multi(const void* x, int32_t x_dtype, const float* norm_weight, float norm_eps,
                       int32_t T, int32_t K, int32_t group, int32_t n_proj,
                       const iq36_u4_projection* proj, void* workspace, size_t workspace_bytes,
                       iq36_stream_t stream);

/* out[t] = sum_{r<k} float(contrib[inv[t*k + r]]) in rank order (fp32 sums of
 * fp16 contribution rows [*, H]); out fp32, bf16 or fp16 [T, H]. The
 * contribution scatter of the grouped prefill on its own, for callers that
 * compute contributions elsewhere (the expert-parallel combine):
 * iq36_scatter_f16_contributions, grouped_s8_u4_f16_contribution_moe.cl:831-845. */
int iq36_moe_combine(const void* contrib_f16, const int32_t* inv, int32_t T, int32_t H, int32_t k,
                     void* out, int32_t out_dtype, iq36_stream_t stream);
size_t iq36_moe_prefill_workspace_bytes(int32_t T, int32_t k, int32_t num_experts,
                                        int32_t hidden, int32_t intermediate);

/* Per-assignment contributions over deduplicated input rows, for the owner
 * side of expert-parallel prefill (no counterpart in the single-device
 * reference): contrib[a] = fp16(weights[a] * Expert_{ids[a]}(x[row_of[a]]))
 * for a < n_assign, x bf16 [n_rows, H], contrib fp16 [n_assign, H] — the same
 * fp16 values iq36_moe_prefill sums, so combining them in slot order with
 * iq36_moe_combine reproduces it bit for bit. row_of entries are clamped to
 * [0, n_rows). n_assign == 0 enqueues nothing. Workspace:
 * iq36_moe_prefill_rows_workspace_bytes. */
int iq36_moe_prefill_rows(const void* x_bf16, int32_t n_rows, int32_t n_assign,
                          const int32_t* row_of, const int32_t* ids, const float* weights,
                          const iq36_expert_bank* routed, void* contrib_f16, void* workspace,
                          size_t workspace_bytes, iq36_stream_t stream);
size_t iq36_moe_prefill_rows_workspace_bytes(int32_t n_assign, int32_t num_experts,
                                             int32_t hidden, int32_t intermediate);

/* ---- (3) paged GQA decode attention ----------------------------------------
 * o[h] = sum_t softmax_t(q[h].k[t,h/grp] * scale) v[t,h/grp], then
 * o *= sigmoid(gate[h]) when gate != NULL. KV cache fp16
 * [num_blocks, block_size, n_kv_heads, head_dim] (K and V separate); token t
 * lives in block block_table[t / block_size], slot t % block_size.
 * Split-K flash decode; follows run_qwen36_full_attention_core
 * (gguf_loader.cpp:6071-6137), the gate run_qwen36_full_attention_gate
 * (:6034-6069) and the split/reduce structure of
 * engine/gpu/opencl/fused_gqa_fp16_kv_decode.cl:16-115.
 * ctx_len_dev (optional, device int32) overrides ctx_len at run time so a
 * captured CUDA graph can be replayed as the context grows; ctx_len is then the
 * capacity that sizes the launch.
 * Requirements: head_dim == 256, n_q_heads / n_kv_heads == 8, block_size == 16. */
int iq36_paged_gqa_decode(const void* q_f16, const void* k_cache, const void* v_cache,
                          const int32_t* block_table, int32_t ctx_len, const int32_t* ctx_len_dev,
                          int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim,
                          int32_t block_size, float scale, const void* gate_f16, void* out,
                          int32_t out_dtype, void* workspace, size_t workspace_bytes,
                          iq36_stream_t stream);
size_t iq36_paged_gqa_workspace_bytes(int32_t max_ctx, int32_t n_q_heads, int32_t n_kv_heads,
                                      int32_t head_dim);

/* Allocation-free form of iq36_paged_gqa_decode. It has no counterpart in the
 * reference. Some callers cannot allocate device memory for a workspace: a
 * graph-plugin host that passes an op only its input and output buffers, or a
 * service held to a fixed device-memory budget with no allocator available to
 * the op. Here the split partials live in one static device array inside the
 * library (4,887,552 bytes, held by every GPU that loads the library until the
 * process exits), sized for n_kv_heads <= 2 (n_q_heads <= 16) at any ctx_len;
 * larger head counts return IQ36_ERR_WORKSPACE. The call allocates nothing.
 * The first call on each device looks up the array's device address (with that
 * device current), so make that first call before any stream capture. All
 * calls share the array and it keeps the last call's contents (nothing in it
 * has to start zeroed); calls whose kernels overlap on the GPU race on it. */
int iq36_paged_gqa_decode_noalloc(const void* q_f16, const void* k_cache, const void* v_cache,
                                  const int32_t* block_table, int32_t ctx_len,
                                  const int32_t* ctx_len_dev, int32_t n_q_heads,
                                  int32_t n_kv_heads, int32_t head_dim, int32_t block_size,
                                  float scale, const void* gate_f16, void* out, int32_t out_dtype,
                                  iq36_stream_t stream);

/* ---- config-4 support ops ---------------------------------------------------*/

/* out[r] = f(in[r] * rsqrt(mean(in[r]^2) + eps) * weight); gguf_loader.cpp:3368-3391
 * (rows of dim), apply_repeated_rms_norm :3410-3439 when weight_len < dim. */
int iq36_rms_norm(const float* in, int32_t rows, int32_t dim, const float* weight,
                  int32_t weight_len, float eps, void* out, int32_t out_dtype,
                  iq36_stream_t stream);

/* Full-attention pre-step for one token: split q_full [n_q, 2, D] into q and
 * gate, per-head RMSNorm of q and k (weights [D]), partial rotate-half RoPE on
 * the first rope_dim dims at position *pos_dev (base rope_base), write q_out
 * [n_q, D] f16 and gate_out [n_q, D] f16, and append k, v (f16 [n_kv, D]) at
 * token *pos_dev of the paged cache. gguf_loader.cpp:5928-5950 (split/norm),
 * engine/openvino/custom/iq36_qk_rope_layout.cl:12-60 (rotate-half on dims <
 * 64), iq36_hot_ring_update.cl:7-28 (slot write). */
int iq36_attn_prep(const void* q_full_f16, const void* k_f16, const void* v_f16,
                   const float* q_norm_w, const float* k_norm_w, float eps,
                   const int32_t* pos_dev, int32_t n_q_heads, int32_t n_kv_heads,
                   int32_t head_dim, int32_t rope_dim, float rope_base,
                   const int32_t* block_table, int32_t block_size, void* k_cache,
                   void* v_cache, void* q_out_f16, void* gate_out_f16, iq36_stream_t stream);

/* iq36_attn_prep for `tokens` consecutive tokens at positions *pos_dev + t
 * (t = 0..tokens-1) in one launch: per token, rows q_full [n_q, 2, D],
 * k/v [n_kv, D], q_out/gate_out [n_q, D] (row-contiguous over tokens). The
 * batched form of the reference's per-token prompt loop over this pre-step. */
int iq36_attn_prep_batch(const void* q_full_f16, const void* k_f16, const void* v_f16,
                         const float* q_norm_w, const float* k_norm_w, float eps,
                         const int32_t* pos_dev, int32_t tokens, int32_t n_q_heads,
                         int32_t n_kv_heads, int32_t head_dim, int32_t rope_dim,
                         float rope_base, const int32_t* block_table, int32_t block_size,
                         void* k_cache, void* v_cache, void* q_out_f16, void* gate_out_f16,
                         iq36_stream_t stream);

/* Causal prompt attention: queries q_f16 [T, n_q, D] at positions
 * *pos_dev + t attend to cache keys 0 .. *pos_dev + t (K/V of the prompt
 * already appended by iq36_attn_prep_batch); out [T, n_q, D] (f32 or f16) =
 * softmax(q k^T * scale) v, times sigmoid(gate [T, n_q, D]) when gate_f16 is
 * not NULL. Equal to iq36_paged_gqa_decode run for each prompt token in turn
 * (run_qwen36_full_attention_core, gguf_loader.cpp:6071-6137; gate :6034-6069).
 * head_dim 256, n_q_heads == 8 * n_kv_heads, block_size 16; num_blocks = the
 * caches' block count (a table entry past it reads zeros). Allocates nothing. */
int iq36_attn_prefill(const void* q_f16, const void* k_cache, const void* v_cache,
                      const int32_t* block_table, int32_t block_size, int32_t num_blocks,
                      const int32_t* pos_dev, int32_t tokens, int32_t n_q_heads,
                      int32_t n_kv_heads, int32_t head_dim, float scale, const void* gate_f16,
                      void* out, int32_t out_dtype, iq36_stream_t stream);

/* DeltaNet pre-step for one token: causal depthwise conv (width 4, carried
 * state [C,4]) + SiLU with the fp16 rounding points of
 * engine/openvino/custom/iq36_linear_conv_swish.cl:12-64, and the gate/beta
 * transform g = -exp(A_log) * softplus(a + dt_bias), beta = sigmoid(b)
 * (gguf_loader.cpp:4875-4912). qkv_act_f16 [C]; g_out, beta_out fp32 [nv]. */
int iq36_delta_prep(const void* qkv_f16, int32_t channels, float* conv_state,
                    const float* conv_w, const void* a_f16, const void* b_f16,
                    const float* a_log, const float* dt_bias, int32_t n_v_heads,
                    void* qkv_act_f16, float* g_out, float* beta_out, iq36_stream_t stream);

/* Gated DeltaNet recurrence for one token, OpenVINO head mapping (key head =
 * value head / (nv/nk)), L2 norm rsqrt(sum+1e-6), q * 1/sqrt(D); state
 * [nv, D(key), D(value)] fp32 updated in place; then gated RMSNorm
 * o * rsqrt(mean(o^2)+eps) * norm_w * silu(z) -> f16.
 * engine/openvino/custom/iq36_gated_delta_net.cl:36-150,
 * gguf_loader.cpp:4770-4786. */
int iq36_delta_step(const void* qkv_act_f16, const float* g, const float* beta, float* state,
                    const void* z_f16, const float* norm_w, float eps, int32_t n_k_heads,
                    int32_t n_v_heads, int32_t head_dim, void* out_f16, iq36_stream_t stream);

/* The DeltaNet block over T prompt tokens: the arithmetic of iq36_delta_prep
 * followed by iq36_delta_step for tokens 0..T-1 in order (conv state and
 * recurrent state carried in and out), in five launches; from 16 chunks of
 * 32 tokens on, the recurrence runs as two segments at once plus a join
 * launch (same result within fp32 rounding, not bit for bit, and more
 * workspace: query it for each token count). Replaces the
 * per-token loop over the reference's linear-attention layer during prompt
 * processing (iq36_linear_conv_swish.cl:12-64, iq36_gated_delta_net.cl:36-150,
 * gguf_loader.cpp:4770-4786 and :4875-4912).
 * qkv_f16 [T, (2nk+nv)*D] (row-contiguous); a_f16/b_f16 [T, *] with row
 * stride gate_stride >= nv halves (the a and b projections may share one
 * padded matrix); z_f16 [T, nv*D]; out_f16 [T, nv*D]. head_dim must be 128;
 * nv % nk == 0; nv <= 256. workspace: iq36_delta_prefill_workspace_bytes. */
int iq36_delta_prefill(const void* qkv_f16, int32_t tokens, int32_t n_k_heads,
                       int32_t n_v_heads, int32_t head_dim, float* conv_state,
                       const float* conv_w, const void* a_f16, const void* b_f16,
                       int32_t gate_stride, const float* a_log, const float* dt_bias,
                       float* state, const void* z_f16, const float* norm_w, float eps,
                       void* out_f16, void* workspace, size_t workspace_bytes,
                       iq36_stream_t stream);
size_t iq36_delta_prefill_workspace_bytes(int32_t tokens, int32_t n_k_heads,
                                          int32_t n_v_heads);

/* Decode-loop position state on the device: *pos_dev += advance (1 after a
 * decode step, the prompt length after a batched prefill, 0 to refresh); then
 * *ctx_dev = *pos_dev + 1 (the attention context of the step at *pos_dev).
 * Lets one captured CUDA graph serve every step of the loop
 * (the reference's per-token loop: engine/service/iq36_server/runtime.py:533-561).
 * advance < 0 returns IQ36_ERR_SHAPE. */
int iq36_decode_positions(int32_t* pos_dev, int32_t* ctx_dev, int32_t advance,
                          iq36_stream_t stream);

/* h[:] = float(embedding[*token_dev, :]) (fp16 table [vocab, H]). */
int iq36_embed(const void* table_f16, int32_t vocab, int32_t hidden, const int32_t* token_dev,
               float* h, iq36_stream_t stream);

/* h[t, :] = float(embedding[tokens_dev[t], :]) for t < T (1 <= T <= 65535):
 * the prompt's embedding rows for the batched prefill. */
int iq36_embed_batch(const void* table_f16, int32_t vocab, int32_t hidden,
                     const int32_t* tokens_dev, int32_t T, float* h, iq36_stream_t stream);

/* u4 layout adapter. The reference's fixed-FC custom op consumes each
 * projection's scales and zero points in group-major order
 * (tools/intel_qwen36_openvino_fixed_fc.py:218-258: scale fp16 [groups, rows],
 * zero points u4 [groups, rows] packed two per byte, low nibble first; the u4
 * weight bytes unchanged). from_group_major writes the row-major layout of
 * this header (scale [rows, groups], zp [rows*groups] packed) from that form;
 * to_group_major is the inverse. rows*groups must be even. No counterpart
 * call in the reference (it repacks on the host while building the graph). */
int iq36_u4_layout_from_group_major(const void* scale_gm_f16, const uint8_t* zp_gm,
                                    int32_t rows, int32_t groups, void* scale_f16, uint8_t* zp,
                                    iq36_stream_t stream);
int iq36_u4_layout_to_group_major(const void* scale_f16, const uint8_t* zp, int32_t rows,
                                  int32_t groups, void* scale_gm_f16, uint8_t* zp_gm,
                                  iq36_stream_t stream);

/* Greedy top-1 over fp32 logits, lowest id on ties: per-block maxima of the
 * 64-bit key (order-preserving fp32 bits, inverted id), then one merge block
 * (engine/openvino/custom/iq36_greedy_top1.cl:8-46 and
 * iq36_greedy_top1_merge.cl). token_out int32[1]; workspace holds the
 * per-block keys (no initialisation needed). */
int iq36_argmax(const float* logits, int32_t n, int32_t* token_out, void* workspace,
                size_t workspace_bytes, iq36_stream_t stream);
size_t iq36_argmax_workspace_bytes(void);

/* ---- LM-head certified greedy top-1 -----------------------------------------
 * The reference's certificate (engine/gpu/opencl/
 * iq36_lm_head_affine_q4_group128_component.cl:126-217 bound scan and
 * candidate selection, :219-300 exact candidates and top-1, the full path as
 * capacity fallback) for the u4 group-128 head. Every row's logit is bounded
 * by sum_g |s_rg| ||q_rg - zp_rg||_2 ||x_g||_2 plus a guard covering the fp32
 * rounding of the full head's group sums. The best row of *seed_token's
 * 16-row chunk, computed in fp32 and lowered by twice its guard, sets the
 * bar; every chunk holding a row whose bound reaches the bar is computed by
 * the full head's own kernel (chunk-list mode), so token_out equals the full
 * head's argmax (lowest id on ties) bit for bit. More than capacity_chunks
 * such chunks: every chunk (the full head). logits [rows] receives the
 * evaluated chunks' logits only; *evaluated_chunks (optional, device) their
 * number. Four launches (prep, bound scan, GEMV, argmax), PDL-chained.
 * Requirements: those of the weight-streaming GEMV (G 128, rows % 16 == 0,
 * K % 512 == 0, K <= 4096). table: iq36_lm_head_cert_table_bytes bytes,
 * written once per head by iq36_lm_head_cert_table ([rows, K/128] fp16
 * |s| * group norm rounded up, then [rows] fp16 max |s|).
 * seed_token may alias token_out (it is read before token_out is written). */
size_t iq36_lm_head_cert_table_bytes(int32_t rows, int32_t K, int32_t G);
int iq36_lm_head_cert_table(const iq36_u4_matrix* w, int32_t K, int32_t G, void* table_f16,
                            iq36_stream_t stream);
size_t iq36_lm_head_top1_certified_workspace_bytes(int32_t rows, int32_t K);
int iq36_lm_head_top1_certified(const void* x_f16, const float* x_f32, const float* norm_weight,
                                float norm_eps, int32_t K, int32_t G, const iq36_u4_matrix* w,
                                const void* table_f16, const int32_t* seed_token,
                                int32_t capacity_chunks, float* logits, int32_t* token_out,
                                int32_t* evaluated_chunks, void* workspace,
                                size_t workspace_bytes, iq36_stream_t stream);

/* Fill device buffers with the synthetic generator of iq36_synth.h.
 * kind: 0 = u8 codes, 1 = fp16 uniform [lo,hi), 2 = fp16 normal(std=lo),
 * 3 = fp32 uniform [lo,hi), 4 = fp32 normal(std=lo). */
int iq36_synth_fill(void* dst, int64_t count, int32_t kind, uint64_t seed, uint64_t tensor,
                    float lo, float hi, iq36_stream_t stream);
/* Tensor naming and distributions of the synthetic model (iq36_synth.h). */
uint64_t iq36_synth_tensor_id(int32_t layer, int32_t slot, int32_t sub);
void iq36_synth_tensor_spec(int32_t slot, int32_t sub, int32_t* kind, float* lo, float* hi);

/* ---- tensor-parallel decode exchange ---------------------------------------
 * No counterpart in the reference (it runs on one device). The north star
 * row-shards the decode GEMVs across 2/4/8 GPUs and completes every
 * row-parallel sub-block with an allreduce over NVLink; these entry points
 * are that exchange, one small kernel each. Every rank owns one device buffer
 * of iq36_tp_comm_bytes(world, hidden) bytes, ZERO-FILLED before first use:
 *   [recv: 2 x world x hidden fp32][flags: world u32, 256-byte region]
 *   [keys: 2 x world u64][counter: u32]
 * shared with the other ranks through CUDA IPC (iq36_ipc_get_handle /
 * iq36_ipc_open_handle). iq36_tp_comm holds, for every rank q, rank q's
 * receive buffer, flag words and key slots as mapped in this process
 * (peer_*[rank] = this rank's own), plus this rank's own buffers and its
 * counter. Exchanges are one-shot: plain peer stores of this rank's data into
 * every rank's slot, then a system-scope release of a per-call sequence
 * number in every rank's flag word, then bounded polling (200 ms) of the
 * world flags of this rank's own buffer; double-buffered by the call parity.
 * All ranks must issue the same sequence of exchanges. A wait that expires is
 * counted by iq36_wait_timeouts and leaves the output untouched; the comm
 * buffers must then be zeroed again on every rank. */
typedef struct {
  int32_t rank, world, hidden;
  float* peer_recv[8];
  uint32_t* peer_flags[8];
  unsigned long long* peer_keys[8];
  float* local_recv;
  uint32_t* local_flags;
  unsigned long long* local_keys;
  uint32_t* counter;
} iq36_tp_comm;
size_t iq36_tp_comm_bytes(int32_t world, int32_t hidden);
/* Set-up only (the one allocating call of this library, made once per rank
 * before any exchange): a zero-filled cudaMalloc allocation of `bytes` for
 * the exchange buffer (an IPC handle must name a whole allocation), and its
 * release after every rank has unmapped it. Synchronises the device. */
int iq36_tp_comm_alloc(size_t bytes, void** dev_ptr);
int iq36_tp_comm_free(void* dev_ptr);
/* 64-byte CUDA IPC handle of a device allocation / its mapping in this
 * process (peer access enabled lazily) / unmapping. */
int iq36_ipc_get_handle(const void* dev_ptr, void* handle_64);
int iq36_ipc_open_handle(const void* handle_64, void** dev_ptr);
int iq36_ipc_close_handle(void* dev_ptr);
/* residual[i] += f16(sum over ranks q, in rank order, of partial_q[i]) on
 * every rank: the allreduce that completes a row-parallel sub-block, with the
 * single-GPU step's fp16 rounding of the sub-block output. partial [hidden]
 * fp32, 16-byte aligned; hidden % 4 == 0; world <= 8. */
int iq36_tp_allreduce_residual(const iq36_tp_comm* comm, float* residual, const float* partial,
                               iq36_stream_t stream);
/* Greedy top-1 over a vocab split: this rank's logits_local [n_local] hold
 * global ids id0 .. id0 + n_local - 1; every rank ends with the global argmax
 * (lowest id on ties, iq36_greedy_top1.cl:8-13) in token_out. key_ws:
 * iq36_tp_argmax_workspace_bytes() device bytes. */
int iq36_tp_argmax(const iq36_tp_comm* comm, const float* logits_local, int32_t n_local,
                   int32_t id0, int32_t* token_out, void* key_ws, iq36_stream_t stream);
size_t iq36_tp_argmax_workspace_bytes(void);

/* Programmatic dependent launch on (default) or off for every later launch
 * of this library in the process. */
void iq36_set_pdl(int enabled);

/* Number of bounded device waits that gave up on the current device since the
 * last reset (decode weight-streaming rings, the tcgen05 GEMM and attention
 * pipelines); a non-zero count means some output of those launches is
 * invalid. reset != 0 clears the counters after reading.
 * No counterpart in the reference (its kernels hold no cross-warp waits). */
int iq36_wait_timeouts(int32_t* count, int32_t reset);

#ifdef __cplusplus
}
#endif

#endif /* IQ36_B200_H */
