// paged_gqa.cu — paged GQA decode attention over an fp16 block-table KV cache.
//
// Semantics: run_qwen36_full_attention_core (engine/src/gguf_loader.cpp:
// 6071-6137; score = q.k * scale, softmax over the history, sum w*v) with the
// output gate of run_qwen36_full_attention_gate (:6034-6069, o *
// sigmoid(gate)). Structure after the reference's split-K decode
// (engine/gpu/opencl/fused_gqa_fp16_kv_decode.cl:16-115: per (kv head, chunk)
// partial max / sum / output, then a reduce with the fused sigmoid gate), with
// the value weights rounded to fp16 before the P.V product as in
// engine/openvino/custom/iq36_full_attention_gqa.cl:26-135.
//
// Layout: K and V caches [num_blocks, 16, n_kv, 256] fp16; token t in block
// block_table[t/16], slot t%16.
//
// Kernel 1 (split): grid (S/4, n_kv), 4 warps; each warp owns one split of
// contiguous 16-token pages and keeps an online softmax for the 8 query heads
// of its KV head. Pages stream through a 3-stage per-warp cp.async ring (K and
// V, 16 KB per page, XOR-swizzled rows for conflict-free ldmatrix).
//   S^T = K Q^T   m16n8k16: M = 16 tokens, N = 8 heads, K = 256 dims;
//   O^T += V^T P^T m16n8k16: M = 16 dims (x16 tiles), N = 8 heads, K = 16 tokens;
// the P tile is transposed in registers with movmatrix. Scores are kept in
// log2 units (scale * log2 e folded in), fp32 throughout, P in fp16.
// Kernel 2 (combine): per (query head, 32-dim slice) merge the S partials
// (max, sum, output), normalise, apply sigmoid(gate), store fp32 or fp16.

#include <atomic>

#include "launch.cuh"
#include "common.cuh"

namespace iq36 {

constexpr int kD = 256;
constexpr int kGrp = 8;
constexpr int kBS = 16;
constexpr int kStages = 3;
constexpr int kPageBytes = kBS * kD * 2;          // one K (or V) page of one kv head
constexpr int kStageBytes = 2 * kPageBytes;       // K + V
constexpr int kWarpSmem = kStages * kStageBytes;  // 48 KB
constexpr int kMaxSplits = 296;

struct GqaArgs {
  const __half* q;
  const __half* kc;
  const __half* vc;
  const int32_t* bt;
  int ctx;
  const int32_t* ctx_dev;
  int n_kv;
  int S;  // splits per kv head (= gridDim.x * 4)
  float scale_log2;
  float* ws_m;
  float* ws_l;
  float* ws_acc;
};

__device__ __forceinline__ void gqa_issue_page(const GqaArgs& a, int kvh, int page, int ctx,
                                               uint32_t stage_base, int lane) {
  const int blk = __ldg(a.bt + page);
  const size_t row_stride = (size_t)a.n_kv * kD;  // halfs between consecutive slots
  const __half* kb = a.kc + ((size_t)blk * kBS) * row_stride + (size_t)kvh * kD;
  const __half* vb = a.vc + ((size_t)blk * kBS) * row_stride + (size_t)kvh * kD;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int c = lane + 32 * i;  // 0..511: 16 rows x 32 chunks of 16 B
    const int r = c >> 5, cc = c & 31;
    const int valid = (page * kBS + r) < ctx ? 16 : 0;
    const uint32_t off = (uint32_t)(r * 512 + ((cc ^ (r & 7)) << 4));
    const size_t goff = (size_t)r * row_stride + (size_t)cc * 8;
    cp_async_16(stage_base + off, kb + goff, valid);
    cp_async_16(stage_base + kPageBytes + off, vb + goff, valid);
  }
}

__global__ void __launch_bounds__(128, 1) gqa_split_kernel(GqaArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int kvh = blockIdx.y;
  const int split = blockIdx.x * 4 + warp;
  const int ctx = a.ctx_dev ? *a.ctx_dev : a.ctx;
  const int n_pages = ctx > 0 ? (ctx + kBS - 1) / kBS : 0;
  const int pps = (n_pages + a.S - 1) / a.S;
  const int p_begin = min(split * pps, n_pages);
  const int p_end = min(p_begin + pps, n_pages);
  const size_t meta = ((size_t)kvh * a.S + split) * kGrp;
  const uint32_t wbase = smem_u32(smem) + warp * kWarpSmem;
  // pages wholly before the newest token do not depend on the previous kernel
  bool pre[kStages - 1];
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    pre[s] = p_begin + s < p_end && (p_begin + s + 1) * kBS <= ctx - 1;
    if (pre[s]) gqa_issue_page(a, kvh, p_begin + s, ctx, wbase + s * kStageBytes, lane);
  }
  pdl_wait();

  // Q^T as the B operand: b0 = q[head g][16kk + 2t..], b1 = q[head g][16kk+8+2t..].
  uint32_t qb[16][2];
  {
    const uint32_t* qh = reinterpret_cast<const uint32_t*>(a.q + (size_t)(kvh * kGrp + g) * kD);
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      qb[kk][0] = qh[(16 * kk + 2 * t) >> 1];
      qb[kk][1] = qh[(16 * kk + 8 + 2 * t) >> 1];
    }
  }
  float acc[16][4];
#pragma unroll
  for (int mt = 0; mt < 16; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (!pre[s] && p_begin + s < p_end)
      gqa_issue_page(a, kvh, p_begin + s, ctx, wbase + s * kStageBytes, lane);
    cp_async_commit();
  }
  pdl_launch_dependents();
  for (int p = p_begin; p < p_end; ++p) {
    const int i = p - p_begin;
    {
      const int pn = p + kStages - 1;
      if (pn < p_end) gqa_issue_page(a, kvh, pn, ctx, wbase + ((i + kStages - 1) % kStages) * kStageBytes, lane);
      cp_async_commit();
    }
    cp_async_wait<kStages - 1>();
    __syncwarp();
    const uint32_t ks = wbase + (i % kStages) * kStageBytes;
    const uint32_t vs = ks + kPageBytes;
    // S^T = K Q^T over 256 dims.
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    {
      const int r = lane & 15;
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) {
        const int cc = 2 * kk + (lane >> 4);
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4(a0, a1, a2, a3, ks + r * 512 + ((cc ^ (r & 7)) << 4));
        mma_16816(s0, s1, s2, s3, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
      }
    }
    // s0=(tok g, head 2t) s1=(tok g, head 2t+1) s2=(tok g+8, 2t) s3=(tok g+8, 2t+1)
    const int tok0 = p * kBS + g, tok1 = tok0 + 8;
    s0 = tok0 < ctx ? s0 * a.scale_log2 : -INFINITY;
    s1 = tok0 < ctx ? s1 * a.scale_log2 : -INFINITY;
    s2 = tok1 < ctx ? s2 * a.scale_log2 : -INFINITY;
    s3 = tok1 < ctx ? s3 * a.scale_log2 : -INFINITY;
    float pm0 = fmaxf(s0, s2), pm1 = fmaxf(s1, s3);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      pm0 = fmaxf(pm0, __shfl_xor_sync(0xffffffffu, pm0, o));
      pm1 = fmaxf(pm1, __shfl_xor_sync(0xffffffffu, pm1, o));
    }
    const float mn0 = fmaxf(m0, pm0), mn1 = fmaxf(m1, pm1);
    const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    const __half p0 = __float2half_rn(exp2f(s0 - mn0));
    const __half p1 = __float2half_rn(exp2f(s1 - mn1));
    const __half p2 = __float2half_rn(exp2f(s2 - mn0));
    const __half p3 = __float2half_rn(exp2f(s3 - mn1));
    // The row sums use the same fp16-rounded weights as the P.V product.
    l0 = l0 * al0 + (__half2float(p0) + __half2float(p2));
    l1 = l1 * al1 + (__half2float(p1) + __half2float(p3));
    const uint32_t pb0 = movmatrix_trans(pack_half2(p0, p1));
    const uint32_t pb1 = movmatrix_trans(pack_half2(p2, p3));
    {
      const int r = (lane & 7) + ((lane >> 4) << 3);
      const int hi = (lane >> 3) & 1;
#pragma unroll
      for (int mt = 0; mt < 16; ++mt) {
        acc[mt][0] *= al0;
        acc[mt][1] *= al1;
        acc[mt][2] *= al0;
        acc[mt][3] *= al1;
        const int cc = 2 * mt + hi;
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4_trans(a0, a1, a2, a3, vs + r * 512 + ((cc ^ (r & 7)) << 4));
        mma_16816(acc[mt][0], acc[mt][1], acc[mt][2], acc[mt][3], a0, a1, a2, a3, pb0, pb1);
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();
  // Full row sums across the 8 lane groups.
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  if (g == 0) {
    a.ws_m[meta + 2 * t] = m0;
    a.ws_m[meta + 2 * t + 1] = m1;
    a.ws_l[meta + 2 * t] = l0;
    a.ws_l[meta + 2 * t + 1] = l1;
  }
  if (p_begin < p_end) {
    float* o = a.ws_acc + meta * kD;
#pragma unroll
    for (int mt = 0; mt < 16; ++mt) {
      const int d0 = 16 * mt + g;
      o[(size_t)(2 * t) * kD + d0] = acc[mt][0];
      o[(size_t)(2 * t + 1) * kD + d0] = acc[mt][1];
      o[(size_t)(2 * t) * kD + d0 + 8] = acc[mt][2];
      o[(size_t)(2 * t + 1) * kD + d0 + 8] = acc[mt][3];
    }
  }
}

// Combine: one CTA per (query head, 32-dim slice), 8 warps. The split
// maxima, weights exp2(m_s - M) and row sums are reduced block-wide; warp w
// then sums the partial outputs of splits w, w+8, ... for its lane's
// dimension, and the 8 warp sums are added in fixed order. Splits that saw
// no page (m = -inf) carry weight 0 and their output rows are never read.
constexpr int kCombWarps = 8;

__global__ void __launch_bounds__(kCombWarps * 32) gqa_combine_kernel(
    const float* ws_m, const float* ws_l, const float* ws_acc, int S, const __half* gate,
    void* out, int out_dtype) {
  __shared__ float sw[kMaxSplits];
  __shared__ float red_m[kCombWarps], red_l[kCombWarps];
  __shared__ float red_o[kCombWarps][32];
  pdl_wait();
  const int h = blockIdx.x, d = blockIdx.y * 32 + (threadIdx.x & 31);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = h / kGrp, hl = h % kGrp;
  const size_t mbase = (size_t)kvh * S * kGrp + hl;
  float m = -INFINITY;
  for (int s = threadIdx.x; s < S; s += kCombWarps * 32) m = fmaxf(m, ws_m[mbase + (size_t)s * kGrp]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red_m[warp] = m;
  __syncthreads();
  float M = red_m[0];
#pragma unroll
  for (int w = 1; w < kCombWarps; ++w) M = fmaxf(M, red_m[w]);
  float l = 0.f;
  for (int s = threadIdx.x; s < S; s += kCombWarps * 32) {
    const float ms = ws_m[mbase + (size_t)s * kGrp];
    const float w = ms == -INFINITY ? 0.f : exp2f(ms - M);
    sw[s] = w;
    if (w != 0.f) l = fmaf(ws_l[mbase + (size_t)s * kGrp], w, l);
  }
  l = warp_sum(l);
  if (lane == 0) red_l[warp] = l;
  __syncthreads();
  // Eight partial rows per batch are loaded before any is used (rows of
  // splits without pages are read but not added), then added in split order.
  float o = 0.f;
  constexpr int kBatch = 8;
  for (int s0 = warp; s0 < S; s0 += kBatch * kCombWarps) {
    float v[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int s = s0 + j * kCombWarps;
      v[j] = s < S ? ws_acc[(mbase + (size_t)s * kGrp) * kD + d] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int s = s0 + j * kCombWarps;
      if (s < S) {
        const float w = sw[s];
        if (w != 0.f) o = fmaf(v[j], w, o);
      }
    }
  }
  red_o[warp][lane] = o;
  __syncthreads();
  pdl_launch_dependents();
  if (warp == 0) {
    float O = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < kCombWarps; ++w) {
      O += red_o[w][lane];
      L += red_l[w];
    }
    float v = L > 0.f ? O / L : 0.f;
    if (gate) v = v * sigmoidf_acc(__half2float(gate[h * kD + d]));
    if (out_dtype == IQ36_F16)
      reinterpret_cast<__half*>(out)[h * kD + d] = __float2half_rn(v);
    else
      reinterpret_cast<float*>(out)[h * kD + d] = v;
  }
}

// Splits per kv head: about two 16-token pages per warp at max_ctx (a warp
// streams its pages through its ring back to back), a multiple of 4 (warps
// per CTA), at most kMaxSplits (longer contexts give each warp more pages).
int gqa_splits(int max_ctx) {
  const int n_pages = (max_ctx + kBS - 1) / kBS;
  int s = (((n_pages + 1) / 2 + 3) / 4) * 4;
  if (s < 4) s = 4;
  if (s > kMaxSplits) s = kMaxSplits;
  return s;
}

size_t gqa_ws_bytes(int max_ctx, int n_q, int n_kv) {
  (void)n_q;
  const size_t S = (size_t)gqa_splits(max_ctx);
  const size_t meta = (size_t)n_kv * S * kGrp;
  const size_t mb = (meta * 4 + 255) / 256 * 256;
  return 2 * mb + meta * kD * 4;
}

int gqa_launch(const void* q, const void* kc, const void* vc, const int32_t* bt, int ctx,
               const int32_t* ctx_dev, int n_q, int n_kv, int D, int bs, float scale,
               const void* gate, void* out, int out_dtype, void* ws, size_t ws_bytes,
               cudaStream_t stream) {
  if (!q || !kc || !vc || !bt || !out) return IQ36_ERR_ARG;
  if (D != kD || bs != kBS || n_kv < 1 || n_q != n_kv * kGrp) return IQ36_ERR_SHAPE;
  if (ctx < 1 || !(scale > 0.f)) return IQ36_ERR_SHAPE;
  if (out_dtype != IQ36_F32 && out_dtype != IQ36_F16) return IQ36_ERR_ARG;
  if (!aligned(q, 16) || !aligned(kc, 16) || !aligned(vc, 16)) return IQ36_ERR_ALIGN;
  const size_t need = gqa_ws_bytes(ctx, n_q, n_kv);
  if (!ws || ws_bytes < need) return IQ36_ERR_WORKSPACE;
  if (!aligned(ws, 256)) return IQ36_ERR_ALIGN;
  // The dynamic shared-memory opt-in is a per-device function attribute.
  static std::atomic<bool> attr_set[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return IQ36_ERR_CUDA;
  if (!attr_set[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(gqa_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             4 * kWarpSmem) != cudaSuccess)
      return IQ36_ERR_CUDA;
    attr_set[dev].store(true, std::memory_order_release);
  }
  const int S = gqa_splits(ctx);
  const size_t meta = (size_t)n_kv * S * kGrp;
  const size_t mb = (meta * 4 + 255) / 256 * 256;
  GqaArgs a;
  a.q = reinterpret_cast<const __half*>(q);
  a.kc = reinterpret_cast<const __half*>(kc);
  a.vc = reinterpret_cast<const __half*>(vc);
  a.bt = bt;
  a.ctx = ctx;
  a.ctx_dev = ctx_dev;
  a.n_kv = n_kv;
  a.S = S;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.ws_m = reinterpret_cast<float*>(ws);
  a.ws_l = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + mb);
  a.ws_acc = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + 2 * mb);
  cudaError_t e = launch(gqa_split_kernel, dim3(S / 4, n_kv), dim3(128), (size_t)4 * kWarpSmem,
                         stream, a);
  if (e != cudaSuccess) return IQ36_ERR_CUDA;
  e = launch(gqa_combine_kernel, dim3(n_q, kD / 32), dim3(kCombWarps * 32), 0, stream,
             (const float*)a.ws_m,
             (const float*)a.ws_l, (const float*)a.ws_acc, S,
             reinterpret_cast<const __half*>(gate), out, out_dtype);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

}  // namespace iq36

extern "C" size_t iq36_paged_gqa_workspace_bytes(int32_t max_ctx, int32_t n_q_heads,
                                                 int32_t n_kv_heads, int32_t head_dim) {
  (void)head_dim;
  return iq36::gqa_ws_bytes(max_ctx, n_q_heads, n_kv_heads);
}

extern "C" int iq36_paged_gqa_decode(const void* q_f16, const void* k_cache, const void* v_cache,
                                     const int32_t* block_table, int32_t ctx_len,
                                     const int32_t* ctx_len_dev, int32_t n_q_heads,
                                     int32_t n_kv_heads, int32_t head_dim, int32_t block_size,
                                     float scale, const void* gate_f16, void* out,
                                     int32_t out_dtype, void* workspace, size_t workspace_bytes,
                                     iq36_stream_t stream) {
  return iq36::gqa_launch(q_f16, k_cache, v_cache, block_table, ctx_len, ctx_len_dev, n_q_heads,
                          n_kv_heads, head_dim, block_size, scale, gate_f16, out, out_dtype,
                          workspace, workspace_bytes, iq36::as_stream(stream));
}

// ---------------------------------------------------------------------------
// Allocation-free paged GQA decode.
//
// For hosts that can hand a kernel only its input and output buffers — for
// example a graph-plugin ABI where the plugin owns every buffer, or a service
// running under a fixed device-memory budget with no allocator reachable from
// the op — this variant keeps the split-K partials (per split and head: max,
// sum and the 256-wide unnormalised output) in one file-scope device array
// instead of a caller workspace. The array is sized for at most 2 KV heads
// (16 query heads) at the largest split count, 4,887,552 bytes; every GPU that
// loads this library holds it until the process exits. All calls on a device
// share it and it keeps the last call's contents; nothing in it needs to start
// at zero because the split kernel writes every max/sum it later reads and the
// combine reads an output partial only for splits that wrote one. Two calls
// whose kernels overlap on the GPU race on the array.
namespace iq36 {

constexpr int kNoAllocMaxKv = 2;
constexpr size_t kNoAllocMeta = (size_t)kNoAllocMaxKv * kMaxSplits * kGrp;
constexpr size_t kNoAllocMetaBytes = (kNoAllocMeta * 4 + 255) / 256 * 256;
constexpr size_t kNoAllocScratchBytes = 2 * kNoAllocMetaBytes + kNoAllocMeta * kD * 4;

static __device__ __align__(256) unsigned char g_gqa_noalloc_scratch[kNoAllocScratchBytes];

// Host code cannot use g_gqa_noalloc_scratch as a device address: resolve it
// once per device, with that device current.
static int noalloc_scratch(void** ptr) {
  static std::atomic<void*> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return IQ36_ERR_CUDA;
  void* p = cached[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    if (cudaGetSymbolAddress(&p, g_gqa_noalloc_scratch) != cudaSuccess || p == nullptr)
      return IQ36_ERR_CUDA;
    cached[dev].store(p, std::memory_order_release);
  }
  *ptr = p;
  return IQ36_OK;
}

}  // namespace iq36

extern "C" int iq36_paged_gqa_decode_noalloc(const void* q_f16, const void* k_cache,
                                             const void* v_cache, const int32_t* block_table,
                                             int32_t ctx_len, const int32_t* ctx_len_dev,
                                             int32_t n_q_heads, int32_t n_kv_heads,
                                             int32_t head_dim, int32_t block_size, float scale,
                                             const void* gate_f16, void* out, int32_t out_dtype,
                                             iq36_stream_t stream) {
  using namespace iq36;
  if (!q_f16 || !k_cache || !v_cache || !block_table || !out) return IQ36_ERR_ARG;
  if (head_dim != kD || block_size != kBS || n_kv_heads < 1 || n_q_heads != n_kv_heads * kGrp ||
      ctx_len < 1 || !(scale > 0.f))
    return IQ36_ERR_SHAPE;
  // Beyond the array's stated maximum: reject before touching the device.
  if (n_kv_heads > kNoAllocMaxKv ||
      gqa_ws_bytes(ctx_len, n_q_heads, n_kv_heads) > kNoAllocScratchBytes)
    return IQ36_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int st = noalloc_scratch(&scratch);
  if (st != IQ36_OK) return st;
  return gqa_launch(q_f16, k_cache, v_cache, block_table, ctx_len, ctx_len_dev, n_q_heads,
                    n_kv_heads, head_dim, block_size, scale, gate_f16, out, out_dtype, scratch,
                    kNoAllocScratchBytes, as_stream(stream));
}
