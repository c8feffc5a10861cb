// attn_prefill.cu — causal GQA attention over T prompt tokens (flash form).
//
// The decode kernel (paged_gqa.cu) attends one query per head to the cached
// context. Prefill attends T queries at positions p0 .. p0+T-1 (p0 = tokens
// already cached) to the keys at positions <= their own, reading K/V from the
// same fp16 paged cache after the batched pre-step wrote the prompt's K/V
// there. Same result as running the decode attention once per prompt token
// (run_qwen36_full_attention_core, gguf_loader.cpp:6071-6137, with the output
// gate of :6034-6069), computed as one causal flash-attention pass.
//
// Tiling: the 8 query heads that share a KV head are packed into the M
// dimension, so every K/V tile staged in shared memory serves all of them.
// CTA = 16 tokens x 8 heads = 128 query rows for one KV head, 8 warps; warp w
// owns tokens t0+2w and t0+2w+1 (fragment rows g -> token t0+2w, g+8 -> token
// t0+2w+1, head g). K/V tiles of 64 keys are gathered through the block table
// with cp.async into a double-buffered, XOR-swizzled ring; QK^T and PV run on
// mma.sync m16n8k16 (fp16 in, fp32 accumulate) with the online softmax in
// registers (P rounded to fp16 as the PV operand). CTAs are issued
// longest-first (latest tokens first) to even out the causal triangle.

#include <atomic>

#include "launch.cuh"
#include "common.cuh"

namespace iq36 {

constexpr int kApD = 256;
constexpr int kApTok = 16;                      // tokens per CTA
constexpr int kApGrp = 8;                       // query heads per KV head
constexpr int kApRows = kApTok * kApGrp;        // 128 query rows per CTA
constexpr int kApKeys = 64;                     // keys per K/V tile
constexpr int kApThreads = 256;
constexpr int kApRowBytes = kApD * 2;           // 512
constexpr int kApQBytes = kApRows * kApRowBytes;
constexpr int kApKVBytes = kApKeys * kApRowBytes;
constexpr int kApSmem = kApQBytes + 4 * kApKVBytes;  // Q + 2 stages of (K, V): 192 KB

// byte offset of 16-byte chunk c of row r in a 512-byte-row swizzled tile
__device__ __forceinline__ uint32_t ap_off(int r, int c) {
  return (uint32_t)(r * kApRowBytes + ((c ^ (r & 7)) << 4));
}

__global__ void __launch_bounds__(kApThreads, 1)
    attn_prefill_kernel(const __half* q, const __half* kc, const __half* vc,
                        const int32_t* bt, int bs, const int32_t* pos_dev, int T, int nq,
                        int nkv, float scale, const __half* gate, void* out, int out_dtype) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int n_tiles = (T + kApTok - 1) / kApTok;
  const int tile = n_tiles - 1 - (int)(blockIdx.x / nkv);
  const int kvh = blockIdx.x % nkv;
  const int t0 = tile * kApTok;
  const uint32_t q_s = smem_u32(smem);
  const uint32_t kv_s = q_s + kApQBytes;

  pdl_wait();
  const int p0 = *pos_dev;
  const int kend = p0 + min(t0 + kApTok, T);  // keys this CTA attends to: [0, kend)
  const int nkb = (kend + kApKeys - 1) / kApKeys;

  // Q rows: R -> token t0 + R/8, head kvh*8 + R%8
  for (int i = tid; i < kApRows * 32; i += kApThreads) {
    const int R = i >> 5, c = i & 31;
    const int tok = t0 + (R >> 3);
    const int tk = min(tok, T - 1);
    cp_async_16(q_s + ap_off(R, c),
                q + ((size_t)tk * nq + kvh * kApGrp + (R & 7)) * kApD + c * 8, tok < T ? 16 : 0);
  }
  auto load_kv = [&](int kb, int stage) {
    const uint32_t ks = kv_s + stage * 2 * kApKVBytes, vs = ks + kApKVBytes;
    for (int i = tid; i < kApKeys * 32; i += kApThreads) {
      const int kr = i >> 5, c = i & 31;
      const int j = kb * kApKeys + kr;
      const bool valid = j < kend;
      size_t slot = 0;
      if (valid) slot = ((size_t)bt[j / bs] * bs + j % bs) * nkv + kvh;
      const size_t off = slot * kApD + c * 8;
      cp_async_16(ks + ap_off(kr, c), kc + off, valid ? 16 : 0);
      cp_async_16(vs + ap_off(kr, c), vc + off, valid ? 16 : 0);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  float o[32][4];
#pragma unroll
  for (int n = 0; n < 32; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float sl2 = scale * 1.4426950408889634f;
  const int pos_a = p0 + t0 + 2 * warp, pos_b = pos_a + 1;

  for (int kb = 0; kb < nkb; ++kb) {
    if (kb + 1 < nkb) {
      load_kv(kb + 1, (kb + 1) & 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t ks = kv_s + (kb & 1) * 2 * kApKVBytes, vs = ks + kApKVBytes;

    // S = Q K^T for this warp's 16 rows x 64 keys
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll 4
    for (int kk = 0; kk < kApD / 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4(a0, a1, a2, a3, q_s + ap_off(16 * warp + (lane & 15), 2 * kk + (lane >> 4)));
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(b0, b1, b2, b3,
                    ks + ap_off(16 * np + ((lane >> 4) << 3) + (lane & 7),
                                2 * kk + ((lane >> 3) & 1)));
        mma_16816(s[2 * np][0], s[2 * np][1], s[2 * np][2], s[2 * np][3], a0, a1, a2, a3, b0, b1);
        mma_16816(s[2 * np + 1][0], s[2 * np + 1][1], s[2 * np + 1][2], s[2 * np + 1][3], a0, a1,
                  a2, a3, b2, b3);
      }
    }
    // causal mask (key j visible to a query at position p iff j <= p)
    const int kbase = kb * kApKeys;
    if (kbase + kApKeys - 1 > pos_a) {
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int j = kbase + 8 * n + 2 * tq + e;
          if (j > pos_a) s[n][e] = -INFINITY;
          if (j > pos_b) s[n][2 + e] = -INFINITY;
        }
    }
    // online softmax (rows g and g+8; a row is spread over the 4 lanes of a quad)
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      mx0 = fmaxf(mx0, fmaxf(s[n][0], s[n][1]));
      mx1 = fmaxf(mx1, fmaxf(s[n][2], s[n][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    // key 0 is visible to every query, so mx is finite from the first tile on
    const float al0 = exp2f((m0 - mx0) * sl2), al1 = exp2f((m1 - mx1) * sl2);
    m0 = mx0;
    m1 = mx1;
    l0 *= al0;
    l1 *= al1;
#pragma unroll
    for (int n = 0; n < 32; ++n) {
      o[n][0] *= al0;
      o[n][1] *= al0;
      o[n][2] *= al1;
      o[n][3] *= al1;
    }
    const float mb0 = mx0 * sl2, mb1 = mx1 * sl2;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      s[n][0] = exp2f(fmaf(s[n][0], sl2, -mb0));
      s[n][1] = exp2f(fmaf(s[n][1], sl2, -mb0));
      s[n][2] = exp2f(fmaf(s[n][2], sl2, -mb1));
      s[n][3] = exp2f(fmaf(s[n][3], sl2, -mb1));
      l0 += s[n][0] + s[n][1];
      l1 += s[n][2] + s[n][3];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < kApKeys / 16; ++kk) {
      const uint32_t pa0 = pack_half2(__float2half_rn(s[2 * kk][0]), __float2half_rn(s[2 * kk][1]));
      const uint32_t pa1 = pack_half2(__float2half_rn(s[2 * kk][2]), __float2half_rn(s[2 * kk][3]));
      const uint32_t pa2 =
          pack_half2(__float2half_rn(s[2 * kk + 1][0]), __float2half_rn(s[2 * kk + 1][1]));
      const uint32_t pa3 =
          pack_half2(__float2half_rn(s[2 * kk + 1][2]), __float2half_rn(s[2 * kk + 1][3]));
#pragma unroll
      for (int dp = 0; dp < 16; ++dp) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(b0, b1, b2, b3,
                          vs + ap_off(16 * kk + (lane & 7) + (((lane >> 3) & 1) << 3),
                                      2 * dp + (lane >> 4)));
        mma_16816(o[2 * dp][0], o[2 * dp][1], o[2 * dp][2], o[2 * dp][3], pa0, pa1, pa2, pa3, b0,
                  b1);
        mma_16816(o[2 * dp + 1][0], o[2 * dp + 1][1], o[2 * dp + 1][2], o[2 * dp + 1][3], pa0,
                  pa1, pa2, pa3, b2, b3);
      }
    }
    __syncthreads();  // this stage is refilled by the next iteration's prefetch
  }
  pdl_launch_dependents();

  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv[2] = {1.f / l0, 1.f / l1};
  const int head = kvh * kApGrp + g;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int tok = t0 + 2 * warp + half;
    if (tok >= T) continue;
    const size_t row = ((size_t)tok * nq + head) * kApD;
#pragma unroll
    for (int n = 0; n < 32; ++n) {
      const int d = 8 * n + 2 * tq;
      float v0 = o[n][2 * half] * inv[half], v1 = o[n][2 * half + 1] * inv[half];
      if (gate) {
        const __half2 gv = *reinterpret_cast<const __half2*>(gate + row + d);
        v0 = v0 * sigmoidf_acc(__low2float(gv));
        v1 = v1 * sigmoidf_acc(__high2float(gv));
      }
      if (out_dtype == IQ36_F16)
        *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(out) + row + d) =
            __floats2half2_rn(v0, v1);
      else
        *reinterpret_cast<float2*>(reinterpret_cast<float*>(out) + row + d) = make_float2(v0, v1);
    }
  }
}

}  // namespace iq36

using namespace iq36;

extern "C" int iq36_attn_prefill(const void* q_f16, const void* k_cache, const void* v_cache,
                                 const int32_t* block_table, int32_t block_size,
                                 const int32_t* pos_dev, int32_t tokens, int32_t n_q_heads,
                                 int32_t n_kv_heads, int32_t head_dim, float scale,
                                 const void* gate_f16, void* out, int32_t out_dtype,
                                 iq36_stream_t stream) {
  if (!q_f16 || !k_cache || !v_cache || !block_table || !pos_dev || !out) return IQ36_ERR_ARG;
  if (head_dim != kApD || tokens < 1 || n_kv_heads < 1 || n_q_heads != kApGrp * n_kv_heads ||
      block_size < 1)
    return IQ36_ERR_SHAPE;
  if (out_dtype != IQ36_F16 && out_dtype != IQ36_F32) return IQ36_ERR_ARG;
  if (!aligned(q_f16, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16) ||
      !aligned(out, 16) || (gate_f16 && !aligned(gate_f16, 16)))
    return IQ36_ERR_ALIGN;
  static std::atomic<bool> attr_set[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return IQ36_ERR_CUDA;
  if (!attr_set[dev].load()) {
    if (cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kApSmem) != cudaSuccess)
      return IQ36_ERR_CUDA;
    attr_set[dev].store(true);
  }
  const int n_tiles = (tokens + kApTok - 1) / kApTok;
  const cudaError_t e =
      launch(attn_prefill_kernel, dim3(n_tiles * n_kv_heads), dim3(kApThreads), (size_t)kApSmem,
             as_stream(stream), reinterpret_cast<const __half*>(q_f16),
             reinterpret_cast<const __half*>(k_cache), reinterpret_cast<const __half*>(v_cache),
             block_table, block_size, pos_dev, tokens, n_q_heads, n_kv_heads, scale,
             reinterpret_cast<const __half*>(gate_f16), out, out_dtype);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}
