// attn_prefill.cu — causal GQA attention over T prompt tokens (flash form) on
// the sm_100a tensor cores (tcgen05).
//
// The decode kernel (paged_gqa.cu) attends one query per head to the cached
// context. Prefill attends T queries at positions p0 .. p0+T-1 (p0 = tokens
// already cached) to the keys at positions <= their own, reading K/V from the
// same fp16 paged cache after the batched pre-step wrote the prompt's K/V
// there. Same result as running the decode attention once per prompt token
// (run_qwen36_full_attention_core, gguf_loader.cpp:6071-6137, with the output
// gate of :6034-6069), computed as one causal flash-attention pass.
//
// CTA = 16 tokens x the 8 query heads of one KV head = 128 query rows (the MMA
// M dimension), so every K/V tile serves all 8 heads. Warp roles:
//   warp 0    TMA: the Q tile once (3-D boxes 64 dims x 8 heads x 16 tokens),
//             then 64-key K and V tiles gathered page by page through the block
//             table (boxes 64 dims x 1 head x 16 keys), K and V in separate
//             double-buffered rings so a K stage refills as soon as its S
//             product is done;
//   warp 1    TMEM allocator and the single MMA-issuing thread:
//             S = Q K^T (M128 N64 K256) into one of two TMEM S buffers, and
//             O += P V (M128 N256 K64, V read MN-major) into TMEM O;
//   warps 2-5 softmax, one query row per thread (= TMEM lane): S from TMEM,
//             causal mask, exp2, P (fp16) to shared memory in the K-major
//             SWIZZLE_128B layout, O rescaled in TMEM only when the row maximum
//             grows by more than 2^8 (otherwise the old maximum stays the
//             reference: exact, P stays <= 256); then the epilogue: O / l,
//             sigmoid(gate), store.
// S(j+1) is computed while the softmax of tile j runs. Every wait is bounded
// and a timeout is counted (iq36_wait_timeouts).

#include <atomic>

#include "launch.cuh"
#include "common.cuh"
#include "tc_sm100.cuh"

namespace iq36 {

constexpr int kApD = 256;
constexpr int kApTok = 16;                      // tokens per CTA
constexpr int kApGrp = 8;                       // query heads per KV head
constexpr int kApRows = kApTok * kApGrp;        // 128 query rows per CTA
constexpr int kApKeys = 64;                     // keys per K/V tile
constexpr int kApThreads = 192;
constexpr int kApQ = kApRows * kApD * 2;        // 64 KB: 4 dim chunks x [128 rows][128 B]
constexpr int kApKV = kApKeys * kApD * 2;       // 32 KB: 4 dim chunks x [64 keys][128 B]
constexpr int kApP = kApRows * kApKeys * 2;     // 16 KB: [128 rows][128 B]
constexpr int kApOffK = kApQ, kApOffV = kApOffK + 2 * kApKV, kApOffP = kApOffV + 2 * kApKV,
              kApOffBar = kApOffP + kApP;
constexpr int kApSmem = kApOffBar + 256 + 1024;  // barriers + 1 KB alignment slack
constexpr uint32_t kApTmemCols = 512;            // S buffers at 0 and 64, O at 256
constexpr uint32_t kIdescS =
    (1u << 4) | ((uint32_t)(kApKeys >> 3) << 17) | ((uint32_t)(kApRows >> 4) << 24);
constexpr uint32_t kIdescO = (1u << 4) | (1u << 16) /* B MN-major */ |
                             ((uint32_t)(kApD >> 3) << 17) | ((uint32_t)(kApRows >> 4) << 24);

__device__ int g_attn_wait_timeouts;

// SWIZZLE_128B descriptor of an MN-major operand: 128-byte rows hold 64 fp16
// along MN, 8-row atoms along K are 1024 B apart (SBO), atoms along MN lbo
// bytes apart (LBO).
__device__ __forceinline__ uint64_t sw128_desc_mn(uint32_t saddr, uint32_t lbo) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__global__ void __launch_bounds__(kApThreads, 1)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const int32_t* bt, int n_blocks,
                        const int32_t* pos_dev, int T, int nq, int nkv, float scale,
                        const __half* gate, void* out, int out_dtype) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_raw = smem_u32(smem_raw);
  const uint32_t base = (base_raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - base_raw);
  const uint32_t q_s = base, k_s = base + kApOffK, v_s = base + kApOffV, p_s = base + kApOffP;
  const uint32_t bar = base + kApOffBar;
  const uint32_t bar_q = bar;          // Q landed (tx)
  const uint32_t bar_k = bar + 8;      // [2] K stage landed (tx)
  const uint32_t bar_ke = bar + 24;    // [2] K stage consumed by S (tcgen05.commit)
  const uint32_t bar_s = bar + 40;     // [2] S buffer written (commit)
  const uint32_t bar_se = bar + 56;    // [2] S buffer read (128 softmax threads)
  const uint32_t bar_p = bar + 72;     // P written and O corrected (128 softmax threads)
  const uint32_t bar_o = bar + 80;     // PV of a tile done (commit)
  const uint32_t bar_done = bar + 88;  // every MMA done (teardown)
  const uint32_t bar_v = bar + 96;     // [2] V stage landed (tx)
  const uint32_t bar_ve = bar + 112;   // [2] V stage consumed by PV (commit)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kApOffBar + 192);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (T + kApTok - 1) / kApTok;
  const int tile = n_tiles - 1 - (int)(blockIdx.x / nkv);  // longest first
  const int kvh = blockIdx.x % nkv;
  const int t0 = tile * kApTok;
  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_k + 8 * s, 1);
      mbar_init(bar_ke + 8 * s, 1);
      mbar_init(bar_v + 8 * s, 1);
      mbar_init(bar_ve + 8 * s, 1);
      mbar_init(bar_s + 8 * s, 1);
      mbar_init(bar_se + 8 * s, 128);
    }
    mbar_init(bar_p, 128);
    mbar_init(bar_o, 1);
    mbar_init(bar_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kApTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  const int p0 = *pos_dev;
  const int kend = p0 + min(t0 + kApTok, T);  // keys this CTA attends to: [0, kend)
  const int nkb = (kend + kApKeys - 1) / kApKeys;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_tx(bar_q, kApQ);
      for (int dc = 0; dc < 4; ++dc)
        tma_load_3d(q_s + dc * (kApRows * 128), &tmQ, dc * 64, kvh * kApGrp, t0, bar_q);
      // per 16-key page and 64-dim chunk one box (64 dims x 1 head x 16 keys)
      // into chunk dc's [64 keys][128 B] operand tile
      auto load_tile = [&](const CUtensorMap* map, uint32_t dst, uint32_t full, int j) {
        mbar_arrive_tx(full, kApKV);
        for (int pg = 0; pg < kApKeys / 16; ++pg) {
          const int key0 = j * kApKeys + pg * 16;
          // a page wholly past the context is read outside the tensor: zeros
          const int row = key0 < kend ? bt[key0 / 16] * 16 : n_blocks * 16;
#pragma unroll
          for (int dc = 0; dc < 4; ++dc)
            tma_load_3d(dst + dc * (kApKeys * 128) + pg * 16 * 128, map, dc * 64, kvh, row, full);
        }
      };
      for (int j = 0; j < nkb && ok; ++j) {
        const int st = j & 1, ph = ((j >> 1) & 1) ^ 1u;
        ok = mbar_wait(bar_ke + 8 * st, ph);
        if (!ok) break;
        load_tile(&tmK, k_s + st * kApKV, bar_k + 8 * st, j);
        ok = mbar_wait(bar_ve + 8 * st, ph);
        if (!ok) break;
        load_tile(&tmV, v_s + st * kApKV, bar_v + 8 * st, j);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      ok = mbar_wait(bar_q, 0);
      auto issue_s = [&](int j) -> bool {
        const int b = j & 1;
        if (!mbar_wait(bar_se + 8 * b, ((j >> 1) & 1) ^ 1u) ||
            !mbar_wait(bar_k + 8 * b, (j >> 1) & 1))
          return false;
        tc_fence_after();
        const uint32_t ks = k_s + b * kApKV;
#pragma unroll
        for (int kk = 0; kk < kApD / 16; ++kk) {
          const uint32_t dc = kk >> 2, sub = kk & 3;
          umma_f16(tmem + b * kApKeys, sw128_desc(q_s + dc * (kApRows * 128) + sub * 32),
                   sw128_desc(ks + dc * (kApKeys * 128) + sub * 32), kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(bar_s + 8 * b);
        umma_commit(bar_ke + 8 * b);  // K of this stage read
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < nkb && ok; ++j) {
        if (j + 1 < nkb && !(ok = issue_s(j + 1))) break;
        ok = mbar_wait(bar_p, j & 1) && mbar_wait(bar_v + 8 * (j & 1), (j >> 1) & 1);
        if (!ok) break;
        tc_fence_after();
        const uint32_t vs = v_s + (j & 1) * kApKV;
#pragma unroll
        for (int kk = 0; kk < kApKeys / 16; ++kk)
          umma_f16(tmem + 256, sw128_desc(p_s + kk * 32),
                   sw128_desc_mn(vs + kk * 16 * 128, kApKeys * 128), kIdescO,
                   (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(bar_ve + 8 * (j & 1));  // V of this stage read
        umma_commit(bar_o);
      }
      umma_commit(bar_done);
      if (!mbar_wait(bar_done, 0)) ok = false;
    }
  } else {
    // softmax, O correction and epilogue: thread = query row = TMEM lane
    const int quarter = warp & 3;  // warps 2,3,4,5 -> TMEM lanes 64.., 96.., 0.., 32..
    const int r = quarter * 32 + lane;
    const int tok = t0 + r / kApGrp, head = kvh * kApGrp + (r % kApGrp);
    const int pos = p0 + tok;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = scale * 1.4426950408889634f;
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < nkb && ok; ++j) {
      const int b = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(bar_s + 8 * b, (j >> 1) & 1));
      if (!ok) break;
      tc_fence_after();
      float s[kApKeys];
#pragma unroll
      for (int c = 0; c < kApKeys; c += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + lane_off + b * kApKeys + c, v);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) s[c + e] = __uint_as_float(v[e]);
      }
      tc_fence_before();
      mbar_arrive(bar_se + 8 * b);  // this S buffer may be rewritten
      const int kbase = j * kApKeys;
      float mx = m;
#pragma unroll
      for (int e = 0; e < kApKeys; ++e) {
        if (kbase + e > pos) s[e] = -INFINITY;
        mx = fmaxf(mx, s[e]);
      }
      // key 0 is visible to every row (rows past T have zero queries), so mx is
      // finite from the first tile on
      const bool first = j == 0;
      const bool grow = !first && (mx - m) * sl2 > 8.f;
      const float mref = (first || grow) ? mx : m;
      const float mb = mref * sl2;
      float sum = 0.f;
      uint32_t ph[kApKeys / 2];
#pragma unroll
      for (int e = 0; e < kApKeys; e += 2) {
        const float a = exp2f(fmaf(s[e], sl2, -mb)), c2 = exp2f(fmaf(s[e + 1], sl2, -mb));
        sum += a + c2;
        ph[e / 2] = pack_half2(__float2half_rn(a), __float2half_rn(c2));
      }
      if (!first) {
        // PV of the previous tile must be done before P is overwritten and O rescaled
        ok = __all_sync(0xffffffffu, mbar_wait(bar_o, (j - 1) & 1));
        if (!ok) break;
        tc_fence_after();
      }
      if (grow) {
        const float alpha = exp2f((m - mref) * sl2);
        l *= alpha;
#pragma unroll 1
        for (int c = 0; c < kApD; c += 16) {
          uint32_t v[16];
          tmem_ld16(tmem + lane_off + 256 + c, v);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
          tmem_st16(tmem + lane_off + 256 + c, v);
        }
        tmem_st_wait();
      }
      m = mref;
      l += sum;
      uint8_t* prow = smem + kApOffP + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) =
            make_uint4(ph[4 * c], ph[4 * c + 1], ph[4 * c + 2], ph[4 * c + 3]);
      fence_proxy_async_smem();  // P is read by the tensor core (async proxy)
      tc_fence_before();
      mbar_arrive(bar_p);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar_o, (nkb - 1) & 1));
    if (ok) {
      tc_fence_after();
      const float inv = 1.f / l;
      const bool store = tok < T;
      const size_t row = ((size_t)(store ? tok : 0) * nq + head) * kApD;
#pragma unroll 1
      for (int c = 0; c < kApD; c += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + lane_off + 256 + c, v);
        tmem_ld_wait();
        if (!store) continue;
        float y[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) y[e] = __uint_as_float(v[e]) * inv;
        if (gate) {
          const uint4* gp = reinterpret_cast<const uint4*>(gate + row + c);
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const uint4 gr = gp[q];
            const __half* gh = reinterpret_cast<const __half*>(&gr);
#pragma unroll
            for (int e = 0; e < 8; ++e) y[8 * q + e] *= sigmoidf_acc(__half2float(gh[e]));
          }
        }
        if (out_dtype == IQ36_F16) {
          uint4 o[2];
          uint32_t* ow = reinterpret_cast<uint32_t*>(o);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            ow[q] = pack_half2(__float2half_rn(y[2 * q]), __float2half_rn(y[2 * q + 1]));
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(out) + row + c);
          dst[0] = o[0];
          dst[1] = o[1];
        } else {
          float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + row + c);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
        }
      }
    }
  }
  if (!ok && lane == 0) atomicAdd(&g_attn_wait_timeouts, 1);
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kApTmemCols);
  }
}

// 3-D fp16 tensor map: {inner (contiguous), mid, outer} with byte strides for
// mid and outer, box {64, box_mid, box_outer}, SWIZZLE_128B.
static bool make_map3(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t mid,
                      uint64_t outer, uint64_t mid_stride, uint64_t outer_stride, uint32_t box_mid,
                      uint32_t box_outer) {
  auto enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[3] = {inner, mid, outer};
  const cuuint64_t strides[2] = {mid_stride, outer_stride};
  const cuuint32_t box[3] = {64u, box_mid, box_outer};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int attn_wait_timeouts(int* count, int reset) {
  if (cudaMemcpyFromSymbol(count, g_attn_wait_timeouts, sizeof(int)) != cudaSuccess)
    return IQ36_ERR_CUDA;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_attn_wait_timeouts, &zero, sizeof(int)) != cudaSuccess)
      return IQ36_ERR_CUDA;
  }
  return IQ36_OK;
}

}  // namespace iq36

using namespace iq36;

extern "C" int iq36_attn_prefill(const void* q_f16, const void* k_cache, const void* v_cache,
                                 const int32_t* block_table, int32_t block_size,
                                 int32_t num_blocks, const int32_t* pos_dev, int32_t tokens,
                                 int32_t n_q_heads,
                                 int32_t n_kv_heads, int32_t head_dim, float scale,
                                 const void* gate_f16, void* out, int32_t out_dtype,
                                 iq36_stream_t stream) {
  if (!q_f16 || !k_cache || !v_cache || !block_table || !pos_dev || !out) return IQ36_ERR_ARG;
  if (head_dim != kApD || tokens < 1 || n_kv_heads < 1 || n_q_heads != kApGrp * n_kv_heads ||
      block_size != 16 || num_blocks < 1 || num_blocks > (1 << 22))
    return IQ36_ERR_SHAPE;
  if (out_dtype != IQ36_F16 && out_dtype != IQ36_F32) return IQ36_ERR_ARG;
  if (!aligned(q_f16, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16) ||
      !aligned(out, 16) || (gate_f16 && !aligned(gate_f16, 16)))
    return IQ36_ERR_ALIGN;
  // the maps span exactly the cache: a block-table entry past it reads zeros
  const uint64_t keys = (uint64_t)num_blocks * 16;
  CUtensorMap mq, mk, mv;
  if (!make_map3(&mq, q_f16, kApD, (uint64_t)n_q_heads, (uint64_t)tokens, kApD * 2,
                 (uint64_t)n_q_heads * kApD * 2, kApGrp, kApTok) ||
      !make_map3(&mk, k_cache, kApD, (uint64_t)n_kv_heads, keys, kApD * 2,
                 (uint64_t)n_kv_heads * kApD * 2, 1, 16) ||
      !make_map3(&mv, v_cache, kApD, (uint64_t)n_kv_heads, keys, kApD * 2,
                 (uint64_t)n_kv_heads * kApD * 2, 1, 16))
    return IQ36_ERR_CUDA;
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
             as_stream(stream), mq, mk, mv, block_table, (int)(keys / 16), pos_dev, tokens,
             n_q_heads, n_kv_heads, scale, reinterpret_cast<const __half*>(gate_f16), out,
             out_dtype);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}
