// moe_prefill.cu — grouped MoE prefill on tcgen05 tensor cores.
//
// Dataflow (reference: Gen-1 schedule grouped_s8_u4_f16_contribution_moe.cl:
// 13-222 -> grouped GEMMs -> deterministic scatter :847-861; the stock
// OpenVINO path gather -> up/gate GEMM with swish*up post-op -> down GEMM ->
// scatter, iq36-pr35924-grouped-postops.patch:15-124), all on the device with
// no host readback:
//   1. pf_hist     per-CTA expert histograms of the T*k assignments;
//   2. pf_scan     expert offsets, per-CTA bases, and the 128-row tile table;
//   3. pf_place    stable position of each assignment (by expert, then token,
//                  then rank), inverse map, permuted token ids and weights;
//   4. pf_gather   Xp[p] = fp16(x[token(p)]) in the permuted operand order;
//   5. GEMM1       per tile: [128 x H] . W_gu,e^T -> [128 x 256] fp32 in TMEM
//                  (128 gate + the matching 128 up columns), SwiGLU epilogue,
//                  act fp16;
//   6. GEMM2       per tile: [128 x I] . W_d,e^T -> [128 x 256] fp32, times the
//                  router weight, contributions Y rounded to fp16;
//   7. pf_scatter  out[t] = sum over ranks r (in order) of Y[inv(t, r)].
//
// GEMM kernel: persistent, one CTA per SM (grid min(148, units)); a unit is
// one or two 128-row M tiles (the grouped modes: one tile of one expert) x
// one 256-wide N tile, taken round-robin.
// Warp roles (23 warps):
//   warp 0      TMA producer of the activation tiles (SWIZZLE_128B, one
//               64-wide k-block of each of the unit's tiles per stage, no
//               multicast) into a 3-deep ring;
//   warp 1      TMEM allocator (2 x 256 columns) and the single-thread
//               tcgen05.mma issuer (kind::f16, M=128 N=256 K=16, fp32
//               accumulate, four MMAs per tile and k-block): a two-tile unit
//               fills both accumulator slots, one-tile units alternate them;
//   warp 2      B-side producer: the raw u4 codes (TMA, 64 bytes x 256 rows
//               per two k-blocks) into a 2-deep ring;
//   warps 3-18  dequant, half a B-tile row per thread: (q - zp) * scale with
//               one fp16 rounding, written in the canonical SW128 K-major
//               layout; each row's scales and zero points are read from
//               global memory, the next group's one group ahead;
//   warps 19-22 epilogue (tcgen05.ld -> registers -> global); for one-tile
//               units it overlaps the next unit's mainloop.
// A ring 3 x 32 KB, B ring 3 x 32 KB, code ring 2 x 16 KB. Per-thread clock
// stamps showed the dequant warps bound a one-tile unit (about 1150 cycles
// per k-block of dequant against 512 of MMA work), so a second tile that
// reuses each dequantised k-block cuts the mainloop time per FLOP by about a
// third (its MMAs add ~26% per stage). All
// rings are synchronised with mbarriers; every wait is time-bounded and
// writes an error word on expiry.
// Buffers that threads read with generic loads and the TMA engine refills
// (codes) are released only after fence.proxy.async.
// GEMM2 stores fp16 contributions (the reference's f16-contribution scatter).

// Operand order: inside each 8-element K chunk both operands hold the
// elements in the order (0,4,1,5,2,6,3,7) — the natural order of the nibble
// unpack — so the dequant needs no permute; the gather (activations) and the
// GEMM1 epilogue (act) write that order.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "launch.cuh"
#include "common.cuh"
#include "tc_sm100.cuh"

namespace iq36 {

constexpr int kPfBM = 128, kPfBN = 256, kPfBK = 64;
// A unit's M extent is one or two 128-row tiles that share each dequantised
// B k-block (eight MMAs per B stage for two tiles): the dequant, not the
// tensor pipe, bounds a one-tile unit, and a second tile's MMAs cost about a
// quarter more time per stage for twice the work.
constexpr int kPfMaxTiles = 2;
constexpr int kPfAStages = 3, kPfBStages = 3, kPfCodeStages = 2;
// A code stage holds two k-blocks of u4 codes for the 256 B-tile rows (TMA
// rows of 64 bytes, half the row requests of 32-byte rows).
constexpr int kPfCodeKB = 2;
constexpr int kPfCodeRow = kPfCodeKB * kPfBK / 2;   // 64 bytes of codes per row
constexpr int kPfASub = kPfBM * kPfBK * 2;          // one k-block of one tile, 16 KB
constexpr int kPfAStage = kPfMaxTiles * kPfASub;    // 32 KB
constexpr int kPfBStage = kPfBN * kPfBK * 2;        // one dequantised k-block, 32 KB
constexpr int kPfCodeStage = kPfBN * kPfCodeRow;    // 16 KB of u4 codes
constexpr int kPfOffB = kPfAStages * kPfAStage;     // B ring after the A ring
constexpr int kPfOffCodes = kPfOffB + kPfBStages * kPfBStage;
constexpr int kPfOffBar = kPfOffCodes + kPfCodeStages * kPfCodeStage;
constexpr int kPfSmem = kPfOffBar + 256 + 1024;
constexpr int kPfDqWarps = 16, kPfEpiWarps = 4;
constexpr int kPfWarpDq0 = 3, kPfWarpEpi0 = kPfWarpDq0 + kPfDqWarps;
constexpr int kPfThreads = (kPfWarpEpi0 + kPfEpiWarps) * 32;  // 736
constexpr int kPfDqThreads = kPfDqWarps * 32;                 // half a B-tile row each
constexpr int kPfChunk = 512;  // assignments per schedule CTA (64 CTAs at 4096 tokens x top-8)
static_assert(kPfChunk % 256 == 0, "placement ranks 256 assignments per round");
constexpr uint32_t kTmemCols = 512;  // two 256-column accumulators

// Instruction descriptor of tcgen05.mma kind::f16: D fp32, A and B fp16, both
// K-major, N = 256, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kPfBN >> 3) << 17) | ((uint32_t)(kPfBM >> 4) << 24);

// ---------------------------------------------------------------------------
// Schedule kernels

struct PfWork {
  int32_t* hist;      // [nC, E]
  int32_t* cbase;     // [nC, E]
  int32_t* offset;    // [E]
  int32_t* tile_count;
  int32_t* tile_expert;
  int32_t* tile_row0;
  int32_t* tile_rows;
  int32_t* inv;       // [P]
  int32_t* perm_tok;  // [P]
  float* perm_w;      // [P]
  int32_t* err;
  __half* xp;         // [P + 128, H]
  __half* act;        // [P + 128, I]
  __half* y;          // [P + 128, H] fp16 contributions
};

__global__ void __launch_bounds__(256) pf_hist_kernel(const int32_t* ids, int P, int E,
                                                      PfWork w) {
  __shared__ int32_t h[256];
  pdl_wait();
  for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
  __syncthreads();
  const int a0 = blockIdx.x * kPfChunk;
  for (int a = a0 + threadIdx.x; a < min(a0 + kPfChunk, P); a += blockDim.x) {
    const int e = min(max(ids[a], 0), E - 1);
    atomicAdd(&h[e], 1);
  }
  __syncthreads();
  pdl_launch_dependents();
  for (int e = threadIdx.x; e < E; e += blockDim.x) w.hist[(size_t)blockIdx.x * E + e] = h[e];
}

// One CTA, thread e = expert (E <= 256). Exclusive scans of the per-expert
// assignment and tile counts: warp shuffles, then the 8 warp totals.
__global__ void __launch_bounds__(256) pf_scan_kernel(int nC, int E, PfWork w) {
  __shared__ int32_t s_wtot[8], s_wtiles[8];
  pdl_wait();
  const int e = threadIdx.x, lane = e & 31, warp = e >> 5;
  int tot = 0;
  if (e < E)
    for (int c = 0; c < nC; ++c) tot += w.hist[(size_t)c * E + e];
  const int tiles = (tot + kPfBM - 1) / kPfBM;
  int inc = tot, tinc = tiles;  // inclusive within the warp
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int a = __shfl_up_sync(0xffffffffu, inc, d), b = __shfl_up_sync(0xffffffffu, tinc, d);
    if (lane >= d) {
      inc += a;
      tinc += b;
    }
  }
  if (lane == 31) {
    s_wtot[warp] = inc;
    s_wtiles[warp] = tinc;
  }
  __syncthreads();
  int off = inc - tot, t0 = tinc - tiles;
  for (int v = 0; v < warp; ++v) {
    off += s_wtot[v];
    t0 += s_wtiles[v];
  }
  if (e == 255) *w.tile_count = t0 + tiles;
  if (e < E) {
    w.offset[e] = off;
    int run = off;
    for (int c = 0; c < nC; ++c) {
      w.cbase[(size_t)c * E + e] = run;
      run += w.hist[(size_t)c * E + e];
    }
    for (int i = 0; off + i * kPfBM < run; ++i) {
      w.tile_expert[t0 + i] = e;
      w.tile_row0[t0 + i] = off + i * kPfBM;
      w.tile_rows[t0 + i] = min(kPfBM, run - (off + i * kPfBM));
    }
  }
  pdl_launch_dependents();
}

// Stable placement: CTA c owns assignments [c*kPfChunk, (c+1)*kPfChunk) in
// order; in rounds of 256 it ranks each assignment among earlier ones of its
// expert. The input row of assignment a is a / k, or row_of[a] (clamped to
// the n_rows rows) when the rows are given per assignment.
__global__ void __launch_bounds__(256) pf_place_kernel(const int32_t* ids, const float* weights,
                                                       int P, int E, int k,
                                                       const int32_t* row_of, int n_rows,
                                                       PfWork w) {
  __shared__ int32_t run[256];
  __shared__ int32_t wc[8][256];
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < E; e += 256) run[e] = w.cbase[(size_t)blockIdx.x * E + e];
  const int a0 = blockIdx.x * kPfChunk;
  for (int r = 0; r < kPfChunk / 256; ++r) {
    for (int i = tid; i < 8 * 256; i += 256) (&wc[0][0])[i] = 0;
    __syncthreads();
    const int a = a0 + r * 256 + tid;
    const bool valid = a < P;
    const int e = valid ? min(max(ids[a], 0), E - 1) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank_w = __popc(peers & ((1u << lane) - 1u));
    if (valid && rank_w == 0) wc[warp][e] = __popc(peers);
    __syncthreads();
    if (valid) {
      int before = 0;
      for (int v = 0; v < warp; ++v) before += wc[v][e];
      const int p = run[e] + before + rank_w;
      w.inv[a] = p;
      w.perm_tok[p] = row_of ? min(max(row_of[a], 0), n_rows - 1) : a / k;
      w.perm_w[p] = weights[a];
    }
    __syncthreads();
    for (int e2 = tid; e2 < E; e2 += 256) {
      int add = 0;
      for (int v = 0; v < 8; ++v) add += wc[v][e2];
      run[e2] += add;
    }
    __syncthreads();
  }
  pdl_launch_dependents();
}

// Xp[p][:] = fp16(x[token(p)][:]) with each 8-chunk stored as (0,4,1,5,2,6,3,7);
// x is bf16 (x_f16 == 0) or fp16.
__global__ void __launch_bounds__(256) pf_gather_kernel(const void* x, int x_f16, int P, int H,
                                                        PfWork w) {
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= P) return;
  const int t = w.perm_tok[warp];
  const uint16_t* src = reinterpret_cast<const uint16_t*>(x) + (size_t)t * H;
  __half* dst = w.xp + (size_t)warp * H;
  for (int c = lane; c < H / 8; c += 32) {
    const uint4 raw = *reinterpret_cast<const uint4*>(src + c * 8);
    __half h[8];
    if (x_f16) {
      const __half* hp = reinterpret_cast<const __half*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) h[j] = hp[j];
    } else {
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) h[j] = __float2half_rn(__bfloat162float(b[j]));
    }
    uint4 o;
    o.x = pack_half2(h[0], h[4]);
    o.y = pack_half2(h[1], h[5]);
    o.z = pack_half2(h[2], h[6]);
    o.w = pack_half2(h[3], h[7]);
    *reinterpret_cast<uint4*>(dst + c * 8) = o;
  }
  pdl_launch_dependents();
}

// out[t][h] = sum_r float(Y[inv(t,r)][h]), ranks in order, fp32 accumulate
// over fp16 contributions (iq36_scatter_f16_contributions,
// grouped_s8_u4_f16_contribution_moe.cl:831-845). Output fp32, bf16 or fp16;
// with accumulate (fp32 only) the sum is added to out (the residual stream).
__global__ void __launch_bounds__(256) pf_scatter_kernel(const int32_t* inv, const __half* y,
                                                         int T, int H, int k, void* out,
                                                         int out_dtype, int accumulate) {
  pdl_wait();
  const int t = blockIdx.x;
  int rows[16];
  for (int r = 0; r < k; ++r) rows[r] = inv[(size_t)t * k + r];
  for (int h = threadIdx.x * 4; h < H; h += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < k; ++r) {
      const uint2 raw = *reinterpret_cast<const uint2*>(y + (size_t)rows[r] * H + h);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
      acc.x += a.x;
      acc.y += a.y;
      acc.z += b.x;
      acc.w += b.y;
    }
    if (out_dtype == IQ36_BF16) {
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out) + (size_t)t * H + h;
      o[0] = __float2bfloat16_rn(acc.x);
      o[1] = __float2bfloat16_rn(acc.y);
      o[2] = __float2bfloat16_rn(acc.z);
      o[3] = __float2bfloat16_rn(acc.w);
    } else if (out_dtype == IQ36_F16) {
      uint2 o;
      o.x = pack_half2(__float2half_rn(acc.x), __float2half_rn(acc.y));
      o.y = pack_half2(__float2half_rn(acc.z), __float2half_rn(acc.w));
      *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(out) + (size_t)t * H + h) = o;
    } else {
      float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)t * H + h);
      if (accumulate) {
        const float4 r = *o;
        acc.x += r.x;
        acc.y += r.y;
        acc.z += r.z;
        acc.w += r.w;
      }
      *o = acc;
    }
  }
}

// ---------------------------------------------------------------------------
// Grouped GEMM

// Count of bounded waits that gave up in the GEMM kernels (read by iq36_wait_timeouts).
__device__ int g_gemm_wait_timeouts;

// MODE 0: grouped gate_up + SwiGLU; MODE 1: grouped down x router weight
// (fp16 contributions); MODE 2: dense u4 GEMM out[T, N] = x W^T (tiles of the
// T rows in order, weight rows nt*256 ..), fp16 store or fp32 accumulate,
// optionally scaled per row by sigmoid(row_gate[t]); MODE 3: dense gate_up +
// SwiGLU, out[T, I] fp16 = SwiGLU(x W[0:I]^T, x W[I:2I]^T).
struct GemmArgs {
  const __half* s;      // scales of the bank (or matrix)
  const uint8_t* z;     // zero points
  int64_t exp_rows;     // weight rows per expert (2I for gate_up, H for down)
  int K;                // reduction length (H or I; the input length for MODE 2)
  int I;                // intermediate size (gate_up row split)
  int H;                // output rows of the down GEMM; N for MODE 2
  PfWork work;
  int T;                // MODE 2: rows of x
  void* out;            // MODE 2: [T, N]
  int out_dtype;        // MODE 2: IQ36_F16 store or IQ36_F32
  int accumulate;       // MODE 2, fp32: out += f16(x W^T)
  const float* row_gate;  // MODE 2: optional per-row logit; output *= sigmoid(logit)
  // MODE 2 over up to 4 projections sharing x: N tile n belongs to projection p
  // with tile_base[p] <= n < tile_base[p + 1] (H = the projections' total rows)
  int n_proj;
  int tile_base[5];
  const __half* ps[4];
  const uint8_t* pz[4];
  void* pout[4];
  int prow[4], pdt[4], pacc[4];
  // Group 64 (one quant group per 64-wide k-block) or 128 (one per two);
  // the dequant threads read a row's scales and zero points from global
  // memory, the next group's while the current one is dequantised.
  int g64;
  // MODE 2/3: 128-row tiles per unit (1 or 2); the grouped modes use 1.
  int mt;
  // MODE 2/3 with mt = 2: the rows from row1 on run as n1 one-tile M rows,
  // ahead of the two-tile rows [0, row1) in the unit order (n1 = 0, row1 = T
  // when every row is in two-tile units).
  int n1, row1;
};

// projection of a MODE-2 N tile and the tile's index inside it
__device__ __forceinline__ void pf_proj(const GemmArgs& g, int nt, int& p, int& ntl) {
  p = 0;
#pragma unroll
  for (int i = 1; i < 4; ++i)
    if (i < g.n_proj && nt >= g.tile_base[i]) p = i;
  ntl = nt - g.tile_base[p];
}

template <int MODE>
__device__ __forceinline__ int pf_units(const GemmArgs& g) {
  const int um = kPfBM * g.mt;  // rows per unit
  const int mrows = g.n1 + (g.row1 + um - 1) / um;
  if (MODE == 2) return mrows * (g.H / kPfBN);
  if (MODE == 3) return mrows * (g.I / 128);
  return *g.work.tile_count * (MODE == 0 ? g.I / 128 : g.H / kPfBN);
}
template <int MODE>
__device__ __forceinline__ void pf_rows(const GemmArgs& g, int mt, int& row0, int& rows) {
  if (MODE >= 2) {
    if (mt < g.n1) {  // one-tile rows at the end of the prompt, scheduled first
      row0 = g.row1 + mt * kPfBM;
      rows = min(kPfBM, g.T - row0);
    } else {
      row0 = (mt - g.n1) * kPfBM * g.mt;
      rows = min(kPfBM * g.mt, g.row1 - row0);
    }
  } else {
    row0 = g.work.tile_row0[mt];
    rows = g.work.tile_rows[mt];
  }
}

// Work unit u (persistent CTAs take u = blockIdx.x, + gridDim.x, ...):
// M tile u / nN of the tile table, N tile u % nN, so the N tiles of one M
// tile (same expert, same activation rows) run side by side.
struct PfUnit {
  int row0, rows;
  int64_t wr0, wr1;  // first weight row of each 128-row half of the B tile
  int proj;          // MODE 2: projection of the tile
};

template <int MODE>
__device__ __forceinline__ PfUnit pf_unit(const GemmArgs& g, int u, int nN) {
  const int mt = u / nN, nt = u - mt * nN;
  PfUnit r;
  pf_rows<MODE>(g, mt, r.row0, r.rows);
  r.proj = 0;
  if (MODE == 2) {
    int ntl;
    pf_proj(g, nt, r.proj, ntl);
    r.wr0 = (int64_t)ntl * kPfBN;
    r.wr1 = r.wr0 + 128;
    return r;
  }
  if (MODE == 3) {
    r.wr0 = (int64_t)nt * 128;  // gate rows
    r.wr1 = r.wr0 + g.I;        // the matching up rows
    return r;
  }
  const int e = g.work.tile_expert[mt];
  if (MODE == 0) {
    r.wr0 = (int64_t)e * g.exp_rows + nt * 128;  // gate rows
    r.wr1 = r.wr0 + g.I;                         // the matching up rows
  } else {
    r.wr0 = (int64_t)e * g.exp_rows + nt * kPfBN;
    r.wr1 = r.wr0 + 128;
  }
  return r;
}

template <int MODE>
__global__ void __launch_bounds__(kPfThreads, 1)
    pf_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmW1,
                   const __grid_constant__ CUtensorMap tmW2,
                   const __grid_constant__ CUtensorMap tmW3, GemmArgs g) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_raw = smem_u32(smem_raw);
  const uint32_t base = (base_raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - base_raw);
  const uint32_t bar_afull = base + kPfOffBar;                 // [kPfAStages]
  const uint32_t bar_aempty = bar_afull + 8 * kPfAStages;      // [kPfAStages]
  const uint32_t bar_full = bar_aempty + 8 * kPfAStages;       // B stages [kPfBStages]
  const uint32_t bar_empty = bar_full + 8 * kPfBStages;        // [kPfBStages]
  const uint32_t bar_cfull = bar_empty + 8 * kPfBStages;       // [kPfCodeStages]
  const uint32_t bar_cempty = bar_cfull + 8 * kPfCodeStages;   // [kPfCodeStages]
  const uint32_t bar_accf = bar_cempty + 8 * kPfCodeStages;    // [2] per accumulator slot
  const uint32_t bar_acce = bar_accf + 16;                     // [2]
  const uint32_t bar_done = bar_acce + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + (bar_done + 8 - base));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPfAStages; ++s) {
      mbar_init(bar_afull + 8 * s, 1);                // A producer (with tx)
      mbar_init(bar_aempty + 8 * s, 1);               // tcgen05.commit
    }
    for (int s = 0; s < kPfBStages; ++s) {
      mbar_init(bar_full + 8 * s, kPfDqThreads);      // dequant threads
      mbar_init(bar_empty + 8 * s, 1);                // tcgen05.commit
    }
    for (int s = 0; s < kPfCodeStages; ++s) {
      mbar_init(bar_cfull + 8 * s, 1);                // code producer (with tx)
      mbar_init(bar_cempty + 8 * s, kPfDqThreads);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_accf + 8 * b, 1);                 // tcgen05.commit
      mbar_init(bar_acce + 8 * b, kPfEpiWarps * 32);  // epilogue threads
    }
    mbar_init(bar_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // the tile table and both operands come from earlier launches
  const int nN = (MODE == 0 || MODE == 3) ? g.I / 128 : g.H / kPfBN;
  const int total = pf_units<MODE>(g);
  const int nkb = g.K / kPfBK;
  const bool g64 = g.g64 != 0;
  const int ng = g64 ? g.K / 64 : g.K / 128;
  bool ok = true;

  if (warp == 0) {
    // ---- activation producer (TMA, SWIZZLE_128B, one k-block of each of
    // the unit's 128-row tiles per stage) ----
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        int row0, rows;
        pf_rows<MODE>(g, u / nN, row0, rows);
        const int mtn = rows > kPfBM ? 2 : 1;
        for (int kb = 0; kb < nkb; ++kb) {
          ok = mbar_wait(bar_aempty + 8 * s, ph ^ 1u);
          if (!ok) break;
          const uint32_t dst = base + s * kPfAStage;
          mbar_arrive_tx(bar_afull + 8 * s, (uint32_t)(mtn * kPfASub));
          for (int t = 0; t < mtn; ++t)
            tma_load_2d(dst + t * kPfASub, &tmA, kb * kPfBK, row0 + t * kPfBM, bar_afull + 8 * s);
          if (++s == kPfAStages) s = 0, ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer: one thread. A two-tile unit accumulates its tiles in
    // both 256-column TMEM slots (its epilogue then runs after the mainloop);
    // one-tile units alternate slots, so their epilogue overlaps the next
    // unit's mainloop. ----
    if (lane == 0) {
      int sa = 0, sb = 0, last = 1;
      uint32_t pha = 0, phb = 0, pu = 0;  // pu bit l: parity of slot l's uses so far
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        int row0, rows;
        pf_rows<MODE>(g, u / nN, row0, rows);
        const int mtn = rows > kPfBM ? 2 : 1;
        const int s0 = mtn == 2 ? 0 : (last ^ 1);
        last = mtn == 2 ? 1 : s0;
        for (int t = 0; t < mtn && ok; ++t) {
          const int sl = s0 + t;
          ok = mbar_wait(bar_acce + 8 * sl, ((pu >> sl) & 1u) ^ 1u);  // previous use drained
          pu ^= 1u << sl;
        }
        if (!ok) break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(s0 * kPfBN);
        for (int kb = 0; kb < nkb; ++kb) {
          ok = mbar_wait(bar_afull + 8 * sa, pha) && mbar_wait(bar_full + 8 * sb, phb);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a_s = base + sa * kPfAStage;
          const uint32_t b_s = base + kPfOffB + sb * kPfBStage;
          for (int t = 0; t < mtn; ++t) {
#pragma unroll
            for (int kk = 0; kk < kPfBK / 16; ++kk)
              umma_f16(acc + (uint32_t)(t * kPfBN), sw128_desc(a_s + t * kPfASub + kk * 32),
                       sw128_desc(b_s + kk * 32), kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(bar_aempty + 8 * sa);  // stages free once these MMAs complete
          umma_commit(bar_empty + 8 * sb);
          if (++sa == kPfAStages) sa = 0, pha ^= 1u;
          if (++sb == kPfBStages) sb = 0, phb ^= 1u;
        }
        if (ok)
          for (int t = 0; t < mtn; ++t) umma_commit(bar_accf + 8 * (s0 + t));  // tile complete
      }
      // every MMA issued above has completed before the teardown
      umma_commit(bar_done);
      if (!mbar_wait(bar_done, 0)) ok = false;
    }
  } else if (warp == 2) {
    // ---- B-side producer: the unit's raw u4 codes by TMA, two k-blocks per
    // 64-byte row ----
    if (lane == 0) {
      int cs = 0;
      uint32_t ph = 0;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const PfUnit un = pf_unit<MODE>(g, u, nN);
        const CUtensorMap* wmap = un.proj == 0 ? &tmW : un.proj == 1 ? &tmW1 : un.proj == 2 ? &tmW2 : &tmW3;
        // nkb is a multiple of kPfCodeKB, so code stages never straddle units
        for (int cb = 0; cb < nkb / kPfCodeKB; ++cb) {
          ok = mbar_wait(bar_cempty + 8 * cs, ph ^ 1u);
          if (!ok) break;
          const uint32_t dst = base + kPfOffCodes + cs * kPfCodeStage;
          mbar_arrive_tx(bar_cfull + 8 * cs, kPfCodeStage);
          tma_load_2d(dst, wmap, cb * kPfCodeRow, (int)un.wr0, bar_cfull + 8 * cs);
          tma_load_2d(dst + kPfCodeStage / 2, wmap, cb * kPfCodeRow, (int)un.wr1,
                      bar_cfull + 8 * cs);
          if (++cs == kPfCodeStages) cs = 0, ph ^= 1u;
        }
      }
    }
  } else if (warp < kPfWarpEpi0) {
    // ---- dequant: thread pair (2n, 2n+1) owns row n of the 256-row B tile,
    // k 0..31 and 32..63 of each k-block, written in the canonical SW128
    // K-major layout. Scales and zero points come from global memory, the
    // next group's requested while the current one is dequantised (a row's
    // scales hit L1 after the first k-block). ----
    const int dt = threadIdx.x - kPfWarpDq0 * 32;
    const int n = dt >> 1, hk = dt & 1;
    const int x8 = n & 7;
    const __half2 sixteenth = __float2half2_rn(0.0625f);
    const uint8_t* const csrc = smem + kPfOffCodes + n * kPfCodeRow + hk * 16;
    uint8_t* const bdst = smem + kPfOffB + n * 128;
    const int gsh = g64 ? 0 : 1;  // k-block -> quant group shift
    int s = 0, cs = 0, sub = 0;
    uint32_t ph = 0, cph = 0;
    for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
      const PfUnit un = pf_unit<MODE>(g, u, nN);
      const int64_t row = n < 128 ? un.wr0 + n : un.wr1 + (n - 128);
      const __half* ssc = (MODE == 2 ? g.ps[un.proj] : g.s) + row * ng;
      const uint8_t* szp = (MODE == 2 ? g.pz[un.proj] : g.z) + row * (ng / 2);
      int grp = 0;
      __half sc = __ldg(ssc);
      uint32_t zb = __ldg(szp);
      for (int kb = 0; kb < nkb; ++kb) {
        ok = mbar_wait(bar_cfull + 8 * cs, cph);
        if (!ok) break;
        const uint4 v =
            *reinterpret_cast<const uint4*>(csrc + cs * kPfCodeStage + sub * (kPfBK / 2));
        const int gn = (kb + 1) >> gsh;
        __half sc_n = sc;
        uint32_t zb_n = zb;
        if (kb + 1 < nkb && gn != grp) {
          sc_n = __ldg(ssc + gn);
          zb_n = __ldg(szp + (gn >> 1));
        }
        ok = mbar_wait(bar_empty + 8 * s, ph ^ 1u);
        if (!ok) break;
        const uint32_t zz = (zb >> ((grp & 1) * 4)) & 15u;
        const __half2 s2 = __halves2half2(sc, sc);
        const __half2 s16 = __hmul2(s2, sixteenth);
        const uint32_t zlo = 0x64006400u | zz | (zz << 16);
        const uint32_t zhi = 0x64006400u | (zz << 4) | (zz << 20);
        uint8_t* bst = bdst + s * kPfBStage;
        const uint32_t* wv = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c = hk * 4 + cc;  // 16-byte chunk of the 128-byte B row
          uint32_t wd = wv[cc];
          uint32_t q0 = hsub2_u32(lop3_and_or(wd, 0x000F000Fu, 0x64006400u), zlo);
          uint32_t q1 = hsub2_u32(lop3_and_or(wd, 0x00F000F0u, 0x64006400u), zhi);
          wd >>= 8;
          uint32_t q2 = hsub2_u32(lop3_and_or(wd, 0x000F000Fu, 0x64006400u), zlo);
          uint32_t q3 = hsub2_u32(lop3_and_or(wd, 0x00F000F0u, 0x64006400u), zhi);
          __half2 r0 = __hmul2(*reinterpret_cast<__half2*>(&q0), s2);
          __half2 r1 = __hmul2(*reinterpret_cast<__half2*>(&q1), s16);
          __half2 r2 = __hmul2(*reinterpret_cast<__half2*>(&q2), s2);
          __half2 r3 = __hmul2(*reinterpret_cast<__half2*>(&q3), s16);
          uint4 o;
          o.x = *reinterpret_cast<uint32_t*>(&r0);
          o.y = *reinterpret_cast<uint32_t*>(&r1);
          o.z = *reinterpret_cast<uint32_t*>(&r2);
          o.w = *reinterpret_cast<uint32_t*>(&r3);
          *reinterpret_cast<uint4*>(bst + ((c ^ x8) << 4)) = o;
        }
        // One proxy fence orders this k-block's generic accesses against the
        // async proxy both ways: the B-tile stores before the MMA reads them,
        // and the code loads before the next TMA overwrites their slot
        // (without it such a write was observed to land first, corrupting
        // rows once units ran back to back).
        fence_proxy_async_smem();
        if (sub == kPfCodeKB - 1) mbar_arrive(bar_cempty + 8 * cs);  // release the code slot
        mbar_arrive(bar_full + 8 * s);
        grp = gn;
        sc = sc_n;
        zb = zb_n;
        if (++s == kPfBStages) s = 0, ph ^= 1u;
        if (++sub == kPfCodeKB) {
          sub = 0;
          if (++cs == kPfCodeStages) cs = 0, cph ^= 1u;
        }
      }
    }
  } else {
    // ---- epilogue: TMEM -> registers -> global, one tile row per thread,
    // the unit's tiles in slot order ----
    const int sp = warp & 3;       // TMEM sub-partition of this warp
    const int m = sp * 32 + lane;  // tile row = TMEM lane
    int last = 1;
    uint32_t pu = 0;
    for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
      const int mt = u / nN, nt = u - mt * nN;
      int urow0, urows;
      pf_rows<MODE>(g, mt, urow0, urows);
      const int mtn = urows > kPfBM ? 2 : 1;
      const int s0 = mtn == 2 ? 0 : (last ^ 1);
      last = mtn == 2 ? 1 : s0;
      for (int t = 0; t < mtn; ++t) {
        const int a = s0 + t;
        // warp-uniform: the TMEM loads below are warp-collective
        ok = __all_sync(0xffffffffu, mbar_wait(bar_accf + 8 * a, (pu >> a) & 1u));
        if (!ok) break;
        pu ^= 1u << a;
        tc_fence_after();
        const int row0 = urow0 + t * kPfBM, rows = min(kPfBM, urows - t * kPfBM);
        const uint32_t tl = tmem + (uint32_t)(a * kPfBN) + ((uint32_t)(sp * 32) << 16);
        if (MODE == 0 || MODE == 3) {
          for (int j = 0; j < 128; j += 16) {
            uint32_t gv[16], uv[16];
            tmem_ld16(tl + j, gv);
            tmem_ld16(tl + 128 + j, uv);
            tmem_ld_wait();
            if (m < rows && MODE == 3) {
              // natural column order, [T, I] fp16
              __half* dst = reinterpret_cast<__half*>(g.out) + (size_t)(row0 + m) * g.I + nt * 128 + j;
              uint32_t hw[8];
#pragma unroll
              for (int c = 0; c < 8; ++c) {
                const float g0 = __uint_as_float(gv[2 * c]), u0 = __uint_as_float(uv[2 * c]);
                const float g1 = __uint_as_float(gv[2 * c + 1]), u1 = __uint_as_float(uv[2 * c + 1]);
                hw[c] = pack_half2(__float2half_rn(g0 * sigmoidf_acc(g0) * u0),
                                   __float2half_rn(g1 * sigmoidf_acc(g1) * u1));
              }
              st_global_32b(dst, make_uint4(hw[0], hw[1], hw[2], hw[3]),
                            make_uint4(hw[4], hw[5], hw[6], hw[7]),
                            (reinterpret_cast<uintptr_t>(g.out) & 31) == 0);
            } else if (m < rows) {
              __half* dst = g.work.act + (size_t)(row0 + m) * g.I + nt * 128 + j;
              uint4 o2[2];
#pragma unroll
              for (int q = 0; q < 2; ++q) {
                __half a8[8];
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                  const float gt = __uint_as_float(gv[8 * q + c]);
                  const float up = __uint_as_float(uv[8 * q + c]);
                  a8[c] = __float2half_rn(gt * sigmoidf_acc(gt) * up);
                }
                uint4 o;
                o.x = pack_half2(a8[0], a8[4]);
                o.y = pack_half2(a8[1], a8[5]);
                o.z = pack_half2(a8[2], a8[6]);
                o.w = pack_half2(a8[3], a8[7]);
                o2[q] = o;
              }
              st_global_32b(dst, o2[0], o2[1], true);  // workspace rows: 256-byte aligned
            }
          }
        } else if (MODE == 2) {
          int pj, ntl;
          pf_proj(g, nt, pj, ntl);
          void* const pout = g.pout[pj];
          const bool pout32 = (reinterpret_cast<uintptr_t>(pout) & 31) == 0;
          const int prow = g.prow[pj], pdt = g.pdt[pj], pacc = g.pacc[pj];
          const float rg =
              (g.row_gate != nullptr && m < rows) ? sigmoidf_acc(g.row_gate[row0 + m]) : 1.f;
          for (int j = 0; j < kPfBN; j += 16) {
            uint32_t yv[16];
            tmem_ld16(tl + j, yv);
            tmem_ld_wait();
            if (g.row_gate != nullptr) {
#pragma unroll
              for (int q = 0; q < 16; ++q) yv[q] = __float_as_uint(__uint_as_float(yv[q]) * rg);
            }
            if (m < rows) {
              const size_t o = (size_t)(row0 + m) * prow + ntl * kPfBN + j;
              if (pdt == IQ36_F16) {
                uint4 h[2];
                uint32_t* hw = reinterpret_cast<uint32_t*>(h);
#pragma unroll
                for (int q = 0; q < 8; ++q)
                  hw[q] = pack_half2(__float2half_rn(__uint_as_float(yv[2 * q])),
                                     __float2half_rn(__uint_as_float(yv[2 * q + 1])));
                st_global_32b(reinterpret_cast<__half*>(pout) + o, h[0], h[1], pout32);
              } else {
                float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(pout) + o);
                float4 v4[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  float4 v = make_float4(__uint_as_float(yv[4 * q]), __uint_as_float(yv[4 * q + 1]),
                                         __uint_as_float(yv[4 * q + 2]),
                                         __uint_as_float(yv[4 * q + 3]));
                  if (pacc) {
                    // residual += the fp16-rounded projection output
                    const float4 r = dst[q];
                    v.x = r.x + __half2float(__float2half_rn(v.x));
                    v.y = r.y + __half2float(__float2half_rn(v.y));
                    v.z = r.z + __half2float(__float2half_rn(v.z));
                    v.w = r.w + __half2float(__float2half_rn(v.w));
                  }
                  v4[q] = v;
                }
                const uint4* u4v = reinterpret_cast<const uint4*>(v4);
                st_global_32b(dst, u4v[0], u4v[1], pout32);
                st_global_32b(dst + 2, u4v[2], u4v[3], pout32);
              }
            }
          }
        } else {
          const float wt = m < rows ? g.work.perm_w[row0 + m] : 0.f;
          for (int j = 0; j < kPfBN; j += 16) {
            uint32_t yv[16];
            tmem_ld16(tl + j, yv);
            tmem_ld_wait();
            if (m < rows) {
              __half* dst = g.work.y + (size_t)(row0 + m) * g.H + nt * kPfBN + j;
              uint4 o2[2];
#pragma unroll
              for (int q = 0; q < 2; ++q) {
                uint4 o;
                o.x = pack_half2(__float2half_rn(__uint_as_float(yv[8 * q]) * wt),
                                 __float2half_rn(__uint_as_float(yv[8 * q + 1]) * wt));
                o.y = pack_half2(__float2half_rn(__uint_as_float(yv[8 * q + 2]) * wt),
                                 __float2half_rn(__uint_as_float(yv[8 * q + 3]) * wt));
                o.z = pack_half2(__float2half_rn(__uint_as_float(yv[8 * q + 4]) * wt),
                                 __float2half_rn(__uint_as_float(yv[8 * q + 5]) * wt));
                o.w = pack_half2(__float2half_rn(__uint_as_float(yv[8 * q + 6]) * wt),
                                 __float2half_rn(__uint_as_float(yv[8 * q + 7]) * wt));
                o2[q] = o;
              }
              st_global_32b(dst, o2[0], o2[1], true);  // workspace rows: 256-byte aligned
            }
          }
        }
        tc_fence_before();
        mbar_arrive(bar_acce + 8 * a);  // this accumulator may be overwritten
      }
    }
  }
  if (!ok) {
    atomicExch(g.work.err, 1);
    if ((threadIdx.x & 31) == 0) atomicAdd(&g_gemm_wait_timeouts, 1);
  }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Router logits over T prompt tokens on tcgen05: logits[t, e] = xn[t] . W[e]
// (fp16 operands, fp32 accumulation in the tensor core), slogit[t] = xn[t] .
// w_sg. One CTA per 128-token tile and nc-column slice of the experts (nc =
// 256, or 128 with two CTAs per tile when the tiles alone would fill fewer
// than half the SMs): warp 0 streams 64-wide K blocks of xn (128 rows), the
// slice of W (nc rows; rows past E read as zeros) and, in the first slice,
// the shared-gate row (a 16-row box, rows past the first read as zeros) into
// a 4-stage ring; warp 1 issues M128 x Nnc and M128 x N16 MMAs into TMEM
// columns [0, nc) and [256, 272); warps 2-5 (thread = token = TMEM lane)
// store the rows.
// The logits equal the decode router's up to fp32 summation order (the
// reference's own router check: max-abs <= 1e-4).
constexpr int kRtM = 128, kRtN = 256, kRtNs = 16, kRtBK = 64, kRtStages = 4;
constexpr int kRtA = kRtM * 128, kRtB = kRtN * 128, kRtBs = kRtNs * 128;
constexpr int kRtStage = kRtA + kRtB + kRtBs;  // 51200 B, every piece 1024-aligned
constexpr int kRtOffBar = kRtStages * kRtStage;
constexpr int kRtSmem = kRtOffBar + 256 + 1024;
constexpr uint32_t kRtIdescS = (1u << 4) | ((uint32_t)(kRtNs >> 3) << 17) | ((uint32_t)(kRtM >> 4) << 24);

__global__ void __launch_bounds__(192, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmS, int has_sg, int T, int H, int E,
                     int nc, float* logits, float* slogit) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_raw = smem_u32(smem_raw);
  const uint32_t base = (base_raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - base_raw);
  const uint32_t bar = base + kRtOffBar;
  const uint32_t bar_full = bar, bar_empty = bar + 8 * kRtStages, bar_done = bar + 16 * kRtStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kRtOffBar + 192);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kRtM, n0 = blockIdx.y * nc;
  const int nk = H / kRtBK;
  const bool sg = has_sg && blockIdx.y == 0;  // the first slice also computes the shared gate
  const uint32_t idesc = (1u << 4) | ((uint32_t)(nc >> 3) << 17) | ((uint32_t)(kRtM >> 4) << 24);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kRtStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  bool ok = true;
  if (warp == 0) {
    if (lane == 0) {
      const uint32_t tx = kRtA + (uint32_t)nc * 128u + (sg ? kRtBs : 0);
      for (int kb = 0; kb < nk && ok; ++kb) {
        const int s = kb % kRtStages;
        ok = mbar_wait(bar_empty + 8 * s, ((kb / kRtStages) & 1) ^ 1u);
        if (!ok) break;
        const uint32_t st = base + s * kRtStage;
        mbar_arrive_tx(bar_full + 8 * s, tx);
        tma_load_2d(st, &tmX, kb * kRtBK, m0, bar_full + 8 * s);
        tma_load_2d(st + kRtA, &tmW, kb * kRtBK, n0, bar_full + 8 * s);
        if (sg) tma_load_2d(st + kRtA + kRtB, &tmS, kb * kRtBK, 0, bar_full + 8 * s);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      for (int kb = 0; kb < nk && ok; ++kb) {
        const int s = kb % kRtStages;
        ok = mbar_wait(bar_full + 8 * s, (kb / kRtStages) & 1);
        if (!ok) break;
        tc_fence_after();
        const uint32_t st = base + s * kRtStage;
#pragma unroll
        for (int kk = 0; kk < kRtBK / 16; ++kk) {
          const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
          umma_f16(tmem, sw128_desc(st + kk * 32), sw128_desc(st + kRtA + kk * 32), idesc, acc);
          if (sg)
            umma_f16(tmem + kRtN, sw128_desc(st + kk * 32), sw128_desc(st + kRtA + kRtB + kk * 32),
                     kRtIdescS, acc);
        }
        umma_commit(bar_empty + 8 * s);
      }
      umma_commit(bar_done);
    }
  } else {
    // thread = token row = TMEM lane; warps 2,3,4,5 own lanes 64.., 96.., 0.., 32..
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane, t = m0 + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    ok = mbar_wait(bar_done, 0);
    if (ok) {
      tc_fence_after();
      const int ncol = min(nc, E - n0);  // this slice's expert columns
      for (int c = 0; c < (ncol + 15) / 16; ++c) {
        uint32_t v[16];
        tmem_ld16(tmem + lane_off + c * 16, v);
        tmem_ld_wait();
        if (t < T) {
          float* dst = logits + (size_t)t * E + n0 + c * 16;
          if ((E & 3) == 0 && c * 16 + 16 <= ncol) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              reinterpret_cast<float4*>(dst)[q] =
                  make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                              __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (c * 16 + j < ncol) dst[j] = __uint_as_float(v[j]);
          }
        }
      }
      if (sg) {
        uint32_t v[16];
        tmem_ld16(tmem + lane_off + kRtN, v);
        tmem_ld_wait();
        if (t < T) slogit[t] = __uint_as_float(v[0]);
      }
    }
  }
  if (!ok && lane == 0) atomicAdd(&g_gemm_wait_timeouts, 1);
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// Host side

struct PfLayout {
  size_t hist, cbase, offset, tile_count, tile_expert, tile_row0, tile_rows, inv, perm_tok,
      perm_w, err, xp, act, y, total;
};

static size_t up256(size_t x) { return (x + 255) / 256 * 256; }

static PfLayout pf_layout(int T, int k, int E, int H, int I) {
  const size_t P = (size_t)T * k;
  const size_t nC = (P + kPfChunk - 1) / kPfChunk;
  const size_t maxt = (P + kPfBM - 1) / kPfBM + E;
  PfLayout L{};
  size_t o = 0;
  L.hist = o; o += up256(nC * E * 4);
  L.cbase = o; o += up256(nC * E * 4);
  L.offset = o; o += up256((size_t)E * 4);
  L.tile_count = o; o += 256;
  L.tile_expert = o; o += up256(maxt * 4);
  L.tile_row0 = o; o += up256(maxt * 4);
  L.tile_rows = o; o += up256(maxt * 4);
  L.inv = o; o += up256(P * 4);
  L.perm_tok = o; o += up256(P * 4);
  L.perm_w = o; o += up256(P * 4);
  L.err = o; o += 256;
  L.xp = o; o += up256((P + kPfBM) * (size_t)H * 2);
  L.act = o; o += up256((P + kPfBM) * (size_t)I * 2);
  L.y = o; o += up256((P + kPfBM) * (size_t)H * 2);
  L.total = o;
  return L;
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D fp16 activation tensor [rows, cols] (cols contiguous), box 64 x 128,
// SWIZZLE_128B (lands in the canonical SW128 K-major layout).
static bool make_act_map(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t cols) {
  auto enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kPfBK, (cuuint32_t)kPfBM};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D fp16 tensor [rows, cols], box 64 columns x box_rows rows, SWIZZLE_128B;
// a box reaching past the rows reads zeros.
static bool make_f16_map(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t cols,
                         uint32_t box_rows) {
  auto enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64u, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// logits [T, E] fp32 (and slogit [T] when w_sg is set) from xn [T, H] fp16.
int router_tc_launch(const __half* xn, int T, int H, const void* w_router, int E,
                     const void* w_sg, float* logits, float* slogit, cudaStream_t stream) {
  if (!xn || !w_router || !logits || (w_sg && !slogit)) return IQ36_ERR_ARG;
  if (T < 1 || E < 1 || E > kRtN || H < kRtBK || H % kRtBK) return IQ36_ERR_SHAPE;
  if (!aligned(xn, 16) || !aligned(w_router, 16) || (w_sg && !aligned(w_sg, 16)) ||
      !aligned(logits, 16))
    return IQ36_ERR_ALIGN;
  int sms = 148, dev0 = 0;
  if (cudaGetDevice(&dev0) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev0) != cudaSuccess)
    return IQ36_ERR_CUDA;
  const int mtiles = (T + kRtM - 1) / kRtM;
  const int nsplit = (E > kRtN / 2 && 2 * mtiles <= sms) ? 2 : 1, nc = kRtN / nsplit;
  CUtensorMap mx, mw, ms;
  if (!make_f16_map(&mx, xn, (uint64_t)T, (uint64_t)H, kRtM) ||
      !make_f16_map(&mw, w_router, (uint64_t)E, (uint64_t)H, (uint32_t)nc) ||
      !make_f16_map(&ms, w_sg ? w_sg : w_router, 1, (uint64_t)H, kRtNs))
    return IQ36_ERR_CUDA;
  static std::atomic<bool> attr_set[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return IQ36_ERR_CUDA;
  if (!attr_set[dev].load()) {
    if (cudaFuncSetAttribute(router_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kRtSmem) != cudaSuccess)
      return IQ36_ERR_CUDA;
    attr_set[dev].store(true);
  }
  const cudaError_t e = launch(router_tc_kernel, dim3(mtiles, nsplit), dim3(192),
                               (size_t)kRtSmem, stream, mx, mw, ms, w_sg ? 1 : 0, T, H, E, nc,
                               logits, slogit);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

// 2-D u8 code tensor [rows, bytes_per_row], box 64 bytes x 128 rows, no swizzle.
static bool make_code_map(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t row_bytes) {
  auto enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[2] = {row_bytes, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)kPfCodeRow, 128u};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t moe_prefill_ws(int T, int k, int E, int H, int I) { return pf_layout(T, k, E, H, I).total; }

int gemm_wait_timeouts(int* count, int reset) {
  if (cudaMemcpyFromSymbol(count, g_gemm_wait_timeouts, sizeof(int)) != cudaSuccess)
    return IQ36_ERR_CUDA;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_gemm_wait_timeouts, &zero, sizeof(int)) != cudaSuccess)
      return IQ36_ERR_CUDA;
  }
  return IQ36_OK;
}

// row_of == nullptr: x is [T, H] and assignment t*k+j reads row t. Otherwise
// (k must be 1) x is [n_rows, H] and assignment a reads row row_of[a].
int moe_prefill_launch(const void* x, int x_dtype, int T, const int32_t* ids,
                       const float* weights, int k, const iq36_expert_bank* b, void* out,
                       int out_dtype, int accumulate, void* ws, size_t ws_bytes,
                       cudaStream_t stream, const int32_t* row_of = nullptr, int n_rows = 0) {
  if (!x || !ids || !weights || !b || !out) return IQ36_ERR_ARG;
  if (row_of && (k != 1 || n_rows < 1)) return IQ36_ERR_SHAPE;
  if (x_dtype != IQ36_BF16 && x_dtype != IQ36_F16) return IQ36_ERR_ARG;
  if (accumulate && out_dtype != IQ36_F32) return IQ36_ERR_ARG;
  if (!b->gate_up_weight || !b->gate_up_scale || !b->gate_up_zp || !b->down_weight ||
      !b->down_scale || !b->down_zp)
    return IQ36_ERR_ARG;
  const int E = b->num_experts, H = b->hidden, I = b->intermediate;
  if ((b->group != 128 && b->group != 64) || T < 1 || k < 1 || k > 16 || E < 1 || E > 256)
    return IQ36_ERR_SHAPE;
  if (H % 256 || I % 128 || H < 256 || I < 128 || H > 2048 || I > 2048 ||
      (int64_t)T * k > (1 << 28))
    return IQ36_ERR_SHAPE;
  if (out_dtype != IQ36_F32 && out_dtype != IQ36_BF16 && out_dtype != IQ36_F16)
    return IQ36_ERR_ARG;
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(b->gate_up_weight, 16) ||
      !aligned(b->down_weight, 16) || !aligned(b->gate_up_scale, 16) ||
      !aligned(b->down_scale, 16) || !aligned(b->gate_up_zp, 16) || !aligned(b->down_zp, 16))
    return IQ36_ERR_ALIGN;
  const PfLayout L = pf_layout(T, k, E, H, I);
  if (!ws || ws_bytes < L.total) return IQ36_ERR_WORKSPACE;
  if (!aligned(ws, 256)) return IQ36_ERR_ALIGN;
  char* base = reinterpret_cast<char*>(ws);
  PfWork w;
  w.hist = reinterpret_cast<int32_t*>(base + L.hist);
  w.cbase = reinterpret_cast<int32_t*>(base + L.cbase);
  w.offset = reinterpret_cast<int32_t*>(base + L.offset);
  w.tile_count = reinterpret_cast<int32_t*>(base + L.tile_count);
  w.tile_expert = reinterpret_cast<int32_t*>(base + L.tile_expert);
  w.tile_row0 = reinterpret_cast<int32_t*>(base + L.tile_row0);
  w.tile_rows = reinterpret_cast<int32_t*>(base + L.tile_rows);
  w.inv = reinterpret_cast<int32_t*>(base + L.inv);
  w.perm_tok = reinterpret_cast<int32_t*>(base + L.perm_tok);
  w.perm_w = reinterpret_cast<float*>(base + L.perm_w);
  w.err = reinterpret_cast<int32_t*>(base + L.err);
  w.xp = reinterpret_cast<__half*>(base + L.xp);
  w.act = reinterpret_cast<__half*>(base + L.act);
  w.y = reinterpret_cast<__half*>(base + L.y);
  const int P = T * k;
  const int nC = (P + kPfChunk - 1) / kPfChunk;
  const int maxt = (P + kPfBM - 1) / kPfBM + E;

  CUtensorMap map_x, map_act, map_gu, map_d;
  if (!make_act_map(&map_x, w.xp, (uint64_t)P + kPfBM, (uint64_t)H) ||
      !make_act_map(&map_act, w.act, (uint64_t)P + kPfBM, (uint64_t)I) ||
      !make_code_map(&map_gu, b->gate_up_weight, (uint64_t)E * 2 * I, (uint64_t)H / 2) ||
      !make_code_map(&map_d, b->down_weight, (uint64_t)E * H, (uint64_t)I / 2))
    return IQ36_ERR_CUDA;
  static std::atomic<bool> attr_set[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return IQ36_ERR_CUDA;
  if (!attr_set[dev].load()) {
    if (cudaFuncSetAttribute(pf_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kPfSmem) != cudaSuccess ||
        cudaFuncSetAttribute(pf_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kPfSmem) != cudaSuccess)
      return IQ36_ERR_CUDA;
    attr_set[dev].store(true);
  }
  if (cudaMemsetAsync(w.err, 0, 4, stream) != cudaSuccess) return IQ36_ERR_CUDA;

  cudaError_t e = launch(pf_hist_kernel, dim3(nC), dim3(256), 0, stream, ids, P, E, w);
  if (e == cudaSuccess) e = launch(pf_scan_kernel, dim3(1), dim3(256), 0, stream, nC, E, w);
  if (e == cudaSuccess)
    e = launch(pf_place_kernel, dim3(nC), dim3(256), 0, stream, ids, weights, P, E, k, row_of,
               n_rows, w);
  if (e == cudaSuccess)
    e = launch(pf_gather_kernel, dim3(ceil_div(P, 8)), dim3(256), 0, stream, x,
               x_dtype == IQ36_F16 ? 1 : 0, P, H, w);
  GemmArgs g1{reinterpret_cast<const __half*>(b->gate_up_scale), b->gate_up_zp, (int64_t)2 * I,
              H, I, H, w};
  g1.g64 = b->group == 64;
  g1.mt = 1;
  g1.n1 = 0;
  g1.row1 = 0;
  // persistent grids: at most one CTA per SM, never more than the units
  int sms = 148;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return IQ36_ERR_CUDA;
  const int grid1 = std::max(1, std::min(sms, maxt * (I / 128)));
  const int grid2 = std::max(1, std::min(sms, maxt * (H / kPfBN)));
  if (e == cudaSuccess)
    e = launch(pf_gemm_kernel<0>, dim3(grid1), dim3(kPfThreads), (size_t)kPfSmem, stream,
               map_x, map_gu, map_gu, map_gu, map_gu, g1);
  GemmArgs g2{reinterpret_cast<const __half*>(b->down_scale), b->down_zp, (int64_t)H, I, I, H, w};
  g2.g64 = b->group == 64;
  g2.mt = 1;
  g2.n1 = 0;
  g2.row1 = 0;
  if (e == cudaSuccess)
    e = launch(pf_gemm_kernel<1>, dim3(grid2), dim3(kPfThreads), (size_t)kPfSmem, stream,
               map_act, map_d, map_d, map_d, map_d, g2);
  if (e == cudaSuccess)
    e = launch(pf_scatter_kernel, dim3(T), dim3(256), 0, stream, (const int32_t*)w.inv,
               (const __half*)w.y, T, H, k, out, out_dtype, accumulate);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Dense u4 GEMM (batched projections): out[T, N] = x W^T.

// Row t of x (fp32, optionally RMS-normalised with weight nw; or fp16) to the
// permuted fp16 operand layout of the GEMM (each 8-chunk as 0,4,1,5,2,6,3,7).
__global__ void __launch_bounds__(256) gemm_xprep_kernel(const void* x, int x_dtype,
                                                         const float* nw, float eps, int K,
                                                         __half* xp) {
  __shared__ float red[9];
  pdl_wait();
  const int t = blockIdx.x, tid = threadIdx.x;
  __half h[8];
  float scale = 1.f;
  const float* xf = reinterpret_cast<const float*>(x) + (size_t)t * K;
  const __half* xh = reinterpret_cast<const __half*>(x) + (size_t)t * K;
  if (x_dtype == IQ36_F32 && nw != nullptr) {
    float ss = 0.f;
    for (int i = tid; i < K; i += 256) ss = fmaf(xf[i], xf[i], ss);
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    if (tid == 0) {
      float v = 0.f;
      for (int w = 0; w < 8; ++w) v += red[w];
      red[8] = rsqrtf(v / (float)K + eps);
    }
    __syncthreads();
    scale = red[8];
  }
  for (int c = tid; c < K / 8; c += 256) {
    if (x_dtype == IQ36_F32) {
      // two 16-byte loads of x (and of nw) per 8-chunk (K % 256 == 0)
      float v[8], w[8];
      *reinterpret_cast<float4*>(v) = reinterpret_cast<const float4*>(xf + c * 8)[0];
      *reinterpret_cast<float4*>(v + 4) = reinterpret_cast<const float4*>(xf + c * 8)[1];
      if (nw != nullptr) {
        *reinterpret_cast<float4*>(w) = reinterpret_cast<const float4*>(nw + c * 8)[0];
        *reinterpret_cast<float4*>(w + 4) = reinterpret_cast<const float4*>(nw + c * 8)[1];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) h[j] = __float2half_rn(nw != nullptr ? v[j] * scale * w[j] : v[j]);
    } else {
      const uint4 raw = *reinterpret_cast<const uint4*>(xh + c * 8);
      const __half* hp = reinterpret_cast<const __half*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) h[j] = hp[j];
    }
    uint4 o;
    o.x = pack_half2(h[0], h[4]);
    o.y = pack_half2(h[1], h[5]);
    o.z = pack_half2(h[2], h[6]);
    o.w = pack_half2(h[3], h[7]);
    *reinterpret_cast<uint4*>(xp + (size_t)t * K + c * 8) = o;
  }
  pdl_launch_dependents();
}

size_t u4_gemm_ws(int T, int K) { return up256((size_t)(T + kPfBM) * K * 2) + 256; }

// Up to 4 projections sharing x (all K columns): out_p[T, rows_p] = x W_p^T.
// swiglu (one projection): W holds [gate; up] (2I rows); out[T, I] fp16 = SwiGLU
// of the two halves. row_gate (fp32 [T], optional, fp32 out only): each output
// row * sigmoid(row_gate[t]).
int u4_gemm_multi_launch(const void* x, int x_dtype, const float* nw, float eps, int T, int K,
                         int G, int n_proj, const iq36_u4_projection* proj, void* ws,
                         size_t ws_bytes, cudaStream_t stream, int swiglu = 0,
                         const float* row_gate = nullptr) {
  if (!x || !proj || n_proj < 1 || n_proj > 4) return IQ36_ERR_ARG;
  if (x_dtype != IQ36_F32 && x_dtype != IQ36_F16) return IQ36_ERR_ARG;
  if (nw && x_dtype != IQ36_F32) return IQ36_ERR_ARG;
  if (swiglu && n_proj != 1) return IQ36_ERR_ARG;
  if (row_gate && n_proj != 1) return IQ36_ERR_ARG;
  if ((G != 128 && G != 64) || T < 1 || K < 256 || K % 256 || K > 4096) return IQ36_ERR_SHAPE;
  if (!aligned(x, 16) || (nw && !aligned(nw, 16))) return IQ36_ERR_ALIGN;
  int total_rows = 0;
  for (int p = 0; p < n_proj; ++p) {
    const iq36_u4_projection& q = proj[p];
    const iq36_u4_matrix* w = &q.m;
    if (!w->weight || !w->scale || !w->zp || !q.out) return IQ36_ERR_ARG;
    if (q.out_dtype != IQ36_F32 && q.out_dtype != IQ36_F16) return IQ36_ERR_ARG;
    if (q.accumulate && q.out_dtype != IQ36_F32) return IQ36_ERR_ARG;
    if (swiglu && (q.out_dtype != IQ36_F16 || q.accumulate)) return IQ36_ERR_ARG;
    if (row_gate && q.out_dtype != IQ36_F32) return IQ36_ERR_ARG;
    if (w->rows < kPfBN || w->rows % kPfBN) return IQ36_ERR_SHAPE;
    if (!aligned(q.out, 16) || !aligned(w->weight, 16) || !aligned(w->scale, 16) ||
        !aligned(w->zp, 16))
      return IQ36_ERR_ALIGN;
    total_rows += w->rows;
  }
  if (!ws || ws_bytes < u4_gemm_ws(T, K)) return IQ36_ERR_WORKSPACE;
  if (!aligned(ws, 256)) return IQ36_ERR_ALIGN;
  __half* xp = reinterpret_cast<__half*>(ws);
  int32_t* err = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(ws) +
                                            up256((size_t)(T + kPfBM) * K * 2));
  CUtensorMap map_x, map_w[4];
  if (!make_act_map(&map_x, xp, (uint64_t)T + kPfBM, (uint64_t)K)) return IQ36_ERR_CUDA;
  for (int p = 0; p < n_proj; ++p)
    if (!make_code_map(&map_w[p], proj[p].m.weight, (uint64_t)proj[p].m.rows, (uint64_t)K / 2))
      return IQ36_ERR_CUDA;
  for (int p = n_proj; p < 4; ++p) map_w[p] = map_w[0];
  static std::atomic<bool> attr_set[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return IQ36_ERR_CUDA;
  if (!attr_set[dev].load()) {
    if (cudaFuncSetAttribute(pf_gemm_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kPfSmem) != cudaSuccess ||
        cudaFuncSetAttribute(pf_gemm_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kPfSmem) != cudaSuccess)
      return IQ36_ERR_CUDA;
    attr_set[dev].store(true);
  }
  int sms = 148;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return IQ36_ERR_CUDA;
  if (cudaMemsetAsync(err, 0, 4, stream) != cudaSuccess) return IQ36_ERR_CUDA;
  cudaError_t e = launch(gemm_xprep_kernel, dim3(T), dim3(256), 0, stream, x, x_dtype, nw, eps, K,
                         xp);
  PfWork wk{};
  wk.err = err;
  const iq36_u4_matrix* w0 = &proj[0].m;
  GemmArgs g{reinterpret_cast<const __half*>(w0->scale), w0->zp, 0, K, w0->rows / 2,
             total_rows, wk, T, proj[0].out, proj[0].out_dtype, proj[0].accumulate, row_gate};
  g.n_proj = n_proj;
  g.g64 = G == 64;
  g.tile_base[0] = 0;
  for (int p = 0; p < 4; ++p) {
    const bool have = p < n_proj;
    g.ps[p] = reinterpret_cast<const __half*>(have ? proj[p].m.scale : w0->scale);
    g.pz[p] = have ? proj[p].m.zp : w0->zp;
    g.pout[p] = have ? proj[p].out : proj[0].out;
    g.prow[p] = have ? proj[p].m.rows : w0->rows;
    g.pdt[p] = have ? proj[p].out_dtype : proj[0].out_dtype;
    g.pacc[p] = have ? proj[p].accumulate : 0;
    g.tile_base[p + 1] = g.tile_base[p] + (have ? proj[p].m.rows / kPfBN : 0);
  }
  // Unit shapes by a simulated makespan of the round-robin schedule: all
  // one-tile units, or two-tile units (a two-tile unit costs ~1.43 one-tile
  // units, measured: its second tile's MMAs plus an epilogue that cannot
  // overlap the next unit) with the last k pairs of rows run as one-tile units
  // first, which evens the CTAs' loads and offsets their write-bound
  // epilogues. The SwiGLU mode keeps one tile (two measured no faster).
  const int nt_units = total_rows / kPfBN;
  const int pairs = (T + 2 * kPfBM - 1) / (2 * kPfBM);
  auto makespan = [&](int mt, int k, int& n1, int& row1) {
    n1 = 0;
    row1 = T;
    if (mt == 2 && k > 0) {
      row1 = (pairs - k) * 2 * kPfBM;
      n1 = (T - row1 + kPfBM - 1) / kPfBM;
    }
    const int um = kPfBM * mt;
    const int mrows = n1 + (row1 + um - 1) / um;
    const int units = mrows * nt_units, grid = std::max(1, std::min(sms, units));
    double worst = 0.0;
    for (int b = 0; b < grid; ++b) {
      double load = 0.0;
      for (int u = b; u < units; u += grid) {
        const int r = u / nt_units;
        const int rows = r < n1 ? kPfBM : std::min(um, row1 - (r - n1) * um);
        load += rows > kPfBM ? 1.43 : 1.0;
      }
      worst = std::max(worst, load);
    }
    return worst;
  };
  int n1 = 0, row1 = T;
  double best = makespan(1, 0, n1, row1);
  g.mt = 1;
  g.n1 = 0;
  g.row1 = T;
  for (int k = 0; !swiglu && k < pairs; ++k) {
    const double m = makespan(2, k, n1, row1);
    if (m < best - 1e-9) {
      best = m;
      g.mt = 2;
      g.n1 = n1;
      g.row1 = row1;
    }
  }
  const int units = (g.n1 + (g.row1 + kPfBM * g.mt - 1) / (kPfBM * g.mt)) * nt_units;
  if (e == cudaSuccess)
    e = launch(swiglu ? pf_gemm_kernel<3> : pf_gemm_kernel<2>,
               dim3(std::max(1, std::min(sms, units))), dim3(kPfThreads), (size_t)kPfSmem, stream,
               map_x, map_w[0], map_w[1], map_w[2], map_w[3], g);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

int u4_gemm_launch(const void* x, int x_dtype, const float* nw, float eps, int T, int K, int G,
                   const iq36_u4_matrix* w, void* out, int out_dtype, int accumulate, void* ws,
                   size_t ws_bytes, cudaStream_t stream, int swiglu = 0,
                   const float* row_gate = nullptr) {
  if (!w) return IQ36_ERR_ARG;
  const iq36_u4_projection p{*w, out, out_dtype, accumulate};
  return u4_gemm_multi_launch(x, x_dtype, nw, eps, T, K, G, 1, &p, ws, ws_bytes, stream, swiglu,
                              row_gate);
}

}  // namespace iq36

extern "C" size_t iq36_u4_gemm_workspace_bytes(int32_t T, int32_t K) {
  return iq36::u4_gemm_ws(T, K);
}

extern "C" int iq36_u4_gemm(const void* x, int32_t x_dtype, const float* norm_weight,
                            float norm_eps, int32_t T, int32_t K, int32_t group,
                            const iq36_u4_matrix* w, void* out, int32_t out_dtype,
                            int32_t accumulate, void* workspace, size_t workspace_bytes,
                            iq36_stream_t stream) {
  return iq36::u4_gemm_launch(x, x_dtype, norm_weight, norm_eps, T, K, group, w, out, out_dtype,
                              accumulate, workspace, workspace_bytes, iq36::as_stream(stream));
}

extern "C" int iq36_u4_gemm_multi(const void* x, int32_t x_dtype, const float* norm_weight,
                                  float norm_eps, int32_t T, int32_t K, int32_t group,
                                  int32_t n_proj, const iq36_u4_projection* proj, void* workspace,
                                  size_t workspace_bytes, iq36_stream_t stream) {
  return iq36::u4_gemm_multi_launch(x, x_dtype, norm_weight, norm_eps, T, K, group, n_proj, proj,
                                    workspace, workspace_bytes, iq36::as_stream(stream));
}

extern "C" int iq36_moe_combine(const void* contrib_f16, const int32_t* inv, int32_t T,
                                int32_t H, int32_t k, void* out, int32_t out_dtype,
                                iq36_stream_t stream) {
  using namespace iq36;
  if (!contrib_f16 || !inv || !out) return IQ36_ERR_ARG;
  if (T < 0 || k < 1 || k > 16 || H < 4 || H % 4) return IQ36_ERR_SHAPE;
  if (out_dtype != IQ36_F32 && out_dtype != IQ36_BF16 && out_dtype != IQ36_F16)
    return IQ36_ERR_ARG;
  if (!aligned(contrib_f16, 8) || !aligned(out, 16)) return IQ36_ERR_ALIGN;
  if (T == 0) return IQ36_OK;
  const cudaError_t e = launch(pf_scatter_kernel, dim3(T), dim3(256), 0, as_stream(stream), inv,
                               reinterpret_cast<const __half*>(contrib_f16), (int)T, (int)H,
                               (int)k, out, (int)out_dtype, 0);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

extern "C" size_t iq36_moe_prefill_workspace_bytes(int32_t T, int32_t k, int32_t num_experts,
                                                   int32_t hidden, int32_t intermediate) {
  return iq36::moe_prefill_ws(T, k, num_experts, hidden, intermediate);
}

extern "C" int iq36_moe_prefill(const void* x_bf16, int32_t T, const int32_t* ids,
                                const float* weights, int32_t k, const iq36_expert_bank* routed,
                                void* out, int32_t out_dtype, void* workspace,
                                size_t workspace_bytes, iq36_stream_t stream) {
  return iq36::moe_prefill_launch(x_bf16, IQ36_BF16, T, ids, weights, k, routed, out, out_dtype,
                                  0, workspace, workspace_bytes, iq36::as_stream(stream));
}

extern "C" size_t iq36_moe_prefill_rows_workspace_bytes(int32_t n_assign, int32_t num_experts,
                                                        int32_t hidden, int32_t intermediate) {
  return iq36::moe_prefill_ws(n_assign, 1, num_experts, hidden, intermediate);
}

extern "C" int iq36_moe_prefill_rows(const void* x_bf16, int32_t n_rows, int32_t n_assign,
                                     const int32_t* row_of, const int32_t* ids,
                                     const float* weights, const iq36_expert_bank* routed,
                                     void* contrib_f16, void* workspace, size_t workspace_bytes,
                                     iq36_stream_t stream) {
  if (!x_bf16 || !row_of || !ids || !weights || !routed || !contrib_f16) return IQ36_ERR_ARG;
  if (n_rows < 0 || n_assign < 0) return IQ36_ERR_SHAPE;
  if (n_assign == 0) return IQ36_OK;
  if (n_rows == 0) return IQ36_ERR_SHAPE;
  return iq36::moe_prefill_launch(x_bf16, IQ36_BF16, n_assign, ids, weights, 1, routed,
                                  contrib_f16, IQ36_F16, 0, workspace, workspace_bytes,
                                  iq36::as_stream(stream), row_of, n_rows);
}

// ---------------------------------------------------------------------------
// The MoE block of one layer over T prompt tokens, residual updated in place:
// router logits on the RMS-normalised fp32 residual (the decode router's fp16
// input bit for bit, logits on tcgen05: equal to the decode step's up to fp32
// summation order; the normalised fp16 input also feeds the experts), top-k
// selection, the grouped routed experts (fp16 contributions summed in rank
// order into the residual), and the shared expert as two dense u4 GEMMs
// (gate_up with SwiGLU, then down scaled by sigmoid(shared logit) and added to
// the residual). run_qwen36_moe_ffn_layer (gguf_loader.cpp:5654-5782) with the
// grouped prefill schedule of grouped_s8_u4_f16_contribution_moe.cl:13-222.

namespace iq36 {
int router_logits_launch(const void* x_f16, const float* x_f32, const float* nw, float eps, int T,
                         int H, const void* w_router, int E, const void* w_sg, float* logits,
                         float* slogit, cudaStream_t stream);
int router_select_launch(const float* logits, int T, int E, int k, int32_t* ids, float* weights,
                         cudaStream_t stream);
int x_norm_launch(const float* x32, const float* nw, float eps, int T, int H, __half* xn,
                  cudaStream_t stream);
int router_tc_launch(const __half* xn, int T, int H, const void* w_router, int E,
                     const void* w_sg, float* logits, float* slogit, cudaStream_t stream);

struct MoeLayerPfLayout {
  size_t slogit, xn, act, gemm, moe, total;
};
static MoeLayerPfLayout moe_layer_pf_layout(int T, int k, int E, int H, int I) {
  MoeLayerPfLayout L{};
  size_t o = 0;
  L.slogit = o; o += up256((size_t)T * 4);
  L.xn = o; o += up256((size_t)T * H * 2);
  L.act = o; o += up256((size_t)T * I * 2);
  L.gemm = o; o += up256(u4_gemm_ws(T, std::max(H, I)));
  L.moe = o; o += up256(pf_layout(T, k, E, H, I).total);
  L.total = o;
  return L;
}
}  // namespace iq36

extern "C" size_t iq36_moe_layer_prefill_workspace_bytes(int32_t T, int32_t k, int32_t num_experts,
                                                         int32_t hidden, int32_t intermediate) {
  if (T < 1 || k < 1 || num_experts < 1 || hidden < 1 || intermediate < 1) return 0;
  return iq36::moe_layer_pf_layout(T, k, num_experts, hidden, intermediate).total;
}

extern "C" int iq36_moe_layer_prefill(float* residual, int32_t T, int32_t hidden,
                                      const float* norm_weight, float norm_eps,
                                      const void* w_router_f16, const void* w_shared_gate_f16,
                                      int32_t k, const iq36_expert_bank* routed,
                                      const iq36_expert_bank* shared, int32_t* ids,
                                      float* weights, float* logits, void* workspace,
                                      size_t workspace_bytes, iq36_stream_t stream) {
  using namespace iq36;
  if (!residual || !norm_weight || !w_router_f16 || !routed || !ids || !weights || !logits ||
      !workspace)
    return IQ36_ERR_ARG;
  if (shared && !w_shared_gate_f16) return IQ36_ERR_ARG;
  const int E = routed->num_experts, H = routed->hidden, I = routed->intermediate;
  if (T < 1 || hidden != H) return IQ36_ERR_SHAPE;
  if (shared && (shared->hidden != H || shared->intermediate != I || shared->group != routed->group))
    return IQ36_ERR_SHAPE;
  const MoeLayerPfLayout L = moe_layer_pf_layout(T, k, E, H, I);
  if (workspace_bytes < L.total) return IQ36_ERR_WORKSPACE;
  if (!aligned(workspace, 256) || !aligned(residual, 16)) return IQ36_ERR_ALIGN;
  char* ws = static_cast<char*>(workspace);
  float* slogit = reinterpret_cast<float*>(ws + L.slogit);
  __half* xn = reinterpret_cast<__half*>(ws + L.xn);
  __half* act = reinterpret_cast<__half*>(ws + L.act);
  const cudaStream_t s = as_stream(stream);
  int st = x_norm_launch(residual, norm_weight, norm_eps, T, H, xn, s);
  if (st == IQ36_OK)
    st = router_tc_launch(xn, T, H, w_router_f16, E, shared ? w_shared_gate_f16 : nullptr, logits,
                          shared ? slogit : nullptr, s);
  if (st == IQ36_OK) st = router_select_launch(logits, T, E, k, ids, weights, s);
  if (st == IQ36_OK)
    st = moe_prefill_launch(xn, IQ36_F16, T, ids, weights, k, routed, residual, IQ36_F32, 1,
                            ws + L.moe, L.total - L.moe, s);
  if (st == IQ36_OK && shared) {
    const iq36_u4_matrix gu{shared->gate_up_weight, shared->gate_up_scale, shared->gate_up_zp,
                            2 * I};
    const iq36_u4_matrix dn{shared->down_weight, shared->down_scale, shared->down_zp, H};
    st = u4_gemm_launch(xn, IQ36_F16, nullptr, 0.f, T, H, shared->group, &gu, act, IQ36_F16, 0,
                        ws + L.gemm, L.moe - L.gemm, s, 1, nullptr);
    if (st == IQ36_OK)
      st = u4_gemm_launch(act, IQ36_F16, nullptr, 0.f, T, I, shared->group, &dn, residual,
                          IQ36_F32, 1, ws + L.gemm, L.moe - L.gemm, s, 0, slogit);
  }
  return st;
}
