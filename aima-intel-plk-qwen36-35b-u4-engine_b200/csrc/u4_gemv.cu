// u4_gemv.cu — multi-output u4 group-wise GEMV (the fixed-FC family).
//
// Replaces IQ36FixedFC{1,3,4} (engine/openvino/custom/
// iq36_fixed_fc_multi_output.cl:6-200; launch geometry and grouping
// tools/intel_qwen36_openvino_fixed_fc.py:180-215,268-378): up to four
// projections of one activation in a single launch, rows of all projections
// concatenated into 16-row blocks.
//
// CTA = 8 warps = (8/KS) row blocks x KS K-splits. The activation (optionally
// RMS-normalised from the fp32 residual) is staged once per CTA; K-split
// partials are summed in fixed order in shared memory, so results are
// deterministic run to run.

#include "launch.cuh"
#include "u4_core.cuh"
#include "u4_stream.cuh"

namespace iq36 {

struct ProjSet {
  const uint8_t* w[4];
  const __half* s[4];
  const uint8_t* z[4];
  void* out[4];
  int rows[4];
  int dtype[4];
  int acc[4];
  int rb_start[5];
  int n_proj;
};

__device__ __forceinline__ void store_out(void* out, int dtype, int acc, int row, float v) {
  if (dtype == IQ36_F16) {
    reinterpret_cast<__half*>(out)[row] = __float2half_rn(v);
  } else if (acc) {
    // Residual update: the projection output is rounded to fp16 (the fixed-FC
    // output type, iq36_fixed_fc_multi_output.cl:198) and added in fp32.
    float* o = reinterpret_cast<float*>(out);
    o[row] = o[row] + __half2float(__float2half_rn(v));
  } else {
    reinterpret_cast<float*>(out)[row] = v;
  }
}

template <int G>
__global__ void __launch_bounds__(256) u4_gemv_multi_kernel(ProjSet ps, const __half* x16,
                                                            const float* x32, const float* nw,
                                                            float eps, int K, int ks_log2) {
  extern __shared__ uint4 xs[];
  __shared__ float red[8][16];
  __shared__ float nred[33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int KS = 1 << ks_log2;
  const int rb = blockIdx.x * (8 >> ks_log2) + (warp >> ks_log2);
  const int ks = warp & (KS - 1);
  const int ng = K / G;
  const int per = ng >> ks_log2;
  const bool valid = rb < ps.rb_start[ps.n_proj];
  float accA = 0.f, accB = 0.f;
  int p = 0, r0 = 0;
  U4Rows rows{};
  U4Chunk<G, 2> first;
  if (valid) {
    // Weights never depend on the previous kernel: start streaming them
    // before waiting on it.
    while (p + 1 < ps.n_proj && rb >= ps.rb_start[p + 1]) ++p;
    r0 = (rb - ps.rb_start[p]) * 16;
    const int nrows = ps.rows[p];
    const int rowA = min(r0 + g, nrows - 1), rowB = min(r0 + g + 8, nrows - 1);
    const uint8_t* w = ps.w[p];
    const __half* s = ps.s[p];
    rows = U4Rows{w + (size_t)rowA * (K / 2), w + (size_t)rowB * (K / 2), s + (size_t)rowA * ng,
                  s + (size_t)rowB * ng, ps.z[p], (int64_t)rowA * ng, (int64_t)rowB * ng};
    u4_load_chunk<G, 2>(first, rows, ks * per, (ks + 1) * per, t);
  }
  pdl_wait();
  stage_x_perm(xs, x16, x32, nw, eps, K, nred);
  pdl_launch_dependents();
  if (valid) u4_dot2_pipelined<G, 2>(first, rows, xs, ks * per, (ks + 1) * per, t, accA, accB);
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
    const int rows = ps.rows[p];
    if (r0 + g < rows) store_out(ps.out[p], ps.dtype[p], ps.acc[p], r0 + g, accA);
    if (r0 + g + 8 < rows) store_out(ps.out[p], ps.dtype[p], ps.acc[p], r0 + g + 8, accB);
  }
}

// K-split factor (log2): split each row block over up to 8 warps while the
// whole grid still fits one wave of 2 CTAs x 8 warps on each of the 148 SMs.
int u4_ks_log2(int total_rb, int ng) {
  constexpr int kWaveWarps = 148 * 2 * 8;
  int l = 0;
  while (l < 3 && (total_rb << (l + 1)) <= kWaveWarps && (ng % (2 << l)) == 0) ++l;
  return l;
}

static int check_matrix(const iq36_u4_matrix& m, int K, int G) {
  if (!m.weight || !m.scale || !m.zp) return IQ36_ERR_ARG;
  if (m.rows < 1) return IQ36_ERR_SHAPE;
  if (((int64_t)m.rows * (K / G)) % 2 != 0) return IQ36_ERR_SHAPE;
  if (!aligned(m.weight, 16) || !aligned(m.scale, 2)) return IQ36_ERR_ALIGN;
  return IQ36_OK;
}

int u4_gemv_multi_launch(const void* x_f16, const float* x_f32, const float* norm_w, float eps,
                         int K, int G, int n_proj, const iq36_u4_projection* proj,
                         cudaStream_t stream) {
  if (n_proj < 1 || n_proj > 4 || !proj) return IQ36_ERR_ARG;
  if (G != 64 && G != 128) return IQ36_ERR_SHAPE;
  if (K < G || K % G != 0 || K > 16384) return IQ36_ERR_SHAPE;
  if (x_f32) {
    if (x_f16 || !norm_w) return IQ36_ERR_ARG;
  } else {
    if (!x_f16) return IQ36_ERR_ARG;
    if (!aligned(x_f16, 16)) return IQ36_ERR_ALIGN;
  }
  ProjSet ps = {};
  ps.n_proj = n_proj;
  int rb = 0;
  for (int i = 0; i < n_proj; ++i) {
    const iq36_u4_projection& p = proj[i];
    const int st = check_matrix(p.m, K, G);
    if (st != IQ36_OK) return st;
    if (!p.out) return IQ36_ERR_ARG;
    if (p.out_dtype != IQ36_F32 && p.out_dtype != IQ36_F16) return IQ36_ERR_ARG;
    if (p.accumulate && p.out_dtype != IQ36_F32) return IQ36_ERR_ARG;
    ps.w[i] = p.m.weight;
    ps.s[i] = reinterpret_cast<const __half*>(p.m.scale);
    ps.z[i] = p.m.zp;
    ps.out[i] = p.out;
    ps.rows[i] = p.m.rows;
    ps.dtype[i] = p.out_dtype;
    ps.acc[i] = p.accumulate;
    ps.rb_start[i] = rb;
    rb += ceil_div(p.m.rows, 16);
  }
  ps.rb_start[n_proj] = rb;
  // Row counts in whole 16-row chunks and 16-byte aligned tensors take the
  // bulk-copy streaming kernel (u4_stream.cu); other shapes this one.
  if (stream_proj_ok(K, G, n_proj, proj))
    return stream_proj_launch(x_f16, x_f32, norm_w, eps, K, G, n_proj, proj, stream);
  const int ng = K / G;
  const int ks_log2 = u4_ks_log2(rb, ng);
  const int rb_per_cta = 8 >> ks_log2;
  const dim3 grid(ceil_div(rb, rb_per_cta));
  const size_t smem = (size_t)K / 8 * sizeof(uint4);
  const __half* xh = reinterpret_cast<const __half*>(x_f16);
  cudaError_t e;
  if (G == 128)
    e = launch(u4_gemv_multi_kernel<128>, grid, dim3(256), smem, stream, ps, xh, x_f32, norm_w,
               eps, K, ks_log2);
  else
    e = launch(u4_gemv_multi_kernel<64>, grid, dim3(256), smem, stream, ps, xh, x_f32, norm_w,
               eps, K, ks_log2);
  return e == cudaSuccess ? IQ36_OK : IQ36_ERR_CUDA;
}

}  // namespace iq36

extern "C" int iq36_u4_gemv(const void* x_f16, int32_t K, int32_t G, const iq36_u4_matrix* w,
                            void* out, int32_t out_dtype, iq36_stream_t stream) {
  if (!w) return IQ36_ERR_ARG;
  iq36_u4_projection p = {*w, out, out_dtype, 0};
  return iq36::u4_gemv_multi_launch(x_f16, nullptr, nullptr, 0.f, K, G, 1, &p,
                                    iq36::as_stream(stream));
}

extern "C" int iq36_u4_gemv_multi(const void* x_f16, const float* x_f32, const float* norm_weight,
                                  float norm_eps, int32_t K, int32_t G, int32_t n_proj,
                                  const iq36_u4_projection* proj, iq36_stream_t stream) {
  return iq36::u4_gemv_multi_launch(x_f16, x_f32, norm_weight, norm_eps, K, G, n_proj, proj,
                                    iq36::as_stream(stream));
}
