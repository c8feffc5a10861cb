/*
 * iq36_synth.h — counter-based synthetic weight generator shared by the CUDA
 * library (device-side model init) and by the CPU checker (host-side
 * regeneration of the same tensors).
 *
 * No counterpart in the reference: the reference loads a locked OpenVINO U4
 * checkpoint. This build runs on random-init weights of the same shapes, so the
 * generator is part of the input specification. Every value is a pure function
 * of (seed, tensor id, element index) computed with integer arithmetic plus at
 * most two correctly-rounded fp32 multiplies, so host and device produce
 * bit-identical tensors without transferring them.
 *
 * Distributions:
 *   u4 codes and u4 zero points: uniform 0..15 (one hash per packed byte);
 *   fp16 group scales: uniform [0.005, 0.02];
 *   "normal" values: Irwin-Hall sum of four 16-bit uniforms, centred and scaled
 *   to unit variance (support +-3.46), times the requested std.
 */
#ifndef IQ36_SYNTH_H
#define IQ36_SYNTH_H

#include <stdint.h>

#if defined(__CUDACC__)
#define IQ36_HD __host__ __device__ __forceinline__
#else
#define IQ36_HD static inline
#endif

IQ36_HD uint64_t iq36_mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* Hash of one element of one tensor. */
IQ36_HD uint64_t iq36_hash(uint64_t seed, uint64_t tensor, uint64_t index) {
  return iq36_mix64(iq36_mix64(seed ^ (tensor * 0xD1B54A32D192ED03ull)) + index);
}

/* One packed byte of u4 codes (two uniform nibbles). */
IQ36_HD uint8_t iq36_synth_u8(uint64_t seed, uint64_t tensor, uint64_t index) {
  return (uint8_t)(iq36_hash(seed, tensor, index) >> 24);
}

/* Separately rounded multiply and add: a compiler may not fuse them into an
 * FMA on one side only (nvcc contracts by default; the CPU checker is built
 * with -ffp-contract=off). */
#if defined(__CUDA_ARCH__)
#define IQ36_SYNTH_MUL(a, b) __fmul_rn((a), (b))
#define IQ36_SYNTH_ADD(a, b) __fadd_rn((a), (b))
#else
#define IQ36_SYNTH_MUL(a, b) ((a) * (b))
#define IQ36_SYNTH_ADD(a, b) ((a) + (b))
#endif

/* Uniform in [lo, hi) as fp32: 24-bit integer times 2^-24 is exact. */
IQ36_HD float iq36_synth_uniform(uint64_t seed, uint64_t tensor, uint64_t index,
                                 float lo, float hi) {
  const uint32_t u = (uint32_t)(iq36_hash(seed, tensor, index) >> 40);
  const float unit = (float)u * (1.0f / 16777216.0f);
  return IQ36_SYNTH_ADD(lo, IQ36_SYNTH_MUL(hi - lo, unit));
}

/* Approximately N(0, std^2): centred Irwin-Hall(4) of 16-bit uniforms.
 * The integer sum is exact; (sum - 131070) is exact in fp32; the two
 * multiplies are IEEE round-to-nearest on host and device alike. */
IQ36_HD float iq36_synth_normal(uint64_t seed, uint64_t tensor, uint64_t index,
                                float std_dev) {
  const uint64_t h = iq36_hash(seed, tensor, index);
  const int32_t s = (int32_t)(h & 0xFFFFu) + (int32_t)((h >> 16) & 0xFFFFu) +
                    (int32_t)((h >> 32) & 0xFFFFu) + (int32_t)((h >> 48) & 0xFFFFu);
  /* Var of one 16-bit uniform = (65536^2 - 1)/12; four of them: (65536^2-1)/3.
   * 1/sqrt((65536^2-1)/3) ~= sqrt(3)/65536. */
  const float z = IQ36_SYNTH_MUL((float)(s - 131070), 2.6429309e-05f);
  return IQ36_SYNTH_MUL(z, std_dev);
}

/* ---- synthetic model tensor spec (BASELINE config 4 shapes) ----------------
 * A tensor is named by (layer, slot, sub); layer -1 holds the global tensors.
 * u4 matrices have three subs: 0 codes (u8), 1 scales (fp16), 2 zero points
 * (u8). Expert banks store all experts contiguously in one tensor. */
enum iq36_slot {
  IQ36_T_EMBED = 1, IQ36_T_LM_HEAD = 2, IQ36_T_FINAL_NORM = 3,
  IQ36_T_IN_NORM = 8, IQ36_T_POST_NORM = 9,
  IQ36_T_Q = 10, IQ36_T_K = 11, IQ36_T_V = 12, IQ36_T_O = 13,
  IQ36_T_QNORM = 14, IQ36_T_KNORM = 15,
  IQ36_T_QKV = 16, IQ36_T_Z = 17, IQ36_T_A = 18, IQ36_T_B = 19, IQ36_T_OUT = 20,
  IQ36_T_CONV = 21, IQ36_T_ALOG = 22, IQ36_T_DTB = 23, IQ36_T_DNORM = 24,
  IQ36_T_ROUTER = 25, IQ36_T_SGATE = 26, IQ36_T_GU = 27, IQ36_T_DOWN = 28,
  IQ36_T_SGU = 29, IQ36_T_SDOWN = 30
};

IQ36_HD uint64_t iq36_tensor_id(int layer, int slot, int sub) {
  return ((uint64_t)(layer + 1) << 16) | ((uint64_t)slot << 4) | (uint64_t)sub;
}

/* Generator kind and parameters of each tensor (kinds as iq36_synth_fill). */
IQ36_HD void iq36_synth_spec(int slot, int sub, int* kind, float* lo, float* hi) {
  switch (slot) {
    case IQ36_T_EMBED: *kind = 2; *lo = 1.0f; *hi = 0.0f; return;
    case IQ36_T_ROUTER:
    case IQ36_T_SGATE: *kind = 2; *lo = 0.02f; *hi = 0.0f; return;
    case IQ36_T_FINAL_NORM: case IQ36_T_IN_NORM: case IQ36_T_POST_NORM:
    case IQ36_T_QNORM: case IQ36_T_KNORM: case IQ36_T_DNORM:
      *kind = 3; *lo = 0.9f; *hi = 1.1f; return;
    case IQ36_T_CONV: *kind = 3; *lo = -0.5f; *hi = 0.5f; return;
    case IQ36_T_ALOG: *kind = 3; *lo = -2.0f; *hi = 1.0f; return;
    case IQ36_T_DTB: *kind = 3; *lo = -1.0f; *hi = 1.0f; return;
    default: /* u4 matrices */
      if (sub == 1) { *kind = 1; *lo = 0.005f; *hi = 0.02f; }
      else { *kind = 0; *lo = 0.0f; *hi = 0.0f; }
      return;
  }
}

#endif /* IQ36_SYNTH_H */
