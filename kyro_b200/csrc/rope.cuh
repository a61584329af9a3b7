// rope.cuh -- the rotary position embedding arithmetic, shared by the paged
// K/V store (rope_kv_write_kernel) and the attention prologue that rotates
// the queries and stores the new keys itself, so that both write the same
// bits.
//
// RotaryEmbedding::apply (src/model/layers.rs:37-61) rotates the two halves
// of every head: y[i] = x[i]*cos(f_i) - x[i+D/2]*sin(f_i) and y[i+D/2] =
// x[i+D/2]*cos(f_i) + x[i]*sin(f_i), with f_i = pos * inv_freq[i] in fp32
// and inv_freq[i] = (float)(1 / theta^(2i/D)) formed in double (:26-33).
// Each product and the sum round to fp32 separately, as the reference's
// broadcast_mul / add do; cos and sin are those of the fp32 angle, rounded
// to fp32 (evaluated in double, so they are the correctly rounded values in
// all but vanishingly rare cases).
#pragma once

#include <stdint.h>

namespace kyro {
namespace rope {

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ uint32_t bf16_pack(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// cos and sin of the fp32 angle pos * inv_freq
__device__ __forceinline__ void angle(float pos, float inv_freq, float& c, float& s) {
  double sd, cd;
  sincos((double)__fmul_rn(pos, inv_freq), &sd, &cd);
  c = (float)cd;
  s = (float)sd;
}

// One bf16 pair of each half: wa holds x[i], x[i+1] and wb holds x[i+D/2],
// x[i+1+D/2]; c0, s0 belong to dim i and c1, s1 to dim i+1.  lo gets the
// rotated first-half pair, hi the second-half pair.
__device__ __forceinline__ void rotate_pair(uint32_t wa, uint32_t wb, float c0, float c1, float s0,
                                            float s1, uint32_t& lo, uint32_t& hi) {
  const float a0 = bf16_lo(wa), a1 = bf16_hi(wa);
  const float b0 = bf16_lo(wb), b1 = bf16_hi(wb);
  lo = bf16_pack(__fadd_rn(__fmul_rn(a0, c0), __fmul_rn(-b0, s0)),
                 __fadd_rn(__fmul_rn(a1, c1), __fmul_rn(-b1, s1)));
  hi = bf16_pack(__fadd_rn(__fmul_rn(b0, c0), __fmul_rn(a0, s0)),
                 __fadd_rn(__fmul_rn(b1, c1), __fmul_rn(a1, s1)));
}

}  // namespace rope
}  // namespace kyro
