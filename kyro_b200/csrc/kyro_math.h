/*
 * kyro_math.h -- arithmetic shared bit-for-bit by the sm_100a kernels and the
 * CPU oracle of the speculative verify step.
 *
 * The reference verifier (src/speculative.rs:286-339) and sampler
 * (src/worker.rs:267-362) draw from an unseeded thread RNG and use candle's
 * softmax, so nothing in the reference fixes the random numbers or the
 * summation order.  This header fixes both, so that a CPU restatement and the
 * GPU kernels make identical accept/reject decisions and emit identical
 * tokens on identical inputs:
 *
 *   1. Philox4x32-10 counter-based uniforms (Salmon, Moraes, Dror, Shaw,
 *      "Parallel Random Numbers: As Easy as 1, 2, 3", SC'11), written from
 *      the paper: S-box multipliers 0xD2511F53 / 0xCD9E8D57, Weyl key bumps
 *      0x9E3779B9 / 0xBB67AE85, ten rounds.
 *      counter = (sequence, position, stream, step), key = seed.
 *      Streams: 0 draft sampling, 1 accept test, 2 resample / bonus token.
 *   2. ky_exp(): an fp32 exponential for x <= 0 built from basic IEEE
 *      operations only (round-to-nearest fma/mul/add and integer ops), so
 *      host and device produce the same bits.  Reduction x = n*ln2 + r,
 *      |r| <= ln2/2, then a degree-5 polynomial whose coefficients were
 *      fitted for this project by iterated weighted least squares
 *      (Lawson's algorithm on the relative error over [-ln2/2, ln2/2],
 *      c0 fixed at 1, stopped early and rounded to fp32; max relative error
 *      9.3e-8 before rounding).  oracle/exp_poly.py restates the fit and
 *      checks these constants.
 *      Inputs below -87 (and NaN) behave as -87; ky_exp(0) == 1 exactly.
 *   3. Fixed summation orders.  A chunk's softmax mass is an fp32 sum in one
 *      prescribed tree (ky_chunk_sum), and a row's normaliser a double sum
 *      in one prescribed butterfly, so a kernel that follows the same trees
 *      gets the same bits.  Inverse-CDF weights are integers,
 *      fix62(w) = floor(w * 2^62) for w in [0,2), whose sums do not depend
 *      on the order in which a kernel adds them.
 *   4. The inverse-CDF threshold: with a uniform u = odd * 2^-24 and integer
 *      total mass W, the sampled index is the smallest i whose inclusive
 *      prefix C_i satisfies u*W <= C_i, i.e. C_i >= ceil(odd*W / 2^24).
 *      This is the exact form of worker.rs:352-360 ("r -= p; if r <= 0").
 *
 * This header compiles as C11 (oracle, gcc) and as CUDA C++ (nvcc).
 */
#ifndef KYRO_MATH_H
#define KYRO_MATH_H

#include <stdint.h>

#if defined(__CUDACC__)
#define KY_HD __host__ __device__ __forceinline__
#else
#include <math.h>
#include <string.h>
#define KY_HD static inline
#endif

/* Round-to-nearest IEEE operations that the compiler may not contract or
 * reassociate.  Host code including this header is compiled with
 * -ffp-contract=off; device code uses the _rn intrinsics, which nvcc never
 * fuses. */
#if defined(__CUDA_ARCH__)
#define KY_FMAF(a, b, c) __fmaf_rn((a), (b), (c))
#define KY_FMUL(a, b) __fmul_rn((a), (b))
#define KY_FADD(a, b) __fadd_rn((a), (b))
#define KY_FSUB(a, b) __fsub_rn((a), (b))
#define KY_FDIV(a, b) __fdiv_rn((a), (b))
#define KY_DMUL(a, b) __dmul_rn((a), (b))
#define KY_DADD(a, b) __dadd_rn((a), (b))
#define KY_DSUB(a, b) __dsub_rn((a), (b))
#define KY_DDIV(a, b) __ddiv_rn((a), (b))
#else
#define KY_FMAF(a, b, c) fmaf((a), (b), (c))
#define KY_FMUL(a, b) ((float)(a) * (float)(b))
#define KY_FADD(a, b) ((float)(a) + (float)(b))
#define KY_FSUB(a, b) ((float)(a) - (float)(b))
#define KY_FDIV(a, b) ((float)(a) / (float)(b))
#define KY_DMUL(a, b) ((double)(a) * (double)(b))
#define KY_DADD(a, b) ((double)(a) + (double)(b))
#define KY_DSUB(a, b) ((double)(a) - (double)(b))
#define KY_DDIV(a, b) ((double)(a) / (double)(b))
#endif

KY_HD uint32_t ky_f2u(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(f);
#else
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
#endif
}

KY_HD float ky_u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}

/* ------------------------------------------------------------------ */
/* Philox4x32-10                                                        */
/* ------------------------------------------------------------------ */
#define KY_PHILOX_M0 0xD2511F53u
#define KY_PHILOX_M1 0xCD9E8D57u
#define KY_PHILOX_W0 0x9E3779B9u
#define KY_PHILOX_W1 0xBB67AE85u

enum {
  KY_STREAM_DRAFT = 0,   /* sampling a draft token from q          */
  KY_STREAM_ACCEPT = 1,  /* the accept test u < p(x)/q(x)           */
  KY_STREAM_RESAMPLE = 2 /* residual resample or bonus token        */
};

KY_HD void ky_mulhilo32(uint32_t a, uint32_t b, uint32_t* hi, uint32_t* lo) {
#if defined(__CUDA_ARCH__)
  *hi = __umulhi(a, b);
  *lo = a * b;
#else
  uint64_t p = (uint64_t)a * (uint64_t)b;
  *hi = (uint32_t)(p >> 32);
  *lo = (uint32_t)p;
#endif
}

/* Ten rounds of Philox4x32 on counter c[0..3] with key (k0, k1). */
KY_HD void ky_philox4x32_10(const uint32_t c_in[4], uint32_t k0, uint32_t k1, uint32_t out[4]) {
  uint32_t c0 = c_in[0], c1 = c_in[1], c2 = c_in[2], c3 = c_in[3];
  for (int round = 0; round < 10; ++round) {
    uint32_t hi0, lo0, hi1, lo1;
    ky_mulhilo32(KY_PHILOX_M0, c0, &hi0, &lo0);
    ky_mulhilo32(KY_PHILOX_M1, c2, &hi1, &lo1);
    uint32_t n0 = hi1 ^ c1 ^ k0;
    uint32_t n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += KY_PHILOX_W0;
    k1 += KY_PHILOX_W1;
  }
  out[0] = c0;
  out[1] = c1;
  out[2] = c2;
  out[3] = c3;
}

/* The odd 24-bit numerator of a uniform in (0,1): u = odd * 2^-24, with
 * odd = 2*(x>>9)+1 taken from the first Philox output word. u is exactly
 * representable in fp32 and never 0 or 1. */
KY_HD uint32_t ky_uniform_odd(uint64_t seed, uint32_t seq, uint32_t pos, uint32_t stream,
                              uint32_t step) {
  uint32_t c[4] = {seq, pos, stream, step};
  uint32_t o[4];
  ky_philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32), o);
  return ((o[0] >> 9) << 1) | 1u;
}

KY_HD float ky_odd_to_float(uint32_t odd) { return KY_FMUL((float)odd, 0x1p-24f); }

/* ------------------------------------------------------------------ */
/* exp for x <= 0                                                       */
/* ------------------------------------------------------------------ */
#define KY_LOG2E 0x1.715476p+0f
#define KY_LN2 0x1.62e430p-1f     /* ln2 rounded to fp32                    */
#define KY_RND_MAGIC 12582912.0f  /* 1.5 * 2^23                             */
#define KY_EXP_C0 0x1.000000p+0f
#define KY_EXP_C1 0x1.fffff6p-1f
#define KY_EXP_C2 0x1.fffdc0p-2f
#define KY_EXP_C3 0x1.555a74p-3f
#define KY_EXP_C4 0x1.573c44p-5f
#define KY_EXP_C5 0x1.0fa6c8p-7f

/* fmaxf returns the non-NaN operand on both host (C99) and device */
#define KY_FMAX(a, b) fmaxf((a), (b))

/* Shared core of ky_exp: x is clamped to [-87, +inf) (NaN -> -87), then
 * x = n*ln2 + r with n = rint(x*log2e) found by the 1.5*2^23 rounding trick
 * (t = 1.5*2^23 + n, so n sits in the low mantissa bits of t), r from one
 * fma with fp32 ln2, and e^r from a degree-5 polynomial fitted for this
 * project (relative error 9.4e-8 on |r| <= ln2/2, leading coefficient 1).
 * Returns the polynomial value; *tbits gets the bits of t. */
KY_HD float ky_exp_core(float x, uint32_t* tbits) {
  const float xc = KY_FMAX(x, -87.0f);
  const float t = KY_FMAF(xc, KY_LOG2E, KY_RND_MAGIC);
  const float nf = KY_FSUB(t, KY_RND_MAGIC);
  const float r = KY_FMAF(-nf, KY_LN2, xc);
  float p = KY_EXP_C5;
  p = KY_FMAF(p, r, KY_EXP_C4);
  p = KY_FMAF(p, r, KY_EXP_C3);
  p = KY_FMAF(p, r, KY_EXP_C2);
  p = KY_FMAF(p, r, KY_EXP_C1);
  p = KY_FMAF(p, r, KY_EXP_C0);
  *tbits = ky_f2u(t);
  return p;
}

/* 2^(n+s) from the bits of t = 1.5*2^23 + n.  The high bits of t's
 * encoding vanish when shifted left by 23, so (bits(t) + 127 + s) << 23
 * is the encoding of 2^(n+s) for -126 <= n+s <= 127. */
KY_HD float ky_pow2_from_t(uint32_t tbits, uint32_t s) {
  return ky_u2f((tbits + 127u + s) << 23);
}

/* e^x for x <= 0 (x below -87 behaves as -87, about 1.6e-38).  Relative
 * error within a few ulp; ky_exp(0) == 1 exactly. */
KY_HD float ky_exp(float x) {
  uint32_t tb;
  const float p = ky_exp_core(x, &tb);
  return KY_FMUL(p, ky_pow2_from_t(tb, 0u));
}

/* ------------------------------------------------------------------ */
/* fixed point                                                          */
/* ------------------------------------------------------------------ */
KY_HD uint64_t ky_f2u64_rz(float v) {
#if defined(__CUDA_ARCH__)
  return __float2ull_rz(v);
#else
  return (uint64_t)v;
#endif
}

/* floor(w * 2^62) for w in [0, 2). */
KY_HD uint64_t ky_fix62(float w) { return ky_f2u64_rz(KY_FMUL(w, 0x1p62f)); }

/* ceil(odd * W / 2^24): the smallest inclusive prefix C_i >= this value
 * marks the sampled index.  1 <= result <= W whenever W >= 1. */
KY_HD uint64_t ky_cdf_threshold(uint32_t odd, uint64_t W) {
  unsigned __int128 p = (unsigned __int128)odd * (unsigned __int128)W;
  p += (unsigned __int128)((1u << 24) - 1u);
  return (uint64_t)(p >> 24);
}

/* ------------------------------------------------------------------ */
/* softmax normaliser contract                                          */
/* ------------------------------------------------------------------ */
/* A vocabulary row is split into shards (tensor-parallel ranks; one shard
 * without TP), and each shard into chunks of KY_CHUNK consecutive entries
 * starting at the shard start (the last chunk may be short).  With
 * s_i = z_i * inv_t:
 *   m_c = max_{i in c} s_i
 *   e_i = ky_exp(s_i - m_c) at each of the chunk's KY_CHUNK positions; a
 *         position past the shard end has s_i = -inf (so e_i = ky_exp(-87))
 *   E_c = ky_chunk_sum(e_c)                   (fp32, the fixed tree below)
 *   M_r = max of m_c over the chunks of shard r
 *   M   = max_r M_r
 *   mass_c = E_c * ky_exp(m_c - M_r)          (double; c in shard r)
 *   S_r = butterfly sum of the chunk masses of shard r:
 *           t[l] = sum of mass_c over c = l, l+32, l+64, ... (in that order,
 *                  starting from 0.0), l = 0..31;
 *           for off = 16, 8, 4, 2, 1: t[l] = t[l] + t[l ^ off];  S_r = t[0]
 *         (the xor-shuffle reduction of a 32-lane warp, every lane ends
 *          with the same value)
 *   S   = sum of S_r * ky_shard_scale(M_r, M) over shards in rank order,
 *         starting from 0.0 (double)
 *   g_c = (float)(ky_exp(m_c - M) / S)        (double division)
 * Each shard's part is taken under its own maximum, so a rank sends its
 * (M_r, S_r) in one exchange round; with one shard, M_0 = M and the scale
 * is exactly 1, so S = S_0.
 *   p_i = e_i * g_c                           (fp32)
 * The same row statistics drive the accept test, the residual and the
 * bonus sample. */
/* 512 entries: one warp holds a chunk in registers (16 per lane), so a
 * chunk's statistics need no exchange between warps. */
#define KY_CHUNK 512

/* fp32 butterfly over 32 partial sums: for off = 16, 8, 4, 2, 1,
 * t[l] = t[l] + t[l ^ off]; returns t[0] (every entry ends equal, since
 * fp32 addition commutes). */
KY_HD float ky_butterfly32f(float t[32]) {
  for (int off = 16; off > 0; off >>= 1) {
    float n[32];
    for (int l = 0; l < 32; ++l) n[l] = KY_FADD(t[l], t[l ^ off]);
    for (int l = 0; l < 32; ++l) t[l] = n[l];
  }
  return t[0];
}

/* The chunk sum E_c.  Position (i*32 + l)*4 + j of the chunk (i = 0..3,
 * l = 0..31, j = 0..3) is term i of column j of lane l -- the float4 that
 * lane l of a warp loads in step i.  Each lane adds its columns' terms in
 * step order, then its four columns as (a0 + a1) + (a2 + a3), and the 32
 * lane totals meet in ky_butterfly32f. */
KY_HD float ky_chunk_sum(const float e[KY_CHUNK]) {
  float lanes[32];
  for (int l = 0; l < 32; ++l) {
    float acc[4];
    for (int j = 0; j < 4; ++j) {
      acc[j] = 0.0f;
      for (int i = 0; i < 4; ++i) acc[j] = KY_FADD(acc[j], e[(i * 32 + l) * 4 + j]);
    }
    lanes[l] = KY_FADD(KY_FADD(acc[0], acc[1]), KY_FADD(acc[2], acc[3]));
  }
  return ky_butterfly32f(lanes);
}

/* inv_t for temperature t > 0: (float)(1/(double)t); candle's `tensor / t`
 * (worker.rs:298) is an affine op multiplying by the reciprocal. */
KY_HD float ky_inv_temperature(float t) { return (float)KY_DDIV(1.0, (double)t); }

KY_HD double ky_chunk_mass(float E, float m_c, float M) {
  return KY_DMUL((double)E, (double)ky_exp(KY_FSUB(m_c, M)));
}

/* The factor that brings shard r's normaliser part S_r (taken under its own
 * maximum M_r) to the row maximum M: exactly 1 when M_r == M (one shard, the
 * shard holding the maximum, or an all -inf row). */
KY_HD double ky_shard_scale(float M_r, float M) {
  return M_r == M ? 1.0 : (double)ky_exp(KY_FSUB(M_r, M));
}

KY_HD float ky_chunk_scale(float m_c, float M, double S) {
  return (float)KY_DDIV((double)ky_exp(KY_FSUB(m_c, M)), S);
}

/* The butterfly combination of 32 partial sums (host side; the device uses
 * __shfl_xor_sync with the same offsets). */
KY_HD double ky_butterfly32(double t[32]) {
  for (int off = 16; off > 0; off >>= 1) {
    double n[32];
    for (int l = 0; l < 32; ++l) n[l] = KY_DADD(t[l], t[l ^ off]);
    for (int l = 0; l < 32; ++l) t[l] = n[l];
  }
  return t[0];
}

/* accept iff u < p/q (Leviathan et al. 2023, Alg. 1; u < min(1,p/q) since u < 1) */
KY_HD int ky_accept(uint32_t odd, float p, float q) {
  float ratio = KY_FDIV(p, q);
  return ky_odd_to_float(odd) < ratio;
}

/* Inverse-CDF weights.  With g62_c = g_c * 2^62 (exact) per chunk:
 *   sampling from p:   w_i = floor(e_i * g62_c)               = fix62(p_i)
 *   residual:          w_i = floor(max(e_i*g62_c - e'_i*g62'_c, 0))
 *                          = fix62(max(p_i - q_i, 0))
 * (scaling by 2^62 commutes with fp32 rounding except where a product is
 * subnormal, and those weights are 0 either way). */
KY_HD float ky_scale62(float g) { return KY_FMUL(g, 0x1p62f); }

KY_HD uint64_t ky_weight_p(float e, float g62) { return ky_f2u64_rz(KY_FMUL(e, g62)); }

KY_HD uint64_t ky_weight_residual(float ep, float g62p, float eq, float g62q) {
  const float d = KY_FSUB(KY_FMUL(ep, g62p), KY_FMUL(eq, g62q));
  return d > 0.0f ? ky_f2u64_rz(d) : 0ull;
}

/* ------------------------------------------------------------------ */
/* tree verification                                                    */
/* ------------------------------------------------------------------ */
/* Multi-candidate rejection sampling over a draft tree (SpecInfer, Miao et
 * al. 2023).  At a node with target distribution p and draft distribution
 * q (the contract's fp32 p_i and q_i, widened to double), the children are
 * tried in index order; child c with token x is accepted iff
 * u_c < p_j(x) / q(x) (double division), where j children have been
 * rejected so far and
 *   p_0(i) = p_i,
 *   p_{j+1}(i) = max(p_j(i) - q_i, 0) / R_j   with   R_j = sum_i max(p_j(i) - q_i, 0),
 * and p_{j+1} = p_j when R_j == 0 (then p_j == q and the next child is
 * accepted).  R_j is summed in one fixed tree: each 512-entry chunk by
 * ky_chunk_sum_d (ky_chunk_sum's tree in double; entries past V are 0),
 * the chunk sums by the 32-lane butterfly of the normaliser (chunks
 * c = l, l+32, ... into lane l, then ky_butterfly32).  A node whose
 * children are all rejected draws from p_J, a leaf from p_0, with integer
 * weights floor(p_J(i) * 2^62) and the chain's inverse-CDF threshold. */

KY_HD double ky_tree_step(double p, double q, double R) {
  if (R == 0.0) return p;
  const double d = KY_DSUB(p, q);
  return d > 0.0 ? KY_DDIV(d, R) : 0.0;
}

/* max(p - q, 0), the term of R_j */
KY_HD double ky_tree_excess(double p, double q) {
  const double d = KY_DSUB(p, q);
  return d > 0.0 ? d : 0.0;
}

/* ky_chunk_sum's lane tree in double */
KY_HD double ky_chunk_sum_d(const double e[KY_CHUNK]) {
  double lanes[32];
  for (int l = 0; l < 32; ++l) {
    double acc[4];
    for (int j = 0; j < 4; ++j) {
      acc[j] = 0.0;
      for (int i = 0; i < 4; ++i) acc[j] = KY_DADD(acc[j], e[(i * 32 + l) * 4 + j]);
    }
    lanes[l] = KY_DADD(KY_DADD(acc[0], acc[1]), KY_DADD(acc[2], acc[3]));
  }
  return ky_butterfly32(lanes);
}

/* floor(w * 2^62) for a probability w in [0, 1] */
KY_HD uint64_t ky_weight_d(double w) {
#if defined(__CUDA_ARCH__)
  return __double2ull_rz(KY_DMUL(w, 0x1p62));
#else
  return (uint64_t)(w * 0x1p62);
#endif
}

#endif /* KYRO_MATH_H */
