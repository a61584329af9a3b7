// sampler.cu -- K2: vocab-wide acceptance sampling for speculative verify,
// and the on-device draft sampler that feeds it.
//
// Replaces SpeculativeDecoder::verify_drafts (src/speculative.rs:286-339),
// which compares argmaxes one position at a time with a host sync per
// position, and sample_token (src/worker.rs:267-362), which copies the row
// to the host.  Everything here stays on the device and is batched.
//
// The normaliser contract of kyro_math.h makes every decision reproducible:
// per-chunk maxima, ky_exp, exact integer (fix40) chunk masses, a fixed-order
// double combination, and integer (fix62) inverse-CDF weights.  Integer
// sums do not depend on how threads are arranged, so the parallel kernels
// below reproduce the sequential oracle bit for bit.
//
// Three launches per call:
//   accept_row_stats_kernel  one CTA per (row, 2048-entry chunk): chunk max
//                            (and argmax), e at the draft token, and the
//                            fix40 chunk mass.  Reads every logit once.
//   accept_decide_kernel     one CTA per sequence: row normalisers, the k
//                            accept tests, the accepted length, and the
//                            descriptor of the row to resample from.
//   accept_final_row_kernel  CTAs over the chunks of each sequence's final
//                            row: fix62 weights (residual or p) and chunk
//                            sums; the last CTA to finish finds the chunk
//                            holding the cut point and scans it.
//
// This file is compiled with --fmad=false; the shared arithmetic also uses
// explicit round-to-nearest intrinsics.
#include "kyro_internal.cuh"
#include "kyro_math.h"

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kChunk = KY_CHUNK;
static_assert(kChunk == kThreads * 8, "a chunk is two float4 per thread");
constexpr int kMaxChunks = 256;  // V <= 524288
constexpr int kMaxDraft = 64;
constexpr int kMaxRows = 2 * kMaxDraft + 1;

struct ChunkStat {
  float m;                 // chunk max of s = z * inv_t (or of z, greedy)
  int32_t arg;             // lowest index attaining m
  unsigned long long E;    // sum of fix40(ky_exp(s - m)) over the chunk
};

// The row a sequence (or a sampled row) draws its emitted token from.
struct FinalRow {
  int64_t p_row;    // row index into the target (or sampled) logits
  int64_t q_row;    // row index into the draft logits, -1 = sample from p
  int64_t p_stat;   // row index into the stats array
  int64_t q_stat;
  float Mp, Mq;
  double Sp, Sq;
  uint32_t odd;     // uniform numerator for the inverse CDF
  int32_t out_index;  // where the token (and its probability) goes
  int32_t skip;     // 1: token already written by the decide kernel
  int32_t _pad;
};

__host__ __device__ inline size_t align_up(size_t x) {
  return (x + 255) & ~size_t(255);
}

struct Workspace {
  ChunkStat* stats;
  float* ex;
  FinalRow* final_rows;
  unsigned long long* W;
  uint32_t* ticket;
  size_t bytes;
};

Workspace carve(void* base, int64_t stat_rows, int64_t nchunks, int64_t final_rows) {
  Workspace w;
  size_t off = 0;
  char* p = (char*)base;
  w.stats = (ChunkStat*)(p + off);
  off += align_up(sizeof(ChunkStat) * (size_t)(stat_rows * nchunks));
  w.ex = (float*)(p + off);
  off += align_up(sizeof(float) * (size_t)stat_rows);
  w.final_rows = (FinalRow*)(p + off);
  off += align_up(sizeof(FinalRow) * (size_t)final_rows);
  w.W = (unsigned long long*)(p + off);
  off += align_up(sizeof(unsigned long long) * (size_t)(final_rows * nchunks));
  w.ticket = (uint32_t*)(p + off);
  off += align_up(sizeof(uint32_t) * (size_t)final_rows);
  w.bytes = off;
  return w;
}

// ------------------------------------------------------------ device helpers

// Exclusive block-wide prefix of a u64 per thread; returns the block total
// through *total.  `sh` holds kWarps entries.
__device__ unsigned long long block_exclusive_scan_u64(unsigned long long v,
                                                       unsigned long long* sh,
                                                       unsigned long long* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    unsigned long long t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  __syncthreads();
  if (lane == 31) sh[warp] = inc;
  __syncthreads();
  unsigned long long warp_base = 0, all = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    unsigned long long s = sh[w];
    if (w < warp) warp_base += s;
    all += s;
  }
  *total = all;
  return warp_base + inc - v;
}

__device__ unsigned long long block_sum_u64(unsigned long long v, unsigned long long* sh) {
  unsigned long long t;
  block_exclusive_scan_u64(v, sh, &t);
  return t;
}

// Load the 8 logits of chunk `c` this thread owns: elements
// c*2048 + g*1024 + 4*tid + i for g in {0,1}, i in {0..3}.
template <bool VEC>
__device__ __forceinline__ void load_chunk(const float* row, int64_t V, int c, float (&v)[8],
                                           int (&idx)[8]) {
  const int64_t base = (int64_t)c * kChunk;
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const int64_t e0 = base + g * 1024 + 4 * threadIdx.x;
    if (VEC && e0 + 3 < V) {
      float4 f = __ldcs(reinterpret_cast<const float4*>(row + e0));
      v[4 * g + 0] = f.x;
      v[4 * g + 1] = f.y;
      v[4 * g + 2] = f.z;
      v[4 * g + 3] = f.w;
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) v[4 * g + i] = (e0 + i < V) ? row[e0 + i] : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) idx[4 * g + i] = (e0 + i < V) ? (int)(e0 + i) : -1;
  }
}

// -------------------------------------------------------------- kernel A

// grid (rows, nchunks).  Rows [0, B*(k+1)) are target rows (b, j); with
// draft logits present, rows [B*(k+1), B*(2k+1)) are draft rows (b, j).
// For the sampler (k_draft_tokens == nullptr) every row is a plain row.
template <bool STOCH, bool VEC>
__global__ void __launch_bounds__(kThreads)
accept_row_stats_kernel(const float* __restrict__ target, const float* __restrict__ draft,
                        const int32_t* __restrict__ draft_tokens, int B, int k, int64_t V,
                        int nchunks, float inv_t, ChunkStat* __restrict__ stats,
                        float* __restrict__ ex, uint32_t* status) {
  __shared__ float sh_m[kWarps];
  __shared__ int sh_arg[kWarps];
  __shared__ unsigned long long sh_E[kWarps];
  const int64_t row = blockIdx.x;
  const int c = blockIdx.y;
  const int64_t tgt_rows = (int64_t)B * (k + 1);
  const float* rowp;
  int x = -1;
  if (row < tgt_rows) {
    rowp = target + row * V;
    if (draft_tokens) {
      const int64_t b = row / (k + 1);
      const int j = (int)(row % (k + 1));
      if (j < k) x = draft_tokens[b * k + j];
    }
  } else {
    const int64_t r2 = row - tgt_rows;
    rowp = draft + r2 * V;
    x = draft_tokens[(r2 / k) * k + (r2 % k)];
  }

  float v[8];
  int idx[8];
  load_chunk<VEC>(rowp, V, c, v, idx);
  float best = -INFINITY;
  int best_i = 0x7fffffff;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (STOCH) v[i] = KY_FMUL(v[i], inv_t);
    if (idx[i] >= 0 && v[i] > best) {
      best = v[i];
      best_i = idx[i];
    }
  }
  kyro::dev::warp_argmax(best, best_i);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sh_m[warp] = best;
    sh_arg[warp] = best_i;
  }
  __syncthreads();
  float m = sh_m[0];
  int arg = sh_arg[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) {
    float ov = sh_m[w];
    int oi = sh_arg[w];
    if (ov > m || (ov == m && oi < arg)) {
      m = ov;
      arg = oi;
    }
  }
  unsigned long long E = 0;
  if (STOCH) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (idx[i] >= 0) {
        float e = ky_exp(KY_FSUB(v[i], m));
        E += ky_fix40(e);
        if (idx[i] == x) ex[row] = e;
      }
    }
    E = kyro::dev::warp_sum_u64(E);
    if (lane == 0) sh_E[warp] = E;
    __syncthreads();
    E = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) E += sh_E[w];
  }
  if (threadIdx.x == 0) {
    ChunkStat s;
    s.m = m;
    s.arg = arg;
    s.E = E;
    stats[row * nchunks + c] = s;
  }
  (void)status;
}

// -------------------------------------------------------------- kernel B

// Row normaliser (M, S) of one stats row, computed by one warp: chunk
// masses in parallel, then lane 0 adds them in chunk order.
__device__ void warp_row_normaliser(const ChunkStat* st, int nchunks, double* scratch, float* M_out,
                                    double* S_out) {
  const int lane = threadIdx.x & 31;
  float M = -INFINITY;
  for (int c = lane; c < nchunks; c += 32) M = fmaxf(M, st[c].m);
  M = kyro::dev::warp_max(M);
  for (int c = lane; c < nchunks; c += 32) scratch[c] = ky_chunk_mass(st[c].E, st[c].m, M);
  __syncwarp();
  if (lane == 0) {
    double S = 0.0;
    for (int c = 0; c < nchunks; ++c) S = KY_DADD(S, scratch[c]);
    *M_out = M;
    *S_out = S;
  }
  __syncwarp();
}

// one CTA per sequence
template <bool STOCH>
__global__ void __launch_bounds__(kThreads)
accept_decide_kernel(const int32_t* __restrict__ draft_tokens, int B, int k, int64_t V,
                     int nchunks, int greedy_ref, uint64_t seed, uint32_t step,
                     int64_t seq_offset, const ChunkStat* __restrict__ stats,
                     const float* __restrict__ ex, FinalRow* __restrict__ final_rows,
                     uint32_t* __restrict__ ticket, int32_t* __restrict__ out_accept_len,
                     int32_t* __restrict__ out_tokens, int32_t* __restrict__ out_num_tokens,
                     float* __restrict__ out_probs, uint32_t* status) {
  __shared__ float sh_M[kMaxRows];
  __shared__ double sh_S[kMaxRows];
  __shared__ int sh_arg[kMaxRows];
  __shared__ int sh_acc[kMaxDraft];
  __shared__ double scratch_all[kWarps][kMaxChunks];
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nrows = STOCH ? 2 * k + 1 : k + 1;  // target rows, then draft rows
  double* scratch = scratch_all[warp];
  const int64_t tgt_rows = (int64_t)B * (k + 1);
  auto stat_row = [&](int r) -> int64_t {
    return r <= k ? (int64_t)b * (k + 1) + r : tgt_rows + (int64_t)b * k + (r - (k + 1));
  };

  for (int r = warp; r < nrows; r += kWarps) {
    const ChunkStat* st = stats + stat_row(r) * nchunks;
    if (STOCH) {
      warp_row_normaliser(st, nchunks, scratch, &sh_M[r], &sh_S[r]);
    } else {
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int c = lane; c < nchunks; c += 32) {
        ChunkStat s = st[c];
        if (s.m > best || (s.m == best && s.arg < bi)) {
          best = s.m;
          bi = s.arg;
        }
      }
      kyro::dev::warp_argmax(best, bi);
      if (lane == 0) sh_arg[r] = bi == 0x7fffffff ? 0 : bi;
    }
  }
  __syncthreads();

  const uint32_t seq = (uint32_t)(seq_offset + b);
  const int32_t* x = draft_tokens + (int64_t)b * k;
  for (int j = threadIdx.x; j < k; j += kThreads) {
    const int xj = x[j];
    const bool ok = xj >= 0 && xj < V;
    if (!ok) kyro::dev::flag(status, KYRO_DEV_BAD_TOKEN);
    if (STOCH) {
      float p = 0.0f, q = 0.0f;
      if (ok) {
        const int cx = xj / kChunk;
        const int64_t pr = stat_row(j), qr = stat_row(k + 1 + j);
        p = KY_FMUL(ex[pr], ky_chunk_scale(stats[pr * nchunks + cx].m, sh_M[j], sh_S[j]));
        q = KY_FMUL(ex[qr], ky_chunk_scale(stats[qr * nchunks + cx].m, sh_M[k + 1 + j],
                                           sh_S[k + 1 + j]));
      }
      if (out_probs) {
        out_probs[((int64_t)b * k + j) * 2 + 0] = p;
        out_probs[((int64_t)b * k + j) * 2 + 1] = q;
      }
      const uint32_t odd = ky_uniform_odd(seed, seq, (uint32_t)j, KY_STREAM_ACCEPT, step);
      sh_acc[j] = ok && ky_accept(odd, p, q);
    } else {
      sh_acc[j] = ok && (sh_arg[j] == xj);
    }
  }
  __syncthreads();

  if (threadIdx.x == 0) {
    int a = k;
    for (int j = 0; j < k; ++j)
      if (!sh_acc[j]) {
        a = j;
        break;
      }
    int32_t* toks = out_tokens + (int64_t)b * (k + 1);
    for (int j = 0; j <= k; ++j) toks[j] = j < a ? x[j] : -1;
    out_accept_len[b] = a;
    FinalRow fr;
    fr.p_row = (int64_t)b * (k + 1) + a;
    fr.p_stat = stat_row(a);
    fr.out_index = b * (k + 1) + a;
    fr.odd = ky_uniform_odd(seed, seq, (uint32_t)a, KY_STREAM_RESAMPLE, step);
    fr._pad = 0;
    if (STOCH) {
      fr.skip = 0;
      fr.Mp = sh_M[a];
      fr.Sp = sh_S[a];
      if (a < k) {
        fr.q_row = (int64_t)b * k + a;
        fr.q_stat = stat_row(k + 1 + a);
        fr.Mq = sh_M[k + 1 + a];
        fr.Sq = sh_S[k + 1 + a];
      } else {
        fr.q_row = -1;
        fr.q_stat = -1;
        fr.Mq = 0.0f;
        fr.Sq = 1.0;
      }
      out_num_tokens[b] = a + 1;
    } else {
      fr.skip = 1;
      if (a == k && greedy_ref && k > 0) {
        out_num_tokens[b] = k;
      } else {
        toks[a] = sh_arg[a];
        out_num_tokens[b] = a + 1;
      }
    }
    final_rows[b] = fr;
    ticket[b] = 0;
  }
}

// Per-row descriptor for the draft sampler: one warp per row.
__global__ void __launch_bounds__(kThreads)
sample_decide_kernel(int64_t nrows, int num_pos, int nchunks, int greedy, uint64_t seed,
                     uint32_t step, int64_t seq_offset, const ChunkStat* __restrict__ stats,
                     FinalRow* __restrict__ final_rows, uint32_t* __restrict__ ticket,
                     int32_t* __restrict__ out_tokens, float* __restrict__ out_probs) {
  __shared__ double scratch_all[kWarps][kMaxChunks];
  __shared__ float shM[kWarps];
  __shared__ double shS[kWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t r = (int64_t)blockIdx.x * kWarps + warp;
  if (r >= nrows) return;
  const ChunkStat* st = stats + r * nchunks;
  FinalRow fr;
  fr.p_row = r;
  fr.p_stat = r;
  fr.q_row = -1;
  fr.q_stat = -1;
  fr.Mq = 0.0f;
  fr.Sq = 1.0;
  fr.out_index = (int32_t)r;
  fr._pad = 0;
  const int64_t b = r / num_pos;
  const int j = (int)(r % num_pos);
  fr.odd = ky_uniform_odd(seed, (uint32_t)(seq_offset + b), (uint32_t)j, KY_STREAM_DRAFT, step);
  if (greedy) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < nchunks; c += 32) {
      ChunkStat s = st[c];
      if (s.m > best || (s.m == best && s.arg < bi)) {
        best = s.m;
        bi = s.arg;
      }
    }
    kyro::dev::warp_argmax(best, bi);
    if (lane == 0) {
      out_tokens[r] = bi == 0x7fffffff ? 0 : bi;
      if (out_probs) out_probs[r] = 1.0f;
      fr.skip = 1;
      fr.Mp = 0.0f;
      fr.Sp = 1.0;
      final_rows[r] = fr;
      ticket[r] = 0;
    }
    return;
  }
  warp_row_normaliser(st, nchunks, scratch_all[warp], &shM[warp], &shS[warp]);
  if (lane == 0) {
    fr.skip = 0;
    fr.Mp = shM[warp];
    fr.Sp = shS[warp];
    final_rows[r] = fr;
    ticket[r] = 0;
  }
}

// -------------------------------------------------------------- kernel C

template <bool VEC>
__device__ __forceinline__ void final_weights(const float* prow, const float* qrow, int64_t V,
                                              int c, float inv_t, float mp, float gp, float mq,
                                              float gq, bool residual, unsigned long long (&w)[8],
                                              int (&idx)[8]) {
  float zp[8], zq[8];
  load_chunk<VEC>(prow, V, c, zp, idx);
  if (residual) {
    int idx2[8];
    load_chunk<VEC>(qrow, V, c, zq, idx2);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float p = KY_FMUL(ky_exp(KY_FSUB(KY_FMUL(zp[i], inv_t), mp)), gp);
    unsigned long long wi;
    if (residual) {
      float q = KY_FMUL(ky_exp(KY_FSUB(KY_FMUL(zq[i], inv_t), mq)), gq);
      wi = ky_residual_w(p, q);
    } else {
      wi = ky_fix62(p);
    }
    w[i] = idx[i] >= 0 ? wi : 0ull;
  }
}

// grid (nsplit, nfinal): CTA x covers chunks [x*per, (x+1)*per) of final row y.
template <bool VEC>
__global__ void __launch_bounds__(kThreads)
accept_final_row_kernel(const float* __restrict__ plogits, const float* __restrict__ qlogits,
                        int64_t V, int nchunks, int chunks_per_cta, float inv_t,
                        const ChunkStat* __restrict__ stats, const FinalRow* __restrict__ final_rows,
                        unsigned long long* __restrict__ Wbuf, uint32_t* __restrict__ ticket,
                        int32_t* __restrict__ out_tokens, float* __restrict__ out_probs) {
  __shared__ unsigned long long sh_red[kWarps];
  __shared__ unsigned long long sh_W[kMaxChunks];
  __shared__ int sh_last, sh_chunk, sh_token;
  __shared__ unsigned long long sh_T;
  __shared__ int sh_residual;
  const int64_t fi = blockIdx.y;
  const FinalRow fr = final_rows[fi];
  if (fr.skip) return;
  const float* prow = plogits + fr.p_row * V;
  const float* qrow = fr.q_row >= 0 ? qlogits + fr.q_row * V : nullptr;
  const ChunkStat* sp = stats + fr.p_stat * nchunks;
  const ChunkStat* sq = fr.q_stat >= 0 ? stats + fr.q_stat * nchunks : nullptr;
  unsigned long long* W = Wbuf + fi * nchunks;

  const int c0 = blockIdx.x * chunks_per_cta;
  const int c1 = min(nchunks, c0 + chunks_per_cta);
  const bool residual = qrow != nullptr;
  for (int c = c0; c < c1; ++c) {
    const float mp = sp[c].m, gp = ky_chunk_scale(mp, fr.Mp, fr.Sp);
    float mq = 0.0f, gq = 0.0f;
    if (residual) {
      mq = sq[c].m;
      gq = ky_chunk_scale(mq, fr.Mq, fr.Sq);
    }
    unsigned long long w[8];
    int idx[8];
    final_weights<VEC>(prow, qrow, V, c, inv_t, mp, gp, mq, gq, residual, w, idx);
    unsigned long long s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += w[i];
    s = block_sum_u64(s, sh_red);
    if (threadIdx.x == 0) W[c] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t t = atomicAdd(&ticket[fi], 1u);
    sh_last = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (!sh_last) return;
  __threadfence();

  // ---- last CTA of this row: locate the chunk, then the index
  for (int c = threadIdx.x; c < nchunks; c += kThreads) sh_W[c] = __ldcg(&W[c]);
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long tot = 0;
    for (int c = 0; c < nchunks; ++c) tot += sh_W[c];
    sh_residual = residual && tot != 0;
  }
  __syncthreads();
  if (residual && !sh_residual) {
    // residual without mass: fall back to sampling from p
    for (int c = 0; c < nchunks; ++c) {
      const float mp = sp[c].m, gp = ky_chunk_scale(mp, fr.Mp, fr.Sp);
      unsigned long long w[8];
      int idx[8];
      final_weights<VEC>(prow, nullptr, V, c, inv_t, mp, gp, 0.0f, 0.0f, false, w, idx);
      unsigned long long s = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) s += w[i];
      s = block_sum_u64(s, sh_red);
      if (threadIdx.x == 0) sh_W[c] = s;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    unsigned long long tot = 0;
    for (int c = 0; c < nchunks; ++c) tot += sh_W[c];
    int chunk = -1;
    unsigned long long T = 0;
    if (tot != 0) {
      T = ky_cdf_threshold(fr.odd, tot);
      unsigned long long cum = 0;
      for (int c = 0; c < nchunks; ++c) {
        if (cum + sh_W[c] >= T) {
          chunk = c;
          T -= cum;
          break;
        }
        cum += sh_W[c];
      }
    }
    sh_chunk = chunk;
    sh_T = T;
    sh_token = (int)V - 1;
  }
  __syncthreads();
  const int chunk = sh_chunk;
  if (chunk >= 0) {
    const bool res = sh_residual;
    const float mp = sp[chunk].m, gp = ky_chunk_scale(mp, fr.Mp, fr.Sp);
    float mq = 0.0f, gq = 0.0f;
    if (res) {
      mq = sq[chunk].m;
      gq = ky_chunk_scale(mq, fr.Mq, fr.Sq);
    }
    unsigned long long w[8];
    int idx[8];
    final_weights<VEC>(prow, qrow, V, chunk, inv_t, mp, gp, mq, gq, res, w, idx);
    const unsigned long long T = sh_T;
    // element order within the chunk: group 0 of all threads, then group 1
    unsigned long long base = 0;
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      unsigned long long s = w[4 * g] + w[4 * g + 1] + w[4 * g + 2] + w[4 * g + 3];
      unsigned long long gtot;
      unsigned long long ex = block_exclusive_scan_u64(s, sh_red, &gtot);
      unsigned long long C = base + ex;
      if (C < T && C + s >= T) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          C += w[4 * g + i];
          if (C >= T) {
            sh_token = idx[4 * g + i];
            break;
          }
        }
      }
      base += gtot;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int tok = sh_token;
    out_tokens[fr.out_index] = tok;
    if (out_probs) {
      // p(token) under the row's normaliser (draft sampler output)
      const int c = tok / kChunk;
      const float mp = sp[c].m;
      out_probs[fr.out_index] =
          KY_FMUL(ky_exp(KY_FSUB(KY_FMUL(prow[tok], inv_t), mp)), ky_chunk_scale(mp, fr.Mp, fr.Sp));
    }
    ticket[fi] = 0;
  }
}

size_t accept_ws_bytes(int64_t B, int64_t k, int64_t V, bool stoch) {
  const int64_t nchunks = (V + kChunk - 1) / kChunk;
  const int64_t stat_rows = stoch ? B * (2 * k + 1) : B * (k + 1);
  return carve(nullptr, stat_rows, nchunks, B).bytes;
}

bool use_vec(const void* a, const void* b, int64_t V) {
  return (V % 4 == 0) && ((uintptr_t)a % 16 == 0) && (b == nullptr || (uintptr_t)b % 16 == 0);
}

}  // namespace

extern "C" {

size_t kyro_spec_accept_workspace_size(const kyro_accept_params* p) {
  if (!p || p->batch < 0 || p->num_draft < 0 || p->vocab <= 0) return 0;
  const bool stoch = p->mode == KYRO_ACCEPT_STOCHASTIC && p->temperature > 0.0f;
  return accept_ws_bytes(p->batch, p->num_draft, p->vocab, stoch);
}

int kyro_spec_accept(kyro_ctx* ctx, const kyro_accept_params* p, const float* target_logits,
                     const float* draft_logits, const int32_t* draft_tokens,
                     int32_t* out_accept_len, int32_t* out_tokens, int32_t* out_num_tokens,
                     float* out_probs, void* workspace, size_t workspace_bytes) {
  KY_TRY(kyro::enter(ctx));
  KY_REQUIRE(p, "kyro_spec_accept: params is NULL");
  KY_REQUIRE(p->batch >= 0, "kyro_spec_accept: batch = %d", p->batch);
  KY_REQUIRE(p->num_draft >= 0 && p->num_draft <= kMaxDraft, "kyro_spec_accept: num_draft = %d (0..64)",
             p->num_draft);
  KY_REQUIRE(p->vocab > 0 && (int64_t)p->vocab <= (int64_t)kMaxChunks * kChunk,
             "kyro_spec_accept: vocab = %d (1..%d)", p->vocab, kMaxChunks * kChunk);
  KY_REQUIRE(p->mode >= 0 && p->mode <= 2, "kyro_spec_accept: mode = %d", p->mode);
  if (p->batch == 0) return KYRO_OK;
  const bool stoch = p->mode == KYRO_ACCEPT_STOCHASTIC && p->temperature > 0.0f;
  const int B = p->batch, k = p->num_draft;
  const int64_t V = p->vocab;
  KY_REQUIRE(target_logits, "kyro_spec_accept: target_logits is NULL");
  KY_REQUIRE(k == 0 || draft_tokens, "kyro_spec_accept: draft_tokens is NULL");
  KY_REQUIRE(!stoch || k == 0 || draft_logits,
             "kyro_spec_accept: stochastic mode needs draft_logits");
  KY_REQUIRE(out_accept_len && out_tokens && out_num_tokens,
             "kyro_spec_accept: an output pointer is NULL");
  const size_t need = accept_ws_bytes(B, k, V, stoch);
  if (workspace_bytes < need || !workspace)
    return kyro::set_error(KYRO_ERR_WORKSPACE, "kyro_spec_accept: workspace %zu < %zu bytes",
                           workspace_bytes, need);
  KY_REQUIRE((uintptr_t)workspace % 256 == 0, "kyro_spec_accept: workspace must be 256-byte aligned");

  const int nchunks = (int)((V + kChunk - 1) / kChunk);
  const int64_t stat_rows = stoch ? (int64_t)B * (2 * k + 1) : (int64_t)B * (k + 1);
  KY_REQUIRE(stat_rows < (1ll << 31), "kyro_spec_accept: too many rows");
  Workspace ws = carve(workspace, stat_rows, nchunks, B);
  const float inv_t = stoch ? ky_inv_temperature(p->temperature) : 1.0f;
  const bool vec = use_vec(target_logits, stoch ? draft_logits : nullptr, V);
  cudaStream_t st = ctx->stream;

  dim3 gridA((unsigned)stat_rows, (unsigned)nchunks);
  const int32_t* xt = k > 0 ? draft_tokens : nullptr;
  if (stoch) {
    if (vec)
      accept_row_stats_kernel<true, true><<<gridA, kThreads, 0, st>>>(
          target_logits, draft_logits, xt, B, k, V, nchunks, inv_t, ws.stats, ws.ex,
          ctx->d_status);
    else
      accept_row_stats_kernel<true, false><<<gridA, kThreads, 0, st>>>(
          target_logits, draft_logits, xt, B, k, V, nchunks, inv_t, ws.stats, ws.ex,
          ctx->d_status);
  } else {
    if (vec)
      accept_row_stats_kernel<false, true><<<gridA, kThreads, 0, st>>>(
          target_logits, nullptr, xt, B, k, V, nchunks, 1.0f, ws.stats, ws.ex, ctx->d_status);
    else
      accept_row_stats_kernel<false, false><<<gridA, kThreads, 0, st>>>(
          target_logits, nullptr, xt, B, k, V, nchunks, 1.0f, ws.stats, ws.ex, ctx->d_status);
  }
  KY_TRY(kyro::check_launch("accept_row_stats_kernel"));

  if (stoch)
    accept_decide_kernel<true><<<B, kThreads, 0, st>>>(
        draft_tokens, B, k, V, nchunks, 0, p->seed, p->step, p->seq_offset, ws.stats, ws.ex,
        ws.final_rows, ws.ticket, out_accept_len, out_tokens, out_num_tokens, out_probs,
        ctx->d_status);
  else
    accept_decide_kernel<false><<<B, kThreads, 0, st>>>(
        draft_tokens, B, k, V, nchunks, p->mode == KYRO_ACCEPT_GREEDY_REF, p->seed, p->step,
        p->seq_offset, ws.stats, ws.ex, ws.final_rows, ws.ticket, out_accept_len, out_tokens,
        out_num_tokens, nullptr, ctx->d_status);
  KY_TRY(kyro::check_launch("accept_decide_kernel"));

  if (stoch) {
    const int per = 4;
    KY_REQUIRE(B <= 65535, "kyro_spec_accept: batch %d > 65535", B);
    dim3 gridC((unsigned)((nchunks + per - 1) / per), (unsigned)B);
    if (vec)
      accept_final_row_kernel<true><<<gridC, kThreads, 0, st>>>(
          target_logits, draft_logits, V, nchunks, per, inv_t, ws.stats, ws.final_rows, ws.W,
          ws.ticket, out_tokens, nullptr);
    else
      accept_final_row_kernel<false><<<gridC, kThreads, 0, st>>>(
          target_logits, draft_logits, V, nchunks, per, inv_t, ws.stats, ws.final_rows, ws.W,
          ws.ticket, out_tokens, nullptr);
    KY_TRY(kyro::check_launch("accept_final_row_kernel"));
  }
  return KYRO_OK;
}

size_t kyro_sample_workspace_size(const kyro_sample_params* p) {
  if (!p || p->batch < 0 || p->num_pos < 0 || p->vocab <= 0) return 0;
  const int64_t rows = (int64_t)p->batch * p->num_pos;
  const int64_t nchunks = (p->vocab + kChunk - 1) / kChunk;
  return carve(nullptr, rows, nchunks, rows).bytes;
}

int kyro_sample_tokens(kyro_ctx* ctx, const kyro_sample_params* p, const float* logits,
                       int32_t* out_tokens, float* out_probs, void* workspace,
                       size_t workspace_bytes) {
  KY_TRY(kyro::enter(ctx));
  KY_REQUIRE(p, "kyro_sample_tokens: params is NULL");
  KY_REQUIRE(p->batch >= 0 && p->num_pos >= 0, "kyro_sample_tokens: batch %d num_pos %d",
             p->batch, p->num_pos);
  KY_REQUIRE(p->vocab > 0 && (int64_t)p->vocab <= (int64_t)kMaxChunks * kChunk,
             "kyro_sample_tokens: vocab = %d", p->vocab);
  const int64_t rows = (int64_t)p->batch * p->num_pos;
  if (rows == 0) return KYRO_OK;
  KY_REQUIRE(rows < (1ll << 31), "kyro_sample_tokens: too many rows");
  KY_REQUIRE(logits && out_tokens, "kyro_sample_tokens: NULL logits or out_tokens");
  const int64_t V = p->vocab;
  const int nchunks = (int)((V + kChunk - 1) / kChunk);
  const size_t need = carve(nullptr, rows, nchunks, rows).bytes;
  if (workspace_bytes < need || !workspace)
    return kyro::set_error(KYRO_ERR_WORKSPACE, "kyro_sample_tokens: workspace %zu < %zu bytes",
                           workspace_bytes, need);
  KY_REQUIRE((uintptr_t)workspace % 256 == 0, "kyro_sample_tokens: workspace must be 256-byte aligned");
  Workspace ws = carve(workspace, rows, nchunks, rows);
  const bool greedy = !(p->temperature > 0.0f);
  const float inv_t = greedy ? 1.0f : ky_inv_temperature(p->temperature);
  const bool vec = use_vec(logits, nullptr, V);
  cudaStream_t st = ctx->stream;
  // rows are plain rows: B*(k+1) with k+1 == 1 per "sequence" slot
  dim3 gridA((unsigned)rows, (unsigned)nchunks);
  if (greedy) {
    if (vec)
      accept_row_stats_kernel<false, true><<<gridA, kThreads, 0, st>>>(
          logits, nullptr, nullptr, (int)rows, 0, V, nchunks, 1.0f, ws.stats, ws.ex, ctx->d_status);
    else
      accept_row_stats_kernel<false, false><<<gridA, kThreads, 0, st>>>(
          logits, nullptr, nullptr, (int)rows, 0, V, nchunks, 1.0f, ws.stats, ws.ex, ctx->d_status);
  } else {
    if (vec)
      accept_row_stats_kernel<true, true><<<gridA, kThreads, 0, st>>>(
          logits, nullptr, nullptr, (int)rows, 0, V, nchunks, inv_t, ws.stats, ws.ex, ctx->d_status);
    else
      accept_row_stats_kernel<true, false><<<gridA, kThreads, 0, st>>>(
          logits, nullptr, nullptr, (int)rows, 0, V, nchunks, inv_t, ws.stats, ws.ex, ctx->d_status);
  }
  KY_TRY(kyro::check_launch("accept_row_stats_kernel(sample)"));
  sample_decide_kernel<<<(unsigned)((rows + kWarps - 1) / kWarps), kThreads, 0, st>>>(
      rows, p->num_pos, nchunks, greedy, p->seed, p->step, p->seq_offset, ws.stats,
      ws.final_rows, ws.ticket, out_tokens, out_probs);
  KY_TRY(kyro::check_launch("sample_decide_kernel"));
  if (!greedy) {
    const int per = 4;
    KY_REQUIRE(rows <= 65535, "kyro_sample_tokens: batch*num_pos %lld > 65535", (long long)rows);
    dim3 gridC((unsigned)((nchunks + per - 1) / per), (unsigned)rows);
    if (vec)
      accept_final_row_kernel<true><<<gridC, kThreads, 0, st>>>(
          logits, nullptr, V, nchunks, per, inv_t, ws.stats, ws.final_rows, ws.W, ws.ticket,
          out_tokens, out_probs);
    else
      accept_final_row_kernel<false><<<gridC, kThreads, 0, st>>>(
          logits, nullptr, V, nchunks, per, inv_t, ws.stats, ws.final_rows, ws.W, ws.ticket,
          out_tokens, out_probs);
    KY_TRY(kyro::check_launch("accept_final_row_kernel(sample)"));
  }
  return KYRO_OK;
}

}  // extern "C"
