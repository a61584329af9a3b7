// sampler.cu -- K2: vocab-wide acceptance sampling for speculative verify,
// and the on-device draft sampler that feeds it.
//
// Replaces SpeculativeDecoder::verify_drafts (src/speculative.rs:286-339),
// which compares argmaxes one position at a time with a host sync per
// position, and sample_token (src/worker.rs:267-362), which copies the row
// to the host.  Everything here stays on the device and is batched.
//
// The normaliser contract of kyro_math.h makes every decision reproducible:
// per-chunk maxima, ky_exp, exact integer (fix40) chunk masses, a fixed
// butterfly combination in double, and integer (fix62) inverse-CDF weights.
// Integer sums do not depend on how threads are arranged, so the parallel
// kernel reproduces the sequential oracle bit for bit.
//
// One persistent launch does the whole step.  Warps take units from an
// atomic work queue in a fixed order:
//   stats unit   one 2048-logit chunk of one row (target or draft) by one
//                warp, 64 logits per lane held in registers: chunk max (or
//                argmax), e at the draft token, fix40 chunk mass.
//   decide       run inline by the warp that finishes a sequence's last
//                stats unit: row normalisers, the k accept tests, the
//                accepted length, and the row to draw the emitted token from.
//   final unit   512 logits of that row: fix62 weights (residual or p) and
//                their sum.  The warp that finishes a row's last final unit
//                locates the sub-range holding the cut point and scans it.
// A sequence's final units are queued kDelta sequences after its stats
// units, so the final row is read again while it is still in L2, and a
// final unit waits (bounded) for its sequence's decision.  Units a waiting
// warp holds always come later in the queue than the unit it waits on, so
// the wait always ends.
//
// This file is compiled with --fmad=false; the shared arithmetic also uses
// explicit round-to-nearest intrinsics.
#include <mutex>

#include "kyro_internal.cuh"
#include "kyro_math.h"

namespace {

constexpr int kChunk = KY_CHUNK;           // logits per stats unit
constexpr int kPerLane = kChunk / 32;      // 64
constexpr int kVecPerLane = kPerLane / 4;  // 16 float4
constexpr int kSub = 512;                  // logits per final unit
constexpr int kSubVec = kSub / 128;        // 4 float4 per lane
constexpr int kSubsPerChunk = kChunk / kSub;
constexpr int kWarps = 4;                  // warps per CTA
constexpr int kThreads = kWarps * 32;
constexpr int kMaxChunks = 256;            // V <= 524288
constexpr int kMaxDraft = 64;
constexpr int kMaxRows = 2 * kMaxDraft + 1;
constexpr int kDelta = 12;                 // sequences between stats and final units
constexpr int kBatch = 2;                  // units taken per queue access

struct ChunkStat {
  float m;               // chunk max of s = z * inv_t (or of z, greedy)
  int32_t arg;           // lowest index attaining m (greedy)
  unsigned long long E;  // sum of fix40(ky_exp(s - m)) over the chunk
};

// The row a sequence (or a sampled row) draws its emitted token from.
struct FinalRow {
  int64_t p_row;      // row index into plog
  int64_t q_row;      // row index into qlog, -1 = sample from p
  int64_t p_stat;     // stats row of p
  int64_t q_stat;     // stats row of q
  float Mp, Mq;
  double Sp, Sq;
  uint32_t odd;       // uniform numerator for the inverse CDF
  int32_t out_index;  // where the token (and its probability) goes
  int32_t skip;       // 1: the decide step already wrote the token
  int32_t _pad;
};

struct Args {
  const float* plog;            // target logits (accept) or the rows to sample
  const float* qlog;            // draft logits (stochastic accept) or null
  const int32_t* draft_tokens;  // [B, k] (accept)
  int B;                        // sequences (accept) or rows (sampler)
  int k;                        // drafts per sequence; 0 for the sampler
  int R;                        // stats rows per sequence
  int64_t V;
  int nchunks, nsub;
  float inv_t;
  int stoch;                    // softmax statistics (else argmax only)
  int greedy_ref;
  int sample;                   // draft-sampler call
  int pos_div;                  // sampler: Philox seq = r / pos_div, pos = r % pos_div
  uint64_t seed;
  uint32_t step;
  int64_t seq_offset;
  int32_t* out_accept_len;
  int32_t* out_tokens;
  int32_t* out_num_tokens;
  float* out_probs;             // accept: [B,k,2] (p,q); sampler: [rows]
  ChunkStat* stats;
  float* ex;
  FinalRow* final_rows;
  unsigned long long* W;
  uint32_t* cnt_a;
  uint32_t* cnt_c;
  uint32_t* ready;
  unsigned long long* queue;
  int ua, uc;                   // stats units and final units per sequence
  long long total;
  uint32_t* status;
};

__host__ __device__ inline size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }

// Workspace: counters first (zeroed before every launch), then the rest.
struct Workspace {
  unsigned long long* queue;
  uint32_t* cnt_a;
  uint32_t* cnt_c;
  uint32_t* ready;
  size_t counter_bytes;
  ChunkStat* stats;
  float* ex;
  FinalRow* final_rows;
  unsigned long long* W;
  size_t bytes;
};

Workspace carve(void* base, int64_t B, int64_t R, int64_t nchunks, int64_t nsub) {
  Workspace w;
  char* p = (char*)base;
  size_t off = 0;
  w.queue = (unsigned long long*)(p + off);
  off += 256;
  w.cnt_a = (uint32_t*)(p + off);
  off += align_up(4 * (size_t)B);
  w.cnt_c = (uint32_t*)(p + off);
  off += align_up(4 * (size_t)B);
  w.ready = (uint32_t*)(p + off);
  off += align_up(4 * (size_t)B);
  w.counter_bytes = off;
  w.stats = (ChunkStat*)(p + off);
  off += align_up(sizeof(ChunkStat) * (size_t)(B * R * nchunks));
  w.ex = (float*)(p + off);
  off += align_up(sizeof(float) * (size_t)(B * R));
  w.final_rows = (FinalRow*)(p + off);
  off += align_up(sizeof(FinalRow) * (size_t)B);
  w.W = (unsigned long long*)(p + off);
  off += align_up(sizeof(unsigned long long) * (size_t)(B * nsub));
  w.bytes = off;
  return w;
}

// ------------------------------------------------------------ warp helpers

__device__ __forceinline__ unsigned long long warp_sum(unsigned long long v) {
  return kyro::dev::warp_sum_u64(v);
}

__device__ __forceinline__ double warp_butterfly(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = KY_DADD(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// inclusive warp scan of a u64
__device__ __forceinline__ unsigned long long warp_inclusive(unsigned long long v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    unsigned long long t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// The 64 logits of chunk c this lane owns: float4 i (0..15) covers elements
// c*2048 + (i*32 + lane)*4 + 0..3.  Entries beyond V read as -inf.
template <bool VEC>
__device__ __forceinline__ void load_chunk(const float* __restrict__ row, int64_t V, int c,
                                           float (&v)[kPerLane]) {
  const int lane = threadIdx.x & 31;
  const int64_t base = (int64_t)c * kChunk;
  if (VEC && base + kChunk <= V) {
    // a whole chunk: no bound checks
    const float4* p4 = reinterpret_cast<const float4*>(row + base) + lane;
#pragma unroll
    for (int i = 0; i < kVecPerLane; ++i) {
      const float4 f = __ldcs(p4 + i * 32);
      v[4 * i + 0] = f.x;
      v[4 * i + 1] = f.y;
      v[4 * i + 2] = f.z;
      v[4 * i + 3] = f.w;
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < kVecPerLane; ++i) {
    const int64_t e0 = base + (i * 32 + lane) * 4;
    if (VEC) {
      float4 f = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      if (e0 < V) f = __ldcs(reinterpret_cast<const float4*>(row + e0));
      v[4 * i + 0] = f.x;
      v[4 * i + 1] = f.y;
      v[4 * i + 2] = f.z;
      v[4 * i + 3] = f.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[4 * i + j] = (e0 + j < V) ? __ldcs(row + e0 + j) : -INFINITY;
    }
  }
}

// 16 logits of final unit `sub`: float4 i (0..3) covers elements
// sub*512 + (i*32 + lane)*4 + 0..3.
template <bool VEC>
__device__ __forceinline__ void load_sub(const float* __restrict__ row, int64_t V, int sub,
                                         float (&v)[kSubVec * 4]) {
  const int lane = threadIdx.x & 31;
  const int64_t base = (int64_t)sub * kSub;
#pragma unroll
  for (int i = 0; i < kSubVec; ++i) {
    const int64_t e0 = base + (i * 32 + lane) * 4;
    if (VEC) {
      float4 f = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      if (e0 < V) f = __ldcg(reinterpret_cast<const float4*>(row + e0));
      v[4 * i + 0] = f.x;
      v[4 * i + 1] = f.y;
      v[4 * i + 2] = f.z;
      v[4 * i + 3] = f.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[4 * i + j] = (e0 + j < V) ? __ldcg(row + e0 + j) : -INFINITY;
    }
  }
}

// Map queue position u to (kind, sequence, index within the sequence).
// Slot s holds the stats units of sequence s (s < B), then the final units
// of sequence s - kDelta (s >= kDelta).  off(s) = ua*min(s,B) + uc*max(0,s-kDelta).
__device__ __forceinline__ long long slot_off(const Args& a, int s) {
  return (long long)a.ua * min(s, a.B) + (long long)a.uc * max(0, s - kDelta);
}

__device__ __forceinline__ void unit_of(const Args& a, long long u, bool& is_stats, int& seq,
                                        int& local) {
  int lo = 0, hi = a.B + kDelta - 1;  // first slot s with off(s+1) > u
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (slot_off(a, mid + 1) > u)
      hi = mid;
    else
      lo = mid + 1;
  }
  const long long rem = u - slot_off(a, lo);
  if (lo < a.B && rem < a.ua) {
    is_stats = true;
    seq = lo;
    local = (int)rem;
  } else {
    is_stats = false;
    seq = lo - kDelta;
    local = (int)(rem - (lo < a.B ? a.ua : 0));
  }
}

__device__ __forceinline__ const float* stats_row_ptr(const Args& a, int b, int r) {
  if (r <= a.k) return a.plog + ((int64_t)b * (a.k + 1) + r) * a.V;
  return a.qlog + ((int64_t)b * a.k + (r - a.k - 1)) * a.V;
}

__device__ __forceinline__ int draft_token_of_row(const Args& a, int b, int r) {
  if (a.sample) return -1;
  if (r < a.k) return a.draft_tokens[(int64_t)b * a.k + r];
  if (r > a.k) return a.draft_tokens[(int64_t)b * a.k + (r - a.k - 1)];
  return -1;
}

// ------------------------------------------------------------ decide step

// Runs in one warp once every stats unit of sequence b is done.
__device__ void decide(const Args& a, int b, float* sM, double* sS, int* sArg) {
  const int lane = threadIdx.x & 31;
  const int R = a.R;
  for (int r = 0; r < R; ++r) {
    const ChunkStat* st = a.stats + ((int64_t)b * R + r) * a.nchunks;
    if (a.stoch) {
      float M = -INFINITY;
      for (int c = lane; c < a.nchunks; c += 32) M = fmaxf(M, __ldcg(&st[c].m));
      M = kyro::dev::warp_max(M);
      double t = 0.0;
      for (int c = lane; c < a.nchunks; c += 32)
        t = KY_DADD(t, ky_chunk_mass(__ldcg(&st[c].E), __ldcg(&st[c].m), M));
      const double S = warp_butterfly(t);
      if (lane == 0) {
        sM[r] = M;
        sS[r] = S;
      }
    } else {
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int c = lane; c < a.nchunks; c += 32) {
        const float m = __ldcg(&st[c].m);
        const int ai = __ldcg(&st[c].arg);
        if (m > best || (m == best && ai < bi)) {
          best = m;
          bi = ai;
        }
      }
      kyro::dev::warp_argmax(best, bi);
      if (lane == 0) sArg[r] = bi == 0x7fffffff ? 0 : bi;
    }
  }
  __syncwarp();

  const int k = a.k;
  FinalRow fr;
  fr._pad = 0;
  if (a.sample) {
    // one row per "sequence": the draft sampler
    const int64_t seq = a.seq_offset + b / a.pos_div;
    const int pos = b % a.pos_div;
    if (lane == 0) {
      fr.p_row = b;
      fr.p_stat = b;
      fr.q_row = -1;
      fr.q_stat = -1;
      fr.Mq = 0.0f;
      fr.Sq = 1.0;
      fr.out_index = b;
      fr.odd = ky_uniform_odd(a.seed, (uint32_t)seq, (uint32_t)pos, KY_STREAM_DRAFT, a.step);
      if (a.stoch) {
        fr.skip = 0;
        fr.Mp = sM[0];
        fr.Sp = sS[0];
      } else {
        fr.skip = 1;
        fr.Mp = 0.0f;
        fr.Sp = 1.0;
        a.out_tokens[b] = sArg[0];
        if (a.out_probs) a.out_probs[b] = 1.0f;
      }
      a.final_rows[b] = fr;
    }
  } else {
    const uint32_t seq = (uint32_t)(a.seq_offset + b);
    const int32_t* x = a.draft_tokens + (int64_t)b * k;
    int first_reject = k;
    for (int j0 = 0; j0 < k; j0 += 32) {
      const int j = j0 + lane;
      bool acc = true;
      if (j < k) {
        const int xj = x[j];
        const bool ok = xj >= 0 && xj < a.V;
        if (!ok) kyro::dev::flag(a.status, KYRO_DEV_BAD_TOKEN);
        if (a.stoch) {
          float p = 0.0f, q = 0.0f;
          if (ok) {
            const int cx = xj / kChunk;
            const int64_t pr = (int64_t)b * a.R + j, qr = (int64_t)b * a.R + k + 1 + j;
            p = KY_FMUL(__ldcg(&a.ex[pr]),
                        ky_chunk_scale(__ldcg(&a.stats[pr * a.nchunks + cx].m), sM[j], sS[j]));
            q = KY_FMUL(__ldcg(&a.ex[qr]),
                        ky_chunk_scale(__ldcg(&a.stats[qr * a.nchunks + cx].m), sM[k + 1 + j],
                                       sS[k + 1 + j]));
          }
          if (a.out_probs) {
            a.out_probs[((int64_t)b * k + j) * 2 + 0] = p;
            a.out_probs[((int64_t)b * k + j) * 2 + 1] = q;
          }
          const uint32_t odd = ky_uniform_odd(a.seed, seq, (uint32_t)j, KY_STREAM_ACCEPT, a.step);
          acc = ok && ky_accept(odd, p, q);
        } else {
          acc = ok && sArg[j] == xj;
        }
      }
      const unsigned rej = __ballot_sync(0xffffffffu, !acc);
      if (first_reject == k && rej) first_reject = j0 + __ffs(rej) - 1;
    }
    const int aa = first_reject;
    if (lane == 0) {
      int32_t* toks = a.out_tokens + (int64_t)b * (k + 1);
      for (int j = 0; j <= k; ++j) toks[j] = j < aa ? x[j] : -1;
      a.out_accept_len[b] = aa;
      fr.p_row = (int64_t)b * (k + 1) + aa;
      fr.p_stat = (int64_t)b * a.R + aa;
      fr.out_index = b * (k + 1) + aa;
      fr.odd = ky_uniform_odd(a.seed, seq, (uint32_t)aa, KY_STREAM_RESAMPLE, a.step);
      if (a.stoch) {
        fr.skip = 0;
        fr.Mp = sM[aa];
        fr.Sp = sS[aa];
        if (aa < k) {
          fr.q_row = (int64_t)b * k + aa;
          fr.q_stat = (int64_t)b * a.R + k + 1 + aa;
          fr.Mq = sM[k + 1 + aa];
          fr.Sq = sS[k + 1 + aa];
        } else {
          fr.q_row = -1;
          fr.q_stat = -1;
          fr.Mq = 0.0f;
          fr.Sq = 1.0;
        }
        a.out_num_tokens[b] = aa + 1;
      } else {
        fr.skip = 1;
        fr.q_row = fr.q_stat = -1;
        fr.Mp = fr.Mq = 0.0f;
        fr.Sp = fr.Sq = 1.0;
        if (aa == k && a.greedy_ref && k > 0) {
          a.out_num_tokens[b] = k;
        } else {
          toks[aa] = sArg[aa];
          a.out_num_tokens[b] = aa + 1;
        }
      }
      a.final_rows[b] = fr;
    }
  }
  if (lane == 0) {
    __threadfence();
    atomicExch(&a.ready[b], 1u);
  }
  __syncwarp();
}

// ------------------------------------------------------------ units

template <bool VEC, bool STOCH>
__device__ void stats_unit(const Args& a, int b, int local, float (&v)[kPerLane], float* sM,
                           double* sS, int* sArg) {
  const int lane = threadIdx.x & 31;
  const int r = local / a.nchunks, c = local % a.nchunks;
  const int64_t srow = (int64_t)b * a.R + r;
  float m = -INFINITY;
  int arg = 0x7fffffff;
  if (STOCH) {
    if (a.inv_t != 1.0f) {
#pragma unroll
      for (int i = 0; i < kPerLane; ++i) v[i] = KY_FMUL(v[i], a.inv_t);
    }
    // independent partial maxima and sums: max and integer addition give the
    // same result in any order, and short chains keep the pipes busy
    float m8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) m8[j] = v[j];
#pragma unroll
    for (int i = 8; i < kPerLane; ++i) m8[i & 7] = fmaxf(m8[i & 7], v[i]);
    m = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
              fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
    m = kyro::dev::warp_max(m);
    unsigned long long e4[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) e4[i & 3] += ky_fix40_exp(KY_FSUB(v[i], m));
    unsigned long long E = (e4[0] + e4[1]) + (e4[2] + e4[3]);
    E = warp_sum(E);
    if (lane == 0) {
      ChunkStat s;
      s.m = m;
      s.arg = 0;
      s.E = E;
      a.stats[srow * a.nchunks + c] = s;
      const int x = draft_token_of_row(a, b, r);
      if (x >= (int64_t)c * kChunk && x < (int64_t)(c + 1) * kChunk && x < a.V) {
        const float* rowp = stats_row_ptr(a, b, r);
        a.ex[srow] = ky_exp(KY_FSUB(KY_FMUL(__ldg(rowp + x), a.inv_t), m));
      }
    }
  } else {
    const int64_t base = (int64_t)c * kChunk;
#pragma unroll
    for (int i = 0; i < kVecPerLane; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (v[4 * i + j] > m) {
          m = v[4 * i + j];
          arg = (int)(base + (i * 32 + lane) * 4 + j);
        }
    kyro::dev::warp_argmax(m, arg);
    if (lane == 0) {
      ChunkStat s;
      s.m = m;
      s.arg = arg;
      s.E = 0;
      a.stats[srow * a.nchunks + c] = s;
    }
  }
  // the warp that completes the sequence's last stats unit decides it
  uint32_t last = 0;
  if (lane == 0) {
    __threadfence();
    last = atomicAdd(&a.cnt_a[b], 1u) == (uint32_t)(a.ua - 1);
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (last) {
    __threadfence();
    decide(a, b, sM, sS, sArg);
  }
}

// fix62 weights of 16 logits of one final unit
template <bool VEC>
__device__ __forceinline__ void final_weights(const Args& a, const FinalRow& fr, bool residual,
                                              int sub, unsigned long long (&w)[kSubVec * 4]) {
  const float* prow = a.plog + fr.p_row * a.V;
  const int c = sub / kSubsPerChunk;
  const ChunkStat* sp = a.stats + fr.p_stat * a.nchunks;
  const float mp = __ldcg(&sp[c].m);
  const float gp62 = ky_scale62(ky_chunk_scale(mp, fr.Mp, fr.Sp));
  float zp[kSubVec * 4];
  load_sub<VEC>(prow, a.V, sub, zp);
  if (a.inv_t != 1.0f) {
#pragma unroll
    for (int i = 0; i < kSubVec * 4; ++i) zp[i] = KY_FMUL(zp[i], a.inv_t);
  }
  if (residual) {
    const float* qrow = a.qlog + fr.q_row * a.V;
    const ChunkStat* sq = a.stats + fr.q_stat * a.nchunks;
    const float mq = __ldcg(&sq[c].m);
    const float gq62 = ky_scale62(ky_chunk_scale(mq, fr.Mq, fr.Sq));
    float zq[kSubVec * 4];
    load_sub<VEC>(qrow, a.V, sub, zq);
    if (a.inv_t != 1.0f) {
#pragma unroll
      for (int i = 0; i < kSubVec * 4; ++i) zq[i] = KY_FMUL(zq[i], a.inv_t);
    }
#pragma unroll
    for (int i = 0; i < kSubVec * 4; ++i)
      w[i] = ky_weight_residual(ky_exp(KY_FSUB(zp[i], mp)), gp62, ky_exp(KY_FSUB(zq[i], mq)),
                                gq62);
  } else {
#pragma unroll
    for (int i = 0; i < kSubVec * 4; ++i) w[i] = ky_weight_p(ky_exp(KY_FSUB(zp[i], mp)), gp62);
  }
}

// Locate the cut point of a final row once all its unit sums are in W.
template <bool VEC>
__device__ void final_search(const Args& a, int b, const FinalRow& fr) {
  const int lane = threadIdx.x & 31;
  unsigned long long* W = a.W + (int64_t)b * a.nsub;
  bool residual = fr.q_row >= 0;
  unsigned long long tot = 0;
  for (int s = lane; s < a.nsub; s += 32) tot += __ldcg(&W[s]);
  tot = warp_sum(tot);
  if (residual && tot == 0) {
    // the residual has no mass: sample from p instead
    residual = false;
    for (int s = 0; s < a.nsub; ++s) {
      unsigned long long w[kSubVec * 4];
      final_weights<VEC>(a, fr, false, s, w);
      unsigned long long t = 0;
#pragma unroll
      for (int i = 0; i < kSubVec * 4; ++i) t += w[i];
      t = warp_sum(t);
      if (lane == 0) W[s] = t;
    }
    __syncwarp();
    __threadfence_block();
    tot = 0;
    for (int s = lane; s < a.nsub; s += 32) tot += __ldcg(&W[s]);
    tot = warp_sum(tot);
  }
  int token = (int)a.V - 1;
  if (tot != 0) {
    unsigned long long T = ky_cdf_threshold(fr.odd, tot);
    // find the unit whose inclusive prefix first reaches T
    int sub = -1;
    unsigned long long base = 0;
    for (int s0 = 0; s0 < a.nsub && sub < 0; s0 += 32) {
      const unsigned long long ws = (s0 + lane < a.nsub) ? __ldcg(&W[s0 + lane]) : 0ull;
      const unsigned long long inc = base + warp_inclusive(ws);
      const unsigned hit = __ballot_sync(0xffffffffu, inc >= T && s0 + lane < a.nsub);
      if (hit) {
        const int l = __ffs(hit) - 1;
        sub = s0 + l;
        const unsigned long long before = __shfl_sync(0xffffffffu, inc - ws, l);
        T -= before;
      } else {
        base = __shfl_sync(0xffffffffu, inc, 31);
      }
    }
    if (sub >= 0) {
      unsigned long long w[kSubVec * 4];
      final_weights<VEC>(a, fr, residual, sub, w);
      unsigned long long cbase = 0;
      int found = -1;
#pragma unroll
      for (int i = 0; i < kSubVec; ++i) {
        const unsigned long long s4 = w[4 * i] + w[4 * i + 1] + w[4 * i + 2] + w[4 * i + 3];
        const unsigned long long inc = warp_inclusive(s4);
        unsigned long long C = cbase + inc - s4;
        int mine = -1;
        if (C < T && C + s4 >= T) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            C += w[4 * i + j];
            if (mine < 0 && C >= T) mine = j;
          }
        }
        const unsigned hit = __ballot_sync(0xffffffffu, mine >= 0);
        if (found < 0 && hit) {
          const int l = __ffs(hit) - 1;
          const int jj = __shfl_sync(0xffffffffu, mine, l);
          found = sub * kSub + (i * 32 + l) * 4 + jj;
        }
        cbase += __shfl_sync(0xffffffffu, inc, 31);
      }
      if (found >= 0) token = found;
    }
  }
  if (lane == 0) {
    a.out_tokens[fr.out_index] = token;
    if (a.sample && a.out_probs) {
      const int c = token / kChunk;
      const float mp = __ldcg(&a.stats[fr.p_stat * a.nchunks + c].m);
      a.out_probs[fr.out_index] =
          KY_FMUL(ky_exp(KY_FSUB(KY_FMUL(__ldg(a.plog + fr.p_row * a.V + token), a.inv_t), mp)),
                  ky_chunk_scale(mp, fr.Mp, fr.Sp));
    }
  }
}

template <bool VEC>
__device__ void final_unit(const Args& a, int b, int sub) {
  const int lane = threadIdx.x & 31;
  // wait (bounded) until the decide step of sequence b has published
  uint32_t ok = 1;
  if (lane == 0) {
    volatile uint32_t* flag = a.ready + b;
    if (*flag == 0) {
      const long long t0 = clock64();
      while (*flag == 0) {
        __nanosleep(200);
        if (clock64() - t0 > kyro::dev::kWaitBudgetCycles) {
          ok = 0;
          break;
        }
      }
    }
    __threadfence();
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (!ok) {
    if (lane == 0) kyro::dev::flag(a.status, KYRO_DEV_WAIT_TIMEOUT);
    return;
  }
  FinalRow fr;
  {
    const FinalRow* src = a.final_rows + b;
    fr.p_row = __ldcg(&src->p_row);
    fr.q_row = __ldcg(&src->q_row);
    fr.p_stat = __ldcg(&src->p_stat);
    fr.q_stat = __ldcg(&src->q_stat);
    fr.Mp = __ldcg(&src->Mp);
    fr.Mq = __ldcg(&src->Mq);
    fr.Sp = __ldcg(&src->Sp);
    fr.Sq = __ldcg(&src->Sq);
    fr.odd = __ldcg(&src->odd);
    fr.out_index = __ldcg(&src->out_index);
    fr.skip = __ldcg(&src->skip);
  }
  if (fr.skip) return;
  unsigned long long w[kSubVec * 4];
  final_weights<VEC>(a, fr, fr.q_row >= 0, sub, w);
  unsigned long long t = 0;
#pragma unroll
  for (int i = 0; i < kSubVec * 4; ++i) t += w[i];
  t = warp_sum(t);
  uint32_t last = 0;
  if (lane == 0) {
    a.W[(int64_t)b * a.nsub + sub] = t;
    __threadfence();
    last = atomicAdd(&a.cnt_c[b], 1u) == (uint32_t)(a.uc - 1);
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (last) {
    __threadfence();
    final_search<VEC>(a, b, fr);
  }
}

// ------------------------------------------------------------ the kernel

struct UnitCursor {
  long long next, end;
};

__device__ __forceinline__ long long take_unit(const Args& a, UnitCursor& cur) {
  const int lane = threadIdx.x & 31;
  if (cur.next >= cur.end) {
    long long g = 0;
    if (lane == 0) g = (long long)atomicAdd(a.queue, (unsigned long long)kBatch);
    g = __shfl_sync(0xffffffffu, g, 0);
    cur.next = g;
    cur.end = g + kBatch;
  }
  return cur.next++;
}

template <bool VEC>
__device__ __forceinline__ void prefetch(const Args& a, long long u, float (&buf)[kPerLane]) {
  if (u >= a.total) return;
  bool is_stats;
  int seq, local;
  unit_of(a, u, is_stats, seq, local);
  if (!is_stats) return;
  const int r = local / a.nchunks, c = local % a.nchunks;
  load_chunk<VEC>(stats_row_ptr(a, seq, r), a.V, c, buf);
}

template <bool VEC, bool STOCH>
__device__ __forceinline__ void run_unit(const Args& a, long long u, float (&buf)[kPerLane],
                                         float* sM, double* sS, int* sArg) {
  bool is_stats;
  int seq, local;
  unit_of(a, u, is_stats, seq, local);
  if (is_stats)
    stats_unit<VEC, STOCH>(a, seq, local, buf, sM, sS, sArg);
  else
    final_unit<VEC>(a, seq, local);
}

template <bool VEC, bool STOCH>
__global__ void __launch_bounds__(kThreads, 3) accept_fused_kernel(Args a) {
  __shared__ float sM_all[kWarps][kMaxRows];
  __shared__ double sS_all[kWarps][kMaxRows];
  __shared__ int sArg_all[kWarps][kMaxRows];
  const int warp = threadIdx.x >> 5;
  float* sM = sM_all[warp];
  double* sS = sS_all[warp];
  int* sArg = sArg_all[warp];
  UnitCursor cur{0, 0};
  float buf[kPerLane];
  for (long long u = take_unit(a, cur); u < a.total; u = take_unit(a, cur)) {
    prefetch<VEC>(a, u, buf);
    run_unit<VEC, STOCH>(a, u, buf, sM, sS, sArg);
  }
}

// ------------------------------------------------------------ host side

bool use_vec(const void* a, const void* b, int64_t V) {
  return (V % 4 == 0) && ((uintptr_t)a % 16 == 0) && (b == nullptr || (uintptr_t)b % 16 == 0);
}

template <bool VEC, bool STOCH>
int resident_ctas(int num_sms) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, accept_fused_kernel<VEC, STOCH>,
                                                    kThreads, 0) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  return num_sms * per_sm;
}

int launch(kyro_ctx* ctx, Args& a, const Workspace& ws, bool vec) {
  cudaStream_t st = ctx->stream;
  // the queue, the per-sequence counters and the ready flags start at zero
  cudaError_t err = cudaMemsetAsync(ws.queue, 0, ws.counter_bytes, st);
  if (err != cudaSuccess) return kyro::cuda_error(err, "cudaMemsetAsync(sampler counters)");
  int resident;
  if (vec && a.stoch)
    resident = resident_ctas<true, true>(ctx->num_sms);
  else if (vec)
    resident = resident_ctas<true, false>(ctx->num_sms);
  else if (a.stoch)
    resident = resident_ctas<false, true>(ctx->num_sms);
  else
    resident = resident_ctas<false, false>(ctx->num_sms);
  const long long useful = (a.total + kWarps * kBatch - 1) / (kWarps * kBatch);
  const int grid = (int)(useful < resident ? useful : resident);
  if (vec && a.stoch)
    accept_fused_kernel<true, true><<<grid, kThreads, 0, st>>>(a);
  else if (vec)
    accept_fused_kernel<true, false><<<grid, kThreads, 0, st>>>(a);
  else if (a.stoch)
    accept_fused_kernel<false, true><<<grid, kThreads, 0, st>>>(a);
  else
    accept_fused_kernel<false, false><<<grid, kThreads, 0, st>>>(a);
  return kyro::check_launch("accept_fused_kernel");
}

void fill_workspace_args(Args& a, const Workspace& ws) {
  a.stats = ws.stats;
  a.ex = ws.ex;
  a.final_rows = ws.final_rows;
  a.W = ws.W;
  a.cnt_a = ws.cnt_a;
  a.cnt_c = ws.cnt_c;
  a.ready = ws.ready;
  a.queue = ws.queue;
}

}  // namespace

extern "C" {

size_t kyro_spec_accept_workspace_size(const kyro_accept_params* p) {
  if (!p || p->batch < 0 || p->num_draft < 0 || p->vocab <= 0) return 0;
  const bool stoch = p->mode == KYRO_ACCEPT_STOCHASTIC && p->temperature > 0.0f;
  const int64_t R = stoch ? 2 * (int64_t)p->num_draft + 1 : (int64_t)p->num_draft + 1;
  const int64_t nchunks = (p->vocab + kChunk - 1) / kChunk;
  const int64_t nsub = (p->vocab + kSub - 1) / kSub;
  return carve(nullptr, p->batch, R, nchunks, nsub).bytes;
}

int kyro_spec_accept(kyro_ctx* ctx, const kyro_accept_params* p, const float* target_logits,
                     const float* draft_logits, const int32_t* draft_tokens,
                     int32_t* out_accept_len, int32_t* out_tokens, int32_t* out_num_tokens,
                     float* out_probs, void* workspace, size_t workspace_bytes) {
  KY_TRY(kyro::enter(ctx));
  KY_REQUIRE(p, "kyro_spec_accept: params is NULL");
  KY_REQUIRE(p->batch >= 0, "kyro_spec_accept: batch = %d", p->batch);
  KY_REQUIRE(p->num_draft >= 0 && p->num_draft <= kMaxDraft,
             "kyro_spec_accept: num_draft = %d (0..%d)", p->num_draft, kMaxDraft);
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
  const int R = stoch ? 2 * k + 1 : k + 1;
  const int nchunks = (int)((V + kChunk - 1) / kChunk);
  const int nsub = (int)((V + kSub - 1) / kSub);
  KY_REQUIRE((int64_t)B * R * nchunks < (1ll << 40), "kyro_spec_accept: batch too large");
  const size_t need = carve(nullptr, B, R, nchunks, nsub).bytes;
  if (workspace_bytes < need || !workspace)
    return kyro::set_error(KYRO_ERR_WORKSPACE, "kyro_spec_accept: workspace %zu < %zu bytes",
                           workspace_bytes, need);
  KY_REQUIRE((uintptr_t)workspace % 256 == 0,
             "kyro_spec_accept: workspace must be 256-byte aligned");
  Workspace ws = carve(workspace, B, R, nchunks, nsub);
  Args a = {};
  a.plog = target_logits;
  a.qlog = stoch ? draft_logits : nullptr;
  a.draft_tokens = draft_tokens;
  a.B = B;
  a.k = k;
  a.R = R;
  a.V = V;
  a.nchunks = nchunks;
  a.nsub = nsub;
  a.inv_t = stoch ? ky_inv_temperature(p->temperature) : 1.0f;
  a.stoch = stoch;
  a.greedy_ref = p->mode == KYRO_ACCEPT_GREEDY_REF;
  a.sample = 0;
  a.pos_div = 1;
  a.seed = p->seed;
  a.step = p->step;
  a.seq_offset = p->seq_offset;
  a.out_accept_len = out_accept_len;
  a.out_tokens = out_tokens;
  a.out_num_tokens = out_num_tokens;
  a.out_probs = stoch ? out_probs : nullptr;
  fill_workspace_args(a, ws);
  a.ua = R * nchunks;
  a.uc = stoch ? nsub : 0;
  a.total = (long long)B * (a.ua + a.uc);
  a.status = ctx->d_status;
  return launch(ctx, a, ws, use_vec(target_logits, a.qlog, V));
}

size_t kyro_sample_workspace_size(const kyro_sample_params* p) {
  if (!p || p->batch < 0 || p->num_pos < 0 || p->vocab <= 0) return 0;
  const int64_t rows = (int64_t)p->batch * p->num_pos;
  const int64_t nchunks = (p->vocab + kChunk - 1) / kChunk;
  const int64_t nsub = (p->vocab + kSub - 1) / kSub;
  return carve(nullptr, rows, 1, nchunks, nsub).bytes;
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
  KY_REQUIRE(rows < (1ll << 30), "kyro_sample_tokens: too many rows");
  KY_REQUIRE(logits && out_tokens, "kyro_sample_tokens: NULL logits or out_tokens");
  const int64_t V = p->vocab;
  const int nchunks = (int)((V + kChunk - 1) / kChunk);
  const int nsub = (int)((V + kSub - 1) / kSub);
  const size_t need = carve(nullptr, rows, 1, nchunks, nsub).bytes;
  if (workspace_bytes < need || !workspace)
    return kyro::set_error(KYRO_ERR_WORKSPACE, "kyro_sample_tokens: workspace %zu < %zu bytes",
                           workspace_bytes, need);
  KY_REQUIRE((uintptr_t)workspace % 256 == 0,
             "kyro_sample_tokens: workspace must be 256-byte aligned");
  Workspace ws = carve(workspace, rows, 1, nchunks, nsub);
  const bool stoch = p->temperature > 0.0f;
  Args a = {};
  a.plog = logits;
  a.qlog = nullptr;
  a.draft_tokens = nullptr;
  a.B = (int)rows;
  a.k = 0;
  a.R = 1;
  a.V = V;
  a.nchunks = nchunks;
  a.nsub = nsub;
  a.inv_t = stoch ? ky_inv_temperature(p->temperature) : 1.0f;
  a.stoch = stoch;
  a.greedy_ref = 0;
  a.sample = 1;
  a.pos_div = p->num_pos;
  a.seed = p->seed;
  a.step = p->step;
  a.seq_offset = p->seq_offset;
  a.out_tokens = out_tokens;
  a.out_probs = out_probs;
  fill_workspace_args(a, ws);
  a.ua = nchunks;
  a.uc = stoch ? nsub : 0;
  a.total = rows * (long long)(a.ua + a.uc);
  a.status = ctx->d_status;
  return launch(ctx, a, ws, use_vec(logits, nullptr, V));
}

}  // extern "C"

// ------------------------------------------------------------ no-allocation entry point
//
// kyro_spec_accept_static serves callers that cannot allocate device memory
// and so cannot pass a workspace.  Its scratch is this file-scope array,
// present on every device that loads the library until the process exits.
// In host code the array's name is only a stand-in, so the device address
// is looked up once per device with cudaGetSymbolAddress while that device
// is current, and that address is what the kernel receives.

namespace {

static __device__ __align__(256) unsigned char g_accept_static_scratch[KYRO_ACCEPT_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_ptr[kMaxDevices] = {};

int static_scratch(int device, void** out) {
  if (device < 0 || device >= kMaxDevices)
    return kyro::set_error(KYRO_ERR_UNSUPPORTED, "kyro_spec_accept_static: device %d", device);
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_ptr[device]) {
    void* p = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&p, g_accept_static_scratch);
    if (err != cudaSuccess)
      return kyro::cuda_error(err, "cudaGetSymbolAddress(static accept scratch)");
    g_static_ptr[device] = p;
  }
  *out = g_static_ptr[device];
  return KYRO_OK;
}

}  // namespace

extern "C" int kyro_spec_accept_static(kyro_ctx* ctx, const kyro_accept_params* p,
                                       const float* target_logits, const float* draft_logits,
                                       const int32_t* draft_tokens, int32_t* out_accept_len,
                                       int32_t* out_tokens, int32_t* out_num_tokens,
                                       float* out_probs) {
  KY_TRY(kyro::enter(ctx));
  KY_REQUIRE(p, "kyro_spec_accept_static: params is NULL");
  const size_t need = kyro_spec_accept_workspace_size(p);
  if (need > KYRO_ACCEPT_STATIC_SCRATCH_BYTES)
    return kyro::set_error(KYRO_ERR_WORKSPACE,
                           "kyro_spec_accept_static: this batch needs %zu bytes of scratch; the "
                           "static scratch holds %u bytes (use kyro_spec_accept with a workspace)",
                           need, (unsigned)KYRO_ACCEPT_STATIC_SCRATCH_BYTES);
  void* scratch = nullptr;
  KY_TRY(static_scratch(ctx->device, &scratch));
  return kyro_spec_accept(ctx, p, target_logits, draft_logits, draft_tokens, out_accept_len,
                          out_tokens, out_num_tokens, out_probs, scratch,
                          KYRO_ACCEPT_STATIC_SCRATCH_BYTES);
}
