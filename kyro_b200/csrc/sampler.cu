// sampler.cu -- K2: vocab-wide acceptance sampling for speculative verify,
// and the on-device draft sampler that feeds it.
//
// Replaces SpeculativeDecoder::verify_drafts (src/speculative.rs:286-339),
// which compares argmaxes one position at a time with a host sync per
// position, and sample_token (src/worker.rs:267-362), which copies the row
// to the host.  Everything here stays on the device and is batched.
//
// The normaliser contract of kyro_math.h makes every decision reproducible:
// per-chunk maxima, ky_exp, chunk sums in one fixed fp32 tree (the lane
// layout of a warp that holds the chunk), a fixed butterfly in double, and
// integer (fix62) inverse-CDF weights.  The kernels follow exactly those
// trees, so they reproduce the sequential oracle bit for bit.
//
// Three launches (the chain acceptance chains them: the decide and final
// kernels start while their predecessor drains and wait for the tagged
// records they read, see "chained acceptance"; the other callers wait for
// the whole predecessor grid):
//   accept_stats_kernel   persistent, one warp per 512-entry chunk of every
//                         row (target and draft), grid-stride.  A lane holds
//                         16 logits in registers: chunk max (or argmax),
//                         chunk sum, and e at the draft token.  Each
//                         warp loads its next chunk while it reduces the
//                         current one.  This kernel reads every logit once
//                         and carries nearly all of the step's HBM traffic.
//   accept_decide_kernel  one CTA per sequence: row normalisers (or argmaxes)
//                         from the chunk statistics, then the k accept tests,
//                         the accepted length and the row to draw from.
//   accept_final_kernel   one warp per 512 entries of each chosen row: fix62
//                         weights (residual or p) and their sum; the warp
//                         that finishes a row's last sum finds the 512-entry
//                         range holding the cut point and scans it.
//
// This file is compiled with --fmad=false; the shared arithmetic also uses
// explicit round-to-nearest intrinsics.
#include <algorithm>
#include <mutex>

#include "kyro_internal.cuh"
#include "kyro_math.h"
#include "xchg.cuh"

namespace {

constexpr int kChunk = KY_CHUNK;     // 512 logits per chunk, one warp
constexpr int kVec = kChunk / 128;   // 4 float4 per lane
constexpr int kPerLane = kChunk / 32;
constexpr int kWarps = 4;            // warps per CTA (stats and final kernels)
constexpr int kThreads = kWarps * 32;
constexpr int kStatsMinCtas = 8;     // resident CTAs per SM the registers allow
constexpr int kMaxChunks = 1024;     // V <= 524288
constexpr int kMaxDraft = 64;
constexpr int kMaxRows = 2 * kMaxDraft + 1;
constexpr int kDecideWarps = 16;
constexpr int kFinalPerWarp = 4;   // chunks per warp in the final kernel
constexpr int kFinalPerCta = kWarps * kFinalPerWarp;
// Resident final CTAs per SM: 7 x 148 holds config 1's 1024 CTAs in one
// wave, so no CTA waits for a slot behind CTAs that wait for their flags.
constexpr int kFinalMinCtas = 7;

static_assert(kChunk == 512, "the kernels assume 16 logits per lane");

// A chunk's statistics, stored as two 64-bit words that each carry a tag in
// their high half: (m, tag) and (E or arg, tag).  Each word is written and
// read as one 64-bit access, so a reader that sees the tag sees the value
// stored with it.  The chained acceptance tags every record with its call's
// tag and its decide kernel waits for those tags (see "chained acceptance");
// the other launches write tag 0, which no chained call uses.
struct ChunkStat {
  float m;        // chunk max of s = z * inv_t (or of z, greedy)
  uint32_t tag;
  float E;        // ky_chunk_sum of ky_exp(s - m) (stochastic); the bits of
                  // the lowest index attaining m (greedy)
  uint32_t tag2;
};

__host__ __device__ inline int32_t stat_arg(const ChunkStat& c) {
#if defined(__CUDA_ARCH__)
  return __float_as_int(c.E);
#else
  int32_t v;
  memcpy(&v, &c.E, 4);
  return v;
#endif
}

struct RowStat {
  float M;      // row max
  int32_t arg;  // row argmax (greedy)
  double S;     // row normaliser
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

// n / d for 0 <= n < 2^31 as (umulhi(n, m) + n) >> s (Granlund and
// Montgomery, "Division by invariant integers using multiplication", 1994).
struct FastDiv {
  uint32_t d, m, s;
};

FastDiv make_fastdiv(uint32_t d) {
  uint32_t s = 0;
  while ((1ull << s) < d) ++s;
  const uint64_t m = ((1ull << 32) * ((1ull << s) - d)) / d + 1;
  return FastDiv{d, (uint32_t)m, s};
}

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
  return (__umulhi(n, f.m) + n) >> f.s;
}

// Tensor-parallel exchange records (one per row or per sequence and rank).
struct TpRow1 {  // round 1 (greedy): this rank's row max and argmax as a global id
  float M;
  int32_t arg;
};
struct TpRow2 {  // round 1 (stochastic): this rank's row max M, its part of
  double S;      // the normaliser under M, and e and the chunk max at the
  float ex;      // draft token when this rank holds the token (else 0)
  float mcx;
  float M;
  int32_t _pad;
};
struct TpSeq3 {  // round 2: this rank's weight totals of the chosen row
  unsigned long long w_res, w_p;
};

struct Args {
  const float* plog;            // target logits (accept) or the rows to sample
  const float* qlog;            // draft logits (stochastic accept) or null
  const int32_t* draft_tokens;  // [B, k] (accept)
  int B;                        // sequences (accept) or rows (sampler)
  int k;                        // drafts per sequence; 0 for the sampler
  int R;                        // stats rows per sequence
  int64_t V;
  int nchunks;
  int nfull;                    // chunks wholly inside V (the rest pad with -inf)
  FastDiv div_chunks, div_rows;  // by nchunks, by R
  float inv_t;
  int stoch;                    // softmax statistics (else argmax only)
  int greedy_ref;
  int sample;                   // draft-sampler call
  int pos_div;                  // sampler: Philox seq = r / pos_div, pos = r % pos_div
  int64_t seq_rows;             // sampler: logits rows from one sequence to the next (>= pos_div)
  uint64_t seed;
  uint32_t step;
  int64_t seq_offset;
  int32_t* out_accept_len;
  int32_t* out_tokens;
  int32_t* out_num_tokens;
  float* out_probs;             // accept: [B,k,2] (p,q); sampler: [rows]
  ChunkStat* stats;             // [B*R][nchunks]
  unsigned long long* ex;       // [B*R] (e at the draft token, tag) as one 64-bit word
  uint32_t* final_ready;        // [B] the call's tag once final_rows[b] is written (poll)
  // Chained acceptance (poll != 0): the decide and final kernels start
  // while their predecessor drains and wait for the records they read
  // instead of the whole grid (see "chained acceptance" below)
  int poll;
  const uint32_t* gen;          // the context's generation count
  uint32_t* done;               // sequences finished in this call
  uint32_t salt;                // the context's tag salt
  FinalRow* final_rows;         // [B]
  unsigned long long* W;        // [B][nchunks] weight sums of the chosen rows
  uint32_t* cnt_c;              // [B] finished weight sums per sequence
  uint32_t units;               // stats units: B * R * nchunks
  // The stats units' counter: [0] the next unit to take, [1] retired warps;
  // both back at zero when the stats kernel ends
  uint32_t* unit_ctr;
  uint32_t* status;
  // tensor parallelism (vocabulary shards): V above is this shard's width
  int64_t V_global;             // the full vocabulary (V without a group)
  int64_t vocab_offset;         // global id of this shard's entry 0
  int tp_rank, tp_world;
  TpRow1 *send1, *recv1;        // [B*R], [world][B*R]
  TpRow2 *send2, *recv2;        // [B*R], [world][B*R]
  TpSeq3 *send3, *recv3;        // [B], [world][B]
  int32_t *send4, *recv4;       // [B]
  unsigned long long* W2;       // [B][nchunks][2]: residual and p weight sums
  // round 1 stored by accept_tp_part_kernel straight into the peers'
  // exchange regions (xpush != 0; recv2 unused): xskip is the round's
  // fault injection, xwait_ns the readers' wait bound
  int xpush, xskip;
  unsigned long long xwait_ns;
  kyro::xchg::Peers xpeers;
  // tree verification: rows per sequence are k+1 = N target rows, then
  // q_rows draft rows (k for the chain)
  int q_rows;
  int tree;
  const int32_t* node_tokens;   // [B, N]
  const int32_t* parents;       // [B, N]
  int32_t* out_path;            // [B, N]
  int32_t* out_path_len;        // [B]
};

__host__ __device__ inline size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }

// Workspace layout.  cnt_c is zeroed by the decide kernel of each call; the
// stats kernel's unit counter (first 8 bytes) is left at zero by every call
// that uses it, and zeroed once when a context first sees the workspace.
struct Workspace {
  uint32_t* unit_ctr;  // 2 words at offset 0 in every layout
  uint32_t* cnt_c;
  size_t counter_bytes;
  ChunkStat* stats;
  unsigned long long* ex;
  uint32_t* final_ready;
  FinalRow* final_rows;
  unsigned long long* W;
  size_t bytes;
};

Workspace carve(void* base, int64_t B, int64_t R, int64_t nchunks) {
  Workspace w;
  char* p = (char*)base;
  size_t off = 0;
  w.unit_ctr = (uint32_t*)(p + off);
  off += 256;
  w.cnt_c = (uint32_t*)(p + off);
  off += align_up(4 * (size_t)B);
  w.counter_bytes = off;
  w.stats = (ChunkStat*)(p + off);
  off += align_up(sizeof(ChunkStat) * (size_t)(B * R * nchunks));
  w.ex = (unsigned long long*)(p + off);
  off += align_up(sizeof(unsigned long long) * (size_t)(B * R));
  w.final_ready = (uint32_t*)(p + off);
  off += align_up(sizeof(uint32_t) * (size_t)B);
  w.final_rows = (FinalRow*)(p + off);
  off += align_up(sizeof(FinalRow) * (size_t)B);
  w.W = (unsigned long long*)(p + off);
  off += align_up(sizeof(unsigned long long) * (size_t)(B * nchunks));
  w.bytes = off;
  return w;
}

// The tensor-parallel call's workspace: the single-GPU layout over this
// rank's columns, then the exchange buffers and the paired chunk sums.
struct TpWorkspace {
  Workspace base;
  TpRow1 *send1, *recv1;
  TpRow2 *send2, *recv2;
  TpSeq3 *send3, *recv3;
  int32_t *send4, *recv4;
  unsigned long long* W2;
  size_t bytes;
};

TpWorkspace carve_tp(void* base, int64_t B, int64_t R, int64_t nchunks, int64_t world) {
  TpWorkspace t;
  t.base = carve(base, B, R, nchunks);
  char* p = (char*)base;
  size_t off = t.base.bytes;
  const int64_t rows = B * R;
  t.send1 = (TpRow1*)(p + off);
  off += align_up(sizeof(TpRow1) * (size_t)rows);
  t.recv1 = (TpRow1*)(p + off);
  off += align_up(sizeof(TpRow1) * (size_t)(rows * world));
  t.send2 = (TpRow2*)(p + off);
  off += align_up(sizeof(TpRow2) * (size_t)rows);
  t.recv2 = (TpRow2*)(p + off);
  off += align_up(sizeof(TpRow2) * (size_t)(rows * world));
  t.send3 = (TpSeq3*)(p + off);
  off += align_up(sizeof(TpSeq3) * (size_t)B);
  t.recv3 = (TpSeq3*)(p + off);
  off += align_up(sizeof(TpSeq3) * (size_t)(B * world));
  t.send4 = (int32_t*)(p + off);
  off += align_up(sizeof(int32_t) * (size_t)B);
  t.recv4 = (int32_t*)(p + off);
  off += align_up(sizeof(int32_t) * (size_t)B);
  t.W2 = (unsigned long long*)(p + off);
  off += align_up(2 * sizeof(unsigned long long) * (size_t)(B * nchunks));
  t.bytes = off;
  return t;
}

// ------------------------------------------------------------ primitives

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

// ky_exp(x), bit for bit, in fewer instructions.  With t = 1.5*2^23 + n,
// bits(t) << 23 == n << 23 (mod 2^32), so adding it to the bits of the
// polynomial value p multiplies p by 2^n exactly whenever p * 2^n is a
// normal number -- and it always is: the clamp at -87 keeps n >= -126, and
// n == -126 only for x < -86.989, where r > 0.336 and so p > 1.  The
// contract's form computes the same product with an fp32 multiply.
__device__ __forceinline__ float exp_fast(float x) {
  const float xc = fmaxf(x, -87.0f);
  const float t = __fmaf_rn(xc, KY_LOG2E, KY_RND_MAGIC);
  const float nf = __fsub_rn(t, KY_RND_MAGIC);
  const float r = __fmaf_rn(-nf, KY_LN2, xc);
  float p = KY_EXP_C5;
  p = __fmaf_rn(p, r, KY_EXP_C4);
  p = __fmaf_rn(p, r, KY_EXP_C3);
  p = __fmaf_rn(p, r, KY_EXP_C2);
  p = __fmaf_rn(p, r, KY_EXP_C1);
  p = __fmaf_rn(p, r, KY_EXP_C0);
  return __uint_as_float(__float_as_uint(p) + (__float_as_uint(t) << 23));
}

// fp32 warp butterfly (the lanes' part of ky_chunk_sum)
__device__ __forceinline__ float warp_butterfly_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- packed pairs of fp32 (sm_100 .f32x2): each half rounds exactly as
// the scalar round-to-nearest operation on it, so a pair computes the same
// bits as two scalar evaluations with half the instructions.
typedef unsigned long long f2_t;  // (lo, hi)

__device__ __forceinline__ f2_t f2_pack(float lo, float hi) {
  f2_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ void f2_unpack(f2_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

__device__ __forceinline__ f2_t f2_fma(f2_t a, f2_t b, f2_t c) {
  f2_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__device__ __forceinline__ f2_t f2_add(f2_t a, f2_t b) {
  f2_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ f2_t f2_sub(f2_t a, f2_t b) {
  f2_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ f2_t f2_mul(f2_t a, f2_t b) {
  f2_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// max of three (NaN inputs are ignored, as by fmaxf)
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// min of three; NaN if any input is NaN
__device__ __forceinline__ float min3_nan(float a, float b, float c) {
  float d;
  asm("min.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start before its predecessor ends; grid_dependency_wait
// blocks until the predecessor grid has completed and its writes are
// visible, and allow_dependents lets the next kernel begin launching.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void allow_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// exp_fast of both halves.  fma(-nf, ln2, x) is written fma(nf, -ln2, x):
// the product is exact inside the fma, so the sign can move to ln2.
// CLAMP = false is for arguments already known to be >= -87 (and not NaN),
// where the clamp is the identity.
template <bool CLAMP = true>
__device__ __forceinline__ f2_t exp_pair(f2_t x) {
  float xl, xh;
  f2_unpack(x, xl, xh);
  const f2_t xc = CLAMP ? f2_pack(fmaxf(xl, -87.0f), fmaxf(xh, -87.0f)) : x;
  const f2_t t = f2_fma(xc, f2_pack(KY_LOG2E, KY_LOG2E), f2_pack(KY_RND_MAGIC, KY_RND_MAGIC));
  const f2_t nf = f2_sub(t, f2_pack(KY_RND_MAGIC, KY_RND_MAGIC));
  const f2_t r = f2_fma(nf, f2_pack(-KY_LN2, -KY_LN2), xc);
  f2_t p = f2_fma(f2_pack(KY_EXP_C5, KY_EXP_C5), r, f2_pack(KY_EXP_C4, KY_EXP_C4));
  p = f2_fma(p, r, f2_pack(KY_EXP_C3, KY_EXP_C3));
  p = f2_fma(p, r, f2_pack(KY_EXP_C2, KY_EXP_C2));
  p = f2_fma(p, r, f2_pack(KY_EXP_C1, KY_EXP_C1));
  p = f2_fma(p, r, f2_pack(KY_EXP_C0, KY_EXP_C0));
  float pl, ph, tl, th;
  f2_unpack(p, pl, ph);
  f2_unpack(t, tl, th);
  return f2_pack(__uint_as_float(__float_as_uint(pl) + (__float_as_uint(tl) << 23)),
                 __uint_as_float(__float_as_uint(ph) + (__float_as_uint(th) << 23)));
}

// The logits row of sampler row b (sequence b / pos_div, position b % pos_div).
__device__ __forceinline__ int64_t sample_row(const Args& a, int b) {
  return (int64_t)(b / a.pos_div) * a.seq_rows + b % a.pos_div;
}

// Chunk statistics, e values and final-row descriptors can be produced by a
// kernel that is still running (the chained acceptance), so they are read
// with ld.global.cg: from L2, never from a possibly stale L1 line.
__device__ __forceinline__ ChunkStat ld_stat(const ChunkStat* p) {
  unsigned long long lo, hi;
  asm volatile("ld.global.cg.v2.u64 {%0, %1}, [%2];" : "=l"(lo), "=l"(hi) : "l"(p) : "memory");
  ChunkStat s;
  s.m = __uint_as_float((uint32_t)lo);
  s.tag = (uint32_t)(lo >> 32);
  s.E = __uint_as_float((uint32_t)hi);
  s.tag2 = (uint32_t)(hi >> 32);
  return s;
}

// Both words of a chunk record, each one 64-bit store.
__device__ __forceinline__ void st_stat(ChunkStat* p, float m, float e, uint32_t tag) {
  const unsigned long long lo = (unsigned long long)__float_as_uint(m) | ((unsigned long long)tag << 32);
  const unsigned long long hi = (unsigned long long)__float_as_uint(e) | ((unsigned long long)tag << 32);
  asm volatile("st.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(lo), "l"(hi) : "memory");
}

__device__ __forceinline__ float ld_ex(const Args& a, int64_t srow) {
  return __uint_as_float((uint32_t)__ldcg(&a.ex[srow]));
}

__device__ __forceinline__ float ld_m(const ChunkStat* p) { return __ldcg(&p->m); }

__device__ __forceinline__ const float* stats_row_ptr(const Args& a, int b, int r) {
  if (a.sample) return a.plog + sample_row(a, b) * a.V;
  if (r <= a.k) return a.plog + ((int64_t)b * (a.k + 1) + r) * a.V;
  return a.qlog + ((int64_t)b * a.q_rows + (r - a.k - 1)) * a.V;
}

__device__ __forceinline__ int draft_token_of_row(const Args& a, int b, int r) {
  if (a.sample || a.tree) return -1;
  if (r < a.k) return a.draft_tokens[(int64_t)b * a.k + r];
  if (r > a.k) return a.draft_tokens[(int64_t)b * a.k + (r - a.k - 1)];
  return -1;
}

// ------------------------------------------------------------ chained acceptance
//
// The chain acceptance's three kernels (stats, decide, final) run with
// programmatic dependent launch: a kernel's CTAs become resident while its
// predecessor drains.  Instead of waiting for the whole predecessor grid,
// they wait for the records they read: every chunk record and every e value
// carries the call's tag in each 64-bit word it is stored in, and a decide
// CTA publishes its final-row descriptor with a tagged flag (release /
// acquire).  So the decide step of a sequence starts as soon as its rows'
// records are in, overlapping the tail of the stats pass, and a final CTA
// as soon as its sequence is decided.  Every wait is for a kernel whose CTAs
// have all been resident since before the waiting CTA launched (a dependent
// grid launches only after every CTA of its predecessor has started), so
// every wait ends; each is also bounded (KYRO_DEV_WAIT_TIMEOUT).  Each kernel
// still calls griddepcontrol.wait before it exits, so it never completes
// before its predecessor.
//
// The tag of a call is a hash of a per-context salt and a generation count
// on the device, read by every CTA at its start; the call's last finished
// sequence advances the count, so every call, and every replay of a
// captured graph, has a new tag, and a record left by an earlier call,
// another context or other data does not match it (a hash collision aside,
// about 2^-32 per record).

constexpr long long kChainWaitNs = 1000000000ll;

__device__ __forceinline__ uint32_t chain_tag(uint32_t gen, uint32_t salt) {
  // murmur3's finaliser: a bijection, so distinct generations give distinct tags
  uint32_t h = gen ^ salt;
  h ^= h >> 16;
  h *= 0x85ebca6bu;
  h ^= h >> 13;
  h *= 0xc2b2ae35u;
  h ^= h >> 16;
  return h == 0u ? 1u : h;  // tag 0 belongs to the unchained launches
}

__device__ __forceinline__ uint32_t ld_acquire_gpu32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long chain_clock() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t call_tag(const Args& a) {
  return a.poll ? chain_tag(ld_acquire_gpu32(a.gen), a.salt) : 0u;
}

__device__ __forceinline__ bool stat_tagged(const ChunkStat* p, uint32_t tag) {
  const ChunkStat c = ld_stat(p);
  return c.tag == tag && c.tag2 == tag;
}

// The whole warp waits until every chunk record of stats row srow carries
// `tag` (bounded).  Lane l watches chunks l, l + 32, ...; its loads go out
// together, then only the records still missing are polled again.
__device__ __forceinline__ void wait_row(const Args& a, int64_t srow, uint32_t tag) {
  const int lane = threadIdx.x & 31;
  const ChunkStat* st = a.stats + srow * a.nchunks;
  const unsigned long long t0 = chain_clock();
  for (int g = 0; g < a.nchunks; g += 256) {
    unsigned missing = 0;  // bit j: chunk g + j*32 + lane not yet tagged
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = g + j * 32 + lane;
      if (c < a.nchunks && !stat_tagged(st + c, tag)) missing |= 1u << j;
    }
    while (__any_sync(0xffffffffu, missing != 0)) {
      if (chain_clock() - t0 > (unsigned long long)kChainWaitNs) {
        if (lane == 0) kyro::dev::flag(a.status, KYRO_DEV_WAIT_TIMEOUT);
        return;
      }
      __nanosleep(256);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if ((missing >> j) & 1u)
          if (stat_tagged(st + g + j * 32 + lane, tag)) missing &= ~(1u << j);
    }
  }
}

// Lane j waits for what accept test j reads (the draft token's e in the
// target and the draft row, and those chunks' records), bounded.  A draft
// token outside the vocabulary has none (and the test reads none).
__device__ __forceinline__ void wait_tests(const Args& a, int b, uint32_t tag) {
  const int lane = threadIdx.x & 31;
  const unsigned long long t0 = chain_clock();
  const int64_t r0 = (int64_t)b * a.R;
  for (int j = lane; j < a.k; j += 32) {
    const int x = a.draft_tokens[(int64_t)b * a.k + j];
    if (x < 0 || x >= a.V) continue;
    const int cx = x / kChunk;
    for (int side = 0; side < 2; ++side) {
      const int64_t srow = side == 0 ? r0 + j : r0 + a.k + 1 + j;
      while ((uint32_t)(__ldcg(&a.ex[srow]) >> 32) != tag ||
             !stat_tagged(a.stats + srow * a.nchunks + cx, tag)) {
        if (chain_clock() - t0 > (unsigned long long)kChainWaitNs) {
          kyro::dev::flag(a.status, KYRO_DEV_WAIT_TIMEOUT);
          break;
        }
        __nanosleep(256);
      }
    }
  }
  __syncwarp();
}

__device__ __forceinline__ FinalRow ld_final_row(const FinalRow* g) {
  FinalRow fr;
  fr.p_row = __ldcg(&g->p_row);
  fr.q_row = __ldcg(&g->q_row);
  fr.p_stat = __ldcg(&g->p_stat);
  fr.q_stat = __ldcg(&g->q_stat);
  fr.Mp = __ldcg(&g->Mp);
  fr.Mq = __ldcg(&g->Mq);
  fr.Sp = __ldcg(&g->Sp);
  fr.Sq = __ldcg(&g->Sq);
  fr.odd = __ldcg(&g->odd);
  fr.out_index = __ldcg(&g->out_index);
  fr.skip = __ldcg(&g->skip);
  fr._pad = 0;
  return fr;
}

// One thread waits until a 32-bit word reads `tag` (bounded).
__device__ __forceinline__ void wait_flag(const Args& a, const uint32_t* word, uint32_t tag) {
  if (ld_acquire_gpu32(word) == tag) return;
  const unsigned long long t0 = chain_clock();
  while (ld_acquire_gpu32(word) != tag) {
    if (chain_clock() - t0 > (unsigned long long)kChainWaitNs) {
      kyro::dev::flag(a.status, KYRO_DEV_WAIT_TIMEOUT);
      return;
    }
    __nanosleep(256);
  }
}

// One more finished sequence; the call's last one advances the generation,
// which gives the next call its tag.  One thread.
__device__ __forceinline__ void chain_seq_done(const Args& a) {
  __threadfence();
  if (atomicAdd(a.done, 1u) == (uint32_t)(a.B - 1)) {
    *a.done = 0u;
    __threadfence();
    atomicAdd(const_cast<uint32_t*>(a.gen), 1u);
  }
}

// ------------------------------------------------------------ stats kernel

// One chunk in flight: its 16 logits per lane and where it belongs.
struct Slice {
  float v[kPerLane];  // float4 i (0..3) holds chunk entries (i*32 + lane)*4 + 0..3
  ChunkStat* dst;     // the chunk's record
  uint32_t srow;      // stats row: b * R + r
  int c;              // chunk index in the row
  int x;              // draft token scored in this row (in [0, V)), -1 if none
};

// Where a batch's first unit lies: its stats row, chunk, draft token and
// logits row.  The batch's other units follow it chunk by chunk (a batch of
// kGrab units crosses into the next row at most once).
struct RowCursor {
  uint32_t u0, srow;
  int c0, x;
  const float* row;
  ChunkStat* st;  // the row's chunk records
};

__device__ __forceinline__ void cursor_at(const Args& a, uint32_t u, RowCursor& rc) {
  const uint32_t srow = fdiv(u, a.div_chunks);
  const int b = (int)fdiv(srow, a.div_rows);
  const int r = (int)(srow - (uint32_t)b * (uint32_t)a.R);
  const int xg = draft_token_of_row(a, b, r);  // global id, -1 for none
  rc.u0 = u;
  rc.srow = srow;
  rc.c0 = (int)(u - srow * (uint32_t)a.nchunks);
  const int64_t xl = xg < 0 ? -1 : (int64_t)xg - a.vocab_offset;
  rc.x = (xl >= 0 && xl < a.V) ? (int)xl : -1;
  rc.row = stats_row_ptr(a, b, r);
  rc.st = a.stats + (int64_t)srow * a.nchunks;
}

// Issue the loads of unit u, a unit of the batch rc starts (entries past V
// read as -inf).
template <bool VEC>
__device__ __forceinline__ void load_slice(const Args& a, const RowCursor& rc, uint32_t u,
                                           Slice& s) {
  const int lane = threadIdx.x & 31;
  int c = rc.c0 + (int)(u - rc.u0);
  uint32_t srow = rc.srow;
  int x = rc.x;
  const float* row = rc.row;
  ChunkStat* st = rc.st;
  if (c >= a.nchunks) {  // past the end of the batch's first row
    RowCursor t;
    cursor_at(a, u, t);
    srow = t.srow;
    c = t.c0;
    x = t.x;
    row = t.row;
    st = t.st;
  }
  s.dst = st + c;
  s.srow = srow;
  s.c = c;
  s.x = x;
  const int64_t base = (int64_t)c * kChunk;
  if (VEC && c < a.nfull) {
    const float4* src = reinterpret_cast<const float4*>(row + base) + lane;
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
      const float4 f = __ldcg(src + i * 32);
      s.v[4 * i + 0] = f.x;
      s.v[4 * i + 1] = f.y;
      s.v[4 * i + 2] = f.z;
      s.v[4 * i + 3] = f.w;
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int64_t e0 = base + (i * 32 + lane) * 4;
    if (VEC) {
      float4 f = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      if (e0 < a.V) f = __ldcg(reinterpret_cast<const float4*>(row + e0));
      s.v[4 * i + 0] = f.x;
      s.v[4 * i + 1] = f.y;
      s.v[4 * i + 2] = f.z;
      s.v[4 * i + 3] = f.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) s.v[4 * i + j] = (e0 + j < a.V) ? __ldcg(row + e0 + j) : -INFINITY;
    }
  }
}

// Reduce one chunk and store its statistics.
template <bool STOCH>
__device__ __forceinline__ void reduce_slice(const Args& a, Slice& s, uint32_t tag) {
  const int lane = threadIdx.x & 31;
  ChunkStat st;
  if (STOCH) {
    // columns (0,1) and (2,3) of each float4 as packed pairs
    f2_t z[2 * kVec];
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
      z[2 * i] = f2_pack(s.v[4 * i], s.v[4 * i + 1]);
      z[2 * i + 1] = f2_pack(s.v[4 * i + 2], s.v[4 * i + 3]);
    }
    if (a.inv_t != 1.0f) {
      const f2_t it = f2_pack(a.inv_t, a.inv_t);
#pragma unroll
      for (int i = 0; i < 2 * kVec; ++i) z[i] = f2_mul(z[i], it);
#pragma unroll
      for (int i = 0; i < kVec; ++i) {
        f2_unpack(z[2 * i], s.v[4 * i], s.v[4 * i + 1]);
        f2_unpack(z[2 * i + 1], s.v[4 * i + 2], s.v[4 * i + 3]);
      }
    }
    // the max is order-free: a tree of three-input maxima
    const float* v = s.v;
    const float m01 = max3(max3(v[0], v[1], v[2]), max3(v[3], v[4], v[5]), v[6]);
    const float m02 = max3(max3(v[7], v[8], v[9]), max3(v[10], v[11], v[12]), v[13]);
    const float m = kyro::dev::warp_max(max3(m01, m02, max3(v[14], v[15], -INFINITY)));
    // ky_chunk_sum's tree: column j of this lane sums steps i = 0..3 in
    // order, then (a0 + a1) + (a2 + a3), then the lane butterfly
    const f2_t m2 = f2_pack(m, m);
    f2_t acc01 = f2_pack(0.0f, 0.0f), acc23 = f2_pack(0.0f, 0.0f);
    // ky_exp clamps its argument at -87.  When the chunk's smallest entry
    // already gives z - m >= -87 (fsub is monotonic, so one check covers
    // every entry; -inf, NaN and an all -inf chunk fail it), the clamp is
    // the identity and the warp skips it.  The vote keeps the branch uniform.
    const float lmin = min3_nan(min3_nan(min3_nan(v[0], v[1], v[2]), min3_nan(v[3], v[4], v[5]),
                                         min3_nan(v[6], v[7], v[8])),
                                min3_nan(min3_nan(v[9], v[10], v[11]),
                                         min3_nan(v[12], v[13], v[14]), v[15]),
                                v[15]);
    if (__all_sync(0xffffffffu, KY_FSUB(lmin, m) >= -87.0f)) {
#pragma unroll
      for (int i = 0; i < kVec; ++i) {
        acc01 = f2_add(acc01, exp_pair<false>(f2_sub(z[2 * i], m2)));
        acc23 = f2_add(acc23, exp_pair<false>(f2_sub(z[2 * i + 1], m2)));
      }
    } else {
#pragma unroll
      for (int i = 0; i < kVec; ++i) {
        acc01 = f2_add(acc01, exp_pair(f2_sub(z[2 * i], m2)));
        acc23 = f2_add(acc23, exp_pair(f2_sub(z[2 * i + 1], m2)));
      }
    }
    float a0, a1, a2, a3;
    f2_unpack(acc01, a0, a1);
    f2_unpack(acc23, a2, a3);
    st.m = m;
    st.E = warp_butterfly_f(__fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3)));
    // e at the draft token, by the lane that holds it (s.v holds z * inv_t);
    // xo is negative for a row without one (s.x == -1)
    const int xo = s.x - s.c * kChunk;
    if ((unsigned)xo < (unsigned)kChunk && lane == ((xo >> 2) & 31)) {
      const int q = ((xo >> 7) << 2) | (xo & 3);
      float z = s.v[0];
#pragma unroll
      for (int i = 1; i < kPerLane; ++i)
        if (i == q) z = s.v[i];
      a.ex[s.srow] = (unsigned long long)__float_as_uint(exp_fast(KY_FSUB(z, m))) |
                     ((unsigned long long)tag << 32);
    }
  } else {
    const int base = s.c * kChunk;  // token ids are int32
    float m = -INFINITY;
    int arg = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i)
      if (s.v[i] > m) {
        m = s.v[i];
        arg = base + ((i >> 2) * 32 + lane) * 4 + (i & 3);
      }
    kyro::dev::warp_argmax(m, arg);
    st.m = m;
    st.E = __int_as_float(arg);
  }
  if (lane == 0) st_stat(s.dst, st.m, st.E, tag);
}

// Units a warp takes from the counter at a time (dynamic distribution).
constexpr uint32_t kGrab = 8;

__device__ __forceinline__ uint32_t take_units(uint32_t* ctr) {
  uint32_t v = 0;
  if ((threadIdx.x & 31) == 0) v = atomicAdd(ctr, kGrab);
  return __shfl_sync(0xffffffffu, v, 0);
}

// Persistent; each warp loads unit i+1 before it reduces unit i.  Warps
// take batches of kGrab consecutive units from one counter (a.unit_ctr, at
// the start of the workspace), one batch ahead, so a warp on an SM that
// streams faster takes more of them and the whole grid still reads the rows
// in order.  Measured on config 1 (acceptance alone): a static split (warp
// w takes units w, w + W, ...) 100.5 us, with warp end times from 48 to
// 71 us; one counter with batches of 2 / 4 / 8 / 12 / 16 / 32 units 132 /
// 100.4 / 99.2 / 102.0 / 101.9 / 149 us (short batches queue on the
// counter, long ones leave warps idle at the end); 16 ranges with a counter
// each, 107-116 us (the grid then reads 16 places at once).  On config 3
// over two ranks the static split's warps ended between 149 and 226 us.
// Every warp retires once it has seen the counter past the last unit; the
// last one to retire sets the counter back to zero for the next call on
// this workspace.
template <bool VEC, bool STOCH>
__global__ void __launch_bounds__(kThreads, kStatsMinCtas) accept_stats_kernel(Args a) {
  allow_dependents();
  const uint32_t tag = call_tag(a);
  Slice s0, s1;
  uint32_t u = take_units(a.unit_ctr);
  uint32_t nxt = take_units(a.unit_ctr);
  if (u < a.units) {
    uint32_t end = min(u + kGrab, a.units);
    RowCursor rc;  // the current batch's position, decoded once per batch
    cursor_at(a, u, rc);
    // the unit after u, or a value >= units when the warp is done
    auto advance = [&](uint32_t cur) -> uint32_t {
      if (cur + 1 < end) return cur + 1;
      const uint32_t n = nxt;
      if (n < a.units) {
        end = min(n + kGrab, a.units);
        nxt = take_units(a.unit_ctr);
        cursor_at(a, n, rc);
      }
      return n;
    };
    load_slice<VEC>(a, rc, u, s0);
    while (true) {
      uint32_t un = advance(u);
      if (un < a.units) load_slice<VEC>(a, rc, un, s1);
      reduce_slice<STOCH>(a, s0, tag);
      if (un >= a.units) break;
      u = un;
      un = advance(u);
      if (un < a.units) load_slice<VEC>(a, rc, un, s0);
      reduce_slice<STOCH>(a, s1, tag);
      if (un >= a.units) break;
      u = un;
    }
  }
  // every take of this warp has returned: retire; the last warp resets
  if ((threadIdx.x & 31) == 0) {
    __threadfence();
    if (atomicAdd(a.unit_ctr + 1, 1u) == gridDim.x * (uint32_t)kWarps - 1u) {
      a.unit_ctr[0] = 0u;
      a.unit_ctr[1] = 0u;
    }
  }
}

// ------------------------------------------------------------ decide kernel

// Row normaliser (or argmax) of stats row srow, by one warp.  Lane l visits
// chunks l, l+32, l+64, ... in that order (the contract's butterfly order);
// loads go out eight at a time so that a pass costs one memory round trip
// per 256 chunks.
__device__ __forceinline__ RowStat row_stat(const Args& a, int64_t srow) {
  const int lane = threadIdx.x & 31;
  const ChunkStat* st = a.stats + srow * a.nchunks;
  const int nc = a.nchunks;
  RowStat rs;
  rs.arg = 0;
  rs.S = 0.0;
  if (a.stoch && nc <= 256) {
    // one round trip: the lane's chunk maxima and sums stay in registers
    // between the maximum and the normaliser
    float mm[8], ee[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = j * 32 + lane;
      mm[j] = -INFINITY;
      ee[j] = 0.0f;
      if (c < nc) {
        const ChunkStat cs = ld_stat(st + c);
        mm[j] = cs.m;
        ee[j] = cs.E;
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) M = fmaxf(M, mm[j]);
    M = kyro::dev::warp_max(M);
    double t = 0.0;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j * 32 + lane < nc) t = KY_DADD(t, ky_chunk_mass(ee[j], mm[j], M));
    rs.M = M;
    rs.S = warp_butterfly(t);
  } else if (a.stoch) {
    float M = -INFINITY;
    for (int g = 0; g < nc; g += 256) {
      float mm[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = g + j * 32 + lane;
        mm[j] = c < nc ? ld_m(st + c) : -INFINITY;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) M = fmaxf(M, mm[j]);
    }
    M = kyro::dev::warp_max(M);
    double t = 0.0;
    for (int g = 0; g < nc; g += 256) {
      float mm[8], ee[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = g + j * 32 + lane;
        const ChunkStat cs = ld_stat(st + (c < nc ? c : 0));
        mm[j] = c < nc ? cs.m : 0.0f;
        ee[j] = c < nc ? cs.E : 0.0f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (g + j * 32 + lane < nc) t = KY_DADD(t, ky_chunk_mass(ee[j], mm[j], M));
    }
    rs.M = M;
    rs.S = warp_butterfly(t);
  } else {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int g = 0; g < nc; g += 256) {
      float mm[8];
      int aa[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = g + j * 32 + lane;
        const ChunkStat cs = ld_stat(st + (c < nc ? c : 0));
        mm[j] = c < nc ? cs.m : -INFINITY;
        aa[j] = c < nc ? stat_arg(cs) : 0x7fffffff;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (mm[j] > best || (mm[j] == best && aa[j] < bi)) {
          best = mm[j];
          bi = aa[j];
        }
    }
    kyro::dev::warp_argmax(best, bi);
    rs.M = best;
    rs.arg = bi == 0x7fffffff ? 0 : bi;
  }
  return rs;
}

// What accept test j reads besides the row statistics: the draft token, e at
// it in the target and the draft row, and those rows' chunk maxima there.
struct TestInputs {
  int x;
  float ep, eq, mp, mq;
};

__device__ __forceinline__ TestInputs load_test(const Args& a, int b, int j) {
  TestInputs t;
  t.x = -1;
  t.ep = t.eq = t.mp = t.mq = 0.0f;
  if (j >= a.k) return t;
  const int64_t r0 = (int64_t)b * a.R;
  t.x = a.draft_tokens[(int64_t)b * a.k + j];
  if (a.stoch && t.x >= 0 && t.x < a.V) {
    const int cx = t.x / kChunk;
    t.ep = ld_ex(a, r0 + j);
    t.eq = ld_ex(a, r0 + a.k + 1 + j);
    t.mp = ld_m(&a.stats[(r0 + j) * a.nchunks + cx]);
    t.mq = ld_m(&a.stats[(r0 + a.k + 1 + j) * a.nchunks + cx]);
  }
  return t;
}

// Warp 0 of a sequence's CTA: the k accept tests (lane j runs test j), the
// accepted prefix, and the descriptor of the row the last token is drawn
// from.  rs holds the sequence's row statistics; t0 / t1 the inputs of
// tests lane and lane + 32.
__device__ __forceinline__ void decide_sequence(const Args& a, int b, const RowStat* rs,
                                                const TestInputs& t0, const TestInputs& t1) {
  const int lane = threadIdx.x & 31;
  const int k = a.k;
  FinalRow fr;
  fr._pad = 0;
  if (a.sample) {
    // one row per "sequence": the draft sampler
    if (lane == 0) {
      const int64_t seq = a.seq_offset + b / a.pos_div;
      const int pos = b % a.pos_div;
      fr.p_row = sample_row(a, b);
      fr.p_stat = b;
      fr.q_row = -1;
      fr.q_stat = -1;
      fr.Mq = 0.0f;
      fr.Sq = 1.0;
      fr.out_index = b;
      fr.odd = ky_uniform_odd(a.seed, (uint32_t)seq, (uint32_t)pos, KY_STREAM_DRAFT, a.step);
      if (a.stoch) {
        fr.skip = 0;
        fr.Mp = rs[0].M;
        fr.Sp = rs[0].S;
      } else {
        fr.skip = 1;
        fr.Mp = 0.0f;
        fr.Sp = 1.0;
        a.out_tokens[b] = rs[0].arg;
        if (a.out_probs) a.out_probs[b] = 1.0f;
      }
      a.final_rows[b] = fr;
    }
    return;
  }
  const uint32_t seq = (uint32_t)(a.seq_offset + b);
  const int64_t r0 = (int64_t)b * a.R;
  // lane j runs accept test j (in rounds of 32)
  int first_reject = k;
  for (int j0 = 0; j0 < k; j0 += 32) {
    const int j = j0 + lane;
    const TestInputs& t = j0 == 0 ? t0 : t1;
    bool acc = true;
    if (j < k) {
      const bool ok = t.x >= 0 && t.x < a.V_global;
      if (!ok) kyro::dev::flag(a.status, KYRO_DEV_BAD_TOKEN);
      if (a.stoch) {
        float p = 0.0f, q = 0.0f;
        if (ok) {
          p = KY_FMUL(t.ep, ky_chunk_scale(t.mp, rs[j].M, rs[j].S));
          q = KY_FMUL(t.eq, ky_chunk_scale(t.mq, rs[k + 1 + j].M, rs[k + 1 + j].S));
        }
        if (a.out_probs) {
          a.out_probs[((int64_t)b * k + j) * 2 + 0] = p;
          a.out_probs[((int64_t)b * k + j) * 2 + 1] = q;
        }
        const uint32_t odd = ky_uniform_odd(a.seed, seq, (uint32_t)j, KY_STREAM_ACCEPT, a.step);
        acc = ok && ky_accept(odd, p, q);
      } else {
        acc = ok && rs[j].arg == t.x;
      }
    }
    const unsigned rej = __ballot_sync(0xffffffffu, !acc);
    if (first_reject == k && rej) first_reject = j0 + __ffs(rej) - 1;
  }
  const int aa = first_reject;
  // lane j writes token slot j (and 32 + j): the accepted drafts, then -1
  int32_t* toks = a.out_tokens + (int64_t)b * (k + 1);
  for (int j = lane; j <= k; j += 32) {
    const TestInputs& t = j < 32 ? t0 : t1;
    toks[j] = j < aa ? t.x : -1;
  }
  __syncwarp();
  if (lane != 0) return;
  a.out_accept_len[b] = aa;
  fr.p_row = (int64_t)b * (k + 1) + aa;
  fr.p_stat = r0 + aa;
  fr.out_index = b * (k + 1) + aa;
  fr.odd = ky_uniform_odd(a.seed, seq, (uint32_t)aa, KY_STREAM_RESAMPLE, a.step);
  if (a.stoch) {
    fr.skip = 0;
    fr.Mp = rs[aa].M;
    fr.Sp = rs[aa].S;
    if (aa < k) {
      fr.q_row = (int64_t)b * k + aa;
      fr.q_stat = r0 + k + 1 + aa;
      fr.Mq = rs[k + 1 + aa].M;
      fr.Sq = rs[k + 1 + aa].S;
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
      toks[aa] = rs[aa].arg;
      a.out_num_tokens[b] = aa + 1;
    }
  }
  a.final_rows[b] = fr;
}

// One CTA per sequence (per row for the sampler): warp 0 loads the accept
// tests' inputs while the other warps compute the row statistics, then warp
// 0 runs the tests and writes the sequence's accepted prefix and the row its
// last token is drawn from.
__global__ void __launch_bounds__(kDecideWarps * 32) accept_decide_kernel(Args a) {
  __shared__ RowStat rs[kMaxRows];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int b = blockIdx.x;
  const uint32_t tag = call_tag(a);
  if (!a.poll) grid_dependency_wait();  // the chunk statistics are complete
  allow_dependents();
  if (threadIdx.x == 0) a.cnt_c[b] = 0;  // the final kernel's last-arriver count
  // warp 0 fetches the test inputs (lane j: tests j and j + 32)
  TestInputs t0, t1;
  if (warp == 0 && !a.sample) {
    if (a.poll && a.stoch) wait_tests(a, b, tag);
    t0 = load_test(a, b, lane);
    t1 = load_test(a, b, lane + 32);
  }
  // the other warps take the rows, so that the test inputs' two dependent
  // loads run beside the row statistics
  const int w0 = (a.sample || nwarps == 1) ? 0 : 1;
  if (warp >= w0) {
    for (int r = warp - w0; r < a.R; r += nwarps - w0) {
      if (a.poll) wait_row(a, (int64_t)b * a.R + r, tag);
      const RowStat s = row_stat(a, (int64_t)b * a.R + r);
      if (lane == 0) rs[r] = s;
    }
  }
  __syncthreads();
  if (warp == 0) {
    decide_sequence(a, b, rs, t0, t1);
    __syncwarp();
    if (a.poll && lane == 0) {
      if (a.stoch) {
        // the descriptor, the zeroed count and the tokens before the flag
        __threadfence();
        asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(a.final_ready + b), "r"(tag)
                     : "memory");
      } else {
        chain_seq_done(a);  // greedy: the decision wrote every token
      }
    }
  }
  if (a.poll) grid_dependency_wait();  // complete only after the stats kernel
}

// ------------------------------------------------------------ final kernel

// Per-chunk factors of a final row: g62 = g_c * 2^62 of p (and of q for
// the residual) at chunk c, from the chunk maxima mp, mq.
struct FinalScale {
  float mp, gp62, mq, gq62;
};

__device__ __forceinline__ FinalScale final_scale(const FinalRow& fr, bool residual, float mp,
                                                  float mq) {
  FinalScale s;
  s.mp = mp;
  s.gp62 = ky_scale62(ky_chunk_scale(mp, fr.Mp, fr.Sp));
  s.mq = mq;
  s.gq62 = residual ? ky_scale62(ky_chunk_scale(mq, fr.Mq, fr.Sq)) : 0.0f;
  return s;
}

// 4 logits at e0..e0+3 of a row (entries past V read as -inf)
template <bool VEC>
__device__ __forceinline__ float4 load4(const float* __restrict__ row, int64_t e0, int64_t V) {
  if (VEC) {
    float4 f = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    if (e0 < V) f = __ldcg(reinterpret_cast<const float4*>(row + e0));
    return f;
  }
  float4 f;
  f.x = e0 + 0 < V ? __ldcg(row + e0 + 0) : -INFINITY;
  f.y = e0 + 1 < V ? __ldcg(row + e0 + 1) : -INFINITY;
  f.z = e0 + 2 < V ? __ldcg(row + e0 + 2) : -INFINITY;
  f.w = e0 + 3 < V ? __ldcg(row + e0 + 3) : -INFINITY;
  return f;
}

// fix62 weights of 4 logits of a final row: residual max(p - q, 0) or p,
// in element order.  Neighbouring elements of one row form the packed pairs
// (x, y) and (z, w), so a float4 splits into pairs without register moves;
// each half rounds as the scalar operation would.  wp_out, if given, gets
// the p weights alone (ky_weight_p of the same e_p).
__device__ __forceinline__ void weights_of4(float inv_t, bool residual, const FinalScale& s,
                                            float4 zp, float4 zq, unsigned long long (&w)[4],
                                            unsigned long long* wp_out = nullptr) {
  const f2_t it = f2_pack(inv_t, inv_t);
  const f2_t mp2 = f2_pack(s.mp, s.mp), gp2 = f2_pack(s.gp62, s.gp62);
  f2_t p01 = f2_pack(zp.x, zp.y), p23 = f2_pack(zp.z, zp.w);
  if (inv_t != 1.0f) {
    p01 = f2_mul(p01, it);
    p23 = f2_mul(p23, it);
  }
  p01 = f2_mul(exp_pair(f2_sub(p01, mp2)), gp2);
  p23 = f2_mul(exp_pair(f2_sub(p23, mp2)), gp2);
  float wp[4];
  f2_unpack(p01, wp[0], wp[1]);
  f2_unpack(p23, wp[2], wp[3]);
  if (residual) {
    const f2_t mq2 = f2_pack(s.mq, s.mq), gq2 = f2_pack(s.gq62, s.gq62);
    f2_t q01 = f2_pack(zq.x, zq.y), q23 = f2_pack(zq.z, zq.w);
    if (inv_t != 1.0f) {
      q01 = f2_mul(q01, it);
      q23 = f2_mul(q23, it);
    }
    q01 = f2_mul(exp_pair(f2_sub(q01, mq2)), gq2);
    q23 = f2_mul(exp_pair(f2_sub(q23, mq2)), gq2);
    float d[4];
    f2_unpack(f2_sub(p01, q01), d[0], d[1]);
    f2_unpack(f2_sub(p23, q23), d[2], d[3]);
    // d > 0 ? d : 0 (a NaN difference weighs 0, as in ky_weight_residual)
#pragma unroll
    for (int j = 0; j < 4; ++j) w[j] = __float2ull_rz(fmaxf(d[j], 0.0f));
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) w[j] = __float2ull_rz(wp[j]);
  }
  if (wp_out) {
#pragma unroll
    for (int j = 0; j < 4; ++j) wp_out[j] = residual ? __float2ull_rz(wp[j]) : w[j];
  }
}

// The 16 logits a lane owns in chunk c of the final row (p and, for the
// residual, q), all loads issued together.
template <bool VEC>
__device__ __forceinline__ void load_final_chunk(const Args& a, const FinalRow& fr, bool residual,
                                                 int c, float4 (&zp)[kVec], float4 (&zq)[kVec]) {
  const int lane = threadIdx.x & 31;
  const float* prow = a.plog + fr.p_row * a.V;
  const float* qrow = residual ? a.qlog + fr.q_row * a.V : prow;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int64_t e0 = (int64_t)c * kChunk + (i * 32 + lane) * 4;
    zp[i] = load4<VEC>(prow, e0, a.V);
    zq[i] = residual ? load4<VEC>(qrow, e0, a.V) : zp[i];
  }
}

// Sum of the fix62 weights of chunk c of a final row over the whole warp.
template <bool VEC>
__device__ __forceinline__ unsigned long long chunk_weight_sum(const Args& a, const FinalRow& fr,
                                                               bool residual, int c) {
  float4 zp[kVec], zq[kVec];
  load_final_chunk<VEC>(a, fr, residual, c, zp, zq);
  const float mp = ld_m(&a.stats[fr.p_stat * a.nchunks + c]);
  const float mq = residual ? ld_m(&a.stats[fr.q_stat * a.nchunks + c]) : 0.0f;
  const FinalScale s = final_scale(fr, residual, mp, mq);
  unsigned long long t = 0;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    unsigned long long w[4];
    weights_of4(a.inv_t, residual, s, zp[i], zq[i], w);
    t += (w[0] + w[1]) + (w[2] + w[3]);
  }
  return warp_sum(t);
}

// Both sums of chunk c over the warp: the weights the row samples from
// (residual or p) and the p weights alone (the residual's fallback).
template <bool VEC>
__device__ __forceinline__ void chunk_weight_sums2(const Args& a, const FinalRow& fr, bool residual,
                                                   int c, unsigned long long& t_w,
                                                   unsigned long long& t_p) {
  float4 zp[kVec], zq[kVec];
  load_final_chunk<VEC>(a, fr, residual, c, zp, zq);
  const float mp = ld_m(&a.stats[fr.p_stat * a.nchunks + c]);
  const float mq = residual ? ld_m(&a.stats[fr.q_stat * a.nchunks + c]) : 0.0f;
  const FinalScale s = final_scale(fr, residual, mp, mq);
  unsigned long long tw = 0, tp = 0;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    unsigned long long w[4], wp[4];
    weights_of4(a.inv_t, residual, s, zp[i], zq[i], w, wp);
    tw += (w[0] + w[1]) + (w[2] + w[3]);
    tp += (wp[0] + wp[1]) + (wp[2] + wp[3]);
  }
  t_w = warp_sum(tw);
  t_p = warp_sum(tp);
}

// The entry (an index into this row's columns) whose inclusive weight
// prefix first reaches T, 1 <= T <= the sum of the chunk sums W[c * wstride]
// (-1 if it does not): find the chunk by a prefix scan over the chunk sums,
// then scan the chunk's float4 groups in index order, lanes in order within.
template <bool VEC>
__device__ __forceinline__ int cut_index(const Args& a, const FinalRow& fr, bool residual,
                                         const unsigned long long* W, int wstride,
                                         unsigned long long T,
                                         const unsigned long long* pre = nullptr) {
  const int lane = threadIdx.x & 31;
  const int nc = a.nchunks;
  int sub = -1;
  unsigned long long base = 0;
  // up to 256 chunk sums load in one round trip (or come preloaded: chunk
  // j*32 + lane in pre[j]), then the scan runs on them
  unsigned long long wr[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int c = j * 32 + lane;
    wr[j] = (c < nc && nc <= 256) ? (pre ? pre[j] : __ldcg(&W[(int64_t)c * wstride])) : 0ull;
  }
  for (int s0 = 0; s0 < nc && sub < 0; s0 += 32) {
    unsigned long long ws;
    if (nc <= 256) {
      ws = 0ull;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j * 32 == s0) ws = wr[j];
    } else {
      ws = (s0 + lane < nc) ? __ldcg(&W[(int64_t)(s0 + lane) * wstride]) : 0ull;
    }
    const unsigned long long inc = base + warp_inclusive(ws);
    const unsigned hit = __ballot_sync(0xffffffffu, inc >= T && s0 + lane < nc);
    if (hit) {
      const int l = __ffs(hit) - 1;
      sub = s0 + l;
      const unsigned long long before = __shfl_sync(0xffffffffu, inc - ws, l);
      T -= before;
    } else {
      base = __shfl_sync(0xffffffffu, inc, 31);
    }
  }
  if (sub < 0) return -1;
  float4 zp[kVec], zq[kVec];
  load_final_chunk<VEC>(a, fr, residual, sub, zp, zq);
  const float mp = ld_m(&a.stats[fr.p_stat * nc + sub]);
  const float mq = residual ? ld_m(&a.stats[fr.q_stat * nc + sub]) : 0.0f;
  const FinalScale sc = final_scale(fr, residual, mp, mq);
  unsigned long long cbase = 0;
  int found = -1;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    unsigned long long w[4];
    weights_of4(a.inv_t, residual, sc, zp[i], zq[i], w);
    const unsigned long long s4 = (w[0] + w[1]) + (w[2] + w[3]);
    const unsigned long long inc = warp_inclusive(s4);
    unsigned long long C = cbase + inc - s4;
    int mine = -1;
    if (C < T && C + s4 >= T) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        C += w[j];
        if (mine < 0 && C >= T) mine = j;
      }
    }
    const unsigned hit = __ballot_sync(0xffffffffu, mine >= 0);
    if (found < 0 && hit) {
      const int l = __ffs(hit) - 1;
      const int jj = __shfl_sync(0xffffffffu, mine, l);
      found = sub * kChunk + (i * 32 + l) * 4 + jj;
    }
    cbase += __shfl_sync(0xffffffffu, inc, 31);
  }
  return found;
}

// Locate the cut point of final row b once all its chunk sums are in W.
template <bool VEC>
__device__ __forceinline__ void final_search(const Args& a, int b, const FinalRow& fr) {
  const int lane = threadIdx.x & 31;
  const int nc = a.nchunks;
  unsigned long long* W = a.W + (int64_t)b * nc;
  bool residual = fr.q_row >= 0;
  unsigned long long tot = 0;
  unsigned long long ww[8];  // the first 256 chunk sums, kept for the search
  for (int g = 0; g < nc; g += 256) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = g + j * 32 + lane;
      ww[j] = c < nc ? __ldcg(&W[c]) : 0ull;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) tot += ww[j];
  }
  tot = warp_sum(tot);
  if (residual && tot == 0) {
    // the residual has no mass: sample from p instead
    residual = false;
    for (int c = 0; c < nc; ++c) {
      const unsigned long long t = chunk_weight_sum<VEC>(a, fr, false, c);
      if (lane == 0) W[c] = t;
    }
    __syncwarp();
    __threadfence_block();
    tot = 0;
    for (int c = lane; c < nc; c += 32) tot += __ldcg(&W[c]);
    tot = warp_sum(tot);
  }
  int token = (int)a.V - 1;
  if (tot != 0) {
    // the sums in ww are the ones just added up, unless the residual had no
    // mass and W was refilled with the p weights
    const bool keep = nc <= 256 && (fr.q_row < 0 || residual);
    const int found = cut_index<VEC>(a, fr, residual, W, 1, ky_cdf_threshold(fr.odd, tot),
                                     keep ? ww : nullptr);
    if (found >= 0) token = found;
  }
  if (lane == 0) {
    a.out_tokens[fr.out_index] = token;
    if (a.sample && a.out_probs) {
      const int c = token / kChunk;
      const float mp = ld_m(&a.stats[fr.p_stat * nc + c]);
      a.out_probs[fr.out_index] =
          KY_FMUL(ky_exp(KY_FSUB(KY_FMUL(__ldg(a.plog + fr.p_row * a.V + token), a.inv_t), mp)),
                  ky_chunk_scale(mp, fr.Mp, fr.Sp));
    }
  }
}

// Weight sums: a CTA covers kFinalPerCta chunks of one sequence's chosen
// row, warp w the chunks w, w + 4, ... of them (neighbouring warps read
// neighbouring chunks).  Sequences run in reverse, so the rows the stats
// kernel read last (the ones most likely still in L2) come first.  The last
// CTA of a row to finish locates the cut point -- or, under tensor
// parallelism (TP), sums this rank's residual and p weights for the
// exchange that precedes the search.
template <bool VEC, bool TP>
__global__ void __launch_bounds__(kThreads, kFinalMinCtas) accept_final_kernel(Args a) {
  __shared__ int last_cta;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_seq = (a.nchunks + kFinalPerCta - 1) / kFinalPerCta;
  const int y = (int)(blockIdx.x / (unsigned)per_seq);
  const int b = a.B - 1 - y;
  const int c0 = (int)(blockIdx.x - (unsigned)y * per_seq) * kFinalPerCta;
  __shared__ FinalRow sh_fr;
  if (a.poll) {
    // this sequence's decision is published (its descriptor, the zeroed count)
    if (threadIdx.x == 0) {
      wait_flag(a, a.final_ready + b, call_tag(a));
      sh_fr = ld_final_row(a.final_rows + b);
    }
    __syncthreads();
  } else {
    grid_dependency_wait();  // the decide kernel has written final_rows and zeroed cnt_c
  }
  allow_dependents();      // the stream's next kernel (e.g. the KV commit) may start launching
  const FinalRow fr = a.poll ? sh_fr : a.final_rows[b];
  if (fr.skip) {  // the same for the whole CTA
    if (a.poll) grid_dependency_wait();
    return;
  }
  const bool residual = fr.q_row >= 0;
#pragma unroll 1
  for (int i = 0; i < kFinalPerWarp; ++i) {
    const int c = c0 + i * kWarps + warp;
    if (c >= a.nchunks) break;
    if (TP) {
      unsigned long long tw, tp;
      chunk_weight_sums2<VEC>(a, fr, residual, c, tw, tp);
      if (lane == 0) {
        a.W2[((int64_t)b * a.nchunks + c) * 2 + 0] = tw;
        a.W2[((int64_t)b * a.nchunks + c) * 2 + 1] = tp;
      }
    } else {
      const unsigned long long t = chunk_weight_sum<VEC>(a, fr, residual, c);
      if (lane == 0) a.W[(int64_t)b * a.nchunks + c] = t;
    }
  }
  if (lane == 0) __threadfence();  // this warp's sums are visible before the count
  __syncthreads();
  if (threadIdx.x == 0) last_cta = atomicAdd(&a.cnt_c[b], 1u) == (uint32_t)(per_seq - 1);
  __syncthreads();
  if (!last_cta || warp != 0) {
    if (a.poll) grid_dependency_wait();  // complete only after the decide kernel
    return;
  }
  __threadfence();  // every other CTA's sums are visible from here on
  if (!TP) {
    final_search<VEC>(a, b, fr);
    if (a.poll) {
      if (lane == 0) chain_seq_done(a);
      grid_dependency_wait();
    }
    return;
  }
  unsigned long long tw = 0, tp = 0;
  for (int c = lane; c < a.nchunks; c += 32) {
    tw += __ldcg(&a.W2[((int64_t)b * a.nchunks + c) * 2 + 0]);
    tp += __ldcg(&a.W2[((int64_t)b * a.nchunks + c) * 2 + 1]);
  }
  tw = warp_sum(tw);
  tp = warp_sum(tp);
  if (lane == 0) a.send3[b] = TpSeq3{tw, tp};
}

// ------------------------------------------------------------ tensor parallelism
//
// Vocabulary shards (DistributedContext::shard_dim, src/distributed.rs:90-98):
// each rank runs the stats kernel on its own columns, then
//   accept_tp_part_kernel   row maxima, the normaliser parts under
//                           them, owner values at the drafts     -> all-gather 1
//   (greedy: accept_tp_max_kernel, row maxima and argmaxes        -> all-gather 1)
//   accept_tp_decide_kernel the decision, the same on every rank
//   accept_final_kernel<TP> this rank's weight totals            -> all-gather 2
//   accept_tp_search_kernel the owner rank finds the token      -> int32 max 3
//   accept_tp_write_kernel  every rank writes it
// Ranks contribute to sums through all-gathers and add the parts in rank
// order, so every rank computes the contract's rank-ordered sums.  Each
// rank's normaliser part is taken under its own row maximum and scaled to
// the row maximum by the receivers (kyro_math.h), which lets the maxima and
// the parts travel in one round.  On peer memory, round 1 is not a separate
// kernel: accept_tp_part_kernel stores its records straight into the peers'
// exchange regions and the decide kernel reads them in place.  Rounds 2
// and 3 stay exchange kernels: their producers are one unit per sequence
// inside the final pass and the search, and a system-scope fence per unit
// under that traffic measured 8 us slower per step on two ranks.

// Row max of stats row srow over this rank's chunks (one warp).
__device__ __forceinline__ float row_max(const Args& a, int64_t srow) {
  const int lane = threadIdx.x & 31;
  const ChunkStat* st = a.stats + srow * a.nchunks;
  float M = -INFINITY;
  for (int g = 0; g < a.nchunks; g += 256) {
    float mm[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = g + j * 32 + lane;
      mm[j] = c < a.nchunks ? st[c].m : -INFINITY;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) M = fmaxf(M, mm[j]);
  }
  return kyro::dev::warp_max(M);
}

// This rank's butterfly part of the normaliser of stats row srow under the
// global row max M (one warp; lane l adds chunks l, l+32, ... in order).
__device__ __forceinline__ double row_sum_part(const Args& a, int64_t srow, float M) {
  const int lane = threadIdx.x & 31;
  const ChunkStat* st = a.stats + srow * a.nchunks;
  double t = 0.0;
  for (int g = 0; g < a.nchunks; g += 256) {
    float mm[8], ee[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = g + j * 32 + lane;
      mm[j] = c < a.nchunks ? st[c].m : 0.0f;
      ee[j] = c < a.nchunks ? st[c].E : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (g + j * 32 + lane < a.nchunks) t = KY_DADD(t, ky_chunk_mass(ee[j], mm[j], M));
  }
  return warp_butterfly(t);
}

// Greedy: this rank's row maxima and argmaxes (one warp per row).
__global__ void __launch_bounds__(kDecideWarps * 32) accept_tp_max_kernel(Args a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int b = blockIdx.x;
  grid_dependency_wait();
  allow_dependents();
  for (int r = warp; r < a.R; r += nwarps) {
    const int64_t srow = (int64_t)b * a.R + r;
    const RowStat rs = row_stat(a, srow);
    TpRow1 v;
    v.M = rs.M;
    v.arg = (int32_t)(rs.arg + a.vocab_offset);
    if (lane == 0) a.send1[srow] = v;
  }
}

// Stochastic: this rank's row maxima, the normaliser parts under them, and
// the owner's values at the draft tokens, for round 1 (one warp per row).
//
// With a.xpush the records go straight into every peer's slot of this rank
// for the round (P2P stores over NVLink, spread over all of the grid's
// CTAs); the CTA that finishes last advances the round counter and raises
// this rank's flag in every peer's region.
__global__ void __launch_bounds__(kDecideWarps * 32) accept_tp_part_kernel(Args a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int b = blockIdx.x;
  __shared__ unsigned long long sh_seq;
  grid_dependency_wait();  // the chunk statistics are complete
  allow_dependents();
  uint8_t* own = a.xpush ? a.xpeers.p[a.tp_rank] : nullptr;
  if (a.xpush) {
    // every CTA reads the round number before the last one advances it
    if (threadIdx.x == 0)
      sh_seq = *reinterpret_cast<volatile unsigned long long*>(kyro::xchg::round_counter(own)) + 1ull;
    __syncthreads();
  }
  const unsigned long long seq = a.xpush ? sh_seq : 0ull;
  const size_t stride = kyro::xchg::slot_stride(sizeof(TpRow2) * (size_t)a.B * a.R);
  for (int r = warp; r < a.R; r += nwarps) {
    const int64_t srow = (int64_t)b * a.R + r;
    TpRow2 v;
    v.M = row_max(a, srow);
    v.S = row_sum_part(a, srow, v.M);
    v.ex = 0.0f;
    v.mcx = 0.0f;
    v._pad = 0;
    const int xg = draft_token_of_row(a, b, r);
    const int64_t xl = (int64_t)xg - a.vocab_offset;
    if (xg >= 0 && xg < a.V_global && xl >= 0 && xl < a.V) {
      v.ex = ld_ex(a, srow);
      v.mcx = a.stats[srow * a.nchunks + xl / kChunk].m;
    }
    if (lane == 0) {
      if (!a.xpush) {
        a.send2[srow] = v;
      } else {
        for (int q = 0; q < a.tp_world; ++q)
          if (a.xskip == 0 || q == a.tp_rank)
            reinterpret_cast<TpRow2*>(kyro::xchg::slot_of(a.xpeers.p[q], seq, a.tp_rank, stride))
                [srow] = v;
      }
    }
  }
  if (!a.xpush) return;
  __threadfence_system();  // this CTA's records are visible in the peers' memory
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* done = reinterpret_cast<uint32_t*>(own + kyro::xchg::kDoneOffset);
    if (atomicAdd(done, 1u) == gridDim.x - 1u) {
      *done = 0u;
      __threadfence();
      *reinterpret_cast<volatile unsigned long long*>(kyro::xchg::round_counter(own)) = seq;
      for (int q = 0; q < a.tp_world; ++q)
        if (a.xskip == 0 || q == a.tp_rank)
          kyro::xchg::st_release_sys(kyro::xchg::flag_of(a.xpeers.p[q], a.tp_rank, seq), seq);
    }
  }
}

// Round 1's records as this rank received them: rank q's record of stats row
// srow, from the exchange's receive buffer or (a.xpush) from rank q's slot in
// this rank's region, read from L2.  `base` is the round's slot 0 in the
// region (pushed rounds only).
__device__ __forceinline__ TpRow2 round1_row(const Args& a, const uint8_t* base, int q,
                                             int64_t srow) {
  const int64_t rows = (int64_t)a.B * a.R;
  if (!a.xpush) return a.recv2[q * rows + srow];
  const size_t stride = kyro::xchg::slot_stride(sizeof(TpRow2) * (size_t)rows);
  const unsigned long long* w =
      reinterpret_cast<const unsigned long long*>(base + (size_t)q * stride) + srow * 3;
  const unsigned long long w0 = __ldcg(w), w1 = __ldcg(w + 1), w2 = __ldcg(w + 2);
  TpRow2 v;
  v.S = __longlong_as_double((long long)w0);
  v.ex = __uint_as_float((uint32_t)w1);
  v.mcx = __uint_as_float((uint32_t)(w1 >> 32));
  v.M = __uint_as_float((uint32_t)w2);
  v._pad = (int32_t)(w2 >> 32);
  return v;
}

// A CTA that reads round 1: with a.xpush, thread 0 waits (bounded) for every
// rank's flag of the round and the CTA gets the round's slot 0 in this
// rank's region; else null (the receive buffer holds the round).
__device__ __forceinline__ const uint8_t* round1_base(const Args& a) {
  __shared__ const uint8_t* sh_base;
  if (!a.xpush) return nullptr;
  if (threadIdx.x == 0) {
    uint8_t* own = a.xpeers.p[a.tp_rank];
    const unsigned long long seq =
        *reinterpret_cast<volatile unsigned long long*>(kyro::xchg::round_counter(own));
    for (int q = 0; q < a.tp_world; ++q)
      if (!kyro::xchg::wait_flag(own, q, seq, a.xwait_ns)) {
        kyro::dev::flag(a.status, KYRO_DEV_WAIT_TIMEOUT);
        break;
      }
    sh_base = kyro::xchg::slot_of(own, seq, 0,
                                  kyro::xchg::slot_stride(sizeof(TpRow2) * (size_t)a.B * a.R));
  }
  __syncthreads();
  return sh_base;
}

// The row's statistics from every rank's round-1 part: M the largest shard
// maximum, S the parts brought to M and added in rank order (kyro_math.h).
__device__ __forceinline__ RowStat gathered_row_stat(const Args& a, const uint8_t* base,
                                                     int64_t srow) {
  RowStat v;
  v.arg = 0;
  v.M = -INFINITY;
  for (int q = 0; q < a.tp_world; ++q) v.M = fmaxf(v.M, round1_row(a, base, q, srow).M);
  v.S = 0.0;
  for (int q = 0; q < a.tp_world; ++q) {
    const TpRow2 r = round1_row(a, base, q, srow);
    v.S = KY_DADD(v.S, KY_DMUL(r.S, ky_shard_scale(r.M, v.M)));
  }
  return v;
}

__device__ __forceinline__ TestInputs tp_test(const Args& a, const uint8_t* base, int b, int j) {
  TestInputs t;
  t.x = -1;
  t.ep = t.eq = t.mp = t.mq = 0.0f;
  if (j >= a.k) return t;
  t.x = a.draft_tokens[(int64_t)b * a.k + j];
  if (a.stoch && t.x >= 0 && t.x < a.V_global) {
    const int owner = (int)(t.x / a.V);
    const TpRow2 pr = round1_row(a, base, owner, (int64_t)b * a.R + j);
    const TpRow2 qr = round1_row(a, base, owner, (int64_t)b * a.R + a.k + 1 + j);
    t.ep = pr.ex;
    t.mp = pr.mcx;
    t.eq = qr.ex;
    t.mq = qr.mcx;
  }
  return t;
}

// One CTA per sequence: global row statistics from the exchanged parts,
// then the same decision as accept_decide_kernel.
__global__ void __launch_bounds__(kDecideWarps * 32) accept_tp_decide_kernel(Args a) {
  __shared__ RowStat rs[kMaxRows];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.x;
  const int64_t rows = (int64_t)a.B * a.R;
  grid_dependency_wait();  // round 1 has landed, or (pushed) its producer is done
  allow_dependents();
  const uint8_t* base = a.stoch ? round1_base(a) : nullptr;
  if (threadIdx.x == 0) a.cnt_c[b] = 0;
  for (int r = threadIdx.x; r < a.R; r += blockDim.x) {
    const int64_t srow = (int64_t)b * a.R + r;
    RowStat v;
    v.S = 0.0;
    v.arg = 0;
    if (a.stoch) {
      v = gathered_row_stat(a, base, srow);
    } else {
      // shards are contiguous: the first strict maximum in rank order is the
      // lowest global index among equal maxima
      v.M = a.recv1[srow].M;
      v.arg = a.recv1[srow].arg;
      for (int q = 1; q < a.tp_world; ++q) {
        const TpRow1 o = a.recv1[q * rows + srow];
        if (o.M > v.M) {
          v.M = o.M;
          v.arg = o.arg;
        }
      }
    }
    rs[r] = v;
  }
  __syncthreads();
  if (warp != 0) return;
  const TestInputs t0 = tp_test(a, base, b, lane), t1 = tp_test(a, base, b, lane + 32);
  decide_sequence(a, b, rs, t0, t1);
}

// One warp per sequence: the global threshold from the exchanged totals;
// the rank whose columns hold it finds the token, the others offer -1.
template <bool VEC>
__global__ void __launch_bounds__(kThreads) accept_tp_search_kernel(Args a) {
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.x * kWarps + (threadIdx.x >> 5);
  grid_dependency_wait();  // round 2 has landed
  allow_dependents();
  if (b >= a.B) return;
  const FinalRow fr = a.final_rows[b];
  int token = -1;
  if (!fr.skip) {
    unsigned long long tot_w = 0, tot_p = 0;
    for (int q = 0; q < a.tp_world; ++q) {
      tot_w += a.recv3[(int64_t)q * a.B + b].w_res;
      tot_p += a.recv3[(int64_t)q * a.B + b].w_p;
    }
    // the residual, or p when there is none (bonus) or it has no mass
    const bool residual = fr.q_row >= 0 && tot_w != 0;
    const unsigned long long tot = residual ? tot_w : tot_p;
    if (tot == 0) {
      if (a.tp_rank == a.tp_world - 1) token = (int)(a.V_global - 1);
    } else {
      const unsigned long long T = ky_cdf_threshold(fr.odd, tot);
      unsigned long long before = 0;
      for (int q = 0; q < a.tp_rank; ++q) {
        const TpSeq3 v = a.recv3[(int64_t)q * a.B + b];
        before += residual ? v.w_res : v.w_p;
      }
      const TpSeq3 mine = a.recv3[(int64_t)a.tp_rank * a.B + b];
      const unsigned long long m = residual ? mine.w_res : mine.w_p;
      if (T > before && T - before <= m) {
        const int local = cut_index<VEC>(a, fr, residual,
                                         a.W2 + (int64_t)b * a.nchunks * 2 + (residual ? 0 : 1), 2,
                                         T - before);
        if (local >= 0) token = (int)(local + a.vocab_offset);
      }
    }
  }
  if (lane == 0) a.send4[b] = token;
}

__global__ void accept_tp_write_kernel(Args a) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  grid_dependency_wait();  // round 3 has landed
  allow_dependents();
  if (b >= a.B) return;
  const FinalRow fr = a.final_rows[b];
  if (!fr.skip) a.out_tokens[fr.out_index] = a.recv4[b];
}

// ------------------------------------------------------------ tree verification
//
// Multi-candidate rejection sampling over a BFS-ordered draft tree
// (SpecInfer), as kyro_math.h states it: one CTA walks one sequence's tree.
// Every node row's chunk statistics come from the stats kernel; a rejection
// costs one CTA-wide pass over the node's target and draft rows that sums
// R_j in the contract's tree (warps own chunks, warp 0 combines them), and
// the final draw sums integer weights per chunk and scans one chunk.

constexpr int kTreeThreads = 1024;
constexpr int kTreeWarps = kTreeThreads / 32;
constexpr int kMaxNodes = 64;

struct TreeShared {
  float mP[kMaxChunks], gP[kMaxChunks], mQ[kMaxChunks], gQ[kMaxChunks];
  double csum[kMaxChunks];  // chunk sums of R_j, or (as u64) of the weights
  double R[kMaxNodes];
  int ch[kMaxNodes];
  int nch, node, accepted, token, done;
};

// The contract's p_i and q_i of 4 entries at e0 (fp32, then widened), and
// p_nr after nr residual steps; entries past V are marked invalid.
template <bool VEC>
__device__ __forceinline__ void tree_values4(const Args& a, const TreeShared& sh,
                                             const float* prow, const float* qrow, int c,
                                             int64_t e0, int nr, double (&pd)[4],
                                             double (&qd)[4], bool (&ok)[4]) {
  const float4 zp = load4<VEC>(prow, e0, a.V);
  const float4 zq = load4<VEC>(qrow, e0, a.V);
  const float p4[4] = {zp.x, zp.y, zp.z, zp.w};
  const float q4[4] = {zq.x, zq.y, zq.z, zq.w};
  const f2_t mm = f2_pack(sh.mP[c], sh.mQ[c]);
  const f2_t gg = f2_pack(sh.gP[c], sh.gQ[c]);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f2_t z = f2_pack(p4[j], q4[j]);
    if (a.inv_t != 1.0f) z = f2_mul(z, f2_pack(a.inv_t, a.inv_t));
    float pf, qf;
    f2_unpack(f2_mul(exp_pair(f2_sub(z, mm)), gg), pf, qf);
    ok[j] = e0 + j < a.V;
    qd[j] = (double)qf;
    double v = (double)pf;
    for (int r = 0; r < nr; ++r) v = ky_tree_step(v, qd[j], sh.R[r]);
    pd[j] = v;
  }
}

template <bool VEC, bool STOCH>
__global__ void __launch_bounds__(kTreeThreads) accept_tree_kernel(Args a) {
  __shared__ TreeShared sh;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.x;
  const int N = a.k + 1;
  const int nc = a.nchunks;
  const uint32_t seq = (uint32_t)(a.seq_offset + b);
  const int32_t* tok = a.node_tokens + (int64_t)b * N;
  const int32_t* par = a.parents + (int64_t)b * N;
  grid_dependency_wait();  // the chunk statistics are complete
  for (int n = threadIdx.x; n < N; n += kTreeThreads) {
    a.out_path[(int64_t)b * N + n] = -1;
    a.out_tokens[(int64_t)b * N + n] = -1;
  }
  int plen = 1, ntok = 0;  // thread 0's counts
  if (threadIdx.x == 0) {
    sh.node = 0;
    sh.done = 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) a.out_path[(int64_t)b * N] = 0;
  while (!sh.done) {
    const int node = sh.node;
    if (threadIdx.x == 0) {
      int m = 0;
      for (int c = node + 1; c < N; ++c)
        if (par[c] == node) sh.ch[m++] = c;
      sh.nch = m;
      sh.accepted = -1;
    }
    if (!STOCH) {
      if (warp == 0) {
        const RowStat rs = row_stat(a, (int64_t)b * a.R + node);
        if (lane == 0) sh.token = rs.arg;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        for (int i = 0; i < sh.nch && sh.accepted < 0; ++i)
          if (tok[sh.ch[i]] == sh.token) sh.accepted = sh.ch[i];
      }
      __syncthreads();
    } else {
      // row statistics of the node's target (warp 0) and draft (warp 1) rows
      if (warp < 2) {
        const RowStat rs = row_stat(a, (int64_t)b * a.R + (warp == 0 ? node : N + node));
        if (lane == 0) {
          if (warp == 0) {
            sh.R[kMaxNodes - 1] = rs.S;  // parked until the chunk factors are made
            sh.mP[0] = rs.M;
          } else {
            sh.csum[0] = rs.S;
            sh.mQ[0] = rs.M;
          }
        }
      }
      __syncthreads();
      const float Mp = sh.mP[0], Mq = sh.mQ[0];
      const double Sp = sh.R[kMaxNodes - 1], Sq = sh.csum[0];
      __syncthreads();
      const ChunkStat* stp = a.stats + ((int64_t)b * a.R + node) * nc;
      const ChunkStat* stq = a.stats + ((int64_t)b * a.R + N + node) * nc;
      for (int c = threadIdx.x; c < nc; c += kTreeThreads) {
        const float mp = stp[c].m, mq = stq[c].m;
        sh.mP[c] = mp;
        sh.gP[c] = ky_chunk_scale(mp, Mp, Sp);
        sh.mQ[c] = mq;
        sh.gQ[c] = ky_chunk_scale(mq, Mq, Sq);
      }
      __syncthreads();
      const float* prow = stats_row_ptr(a, b, node);
      const float* qrow = stats_row_ptr(a, b, N + node);
      int nr = 0;
      for (int i = 0; i < sh.nch; ++i) {
        const int c = sh.ch[i];
        if (threadIdx.x == 0) {
          const int x = tok[c];
          if (x >= 0 && x < a.V) {
            const int cx = x / kChunk;
            float sp = prow[x], sq = qrow[x];
            if (a.inv_t != 1.0f) {
              sp = KY_FMUL(sp, a.inv_t);
              sq = KY_FMUL(sq, a.inv_t);
            }
            const double qx = (double)KY_FMUL(exp_fast(KY_FSUB(sq, sh.mQ[cx])), sh.gQ[cx]);
            double px = (double)KY_FMUL(exp_fast(KY_FSUB(sp, sh.mP[cx])), sh.gP[cx]);
            for (int r = 0; r < nr; ++r) px = ky_tree_step(px, qx, sh.R[r]);
            const double u =
                (double)ky_odd_to_float(ky_uniform_odd(a.seed, seq, (uint32_t)c, KY_STREAM_ACCEPT,
                                                       a.step));
            if (u < KY_DDIV(px, qx)) sh.accepted = c;
          } else {
            kyro::dev::flag(a.status, KYRO_DEV_BAD_TOKEN);
          }
        }
        __syncthreads();
        if (sh.accepted >= 0) break;
        // rejected: R_nr over the vocabulary in the contract's tree
        for (int cc = warp; cc < nc; cc += kTreeWarps) {
          double acc[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
          for (int g = 0; g < kVec; ++g) {
            double pd[4], qd[4];
            bool ok[4];
            tree_values4<VEC>(a, sh, prow, qrow, cc,
                              (int64_t)cc * kChunk + (g * 32 + lane) * 4, nr, pd, qd, ok);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              acc[j] = KY_DADD(acc[j], ok[j] ? ky_tree_excess(pd[j], qd[j]) : 0.0);
          }
          const double t =
              warp_butterfly(KY_DADD(KY_DADD(acc[0], acc[1]), KY_DADD(acc[2], acc[3])));
          if (lane == 0) sh.csum[cc] = t;
        }
        __syncthreads();
        if (warp == 0) {
          double t = 0.0;
          for (int cc = lane; cc < nc; cc += 32) t = KY_DADD(t, sh.csum[cc]);
          t = warp_butterfly(t);
          if (lane == 0) sh.R[nr] = t;
        }
        __syncthreads();
        ++nr;
      }
      if (sh.accepted < 0) {
        // draw from p_nr: integer weights, chunk sums, then one chunk's scan
        unsigned long long* wsum = reinterpret_cast<unsigned long long*>(sh.csum);
        for (int cc = warp; cc < nc; cc += kTreeWarps) {
          unsigned long long t = 0;
#pragma unroll
          for (int g = 0; g < kVec; ++g) {
            double pd[4], qd[4];
            bool ok[4];
            tree_values4<VEC>(a, sh, prow, qrow, cc,
                              (int64_t)cc * kChunk + (g * 32 + lane) * 4, nr, pd, qd, ok);
#pragma unroll
            for (int j = 0; j < 4; ++j) t += ok[j] ? ky_weight_d(pd[j]) : 0ull;
          }
          t = warp_sum(t);
          if (lane == 0) wsum[cc] = t;
        }
        __syncthreads();
        if (warp == 0) {
          unsigned long long tot = 0;
          for (int cc = lane; cc < nc; cc += 32) tot += wsum[cc];
          tot = warp_sum(tot);
          int token = (int)a.V - 1;
          if (tot != 0) {
            unsigned long long T = ky_cdf_threshold(
                ky_uniform_odd(a.seed, seq, (uint32_t)node, KY_STREAM_RESAMPLE, a.step), tot);
            int sub = -1;
            unsigned long long base = 0;
            for (int s0 = 0; s0 < nc && sub < 0; s0 += 32) {
              const unsigned long long ws = s0 + lane < nc ? wsum[s0 + lane] : 0ull;
              const unsigned long long inc = base + warp_inclusive(ws);
              const unsigned hit = __ballot_sync(0xffffffffu, inc >= T && s0 + lane < nc);
              if (hit) {
                const int l = __ffs(hit) - 1;
                sub = s0 + l;
                T -= __shfl_sync(0xffffffffu, inc - ws, l);
              } else {
                base = __shfl_sync(0xffffffffu, inc, 31);
              }
            }
            if (sub >= 0) {
              unsigned long long cbase = 0;
              int found = -1;
              for (int g = 0; g < kVec; ++g) {
                double pd[4], qd[4];
                bool ok[4];
                tree_values4<VEC>(a, sh, prow, qrow, sub,
                                  (int64_t)sub * kChunk + (g * 32 + lane) * 4, nr, pd, qd, ok);
                unsigned long long w[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) w[j] = ok[j] ? ky_weight_d(pd[j]) : 0ull;
                const unsigned long long s4 = (w[0] + w[1]) + (w[2] + w[3]);
                const unsigned long long inc = warp_inclusive(s4);
                unsigned long long C = cbase + inc - s4;
                int mine = -1;
                if (C < T && C + s4 >= T) {
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    C += w[j];
                    if (mine < 0 && C >= T) mine = j;
                  }
                }
                const unsigned hit = __ballot_sync(0xffffffffu, mine >= 0);
                if (found < 0 && hit) {
                  const int l = __ffs(hit) - 1;
                  found = sub * kChunk + (g * 32 + l) * 4 + __shfl_sync(0xffffffffu, mine, l);
                }
                cbase += __shfl_sync(0xffffffffu, inc, 31);
              }
              if (found >= 0) token = found;
            }
          }
          if (lane == 0) sh.token = token;
        }
        __syncthreads();
      }
    }
    if (threadIdx.x == 0) {
      const int c = sh.accepted;
      if (c >= 0) {
        a.out_path[(int64_t)b * N + plen++] = c;
        a.out_tokens[(int64_t)b * N + ntok++] = tok[c];
        sh.node = c;
      } else {
        a.out_tokens[(int64_t)b * N + ntok++] = sh.token;
        sh.done = 1;
        a.out_path_len[b] = plen;
        a.out_num_tokens[b] = ntok;
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------ clustered tree walk
//
// The stochastic walk of accept_tree_kernel on a cluster of kTreeC CTAs per
// sequence.  CTA `rank` owns chunks [rank * cpc, rank * cpc + cpc) of the
// vocabulary and keeps their p (fp64, the current residual p_nr) and q (fp32,
// exact in fp64) in shared memory, so a residual step costs one division per
// entry instead of the whole chain from p_0.  Every CTA takes the same
// decisions from the same inputs in the same order (row statistics, child
// tests, thresholds); per-chunk sums cross the cluster through distributed
// shared memory (double-buffered, one cluster barrier per exchange) and each
// CTA adds them in the contract's order (chunks l, l+32, ... into lane l,
// then the butterfly), so all ranks hold bit-identical R_j.  Rank 0 writes
// the path, the CTA owning the drawn token's chunk writes that token.

constexpr int kTreeCMaxChunks = 32;  // chunks per CTA (one warp each)

__device__ __forceinline__ uint32_t tc_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t tc_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void tc_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}
// A 64-bit word of CTA `rank`'s shared memory at this CTA's offset `local`.
__device__ __forceinline__ unsigned long long tc_ld_remote(const void* local, uint32_t rank) {
  uint32_t la = (uint32_t)__cvta_generic_to_shared(local), ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(la), "r"(rank));
  unsigned long long v;
  asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(ra) : "memory");
  return v;
}

struct TreeClusterShared {
  float mP[kTreeCMaxChunks], gP[kTreeCMaxChunks], mQ[kTreeCMaxChunks], gQ[kTreeCMaxChunks];
  unsigned long long xsum[2][kTreeCMaxChunks];  // exchanged chunk sums (f64 bits or u64)
  double R[kMaxNodes];
  int ch[kMaxNodes];
  float Mp, Mq;
  double Sp, Sq;
  int nch, node, accepted, token, done, sub;
  unsigned long long T;
};

template <bool VEC>
__global__ void __launch_bounds__(kTreeThreads) accept_tree_cluster_kernel(Args a, int cpc) {
  extern __shared__ __align__(16) uint8_t tree_smem[];
  TreeClusterShared& sh = *reinterpret_cast<TreeClusterShared*>(tree_smem);
  double* pv = reinterpret_cast<double*>(tree_smem + ((sizeof(TreeClusterShared) + 15) & ~size_t(15)));
  float* qv = reinterpret_cast<float*>(pv + (size_t)cpc * kChunk);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t rank = tc_rank(), C = tc_size();
  const int b = (int)(blockIdx.x / C);
  const int N = a.k + 1;
  const int nc = a.nchunks;
  const int c0 = (int)rank * cpc;
  const int ncc = max(0, min(nc, c0 + cpc) - c0);  // chunks of this CTA
  const uint32_t seq = (uint32_t)(a.seq_offset + b);
  const int32_t* tok = a.node_tokens + (int64_t)b * N;
  const int32_t* par = a.parents + (int64_t)b * N;
  grid_dependency_wait();  // the chunk statistics are complete
  if (rank == 0)
    for (int n = threadIdx.x; n < N; n += kTreeThreads) {
      a.out_path[(int64_t)b * N + n] = -1;
      a.out_tokens[(int64_t)b * N + n] = -1;
    }
  int plen = 1, ntok = 0, xbuf = 0;  // thread 0's counts; the exchange buffer (uniform)
  if (threadIdx.x == 0) {
    sh.node = 0;
    sh.done = 0;
  }
  __syncthreads();
  if (rank == 0 && threadIdx.x == 0) a.out_path[(int64_t)b * N] = 0;
  // sums of all chunks from their owners, in the contract's lane order
  auto gather_f64 = [&](int buf) -> double {
    double t = 0.0;
    for (int cc = lane; cc < nc; cc += 32)
      t = KY_DADD(t, __longlong_as_double((long long)tc_ld_remote(&sh.xsum[buf][cc % cpc],
                                                                   (uint32_t)(cc / cpc))));
    return warp_butterfly(t);
  };
  // a path visits at most N nodes; every CTA of the cluster takes the same
  // number of steps
  for (int walk = 0; walk <= N && !sh.done; ++walk) {
    const int node = sh.node;
    if (threadIdx.x == 0) {
      int m = 0;
      for (int c = node + 1; c < N; ++c)
        if (par[c] == node) sh.ch[m++] = c;
      sh.nch = m;
      sh.accepted = -1;
    }
    // row statistics of the node's target (warp 0) and draft (warp 1) rows
    if (warp < 2) {
      const RowStat rs = row_stat(a, (int64_t)b * a.R + (warp == 0 ? node : N + node));
      if (lane == 0) {
        if (warp == 0) {
          sh.Mp = rs.M;
          sh.Sp = rs.S;
        } else {
          sh.Mq = rs.M;
          sh.Sq = rs.S;
        }
      }
    }
    __syncthreads();
    const ChunkStat* stp = a.stats + ((int64_t)b * a.R + node) * nc;
    const ChunkStat* stq = a.stats + ((int64_t)b * a.R + N + node) * nc;
    if ((int)threadIdx.x < ncc) {
      const int c = c0 + threadIdx.x;
      const float mp = stp[c].m, mq = stq[c].m;
      sh.mP[threadIdx.x] = mp;
      sh.gP[threadIdx.x] = ky_chunk_scale(mp, sh.Mp, sh.Sp);
      sh.mQ[threadIdx.x] = mq;
      sh.gQ[threadIdx.x] = ky_chunk_scale(mq, sh.Mq, sh.Sq);
    }
    __syncthreads();
    const float* prow = stats_row_ptr(a, b, node);
    const float* qrow = stats_row_ptr(a, b, N + node);
    // p_0 and q of this CTA's entries (entries past V hold 0, which adds 0
    // to every sum below)
    if (warp < ncc) {
      const int cc = c0 + warp;
      const f2_t mm = f2_pack(sh.mP[warp], sh.mQ[warp]);
      const f2_t gg = f2_pack(sh.gP[warp], sh.gQ[warp]);
#pragma unroll
      for (int g = 0; g < kVec; ++g) {
        const int64_t e0 = (int64_t)cc * kChunk + (g * 32 + lane) * 4;
        const float4 zp = load4<VEC>(prow, e0, a.V);
        const float4 zq = load4<VEC>(qrow, e0, a.V);
        const float p4[4] = {zp.x, zp.y, zp.z, zp.w};
        const float q4[4] = {zq.x, zq.y, zq.z, zq.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          f2_t z = f2_pack(p4[j], q4[j]);
          if (a.inv_t != 1.0f) z = f2_mul(z, f2_pack(a.inv_t, a.inv_t));
          float pf, qf;
          f2_unpack(f2_mul(exp_pair(f2_sub(z, mm)), gg), pf, qf);
          const bool ok = e0 + j < a.V;
          const int idx = warp * kChunk + (g * 32 + lane) * 4 + j;
          pv[idx] = ok ? (double)pf : 0.0;
          qv[idx] = ok ? qf : 0.0f;
        }
      }
    }
    __syncthreads();
    int nr = 0;
    for (int i = 0; i < sh.nch; ++i) {
      const int c = sh.ch[i];
      if (threadIdx.x == 0) {
        const int x = tok[c];
        if (x >= 0 && x < a.V) {
          const int cx = x / kChunk;
          const float mpx = stp[cx].m, mqx = stq[cx].m;
          float sp = prow[x], sq = qrow[x];
          if (a.inv_t != 1.0f) {
            sp = KY_FMUL(sp, a.inv_t);
            sq = KY_FMUL(sq, a.inv_t);
          }
          const double qx =
              (double)KY_FMUL(exp_fast(KY_FSUB(sq, mqx)), ky_chunk_scale(mqx, sh.Mq, sh.Sq));
          double px =
              (double)KY_FMUL(exp_fast(KY_FSUB(sp, mpx)), ky_chunk_scale(mpx, sh.Mp, sh.Sp));
          for (int r = 0; r < nr; ++r) px = ky_tree_step(px, qx, sh.R[r]);
          const double u =
              (double)ky_odd_to_float(ky_uniform_odd(a.seed, seq, (uint32_t)c, KY_STREAM_ACCEPT,
                                                     a.step));
          if (u < KY_DDIV(px, qx)) sh.accepted = c;
        } else if (rank == 0) {
          kyro::dev::flag(a.status, KYRO_DEV_BAD_TOKEN);
        }
      }
      __syncthreads();
      if (sh.accepted >= 0) break;
      // rejected: p_nr from the stored p_{nr-1}, then R_nr = sum max(p_nr - q, 0)
      if (warp < ncc) {
        double acc[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
        for (int g = 0; g < kVec; ++g)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int idx = warp * kChunk + (g * 32 + lane) * 4 + j;
            double p = pv[idx];
            const double q = (double)qv[idx];
            if (nr > 0) {
              p = ky_tree_step(p, q, sh.R[nr - 1]);
              pv[idx] = p;
            }
            acc[j] = KY_DADD(acc[j], ky_tree_excess(p, q));
          }
        const double t = warp_butterfly(KY_DADD(KY_DADD(acc[0], acc[1]), KY_DADD(acc[2], acc[3])));
        if (lane == 0) sh.xsum[xbuf][warp] = (unsigned long long)__double_as_longlong(t);
      }
      tc_cluster_sync();
      if (warp == 0) {
        const double t = gather_f64(xbuf);
        if (lane == 0) sh.R[nr] = t;
      }
      xbuf ^= 1;
      __syncthreads();
      ++nr;
    }
    if (sh.accepted < 0) {
      // draw from p_nr: integer weights, chunk sums, then one chunk's scan
      if (warp < ncc) {
        unsigned long long t = 0;
#pragma unroll
        for (int g = 0; g < kVec; ++g)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int idx = warp * kChunk + (g * 32 + lane) * 4 + j;
            double p = pv[idx];
            if (nr > 0) {
              p = ky_tree_step(p, (double)qv[idx], sh.R[nr - 1]);
              pv[idx] = p;
            }
            t += ky_weight_d(p);
          }
        t = warp_sum(t);
        if (lane == 0) sh.xsum[xbuf][warp] = t;
      }
      tc_cluster_sync();
      if (warp == 0) {
        unsigned long long tot = 0;
        for (int cc = lane; cc < nc; cc += 32)
          tot += tc_ld_remote(&sh.xsum[xbuf][cc % cpc], (uint32_t)(cc / cpc));
        tot = warp_sum(tot);
        int sub = -1;
        unsigned long long T = 0;
        if (tot != 0) {
          T = ky_cdf_threshold(
              ky_uniform_odd(a.seed, seq, (uint32_t)node, KY_STREAM_RESAMPLE, a.step), tot);
          unsigned long long base = 0;
          for (int s0 = 0; s0 < nc && sub < 0; s0 += 32) {
            const unsigned long long ws =
                s0 + lane < nc ? tc_ld_remote(&sh.xsum[xbuf][(s0 + lane) % cpc],
                                              (uint32_t)((s0 + lane) / cpc))
                               : 0ull;
            const unsigned long long inc = base + warp_inclusive(ws);
            const unsigned hit = __ballot_sync(0xffffffffu, inc >= T && s0 + lane < nc);
            if (hit) {
              const int l = __ffs(hit) - 1;
              sub = s0 + l;
              T -= __shfl_sync(0xffffffffu, inc - ws, l);
            } else {
              base = __shfl_sync(0xffffffffu, inc, 31);
            }
          }
        }
        if (lane == 0) {
          sh.sub = sub;
          sh.T = T;
        }
      }
      __syncthreads();
      // the token: in the cut chunk by its owner, V - 1 when p_nr has no mass
      const int sub = sh.sub;
      const uint32_t owner = sub >= 0 ? (uint32_t)(sub / cpc) : 0u;
      if (warp == 0 && rank == owner) {
        int token = (int)a.V - 1;
        if (sub >= 0) {
          const unsigned long long T = sh.T;
          const int w = sub - c0;
          unsigned long long cbase = 0;
          int found = -1;
          for (int g = 0; g < kVec; ++g) {
            unsigned long long wj[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
              wj[j] = ky_weight_d(pv[w * kChunk + (g * 32 + lane) * 4 + j]);
            const unsigned long long s4 = (wj[0] + wj[1]) + (wj[2] + wj[3]);
            const unsigned long long inc = warp_inclusive(s4);
            unsigned long long Cc = cbase + inc - s4;
            int mine = -1;
            if (Cc < T && Cc + s4 >= T) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                Cc += wj[j];
                if (mine < 0 && Cc >= T) mine = j;
              }
            }
            const unsigned hit = __ballot_sync(0xffffffffu, mine >= 0);
            if (found < 0 && hit) {
              const int l = __ffs(hit) - 1;
              found = sub * kChunk + (g * 32 + l) * 4 + __shfl_sync(0xffffffffu, mine, l);
            }
            cbase += __shfl_sync(0xffffffffu, inc, 31);
          }
          if (found >= 0) token = found;
        }
        if (lane == 0) a.out_tokens[(int64_t)b * N + ntok] = token;
      }
      xbuf ^= 1;
    }
    if (threadIdx.x == 0) {
      const int c = sh.accepted;
      if (c >= 0) {
        if (rank == 0) {
          a.out_path[(int64_t)b * N + plen] = c;
          a.out_tokens[(int64_t)b * N + ntok] = tok[c];
        }
        ++plen;
        ++ntok;
        sh.node = c;
      } else {
        ++ntok;
        sh.done = 1;
        if (rank == 0) {
          a.out_path_len[b] = plen;
          a.out_num_tokens[b] = ntok;
        }
      }
    }
    __syncthreads();
  }
  // no CTA leaves while another may still read its shared memory
  tc_cluster_sync();
}

// ------------------------------------------------------------ host side

bool use_vec(const void* a, const void* b, int64_t V) {
  return (V % 4 == 0) && ((uintptr_t)a % 16 == 0) && (b == nullptr || (uintptr_t)b % 16 == 0);
}

// CTAs a stats launch needs: one warp per batch of kGrab units (more warps
// would only find the counter exhausted); capped by the resident count.
long long stats_ctas_needed(uint32_t units) {
  const long long per_cta = (long long)kGrab * kWarps;
  return ((long long)units + per_cta - 1) / per_cta;
}

template <bool VEC, bool STOCH>
int resident_ctas(int num_sms) {
  // one occupancy query per kernel (not repeated inside a graph capture)
  static int per_sm = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, accept_stats_kernel<VEC, STOCH>,
                                                      kThreads, 0) != cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
  });
  return num_sms * per_sm;
}

// Launch a kernel that may begin while its predecessor on the stream drains
// (it calls grid_dependency_wait before it reads the predecessor's output).
template <typename Kernel>
int launch_dependent(Kernel kernel, unsigned grid, unsigned block, cudaStream_t stream,
                     const Args& a, const char* name) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, a);
  if (err != cudaSuccess) return kyro::cuda_error(err, name);
  return KYRO_OK;
}

// The clustered tree walk: clusters of 4 CTAs (up to 64 chunks) or 8 (up to
// 256), each CTA holding its chunks' p and q in shared memory.  Returns
// false when the vocabulary is too large for it.
template <bool VEC>
bool launch_tree_cluster(int B, const Args& a, cudaStream_t stream, int* rc) {
  const int nc = a.nchunks;
  if (nc > 8 * kTreeCMaxChunks) return false;
  const int C = nc <= 4 * 16 ? 4 : 8;
  const int cpc = (nc + C - 1) / C;
  const size_t smem = ((sizeof(TreeClusterShared) + 15) & ~size_t(15)) +
                      (size_t)cpc * kChunk * (sizeof(double) + sizeof(float));
  static std::once_flag once;  // one host call per kernel, never inside a graph capture
  std::call_once(once, [] {
    cudaFuncSetAttribute(accept_tree_cluster_kernel<VEC>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(B * C));
  cfg.blockDim = dim3(kTreeThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, accept_tree_cluster_kernel<VEC>, a, cpc);
  *rc = err == cudaSuccess ? KYRO_OK : kyro::cuda_error(err, "accept_tree_cluster_kernel");
  return true;
}

// Every stats launch distributes its units dynamically, through the counter
// at the start of the workspace.  Each call leaves it at zero; a context
// zeroes it the first time it sees a workspace (it remembers the last few).
int use_unit_counter(kyro_ctx* ctx, Args& a, const Workspace& ws, const void* base) {
  a.unit_ctr = ws.unit_ctr;
  for (int i = 0; i < KYRO_ZEROED_WS; ++i)
    if (ctx->stats_ws_zeroed[i] == base) return KYRO_OK;
  const cudaError_t err = cudaMemsetAsync(ws.unit_ctr, 0, 8, ctx->stream);
  if (err != cudaSuccess) return kyro::cuda_error(err, "cudaMemsetAsync(stats unit counter)");
  ctx->stats_ws_zeroed[ctx->stats_ws_next] = base;
  ctx->stats_ws_next = (ctx->stats_ws_next + 1) % KYRO_ZEROED_WS;
  return KYRO_OK;
}

// The KV commit (and next reserve) that kyro_spec_accept_commit runs inside
// the acceptance, right after the decide kernel.
struct CommitSpec {
  const kyro_kv_params* kv;
  int32_t num_new, num_new_next;
  int64_t* block_table;
  int64_t* context_lens;
  int32_t *free_stack, *free_top, *ref_counts, *out_ok;
};

template <bool VEC, bool STOCH>
int launch_t(kyro_ctx* ctx, const Args& a, const CommitSpec* commit) {
  const long long need = stats_ctas_needed(a.units);
  const int resident = resident_ctas<VEC, STOCH>(ctx->num_sms);
  const int grid = (int)(need < resident ? need : resident);
  // launched plainly: a persistent grid launched early would take SM slots
  // in a long predecessor's last wave (measured 5 us slower behind attention)
  accept_stats_kernel<VEC, STOCH><<<grid, kThreads, 0, ctx->stream>>>(a);
  KY_TRY(kyro::check_launch("accept_stats_kernel"));
  const int dwarps = min(a.R + (a.sample ? 0 : 1), kDecideWarps);
  KY_TRY(launch_dependent(accept_decide_kernel, (unsigned)a.B, (unsigned)dwarps * 32, ctx->stream,
                          a, "accept_decide_kernel"));
  // the commit needs only the accept lengths: it waits for the decide kernel
  // and runs beside the final pass (which waits for its flags, not for it)
  if (commit)
    KY_TRY(kyro::kv::launch_commit_reserve(ctx, commit->kv, commit->num_new, commit->num_new_next,
                                           a.out_accept_len, commit->block_table,
                                           commit->context_lens, commit->free_stack,
                                           commit->free_top, commit->ref_counts, commit->out_ok));
  if (!STOCH) return KYRO_OK;  // greedy: the decide step wrote every token
  const unsigned nfinal = (unsigned)a.B * (unsigned)((a.nchunks + kFinalPerCta - 1) / kFinalPerCta);
  return launch_dependent(accept_final_kernel<VEC, false>, nfinal, kThreads, ctx->stream, a,
                          "accept_final_kernel");
}

int launch(kyro_ctx* ctx, Args& a, const Workspace& ws, bool vec,
           const CommitSpec* commit = nullptr) {
  (void)ws;
  if (vec && a.stoch) return launch_t<true, true>(ctx, a, commit);
  if (vec) return launch_t<true, false>(ctx, a, commit);
  if (a.stoch) return launch_t<false, true>(ctx, a, commit);
  return launch_t<false, false>(ctx, a, commit);
}

// The tensor-parallel sequence (kernels and collectives on the context's
// stream; every rank issues the same collectives in the same order).
template <bool VEC, bool STOCH>
int launch_tp(kyro_ctx* ctx, const Args& a_in) {
  Args a = a_in;
  const int64_t rows = (int64_t)a.B * a.R;
  // round 1 (stochastic) goes straight into the peers' regions when the
  // context's exchange is on peer memory
  a.xpush = 0;
  if (STOCH && kyro::xchg::push_round(ctx, sizeof(TpRow2) * (size_t)rows, &a.xpeers, &a.xskip)) {
    a.xpush = 1;
    a.xwait_ns = (unsigned long long)ctx->wait_ns;
  }
  const long long need = stats_ctas_needed(a.units);
  const int resident = resident_ctas<VEC, STOCH>(ctx->num_sms);
  const int grid = (int)(need < resident ? need : resident);
  accept_stats_kernel<VEC, STOCH><<<grid, kThreads, 0, ctx->stream>>>(a);
  KY_TRY(kyro::check_launch("accept_stats_kernel"));
  const unsigned dthreads = 32u * (unsigned)(a.R < kDecideWarps ? a.R : kDecideWarps);
  if (STOCH) {
    KY_TRY(launch_dependent(accept_tp_part_kernel, (unsigned)a.B, dthreads, ctx->stream, a,
                            "accept_tp_part_kernel"));
    if (!a.xpush)
      KY_TRY(kyro::xchg::all_gather(ctx, a.send2, a.recv2, sizeof(TpRow2) * rows,
                                    "kyro_spec_accept_tp: row maxima and normaliser parts"));
  } else {
    KY_TRY(launch_dependent(accept_tp_max_kernel, (unsigned)a.B, dthreads, ctx->stream, a,
                            "accept_tp_max_kernel"));
    KY_TRY(kyro::xchg::all_gather(ctx, a.send1, a.recv1, sizeof(TpRow1) * rows,
                                  "kyro_spec_accept_tp: row maxima"));
  }
  KY_TRY(launch_dependent(accept_tp_decide_kernel, (unsigned)a.B, dthreads, ctx->stream, a,
                          "accept_tp_decide_kernel"));
  if (!STOCH) return KYRO_OK;  // greedy: the decide step wrote every token
  const unsigned nfinal = (unsigned)a.B * (unsigned)((a.nchunks + kFinalPerCta - 1) / kFinalPerCta);
  KY_TRY(launch_dependent(accept_final_kernel<VEC, true>, nfinal, kThreads, ctx->stream, a,
                          "accept_final_kernel"));
  KY_TRY(kyro::xchg::all_gather(ctx, a.send3, a.recv3, sizeof(TpSeq3) * (size_t)a.B,
                                "kyro_spec_accept_tp: weight totals"));
  KY_TRY(launch_dependent(accept_tp_search_kernel<VEC>, (unsigned)((a.B + kWarps - 1) / kWarps),
                          kThreads, ctx->stream, a, "accept_tp_search_kernel"));
  KY_TRY(kyro::xchg::all_reduce_max_i32(ctx, a.send4, a.recv4, (size_t)a.B,
                                        "kyro_spec_accept_tp: token"));
  return launch_dependent(accept_tp_write_kernel, (unsigned)((a.B + 127) / 128), 128u,
                          ctx->stream, a, "accept_tp_write_kernel");
}

void fill_common(Args& a, const Workspace& ws, int64_t V, int B, int R) {
  a.V = V;
  a.B = B;
  a.R = R;
  a.nchunks = (int)((V + kChunk - 1) / kChunk);
  a.nfull = (int)(V / kChunk);
  a.div_chunks = make_fastdiv((uint32_t)a.nchunks);
  a.div_rows = make_fastdiv((uint32_t)R);
  a.units = (uint32_t)((int64_t)B * R * a.nchunks);
  a.stats = ws.stats;
  a.ex = ws.ex;
  a.final_ready = ws.final_ready;
  a.final_rows = ws.final_rows;
  a.W = ws.W;
  a.cnt_c = ws.cnt_c;
  a.V_global = V;
  a.vocab_offset = 0;
  a.tp_rank = 0;
  a.tp_world = 1;
  a.q_rows = 0;
  a.tree = 0;
}

}  // namespace

extern "C" {

size_t kyro_spec_accept_workspace_size(const kyro_accept_params* p) {
  if (!p || p->batch < 0 || p->num_draft < 0 || p->vocab <= 0) return 0;
  const bool stoch = p->mode == KYRO_ACCEPT_STOCHASTIC && p->temperature > 0.0f;
  const int64_t R = stoch ? 2 * (int64_t)p->num_draft + 1 : (int64_t)p->num_draft + 1;
  const int64_t nchunks = (p->vocab + kChunk - 1) / kChunk;
  return carve(nullptr, p->batch, R, nchunks).bytes;
}

}  // extern "C"

namespace {

int accept_impl(kyro_ctx* ctx, const kyro_accept_params* p, const float* target_logits,
                const float* draft_logits, const int32_t* draft_tokens, int32_t* out_accept_len,
                int32_t* out_tokens, int32_t* out_num_tokens, float* out_probs, void* workspace,
                size_t workspace_bytes, const CommitSpec* commit) {
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
  const int64_t nchunks = (V + kChunk - 1) / kChunk;
  KY_REQUIRE((int64_t)B * R * nchunks < (1ll << 31), "kyro_spec_accept: batch too large");
  const size_t need = carve(nullptr, B, R, nchunks).bytes;
  if (workspace_bytes < need || !workspace)
    return kyro::set_error(KYRO_ERR_WORKSPACE, "kyro_spec_accept: workspace %zu < %zu bytes",
                           workspace_bytes, need);
  KY_REQUIRE((uintptr_t)workspace % 256 == 0,
             "kyro_spec_accept: workspace must be 256-byte aligned");
  Workspace ws = carve(workspace, B, R, nchunks);
  Args a = {};
  fill_common(a, ws, V, B, R);
  a.plog = target_logits;
  a.qlog = stoch ? draft_logits : nullptr;
  a.draft_tokens = draft_tokens;
  a.k = k;
  a.q_rows = k;
  a.inv_t = stoch ? ky_inv_temperature(p->temperature) : 1.0f;
  a.stoch = stoch;
  a.greedy_ref = p->mode == KYRO_ACCEPT_GREEDY_REF;
  a.sample = 0;
  a.pos_div = 1;
  a.seq_rows = 1;
  a.seed = p->seed;
  a.step = p->step;
  a.seq_offset = p->seq_offset;
  a.out_accept_len = out_accept_len;
  a.out_tokens = out_tokens;
  a.out_num_tokens = out_num_tokens;
  a.out_probs = stoch ? out_probs : nullptr;
  a.status = ctx->d_status;
  // chained: the decide and final kernels wait for tagged records
  a.poll = 1;
  KY_TRY(use_unit_counter(ctx, a, ws, workspace));
  a.gen = ctx->d_pipe_counts;
  a.done = ctx->d_pipe_counts + 1;
  a.salt = ctx->pipe_salt;
  return launch(ctx, a, ws, use_vec(target_logits, a.qlog, V), commit);
}

}  // namespace

extern "C" {

int kyro_spec_accept(kyro_ctx* ctx, const kyro_accept_params* p, const float* target_logits,
                     const float* draft_logits, const int32_t* draft_tokens,
                     int32_t* out_accept_len, int32_t* out_tokens, int32_t* out_num_tokens,
                     float* out_probs, void* workspace, size_t workspace_bytes) {
  KY_NVTX("kyro_spec_accept");
  return accept_impl(ctx, p, target_logits, draft_logits, draft_tokens, out_accept_len,
                     out_tokens, out_num_tokens, out_probs, workspace, workspace_bytes, nullptr);
}

int kyro_spec_accept_commit(kyro_ctx* ctx, const kyro_accept_params* p,
                            const float* target_logits, const float* draft_logits,
                            const int32_t* draft_tokens, int32_t* out_accept_len,
                            int32_t* out_tokens, int32_t* out_num_tokens, float* out_probs,
                            void* workspace, size_t workspace_bytes, const kyro_kv_params* kv,
                            int32_t num_new, int32_t num_new_next, int64_t* block_table,
                            int64_t* context_lens, int32_t* free_stack, int32_t* free_top,
                            int32_t* ref_counts, int32_t* out_ok) {
  KY_NVTX("kyro_spec_accept_commit");
  KY_TRY(kyro::enter(ctx));
  KY_REQUIRE(p && kv, "kyro_spec_accept_commit: params is NULL");
  KY_REQUIRE(kv->batch == p->batch, "kyro_spec_accept_commit: kv batch %d != accept batch %d",
             kv->batch, p->batch);
  KY_TRY(kyro::kv::check_commit_args(kv, num_new, num_new_next, out_accept_len, block_table,
                                     context_lens, free_stack, free_top, ref_counts,
                                     "kyro_spec_accept_commit"));
  const CommitSpec commit{kv, num_new, num_new_next, block_table, context_lens,
                          free_stack, free_top, ref_counts, out_ok};
  return accept_impl(ctx, p, target_logits, draft_logits, draft_tokens, out_accept_len,
                     out_tokens, out_num_tokens, out_probs, workspace, workspace_bytes, &commit);
}

size_t kyro_sample_workspace_size(const kyro_sample_params* p) {
  if (!p || p->batch < 0 || p->num_pos < 0 || p->vocab <= 0) return 0;
  const int64_t rows = (int64_t)p->batch * p->num_pos;
  const int64_t nchunks = (p->vocab + kChunk - 1) / kChunk;
  return carve(nullptr, rows, 1, nchunks).bytes;
}

int kyro_sample_tokens(kyro_ctx* ctx, const kyro_sample_params* p, const float* logits,
                       int32_t* out_tokens, float* out_probs, void* workspace,
                       size_t workspace_bytes) {
  KY_NVTX("kyro_sample_tokens");
  KY_TRY(kyro::enter(ctx));
  KY_REQUIRE(p, "kyro_sample_tokens: params is NULL");
  KY_REQUIRE(p->batch >= 0 && p->num_pos >= 0, "kyro_sample_tokens: batch %d num_pos %d",
             p->batch, p->num_pos);
  KY_REQUIRE(p->vocab > 0 && (int64_t)p->vocab <= (int64_t)kMaxChunks * kChunk,
             "kyro_sample_tokens: vocab = %d", p->vocab);
  const int64_t rows = (int64_t)p->batch * p->num_pos;
  if (rows == 0) return KYRO_OK;
  const int64_t V = p->vocab;
  const int64_t nchunks = (V + kChunk - 1) / kChunk;
  KY_REQUIRE(rows * nchunks < (1ll << 31), "kyro_sample_tokens: too many rows");
  KY_REQUIRE(logits && out_tokens, "kyro_sample_tokens: NULL logits or out_tokens");
  KY_REQUIRE(p->seq_stride == 0 || p->seq_stride >= (uint32_t)p->num_pos,
             "kyro_sample_tokens: seq_stride %u < num_pos %d", p->seq_stride, p->num_pos);
  const size_t need = carve(nullptr, rows, 1, nchunks).bytes;
  if (workspace_bytes < need || !workspace)
    return kyro::set_error(KYRO_ERR_WORKSPACE, "kyro_sample_tokens: workspace %zu < %zu bytes",
                           workspace_bytes, need);
  KY_REQUIRE((uintptr_t)workspace % 256 == 0,
             "kyro_sample_tokens: workspace must be 256-byte aligned");
  Workspace ws = carve(workspace, rows, 1, nchunks);
  const bool stoch = p->temperature > 0.0f;
  Args a = {};
  fill_common(a, ws, V, (int)rows, 1);
  a.plog = logits;
  a.qlog = nullptr;
  a.draft_tokens = nullptr;
  a.k = 0;
  a.inv_t = stoch ? ky_inv_temperature(p->temperature) : 1.0f;
  a.stoch = stoch;
  a.greedy_ref = 0;
  a.sample = 1;
  a.pos_div = p->num_pos;
  a.seq_rows = p->seq_stride ? (int64_t)p->seq_stride : (int64_t)p->num_pos;
  a.seed = p->seed;
  a.step = p->step;
  a.seq_offset = p->seq_offset;
  a.out_tokens = out_tokens;
  a.out_probs = out_probs;
  a.status = ctx->d_status;
  KY_TRY(use_unit_counter(ctx, a, ws, workspace));
  return launch(ctx, a, ws, use_vec(logits, nullptr, V));
}

size_t kyro_spec_accept_tp_workspace_size(const kyro_accept_params* p, int world) {
  if (!p || world < 1 || p->batch < 0 || p->num_draft < 0 || p->vocab <= 0 ||
      p->vocab % world != 0)
    return 0;
  const bool stoch = p->mode == KYRO_ACCEPT_STOCHASTIC && p->temperature > 0.0f;
  const int64_t R = stoch ? 2 * (int64_t)p->num_draft + 1 : (int64_t)p->num_draft + 1;
  const int64_t nchunks = (p->vocab / world + kChunk - 1) / kChunk;
  return carve_tp(nullptr, p->batch, R, nchunks, world).bytes;
}

int kyro_spec_accept_tp(kyro_ctx* ctx, const kyro_accept_params* p, const float* target_shard,
                        const float* draft_shard, const int32_t* draft_tokens,
                        int32_t* out_accept_len, int32_t* out_tokens, int32_t* out_num_tokens,
                        float* out_probs, void* workspace, size_t workspace_bytes) {
  KY_NVTX("kyro_spec_accept_tp");
  KY_TRY(kyro::enter(ctx));
  KY_REQUIRE(p, "kyro_spec_accept_tp: params is NULL");
  const int world = ctx->tp_world;
  if (world == 1)  // no group: the single-GPU call on the full rows
    return kyro_spec_accept(ctx, p, target_shard, draft_shard, draft_tokens, out_accept_len,
                            out_tokens, out_num_tokens, out_probs, workspace, workspace_bytes);
  KY_REQUIRE(ctx->nccl_comm, "kyro_spec_accept_tp: the context has no group");
  if (ctx->tp_aborted)
    return kyro::set_error(KYRO_ERR_TIMEOUT,
                           "kyro_spec_accept_tp: a collective of this group exceeded the wait "
                           "bound and the group was aborted; destroy the context and form the "
                           "group again");
  KY_REQUIRE(p->batch >= 0, "kyro_spec_accept_tp: batch = %d", p->batch);
  KY_REQUIRE(p->num_draft >= 0 && p->num_draft <= kMaxDraft,
             "kyro_spec_accept_tp: num_draft = %d (0..%d)", p->num_draft, kMaxDraft);
  KY_REQUIRE(p->vocab > 0 && p->vocab % world == 0 &&
                 (int64_t)(p->vocab / world) <= (int64_t)kMaxChunks * kChunk,
             "kyro_spec_accept_tp: vocab = %d over %d ranks (a multiple of the group size, "
             "at most %d per rank)",
             p->vocab, world, kMaxChunks * kChunk);
  KY_REQUIRE(p->mode >= 0 && p->mode <= 2, "kyro_spec_accept_tp: mode = %d", p->mode);
  if (p->batch == 0) return KYRO_OK;
  const bool stoch = p->mode == KYRO_ACCEPT_STOCHASTIC && p->temperature > 0.0f;
  const int B = p->batch, k = p->num_draft;
  const int64_t V = p->vocab, Vl = V / world;
  KY_REQUIRE(target_shard, "kyro_spec_accept_tp: target_shard is NULL");
  KY_REQUIRE(k == 0 || draft_tokens, "kyro_spec_accept_tp: draft_tokens is NULL");
  KY_REQUIRE(!stoch || k == 0 || draft_shard,
             "kyro_spec_accept_tp: stochastic mode needs draft_shard");
  KY_REQUIRE(out_accept_len && out_tokens && out_num_tokens,
             "kyro_spec_accept_tp: an output pointer is NULL");
  const int R = stoch ? 2 * k + 1 : k + 1;
  const int64_t nchunks = (Vl + kChunk - 1) / kChunk;
  KY_REQUIRE((int64_t)B * R * nchunks < (1ll << 31) && (int64_t)B * R * world < (1ll << 31),
             "kyro_spec_accept_tp: batch too large");
  const size_t need = carve_tp(nullptr, B, R, nchunks, world).bytes;
  if (workspace_bytes < need || !workspace)
    return kyro::set_error(KYRO_ERR_WORKSPACE, "kyro_spec_accept_tp: workspace %zu < %zu bytes",
                           workspace_bytes, need);
  KY_REQUIRE((uintptr_t)workspace % 256 == 0,
             "kyro_spec_accept_tp: workspace must be 256-byte aligned");
  const TpWorkspace ws = carve_tp(workspace, B, R, nchunks, world);
  Args a = {};
  fill_common(a, ws.base, Vl, B, R);
  a.plog = target_shard;
  a.qlog = stoch ? draft_shard : nullptr;
  a.draft_tokens = draft_tokens;
  a.k = k;
  a.q_rows = k;
  a.inv_t = stoch ? ky_inv_temperature(p->temperature) : 1.0f;
  a.stoch = stoch;
  a.greedy_ref = p->mode == KYRO_ACCEPT_GREEDY_REF;
  a.sample = 0;
  a.pos_div = 1;
  a.seq_rows = 1;
  a.seed = p->seed;
  a.step = p->step;
  a.seq_offset = p->seq_offset;
  a.out_accept_len = out_accept_len;
  a.out_tokens = out_tokens;
  a.out_num_tokens = out_num_tokens;
  a.out_probs = stoch ? out_probs : nullptr;
  a.status = ctx->d_status;
  a.V_global = V;
  a.vocab_offset = (int64_t)ctx->tp_rank * Vl;
  a.tp_rank = ctx->tp_rank;
  a.tp_world = world;
  a.send1 = ws.send1;
  a.recv1 = ws.recv1;
  a.send2 = ws.send2;
  a.recv2 = ws.recv2;
  a.send3 = ws.send3;
  a.recv3 = ws.recv3;
  a.send4 = ws.send4;
  a.recv4 = ws.recv4;
  a.W2 = ws.W2;
  KY_TRY(use_unit_counter(ctx, a, ws.base, workspace));
  const bool vec = use_vec(target_shard, a.qlog, Vl);
  int st;
  if (vec && stoch) st = launch_tp<true, true>(ctx, a);
  else if (vec) st = launch_tp<true, false>(ctx, a);
  else if (stoch) st = launch_tp<false, true>(ctx, a);
  else st = launch_tp<false, false>(ctx, a);
  if (st == KYRO_OK) kyro::nccl::watch(ctx);
  return st;
}

size_t kyro_spec_accept_tree_workspace_size(const kyro_tree_params* p) {
  if (!p || p->batch < 0 || p->num_nodes < 1 || p->vocab <= 0) return 0;
  const bool stoch = p->mode == KYRO_ACCEPT_STOCHASTIC && p->temperature > 0.0f;
  const int64_t R = stoch ? 2 * (int64_t)p->num_nodes : (int64_t)p->num_nodes;
  const int64_t nchunks = (p->vocab + kChunk - 1) / kChunk;
  return carve(nullptr, p->batch, R, nchunks).bytes;
}

int kyro_spec_accept_tree(kyro_ctx* ctx, const kyro_tree_params* p, const float* target_logits,
                          const float* draft_logits, const int32_t* node_tokens,
                          const int32_t* parents, int32_t* out_path, int32_t* out_path_len,
                          int32_t* out_tokens, int32_t* out_num_tokens, void* workspace,
                          size_t workspace_bytes) {
  KY_NVTX("kyro_spec_accept_tree");
  KY_TRY(kyro::enter(ctx));
  KY_REQUIRE(p, "kyro_spec_accept_tree: params is NULL");
  KY_REQUIRE(p->batch >= 0, "kyro_spec_accept_tree: batch = %d", p->batch);
  KY_REQUIRE(p->num_nodes >= 1 && p->num_nodes <= kMaxNodes,
             "kyro_spec_accept_tree: num_nodes = %d (1..%d)", p->num_nodes, kMaxNodes);
  KY_REQUIRE(p->vocab > 0 && (int64_t)p->vocab <= (int64_t)kMaxChunks * kChunk,
             "kyro_spec_accept_tree: vocab = %d (1..%d)", p->vocab, kMaxChunks * kChunk);
  KY_REQUIRE(p->mode >= 0 && p->mode <= 2, "kyro_spec_accept_tree: mode = %d", p->mode);
  if (p->batch == 0) return KYRO_OK;
  const bool stoch = p->mode == KYRO_ACCEPT_STOCHASTIC && p->temperature > 0.0f;
  const int B = p->batch, N = p->num_nodes;
  const int64_t V = p->vocab;
  KY_REQUIRE(target_logits && node_tokens && parents,
             "kyro_spec_accept_tree: target_logits, node_tokens and parents are required");
  KY_REQUIRE(!stoch || draft_logits, "kyro_spec_accept_tree: stochastic mode needs draft_logits");
  KY_REQUIRE(out_path && out_path_len && out_tokens && out_num_tokens,
             "kyro_spec_accept_tree: an output pointer is NULL");
  const int R = stoch ? 2 * N : N;
  const int64_t nchunks = (V + kChunk - 1) / kChunk;
  KY_REQUIRE((int64_t)B * R * nchunks < (1ll << 31), "kyro_spec_accept_tree: batch too large");
  const size_t need = carve(nullptr, B, R, nchunks).bytes;
  if (workspace_bytes < need || !workspace)
    return kyro::set_error(KYRO_ERR_WORKSPACE, "kyro_spec_accept_tree: workspace %zu < %zu bytes",
                           workspace_bytes, need);
  KY_REQUIRE((uintptr_t)workspace % 256 == 0,
             "kyro_spec_accept_tree: workspace must be 256-byte aligned");
  Workspace ws = carve(workspace, B, R, nchunks);
  Args a = {};
  fill_common(a, ws, V, B, R);
  a.plog = target_logits;
  a.qlog = stoch ? draft_logits : nullptr;
  a.k = N - 1;
  a.q_rows = stoch ? N : 0;
  a.tree = 1;
  a.inv_t = stoch ? ky_inv_temperature(p->temperature) : 1.0f;
  a.stoch = stoch;
  a.seed = p->seed;
  a.step = p->step;
  a.seq_offset = p->seq_offset;
  a.node_tokens = node_tokens;
  a.parents = parents;
  a.out_path = out_path;
  a.out_path_len = out_path_len;
  a.out_tokens = out_tokens;
  a.out_num_tokens = out_num_tokens;
  a.status = ctx->d_status;
  KY_TRY(use_unit_counter(ctx, a, ws, workspace));
  const bool vec = use_vec(target_logits, a.qlog, V);
  if (vec && stoch) {
    const int resident = resident_ctas<true, true>(ctx->num_sms);
    const long long need_ctas = stats_ctas_needed(a.units);
    accept_stats_kernel<true, true><<<(int)(need_ctas < resident ? need_ctas : resident),
                                      kThreads, 0, ctx->stream>>>(a);
    KY_TRY(kyro::check_launch("accept_stats_kernel"));
    int rc = KYRO_OK;
    if (launch_tree_cluster<true>(B, a, ctx->stream, &rc)) return rc;
    return launch_dependent(accept_tree_kernel<true, true>, (unsigned)B, kTreeThreads, ctx->stream,
                            a, "accept_tree_kernel");
  }
  if (vec) {
    const int resident = resident_ctas<true, false>(ctx->num_sms);
    const long long need_ctas = stats_ctas_needed(a.units);
    accept_stats_kernel<true, false><<<(int)(need_ctas < resident ? need_ctas : resident),
                                       kThreads, 0, ctx->stream>>>(a);
    KY_TRY(kyro::check_launch("accept_stats_kernel"));
    return launch_dependent(accept_tree_kernel<true, false>, (unsigned)B, kTreeThreads,
                            ctx->stream, a, "accept_tree_kernel");
  }
  if (stoch) {
    const int resident = resident_ctas<false, true>(ctx->num_sms);
    const long long need_ctas = stats_ctas_needed(a.units);
    accept_stats_kernel<false, true><<<(int)(need_ctas < resident ? need_ctas : resident),
                                       kThreads, 0, ctx->stream>>>(a);
    KY_TRY(kyro::check_launch("accept_stats_kernel"));
    int rc = KYRO_OK;
    if (launch_tree_cluster<false>(B, a, ctx->stream, &rc)) return rc;
    return launch_dependent(accept_tree_kernel<false, true>, (unsigned)B, kTreeThreads,
                            ctx->stream, a, "accept_tree_kernel");
  }
  const int resident = resident_ctas<false, false>(ctx->num_sms);
  const long long need_ctas = stats_ctas_needed(a.units);
  accept_stats_kernel<false, false><<<(int)(need_ctas < resident ? need_ctas : resident),
                                      kThreads, 0, ctx->stream>>>(a);
  KY_TRY(kyro::check_launch("accept_stats_kernel"));
  return launch_dependent(accept_tree_kernel<false, false>, (unsigned)B, kTreeThreads, ctx->stream,
                          a, "accept_tree_kernel");
}

}  // extern "C"

// ------------------------------------------------------------ exp self-check
//
// The kernels evaluate ky_exp through exp_fast and exp_pair.  This kernel
// compares both with the contract's ky_exp on every fp32 x in [-100, 0]
// (the bit patterns 0x80000000 .. 0xC2C80000) and on -inf and both NaN
// signs, and counts the inputs whose bits differ.

namespace {

constexpr uint32_t kSelfFirst = 0x80000000u;  // -0.0f
constexpr uint32_t kSelfLast = 0xC2C80000u;   // -100.0f
constexpr uint64_t kSelfRange = (uint64_t)(kSelfLast - kSelfFirst) + 1;
constexpr uint64_t kSelfCount = kSelfRange + 3;

__device__ __forceinline__ float selftest_input(uint64_t i) {
  if (i < kSelfRange) return __uint_as_float(kSelfFirst + (uint32_t)i);
  const uint32_t special[3] = {0xFF800000u, 0x7FC00000u, 0xFFC00000u};
  return __uint_as_float(special[i - kSelfRange]);
}

__global__ void __launch_bounds__(256) exp_selftest_kernel(unsigned long long* counts) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  unsigned long long bad_fast = 0, bad_pair = 0;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < kSelfCount; i += stride) {
    const float x = selftest_input(i), y = selftest_input(kSelfCount - 1 - i);
    const uint32_t rx = __float_as_uint(ky_exp(x)), ry = __float_as_uint(ky_exp(y));
    bad_fast += __float_as_uint(exp_fast(x)) != rx;
    float px, py;
    f2_unpack(exp_pair(f2_pack(x, y)), px, py);
    bad_pair += (__float_as_uint(px) != rx) + (__float_as_uint(py) != ry);
  }
  bad_fast = warp_sum(bad_fast);
  bad_pair = warp_sum(bad_pair);
  if ((threadIdx.x & 31) == 0) {
    if (bad_fast) atomicAdd(&counts[0], bad_fast);
    if (bad_pair) atomicAdd(&counts[1], bad_pair);
  }
}

}  // namespace

extern "C" int kyro_selftest_exp(kyro_ctx* ctx, unsigned long long* counts) {
  KY_TRY(kyro::enter(ctx));
  KY_REQUIRE(counts, "kyro_selftest_exp: counts is NULL");
  cudaError_t err = cudaMemsetAsync(counts, 0, 2 * sizeof(unsigned long long), ctx->stream);
  if (err != cudaSuccess) return kyro::cuda_error(err, "cudaMemsetAsync(selftest counts)");
  exp_selftest_kernel<<<ctx->num_sms * 8, 256, 0, ctx->stream>>>(counts);
  return kyro::check_launch("exp_selftest_kernel");
}

// ------------------------------------------------------------ no-allocation entry point
//
// kyro_spec_accept_static serves callers that cannot allocate device memory
// and so cannot pass a workspace.  Its scratch is this file-scope array,
// present on every device that loads the library until the process exits.
// In host code the array's name is only a stand-in, so the device address
// is looked up once per device with cudaGetSymbolAddress while that device
// is current, and that address is what the kernels receive.

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

// A device reset (cudaDeviceReset, or the primary context torn down and made
// again) moves the array, so the cached address must not outlive it.  A
// reset also ends every kyro_ctx on the device, and any later call needs a
// new one: kyro_ctx_create calls this, and the next static call looks the
// address up again.
void kyro::static_scratch_forget(int device) {
  if (device < 0 || device >= kMaxDevices) return;
  std::lock_guard<std::mutex> lock(g_static_mu);
  g_static_ptr[device] = nullptr;
}

extern "C" int kyro_spec_accept_static(kyro_ctx* ctx, const kyro_accept_params* p,
                                       const float* target_logits, const float* draft_logits,
                                       const int32_t* draft_tokens, int32_t* out_accept_len,
                                       int32_t* out_tokens, int32_t* out_num_tokens,
                                       float* out_probs) {
  KY_NVTX("kyro_spec_accept_static");
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
