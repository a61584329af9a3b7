// attention.cu -- K1: paged multi-query verify attention for sm_100a.
//
// Replaces PagedAttention::forward / paged_attention_kernel
// (src/model/attention_kernel.rs:22-136), which walks the block table one
// scalar at a time with a host sync per block and makes two passes over
// K/V.  Here one pass streams each 16-token K and V block of a KV head once
// for all query rows that share it (GQA group x verify positions).
//
// Work item: (sequence b, KV head, row group of <= 32 query rows, KV
// split).  A CTA has four warps and each warp streams its own share of the
// item's KV blocks (blocks w, w+4, w+8, ...) through a private shared-memory
// ring with 16-byte cp.async copies.  Paged blocks are scattered 4 KB tiles,
// and HBM bandwidth on this pattern follows the number of independent
// warps issuing loads, so every warp is its own producer; three CTAs per SM
// keep twelve streams in flight.  Tiles land XOR-swizzled (16-byte chunk
// index ^ row) so ldmatrix reads them without bank conflicts.
//
// Per block a warp computes, with bf16 mma.sync (m16n8k16):
//     S^T = K Q^T      (M = 16 tokens, N = query rows, K = head_dim)
//     O^T += V^T P^T   (M = head_dim, N = query rows, K = 16 tokens)
// so the query rows (24 for GQA 4 x 6 positions) sit in the N dimension in
// 8-wide tiles without padding to 16; movmatrix turns P^T into the B
// operand.  Online softmax runs per query column in the log2 domain.  The
// four warps' states merge in shared memory in one pass (each warp
// publishes its (O, m, l), per-column factors are formed once, then every
// thread combines four dims at a time); when a sequence needs more than one
// split, every split takes an epoch-tagged ticket, and the one whose ticket
// completes the count merges them all from its own state on chip and the
// partial states the other splits store in the workspace (each raises a
// ready flag once its partial is out).
#include <cuda_bf16.h>

#include <cmath>
#include <mutex>

#include "kyro_internal.cuh"
#include "ptx.cuh"
#include "rope.cuh"

namespace {

constexpr int kBS = 16;               // tokens per KV block
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxCols = 32;          // query rows per work item
constexpr int kMaxSplitBlocks = 256;  // KV blocks per work item
constexpr int kMaxSplits = 64;        // work items per (sequence, KV head, row group)
// 64-bit words of a work item's ticket region: the ticket, then a 32-bit
// ready flag per split
__host__ __device__ constexpr int ticket_words(int max_splits) { return 1 + (max_splits + 1) / 2; }
constexpr float kLazyRescale = 8.0f;  // log2 headroom before a column's running max moves

// Shared-memory geometry for head_dim D (64 or 128) and NS ring stages.
template <int D, int NS>
struct Geo {
  static constexpr int kTileBytes = kBS * D * 2;      // one K or V block of one head
  static constexpr int kSlotBytes = 2 * kTileBytes;   // K + V
  static constexpr int kWarpRing = NS * kSlotBytes;
  static constexpr int kRingBytes = kWarps * kWarpRing;
  static constexpr int kQStride = D + 8;              // padded bf16 row stride of the Q tile
  static constexpr int kQBytes = kMaxCols * kQStride * 2;
  // warp merge: the four warps' (O, m, l), merge factors and the merged
  // (m, l), over the ring and the Q tile (both free by then).  O is stored
  // [col][D + 4] so a warp's accumulator fragment (8 dims x 4 column pairs)
  // hits 32 different banks.
  static constexpr int kMoStride = D + 4;
  static constexpr int kMergeBytes =
      (kWarps * kMaxCols * kMoStride + 3 * kWarps * kMaxCols + 2 * kMaxCols) * 4;
  static_assert(kMergeBytes <= kRingBytes + kQBytes, "the warp merge reuses the ring and Q tile");
  static constexpr int kSmemBytes =
      kRingBytes + kQBytes + kMaxCols * 8 + kMaxSplitBlocks * 4 + 16;
};

struct AttnArgs {
  int B, nq, hq, hkv, group, rows, ngroups, max_blocks, num_blocks, split_blocks, max_splits;
  float scale_log2;
  int d;
  uint32_t epoch;  // nonzero, new on every call: split tickets of older calls count as zero
};

// The rotary embedding fused into the prologue (kyro_verify_attention_rope):
// the unrotated new keys and values, the caches they are stored into, and
// the rotary frequencies (D <= 128).
struct RopeIn {
  const uint4* k_new;          // bf16 [B, nq, Hkv, D]
  const uint4* v_new;
  const int32_t* pos_offsets;  // [nq] or NULL (offset j)
  uint8_t* k_cache;
  uint8_t* v_cache;
  float inv_freq[64];
};

// byte offset of (token row, 16-byte chunk along D) inside a swizzled tile:
// 64-column halves of 2 KB, rows of 128 B, chunk index XOR (row & 7)
__device__ __forceinline__ uint32_t kv_off(int row, int cidx) {
  return (uint32_t)((cidx >> 3) * 2048 + row * 128 + (((cidx & 7) ^ (row & 7)) << 4));
}

// Issue the cp.async copies of one block's K and V tiles (one KV head) into
// a slot; every lane copies its share of 16-byte chunks.
template <int D>
__device__ __forceinline__ void load_block(uint32_t slot, const uint8_t* __restrict__ k_base,
                                           const uint8_t* __restrict__ v_base, int64_t tile_off,
                                           int lane) {
  constexpr int kTile = kBS * D * 2;
  constexpr int kChunks = kTile / 16;   // 256 (D=128) or 128 (D=64)
  constexpr int kPerRow = D / 8;        // 16-byte chunks per token row
  const uint8_t* ks = k_base + tile_off;
  const uint8_t* vs = v_base + tile_off;
#pragma unroll
  for (int i = 0; i < kChunks / 32; ++i) {
    const int c = lane + 32 * i;
    const uint32_t off = kv_off(c / kPerRow, c % kPerRow);
    kyro::ptx::cp_async_16(slot + off, ks + c * 16);
    kyro::ptx::cp_async_16(slot + kTile + off, vs + c * 16);
  }
}

// The end of a work item after its warp merge, out of line so that its
// registers do not weigh on the streaming loop's: a single split writes its
// rows; with more than one split, the split whose ticket completes the count
// merges them all.  The ticket comes first, so the merging split keeps its
// own state on chip; every other split stores its partial and raises its
// ready flag.  A ticket is (epoch << 32 | splits done); a ticket of another
// epoch (a workspace that held other data) counts as zero.
template <int D, int NS>
__device__ __noinline__ void split_merge(const AttnArgs a, const float* mo, const float* mf,
                                         const float* mM, const float* mL, int* sh_last, int b,
                                         int kvh, int grp, int split, int nsplit, int ncols,
                                         int col0, __nv_bfloat16* __restrict__ out,
                                         float* __restrict__ part_o, float* __restrict__ part_ml,
                                         unsigned long long* __restrict__ tickets,
                                         uint32_t* status) {
  constexpr int kD = D;
  constexpr int kMoStride = Geo<D, NS>::kMoStride;
  const int tid = threadIdx.x;
  const bool single = nsplit == 1;
  const int64_t item = ((int64_t)b * a.hkv + kvh) * a.ngroups + grp;
  float* po = part_o + item * a.max_splits * (kMaxCols * kD);
  float* pml = part_ml + item * a.max_splits * (kMaxCols * 2);
  // the item's ticket and its splits' ready flags (ticket_words per item)
  unsigned long long* tkt = tickets + item * ticket_words(a.max_splits);
  uint32_t* ready = reinterpret_cast<uint32_t*>(tkt + 1);

  bool last = single;
  if (!single) {
    if (tid == 0) {
      // guess that this split completes the count: one CAS when it does
      unsigned long long cur = ((unsigned long long)a.epoch << 32) | (uint32_t)(nsplit - 1);
      uint32_t done;
      for (;;) {
        done = (uint32_t)(cur >> 32) == a.epoch ? (uint32_t)cur + 1u : 1u;
        const unsigned long long nw = ((unsigned long long)a.epoch << 32) | done;
        const unsigned long long prev = atomicCAS(tkt, cur, nw);
        if (prev == cur) break;
        cur = prev;
      }
      *sh_last = done == (uint32_t)nsplit;
    }
    __syncthreads();
    last = *sh_last != 0;
  }

  // this split's merged O at (col, d4..d4+3), formed from the warps' states
  // in shared memory wherever it is needed (the same operations each time);
  // a thread's entries are tid, tid + kThreads, ... (four dims each)
  constexpr int kEnt = kMaxCols * (kD / 4) / kThreads;
  auto own_o = [&](int col, int d4) -> float4 {
    float4 O = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = mf[w * kMaxCols + col];
      const float4 v = *reinterpret_cast<const float4*>(&mo[(w * kMaxCols + col) * kMoStride + d4]);
      O.x += f * v.x;
      O.y += f * v.y;
      O.z += f * v.z;
      O.w += f * v.w;
    }
    return O;
  };
  auto store_out = [&](int col, int d4, float4 O, float inv) {
    const int r = col0 + col, j = r / a.group, gi = r % a.group;
    const int h = kvh * a.group + gi;
    *reinterpret_cast<uint2*>(&out[(((int64_t)b * a.nq + j) * a.hq + h) * kD + d4]) =
        make_uint2(kyro::ptx::pack_bf16x2(O.x * inv, O.y * inv),
                   kyro::ptx::pack_bf16x2(O.z * inv, O.w * inv));
  };
  if (single) {
#pragma unroll
    for (int e = 0; e < kEnt; ++e) {
      const int i4 = tid + e * kThreads;
      const int col = i4 / (kD / 4), d4 = (i4 % (kD / 4)) * 4;
      if (col >= ncols) continue;
      const float L = mL[col];
      store_out(col, d4, own_o(col, d4), L > 0.0f ? 1.0f / L : 0.0f);
    }
    return;
  }
  if (!last) {
#pragma unroll
    for (int e = 0; e < kEnt; ++e) {
      const int i4 = tid + e * kThreads;
      const int col = i4 / (kD / 4), d4 = (i4 % (kD / 4)) * 4;
      if (col >= ncols) continue;
      *reinterpret_cast<float4*>(&po[(split * kMaxCols + col) * kD + d4]) = own_o(col, d4);
      if (d4 == 0) {
        pml[(split * kMaxCols + col) * 2 + 0] = mM[col];
        pml[(split * kMaxCols + col) * 2 + 1] = mL[col];
      }
    }
    __syncthreads();
    if (tid == 0) {
      __threadfence();  // every thread's partial (observed through the barrier) first
      asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(ready + split), "r"(a.epoch)
                   : "memory");
    }
    return;
  }
  // the merging split: the others' ready flags (each split took its ticket
  // before this one and stores without waiting, so the wait is short;
  // bounded all the same)
  if (tid < nsplit && tid != split) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ready + tid) : "memory");
    if (v != a.epoch) {
      unsigned long long t0, t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
      while (true) {
        __nanosleep(64);
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ready + tid) : "memory");
        if (v == a.epoch) break;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (t - t0 > 1000000000ull) {
          kyro::dev::flag(status, KYRO_DEV_WAIT_TIMEOUT);
          break;
        }
      }
    }
  }
  __syncthreads();
  // every thread merges its own entries: the splits' maxima of its columns,
  // then factors, sums and O in split order (this split's own state in place
  // of its partial)
  float Mu[kEnt];
#pragma unroll
  for (int e = 0; e < kEnt; ++e) {
    const int col = min((tid + e * kThreads) / (kD / 4), kMaxCols - 1);
    Mu[e] = mM[col];
  }
#pragma unroll 1
  for (int sp = 0; sp < nsplit; ++sp) {
    if (sp == split) continue;
#pragma unroll
    for (int e = 0; e < kEnt; ++e) {
      const int col = min((tid + e * kThreads) / (kD / 4), kMaxCols - 1);
      Mu[e] = fmaxf(Mu[e], __ldcg(&pml[(sp * kMaxCols + col) * 2]));
    }
  }
  float Ls[kEnt];
  float4 O[kEnt];
#pragma unroll
  for (int e = 0; e < kEnt; ++e) {
    if (Mu[e] == -INFINITY) Mu[e] = 0.0f;
    Ls[e] = 0.0f;
    O[e] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
#pragma unroll 1
  for (int sp = 0; sp < nsplit; ++sp) {
#pragma unroll
    for (int e = 0; e < kEnt; ++e) {
      const int i4 = tid + e * kThreads;
      const int col = min(i4 / (kD / 4), kMaxCols - 1), d4 = (i4 % (kD / 4)) * 4;
      float m, l;
      float4 v;
      if (sp == split) {
        m = mM[col];
        l = mL[col];
        v = own_o(col, d4);
      } else {
        m = __ldcg(&pml[(sp * kMaxCols + col) * 2]);
        l = __ldcg(&pml[(sp * kMaxCols + col) * 2 + 1]);
        v = __ldcg(reinterpret_cast<const float4*>(&po[(sp * kMaxCols + col) * kD + d4]));
      }
      const float f = kyro::ptx::fast_exp2(m - Mu[e]);
      Ls[e] += f * l;
      O[e].x += f * v.x;
      O[e].y += f * v.y;
      O[e].z += f * v.z;
      O[e].w += f * v.w;
    }
  }
#pragma unroll
  for (int e = 0; e < kEnt; ++e) {
    const int i4 = tid + e * kThreads;
    const int col = i4 / (kD / 4), d4 = (i4 % (kD / 4)) * 4;
    if (col >= ncols) continue;
    store_out(col, d4, O[e], Ls[e] > 0.0f ? 1.0f / Ls[e] : 0.0f);
  }
  // back to zero for the next call (a replayed graph reuses its epoch)
  if (tid < nsplit && tid != split) ready[tid] = 0u;
  if (tid == 0) *tkt = 0ull;
}

// ROPE: the queries arrive unrotated and this step's keys and values are not
// in the cache yet.  The prologue rotates the CTA's query rows, and a CTA
// whose blocks hold new slots rotates those keys and stores them with their
// values before it streams the blocks (the cache is read only by cp.async,
// after a fence and a barrier).
template <int NT, int D, int NS, bool ROPE>
__global__ void __launch_bounds__(kThreads, 3)
verify_attention_kernel(const __nv_bfloat16* __restrict__ q,
                        const uint8_t* k_base, const uint8_t* v_base,
                        const int64_t* __restrict__ block_table,
                        const int64_t* __restrict__ context_lens,
                        const uint64_t* __restrict__ tree_mask, __nv_bfloat16* __restrict__ out,
                        float* __restrict__ part_o, float* __restrict__ part_ml,
                        unsigned long long* __restrict__ tickets, AttnArgs a, RopeIn r,
                        uint32_t* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  using G = Geo<D, NS>;
  constexpr int kD = D;
  constexpr int kTileBytes = G::kTileBytes, kSlotBytes = G::kSlotBytes;
  constexpr int kQStride = G::kQStride, kQBytes = G::kQBytes;
  constexpr int kMT = D / 16;   // m-tiles of O^T along head_dim
  constexpr int kKK = D / 16;   // k-steps of S^T along head_dim
  const int split = blockIdx.x;
  const int kvh = blockIdx.y / a.ngroups;
  const int grp = blockIdx.y % a.ngroups;
  const int b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // launched behind the stream's previous kernel (programmatic dependent
  // launch): nothing is read or written before it has completed
  kyro::dev::pdl_wait();
  kyro::dev::pdl_trigger();

  // this warp's first block ids load together with the context length (the
  // split's start does not depend on it); entries past the table row are
  // not read
  const int64_t* bt = block_table + (int64_t)b * a.max_blocks + (int64_t)split * a.split_blocks;
  int64_t first_ids[NS - 1];
#pragma unroll
  for (int p = 0; p < NS - 1; ++p)
    first_ids[p] = split * a.split_blocks + p * kWarps + warp < a.max_blocks ? bt[p * kWarps + warp]
                                                                             : 0;
  // the rest of the split's block ids (entries tid, tid + kThreads of the
  // split's span of the table row) and the CTA's Q rows do not depend on the
  // context length either: they load in the same round trip
  constexpr int kIdsPerThread = kMaxSplitBlocks / kThreads;
  constexpr int kQPerThread = kMaxCols * (D / 8) / kThreads;
  const int span = min(a.split_blocks, a.max_blocks - split * a.split_blocks);
  int64_t my_ids[kIdsPerThread];
#pragma unroll
  for (int j = 0; j < kIdsPerThread; ++j)
    my_ids[j] = tid + j * kThreads < span ? bt[tid + j * kThreads] : 0;
  const int col0 = grp * kMaxCols;
  const int ncols = min(kMaxCols, a.rows - col0);
  uint4 my_q[kQPerThread];
#pragma unroll
  for (int j = 0; j < kQPerThread; ++j) {
    const int i = tid + j * kThreads;
    const int col = i / (D / 8), ch = i % (D / 8);
    my_q[j] = make_uint4(0, 0, 0, 0);
    if (col < ncols) {
      const int r = col0 + col, jq = r / a.group, gi = r % a.group;
      const int h = kvh * a.group + gi;
      my_q[j] =
          *reinterpret_cast<const uint4*>(q + (((int64_t)b * a.nq + jq) * a.hq + h) * D + ch * 8);
    }
  }
  // ROPE: this KV head's new K/V rows load in the same round trip (which of
  // them fall in this split depends on the context length).  Item it of
  // kRowItems per row: a K piece and its partner half, or one V piece;
  // thread tid holds items tid and tid + kThreads, the rest load later.
  constexpr int kHalfPieces = kD / 16;
  constexpr int kRowItems = kHalfPieces + kD / 8;
  constexpr int kNewPre = 2;
  uint4 pre1[kNewPre], pre2[kNewPre];
#pragma unroll
  for (int u = 0; u < kNewPre; ++u) {
    pre1[u] = pre2[u] = make_uint4(0, 0, 0, 0);
    const int it = tid + u * kThreads;
    if (ROPE && it < a.nq * kRowItems) {
      const int j = it / kRowItems, c0 = it - j * kRowItems;
      const int64_t src = (((int64_t)b * a.nq + j) * a.hkv + kvh) * (kD / 8);
      if (c0 < kHalfPieces) {
        pre1[u] = r.k_new[src + c0];
        pre2[u] = r.k_new[src + kHalfPieces + c0];
      } else {
        pre1[u] = r.v_new[src + c0 - kHalfPieces];
      }
    }
  }
  const int64_t ctx = context_lens[b];
  const int64_t total = ctx + a.nq;
  if (ctx < 0 || (total + kBS - 1) / kBS > a.max_blocks) {
    if (tid == 0 && split == 0) kyro::dev::flag(status, KYRO_DEV_BAD_LENGTH);
    return;
  }
  const int nblk = (int)((total + kBS - 1) / kBS);
  const int nsplit = (nblk + a.split_blocks - 1) / a.split_blocks;
  if (split >= nsplit) return;
  const int blk0 = split * a.split_blocks;
  const int nb = min(nblk, blk0 + a.split_blocks) - blk0;

  uint8_t* ring = smem;
  uint8_t* qtile = ring + G::kRingBytes;
  uint64_t* col_mask = reinterpret_cast<uint64_t*>(qtile + kQBytes);
  int32_t* ids = reinterpret_cast<int32_t*>(col_mask + kMaxCols);
  int* sh_last = reinterpret_cast<int*>(ids + kMaxSplitBlocks);
  const uint32_t ring_s = kyro::ptx::smem_addr(ring);
  const uint32_t q_s = ring_s + G::kRingBytes;

  // ---- this warp's first blocks go out before the setup below, so their
  // latency overlaps it.  With ROPE, a block from ctx / kBS on receives new
  // keys below: its load waits until they are stored ("late").
  const int nmy = nb > warp ? (nb - warp + kWarps - 1) / kWarps : 0;
  const uint32_t wring0 = kyro::ptx::smem_addr(smem) + warp * G::kWarpRing;
  uint32_t late = 0;
#pragma unroll
  for (int p = 0; p < NS - 1; ++p) {
    if (p < nmy) {
      if (ROPE && blk0 + p * kWarps + warp >= ctx / kBS) {
        late |= 1u << p;
      } else {
        int64_t phys = first_ids[p];
        if (phys < 0 || phys >= a.num_blocks) phys = 0;  // flagged below
        load_block<D>(wring0 + p * kSlotBytes, k_base, v_base, (phys * a.hkv + kvh) * kTileBytes,
                      lane);
      }
    }
    kyro::ptx::cp_async_commit();
  }

  // ---- block ids of this split, Q rows, column masks into shared memory
  int bad_id = 0;
#pragma unroll
  for (int j = 0; j < kIdsPerThread; ++j) {
    const int i = tid + j * kThreads;
    if (i < nb) {
      int64_t phys = my_ids[j];
      if (phys < 0 || phys >= a.num_blocks) {
        kyro::dev::flag(status, KYRO_DEV_BAD_BLOCK);
        phys = 0;
        bad_id = 1;
      }
      ids[i] = (int32_t)phys;
    }
  }
  if (!ROPE) {
#pragma unroll
    for (int j = 0; j < kQPerThread; ++j) {
      const int i = tid + j * kThreads;
      const int col = i / (kD / 8), ch = i % (kD / 8);
      *reinterpret_cast<uint4*>(qtile + col * kQStride * 2 + ch * 16) = my_q[j];
    }
  }
  for (int col = tid; col < kMaxCols; col += kThreads) {
    uint64_t m = 0;
    if (col < ncols) {
      const int j = (col0 + col) / a.group;
      m = tree_mask ? tree_mask[(int64_t)b * a.nq + j]
                    : (j >= 63 ? ~0ull : ((1ull << (j + 1)) - 1ull));
    }
    col_mask[col] = m;
  }
  // ROPE: cos and sin of every new position, in the ring slot that no
  // prefetch fills (slot NS-1 of each warp; position p in warp p / kTabRows)
  constexpr int kHalf = kD / 2;
  constexpr int kTabRowBytes = kHalf * 8;
  constexpr int kTabRows = kSlotBytes / kTabRowBytes;
  static_assert(kWarps * kTabRows >= 64, "the table holds 64 positions");
  auto tab = [&](int p) -> const float2* {
    return reinterpret_cast<const float2*>(ring + (p / kTabRows) * G::kWarpRing +
                                           (NS - 1) * kSlotBytes + (p % kTabRows) * kTabRowBytes);
  };
  if (ROPE) {
    for (int idx = tid; idx < a.nq * kHalf; idx += kThreads) {
      const int p = idx / kHalf, i = idx - p * kHalf;
      // the rotary position: (index + offset) as f32 (layers.rs:45)
      const float pf = (float)(ctx + (r.pos_offsets ? r.pos_offsets[p] : p));
      float c, sn;
      kyro::rope::angle(pf, r.inv_freq[i], c, sn);
      const_cast<float2*>(tab(p))[i] = make_float2(c, sn);
    }
  }
  const int any_bad_id = __syncthreads_or(bad_id);  // the ids, the mask and the table are in place
  if (ROPE) {
    // the query rows: thread tid holds 16-byte piece ch of row col (i = tid
    // + j * kThreads); the piece with the other half of the same dims sits
    // in thread tid ^ kHalfPieces
#pragma unroll
    for (int j = 0; j < kQPerThread; ++j) {
      const int i = tid + j * kThreads;
      const int col = i / (kD / 8), ch = i % (kD / 8);
      const uint4 x = my_q[j];
      uint4 y;
      y.x = __shfl_xor_sync(0xffffffffu, x.x, kHalfPieces);
      y.y = __shfl_xor_sync(0xffffffffu, x.y, kHalfPieces);
      y.z = __shfl_xor_sync(0xffffffffu, x.z, kHalfPieces);
      y.w = __shfl_xor_sync(0xffffffffu, x.w, kHalfPieces);
      uint4 o = make_uint4(0, 0, 0, 0);
      if (col < ncols) {
        const bool first = ch < kHalfPieces;
        const uint4 wa = first ? x : y, wb = first ? y : x;
        const uint32_t a4[4] = {wa.x, wa.y, wa.z, wa.w}, b4[4] = {wb.x, wb.y, wb.z, wb.w};
        const float2* cs = tab((col0 + col) / a.group) + (first ? ch : ch - kHalfPieces) * 8;
        uint32_t o4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 t0 = cs[2 * e], t1 = cs[2 * e + 1];
          uint32_t lo, hi;
          kyro::rope::rotate_pair(a4[e], b4[e], t0.x, t1.x, t0.y, t1.y, lo, hi);
          o4[e] = first ? lo : hi;
        }
        o = make_uint4(o4[0], o4[1], o4[2], o4[3]);
      }
      *reinterpret_cast<uint4*>(qtile + col * kQStride * 2 + ch * 16) = o;
    }
    // the new slots ctx + j that fall in this split's blocks: rotated keys
    // (a piece and its partner half per item) and values (one piece per
    // item), the items numbered as their speculative loads above
    const int64_t s_lo = (int64_t)blk0 * kBS - ctx, s_hi = (int64_t)(blk0 + nb) * kBS - ctx;
    const int j_lo = (int)(s_lo > 0 ? s_lo : 0);
    const int j_hi = (int)(s_hi < a.nq ? s_hi : a.nq);
    bool stored = false;
    if (j_lo < j_hi) {
      for (int it = tid, u = 0; it < a.nq * kRowItems; it += kThreads, ++u) {
        const int j = it / kRowItems, c0 = it - j * kRowItems;
        if (j < j_lo || j >= j_hi) continue;
        const int64_t slot = ctx + j;
        int64_t phys = ids[slot / kBS - blk0];
        if (any_bad_id) {  // ids of bad entries read 0 in shared memory: check the table
          phys = block_table[(int64_t)b * a.max_blocks + slot / kBS];
          if (phys < 0 || phys >= a.num_blocks) continue;  // flagged with the block ids
        }
        const int64_t row = ((phys * a.hkv + kvh) * kBS + slot % kBS) * (kD / 8);  // uint4 units
        const int64_t src = (((int64_t)b * a.nq + j) * a.hkv + kvh) * (kD / 8);
        const bool is_k = c0 < kHalfPieces;
        uint4 x1, x2;
        if (u == 0) {
          x1 = pre1[0];
          x2 = pre2[0];
        } else if (u == 1) {
          x1 = pre1[kNewPre - 1];
          x2 = pre2[kNewPre - 1];
        } else if (is_k) {
          x1 = r.k_new[src + c0];
          x2 = r.k_new[src + kHalfPieces + c0];
        } else {
          x1 = r.v_new[src + c0 - kHalfPieces];
        }
        if (is_k) {
          const int c = c0;
          const uint32_t a4[4] = {x1.x, x1.y, x1.z, x1.w}, b4[4] = {x2.x, x2.y, x2.z, x2.w};
          const float2* cs = tab(j) + c * 8;
          uint32_t lo[4], hi[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 t0 = cs[2 * e], t1 = cs[2 * e + 1];
            kyro::rope::rotate_pair(a4[e], b4[e], t0.x, t1.x, t0.y, t1.y, lo[e], hi[e]);
          }
          uint4* dst = reinterpret_cast<uint4*>(r.k_cache) + row;
          dst[c] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
          dst[kHalfPieces + c] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        } else {
          reinterpret_cast<uint4*>(r.v_cache)[row + c0 - kHalfPieces] = x1;
        }
        stored = true;
      }
    }
    // the stores reach L2 before any cp.async of this CTA reads the blocks
    // (only a thread that stored has anything to fence); the table's slot is
    // free again after the barrier
    if (stored) __threadfence();
    __syncthreads();
    // the late blocks: one copy group for every prefetch position from the
    // first late one on (empty where the warp has no block), in order, so
    // that the ring's group count still finds block i complete at iteration i
    if (late) {
      const int p0 = __ffs(late) - 1;
#pragma unroll
      for (int p = 0; p < NS - 1; ++p) {
        if (p < p0) continue;
        if (late & (1u << p))
          load_block<D>(wring0 + p * kSlotBytes, k_base, v_base,
                        ((int64_t)ids[p * kWarps + warp] * a.hkv + kvh) * kTileBytes, lane);
        kyro::ptx::cp_async_commit();
      }
    }
  }

  // ---- this warp's blocks: w, w + 4, w + 8, ... of the split (the first
  // NS-1 already in flight)
  const uint32_t wring = ring_s + warp * G::kWarpRing;
  auto tile_off = [&](int i) -> int64_t {
    return ((int64_t)ids[i * kWarps + warp] * a.hkv + kvh) * kTileBytes;
  };

  float o[kMT][NT][4];
  float m_run[NT][2], l_run[NT][2];
#pragma unroll
  for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[mt][nt][e] = 0.0f;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m_run[nt][0] = m_run[nt][1] = -INFINITY;
    l_run[nt][0] = l_run[nt][1] = 0.0f;
  }
  const int g8 = lane >> 3, r8 = lane & 7;
  for (int i = 0; i < nmy; ++i) {
    // keep NS-1 blocks in flight: issue block i+NS-1 into the slot freed last iteration
    const int pf = i + NS - 1;
    if (pf < nmy) load_block<D>(wring + (pf % NS) * kSlotBytes, k_base, v_base, tile_off(pf), lane);
    kyro::ptx::cp_async_commit();
    kyro::ptx::cp_async_wait<NS - 1>();  // block i has landed (this lane's copies)
    __syncwarp();                        // ... and every lane's
    const int blk = blk0 + i * kWarps + warp;
    const uint32_t ks = wring + (i % NS) * kSlotBytes;
    const uint32_t vs = ks + kTileBytes;
    // ---- S^T = K Q^T
    float sc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[nt][e] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < kKK; kk += 2) {
      uint32_t qb[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        kyro::ptx::ldsm_x4(q_s + (uint32_t)((nt * 8 + r8) * kQStride * 2 + (2 * kk + g8) * 16),
                           qb[nt][0], qb[nt][1], qb[nt][2], qb[nt][3]);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t a0, a1, a2, a3;
        // matrices: (tokens 0-7 | 8-15) x (dims lo | hi) of k-step kk+h
        kyro::ptx::ldsm_x4(ks + kv_off((g8 & 1) * 8 + r8, 2 * (kk + h) + (g8 >> 1)), a0, a1, a2,
                           a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          kyro::ptx::mma_bf16_16816(sc[nt], a0, a1, a2, a3, qb[nt][2 * h], qb[nt][2 * h + 1]);
      }
    }
    // ---- scale, mask, online softmax (per query column)
    const int64_t tok0 = (int64_t)blk * kBS;
    const bool need_mask = tok0 + kBS > ctx;
    const int trow = lane >> 2;
    bool over = false;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = sc[nt][e] * a.scale_log2;
        if (need_mask) {
          const int64_t t = tok0 + trow + (e >> 1) * 8;
          const int col = nt * 8 + 2 * (lane & 3) + (e & 1);
          const int64_t rel = t - ctx;
          const bool ok = t < ctx || (rel < a.nq && ((col_mask[col] >> rel) & 1ull));
          if (!ok) v = -INFINITY;
        }
        sc[nt][e] = v;
        over |= v > m_run[nt][e & 1] + kLazyRescale;
      }
    }
    // The running max of a column moves only when a score passes it by more
    // than kLazyRescale (log2 units), so P stays below 2^kLazyRescale; most
    // blocks skip the column reductions and the O rescale.
    if (__any_sync(0xffffffffu, over)) {
      float alpha[NT][2];
      bool moved = false;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float cm = fmaxf(sc[nt][c], sc[nt][c + 2]);
          cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 4));
          cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 8));
          cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 16));
          const float m_new = fmaxf(m_run[nt][c], cm);
          const float m_use = m_new == -INFINITY ? 0.0f : m_new;
          alpha[nt][c] = kyro::ptx::fast_exp2(m_run[nt][c] - m_use);
          moved |= m_new != m_run[nt][c];
          l_run[nt][c] *= alpha[nt][c];
          m_run[nt][c] = m_new;
        }
      // rescale O only when some running max moved (alpha == 1 otherwise)
      if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
        for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            o[mt][nt][0] *= alpha[nt][0];
            o[mt][nt][1] *= alpha[nt][1];
            o[mt][nt][2] *= alpha[nt][0];
            o[mt][nt][3] *= alpha[nt][1];
          }
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const float m_use = m_run[nt][c] == -INFINITY ? 0.0f : m_run[nt][c];
        const float p0 = kyro::ptx::fast_exp2(sc[nt][c] - m_use);
        const float p1 = kyro::ptx::fast_exp2(sc[nt][c + 2] - m_use);
        sc[nt][c] = p0;
        sc[nt][c + 2] = p1;
        l_run[nt][c] += p0 + p1;
      }
    // P^T fragment (tokens x cols) -> B operand (k = tokens, n = cols)
    uint32_t pb[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      pb[nt][0] = kyro::ptx::movmatrix_trans(kyro::ptx::pack_bf16x2(sc[nt][0], sc[nt][1]));
      pb[nt][1] = kyro::ptx::movmatrix_trans(kyro::ptx::pack_bf16x2(sc[nt][2], sc[nt][3]));
    }
    // ---- O^T += V^T P^T
#pragma unroll
    for (int mt = 0; mt < kMT; ++mt) {
      uint32_t a0, a1, a2, a3;
      // matrices: (tokens 0-7 | 8-15) x (dims 16mt.. | 16mt+8..), transposed
      kyro::ptx::ldsm_x4_trans(vs + kv_off((g8 >> 1) * 8 + r8, 2 * mt + (g8 & 1)), a0, a1, a2, a3);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        kyro::ptx::mma_bf16_16816(o[mt][nt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
    }
    __syncwarp();  // every lane is done with this slot before it is refilled
  }
  kyro::ptx::cp_async_wait<0>();
  // reduce the per-thread partial sums over the 8 lanes sharing a column
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float l = l_run[nt][c];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      l_run[nt][c] = l;
    }
  __syncthreads();  // the ring is free

  // ---- merge the four warps in one pass: each publishes its state, the
  // first ncols threads form the per-column factors, then every thread
  // combines four dims at a time
  constexpr int kMoStride = G::kMoStride;
  float* mo = reinterpret_cast<float*>(ring);           // [warp][col][kMoStride]
  float* mm = mo + kWarps * kMaxCols * kMoStride;       // [warp][col]
  float* ml = mm + kWarps * kMaxCols;                   // [warp][col]
  float* mf = ml + kWarps * kMaxCols;                   // [warp][col] merge factors
  float* mM = mf + kWarps * kMaxCols;                   // [col] merged max
  float* mL = mM + kMaxCols;                            // [col] merged sum
  {
    float* wo = mo + warp * kMaxCols * kMoStride;
#pragma unroll
    for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int d = mt * 16 + (lane >> 2) + (e >> 1) * 8;
          const int col = nt * 8 + 2 * (lane & 3) + (e & 1);
          wo[col * kMoStride + d] = o[mt][nt][e];
        }
    if (lane < 4) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int col = nt * 8 + 2 * lane + c;
          mm[warp * kMaxCols + col] = m_run[nt][c];
          ml[warp * kMaxCols + col] = l_run[nt][c];
        }
    }
  }
  __syncthreads();
  if (tid < ncols) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mm[w * kMaxCols + tid]);
    const float Mu = M == -INFINITY ? 0.0f : M;
    float L = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = kyro::ptx::fast_exp2(mm[w * kMaxCols + tid] - Mu);
      mf[w * kMaxCols + tid] = f;
      L += f * ml[w * kMaxCols + tid];
    }
    mM[tid] = M;
    mL[tid] = L;
  }
  __syncthreads();

  split_merge<D, NS>(a, mo, mf, mM, mL, sh_last, b, kvh, grp, split, nsplit, ncols, col0, out,
                     part_o, part_ml, tickets, status);
}

// ------------------------------------------------------------------ host

// ring stages per warp: a D = 64 block is half the bytes of a D = 128 one,
// so it keeps one more block in flight (measured on 512 sequences of
// lognormal context: 2% faster with 5 query rows, equal with 1; a fourth
// stage costs CTAs per SM when the splits are short)
template <int D>
constexpr int stages_for() { return D == 64 ? 3 : 2; }

struct Plan {
  AttnArgs a;
  int nt;
  size_t part_o_bytes, part_ml_bytes, ticket_bytes;
};

int plan(const kyro_attn_params* p, int num_sms, Plan* out) {
  KY_REQUIRE(p, "kyro_verify_attention: params is NULL");
  KY_REQUIRE(p->batch >= 0, "kyro_verify_attention: batch = %d", p->batch);
  KY_REQUIRE(p->num_query >= 1 && p->num_query <= 64,
             "kyro_verify_attention: num_query = %d (1..64)", p->num_query);
  KY_REQUIRE(p->head_dim == 64 || p->head_dim == 128,
             "kyro_verify_attention: head_dim = %d (64 or 128 supported)", p->head_dim);
  KY_REQUIRE(p->block_size == kBS, "kyro_verify_attention: block_size = %d (only %d supported)",
             p->block_size, kBS);
  KY_REQUIRE(p->num_heads > 0 && p->num_kv_heads > 0 && p->num_heads % p->num_kv_heads == 0,
             "kyro_verify_attention: num_heads %d not a multiple of num_kv_heads %d",
             p->num_heads, p->num_kv_heads);
  KY_REQUIRE(p->max_blocks_per_seq > 0, "kyro_verify_attention: max_blocks_per_seq = %d",
             p->max_blocks_per_seq);
  KY_REQUIRE(p->num_blocks > 0, "kyro_verify_attention: num_blocks = %d", p->num_blocks);
  KY_REQUIRE((int64_t)p->num_blocks * p->num_kv_heads < (1ll << 31),
             "kyro_verify_attention: num_blocks * num_kv_heads must fit in 31 bits");
  KY_REQUIRE(p->kv_split_blocks >= 0, "kyro_verify_attention: kv_split_blocks = %d",
             p->kv_split_blocks);
  Plan pl;
  AttnArgs& a = pl.a;
  a.B = p->batch;
  a.nq = p->num_query;
  a.hq = p->num_heads;
  a.hkv = p->num_kv_heads;
  a.group = p->num_heads / p->num_kv_heads;
  a.rows = a.group * a.nq;
  a.ngroups = (a.rows + kMaxCols - 1) / kMaxCols;
  a.max_blocks = p->max_blocks_per_seq;
  a.num_blocks = p->num_blocks;
  const float scale = p->scale > 0.0f ? p->scale : 1.0f / sqrtf((float)p->head_dim);
  a.scale_log2 = scale * 1.4426950408889634f;
  a.d = p->head_dim;
  int64_t split = p->kv_split_blocks;
  if (split == 0) {
    // aim for about 1.6 waves of work items at three CTAs per SM, assuming
    // half the table width is used on average.  Measured with the RoPE
    // prologue on 64 sequences of U[512, 4096] context (Hq 32 / Hkv 8, 320
    // table columns): splits of 112 / 120 / 124 / 128 blocks 115.7 / 116.4 /
    // 116.5 / 117.0 us, the two-wave choice (92 blocks) 120.0 us, and 64 /
    // 80 / 96 / 144 / 160 blocks 119.8 / 125.6 / 120.6 / 121.2 / 121.3 us
    const int64_t items = (int64_t)a.B * a.hkv * a.ngroups;
    const int64_t avg_blocks = (a.max_blocks + 1) / 2;
    const int64_t target = (int64_t)num_sms * 3 * 8 / 5;
    split = (items * avg_blocks + target - 1) / (target > 0 ? target : 1);
    split = (split + kWarps - 1) / kWarps * kWarps;
    if (split < 16) split = 16;
  }
  // a work item holds at most kMaxSplitBlocks block ids, and a sequence at
  // most kMaxSplits work items
  if (split > kMaxSplitBlocks) split = kMaxSplitBlocks;
  const int64_t min_split = (a.max_blocks + kMaxSplits - 1) / kMaxSplits;
  if (split < min_split) split = min_split;
  KY_REQUIRE(split <= kMaxSplitBlocks,
             "kyro_verify_attention: max_blocks_per_seq %d needs more than %d work items",
             a.max_blocks, kMaxSplits);
  a.split_blocks = (int)split;
  a.max_splits = (int)((a.max_blocks + split - 1) / split);
  pl.nt = a.rows >= kMaxCols ? 4 : (a.rows + 7) / 8;
  const int64_t groups = (int64_t)a.B * a.hkv * a.ngroups;
  const int64_t items = groups * (a.max_splits > 1 ? a.max_splits : 0);
  pl.part_o_bytes = (size_t)items * kMaxCols * p->head_dim * 4;
  pl.part_ml_bytes = (size_t)items * kMaxCols * 2 * 4;
  pl.ticket_bytes = a.max_splits > 1 ? (size_t)groups * 8 * ticket_words(a.max_splits) : 0;
  *out = pl;
  return KYRO_OK;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

size_t ws_bytes(const Plan& pl) {
  return align256(pl.part_o_bytes) + align256(pl.part_ml_bytes) + align256(pl.ticket_bytes);
}

template <int NT, int D, bool ROPE>
void launch(const Plan& pl, dim3 grid, cudaStream_t st, const void* q, const void* kc,
            const void* vc, const int64_t* bt, const int64_t* cl, const uint64_t* tm, void* out,
            float* po, float* pml, unsigned long long* tk, const RopeIn& r, uint32_t* status) {
  constexpr int kStages = stages_for<D>();
  constexpr int smem = Geo<D, kStages>::kSmemBytes;
  static std::once_flag attr_once;  // one host call per kernel, never inside a graph capture
  std::call_once(attr_once, [] {
    cudaFuncSetAttribute(verify_attention_kernel<NT, D, kStages, ROPE>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  });
  kyro::launch_pdl(verify_attention_kernel<NT, D, kStages, ROPE>, grid, dim3(kThreads), smem, st,
                   "verify_attention_kernel", (const __nv_bfloat16*)q, (const uint8_t*)kc,
                   (const uint8_t*)vc, bt, cl, tm, (__nv_bfloat16*)out, po, pml, tk, pl.a, r,
                   status);
}

template <int D, bool ROPE>
void launch_d(const Plan& pl, dim3 grid, cudaStream_t st, const void* q, const void* kc,
              const void* vc, const int64_t* bt, const int64_t* cl, const uint64_t* tm,
              void* out, float* po, float* pml, unsigned long long* tk, const RopeIn& r,
              uint32_t* status) {
  switch (pl.nt) {
    case 1: launch<1, D, ROPE>(pl, grid, st, q, kc, vc, bt, cl, tm, out, po, pml, tk, r, status); break;
    case 2: launch<2, D, ROPE>(pl, grid, st, q, kc, vc, bt, cl, tm, out, po, pml, tk, r, status); break;
    case 3: launch<3, D, ROPE>(pl, grid, st, q, kc, vc, bt, cl, tm, out, po, pml, tk, r, status); break;
    default: launch<4, D, ROPE>(pl, grid, st, q, kc, vc, bt, cl, tm, out, po, pml, tk, r, status); break;
  }
}

// The split-KV kernel (not the tcgen05 tree kernel) on a planned call; r
// non-null fuses the rotary embedding.
int run_split_kernel(kyro_ctx* ctx, const kyro_attn_params* p, Plan& pl, const void* q,
                     const void* k_cache, const void* v_cache, const int64_t* block_table,
                     const int64_t* context_lens, const uint64_t* tree_mask, void* out,
                     void* workspace, size_t workspace_bytes, const RopeIn* r, const char* fn) {
  const size_t need = ws_bytes(pl);
  if (need > 0 && (workspace_bytes < need || !workspace))
    return kyro::set_error(KYRO_ERR_WORKSPACE, "%s: workspace %zu < %zu bytes", fn,
                           workspace_bytes, need);
  KY_REQUIRE(need == 0 || (uintptr_t)workspace % 256 == 0,
             "%s: workspace must be 256-byte aligned", fn);
  float* po = (float*)workspace;
  float* pml = (float*)((char*)workspace + align256(pl.part_o_bytes));
  unsigned long long* tk = (unsigned long long*)((char*)workspace + align256(pl.part_o_bytes) +
                                                 align256(pl.part_ml_bytes));
  dim3 grid((unsigned)pl.a.max_splits, (unsigned)(pl.a.hkv * pl.a.ngroups), (unsigned)pl.a.B);
  cudaStream_t st = ctx->stream;
  // split tickets carry the call's epoch, so one workspace needs zeroing
  // only the first time this context sees it (a zeroed ticket holds epoch 0,
  // which no call uses)
  if (++ctx->attn_epoch == 0) ctx->attn_epoch = 1;
  pl.a.epoch = ctx->attn_epoch;
  if (pl.ticket_bytes && workspace != ctx->attn_ws_zeroed) {
    cudaError_t err = cudaMemsetAsync(tk, 0, pl.ticket_bytes, st);
    if (err != cudaSuccess) return kyro::cuda_error(err, "cudaMemsetAsync(attention tickets)");
    ctx->attn_ws_zeroed = workspace;
  }
  RopeIn none{};
  const RopeIn& rr = r ? *r : none;
  if (p->head_dim == 128) {
    if (r)
      launch_d<128, true>(pl, grid, st, q, k_cache, v_cache, block_table, context_lens, tree_mask,
                          out, po, pml, tk, rr, ctx->d_status);
    else
      launch_d<128, false>(pl, grid, st, q, k_cache, v_cache, block_table, context_lens, tree_mask,
                           out, po, pml, tk, rr, ctx->d_status);
  } else {
    if (r)
      launch_d<64, true>(pl, grid, st, q, k_cache, v_cache, block_table, context_lens, tree_mask,
                         out, po, pml, tk, rr, ctx->d_status);
    else
      launch_d<64, false>(pl, grid, st, q, k_cache, v_cache, block_table, context_lens, tree_mask,
                          out, po, pml, tk, rr, ctx->d_status);
  }
  return kyro::check_launch("verify_attention_kernel");
}

}  // namespace

extern "C" {

size_t kyro_verify_attention_workspace_size(const kyro_attn_params* p) {
  Plan pl;
  if (plan(p, 148, &pl) != KYRO_OK) return 0;
  return ws_bytes(pl);
}

int kyro_verify_attention(kyro_ctx* ctx, const kyro_attn_params* p, const void* q,
                          const void* k_cache, const void* v_cache, const int64_t* block_table,
                          const int64_t* context_lens, const uint64_t* tree_mask, void* out,
                          void* workspace, size_t workspace_bytes) {
  KY_NVTX("kyro_verify_attention");
  KY_TRY(kyro::enter(ctx));
  Plan pl;
  // plan with the SM count the workspace size was computed for, so that
  // kyro_verify_attention_workspace_size() and this call agree
  KY_TRY(plan(p, 148, &pl));
  if (p->batch == 0) return KYRO_OK;
  KY_REQUIRE(q && k_cache && v_cache && block_table && context_lens && out,
             "kyro_verify_attention: a required pointer is NULL");
  KY_REQUIRE((uintptr_t)k_cache % 16 == 0 && (uintptr_t)v_cache % 16 == 0 &&
                 (uintptr_t)q % 16 == 0,
             "kyro_verify_attention: q and the caches must be 16-byte aligned");
  KY_REQUIRE(pl.a.B <= 65535, "kyro_verify_attention: batch %d > 65535", pl.a.B);
  // enough query rows per KV head to fill 128-row tensor-core tiles (draft
  // trees): the tcgen05 kernel, which needs no workspace
  if (kyro::tree_attention_eligible(p))
    return kyro::tree_attention_launch(ctx, p, q, k_cache, v_cache, block_table, context_lens,
                                       tree_mask, out);
  return run_split_kernel(ctx, p, pl, q, k_cache, v_cache, block_table, context_lens, tree_mask,
                          out, workspace, workspace_bytes, nullptr, "kyro_verify_attention");
}

int kyro_verify_attention_rope(kyro_ctx* ctx, const kyro_attn_params* p, float rope_theta,
                               const int32_t* pos_offsets, const void* q, const void* k_new,
                               const void* v_new, void* k_cache, void* v_cache,
                               const int64_t* block_table, const int64_t* context_lens,
                               const uint64_t* tree_mask, void* out, void* workspace,
                               size_t workspace_bytes) {
  KY_NVTX("kyro_verify_attention_rope");
  KY_TRY(kyro::enter(ctx));
  Plan pl;
  KY_TRY(plan(p, 148, &pl));
  KY_REQUIRE(rope_theta > 0.0f, "kyro_verify_attention_rope: rope_theta = %g",
             (double)rope_theta);
  KY_REQUIRE(!kyro::tree_attention_eligible(p),
             "kyro_verify_attention_rope: this shape runs on the tensor-core tree kernel; "
             "use kyro_rope_kv_write and kyro_verify_attention");
  if (p->batch == 0) return KYRO_OK;
  KY_REQUIRE(q && k_new && v_new && k_cache && v_cache && block_table && context_lens && out,
             "kyro_verify_attention_rope: a required pointer is NULL");
  KY_REQUIRE((uintptr_t)k_cache % 16 == 0 && (uintptr_t)v_cache % 16 == 0 &&
                 (uintptr_t)q % 16 == 0 && (uintptr_t)k_new % 16 == 0 &&
                 (uintptr_t)v_new % 16 == 0,
             "kyro_verify_attention_rope: q, k_new, v_new and the caches must be 16-byte "
             "aligned");
  KY_REQUIRE(pl.a.B <= 65535, "kyro_verify_attention_rope: batch %d > 65535", pl.a.B);
  RopeIn r{};
  r.k_new = (const uint4*)k_new;
  r.v_new = (const uint4*)v_new;
  r.pos_offsets = pos_offsets;
  r.k_cache = (uint8_t*)k_cache;
  r.v_cache = (uint8_t*)v_cache;
  // RotaryEmbedding::new (layers.rs:26-33): 1 / theta^(2i/D) in double, then fp32
  for (int i = 0; i < 64; ++i)
    r.inv_freq[i] = i < p->head_dim / 2
                        ? (float)(1.0 / std::pow((double)rope_theta, 2.0 * i / p->head_dim))
                        : 0.0f;
  return run_split_kernel(ctx, p, pl, q, k_cache, v_cache, block_table, context_lens, tree_mask,
                          out, workspace, workspace_bytes, &r, "kyro_verify_attention_rope");
}

}  // extern "C"
