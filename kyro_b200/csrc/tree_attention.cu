// tree_attention.cu -- K1 for many query rows per KV head (tree
// verification), on the sm_100 tensor cores: tcgen05.mma with the score and
// output accumulators in tensor memory (TMEM).
//
// Replaces PagedAttention::forward (src/model/attention_kernel.rs:22-136) for
// the tree case: N draft-tree nodes x (Hq/Hkv) query heads share each KV
// head, 512 rows for config 2, which fill 128-row MMA tiles.  The chain case
// (24 rows) stays on the mma.sync kernel of attention.cu.
//
// A cluster of two CTAs (an SM pair) = (four 128-row query tiles, one KV
// head, one sequence).  Rows are ordered node-major: row r = node_local *
// group + head_in_group, so a Q tile is a TMA box of (128/group nodes) x
// (group heads) x 128 dims.  CTA `rank` of pair p holds tiles 4p + 2h + rank
// (h = 0, 1); the pair's MMAs are tcgen05.mma.cta_group::2 with M = 256, one
// instruction covering tile h of both CTAs, which runs about 1.5x faster per
// SM than two M = 128 instructions.  For S = Q K^T each CTA holds 64 of a
// KV tile's 128 tokens of K, for O += P V all 128 tokens of one 64-dim slab
// of V, so every K/V byte is loaded once per (sequence, KV head).  Per
// 128-token KV tile j (8 paged blocks):
//   warps 0-3, 4-7     the softmax of tile 0 and of tile 1, one query row
//                      per thread (its TMEM lane, so warp w reads lanes
//                      32*(w%4)..): mask, online max and sum, P = exp2(s - m)
//                      written back over the scores as bf16 in two 64-token
//                      halves, and the O rescale when the running max grows
//                      by more than 2^8.  A row's scores are read from TMEM
//                      twice (all 128 for the maximum, then 64 at a time),
//                      which keeps a thread within 168 registers.
//   warp 8 (producer)  TMA loads of this CTA's half of K_j and V_j into a
//                      ring of 16 KB slots (128-byte swizzle, no multicast;
//                      the .cta_group::2 form completes them on the leader
//                      CTA's barrier, which expects both halves)
//   warp 9 (MMA)       in the leader only: S_h = Q_h K_j^T, and after each
//                      half of tile h's softmax (both CTAs) O_h += P_h V_j
//                      with P read from TMEM and V from shared memory
//                      (MN-major).  The order S0 S1 | O0 S0' | O1 S1' lets
//                      one tile's softmax run while the other's MMAs do.
//                      Commits reach both CTAs' barriers (multicast commit).
//                      Warp 9 of each CTA also owns the pair's TMEM.
// The output is O / l, written as bf16.  Every wait is bounded; a wait that
// runs out sets KYRO_DEV_WAIT_TIMEOUT, and both CTAs still wait (bounded)
// for the leader's MMAs before they free TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <mutex>

#include "kyro_internal.cuh"
#include "ptx.cuh"

namespace {

constexpr int kBS = 16;                       // tokens per paged block
constexpr int kD = 128;                       // head dim
constexpr int kTM = 128;                      // query rows per CTA
constexpr int kTN = 128;                      // KV tokens per tile
constexpr int kTileBlocks = kTN / kBS;        // 8
constexpr int kTcThreads = 320;
constexpr int kProducerWarp = 8, kMmaWarp = 9;
constexpr int kTilesPerCta = 2;
constexpr uint32_t kSlab = 128 * 128;         // one 64-column slab of a 128-row tile
constexpr uint32_t kTile = 2 * kSlab;         // 128 rows x 128 bf16
constexpr uint32_t kItem = 16384;             // one CTA's half of a K or V tile
constexpr uint32_t kKSlab = 64 * 128;         // 64 tokens x 64 dims of K
// K and V halves share one ring of kSlots buffers, filled in the order
// K_0 V_0 K_1 V_1 ... (item n: K_{n/2} for even n, V_{n/2} for odd n) and
// released in the same order.  The ring comes first and the Q tiles after
// it, so every operand read stays inside the allocation.
constexpr int kSlots = 10;
constexpr uint32_t kOffRing = 0;                             // slot s at s * kItem
constexpr uint32_t kOffQ = kSlots * kItem;                   // Q tile h at + h * kTile
constexpr uint32_t kTilesBytes = kOffQ + 2 * kTile;          // 224 KB
constexpr uint32_t kSmemTc = kTilesBytes + 512 + 1024;       // + barriers, alignment slack
constexpr uint32_t kTmemCols = 512;           // S_h at h*128, O_h at 256 + h*128
constexpr uint32_t kColO = 256;
constexpr long long kTcWaitBudget = 2000000000ll;

struct TcArgs {
  int B, nq, hq, hkv, group, max_blocks, num_blocks;
  float scale_log2;
};

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// ---------------------------------------------------------------- CTA pair
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}
// The leader CTA's (rank 0) copy of a shared-memory object, as a
// shared::cluster address.
__device__ __forceinline__ uint32_t leader_addr(uint32_t local) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(local));
  return r;
}
// Arrive on a barrier of either CTA of the pair (default semantics, release
// at CTA scope).  TMEM written before it is ordered by tcgen05.wait::st and
// tcgen05.fence::before_thread_sync, and the MMA issued after the matching
// wait by tcgen05.fence::after_thread_sync; a cluster-scope release here
// costs about a thousand cycles per arrive and orders nothing more.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// 3-D tile load into this CTA's shared memory that completes on a barrier of
// either CTA of the pair (.cta_group::2; no multicast).
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, int32_t x,
                                                 int32_t y, int32_t z, uint32_t cluster_bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(cluster_bar)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc2(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// D (+)= A[smem] * B[smem] over the pair: each CTA supplies its 128 rows of A
// and half of B's N columns at the same shared-memory offsets.
__device__ __forceinline__ void umma2_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// D (+)= A[tmem] * B[smem] over the pair (A: each CTA's own TMEM rows).
__device__ __forceinline__ void umma2_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc,
                                         uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// Arrive on `bar` in both CTAs when every MMA issued so far is done.
__device__ __forceinline__ void umma2_commit_both(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(bar),
      "h"((uint16_t)3)
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptors (tcgen05 format: version 1, 128-byte
// swizzle).  K-major (rows of 64 contiguous bf16 along K): the stride between
// 8-row groups is 1024 B and the leading offset is unused (16 B).  MN-major
// (64 contiguous bf16 along N): the leading offset steps between 64-column
// slabs along N, the stride between 8-row groups along K.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor of kind::f16: bf16 A and B, fp32 accumulate,
// M = 256 (a CTA pair), N = 128; b_mn selects an MN-major B.
__host__ __device__ constexpr uint32_t idesc_bf16(bool b_mn) {
  return (1u << 4)              // D fp32
         | (1u << 7)            // A bf16
         | (1u << 10)           // B bf16
         | ((b_mn ? 1u : 0u) << 16)
         | ((uint32_t)(kTN >> 3) << 17)   // N = 128
         | ((uint32_t)((2 * kTM) >> 4) << 24);  // M = 256
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Maximum of a row's 128 scores (raw units): four max3 chains.
__device__ __forceinline__ float row_max128(const uint32_t (&r)[128]) {
  float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
  for (int i = 0; i < 128; i += 8) {
    m0 = fmax3(m0, __uint_as_float(r[i]), __uint_as_float(r[i + 1]));
    m1 = fmax3(m1, __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
    m2 = fmax3(m2, __uint_as_float(r[i + 4]), __uint_as_float(r[i + 5]));
    m3 = fmax3(m3, __uint_as_float(r[i + 6]), __uint_as_float(r[i + 7]));
  }
  return fmax3(fmax3(m0, m1, m2), m3, -INFINITY);
}

// 2^x on the FMA pipe, for a share of the probabilities so that the
// special-function unit is not the only exp2 engine.  x is rounded to
// n + f with |f| <= 1/2 (the 1.5 * 2^23 addition), 2^f is a degree-3
// polynomial fitted here for minimum relative error on [-1/2, 1/2]
// (7.5e-5, far below the bf16 rounding of P), and n is added to the
// exponent field.  x is clamped at -120 so the result stays normal; such
// terms (< 2^-119 against a row maximum of 1) vanish in bf16 sums.
__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -120.0f);
  const float t = x + 12582912.0f;
  const float f = x - (t - 12582912.0f);
  float p = fmaf(0.0551716685f, f, 0.2426111251f);
  p = fmaf(p, f, 0.6932609677f);
  p = fmaf(p, f, 0.9999280572f);
  return __int_as_float(__float_as_int(p) + ((__float_as_int(t) - 0x4B400000) << 23));
}

// Pairs of probabilities per 16 whose exp2 runs on the FMA pipe.
constexpr int kPolyPairs = 0;

// P = 2^(s * sl2 - m) for 64 scores (one half of a row's tile), written as
// bf16 pairs over the first 32 of their TMEM columns at pc; returns their
// sum.  With kPoly (tiles without masked scores) kPolyPairs of every 16
// pairs use exp2_poly.
template <bool kPoly>
__device__ __forceinline__ float exp_half(const uint32_t (&q)[64], float sl2, float nref,
                                          uint32_t pc) {
  float l4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float x0 = fmaf(__uint_as_float(q[c * 32 + 2 * i]), sl2, nref);
      const float x1 = fmaf(__uint_as_float(q[c * 32 + 2 * i + 1]), sl2, nref);
      const bool poly = kPoly && ((i * kPolyPairs) % 16) < kPolyPairs;
      const float p0 = poly ? exp2_poly(x0) : kyro::ptx::fast_exp2(x0);
      const float p1 = poly ? exp2_poly(x1) : kyro::ptx::fast_exp2(x1);
      l4[i & 3] += p0 + p1;
      pk[i] = kyro::ptx::pack_bf16x2(p0, p1);
    }
    tmem_st16(pc + c * 16, pk);
  }
  return (l4[0] + l4[1]) + (l4[2] + l4[3]);
}

__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, int* err, uint32_t* status) {
  if (kyro::ptx::mbar_wait_bounded(bar, parity, kTcWaitBudget)) return true;
  *(volatile int*)err = 1;
  kyro::dev::flag(status, KYRO_DEV_WAIT_TIMEOUT);
  return false;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTcThreads, 1)
tree_attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                         const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, TcArgs a,
                         const int64_t* __restrict__ block_table,
                         const int64_t* __restrict__ context_lens,
                         const uint64_t* __restrict__ tree_mask, __nv_bfloat16* __restrict__ out,
                         uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = kyro::ptx::smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + kTilesBytes;
  // leader-side barriers (only the leader's copies are used): Q and ring
  // slots filled (both CTAs' bytes), P halves written (both CTAs' threads)
  auto q_full = [&]() { return bar0; };
  auto slot_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto p_full = [&](int h, int half) { return bar0 + 8u * (1 + kSlots + 2 * h + half); };
  // barriers of both CTAs, signalled by multicast commits of the leader's MMAs
  auto slot_empty = [&](int s) { return bar0 + 8u * (5 + kSlots + s); };
  auto s_full = [&](int h) { return bar0 + 8u * (5 + 2 * kSlots + h); };
  auto o_done = [&](int h) { return bar0 + 8u * (7 + 2 * kSlots + h); };
  const uint32_t mma_done = bar0 + 8u * (9 + 2 * kSlots);
  // ring item n lives in slot n % kSlots; its fill is that slot's phase n / kSlots
  auto item_slot = [](int n) { return n % kSlots; };
  auto item_parity = [](int n) { return (uint32_t)((n / kSlots) & 1); };
  auto item_addr = [&](int n) { return base + kOffRing + (uint32_t)(n % kSlots) * kItem; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + kTilesBytes + 480);
  int* err = reinterpret_cast<int*>(gbase + kTilesBytes + 484);
  int* issued_out = reinterpret_cast<int*>(gbase + kTilesBytes + 488);  // the producer's count

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();  // 0: the leader, which issues the MMAs
  const int pair = blockIdx.x >> 1;
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int64_t ctx = context_lens[b];
  const int64_t T = ctx + a.nq;
  if (ctx < 0 || (T + kBS - 1) / kBS > a.max_blocks) {  // the same decision in both CTAs
    if (threadIdx.x == 0 && blockIdx.x == 0 && kvh == 0)
      kyro::dev::flag(status, KYRO_DEV_BAD_LENGTH);
    return;
  }
  const int nblk = (int)((T + kBS - 1) / kBS);
  const int ntiles = (int)((T + kTN - 1) / kTN);
  const int nodes_per_tile = kTM / a.group;
  const int mtiles = a.nq * a.group / kTM;
  // the pair's query tiles: 4*pair + 2*h + rank for h < ntq; a CTA whose
  // tile h lies past mtiles computes padding rows and writes nothing for them
  const int left = (mtiles - 4 * pair + 1) / 2;
  const int ntq = left < kTilesPerCta ? left : kTilesPerCta;  // 1 or 2
  auto tile_of = [&](int h) { return 4 * pair + 2 * h + (int)rank; };

  if (threadIdx.x == 0) {
    kyro::ptx::mbar_init(q_full(), 1);
    for (int i = 0; i < kSlots; ++i) {
      kyro::ptx::mbar_init(slot_full(i), 1);
      kyro::ptx::mbar_init(slot_empty(i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      kyro::ptx::mbar_init(s_full(i), 1);
      kyro::ptx::mbar_init(p_full(i, 0), 256);
      kyro::ptx::mbar_init(p_full(i, 1), 256);
      kyro::ptx::mbar_init(o_done(i), 1);
    }
    kyro::ptx::mbar_init(mma_done, 1);
    *err = 0;
    *issued_out = 0;
    kyro::ptx::fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc2(kyro::ptx::smem_addr(tmem_slot), kTmemCols);
    tmem_relinquish2();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before either signals the other
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducerWarp) {
    // ------------------------------------------------ producer (one thread per CTA)
    if (lane == 0) {
      kyro::ptx::prefetch_tensormap(&tmQ);
      kyro::ptx::prefetch_tensormap(&tmK);
      kyro::ptx::prefetch_tensormap(&tmV);
      // every load completes on the leader's barrier, which expects both CTAs' bytes
      const uint32_t lq = leader_addr(q_full());
      if (rank == 0) kyro::ptx::mbar_arrive_expect_tx(q_full(), 2u * (uint32_t)ntq * kTile);
      for (int h = 0; h < ntq; ++h) {
        // a padding tile reads some other rows (or the zero fill past the end)
        const int32_t qz = (int32_t)((int64_t)b * a.nq + tile_of(h) * nodes_per_tile);
        const uint32_t qd = base + kOffQ + (uint32_t)h * kTile;
        tma_load_3d_pair(qd, &tmQ, 0, kvh * a.group, qz, lq);
        tma_load_3d_pair(qd + kSlab, &tmQ, 64, kvh * a.group, qz, lq);
      }
      const int64_t* bt = block_table + (int64_t)b * a.max_blocks;
      // a tile's 8 block ids are loaded together, one tile ahead of use
      int64_t ids[kTileBlocks];
      auto fetch_ids = [&](int j) {
#pragma unroll
        for (int i = 0; i < kTileBlocks; ++i) {
          const int tb = j * kTileBlocks + i;
          ids[i] = __ldg(&bt[tb < nblk ? tb : 0]);  // blocks past the end: any block, masked
        }
      };
      auto zrow = [&](int64_t bid) -> int32_t {
        if (bid < 0 || bid >= a.num_blocks) {
          kyro::dev::flag(status, KYRO_DEV_BAD_BLOCK);
          bid = 0;
        }
        return (int32_t)(bid * a.hkv + kvh);
      };
      // item 2j: this CTA's 64 tokens of K_j (both 64-dim slabs, 8 KB each);
      // item 2j+1: all 128 tokens of V_j in this CTA's 64-dim slab
      auto load_item = [&](int n, const int64_t (&bids)[kTileBlocks]) {
        const uint32_t dst = item_addr(n), lb = leader_addr(slot_full(item_slot(n)));
        if (rank == 0) kyro::ptx::mbar_arrive_expect_tx(slot_full(item_slot(n)), 2u * kItem);
        if ((n & 1) == 0) {
#pragma unroll
          for (int i = 0; i < kTileBlocks / 2; ++i) {
            const int32_t z = zrow(bids[(kTileBlocks / 2) * rank + i]);
            const uint32_t off = (uint32_t)i * kBS * 128;
            tma_load_3d_pair(dst + off, &tmK, 0, 0, z, lb);
            tma_load_3d_pair(dst + kKSlab + off, &tmK, 64, 0, z, lb);
          }
        } else {
#pragma unroll
          for (int i = 0; i < kTileBlocks; ++i)
            tma_load_3d_pair(dst + (uint32_t)i * kBS * 128, &tmV, 64 * (int32_t)rank, 0,
                             zrow(bids[i]), lb);
        }
      };
      fetch_ids(0);
      int issued = 0;  // ring items whose loads this CTA has issued
      for (int j = 0; j < ntiles; ++j) {
        int64_t cur[kTileBlocks];
#pragma unroll
        for (int i = 0; i < kTileBlocks; ++i) cur[i] = ids[i];
        if (j + 1 < ntiles) fetch_ids(j + 1);
        bool stop = false;
        for (int n = 2 * j; n < 2 * j + 2; ++n) {
          if (n >= kSlots && !wait_bar(slot_empty(item_slot(n)), item_parity(n - kSlots), err, status)) {
            stop = true;
            break;
          }
          if (*(volatile int*)err) {
            stop = true;
            break;
          }
          load_item(n, cur);
          issued = n + 1;
        }
        if (stop) break;
      }
      *issued_out = issued;
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------ MMA issuer (the leader's one thread)
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idS = idesc_bf16(false), idO = idesc_bf16(true);
      auto s_mma = [&](int h, int j) {
        const uint32_t ks = item_addr(2 * j);
        const uint32_t qs = base + kOffQ + (uint32_t)h * kTile;
#pragma unroll
        for (int k = 0; k < kD / 16; ++k) {
          const uint32_t qoff = (uint32_t)(k >> 2) * kSlab + (uint32_t)(k & 3) * 32;
          const uint32_t koff = (uint32_t)(k >> 2) * kKSlab + (uint32_t)(k & 3) * 32;
          umma2_ss(tmem + (uint32_t)h * 128, desc_sw128(qs + qoff, 16, 1024),
                   desc_sw128(ks + koff, 16, 1024), idS, k > 0 ? 1u : 0u);
        }
        umma2_commit_both(s_full(h));
        if (h == ntq - 1) umma2_commit_both(slot_empty(item_slot(2 * j)));  // K_j no longer read
      };
      auto o_mma = [&](int h, int j) -> bool {
        const uint32_t vs = item_addr(2 * j + 1);
        for (int half = 0; half < 2; ++half) {
          if (!wait_bar(p_full(h, half), j & 1, err, status)) return false;
          if (half == 0 && h == 0 &&
              !wait_bar(slot_full(item_slot(2 * j + 1)), item_parity(2 * j + 1), err, status))
            return false;
          tc_fence_after();
#pragma unroll
          for (int k = 4 * half; k < 4 * half + 4; ++k) {
            const uint64_t bd = desc_sw128(vs + (uint32_t)k * 16 * 128, kSlab, 1024);
            umma2_ts(tmem + kColO + (uint32_t)h * 128, tmem + (uint32_t)h * 128 + (uint32_t)k * 8,
                     bd, idO, (j > 0 || k > 0) ? 1u : 0u);
          }
        }
        umma2_commit_both(o_done(h));
        if (h == ntq - 1) umma2_commit_both(slot_empty(item_slot(2 * j + 1)));  // V_j no longer read
        return true;
      };
      bool ok = wait_bar(q_full(), 0, err, status) && wait_bar(slot_full(0), 0, err, status);
      if (ok) {
        tc_fence_after();
        for (int h = 0; h < ntq; ++h) s_mma(h, 0);
      }
      for (int j = 0; ok && j < ntiles; ++j) {
        // a timeout recorded by another warp of this CTA: issue nothing more
        if (*(volatile int*)err) {
          ok = false;
          break;
        }
        const bool more = j + 1 < ntiles;
        for (int h = 0; ok && h < ntq; ++h) {
          if (!o_mma(h, j)) {
            ok = false;
            break;
          }
          if (more) {
            if (h == 0) {
              const int nk = 2 * (j + 1);
              if (!wait_bar(slot_full(item_slot(nk)), item_parity(nk), err, status)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
            s_mma(h, j + 1);  // overwrites P_h of tile j, consumed by the O MMA above
          }
        }
      }
      // every MMA issued above is complete before either CTA frees TMEM
      umma2_commit_both(mma_done);
    }
    if (lane == 0) wait_bar(mma_done, 0, err, status);
    __syncwarp();
  } else if (warp < 8 && warp / 4 < ntq) {
    // ------------------------------------------------ softmax of tile h, one row per thread
    const int h = warp / 4;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const bool real = tile_of(h) < mtiles;  // padding rows take part but write nothing
    const int node = real ? tile_of(h) * nodes_per_tile + row / a.group : 0;
    const int g = row % a.group;
    // bit i: the row sees draft node i (its ancestors and itself under a
    // tree mask, nodes 0..node for a chain); nothing at or past nq
    uint64_t tbits = tree_mask ? tree_mask[(int64_t)b * a.nq + node]
                               : (node >= 63 ? ~0ull : (1ull << (node + 1)) - 1ull);
    if (a.nq < 64) tbits &= (1ull << a.nq) - 1ull;
    // visibility of tokens tw .. tw+31: the context below ctx, then tbits
    auto vis_word = [&](int64_t tw) -> uint32_t {
      const int64_t d = ctx - tw;
      const uint32_t wc = d >= 32 ? 0xffffffffu : d <= 0 ? 0u : ((1u << (uint32_t)d) - 1u);
      const int64_t rel = tw - ctx;
      uint32_t wt = 0;
      if (rel >= 0 && rel < 64) wt = (uint32_t)(tbits >> rel);
      else if (rel < 0 && rel > -32) wt = (uint32_t)(tbits << (uint32_t)(-rel));
      return wc | wt;
    };
    const float sl2 = a.scale_log2;
    const uint32_t sc = tmem + lane_base + (uint32_t)h * 128;
    const uint32_t oc = tmem + lane_base + kColO + (uint32_t)h * 128;
    // P halves are reported on the leader's barriers
    const uint32_t pf0 = leader_addr(p_full(h, 0)), pf1 = leader_addr(p_full(h, 1));
    float m_used = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      if (!wait_bar(s_full(h), j & 1, err, status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int64_t t0 = (int64_t)j * kTN;
      const bool whole = t0 + kTN <= ctx;  // no masked score in the tile
      // first pass: the row's 128 scores for the maximum (four loads in flight)
      uint32_t r[128];
      tmem_ld32(sc + 0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      tmem_ld32(sc + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      tmem_ld32(sc + 64, *reinterpret_cast<uint32_t(*)[32]>(&r[64]));
      tmem_ld32(sc + 96, *reinterpret_cast<uint32_t(*)[32]>(&r[96]));
      tmem_ld_wait();
      uint32_t vis[4] = {~0u, ~0u, ~0u, ~0u};
      if (!whole) {
#pragma unroll
        for (int w = 0; w < 4; ++w) vis[w] = vis_word(t0 + 32 * w);
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (!((vis[i >> 5] >> (i & 31)) & 1u)) r[i] = 0xff800000u;  // -inf
      }
      // scores stay raw; the log2 scale enters the max and the exp2 argument
      const float m_new = fmaxf(m_used, row_max128(r) * sl2);
      bool need = false;
      if (j == 0) {
        m_used = m_new;
      } else {
        need = m_new > m_used + 8.0f;
      }
      if (__any_sync(0xffffffffu, need)) {
        // S_h of tile j was issued after O_h of tile j-1, so O_h is final
        // for tile j-1 by now; the wait only confirms it
        if (!wait_bar(o_done(h), (j - 1) & 1, err, status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float alpha = need ? kyro::ptx::fast_exp2(m_used - m_new) : 1.0f;
        if (need) {
          m_used = m_new;
          l *= alpha;
        }
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(oc + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(oc + c * 32, o);
        }
        tmem_st_wait();
      }
      const float nref = m_used == -INFINITY ? 0.0f : -m_used;
      // second pass, 64 tokens at a time: the first half's P goes to the MMA
      // warp while the second half is computed.  P of tokens 64*half.. lands
      // on score columns 32*half.., which this thread has already read.
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t q[64];
        tmem_ld32(sc + 64 * half, *reinterpret_cast<uint32_t(*)[32]>(&q[0]));
        tmem_ld32(sc + 64 * half + 32, *reinterpret_cast<uint32_t(*)[32]>(&q[32]));
        tmem_ld_wait();
        if (!whole) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (!((vis[2 * half + (i >> 5)] >> (i & 31)) & 1u)) q[i] = 0xff800000u;
        }
        const uint32_t pc = sc + 32 * half;
        l += whole ? exp_half<true>(q, sl2, nref, pc) : exp_half<false>(q, sl2, nref, pc);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive_cluster(half == 0 ? pf0 : pf1);
      }
    }
    if (ok && real && ntiles > 0 && wait_bar(o_done(h), (ntiles - 1) & 1, err, status)) {
      tc_fence_after();
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      __nv_bfloat16* orow =
          out + (((int64_t)b * a.nq + node) * a.hq + (int64_t)kvh * a.group + g) * kD;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(oc + c * 32, o);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = kyro::ptx::pack_bf16x2(__uint_as_float(o[2 * i]) * inv,
                                         __uint_as_float(o[2 * i + 1]) * inv);
        uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
        for (int v = 0; v < 4; ++v)
          dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
      }
    }
  }
  // neither CTA leaves (or frees TMEM) while the leader's MMAs may still
  // read the other's shared memory or TMEM, or its commits may still arrive
  tc_fence_before();
  __syncthreads();
  // After a timeout the consumers may have stopped before the last loads
  // landed.  The leader's slot barriers count both CTAs' bytes, so the
  // leader waits (bounded) for every item still in the ring, while the
  // cluster barrier below keeps the peer resident: no CTA leaves while a
  // bulk copy may still write its shared memory.
  if (rank == 0 && warp == kProducerWarp && lane == 0 && *(volatile int*)err) {
    const int issued = *(volatile int*)issued_out;
    for (int n = issued > kSlots ? issued - kSlots : 0; n < issued; ++n)
      kyro::ptx::mbar_wait_bounded(slot_full(item_slot(n)), item_parity(n), kTcWaitBudget);
  }
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc2(tmem, kTmemCols);
}

// ---------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// 3-D bf16 map with 128-byte swizzle: dims (innermost first), strides of the
// outer two dims in bytes, box (64, box1, box2).
int make_map3(CUtensorMap* map, const void* ptr, uint64_t d0, uint64_t d1, uint64_t d2,
              uint64_t s1, uint64_t s2, uint32_t box1, uint32_t box2) {
  auto enc = encode_fn();
  if (!enc) return kyro::set_error(KYRO_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {64, box1, box2};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return kyro::set_error(KYRO_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return KYRO_OK;
}

}  // namespace

namespace kyro {

// The shapes this kernel takes: head_dim 128, 16-token blocks, and query
// rows that fill 128-row tiles node-major (group divides 128, and the tree
// size is a multiple of 128/group).
bool tree_attention_eligible(const kyro_attn_params* p) {
  if (!p || p->head_dim != kD || p->block_size != kBS || p->num_kv_heads <= 0) return false;
  if (p->num_heads % p->num_kv_heads) return false;
  const int group = p->num_heads / p->num_kv_heads;
  if (group > kTM || kTM % group) return false;
  const int npt = kTM / group;
  return p->num_query >= npt && p->num_query % npt == 0 && p->num_query <= 64;
}

int tree_attention_launch(kyro_ctx* ctx, const kyro_attn_params* p, const void* q,
                          const void* k_cache, const void* v_cache, const int64_t* block_table,
                          const int64_t* context_lens, const uint64_t* tree_mask, void* out) {
  const int group = p->num_heads / p->num_kv_heads;
  KY_REQUIRE((uintptr_t)q % 16 == 0 && (uintptr_t)k_cache % 16 == 0 &&
                 (uintptr_t)v_cache % 16 == 0 && (uintptr_t)out % 16 == 0,
             "kyro_verify_attention: q, caches and out must be 16-byte aligned");
  CUtensorMap mq, mk, mv;
  // Q [B*nq nodes][Hq heads][128]: box (64, group heads, 128/group nodes)
  KY_TRY(make_map3(&mq, q, kD, (uint64_t)p->num_heads, (uint64_t)p->batch * p->num_query,
                   (uint64_t)kD * 2, (uint64_t)p->num_heads * kD * 2, (uint32_t)group,
                   (uint32_t)(kTM / group)));
  // K, V [blocks*Hkv][16 tokens][128]: box (64, 16, 1)
  const uint64_t rows = (uint64_t)p->num_blocks * p->num_kv_heads;
  KY_TRY(make_map3(&mk, k_cache, kD, kBS, rows, (uint64_t)kD * 2, (uint64_t)kBS * kD * 2, kBS, 1));
  KY_TRY(make_map3(&mv, v_cache, kD, kBS, rows, (uint64_t)kD * 2, (uint64_t)kBS * kD * 2, kBS, 1));
  TcArgs a;
  a.B = p->batch;
  a.nq = p->num_query;
  a.hq = p->num_heads;
  a.hkv = p->num_kv_heads;
  a.group = group;
  a.max_blocks = p->max_blocks_per_seq;
  a.num_blocks = p->num_blocks;
  const float scale = p->scale > 0.0f ? p->scale : 1.0f / sqrtf((float)kD);
  a.scale_log2 = scale * 1.4426950408889634f;
  static std::once_flag attr_once;
  std::call_once(attr_once, [] {
    cudaFuncSetAttribute(tree_attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kSmemTc);
  });
  const int mtiles = p->num_query * group / kTM;
  // CTA pairs (the kernel's cluster shape), each covering four query tiles
  const dim3 grid((unsigned)(2 * ((mtiles + 3) / 4)), (unsigned)p->num_kv_heads,
                  (unsigned)p->batch);
  tree_attention_tc_kernel<<<grid, kTcThreads, kSmemTc, ctx->stream>>>(
      mq, mk, mv, a, block_table, context_lens, tree_mask, (__nv_bfloat16*)out, ctx->d_status);
  return kyro::check_launch("tree_attention_tc_kernel");
}

}  // namespace kyro
