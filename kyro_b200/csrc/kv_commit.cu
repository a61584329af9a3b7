// kv_commit.cu -- K3: KV-slot reserve / commit / rollback on the device
// mirror of BlockManager (src/scheduler/block_manager.rs:15-153).
//
// The reference allocates a request's blocks once, at admission, by
// popping Vec free_gpu_blocks from the back with ref_count = 1 (:92-98,
// :115-121), and returns them on free when the ref count reaches zero, in
// table order (:133-150).  It never grows a sequence during decode and
// never rolls back.  The verify step needs both: reserve k+1 slots before
// the target forward, keep the accepted ones after, release the rest.
//
// Both operations run as one CTA that walks the batch in tiles of one
// sequence per thread (up to kTile).  Within a tile, per-sequence block
// counts go through a block-wide exclusive scan, which gives every sequence
// the same stack
// positions a sequential loop in batch order would: sequence b pops
// free_stack[top-1-off_b-i] for its i-th block and pushes released block i
// at free_stack[top+off_b+i].  When the fast path's preconditions fail
// (the pool runs out inside the tile, or a released block is shared), the
// tile is done by one thread in batch order, which is the reference's
// semantics exactly.
#include <algorithm>
#include <cmath>

#include "kyro_internal.cuh"
#include "rope.cuh"

namespace {

constexpr int kTile = 1024;

__device__ __forceinline__ int64_t blocks_for(int64_t tokens, int bs) {
  return (tokens + bs - 1) / bs;
}

// Block-wide exclusive scan of an int over the block's threads (a multiple
// of 32, at most kTile).
__device__ int block_exclusive_scan(int v, int* sh, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  __syncthreads();
  if (lane == 31) sh[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nwarps ? sh[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    sh[32 + lane] = wi - w;  // exclusive warp offsets
    if (lane == 31) sh[64] = wi;
  }
  __syncthreads();
  *total = sh[64];
  return sh[32 + warp] + inc - v;
}

// COW (copy-on-write): a sequence whose last block is partly filled and
// shared (ref count > 1, a prefix held by the radix cache or another
// request, block_manager.rs:60-63) gets a fresh block for it before its new
// blocks; the shared block's ref count drops by one and the pair (shared,
// fresh) goes to cow[b] for the copy kernel (-1, -1 when there is none).  A
// tile with such a sequence takes the one-thread path, so that sequences
// sharing one block see each other's decrements in batch order.
template <bool COW>
__device__ __forceinline__ void reserve_body(int B, int bs, int max_blocks, int num_blocks,
                                             int num_new, int64_t* __restrict__ block_table,
                                             const int64_t* __restrict__ context_lens,
                                             const int32_t* __restrict__ free_stack,
                                             int32_t* __restrict__ free_top,
                                             int32_t* __restrict__ ref_counts,
                                             int32_t* __restrict__ out_ok,
                                             int32_t* __restrict__ cow, uint32_t* status) {
  __shared__ int sh[72];
  __shared__ int sh_top, sh_fast;
  if (threadIdx.x == 0) {
    int t = *free_top;
    if (t < 0 || t > num_blocks) {
      kyro::dev::flag(status, KYRO_DEV_STACK_OVERFLOW);
      t = t < 0 ? 0 : num_blocks;
    }
    sh_top = t;
  }
  __syncthreads();
  for (int base = 0; base < B; base += (int)blockDim.x) {
    const int b = base + threadIdx.x;
    int64_t have = 0, need = 0;
    bool fits_table = true, shared_last = false;
    if (b < B) {
      const int64_t len = context_lens[b];
      have = blocks_for(len, bs);
      const int64_t want = blocks_for(len + num_new, bs);
      need = want - have;
      fits_table = len >= 0 && want <= max_blocks;
      if (!fits_table) kyro::dev::flag(status, KYRO_DEV_BAD_LENGTH);
      if constexpr (COW) {
        if (fits_table && len % bs != 0) {
          const int64_t old = block_table[(int64_t)b * max_blocks + have - 1];
          shared_last = old >= 0 && old < num_blocks && ref_counts[old] > 1;
        }
      }
    }
    int total;
    const int off = block_exclusive_scan(fits_table ? (int)need : 0, sh, &total);
    const int top = sh_top;
    if (threadIdx.x == 0) sh_fast = 1;
    __syncthreads();
    if (b < B && (!fits_table || shared_last)) sh_fast = 0;
    __syncthreads();
    const bool fast = sh_fast && total <= top;
    if (fast) {
      if (b < B) {
        for (int64_t i = 0; i < need; ++i) {
          const int32_t blk = free_stack[top - 1 - off - i];
          if (blk < 0 || blk >= num_blocks) {
            kyro::dev::flag(status, KYRO_DEV_BAD_BLOCK);
            continue;
          }
          ref_counts[blk] = 1;
          block_table[(int64_t)b * max_blocks + have + i] = blk;
        }
        if (out_ok) out_ok[b] = 1;
        if constexpr (COW) {
          cow[2 * b] = -1;
          cow[2 * b + 1] = -1;
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) sh_top = top - total;
      __syncthreads();
    } else {
      __syncthreads();
      if (threadIdx.x == 0) {
        int t = top;
        const int end = min(B, base + (int)blockDim.x);
        for (int bb = base; bb < end; ++bb) {
          const int64_t len = context_lens[bb];
          const int64_t h = blocks_for(len, bs);
          const int64_t w = blocks_for(len + num_new, bs);
          int64_t n = w - h;
          int64_t old = -1;
          if constexpr (COW) {
            cow[2 * bb] = -1;
            cow[2 * bb + 1] = -1;
            if (len >= 0 && w <= max_blocks && len % bs != 0) {
              const int64_t o = block_table[(int64_t)bb * max_blocks + h - 1];
              if (o >= 0 && o < num_blocks && ref_counts[o] > 1) old = o;
            }
          }
          if (len < 0 || w > max_blocks || n + (old >= 0) > t) {
            if (out_ok) out_ok[bb] = 0;
            continue;
          }
          if constexpr (COW) {
            if (old >= 0) {
              const int32_t blk = free_stack[--t];
              if (blk < 0 || blk >= num_blocks) {
                kyro::dev::flag(status, KYRO_DEV_BAD_BLOCK);
              } else {
                ref_counts[blk] = 1;
                ref_counts[old] -= 1;
                block_table[(int64_t)bb * max_blocks + h - 1] = blk;
                cow[2 * bb] = (int32_t)old;
                cow[2 * bb + 1] = blk;
              }
            }
          }
          for (int64_t i = 0; i < n; ++i) {
            const int32_t blk = free_stack[--t];
            if (blk < 0 || blk >= num_blocks) {
              kyro::dev::flag(status, KYRO_DEV_BAD_BLOCK);
              continue;
            }
            ref_counts[blk] = 1;
            block_table[(int64_t)bb * max_blocks + h + i] = blk;
          }
          if (out_ok) out_ok[bb] = 1;
        }
        sh_top = t;
      }
      __syncthreads();
    }
  }
  if (threadIdx.x == 0) *free_top = sh_top;
  __syncthreads();
}

template <bool COW>
__global__ void __launch_bounds__(kTile)
kv_reserve_kernel(int B, int bs, int max_blocks, int num_blocks, int num_new,
                  int64_t* __restrict__ block_table, const int64_t* __restrict__ context_lens,
                  const int32_t* __restrict__ free_stack, int32_t* __restrict__ free_top,
                  int32_t* __restrict__ ref_counts, int32_t* __restrict__ out_ok,
                  int32_t* __restrict__ cow, uint32_t* status) {
  kyro::dev::pdl_wait();
  kyro::dev::pdl_trigger();
  reserve_body<COW>(B, bs, max_blocks, num_blocks, num_new, block_table, context_lens, free_stack,
                    free_top, ref_counts, out_ok, cow, status);
}

// accept_len[b] (accepted drafts) or path_len[b] (accepted path length
// including the root) gives the number of reserved slots to keep.
__device__ __forceinline__ void commit_body(int B, int bs, int max_blocks, int num_blocks,
                                            int num_new, const int32_t* __restrict__ accept_len,
                                            const int32_t* __restrict__ path_len,
                                            int64_t* __restrict__ block_table,
                                            int64_t* __restrict__ context_lens,
                                            int32_t* __restrict__ free_stack,
                                            int32_t* __restrict__ free_top,
                                            int32_t* __restrict__ ref_counts, uint32_t* status) {
  __shared__ int sh[72];
  __shared__ int sh_top, sh_fast;
  if (threadIdx.x == 0) {
    int t = *free_top;
    if (t < 0 || t > num_blocks) {
      kyro::dev::flag(status, KYRO_DEV_STACK_OVERFLOW);
      t = t < 0 ? 0 : num_blocks;
    }
    sh_top = t;
  }
  __syncthreads();
  for (int base = 0; base < B; base += (int)blockDim.x) {
    const int b = base + threadIdx.x;
    int64_t len = 0, keep = 0, had = 0, new_len = 0;
    bool active = false;
    int nrel = 0;
    if (threadIdx.x == 0) sh_fast = 1;
    __syncthreads();
    if (b < B) {
      const int a = accept_len ? accept_len[b] : (path_len ? path_len[b] - 1 : -1);
      len = context_lens[b];
      if (a >= 0 && len < 0) kyro::dev::flag(status, KYRO_DEV_BAD_LENGTH);
      if (a >= 0 && len >= 0) {
        active = true;
        const int64_t kept = min((int64_t)a + 1, (int64_t)num_new);
        new_len = len + kept;
        keep = blocks_for(new_len, bs);
        had = min(blocks_for(len + num_new, bs), (int64_t)max_blocks);
        for (int64_t i = keep; i < had; ++i) {
          const int64_t blk = block_table[(int64_t)b * max_blocks + i];
          if (blk < 0) continue;
          if (blk >= num_blocks) {
            kyro::dev::flag(status, KYRO_DEV_BAD_BLOCK);
            continue;
          }
          if (ref_counts[blk] != 1) sh_fast = 0;  // shared (or inconsistent) block
          ++nrel;
        }
      }
    }
    int total;
    const int off = block_exclusive_scan(nrel, sh, &total);
    const int top = sh_top;
    const bool fast = sh_fast && (top + total <= num_blocks);
    if (fast) {
      if (active) {
        int k = 0;
        for (int64_t i = keep; i < had; ++i) {
          int64_t* slot = &block_table[(int64_t)b * max_blocks + i];
          const int64_t blk = *slot;
          *slot = -1;
          if (blk < 0 || blk >= num_blocks) continue;
          ref_counts[blk] = 0;
          free_stack[top + off + k] = (int32_t)blk;
          ++k;
        }
        context_lens[b] = new_len;
      }
      __syncthreads();
      if (threadIdx.x == 0) sh_top = top + total;
      __syncthreads();
    } else {
      __syncthreads();
      if (threadIdx.x == 0) {
        int t = top;
        const int end = min(B, base + (int)blockDim.x);
        for (int bb = base; bb < end; ++bb) {
          const int a = accept_len ? accept_len[bb] : (path_len ? path_len[bb] - 1 : -1);
          const int64_t l0 = context_lens[bb];
          if (a < 0 || l0 < 0) continue;
          const int64_t nl = l0 + min((int64_t)a + 1, (int64_t)num_new);
          const int64_t kp = blocks_for(nl, bs);
          const int64_t hd = min(blocks_for(l0 + num_new, bs), (int64_t)max_blocks);
          for (int64_t i = kp; i < hd; ++i) {
            int64_t* slot = &block_table[(int64_t)bb * max_blocks + i];
            const int64_t blk = *slot;
            *slot = -1;
            if (blk < 0 || blk >= num_blocks) continue;
            if (ref_counts[blk] > 0) ref_counts[blk] -= 1;
            if (ref_counts[blk] == 0) {
              if (t < num_blocks)
                free_stack[t++] = (int32_t)blk;
              else
                kyro::dev::flag(status, KYRO_DEV_STACK_OVERFLOW);
            }
          }
          context_lens[bb] = nl;
        }
        sh_top = t;
      }
      __syncthreads();
    }
  }
  if (threadIdx.x == 0) *free_top = sh_top;
  __syncthreads();
}

__global__ void __launch_bounds__(kTile)
kv_commit_kernel(int B, int bs, int max_blocks, int num_blocks, int num_new,
                 const int32_t* __restrict__ accept_len, const int32_t* __restrict__ path_len,
                 int64_t* __restrict__ block_table, int64_t* __restrict__ context_lens,
                 int32_t* __restrict__ free_stack, int32_t* __restrict__ free_top,
                 int32_t* __restrict__ ref_counts, uint32_t* status) {
  kyro::dev::pdl_wait();
  kyro::dev::pdl_trigger();
  commit_body(B, bs, max_blocks, num_blocks, num_new, accept_len, path_len, block_table,
              context_lens, free_stack, free_top, ref_counts, status);
}

// The commit of this step's slots, then the reserve of num_new_next slots
// for the next step, in one launch: a decoding loop always reserves right
// after it commits.  The two phases run in the same CTA, in the same order
// as kv_commit_kernel followed by kv_reserve_kernel.  Launched between the
// acceptance's decide and final kernels (kyro_spec_accept_commit): it lets
// the final kernel launch before it waits for the accept lengths, since the
// final kernel waits for its own records and touches none of the KV state.
__global__ void __launch_bounds__(kTile)
kv_commit_reserve_kernel(int B, int bs, int max_blocks, int num_blocks, int num_new,
                         int num_new_next, const int32_t* __restrict__ accept_len,
                         int64_t* __restrict__ block_table, int64_t* __restrict__ context_lens,
                         int32_t* __restrict__ free_stack, int32_t* __restrict__ free_top,
                         int32_t* __restrict__ ref_counts, int32_t* __restrict__ out_ok,
                         uint32_t* status) {
  kyro::dev::pdl_trigger();
  kyro::dev::pdl_wait();
  commit_body(B, bs, max_blocks, num_blocks, num_new, accept_len, nullptr, block_table,
              context_lens, free_stack, free_top, ref_counts, status);
  if (num_new_next > 0)
    reserve_body<false>(B, bs, max_blocks, num_blocks, num_new_next, block_table, context_lens,
                        free_stack, free_top, ref_counts, out_ok, nullptr, status);
}

constexpr int kMaxLayerPtrs = 32;
struct CachePtrs {
  uint8_t* p[2 * kMaxLayerPtrs];  // K caches then V caches of up to 32 layers
};

// grid (B, 2 * layers in this launch); moves the accepted path's rows to
// consecutive positions.  Every source row of a head is read into shared
// memory before any destination is written.
__global__ void __launch_bounds__(256)
kv_tree_move_kernel(CachePtrs caches, int nlayers, int num_nodes, int hkv, int d, int bs,
                    int max_blocks, int num_blocks, const int32_t* __restrict__ path,
                    const int32_t* __restrict__ path_len, const int64_t* __restrict__ block_table,
                    const int64_t* __restrict__ context_lens, uint32_t* status) {
  extern __shared__ uint4 rows[];  // [num_nodes][d*2/16]
  const int b = blockIdx.x;
  const int which = blockIdx.y;  // 0..2*nlayers-1
  uint8_t* cache = caches.p[which < nlayers ? which : kMaxLayerPtrs + (which - nlayers)];
  const int L = min(path_len[b], num_nodes);
  if (L <= 1) return;
  const int64_t ctx = context_lens[b];
  if (ctx < 0 || (ctx + num_nodes + bs - 1) / bs > max_blocks) {
    if (threadIdx.x == 0 && which == 0) kyro::dev::flag(status, KYRO_DEV_BAD_LENGTH);
    return;
  }
  const int64_t* bt = block_table + (int64_t)b * max_blocks;
  const int row_chunks = d * 2 / 16;
  const int32_t* pb = path + (int64_t)b * num_nodes;
  for (int h = 0; h < hkv; ++h) {
    for (int i = threadIdx.x; i < L * row_chunks; i += blockDim.x) {
      const int n = i / row_chunks, ch = i % row_chunks;
      int node = pb[n];
      if (node < 0 || node >= num_nodes) {
        kyro::dev::flag(status, KYRO_DEV_BAD_LENGTH);
        node = n;
      }
      const int64_t pos = ctx + node;
      const int64_t blk = bt[pos / bs];
      uint4 v = make_uint4(0, 0, 0, 0);
      if (blk >= 0 && blk < num_blocks)
        v = *reinterpret_cast<const uint4*>(cache + (((blk * hkv + h) * bs + pos % bs) * d) * 2 +
                                            ch * 16);
      else
        kyro::dev::flag(status, KYRO_DEV_BAD_BLOCK);
      rows[n * row_chunks + ch] = v;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < L * row_chunks; i += blockDim.x) {
      const int n = i / row_chunks, ch = i % row_chunks;
      if (n == 0 || pb[n] == n) continue;  // already in place
      const int64_t pos = ctx + n;
      const int64_t blk = bt[pos / bs];
      if (blk < 0 || blk >= num_blocks) continue;
      *reinterpret_cast<uint4*>(cache + (((blk * hkv + h) * bs + pos % bs) * d) * 2 + ch * 16) =
          rows[n * row_chunks + ch];
    }
    __syncthreads();
  }
}

// grid (B, 2 * layers): the copy half of a copy-on-write reserve -- every
// slot of the shared block cow[2b] into the fresh block cow[2b+1], in one
// layer's K or V cache.
__global__ void __launch_bounds__(256)
kv_block_copy_kernel(CachePtrs caches, int nlayers, int hkv, int d, int bs, int num_blocks,
                     const int32_t* __restrict__ cow) {
  const int b = blockIdx.x, which = blockIdx.y;
  const int32_t src = cow[2 * b], dst = cow[2 * b + 1];
  if (src < 0 || dst < 0 || src >= num_blocks || dst >= num_blocks) return;
  uint8_t* cache = caches.p[which < nlayers ? which : kMaxLayerPtrs + (which - nlayers)];
  const int64_t n16 = (int64_t)hkv * bs * d * 2 / 16;
  const uint4* s = reinterpret_cast<const uint4*>(cache) + (int64_t)src * n16;
  uint4* t = reinterpret_cast<uint4*>(cache) + (int64_t)dst * n16;
  for (int64_t i = threadIdx.x; i < n16; i += blockDim.x) t[i] = s[i];
}

// grid (B, num_new): one CTA copies the K and V rows of one new token.
__global__ void __launch_bounds__(256)
kv_write_kernel(int num_new, int hkv, int d, int bs, int max_blocks, int num_blocks,
                const uint4* __restrict__ k_new, const uint4* __restrict__ v_new,
                const int64_t* __restrict__ block_table, const int64_t* __restrict__ context_lens,
                uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache, uint32_t* status) {
  const int b = blockIdx.x, j = blockIdx.y;
  kyro::dev::pdl_wait();
  kyro::dev::pdl_trigger();
  const int64_t ctx = context_lens[b];
  const int64_t pos = ctx + j;
  if (ctx < 0 || pos / bs >= max_blocks) {
    if (threadIdx.x == 0) kyro::dev::flag(status, KYRO_DEV_BAD_LENGTH);
    return;
  }
  const int64_t blk = block_table[(int64_t)b * max_blocks + pos / bs];
  if (blk < 0 || blk >= num_blocks) {
    if (threadIdx.x == 0) kyro::dev::flag(status, KYRO_DEV_BAD_BLOCK);
    return;
  }
  const int row_chunks = d * 2 / 16;
  const int64_t src0 = ((int64_t)b * num_new + j) * hkv * row_chunks;
  for (int i = threadIdx.x; i < hkv * row_chunks; i += blockDim.x) {
    const int h = i / row_chunks, ch = i % row_chunks;
    const int64_t dst = (((blk * hkv + h) * bs + pos % bs) * d) * 2 + ch * 16;
    *reinterpret_cast<uint4*>(k_cache + dst) = k_new[src0 + i];
    *reinterpret_cast<uint4*>(v_cache + dst) = v_new[src0 + i];
  }
}

// Rotary position embedding of the new tokens, fused with the paged K/V
// store (LlamaAttention::forward, src/model/llama.rs:77-82, then append_kv);
// the arithmetic is kyro::rope's (rope.cuh).
constexpr int kRopeMaxHalf = 128;  // head_dim <= 256
constexpr int kRopeThreads = 256;
constexpr int kRopePrefetch = 2;   // rotation pieces per thread loaded before the angles

struct RopeArgs {
  int num_new, hq, hkv, d, bs, max_blocks, num_blocks;
  float inv_freq[kRopeMaxHalf];
};

// grid (B, num_new): one CTA rotates the query and key heads of one new
// token, writes the queries to q_out and the rotated keys and the values to
// the token's paged slot.
__global__ void __launch_bounds__(kRopeThreads)
rope_kv_write_kernel(RopeArgs a, const int32_t* __restrict__ pos_offsets,
                     const uint4* q /* q_out may alias it */,
                     const uint4* __restrict__ k_new, const uint4* __restrict__ v_new,
                     const int64_t* __restrict__ block_table,
                     const int64_t* __restrict__ context_lens, uint4* q_out, uint8_t* k_cache,
                     uint8_t* v_cache, uint32_t* status) {
  __shared__ float cs[kRopeMaxHalf], sn[kRopeMaxHalf];
  const int b = blockIdx.x, j = blockIdx.y;
  kyro::dev::pdl_wait();
  kyro::dev::pdl_trigger();
  const int half = a.d / 2;
  const int hv = half / 8;    // 16-byte pieces per half row
  const int row16 = a.d / 8;  // 16-byte pieces per row
  const int64_t tok = (int64_t)b * a.num_new + j;
  const int nrot = (a.hq + a.hkv) * hv;
  const int nv = a.hkv * row16;
  // the inputs do not depend on the position: their loads go out first, and
  // the angles are computed while they are in flight
  uint4 x1[kRopePrefetch], x2[kRopePrefetch], xv;
#pragma unroll
  for (int u = 0; u < kRopePrefetch; ++u) {
    const int it = threadIdx.x + u * blockDim.x;
    if (it < nrot) {
      const int h = it / hv, c = it - h * hv;
      const uint4* src = h < a.hq ? q + (tok * a.hq + h) * row16
                                  : k_new + (tok * a.hkv + (h - a.hq)) * row16;
      x1[u] = src[c];
      x2[u] = src[hv + c];
    }
  }
  if (threadIdx.x < nv) xv = v_new[tok * nv + threadIdx.x];
  const int64_t ctx = context_lens[b];
  const int64_t pos = ctx + j;  // the cache slot
  // the rotary position: (index + i) as f32 (layers.rs:45), index = the
  // sequence's cached length, i = the token's offset (its depth in a tree)
  const float pf = (float)(ctx + (pos_offsets ? pos_offsets[j] : j));
  bool slot_ok = ctx >= 0 && pos / a.bs < a.max_blocks;
  int64_t blk = -1;
  if (slot_ok) blk = block_table[(int64_t)b * a.max_blocks + pos / a.bs];
  for (int i = threadIdx.x; i < half; i += blockDim.x)
    kyro::rope::angle(pf, a.inv_freq[i], cs[i], sn[i]);
  if (slot_ok && (blk < 0 || blk >= a.num_blocks)) {
    if (threadIdx.x == 0) kyro::dev::flag(status, KYRO_DEV_BAD_BLOCK);
    slot_ok = false;
  } else if (!slot_ok && threadIdx.x == 0) {
    kyro::dev::flag(status, KYRO_DEV_BAD_LENGTH);
  }
  __syncthreads();
  for (int it = threadIdx.x, u = 0; it < nrot; it += blockDim.x, ++u) {
    const int h = it / hv, c = it - h * hv;
    const bool is_q = h < a.hq;
    if (!is_q && !slot_ok) continue;
    uint4 v1, v2;
    if (u < kRopePrefetch) {
      // static register indexing: u is 0 or 1 here
      v1 = u == 0 ? x1[0] : x1[kRopePrefetch - 1];
      v2 = u == 0 ? x2[0] : x2[kRopePrefetch - 1];
    } else {
      const uint4* src = is_q ? q + (tok * a.hq + h) * row16
                              : k_new + (tok * a.hkv + (h - a.hq)) * row16;
      v1 = src[c];
      v2 = src[hv + c];
    }
    const uint32_t w1[4] = {v1.x, v1.y, v1.z, v1.w};
    const uint32_t w2[4] = {v2.x, v2.y, v2.z, v2.w};
    uint32_t y1[4], y2[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i0 = c * 8 + 2 * e;
      kyro::rope::rotate_pair(w1[e], w2[e], cs[i0], cs[i0 + 1], sn[i0], sn[i0 + 1], y1[e], y2[e]);
    }
    const uint4 o1 = make_uint4(y1[0], y1[1], y1[2], y1[3]);
    const uint4 o2 = make_uint4(y2[0], y2[1], y2[2], y2[3]);
    uint4* dst = is_q ? q_out + (tok * a.hq + h) * row16
                      : reinterpret_cast<uint4*>(
                            k_cache + (((blk * a.hkv + (h - a.hq)) * a.bs + pos % a.bs) * a.d) * 2);
    dst[c] = o1;
    dst[hv + c] = o2;
  }
  if (!slot_ok) return;
  for (int it = threadIdx.x; it < nv; it += blockDim.x) {
    const int h = it / row16, c = it - h * row16;
    uint4* dst = reinterpret_cast<uint4*>(
        v_cache + (((blk * a.hkv + h) * a.bs + pos % a.bs) * a.d) * 2);
    dst[c] = it == threadIdx.x ? xv : v_new[tok * nv + it];
  }
}

int check_kv(const kyro_kv_params* p, const char* fn) {
  KY_REQUIRE(p, "%s: params is NULL", fn);
  KY_REQUIRE(p->batch >= 0, "%s: batch = %d", fn, p->batch);
  KY_REQUIRE(p->block_size > 0, "%s: block_size = %d", fn, p->block_size);
  KY_REQUIRE(p->max_blocks_per_seq > 0, "%s: max_blocks_per_seq = %d", fn, p->max_blocks_per_seq);
  KY_REQUIRE(p->num_blocks > 0, "%s: num_blocks = %d", fn, p->num_blocks);
  return KYRO_OK;
}

}  // namespace

namespace kyro {
namespace kv {

int check_commit_args(const kyro_kv_params* p, int32_t num_new, int32_t num_new_next,
                      const int32_t* accept_len, const int64_t* block_table,
                      const int64_t* context_lens, const int32_t* free_stack,
                      const int32_t* free_top, const int32_t* ref_counts, const char* what) {
  KY_TRY(check_kv(p, what));
  KY_REQUIRE(num_new >= 0 && num_new_next >= 0, "%s: num_new = %d, num_new_next = %d", what,
             num_new, num_new_next);
  KY_REQUIRE(accept_len && block_table && context_lens && free_stack && free_top && ref_counts,
             "%s: a required KV pointer is NULL", what);
  return KYRO_OK;
}

int launch_commit_reserve(kyro_ctx* ctx, const kyro_kv_params* p, int32_t num_new,
                          int32_t num_new_next, const int32_t* accept_len, int64_t* block_table,
                          int64_t* context_lens, int32_t* free_stack, int32_t* free_top,
                          int32_t* ref_counts, int32_t* out_ok) {
  if (p->batch == 0) return KYRO_OK;
  // a CTA no larger than the batch: it launches between the acceptance's
  // decide and final kernels and must find room on an SM beside them
  const int threads = std::min(kTile, std::max(32, (p->batch + 31) / 32 * 32));
  return kyro::launch_pdl(kv_commit_reserve_kernel, dim3(1), dim3(threads), 0, ctx->stream,
                          "kv_commit_reserve_kernel", p->batch, p->block_size,
                          p->max_blocks_per_seq, p->num_blocks, (int)num_new, (int)num_new_next,
                          accept_len, block_table, context_lens, free_stack, free_top,
                          ref_counts, out_ok, ctx->d_status);
}

}  // namespace kv
}  // namespace kyro

extern "C" {

int kyro_kv_reserve(kyro_ctx* ctx, const kyro_kv_params* p, int32_t num_new,
                    int64_t* block_table, const int64_t* context_lens, int32_t* free_stack,
                    int32_t* free_top, int32_t* ref_counts, int32_t* out_ok) {
  KY_NVTX("kyro_kv_reserve");
  KY_TRY(kyro::enter(ctx));
  KY_TRY(check_kv(p, "kyro_kv_reserve"));
  KY_REQUIRE(num_new >= 0, "kyro_kv_reserve: num_new = %d", num_new);
  if (p->batch == 0) return KYRO_OK;
  KY_REQUIRE(block_table && context_lens && free_stack && free_top && ref_counts,
             "kyro_kv_reserve: a required pointer is NULL");
  return kyro::launch_pdl(kv_reserve_kernel<false>, dim3(1), dim3(kTile), 0, ctx->stream,
                          "kv_reserve_kernel", p->batch, p->block_size, p->max_blocks_per_seq,
                          p->num_blocks, num_new, block_table, context_lens,
                          (const int32_t*)free_stack, free_top, ref_counts, out_ok,
                          (int32_t*)nullptr, ctx->d_status);
}

int kyro_kv_commit(kyro_ctx* ctx, const kyro_kv_params* p, int32_t num_new,
                   const int32_t* accept_len, int64_t* block_table, int64_t* context_lens,
                   int32_t* free_stack, int32_t* free_top, int32_t* ref_counts) {
  KY_NVTX("kyro_kv_commit");
  KY_TRY(kyro::enter(ctx));
  KY_TRY(check_kv(p, "kyro_kv_commit"));
  KY_REQUIRE(num_new >= 0, "kyro_kv_commit: num_new = %d", num_new);
  if (p->batch == 0) return KYRO_OK;
  KY_REQUIRE(accept_len && block_table && context_lens && free_stack && free_top && ref_counts,
             "kyro_kv_commit: a required pointer is NULL");
  return kyro::launch_pdl(kv_commit_kernel, dim3(1), dim3(kTile), 0, ctx->stream,
                          "kv_commit_kernel", p->batch, p->block_size, p->max_blocks_per_seq,
                          p->num_blocks, num_new, accept_len, (const int32_t*)nullptr, block_table,
                          context_lens, free_stack, free_top, ref_counts, ctx->d_status);
}

int kyro_kv_write(kyro_ctx* ctx, const kyro_kv_params* p, int32_t num_new, int32_t num_kv_heads,
                  int32_t head_dim, const void* k_new, const void* v_new,
                  const int64_t* block_table, const int64_t* context_lens, void* k_cache,
                  void* v_cache) {
  KY_NVTX("kyro_kv_write");
  KY_TRY(kyro::enter(ctx));
  KY_TRY(check_kv(p, "kyro_kv_write"));
  KY_REQUIRE(num_new >= 0 && num_new <= 65535, "kyro_kv_write: num_new = %d", num_new);
  KY_REQUIRE(num_kv_heads > 0 && head_dim > 0 && (head_dim * 2) % 16 == 0,
             "kyro_kv_write: num_kv_heads %d head_dim %d", num_kv_heads, head_dim);
  if (p->batch == 0 || num_new == 0) return KYRO_OK;
  KY_REQUIRE(k_new && v_new && block_table && context_lens && k_cache && v_cache,
             "kyro_kv_write: a required pointer is NULL");
  KY_REQUIRE((uintptr_t)k_new % 16 == 0 && (uintptr_t)v_new % 16 == 0 &&
                 (uintptr_t)k_cache % 16 == 0 && (uintptr_t)v_cache % 16 == 0,
             "kyro_kv_write: tensors must be 16-byte aligned");
  dim3 grid((unsigned)p->batch, (unsigned)num_new);
  return kyro::launch_pdl(kv_write_kernel, grid, dim3(256), 0, ctx->stream, "kv_write_kernel",
                          (int)num_new, (int)num_kv_heads, (int)head_dim, p->block_size,
                          p->max_blocks_per_seq, p->num_blocks, (const uint4*)k_new,
                          (const uint4*)v_new, block_table, context_lens, (uint8_t*)k_cache,
                          (uint8_t*)v_cache, ctx->d_status);
}

int kyro_kv_commit_tree(kyro_ctx* ctx, const kyro_kv_params* p, int32_t num_nodes,
                        const int32_t* path, const int32_t* path_len, int32_t num_layers,
                        void* const* k_caches, void* const* v_caches, int32_t num_kv_heads,
                        int32_t head_dim, int64_t* block_table, int64_t* context_lens,
                        int32_t* free_stack, int32_t* free_top, int32_t* ref_counts) {
  KY_NVTX("kyro_kv_commit_tree");
  KY_TRY(kyro::enter(ctx));
  KY_TRY(check_kv(p, "kyro_kv_commit_tree"));
  KY_REQUIRE(num_nodes >= 1 && num_nodes <= 64, "kyro_kv_commit_tree: num_nodes = %d (1..64)",
             num_nodes);
  KY_REQUIRE(num_layers >= 0, "kyro_kv_commit_tree: num_layers = %d", num_layers);
  KY_REQUIRE(num_kv_heads > 0 && head_dim > 0 && head_dim <= 256 && (head_dim * 2) % 16 == 0,
             "kyro_kv_commit_tree: num_kv_heads %d head_dim %d (head_dim*2 must be a multiple "
             "of 16)",
             num_kv_heads, head_dim);
  if (p->batch == 0) return KYRO_OK;
  KY_REQUIRE(path && path_len && block_table && context_lens && free_stack && free_top &&
                 ref_counts,
             "kyro_kv_commit_tree: a required pointer is NULL");
  KY_REQUIRE(num_layers == 0 || (k_caches && v_caches), "kyro_kv_commit_tree: cache arrays NULL");
  KY_REQUIRE(p->batch <= 65535 * 32, "kyro_kv_commit_tree: batch too large");
  const size_t smem = (size_t)num_nodes * head_dim * 2;
  for (int l0 = 0; l0 < num_layers; l0 += kMaxLayerPtrs) {
    const int nl = min(kMaxLayerPtrs, num_layers - l0);
    CachePtrs cp = {};
    for (int i = 0; i < nl; ++i) {
      KY_REQUIRE(k_caches[l0 + i] && v_caches[l0 + i] &&
                     (uintptr_t)k_caches[l0 + i] % 16 == 0 && (uintptr_t)v_caches[l0 + i] % 16 == 0,
                 "kyro_kv_commit_tree: layer %d cache pointer NULL or not 16-byte aligned", l0 + i);
      cp.p[i] = (uint8_t*)k_caches[l0 + i];
      cp.p[kMaxLayerPtrs + i] = (uint8_t*)v_caches[l0 + i];
    }
    dim3 grid((unsigned)p->batch, (unsigned)(2 * nl));
    kv_tree_move_kernel<<<grid, 256, smem, ctx->stream>>>(
        cp, nl, num_nodes, num_kv_heads, head_dim, p->block_size, p->max_blocks_per_seq,
        p->num_blocks, path, path_len, block_table, context_lens, ctx->d_status);
    KY_TRY(kyro::check_launch("kv_tree_move_kernel"));
  }
  kv_commit_kernel<<<1, kTile, 0, ctx->stream>>>(p->batch, p->block_size, p->max_blocks_per_seq,
                                                 p->num_blocks, num_nodes, nullptr, path_len,
                                                 block_table, context_lens, free_stack, free_top,
                                                 ref_counts, ctx->d_status);
  return kyro::check_launch("kv_commit_kernel");
}

int kyro_rope_kv_write(kyro_ctx* ctx, const kyro_kv_params* p, int32_t num_new,
                       int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                       float rope_theta, const int32_t* pos_offsets, const void* q,
                       const void* k_new, const void* v_new, const int64_t* block_table,
                       const int64_t* context_lens, void* q_out, void* k_cache, void* v_cache) {
  KY_NVTX("kyro_rope_kv_write");
  KY_TRY(kyro::enter(ctx));
  KY_TRY(check_kv(p, "kyro_rope_kv_write"));
  KY_REQUIRE(num_new >= 0 && num_new <= 65535, "kyro_rope_kv_write: num_new = %d", num_new);
  KY_REQUIRE(num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0,
             "kyro_rope_kv_write: num_heads %d num_kv_heads %d", num_heads, num_kv_heads);
  KY_REQUIRE(head_dim > 0 && head_dim % 16 == 0 && head_dim / 2 <= kRopeMaxHalf,
             "kyro_rope_kv_write: head_dim %d (a multiple of 16, at most %d)", head_dim,
             2 * kRopeMaxHalf);
  KY_REQUIRE(rope_theta > 0.0f, "kyro_rope_kv_write: rope_theta = %g", (double)rope_theta);
  if (p->batch == 0 || num_new == 0) return KYRO_OK;
  KY_REQUIRE(q && k_new && v_new && block_table && context_lens && q_out && k_cache && v_cache,
             "kyro_rope_kv_write: a required pointer is NULL");
  KY_REQUIRE((uintptr_t)q % 16 == 0 && (uintptr_t)k_new % 16 == 0 && (uintptr_t)v_new % 16 == 0 &&
                 (uintptr_t)q_out % 16 == 0 && (uintptr_t)k_cache % 16 == 0 &&
                 (uintptr_t)v_cache % 16 == 0,
             "kyro_rope_kv_write: tensors must be 16-byte aligned");
  RopeArgs a;
  a.num_new = num_new;
  a.hq = num_heads;
  a.hkv = num_kv_heads;
  a.d = head_dim;
  a.bs = p->block_size;
  a.max_blocks = p->max_blocks_per_seq;
  a.num_blocks = p->num_blocks;
  // RotaryEmbedding::new (layers.rs:26-33): 1 / theta^(2i/D) in double, then fp32
  for (int i = 0; i < kRopeMaxHalf; ++i)
    a.inv_freq[i] = i < head_dim / 2
                        ? (float)(1.0 / std::pow((double)rope_theta, 2.0 * i / head_dim))
                        : 0.0f;
  dim3 grid((unsigned)p->batch, (unsigned)num_new);
  return kyro::launch_pdl(rope_kv_write_kernel, grid, dim3(kRopeThreads), 0, ctx->stream,
                          "rope_kv_write_kernel", a, pos_offsets, (const uint4*)q,
                          (const uint4*)k_new, (const uint4*)v_new, block_table, context_lens,
                          (uint4*)q_out, (uint8_t*)k_cache, (uint8_t*)v_cache, ctx->d_status);
}

int kyro_kv_reserve_cow(kyro_ctx* ctx, const kyro_kv_params* p, int32_t num_new,
                        int32_t num_layers, void* const* k_caches, void* const* v_caches,
                        int32_t num_kv_heads, int32_t head_dim, int64_t* block_table,
                        const int64_t* context_lens, int32_t* free_stack, int32_t* free_top,
                        int32_t* ref_counts, int32_t* out_ok, int32_t* out_cow) {
  KY_NVTX("kyro_kv_reserve_cow");
  KY_TRY(kyro::enter(ctx));
  KY_TRY(check_kv(p, "kyro_kv_reserve_cow"));
  KY_REQUIRE(num_new >= 0, "kyro_kv_reserve_cow: num_new = %d", num_new);
  KY_REQUIRE(num_layers >= 0, "kyro_kv_reserve_cow: num_layers = %d", num_layers);
  KY_REQUIRE(num_kv_heads > 0 && head_dim > 0 && (head_dim * 2) % 16 == 0,
             "kyro_kv_reserve_cow: num_kv_heads %d head_dim %d (head_dim*2 must be a multiple "
             "of 16)",
             num_kv_heads, head_dim);
  if (p->batch == 0) return KYRO_OK;
  KY_REQUIRE(block_table && context_lens && free_stack && free_top && ref_counts && out_cow,
             "kyro_kv_reserve_cow: a required pointer is NULL");
  KY_REQUIRE(num_layers == 0 || (k_caches && v_caches), "kyro_kv_reserve_cow: cache arrays NULL");
  KY_REQUIRE(p->batch <= 2147483647 / 2, "kyro_kv_reserve_cow: batch too large");
  for (int i = 0; i < num_layers; ++i)
    KY_REQUIRE(k_caches[i] && v_caches[i] && (uintptr_t)k_caches[i] % 16 == 0 &&
                   (uintptr_t)v_caches[i] % 16 == 0,
               "kyro_kv_reserve_cow: layer %d cache pointer NULL or not 16-byte aligned", i);
  KY_TRY(kyro::launch_pdl(kv_reserve_kernel<true>, dim3(1), dim3(kTile), 0, ctx->stream,
                          "kv_reserve_kernel", p->batch, p->block_size, p->max_blocks_per_seq,
                          p->num_blocks, num_new, block_table, context_lens,
                          (const int32_t*)free_stack, free_top, ref_counts, out_ok, out_cow,
                          ctx->d_status));
  for (int l0 = 0; l0 < num_layers; l0 += kMaxLayerPtrs) {
    const int nl = min(kMaxLayerPtrs, num_layers - l0);
    CachePtrs cp = {};
    for (int i = 0; i < nl; ++i) {
      cp.p[i] = (uint8_t*)k_caches[l0 + i];
      cp.p[kMaxLayerPtrs + i] = (uint8_t*)v_caches[l0 + i];
    }
    dim3 grid((unsigned)p->batch, (unsigned)(2 * nl));
    kv_block_copy_kernel<<<grid, 256, 0, ctx->stream>>>(cp, nl, num_kv_heads, head_dim,
                                                        p->block_size, p->num_blocks, out_cow);
    KY_TRY(kyro::check_launch("kv_block_copy_kernel"));
  }
  return KYRO_OK;
}

}  // extern "C"
