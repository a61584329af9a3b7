/*
 * block_manager.c -- CPU restatement of the KV slot bookkeeping
 * (TEST INFRASTRUCTURE: the checker for the sm_100a commit kernels).
 *
 * Mirrors BlockManager, src/scheduler/block_manager.rs:
 *   free list is a Vec popped from the back        (:36, :92-98, :115-121)
 *   a newly allocated block gets ref_count = 1      (:97, :120)
 *   allocation fails as a whole when too few blocks are free (:111-113)
 *   release decrements ref_count and returns the block to the free list
 *   when it reaches zero, in table order            (:133-150)
 * The reference never grows a sequence after its prompt and never rolls
 * back; reserve/commit apply the same rules to the k+1 verify slots.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "kyro_oracle.h"

static int64_t blocks_for(int64_t tokens, int32_t bs) { return (tokens + bs - 1) / bs; }

void ko_kv_reserve(int32_t batch, int32_t bs, int32_t max_blocks, int32_t num_blocks,
                   int32_t num_new, int64_t* block_table, const int64_t* context_lens,
                   int32_t* free_stack, int32_t* free_top, int32_t* ref_counts,
                   int32_t* out_ok) {
  int32_t top = *free_top;
  for (int32_t b = 0; b < batch; ++b) {
    int64_t have = blocks_for(context_lens[b], bs);
    int64_t want = blocks_for(context_lens[b] + num_new, bs);
    int64_t need = want - have;
    if (want > max_blocks || need > top) {
      if (out_ok) out_ok[b] = 0;
      continue;
    }
    for (int64_t i = 0; i < need; ++i) {
      int32_t blk = free_stack[--top];
      if (blk < 0 || blk >= num_blocks) continue; /* the kernel flags KYRO_DEV_BAD_BLOCK */
      ref_counts[blk] = 1;
      block_table[(size_t)b * max_blocks + have + i] = blk;
    }
    if (out_ok) out_ok[b] = 1;
  }
  *free_top = top;
}

/* kv_reserve with copy-on-write of a shared, partly filled last block (the
 * prefix blocks allocate_with_prefix hands out with ref_count += 1,
 * block_manager.rs:60-63): in batch order, such a sequence first pops a
 * fresh block for it (ref 1, the shared block's ref count - 1, the table
 * entry replaced, every layer's K/V slots of the block copied), then its new
 * blocks as ko_kv_reserve does.  cow[2b], cow[2b+1] = (shared, fresh) or -1. */
void ko_kv_reserve_cow(int32_t batch, int32_t bs, int32_t max_blocks, int32_t num_blocks,
                       int32_t num_new, int32_t num_layers, uint16_t* const* k_caches,
                       uint16_t* const* v_caches, int32_t hkv, int32_t d, int64_t* block_table,
                       const int64_t* context_lens, int32_t* free_stack, int32_t* free_top,
                       int32_t* ref_counts, int32_t* out_ok, int32_t* cow) {
  int32_t top = *free_top;
  size_t block_elems = (size_t)hkv * bs * d;
  for (int32_t b = 0; b < batch; ++b) {
    int64_t len = context_lens[b];
    int64_t have = blocks_for(len, bs);
    int64_t want = blocks_for(len + num_new, bs);
    int64_t need = want - have;
    int64_t old = -1;
    cow[2 * b] = cow[2 * b + 1] = -1;
    if (len >= 0 && want <= max_blocks && len % bs != 0) {
      int64_t o = block_table[(size_t)b * max_blocks + have - 1];
      if (o >= 0 && o < num_blocks && ref_counts[o] > 1) old = o;
    }
    if (len < 0 || want > max_blocks || need + (old >= 0) > top) {
      if (out_ok) out_ok[b] = 0;
      continue;
    }
    if (old >= 0) {
      int32_t blk = free_stack[--top];
      if (blk >= 0 && blk < num_blocks) {
        ref_counts[blk] = 1;
        ref_counts[old] -= 1;
        block_table[(size_t)b * max_blocks + have - 1] = blk;
        cow[2 * b] = (int32_t)old;
        cow[2 * b + 1] = blk;
        for (int32_t l = 0; l < num_layers; ++l) {
          memcpy(k_caches[l] + (size_t)blk * block_elems, k_caches[l] + (size_t)old * block_elems,
                 sizeof(uint16_t) * block_elems);
          memcpy(v_caches[l] + (size_t)blk * block_elems, v_caches[l] + (size_t)old * block_elems,
                 sizeof(uint16_t) * block_elems);
        }
      }
    }
    for (int64_t i = 0; i < need; ++i) {
      int32_t blk = free_stack[--top];
      if (blk < 0 || blk >= num_blocks) continue;
      ref_counts[blk] = 1;
      block_table[(size_t)b * max_blocks + have + i] = blk;
    }
    if (out_ok) out_ok[b] = 1;
  }
  *free_top = top;
}

static void release_tail(int32_t b, int32_t bs, int32_t max_blocks, int32_t num_blocks,
                         int64_t old_len,
                         int64_t reserved_len, int64_t new_len, int64_t* block_table,
                         int32_t* free_stack, int32_t* top, int32_t* ref_counts) {
  (void)old_len;
  int64_t keep = blocks_for(new_len, bs);
  int64_t had = blocks_for(reserved_len, bs);
  if (had > max_blocks) had = max_blocks;
  for (int64_t i = keep; i < had; ++i) {
    int64_t* slot = &block_table[(size_t)b * max_blocks + i];
    int64_t blk = *slot;
    *slot = -1;
    if (blk < 0 || blk >= num_blocks) continue;
    if (ref_counts[blk] > 0) ref_counts[blk] -= 1;
    if (ref_counts[blk] == 0 && *top < num_blocks) free_stack[(*top)++] = (int32_t)blk;
  }
}

void ko_kv_commit(int32_t batch, int32_t bs, int32_t max_blocks, int32_t num_blocks,
                  int32_t num_new, const int32_t* accept_len, int64_t* block_table,
                  int64_t* context_lens, int32_t* free_stack, int32_t* free_top,
                  int32_t* ref_counts) {
  int32_t top = *free_top;
  for (int32_t b = 0; b < batch; ++b) {
    int32_t a = accept_len[b];
    if (a < 0) continue;
    int64_t kept = (int64_t)a + 1 < num_new ? (int64_t)a + 1 : num_new;
    int64_t old_len = context_lens[b];
    int64_t new_len = old_len + kept;
    release_tail(b, bs, max_blocks, num_blocks, old_len, old_len + num_new, new_len, block_table,
                 free_stack, &top, ref_counts);
    context_lens[b] = new_len;
  }
  *free_top = top;
}

void ko_kv_commit_tree(int32_t batch, int32_t bs, int32_t max_blocks, int32_t num_blocks,
                       int32_t num_nodes, const int32_t* path, const int32_t* path_len,
                       int32_t num_layers, uint16_t* const* k_caches, uint16_t* const* v_caches,
                       int32_t hkv, int32_t d, int64_t* block_table, int64_t* context_lens,
                       int32_t* free_stack, int32_t* free_top, int32_t* ref_counts) {
  /* 1. move the accepted path's K/V rows to consecutive positions (read all
   *    sources before writing any destination) */
  size_t row = (size_t)d;
  uint16_t* tmp = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)num_nodes * hkv * row);
  for (int32_t b = 0; b < batch; ++b) {
    int32_t L = path_len[b] < num_nodes ? path_len[b] : num_nodes;
    if (L <= 1) continue;
    int64_t ctx = context_lens[b];
    for (int32_t layer = 0; layer < num_layers; ++layer) {
      for (int32_t which = 0; which < 2; ++which) {
        uint16_t* cache = which ? v_caches[layer] : k_caches[layer];
        for (int32_t i = 0; i < L; ++i) {
          int32_t node = path[(size_t)b * num_nodes + i];
          if (node < 0 || node >= num_nodes) node = i;
          int64_t pos = ctx + node;
          int64_t blk = block_table[(size_t)b * max_blocks + pos / bs];
          if (blk < 0 || blk >= num_blocks) {
            memset(tmp + (size_t)i * hkv * row, 0, sizeof(uint16_t) * hkv * row);
            continue;
          }
          for (int32_t h = 0; h < hkv; ++h)
            memcpy(tmp + ((size_t)i * hkv + h) * row,
                   cache + (((size_t)blk * hkv + h) * bs + (size_t)(pos % bs)) * row,
                   sizeof(uint16_t) * row);
        }
        for (int32_t i = 1; i < L; ++i) {
          if (path[(size_t)b * num_nodes + i] == i) continue; /* already in place */
          int64_t pos = ctx + i;
          int64_t blk = block_table[(size_t)b * max_blocks + pos / bs];
          if (blk < 0 || blk >= num_blocks) continue;
          for (int32_t h = 0; h < hkv; ++h)
            memcpy(cache + (((size_t)blk * hkv + h) * bs + (size_t)(pos % bs)) * row,
                   tmp + ((size_t)i * hkv + h) * row, sizeof(uint16_t) * row);
        }
      }
    }
  }
  free(tmp);
  /* 2. commit path_len slots */
  int32_t* acc = (int32_t*)malloc(sizeof(int32_t) * (size_t)(batch > 0 ? batch : 1));
  for (int32_t b = 0; b < batch; ++b) acc[b] = path_len[b] > 0 ? path_len[b] - 1 : -1;
  ko_kv_commit(batch, bs, max_blocks, num_blocks, num_nodes, acc, block_table, context_lens,
               free_stack, free_top, ref_counts);
  free(acc);
}

void ko_kv_write(int32_t batch, int32_t bs, int32_t max_blocks, int32_t num_blocks,
                 int32_t num_new, int32_t hkv, int32_t d, const uint16_t* k_new,
                 const uint16_t* v_new, const int64_t* block_table, const int64_t* context_lens,
                 uint16_t* k_cache, uint16_t* v_cache) {
  /* KVCacheManager::append_kv (src/model/kv_cache.rs:49-75) appends the
   * [batch, seq, Hkv, D] rows after the cached ones; here each row goes to
   * its paged slot context_len + j. */
  for (int32_t b = 0; b < batch; ++b) {
    int64_t ctx = context_lens[b];
    for (int32_t j = 0; j < num_new; ++j) {
      int64_t pos = ctx + j;
      if (ctx < 0 || pos / bs >= max_blocks) continue;
      int64_t blk = block_table[(size_t)b * max_blocks + pos / bs];
      if (blk < 0 || blk >= num_blocks) continue;
      for (int32_t h = 0; h < hkv; ++h) {
        size_t src = (((size_t)b * num_new + j) * hkv + h) * (size_t)d;
        size_t dst = (((size_t)blk * hkv + h) * bs + (size_t)(pos % bs)) * (size_t)d;
        memcpy(k_cache + dst, k_new + src, sizeof(uint16_t) * (size_t)d);
        memcpy(v_cache + dst, v_new + src, sizeof(uint16_t) * (size_t)d);
      }
    }
  }
}

/* ---- rotary position embedding + paged K/V store ---------------------- */

static float rope_bf16_to_f32(uint16_t v) {
  uint32_t u = (uint32_t)v << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* fp32 -> bf16, round to nearest even (NaN kept quiet) */
static uint16_t rope_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* One head row: RotaryEmbedding::apply (src/model/layers.rs:37-61) on the
 * [x1 | x2] halves, y = x*cos + cat(-x2, x1)*sin, each product and the sum
 * rounded to fp32 (-ffp-contract=off keeps them unfused). */
static void rope_row(const uint16_t* x, uint16_t* y, int32_t d, const float* cs, const float* sn) {
  int32_t half = d / 2;
  for (int32_t i = 0; i < half; ++i) {
    float a = rope_bf16_to_f32(x[i]), b = rope_bf16_to_f32(x[i + half]);
    float t1 = a * cs[i], t2 = (-b) * sn[i];
    float u1 = b * cs[i], u2 = a * sn[i];
    y[i] = rope_f32_to_bf16(t1 + t2);
    y[i + half] = rope_f32_to_bf16(u1 + u2);
  }
}

void ko_rope_kv_write(int32_t batch, int32_t bs, int32_t max_blocks, int32_t num_blocks,
                      int32_t num_new, int32_t hq, int32_t hkv, int32_t d, float theta,
                      const int32_t* pos_offsets, const uint16_t* q, const uint16_t* k_new,
                      const uint16_t* v_new, const int64_t* block_table,
                      const int64_t* context_lens, uint16_t* q_out, uint16_t* k_cache,
                      uint16_t* v_cache) {
  /* LlamaAttention::forward (src/model/llama.rs:73-82): rope on q and k at
   * index + i, then append_kv; here index = context_lens[b] and the rows go
   * to their paged slots context_len + j. */
  int32_t half = d / 2;
  float inv_freq[128], cs[128], sn[128];
  uint16_t row[256];
  for (int32_t i = 0; i < half; ++i)  /* RotaryEmbedding::new, layers.rs:26-33 */
    inv_freq[i] = (float)(1.0 / pow((double)theta, 2.0 * i / d));
  for (int32_t b = 0; b < batch; ++b) {
    int64_t ctx = context_lens[b];
    for (int32_t j = 0; j < num_new; ++j) {
      float pf = (float)(ctx + (pos_offsets ? pos_offsets[j] : j));
      for (int32_t i = 0; i < half; ++i) {
        float f = pf * inv_freq[i];
        cs[i] = (float)cos((double)f);
        sn[i] = (float)sin((double)f);
      }
      size_t tok = (size_t)b * num_new + j;
      for (int32_t h = 0; h < hq; ++h) {
        rope_row(q + (tok * hq + h) * (size_t)d, row, d, cs, sn);
        memcpy(q_out + (tok * hq + h) * (size_t)d, row, sizeof(uint16_t) * (size_t)d);
      }
      int64_t pos = ctx + j;
      if (ctx < 0 || pos / bs >= max_blocks) continue;
      int64_t blk = block_table[(size_t)b * max_blocks + pos / bs];
      if (blk < 0 || blk >= num_blocks) continue;
      for (int32_t h = 0; h < hkv; ++h) {
        size_t src = (tok * hkv + h) * (size_t)d;
        size_t dst = (((size_t)blk * hkv + h) * bs + (size_t)(pos % bs)) * (size_t)d;
        rope_row(k_new + src, k_cache + dst, d, cs, sn);
        memcpy(v_cache + dst, v_new + src, sizeof(uint16_t) * (size_t)d);
      }
    }
  }
}
