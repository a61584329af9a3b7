/*
 * attention.c -- CPU restatement of paged multi-query verify attention
 * (TEST INFRASTRUCTURE: the checker for the sm_100a attention kernel).
 *
 * Mathematics of PagedAttention::paged_attention_kernel,
 * src/model/attention_kernel.rs:59-136: for every query head h the KV head
 * is h / (Hq/Hkv) (:39-46); the token at position t lives in block
 * block_table[b][t / block_size], slot t % block_size (:89-93); scores are
 * q.k * scale with scale = 1/sqrt(D) (:69, :98-102); softmax over the
 * positions (:112); output = sum of weights * V (:116-130).  The
 * reference's reinterpretation of its score buffer (:104-111) mixes heads;
 * this restatement computes the intended per-head softmax instead.
 *
 * Generalised to num_query positions per sequence: query j sits at
 * position context_len + j and sees every cached position plus new
 * position i iff bit i of its mask is set (chain default: i <= j).
 * Accumulation is in double precision.
 */
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include "kyro_oracle.h"

static float bf16_to_float(uint16_t v) {
  uint32_t u = (uint32_t)v << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

typedef struct {
  int32_t batch, nq, hq, hkv, d, bs, max_blocks;
  float scale;
  const uint16_t *q, *k_cache, *v_cache;
  const int64_t* block_table;
  const int64_t* context_lens;
  const uint64_t* tree_mask;
  float* out;
  int32_t w0, w1; /* work range over (b, h) pairs */
} attn_job;

static void* attn_thread(void* arg) {
  const attn_job* J = (const attn_job*)arg;
  const int32_t group = J->hq / J->hkv;
  double* sc = NULL;
  size_t sc_cap = 0;
  double* acc = (double*)malloc(sizeof(double) * (size_t)J->d);
  float* qf = (float*)malloc(sizeof(float) * (size_t)J->d);
  for (int32_t w = J->w0; w < J->w1; ++w) {
    int32_t b = w / J->hq, h = w % J->hq;
    int32_t kvh = h / group;
    int64_t ctx = J->context_lens[b];
    int64_t total = ctx + J->nq;
    if ((size_t)total > sc_cap) {
      sc_cap = (size_t)total;
      sc = (double*)realloc(sc, sizeof(double) * sc_cap);
    }
    for (int32_t j = 0; j < J->nq; ++j) {
      const uint16_t* qrow = J->q + (((size_t)b * J->nq + j) * J->hq + h) * J->d;
      for (int32_t e = 0; e < J->d; ++e) qf[e] = bf16_to_float(qrow[e]);
      uint64_t mask = J->tree_mask ? J->tree_mask[(size_t)b * J->nq + j]
                                   : (j >= 63 ? ~0ull : ((1ull << (j + 1)) - 1ull));
      double mx = -INFINITY;
      for (int64_t t = 0; t < total; ++t) {
        int allowed = t < ctx || ((mask >> (t - ctx)) & 1ull);
        if (!allowed) {
          sc[t] = -INFINITY;
          continue;
        }
        int64_t blk = J->block_table[(size_t)b * J->max_blocks + t / J->bs];
        const uint16_t* krow =
            J->k_cache + (((size_t)blk * J->hkv + kvh) * J->bs + (size_t)(t % J->bs)) * J->d;
        double s = 0.0;
        for (int32_t e = 0; e < J->d; ++e) s += (double)qf[e] * (double)bf16_to_float(krow[e]);
        s *= (double)J->scale;
        sc[t] = s;
        if (s > mx) mx = s;
      }
      double l = 0.0;
      for (int32_t e = 0; e < J->d; ++e) acc[e] = 0.0;
      for (int64_t t = 0; t < total; ++t) {
        if (sc[t] == -INFINITY) continue;
        double p = exp(sc[t] - mx);
        l += p;
        int64_t blk = J->block_table[(size_t)b * J->max_blocks + t / J->bs];
        const uint16_t* vrow =
            J->v_cache + (((size_t)blk * J->hkv + kvh) * J->bs + (size_t)(t % J->bs)) * J->d;
        for (int32_t e = 0; e < J->d; ++e) acc[e] += p * (double)bf16_to_float(vrow[e]);
      }
      float* orow = J->out + (((size_t)b * J->nq + j) * J->hq + h) * J->d;
      for (int32_t e = 0; e < J->d; ++e) orow[e] = l > 0.0 ? (float)(acc[e] / l) : 0.0f;
    }
  }
  free(sc);
  free(acc);
  free(qf);
  return NULL;
}

void ko_paged_attention(int32_t batch, int32_t nq, int32_t hq, int32_t hkv, int32_t d,
                        int32_t bs, int32_t max_blocks, float scale, const uint16_t* q,
                        const uint16_t* k_cache, const uint16_t* v_cache,
                        const int64_t* block_table, const int64_t* context_lens,
                        const uint64_t* tree_mask, float* out, int32_t nthreads) {
  int32_t work = batch * hq;
  int32_t nt = nthreads < 1 ? 1 : nthreads;
  if (nt > work) nt = work > 0 ? work : 1;
  attn_job* jobs = (attn_job*)calloc((size_t)nt, sizeof(attn_job));
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nt);
  for (int32_t t = 0; t < nt; ++t) {
    attn_job J = {batch, nq, hq, hkv, d, bs, max_blocks, scale, q, k_cache, v_cache,
                  block_table, context_lens, tree_mask, out,
                  (int32_t)((int64_t)work * t / nt), (int32_t)((int64_t)work * (t + 1) / nt)};
    jobs[t] = J;
  }
  for (int32_t t = 1; t < nt; ++t) pthread_create(&th[t], NULL, attn_thread, &jobs[t]);
  attn_thread(&jobs[0]);
  for (int32_t t = 1; t < nt; ++t) pthread_join(th[t], NULL);
  free(th);
  free(jobs);
}
