/*
 * sampler.c -- CPU restatement of the acceptance step (TEST INFRASTRUCTURE:
 * the checker for the sm_100a sampler kernels, never the shipped path).
 *
 * Rules restated:
 *   greedy verify       src/speculative.rs:296-305 (k == 0), :314-323
 *   sampling helpers    src/worker.rs:290-296 (argmax), :298 (logits / T),
 *                       :314-323 (max-subtracted softmax), :352-360
 *                       (inverse CDF, first id where the running remainder
 *                       reaches <= 0)
 *   rejection sampling  Leviathan et al. 2023, Alg. 1; Chen et al. 2023
 * Arithmetic (exp, fixed-point sums, Philox) comes from kyro_math.h so that
 * the oracle and the kernels decide identically.
 */
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include "kyro_math.h"
#include "kyro_oracle.h"

#define KO_MODE_STOCHASTIC 0
#define KO_MODE_GREEDY 1
#define KO_MODE_GREEDY_REF 2

void ko_philox4x32_10(const uint32_t ctr[4], uint64_t key, uint32_t out[4]) {
  ky_philox4x32_10(ctr, (uint32_t)key, (uint32_t)(key >> 32), out);
}

float ko_uniform(uint64_t seed, uint32_t seq, uint32_t pos, uint32_t stream, uint32_t step) {
  return ky_odd_to_float(ky_uniform_odd(seed, seq, pos, stream, step));
}

float ko_exp(float x) { return ky_exp(x); }

/* ------------------------------------------------------------------ */
/* row statistics under the normaliser contract (kyro_math.h)          */
/* ------------------------------------------------------------------ */
typedef struct {
  const float* row;
  int32_t vocab, num_shards, shard_len, chunks_per_shard;
  float inv_t;
  float* m;    /* per chunk max of s                        */
  float* g;    /* per chunk probability scale g_c            */
  float* g62;  /* g_c * 2^62                                 */
  float M;
  double S;
} ko_rowstat;

static int32_t chunk_of(const ko_rowstat* st, int32_t i) {
  int32_t r = i / st->shard_len;
  int32_t local = i - r * st->shard_len;
  return r * st->chunks_per_shard + local / KY_CHUNK;
}

static void rowstat_init(ko_rowstat* st, const float* row, int32_t vocab, int32_t num_shards,
                         float inv_t) {
  st->row = row;
  st->vocab = vocab;
  st->num_shards = num_shards;
  st->shard_len = vocab / num_shards;
  st->chunks_per_shard = (st->shard_len + KY_CHUNK - 1) / KY_CHUNK;
  st->inv_t = inv_t;
  int32_t nc = st->chunks_per_shard * num_shards;
  st->m = (float*)malloc(sizeof(float) * (size_t)nc);
  st->g = (float*)malloc(sizeof(float) * (size_t)nc);
  st->g62 = (float*)malloc(sizeof(float) * (size_t)nc);
  float* E = (float*)malloc(sizeof(float) * (size_t)nc);
  /* chunk maxima */
  for (int32_t c = 0; c < nc; ++c) st->m[c] = -INFINITY;
  for (int32_t i = 0; i < vocab; ++i) {
    float s = KY_FMUL(row[i], inv_t);
    int32_t c = chunk_of(st, i);
    if (s > st->m[c]) st->m[c] = s;
  }
  /* chunk sums: every position of a chunk, -inf past the shard end */
  for (int32_t r = 0; r < num_shards; ++r) {
    for (int32_t lc = 0; lc < st->chunks_per_shard; ++lc) {
      int32_t gc = r * st->chunks_per_shard + lc;
      float e[KY_CHUNK];
      for (int32_t p = 0; p < KY_CHUNK; ++p) {
        int32_t local = lc * KY_CHUNK + p;
        float s = local < st->shard_len ? KY_FMUL(row[r * st->shard_len + local], inv_t) : -INFINITY;
        e[p] = ky_exp(KY_FSUB(s, st->m[gc]));
      }
      E[gc] = ky_chunk_sum(e);
    }
  }
  /* shard maxima M_r, the row max M, and each shard's part under its own
   * maximum, brought to M in rank order (kyro_math.h) */
  float* Mr = (float*)malloc(sizeof(float) * (size_t)num_shards);
  float M = -INFINITY;
  for (int32_t r = 0; r < num_shards; ++r) {
    Mr[r] = -INFINITY;
    for (int32_t c = 0; c < st->chunks_per_shard; ++c) {
      int32_t gc = r * st->chunks_per_shard + c;
      if (st->m[gc] > Mr[r]) Mr[r] = st->m[gc];
    }
    if (Mr[r] > M) M = Mr[r];
  }
  double S = 0.0;
  for (int32_t r = 0; r < num_shards; ++r) {
    double t[32];
    for (int32_t l = 0; l < 32; ++l) {
      t[l] = 0.0;
      for (int32_t c = l; c < st->chunks_per_shard; c += 32) {
        int32_t gc = r * st->chunks_per_shard + c;
        t[l] = KY_DADD(t[l], ky_chunk_mass(E[gc], st->m[gc], Mr[r]));
      }
    }
    S = KY_DADD(S, KY_DMUL(ky_butterfly32(t), ky_shard_scale(Mr[r], M)));
  }
  free(Mr);
  for (int32_t c = 0; c < nc; ++c) {
    st->g[c] = ky_chunk_scale(st->m[c], M, S);
    st->g62[c] = ky_scale62(st->g[c]);
  }
  st->M = M;
  st->S = S;
  free(E);
}

static void rowstat_free(ko_rowstat* st) {
  free(st->m);
  free(st->g);
  free(st->g62);
}

static float rowstat_e(const ko_rowstat* st, int32_t i) {
  int32_t c = chunk_of(st, i);
  return ky_exp(KY_FSUB(KY_FMUL(st->row[i], st->inv_t), st->m[c]));
}

/* inverse-CDF weight of entry i for sampling from p */
static uint64_t rowstat_wp(const ko_rowstat* st, int32_t i) {
  return ky_weight_p(rowstat_e(st, i), st->g62[chunk_of(st, i)]);
}

static float rowstat_p(const ko_rowstat* st, int32_t i) {
  int32_t c = chunk_of(st, i);
  float s = KY_FMUL(st->row[i], st->inv_t);
  return KY_FMUL(ky_exp(KY_FSUB(s, st->m[c])), st->g[c]);
}

static int32_t argmax_row(const float* row, int32_t vocab) {
  int32_t best = 0;
  float bv = row[0];
  for (int32_t i = 1; i < vocab; ++i)
    if (row[i] > bv) {
      bv = row[i];
      best = i;
    }
  return best;
}

/* smallest i with inclusive prefix sum of w >= threshold(odd, W);
 * the last index when W == 0 (worker.rs:361 falls back to the last id). */
static int32_t inverse_cdf(const uint64_t* w, int32_t n, uint32_t odd) {
  uint64_t W = 0;
  for (int32_t i = 0; i < n; ++i) W += w[i];
  if (W == 0) return n - 1;
  uint64_t T = ky_cdf_threshold(odd, W);
  uint64_t C = 0;
  for (int32_t i = 0; i < n; ++i) {
    C += w[i];
    if (C >= T) return i;
  }
  return n - 1;
}

void ko_softmax_row(const float* row, int32_t vocab, int32_t num_shards, float temperature,
                    float* out_p) {
  ko_rowstat st;
  rowstat_init(&st, row, vocab, num_shards, ky_inv_temperature(temperature));
  for (int32_t i = 0; i < vocab; ++i) out_p[i] = rowstat_p(&st, i);
  rowstat_free(&st);
}

/* ------------------------------------------------------------------ */
/* one rank's columns under tensor parallelism                          */
/* ------------------------------------------------------------------ */
/* The pieces each rank of a vocabulary-sharded group computes on its own
 * columns (a contiguous shard, chunks starting at the shard start; the
 * shard rule of src/distributed.rs:90-98).  Combined across ranks in rank
 * order they give exactly the num_shards statistics of rowstat_init. */

/* chunk maxima and sums of one shard */
static int32_t shard_chunks(const float* shard, int32_t len, float inv_t, float** m_out,
                            float** E_out) {
  ko_rowstat st;
  rowstat_init(&st, shard, len, 1, inv_t);
  int32_t nc = st.chunks_per_shard;
  float* E = (float*)malloc(sizeof(float) * (size_t)nc);
  for (int32_t c = 0; c < nc; ++c) {
    float e[KY_CHUNK];
    for (int32_t p = 0; p < KY_CHUNK; ++p) {
      int32_t i = c * KY_CHUNK + p;
      float s = i < len ? KY_FMUL(shard[i], inv_t) : -INFINITY;
      e[p] = ky_exp(KY_FSUB(s, st.m[c]));
    }
    E[c] = ky_chunk_sum(e);
  }
  float* m = (float*)malloc(sizeof(float) * (size_t)nc);
  memcpy(m, st.m, sizeof(float) * (size_t)nc);
  rowstat_free(&st);
  *m_out = m;
  *E_out = E;
  return nc;
}

float ko_tp_row_max(const float* shard, int32_t len, float temperature) {
  float *m, *E;
  int32_t nc = shard_chunks(shard, len, ky_inv_temperature(temperature), &m, &E);
  float M = -INFINITY;
  for (int32_t c = 0; c < nc; ++c)
    if (m[c] > M) M = m[c];
  free(m);
  free(E);
  return M;
}

double ko_tp_row_sum_part(const float* shard, int32_t len, float temperature, float M) {
  float *m, *E;
  int32_t nc = shard_chunks(shard, len, ky_inv_temperature(temperature), &m, &E);
  double t[32];
  for (int32_t l = 0; l < 32; ++l) {
    t[l] = 0.0;
    for (int32_t c = l; c < nc; c += 32) t[l] = KY_DADD(t[l], ky_chunk_mass(E[c], m[c], M));
  }
  free(m);
  free(E);
  return ky_butterfly32(t);
}

void ko_tp_entry(const float* shard, int32_t len, float temperature, int32_t idx, float* e,
                 float* m_c) {
  float inv_t = ky_inv_temperature(temperature);
  float *m, *E;
  shard_chunks(shard, len, inv_t, &m, &E);
  *m_c = m[idx / KY_CHUNK];
  *e = ky_exp(KY_FSUB(KY_FMUL(shard[idx], inv_t), *m_c));
  free(m);
  free(E);
}

/* Weights of the shard under the global row statistics (Mp, Sp) of p and
 * (Mq, Sq) of q; q_shard NULL samples from p.  w[i] = residual (or p)
 * weight, wp[i] = p weight. */
static void shard_weights(const float* p_shard, const float* q_shard, int32_t len, float inv_t,
                          float Mp, double Sp, float Mq, double Sq, uint64_t* w, uint64_t* wp) {
  float *mp, *Ep, *mq = NULL, *Eq = NULL;
  shard_chunks(p_shard, len, inv_t, &mp, &Ep);
  if (q_shard) shard_chunks(q_shard, len, inv_t, &mq, &Eq);
  for (int32_t i = 0; i < len; ++i) {
    int32_t c = i / KY_CHUNK;
    float ep = ky_exp(KY_FSUB(KY_FMUL(p_shard[i], inv_t), mp[c]));
    float gp62 = ky_scale62(ky_chunk_scale(mp[c], Mp, Sp));
    wp[i] = ky_weight_p(ep, gp62);
    if (q_shard) {
      float eq = ky_exp(KY_FSUB(KY_FMUL(q_shard[i], inv_t), mq[c]));
      w[i] = ky_weight_residual(ep, gp62, eq, ky_scale62(ky_chunk_scale(mq[c], Mq, Sq)));
    } else {
      w[i] = wp[i];
    }
  }
  free(mp);
  free(Ep);
  free(mq);
  free(Eq);
}

void ko_tp_weight_totals(const float* p_shard, const float* q_shard, int32_t len,
                         float temperature, float Mp, double Sp, float Mq, double Sq,
                         uint64_t* w_res, uint64_t* w_p) {
  uint64_t* w = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)len);
  uint64_t* wp = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)len);
  shard_weights(p_shard, q_shard, len, ky_inv_temperature(temperature), Mp, Sp, Mq, Sq, w, wp);
  uint64_t a = 0, b = 0;
  for (int32_t i = 0; i < len; ++i) {
    a += w[i];
    b += wp[i];
  }
  *w_res = a;
  *w_p = b;
  free(w);
  free(wp);
}

int32_t ko_tp_cut(const float* p_shard, const float* q_shard, int32_t len, float temperature,
                  float Mp, double Sp, float Mq, double Sq, int32_t residual, uint64_t T) {
  uint64_t* w = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)len);
  uint64_t* wp = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)len);
  shard_weights(p_shard, q_shard, len, ky_inv_temperature(temperature), Mp, Sp, Mq, Sq, w, wp);
  const uint64_t* use = residual ? w : wp;
  int32_t found = -1;
  uint64_t C = 0;
  for (int32_t i = 0; i < len && found < 0; ++i) {
    C += use[i];
    if (C >= T) found = i;
  }
  free(w);
  free(wp);
  return found;
}

/* ------------------------------------------------------------------ */
/* draft sampler                                                        */
/* ------------------------------------------------------------------ */
typedef struct {
  int32_t batch, num_pos, vocab;
  float temperature;
  uint64_t seed;
  uint32_t step;
  int64_t seq_offset;
  const float* logits;
  int32_t* out_tokens;
  float* out_probs;
  int32_t b0, b1;
} sample_job;

static void sample_range(const sample_job* J) {
  uint64_t* w = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)J->vocab);
  for (int32_t b = J->b0; b < J->b1; ++b) {
    for (int32_t j = 0; j < J->num_pos; ++j) {
      const float* row = J->logits + ((size_t)b * J->num_pos + j) * (size_t)J->vocab;
      int32_t tok;
      float prob = 1.0f;
      if (!(J->temperature > 0.0f)) {
        tok = argmax_row(row, J->vocab);
      } else {
        ko_rowstat st;
        rowstat_init(&st, row, J->vocab, 1, ky_inv_temperature(J->temperature));
        for (int32_t i = 0; i < J->vocab; ++i) w[i] = rowstat_wp(&st, i);
        uint32_t odd = ky_uniform_odd(J->seed, (uint32_t)(J->seq_offset + b), (uint32_t)j,
                                      KY_STREAM_DRAFT, J->step);
        tok = inverse_cdf(w, J->vocab, odd);
        prob = rowstat_p(&st, tok);
        rowstat_free(&st);
      }
      J->out_tokens[(size_t)b * J->num_pos + j] = tok;
      if (J->out_probs) J->out_probs[(size_t)b * J->num_pos + j] = prob;
    }
  }
  free(w);
}

static void* sample_thread(void* arg) {
  sample_range((const sample_job*)arg);
  return NULL;
}

/* run fn over [0, batch) split into nthreads contiguous ranges */
typedef void* (*ko_thread_fn)(void*);
static void run_parallel(void* jobs, size_t job_size, int32_t batch, int32_t nthreads,
                         ko_thread_fn fn, void (*set_range)(void*, int32_t, int32_t)) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > batch) nthreads = batch > 0 ? batch : 1;
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
  for (int32_t t = 0; t < nthreads; ++t) {
    int32_t b0 = (int32_t)((int64_t)batch * t / nthreads);
    int32_t b1 = (int32_t)((int64_t)batch * (t + 1) / nthreads);
    set_range((char*)jobs + job_size * (size_t)t, b0, b1);
  }
  for (int32_t t = 1; t < nthreads; ++t)
    pthread_create(&th[t], NULL, fn, (char*)jobs + job_size * (size_t)t);
  fn(jobs);
  for (int32_t t = 1; t < nthreads; ++t) pthread_join(th[t], NULL);
  free(th);
}

static void sample_set_range(void* j, int32_t b0, int32_t b1) {
  ((sample_job*)j)->b0 = b0;
  ((sample_job*)j)->b1 = b1;
}

void ko_sample_tokens(int32_t batch, int32_t num_pos, int32_t vocab, float temperature,
                      uint64_t seed, uint32_t step, int64_t seq_offset, const float* logits,
                      int32_t* out_tokens, float* out_probs, int32_t nthreads) {
  int32_t nt = nthreads < 1 ? 1 : nthreads;
  sample_job* jobs = (sample_job*)calloc((size_t)nt, sizeof(sample_job));
  for (int32_t t = 0; t < nt; ++t) {
    sample_job J = {batch, num_pos, vocab, temperature, seed, step, seq_offset,
                    logits, out_tokens, out_probs, 0, 0};
    jobs[t] = J;
  }
  run_parallel(jobs, sizeof(sample_job), batch, nt, sample_thread, sample_set_range);
  free(jobs);
}

/* ------------------------------------------------------------------ */
/* chain acceptance                                                     */
/* ------------------------------------------------------------------ */
typedef struct {
  int32_t batch, k, vocab, mode;
  float temperature;
  uint64_t seed;
  uint32_t step;
  int64_t seq_offset;
  int32_t num_shards;
  const float* target;
  const float* draft;
  const int32_t* draft_tokens;
  int32_t* out_accept_len;
  int32_t* out_tokens;
  int32_t* out_num_tokens;
  float* out_probs;
  int32_t b0, b1;
} accept_job;

static void accept_one_greedy(const accept_job* J, int32_t b) {
  const int32_t k = J->k, V = J->vocab;
  const float* tgt = J->target + (size_t)b * (k + 1) * V;
  const int32_t* x = J->draft_tokens + (size_t)b * k;
  int32_t* toks = J->out_tokens + (size_t)b * (k + 1);
  for (int32_t j = 0; j <= k; ++j) toks[j] = -1;
  int32_t a = 0;
  int32_t last = -1;
  for (; a < k; ++a) {
    int32_t top = argmax_row(tgt + (size_t)a * V, V);
    if (top != x[a]) {
      last = top;
      break;
    }
    toks[a] = x[a];
  }
  int32_t num;
  if (a < k) {
    toks[a] = last;
    num = a + 1;
  } else if (J->mode == KO_MODE_GREEDY_REF && k > 0) {
    num = k; /* reference: no bonus token */
  } else {
    toks[k] = argmax_row(tgt + (size_t)k * V, V);
    num = k + 1;
  }
  J->out_accept_len[b] = a;
  J->out_num_tokens[b] = num;
}

static void accept_one_stochastic(const accept_job* J, int32_t b, uint64_t* w) {
  const int32_t k = J->k, V = J->vocab;
  const float inv_t = ky_inv_temperature(J->temperature);
  const float* tgt = J->target + (size_t)b * (k + 1) * V;
  const float* drf = J->draft + (size_t)b * k * V;
  const int32_t* x = J->draft_tokens + (size_t)b * k;
  int32_t* toks = J->out_tokens + (size_t)b * (k + 1);
  const uint32_t seq = (uint32_t)(J->seq_offset + b);
  for (int32_t j = 0; j <= k; ++j) toks[j] = -1;

  int32_t a = k;
  for (int32_t j = 0; j < k; ++j) {
    ko_rowstat P, Q;
    rowstat_init(&P, tgt + (size_t)j * V, V, J->num_shards, inv_t);
    rowstat_init(&Q, drf + (size_t)j * V, V, J->num_shards, inv_t);
    int32_t xj = x[j];
    float p = 0.0f, q = 0.0f;
    if (xj >= 0 && xj < V) {
      p = rowstat_p(&P, xj);
      q = rowstat_p(&Q, xj);
    }
    if (J->out_probs) {
      J->out_probs[((size_t)b * k + j) * 2 + 0] = p;
      J->out_probs[((size_t)b * k + j) * 2 + 1] = q;
    }
    uint32_t odd = ky_uniform_odd(J->seed, seq, (uint32_t)j, KY_STREAM_ACCEPT, J->step);
    int acc = (xj >= 0 && xj < V) && ky_accept(odd, p, q);
    if (a == k && !acc) a = j;
    rowstat_free(&P);
    rowstat_free(&Q);
  }
  for (int32_t j = 0; j < a; ++j) toks[j] = x[j];

  ko_rowstat P;
  rowstat_init(&P, tgt + (size_t)a * V, V, J->num_shards, inv_t);
  uint64_t W = 0;
  if (a < k) {
    ko_rowstat Q;
    rowstat_init(&Q, drf + (size_t)a * V, V, J->num_shards, inv_t);
    for (int32_t i = 0; i < V; ++i) {
      w[i] = ky_weight_residual(rowstat_e(&P, i), P.g62[chunk_of(&P, i)], rowstat_e(&Q, i),
                                Q.g62[chunk_of(&Q, i)]);
      W += w[i];
    }
    rowstat_free(&Q);
  }
  if (W == 0) /* bonus row, or a residual with no mass: sample from p */
    for (int32_t i = 0; i < V; ++i) w[i] = rowstat_wp(&P, i);
  rowstat_free(&P);
  uint32_t odd = ky_uniform_odd(J->seed, seq, (uint32_t)a, KY_STREAM_RESAMPLE, J->step);
  toks[a] = inverse_cdf(w, V, odd);
  J->out_accept_len[b] = a;
  J->out_num_tokens[b] = a + 1;
}

static void* accept_thread(void* arg) {
  const accept_job* J = (const accept_job*)arg;
  uint64_t* w = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)J->vocab);
  for (int32_t b = J->b0; b < J->b1; ++b) {
    if (J->mode == KO_MODE_STOCHASTIC && J->temperature > 0.0f)
      accept_one_stochastic(J, b, w);
    else
      accept_one_greedy(J, b);
  }
  free(w);
  return NULL;
}

static void accept_set_range(void* j, int32_t b0, int32_t b1) {
  ((accept_job*)j)->b0 = b0;
  ((accept_job*)j)->b1 = b1;
}

void ko_spec_accept(int32_t batch, int32_t k, int32_t vocab, int32_t mode, float temperature,
                    uint64_t seed, uint32_t step, int64_t seq_offset, int32_t num_shards,
                    const float* target_logits, const float* draft_logits,
                    const int32_t* draft_tokens, int32_t* out_accept_len, int32_t* out_tokens,
                    int32_t* out_num_tokens, float* out_probs, int32_t nthreads) {
  int32_t nt = nthreads < 1 ? 1 : nthreads;
  accept_job* jobs = (accept_job*)calloc((size_t)nt, sizeof(accept_job));
  int32_t eff_mode = mode;
  if (mode == KO_MODE_STOCHASTIC && !(temperature > 0.0f)) eff_mode = KO_MODE_GREEDY;
  for (int32_t t = 0; t < nt; ++t) {
    accept_job J = {batch,        k,
                    vocab,        eff_mode,
                    temperature,  seed,
                    step,         seq_offset,
                    num_shards < 1 ? 1 : num_shards,
                    target_logits, draft_logits,
                    draft_tokens, out_accept_len,
                    out_tokens,   out_num_tokens,
                    out_probs,    0,
                    0};
    jobs[t] = J;
  }
  run_parallel(jobs, sizeof(accept_job), batch, nt, accept_thread, accept_set_range);
  free(jobs);
}

/* ------------------------------------------------------------------ */
/* tree acceptance                                                      */
/* ------------------------------------------------------------------ */
/* Multi-candidate rejection sampling over a BFS-ordered draft tree
 * (SpecInfer, Miao et al. 2023), as kyro_math.h states it.  The reference
 * has no tree code; the greedy variant accepts the first child whose token
 * is the target's argmax (speculative.rs:314-323 applied per node). */

/* p_j(i): p_i after j residual steps */
static double tree_pj(const ko_rowstat* P, const ko_rowstat* Q, const double* R, int32_t nr,
                      int32_t i) {
  double v = (double)rowstat_p(P, i);
  const double q = (double)rowstat_p(Q, i);
  for (int32_t j = 0; j < nr; ++j) v = ky_tree_step(v, q, R[j]);
  return v;
}

/* R_nr = sum_i max(p_nr(i) - q_i, 0) in the contract's tree */
static double tree_residual_sum(const ko_rowstat* P, const ko_rowstat* Q, const double* R,
                                int32_t nr, int32_t V) {
  int32_t nc = (V + KY_CHUNK - 1) / KY_CHUNK;
  double t[32];
  for (int32_t l = 0; l < 32; ++l) t[l] = 0.0;
  for (int32_t c = 0; c < nc; ++c) {
    double e[KY_CHUNK];
    for (int32_t p = 0; p < KY_CHUNK; ++p) {
      int32_t i = c * KY_CHUNK + p;
      e[p] = i < V ? ky_tree_excess(tree_pj(P, Q, R, nr, i), (double)rowstat_p(Q, i)) : 0.0;
    }
    t[c % 32] = KY_DADD(t[c % 32], ky_chunk_sum_d(e));
  }
  return ky_butterfly32(t);
}

typedef struct {
  int32_t batch, num_nodes, vocab, greedy;
  float temperature;
  uint64_t seed;
  uint32_t step;
  int64_t seq_offset;
  const float* target;
  const float* draft;
  const int32_t* node_tokens;
  const int32_t* parents;
  int32_t* out_path;
  int32_t* out_path_len;
  int32_t* out_tokens;
  int32_t* out_num_tokens;
  int32_t b0, b1;
} tree_job;

static void tree_one(const tree_job* J, int32_t b, uint64_t* w) {
  const int32_t N = J->num_nodes, V = J->vocab;
  const float inv_t = ky_inv_temperature(J->temperature);
  const float* tgt = J->target + (size_t)b * N * V;
  const float* drf = J->draft + (size_t)b * N * V;
  const int32_t* tok = J->node_tokens + (size_t)b * N;
  const int32_t* par = J->parents + (size_t)b * N;
  int32_t* path = J->out_path + (size_t)b * N;
  int32_t* toks = J->out_tokens + (size_t)b * N;
  const uint32_t seq = (uint32_t)(J->seq_offset + b);
  for (int32_t n = 0; n < N; ++n) path[n] = toks[n] = -1;
  int32_t node = 0, plen = 1, ntok = 0;
  path[0] = 0;
  for (;;) {
    int32_t ch[64], nch = 0;
    for (int32_t c = node + 1; c < N; ++c)
      if (par[c] == node) ch[nch++] = c;
    int32_t accepted = -1;
    if (J->greedy) {
      const int32_t top = argmax_row(tgt + (size_t)node * V, V);
      for (int32_t i = 0; i < nch && accepted < 0; ++i)
        if (tok[ch[i]] == top) accepted = ch[i];
      if (accepted < 0) {
        toks[ntok++] = top;
        break;
      }
    } else {
      ko_rowstat P, Q;
      rowstat_init(&P, tgt + (size_t)node * V, V, 1, inv_t);
      rowstat_init(&Q, drf + (size_t)node * V, V, 1, inv_t);
      double R[64];
      int32_t nr = 0;
      for (int32_t i = 0; i < nch; ++i) {
        const int32_t c = ch[i], x = tok[c];
        if (x >= 0 && x < V) {
          const double px = tree_pj(&P, &Q, R, nr, x);
          const double qx = (double)rowstat_p(&Q, x);
          const double u =
              (double)ky_odd_to_float(ky_uniform_odd(J->seed, seq, (uint32_t)c, KY_STREAM_ACCEPT,
                                                     J->step));
          if (u < KY_DDIV(px, qx)) {
            accepted = c;
            break;
          }
        }
        R[nr] = tree_residual_sum(&P, &Q, R, nr, V);
        ++nr;
      }
      if (accepted < 0) {
        for (int32_t i = 0; i < V; ++i) w[i] = ky_weight_d(tree_pj(&P, &Q, R, nr, i));
        const uint32_t odd =
            ky_uniform_odd(J->seed, seq, (uint32_t)node, KY_STREAM_RESAMPLE, J->step);
        toks[ntok++] = inverse_cdf(w, V, odd);
      }
      rowstat_free(&P);
      rowstat_free(&Q);
      if (accepted < 0) break;
    }
    path[plen++] = accepted;
    toks[ntok++] = tok[accepted];
    node = accepted;
  }
  J->out_path_len[b] = plen;
  J->out_num_tokens[b] = ntok;
}

static void* tree_thread(void* arg) {
  const tree_job* J = (const tree_job*)arg;
  uint64_t* w = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)J->vocab);
  for (int32_t b = J->b0; b < J->b1; ++b) tree_one(J, b, w);
  free(w);
  return NULL;
}

static void tree_set_range(void* j, int32_t b0, int32_t b1) {
  ((tree_job*)j)->b0 = b0;
  ((tree_job*)j)->b1 = b1;
}

void ko_spec_accept_tree(int32_t batch, int32_t num_nodes, int32_t vocab, int32_t mode,
                         float temperature, uint64_t seed, uint32_t step, int64_t seq_offset,
                         const float* target_logits, const float* draft_logits,
                         const int32_t* node_tokens, const int32_t* parents, int32_t* out_path,
                         int32_t* out_path_len, int32_t* out_tokens, int32_t* out_num_tokens,
                         int32_t nthreads) {
  int32_t nt = nthreads < 1 ? 1 : nthreads;
  tree_job* jobs = (tree_job*)calloc((size_t)nt, sizeof(tree_job));
  const int32_t greedy = !(mode == KO_MODE_STOCHASTIC && temperature > 0.0f);
  for (int32_t t = 0; t < nt; ++t) {
    tree_job J = {batch,        num_nodes,     vocab,       greedy,        temperature,
                  seed,         step,          seq_offset,  target_logits, draft_logits,
                  node_tokens,  parents,       out_path,    out_path_len,  out_tokens,
                  out_num_tokens, 0,           0};
    jobs[t] = J;
  }
  run_parallel(jobs, sizeof(tree_job), batch, nt, tree_thread, tree_set_range);
  free(jobs);
}
