/*
 * kyro_oracle.h -- CPU restatement of the speculative verify step.
 *
 * TEST INFRASTRUCTURE ONLY.  The oracle is the checker for the sm_100a
 * kernels; it is never the measured or shipped path.  Only tests/,
 * __graft_entry__.smoke() and bench.py (its cpu_baseline leg and
 * `--impl reference`) may load it.
 *
 * What it restates (reference paths are within khulnasoft-research/kyro):
 *   - greedy verification, exactly: src/speculative.rs:286-339
 *     (argmax compare :314-323, k == 0 case :296-305);
 *   - sampling conventions of sample_token, src/worker.rs:267-362
 *     (argmax at T <= 0 :290-296, logits * (1/T) :298, max-subtracted
 *     softmax :314-323, inverse-CDF "r -= p; if r <= 0" :352-360);
 *   - stochastic rejection sampling, which the reference does not have:
 *     Leviathan, Kalman & Matias 2023 (Alg. 1) / Chen et al. 2023;
 *   - paged attention mathematics of src/model/attention_kernel.rs:22-136
 *     (layouts :52-57, GQA map h / (Hq/Hkv) :39-46, scale 1/sqrt(D) :69,
 *     block walk with a partial last block :86-93), without the score
 *     layout bug of :104-111;
 *   - BlockManager free-list / ref-count bookkeeping,
 *     src/scheduler/block_manager.rs:33-153.
 *
 * Parity pin: the reference is Rust with un-vendored candle 0.10.2 and no
 * cargo here, so it cannot be run.  The oracle is pinned against the
 * reference's own known-answer tests, read as text (tests/golden/): the
 * sample_token argmax cases (src/worker.rs:395-422), the peaked-row cases
 * (:425-440), the BlockManager counts (src/scheduler/block_manager.rs:
 * 164-235) and the attention shape cases (src/model/attention_kernel.rs:
 * 163-227, with the value check that all-ones K/V gives all-ones output).
 * The stochastic rule has no counterpart in the reference: for it parity is
 * unpinned by the reference and is checked against the published method's
 * distributional property (the emitted token is distributed as p).
 */
#ifndef KYRO_ORACLE_H
#define KYRO_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Philox uniforms, for cross-checking the device generator. */
void ko_philox4x32_10(const uint32_t ctr[4], uint64_t key, uint32_t out[4]);
float ko_uniform(uint64_t seed, uint32_t seq, uint32_t pos, uint32_t stream, uint32_t step);
float ko_exp(float x);

/* Softmax probabilities of one row under the normaliser contract of
 * kyro_math.h (num_shards equal contiguous shards of the row). */
void ko_softmax_row(const float* row, int32_t vocab, int32_t num_shards, float temperature,
                    float* out_p);

/* Draft sampler: logits [B, P, V] -> tokens [B, P] (+ q(token)). */
void ko_sample_tokens(int32_t batch, int32_t num_pos, int32_t vocab, float temperature,
                      uint64_t seed, uint32_t step, int64_t seq_offset, const float* logits,
                      int32_t* out_tokens, float* out_probs, int32_t nthreads);

/* Chain acceptance: same arguments and outputs as kyro_spec_accept, plus
 * the number of vocabulary shards the normaliser is defined over. */
void ko_spec_accept(int32_t batch, int32_t k, int32_t vocab, int32_t mode, float temperature,
                    uint64_t seed, uint32_t step, int64_t seq_offset, int32_t num_shards,
                    const float* target_logits, const float* draft_logits,
                    const int32_t* draft_tokens, int32_t* out_accept_len, int32_t* out_tokens,
                    int32_t* out_num_tokens, float* out_probs, int32_t nthreads);

/* Tree acceptance: node n of sequence b has token node_tokens[b][n], parent
 * parents[b][n] (-1 for the root, node 0; parents precede children), and
 * target / draft next-token logits rows [b][n][V].  Outputs: the accepted
 * path (node ids, root first, -1 padded) [B, N], its length [B], the
 * emitted tokens [B, N] (-1 padded) and their count [B]. */
void ko_spec_accept_tree(int32_t batch, int32_t num_nodes, int32_t vocab, int32_t mode,
                         float temperature, uint64_t seed, uint32_t step, int64_t seq_offset,
                         const float* target_logits, const float* draft_logits,
                         const int32_t* node_tokens, const int32_t* parents, int32_t* out_path,
                         int32_t* out_path_len, int32_t* out_tokens, int32_t* out_num_tokens,
                         int32_t nthreads);

/* One rank's pieces of a vocabulary-sharded row (its contiguous columns,
 * len entries): the shard's row max M_r; its butterfly part of the
 * normaliser under a given max M (the protocol passes M_r, and every rank
 * brings the parts to the row max with ky_shard_scale); e and the chunk max
 * at one of its entries; its
 * residual (q_shard != NULL) and p weight totals under the global row
 * statistics; and the entry where its weights first reach T. */
float ko_tp_row_max(const float* shard, int32_t len, float temperature);
double ko_tp_row_sum_part(const float* shard, int32_t len, float temperature, float M);
void ko_tp_entry(const float* shard, int32_t len, float temperature, int32_t idx, float* e,
                 float* m_c);
void ko_tp_weight_totals(const float* p_shard, const float* q_shard, int32_t len,
                         float temperature, float Mp, double Sp, float Mq, double Sq,
                         uint64_t* w_res, uint64_t* w_p);
int32_t ko_tp_cut(const float* p_shard, const float* q_shard, int32_t len, float temperature,
                  float Mp, double Sp, float Mq, double Sq, int32_t residual, uint64_t T);

/* Paged multi-query attention in double precision.
 * q bf16 bits [B, nq, Hq, D]; caches bf16 bits [NB, Hkv, bs, D];
 * out fp32 [B, nq, Hq, D]; tree_mask may be NULL (chain). */
void ko_paged_attention(int32_t batch, int32_t nq, int32_t hq, int32_t hkv, int32_t d,
                        int32_t bs, int32_t max_blocks, float scale, const uint16_t* q,
                        const uint16_t* k_cache, const uint16_t* v_cache,
                        const int64_t* block_table, const int64_t* context_lens,
                        const uint64_t* tree_mask, float* out, int32_t nthreads);

/* BlockManager mirror: same semantics as kyro_kv_reserve / _commit. */
void ko_kv_reserve(int32_t batch, int32_t bs, int32_t max_blocks, int32_t num_blocks,
                   int32_t num_new, int64_t* block_table, const int64_t* context_lens,
                   int32_t* free_stack, int32_t* free_top, int32_t* ref_counts,
                   int32_t* out_ok);
/* kv_reserve with copy-on-write of a shared, partly filled last block */
void ko_kv_reserve_cow(int32_t batch, int32_t bs, int32_t max_blocks, int32_t num_blocks,
                       int32_t num_new, int32_t num_layers, uint16_t* const* k_caches,
                       uint16_t* const* v_caches, int32_t hkv, int32_t d, int64_t* block_table,
                       const int64_t* context_lens, int32_t* free_stack, int32_t* free_top,
                       int32_t* ref_counts, int32_t* out_ok, int32_t* cow);
void ko_kv_commit(int32_t batch, int32_t bs, int32_t max_blocks, int32_t num_blocks,
                  int32_t num_new, const int32_t* accept_len, int64_t* block_table,
                  int64_t* context_lens, int32_t* free_stack, int32_t* free_top,
                  int32_t* ref_counts);
void ko_kv_write(int32_t batch, int32_t bs, int32_t max_blocks, int32_t num_blocks,
                 int32_t num_new, int32_t hkv, int32_t d, const uint16_t* k_new,
                 const uint16_t* v_new, const int64_t* block_table, const int64_t* context_lens,
                 uint16_t* k_cache, uint16_t* v_cache);
/* rotary position embedding (layers.rs:37-61) + paged K/V store */
void ko_rope_kv_write(int32_t batch, int32_t bs, int32_t max_blocks, int32_t num_blocks,
                      int32_t num_new, int32_t hq, int32_t hkv, int32_t d, float theta,
                      const int32_t* pos_offsets, const uint16_t* q, const uint16_t* k_new,
                      const uint16_t* v_new, const int64_t* block_table,
                      const int64_t* context_lens, uint16_t* q_out, uint16_t* k_cache,
                      uint16_t* v_cache);
void ko_kv_commit_tree(int32_t batch, int32_t bs, int32_t max_blocks, int32_t num_blocks,
                       int32_t num_nodes, const int32_t* path, const int32_t* path_len,
                       int32_t num_layers, uint16_t* const* k_caches, uint16_t* const* v_caches,
                       int32_t hkv, int32_t d, int64_t* block_table, int64_t* context_lens,
                       int32_t* free_stack, int32_t* free_top, int32_t* ref_counts);

#ifdef __cplusplus
}
#endif

#endif
