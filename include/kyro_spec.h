/*
 * kyro_spec.h -- C ABI of the B200 (sm_100a) speculative-decoding verify step.
 *
 * Three kernels families sit behind this header:
 *   K1  paged multi-query verify attention (chain of k+1 positions, or the
 *       nodes of a draft tree under an ancestor mask);
 *   K2  vocab-wide rejection sampling (accept test, residual resample, bonus
 *       token), plus the draft-token sampler that feeds it;
 *   K3  KV-slot reserve / commit / rollback on the BlockManager block table.
 *
 * Conventions
 *   - Every function returns an int status (KYRO_OK == 0).  Arguments are
 *     validated on the host before anything is launched; kyro_last_error()
 *     returns a message for the calling thread.
 *   - The caller owns every device buffer (inputs, outputs, KV cache, block
 *     tables, workspace).  Nothing on these entry points allocates device
 *     memory; *_workspace_size() says how much scratch to pass.
 *   - Calls enqueue on the context's stream and return without a host sync.
 *   - One kyro_ctx per GPU; a context is not re-entrant, distinct contexts
 *     are independent.
 *   - Device-side range checks (block ids, token ids) set bits in a status
 *     word instead of trapping; kyro_ctx_device_status() reads it.
 *
 * The reference (an all-Rust server) has no native code for this path; each
 * declaration cites the Rust item whose role it takes.
 */
#ifndef KYRO_SPEC_H
#define KYRO_SPEC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KYRO_VERSION 1

/* Status codes.  The Rust wrapper maps each to candle_core::Error::Msg
 * (src/speculative.rs:224 builds errors the same way). */
#define KYRO_OK 0
#define KYRO_ERR_INVALID_ARG 1
#define KYRO_ERR_CUDA 2
#define KYRO_ERR_NCCL 3
#define KYRO_ERR_TIMEOUT 4
#define KYRO_ERR_OOB 5
#define KYRO_ERR_OOM 6
#define KYRO_ERR_UNSUPPORTED 7
#define KYRO_ERR_WORKSPACE 8

/* Bits of the device status word. */
#define KYRO_DEV_BAD_TOKEN 0x1u      /* a draft token outside [0, vocab)        */
#define KYRO_DEV_BAD_BLOCK 0x2u      /* a block id outside [0, num_blocks)      */
#define KYRO_DEV_BAD_LENGTH 0x4u     /* context length beyond the block table   */
#define KYRO_DEV_WAIT_TIMEOUT 0x8u   /* a bounded device-side wait gave up      */
#define KYRO_DEV_STACK_OVERFLOW 0x10u /* free-stack push beyond num_blocks      */

typedef struct kyro_ctx kyro_ctx;

/* ---------------------------------------------------------------- context */

/* Create a context bound to `device` and enqueueing on `stream`
 * (a cudaStream_t; NULL = legacy default stream).  Allocates only the
 * 16-byte device status word. */
int kyro_ctx_create(int device, void* stream, kyro_ctx** out);
int kyro_ctx_destroy(kyro_ctx* ctx);
int kyro_ctx_set_stream(kyro_ctx* ctx, void* stream);
/* Synchronise the context's stream, return the device status word in
 * *out_flags (KYRO_DEV_* bits) and clear it when `clear` != 0. */
int kyro_ctx_device_status(kyro_ctx* ctx, uint32_t* out_flags, int clear);
/* Bound, in milliseconds (1..600000), of every wait this context makes on
 * another rank: a device-side wait for a peer's flag in the exchange rounds
 * sets KYRO_DEV_WAIT_TIMEOUT and returns when it runs out, and the host
 * watchdog aborts an NCCL collective that has not completed within it (the
 * group's TP calls then return KYRO_ERR_TIMEOUT).  The role of the
 * reference's request deadlines (src/scheduler/continuous_batching.rs:
 * 83-100), for the step's collectives.  A new context takes
 * KYRO_WAIT_TIMEOUT_MS from the environment, else 2000.  After a timeout
 * the ranks' exchange state no longer agrees: destroy the context and form
 * the group again. */
int kyro_ctx_set_wait_timeout(kyro_ctx* ctx, uint32_t ms);
/* Copy the calling thread's last error message into buf (NUL-terminated);
 * returns the full message length. */
size_t kyro_last_error(char* buf, size_t len);
const char* kyro_status_string(int status);
int kyro_version(void);
/* Names of the kernels this library launches, ';'-separated. */
const char* kyro_kernel_names(void);

/* ------------------------------------------------ K2: acceptance sampling */

/* Accept modes.
 *  STOCHASTIC  rejection sampling (Leviathan et al. 2023 / Chen et al. 2023):
 *              accept draft x_j iff u_j < p_j(x_j)/q_j(x_j); at the first
 *              rejection resample from norm(max(p_j - q_j, 0)); if all k are
 *              accepted, sample a bonus token from p_k.  temperature <= 0
 *              falls back to GREEDY, as sample_token does
 *              (src/worker.rs:290-296).
 *  GREEDY      accept x_j iff x_j == argmax p_j; emit argmax at the first
 *              mismatch, or the bonus argmax p_k when all match.
 *  GREEDY_REF  exactly the reference rule of verify_drafts
 *              (src/speculative.rs:314-323): like GREEDY but no bonus token
 *              when every draft matches, and k == 0 emits argmax of row 0
 *              (src/speculative.rs:296-305).
 * argmax ties resolve to the lowest index. */
#define KYRO_ACCEPT_STOCHASTIC 0
#define KYRO_ACCEPT_GREEDY 1
#define KYRO_ACCEPT_GREEDY_REF 2

typedef struct kyro_accept_params {
  int32_t batch;       /* B sequences in this call                          */
  int32_t num_draft;   /* k draft tokens per sequence (0..64)               */
  int32_t vocab;       /* V entries per logits row held by this process     */
  int32_t mode;        /* KYRO_ACCEPT_*                                     */
  float temperature;   /* softmax temperature for p and q (stochastic mode) */
  uint32_t step;       /* Philox counter word 3 (the caller's step number)  */
  uint64_t seed;       /* Philox key                                        */
  int64_t seq_offset;  /* global index of sequence 0 (Philox counter word 0)*/
} kyro_accept_params;

size_t kyro_spec_accept_workspace_size(const kyro_accept_params* p);

/* Replaces SpeculativeDecoder::verify_drafts (src/speculative.rs:286-339),
 * batched over B sequences, with the sampling conventions of sample_token
 * (src/worker.rs:298 temperature, :314-323 max-subtracted softmax,
 * :352-360 inverse CDF).
 *   target_logits  fp32 [B, k+1, V]   row j scores position j; row k is the
 *                                     bonus row (unused by GREEDY_REF)
 *   draft_logits   fp32 [B, k, V]     draft model logits (STOCHASTIC only;
 *                                     may be NULL otherwise)
 *   draft_tokens   int32 [B, k]
 *   out_accept_len int32 [B]          accepted drafts a in [0, k]
 *   out_tokens     int32 [B, k+1]     x_0..x_{a-1}, then the resampled /
 *                                     bonus / argmax token; -1 padded
 *   out_num_tokens int32 [B]          tokens emitted (a+1, or k for
 *                                     GREEDY_REF when all match)
 *   out_probs      fp32 [B, k, 2]     optional (NULL): (p_j(x_j), q_j(x_j)) */
int kyro_spec_accept(kyro_ctx* ctx, const kyro_accept_params* p, const float* target_logits,
                     const float* draft_logits, const int32_t* draft_tokens,
                     int32_t* out_accept_len, int32_t* out_tokens, int32_t* out_num_tokens,
                     float* out_probs, void* workspace, size_t workspace_bytes);

/* kyro_spec_accept_static: kyro_spec_accept for callers that cannot
 * allocate device memory.  No counterpart in the reference.  Some hosts
 * hand this library only their own tensors and own every other byte of
 * device memory themselves (a serving runtime with a fixed arena, or a
 * real-time loop that must not call the allocator), so they have no
 * workspace to pass.  This entry point takes the same inputs and outputs
 * and uses instead a scratch buffer that the library keeps in a file-scope
 * __device__ array of KYRO_ACCEPT_STATIC_SCRATCH_BYTES (8 MiB) on every GPU
 * that loads it, held until the process exits.  It allocates nothing.
 *   - Calls whose kyro_spec_accept_workspace_size() exceeds that size are
 *     rejected with KYRO_ERR_WORKSPACE before anything is launched.
 *   - The first call on a device looks up the buffer's device address (a
 *     host-side runtime query, no allocation); make that first call before
 *     capturing a stream into a CUDA graph.  The address is kept until the
 *     next kyro_ctx_create on that device: a device reset moves the array
 *     and ends every context, so the first call through a new context looks
 *     it up again.
 *   - Every call on a device shares the one buffer and its counters are
 *     cleared at the start of each call: calls that overlap on the GPU
 *     (different streams, or different contexts on one device) race. */
#define KYRO_ACCEPT_STATIC_SCRATCH_BYTES (8u << 20)
int kyro_spec_accept_static(kyro_ctx* ctx, const kyro_accept_params* p,
                            const float* target_logits, const float* draft_logits,
                            const int32_t* draft_tokens, int32_t* out_accept_len,
                            int32_t* out_tokens, int32_t* out_num_tokens, float* out_probs);

/* Draft sampler: one token per row from softmax(logits / T) with Philox
 * stream 0 (counter (seq_offset + b, pos, 0, step)); temperature <= 0 is
 * argmax.  Replaces the draft loop's argmax (src/speculative.rs:229-241)
 * with on-device sampling.
 *   logits fp32 [B, num_pos, V] -> out_tokens int32 [B, num_pos]
 *   out_probs fp32 [B, num_pos] optional: q(token).
 * seq_stride: logits rows from sequence b's first row to sequence b+1's;
 * 0 means num_pos (dense rows).  A draft loop that writes position i's
 * logits straight into column i of a [B, k, V] buffer samples it with
 * num_pos 1 and seq_stride k. */
typedef struct kyro_sample_params {
  int32_t batch;
  int32_t num_pos;
  int32_t vocab;
  float temperature;
  uint32_t step;
  uint32_t seq_stride;
  uint64_t seed;
  int64_t seq_offset;
} kyro_sample_params;

size_t kyro_sample_workspace_size(const kyro_sample_params* p);
int kyro_sample_tokens(kyro_ctx* ctx, const kyro_sample_params* p, const float* logits,
                       int32_t* out_tokens, float* out_probs, void* workspace,
                       size_t workspace_bytes);

/* ------------------------------------------- K1: paged verify attention */

typedef struct kyro_attn_params {
  int32_t batch;              /* B                                              */
  int32_t num_query;          /* query positions per sequence: k+1 (chain) or
                                 tree nodes (<= 64)                             */
  int32_t num_heads;          /* Hq                                             */
  int32_t num_kv_heads;       /* Hkv; Hq % Hkv == 0                             */
  int32_t head_dim;           /* D (128 supported)                              */
  int32_t block_size;         /* tokens per KV block (16 supported)             */
  int32_t max_blocks_per_seq; /* width of block_table                           */
  int32_t num_blocks;         /* KV cache capacity in blocks                    */
  float scale;                /* softmax scale; 0 selects 1/sqrt(D)             */
  int32_t kv_split_blocks;    /* KV blocks per work item; 0 = automatic         */
} kyro_attn_params;

size_t kyro_verify_attention_workspace_size(const kyro_attn_params* p);

/* Replaces PagedAttention::forward (src/model/attention_kernel.rs:22-31) for
 * num_query query positions per sequence, with the reference layouts
 * (:52-57):
 *   q            bf16 [B, num_query, Hq, D]
 *   k_cache      bf16 [num_blocks, Hkv, block_size, D]
 *   v_cache      bf16 [num_blocks, Hkv, block_size, D]
 *   block_table  int64 [B, max_blocks_per_seq]
 *   context_lens int64 [B]   tokens cached before the new ones
 *   tree_mask    uint64 [B, num_query] or NULL.  Query j sits at position
 *                context_len + j; its K/V must already be in the cache.
 *                Query j attends every cached position and new position i
 *                iff bit i of tree_mask[b][j] is set.  NULL means the chain
 *                mask (i <= j).
 *   out          bf16 [B, num_query, Hq, D]
 * Query head h reads KV head h / (Hq/Hkv) (attention_kernel.rs:39-46);
 * fp32 accumulation; scale 1/sqrt(D) (attention_kernel.rs:69). */
int kyro_verify_attention(kyro_ctx* ctx, const kyro_attn_params* p, const void* q,
                          const void* k_cache, const void* v_cache, const int64_t* block_table,
                          const int64_t* context_lens, const uint64_t* tree_mask, void* out,
                          void* workspace, size_t workspace_bytes);

/* LlamaAttention::forward's rotary embedding, new-token KV append and
 * attention (src/model/llama.rs:73-90) in one launch: q, k_new and v_new
 * (bf16 [B, num_query, Hq or Hkv, D]) arrive unrotated; query and key j are
 * rotated at position context_len + pos_offsets[j] (pos_offsets NULL: + j),
 * the keys and values are stored at slot context_len + j of the paged cache
 * (the slots must be reserved), and the attention runs as in
 * kyro_verify_attention.  The cache ends, and out is, bit for bit what
 * kyro_rope_kv_write followed by kyro_verify_attention give; the rotated
 * queries are not written out.  Same workspace as kyro_verify_attention.
 * Shapes that take the tensor-core tree kernel (kyro_verify_attention on
 * draft trees of >= 128 query rows per KV head) are rejected with
 * KYRO_ERR_INVALID_ARG. */
int kyro_verify_attention_rope(kyro_ctx* ctx, const kyro_attn_params* p, float rope_theta,
                               const int32_t* pos_offsets, const void* q, const void* k_new,
                               const void* v_new, void* k_cache, void* v_cache,
                               const int64_t* block_table, const int64_t* context_lens,
                               const uint64_t* tree_mask, void* out, void* workspace,
                               size_t workspace_bytes);

/* ------------------------------------------------ K3: KV commit / rollback */

typedef struct kyro_kv_params {
  int32_t batch;              /* B sequences                         */
  int32_t block_size;         /* tokens per block                    */
  int32_t max_blocks_per_seq; /* width of block_table                */
  int32_t num_blocks;         /* pool size                           */
} kyro_kv_params;

/* Device mirror of BlockManager (src/scheduler/block_manager.rs:15-30):
 *   block_table  int64 [B, max_blocks_per_seq]  seq b holds
 *                ceil(context_lens[b]/block_size) blocks in entries 0..;
 *                unused entries are -1
 *   context_lens int64 [B]
 *   free_stack   int32 [num_blocks]   free_gpu_blocks; entries
 *                [0, *free_top) are free, the top is popped first
 *                (Vec::pop, block_manager.rs:92-98)
 *   free_top     int32 [1]
 *   ref_counts   int32 [num_blocks]   (block_manager.rs:29)
 *
 * kyro_kv_reserve: make room for num_new more token slots in every
 * sequence, popping new blocks in sequence order with ref_count = 1
 * (allocate, block_manager.rs:109-125).  A sequence whose blocks do not fit
 * in what is left of the free list gets nothing and out_ok[b] = 0 (out_ok
 * may be NULL), like allocate() returning None (:111-113); later sequences
 * are still served in order.  context_lens is not changed. */
int kyro_kv_reserve(kyro_ctx* ctx, const kyro_kv_params* p, int32_t num_new,
                    int64_t* block_table, const int64_t* context_lens, int32_t* free_stack,
                    int32_t* free_top, int32_t* ref_counts, int32_t* out_ok);

/* kyro_kv_reserve_cow: kyro_kv_reserve for block tables that share prefix
 * blocks.  allocate_with_prefix (block_manager.rs:53-105) hands a request the
 * radix cache's blocks with ref_count += 1 (:60-63), so a sequence's last,
 * partly filled block can be shared; growing into it would overwrite the
 * other holders' tokens.  Here, in sequence order, such a sequence first
 * pops a fresh block (ref_count 1) for it, the shared block's ref_count drops
 * by one, its table entry is replaced, and every slot of the block is copied
 * in each of the num_layers K and V caches (copy-on-write); then its new
 * blocks are popped as kyro_kv_reserve does.  A sequence that cannot get all
 * of its blocks gets none (out_ok[b] = 0).  out_cow int32 [B, 2] receives the
 * (shared, fresh) pair of each sequence, or (-1, -1).  k_caches / v_caches
 * are host arrays of device pointers as in kyro_kv_commit_tree. */
int kyro_kv_reserve_cow(kyro_ctx* ctx, const kyro_kv_params* p, int32_t num_new,
                        int32_t num_layers, void* const* k_caches, void* const* v_caches,
                        int32_t num_kv_heads, int32_t head_dim, int64_t* block_table,
                        const int64_t* context_lens, int32_t* free_stack, int32_t* free_top,
                        int32_t* ref_counts, int32_t* out_ok, int32_t* out_cow);

/* kyro_kv_commit: after verification keep accept_len[b] + 1 of the num_new
 * reserved slots (the last accepted token plus the accepted drafts),
 * advance context_lens, and release the blocks that now lie wholly beyond
 * the new length: ref_count -= 1 and, at zero, push onto the free stack in
 * sequence order and ascending table position (free, block_manager.rs:
 * 129-153).  accept_len[b] < 0 leaves sequence b untouched. */
int kyro_kv_commit(kyro_ctx* ctx, const kyro_kv_params* p, int32_t num_new,
                   const int32_t* accept_len, int64_t* block_table, int64_t* context_lens,
                   int32_t* free_stack, int32_t* free_top, int32_t* ref_counts);

/* kyro_spec_accept_commit: kyro_spec_accept, then kyro_kv_commit of the
 * accepted slots and, when num_new_next > 0, kyro_kv_reserve of the next
 * step's num_new_next slots, in one call.  The end of
 * SpeculativeDecoder::step (src/speculative.rs:342-353) in a decode loop,
 * where every step reserves right after it commits.  The commit needs only
 * the accept lengths, so it runs beside the acceptance's final pass
 * instead of after it, and the commit and the reserve are one launch.
 * Results equal kyro_spec_accept followed by kyro_kv_commit (num_new) and
 * kyro_kv_reserve (num_new_next); kv->batch must equal p->batch, and
 * out_ok (may be NULL) gets the reserve's per-sequence result. */
int kyro_spec_accept_commit(kyro_ctx* ctx, const kyro_accept_params* p,
                            const float* target_logits, const float* draft_logits,
                            const int32_t* draft_tokens, int32_t* out_accept_len,
                            int32_t* out_tokens, int32_t* out_num_tokens, float* out_probs,
                            void* workspace, size_t workspace_bytes, const kyro_kv_params* kv,
                            int32_t num_new, int32_t num_new_next, int64_t* block_table,
                            int64_t* context_lens, int32_t* free_stack, int32_t* free_top,
                            int32_t* ref_counts, int32_t* out_ok);

/* kyro_kv_commit_tree: tree verification wrote node n's K/V at position
 * context_len + n.  For the accepted root-to-leaf path path[b][0..len-1]
 * (path[b][0] == 0), move node path[b][i]'s K/V rows to position
 * context_len + i in every one of the num_layers caches, then commit
 * path_len[b] slots as kyro_kv_commit does.  k_caches / v_caches are host
 * arrays of num_layers device pointers, each bf16
 * [num_blocks, num_kv_heads, block_size, head_dim]. */
int kyro_kv_commit_tree(kyro_ctx* ctx, const kyro_kv_params* p, int32_t num_nodes,
                        const int32_t* path, const int32_t* path_len, int32_t num_layers,
                        void* const* k_caches, void* const* v_caches, int32_t num_kv_heads,
                        int32_t head_dim, int64_t* block_table, int64_t* context_lens,
                        int32_t* free_stack, int32_t* free_top, int32_t* ref_counts);

/* kyro_kv_write: store the K/V rows of the num_new new tokens of every
 * sequence at positions context_lens[b] .. context_lens[b]+num_new-1 of its
 * block table (slots made by kyro_kv_reserve).  Replaces
 * KVCacheManager::append_kv (src/model/kv_cache.rs:49-75), which
 * concatenates dense per-request tensors, with a paged scatter.
 *   k_new, v_new bf16 [B, num_new, num_kv_heads, head_dim]
 *                (the [batch, seq, Hkv, D] layout append_kv takes, :47-48)
 *   k_cache, v_cache bf16 [num_blocks, num_kv_heads, block_size, head_dim] */
int kyro_kv_write(kyro_ctx* ctx, const kyro_kv_params* p, int32_t num_new, int32_t num_kv_heads,
                  int32_t head_dim, const void* k_new, const void* v_new,
                  const int64_t* block_table, const int64_t* context_lens, void* k_cache,
                  void* v_cache);

/* kyro_rope_kv_write: the steps between the q/k/v projections and attention
 * in LlamaAttention::forward (src/model/llama.rs:73-82) for the num_new new
 * tokens of every sequence: rotary position embedding of the query and key
 * heads (RotaryEmbedding::apply, src/model/layers.rs:37-61, with
 * inv_freq[i] = 1 / rope_theta^(2i/head_dim) as in :26-33; llama.rs:45 uses
 * theta 10000), then the rotated keys and the values stored in the paged
 * slots context_lens[b] + j as kyro_kv_write does (append_kv), and the
 * rotated queries written to q_out (which may be q itself).  Token j of
 * sequence b is rotated at position context_lens[b] + pos_offsets[j]
 * (the reference's index + i, layers.rs:45); pos_offsets NULL means j, and a
 * draft tree passes each node's depth.
 *   q       bf16 [B, num_new, num_heads, head_dim]     (q_proj, reshaped :73)
 *   k_new   bf16 [B, num_new, num_kv_heads, head_dim]  (k_proj, :74)
 *   v_new   bf16 [B, num_new, num_kv_heads, head_dim]  (v_proj, :75)
 *   q_out   bf16 [B, num_new, num_heads, head_dim]
 *   k_cache, v_cache bf16 [num_blocks, num_kv_heads, block_size, head_dim]
 * head_dim is a multiple of 16 and at most 256.  Each rotated element is
 * x*cos + (-/+)x'*sin with each product and the sum rounded to fp32 (the
 * reference's broadcast_mul and add), then rounded to bf16. */
int kyro_rope_kv_write(kyro_ctx* ctx, const kyro_kv_params* p, int32_t num_new,
                       int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                       float rope_theta, const int32_t* pos_offsets, const void* q,
                       const void* k_new, const void* v_new, const int64_t* block_table,
                       const int64_t* context_lens, void* q_out, void* k_cache, void* v_cache);

/* ------------------------------------------------- tree acceptance */

/* Verification of a draft tree instead of a chain.  The reference has no
 * tree path; the rule is multi-candidate rejection sampling (SpecInfer,
 * Miao et al. 2023) with the arithmetic of kyro_math.h: at each node the
 * children are tried in index order against the target / draft
 * distributions of their parent, each rejection replaces p by
 * norm(max(p - q, 0)), an accepted child becomes the next node, and when
 * every child is rejected (or the node is a leaf) one token is drawn from
 * the current p.  Greedy modes accept the first child whose token is the
 * target's argmax and otherwise emit the argmax (speculative.rs:314-323 per
 * node). */
typedef struct kyro_tree_params {
  int32_t batch;       /* B                                                */
  int32_t num_nodes;   /* N <= 64, BFS order, node 0 = the root            */
  int32_t vocab;       /* V                                                */
  int32_t mode;        /* KYRO_ACCEPT_*                                    */
  float temperature;
  uint32_t step;       /* Philox counter word 3                            */
  uint64_t seed;       /* Philox key                                       */
  int64_t seq_offset;  /* global index of sequence 0                       */
} kyro_tree_params;

size_t kyro_spec_accept_tree_workspace_size(const kyro_tree_params* p);

/*   target_logits fp32 [B, N, V]  the target's next-token logits at node n
 *   draft_logits  fp32 [B, N, V]  the draft's, which node n's children were
 *                                 sampled from (NULL in greedy modes)
 *   node_tokens   int32 [B, N]    the token of node n (the root's is unused)
 *   parents       int32 [B, N]    parent of node n; -1 for the root; a
 *                                 parent precedes its children
 * Outputs: out_path [B, N] the accepted nodes, root first, -1 padded (the
 * path kyro_kv_commit_tree takes); out_path_len [B]; out_tokens [B, N] the
 * emitted tokens (the path's tokens after the root, then the drawn one),
 * -1 padded; out_num_tokens [B] (== out_path_len). */
int kyro_spec_accept_tree(kyro_ctx* ctx, const kyro_tree_params* p, const float* target_logits,
                          const float* draft_logits, const int32_t* node_tokens,
                          const int32_t* parents, int32_t* out_path, int32_t* out_path_len,
                          int32_t* out_tokens, int32_t* out_num_tokens, void* workspace,
                          size_t workspace_bytes);

/* ------------------------------------- tensor parallelism (vocab shards) */

/* The lm_head / vocabulary dimension split over a tensor-parallel group as
 * DistributedContext::shard_dim does it (src/distributed.rs:90-98): rank r
 * holds vocabulary entries [r*V/R, (r+1)*V/R).  The reference's all_reduce
 * (:61-79) is a stub; here a context joins its group through an NCCL
 * communicator it creates from a unique id that the caller's launcher
 * hands to every rank (rank 0 calls kyro_tp_unique_id).  NCCL is opened at
 * run time: libnccl.so.2, or the path in the KYRO_NCCL_LIBRARY variable. */
#define KYRO_TP_UNIQUE_ID_BYTES 128
int kyro_tp_unique_id(void* out /* KYRO_TP_UNIQUE_ID_BYTES bytes */);
/* Blocking: returns once all `world` ranks have joined.  With 2..8 ranks on
 * distinct GPUs that can map each other's memory (CUDA IPC over NVLink), the
 * sampler's exchange rounds then run as peer-memory stores with per-sender
 * flags instead of NCCL collectives; KYRO_TP_TRANSPORT=nccl in the
 * environment keeps NCCL.  The group agrees on one transport. */
int kyro_ctx_tp_init(kyro_ctx* ctx, const void* unique_id, int rank, int world);
/* The transport of the context's exchange rounds: 0 no group, 1 NCCL,
 * 2 NVLink peer memory. */
int kyro_ctx_tp_transport(kyro_ctx* ctx);

/* Failure injection and self-tests of the bounded waits.  No counterpart in
 * the reference, whose failure handling is host-side (deadlines,
 * src/scheduler/continuous_batching.rs:83-100; worker errors logged,
 * src/main.rs:146-148).  None of them faults or hangs a GPU.
 *
 * kyro_ctx_tp_inject_skip: this rank skips its next `rounds` peer-memory
 * exchange rounds while staying alive (it neither stores its payload nor
 * raises its flags), so its peers' waits run into the wait bound.  Only for
 * contexts whose exchange runs on peer memory.
 *
 * kyro_selftest_exchange_timeout: on one GPU, runs the exchange kernel as a
 * one-rank group over `region` (>= 4096 bytes of device memory, 256-byte
 * aligned, cleared by the call) with the round skipped, so it waits for a
 * flag that nothing sets; after the wait bound it sets
 * KYRO_DEV_WAIT_TIMEOUT and returns, leaving the context usable.
 *
 * kyro_selftest_watchdog: the host watchdog that guards NCCL collectives,
 * run on the caller's probe: arms `poll` with a bound of timeout_ms and
 * blocks until poll(user) returns nonzero (KYRO_OK) or the bound passes and
 * on_abort(user) has run once (KYRO_ERR_TIMEOUT).  Needs no GPU. */
int kyro_ctx_tp_inject_skip(kyro_ctx* ctx, int32_t rounds);
int kyro_selftest_exchange_timeout(kyro_ctx* ctx, void* region, size_t region_bytes);
int kyro_selftest_watchdog(uint32_t timeout_ms, int (*poll)(void* user),
                           void (*on_abort)(void* user), void* user);

/* Vocabulary-sharded kyro_spec_accept: p->vocab is the FULL vocabulary V
 * (divisible by the group size R); target_shard [B, k+1, V/R] and
 * draft_shard [B, k, V/R] are this rank's columns; draft_tokens hold global
 * ids.  Every rank passes identical params and gets identical outputs
 * (accept lengths, tokens with global ids, p/q at the drafts).  The
 * normaliser contract is then taken over R shards (chunks start at each
 * shard's first column; shard sums add in rank order), so the outputs equal
 * the CPU restatement with num_shards = R bit for bit; they can differ from
 * kyro_spec_accept on the full rows in the last bits of p and q, and so in
 * a decision whose test lands within those bits.  Four small collectives on the
 * context's stream: all-gathers of per-row maxima, per-row normaliser parts
 * with the owner rank's values at the draft tokens, per-sequence weight
 * totals, and an int32 max of the token id.  A rank that returns an error
 * before its collectives leaves the others waiting in NCCL, so callers
 * check arguments identically on every rank. */
size_t kyro_spec_accept_tp_workspace_size(const kyro_accept_params* p, int world);
int kyro_spec_accept_tp(kyro_ctx* ctx, const kyro_accept_params* p, const float* target_shard,
                        const float* draft_shard, const int32_t* draft_tokens,
                        int32_t* out_accept_len, int32_t* out_tokens, int32_t* out_num_tokens,
                        float* out_probs, void* workspace, size_t workspace_bytes);

/* Philox4x32-10 uniforms exactly as the kernels draw them (test aid):
 * out[i] = u for counter (seq, pos0 + i, stream, step), i < n. */
int kyro_philox_uniforms(kyro_ctx* ctx, uint64_t seed, uint32_t seq, uint32_t pos0,
                         uint32_t stream, uint32_t step, int32_t n, float* out);

/* Self-check of the sampler's arithmetic (test aid, no reference
 * counterpart): the kernels evaluate the contract's ky_exp in two faster
 * forms (exponent add; packed fp32x2 pairs).  This compares both with
 * ky_exp on every fp32 input in [-100, 0] and on -inf / NaN, on the
 * context's stream.  counts: device array of 2 u64, set to the number of
 * mismatching inputs of each form (0 and 0 when the forms agree). */
int kyro_selftest_exp(kyro_ctx* ctx, unsigned long long* counts);

#ifdef __cplusplus
}
#endif

#endif /* KYRO_SPEC_H */
