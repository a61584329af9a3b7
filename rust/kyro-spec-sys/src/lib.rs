//! Raw declarations of the C ABI in `include/kyro_spec.h`, one to one.
//!
//! The verify step of `SpeculativeDecoder` (Kyro's `src/speculative.rs`)
//! calls these through the safe wrapper crate `kyro-spec`.  Every function
//! returns an `int` status (`KYRO_OK` = 0); `kyro_last_error` gives the
//! calling thread's message.  The caller owns every device buffer; calls
//! enqueue on the context's CUDA stream and return without a host sync.
//! `tests/test_rust_bindings.py` checks these declarations against the
//! header (names, argument counts, struct fields).
#![allow(non_camel_case_types)]
#![no_std]

use core::ffi::{c_char, c_int, c_void};

pub const KYRO_VERSION: c_int = 1;

pub const KYRO_OK: c_int = 0;
pub const KYRO_ERR_INVALID_ARG: c_int = 1;
pub const KYRO_ERR_CUDA: c_int = 2;
pub const KYRO_ERR_NCCL: c_int = 3;
pub const KYRO_ERR_TIMEOUT: c_int = 4;
pub const KYRO_ERR_OOB: c_int = 5;
pub const KYRO_ERR_OOM: c_int = 6;
pub const KYRO_ERR_UNSUPPORTED: c_int = 7;
pub const KYRO_ERR_WORKSPACE: c_int = 8;

pub const KYRO_DEV_BAD_TOKEN: u32 = 0x1;
pub const KYRO_DEV_BAD_BLOCK: u32 = 0x2;
pub const KYRO_DEV_BAD_LENGTH: u32 = 0x4;
pub const KYRO_DEV_WAIT_TIMEOUT: u32 = 0x8;
pub const KYRO_DEV_STACK_OVERFLOW: u32 = 0x10;

pub const KYRO_ACCEPT_STOCHASTIC: i32 = 0;
pub const KYRO_ACCEPT_GREEDY: i32 = 1;
pub const KYRO_ACCEPT_GREEDY_REF: i32 = 2;

pub const KYRO_ACCEPT_STATIC_SCRATCH_BYTES: usize = 8 << 20;
pub const KYRO_TP_UNIQUE_ID_BYTES: usize = 128;

/// Opaque per-GPU context.
#[repr(C)]
pub struct kyro_ctx {
    _private: [u8; 0],
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct kyro_accept_params {
    pub batch: i32,
    pub num_draft: i32,
    pub vocab: i32,
    pub mode: i32,
    pub temperature: f32,
    pub step: u32,
    pub seed: u64,
    pub seq_offset: i64,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct kyro_sample_params {
    pub batch: i32,
    pub num_pos: i32,
    pub vocab: i32,
    pub temperature: f32,
    pub step: u32,
    pub seq_stride: u32,
    pub seed: u64,
    pub seq_offset: i64,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct kyro_attn_params {
    pub batch: i32,
    pub num_query: i32,
    pub num_heads: i32,
    pub num_kv_heads: i32,
    pub head_dim: i32,
    pub block_size: i32,
    pub max_blocks_per_seq: i32,
    pub num_blocks: i32,
    pub scale: f32,
    pub kv_split_blocks: i32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct kyro_kv_params {
    pub batch: i32,
    pub block_size: i32,
    pub max_blocks_per_seq: i32,
    pub num_blocks: i32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct kyro_tree_params {
    pub batch: i32,
    pub num_nodes: i32,
    pub vocab: i32,
    pub mode: i32,
    pub temperature: f32,
    pub step: u32,
    pub seed: u64,
    pub seq_offset: i64,
}

extern "C" {
    // ------------------------------------------------------------ context
    pub fn kyro_ctx_create(device: c_int, stream: *mut c_void, out: *mut *mut kyro_ctx) -> c_int;
    pub fn kyro_ctx_destroy(ctx: *mut kyro_ctx) -> c_int;
    pub fn kyro_ctx_set_stream(ctx: *mut kyro_ctx, stream: *mut c_void) -> c_int;
    pub fn kyro_ctx_device_status(ctx: *mut kyro_ctx, out_flags: *mut u32, clear: c_int) -> c_int;
    pub fn kyro_ctx_set_wait_timeout(ctx: *mut kyro_ctx, ms: u32) -> c_int;
    pub fn kyro_last_error(buf: *mut c_char, len: usize) -> usize;
    pub fn kyro_status_string(status: c_int) -> *const c_char;
    pub fn kyro_version() -> c_int;
    pub fn kyro_kernel_names() -> *const c_char;

    // ------------------------------------------------------------ K2: acceptance
    pub fn kyro_spec_accept_workspace_size(p: *const kyro_accept_params) -> usize;
    pub fn kyro_spec_accept(
        ctx: *mut kyro_ctx, p: *const kyro_accept_params, target_logits: *const f32,
        draft_logits: *const f32, draft_tokens: *const i32, out_accept_len: *mut i32,
        out_tokens: *mut i32, out_num_tokens: *mut i32, out_probs: *mut f32,
        workspace: *mut c_void, workspace_bytes: usize,
    ) -> c_int;
    pub fn kyro_spec_accept_static(
        ctx: *mut kyro_ctx, p: *const kyro_accept_params, target_logits: *const f32,
        draft_logits: *const f32, draft_tokens: *const i32, out_accept_len: *mut i32,
        out_tokens: *mut i32, out_num_tokens: *mut i32, out_probs: *mut f32,
    ) -> c_int;
    pub fn kyro_spec_accept_commit(
        ctx: *mut kyro_ctx, p: *const kyro_accept_params, target_logits: *const f32,
        draft_logits: *const f32, draft_tokens: *const i32, out_accept_len: *mut i32,
        out_tokens: *mut i32, out_num_tokens: *mut i32, out_probs: *mut f32,
        workspace: *mut c_void, workspace_bytes: usize, kv: *const kyro_kv_params, num_new: i32,
        num_new_next: i32, block_table: *mut i64, context_lens: *mut i64, free_stack: *mut i32,
        free_top: *mut i32, ref_counts: *mut i32, out_ok: *mut i32,
    ) -> c_int;
    pub fn kyro_sample_workspace_size(p: *const kyro_sample_params) -> usize;
    pub fn kyro_sample_tokens(
        ctx: *mut kyro_ctx, p: *const kyro_sample_params, logits: *const f32,
        out_tokens: *mut i32, out_probs: *mut f32, workspace: *mut c_void, workspace_bytes: usize,
    ) -> c_int;

    // ------------------------------------------------------------ K1: verify attention
    pub fn kyro_verify_attention_workspace_size(p: *const kyro_attn_params) -> usize;
    pub fn kyro_verify_attention(
        ctx: *mut kyro_ctx, p: *const kyro_attn_params, q: *const c_void, k_cache: *const c_void,
        v_cache: *const c_void, block_table: *const i64, context_lens: *const i64,
        tree_mask: *const u64, out: *mut c_void, workspace: *mut c_void, workspace_bytes: usize,
    ) -> c_int;
    pub fn kyro_verify_attention_rope(
        ctx: *mut kyro_ctx, p: *const kyro_attn_params, rope_theta: f32, pos_offsets: *const i32,
        q: *const c_void, k_new: *const c_void, v_new: *const c_void, k_cache: *mut c_void,
        v_cache: *mut c_void, block_table: *const i64, context_lens: *const i64,
        tree_mask: *const u64, out: *mut c_void, workspace: *mut c_void, workspace_bytes: usize,
    ) -> c_int;

    // ------------------------------------------------------------ K3: KV commit / rollback
    pub fn kyro_kv_reserve(
        ctx: *mut kyro_ctx, p: *const kyro_kv_params, num_new: i32, block_table: *mut i64,
        context_lens: *const i64, free_stack: *mut i32, free_top: *mut i32,
        ref_counts: *mut i32, out_ok: *mut i32,
    ) -> c_int;
    pub fn kyro_kv_reserve_cow(
        ctx: *mut kyro_ctx, p: *const kyro_kv_params, num_new: i32, num_layers: i32,
        k_caches: *const *mut c_void, v_caches: *const *mut c_void, num_kv_heads: i32,
        head_dim: i32, block_table: *mut i64, context_lens: *const i64, free_stack: *mut i32,
        free_top: *mut i32, ref_counts: *mut i32, out_ok: *mut i32, out_cow: *mut i32,
    ) -> c_int;
    pub fn kyro_kv_commit(
        ctx: *mut kyro_ctx, p: *const kyro_kv_params, num_new: i32, accept_len: *const i32,
        block_table: *mut i64, context_lens: *mut i64, free_stack: *mut i32, free_top: *mut i32,
        ref_counts: *mut i32,
    ) -> c_int;
    pub fn kyro_kv_commit_tree(
        ctx: *mut kyro_ctx, p: *const kyro_kv_params, num_nodes: i32, path: *const i32,
        path_len: *const i32, num_layers: i32, k_caches: *const *mut c_void,
        v_caches: *const *mut c_void, num_kv_heads: i32, head_dim: i32, block_table: *mut i64,
        context_lens: *mut i64, free_stack: *mut i32, free_top: *mut i32, ref_counts: *mut i32,
    ) -> c_int;
    pub fn kyro_kv_write(
        ctx: *mut kyro_ctx, p: *const kyro_kv_params, num_new: i32, num_kv_heads: i32,
        head_dim: i32, k_new: *const c_void, v_new: *const c_void, block_table: *const i64,
        context_lens: *const i64, k_cache: *mut c_void, v_cache: *mut c_void,
    ) -> c_int;
    pub fn kyro_rope_kv_write(
        ctx: *mut kyro_ctx, p: *const kyro_kv_params, num_new: i32, num_heads: i32,
        num_kv_heads: i32, head_dim: i32, rope_theta: f32, pos_offsets: *const i32,
        q: *const c_void, k_new: *const c_void, v_new: *const c_void, block_table: *const i64,
        context_lens: *const i64, q_out: *mut c_void, k_cache: *mut c_void, v_cache: *mut c_void,
    ) -> c_int;

    // ------------------------------------------------------------ tree acceptance
    pub fn kyro_spec_accept_tree_workspace_size(p: *const kyro_tree_params) -> usize;
    pub fn kyro_spec_accept_tree(
        ctx: *mut kyro_ctx, p: *const kyro_tree_params, target_logits: *const f32,
        draft_logits: *const f32, node_tokens: *const i32, parents: *const i32,
        out_path: *mut i32, out_path_len: *mut i32, out_tokens: *mut i32,
        out_num_tokens: *mut i32, workspace: *mut c_void, workspace_bytes: usize,
    ) -> c_int;

    // ------------------------------------------------------------ tensor parallelism
    pub fn kyro_tp_unique_id(out: *mut c_void) -> c_int;
    pub fn kyro_ctx_tp_init(ctx: *mut kyro_ctx, unique_id: *const c_void, rank: c_int,
                            world: c_int) -> c_int;
    pub fn kyro_ctx_tp_transport(ctx: *mut kyro_ctx) -> c_int;
    pub fn kyro_ctx_tp_inject_skip(ctx: *mut kyro_ctx, rounds: i32) -> c_int;
    pub fn kyro_selftest_exchange_timeout(ctx: *mut kyro_ctx, region: *mut c_void,
                                          region_bytes: usize) -> c_int;
    pub fn kyro_selftest_watchdog(
        timeout_ms: u32, poll: Option<unsafe extern "C" fn(*mut c_void) -> c_int>,
        on_abort: Option<unsafe extern "C" fn(*mut c_void)>, user: *mut c_void,
    ) -> c_int;
    pub fn kyro_spec_accept_tp_workspace_size(p: *const kyro_accept_params, world: c_int) -> usize;
    pub fn kyro_spec_accept_tp(
        ctx: *mut kyro_ctx, p: *const kyro_accept_params, target_shard: *const f32,
        draft_shard: *const f32, draft_tokens: *const i32, out_accept_len: *mut i32,
        out_tokens: *mut i32, out_num_tokens: *mut i32, out_probs: *mut f32,
        workspace: *mut c_void, workspace_bytes: usize,
    ) -> c_int;

    // ------------------------------------------------------------ test aids
    pub fn kyro_philox_uniforms(ctx: *mut kyro_ctx, seed: u64, seq: u32, pos0: u32, stream: u32,
                                step: u32, n: i32, out: *mut f32) -> c_int;
    pub fn kyro_selftest_exp(ctx: *mut kyro_ctx, counts: *mut u64) -> c_int;
}
