//! The batched verify step of the worker's speculative branch
//! (`Worker::run_loop`, src/worker.rs:134-205, with `SpeculativeDecoder::step`,
//! src/speculative.rs:342-353), on device pointers the worker owns:
//!
//! 1. `kyro_kv_reserve`: k + 1 slots per sequence (BlockManager::allocate,
//!    src/scheduler/block_manager.rs:109-125, at decode time);
//! 2. per attention layer of the target forward: `kyro_rope_kv_write`
//!    (RoPE at `index + i` and the paged store, src/model/llama.rs:73-82)
//!    then `kyro_verify_attention` (the k + 1 query rows);
//! 3. `kyro_spec_accept` on the lm_head's logits;
//! 4. `kyro_kv_commit`: keep accept_len + 1 slots, free the rest.
//!
//! One host read per step, of the emitted tokens, after `commit`.
use core::ffi::c_void;

use crate::{check, sys, AcceptOut, Result, VerifyCtx, Workspace};

/// The worker's device mirror of BlockManager for one batch.
pub struct KvState {
    pub block_table: *mut i64,  // [B, max_blocks]
    pub context_lens: *mut i64, // [B]
    pub free_stack: *mut i32,   // [num_blocks]
    pub free_top: *mut i32,     // [1]
    pub ref_counts: *mut i32,   // [num_blocks]
    pub kv: sys::kyro_kv_params,
}

/// One attention layer's inputs and outputs for the verify forward.
pub struct LayerIo {
    pub q: *const c_void,     // bf16 [B, k+1, Hq, D], un-rotated (q_proj)
    pub k_new: *const c_void, // bf16 [B, k+1, Hkv, D] (k_proj)
    pub v_new: *const c_void, // bf16 [B, k+1, Hkv, D] (v_proj)
    pub q_rot: *mut c_void,   // bf16 [B, k+1, Hq, D]
    pub k_cache: *mut c_void, // bf16 [num_blocks, Hkv, block_size, D]
    pub v_cache: *mut c_void,
    pub out: *mut c_void,     // bf16 [B, k+1, Hq, D]
}

pub struct VerifyStep<'a> {
    pub ctx: &'a VerifyCtx,
    pub attn: sys::kyro_attn_params,
    pub rope_theta: f32,
}

impl<'a> VerifyStep<'a> {
    /// Step 1: reserve k + 1 slots in every sequence.  `ok[b] == 0` marks a
    /// sequence the free list could not serve (allocate() -> None).
    ///
    /// # Safety
    /// The state's pointers address this context's device memory.
    pub unsafe fn reserve(&self, st: &KvState, ok: *mut i32) -> Result<()> {
        check(sys::kyro_kv_reserve(self.ctx.raw(), &st.kv, self.attn.num_query, st.block_table,
                                   st.context_lens, st.free_stack, st.free_top, st.ref_counts,
                                   ok))
    }

    /// Step 2, for one layer: RoPE + paged store, then verify attention.
    ///
    /// # Safety
    /// As for `reserve`; `io` holds device pointers of the documented shapes.
    pub unsafe fn layer(&self, st: &KvState, io: &LayerIo, ws: Workspace) -> Result<()> {
        let a = &self.attn;
        check(sys::kyro_rope_kv_write(self.ctx.raw(), &st.kv, a.num_query, a.num_heads,
                                      a.num_kv_heads, a.head_dim, self.rope_theta,
                                      core::ptr::null(), io.q, io.k_new, io.v_new,
                                      st.block_table, st.context_lens, io.q_rot, io.k_cache,
                                      io.v_cache))?;
        check(sys::kyro_verify_attention(self.ctx.raw(), a, io.q_rot, io.k_cache, io.v_cache,
                                         st.block_table, st.context_lens, core::ptr::null(),
                                         io.out, ws.ptr, ws.bytes))
    }

    /// Steps 3 and 4: acceptance on the target / draft logits, then commit.
    ///
    /// # Safety
    /// As for `reserve`; logits and tokens are device pointers.
    pub unsafe fn accept_and_commit(&self, st: &KvState, p: &sys::kyro_accept_params,
                                    target_logits: *const f32, draft_logits: *const f32,
                                    draft_tokens: *const i32, out: &AcceptOut, ws: Workspace)
                                    -> Result<()> {
        self.ctx.accept(p, target_logits, draft_logits, draft_tokens, out, ws)?;
        check(sys::kyro_kv_commit(self.ctx.raw(), &st.kv, self.attn.num_query, out.accept_len,
                                  st.block_table, st.context_lens, st.free_stack, st.free_top,
                                  st.ref_counts))
    }
}
