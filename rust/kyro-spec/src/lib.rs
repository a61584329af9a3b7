//! Safe wrapper of `libkyro_spec` for Kyro's speculative verifier.
//!
//! `VerifyCtx` owns one `kyro_ctx` (one per GPU worker; not `Sync`).  Its
//! methods take device pointers (from candle's `CudaStorage` in Kyro) and
//! enqueue on the context's stream.  Errors carry the library's message; the
//! verifier maps them to `candle_core::Error::Msg`, the error
//! `SpeculativeDecoder` already returns (src/speculative.rs:224):
//!
//! ```ignore
//! ctx.accept(&p, tgt, drf, drafts, &out, ws).map_err(|e| candle_core::Error::Msg(e.to_string()))?;
//! ```
//!
//! `step::VerifyStep` composes the batched verify step the worker's spec
//! branch runs (reserve -> RoPE + paged store -> attention -> accept ->
//! commit), as `kyro_b200/step.py` does for the Python harness.
use core::ffi::c_void;
use std::fmt;

pub use kyro_spec_sys as sys;

pub mod step;

/// A failed library call: the status code and the thread's last message.
#[derive(Debug, Clone)]
pub struct KyroError {
    pub status: i32,
    pub message: String,
}

impl fmt::Display for KyroError {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        write!(f, "kyro status {}: {}", self.status, self.message)
    }
}

impl std::error::Error for KyroError {}

pub type Result<T> = std::result::Result<T, KyroError>;

/// Map a status to `Ok` or the thread's last error message.
pub fn check(status: i32) -> Result<()> {
    if status == sys::KYRO_OK {
        return Ok(());
    }
    let mut buf = vec![0u8; 512];
    let n = unsafe { sys::kyro_last_error(buf.as_mut_ptr() as *mut _, buf.len()) };
    buf.truncate(n.min(511));
    Err(KyroError { status, message: String::from_utf8_lossy(&buf).into_owned() })
}

/// Device outputs of one acceptance call.
pub struct AcceptOut {
    pub accept_len: *mut i32, // [B]
    pub tokens: *mut i32,     // [B, k+1]
    pub num_tokens: *mut i32, // [B]
    pub probs: *mut f32,      // [B, k, 2] or null
}

/// A caller-owned device buffer the library may use as scratch.
#[derive(Clone, Copy)]
pub struct Workspace {
    pub ptr: *mut c_void,
    pub bytes: usize,
}

pub struct VerifyCtx {
    raw: *mut sys::kyro_ctx,
}

impl VerifyCtx {
    /// A context on `device`, enqueueing on `stream` (a `cudaStream_t`).
    pub fn new(device: i32, stream: *mut c_void) -> Result<Self> {
        let mut raw = core::ptr::null_mut();
        check(unsafe { sys::kyro_ctx_create(device, stream, &mut raw) })?;
        Ok(Self { raw })
    }

    pub fn raw(&self) -> *mut sys::kyro_ctx {
        self.raw
    }

    pub fn set_stream(&self, stream: *mut c_void) -> Result<()> {
        check(unsafe { sys::kyro_ctx_set_stream(self.raw, stream) })
    }

    /// Bound of this context's waits on other ranks, in milliseconds.
    pub fn set_wait_timeout(&self, ms: u32) -> Result<()> {
        check(unsafe { sys::kyro_ctx_set_wait_timeout(self.raw, ms) })
    }

    /// Synchronise the stream and read (and clear) the device status word.
    pub fn device_status(&self) -> Result<u32> {
        let mut flags = 0u32;
        check(unsafe { sys::kyro_ctx_device_status(self.raw, &mut flags, 1) })?;
        Ok(flags)
    }

    /// Bytes of scratch `accept` needs for these parameters.
    pub fn accept_workspace_size(p: &sys::kyro_accept_params) -> usize {
        unsafe { sys::kyro_spec_accept_workspace_size(p) }
    }

    /// Batched `SpeculativeDecoder::verify_drafts` (src/speculative.rs:286-339):
    /// target logits [B,k+1,V] f32, draft logits [B,k,V] f32 (stochastic
    /// mode), draft tokens [B,k] i32, all device pointers.
    ///
    /// # Safety
    /// Every pointer must address device memory of the documented shape on
    /// this context's device, valid until the stream reaches this call.
    pub unsafe fn accept(&self, p: &sys::kyro_accept_params, target_logits: *const f32,
                         draft_logits: *const f32, draft_tokens: *const i32, out: &AcceptOut,
                         ws: Workspace) -> Result<()> {
        check(sys::kyro_spec_accept(self.raw, p, target_logits, draft_logits, draft_tokens,
                                    out.accept_len, out.tokens, out.num_tokens, out.probs,
                                    ws.ptr, ws.bytes))
    }

    /// `accept` without a workspace, for hosts that cannot allocate device
    /// memory (the library's static scratch; one call at a time per GPU).
    ///
    /// # Safety
    /// As for `accept`.
    pub unsafe fn accept_static(&self, p: &sys::kyro_accept_params, target_logits: *const f32,
                                draft_logits: *const f32, draft_tokens: *const i32,
                                out: &AcceptOut) -> Result<()> {
        check(sys::kyro_spec_accept_static(self.raw, p, target_logits, draft_logits,
                                           draft_tokens, out.accept_len, out.tokens,
                                           out.num_tokens, out.probs))
    }

    /// On-device draft sampling (Philox stream 0), replacing the draft loop's
    /// argmax and host sync (src/speculative.rs:229-241).
    ///
    /// # Safety
    /// As for `accept`.
    pub unsafe fn sample(&self, p: &sys::kyro_sample_params, logits: *const f32,
                         out_tokens: *mut i32, out_probs: *mut f32, ws: Workspace) -> Result<()> {
        check(sys::kyro_sample_tokens(self.raw, p, logits, out_tokens, out_probs, ws.ptr,
                                      ws.bytes))
    }
}

impl Drop for VerifyCtx {
    fn drop(&mut self) {
        unsafe {
            sys::kyro_ctx_destroy(self.raw);
        }
    }
}
