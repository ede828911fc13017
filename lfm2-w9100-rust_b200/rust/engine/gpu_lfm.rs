//! Drop-in replacement of the reference's `engine/src/gpu_lfm.rs` (and its
//! `gpu_lfm/resident_graph.rs` submodule): the same public `GpuEngine` methods
//! that `main.rs`, `bin/api_stream.rs` and `bin/persistent.rs` call, over the
//! B200 engine's C ABI (`lfm2-cuda-sys`, include/lfm_cuda.h). The callers keep
//! compiling unchanged: `engine.gpu.device_name`, `engine.gpu.dispatch_count()`
//! and the W9100 submission hooks `engine.gpu.ctx.set_submission_context(..)` /
//! `engine.gpu.ctx.profile_forward(..)` exist (the hooks do nothing on B200).
//!
//! Errors cross the boundary as a status plus the engine's message; no C++
//! exception or Rust panic crosses it. `set_ctx` keeps the reference's
//! infallible signature (gpu_lfm.rs:117-119); a rejected context length
//! (above 4096) is reported by the next `forward` / `forward_token` call, and
//! `try_set_ctx` returns it at once.
use crate::{lfm::Hyperparams, model_file::ModelFile};
use anyhow::{anyhow, Result};
use lfm2_cuda_sys as sys;
use std::ffi::{CStr, CString};

/// The W9100 submission context of the reference (vulkan.rs); no-ops here.
pub struct SubmissionCtx;
impl SubmissionCtx {
    pub fn set_submission_context(&self, _phase: &str, _prompt_tokens: usize) {}
    pub fn profile_forward(&self, _t0_ns: u64, _t1_ns: u64, _pos: usize, _n: usize) -> Result<()> {
        Ok(())
    }
}

/// What callers read from `engine.gpu` (ops.rs GpuOps fields they touch).
pub struct GpuStats {
    pub device_name: String,
    pub ctx: SubmissionCtx,
    e: *mut sys::lfm_engine,
}
impl GpuStats {
    fn counters(&self) -> sys::lfm_counters {
        let mut c = sys::lfm_counters::default();
        unsafe { sys::lfm_counters_get(self.e, &mut c) };
        c
    }
    /// gpu_dispatch_count of the result lines (kernel launches on B200).
    pub fn dispatch_count(&self) -> u64 {
        self.counters().kernel_launches
    }
    pub fn gpu_argmax_dispatches(&self) -> u64 {
        self.counters().gpu_argmax
    }
    pub fn decode_command_buffer_reuses(&self) -> u64 {
        self.counters().graph_replays
    }
}

pub struct GpuEngine {
    e: *mut sys::lfm_engine,
    pub hp: Hyperparams,
    pub gpu: GpuStats,
    pending: Option<anyhow::Error>,
}

fn message(e: *mut sys::lfm_engine) -> String {
    let p = unsafe { if e.is_null() { sys::lfm_global_error() } else { sys::lfm_last_error(e) } };
    unsafe { CStr::from_ptr(p) }.to_string_lossy().into_owned()
}
fn check(e: *mut sys::lfm_engine, st: sys::lfm_status) -> Result<()> {
    if st == sys::LFM_OK {
        Ok(())
    } else {
        Err(anyhow!("{} (status {st})", message(e)))
    }
}

impl GpuEngine {
    /// gpu_lfm.rs:51-115: parse, validate the geometry (lfm.rs:102-145, the
    /// same checks the library repeats), repack and upload every weight.
    pub fn load(model: &ModelFile) -> Result<Self> {
        let hp = crate::lfm::load_hyperparams(model)?;
        let path = CString::new(model.file_path())?;
        let device = std::env::var("LFM_CUDA_DEVICE").ok().and_then(|v| v.parse().ok()).unwrap_or(0);
        let mut e = std::ptr::null_mut();
        check(std::ptr::null_mut(), unsafe { sys::lfm_engine_create(path.as_ptr(), device, &mut e) })?;
        let name = unsafe { CStr::from_ptr(sys::lfm_device_name(e)) }.to_string_lossy().into_owned();
        Ok(GpuEngine { e, hp, gpu: GpuStats { device_name: name, ctx: SubmissionCtx, e }, pending: None })
    }

    /// gpu_lfm.rs:117-119 (infallible there); a rejected length is returned
    /// by the next forward call.
    pub fn set_ctx(&mut self, ctx: usize) {
        if let Err(err) = self.try_set_ctx(ctx) {
            self.pending = Some(err);
        }
    }

    /// set_ctx with the library's status (ctx must be 1..=4096).
    pub fn try_set_ctx(&mut self, ctx: usize) -> Result<()> {
        let c = u32::try_from(ctx).map_err(|_| anyhow!("context length {ctx} out of range"))?;
        let r = check(self.e, unsafe { sys::lfm_engine_set_ctx(self.e, c) });
        if r.is_ok() {
            self.pending = None;
        }
        r
    }

    fn take_pending(&mut self) -> Result<()> {
        match self.pending.take() {
            Some(err) => Err(err),
            None => Ok(()),
        }
    }

    pub fn device_name(&self) -> String {
        self.gpu.device_name.clone()
    }

    /// gpu_lfm.rs:243-245: full logits of the last token.
    pub fn forward(&mut self, ids: &[u32], start_pos: i64) -> Result<Vec<f32>> {
        self.take_pending()?;
        let mut out = vec![0f32; self.hp.vocab];
        check(self.e, unsafe {
            sys::lfm_forward_logits(self.e, ids.as_ptr(), ids.len() as u32, start_pos, out.as_mut_ptr())
        })?;
        Ok(out)
    }

    /// resident_graph.rs:90-101: device argmax of the last token (1..=64 ids).
    pub fn forward_token(&mut self, ids: &[u32], position: usize) -> Result<u32> {
        self.take_pending()?;
        let mut next = 0u32;
        check(self.e, unsafe {
            sys::lfm_forward_token(self.e, ids.as_ptr(), ids.len() as u32, position as u32, &mut next)
        })?;
        Ok(next)
    }

    /// resident_graph.rs:105-115
    pub fn reset_session(&mut self) -> Result<()> {
        check(self.e, unsafe { sys::lfm_reset_session(self.e) })
    }

    /// resident_graph.rs:119-158
    pub fn restore_session(&self, valid_tokens: usize, bytes: &[u8]) -> Result<()> {
        check(self.e, unsafe { sys::lfm_restore_cache(self.e, valid_tokens as u32, bytes.as_ptr(), bytes.len()) })
    }

    /// resident_graph.rs:572-602 (same byte layout)
    pub fn snapshot_resident_cache(&self, valid_tokens: usize) -> Result<Vec<u8>> {
        let mut len = 0usize;
        check(self.e, unsafe {
            sys::lfm_snapshot_cache(self.e, valid_tokens as u32, std::ptr::null_mut(), 0, &mut len)
        })?;
        let mut buf = vec![0u8; len];
        check(self.e, unsafe {
            sys::lfm_snapshot_cache(self.e, valid_tokens as u32, buf.as_mut_ptr(), len, &mut len)
        })?;
        Ok(buf)
    }

    /// resident_graph.rs:561-568
    pub fn snapshot_resident_logits(&self) -> Result<Vec<f32>> {
        let mut out = vec![0f32; self.hp.vocab];
        check(self.e, unsafe { sys::lfm_snapshot_logits(self.e, out.as_mut_ptr()) })?;
        Ok(out)
    }

    /// Device-resident greedy decode (no reference counterpart: the
    /// reference reads the argmax back every step): `steps` tokens fed back
    /// on the device, returned with the device time of the loop.
    pub fn decode_loop(&mut self, first_token: u32, start_pos: usize, steps: usize) -> Result<(Vec<u32>, f32)> {
        self.take_pending()?;
        let mut out = vec![0u32; steps];
        let mut ms = 0f32;
        check(self.e, unsafe {
            sys::lfm_decode_loop(self.e, first_token, start_pos as u32, steps as u32, out.as_mut_ptr(), &mut ms)
        })?;
        Ok((out, ms))
    }
}

impl Drop for GpuEngine {
    fn drop(&mut self) {
        unsafe { sys::lfm_engine_destroy(self.e) }
    }
}
