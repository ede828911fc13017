//! Raw bindings of `include/lfm_cuda.h`, the C ABI of the B200 engine that
//! replaces the reference's `lfm2_engine::gpu_lfm::GpuEngine`
//! (engine/src/gpu_lfm.rs:23-245, engine/src/gpu_lfm/resident_graph.rs:90-602).
//! Every declaration mirrors the header one to one (same order of arguments,
//! same widths); `tests/test_c_abi.py` checks the function list, the argument
//! counts and the `#[repr(C)]` struct layouts against the header.
#![allow(non_camel_case_types)]
use std::os::raw::{c_char, c_int, c_void};

pub type lfm_status = i32;
pub const LFM_OK: lfm_status = 0;
pub const LFM_ERR_ARG: lfm_status = 1;
pub const LFM_ERR_MODEL: lfm_status = 2;
pub const LFM_ERR_CUDA: lfm_status = 3;
pub const LFM_ERR_STATE: lfm_status = 4;
pub const LFM_ERR_DEVICE: lfm_status = 5;
pub const LFM_MAX_CTX: u32 = 4096;
pub const LFM_PREFILL_CHUNK: u32 = 64;
pub const LFM_EP_OWN_SESSION: u32 = 0xFFFF_FFFF;

/// Opaque engine handle.
#[repr(C)]
pub struct lfm_engine {
    _p: [u8; 0],
}

/// Opaque streaming-text handle.
#[repr(C)]
pub struct lfm_text {
    _p: [u8; 0],
}

/// `lfm_hparams` (engine/src/lfm.rs:31-49).
#[repr(C)]
#[derive(Clone, Copy)]
pub struct lfm_hparams {
    pub dim: u32,
    pub heads: u32,
    pub head_dim: u32,
    pub n_layers: u32,
    pub vocab: u32,
    pub n_expert: u32,
    pub n_used: u32,
    pub expert_ff: u32,
    pub n_ff: u32,
    pub dense_lead: u32,
    pub conv_l_cache: u32,
    pub eos: u32,
    pub eps: f32,
    pub rope_theta: f32,
    pub kv_heads: [u32; 64],
}

/// `lfm_counters` (the counters of main.rs:273-280 and persistent.rs:230-242).
#[repr(C)]
#[derive(Clone, Copy, Default)]
pub struct lfm_counters {
    pub kernel_launches: u64,
    pub gpu_argmax: u64,
    pub graph_replays: u64,
    pub graph_captures: u64,
    pub prefill_tokens: u64,
    pub expert_grouped_launches: u64,
}

extern "C" {
    // ---- engine lifetime and the GpuEngine surface
    pub fn lfm_model_inspect(gguf_path: *const c_char, out: *mut lfm_hparams) -> lfm_status;
    pub fn lfm_engine_create(gguf_path: *const c_char, device: c_int, out: *mut *mut lfm_engine) -> lfm_status;
    pub fn lfm_engine_destroy(e: *mut lfm_engine);
    pub fn lfm_engine_set_ctx(e: *mut lfm_engine, ctx: u32) -> lfm_status;
    pub fn lfm_hparams_get(e: *mut lfm_engine, out: *mut lfm_hparams) -> lfm_status;
    pub fn lfm_forward_logits(e: *mut lfm_engine, ids: *const u32, n: u32, start_pos: i64, logits: *mut f32)
        -> lfm_status;
    pub fn lfm_forward_token(e: *mut lfm_engine, ids: *const u32, n: u32, position: u32, next_token: *mut u32)
        -> lfm_status;
    pub fn lfm_generate(e: *mut lfm_engine, prompt: *const u32, prompt_len: u32, n: u32, eos: u32,
                        out_tokens: *mut u32, n_out: *mut u32) -> lfm_status;
    pub fn lfm_decode_loop(e: *mut lfm_engine, first_token: u32, start_pos: u32, steps: u32, out_tokens: *mut u32,
                           device_ms: *mut f32) -> lfm_status;
    pub fn lfm_last_device_ms(e: *mut lfm_engine) -> f32;
    // ---- independent sessions decoded together
    pub fn lfm_batch_create(e: *mut lfm_engine, n_sessions: u32) -> lfm_status;
    pub fn lfm_batch_prefill(e: *mut lfm_engine, session: u32, ids: *const u32, n: u32, next_token: *mut u32)
        -> lfm_status;
    pub fn lfm_batch_prefill_many(e: *mut lfm_engine, sessions: *const u32, ids: *const u32, lens: *const u32,
                                  count: u32, next_tokens: *mut u32) -> lfm_status;
    pub fn lfm_batch_decode(e: *mut lfm_engine, sessions: *const u32, tokens: *const u32, positions: *const u32,
                            count: u32, next_tokens: *mut u32) -> lfm_status;
    pub fn lfm_batch_logits(e: *mut lfm_engine, index: u32, logits: *mut f32) -> lfm_status;
    // ---- expert-parallel prompt path (one process per GPU)
    pub fn lfm_ep_unique_id(id_out: *mut u8) -> lfm_status;
    pub fn lfm_ep_init(e: *mut lfm_engine, id: *const u8, rank: c_int, world: c_int) -> lfm_status;
    pub fn lfm_ep_prefill(e: *mut lfm_engine, session: u32, ids: *const u32, n: u32, next_token: *mut u32)
        -> lfm_status;
    pub fn lfm_ep_plan(sel: *const i32, nslots: u32, world: u32, counts: *mut i32, order: *mut i32) -> lfm_status;
    pub fn lfm_ep_finalize(e: *mut lfm_engine) -> lfm_status;
    // ---- diagnostics
    pub fn lfm_step_trace(e: *mut lfm_engine, enable: c_int, out: *mut u64, cap: usize, n_stages: *mut u32,
                          n_ctas: *mut u32) -> lfm_status;
    pub fn lfm_engine_info(e: *mut lfm_engine) -> *const c_char;
    // ---- session state
    pub fn lfm_reset_session(e: *mut lfm_engine) -> lfm_status;
    pub fn lfm_snapshot_cache(e: *mut lfm_engine, valid: u32, buf: *mut u8, cap: usize, len: *mut usize)
        -> lfm_status;
    pub fn lfm_restore_cache(e: *mut lfm_engine, valid: u32, buf: *const u8, len: usize) -> lfm_status;
    pub fn lfm_snapshot_logits(e: *mut lfm_engine, logits: *mut f32) -> lfm_status;
    pub fn lfm_counters_get(e: *mut lfm_engine, out: *mut lfm_counters) -> lfm_status;
    pub fn lfm_device_name(e: *mut lfm_engine) -> *const c_char;
    pub fn lfm_last_error(e: *mut lfm_engine) -> *const c_char;
    pub fn lfm_global_error() -> *const c_char;
    // ---- kernel-level entry points (device pointers, optional cudaStream_t)
    pub fn lfm_q6k_device_bytes(in_dim: u32, rows: u32) -> usize;
    pub fn lfm_q6k_upload(gguf_rows: *const u8, in_dim: u32, rows: u32, dst_dev: *mut c_void) -> lfm_status;
    pub fn lfm_q6k_dequant(w_dev: *const c_void, in_dim: u32, rows: u32, row0: u32, nrows: u32, out_dev: *mut f32,
                           stream: *mut c_void) -> lfm_status;
    pub fn lfm_q6k_matmul(w_dev: *const c_void, in_dim: u32, rows: u32, x_dev: *const f32, n: u32, y_dev: *mut f32,
                          stream: *mut c_void) -> lfm_status;
    pub fn lfm_q6k_routed(w_dev: *const c_void, in_dim: u32, rows: u32, n_expert: u32, expert_ids_dev: *const i32,
                          x_dev: *const f32, x_stride: u32, y_dev: *mut f32, stream: *mut c_void) -> lfm_status;
    pub fn lfm_route(logits_dev: *const f32, bias_dev: *const f32, n_expert: u32, n: u32, sel_ids_dev: *mut i32,
                     sel_w_dev: *mut f32, stream: *mut c_void) -> lfm_status;
    pub fn lfm_argmax(x_dev: *const f32, n: u32, out_dev: *mut u32, stream: *mut c_void) -> lfm_status;
    pub fn lfm_argmax_noalloc(x_dev: *const f32, n: u32, out_dev: *mut u32, stream: *mut c_void) -> lfm_status;
    pub fn lfm_tc_gemm_f16(a_dev: *const c_void, b_dev: *const c_void, m: u32, n: u32, k: u32, c_dev: *mut f32,
                           stream: *mut c_void) -> lfm_status;
    pub fn lfm_tc_gemm_f16_bmn(a_dev: *const c_void, b_dev: *const c_void, m: u32, k: u32, c_dev: *mut f32,
                               stream: *mut c_void) -> lfm_status;
    pub fn lfm_attention_prefill(q_dev: *const f32, q_stride: u32, k_cache: *const c_void, v_cache: *const c_void,
                                 ctx: u32, start: u32, n: u32, out_dev: *mut f32, out_stride: u32,
                                 stream: *mut c_void) -> lfm_status;
    pub fn lfm_q6k_prompt_gemm(w_dev: *const c_void, in_dim: u32, rows: u32, x_dev: *const f32, n: u32,
                               y_dev: *mut f32, stream: *mut c_void) -> lfm_status;
    pub fn lfm_q6k_prompt_grouped(w_dev: *const c_void, in_dim: u32, rows: u32, n_expert: u32,
                                  expert_ids_dev: *const i32, x_dev: *const f32, x_div: u32, n: u32,
                                  y_dev: *mut f32, stream: *mut c_void) -> lfm_status;
    pub fn lfm_q6k_expand_f16(w_dev: *const c_void, in_dim: u32, rows: u32, out_dev: *mut c_void,
                              stream: *mut c_void) -> lfm_status;
    pub fn lfm_q6k_prompt_gemm_x16(w_dev: *const c_void, w16_dev: *const c_void, in_dim: u32, rows: u32,
                                   x_dev: *const f32, n: u32, y_dev: *mut f32, stream: *mut c_void) -> lfm_status;
    pub fn lfm_q6k_prompt_grouped_x16(w_dev: *const c_void, w16_dev: *const c_void, in_dim: u32, rows: u32,
                                      n_expert: u32, expert_ids_dev: *const i32, x_dev: *const f32, x_div: u32,
                                      n: u32, y_dev: *mut f32, stream: *mut c_void) -> lfm_status;
    pub fn lfm_selftest_wait_timeout(status: *mut u32, cycles: *mut u64) -> lfm_status;
    pub fn lfm_ops_error() -> *const c_char;
    // ---- streaming text of sessions decoded together (host only)
    pub fn lfm_text_create(piece_bytes: *const u8, piece_off: *const u64, n_tokens: u32, n_sessions: u32,
                           clean_spaces: c_int, replace_invalid: c_int, out: *mut *mut lfm_text) -> lfm_status;
    pub fn lfm_text_destroy(t: *mut lfm_text);
    pub fn lfm_text_push(t: *mut lfm_text, sessions: *const u32, tokens: *const u32, count: u32, out: *mut c_char,
                         cap: usize, out_off: *mut u64) -> lfm_status;
    pub fn lfm_text_finish(t: *mut lfm_text, session: u32, out: *mut c_char, cap: usize, len: *mut usize)
        -> lfm_status;
    pub fn lfm_text_reset(t: *mut lfm_text, session: u32) -> lfm_status;
    pub fn lfm_text_error() -> *const c_char;
}
