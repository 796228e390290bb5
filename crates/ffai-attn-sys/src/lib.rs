//! Raw bindings to `libffai_attn`, the B200 (sm_100a) attention library that
//! takes over the fused attention of `ffai-mercury` (`asr/flash_attn.rs`)
//! when its tensors live on a CUDA device, plus the projections and GEMVs
//! around it.  Every declaration mirrors `include/ffai_attn.h` one for one
//! (names, argument order, `#[repr(C)]` field order); a CPU test of the
//! repository parses both files and compares them.
//!
//! Statuses: [`FFAI_ATTN_OK`] served; [`FFAI_ATTN_DECLINED`] not a shape the
//! library serves (the reference's `Ok(None)`: take the fallback path);
//! negative values are errors, described by [`ffai_attn_last_error`].
//!
//! Threading: one context per device; calls on one context must not overlap
//! on the GPU.  [`ctx`] hands out one mutex-guarded context per device, the
//! contract the reference's engine already keeps behind its own mutex.

#![allow(non_camel_case_types)]

use std::ffi::{c_char, c_int, c_void};

pub const FFAI_ATTN_ABI_VERSION: c_int = 1;

pub const FFAI_ATTN_OK: c_int = 0;
pub const FFAI_ATTN_DECLINED: c_int = 1;
pub const FFAI_ATTN_ERR_INVALID: c_int = -1;
pub const FFAI_ATTN_ERR_CUDA: c_int = -2;
pub const FFAI_ATTN_ERR_TIMEOUT: c_int = -3;
pub const FFAI_ATTN_ERR_NOMEM: c_int = -4;
pub const FFAI_ATTN_ERR_NO_DEVICE: c_int = -5;

pub const FFAI_DT_F32: i32 = 0;
pub const FFAI_DT_BF16: i32 = 1;
pub const FFAI_DT_F16: i32 = 2;

pub const FFAI_LAYOUT_HEADS_SPLIT: i32 = 0;
pub const FFAI_LAYOUT_TOKEN_MAJOR: i32 = 1;
pub const FFAI_LAYOUT_KT: i32 = 2;

pub const FFAI_ATTN_FLAG_CHECKED_F32: u32 = 0x1;
pub const FFAI_ATTN_FLAG_KV_STABLE: u32 = 0x2;
pub const FFAI_ATTN_FLAG_KV_APPEND_ONLY: u32 = 0x4;
pub const FFAI_ATTN_FLAG_INPUTS_STABLE: u32 = 0x8;

pub const FFAI_OP_PREFILL: c_int = 0;
pub const FFAI_OP_DECODE: c_int = 1;
pub const FFAI_OP_VARLEN: c_int = 2;

pub const FFAI_PAGE_KEYS: i32 = 64;
pub const FFAI_INT8_FLAG_WEIGHTS_STABLE: u32 = 0x2;
pub const FFAI_GEMV_FLAG_WEIGHTS_STABLE: u32 = 0x2;
pub const FFAI_GEMM_ACT_NONE: i32 = 0;
pub const FFAI_GEMM_ACT_FAST_GELU: i32 = 1;

/// `ffai_attn_desc`: the shape, types and layouts of one attention call.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct ffai_attn_desc {
    pub batch: i32,
    pub heads: i32,
    pub q_len: i32,
    pub kv_len: i32,
    pub head_dim: i32,
    pub kv_capacity: i32,
    pub q_dtype: i32,
    pub kv_dtype: i32,
    pub out_dtype: i32,
    pub q_layout: i32,
    pub k_layout: i32,
    pub v_layout: i32,
    pub out_layout: i32,
    pub causal: i32,
    pub q_offset: i32,
    pub scale: f32,
    pub flags: u32,
    pub token_stride: i32,
}

impl ffai_attn_desc {
    /// The library's defaults (`ffai_attn_desc_init`).
    #[must_use]
    pub fn new() -> Self {
        let mut d = Self::default();
        // SAFETY: `d` is a valid, writable descriptor.
        unsafe { ffai_attn_desc_init(&raw mut d) };
        d
    }
}

/// `ffai_tensor4`: a contiguous 4-d tensor as candle presents it.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct ffai_tensor4 {
    pub data: *mut c_void,
    pub dims: [i64; 4],
    pub dtype: i32,
    pub device: i32,
}

/// Opaque per-device context.
#[repr(C)]
pub struct ffai_attn_ctx {
    _private: [u8; 0],
}

unsafe extern "C" {
    pub fn ffai_attn_version() -> *const c_char;
    pub fn ffai_attn_desc_init(d: *mut ffai_attn_desc);
    pub fn ffai_attn_check(d: *const ffai_attn_desc, op: c_int) -> c_int;
    pub fn ffai_attn_create(device: c_int, status: *mut c_int) -> *mut ffai_attn_ctx;
    pub fn ffai_attn_destroy(ctx: *mut ffai_attn_ctx);
    pub fn ffai_attn_prefill(ctx: *mut ffai_attn_ctx, d: *const ffai_attn_desc, q: *const c_void,
                             k: *const c_void, v: *const c_void, o: *mut c_void, lse: *mut f32,
                             stream: *mut c_void) -> c_int;
    pub fn ffai_attn_decode(ctx: *mut ffai_attn_ctx, d: *const ffai_attn_desc, q: *const c_void,
                            k: *const c_void, v: *const c_void, o: *mut c_void, lse: *mut f32,
                            num_splits: i32, stream: *mut c_void) -> c_int;
    pub fn ffai_attn_decode_prefetch(ctx: *mut ffai_attn_ctx, d: *const ffai_attn_desc,
                                     q: *const c_void, k: *const c_void, v: *const c_void,
                                     next_k: *const c_void, next_v: *const c_void,
                                     o: *mut c_void, lse: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ffai_attn_decode_static(d: *const ffai_attn_desc, q: *const c_void, k: *const c_void,
                                   v: *const c_void, o: *mut c_void, lse: *mut f32,
                                   num_splits: i32, stream: *mut c_void) -> c_int;
    pub fn ffai_attn_decode_paged(ctx: *mut ffai_attn_ctx, d: *const ffai_attn_desc,
                                  q: *const c_void, k_pool: *const c_void,
                                  v_pool: *const c_void, num_pages: i32,
                                  block_table: *const i32, seq_lens: *const i32, max_pages: i32,
                                  o: *mut c_void, lse: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ffai_kv_append(ctx: *mut ffai_attn_ctx, d: *const ffai_attn_desc, k_pool: *mut c_void,
                          v_pool: *mut c_void, num_pages: i32, block_table: *const i32,
                          seq_lens: *mut i32, max_pages: i32, k_new: *const c_void,
                          v_new: *const c_void, stream: *mut c_void) -> c_int;
    pub fn ffai_kv_copy_pages(ctx: *mut ffai_attn_ctx, d: *const ffai_attn_desc,
                              k_pool: *mut c_void, v_pool: *mut c_void, num_pages: i32,
                              src: *const i32, dst: *const i32, n: i32,
                              stream: *mut c_void) -> c_int;
    pub fn ffai_int8_gemv_layout(rows: i32, cols: i32, blk: i32, packed_bytes: *mut i64,
                                 corr_count: *mut i64) -> c_int;
    pub fn ffai_int8_gemv_quantize(ctx: *mut ffai_attn_ctx, w: *const c_void, w_dtype: i32,
                                   rows: i32, cols: i32, blk: i32, packed: *mut c_void,
                                   corr: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ffai_int8_gemv(ctx: *mut ffai_attn_ctx, x: *const f32, batch: i32,
                          packed: *const c_void, corr: *const f32, rows: i32, cols: i32,
                          blk: i32, out: *mut f32, flags: u32, stream: *mut c_void) -> c_int;
    pub fn ffai_f16_gemv_layout(rows: i32, cols: i32, packed_bytes: *mut i64) -> c_int;
    pub fn ffai_f16_gemv_pack(ctx: *mut ffai_attn_ctx, w: *const c_void, w_dtype: i32,
                              rows: i32, cols: i32, packed: *mut c_void,
                              stream: *mut c_void) -> c_int;
    pub fn ffai_f16_gemv(ctx: *mut ffai_attn_ctx, x: *const f32, batch: i32,
                         packed: *const c_void, bias: *const f32, rows: i32, cols: i32,
                         out: *mut f32, flags: u32, stream: *mut c_void) -> c_int;
    pub fn ffai_gemm_bf16(ctx: *mut ffai_attn_ctx, a: *const c_void, lda: i64, b: *const c_void,
                          ldb: i64, bias: *const f32, residual: *const c_void, ldr: i64,
                          out: *mut c_void, ldo: i64, m: i32, n: i32, k: i32, out_dtype: i32,
                          act: i32, stream: *mut c_void) -> c_int;
    pub fn ffai_attn_varlen(ctx: *mut ffai_attn_ctx, d: *const ffai_attn_desc,
                            cu_seqlens_q: *const i32, cu_seqlens_k: *const i32, n_seg: i32,
                            q: *const c_void, k: *const c_void, v: *const c_void,
                            o: *mut c_void, lse: *mut f32, stream: *mut c_void) -> c_int;
    pub fn ffai_attn_prefill_host(ctx: *mut ffai_attn_ctx, d: *const ffai_attn_desc,
                                  q: *const c_void, k: *const c_void, v: *const c_void,
                                  o: *mut c_void, lse: *mut f32) -> c_int;
    pub fn ffai_attn_multi_prefill_host(ctxs: *const *mut ffai_attn_ctx, n_ctx: i32,
                                        d: *const ffai_attn_desc, q: *const c_void,
                                        k: *const c_void, v: *const c_void, o: *mut c_void,
                                        lse: *mut f32, chunk_segments: i32,
                                        failed_workers: *mut i32) -> c_int;
    pub fn ffai_attn_chunk_queue_selftest(n_workers: i32, n_chunks: i32, fail_mask: u32,
                                          owner: *mut i32, failed_workers: *mut i32) -> c_int;
    pub fn ffai_attn_profile(ctx: *mut ffai_attn_ctx, enable: i32, ms: *mut f64,
                             launches: *mut i64) -> c_int;
    pub fn ffai_attn_sync(ctx: *mut ffai_attn_ctx, stream: *mut c_void) -> c_int;
    pub fn ffai_attn_last_error(ctx: *const ffai_attn_ctx, buf: *mut c_char, n: usize) -> c_int;
    pub fn ffai_flash_serves(kt: *const ffai_tensor4, v: *const ffai_tensor4) -> c_int;
    pub fn ffai_flash_attend(ctx: *mut ffai_attn_ctx, q: *const ffai_tensor4,
                             kt: *const ffai_tensor4, v: *const ffai_tensor4, masked: i32,
                             out: *mut ffai_tensor4, stream: *mut c_void) -> c_int;
    pub fn ffai_flash_attend_merged(ctx: *mut ffai_attn_ctx, q: *const ffai_tensor4,
                                    kt: *const ffai_tensor4, v: *const ffai_tensor4,
                                    out: *mut ffai_tensor4, stream: *mut c_void) -> c_int;
    pub fn ffai_flash_check(q: *const ffai_tensor4, kt: *const ffai_tensor4,
                            v: *const ffai_tensor4, masked: i32, merged: i32) -> c_int;
}

/// The message of the last error or decline of `ctx` (null: this thread's).
#[must_use]
pub fn last_error(ctx: *const ffai_attn_ctx) -> String {
    let mut buf = [0 as c_char; 512];
    // SAFETY: `buf` is writable for its length; the library NUL-terminates.
    unsafe { ffai_attn_last_error(ctx, buf.as_mut_ptr(), buf.len()) };
    // SAFETY: NUL-terminated within `buf`.
    unsafe { std::ffi::CStr::from_ptr(buf.as_ptr()) }.to_string_lossy().into_owned()
}

/// A device's context.  The raw pointer is only used under the mutex that
/// [`ctx`] wraps it in, which is what makes sharing it across threads sound.
pub struct Ctx(pub *mut ffai_attn_ctx);

// SAFETY: the library's contexts may be used from any thread as long as calls
// on one context do not overlap; `ctx` serialises them with a mutex.
unsafe impl Send for Ctx {}

/// Upper bound on device ordinals served (contexts are created lazily).
pub const MAX_DEVICES: usize = 64;

/// The context of CUDA device `device`, created on first use.  Errors
/// (no such device, no GPU) come back as the library's message.
pub fn ctx(device: usize) -> Result<&'static std::sync::Mutex<Ctx>, String> {
    use std::sync::{Mutex, OnceLock};
    static CTXS: OnceLock<Vec<OnceLock<Mutex<Ctx>>>> = OnceLock::new();
    let slots = CTXS.get_or_init(|| (0..MAX_DEVICES).map(|_| OnceLock::new()).collect());
    let slot = slots.get(device).ok_or_else(|| format!("device {device} out of range"))?;
    if let Some(m) = slot.get() {
        return Ok(m);
    }
    let mut st: c_int = 0;
    let dev = c_int::try_from(device).map_err(|e| e.to_string())?;
    // SAFETY: `st` is writable; a null return carries its status in `st`.
    let p = unsafe { ffai_attn_create(dev, &raw mut st) };
    if p.is_null() {
        return Err(format!("ffai_attn_create({device}): status {st}: {}",
                           last_error(std::ptr::null())));
    }
    if slot.set(Mutex::new(Ctx(p))).is_err() {
        // Another thread created this device's context first: keep theirs.
        // SAFETY: `p` came from ffai_attn_create and is used nowhere else.
        unsafe { ffai_attn_destroy(p) };
    }
    Ok(slot.get().expect("set above"))
}

#[cfg(feature = "candle")]
pub mod candle_ops;
