//! The CUDA side of `ffai-mercury`'s `asr/flash_attn.rs`: candle custom ops
//! named like the reference's ("flash-attn", "flash-attn-merged") whose
//! `cuda_fwd` calls this library, and the CUDA branches of the three
//! functions the Whisper engines call (`serves`, `attend`, `attend_merged`,
//! flash_attn.rs:104, :218, :135).  `patches/flash_attn_cuda.patch` adds one
//! early branch to each of those functions that hands CUDA tensors here; CPU
//! tensors keep the reference's AVX2 path unchanged.
//!
//! Semantics follow the reference: `Ok(None)` where it declines (decided by
//! `ffai_flash_check` before the op is applied, the same rules the library
//! applies when it runs), q pre-scaled f32, K given as K^T, f32 output.  At
//! the encoder shape the f32 operands are rounded to bf16 on the device
//! (`ffai_flash_attend` in `include/ffai_attn.h` states the error);
//! `FFAI_ATTN_CHECKED_F32=1` selects the f32 kernel.

use std::ffi::c_void;

use candle_core::backend::BackendStorage;
use candle_core::cuda_backend::cudarc::driver::DevicePtr;
use candle_core::{
    CpuStorage, CudaStorage, CustomOp3, DType, Device, Layout, Result, Shape, Tensor, bail,
};

use crate::{
    FFAI_ATTN_DECLINED, FFAI_ATTN_OK, FFAI_DT_BF16, FFAI_DT_F16, FFAI_DT_F32, ffai_flash_attend,
    ffai_flash_attend_merged, ffai_flash_check, ffai_flash_serves, ffai_tensor4, last_error,
};

fn dtype_code(dt: DType) -> Option<i32> {
    match dt {
        DType::F32 => Some(FFAI_DT_F32),
        DType::BF16 => Some(FFAI_DT_BF16),
        DType::F16 => Some(FFAI_DT_F16),
        _ => None,
    }
}

fn ordinal(dev: &Device) -> Option<i32> {
    match dev {
        Device::Cuda(d) => i32::try_from(d.ordinal()).ok(),
        _ => None,
    }
}

/// A tensor's shape and type for the library's gate (no data pointer: the
/// gate reads dims, dtype and device only).
fn shape_of(t: &Tensor) -> Option<ffai_tensor4> {
    let (a, b, c, d) = t.dims4().ok()?;
    let dims = [a, b, c, d].map(|x| i64::try_from(x).unwrap_or(i64::MAX));
    Some(ffai_tensor4 {
        data: std::ptr::null_mut(),
        dims,
        dtype: dtype_code(t.dtype())?,
        device: ordinal(t.device())?,
    })
}

/// The CUDA branch of `flash_attn::serves`: whether the decode kernel will
/// read this K^T / V pair, so the engine picks the cache dtype it serves.
#[must_use]
pub fn serves(kt: &Tensor, v: &Tensor) -> bool {
    match (shape_of(kt), shape_of(v)) {
        // SAFETY: both descriptors are valid for the call.
        (Some(a), Some(b)) => unsafe { ffai_flash_serves(&raw const a, &raw const b) } == 1,
        _ => false,
    }
}

fn gate(q: &Tensor, kt: &Tensor, v: &Tensor, masked: bool, merged: bool) -> Result<bool> {
    let (Some(a), Some(b), Some(c)) = (shape_of(q), shape_of(kt), shape_of(v)) else {
        return Ok(false);
    };
    if !q.is_contiguous() || !kt.is_contiguous() || !v.is_contiguous() {
        return Ok(false);
    }
    // SAFETY: the three descriptors are valid for the call.
    let st = unsafe {
        ffai_flash_check(&raw const a, &raw const b, &raw const c, i32::from(masked),
                         i32::from(merged))
    };
    match st {
        FFAI_ATTN_OK => Ok(true),
        FFAI_ATTN_DECLINED => Ok(false),
        _ => bail!("flash-attn (cuda): {}", last_error(std::ptr::null())),
    }
}

/// The CUDA branch of `flash_attn::attend`: `Ok(None)` where the reference
/// declines, else the (1, heads, qlen, 64) f32 output.
pub fn attend(q: &Tensor, kt: &Tensor, v: &Tensor, masked: bool) -> Result<Option<Tensor>> {
    if !gate(q, kt, v, masked, false)? {
        return Ok(None);
    }
    Ok(Some(q.apply_op3(kt, v, CudaFlashAttnOp)?))
}

/// The CUDA branch of `flash_attn::attend_merged`: (1, seq, heads*64) f32.
pub fn attend_merged(q: &Tensor, kt: &Tensor, v: &Tensor) -> Result<Option<Tensor>> {
    if !gate(q, kt, v, false, true)? {
        return Ok(None);
    }
    Ok(Some(q.apply_op3(kt, v, CudaMergedAttnOp)?))
}

/// Device address of a contiguous operand's first element.
fn operand(s: &CudaStorage, l: &Layout) -> Result<(*mut c_void, i32)> {
    if !l.is_contiguous() {
        bail!("flash-attn (cuda): contiguous operands only")
    }
    let stream = s.device().cuda_stream();
    let (ptr, dt, elt) = match s.dtype() {
        DType::F32 => {
            let (p, _sync) = s.as_cuda_slice::<f32>()?.device_ptr(&stream);
            (p, FFAI_DT_F32, 4)
        }
        DType::BF16 => {
            let (p, _sync) = s.as_cuda_slice::<half::bf16>()?.device_ptr(&stream);
            (p, FFAI_DT_BF16, 2)
        }
        DType::F16 => {
            let (p, _sync) = s.as_cuda_slice::<half::f16>()?.device_ptr(&stream);
            (p, FFAI_DT_F16, 2)
        }
        dt => bail!("flash-attn (cuda): unsupported dtype {dt:?}"),
    };
    let addr = ptr + (l.start_offset() * elt) as u64;
    Ok((addr as usize as *mut c_void, dt))
}

fn tensor4(ptr: *mut c_void, dims: &[usize], dtype: i32, device: i32) -> Result<ffai_tensor4> {
    let &[a, b, c, d] = dims else { bail!("flash-attn (cuda): 4-d operands only") };
    let dims = [a, b, c, d].map(|x| i64::try_from(x).unwrap_or(i64::MAX));
    Ok(ffai_tensor4 { data: ptr, dims, dtype, device })
}

/// Runs one served call on the operands' device and stream.
fn run(s1: &CudaStorage, l1: &Layout, s2: &CudaStorage, l2: &Layout, s3: &CudaStorage,
       l3: &Layout, merged: bool) -> Result<(CudaStorage, Shape)> {
    let dev = s1.device().clone();
    let ord = i32::try_from(dev.ordinal()).map_err(candle_core::Error::wrap)?;
    let (qp, qdt) = operand(s1, l1)?;
    let (kp, kdt) = operand(s2, l2)?;
    let (vp, vdt) = operand(s3, l3)?;
    let (_, heads, qlen, hd) = l1.shape().dims4()?;
    // The merged output (1, seq, heads * 64) is 3-d: its fourth extent is 0.
    let out_dims = if merged { [1, qlen, heads * hd, 0] } else { [1, heads, qlen, hd] };
    let out = dev.alloc_zeros::<f32>(heads * qlen * hd)?;
    let stream = dev.cuda_stream();
    let (op, _sync) = out.device_ptr(&stream);
    let tq = tensor4(qp, l1.shape().dims(), qdt, ord)?;
    let tk = tensor4(kp, l2.shape().dims(), kdt, ord)?;
    let tv = tensor4(vp, l3.shape().dims(), vdt, ord)?;
    let mut to = tensor4(op as usize as *mut c_void, &out_dims, FFAI_DT_F32, ord)?;
    let ctx = crate::ctx(dev.ordinal()).map_err(candle_core::Error::msg)?;
    let guard = ctx.lock().map_err(|e| candle_core::Error::msg(e.to_string()))?;
    let cu_stream = stream.cu_stream() as *mut c_void;
    // SAFETY: every pointer addresses a live device buffer of the shape its
    // descriptor states, on the context's device; the mutex serialises calls.
    let st = unsafe {
        if merged {
            ffai_flash_attend_merged(guard.0, &raw const tq, &raw const tk, &raw const tv,
                                     &raw mut to, cu_stream)
        } else {
            ffai_flash_attend(guard.0, &raw const tq, &raw const tk, &raw const tv, 0,
                              &raw mut to, cu_stream)
        }
    };
    if st != FFAI_ATTN_OK {
        bail!("flash-attn (cuda): status {st}: {}", last_error(guard.0))
    }
    drop(guard);
    let shape = if merged {
        Shape::from_dims(&[1, qlen, heads * hd])
    } else {
        Shape::from_dims(&[1, heads, qlen, hd])
    };
    Ok((CudaStorage::wrap_cuda_slice(out, dev), shape))
}

/// "flash-attn" on CUDA tensors.
pub struct CudaFlashAttnOp;

impl CustomOp3 for CudaFlashAttnOp {
    fn name(&self) -> &'static str {
        "flash-attn"
    }

    fn cpu_fwd(&self, _: &CpuStorage, _: &Layout, _: &CpuStorage, _: &Layout, _: &CpuStorage,
               _: &Layout) -> Result<(CpuStorage, Shape)> {
        bail!("flash-attn (cuda): CPU tensors take flash_attn.rs's own op")
    }

    fn cuda_fwd(&self, s1: &CudaStorage, l1: &Layout, s2: &CudaStorage, l2: &Layout,
                s3: &CudaStorage, l3: &Layout) -> Result<(CudaStorage, Shape)> {
        run(s1, l1, s2, l2, s3, l3, false)
    }
}

/// "flash-attn-merged" on CUDA tensors.
pub struct CudaMergedAttnOp;

impl CustomOp3 for CudaMergedAttnOp {
    fn name(&self) -> &'static str {
        "flash-attn-merged"
    }

    fn cpu_fwd(&self, _: &CpuStorage, _: &Layout, _: &CpuStorage, _: &Layout, _: &CpuStorage,
               _: &Layout) -> Result<(CpuStorage, Shape)> {
        bail!("flash-attn-merged (cuda): CPU tensors take flash_attn.rs's own op")
    }

    fn cuda_fwd(&self, s1: &CudaStorage, l1: &Layout, s2: &CudaStorage, l2: &Layout,
                s3: &CudaStorage, l3: &Layout) -> Result<(CudaStorage, Shape)> {
        run(s1, l1, s2, l2, s3, l3, true)
    }
}
