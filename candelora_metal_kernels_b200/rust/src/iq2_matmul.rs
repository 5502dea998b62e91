//! The IQ2 public functions of candelora-metal-kernels (its src/iq2_matmul.rs:535-670), same names
//! and signatures, on CUDA tensors: the body that dispatched Metal kernels (iq2_matmul_metal,
//! :197-365) is replaced by `Iq2MatmulOp`, a candle `CustomOp3` over (x, weight_bytes,
//! weight_scales) whose `cuda_fwd` calls the C ABI on candle's stream for the device. There is no
//! CPU path: `cpu_fwd` bails, like the reference without its `metal` feature (:507-520).
//!
//! Written against candle-core 0.9.2 (the reference's pin) with its `cuda` feature; this
//! repository's image has no Rust toolchain, so this file is not compiled here: the argument
//! lists of the FFI it calls are checked against the C header by tests/test_rust_binding.py.
use std::ffi::c_void;

use candle_core::backend::BackendStorage;
use candle_core::cuda_backend::cudarc::driver::DevicePtr;
use candle_core::cuda_backend::{CudaStorageSlice, WrapErr};
use candle_core::{bail, CpuStorage, CudaStorage, CustomOp3, DType, Layout, Result, Shape, Tensor};

use crate::activation_quant::{ActivationQuantConfig, ActivationQuantMode};
use crate::iq2_cuda_ffi as ffi;

/// Iq2MatmulVariant (reference src/iq2_matmul.rs:31-37).
#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub enum Iq2MatmulVariant {
    Iq2Xxs,
    Iq2Xs,
    Iq2S,
    Iq3S,
}

impl Iq2MatmulVariant {
    fn code(self) -> i32 {
        match self {
            Self::Iq2Xxs => 0,
            Self::Iq2Xs => 1,
            Self::Iq2S => 2,
            Self::Iq3S => 3,
        }
    }
}

fn check(rc: i32) -> Result<()> {
    if rc == ffi::IQ2_OK {
        Ok(())
    } else {
        Err(candle_core::Error::msg(ffi::last_error()))
    }
}

fn x_dtype_code(dtype: DType) -> Result<i32> {
    Ok(match dtype {
        DType::F32 => ffi::IQ2_DTYPE_F32,
        DType::F16 => ffi::IQ2_DTYPE_F16,
        DType::BF16 => ffi::IQ2_DTYPE_BF16,
        other => bail!("unsupported x dtype for iq2 matmul: {other:?}"),
    })
}

/// Device address of the first element of a contiguous storage view, and its length in elements.
fn device_view(s: &CudaStorage, l: &Layout) -> Result<(u64, usize)> {
    if !l.is_contiguous() {
        bail!("iq2_matmul expects contiguous layouts");
    }
    let stream = s.device.cuda_stream();
    let off = l.start_offset();
    let n = l.shape().elem_count();
    let (base, esz) = match &s.slice {
        CudaStorageSlice::U8(v) => (v.device_ptr(&stream).0, 1u64),
        CudaStorageSlice::F32(v) => (v.device_ptr(&stream).0, 4),
        CudaStorageSlice::F16(v) => (v.device_ptr(&stream).0, 2),
        CudaStorageSlice::BF16(v) => (v.device_ptr(&stream).0, 2),
        _ => bail!("iq2_matmul: unsupported storage dtype {:?}", s.dtype()),
    };
    Ok((base + off as u64 * esz, n))
}

/// The op form of the matmul (x, weight_bytes, weight_scales) -> f32 [m, out_dim].
struct Iq2MatmulOp {
    m: usize,
    out_dim: usize,
    in_dim: usize,
    variant: Iq2MatmulVariant,
    act_mode: i32,
    strict: bool,
}

impl CustomOp3 for Iq2MatmulOp {
    fn name(&self) -> &'static str {
        "candelora-iq2-matmul"
    }

    fn cpu_fwd(
        &self,
        _: &CpuStorage,
        _: &Layout,
        _: &CpuStorage,
        _: &Layout,
        _: &CpuStorage,
        _: &Layout,
    ) -> Result<(CpuStorage, Shape)> {
        bail!("iq2_matmul requires a CUDA device")
    }

    fn cuda_fwd(
        &self,
        x: &CudaStorage,
        xl: &Layout,
        wb: &CudaStorage,
        wbl: &Layout,
        ws: &CudaStorage,
        wsl: &Layout,
    ) -> Result<(CudaStorage, Shape)> {
        if wb.dtype() != DType::U8 || ws.dtype() != DType::U8 {
            bail!("iq2_matmul expects U8 weight bytes/scales, got bytes={:?}, scales={:?}", wb.dtype(), ws.dtype());
        }
        let dev = x.device.clone();
        let stream = dev.cuda_stream();
        let xd = x_dtype_code(x.dtype())?;
        let (xp, _) = device_view(x, xl)?;
        let (wbp, wbn) = device_view(wb, wbl)?;
        let (wsp, wsn) = device_view(ws, wsl)?;
        // the op owns its output (src/iq2_matmul.rs:261); every element is written by the kernel
        let out = unsafe { dev.alloc::<f32>(self.m * self.out_dim) }.w()?;
        let need = unsafe {
            ffi::iq2_matmul_with_activation_quant_workspace_size(
                self.m as u32,
                self.out_dim as u32,
                self.in_dim as u32,
                xd,
                self.variant.code(),
                self.act_mode,
            )
        };
        let workspace = unsafe { dev.alloc::<u8>(need.max(1)) }.w()?;
        let (op, _g0) = out.device_ptr(&stream);
        let (wp, _g1) = workspace.device_ptr(&stream);
        check(unsafe {
            ffi::iq2_matmul_with_activation_quant(
                xp as *const c_void,
                xd,
                self.m as u32,
                wbp as *const u8,
                wbn,
                wsp as *const u8,
                wsn,
                self.out_dim as u32,
                self.in_dim as u32,
                self.variant.code(),
                self.act_mode,
                self.strict as i32,
                op as *mut f32,
                wp as *mut c_void,
                need,
                stream.cu_stream() as *mut c_void,
            )
        })?;
        drop(workspace); // stream-ordered free, after the kernels that use it
        Ok((CudaStorage::wrap_cuda_slice(out, dev), Shape::from((self.m, self.out_dim))))
    }
}

/// parse_x_shape (reference src/iq2_matmul.rs:170-195): [K] -> ([1, K], squeeze) or [M, K].
fn parse_x_shape(x: &Tensor, in_dim: usize) -> Result<(Tensor, usize, bool)> {
    match x.dims() {
        [k] => {
            if *k != in_dim {
                bail!("iq2_matmul input mismatch: x dim={k} expected in_dim={in_dim}");
            }
            Ok((x.reshape((1, in_dim))?, 1, true))
        }
        [m, k] => {
            if *k != in_dim {
                bail!("iq2_matmul input mismatch: x last dim={k} expected in_dim={in_dim}");
            }
            Ok((x.clone(), *m, false))
        }
        dims => bail!("iq2_matmul expects x rank 1 or 2, got shape {dims:?}"),
    }
}

fn matmul_impl(
    x: &Tensor,
    weight_bytes: &Tensor,
    weight_scales: &Tensor,
    out_dim: usize,
    in_dim: usize,
    variant: Iq2MatmulVariant,
    act_mode: i32,
    strict: bool,
) -> Result<Tensor> {
    if out_dim == 0 || in_dim == 0 {
        bail!("iq2_matmul expects non-zero dimensions");
    }
    if !x.device().is_cuda() {
        bail!("iq2_matmul requires a CUDA device");
    }
    if !x.device().same_device(weight_bytes.device()) || !x.device().same_device(weight_scales.device()) {
        bail!("iq2_matmul device mismatch");
    }
    let (x2, m, squeeze) = parse_x_shape(x, in_dim)?;
    let x2 = x2.contiguous()?;
    let op = Iq2MatmulOp { m, out_dim, in_dim, variant, act_mode, strict };
    let out = x2.apply_op3_no_bwd(&weight_bytes.contiguous()?, &weight_scales.contiguous()?, &op)?;
    if squeeze {
        out.squeeze(0)
    } else {
        Ok(out)
    }
}

/// Reference src/iq2_matmul.rs:535-553.
pub fn iq2_matmul(
    x: &Tensor,
    weight_bytes: &Tensor,
    weight_scales: &Tensor,
    out_dim: usize,
    in_dim: usize,
    variant: Iq2MatmulVariant,
) -> Result<Tensor> {
    matmul_impl(x, weight_bytes, weight_scales, out_dim, in_dim, variant, ffi::IQ2_ACT_QUANT_OFF, false)
}

/// Reference src/iq2_matmul.rs:555-591: Off and non-strict W4A8 run the float path, strict W4A8
/// fails with the reference's message, W8A8 quantises every x row to int8 first.
pub fn iq2_matmul_with_activation_quant(
    x: &Tensor,
    weight_bytes: &Tensor,
    weight_scales: &Tensor,
    out_dim: usize,
    in_dim: usize,
    variant: Iq2MatmulVariant,
    activation_quant: &ActivationQuantConfig,
) -> Result<Tensor> {
    let mode = match activation_quant.mode {
        ActivationQuantMode::Off => ffi::IQ2_ACT_QUANT_OFF,
        ActivationQuantMode::W8A8 => ffi::IQ2_ACT_QUANT_W8A8,
        ActivationQuantMode::W4A8 => ffi::IQ2_ACT_QUANT_W4A8,
    };
    matmul_impl(x, weight_bytes, weight_scales, out_dim, in_dim, variant, mode, activation_quant.strict)
}

/// Reference src/iq2_matmul.rs:593-602: dense f16 [out_dim, in_dim], bit-identical to the
/// reference's iq2_xxs_dequantize_f16 kernel.
pub fn iq2_dequantize_to_f16(
    weight_bytes: &Tensor,
    weight_scales: &Tensor,
    out_dim: usize,
    in_dim: usize,
    variant: Iq2MatmulVariant,
) -> Result<Tensor> {
    struct DequantOp {
        out_dim: usize,
        in_dim: usize,
        variant: Iq2MatmulVariant,
    }
    impl candle_core::CustomOp2 for DequantOp {
        fn name(&self) -> &'static str {
            "candelora-iq2-dequantize-f16"
        }
        fn cpu_fwd(&self, _: &CpuStorage, _: &Layout, _: &CpuStorage, _: &Layout) -> Result<(CpuStorage, Shape)> {
            bail!("iq2_dequantize_to_f16 requires a CUDA device")
        }
        fn cuda_fwd(&self, wb: &CudaStorage, wbl: &Layout, ws: &CudaStorage, wsl: &Layout) -> Result<(CudaStorage, Shape)> {
            let dev = wb.device.clone();
            let stream = dev.cuda_stream();
            let (wbp, wbn) = device_view(wb, wbl)?;
            let (wsp, wsn) = device_view(ws, wsl)?;
            let out = unsafe { dev.alloc::<half::f16>(self.out_dim * self.in_dim) }.w()?;
            let (op, _g) = out.device_ptr(&stream);
            check(unsafe {
                ffi::iq2_dequantize(
                    wbp as *const u8,
                    wbn,
                    wsp as *const u8,
                    wsn,
                    self.out_dim as u32,
                    self.in_dim as u32,
                    self.variant.code(),
                    op as *mut c_void,
                    ffi::IQ2_DTYPE_F16,
                    stream.cu_stream() as *mut c_void,
                )
            })?;
            Ok((CudaStorage::wrap_cuda_slice(out, dev), Shape::from((self.out_dim, self.in_dim))))
        }
    }
    if out_dim == 0 || in_dim == 0 {
        bail!("iq2_dequantize_to_f16 expects non-zero dimensions");
    }
    weight_bytes.contiguous()?.apply_op2_no_bwd(&weight_scales.contiguous()?, &DequantOp { out_dim, in_dim, variant })
}

/// Reference src/iq2_matmul.rs:604-619.
pub fn iq2_xxs_matmul(x: &Tensor, weight_bytes: &Tensor, weight_scales: &Tensor, out_dim: usize, in_dim: usize) -> Result<Tensor> {
    iq2_matmul(x, weight_bytes, weight_scales, out_dim, in_dim, Iq2MatmulVariant::Iq2Xxs)
}

/// Reference src/iq2_matmul.rs:621-636.
pub fn iq2_xs_matmul(x: &Tensor, weight_bytes: &Tensor, weight_scales: &Tensor, out_dim: usize, in_dim: usize) -> Result<Tensor> {
    iq2_matmul(x, weight_bytes, weight_scales, out_dim, in_dim, Iq2MatmulVariant::Iq2Xs)
}

/// Reference src/iq2_matmul.rs:638-653.
pub fn iq2_s_matmul(x: &Tensor, weight_bytes: &Tensor, weight_scales: &Tensor, out_dim: usize, in_dim: usize) -> Result<Tensor> {
    iq2_matmul(x, weight_bytes, weight_scales, out_dim, in_dim, Iq2MatmulVariant::Iq2S)
}

/// Reference src/iq2_matmul.rs:655-670.
pub fn iq3_s_matmul(x: &Tensor, weight_bytes: &Tensor, weight_scales: &Tensor, out_dim: usize, in_dim: usize) -> Result<Tensor> {
    iq2_matmul(x, weight_bytes, weight_scales, out_dim, in_dim, Iq2MatmulVariant::Iq3S)
}
