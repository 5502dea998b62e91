//! candelora-iq2-cuda: the IQ2 matmul of candelora-metal-kernels on B200 (sm_100a) GPUs, as a
//! Rust/candle library with the reference crate's public IQ2 API (`iq2_matmul`,
//! `iq2_matmul_with_activation_quant`, `iq2_dequantize_to_f16`, `iq2_xxs_matmul`, ...). The
//! kernels are this repository's CUDA sources, compiled by build.rs; `iq2_cuda_ffi` is their C ABI.
pub mod activation_quant;
pub mod iq2_cuda_ffi;
pub mod iq2_matmul;

pub use activation_quant::{ActivationQuantConfig, ActivationQuantMode};
pub use iq2_matmul::{
    iq2_dequantize_to_f16, iq2_matmul, iq2_matmul_with_activation_quant, iq2_s_matmul, iq2_xs_matmul,
    iq2_xxs_matmul, iq3_s_matmul, Iq2MatmulVariant,
};
