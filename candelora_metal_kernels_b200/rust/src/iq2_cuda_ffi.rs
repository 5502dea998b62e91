//! The C ABI of libcandelora_iq2 (include/candelora_iq2.h and include/candelora_iq2_testing.h),
//! declared for Rust. Every declaration has the header's argument order and types
//! (tests/test_rust_binding.py compares the two); `*mut c_void` stands for `iq2_stream_t` (a
//! `cudaStream_t`) and for `iq2_comm_t`.
#![allow(dead_code)]

use std::ffi::{c_char, c_int, c_void};

pub const IQ2_OK: c_int = 0;
pub const IQ2_ERR_INVALID_ARGUMENT: c_int = 1;
pub const IQ2_ERR_ZERO_DIM: c_int = 2;
pub const IQ2_ERR_DEVICE: c_int = 3;
pub const IQ2_ERR_DTYPE: c_int = 4;
pub const IQ2_ERR_OVERFLOW: c_int = 5;
pub const IQ2_ERR_TOO_SMALL: c_int = 6;
pub const IQ2_ERR_UNSUPPORTED: c_int = 7;
pub const IQ2_ERR_WORKSPACE: c_int = 8;
pub const IQ2_ERR_CUDA: c_int = 9;
pub const IQ2_ERR_COMM: c_int = 10;
pub const IQ2_ERR_TIMEOUT: c_int = 11;

pub const IQ2_DTYPE_F32: c_int = 0;
pub const IQ2_DTYPE_F16: c_int = 1;
pub const IQ2_DTYPE_BF16: c_int = 2;

pub const IQ2_ACT_QUANT_OFF: c_int = 0;
pub const IQ2_ACT_QUANT_W8A8: c_int = 1;
pub const IQ2_ACT_QUANT_W4A8: c_int = 2;

pub const IQ2_COMM_ID_BYTES: usize = 128;
pub const IQ2_NOALLOC_SCRATCH_BYTES: usize = 8 * 1024 * 1024;

/// struct iq2_matmul_problem (one projection of a grouped call).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct Iq2MatmulProblem {
    pub x: *const c_void,
    pub weight_bytes: *const u8,
    pub weight_bytes_len: usize,
    pub weight_scales: *const u8,
    pub weight_scales_len: usize,
    pub out_dim: u32,
    pub in_dim: u32,
    pub out: *mut f32,
}

#[link(name = "candelora_iq2", kind = "static")]
extern "C" {
    pub fn iq2_last_error() -> *const c_char;
    pub fn iq2_abi_version() -> c_int;
    pub fn iq2_device_check() -> c_int;
    pub fn iq2_matmul_workspace_size(m: u32, out_dim: u32, in_dim: u32, x_dtype: c_int, variant: c_int) -> usize;
    pub fn iq2_matmul(
        x: *const c_void,
        x_dtype: c_int,
        m: u32,
        weight_bytes: *const u8,
        weight_bytes_len: usize,
        weight_scales: *const u8,
        weight_scales_len: usize,
        out_dim: u32,
        in_dim: u32,
        variant: c_int,
        out: *mut f32,
        workspace: *mut c_void,
        workspace_bytes: usize,
        stream: *mut c_void,
    ) -> c_int;
    pub fn iq2_matmul_with_activation_quant(
        x: *const c_void,
        x_dtype: c_int,
        m: u32,
        weight_bytes: *const u8,
        weight_bytes_len: usize,
        weight_scales: *const u8,
        weight_scales_len: usize,
        out_dim: u32,
        in_dim: u32,
        variant: c_int,
        act_mode: c_int,
        strict: c_int,
        out: *mut f32,
        workspace: *mut c_void,
        workspace_bytes: usize,
        stream: *mut c_void,
    ) -> c_int;
    pub fn iq2_matmul_with_activation_quant_workspace_size(
        m: u32,
        out_dim: u32,
        in_dim: u32,
        x_dtype: c_int,
        variant: c_int,
        act_mode: c_int,
    ) -> usize;
    pub fn iq2_matmul_grouped_workspace_size(
        problems: *const Iq2MatmulProblem,
        count: u32,
        m: u32,
        x_dtype: c_int,
    ) -> usize;
    pub fn iq2_matmul_grouped(
        problems: *const Iq2MatmulProblem,
        count: u32,
        m: u32,
        x_dtype: c_int,
        workspace: *mut c_void,
        workspace_bytes: usize,
        stream: *mut c_void,
    ) -> c_int;
    pub fn iq2_matmul_noalloc(
        x: *const c_void,
        x_dtype: c_int,
        m: u32,
        weight_bytes: *const u8,
        weight_bytes_len: usize,
        weight_scales: *const u8,
        weight_scales_len: usize,
        out_dim: u32,
        in_dim: u32,
        out: *mut f32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn iq2_dequantize(
        weight_bytes: *const u8,
        weight_bytes_len: usize,
        weight_scales: *const u8,
        weight_scales_len: usize,
        out_dim: u32,
        in_dim: u32,
        variant: c_int,
        out: *mut c_void,
        out_dtype: c_int,
        stream: *mut c_void,
    ) -> c_int;
    pub fn iq2_gather_columns(
        gathered: *const f32,
        shards: u32,
        m: u32,
        shard_cols: u32,
        out: *mut f32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn iq2_split_interleaved(
        blocks: *const u8,
        blocks_len: usize,
        nblocks: u64,
        variant: c_int,
        weight_bytes: *mut u8,
        weight_scales: *mut u8,
        stream: *mut c_void,
    ) -> c_int;
    pub fn iq2_comm_unique_id(id: *mut u8) -> c_int;
    pub fn iq2_comm_init_with_timeout(
        id: *const u8,
        world: c_int,
        rank: c_int,
        timeout_ms: u32,
        comm: *mut *mut c_void,
    ) -> c_int;
    pub fn iq2_comm_init(id: *const u8, world: c_int, rank: c_int, comm: *mut *mut c_void) -> c_int;
    pub fn iq2_comm_destroy(comm: *mut c_void) -> c_int;
    pub fn iq2_comm_symmetric_alloc(comm: *mut c_void, bytes: usize, ptr: *mut *mut c_void) -> c_int;
    pub fn iq2_comm_check(comm: *mut c_void) -> c_int;
    pub fn iq2_matmul_grouped_sharded_workspace_size(
        problems: *const Iq2MatmulProblem,
        count: u32,
        m: u32,
        x_dtype: c_int,
        world: c_int,
    ) -> usize;
    pub fn iq2_matmul_grouped_sharded(
        comm: *mut c_void,
        problems: *const Iq2MatmulProblem,
        count: u32,
        m: u32,
        x_dtype: c_int,
        workspace: *mut c_void,
        workspace_bytes: usize,
        stream: *mut c_void,
    ) -> c_int;
    pub fn iq2_testing_set_gemm_stall(wait_limit_ns: u64, stall_stage: u32) -> c_int;
}

/// The calling thread's message for the last failed call.
pub fn last_error() -> String {
    // SAFETY: the library returns a NUL-terminated thread-local string, valid until the next call.
    unsafe { std::ffi::CStr::from_ptr(iq2_last_error()) }.to_string_lossy().into_owned()
}
