//! `vmlm-ops-cuda`: the GEMM operators of `vmlm_ops::kernels` on a B200.
//!
//! The functions in [`kernels`] keep the signatures of the reference
//! operators (ops/src/kernels.rs:1200-1204 `gemm_nt_bf16`, :1256-1261
//! `gemm_nt_int8`, :987-995 `gemm_nt`, :407-415 `gemm`), so the VM's OP_GEMM
//! arm (core/src/interp.rs:764, 801, 808, 810) calls them unchanged once the
//! re-export in core/src/kernels.rs:1-3 points here. They call the C ABI of
//! libvmlm_cuda.so; a non-zero status is reported the way the VM reports
//! misuse: the message is printed and the process exits with code 9
//! (core/src/interp.rs:752-806).
#![no_std]
#![allow(clippy::missing_safety_doc)]

use core::ffi::{c_char, c_int, c_uint, c_void};

/// The C ABI (include/vmlm_cuda.h), the entry points a VM build needs.
pub mod ffi {
    use super::*;

    /// A VM slot as OP_GEMM reads it: row-major [rows, cols] of `dtype`.
    #[repr(C)]
    pub struct vmlm_slot {
        pub ptr: *mut c_void,
        pub rows: usize,
        pub cols: usize,
        pub dtype: c_int,
    }

    /// One independent Q8 call of a batch (device pointers).
    #[repr(C)]
    pub struct vmlm_q8_call {
        pub a: *const f32,
        pub q: *const i8,
        pub scale: *const f32,
        pub c: *mut f32,
        pub m: usize,
        pub n: usize,
        pub k: usize,
    }

    /// Opaque device constant pool of a .vmb program.
    #[repr(C)]
    pub struct vmlm_pool {
        _private: [u8; 0],
    }

    #[link(name = "vmlm_cuda")]
    extern "C" {
        pub fn vmlm_version() -> c_int;
        pub fn vmlm_init(device: c_int) -> c_int;
        pub fn vmlm_shutdown() -> c_int;
        pub fn vmlm_last_error() -> *const c_char;
        pub fn vmlm_register_weight(host_ptr: *const c_void, bytes: usize) -> c_int;
        pub fn vmlm_unregister_weight(host_ptr: *const c_void) -> c_int;
        pub fn vmlm_unregister_all() -> c_int;
        pub fn vmlm_gemm_nt_int8(a: *const f32, q: *const i8, scale: *const f32, c: *mut f32, m: usize, n: usize,
                                 k: usize) -> c_int;
        pub fn vmlm_gemm_nt_bf16(a: *const f32, b: *const u16, c: *mut f32, m: usize, n: usize, k: usize) -> c_int;
        pub fn vmlm_gemm_nt_f32(a: *const f32, b: *const f32, c: *mut f32, m: usize, n: usize, k: usize,
                                acc: c_int) -> c_int;
        pub fn vmlm_gemm_f32(a: *const f32, b: *const f32, c: *mut f32, m: usize, n: usize, k: usize,
                             acc: c_int) -> c_int;
        pub fn vmlm_gemm_i8i8(x: *const i8, w: *const i8, scale: *const f32, c: *mut f32, acc: *mut i32, m: usize,
                              n: usize, k: usize) -> c_int;
        pub fn vmlm_rmsnorm_gemm_nt_int8(a: *const f32, g: *const f32, eps: f32, q: *const i8, scale: *const f32,
                                         c: *mut f32, m: usize, n: usize, k: usize) -> c_int;
        pub fn vmlm_gemv_f32(a: *const f32, b: *const f32, c: *mut f32, m: usize, k: usize) -> c_int;
        pub fn vmlm_emb(table: *const c_void, dtype: c_int, rows: usize, cols: usize, idx: *const f32, m: usize,
                        out: *mut f32) -> c_int;
        pub fn vmlm_gemm_nt_int4_gs(a: *const f32, packed: *const u8, scale: *const f32, c: *mut f32, m: usize,
                                    n: usize, k: usize, group: usize, order: c_int) -> c_int;
        pub fn vmlm_gemm_nt_int8_outlier(a: *const f32, q: *const i8, scale: *const f32, w: *const f32,
                                         idx: *const u32, n_idx: usize, c: *mut f32, m: usize, n: usize,
                                         k: usize) -> c_int;
        pub fn vmlm_op_gemm(fl: c_uint, d: *const vmlm_slot, a: *const vmlm_slot, b: *const vmlm_slot,
                            scale: *const vmlm_slot) -> c_int;
        pub fn vmlm_gemm_nt_int8_batch_dev(calls: *const vmlm_q8_call, count: usize, stream: *mut c_void) -> c_int;
        pub fn vmlm_pool_load(vmb: *const c_void, len: usize, weights: *const c_void, weights_len: usize,
                              out: *mut *mut vmlm_pool) -> c_int;
        pub fn vmlm_pool_free(pool: *mut vmlm_pool) -> c_int;
        pub fn vmlm_pool_layerb(pool: *mut vmlm_pool, delta: f32) -> c_int;
        pub fn vmlm_pool_gemm(pool: *mut vmlm_pool, ins: *const c_void, stream: *mut c_void) -> c_int;
        pub fn vmlm_sync(stream: *mut c_void) -> c_int;
    }
}

/// The VM's convention for misuse: print the message and exit with code 9.
pub unsafe fn check(rc: c_int) {
    if rc != 0 {
        vmlm_sys::print(b"vmlm_cuda: ");
        let msg = ffi::vmlm_last_error() as *const u8;
        let mut n = 0usize;
        while *msg.add(n) != 0 {
            n += 1;
        }
        vmlm_sys::print(core::slice::from_raw_parts(msg, n));
        vmlm_sys::print(b"\n");
        vmlm_sys::exit_i(9);
    }
}

/// Same names and signatures as `vmlm_ops::kernels`.
pub mod kernels {
    use super::{check, ffi};
    use core::ffi::c_int;

    /// ops/src/kernels.rs:1256-1261: C[i][j] = (sum_k a[i][k] * q[j][k]) * scale[j], C overwritten.
    pub unsafe fn gemm_nt_int8(a: *const f32, q: *const i8, scale: *const f32, c: *mut f32, m: usize, n: usize,
                               k: usize) {
        check(ffi::vmlm_gemm_nt_int8(a, q, scale, c, m, n, k));
    }

    /// ops/src/kernels.rs:1200-1204: C[i][j] = sum_k a[i][k] * widen(b[j][k]), C overwritten.
    pub unsafe fn gemm_nt_bf16(a: *const f32, b: *const u16, c: *mut f32, m: usize, n: usize, k: usize) {
        check(ffi::vmlm_gemm_nt_bf16(a, b, c, m, n, k));
    }

    /// ops/src/kernels.rs:987-995: C = A . B^T (+ C when acc), B [n, k].
    pub unsafe fn gemm_nt(a: *const f32, b: *const f32, c: *mut f32, m: usize, n: usize, k: usize, acc: bool) {
        check(ffi::vmlm_gemm_nt_f32(a, b, c, m, n, k, acc as c_int));
    }

    /// ops/src/kernels.rs:407-415: C = A . B (+ C when acc), B [k, n].
    pub unsafe fn gemm(a: *const f32, b: *const f32, c: *mut f32, m: usize, n: usize, k: usize, acc: bool) {
        check(ffi::vmlm_gemm_f32(a, b, c, m, n, k, acc as c_int));
    }
}
