/*
 * libmusapy_b200 - musapy's kernel C-ABI, reproduced symbol for symbol.
 *
 * Every declaration below has the name, argument order and argument types of
 * the extern "C" kernel wrapper musapy's operator layer binds in
 * rust/musapy-ops/src/kernels.rs (cited per symbol), with musaStream_t
 * replaced by a CUDA stream, so a CUDA build of musapy's Rust layers can link
 * this library in place of libmusapy_kernels.a. Each wrapper routes to the
 * engine behind include/musapy_b200.h (collapsed geometry, fused casts,
 * sm_100a kernels).
 *
 * Contract (docs/adr/ADR.md:322-338): void return; strides in elements (0 or
 * negative allowed); pointers pre-adjusted by the view offset; outputs
 * C-contiguous; shape/stride arrays are host memory. A launch failure stays
 * visible to the caller's cudaGetLastError() as before; requests the engine
 * rejects (e.g. more than 32 dims) launch nothing and are described by
 * mpb_last_error().
 *
 * Semantics where the engine is stricter than musapy's GPU kernels:
 * max/min/argmax/argmin follow musapy's CPU rule (first occurrence, NaN only
 * when it is the first element) in every variant; cumsum has no 256^3 length
 * limit. The partial/mid/final stages keep their musapy layouts
 * ([out_size][tiles] partials): the partial stage writes the whole reduction
 * of each output into tile 0 and the identity (or a copy, for max/min/arg) into
 * the other tiles, so any sequence of mid/final calls musapy makes returns the
 * same result.
 *
 * Not reproduced (outside this path): musapy_resize_c64_v2 (kernels.rs:126), musapy_resize_c128_v2 (kernels.rs:127), musapy_resize_f32_real_v2 (kernels.rs:129), musapy_resize_f64_real_v2 (kernels.rs:130), musapy_cast_resize_f32_c64_v2 (kernels.rs:132), musapy_cast_resize_f64_c128_v2 (kernels.rs:133), musapy_scale_c64_v2 (kernels.rs:135), musapy_scale_c128_v2 (kernels.rs:136), musapy_gather_f32_v2 (kernels.rs:309), musapy_gather_f64_v2 (kernels.rs:310), musapy_gather_i32_v2 (kernels.rs:311), musapy_gather_i64_v2 (kernels.rs:312), musapy_scatter_f32_v2 (kernels.rs:315), musapy_scatter_f64_v2 (kernels.rs:316), musapy_scatter_i32_v2 (kernels.rs:317), musapy_scatter_i64_v2 (kernels.rs:318), musapy_extract_diag_f32_v1 (kernels.rs:334), musapy_extract_diag_f64_v1 (kernels.rs:335), musapy_adv_gather_f32_v2 (kernels.rs:341), musapy_adv_gather_f64_v2 (kernels.rs:342), musapy_adv_gather_i32_v2 (kernels.rs:343).
 */
#ifndef MUSAPY_KERNELS_V2_H
#define MUSAPY_KERNELS_V2_H

#include <stddef.h>
#include <stdint.h>

#include "musapy_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Interleaved {re, im} layout of muComplex / muDoubleComplex. */
typedef struct { float re, im; } musapy_complex64;
typedef struct { double re, im; } musapy_complex128;

/* ---- Binary arithmetic (kernels.rs:19-28, :102-109) */
/* kernels.rs:19 */
void musapy_add_f32_v2(const float* a, const float* b, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:20 */
void musapy_add_f64_v2(const double* a, const double* b, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:21 */
void musapy_sub_f32_v2(const float* a, const float* b, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:22 */
void musapy_sub_f64_v2(const double* a, const double* b, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:23 */
void musapy_mul_f32_v2(const float* a, const float* b, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:24 */
void musapy_mul_f64_v2(const double* a, const double* b, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:25 */
void musapy_div_f32_v2(const float* a, const float* b, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:26 */
void musapy_div_f64_v2(const double* a, const double* b, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:27 */
void musapy_pow_f32_v2(const float* a, const float* b, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:28 */
void musapy_pow_f64_v2(const double* a, const double* b, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:102 */
void musapy_add_c64_v2(const musapy_complex64* a, const musapy_complex64* b, musapy_complex64* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:103 */
void musapy_add_c128_v2(const musapy_complex128* a, const musapy_complex128* b, musapy_complex128* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:104 */
void musapy_sub_c64_v2(const musapy_complex64* a, const musapy_complex64* b, musapy_complex64* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:105 */
void musapy_sub_c128_v2(const musapy_complex128* a, const musapy_complex128* b, musapy_complex128* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:106 */
void musapy_mul_c64_v2(const musapy_complex64* a, const musapy_complex64* b, musapy_complex64* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:107 */
void musapy_mul_c128_v2(const musapy_complex128* a, const musapy_complex128* b, musapy_complex128* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:108 */
void musapy_div_c64_v2(const musapy_complex64* a, const musapy_complex64* b, musapy_complex64* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:109 */
void musapy_div_c128_v2(const musapy_complex128* a, const musapy_complex128* b, musapy_complex128* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);

/* ---- Unary math and clamp (kernels.rs:31-48, :110-113) */
/* kernels.rs:31 */
void musapy_sin_f32_v2(const float* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:32 */
void musapy_sin_f64_v2(const double* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:33 */
void musapy_cos_f32_v2(const float* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:34 */
void musapy_cos_f64_v2(const double* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:35 */
void musapy_exp_f32_v2(const float* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:36 */
void musapy_exp_f64_v2(const double* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:37 */
void musapy_log_f32_v2(const float* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:38 */
void musapy_log_f64_v2(const double* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:39 */
void musapy_abs_f32_v2(const float* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:40 */
void musapy_abs_f64_v2(const double* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:41 */
void musapy_sign_f32_v2(const float* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:42 */
void musapy_sign_f64_v2(const double* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:43 */
void musapy_neg_f32_v2(const float* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:44 */
void musapy_neg_f64_v2(const double* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:47 */
void musapy_clamp_f32_v2(const float* a, float* c, float lo, float hi, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:48 */
void musapy_clamp_f64_v2(const double* a, double* c, double lo, double hi, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:110 */
void musapy_neg_c64_v2(const musapy_complex64* a, musapy_complex64* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:111 */
void musapy_neg_c128_v2(const musapy_complex128* a, musapy_complex128* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:112 */
void musapy_abs_c64_v2(const musapy_complex64* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:113 */
void musapy_abs_c128_v2(const musapy_complex128* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);

/* ---- Casts (kernels.rs:51-81, :119-124) */
/* kernels.rs:51 */
void musapy_cast_i8_f32_v2(const int8_t* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:52 */
void musapy_cast_i16_f32_v2(const int16_t* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:53 */
void musapy_cast_i32_f32_v2(const int32_t* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:54 */
void musapy_cast_i64_f32_v2(const int64_t* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:55 */
void musapy_cast_u8_f32_v2(const uint8_t* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:56 */
void musapy_cast_u16_f32_v2(const uint16_t* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:57 */
void musapy_cast_u32_f32_v2(const uint32_t* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:58 */
void musapy_cast_u64_f32_v2(const uint64_t* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:59 */
void musapy_cast_f64_f32_v2(const double* a, float* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:62 */
void musapy_cast_i8_f64_v2(const int8_t* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:63 */
void musapy_cast_i16_f64_v2(const int16_t* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:64 */
void musapy_cast_i32_f64_v2(const int32_t* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:65 */
void musapy_cast_i64_f64_v2(const int64_t* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:66 */
void musapy_cast_u8_f64_v2(const uint8_t* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:67 */
void musapy_cast_u16_f64_v2(const uint16_t* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:68 */
void musapy_cast_u32_f64_v2(const uint32_t* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:69 */
void musapy_cast_u64_f64_v2(const uint64_t* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:70 */
void musapy_cast_f32_f64_v2(const float* a, double* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:73 */
void musapy_cast_i8_i64_v2(const int8_t* a, int64_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:74 */
void musapy_cast_i16_i64_v2(const int16_t* a, int64_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:75 */
void musapy_cast_i32_i64_v2(const int32_t* a, int64_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:76 */
void musapy_cast_u8_i64_v2(const uint8_t* a, int64_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:77 */
void musapy_cast_u16_i64_v2(const uint16_t* a, int64_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:78 */
void musapy_cast_u32_i64_v2(const uint32_t* a, int64_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:79 */
void musapy_cast_u64_i64_v2(const uint64_t* a, int64_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:80 */
void musapy_cast_f32_i64_v2(const float* a, int64_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:81 */
void musapy_cast_f64_i64_v2(const double* a, int64_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:119 */
void musapy_cast_f32_c64_v2(const float* a, musapy_complex64* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:120 */
void musapy_cast_f32_c128_v2(const float* a, musapy_complex128* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:121 */
void musapy_cast_f64_c64_v2(const double* a, musapy_complex64* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:122 */
void musapy_cast_f64_c128_v2(const double* a, musapy_complex128* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);
/* kernels.rs:124 */
void musapy_cast_c64_c128_v2(const musapy_complex64* a, musapy_complex128* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, mpb_stream_t stream);

/* ---- Comparisons (kernels.rs:84-95, :114-117) */
/* kernels.rs:84 */
void musapy_eq_f32_v2(const float* a, const float* b, uint8_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:85 */
void musapy_eq_f64_v2(const double* a, const double* b, uint8_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:86 */
void musapy_ne_f32_v2(const float* a, const float* b, uint8_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:87 */
void musapy_ne_f64_v2(const double* a, const double* b, uint8_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:88 */
void musapy_lt_f32_v2(const float* a, const float* b, uint8_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:89 */
void musapy_lt_f64_v2(const double* a, const double* b, uint8_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:90 */
void musapy_gt_f32_v2(const float* a, const float* b, uint8_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:91 */
void musapy_gt_f64_v2(const double* a, const double* b, uint8_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:92 */
void musapy_le_f32_v2(const float* a, const float* b, uint8_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:93 */
void musapy_le_f64_v2(const double* a, const double* b, uint8_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:94 */
void musapy_ge_f32_v2(const float* a, const float* b, uint8_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:95 */
void musapy_ge_f64_v2(const double* a, const double* b, uint8_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:114 */
void musapy_eq_c64_v2(const musapy_complex64* a, const musapy_complex64* b, uint8_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:115 */
void musapy_eq_c128_v2(const musapy_complex128* a, const musapy_complex128* b, uint8_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:116 */
void musapy_ne_c64_v2(const musapy_complex64* a, const musapy_complex64* b, uint8_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);
/* kernels.rs:117 */
void musapy_ne_c128_v2(const musapy_complex128* a, const musapy_complex128* b, uint8_t* c, int32_t ndim, const size_t* shape, const ptrdiff_t* a_strides, const ptrdiff_t* b_strides, mpb_stream_t stream);

/* ---- Reductions, one launch per call (kernels.rs:139-180, :259-264) */
/* kernels.rs:139 */
void musapy_sum_i64_v2(const int64_t* a, int64_t* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:140 */
void musapy_sum_f32_v2(const float* a, float* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:141 */
void musapy_sum_f64_v2(const double* a, double* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:142 */
void musapy_prod_i64_v2(const int64_t* a, int64_t* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:143 */
void musapy_prod_f32_v2(const float* a, float* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:144 */
void musapy_prod_f64_v2(const double* a, double* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:145 */
void musapy_max_i64_v2(const int64_t* a, int64_t* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:146 */
void musapy_max_f32_v2(const float* a, float* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:147 */
void musapy_max_f64_v2(const double* a, double* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:148 */
void musapy_min_i64_v2(const int64_t* a, int64_t* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:149 */
void musapy_min_f32_v2(const float* a, float* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:150 */
void musapy_min_f64_v2(const double* a, double* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:151 */
void musapy_mean_f32_v2(const float* a, float* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:152 */
void musapy_mean_f64_v2(const double* a, double* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:154 */
void musapy_sum_c64_v2(const musapy_complex64* a, musapy_complex64* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:155 */
void musapy_sum_c128_v2(const musapy_complex128* a, musapy_complex128* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:156 */
void musapy_prod_c64_v2(const musapy_complex64* a, musapy_complex64* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:157 */
void musapy_prod_c128_v2(const musapy_complex128* a, musapy_complex128* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:158 */
void musapy_mean_c64_v2(const musapy_complex64* a, musapy_complex64* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:159 */
void musapy_mean_c128_v2(const musapy_complex128* a, musapy_complex128* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:161 */
void musapy_sum_small_axis_i64_v2(const int64_t* a, int64_t* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:162 */
void musapy_sum_small_axis_f32_v2(const float* a, float* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:163 */
void musapy_sum_small_axis_f64_v2(const double* a, double* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:164 */
void musapy_prod_small_axis_i64_v2(const int64_t* a, int64_t* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:165 */
void musapy_prod_small_axis_f32_v2(const float* a, float* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:166 */
void musapy_prod_small_axis_f64_v2(const double* a, double* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:167 */
void musapy_max_small_axis_i64_v2(const int64_t* a, int64_t* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:168 */
void musapy_max_small_axis_f32_v2(const float* a, float* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:169 */
void musapy_max_small_axis_f64_v2(const double* a, double* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:170 */
void musapy_min_small_axis_i64_v2(const int64_t* a, int64_t* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:171 */
void musapy_min_small_axis_f32_v2(const float* a, float* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:172 */
void musapy_min_small_axis_f64_v2(const double* a, double* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:173 */
void musapy_mean_small_axis_f32_v2(const float* a, float* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:174 */
void musapy_mean_small_axis_f64_v2(const double* a, double* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:175 */
void musapy_argmax_i64_v2(const int64_t* a, int64_t* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:176 */
void musapy_argmax_f32_v2(const float* a, int64_t* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:177 */
void musapy_argmax_f64_v2(const double* a, int64_t* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:178 */
void musapy_argmin_i64_v2(const int64_t* a, int64_t* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:179 */
void musapy_argmin_f32_v2(const float* a, int64_t* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:180 */
void musapy_argmin_f64_v2(const double* a, int64_t* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:259 */
void musapy_sum_small_axis_c64_v2(const musapy_complex64* a, musapy_complex64* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:260 */
void musapy_sum_small_axis_c128_v2(const musapy_complex128* a, musapy_complex128* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:261 */
void musapy_prod_small_axis_c64_v2(const musapy_complex64* a, musapy_complex64* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:262 */
void musapy_prod_small_axis_c128_v2(const musapy_complex128* a, musapy_complex128* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:263 */
void musapy_mean_small_axis_c64_v2(const musapy_complex64* a, musapy_complex64* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);
/* kernels.rs:264 */
void musapy_mean_small_axis_c128_v2(const musapy_complex128* a, musapy_complex128* c, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, int32_t group_size, mpb_stream_t stream);

/* ---- Reductions, partial / mid / final stages (kernels.rs:222-304) */
/* kernels.rs:222 */
void musapy_sum_partial_i64_v2(const int64_t* a, int64_t* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:223 */
void musapy_sum_partial_f32_v2(const float* a, float* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:224 */
void musapy_sum_partial_f64_v2(const double* a, double* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:225 */
void musapy_prod_partial_i64_v2(const int64_t* a, int64_t* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:226 */
void musapy_prod_partial_f32_v2(const float* a, float* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:227 */
void musapy_prod_partial_f64_v2(const double* a, double* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:228 */
void musapy_max_partial_i64_v2(const int64_t* a, int64_t* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:229 */
void musapy_max_partial_f32_v2(const float* a, float* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:230 */
void musapy_max_partial_f64_v2(const double* a, double* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:231 */
void musapy_min_partial_i64_v2(const int64_t* a, int64_t* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:232 */
void musapy_min_partial_f32_v2(const float* a, float* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:233 */
void musapy_min_partial_f64_v2(const double* a, double* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:235 */
void musapy_mean_partial_f32_v2(const float* a, float* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:236 */
void musapy_mean_partial_f64_v2(const double* a, double* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:240 */
void musapy_sum_final_i64_v2(const int64_t* partials, int64_t* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:241 */
void musapy_sum_final_f32_v2(const float* partials, float* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:242 */
void musapy_sum_final_f64_v2(const double* partials, double* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:243 */
void musapy_prod_final_i64_v2(const int64_t* partials, int64_t* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:244 */
void musapy_prod_final_f32_v2(const float* partials, float* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:245 */
void musapy_prod_final_f64_v2(const double* partials, double* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:246 */
void musapy_max_final_i64_v2(const int64_t* partials, int64_t* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:247 */
void musapy_max_final_f32_v2(const float* partials, float* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:248 */
void musapy_max_final_f64_v2(const double* partials, double* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:249 */
void musapy_min_final_i64_v2(const int64_t* partials, int64_t* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:250 */
void musapy_min_final_f32_v2(const float* partials, float* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:251 */
void musapy_min_final_f64_v2(const double* partials, double* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:254 */
void musapy_mean_final_f32_v2(const float* partials, float* c, size_t num_partials, size_t out_size, size_t axis_len, mpb_stream_t stream);
/* kernels.rs:255 */
void musapy_mean_final_f64_v2(const double* partials, double* c, size_t num_partials, size_t out_size, size_t axis_len, mpb_stream_t stream);
/* kernels.rs:265 */
void musapy_sum_partial_c64_v2(const musapy_complex64* a, musapy_complex64* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:266 */
void musapy_sum_partial_c128_v2(const musapy_complex128* a, musapy_complex128* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:267 */
void musapy_prod_partial_c64_v2(const musapy_complex64* a, musapy_complex64* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:268 */
void musapy_prod_partial_c128_v2(const musapy_complex128* a, musapy_complex128* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:269 */
void musapy_mean_partial_c64_v2(const musapy_complex64* a, musapy_complex64* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:270 */
void musapy_mean_partial_c128_v2(const musapy_complex128* a, musapy_complex128* partials, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:271 */
void musapy_sum_final_c64_v2(const musapy_complex64* partials, musapy_complex64* c, size_t num_partials, size_t out_size, size_t axis_len, mpb_stream_t stream);
/* kernels.rs:272 */
void musapy_sum_final_c128_v2(const musapy_complex128* partials, musapy_complex128* c, size_t num_partials, size_t out_size, size_t axis_len, mpb_stream_t stream);
/* kernels.rs:273 */
void musapy_prod_final_c64_v2(const musapy_complex64* partials, musapy_complex64* c, size_t num_partials, size_t out_size, size_t axis_len, mpb_stream_t stream);
/* kernels.rs:274 */
void musapy_prod_final_c128_v2(const musapy_complex128* partials, musapy_complex128* c, size_t num_partials, size_t out_size, size_t axis_len, mpb_stream_t stream);
/* kernels.rs:275 */
void musapy_mean_final_c64_v2(const musapy_complex64* partials, musapy_complex64* c, size_t num_partials, size_t out_size, size_t axis_len, mpb_stream_t stream);
/* kernels.rs:276 */
void musapy_mean_final_c128_v2(const musapy_complex128* partials, musapy_complex128* c, size_t num_partials, size_t out_size, size_t axis_len, mpb_stream_t stream);
/* kernels.rs:280 */
void musapy_argmax_partial_i64_v2(const int64_t* a, int64_t* partials_val, int64_t* partials_idx, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:281 */
void musapy_argmax_partial_f32_v2(const float* a, float* partials_val, int64_t* partials_idx, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:282 */
void musapy_argmax_partial_f64_v2(const double* a, double* partials_val, int64_t* partials_idx, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:283 */
void musapy_argmin_partial_i64_v2(const int64_t* a, int64_t* partials_val, int64_t* partials_idx, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:284 */
void musapy_argmin_partial_f32_v2(const float* a, float* partials_val, int64_t* partials_idx, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:285 */
void musapy_argmin_partial_f64_v2(const double* a, double* partials_val, int64_t* partials_idx, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, size_t tiles_per_output, mpb_stream_t stream);
/* kernels.rs:289 */
void musapy_argmax_final_i64_v2(const int64_t* partials_val, const int64_t* partials_idx, int64_t* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:290 */
void musapy_argmax_final_f32_v2(const float* partials_val, const int64_t* partials_idx, int64_t* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:291 */
void musapy_argmax_final_f64_v2(const double* partials_val, const int64_t* partials_idx, int64_t* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:292 */
void musapy_argmin_final_i64_v2(const int64_t* partials_val, const int64_t* partials_idx, int64_t* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:293 */
void musapy_argmin_final_f32_v2(const float* partials_val, const int64_t* partials_idx, int64_t* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:294 */
void musapy_argmin_final_f64_v2(const double* partials_val, const int64_t* partials_idx, int64_t* c, size_t num_partials, size_t out_size, mpb_stream_t stream);
/* kernels.rs:299 */
void musapy_argmax_mid_i64_v2(const int64_t* partials_val, const int64_t* partials_idx, int64_t* out_val, int64_t* out_idx, size_t out_size, size_t tiles_per_output, size_t axis_len, mpb_stream_t stream);
/* kernels.rs:300 */
void musapy_argmax_mid_f32_v2(const float* partials_val, const int64_t* partials_idx, float* out_val, int64_t* out_idx, size_t out_size, size_t tiles_per_output, size_t axis_len, mpb_stream_t stream);
/* kernels.rs:301 */
void musapy_argmax_mid_f64_v2(const double* partials_val, const int64_t* partials_idx, double* out_val, int64_t* out_idx, size_t out_size, size_t tiles_per_output, size_t axis_len, mpb_stream_t stream);
/* kernels.rs:302 */
void musapy_argmin_mid_i64_v2(const int64_t* partials_val, const int64_t* partials_idx, int64_t* out_val, int64_t* out_idx, size_t out_size, size_t tiles_per_output, size_t axis_len, mpb_stream_t stream);
/* kernels.rs:303 */
void musapy_argmin_mid_f32_v2(const float* partials_val, const int64_t* partials_idx, float* out_val, int64_t* out_idx, size_t out_size, size_t tiles_per_output, size_t axis_len, mpb_stream_t stream);
/* kernels.rs:304 */
void musapy_argmin_mid_f64_v2(const double* partials_val, const int64_t* partials_idx, double* out_val, int64_t* out_idx, size_t out_size, size_t tiles_per_output, size_t axis_len, mpb_stream_t stream);

/* ---- Cumsum (kernels.rs:185-187) */
/* kernels.rs:185 */
void musapy_cumsum_i64_v3(const int64_t* a, int64_t* c, int64_t* tmp, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:186 */
void musapy_cumsum_f32_v3(const float* a, float* c, float* tmp, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);
/* kernels.rs:187 */
void musapy_cumsum_f64_v3(const double* a, double* c, double* tmp, int32_t ndim, const size_t* in_shape, const ptrdiff_t* in_strides, int32_t axis, size_t axis_len, size_t out_size, mpb_stream_t stream);

/* ---- Creation (kernels.rs:193-218) */
/* kernels.rs:193 */
void musapy_fill_f32(float* out, float value, size_t n, mpb_stream_t stream);
/* kernels.rs:194 */
void musapy_fill_f64(double* out, double value, size_t n, mpb_stream_t stream);
/* kernels.rs:195 */
void musapy_fill_i64(int64_t* out, int64_t value, size_t n, mpb_stream_t stream);
/* kernels.rs:196 */
void musapy_fill_i32(int32_t* out, int32_t value, size_t n, mpb_stream_t stream);
/* kernels.rs:197 */
void musapy_fill_i16(int16_t* out, int16_t value, size_t n, mpb_stream_t stream);
/* kernels.rs:198 */
void musapy_fill_i8(int8_t* out, int8_t value, size_t n, mpb_stream_t stream);
/* kernels.rs:199 */
void musapy_fill_u64(uint64_t* out, uint64_t value, size_t n, mpb_stream_t stream);
/* kernels.rs:200 */
void musapy_fill_u32(uint32_t* out, uint32_t value, size_t n, mpb_stream_t stream);
/* kernels.rs:201 */
void musapy_fill_u16(uint16_t* out, uint16_t value, size_t n, mpb_stream_t stream);
/* kernels.rs:202 */
void musapy_fill_u8(uint8_t* out, uint8_t value, size_t n, mpb_stream_t stream);
/* kernels.rs:205 */
void musapy_arange_f32(float* out, float start, float step, size_t n, mpb_stream_t stream);
/* kernels.rs:206 */
void musapy_arange_f64(double* out, double start, double step, size_t n, mpb_stream_t stream);
/* kernels.rs:207 */
void musapy_arange_i64(int64_t* out, int64_t start, int64_t step, size_t n, mpb_stream_t stream);
/* kernels.rs:208 */
void musapy_arange_i32(int32_t* out, int32_t start, int32_t step, size_t n, mpb_stream_t stream);
/* kernels.rs:211 */
void musapy_linspace_f32(float* out, float start, float stop, size_t n, mpb_stream_t stream);
/* kernels.rs:212 */
void musapy_linspace_f64(double* out, double start, double stop, size_t n, mpb_stream_t stream);
/* kernels.rs:215 */
void musapy_eye_f32(float* out, size_t n, size_t m, int32_t k, mpb_stream_t stream);
/* kernels.rs:216 */
void musapy_eye_f64(double* out, size_t n, size_t m, int32_t k, mpb_stream_t stream);
/* kernels.rs:217 */
void musapy_eye_i64(int64_t* out, size_t n, size_t m, int32_t k, mpb_stream_t stream);
/* kernels.rs:218 */
void musapy_eye_i32(int32_t* out, size_t n, size_t m, int32_t k, mpb_stream_t stream);

/* ---- Strided copy and 2-D transpose copy (kernels.rs:321-330) */
/* kernels.rs:321 */
void musapy_copy_f32(const float* input, float* output, int32_t ndim, const size_t* shape, const ptrdiff_t* in_strides, mpb_stream_t stream);
/* kernels.rs:322 */
void musapy_copy_f64(const double* input, double* output, int32_t ndim, const size_t* shape, const ptrdiff_t* in_strides, mpb_stream_t stream);
/* kernels.rs:323 */
void musapy_copy_i32(const int32_t* input, int32_t* output, int32_t ndim, const size_t* shape, const ptrdiff_t* in_strides, mpb_stream_t stream);
/* kernels.rs:324 */
void musapy_copy_i64(const int64_t* input, int64_t* output, int32_t ndim, const size_t* shape, const ptrdiff_t* in_strides, mpb_stream_t stream);
/* kernels.rs:327 */
void musapy_copy_transpose2d_f32(const float* src, float* dst, size_t rows, size_t cols, mpb_stream_t stream);
/* kernels.rs:328 */
void musapy_copy_transpose2d_f64(const double* src, double* dst, size_t rows, size_t cols, mpb_stream_t stream);
/* kernels.rs:329 */
void musapy_copy_transpose2d_i32(const int32_t* src, int32_t* dst, size_t rows, size_t cols, mpb_stream_t stream);
/* kernels.rs:330 */
void musapy_copy_transpose2d_i64(const int64_t* src, int64_t* dst, size_t rows, size_t cols, mpb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MUSAPY_KERNELS_V2_H */
