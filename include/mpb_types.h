// Shared enums and limits of the musapy-b200 engine (host, device and the
// public C-ABI in musapy_b200.h).
//
// The dtype numbering follows the declaration order of musapy's `Dtype`
// enum (rust/musapy-core/src/dtype.rs:25-41) so that a tag crossing the
// C-ABI means the same thing on both sides.
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum mpb_dtype {
  MPB_BOOL = 0,
  MPB_I8 = 1,
  MPB_I16 = 2,
  MPB_I32 = 3,
  MPB_I64 = 4,
  MPB_U8 = 5,
  MPB_U16 = 6,
  MPB_U32 = 7,
  MPB_U64 = 8,
  MPB_F16 = 9,
  MPB_F32 = 10,
  MPB_F64 = 11,
  MPB_BF16 = 12,
  MPB_C64 = 13,
  MPB_C128 = 14,
  MPB_NUM_DTYPES = 15
};

// Elementwise operators. Binary arithmetic, comparisons, unary math,
// clamp and cast share one engine; the op decides arity and output kind.
enum mpb_ew_op {
  MPB_ADD = 0,
  MPB_SUB = 1,
  MPB_MUL = 2,
  MPB_DIV = 3,
  MPB_POW = 4,
  MPB_EQ = 10,
  MPB_NE = 11,
  MPB_LT = 12,
  MPB_GT = 13,
  MPB_LE = 14,
  MPB_GE = 15,
  MPB_SIN = 20,
  MPB_COS = 21,
  MPB_EXP = 22,
  MPB_LOG = 23,
  MPB_ABS = 24,
  MPB_SIGN = 25,
  MPB_NEG = 26,
  MPB_CLAMP = 30,
  MPB_CAST = 31,  // identity in the compute type: a dtype conversion / strided copy
  MPB_FILL = 32   // no input: out[i] = p0 (creation kernels)
};

// Reductions (rust/musapy-ops/src/op_builder.rs:2162-2171 ReduceKernel).
enum mpb_red_op {
  MPB_R_SUM = 0,
  MPB_R_PROD = 1,
  MPB_R_MAX = 2,
  MPB_R_MIN = 3,
  MPB_R_MEAN = 4,
  MPB_R_ARGMAX = 5,
  MPB_R_ARGMIN = 6,
  // (value, index) record per output, 16 bytes: used to combine shards
  MPB_R_ARGMAX_REC = 7,
  MPB_R_ARGMIN_REC = 8
};

// Status codes returned by every extended entry point.
enum mpb_status {
  MPB_OK = 0,
  MPB_ERR_INVALID = 1,      // malformed arguments (ndim, null pointer, axis)
  MPB_ERR_DTYPE = 2,        // dtype / op combination not supported
  MPB_ERR_SHAPE = 3,        // shape / stride problem (e.g. too many dims)
  MPB_ERR_SCRATCH = 4,      // caller scratch smaller than *_scratch_bytes()
  MPB_ERR_CUDA = 5,         // CUDA launch / runtime error
  MPB_ERR_TIMEOUT = 6,      // a bounded device-side wait gave up
  MPB_ERR_UNSUPPORTED = 7   // valid request outside the implemented kernels
};

#define MPB_MAX_DIMS 32

#ifdef __cplusplus
}
#endif
