// CPython binding of the per-op entry points of libmusapy_b200.
//
// musapy's Python surface calls its Rust ops layer through PyO3
// (rust/musapy-python/src/ops.rs), a compiled binding whose per-call cost is
// argument extraction plus the launch. The ctypes route costs several
// microseconds per call for a 15-argument function (argument conversion
// objects, a libffi call frame), which on a small op is as long as the
// kernel. This module is the compiled binding for the calls made on every
// op: shapes and strides arrive as Python tuples of ints and are unpacked
// into stack arrays, pointers and dtype codes as ints, and the C-ABI is
// called directly (METH_FASTCALL: no argument tuple is built). The GIL stays
// held, as in the reference: a launch returns in microseconds.
//
// Functions (all return the mpb status code; 0 = MPB_OK):
//   elementwise(op, shape, a, a_dtype, a_strides, b, b_dtype, b_strides,
//               out, out_dtype, compute_dtype, p0, p1, stream)
//   elementwise_bc(op, out_shape, a, a_dtype, a_shape, a_strides, b,
//                  b_dtype, b_shape, b_strides, out, out_dtype,
//                  compute_dtype, p0, p1, stream)   (broadcast here)
//   reduce_scratch_bytes(op, shape, strides, a, in_dtype, axes_mask,
//                        compute_dtype) -> bytes
//   reduce(op, shape, strides, a, in_dtype, axes_mask, out, out_dtype,
//          compute_dtype, nan_first_rule, scratch, scratch_bytes, stream)
// Pointers and streams are ints (0 or None for none); a_strides / b_strides
// may be None where the C-ABI accepts a null array.
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <cstdint>

#include "musapy_b200.h"

namespace {

constexpr int kMaxDims = 32;

// tuple/list of ints -> out[0..n); returns n, or -1 with a Python error set
int dims(PyObject* o, int64_t* out, const char* what) {
  if (o == Py_None) return 0;
  PyObject* seq = PySequence_Fast(o, what);
  if (!seq) return -1;
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(seq);
  if (n > kMaxDims) {
    Py_DECREF(seq);
    PyErr_Format(PyExc_ValueError, "%s: %zd dims (at most %d)", what, n, kMaxDims);
    return -1;
  }
  PyObject** items = PySequence_Fast_ITEMS(seq);
  for (Py_ssize_t i = 0; i < n; ++i) {
    out[i] = PyLong_AsLongLong(items[i]);
    if (out[i] == -1 && PyErr_Occurred()) {
      Py_DECREF(seq);
      return -1;
    }
  }
  Py_DECREF(seq);
  return (int)n;
}

bool ptr(PyObject* o, void** out) {
  if (o == Py_None) {
    *out = nullptr;
    return true;
  }
  *out = PyLong_AsVoidPtr(o);
  return !(*out == nullptr && PyErr_Occurred());
}

bool i32(PyObject* o, int* out) {
  const long v = PyLong_AsLong(o);
  if (v == -1 && PyErr_Occurred()) return false;
  *out = (int)v;
  return true;
}

bool u64(PyObject* o, uint64_t* out) {
  const unsigned long long v = PyLong_AsUnsignedLongLong(o);
  if (v == (unsigned long long)-1 && PyErr_Occurred()) return false;
  *out = v;
  return true;
}

bool nargs(Py_ssize_t n, Py_ssize_t want, const char* fn) {
  if (n == want) return true;
  PyErr_Format(PyExc_TypeError, "%s() takes %zd arguments (%zd given)", fn, want, n);
  return false;
}

PyObject* py_elementwise(PyObject*, PyObject* const* args, Py_ssize_t n) {
  if (!nargs(n, 14, "elementwise")) return nullptr;
  int op, a_dt, b_dt, out_dt, cdt;
  int64_t shape[kMaxDims], as[kMaxDims], bs[kMaxDims];
  void *a, *b, *out, *stream;
  if (!i32(args[0], &op)) return nullptr;
  const int nd = dims(args[1], shape, "shape");
  if (nd < 0 || !ptr(args[2], &a) || !i32(args[3], &a_dt)) return nullptr;
  const bool has_as = args[4] != Py_None, has_bs = args[7] != Py_None;
  const int na = dims(args[4], as, "a_strides");
  if (na < 0 || !ptr(args[5], &b) || !i32(args[6], &b_dt)) return nullptr;
  const int nb = dims(args[7], bs, "b_strides");
  if (nb < 0 || !ptr(args[8], &out) || !i32(args[9], &out_dt) || !i32(args[10], &cdt)) return nullptr;
  if ((has_as && na != nd) || (has_bs && nb != nd)) {
    PyErr_SetString(PyExc_ValueError, "elementwise: strides and shape differ in length");
    return nullptr;
  }
  const double p0 = PyFloat_AsDouble(args[11]);
  if (p0 == -1.0 && PyErr_Occurred()) return nullptr;
  const double p1 = PyFloat_AsDouble(args[12]);
  if (p1 == -1.0 && PyErr_Occurred()) return nullptr;
  if (!ptr(args[13], &stream)) return nullptr;
  const int rc = mpb_elementwise(op, nd, shape, a, a_dt, has_as ? as : nullptr, b, b_dt, has_bs ? bs : nullptr, out,
                                 out_dt, cdt, p0, p1, (mpb_stream_t)stream);
  return PyLong_FromLong(rc);
}

// broadcast_strides (broadcast.rs:57-92): the strides of an operand of
// shape in[0..ni) (strides st) on the output shape out[0..nd): 0 where a
// dim is added on the left or stretched from extent 1.
bool bcast_strides(const int64_t* out, int nd, const int64_t* in, const int64_t* st, int ni, int64_t* res) {
  if (ni > nd) {
    PyErr_SetString(PyExc_ValueError, "elementwise_bc: operand has more dims than the output");
    return false;
  }
  for (int i = 0; i < nd; ++i) {
    const int j = i - (nd - ni);
    if (j < 0 || (in[j] == 1 && out[i] != 1)) {
      res[i] = 0;
    } else if (in[j] == out[i]) {
      res[i] = st[j];
    } else {
      PyErr_Format(PyExc_ValueError, "elementwise_bc: extent %lld does not broadcast to %lld", (long long)in[j],
                   (long long)out[i]);
      return false;
    }
  }
  return true;
}

// elementwise_bc(op, out_shape, a, a_dtype, a_shape, a_strides, b, b_dtype,
//                b_shape, b_strides, out, out_dtype, compute_dtype, p0, p1,
//                stream): a binary op with the operands' own shapes and
// strides, broadcast here onto out_shape.
PyObject* py_elementwise_bc(PyObject*, PyObject* const* args, Py_ssize_t n) {
  if (!nargs(n, 16, "elementwise_bc")) return nullptr;
  int op, a_dt, b_dt, out_dt, cdt;
  int64_t shape[kMaxDims], ash[kMaxDims], ast[kMaxDims], bsh[kMaxDims], bst[kMaxDims];
  int64_t as[kMaxDims], bs[kMaxDims];
  void *a, *b, *out, *stream;
  if (!i32(args[0], &op)) return nullptr;
  const int nd = dims(args[1], shape, "out_shape");
  if (nd < 0 || !ptr(args[2], &a) || !i32(args[3], &a_dt)) return nullptr;
  const int na = dims(args[4], ash, "a_shape");
  if (na < 0 || dims(args[5], ast, "a_strides") != na) {
    if (!PyErr_Occurred()) PyErr_SetString(PyExc_ValueError, "elementwise_bc: a_strides and a_shape differ");
    return nullptr;
  }
  if (!ptr(args[6], &b) || !i32(args[7], &b_dt)) return nullptr;
  const int nb = dims(args[8], bsh, "b_shape");
  if (nb < 0 || dims(args[9], bst, "b_strides") != nb) {
    if (!PyErr_Occurred()) PyErr_SetString(PyExc_ValueError, "elementwise_bc: b_strides and b_shape differ");
    return nullptr;
  }
  if (!ptr(args[10], &out) || !i32(args[11], &out_dt) || !i32(args[12], &cdt)) return nullptr;
  const double p0 = PyFloat_AsDouble(args[13]);
  if (p0 == -1.0 && PyErr_Occurred()) return nullptr;
  const double p1 = PyFloat_AsDouble(args[14]);
  if (p1 == -1.0 && PyErr_Occurred()) return nullptr;
  if (!ptr(args[15], &stream)) return nullptr;
  if (!bcast_strides(shape, nd, ash, ast, na, as) || !bcast_strides(shape, nd, bsh, bst, nb, bs)) return nullptr;
  const int rc = mpb_elementwise(op, nd, shape, a, a_dt, as, b, b_dt, bs, out, out_dt, cdt, p0, p1,
                                 (mpb_stream_t)stream);
  return PyLong_FromLong(rc);
}

// shared head of the two reduce calls: op, shape, strides, a, in_dtype, mask
struct RedHead {
  int op, nd, in_dt;
  int64_t shape[kMaxDims], strides[kMaxDims];
  void* a;
  uint64_t mask;
};

bool red_head(PyObject* const* args, RedHead* h) {
  if (!i32(args[0], &h->op)) return false;
  h->nd = dims(args[1], h->shape, "shape");
  if (h->nd < 0) return false;
  const int ns = dims(args[2], h->strides, "strides");
  if (ns < 0) return false;
  if (ns != h->nd) {
    PyErr_SetString(PyExc_ValueError, "reduce: strides and shape differ in length");
    return false;
  }
  return ptr(args[3], &h->a) && i32(args[4], &h->in_dt) && u64(args[5], &h->mask);
}

PyObject* py_reduce_scratch_bytes(PyObject*, PyObject* const* args, Py_ssize_t n) {
  if (!nargs(n, 7, "reduce_scratch_bytes")) return nullptr;
  RedHead h;
  int cdt;
  if (!red_head(args, &h) || !i32(args[6], &cdt)) return nullptr;
  return PyLong_FromSize_t(mpb_reduce_scratch_bytes(h.op, h.nd, h.shape, h.strides, h.a, h.in_dt, h.mask, cdt));
}

PyObject* py_reduce(PyObject*, PyObject* const* args, Py_ssize_t n) {
  if (!nargs(n, 13, "reduce")) return nullptr;
  RedHead h;
  int out_dt, cdt, nan_first;
  void *out, *scratch, *stream;
  if (!red_head(args, &h) || !ptr(args[6], &out) || !i32(args[7], &out_dt) || !i32(args[8], &cdt) ||
      !i32(args[9], &nan_first) || !ptr(args[10], &scratch))
    return nullptr;
  const size_t sbytes = PyLong_AsSize_t(args[11]);
  if (sbytes == (size_t)-1 && PyErr_Occurred()) return nullptr;
  if (!ptr(args[12], &stream)) return nullptr;
  const int rc = mpb_reduce(h.op, h.nd, h.shape, h.strides, h.a, h.in_dt, h.mask, out, out_dt, cdt, nan_first, scratch,
                            sbytes, (mpb_stream_t)stream);
  return PyLong_FromLong(rc);
}

PyMethodDef kMethods[] = {
    {"elementwise", (PyCFunction)(void (*)(void))py_elementwise, METH_FASTCALL,
     "mpb_elementwise with shapes and strides as tuples"},
    {"elementwise_bc", (PyCFunction)(void (*)(void))py_elementwise_bc, METH_FASTCALL,
     "mpb_elementwise of a binary op, broadcasting the operands' shapes and strides"},
    {"reduce_scratch_bytes", (PyCFunction)(void (*)(void))py_reduce_scratch_bytes, METH_FASTCALL,
     "mpb_reduce_scratch_bytes with shapes and strides as tuples"},
    {"reduce", (PyCFunction)(void (*)(void))py_reduce, METH_FASTCALL, "mpb_reduce with shapes and strides as tuples"},
    {nullptr, nullptr, 0, nullptr},
};

PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_native", "Compiled per-op binding of libmusapy_b200", -1, kMethods};

}  // namespace

PyMODINIT_FUNC PyInit__native(void) { return PyModule_Create(&kModule); }
