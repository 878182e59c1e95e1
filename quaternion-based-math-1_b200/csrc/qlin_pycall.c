/* CPython binding of qlin_forward_ex (and qlin_forward_host) for the package's per-call path.
 *
 * The ctypes binding converts its 23 arguments in Python for every call
 * (about 8 us on the GPU host); this vectorcall function does the same
 * conversion in C.  It links against libqlin_b200.so (same directory), so
 * the process keeps one copy of the library and its device state.
 * Arguments (positional, all ints except lora_scale; pointer arguments may
 * be None): dtype, x, ld_x, wr, wi, wj, wk, ld_w, bias, lora_a, lora_b, rank,
 * lora_scale, y, ld_y, M, K_g, N_g, workspace, workspace_bytes, algo, flags,
 * stream.  Returns the status code. */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>

#include "qlin_b200.h"

static int as_ptr(PyObject* o, void** out) {
  if (o == Py_None) {
    *out = NULL;
    return 0;
  }
  unsigned long long v = PyLong_AsUnsignedLongLong(o);
  if (v == (unsigned long long)-1 && PyErr_Occurred()) return -1;
  *out = (void*)(uintptr_t)v;
  return 0;
}

static int as_i64(PyObject* o, int64_t* out) {
  long long v = PyLong_AsLongLong(o);
  if (v == -1 && PyErr_Occurred()) return -1;
  *out = (int64_t)v;
  return 0;
}

static PyObject* forward_ex(PyObject* self, PyObject* const* a, Py_ssize_t n) {
  (void)self;
  if (n != 23) {
    PyErr_SetString(PyExc_TypeError, "forward_ex takes 23 arguments");
    return NULL;
  }
  int64_t dtype, ld_x, ld_w, rank, ld_y, M, K_g, N_g, ws_bytes, algo, flags;
  void *x, *wr, *wi, *wj, *wk, *bias, *la, *lb, *y, *ws, *stream;
  if (as_i64(a[0], &dtype) || as_ptr(a[1], &x) || as_i64(a[2], &ld_x) || as_ptr(a[3], &wr) ||
      as_ptr(a[4], &wi) || as_ptr(a[5], &wj) || as_ptr(a[6], &wk) || as_i64(a[7], &ld_w) ||
      as_ptr(a[8], &bias) || as_ptr(a[9], &la) || as_ptr(a[10], &lb) || as_i64(a[11], &rank))
    return NULL;
  double scale = PyFloat_AsDouble(a[12]);
  if (scale == -1.0 && PyErr_Occurred()) return NULL;
  if (as_ptr(a[13], &y) || as_i64(a[14], &ld_y) || as_i64(a[15], &M) || as_i64(a[16], &K_g) ||
      as_i64(a[17], &N_g) || as_ptr(a[18], &ws) || as_i64(a[19], &ws_bytes) || as_i64(a[20], &algo) ||
      as_i64(a[21], &flags) || as_ptr(a[22], &stream))
    return NULL;
  const int st = qlin_forward_ex((int)dtype, x, ld_x, wr, wi, wj, wk, ld_w, bias, la, lb, (int)rank,
                                 (float)scale, y, ld_y, M, K_g, N_g, ws, (size_t)ws_bytes, (int)algo,
                                 (int)flags, stream);
  return PyLong_FromLong(st);
}

/* qlin_forward_host: the same 23 arguments, x and y host addresses. */
static PyObject* forward_host(PyObject* self, PyObject* const* a, Py_ssize_t n) {
  (void)self;
  if (n != 23) {
    PyErr_SetString(PyExc_TypeError, "forward_host takes 23 arguments");
    return NULL;
  }
  int64_t dtype, ld_x, ld_w, rank, ld_y, M, K_g, N_g, ws_bytes, algo, flags;
  void *x, *wr, *wi, *wj, *wk, *bias, *la, *lb, *y, *ws, *stream;
  if (as_i64(a[0], &dtype) || as_ptr(a[1], &x) || as_i64(a[2], &ld_x) || as_ptr(a[3], &wr) ||
      as_ptr(a[4], &wi) || as_ptr(a[5], &wj) || as_ptr(a[6], &wk) || as_i64(a[7], &ld_w) ||
      as_ptr(a[8], &bias) || as_ptr(a[9], &la) || as_ptr(a[10], &lb) || as_i64(a[11], &rank))
    return NULL;
  double scale = PyFloat_AsDouble(a[12]);
  if (scale == -1.0 && PyErr_Occurred()) return NULL;
  if (as_ptr(a[13], &y) || as_i64(a[14], &ld_y) || as_i64(a[15], &M) || as_i64(a[16], &K_g) ||
      as_i64(a[17], &N_g) || as_ptr(a[18], &ws) || as_i64(a[19], &ws_bytes) || as_i64(a[20], &algo) ||
      as_i64(a[21], &flags) || as_ptr(a[22], &stream))
    return NULL;
  const int st = qlin_forward_host((int)dtype, x, ld_x, wr, wi, wj, wk, ld_w, bias, la, lb, (int)rank,
                                   (float)scale, y, ld_y, M, K_g, N_g, ws, (size_t)ws_bytes, (int)algo,
                                   (int)flags, stream);
  return PyLong_FromLong(st);
}

static PyMethodDef methods[] = {
    {"forward_ex", (PyCFunction)(void (*)(void))forward_ex, METH_FASTCALL, "qlin_forward_ex (see qlin_b200.h)"},
    {"forward_host", (PyCFunction)(void (*)(void))forward_host, METH_FASTCALL, "qlin_forward_host (see qlin_b200.h)"},
    {NULL, NULL, 0, NULL}};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_qlin_call", NULL, -1, methods};

PyMODINIT_FUNC PyInit__qlin_call(void) { return PyModule_Create(&module); }
