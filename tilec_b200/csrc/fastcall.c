/* fastcall.c -- CPython entry points for the per-call path of tilec_b200.ext.
 *
 * The same two C ABI calls the ctypes binding makes for every matrix_mul
 * (tilec_mm_workspace_bytes, tilec_mm_f32; include/tilec_mm.h), without ctypes' per-argument
 * conversion, which costs about 1.4 us of the binding's per-call time.  The functions are
 * not linked: tilec_b200._native hands over the addresses of the ones in the already
 * loaded libtilec_mm.so (install()), so both bindings drive the same library instance.
 *
 *   install(addr_mm_f32, addr_workspace_bytes) -> None
 *   mm(a, b, c, M, N, K, lda, ldb, ldc, variant, split_k, flags, ws, ws_bytes, stream) -> int
 *   ws_bytes(a, b, c, M, N, K, lda, ldb, ldc, variant, split_k, flags) -> int
 *
 * Pointers (a, b, c, ws, stream) are Python ints (0 or None for NULL); the rest are ints.
 * Return values are the C ABI's status codes and byte counts, unchanged.
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>

#include "../../include/tilec_mm.h"

typedef int (*mm_f32_fn)(const float*, const float*, float*, int64_t, int64_t, int64_t, int64_t, int64_t,
                         int64_t, const tilec_mm_cfg*, void*, size_t, void*);
typedef size_t (*ws_bytes_fn)(const float*, const float*, const float*, int64_t, int64_t, int64_t, int64_t,
                              int64_t, int64_t, const tilec_mm_cfg*);

static mm_f32_fn g_mm = NULL;
static ws_bytes_fn g_ws = NULL;

static int as_ptr(PyObject* o, void** out) {
  if (o == Py_None) {
    *out = NULL;
    return 0;
  }
  const unsigned long long v = PyLong_AsUnsignedLongLong(o);
  if (v == (unsigned long long)-1 && PyErr_Occurred()) return -1;
  *out = (void*)(uintptr_t)v;
  return 0;
}

static int as_i64(PyObject* o, int64_t* out) {
  const long long v = PyLong_AsLongLong(o);
  if (v == -1 && PyErr_Occurred()) return -1;
  *out = (int64_t)v;
  return 0;
}

/* Parses the 12 leading arguments shared by mm() and ws_bytes(). */
static int parse_problem(PyObject* const* args, void** p, int64_t* d, tilec_mm_cfg* cfg) {
  for (int i = 0; i < 3; ++i)
    if (as_ptr(args[i], &p[i])) return -1;
  for (int i = 0; i < 6; ++i)
    if (as_i64(args[3 + i], &d[i])) return -1;
  int64_t v[3];
  for (int i = 0; i < 3; ++i)
    if (as_i64(args[9 + i], &v[i])) return -1;
  cfg->variant = (int32_t)v[0];
  cfg->split_k = (int32_t)v[1];
  cfg->flags = (int32_t)v[2];
  cfg->activation = 0;
  for (int i = 0; i < 4; ++i) cfg->reserved[i] = 0;
  return 0;
}

static PyObject* py_install(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  if (nargs != 2) {
    PyErr_SetString(PyExc_TypeError, "install(addr_mm_f32, addr_workspace_bytes)");
    return NULL;
  }
  void* a = NULL;
  void* b = NULL;
  if (as_ptr(args[0], &a) || as_ptr(args[1], &b)) return NULL;
  if (a == NULL || b == NULL) {
    PyErr_SetString(PyExc_ValueError, "install: null function address");
    return NULL;
  }
  g_mm = (mm_f32_fn)a;
  g_ws = (ws_bytes_fn)b;
  Py_RETURN_NONE;
}

static PyObject* py_mm(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  if (nargs != 15) {
    PyErr_SetString(PyExc_TypeError, "mm() takes 15 arguments");
    return NULL;
  }
  if (g_mm == NULL) {
    PyErr_SetString(PyExc_RuntimeError, "tilec fastcall: install() was not called");
    return NULL;
  }
  void* p[3];
  int64_t d[6];
  tilec_mm_cfg cfg;
  if (parse_problem(args, p, d, &cfg)) return NULL;
  void* ws = NULL;
  void* stream = NULL;
  int64_t ws_bytes = 0;
  if (as_ptr(args[12], &ws) || as_i64(args[13], &ws_bytes) || as_ptr(args[14], &stream)) return NULL;
  if (ws_bytes < 0) {
    PyErr_SetString(PyExc_ValueError, "mm: negative workspace size");
    return NULL;
  }
  int rc;
  /* The GIL is released around the launch, as ctypes does, so other host threads run. */
  Py_BEGIN_ALLOW_THREADS
  rc = g_mm((const float*)p[0], (const float*)p[1], (float*)p[2], d[0], d[1], d[2], d[3], d[4], d[5], &cfg, ws,
            (size_t)ws_bytes, stream);
  Py_END_ALLOW_THREADS
  return PyLong_FromLong(rc);
}

static PyObject* py_ws_bytes(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  if (nargs != 12) {
    PyErr_SetString(PyExc_TypeError, "ws_bytes() takes 12 arguments");
    return NULL;
  }
  if (g_ws == NULL) {
    PyErr_SetString(PyExc_RuntimeError, "tilec fastcall: install() was not called");
    return NULL;
  }
  void* p[3];
  int64_t d[6];
  tilec_mm_cfg cfg;
  if (parse_problem(args, p, d, &cfg)) return NULL;
  const size_t n = g_ws((const float*)p[0], (const float*)p[1], (const float*)p[2], d[0], d[1], d[2], d[3], d[4],
                        d[5], &cfg);
  return PyLong_FromSize_t(n);
}

static PyMethodDef kMethods[] = {
    {"install", (PyCFunction)(void (*)(void))py_install, METH_FASTCALL, "install(addr_mm_f32, addr_workspace_bytes)"},
    {"mm", (PyCFunction)(void (*)(void))py_mm, METH_FASTCALL,
     "mm(a, b, c, M, N, K, lda, ldb, ldc, variant, split_k, flags, ws, ws_bytes, stream) -> status"},
    {"ws_bytes", (PyCFunction)(void (*)(void))py_ws_bytes, METH_FASTCALL,
     "ws_bytes(a, b, c, M, N, K, lda, ldb, ldc, variant, split_k, flags) -> bytes"},
    {NULL, NULL, 0, NULL},
};

static struct PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_tilec_fast", NULL, -1, kMethods, NULL, NULL, NULL, NULL};

PyMODINIT_FUNC PyInit__tilec_fast(void) { return PyModule_Create(&kModule); }
