/*
 * chol_pyext.c — CPython fast-call binding of the hot C-ABI entry point, used by the
 * Python drop-in (linalg_kernels_b200/cholesky.py) instead of ctypes: one call with eight
 * integer arguments costs ~0.3 us here against several us of ctypes marshalling, which
 * matters when a whole batch of n = 32 matrices factors in ~10 us.
 *
 *   potrf_ws(A, L, batch, n, info, ws, ws_bytes, queue) -> status
 *     all arguments are Python ints (device addresses, sizes; 0 for NULL)
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>

#include "../../include/chol_b200.h"

static PyObject* potrf_ws(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  if (nargs != 8) {
    PyErr_SetString(PyExc_TypeError, "potrf_ws expects 8 integer arguments");
    return NULL;
  }
  unsigned long long v[8];
  for (int i = 0; i < 8; ++i) {
    v[i] = PyLong_AsUnsignedLongLongMask(args[i]);
    if (v[i] == (unsigned long long)-1 && PyErr_Occurred()) return NULL;
  }
  int st = chol_potrf_batched_ws_f32((const float*)(uintptr_t)v[0], (float*)(uintptr_t)v[1],
                                     (int64_t)v[2], (int64_t)v[3], (int*)(uintptr_t)v[4],
                                     (void*)(uintptr_t)v[5], (size_t)v[6], (void*)(uintptr_t)v[7]);
  return PyLong_FromLong(st);
}

static PyMethodDef methods[] = {
    {"potrf_ws", (PyCFunction)(void (*)(void))potrf_ws, METH_FASTCALL,
     "chol_potrf_batched_ws_f32 with integer arguments"},
    {NULL, NULL, 0, NULL}};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_cholpy", NULL, -1, methods};

PyMODINIT_FUNC PyInit__cholpy(void) { return PyModule_Create(&module); }
