/* fastcall.c -- a CPython binding of the prefill entry point of libb200attn.so.
 *
 * b200attn.attention calls the C-ABI through ctypes; converting its fifteen
 * arguments costs a few microseconds per call, which is as much as the kernel
 * launch itself and dominates small prefill calls.  This module parses the
 * same arguments with PyArg_ParseTuple and calls the same exported function
 * (b2a_prefill_fwd_kv), so both routes run identical library code.
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>

#include "../../include/b200attn.h"

/* prefill_fwd_kv(q, k, v, o, lse, B, H, Hkv, N, Nk, D, dtype, causal, scale, stream) -> status
 * pointers and the stream are integers (lse may be 0 for the O-only path). */
static PyObject* prefill_fwd_kv(PyObject* self, PyObject* args) {
  unsigned long long q, k, v, o, lse, stream;
  int B, H, Hkv, N, Nk, D, dtype, causal;
  float scale;
  (void)self;
  if (!PyArg_ParseTuple(args, "KKKKKiiiiiiiifK", &q, &k, &v, &o, &lse, &B, &H, &Hkv, &N, &Nk, &D,
                        &dtype, &causal, &scale, &stream))
    return NULL;
  const int rc = b2a_prefill_fwd_kv((const void*)(uintptr_t)q, (const void*)(uintptr_t)k,
                                    (const void*)(uintptr_t)v, (void*)(uintptr_t)o,
                                    (float*)(uintptr_t)lse, B, H, Hkv, N, Nk, D, dtype, causal,
                                    scale, (void*)(uintptr_t)stream);
  return PyLong_FromLong(rc);
}

static PyMethodDef kMethods[] = {
    {"prefill_fwd_kv", prefill_fwd_kv, METH_VARARGS,
     "b2a_prefill_fwd_kv(q, k, v, o, lse, B, H, Hkv, N, Nk, D, dtype, causal, scale, stream)"},
    {NULL, NULL, 0, NULL}};

static struct PyModuleDef kModule = {PyModuleDef_HEAD_INIT, "_fastcall",
                                     "CPython binding of b2a_prefill_fwd_kv", -1, kMethods};

PyMODINIT_FUNC PyInit__fastcall(void) { return PyModule_Create(&kModule); }
