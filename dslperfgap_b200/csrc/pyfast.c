/* pyfast.c — a CPython extension (`_dslpg_fast`) exposing the per-call entry
 * points of libdslpg_b200.so with METH_FASTCALL argument parsing, so a call
 * from the Python wrappers costs a few hundred nanoseconds of binding instead
 * of ctypes' per-argument conversions. Each function has the C entry point's
 * name and takes its arguments in order (device pointers and the stream as
 * Python ints, floats as Python floats) and returns its int status; the
 * wrappers raise on a non-zero status. ctypes binds the rest of the ABI.
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <string.h>

#include "dslpg_b200.h"

typedef union {
  void* p;
  int64_t l;
  int i;
  float f;
} Arg;

/* Parse `n` arguments by `spec`: p = pointer, l = int64, i = int, f = float. */
static int parse(PyObject* const* a, Py_ssize_t n, const char* spec, Arg* out, const char* name) {
  const Py_ssize_t want = (Py_ssize_t)strlen(spec);
  if (n != want) {
    PyErr_Format(PyExc_TypeError, "%s: expected %zd arguments, got %zd", name, want, n);
    return 0;
  }
  for (Py_ssize_t k = 0; k < n; ++k) {
    switch (spec[k]) {
      case 'p':
        out[k].p = a[k] == Py_None ? NULL : PyLong_AsVoidPtr(a[k]);
        break;
      case 'l':
        out[k].l = (int64_t)PyLong_AsLongLong(a[k]);
        break;
      case 'i':
        out[k].i = (int)PyLong_AsLong(a[k]);
        break;
      case 'f':
        out[k].f = (float)PyFloat_AsDouble(a[k]);
        break;
      default:
        PyErr_Format(PyExc_SystemError, "%s: bad argument spec", name);
        return 0;
    }
    if (PyErr_Occurred()) return 0;
  }
  return 1;
}

#define STREAM(v) ((cudaStream_t)(v).p)
#define ENTRY(fname, spec, call)                                             \
  static PyObject* w_##fname(PyObject* self, PyObject* const* a, Py_ssize_t n) { \
    Arg v[32];                                                               \
    (void)self;                                                              \
    if (!parse(a, n, spec, v, #fname)) return NULL;                          \
    return PyLong_FromLong(call);                                            \
  }

ENTRY(dslpg_layer_norm_fwd, "ppppllllfp",
      dslpg_layer_norm_fwd(v[0].p, v[1].p, v[2].p, v[3].p, v[4].l, v[5].l, (int)v[6].l, (int)v[7].l, v[8].f,
                           STREAM(v[9])))
ENTRY(dslpg_rms_norm_fwd, "pppllllfp",
      dslpg_rms_norm_fwd(v[0].p, v[1].p, v[2].p, v[3].l, v[4].l, (int)v[5].l, (int)v[6].l, v[7].f, STREAM(v[8])))
ENTRY(dslpg_softmax_fwd, "ppllip", dslpg_softmax_fwd(v[0].p, v[1].p, v[2].l, v[3].l, v[4].i, STREAM(v[5])))
ENTRY(dslpg_log_softmax_fwd, "pplllllp",
      dslpg_log_softmax_fwd(v[0].p, v[1].p, v[2].l, v[3].l, v[4].l, (int)v[5].l, (int)v[6].l, STREAM(v[7])))
ENTRY(dslpg_logsumexp_fwd, "ppllip", dslpg_logsumexp_fwd(v[0].p, v[1].p, v[2].l, v[3].l, v[4].i, STREAM(v[5])))
ENTRY(dslpg_cross_entropy_fwd, "ppppplllllffflfllllp",
      dslpg_cross_entropy_fwd(v[0].p, v[1].p, (float*)v[2].p, (float*)v[3].p, (float*)v[4].p, v[5].l, v[6].l, v[7].l,
                              (int)v[8].l, (int)v[9].l, v[10].f, v[11].f, v[12].f, v[13].l, v[14].f, v[15].l, v[16].l,
                              (int)v[17].l, (int)v[18].l, STREAM(v[19])))
ENTRY(dslpg_cross_entropy_bwd, "pllppppllllllffflfllp",
      dslpg_cross_entropy_bwd(v[0].p, (int)v[1].l, v[2].l, v[3].p, (const float*)v[4].p, v[5].p, v[6].p, v[7].l,
                              v[8].l, v[9].l, v[10].l, (int)v[11].l, (int)v[12].l, v[13].f, v[14].f, v[15].f, v[16].l,
                              v[17].f, v[18].l, (int)v[19].l, STREAM(v[20])))
ENTRY(dslpg_cross_entropy_fwd_bwd, "ppplpppppllllllffflfllp",
      dslpg_cross_entropy_fwd_bwd(v[0].p, v[1].p, v[2].p, (int)v[3].l, v[4].l, (float*)v[5].p, (float*)v[6].p,
                                  (float*)v[7].p, v[8].p, v[9].l, v[10].l, v[11].l, v[12].l, (int)v[13].l,
                                  (int)v[14].l, v[15].f, v[16].f, v[17].f, v[18].l, v[19].f, v[20].l, (int)v[21].l,
                                  STREAM(v[22])))
ENTRY(dslpg_mean_reduction, "pplllllp",
      dslpg_mean_reduction(v[0].p, v[1].p, v[2].l, v[3].l, v[4].l, (int)v[5].l, (int)v[6].l, STREAM(v[7])))
ENTRY(dslpg_max_reduction, "ppplllip",
      dslpg_max_reduction(v[0].p, v[1].p, (int64_t*)v[2].p, v[3].l, v[4].l, v[5].l, v[6].i, STREAM(v[7])))
ENTRY(dslpg_argmax, "pplllip", dslpg_argmax(v[0].p, (int64_t*)v[1].p, v[2].l, v[3].l, v[4].l, v[5].i, STREAM(v[6])))
ENTRY(dslpg_kernel_ff, "ppppplllplp",
      dslpg_kernel_ff(v[0].p, v[1].p, v[2].p, v[3].p, v[4].p, v[5].l, v[6].l, v[7].l, v[8].p, v[9].l, STREAM(v[10])))

#define M(fname) {#fname, (PyCFunction)(void (*)(void))w_##fname, METH_FASTCALL, NULL}
static PyMethodDef methods[] = {
    M(dslpg_layer_norm_fwd), M(dslpg_rms_norm_fwd),      M(dslpg_softmax_fwd),
    M(dslpg_log_softmax_fwd), M(dslpg_logsumexp_fwd),    M(dslpg_cross_entropy_fwd),
    M(dslpg_cross_entropy_bwd), M(dslpg_mean_reduction), M(dslpg_max_reduction),
    M(dslpg_argmax),          M(dslpg_kernel_ff),        M(dslpg_cross_entropy_fwd_bwd),
    {NULL, NULL, 0, NULL}};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_dslpg_fast",
                                    "METH_FASTCALL bindings of libdslpg_b200's per-call entry points", -1, methods,
                                    NULL, NULL, NULL, NULL};

PyMODINIT_FUNC PyInit__dslpg_fast(void) { return PyModule_Create(&module); }
