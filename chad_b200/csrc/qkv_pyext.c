/*
 * chad_b200._qkvext: CPython bindings of the per-layer entry points of libqkv.so.
 *
 * The same C ABI as the ctypes table in chad_b200/_lib.py, called with the prototypes of
 * include/qkv.h through function pointers bound at load time to the library instance the
 * process loaded (bind(name, address)). ctypes converts its ~30 arguments per call in about
 * 8 us, which is most of a decode layer's host time; parsing them here costs well under
 * 1 us. Arguments: device pointers and streams as Python ints (0 or None for NULL), the
 * rest as ints, one float (the softmax scale).
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>
#include <string.h>

#include "../../include/qkv.h"

static __typeof__(&qkv_attention) p_attention;
static __typeof__(&qkv_prefill) p_prefill;
static __typeof__(&qkv_quantize_append_kv) p_append_kv;
static __typeof__(&qkv_combine) p_combine;
static __typeof__(&qkv_gather_combine) p_gather_combine;

typedef union {
  void* p;
  long long l;
  int i;
  float f;
  size_t z;
} Arg;

/* fmt: one letter per argument. p pointer (int or None), i int, l long long, z size_t,
 * f float. */
static int parse(PyObject* const* args, Py_ssize_t n, const char* fmt, Arg* out) {
  const Py_ssize_t k = (Py_ssize_t)strlen(fmt);
  if (n != k) {
    PyErr_Format(PyExc_TypeError, "expected %zd arguments, got %zd", k, n);
    return -1;
  }
  for (Py_ssize_t j = 0; j < k; ++j) {
    PyObject* o = args[j];
    switch (fmt[j]) {
      case 'p':
        if (o == Py_None) {
          out[j].p = NULL;
        } else {
          const unsigned long long v = PyLong_AsUnsignedLongLong(o);
          if (v == (unsigned long long)-1 && PyErr_Occurred()) return -1;
          out[j].p = (void*)(uintptr_t)v;
        }
        break;
      case 'i': {
        const long v = PyLong_AsLong(o);
        if (v == -1 && PyErr_Occurred()) return -1;
        if (v < INT32_MIN || v > INT32_MAX) {
          PyErr_Format(PyExc_OverflowError, "argument %zd out of int range", j);
          return -1;
        }
        out[j].i = (int)v;
        break;
      }
      case 'l': {
        const long long v = PyLong_AsLongLong(o);
        if (v == -1 && PyErr_Occurred()) return -1;
        out[j].l = v;
        break;
      }
      case 'z': {
        const unsigned long long v = PyLong_AsUnsignedLongLong(o);
        if (v == (unsigned long long)-1 && PyErr_Occurred()) return -1;
        out[j].z = (size_t)v;
        break;
      }
      case 'f': {
        const double v = PyFloat_AsDouble(o);
        if (v == -1.0 && PyErr_Occurred()) return -1;
        out[j].f = (float)v;
        break;
      }
      default:
        PyErr_SetString(PyExc_SystemError, "bad argument format");
        return -1;
    }
  }
  return 0;
}

static int unbound(const char* name) {
  PyErr_Format(PyExc_RuntimeError, "%s is not bound to libqkv.so", name);
  return -1;
}

static PyObject* w_attention(PyObject* self, PyObject* const* args, Py_ssize_t n) {
  Arg a[33];
  (void)self;
  if (!p_attention) return unbound("qkv_attention"), NULL;
  if (parse(args, n, "pppppppp" "iiiiiii" "ppp" "iiif" "ipilll" "iipzp", a)) return NULL;
  const int rc = p_attention(a[0].p, a[1].p, a[2].p, a[3].p, a[4].p, a[5].p, a[6].p, a[7].p,
                             a[8].i, a[9].i, a[10].i, a[11].i, a[12].i, a[13].i, a[14].i,
                             (const int*)a[15].p, (const int*)a[16].p, (const int*)a[17].p,
                             a[18].i, a[19].i, a[20].i, a[21].f, a[22].i, a[23].p, a[24].i,
                             a[25].l, a[26].l, a[27].l, a[28].i, a[29].i, a[30].p, a[31].z,
                             a[32].p);
  return PyLong_FromLong(rc);
}

static PyObject* w_prefill(PyObject* self, PyObject* const* args, Py_ssize_t n) {
  Arg a[24];
  (void)self;
  if (!p_prefill) return unbound("qkv_prefill"), NULL;
  if (parse(args, n, "pppppppppp" "iiiiiiiiii" "f" "pzp", a)) return NULL;
  const int rc = p_prefill(a[0].p, a[1].p, a[2].p, a[3].p, a[4].p, a[5].p, a[6].p, a[7].p,
                           a[8].p, a[9].p, a[10].i, a[11].i, a[12].i, a[13].i, a[14].i,
                           a[15].i, a[16].i, a[17].i, a[18].i, a[19].i, a[20].f, a[21].p,
                           a[22].z, a[23].p);
  return PyLong_FromLong(rc);
}

static PyObject* w_append_kv(PyObject* self, PyObject* const* args, Py_ssize_t n) {
  Arg a[19];
  (void)self;
  if (!p_append_kv) return unbound("qkv_quantize_append_kv"), NULL;
  if (parse(args, n, "ppi" "pppppp" "iiiiiiiii" "p", a)) return NULL;
  const int rc = p_append_kv(a[0].p, a[1].p, a[2].i, a[3].p, a[4].p, a[5].p, a[6].p, a[7].p,
                             a[8].p, a[9].i, a[10].i, a[11].i, a[12].i, a[13].i, a[14].i,
                             a[15].i, a[16].i, a[17].i, a[18].p);
  return PyLong_FromLong(rc);
}

static PyObject* w_combine(PyObject* self, PyObject* const* args, Py_ssize_t n) {
  Arg a[8];
  (void)self;
  if (!p_combine) return unbound("qkv_combine"), NULL;
  if (parse(args, n, "pilipiip", a)) return NULL;
  const int rc = p_combine((const float*)a[0].p, a[1].i, a[2].l, a[3].i, a[4].p, a[5].i,
                           a[6].i, a[7].p);
  return PyLong_FromLong(rc);
}

static PyObject* w_gather_combine(PyObject* self, PyObject* const* args, Py_ssize_t n) {
  Arg a[11];
  (void)self;
  if (!p_gather_combine) return unbound("qkv_gather_combine"), NULL;
  if (parse(args, n, "pli" "pp" "ii" "piip", a)) return NULL;
  const int rc = p_gather_combine((const float*)a[0].p, a[1].l, a[2].i, (void* const*)a[3].p,
                                  a[4].p, a[5].i, a[6].i, a[7].p, a[8].i, a[9].i, a[10].p);
  return PyLong_FromLong(rc);
}

/* bind(name, address): point the wrapper of `name` at the loaded library's symbol */
static PyObject* w_bind(PyObject* self, PyObject* args) {
  const char* name;
  unsigned long long addr;
  (void)self;
  if (!PyArg_ParseTuple(args, "sK", &name, &addr)) return NULL;
  void* f = (void*)(uintptr_t)addr;
  if (!strcmp(name, "qkv_attention")) p_attention = (__typeof__(p_attention))f;
  else if (!strcmp(name, "qkv_prefill")) p_prefill = (__typeof__(p_prefill))f;
  else if (!strcmp(name, "qkv_quantize_append_kv")) p_append_kv = (__typeof__(p_append_kv))f;
  else if (!strcmp(name, "qkv_combine")) p_combine = (__typeof__(p_combine))f;
  else if (!strcmp(name, "qkv_gather_combine")) p_gather_combine = (__typeof__(p_gather_combine))f;
  else return PyErr_Format(PyExc_KeyError, "no binding for %s", name);
  Py_RETURN_NONE;
}

static PyMethodDef methods[] = {
    {"bind", (PyCFunction)w_bind, METH_VARARGS, "bind(name, address)"},
    {"attention", (PyCFunction)(void (*)(void))w_attention, METH_FASTCALL, "qkv_attention"},
    {"prefill", (PyCFunction)(void (*)(void))w_prefill, METH_FASTCALL, "qkv_prefill"},
    {"quantize_append_kv", (PyCFunction)(void (*)(void))w_append_kv, METH_FASTCALL,
     "qkv_quantize_append_kv"},
    {"combine", (PyCFunction)(void (*)(void))w_combine, METH_FASTCALL, "qkv_combine"},
    {"gather_combine", (PyCFunction)(void (*)(void))w_gather_combine, METH_FASTCALL,
     "qkv_gather_combine"},
    {NULL, NULL, 0, NULL}};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_qkvext", NULL, -1, methods,
                                    NULL, NULL, NULL, NULL};

PyMODINIT_FUNC PyInit__qkvext(void) { return PyModule_Create(&module); }
