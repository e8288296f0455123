/* kvs_fastcall.c -- CPython entry points for the per-call hot path of the Python facade.
 *
 * Client.get_blocks / put_blocks / exists_batch on one or a few blocks are latency-bound: through
 * ctypes each call pays for argument conversion (a few hundred ns per pointer) on top of the C ABI
 * call itself. The reference binds its client to Python with a compiled module (nanobind,
 * src/python/bindings.cpp); this module plays that part for these three calls. It calls the
 * functions of libkvs_b200.so through pointers that the package hands over once (bind), so both
 * the ctypes binding and this module use the one loaded library.
 *
 * Each call takes its arrays through the buffer protocol, exactly typed (keys: 8-byte unsigned,
 * block ids: 8-byte signed, one dimension, C-contiguous); anything else returns NotImplemented and
 * the facade converts it and takes its ctypes path. A failing C ABI call returns its error code as
 * an int (the facade raises KvsError with the library's message); success returns the result. The
 * GIL is released around every C ABI call, as ctypes does. */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#define NPY_NO_DEPRECATED_API NPY_1_7_API_VERSION
#include <numpy/arrayobject.h>

#include <stdint.h>
#include <string.h>

typedef int (*put_blocks_fn)(void *, const void *, uint32_t, const uint64_t *, const int64_t *, int, void *);
typedef int (*get_blocks_fn)(void *, const void *, uint32_t, const uint64_t *, const int64_t *, uint8_t *, void *);
typedef int (*exists_batch_fn)(void *, uint32_t, const uint64_t *, uint8_t *);

static put_blocks_fn g_put_blocks;
static get_blocks_fn g_get_blocks;
static exists_batch_fn g_exists_batch;

/* 1-D, C-contiguous, 8-byte items of the wanted signedness ('Q'/'L' unsigned, 'q'/'l' signed). */
static int take_u64_or_i64(PyObject *o, Py_buffer *view, int want_signed) {
  if (!PyObject_CheckBuffer(o)) return 0;
  if (PyObject_GetBuffer(o, view, PyBUF_C_CONTIGUOUS | PyBUF_FORMAT) != 0) {
    PyErr_Clear();
    return 0;
  }
  const char *f = view->format ? view->format : "B";
  if (*f == '<' || *f == '=' || *f == '@') ++f;
  const int ok = view->ndim == 1 && view->itemsize == 8 && f[1] == '\0' &&
                 (want_signed ? (f[0] == 'q' || f[0] == 'l') : (f[0] == 'Q' || f[0] == 'L'));
  if (!ok) {
    PyBuffer_Release(view);
    return 0;
  }
  return 1;
}

static PyObject *bind(PyObject *self, PyObject *args) {
  unsigned long long put, get, exists;
  if (!PyArg_ParseTuple(args, "KKK", &put, &get, &exists)) return NULL;
  g_put_blocks = (put_blocks_fn)(uintptr_t)put;
  g_get_blocks = (get_blocks_fn)(uintptr_t)get;
  g_exists_batch = (exists_batch_fn)(uintptr_t)exists;
  Py_RETURN_NONE;
}

/* get_blocks(client, layout, keys, block_ids, stream) -> found (bool ndarray) | rc | NotImplemented */
static PyObject *get_blocks(PyObject *self, PyObject *const *args, Py_ssize_t nargs) {
  if (nargs != 5) {
    PyErr_SetString(PyExc_TypeError, "get_blocks takes 5 arguments");
    return NULL;
  }
  if (!g_get_blocks) Py_RETURN_NOTIMPLEMENTED;
  void *client = PyLong_AsVoidPtr(args[0]);
  const void *layout = PyLong_AsVoidPtr(args[1]);
  void *stream = PyLong_AsVoidPtr(args[4]);
  if (PyErr_Occurred()) return NULL;
  Py_buffer k, b;
  if (!take_u64_or_i64(args[2], &k, 0)) Py_RETURN_NOTIMPLEMENTED;
  if (!take_u64_or_i64(args[3], &b, 1)) {
    PyBuffer_Release(&k);
    Py_RETURN_NOTIMPLEMENTED;
  }
  const Py_ssize_t n = k.shape ? k.shape[0] : k.len / 8;
  if ((b.shape ? b.shape[0] : b.len / 8) != n || n > (Py_ssize_t)UINT32_MAX) {
    PyBuffer_Release(&k);
    PyBuffer_Release(&b);
    Py_RETURN_NOTIMPLEMENTED; /* the facade reports the mismatch */
  }
  npy_intp dims[1] = {(npy_intp)n};
  PyObject *found = PyArray_SimpleNew(1, dims, NPY_BOOL);
  if (!found) {
    PyBuffer_Release(&k);
    PyBuffer_Release(&b);
    return NULL;
  }
  uint8_t *fp = (uint8_t *)PyArray_DATA((PyArrayObject *)found);
  if (n) memset(fp, 0, (size_t)n);
  int rc;
  Py_BEGIN_ALLOW_THREADS
  rc = g_get_blocks(client, layout, (uint32_t)n, (const uint64_t *)k.buf, (const int64_t *)b.buf, fp, stream);
  Py_END_ALLOW_THREADS
  PyBuffer_Release(&k);
  PyBuffer_Release(&b);
  if (rc != 0) {
    Py_DECREF(found);
    return PyLong_FromLong(rc);
  }
  return found;
}

/* put_blocks(client, layout, keys, block_ids, sync_commit, stream) -> 0 | rc | NotImplemented */
static PyObject *put_blocks(PyObject *self, PyObject *const *args, Py_ssize_t nargs) {
  if (nargs != 6) {
    PyErr_SetString(PyExc_TypeError, "put_blocks takes 6 arguments");
    return NULL;
  }
  if (!g_put_blocks) Py_RETURN_NOTIMPLEMENTED;
  void *client = PyLong_AsVoidPtr(args[0]);
  const void *layout = PyLong_AsVoidPtr(args[1]);
  const int sync_commit = PyObject_IsTrue(args[4]);
  if (sync_commit < 0) return NULL;
  void *stream = PyLong_AsVoidPtr(args[5]);
  if (PyErr_Occurred()) return NULL;
  Py_buffer k, b;
  if (!take_u64_or_i64(args[2], &k, 0)) Py_RETURN_NOTIMPLEMENTED;
  if (!take_u64_or_i64(args[3], &b, 1)) {
    PyBuffer_Release(&k);
    Py_RETURN_NOTIMPLEMENTED;
  }
  const Py_ssize_t n = k.shape ? k.shape[0] : k.len / 8;
  if ((b.shape ? b.shape[0] : b.len / 8) != n || n > (Py_ssize_t)UINT32_MAX) {
    PyBuffer_Release(&k);
    PyBuffer_Release(&b);
    Py_RETURN_NOTIMPLEMENTED;
  }
  int rc;
  Py_BEGIN_ALLOW_THREADS
  rc = g_put_blocks(client, layout, (uint32_t)n, (const uint64_t *)k.buf, (const int64_t *)b.buf, sync_commit, stream);
  Py_END_ALLOW_THREADS
  PyBuffer_Release(&k);
  PyBuffer_Release(&b);
  return PyLong_FromLong(rc);
}

/* exists_batch(client, keys) -> found (bool ndarray) | rc | NotImplemented */
static PyObject *exists_batch(PyObject *self, PyObject *const *args, Py_ssize_t nargs) {
  if (nargs != 2) {
    PyErr_SetString(PyExc_TypeError, "exists_batch takes 2 arguments");
    return NULL;
  }
  if (!g_exists_batch) Py_RETURN_NOTIMPLEMENTED;
  void *client = PyLong_AsVoidPtr(args[0]);
  if (PyErr_Occurred()) return NULL;
  Py_buffer k;
  if (!take_u64_or_i64(args[1], &k, 0)) Py_RETURN_NOTIMPLEMENTED;
  const Py_ssize_t n = k.shape ? k.shape[0] : k.len / 8;
  if (n > (Py_ssize_t)UINT32_MAX) {
    PyBuffer_Release(&k);
    Py_RETURN_NOTIMPLEMENTED;
  }
  npy_intp dims[1] = {(npy_intp)n};
  PyObject *found = PyArray_SimpleNew(1, dims, NPY_BOOL);
  if (!found) {
    PyBuffer_Release(&k);
    return NULL;
  }
  uint8_t *fp = (uint8_t *)PyArray_DATA((PyArrayObject *)found);
  if (n) memset(fp, 0, (size_t)n);
  int rc;
  Py_BEGIN_ALLOW_THREADS
  rc = g_exists_batch(client, (uint32_t)n, (const uint64_t *)k.buf, fp);
  Py_END_ALLOW_THREADS
  PyBuffer_Release(&k);
  if (rc != 0) {
    Py_DECREF(found);
    return PyLong_FromLong(rc);
  }
  return found;
}

static PyMethodDef methods[] = {
    {"bind", bind, METH_VARARGS, "bind(put_blocks, get_blocks, exists_batch): C ABI function addresses"},
    {"get_blocks", (PyCFunction)(void (*)(void))get_blocks, METH_FASTCALL,
     "get_blocks(client, layout, keys, block_ids, stream) -> found | rc | NotImplemented"},
    {"put_blocks", (PyCFunction)(void (*)(void))put_blocks, METH_FASTCALL,
     "put_blocks(client, layout, keys, block_ids, sync_commit, stream) -> rc | NotImplemented"},
    {"exists_batch", (PyCFunction)(void (*)(void))exists_batch, METH_FASTCALL,
     "exists_batch(client, keys) -> found | rc | NotImplemented"},
    {NULL, NULL, 0, NULL},
};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_fastcall",
                                    "CPython entry points of the block calls (see kvs_fastcall.c)", -1, methods};

PyMODINIT_FUNC PyInit__fastcall(void) {
  import_array();
  return PyModule_Create(&module);
}
