/*
 * _hostpack: native packing of one step's host metadata.
 *
 * Reads Tokquay Sequence objects (any object with num_cached_tokens,
 * block_table, prompt_token_ids and output_token_ids; the reference's
 * tokquay/sequence.py:34-81 contract) and writes the int32 arrays
 * tq_plan_step takes: start[B], q_len[B], table_offsets[B+1],
 * table_data[sum of table lengths] and token_ids[sum of q_len].  The Python
 * equivalent walks every block id and token id through the interpreter; this
 * walks the lists' items in C.
 *
 *   pack_step(seqs, new_lens or None) -> (starts, lens, offsets, tables, ids)
 *
 * Each result is a bytearray of int32 (native byte order) of exactly the
 * array's length (ids holds the tokens of rows with q_len >= 1).  new_lens None
 * means each sequence feeds all its uncached tokens, as in
 * tokquay/kv_cache.py:122-127.
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>
#include <string.h>

static int get_long_attr(PyObject* o, PyObject* name, long* out) {
  PyObject* v = PyObject_GetAttr(o, name);
  if (!v) return -1;
  *out = PyLong_AsLong(v);
  Py_DECREF(v);
  return (*out == -1 && PyErr_Occurred()) ? -1 : 0;
}

/* Borrowed list attribute; caller must Py_DECREF the returned object. */
static PyObject* get_list_attr(PyObject* o, PyObject* name) {
  PyObject* v = PyObject_GetAttr(o, name);
  if (v && !PyList_Check(v)) {
    PyErr_Format(PyExc_TypeError, "%U must be a list", name);
    Py_DECREF(v);
    return NULL;
  }
  return v;
}

static int put_ints(PyObject* list, Py_ssize_t begin, Py_ssize_t end, int32_t* dst) {
  for (Py_ssize_t i = begin; i < end; ++i) {
    long v = PyLong_AsLong(PyList_GET_ITEM(list, i));
    if (v == -1 && PyErr_Occurred()) return -1;
    if (v < INT32_MIN || v > INT32_MAX) {
      PyErr_SetString(PyExc_OverflowError, "value does not fit int32");
      return -1;
    }
    *dst++ = (int32_t)v;
  }
  return 0;
}

static PyObject* pack_step(PyObject* self, PyObject* args) {
  (void)self;
  PyObject *seqs, *new_lens;
  if (!PyArg_ParseTuple(args, "OO", &seqs, &new_lens)) return NULL;
  PyObject* seq_fast = PySequence_Fast(seqs, "seqs must be a sequence");
  if (!seq_fast) return NULL;
  PyObject* lens_fast = NULL;
  const Py_ssize_t B = PySequence_Fast_GET_SIZE(seq_fast);
  if (new_lens != Py_None) {
    lens_fast = PySequence_Fast(new_lens, "new_lens must be a sequence");
    if (!lens_fast) goto fail0;
    if (PySequence_Fast_GET_SIZE(lens_fast) != B) {
      PyErr_SetString(PyExc_ValueError, "block_tables, start and new_lens must be non-empty and the same length");
      goto fail0;
    }
  }
  PyObject* s_cached = PyUnicode_InternFromString("num_cached_tokens");
  PyObject* s_table = PyUnicode_InternFromString("block_table");
  PyObject* s_prompt = PyUnicode_InternFromString("prompt_token_ids");
  PyObject* s_output = PyUnicode_InternFromString("output_token_ids");
  PyObject *starts = NULL, *lens = NULL, *offs = NULL, *tables = NULL, *ids = NULL, *result = NULL;
  if (!s_cached || !s_table || !s_prompt || !s_output) goto fail1;

  /* Pass 1: sizes. */
  Py_ssize_t n_tab = 0, n_tok = 0;
  starts = PyByteArray_FromStringAndSize(NULL, B * 4);
  lens = PyByteArray_FromStringAndSize(NULL, B * 4);
  offs = PyByteArray_FromStringAndSize(NULL, (B + 1) * 4);
  if (!starts || !lens || !offs) goto fail1;
  int32_t* st = (int32_t*)PyByteArray_AS_STRING(starts);
  int32_t* ln = (int32_t*)PyByteArray_AS_STRING(lens);
  int32_t* of = (int32_t*)PyByteArray_AS_STRING(offs);
  of[0] = 0;
  for (Py_ssize_t b = 0; b < B; ++b) {
    PyObject* s = PySequence_Fast_GET_ITEM(seq_fast, b);
    long cached;
    if (get_long_attr(s, s_cached, &cached) < 0) goto fail1;
    PyObject* tbl = get_list_attr(s, s_table);
    if (!tbl) goto fail1;
    const Py_ssize_t nt = PyList_GET_SIZE(tbl);
    Py_DECREF(tbl);
    long n;
    if (lens_fast) {
      n = PyLong_AsLong(PySequence_Fast_GET_ITEM(lens_fast, b));
      if (n == -1 && PyErr_Occurred()) goto fail1;
    } else {
      PyObject* pr = get_list_attr(s, s_prompt);
      if (!pr) goto fail1;
      PyObject* ou = get_list_attr(s, s_output);
      if (!ou) {
        Py_DECREF(pr);
        goto fail1;
      }
      n = (long)(PyList_GET_SIZE(pr) + PyList_GET_SIZE(ou)) - cached;
      Py_DECREF(pr);
      Py_DECREF(ou);
    }
    st[b] = (int32_t)cached;
    ln[b] = (int32_t)n;
    n_tab += nt;
    if (n > 0) n_tok += n;
    if (n_tab > INT32_MAX || n_tok > INT32_MAX) {
      PyErr_SetString(PyExc_OverflowError, "step too large");
      goto fail1;
    }
    of[b + 1] = (int32_t)n_tab;
  }

  /* Pass 2: block ids and token ids. */
  tables = PyByteArray_FromStringAndSize(NULL, n_tab * 4);
  ids = PyByteArray_FromStringAndSize(NULL, n_tok * 4);
  if (!tables || !ids) goto fail1;
  int32_t* tb = (int32_t*)PyByteArray_AS_STRING(tables);
  int32_t* id = (int32_t*)PyByteArray_AS_STRING(ids);
  for (Py_ssize_t b = 0; b < B; ++b) {
    PyObject* s = PySequence_Fast_GET_ITEM(seq_fast, b);
    PyObject* tbl = get_list_attr(s, s_table);
    if (!tbl) goto fail1;
    int rc = put_ints(tbl, 0, PyList_GET_SIZE(tbl), tb + of[b]);
    Py_DECREF(tbl);
    if (rc < 0) goto fail1;
    const long begin = st[b], n = ln[b];
    if (n <= 0 || begin < 0) continue; /* the planner rejects these with the reference's message */
    PyObject* pr = get_list_attr(s, s_prompt);
    if (!pr) goto fail1;
    PyObject* ou = get_list_attr(s, s_output);
    if (!ou) {
      Py_DECREF(pr);
      goto fail1;
    }
    const Py_ssize_t np_ = PyList_GET_SIZE(pr), no = PyList_GET_SIZE(ou);
    const Py_ssize_t end = begin + n;
    if (end > np_ + no) {
      Py_DECREF(pr);
      Py_DECREF(ou);
      PyErr_SetString(PyExc_ValueError, "a sequence feeds more tokens than it has");
      goto fail1;
    }
    /* tokens [begin, end) of prompt + output */
    rc = 0;
    if (begin < np_) rc = put_ints(pr, begin, end < np_ ? end : np_, id);
    if (rc == 0 && end > np_)
      rc = put_ints(ou, begin > np_ ? begin - np_ : 0, end - np_, id + (begin < np_ ? np_ - begin : 0));
    id += n;
    Py_DECREF(pr);
    Py_DECREF(ou);
    if (rc < 0) goto fail1;
  }
  result = PyTuple_Pack(5, starts, lens, offs, tables, ids);
fail1:
  Py_XDECREF(starts);
  Py_XDECREF(lens);
  Py_XDECREF(offs);
  Py_XDECREF(tables);
  Py_XDECREF(ids);
  Py_XDECREF(s_cached);
  Py_XDECREF(s_table);
  Py_XDECREF(s_prompt);
  Py_XDECREF(s_output);
fail0:
  Py_XDECREF(lens_fast);
  Py_DECREF(seq_fast);
  return result;
}

static PyMethodDef methods[] = {
    {"pack_step", pack_step, METH_VARARGS,
     "pack_step(seqs, new_lens or None) -> (starts, lens, offsets, tables, ids) int32 bytearrays"},
    {NULL, NULL, 0, NULL}};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_hostpack",
                                    "Native packing of one paged step's host metadata.", -1, methods};

PyMODINIT_FUNC PyInit__hostpack(void) { return PyModule_Create(&module); }
