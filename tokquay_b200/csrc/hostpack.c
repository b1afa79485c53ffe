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
 *
 *   plan_sequences(plan_fn, seqs, new_lens or None, block_size, num_blocks,
 *                  n_head, vocab_size, n_ctas, min_split_chunks, caps, out,
 *                  out_capacity, layout) -> status
 *
 * packs the same arrays into buffers kept by this module and hands them
 * straight to the planner (plan_fn: the address of tq_plan_step; caps, out and
 * layout: addresses of int32 host buffers, caps 0 for none), so one decode
 * step's host planning makes no Python objects at all.  Returns the planner's
 * status (0 = TQ_OK).  With decode_max_ctx > 0 only a decode step (one new
 * token per sequence, contexts <= decode_max_ctx) is planned; any other step
 * returns -2 and plans nothing.
 *
 *   advance_cached(seqs)
 *
 * adds each sequence's q_len of the step plan_sequences last planned to its
 * num_cached_tokens (tokquay/generate.py:85-86).
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

/* Growable int32 buffers owned by this module (the GIL serialises callers). */
typedef struct {
  int32_t* p;
  Py_ssize_t cap;
} IntBuf;

static int32_t* grow(IntBuf* b, Py_ssize_t n) {
  if (n <= b->cap) return b->p;
  Py_ssize_t cap = b->cap ? b->cap : 256;
  while (cap < n) cap *= 2;
  int32_t* q = (int32_t*)PyMem_Realloc(b->p, (size_t)cap * sizeof(int32_t));
  if (!q) {
    PyErr_NoMemory();
    return NULL;
  }
  b->p = q;
  b->cap = cap;
  return q;
}

static PyObject *s_cached, *s_table, *s_prompt, *s_output;

/* Packs seqs (and new_lens, NULL for "all uncached") into st/ln/of (B, B, B+1
 * entries, caller-sized) and the growable table / id buffers.  Returns 0, or
 * -1 with a Python exception set. */
static int pack_into(PyObject* seq_fast, PyObject* lens_fast, int32_t* st, int32_t* ln, int32_t* of, IntBuf* tabs,
                     IntBuf* toks, Py_ssize_t* n_tab_out, Py_ssize_t* n_tok_out) {
  const Py_ssize_t B = PySequence_Fast_GET_SIZE(seq_fast);
  /* Pass 1: sizes. */
  Py_ssize_t n_tab = 0, n_tok = 0;
  of[0] = 0;
  for (Py_ssize_t b = 0; b < B; ++b) {
    PyObject* s = PySequence_Fast_GET_ITEM(seq_fast, b);
    long cached;
    if (get_long_attr(s, s_cached, &cached) < 0) return -1;
    PyObject* tbl = get_list_attr(s, s_table);
    if (!tbl) return -1;
    const Py_ssize_t nt = PyList_GET_SIZE(tbl);
    Py_DECREF(tbl);
    long n;
    if (lens_fast) {
      n = PyLong_AsLong(PySequence_Fast_GET_ITEM(lens_fast, b));
      if (n == -1 && PyErr_Occurred()) return -1;
    } else {
      PyObject* pr = get_list_attr(s, s_prompt);
      if (!pr) return -1;
      PyObject* ou = get_list_attr(s, s_output);
      if (!ou) {
        Py_DECREF(pr);
        return -1;
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
      return -1;
    }
    of[b + 1] = (int32_t)n_tab;
  }
  /* Pass 2: block ids and token ids. */
  int32_t* tb = grow(tabs, n_tab > 0 ? n_tab : 1);
  int32_t* id = grow(toks, n_tok > 0 ? n_tok : 1);
  if (!tb || !id) return -1;
  for (Py_ssize_t b = 0; b < B; ++b) {
    PyObject* s = PySequence_Fast_GET_ITEM(seq_fast, b);
    PyObject* tbl = get_list_attr(s, s_table);
    if (!tbl) return -1;
    int rc = put_ints(tbl, 0, PyList_GET_SIZE(tbl), tb + of[b]);
    Py_DECREF(tbl);
    if (rc < 0) return -1;
    const long begin = st[b], n = ln[b];
    if (n <= 0 || begin < 0) continue; /* the planner rejects these with the reference's message */
    PyObject* pr = get_list_attr(s, s_prompt);
    if (!pr) return -1;
    PyObject* ou = get_list_attr(s, s_output);
    if (!ou) {
      Py_DECREF(pr);
      return -1;
    }
    const Py_ssize_t np_ = PyList_GET_SIZE(pr), no = PyList_GET_SIZE(ou);
    const Py_ssize_t end = begin + n;
    if (end > np_ + no) {
      Py_DECREF(pr);
      Py_DECREF(ou);
      PyErr_SetString(PyExc_ValueError, "a sequence feeds more tokens than it has");
      return -1;
    }
    /* tokens [begin, end) of prompt + output */
    rc = 0;
    if (begin < np_) rc = put_ints(pr, begin, end < np_ ? end : np_, id);
    if (rc == 0 && end > np_)
      rc = put_ints(ou, begin > np_ ? begin - np_ : 0, end - np_, id + (begin < np_ ? np_ - begin : 0));
    id += n;
    Py_DECREF(pr);
    Py_DECREF(ou);
    if (rc < 0) return -1;
  }
  *n_tab_out = n_tab;
  *n_tok_out = n_tok;
  return 0;
}

/* seqs / new_lens as fast sequences; lens_fast NULL for None.  Returns -1 with
 * an exception set on error. */
static int open_args(PyObject* seqs, PyObject* new_lens, PyObject** seq_fast, PyObject** lens_fast) {
  *seq_fast = PySequence_Fast(seqs, "seqs must be a sequence");
  *lens_fast = NULL;
  if (!*seq_fast) return -1;
  if (new_lens != Py_None) {
    *lens_fast = PySequence_Fast(new_lens, "new_lens must be a sequence");
    if (!*lens_fast) return -1;
    if (PySequence_Fast_GET_SIZE(*lens_fast) != PySequence_Fast_GET_SIZE(*seq_fast)) {
      PyErr_SetString(PyExc_ValueError, "block_tables, start and new_lens must be non-empty and the same length");
      return -1;
    }
  }
  return 0;
}

static IntBuf g_tabs, g_toks, g_small;

static PyObject* pack_step(PyObject* self, PyObject* args) {
  (void)self;
  PyObject *seqs, *new_lens, *seq_fast = NULL, *lens_fast = NULL, *result = NULL;
  if (!PyArg_ParseTuple(args, "OO", &seqs, &new_lens)) return NULL;
  if (open_args(seqs, new_lens, &seq_fast, &lens_fast) < 0) goto done;
  const Py_ssize_t B = PySequence_Fast_GET_SIZE(seq_fast);
  PyObject* starts = PyByteArray_FromStringAndSize(NULL, B * 4);
  PyObject* lens = PyByteArray_FromStringAndSize(NULL, B * 4);
  PyObject* offs = PyByteArray_FromStringAndSize(NULL, (B + 1) * 4);
  PyObject *tables = NULL, *ids = NULL;
  Py_ssize_t n_tab = 0, n_tok = 0;
  if (starts && lens && offs &&
      pack_into(seq_fast, lens_fast, (int32_t*)PyByteArray_AS_STRING(starts), (int32_t*)PyByteArray_AS_STRING(lens),
                (int32_t*)PyByteArray_AS_STRING(offs), &g_tabs, &g_toks, &n_tab, &n_tok) == 0) {
    tables = PyByteArray_FromStringAndSize((const char*)g_tabs.p, n_tab * 4);
    ids = PyByteArray_FromStringAndSize((const char*)g_toks.p, n_tok * 4);
    if (tables && ids) result = PyTuple_Pack(5, starts, lens, offs, tables, ids);
  }
  Py_XDECREF(starts);
  Py_XDECREF(lens);
  Py_XDECREF(offs);
  Py_XDECREF(tables);
  Py_XDECREF(ids);
done:
  Py_XDECREF(lens_fast);
  Py_XDECREF(seq_fast);
  return result;
}

/* plan_sequences' answer for a step that is not a decode step (decode_max_ctx). */
#define NOT_A_DECODE_STEP (-2)

/* The planner's C signature (include/tokquay_b200.h, tq_plan_step). */
typedef int (*plan_fn_t)(int32_t, const int32_t*, const int32_t*, const int32_t*, const int32_t*, const int32_t*,
                         int32_t, int64_t, int32_t, int32_t, int32_t, int32_t, const int32_t*, int32_t*, int64_t,
                         int32_t*);

/* q_len of the last step plan_sequences packed (for advance_cached). */
static Py_ssize_t g_last_B = -1;

static PyObject* plan_sequences(PyObject* self, PyObject* args) {
  (void)self;
  unsigned long long fn, caps, out, layout;
  PyObject *seqs, *new_lens, *seq_fast = NULL, *lens_fast = NULL, *result = NULL;
  int block_size, n_head, vocab, n_ctas, min_split, decode_max_ctx = 0;
  long long num_blocks, out_cap;
  if (!PyArg_ParseTuple(args, "KOOiLiiiiKKLK|i", &fn, &seqs, &new_lens, &block_size, &num_blocks, &n_head, &vocab,
                        &n_ctas, &min_split, &caps, &out, &out_cap, &layout, &decode_max_ctx))
    return NULL;
  g_last_B = -1;
  if (!fn || !out || !layout) {
    PyErr_SetString(PyExc_ValueError, "plan_fn, out and layout must be non-zero addresses");
    return NULL;
  }
  if (open_args(seqs, new_lens, &seq_fast, &lens_fast) < 0) goto done;
  const Py_ssize_t B = PySequence_Fast_GET_SIZE(seq_fast);
  int32_t* small = grow(&g_small, 3 * B + 1);
  if (!small) goto done;
  Py_ssize_t n_tab = 0, n_tok = 0;
  if (pack_into(seq_fast, lens_fast, small, small + B, small + 2 * B, &g_tabs, &g_toks, &n_tab, &n_tok) < 0)
    goto done;
  if (decode_max_ctx > 0) { /* only a decode step (one token each, context <= decode_max_ctx) is planned */
    for (Py_ssize_t b = 0; b < B; ++b)
      if (small[B + b] != 1 || small[b] < 0 || small[b] + 1 > decode_max_ctx) {
        result = PyLong_FromLong(NOT_A_DECODE_STEP);
        goto done;
      }
  }
  const int status = ((plan_fn_t)(uintptr_t)fn)(
      (int32_t)B, small, small + B, small + 2 * B, g_tabs.p, g_toks.p, block_size, num_blocks, n_head, vocab, n_ctas,
      min_split, caps ? (const int32_t*)(uintptr_t)caps : NULL, (int32_t*)(uintptr_t)out, out_cap,
      (int32_t*)(uintptr_t)layout);
  if (status == 0) g_last_B = B;
  result = PyLong_FromLong(status);
done:
  Py_XDECREF(lens_fast);
  Py_XDECREF(seq_fast);
  return result;
}

/* advance_cached(seqs): num_cached_tokens += q_len for each sequence of the
 * step plan_sequences last planned successfully (the same list). */
static PyObject* advance_cached(PyObject* self, PyObject* args) {
  (void)self;
  PyObject* seqs;
  if (!PyArg_ParseTuple(args, "O", &seqs)) return NULL;
  PyObject* seq_fast = PySequence_Fast(seqs, "seqs must be a sequence");
  if (!seq_fast) return NULL;
  const Py_ssize_t B = PySequence_Fast_GET_SIZE(seq_fast);
  if (B != g_last_B) {
    Py_DECREF(seq_fast);
    PyErr_SetString(PyExc_RuntimeError, "advance_cached: not the step plan_sequences last planned");
    return NULL;
  }
  g_last_B = -1;
  for (Py_ssize_t b = 0; b < B; ++b) {
    PyObject* v = PyLong_FromLong((long)g_small.p[b] + g_small.p[B + b]);
    if (!v || PyObject_SetAttr(PySequence_Fast_GET_ITEM(seq_fast, b), s_cached, v) < 0) {
      Py_XDECREF(v);
      Py_DECREF(seq_fast);
      return NULL;
    }
    Py_DECREF(v);
  }
  Py_DECREF(seq_fast);
  Py_RETURN_NONE;
}

static PyMethodDef methods[] = {
    {"pack_step", pack_step, METH_VARARGS,
     "pack_step(seqs, new_lens or None) -> (starts, lens, offsets, tables, ids) int32 bytearrays"},
    {"plan_sequences", plan_sequences, METH_VARARGS,
     "plan_sequences(plan_fn, seqs, new_lens or None, block_size, num_blocks, n_head, vocab_size, n_ctas, "
     "min_split_chunks, caps, out, out_capacity, layout[, decode_max_ctx]) -> status "
     "(-2: not a decode step within decode_max_ctx, nothing planned)"},
    {"advance_cached", advance_cached, METH_VARARGS,
     "advance_cached(seqs): num_cached_tokens += q_len of the step plan_sequences last planned"},
    {NULL, NULL, 0, NULL}};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_hostpack",
                                    "Native packing of one paged step's host metadata.", -1, methods};

PyMODINIT_FUNC PyInit__hostpack(void) {
  s_cached = PyUnicode_InternFromString("num_cached_tokens");
  s_table = PyUnicode_InternFromString("block_table");
  s_prompt = PyUnicode_InternFromString("prompt_token_ids");
  s_output = PyUnicode_InternFromString("output_token_ids");
  if (!s_cached || !s_table || !s_prompt || !s_output) return NULL;
  return PyModule_Create(&module);
}
