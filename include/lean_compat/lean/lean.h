/* Minimal Lean-4 runtime object API, written for this project.
 *
 * It provides the handful of `lean.h` names that a Lean `@[extern]` C function on the
 * PPO+Muon update path touches: scalar arrays (`FloatArray`), boxed scalars, constructor
 * objects (`Prod`, IO results) and strings. The struct layouts follow the object header
 * that Lean 4 documents (reference count, other/tag bytes, then the payload), so a
 * function compiled against this header reads a real `FloatArray` the same way.
 *
 * Allocation here is plain malloc/free. Inside a real Lean executable the adapter must be
 * compiled against Lean's own lean.h instead (its allocator owns the objects); this header
 * exists so the adapter and the reference's C kernels can be compiled and exercised on a
 * machine without a Lean toolchain. */
#ifndef PL_LEAN_COMPAT_LEAN_H
#define PL_LEAN_COMPAT_LEAN_H

#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef LEAN_EXPORT
#define LEAN_EXPORT __attribute__((visibility("default")))
#endif

#define PL_LEAN_COMPAT 1
#define LeanMaxCtorTag 244
#define LeanScalarArray 248
#define LeanString 249

typedef struct {
  int m_rc;
  unsigned m_cs_sz : 16;
  unsigned m_other : 8;
  unsigned m_tag : 8;
} lean_object;

typedef struct {
  lean_object m_header;
  size_t m_size;
  size_t m_capacity;
  uint8_t m_data[1];
} lean_sarray_object;

typedef struct {
  lean_object m_header;
  lean_object* m_objs[1];
} lean_ctor_object;

typedef struct {
  lean_object m_header;
  size_t m_size;     /* bytes including the terminating 0 */
  size_t m_capacity;
  size_t m_length;   /* code points */
  char m_data[1];
} lean_string_object;

typedef lean_object* lean_obj_arg;
typedef lean_object* b_lean_obj_arg;
typedef lean_object* lean_obj_res;
typedef lean_object* b_lean_obj_res;

static inline int lean_is_scalar(const lean_object* o) { return ((size_t)o & 1) == 1; }
static inline lean_object* lean_box(size_t n) { return (lean_object*)((n << 1) | 1); }
static inline size_t lean_unbox(const lean_object* o) { return (size_t)o >> 1; }

static inline lean_sarray_object* lean_to_sarray(lean_object* o) { return (lean_sarray_object*)o; }
static inline lean_ctor_object* lean_to_ctor(lean_object* o) { return (lean_ctor_object*)o; }
static inline lean_string_object* lean_to_string(lean_object* o) { return (lean_string_object*)o; }
static inline unsigned lean_ptr_tag(const lean_object* o) { return o->m_tag; }
static inline unsigned lean_ptr_other(const lean_object* o) { return o->m_other; }
static inline unsigned lean_obj_tag(const lean_object* o) {
  return lean_is_scalar(o) ? (unsigned)lean_unbox(o) : o->m_tag;
}

static inline lean_object* pl_lean_compat_alloc(size_t bytes, unsigned tag, unsigned other) {
  lean_object* o = (lean_object*)malloc(bytes < sizeof(lean_object) ? sizeof(lean_object) : bytes);
  if (!o) abort();
  o->m_rc = 1;
  o->m_tag = tag;
  o->m_other = other;
  o->m_cs_sz = 0;
  return o;
}

static inline lean_object* lean_alloc_sarray(unsigned elem_size, size_t size, size_t capacity) {
  size_t bytes = offsetof(lean_sarray_object, m_data) + (size_t)elem_size * (capacity ? capacity : 1);
  lean_object* o = pl_lean_compat_alloc(bytes, LeanScalarArray, elem_size);
  lean_to_sarray(o)->m_size = size;
  lean_to_sarray(o)->m_capacity = capacity;
  return o;
}
static inline size_t lean_sarray_size(b_lean_obj_arg o) { return lean_to_sarray(o)->m_size; }
static inline uint8_t* lean_sarray_cptr(lean_object* o) { return lean_to_sarray(o)->m_data; }
static inline double* lean_float_array_cptr(b_lean_obj_arg a) { return (double*)lean_to_sarray(a)->m_data; }

static inline lean_object* lean_alloc_ctor(unsigned tag, unsigned num_objs, unsigned scalar_sz) {
  size_t bytes = offsetof(lean_ctor_object, m_objs) + sizeof(lean_object*) * num_objs + scalar_sz;
  return pl_lean_compat_alloc(bytes, tag, num_objs);
}
static inline void lean_ctor_set(b_lean_obj_arg o, unsigned i, lean_obj_arg v) { lean_to_ctor(o)->m_objs[i] = v; }
static inline lean_object* lean_ctor_get(b_lean_obj_arg o, unsigned i) { return lean_to_ctor(o)->m_objs[i]; }

static inline void lean_inc(lean_object* o) { if (!lean_is_scalar(o)) o->m_rc++; }
static inline void lean_dec(lean_object* o) {
  if (lean_is_scalar(o) || o == NULL) return;
  if (--o->m_rc > 0) return;
  if (o->m_tag <= LeanMaxCtorTag) {
    unsigned n = o->m_other;
    for (unsigned i = 0; i < n; i++) lean_dec(lean_to_ctor(o)->m_objs[i]);
  }
  free(o);
}

static inline lean_object* lean_box_usize(size_t v) {
  lean_object* o = lean_alloc_ctor(0, 0, sizeof(size_t));
  memcpy((char*)o + offsetof(lean_ctor_object, m_objs), &v, sizeof(size_t));
  return o;
}
static inline size_t lean_unbox_usize(b_lean_obj_arg o) {
  if (lean_is_scalar(o)) return lean_unbox(o);
  size_t v;
  memcpy(&v, (char*)o + offsetof(lean_ctor_object, m_objs), sizeof(size_t));
  return v;
}

static inline lean_object* lean_mk_string(const char* s) {
  size_t n = strlen(s);
  size_t bytes = offsetof(lean_string_object, m_data) + n + 1;
  lean_object* o = pl_lean_compat_alloc(bytes, LeanString, 0);
  lean_to_string(o)->m_size = n + 1;
  lean_to_string(o)->m_capacity = n + 1;
  lean_to_string(o)->m_length = n;
  memcpy(lean_to_string(o)->m_data, s, n + 1);
  return o;
}
static inline const char* lean_string_cstr(b_lean_obj_arg o) { return lean_to_string(o)->m_data; }

/* IO results: constructor 0 = ok (value, world), constructor 1 = error (error, world). */
static inline lean_object* lean_io_result_mk_ok(lean_obj_arg a) {
  lean_object* r = lean_alloc_ctor(0, 2, 0);
  lean_ctor_set(r, 0, a);
  lean_ctor_set(r, 1, lean_box(0));
  return r;
}
static inline lean_object* lean_io_result_mk_error(lean_obj_arg e) {
  lean_object* r = lean_alloc_ctor(1, 2, 0);
  lean_ctor_set(r, 0, e);
  lean_ctor_set(r, 1, lean_box(0));
  return r;
}
static inline int lean_io_result_is_ok(b_lean_obj_arg r) { return lean_ptr_tag(r) == 0; }
static inline lean_object* lean_io_result_get_value(b_lean_obj_arg r) { return lean_ctor_get(r, 0); }
/* `IO.userError msg`: a one-field constructor carrying the message string. */
static inline lean_object* lean_mk_io_user_error(lean_obj_arg str) {
  lean_object* e = lean_alloc_ctor(7, 1, 0);
  lean_ctor_set(e, 0, str);
  return e;
}

#ifdef __cplusplus
}
#endif
#endif
