/* TEST STUB, not CRoaring: just enough of CRoaring's public C API for the
 * drop-in header's guarded upload() / get_meta() overloads
 * (include/cu_roaring/detail/upload.cuh) to compile and run in a test
 * program here, where CRoaring itself is absent. The bitmap is a sorted list
 * of IDs and its portable serialization comes from the CPU oracle's writer
 * (oracle/roaring_oracle.c, or_serialize_portable), which the tests pin to
 * the published format specification. */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

uint64_t or_serialize_portable(const uint32_t* ids, uint64_t n, int allow_runs, uint8_t* out, uint64_t cap);

typedef struct roaring_bitmap_s {
  const uint32_t* ids; /* sorted, unique */
  uint64_t n;
} roaring_bitmap_t;

static inline size_t roaring_bitmap_portable_size_in_bytes(const roaring_bitmap_t* r)
{
  return (size_t)or_serialize_portable(r->ids, r->n, 1, NULL, 0);
}

static inline size_t roaring_bitmap_portable_serialize(const roaring_bitmap_t* r, char* buf)
{
  const uint64_t n = or_serialize_portable(r->ids, r->n, 1, NULL, 0);
  return (size_t)or_serialize_portable(r->ids, r->n, 1, (uint8_t*)buf, n);
}

#ifdef __cplusplus
}
#endif
