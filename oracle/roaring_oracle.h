/*
 * CPU oracle for the cu_roaring B200 engine — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's semantics for the hot path
 * (upload, promotion, set algebra, point queries, decompress, enumerate,
 * filtered top-k). Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference arm may load it, and only as the checker or the
 * timed CPU baseline; the product path never calls it.
 *
 * Images: an or_image is the host copy of a GpuRoaring in the exact packed
 * layout the engine produces (keys/types/offsets/cards/key_index and the
 * three pools), so a downloaded device result can be compared byte for byte.
 *
 * Parity pins: the known-answer cases of the reference's own test suite
 * (test/test_promote.cu, test/test_complement.cu, test/test_decompress.cu,
 * test/test_set_ops.cu, test/test_device_query.cu) are replayed against this
 * oracle by tests/test_oracle_golden.py; CRoaring (the reference's own
 * oracle, an absent git submodule) is not available, so container-type
 * parity with CRoaring itself is unpinned.
 */
#ifndef ROARING_ORACLE_H
#define ROARING_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct or_image {
  uint32_t n_containers, universe_size;
  uint64_t total_cardinality;
  uint32_t n_bitmap, n_array, n_run;
  uint32_t array_pool_bytes, run_pool_bytes, max_key;
  int32_t negated;
  uint16_t* keys;
  uint8_t* types;
  uint32_t* offsets;
  uint16_t* cards;
  uint16_t* key_index; /* max_key + 1 entries, NULL when n_containers == 0 */
  uint64_t* bitmap;    /* n_bitmap * 1024 */
  uint16_t* array;     /* array_pool_bytes / 2 */
  uint16_t* run;       /* run_pool_bytes / 2 */
} or_image;

void or_image_free(or_image* im);

/* Canonical container type for a non-empty chunk (popcount c, run count r)
 * under the resolved threshold t. Returns 0 ARRAY, 1 BITMAP, 2 RUN. */
int or_container_type(uint32_t c, uint32_t r, uint32_t t);

/* resolve_auto_threshold (reference src/promote.cu:334-367). */
uint32_t or_resolve_auto_threshold(uint32_t universe_size, uint64_t l2_bytes);

/* upload_from_ids / upload_from_bitset. `l2_bytes` feeds PROMOTE_AUTO.
 * Returns 0, or -4 when an ID is >= universe_size. */
int or_from_ids(const uint32_t* ids, uint64_t n, uint32_t universe_size, uint32_t threshold,
                uint64_t l2_bytes, or_image* out);
int or_from_bitset(const uint32_t* words, uint64_t n_words, uint32_t universe_size,
                   uint32_t threshold, uint64_t l2_bytes, or_image* out);

/* Set algebra. op: 0 AND, 1 OR, 2 ANDNOT, 3 XOR. */
int or_set_operation(const or_image* a, const or_image* b, int op, or_image* out);
int or_multi_and(const or_image* const* ims, uint32_t count, or_image* out);
int or_multi_or(const or_image* const* ims, uint32_t count, or_image* out);

int or_promote_to_bitmap(const or_image* in, or_image* out);

/* Logical membership, bitset and sorted IDs. */
void or_contains_batch(const or_image* im, const uint32_t* ids, uint64_t n, uint32_t* out_bits,
                       int n_threads);
void or_decompress(const or_image* im, uint32_t* out_words, uint64_t n_words);
uint64_t or_enumerate(const or_image* im, uint32_t* out_ids); /* returns count */

/* Structural validation of an image; returns 0 or a negative code. */
int or_validate(const or_image* im);

/* Exact fp32 filtered top-k. db/queries are fp16 bit patterns.
 * pass_bits: bit r set = row r passes (NULL = all pass). Ties -> smaller id.
 * metric 0 = IP (descending score), 1 = L2 (ascending distance). */
void or_topk(const uint16_t* db, uint64_t n_rows, uint32_t dim, const uint16_t* queries,
             uint32_t n_queries, const uint32_t* pass_bits, uint32_t k, int metric,
             float* out_dist, int64_t* out_ids, int n_threads);

/* Same with a pre-widened fp32 database and its squared norms (so a timed
 * CPU baseline does not re-widen the database every call). */
void or_topk_f32(const float* dbf, const float* norms, uint64_t n_rows, uint32_t dim,
                 const uint16_t* queries, uint32_t n_queries, const uint32_t* pass_bits, uint32_t k,
                 int metric, float* out_dist, int64_t* out_ids, int n_threads);
/* The portable Roaring serialization (the published, library-independent
 * "RoaringFormatSpec") of the sorted distinct ids[0..n): one container per
 * 65536-ID chunk, typed as that format's writers do: RUN (when allow_runs)
 * if 2 + 4*runs bytes is smaller than the alternative, else ARRAY up to 4096
 * members, else BITMAP. Cookie 12347 with run flags when any container is a
 * RUN (offsets only from 4 containers on), else 12346 with offsets. Returns
 * the byte count; writes only when out != NULL and cap suffices. */
uint64_t or_serialize_portable(const uint32_t* ids, uint64_t n, int allow_runs, uint8_t* out, uint64_t cap);

void or_widen_f16(const uint16_t* src, uint64_t n, float* dst);
void or_row_norms_f32(const float* dbf, uint64_t n_rows, uint32_t dim, float* norms);

#ifdef __cplusplus
}
#endif
#endif
