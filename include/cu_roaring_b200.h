/*
 * cu_roaring B200 engine — C ABI of libcuroaring_b200.so.
 *
 * Every host entry point of the reference C++ API has one `cr_*` function
 * here (plain pointers and sizes, no C++ types), so that a C++ shim
 * (include/cu_roaring/detail/\*.cuh), a ctypes/cffi binding or any other FFI
 * can bind it. Each function returns CR_OK (0) or a negative cr_status; the
 * message of the last failure on the calling thread is cr_last_error_string().
 *
 * Ownership: functions with a `cr_gpu_roaring* out` parameter allocate ONE
 * stream-ordered device block (cudaMallocAsync on `stream`) and store its
 * base in out->_alloc_base; release it with cr_gpu_roaring_free[_async].
 * Functions that build a new bitmap synchronise `stream` (its host-side
 * fields — counts and sizes — must be known on return); all others are purely
 * stream-ordered.
 *
 * Streams are passed as cr_stream_t, which is ABI-identical to cudaStream_t
 * (NULL = the legacy default stream).
 */
#ifndef CU_ROARING_B200_H
#define CU_ROARING_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* cr_stream_t;

/* Byte-for-byte the layout of cu_roaring::GpuRoaring
 * (reference include/cu_roaring/types.cuh:15-54). `types` points at u8 tags
 * (0 ARRAY, 1 BITMAP, 2 RUN); `negated` is a C++ bool (one byte). */
typedef struct cr_gpu_roaring {
  uint16_t* keys;
  uint8_t*  types;
  uint32_t* offsets;
  uint16_t* cardinalities;
  uint32_t  n_containers;
  uint32_t  universe_size;
  uint64_t  total_cardinality;
  uint64_t* bitmap_data;
  uint32_t  n_bitmap_containers;
  uint16_t* array_data;
  uint32_t  n_array_containers;
  uint32_t  array_pool_bytes;
  uint16_t* run_data;
  uint32_t  n_run_containers;
  uint32_t  run_pool_bytes;
  uint16_t* key_index;
  uint32_t  max_key;
  uint8_t   negated;
  void*     _alloc_base;
} cr_gpu_roaring;

typedef enum cr_status {
  CR_OK              = 0,
  CR_ERR_INVALID     = -1, /* bad argument (null pointer, size, op code)      */
  CR_ERR_CUDA        = -2, /* a CUDA runtime call failed                       */
  CR_ERR_OOM         = -3, /* device allocation failed                          */
  CR_ERR_RANGE       = -4, /* an input ID is >= universe_size                   */
  CR_ERR_DEVICE      = -5, /* a kernel raised its device-side error flag        */
  CR_ERR_UNSUPPORTED = -6, /* configuration not supported by this build         */
  CR_ERR_COMM        = -7  /* a collective between ranks failed (NCCL)         */
} cr_status;

/* Promotion thresholds (reference include/cu_roaring/detail/promote.cuh:38-40). */
#define CR_PROMOTE_KEEP_DEFAULT 4096u
#define CR_PROMOTE_ALL          0u
#define CR_PROMOTE_AUTO         0xFFFFFFFFu

/* Set operations (reference include/cu_roaring/detail/set_ops.cuh:7-12). */
#define CR_OP_AND    0
#define CR_OP_OR     1
#define CR_OP_ANDNOT 2
#define CR_OP_XOR    3

const char* cr_last_error_string(void);
/* Library version string ("cu_roaring_b200 <semver> sm_100a"). */
const char* cr_version(void);

/* ---- Construction --------------------------------------------------------- */

/* Replaces upload_from_ids (reference src/upload_ids.cu:567-591,
 * include/cu_roaring/detail/upload_ids.cuh:19-24). Unsorted IDs with
 * duplicates, in HOST memory. Stores the complement when the unique count is
 * > universe_size/2. IDs >= universe_size are rejected with CR_ERR_RANGE. */
int cr_upload_from_ids(const uint32_t* host_ids, uint32_t n_ids, uint32_t universe_size,
                       cr_stream_t stream, uint32_t bitmap_threshold, cr_gpu_roaring* out);

/* Same, IDs already in DEVICE memory (no reference counterpart; the reference
 * always copies from the host, src/upload_ids.cu:302-313). */
int cr_upload_from_device_ids(const uint32_t* d_ids, uint64_t n_ids, uint32_t universe_size,
                              cr_stream_t stream, uint32_t bitmap_threshold,
                              cr_gpu_roaring* out);

/* A bitmap in the portable Roaring serialization (the published,
 * library-independent format: cookie 12346 / 12347, (key, cardinality - 1)
 * headers, optional offsets, ARRAY / BITMAP / RUN payloads) -> GpuRoaring
 * with canonical container types under bitmap_threshold and the complement
 * above half density. Replaces loading through CRoaring and
 * upload(const roaring_bitmap_t*) (reference src/upload.cpp:89-225, 290-296;
 * bench/bench_from_disk.cu). Returns CR_ERR_INVALID for a malformed buffer
 * and CR_ERR_RANGE for members >= universe_size. */
int cr_upload_portable(const void* data, uint64_t n_bytes, uint32_t universe_size, cr_stream_t stream,
                       uint32_t bitmap_threshold, cr_gpu_roaring* out);

/* cr_upload_portable with flags. CR_PORTABLE_KEEP_UNCOMPLEMENTED: never
 * store the complement, whatever the density (the reference's
 * upload(const roaring_bitmap_t*, stream, threshold) without a universe
 * never complements, src/upload.cpp:290-294). */
#define CR_PORTABLE_KEEP_UNCOMPLEMENTED 1u
int cr_upload_portable_ex(const void* data, uint64_t n_bytes, uint32_t universe_size, cr_stream_t stream,
                          uint32_t bitmap_threshold, uint32_t flags, cr_gpu_roaring* out);

/* Container counts and device footprint of a portable serialization, read
 * from its header on the host (no device work): replaces
 * get_meta(const roaring_bitmap_t*) (reference src/upload.cpp:31-71), whose
 * fields it fills the same way (universe_size = (max key + 1) << 16 in u32
 * arithmetic; total_bytes = 9 B per container + 8 KiB per BITMAP + 2 B per
 * ARRAY member + 4 B per run). */
typedef struct cr_roaring_meta {
  uint32_t n_containers, n_bitmap_containers, n_array_containers, n_run_containers;
  uint32_t universe_size, max_key;
  uint64_t total_bytes, total_cardinality;
} cr_roaring_meta;
int cr_portable_meta(const void* data, uint64_t n_bytes, cr_roaring_meta* out);

/* Replace upload_from_bitset / upload_from_device_bitset (reference
 * src/upload_ids.cu:806-893, include/cu_roaring/detail/upload_ids.cuh:48-56).
 * Bit i is (words[i/32] >> (i%32)) & 1. Bits >= universe_size are ignored.
 * bitmap_threshold is an addition (the reference always builds all-BITMAP). */
int cr_upload_from_bitset(const uint32_t* host_bitset, uint32_t n_words,
                          uint32_t universe_size, cr_stream_t stream,
                          uint32_t bitmap_threshold, cr_gpu_roaring* out);
int cr_upload_from_device_bitset(const uint32_t* d_bitset, uint32_t n_words,
                                 uint32_t universe_size, cr_stream_t stream,
                                 uint32_t bitmap_threshold, cr_gpu_roaring* out);

/* Replaces gpu_roaring_free / gpu_roaring_free_async (reference
 * src/upload.cpp:318-350). Resets *bm to the empty state. */
int cr_gpu_roaring_free(cr_gpu_roaring* bm);
int cr_gpu_roaring_free_async(cr_gpu_roaring* bm, cr_stream_t stream);

/* ---- Promotion ------------------------------------------------------------- */

/* Replaces resolve_auto_threshold (reference src/promote.cu:334-367):
 * PROMOTE_ALL iff 2*ceil(U/8) > L2 bytes of the device (-1 = current). */
int cr_resolve_auto_threshold(uint32_t universe_size, int device_id, uint32_t* out_threshold);
/* Replace promote_to_bitmap, promote_auto, gpu_roaring_deep_copy
 * (reference src/promote.cu:173-385). Stream-ordered, no host sync. */
int cr_promote_to_bitmap(const cr_gpu_roaring* bm, cr_stream_t stream, cr_gpu_roaring* out);
int cr_promote_auto(const cr_gpu_roaring* bm, cr_stream_t stream, int device_id,
                    cr_gpu_roaring* out);
int cr_deep_copy(const cr_gpu_roaring* bm, cr_stream_t stream, cr_gpu_roaring* out);

/* ---- Set algebra ----------------------------------------------------------- */

/* Replaces set_operation (reference src/set_ops.cu:567-1207). */
int cr_set_operation(const cr_gpu_roaring* a, const cr_gpu_roaring* b, int op,
                     cr_stream_t stream, cr_gpu_roaring* out);
/* Replace multi_and / multi_or (reference src/set_ops.cu:1715-1762).
 * Any count: more than 64 inputs are combined 64 per pass (the first pass,
 * then the running result with the next 63). */
int cr_multi_and(const cr_gpu_roaring* bitmaps, uint32_t count, cr_stream_t stream,
                 cr_gpu_roaring* out);
int cr_multi_or(const cr_gpu_roaring* bitmaps, uint32_t count, cr_stream_t stream,
                cr_gpu_roaring* out);

/* ---- Key-range sharding across GPUs (no reference counterpart: the
 * reference has no multi-GPU path) --------------------------------------------
 * Set operations, multi_and / multi_or and point queries work chunk by chunk
 * (65536 IDs per key), so G ranks split every operand at chunk boundaries,
 * rank g holding keys [g*K/G, (g+1)*K/G) with K = ceil(universe / 65536),
 * and compute with no communication; the result slices laid end to end are
 * the unsharded result, container for container.
 * cr_key_range gives a rank's key range; cr_key_slice copies a bitmap's
 * containers in [key_lo, key_hi) into a new bitmap (same universe, types and
 * complement flag); cr_concat_key_slices lays slices with ascending,
 * disjoint key ranges end to end (pool offsets rebased, key index rebuilt).
 * total_cardinality of a slice or a concatenation counts as if it were the
 * whole bitmap (U minus the stored members when the complement is stored).
 * Both synchronise `stream` (they plan the copy on the host). */
int cr_key_range(uint32_t universe_size, uint32_t rank, uint32_t n_ranks, uint32_t* key_lo, uint32_t* key_hi);
int cr_key_slice(const cr_gpu_roaring* bm, uint32_t key_lo, uint32_t key_hi, cr_stream_t stream,
                 cr_gpu_roaring* out);
int cr_concat_key_slices(const cr_gpu_roaring* slices, uint32_t n, cr_stream_t stream, cr_gpu_roaring* out);

/* ---- Export ------------------------------------------------------------------ */

/* Replaces decompress_to_bitset (reference src/decompress.cu:104-162).
 * Writes all output_words words (bits >= universe_size are zero). */
int cr_decompress_to_bitset(const cr_gpu_roaring* bm, uint32_t* d_output,
                            uint32_t output_words, cr_stream_t stream);
/* Allocating form: ceil(U/32) words via cudaMallocAsync; free with cudaFree
 * (or cudaFreeAsync). *out is NULL when universe_size == 0. */
int cr_decompress_to_bitset_alloc(const cr_gpu_roaring* bm, cr_stream_t stream,
                                  uint32_t** d_out);

/* Replace enumerate_ids (reference src/to_csr.cu:161-220): the sorted IDs of
 * the LOGICAL set (negation honoured), exactly total_cardinality values.
 * The u32 form is an addition. */
int cr_enumerate_ids_i64(const cr_gpu_roaring* bm, int64_t* d_output, cr_stream_t stream);
int cr_enumerate_ids_u32(const cr_gpu_roaring* bm, uint32_t* d_output, cr_stream_t stream);
int cr_enumerate_ids_alloc(const cr_gpu_roaring* bm, cr_stream_t stream, int64_t** d_out);

/* Allocation-free form of cr_enumerate_ids_u32 (no counterpart in the
 * reference). For callers that must not allocate device memory while they
 * run, e.g. a server that gave all GPU memory to its own pool at start-up or
 * a latency-critical path that forbids allocator calls. Its scratch is one
 * fixed array of 918,016 bytes (0.875 MiB) inside the library, resident on every GPU that
 * loads it; it covers any valid bitmap (at most 65536 containers/chunks) and
 * larger inputs are rejected with CR_ERR_INVALID. The first call on a device
 * looks up that array's device address; make that first call before any
 * stream capture. All calls share the array, so calls that overlap on the GPU
 * (different streams, or different host threads) race: serialise them. */
int cr_enumerate_ids_u32_noalloc(const cr_gpu_roaring* bm, uint32_t* d_output, cr_stream_t stream);

/* ---- Bulk point queries ------------------------------------------------------ */

/* Bulk form of GpuRoaringView::contains / warp_contains (reference
 * include/cu_roaring/device/roaring_view.cuh:39, roaring_warp_query.cuh:16),
 * as the reference benches use them (bench/bench_point_query.cu:123-146):
 * bit i of d_out_bits (u32 words, ceil(n/32)) = contains(d_ids[i]).
 * mode 0 = per-thread contains, 1 = warp_contains. */
int cr_contains_batch(const cr_gpu_roaring* bm, const uint32_t* d_ids, uint64_t n,
                      uint32_t* d_out_bits, int mode, cr_stream_t stream);

/* ---- Fused filtered brute-force top-k (no reference counterpart; the
 * reference only describes it, README.md:265-285) ---------------------------- */

#define CR_METRIC_IP 0  /* larger inner product is better          */
#define CR_METRIC_L2 1  /* smaller squared euclidean distance is better */

/* Exact top-k over the database rows that the filter contains.
 *   d_db      fp16 [n_rows x dim], row-major (dim == 128)
 *   d_db_norms fp32 [n_rows] squared norms (L2 only; may be NULL for IP)
 *   d_queries fp16 [n_queries x dim]
 *   filter    rows r with contains(r) take part; NULL = all rows
 *   row_offset global ID of row 0 (for sharded databases); the filter is
 *             queried with row_offset + r and output IDs include it
 *   k         1..256
 *   d_out_dist fp32 [n_queries x k], best first (IP: scores, L2: distances)
 *   d_out_ids  int64 [n_queries x k], -1 where fewer than k rows pass
 * Stream-ordered: the call returns without waiting for the device (the
 * search plan, including the pre-filter's choice between compacted and
 * masked rows, is made on the device, and the exact redo for degenerate
 * score distributions is queued behind the first pass and skipped by the
 * device unless needed). Scratch is allocated stream-ordered on `stream`.
 * A device-side failure (a bounded pipeline wait that ran out) is reported
 * by the next cr_filtered_topk call on the same host thread or by
 * cr_filtered_topk_check. */
int cr_filtered_topk(const uint16_t* d_db, const float* d_db_norms, uint64_t n_rows,
                     uint32_t dim, const uint16_t* d_queries, uint32_t n_queries,
                     const cr_gpu_roaring* filter, uint64_t row_offset, uint32_t k,
                     int metric, float* d_out_dist, int64_t* d_out_ids, cr_stream_t stream);

/* cr_topk_merge over parts that each sit in one packed block, as a single
 * collective (e.g. an NCCL all-gather of each shard's block) leaves them:
 * part p starts at (char*)d_parts + p * part_bytes and holds fp32 distances
 * [n_queries x k] followed by int64 ids [n_queries x k] (n_queries * k even,
 * part_bytes a multiple of 8 and >= 12 * n_queries * k). No reference
 * counterpart (the reference has no multi-GPU path). */
int cr_topk_merge_packed(const void* d_parts, uint64_t part_bytes, uint32_t n_parts, uint32_t n_queries,
                         uint32_t k, int metric, float* d_out_dist, int64_t* d_out_ids, cr_stream_t stream);

/* Waits for this host thread's outstanding cr_filtered_topk searches and
 * returns CR_ERR_DEVICE if any of them failed on the device. */
int cr_filtered_topk_check(void);

/* ---- Row-sharded top-k over several GPUs (no reference counterpart: the
 * reference has neither a top-k nor a multi-GPU path) ------------------------
 * One process (rank) per GPU. A communicator is made once per rank:
 * rank 0 calls cr_topk_comm_unique_id, hands the CR_TOPK_COMM_ID_BYTES bytes
 * to every rank by any host channel, and every rank calls cr_topk_comm_init
 * with its device current (all ranks together: the call waits for the
 * others). NCCL is loaded at run time; without it these calls return
 * CR_ERR_UNSUPPORTED. */
#define CR_TOPK_COMM_ID_BYTES 128
typedef struct cr_topk_comm_st* cr_topk_comm;
int cr_topk_comm_unique_id(void* out_id, uint32_t n_bytes);
int cr_topk_comm_init(const void* unique_id, int n_ranks, int rank, cr_topk_comm* out);
int cr_topk_comm_size(cr_topk_comm comm, int* n_ranks, int* rank);
/* Waits for the device, frees the communicator and its gather buffer. */
int cr_topk_comm_destroy(cr_topk_comm comm);

/* Every rank calls this with its own rows [row_offset, row_offset +
 * shard_rows) of the database (d_db holds just those rows) and the same
 * queries, filter, k and metric. Each rank searches its rows like
 * cr_filtered_topk (filter queried with global row IDs, output IDs global);
 * the per-rank [n_queries x k] lists go to `root` in one NCCL group of
 * point-to-point transfers and the root writes the merged top-k to
 * d_out_dist / d_out_ids (the other ranks' output pointers are not used and
 * may be NULL). Stream-ordered on every rank, no host wait. */
int cr_filtered_topk_sharded(cr_topk_comm comm, int root, const uint16_t* d_db, const float* d_db_norms,
                             uint64_t shard_rows, uint32_t dim, const uint16_t* d_queries, uint32_t n_queries,
                             const cr_gpu_roaring* filter, uint64_t row_offset, uint32_t k, int metric,
                             float* d_out_dist, int64_t* d_out_ids, cr_stream_t stream);

/* Squared L2 norms of fp16 rows (fp32 accumulate) for the L2 metric. */
int cr_row_norms(const uint16_t* d_db, uint64_t n_rows, uint32_t dim, float* d_out,
                 cr_stream_t stream);

/* Merge `n_parts` per-shard top-k lists ([n_parts x n_queries x k], device)
 * into one [n_queries x k] list (same ordering rules as cr_filtered_topk). */
int cr_topk_merge(const float* d_dist_parts, const int64_t* d_id_parts, uint32_t n_parts,
                  uint32_t n_queries, uint32_t k, int metric, float* d_out_dist,
                  int64_t* d_out_ids, cr_stream_t stream);

/* ---- Batches of bitmaps (replace the reference's v2 API,
 * v2/include/cu_roaring_v2/api.hpp:22-69) ------------------------------------
 * cr_roaring_batch has the exact layout of cu_roaring::v2::GpuRoaringBatch
 * (include/cu_roaring_v2/types.cuh): N bitmaps in one device block, CSR
 * offsets per bitmap, shared pools, no complement, host mirrors of the
 * per-bitmap scalars. */
typedef struct cr_roaring_batch {
  uint32_t n_bitmaps, total_containers, n_bitmap_containers_total;
  uint32_t array_pool_bytes, run_pool_bytes;
  uint32_t* container_starts;
  uint32_t* key_index_starts;
  uint16_t* keys;
  uint8_t* types;
  uint32_t* offsets;
  uint16_t* cardinalities;
  uint16_t* key_indices;
  uint64_t* bitmap_data;
  uint16_t* array_data;
  uint16_t* run_data;
  const uint64_t* host_total_cardinalities;
  const uint32_t* host_universe_sizes;
  const uint32_t* host_container_starts;
  const uint32_t* host_key_index_starts;
  const uint32_t* host_n_bitmap_containers;
  void* _alloc_base;
  void* _host_meta_base;
} cr_roaring_batch;

/* N bitmaps in the portable Roaring serialization -> one batch (one device
 * allocation, one host-to-device copy). Container types are kept as
 * serialized. Replaces upload_batch(const roaring_bitmap_t* const*, n)
 * (v2/include/cu_roaring_v2/api.hpp:22-25), whose CRoaring input is absent
 * here; n == 0 gives an empty batch. */
int cr_batch_upload_portable(const void* const* buffers, const uint64_t* sizes, uint32_t n, cr_stream_t stream,
                             cr_roaring_batch* out);
/* Frees both blocks of a batch and zeroes it (api.hpp:29). */
int cr_batch_free(cr_roaring_batch* batch);
/* Every ARRAY / RUN container of every bitmap becomes a BITMAP container
 * (api.hpp:31-38); a new batch, the input untouched. */
int cr_batch_promote(const cr_roaring_batch* in, cr_stream_t stream, cr_roaring_batch* out);
/* AND of the bitmaps in[indices[0..n)) (all of them all-BITMAP), a
 * one-bitmap batch without empty containers (api.hpp:46-55). */
int cr_batch_multi_and(const cr_roaring_batch* in, const uint32_t* indices, uint32_t n, cr_stream_t stream,
                       cr_roaring_batch* out);
/* Bitmap b -> d_bitsets[b * words_each ..), u64 words (api.hpp:57-67): only
 * the windows of present containers are written; words_each must cover
 * every bitmap's universe. */
int cr_batch_decompress(const cr_roaring_batch* in, uint64_t* d_bitsets, uint64_t words_each, cr_stream_t stream);
/* Bit i of d_out_bits = contains(batch, d_bitmap_idx[i], d_ids[i]) (the
 * query.cuh device test, run over n pairs; no reference counterpart). */
int cr_batch_contains(const cr_roaring_batch* in, const uint32_t* d_bitmap_idx, const uint32_t* d_ids, uint64_t n,
                      uint32_t* d_out_bits, cr_stream_t stream);

/* ---- Fault injection for tests (no reference counterpart) -------------------
 * After `after` more successful device allocations, every later one inside
 * the library fails as if the device were out of memory (CR_ERR_OOM);
 * after < 0 switches injection off. Process-wide. For testing callers'
 * error paths: no call may leak or leave a half-built bitmap behind. */
int cr_test_fail_allocations(int64_t after);

/* ---- Measurement hooks (no reference counterpart) ---------------------------
 * When enabled, the library brackets its dominant kernels with CUDA events on
 * the launching stream; cr_profile_last_ms returns the device time of the
 * most recent launch of `kernel` on the calling thread (waits for it).
 * Kernel ids: CR_KERNEL_TOPK, CR_KERNEL_CONTAINS, CR_KERNEL_SETOP, CR_KERNEL_UPLOAD_SCATTER,
 * CR_KERNEL_UPLOAD_EMIT, CR_KERNEL_DECOMPRESS, CR_KERNEL_TOPK_MERGE, CR_KERNEL_TOPK_COMPACT. */
#define CR_KERNEL_TOPK 0
#define CR_KERNEL_CONTAINS 1
#define CR_KERNEL_SETOP 2
#define CR_KERNEL_UPLOAD_SCATTER 3
#define CR_KERNEL_UPLOAD_EMIT 4
#define CR_KERNEL_DECOMPRESS 5
#define CR_KERNEL_TOPK_MERGE 6
#define CR_KERNEL_TOPK_COMPACT 7 /* pass-row compaction plus the row copy of the pre-filter */
int cr_profile_enable(int on);
/* Restricts the bracketing to the kernel ids whose bit is set in `mask`
 * (default: all). Each bracket is two event records on the launching
 * stream, which cost device time between short kernels. No reference
 * counterpart (measurement support). */
int cr_profile_kinds(uint32_t mask);
int cr_profile_last_ms(int kernel, float* ms);
/* Sum of the device times of every profiled launch of `kernel` since
 * profiling was last switched on, and their number (waits for them). */
int cr_profile_sum_ms(int kernel, float* total_ms, uint32_t* count);

#ifdef __cplusplus
}
#endif
#endif /* CU_ROARING_B200_H */
