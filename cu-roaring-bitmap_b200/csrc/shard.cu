// cu_roaring B200 engine — the row-sharded filtered top-k over several GPUs.
//
// No reference counterpart (the reference has no multi-GPU path and no
// top-k). One process per GPU; every rank holds a contiguous range of
// database rows [row_offset, row_offset + shard_rows) and the same queries.
// Per call:
//   1. each rank runs the fused filtered top-k over its rows (global row IDs)
//      into one packed block: fp32 distances [Q x k], then int64 ids [Q x k];
//      the root's block is written straight into its slot of the gather
//      buffer;
//   2. one NCCL group of point-to-point transfers brings every other rank's
//      block into the root's gather buffer (NVLink through NVSwitch on one
//      B200 box; plain local buffers on both sides, no peer loads);
//   3. the root merges the n_ranks sorted lists per query (k_merge).
// Everything is stream-ordered on the caller's stream; nothing waits on the
// host.
//
// NCCL is opened at run time (dlopen of libnccl.so.2, reusing a copy that the
// process already loaded, e.g. PyTorch's), so the library loads and every
// single-GPU entry point works on hosts without NCCL.
#include <dlfcn.h>
#include <nccl.h>  // types and constants only; the functions come from dlopen

#include <mutex>
#include <string>

#include "common.cuh"

namespace crb {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  std::string why;  // empty when every symbol resolved

  static NcclApi& get()
  {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] { api.open(); });
    if (!api.why.empty()) fail(CR_ERR_UNSUPPORTED, "NCCL is not available: " + api.why);
    return api;
  }

 private:
  template <class F> bool sym(void* h, const char* name, F& f)
  {
    f = reinterpret_cast<F>(dlsym(h, name));
    if (!f) why = std::string("missing symbol ") + name;
    return f != nullptr;
  }
  void open()
  {
    // A copy already in the process first (same communicator ABI as the
    // caller's other NCCL users), then the default search path.
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      const char* e = dlerror();
      why = e ? e : "dlopen(libnccl.so.2) failed";
      return;
    }
    sym(h, "ncclGetUniqueId", get_unique_id) && sym(h, "ncclCommInitRank", comm_init_rank) &&
        sym(h, "ncclCommDestroy", comm_destroy) && sym(h, "ncclGroupStart", group_start) &&
        sym(h, "ncclGroupEnd", group_end) && sym(h, "ncclSend", send) && sym(h, "ncclRecv", recv) &&
        sym(h, "ncclGetErrorString", error_string);
  }
};

void nccl_check(ncclResult_t r, const char* what)
{
  if (r == ncclSuccess) return;
  const NcclApi& api = NcclApi::get();
  fail(CR_ERR_COMM, std::string(what) + " failed: " + (api.error_string ? api.error_string(r) : "?"));
}

// Packed block of one shard's result: distances, then ids 16-byte aligned.
struct BlockLayout {
  uint64_t dist_bytes, id_off, bytes;
  BlockLayout(uint32_t nq, uint32_t k)
  {
    dist_bytes = uint64_t(nq) * k * 4;
    id_off = (dist_bytes + 255) & ~uint64_t(255);
    bytes = (id_off + uint64_t(nq) * k * 8 + 255) & ~uint64_t(255);
  }
};

}  // namespace
}  // namespace crb

// The communicator: NCCL's, plus this rank's gather buffer (allocated on the
// first call that needs it, grown when a call needs more, freed with the
// communicator).
struct cr_topk_comm_st {
  ncclComm_t comm = nullptr;
  int n_ranks = 0, rank = 0, device = 0;
  char* buf = nullptr;
  size_t buf_bytes = 0;
};

using namespace crb;

extern "C" int cr_topk_comm_unique_id(void* out_id, uint32_t n_bytes)
{
  CR_API_BEGIN
  CR_REQUIRE(out_id != nullptr && n_bytes >= CR_TOPK_COMM_ID_BYTES, "cr_topk_comm_unique_id: buffer too small");
  ncclUniqueId id;
  nccl_check(NcclApi::get().get_unique_id(&id), "ncclGetUniqueId");
  std::memcpy(out_id, &id, sizeof(id));
  CR_API_END
}

extern "C" int cr_topk_comm_init(const void* unique_id, int n_ranks, int rank, cr_topk_comm* out)
{
  CR_API_BEGIN
  CR_REQUIRE(unique_id && out, "cr_topk_comm_init: null argument");
  CR_REQUIRE(n_ranks >= 1 && rank >= 0 && rank < n_ranks, "cr_topk_comm_init: bad rank / n_ranks");
  *out = nullptr;
  auto* c = new cr_topk_comm_st();
  c->n_ranks = n_ranks;
  c->rank = rank;
  CR_CUDA(cudaGetDevice(&c->device));
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  const ncclResult_t r = NcclApi::get().comm_init_rank(&c->comm, n_ranks, id, rank);
  if (r != ncclSuccess) {
    delete c;
    nccl_check(r, "ncclCommInitRank");
  }
  *out = c;
  CR_API_END
}

extern "C" int cr_topk_comm_destroy(cr_topk_comm comm)
{
  CR_API_BEGIN
  if (!comm) return CR_OK;
  int prev = 0;
  CR_CUDA(cudaGetDevice(&prev));
  CR_CUDA(cudaSetDevice(comm->device));
  if (comm->buf) {
    CR_CUDA(cudaDeviceSynchronize());
    CR_CUDA(cudaFree(comm->buf));
  }
  const ncclResult_t r = comm->comm ? NcclApi::get().comm_destroy(comm->comm) : ncclSuccess;
  delete comm;
  CR_CUDA(cudaSetDevice(prev));
  nccl_check(r, "ncclCommDestroy");
  CR_API_END
}

extern "C" int cr_topk_comm_size(cr_topk_comm comm, int* n_ranks, int* rank)
{
  CR_API_BEGIN
  CR_REQUIRE(comm && n_ranks && rank, "cr_topk_comm_size: null argument");
  *n_ranks = comm->n_ranks;
  *rank = comm->rank;
  CR_API_END
}

extern "C" int cr_filtered_topk_sharded(cr_topk_comm comm, int root, const uint16_t* d_db, const float* d_db_norms,
                                        uint64_t shard_rows, uint32_t dim, const uint16_t* d_queries,
                                        uint32_t n_queries, const cr_gpu_roaring* filter, uint64_t row_offset,
                                        uint32_t k, int metric, float* d_out_dist, int64_t* d_out_ids,
                                        cr_stream_t stream)
{
  CR_API_BEGIN
  CR_REQUIRE(comm != nullptr, "cr_filtered_topk_sharded: null communicator");
  CR_REQUIRE(root >= 0 && root < comm->n_ranks, "cr_filtered_topk_sharded: root out of range");
  CR_REQUIRE(k >= 1 && k <= 256 && n_queries >= 1, "cr_filtered_topk_sharded: bad k or n_queries");
  int dev = 0;
  CR_CUDA(cudaGetDevice(&dev));
  CR_REQUIRE(dev == comm->device, "cr_filtered_topk_sharded: the current device is not the communicator's");
  const bool is_root = comm->rank == root;
  CR_REQUIRE(!is_root || (d_out_dist && d_out_ids), "cr_filtered_topk_sharded: the root needs output buffers");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const BlockLayout L(n_queries, k);
  const int n = comm->n_ranks;
  if (n == 1) {  // one rank: the search's own merge is the answer
    filtered_topk_enqueue(d_db, d_db_norms, shard_rows, dim, d_queries, n_queries, filter, row_offset, k, metric,
                          d_out_dist, d_out_ids, s);
    return CR_OK;
  }
  const size_t need = is_root ? size_t(n) * L.bytes : L.bytes;
  if (comm->buf_bytes < need) {
    if (comm->buf) {
      CR_CUDA(cudaStreamSynchronize(s));  // the previous calls' transfers have finished
      CR_CUDA(cudaFree(comm->buf));
      comm->buf = nullptr;
      comm->buf_bytes = 0;
    }
    void* p = nullptr;
    const cudaError_t e = cudaMalloc(&p, need);
    if (e != cudaSuccess) {
      cudaGetLastError();
      fail(e == cudaErrorMemoryAllocation ? CR_ERR_OOM : CR_ERR_CUDA,
           std::string("cr_filtered_topk_sharded: gather buffer: ") + cudaGetErrorString(e));
    }
    comm->buf = static_cast<char*>(p);
    comm->buf_bytes = need;
  }
  // This rank's block: its own slot of the gather buffer on the root.
  char* mine = comm->buf + (is_root ? size_t(root) * L.bytes : 0);
  filtered_topk_enqueue(d_db, d_db_norms, shard_rows, dim, d_queries, n_queries, filter, row_offset, k, metric,
                        reinterpret_cast<float*>(mine), reinterpret_cast<int64_t*>(mine + L.id_off), s);
  const NcclApi& api = NcclApi::get();
  nccl_check(api.group_start(), "ncclGroupStart");
  if (is_root) {
    for (int p = 0; p < n; ++p)
      if (p != root) {
        const ncclResult_t r = api.recv(comm->buf + size_t(p) * L.bytes, L.bytes, ncclUint8, p, comm->comm, s);
        if (r != ncclSuccess) {
          api.group_end();
          nccl_check(r, "ncclRecv");
        }
      }
  } else {
    const ncclResult_t r = api.send(mine, L.bytes, ncclUint8, root, comm->comm, s);
    if (r != ncclSuccess) {
      api.group_end();
      nccl_check(r, "ncclSend");
    }
  }
  nccl_check(api.group_end(), "ncclGroupEnd");
  if (is_root)
    topk_merge_enqueue(reinterpret_cast<const float*>(comm->buf),
                       reinterpret_cast<const int64_t*>(comm->buf + L.id_off), L.bytes / 4, L.bytes / 8, uint32_t(n),
                       n_queries, k, metric, d_out_dist, d_out_ids, s);
  CR_API_END
}
