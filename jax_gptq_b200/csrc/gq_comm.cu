// Per-device handle with an optional NCCL communicator, and the in-place fp32
// all-reduce that sums token-sharded Hessians across GPUs.  The reference has
// no multi-device path; these are the C-ABI counterparts of what
// jax_gptq_b200/distributed.py does through torch.distributed.
//
// NCCL is opened with dlopen on first use (an already-loaded copy in the
// process is reused, e.g. the one a framework brought), so the library itself
// does not depend on libnccl and loads on hosts without it.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "gq_common.cuh"

namespace gq {
int64_t sym_packed_size(int64_t d);
int sym_pack(const float* h, int64_t d, int64_t ldh, float* packed, cudaStream_t st);
int sym_unpack(const float* packed, int64_t d, float* h, int64_t ldh, cudaStream_t st);
}  // namespace gq

struct gq_handle {
  int device;
  ncclComm_t comm;  // NULL: no collectives
  int owns_comm;
  int nranks;
  int rank;
  int aborted;      // the communicator was aborted (gq_comm_check / gq_handle_abort)
};

namespace gq {
namespace comm {

struct Api {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_count)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*comm_user_rank)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  bool ok = false;
};

static const Api& api() {
  static Api a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    a.comm_count = reinterpret_cast<decltype(a.comm_count)>(dlsym(h, "ncclCommCount"));
    a.comm_user_rank = reinterpret_cast<decltype(a.comm_user_rank)>(dlsym(h, "ncclCommUserRank"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    a.get_async_error =
        reinterpret_cast<decltype(a.get_async_error)>(dlsym(h, "ncclCommGetAsyncError"));
    a.comm_abort = reinterpret_cast<decltype(a.comm_abort)>(dlsym(h, "ncclCommAbort"));
    a.ok = a.get_unique_id && a.comm_init_rank && a.comm_destroy && a.comm_count &&
           a.comm_user_rank && a.all_reduce && a.error_string && a.get_async_error &&
           a.comm_abort;
  });
  return a;
}

static int nccl_fail(const char* what, ncclResult_t r) {
  return fail(GQ_ENCCL, "%s: %s", what, api().error_string ? api().error_string(r) : "NCCL error");
}

// Makes `device` current for the scope and restores the previous device.
struct DeviceScope {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit DeviceScope(int device) {
    err = cudaGetDevice(&prev);
    if (err == cudaSuccess && prev != device) err = cudaSetDevice(device);
  }
  ~DeviceScope() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace comm
}  // namespace gq

extern "C" {

int gq_nccl_unique_id(void* id_out, int64_t id_bytes) {
  GQ_REQUIRE(id_out != nullptr && id_bytes >= (int64_t)sizeof(ncclUniqueId),
             "gq_nccl_unique_id: need a buffer of at least %d bytes", (int)sizeof(ncclUniqueId));
  const auto& a = gq::comm::api();
  if (!a.ok) return gq::fail(GQ_ENCCL, "gq_nccl_unique_id: libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  ncclResult_t r = a.get_unique_id(&id);
  if (r != ncclSuccess) return gq::comm::nccl_fail("ncclGetUniqueId", r);
  std::memcpy(id_out, &id, sizeof(id));
  return GQ_OK;
}

int gq_handle_create(int device, void* nccl_comm, gq_handle** out) {
  GQ_REQUIRE(out != nullptr, "gq_handle_create: NULL out");
  GQ_REQUIRE(device >= 0, "gq_handle_create: bad device %d", device);
  int nranks = 1, rank = 0;
  if (nccl_comm) {
    const auto& a = gq::comm::api();
    if (!a.ok) return gq::fail(GQ_ENCCL, "gq_handle_create: libnccl.so.2 could not be loaded");
    ncclResult_t r = a.comm_count(static_cast<ncclComm_t>(nccl_comm), &nranks);
    if (r == ncclSuccess) r = a.comm_user_rank(static_cast<ncclComm_t>(nccl_comm), &rank);
    if (r != ncclSuccess) return gq::comm::nccl_fail("gq_handle_create", r);
  }
  *out = new gq_handle{device, static_cast<ncclComm_t>(nccl_comm), 0, nranks, rank, 0};
  return GQ_OK;
}

int gq_handle_create_nccl(int device, const void* unique_id, int nranks, int rank,
                          gq_handle** out) {
  GQ_REQUIRE(out != nullptr && unique_id != nullptr, "gq_handle_create_nccl: NULL argument");
  GQ_REQUIRE(device >= 0 && nranks >= 1 && rank >= 0 && rank < nranks,
             "gq_handle_create_nccl: bad device %d / rank %d of %d", device, rank, nranks);
  const auto& a = gq::comm::api();
  if (!a.ok) return gq::fail(GQ_ENCCL, "gq_handle_create_nccl: libnccl.so.2 could not be loaded");
  gq::comm::DeviceScope scope(device);
  GQ_CHECK_CUDA(scope.err);
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  ncclComm_t comm = nullptr;
  ncclResult_t r = a.comm_init_rank(&comm, nranks, id, rank);
  if (r != ncclSuccess) return gq::comm::nccl_fail("ncclCommInitRank", r);
  *out = new gq_handle{device, comm, 1, nranks, rank, 0};
  return GQ_OK;
}

int gq_handle_destroy(gq_handle* h) {
  if (!h) return GQ_OK;
  int status = GQ_OK;
  if (h->comm && h->owns_comm) {
    gq::comm::DeviceScope scope(h->device);
    ncclResult_t r = gq::comm::api().comm_destroy(h->comm);
    if (r != ncclSuccess) status = gq::comm::nccl_fail("ncclCommDestroy", r);
  }
  delete h;
  return status;
}

int gq_handle_ranks(const gq_handle* h, int* nranks, int* rank) {
  GQ_REQUIRE(h != nullptr, "gq_handle_ranks: NULL handle");
  if (nranks) *nranks = h->nranks;
  if (rank) *rank = h->rank;
  return GQ_OK;
}

int gq_comm_check(gq_handle* h, int abort_on_error) {
  GQ_REQUIRE(h != nullptr, "gq_comm_check: NULL handle");
  if (h->aborted) return gq::fail(GQ_ENCCL, "gq_comm_check: the communicator was aborted");
  if (h->comm == nullptr) return GQ_OK;
  const auto& a = gq::comm::api();
  ncclResult_t async = ncclSuccess;
  ncclResult_t r = a.get_async_error(h->comm, &async);
  if (r != ncclSuccess) return gq::comm::nccl_fail("ncclCommGetAsyncError", r);
  if (async == ncclSuccess || async == ncclInProgress) return GQ_OK;
  if (abort_on_error && h->owns_comm) {
    gq::comm::DeviceScope scope(h->device);
    a.comm_abort(h->comm);  // ends this rank's outstanding collectives
    h->comm = nullptr;
    h->aborted = 1;
  }
  return gq::fail(GQ_ENCCL, "NCCL asynchronous error on rank %d of %d: %s%s", h->rank, h->nranks,
                  a.error_string(async), h->aborted ? " (communicator aborted)" : "");
}

int gq_handle_abort(gq_handle* h) {
  GQ_REQUIRE(h != nullptr, "gq_handle_abort: NULL handle");
  GQ_REQUIRE(h->owns_comm || h->comm == nullptr,
             "gq_handle_abort: the communicator belongs to the caller; abort it there");
  if (h->comm) {
    gq::comm::DeviceScope scope(h->device);
    ncclResult_t r = gq::comm::api().comm_abort(h->comm);
    h->comm = nullptr;
    h->aborted = 1;
    if (r != ncclSuccess) return gq::comm::nccl_fail("ncclCommAbort", r);
  }
  h->aborted = 1;
  return GQ_OK;
}

int gq_allreduce_sum_f32(gq_handle* h, float* buf, int64_t count, void* stream) {
  GQ_REQUIRE(h != nullptr, "gq_allreduce_sum_f32: NULL handle");
  if (h->aborted) return gq::fail(GQ_ENCCL, "gq_allreduce_sum_f32: the communicator was aborted");
  GQ_REQUIRE(h->comm != nullptr, "gq_allreduce_sum_f32: the handle has no communicator");
  GQ_REQUIRE(count >= 0 && (count == 0 || buf != nullptr), "gq_allreduce_sum_f32: bad buffer");
  if (count == 0) return GQ_OK;
  gq::comm::DeviceScope scope(h->device);
  GQ_CHECK_CUDA(scope.err);
  ncclResult_t r = gq::comm::api().all_reduce(buf, buf, (size_t)count, ncclFloat32, ncclSum,
                                              h->comm, gq::as_stream(stream));
  if (r != ncclSuccess) return gq::comm::nccl_fail("ncclAllReduce", r);
  return GQ_OK;
}

int gq_allreduce_sym_f32(gq_handle* h, float* x, int64_t d, int64_t ldx, float* packed,
                         void* stream) {
  GQ_REQUIRE(h != nullptr, "gq_allreduce_sym_f32: NULL handle");
  if (h->aborted) return gq::fail(GQ_ENCCL, "gq_allreduce_sym_f32: the communicator was aborted");
  GQ_REQUIRE(h->comm != nullptr, "gq_allreduce_sym_f32: the handle has no communicator");
  GQ_REQUIRE(d >= 0 && d <= (int64_t)INT32_MAX && (d == 0 || (x != nullptr && packed != nullptr &&
                                                               ldx >= d)),
             "gq_allreduce_sym_f32: bad arguments (d=%lld ldx=%lld)", (long long)d,
             (long long)ldx);
  if (d == 0) return GQ_OK;
  gq::comm::DeviceScope scope(h->device);
  GQ_CHECK_CUDA(scope.err);
  cudaStream_t st = gq::as_stream(stream);
  GQ_TRY(gq::sym_pack(x, d, ldx, packed, st));
  ncclResult_t r = gq::comm::api().all_reduce(packed, packed, (size_t)gq::sym_packed_size(d),
                                              ncclFloat32, ncclSum, h->comm, st);
  if (r != ncclSuccess) return gq::comm::nccl_fail("ncclAllReduce", r);
  return gq::sym_unpack(packed, d, x, ldx, st);
}

}  // extern "C"
