// comm.cu -- the output all-gather of sample-sharded evaluation, over NCCL.
//
// Samples are independent, so a batch is split into contiguous shards, one per GPU (every GPU
// holds a full key replica generated from the same seed), each GPU evaluates its shard, and one
// all-gather of the output ciphertexts reassembles the batch on every rank.  The reference
// evaluates one sample on one CPU process (runtime/src/eval.rs:86-166) and has no collective;
// this is the exchange step that batching across GPUs adds.
//
// NCCL is opened at run time (dlopen of libnccl.so.2): a process that already loaded NCCL --
// PyTorch does -- shares that copy, one without it loads the system library, and a process that
// never creates a communicator needs no NCCL at all.  Equal shards go through one ncclAllGather;
// ragged ones through one grouped ncclBroadcast per rank straight into place (an all-gather-v),
// so no staging buffer is needed.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <new>

#include "pnb_internal.cuh"

namespace pnb {
void set_error(const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);
}  // namespace pnb
using pnb::set_error;

namespace {

struct Nccl {
  bool ok = false;
  const char* why = "not loaded";
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

Nccl& nccl() {
  static Nccl lib;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      lib.why = "libnccl.so.2 could not be opened";
      return;
    }
    bool all = true;
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      all = all && fn != nullptr;
    };
    sym(lib.get_unique_id, "ncclGetUniqueId");
    sym(lib.comm_init_rank, "ncclCommInitRank");
    sym(lib.comm_destroy, "ncclCommDestroy");
    sym(lib.comm_abort, "ncclCommAbort");
    sym(lib.comm_get_async_error, "ncclCommGetAsyncError");
    sym(lib.all_gather, "ncclAllGather");
    sym(lib.broadcast, "ncclBroadcast");
    sym(lib.group_start, "ncclGroupStart");
    sym(lib.group_end, "ncclGroupEnd");
    sym(lib.error_string, "ncclGetErrorString");
    lib.ok = all;
    if (!all) lib.why = "libnccl.so.2 lacks an expected entry point";
  });
  return lib;
}

int nccl_status(ncclResult_t r, const char* what) {
  set_error("%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
  return PNB_ERR_CUDA;
}

int need_nccl(const char* what) {
  if (nccl().ok) return PNB_OK;
  set_error("%s: NCCL unavailable (%s)", what, nccl().why);
  return PNB_ERR_UNSUPPORTED;
}

}  // namespace

struct pnb_comm {
  ncclComm_t comm = nullptr;
  int device = 0, world = 1, rank = 0;
};

extern "C" {

int pnb_shard(int64_t batch, int world, int rank, int64_t* start, int64_t* stop) {
  if (batch < 0 || world < 1 || rank < 0 || rank >= world || !start || !stop) {
    set_error("pnb_shard: need batch >= 0, 0 <= rank < world and output pointers");
    return PNB_ERR_INVALID;
  }
  const int64_t base = batch / world, extra = batch % world;
  *start = rank * base + (rank < extra ? rank : extra);
  *stop = *start + base + (rank < extra ? 1 : 0);
  return PNB_OK;
}

int pnb_comm_unique_id(void* id_out) {
  if (!id_out) {
    set_error("pnb_comm_unique_id: NULL output");
    return PNB_ERR_INVALID;
  }
  if (int rc = need_nccl("pnb_comm_unique_id")) return rc;
  ncclUniqueId id;
  ncclResult_t r = nccl().get_unique_id(&id);
  if (r != ncclSuccess) return nccl_status(r, "ncclGetUniqueId");
  static_assert(sizeof(id) == PNB_COMM_ID_BYTES, "NCCL unique id size");
  memcpy(id_out, &id, sizeof id);
  return PNB_OK;
}

int pnb_comm_create(int device, int world, int rank, const void* id, pnb_comm** out) {
  if (!id || !out || world < 1 || rank < 0 || rank >= world) {
    set_error("pnb_comm_create: need an id, an output pointer and 0 <= rank < world");
    return PNB_ERR_INVALID;
  }
  *out = nullptr;
  if (int rc = need_nccl("pnb_comm_create")) return rc;
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return pnb::cuda_status(e, "cudaGetDevice");
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return pnb::cuda_status(e, "cudaSetDevice");
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof uid);
  pnb_comm* c = new (std::nothrow) pnb_comm;
  int rc = PNB_OK;
  if (!c) {
    set_error("pnb_comm_create: out of host memory");
    rc = PNB_ERR_OOM;
  } else {
    ncclResult_t r = nccl().comm_init_rank(&c->comm, world, uid, rank);
    if (r != ncclSuccess) {
      rc = nccl_status(r, "ncclCommInitRank");
      delete c;
      c = nullptr;
    } else {
      c->device = device;
      c->world = world;
      c->rank = rank;
    }
  }
  if (prev >= 0 && prev != device) cudaSetDevice(prev);
  *out = c;
  return rc;
}

int pnb_comm_free(pnb_comm* c) {
  if (!c) return PNB_OK;
  int rc = PNB_OK;
  if (c->comm) {
    ncclResult_t r = nccl().comm_destroy(c->comm);
    if (r != ncclSuccess) rc = nccl_status(r, "ncclCommDestroy");
  }
  delete c;
  return rc;
}

int pnb_comm_abort(pnb_comm* c) {
  if (!c) return PNB_OK;
  int rc = PNB_OK;
  if (c->comm) {
    ncclResult_t r = nccl().comm_abort(c->comm);
    if (r != ncclSuccess) rc = nccl_status(r, "ncclCommAbort");
  }
  delete c;
  return rc;
}

int pnb_comm_info(const pnb_comm* c, int* device, int* world, int* rank) {
  if (!c) {
    set_error("pnb_comm_info: NULL communicator");
    return PNB_ERR_INVALID;
  }
  if (device) *device = c->device;
  if (world) *world = c->world;
  if (rank) *rank = c->rank;
  return PNB_OK;
}

int pnb_comm_status(const pnb_comm* c) {
  if (!c || !c->comm) {
    set_error("pnb_comm_status: NULL communicator");
    return PNB_ERR_INVALID;
  }
  ncclResult_t async = ncclSuccess;
  ncclResult_t r = nccl().comm_get_async_error(c->comm, &async);
  if (r != ncclSuccess) return nccl_status(r, "ncclCommGetAsyncError");
  if (async != ncclSuccess && async != ncclInProgress)
    return nccl_status(async, "pnb_comm_status (asynchronous error)");
  return PNB_OK;
}

int pnb_allgather(pnb_comm* c, const uint64_t* local_dev, uint64_t* out_dev, int64_t batch,
                  int64_t row_words, void* stream) {
  if (!c || !c->comm || batch < 0 || row_words <= 0 || (!out_dev && batch > 0)) {
    set_error("pnb_allgather: need a communicator, batch >= 0, row_words > 0 and an output");
    return PNB_ERR_INVALID;
  }
  int64_t s0 = 0, e0 = 0;
  pnb_shard(batch, c->world, c->rank, &s0, &e0);
  if (e0 > s0 && !local_dev) {
    set_error("pnb_allgather: this rank holds %lld rows but local_dev is NULL",
              (long long)(e0 - s0));
    return PNB_ERR_INVALID;
  }
  if (batch == 0) return PNB_OK;
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return pnb::cuda_status(e, "cudaGetDevice");
  if (prev != c->device && (e = cudaSetDevice(c->device)) != cudaSuccess)
    return pnb::cuda_status(e, "cudaSetDevice");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = PNB_OK;
  ncclResult_t r;
  if (batch % c->world == 0) {
    const size_t words = (size_t)(batch / c->world) * (size_t)row_words;
    r = nccl().all_gather(local_dev, out_dev, words, ncclUint64, c->comm, st);
    if (r != ncclSuccess) rc = nccl_status(r, "ncclAllGather");
  } else {
    r = nccl().group_start();
    if (r != ncclSuccess) {
      rc = nccl_status(r, "ncclGroupStart");
    } else {
      for (int q = 0; q < c->world && rc == PNB_OK; ++q) {
        int64_t a = 0, b = 0;
        pnb_shard(batch, c->world, q, &a, &b);
        if (b == a) continue;  // every rank computes the same shards, so all skip alike
        uint64_t* dst = out_dev + (size_t)a * (size_t)row_words;
        r = nccl().broadcast(q == c->rank ? local_dev : dst, dst,
                             (size_t)(b - a) * (size_t)row_words, ncclUint64, q, c->comm, st);
        if (r != ncclSuccess) rc = nccl_status(r, "ncclBroadcast");
      }
      r = nccl().group_end();
      if (r != ncclSuccess && rc == PNB_OK) rc = nccl_status(r, "ncclGroupEnd");
    }
  }
  if (prev >= 0 && prev != c->device) cudaSetDevice(prev);
  return rc;
}

}  // extern "C"
