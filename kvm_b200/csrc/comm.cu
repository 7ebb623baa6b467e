// Collectives of the kernel dialect over NCCL (NVLink / NVSwitch on one
// node): kernel.comm.all_reduce.sum / .max, all_gather, broadcast,
// all_to_all, send, recv (src/ir/dialect/kernel/dialect.cpp:58-64; rank
// sets on kernel/ops.h:39-88). One process per GPU; a communicator per rank
// set (split from the world communicator).
//
// NCCL is opened at run time (libnccl.so.2): inside a Python process that
// already loaded torch's NCCL the same library is used, and the C ABI keeps
// no link-time dependency. Communicator setup is non-blocking and bounded:
// a rank that never joins makes init fail with KVM_ERR_TIMEOUT instead of
// hanging.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include "runtime.h"

struct kvm_comm {
  ncclComm_t comm = nullptr;
  int rank = 0;
  int nranks = 0;
};

namespace kvm {
namespace {

struct Nccl {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int,
                                     ncclConfig_t*) = nullptr;
  ncclResult_t (*CommSplit)(ncclComm_t, int, int, ncclComm_t*, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                            ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t,
                       cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t,
                       cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  std::string error;
};

template <typename F>
bool sym(void* h, const char* name, F* out) {
  *out = reinterpret_cast<F>(dlsym(h, name));
  return *out != nullptr;
}

const Nccl* nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      n.error = std::string("cannot open libnccl.so.2: ") + dlerror();
      return;
    }
    bool ok = sym(h, "ncclGetUniqueId", &n.GetUniqueId) &&
              sym(h, "ncclCommInitRankConfig", &n.CommInitRankConfig) &&
              sym(h, "ncclCommSplit", &n.CommSplit) &&
              sym(h, "ncclCommGetAsyncError", &n.CommGetAsyncError) &&
              sym(h, "ncclCommAbort", &n.CommAbort) &&
              sym(h, "ncclCommDestroy", &n.CommDestroy) &&
              sym(h, "ncclAllReduce", &n.AllReduce) &&
              sym(h, "ncclAllGather", &n.AllGather) &&
              sym(h, "ncclBroadcast", &n.Broadcast) && sym(h, "ncclSend", &n.Send) &&
              sym(h, "ncclRecv", &n.Recv) && sym(h, "ncclGroupStart", &n.GroupStart) &&
              sym(h, "ncclGroupEnd", &n.GroupEnd) &&
              sym(h, "ncclGetErrorString", &n.GetErrorString);
    if (!ok) n.error = "libnccl.so.2 lacks a required symbol (NCCL >= 2.18 needed)";
  });
  if (!n.error.empty()) {
    fail(KVM_ERR_UNSUPPORTED, n.error);
    return nullptr;
  }
  return &n;
}

int nccl_fail(const Nccl* n, ncclResult_t r, const char* what) {
  return fail(KVM_ERR_NCCL, std::string(what) + ": " + n->GetErrorString(r));
}

bool nccl_dtype(int dtype, ncclDataType_t* t, int* bytes) {
  switch (dtype) {
    case KVM_EW_BF16: *t = ncclBfloat16; *bytes = 2; return true;
    case KVM_EW_F16: *t = ncclFloat16; *bytes = 2; return true;
    case KVM_EW_F32: *t = ncclFloat32; *bytes = 4; return true;
    case KVM_EW_I32: *t = ncclInt32; *bytes = 4; return true;
    default: return false;
  }
}

// Wait (bounded) for a non-blocking communicator to finish its setup.
int wait_ready(const Nccl* n, ncclComm_t c, double seconds) {
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = n->CommGetAsyncError(c, &st);
    if (r != ncclSuccess) return nccl_fail(n, r, "ncclCommGetAsyncError");
    if (st == ncclSuccess) return KVM_OK;
    if (st != ncclInProgress) return nccl_fail(n, st, "communicator setup");
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() >
        seconds) {
      n->CommAbort(c);
      return fail(KVM_ERR_TIMEOUT, "communicator setup: a rank did not join in time");
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
}

// After enqueueing on a non-blocking communicator: ncclInProgress means the
// operation is queued; anything else but success is an error.
int enqueued(const Nccl* n, kvm_comm* c, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return KVM_OK;
  if (r == ncclInProgress) return wait_ready(n, c->comm, 60.0);
  return nccl_fail(n, r, what);
}

constexpr double kJoinSeconds = 60.0;

}  // namespace
}  // namespace kvm

using namespace kvm;

extern "C" int kvm_sm100_comm_unique_id(void* id) {
  const Nccl* n = nccl();
  if (!n) return KVM_ERR_UNSUPPORTED;
  if (!id) return fail(KVM_ERR_INVALID_ARG, "comm_unique_id: NULL");
  static_assert(sizeof(ncclUniqueId) == KVM_COMM_ID_BYTES, "unique id size");
  ncclResult_t r = n->GetUniqueId(static_cast<ncclUniqueId*>(id));
  return r == ncclSuccess ? KVM_OK : nccl_fail(n, r, "ncclGetUniqueId");
}

extern "C" int kvm_sm100_comm_init(int nranks, int rank, const void* id, kvm_comm** out) {
  const Nccl* n = nccl();
  if (!n) return KVM_ERR_UNSUPPORTED;
  if (!id || !out || nranks < 1 || rank < 0 || rank >= nranks)
    return fail(KVM_ERR_INVALID_ARG, "comm_init: bad argument");
  *out = nullptr;
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  auto* c = new kvm_comm;
  c->rank = rank;
  c->nranks = nranks;
  ncclResult_t r = n->CommInitRankConfig(&c->comm, nranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    delete c;
    return nccl_fail(n, r, "ncclCommInitRankConfig");
  }
  int rc = wait_ready(n, c->comm, kJoinSeconds);
  if (rc != KVM_OK) {
    delete c;
    return rc;
  }
  *out = c;
  return KVM_OK;
}

extern "C" int kvm_sm100_comm_split(kvm_comm* parent, const int32_t* ranks, int n_ranks,
                                    kvm_comm** out) {
  const Nccl* n = nccl();
  if (!n) return KVM_ERR_UNSUPPORTED;
  if (!parent || !ranks || n_ranks < 1 || !out)
    return fail(KVM_ERR_INVALID_ARG, "comm_split: bad argument");
  *out = nullptr;
  int key = -1;
  for (int i = 0; i < n_ranks; ++i) {
    if (ranks[i] < 0 || ranks[i] >= parent->nranks)
      return fail(KVM_ERR_INVALID_ARG, "comm_split: rank outside the communicator");
    if (ranks[i] == parent->rank) key = i;
  }
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t sub = nullptr;
  // Every rank of the parent takes part; non-members pass NCCL_SPLIT_NOCOLOR.
  ncclResult_t r = n->CommSplit(parent->comm, key >= 0 ? 0 : NCCL_SPLIT_NOCOLOR,
                                key >= 0 ? key : 0, &sub, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(n, r, "ncclCommSplit");
  int rc = wait_ready(n, parent->comm, kJoinSeconds);
  if (rc != KVM_OK) return rc;
  if (key < 0 || !sub) return KVM_OK;  // not a member: *out stays NULL
  rc = wait_ready(n, sub, kJoinSeconds);
  if (rc != KVM_OK) return rc;
  auto* c = new kvm_comm;
  c->comm = sub;
  c->rank = key;
  c->nranks = n_ranks;
  *out = c;
  return KVM_OK;
}

extern "C" int kvm_sm100_comm_rank(const kvm_comm* comm, int* rank, int* nranks) {
  if (!comm) return fail(KVM_ERR_INVALID_ARG, "comm_rank: NULL");
  if (rank) *rank = comm->rank;
  if (nranks) *nranks = comm->nranks;
  return KVM_OK;
}

extern "C" int kvm_sm100_comm_destroy(kvm_comm* comm) {
  if (!comm) return KVM_OK;
  const Nccl* n = nccl();
  if (!n) return KVM_ERR_UNSUPPORTED;
  ncclResult_t r = n->CommDestroy(comm->comm);
  delete comm;
  return r == ncclSuccess ? KVM_OK : nccl_fail(n, r, "ncclCommDestroy");
}

extern "C" int kvm_sm100_all_reduce(kvm_comm* comm, const void* send, void* recv,
                                    int64_t count, int dtype, int op, kvm_stream_t stream) {
  const Nccl* n = nccl();
  if (!n) return KVM_ERR_UNSUPPORTED;
  ncclDataType_t t;
  int es;
  if (!comm || !send || !recv || count < 0 || !nccl_dtype(dtype, &t, &es) ||
      (op != KVM_RED_SUM && op != KVM_RED_MAX))
    return fail(KVM_ERR_INVALID_ARG, "all_reduce: bad argument");
  return enqueued(n, comm,
                  n->AllReduce(send, recv, size_t(count), t, op == KVM_RED_SUM ? ncclSum : ncclMax,
                               comm->comm, static_cast<cudaStream_t>(stream)),
                  "ncclAllReduce");
}

extern "C" int kvm_sm100_all_gather(kvm_comm* comm, const void* send, void* recv,
                                    int64_t count, int dtype, kvm_stream_t stream) {
  const Nccl* n = nccl();
  if (!n) return KVM_ERR_UNSUPPORTED;
  ncclDataType_t t;
  int es;
  if (!comm || !send || !recv || count < 0 || !nccl_dtype(dtype, &t, &es))
    return fail(KVM_ERR_INVALID_ARG, "all_gather: bad argument");
  return enqueued(n, comm,
                  n->AllGather(send, recv, size_t(count), t, comm->comm,
                               static_cast<cudaStream_t>(stream)),
                  "ncclAllGather");
}

extern "C" int kvm_sm100_broadcast(kvm_comm* comm, const void* send, void* recv,
                                   int64_t count, int dtype, int root, kvm_stream_t stream) {
  const Nccl* n = nccl();
  if (!n) return KVM_ERR_UNSUPPORTED;
  ncclDataType_t t;
  int es;
  if (!comm || !recv || count < 0 || !nccl_dtype(dtype, &t, &es) || root < 0 ||
      root >= comm->nranks || (comm->rank == root && !send))
    return fail(KVM_ERR_INVALID_ARG, "broadcast: bad argument");
  return enqueued(n, comm,
                  n->Broadcast(send, recv, size_t(count), t, root, comm->comm,
                               static_cast<cudaStream_t>(stream)),
                  "ncclBroadcast");
}

extern "C" int kvm_sm100_send(kvm_comm* comm, const void* buf, int64_t count, int dtype,
                              int peer, kvm_stream_t stream) {
  const Nccl* n = nccl();
  if (!n) return KVM_ERR_UNSUPPORTED;
  ncclDataType_t t;
  int es;
  if (!comm || !buf || count < 0 || !nccl_dtype(dtype, &t, &es) || peer < 0 ||
      peer >= comm->nranks || peer == comm->rank)
    return fail(KVM_ERR_INVALID_ARG, "send: bad argument");
  return enqueued(n, comm,
                  n->Send(buf, size_t(count), t, peer, comm->comm,
                          static_cast<cudaStream_t>(stream)),
                  "ncclSend");
}

extern "C" int kvm_sm100_recv(kvm_comm* comm, void* buf, int64_t count, int dtype, int peer,
                              kvm_stream_t stream) {
  const Nccl* n = nccl();
  if (!n) return KVM_ERR_UNSUPPORTED;
  ncclDataType_t t;
  int es;
  if (!comm || !buf || count < 0 || !nccl_dtype(dtype, &t, &es) || peer < 0 ||
      peer >= comm->nranks || peer == comm->rank)
    return fail(KVM_ERR_INVALID_ARG, "recv: bad argument");
  return enqueued(n, comm,
                  n->Recv(buf, size_t(count), t, peer, comm->comm,
                          static_cast<cudaStream_t>(stream)),
                  "ncclRecv");
}

extern "C" int kvm_sm100_all_to_all(kvm_comm* comm, const void* send, void* recv,
                                    int64_t count, int dtype, kvm_stream_t stream) {
  const Nccl* n = nccl();
  if (!n) return KVM_ERR_UNSUPPORTED;
  ncclDataType_t t;
  int es;
  if (!comm || !send || !recv || count < 0 || !nccl_dtype(dtype, &t, &es))
    return fail(KVM_ERR_INVALID_ARG, "all_to_all: bad argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const char* s = static_cast<const char*>(send);
  char* r = static_cast<char*>(recv);
  const size_t chunk = size_t(count) * es;
  ncclResult_t g = n->GroupStart();
  if (g != ncclSuccess) return nccl_fail(n, g, "ncclGroupStart");
  for (int p = 0; p < comm->nranks; ++p) {
    ncclResult_t e1 = n->Send(s + p * chunk, size_t(count), t, p, comm->comm, st);
    ncclResult_t e2 = n->Recv(r + p * chunk, size_t(count), t, p, comm->comm, st);
    if ((e1 != ncclSuccess && e1 != ncclInProgress) ||
        (e2 != ncclSuccess && e2 != ncclInProgress)) {
      n->GroupEnd();
      return nccl_fail(n, e1 != ncclSuccess && e1 != ncclInProgress ? e1 : e2,
                       "all_to_all send/recv");
    }
  }
  return enqueued(n, comm, n->GroupEnd(), "ncclGroupEnd");
}
