// K9: the cross-GPU gradient mean. boonta never calls a collective itself: XLA's SPMD
// partitioner inserts an all-reduce because params are replicated and the batch is
// sharded on "data" (boonta/podracers/anakin.py:165-186). Here each learner handle owns
// one NCCL communicator (one rank per GPU of an NVLink/NVSwitch box) and the learner
// issues one ncclAllReduce(sum, fp32) per minibatch on the flat gradient buffer, on the
// learner's stream. Because every rank's loss terms are already scaled by 1/mb_global,
// the sum is the exact global-minibatch gradient, and the identical reduced bytes keep
// the replicated parameters bitwise equal on every rank.
//
// NCCL is resolved with dlopen at communicator creation, so single-GPU use of the
// library carries no NCCL dependency.
#include <dlfcn.h>

#include "learner.h"
#include "nccl.h"

namespace bt {

struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

static NcclApi g_nccl;

static int load_nccl() {
  if (g_nccl.handle) return BT_OK;
  const char* names[] = {"libnccl.so.2", "libnccl.so"};
  void* h = nullptr;
  for (const char* n : names) {
    h = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
    if (h) break;
  }
  if (!h) {
    set_error("could not load NCCL (libnccl.so.2): %s", dlerror());
    return BT_ERR_NCCL;
  }
  g_nccl.GetUniqueId = (decltype(g_nccl.GetUniqueId))dlsym(h, "ncclGetUniqueId");
  g_nccl.CommInitRank = (decltype(g_nccl.CommInitRank))dlsym(h, "ncclCommInitRank");
  g_nccl.AllReduce = (decltype(g_nccl.AllReduce))dlsym(h, "ncclAllReduce");
  g_nccl.AllGather = (decltype(g_nccl.AllGather))dlsym(h, "ncclAllGather");
  g_nccl.CommDestroy = (decltype(g_nccl.CommDestroy))dlsym(h, "ncclCommDestroy");
  g_nccl.GetErrorString = (decltype(g_nccl.GetErrorString))dlsym(h, "ncclGetErrorString");
  if (!g_nccl.GetUniqueId || !g_nccl.CommInitRank || !g_nccl.AllReduce || !g_nccl.AllGather ||
      !g_nccl.CommDestroy ||
      !g_nccl.GetErrorString) {
    set_error("NCCL library lacks a required symbol");
    return BT_ERR_NCCL;
  }
  g_nccl.handle = h;
  return BT_OK;
}

#define BT_NCCL(call)                                                                    \
  do {                                                                                   \
    ncclResult_t r_ = (call);                                                            \
    if (r_ != ncclSuccess) {                                                             \
      set_error("%s:%d: %s failed: %s", __FILE__, __LINE__, #call,                       \
                g_nccl.GetErrorString ? g_nccl.GetErrorString(r_) : "?");                \
      return BT_ERR_NCCL;                                                                \
    }                                                                                    \
  } while (0)

}  // namespace bt

struct Comm {
  ncclComm_t comm = nullptr;
  int rank = 0, size = 1;
};

namespace bt {

int comm_allreduce_f32(Comm* c, float* buf, size_t n, cudaStream_t stream) {
  BT_NCCL(g_nccl.AllReduce(buf, buf, n, ncclFloat32, ncclSum, c->comm, stream));
  return BT_OK;
}

int comm_allreduce_f64(Comm* c, double* buf, size_t n, cudaStream_t stream) {
  BT_NCCL(g_nccl.AllReduce(buf, buf, n, ncclFloat64, ncclSum, c->comm, stream));
  return BT_OK;
}

// Blocking all-gather of `bytes` host bytes per rank through the communicator (set-up only).
static int comm_allgather_host(void* ctx, const void* send, void* recv, size_t bytes) {
  Comm* c = static_cast<Comm*>(ctx);
  uint8_t* d = nullptr;
  BT_CUDA(cudaMalloc(&d, bytes * (c->size + 1)));
  int rc = BT_OK;
  if (cudaMemcpy(d, send, bytes, cudaMemcpyHostToDevice) != cudaSuccess) rc = BT_ERR_CUDA;
  if (rc == BT_OK) {
    ncclResult_t r = g_nccl.AllGather(d, d + bytes, bytes, ncclUint8, c->comm, 0);
    if (r != ncclSuccess) {
      set_error("ncclAllGather failed: %s", g_nccl.GetErrorString(r));
      rc = BT_ERR_NCCL;
    }
  }
  if (rc == BT_OK && cudaStreamSynchronize(0) != cudaSuccess) rc = BT_ERR_CUDA;
  if (rc == BT_OK &&
      cudaMemcpy(recv, d + bytes, bytes * c->size, cudaMemcpyDeviceToHost) != cudaSuccess)
    rc = BT_ERR_CUDA;
  if (rc == BT_ERR_CUDA) set_error("comm_allgather_host: CUDA copy failed");
  cudaFree(d);
  return rc;
}

void comm_destroy(Comm* c) {
  if (c && c->comm && g_nccl.CommDestroy) g_nccl.CommDestroy(c->comm);
  delete c;
}

}  // namespace bt

using namespace bt;

extern "C" int bt_nccl_unique_id(void* out, int32_t size) {
  BT_CHECK_ARG(out && size >= (int32_t)sizeof(ncclUniqueId), "unique id buffer of %d bytes",
               size);
  BT_TRY(load_nccl());
  ncclUniqueId id;
  BT_NCCL(g_nccl.GetUniqueId(&id));
  memcpy(out, &id, sizeof(id));
  return BT_OK;
}

extern "C" int bt_learner_comm_init(bt_learner* L, const void* unique_id, int32_t size) {
  BT_CHECK_ARG(L && unique_id && size >= (int32_t)sizeof(ncclUniqueId),
               "bt_learner_comm_init: bad argument");
  BT_CHECK_ARG(L->comm == nullptr, "communicator already initialised");
  BT_TRY(load_nccl());
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  Comm* c = new Comm();
  c->rank = L->cfg.rank;
  c->size = L->cfg.world_size;
  ncclResult_t r = g_nccl.CommInitRank(&c->comm, c->size, id, c->rank);
  if (r != ncclSuccess) {
    set_error("ncclCommInitRank(rank %d of %d) failed: %s", c->rank, c->size,
              g_nccl.GetErrorString(r));
    delete c;
    return BT_ERR_NCCL;
  }
  L->comm = c;
  // the NVLink peer-memory exchange (exchange.cu) when every rank can map every peer
  return exchange_create(L, comm_allgather_host, c);
}
