// comm.cu -- the collectives of a sharded decode step over NCCL (NVLink / NVSwitch), loaded at
// run time so the library itself loads where NCCL is absent (the entry points then fail with
// UGB_EBACKEND).
//
// The hot path shards in two places (the reference runs on one GPU; these are the B200 forms
// of its expert loop and vocabulary projection):
//   * expert parallelism: each device holds a range of every MoE layer's experts and computes
//     the weighted sum of the held experts' outputs; one all-reduce (sum) of the layer's
//     [batch][hidden] output combines the devices;
//   * vocabulary row split: each device holds a range of head rows and finds the greedy
//     (value, lowest id) key of its range; one all-reduce (max) of the batch's 64-bit keys gives
//     the global greedy token -- exactly the argmax of the all-gathered logits, for 8 bytes per
//     sequence instead of 4 * n_vocab.
// Both are plain NCCL calls on the decode stream, so they are captured in the decoder's CUDA
// graph with the kernels around them.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <new>

#include "internal.hpp"

struct ugb_comm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, device = 0;
};

namespace ugb {
namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
};

NcclApi &nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    // the process's NCCL if one is loaded already (torch's), else the system one
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce;
  });
  return api;
}

}  // namespace

ugb_status comm_allreduce_sum_f32(ugb_comm *c, float *buf, size_t n, cudaStream_t stream) {
  if (!c || !nccl().ok) return UGB_EBACKEND;
  return nccl().all_reduce(buf, buf, n, ncclFloat32, ncclSum, c->comm, stream) == ncclSuccess ? UGB_OK
                                                                                               : UGB_EBACKEND;
}

ugb_status comm_allreduce_max_u64(ugb_comm *c, unsigned long long *buf, size_t n, cudaStream_t stream) {
  if (!c || !nccl().ok) return UGB_EBACKEND;
  return nccl().all_reduce(buf, buf, n, ncclUint64, ncclMax, c->comm, stream) == ncclSuccess ? UGB_OK
                                                                                              : UGB_EBACKEND;
}

int comm_world(const ugb_comm *c) { return c ? c->world : 1; }

}  // namespace ugb

using namespace ugb;

extern "C" {

ugb_status ugb_comm_unique_id(uint8_t *id_out) {
  if (!id_out) return UGB_EALIGN;
  if (!nccl().ok) return UGB_EBACKEND;
  ncclUniqueId id;
  if (nccl().get_unique_id(&id) != ncclSuccess) return UGB_EBACKEND;
  std::memcpy(id_out, id.internal, UGB_COMM_ID_BYTES);
  return UGB_OK;
}

ugb_status ugb_comm_init(ugb_ctx *ctx, int rank, int world, const uint8_t *id, ugb_comm **out) {
  if (!ctx || !out) return UGB_ECONTEXT;
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world || !id) return UGB_ESHAPE;
  if (!nccl().ok) return UGB_EBACKEND;
  if (cudaSetDevice(ctx->device) != cudaSuccess) return UGB_EBACKEND;
  ncclUniqueId uid;
  std::memcpy(uid.internal, id, UGB_COMM_ID_BYTES);
  ugb_comm *c = new (std::nothrow) ugb_comm();
  if (!c) return UGB_EBACKEND;
  if (nccl().comm_init_rank(&c->comm, world, uid, rank) != ncclSuccess) {
    delete c;
    return UGB_EBACKEND;
  }
  c->rank = rank;
  c->world = world;
  c->device = ctx->device;
  *out = c;
  return UGB_OK;
}

ugb_status ugb_comm_destroy(ugb_comm *c) {
  if (!c) return UGB_ECONTEXT;
  if (nccl().ok && c->comm) nccl().comm_destroy(c->comm);
  delete c;
  return UGB_OK;
}

}  // extern "C"
