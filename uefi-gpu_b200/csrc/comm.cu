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
// Both collectives are the library's own one-shot kernels over NVLink peer memory: every rank
// pushes its slice of the data into a slot of every rank's receive area with plain peer stores,
// raises a flag there (release, system scope), waits for every rank's flag of the slice (acquire,
// bounded by the wait limit) and reduces the slots in rank order -- so every rank computes the
// same bits, in about one NVLink round trip, as an ordinary kernel captured in the decode graph.
// Receive areas are double-buffered by the parity of a per-CTA epoch, so a rank can run one call
// ahead of a peer without overwriting data the peer still reads.  NCCL (loaded at run time) only
// creates the communicator and exchanges the areas' IPC handles once.  No multicast, no TMA.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "common.cuh"
#include "internal.hpp"

namespace ugb {

constexpr int kCommMaxRanks = 8;
constexpr int kCommMaxCtas = 32;          // slices of one call
constexpr int kCommSlice = 1024;          // 4-byte words per CTA slice
constexpr int64_t kCommCapWords = static_cast<int64_t>(kCommMaxCtas) * kCommSlice;  // per slot

// Receive area of one rank: data [parity 2][rank][kCommCapWords] words, then flags [2][rank][CTA].
struct PeerArea {
  uint32_t *base[kCommMaxRanks];  // each rank's area, mapped into this process
};
constexpr size_t comm_area_data_words() { return 2ull * kCommMaxRanks * kCommCapWords; }
constexpr size_t comm_area_bytes() {
  return (comm_area_data_words() + 2ull * kCommMaxRanks * kCommMaxCtas) * sizeof(uint32_t);
}

}  // namespace ugb

struct ugb_comm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, device = 0;
  uint32_t *area = nullptr;     // this rank's receive area (peers write into it)
  uint32_t *epochs = nullptr;   // [kCommMaxCtas] calls completed, per CTA slice
  ugb::PeerArea peers{};        // every rank's area as mapped here (peers' through IPC)
  uint64_t wait_ns = ugb::kWaitLimitNs;
  uint32_t *status = nullptr;   // the context's status word
};

namespace ugb {
namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
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
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather;
  });
  return api;
}

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

enum : int { kOpSumF32 = 0, kOpMaxU64 = 1 };

struct AllReduceArgs {
  PeerArea peers;
  uint32_t *buf;      // local data, reduced in place: n 4-byte words (f32) or n/2 u64
  uint32_t *epochs;   // [kCommMaxCtas]
  uint32_t *status;
  uint64_t wait_ns;
  int64_t n;          // 4-byte words
  int rank, world;
};

// CTA c reduces words [c * kCommSlice, ...) of the buffer over the ranks.
template <int OP>
__global__ void __launch_bounds__(256) p2p_allreduce_kernel(const AllReduceArgs a) {
  __shared__ int ok_s;
  const int c = blockIdx.x, tid = threadIdx.x;
  const int64_t w0 = static_cast<int64_t>(c) * kCommSlice;
  const int len = static_cast<int>(a.n - w0 < kCommSlice ? a.n - w0 : kCommSlice);
  const uint32_t e = a.epochs[c] + 1;
  const int par = e & 1;
  // 1. this rank's slice into slot [par][rank] of every rank's area (the own one included)
  const bool vec = (reinterpret_cast<uintptr_t>(a.buf) & 15) == 0;  // slots are 16-byte aligned
  for (int r = 0; r < a.world; ++r) {
    uint32_t *dst = a.peers.base[r] + (static_cast<int64_t>(par) * kCommMaxRanks + a.rank) * kCommCapWords + w0;
    const int nv = vec ? len / 4 : 0;
    for (int i = tid; i < nv; i += blockDim.x)
      reinterpret_cast<uint4 *>(dst)[i] = reinterpret_cast<const uint4 *>(a.buf + w0)[i];
    for (int i = nv * 4 + tid; i < len; i += blockDim.x) dst[i] = a.buf[w0 + i];
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();  // the slice's stores before the flags, at system scope
    for (int r = 0; r < a.world; ++r)
      st_release_sys(a.peers.base[r] + comm_area_data_words() + (par * kCommMaxRanks + a.rank) * kCommMaxCtas + c, e);
    // 2. every rank's flag for this slice, in this rank's own area (bounded wait)
    const uint32_t *flags = a.peers.base[a.rank] + comm_area_data_words() + par * kCommMaxRanks * kCommMaxCtas + c;
    const uint64_t t0 = globaltimer_ns();
    int ok = 1;
    for (int r = 0; r < a.world && ok; ++r)
      while (ld_acquire_sys(flags + r * kCommMaxCtas) != e)
        if (globaltimer_ns() - t0 > a.wait_ns) {
          ok = 0;
          status_or(a.status, ST_TIMEOUT);
          break;
        }
    ok_s = ok;
  }
  __syncthreads();
  if (!ok_s) return;  // a peer never arrived: the result is not valid (status says so)
  // 3. the slots reduced in rank order
  // (through L2: the slots were written by other GPUs since this SM last read them)
  const uint32_t *slots = a.peers.base[a.rank] + static_cast<int64_t>(par) * kCommMaxRanks * kCommCapWords + w0;
  if (OP == kOpSumF32) {
    for (int i = tid; i < len; i += blockDim.x) {
      float v = __uint_as_float(__ldcg(slots + i));
      for (int r = 1; r < a.world; ++r) v += __uint_as_float(__ldcg(slots + r * kCommCapWords + i));
      a.buf[w0 + i] = __float_as_uint(v);
    }
  } else {
    for (int i = tid; 2 * i < len; i += blockDim.x) {
      unsigned long long v = __ldcg(reinterpret_cast<const unsigned long long *>(slots) + i);
      for (int r = 1; r < a.world; ++r)
        v = max(v, __ldcg(reinterpret_cast<const unsigned long long *>(slots + r * kCommCapWords) + i));
      reinterpret_cast<unsigned long long *>(a.buf + w0)[i] = v;
    }
  }
  __syncthreads();
  if (tid == 0) a.epochs[c] = e;
}

ugb_status launch_allreduce(ugb_comm *c, int op, uint32_t *buf, int64_t words, cudaStream_t stream) {
  if (!c || !c->area) return UGB_EBACKEND;
  if (words < 1 || words > kCommCapWords || (op == kOpMaxU64 && (words & 1))) return UGB_ESHAPE;
  if ((reinterpret_cast<uintptr_t>(buf) & (op == kOpMaxU64 ? 7 : 3)) != 0) return UGB_EALIGN;
  AllReduceArgs a;
  a.peers = c->peers;
  a.buf = buf;
  a.epochs = c->epochs;
  a.status = c->status;
  a.wait_ns = c->wait_ns;
  a.n = words;
  a.rank = c->rank;
  a.world = c->world;
  const unsigned ctas = static_cast<unsigned>((words + kCommSlice - 1) / kCommSlice);
  if (op == kOpSumF32)
    p2p_allreduce_kernel<kOpSumF32><<<ctas, 256, 0, stream>>>(a);
  else
    p2p_allreduce_kernel<kOpMaxU64><<<ctas, 256, 0, stream>>>(a);
  return cuda_status(cudaGetLastError());
}

}  // namespace

ugb_status comm_allreduce_sum_f32(ugb_comm *c, float *buf, size_t n, cudaStream_t stream) {
  return launch_allreduce(c, kOpSumF32, reinterpret_cast<uint32_t *>(buf), static_cast<int64_t>(n), stream);
}

ugb_status comm_allreduce_max_u64(ugb_comm *c, unsigned long long *buf, size_t n, cudaStream_t stream) {
  return launch_allreduce(c, kOpMaxU64, reinterpret_cast<uint32_t *>(buf), 2 * static_cast<int64_t>(n), stream);
}

int comm_world(const ugb_comm *c) { return c ? c->world : 1; }

}  // namespace ugb

namespace ugb {
namespace {

// This rank's receive area (zeroed) and its IPC handle all-gathered over NCCL; every peer's area
// mapped into this process.  The all-gather also orders every rank's zeroing before any write.
ugb_status open_areas(ugb_comm *c) {
  if (c->world > kCommMaxRanks) return UGB_ESHAPE;
  if (cudaMalloc(reinterpret_cast<void **>(&c->area), comm_area_bytes()) != cudaSuccess ||
      cudaMemset(c->area, 0, comm_area_bytes()) != cudaSuccess ||
      cudaMalloc(reinterpret_cast<void **>(&c->epochs), kCommMaxCtas * sizeof(uint32_t)) != cudaSuccess ||
      cudaMemset(c->epochs, 0, kCommMaxCtas * sizeof(uint32_t)) != cudaSuccess)
    return UGB_EBACKEND;
  c->peers.base[c->rank] = c->area;
  if (c->world == 1) return UGB_OK;
  cudaIpcMemHandle_t mine;
  if (cudaIpcGetMemHandle(&mine, c->area) != cudaSuccess) return UGB_EBACKEND;
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  void *dev = nullptr;
  if (cudaMalloc(&dev, hb * (c->world + 1)) != cudaSuccess) return UGB_EBACKEND;
  std::vector<uint8_t> all(hb * c->world);
  bool ok = cudaMemcpy(dev, &mine, hb, cudaMemcpyHostToDevice) == cudaSuccess &&
            nccl().all_gather(dev, static_cast<uint8_t *>(dev) + hb, hb, ncclUint8, c->comm, nullptr) == ncclSuccess &&
            cudaDeviceSynchronize() == cudaSuccess &&
            cudaMemcpy(all.data(), static_cast<uint8_t *>(dev) + hb, all.size(), cudaMemcpyDeviceToHost) == cudaSuccess;
  cudaFree(dev);
  for (int r = 0; ok && r < c->world; ++r) {
    if (r == c->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, all.data() + r * hb, hb);
    void *p = nullptr;
    ok = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    c->peers.base[r] = static_cast<uint32_t *>(p);
  }
  return ok ? UGB_OK : UGB_EBACKEND;
}

}  // namespace
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
  c->status = ctx->status;
  const ugb_status st = open_areas(c);
  if (st != UGB_OK) {
    ugb_comm_destroy(c);
    return st;
  }
  *out = c;
  return UGB_OK;
}

ugb_status ugb_comm_destroy(ugb_comm *c) {
  if (!c) return UGB_ECONTEXT;
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  for (int r = 0; r < c->world && r < kCommMaxRanks; ++r)
    if (r != c->rank && c->peers.base[r]) cudaIpcCloseMemHandle(c->peers.base[r]);
  if (nccl().ok && c->comm) nccl().comm_destroy(c->comm);  // a barrier of sorts: peers are done
  if (c->area) cudaFree(c->area);
  if (c->epochs) cudaFree(c->epochs);
  delete c;
  return UGB_OK;
}

ugb_status ugb_comm_allreduce_f32(ugb_comm *c, ugb_stream stream, float *buf_dev, int64_t n) {
  if (!c) return UGB_ECONTEXT;
  if (cudaSetDevice(c->device) != cudaSuccess) return UGB_EBACKEND;
  return comm_allreduce_sum_f32(c, buf_dev, static_cast<size_t>(n), stream);
}

ugb_status ugb_comm_allreduce_max_u64(ugb_comm *c, ugb_stream stream, uint64_t *buf_dev, int64_t n) {
  if (!c) return UGB_ECONTEXT;
  if (cudaSetDevice(c->device) != cudaSuccess) return UGB_EBACKEND;
  return comm_allreduce_max_u64(c, reinterpret_cast<unsigned long long *>(buf_dev), static_cast<size_t>(n), stream);
}

}  // extern "C"
