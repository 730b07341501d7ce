// linear_static.cu -- ugb_linear_static: the host-buffer linear layer of ugb_linear, with its
// device scratch in a fixed array compiled into the library instead of a workspace grown with
// cudaMalloc.
//
// Why a second form exists: ugb_linear grows a per-context workspace (cudaMalloc and pinned
// cudaMallocHost) the first time it meets a larger k or m.  Some callers cannot let a library
// allocate behind their back: a host that plans all device memory up front (as the reference's
// firmware host does with fixed VRAM arenas), a serving loop that must not see the implicit
// device synchronisation or the out-of-memory failure an allocation can bring mid-run, or code
// running where allocation calls are not allowed.  This form touches no allocator at all: the
// scratch is a file-scope __device__ array, its address is looked up once per device with
// cudaGetSymbolAddress, and the host buffers are copied directly.
//
// Limits: k <= UGB_LINEAR_STATIC_MAX_K (16384, the reference's n cap) and m <=
// UGB_LINEAR_STATIC_MAX_M (524288, i.e. m*4 <= 2 MiB, the reference's output cap,
// frontier_backend.rs:245-248); the array is 2,183,168 bytes.  Nothing in it has to start at
// zero: every byte a call reads was written earlier in the same call.  The array is shared by
// every context and stream on a device, so calls that overlap in time on one device race.
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "internal.hpp"

namespace ugb {
namespace {

constexpr int64_t kStaticMaxK = UGB_LINEAR_STATIC_MAX_K;
constexpr int64_t kStaticMaxM = UGB_LINEAR_STATIC_MAX_M;
// [x: f32 k][xq: Q8_1 of k][y: f32 m], each region 256-byte aligned.
constexpr size_t kXBytes = kStaticMaxK * 4;                                  // 65,536
constexpr size_t kXqBytes = kStaticMaxK + 2 * ((kStaticMaxK / 32 * 4 + 255) / 256 * 256);  // 20,480
constexpr size_t kYBytes = kStaticMaxM * 4;                                  // 2,097,152
constexpr size_t kXqOff = kXBytes;
constexpr size_t kYOff = kXqOff + kXqBytes;
constexpr size_t kScratchBytes = kYOff + kYBytes;                            // 2,183,168
static_assert(kXqOff % 256 == 0 && kYOff % 256 == 0, "scratch regions must stay 256-byte aligned");

__device__ __align__(256) unsigned char g_linear_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_addr_mu;
void *g_addr[kMaxDevices] = {};

// Address of the scratch array on the current device (ctx's, made current by check_ctx), looked
// up on the first call for that device and cached for the life of the process.  The cache
// assumes the device's primary context lives that long: after cudaDeviceReset the array would
// move, and this form must not be used again in that process.
ugb_status scratch_address(const ugb_ctx *ctx, uint8_t **out) {
  if (ctx->device < 0 || ctx->device >= kMaxDevices) return UGB_ECONTEXT;
  std::lock_guard<std::mutex> lock(g_addr_mu);
  if (!g_addr[ctx->device]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_linear_scratch) != cudaSuccess || !p) return UGB_EBACKEND;
    g_addr[ctx->device] = p;
  }
  *out = static_cast<uint8_t *>(g_addr[ctx->device]);
  return UGB_OK;
}

}  // namespace
}  // namespace ugb

using namespace ugb;

extern "C" ugb_status ugb_linear_static(ugb_ctx *ctx, ugb_stream stream, uint32_t kind, const void *w_dev,
                                        int64_t row_bytes, const float *x_host, float *y_host, int64_t k,
                                        int64_t m) {
  ugb_status st = check_ctx(ctx);  // ctx's device current on every call, as every entry point
  if (st != UGB_OK) return st;
  st = check_weights(kind, w_dev, row_bytes, k, m);
  if (st != UGB_OK) return st;
  if (k > kStaticMaxK || m > kStaticMaxM) return UGB_ESHAPE;  // beyond the fixed scratch
  if (!x_host || !y_host) return UGB_EALIGN;
  std::lock_guard<std::mutex> lock(ctx->mu);
  uint8_t *base = nullptr;
  st = scratch_address(ctx, &base);
  if (st != UGB_OK) return st;
  if (q8act_layout(k, 1).bytes > kXqBytes) return UGB_ESHAPE;
  float *x_dev = reinterpret_cast<float *>(base);
  uint8_t *xq = base + kXqOff;
  float *y_dev = reinterpret_cast<float *>(base + kYOff);
  if (cudaMemcpyAsync(x_dev, x_host, static_cast<size_t>(k) * 4, cudaMemcpyHostToDevice, stream) != cudaSuccess)
    return UGB_EBACKEND;
  st = launch_quant_q8_1(ctx, stream, x_dev, xq, k, 1, false);
  if (st != UGB_OK) return st;
  MatvecArgs a;
  a.kind = kind;
  a.w = static_cast<const uint8_t *>(w_dev);
  a.row_bytes = row_bytes;
  a.k = k;
  a.m = m;
  a.xq = xq;
  a.xl = q8act_layout(k, 1);
  a.y = y_dev;
  a.ldy = m;
  a.batch = 1;
  st = launch_matvec(ctx, stream, a);
  if (st != UGB_OK) return st;
  if (cudaMemcpyAsync(y_host, y_dev, static_cast<size_t>(m) * 4, cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return UGB_EBACKEND;
  return read_status_bits(ctx, stream, nullptr);  // synchronises the stream
}
