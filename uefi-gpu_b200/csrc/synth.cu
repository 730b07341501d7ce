// synth.cu -- seeded synthetic GGUF weight blocks, generated on the device.
//
// Benchmarks run on synthetic weights with the shapes and value distributions of the
// configurations (no model files are available): quants uniform over each format's code
// range, fp16 block scales |N(0,1)| * 0.002.  Every output byte is a pure function of
// (seed, byte index), so a matrix is reproducible and can be generated in parallel.
#include "common.cuh"
#include "internal.hpp"

namespace ugb {
namespace {

// fp16 bits of 0.002 * |Z| at the half-normal quantiles (i + 0.5) / 256, i = 0..255.
__constant__ uint16_t kScaleTable[256] = {
    0x0052, 0x00f6, 0x019b, 0x023f, 0x02e3, 0x0388, 0x042c, 0x04d0, 0x0575, 0x0619, 0x06be,
    0x0762, 0x0803, 0x0856, 0x08a8, 0x08fa, 0x094d, 0x099f, 0x09f2, 0x0a44, 0x0a97, 0x0ae9,
    0x0b3c, 0x0b8f, 0x0be1, 0x0c1a, 0x0c43, 0x0c6d, 0x0c96, 0x0cc0, 0x0ce9, 0x0d13, 0x0d3c,
    0x0d66, 0x0d90, 0x0db9, 0x0de3, 0x0e0d, 0x0e37, 0x0e60, 0x0e8a, 0x0eb4, 0x0ede, 0x0f08,
    0x0f32, 0x0f5c, 0x0f86, 0x0fb1, 0x0fdb, 0x1003, 0x1018, 0x102d, 0x1042, 0x1057, 0x106d,
    0x1082, 0x1097, 0x10ad, 0x10c2, 0x10d8, 0x10ed, 0x1103, 0x1118, 0x112e, 0x1143, 0x1159,
    0x116f, 0x1184, 0x119a, 0x11b0, 0x11c6, 0x11dc, 0x11f1, 0x1207, 0x121d, 0x1233, 0x124a,
    0x1260, 0x1276, 0x128c, 0x12a2, 0x12b9, 0x12cf, 0x12e5, 0x12fc, 0x1312, 0x1329, 0x1340,
    0x1356, 0x136d, 0x1384, 0x139b, 0x13b1, 0x13c8, 0x13df, 0x13f7, 0x1407, 0x1412, 0x141e,
    0x142a, 0x1435, 0x1441, 0x144d, 0x1459, 0x1465, 0x1470, 0x147c, 0x1488, 0x1494, 0x14a0,
    0x14ac, 0x14b8, 0x14c5, 0x14d1, 0x14dd, 0x14e9, 0x14f6, 0x1502, 0x150e, 0x151b, 0x1527,
    0x1534, 0x1540, 0x154d, 0x155a, 0x1566, 0x1573, 0x1580, 0x158d, 0x159a, 0x15a7, 0x15b4,
    0x15c1, 0x15ce, 0x15db, 0x15e9, 0x15f6, 0x1604, 0x1611, 0x161f, 0x162c, 0x163a, 0x1648,
    0x1655, 0x1663, 0x1671, 0x167f, 0x168d, 0x169b, 0x16aa, 0x16b8, 0x16c6, 0x16d5, 0x16e4,
    0x16f2, 0x1701, 0x1710, 0x171f, 0x172e, 0x173d, 0x174c, 0x175b, 0x176b, 0x177a, 0x178a,
    0x179a, 0x17aa, 0x17ba, 0x17ca, 0x17da, 0x17ea, 0x17fb, 0x1806, 0x180e, 0x1816, 0x181f,
    0x1827, 0x1830, 0x1839, 0x1841, 0x184a, 0x1853, 0x185c, 0x1865, 0x186e, 0x1878, 0x1881,
    0x188b, 0x1894, 0x189e, 0x18a7, 0x18b1, 0x18bb, 0x18c5, 0x18cf, 0x18da, 0x18e4, 0x18ef,
    0x18f9, 0x1904, 0x190f, 0x191a, 0x1925, 0x1931, 0x193c, 0x1948, 0x1954, 0x1960, 0x196c,
    0x1979, 0x1985, 0x1992, 0x199f, 0x19ac, 0x19ba, 0x19c8, 0x19d6, 0x19e4, 0x19f3, 0x1a01,
    0x1a11, 0x1a20, 0x1a30, 0x1a40, 0x1a51, 0x1a62, 0x1a74, 0x1a86, 0x1a98, 0x1aab, 0x1abf,
    0x1ad3, 0x1ae8, 0x1afe, 0x1b14, 0x1b2b, 0x1b43, 0x1b5d, 0x1b77, 0x1b93, 0x1bb0, 0x1bcf,
    0x1bef, 0x1c09, 0x1c1b, 0x1c2f, 0x1c45, 0x1c5d, 0x1c77, 0x1c94, 0x1cb6, 0x1cdd, 0x1d0d,
    0x1d4b, 0x1da5, 0x1e58};

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  // splitmix64 finaliser
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ uint32_t hash32(uint64_t seed, uint64_t block, uint64_t lane) {
  return static_cast<uint32_t>(mix64(seed ^ mix64(block * 0x9e3779b97f4a7c15ull + lane)) >> 16);
}

// Byte j of block b.
template <int KIND>
__device__ __forceinline__ uint8_t synth_byte(uint64_t seed, uint64_t b, int j) {
  if constexpr (KIND == UGB_Q8_0) {
    if (j < 2) {
      const uint16_t h = kScaleTable[hash32(seed, b, 1000) & 255];
      return static_cast<uint8_t>(j == 0 ? h & 0xff : h >> 8);
    }
    const uint32_t r = hash32(seed, b, j) & 0xffff;
    return static_cast<uint8_t>(static_cast<int8_t>(static_cast<int>((r * 255u) >> 16) - 127));
  } else {
    // where the block's fp16 scale d sits; every other byte is uniform (all patterns are valid)
    constexpr int d_at = KIND == UGB_Q3_K ? 108 : KIND == UGB_Q6_K ? 208 : 0;
    if (j >= d_at && j < d_at + 2) {
      const uint16_t h = kScaleTable[hash32(seed, b, 1000) & 255];
      return static_cast<uint8_t>(j == d_at ? h & 0xff : h >> 8);
    }
    if (KIND == UGB_Q4_K && (j == 2 || j == 3)) {
      const uint16_t h = kScaleTable[hash32(seed, b, 1001) & 255];
      return static_cast<uint8_t>(j == 2 ? h & 0xff : h >> 8);
    }
    return static_cast<uint8_t>(hash32(seed, b, j) & 0xff);
  }
}

template <int KIND, int BYTES>
__global__ void fill_kernel(uint8_t *w, uint64_t total, uint64_t seed) {
  const uint64_t i = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (i >= total) return;
  uint32_t word = 0;
  for (int t = 0; t < 4; ++t) {
    const uint64_t o = i + t;
    if (o < total) word |= static_cast<uint32_t>(synth_byte<KIND>(seed, o / BYTES, static_cast<int>(o % BYTES))) << (8 * t);
  }
  if (i + 4 <= total) {
    *reinterpret_cast<uint32_t *>(w + i) = word;
  } else {
    for (int t = 0; i + t < total; ++t) w[i + t] = static_cast<uint8_t>(word >> (8 * t));
  }
}

}  // namespace

ugb_status launch_fill_synthetic(ugb_ctx *, cudaStream_t stream, uint32_t kind, uint8_t *w,
                                 int64_t k, int64_t m, uint64_t seed) {
  const int64_t rb = ugb_row_bytes(kind, k);
  const uint64_t total = static_cast<uint64_t>(rb) * static_cast<uint64_t>(m);
  const uint64_t threads = (total + 3) / 4;
  const dim3 grid(static_cast<unsigned>((threads + 255) / 256));
  switch (kind) {
    case UGB_Q8_0: fill_kernel<UGB_Q8_0, 34><<<grid, 256, 0, stream>>>(w, total, seed); break;
    case UGB_Q4_K: fill_kernel<UGB_Q4_K, 144><<<grid, 256, 0, stream>>>(w, total, seed); break;
    case UGB_Q3_K: fill_kernel<UGB_Q3_K, 110><<<grid, 256, 0, stream>>>(w, total, seed); break;
    case UGB_Q6_K: fill_kernel<UGB_Q6_K, 210><<<grid, 256, 0, stream>>>(w, total, seed); break;
    case UGB_IQ3_XXS: fill_kernel<UGB_IQ3_XXS, 98><<<grid, 256, 0, stream>>>(w, total, seed); break;
    case UGB_IQ4_NL: fill_kernel<UGB_IQ4_NL, 18><<<grid, 256, 0, stream>>>(w, total, seed); break;
    case UGB_IQ4_XS: fill_kernel<UGB_IQ4_XS, 136><<<grid, 256, 0, stream>>>(w, total, seed); break;
    default: return UGB_EQUANT;
  }
  return cuda_status(cudaGetLastError());
}

}  // namespace ugb
