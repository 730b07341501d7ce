// prefill_quant.cuh -- the block-32 activation quantiser of the prefill GEMM's packed operand,
// shared by the standalone quant kernel (prefill.cu) and the glue kernels that quantise their
// own output (prefill_step.cu), so every form writes the same bits.
#pragma once
#include <cmath>

#include "common.cuh"
#include "prefill.hpp"

namespace ugb {

// Byte offset of (row r, K byte j) inside one canonical 128 x 32-byte block: 16-byte
// core-matrix rows, the two 16-byte K halves 128 B apart, 8-row groups 256 B apart.
__host__ __device__ __forceinline__ uint32_t canon_off(int r, int j) {
  return static_cast<uint32_t>((r >> 3) * 256 + (j >> 4) * 128 + (r & 7) * 16 + (j & 15));
}

// One warp, one element per lane: quantise block b of token t (quant_act's arithmetic:
// a = max|x|, d = a/127, q = clamp(rint(x * 127/a), +-127), non-finite x -> 0) into the packed
// operand whose quants start at q_out and scales at s_out (nb blocks per row).  Returns whether
// any element was non-finite.
__device__ __forceinline__ bool pf_quant_block(float val, int lane, int64_t t, int b, int nb, uint8_t *q_out,
                                               float *s_out) {
  const bool fin = isfinite(val);
  float a = fin ? fabsf(val) : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  const float inv = a > 0.f ? 127.0f / a : 0.0f;
  int qi = fin ? __float2int_rn(val * inv) : 0;
  qi = max(-127, min(127, qi));
  // gather four consecutive quants into lane 4w's word
  uint32_t word = static_cast<uint32_t>(qi) & 0xFFu;
  word |= (__shfl_down_sync(0xffffffffu, static_cast<uint32_t>(qi) & 0xFFu, 1) << 8);
  word |= (__shfl_down_sync(0xffffffffu, static_cast<uint32_t>(qi) & 0xFFu, 2) << 16);
  word |= (__shfl_down_sync(0xffffffffu, static_cast<uint32_t>(qi) & 0xFFu, 3) << 24);
  const int64_t tile = t / kPrefillTile;
  const int r = static_cast<int>(t % kPrefillTile);
  if ((lane & 3) == 0)
    *reinterpret_cast<uint32_t *>(q_out + (tile * nb + b) * kPrefillTileBytes + canon_off(r, lane)) = word;
  if (lane == 0) s_out[(tile * nb + b) * kPrefillTile + r] = a / 127.0f;
  return __any_sync(0xffffffffu, !fin);
}

}  // namespace ugb
