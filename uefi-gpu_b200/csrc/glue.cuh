// glue.cuh -- device helpers shared by the matvec kernels (matvec.cu), the decode glue kernels
// (decode.cu) and the persistent token kernel (token.cu): Q8_1 block quantisation of a
// warp-held block, the greedy key, and warp reductions of row partials.
#pragma once
#include <cuda_fp16.h>
#include <cfloat>
#include <cmath>

#include "common.cuh"

namespace ugb {

// ---- correctly rounded divisions of the quantiser ------------------------------------------
//
// The activation quantiser (gpu_dp4a.cu:23-31) forms d = amax / 127 and inv = 127 / amax with
// IEEE division.  The compiler's general division is a long sequence with a slow-path branch,
// and it dominated the quantiser's latency (a warp quantises its blocks one after another).
// Both quotients are computed here with Markstein's method (P. Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990):
// a reciprocal approximation refined by one Newton step, the quotient, its exact remainder by
// FMA, and one correction.  They were checked bit for bit against __fdiv_rn for every positive
// finite float (and 0 maps to 0 in the callers).

__device__ __forceinline__ float rcp_approx_ftz(float a) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(a));
  return y;
}

// 127 / a for finite a > 0.  The divisor is first scaled by an exact power of two into
// [2^-64, 2^100] (no rounding), where the Markstein sequence is exact, and the quotient scaled
// back (exact while it stays normal; an overflow rounds to infinity exactly as the IEEE
// quotient does).  Branch-free.
__device__ __forceinline__ float div_127_by(float a) {
  const float s = a < 0x1p-64f ? 0x1p64f : (a > 0x1p100f ? 0x1p-64f : 1.0f);
  const float as = a * s;
  const float y0 = rcp_approx_ftz(as);
  const float y1 = __fmaf_rn(y0, __fmaf_rn(-as, y0, 1.0f), y0);
  const float q0 = __fmul_rn(127.0f, y1);
  const float q1 = __fmaf_rn(__fmaf_rn(-as, q0, 127.0f), y1, q0);
  return q1 * s;
}

// a / 127 for finite a >= 0: q0 = a * RN(1/127), corrected once by the exact remainder.  Below
// 2^-119 the quotient is subnormal and the correction may round twice, so such (never seen in
// practice) maxima take the IEEE division.
__device__ __forceinline__ float div_by_127(float a) {
  if (a < 0x1p-119f) return __fdiv_rn(a, 127.0f);
  const float c = 1.0f / 127.0f;
  const float q0 = __fmul_rn(a, c);
  return __fmaf_rn(__fmaf_rn(-127.0f, q0, a), c, q0);
}

// Q8_1 block-32 quantisation of one 32-element block held one value per lane (the
// quant_act arithmetic, gpu_dp4a.cu:23-31): amax over the block (non-finite values count as
// 0 and are reported), d = amax / 127, q = round-half-even(v * (127 / amax)) clamped to
// [-127, 127], s = sum(q).  The block maximum is one redux over the bit patterns of |v| (for
// non-negative floats the bit order is the value order).  Writes quants, scale and sum of
// block b.
// The values alone: this lane's quant, and (every lane) the block's scale and sum.
__device__ __forceinline__ bool quant_block_values(float v, int &qi, float &d, int &sum) {
  const bool fin = isfinite(v);
  const float a = __uint_as_float(__reduce_max_sync(0xffffffffu, fin ? __float_as_uint(fabsf(v)) : 0u));
  const float inv = a > 0.f ? div_127_by(a) : 0.0f;
  qi = fin ? __float2int_rn(v * inv) : 0;
  qi = max(-127, min(127, qi));
  sum = __reduce_add_sync(0xffffffffu, qi);
  d = div_by_127(a);
  return __any_sync(0xffffffffu, !fin);
}

__device__ __forceinline__ bool quant_block(float v, int lane, int8_t *q, float *d, int32_t *s, int b) {
  int qi, sum;
  float dd;
  const bool bad = quant_block_values(v, qi, dd, sum);
  q[b * 32 + lane] = static_cast<int8_t>(qi);
  if (lane == 0) {
    d[b] = dd;
    s[b] = sum;
  }
  return bad;
}

// NB blocks quantised together by one warp (block k's value in v[k], lane = element): the same
// arithmetic as quant_block, with the NB dependency chains interleaved (every operation runs for
// every k; only the stores are skipped for blocks with live[k] false).  A warp quantising its
// blocks one at a time waits out each block's redux / divide / redux chain in turn.
template <int NB>
__device__ __forceinline__ bool quant_blocks(const float (&v)[NB], const int (&b)[NB], const bool (&live)[NB], int lane,
                                             int8_t *q, float *d, int32_t *s) {
  float a[NB];
  bool bad = false;
#pragma unroll
  for (int k = 0; k < NB; ++k) {
    const bool fin = isfinite(v[k]);
    bad |= live[k] && !fin;
    a[k] = __uint_as_float(__reduce_max_sync(0xffffffffu, fin ? __float_as_uint(fabsf(v[k])) : 0u));
  }
  int qi[NB], sum[NB];
#pragma unroll
  for (int k = 0; k < NB; ++k) {
    const float inv = a[k] > 0.f ? div_127_by(a[k]) : 0.0f;
    const int t = isfinite(v[k]) ? __float2int_rn(v[k] * inv) : 0;
    qi[k] = max(-127, min(127, t));
  }
#pragma unroll
  for (int k = 0; k < NB; ++k) sum[k] = __reduce_add_sync(0xffffffffu, qi[k]);
#pragma unroll
  for (int k = 0; k < NB; ++k) {
    if (live[k]) {
      q[b[k] * 32 + lane] = static_cast<int8_t>(qi[k]);
      if (lane == 0) {
        d[b[k]] = div_by_127(a[k]);
        s[b[k]] = sum[k];
      }
    }
  }
  return __any_sync(0xffffffffu, bad);
}

// Element access of a KV cache of fp32 or fp16 (round to nearest even on store).  round()
// is the value a store followed by a load gives back.
template <typename KV>
struct KvIO;
template <>
struct KvIO<float> {
  static __device__ __forceinline__ float round(float v) { return v; }
  static __device__ __forceinline__ void store(float *p, float v) { *p = v; }
  static __device__ __forceinline__ float load(const float *p) { return *p; }
  static __device__ __forceinline__ float4 load4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
};
template <>
struct KvIO<__half> {
  static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
  static __device__ __forceinline__ void store(__half *p, float v) { *p = __float2half_rn(v); }
  static __device__ __forceinline__ float load(const __half *p) { return __half2float(*p); }
  static __device__ __forceinline__ float4 load4(const __half *p) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
};

// Greedy key: value bits made order-preserving as an unsigned integer, then the complemented
// id, so the larger key is the larger value and, for equal values, the lower id (the
// reference keeps the first maximum, llm.rs:383-385).
__device__ __forceinline__ uint64_t greedy_key(float v, uint32_t id) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<uint64_t>(b) << 32) | static_cast<uint64_t>(~id);
}

__device__ __forceinline__ uint32_t key_id(uint64_t key) { return ~static_cast<uint32_t>(key); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Totals of RW per-lane row partials v[0..RW) over the warp with one transposed shuffle tree
// (RW=4: 6 shuffles instead of 20).  The total of row r ends in lane r * (32 / RW); the lane
// returns the total of its row in *out and whether it owns one.
template <int RW>
__device__ __forceinline__ bool reduce_rows(const float (&v)[RW], int lane, float &out) {
  float c;
  if constexpr (RW == 1) {
    c = v[0];
  } else if constexpr (RW == 2) {
    const bool hi = lane & 16;
    const float r = __shfl_xor_sync(0xffffffffu, hi ? v[0] : v[1], 16);
    c = (hi ? v[1] : v[0]) + r;  // row (hi ? 1 : 0)
  } else {
    const bool hi = lane & 16;
    const float r0 = __shfl_xor_sync(0xffffffffu, hi ? v[0] : v[2], 16);
    const float r1 = __shfl_xor_sync(0xffffffffu, hi ? v[1] : v[3], 16);
    const float a = (hi ? v[2] : v[0]) + r0;  // row (hi ? 2 : 0)
    const float b = (hi ? v[3] : v[1]) + r1;  // row (hi ? 3 : 1)
    const bool h8 = lane & 8;
    const float r = __shfl_xor_sync(0xffffffffu, h8 ? a : b, 8);
    c = (h8 ? b : a) + r;  // row (hi ? 2 : 0) + (h8 ? 1 : 0)
  }
#pragma unroll
  for (int o = 32 / RW / 2; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  out = c;
  return (lane & (32 / RW - 1)) == 0;
}


}  // namespace ugb
