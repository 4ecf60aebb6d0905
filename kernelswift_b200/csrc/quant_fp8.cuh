// e4m3 (fp8) quantisation of bf16 rows with one power-of-two scale per row: the
// input side of the FP8 indexer (ModelArgs.dtype = "fp8", scale_fmt = "ue8m0" in
// baseline/indexer.py:14-17).
//
//   amax  = max(max_i |x_i|, 1e-4)
//   scale = the smallest power of two >= amax / 448   (448 = largest finite e4m3;
//           a power of two is what a ue8m0 scale byte can hold)
//   q_i   = e4m3(x_i / scale), round to nearest even, saturating to +-448
//
// x / scale is exact (a power-of-two scaling of a bf16 value), so the only
// rounding is the final conversion.  One warp per row, 8-byte loads.
#pragma once
#include "ks_device.cuh"

namespace ks {

constexpr int QF_WARPS = 8;

// Two fp32 -> e4m3x2 with round to nearest even and saturation (lo in bits 0-7).
__device__ __forceinline__ uint16_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

__global__ void __launch_bounds__(QF_WARPS * 32)
    quant_fp8_rows_kernel(const uint16_t* __restrict__ x, uint8_t* __restrict__ x8,
                          float* __restrict__ scale, int64_t rows, int D) {
  const int64_t row = (int64_t)blockIdx.x * QF_WARPS + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint16_t* xr = x + row * D;
  float amax = 0.f;
  for (int i = lane * 4; i < D; i += 128) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(xr + i));
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(bf16lo_f32(v.x)), fabsf(bf16hi_f32(v.x))),
                             fmaxf(fabsf(bf16lo_f32(v.y)), fabsf(bf16hi_f32(v.y)))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  // smallest power of two >= v (v is a positive normal number)
  const float v = __fdiv_rn(fmaxf(amax, 1e-4f), 448.f);
  const uint32_t vb = __float_as_uint(v);
  const uint32_t e = vb & 0x7F800000u;
  const float s = (vb & 0x007FFFFFu) ? __uint_as_float(e + 0x00800000u) : v;
  const float inv = __frcp_rn(s);  // exact: s is a power of two
  uint8_t* yr = x8 + row * D;
  for (int i = lane * 4; i < D; i += 128) {
    const uint2 v2 = __ldg(reinterpret_cast<const uint2*>(xr + i));
    const uint32_t lo = cvt_e4m3x2(bf16lo_f32(v2.x) * inv, bf16hi_f32(v2.x) * inv);
    const uint32_t hi = cvt_e4m3x2(bf16lo_f32(v2.y) * inv, bf16hi_f32(v2.y) * inv);
    *reinterpret_cast<uint32_t*>(yr + i) = lo | (hi << 16);
  }
  if (lane == 0) scale[row] = s;
}

}  // namespace ks
