// RMSNorm: y = x * rsqrt(mean(x^2) + eps) * w, bf16 out.
//
// Reference: designs/granite_gemv/granite_rmsnorm.h:45-80 (fp32 sum of squares,
// inverse square root, x*w scaled, one rounding to bf16 at the store); oracle
// granite_rmsnorm.py:112-113.  eps is a runtime argument here (the reference
// fixes it at compile time, granite_rmsnorm.h:37-39).  x may be bf16 or fp32
// (the decode step keeps its residual stream in fp32).  One CTA per row.
#pragma once

#include "b2_common.cuh"

namespace b2 {

constexpr int kNormThreads = 256;

template <bool XF32>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const void* __restrict__ x, int ldx,
                                                               const __nv_bfloat16* __restrict__ w, float eps,
                                                               int n, __nv_bfloat16* __restrict__ y, int ldy) {
  __shared__ float red[kNormThreads / 32];
  const int row = blockIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  auto xat = [&](int i) -> float {
    if (XF32) return static_cast<const float*>(x)[static_cast<size_t>(row) * ldx + i];
    return __bfloat162float(static_cast<const __nv_bfloat16*>(x)[static_cast<size_t>(row) * ldx + i]);
  };
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += kNormThreads) {
    const float v = xat(i);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float inv = rsqrtf(tot / static_cast<float>(n) + eps);
  for (int i = threadIdx.x; i < n; i += kNormThreads)
    y[static_cast<size_t>(row) * ldy + i] = __float2bfloat16_rn(xat(i) * __bfloat162float(w[i]) * inv);
}

}  // namespace b2
