// Bit-exact q4nx tile decode on the device (test/debug path and the GPU form of
// Q4NX.tensor()).
//
// Per weight i of a tile (rb = i/4096, k = (i/16)%256, r = i%16):
//   scale entry  e = (k/32)*32 + rb*16 + r
//   q4  w = code*d[e] + m[e]   code = nibble (i even: low, i odd: high) of byte i/2
//   q8  w = code*s[e]          code = int8 byte i
// code*d and code*s are exact in fp32 (at most 12 and 16 significant bits), so
// fmaf(code, d, m) rounds exactly once, like numpy's `code*d + m` in float32
// (tools/q4nx.py:127-143).  The bf16 forms round that float32 with RNE, like
// `.astype(bfloat16)` (tools/q4nx.py:97-111, designs/q4nx_unpack/q4nx_unpack.cc).
#pragma once

#include "b2_common.cuh"

namespace b2 {

template <int QT>
__device__ __forceinline__ float dequant_one(const uint8_t* tile, const float* scale, const float* minv,
                                             int i) {
  const int e = (((i >> 4) & 255) >> 5) * 32 + (i >> 12) * 16 + (i & 15);
  if (QT == 0) {
    const uint8_t byte = tile[1024 + (i >> 1)];
    const float code = static_cast<float>((i & 1) ? (byte >> 4) : (byte & 15));
    return fmaf(code, scale[e], minv[e]);
  } else {
    const float code = static_cast<float>(static_cast<int8_t>(tile[512 + i]));
    return code * scale[e];
  }
}

// Load one tile and its scale planes into shared memory.
template <int QT>
__device__ __forceinline__ void stage_tile(const uint8_t* src, uint8_t* tile_s, float* scale_s, float* min_s) {
  constexpr int TILE = QT == 0 ? 5120 : 8704;
  for (int v = threadIdx.x; v < TILE / 16; v += blockDim.x)
    reinterpret_cast<uint4*>(tile_s)[v] = reinterpret_cast<const uint4*>(src)[v];
  __syncthreads();
  for (int e = threadIdx.x; e < 256; e += blockDim.x) {
    const uint16_t* d = reinterpret_cast<const uint16_t*>(tile_s);
    scale_s[e] = __uint_as_float(static_cast<uint32_t>(d[e]) << 16);
    if (QT == 0) min_s[e] = __uint_as_float(static_cast<uint32_t>(d[256 + e]) << 16);
  }
  __syncthreads();
}

// tiles [n_tiles][tile] -> out [n_tiles][8192] bf16 in weight-index order.
template <int QT>
__global__ void __launch_bounds__(256) dequant_tiles_bf16_kernel(const uint8_t* __restrict__ tiles,
                                                                 int64_t n_tiles,
                                                                 __nv_bfloat16* __restrict__ out) {
  constexpr int TILE = QT == 0 ? 5120 : 8704;
  __shared__ __align__(16) uint8_t tile_s[TILE];
  __shared__ float scale_s[256], min_s[256];
  for (int64_t tix = blockIdx.x; tix < n_tiles; tix += gridDim.x) {
    stage_tile<QT>(tiles + tix * TILE, tile_s, scale_s, min_s);
    __nv_bfloat16* o = out + tix * 8192;
    for (int i0 = threadIdx.x * 8; i0 < 8192; i0 += blockDim.x * 8) {
      alignas(16) __nv_bfloat16 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __float2bfloat16_rn(dequant_one<QT>(tile_s, scale_s, min_s, i0 + j));
      *reinterpret_cast<uint4*>(o + i0) = *reinterpret_cast<const uint4*>(v);
    }
    __syncthreads();
  }
}

// tiles [n_t][k_t][tile] -> out float32 [n_t*32][ld], untiled (row n, column k).
template <int QT>
__global__ void __launch_bounds__(256) dequant_matrix_f32_kernel(const uint8_t* __restrict__ tiles, int n_t,
                                                                 int k_t, float* __restrict__ out,
                                                                 int64_t ld) {
  constexpr int TILE = QT == 0 ? 5120 : 8704;
  __shared__ __align__(16) uint8_t tile_s[TILE];
  __shared__ float scale_s[256], min_s[256];
  const int64_t n_tiles = static_cast<int64_t>(n_t) * k_t;
  for (int64_t tix = blockIdx.x; tix < n_tiles; tix += gridDim.x) {
    const int64_t tr = tix / k_t, kt = tix % k_t;
    stage_tile<QT>(tiles + tix * TILE, tile_s, scale_s, min_s);
    // thread -> (row, 32 consecutive k)
    const int row = threadIdx.x >> 3, k0 = (threadIdx.x & 7) * 32;
    const int rb = row >> 4, r = row & 15;
    float* o = out + (tr * 32 + row) * ld + kt * 256 + k0;
#pragma unroll 4
    for (int k = 0; k < 32; ++k) o[k] = dequant_one<QT>(tile_s, scale_s, min_s, rb * 4096 + (k0 + k) * 16 + r);
    __syncthreads();
  }
}

}  // namespace b2
