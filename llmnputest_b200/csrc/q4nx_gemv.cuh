// q4nx W4A16 / W8A16 GEMV for sm_100a, reading FastFlowLM's tiles as stored.
//
//   y[b][n] = sum_k W[n][k] * x[b][k],   b < batch <= 16, fp32 accumulate
//
// Tile format (one tile = 32 output rows x 256 k, row index fastest):
//   q4 5120 B: d[256] bf16 | m[256] bf16 | 4096 B nibbles,  w = code*d + m
//   q8 8704 B: s[256] bf16 | 8192 B int8 codes,             w = code*s
//   weight i = rb*4096 + k*16 + r (rb = row-block 0..1, r = 0..15), its scale
//   entry (k/32)*32 + rb*16 + r; q4 byte i/2, low nibble = even i.
// (tools/q4nx.py:1-33, designs/granite_gemv/granite_gemv.h:31-45,
//  designs/lm_head/lm_head.h:19-32.)
//
// The quantisation block factors out of the dot product as in the reference
// kernel (granite_gemv.h:19-29):
//   y[r] = sum_kb  d[kb][r] * (sum_{k in kb} code*x)  +  m[kb][r] * (sum_{k in kb} x)
// The inner sums run on the tensor core (mma.sync m16n8k16, fp16 operands, fp32
// accumulate) with EXACT operands:
//   * x is staged as fp16 x' = x * 2^e, e chosen per token and per K slice so
//     that max|x'| lies in [2^14, 2^15): a bf16 value (8 significant bits)
//     times a power of two is exact in fp16; e is undone exactly at the end.
//   * a q4 byte holds rows 2j (low nibble) and 2j+1 (high nibble) at one k.  One
//     LOP3 per nibble against an fp16 exponent pattern yields an exact value
//     with no shift: low nibble n | 0x6400 = 1024 + n, high nibble (n<<4) |
//     0x5400 = 64 + n; an exact f16x2 subtract leaves n.
//   * a q8 byte c becomes one exact fp16 with one LOP3: (c & 0xFF) ^ 0x6480 =
//     0x6400 | (c + 128) = 1152 + c; one MMA against x' gives (1152 + c)*x', and
//     the constant 1152*s folds into the sum-of-x term (m = -1152*s).
// Every product is exact in fp32; the only rounding is fp32 accumulation.
//
// Data flow per CTA (a "row group" = 4 tile-rows = 128 outputs, or for the
// fused SwiGLU 2 gate + 2 up tile-rows with matching rows):
//   producer warp: cp.async.bulk (TMA engine, no multicast) of the group's 4
//                  tiles at one K-tile into a stage of a shared-memory ring;
//                  mbarrier complete_tx; L2 evict-first (weights stream once);
//   8 consumer warps: warp w = (row-block rb = w&1, k-block pair kp = w>>1).
//                  Lane (g,t) owns rows h*8..h*8+7 (h = g>>2) of row-block rb
//                  of tile g&3, and k-pairs {2t,2t+1}, {2t+8,2t+9} of each
//                  16-k MMA step: four 32-bit shared loads, PRMT pairs two k,
//                  LOP3 decodes, 4 MMAs (the 16 "M" rows are rows 2s,2s+1 of
//                  8 row-block halves), x' as the B operand (N = batch);
//                  after each 32-k block the d/m scaling into fp32 totals;
//   epilogue:      warp totals -> shared memory -> CTA sum (fixed order) ->
//                  split-K: SwiGLU sums the cluster's partials through
//                  distributed shared memory (fixed order, deterministic);
//                  f32 adds them into y with global reductions (the order of
//                  those fp32 adds, and so the last bits, vary between runs).
// Split-K across CTAs uses a cluster (no global workspace); when the groups
// outnumber the SMs the grid is persistent and the producer runs ahead across
// group boundaries.
#pragma once

#include "b2_common.cuh"

namespace b2 {

enum QType : int { kQ4 = 0, kQ8 = 1 };
enum GemvEpi : int { kEpiF32 = 0, kEpiSwiglu = 1 };

template <int QT>
struct QTraits;
template <>
struct QTraits<kQ4> {
  static constexpr int kTile = 5120;
  // +32 B: the 4 tiles of a stage start 32 B apart modulo 128, which with the
  // per-tile load order below makes every 32-bit nibble load conflict-free
  static constexpr int kSlot = 5152;
};
template <>
struct QTraits<kQ8> {
  static constexpr int kTile = 8704;
  static constexpr int kSlot = 8720;
};

constexpr int kGemvConsumerWarps = 8;
constexpr int kGemvConsumers = kGemvConsumerWarps * 32;
constexpr int kGemvThreads = kGemvConsumers + 32;
constexpr int kGroupRows = 128;
constexpr int kMaxStages = 8;
constexpr int kMaxBatch = 16;

struct GemvParams {
  const uint8_t* w0;  // tile-rows [n_tile_rows][k_tiles][tile]
  const uint8_t* w1;  // second source (fused SwiGLU: up), else null
  int n_tile_rows;    // per source
  int k_tiles;
  const __nv_bfloat16* x;  // [batch][ldx]
  int batch;
  int ldx;
  void* y;  // f32 [batch][ldy] or, for SwiGLU, bf16 [batch][ldy]
  int ldy;
  int accumulate;    // f32 epilogue: y += W x instead of y = W x
  int kt_per_split;  // K-tiles per CTA of a cluster
  int n_splits;      // cluster size (split-K), 1 = no cluster
  int n_groups;
  int stages;
  int x_stride;              // fp16 per shared-memory x row = kt_per_split*256 + 8
  int prefetch_before_wait;  // weights may stream before the PDL wait
  const float* xf;           // fused RMSNorm: fp32 input rows [batch][ldx] instead of x
  const __nv_bfloat16* norm_w;  // [K] RMSNorm weight
  float eps;
};

// Shared-memory layout (bytes), computed identically on host and device.
struct GemvSmem {
  int ring, x, xs, red, csum, gather, misc, xf, nw, bar, flag, total;
  int ncol;  // batch rounded up to even
  // norm_k > 0: batch-1 fused RMSNorm with the fp32 row (norm_k floats) and this
  // CTA's slice of the norm weight copied into shared memory
  __host__ __device__ GemvSmem(int slot, int nb, int stages, int x_stride, int kt_per_split, int batch,
                               int norm_k = 0) {
    ncol = (batch + 1) & ~1;
    ring = 0;
    x = stages * 4 * slot;
    xs = x + ((batch * x_stride * 2 + 15) & ~15);
    red = xs + kt_per_split * 8 * 8 * nb * 4;
    csum = red + kGemvConsumerWarps * 64 * ncol * 4;
    gather = csum + kGroupRows * ncol * 4;  // split-K partials pushed by the cluster's ranks
    misc = gather + 160 * ncol * 4;         // [kMaxBatch] max bits, [kMaxBatch] exponents
    xf = (misc + 2 * kMaxBatch * 4 + 15) & ~15;
    nw = xf + norm_k * 4;
    bar = nw + (norm_k > 0 ? kt_per_split * 256 * 2 : 0);
    bar = (bar + 15) & ~15;
    flag = bar + (2 * stages + 1) * 8;  // full[stages], empty[stages], x
    total = flag + 16;
  }
};

__device__ __forceinline__ uint32_t pack_bf16x2_rn(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ float absmax8_bf16(uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) m = fmaxf(m, fmaxf(fabsf(bf16lo_to_f32(w[i])), fabsf(bf16hi_to_f32(w[i]))));
  return m;
}

// Scale exponent for a row whose max |x| has bit pattern `bits`: x*2^e has its
// max in [2^14, 2^15).  Clamped so that 2^e and 2^-e are normal floats.
__device__ __forceinline__ int gemv_scale_exp(uint32_t bits) {
  const int ex = static_cast<int>((bits >> 23) & 255);
  if (bits == 0 || ex == 255) return 0;
  const int e = 14 - (ex - 127);
  return max(-126, min(126, e));
}
__device__ __forceinline__ float pow2f(int e) { return __uint_as_float(static_cast<uint32_t>(e + 127) << 23); }

// q4: decode the 8 rows of one k-pair from two 32-bit words (k_a and k_b bytes of
// rows h*8..h*8+7, 2 rows per byte); out[r] = f16x2 (row r @ k_a, row r @ k_b).
// Even rows come out as 1024 + n (low nibble under the 1024 exponent pattern),
// odd rows as 64 + n (high nibble under 64's): both exact in f16, no subtract;
// the caller folds the offsets into the m term.
__device__ __forceinline__ void decode_q4_pair_biased(uint32_t w1, uint32_t w2, uint32_t sel_lo, uint32_t sel_hi,
                                                      uint32_t (&a)[8]) {
  constexpr uint32_t kLoMagic = 0x64006400u, kHiMagic = 0x54005400u;
  const uint32_t r0 = prmt(w1, w2, sel_lo), r1 = prmt(w1, w2, sel_hi);
  const uint32_t r0s = r0 >> 8, r1s = r1 >> 8;
  a[0] = lop3<kLutAndOr>(r0, 0x000F000Fu, kLoMagic);
  a[1] = lop3<kLutAndOr>(r0, 0x00F000F0u, kHiMagic);
  a[2] = lop3<kLutAndOr>(r0s, 0x000F000Fu, kLoMagic);
  a[3] = lop3<kLutAndOr>(r0s, 0x00F000F0u, kHiMagic);
  a[4] = lop3<kLutAndOr>(r1, 0x000F000Fu, kLoMagic);
  a[5] = lop3<kLutAndOr>(r1, 0x00F000F0u, kHiMagic);
  a[6] = lop3<kLutAndOr>(r1s, 0x000F000Fu, kLoMagic);
  a[7] = lop3<kLutAndOr>(r1s, 0x00F000F0u, kHiMagic);
}

// q8: a PRMT result [row A @k, row B @k, row A @k+1, row B @k+1] -> f16x2
// (A @k, A @k+1) and (B @k, B @k+1), each code c as 1152 + c (exact).
__device__ __forceinline__ void decode_q8_pair(uint32_t res, uint32_t& ra, uint32_t& rb) {
  constexpr uint32_t kMagicFlip = 0x64806480u;  // 0x6400 | flip of bit 7 (c ^ 0x80 = c + 128)
  ra = lop3<kLutAndXor>(res, 0x00FF00FFu, kMagicFlip);
  rb = lop3<kLutAndXor>(res >> 8, 0x00FF00FFu, kMagicFlip);
}

// q4 nibbles of 4 rows at (k_a, k_b) -> bf16x2 codes 128 + n (exact, no subtract:
// the offset folds into the m term).  r = PRMT of the two k words; bf16 has 7
// mantissa bits, so each nibble is shifted to bits 0-3 first.
__device__ __forceinline__ void decode_q4_half_bf16(uint32_t w1, uint32_t w2, uint32_t sel, uint32_t (&a)[4]) {
  constexpr uint32_t kMagic = 0x43004300u;  // bf16x2 (128, 128): n | magic = 128 + n
  const uint32_t r = prmt(w1, w2, sel);
  a[0] = lop3<kLutAndOr>(r, 0x000F000Fu, kMagic);
  a[1] = lop3<kLutAndOr>(r >> 4, 0x000F000Fu, kMagic);
  a[2] = lop3<kLutAndOr>(r >> 8, 0x000F000Fu, kMagic);
  a[3] = lop3<kLutAndOr>(r >> 12, 0x000F000Fu, kMagic);
}

template <int QT, int NB, int EPI>
__global__ void __launch_bounds__(kGemvThreads, NB == 1 ? 2 : 1) q4nx_gemv_kernel(const GemvParams p) {
  constexpr int TILE = QTraits<QT>::kTile;
  constexpr int SLOT = QTraits<QT>::kSlot;
  constexpr int STAGE = 4 * SLOT;
  extern __shared__ __align__(128) uint8_t smem[];

  // batch 1 with the fused norm (q4): the fp32 row and the norm weight slice are
  // bulk-copied after the PDL wait and the norm is reduced by all consumer threads
  const bool x_norm_bulk = QT == kQ4 && NB == 1 && p.batch == 1 && p.xf != nullptr;
  const GemvSmem L(SLOT, NB, p.stages, p.x_stride, p.kt_per_split, p.batch, x_norm_bulk ? p.k_tiles * 256 : 0);
  uint8_t* ring = smem + L.ring;
  __half* x_s = reinterpret_cast<__half*>(smem + L.x);
  float* xs_s = reinterpret_cast<float*>(smem + L.xs);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* csum = reinterpret_cast<float*>(smem + L.csum);
  uint32_t* maxbits = reinterpret_cast<uint32_t*>(smem + L.misc);
  int* exps = reinterpret_cast<int*>(smem + L.misc) + kMaxBatch;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.flag);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int stages = p.stages;
  const int batch = p.batch;
  const int ncol = L.ncol;
  const bool clustered = p.n_splits > 1;
  const int split = clustered ? static_cast<int>(cluster_ctarank()) : 0;
  const int kt0 = split * p.kt_per_split;
  const int kt_cnt = min(p.kt_per_split, p.k_tiles - kt0);  // >= 1 by construction
  // cluster protocol (split-K).  f32: partials are added into y with global
  // reductions; unless y is accumulated into, rank 0's producer warp zeroes the
  // group's rows once its loads are issued (after its PDL wait) and arrives on a
  // cluster barrier that the consumers only wait on just before their adds, so
  // the zeroing stays off the consumers' path.  SwiGLU: partials are pushed to
  // the owning rank's shared memory and summed after one cluster barrier.
  // Clustered launches always give each CTA exactly one group.
  const int cl_mode = !clustered ? 0 : (EPI == kEpiSwiglu ? 2 : (p.accumulate ? 0 : 1));
  // Batch 1 (q4): each 32-k block of a K-tile gets its own MMA column (x in
  // column j, zero elsewhere), so one accumulator holds the eight block sums and
  // the d/m fold runs once per K-tile instead of once per block.  Warps split a
  // stage by (row block, half of the k-blocks) and take alternate stages.
  constexpr bool kB1able = (QT == kQ4 && NB == 1);
  const bool b1 = kB1able && batch == 1;
  // batch 1 without the fused norm: x needs no conversion, so the producer copies
  // the K slice into shared memory right after its PDL wait (one bulk copy)
  const bool x_bulk = b1 && !p.xf;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&bars[s]), 1);                             // full: producer + tx
      mbar_init(smem_u32(&bars[stages + s]), b1 ? 4 : kGemvConsumerWarps);  // empty: one per consuming warp
    }
    mbar_init(smem_u32(&bars[2 * stages]), 1);  // x slice
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < kMaxBatch) maxbits[threadIdx.x] = 0;
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kGemvConsumerWarps) {
    // ------------------------------------------------------------ producer
    const uint64_t policy = l2_evict_first_policy();
    // Called by the whole warp exactly once: after the PDL wait x and y are
    // final/free, so copy this CTA's x slice (batch 1, no norm), zero the
    // group's y rows (rank 0 of an f32 split-K cluster) and arrive on the
    // cluster barrier the consumers wait on before their adds.
    auto wait_and_copy_x = [&]() {
      __syncwarp();
      pdl_wait();
      if (x_bulk && lane == 0) {
        const uint32_t xb = smem_u32(&bars[2 * stages]);
        mbar_arrive_expect_tx(xb, static_cast<uint32_t>(kt_cnt) * 512);
        bulk_g2s(smem_u32(x_s), p.x + static_cast<size_t>(kt0) * 256, static_cast<uint32_t>(kt_cnt) * 512, xb,
                 l2_evict_last_policy());
      }
      if (x_norm_bulk && lane == 0) {  // the whole fp32 row (for the norm) and this CTA's weight slice
        const uint32_t xb = smem_u32(&bars[2 * stages]);
        const uint32_t row_bytes = static_cast<uint32_t>(p.k_tiles) * 1024, w_bytes = static_cast<uint32_t>(kt_cnt) * 512;
        mbar_arrive_expect_tx(xb, row_bytes + w_bytes);
        bulk_g2s(smem_u32(smem + L.xf), p.xf, row_bytes, xb, l2_evict_last_policy());
        bulk_g2s(smem_u32(smem + L.nw), p.norm_w + static_cast<size_t>(kt0) * 256, w_bytes, xb,
                 l2_evict_last_policy());
      }
      if (cl_mode == 1) {
        if (split == 0) {
          float* y = static_cast<float*>(p.y);
          for (int e = lane; e < kGroupRows * p.batch; e += 32) {
            const int row = e % kGroupRows, b = e / kGroupRows;
            if (blockIdx.y * 4 + (row >> 5) < p.n_tile_rows)
              y[static_cast<size_t>(b) * p.ldy + blockIdx.y * kGroupRows + row] = 0.f;
          }
        }
        __syncwarp();
        cluster_arrive_release();
      }
    };
    uint32_t seq = 0;
    bool waited_pdl = false;
    if (!p.prefetch_before_wait) {
      wait_and_copy_x();
      waited_pdl = true;
    } else if (x_bulk && lane == 0) {
      bulk_prefetch_l2(p.x + static_cast<size_t>(kt0) * 256, static_cast<uint32_t>(kt_cnt) * 512);  // L2 only
    } else if (x_norm_bulk && lane == 0) {
      bulk_prefetch_l2(p.xf, static_cast<uint32_t>(p.k_tiles) * 1024);
    }
    for (int grp = blockIdx.y; grp < p.n_groups; grp += gridDim.y) {
      for (int kk = 0; kk < kt_cnt; ++kk, ++seq) {
        if (seq >= static_cast<uint32_t>(stages) && !waited_pdl) {  // warp-uniform
          wait_and_copy_x();  // ring full: nothing more to prefetch before the dependency
          waited_pdl = true;
        }
        if (lane == 0 && !*abort_flag) {
          const int slot = seq % stages;
          const uint32_t ph = (seq / stages) & 1;
          bool ok = true;
          if (seq >= static_cast<uint32_t>(stages))
            ok = mbar_wait_bounded(smem_u32(&bars[stages + slot]), ph ^ 1, abort_flag, kDevTimeoutEmpty);
          if (ok) {
            const int kt = kt0 + kk;
            const uint8_t* src[4];
            uint32_t bytes = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              int tr;
              const uint8_t* base;
              if (EPI == kEpiSwiglu) {
                tr = grp * 2 + (j & 1);
                base = (j < 2) ? p.w0 : p.w1;
              } else {
                tr = grp * 4 + j;
                base = p.w0;
              }
              src[j] = (tr < p.n_tile_rows) ? base + (static_cast<size_t>(tr) * p.k_tiles + kt) * TILE : nullptr;
              bytes += src[j] ? TILE : 0;
            }
            const uint32_t full = smem_u32(&bars[slot]);
            mbar_arrive_expect_tx(full, bytes);
            const uint32_t dst = smem_u32(ring + slot * STAGE);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              if (src[j]) bulk_g2s(dst + j * SLOT, src[j], TILE, full, policy);
          }
        }
      }
      __syncwarp();
    }
    __syncwarp();
    if (!waited_pdl) wait_and_copy_x();  // the whole slice fit the ring
    __syncwarp();
    if (cl_mode == 1) cluster_wait_acquire();  // completes this thread's barrier phase
    if (cl_mode == 2) cluster_sync_all();
    if (lane == 0 && *abort_flag && (x_bulk || x_norm_bulk)) {
      // lane 0 has issued the x copy by now, right after its PDL wait
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(smem_u32(&bars[2 * stages]), 0)) {
        if (globaltimer() - t0 > B2_WAIT_TIMEOUT_NS) {
          record_error(kDevTimeoutDrain);
          break;
        }
      }
    }
    if (lane == 0 && *abort_flag) {
      // abort path: let every copy this CTA issued land before the CTA exits
      const uint32_t first = seq > static_cast<uint32_t>(stages) ? seq - stages : 0;
      for (uint32_t s = first; s < seq; ++s) {
        const uint32_t bar = smem_u32(&bars[s % stages]);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(bar, (s / stages) & 1)) {
          if (globaltimer() - t0 > B2_WAIT_TIMEOUT_NS) {
            record_error(kDevTimeoutDrain);
            break;
          }
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  pdl_wait();
  const int ctid = threadIdx.x;
  if (cl_mode == 1) cluster_arrive_relaxed();  // nothing to publish: the producer carries the zeroing
  const int L_cta = kt_cnt * 256;
  if (!x_bulk && !x_norm_bulk) {
    // x rows as bf16: given (p.x), or bf16(rmsnorm(p.xf) * norm_w) computed here
    // (the norm fused into the GEMV, granite_rmsnorm.h:45-80 arithmetic).
    const int vec_per_row = L_cta / 8;  // 16-byte vectors of 8 values, a multiple of 32
    float* inv_rms = reinterpret_cast<float*>(maxbits);
    if (p.xf) {
      const int K = p.k_tiles * 256;
      for (int b = warp; b < batch; b += kGemvConsumerWarps) {
        const float4* xr = reinterpret_cast<const float4*>(p.xf + static_cast<size_t>(b) * p.ldx);
        float ss = 0.f;
        for (int c = lane; c < K / 4; c += 32) {
          const float4 v = xr[c];
          ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) inv_rms[b] = rsqrtf(ss / static_cast<float>(K) + p.eps);
      }
      named_barrier(1, kGemvConsumers);
    }
    auto xvec = [&](int b, int c) -> uint4 {
      if (!p.xf) return reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(b) * p.ldx + kt0 * 256)[c];
      const int k0 = kt0 * 256 + c * 8;
      const float4 a0 = *reinterpret_cast<const float4*>(p.xf + static_cast<size_t>(b) * p.ldx + k0);
      const float4 a1 = *reinterpret_cast<const float4*>(p.xf + static_cast<size_t>(b) * p.ldx + k0 + 4);
      const uint4 wv = *reinterpret_cast<const uint4*>(p.norm_w + k0);
      const float r = inv_rms[b];
      auto nb = [&](float xv, float wf) { return xv * r * wf; };
      uint4 o;
      o.x = pack_bf16x2_rn(nb(a0.x, bf16lo_to_f32(wv.x)), nb(a0.y, bf16hi_to_f32(wv.x)));
      o.y = pack_bf16x2_rn(nb(a0.z, bf16lo_to_f32(wv.y)), nb(a0.w, bf16hi_to_f32(wv.y)));
      o.z = pack_bf16x2_rn(nb(a1.x, bf16lo_to_f32(wv.z)), nb(a1.y, bf16hi_to_f32(wv.z)));
      o.w = pack_bf16x2_rn(nb(a1.z, bf16lo_to_f32(wv.w)), nb(a1.w, bf16hi_to_f32(wv.w)));
      return o;
    };
    // x' = fp16(x * 2^e) for this warp's K-tiles and the per-32-k sums of x'
    auto put = [&](int b, int c, uint4 in, float sc) {
      const uint32_t w[4] = {in.x, in.y, in.z, in.w};
      uint32_t o[4];
      float s8 = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (b1) {  // bf16 kept as is
          o[i] = w[i];
          s8 += bf16lo_to_f32(w[i]);
          s8 += bf16hi_to_f32(w[i]);
        } else {
          const __half2 hv = __floats2half2_rn(bf16lo_to_f32(w[i]) * sc, bf16hi_to_f32(w[i]) * sc);
          o[i] = *reinterpret_cast<const uint32_t*>(&hv);
          const float2 f = __half22float2(hv);
          s8 += f.x;
          s8 += f.y;
        }
      }
      *reinterpret_cast<uint4*>(x_s + b * p.x_stride + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
      s8 += __shfl_xor_sync(0xffffffffu, s8, 1);
      s8 += __shfl_xor_sync(0xffffffffu, s8, 2);
      if ((lane & 3) == 0) xs_s[(c >> 2) * 8 * NB + b] = s8;
    };
    constexpr int kVecLane = 8;  // a slice of up to 8 K-tiles is held in registers
    if (batch > 1) {
      // one warp per row: the rows' loads, maxima and conversions run in parallel
      for (int b = warp; b < batch; b += kGemvConsumerWarps) {
        float mx = 0.f;
        if (vec_per_row <= 32 * kVecLane) {
          uint4 v[kVecLane];
#pragma unroll
          for (int i = 0; i < kVecLane; ++i)
            if (32 * i < vec_per_row) {
              v[i] = xvec(b, lane + 32 * i);
              mx = fmaxf(mx, absmax8_bf16(v[i]));
            }
          mx = warp_max(mx);
          const int e = gemv_scale_exp(__float_as_uint(mx));
          const float sc = pow2f(e);
          if (lane == 0) exps[b] = e;
#pragma unroll
          for (int i = 0; i < kVecLane; ++i)
            if (32 * i < vec_per_row) put(b, lane + 32 * i, v[i], sc);
        } else {
          for (int c = lane; c < vec_per_row; c += 32) mx = fmaxf(mx, absmax8_bf16(xvec(b, c)));
          mx = warp_max(mx);
          const int e = gemv_scale_exp(__float_as_uint(mx));
          const float sc = pow2f(e);
          if (lane == 0) exps[b] = e;
          for (int c = lane; c < vec_per_row; c += 32) put(b, c, xvec(b, c), sc);
        }
      }
    }
    for (int b = 0; b < (batch > 1 ? 0 : batch); ++b) {
      if (vec_per_row <= 32 * kVecLane) {
        // one pass: every warp loads the whole slice (one L2 round trip), finds the
        // max itself (no barrier), and converts its own K-tiles from registers
        uint4 v[kVecLane];
        float mx = 0.f;
#pragma unroll
        for (int i = 0; i < kVecLane; ++i)
          if (32 * i < vec_per_row) {
            v[i] = xvec(b, lane + 32 * i);
            mx = fmaxf(mx, absmax8_bf16(v[i]));
          }
        mx = warp_max(mx);
        const int e = gemv_scale_exp(__float_as_uint(mx));
        const float sc = pow2f(e);
        if (warp == 0 && lane == 0) exps[b] = b1 ? 0 : e;
#pragma unroll
        for (int i = 0; i < kVecLane; ++i)
          if (32 * i < vec_per_row && (i % kGemvConsumerWarps) == warp) put(b, lane + 32 * i, v[i], sc);
      } else {
        float mx = 0.f;
        for (int c = lane; c < vec_per_row; c += 32) mx = fmaxf(mx, absmax8_bf16(xvec(b, c)));
        mx = warp_max(mx);
        const int e = gemv_scale_exp(__float_as_uint(mx));
        const float sc = pow2f(e);
        if (warp == 0 && lane == 0) exps[b] = b1 ? 0 : e;
        for (int c = warp * 32 + lane; c < vec_per_row; c += kGemvConsumers) put(b, c, xvec(b, c), sc);
      }
    }
    for (int v = ctid; v < kt_cnt * 8 * 8 * NB; v += kGemvConsumers)
      if (v % (8 * NB) >= batch) xs_s[v] = 0.f;
    named_barrier(1, kGemvConsumers);
  }

  const int g = lane >> 2, t = lane & 3;
  const int tile = g & 3, h = g >> 2, odd = tile & 1;
  const int rb = warp & 1, kp = warp >> 1;
  // load order: odd tiles read the k_b word first (bank spreading); the PRMT
  // selector undoes the swap so r = [k_a bytes | k_b bytes] either way
  const uint32_t sel_lo = odd ? 0x1054u : 0x5410u;
  const uint32_t sel_hi = odd ? 0x3276u : 0x7632u;
  const int off_first = odd ? 8 : 0, off_second = odd ? 0 : 8;
  const uint32_t* x32 = reinterpret_cast<const uint32_t*>(x_s);
  const int xw_stride = p.x_stride / 2;

  if (x_bulk || x_norm_bulk) mbar_wait_bounded(smem_u32(&bars[2 * stages]), 0, abort_flag, kDevTimeoutFull);
  float inv_rms1 = 0.f;
  if (x_norm_bulk) {
    // sum of squares of the fp32 row by all consumer threads (granite_rmsnorm.h:45-80 arithmetic)
    const float4* xr = reinterpret_cast<const float4*>(smem + L.xf);
    float ss = 0.f;
    for (int c = ctid; c < p.k_tiles * 64; c += kGemvConsumers) {
      const float4 v = xr[c];
      ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;  // red is free until the first park
    named_barrier(1, kGemvConsumers);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kGemvConsumerWarps; ++w) tot += red[w];
    inv_rms1 = rsqrtf(tot / static_cast<float>(p.k_tiles * 256) + p.eps);
  }
  if (b1) {
    // x (bf16, this CTA's K slice) -> f16 in place, scaled per 32-k block by 2^e
    // (exact: bf16's 8-bit mantissa fits f16's 11), with the block's sum of x and
    // 2^-e beside it: xs_s[block * 8 + 0 / 1].  Four lanes hold one block.
    uint4* xv = reinterpret_cast<uint4*>(x_s);
    for (int v = ctid; v < kt_cnt * 32; v += kGemvConsumers) {  // warp-uniform trip count
      uint4 u;
      if (x_norm_bulk) {  // bf16(x * inv_rms * w) from the row and weight slice in shared memory
        const float4 a0 = reinterpret_cast<const float4*>(smem + L.xf)[kt0 * 64 + 2 * v];
        const float4 a1 = reinterpret_cast<const float4*>(smem + L.xf)[kt0 * 64 + 2 * v + 1];
        const uint4 wv = reinterpret_cast<const uint4*>(smem + L.nw)[v];
        auto nb = [&](float xv_, float wf) { return xv_ * inv_rms1 * wf; };
        u.x = pack_bf16x2_rn(nb(a0.x, bf16lo_to_f32(wv.x)), nb(a0.y, bf16hi_to_f32(wv.x)));
        u.y = pack_bf16x2_rn(nb(a0.z, bf16lo_to_f32(wv.y)), nb(a0.w, bf16hi_to_f32(wv.y)));
        u.z = pack_bf16x2_rn(nb(a1.x, bf16lo_to_f32(wv.z)), nb(a1.y, bf16hi_to_f32(wv.z)));
        u.w = pack_bf16x2_rn(nb(a1.z, bf16lo_to_f32(wv.w)), nb(a1.w, bf16hi_to_f32(wv.w)));
      } else {
        u = xv[v];
      }
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
      float f[8], mx = 0.f, sm = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        f[2 * i] = bf16lo_to_f32(w[i]);
        f[2 * i + 1] = bf16hi_to_f32(w[i]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        mx = fmaxf(mx, fabsf(f[i]));
        sm += f[i];
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      sm += __shfl_xor_sync(0xffffffffu, sm, 1);
      sm += __shfl_xor_sync(0xffffffffu, sm, 2);
      const int e = gemv_scale_exp(__float_as_uint(mx));
      const float sc = pow2f(e);
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __half2 hv = __floats2half2_rn(f[2 * i] * sc, f[2 * i + 1] * sc);
        o[i] = *reinterpret_cast<const uint32_t*>(&hv);
      }
      xv[v] = make_uint4(o[0], o[1], o[2], o[3]);
      if ((lane & 3) == 0) {
        xs_s[(v >> 2) * 8] = sm;
        xs_s[(v >> 2) * 8 + 1] = pow2f(-e);
      }
    }
    named_barrier(1, kGemvConsumers);
  }
  uint32_t seq = 0;
  for (int grp = blockIdx.y; grp < p.n_groups; grp += gridDim.y) {
    if (kB1able && b1) {
      // warp = (row block rb, k-block half kh, stage parity phs): 4 warps share a
      // stage.  Block 4*kh + j of a K-tile goes to MMA column 2*j + kh, so lane t
      // folds exactly one block (4*kh + t) and lanes with g = 2*j + kh feed B.
      const int kh = (warp >> 1) & 1, phs = warp >> 2;
      const int xblk = 4 * kh + (g >> 1);  // the block whose x this lane feeds
      float tb[4][2];
#pragma unroll
      for (int s = 0; s < 4; ++s) tb[s][0] = tb[s][1] = 0.f;
      const uint32_t seq0 = seq;
      for (int kk = 0; kk < kt_cnt; ++kk) {
        const uint32_t sq = seq0 + kk;
        if (static_cast<int>(sq & 1) != phs) continue;
        const int slot = sq % stages;
        uint32_t xw[2][2];
#pragma unroll
        for (int st = 0; st < 2; ++st) {
          const uint32_t* xr = x32 + (kk * 256 + xblk * 32 + st * 16) / 2 + t;
          xw[st][0] = xr[0];
          xw[st][1] = xr[4];
        }
        mbar_wait_bounded(smem_u32(&bars[slot]), (sq / stages) & 1, abort_flag, kDevTimeoutFull);
        const uint8_t* tl = ring + slot * STAGE + tile * SLOT;
        float acc[4][4];
#pragma unroll
        for (int s = 0; s < 4; ++s) acc[s][0] = acc[s][1] = acc[s][2] = acc[s][3] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint8_t* nbj = tl + 1024 + rb * 2048 + (4 * kh + j) * 256 + 16 * t + 4 * h;
          const bool mine = g == 2 * j + kh;
#pragma unroll
          for (int st = 0; st < 2; ++st) {
            const uint8_t* nb = nbj + st * 128;
            const uint32_t p1 = *reinterpret_cast<const uint32_t*>(nb + off_first);
            const uint32_t p2 = *reinterpret_cast<const uint32_t*>(nb + off_second);
            const uint32_t q1 = *reinterpret_cast<const uint32_t*>(nb + 64 + off_first);
            const uint32_t q2 = *reinterpret_cast<const uint32_t*>(nb + 64 + off_second);
            uint32_t aP[8], aQ[8];
            decode_q4_pair_biased(p1, p2, sel_lo, sel_hi, aP);
            decode_q4_pair_biased(q1, q2, sel_lo, sel_hi, aQ);
            const uint32_t b0 = mine ? xw[st][0] : 0u, b1v = mine ? xw[st][1] : 0u;
#pragma unroll
            for (int s = 0; s < 4; ++s)
              mma_f16_m16n8k16(acc[s][0], acc[s][1], acc[s][2], acc[s][3], aP[2 * s], aP[2 * s + 1], aQ[2 * s],
                               aQ[2 * s + 1], b0, b1v);
          }
        }
        // fold block 4*kh + t (column 2t + kh): rows 2s (c0/c1) and 2s + 1 (c2/c3)
        // of the lane's 8.  Codes carry +1024 (even rows) / +64 (odd rows):
        // y += d * 2^-e * acc + (m - off * d) * sum(x)
        {
          const int kbl = 4 * kh + t;
          const uint8_t* meta = tl + (kbl * 32 + rb * 16 + h * 8) * 2;
          const uint4 dv = *reinterpret_cast<const uint4*>(meta);
          const uint4 mv = *reinterpret_cast<const uint4*>(meta + 512);
          const float2 si = *reinterpret_cast<const float2*>(xs_s + (kk * 8 + kbl) * 8);  // sum, 2^-e
          const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w}, mw[4] = {mv.x, mv.y, mv.z, mv.w};
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const float da = bf16lo_to_f32(dw[s]), db = bf16hi_to_f32(dw[s]);
            const float ca = kh ? acc[s][1] : acc[s][0], cb = kh ? acc[s][3] : acc[s][2];
            tb[s][0] = fmaf(da * si.y, ca, fmaf(fmaf(-1024.f, da, bf16lo_to_f32(mw[s])), si.x, tb[s][0]));
            tb[s][1] = fmaf(db * si.y, cb, fmaf(fmaf(-64.f, db, bf16hi_to_f32(mw[s])), si.x, tb[s][1]));
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bars[stages + slot]));
      }
      seq = seq0 + kt_cnt;
      // sum the four t lanes (their blocks) and park this warp's 8 rows per lane
#pragma unroll
      for (int s = 0; s < 4; ++s)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          tb[s][e] += __shfl_xor_sync(0xffffffffu, tb[s][e], 1);
          tb[s][e] += __shfl_xor_sync(0xffffffffu, tb[s][e], 2);
        }
      if (t == 0) {
        float* rw = red + warp * 64 * ncol;
#pragma unroll
        for (int s = 0; s < 4; ++s)
#pragma unroll
          for (int e = 0; e < 2; ++e) rw[(tile * 16 + h * 8 + 2 * s + e) * ncol] = tb[s][e];
      }
    } else {
    float tot[4][4 * NB];
#pragma unroll
    for (int s = 0; s < 4; ++s)
#pragma unroll
      for (int c = 0; c < 4 * NB; ++c) tot[s][c] = 0.f;

    for (int kk = 0; kk < kt_cnt; ++kk, ++seq) {
      const int slot = seq % stages;
      const uint32_t ph = (seq / stages) & 1;
      mbar_wait_bounded(smem_u32(&bars[slot]), ph, abort_flag, kDevTimeoutFull);
      const uint8_t* tl = ring + slot * STAGE + tile * SLOT;

#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int kb = 2 * kp + j;
        float part[4][4 * NB];
#pragma unroll
        for (int s = 0; s < 4; ++s)
#pragma unroll
          for (int c = 0; c < 4 * NB; ++c) part[s][c] = 0.f;

#pragma unroll
        for (int st = 0; st < 2; ++st) {
          const int kl = kk * 256 + kb * 32 + st * 16;
          uint32_t bx[NB][2];
#pragma unroll
          for (int n = 0; n < NB; ++n) {
            const int row = g + 8 * n;
            const uint32_t* xr = x32 + row * xw_stride + kl / 2 + t;
            bx[n][0] = row < batch ? xr[0] : 0u;
            bx[n][1] = row < batch ? xr[4] : 0u;
          }
          if (QT == kQ4) {
            const uint8_t* nb = tl + 1024 + rb * 2048 + kb * 256 + st * 128 + 16 * t + 4 * h;
            const uint32_t p1 = *reinterpret_cast<const uint32_t*>(nb + off_first);
            const uint32_t p2 = *reinterpret_cast<const uint32_t*>(nb + off_second);
            const uint32_t q1 = *reinterpret_cast<const uint32_t*>(nb + 64 + off_first);
            const uint32_t q2 = *reinterpret_cast<const uint32_t*>(nb + 64 + off_second);
            uint32_t aP[8], aQ[8];  // codes + 1024 (even rows) / + 64 (odd rows), folded below
            decode_q4_pair_biased(p1, p2, sel_lo, sel_hi, aP);
            decode_q4_pair_biased(q1, q2, sel_lo, sel_hi, aQ);
#pragma unroll
            for (int s = 0; s < 4; ++s)
#pragma unroll
              for (int n = 0; n < NB; ++n)
                mma_f16_m16n8k16(part[s][4 * n], part[s][4 * n + 1], part[s][4 * n + 2], part[s][4 * n + 3],
                                 aP[2 * s], aP[2 * s + 1], aQ[2 * s], aQ[2 * s + 1], bx[n][0], bx[n][1]);
          } else {
            // 16 bytes = 16 rows at one k; this lane reads rows h*8..h*8+7 (8 bytes)
            const uint8_t* cb = tl + 512 + rb * 4096 + kb * 512 + st * 256 + 8 * h + 32 * t;
            const uint2 pa = *reinterpret_cast<const uint2*>(cb);        // k = 2t
            const uint2 pb = *reinterpret_cast<const uint2*>(cb + 16);   // k = 2t+1
            const uint2 qa = *reinterpret_cast<const uint2*>(cb + 128);  // k = 2t+8
            const uint2 qb = *reinterpret_cast<const uint2*>(cb + 144);  // k = 2t+9
            const uint32_t paw[2] = {pa.x, pa.y}, pbw[2] = {pb.x, pb.y};
            const uint32_t qaw[2] = {qa.x, qa.y}, qbw[2] = {qb.x, qb.y};
#pragma unroll
            for (int q = 0; q < 2; ++q) {    // rows 4q..4q+3 of the lane's 8
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {  // rows 4q+2hh, 4q+2hh+1 = MMA s
                const uint32_t sel = hh ? 0x7632u : 0x5410u;
                uint32_t pA, pB, qA, qB;  // rows 4q+2hh (A) and 4q+2hh+1 (B) at (k, k+1), (k+8, k+9)
                decode_q8_pair(prmt(paw[q], pbw[q], sel), pA, pB);
                decode_q8_pair(prmt(qaw[q], qbw[q], sel), qA, qB);
                const int s = 2 * q + hh;
#pragma unroll
                for (int n = 0; n < NB; ++n)
                  mma_f16_m16n8k16(part[s][4 * n], part[s][4 * n + 1], part[s][4 * n + 2], part[s][4 * n + 3],
                                   pA, pB, qA, qB, bx[n][0], bx[n][1]);
              }
            }
          }
        }

        // fold this k-block: tot += d*part + m'*sum(x'), m' = m - code offset * d
        // (q4: offset 1024 for even rows, 64 for odd rows; q8: m' = -1152*s)
        const uint8_t* meta = tl + (kb * 32 + rb * 16 + h * 8) * 2;
        const uint4 dv = *reinterpret_cast<const uint4*>(meta);
        const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
        uint32_t mw[4] = {0, 0, 0, 0};
        if (QT == kQ4) {
          const uint4 mv = *reinterpret_cast<const uint4*>(meta + 512);
          mw[0] = mv.x; mw[1] = mv.y; mw[2] = mv.z; mw[3] = mv.w;
        }
        float2 xsv[NB];
#pragma unroll
        for (int n = 0; n < NB; ++n)
          xsv[n] = *reinterpret_cast<const float2*>(xs_s + (kk * 8 + kb) * 8 * NB + 8 * n + 2 * t);
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const float da = bf16lo_to_f32(dw[s]), db = bf16hi_to_f32(dw[s]);
          float ma, mb;
          if (QT == kQ4) {
            ma = fmaf(-1024.f, da, bf16lo_to_f32(mw[s]));
            mb = fmaf(-64.f, db, bf16hi_to_f32(mw[s]));
          } else {
            ma = -1152.f * da;
            mb = -1152.f * db;
          }
#pragma unroll
          for (int n = 0; n < NB; ++n) {
            tot[s][4 * n + 0] = fmaf(da, part[s][4 * n + 0], fmaf(ma, xsv[n].x, tot[s][4 * n + 0]));
            tot[s][4 * n + 1] = fmaf(da, part[s][4 * n + 1], fmaf(ma, xsv[n].y, tot[s][4 * n + 1]));
            tot[s][4 * n + 2] = fmaf(db, part[s][4 * n + 2], fmaf(mb, xsv[n].x, tot[s][4 * n + 2]));
            tot[s][4 * n + 3] = fmaf(db, part[s][4 * n + 3], fmaf(mb, xsv[n].y, tot[s][4 * n + 3]));
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars[stages + slot]));
    }

    // ------------------------------------------------------------ epilogue
    {
      // undo the x scale (exact power of two) and park the warp's totals:
      // red[warp][64 local rows = tile*16 + h*8 + r][ncol]
      float* rw = red + warp * 64 * ncol;
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        const int c0 = 8 * n + 2 * t;
        if (c0 < batch) {
          const float u0 = pow2f(-exps[c0]);
          const float u1 = (c0 + 1 < batch) ? pow2f(-exps[c0 + 1]) : 0.f;
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const int lr = tile * 16 + h * 8 + 2 * s;
            *reinterpret_cast<float2*>(rw + lr * ncol + c0) = make_float2(tot[s][4 * n] * u0, tot[s][4 * n + 1] * u1);
            *reinterpret_cast<float2*>(rw + (lr + 1) * ncol + c0) =
                make_float2(tot[s][4 * n + 2] * u0, tot[s][4 * n + 3] * u1);
          }
        }
      }
    }
    }  // batch-1 / general stage loop
    named_barrier(1, kGemvConsumers);
    // CTA sum over the 4 warps that hold each row (fixed order).
    const int nsp = p.n_splits;
    const bool do_store = !*abort_flag;
    if (EPI == kEpiF32) {
      float* y = static_cast<float*>(p.y);
      if (!clustered) {
        for (int e = ctid; e < kGroupRows * batch; e += kGemvConsumers) {
          const int row = e % kGroupRows, b = e / kGroupRows;
          const int rbr = (row >> 4) & 1, lr = (row >> 5) * 16 + (row & 15);
          float v = 0.f;
#pragma unroll
          for (int q = 0; q < 4; ++q) v += red[(2 * q + rbr) * 64 * ncol + lr * ncol + b];
          const int tr = grp * 4 + (row >> 5);
          if (do_store && tr < p.n_tile_rows) {
            float* dst = y + static_cast<size_t>(b) * p.ldy + grp * kGroupRows + row;
            *dst = p.accumulate ? *dst + v : v;
          }
        }
        named_barrier(1, kGemvConsumers);  // red is rewritten by the next group
      } else {
        if (cl_mode == 1) cluster_wait_acquire();  // rank 0 has zeroed y
        for (int e = ctid; e < kGroupRows * batch; e += kGemvConsumers) {
          const int row = e % kGroupRows, b = e / kGroupRows;
          const int rbr = (row >> 4) & 1, lr = (row >> 5) * 16 + (row & 15);
          float v = 0.f;
#pragma unroll
          for (int q = 0; q < 4; ++q) v += red[(2 * q + rbr) * 64 * ncol + lr * ncol + b];
          const int tr = grp * 4 + (row >> 5);
          if (do_store && tr < p.n_tile_rows)
            atomicAdd(y + static_cast<size_t>(b) * p.ldy + grp * kGroupRows + row, v);
        }
      }
    } else {
      // SwiGLU: sum rows 0..63 are gate rows grp*64.., rows 64..127 the matching up rows.
      // Clustered: push to the owning rank (gather[src rank][owned row][g|u]).
      const int rows_per = (64 + nsp - 1) / nsp;
      float* gather = reinterpret_cast<float*>(smem + L.gather);
      const uint32_t gather_addr = smem_u32(gather);
      for (int e = ctid; e < kGroupRows * ncol; e += kGemvConsumers) {
        const int row = e / ncol, col = e % ncol;
        const int rbr = (row >> 4) & 1, lr = (row >> 5) * 16 + (row & 15);
        float v = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) v += red[(2 * q + rbr) * 64 * ncol + lr * ncol + col];
        if (!clustered) {
          csum[e] = v;
        } else {
          const int orow = row & 63;
          const int o = orow / rows_per, ol = orow - o * rows_per;
          st_dsmem_f32(gather_addr + (((split * rows_per + ol) * 2 + (row >> 6)) * ncol + col) * 4, o, v);
        }
      }
      if (clustered)
        cluster_sync_all();
      else
        named_barrier(1, kGemvConsumers);
      const int r_lo = split * rows_per, r_hi = min(64, r_lo + rows_per);
      const int nrow = r_hi - r_lo;
      __nv_bfloat16* hout = static_cast<__nv_bfloat16*>(p.y);
      for (int e = ctid; e < nrow * batch; e += kGemvConsumers) {
        const int ol = e % nrow, b = e / nrow, row = r_lo + ol;
        float gv = 0.f, uv = 0.f;
        if (clustered) {
          for (int q = 0; q < nsp; ++q) {
            gv += gather[((q * rows_per + ol) * 2 + 0) * ncol + b];
            uv += gather[((q * rows_per + ol) * 2 + 1) * ncol + b];
          }
        } else {
          gv = csum[row * ncol + b];
          uv = csum[(row + 64) * ncol + b];
        }
        // the reference narrows both accumulators to bf16 before SiLU (granite_mlp.py:172-181)
        const float gb = __bfloat162float(__float2bfloat16_rn(gv));
        const float ub = __bfloat162float(__float2bfloat16_rn(uv));
        const float hv = gb / (1.f + expf(-gb)) * ub;
        const int tr = grp * 2 + (row >> 5);
        if (do_store && tr < p.n_tile_rows)
          hout[static_cast<size_t>(b) * p.ldy + grp * 64 + row] = __float2bfloat16_rn(hv);
      }
      if (!clustered) named_barrier(1, kGemvConsumers);  // csum is rewritten by the next group
    }
  }
}

}  // namespace b2
