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
// The quantisation block factors out of the dot product exactly as in the
// reference kernel (granite_gemv.h:19-29):
//   y[r] = sum_kb  d[kb][r] * (sum_{k in kb} code*x)  +  m[kb][r] * (sum_{k in kb} x)
// The inner sums run on the tensor core with *exact* bf16 codes:
//   * a nibble n is turned into the bf16 value 128+n by one LOP3 against the
//     exponent pattern 0x4300 (a bf16 in [128,256) has an ulp of 1) and 128 is
//     subtracted exactly, so A holds the integer code itself;
//   * q8 codes are split as c = 16*uh + ul - 128 (uh, ul the nibbles of c^0x80),
//     two exact MMAs against x and 16*x, and the -128 folds into the sum-of-x term.
// Products code*x are exact in fp32, so the only rounding is fp32 accumulation.
//
// Data flow per CTA (one "row group" = 4 tile-rows = 128 outputs, or for the
// fused SwiGLU 2 gate + 2 up tile-rows):
//   producer warp: cp.async.bulk (TMA, no multicast) of the group's 4 tiles at
//                  one K-tile into a stage of a shared-memory ring, mbarrier
//                  complete_tx; L2 evict-first (weights are streamed once);
//   8 consumer warps: warp w owns k-block w of every K-tile.  A thread (g,t)
//                  of the warp owns row-block g of the stage (tile g%4, rb g/4)
//                  and k-pairs {2t,2t+1}, {2t+8,2t+9} of each 16-k MMA step:
//                  two 16-byte shared loads, PRMT+LOP3 into A fragments, 8 MMAs
//                  (m16n8k16; the 16 "M" rows are rows 2s,2s+1 of 8 row-blocks)
//                  with x as the B operand (N = batch), then the d/m scaling
//                  into fp32 totals;
//   epilogue:      warp totals -> shared memory -> CTA sum (fixed order) ->
//                  split-K sum across a thread-block cluster through
//                  distributed shared memory (fixed order) -> store.
// Split-K across CTAs uses a cluster (no global workspace, deterministic);
// groups larger than the GPU use a persistent grid with the producer running
// ahead across group boundaries.
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
  static constexpr int kSlot = 5184;  // +64 B: row-blocks of adjacent tiles hit disjoint banks
};
template <>
struct QTraits<kQ8> {
  static constexpr int kTile = 8704;
  static constexpr int kSlot = 8720;  // +16 B, same reason for the 32-byte q8 reads
};

constexpr int kGemvConsumerWarps = 8;  // one per 32-k block of a K-tile
constexpr int kGemvThreads = (kGemvConsumerWarps + 1) * 32;
constexpr int kGroupRows = 128;
constexpr int kMaxStages = 8;

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
  int x_stride;  // bf16 per shared-memory x row = kt_per_split*256 + 8
  int prefetch_before_wait;  // weights may stream before the PDL wait
};

// Shared-memory layout (bytes), computed identically on host and device.
struct GemvSmem {
  int ring, x, xs, red, csum, bar, flag, total;
  __host__ __device__ static constexpr int red_warp_floats(int nb) { return kGroupRows * 8 * nb + 24; }
  __host__ __device__ GemvSmem(int qt_slot, int nb, int stages, int x_stride, int kt_per_split) {
    ring = 0;
    x = stages * 4 * qt_slot;
    xs = x + 8 * nb * x_stride * 2;
    red = xs + kt_per_split * 8 * 8 * nb * 4;
    csum = red + kGemvConsumerWarps * red_warp_floats(nb) * 4;
    bar = csum + kGroupRows * 8 * nb * 4;
    bar = (bar + 15) & ~15;
    flag = bar + 2 * stages * 8;
    total = flag + 16;
  }
};

__device__ __forceinline__ int red_index(int row, int col, int nb) {
  // row-major [128][8nb], each 32-row tile shifted by 8 floats so that the
  // 4 tiles written by one quarter-warp land in different banks
  return row * 8 * nb + col + 8 * (row >> 5);
}

template <int QT, int NB, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 1) q4nx_gemv_kernel(const GemvParams p) {
  constexpr int TILE = QTraits<QT>::kTile;
  constexpr int SLOT = QTraits<QT>::kSlot;
  constexpr int STAGE = 4 * SLOT;
  extern __shared__ __align__(128) uint8_t smem[];

  const GemvSmem L(SLOT, NB, p.stages, p.x_stride, p.kt_per_split);
  uint8_t* ring = smem + L.ring;
  __nv_bfloat16* x_s = reinterpret_cast<__nv_bfloat16*>(smem + L.x);
  float* xs_s = reinterpret_cast<float*>(smem + L.xs);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* csum = reinterpret_cast<float*>(smem + L.csum);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.flag);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int stages = p.stages;
  const bool clustered = p.n_splits > 1;
  const int split = clustered ? static_cast<int>(cluster_ctarank()) : 0;
  const int kt0 = split * p.kt_per_split;
  const int kt_cnt = min(p.kt_per_split, p.k_tiles - kt0);  // >= 1 by construction

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&bars[s]), 1);                             // full: producer + tx
      mbar_init(smem_u32(&bars[stages + s]), kGemvConsumerWarps);  // empty: one per warp
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kGemvConsumerWarps) {
    // ------------------------------------------------------------ producer
    const uint64_t policy = l2_evict_first_policy();
    uint32_t seq = 0;
    bool waited_pdl = false;
    if (!p.prefetch_before_wait) {
      pdl_wait();
      waited_pdl = true;
    }
    for (int grp = blockIdx.y; grp < p.n_groups; grp += gridDim.y) {
      for (int kk = 0; kk < kt_cnt; ++kk, ++seq) {
        if (lane == 0 && !*abort_flag) {
          const int slot = seq % stages;
          const uint32_t ph = (seq / stages) & 1;
          bool ok = true;
          if (seq >= static_cast<uint32_t>(stages)) {
            if (!waited_pdl) {  // ring full: nothing more to prefetch before the dependency
              pdl_wait();
              waited_pdl = true;
            }
            ok = mbar_wait_bounded(smem_u32(&bars[stages + slot]), ph ^ 1, abort_flag, kDevTimeoutEmpty);
          }
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
      if (clustered) {  // mirror the consumers' two cluster barriers of this group
        cluster_sync_all();
        cluster_sync_all();
      }
    }
    if (!waited_pdl) pdl_wait();
    __syncwarp();
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
  const int ctid = threadIdx.x;  // 0..255
  const int L_cta = kt_cnt * 256;
  {
    // stage x[b][kt0*256 .. +L_cta) (zero rows for b >= batch), 16 bytes a thread at a time
    const int vec_per_row = L_cta / 8;
    for (int v = ctid; v < 8 * NB * vec_per_row; v += kGemvConsumerWarps * 32) {
      const int b = v / vec_per_row, c = v % vec_per_row;
      uint4 val = make_uint4(0, 0, 0, 0);
      if (b < p.batch)
        val = *reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(b) * p.ldx + kt0 * 256 + c * 8);
      *reinterpret_cast<uint4*>(x_s + b * p.x_stride + c * 8) = val;
    }
    named_barrier(1, kGemvConsumerWarps * 32);
    // per-32-k-block sums of x (fp32), [kb_local][8*NB]
    const int nsum = kt_cnt * 8 * 8 * NB;
    for (int v = ctid; v < nsum; v += kGemvConsumerWarps * 32) {
      const int kbl = v / (8 * NB), b = v % (8 * NB);
      const __nv_bfloat16* xr = x_s + b * p.x_stride + kbl * 32;
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) acc += __bfloat162float(xr[j]);
      xs_s[v] = acc;
    }
    named_barrier(1, kGemvConsumerWarps * 32);
  }

  const int g = lane >> 2, t = lane & 3;
  const int tslot = g & 3, rb = g >> 2;
  const int kb = warp;
  const uint32_t* x32 = reinterpret_cast<const uint32_t*>(x_s);
  const int xw_stride = p.x_stride / 2;
  const uint32_t kMagic = 0x43004300u;  // bf16x2 (128, 128)
  const uint32_t kSixteen = 0x41804180u;  // bf16x2 (16, 16)

  uint32_t seq = 0;
  for (int grp = blockIdx.y; grp < p.n_groups; grp += gridDim.y) {
    float tot[8][4 * NB];
#pragma unroll
    for (int s = 0; s < 8; ++s)
#pragma unroll
      for (int c = 0; c < 4 * NB; ++c) tot[s][c] = 0.f;

    for (int kk = 0; kk < kt_cnt; ++kk, ++seq) {
      const int slot = seq % stages;
      const uint32_t ph = (seq / stages) & 1;
      mbar_wait_bounded(smem_u32(&bars[slot]), ph, abort_flag, kDevTimeoutFull);

      const uint8_t* tile = ring + slot * STAGE + tslot * SLOT;
      const int kl = kk * 256 + kb * 32;  // local k of this k-block
      float part[8][4 * NB];
#pragma unroll
      for (int s = 0; s < 8; ++s)
#pragma unroll
        for (int c = 0; c < 4 * NB; ++c) part[s][c] = 0.f;

#pragma unroll
      for (int st = 0; st < 2; ++st) {
        uint32_t bx[NB][2];
#pragma unroll
        for (int n = 0; n < NB; ++n) {
          const uint32_t* xr = x32 + (g + 8 * n) * xw_stride + (kl + st * 16) / 2 + t;
          bx[n][0] = xr[0];
          bx[n][1] = xr[4];
        }
        if (QT == kQ4) {
          const uint8_t* nb = tile + 1024 + rb * 2048 + kb * 256 + st * 128;
          const uint4 P = *reinterpret_cast<const uint4*>(nb + 16 * t);
          const uint4 Q = *reinterpret_cast<const uint4*>(nb + 64 + 16 * t);
          uint32_t aP[16], aQ[16];
          // P = [k_a rows 0-7 | k_a rows 8-15 | k_b rows 0-7 | k_b rows 8-15], 4 bytes each
          const uint32_t pw[4] = {P.x, P.y, P.z, P.w};
          const uint32_t qw[4] = {Q.x, Q.y, Q.z, Q.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t sel = (q & 1) ? 0x7632u : 0x5410u;
            const uint32_t rp = prmt(pw[q >> 1], pw[2 + (q >> 1)], sel);
            const uint32_t rq = prmt(qw[q >> 1], qw[2 + (q >> 1)], sel);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              aP[4 * q + j] = bf16x2_sub(lop3<kLutAndOr>(rp >> (4 * j), 0x000F000Fu, kMagic), kMagic);
              aQ[4 * q + j] = bf16x2_sub(lop3<kLutAndOr>(rq >> (4 * j), 0x000F000Fu, kMagic), kMagic);
            }
          }
#pragma unroll
          for (int s = 0; s < 8; ++s)
#pragma unroll
            for (int n = 0; n < NB; ++n)
              mma_bf16_m16n8k16(part[s][4 * n], part[s][4 * n + 1], part[s][4 * n + 2], part[s][4 * n + 3],
                                aP[2 * s], aP[2 * s + 1], aQ[2 * s], aQ[2 * s + 1], bx[n][0], bx[n][1]);
        } else {
          // q8: 16 bytes = 16 rows at one k; k_a, k_b (pair P) then k_c, k_d (pair Q)
          const uint8_t* cb = tile + 512 + rb * 4096 + kb * 512 + st * 256;
          const uint4 A = *reinterpret_cast<const uint4*>(cb + 32 * t);
          const uint4 B = *reinterpret_cast<const uint4*>(cb + 32 * t + 16);
          const uint4 C = *reinterpret_cast<const uint4*>(cb + 128 + 32 * t);
          const uint4 D = *reinterpret_cast<const uint4*>(cb + 128 + 32 * t + 16);
          const uint32_t aw[4] = {A.x, A.y, A.z, A.w}, bw[4] = {B.x, B.y, B.z, B.w};
          const uint32_t cw[4] = {C.x, C.y, C.z, C.w}, dw[4] = {D.x, D.y, D.z, D.w};
          uint32_t bx16[NB][2];
#pragma unroll
          for (int n = 0; n < NB; ++n) {
            bx16[n][0] = bf16x2_mul(bx[n][0], kSixteen);
            bx16[n][1] = bf16x2_mul(bx[n][1], kSixteen);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {     // word q = rows 4q..4q+3
#pragma unroll
            for (int h = 0; h < 2; ++h) {   // rows 4q+2h, 4q+2h+1
              const uint32_t sel = h ? 0x7632u : 0x5410u;
              const uint32_t rp = prmt(aw[q], bw[q], sel);
              const uint32_t rq = prmt(cw[q], dw[q], sel);
              // low nibbles (ul) and flipped high nibbles (uh = (c^0x80)>>4)
              const uint32_t pl0 = bf16x2_sub(lop3<kLutAndOr>(rp, 0x000F000Fu, kMagic), kMagic);
              const uint32_t pl1 = bf16x2_sub(lop3<kLutAndOr>(rp >> 8, 0x000F000Fu, kMagic), kMagic);
              const uint32_t ph0 = bf16x2_sub(lop3<kLutAndXor>(rp >> 4, 0x000F000Fu, 0x43084308u), kMagic);
              const uint32_t ph1 = bf16x2_sub(lop3<kLutAndXor>(rp >> 12, 0x000F000Fu, 0x43084308u), kMagic);
              const uint32_t ql0 = bf16x2_sub(lop3<kLutAndOr>(rq, 0x000F000Fu, kMagic), kMagic);
              const uint32_t ql1 = bf16x2_sub(lop3<kLutAndOr>(rq >> 8, 0x000F000Fu, kMagic), kMagic);
              const uint32_t qh0 = bf16x2_sub(lop3<kLutAndXor>(rq >> 4, 0x000F000Fu, 0x43084308u), kMagic);
              const uint32_t qh1 = bf16x2_sub(lop3<kLutAndXor>(rq >> 12, 0x000F000Fu, 0x43084308u), kMagic);
              const int s = 2 * q + h;  // MMA index: rows 2s, 2s+1
#pragma unroll
              for (int n = 0; n < NB; ++n) {
                mma_bf16_m16n8k16(part[s][4 * n], part[s][4 * n + 1], part[s][4 * n + 2],
                                  part[s][4 * n + 3], pl0, pl1, ql0, ql1, bx[n][0], bx[n][1]);
                mma_bf16_m16n8k16(part[s][4 * n], part[s][4 * n + 1], part[s][4 * n + 2],
                                  part[s][4 * n + 3], ph0, ph1, qh0, qh1, bx16[n][0], bx16[n][1]);
              }
            }
          }
        }
      }

      // fold this k-block: tot += d*part + m*sum(x)   (q8: m = -128*s)
      {
        const uint8_t* meta = tile + (kb * 32 + rb * 16) * 2;
        const uint4 d0 = *reinterpret_cast<const uint4*>(meta);
        const uint4 d1 = *reinterpret_cast<const uint4*>(meta + 16);
        const uint32_t dw[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
        uint32_t mw[8];
        if (QT == kQ4) {
          const uint4 m0 = *reinterpret_cast<const uint4*>(meta + 512);
          const uint4 m1 = *reinterpret_cast<const uint4*>(meta + 528);
          mw[0] = m0.x; mw[1] = m0.y; mw[2] = m0.z; mw[3] = m0.w;
          mw[4] = m1.x; mw[5] = m1.y; mw[6] = m1.z; mw[7] = m1.w;
        }
        float2 xsv[NB];
#pragma unroll
        for (int n = 0; n < NB; ++n)
          xsv[n] = *reinterpret_cast<const float2*>(xs_s + (kk * 8 + kb) * 8 * NB + 8 * n + 2 * t);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const float da = bf16lo_to_f32(dw[s]), db = bf16hi_to_f32(dw[s]);
          float ma, mb;
          if (QT == kQ4) {
            ma = bf16lo_to_f32(mw[s]);
            mb = bf16hi_to_f32(mw[s]);
          } else {
            ma = -128.f * da;
            mb = -128.f * db;
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
      float* rw = red + warp * GemvSmem::red_warp_floats(NB);
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const int r0 = tslot * 32 + rb * 16 + 2 * s;
#pragma unroll
        for (int n = 0; n < NB; ++n) {
          *reinterpret_cast<float2*>(rw + red_index(r0, 8 * n + 2 * t, NB)) =
              make_float2(tot[s][4 * n + 0], tot[s][4 * n + 1]);
          *reinterpret_cast<float2*>(rw + red_index(r0 + 1, 8 * n + 2 * t, NB)) =
              make_float2(tot[s][4 * n + 2], tot[s][4 * n + 3]);
        }
      }
    }
    named_barrier(1, kGemvConsumerWarps * 32);
    for (int e = ctid; e < kGroupRows * 8 * NB; e += kGemvConsumerWarps * 32) {
      const int row = e / (8 * NB), col = e % (8 * NB);
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kGemvConsumerWarps; ++w) v += red[w * GemvSmem::red_warp_floats(NB) + red_index(row, col, NB)];
      csum[e] = v;
    }
    if (clustered)
      cluster_sync_all();
    else
      named_barrier(1, kGemvConsumerWarps * 32);

    // split-K sum over the cluster (fixed rank order), then the epilogue
    const int nsp = p.n_splits;
    const bool do_store = !*abort_flag;
    const uint32_t csum_addr = smem_u32(csum);
    if (EPI == kEpiF32) {
      const int rows_per = (kGroupRows + nsp - 1) / nsp;
      const int r_lo = split * rows_per, r_hi = min(kGroupRows, r_lo + rows_per);
      const int nrow = r_hi - r_lo;
      float* y = static_cast<float*>(p.y);
      for (int e = ctid; e < nrow * p.batch; e += kGemvConsumerWarps * 32) {
        const int row = r_lo + e % nrow, b = e / nrow;
        const int idx = row * 8 * NB + b;
        float v = 0.f;
        if (clustered) {
          for (int q = 0; q < nsp; ++q) v += ld_dsmem_f32(csum_addr + idx * 4, q);
        } else {
          v = csum[idx];
        }
        const int tr = grp * 4 + (row >> 5);
        if (do_store && tr < p.n_tile_rows) {
          float* dst = y + static_cast<size_t>(b) * p.ldy + grp * kGroupRows + row;
          *dst = p.accumulate ? *dst + v : v;
        }
      }
    } else {
      // SwiGLU: sum rows 0..63 are gate rows grp*64.., rows 64..127 the matching up rows
      const int rows_per = (64 + nsp - 1) / nsp;
      const int r_lo = split * rows_per, r_hi = min(64, r_lo + rows_per);
      const int nrow = r_hi - r_lo;
      __nv_bfloat16* h = static_cast<__nv_bfloat16*>(p.y);
      for (int e = ctid; e < nrow * p.batch; e += kGemvConsumerWarps * 32) {
        const int row = r_lo + e % nrow, b = e / nrow;
        const int ig = row * 8 * NB + b, iu = (row + 64) * 8 * NB + b;
        float gv = 0.f, uv = 0.f;
        if (clustered) {
          for (int q = 0; q < nsp; ++q) {
            gv += ld_dsmem_f32(csum_addr + ig * 4, q);
            uv += ld_dsmem_f32(csum_addr + iu * 4, q);
          }
        } else {
          gv = csum[ig];
          uv = csum[iu];
        }
        // the reference narrows both accumulators to bf16 before SiLU (granite_mlp.py:172-181)
        const float gb = __bfloat162float(__float2bfloat16_rn(gv));
        const float ub = __bfloat162float(__float2bfloat16_rn(uv));
        const float hv = gb / (1.f + expf(-gb)) * ub;
        const int tr = grp * 2 + (row >> 5);
        if (do_store && tr < p.n_tile_rows)
          h[static_cast<size_t>(b) * p.ldy + grp * 64 + row] = __float2bfloat16_rn(hv);
      }
    }
    if (clustered) cluster_sync_all();
  }
}

}  // namespace b2
