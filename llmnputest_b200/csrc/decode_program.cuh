// Persistent decode program for sm_100a: one cooperative launch runs a list of
// phases -- q4nx GEMVs, GQA decode attention, a preparation step -- with a
// grid-wide barrier after every phase whose outputs the next one reads.
//
// Why: at batch 1 the decode step of a 3B model is ~200 small dependent
// operations (QKV 5.7 MB, O 4.1 MB of tiles ...), each shorter than a kernel
// launch plus its prologue.  Weights do not depend on activations, so one
// producer warp per SM streams every phase's tiles into the shared-memory ring
// without waiting for the barriers; only the consumers wait.  The ring (7-9
// stages of 20 KB) covers the barrier latency, and HBM keeps streaming across
// the phase boundaries.
//
// A step of the dense GQA decoder (designs/granite_gemv/granite_layer.py:54-59):
//   (a small kernel before the launch: RoPE cos/sin per sequence, fp64 angles
//   rounded to fp32 as in the one-shot attention kernel)
//   prep    resid = x_in; zero the first split-K targets; barrier
//   per layer
//     GEMV  qkv[l&1] += W_qkv bf16(rmsnorm(resid))           barrier
//     ATTN  rope(q), rope(k) -> cache, v -> cache; split partials (o, m, l)
//           zero qkv[(l+1)&1], gu[(l+1)&1] for the next layer  barrier
//     GEMV  resid += W_o bf16(merge of the partials)         barrier
//     GEMV  gu[l&1][:, :I] += W_gate bf16(rmsnorm(resid))    (no barrier)
//     GEMV  gu[l&1][:, I:] += W_up   bf16(rmsnorm(resid))    barrier
//     GEMV  resid += W_down bf16(silu(bf16 g) * bf16 u)      barrier
// (the final norm + q8 lm_head run as the next launch).  Every GEMV output is
// a split-K sum with fp32 atomics into a zeroed buffer or the residual, so a
// CTA can take any contiguous run of (tile-row group, K-tile) stages and all
// 148 SMs share every phase evenly.  The merge of attention splits and the
// SwiGLU nonlinearity run in the prologue of the GEMV that consumes them.
//
// Arithmetic per element matches the one-launch-per-op kernels: exact
// code * x products on the tensor core with fp32 accumulation (here bf16
// operands: codes 0..15 and the bf16 x are both exact in bf16, so x needs no
// per-row rescaling), the same q4_1 factoring, RMSNorm, SwiGLU, RoPE and online
// softmax (q4nx_gemv.cuh, gqa_decode.cuh); only fp32 summation order differs.
// Consumers: 12 warps.  Batch >= 2: 8 of them split each stage by (row-block,
// pair of 32-k blocks).  Batch 1: a different split (prog_gemv_phase_b1).  A
// unit's warp sums meet in shared memory and leave as one fp32 reduction per
// output at L2.
//
// Synchronisation: the grid barrier is an arrival counter in caller memory
// (zeroed before each launch) released with a gpu-scope fence and polled with
// ld.acquire.gpu by one thread per CTA, which then releases its CTA with a CTA
// barrier.  Data written earlier in the launch is read with ordinary loads:
// the acquire orders them after the other CTAs' writes (PTX memory model:
// release -> acquire -> bar.sync is causality order), and no phase reads what
// another CTA writes in the same phase.  Every wait is bounded
// (B2_WAIT_TIMEOUT_NS): a barrier that times out records kDevTimeoutGrid,
// raises the launch-wide abort word, and every CTA leaves at its next barrier;
// producers drain their copies in flight before exiting.  All CTAs must be
// resident at once: the launch is cooperative, one CTA per SM.
#pragma once

#include "gqa_decode.cuh"
#include "q4nx_gemv.cuh"

namespace b2 {

enum ProgKind : int { kPhGemv = 0, kPhAttn = 1, kPhPrep = 2 };
enum ProgXSrc : int { kXBf16 = 0, kXNorm = 1, kXAttn = 2, kXSwiglu = 3 };

// Consumer warps.  13 warps per CTA (with the producer) are budgeted as 16 by the
// register allocator, so each thread may hold 128 registers.
constexpr int kProgWarps = 12;
constexpr int kNbWarps = 8;  // batch >= 2: warps (row-block, pair of 32-k blocks) of a stage
constexpr int kProgConsumers = kProgWarps * 32;
constexpr int kProgThreads = kProgConsumers + 32;
constexpr int kProgMaxBatch = 8;
constexpr int kProgUnitKt = 8;  // K-tiles of one unit at most (its x slice is staged in shared memory)
// K-tiles per unit for a batch: the staged x of two units must leave room for the ring
__host__ __device__ constexpr int prog_unit_kt(int batch) { return batch <= 4 ? kProgUnitKt : kProgUnitKt / 2; }
constexpr int kProgSlot = QTraits<kQ4>::kSlot;
constexpr int kProgStage = 4 * kProgSlot;
__host__ __device__ constexpr int prog_x_stride(int batch) { return prog_unit_kt(batch) * 256 + 8; }  // bf16 per x row
constexpr int kProgMaxStages = 12;
constexpr int kAttnQW = 64 / 2 + 4;  // q_s row stride in 32-bit words
constexpr int kProgAttnBytes = 16 * kAttnQW * 4 + 2 * kProgWarps * 16 * 4 + kProgWarps * 8 * 65 * 4;
constexpr int kPartStride = 64 + 2;  // floats per (split, q head) partial: o[64], m, l

// Device mirror of b2_phase (include/b2q4nx.h): same fields, order and sizes.
struct ProgPhase {
  int32_t kind, x_source, barrier_after, n_tile_rows;
  int32_t k_tiles, ldx, half, ldy;
  int32_t n_q_heads, n_kv_heads, n_splits, split_len;
  int32_t ld_qkv, ctx_max, zero0_n, zero1_n;
  int32_t copy_n;
  float eps;
  float scale_log2;
  int32_t reserved;
  const uint8_t* w;
  const void* x;
  const __nv_bfloat16* norm_w;
  float* y;
  float* part;
  const float* qkv;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  float* zero0;
  float* zero1;
  const float* copy_src;
  float* copy_dst;
};

struct ProgParams {
  const ProgPhase* phases;
  int n_phases;
  int batch;
  int stages;
  float theta;
  const int* pos;         // [batch] position of the new token
  float* rope;            // [batch][32][2] cos, sin (written by prog_rope_kernel)
  unsigned int* barrier;  // [0] arrivals, [1] abort word; zeroed before the launch
};

// Shared-memory layout (bytes), identical on host and device.  The work area is
// used either by GEMV units (two slots of staged x and per-32-k sums, so one
// unit's staging never waits for the previous unit's readers; misc) or by an
// attention unit (q heads, per-warp m/l/o); the two never overlap in time.
struct ProgSmem {
  int ring, work, xslot, xs, xs_slot, red, misc, bar, flag, total;
  __host__ __device__ ProgSmem(int stages, int batch) {
    const int ncol = (batch + 1) & ~1;
    ring = 0;
    work = stages * kProgStage;
    xslot = (batch * prog_x_stride(batch) * 2 + 15) & ~15;  // bytes of one x slot
    xs = work + 2 * xslot;
    xs_slot = prog_unit_kt(batch) * 8 * 8 * 4;
    red = xs + 2 * xs_slot;  // warp partial sums [warp][64 rows][ncol]
    misc = red + kProgWarps * 64 * ncol * 4;
    const int gemv_end = misc + (kProgMaxBatch + kProgMaxBatch * kProgWarps) * 4;
    const int attn_end = work + kProgAttnBytes;
    bar = ((gemv_end > attn_end ? gemv_end : attn_end) + 15) & ~15;
    flag = bar + 2 * stages * 8;  // [0] abort flag, [1] grid-barrier verdict
    total = flag + 16;
  }
};

// The CTA's contiguous share of a GEMV phase's (group, K-tile) stages, cut into
// units that stay inside one group and one aligned run of kProgUnitKt K-tiles.
struct ProgUnits {
  long long s, s_end;
  int kt, ukt;
  __device__ ProgUnits(int groups, int k_tiles, int cta, int n_cta, int unit_kt) {
    const long long total = static_cast<long long>(groups) * k_tiles;
    s = total * cta / n_cta;
    s_end = total * (cta + 1) / n_cta;
    kt = k_tiles;
    ukt = unit_kt;
  }
  __device__ bool next(int& grp, int& ka, int& kb) {
    if (s >= s_end) return false;
    grp = static_cast<int>(s / kt);
    ka = static_cast<int>(s % kt);
    const int lim = min(kt, (ka / ukt + 1) * ukt);
    kb = static_cast<int>(min(static_cast<long long>(lim), ka + (s_end - s)));
    s += kb - ka;
    return true;
  }
};

__device__ __forceinline__ uint32_t ld_acquire_gpu(const unsigned int* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid barrier among the consumer warps of every CTA (the producers never wait
// on it).  Returns false when the launch is aborting.  The verdict is broadcast
// through its own shared word (written only by thread 0 before the closing
// barrier), so every consumer thread takes the same branch even if the
// producer raises the abort flag meanwhile.
__device__ __forceinline__ bool prog_grid_barrier(unsigned int* bar, unsigned int target, volatile int* abort_flag,
                                                  volatile int* verdict) {
  named_barrier(1, kProgConsumers);
  if (threadIdx.x == 0) {
    volatile unsigned int* abort_g = bar + 1;
    if (*abort_flag) {
      atomicExch(bar + 1, 1u);
    } else {
      __threadfence();
      atomicAdd(bar, 1u);
      const uint64_t t0 = globaltimer();
      while (ld_acquire_gpu(bar) < target) {
        if (*abort_g) {
          *abort_flag = 1;
          break;
        }
        if (globaltimer() - t0 > B2_WAIT_TIMEOUT_NS) {
          record_error(kDevTimeoutGrid);
          atomicExch(bar + 1, 1u);
          *abort_flag = 1;
          break;
        }
      }
      __threadfence();
    }
    *verdict = *abort_flag ? 0 : 1;
  }
  named_barrier(1, kProgConsumers);
  return *verdict != 0;
}

// Eight bf16 inputs of GEMV row b at k = K0 + 8c .. K0 + 8c + 7, from the phase's source.
__device__ __forceinline__ uint4 prog_x_vec(const ProgPhase& P, int b, int K0, int c, const float* inv_rms) {
  const int k = K0 + c * 8;
  switch (P.x_source) {
    case kXNorm: {
      // bf16(x * rsqrt(mean(x^2) + eps) * w)   (granite_rmsnorm.h:45-80)
      const float* xr = static_cast<const float*>(P.x) + static_cast<size_t>(b) * P.ldx + k;
      const float4 a0 = *reinterpret_cast<const float4*>(xr);
      const float4 a1 = *reinterpret_cast<const float4*>(xr + 4);
      const uint4 wv = *reinterpret_cast<const uint4*>(P.norm_w + k);
      const float r = inv_rms[b];
      auto nb = [&](float xv, float wf) { return xv * r * wf; };
      uint4 o;
      o.x = pack_bf16x2_rn(nb(a0.x, bf16lo_to_f32(wv.x)), nb(a0.y, bf16hi_to_f32(wv.x)));
      o.y = pack_bf16x2_rn(nb(a0.z, bf16lo_to_f32(wv.y)), nb(a0.w, bf16hi_to_f32(wv.y)));
      o.z = pack_bf16x2_rn(nb(a1.x, bf16lo_to_f32(wv.z)), nb(a1.y, bf16hi_to_f32(wv.z)));
      o.w = pack_bf16x2_rn(nb(a1.z, bf16lo_to_f32(wv.w)), nb(a1.w, bf16hi_to_f32(wv.w)));
      return o;
    }
    case kXSwiglu: {
      // h = silu(bf16 g) * bf16 u, both accumulators narrowed first (granite_mlp.py:172-181)
      const float* gp = static_cast<const float*>(P.x) + static_cast<size_t>(b) * P.ldx + k;
      const float* up = gp + P.half;
      const float4 g0 = *reinterpret_cast<const float4*>(gp);
      const float4 g1 = *reinterpret_cast<const float4*>(gp + 4);
      const float4 u0 = *reinterpret_cast<const float4*>(up);
      const float4 u1 = *reinterpret_cast<const float4*>(up + 4);
      const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      const float uv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float hv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float gb = __bfloat162float(__float2bfloat16_rn(gv[2 * i + e]));
          const float ub = __bfloat162float(__float2bfloat16_rn(uv[2 * i + e]));
          hv[e] = gb / (1.f + expf(-gb)) * ub;
        }
        o[i] = pack_bf16x2_rn(hv[0], hv[1]);
      }
      return make_uint4(o[0], o[1], o[2], o[3]);
    }
    case kXAttn: {
      // log-sum-exp merge of the attention splits of q head k/64, d = k%64 .. +7
      const int head = k >> 6, d0 = k & 63;
      const int grp = P.n_q_heads / P.n_kv_heads;
      const int kvh = head / grp, j = head - kvh * grp;
      const float* base = P.part +
                          ((static_cast<size_t>(b) * P.n_kv_heads + kvh) * P.n_splits * grp + j) * kPartStride;
      const size_t stride = static_cast<size_t>(grp) * kPartStride;
      // splits in groups of 8: all loads of a group are issued before any is used
      float M = -INFINITY;
      for (int s0 = 0; s0 < P.n_splits; s0 += 8) {
        float mv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mv[i] = s0 + i < P.n_splits ? base[(s0 + i) * stride + 64] : -INFINITY;
#pragma unroll
        for (int i = 0; i < 8; ++i) M = fmaxf(M, mv[i]);
      }
      float Lsum = 0.f, O[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int s0 = 0; s0 < P.n_splits; s0 += 4) {
        float2 ml[4];
        float4 ov[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float* ps = base + min(s0 + i, P.n_splits - 1) * stride;
          ml[i] = *reinterpret_cast<const float2*>(ps + 64);
          const float2 a = *reinterpret_cast<const float2*>(ps + d0), b2 = *reinterpret_cast<const float2*>(ps + d0 + 2);
          const float2 c = *reinterpret_cast<const float2*>(ps + d0 + 4), e = *reinterpret_cast<const float2*>(ps + d0 + 6);
          ov[i][0] = make_float4(a.x, a.y, b2.x, b2.y);
          ov[i][1] = make_float4(c.x, c.y, e.x, e.y);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          // a split past the sequence end (m = -inf), or past n_splits, adds 0
          const float f = (s0 + i >= P.n_splits || ml[i].x == -INFINITY) ? 0.f : exp2f(ml[i].x - M);
          Lsum += ml[i].y * f;
          O[0] += ov[i][0].x * f;
          O[1] += ov[i][0].y * f;
          O[2] += ov[i][0].z * f;
          O[3] += ov[i][0].w * f;
          O[4] += ov[i][1].x * f;
          O[5] += ov[i][1].y * f;
          O[6] += ov[i][1].z * f;
          O[7] += ov[i][1].w * f;
        }
      }
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = pack_bf16x2_rn(O[2 * i] / Lsum, O[2 * i + 1] / Lsum);
      return make_uint4(o[0], o[1], o[2], o[3]);
    }
    default:
      return *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(P.x) + static_cast<size_t>(b) * P.ldx +
                                             k);
  }
}

// ---------------------------------------------------------------- GEMV unit
// q4 nibbles -> exact bf16 codes.  r = [k_a byte j | k_a byte j+1 | k_b byte j |
// k_b byte j+1] after the PRMT; each byte holds rows 2i (low nibble) and 2i+1
// (high nibble).  n | 0x4300 is the bf16 128 + n; bf16 has 7 mantissa bits, so
// each nibble is shifted to bits 0-3 first; the exact subtract leaves n.
__device__ __forceinline__ void decode_q4_pair_bf16(uint32_t w1, uint32_t w2, uint32_t sel_lo, uint32_t sel_hi,
                                                    uint32_t (&a)[8]) {
  constexpr uint32_t kMagic = 0x43004300u;  // bf16x2 (128, 128)
  const uint32_t r0 = prmt(w1, w2, sel_lo);  // rows 0-3 at (k_a, k_b)
  const uint32_t r1 = prmt(w1, w2, sel_hi);  // rows 4-7
  a[0] = bf16x2_sub(lop3<kLutAndOr>(r0, 0x000F000Fu, kMagic), kMagic);
  a[1] = bf16x2_sub(lop3<kLutAndOr>(r0 >> 4, 0x000F000Fu, kMagic), kMagic);
  a[2] = bf16x2_sub(lop3<kLutAndOr>(r0 >> 8, 0x000F000Fu, kMagic), kMagic);
  a[3] = bf16x2_sub(lop3<kLutAndOr>(r0 >> 12, 0x000F000Fu, kMagic), kMagic);
  a[4] = bf16x2_sub(lop3<kLutAndOr>(r1, 0x000F000Fu, kMagic), kMagic);
  a[5] = bf16x2_sub(lop3<kLutAndOr>(r1 >> 4, 0x000F000Fu, kMagic), kMagic);
  a[6] = bf16x2_sub(lop3<kLutAndOr>(r1 >> 8, 0x000F000Fu, kMagic), kMagic);
  a[7] = bf16x2_sub(lop3<kLutAndOr>(r1 >> 12, 0x000F000Fu, kMagic), kMagic);
}

// Stage the unit's bf16 x slice into x slot `slot` and the fp32 sums of each
// 32-k block (for the m * sum(x) term).  Products code * x (4 x 8 significant
// bits) are exact in the fp32 tensor-core accumulate, so x needs no rescaling.
__device__ __forceinline__ void prog_stage_x(const ProgPhase& P, int batch, int ka, int kb, bool first_unit,
                                             int slot, uint8_t* smem, const ProgSmem& L) {
  const int x_stride = prog_x_stride(batch);
  const int ctid = threadIdx.x, warp = ctid >> 5, lane = ctid & 31;
  __nv_bfloat16* x_s = reinterpret_cast<__nv_bfloat16*>(smem + L.work + slot * L.xslot);
  float* xs_s = reinterpret_cast<float*>(smem + L.xs + slot * L.xs_slot);
  float* inv_rms = reinterpret_cast<float*>(smem + L.misc);
  const int nvec = (kb - ka) * 32;  // 16-byte vectors per row, a multiple of 32 (warp-uniform tests)
  const int K0 = ka * 256;

  if (P.x_source == kXNorm && first_unit) {
    // 1/rms of whole rows, once per phase (kept in misc): every thread sums a few
    // float4 of each row (one L2 round trip), warps reduce, then one thread per row
    float* wss = inv_rms + kProgMaxBatch;  // [batch][kProgWarps]
    const int K = P.k_tiles * 256;
    for (int b = 0; b < batch; ++b) {
      const float4* xr = reinterpret_cast<const float4*>(static_cast<const float*>(P.x) + static_cast<size_t>(b) * P.ldx);
      float ss = 0.f;
#pragma unroll 2
      for (int q = ctid; q < K / 4; q += kProgConsumers) {
        const float4 v = xr[q];
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) wss[b * kProgWarps + warp] = ss;
    }
    named_barrier(1, kProgConsumers);
    if (ctid < batch) {
      float ss = 0.f;
#pragma unroll
      for (int w = 0; w < kProgWarps; ++w) ss += wss[ctid * kProgWarps + w];
      inv_rms[ctid] = rsqrtf(ss / static_cast<float>(K) + P.eps);
    }
    named_barrier(1, kProgConsumers);
  }
  for (int e = ctid; e < batch * nvec; e += kProgConsumers) {  // nvec % 32 == 0: a warp stays in one row
    const int b = e / nvec, c = e - b * nvec;
    const uint4 v = prog_x_vec(P, b, K0, c, inv_rms);
    *reinterpret_cast<uint4*>(x_s + b * x_stride + c * 8) = v;
    float s8 = bf16lo_to_f32(v.x) + bf16hi_to_f32(v.x) + bf16lo_to_f32(v.y) + bf16hi_to_f32(v.y) +
               bf16lo_to_f32(v.z) + bf16hi_to_f32(v.z) + bf16lo_to_f32(v.w) + bf16hi_to_f32(v.w);
    s8 += __shfl_xor_sync(0xffffffffu, s8, 1);
    s8 += __shfl_xor_sync(0xffffffffu, s8, 2);
    if ((lane & 3) == 0) xs_s[(c >> 2) * 8 + b] = s8;
  }
  named_barrier(1, kProgConsumers);
}

__device__ __forceinline__ void prog_gemv_phase(const ProgParams& p, const ProgPhase& P, uint8_t* smem,
                                                const ProgSmem& L, uint64_t* bars, volatile int* abort_flag,
                                                uint32_t& seq, uint32_t& unit_seq) {
  const int ctid = threadIdx.x, warp = ctid >> 5, lane = ctid & 31;
  const int batch = p.batch, stages = p.stages;
  const int ncol = (batch + 1) & ~1;
  const int xw_stride = prog_x_stride(batch) / 2;
  float* red = reinterpret_cast<float*>(smem + L.red);

  // warps 0-7 = (row-block rb, 32-k blocks 2kp and 2kp+1); lane (g, t): tile g&3,
  // rows h*8.. of the row-block, k pairs {2t, 2t+1} and {2t+8, 2t+9} of each
  // 16-k MMA step.  Warps 8-11 only stage x.
  const int g = lane >> 2, t = lane & 3;
  const int tile = g & 3, h = g >> 2, odd = tile & 1;
  const int rb = warp & 1, kp = (warp >> 1) & 3;
  const bool mma_warp = warp < kNbWarps;
  const uint32_t sel_lo = odd ? 0x1054u : 0x5410u;
  const uint32_t sel_hi = odd ? 0x3276u : 0x7632u;
  const int off_first = odd ? 8 : 0, off_second = odd ? 0 : 8;

  ProgUnits it((P.n_tile_rows + 3) / 4, P.k_tiles, blockIdx.x, gridDim.x, prog_unit_kt(p.batch));
  int grp, ka, kb;
  bool first_unit = true;
  while (it.next(grp, ka, kb)) {
    const int slot = unit_seq & 1;
    ++unit_seq;
    prog_stage_x(P, batch, ka, kb, first_unit, slot, smem, L);
    first_unit = false;
    const uint32_t* x32 = reinterpret_cast<const uint32_t*>(smem + L.work + slot * L.xslot);
    const float* xs_s = reinterpret_cast<const float*>(smem + L.xs + slot * L.xs_slot);
    float tot[4][4];
#pragma unroll
    for (int s = 0; s < 4; ++s) tot[s][0] = tot[s][1] = tot[s][2] = tot[s][3] = 0.f;

    for (int kk = 0; kk < kb - ka && mma_warp; ++kk) {
      const uint32_t sq = seq + kk;
      const int rs = sq % stages;
      mbar_wait_bounded(smem_u32(&bars[rs]), (sq / stages) & 1, abort_flag, kDevTimeoutFull);
      const uint8_t* tl = smem + L.ring + rs * kProgStage + tile * kProgSlot;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int kblk = 2 * kp + j;
        float part[4][4];
#pragma unroll
        for (int s = 0; s < 4; ++s) part[s][0] = part[s][1] = part[s][2] = part[s][3] = 0.f;
#pragma unroll
        for (int st = 0; st < 2; ++st) {
          const int kl = kk * 256 + kblk * 32 + st * 16;
          const uint32_t* xr = x32 + g * xw_stride + kl / 2 + t;
          const uint32_t bx0 = g < batch ? xr[0] : 0u;
          const uint32_t bx1 = g < batch ? xr[4] : 0u;
          const uint8_t* nb = tl + 1024 + rb * 2048 + kblk * 256 + st * 128 + 16 * t + 4 * h;
          const uint32_t p1 = *reinterpret_cast<const uint32_t*>(nb + off_first);
          const uint32_t p2 = *reinterpret_cast<const uint32_t*>(nb + off_second);
          const uint32_t q1 = *reinterpret_cast<const uint32_t*>(nb + 64 + off_first);
          const uint32_t q2 = *reinterpret_cast<const uint32_t*>(nb + 64 + off_second);
          uint32_t aP[8], aQ[8];
          decode_q4_pair_bf16(p1, p2, sel_lo, sel_hi, aP);
          decode_q4_pair_bf16(q1, q2, sel_lo, sel_hi, aQ);
#pragma unroll
          for (int s = 0; s < 4; ++s)
            mma_bf16_m16n8k16(part[s][0], part[s][1], part[s][2], part[s][3], aP[2 * s], aP[2 * s + 1], aQ[2 * s],
                              aQ[2 * s + 1], bx0, bx1);
        }
        // tot += d*part + m*sum(x) for this 32-k block
        const uint8_t* meta = tl + (kblk * 32 + rb * 16 + h * 8) * 2;
        const uint4 dv = *reinterpret_cast<const uint4*>(meta);
        const uint4 mv = *reinterpret_cast<const uint4*>(meta + 512);
        const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
        const uint32_t mw[4] = {mv.x, mv.y, mv.z, mv.w};
        const float2 xsv = *reinterpret_cast<const float2*>(xs_s + (kk * 8 + kblk) * 8 + 2 * t);
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const float da = bf16lo_to_f32(dw[s]), db = bf16hi_to_f32(dw[s]);
          const float ma = bf16lo_to_f32(mw[s]), mb = bf16hi_to_f32(mw[s]);
          tot[s][0] = fmaf(da, part[s][0], fmaf(ma, xsv.x, tot[s][0]));
          tot[s][1] = fmaf(da, part[s][1], fmaf(ma, xsv.y, tot[s][1]));
          tot[s][2] = fmaf(db, part[s][2], fmaf(mb, xsv.x, tot[s][2]));
          tot[s][3] = fmaf(db, part[s][3], fmaf(mb, xsv.y, tot[s][3]));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars[stages + rs]));
    }
    seq += kb - ka;

    // park the warp's sums: red[warp][64 local rows = tile*16 + h*8 + r][ncol]
    if (mma_warp) {
      float* rw = red + warp * 64 * ncol;
      const int c0 = 2 * t;
      if (c0 < batch) {
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const int lr = tile * 16 + h * 8 + 2 * s;
          *reinterpret_cast<float2*>(rw + lr * ncol + c0) = make_float2(tot[s][0], tot[s][1]);
          *reinterpret_cast<float2*>(rw + (lr + 1) * ncol + c0) = make_float2(tot[s][2], tot[s][3]);
        }
      }
    }
    named_barrier(1, kProgConsumers);
    // CTA sum over the 8 warps holding each row, one coalesced fp32 reduction per output
    if (!*abort_flag) {
      for (int e = ctid; e < kGroupRows * batch; e += kProgConsumers) {
        const int row = e % kGroupRows, b = e / kGroupRows;
        const int rbr = (row >> 4) & 1, lr = (row >> 5) * 16 + (row & 15);
        float v = 0.f;
#pragma unroll
        for (int q = 0; q < kNbWarps / 2; ++q) v += red[(2 * q + rbr) * 64 * ncol + lr * ncol + b];
        if (grp * 4 + (row >> 5) < P.n_tile_rows)
          atomicAdd(P.y + static_cast<size_t>(b) * P.ldy + grp * kGroupRows + row, v);
      }
    }
  }
}

// ------------------------------------------------------- GEMV unit, batch 1
// At batch 1 seven of the MMA's eight N columns would be padding.  Here column
// j of the B operand carries x of 32-k block j of the K-tile (x in column j,
// zero elsewhere), so one m16n8 accumulator collects all eight per-block dot
// products of the K-tile and the d/m scale fold runs once per K-tile instead of
// once per block.  Codes enter the MMA as the bf16 value 128 + n (no subtract);
// the 128 * sum(x) this adds folds into the m term: y += d*D + (m - 128 d)*S.
// Warp w: row-block rb = w & 1, rows half sh = (w >> 1) & 1 (rows 0-3 or 4-7 of
// each lane's 8-row group), stage phase ph = w >> 2 (stages with seq % 3 == ph).
constexpr int kB1Phases = kProgWarps / 4;

__device__ __forceinline__ void prog_gemv_phase_b1(const ProgPhase& P, uint8_t* smem, const ProgSmem& L,
                                                   uint64_t* bars, volatile int* abort_flag, int stages,
                                                   uint32_t& seq, uint32_t& unit_seq) {
  const int ctid = threadIdx.x, warp = ctid >> 5, lane = ctid & 31;
  constexpr int ncol = 2;
  float* red = reinterpret_cast<float*>(smem + L.red);
  const int g = lane >> 2, t = lane & 3;
  const int tile = g & 3, h = g >> 2, odd = tile & 1;
  const int rb = warp & 1, sh = (warp >> 1) & 1, ph = warp >> 2;
  const uint32_t sel = sh ? (odd ? 0x3276u : 0x7632u) : (odd ? 0x1054u : 0x5410u);
  const int off_first = odd ? 8 : 0, off_second = odd ? 0 : 8;

  ProgUnits it((P.n_tile_rows + 3) / 4, P.k_tiles, blockIdx.x, gridDim.x, prog_unit_kt(1));
  int grp, ka, kb;
  bool first_unit = true;
  while (it.next(grp, ka, kb)) {
    const int slot = unit_seq & 1;
    ++unit_seq;
    prog_stage_x(P, 1, ka, kb, first_unit, slot, smem, L);
    first_unit = false;
    const uint32_t* x32 = reinterpret_cast<const uint32_t*>(smem + L.work + slot * L.xslot);
    const float* xs_s = reinterpret_cast<const float*>(smem + L.xs + slot * L.xs_slot);
    float tot[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    const uint32_t seq0 = seq;
    const int n_st = kb - ka;
    for (int kk = 0; kk < n_st; ++kk) {
      const uint32_t sq = seq0 + kk;
      if (static_cast<int>(sq % kB1Phases) != ph) continue;
      const int rs = sq % stages;
      mbar_wait_bounded(smem_u32(&bars[rs]), (sq / stages) & 1, abort_flag, kDevTimeoutFull);
      const uint8_t* tl = smem + L.ring + rs * kProgStage + tile * kProgSlot;
      // x of block g (this lane's column) at k = g*32 + st*16 + {2t, 2t+8}
      uint32_t xw[2][2];
#pragma unroll
      for (int st = 0; st < 2; ++st) {
        const uint32_t* xr = x32 + (kk * 256 + g * 32 + st * 16) / 2 + t;
        xw[st][0] = xr[0];
        xw[st][1] = xr[4];
      }
      float acc[2][4];
#pragma unroll
      for (int s = 0; s < 2; ++s) acc[s][0] = acc[s][1] = acc[s][2] = acc[s][3] = 0.f;
#pragma unroll
      for (int kblk = 0; kblk < 8; ++kblk) {
        const bool mine = g == kblk;
#pragma unroll
        for (int st = 0; st < 2; ++st) {
          const uint8_t* nb = tl + 1024 + rb * 2048 + kblk * 256 + st * 128 + 16 * t + 4 * h;
          const uint32_t p1 = *reinterpret_cast<const uint32_t*>(nb + off_first);
          const uint32_t p2 = *reinterpret_cast<const uint32_t*>(nb + off_second);
          const uint32_t q1 = *reinterpret_cast<const uint32_t*>(nb + 64 + off_first);
          const uint32_t q2 = *reinterpret_cast<const uint32_t*>(nb + 64 + off_second);
          uint32_t aP[4], aQ[4];
          decode_q4_half_bf16(p1, p2, sel, aP);
          decode_q4_half_bf16(q1, q2, sel, aQ);
          const uint32_t b0 = mine ? xw[st][0] : 0u, b1 = mine ? xw[st][1] : 0u;
#pragma unroll
          for (int s = 0; s < 2; ++s)
            mma_bf16_m16n8k16(acc[s][0], acc[s][1], acc[s][2], acc[s][3], aP[2 * s], aP[2 * s + 1], aQ[2 * s],
                              aQ[2 * s + 1], b0, b1);
        }
      }
      // fold columns 2t, 2t+1 (blocks 2t + c): rows 4sh + 2s (c0, c1) and 4sh + 2s + 1 (c2, c3)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int kbl = 2 * t + c;
        const uint8_t* meta = tl + (kbl * 32 + rb * 16 + h * 8 + 4 * sh) * 2;
        const uint2 dv = *reinterpret_cast<const uint2*>(meta);
        const uint2 mv = *reinterpret_cast<const uint2*>(meta + 512);
        const float sx = xs_s[(kk * 8 + kbl) * 8];
        const uint32_t dw[2] = {dv.x, dv.y}, mw[2] = {mv.x, mv.y};
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          const float da = bf16lo_to_f32(dw[s]), db = bf16hi_to_f32(dw[s]);
          const float ma = fmaf(-128.f, da, bf16lo_to_f32(mw[s]));
          const float mb = fmaf(-128.f, db, bf16hi_to_f32(mw[s]));
          tot[s][0] = fmaf(da, acc[s][c], fmaf(ma, sx, tot[s][0]));
          tot[s][1] = fmaf(db, acc[s][2 + c], fmaf(mb, sx, tot[s][1]));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars[stages + rs]));
    }
    seq = seq0 + n_st;

    // sum the four t lanes (their block columns), park, then sum the stage phases
#pragma unroll
    for (int s = 0; s < 2; ++s)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        tot[s][e] += __shfl_xor_sync(0xffffffffu, tot[s][e], 1);
        tot[s][e] += __shfl_xor_sync(0xffffffffu, tot[s][e], 2);
      }
    if (t == 0) {
      float* rw = red + warp * 64 * ncol;
#pragma unroll
      for (int s = 0; s < 2; ++s)
#pragma unroll
        for (int e = 0; e < 2; ++e) rw[(tile * 16 + h * 8 + 4 * sh + 2 * s + e) * ncol] = tot[s][e];
    }
    named_barrier(1, kProgConsumers);
    if (!*abort_flag && ctid < kGroupRows) {
      const int row = ctid;
      const int rbr = (row >> 4) & 1, lr = (row >> 5) * 16 + (row & 15), shr = (row >> 2) & 1;
      float v = 0.f;
#pragma unroll
      for (int q = 0; q < kB1Phases; ++q) v += red[(rbr + 2 * shr + 4 * q) * 64 * ncol + lr * ncol];
      if (grp * 4 + (row >> 5) < P.n_tile_rows) atomicAdd(P.y + grp * kGroupRows + row, v);
    }
  }
}

// ----------------------------------------------------------- attention unit
// CTA unit (sequence b, kv head, split): 8 warps over the split's positions,
// merged in shared memory, partial (o, m, l) per q head to P.part.  The inner
// loop is that of gqa_decode_kernel (mma.sync bf16, log2-domain online softmax,
// P split hi + lo); RoPE uses the launch's cos/sin table.
__device__ __forceinline__ void prog_attention_phase(const ProgParams& p, const ProgPhase& P, uint8_t* work) {
  constexpr int D = 64;
  uint32_t* q_s = reinterpret_cast<uint32_t*>(work);
  float* wm = reinterpret_cast<float*>(work + 16 * kAttnQW * 4);
  float* wl = wm + kProgWarps * 16;
  float* wo = wl + kProgWarps * 16;  // [warp][8 head rows][D + 1]
  const int ctid = threadIdx.x, warp = ctid >> 5, lane = ctid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int hq = P.n_q_heads, hkv = P.n_kv_heads, grp = hq / hkv;
  const int units = p.batch * hkv * P.n_splits;
  named_barrier(1, kProgConsumers);  // the work area may still hold a GEMV unit's x being read

  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    const int split = u % P.n_splits;
    const int kvh = (u / P.n_splits) % hkv;
    const int b = u / (P.n_splits * hkv);
    const int pos = p.pos[b];
    // a position outside the cache makes the unit empty (no keys, no append), as a split
    // past pos is: every barrier of the launch is still reached
    const bool bad_pos = pos < 0 || pos >= P.ctx_max;
    if (bad_pos && split == 0 && kvh == 0 && ctid == 0) record_error(5);
    const int len = bad_pos ? 0 : pos + 1;
    const int lo = split * P.split_len;
    const int hi = min(len, lo + P.split_len);
    const float* rope = p.rope + b * 64;
    auto rot = [&](const float* src, __nv_bfloat16* dst, int i) {
      const float c = rope[2 * i], s = rope[2 * i + 1];
      const float x0 = src[i], x1 = src[i + D / 2];
      dst[i] = __float2bfloat16_rn(x0 * c - x1 * s);
      dst[i + D / 2] = __float2bfloat16_rn(x1 * c + x0 * s);
    };

    __nv_bfloat16* qh = reinterpret_cast<__nv_bfloat16*>(q_s);
    for (int e = ctid; e < 16 * kAttnQW * 2; e += kProgConsumers) qh[e] = __float2bfloat16_rn(0.f);
    named_barrier(1, kProgConsumers);
    const float* qrow = P.qkv + static_cast<size_t>(b) * P.ld_qkv;
    for (int e = ctid; e < grp * (D / 2); e += kProgConsumers) {
      const int j = e / (D / 2), i = e % (D / 2);
      rot(qrow + (kvh * grp + j) * D, qh + j * kAttnQW * 2, i);
    }
    if (!bad_pos && pos >= lo && pos < hi) {  // append the new token's k (rotated) and v
      const size_t row = ((static_cast<size_t>(b) * hkv + kvh) * P.ctx_max + pos) * D;
      const float* ks = qrow + hq * D + kvh * D;
      const float* vs = qrow + (hq + hkv) * D + kvh * D;
      if (ctid < D / 2) rot(ks, P.k_cache + row, ctid);
      if (ctid < D) P.v_cache[row + ctid] = __float2bfloat16_rn(vs[ctid]);
    }
    named_barrier(1, kProgConsumers);

    uint32_t qa[4][2];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      qa[j][0] = q_s[g * kAttnQW + 8 * t + 2 * j];
      qa[j][1] = q_s[g * kAttnQW + 8 * t + 2 * j + 1];
    }
    const int n = max(0, hi - lo);
    const int per_warp = ((n + kProgWarps * kAttnChunk - 1) / (kProgWarps * kAttnChunk)) * kAttnChunk;
    const int w_lo = lo + warp * per_warp;
    const int w_hi = min(hi, w_lo + per_warp);
    const __nv_bfloat16* kbase = P.k_cache + (static_cast<size_t>(b) * hkv + kvh) * P.ctx_max * D;
    const __nv_bfloat16* vbase = P.v_cache + (static_cast<size_t>(b) * hkv + kvh) * P.ctx_max * D;

    float m_run = -INFINITY, l_run = 0.f;
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

    auto load_chunk = [&](int c0, uint4 (&kr)[4], uint4 (&vr)[4]) {
      const int last = w_hi - 1;
      const int r0 = min(c0 + g, last), r1 = min(c0 + 8 + g, last);
      kr[0] = *reinterpret_cast<const uint4*>(kbase + static_cast<size_t>(r0) * D + 16 * t);
      kr[1] = *reinterpret_cast<const uint4*>(kbase + static_cast<size_t>(r0) * D + 16 * t + 8);
      kr[2] = *reinterpret_cast<const uint4*>(kbase + static_cast<size_t>(r1) * D + 16 * t);
      kr[3] = *reinterpret_cast<const uint4*>(kbase + static_cast<size_t>(r1) * D + 16 * t + 8);
      const int v0 = min(c0 + 2 * t, last), v1 = min(c0 + 2 * t + 1, last);
      const int v2 = min(c0 + 8 + 2 * t, last), v3 = min(c0 + 9 + 2 * t, last);
      vr[0] = *reinterpret_cast<const uint4*>(vbase + static_cast<size_t>(v0) * D + 8 * g);
      vr[1] = *reinterpret_cast<const uint4*>(vbase + static_cast<size_t>(v1) * D + 8 * g);
      vr[2] = *reinterpret_cast<const uint4*>(vbase + static_cast<size_t>(v2) * D + 8 * g);
      vr[3] = *reinterpret_cast<const uint4*>(vbase + static_cast<size_t>(v3) * D + 8 * g);
    };

    if (w_lo < w_hi) {
      // one chunk in flight per warp; 16 warps per SM keep enough loads outstanding
      for (int c0 = w_lo; c0 < w_hi; c0 += kAttnChunk) {
        uint4 kr[4], vr[4];
        load_chunk(c0, kr, vr);
        float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const uint32_t kw[8] = {kr[2 * nt].x,     kr[2 * nt].y,     kr[2 * nt].z,     kr[2 * nt].w,
                                  kr[2 * nt + 1].x, kr[2 * nt + 1].y, kr[2 * nt + 1].z, kr[2 * nt + 1].w};
#pragma unroll
          for (int j = 0; j < 4; ++j)
            mma_bf16_m16n8k16(s[nt][0], s[nt][1], s[nt][2], s[nt][3], qa[j][0], 0u, qa[j][1], 0u, kw[2 * j],
                              kw[2 * j + 1]);
        }
        float sc[4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int pp = c0 + 8 * nt + 2 * t + e;
            sc[2 * nt + e] = pp < w_hi ? s[nt][e] * P.scale_log2 : -INFINITY;
          }
        float mc = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
        mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, 1));
        mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, 2));
        const float m_new = fmaxf(m_run, mc);
        const float corr = exp2f(m_run - m_new);
        float pr[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) pr[e] = exp2f(sc[e] - m_new);
        l_run = l_run * corr + (pr[0] + pr[1] + pr[2] + pr[3]);
        m_run = m_new;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          o[i][0] *= corr;
          o[i][1] *= corr;
        }
        const uint32_t ph0 = pack_bf16x2(pr[0], pr[1]), ph1 = pack_bf16x2(pr[2], pr[3]);
        const uint32_t pl0 = pack_bf16x2(pr[0] - bf16lo_to_f32(ph0), pr[1] - bf16hi_to_f32(ph0));
        const uint32_t pl1 = pack_bf16x2(pr[2] - bf16lo_to_f32(ph1), pr[3] - bf16hi_to_f32(ph1));
        const uint32_t va[4] = {vr[0].x, vr[0].y, vr[0].z, vr[0].w}, vb[4] = {vr[1].x, vr[1].y, vr[1].z, vr[1].w};
        const uint32_t vc[4] = {vr[2].x, vr[2].y, vr[2].z, vr[2].w}, vd[4] = {vr[3].x, vr[3].y, vr[3].z, vr[3].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t sel = (i & 1) ? 0x7632u : 0x5410u;
          const uint32_t b0 = prmt(va[i >> 1], vb[i >> 1], sel);
          const uint32_t b1 = prmt(vc[i >> 1], vd[i >> 1], sel);
          mma_bf16_m16n8k16(o[i][0], o[i][1], o[i][2], o[i][3], ph0, 0u, ph1, 0u, b0, b1);
          mma_bf16_m16n8k16(o[i][0], o[i][1], o[i][2], o[i][3], pl0, 0u, pl1, 0u, b0, b1);
        }
      }
    }
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    if (t == 0) {
      wm[warp * 16 + g] = m_run;
      wl[warp * 16 + g] = l_run;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {  // head rows g (rows g + 8 are the zero padding of M)
      wo[(warp * 8 + g) * (D + 1) + 16 * t + i] = o[i][0];
      wo[(warp * 8 + g) * (D + 1) + 16 * t + 8 + i] = o[i][1];
    }
    named_barrier(1, kProgConsumers);
    for (int e = ctid; e < grp * D; e += kProgConsumers) {
      const int j = e / D, d = e % D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kProgWarps; ++w) M = fmaxf(M, wm[w * 16 + j]);
      float Ls = 0.f, O = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < kProgWarps; ++w) {
          const float mw = wm[w * 16 + j];
          const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
          Ls += wl[w * 16 + j] * f;
          O += wo[(w * 8 + j) * (D + 1) + d] * f;
        }
      }
      float* pr = P.part + (((static_cast<size_t>(b) * hkv + kvh) * P.n_splits + split) * grp + j) * kPartStride;
      pr[d] = O;
      if (d == 0) {
        pr[D] = M;
        pr[D + 1] = Ls;
      }
    }
    named_barrier(1, kProgConsumers);  // q_s / wo are rewritten by the next unit
  }
}

// RoPE cos/sin of each sequence's position, half-split pairs i = 0..31
// (granite_elementwise.py:135-138): fp64 angle, rounded to fp32 exactly as the
// one-shot attention kernel does.  One block of 32 threads per sequence.
__global__ void prog_rope_kernel(const int* pos, float theta, float* rope) {
  const int b = blockIdx.x, i = threadIdx.x;
  const double inv = pow(static_cast<double>(theta), -2.0 * i / 64);
  double sn, cs;
  sincos(static_cast<double>(pos[b]) * inv, &sn, &cs);
  rope[(b * 32 + i) * 2] = static_cast<float>(cs);
  rope[(b * 32 + i) * 2 + 1] = static_cast<float>(sn);
}

__global__ void __launch_bounds__(kProgThreads, 1) decode_program_kernel(const ProgParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const ProgSmem L(p.stages, p.batch);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.flag);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int stages = p.stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&bars[s]), 1);
      // empty: the 8 MMA warps per stage, or at batch 1 the four warps of the stage's phase
      mbar_init(smem_u32(&bars[stages + s]), p.batch == 1 ? 4 : kNbWarps);
    }
    abort_flag[0] = 0;
    abort_flag[1] = 1;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kProgWarps) {
    // ------------------------------------------------------------ producer
    const uint64_t policy = l2_evict_first_policy();
    uint32_t seq = 0, issued = 0;
    for (int ph = 0; ph < p.n_phases && !*abort_flag; ++ph) {
      const ProgPhase& P = p.phases[ph];
      if (P.kind != kPhGemv) continue;
      ProgUnits it((P.n_tile_rows + 3) / 4, P.k_tiles, blockIdx.x, gridDim.x, prog_unit_kt(p.batch));
      int grp, ka, kb;
      while (it.next(grp, ka, kb)) {
        for (int kt = ka; kt < kb; ++kt, ++seq) {
          if (lane == 0 && !*abort_flag) {
            const int slot = seq % stages;
            bool ok = true;
            if (seq >= static_cast<uint32_t>(stages))
              ok = mbar_wait_bounded(smem_u32(&bars[stages + slot]), ((seq / stages) & 1) ^ 1, abort_flag,
                                     kDevTimeoutEmpty);
            if (ok) {
              const uint8_t* src[4];
              uint32_t bytes = 0;
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int tr = grp * 4 + j;
                src[j] = tr < P.n_tile_rows ? P.w + (static_cast<size_t>(tr) * P.k_tiles + kt) * QTraits<kQ4>::kTile
                                            : nullptr;
                bytes += src[j] ? QTraits<kQ4>::kTile : 0;
              }
              const uint32_t full = smem_u32(&bars[slot]);
              mbar_arrive_expect_tx(full, bytes);
              const uint32_t dst = smem_u32(smem + L.ring + slot * kProgStage);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                if (src[j]) bulk_g2s(dst + j * kProgSlot, src[j], QTraits<kQ4>::kTile, full, policy);
              issued = seq + 1;
            }
          }
        }
        __syncwarp();
      }
    }
    if (lane == 0 && *abort_flag) {
      // let every copy this CTA issued land before the CTA exits
      const uint32_t first = issued > static_cast<uint32_t>(stages) ? issued - stages : 0;
      for (uint32_t s = first; s < issued; ++s) {
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
  const int ctid = threadIdx.x;
  uint32_t seq = 0, unit_seq = 0;
  unsigned int n_barriers = 0;
  for (int ph = 0; ph < p.n_phases; ++ph) {
    const ProgPhase& P = p.phases[ph];
    {
      // side tasks, spread over the whole grid
      const int gtid = blockIdx.x * kProgConsumers + ctid, gstride = gridDim.x * kProgConsumers;
      for (int i = gtid; i < P.zero0_n; i += gstride) P.zero0[i] = 0.f;
      for (int i = gtid; i < P.zero1_n; i += gstride) P.zero1[i] = 0.f;
      for (int i = gtid; i < P.copy_n; i += gstride) P.copy_dst[i] = P.copy_src[i];
    }
    if (P.kind == kPhPrep) {
      // side tasks only (the RoPE table comes from prog_rope_kernel, launched just before)
    } else if (P.kind == kPhAttn) {
      prog_attention_phase(p, P, smem + L.work);
    } else {
      if (p.batch == 1)
        prog_gemv_phase_b1(P, smem, L, bars, abort_flag, stages, seq, unit_seq);
      else
        prog_gemv_phase(p, P, smem, L, bars, abort_flag, seq, unit_seq);
    }
    if (P.barrier_after) {
      ++n_barriers;
      if (!prog_grid_barrier(p.barrier, n_barriers * gridDim.x, abort_flag, abort_flag + 1)) break;
    }
  }
}

}  // namespace b2
