// q4nx W4A16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), for
// decode batches where the GEMV becomes a dense contraction (16 < B <= 256).
//
//   y[b][n] = sum_k W[n][k] * x[b][k]        (or, fused, h = silu(bf16 g) * bf16 u)
//
// Operands (both fp16, as one tcgen05.mma kind::f16 requires):
//   A = weights, M = 128 rows of a CTA tile (4 q4nx tile-rows), dequantised in
//       shared memory by 8 warps: w = code*d + m in fp32, rounded once to fp16
//       (relative error <= 2^-11 per weight; codes and the block scales come
//       from the tiles exactly as stored, tools/q4nx.py:80-111).
//   B = x, N = batch rounded up to 16 (<= 256): staged by a pre-pass as fp16
//       x*2^e (e per token, exact power of two, undone in the epilogue) in the
//       exact byte image of the shared-memory operand (K-major, 128-byte
//       swizzle), so a plain 1-D bulk copy (cp.async.bulk, no multicast, no
//       tensor map) lands each 64-k slice ready for the tensor core.
//   D = fp32 in TMEM, 2 x N columns (double-buffered across row tiles).
//
// Warp roles (15 warps):
//   warp 0       producer: bulk copies of the raw tiles (one K-tile stage) and
//                of the x slices, mbarrier complete_tx
//   warp 1       TMEM allocation; lane 0 issues tcgen05.mma (4 per 64-k slice)
//                and tcgen05.commit to release the slices and publish D
//   warps 2-5    epilogue: tcgen05.ld 32x32b (warp w reads TMEM lanes
//                32*(w%4) ..), scale by 2^-e, store y / SwiGLU through smem
//   warps 6-13   dequant: four pairs, pair j converts 64-k slice j of every
//                K-tile (raw ring -> A ring slot j)
//   warp 14      packed form: lane 0 is the second MMA issuer (below); idle otherwise
// Every mbarrier wait is bounded; on a timeout the kernel records an error,
// stops issuing, waits (bounded) for the MMAs it issued, frees TMEM and exits.
//
// Packed form (TA): the same arithmetic from tiles repacked once per weight into a
// lane-per-row layout (tc_pack_kernel below).  The dequant warps then decode their
// own row with one conflict-free 16-byte load per 32 k and write A straight into
// tensor memory (tcgen05.st, 32x32b: TMEM lane = weight row); tcgen05.mma reads A
// from TMEM and only x from shared memory.  TMEM: columns 0-255 hold D (two
// buffers of up to 128 columns, or one of 256), columns 256-511 two K-tile A
// buffers of 128 columns (256 k as fp16 pairs).  Warp w (w % 4 = its TMEM lane
// quarter = tile-row slot q) decodes k 128*h .. 128*h + 127 of each K-tile, h = 0
// for warps 6-9 and 1 for warps 10-13.  A single issuing thread sustains one
// tcgen05.mma (M=128, K=16) per ~53 cycles whatever N <= 64, well below the tensor
// pipe's rate at small N; two issuers (warp 1 lane 0 and warp 14 lane 0) take the
// odd and even K-tiles of each item into two partial accumulators, which the
// epilogue adds (TMEM columns allowing: 2 x N <= 256).
#pragma once

#include "b2_common.cuh"
#include "q4nx_gemv.cuh"
#include "tp_exchange.cuh"

namespace b2 {

constexpr int kTcM = 128;
constexpr int kTcWarps = 15;
constexpr int kTcMma2Warp = 14;             // packed form: the second MMA issuer
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kTcEpiWarp0 = 2;
constexpr int kTcDqWarp0 = 6;
constexpr int kTcMaxASlots = 8;              // per 64-k slice of a K-tile: 1 or 2 (double-buffered)
constexpr int kTcASlotBytes = kTcM * 128;    // 128 rows x 64 fp16
constexpr int kTcRawSlot = QTraits<kQ4>::kSlot;
constexpr int kTcRawStage = 4 * kTcRawSlot;
constexpr int kTcMaxN = 256;
constexpr int kTcXchgStride = 33;            // SwiGLU exchange row stride in floats (bank spread)
constexpr int kTcXchgBytes = 64 * kTcXchgStride * 4 + 256 * 4;  // 64 rows x 32 tokens, then 2^-e per token
constexpr int kTcTmemACol = 256;             // packed form: first A column in TMEM with 2 A buffers
constexpr int kTcTmemABuf = 128;             // packed form: columns per A buffer (one K-tile)
// packed form: the a_bufs A buffers take the top a_bufs x 128 of the 512 TMEM columns (2:
// from column 256; 3, when the accumulators fit in 128 columns: from column 128)

// Packed weight: the tiles of a [n_tile_rows][k_tiles] weight reordered pair-major,
// tile (tr, kt) at position (tr/2)*2*k_tiles + kt*np + tr%2 (np = tiles in tr's pair,
// 2 or, for a last odd tile-row, 1), so that both tile-rows of a pair at one K-tile are
// one contiguous copy; inside each tile (5120 bytes, same size as a q4nx tile), for 32
// rows x 256 k:
//   bytes    0..1023  scales: entry s*32 + l = bf16 d | bf16 m << 16 of row l, 32-k block s
//   bytes 1024..5119  codes:  16 bytes at 1024 + (s*32 + l)*16 = row l, k 32s .. 32s+31 as
//                     four words w; nibble i of word w is k = 32s + 8w + 2i (i < 4) or
//                     32s + 8w + 2(i-4) + 1 (i >= 4), so (word >> 4p) & 0x000F000F holds
//                     the codes of k = 32s + 8w + 2p and k + 1.
// q8 packed tile (8704 bytes): bytes 0..511 the bf16 scale of row l, block s at
// (s*32 + l)*2; bytes 512..8703 row l's 32 int8 codes of block s (k = 32s + j at byte j)
// at 512 + (s*32 + l)*32.
__host__ __device__ constexpr int tc_packed_scale_off(int s, int l) { return (s * 32 + l) * 4; }
__host__ __device__ constexpr int tc_packed8_scale_off(int s, int l) { return (s * 32 + l) * 2; }
__host__ __device__ constexpr int tc_packed8_code_off(int s, int l) { return 512 + (s * 32 + l) * 32; }
__host__ __device__ inline long long tc_packed_tile(int tr, int kt, int n_tile_rows, int k_tiles) {
  const int pr = tr >> 1;
  const int np = (n_tile_rows - 2 * pr) >= 2 ? 2 : 1;
  return static_cast<long long>(pr) * 2 * k_tiles + static_cast<long long>(kt) * np + (tr & 1);
}
__host__ __device__ constexpr int tc_packed_code_off(int s, int l) { return 1024 + (s * 32 + l) * 16; }

enum TcEpi : int { kTcEpiF32 = 0, kTcEpiSwiglu = 1 };

struct TcParams {
  const uint8_t* w0;  // [n_tile_rows][k_tiles][5120]
  const uint8_t* w1;  // SwiGLU: up tiles (w0 = gate), else null
  int n_tile_rows;    // per source
  int k_tiles;
  const uint8_t* xsw;  // x image [k_tiles*4][npad][64] fp16, swizzled
  const int* xexp;     // [npad] exponents e (x' = x * 2^e)
  int batch, npad;
  int raw_stages, x_stages;
  int pre_raw;  // raw stages issued before the wait on the preceding kernel (<= raw_stages)
  int a_bufs;  // A slots per 64-k slice (1 or 2)
  void* y;     // fp32 [batch][ldy], or SwiGLU bf16 [batch][ldy]
  int ldy;
  int accumulate;
  int n_row_tiles;  // CTA tiles of 128 output rows (SwiGLU: 64 gate + 64 up rows)
  int n_splits;     // split-K: work item = (row tile, K range); partials added with fp32 reductions
  int kt_per_split;
  int n_nsplit;     // token columns split over CTAs: item = (row tile, K range, column block)
  int ncta;         // token columns per CTA (npad / n_nsplit, a multiple of 16)
  int prefetch;     // the weights are constant: the first raw stages stream (and are
                    // dequantised) before the wait on the preceding kernel
  int d_bufs;       // accumulator buffers in TMEM (2, or 1 for 256 columns in the packed form)
  int n_issuers;    // packed form: MMA issuing threads (1 or 2), each with its own partial
  void* const* seam_peers;  // non-null: advance pulled seam `seam` of rank `seam_rank` (its pre-pass consumed it)
  int seam, seam_rank, seam_world;
};

struct TcSmem {
  int a, x, raw, xchg, bar, total;
  // x_slices: 64-k slices per x stage (1; packed form 4, a whole K-tile)
  __host__ __device__ TcSmem(int npad, int raw_stages, int x_stages, int a_bufs, int x_slices = 1,
                             int raw_stage_bytes = kTcRawStage) {
    a = 0;  // 1024-aligned base (the kernel aligns the dynamic smem pointer)
    x = a + 4 * a_bufs * kTcASlotBytes;
    raw = x + x_stages * x_slices * npad * 128;
    xchg = raw + raw_stages * raw_stage_bytes;
    bar = (xchg + kTcXchgBytes + 15) & ~15;
    // raw full/empty, a full/empty, x full/empty, acc full/empty x2, done, tmem addr
    total = bar + (2 * raw_stages + 2 * kTcMaxASlots + 2 * x_stages + 4 + 2) * 8 + 16;
  }
};

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, fp16 x fp16 -> fp32
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T, fp16 x fp16 -> fp32 (A: M lanes x 16 k as 8 columns)
__device__ __forceinline__ void tc_mma_f16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 16 consecutive columns of this thread's TMEM lane (32x32b shape: lane = thread of the warp)
__device__ __forceinline__ void tmem_st32x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// arrive on `bar` once every MMA this thread issued so far has completed
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms of
// 1024 B (stride between atoms = 1024 B), start 16-byte aligned.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}
// Instruction descriptor, kind::f16: D fp32, A and B fp16, both K-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int m, int n) {
  return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// Byte offset of element (row, k) of a [rows][64] fp16 operand slice in the
// K-major 128-byte-swizzle layout: 16-byte chunk c of row r sits at chunk c ^ (r % 8).
__host__ __device__ __forceinline__ uint32_t sw128_offset(int row, int k) {
  return static_cast<uint32_t>((row >> 3) * 1024 + (row & 7) * 128 + ((((k >> 3) ^ row) & 7) << 4) + (k & 7) * 2);
}

// ------------------------------------------------------------ x pre-pass
// One CTA per token row n < npad: e = exponent putting max|x| in [2^14, 2^15),
// x' = fp16(x * 2^e) written into the swizzled slice image; rows >= batch are 0.
// With xf (fused RMSNorm) the row is bf16(xf * rsqrt(mean(xf^2) + eps) * norm_w), the
// arithmetic of granite_rms_norm (designs/granite_gemv/granite_rmsnorm.h:45-80), from the
// fp32 row xf [batch][ldx] instead of x.  With gu (SwiGLU input) the row is
// bf16(silu(bf16 g) * bf16 u) of the fp32 gate/up projections g = gu[n][k] and
// u = gu[n][gu_half + k]: the SwiGLU epilogue's arithmetic (granite_mlp.py:172-181), here
// run on the outputs of a plain split-K gate+up GEMM.
struct TcPrep {
  const __nv_bfloat16* x;
  const float* xf;
  const float* gu;
  int gu_half;
  const __nv_bfloat16* norm_w;
  float eps;
  int ldx, batch, k, npad;
  uint8_t* xsw;
  int* xexp;
  float* yzero;
  int ldy, n_out;
  int early;  // release the GEMM before this pass's own wait (see the kernel)
  // pulled seam (tensor-parallel decode; with xf only): before the norm, the fp32 row
  // becomes xf + sum over ranks r (in rank order) of r's partial at byte `part_off` of
  // its peer region ([batch][ld_part] fp32) and is written back to xf_out (= xf)
  void* const* peers;  // null: no seam
  int world, rank, seam, ld_part;
  long long part_off;
  float* xf_out;
  unsigned long long timeout_ns;
  int stage;  // stage every rank's row in dynamic shared memory (world * k floats), one round trip
};

// Rows of up to kPrepRegChunks * 256 chunks of 8 (K <= 16384) are read from global
// memory once into registers; longer rows take three passes over it.
constexpr int kPrepRegChunks = 8;

__global__ void __launch_bounds__(256) tc_x_prep_kernel(const TcPrep a) {
  __shared__ float wred[8];
  extern __shared__ __align__(16) float4 seam_rows[];  // [world][k / 4] when a.stage
  const int n = blockIdx.x;
  const int k = a.k;
  const int nc = k / 8;  // chunks of 8 values
  // early: the GEMM's CTAs may start (set up, prefetch and dequantise weights) while
  // this runs, they read the x image only after this grid completed.  Not after a
  // kernel whose CTAs still wait for SMs: the GEMM's (over half an SM's shared memory
  // each) would hold SMs that kernel needs.
  if (a.early) pdl_launch_dependents();
  pdl_wait();
  if (!a.early) pdl_launch_dependents();
  const bool live = n < a.batch;
  if (a.peers) {
    // this rank's partial is final (its producer grid completed before our wait): post
    // it, then wait until every rank's has landed
    if (blockIdx.x == 0) tp_seam_post(a.peers, a.world, a.rank, a.seam);
    tp_seam_wait(a.peers, a.world, a.rank, a.seam, a.timeout_ns);
    if (a.stage && live) {
      // every rank's row in flight at once (one NVLink round trip, not one per rank)
      const int k4 = k / 4;
      for (int q = 0; q < a.world; ++q) {
        const float* pr = reinterpret_cast<const float*>(static_cast<const uint8_t*>(a.peers[q]) + a.part_off) +
                          static_cast<size_t>(n) * a.ld_part;
        for (int u = threadIdx.x; u < k4; u += blockDim.x) cp_async16(smem_u32(&seam_rows[q * k4 + u]), pr + u * 4);
      }
      cp_async_commit();
      cp_async_wait<0>();
    }
    __syncthreads();
  }
  // chunk c (8 values) of the seam's sum over ranks, in rank order
  auto seam_sum = [&](int c, float4& s0, float4& s1) {
    const size_t e = static_cast<size_t>(n) * a.ld_part + c * 8;
    for (int q = 0; q < a.world; ++q) {
      float4 t0, t1;
      if (a.stage) {
        t0 = seam_rows[q * (k / 4) + 2 * c];
        t1 = seam_rows[q * (k / 4) + 2 * c + 1];
      } else {
        const float* pr = reinterpret_cast<const float*>(static_cast<const uint8_t*>(a.peers[q]) + a.part_off) + e;
        t0 = *reinterpret_cast<const float4*>(pr);
        t1 = *reinterpret_cast<const float4*>(pr + 4);
      }
      if (q == 0) {
        s0 = t0;
        s1 = t1;
      } else {
        s0.x += t0.x; s0.y += t0.y; s0.z += t0.z; s0.w += t0.w;
        s1.x += t1.x; s1.y += t1.y; s1.z += t1.z; s1.w += t1.w;
      }
    }
  };
  auto block_sum = [&](float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) wred[threadIdx.x >> 5] = v;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += wred[i];
    __syncthreads();  // wred is reused
    return tot;
  };
  auto block_max = [&](float v) {
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0) wred[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, wred[i]);
    return m;
  };
  // x' = fp16(x * 2^e) of one chunk, stored into the swizzled slice image
  auto store_chunk = [&](int c, uint4 v, float sc, bool zero) {
    uint4 o = make_uint4(0u, 0u, 0u, 0u);
    if (!zero) {
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint32_t h[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __half2 hv = __floats2half2_rn(bf16lo_to_f32(w[i]) * sc, bf16hi_to_f32(w[i]) * sc);
        h[i] = *reinterpret_cast<const uint32_t*>(&hv);
      }
      o = make_uint4(h[0], h[1], h[2], h[3]);
    }
    const int kc = (c * 8) >> 6, kin = (c * 8) & 63;
    *reinterpret_cast<uint4*>(a.xsw + static_cast<size_t>(kc) * a.npad * 128 + sw128_offset(n, kin)) = o;
  };
  // bf16(xf * inv * w) of one chunk (fused RMSNorm), with the chunk's 8 norm weights wv
  auto norm_chunk_w = [&](uint4 wv, float4 a0, float4 a1, float inv) {
    auto nb = [&](float xv, float wf) { return xv * inv * wf; };
    uint4 o;
    o.x = pack_bf16x2_rn(nb(a0.x, bf16lo_to_f32(wv.x)), nb(a0.y, bf16hi_to_f32(wv.x)));
    o.y = pack_bf16x2_rn(nb(a0.z, bf16lo_to_f32(wv.y)), nb(a0.w, bf16hi_to_f32(wv.y)));
    o.z = pack_bf16x2_rn(nb(a1.x, bf16lo_to_f32(wv.z)), nb(a1.y, bf16hi_to_f32(wv.z)));
    o.w = pack_bf16x2_rn(nb(a1.z, bf16lo_to_f32(wv.w)), nb(a1.w, bf16hi_to_f32(wv.w)));
    return o;
  };
  auto norm_chunk = [&](int c, float4 a0, float4 a1, float inv) {
    return norm_chunk_w(*reinterpret_cast<const uint4*>(a.norm_w + c * 8), a0, a1, inv);
  };
  // bf16(silu(bf16 g) * bf16 u) of one chunk (SwiGLU input), as the fused epilogue
  auto swiglu_chunk = [&](int c) {
    const float* gr = a.gu + static_cast<size_t>(n) * a.ldx + c * 8;
    const float4 g0 = *reinterpret_cast<const float4*>(gr), g1 = *reinterpret_cast<const float4*>(gr + 4);
    const float4 u0 = *reinterpret_cast<const float4*>(gr + a.gu_half);
    const float4 u1 = *reinterpret_cast<const float4*>(gr + a.gu_half + 4);
    auto h = [](float g, float u) {
      const float gb = __bfloat162float(__float2bfloat16_rn(g));
      const float ub = __bfloat162float(__float2bfloat16_rn(u));
      return __fdividef(gb, 1.f + __expf(-gb)) * ub;
    };
    uint4 o;
    o.x = pack_bf16x2_rn(h(g0.x, u0.x), h(g0.y, u0.y));
    o.y = pack_bf16x2_rn(h(g0.z, u0.z), h(g0.w, u0.w));
    o.z = pack_bf16x2_rn(h(g1.x, u1.x), h(g1.y, u1.y));
    o.w = pack_bf16x2_rn(h(g1.z, u1.z), h(g1.w, u1.w));
    return o;
  };
  auto finish_row = [&](float m) {  // exponent, and the zeroed output row for split-K
    const int e = live ? gemv_scale_exp(__float_as_uint(m)) : 0;
    if (threadIdx.x == 0) a.xexp[n] = e;
    if (a.yzero && live) {  // split-K partials are added into y: start it at zero
      float* yr = a.yzero + static_cast<size_t>(n) * a.ldy;
      if ((reinterpret_cast<uintptr_t>(yr) & 15) == 0)  // n_out is a multiple of 32
        for (int i = threadIdx.x; i < a.n_out / 4; i += blockDim.x)
          reinterpret_cast<float4*>(yr)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      else
        for (int i = threadIdx.x; i < a.n_out; i += blockDim.x) yr[i] = 0.f;
    }
    return pow2f(e);
  };

  if (nc <= kPrepRegChunks * 256) {
    // one read of the row: chunk c = threadIdx.x + 256 i lives in registers
    uint4 v[kPrepRegChunks];
#pragma unroll
    for (int i = 0; i < kPrepRegChunks; ++i) v[i] = make_uint4(0u, 0u, 0u, 0u);
    if (a.gu) {
#pragma unroll
      for (int i = 0; i < kPrepRegChunks; ++i) {
        const int c = threadIdx.x + 256 * i;
        if (live && c < nc) v[i] = swiglu_chunk(c);
      }
    } else if (a.xf) {
      float4 f[kPrepRegChunks][2];
      uint4 wv[kPrepRegChunks];  // the norm weights, loaded with the row (not after its reduction)
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < kPrepRegChunks; ++i) {
        const int c = threadIdx.x + 256 * i;
        if (live && c < nc) {
          const float* xr = a.xf + static_cast<size_t>(n) * a.ldx + c * 8;
          f[i][0] = *reinterpret_cast<const float4*>(xr);
          f[i][1] = *reinterpret_cast<const float4*>(xr + 4);
          wv[i] = *reinterpret_cast<const uint4*>(a.norm_w + c * 8);
        }
      }
      if (a.peers) {  // the residual plus the seam's sum, kept for the next seam
#pragma unroll
        for (int i = 0; i < kPrepRegChunks; ++i) {
          const int c = threadIdx.x + 256 * i;
          if (live && c < nc) {
            float4 s0, s1;
            seam_sum(c, s0, s1);
            f[i][0].x += s0.x; f[i][0].y += s0.y; f[i][0].z += s0.z; f[i][0].w += s0.w;
            f[i][1].x += s1.x; f[i][1].y += s1.y; f[i][1].z += s1.z; f[i][1].w += s1.w;
            float* xo = a.xf_out + static_cast<size_t>(n) * a.ldx + c * 8;
            *reinterpret_cast<float4*>(xo) = f[i][0];
            *reinterpret_cast<float4*>(xo + 4) = f[i][1];
          }
        }
      }
#pragma unroll
      for (int i = 0; i < kPrepRegChunks; ++i) {
        const int c = threadIdx.x + 256 * i;
        if (live && c < nc)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float4 q = f[i][h];
            ss = fmaf(q.x, q.x, fmaf(q.y, q.y, fmaf(q.z, q.z, fmaf(q.w, q.w, ss))));
          }
      }
      const float inv = rsqrtf(block_sum(ss) / static_cast<float>(k) + a.eps);
#pragma unroll
      for (int i = 0; i < kPrepRegChunks; ++i) {
        const int c = threadIdx.x + 256 * i;
        if (live && c < nc) v[i] = norm_chunk_w(wv[i], f[i][0], f[i][1], inv);
      }
    } else {
#pragma unroll
      for (int i = 0; i < kPrepRegChunks; ++i) {
        const int c = threadIdx.x + 256 * i;
        if (live && c < nc) v[i] = *reinterpret_cast<const uint4*>(a.x + static_cast<size_t>(n) * a.ldx + c * 8);
      }
    }
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < kPrepRegChunks; ++i) m = fmaxf(m, absmax8_bf16(v[i]));  // zero chunks add nothing
    const float sc = finish_row(block_max(m));
#pragma unroll
    for (int i = 0; i < kPrepRegChunks; ++i) {
      const int c = threadIdx.x + 256 * i;
      if (c < nc) store_chunk(c, v[i], sc, !live);
    }
    return;
  }

  // long rows: sum of squares, max and conversion as three passes over the row
  float inv = 0.f;
  if (live && a.xf) {
    const float4* xr = reinterpret_cast<const float4*>(a.xf + static_cast<size_t>(n) * a.ldx);
    float ss = 0.f;
    for (int c = threadIdx.x; c < k / 4; c += blockDim.x) {
      const float4 q = xr[c];
      ss = fmaf(q.x, q.x, fmaf(q.y, q.y, fmaf(q.z, q.z, fmaf(q.w, q.w, ss))));
    }
    inv = rsqrtf(block_sum(ss) / static_cast<float>(k) + a.eps);
  }
  auto row8 = [&](int c) -> uint4 {
    if (a.gu) return swiglu_chunk(c);
    if (!a.xf) return *reinterpret_cast<const uint4*>(a.x + static_cast<size_t>(n) * a.ldx + c * 8);
    const float* xr = a.xf + static_cast<size_t>(n) * a.ldx + c * 8;
    return norm_chunk(c, *reinterpret_cast<const float4*>(xr), *reinterpret_cast<const float4*>(xr + 4), inv);
  };
  float m = 0.f;
  if (live)
    for (int c = threadIdx.x; c < nc; c += blockDim.x) m = fmaxf(m, absmax8_bf16(row8(c)));
  const float sc = finish_row(block_max(m));
  for (int c = threadIdx.x; c < nc; c += blockDim.x) store_chunk(c, live ? row8(c) : make_uint4(0u, 0u, 0u, 0u), sc, !live);
}

// ------------------------------------------------------------ the GEMM
// QT: kQ4, or kQ8 (packed form, fp32 epilogue only)
template <int EPI, bool TA, int QT = kQ4>
__global__ void __launch_bounds__(kTcThreads, 1) q4_gemm_tc_kernel(const TcParams p) {
  constexpr int TILE = QTraits<QT>::kTile;
  constexpr int RAW_STAGE = TA ? 4 * TILE : kTcRawStage;  // packed: tiles back to back
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled operand slices
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const TcSmem L(p.ncta, p.raw_stages, p.x_stages, TA ? 0 : p.a_bufs, TA ? 4 : 1, RAW_STAGE);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar);
  const int RS = p.raw_stages, XS = p.x_stages;
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = raw_full + RS;
  uint64_t* a_full = raw_empty + RS;
  uint64_t* a_empty = a_full + kTcMaxASlots;
  uint64_t* x_full = a_empty + kTcMaxASlots;
  uint64_t* x_empty = x_full + XS;
  uint64_t* acc_full = x_empty + XS;  // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint64_t* mma_done = acc_empty + 2;  // [2]: one per MMA issuer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int npad = p.npad, ncta = p.ncta;
  const uint32_t ncols = ncta <= 32 ? 32u : (ncta <= 64 ? 64u : (ncta <= 128 ? 128u : 256u));  // per buffer
  const uint32_t tcols = TA ? 512u : 2 * ncols;  // TMEM columns allocated
  const int DB = p.d_bufs;                       // accumulator buffers (1 or 2)
  const int NI = TA ? p.n_issuers : 1;           // MMA issuers = partial accumulators per buffer
  const uint32_t dstride = NI * ncols;           // TMEM columns per accumulator buffer

  if (threadIdx.x == 0) {
    for (int s = 0; s < RS; ++s) {
      mbar_init(smem_u32(&raw_full[s]), 1);
      mbar_init(smem_u32(&raw_empty[s]), 8);  // the 8 dequant warps
    }
    for (int s = 0; s < kTcMaxASlots; ++s) {
      // the dequant pair of slice s % 4, buffer s / 4; packed form: all 8 dequant warps, buffer s
      mbar_init(smem_u32(&a_full[s]), TA ? 8 : 2);
      mbar_init(smem_u32(&a_empty[s]), 1);  // [0..1]: buffer free again (tcgen05.commit per K-tile)
    }
    for (int s = 0; s < XS; ++s) {
      mbar_init(smem_u32(&x_full[s]), 1);
      mbar_init(smem_u32(&x_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&acc_full[s]), NI);  // each MMA issuer's commit
      mbar_init(smem_u32(&acc_empty[s]), 4);  // the 4 epilogue warps
      mbar_init(smem_u32(&mma_done[s]), 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), tcols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();

  const int KT = p.k_tiles;
  const int n_items = p.n_row_tiles * p.n_splits * p.n_nsplit;  // -> (row tile, K-tile range, column block)
  const int AB = p.a_bufs;
  const uint32_t a_base = TA ? 512u - static_cast<uint32_t>(AB) * kTcTmemABuf : 0u;  // first A column
  auto item_tile = [&](int it) { return (it / p.n_nsplit) / p.n_splits; };
  auto item_k0 = [&](int it) { return ((it / p.n_nsplit) % p.n_splits) * p.kt_per_split; };
  auto item_n0 = [&](int it) { return (it % p.n_nsplit) * ncta; };
  auto item_k1 = [&](int it) { return min(KT, item_k0(it) + p.kt_per_split); };

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t policy = l2_evict_first_policy();  // weights stream once
      const uint64_t keep = l2_evict_last_policy();     // every CTA reads the same x slices
      // raw tiles of K-tile kt of row tile `tile` into raw stage rs (no dependency on x)
      auto issue_raw = [&](int tile, int kt, int rs) {
        const uint8_t* src[4];
        uint32_t bytes = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          int tr;
          const uint8_t* base;
          if (EPI == kTcEpiSwiglu) {
            tr = tile * 2 + (j & 1);
            base = j < 2 ? p.w0 : p.w1;
          } else {
            tr = tile * 4 + j;
            base = p.w0;
          }
          src[j] = tr < p.n_tile_rows ? base + (static_cast<size_t>(tr) * KT + kt) * TILE : nullptr;
          bytes += src[j] ? TILE : 0;
        }
        const uint32_t dst = smem_u32(smem + L.raw + rs * RAW_STAGE);
        if constexpr (TA) {
          // packed: slots 0-1 and 2-3 are each one tile-row pair, contiguous at this K-tile
          mbar_arrive_expect_tx(smem_u32(&raw_full[rs]), bytes);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint8_t* b = EPI == kTcEpiSwiglu ? (h ? p.w1 : p.w0) : p.w0;
            const int tr0 = EPI == kTcEpiSwiglu ? tile * 2 : tile * 4 + 2 * h;
            if (tr0 >= p.n_tile_rows) continue;
            const int np = p.n_tile_rows - tr0 >= 2 ? 2 : 1;
            bulk_g2s(dst + 2 * h * TILE, b + tc_packed_tile(tr0, kt, p.n_tile_rows, KT) * TILE, np * TILE,
                     smem_u32(&raw_full[rs]), policy);
          }
        } else {
          mbar_arrive_expect_tx(smem_u32(&raw_full[rs]), bytes);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (src[j]) bulk_g2s(dst + j * kTcRawSlot, src[j], TILE, smem_u32(&raw_full[rs]), policy);
        }
      };
      // The raw ring (per K-tile) and the x ring (per 64-k slice) advance independently:
      // each is refilled as soon as its consumers free a slot, so the raw prefetch runs
      // the full ring ahead of the MMAs instead of waiting behind x slots.  With prefetch
      // the first RS raw stages go out before the wait on the preceding kernel (the
      // dequant warps need nothing else), the x slices only after it.
      int it_r = blockIdx.x, kt_r = it_r < n_items ? item_k0(it_r) : 0;  // raw cursor
      uint32_t r_next = 0, n_k = 0;
      for (int it = blockIdx.x; it < n_items; it += gridDim.x) n_k += static_cast<uint32_t>(item_k1(it) - item_k0(it));
      auto advance_r = [&]() {
        if (++kt_r == item_k1(it_r)) {
          it_r += gridDim.x;
          if (it_r < n_items) kt_r = item_k0(it_r);
        }
        ++r_next;
      };
      if (p.prefetch)
        while (r_next < n_k && r_next < static_cast<uint32_t>(p.pre_raw)) {
          issue_raw(item_tile(it_r), kt_r, static_cast<int>(r_next));
          advance_r();
        }
      pdl_wait();  // x image comes from the pre-pass
      if (p.seam_peers && blockIdx.x == 0) tp_seam_advance(p.seam_peers, p.seam_world, p.seam_rank, p.seam);
      int it_x = blockIdx.x, kt_x = it_x < n_items ? item_k0(it_x) : 0, js_x = 0;  // x cursor
      uint32_t x_next = 0;
      // stages: one 64-k slice, or (packed form) the four slices of a K-tile
      const uint32_t n_x = TA ? n_k : 4 * n_k;
      const uint32_t xbytes = static_cast<uint32_t>(ncta) * 128;
      const uint32_t xstage = TA ? 4 * xbytes : xbytes;
      uint64_t t_prog = globaltimer();
      while ((r_next < n_k || x_next < n_x) && !*abort_flag) {
        bool progressed = false;
        // one x stage, then one raw stage, per pass: the MMAs wait on x while the raw ring
        // already runs up to RS K-tiles ahead (prefetched before the wait), so x goes first
        if (x_next < n_x) {
          const int xs = static_cast<int>(x_next % XS);
          if (x_next < static_cast<uint32_t>(XS) || mbar_test_wait(smem_u32(&x_empty[xs]), ((x_next / XS) & 1) ^ 1)) {
            // this CTA's token rows n0.. of the slice: contiguous, and their swizzle
            // pattern is the slice's (n0 is a multiple of 8 rows)
            mbar_arrive_expect_tx(smem_u32(&x_full[xs]), xstage);
            if (TA && ncta == npad) {  // the K-tile's four slices are contiguous in the image
              bulk_g2s(smem_u32(smem + L.x + xs * xstage), p.xsw + static_cast<size_t>(kt_x) * 4 * npad * 128, xstage,
                       smem_u32(&x_full[xs]), keep);
            } else {
              const int nsl = TA ? 4 : 1;
              for (int j = 0; j < nsl; ++j)
                bulk_g2s(smem_u32(smem + L.x + xs * xstage + j * xbytes),
                         p.xsw + (static_cast<size_t>(kt_x * 4 + js_x + j) * npad + item_n0(it_x)) * 128, xbytes,
                         smem_u32(&x_full[xs]), keep);
            }
            if (TA) js_x = 3;  // a whole K-tile per stage
            if (++js_x == 4) {
              js_x = 0;
              if (++kt_x == item_k1(it_x)) {
                it_x += gridDim.x;
                if (it_x < n_items) kt_x = item_k0(it_x);
              }
            }
            ++x_next;
            progressed = true;
          }
        }
        if (r_next < n_k) {
          const int rs = static_cast<int>(r_next % RS);
          if (r_next < static_cast<uint32_t>(RS) || mbar_test_wait(smem_u32(&raw_empty[rs]), ((r_next / RS) & 1) ^ 1)) {
            issue_raw(item_tile(it_r), kt_r, rs);
            advance_r();
            progressed = true;
          }
        }
        if (progressed) {
          t_prog = globaltimer();
        } else if (globaltimer() - t_prog > B2_WAIT_TIMEOUT_NS) {
          *abort_flag = 1;
          record_error(kDevTimeoutEmpty);
        } else {
          __nanosleep(64);  // leave the issue slots to the dequant warps between probes
        }
      }
    }
  } else if (TA && (warp == 1 || warp == kTcMma2Warp)) {
    // --------------------------------------------- MMA, packed form (A in TMEM)
    // issuer e takes the K-tiles kt of each item with (kt - k0) % NI == e into partial e;
    // A buffer and x stage follow the CTA's K-tile sequence rseq (shared with the
    // producer and the dequant warps)
    const int e = warp == 1 ? 0 : 1;
    if (lane == 0 && e < NI) {
      pdl_wait();
      const uint32_t idesc = umma_idesc_f16(kTcM, ncta);
      const uint32_t x0 = smem_u32(smem + L.x);
      const uint32_t xbytes = static_cast<uint32_t>(ncta) * 128;
      bool issued_any = false;
      uint32_t rseq = 0, t_it = 0;
      int ab_c = 0;          // A buffer of K-tile rseq
      uint32_t aph_c = 0u;   // its phase
      for (int it = blockIdx.x; it < n_items && !*abort_flag; it += gridDim.x, ++t_it) {
        const int buf = DB == 2 ? static_cast<int>(t_it & 1) : 0;
        const uint32_t uses = DB == 2 ? t_it >> 1 : t_it;  // earlier items on this buffer
        if (t_it >= static_cast<uint32_t>(DB))
          mbar_wait_bounded(smem_u32(&acc_empty[buf]), (uses & 1) ^ 1, abort_flag, kDevTimeoutEmpty);
        const uint32_t d_tmem = tmem_base + buf * dstride + e * ncols;
        const int k0 = item_k0(it), k1 = item_k1(it);
        uint32_t acc = 0;  // the partial's first MMA of the item starts it
        for (int kt = k0; kt < k1; ++kt, ++rseq) {
          // A buffer rseq % AB and its phase, kept by increments (no division here)
          const int ab = ab_c;
          const uint32_t aph = aph_c;
          if (++ab_c == AB) {
            ab_c = 0;
            aph_c ^= 1u;
          }
          if ((kt - k0) % NI != e) continue;
          const int xs = static_cast<int>(rseq % XS);
          const uint32_t xph = (rseq / XS) & 1;
          // a failed wait has set the abort flag, checked below
          if (!mbar_wait_bounded(smem_u32(&a_full[ab]), aph, abort_flag, kDevTimeoutFull) ||
              !mbar_wait_bounded(smem_u32(&x_full[xs]), xph, abort_flag, kDevTimeoutFull))
            break;
          tc_fence_after();
          const uint32_t a_tmem = tmem_base + a_base + ab * kTcTmemABuf;
#pragma unroll
          for (int js = 0; js < 4; ++js) {
            const uint64_t bd = umma_desc_sw128(x0 + (4 * xs + js) * xbytes);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {  // 16 k = 8 TMEM columns of A; +32 bytes along K of x
              tc_mma_f16_ta(d_tmem, a_tmem + js * 32 + kk * 8, bd + 2 * kk, idesc, acc);
              acc = 1;
            }
          }
          issued_any = true;
          tc_commit(smem_u32(&x_empty[xs]));
          tc_commit(smem_u32(&a_empty[ab]));
        }
        if (*abort_flag) break;
        tc_commit(smem_u32(&acc_full[buf]));
      }
      // every MMA issued here has completed before TMEM is released
      if (issued_any) {
        tc_commit(smem_u32(&mma_done[e]));
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(smem_u32(&mma_done[e]), 0)) {
          if (globaltimer() - t0 > B2_WAIT_TIMEOUT_NS) {
            record_error(kDevTimeoutDrain);
            break;
          }
        }
      }
    }
  } else if (warp == kTcMma2Warp) {
    // shared-memory form: no second issuer
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    if (lane == 0) {
      pdl_wait();
      const uint32_t idesc = umma_idesc_f16(kTcM, ncta);
      // ring positions advance by increments (no division in the issue loop: the
      // tensor pipe drains if the issuing thread spends ~100 cycles between MMAs)
      int ab = 0, xs = 0;
      uint32_t aph = 0, xph = 0, t_it = 0;
      const uint32_t a0 = smem_u32(smem + L.a), x0 = smem_u32(smem + L.x);
      const uint32_t xbytes = static_cast<uint32_t>(ncta) * 128;
      bool issued_any = false;
      for (int it = blockIdx.x; it < n_items && !*abort_flag; it += gridDim.x, ++t_it) {
        const int buf = DB == 2 ? static_cast<int>(t_it & 1) : 0;
        const uint32_t uses = DB == 2 ? t_it >> 1 : t_it;  // earlier items on this buffer
        if (t_it >= static_cast<uint32_t>(DB))
          mbar_wait_bounded(smem_u32(&acc_empty[buf]), (uses & 1) ^ 1, abort_flag, kDevTimeoutEmpty);
        const uint32_t d_tmem = tmem_base + buf * ncols;
        const int k0 = item_k0(it), k1 = item_k1(it);
        for (int kt = k0; kt < k1; ++kt) {
          for (int js = 0; js < 4; ++js) {
            const bool ok_a = mbar_wait_bounded(smem_u32(&a_full[4 * ab + js]), aph, abort_flag, kDevTimeoutFull);
            const bool ok_x = mbar_wait_bounded(smem_u32(&x_full[xs]), xph, abort_flag, kDevTimeoutFull);
            if (!ok_a || !ok_x) break;
            tc_fence_after();
            const uint64_t ad = umma_desc_sw128(a0 + (4 * ab + js) * kTcASlotBytes);
            const uint64_t bd = umma_desc_sw128(x0 + xs * xbytes);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)  // +32 bytes along K = +2 in the descriptor's address field
              tc_mma_f16(d_tmem, ad + 2 * kk, bd + 2 * kk, idesc, ((kt - k0) | js | kk) != 0);
            issued_any = true;
            tc_commit(smem_u32(&x_empty[xs]));
            if (++xs == XS) {
              xs = 0;
              xph ^= 1;
            }
          }
          if (*abort_flag) break;
          tc_commit(smem_u32(&a_empty[ab]));
          if (++ab == AB) {
            ab = 0;
            aph ^= 1;
          }
        }
        if (*abort_flag) break;
        tc_commit(smem_u32(&acc_full[buf]));
      }
      // every MMA issued here has completed before TMEM is released
      if (issued_any) {
        tc_commit(smem_u32(&mma_done[0]));
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(smem_u32(&mma_done[0]), 0)) {
          if (globaltimer() - t0 > B2_WAIT_TIMEOUT_NS) {
            record_error(kDevTimeoutDrain);
            break;
          }
        }
      }
    }
  } else if (warp < kTcDqWarp0) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may read
    const int row_local = q * 32 + lane;
    float* xchg = reinterpret_cast<float*>(smem + L.xchg);
    float* inv_sc = xchg + 64 * kTcXchgStride;  // [npad] 2^-e per token column
    pdl_wait();  // the exponents come from the pre-pass
    for (int i = threadIdx.x - 64; i < npad; i += 128) inv_sc[i] = pow2f(-p.xexp[i]);  // xexp has npad entries
    named_barrier(2, 128);
    uint32_t t_it = 0;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x, ++t_it) {
      const int tile = item_tile(it);
      const int n0 = item_n0(it);
      const int buf = DB == 2 ? static_cast<int>(t_it & 1) : 0;
      const uint32_t uses = DB == 2 ? t_it >> 1 : t_it;
      const bool ok = mbar_wait_bounded(smem_u32(&acc_full[buf]), uses & 1, abort_flag, kDevTimeoutFull);
      tc_fence_after();
      const uint32_t t_row = tmem_base + buf * dstride + (static_cast<uint32_t>(q * 32) << 16);
      const bool two = NI == 2 && item_k1(it) - item_k0(it) >= 2;  // partial 1 was written
      for (int c0 = n0; c0 < n0 + ncta; c0 += 32) {  // c0: global token column
        uint32_t r[32];
        tmem_ld32(t_row + (c0 - n0), r);
        if (two) {
          uint32_t r1[32];
          tmem_ld32(t_row + ncols + (c0 - n0), r1);
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) + __uint_as_float(r1[j]));
        }
        if (EPI == kTcEpiF32) {
          const int tr = tile * 4 + (row_local >> 5);
          const int grow = tile * kTcM + row_local;
          if (ok && !*abort_flag && tr < p.n_tile_rows) {
            float* y = static_cast<float*>(p.y) + grow;
#pragma unroll
            for (int hh = 0; hh < 32; hh += 16) {
              float u2v[16];  // the half's x scales (shared table)
#pragma unroll
              for (int j = 0; j < 16; ++j) u2v[j] = inv_sc[c0 + hh + j];
              if (p.n_splits > 1) {
#pragma unroll
                for (int j = 0; j < 16; ++j)  // zeroed by the pre-pass unless accumulating
                  if (c0 + hh + j < p.batch)
                    atomicAdd(y + static_cast<size_t>(c0 + hh + j) * p.ldy, __uint_as_float(r[hh + j]) * u2v[j]);
              } else {
                float old[16];  // the half's loads before its first store (no load waits behind a store)
#pragma unroll
                for (int j = 0; j < 16; ++j)
                  old[j] = (p.accumulate && c0 + hh + j < p.batch) ? y[static_cast<size_t>(c0 + hh + j) * p.ldy] : 0.f;
#pragma unroll
                for (int j = 0; j < 16; ++j)
                  if (c0 + hh + j < p.batch)
                    y[static_cast<size_t>(c0 + hh + j) * p.ldy] = old[j] + __uint_as_float(r[hh + j]) * u2v[j];
              }
            }
          }
        } else {
          // the 32 columns' x scales (shared table), read before any store below
          float u2v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) u2v[j] = inv_sc[c0 + j];
          // rows 0-63 gate, 64-127 the matching up rows.  Gate warps finish columns
          // 0-15 of the chunk and up warps columns 16-31: each hands the other half
          // of its values over (disjoint columns of the exchange rows).  Indices stay
          // compile-time (warp-uniform branches), all loads precede the stores.
          const bool gate_w = q < 2;
          const int orow = gate_w ? row_local : row_local - 64;  // output row 0..63
          float* xrow = xchg + orow * kTcXchgStride;
          if (gate_w) {
#pragma unroll
            for (int j = 0; j < 16; ++j) xrow[16 + j] = __uint_as_float(r[16 + j]);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) xrow[j] = __uint_as_float(r[j]);
          }
          named_barrier(2, 128);
          float hv[16];
          if (gate_w) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              // both accumulators narrowed to bf16 before SiLU (granite_mlp.py:172-181)
              const float gb = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[j]) * u2v[j]));
              const float ub = __bfloat162float(__float2bfloat16_rn(xrow[j] * u2v[j]));
              hv[j] = __fdividef(gb, 1.f + __expf(-gb)) * ub;  // error ~2^-21, far below bf16's
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float gb = __bfloat162float(__float2bfloat16_rn(xrow[16 + j] * u2v[16 + j]));
              const float ub = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[16 + j]) * u2v[16 + j]));
              hv[j] = __fdividef(gb, 1.f + __expf(-gb)) * ub;
            }
          }
          const int jm = gate_w ? 0 : 16;  // this warp's columns
          const int tr = tile * 2 + (orow >> 5);
          const int grow = tile * 64 + orow;
          if (ok && !*abort_flag && tr < p.n_tile_rows) {
            __nv_bfloat16* h = static_cast<__nv_bfloat16*>(p.y);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int n = c0 + jm + j;
              if (n < p.batch) h[static_cast<size_t>(n) * p.ldy + grow] = __float2bfloat16_rn(hv[j]);
            }
          }
          named_barrier(2, 128);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&acc_empty[buf]));
    }
  } else if constexpr (TA) {
    // ------------------------------------------------- dequant, packed form
    // warp w: TMEM lane quarter q = w % 4 = tile-row slot q of the raw stage, row = lane;
    // half hh of each K-tile: 32-k blocks 4 hh .. 4 hh + 3 (TMEM columns 64 hh ..)
    const int q = warp & 3;
    const int hh = (warp - kTcDqWarp0) >> 2;
    const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
    uint32_t rseq = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
      for (int kt = item_k0(it); kt < item_k1(it); ++kt, ++rseq) {
        const int rs = rseq % RS;
        const int abuf = static_cast<int>(rseq % AB);
        ok = ok && mbar_wait_bounded(smem_u32(&raw_full[rs]), (rseq / RS) & 1, abort_flag, kDevTimeoutFull);
        if (rseq >= static_cast<uint32_t>(AB))
          ok = ok && mbar_wait_bounded(smem_u32(&a_empty[abuf]), ((rseq / AB) & 1) ^ 1, abort_flag,
                                       kDevTimeoutEmpty);
        ok = __all_sync(0xffffffffu, ok);  // the TMEM stores below are warp-collective
        if (ok) {
          tc_fence_after();  // the MMAs that read this A buffer have completed
          const uint8_t* tl = smem + L.raw + rs * RAW_STAGE + q * TILE;
          const uint32_t a_col = tmem_base + t_lane + a_base + abuf * kTcTmemABuf;
#pragma unroll
          for (int sb = 0; sb < 4; ++sb) {
            const int s = 4 * hh + sb;  // 32-k block of the K-tile
            if constexpr (QT == kQ8) {
              // int8 code c: byte ^ 0x80 = c + 128 placed under 0x64 is fp16 1024 + c + 128,
              // less 1152 is c exactly; times the block scale, rounded once
              const float sv = __uint_as_float(static_cast<uint32_t>(
                                   *reinterpret_cast<const uint16_t*>(tl + tc_packed8_scale_off(s, lane))) << 16);
              const __half2 s2 = __floats2half2_rn(sv, sv);
              const uint4 c0 = *reinterpret_cast<const uint4*>(tl + tc_packed8_code_off(s, lane));
              const uint4 c1 = *reinterpret_cast<const uint4*>(tl + tc_packed8_code_off(s, lane) + 16);
              const uint32_t wv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
              uint32_t a[16];
#pragma unroll
              for (int w = 0; w < 8; ++w) {
                const uint32_t u = wv[w] ^ 0x80808080u;
#pragma unroll
                for (int hp = 0; hp < 2; ++hp) {  // bytes (0, 1) and (2, 3): k = 4w + 2hp, +1
                  const uint32_t h = prmt(u, 0x64646464u, hp ? 0x4342u : 0x4140u);
                  const uint32_t cc = f16x2_sub(h, 0x64806480u);
                  const __half2 wh = __hmul2(*reinterpret_cast<const __half2*>(&cc), s2);
                  a[2 * w + hp] = *reinterpret_cast<const uint32_t*>(&wh);
                }
              }
              tmem_st32x16(a_col + s * 16, a);
              continue;
            }
            const uint32_t sc = *reinterpret_cast<const uint32_t*>(tl + tc_packed_scale_off(s, lane));
            const uint4 nv = *reinterpret_cast<const uint4*>(tl + tc_packed_code_off(s, lane));
            const float dv = bf16lo_to_f32(sc), mv = bf16hi_to_f32(sc);
            const __half2 d2 = __floats2half2_rn(dv, dv), m2 = __floats2half2_rn(mv, mv);
            const uint32_t wv[4] = {nv.x, nv.y, nv.z, nv.w};
            uint32_t a[16];
#pragma unroll
            for (int w = 0; w < 4; ++w)
#pragma unroll
              for (int pp = 0; pp < 4; ++pp) {
                const uint32_t code = f16x2_sub(lop3<kLutAndOr>(wv[w] >> (4 * pp), 0x000F000Fu, 0x64006400u), 0x64006400u);
                const __half2 wh = __hfma2(*reinterpret_cast<const __half2*>(&code), d2, m2);
                a[4 * w + pp] = *reinterpret_cast<const uint32_t*>(&wh);
              }
            tmem_st32x16(a_col + s * 16, a);
          }
          tmem_wait_st();
          tc_fence_before();
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(smem_u32(&a_full[abuf]));
          mbar_arrive(smem_u32(&raw_empty[rs]));
        }
      }
    }
  } else {
    // ------------------------------------------------------------ dequant
    // pair js (warps 6+2js, 7+2js) converts slice js (k 64*js .. +63) of every K-tile.
    // thread: chunk c = 8 k (lane & 7), tile-row t and row-block rb (idx >> 3)
    const int idx = threadIdx.x - kTcDqWarp0 * 32;  // 0..255
    const int js = idx >> 6;
    const int pidx = idx & 63;
    const int c = pidx & 7, qq = pidx >> 3;
    const int t = qq >> 1, rb = qq & 1;
    const int row0 = t * 32 + rb * 16;          // first of this thread's 16 A rows
    const int kb = (js * 64 + c * 8) >> 5;      // this chunk's 32-k block
    uint32_t rseq = 0;  // K-tiles of this CTA so far (= the MMA thread's kseq)
    bool ok = true;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
      for (int kt = item_k0(it); kt < item_k1(it); ++kt, ++rseq) {
        const int rs = rseq % RS;
        const int abuf = static_cast<int>(rseq % AB);
        const int as = js + 4 * abuf;
        ok = ok && mbar_wait_bounded(smem_u32(&raw_full[rs]), (rseq / RS) & 1, abort_flag, kDevTimeoutFull);
        if (rseq >= static_cast<uint32_t>(AB))
          ok = ok && mbar_wait_bounded(smem_u32(&a_empty[abuf]), ((rseq / AB) & 1) ^ 1, abort_flag,
                                       kDevTimeoutEmpty);
        if (ok) {
          const uint8_t* tl = smem + L.raw + rs * RAW_STAGE + t * kTcRawSlot;
          // scales of the 16 rows at block kb: d, m bf16 -> fp16 pairs (d, d), (m, m)
          const uint4* dp = reinterpret_cast<const uint4*>(tl + (kb * 32 + rb * 16) * 2);
          const uint4 d0 = dp[0], d1 = dp[1], m0 = dp[32], m1 = dp[33];
          const uint32_t dw[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
          const uint32_t mw[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
          // nibbles of k = 64 js + 8 c + 2i (+1): 16 bytes = 16 rows at k, then at k + 1
          uint4 nv[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            nv[i] = *reinterpret_cast<const uint4*>(tl + 1024 + rb * 2048 + (js * 64 + c * 8 + 2 * i) * 8);
          uint8_t* a_slot = smem + L.a + as * kTcASlotBytes;
#pragma unroll
          for (int rp = 0; rp < 8; ++rp) {  // row pair (2 rp, 2 rp + 1) = byte rp of each 8-byte row group
            const float de = bf16lo_to_f32(dw[rp]), dodd = bf16hi_to_f32(dw[rp]);
            const float me = bf16lo_to_f32(mw[rp]), modd = bf16hi_to_f32(mw[rp]);
            const __half2 de2 = __floats2half2_rn(de, de), do2 = __floats2half2_rn(dodd, dodd);
            const __half2 me2 = __floats2half2_rn(me, me), mo2 = __floats2half2_rn(modd, modd);
            uint32_t ev[4], ov[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t wl = (rp < 4) ? nv[i].x : nv[i].y;  // k bytes 0-7
              const uint32_t wh = (rp < 4) ? nv[i].z : nv[i].w;  // k+1 bytes 8-15
              const uint32_t bsel = static_cast<uint32_t>(rp & 3);
              const uint32_t r2 = prmt(wl, wh, bsel | ((bsel + 4) << 8));  // k byte -> bits 0-7, k+1 byte -> 16-23
              const uint32_t lo = f16x2_sub(lop3<kLutAndOr>(r2, 0x000F000Fu, 0x64006400u), 0x64006400u);
              const uint32_t hi = f16x2_sub(lop3<kLutAndOr>(r2, 0x00F000F0u, 0x54005400u), 0x54005400u);
              const __half2 we = __hfma2(*reinterpret_cast<const __half2*>(&lo), de2, me2);
              const __half2 wo = __hfma2(*reinterpret_cast<const __half2*>(&hi), do2, mo2);
              ev[i] = *reinterpret_cast<const uint32_t*>(&we);
              ov[i] = *reinterpret_cast<const uint32_t*>(&wo);
            }
            const int re = row0 + 2 * rp;
            *reinterpret_cast<uint4*>(a_slot + sw128_offset(re, c * 8)) = make_uint4(ev[0], ev[1], ev[2], ev[3]);
            *reinterpret_cast<uint4*>(a_slot + sw128_offset(re + 1, c * 8)) = make_uint4(ov[0], ov[1], ov[2], ov[3]);
          }
        }
        fence_async_smem();  // generic-proxy stores -> visible to the tensor core
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(smem_u32(&a_full[as]));
          mbar_arrive(smem_u32(&raw_empty[rs]));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tcols);
  }
}

// ------------------------------------------------------------ packing
// q4nx weight -> packed weight (the layout above): one CTA of 256 threads per tile,
// thread (s, l) = (threadIdx.x / 32, threadIdx.x % 32) writes row l's 32-k block s.
// A pure byte permutation: every code, d and m keeps its bits.
__global__ void __launch_bounds__(256) tc_pack_kernel(const uint8_t* __restrict__ in, uint8_t* __restrict__ out,
                                                      int n_tile_rows, int k_tiles) {
  const int s = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int rb = l >> 4, r = l & 15;
  const long long n_tiles = static_cast<long long>(n_tile_rows) * k_tiles;
  for (long long t = blockIdx.x; t < n_tiles; t += gridDim.x) {
    const int tr = static_cast<int>(t / k_tiles), kt = static_cast<int>(t % k_tiles);
    const uint8_t* ti = in + t * QTraits<kQ4>::kTile;
    uint8_t* to = out + tc_packed_tile(tr, kt, n_tile_rows, k_tiles) * QTraits<kQ4>::kTile;
    const uint16_t* dm = reinterpret_cast<const uint16_t*>(ti);
    const uint32_t d = dm[s * 32 + l], m = dm[256 + s * 32 + l];  // entry (k/32)*32 + row
    *reinterpret_cast<uint32_t*>(to + tc_packed_scale_off(s, l)) = d | (m << 16);
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int j = 0; j < 32; ++j) {  // k = 32 s + j
      const int k = 32 * s + j;
      const int i = rb * 4096 + k * 16 + r;  // nibble index in the q4nx tile
      const uint32_t code = (ti[1024 + (i >> 1)] >> ((i & 1) * 4)) & 0xFu;
      const int wi = j >> 3, jj = j & 7;
      const int pos = (jj & 1) ? 4 + (jj >> 1) : (jj >> 1);
      w[wi] |= code << (4 * pos);
    }
    *reinterpret_cast<uint4*>(to + tc_packed_code_off(s, l)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}


// q8 weight -> packed q8 weight: thread (s, l) writes row l's scale and 32 codes of block s
__global__ void __launch_bounds__(256) tc_pack8_kernel(const uint8_t* __restrict__ in, uint8_t* __restrict__ out,
                                                       int n_tile_rows, int k_tiles) {
  constexpr int T8 = QTraits<kQ8>::kTile;
  const int s = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int rb = l >> 4, r = l & 15;
  const long long n_tiles = static_cast<long long>(n_tile_rows) * k_tiles;
  for (long long t = blockIdx.x; t < n_tiles; t += gridDim.x) {
    const int tr = static_cast<int>(t / k_tiles), kt = static_cast<int>(t % k_tiles);
    const uint8_t* ti = in + t * T8;
    uint8_t* to = out + tc_packed_tile(tr, kt, n_tile_rows, k_tiles) * T8;
    *reinterpret_cast<uint16_t*>(to + tc_packed8_scale_off(s, l)) =
        reinterpret_cast<const uint16_t*>(ti)[s * 32 + l];  // entry (k/32)*32 + row
    uint32_t w[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      uint32_t v = 0u;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int k = 32 * s + 4 * q + b;
        v |= static_cast<uint32_t>(ti[512 + rb * 4096 + k * 16 + r]) << (8 * b);  // code index rb*4096 + k*16 + r
      }
      w[q] = v;
    }
    *reinterpret_cast<uint4*>(to + tc_packed8_code_off(s, l)) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(to + tc_packed8_code_off(s, l) + 16) = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

}  // namespace b2
