// GQA decode attention (flash-decode) for sm_100a, with RoPE fused on the
// query/key load and the new token's K/V appended to the cache.
//
// Reference: designs/granite_gemv/granite_attention.h:80-213 (one q head
// against a streamed KV cache, online softmax in log2 units, final divide),
// oracle granite_attention.py:163-167; RoPE half-split granite_elementwise.h:40-75
// with the table of granite_elementwise.py:136-138; q/k rotated, v not
// (granite_qkv.py:176-207).
//
//   for each sequence b, kv head h, q head j of h's group (Hq/Hkv heads):
//     q  = bf16(rope(q_new[b][j], pos_b)),  k_pos = bf16(rope(k_new[b][h], pos_b)),
//     v_pos = bf16(v_new[b][h]);  cache[b][h][pos_b] = (k_pos, v_pos)
//     s[t] = scale * q . K[t],  t = 0..pos_b  (causal: the new token sees itself)
//     out  = sum_t softmax(s)[t] * V[t]                       (fp32 softmax)
//
// Layout: K, V caches bf16 [B][Hkv][ctx_max][D]; q/k/v of the new token fp32
// rows (the QKV GEMV output), row stride ld_new; out bf16 [B][Hq*D].
//
// Work split: CTA (split, kv head, sequence), 4 warps, each warp a contiguous
// run of positions in 16-position chunks.  The group's q heads are the 16 "M"
// rows of mma.sync m16n8k16 (bf16 in, fp32 out), so every K/V byte is loaded
// once for the whole group.  Per chunk: S = Q K^T (2 n-tiles x 4 k-steps), the
// online softmax on the accumulator fragments (scores pre-scaled by log2 e,
// exp2), P reused from the accumulator layout as the A operand of O += P V
// (8 n-tiles of d), P split as bf16 hi + lo so the product keeps ~2^-17 of P.
// K/V stream through a ring of shared-memory stages per warp, filled with
// 16-byte asynchronous copies (cp.async, coalesced rows) several chunks ahead of
// the math, so the loads in flight do not cost registers.  Warps merge in shared
// memory; splits merge in a cluster or in a second kernel from a caller-provided
// workspace (log-sum-exp).
#pragma once

#include "b2_common.cuh"

namespace b2 {

// Warps per CTA (template W): 8 when a launch has at most one CTA per SM, else 4.
constexpr int kAttnMaxWarps = 8;
constexpr int kAttnChunk = 16;  // positions per inner step

struct AttnParams {
  const float* q;      // [B][ld_new] rows, q head j at q + b*ld_new + j*D
  const float* k_new;  // kv head h at k_new + b*ld_new + h*D
  const float* v_new;
  int ld_new;
  __nv_bfloat16* k_cache;  // [B][Hkv][ctx_max][D]
  __nv_bfloat16* v_cache;
  const int* pos;  // [B] position of the new token; attention length = pos + 1
  int batch, hq, hkv, ctx_max;
  float theta;
  float scale_log2;  // scale * log2(e)
  __nv_bfloat16* out;  // [B][ldo], q head j at out + b*ldo + j*D
  int ldo;
  float* part;   // [B][Hkv][n_splits][grp][D + 2] partials (o, m, l) when n_splits > 1
  int n_splits;  // CTAs per (sequence, kv head)
  int split_len;  // positions per split (multiple of 16)
  int append;     // write the new token's k/v into the cache
  int rope;       // rotate the new q/k (0: use them as given)
  int out_f32;    // out is fp32 instead of bf16
  int clustered;  // splits of one (sequence, kv head) form a cluster and merge in rank 0's smem
  int prefetch_kv;  // pos[] and cache rows < pos are final at launch: load them before the PDL wait
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Half-split RoPE: the angle of pair (i, i + D/2) at pos, evaluated in fp64 and
// rounded to fp32 cos/sin.
template <int D>
__device__ __forceinline__ void rope_angle(int pos, float theta, int i, float& c, float& s) {
  const double inv = pow(static_cast<double>(theta), -2.0 * i / D);
  double sn, cs;
  sincos(static_cast<double>(pos) * inv, &sn, &cs);
  c = static_cast<float>(cs);
  s = static_cast<float>(sn);
}

// Rotation of one head's pair (i, i + D/2) (D fp32 values at src) by the angle
// (c, s) of pair i into bf16 dst; rope == 0 rounds without rotating.
template <int D>
__device__ __forceinline__ void rope_apply_bf16(const float* src, __nv_bfloat16* dst, int i, float c, float s,
                                                int rope) {
  const float x0 = src[i], x1 = src[i + D / 2];
  dst[i] = __float2bfloat16_rn(rope ? x0 * c - x1 * s : x0);
  dst[i + D / 2] = __float2bfloat16_rn(rope ? x1 * c + x0 * s : x1);
}


// K/V ring of one warp: kAttnStages(W) stages of one 16-position chunk, K rows then V
// rows (128 bytes each); 16-byte piece c of row r sits at piece c ^ (r % 8), so the
// fragment reads below (8 rows x 4 pieces, or 4 rows x 8 pieces per load) hit every
// bank once per wavefront.  Every warp has the same ring bytes: 2 stages at 8 warps,
// 4 at 4 warps (64 KB per CTA), the loads in flight per warp that a 4-warp CTA, three
// per SM, can keep deeper.
constexpr int kAttnStageBytes = 2 * kAttnChunk * 128;
__host__ __device__ constexpr int attn_stages(int w) { return w == 8 ? 2 : 4; }
__host__ __device__ constexpr int attn_ring_bytes(int w) { return w * attn_stages(w) * kAttnStageBytes; }
__device__ __forceinline__ uint32_t attn_swz(int row, int piece) {
  return static_cast<uint32_t>(row * 128 + ((piece ^ (row & 7)) << 4));
}

template <int D, int W>
__global__ void __launch_bounds__(W * 32, W == 8 ? 2 : 3) gqa_decode_kernel(const AttnParams p) {
  constexpr int kAttnWarps = W, kAttnThreads = W * 32;
  constexpr int NS = attn_stages(W);
  static_assert(D == 64, "this kernel is written for head_dim 64");
  // dynamic: the cluster merge buffer (clustered: [n_splits][grp][D + 2] floats on rank
  // 0), then at a 128-byte boundary the warps' K/V rings, reused for the warp merge
  extern __shared__ __align__(128) float gather[];
  constexpr int QW = D / 2 + 4;  // q_s row stride in 32-bit words (bank spread)
  __shared__ __align__(16) uint32_t q_s[16 * QW];        // bf16x2, 16 head rows (rows >= grp zero)
  __shared__ float wm[kAttnWarps][16], wl[kAttnWarps][16];
  __shared__ float rope_cs[2][D / 2];  // cos, sin of each pair's angle at pos

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int grp = p.hq / p.hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  if (!p.prefetch_kv) pdl_wait();  // q/k/v come from the previous kernel
  pdl_launch_dependents();
  const int pos = p.pos[b];
  if (pos < 0 || pos >= p.ctx_max) {  // outside the cache: record, read and write nothing
    if (p.prefetch_kv) pdl_wait();     // leave only after the preceding kernel, as every path does
    if (threadIdx.x == 0) record_error(5);
    return;  // uniform over the CTA and its cluster (one sequence), before any barrier
  }
  const int len = pos + 1;
  const int lo = split * p.split_len;
  const int hi = min(len, lo + p.split_len);

  // ---- this warp's positions
  const int n = max(0, hi - lo);
  const int per_warp = ((n + kAttnWarps * kAttnChunk - 1) / (kAttnWarps * kAttnChunk)) * kAttnChunk;
  const int w_lo = lo + warp * per_warp;
  const int w_hi = min(hi, w_lo + per_warp);
  const __nv_bfloat16* kbase = p.k_cache + (static_cast<size_t>(b) * p.hkv + kvh) * p.ctx_max * D;
  const __nv_bfloat16* vbase = p.v_cache + (static_cast<size_t>(b) * p.hkv + kvh) * p.ctx_max * D;

  // this warp's ring; stage ci % NS holds chunk ci (positions w_lo + 16 ci ..)
  const int gbytes = p.clustered ? ((p.n_splits * grp * (D + 2) * 4 + 127) & ~127) : 0;
  uint8_t* rings = reinterpret_cast<uint8_t*>(gather) + gbytes;
  const uint32_t ring_s = smem_u32(rings) + warp * NS * kAttnStageBytes;
  const int n_chunks = w_hi > w_lo ? (w_hi - w_lo + kAttnChunk - 1) / kAttnChunk : 0;
  // chunk ci: 16 K rows then 16 V rows, 8 pieces each, 8 pieces per lane.  Rows past the
  // end are the last valid row (their scores are masked).  One commit group per chunk
  // index, empty past the end, so the group count stays in step with the chunks.
  auto issue_chunk = [&](int ci) {
    if (ci < n_chunks) {
      const int c0 = w_lo + ci * kAttnChunk, last = w_hi - 1;
      const uint32_t st = ring_s + (ci % NS) * kAttnStageBytes;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int pc = lane + 32 * j;
        const int kv = pc >> 7, row = (pc >> 3) & 15, pce = pc & 7;
        const int r = min(c0 + row, last);
        cp_async16(st + kv * (kAttnChunk * 128) + attn_swz(row, pce),
                   (kv ? vbase : kbase) + static_cast<size_t>(r) * D + pce * 8);
      }
    }
    cp_async_commit();
  };
  // With prefetch_kv the warp's first chunks are issued before the PDL wait, unless a
  // chunk reaches row pos (appended below, after the wait): rows read are
  // min(c0 + r, w_hi - 1), which include pos only when w_hi == len.
  auto early_ok = [&](int c0) { return p.prefetch_kv && (w_hi != len || c0 + kAttnChunk - 1 < pos); };
  int n_pre = 0;
  while (n_pre < NS - 1 && n_pre < n_chunks && early_ok(w_lo + n_pre * kAttnChunk)) issue_chunk(n_pre++);
  // the rotation angles depend on pos only: with prefetch_kv (pos final at launch)
  // their fp64 evaluation runs before the wait, off the dependent path
  if (p.prefetch_kv && threadIdx.x < D / 2 && p.rope) rope_angle<D>(pos, p.theta, threadIdx.x, rope_cs[0][threadIdx.x], rope_cs[1][threadIdx.x]);
  if (p.prefetch_kv) pdl_wait();
  if (!p.prefetch_kv && threadIdx.x < D / 2 && p.rope) rope_angle<D>(pos, p.theta, threadIdx.x, rope_cs[0][threadIdx.x], rope_cs[1][threadIdx.x]);

  // ---- q heads of the group: rope -> bf16 -> shared (rows >= grp are zero)
  {
    __nv_bfloat16* qh = reinterpret_cast<__nv_bfloat16*>(q_s);
    for (int e = threadIdx.x; e < 16 * QW * 2; e += kAttnThreads) qh[e] = __float2bfloat16_rn(0.f);
    __syncthreads();  // also publishes rope_cs
    for (int e = threadIdx.x; e < grp * (D / 2); e += kAttnThreads) {
      const int j = e / (D / 2), i = e % (D / 2);
      const float* src = p.q + static_cast<size_t>(b) * p.ld_new + (kvh * grp + j) * D;
      rope_apply_bf16<D>(src, qh + j * QW * 2, i, rope_cs[0][i], rope_cs[1][i], p.rope);
    }
    // the split that holds the new position appends its k (rotated) and v
    if (p.append && pos >= lo && pos < hi) {
      const size_t row = ((static_cast<size_t>(b) * p.hkv + kvh) * p.ctx_max + pos) * D;
      const float* ks = p.k_new + static_cast<size_t>(b) * p.ld_new + kvh * D;
      const float* vs = p.v_new + static_cast<size_t>(b) * p.ld_new + kvh * D;
      for (int i = threadIdx.x; i < D / 2; i += kAttnThreads)
        rope_apply_bf16<D>(ks, p.k_cache + row, i, rope_cs[0][i], rope_cs[1][i], p.rope);
      for (int i = threadIdx.x; i < D; i += kAttnThreads) p.v_cache[row + i] = __float2bfloat16_rn(vs[i]);
    }
    __syncthreads();
  }

  // Q A-fragments: logical d pair (2t,2t+1) of k-step j <-> physical d 16t+4j+{0,1},
  // (2t+8,2t+9) <-> 16t+4j+{2,3}; head rows g+8 are always zero (grp <= 8).
  uint32_t qa[4][2];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    qa[j][0] = q_s[g * QW + 8 * t + 2 * j];
    qa[j][1] = q_s[g * QW + 8 * t + 2 * j + 1];
  }

  float m_run = -INFINITY, l_run = 0.f;
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  if (n_chunks > 0) {
    for (int ci = n_pre; ci < NS - 1; ++ci) issue_chunk(ci);  // the rest of the first NS - 1 chunks
    for (int c0 = w_lo; c0 < w_hi; c0 += kAttnChunk) {
      const int ci = (c0 - w_lo) / kAttnChunk;
      __syncwarp();  // every lane is done with stage (ci - 1) % NS, refilled next
      issue_chunk(ci + NS - 1);
      cp_async_wait<NS - 1>();
      __syncwarp();  // every lane's copies of chunk ci are visible to the warp
      uint4 kr[4], vr[4];
      {
        const uint8_t* st = rings + warp * NS * kAttnStageBytes + (ci % NS) * kAttnStageBytes;
        kr[0] = *reinterpret_cast<const uint4*>(st + attn_swz(g, 2 * t));
        kr[1] = *reinterpret_cast<const uint4*>(st + attn_swz(g, 2 * t + 1));
        kr[2] = *reinterpret_cast<const uint4*>(st + attn_swz(8 + g, 2 * t));
        kr[3] = *reinterpret_cast<const uint4*>(st + attn_swz(8 + g, 2 * t + 1));
        const uint8_t* sv = st + kAttnChunk * 128;
        vr[0] = *reinterpret_cast<const uint4*>(sv + attn_swz(2 * t, g));
        vr[1] = *reinterpret_cast<const uint4*>(sv + attn_swz(2 * t + 1, g));
        vr[2] = *reinterpret_cast<const uint4*>(sv + attn_swz(8 + 2 * t, g));
        vr[3] = *reinterpret_cast<const uint4*>(sv + attn_swz(9 + 2 * t, g));
      }
      // S = Q K^T for positions c0..c0+7 (n-tile 0) and c0+8..c0+15 (n-tile 1)
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const uint32_t kw[8] = {kr[2 * nt].x, kr[2 * nt].y, kr[2 * nt].z, kr[2 * nt].w,
                                kr[2 * nt + 1].x, kr[2 * nt + 1].y, kr[2 * nt + 1].z, kr[2 * nt + 1].w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          mma_bf16_m16n8k16(s[nt][0], s[nt][1], s[nt][2], s[nt][3], qa[j][0], 0u, qa[j][1], 0u, kw[2 * j],
                            kw[2 * j + 1]);
      }
      // scores (log2 units) with the causal / range mask; this lane: head g,
      // positions c0 + 8nt + 2t + {0,1}
      float sc[4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int pp = c0 + 8 * nt + 2 * t + e;
          sc[2 * nt + e] = pp < w_hi ? s[nt][e] * p.scale_log2 : -INFINITY;
        }
      float mc = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
      mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, 1));
      mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, 2));
      const float m_new = fmaxf(m_run, mc);  // finite: every chunk holds >= 1 valid position
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
      // P as the A operand (rows = heads, k = positions), split bf16 hi + lo
      const uint32_t ph0 = pack_bf16x2(pr[0], pr[1]), ph1 = pack_bf16x2(pr[2], pr[3]);
      const uint32_t pl0 = pack_bf16x2(pr[0] - bf16lo_to_f32(ph0), pr[1] - bf16hi_to_f32(ph0));
      const uint32_t pl1 = pack_bf16x2(pr[2] - bf16lo_to_f32(ph1), pr[3] - bf16hi_to_f32(ph1));
      const uint32_t va[4] = {vr[0].x, vr[0].y, vr[0].z, vr[0].w}, vb[4] = {vr[1].x, vr[1].y, vr[1].z, vr[1].w};
      const uint32_t vc[4] = {vr[2].x, vr[2].y, vr[2].z, vr[2].w}, vd[4] = {vr[3].x, vr[3].y, vr[3].z, vr[3].w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {  // n-tile i: column g <-> d = 8g + i
        const uint32_t sel = (i & 1) ? 0x7632u : 0x5410u;
        const uint32_t b0 = prmt(va[i >> 1], vb[i >> 1], sel);
        const uint32_t b1 = prmt(vc[i >> 1], vd[i >> 1], sel);
        mma_bf16_m16n8k16(o[i][0], o[i][1], o[i][2], o[i][3], ph0, 0u, ph1, 0u, b0, b1);
        mma_bf16_m16n8k16(o[i][0], o[i][1], o[i][2], o[i][3], pl0, 0u, pl1, 0u, b0, b1);
      }
    }
    cp_async_wait<0>();  // no copy into the rings is left in flight (the merge reuses them)
  }
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);

  // ---- merge the warps (head g rows; lane t holds d = 16t + i and 16t + 8 + i) through
  // the ring bytes, once every warp is done with its ring
  float (*wo)[16][D + 1] = reinterpret_cast<float (*)[16][D + 1]>(rings);
  static_assert(kAttnWarps * 16 * (D + 1) * 4 <= attn_ring_bytes(kAttnWarps), "merge buffer fits the rings");
  __syncthreads();
  if (t == 0) {
    wm[warp][g] = m_run;
    wl[warp][g] = l_run;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    wo[warp][g][16 * t + i] = o[i][0];
    wo[warp][g][16 * t + 8 + i] = o[i][1];
  }
  __syncthreads();
  const uint32_t gather_addr = smem_u32(gather);
  for (int e = threadIdx.x; e < grp * D; e += kAttnThreads) {
    const int j = e / D, d = e % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w][j]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        const float f = wm[w][j] == -INFINITY ? 0.f : exp2f(wm[w][j] - M);
        L += wl[w][j] * f;
        O += wo[w][j][d] * f;
      }
    }
    const int qhead = kvh * grp + j;
    if (p.n_splits == 1) {
      const size_t oi = static_cast<size_t>(b) * p.ldo + qhead * D + d;
      if (p.out_f32)
        reinterpret_cast<float*>(p.out)[oi] = O / L;
      else
        p.out[oi] = __float2bfloat16_rn(O / L);
    } else if (p.clustered) {
      // push (o, m, l) into rank 0's gather[split][j]
      const uint32_t base = gather_addr + ((split * grp + j) * (D + 2)) * 4;
      st_dsmem_f32(base + d * 4, 0, O);
      if (d == 0) {
        st_dsmem_f32(base + D * 4, 0, M);
        st_dsmem_f32(base + (D + 1) * 4, 0, L);
      }
    } else {
      float* pr = p.part + ((((static_cast<size_t>(b) * p.hkv + kvh) * p.n_splits + split) * grp + j) * (D + 2));
      pr[d] = O;
      if (d == 0) {
        pr[D] = M;
        pr[D + 1] = L;
      }
    }
  }
  if (p.clustered) {
    cluster_arrive_release();
    if (split != 0) return;  // nothing reads this CTA's shared memory
    cluster_wait_acquire();
    for (int e = threadIdx.x; e < grp * D; e += kAttnThreads) {
      const int j = e / D, d = e % D;
      float M = -INFINITY;
      for (int sp = 0; sp < p.n_splits; ++sp) M = fmaxf(M, gather[(sp * grp + j) * (D + 2) + D]);
      float L = 0.f, O = 0.f;
      for (int sp = 0; sp < p.n_splits; ++sp) {
        const float* g = gather + (sp * grp + j) * (D + 2);
        if (g[D] == -INFINITY) continue;  // split past this sequence's end
        const float f = exp2f(g[D] - M);
        L += g[D + 1] * f;
        O += g[d] * f;
      }
      const size_t oi = static_cast<size_t>(b) * p.ldo + (kvh * grp + j) * D + d;
      if (p.out_f32)
        reinterpret_cast<float*>(p.out)[oi] = O / L;
      else
        p.out[oi] = __float2bfloat16_rn(O / L);
    }
  }
}

// Log-sum-exp merge of the split partials: one CTA per (q head, sequence).
template <int D>
__global__ void __launch_bounds__(D) gqa_combine_kernel(const AttnParams p) {
  const int qhead = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int grp = p.hq / p.hkv;
  const int kvh = qhead / grp, j = qhead % grp;
  pdl_wait();
  pdl_launch_dependents();
  const float* base = p.part + ((static_cast<size_t>(b) * p.hkv + kvh) * p.n_splits * grp + j) * (D + 2);
  const size_t stride = static_cast<size_t>(grp) * (D + 2);
  float M = -INFINITY;
  for (int s = 0; s < p.n_splits; ++s) M = fmaxf(M, base[s * stride + D]);
  float L = 0.f, O = 0.f;
  for (int s = 0; s < p.n_splits; ++s) {
    const float ms = base[s * stride + D];
    if (ms == -INFINITY) continue;  // split past this sequence's end
    const float f = exp2f(ms - M);
    L += base[s * stride + D + 1] * f;
    O += base[s * stride + d] * f;
  }
  const size_t oi = static_cast<size_t>(b) * p.ldo + qhead * D + d;
  if (p.out_f32)
    reinterpret_cast<float*>(p.out)[oi] = O / L;
  else
    p.out[oi] = __float2bfloat16_rn(O / L);
}

}  // namespace b2
