// Qwen3.5 gated full-attention decode (head_dim 256): q/k RMSNorm (1 + w) ->
// partial RoPE -> KV-cache append -> softmax(q K^T / 16) V -> * sigmoid(gate).
//
// Reference arithmetic: transformers 5.5.0 Qwen3_5Attention.forward
// (models/qwen3_5/modeling_qwen3_5.py:647-692) between q/k/v_proj and o_proj,
// run by the reference in float32 (reference/from_q4nx.py:140-171): Qwen3_5RMSNorm
// (:711-725), apply_rotary_pos_emb with rotate_half on the first rotary dims
// (:544-579), the rotary frequencies of Qwen3_5TextRotaryEmbedding (:85-155,
// passed in as its inv_freq buffer), eager attention (:594-617).  The KV cache is
// bf16 (the decode path's cache layout); the appended row is rounded once.
//
// One CTA per (split, kv head, sequence), 8 warps.  The G = nq / nkv q heads of a
// kv head share each K and V row, read once: lane l owns dims 8l..8l+7, so a
// warp's 16-byte loads cover one 512-byte row per instruction.  Per chunk of
// 16 / G keys a lane forms 16 partial dot products (key x head), and a butterfly
// reduce-scatter over the warp (4 exchange steps + one add) leaves lane l with
// the full score of value (l >> 1): about one shuffle per score.  Online softmax
// per head, the warps' (max, sum, o) merged in shared memory; with one split the
// CTA applies the gate and stores, else it leaves fp32 partials for
// gated_attn_combine_kernel.
#pragma once

#include "b2_common.cuh"

namespace b2 {

constexpr int kGaThreads = 256;
constexpr int kGaWarps = kGaThreads / 32;
constexpr int kGaD = 256;

struct GatedAttnParams {
  const float* qg;  // [B][ld_qg]; q head h at h*512: q (256) | gate (256)
  const float* k_new;
  const float* v_new;  // [B][ld_kv], kv head g at g*256
  const float* q_norm_w;
  const float* k_norm_w;  // [256], applied as (1 + w)
  const float* inv_freq;  // [rot_half]: pair (i, i + rot_half) turns by pos * inv_freq[i]
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;  // [B][nkv][ctx_max][256]
  const int* pos;          // [B]: the new token's position; cache rows 0..pos-1 are valid
  void* out;               // [B][ldo] bf16 or fp32: attention * sigmoid(gate), nq*256 used
  float* part;             // [B][nkv][n_splits][G][258] (max, sum, o[256]) when n_splits > 1
  int ld_qg, ld_kv, ldo;
  int rot_half, ctx_max, max_len;
  int nq, nkv;
  int n_splits, split_len;
  float eps;
  int out_f32;
};

__device__ __forceinline__ void bf16x8_to_f32(const uint4 r, float (&f)[8]) {
  f[0] = bf16lo_to_f32(r.x); f[1] = bf16hi_to_f32(r.x);
  f[2] = bf16lo_to_f32(r.y); f[3] = bf16hi_to_f32(r.y);
  f[4] = bf16lo_to_f32(r.z); f[5] = bf16hi_to_f32(r.z);
  f[6] = bf16lo_to_f32(r.w); f[7] = bf16hi_to_f32(r.w);
}

__device__ __forceinline__ void gated_store(const GatedAttnParams& p, int b, int hq, int d, float attn) {
  const float gate = p.qg[(size_t)b * p.ld_qg + (size_t)hq * 2 * kGaD + kGaD + d];
  const float y = attn / (1.f + expf(-gate));
  const size_t oi = (size_t)b * p.ldo + (size_t)hq * kGaD + d;
  if (p.out_f32) static_cast<float*>(p.out)[oi] = y;
  else static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(y);
}

template <int G>
__global__ void __launch_bounds__(kGaThreads, 2) gated_attn_kernel(const GatedAttnParams p) {
  static_assert(G == 1 || G == 2 || G == 4, "q heads per kv head: 1, 2 or 4");
  constexpr int D = kGaD, KC = 16 / G, LG = G == 1 ? 0 : (G == 2 ? 1 : 2);
  constexpr unsigned FULL = 0xffffffffu;
  __shared__ __align__(16) float qs[G][D];
  __shared__ float ks[D], vs[D];
  __shared__ __align__(16) float o_s[kGaWarps][G][D];
  __shared__ float ml_s[kGaWarps][G][2];

  const int s = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();  // q/k/v come from the projection launched before
  pdl_launch_dependents();
  const int pos = p.pos[b];
  if (pos < 0 || pos >= p.max_len) {  // outside the planned key range: record, write nothing
    if (tid == 0) record_error(5);
    return;
  }
  const int t_begin = s * p.split_len;
  const int t_end = min(t_begin + p.split_len, pos + 1);  // keys [t_begin, t_end)

  // ---- q heads (warps 0..G-1) and k (warp 4) through RMSNorm (1 + w); v (warp 5) as is
  if (warp < G || warp == 4 || warp == 5) {
    const float* src;
    const float* w = nullptr;
    float* dst;
    if (warp < G) {
      src = p.qg + (size_t)b * p.ld_qg + (size_t)(g * G + warp) * 2 * D;
      w = p.q_norm_w;
      dst = qs[warp];
    } else if (warp == 4) {
      src = p.k_new + (size_t)b * p.ld_kv + (size_t)g * D;
      w = p.k_norm_w;
      dst = ks;
    } else {
      src = p.v_new + (size_t)b * p.ld_kv + (size_t)g * D;
      dst = vs;
    }
    float x[8], ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      x[e] = src[lane + 32 * e];
      ss = fmaf(x[e], x[e], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(FULL, ss, o);
    const float r = 1.f / sqrtf(ss / (float)D + p.eps);
#pragma unroll
    for (int e = 0; e < 8; ++e) dst[lane + 32 * e] = w ? x[e] * r * (1.f + w[lane + 32 * e]) : x[e];
  }
  __syncthreads();
  // ---- RoPE on the first 2*rot_half dims of the q heads and k (rotate_half pairs)
  const int rh = p.rot_half;
  for (int it = tid; it < (G + 1) * rh; it += kGaThreads) {
    const int j = it / rh, i = it - j * rh;
    float* v = j < G ? qs[j] : ks;
    float sn, cs;
    sincosf((float)pos * p.inv_freq[i], &sn, &cs);
    const float x0 = v[i], x1 = v[i + rh];
    v[i] = x0 * cs - x1 * sn;
    v[i + rh] = x1 * cs + x0 * sn;
  }
  __syncthreads();
  // q takes the 1/sqrt(256) score scale (a power of two: exact)
  for (int i = tid; i < G * D; i += kGaThreads) (&qs[0][0])[i] *= 0.0625f;
  // the split holding pos appends the new row; its warps read it back below
  const size_t head_base = ((size_t)b * p.nkv + g) * p.ctx_max * D;
  if (pos >= t_begin && pos < t_begin + p.split_len) {
    p.k_cache[head_base + (size_t)pos * D + tid] = __float2bfloat16_rn(ks[tid]);
    p.v_cache[head_base + (size_t)pos * D + tid] = __float2bfloat16_rn(vs[tid]);
  }
  __syncthreads();

  // ---- keys: warp w takes a contiguous run of the CTA's range, KC keys per step
  const int n_keys = max(0, t_end - t_begin);
  const int per_warp = ((n_keys + kGaWarps - 1) / kGaWarps + KC - 1) / KC * KC;
  const int w0 = t_begin + warp * per_warp;
  const int w1 = min(w0 + per_warp, t_end);
  const __nv_bfloat16* kb = p.k_cache + head_base + 8 * lane;
  const __nv_bfloat16* vb = p.v_cache + head_base + 8 * lane;
  float m_run[G], l_run[G], o[G][8];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m_run[h] = -INFINITY;
    l_run[h] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[h][e] = 0.f;
  }
  const int my_v = lane >> 1, my_j = my_v >> LG, my_h = my_v & (G - 1);
  for (int t0 = w0; t0 < w1; t0 += KC) {
    uint4 kr[KC], vr[KC];
#pragma unroll
    for (int j = 0; j < KC; ++j) {
      const int t = min(t0 + j, w1 - 1);
      kr[j] = *reinterpret_cast<const uint4*>(kb + (size_t)t * D);
      vr[j] = *reinterpret_cast<const uint4*>(vb + (size_t)t * D);
    }
    float vals[16];
#pragma unroll
    for (int j = 0; j < KC; ++j) {
      float kf[8];
      bf16x8_to_f32(kr[j], kf);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float4 q0 = *reinterpret_cast<const float4*>(&qs[h][8 * lane]);
        const float4 q1 = *reinterpret_cast<const float4*>(&qs[h][8 * lane + 4]);
        float acc = q0.x * kf[0];
        acc = fmaf(q0.y, kf[1], acc); acc = fmaf(q0.z, kf[2], acc); acc = fmaf(q0.w, kf[3], acc);
        acc = fmaf(q1.x, kf[4], acc); acc = fmaf(q1.y, kf[5], acc); acc = fmaf(q1.z, kf[6], acc);
        acc = fmaf(q1.w, kf[7], acc);
        vals[j * G + h] = acc;
      }
    }
    // reduce-scatter: after the masks 16, 8, 4, 2 lane l holds value (l >> 1) summed over
    // the 16 lanes sharing bit 0; the xor-1 add completes the sum over all 32
#pragma unroll
    for (int st = 0; st < 4; ++st) {
      const int mask = 16 >> st, half = 8 >> st;
      const bool up = (lane & mask) != 0;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = up ? vals[i] : vals[i + half];
        const float keep = up ? vals[i + half] : vals[i];
        vals[i] = keep + __shfl_xor_sync(FULL, send, mask);
      }
    }
    // every lane takes part in each exchange: the key-validity select comes after it
    const float tot = vals[0] + __shfl_xor_sync(FULL, vals[0], 1);
    const bool valid = t0 + my_j < w1;
    const float sc = valid ? tot : -INFINITY;
    // per-head chunk max over the lanes holding that head's keys (lane bits above 1 + log2 G)
    float mx = sc;
#pragma unroll
    for (int mask = 2 * G; mask <= 16; mask <<= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, mask));
    float mnew[G], alpha[G], my_m = 0.f;
#pragma unroll
    for (int h = 0; h < G; ++h) {
      mnew[h] = fmaxf(m_run[h], __shfl_sync(FULL, mx, 2 * h));  // key t0 is valid: finite
      alpha[h] = m_run[h] == -INFINITY ? 0.f : expf(m_run[h] - mnew[h]);
      if (my_h == h) my_m = mnew[h];
    }
    const float pr = valid ? expf(sc - my_m) : 0.f;
    float sm = pr;
#pragma unroll
    for (int mask = 2 * G; mask <= 16; mask <<= 1) sm += __shfl_xor_sync(FULL, sm, mask);
#pragma unroll
    for (int h = 0; h < G; ++h) {
      l_run[h] = fmaf(l_run[h], alpha[h], __shfl_sync(FULL, sm, 2 * h));
      m_run[h] = mnew[h];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[h][e] *= alpha[h];
    }
#pragma unroll
    for (int j = 0; j < KC; ++j) {
      float vf[8];
      bf16x8_to_f32(vr[j], vf);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float pj = __shfl_sync(FULL, pr, 2 * (j * G + h));  // 0 for keys past the run
#pragma unroll
        for (int e = 0; e < 8; ++e) o[h][e] = fmaf(pj, vf[e], o[h][e]);
      }
    }
  }

  // ---- merge the warps (thread = dim); apply the gate or leave split partials
#pragma unroll
  for (int h = 0; h < G; ++h) {
    *reinterpret_cast<float4*>(&o_s[warp][h][8 * lane]) = make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
    *reinterpret_cast<float4*>(&o_s[warp][h][8 * lane + 4]) = make_float4(o[h][4], o[h][5], o[h][6], o[h][7]);
    if (lane == 0) {
      ml_s[warp][h][0] = m_run[h];
      ml_s[warp][h][1] = l_run[h];
    }
  }
  __syncthreads();
  const int d = tid;
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kGaWarps; ++w) M = fmaxf(M, ml_s[w][h][0]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kGaWarps; ++w) {
      const float mw = ml_s[w][h][0];
      if (mw != -INFINITY) {
        const float f = expf(mw - M);
        L = fmaf(ml_s[w][h][1], f, L);
        O = fmaf(o_s[w][h][d], f, O);
      }
    }
    if (p.n_splits == 1) {
      gated_store(p, b, g * G + h, d, O / L);
    } else {
      float* dst = p.part + ((((size_t)b * p.nkv + g) * p.n_splits + s) * G + h) * (D + 2);
      dst[2 + d] = O;
      if (d == 0) {
        dst[0] = M;
        dst[1] = L;
      }
    }
  }
}

// Merge the splits of one (q head, sequence): thread = dim.
__global__ void __launch_bounds__(kGaThreads) gated_attn_combine_kernel(const GatedAttnParams p) {
  constexpr int D = kGaD;
  const int hq = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  const int pos = p.pos[b];
  if (pos < 0 || pos >= p.max_len) return;  // recorded by the attention kernel
  const int G = p.nq / p.nkv, g = hq / G, h = hq - g * G;
  const float* base = p.part + (((size_t)b * p.nkv + g) * p.n_splits * G + h) * (D + 2);
  const size_t stride = (size_t)G * (D + 2);
  float M = -INFINITY;
  for (int s = 0; s < p.n_splits; ++s) M = fmaxf(M, base[s * stride]);
  float L = 0.f, O = 0.f;
  for (int s = 0; s < p.n_splits; ++s) {
    const float mw = base[s * stride];
    if (mw != -INFINITY) {
      const float f = expf(mw - M);
      L = fmaf(base[s * stride + 1], f, L);
      O = fmaf(base[s * stride + 2 + d], f, O);
    }
  }
  gated_store(p, b, hq, d, O / L);
}

}  // namespace b2
