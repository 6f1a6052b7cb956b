// Gated DeltaNet (linear attention) decode step: conv update -> q/k l2norm ->
// gated delta rule on the recurrent state -> gated RMSNorm, one kernel.
//
// Reference arithmetic: transformers 5.5.0 Qwen3_5GatedDeltaNet.forward on its
// decode branch (models/qwen3_5/modeling_qwen3_5.py:422-533), which the
// reference runs in float32 (reference/from_q4nx.py:140-171): the conv update
// torch_causal_conv1d_update (:210-225), l2norm (:228-231), the recurrence
// torch_recurrent_gated_delta_rule (:314-353) and Qwen3_5RMSNormGated (:175-190).
//
// One CTA per (v head, sequence), 8 warps.  The head's recurrent state
// S[dk=128][dv=128] fp32 (64 KB, row-major as transformers' cache holds it) is
// the only large operand: warp w owns rows 16w..16w+15, lane l owns columns
// 4l..4l+3, so each load/store instruction of a warp moves one 512-byte row.
// The 16 float4 loads of a thread are issued before anything else (before the
// PDL wait when the caller marks the state final), the state lives in
// registers through the decay, the kv_mem reduction, the rank-1 update and the
// output reduction, and is stored once: 128 KB of HBM traffic per (head,
// sequence) and step, which bounds the kernel.
//
// The conv state [B][conv_dim][4] holds the last four conv inputs per channel.
// When k heads are repeated over several v heads (nv / nk = ratio > 1) the
// ratio CTAs of one k head form a cluster: each computes the q/k conv from the
// old state, and rank 0 writes the shifted q/k state only after a cluster
// barrier that every CTA passes after its reads.
#pragma once

#include "b2_common.cuh"

namespace b2 {

constexpr int kDeltaThreads = 256;
constexpr int kDeltaHeadDim = 128;  // dk = dv (Qwen3.5 / Qwen3-Next linear attention)
constexpr int kDeltaConvWidth = 4;

struct DeltaParams {
  const float* qkv;  // [B][ld_qkv]: q (nk*128) | k (nk*128) | v (nv*128), before the conv
  const float* z;    // [B][ld_z] gate, nv*128
  const float* b;    // [B][ld_ab] -> beta = sigmoid(b)
  const float* a;    // [B][ld_ab] -> g = -exp(A_log) * softplus(a + dt_bias)
  float* conv_state;     // [B][conv_dim][4]
  const float* conv_w;   // [conv_dim][4]
  const float* A_log;    // [nv]
  const float* dt_bias;  // [nv]
  const float* norm_w;   // [128]
  float* state;          // [B][nv][128][128]
  void* out;             // [B][ldo] bf16 or fp32, nv*128 used
  int ld_qkv, ld_z, ld_ab, ldo;
  int nk, nv;
  float eps;
  int out_f32;
  int prefetch_state;  // the state and conv state are final at launch: load before the PDL wait
};

__device__ __forceinline__ float silu_f32(float x) { return x / (1.f + expf(-x)); }

__global__ void __launch_bounds__(kDeltaThreads, 2) gated_delta_step_kernel(const DeltaParams p) {
  constexpr int D = kDeltaHeadDim, W = kDeltaConvWidth;
  __shared__ float qn[D], kn[D], vs[D];
  __shared__ float red[kDeltaThreads / 32][D];
  __shared__ float part[kDeltaThreads / 32][2];
  __shared__ float gates[2];  // decay = exp(g), beta

  const int h = blockIdx.x, bt = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ratio = p.nv / p.nk, kh = h / ratio;
  const int key_dim = p.nk * D, conv_dim = 2 * key_dim + p.nv * D;

  float4* srow = reinterpret_cast<float4*>(p.state + ((size_t)bt * p.nv + h) * D * D) + warp * 16 * (D / 4) + lane;
  float4 S[16];
  auto load_state = [&]() {
#pragma unroll
    for (int i = 0; i < 16; ++i) S[i] = srow[i * (D / 4)];
  };
  // q/k channel of this thread (threads 0..127 q, 128..255 k) and the v channel of threads 0..127
  const int qk_ch = tid < D ? kh * D + tid : key_dim + kh * D + (tid - D);
  const int v_ch = 2 * key_dim + h * D + (tid & (D - 1));
  float4* cs_qk = reinterpret_cast<float4*>(p.conv_state + ((size_t)bt * conv_dim + qk_ch) * W);
  float4* cs_v = reinterpret_cast<float4*>(p.conv_state + ((size_t)bt * conv_dim + v_ch) * W);
  float4 c_qk, c_v;
  if (p.prefetch_state) {
    load_state();
    c_qk = *cs_qk;
    if (tid < D) c_v = *cs_v;
  }
  pdl_wait();
  pdl_launch_dependents();
  if (!p.prefetch_state) {
    load_state();
    c_qk = *cs_qk;
    if (tid < D) c_v = *cs_v;
  }

  // ---- conv update + silu (torch_causal_conv1d_update): window = last 3 states + the new input
  const float* xrow = p.qkv + (size_t)bt * p.ld_qkv;
  const float x_qk = xrow[qk_ch];
  const float4 w_qk = reinterpret_cast<const float4*>(p.conv_w)[qk_ch];
  const float y_qk = silu_f32(w_qk.x * c_qk.y + w_qk.y * c_qk.z + w_qk.z * c_qk.w + w_qk.w * x_qk);
  float x_v = 0.f;
  if (tid < D) {
    x_v = xrow[v_ch];
    const float4 w_v = reinterpret_cast<const float4*>(p.conv_w)[v_ch];
    vs[tid] = silu_f32(w_v.x * c_v.y + w_v.y * c_v.z + w_v.z * c_v.w + w_v.w * x_v);
    *cs_v = make_float4(c_v.y, c_v.z, c_v.w, x_v);  // v channels belong to this head alone
  }
  if (ratio > 1) cluster_arrive_release();  // this CTA's reads of the shared q/k conv state are done
  else *cs_qk = make_float4(c_qk.y, c_qk.z, c_qk.w, x_qk);

  // ---- l2norm of q (warps 0-3) and k (warps 4-7); q also takes 1/sqrt(dk)
  float ss = y_qk * y_qk;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) part[warp][0] = ss;
  if (tid == 0) {
    const float av = p.a[(size_t)bt * p.ld_ab + h] + p.dt_bias[h];
    const float sp = av > 20.f ? av : log1pf(expf(av));  // torch softplus, threshold 20
    gates[0] = expf(-expf(p.A_log[h]) * sp);
    gates[1] = 1.f / (1.f + expf(-p.b[(size_t)bt * p.ld_ab + h]));
  }
  __syncthreads();
  {
    const int g0 = tid < D ? 0 : 4;
    const float tot = part[g0][0] + part[g0 + 1][0] + part[g0 + 2][0] + part[g0 + 3][0];
    const float inv = 1.f / sqrtf(tot + 1e-6f);
    if (tid < D) qn[tid] = y_qk * inv * 0.08838834764831845f;  // 1/sqrt(128)
    else kn[tid - D] = y_qk * inv;
  }
  __syncthreads();
  const float decay = gates[0], beta = gates[1];

  // ---- S *= exp(g); kv_mem = S^T k
  const int r0 = warp * 16;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    S[i].x *= decay; S[i].y *= decay; S[i].z *= decay; S[i].w *= decay;
    const float kk = kn[r0 + i];
    acc.x = fmaf(S[i].x, kk, acc.x); acc.y = fmaf(S[i].y, kk, acc.y);
    acc.z = fmaf(S[i].z, kk, acc.z); acc.w = fmaf(S[i].w, kk, acc.w);
  }
  reinterpret_cast<float4*>(red[warp])[lane] = acc;
  __syncthreads();
  float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int w = 0; w < kDeltaThreads / 32; ++w) {
    const float4 r = reinterpret_cast<const float4*>(red[w])[lane];
    kv.x += r.x; kv.y += r.y; kv.z += r.z; kv.w += r.w;
  }
  const float4 vv = reinterpret_cast<const float4*>(vs)[lane];
  const float4 dl = make_float4((vv.x - kv.x) * beta, (vv.y - kv.y) * beta, (vv.z - kv.z) * beta,
                                (vv.w - kv.w) * beta);
  __syncthreads();  // red is reused below

  // ---- S += k delta^T; o = S^T q; store S
  acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float kk = kn[r0 + i], qq = qn[r0 + i];
    S[i].x = fmaf(kk, dl.x, S[i].x); S[i].y = fmaf(kk, dl.y, S[i].y);
    S[i].z = fmaf(kk, dl.z, S[i].z); S[i].w = fmaf(kk, dl.w, S[i].w);
    acc.x = fmaf(S[i].x, qq, acc.x); acc.y = fmaf(S[i].y, qq, acc.y);
    acc.z = fmaf(S[i].z, qq, acc.z); acc.w = fmaf(S[i].w, qq, acc.w);
    srow[i * (D / 4)] = S[i];
  }
  reinterpret_cast<float4*>(red[warp])[lane] = acc;
  __syncthreads();

  // ---- gated RMSNorm over the head's 128 outputs (threads 0..127, one column each)
  float o = 0.f;
  if (tid < D) {
#pragma unroll
    for (int w = 0; w < kDeltaThreads / 32; ++w) o += red[w][tid];
    float s2 = o * o;
#pragma unroll
    for (int k = 16; k > 0; k >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, k);
    if (lane == 0) part[warp][1] = s2;
  }
  __syncthreads();
  if (tid < D) {
    const float ms = (part[0][1] + part[1][1] + part[2][1] + part[3][1]) / (float)D;
    const float zz = p.z[(size_t)bt * p.ld_z + h * D + tid];
    const float y = o * rsqrtf(ms + p.eps) * p.norm_w[tid] * silu_f32(zz);
    const size_t oi = (size_t)bt * p.ldo + h * D + tid;
    if (p.out_f32) static_cast<float*>(p.out)[oi] = y;
    else static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(y);
  }

  // ---- the shared q/k conv state: rank 0 of the cluster shifts it once every CTA has read it
  if (ratio > 1) {
    cluster_wait_acquire();
    if (cluster_ctarank() == 0) *cs_qk = make_float4(c_qk.y, c_qk.z, c_qk.w, x_qk);
  }
}

}  // namespace b2
