// b2q4nx: the C-ABI shared library (one translation unit; the kernels live in
// the .cuh files it includes so that the device error word is a single symbol).
//
// Host responsibilities per call: validate shapes/alignment, pick the launch
// plan (split-K cluster size, persistent grid, pipeline depth) from the device's
// SM count and shared-memory limit, and launch on the caller's stream.

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/b2q4nx.h"
#include "b2_common.cuh"
#include "q4_gemm_tc.cuh"
#include "q4nx_dequant.cuh"
#include "gated_attention.cuh"
#include "gated_delta.cuh"
#include "gqa_decode.cuh"
#include "q4nx_gemv.cuh"
#include "rmsnorm.cuh"
#include "tp_exchange.cuh"

namespace {

thread_local char g_msg[512] = "";
int g_pdl = 1;
unsigned long long g_peer_timeout_ns = B2_WAIT_TIMEOUT_NS;  // bounded waits on other ranks (b2_set_peer_timeout_ms)

// A pulled seam for the _rmsnorm GEMMs' x pre-pass (tensor-parallel decode): the residual
// rows gain the sum over ranks of the fp32 partials at part_off of every peer region.
// a seam's rows from every rank are staged in the pre-pass's shared memory up to this size
constexpr size_t kSeamStageMax = 160 * 1024;
struct SeamArgs {
  void* const* peers;
  int world, rank, seam, ld_part;
  long long part_off;
};

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  cudaGetLastError();  // clear the sticky-free error so later calls see their own
  return fail(B2_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

struct DevInfo {
  int ok = 0;
  int sms = 0;
  int smem_optin = 0;
  int smem_per_sm = 0;
  int smem_reserved = 0;
  int major = 0, minor = 0;
};

std::mutex g_mu;
DevInfo g_dev[64];

// Current device's properties; B2_OK or an error status.
int device_info(DevInfo* out) {
  int d = -1;
  cudaError_t e = cudaGetDevice(&d);
  if (e != cudaSuccess || d < 0) return fail(B2_ERR_NO_DEVICE, "no current CUDA device (%s)", cudaGetErrorString(e));
  if (d >= 64) return fail(B2_ERR_NO_DEVICE, "device ordinal %d out of range", d);
  std::lock_guard<std::mutex> lk(g_mu);
  DevInfo& di = g_dev[d];
  if (!di.ok) {
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, d);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
    di.sms = prop.multiProcessorCount;
    di.smem_optin = static_cast<int>(prop.sharedMemPerBlockOptin);
    di.smem_per_sm = static_cast<int>(prop.sharedMemPerMultiprocessor);
    di.smem_reserved = static_cast<int>(prop.reservedSharedMemPerBlock);
    di.major = prop.major;
    di.minor = prop.minor;
    di.ok = 1;
  }
  if (di.major != 10) return fail(B2_ERR_UNSUPPORTED, "device is sm_%d%d; this library is built for sm_100a", di.major, di.minor);
  *out = di;
  return B2_OK;
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Launch-plan knobs, read once from the environment (for tuning experiments):
//   B2Q4NX_MAX_CLUSTER   largest split-K cluster (1..16, default 16)
//   B2Q4NX_CTAS_PER_SM   force 1 or 2 GEMV CTAs per SM (default: 2 when they fit)
//   B2Q4NX_MAX_STAGES    cap on the shared-memory pipeline depth (1..8)
//   B2Q4NX_TC_SPLITS / _TC_RAW / _TC_XSTAGES / _TC_ABUFS   tensor-core GEMM split-K
//                        count, raw (<= 10) and x pipeline depths, A buffers per slice
//   B2Q4NX_TC_PRE_RAW    raw stages the GEMM issues before its PDL wait (default: its
//                        whole raw ring; 2-4 measured the same, 1 slower)
//   B2Q4NX_TC_PREP_EARLY 1: the GEMM's x pre-pass releases the GEMM before its own wait
//   B2Q4NX_PDL_MASK      launch kinds that use PDL: 1 GEMV, 2 GEMM pre-pass, 4 GEMM,
//                        8 attention, 16 exchange, 32 other (default 0x37)
//   B2Q4NX_ATTN_WAVE     0: attention splits as many as the 4-CTAs-per-SM target asks
//                        (default 1: launches capped at one wave of resident CTAs)
struct Tuning {
  int max_cluster = 16;
  int ctas_per_sm = 0;
  int max_stages = b2::kMaxStages;
  int tc_splits = 0, tc_raw = 0, tc_xst = 0, tc_abufs = 0;  // tensor-core GEMM overrides (0 = plan)
  int tc_pre_raw = 0;  // raw stages the GEMM issues before its PDL wait (0 = all of its ring)
  // GEMM x pre-pass releases the GEMM before its own PDL wait (off: after an attention
  // call the GEMM's CTAs, over half an SM's shared memory each, would take SMs from it)
  int tc_prep_early = 0;
  // launch kinds that use PDL (PdlKind bits).  Not attention: launched early behind a
  // tensor-core GEMM its CTAs contend with the GEMM's, and a batch-32 decode step of
  // config 4 measured 4.78 ms without it against 5.45 ms with it (batch 1: equal,
  // batch 8: 2.87 against 2.93 ms)
  int pdl_mask = 0x37;
  int attn_wave = 1;  // attention: cap unclustered splits at one wave of resident CTAs
  // attention warps per CTA: 1 always 8 (default: measured equal or faster at every
  // bench shape), 2 always 4, 0 by launch shape (8 when the launch has at most one CTA
  // per SM, else 4)
  int attn_wide = 1;
  int gated_min_split = 256;  // gated attention: fewest keys per split
};
// PDL per launch kind (B2Q4NX_PDL_MASK, default all but attention): a kind's launches
// may start before the preceding kernel completes
enum PdlKind : int {
  kPdlGemv = 1, kPdlGemmPrep = 2, kPdlGemm = 4, kPdlAttention = 8, kPdlExchange = 16, kPdlOther = 32
};
const Tuning& tuning();
bool pdl_for(int kind) { return g_pdl && (tuning().pdl_mask & kind) != 0; }

const Tuning& tuning() {
  static const Tuning t = [] {
    Tuning v;
    if (const char* e = getenv("B2Q4NX_MAX_CLUSTER")) v.max_cluster = std::max(1, std::min(16, atoi(e)));
    if (const char* e = getenv("B2Q4NX_CTAS_PER_SM")) v.ctas_per_sm = std::max(0, std::min(2, atoi(e)));
    if (const char* e = getenv("B2Q4NX_MAX_STAGES")) v.max_stages = std::max(1, std::min(b2::kMaxStages, atoi(e)));
    if (const char* e = getenv("B2Q4NX_TC_SPLITS")) v.tc_splits = std::max(0, atoi(e));
    if (const char* e = getenv("B2Q4NX_TC_RAW")) v.tc_raw = std::max(0, std::min(10, atoi(e)));
    if (const char* e = getenv("B2Q4NX_TC_XSTAGES")) v.tc_xst = std::max(0, std::min(8, atoi(e)));
    if (const char* e = getenv("B2Q4NX_TC_ABUFS")) v.tc_abufs = std::max(0, std::min(2, atoi(e)));
    if (const char* e = getenv("B2Q4NX_TC_PRE_RAW")) v.tc_pre_raw = std::max(0, std::min(8, atoi(e)));
    if (const char* e = getenv("B2Q4NX_TC_PREP_EARLY")) v.tc_prep_early = atoi(e) != 0;
    if (const char* e = getenv("B2Q4NX_PDL_MASK")) v.pdl_mask = static_cast<int>(strtol(e, nullptr, 0)) & 0x3F;
    if (const char* e = getenv("B2Q4NX_ATTN_WAVE")) v.attn_wave = atoi(e) != 0;
    if (const char* e = getenv("B2Q4NX_ATTN_WIDE")) v.attn_wide = std::max(0, std::min(2, atoi(e)));
    if (const char* e = getenv("B2Q4NX_GATED_MIN_SPLIT")) v.gated_min_split = std::max(64, std::min(4096, atoi(e)));
    return v;
  }();
  return t;
}

// ------------------------------------------------------------------ GEMV
template <int QT, int NB, int EPI>
int launch_gemv_t(b2::GemvParams p, const DevInfo& di, cudaStream_t stream) {
  using namespace b2;
  auto kernel = q4nx_gemv_kernel<QT, NB, EPI>;
  constexpr int SLOT = QTraits<QT>::kSlot;
  constexpr int STAGE = 4 * SLOT;
  static int attr_set[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, di.smem_optin);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemv)");
    attr_set[dev] = 1;
  }

  const int G = p.n_groups;
  const int batch = p.batch;
  // batch-1 q4 with the fused norm keeps the fp32 row in shared memory (kernel: x_norm_bulk)
  const int norm_k = (QT == kQ4 && NB == 1 && batch == 1 && p.xf) ? p.k_tiles * 256 : 0;
  // largest K slice whose staged x (batch rows, fp16) stays within 48 KB
  const int kt_cap = std::max(1, (48 * 1024) / (batch * 512 + 16));
  // CTAs per SM: two when the register budget (NB == 1) and shared memory allow
  auto fixed_bytes = [&](int ktps) {
    const GemvSmem base(SLOT, NB, 0, ktps * 256 + 8, ktps, batch, norm_k);
    return base.total + 2 * kMaxStages * 8;
  };
  const int per_cta_2 = di.smem_per_sm / 2 - di.smem_reserved;

  const Tuning& tu = tuning();
  // Plans, in order of preference.  Chained (weights may stream before the PDL
  // wait): one CTA per SM in at most half of its shared memory, so the next
  // kernel's CTAs can be resident alongside and prefetch their weights while
  // this one runs.  Otherwise: two CTAs per SM if they fit, else one.
  // The chained plan is used only when every CTA's whole weight slice fits its
  // ring (complete prefetch); large GEMVs are bandwidth-bound and keep two CTAs/SM.
  bool chained = false;
  if (p.prefetch_before_wait && G <= di.sms) {
    int S1 = std::min(std::min(tu.max_cluster, p.k_tiles), std::max(1, di.sms / G));
    S1 = std::max(S1, (p.k_tiles + kt_cap - 1) / kt_cap);
    const int kt1 = (p.k_tiles + S1 - 1) / S1;
    chained = fixed_bytes(kt1) + kt1 * STAGE <= per_cta_2;
  }
  int cps = 1, S = 1, ktps = p.k_tiles, budget = di.smem_optin;
  for (int attempt = 0; attempt < 2; ++attempt) {
    if (chained) {
      cps = 1;
      budget = attempt == 0 ? per_cta_2 : di.smem_optin;
    } else {
      cps = (attempt == 0 && NB == 1 && tu.ctas_per_sm != 1) ? 2 : 1;
      if (attempt == 1 && tu.ctas_per_sm == 2 && NB == 1) cps = 2;
      budget = cps == 2 ? per_cta_2 : di.smem_optin;
    }
    const int cap = cps * di.sms;
    S = 1;
    if (G < cap) S = std::min(std::min(tu.max_cluster, p.k_tiles), std::max(1, cap / G));
    S = std::max(S, (p.k_tiles + kt_cap - 1) / kt_cap);
    S = std::min(S, p.k_tiles);
    ktps = (p.k_tiles + S - 1) / S;
    S = (p.k_tiles + ktps - 1) / ktps;
    const int want = std::min(2, ktps);  // at least double-buffered, or the whole slice
    if (fixed_bytes(ktps) + want * STAGE <= budget) break;
  }
  if (S > 16) return fail(B2_ERR_ARG, "K too large for one cluster (k_tiles=%d, batch=%d)", p.k_tiles, batch);

  const int x_stride = ktps * 256 + 8;
  int grid_y;
  if (S == 1) {
    grid_y = std::min(G, cps * di.sms);  // persistent over groups
  } else {
    if (G > 65535) return fail(B2_ERR_ARG, "too many row groups (%d) for a split-K grid", G);
    grid_y = G;
  }
  const int groups_per_cta = (G + grid_y - 1) / grid_y;
  const int total_stages = ktps * groups_per_cta;
  int stages = std::min(tu.max_stages, (budget - fixed_bytes(ktps)) / STAGE);
  stages = std::min(stages, total_stages);
  if (stages < 1) return fail(B2_ERR_ARG, "K slice too large for shared memory");
  const GemvSmem L(SLOT, NB, stages, x_stride, ktps, batch, norm_k);

  p.kt_per_split = ktps;
  p.n_splits = S;
  p.stages = stages;
  p.x_stride = x_stride;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S, grid_y, 1);
  cfg.blockDim = dim3(kGemvThreads, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (S > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = S;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl_for(kPdlGemv)) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, p);
  if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
  return B2_OK;
}

int gemv_common(int qt, int epi, const uint8_t* w0, const uint8_t* w1, int n_tile_rows, int k_tiles,
                const uint16_t* x, int batch, int ldx, void* y, int ldy, int flags, void* stream,
                const float* xf = nullptr, const uint16_t* norm_w = nullptr, float eps = 0.f) {
  DevInfo di;
  int st = device_info(&di);
  if (st != B2_OK) return st;
  if (xf) {  // fused RMSNorm: x is the fp32 residual row, normalised in the prologue
    if (!norm_w) return fail(B2_ERR_ARG, "null norm weight");
    if (!aligned(xf, 16) || (ldx % 4) || !aligned(norm_w, 16)) return fail(B2_ERR_ALIGN, "x/norm weight alignment");
    if (!(eps >= 0.f)) return fail(B2_ERR_ARG, "eps must be >= 0");
    x = reinterpret_cast<const uint16_t*>(xf);  // satisfies the checks below; the kernel reads xf
  }
  if (!w0 || !x || !y || (epi == b2::kEpiSwiglu && !w1)) return fail(B2_ERR_ARG, "null pointer argument");
  if (n_tile_rows < 1 || k_tiles < 1) return fail(B2_ERR_ARG, "n_tile_rows=%d k_tiles=%d", n_tile_rows, k_tiles);
  if (batch < 1 || batch > 16) return fail(B2_ERR_ARG, "batch %d outside 1..16", batch);
  if (ldx < k_tiles * 256) return fail(B2_ERR_ARG, "ldx %d < K %d", ldx, k_tiles * 256);
  if (ldy < n_tile_rows * 32) return fail(B2_ERR_ARG, "ldy %d < N %d", ldy, n_tile_rows * 32);
  if (!aligned(w0, 16) || (w1 && !aligned(w1, 16))) return fail(B2_ERR_ALIGN, "weights must be 16-byte aligned");
  if (!aligned(x, 16) || (ldx % 8)) return fail(B2_ERR_ALIGN, "x must be 16-byte aligned with ldx %% 8 == 0");
  if (!aligned(y, epi == b2::kEpiSwiglu ? 2 : 4)) return fail(B2_ERR_ALIGN, "y misaligned");
  if ((flags & ~(B2_GEMV_ACCUMULATE | B2_GEMV_PREFETCH)) != 0) return fail(B2_ERR_ARG, "unknown flags 0x%x", flags);
  if (epi == b2::kEpiSwiglu && (flags & B2_GEMV_ACCUMULATE)) return fail(B2_ERR_ARG, "SwiGLU cannot accumulate");

  b2::GemvParams p = {};
  p.w0 = w0;
  p.w1 = w1;
  p.n_tile_rows = n_tile_rows;
  p.k_tiles = k_tiles;
  p.x = reinterpret_cast<const __nv_bfloat16*>(x);
  p.batch = batch;
  p.ldx = ldx;
  p.y = y;
  p.ldy = ldy;
  p.accumulate = (flags & B2_GEMV_ACCUMULATE) ? 1 : 0;
  p.prefetch_before_wait = (flags & B2_GEMV_PREFETCH) ? 1 : 0;
  p.n_groups = epi == b2::kEpiSwiglu ? (n_tile_rows + 1) / 2 : (n_tile_rows + 3) / 4;
  p.xf = xf;
  p.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w);
  p.eps = eps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nb = batch <= 8 ? 1 : 2;
  if (qt == b2::kQ4 && epi == b2::kEpiF32)
    return nb == 1 ? launch_gemv_t<b2::kQ4, 1, b2::kEpiF32>(p, di, s) : launch_gemv_t<b2::kQ4, 2, b2::kEpiF32>(p, di, s);
  if (qt == b2::kQ8 && epi == b2::kEpiF32)
    return nb == 1 ? launch_gemv_t<b2::kQ8, 1, b2::kEpiF32>(p, di, s) : launch_gemv_t<b2::kQ8, 2, b2::kEpiF32>(p, di, s);
  if (qt == b2::kQ4 && epi == b2::kEpiSwiglu)
    return nb == 1 ? launch_gemv_t<b2::kQ4, 1, b2::kEpiSwiglu>(p, di, s)
                   : launch_gemv_t<b2::kQ4, 2, b2::kEpiSwiglu>(p, di, s);
  return fail(B2_ERR_ARG, "unsupported gemv variant");
}

// --------------------------------------------------------------- dequant
int dequant_tiles(int qt, const uint8_t* tiles, int64_t n_tiles, uint16_t* out, void* stream) {
  DevInfo di;
  int st = device_info(&di);
  if (st != B2_OK) return st;
  if (!tiles || !out || n_tiles < 1) return fail(B2_ERR_ARG, "bad dequant arguments");
  if (!aligned(tiles, 16) || !aligned(out, 16)) return fail(B2_ERR_ALIGN, "tiles and out must be 16-byte aligned");
  const int grid = static_cast<int>(std::min<int64_t>(n_tiles, 8LL * di.sms));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out);
  if (qt == 0)
    b2::dequant_tiles_bf16_kernel<0><<<grid, 256, 0, s>>>(tiles, n_tiles, o);
  else
    b2::dequant_tiles_bf16_kernel<1><<<grid, 256, 0, s>>>(tiles, n_tiles, o);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "dequant launch");
  return B2_OK;
}

int dequant_matrix(int qt, const uint8_t* tiles, int n_t, int k_t, float* out, int64_t ld, void* stream) {
  DevInfo di;
  int st = device_info(&di);
  if (st != B2_OK) return st;
  if (!tiles || !out || n_t < 1 || k_t < 1 || ld < static_cast<int64_t>(k_t) * 256)
    return fail(B2_ERR_ARG, "bad dequant arguments");
  if (!aligned(tiles, 16) || !aligned(out, 4)) return fail(B2_ERR_ALIGN, "tiles must be 16-byte aligned");
  const int64_t n_tiles = static_cast<int64_t>(n_t) * k_t;
  const int grid = static_cast<int>(std::min<int64_t>(n_tiles, 8LL * di.sms));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (qt == 0)
    b2::dequant_matrix_f32_kernel<0><<<grid, 256, 0, s>>>(tiles, n_t, k_t, out, ld);
  else
    b2::dequant_matrix_f32_kernel<1><<<grid, 256, 0, s>>>(tiles, n_t, k_t, out, ld);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "dequant launch");
  return B2_OK;
}

// ------------------------------------------------------------- attention
struct AttnPlan {
  int n_splits;
  int split_len;
  int clustered;  // splits merge through a thread-block cluster (<= 16 CTAs), no workspace
  size_t ws_bytes;
};

// Context split: enough CTAs to cover the SMs.  When one layer's KV is small
// (decode-sized, < 64 MB) the splits of a (sequence, kv head) are capped at 16
// and merged inside a cluster -- one launch; larger contexts take more splits
// and merge in a second kernel through the caller's workspace.
// warps per attention CTA: 8 when the launch has at most one CTA per SM, else 4
// (three resident per SM; the tuning switch forces either)
bool attn_wide(long long n_cta, int split_len, int sms) {
  (void)split_len;
  if (tuning().attn_wide) return tuning().attn_wide == 1;
  return n_cta <= sms;
}

// wave_cap: unclustered launches use at most one wave of resident CTAs (fewer,
// longer splits); the cap only ever lowers the split count, never the scratch need
AttnPlan attn_plan(int batch, int hq, int hkv, int head_dim, int max_len, int sms, bool wave_cap) {
  AttnPlan pl;
  const int pairs = batch * hkv;
  const int target = 4 * sms;
  const int max_splits = (max_len + 63) / 64;
  const double kv_bytes = static_cast<double>(pairs) * max_len * head_dim * 4;
  int S = std::max(1, std::min(max_splits, (target + pairs - 1) / pairs));
  pl.clustered = 0;
  if (S > 1 && kv_bytes < 64.0 * (1 << 20)) {
    S = std::min(S, 16);
    pl.clustered = 1;
  }
  int sl = (max_len + S - 1) / S;
  sl = (sl + 63) / 64 * 64;
  S = (max_len + sl - 1) / sl;
  if (wave_cap) {
    // at most one wave of resident CTAs: 8-warp CTAs fit two per SM, 4-warp ones
    // three (the launcher's choice of warps, which itself depends on the split).
    // Clustered launches too: a tensor-parallel shard's few pairs (32 at TP = 8, B = 32)
    // in 16-CTA clusters made 512 CTAs on 296 slots, 21 us for 33.5 MB of K/V
    while (S > 1) {
      const long long n_cta = static_cast<long long>(S) * pairs;
      const bool wide = attn_wide(n_cta, sl, sms);
      const long long slots = static_cast<long long>(wide ? 2 : 3) * sms;
      if (n_cta <= slots) break;
      const int S2 = std::max(1, std::min(S - 1, static_cast<int>(slots / pairs)));
      sl = (max_len + S2 - 1) / S2;
      sl = (sl + 63) / 64 * 64;
      S = (max_len + sl - 1) / sl;
    }
    // a one-wave launch with few splits merges them in a cluster (DSMEM) rather than
    // through the workspace and a second kernel
    if (S > 1 && S <= 16) pl.clustered = 1;
  }
  pl.n_splits = S;
  pl.split_len = sl;
  if (S == 1) pl.clustered = 0;
  pl.ws_bytes = (S > 1 && !pl.clustered)
                    ? static_cast<size_t>(batch) * hkv * S * (hq / hkv) * (head_dim + 2) * sizeof(float)
                    : 0;
  return pl;
}

int attn_check(int batch, int hq, int hkv, int head_dim, int ctx_max, int max_len) {
  if (batch < 1 || hq < 1 || hkv < 1 || hq % hkv) return fail(B2_ERR_ARG, "bad head counts hq=%d hkv=%d", hq, hkv);
  if (hq / hkv > 8) return fail(B2_ERR_ARG, "GQA group %d > 8 is not supported", hq / hkv);
  if (head_dim != 64) return fail(B2_ERR_ARG, "head_dim %d: only 64 is built", head_dim);
  if (max_len < 1 || max_len > ctx_max) return fail(B2_ERR_ARG, "max_len %d outside 1..ctx_max %d", max_len, ctx_max);
  return B2_OK;
}

// ------------------------------------------ attention with static scratch
// Device scratch for b2_gqa_decode_static, for callers that cannot allocate
// device memory.  Every GPU that loads this library holds these 2 MiB until the
// process exits.  Host code must not pass the symbol itself to a kernel (on the
// host it is only a stand-in); its device address is looked up once per device.
constexpr size_t kAttnStaticScratchBytes = size_t(2) << 20;
static __device__ __align__(256) unsigned char g_attn_static_scratch[kAttnStaticScratchBytes];
static void* g_attn_static_ptr[64] = {};

// Device address of the static scratch on the current device (set up on first use).
int attn_static_scratch(void** out) {
  int d = -1;
  cudaError_t e = cudaGetDevice(&d);
  if (e != cudaSuccess || d < 0 || d >= 64) return fail(B2_ERR_NO_DEVICE, "no current CUDA device");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_attn_static_ptr[d]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_attn_static_scratch);
    if (e != cudaSuccess || !ptr) return cuda_fail(e, "cudaGetSymbolAddress(static attention scratch)");
    g_attn_static_ptr[d] = ptr;
  }
  *out = g_attn_static_ptr[d];
  return B2_OK;
}

// ------------------------------------------------- tcgen05 GEMM (large batch)
inline int tc_npad(int batch) { return (batch + 15) / 16 * 16; }
inline size_t tc_ws_bytes(int batch, int k_tiles) {
  const size_t img = static_cast<size_t>(tc_npad(batch)) * k_tiles * 256 * 2;
  return ((img + 255) & ~static_cast<size_t>(255)) + static_cast<size_t>(tc_npad(batch)) * sizeof(int);
}

// xf (with norm_w, eps): the fused RMSNorm input, fp32 rows [batch][ldx] in place of x
// qt: b2::kQ4, or b2::kQ8 (packed tiles and the fp32 form only)
int tc_gemm_common(int epi, const uint8_t* w0, const uint8_t* w1, int n_tile_rows, int k_tiles, const uint16_t* x,
                   int batch, int ldx, void* y, int ldy, int flags, void* workspace, size_t ws_bytes,
                   void* stream, const float* xf = nullptr, const uint16_t* norm_w = nullptr, float eps = 0.f,
                   int qt = b2::kQ4, const float* gu = nullptr, const SeamArgs* seam = nullptr) {
  DevInfo di;
  int st = device_info(&di);
  if (st != B2_OK) return st;
  if (xf) {
    if (!norm_w) return fail(B2_ERR_ARG, "null norm weight");
    if (!aligned(xf, 16) || (ldx % 4) || !aligned(norm_w, 16)) return fail(B2_ERR_ALIGN, "x/norm weight alignment");
    if (!(eps >= 0.f)) return fail(B2_ERR_ARG, "eps must be >= 0");
    x = reinterpret_cast<const uint16_t*>(xf);  // satisfies the checks below; the pre-pass reads xf
  }
  if (seam) {
    if (!xf) return fail(B2_ERR_ARG, "a pulled seam needs the _rmsnorm form");
    if (!seam->peers) return fail(B2_ERR_ARG, "null peers");
    if (seam->world < 1 || seam->world > b2::kPeerMaxRanks || seam->rank < 0 || seam->rank >= seam->world)
      return fail(B2_ERR_ARG, "rank %d of world %d", seam->rank, seam->world);
    if (seam->seam < 0 || seam->seam >= b2::kPeerMaxSeams) return fail(B2_ERR_ARG, "seam %d outside 0..%d", seam->seam, b2::kPeerMaxSeams - 1);
    if (seam->part_off < b2::kPeerCtlBytes || seam->part_off % 16) return fail(B2_ERR_ALIGN, "partial offset %lld", seam->part_off);
    if (seam->ld_part < k_tiles * 256 || seam->ld_part % 4) return fail(B2_ERR_ARG, "ld_part %d (K %d)", seam->ld_part, k_tiles * 256);
    if (k_tiles * 256 > b2::kPrepRegChunks * 256 * 8) return fail(B2_ERR_ARG, "a pulled seam takes K <= %d", b2::kPrepRegChunks * 2048);
  }
  if (gu) {  // SwiGLU input: fp32 rows [batch][ldx] holding g at column k and u at K + k
    if (xf || epi != b2::kTcEpiF32 || qt != b2::kQ4) return fail(B2_ERR_ARG, "SwiGLU input is for the plain q4 GEMM");
    if (!aligned(gu, 16) || (ldx % 4)) return fail(B2_ERR_ALIGN, "gu must be 16-byte aligned with ldx %% 4 == 0");
    if (ldx < 2 * k_tiles * 256) return fail(B2_ERR_ARG, "ldx %d < 2K %d (gate and up halves)", ldx, 2 * k_tiles * 256);
    x = reinterpret_cast<const uint16_t*>(gu);  // satisfies the checks below; the pre-pass reads gu
  }
  if (!w0 || !x || !y || (epi == b2::kTcEpiSwiglu && !w1)) return fail(B2_ERR_ARG, "null pointer argument");
  if (n_tile_rows < 1 || k_tiles < 1) return fail(B2_ERR_ARG, "bad tile shape %d x %d", n_tile_rows, k_tiles);
  if (batch < 1 || batch > b2::kTcMaxN) return fail(B2_ERR_ARG, "batch %d outside 1..%d", batch, b2::kTcMaxN);
  if (ldx < k_tiles * 256 || ldx % ((xf || gu) ? 4 : 8)) return fail(B2_ERR_ALIGN, "ldx %d: need >= K and aligned rows", ldx);
  if (ldy < n_tile_rows * 32) return fail(B2_ERR_ARG, "ldy %d < output rows %d", ldy, n_tile_rows * 32);
  if (!aligned(w0, 16) || (w1 && !aligned(w1, 16)) || !aligned(x, 16)) return fail(B2_ERR_ALIGN, "tiles and x must be 16-byte aligned");
  if (flags & ~(B2_GEMV_ACCUMULATE | B2_GEMV_PREFETCH | B2_GEMM_PACKED))
    return fail(B2_ERR_ARG, "unknown flags 0x%x", flags);
  if (epi == b2::kTcEpiSwiglu && (flags & B2_GEMV_ACCUMULATE)) return fail(B2_ERR_ARG, "SwiGLU output cannot accumulate");
  const bool packed = (flags & B2_GEMM_PACKED) != 0;
  if (qt == b2::kQ8 && (!packed || epi != b2::kTcEpiF32))
    return fail(B2_ERR_ARG, "the q8 tensor-core GEMM takes packed tiles (B2_GEMM_PACKED), fp32 form");
  const int tile_bytes = qt == b2::kQ8 ? b2::QTraits<b2::kQ8>::kTile : b2::QTraits<b2::kQ4>::kTile;
  const size_t need = tc_ws_bytes(batch, k_tiles);
  if (!workspace || ws_bytes < need) return fail(B2_ERR_WORKSPACE, "workspace of %zu bytes needed", need);
  if (!aligned(workspace, 256)) return fail(B2_ERR_ALIGN, "workspace must be 256-byte aligned");

  const int npad = tc_npad(batch);
  const int n_row_tiles = epi == b2::kTcEpiSwiglu ? (n_tile_rows + 1) / 2 : (n_tile_rows + 3) / 4;
  // SwiGLU cannot split K (its epilogue needs whole sums), so when the row tiles
  // leave SMs idle the token columns are split over CTAs instead (each CTA
  // dequantises the same tiles, runs 1/n of the MMAs and reads 1/n of x)
  int n_nsplit = 1;
  if (epi == b2::kTcEpiSwiglu)
    while (npad % (2 * n_nsplit * 16) == 0 && npad / (2 * n_nsplit) >= 64 && n_row_tiles * 2 * n_nsplit <= di.sms)
      n_nsplit *= 2;  // columns per CTA stay a multiple of 16 (MMA N) and >= 64
  const int ncta = npad / n_nsplit;
  const int budget = di.smem_optin - 1024;  // alignment slack for the 1024-byte operand atoms
  int raw_stages = 0, x_stages = 0, a_bufs = tuning().tc_abufs > 0 ? tuning().tc_abufs : 2;
  const int max_x = tuning().tc_xst > 0 ? tuning().tc_xst : 8;
  int smem = 0;
  if (packed) {
    // A lives in TMEM (two K-tile buffers): shared memory holds only the raw and x rings,
    // so the raw ring can run deeper
    // x stages are whole K-tiles: the deepest raw ring that leaves two of them
    a_bufs = 2;
    const int max_raw = tuning().tc_raw > 0 ? tuning().tc_raw : 6;
    const int max_xp = tuning().tc_xst > 0 ? tuning().tc_xst : 4;
    auto x_fit = [&](int rs) {
      return std::min(max_xp, (budget - b2::TcSmem(ncta, rs, 0, 0, 4, 4 * tile_bytes).total) / (4 * ncta * 128 + 16));
    };
    raw_stages = max_raw;
    while (raw_stages > 2 && x_fit(raw_stages) < std::min(2, max_xp)) --raw_stages;
    x_stages = x_fit(raw_stages);
    if (x_stages < 1) return fail(B2_ERR_UNSUPPORTED, "shared memory too small for the tensor-core GEMM");
    // more than half of an SM's shared memory: two of these CTAs (each allocating all
    // 512 TMEM columns) are never resident on one SM
    smem = std::max(b2::TcSmem(ncta, raw_stages, x_stages, 0, 4, 4 * tile_bytes).total + 1024,
                    di.smem_per_sm / 2 + 1024);
  } else {
    // pipeline: double-buffered A slices when they fit beside >= 2 raw and >= 2 x stages
    const int max_raw = tuning().tc_raw > 0 ? tuning().tc_raw : 3;
    for (; a_bufs >= 1 && x_stages < 2; --a_bufs) {
      for (raw_stages = max_raw; raw_stages >= 2; --raw_stages) {
        const b2::TcSmem base(ncta, raw_stages, 0, a_bufs);
        x_stages = std::min(max_x, (budget - base.total) / (ncta * 128 + 16));
        if (x_stages >= 2) break;
      }
    }
    ++a_bufs;  // undo the loop's last decrement
    if (x_stages < 2) return fail(B2_ERR_UNSUPPORTED, "shared memory too small for the tensor-core GEMM");
    smem = b2::TcSmem(ncta, raw_stages, x_stages, a_bufs).total + 1024;
  }
  // split-K (fp32 form only) so that small projections still occupy every SM, in
  // one wave: row tiles x splits <= SMs
  int n_splits = 1, kt_per_split = k_tiles;
  if (epi == b2::kTcEpiF32 && 2 * n_row_tiles <= di.sms) {
    n_splits = std::min(k_tiles, di.sms / n_row_tiles);
    kt_per_split = (k_tiles + n_splits - 1) / n_splits;
    n_splits = (k_tiles + kt_per_split - 1) / kt_per_split;
  }
  if (tuning().tc_splits > 0) {  // tuning experiments
    n_splits = std::min(k_tiles, tuning().tc_splits);
    kt_per_split = (k_tiles + n_splits - 1) / n_splits;
    n_splits = (k_tiles + kt_per_split - 1) / kt_per_split;
  }
  float* yzero = (n_splits > 1 && !(flags & B2_GEMV_ACCUMULATE)) ? static_cast<float*>(y) : nullptr;

  uint8_t* xsw = static_cast<uint8_t*>(workspace);
  int* xexp = reinterpret_cast<int*>(xsw + ((static_cast<size_t>(npad) * k_tiles * 512 + 255) & ~static_cast<size_t>(255)));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(npad, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_for(kPdlGemmPrep) ? 1 : 0;
  b2::TcPrep pp = {};
  pp.x = (xf || gu) ? nullptr : reinterpret_cast<const __nv_bfloat16*>(x);
  pp.xf = xf;
  pp.gu = gu;
  pp.gu_half = k_tiles * 256;
  if (seam) {
    pp.peers = seam->peers;
    pp.world = seam->world;
    pp.rank = seam->rank;
    pp.seam = seam->seam;
    pp.ld_part = seam->ld_part;
    pp.part_off = seam->part_off;
    pp.xf_out = const_cast<float*>(xf);
    pp.timeout_ns = g_peer_timeout_ns;
    const size_t stage_bytes = static_cast<size_t>(seam->world) * k_tiles * 256 * sizeof(float);
    if (stage_bytes <= kSeamStageMax) {
      static int prep_attr[64] = {0};
      int dev = 0;
      cudaGetDevice(&dev);
      if (!prep_attr[dev]) {
        cudaError_t ea = cudaFuncSetAttribute(b2::tc_x_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              static_cast<int>(kSeamStageMax));
        if (ea != cudaSuccess) return cuda_fail(ea, "cudaFuncSetAttribute(x pre-pass)");
        prep_attr[dev] = 1;
      }
      pp.stage = 1;
      cfg.dynamicSmemBytes = stage_bytes;
    }
  }
  pp.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w);
  pp.eps = eps;
  pp.ldx = ldx;
  pp.batch = batch;
  pp.k = k_tiles * 256;
  pp.npad = npad;
  pp.xsw = xsw;
  pp.xexp = xexp;
  pp.yzero = yzero;
  pp.ldy = ldy;
  pp.n_out = n_tile_rows * 32;
  pp.early = tuning().tc_prep_early;
  cudaError_t e = cudaLaunchKernelEx(&cfg, b2::tc_x_prep_kernel, pp);
  if (e != cudaSuccess) return cuda_fail(e, "x pre-pass launch");

  b2::TcParams p = {};
  p.w0 = w0;
  p.w1 = w1;
  p.n_tile_rows = n_tile_rows;
  p.k_tiles = k_tiles;
  p.xsw = xsw;
  p.xexp = xexp;
  p.batch = batch;
  p.npad = npad;
  p.raw_stages = raw_stages;
  p.pre_raw = tuning().tc_pre_raw > 0 ? std::min(raw_stages, tuning().tc_pre_raw) : raw_stages;
  p.x_stages = x_stages;
  p.a_bufs = a_bufs;
  p.y = y;
  p.ldy = ldy;
  p.accumulate = (flags & B2_GEMV_ACCUMULATE) ? 1 : 0;
  p.n_row_tiles = n_row_tiles;
  p.n_splits = n_splits;
  p.kt_per_split = kt_per_split;
  p.n_nsplit = n_nsplit;
  p.ncta = ncta;
  p.prefetch = (flags & B2_GEMV_PREFETCH) ? 1 : 0;
  if (seam) {  // the GEMM advances the seam its pre-pass consumed
    p.seam_peers = seam->peers;
    p.seam = seam->seam;
    p.seam_rank = seam->rank;
    p.seam_world = seam->world;
  }
  {
    const int nc = ncta <= 32 ? 32 : (ncta <= 64 ? 64 : (ncta <= 128 ? 128 : 256));
    // packed: two MMA issuers (two partials) while 2 x N columns fit the D region, and two
    // accumulator buffers while those fit too
    p.n_issuers = (packed && 2 * nc <= b2::kTcTmemACol) ? 2 : 1;
    p.d_bufs = (!packed || 2 * p.n_issuers * nc <= b2::kTcTmemACol) ? 2 : 1;
    // packed: a third A buffer when the accumulators leave 3 x 128 TMEM columns, so the
    // dequant of K-tile j + 2 need not wait for the MMAs of K-tile j (B2Q4NX_TC_ABUFS=2: two)
    if (packed)
      p.a_bufs = (p.d_bufs * p.n_issuers * nc + 3 * b2::kTcTmemABuf <= 512 && tuning().tc_abufs != 2) ? 3 : 2;
  }
  auto kernel = qt == b2::kQ8 ? b2::q4_gemm_tc_kernel<b2::kTcEpiF32, true, b2::kQ8>
                : epi == b2::kTcEpiSwiglu
                    ? (packed ? b2::q4_gemm_tc_kernel<b2::kTcEpiSwiglu, true> : b2::q4_gemm_tc_kernel<b2::kTcEpiSwiglu, false>)
                    : (packed ? b2::q4_gemm_tc_kernel<b2::kTcEpiF32, true> : b2::q4_gemm_tc_kernel<b2::kTcEpiF32, false>);
  static int attr_set[64][5] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int variant = qt == b2::kQ8 ? 4 : epi * 2 + (packed ? 1 : 0);
  if (!attr_set[dev][variant]) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, di.smem_optin);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(tensor-core GEMM)");
    attr_set[dev][variant] = 1;
  }
  cfg.gridDim = dim3(std::min(n_row_tiles * n_splits * n_nsplit, di.sms), 1, 1);
  cfg.blockDim = dim3(b2::kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.numAttrs = pdl_for(kPdlGemm) ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, kernel, p);
  if (e != cudaSuccess) return cuda_fail(e, "tensor-core GEMM launch");
  return B2_OK;
}

}  // namespace

// ------------------------------------------------------------------ C ABI
extern "C" {

int b2_version(void) { return (0 << 16) | (1 << 8) | 0; }

const char* b2_status_string(int status) {
  switch (status) {
    case B2_OK: return "ok";
    case B2_ERR_ARG: return "invalid argument";
    case B2_ERR_ALIGN: return "misaligned pointer or leading dimension";
    case B2_ERR_CUDA: return "CUDA error";
    case B2_ERR_NO_DEVICE: return "no CUDA device";
    case B2_ERR_UNSUPPORTED: return "unsupported device (needs sm_100)";
    case B2_ERR_WORKSPACE: return "workspace missing or too small";
    case B2_ERR_DEVICE: return "device-side error recorded";
    default: return "unknown status";
  }
}

const char* b2_last_error_message(void) { return g_msg; }

int b2_set_launch_options(int pdl) {
  g_pdl = pdl ? 1 : 0;
  return B2_OK;
}

int b2_read_device_error(int* code, void* stream) {
  if (!code) return fail(B2_ERR_ARG, "null code pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, b2::g_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  const int zero = 0;
  e = cudaMemcpyToSymbolAsync(b2::g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "clearing the device error word");
  *code = v;
  return B2_OK;
}

int b2_q4_gemv(const uint8_t* tiles, int n_tile_rows, int k_tiles, const uint16_t* x, int batch, int ldx,
               float* y, int ldy, int flags, void* stream) {
  return gemv_common(b2::kQ4, b2::kEpiF32, tiles, nullptr, n_tile_rows, k_tiles, x, batch, ldx, y, ldy, flags,
                     stream);
}

int b2_q8_gemv(const uint8_t* tiles, int n_tile_rows, int k_tiles, const uint16_t* x, int batch, int ldx,
               float* y, int ldy, int flags, void* stream) {
  return gemv_common(b2::kQ8, b2::kEpiF32, tiles, nullptr, n_tile_rows, k_tiles, x, batch, ldx, y, ldy, flags,
                     stream);
}

int b2_q4_swiglu_gemv(const uint8_t* gate, const uint8_t* up, int n_tile_rows, int k_tiles, const uint16_t* x,
                      int batch, int ldx, uint16_t* h, int ldh, int flags, void* stream) {
  return gemv_common(b2::kQ4, b2::kEpiSwiglu, gate, up, n_tile_rows, k_tiles, x, batch, ldx, h, ldh, flags,
                     stream);
}

int b2_gqa_decode_workspace_size(int batch, int n_q_heads, int n_kv_heads, int head_dim, int max_len,
                                 size_t* bytes) {
  DevInfo di;
  int st = device_info(&di);
  if (st != B2_OK) return st;
  if (!bytes) return fail(B2_ERR_ARG, "null bytes pointer");
  st = attn_check(batch, n_q_heads, n_kv_heads, head_dim, max_len, max_len);
  if (st != B2_OK) return st;
  *bytes = attn_plan(batch, n_q_heads, n_kv_heads, head_dim, max_len, di.sms, tuning().attn_wave != 0).ws_bytes;
  return B2_OK;
}

static int gqa_decode_impl(const float* q, const float* k_new, const float* v_new, int ld_new, uint16_t* k_cache,
                           uint16_t* v_cache, const int32_t* pos, int batch, int n_q_heads, int n_kv_heads,
                           int head_dim, int ctx_max, int max_len, float theta, float scale, uint16_t* out, int ldo,
                           void* workspace, size_t workspace_bytes, int flags, void* stream, bool wave_cap) {
  DevInfo di;
  int st = device_info(&di);
  if (st != B2_OK) return st;
  st = attn_check(batch, n_q_heads, n_kv_heads, head_dim, ctx_max, max_len);
  if (st != B2_OK) return st;
  if (!q || !k_new || !v_new || !k_cache || !v_cache || !pos || !out) return fail(B2_ERR_ARG, "null pointer argument");
  if (ld_new < n_q_heads * head_dim) return fail(B2_ERR_ARG, "ld_new %d < Hq*D", ld_new);
  if (ldo < n_q_heads * head_dim) return fail(B2_ERR_ARG, "ldo %d < Hq*D", ldo);
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16)) return fail(B2_ERR_ALIGN, "KV caches must be 16-byte aligned");
  if ((flags & ~(B2_ATTN_NO_APPEND | B2_ATTN_NO_ROPE | B2_ATTN_OUT_F32 | B2_ATTN_PREFETCH_KV)) != 0)
    return fail(B2_ERR_ARG, "unknown flags 0x%x", flags);
  const AttnPlan pl = attn_plan(batch, n_q_heads, n_kv_heads, head_dim, max_len, di.sms, wave_cap);
  if (pl.n_splits > 1 && (!workspace || workspace_bytes < pl.ws_bytes))
    return fail(B2_ERR_WORKSPACE, "workspace of %zu bytes needed (b2_gqa_decode_workspace_size)", pl.ws_bytes);
  if (pl.n_splits > 65535) return fail(B2_ERR_ARG, "too many context splits");

  b2::AttnParams p = {};
  p.q = q;
  p.k_new = k_new;
  p.v_new = v_new;
  p.ld_new = ld_new;
  p.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache);
  p.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache);
  p.pos = pos;
  p.batch = batch;
  p.hq = n_q_heads;
  p.hkv = n_kv_heads;
  p.ctx_max = ctx_max;
  p.theta = theta;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.part = static_cast<float*>(workspace);
  p.n_splits = pl.n_splits;
  p.split_len = pl.split_len;
  p.append = (flags & B2_ATTN_NO_APPEND) ? 0 : 1;
  p.rope = (flags & B2_ATTN_NO_ROPE) ? 0 : 1;
  p.out_f32 = (flags & B2_ATTN_OUT_F32) ? 1 : 0;
  p.clustered = pl.clustered;
  p.prefetch_kv = (flags & B2_ATTN_PREFETCH_KV) ? 1 : 0;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long n_cta = static_cast<long long>(pl.n_splits) * n_kv_heads * batch;
  const bool wide = attn_wide(n_cta, pl.split_len, di.sms);
  auto kernel = wide ? b2::gqa_decode_kernel<64, 8> : b2::gqa_decode_kernel<64, 4>;
  static int attr_set[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    for (auto kf : {b2::gqa_decode_kernel<64, 8>, b2::gqa_decode_kernel<64, 4>}) {
      cudaError_t e = cudaFuncSetAttribute(kf, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      // the cluster merge buffer (<= 16 splits x 8 heads x 66 floats) and the 64 KB of K/V rings
      if (e == cudaSuccess) e = cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, 128 * 1024);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(attention)");
    }
    attr_set[dev] = 1;
  }
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl_for(kPdlAttention)) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (pl.clustered) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = pl.n_splits;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.n_splits, n_kv_heads, batch);
  cfg.blockDim = dim3(wide ? 256 : 128, 1, 1);
  {
    const size_t gather = pl.clustered ? pl.n_splits * (n_q_heads / n_kv_heads) * (head_dim + 2) * sizeof(float) : 0;
    cfg.dynamicSmemBytes = ((gather + 127) & ~static_cast<size_t>(127)) + b2::attn_ring_bytes(wide ? 8 : 4);
  }
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = na;  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, p);
  if (e != cudaSuccess) return cuda_fail(e, "attention launch");
  if (pl.n_splits > 1 && !pl.clustered) {
    cfg.numAttrs = pdl_for(kPdlAttention) ? 1 : 0;  // the combine kernel is not clustered
    cfg.gridDim = dim3(n_q_heads, batch, 1);
    cfg.blockDim = dim3(64, 1, 1);
    cfg.dynamicSmemBytes = 0;
    e = cudaLaunchKernelEx(&cfg, b2::gqa_combine_kernel<64>, p);
    if (e != cudaSuccess) return cuda_fail(e, "attention combine launch");
  }
  return B2_OK;
}

int b2_gqa_decode(const float* q, const float* k_new, const float* v_new, int ld_new, uint16_t* k_cache,
                  uint16_t* v_cache, const int32_t* pos, int batch, int n_q_heads, int n_kv_heads, int head_dim,
                  int ctx_max, int max_len, float theta, float scale, uint16_t* out, int ldo, void* workspace,
                  size_t workspace_bytes, int flags, void* stream) {
  return gqa_decode_impl(q, k_new, v_new, ld_new, k_cache, v_cache, pos, batch, n_q_heads, n_kv_heads, head_dim,
                         ctx_max, max_len, theta, scale, out, ldo, workspace, workspace_bytes, flags, stream,
                         tuning().attn_wave != 0);
}

int b2_gqa_decode_static(const float* q, const float* k_new, const float* v_new, int ld_new, uint16_t* k_cache,
                         uint16_t* v_cache, const int32_t* pos, int batch, int n_q_heads, int n_kv_heads,
                         int head_dim, int ctx_max, int max_len, float theta, float scale, uint16_t* out, int ldo,
                         int flags, void* stream) {
  DevInfo di;
  int st = device_info(&di);
  if (st != B2_OK) return st;
  st = attn_check(batch, n_q_heads, n_kv_heads, head_dim, ctx_max, max_len);
  if (st != B2_OK) return st;
  // the same plan as b2_gqa_decode, so b2_gqa_decode_workspace_size() is exactly
  // this call's scratch need and the limit below can be checked in advance
  const bool wave_cap = tuning().attn_wave != 0;
  const AttnPlan pl = attn_plan(batch, n_q_heads, n_kv_heads, head_dim, max_len, di.sms, wave_cap);
  if (pl.ws_bytes > kAttnStaticScratchBytes)
    return fail(B2_ERR_WORKSPACE,
                "this call needs %zu bytes of scratch, more than the %zu-byte static scratch of "
                "b2_gqa_decode_static; call b2_gqa_decode with a workspace instead",
                pl.ws_bytes, kAttnStaticScratchBytes);
  void* ws = nullptr;
  st = attn_static_scratch(&ws);
  if (st != B2_OK) return st;
  return gqa_decode_impl(q, k_new, v_new, ld_new, k_cache, v_cache, pos, batch, n_q_heads, n_kv_heads, head_dim,
                         ctx_max, max_len, theta, scale, out, ldo, ws, kAttnStaticScratchBytes, flags, stream,
                         wave_cap);
}

// ------------------------------------------------- tensor-parallel exchanges
namespace {
int xchg_check(void* const* peers, int world, int rank, const void* src, int rows, int cols, int ld_src,
               long long dst_offset) {
  if (!peers || !src) return fail(B2_ERR_ARG, "null pointer argument");
  if (world < 1 || world > b2::kPeerMaxRanks || rank < 0 || rank >= world)
    return fail(B2_ERR_ARG, "rank %d of world %d", rank, world);
  if (rows < 1 || cols < 1 || ld_src < cols) return fail(B2_ERR_ARG, "bad block %dx%d (ld %d)", rows, cols, ld_src);
  if (dst_offset < b2::kPeerCtlBytes) return fail(B2_ERR_ARG, "dst_offset inside the control words");
  static_assert(b2::kPeerCtlBytes == B2_PEER_CTL_BYTES, "control block size");
  static_assert(b2::kPeerMaxRanks == B2_PEER_MAX_RANKS, "rank limit");
  return B2_OK;
}

// Units (16-byte vectors when every row start and the width allow, else elements) and
// CTAs: one unit per thread up to kPeerMaxChunks CTAs, more units per thread beyond.
void xchg_plan(b2::XchgParams& p, int elem_bytes, bool vec_ok) {
  const bool vec = vec_ok && (static_cast<long long>(p.cols) * elem_bytes) % 16 == 0 &&
                   (static_cast<long long>(p.ld_src) * elem_bytes) % 16 == 0 && aligned(p.src, 16);
  p.vec = vec ? 1 : 0;
  const long long units = static_cast<long long>(p.rows) * (vec ? p.cols * elem_bytes / 16 : p.cols);
  const long long c = (units + b2::kXchgThreads - 1) / b2::kXchgThreads;
  p.chunks = static_cast<int>(std::max(1LL, std::min<long long>(c, b2::kPeerMaxChunks)));
}

int xchg_launch(const void* kernel, const b2::XchgParams& p, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.chunks, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_for(kPdlExchange) ? 1 : 0;
  void* args[] = {const_cast<b2::XchgParams*>(&p)};
  cudaError_t e = cudaLaunchKernelExC(&cfg, kernel, args);
  if (e != cudaSuccess) return cuda_fail(e, "exchange launch");
  return B2_OK;
}
}  // namespace

int b2_peer_alloc(size_t bytes, void** ptr, uint8_t* ipc_handle) {
  DevInfo di;
  int st = device_info(&di);
  if (st != B2_OK) return st;
  if (!ptr || !ipc_handle || bytes < static_cast<size_t>(b2::kPeerCtlBytes))
    return fail(B2_ERR_ARG, "peer region needs >= %d bytes and out pointers", b2::kPeerCtlBytes);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(peer region)");
  e = cudaMemset(p, 0, b2::kPeerCtlBytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "peer region set-up");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == B2_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return B2_OK;
}

int b2_peer_free(void* ptr) {
  if (!ptr) return B2_OK;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? B2_OK : cuda_fail(e, "cudaFree(peer region)");
}

int b2_peer_open(const uint8_t* ipc_handle, void** ptr) {
  if (!ipc_handle || !ptr) return fail(B2_ERR_ARG, "null pointer argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? B2_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

int b2_peer_close(void* ptr) {
  if (!ptr) return B2_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? B2_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int b2_set_peer_timeout_ms(int ms) {
  if (ms < 1) return fail(B2_ERR_ARG, "timeout must be >= 1 ms");
  g_peer_timeout_ns = static_cast<unsigned long long>(ms) * 1000000ull;
  return B2_OK;
}

int b2_tp_gather(void* const* peers, int world, int rank, const void* src, int rows, int cols, int ld_src,
                 int elem_bytes, long long dst_offset, int ld_dst, const float* add_base, void* stream) {
  DevInfo di;
  int st = device_info(&di);
  if (st != B2_OK) return st;
  st = xchg_check(peers, world, rank, src, rows, cols, ld_src, dst_offset);
  if (st != B2_OK) return st;
  if (elem_bytes != 2 && elem_bytes != 4) return fail(B2_ERR_ARG, "elem_bytes %d (2 or 4)", elem_bytes);
  if (add_base && elem_bytes != 4) return fail(B2_ERR_ARG, "add_base needs fp32 elements");
  if (ld_dst < cols * world) return fail(B2_ERR_ARG, "ld_dst %d < cols*world %d", ld_dst, cols * world);
  if (dst_offset % elem_bytes) return fail(B2_ERR_ALIGN, "dst_offset misaligned");
  b2::XchgParams p = {};
  p.peers = peers;
  p.world = world;
  p.rank = rank;
  p.src = src;
  p.rows = rows;
  p.cols = cols;
  p.ld_src = ld_src;
  p.dst_offset = dst_offset;
  p.ld_dst = ld_dst;
  p.add_base = add_base;
  // 16-byte units need every destination row start aligned too (region bases are
  // 256-byte aligned allocations), and the add base's rows
  const bool vec_ok = dst_offset % 16 == 0 && (static_cast<long long>(ld_dst) * elem_bytes) % 16 == 0 &&
                      (static_cast<long long>(rank) * cols * elem_bytes) % 16 == 0 && (!add_base || aligned(add_base, 16));
  xchg_plan(p, elem_bytes, vec_ok);
  p.timeout_ns = g_peer_timeout_ns;
  const void* k = elem_bytes == 2 ? reinterpret_cast<const void*>(b2::tp_gather_kernel<uint16_t>)
                                  : reinterpret_cast<const void*>(b2::tp_gather_kernel<uint32_t>);
  return xchg_launch(k, p, static_cast<cudaStream_t>(stream));
}

int b2_tp_allreduce(void* const* peers, int world, int rank, const float* src, int rows, int cols, int ld_src,
                    long long slots_offset, float* y, int ldy, void* stream) {
  DevInfo di;
  int st = device_info(&di);
  if (st != B2_OK) return st;
  st = xchg_check(peers, world, rank, src, rows, cols, ld_src, slots_offset);
  if (st != B2_OK) return st;
  if (!y || ldy < cols) return fail(B2_ERR_ARG, "bad output (ldy %d < cols %d)", ldy, cols);
  if (slots_offset % 16) return fail(B2_ERR_ALIGN, "slots_offset must be 16-byte aligned");
  b2::XchgParams p = {};
  p.peers = peers;
  p.world = world;
  p.rank = rank;
  p.src = src;
  p.rows = rows;
  p.cols = cols;
  p.ld_src = ld_src;
  p.dst_offset = slots_offset;
  p.ld_dst = cols;
  p.y = y;
  p.ldy = ldy;
  // slots rows are cols floats apart; y rows ldy floats apart
  const bool vec_ok = (static_cast<long long>(rows) * cols * 4) % 16 == 0 && ldy % 4 == 0 && aligned(y, 16);
  xchg_plan(p, 4, vec_ok);
  p.timeout_ns = g_peer_timeout_ns;
  return xchg_launch(reinterpret_cast<const void*>(b2::tp_allreduce_kernel), p, static_cast<cudaStream_t>(stream));
}

int b2_rmsnorm(const void* x, int x_is_f32, int ldx, const uint16_t* w, float eps, int batch, int n, uint16_t* y,
               int ldy, void* stream) {
  DevInfo di;
  int st = device_info(&di);
  if (st != B2_OK) return st;
  if (!x || !w || !y) return fail(B2_ERR_ARG, "null pointer argument");
  if (batch < 1 || n < 1 || ldx < n || ldy < n) return fail(B2_ERR_ARG, "bad rmsnorm shape");
  if (!(eps >= 0.f)) return fail(B2_ERR_ARG, "eps must be >= 0");
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(batch, 1, 1);
  cfg.blockDim = dim3(b2::kNormThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = pdl_for(kPdlOther) ? 1 : 0;
  const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(w);
  __nv_bfloat16* yb = reinterpret_cast<__nv_bfloat16*>(y);
  cudaError_t e = x_is_f32 ? cudaLaunchKernelEx(&cfg, b2::rmsnorm_kernel<true>, x, ldx, wb, eps, n, yb, ldy)
                           : cudaLaunchKernelEx(&cfg, b2::rmsnorm_kernel<false>, x, ldx, wb, eps, n, yb, ldy);
  if (e != cudaSuccess) return cuda_fail(e, "rmsnorm launch");
  return B2_OK;
}

// splits of the gated attention: one per (kv head, sequence) when those fill the SMs,
// else enough for about two CTAs per SM, each at least tuning().gated_min_split keys
static void gated_attn_plan(int batch, int nkv, int max_len, int sms, int* n_splits, int* split_len) {
  const long long pairs = (long long)batch * nkv;
  int S = 1;
  const int mk = tuning().gated_min_split;
  if (pairs < sms) S = (int)std::max(1LL, std::min<long long>((2LL * sms + pairs - 1) / pairs, (max_len + mk - 1) / mk));
  int sl = (max_len + S - 1) / S;
  sl = (sl + 63) / 64 * 64;
  *split_len = sl;
  *n_splits = (max_len + sl - 1) / sl;
}

static size_t gated_attn_ws_bytes(int batch, int nq, int nkv, int n_splits) {
  return n_splits > 1 ? (size_t)batch * nq * n_splits * (b2::kGaD + 2) * sizeof(float) : 0;
}

int b2_gated_attn_decode_workspace_size(int batch, int n_q_heads, int n_kv_heads, int head_dim, int max_len,
                                        size_t* bytes) {
  if (!bytes) return fail(B2_ERR_ARG, "null bytes");
  if (batch < 1 || n_kv_heads < 1 || n_q_heads < n_kv_heads || max_len < 1 || head_dim != b2::kGaD)
    return fail(B2_ERR_ARG, "bad gated attention shape");
  DevInfo di;
  int st = device_info(&di);
  if (st != B2_OK) return st;
  int S, sl;
  gated_attn_plan(batch, n_kv_heads, max_len, di.sms, &S, &sl);
  *bytes = gated_attn_ws_bytes(batch, n_q_heads, n_kv_heads, S);
  return B2_OK;
}

int b2_gated_attn_decode(const float* qg, int ld_qg, const float* k_new, const float* v_new, int ld_kv,
                         const float* q_norm_w, const float* k_norm_w, const float* inv_freq, int rot_dim,
                         uint16_t* k_cache, uint16_t* v_cache, const int32_t* pos, int batch, int n_q_heads,
                         int n_kv_heads, int head_dim, int ctx_max, int max_len, float eps, void* out, int ldo,
                         int flags, void* workspace, size_t workspace_bytes, void* stream) {
  DevInfo di;
  int st = device_info(&di);
  if (st != B2_OK) return st;
  if (!qg || !k_new || !v_new || !q_norm_w || !k_norm_w || !inv_freq || !k_cache || !v_cache || !pos || !out)
    return fail(B2_ERR_ARG, "null pointer argument");
  if (head_dim != b2::kGaD) return fail(B2_ERR_ARG, "head_dim %d: only 256 is built", head_dim);
  if (batch < 1 || batch > 65535 || n_kv_heads < 1 || n_kv_heads > 65535 || n_q_heads % n_kv_heads)
    return fail(B2_ERR_ARG, "bad gated attention heads (q %d, kv %d)", n_q_heads, n_kv_heads);
  const int G = n_q_heads / n_kv_heads;
  if (G != 1 && G != 2 && G != 4) return fail(B2_ERR_ARG, "q heads per kv head %d: 1, 2 or 4 are built", G);
  if (rot_dim < 2 || rot_dim > head_dim || rot_dim % 2) return fail(B2_ERR_ARG, "bad rotary dim %d", rot_dim);
  if (ctx_max < 1 || max_len < 1 || max_len > ctx_max) return fail(B2_ERR_ARG, "need 1 <= max_len <= ctx_max");
  if (ld_qg < n_q_heads * 2 * head_dim || ld_kv < n_kv_heads * head_dim || ldo < n_q_heads * head_dim)
    return fail(B2_ERR_ARG, "leading dimension too small");
  if (!(eps >= 0.f)) return fail(B2_ERR_ARG, "eps must be >= 0");
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15)
    return fail(B2_ERR_ALIGN, "k_cache and v_cache must be 16-byte aligned");
  int S, sl;
  gated_attn_plan(batch, n_kv_heads, max_len, di.sms, &S, &sl);
  const size_t need = gated_attn_ws_bytes(batch, n_q_heads, n_kv_heads, S);
  if (need && (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15)))
    return fail(B2_ERR_WORKSPACE, "gated attention needs %zu bytes of 16-byte aligned workspace", need);
  b2::GatedAttnParams p = {};
  p.qg = qg;
  p.k_new = k_new;
  p.v_new = v_new;
  p.q_norm_w = q_norm_w;
  p.k_norm_w = k_norm_w;
  p.inv_freq = inv_freq;
  p.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache);
  p.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache);
  p.pos = pos;
  p.out = out;
  p.part = static_cast<float*>(workspace);
  p.ld_qg = ld_qg;
  p.ld_kv = ld_kv;
  p.ldo = ldo;
  p.rot_half = rot_dim / 2;
  p.ctx_max = ctx_max;
  p.max_len = max_len;
  p.nq = n_q_heads;
  p.nkv = n_kv_heads;
  p.n_splits = S;
  p.split_len = sl;
  p.eps = eps;
  p.out_f32 = (flags & B2_GATED_OUT_F32) ? 1 : 0;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S, n_kv_heads, batch);
  cfg.blockDim = dim3(b2::kGaThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = pdl_for(kPdlOther) ? 1 : 0;
  cudaError_t e = G == 4   ? cudaLaunchKernelEx(&cfg, b2::gated_attn_kernel<4>, p)
                  : G == 2 ? cudaLaunchKernelEx(&cfg, b2::gated_attn_kernel<2>, p)
                           : cudaLaunchKernelEx(&cfg, b2::gated_attn_kernel<1>, p);
  if (e != cudaSuccess) return cuda_fail(e, "gated attention launch");
  if (S > 1) {
    cfg.gridDim = dim3(n_q_heads, batch, 1);
    e = cudaLaunchKernelEx(&cfg, b2::gated_attn_combine_kernel, p);
    if (e != cudaSuccess) return cuda_fail(e, "gated attention combine launch");
  }
  return B2_OK;
}

int b2_gated_delta_step(const float* qkv, int ld_qkv, const float* z, int ld_z, const float* b, const float* a,
                        int ld_ab, float* conv_state, const float* conv_w, const float* A_log, const float* dt_bias,
                        const float* norm_w, float* state, int batch, int n_k_heads, int n_v_heads, int head_dim,
                        float eps, void* out, int ldo, int flags, void* stream) {
  DevInfo di;
  int st = device_info(&di);
  if (st != B2_OK) return st;
  if (!qkv || !z || !b || !a || !conv_state || !conv_w || !A_log || !dt_bias || !norm_w || !state || !out)
    return fail(B2_ERR_ARG, "null pointer argument");
  if (head_dim != b2::kDeltaHeadDim) return fail(B2_ERR_ARG, "head_dim %d: only 128 is built", head_dim);
  if (batch < 1 || batch > 65535 || n_k_heads < 1 || n_v_heads < n_k_heads || n_v_heads % n_k_heads)
    return fail(B2_ERR_ARG, "bad gated delta shape (batch %d, k heads %d, v heads %d)", batch, n_k_heads,
                n_v_heads);
  const int ratio = n_v_heads / n_k_heads;
  if (ratio > 8) return fail(B2_ERR_ARG, "v heads per k head %d > 8", ratio);
  const long long conv_dim = 2LL * n_k_heads * head_dim + (long long)n_v_heads * head_dim;
  if (ld_qkv < conv_dim || ld_z < n_v_heads * head_dim || ld_ab < n_v_heads || ldo < n_v_heads * head_dim)
    return fail(B2_ERR_ARG, "leading dimension too small");
  if (!(eps >= 0.f)) return fail(B2_ERR_ARG, "eps must be >= 0");
  if ((reinterpret_cast<uintptr_t>(conv_state) | reinterpret_cast<uintptr_t>(conv_w) |
       reinterpret_cast<uintptr_t>(state)) & 15)
    return fail(B2_ERR_ALIGN, "conv_state, conv_w and state must be 16-byte aligned");
  b2::DeltaParams p = {};
  p.qkv = qkv;
  p.z = z;
  p.b = b;
  p.a = a;
  p.conv_state = conv_state;
  p.conv_w = conv_w;
  p.A_log = A_log;
  p.dt_bias = dt_bias;
  p.norm_w = norm_w;
  p.state = state;
  p.out = out;
  p.ld_qkv = ld_qkv;
  p.ld_z = ld_z;
  p.ld_ab = ld_ab;
  p.ldo = ldo;
  p.nk = n_k_heads;
  p.nv = n_v_heads;
  p.eps = eps;
  p.out_f32 = (flags & B2_DELTA_OUT_F32) ? 1 : 0;
  p.prefetch_state = (flags & B2_DELTA_PREFETCH_STATE) ? 1 : 0;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl_for(kPdlOther)) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (ratio > 1) {  // the v heads of one k head share its q/k conv state
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = ratio;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_v_heads, batch, 1);
  cfg.blockDim = dim3(b2::kDeltaThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, b2::gated_delta_step_kernel, p);
  if (e != cudaSuccess) return cuda_fail(e, "gated delta launch");
  return B2_OK;
}

int b2_q4_gemv_rmsnorm(const uint8_t* tiles, int n_tile_rows, int k_tiles, const float* x, int batch, int ldx,
                       const uint16_t* norm_w, float eps, float* y, int ldy, int flags, void* stream) {
  return gemv_common(b2::kQ4, b2::kEpiF32, tiles, nullptr, n_tile_rows, k_tiles, nullptr, batch, ldx, y, ldy,
                     flags, stream, x, norm_w, eps);
}

int b2_q8_gemv_rmsnorm(const uint8_t* tiles, int n_tile_rows, int k_tiles, const float* x, int batch, int ldx,
                       const uint16_t* norm_w, float eps, float* y, int ldy, int flags, void* stream) {
  return gemv_common(b2::kQ8, b2::kEpiF32, tiles, nullptr, n_tile_rows, k_tiles, nullptr, batch, ldx, y, ldy,
                     flags, stream, x, norm_w, eps);
}

int b2_q4_swiglu_gemv_rmsnorm(const uint8_t* gate, const uint8_t* up, int n_tile_rows, int k_tiles, const float* x,
                              int batch, int ldx, const uint16_t* norm_w, float eps, uint16_t* h, int ldh,
                              int flags, void* stream) {
  return gemv_common(b2::kQ4, b2::kEpiSwiglu, gate, up, n_tile_rows, k_tiles, nullptr, batch, ldx, h, ldh, flags,
                     stream, x, norm_w, eps);
}

int b2_q4_gemm_workspace_size(int batch, int k_tiles, size_t* bytes) {
  if (!bytes) return fail(B2_ERR_ARG, "null bytes pointer");
  if (batch < 1 || batch > b2::kTcMaxN || k_tiles < 1) return fail(B2_ERR_ARG, "bad batch %d / k_tiles %d", batch, k_tiles);
  *bytes = tc_ws_bytes(batch, k_tiles);
  return B2_OK;
}

int b2_q4_gemm(const uint8_t* tiles, int n_tile_rows, int k_tiles, const uint16_t* x, int batch, int ldx, float* y,
               int ldy, int flags, void* workspace, size_t workspace_bytes, void* stream) {
  return tc_gemm_common(b2::kTcEpiF32, tiles, nullptr, n_tile_rows, k_tiles, x, batch, ldx, y, ldy, flags,
                        workspace, workspace_bytes, stream);
}

int b2_q4_swiglu_gemm(const uint8_t* gate, const uint8_t* up, int n_tile_rows, int k_tiles, const uint16_t* x,
                      int batch, int ldx, uint16_t* h, int ldh, int flags, void* workspace, size_t workspace_bytes,
                      void* stream) {
  return tc_gemm_common(b2::kTcEpiSwiglu, gate, up, n_tile_rows, k_tiles, x, batch, ldx, h, ldh, flags, workspace,
                        workspace_bytes, stream);
}

int b2_q4_gemm_swiglu_in(const uint8_t* tiles, int n_tile_rows, int k_tiles, const float* gu, int batch, int ldgu,
                          float* y, int ldy, int flags, void* workspace, size_t workspace_bytes, void* stream) {
  return tc_gemm_common(b2::kTcEpiF32, tiles, nullptr, n_tile_rows, k_tiles, nullptr, batch, ldgu, y, ldy, flags,
                        workspace, workspace_bytes, stream, nullptr, nullptr, 0.f, b2::kQ4, gu);
}

int b2_q4_gemm_rmsnorm(const uint8_t* tiles, int n_tile_rows, int k_tiles, const float* x, int batch, int ldx,
                       const uint16_t* norm_w, float eps, float* y, int ldy, int flags, void* workspace,
                       size_t workspace_bytes, void* stream) {
  return tc_gemm_common(b2::kTcEpiF32, tiles, nullptr, n_tile_rows, k_tiles, nullptr, batch, ldx, y, ldy, flags,
                        workspace, workspace_bytes, stream, x, norm_w, eps);
}

int b2_q4_swiglu_gemm_rmsnorm(const uint8_t* gate, const uint8_t* up, int n_tile_rows, int k_tiles, const float* x,
                              int batch, int ldx, const uint16_t* norm_w, float eps, uint16_t* h, int ldh, int flags,
                              void* workspace, size_t workspace_bytes, void* stream) {
  return tc_gemm_common(b2::kTcEpiSwiglu, gate, up, n_tile_rows, k_tiles, nullptr, batch, ldx, h, ldh, flags,
                        workspace, workspace_bytes, stream, x, norm_w, eps);
}

namespace {
int gemm_pack(int qt, const uint8_t* tiles, int n_tile_rows, int k_tiles, uint8_t* packed, void* stream) {
  DevInfo di;
  int st = device_info(&di);
  if (st != B2_OK) return st;
  if (!tiles || !packed || n_tile_rows < 1 || k_tiles < 1) return fail(B2_ERR_ARG, "bad pack arguments");
  const int64_t n_tiles = static_cast<int64_t>(n_tile_rows) * k_tiles;
  if (!aligned(tiles, 16) || !aligned(packed, 16)) return fail(B2_ERR_ALIGN, "tiles and packed must be 16-byte aligned");
  const int64_t tb = qt == b2::kQ8 ? b2::QTraits<b2::kQ8>::kTile : b2::QTraits<b2::kQ4>::kTile;
  if (tiles < packed + n_tiles * tb && packed < tiles + n_tiles * tb) return fail(B2_ERR_ARG, "packing cannot run in place");
  const int grid = static_cast<int>(std::min<int64_t>(n_tiles, 16LL * di.sms));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (qt == b2::kQ8)
    b2::tc_pack8_kernel<<<grid, 256, 0, s>>>(tiles, packed, n_tile_rows, k_tiles);
  else
    b2::tc_pack_kernel<<<grid, 256, 0, s>>>(tiles, packed, n_tile_rows, k_tiles);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? B2_OK : cuda_fail(e, "pack launch");
}
}  // namespace

int b2_q4_gemm_pack(const uint8_t* tiles, int n_tile_rows, int k_tiles, uint8_t* packed, void* stream) {
  return gemm_pack(b2::kQ4, tiles, n_tile_rows, k_tiles, packed, stream);
}
int b2_q8_gemm_pack(const uint8_t* tiles, int n_tile_rows, int k_tiles, uint8_t* packed, void* stream) {
  return gemm_pack(b2::kQ8, tiles, n_tile_rows, k_tiles, packed, stream);
}

int b2_q8_gemm(const uint8_t* tiles, int n_tile_rows, int k_tiles, const uint16_t* x, int batch, int ldx, float* y,
               int ldy, int flags, void* workspace, size_t workspace_bytes, void* stream) {
  return tc_gemm_common(b2::kTcEpiF32, tiles, nullptr, n_tile_rows, k_tiles, x, batch, ldx, y, ldy, flags, workspace,
                        workspace_bytes, stream, nullptr, nullptr, 0.f, b2::kQ8);
}

int b2_q8_gemm_rmsnorm(const uint8_t* tiles, int n_tile_rows, int k_tiles, const float* x, int batch, int ldx,
                       const uint16_t* norm_w, float eps, float* y, int ldy, int flags, void* workspace,
                       size_t workspace_bytes, void* stream) {
  return tc_gemm_common(b2::kTcEpiF32, tiles, nullptr, n_tile_rows, k_tiles, nullptr, batch, ldx, y, ldy, flags,
                        workspace, workspace_bytes, stream, x, norm_w, eps, b2::kQ8);
}

int b2_gemm_rmsnorm_seam(int form, const uint8_t* w0, const uint8_t* w1, int n_tile_rows, int k_tiles, float* x,
                         int batch, int ldx, const uint16_t* norm_w, float eps, void* y, int ldy, int flags,
                         void* workspace, size_t workspace_bytes, void* const* peers, int world, int rank,
                         long long part_offset, int ld_part, int seam, void* stream) {
  const SeamArgs sa = {peers, world, rank, seam, ld_part, part_offset};
  switch (form) {
    case B2_SEAM_Q4_F32:
      return tc_gemm_common(b2::kTcEpiF32, w0, nullptr, n_tile_rows, k_tiles, nullptr, batch, ldx, y, ldy, flags,
                            workspace, workspace_bytes, stream, x, norm_w, eps, b2::kQ4, nullptr, &sa);
    case B2_SEAM_Q4_SWIGLU:
      return tc_gemm_common(b2::kTcEpiSwiglu, w0, w1, n_tile_rows, k_tiles, nullptr, batch, ldx, y, ldy, flags,
                            workspace, workspace_bytes, stream, x, norm_w, eps, b2::kQ4, nullptr, &sa);
    case B2_SEAM_Q8_F32:
      return tc_gemm_common(b2::kTcEpiF32, w0, nullptr, n_tile_rows, k_tiles, nullptr, batch, ldx, y, ldy, flags,
                            workspace, workspace_bytes, stream, x, norm_w, eps, b2::kQ8, nullptr, &sa);
    default:
      return fail(B2_ERR_ARG, "unknown form %d", form);
  }
}

int b2_q4_dequant_tiles(const uint8_t* tiles, int64_t n_tiles, uint16_t* out, void* stream) {
  return dequant_tiles(0, tiles, n_tiles, out, stream);
}
int b2_q8_dequant_tiles(const uint8_t* tiles, int64_t n_tiles, uint16_t* out, void* stream) {
  return dequant_tiles(1, tiles, n_tiles, out, stream);
}
int b2_q4_dequant_matrix(const uint8_t* tiles, int n_tile_rows, int k_tiles, float* out, int64_t ld,
                         void* stream) {
  return dequant_matrix(0, tiles, n_tile_rows, k_tiles, out, ld, stream);
}
int b2_q8_dequant_matrix(const uint8_t* tiles, int n_tile_rows, int k_tiles, float* out, int64_t ld,
                         void* stream) {
  return dequant_matrix(1, tiles, n_tile_rows, k_tiles, out, ld, stream);
}

}  // extern "C"
