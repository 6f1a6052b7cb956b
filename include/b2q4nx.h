/*
 * b2q4nx -- C ABI of the B200 decode-path library for FastFlowLM q4nx weights.
 *
 * This is the drop-in boundary of the framework: plain pointers, sizes and a
 * CUDA stream passed as `void*`; no torch or CUDA types in any signature.  The
 * Python host layer (llmnputest_b200.npu / .ops) binds it with ctypes; any other
 * host language binds the same symbols through its own C FFI.
 *
 * Conventions shared by every entry point:
 *   - All data pointers are DEVICE pointers owned by the caller.  The library
 *     allocates no device memory per call.
 *   - bf16 values are passed as `uint16_t` bit patterns.
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream).  Calls are
 *     stream-ordered and asynchronous; nothing synchronises the host except
 *     b2_read_device_error().
 *   - Return value: B2_OK (0) or a negative b2_status.  b2_last_error_message()
 *     describes the last failure on the calling thread.
 *   - Weights are q4nx tiles exactly as stored in the .q4nx file: tile-row major
 *     [n_tile_rows][k_tiles][tile_bytes] (tile_bytes 5120 for q4, 8704 for q8),
 *     32 output rows x 256 k per tile.  They must be 16-byte aligned.
 *
 * Reference interfaces replaced (file:line in vegah/LLMNpuTest):
 *   NpuDesign.upload/run/download   reference/npu.py:89-114
 *   NpuLmHead.forward               reference/npu.py:137-150
 *   lmhead_q8_k{0..3}               designs/lm_head/lm_head.h:106-115
 *   granite_gemv_p{P}b{B}_k{N}      designs/granite_gemv/granite_gemv.h:282-302
 *   q4nx_unpack_tile                designs/q4nx_unpack/q4nx_unpack.cc:40-92
 *   Q4NX.tensor dequant             tools/q4nx.py:127-197
 */
#ifndef B2Q4NX_H_
#define B2Q4NX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum b2_status {
  B2_OK = 0,
  B2_ERR_ARG = -1,         /* a size or pointer argument is invalid */
  B2_ERR_ALIGN = -2,       /* a pointer or leading dimension is misaligned */
  B2_ERR_CUDA = -3,        /* a CUDA runtime call or kernel launch failed */
  B2_ERR_NO_DEVICE = -4,   /* no CUDA device is current */
  B2_ERR_UNSUPPORTED = -5, /* the current device is not sm_100 (B200) */
  B2_ERR_WORKSPACE = -6,   /* workspace missing or too small */
  B2_ERR_DEVICE = -7       /* a kernel recorded a device-side error (bounded wait ran out) */
} b2_status;

/* Library version, (major << 16) | (minor << 8) | patch. */
int b2_version(void);

/* Human-readable text for a b2_status, and the detail of the last failure on
 * this thread (empty string if none). */
const char* b2_status_string(int status);
const char* b2_last_error_message(void);

/* Launch options for every later call on this process:
 *   pdl != 0: launch with programmatic dependent launch, so a kernel's prologue
 *   overlaps the tail of the previous kernel in the stream (default on). */
int b2_set_launch_options(int pdl);

/* Read and clear the device error word (0 = none; the first error wins): 1-4 a
 * bounded wait gave up (1 full-wait, 2 empty-wait, 3 drain; 4 unused), 5 an
 * attention call met a sequence position outside its cache or planned length, 6 a
 * tensor-parallel exchange waited too long for another rank (b2_tp_*).
 * Synchronises `stream`.  Returns B2_OK or B2_ERR_CUDA. */
int b2_read_device_error(int* code, void* stream);

/* Flags for the GEMV entry points. */
#define B2_GEMV_ACCUMULATE 1 /* y += W x (residual add) instead of y = W x */
#define B2_GEMV_PREFETCH 2   /* weights are not written by earlier kernels in the
                                stream: they may be streamed before the PDL wait */
#define B2_GEMM_PACKED 4     /* tensor-core GEMM only: the tiles are in the packed
                                layout of b2_q4_gemm_pack */

/* y[b][n] = sum_k W[n][k] x[b][k] for a q4nx q4 (W4A16) weight.
 *   tiles     [n_tile_rows][k_tiles][5120] bytes
 *   x         bf16 [batch][ldx], 16-byte aligned, ldx % 8 == 0, ldx >= 256*k_tiles
 *   y         fp32 [batch][ldy], ldy >= 32*n_tile_rows
 *   batch     1..16
 * Replaces granite_gemv_p{P}b{B}_k{N} (designs/granite_gemv/granite_gemv.h:282-302)
 * and its host oracle granite_gemv.reference (granite_gemv.py:256-272). */
int b2_q4_gemv(const uint8_t* tiles, int n_tile_rows, int k_tiles, const uint16_t* x, int batch, int ldx,
               float* y, int ldy, int flags, void* stream);

/* Same for a q4nx q8 (W8A16) weight, tiles [n_tile_rows][k_tiles][8704].
 * Replaces lmhead_q8_k{0..3} (designs/lm_head/lm_head.h:53-115) and
 * lm_head.reference (designs/lm_head/lm_head.py:129-144). */
int b2_q8_gemv(const uint8_t* tiles, int n_tile_rows, int k_tiles, const uint16_t* x, int batch, int ldx,
               float* y, int ldy, int flags, void* stream);

/* Fused gate/up GEMV + SwiGLU: h[b][n] = silu(bf16(G x)) * bf16(U x), bf16 out.
 *   gate, up  q4 tiles [n_tile_rows][k_tiles][5120] each (same shape)
 *   h         bf16 [batch][ldh], ldh >= 32*n_tile_rows
 * Replaces the gate+up+SwiGLU design (designs/granite_gemv/granite_mlp.py:48-133,
 * granite_swiglu_f32.h:27-51). */
int b2_q4_swiglu_gemv(const uint8_t* gate, const uint8_t* up, int n_tile_rows, int k_tiles, const uint16_t* x,
                      int batch, int ldx, uint16_t* h, int ldh, int flags, void* stream);

/* The three GEMVs above with RMSNorm fused into their input: the kernel reads the
 * fp32 rows x [batch][ldx] (e.g. the residual stream; 16-byte aligned, ldx % 4 == 0),
 * forms bf16(x * rsqrt(mean(x^2) + eps) * norm_w) (norm_w bf16 [K]) and multiplies
 * that, as b2_rmsnorm followed by the plain GEMV would, without the extra launch.
 * The norm is granite_rms_norm (designs/granite_gemv/granite_rmsnorm.h:45-80); the
 * composition is the layer order of designs/granite_gemv/granite_layer.py:54-59. */
int b2_q4_gemv_rmsnorm(const uint8_t* tiles, int n_tile_rows, int k_tiles, const float* x, int batch, int ldx,
                       const uint16_t* norm_w, float eps, float* y, int ldy, int flags, void* stream);
int b2_q8_gemv_rmsnorm(const uint8_t* tiles, int n_tile_rows, int k_tiles, const float* x, int batch, int ldx,
                       const uint16_t* norm_w, float eps, float* y, int ldy, int flags, void* stream);
int b2_q4_swiglu_gemv_rmsnorm(const uint8_t* gate, const uint8_t* up, int n_tile_rows, int k_tiles, const float* x,
                              int batch, int ldx, const uint16_t* norm_w, float eps, uint16_t* h, int ldh,
                              int flags, void* stream);

/* Tile decode, weight-index order: out bf16 [n_tiles][8192] = RNE(code*d + m)
 * (q4) or RNE(code*s) (q8).  Bit-exact with tools/q4nx.py dequant_q4 / dequant_q8
 * (:97-111) and designs/q4nx_unpack/q4nx_unpack.cc:40-92. */
int b2_q4_dequant_tiles(const uint8_t* tiles, int64_t n_tiles, uint16_t* out, void* stream);
int b2_q8_dequant_tiles(const uint8_t* tiles, int64_t n_tiles, uint16_t* out, void* stream);

/* Whole-tensor decode to an untiled fp32 matrix out[n_tile_rows*32][ld]
 * (column k), bit-exact with Q4NX.tensor (tools/q4nx.py:127-197). */
int b2_q4_dequant_matrix(const uint8_t* tiles, int n_tile_rows, int k_tiles, float* out, int64_t ld,
                         void* stream);
int b2_q8_dequant_matrix(const uint8_t* tiles, int n_tile_rows, int k_tiles, float* out, int64_t ld,
                         void* stream);

/* GQA decode attention over a bf16 KV cache, RoPE fused on the new token's q/k.
 *   q, k_new, v_new  fp32 rows of the new token, row stride ld_new floats per
 *                    sequence (q head j at q + b*ld_new + j*D, kv head h at
 *                    k_new/v_new + b*ld_new + h*D) -- e.g. slices of the QKV
 *                    GEMV output [B][(Hq + 2*Hkv)*D]
 *   k_cache, v_cache bf16 [B][Hkv][ctx_max][D]; the new token's rotated k and
 *                    its v are written at position pos[b] (unless
 *                    B2_ATTN_NO_APPEND), and positions 0..pos[b] are attended
 *   pos              int32 [B] device array; max_len >= max(pos) + 1 sizes the
 *                    context split (<= ctx_max).  A kernel records device
 *                    error 5 and reads and writes nothing for a sequence
 *                    whose pos lies outside 0..ctx_max-1
 *   theta, scale     RoPE base (half-split convention) and the score scale
 *                    (head_dim^-0.5 for the reference model)
 *   out              bf16 [B][ldo] (fp32 with B2_ATTN_OUT_F32), q head j at
 *                    out + b*ldo + j*D
 *   workspace        b2_gqa_decode_workspace_size() bytes (may be 0 bytes)
 * head_dim 64, Hq/Hkv <= 8.  fp32 softmax and accumulation.
 * Replaces granite_attn_block/_finish (designs/granite_gemv/granite_attention.h:80-213,
 * design granite_attention.py:50-121) and the RoPE epilogues granite_rope /
 * granite_qkv_rope (granite_elementwise.h:48-75, granite_qkv_rope.h:49-71). */
#define B2_ATTN_NO_APPEND 1 /* the cache already holds position pos[b]; write nothing */
#define B2_ATTN_NO_ROPE 2   /* use the new q/k as given (no rotation) */
#define B2_ATTN_OUT_F32 4   /* fp32 output */
#define B2_ATTN_PREFETCH_KV 8 /* pos[] and the cache rows before pos[b] are final when the
                               * call is launched (no kernel still in flight writes them):
                               * their first chunks are read before the wait on the
                               * preceding kernel (programmatic dependent launch) */
int b2_gqa_decode_workspace_size(int batch, int n_q_heads, int n_kv_heads, int head_dim, int max_len,
                                 size_t* bytes);
int b2_gqa_decode(const float* q, const float* k_new, const float* v_new, int ld_new, uint16_t* k_cache,
                  uint16_t* v_cache, const int32_t* pos, int batch, int n_q_heads, int n_kv_heads, int head_dim,
                  int ctx_max, int max_len, float theta, float scale, uint16_t* out, int ldo, void* workspace,
                  size_t workspace_bytes, int flags, void* stream);

/* b2_gqa_decode without a workspace argument, for callers that cannot allocate
 * device memory: code that only receives input and output buffers from a host
 * framework that owns the GPU allocator, or a service that forbids device
 * allocation after start-up because cudaMalloc can block and synchronise the
 * device.  It has no counterpart in the reference.
 *   - Same arguments and results as b2_gqa_decode, minus the workspace.
 *   - Its scratch is a fixed 2 MiB array inside the library, held by every GPU
 *     that loads the library until the process exits.  It plans its splits
 *     exactly as b2_gqa_decode does, so b2_gqa_decode_workspace_size() is its
 *     scratch need: a call needing more than 2 MiB returns B2_ERR_WORKSPACE
 *     without launching anything.  (With the default plan, at most one wave of
 *     resident CTAs, no call on a 148-SM B200 needs more than about 0.65 MiB.)
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture on the device.
 *   - It allocates nothing: no cudaMalloc, cudaFree or allocating library call.
 *   - All calls share the one array.  Each call writes every partial it later
 *     reads, so nothing needs to start at zero, but calls that overlap on the
 *     GPU (other streams, other threads) race on it: serialise them. */
int b2_gqa_decode_static(const float* q, const float* k_new, const float* v_new, int ld_new, uint16_t* k_cache,
                         uint16_t* v_cache, const int32_t* pos, int batch, int n_q_heads, int n_kv_heads,
                         int head_dim, int ctx_max, int max_len, float theta, float scale, uint16_t* out, int ldo,
                         int flags, void* stream);

/* ---- Tensor-parallel exchanges over NVLink peer memory (one process per GPU) ----
 * The collective seams of tensor-parallel decode (designs/granite_gemv/granite_layer.py
 * gives the layer; the shards are the q4nx tiles' natural cuts: kv heads, output rows,
 * K-tiles, vocab rows), as small kernels that store straight into the other GPUs'
 * memory instead of NCCL calls.  No reference counterpart: the reference runs on one
 * NPU.
 *
 * Peer regions: each rank allocates one with b2_peer_alloc (device memory plus a CUDA
 * IPC handle of B2_IPC_HANDLE_BYTES bytes), hands the handle to the other ranks (any
 * host channel), and maps theirs with b2_peer_open.  Plain peer mappings: no multicast
 * object.  The first B2_PEER_CTL_BYTES of a region are control words (zeroed by the
 * allocation); exchanged buffers sit at higher offsets, the same on every rank.
 * `peers` below is a DEVICE array of `world` (<= B2_PEER_MAX_RANKS) pointers: the
 * regions as mapped in the calling process, peers[rank] being its own.
 *
 * Every rank must issue the same exchanges in the same order.  An exchange is split
 * into chunks, one per CTA; each chunk waits only for the same chunk of the other
 * ranks, with a bounded spin (b2_set_peer_timeout_ms, default 2000 ms); when it runs
 * out the kernel records device error 6 (b2_read_device_error) and returns without
 * waiting further. */
#define B2_IPC_HANDLE_BYTES 64
#define B2_PEER_CTL_BYTES 65536
#define B2_PEER_MAX_RANKS 16
int b2_peer_alloc(size_t bytes, void** ptr, uint8_t* ipc_handle);
int b2_peer_free(void* ptr);
int b2_peer_open(const uint8_t* ipc_handle, void** ptr);
int b2_peer_close(void* ptr);
int b2_set_peer_timeout_ms(int ms);

/* All-gather of column blocks: src [rows][cols] (elem_bytes 2 or 4, row stride ld_src
 * elements) of every rank lands in every rank's region at dst_offset as
 * [rows][ld_dst] with this rank's block at column rank*cols.  With add_base (fp32
 * only), the value stored is add_base[r][rank*cols + c] + src[r][c]: add_base is this
 * rank's copy of a buffer every rank holds identically, so the exchange adds each
 * rank's block into all copies (the residual stream after a row-sharded projection).
 * Replaces NCCL all_gather at the attention, O and lm_head seams. */
int b2_tp_gather(void* const* peers, int world, int rank, const void* src, int rows, int cols, int ld_src,
                 int elem_bytes, long long dst_offset, int ld_dst, const float* add_base, void* stream);

/* All-reduce (sum) into a replicated fp32 buffer: y[r][c] += sum over ranks of their
 * src[r][c], added in rank order on every rank so all copies stay bit-identical.  The
 * partials pass through world * rows * cols floats at slots_offset of every region.
 * Replaces NCCL all_reduce after the K-sharded down projection. */
int b2_tp_allreduce(void* const* peers, int world, int rank, const float* src, int rows, int cols, int ld_src,
                    long long slots_offset, float* y, int ldy, void* stream);

/* The all-reduce fused into the tensor-core GEMM that consumes it (a "pulled seam"):
 * the _rmsnorm GEMM of `form` (B2_SEAM_Q4_F32: b2_q4_gemm_rmsnorm, y fp32;
 * B2_SEAM_Q4_SWIGLU: b2_q4_swiglu_gemm_rmsnorm with w0 = gate, w1 = up, y = h bf16;
 * B2_SEAM_Q8_F32: b2_q8_gemm_rmsnorm) whose x pre-pass first makes every residual row
 *   x[b] += sum over ranks r, in rank order, of r's fp32 partial [batch][ld_part] at byte
 *   part_offset of r's region
 * (read over NVLink through `peers`) and writes it back to x -- bit-identical on every
 * rank -- then normalises it.  The partial is the output of the kernel just before, on
 * every rank (the K-sharded O or down projection); the pre-pass signals that its own is
 * final and waits (bounded: device error 6) for the others', per `seam` (0 ..
 * B2_PEER_MAX_SEAMS - 1, its own counters in the control words).  A rank rewrites a
 * partial only after every rank has read it: alternate two seams (O, then down) per
 * layer, each in its own buffer.  x: K <= 16384, the region offset 16-byte aligned and
 * past the control words, ld_part >= K and a multiple of 4.  Replaces the reference's
 * single-device residual add, as b2_tp_allreduce does, with no launch of its own. */
#define B2_PEER_MAX_SEAMS 8
#define B2_SEAM_Q4_F32 0
#define B2_SEAM_Q4_SWIGLU 1
#define B2_SEAM_Q8_F32 2
int b2_gemm_rmsnorm_seam(int form, const uint8_t* w0, const uint8_t* w1, int n_tile_rows, int k_tiles, float* x,
                         int batch, int ldx, const uint16_t* norm_w, float eps, void* y, int ldy, int flags,
                         void* workspace, size_t workspace_bytes, void* const* peers, int world, int rank,
                         long long part_offset, int ld_part, int seam, void* stream);

/* RMSNorm y = x * rsqrt(mean(x^2) + eps) * w over rows of n, bf16 out.
 *   x  bf16 (x_is_f32 = 0) or fp32 (x_is_f32 = 1), [batch][ldx];  w bf16 [n]
 * Replaces granite_rms_norm (designs/granite_gemv/granite_rmsnorm.h:45-80). */
int b2_rmsnorm(const void* x, int x_is_f32, int ldx, const uint16_t* w, float eps, int batch, int n, uint16_t* y,
               int ldy, void* stream);

/* Decode step of Qwen3.5's gated full-attention layer (head_dim 256), between its
 * q/k/v projections and o_proj, for one new token per sequence at pos[b]:
 *   q_h, k: RMSNorm over the head with weight (1 + w) (q_norm_w, k_norm_w fp32 [256]);
 *   RoPE (rotate_half) on the first rot_dim dims, pair (i, i + rot_dim/2) turned by
 *   pos * inv_freq[i] (inv_freq fp32 [rot_dim/2], the rotary module's own buffer);
 *   the rotated k and the raw v appended to the bf16 cache at row pos[b];
 *   out_h = softmax(q_h K^T / 16) V * sigmoid(gate_h).
 *   qg     fp32 [batch][ld_qg]: q head h at h*512 is q (256) | gate (256), the q_proj
 *          output as transformers lays it out
 *   k_new, v_new  fp32 [batch][ld_kv], kv head g at g*256
 *   k_cache, v_cache  bf16 [batch][n_kv_heads][ctx_max][256], 16-byte aligned
 *   pos    int32 [batch], 0 <= pos < max_len <= ctx_max (a kernel records device
 *          error 5 and writes nothing for a sequence outside that range)
 *   out    bf16 (fp32 with B2_GATED_OUT_F32) [batch][ldo], n_q_heads*256 used
 *   n_q_heads / n_kv_heads in {1, 2, 4}.
 *   workspace: b2_gated_attn_decode_workspace_size bytes, 16-byte aligned (0 when
 *   the (kv head, sequence) pairs fill the SMs and no split is needed).
 * The reference has no kernel for it: it runs transformers 5.5.0's
 * Qwen3_5Attention.forward (models/qwen3_5/modeling_qwen3_5.py:647-692) in float32
 * (reference/from_q4nx.py:140-171). */
#define B2_GATED_OUT_F32 1
int b2_gated_attn_decode_workspace_size(int batch, int n_q_heads, int n_kv_heads, int head_dim, int max_len,
                                        size_t* bytes);
int b2_gated_attn_decode(const float* qg, int ld_qg, const float* k_new, const float* v_new, int ld_kv,
                         const float* q_norm_w, const float* k_norm_w, const float* inv_freq, int rot_dim,
                         uint16_t* k_cache, uint16_t* v_cache, const int32_t* pos, int batch, int n_q_heads,
                         int n_kv_heads, int head_dim, int ctx_max, int max_len, float eps, void* out, int ldo,
                         int flags, void* workspace, size_t workspace_bytes, void* stream);

/* One decode step of a gated DeltaNet (linear-attention) layer, fused: conv
 * update + silu over q|k|v, q/k l2norm (q scaled by 1/sqrt(128)), the gated delta
 * rule on the recurrent state, and the gated RMSNorm of the output.  Per
 * sequence b and v head h (k head h / (n_v_heads / n_k_heads)):
 *   beta = sigmoid(b), decay = exp(-exp(A_log[h]) * softplus(a + dt_bias[h]))
 *   S = decay * S;  S += k (beta (v - S^T k))^T;  o = S^T q
 *   out = o * rsqrt(mean(o^2) + eps) * norm_w * silu(z)
 *   qkv         fp32 [batch][ld_qkv]: q (nk*128) | k (nk*128) | v (nv*128), the
 *               in_proj_qkv output before the conv
 *   z           fp32 [batch][ld_z], nv*128;  b, a  fp32 [batch][ld_ab], nv
 *   conv_state  fp32 [batch][conv_dim = 2*nk*128 + nv*128][4], updated in place
 *   conv_w      fp32 [conv_dim][4];  A_log, dt_bias fp32 [nv];  norm_w fp32 [128]
 *   state       fp32 [batch][nv][128][128] (transformers' cache layout), updated
 *   out         bf16 (fp32 with B2_DELTA_OUT_F32) [batch][ldo], nv*128 used
 *   head_dim 128 only; n_v_heads a multiple of n_k_heads, at most 8x.
 *   conv_state, conv_w and state 16-byte aligned.
 * The reference has no kernel for it: it runs transformers 5.5.0's
 * Qwen3_5GatedDeltaNet.forward (models/qwen3_5/modeling_qwen3_5.py:422-533) in
 * float32 (reference/from_q4nx.py:140-171, chat.py:74-78); this replaces that
 * call's decode branch between in_proj_* and out_proj. */
#define B2_DELTA_OUT_F32 1        /* fp32 output */
#define B2_DELTA_PREFETCH_STATE 2 /* state and conv_state are final at launch (no earlier kernel in
                                     the PDL chain writes them): read them before the PDL wait */
int b2_gated_delta_step(const float* qkv, int ld_qkv, const float* z, int ld_z, const float* b, const float* a,
                        int ld_ab, float* conv_state, const float* conv_w, const float* A_log, const float* dt_bias,
                        const float* norm_w, float* state, int batch, int n_k_heads, int n_v_heads, int head_dim,
                        float eps, void* out, int ldo, int flags, void* stream);

/* ------------------------------------------------------------------------
 * Large-batch W4A16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM):
 * the GEMV entry points' arithmetic for batches up to 256, where the
 * projection is a dense contraction (granite_gemv32.py:90-100
 * is the reference's batched layout).  Weights are dequantised in shared memory
 * to fp16 (w = code*d + m rounded once, relative error <= 2^-11) and x is staged
 * as fp16 x*2^e per token; accumulation fp32.
 *   y   fp32 [batch][ldy] = (or += with B2_GEMV_ACCUMULATE) W x
 *   h   bf16 [batch][ldh] = silu(bf16(G x)) * bf16(U x)        (SwiGLU form)
 *   batch 1..256; x bf16 [batch][ldx], 16-byte aligned, ldx % 8 == 0.
 *   workspace: device memory of b2_q4_gemm_workspace_size bytes, 256-byte
 *   aligned (the staged fp16 x and exponents); not kept between calls.
 *   flags: B2_GEMV_ACCUMULATE (fp32 form); B2_GEMV_PREFETCH (the weights are not
 *   written by kernels in flight: their first stages stream, and are dequantised,
 *   before the wait on the preceding kernel); B2_GEMM_PACKED (tiles from
 *   b2_q4_gemm_pack; A is dequantised into tensor memory).
 * Each call is two launches: a pre-pass that stages x (per token, one CTA) and the
 * GEMM.  The _rmsnorm forms read fp32 rows x [batch][ldx] (16-byte aligned, ldx % 4
 * == 0) and stage bf16(x * rsqrt(mean(x^2) + eps) * norm_w) in that pre-pass, as
 * b2_q4_gemv_rmsnorm does for the GEMV (designs/granite_gemv/granite_rmsnorm.h:45-80),
 * without a separate RMSNorm launch. */
int b2_q4_gemm_workspace_size(int batch, int k_tiles, size_t* bytes);

/* Packed layout for the tensor-core GEMM: the same codes and scales of a q4nx weight
 * [n_tile_rows][k_tiles] (5120 bytes per tile in and out), reordered so that each
 * weight row's codes for 32 consecutive k sit in 16 contiguous bytes (with that
 * block's d and m beside them) and the two tile-rows of each pair are contiguous at
 * every K-tile (one copy per pair).
 * With B2_GEMM_PACKED the GEMM dequantises every row in one thread and writes A
 * straight into tensor memory, where the tensor cores read it (no shared-memory pass
 * for the dequantised weights).  Repack once per weight (a load-time step); a pure
 * byte permutation, so results equal the GEMM on the original tiles.  Not in place.
 * No reference counterpart: the reference reads the tiles as stored. */
int b2_q4_gemm_pack(const uint8_t* tiles, int n_tile_rows, int k_tiles, uint8_t* packed, void* stream);

/* The q8 form (the lm_head): b2_q8_gemm_pack packs a q8 weight (8704-byte tiles: each
 * row's bf16 scale and 32 int8 codes of a 32-k block contiguous, tile-row pairs
 * contiguous per K-tile); b2_q8_gemm / b2_q8_gemm_rmsnorm are the fp32 form of the
 * GEMM above on those tiles, w = fp16(code * scale) rounded once (the q8 GEMV's
 * arithmetic, b2_q8_gemv), flags must include B2_GEMM_PACKED.  Replaces the reference's
 * batched lm_head GEMV (designs/lm_head/lm_head.py:129-144) for large decode batches. */
int b2_q8_gemm_pack(const uint8_t* tiles, int n_tile_rows, int k_tiles, uint8_t* packed, void* stream);
int b2_q8_gemm(const uint8_t* tiles, int n_tile_rows, int k_tiles, const uint16_t* x, int batch, int ldx, float* y,
               int ldy, int flags, void* workspace, size_t workspace_bytes, void* stream);
int b2_q8_gemm_rmsnorm(const uint8_t* tiles, int n_tile_rows, int k_tiles, const float* x, int batch, int ldx,
                       const uint16_t* norm_w, float eps, float* y, int ldy, int flags, void* workspace,
                       size_t workspace_bytes, void* stream);
int b2_q4_gemm(const uint8_t* tiles, int n_tile_rows, int k_tiles, const uint16_t* x, int batch, int ldx, float* y,
               int ldy, int flags, void* workspace, size_t workspace_bytes, void* stream);
int b2_q4_swiglu_gemm(const uint8_t* gate, const uint8_t* up, int n_tile_rows, int k_tiles, const uint16_t* x,
                      int batch, int ldx, uint16_t* h, int ldh, int flags, void* workspace, size_t workspace_bytes,
                      void* stream);
int b2_q4_gemm_rmsnorm(const uint8_t* tiles, int n_tile_rows, int k_tiles, const float* x, int batch, int ldx,
                       const uint16_t* norm_w, float eps, float* y, int ldy, int flags, void* workspace,
                       size_t workspace_bytes, void* stream);
int b2_q4_swiglu_gemm_rmsnorm(const uint8_t* gate, const uint8_t* up, int n_tile_rows, int k_tiles, const float* x,
                              int batch, int ldx, const uint16_t* norm_w, float eps, uint16_t* h, int ldh, int flags,
                              void* workspace, size_t workspace_bytes, void* stream);

/* The down projection with the SwiGLU in its x pre-pass: y = W h (fp32 form, flags as
 * b2_q4_gemm) with h[b][k] = bf16(silu(bf16 g) * bf16 u), g = gu[b][k] and
 * u = gu[b][K + k] (K = k_tiles*256): the SwiGLU epilogue's arithmetic
 * (designs/granite_gemv/granite_mlp.py:172-181) applied to the fp32 outputs of a plain
 * GEMM over the gate and up tile-rows stacked as one weight.  That GEMM can split K
 * across CTAs (the fused SwiGLU form cannot: its epilogue needs whole sums), which
 * fills the SMs when a tensor-parallel shard leaves few row tiles.
 *   gu fp32 [batch][ldgu], 16-byte aligned, ldgu % 4 == 0, ldgu >= 2K. */
int b2_q4_gemm_swiglu_in(const uint8_t* tiles, int n_tile_rows, int k_tiles, const float* gu, int batch, int ldgu,
                          float* y, int ldy, int flags, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B2Q4NX_H_ */
