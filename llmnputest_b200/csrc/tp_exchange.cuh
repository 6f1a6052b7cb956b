// Tensor-parallel exchanges over NVLink peer memory (one process per GPU).
//
// Every rank owns one peer region (cudaMalloc'd, shared with the other ranks by CUDA
// IPC: plain peer mappings, no multicast object).  Its first kPeerCtlBytes are
// control words:
//   sig[src][c]  u64  chunk c of an exchange received from rank src (monotonic count)
//   exp[src][c]  u64  of those, how many this rank has consumed
//   seam_sig[src][z], seam_exp[src][z], seam_done[z]   the same for a seam z whose sum
//                is pulled by a consumer kernel (tp_seam_* below)
// The rest holds the exchanged buffers at offsets the host chooses (the same layout on
// every rank).  `peers` is a device array of the W region bases as mapped in this
// process (peers[rank] is the own base).
//
// An exchange is one launch of C CTAs, C from the block size (one 16-byte unit per
// thread up to kPeerMaxChunks CTAs).  CTA c owns chunk c: a contiguous run of 16-byte
// units of this rank's block, the same run on every rank.  It
//   1. loads its units (all loads before any store), stores each to every rank's
//      region (W stores per unit, over NVLink for the peers);
//   2. after a CTA barrier, thread q adds 1 to sig[rank][c] of rank q with a
//      release at system scope (the barrier orders the CTA's stores before it);
//   3. thread s waits (bounded, acquire at system scope) until sig[s][c] on this rank
//      exceeds exp[s][c], then advances exp[s][c]: chunk c of every rank has landed;
//   4. (all-reduce) sums chunk c of the W slots in rank order into y.
// Waits are per chunk: a CTA depends only on the same chunk of the other ranks, never
// on the whole exchange.  Every rank runs the same exchanges in the same order, so the
// counters of each (source, chunk) advance together.  A buffer is rewritten only by a
// later exchange that every rank has entered after finishing its reads of it.
//
// Two kinds, for the seams of tensor-parallel decode (the q4nx tiles' natural cuts:
// kv heads, output rows, K-tiles, vocab rows):
//   gather     block [rows][cols] of each rank -> every rank's dst [rows][cols*W] at
//              column rank*cols (attention heads, O rows, logits).  With add_base the
//              pushed value is add_base[r][rank*cols + c] + src[r][c]: an add into a
//              buffer every rank holds identically (the residual stream).
//   allreduce  fp32 partial [rows][cols] of each rank -> every rank: y += sum over
//              ranks, summed in rank order so that every rank's y is bit-identical.
//              The partials travel through W slots of [rows][cols] in each region.
#pragma once

#include "b2_common.cuh"

namespace b2 {

constexpr int kPeerMaxRanks = 16;
constexpr int kPeerMaxChunks = 240;
constexpr int kPeerMaxSeams = 8;
constexpr int kPeerCtlBytes = 65536;
constexpr int kXchgThreads = 256;
constexpr int kXchgUnroll = 4;      // units in flight per thread (loads before stores)
constexpr int kDevTimeoutPeer = 6;  // device error: a peer's signal never came

struct PeerCtl {
  unsigned long long sig[kPeerMaxRanks][kPeerMaxChunks];
  unsigned long long exp[kPeerMaxRanks][kPeerMaxChunks];
  unsigned long long seam_sig[kPeerMaxRanks][kPeerMaxSeams];
  unsigned long long seam_exp[kPeerMaxRanks][kPeerMaxSeams];
  unsigned long long seam_done[kPeerMaxSeams];
  unsigned long long pad[(kPeerCtlBytes - (2 * kPeerMaxRanks * kPeerMaxChunks + 2 * kPeerMaxRanks * kPeerMaxSeams +
                                           kPeerMaxSeams) * 8) / 8];
};
static_assert(sizeof(PeerCtl) == kPeerCtlBytes, "control block layout");

struct XchgParams {
  void* const* peers;  // [world] region bases
  int world, rank, chunks;
  const void* src;
  int rows, cols, ld_src;  // elements
  int vec;                 // 16-byte units (every row start and width aligned), else single elements
  long long dst_offset;    // bytes into every region
  int ld_dst;              // elements (gather: >= cols*world)
  const float* add_base;   // gather: replicated base to add to (fp32), or null
  float* y;                // allreduce: this rank's replicated fp32 output
  int ldy;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ PeerCtl* peer_ctl(void* base) { return reinterpret_cast<PeerCtl*>(base); }

__device__ __forceinline__ void red_release_sys(unsigned long long* a) {
  asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(a) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* a) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}

// Units [u0, u1) of chunk c: units are 16-byte vectors (vec) or single elements of the
// [rows][cols] block in row-major order.
struct ChunkRange {
  long long u0, u1;
  int per_row;  // units per row
};
__device__ __forceinline__ ChunkRange chunk_range(const XchgParams& p, int elem_bytes, int c) {
  ChunkRange r;
  r.per_row = p.vec ? p.cols * elem_bytes / 16 : p.cols;
  const long long U = static_cast<long long>(p.rows) * r.per_row;
  r.u0 = U * c / p.chunks;
  r.u1 = U * (c + 1) / p.chunks;
  return r;
}

// Step 1: this CTA's units of the rank's block to every rank's region at byte offset
// dst_off (row stride ld_dst elements, the block at column col0).  Each value is read
// once and the same value stored to all W copies, so with add_base (which may be this
// rank's own copy of the destination) every copy gets the same base + src.
template <typename T>
__device__ __forceinline__ void push_chunk(const XchgParams& p, long long dst_off, int ld_dst, int col0,
                                           const float* add_base, const ChunkRange& cr) {
  const T* src = static_cast<const T*>(p.src);
  if (p.vec) {
    constexpr int V = 16 / sizeof(T);
    for (long long ub = cr.u0; ub < cr.u1; ub += kXchgThreads * kXchgUnroll) {
      uint4 val[kXchgUnroll];
      size_t di[kXchgUnroll];
#pragma unroll
      for (int j = 0; j < kXchgUnroll; ++j) {
        const long long u = ub + j * kXchgThreads + threadIdx.x;
        if (u < cr.u1) {
          const int r = static_cast<int>(u / cr.per_row), v = static_cast<int>(u % cr.per_row);
          di[j] = static_cast<size_t>(r) * ld_dst + col0 + v * V;
          val[j] = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(r) * p.ld_src + v * V);
          if (sizeof(T) == 4 && add_base) {
            const float4 b = *reinterpret_cast<const float4*>(add_base + di[j]);
            float4 f = *reinterpret_cast<float4*>(&val[j]);
            f.x += b.x;
            f.y += b.y;
            f.z += b.z;
            f.w += b.w;
            val[j] = *reinterpret_cast<uint4*>(&f);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kXchgUnroll; ++j) {
        if (ub + j * kXchgThreads + threadIdx.x < cr.u1)
          for (int q = 0; q < p.world; ++q) {
            T* dst = reinterpret_cast<T*>(static_cast<uint8_t*>(p.peers[q]) + dst_off);
            *reinterpret_cast<uint4*>(dst + di[j]) = val[j];
          }
      }
    }
  } else {
    for (long long ub = cr.u0; ub < cr.u1; ub += kXchgThreads * kXchgUnroll) {
      T val[kXchgUnroll];
      size_t di[kXchgUnroll];
#pragma unroll
      for (int j = 0; j < kXchgUnroll; ++j) {
        const long long u = ub + j * kXchgThreads + threadIdx.x;
        if (u < cr.u1) {
          const int r = static_cast<int>(u / cr.per_row), c = static_cast<int>(u % cr.per_row);
          di[j] = static_cast<size_t>(r) * ld_dst + col0 + c;
          val[j] = src[static_cast<size_t>(r) * p.ld_src + c];
          if (sizeof(T) == 4 && add_base) {
            const float f = *reinterpret_cast<const float*>(&val[j]) + add_base[di[j]];
            val[j] = *reinterpret_cast<const T*>(&f);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kXchgUnroll; ++j) {
        if (ub + j * kXchgThreads + threadIdx.x < cr.u1)
          for (int q = 0; q < p.world; ++q)
            reinterpret_cast<T*>(static_cast<uint8_t*>(p.peers[q]) + dst_off)[di[j]] = val[j];
      }
    }
  }
}

// Steps 2-3 for chunk c; returns (to every thread) whether chunk c of every rank landed.
__device__ __forceinline__ bool signal_and_wait(const XchgParams& p, int c) {
  __shared__ int ok;
  // the CTA barrier orders every thread's stores before thread q's release: a peer
  // that acquires the signal sees the whole chunk
  __syncthreads();
  if (threadIdx.x == 0) ok = 1;
  if (threadIdx.x < p.world) red_release_sys(&peer_ctl(p.peers[threadIdx.x])->sig[p.rank][c]);
  __syncthreads();
  if (threadIdx.x < p.world) {
    PeerCtl* ctl = peer_ctl(p.peers[p.rank]);
    const int s = threadIdx.x;
    const unsigned long long want = ctl->exp[s][c] + 1ull;
    const uint64_t t0 = globaltimer();
    bool got = true;
    while (ld_acquire_sys(&ctl->sig[s][c]) < want) {
      if (globaltimer() - t0 > p.timeout_ns) {
        record_error(kDevTimeoutPeer);
        got = false;
        break;
      }
    }
    if (got)
      ctl->exp[s][c] = want;
    else
      ok = 0;
  }
  __syncthreads();
  return ok != 0;
}

// grid = chunks: CTA c pushes chunk c to every rank, signals, and waits for chunk c of
// every rank; the launch completes once every rank's block has landed here
template <typename T>
__global__ void __launch_bounds__(kXchgThreads) tp_gather_kernel(const XchgParams p) {
  pdl_wait();  // the block to send is the preceding kernel's output
  pdl_launch_dependents();
  const ChunkRange cr = chunk_range(p, sizeof(T), blockIdx.x);
  push_chunk<T>(p, p.dst_offset, p.ld_dst, p.rank * p.cols, p.add_base, cr);
  signal_and_wait(p, blockIdx.x);
}

// slots: W x [rows][cols] fp32 at dst_offset of every region (slot s = rank s's
// partial); CTA c sums chunk c of the slots in rank order into y
__global__ void __launch_bounds__(kXchgThreads) tp_allreduce_kernel(const XchgParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const size_t slot_elems = static_cast<size_t>(p.rows) * p.cols;
  const ChunkRange cr = chunk_range(p, 4, blockIdx.x);
  push_chunk<float>(p, p.dst_offset + static_cast<long long>(p.rank) * slot_elems * 4, p.cols, 0, nullptr, cr);
  if (!signal_and_wait(p, blockIdx.x)) return;
  const float* slots = reinterpret_cast<const float*>(static_cast<const uint8_t*>(p.peers[p.rank]) + p.dst_offset);
  if (p.vec) {
    for (long long u = cr.u0 + threadIdx.x; u < cr.u1; u += kXchgThreads) {
      const int r = static_cast<int>(u / cr.per_row), v = static_cast<int>(u % cr.per_row);
      const size_t e = static_cast<size_t>(r) * p.cols + v * 4;
      float4 s = *reinterpret_cast<const float4*>(slots + e);
      for (int q = 1; q < p.world; ++q) {
        const float4 t = *reinterpret_cast<const float4*>(slots + q * slot_elems + e);
        s.x += t.x;
        s.y += t.y;
        s.z += t.z;
        s.w += t.w;
      }
      float4* yp = reinterpret_cast<float4*>(p.y + static_cast<size_t>(r) * p.ldy + v * 4);
      float4 yv = *yp;
      yv.x += s.x;
      yv.y += s.y;
      yv.z += s.z;
      yv.w += s.w;
      *yp = yv;
    }
  } else {
    for (long long u = cr.u0 + threadIdx.x; u < cr.u1; u += kXchgThreads) {
      const int r = static_cast<int>(u / cr.per_row), c = static_cast<int>(u % cr.per_row);
      const size_t e = static_cast<size_t>(r) * p.cols + c;
      float s = slots[e];
      for (int q = 1; q < p.world; ++q) s += slots[q * slot_elems + e];
      p.y[static_cast<size_t>(r) * p.ldy + c] += s;
    }
  }
}


// ------------------------------------------------------------------ pulled seams
// A seam whose fp32 partials [rows][ld] sit in every rank's region at one offset and
// are summed by the kernel that consumes them (the tensor-core GEMM's x pre-pass), so
// the all-reduce costs no kernel of its own.  Per use of seam z:
//   post  (one thread per rank q, in the consumer, once the producer grid has
//         completed): seam_sig[rank][z] += 1 on rank q, a system-scope release;
//   wait  (thread s of every consumer CTA): until seam_sig[s][z] here exceeds
//         seam_exp[s][z] (bounded; device error kDevTimeoutPeer);
//   advance (one thread of the next kernel, past its PDL wait): seam_exp[.][z] += 1.
// A rank rewrites its partial only in a later use of the same seam, after it has
// waited in another seam that every rank posts only after finishing this one's reads:
// decoders alternate two seams (O and down) per layer.
__device__ __forceinline__ void tp_seam_post(void* const* peers, int world, int rank, int z) {
  // the release orders the producer grid's partial (complete at our PDL wait) before the
  // signal; one system-scope fence, no second one before it (it costs ~1.5 us)
  if (threadIdx.x < world) red_release_sys(&peer_ctl(peers[threadIdx.x])->seam_sig[rank][z]);
}

// Every thread of the CTA calls it; true when every rank's partial has landed.  The
// consumed counts seam_exp[.][z] stay as they are for the whole consumer grid: the kernel
// after it advances them (tp_seam_advance), so no CTA contends on a shared counter here.
__device__ __forceinline__ bool tp_seam_wait(void* const* peers, int world, int rank, int z,
                                             unsigned long long timeout_ns) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (threadIdx.x < world) {
    PeerCtl* ctl = peer_ctl(peers[rank]);
    const int s = threadIdx.x;
    const unsigned long long want = ctl->seam_exp[s][z] + 1ull;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_sys(&ctl->seam_sig[s][z]) < want) {
      if (globaltimer() - t0 > timeout_ns) {
        record_error(kDevTimeoutPeer);
        ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

// One thread of the kernel launched right after the consumer grid (which has completed
// once that kernel is past its PDL wait): every rank's use of seam z counted consumed.
__device__ __forceinline__ void tp_seam_advance(void* const* peers, int world, int rank, int z) {
  PeerCtl* ctl = peer_ctl(peers[rank]);
  for (int q = 0; q < world; ++q) ctl->seam_exp[q][z] += 1ull;
}

}  // namespace b2
