// Tensor-parallel exchanges over NVLink peer memory (one process per GPU).
//
// Every rank owns one peer region (cudaMalloc'd, shared with the other ranks by CUDA
// IPC: plain peer mappings, no multicast object).  Its first 4 KB are control words:
//   sig[64]  u64  signals received, one monotonic counter per source rank
//   exp[64]  u64  signals consumed so far, per source rank (this rank's own count)
//   ticket   u32  last-CTA election of the all-reduce
// The rest holds the exchanged buffers at offsets the host chooses (the same layout on
// every rank).  `peers` is a device array of the W region bases as mapped in this
// process (peers[rank] is the own base).
//
// An exchange is one launch of `chunks` CTAs: CTA c reads its rows of this rank's block
// once and stores them into every rank's region (16-byte stores, over NVLink for the
// peers), then fences at system scope and adds 1 to every rank's sig[rank].  Every
// rank runs the same exchanges in the same order, so after an exchange with C chunks each sig[src] has
// grown by C; a waiter spins (bounded) until sig[src] >= exp[src] + C for all src, then
// exp[src] += C.  Buffers are reused only after a later exchange that every rank has
// entered, so a push never overwrites data a peer has yet to read.
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

constexpr int kPeerMaxRanks = 64;
constexpr int kPeerCtlBytes = 4096;
constexpr int kDevTimeoutPeer = 6;  // device error: a peer's signal never came

struct PeerCtl {
  unsigned long long sig[kPeerMaxRanks];
  unsigned long long exp[kPeerMaxRanks];
  unsigned int ticket;
};

struct XchgParams {
  void* const* peers;  // [world] region bases
  int world, rank, chunks;
  const void* src;
  int rows, cols, ld_src;  // elements
  int elem_bytes;          // 2 or 4
  long long dst_offset;    // bytes into every region
  int ld_dst;              // elements (gather: >= cols*world)
  const float* add_base;   // gather: replicated base to add to (fp32), or null
  float* y;                // allreduce: this rank's replicated fp32 output
  int ldy;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ PeerCtl* peer_ctl(void* base) { return reinterpret_cast<PeerCtl*>(base); }

__device__ __forceinline__ void signal_peer(void* peer_base, int rank) {
  __threadfence_system();
  unsigned long long* s = &peer_ctl(peer_base)->sig[rank];
  asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(s) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* a) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}

// Bounded wait for `chunks` new signals from every rank; true when they all arrived.
// Called by one thread; does not update exp (the caller does, once per exchange).
__device__ bool wait_peers(PeerCtl* ctl, int world, int chunks, unsigned long long timeout_ns) {
  const uint64_t t0 = globaltimer();
  for (int src = 0; src < world; ++src) {
    const unsigned long long want = ctl->exp[src] + static_cast<unsigned long long>(chunks);
    while (ld_acquire_sys(&ctl->sig[src]) < want) {
      if (globaltimer() - t0 > timeout_ns) {
        record_error(kDevTimeoutPeer);
        return false;
      }
    }
  }
  return true;
}

// Push this CTA's rows of the rank's block to every rank's region at byte offset
// `dst_off` (row stride ld_dst elements, this rank's block at column col0).  Each value
// is read once and stored to all W destinations, so with add_base (which may be this
// rank's own copy of the destination) every copy gets the same base + src.
template <typename T>
__device__ void push_rows_all(const XchgParams& p, long long dst_off, int ld_dst, int col0, const float* add_base,
                              int chunk) {
  const int r0 = static_cast<int>(static_cast<long long>(chunk) * p.rows / p.chunks);
  const int r1 = static_cast<int>(static_cast<long long>(chunk + 1) * p.rows / p.chunks);
  const T* src = static_cast<const T*>(p.src);
  constexpr int V = 16 / sizeof(T);
  const bool vec = (p.cols % V) == 0 && (p.ld_src % V) == 0 && (ld_dst % V) == 0 && (col0 % V) == 0 &&
                   (dst_off % 16) == 0 && (reinterpret_cast<uintptr_t>(src) % 16) == 0 &&
                   (!add_base || (reinterpret_cast<uintptr_t>(add_base) % 16) == 0);
  if (vec) {
    const int nv = p.cols / V;
    for (long long e = threadIdx.x; e < static_cast<long long>(r1 - r0) * nv; e += blockDim.x) {
      const int r = r0 + static_cast<int>(e / nv), v = static_cast<int>(e % nv);
      const size_t di = static_cast<size_t>(r) * ld_dst + col0 + v * V;
      uint4 val = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(r) * p.ld_src + v * V);
      if (sizeof(T) == 4 && add_base) {
        const float4 b = *reinterpret_cast<const float4*>(add_base + di);
        float4 f = *reinterpret_cast<float4*>(&val);
        f.x += b.x; f.y += b.y; f.z += b.z; f.w += b.w;
        val = *reinterpret_cast<uint4*>(&f);
      }
      for (int q = 0; q < p.world; ++q) {
        T* dst = reinterpret_cast<T*>(static_cast<uint8_t*>(p.peers[q]) + dst_off);
        *reinterpret_cast<uint4*>(dst + di) = val;
      }
    }
  } else {
    for (long long e = threadIdx.x; e < static_cast<long long>(r1 - r0) * p.cols; e += blockDim.x) {
      const int r = r0 + static_cast<int>(e / p.cols), c = static_cast<int>(e % p.cols);
      const size_t di = static_cast<size_t>(r) * ld_dst + col0 + c;
      T val = src[static_cast<size_t>(r) * p.ld_src + c];
      if (sizeof(T) == 4 && add_base) {
        const float f = *reinterpret_cast<float*>(&val) + add_base[di];
        val = *reinterpret_cast<const T*>(&f);
      }
      for (int q = 0; q < p.world; ++q)
        reinterpret_cast<T*>(static_cast<uint8_t*>(p.peers[q]) + dst_off)[di] = val;
    }
  }
}

// grid = chunks: CTA c pushes its rows to every rank, then signals every rank
template <typename T>
__global__ void __launch_bounds__(256) tp_gather_kernel(const XchgParams p) {
  pdl_wait();  // the block to send is the preceding kernel's output
  pdl_launch_dependents();
  push_rows_all<T>(p, p.dst_offset, p.ld_dst, p.rank * p.cols, p.add_base, blockIdx.x);
  __syncthreads();
  if (threadIdx.x < p.world) signal_peer(p.peers[threadIdx.x], p.rank);
  // one waiter: the launch completes only when every rank's pushes into this region landed
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    PeerCtl* ctl = peer_ctl(p.peers[p.rank]);
    if (wait_peers(ctl, p.world, p.chunks, p.timeout_ns))
      for (int src = 0; src < p.world; ++src) ctl->exp[src] += static_cast<unsigned long long>(p.chunks);
  }
}

// slots: W x [rows][cols] fp32 at dst_offset of every region (slot s = rank s's partial)
__global__ void __launch_bounds__(256) tp_allreduce_kernel(const XchgParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const size_t slot_elems = static_cast<size_t>(p.rows) * p.cols;
  push_rows_all<float>(p, p.dst_offset + static_cast<long long>(p.rank) * slot_elems * 4, p.cols, 0, nullptr,
                       blockIdx.x);
  __syncthreads();
  if (threadIdx.x < p.world) signal_peer(p.peers[threadIdx.x], p.rank);
  // every CTA waits for all partials, then sums its share of the elements in rank order
  __shared__ int ok;
  PeerCtl* ctl = peer_ctl(p.peers[p.rank]);
  if (threadIdx.x == 0) ok = wait_peers(ctl, p.world, p.chunks, p.timeout_ns) ? 1 : 0;
  __syncthreads();
  if (ok) {
    const float* slots = reinterpret_cast<const float*>(static_cast<const uint8_t*>(p.peers[p.rank]) + p.dst_offset);
    const long long n = static_cast<long long>(slot_elems);
    const long long e0 = n * blockIdx.x / gridDim.x, e1 = n * (blockIdx.x + 1) / gridDim.x;
    for (long long e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
      float s = 0.f;
      for (int r = 0; r < p.world; ++r) s += slots[static_cast<size_t>(r) * slot_elems + e];
      const int row = static_cast<int>(e / p.cols), col = static_cast<int>(e % p.cols);
      p.y[static_cast<size_t>(row) * p.ldy + col] += s;
    }
  }
  // the last CTA past its wait consumes the signals (every CTA has read exp by then)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int t = atomicAdd(&ctl->ticket, 1u);
    if (t == gridDim.x - 1) {
      for (int src = 0; src < p.world; ++src) ctl->exp[src] += static_cast<unsigned long long>(p.chunks);
      ctl->ticket = 0;
      __threadfence();
    }
  }
}

}  // namespace b2
