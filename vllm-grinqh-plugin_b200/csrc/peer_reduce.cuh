// Peer buffers of the fused row-parallel all-reduce: the kernel that computes a
// rank's partial y also stores it into every rank's buffer over NVLink and sums the
// ranks' partials (decode_m1.cu for one row, gemm_skinny.cu for 2..64 rows). Plain
// 64-bit peer stores and loads only: no multicast, no bulk copy from peer memory.
//
// Buffer of a rank: word 0 = epoch of its last completed fused launch, word 1 = count
// of the current launch's CTAs that have finished (the last one publishes the epoch and
// clears the count); at kArParts the partial sums [2 (epoch parity)][world][cap], each
// a 64-bit word {fp32 bits, epoch} written by the rank that computed it. cap counts
// output elements (rows x columns) of one launch; entry m * N + n holds y[m, n].
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __CUDACC__
#include "ptx.cuh"
#endif

namespace grinqh {

constexpr int kArMaxRanks = 8;
constexpr size_t kArParts = 256;

struct PeerReduce {
  unsigned char* buf[kArMaxRanks];  // every rank's buffer as mapped in this process
  int rank, world;
  long long cap;                    // output elements a launch may write (the buffers' capacity)
  unsigned long long wait_ns;       // a peer's partial not seen after this long: give up
};

inline size_t peer_reduce_buffer_bytes(int world, int64_t cap) {
  return kArParts + 2 * (size_t)world * (size_t)cap * sizeof(uint64_t);
}

#ifdef __CUDACC__
// A naturally aligned 64-bit store is single-copy atomic, so a reader that sees this
// launch's epoch in a word also sees the value stored with it, without a fence or a
// separate flag.
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Epoch of this launch: one more than the last completed one. Read after
// griddepcontrol.wait (the previous launch on the stream has completed).
__device__ __forceinline__ unsigned peer_epoch(const PeerReduce& ar) {
  return *reinterpret_cast<volatile unsigned*>(ar.buf[ar.rank]) + 1u;
}

// Rank `writer`'s block of the partials of launch `epoch` in rank `owner`'s buffer.
__device__ __forceinline__ unsigned long long* peer_parts(const PeerReduce& ar, int owner, int writer,
                                                          unsigned epoch) {
  return reinterpret_cast<unsigned long long*>(ar.buf[owner] + kArParts) +
         ((size_t)(epoch & 1u) * ar.world + writer) * (size_t)ar.cap;
}

// This rank's partial of output entry e, into every rank's buffer (NVLink stores).
__device__ __forceinline__ void peer_publish(const PeerReduce& ar, unsigned epoch, size_t e, float v) {
  const unsigned long long word = ((unsigned long long)epoch << 32) | __float_as_uint(v);
  for (int r = 0; r < ar.world; ++r) st_relaxed_sys_u64(peer_parts(ar, r, ar.rank, epoch) + e, word);
}

// Every rank's partial of the kE entries e[i] (skipped where !ok[i]) of launch `epoch`,
// summed in rank order -- the same order on every rank, so all ranks get the same bits.
// Two ranks' words are in flight at a time; each wait is bounded: after any wait of
// this file gave up, or after ar.wait_ns, it gives up (counting one timeout) and the
// sums are invalid. Returns false then.
template <int kE>
__device__ bool peer_sum(const PeerReduce& ar, unsigned epoch, const size_t (&e)[kE], const bool (&ok)[kE],
                         float (&v)[kE]) {
#pragma unroll
  for (int i = 0; i < kE; ++i) v[i] = 0.f;
  uint64_t t0 = 0;
  for (int r0 = 0; r0 < ar.world; r0 += 2) {
    const int nr = min(2, ar.world - r0);
    const unsigned long long* src[2] = {peer_parts(ar, ar.rank, r0, epoch),
                                        peer_parts(ar, ar.rank, r0 + (nr > 1 ? 1 : 0), epoch)};
    unsigned long long q[2][kE];
    for (uint32_t it = 0;; ++it) {
      bool all = true;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int i = 0; i < kE; ++i)
          if (j < nr && ok[i] && (it == 0 || (unsigned)(q[j][i] >> 32) != epoch)) q[j][i] = ld_relaxed_sys_u64(src[j] + e[i]);
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int i = 0; i < kE; ++i)
          if (j < nr && ok[i] && (unsigned)(q[j][i] >> 32) != epoch) all = false;
      if (all) break;
      if (t0 == 0) t0 = globaltimer_ns();
      if ((it & 63u) == 63u) {
        if (*reinterpret_cast<volatile unsigned*>(&g_wait_timeouts) != 0u || globaltimer_ns() - t0 > ar.wait_ns) {
          if (*reinterpret_cast<volatile unsigned*>(&g_wait_timeouts) == 0u) atomicAdd(&g_wait_timeouts, 1u);
          return false;  // a rank never arrived
        }
      }
      __nanosleep(32);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int i = 0; i < kE; ++i)
        if (j < nr && ok[i]) v[i] += __uint_as_float((unsigned)q[j][i]);
  }
  return true;
}

// Every CTA of a fused launch calls this as it exits. The epoch of a launch is read by
// each CTA when it starts its reduction, so the next epoch may only be published once
// every CTA of the grid has read it: the last CTA to finish (the count in word 1)
// publishes it and clears the count. The next launch reads it after
// griddepcontrol.wait, i.e. after this grid has completed.
template <bool kAR>
__device__ __forceinline__ void peer_cta_done(const PeerReduce& ar, unsigned epoch) {
  if constexpr (kAR) {
    if (threadIdx.x == 0) {
      unsigned* words = reinterpret_cast<unsigned*>(ar.buf[ar.rank]);
      __threadfence();  // this CTA's read of the epoch is ordered before its count
      if (atomicAdd(words + 1, 1u) == gridDim.x * gridDim.y - 1u) {
        words[1] = 0u;
        *reinterpret_cast<volatile unsigned*>(words) = epoch;
      }
    }
  }
}
#endif

}  // namespace grinqh
