// Block-wide exact top-K with a shared-memory candidate buffer.
//
// Threads offer (score, id) pairs in rounds of at most one offer per thread
// of the group.  A pair
// is kept only if it beats the current K-th best of the buffer (the total order
// of pqb::better); when the buffer could overflow in the next round it is
// bitonic-sorted and cut back to K.  Rejections are exact: a pair worse than
// the buffer's K-th best can never enter the final top-K.  The result is the
// top-K under (score desc, id asc), independent of the offer order.
#pragma once
#include "common.cuh"

namespace pqb {

// The threads that share one top-K buffer: the whole CTA ...
struct CtaGroup {
  __device__ __forceinline__ int rank() const { return threadIdx.x; }
  __device__ __forceinline__ int size() const { return blockDim.x; }
  __device__ __forceinline__ void sync() const { __syncthreads(); }
};

// ... or NT consecutive threads from `first` (whole warps) meeting at named
// barrier ID (1..15), while the CTA's other warps do other work.
template <int ID, int NT>
struct WarpsGroup {
  int first;
  __device__ __forceinline__ int rank() const { return (int)threadIdx.x - first; }
  __device__ __forceinline__ int size() const { return NT; }
  __device__ __forceinline__ void sync() const {
    asm volatile("bar.sync %0, %1;" ::"n"(ID), "n"(NT) : "memory");
  }
};

template <class G>
struct TopKT {
  G g;
  float* s;         // [cap]
  long long* id;    // [cap]
  int* count;       // number of filled slots
  float* ts;        // score of the K-th best after the last compaction (-inf before)
  long long* tid;   // its id
  int K, cap;

  static __host__ __device__ size_t smem_bytes(int cap) {
    return (size_t)cap * (sizeof(float) + sizeof(long long)) + 64;
  }

  // Buffer capacity for a given K: a power of two >= 2*max(K, blockDim).
  static __host__ __device__ int cap_for(int K, int threads) {
    int c = 1;
    int need = 2 * (K > threads ? K : threads);
    while (c < need) c <<= 1;
    return c;
  }

  __device__ void init(char* smem, int K_, int cap_) {
    K = K_;
    cap = cap_;
    id = reinterpret_cast<long long*>(smem);
    s = reinterpret_cast<float*>(smem + (size_t)cap * sizeof(long long));
    char* tail = smem + (size_t)cap * (sizeof(long long) + sizeof(float));
    count = reinterpret_cast<int*>(tail);
    ts = reinterpret_cast<float*>(tail + 8);
    tid = reinterpret_cast<long long*>(tail + 16);
    if (g.rank() == 0) {
      *count = 0;
      *ts = -INFINITY;
      *tid = -1;
    }
    g.sync();
  }

  // Called by every thread; `valid` marks whether this thread has an offer.
  // Returns whether the pair went into the buffer.
  __device__ __forceinline__ bool offer(bool valid, float sc, long long ident) {
    if (valid && (*tid < 0 || better(sc, ident, *ts, *tid))) {
      int slot = atomicAdd(count, 1);
      s[slot] = sc;
      id[slot] = ident;
      return true;
    }
    return false;
  }

  // Block-wide: bitonic sort of the whole buffer, best first.
  __device__ void sort_all() {
    const int n = *count;
    for (int i = n + g.rank(); i < cap; i += g.size()) {
      s[i] = -INFINITY;
      id[i] = -1;
    }
    g.sync();
    for (int k = 2; k <= cap; k <<= 1) {
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = g.rank(); i < cap; i += g.size()) {
          const int l = i ^ j;
          if (l > i) {
            const bool desc = (i & k) == 0;
            const float si = s[i], sl = s[l];
            const long long ii = id[i], il = id[l];
            const bool sw = desc ? better(sl, il, si, ii) : better(si, ii, sl, il);
            if (sw) {
              s[i] = sl; s[l] = si;
              id[i] = il; id[l] = ii;
            }
          }
        }
        g.sync();
      }
    }
  }

  // Block-wide: keep the best K.
  __device__ void compact() {
    sort_all();
    if (g.rank() == 0) {
      int n = *count;
      if (n >= K) {
        n = K;
        *ts = s[K - 1];
        *tid = id[K - 1];
      }
      *count = n;
    }
    g.sync();
  }

  // Block-wide, after a round of offers: compact if the next round could overflow.
  __device__ __forceinline__ void end_round() {
    g.sync();
    if (*count > cap - (int)g.size()) compact();
  }

  // Block-wide: final sort; writes K results (id -1 / -inf past the filled count).
  __device__ void write(float* out_s, long long* out_id, long long id_offset) {
    compact();
    const int n = *count;
    for (int i = g.rank(); i < K; i += g.size()) {
      if (i < n) {
        out_s[i] = s[i];
        out_id[i] = id[i] + id_offset;
      } else {
        out_s[i] = -INFINITY;
        out_id[i] = -1;
      }
    }
  }
};

using BlockTopK = TopKT<CtaGroup>;

}  // namespace pqb
