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

// Order-preserving map of a score to 32 bits (a larger score gives a larger
// key; -0 and +0 share a key, as they compare equal; NaN, which `better`
// never prefers, gets the lowest).
__device__ __forceinline__ uint32_t topk_key(float f) {
  if (f != f) return 0u;
  if (f == 0.f) f = 0.f;
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float topk_key_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Shared-memory words a group needs for TopKT::select_compact.
constexpr int kTopkSelectWords = 264;
// Buffer entries per thread select_compact handles (cap <= this x threads).
constexpr int kTopkSelectPerThread = 8;

template <class G>
struct TopKT {
  G g;
  uint32_t* sel;  // select_compact scratch (kTopkSelectWords words)
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

  // Group-wide: keeps the best K of n > K entries without sorting them.  A
  // radix selection (4 passes of 8 bits over topk_key) finds the key T of the
  // K-th best score and how many entries with key T stay; among those, the
  // ones with the smallest ids (unsigned, as `better`).  The threshold becomes
  // the K-th best entry.  Needs `sel` and cap <= E x size (E <= 8).
  template <int E = kTopkSelectPerThread>
  __device__ void select_compact() {
    const int n = *count, t = g.rank(), nt = g.size();
    float es[E];
    long long ei[E];
    uint32_t ek[E];
    bool ev[E];
#pragma unroll
    for (int u = 0; u < E; ++u) {
      const int i = t + u * nt;
      ev[u] = i < n;
      es[u] = ev[u] ? s[i] : 0.f;
      ei[u] = ev[u] ? id[i] : -1;
      ek[u] = ev[u] ? topk_key(es[u]) : 0u;
    }
    uint32_t prefix = 0;
    int remaining = K;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = t; b < 256; b += nt) sel[b] = 0u;
      g.sync();
      const uint32_t hmask = shift == 24 ? 0u : (0xffffffffu << (shift + 8));
#pragma unroll
      for (int u = 0; u < E; ++u)
        if (ev[u] && (ek[u] & hmask) == (prefix & hmask))
          atomicAdd(&sel[(ek[u] >> shift) & 255u], 1u);
      g.sync();
      if (t < 32) {
        // Lane l holds bins 255 - 8l .. 248 - 8l (descending keys).
        uint32_t c[8], sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          c[j] = sel[255 - 8 * t - j];
          sum += c[j];
        }
        uint32_t incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
          if (t >= o) incl += y;
        }
        const uint32_t excl = incl - sum, rem = (uint32_t)remaining;
        if (excl < rem && rem <= incl) {
          uint32_t acc = excl;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (acc < rem && rem <= acc + c[j]) {
              sel[256] = (uint32_t)(255 - 8 * t - j);
              sel[257] = rem - acc;
            }
            acc += c[j];
          }
        }
      }
      g.sync();
      prefix |= sel[256] << shift;
      remaining = (int)sel[257];
      g.sync();
    }
    const uint32_t T = prefix;
    const uint32_t eq = sel[T & 255u];  // entries with key T (the last pass's bin)
    const int need = remaining;         // of which the first `need` by id stay
    bool keep[E];
#pragma unroll
    for (int u = 0; u < E; ++u) {
      keep[u] = ev[u] && ek[u] > T;
      if (ev[u] && ek[u] == T) {
        if ((int)eq == need) {
          keep[u] = true;
        } else {
          int rank = 0;
          for (int j = 0; j < n; ++j)
            if (topk_key(s[j]) == T && (unsigned long long)id[j] < (unsigned long long)ei[u])
              ++rank;
          keep[u] = rank < need;
        }
      }
    }
    unsigned long long* worst = reinterpret_cast<unsigned long long*>(sel + 260);
    if (t == 0) {
      sel[258] = 0u;
      *worst = 0ull;
    }
    g.sync();  // every entry was read before the buffer is rewritten
#pragma unroll
    for (int u = 0; u < E; ++u) {
      if (!keep[u]) continue;
      const uint32_t slot = atomicAdd(&sel[258], 1u);
      s[slot] = es[u];
      id[slot] = ei[u];
      if (ek[u] == T) atomicMax(worst, (unsigned long long)ei[u]);
    }
    g.sync();
    if (t == 0) {
      *count = K;
      *ts = topk_key_float(T);
      *tid = (long long)*worst;
    }
    g.sync();
  }

  // Block-wide, after a round of offers: compact if the next round could overflow.
  __device__ __forceinline__ void end_round() {
    g.sync();
    if (*count > cap - (int)g.size()) compact();
  }

  // end_round with select_compact (kernels that give `sel` scratch and have
  // cap <= E x group size): no sort until write().
  template <int E = kTopkSelectPerThread>
  __device__ __forceinline__ void end_round_select() {
    g.sync();
    if (*count > cap - (int)g.size()) select_compact<E>();
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
