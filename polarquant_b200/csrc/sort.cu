// Large-k path of the ADC search (k > PQ_TOPK_MAX, e.g. k >= n, where the
// reference falls back to a full argsort, remex/core.py:575-577, :631-633):
// every row's score is written as a 64-bit key that sorts ascending in the
// library's order (score descending, then row ascending), the keys are
// bitonic-sorted on the device, and the first k are emitted.
#include "codes.cuh"

namespace pqb {

__device__ __forceinline__ unsigned long long score_key(float s, long long row) {
  uint32_t u = __float_as_uint(s);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // ascending in s
  return ((unsigned long long)(~u) << 32) | (unsigned long long)(uint32_t)row;
}

__device__ __forceinline__ float key_score(unsigned long long k) {
  uint32_t u = ~(uint32_t)(k >> 32);
  u = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
  return __uint_as_float(u);
}

template <int B, int P>
__global__ void __launch_bounds__(256)
score_keys_kernel(const uint8_t* __restrict__ packed, int64_t ldb, const float* __restrict__ norms,
                  int64_t n, int d, const float* __restrict__ q, const float* __restrict__ cent,
                  unsigned long long* __restrict__ keys, int64_t npad) {
  extern __shared__ __align__(16) char smem[];
  float* st = reinterpret_cast<float*>(smem);
  build_query_state<P>(q, d, cent, st, st, st + d);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < npad;
       r += (int64_t)gridDim.x * blockDim.x) {
    if (r < n) {
      const float sc = score_row<B, P>(packed + r * ldb, d, st, st, st + d, lane) * __ldg(norms + r);
      keys[r] = score_key(sc, r);
    } else {
      keys[r] = ~0ull;
    }
  }
}

// One compare-exchange step of the bitonic network over the whole array.
__global__ void bitonic_global_kernel(unsigned long long* __restrict__ a, int64_t npad, int64_t k,
                                      int64_t j) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < npad;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t l = i ^ j;
    if (l > i) {
      const bool asc = (i & k) == 0;
      const unsigned long long x = a[i], y = a[l];
      if ((x > y) == asc) {
        a[i] = y;
        a[l] = x;
      }
    }
  }
}

// All steps j <= 1024 of stage k inside one 2048-element tile in shared memory.
// When k <= 2048 this runs every stage up to k (the initial local sort).
__global__ void __launch_bounds__(1024)
bitonic_shared_kernel(unsigned long long* __restrict__ a, int64_t k_stage, int full_local) {
  __shared__ unsigned long long t[2048];
  const int64_t base = (int64_t)blockIdx.x * 2048;
  t[threadIdx.x] = a[base + threadIdx.x];
  t[threadIdx.x + 1024] = a[base + threadIdx.x + 1024];
  __syncthreads();
  const int64_t k_lo = full_local ? 2 : k_stage;
  for (int64_t k = k_lo; k <= k_stage; k <<= 1) {
    for (int64_t j = (k == k_stage && !full_local) ? 1024 : (k >> 1); j > 0; j >>= 1) {
      if (j > 1024) continue;
      const int i = (int)((threadIdx.x / j) * 2 * j + (threadIdx.x % j));
      const int l = i + (int)j;
      const bool asc = ((base + i) & k) == 0;
      const unsigned long long x = t[i], y = t[l];
      if ((x > y) == asc) {
        t[i] = y;
        t[l] = x;
      }
      __syncthreads();
    }
  }
  a[base + threadIdx.x] = t[threadIdx.x];
  a[base + threadIdx.x + 1024] = t[threadIdx.x + 1024];
}

__global__ void emit_topk_kernel(const unsigned long long* __restrict__ keys, int K,
                                 long long row_offset, float* __restrict__ out_s,
                                 long long* __restrict__ out_id) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < K; i += gridDim.x * blockDim.x) {
    const unsigned long long k = keys[i];
    if (k == ~0ull) {
      out_s[i] = -INFINITY;
      out_id[i] = -1;
    } else {
      out_s[i] = key_score(k);
      out_id[i] = (long long)(uint32_t)k + row_offset;
    }
  }
}

static int64_t pow2_at_least(int64_t x) {
  int64_t p = 2048;
  while (p < x) p <<= 1;
  return p;
}

// Ascending bitonic sort of npad (power of two, >= 2048) keys.
static int bitonic_sort(unsigned long long* a, int64_t npad, cudaStream_t st) {
  const int tiles = (int)(npad / 2048);
  bitonic_shared_kernel<<<tiles, 1024, 0, st>>>(a, 2048, 1);
  PQ_LAUNCH_CHECK("bitonic_shared_kernel");
  int64_t g = npad / 256;
  if (g > (int64_t)num_sms() * 64) g = (int64_t)num_sms() * 64;
  for (int64_t k = 4096; k <= npad; k <<= 1) {
    for (int64_t j = k >> 1; j > 1024; j >>= 1) {
      bitonic_global_kernel<<<(int)g, 256, 0, st>>>(a, npad, k, j);
      PQ_LAUNCH_CHECK("bitonic_global_kernel");
    }
    bitonic_shared_kernel<<<tiles, 1024, 0, st>>>(a, k, 0);
    PQ_LAUNCH_CHECK("bitonic_shared_kernel");
  }
  return PQ_OK;
}

}  // namespace pqb

// Called by pq_adc_scan when k > PQ_TOPK_MAX: one query at a time.
static int adc_large_k(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                       int bits, int precision, const float* qrot, int nq, const float* cent,
                       int k, int64_t row_offset, float* out_s, int64_t* out_ids, void* ws,
                       cudaStream_t st) {
  using namespace pqb;
  const int64_t npad = pow2_at_least(n);
  unsigned long long* keys = (unsigned long long*)ws;
  const size_t sm = align_up(((precision <= 4) ? (size_t)d * 16
                                               : (size_t)d + (size_t)(1 << precision) * 32) * 4,
                             16);
  int64_t g = (npad + 255) / 256;
  if (g > (int64_t)num_sms() * 16) g = (int64_t)num_sms() * 16;
  for (int q = 0; q < nq; ++q) {
    int rc = PQ_OK;
    PQ_DISPATCH_BP(bits, precision, {
      auto kern = score_keys_kernel<B_, P_>;
      rc = set_smem(kern, sm);
      if (rc) return rc;
      kern<<<(int)g, 256, sm, st>>>(packed, ldb, norms, n, d, qrot + (size_t)q * d, cent, keys,
                                    npad);
    });
    PQ_LAUNCH_CHECK("score_keys_kernel");
    rc = bitonic_sort(keys, npad, st);
    if (rc) return rc;
    emit_topk_kernel<<<(k + 255) / 256, 256, 0, st>>>(keys, k, row_offset, out_s + (size_t)q * k,
                                                      (long long*)out_ids + (size_t)q * k);
    PQ_LAUNCH_CHECK("emit_topk_kernel");
  }
  return PQ_OK;
}
