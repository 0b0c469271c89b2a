// Large-k path of the ADC search (k > PQ_TOPK_MAX, e.g. k >= n, where the
// reference falls back to a full argsort, remex/core.py:575-577, :631-633):
// every row's score is written as a 64-bit key that sorts ascending in the
// library's order (score descending, then row ascending), the keys are
// bitonic-sorted on the device, and the first k are emitted.
#include <vector>

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

// Keys of rows to rank: element e < m is row e (rows == nullptr) or row
// rows[e] (rows outside [0, n), e.g. the -1 of an unused slot, get the key
// that sorts last).  Elements [m, npad) are padding with the same key.
template <int B, int P>
__global__ void __launch_bounds__(256)
score_keys_kernel(const uint8_t* __restrict__ packed, int64_t ldb, const float* __restrict__ norms,
                  int64_t n, int d, const float* __restrict__ q, const float* __restrict__ cent,
                  const long long* __restrict__ rows, int64_t m,
                  unsigned long long* __restrict__ keys, int64_t npad) {
  extern __shared__ __align__(16) char smem[];
  float* st = reinterpret_cast<float*>(smem);
  build_query_state<P>(q, d, cent, st, st, st + d);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < npad;
       e += (int64_t)gridDim.x * blockDim.x) {
    const long long r = e < m ? (rows ? rows[e] : e) : -1;
    if (r >= 0 && r < n) {
      const float sc = score_row<B, P>(packed + r * ldb, d, st, st, st + d, lane) * __ldg(norms + r);
      keys[e] = score_key(sc, r);
    } else {
      keys[e] = ~0ull;
    }
  }
}

// Keys of the rows of one query's probed IVF cells (the concatenation of
// their CSR ranges; pre = prefix sums of the probed cells' sizes, cstart =
// each probed cell's CSR start).  With cell_rows the rows are read from the
// CSR-ordered copy of the corpus.  The key's id is the corpus row.
template <int B, int P>
__global__ void __launch_bounds__(256)
ivf_keys_kernel(const uint8_t* __restrict__ packed, int64_t ldb, const float* __restrict__ norms,
                const uint8_t* __restrict__ cell_rows, const float* __restrict__ cell_norms, int d,
                const float* __restrict__ q, const float* __restrict__ cent,
                const long long* __restrict__ pre, const long long* __restrict__ cstart,
                int nprobe, const long long* __restrict__ sorted_idx,
                unsigned long long* __restrict__ keys, int64_t npad) {
  extern __shared__ __align__(16) char smem[];
  float* st = reinterpret_cast<float*>(smem);
  build_query_state<P>(q, d, cent, st, st, st + d);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const long long T = pre[nprobe];
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < npad;
       e += (int64_t)gridDim.x * blockDim.x) {
    if (e >= T) {
      keys[e] = ~0ull;
      continue;
    }
    int a = 0, b = nprobe;  // pre[a] <= e < pre[b]
    while (b - a > 1) {
      const int mid = (a + b) >> 1;
      if (pre[mid] <= e) a = mid; else b = mid;
    }
    const long long pos = cstart[a] + (e - pre[a]);
    const long long r = sorted_idx[pos];
    const float sc = cell_rows
        ? score_row<B, P>(cell_rows + pos * ldb, d, st, st, st + d, lane) * __ldg(cell_norms + pos)
        : score_row<B, P>(packed + r * ldb, d, st, st, st + d, lane) * __ldg(norms + r);
    keys[e] = score_key(sc, r);
  }
}

// Prefix sums of the probed cells' sizes of query q (one thread; nprobe is
// at most the cell count) and each probed cell's CSR start.
__global__ void ivf_probe_prefix_kernel(const int* __restrict__ probe, int nprobe,
                                        const long long* __restrict__ offsets,
                                        long long* __restrict__ pre, long long* __restrict__ cstart,
                                        long long* __restrict__ total) {
  long long acc = 0;
  pre[0] = 0;
  for (int j = 0; j < nprobe; ++j) {
    const int c = probe[j];
    cstart[j] = offsets[c];
    acc += offsets[c + 1] - offsets[c];
    pre[j + 1] = acc;
  }
  if (total) *total = acc;
}

// Row ids of the first m sorted keys (-1 for padding keys).
// Keys past `avail` (the sorted array's length) count as padding.
__global__ void keys_to_rows_kernel(const unsigned long long* __restrict__ keys, int64_t avail,
                                    int64_t m, long long* __restrict__ rows) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m;
       i += (int64_t)gridDim.x * blockDim.x) {
    const unsigned long long k = i < avail ? keys[i] : ~0ull;
    rows[i] = (k == ~0ull) ? -1 : (long long)(uint32_t)k;
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

// The first K of the sorted keys (keys past `avail`, the array's length,
// count as padding) as scores and ids + row_offset; padding -> -inf / -1.
__global__ void emit_topk_kernel(const unsigned long long* __restrict__ keys, int64_t avail, int K,
                                 long long row_offset, float* __restrict__ out_s,
                                 long long* __restrict__ out_id) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < K; i += gridDim.x * blockDim.x) {
    const unsigned long long k = i < avail ? keys[i] : ~0ull;
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
      kern<<<(int)g, 256, sm, st>>>(packed, ldb, norms, n, d, qrot + (size_t)q * d, cent, nullptr,
                                    n, keys, npad);
    });
    PQ_LAUNCH_CHECK("score_keys_kernel");
    rc = bitonic_sort(keys, npad, st);
    if (rc) return rc;
    emit_topk_kernel<<<(k + 255) / 256, 256, 0, st>>>(keys, npad, k, row_offset,
                                                      out_s + (size_t)q * k,
                                                      (long long*)out_ids + (size_t)q * k);
    PQ_LAUNCH_CHECK("emit_topk_kernel");
  }
  return PQ_OK;
}

// Keys of m rows (rows == nullptr: rows 0..m-1) of one query at precision P,
// into npad keys (padding sorts last).
static int launch_row_keys(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                           int bits, int precision, const float* q, const float* cent,
                           const long long* rows, int64_t m, unsigned long long* keys,
                           int64_t npad, cudaStream_t st) {
  using namespace pqb;
  const size_t sm = align_up(((precision <= 4) ? (size_t)d * 16
                                               : (size_t)d + (size_t)(1 << precision) * 32) * 4,
                             16);
  int64_t g = (npad + 255) / 256;
  if (g > (int64_t)num_sms() * 16) g = (int64_t)num_sms() * 16;
  int rc = PQ_OK;
  PQ_DISPATCH_BP(bits, precision, {
    auto kern = score_keys_kernel<B_, P_>;
    rc = set_smem(kern, sm);
    if (rc) return rc;
    kern<<<(int)g, 256, sm, st>>>(packed, ldb, norms, n, d, q, cent, rows, m, keys, npad);
  });
  PQ_LAUNCH_CHECK("score_keys_kernel");
  return PQ_OK;
}

// Full-precision rescoring of m candidate rows (-1 = empty slot) of one query,
// sorted; the first k are written (score desc, id asc; id + row_offset).
static int rescore_sorted(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                          int bits, const float* q, const float* cent_full, const long long* rows,
                          int64_t m, int k, int64_t row_offset, unsigned long long* keys2,
                          float* out_s, long long* out_id, cudaStream_t st) {
  using namespace pqb;
  const int64_t npad2 = pow2_at_least(m);
  int rc = launch_row_keys(packed, ldb, norms, n, d, bits, bits, q, cent_full, rows, m, keys2,
                           npad2, st);
  if (rc) return rc;
  rc = bitonic_sort(keys2, npad2, st);
  if (rc) return rc;
  emit_topk_kernel<<<(k + 255) / 256, 256, 0, st>>>(keys2, npad2, k, row_offset, out_s, out_id);
  PQ_LAUNCH_CHECK("emit_topk_kernel");
  return PQ_OK;
}

// Two-stage search with more than PQ_TOPK_MAX candidates (remex/core.py:
// 638-719 takes any count): per query the coarse keys of every row are
// sorted, the first C rows are rescored at full precision and sorted, and
// the first k are written.
static size_t large_twostage_ws(int64_t n, int C) {
  using namespace pqb;
  return align_up((size_t)pow2_at_least(n) * 8, 256) + align_up((size_t)C * 8, 256) +
         (size_t)pow2_at_least(C) * 8 + 512;
}

static int large_twostage(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                          int bits, int cp, const float* qrot, int nq, const float* cent_coarse,
                          const float* cent_full, int C, int k, int64_t row_offset, float* out_s,
                          int64_t* out_ids, void* ws, cudaStream_t st) {
  using namespace pqb;
  const int64_t npad = pow2_at_least(n);
  Carve cv(ws, large_twostage_ws(n, C));
  unsigned long long* keys = cv.take<unsigned long long>((size_t)npad);
  long long* rows = cv.take<long long>((size_t)C);
  unsigned long long* keys2 = cv.take<unsigned long long>((size_t)pow2_at_least(C));
  const int gr = (int)((C + 255) / 256);
  for (int q = 0; q < nq; ++q) {
    const float* qv = qrot + (size_t)q * d;
    int rc = launch_row_keys(packed, ldb, norms, n, d, bits, cp, qv, cent_coarse, nullptr, n, keys,
                             npad, st);
    if (rc) return rc;
    rc = bitonic_sort(keys, npad, st);
    if (rc) return rc;
    keys_to_rows_kernel<<<gr < 1024 ? gr : 1024, 256, 0, st>>>(keys, npad, C, rows);
    PQ_LAUNCH_CHECK("keys_to_rows_kernel");
    rc = rescore_sorted(packed, ldb, norms, n, d, bits, qv, cent_full, rows, C, k, row_offset,
                        keys2, out_s + (size_t)q * k, (long long*)out_ids + (size_t)q * k, st);
    if (rc) return rc;
  }
  return PQ_OK;
}

// IVF search with more than PQ_TOPK_MAX candidates (or coarse results):
// per query the coarse keys of the probed cells' rows are sorted; search_coarse
// writes the first k, search_twostage rescores the first C at full precision
// (remex/ivf.py:301-436).  The probed-row counts are read back to the host
// once (one stream synchronisation) to size each query's sort.
static size_t large_ivf_ws(int64_t n, int nq, int nprobe, int C) {
  using namespace pqb;
  return align_up((size_t)nq * nprobe * sizeof(int), 256) +
         align_up((size_t)nq * (nprobe + 1) * 8, 256) + align_up((size_t)nq * nprobe * 8, 256) +
         align_up((size_t)nq * 8, 256) + align_up((size_t)pow2_at_least(n) * 8, 256) +
         align_up((size_t)C * 8, 256) + (size_t)pow2_at_least(C) * 8 + 1024;
}

static int large_ivf(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                     int bits, int cp, const float* qrot, int nq, const float* cent_coarse,
                     const float* cent_full, int n_bits, int mode, const float* hyperplanes,
                     const long long* sorted_idx, const long long* offsets,
                     const uint8_t* cell_rows, const float* cell_norms, int nprobe, int C, int k,
                     int rerank, float* out_s, int64_t* out_ids, void* ws, size_t ws_bytes,
                     cudaStream_t st) {
  using namespace pqb;
  Carve cv(ws, ws_bytes);
  int* probe = cv.take<int>((size_t)nq * nprobe);
  long long* pre = cv.take<long long>((size_t)nq * (nprobe + 1));
  long long* cstart = cv.take<long long>((size_t)nq * nprobe);
  long long* totals = cv.take<long long>((size_t)nq);
  unsigned long long* keys = cv.take<unsigned long long>((size_t)pow2_at_least(n));
  long long* rows = cv.take<long long>((size_t)C);
  unsigned long long* keys2 = cv.take<unsigned long long>((size_t)pow2_at_least(C));
  if (!cv.ok()) return fail(PQ_ERR_WORKSPACE, "IVF search needs %zu workspace bytes", cv.off);
  int rc = pq_ivf_probe(qrot, nq, d, n_bits, mode, hyperplanes, nprobe, probe, nullptr, st);
  if (rc) return rc;
  for (int q = 0; q < nq; ++q) {
    ivf_probe_prefix_kernel<<<1, 1, 0, st>>>(probe + (size_t)q * nprobe, nprobe, offsets,
                                             pre + (size_t)q * (nprobe + 1),
                                             cstart + (size_t)q * nprobe, totals + q);
    PQ_LAUNCH_CHECK("ivf_probe_prefix_kernel");
  }
  std::vector<long long> T(nq);
  PQ_CUDA_TRY(cudaMemcpyAsync(T.data(), totals, sizeof(long long) * nq, cudaMemcpyDeviceToHost,
                              st));
  PQ_CUDA_TRY(cudaStreamSynchronize(st));
  const size_t sm = align_up(((cp <= 4) ? (size_t)d * 16 : (size_t)d + (size_t)(1 << cp) * 32) * 4,
                             16);
  for (int q = 0; q < nq; ++q) {
    const float* qv = qrot + (size_t)q * d;
    const int64_t npad = pow2_at_least(T[q] > 0 ? T[q] : 1);
    int64_t g = (npad + 255) / 256;
    if (g > (int64_t)num_sms() * 16) g = (int64_t)num_sms() * 16;
    PQ_DISPATCH_BP(bits, cp, {
      auto kern = ivf_keys_kernel<B_, P_>;
      rc = set_smem(kern, sm);
      if (rc) return rc;
      kern<<<(int)g, 256, sm, st>>>(packed, ldb, norms, cell_rows, cell_norms, d, qv, cent_coarse,
                                    pre + (size_t)q * (nprobe + 1), cstart + (size_t)q * nprobe,
                                    nprobe, sorted_idx, keys, npad);
    });
    PQ_LAUNCH_CHECK("ivf_keys_kernel");
    rc = bitonic_sort(keys, npad, st);
    if (rc) return rc;
    float* os = out_s + (size_t)q * k;
    long long* oi = (long long*)out_ids + (size_t)q * k;
    if (!rerank) {
      emit_topk_kernel<<<(k + 255) / 256, 256, 0, st>>>(keys, npad, k, 0, os, oi);
      PQ_LAUNCH_CHECK("emit_topk_kernel");
      continue;
    }
    const int gr = (C + 255) / 256;
    keys_to_rows_kernel<<<gr < 1024 ? gr : 1024, 256, 0, st>>>(keys, npad, C, rows);
    PQ_LAUNCH_CHECK("keys_to_rows_kernel");
    rc = rescore_sorted(packed, ldb, norms, n, d, bits, qv, cent_full, rows, C, k, 0, keys2, os,
                        oi, st);
    if (rc) return rc;
  }
  return PQ_OK;
}
