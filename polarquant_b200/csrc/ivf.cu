// IVF coarse index over the Matryoshka tier (remex/ivf.py): device index build
// (cell ids) and the query path (query cell, Hamming-ranked probe cells,
// gather-ADC over the probed cells' CSR rows, top-C, full-precision rerank).
#include "codes.cuh"
#include "topk.cuh"

namespace pqb {

// Cell id of every corpus row (remex/ivf.py:162-214).  mode 0 = lsh: bit b is
// sign(sum_j H[b, j] * (2*msb_j - 1)) > 0 over the MSBs of the codes; the
// +-1 x f32 products are exact and summed in f64.  mode 1 = rotated_prefix:
// bit b is the MSB of code b.
__global__ void ivf_cell_ids_kernel(const uint8_t* __restrict__ packed, int64_t ldb, int64_t n,
                                    int d, int B, int n_bits, int mode,
                                    const float* __restrict__ H, uint16_t* __restrict__ cells) {
  extern __shared__ float sH[];  // n_bits x d (lsh)
  if (mode == 0)
    for (int i = threadIdx.x; i < n_bits * d; i += blockDim.x) sH[i] = H[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n;
       r += warps) {
    const uint8_t* row = packed + r * ldb;
    uint32_t cell = 0;
    if (mode == 1) {
      if (lane < n_bits) {
        const int p = lane * B;  // MSB of code `lane` is stream bit p
        const uint32_t bit = (row[p >> 3] >> (7 - (p & 7))) & 1u;
        cell = bit << lane;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) cell |= __shfl_xor_sync(0xffffffffu, cell, o);
    } else {
      double acc[16];
#pragma unroll
      for (int b = 0; b < 16; ++b) acc[b] = 0.0;
      for (int j = lane; j < d; j += 32) {
        const int p = j * B;
        const float sgn = ((row[p >> 3] >> (7 - (p & 7))) & 1u) ? 1.f : -1.f;
#pragma unroll
        for (int b = 0; b < 16; ++b)
          if (b < n_bits) acc[b] += (double)(sgn * sH[b * d + j]);
      }
#pragma unroll
      for (int b = 0; b < 16; ++b) {
        double v = acc[b];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (b < n_bits && v > 0.0) cell |= 1u << b;
      }
    }
    if (lane == 0) cells[r] = (uint16_t)cell;
  }
}

// Query cell and probe list of every query (remex/ivf.py:230-265): one warp
// per query.  The probe list holds the nprobe cells of smallest Hamming
// distance to the query cell, ties by cell id, written in that order.
__global__ void ivf_probe_kernel(const float* __restrict__ qrot, int nq, int d, int n_bits,
                                 int mode, const float* __restrict__ H, int nprobe,
                                 int* __restrict__ probe, int* __restrict__ qcell_out) {
  const int lane = threadIdx.x & 31;
  const int q = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (q >= nq) return;
  const float* x = qrot + (size_t)q * d;
  uint32_t qc = 0;
  if (mode == 1) {
    if (lane < n_bits && x[lane] > 0.f) qc = 1u << lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) qc |= __shfl_xor_sync(0xffffffffu, qc, o);
  } else {
    for (int b = 0; b < n_bits; ++b) {
      double v = 0.0;
      for (int j = lane; j < d; j += 32) v += (double)H[b * d + j] * (double)x[j];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (v > 0.0) qc |= 1u << b;
    }
  }
  if (lane == 0 && qcell_out) qcell_out[q] = (int)qc;
  const int n_cells = 1 << n_bits;
  int* out = probe + (size_t)q * nprobe;
  int written = 0;
  for (int h = 0; h <= n_bits && written < nprobe; ++h) {
    for (int c0 = 0; c0 < n_cells && written < nprobe; c0 += 32) {
      const int c = c0 + lane;
      const bool hit = c < n_cells && __popc((uint32_t)c ^ qc) == h;
      const uint32_t m = __ballot_sync(0xffffffffu, hit);
      const int pos = written + __popc(m & ((1u << lane) - 1u));
      if (hit && pos < nprobe) out[pos] = c;
      written += __popc(m);
    }
  }
}

// Grouped gather-ADC (remex/ivf.py:348-374 coarse scoring over the probed
// cells' rows): block (g, q) scores share g of query q's probe-row list -- the
// concatenation of its nprobe cells' CSR ranges, split into G equal parts --
// at precision P and keeps its top-K.  With `cell_rows` (the packed rows and
// norms copied in CSR order) each probed cell is read as one contiguous run;
// without it rows are gathered through sorted_idx.  Output ids are corpus rows.
template <int B, int P>
__global__ void __launch_bounds__(256)
ivf_group_scan_kernel(const uint8_t* __restrict__ packed, int64_t ldb,
                      const float* __restrict__ norms, const uint8_t* __restrict__ cell_rows,
                      const float* __restrict__ cell_norms, int d,
                      const float* __restrict__ qrot, const float* __restrict__ cent,
                      const int* __restrict__ probe, int nprobe, int G,
                      const long long* __restrict__ sorted_idx,
                      const long long* __restrict__ offsets, int K, float* __restrict__ out_s,
                      long long* __restrict__ out_id) {
  extern __shared__ __align__(16) char smem[];
  const int q = blockIdx.y, g = blockIdx.x;
  const size_t st_floats = query_state_floats<P>(d);
  float* st = reinterpret_cast<float*>(smem);
  long long* pre = reinterpret_cast<long long*>(smem + align_up(st_floats * sizeof(float), 16));
  long long* cstart = pre + (nprobe + 1);
  build_query_state<P>(qrot + (size_t)q * d, d, cent, st, st, st + d);
  for (int j = threadIdx.x; j < nprobe; j += blockDim.x) {
    const int c = probe[(size_t)q * nprobe + j];
    cstart[j] = offsets[c];
    pre[j + 1] = offsets[c + 1] - offsets[c];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    pre[0] = 0;
    for (int j = 0; j < nprobe; ++j) pre[j + 1] += pre[j];
  }
  BlockTopK tk;
  tk.init(reinterpret_cast<char*>(cstart + nprobe), K, BlockTopK::cap_for(K, blockDim.x));
  const long long T = pre[nprobe];
  const long long lo = T * g / G, hi = T * (g + 1) / G;
  const int lane = threadIdx.x & 31;
  // Cell of the thread's first element by binary search, then advanced as the
  // element index grows.
  int j = 0;
  {
    const long long e0 = lo + threadIdx.x;
    int a = 0, b = nprobe;  // pre[a] <= e0 < pre[b]
    while (b - a > 1) {
      const int m = (a + b) >> 1;
      if (pre[m] <= e0) a = m; else b = m;
    }
    j = a;
  }
  for (long long base = lo; base < hi; base += blockDim.x) {
    const long long e = base + threadIdx.x;
    const bool valid = e < hi;
    float sc = 0.f;
    long long r = -1;
    if (valid) {
      while (e >= pre[j + 1]) ++j;
      const long long pos = cstart[j] + (e - pre[j]);
      r = sorted_idx[pos];
      if (cell_rows) {
        sc = score_row<B, P>(cell_rows + pos * ldb, d, st, st, st + d, lane) *
             __ldg(cell_norms + pos);
      } else {
        sc = score_row<B, P>(packed + r * ldb, d, st, st, st + d, lane) * __ldg(norms + r);
      }
    }
    tk.offer(valid, sc, r);
    tk.end_round();
  }
  const size_t o = ((size_t)q * G + g) * K;
  tk.write(out_s + o, out_id + o, 0);
}

}  // namespace pqb

using namespace pqb;

extern "C" {

int pq_ivf_cell_ids(const uint8_t* packed, int64_t ldb, int64_t n, int d, int bits, int n_bits,
                    int mode, const float* hyperplanes, uint16_t* cells, void* stream) {
  PQ_CHECK_ARG(supported_bits(bits), "bits must be one of 1,2,3,4,8 (got %d)", bits);
  PQ_CHECK_ARG(n_bits >= 1 && n_bits <= 16, "n_bits must be 1-16, got %d", n_bits);
  PQ_CHECK_ARG(mode == 0 || mode == 1, "mode must be 0 (lsh) or 1 (rotated_prefix)");
  PQ_CHECK_ARG(mode == 0 || n_bits <= d, "n_bits=%d exceeds d=%d for rotated_prefix mode",
               n_bits, d);
  PQ_CHECK_ARG(ldb >= row_bytes(d, bits), "ldb too small");
  if (n == 0) return PQ_OK;
  PQ_CHECK_ARG(packed && cells && (mode == 1 || hyperplanes), "null pointer argument");
  const size_t sm = mode == 0 ? (size_t)n_bits * d * sizeof(float) : 0;
  if (sm > 227 * 1024) return fail(PQ_ERR_UNSUPPORTED, "hyperplanes too large for shared memory");
  PQ_CUDA_TRY(cudaFuncSetAttribute(ivf_cell_ids_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  int64_t g = (n + 7) / 8;
  if (g > (int64_t)num_sms() * 8) g = (int64_t)num_sms() * 8;
  ivf_cell_ids_kernel<<<(int)g, 256, sm, (cudaStream_t)stream>>>(packed, ldb, n, d, bits, n_bits,
                                                                  mode, hyperplanes, cells);
  PQ_LAUNCH_CHECK("ivf_cell_ids_kernel");
  return PQ_OK;
}

int pq_ivf_probe(const float* qrot, int nq, int d, int n_bits, int mode, const float* hyperplanes,
                 int nprobe, int* probe, int* query_cells, void* stream) {
  PQ_CHECK_ARG(n_bits >= 1 && n_bits <= 16, "n_bits must be 1-16, got %d", n_bits);
  PQ_CHECK_ARG(mode == 0 || mode == 1, "mode must be 0 (lsh) or 1 (rotated_prefix)");
  PQ_CHECK_ARG(nprobe >= 1 && nprobe <= (1 << n_bits), "nprobe must be in [1, n_cells]");
  if (nq == 0) return PQ_OK;
  PQ_CHECK_ARG(qrot && probe && (mode == 1 || hyperplanes), "null pointer argument");
  ivf_probe_kernel<<<(nq + 7) / 8, 256, 0, (cudaStream_t)stream>>>(
      qrot, nq, d, n_bits, mode, hyperplanes, nprobe, probe, query_cells);
  PQ_LAUNCH_CHECK("ivf_probe_kernel");
  return PQ_OK;
}

size_t pq_ivf_workspace_bytes(int nq, int nprobe, int splits, int candidates) {
  const size_t c = (size_t)nq * splits * candidates;
  return align_up((size_t)nq * nprobe * sizeof(int), 256) + align_up(c * sizeof(float), 256) +
         c * sizeof(long long) + 1024;
}

int pq_ivf_search(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                  int bits, int coarse_precision, const float* qrot, int nq,
                  const float* cent_coarse, const float* cent_full, int n_bits, int mode,
                  const float* hyperplanes, const int64_t* sorted_idx, const int64_t* offsets,
                  const uint8_t* cell_rows, const float* cell_norms, int nprobe, int splits,
                  int candidates, int k, int rerank, float* out_scores, int64_t* out_ids,
                  void* ws, size_t ws_bytes, void* stream) {
  int rc = check_corpus(packed, ldb, norms, n, d, bits);
  if (rc) return rc;
  PQ_CHECK_ARG(coarse_precision >= 1 && coarse_precision <= bits,
               "precision must be 1-%d, got %d", bits, coarse_precision);
  PQ_CHECK_ARG(n_bits >= 1 && n_bits <= 16, "n_bits must be 1-16, got %d", n_bits);
  PQ_CHECK_ARG(nprobe >= 1 && nprobe <= (1 << n_bits), "nprobe must be in [1, n_cells]");
  PQ_CHECK_ARG(splits >= 1 && splits <= 64, "splits must be in [1, 64]");
  PQ_CHECK_ARG(candidates >= 1 && candidates <= PQ_TOPK_MAX,
               "candidates must be in [1, %d] (got %d)", PQ_TOPK_MAX, candidates);
  PQ_CHECK_ARG(k >= 1 && k <= candidates, "k must be in [1, candidates] (got %d)", k);
  if (nq == 0) return PQ_OK;
  PQ_CHECK_ARG(qrot && cent_coarse && sorted_idx && offsets && out_scores && out_ids && ws,
               "null pointer argument");
  PQ_CHECK_ARG(!rerank || cent_full, "null full-precision centroids");
  PQ_CHECK_ARG((cell_rows == nullptr) == (cell_norms == nullptr),
               "cell_rows and cell_norms must both be given or both be null");
  PQ_CHECK_ARG(cell_rows == nullptr || ((uintptr_t)cell_rows & 15) == 0,
               "cell_rows must be 16-byte aligned");
  const size_t need = pq_ivf_workspace_bytes(nq, nprobe, splits, candidates);
  if (ws_bytes < need)
    return fail(PQ_ERR_WORKSPACE, "pq_ivf_search needs %zu workspace bytes, got %zu", need,
                ws_bytes);
  cudaStream_t st = (cudaStream_t)stream;
  Carve cv(ws, ws_bytes);
  int* probe = cv.take<int>((size_t)nq * nprobe);
  const size_t c = (size_t)nq * splits * candidates;
  float* cs = cv.take<float>(c);
  long long* ci = cv.take<long long>(c);
  rc = pq_ivf_probe(qrot, nq, d, n_bits, mode, hyperplanes, nprobe, probe, nullptr, stream);
  if (rc) return rc;
  // `splits` row groups per query, each a 1/splits share of the query's
  // probed rows (the prefix sums of the probed cells' sizes live in shared
  // memory next to the query table).
  const size_t sm = scan_smem(d, coarse_precision, candidates) +
                    align_up(((size_t)2 * nprobe + 1) * sizeof(long long), 16);
  dim3 grid(splits, nq);
  PQ_DISPATCH_BP(bits, coarse_precision, {
    auto kern = ivf_group_scan_kernel<B_, P_>;
    rc = set_smem(kern, sm);
    if (rc) return rc;
    kern<<<grid, kScanThreads, sm, st>>>(packed, ldb, norms, cell_rows, cell_norms, d, qrot,
                                         cent_coarse, probe, nprobe, splits,
                                         (const long long*)sorted_idx,
                                         (const long long*)offsets, candidates, cs, ci);
  });
  PQ_LAUNCH_CHECK("ivf_group_scan_kernel");
  const int parts = splits;
  if (!rerank)  // search_coarse: merged coarse top-k
    return launch_merge(cs, ci, parts, candidates, (long long)parts * candidates, candidates, nq,
                        k, 0, out_scores, (long long*)out_ids, st);
  const size_t smr = rerank_smem(d, bits, candidates, k);
  PQ_DISPATCH_B(bits, {
    auto kern = rerank_kernel<B_, B_>;
    rc = set_smem(kern, smr);
    if (rc) return rc;
    kern<<<nq, kScanThreads, smr, st>>>(packed, ldb, norms, n, d, qrot, cent_full, cs, ci, parts,
                                        nullptr, candidates, k, 0, out_scores,
                                        (long long*)out_ids);
  });
  PQ_LAUNCH_CHECK("rerank_kernel");
  return PQ_OK;
}

}  // extern "C"
