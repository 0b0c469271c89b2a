// 1-bit popcount coarse scorer (the coarse tier the reference recommends for
// very large corpora, bench/RESULTS.md:153-161: "The coarse score is
// popcount(query_signs XOR coarse_signs) -- no Lloyd-Max lookup needed").
// The reference describes it but ships no implementation, so its parity
// definition is this library's:
//
//   coarse sign of row r, coordinate j = MSB of code j (the 1-bit Matryoshka
//     level, remex/core.py:894-901; 1 <=> the rotated coordinate was > 0,
//     since the middle Lloyd-Max boundary is 0 and searchsorted is side='left')
//   query sign j = q_rot[j] > 0
//   score(r) = d - 2 * popcount(query_signs XOR coarse_signs)
//            = sum_j s_q[j] * s_r[j] with s = +-1 (an integer in [-d, d])
//   top-k by score descending, ties by row ascending (exact integers, so the
//   order is fully determined and compared bit for bit).
//
// The scan reads the 1-bit rows (the corpus's at_precision(1) tier, MSB-first
// bits, row stride ldb a multiple of 16) with 128-bit loads: d/8 bytes per row
// instead of d*b/8, one XOR + POPC per 32 coordinates.  Two-stage search
// rescores the top `candidates` at full precision with the rerank kernel.
#include "codes.cuh"
#include "topk.cuh"

namespace pqb {

// Query sign words in the rows' layout: code j is bit (7 - j % 8) of byte
// j / 8; word w holds bytes 4w..4w+3 (little-endian).  mask marks the bits
// of coordinates < d (the row padding past d is not read as data).
__device__ __forceinline__ void sign_words(const float* __restrict__ q, int d, int nw,
                                           uint32_t* qw, uint32_t* mw) {
  for (int w = threadIdx.x; w < nw; w += blockDim.x) {
    uint32_t v = 0, m = 0;
#pragma unroll 4
    for (int t = 0; t < 32; ++t) {
      const int j = 32 * w + t;
      const int byte = t >> 3, bit = 7 - (t & 7);
      if (j < d) {
        m |= 1u << (8 * byte + bit);
        if (__ldg(q + j) > 0.f) v |= 1u << (8 * byte + bit);
      }
    }
    qw[w] = v;
    mw[w] = m;
  }
}

__global__ void __launch_bounds__(256)
hamming_scan_kernel(const uint8_t* __restrict__ signs, int64_t ldb, int64_t n, int d,
                    const float* __restrict__ qrot, int K, int64_t rows_per_block, int nblk,
                    float* __restrict__ cand_s, long long* __restrict__ cand_id) {
  extern __shared__ __align__(16) char smem[];
  const int q = blockIdx.y, b = blockIdx.x;
  const int nw = (d + 31) / 32;
  const int nw4 = (nw + 3) / 4;
  uint32_t* qw = reinterpret_cast<uint32_t*>(smem);
  uint32_t* mw = qw + 4 * nw4;
  for (int w = nw + threadIdx.x; w < 4 * nw4; w += blockDim.x) qw[w] = mw[w] = 0u;
  sign_words(qrot + (size_t)q * d, d, nw, qw, mw);
  BlockTopK tk;
  tk.init(smem + align_up((size_t)8 * 4 * nw4, 16), K, BlockTopK::cap_for(K, blockDim.x));
  const int64_t r0 = (int64_t)b * rows_per_block;
  const int64_t r1 = min(n, r0 + rows_per_block);
  const uint4* q4 = reinterpret_cast<const uint4*>(qw);
  const uint4* m4 = reinterpret_cast<const uint4*>(mw);
  for (int64_t base = r0; base < r1; base += blockDim.x) {
    const int64_t r = base + threadIdx.x;
    const bool valid = r < r1;
    float sc = 0.f;
    if (valid) {
      const uint4* row = reinterpret_cast<const uint4*>(signs + r * ldb);
      int ham = 0;
      for (int c = 0; c < nw4; ++c) {
        const uint4 v = __ldg(row + c), a = q4[c], m = m4[c];
        ham += __popc((v.x ^ a.x) & m.x) + __popc((v.y ^ a.y) & m.y) +
               __popc((v.z ^ a.z) & m.z) + __popc((v.w ^ a.w) & m.w);
      }
      sc = (float)(d - 2 * ham);
    }
    tk.offer(valid, sc, r);
    tk.end_round();
  }
  const size_t o = ((size_t)q * nblk + b) * K;
  tk.write(cand_s + o, cand_id + o, 0);
}

static size_t hamming_smem(int d, int K) {
  const int nw4 = ((d + 31) / 32 + 3) / 4;
  return align_up((size_t)8 * 4 * nw4, 16) +
         BlockTopK::smem_bytes(BlockTopK::cap_for(K, kScanThreads));
}

static int check_signs(const uint8_t* signs, int64_t ldb, int64_t n, int d) {
  PQ_CHECK_ARG(d > 0, "d must be positive (got %d)", d);
  PQ_CHECK_ARG(n >= 0 && n < (1ll << 31), "n=%lld out of range", (long long)n);
  PQ_CHECK_ARG(ldb % 16 == 0 && ldb >= ((int64_t)(d + 127) / 128) * 16,
               "sign-row stride ldb=%lld must be a multiple of 16 covering d=%d bits "
               "rounded up to 128", (long long)ldb, d);
  PQ_CHECK_ARG(n == 0 || signs, "null sign rows");
  PQ_CHECK_ARG(((uintptr_t)signs & 15) == 0, "sign rows must be 16-byte aligned");
  return PQ_OK;
}

// Scans all rows for nq queries, leaving per-block top-K lists in cs/ci
// (layout [nq][nblk][K]).
static int run_hamming(const uint8_t* signs, int64_t ldb, int64_t n, int d, const float* qrot,
                       int nq, int K, float* cs, long long* ci, int* nblk_out, cudaStream_t st) {
  const int64_t per = scan_rows_per_block(n, nq);
  const int nblk = scan_blocks(n, nq);
  *nblk_out = nblk;
  const size_t sm = hamming_smem(d, K);
  int rc = set_smem(hamming_scan_kernel, sm);
  if (rc) return rc;
  hamming_scan_kernel<<<dim3(nblk, nq), kScanThreads, sm, st>>>(signs, ldb, n, d, qrot, K, per,
                                                                 nblk, cs, ci);
  PQ_LAUNCH_CHECK("hamming_scan_kernel");
  return PQ_OK;
}

}  // namespace pqb

using namespace pqb;

extern "C" {

size_t pq_hamming_workspace_bytes(int64_t n, int nq, int k) {
  if (n <= 0 || nq <= 0 || k <= 0) return 256;
  const size_t c = (size_t)nq * scan_blocks(n, nq) * k;
  return align_up(c * sizeof(float), 256) + c * sizeof(long long) + 512;
}

int pq_hamming_scan(const uint8_t* signs, int64_t ldb, int64_t n, int d, const float* qrot,
                    int nq, int k, int64_t row_offset, float* out_scores, int64_t* out_ids,
                    void* ws, size_t ws_bytes, void* stream) {
  int rc = check_signs(signs, ldb, n, d);
  if (rc) return rc;
  PQ_CHECK_ARG(k >= 1 && k <= n && k <= PQ_TOPK_MAX, "k must be in [1, min(n, %d)] (got %d)",
               PQ_TOPK_MAX, k);
  PQ_CHECK_ARG(nq >= 0, "nq must be >= 0");
  if (nq == 0) return PQ_OK;
  PQ_CHECK_ARG(qrot && out_scores && out_ids, "null pointer argument");
  const size_t need = pq_hamming_workspace_bytes(n, nq, k);
  if (!ws || ws_bytes < need)
    return fail(PQ_ERR_WORKSPACE, "pq_hamming_scan needs %zu workspace bytes, got %zu", need,
                ws_bytes);
  cudaStream_t st = (cudaStream_t)stream;
  Carve cv(ws, ws_bytes);
  const size_t c = (size_t)nq * scan_blocks(n, nq) * k;
  float* cs = cv.take<float>(c);
  long long* ci = cv.take<long long>(c);
  int nblk = 0;
  rc = run_hamming(signs, ldb, n, d, qrot, nq, k, cs, ci, &nblk, st);
  if (rc) return rc;
  return launch_merge_sorted(cs, ci, nblk, k, (long long)nblk * k, k, nq, k, row_offset, out_scores,
                      (long long*)out_ids, st);
}

int pq_hamming_twostage(const uint8_t* signs, int64_t ldb_signs, const uint8_t* packed,
                        int64_t ldb, const float* norms, int64_t n, int d, int bits,
                        const float* qrot, int nq, const float* cent_full, int candidates, int k,
                        int64_t row_offset, float* out_scores, int64_t* out_ids, void* ws,
                        size_t ws_bytes, void* stream) {
  int rc = check_signs(signs, ldb_signs, n, d);
  if (rc) return rc;
  rc = check_corpus(packed, ldb, norms, n, d, bits);
  if (rc) return rc;
  PQ_CHECK_ARG(candidates >= 1 && candidates <= n && candidates <= PQ_TOPK_MAX,
               "candidates must be in [1, min(n, %d)] (got %d)", PQ_TOPK_MAX, candidates);
  PQ_CHECK_ARG(k >= 1 && k <= candidates, "k must be in [1, candidates] (got %d)", k);
  if (nq == 0) return PQ_OK;
  PQ_CHECK_ARG(qrot && cent_full && out_scores && out_ids, "null pointer argument");
  const size_t need = pq_hamming_workspace_bytes(n, nq, candidates);
  if (!ws || ws_bytes < need)
    return fail(PQ_ERR_WORKSPACE, "pq_hamming_twostage needs %zu workspace bytes, got %zu", need,
                ws_bytes);
  cudaStream_t st = (cudaStream_t)stream;
  Carve cv(ws, ws_bytes);
  const size_t c = (size_t)nq * scan_blocks(n, nq) * candidates;
  float* cs = cv.take<float>(c);
  long long* ci = cv.take<long long>(c);
  int nblk = 0;
  rc = run_hamming(signs, ldb_signs, n, d, qrot, nq, candidates, cs, ci, &nblk, st);
  if (rc) return rc;
  // Top-`candidates` of the coarse lists (score desc, row asc), rescored at
  // full precision with the f32 table sums, top-k.
  const size_t sm = rerank_smem(d, bits, candidates, k);
  PQ_DISPATCH_B(bits, {
    auto kern = rerank_kernel<B_, B_>;
    rc = set_smem(kern, sm);
    if (rc) return rc;
    kern<<<nq, kScanThreads, sm, st>>>(packed, ldb, norms, n, d, qrot, cent_full, cs, ci, nblk,
                                       nullptr, candidates, k, row_offset, out_scores,
                                       (long long*)out_ids, 1);
  });
  PQ_LAUNCH_CHECK("rerank_kernel");
  return PQ_OK;
}

}  // extern "C"
