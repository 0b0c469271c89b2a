// ADC scan, top-k, merge and rerank kernels (single-query semantics, any
// number of queries per launch).  HBM-bound: each block streams a contiguous
// slice of packed rows once per query with 128-bit loads, scores each row
// against a per-query table held in shared memory, and keeps an exact block
// top-K; a second kernel merges the per-block lists.
#include "codes.cuh"
#include "topk.cuh"

namespace pqb {

constexpr int kScanThreads = 256;

// Rows handled by one block of the scan (a multiple of the block size), chosen
// so that nq * blocks covers the GPU several times over.
static int64_t scan_rows_per_block(int64_t n, int nq) {
  const int64_t target = (int64_t)num_sms() * 8;
  int64_t per = (n * (int64_t)nq + target - 1) / target;
  if (per < 2048) per = 2048;
  per = (per + kScanThreads - 1) / kScanThreads * kScanThreads;
  return per;
}

static int scan_blocks(int64_t n, int nq) {
  const int64_t per = scan_rows_per_block(n, nq);
  return (int)((n + per - 1) / per);
}

template <int B, int P>
__global__ void __launch_bounds__(kScanThreads)
scan_topk_kernel(const uint8_t* __restrict__ packed, int64_t ldb, const float* __restrict__ norms,
                 int64_t n, int d, const float* __restrict__ qrot, const float* __restrict__ cent,
                 int K, int64_t rows_per_block, int nblk, float* __restrict__ cand_s,
                 long long* __restrict__ cand_id) {
  extern __shared__ __align__(16) char smem[];
  const int q = blockIdx.y, b = blockIdx.x;
  const size_t st_floats = query_state_floats<P>(d);
  float* st = reinterpret_cast<float*>(smem);
  build_query_state<P>(qrot + (size_t)q * d, d, cent, st, st, st + d);
  BlockTopK tk;
  tk.init(smem + align_up(st_floats * sizeof(float), 16), K,
          BlockTopK::cap_for(K, blockDim.x));  // init() syncs, covering the state build
  const int64_t r0 = (int64_t)b * rows_per_block;
  const int64_t r1 = min(n, r0 + rows_per_block);
  const int lane = threadIdx.x & 31;
  for (int64_t base = r0; base < r1; base += blockDim.x) {
    const int64_t r = base + threadIdx.x;
    const bool valid = r < r1;
    float sc = 0.f;
    if (valid) sc = score_row<B, P>(packed + r * ldb, d, st, st, st + d, lane) * __ldg(norms + r);
    tk.offer(valid, sc, r);
    tk.end_round();
  }
  const size_t o = ((size_t)q * nblk + b) * K;
  tk.write(cand_s + o, cand_id + o, 0);
}

// Merge: candidate (q, part, i) lives at q*q_stride + part*part_stride + i.
__global__ void __launch_bounds__(kScanThreads)
merge_topk_kernel(const float* __restrict__ in_s, const long long* __restrict__ in_id, int parts,
                  int kin, long long q_stride, long long part_stride, int K,
                  long long id_offset, float* __restrict__ out_s, long long* __restrict__ out_id) {
  extern __shared__ __align__(16) char smem[];
  const int q = blockIdx.x;
  BlockTopK tk;
  tk.init(smem, K, BlockTopK::cap_for(K, blockDim.x));
  const long long total = (long long)parts * kin;
  for (long long base = 0; base < total; base += blockDim.x) {
    const long long e = base + threadIdx.x;
    bool valid = e < total;
    float sc = 0.f;
    long long ident = -1;
    if (valid) {
      const long long off = q * q_stride + (e / kin) * part_stride + (e % kin);
      ident = in_id[off];
      sc = in_s[off];
      valid = ident >= 0;
    }
    tk.offer(valid, sc, ident);
    tk.end_round();
  }
  tk.write(out_s + (size_t)q * K, out_id + (size_t)q * K, id_offset);
}

// Merge of lists that are each sorted best first (BlockTopK::write output,
// padded with id -1): thread t walks list t of a chunk of blockDim lists,
// offering its elements in order and stopping at the first one the block's
// top-K rejects (every later element of the list is worse), so a query costs
// about K + parts offers instead of parts * kin.  Same result as
// merge_topk_kernel.  Query q's top-K goes to out + q * out_q_stride.
__global__ void __launch_bounds__(kScanThreads)
merge_sorted_kernel(const float* __restrict__ in_s, const long long* __restrict__ in_id,
                    int parts, int kin, long long q_stride, long long part_stride, int K,
                    long long id_offset, float* __restrict__ out_s, long long* __restrict__ out_id,
                    long long out_q_stride) {
  extern __shared__ __align__(16) char smem[];
  const int q = blockIdx.x;
  BlockTopK tk;
  tk.init(smem, K, BlockTopK::cap_for(K, blockDim.x));
  for (int p0 = 0; p0 < parts; p0 += blockDim.x) {
    const int part = p0 + threadIdx.x;
    bool active = part < parts;
    const long long row = q * q_stride + (long long)part * part_stride;
    for (int j = 0; j < kin; ++j) {
      if (!__syncthreads_or(active)) break;  // block-uniform
      float sc = 0.f;
      long long ident = -1;
      if (active) {
        ident = in_id[row + j];
        sc = in_s[row + j];
      }
      const bool valid = active && ident >= 0;
      const bool taken = tk.offer(valid, sc, ident);
      tk.end_round();
      active = valid && taken;
    }
  }
  tk.write(out_s + q * out_q_stride, out_id + q * out_q_stride, id_offset);
}

// Rescoring of a candidate row list at precision P (exact f32 table sums,
// P = B: full precision), then top-K.  When `coarse` is non-null the list is
// first selected as the top-C of the per-part candidate lists (two-stage
// search, or the candidates of the int8 batched kernel), one block per query.
template <int B, int P>
__global__ void __launch_bounds__(kScanThreads)
rerank_kernel(const uint8_t* __restrict__ packed, int64_t ldb, const float* __restrict__ norms,
              int64_t n, int d, const float* __restrict__ qrot, const float* __restrict__ cent_full,
              const float* __restrict__ coarse_s, const long long* __restrict__ coarse_id,
              int coarse_parts, const long long* __restrict__ cand, int C, int K,
              long long id_offset, float* __restrict__ out_s, long long* __restrict__ out_id,
              int coarse_sorted) {
  extern __shared__ __align__(16) char smem[];
  const int q = blockIdx.x;
  const size_t st_floats = query_state_floats<P>(d);
  float* st = reinterpret_cast<float*>(smem);
  long long* rows = reinterpret_cast<long long*>(smem + align_up(st_floats * sizeof(float), 16));
  char* tk_mem = reinterpret_cast<char*>(rows + align_up((size_t)C, 2));
  BlockTopK tk;
  int nrows = 0;
  if (coarse_s != nullptr) {
    // Stage 1 selection: top-C of coarse_parts x C candidates of this query.
    tk.init(tk_mem, C, BlockTopK::cap_for(C, blockDim.x));
    const long long total = (long long)coarse_parts * C;
    const long long qoff = (long long)q * total;
    if (coarse_sorted) {
      // Lists sorted best first: as merge_sorted_kernel, each thread walks
      // one list until the top-C rejects an element.
      for (int p0 = 0; p0 < coarse_parts; p0 += blockDim.x) {
        const int part = p0 + threadIdx.x;
        bool active = part < coarse_parts;
        const long long lrow = qoff + (long long)part * C;
        for (int j = 0; j < C; ++j) {
          if (!__syncthreads_or(active)) break;  // block-uniform
          float sc = 0.f;
          long long ident = -1;
          if (active) {
            ident = coarse_id[lrow + j];
            sc = coarse_s[lrow + j];
          }
          const bool valid = active && ident >= 0;
          const bool taken = tk.offer(valid, sc, ident);
          tk.end_round();
          active = valid && taken;
        }
      }
    }
    for (long long base = 0; !coarse_sorted && base < total; base += blockDim.x) {
      const long long e = base + threadIdx.x;
      bool valid = e < total;
      float sc = 0.f;
      long long ident = -1;
      if (valid) {
        ident = coarse_id[qoff + e];
        sc = coarse_s[qoff + e];
        valid = ident >= 0;
      }
      tk.offer(valid, sc, ident);
      tk.end_round();
    }
    tk.compact();
    nrows = *tk.count;
    for (int i = threadIdx.x; i < nrows; i += blockDim.x) rows[i] = tk.id[i];
  } else {
    // Candidate ids are global; rows owned by this shard map to [0, n).
    for (int i = threadIdx.x; i < C; i += blockDim.x) {
      const long long g = cand[(size_t)q * C + i];
      rows[i] = (g < 0) ? -1 : g - id_offset;
    }
    nrows = C;
  }
  build_query_state<P>(qrot + (size_t)q * d, d, cent_full, st, st, st + d);
  __syncthreads();
  tk.init(tk_mem, K, BlockTopK::cap_for(K, blockDim.x));
  const int lane = threadIdx.x & 31;
  for (int base = 0; base < nrows; base += blockDim.x) {
    const int i = base + threadIdx.x;
    long long r = -1;
    if (i < nrows) r = rows[i];
    const bool valid = r >= 0 && r < n;
    float sc = 0.f;
    if (valid) sc = score_row<B, P>(packed + r * ldb, d, st, st, st + d, lane) * __ldg(norms + r);
    tk.offer(valid, sc, r);
    tk.end_round();
  }
  tk.write(out_s + (size_t)q * K, out_id + (size_t)q * K, id_offset);
}

// ---------------------------------------------------------------------------
// Packed-row utilities
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t read_code(const uint8_t* row, int j, int B) {
  const int p = j * B;
  const uint32_t v = ((uint32_t)row[p >> 3] << 8) | (uint32_t)row[(p >> 3) + 1];
  return (v >> (16 - B - (p & 7))) & ((1u << B) - 1u);
}

__global__ void unpack_kernel(const uint8_t* __restrict__ packed, int64_t ldb,
                              const long long* __restrict__ idx, int64_t m, int d, int B,
                              int shift, uint8_t* __restrict__ out) {
  const int64_t total = m * (int64_t)d;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = t / d;
    const int j = (int)(t - r * d);
    const int64_t src = idx ? idx[r] : r;
    out[t] = (uint8_t)(read_code(packed + src * ldb, j, B) >> shift);
  }
}

// One thread per output byte: bit i of the byte is bit (i) of the MSB-first
// stream of codes (src >> shift) at width T.
__global__ void pack_bits_kernel(const uint8_t* __restrict__ packed, int64_t ldb, int Bsrc,
                                 int shift, const uint8_t* __restrict__ codes, int64_t n, int d,
                                 int T, uint8_t* __restrict__ out, int64_t ldb_out) {
  const int64_t rbo = (int64_t)ldb_out;
  const int64_t total = n * rbo;
  const int64_t used = ((int64_t)d * T + 7) / 8;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = t / rbo;
    const int o = (int)(t - r * rbo);
    uint32_t byte = 0;
    if (o < used) {
      for (int i = 0; i < 8; ++i) {
        const int pos = o * 8 + i;
        const int j = pos / T, bit = pos % T;
        uint32_t c = 0;
        if (j < d) {
          c = codes ? (uint32_t)codes[r * d + j] & ((1u << T) - 1u)
                    : (read_code(packed + r * ldb, j, Bsrc) >> shift);
        }
        byte |= ((c >> (T - 1 - bit)) & 1u) << (7 - i);
      }
    }
    out[t] = (uint8_t)byte;
  }
}

}  // namespace pqb

using namespace pqb;

// ---------------------------------------------------------------------------
// Dispatch helpers
// ---------------------------------------------------------------------------

#define PQ_DISPATCH_BP(B, P, ...)                                              \
  switch (B * 16 + P) {                                                         \
    case 0x11: { constexpr int B_ = 1, P_ = 1; __VA_ARGS__; } break;                   \
    case 0x21: { constexpr int B_ = 2, P_ = 1; __VA_ARGS__; } break;                   \
    case 0x22: { constexpr int B_ = 2, P_ = 2; __VA_ARGS__; } break;                   \
    case 0x31: { constexpr int B_ = 3, P_ = 1; __VA_ARGS__; } break;                   \
    case 0x32: { constexpr int B_ = 3, P_ = 2; __VA_ARGS__; } break;                   \
    case 0x33: { constexpr int B_ = 3, P_ = 3; __VA_ARGS__; } break;                   \
    case 0x41: { constexpr int B_ = 4, P_ = 1; __VA_ARGS__; } break;                   \
    case 0x42: { constexpr int B_ = 4, P_ = 2; __VA_ARGS__; } break;                   \
    case 0x43: { constexpr int B_ = 4, P_ = 3; __VA_ARGS__; } break;                   \
    case 0x44: { constexpr int B_ = 4, P_ = 4; __VA_ARGS__; } break;                   \
    case 0x81: { constexpr int B_ = 8, P_ = 1; __VA_ARGS__; } break;                   \
    case 0x82: { constexpr int B_ = 8, P_ = 2; __VA_ARGS__; } break;                   \
    case 0x83: { constexpr int B_ = 8, P_ = 3; __VA_ARGS__; } break;                   \
    case 0x84: { constexpr int B_ = 8, P_ = 4; __VA_ARGS__; } break;                   \
    case 0x85: { constexpr int B_ = 8, P_ = 5; __VA_ARGS__; } break;                   \
    case 0x86: { constexpr int B_ = 8, P_ = 6; __VA_ARGS__; } break;                   \
    case 0x87: { constexpr int B_ = 8, P_ = 7; __VA_ARGS__; } break;                   \
    case 0x88: { constexpr int B_ = 8, P_ = 8; __VA_ARGS__; } break;                   \
    default: return fail(PQ_ERR_INVALID, "unsupported bits/precision %d/%d", B, P); \
  }

#define PQ_DISPATCH_B(B, ...)                                   \
  switch (B) {                                                   \
    case 1: { constexpr int B_ = 1; __VA_ARGS__; } break;               \
    case 2: { constexpr int B_ = 2; __VA_ARGS__; } break;               \
    case 3: { constexpr int B_ = 3; __VA_ARGS__; } break;               \
    case 4: { constexpr int B_ = 4; __VA_ARGS__; } break;               \
    case 8: { constexpr int B_ = 8; __VA_ARGS__; } break;               \
    default: return fail(PQ_ERR_INVALID, "unsupported bits %d", B); \
  }

static int check_corpus(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                        int bits) {
  PQ_CHECK_ARG(supported_bits(bits), "bits must be one of 1,2,3,4,8 (got %d)", bits);
  PQ_CHECK_ARG(d > 0, "d must be positive (got %d)", d);
  PQ_CHECK_ARG(n >= 0, "n must be >= 0");
  PQ_CHECK_ARG(ldb >= row_bytes(d, bits) && ldb % 16 == 0,
               "row stride ldb=%lld must be a multiple of 16 and >= %lld", (long long)ldb,
               (long long)row_bytes(d, bits));
  PQ_CHECK_ARG(n == 0 || (packed && norms), "null corpus pointer");
  PQ_CHECK_ARG(((uintptr_t)packed & 15) == 0, "packed rows must be 16-byte aligned");
  return PQ_OK;
}

template <class Kern>
static int set_smem(Kern k, size_t bytes) {
  if (bytes > 227 * 1024)
    return fail(PQ_ERR_UNSUPPORTED, "kernel needs %zu bytes of shared memory", bytes);
  PQ_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  return PQ_OK;
}

static size_t scan_smem(int d, int P, int K) {
  const size_t st = (P <= 4) ? (size_t)d * 16 : (size_t)d + (size_t)(1 << P) * 32;
  return align_up(st * 4, 16) + BlockTopK::smem_bytes(BlockTopK::cap_for(K, kScanThreads));
}

static int launch_merge(const float* in_s, const long long* in_id, int parts, int kin,
                        long long q_stride, long long part_stride, int nq, int K,
                        long long id_offset, float* out_s, long long* out_id, cudaStream_t st) {
  const size_t sm = BlockTopK::smem_bytes(BlockTopK::cap_for(K, kScanThreads));
  int rc = set_smem(merge_topk_kernel, sm);
  if (rc) return rc;
  merge_topk_kernel<<<nq, kScanThreads, sm, st>>>(in_s, in_id, parts, kin, q_stride, part_stride,
                                                  K, id_offset, out_s, out_id);
  PQ_LAUNCH_CHECK("merge_topk_kernel");
  return PQ_OK;
}

// launch_merge for lists each sorted best first (the scans' BlockTopK lists);
// query q's result at out + q * out_q_stride (K when out_q_stride is 0).
static int launch_merge_sorted(const float* in_s, const long long* in_id, int parts, int kin,
                               long long q_stride, long long part_stride, int nq, int K,
                               long long id_offset, float* out_s, long long* out_id,
                               cudaStream_t st, long long out_q_stride = 0) {
  const size_t sm = BlockTopK::smem_bytes(BlockTopK::cap_for(K, kScanThreads));
  int rc = set_smem(merge_sorted_kernel, sm);
  if (rc) return rc;
  merge_sorted_kernel<<<nq, kScanThreads, sm, st>>>(in_s, in_id, parts, kin, q_stride,
                                                    part_stride, K, id_offset, out_s, out_id,
                                                    out_q_stride > 0 ? out_q_stride : K);
  PQ_LAUNCH_CHECK("merge_sorted_kernel");
  return PQ_OK;
}

static int try_scan2(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                     int bits, int precision, const float* qrot, int nq, const float* cent,
                     int K, float* cand_s, long long* cand_id, cudaStream_t st, int* nblk,
                     bool* used);
static size_t bt_tables_bytes(int64_t n, int d, int nq, int k);
static int try_scan_bt(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                       int bits, int precision, const float* qrot, int nq, const float* cent,
                       int K, float* cand_s, long long* cand_id, void* tables,
                       size_t tables_bytes, cudaStream_t st, int* nblk, bool* used);

// Scan every query against all rows, leaving per-block candidates in ws:
// list b of query q at (q * nblk + b) * K, *nblk_out <= scan_blocks(n, nq).
// 1-, 2-, 4- and 8-bit corpora of 2^18+ rows run the byte-table scan
// (scan_bt.cu) when `tables` has room for its tables; other 4- and 8-bit
// corpora the TMA-staged scan (scan2.cu) when it fits; the rest the generic
// scan below.
static int run_scan(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                    int bits, int precision, const float* qrot, int nq, const float* cent, int K,
                    float* cand_s, long long* cand_id, void* tables, size_t tables_bytes,
                    cudaStream_t st, int* nblk_out) {
  bool used = false;
  int rc = try_scan_bt(packed, ldb, norms, n, d, bits, precision, qrot, nq, cent, K, cand_s,
                       cand_id, tables, tables_bytes, st, nblk_out, &used);
  if (rc || used) return rc;
  rc = try_scan2(packed, ldb, norms, n, d, bits, precision, qrot, nq, cent, K, cand_s,
                 cand_id, st, nblk_out, &used);
  if (rc || used) return rc;
  const int64_t per = scan_rows_per_block(n, nq);
  const int nblk = scan_blocks(n, nq);
  *nblk_out = nblk;
  const size_t sm = scan_smem(d, precision, K);
  dim3 grid(nblk, nq);
  PQ_DISPATCH_BP(bits, precision, {
    auto kern = scan_topk_kernel<B_, P_>;
    rc = set_smem(kern, sm);
    if (rc) return rc;
    kern<<<grid, kScanThreads, sm, st>>>(packed, ldb, norms, n, d, qrot, cent, K, per, nblk,
                                         cand_s, cand_id);
  });
  PQ_LAUNCH_CHECK("scan_topk_kernel");
  return PQ_OK;
}

// Batched ADC (tensor cores): per-(query, row chunk) candidate lists of
// *kpart entries each in ws, layout [nq][*nparts][*kpart], ids local (+
// row_offset).  *kpart == K: the lists hold exact scores and the top-K of each
// chunk.  *kpart > K: the lists hold the top-*kpart of each chunk by an
// approximate score (int8 kernel); rescore_candidates() then gives the exact
// top-K.
static int run_batched(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                       int bits, int precision, const float* qrot, int nq, const float* cent, int K,
                       int64_t row_offset, void* ws, size_t ws_bytes, cudaStream_t st,
                       float** parts_s, long long** parts_id, int* nparts, int* kpart);

static int adc_large_k(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                       int bits, int precision, const float* qrot, int nq, const float* cent,
                       int k, int64_t row_offset, float* out_s, int64_t* out_ids, void* ws,
                       cudaStream_t st);

// Two-stage search with more than PQ_TOPK_MAX candidates (sort.cu).
static size_t large_twostage_ws(int64_t n, int C);
static int large_twostage(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                          int bits, int cp, const float* qrot, int nq, const float* cent_coarse,
                          const float* cent_full, int C, int k, int64_t row_offset, float* out_s,
                          int64_t* out_ids, void* ws, cudaStream_t st);

extern "C" {

}  // extern "C"

// Candidate lists of the streaming scans (the part of the workspace every
// scan needs).
static size_t scan_ws_base(int64_t n, int nq, int k) {
  const size_t c = (size_t)nq * scan_blocks(n, nq) * k;
  return align_up(align_up(c * sizeof(float), 256) + c * sizeof(long long) + 512, 256);
}

extern "C" {

size_t pq_adc_scan_workspace_bytes(int64_t n, int d, int nq, int k) {
  if (n <= 0 || nq <= 0 || k <= 0) return 256;
  if (k > PQ_TOPK_MAX) {
    size_t p = 2048;
    while ((int64_t)p < n) p <<= 1;
    return p * sizeof(unsigned long long) + 256;
  }
  // + the byte-table scan's tables where it may run (a smaller workspace
  // holding at least the candidate lists is accepted: the call then uses
  // the other scans).
  return scan_ws_base(n, nq, k) + bt_tables_bytes(n, d, nq, k);
}

int pq_adc_scan(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d, int bits,
                int precision, const float* qrot, int nq, const float* cent, int k,
                int64_t row_offset, float* out_scores, int64_t* out_ids, void* ws,
                size_t ws_bytes, void* stream) {
  int rc = check_corpus(packed, ldb, norms, n, d, bits);
  if (rc) return rc;
  PQ_CHECK_ARG(precision >= 1 && precision <= bits, "precision must be 1-%d, got %d", bits,
               precision);
  PQ_CHECK_ARG(nq >= 0, "nq must be >= 0");
  PQ_CHECK_ARG(k >= 1, "k must be >= 1 (got %d)", k);
  PQ_CHECK_ARG(k <= n, "k=%d exceeds n=%lld", k, (long long)n);
  PQ_CHECK_ARG(n < (1ll << 31), "n=%lld rows exceed one launch; shard the corpus", (long long)n);
  if (nq == 0) return PQ_OK;
  PQ_CHECK_ARG(qrot && cent && out_scores && out_ids, "null pointer argument");
  const size_t need = k > PQ_TOPK_MAX ? pq_adc_scan_workspace_bytes(n, d, nq, k)
                                      : scan_ws_base(n, nq, k);
  if (ws_bytes < need || !ws)
    return fail(PQ_ERR_WORKSPACE, "pq_adc_scan needs %zu workspace bytes, got %zu", need, ws_bytes);
  cudaStream_t st = (cudaStream_t)stream;
  if (k > PQ_TOPK_MAX)
    return adc_large_k(packed, ldb, norms, n, d, bits, precision, qrot, nq, cent, k, row_offset,
                       out_scores, out_ids, ws, st);
  int nblk = scan_blocks(n, nq);
  Carve cv(ws, ws_bytes);
  const size_t c = (size_t)nq * nblk * k;
  float* cs = cv.take<float>(c);
  long long* ci = cv.take<long long>(c);
  char* tables = (char*)ws + need;
  rc = run_scan(packed, ldb, norms, n, d, bits, precision, qrot, nq, cent, k, cs, ci, tables,
                ws_bytes - need, st, &nblk);
  if (rc) return rc;
  return launch_merge_sorted(cs, ci, nblk, k, (long long)nblk * k, k, nq, k, row_offset,
                             out_scores, (long long*)out_ids, st);
}

// Query batches at least this large run the coarse stage of two-stage search
// on the tensor cores (batched ADC); smaller ones use the streaming scan.
constexpr int kTwostageBatchMin = 64;
// ... and on corpora of at least kTwostageLargeRows rows from this many: one
// pass of the batched kernels costs a few single-query scans there.
constexpr int kTwostageBatchMinLarge = 8;
constexpr int64_t kTwostageLargeRows = 1 << 20;

static bool twostage_batched(int64_t n, int nq, int candidates) {
  return candidates <= 256 &&
         (nq >= kTwostageBatchMin || (nq >= kTwostageBatchMinLarge && n >= kTwostageLargeRows));
}

static size_t batched_ws(int64_t n, int d, int nq, int k);

// Offset of the exact coarse candidates (nq x candidates scores + ids) that
// follow the batched workspace in two-stage search.
static size_t twostage_exact_offset(int64_t n, int d, int nq, int candidates) {
  return align_up(batched_ws(n, d, nq, candidates), 256);
}

size_t pq_twostage_workspace_bytes(int64_t n, int d, int nq, int candidates) {
  if (candidates > PQ_TOPK_MAX) return large_twostage_ws(n, candidates);
  const size_t a = pq_adc_scan_workspace_bytes(n, d, nq, candidates);
  if (twostage_batched(n, nq, candidates)) {
    const size_t b = twostage_exact_offset(n, d, nq, candidates) +
                     align_up((size_t)nq * candidates * sizeof(float), 256) +
                     (size_t)nq * candidates * sizeof(long long) + 256;
    return a > b ? a : b;
  }
  return a;
}

// Shared memory of rerank_kernel<B, P> with `bits` = P.
static size_t rerank_smem(int d, int bits, int C, int K) {
  const size_t st = (bits <= 4) ? (size_t)d * 16 : (size_t)d + (size_t)(1 << bits) * 32;
  const int cap = BlockTopK::cap_for(C > K ? C : K, kScanThreads);
  return align_up(st * 4, 16) + align_up((size_t)C, 2) * 8 + BlockTopK::smem_bytes(cap);
}

// Exact top-K of approximate candidate lists (layout [nq][parts][C], local
// row ids, each list sorted best first as the batched kernels write them):
// per query the top-C of all lists by the approximate score, each
// rescored at precision P with the f32 table sums of the streaming scan,
// then the top-K; output ids + id_offset.
static int rescore_candidates(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n,
                              int d, int bits, int precision, const float* qrot, int nq,
                              const float* cent, const float* cs, const long long* ci, int parts,
                              int C, int K, int64_t id_offset, float* out_s, long long* out_id,
                              cudaStream_t st) {
  const size_t sm = rerank_smem(d, precision, C, K);
  int rc = PQ_OK;
  PQ_DISPATCH_BP(bits, precision, {
    auto kern = rerank_kernel<B_, P_>;
    rc = set_smem(kern, sm);
    if (rc) return rc;
    kern<<<nq, kScanThreads, sm, st>>>(packed, ldb, norms, n, d, qrot, cent, cs, ci, parts,
                                       nullptr, C, K, id_offset, out_s, out_id, 1);
  });
  PQ_LAUNCH_CHECK("rerank_kernel");
  return PQ_OK;
}

int pq_twostage(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d, int bits,
                int coarse_precision, const float* qrot, int nq, const float* cent_coarse,
                const float* cent_full, int candidates, int k, int64_t row_offset,
                float* out_scores, int64_t* out_ids, void* ws, size_t ws_bytes, void* stream) {
  int rc = check_corpus(packed, ldb, norms, n, d, bits);
  if (rc) return rc;
  PQ_CHECK_ARG(coarse_precision >= 1 && coarse_precision <= bits,
               "precision must be 1-%d, got %d", bits, coarse_precision);
  PQ_CHECK_ARG(candidates >= 1 && candidates <= n,
               "candidates must be in [1, n] (got %d)", candidates);
  PQ_CHECK_ARG(k >= 1 && k <= candidates, "k must be in [1, candidates] (got %d)", k);
  PQ_CHECK_ARG(n < (1ll << 31), "n=%lld rows exceed one launch; shard the corpus", (long long)n);
  if (nq == 0) return PQ_OK;
  PQ_CHECK_ARG(qrot && cent_coarse && cent_full && out_scores && out_ids, "null pointer argument");
  const size_t need = pq_twostage_workspace_bytes(n, d, nq, candidates);
  if (ws_bytes < need || !ws)
    return fail(PQ_ERR_WORKSPACE, "pq_twostage needs %zu workspace bytes, got %zu", need, ws_bytes);
  cudaStream_t st = (cudaStream_t)stream;
  if (candidates > PQ_TOPK_MAX)
    return large_twostage(packed, ldb, norms, n, d, bits, coarse_precision, qrot, nq, cent_coarse,
                          cent_full, candidates, k, row_offset, out_scores, out_ids, ws, st);
  float* cs;
  long long* ci;
  int nblk;
  // Every coarse candidate list is sorted best first: the streaming scans'
  // (BlockTopK::write) and the batched kernels' (warp_compact).
  const int sorted_lists = 1;
  if (twostage_batched(n, nq, candidates)) {
    int kpart = candidates;
    rc = run_batched(packed, ldb, norms, n, d, bits, coarse_precision, qrot, nq, cent_coarse,
                     candidates, 0, ws, ws_bytes, st, &cs, &ci, &nblk, &kpart);
    if (rc) return rc;
    if (kpart != candidates) {
      // Approximate coarse lists: exact coarse scores of the best kpart, top
      // `candidates` of them (global ids), then the full-precision rerank.
      float* es = reinterpret_cast<float*>((char*)ws + twostage_exact_offset(n, d, nq, candidates));
      long long* ei = reinterpret_cast<long long*>(
          (char*)es + align_up((size_t)nq * candidates * sizeof(float), 256));
      rc = rescore_candidates(packed, ldb, norms, n, d, bits, coarse_precision, qrot, nq,
                              cent_coarse, cs, ci, nblk, kpart, candidates, row_offset, es, ei, st);
      if (rc) return rc;
      const size_t sm = rerank_smem(d, bits, candidates, k);
      PQ_DISPATCH_B(bits, {
        auto kern = rerank_kernel<B_, B_>;
        rc = set_smem(kern, sm);
        if (rc) return rc;
        kern<<<nq, kScanThreads, sm, st>>>(packed, ldb, norms, n, d, qrot, cent_full, nullptr,
                                           nullptr, 0, ei, candidates, k, row_offset, out_scores,
                                           (long long*)out_ids, 0);
      });
      PQ_LAUNCH_CHECK("rerank_kernel");
      return PQ_OK;
    }
  } else {
    nblk = scan_blocks(n, nq);
    Carve cv(ws, ws_bytes);
    const size_t c = (size_t)nq * nblk * candidates;
    cs = cv.take<float>(c);
    ci = cv.take<long long>(c);
    const size_t base = scan_ws_base(n, nq, candidates);
    rc = run_scan(packed, ldb, norms, n, d, bits, coarse_precision, qrot, nq, cent_coarse,
                  candidates, cs, ci, ws_bytes > base ? (char*)ws + base : nullptr,
                  ws_bytes > base ? ws_bytes - base : 0, st, &nblk);
  }
  if (rc) return rc;
  const size_t sm = rerank_smem(d, bits, candidates, k);
  PQ_DISPATCH_B(bits, {
    auto kern = rerank_kernel<B_, B_>;
    rc = set_smem(kern, sm);
    if (rc) return rc;
    kern<<<nq, kScanThreads, sm, st>>>(packed, ldb, norms, n, d, qrot, cent_full, cs, ci, nblk,
                                       nullptr, candidates, k, row_offset, out_scores,
                                       (long long*)out_ids, sorted_lists);
  });
  PQ_LAUNCH_CHECK("rerank_kernel");
  return PQ_OK;
}

int pq_rerank(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d, int bits,
              const float* qrot, int nq, const float* cent_full, const int64_t* cand, int C, int k,
              int64_t row_offset, float* out_scores, int64_t* out_ids, void* stream) {
  int rc = check_corpus(packed, ldb, norms, n, d, bits);
  if (rc) return rc;
  PQ_CHECK_ARG(C >= 1 && C <= 8 * PQ_TOPK_MAX, "C must be in [1, %d] (got %d)", 8 * PQ_TOPK_MAX, C);
  PQ_CHECK_ARG(k >= 1 && k <= PQ_TOPK_MAX, "k must be in [1, %d] (got %d)", PQ_TOPK_MAX, k);
  if (nq == 0) return PQ_OK;
  PQ_CHECK_ARG(qrot && cent_full && cand && out_scores && out_ids, "null pointer argument");
  cudaStream_t st = (cudaStream_t)stream;
  const size_t st_f = (bits <= 4) ? (size_t)d * 16 : (size_t)d + (size_t)(1 << bits) * 32;
  const size_t sm = align_up(st_f * 4, 16) + align_up((size_t)C, 2) * 8 +
                    BlockTopK::smem_bytes(BlockTopK::cap_for(k, kScanThreads));
  PQ_DISPATCH_B(bits, {
    auto kern = rerank_kernel<B_, B_>;
    rc = set_smem(kern, sm);
    if (rc) return rc;
    kern<<<nq, kScanThreads, sm, st>>>(packed, ldb, norms, n, d, qrot, cent_full, nullptr, nullptr,
                                       0, (const long long*)cand, C, k, row_offset, out_scores,
                                       (long long*)out_ids, 0);
  });
  PQ_LAUNCH_CHECK("rerank_kernel");
  return PQ_OK;
}

int pq_topk_merge(const float* in_s, const int64_t* in_ids, int parts, int nq, int kin, int k,
                  float* out_s, int64_t* out_ids, void* stream) {
  PQ_CHECK_ARG(parts >= 1 && kin >= 1 && nq >= 0, "bad merge shape");
  PQ_CHECK_ARG(k >= 1 && k <= PQ_TOPK_MAX && (long long)k <= (long long)kin * parts,
               "k must be in [1, min(%d, parts*kin)] (got %d)", PQ_TOPK_MAX, k);
  if (nq == 0) return PQ_OK;
  PQ_CHECK_ARG(in_s && in_ids && out_s && out_ids, "null pointer argument");
  return launch_merge(in_s, (const long long*)in_ids, parts, kin, kin, (long long)nq * kin, nq, k,
                      0, out_s, (long long*)out_ids, (cudaStream_t)stream);
}

static int util_grid(int64_t work) {
  int64_t g = (work + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 32;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

int pq_unpack_rows(const uint8_t* packed, int64_t ldb, int64_t n, int d, int bits, int shift,
                   uint8_t* out, void* stream) {
  int rc = check_corpus(packed, ldb, (const float*)1, n, d, bits);
  if (rc) return rc;
  PQ_CHECK_ARG(shift >= 0 && shift < bits, "shift out of range");
  if (n == 0) return PQ_OK;
  unpack_kernel<<<util_grid(n * d), 256, 0, (cudaStream_t)stream>>>(packed, ldb, nullptr, n, d,
                                                                     bits, shift, out);
  PQ_LAUNCH_CHECK("unpack_kernel");
  return PQ_OK;
}

int pq_unpack_at(const uint8_t* packed, int64_t ldb, const int64_t* idx, int64_t m, int d,
                 int bits, int shift, uint8_t* out, void* stream) {
  int rc = check_corpus(packed, ldb, (const float*)1, m > 0 ? 1 : 0, d, bits);
  if (rc) return rc;
  PQ_CHECK_ARG(shift >= 0 && shift < bits, "shift out of range");
  if (m == 0) return PQ_OK;
  PQ_CHECK_ARG(idx && out, "null pointer argument");
  unpack_kernel<<<util_grid(m * d), 256, 0, (cudaStream_t)stream>>>(
      packed, ldb, (const long long*)idx, m, d, bits, shift, out);
  PQ_LAUNCH_CHECK("unpack_kernel");
  return PQ_OK;
}

int pq_repack(const uint8_t* packed, int64_t ldb, int64_t n, int d, int bits, int target_bits,
              uint8_t* out, int64_t ldb_out, void* stream) {
  int rc = check_corpus(packed, ldb, (const float*)1, n, d, bits);
  if (rc) return rc;
  PQ_CHECK_ARG(target_bits >= 1 && target_bits <= bits && supported_bits(target_bits),
               "target_bits must be a supported width in 1-%d", bits);
  PQ_CHECK_ARG(ldb_out >= row_bytes(d, target_bits) && ldb_out % 16 == 0, "bad ldb_out");
  if (n == 0) return PQ_OK;
  pack_bits_kernel<<<util_grid(n * ldb_out), 256, 0, (cudaStream_t)stream>>>(
      packed, ldb, bits, bits - target_bits, nullptr, n, d, target_bits, out, ldb_out);
  PQ_LAUNCH_CHECK("pack_bits_kernel");
  return PQ_OK;
}

int pq_pack_codes(const uint8_t* codes, int64_t n, int d, int bits, uint8_t* out, int64_t ldb,
                  void* stream) {
  PQ_CHECK_ARG(supported_bits(bits), "bits must be one of 1,2,3,4,8 (got %d)", bits);
  PQ_CHECK_ARG(ldb >= row_bytes(d, bits) && ldb % 16 == 0, "bad ldb");
  if (n == 0) return PQ_OK;
  PQ_CHECK_ARG(codes && out, "null pointer argument");
  pack_bits_kernel<<<util_grid(n * ldb), 256, 0, (cudaStream_t)stream>>>(
      nullptr, 0, bits, 0, codes, n, d, bits, out, ldb);
  PQ_LAUNCH_CHECK("pack_bits_kernel");
  return PQ_OK;
}

}  // extern "C"
