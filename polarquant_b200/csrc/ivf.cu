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
  if constexpr (PairTab<B, P>::on)
    build_pair_tables<P>(qrot + (size_t)q * d, d, cent, st);
  else
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
  const int cap = BlockTopK::cap_for(K, blockDim.x);
  tk.init(reinterpret_cast<char*>(cstart + nprobe), K, cap);
  // Candidate lists up to 4 x blockDim entries compact by selection (no
  // sort until the end); larger ones by the bitonic sort.
  tk.sel = reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(cstart + nprobe) +
                                       BlockTopK::smem_bytes(cap));
  const bool select = cap <= 4 * (int)blockDim.x;
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
      const uint8_t* rp = cell_rows ? cell_rows + pos * ldb : packed + r * ldb;
      const float nv = cell_rows ? __ldg(cell_norms + pos) : __ldg(norms + r);
      if constexpr (PairTab<B, P>::on)
        sc = score_row_pair<P>(rp, d, st) * nv;
      else
        sc = score_row<B, P>(rp, d, st, st, st + d, lane) * nv;
    }
    tk.offer(valid, sc, r);
    if (select)
      tk.end_round_select<4>();
    else
      tk.end_round();
  }
  const size_t o = ((size_t)q * G + g) * K;
  tk.write(out_s + o, out_id + o, 0);
}


// ---------------------------------------------------------------------------
// CSR build (remex/ivf.py:216-224: stable argsort of the cell ids, bincount,
// cumsum) as a stable counting sort: the rows are cut into tiles; each tile
// counts its rows per cell; the counts are scanned per cell over the tiles and
// over the cells; then one warp per tile walks its rows in order, 32 at a
// time, and places each row at its cell's next slot (rows of one cell keep
// their order: stable).  Then the packed rows and norms are copied in CSR
// order.  tile_counts is cell-major: entry (c, t) at c * ntiles + t.
// ---------------------------------------------------------------------------

// Cells of at most this many fit the per-block shared counters.
constexpr int kCsrSmemCells = 16384;

__global__ void __launch_bounds__(256)
csr_hist_kernel(const uint16_t* __restrict__ cells, int64_t n, int n_cells, int64_t tile,
                int ntiles, int* __restrict__ tile_counts) {
  extern __shared__ int h[];
  const int t = blockIdx.x;
  const int64_t r0 = (int64_t)t * tile, r1 = min(n, r0 + tile);
  const bool sm = n_cells <= kCsrSmemCells;
  if (sm) {
    for (int i = threadIdx.x; i < n_cells; i += blockDim.x) h[i] = 0;
    __syncthreads();
  }
  for (int64_t r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
    const int c = cells[r];
    if (sm) atomicAdd(&h[c], 1);
    else atomicAdd(&tile_counts[(size_t)c * ntiles + t], 1);  // zeroed by the host
  }
  if (sm) {
    __syncthreads();
    for (int i = threadIdx.x; i < n_cells; i += blockDim.x)
      tile_counts[(size_t)i * ntiles + t] = h[i];
  }
}

// One warp per cell: exclusive scan of the cell's tile counts in place, and
// the cell's total.
__global__ void __launch_bounds__(256)
csr_tile_scan_kernel(int* __restrict__ tile_counts, int ntiles, int n_cells,
                     long long* __restrict__ counts) {
  const int lane = threadIdx.x & 31;
  const int c = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (c >= n_cells) return;
  int* row = tile_counts + (size_t)c * ntiles;
  long long run = 0;
  for (int b = 0; b < ntiles; b += 32) {
    const int i = b + lane;
    const int v = i < ntiles ? row[i] : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (i < ntiles) row[i] = (int)(run + x - v);
    run += __shfl_sync(0xffffffffu, x, 31);
  }
  if (lane == 0) counts[c] = run;
}

// offsets[0] = 0, offsets[c + 1] = offsets[c] + counts[c] (one block of 1024).
__global__ void __launch_bounds__(1024)
csr_offsets_kernel(const long long* __restrict__ counts, int n_cells,
                   long long* __restrict__ offsets) {
  __shared__ long long part[1024];
  const int per = (n_cells + 1023) / 1024;
  const int c0 = threadIdx.x * per, c1 = min(n_cells, c0 + per);
  long long s = 0;
  for (int c = c0; c < c1; ++c) s += counts[c];
  part[threadIdx.x] = s;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    const long long y = threadIdx.x >= o ? part[threadIdx.x - o] : 0;
    __syncthreads();
    part[threadIdx.x] += y;
    __syncthreads();
  }
  long long run = part[threadIdx.x] - s;  // exclusive prefix of this thread's chunk
  if (threadIdx.x == 0) offsets[0] = 0;
  for (int c = c0; c < c1; ++c) {
    run += counts[c];
    offsets[c + 1] = run;
  }
}

// One warp per tile: rows in order, 32 at a time; lanes with equal cells
// (__match_any_sync) take consecutive slots in lane order after the cell's
// running position, which the lowest such lane advances.
__global__ void __launch_bounds__(32)
csr_scatter_kernel(const uint16_t* __restrict__ cells, int64_t n, int64_t tile, int ntiles,
                   int* __restrict__ tile_prefix, const long long* __restrict__ offsets,
                   int n_cells, long long* __restrict__ sorted_idx) {
  extern __shared__ long long run_s[];
  const int t = blockIdx.x, lane = threadIdx.x;
  const int64_t r0 = (int64_t)t * tile, r1 = min(n, r0 + tile);
  const bool sm = n_cells <= kCsrSmemCells;
  if (sm) {
    for (int c = lane; c < n_cells; c += 32)
      run_s[c] = offsets[c] + tile_prefix[(size_t)c * ntiles + t];
    __syncwarp();
  }
  for (int64_t b = r0; b < r1; b += 32) {
    const int64_t r = b + lane;
    const bool valid = r < r1;
    const int c = valid ? (int)cells[r] : n_cells + lane;  // invalid lanes match nobody
    const unsigned peers = __match_any_sync(0xffffffffu, c);
    const int leader = __ffs(peers) - 1;
    const int rank = __popc(peers & ((1u << lane) - 1u));
    long long old = 0;
    if (valid && lane == leader) {
      if (sm) {
        old = run_s[c];
        run_s[c] = old + __popc(peers);
      } else {
        int* p = tile_prefix + (size_t)c * ntiles + t;
        old = offsets[c] + *p;
        *p += __popc(peers);
      }
    }
    old = __shfl_sync(0xffffffffu, old, leader);
    if (valid) sorted_idx[old + rank] = r;
    __syncwarp();
  }
}

// The packed rows (ldb bytes, a multiple of 16) and norms in CSR order: one
// warp per output row, 16 bytes per lane.
__global__ void __launch_bounds__(256)
csr_gather_rows_kernel(const uint8_t* __restrict__ packed, int64_t ldb,
                       const float* __restrict__ norms, const long long* __restrict__ sorted_idx,
                       int64_t n, uint8_t* __restrict__ cell_rows, float* __restrict__ cell_norms) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int chunks = (int)(ldb / 16);
  for (int64_t p = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < n;
       p += warps) {
    const long long r = sorted_idx[p];
    const uint4* src = reinterpret_cast<const uint4*>(packed + r * ldb);
    uint4* dst = reinterpret_cast<uint4*>(cell_rows + p * ldb);
    for (int i = lane; i < chunks; i += 32) dst[i] = __ldg(src + i);
    if (lane == 0) cell_norms[p] = __ldg(norms + r);
  }
}

static int64_t csr_tile(int64_t n, int n_cells) {
  // At least 8192 rows per tile, and few enough tiles that the count table
  // (n_cells x tiles ints) stays within 2^26 entries.
  int64_t t = 8192;
  const int64_t need = (n * (int64_t)n_cells + (1ll << 26) - 1) >> 26;
  if (t < need) t = (need + 31) / 32 * 32;
  return t;
}

}  // namespace pqb

using namespace pqb;

extern "C" {

size_t pq_ivf_csr_workspace_bytes(int64_t n, int n_bits) {
  if (n <= 0 || n_bits < 1 || n_bits > 16) return 256;
  const int n_cells = 1 << n_bits;
  const int64_t tile = csr_tile(n, n_cells);
  const int64_t ntiles = (n + tile - 1) / tile;
  return align_up((size_t)n_cells * ntiles * sizeof(int), 256) +
         (size_t)n_cells * sizeof(long long) + 512;
}

int pq_ivf_build_csr(const uint16_t* cells, int64_t n, int n_bits, int64_t* sorted_idx,
                     int64_t* offsets, const uint8_t* packed, int64_t ldb, const float* norms,
                     uint8_t* cell_rows, float* cell_norms, void* ws, size_t ws_bytes,
                     void* stream) {
  PQ_CHECK_ARG(n_bits >= 1 && n_bits <= 16, "n_bits must be 1-16, got %d", n_bits);
  PQ_CHECK_ARG(n >= 0 && n < (1ll << 31), "n=%lld out of range", (long long)n);
  PQ_CHECK_ARG(offsets, "null offsets");
  PQ_CHECK_ARG((cell_rows == nullptr) == (cell_norms == nullptr),
               "cell_rows and cell_norms must both be given or both be null");
  PQ_CHECK_ARG(cell_rows == nullptr || (packed && norms && ldb % 16 == 0 &&
                                        ((uintptr_t)packed & 15) == 0 &&
                                        ((uintptr_t)cell_rows & 15) == 0),
               "the CSR-order copy needs 16-byte aligned rows of a 16-byte stride");
  const int n_cells = 1 << n_bits;
  cudaStream_t st = (cudaStream_t)stream;
  if (n == 0) {
    PQ_CUDA_TRY(cudaMemsetAsync(offsets, 0, sizeof(int64_t) * (n_cells + 1), st));
    return PQ_OK;
  }
  PQ_CHECK_ARG(cells && sorted_idx, "null pointer argument");
  const size_t need = pq_ivf_csr_workspace_bytes(n, n_bits);
  if (!ws || ws_bytes < need)
    return fail(PQ_ERR_WORKSPACE, "pq_ivf_build_csr needs %zu workspace bytes, got %zu", need,
                ws_bytes);
  const int64_t tile = csr_tile(n, n_cells);
  const int ntiles = (int)((n + tile - 1) / tile);
  Carve cv(ws, ws_bytes);
  int* tile_counts = cv.take<int>((size_t)n_cells * ntiles);
  long long* counts = cv.take<long long>((size_t)n_cells);
  const bool sm = n_cells <= kCsrSmemCells;
  if (!sm)
    PQ_CUDA_TRY(cudaMemsetAsync(tile_counts, 0, sizeof(int) * (size_t)n_cells * ntiles, st));
  const size_t hsm = sm ? (size_t)n_cells * sizeof(int) : 0;
  int rc = set_smem(csr_hist_kernel, hsm);
  if (rc) return rc;
  csr_hist_kernel<<<ntiles, 256, hsm, st>>>(cells, n, n_cells, tile, ntiles, tile_counts);
  PQ_LAUNCH_CHECK("csr_hist_kernel");
  csr_tile_scan_kernel<<<(n_cells + 7) / 8, 256, 0, st>>>(tile_counts, ntiles, n_cells, counts);
  PQ_LAUNCH_CHECK("csr_tile_scan_kernel");
  csr_offsets_kernel<<<1, 1024, 0, st>>>(counts, n_cells, (long long*)offsets);
  PQ_LAUNCH_CHECK("csr_offsets_kernel");
  const size_t ssm = sm ? (size_t)n_cells * sizeof(long long) : 0;
  rc = set_smem(csr_scatter_kernel, ssm);
  if (rc) return rc;
  csr_scatter_kernel<<<ntiles, 32, ssm, st>>>(cells, n, tile, ntiles, tile_counts,
                                              (const long long*)offsets, n_cells,
                                              (long long*)sorted_idx);
  PQ_LAUNCH_CHECK("csr_scatter_kernel");
  if (cell_rows) {
    int64_t g = (n + 7) / 8;
    if (g > (int64_t)num_sms() * 16) g = (int64_t)num_sms() * 16;
    csr_gather_rows_kernel<<<(int)g, 256, 0, st>>>(packed, ldb, norms, (const long long*)sorted_idx,
                                                   n, cell_rows, cell_norms);
    PQ_LAUNCH_CHECK("csr_gather_rows_kernel");
  }
  return PQ_OK;
}

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

size_t pq_ivf_workspace_bytes(int64_t n, int nq, int nprobe, int splits, int candidates) {
  if (candidates > PQ_TOPK_MAX) return large_ivf_ws(n, nq, nprobe, candidates);
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
  PQ_CHECK_ARG(candidates >= 1, "candidates must be >= 1 (got %d)", candidates);
  PQ_CHECK_ARG(n < (1ll << 31), "n=%lld rows exceed one launch; shard the corpus", (long long)n);
  PQ_CHECK_ARG(k >= 1 && k <= candidates, "k must be in [1, candidates] (got %d)", k);
  if (nq == 0) return PQ_OK;
  PQ_CHECK_ARG(qrot && cent_coarse && sorted_idx && offsets && out_scores && out_ids && ws,
               "null pointer argument");
  PQ_CHECK_ARG(!rerank || cent_full, "null full-precision centroids");
  PQ_CHECK_ARG((cell_rows == nullptr) == (cell_norms == nullptr),
               "cell_rows and cell_norms must both be given or both be null");
  PQ_CHECK_ARG(cell_rows == nullptr || ((uintptr_t)cell_rows & 15) == 0,
               "cell_rows must be 16-byte aligned");
  const size_t need = pq_ivf_workspace_bytes(n, nq, nprobe, splits, candidates);
  if (ws_bytes < need)
    return fail(PQ_ERR_WORKSPACE, "pq_ivf_search needs %zu workspace bytes, got %zu", need,
                ws_bytes);
  cudaStream_t st = (cudaStream_t)stream;
  if (candidates > PQ_TOPK_MAX)
    return large_ivf(packed, ldb, norms, n, d, bits, coarse_precision, qrot, nq, cent_coarse,
                     cent_full, n_bits, mode, hyperplanes, (const long long*)sorted_idx,
                     (const long long*)offsets, cell_rows, cell_norms, nprobe, candidates, k,
                     rerank, out_scores, out_ids, ws, ws_bytes, st);
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
                    align_up(((size_t)2 * nprobe + 1) * sizeof(long long), 16) +
                    kTopkSelectWords * sizeof(uint32_t);
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
    return launch_merge_sorted(cs, ci, parts, candidates, (long long)parts * candidates, candidates, nq,
                        k, 0, out_scores, (long long*)out_ids, st);
  const size_t smr = rerank_smem(d, bits, candidates, k);
  PQ_DISPATCH_B(bits, {
    auto kern = rerank_kernel<B_, B_>;
    rc = set_smem(kern, smr);
    if (rc) return rc;
    kern<<<nq, kScanThreads, smr, st>>>(packed, ldb, norms, n, d, qrot, cent_full, cs, ci, parts,
                                        nullptr, candidates, k, 0, out_scores,
                                        (long long*)out_ids, 1);
  });
  PQ_LAUNCH_CHECK("rerank_kernel");
  return PQ_OK;
}

}  // extern "C"
