/*
 * polarquant_b200 -- C ABI of the B200 (sm_100a) encode and ADC-search library.
 *
 * Drop-in boundary for the hot path of the `remex` package
 * (oaustegard/polarquant).  The reference is pure Python/NumPy, so it has no
 * FFI of its own; each entry point below replaces the NumPy expression named
 * in its comment, and the Python package `polarquant_b200` binds these
 * symbols through ctypes behind the reference's Quantizer / CompressedVectors
 * / PackedVectors / IVFCoarseIndex API.
 *
 * Conventions
 *  - Every pointer is device memory owned by the caller, except where noted.
 *  - Packed corpora use the reference's MSB-first row layout
 *    (remex/packing.py:18-75, row-padded as remex/core.py:203-223) with a
 *    device row stride `ldb` (bytes, a multiple of 16, >= packed bytes of one
 *    row); buffers holding packed rows carry >= 64 bytes of slack after the
 *    last row.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls are
 *    asynchronous: they enqueue work and return.
 *  - Return value: PQ_OK (0) or a negative PQ_ERR_* code; pq_last_error()
 *    gives the message of the last failure on the calling thread.  No C++
 *    exception crosses the ABI.
 *  - Scratch memory is caller-provided (`ws`, `ws_bytes`); the matching
 *    *_workspace_bytes() function gives the size needed.
 *  - Top-k outputs are ordered by score descending, ties by id ascending;
 *    unused slots hold id -1 and score -inf.
 */
#ifndef POLARQUANT_B200_H
#define POLARQUANT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PQ_OK 0
#define PQ_ERR_INVALID (-1)     /* bad argument (message says which) */
#define PQ_ERR_CUDA (-2)        /* CUDA runtime / launch failure */
#define PQ_ERR_WORKSPACE (-3)   /* workspace too small */
#define PQ_ERR_UNSUPPORTED (-4) /* shape outside what the kernels handle */
#define PQ_ERR_DEVICE (-5)      /* a kernel reported a device-side failure */

/* Largest k (or candidate count) of the fused top-k kernels. */
#define PQ_TOPK_MAX 2048

/* Library version (major*10000 + minor*100 + patch). */
int pq_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* pq_last_error(void);

/* Codes a kernel records in the device error word when one of its bounded
 * waits (~2 s of SM clock) runs out: the CTA stops, drains its in-flight
 * copies and MMAs (bounded), frees its TMEM and returns -- no trap, no hang. */
#define PQ_DEVICE_ERR_WAIT_TMA_FULL 101    /* a TMA copy never landed */
#define PQ_DEVICE_ERR_WAIT_STAGE_EMPTY 102 /* a pipeline stage was never released */
#define PQ_DEVICE_ERR_WAIT_ACC_FULL 103    /* an MMA accumulator never completed */
#define PQ_DEVICE_ERR_WAIT_ACC_EMPTY 104   /* an accumulator was never drained */
#define PQ_DEVICE_ERR_WAIT_SELFTEST 105    /* pq_selftest_wait_timeout */

/* Synchronises the current device and reports (then clears) the first
 * device-side failure recorded by a kernel whose bounded wait ran out:
 * *code = 0 when none.  Returns PQ_ERR_CUDA if the synchronisation fails. */
int pq_device_status(int* code);

/* Self-test of the bounded waits (no counterpart in the reference): one block
 * waits on an mbarrier that nothing arrives at, through the same wait routine
 * as the tensor-core kernels but with a limit of `limit_cycles` SM clock
 * cycles (1e3 .. 4e9).  The wait runs out, PQ_DEVICE_ERR_WAIT_SELFTEST is
 * recorded for pq_device_status() and the kernel returns normally. */
int pq_selftest_wait_timeout(int64_t limit_cycles, void* stream);

/* Number of kernels the library has launched in this process (all devices). */
int64_t pq_launch_count(void);

/* Packed bytes of one row of d codes at `bits` (remex/packing.py:130-150). */
int64_t pq_row_bytes(int d, int bits);

/* ---------------------------------------------------------------------------
 * Encode.  Replaces Quantizer.encode (remex/core.py:484-511) followed by the
 * row packing of PackedVectors.from_compressed (remex/core.py:203-223):
 *   norms = f32(sqrt(sum_f64(x^2)));  x_unit = x / max(norms, 1e-8)  (f32)
 *   codes = searchsorted(boundaries, x_unit @ R^T)   (side='left')
 *   packed rows (stride ldb) of the MSB-first code stream.
 * `planes` is the rotation prepared once per (R, d) by pq_prepare_rotation
 * (R * 2^14 split into fp16 hi/lo planes, pq_rotation_planes_bytes(d) bytes);
 * R itself (d x d f32) is read for the exact recomputation of coordinates
 * that land within 1e-6 of a boundary.
 * X: n x d f32 row-major; norms: n f32 out; boundaries: 2^bits - 1 f32.
 * Workspace: pq_encode_workspace_bytes(n, d) (rows are processed in chunks).
 * ------------------------------------------------------------------------- */
size_t pq_rotation_planes_bytes(int d);
int pq_prepare_rotation(const float* R, int d, void* planes, size_t planes_bytes, void* stream);
size_t pq_encode_workspace_bytes(int64_t n, int d);
int pq_encode(const float* X, int64_t n, int d, const float* R, const void* planes,
              const float* boundaries, int bits, uint8_t* packed, int64_t ldb, float* norms,
              void* ws, size_t ws_bytes, void* stream);

/* Tensor-core rotation Y = X @ R^T (f32) through the encode GEMM, with the
 * planes that pq_prepare_rotation made of R (same workspace as pq_encode):
 * the `X @ R.T` of remex/core.py:507 without the coding, for many rows at
 * once (pq_rotate below is the exact f64-accumulated path for queries). */
int pq_rotate_tc(const float* X, int64_t n, int d, const void* planes, float* Y, void* ws,
                 size_t ws_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Query rotation: Y = X @ R^T (nq x d, f32), i.e. q_rot = R @ q per query.
 * Replaces `self.R @ query` (remex/core.py:570, :615, :682; remex/ivf.py:249,
 * :331) and `queries @ self.R.T` (remex/core.py:759).  Exact f32 products
 * accumulated in f64, rounded once to f32.
 * ------------------------------------------------------------------------- */
int pq_rotate(const float* X, int64_t nq, int d, const float* R, float* Y, void* stream);

/* ---------------------------------------------------------------------------
 * Decode (remex/core.py:513-532): out = (cent[codes >> (bits-precision)] @ R)
 * * norms, n x d f32.  RT is R transposed (d x d f32, device); cent holds the
 * 2^precision centroids.  Workspace: pq_decode_workspace_bytes(n, d).
 * ------------------------------------------------------------------------- */
size_t pq_decode_workspace_bytes(int64_t n, int d);
int pq_decode(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d, int bits,
              int precision, const float* cent, const float* RT, float* out, void* ws,
              size_t ws_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * ADC scan + top-k.  Replaces, per query,
 *   table = np.outer(R @ q, centroids)                     (remex/core.py:615-618)
 *   scores = table[arange(d), codes >> shift].sum(1)*norms  (remex/core.py:792-859)
 *   argpartition/argsort top-k                              (remex/core.py:631-636)
 * for `search_adc` and (same scores, remex/core.py:534-580) `search`.
 *
 * packed/norms: n rows (stride ldb); qrot: nq x d rotated queries (f32);
 * cent: 2^precision centroids of the Matryoshka level (remex/core.py:882-901);
 * shift = bits - precision.  1 <= k <= n; k > PQ_TOPK_MAX (e.g. k >= n, the
 * reference's full-argsort case) takes a sort-based path one query at a time.
 * Output: nq x k, ids are row + row_offset.
 * ------------------------------------------------------------------------- */
size_t pq_adc_scan_workspace_bytes(int64_t n, int d, int nq, int k);
/* Which kernel pq_adc_scan runs for this shape (with the workspace that
 * pq_adc_scan_workspace_bytes gives): 4 = byte-table scan (1-, 2-, 4- and
 * 8-bit codes, rows of at most 1024 bytes, n >= 2^18, nq <= 64, k <= 512:
 * one lookup per packed byte; its workspace holds the byte tables, 1 KB per
 * byte position per query, and the per-slice row sums of up to 256 MB of
 * rows), 2 = TMA-staged streaming scan (4- and 8-bit codes, n >= 256,
 * ldb >= 128, table fits in shared memory), 1 = generic streaming scan,
 * 3 = full sort (k > PQ_TOPK_MAX).  Diagnostic.  A workspace smaller than
 * pq_adc_scan_workspace_bytes but holding the candidate lists is accepted:
 * the call then skips the byte-table scan. */
int pq_adc_scan_kernel(int64_t n, int d, int bits, int precision, int nq, int k, int64_t ldb);
int pq_adc_scan(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                int bits, int precision, const float* qrot, int nq, const float* cent, int k,
                int64_t row_offset, float* out_scores, int64_t* out_ids, void* ws,
                size_t ws_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Batched ADC on the tensor cores (tcgen05): scores of nq queries against
 * all n rows as one GEMM over decoded code tiles.  Replaces
 * Quantizer.search_batch (remex/core.py:721-778: `Q_rot @ X_hat_rot.T *
 * norms` and the per-row argpartition/argsort).  For d >= 1024 and 2-, 4- or
 * 8-bit codes (k <= 224) the GEMM runs on int8 digit planes of 16-bit fixed
 * point and keeps the top k + 32 candidates per query, which are rescored
 * with the f32 table sums of pq_adc_scan and cut to k; otherwise an fp16
 * hi/lo split (three MMAs per K step, f32 accumulation) with the exact top-k
 * fused in the epilogue.  Scores equal pq_adc_scan's up to f32 summation order.
 * Same arguments and output as pq_adc_scan; 1 <= k <= 256, k <= n.
 * ------------------------------------------------------------------------- */
size_t pq_adc_batch_workspace_bytes(int64_t n, int d, int nq, int k);
/* Which kernel pq_adc_batch runs for this shape: 1 = int8 CTA-pair kernel
 * (candidates rescored exactly), 2 = fp16 hi/lo CTA-pair kernel, 3 = fp16
 * one-CTA kernel.  Diagnostic (queries the device's cluster occupancy). */
int pq_adc_batch_kernel(int64_t n, int d, int bits, int precision, int k, int64_t ldb);
int pq_adc_batch(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                 int bits, int precision, const float* qrot, int nq, const float* cent, int k,
                 int64_t row_offset, float* out_scores, int64_t* out_ids, void* ws,
                 size_t ws_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Allocation-free variant of pq_adc_scan.  No counterpart in the reference:
 * it exists for callers that cannot allocate device memory -- hosts that
 * reserve the GPU's memory for their own pool up front, and latency-critical
 * paths that cannot pay for cudaMalloc/cudaFree (which may synchronise the
 * device).  The caller passes only inputs and outputs; the scan's scratch is
 * a built-in device array of pq_adc_scan_noalloc_scratch_bytes() (16 MiB)
 * that every GPU loading the library holds until the process exits.  A call
 * is accepted when the scan's candidate lists fit in it, else rejected with
 * PQ_ERR_WORKSPACE (and k > PQ_TOPK_MAX with PQ_ERR_INVALID): the scan splits
 * the rows into about 8 blocks per SM in total, over all queries, each
 * keeping k candidates of 12 bytes, so on corpora of more than about 2.4
 * million rows the limit is k <= ~16 MiB / (12 * 8 * SMs), i.e. k <= ~1,180
 * on a 148-SM B200 whatever the query count; smaller corpora (fewer blocks)
 * allow k up to PQ_TOPK_MAX.  The byte-table scan runs when the rest of the
 * array also holds its tables and partial sums, else a scan that needs no
 * more space (as pq_adc_scan does with a workspace smaller than
 * pq_adc_scan_workspace_bytes).  The first call on each device
 * (and the first after the device's context is re-created) looks up the
 * array's device address (cudaGetSymbolAddress) and should come before any
 * stream capture.  All calls on a device share the array, so calls that
 * overlap on the GPU race and must be serialised by the caller.  Arguments
 * and results are those of pq_adc_scan.
 * ------------------------------------------------------------------------- */
size_t pq_adc_scan_noalloc_scratch_bytes(void);
int pq_adc_scan_noalloc(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                        int bits, int precision, const float* qrot, int nq, const float* cent,
                        int k, int64_t row_offset, float* out_scores, int64_t* out_ids,
                        void* stream);

/* ---------------------------------------------------------------------------
 * Two-stage Matryoshka search.  Replaces Quantizer.search_twostage
 * (remex/core.py:638-719): coarse ADC at `coarse_precision` over all rows,
 * top-`candidates` (unordered, any tie order), then full-precision rescoring
 * sum_j q_rot[j]*cent_full[code_j]*norm of those rows, top-k.
 * 1 <= candidates <= n, k <= candidates; more than PQ_TOPK_MAX candidates
 * take a sort-based path one query at a time (every row's coarse score
 * sorted, the first `candidates` rescored and sorted).
 * cent_coarse: 2^coarse_precision centroids; cent_full: 2^bits centroids.
 * With candidates <= 256, batches of >= 64 queries (>= 8 on corpora of at
 * least 2^20 rows) run the coarse stage on the tensor cores (as
 * pq_adc_batch); other batches use the streaming scan.
 * ------------------------------------------------------------------------- */
size_t pq_twostage_workspace_bytes(int64_t n, int d, int nq, int candidates);
int pq_twostage(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                int bits, int coarse_precision, const float* qrot, int nq,
                const float* cent_coarse, const float* cent_full, int candidates, int k,
                int64_t row_offset, float* out_scores, int64_t* out_ids, void* ws,
                size_t ws_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Full-precision rescoring of given rows + top-k (stage 2 of
 * remex/core.py:706-719 and remex/ivf.py:422-436).  cand: nq x C global row
 * ids; the local row is id - row_offset and ids outside this shard's
 * [row_offset, row_offset + n) (or < 0) are skipped, so a row-sharded corpus
 * reranks each candidate on the rank that owns it.  Output ids are global.
 * ------------------------------------------------------------------------- */
int pq_rerank(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
              int bits, const float* qrot, int nq, const float* cent_full, const int64_t* cand,
              int C, int k, int64_t row_offset, float* out_scores, int64_t* out_ids,
              void* stream);

/* ---------------------------------------------------------------------------
 * IVF coarse index (remex/ivf.py).  mode 0 = 'lsh', 1 = 'rotated_prefix'.
 * pq_ivf_cell_ids: cell id (uint16) of every row from the MSBs of its codes
 *   (remex/ivf.py:162-214); lsh projections onto hyperplanes (n_bits x d f32)
 *   are summed exactly in f64.
 * pq_ivf_probe: per query the nprobe cells closest in Hamming distance to the
 *   query cell, ties by cell id (remex/ivf.py:230-265); probe is nq x nprobe.
 * pq_ivf_search: IVFCoarseIndex.search_coarse (rerank = 0: top-k of the coarse
 *   ADC scores over the probed cells' rows, remex/ivf.py:301-374) or
 *   .search_twostage (rerank = 1: top-`candidates` coarse rows, full-precision
 *   rescoring, top-k, remex/ivf.py:376-436).  sorted_idx/offsets: the CSR
 *   layout (rows grouped by cell, offsets n_cells + 1).  cell_rows/cell_norms
 *   (optional, both or neither): the packed rows (stride ldb, >= 64 bytes of
 *   slack) and norms copied in CSR order, so each probed cell is read as one
 *   contiguous run; without them rows are gathered through sorted_idx.  Each
 *   query's probed rows are split into `splits` equal groups, one block and
 *   one candidate list each.  Slots past a query's candidate count hold id -1.
 *   candidates (the coarse k of search_coarse) may exceed PQ_TOPK_MAX: such
 *   calls sort each query's probed rows by coarse score instead of keeping a
 *   fused top-C, and synchronise `stream` once to read the probed-row counts.
 *   Workspace: pq_ivf_workspace_bytes(n, nq, nprobe, splits, C).
 * ------------------------------------------------------------------------- */
int pq_ivf_cell_ids(const uint8_t* packed, int64_t ldb, int64_t n, int d, int bits, int n_bits,
                    int mode, const float* hyperplanes, uint16_t* cells, void* stream);
int pq_ivf_probe(const float* qrot, int nq, int d, int n_bits, int mode, const float* hyperplanes,
                 int nprobe, int* probe, int* query_cells, void* stream);
/* CSR layout of the cell ids (remex/ivf.py:216-224: sorted_idx =
 * argsort(cell_ids, kind="stable"), offsets = [0, cumsum(bincount)]) by a
 * stable counting sort on the device: sorted_idx (n int64), offsets
 * (2^n_bits + 1 int64).  With cell_rows/cell_norms (both or neither) the
 * packed rows (stride ldb, 16-byte aligned) and norms are also copied in CSR
 * order (the layout pq_ivf_search reads; no reference counterpart).
 * Workspace: pq_ivf_csr_workspace_bytes(n, n_bits). */
size_t pq_ivf_csr_workspace_bytes(int64_t n, int n_bits);
int pq_ivf_build_csr(const uint16_t* cells, int64_t n, int n_bits, int64_t* sorted_idx,
                     int64_t* offsets, const uint8_t* packed, int64_t ldb, const float* norms,
                     uint8_t* cell_rows, float* cell_norms, void* ws, size_t ws_bytes,
                     void* stream);
size_t pq_ivf_workspace_bytes(int64_t n, int nq, int nprobe, int splits, int candidates);
int pq_ivf_search(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                  int bits, int coarse_precision, const float* qrot, int nq,
                  const float* cent_coarse, const float* cent_full, int n_bits, int mode,
                  const float* hyperplanes, const int64_t* sorted_idx, const int64_t* offsets,
                  const uint8_t* cell_rows, const float* cell_norms, int nprobe, int splits,
                  int candidates, int k, int rerank, float* out_scores, int64_t* out_ids,
                  void* ws, size_t ws_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * 1-bit popcount coarse scorer.  The reference recommends this coarse tier
 * for very large corpora (bench/RESULTS.md:153-161: "popcount(query_signs
 * XOR coarse_signs) -- no Lloyd-Max lookup needed") but ships no code for
 * it, so its semantics are defined here:
 *   score(row) = d - 2 * popcount(query_signs XOR row_signs), an integer in
 *   [-d, d] (the +-1 inner product of the sign vectors), where row_signs are
 *   the MSBs of the row's codes (its 1-bit Matryoshka level) and query bit j
 *   is q_rot[j] > 0; top-k by score descending, ties by row ascending.
 * signs: the corpus's 1-bit rows (MSB-first bits, e.g. pq_repack to 1 bit),
 * stride ldb (a multiple of 16, >= ceil(d / 128) * 16).  k <= PQ_TOPK_MAX.
 * pq_hamming_twostage: the top `candidates` (<= PQ_TOPK_MAX) by that score,
 * rescored at full precision as pq_twostage's second stage
 * (remex/core.py:706-719), top-k.  Workspace:
 * pq_hamming_workspace_bytes(n, nq, k or candidates).
 * ------------------------------------------------------------------------- */
size_t pq_hamming_workspace_bytes(int64_t n, int nq, int k);
int pq_hamming_scan(const uint8_t* signs, int64_t ldb, int64_t n, int d, const float* qrot,
                    int nq, int k, int64_t row_offset, float* out_scores, int64_t* out_ids,
                    void* ws, size_t ws_bytes, void* stream);
int pq_hamming_twostage(const uint8_t* signs, int64_t ldb_signs, const uint8_t* packed,
                        int64_t ldb, const float* norms, int64_t n, int d, int bits,
                        const float* qrot, int nq, const float* cent_full, int candidates, int k,
                        int64_t row_offset, float* out_scores, int64_t* out_ids, void* ws,
                        size_t ws_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Merge of per-part top-k lists: in_s/in_ids are parts x nq x kin (as written
 * by the per-rank scans, ids already global); out is nq x k, k <= kin*parts,
 * k <= PQ_TOPK_MAX.  Used after the NCCL all-gather of the row-sharded search.
 * ------------------------------------------------------------------------- */
int pq_topk_merge(const float* in_s, const int64_t* in_ids, int parts, int nq, int kin, int k,
                  float* out_s, int64_t* out_ids, void* stream);

/* ---------------------------------------------------------------------------
 * Packed-row utilities (remex/core.py:161-201, :254-293).
 * pq_unpack_rows: codes (n x d uint8, row stride d) = row codes >> shift.
 * pq_unpack_at: same for rows idx[0..m) (gather).
 * pq_repack: Matryoshka at_precision(target_bits): rows re-packed at
 *   target_bits from codes >> (bits - target_bits); out stride ldb_out.
 * pq_pack_codes: pack an (n x d) uint8 code matrix into rows of stride ldb.
 * ------------------------------------------------------------------------- */
int pq_unpack_rows(const uint8_t* packed, int64_t ldb, int64_t n, int d, int bits, int shift,
                   uint8_t* out, void* stream);
int pq_unpack_at(const uint8_t* packed, int64_t ldb, const int64_t* idx, int64_t m, int d,
                 int bits, int shift, uint8_t* out, void* stream);
int pq_repack(const uint8_t* packed, int64_t ldb, int64_t n, int d, int bits, int target_bits,
              uint8_t* out, int64_t ldb_out, void* stream);
int pq_pack_codes(const uint8_t* codes, int64_t n, int d, int bits, uint8_t* out, int64_t ldb,
                  void* stream);

#ifdef __cplusplus
}
#endif

#endif /* POLARQUANT_B200_H */
