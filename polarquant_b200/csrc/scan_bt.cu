// Streaming ADC scan through byte tables (remex/core.py:597-636 search_adc
// semantics, one corpus pass per query) for 1-, 2-, 4- and 8-bit codes.
//
// One shared-memory lookup per code is the ceiling of a table-per-coordinate
// scan: at 32 lookups per SM cycle it cannot stream 4-bit codes much faster
// than ~0.7 of HBM even with nothing else to do.  Here every lookup covers a
// whole byte of the packed row: for byte position p and byte value e the
// table holds the sum of the products of every code packed in that byte,
//   T[p][e] = sum_t fl(q_rot[j_t] * cent[code_t(e) >> shift])
// (2 codes at 4 bits, 1 at 8, 4 at 2, 8 at 1; the products are the
// reference's np.outer table entries, remex/core.py:618, added in another
// order), so a row's score is sum_p T[p][row[p]] * norm: one lookup per byte.
//
// Tables: 1 KB per byte position, rb KB per query (768 KB at d=1536 4-bit),
// built in global memory by bt_table_kernel.  A block streams a contiguous
// range of rows in chunks of kBtChunk rows, slice-major: for each 64-byte
// column slice of the row it copies that slice's 64 KB of tables into shared
// memory (cp.async.bulk), streams the slice of the chunk's rows through a
// TMA ring (256 rows x 64 bytes per stage, 6 stages: ~96 KB in flight per
// SM, what HBM latency needs at full bandwidth), and adds each row's slice
// sum to a per-row partial in shared memory; after the last slice the
// chunk's rows are scored (partial * norm) into the block's top-K.
//
// A warp instruction covers two rows: lanes 0-15 take the 16 words of row A's
// slice, lanes 16-31 those of row B, which walk their word's bytes in the
// order 2, 3, 0, 1.  Byte i of word l' (byte position p = 4l' + i) has its
// 256 entries in bank (l' + 8i) mod 32, layer i & 1, so at every step the 16
// lanes of row A hit banks 8i .. 8i+15 and those of row B the other 16:
// conflict-free whatever the codes.  A warp takes 16 rows (8 pairs) per
// stage; the 16 lanes' partial sums of each row are reduced by a transposed
// butterfly.  No block-wide barrier per stage: each warp runs through the
// stages on its own, up to the ring depth apart.
#include "codes.cuh"
#include "tc.cuh"
#include "topk.cuh"

namespace pqb {

constexpr int kBtThreads = 512;                 // 16 warps
constexpr int kBtSlab = 64;                     // bytes of a row slice
constexpr int kBtRows = 256;                    // rows per stage (16 per warp)
constexpr int kBtStages = 6;                    // TMA ring depth
constexpr int kBtChunk = 8192;                  // rows per chunk (partials in shared memory)
constexpr int kBtTableBytes = kBtSlab * 256 * 4;  // 64 KB of tables per slice
constexpr int kBtTableCopies = 2;               // bulk copies per table slice (32 KB each)

// Word offset of entry e of byte position p (0..63) inside a slice's table.
__host__ __device__ __forceinline__ uint32_t bt_word(int p, int e) {
  const int l = p >> 2, i = p & 3;
  return (uint32_t)((l + 8 * i) & 31) + 32u * (uint32_t)(e + 256 * (i & 1));
}

// T[q][slice][word]: the byte tables of every query, in the shared-memory
// layout above.  One thread per (query, byte position, byte value).
template <int B>
__global__ void __launch_bounds__(256)
bt_table_kernel(const float* __restrict__ qrot, int nq, int d, int64_t rb, int nslices,
                const float* __restrict__ cent, int shift, float* __restrict__ tables) {
  constexpr int PER = 8 / B;  // codes per byte
  const int64_t per_q = (int64_t)nslices * kBtSlab * 256;
  const int64_t total = per_q * nq;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int q = (int)(t / per_q);
    const int64_t r = t - (int64_t)q * per_q;
    const int s = (int)(r / (kBtSlab * 256));
    const int pe = (int)(r - (int64_t)s * kBtSlab * 256);
    const int p = pe >> 8, e = pe & 255;
    const int64_t gb = (int64_t)s * kBtSlab + p;  // byte position in the row
    float v = 0.f;
    if (gb < rb) {
      const float* qv = qrot + (size_t)q * d;
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int64_t j = gb * PER + u;  // MSB-first: code u of the byte
        if (j < d) {
          const uint32_t code = ((uint32_t)e >> (8 - B * (u + 1))) & ((1u << B) - 1u);
          v = __fadd_rn(v, __fmul_rn(__ldg(qv + j), __ldg(cent + (code >> shift))));
        }
      }
    }
    tables[(size_t)q * per_q + (size_t)s * (kBtSlab * 256) + bt_word(p, e)] = v;
  }
}

__device__ __forceinline__ float bt_lds(uint32_t addr) {
  float v;
  asm("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint32_t bt_lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

// One 1-D bulk copy global -> shared completing on `bar` (no multicast).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}

// Half-warp partial sums of 8 row pairs -> the full sum of row
// 2 * pair + (lane >> 4), pair = bits 3..1 of the lane (in 2 lanes each).
__device__ __forceinline__ float bt_reduce_pairs(float (&p)[8], int lane) {
#pragma unroll
  for (int lvl = 0; lvl < 3; ++lvl) {
    const int half = 4 >> lvl;   // values kept after this level
    const int mask = 8 >> lvl;   // partner lane (within the half-warp)
    const bool hi = (lane & mask) != 0;
#pragma unroll
    for (int r = 0; r < half; ++r) {
      const float send = hi ? p[r] : p[r + half];
      const float keep = hi ? p[r + half] : p[r];
      p[r] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
    }
  }
  return p[0] + __shfl_xor_sync(0xffffffffu, p[0], 1);
}

__global__ void __launch_bounds__(kBtThreads, 1)
scan_bt_kernel(const __grid_constant__ CUtensorMap tmap, const float* __restrict__ norms,
               int64_t n, const float* __restrict__ tables, int nslices, int K,
               int64_t rows_per_block, int nblk, float* __restrict__ cand_s,
               long long* __restrict__ cand_id) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  constexpr uint32_t STAGE = kBtRows * kBtSlab;  // 16 KB
  constexpr int NW = kBtThreads / 32;
  const uint32_t raw = tc::smem_u32(smem_raw);
  // [table 128 KB][slab ring][partials kBtChunk f32][barriers + counters 128 B][top-k]
  const uint32_t tab = (raw + 1023u) & ~1023u;
  const uint32_t slabs = tab + kBtTableBytes;
  const uint32_t part_a = slabs + kBtStages * STAGE;
  float* part = reinterpret_cast<float*>(smem_raw + (part_a - raw));
  const uint32_t bars = part_a + kBtChunk * 4;
  uint8_t* gbars = smem_raw + (bars - raw);
  const uint32_t TBAR = bars + 8u * kBtStages;  // table slice landed
  int* slot_cnt = reinterpret_cast<int*>(gbars + 8 * (kBtStages + 1));  // warps done per slot
  int* slice_cnt = slot_cnt + kBtStages;                                // warps done with a slice
  int* slot_iss = slice_cnt + 1;                                        // copies issued per slot
  int* tab_iss = slot_iss + kBtStages;                                  // table copies issued
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tab_iss + 1);
  char* gtk = reinterpret_cast<char*>(gbars + 128);
  const int q = blockIdx.y, b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* qtab = tables + (size_t)q * nslices * (kBtTableBytes / 4);

  const int64_t r0 = (int64_t)b * rows_per_block;
  const int64_t r1 = min(n, r0 + rows_per_block);
  const int nchunks = (int)((r1 - r0 + kBtChunk - 1) / kBtChunk);
  constexpr int FULL_NS = kBtChunk / kBtRows;  // stages per slice of a full chunk
  auto chunk_stages = [&](int c) {
    const int64_t c0 = r0 + (int64_t)c * kBtChunk;
    const int64_t rows = min((int64_t)kBtChunk, r1 - c0);
    return (int)((rows + kBtRows - 1) / kBtRows);
  };
  const int total = (nchunks - 1) * FULL_NS * nslices + chunk_stages(nchunks - 1) * nslices;
  // Stage L of the sequence (chunk-major, then slice, then stage) -> TMA
  // coordinates of its slab.
  auto issue = [&](int L) {
    const int c = L / (FULL_NS * nslices);
    const int rem = L - c * FULL_NS * nslices;
    const int ns = chunk_stages(c);
    const int sl = rem / ns, t = rem - sl * ns;
    const int slot = L % kBtStages;
    const int64_t y = r0 + (int64_t)c * kBtChunk + (int64_t)t * kBtRows;
    ++slot_iss[slot];
    tc::mbar_arrive_expect_tx(bars + 8u * slot, STAGE);
    tc::tma_load_2d(slabs + (uint32_t)slot * STAGE, &tmap, sl * kBtSlab, (int)y,
                    bars + 8u * slot);
  };
  auto load_table = [&](int sl) {
    ++*tab_iss;
    tc::mbar_arrive_expect_tx(TBAR, (uint32_t)kBtTableBytes);
    const char* src = reinterpret_cast<const char*>(qtab) + (size_t)sl * kBtTableBytes;
#pragma unroll
    for (int u = 0; u < kBtTableCopies; ++u)
      bulk_load(tab + (uint32_t)u * (kBtTableBytes / kBtTableCopies),
                src + (size_t)u * (kBtTableBytes / kBtTableCopies),
                (uint32_t)(kBtTableBytes / kBtTableCopies), TBAR);
  };

  if (tid == 0) {
    for (int s = 0; s < kBtStages; ++s) {
      tc::mbar_init(bars + 8u * s, 1);
      slot_cnt[s] = 0;
      slot_iss[s] = 0;
    }
    tc::mbar_init(TBAR, 1);
    *slice_cnt = 0;
    *tab_iss = 0;
    *abort_flag = 0;
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmap);
  }
  BlockTopK tk;
  tk.init(gtk, K, BlockTopK::cap_for(K, kBtThreads));  // syncs: barriers ready
  if (tid == 0) {
    load_table(0);
    for (int L = 0; L < kBtStages && L < total; ++L) issue(L);
  }

  // Per lane: its word l' of the slice, the half-warp's row h, and for its
  // k-th lookup (byte i = k for row A, (k + 2) & 3 for row B) the address of
  // entry 0 -- layer i & 1 plus the bank (l' + 8i) mod 32; entry e is
  // 128 * e further.
  const int lw = lane & 15, h = lane >> 4;
  uint32_t tb[4], sel[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = h ? ((k + 2) & 3) : k;
    tb[k] = tab + 32768u * (uint32_t)(i & 1) + 4u * (uint32_t)((lw + 8 * i) & 31);
    sel[k] = 0x4440u + (uint32_t)i;
  }

  // No block-wide barrier per stage: each warp runs through the stages on its
  // own (up to the ring depth apart).  The last warp to finish a slot issues
  // the copy of the stage kBtStages later into it; the last warp to finish a
  // slice issues the copy of the next slice's table, which every warp waits
  // for before its first stage of that slice.  The block meets only at chunk
  // ends, to score the chunk's rows.
  int seq = 0, tcount = 0;
  for (int c = 0; c < nchunks; ++c) {
    const int64_t c0 = r0 + (int64_t)c * kBtChunk;
    const int ns = chunk_stages(c);
    for (int s = 0; s < nslices; ++s, ++tcount) {
      if (!tc::mbar_wait(TBAR, (uint32_t)tcount & 1u, abort_flag, tc::kErrWaitTmaFull)) {
        // Aborted: skip the work, keep the block's meeting points.
        seq += ns;
        continue;
      }
      for (int t = 0; t < ns; ++t, ++seq) {
        const int slot = seq % kBtStages;
        const bool ok = tc::mbar_wait(bars + 8u * slot, (uint32_t)(seq / kBtStages) & 1u,
                                      abort_flag, tc::kErrWaitTmaFull);
        if (ok) {
          // Warp w: rows w*16 .. w*16+15 of the stage as 8 pairs (2j, 2j+1);
          // lane: word lw of row 2j + h.
          const uint32_t rowa = slabs + (uint32_t)slot * STAGE +
                                (uint32_t)(warp * 16 + h) * kBtSlab + 4u * (uint32_t)lw;
          float p[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t w = bt_lds_u32(rowa + (uint32_t)(2 * j) * kBtSlab);
            // byte of w (PRMT isolates it) -> its entry, 128 bytes apart
            const float v0 = bt_lds(tb[0] + __byte_perm(w, 0u, sel[0]) * 128u);
            const float v1 = bt_lds(tb[1] + __byte_perm(w, 0u, sel[1]) * 128u);
            const float v2 = bt_lds(tb[2] + __byte_perm(w, 0u, sel[2]) * 128u);
            const float v3 = bt_lds(tb[3] + __byte_perm(w, 0u, sel[3]) * 128u);
            p[j] = (v0 + v1) + (v2 + v3);
          }
          const float sum = bt_reduce_pairs(p, lane);
          if ((lane & 1) == 0) {
            const int pr = (lane >> 1) & 7;  // the pair whose sum this lane holds
            const int lr = t * kBtRows + warp * 16 + 2 * pr + h;  // row within the chunk
            part[lr] = (s == 0) ? sum : part[lr] + sum;
          }
        }
        // This warp is done with the slot (its loads were consumed above).
        __syncwarp();
        if (lane == 0) {
          __threadfence_block();
          if (atomicAdd(&slot_cnt[slot], 1) == NW - 1) {
            slot_cnt[slot] = 0;
            __threadfence_block();
            if (!*abort_flag && seq + kBtStages < total) {
              asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
              issue(seq + kBtStages);
            }
          }
        }
      }
      // This warp is done with the slice's table.
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        if (atomicAdd(slice_cnt, 1) == NW - 1) {
          *slice_cnt = 0;
          __threadfence_block();
          const bool more = s + 1 < nslices || c + 1 < nchunks;
          if (!*abort_flag && more) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            load_table(s + 1 < nslices ? s + 1 : 0);
          }
        }
      }
    }
    // The chunk's rows are complete: score and offer them (block-wide).
    __syncthreads();
    const bool ok = !*abort_flag;
    const int64_t rows = min((int64_t)kBtChunk, r1 - c0);
    for (int base = 0; base < rows; base += kBtThreads) {
      const int lr = base + tid;
      const bool valid = ok && lr < rows;
      const float sc = valid ? part[lr] * __ldg(norms + c0 + lr) : 0.f;
      tk.offer(valid, sc, c0 + lr);
      tk.end_round();
    }
  }
  // After an abort, copies still in flight must land before the block exits:
  // every issued slab and table copy is waited for (bounded).
  __syncthreads();
  if (tid == 0 && *abort_flag) {
    volatile int never = 0;
    for (int s = 0; s < kBtStages; ++s)  // the phase of each slot's last copy
      if (slot_iss[s] > 0)
        tc::mbar_wait(bars + 8u * s, (uint32_t)(slot_iss[s] - 1) & 1u, &never,
                      tc::kErrWaitTmaFull);
    if (*tab_iss > 0)
      tc::mbar_wait(TBAR, (uint32_t)(*tab_iss - 1) & 1u, &never, tc::kErrWaitTmaFull);
  }
  __syncthreads();
  const size_t o = ((size_t)q * nblk + b) * K;
  tk.write(cand_s + o, cand_id + o, 0);
}

}  // namespace pqb

using namespace pqb;

// Queries per call up to which the byte-table scan is used (its tables take
// rb KB per query of workspace) and the smallest corpus (the tables' build and
// per-block loads are amortised over many rows).
constexpr int kBtMaxQueries = 64;
constexpr int64_t kBtMinRows = 1 << 18;
constexpr int kBtMaxK = 512;

// Workspace the byte tables of nq queries may need (sized for 8-bit rows of d
// bytes, the widest) when the byte-table scan can take the call; else 0.
static size_t bt_tables_bytes(int64_t n, int d, int nq) {
  if (nq < 1 || nq > kBtMaxQueries || n < kBtMinRows) return 0;
  const size_t slices = (size_t)(d + kBtSlab - 1) / kBtSlab;
  return (size_t)nq * slices * kBtTableBytes;
}

struct BtPlan {
  bool ok;
  int nslices, nblk;
  int64_t per, rb;
  size_t smem;
};

static BtPlan bt_plan(int64_t n, int d, int bits, int nq, int K, int64_t ldb, size_t tables_avail) {
  BtPlan p{};
  p.ok = false;
  if (!(bits == 1 || bits == 2 || bits == 4 || bits == 8) || K > kBtMaxK || ldb < kBtSlab ||
      nq > kBtMaxQueries || n < kBtMinRows)
    return p;
  p.rb = row_bytes(d, bits);
  p.nslices = (int)((p.rb + kBtSlab - 1) / kBtSlab);
  if ((size_t)nq * p.nslices * kBtTableBytes > tables_avail) return p;
  const size_t tk = BlockTopK::smem_bytes(BlockTopK::cap_for(K, kBtThreads));
  p.smem = 1024 + (size_t)kBtTableBytes + (size_t)kBtStages * kBtRows * kBtSlab +
           (size_t)kBtChunk * 4 + 128 + tk;
  if (p.smem > 227 * 1024) return p;
  // One block per SM: blocks per query so that nq * blocks fills whole waves
  // of the SMs (>= 95% of the last wave busy); never more blocks than the
  // candidate workspace holds (scan_blocks).
  const int64_t sms = num_sms();
  int64_t bq = 1;
  double best = -1.0;
  const int64_t hi = 4 * ((sms + nq - 1) / nq);
  for (int64_t c = 1; c <= hi; ++c) {
    const int64_t tot = c * nq;
    const double eff = (double)tot / (double)(((tot + sms - 1) / sms) * sms);
    if (eff > best + 1e-9) {
      best = eff;
      bq = c;
    }
    if (eff >= 0.95) break;
  }
  int64_t per = ((n + bq - 1) / bq + kBtRows - 1) / kBtRows * kBtRows;
  const int64_t gen = scan_rows_per_block(n, nq);
  if (per < gen) per = gen;
  p.per = per;
  p.nblk = (int)((n + per - 1) / per);
  p.ok = true;
  return p;
}

// Runs the byte-table scan when it covers the shape and `tables` has room;
// *used = false otherwise.  *nblk receives the per-query candidate lists written.
static int try_scan_bt(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                       int bits, int precision, const float* qrot, int nq, const float* cent,
                       int K, float* cand_s, long long* cand_id, void* tables,
                       size_t tables_bytes, cudaStream_t st, int* nblk, bool* used) {
  *used = false;
  if (!tables) return PQ_OK;
  const BtPlan p = bt_plan(n, d, bits, nq, K, ldb, tables_bytes);
  if (!p.ok) return PQ_OK;
  auto fn = get_encode_fn();
  if (!fn) return PQ_OK;
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)ldb, (cuuint64_t)n};
  cuuint64_t strides[1] = {(cuuint64_t)ldb};
  cuuint32_t box[2] = {(cuuint32_t)kBtSlab, (cuuint32_t)kBtRows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(packed), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  // No L2 promotion: a promoted fetch would also bring in
                  // the next column slice of each row, which is read only in
                  // the next slice pass (after the chunk's other rows) and
                  // by then evicted -- up to 2x the DRAM reads.
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PQ_ERR_CUDA, "cuTensorMapEncodeTiled (byte-table scan rows) failed (%d)", (int)r);
  float* tab = reinterpret_cast<float*>(tables);
  const int64_t entries = (int64_t)nq * p.nslices * kBtSlab * 256;
  int64_t g = (entries + 255) / 256;
  if (g > (int64_t)num_sms() * 32) g = (int64_t)num_sms() * 32;
  const int shift = bits - precision;
  switch (bits) {
#define PQ_BT_CASE(BB)                                                                          \
  case BB:                                                                                      \
    bt_table_kernel<BB><<<(int)g, 256, 0, st>>>(qrot, nq, d, p.rb, p.nslices, cent, shift, tab); \
    break;
    PQ_BT_CASE(1)
    PQ_BT_CASE(2)
    PQ_BT_CASE(4)
    PQ_BT_CASE(8)
#undef PQ_BT_CASE
    default:
      return PQ_OK;
  }
  PQ_LAUNCH_CHECK("bt_table_kernel");
  int rc = set_smem(scan_bt_kernel, p.smem);
  if (rc) return rc;
  scan_bt_kernel<<<dim3(p.nblk, nq), kBtThreads, p.smem, st>>>(map, norms, n, tab, p.nslices, K,
                                                              p.per, p.nblk, cand_s, cand_id);
  PQ_LAUNCH_CHECK("scan_bt_kernel");
  *nblk = p.nblk;
  *used = true;
  return PQ_OK;
}

extern "C" int pq_adc_scan_kernel(int64_t n, int d, int bits, int precision, int nq, int k,
                                  int64_t ldb) {
  if (k > PQ_TOPK_MAX) return 3;
  if (precision < 1 || precision > bits) return 1;
  if (bt_plan(n, d, bits, nq, k, ldb, bt_tables_bytes(n, d, nq)).ok) return 4;
  const S2Plan p = s2_plan(n, d, bits, precision, nq, k, ldb);
  return p.ok ? 2 : 1;
}
