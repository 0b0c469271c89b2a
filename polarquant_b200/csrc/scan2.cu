// Streaming ADC scan for 4- and 8-bit codes, staged through shared memory by
// TMA (remex/core.py:597-636 search_adc semantics, one corpus pass per query).
//
// Each block streams a contiguous range of rows, 256 rows (one per thread) at a
// time, as 128-byte column slabs: TMA copies a 256-row x 128-byte box of the
// packed corpus into shared memory with 128-byte swizzle (16-byte chunk c of
// row r lands at chunk c ^ (r % 8)), so the 8 threads of a quarter-warp that
// read chunk c of 8 consecutive rows hit 8 different bank groups.  Several
// slabs are in flight per block; a thread keeps its row's partial sums in
// registers across the slabs of the row.  Bytes past the row (or past the last
// row) arrive as zeros and score 0 (their table entries are zero).
//
// Table mode (precision P <= 4): T[j][c] = fl(q_rot[j] * cent[c]), the
// reference's np.outer table (remex/core.py:618), 16 floats (64 bytes) per
// coordinate, in shared memory.  The byte offset of T[j][code] inside its
// 256-byte page ((j % 4) * 64 + code * 4) is formed for four codes at once
// with a shift, a mask and an OR, and spliced into the table address with one
// PRMT; the page number is a compile-time offset.  A code costs PRMT + LDS +
// FADD.  All lanes read the same coordinate at once, so the lookups are
// bank-conflict free.
//
// Direct mode (8-bit codes, P = 5..8): cent[c] replicated per lane
// (C[c][lane], 128 bytes per code: conflict free), q_rot[j] read four at a
// time with a broadcast load, products fused into the sum.
#include "codes.cuh"
#include "tc.cuh"
#include "topk.cuh"

namespace pqb {

constexpr int kS2Rows = 256;     // rows per tile
constexpr int kS2Threads = 512;  // two threads per row
constexpr int kS2Slab = 128;  // bytes per row per slab

// Table lookups: the table is written once before the block's first
// __syncthreads and only read afterwards, so these loads may be scheduled
// freely (their addresses depend on slab data read after the copy's wait).
__device__ __forceinline__ float lds_f32(uint32_t addr) {
  float v;
  asm("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint4 lds_u128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Low address bytes of the table entries of the four codes in word w (one per
// byte lane k): code * 4 (shifted down to precision P) OR'd with the entry's
// position inside its 256-byte page, `pos` (one byte per lane k, see below).
template <int B, int P, bool HIGH>
__device__ __forceinline__ uint32_t code_offsets(uint32_t w, uint32_t pos) {
  constexpr uint32_t rep = 0x01010101u;
  if constexpr (B == 8) {
    constexpr uint32_t m = ((((1u << P) - 1u) << 2)) * rep;
    return ((w >> (6 - P)) & m) | pos;  // (byte >> (8 - P)) << 2
  } else {
    constexpr int sh = B - P;  // 0..3
    constexpr uint32_t m = ((15u >> sh) << 2) * rep;
    if constexpr (HIGH) {
      return ((w >> (2 + sh)) & m) | pos;
    } else {
      uint32_t v;
      if constexpr (sh <= 2) v = (w << (2 - sh)) & m;
      else v = (w >> (sh - 2)) & m;
      return v | pos;
    }
  }
}

// Table position of T[j][c]: j * 64 + c * 4 bytes, except that in the second
// half of each slab (the half read by the odd half-warps) the two 64-byte
// rows of each 128-byte pair are swapped, so the two half-warps of a warp,
// which look up coordinates of equal parity at the same time, read opposite
// halves of the 32 banks.
__host__ __device__ __forceinline__ int s2_tab_index(int j, int c, int cpr) {
  const int t = j * 16 + c;
  return ((j % cpr) >= cpr / 2) ? (t ^ 16) : t;
}

// The query's table in shared memory (all threads of the block).  Table mode
// (P <= 4): T[j][c] = fl(q_rot[j] * cent[c]) at s2_tab_index(j, c).  Direct
// mode: cent[c] replicated per lane, then q_rot per slab as
// [first half][4 pad][second half][4 pad] (CPR + 8 floats), so the two
// half-warps' broadcast reads fall in different banks.
template <int B, int P>
__device__ __forceinline__ void s2_fill_table(float* gtab, const float* __restrict__ qv,
                                              const float* __restrict__ cent, int d, int slabs) {
  constexpr int CPR = kS2Slab * 8 / B;
  const int jmax = slabs * CPR;
  if constexpr (P <= 4) {
    for (int i = threadIdx.x; i < jmax * 16; i += blockDim.x) {
      const int j = i >> 4, c = i & 15;
      gtab[s2_tab_index(j, c, CPR)] =
          (j < d && c < (1 << P)) ? __fmul_rn(__ldg(qv + j), __ldg(cent + c)) : 0.f;
    }
  } else {
    for (int i = threadIdx.x; i < (1 << P) * 32; i += blockDim.x) gtab[i] = __ldg(cent + (i >> 5));
    float* Q = gtab + (1 << P) * 32;
    for (int i = threadIdx.x; i < jmax; i += blockDim.x) {
      const int sl = i / CPR, jl = i % CPR;
      Q[sl * (CPR + 8) + jl + ((jl >= CPR / 2) ? 4 : 0)] = (i < d) ? __ldg(qv + i) : 0.f;
    }
  }
}

// Adds the row's partial sums over one 128-byte slab (two threads per row:
// half h of the slab) to a0..a3.  buf: shared address of the row's slab in the
// stage; tab: the query table; the rest as in scan2_kernel.
template <int B, int P>
__device__ __forceinline__ void s2_slab(uint32_t buf, uint32_t swz, uint32_t tab, int slab, int h,
                                        int lane, float& a0, float& a1, float& a2, float& a3) {
  constexpr bool TABLE = P <= 4;
  constexpr int CPR = kS2Slab * 8 / B;
  const uint32_t pos_hi = h ? 0xC040C040u : 0x80008000u;
  const uint32_t pos_lo = h ? 0x80008000u : 0xC040C040u;
  const uint32_t pos_b = h ? 0x80C00040u : 0xC0804000u;
  if constexpr (TABLE) {
    // 256-aligned base of this half's table pages
    const uint32_t tbs = tab + (uint32_t)(slab * CPR) * 64u + (uint32_t)h * (CPR / 2) * 64u;
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      const uint32_t c = (uint32_t)(4 * h + cc);
      const uint4 v = lds_u128(buf + ((c ^ swz) << 4));
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if constexpr (B == 4) {
          const uint32_t oh = code_offsets<4, P, true>(w[i], pos_hi);
          const uint32_t ol = code_offsets<4, P, false>(w[i], pos_lo);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t pg = 256u * (uint32_t)(8 * cc + 2 * i + (k >> 1));
            const uint32_t sel = 0x7650u | (uint32_t)k;
            const float th = lds_f32(__byte_perm(oh, tbs, sel) + pg);
            const float tl = lds_f32(__byte_perm(ol, tbs, sel) + pg);
            if (k & 1) { a1 += th; a3 += tl; } else { a0 += th; a2 += tl; }
          }
        } else {
          const uint32_t o = code_offsets<8, P, true>(w[i], pos_b);
          const uint32_t pg = 256u * (uint32_t)(4 * cc + i);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float t = lds_f32(__byte_perm(o, tbs, 0x7650u | (uint32_t)k) + pg);
            if (k == 0) a0 += t; else if (k == 1) a1 += t; else if (k == 2) a2 += t; else a3 += t;
          }
        }
      }
    }
  } else {
    const uint32_t cb = tab + (uint32_t)lane * 4u;
    const uint32_t qb = tab + (uint32_t)(1 << P) * 128u +
                        (uint32_t)(slab * (CPR + 8) + h * (CPR / 2 + 4)) * 4u;
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      const uint32_t c = (uint32_t)(4 * h + cc);
      const uint4 v = lds_u128(buf + ((c ^ swz) << 4));
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 qq = lds_u128(qb + (uint32_t)(16 * cc + 4 * i) * 4u);
        const float qf[4] = {__uint_as_float(qq.x), __uint_as_float(qq.y),
                             __uint_as_float(qq.z), __uint_as_float(qq.w)};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t code = (w[i] >> (8 * k + 8 - P)) & ((1u << P) - 1u);
          const float cv = lds_f32(cb + code * 128u);
          if (k == 0) a0 = fmaf(qf[k], cv, a0);
          else if (k == 1) a1 = fmaf(qf[k], cv, a1);
          else if (k == 2) a2 = fmaf(qf[k], cv, a2);
          else a3 = fmaf(qf[k], cv, a3);
        }
      }
    }
  }
}

template <int B, int P>
__global__ void __launch_bounds__(kS2Threads, 1)
scan2_kernel(const __grid_constant__ CUtensorMap tmap, const float* __restrict__ norms,
             int64_t n, int d, const float* __restrict__ qrot, const float* __restrict__ cent,
             int K, int64_t rows_per_block, int nblk, int slabs, int stages, int lut_bytes,
             float* __restrict__ cand_s, long long* __restrict__ cand_id) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  constexpr uint32_t STAGE = kS2Rows * kS2Slab;
  const uint32_t raw = tc::smem_u32(smem_raw);
  // [slab buffers, 1024-aligned][table][8 x 8-byte barriers][top-k buffer]
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  const uint32_t tab = sbase + (uint32_t)stages * STAGE;
  float* gtab = reinterpret_cast<float*>(smem_raw + (tab - raw));
  const uint32_t bars = tab + (uint32_t)lut_bytes;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem_raw + (bars - raw) + 56);
  char* gtk = reinterpret_cast<char*>(smem_raw + (bars - raw) + 64);
  const int q = blockIdx.y, b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31;
  const float* qv = qrot + (size_t)q * d;
  s2_fill_table<B, P>(gtab, qv, cent, d, slabs);
  if (tid == 0) {
    for (int s = 0; s < stages; ++s) tc::mbar_init(bars + 8u * s, 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmap);
  }
  BlockTopK tk;
  tk.init(gtk, K, BlockTopK::cap_for(K, kS2Threads));  // syncs: table and barriers ready

  const int64_t r0 = (int64_t)b * rows_per_block;
  const int64_t r1 = min(n, r0 + rows_per_block);
  const int tiles = (int)((r1 - r0 + kS2Rows - 1) / kS2Rows);
  const int total = tiles * slabs;
  int issued = 0, confirmed = 0;  // thread 0's copy bookkeeping
  if (tid == 0) {
    for (; issued < stages && issued < total; ++issued) {
      const int s = issued % stages;
      tc::mbar_arrive_expect_tx(bars + 8u * s, STAGE);
      tc::tma_load_2d(sbase + (uint32_t)s * STAGE, &tmap, (issued % slabs) * kS2Slab,
                      (int)(r0 + (int64_t)(issued / slabs) * kS2Rows), bars + 8u * s);
    }
  }

  // Two threads per row: the row's first 64 bytes of each slab go to the even
  // half-warp (h = 0), the last 64 to the odd one (h = 1).
  const int h = lane >> 4;
  const int rt = (tid >> 5) * 16 + (lane & 15);  // row within the tile
  const uint32_t swz = (uint32_t)(rt & 7);
  const uint32_t rowoff = (uint32_t)rt * kS2Slab;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  bool ok = true;
  int slab = 0;
  for (int it = 0; it < total; ++it) {
    const int s = it % stages;
    if (ok) {
      ok = tc::mbar_wait(bars + 8u * s, (uint32_t)(it / stages) & 1u, abort_flag,
                         tc::kErrWaitTmaFull);
      if (ok && tid == 0) confirmed = it + 1;
    }
    if (ok) {
      s2_slab<B, P>(sbase + (uint32_t)s * STAGE + rowoff, swz, tab, slab, h, lane, a0, a1, a2,
                    a3);
    }
    __syncthreads();  // every thread is done with stage s
    if (tid == 0 && ok && issued < total) {
      const int sn = issued % stages;  // == s
      tc::mbar_arrive_expect_tx(bars + 8u * sn, STAGE);
      tc::tma_load_2d(sbase + (uint32_t)sn * STAGE, &tmap, (issued % slabs) * kS2Slab,
                      (int)(r0 + (int64_t)(issued / slabs) * kS2Rows), bars + 8u * sn);
      ++issued;
    }
    if (++slab == slabs) {
      slab = 0;
      const float part = (a0 + a1) + (a2 + a3);
      const float other = __shfl_xor_sync(0xffffffffu, part, 16);
      const int64_t row = r0 + (int64_t)(it / slabs) * kS2Rows + rt;
      const bool valid = ok && h == 0 && row < r1;
      const float sc = valid ? (part + other) * __ldg(norms + row) : 0.f;
      tk.offer(valid, sc, row);
      tk.end_round();
      a0 = a1 = a2 = a3 = 0.f;
    }
  }
  // After an abort, copies still in flight must land before the block exits.
  if (tid == 0) {
    volatile int never = 0;
    for (int it = confirmed; it < issued; ++it)
      tc::mbar_wait(bars + 8u * (it % stages), (uint32_t)(it / stages) & 1u, &never,
                    tc::kErrWaitTmaFull);
  }
  __syncthreads();
  const size_t o = ((size_t)q * nblk + b) * K;
  tk.write(cand_s + o, cand_id + o, 0);
}


}  // namespace pqb

using namespace pqb;

// Layout of one scan2 launch; ok == false when the shape is not covered.
struct S2Plan {
  bool ok;
  int slabs, stages, lut_bytes, nblk;
  int64_t per;
  size_t smem;
};

static S2Plan s2_plan(int64_t n, int d, int bits, int precision, int nq, int K, int64_t ldb) {
  S2Plan p{};
  p.ok = false;
  if (!(bits == 4 || bits == 8) || n < kS2Rows || ldb < kS2Slab || K > PQ_TOPK_MAX) return p;
  const int64_t rb = row_bytes(d, bits);
  p.slabs = (int)((rb + kS2Slab - 1) / kS2Slab);
  const int jmax = p.slabs * (kS2Slab * 8 / bits);
  if (precision <= 4) p.lut_bytes = (int)align_up((size_t)jmax * 64, 1024);
  else p.lut_bytes = (int)align_up(((size_t)(1 << precision) * 32 + (size_t)p.slabs * ((kS2Slab * 8 / bits) + 8)) * 4, 1024);
  const size_t tk = BlockTopK::smem_bytes(BlockTopK::cap_for(K, kS2Threads));
  const size_t fixed = 1024 + (size_t)p.lut_bytes + 64 + tk;
  const size_t cap = 227 * 1024;
  int st = 4;
  while (st >= 2 && fixed + (size_t)st * kS2Rows * kS2Slab > cap) --st;
  if (st < 2) return p;
  p.stages = st;
  p.smem = fixed + (size_t)st * kS2Rows * kS2Slab;
  // One block per SM (the shared memory allows no more): blocks per query
  // chosen so nq * blocks fills whole waves of the SMs (>= 95% of the last
  // wave busy, else the best found); never more blocks than the generic scan
  // would use (its workspace size bounds the candidate lists).
  const int64_t sms = num_sms();
  int64_t blocks_q = 1;
  double best = -1.0;
  const int64_t hi = 4 * ((sms + nq - 1) / nq);
  for (int64_t bq = 1; bq <= hi; ++bq) {
    const int64_t tot = bq * nq;
    const double eff = (double)tot / (double)(((tot + sms - 1) / sms) * sms);
    if (eff > best + 1e-9) {
      best = eff;
      blocks_q = bq;
    }
    if (eff >= 0.95) break;
  }
  int64_t per = ((n + blocks_q - 1) / blocks_q + kS2Rows - 1) / kS2Rows * kS2Rows;
  const int64_t gen = scan_rows_per_block(n, nq);
  if (per < gen) per = gen;
  p.per = per;
  p.nblk = (int)((n + per - 1) / per);
  p.ok = true;
  return p;
}

// Runs the TMA-staged scan when it covers the shape; *used = false otherwise
// (the caller then runs the generic scan).  *nblk receives the number of
// per-query candidate lists written.
static int try_scan2(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                     int bits, int precision, const float* qrot, int nq, const float* cent,
                     int K, float* cand_s, long long* cand_id, cudaStream_t st, int* nblk,
                     bool* used) {
  *used = false;
  const S2Plan p = s2_plan(n, d, bits, precision, nq, K, ldb);
  if (!p.ok) return PQ_OK;
  auto fn = get_encode_fn();
  if (!fn) return PQ_OK;
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)ldb, (cuuint64_t)n};
  cuuint64_t strides[1] = {(cuuint64_t)ldb};
  cuuint32_t box[2] = {(cuuint32_t)kS2Slab, (cuuint32_t)kS2Rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(packed), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PQ_ERR_CUDA, "cuTensorMapEncodeTiled (packed rows) failed (%d)", (int)r);
  dim3 grid(p.nblk, nq);
  int rc = PQ_OK;
#define PQ_S2_CASE(BB, PP)                                                                 \
  case BB * 16 + PP: {                                                                     \
    auto kern = scan2_kernel<BB, PP>;                                                      \
    rc = set_smem(kern, p.smem);                                                           \
    if (rc) return rc;                                                                     \
    kern<<<grid, kS2Threads, p.smem, st>>>(map, norms, n, d, qrot, cent, K, p.per, p.nblk,    \
                                        p.slabs, p.stages, p.lut_bytes, cand_s, cand_id);  \
  } break;
  switch (bits * 16 + precision) {
    PQ_S2_CASE(4, 1) PQ_S2_CASE(4, 2) PQ_S2_CASE(4, 3) PQ_S2_CASE(4, 4)
    PQ_S2_CASE(8, 1) PQ_S2_CASE(8, 2) PQ_S2_CASE(8, 3) PQ_S2_CASE(8, 4)
    PQ_S2_CASE(8, 5) PQ_S2_CASE(8, 6) PQ_S2_CASE(8, 7) PQ_S2_CASE(8, 8)
    default:
      return PQ_OK;
  }
#undef PQ_S2_CASE
  PQ_LAUNCH_CHECK("scan2_kernel");
  *nblk = p.nblk;
  *used = true;
  return PQ_OK;
}
