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
// The tables take 1 KB per byte position (768 KB per query at d=1536 4-bit),
// more than one SM holds, so the rows are cut into C = ceil(row_bytes / 128)
// column slices and the work into groups of C CTAs: CTA r of a group keeps
// the r-th slice's 128 KB of tables in shared memory for the whole launch
// and streams only that 128-byte slice of the group's rows through a TMA
// ring (stages of 128 rows x 128 bytes), writing each row's slice sum to a
// partial-sum buffer P[query][slice][row] in global memory.  Each CTA reads
// exactly one 128-byte line per row, and nothing couples the CTAs while they
// stream.  bt_score_kernel then adds the C slice sums of each row in slice
// order, multiplies by the norm and keeps each block's top-K.  Corpora whose
// partial sums would not fit the buffer are scanned in row chunks.
//
// Lookups: lane 8*rho + g of a consumer warp holds the 16-byte group g of row
// rho (4 rows per warp instruction, two such row groups per warp and stage).
// At step (k, i') it looks up byte i = (i' + rho) mod 4 of word k, byte
// position p = 16g + 4k + i.  Position p has its 256 entries in bank 4g + i,
// so the 32 lanes of every lookup hit 32 banks whatever the codes.  The table
// sits at a 64 KB-aligned shared address with a 256-byte entry stride, so the
// lookup address is the lane's base with byte 1 replaced by the code byte:
// one PRMT per lookup, and one packed f32x2 add per two rows' lookups.
//
// Warp roles (544 threads): warps 0-15 consume stages (8 rows each), warp 16
// issues the TMA loads.  Every wait is bounded; a CTA that gives up records
// the error, stops issuing and waits for its copies in flight.
#include "codes.cuh"
#include "tc.cuh"
#include "topk.cuh"

namespace pqb {

constexpr int kBtConsumerWarps = 16;
constexpr int kBtProducerWarp = 16;
constexpr int kBtThreads = 32 * (kBtConsumerWarps + 1);  // 544
constexpr int kBtSlab = 128;                      // bytes of a row slice (one CTA)
constexpr int kBtRows = 128;                      // rows per stage
constexpr uint32_t kBtStage = kBtRows * kBtSlab;  // 16 KB
constexpr int kBtMaxStages = 6;
constexpr int kBtMinStages = 3;
constexpr int kBtMaxSlices = 8;                   // row_bytes <= 1024
constexpr uint32_t kBtTableBytes = kBtSlab * 256 * 4;  // 128 KB per slice
constexpr int kBtTableCopies = 4;
constexpr uint32_t kBtSmem = 227 * 1024;
constexpr uint32_t kBtSmallBytes = 1024;          // barriers and flags

// Word offset of entry e of byte position p (0..127) inside a slice's table:
// layer k & 1 (64 KB each), entry stride 64 words, column 4g + i + 32 (k >> 1)
// -- bank 4g + i.
__host__ __device__ __forceinline__ uint32_t bt_word(int p, int e) {
  const int g = p >> 4, k = (p >> 2) & 3, i = p & 3;
  return 16384u * (uint32_t)(k & 1) + 64u * (uint32_t)e +
         (uint32_t)(4 * g + i + 32 * (k >> 1));
}

// T[q][slice][word]: the byte tables of every query, in the shared-memory
// layout above.  One thread per output word (coalesced writes).
template <int B>
__global__ void __launch_bounds__(256)
bt_table_kernel(const float* __restrict__ qrot, int nq, int d, int64_t rb, int nslices,
                const float* __restrict__ cent, int shift, float* __restrict__ tables) {
  constexpr int PER = 8 / B;  // codes per byte
  constexpr int W = kBtTableBytes / 4;
  const int64_t total = (int64_t)nq * nslices * W;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t qs = t / W;
    const int w = (int)(t - qs * W);
    const int q = (int)(qs / nslices), s = (int)(qs - (int64_t)q * nslices);
    // Invert bt_word: layer, entry, column -> byte position.
    const int layer = w >> 14, e = (w >> 6) & 255, col = w & 63;
    const int bank = col & 31, h = col >> 5;
    const int g = bank >> 2, i = bank & 3, k = 2 * h + layer;
    const int p = 16 * g + 4 * k + i;
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
    tables[t] = v;
  }
}

__device__ __forceinline__ float bt_lds(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint4 bt_lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// (a0, a1) += (b0, b1) as one packed f32x2 add (round-to-nearest, the same
// results as two scalar adds).
__device__ __forceinline__ void bt_add2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 x, y;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %3};\n\t"
      "add.rn.f32x2 x, x, y;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1));
}

// Bounded mbarrier wait whose polls suspend the thread until the phase
// completes or `kBtHintNs` pass, instead of spinning (a waiting producer
// would otherwise take issue slots from the streaming warps).
constexpr uint32_t kBtHintNs = 20000;

__device__ __forceinline__ bool bt_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kBtHintNs)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool bt_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                                        int err) {
  if (bt_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (bt_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (clock64() - t0 > tc::kWaitCycles) {
      *abort = err;
      device_fail(err);
      return false;
    }
  }
}

// One 1-D bulk copy global -> shared completing on `bar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}

// Shared-memory plan of one CTA, from the address of its dynamic shared
// memory: the table at the first 64 KB boundary, the small region (barriers,
// flags) and the ring stages in the space before and after it.  Same on the
// host (feasibility) and in the kernel.
struct BtLayout {
  uint32_t tab, small, run1, run2;
  int n1, n2, stages;
};

__host__ __device__ inline int bt_fit(uint32_t a, uint32_t b, uint32_t* start) {
  a = (a + 1023u) & ~1023u;
  *start = a;
  return a < b ? (int)((b - a) / kBtStage) : 0;
}

__host__ __device__ inline BtLayout bt_layout(uint32_t raw, uint32_t small_bytes) {
  BtLayout L{};
  const uint32_t end = raw + kBtSmem;
  L.tab = (raw + 0xFFFFu) & ~0xFFFFu;
  L.stages = 0;
  if (L.tab + kBtTableBytes > end) return L;
  const uint32_t g1s = raw, g1e = L.tab, g2s = L.tab + kBtTableBytes, g2e = end;
  // Option A: small region at the start of the space after the table;
  // option B: at the start of the space before it.  The one leaving more
  // ring stages wins.
  uint32_t a1 = 0, a2 = 0, b1 = 0, b2 = 0;
  int na = -1, nb = -1, na1 = 0, nb1 = 0;
  if (g2s + small_bytes <= g2e) {
    na1 = bt_fit(g1s, g1e, &a1);
    na = na1 + bt_fit(g2s + small_bytes, g2e, &a2);
  }
  if (g1s + small_bytes <= g1e) {
    nb1 = bt_fit(g1s + small_bytes, g1e, &b1);
    nb = nb1 + bt_fit(g2s, g2e, &b2);
  }
  if (na < 0 && nb < 0) return L;
  if (na >= nb) {
    L.small = g2s;
    L.run1 = a1;
    L.n1 = na1;
    L.run2 = a2;
    L.n2 = na - na1;
  } else {
    L.small = g1s;
    L.run1 = b1;
    L.n1 = nb1;
    L.run2 = b2;
    L.n2 = nb - nb1;
  }
  L.stages = L.n1 + L.n2 < kBtMaxStages ? L.n1 + L.n2 : kBtMaxStages;
  return L;
}


// Streaming kernel.  Grid (C x groups, nq): CTA x streams slice r = x mod C
// of rows [row0, row1) of group x / C (rows counted from corpus row `base`,
// where the chunk starts) and writes their slice sums to
// P[(q * C + r) * pstride + row].
__global__ void __launch_bounds__(kBtThreads, 1)
scan_bt_kernel(const __grid_constant__ CUtensorMap tmap, const float* __restrict__ tables,
               int C, int64_t base, int64_t rows, int64_t per, float* __restrict__ P,
               int64_t pstride) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t raw = tc::smem_u32(smem_raw);
  const BtLayout lay = bt_layout(raw, kBtSmallBytes);
  const int S = lay.stages;
  // Small region: [full x 6][empty x 6][table] barriers, then flags at 512.
  const uint32_t FULL = lay.small, EMPTY = FULL + 8u * kBtMaxStages;
  const uint32_t TBAR = EMPTY + 8u * kBtMaxStages;
  uint8_t* small = smem_raw + (lay.small - raw);
  int* flags = reinterpret_cast<int*>(small + 512);
  volatile int* abort_flag = flags;
  int* iss = flags + 1;  // copies issued per slot [kBtMaxStages], then the table's

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int q = blockIdx.y;
  const int rank = (int)(blockIdx.x % (unsigned)C);
  const int64_t row0 = (int64_t)(blockIdx.x / (unsigned)C) * per;
  const int64_t row1 = min(rows, row0 + per);
  const int T = row0 < row1 ? (int)((row1 - row0 + kBtRows - 1) / kBtRows) : 0;
  auto slot_addr = [&](int slot) {
    return slot < lay.n1 ? lay.run1 + (uint32_t)slot * kBtStage
                         : lay.run2 + (uint32_t)(slot - lay.n1) * kBtStage;
  };

  if (tid == 0) {
    *abort_flag = 0;
    for (int s = 0; s <= kBtMaxStages; ++s) iss[s] = 0;
    if (S < kBtMinStages) {
      *abort_flag = tc::kErrWaitTmaFull;
      device_fail(tc::kErrWaitTmaFull);
    }
    for (int s = 0; s < kBtMaxStages; ++s) {
      tc::mbar_init(FULL + 8u * s, 1);
      tc::mbar_init(EMPTY + 8u * s, kBtConsumerWarps);
    }
    tc::mbar_init(TBAR, 1);
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmap);
  }
  __syncthreads();

  if (warp == kBtProducerWarp) {
    if (lane == 0 && T > 0 && !*abort_flag) {
      const char* src = reinterpret_cast<const char*>(tables) +
                        ((size_t)q * C + rank) * kBtTableBytes;
      iss[kBtMaxStages] = 1;
      tc::mbar_arrive_expect_tx(TBAR, kBtTableBytes);
#pragma unroll
      for (int u = 0; u < kBtTableCopies; ++u)
        bulk_load(lay.tab + (uint32_t)u * (kBtTableBytes / kBtTableCopies),
                  src + (size_t)u * (kBtTableBytes / kBtTableCopies),
                  kBtTableBytes / kBtTableCopies, TBAR);
      int slot = 0;
      uint32_t eph = 0;  // parity of the slot's previous consumption
      for (int L = 0; L < T; ++L) {
        if (L >= S && !bt_wait(EMPTY + 8u * slot, eph, abort_flag, tc::kErrWaitStageEmpty))
          break;
        if (*abort_flag) break;
        ++iss[slot];
        tc::mbar_arrive_expect_tx(FULL + 8u * slot, kBtStage);
        tc::tma_load_2d(slot_addr(slot), &tmap, rank * kBtSlab,
                        (int)(base + row0 + (int64_t)L * kBtRows), FULL + 8u * slot);
        if (++slot == S) {
          slot = 0;
          if (L >= S) eph ^= 1u;
        }
      }
    }
  } else {
    // Lane 8 rho + g: 16-byte group g of row rho of each 4-row group.
    const int rho = lane >> 3, g = lane & 7;
    uint32_t base_a[4][4], sel[4];
#pragma unroll
    for (int ip = 0; ip < 4; ++ip) {
      const int i = (ip + rho) & 3;
      sel[ip] = 0x7604u | ((uint32_t)i << 4);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        base_a[k][ip] = lay.tab + 65536u * (uint32_t)(k & 1) + 4u * (uint32_t)(4 * g + i) +
                        128u * (uint32_t)(k >> 1);
    }
    // Waits are made warp-uniform (a lane whose wait gave up takes the whole
    // warp out of the loop, so every __syncwarp below has all 32 lanes).
    bool ok = T > 0 && __all_sync(0xffffffffu,
                                  bt_wait(TBAR, 0u, abort_flag, tc::kErrWaitTmaFull));
    int slot = 0;
    uint32_t fph = 0;
    // This lane's 16 bytes of row 8 warp + rho in ring slot 0 (the slot's
    // address advances with the slot); lanes 0 and 4 store rows 8 warp .. +3
    // and 8 warp + 4 .. +7 of each stage.
    const uint32_t lane_off = (uint32_t)(8 * warp + rho) * kBtSlab + 16u * g;
    uint32_t ra = slot_addr(0) + lane_off;
    float* pout = P + ((size_t)q * C + rank) * pstride + row0 + 8 * warp + 4 * (g >> 2);
    for (int L = 0; L < T && ok; ++L) {
      if (!__all_sync(0xffffffffu,
                      bt_wait(FULL + 8u * slot, fph, abort_flag, tc::kErrWaitTmaFull)))
        break;
      // Rows 8 warp + 4 j + rho of the stage, j = 0, 1.
      const uint4 x0 = bt_lds128(ra), x1 = bt_lds128(ra + 4u * kBtSlab);
      const uint32_t w0[4] = {x0.x, x0.y, x0.z, x0.w}, w1[4] = {x1.x, x1.y, x1.z, x1.w};
      float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
#pragma unroll
        for (int ip = 0; ip < 4; ++ip)
          bt_add2(a0[ip], a1[ip], bt_lds(__byte_perm(w0[k], base_a[k][ip], sel[ip])),
                  bt_lds(__byte_perm(w1[k], base_a[k][ip], sel[ip])));
      }
      // The slab is consumed (its words are in registers).
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(EMPTY + 8u * slot);
      bt_add2(a0[0], a1[0], a0[1], a1[1]);
      bt_add2(a0[2], a1[2], a0[3], a1[3]);
      bt_add2(a0[0], a1[0], a0[2], a1[2]);
      const float r0 = a0[0], r1 = a1[0];
      // Transposed reduction over the 8 lanes of each row: lanes g < 4 end
      // with row j = 0's slice sum, g >= 4 with row j = 1's.
      const bool up = (g & 4) != 0;
      float v = (up ? r1 : r0) + __shfl_xor_sync(0xffffffffu, up ? r0 : r1, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      // Rows 8 warp + 4 j .. +3 (rho = 0..3) are in lanes 8 rho + 4 j: lane
      // 4 j gathers them and stores 16 bytes.
      const float v1 = __shfl_down_sync(0xffffffffu, v, 8);
      const float v2 = __shfl_down_sync(0xffffffffu, v, 16);
      const float v3 = __shfl_down_sync(0xffffffffu, v, 24);
      if (lane < 8 && (g & 3) == 0)
        *reinterpret_cast<float4*>(pout + (int64_t)L * kBtRows) = make_float4(v, v1, v2, v3);
      if (++slot == S) {
        slot = 0;
        fph ^= 1u;
        ra = slot_addr(0) + lane_off;
      } else {
        ra = slot == lay.n1 ? lay.run2 + lane_off : ra + kBtStage;
      }
    }
  }

  // After an abort, copies still in flight land before the CTA exits.
  __syncthreads();
  if (tid == 0 && *abort_flag) {
    volatile int never = 0;
    for (int s = 0; s < kBtMaxStages; ++s)
      if (iss[s] > 0)
        tc::mbar_wait(FULL + 8u * s, (uint32_t)(iss[s] - 1) & 1u, &never, tc::kErrWaitTmaFull);
    if (iss[kBtMaxStages] > 0) tc::mbar_wait(TBAR, 0u, &never, tc::kErrWaitTmaFull);
  }
}

// Scoring kernel.  Grid (nb, nq), kBtScoreThreads threads: block b scores
// rows [b * per2, min(rows, (b + 1) * per2)) of the chunk -- the C slice sums
// of each row added in slice order, times the row's norm -- and writes its
// top-K to candidate list list0 + b of query q.
constexpr int kBtScoreThreads = 512;
constexpr int kBtScoreGroup = 4;  // rounds whose loads are in flight together

__global__ void __launch_bounds__(kBtScoreThreads)
bt_score_kernel(const float* __restrict__ P, int64_t pstride, int C,
                const float* __restrict__ norms, int64_t base, int64_t rows, int64_t per2,
                int K, int nlists, int list0, float* __restrict__ cand_s,
                long long* __restrict__ cand_id) {
  extern __shared__ __align__(16) char tk_smem[];
  BlockTopK tk;
  const int cap = BlockTopK::cap_for(K, kBtScoreThreads);
  tk.init(tk_smem, K, cap);
  tk.sel = reinterpret_cast<uint32_t*>(tk_smem + BlockTopK::smem_bytes(cap));
  const int q = blockIdx.y;
  const int64_t r0 = (int64_t)blockIdx.x * per2, r1 = min(rows, r0 + per2);
  const float* pq = P + (size_t)q * C * pstride;
  // Rows go in groups of kBtScoreGroup rounds: the next group's slice sums
  // and norms (up to 9 x kBtScoreGroup loads a thread) are in flight while
  // the current group's scores are offered to the top-K.
  constexpr int G = kBtScoreGroup, T = kBtScoreThreads;
  float xr[G][kBtMaxSlices], nr[G], cur[G];
  auto issue = [&](int64_t g0) {
#pragma unroll
    for (int u = 0; u < G; ++u) {
      const int64_t r = g0 + (int64_t)u * T + threadIdx.x;
      const bool ok = r < r1;
#pragma unroll
      for (int c = 0; c < kBtMaxSlices; ++c)
        xr[u][c] = (ok && c < C) ? __ldg(pq + (size_t)c * pstride + r) : 0.f;
      nr[u] = ok ? __ldg(norms + base + r) : 0.f;
    }
  };
  auto finish = [&]() {
#pragma unroll
    for (int u = 0; u < G; ++u) {
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < kBtMaxSlices; ++c) s += xr[u][c];  // slice order (zeros past C)
      cur[u] = s * nr[u];
    }
  };
  issue(r0);
  finish();
  for (int64_t g0 = r0; g0 < r1; g0 += (int64_t)G * T) {  // the same trip count in every thread
    issue(g0 + (int64_t)G * T);
#pragma unroll
    for (int u = 0; u < G; ++u) {
      const int64_t r = g0 + (int64_t)u * T + threadIdx.x;
      tk.offer(r < r1, cur[u], base + r);
      tk.end_round_select<2>();  // cap = 2 x max(K, 512) = 1024 for K <= 512
    }
    finish();
  }
  const size_t o = ((size_t)q * nlists + list0 + blockIdx.x) * K;
  tk.write(cand_s + o, cand_id + o, 0);
}

}  // namespace pqb

using namespace pqb;

// Queries per call up to which the byte-table scan is used (its tables take
// 1 KB per byte position per query of workspace) and the smallest corpus (the
// tables' build and loads are amortised over many rows).
constexpr int kBtMaxQueries = 64;
constexpr int64_t kBtMinRows = 1 << 18;
constexpr int kBtMaxK = 512;
// Largest partial-sum buffer (slice sums of one row chunk, every query);
// bigger corpora are scanned in chunks of rows.
constexpr size_t kBtPartialCap = (size_t)256 << 20;
// Rows a CTA streams at least when the rows are split into more groups to
// fill the waves (its 128 KB table load stays under ~6 % of its traffic).
constexpr int64_t kBtMinGroupRows = 16384;

static int bt_slices(int d, int bits) {
  return (int)((row_bytes(d, bits) + kBtSlab - 1) / kBtSlab);
}

static int64_t round_rows(int64_t r) { return (r + kBtRows - 1) / kBtRows * kBtRows; }

// Rows per chunk for C slices and nq queries (a multiple of the stage): the
// fewest chunks whose partial sums fit the buffer, of equal size.
static int64_t bt_chunk_rows(int64_t n, int nq, int C) {
  int64_t cap = (int64_t)(kBtPartialCap / ((size_t)nq * C * sizeof(float)));
  cap = cap / kBtRows * kBtRows;
  const int64_t all = round_rows(n);
  if (cap >= all) return all;
  const int64_t chunks = (all + cap - 1) / cap;
  return round_rows((n + chunks - 1) / chunks);
}

// Scoring blocks per query and chunk: one per SM in all (fewer top-K
// compactions), at least 4 x kBtScoreThreads rows each.
static int bt_score_width(int64_t chunk, int nq) {
  int w = (num_sms() + nq - 1) / nq;
  const int64_t minper = 4 * kBtScoreThreads;
  const int64_t cap = (chunk + minper - 1) / minper;
  if (w > cap) w = (int)cap;
  return w < 1 ? 1 : w;
}

// Candidate-list staging of a multi-chunk scan: each chunk's scoring blocks
// write bt_score_width lists per query there, merged into one list per chunk.
static size_t bt_stage_bytes(int64_t n, int nq, int C, int K) {
  const int64_t chunk = bt_chunk_rows(n, nq, C);
  if (chunk >= round_rows(n)) return 0;
  const size_t c = (size_t)nq * bt_score_width(chunk, nq) * K;
  return align_up(c * sizeof(float), 256) + align_up(c * sizeof(long long), 256);
}

// Tables + partial sums (+ list staging) of the scan with C slices.
static size_t bt_ws_for(int64_t n, int nq, int C, int K) {
  return align_up((size_t)nq * C * kBtTableBytes, 256) +
         align_up((size_t)nq * C * bt_chunk_rows(n, nq, C) * sizeof(float), 256) +
         bt_stage_bytes(n, nq, C, K);
}

// Workspace the byte-table scan may need (sized for the widest code width
// whose rows it takes at this d) when it can take the call; else 0.
static size_t bt_tables_bytes(int64_t n, int d, int nq, int k) {
  if (nq < 1 || nq > kBtMaxQueries || n < kBtMinRows || k < 1 || k > kBtMaxK) return 0;
  size_t w = 0;
  for (int b : {1, 2, 4, 8}) {
    const int c = bt_slices(d, b);
    if (c <= kBtMaxSlices) {
      const size_t x = bt_ws_for(n, nq, c, k);
      if (x > w) w = x;
    }
  }
  return w;
}

struct BtPlan {
  bool ok, merge;
  int C, groups, chunks, nb2;
  int64_t rb, chunk, per, per2;
};

static BtPlan bt_plan(int64_t n, int d, int bits, int nq, int K, int64_t ldb, size_t ws_avail) {
  BtPlan p{};
  p.ok = false;
  if (!(bits == 1 || bits == 2 || bits == 4 || bits == 8) || K < 1 || K > kBtMaxK ||
      nq < 1 || nq > kBtMaxQueries || n < kBtMinRows || n >= ((int64_t)1 << 31))
    return p;
  p.rb = row_bytes(d, bits);
  p.C = bt_slices(d, bits);
  if (p.C > kBtMaxSlices || ldb < p.rb || (ldb & 15) != 0) return p;
  if (bt_ws_for(n, nq, p.C, K) > ws_avail) return p;
  // The ring must fit wherever the dynamic shared memory starts (0 or past
  // a reserved first kilobyte).
  for (uint32_t raw : {0u, 1024u})
    if (bt_layout(raw, kBtSmallBytes).stages < kBtMinStages) return p;
  p.chunk = bt_chunk_rows(n, nq, p.C);
  p.chunks = (int)((n + p.chunk - 1) / p.chunk);
  // One CTA per SM (each holds 227 KB of shared memory) in groups of C CTAs
  // per query: a chunk's launch takes ceil(nq x C x groups / sms) waves of
  // CTAs that each stream chunk / groups rows, so the group count is the one
  // (from sms / (nq x C) up) whose CTAs fill their waves best.
  const int sms = num_sms();
  const int64_t unit = (int64_t)p.C * nq;
  int g0 = (int)(sms / unit);
  if (g0 < 1) g0 = 1;
  double best = -1.0;
  for (int g = g0; g <= (4 * g0 > 8 ? 4 * g0 : 8); ++g) {
    const int64_t per = round_rows((p.chunk + g - 1) / g);
    if (g > g0 && per < kBtMinGroupRows) break;
    const int64_t groups = (p.chunk + per - 1) / per;
    const int64_t ctas = unit * groups, waves = (ctas + sms - 1) / sms;
    const double fill = (double)ctas / (double)(waves * sms);
    if (fill > best + 1e-9) {
      best = fill;
      p.per = per;
      p.groups = (int)groups;
    }
    if (fill >= 0.95) break;
  }
  // Candidate lists: the scan workspace holds scan_blocks(n, nq) per query,
  // shared by the chunks.  When a chunk's share would leave the scoring grid
  // under half its width, the chunk's blocks write to the staging area and a
  // merge leaves one list per chunk.
  const int lists = scan_blocks(n, nq) / p.chunks;
  if (lists < 1) return p;
  const int want = bt_score_width(p.chunk, nq);
  p.merge = p.chunks > 1 && 2 * lists < want;
  int nb2 = p.merge || want < lists ? want : lists;
  p.per2 = (p.chunk + nb2 - 1) / nb2;
  p.nb2 = (int)((p.chunk + p.per2 - 1) / p.per2);
  p.ok = true;
  return p;
}

// Runs the byte-table scan when it covers the shape and `ws` (after the
// candidate lists) has room for its tables and partial sums; *used = false
// otherwise.  *nblk receives the per-query candidate lists written.
static int try_scan_bt(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                       int bits, int precision, const float* qrot, int nq, const float* cent,
                       int K, float* cand_s, long long* cand_id, void* ws, size_t ws_bytes,
                       cudaStream_t st, int* nblk, bool* used) {
  *used = false;
  if (!ws) return PQ_OK;
  const BtPlan p = bt_plan(n, d, bits, nq, K, ldb, ws_bytes);
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
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PQ_ERR_CUDA, "cuTensorMapEncodeTiled (byte-table scan rows) failed (%d)", (int)r);
  Carve cv(ws, ws_bytes);
  float* tab = cv.take<float>((size_t)nq * p.C * (kBtTableBytes / 4));
  float* P = cv.take<float>((size_t)nq * p.C * p.chunk);
  float* stage_s = nullptr;
  long long* stage_id = nullptr;
  if (p.merge) {
    stage_s = cv.take<float>((size_t)nq * p.nb2 * K);
    stage_id = cv.take<long long>((size_t)nq * p.nb2 * K);
  }
  if (!cv.ok()) return PQ_OK;
  const int64_t words = (int64_t)nq * p.C * (kBtTableBytes / 4);
  int64_t g = (words + 255) / 256;
  if (g > (int64_t)num_sms() * 32) g = (int64_t)num_sms() * 32;
  const int shift = bits - precision;
  switch (bits) {
#define PQ_BT_CASE(BB)                                                                     \
  case BB:                                                                                 \
    bt_table_kernel<BB><<<(int)g, 256, 0, st>>>(qrot, nq, d, p.rb, p.C, cent, shift, tab); \
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
  int rc = set_smem(scan_bt_kernel, kBtSmem);
  if (rc) return rc;
  const size_t tk_smem = BlockTopK::smem_bytes(BlockTopK::cap_for(K, kBtScoreThreads)) +
                         kTopkSelectWords * sizeof(uint32_t);
  rc = set_smem(bt_score_kernel, tk_smem);
  if (rc) return rc;
  // Candidate lists per query: nb2 per chunk, or one per chunk (merged).
  const int nlists = p.merge ? p.chunks : p.chunks * p.nb2;
  for (int c = 0; c < p.chunks; ++c) {
    const int64_t base = (int64_t)c * p.chunk;
    const int64_t rows = n - base < p.chunk ? n - base : p.chunk;
    const int64_t groups = (rows + p.per - 1) / p.per;
    scan_bt_kernel<<<dim3((unsigned)(p.C * groups), nq), kBtThreads, kBtSmem, st>>>(
        map, tab, p.C, base, rows, p.per, P, p.chunk);
    PQ_LAUNCH_CHECK("scan_bt_kernel");
    // Every chunk launches nb2 scoring blocks: those past a short last
    // chunk's rows write empty lists.
    if (p.merge) {
      bt_score_kernel<<<dim3(p.nb2, nq), kBtScoreThreads, tk_smem, st>>>(
          P, p.chunk, p.C, norms, base, rows, p.per2, K, p.nb2, 0, stage_s, stage_id);
      PQ_LAUNCH_CHECK("bt_score_kernel");
      rc = launch_merge_sorted(stage_s, stage_id, p.nb2, K, (long long)p.nb2 * K, K, nq, K, 0,
                               cand_s + (size_t)c * K, cand_id + (size_t)c * K, st,
                               (long long)nlists * K);
      if (rc) return rc;
    } else {
      bt_score_kernel<<<dim3(p.nb2, nq), kBtScoreThreads, tk_smem, st>>>(
          P, p.chunk, p.C, norms, base, rows, p.per2, K, nlists, c * p.nb2, cand_s, cand_id);
      PQ_LAUNCH_CHECK("bt_score_kernel");
    }
  }
  *nblk = nlists;
  *used = true;
  return PQ_OK;
}

extern "C" int pq_adc_scan_kernel(int64_t n, int d, int bits, int precision, int nq, int k,
                                  int64_t ldb) {
  if (k > PQ_TOPK_MAX) return 3;
  if (precision < 1 || precision > bits) return 1;
  if (bt_plan(n, d, bits, nq, k, ldb, bt_tables_bytes(n, d, nq, k)).ok) return 4;
  const S2Plan p = s2_plan(n, d, bits, precision, nq, k, ldb);
  return p.ok ? 2 : 1;
}
