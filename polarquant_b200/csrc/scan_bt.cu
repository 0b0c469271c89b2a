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
// more than one SM holds, so a thread-block cluster of C CTAs shares the work
// of one row range: CTA r of the cluster owns the r-th 128-byte column slice
// of every row and keeps that slice's 128 KB of tables in its shared memory
// for the whole kernel.  Each CTA streams its slice of the range's rows
// through a TMA ring (stages of 128 rows x 128 bytes) and computes every
// row's slice sum.  The rows of stage L are scored by CTA L mod C (their
// owner): each CTA stores its 128 slice sums of the stage into the owner's
// shared memory with st.async, which completes bytes on the owner's mbarrier
// (no fence on the streaming warps' path); the owner's scorer warps add the
// C sums of each row in slice order, multiply by the norm, keep the CTA's
// top-K and release the slot to the writers.  All slices of a row are read
// by the cluster at about the same time, so DRAM pages and L2 lines are
// fetched once.
//
// Lookups: lane 8*rho + g of a consumer warp holds the 16-byte group g of row
// rho (4 rows per warp instruction).  At step (k, i') it looks up byte
// i = (i' + rho) mod 4 of word k, byte position p = 16g + 4k + i.  Position p
// has its 256 entries in bank 4g + i, so the 32 lanes of every lookup hit 32
// banks whatever the codes.  The table sits at a 64 KB-aligned shared
// address with a 256-byte entry stride, so the lookup address is the lane's
// base with byte 1 replaced by the code byte: one PRMT per lookup.
//
// Warp roles (672 threads): warps 0-15 consume stages (8 rows each), warp 16
// issues the TMA loads, warps 17-20 score the rows of the stages this CTA
// owns.  Every wait is bounded; a CTA that gives up records the error, stops
// issuing, waits for its copies in flight and meets the cluster at the end.
#include "codes.cuh"
#include "tc.cuh"
#include "topk.cuh"

namespace pqb {

constexpr int kBtConsumerWarps = 16;
constexpr int kBtProducerWarp = 16;
constexpr int kBtScorerWarp0 = 17;
constexpr int kBtScorers = 128;
constexpr int kBtThreads = 32 * (kBtConsumerWarps + 1) + kBtScorers;  // 672
constexpr int kBtSlab = 128;                     // bytes of a row slice (one CTA)
constexpr int kBtRows = 128;                     // rows per stage
constexpr uint32_t kBtStage = kBtRows * kBtSlab;  // 16 KB
constexpr int kBtMaxStages = 8;
constexpr int kBtMinStages = 3;
constexpr int kBtMaxCluster = 8;
constexpr int kBtOwnSlots = 3;                   // stage_full slots per owner
constexpr uint32_t kBtTableBytes = kBtSlab * 256 * 4;  // 128 KB per slice
constexpr int kBtTableCopies = 4;
constexpr uint32_t kBtSmem = 227 * 1024;

using BtTopK = TopKT<WarpsGroup<1, kBtScorers>>;

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

__device__ __forceinline__ float bt_ld_cluster(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
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
// completes or `kBtHintNs` pass (instead of spinning: the scorer, producer
// and waiting consumer warps would otherwise take issue slots from the
// streaming warps).  CLUSTER: acquire at cluster scope (the barrier receives
// arrivals or st.async bytes from other CTAs).
constexpr uint32_t kBtHintNs = 20000;

template <bool CLUSTER>
__device__ __forceinline__ bool bt_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  if constexpr (CLUSTER)
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(kBtHintNs)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(kBtHintNs)
        : "memory");
  return ok != 0;
}

template <bool CLUSTER = false>
__device__ __forceinline__ bool bt_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                                        int err) {
  if (bt_try_wait<CLUSTER>(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (bt_try_wait<CLUSTER>(bar, parity)) return true;
    if (*abort) return false;
    if (clock64() - t0 > tc::kWaitCycles) {
      *abort = err;
      device_fail(err);
      return false;
    }
  }
}

// 4-byte store into another CTA's shared memory (addresses from mapa) that
// performs complete_tx of its bytes on that CTA's mbarrier `bar`.
__device__ __forceinline__ void bt_st_async(uint32_t addr, float v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(
                   addr),
               "r"(__float_as_uint(v)), "r"(bar)
               : "memory");
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
// flags, partial sums, top-K) and the ring stages in the space before and
// after it.  Same on the host (feasibility) and in the kernel.
struct BtLayout {
  uint32_t tab, small, run1, run2;
  int n1, n2, stages;
};

__host__ __device__ inline uint32_t bt_small_bytes(int C, int tkbytes) {
  const uint32_t nb = (uint32_t)(C * kBtOwnSlots);
  return (512u + 64u + nb * kBtRows * 4u + (uint32_t)tkbytes + 1023u) & ~1023u;
}

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

__global__ void __launch_bounds__(kBtThreads, 1)
scan_bt_kernel(const __grid_constant__ CUtensorMap tmap, const float* __restrict__ norms,
               int64_t n, const float* __restrict__ tables, int C, int K, int64_t per, int nblk,
               float* __restrict__ cand_s, long long* __restrict__ cand_id) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t raw = tc::smem_u32(smem_raw);
  const int tkcap = BtTopK::cap_for(K, kBtScorers);
  const BtLayout lay = bt_layout(raw, bt_small_bytes(C, (int)BtTopK::smem_bytes(tkcap)));
  const int S = lay.stages;
  // Small region: [barriers 512 B][flags 64 B][slice sums NU x C x 128 f32][top-K]
  const uint32_t FULL = lay.small, EMPTY = FULL + 8u * kBtMaxStages;
  const uint32_t TBAR = EMPTY + 8u * kBtMaxStages;
  const uint32_t OWNF = TBAR + 8u;                 // sums landed [NU]
  const uint32_t FREE = OWNF + 8u * kBtOwnSlots;   // owner o's slot s free [C][NU]
  uint8_t* small = smem_raw + (lay.small - raw);
  int* flags = reinterpret_cast<int*>(small + 512);
  volatile int* abort_flag = flags;
  int* iss = flags + 1;  // copies issued per slot [kBtMaxStages], then the table's
  const uint32_t OPART = lay.small + 576u;
  char* tkmem = reinterpret_cast<char*>(small + 576 + kBtOwnSlots * C * kBtRows * 4);
  const uint32_t SUMS_BYTES = (uint32_t)C * kBtRows * 4u;  // one owned stage's sums

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int q = blockIdx.y;
  const int rank = (int)tc::cluster_ctarank();
  const int64_t cl = blockIdx.x / C;
  const int64_t row0 = cl * per;
  const int64_t row1 = min(n, row0 + per);
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
    // OWNF[s]: one arrival (this CTA's, carrying the expected bytes) plus
    // the C x 128 slice sums of one owned stage stored into it by the
    // cluster's CTAs; the first phase of each is armed here.
    for (int u = 0; u < kBtOwnSlots; ++u) {
      tc::mbar_init(OWNF + 8u * u, 1);
      tc::mbar_arrive_expect_tx(OWNF + 8u * u, SUMS_BYTES);
    }
    for (int b = 0; b < C * kBtOwnSlots; ++b) tc::mbar_init(FREE + 8u * b, 1);
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmap);
  }
  __syncthreads();
  // Every CTA's barriers are initialised before any CTA arrives remotely.
  tc::cluster_sync();

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
                        (int)(row0 + (int64_t)L * kBtRows), FULL + 8u * slot);
        if (++slot == S) {
          slot = 0;
          if (L >= S) eph ^= 1u;
        }
      }
    }
  } else if (warp < kBtConsumerWarps) {
    // Lane 8 rho + g: 16-byte group g of row rho of each 4-row group.
    const int rho = lane >> 3, g = lane & 7;
    uint32_t base[4][4], sel[4];
#pragma unroll
    for (int ip = 0; ip < 4; ++ip) {
      const int i = (ip + rho) & 3;
      sel[ip] = 0x7604u | ((uint32_t)i << 4);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        base[k][ip] = lay.tab + 65536u * (uint32_t)(k & 1) + 4u * (uint32_t)(4 * g + i) +
                      128u * (uint32_t)(k >> 1);
    }
    // Waits are made warp-uniform (a lane whose wait gave up takes the whole
    // warp out of the loop, so every __syncwarp below has all 32 lanes).
    bool ok = T > 0 && __all_sync(0xffffffffu,
                                  bt_wait(TBAR, 0u, abort_flag, tc::kErrWaitTmaFull));
    // Incremental stage state: ring slot and its parity; owner L mod C, the
    // owned-stage index u = L / C as slot u mod NU, its reuse parity and
    // whether the slot was used before.
    int slot = 0, owner = 0, oslot = 0;
    uint32_t fph = 0, rph = 0;
    bool reuse = false;
    const int myrow = 8 * warp + 4 * (g >> 2) + rho;  // row of this lane's sum (g % 4 == 0)
    // This lane's 16 bytes of row 8 warp + rho in ring slot 0 (the slot's
    // address advances with the slot).
    const uint32_t lane_off = (uint32_t)(8 * warp + rho) * kBtSlab + 16u * g;
    uint32_t ra = slot_addr(0) + lane_off;
    const uint32_t dst0 = OPART + 4u * (uint32_t)(rank * kBtRows + myrow);
    const uint32_t oslot_bytes = (uint32_t)C * kBtRows * 4u;
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
          bt_add2(a0[ip], a1[ip], bt_lds(__byte_perm(w0[k], base[k][ip], sel[ip])),
                  bt_lds(__byte_perm(w1[k], base[k][ip], sel[ip])));
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
      // The owner's slot must have been read (its previous use) before this
      // stage's sums are stored into it.
      if (reuse) {
        bool fr = true;
        if (lane == 0)
          fr = bt_wait<true>(FREE + 8u * (uint32_t)(owner * kBtOwnSlots + oslot), rph,
                                     abort_flag, tc::kErrWaitAccEmpty);
        if (!__shfl_sync(0xffffffffu, fr, 0)) break;
      }
      if ((g & 3) == 0)
        bt_st_async(tc::mapa(dst0 + (uint32_t)oslot * oslot_bytes, (uint32_t)owner), v,
                    tc::mapa(OWNF + 8u * (uint32_t)oslot, (uint32_t)owner));
      if (++slot == S) {
        slot = 0;
        fph ^= 1u;
        ra = slot_addr(0) + lane_off;
      } else {
        ra = slot == lay.n1 ? lay.run2 + lane_off : ra + kBtStage;
      }
      if (++owner == C) {
        owner = 0;
        if (++oslot == kBtOwnSlots) {
          oslot = 0;
          if (reuse) rph ^= 1u;
          reuse = true;
        }
      }
    }
  } else {
    // Scorers: thread t <-> row t of each owned stage.
    BtTopK tk;
    tk.g.first = 32 * kBtScorerWarp0;
    tk.init(tkmem, K, tkcap);
    const int t = tid - 32 * kBtScorerWarp0;
    bool ok = true;
    int oslot = 0;
    uint32_t oph = 0;
    for (int L = rank; L < T; L += C) {
      ok = ok && bt_wait<true>(OWNF + 8u * (uint32_t)oslot, oph, abort_flag,
                               tc::kErrWaitAccFull);
      float s = 0.f;
      if (ok) {
        const uint32_t pa = OPART + 4u * (uint32_t)(oslot * C * kBtRows + t);
        for (int c = 0; c < C; ++c) s += bt_lds(pa + 4u * (uint32_t)(c * kBtRows));  // slice order
      }
      // Arm the slot's next phase (its sums are only stored after the
      // releases below, so they cannot reach it earlier).
      if (t == 0 && ok) tc::mbar_arrive_expect_tx(OWNF + 8u * (uint32_t)oslot, SUMS_BYTES);
      tk.g.sync();  // every scorer has read the slot
      if (ok && t < C)
        tc::mbar_arrive_cluster(
            tc::mapa(FREE + 8u * (uint32_t)(rank * kBtOwnSlots + oslot), (uint32_t)t));
      const int64_t row = row0 + (int64_t)L * kBtRows + t;
      const bool valid = ok && row < row1;
      const float sc = valid ? s * __ldg(norms + row) : 0.f;
      tk.offer(valid, sc, row);
      tk.end_round();
      if (++oslot == kBtOwnSlots) {
        oslot = 0;
        oph ^= 1u;
      }
    }
    const size_t o = ((size_t)q * nblk + blockIdx.x) * K;
    tk.write(cand_s + o, cand_id + o, 0);
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
  // After an abort, slice sums already stored towards this CTA may still be
  // in flight (their owner no longer waits for them): give them time to land
  // before the cluster is released.
  if (*abort_flag) {
    const long long t0 = clock64();
    while (clock64() - t0 < 200000) {
    }
  }
  // No CTA leaves while another may still store its slice sums into it or
  // arrive on its barriers.
  __syncthreads();
  tc::cluster_sync();
}

}  // namespace pqb

using namespace pqb;

// Queries per call up to which the byte-table scan is used (its tables take
// 1 KB per byte position per query of workspace) and the smallest corpus (the
// tables' build and loads are amortised over many rows).
constexpr int kBtMaxQueries = 64;
constexpr int64_t kBtMinRows = 1 << 18;
constexpr int kBtMaxK = 512;

static int bt_cluster_size(int d, int bits) {
  return (int)((row_bytes(d, bits) + kBtSlab - 1) / kBtSlab);
}

// Workspace the byte tables of nq queries may need (sized for the widest
// code width whose rows the scan takes at this d) when the byte-table scan
// can take the call; else 0.
static size_t bt_tables_bytes(int64_t n, int d, int nq) {
  if (nq < 1 || nq > kBtMaxQueries || n < kBtMinRows) return 0;
  int c = 0;
  for (int b : {1, 2, 4, 8}) {
    const int cb = bt_cluster_size(d, b);
    if (cb <= kBtMaxCluster && cb > c) c = cb;
  }
  return (size_t)nq * c * kBtTableBytes;
}

static void bt_config(cudaLaunchConfig_t* cfg, cudaLaunchAttribute* at, dim3 grid, int C,
                      cudaStream_t st) {
  *cfg = cudaLaunchConfig_t{};
  cfg->gridDim = grid;
  cfg->blockDim = dim3(kBtThreads);
  cfg->dynamicSmemBytes = kBtSmem;
  cfg->stream = st;
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = C;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg->attrs = at;
  cfg->numAttrs = 1;
}

// Clusters of C byte-table CTAs that fit on the GPU at once (0: unavailable).
static int bt_active_clusters(int C) {
  static int cache[kBtMaxCluster + 1] = {-1, -1, -1, -1, -1, -1, -1, -1, -1};
  if (C < 1 || C > kBtMaxCluster) return 0;
  if (cache[C] < 0) {
    int c = 0;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute at[1];
    bt_config(&cfg, at, dim3(C * (num_sms() / C)), C, 0);
    if (cudaFuncSetAttribute(scan_bt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kBtSmem) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&c, (void*)scan_bt_kernel, &cfg) != cudaSuccess) {
      cudaGetLastError();
      c = 0;
    }
    cache[C] = c;
  }
  return cache[C];
}

struct BtPlan {
  bool ok;
  int C, ncl, nblk;
  int64_t per, rb;
};

static BtPlan bt_plan(int64_t n, int d, int bits, int nq, int K, int64_t ldb, size_t tables_avail) {
  BtPlan p{};
  p.ok = false;
  if (!(bits == 1 || bits == 2 || bits == 4 || bits == 8) || K < 1 || K > kBtMaxK ||
      nq < 1 || nq > kBtMaxQueries || n < kBtMinRows || n >= ((int64_t)1 << 31))
    return p;
  p.rb = row_bytes(d, bits);
  p.C = bt_cluster_size(d, bits);
  if (p.C > kBtMaxCluster || ldb < p.rb || (ldb & 15) != 0) return p;
  if ((size_t)nq * p.C * kBtTableBytes > tables_avail) return p;
  // The shared-memory plan must leave room for the ring wherever the dynamic
  // shared memory starts (0 or past a reserved first kilobyte).
  const uint32_t sb = bt_small_bytes(p.C, (int)BtTopK::smem_bytes(BtTopK::cap_for(K, kBtScorers)));
  for (uint32_t raw : {0u, 1024u})
    if (bt_layout(raw, sb).stages < kBtMinStages) return p;
  const int active = bt_active_clusters(p.C);
  if (active < 1) return p;
  // Clusters per query: enough to fill the GPU's cluster slots once, never
  // more candidate lists than the scan workspace holds (scan_blocks).
  int ncl = active / nq;
  if (ncl < 1) ncl = 1;
  const int maxcl = scan_blocks(n, nq) / p.C;
  if (maxcl < 1) return p;
  if (ncl > maxcl) ncl = maxcl;
  int64_t per = (n + ncl - 1) / ncl;
  per = (per + kBtRows - 1) / kBtRows * kBtRows;
  p.ncl = (int)((n + per - 1) / per);
  p.per = per;
  p.nblk = p.C * p.ncl;
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
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PQ_ERR_CUDA, "cuTensorMapEncodeTiled (byte-table scan rows) failed (%d)", (int)r);
  float* tab = reinterpret_cast<float*>(tables);
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
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute at[1];
  bt_config(&cfg, at, dim3(p.nblk, nq), p.C, st);
  PQ_CUDA_TRY(cudaFuncSetAttribute(scan_bt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)kBtSmem));
  PQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, scan_bt_kernel, map, norms, n, (const float*)tab, p.C, K,
                                 p.per, p.nblk, cand_s, cand_id));
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
