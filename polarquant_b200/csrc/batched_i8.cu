// Batched ADC on CTA pairs with 8-bit integer tensor-core operands
// (tcgen05 .kind::i8, .cta_group::2): candidate lists for
// Quantizer.search_batch (remex/core.py:721-778, S = Q_rot @ X_hat_rot^T *
// norms) at half the tensor-pipe and shared-memory cost per multiply-add of
// the fp16 hi/lo pair kernel.  The epilogue keeps each query's top K + 32 by
// a fixed-point score; rescore_candidates() recomputes those rows with the
// f32 table sums of the streaming scan and cuts them to the exact top K.
//
// Fixed point.  Each rotated query is scaled by sq = max|q| / 32639 and
// rounded to an integer in [-32639, 32639]; the 2^P centroids of the
// Matryoshka level likewise with sx = max|c| / 32639.  An integer v splits
// into two signed 8-bit digits v = 256 * hi + lo (hi in [-127, 127], lo in
// [-128, 127]).  Three int8 MMAs per 32-wide K step accumulate exactly in s32
// TMEM: HH = sum qhi*xhi and X = sum (qhi*xlo + qlo*xhi); the lo*lo term
// (weight 2^-16 of the result) is dropped.  The epilogue forms
// score = float(HH + round(X / 256)) * sq * sx * 65536 * norm.  The dropped
// lo*lo sum dominates the error: ~2e-6 rms, ~1e-5 at most, absolute, on
// unit-norm data -- too coarse to report as a score (1e-4 relative of the
// small top scores of unclustered data), fine for choosing candidates.
//
// Tiles.  One pair MMA computes 256 queries x 256 rows x 32: each CTA holds
// 128 queries and 128 rows per stage as 128-byte K rows (one 128B swizzle
// atom = 128 codes), receives 128 queries x 256 rows of both accumulators in
// its TMEM (HH in columns 0-255, X in 256-511: the whole TMEM, so the
// accumulators are single-buffered and the MMAs of the next tile wait for the
// epilogue to read them).
//
// Decoding.  4-bit codes: the 16-entry digit tables live in 8 registers per
// thread and PRMT looks up four codes at once (no shared-memory table, no
// bank conflicts); the lookup yields each byte's two codes swapped, so the
// query planes are stored with coordinates swapped in pairs to match (the dot
// product is unchanged).  8-bit codes at precision <= 4 use the same register
// tables after gathering four shifted codes into PRMT selector nibbles.  2-bit
// codes and 8-bit codes at precision >= 5: a shared table of the 2^P digit
// pairs indexed by the shifted code.
//
// Roles per CTA (480 threads): warp 0 loads this CTA's query planes by TMA
// (each CTA its own copy); warp 1 issues the pair MMAs (even CTA) or relays "stage
// landed" to the even CTA (odd CTA); warps 2-9 run the top-k epilogue of this
// CTA's 128 queries (two warps per TMEM lane quadrant, one per half of the
// tile's columns); warps 10-13 decode this CTA's 128 rows of each stage;
// warp 14 streams raw code tiles by TMA into a ring.  Every wait is bounded.
#include "tc.cuh"
#include "topk.cuh"

namespace pqb {

constexpr int kQM = 128;        // queries per CTA (256 per pair)
constexpr int kQN = 256;        // rows per pair tile
constexpr int kQNh = 128;       // rows per CTA
constexpr int kQBK = 128;       // K (codes) per stage: one 128-byte swizzle row of int8
constexpr int kQThreads = 15 * 32;
constexpr int kQDigitMax = 32639;  // largest |fixed-point value| (both digits fit int8)

template <int B>
struct I8Geo {
  static constexpr int STAGES = (B == 8) ? 2 : 3;
  static constexpr int RB = kQBK * B / 8;             // raw bytes of one row per K block
  static constexpr int RAWSTAGE = kQNh * RB;          // this CTA's rows of one K block
  static constexpr int RAWBYTES = (B == 8) ? 3 * 16384 : 16384;
  static constexpr int RAW = RAWBYTES / RAWSTAGE;     // ring slots: 4 (2-bit), 2 (4-bit), 3 (8-bit)
  static constexpr int DW = 4;                        // decoder warps
  // Raw segment per decoder task: 8 bytes for 4-bit codes (16 codes -> one
  // 16-byte output chunk, so 8 consecutive lanes write one whole 128-byte row
  // of a plane: conflict-free for any 8-lane phase), else 16 bytes.
  static constexpr int SEGB = (B == 4) ? 8 : 16;
  static constexpr int SPR = RB / SEGB;               // raw segments per row per K block
  static constexpr int UPT = kQNh * SPR / (DW * 32);  // segments per decoder thread per stage
  static constexpr int CPS = SEGB * 8 / B / 16;       // 16-code output chunks per segment
  static_assert(RAW >= 2 && UPT >= 1 && UPT * DW * 32 == kQNh * SPR, "decoder geometry");
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(s));
  return r;
}

// The eight 4-bit codes of word w (MSB-first stream: byte b holds codes 2b
// (high nibble) and 2b+1) looked up in a 16-entry byte table T held as four
// registers (entry c is byte c % 4 of T[c / 4]).  Returns the entries in the
// order of the nibbles, i.e. codes (1,0,3,2) in o0 and (5,4,7,6) in o1.
// PRMT selects bytes 0-7 with the low three bits of each selector nibble; the
// entries 8-15 come from a second PRMT and are chosen byte-wise by a mask
// built with PRMT's sign-replicate mode from each code's top bit.
__device__ __forceinline__ void nib_masks(uint32_t w, uint32_t& s, uint32_t& m0, uint32_t& m1) {
  s = w & 0x77777777u;
  const uint32_t w4 = w << 4;
  m0 = prmt(w, w4, 0x9D8Cu);  // byte i = sign of the top bit of nibble i (i = 0..3)
  m1 = prmt(w, w4, 0xBFAEu);  // nibbles 4..7
}

__device__ __forceinline__ void nib_lookup(const uint32_t (&T)[4], uint32_t s, uint32_t m0,
                                           uint32_t m1, uint32_t& o0, uint32_t& o1) {
  const uint32_t s1 = s >> 16;
  o0 = (prmt(T[0], T[1], s) & ~m0) | (prmt(T[2], T[3], s) & m0);
  o1 = (prmt(T[0], T[1], s1) & ~m1) | (prmt(T[2], T[3], s1) & m1);
}

// Inverse of ordered_key() for keys != 0.
__device__ __forceinline__ float key_to_float(unsigned k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// bar.sync on named barrier `id` for `count` threads (whole warps).
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Four 8-bit codes of word w (one per byte, in K order) shifted down to a
// precision P <= 4 (shift = 8 - P, mask = 2^P - 1 in every byte) and looked
// up in the same register tables: the codes are gathered into the four
// selector nibbles, bytes returned in K order.
__device__ __forceinline__ void byte_lookup(uint32_t w, int shift, uint32_t mask,
                                            const uint32_t (&TH)[4], const uint32_t (&TL)[4],
                                            uint32_t& h, uint32_t& l) {
  const uint32_t t = (w >> shift) & mask;      // code k in the low nibble of byte k
  const uint32_t u = t | (t >> 4);             // byte 0 = c0 | c1 << 4, byte 2 = c2 | c3 << 4
  const uint32_t s = prmt(u, 0u, 0x0020u) & 0x7777u;
  const uint32_t m = prmt(t << 4, 0u, 0xBA98u);  // byte k = sign of code k's top bit
  h = (prmt(TH[0], TH[1], s) & ~m) | (prmt(TH[2], TH[3], s) & m);
  l = (prmt(TL[0], TL[1], s) & ~m) | (prmt(TL[2], TL[3], s) & m);
}

// 16-byte shared-memory load / store at a shared-window address.
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ uint2 ld_shared_v2(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

struct PairWalkI8 {
  int t, tile, kb, tiles;
  int64_t r0, r1;
};

__device__ __forceinline__ void i8_task(PairWalkI8& w, const BatArgs& p) {
  const int rc = w.t / p.qtiles;
  w.r0 = (int64_t)rc * p.rows_per_chunk;
  w.r1 = min(p.n, w.r0 + p.rows_per_chunk);
  w.tiles = (int)((w.r1 - w.r0 + kQN - 1) / kQN);
}

__device__ __forceinline__ void i8_next(PairWalkI8& w, const BatArgs& p, int ntasks, int npairs) {
  if (++w.kb == p.nk) {
    w.kb = 0;
    if (++w.tile == w.tiles) {
      w.tile = 0;
      w.t += npairs;
      if (w.t < ntasks) i8_task(w, p);
    }
  }
}

template <int B>
__global__ void __launch_bounds__(kQThreads, 1)
pair_i8_kernel(const __grid_constant__ CUtensorMap tmQhi, const __grid_constant__ CUtensorMap tmQlo,
               const __grid_constant__ CUtensorMap tmRaw, const BatArgs p) {
  using G = I8Geo<B>;
  constexpr int S = G::STAGES;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t raw = tc::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  constexpr uint32_t QPLANE = kQM * 128;   // 16 KB: 128 queries x 128 int8
  constexpr uint32_t XPLANE = kQNh * 128;  // 16 KB: 128 rows x 128 int8
  constexpr uint32_t STAGE = 2 * QPLANE + 2 * XPLANE;
  const uint32_t meta = base + S * STAGE;
  uint8_t* gmeta = gbase + S * STAGE;
  auto bar = [&](int i) { return meta + 8u * (uint32_t)i; };
  constexpr int FULLA = 0, FULLB = S, PEER = 2 * S, EMPTY = 3 * S, TFULL = 4 * S,
                TEMPTY = 4 * S + 1, DRAIN = 4 * S + 2, RAWFULL = 4 * S + 3,
                RAWEMPTY = RAWFULL + G::RAW, NBAR = RAWEMPTY + G::RAW;
  constexpr int NBAR_MAX = 32;
  static_assert(NBAR <= NBAR_MAX, "barrier area");
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(gmeta + 8 * NBAR_MAX);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gmeta + 8 * NBAR_MAX + 4);
  uint32_t* slut = reinterpret_cast<uint32_t*>(gmeta + 8 * NBAR_MAX + 16);       // 256 entries
  float* scratch_s = reinterpret_cast<float*>(gmeta + 8 * NBAR_MAX + 16 + 1024);  // 4 x 512 (sort)
  int* scratch_i = reinterpret_cast<int*>(gmeta + 8 * NBAR_MAX + 16 + 1024 + 4 * kBatScratch * 4);
  const uint32_t raw_ring =
      (meta + 8 * NBAR_MAX + 16 + 1024 + 4 * kBatScratch * 8 + 127u) & ~127u;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      tc::mbar_init(bar(FULLA + s), 1);
      tc::mbar_init(bar(FULLB + s), G::DW);
      tc::mbar_init(bar(PEER + s), 1);
      tc::mbar_init(bar(EMPTY + s), 1);
    }
    tc::mbar_init(bar(TFULL), 1);
    tc::mbar_init(bar(TEMPTY), 16);  // 8 epilogue warps in each CTA
    tc::mbar_init(bar(DRAIN), 1);
    for (int r = 0; r < G::RAW; ++r) {
      tc::mbar_init(bar(RAWFULL + r), 1);
      tc::mbar_init(bar(RAWEMPTY + r), G::DW);
    }
    *abort_flag = 0;
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmQhi);
    tc::prefetch_tmap(&tmQlo);
    tc::prefetch_tmap(&tmRaw);
  }
  if constexpr (B != 4)
    for (int i = threadIdx.x; i < p.lut_size; i += blockDim.x) slut[i] = p.lut[i];
  if (warp == 1) tc::tmem_alloc_pair(tc::smem_u32(tmem_holder), 512u);
  tc::tc_fence_before();
  tc::cluster_sync();  // barriers of both CTAs initialised, TMEM address published
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint32_t lead_meta = tc::mapa(meta, 0);  // the even CTA's barriers
  auto lead_bar = [&](int i) { return lead_meta + 8u * (uint32_t)i; };

  const int ntasks = p.qtiles * p.rchunks;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: this CTA's 128 queries ----------------
      int it = 0;
      bool ok = true;
      for (int t = pair; t < ntasks && ok; t += npairs) {
        const int rc = t / p.qtiles, qt = t % p.qtiles;
        const int64_t r0 = (int64_t)rc * p.rows_per_chunk;
        const int64_t r1 = min(p.n, r0 + p.rows_per_chunk);
        const int tiles = (int)((r1 - r0 + kQN - 1) / kQN);
        const int qrow = qt * 2 * kQM + (int)rank * kQM;
        for (int tile = 0; tile < tiles && ok; ++tile) {
          for (int kb = 0; kb < p.nk; ++kb, ++it) {
            const int s = it % S;
            const uint32_t ph = (uint32_t)(it / S) & 1u;
            if (!tc::mbar_wait(bar(EMPTY + s), ph ^ 1u, abort_flag, tc::kErrWaitStageEmpty)) {
              ok = false;
              break;
            }
            const uint32_t st = base + (uint32_t)s * STAGE;
            tc::mbar_arrive_expect_tx(bar(FULLA + s), 2 * QPLANE);
            tc::tma_load_2d(st, &tmQhi, kb * kQBK, qrow, bar(FULLA + s));
            tc::tma_load_2d(st + QPLANE, &tmQlo, kb * kQBK, qrow, bar(FULLA + s));
          }
        }
      }
      for (int j = it - S; j < it; ++j) {
        if (j < 0) continue;
        volatile int never = 0;
        tc::mbar_wait(bar(FULLA + j % S), (uint32_t)(j / S) & 1u, &never, tc::kErrWaitTmaFull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && !leader) {
      // ---------------- relay (odd CTA): stage s of this CTA is complete ----------------
      int it = 0;
      bool ok = true;
      for (int t = pair; t < ntasks && ok; t += npairs) {
        const int rc = t / p.qtiles;
        const int64_t r0 = (int64_t)rc * p.rows_per_chunk;
        const int64_t r1 = min(p.n, r0 + p.rows_per_chunk);
        const int tiles = (int)((r1 - r0 + kQN - 1) / kQN);
        for (int tile = 0; tile < tiles && ok; ++tile) {
          for (int kb = 0; kb < p.nk; ++kb, ++it) {
            const int s = it % S;
            const uint32_t ph = (uint32_t)(it / S) & 1u;
            if (!tc::mbar_wait(bar(FULLA + s), ph, abort_flag, tc::kErrWaitTmaFull) ||
                !tc::mbar_wait(bar(FULLB + s), ph, abort_flag, tc::kErrWaitTmaFull)) {
              ok = false;
              break;
            }
            tc::mbar_arrive_cluster(lead_bar(PEER + s));
          }
        }
      }
    } else if (lane == 0) {
      // ---------------- pair MMA issuer (even CTA) ----------------
      const uint32_t idesc = tc::idesc_i8_s32(2 * kQM, kQN);
      const uint32_t d_hh = tmem_base, d_x = tmem_base + (uint32_t)kQN;
      int it = 0, tcount = 0;
      bool ok = true;
      for (int t = pair; t < ntasks && ok; t += npairs) {
        const int rc = t / p.qtiles;
        const int64_t r0 = (int64_t)rc * p.rows_per_chunk;
        const int64_t r1 = min(p.n, r0 + p.rows_per_chunk);
        const int tiles = (int)((r1 - r0 + kQN - 1) / kQN);
        for (int tile = 0; tile < tiles && ok; ++tile, ++tcount) {
          const uint32_t tph = (uint32_t)tcount & 1u;
          if (!tc::mbar_wait_cluster(bar(TEMPTY), tph ^ 1u, abort_flag, tc::kErrWaitAccEmpty)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          for (int kb = 0; kb < p.nk; ++kb, ++it) {
            const int s = it % S;
            const uint32_t ph = (uint32_t)(it / S) & 1u;
            if (!tc::mbar_wait(bar(FULLA + s), ph, abort_flag, tc::kErrWaitTmaFull) ||
                !tc::mbar_wait(bar(FULLB + s), ph, abort_flag, tc::kErrWaitTmaFull) ||
                !tc::mbar_wait_cluster(bar(PEER + s), ph, abort_flag, tc::kErrWaitTmaFull)) {
              ok = false;
              break;
            }
            tc::tc_fence_after();
            const uint32_t st = base + (uint32_t)s * STAGE;
            const uint32_t q_hi = st, q_lo = st + QPLANE;
            const uint32_t x_hi = st + 2 * QPLANE, x_lo = x_hi + XPLANE;
#pragma unroll
            for (int kk = 0; kk < kQBK / 32; ++kk) {
              const uint32_t off = (uint32_t)kk * 32u;
              const uint32_t acc = (kb | kk) != 0;
              tc::mma_i8_pair(d_hh, tc::sw128_desc(q_hi + off), tc::sw128_desc(x_hi + off), idesc,
                              acc);
              tc::mma_i8_pair(d_x, tc::sw128_desc(q_hi + off), tc::sw128_desc(x_lo + off), idesc,
                              acc);
              tc::mma_i8_pair(d_x, tc::sw128_desc(q_lo + off), tc::sw128_desc(x_hi + off), idesc,
                              1);
            }
            tc::mma_commit_pair(bar(EMPTY + s), 3);
          }
          if (ok) tc::mma_commit_pair(bar(TFULL), 3);
        }
      }
      tc::mma_commit_pair(bar(DRAIN), 1);
      volatile int never = 0;
      tc::mbar_wait(bar(DRAIN), 0, &never, tc::kErrWaitAccFull);
    }
  } else if (warp == 14) {
    if (lane == 0) {
      // ---------------- TMA producer: raw code tiles of this CTA's 128 rows ----------------
      const int half = (int)rank * kQNh;
      int it = 0;
      bool ok = true;
      for (int t = pair; t < ntasks && ok; t += npairs) {
        const int rc = t / p.qtiles;
        const int64_t r0 = (int64_t)rc * p.rows_per_chunk;
        const int64_t r1 = min(p.n, r0 + p.rows_per_chunk);
        const int tiles = (int)((r1 - r0 + kQN - 1) / kQN);
        for (int tile = 0; tile < tiles && ok; ++tile) {
          const int y = (int)(r0 + (int64_t)tile * kQN + half);
          for (int kb = 0; kb < p.nk; ++kb, ++it) {
            const int r = it % G::RAW;
            const uint32_t ph = (uint32_t)(it / G::RAW) & 1u;
            if (!tc::mbar_wait(bar(RAWEMPTY + r), ph ^ 1u, abort_flag, tc::kErrWaitStageEmpty)) {
              ok = false;
              break;
            }
            tc::mbar_arrive_expect_tx(bar(RAWFULL + r), (uint32_t)G::RAWSTAGE);
            tc::tma_load_2d(raw_ring + (uint32_t)(r * G::RAWSTAGE), &tmRaw, kb * G::RB, y,
                            bar(RAWFULL + r));
          }
        }
      }
      for (int j = it - G::RAW; j < it; ++j) {
        if (j < 0) continue;
        volatile int never = 0;
        tc::mbar_wait(bar(RAWFULL + j % G::RAW), (uint32_t)(j / G::RAW) & 1u, &never,
                      tc::kErrWaitTmaFull);
      }
    }
  } else if (warp >= 10) {
    // ---------------- decoder: this CTA's 128 rows of each stage ----------------
    // Thread dt owns UPT raw segments u = dt + i * 128 of the stage's raw
    // tile (row u / SPR, segment u % SPR) and writes their digits into the
    // swizzled hi/lo planes.  Rows past the chunk decode to finite digits and
    // are ignored by the epilogue.
    const int dt = threadIdx.x - 10 * 32;
    uint32_t TH[4] = {0u, 0u, 0u, 0u}, TL[4] = {0u, 0u, 0u, 0u};
    const bool regs = (B == 4) || (B == 8 && p.shift >= 4);  // register-table decode
    const uint32_t bmask = ((1u << (8 - p.shift)) - 1u) * 0x01010101u;
    if (regs) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        TH[i] = p.lut[256 + i];
        TL[i] = p.lut[260 + i];
      }
    }
    PairWalkI8 w;
    w.t = pair;
    w.tile = 0;
    w.kb = 0;
    if (w.t < ntasks) i8_task(w, p);
    for (int it = 0; w.t < ntasks; ++it) {
      const int rr = it % G::RAW;
      const uint32_t rph = (uint32_t)(it / G::RAW) & 1u;
      i8_next(w, p, ntasks, npairs);
      const int s = it % S;
      const uint32_t ph = (uint32_t)(it / S) & 1u;
      if (!tc::mbar_wait(bar(RAWFULL + rr), rph, abort_flag, tc::kErrWaitTmaFull)) break;
      uint32_t cur[G::UPT][4];
      const uint32_t rawa = raw_ring + (uint32_t)(rr * G::RAWSTAGE);
#pragma unroll
      for (int i = 0; i < G::UPT; ++i) {
        const uint32_t a = rawa + (uint32_t)(dt + i * G::DW * 32) * (uint32_t)G::SEGB;
        if constexpr (G::SEGB == 8) {
          const uint2 v = ld_shared_v2(a);
          cur[i][0] = v.x; cur[i][1] = v.y; cur[i][2] = 0u; cur[i][3] = 0u;
        } else {
          const uint4 v = ld_shared_v4(a);
          cur[i][0] = v.x; cur[i][1] = v.y; cur[i][2] = v.z; cur[i][3] = v.w;
        }
      }
      if (!tc::mbar_wait(bar(EMPTY + s), ph ^ 1u, abort_flag, tc::kErrWaitStageEmpty)) break;
      const uint32_t xh = base + (uint32_t)s * STAGE + 2 * QPLANE;
      const uint32_t xl = xh + XPLANE;
#pragma unroll
      for (int i = 0; i < G::UPT; ++i) {
        const int u = dt + i * G::DW * 32;
        const int r = u / G::SPR, sg = u % G::SPR;
#pragma unroll
        for (int ch = 0; ch < G::CPS; ++ch) {
          uint32_t hw[4], lw[4];
          if constexpr (B == 4) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              uint32_t sel, m0, m1;
              nib_masks(cur[i][2 * ch + j], sel, m0, m1);
              nib_lookup(TH, sel, m0, m1, hw[2 * j], hw[2 * j + 1]);
              nib_lookup(TL, sel, m0, m1, lw[2 * j], lw[2 * j + 1]);
            }
          } else if (B == 8 && regs) {
#pragma unroll
            for (int g = 0; g < 4; ++g)
              byte_lookup(cur[i][g], p.shift, bmask, TH, TL, hw[g], lw[g]);
          } else {
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint32_t e[4];
#pragma unroll
              for (int k = 0; k < 4; ++k)
                e[k] = slut[seg_code<B>(cur[i], ch * 16 + 4 * g + k) >> p.shift];
              const uint32_t x01 = prmt(e[0], e[1], 0x5140u), x23 = prmt(e[2], e[3], 0x5140u);
              hw[g] = prmt(x01, x23, 0x5410u);
              lw[g] = prmt(x01, x23, 0x7632u);
            }
          }
          const int c = sg * G::CPS + ch;
          const uint32_t off = (uint32_t)r * 128u + ((uint32_t)(c ^ (r & 7)) << 4);
          st_shared_v4(xh + off, hw[0], hw[1], hw[2], hw[3]);
          st_shared_v4(xl + off, lw[0], lw[1], lw[2], lw[3]);
        }
      }
      // Generic-proxy stores become visible to the tensor core (async proxy);
      // the odd CTA's relay forwards completion to the even CTA.  The raw
      // slot is released only now, after the stores that consume its bytes:
      // released right after the shared-memory loads (before their values
      // were used), the next TMA write into the slot -- an async-proxy write,
      // which the mbarrier's release does not order after generic-proxy
      // loads -- overwrote codes still being read (measured: 30-130 of 520
      // queries lost rows at d=256).
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(bar(FULLB + s));
        tc::mbar_arrive(bar(RAWEMPTY + rr));
      }
    }
  } else {
    // ---------------- epilogue: warps 2..9, thread = query ----------------
    // Warps w and w + 4 read the same TMEM lanes (queries), w the tile's
    // columns 0-127 and w + 4 columns 128-255, and keep separate candidate
    // buffers and output lists (list 2 * chunk + half).  Per 16 rows a bound
    // float(max v) * qs * (max or min norm) -- an upper bound of every score of
    // the group, since IEEE rounding is monotonic -- skips groups that cannot
    // beat the query's threshold; only the others are scored row by row.
    const int ew = warp - 2;
    const int quad = warp & 3, half = ew >> 2;
    const int q_lane = 32 * quad + lane;
    float* ss = scratch_s + quad * kBatScratch;  // shared by the two halves, used in turn
    int* si = scratch_i + quad * kBatScratch;
    const float csc = p.cscale[0];
    const int mch = (int)p.cscale[1], mcl = (int)p.cscale[2];
    auto buf_of = [&](int ql) { return (((size_t)blockIdx.x * kQM + ql) * 2 + half) * p.cap; };
    int tcount = 0;
    bool ok = true;
    for (int t = pair; t < ntasks; t += npairs) {
      const int rc = t / p.qtiles, qt = t % p.qtiles;
      const int64_t r0 = (int64_t)rc * p.rows_per_chunk;
      const int64_t r1 = min(p.n, r0 + p.rows_per_chunk);
      const int tiles = (int)((r1 - r0 + kQN - 1) / kQN);
      const int qbase = qt * 2 * kQM + (int)rank * kQM;
      const int qg = qbase + q_lane;
      const bool qv = qg < p.nq;
      const float qs = qv ? p.qinv[qg] * csc : 0.f;
      // v = HH + round(X / 256) <= HH + xb: |X| <= sum|q_hi| max|c_lo| +
      // sum|q_lo| max|c_hi|, so a group is bounded by its HH values alone.
      const int xb = qv ? (p.qdig[2 * qg] * mcl + p.qdig[2 * qg + 1] * mch + 128) >> 8 : 0;
      float* bs = p.buf_s + buf_of(q_lane);
      int* bi = p.buf_i + buf_of(q_lane);
      int cnt = 0;
      float thr = -INFINITY;
      // After an abort the warps keep walking the remaining tasks (every wait
      // then fails at once) so that both halves still meet at each named
      // barrier below.
      for (int tile = 0; tile < tiles; ++tile, ++tcount) {
        const int64_t hr0 = r0 + (int64_t)tile * kQN + half * (kQN / 2);  // this half's rows
        // The half's 128 norms, loaded before the accumulator wait (which
        // hides their latency): register c holds row hr0 + 32 c + lane.
        float nrm[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int64_t row = hr0 + 32 * c + lane;
          nrm[c] = (ok && row < r1) ? __ldg(p.norms + row) : 0.f;
        }
        const unsigned gkey = (ok && qv) ? __ldcg(p.gthr + qg) : 0u;
        // Norm range of each 8-row group, also before the wait: after the
        // reduction lanes 8j..8j+7 of register c hold group 4c+j's.
        float nmx[4], nmn[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          nmx[c] = nrm[c];
          nmn[c] = nrm[c];
#pragma unroll
          for (int o = 4; o > 0; o >>= 1) {
            nmx[c] = fmaxf(nmx[c], __shfl_xor_sync(0xffffffffu, nmx[c], o));
            nmn[c] = fminf(nmn[c], __shfl_xor_sync(0xffffffffu, nmn[c], o));
          }
        }
        if (ok && !tc::mbar_wait(bar(TFULL), (uint32_t)tcount & 1u, abort_flag,
                                 tc::kErrWaitAccFull))
          ok = false;
        ok = __all_sync(0xffffffffu, ok);  // the TMEM loads below are warp-collective
        if (!ok) continue;
        tc::tc_fence_after();
        // The best threshold any task of this query has published: at least
        // K approximate scores (in some row chunk) reach it, so rows below it
        // cannot enter the query's overall top K.
        if (gkey != 0u) thr = fmaxf(thr, key_to_float(gkey));
        const uint32_t taddr =
            tmem_base + ((uint32_t)(32 * quad) << 16) + (uint32_t)(half * (kQN / 2));
        // The half's 128 columns in four 32-column chunks, 8-row groups of a
        // chunk: one TMEM load of the chunk's HH values (load latency, not
        // arithmetic, bounds this loop), then per group two bounds of its
        // scores -- HH + xb (loose by the worst case of the cross terms) and,
        // for groups that pass it, the group's largest v after loading its
        // cross terms -- and only the rows of groups that pass both are
        // scored.  float(v) * qs * norm is monotonic in v and in the norm
        // (IEEE rounding is), so both are upper bounds of every score of the
        // group.
        auto room = [&]() {
          // Room for 32 more candidates in every buffer of the warp.
          uint32_t need = __ballot_sync(0xffffffffu, qv && cnt + 32 > p.cap);
          while (need) {
            const int src = __ffs(need) - 1;
            need &= need - 1;
            const float before = thr;
            warp_select(src, lane, cnt, p.buf_s + buf_of(32 * quad + src),
                        p.buf_i + buf_of(32 * quad + src), p.K, cnt, thr);
            if (lane == src) {
              thr = fmaxf(thr, before);  // never below a threshold already adopted
              atomicMax(p.gthr + qg, ordered_key(thr));  // publish
            }
          }
        };
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          room();
          uint32_t h[32];
          __syncwarp();
          tc::tmem_ld32(taddr + (uint32_t)(32 * c), h);
          tc::tmem_ld_wait(h);
          const float nr_all = c == 0 ? nrm[0] : c == 1 ? nrm[1] : c == 2 ? nrm[2] : nrm[3];
          const float nmx_c = c == 0 ? nmx[0] : c == 1 ? nmx[1] : c == 2 ? nmx[2] : nmx[3];
          const float nmn_c = c == 0 ? nmn[0] : c == 1 ? nmn[1] : c == 2 ? nmn[2] : nmn[3];
          // The four groups' first bounds side by side (independent chains),
          // then one warp-wide OR of the per-thread group masks.
          float gmx[4], gmn[4];
          unsigned wbits = 0u;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            gmx[j] = __shfl_sync(0xffffffffu, nmx_c, 8 * j);
            gmn[j] = __shfl_sync(0xffffffffu, nmn_c, 8 * j);
            int t4[4];                                 // tree max of the group's 8 HH values
#pragma unroll
            for (int i = 0; i < 4; ++i) t4[i] = max((int)h[8 * j + i], (int)h[8 * j + i + 4]);
            const int hmax = max(max(t4[0], t4[2]), max(t4[1], t4[3])) + xb;
            if (qv && (__int2float_rn(hmax) * qs) * (hmax >= 0 ? gmx[j] : gmn[j]) > thr)
              wbits |= 1u << j;
          }
          const unsigned groups = __reduce_or_sync(0xffffffffu, wbits);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (!((groups >> j) & 1u)) continue;
            const float gmax = gmx[j], gmin = gmn[j];
            bool want = (wbits >> j) & 1u;
            uint32_t x[8];
            __syncwarp();
            tc::tmem_ld8(taddr + (uint32_t)(kQN + 32 * c + 8 * j), x);
            tc::tmem_ld_wait(x);
            int vmax = (int)h[8 * j] + (((int)x[0] + 128) >> 8);
#pragma unroll
            for (int i = 1; i < 8; ++i)
              vmax = max(vmax, (int)h[8 * j + i] + (((int)x[i] + 128) >> 8));
            want = want && (__int2float_rn(vmax) * qs) * (vmax >= 0 ? gmax : gmin) > thr;
            if (!__any_sync(0xffffffffu, want)) continue;
            // Every row of the group scored exactly; passing rows appended
            // with predicated stores (no per-row branch).
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float nr = __shfl_sync(0xffffffffu, nr_all, 8 * j + i);
              const int64_t row = hr0 + 32 * c + 8 * j + i;
              const int v = (int)h[8 * j + i] + (((int)x[i] + 128) >> 8);
              const float sc = (__int2float_rn(v) * qs) * nr;
              const bool pass = want && row < r1 && sc > thr;
              if (pass) {
                bs[cnt] = sc;
                bi[cnt] = (int)row;
              }
              cnt += pass ? 1 : 0;
            }
          }
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader) tc::mbar_arrive(bar(TEMPTY));
          else tc::mbar_arrive_cluster(lead_bar(TEMPTY));
        }
      }
      // Task end: each half writes the best K of its buffer per query.  The
      // two halves of a quadrant share one sort scratch and take turns, half
      // 0 then half 1, and neither goes on before both are done: half 0 could
      // otherwise finish a following one-tile task and sort into the scratch
      // while half 1 is still sorting this task's lists.
      for (int turn = 0; turn < 2; ++turn) {
        if (turn == half && ok) {
          __syncwarp();
          uint32_t pend = __ballot_sync(0xffffffffu, qv);
          while (pend) {
            const int src = __ffs(pend) - 1;
            pend &= pend - 1;
            const int sq = qbase + 32 * quad + src;
            const size_t o = ((size_t)sq * p.out_parts + p.part_base + 2 * rc + half) * p.K;
            warp_compact(src, lane, cnt, p.buf_s + buf_of(32 * quad + src),
                         p.buf_i + buf_of(32 * quad + src), p.K, ss, si, cnt, thr,
                         p.out_s + o, p.out_id + o, p.row_offset);
          }
        }
        named_sync(1, 256);
      }
    }
  }
  tc::tc_fence_before();
  tc::cluster_sync();  // both CTAs done with each other's shared memory and the TMEM
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc_pair(tmem_base, 512u);
  }
}

// Rotated queries -> 16-bit fixed point split into two int8 planes (rows of
// ldk bytes, zero past d), one warp per query; qscale[q] = max|q| / 32639 and
// qdig[2q], qdig[2q+1] = the sums of |hi| and |lo| digits (for the epilogue's
// bound on the cross-term accumulator).  swap != 0 stores coordinate j at
// position j ^ 1 (the 4-bit decoder's order).
__global__ void __launch_bounds__(256)
qsplit_i8_kernel(const float* __restrict__ qrot, int nq, int d, int ldk, int swap,
                 int8_t* __restrict__ qhi, int8_t* __restrict__ qlo, float* __restrict__ qscale,
                 int* __restrict__ qdig) {
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int q = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); q < nq; q += warps) {
    const float* v = qrot + (size_t)q * d;
    float mx = 0.f;
    for (int j = lane; j < d; j += 32) mx = fmaxf(mx, fabsf(__ldg(v + j)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float inv = mx > 0.f ? (float)kQDigitMax / mx : 0.f;
    uint32_t* hp = reinterpret_cast<uint32_t*>(qhi + (size_t)q * ldk);
    uint32_t* lp = reinterpret_cast<uint32_t*>(qlo + (size_t)q * ldk);
    int shi = 0, slo = 0;
    for (int p0 = 4 * lane; p0 < ldk; p0 += 128) {
      uint32_t hw = 0, lw = 0;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int j = (p0 + t) ^ swap;
        const float f = j < d ? __ldg(v + j) : 0.f;
        int qi = __float2int_rn(f * inv);
        qi = max(-kQDigitMax, min(kQDigitMax, qi));
        const int hi = (qi + 128) >> 8;
        const int lo = qi - (hi << 8);
        shi += abs(hi);
        slo += abs(lo);
        hw |= (uint32_t)(hi & 255) << (8 * t);
        lw |= (uint32_t)(lo & 255) << (8 * t);
      }
      hp[p0 >> 2] = hw;
      lp[p0 >> 2] = lw;
    }
    shi = (int)__reduce_add_sync(0xffffffffu, (unsigned)shi);
    slo = (int)__reduce_add_sync(0xffffffffu, (unsigned)slo);
    if (lane == 0) {
      qscale[q] = mx > 0.f ? mx / (float)kQDigitMax : 0.f;
      qdig[2 * q] = shi;
      qdig[2 * q + 1] = slo;
    }
  }
}

// Digit tables of the 2^P centroids: lut[c] = hi | lo << 8 (bytes) of
// round(cent[c] * 32639 / max|cent|); lut[256..263] = the register tables
// (hi bytes, then lo bytes) of 16 entries c -> cent[c >> reg_shift] (0 past
// the table): reg_shift = bits - P for 4-bit codes (indexed by the stored
// code), 0 for 8-bit codes (indexed by the shifted code);
// cscale[0] = max|cent| / 32639 * 65536, cscale[1] / [2] = the largest |hi| /
// |lo| digit.
__global__ void lut_i8_kernel(const float* __restrict__ cent, int size, int reg_shift,
                              uint32_t* __restrict__ lut, float* __restrict__ cscale) {
  __shared__ float mx;
  __shared__ uint32_t ent[256];
  if (threadIdx.x == 0) {
    float m = 0.f;
    for (int i = 0; i < size; ++i) m = fmaxf(m, fabsf(cent[i]));
    mx = m;
  }
  __syncthreads();
  const float inv = mx > 0.f ? (float)kQDigitMax / mx : 0.f;
  for (int i = threadIdx.x; i < size; i += blockDim.x) {
    int ci = __float2int_rn(cent[i] * inv);
    ci = max(-kQDigitMax, min(kQDigitMax, ci));
    const int hi = (ci + 128) >> 8;
    const int lo = ci - (hi << 8);
    ent[i] = (uint32_t)(hi & 255) | ((uint32_t)(lo & 255) << 8);
    lut[i] = ent[i];
  }
  __syncthreads();
  if (threadIdx.x < 8) {
    const int plane = threadIdx.x >> 2, wd = threadIdx.x & 3;
    uint32_t v = 0;
    for (int b = 0; b < 4; ++b) {
      const int e = (4 * wd + b) >> reg_shift;
      if (e < size) v |= ((ent[e] >> (8 * plane)) & 255u) << (8 * b);
    }
    lut[256 + threadIdx.x] = v;
  }
  if (threadIdx.x == 0) {
    cscale[0] = mx / (float)kQDigitMax * 65536.f;
    int mh = 0, ml = 0;  // largest |hi| and |lo| digit of the table
    for (int i = 0; i < size; ++i) {
      mh = max(mh, abs((int)(int8_t)(ent[i] & 255u)));
      ml = max(ml, abs((int)(int8_t)((ent[i] >> 8) & 255u)));
    }
    cscale[1] = (float)mh;
    cscale[2] = (float)ml;
  }
}

struct I8Plan {
  int ldk, nk, nq_pad, qtiles, rchunks, grid, cap;
  int64_t rpc;
  size_t smem;
};

template <int B>
static constexpr size_t i8_smem() {
  return 1024 + (size_t)I8Geo<B>::STAGES * (2 * kQM * 128 + 2 * kQNh * 128) + 8 * 32 + 16 + 1024 +
         (size_t)4 * kBatScratch * 8 + 128 + I8Geo<B>::RAWBYTES;
}

static size_t i8_smem_for(int bits) {
  return bits == 8 ? i8_smem<8>() : bits == 2 ? i8_smem<2>() : i8_smem<4>();
}

static void i8_config(cudaLaunchConfig_t* cfg, cudaLaunchAttribute* at, int grid, size_t smem,
                      cudaStream_t st) {
  *cfg = cudaLaunchConfig_t{};
  cfg->gridDim = dim3(grid);
  cfg->blockDim = dim3(kQThreads);
  cfg->dynamicSmemBytes = smem;
  cfg->stream = st;
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg->attrs = at;
  cfg->numAttrs = 1;
}

// CTA pairs of the int8 kernel that fit on the GPU at once; 0 when pair
// launches are unavailable.  (The 4-bit kernel has the largest footprint.)
static int i8_slots() {
  static int slots = -1;
  if (slots < 0) {
    int c = 0;
    auto kern = pair_i8_kernel<4>;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute at[1];
    i8_config(&cfg, at, 2 * (num_sms() / 2), i8_smem<4>(), 0);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)i8_smem<4>()) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&c, (void*)kern, &cfg) != cudaSuccess) {
      cudaGetLastError();
      c = 0;
    }
    slots = c < num_sms() / 2 ? c : num_sms() / 2;
  }
  return slots;
}

// Extra candidates the int8 kernel keeps per list beyond the K asked for.
// Its scores are within ~1e-5 (absolute, unit-norm data) of the exact f32
// sums; the lists are rescored exactly and cut to K, so a row of the exact
// top-K can only be lost if more than kI8Margin other rows score within
// twice that error of it, i.e. inside the score-tie band.
constexpr int kI8Margin = 32;

// Smallest dimension for which the int8 kernel is used.  Its two
// accumulators fill the TMEM, so a tile's epilogue (~7.5 k cycles with the
// hand-offs) does not overlap the next tile's MMAs (~1.6 k cycles per 128 of
// d); the fp16 pair kernel double-buffers its accumulator but needs twice the
// MMA time.  Measured on the B200: int8 1.45x faster at d=1536 (4-bit), fp16
// 1.2x faster at d=768 (8-bit codes at precision 4).
constexpr int kI8MinDim = 1024;

// Shapes the int8 kernel takes: 2-, 4- and 8-bit codes, d >= kI8MinDim, at
// least one pair tile of rows, a row stride of at least one raw K block (the
// TMA box), and K + margin within the epilogue's selection limit.
static bool i8_eligible(int64_t n, int d, int64_t ldb, int bits, int K) {
  return (bits == 2 || bits == 4 || bits == 8) && d >= kI8MinDim && n >= kQN &&
         ldb >= kQBK * bits / 8 && K + kI8Margin <= kBatMaxK;
}

static I8Plan i8_plan(int64_t n, int d, int nq, int k, int slots, int bits) {
  I8Plan b;
  b.ldk = (d + kQBK - 1) / kQBK * kQBK;
  b.nk = b.ldk / kQBK;
  b.qtiles = (nq + 2 * kQM - 1) / (2 * kQM);
  b.nq_pad = b.qtiles * 2 * kQM;
  // Row chunks per query tile: the smallest count whose task total fills the
  // pair slots in whole waves (>= 97% of the last wave busy); tasks stay >= 4
  // row tiles long.
  const int64_t min_rows = 4 * kQN;
  const int64_t max_rc = (n + min_rows - 1) / min_rows < 1 ? 1 : (n + min_rows - 1) / min_rows;
  int rc = 1;
  double best = -1.0;
  const int lo = (slots + b.qtiles - 1) / b.qtiles;
  for (int c = lo < 1 ? 1 : lo; c <= 16 * lo + 16 && c <= max_rc; ++c) {
    const int64_t tasks = (int64_t)c * b.qtiles;
    const double eff = (double)tasks / (double)(((tasks + slots - 1) / slots) * slots);
    if (eff > best + 1e-9) {
      best = eff;
      rc = c;
    }
    if (eff >= 0.97) break;
  }
  if (best < 0) rc = (int)(max_rc < lo ? max_rc : lo);
  b.rpc = ((n + rc - 1) / rc + kQN - 1) / kQN * kQN;
  if (b.rpc < kQN) b.rpc = kQN;
  b.rchunks = (int)((n + b.rpc - 1) / b.rpc);
  if (b.rchunks < 1) b.rchunks = 1;
  const int tasks = b.qtiles * b.rchunks;
  b.grid = 2 * (tasks < slots ? tasks : slots);
  b.cap = 2 * k;
  if (b.cap < 64) b.cap = 64;
  b.smem = i8_smem_for(bits);
  return b;
}

struct I8Ws {
  int8_t *qhi, *qlo;
  float *qscale, *cscale, *buf_s, *out_s, *seed_s;
  uint32_t* lut;
  unsigned int* gthr;
  int* qdig;
  int* buf_i;
  long long *out_id, *seed_id;
};

// Rows of a first pass whose merged lists seed every query's threshold before
// the rest of the corpus is scanned (0 = a single pass).  Without it each
// task's threshold starts at -inf and rises only as the task's own rows (or
// other tasks' of the same query) fill its list, so on shards of a few
// million rows -- where a row chunk holds few rows close to a clustered
// query -- most of the scan runs with a loose threshold and the epilogue
// scores many groups row by row.  The K'-th best approximate score over the
// first pass's rows is a lower bound of the K'-th best over all rows, so it
// is a valid starting threshold.
static int64_t i8_pilot_rows(int64_t n) {
  if (n < ((int64_t)4 << 20)) return 0;
  int64_t s = n / 8;
  if (s < ((int64_t)1 << 20)) s = (int64_t)1 << 20;
  if (s > ((int64_t)4 << 20)) s = (int64_t)4 << 20;
  return s / kQN * kQN;
}

struct I8Run {
  int npass, parts, grid_max;
  int64_t first[2], rows[2];
  I8Plan p[2];
};

static I8Run i8_run_plan(int64_t n, int d, int nq, int K, int slots, int bits) {
  I8Run r;
  const int64_t S = i8_pilot_rows(n);
  r.npass = S > 0 ? 2 : 1;
  r.first[0] = 0;
  r.rows[0] = S > 0 ? S : n;
  r.first[1] = S;
  r.rows[1] = n - S;
  r.parts = 0;
  r.grid_max = 0;
  for (int i = 0; i < r.npass; ++i) {
    r.p[i] = i8_plan(r.rows[i], d, nq, K, slots, bits);
    r.parts += 2 * r.p[i].rchunks;
    if (r.p[i].grid > r.grid_max) r.grid_max = r.p[i].grid;
  }
  return r;
}

static size_t i8_ws_carve(const I8Run& r, int nq, int K, void* ws, size_t ws_bytes, I8Ws* w) {
  const I8Plan& b = r.p[0];  // nq_pad, ldk and cap are the same for both passes
  Carve cv(ws, ws_bytes);
  w->qhi = cv.take<int8_t>((size_t)b.nq_pad * b.ldk);
  w->qlo = cv.take<int8_t>((size_t)b.nq_pad * b.ldk);
  w->qscale = cv.take<float>((size_t)b.nq_pad);
  w->cscale = cv.take<float>(4);
  w->lut = cv.take<uint32_t>(256 + 8);
  w->gthr = cv.take<unsigned int>((size_t)b.nq_pad);
  w->qdig = cv.take<int>((size_t)2 * b.nq_pad);
  w->buf_s = cv.take<float>((size_t)r.grid_max * kQM * 2 * b.cap);
  w->buf_i = cv.take<int>((size_t)r.grid_max * kQM * 2 * b.cap);
  w->out_s = cv.take<float>((size_t)nq * r.parts * K);
  w->out_id = cv.take<long long>((size_t)nq * r.parts * K);
  w->seed_s = r.npass > 1 ? cv.take<float>((size_t)nq * K) : nullptr;
  w->seed_id = r.npass > 1 ? cv.take<long long>((size_t)nq * K) : nullptr;
  return cv.off + 256;
}

// gthr[q] = the K-th best of query q's merged first-pass lists (when it has K).
__global__ void i8_seed_kernel(const float* __restrict__ s, const long long* __restrict__ id,
                               int nq, int K, unsigned int* __restrict__ gthr) {
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  const size_t o = (size_t)q * K + K - 1;
  if (id[o] >= 0) gthr[q] = ordered_key(s[o]);
}

// 2-D uint8 tensor map (rows x width bytes, row stride `stride`), box
// {box_x bytes, box_rows}, optional 128-byte swizzle.
static int make_map_u8(CUtensorMap* map, const void* ptr, int64_t rows, int64_t width,
                       int64_t stride, int box_x, int box_rows, bool swizzle) {
  auto fn = get_encode_fn();
  if (!fn) return fail(PQ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  PQ_CHECK_ARG(((uintptr_t)ptr & 15) == 0, "TMA base must be 16-byte aligned");
  cuuint64_t dims[2] = {(cuuint64_t)width, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)stride};
  cuuint32_t box[2] = {(cuuint32_t)box_x, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PQ_ERR_CUDA, "cuTensorMapEncodeTiled (uint8) failed (%d)", (int)r);
  return PQ_OK;
}

}  // namespace pqb

using namespace pqb;

// Runs the int8 pair kernel (a threshold-seeding first pass and the main
// pass on corpora of 4M+ rows, see i8_pilot_rows); leaves per-(query, row
// chunk) top-K lists in ws (layout [nq][parts][K], ids local + row_offset) and
// returns their location.
static int run_batched_i8(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                          int bits, int precision, const float* qrot, int nq, const float* cent,
                          int K, int64_t row_offset, void* ws, size_t ws_bytes, cudaStream_t st,
                          int slots, float** parts_s, long long** parts_id, int* nparts) {
  const I8Run r = i8_run_plan(n, d, nq, K, slots, bits);
  const I8Plan& b0 = r.p[0];
  I8Ws w;
  const size_t need = i8_ws_carve(r, nq, K, ws, (size_t)-1 / 2, &w);
  if (ws_bytes < need) return fail(PQ_ERR_WORKSPACE, "batched ADC needs %zu workspace bytes", need);
  i8_ws_carve(r, nq, K, ws, ws_bytes, &w);
  PQ_CUDA_TRY(cudaMemsetAsync(w.qhi, 0, (size_t)b0.nq_pad * b0.ldk, st));
  PQ_CUDA_TRY(cudaMemsetAsync(w.qlo, 0, (size_t)b0.nq_pad * b0.ldk, st));
  PQ_CUDA_TRY(cudaMemsetAsync(w.gthr, 0, (size_t)b0.nq_pad * sizeof(unsigned int), st));
  {
    const int pg = (nq + 7) / 8 < num_sms() * 16 ? (nq + 7) / 8 : num_sms() * 16;
    qsplit_i8_kernel<<<pg, 256, 0, st>>>(qrot, nq, d, b0.ldk, bits == 4 ? 1 : 0, w.qhi, w.qlo,
                                         w.qscale, w.qdig);
    PQ_LAUNCH_CHECK("qsplit_i8_kernel");
  }
  const int lut_size = 1 << precision;
  lut_i8_kernel<<<1, 256, 0, st>>>(cent, lut_size, bits == 4 ? bits - precision : 0, w.lut,
                                   w.cscale);
  PQ_LAUNCH_CHECK("lut_i8_kernel");
  CUtensorMap mhi, mlo;
  int rc;
  if ((rc = make_map_u8(&mhi, w.qhi, b0.nq_pad, b0.ldk, b0.ldk, kQBK, kQM, true))) return rc;
  if ((rc = make_map_u8(&mlo, w.qlo, b0.nq_pad, b0.ldk, b0.ldk, kQBK, kQM, true))) return rc;
  int part_base = 0;
  for (int pass = 0; pass < r.npass; ++pass) {
    const I8Plan& b = r.p[pass];
    const int64_t f = r.first[pass];
    if (pass == 1) {
      // Seed each query's threshold with the K-th best of the first pass
      // (its lists are sorted best first).
      rc = launch_merge_sorted(w.out_s, w.out_id, part_base, K, (long long)r.parts * K, K, nq, K,
                               0, w.seed_s, w.seed_id, st);
      if (rc) return rc;
      i8_seed_kernel<<<(nq + 255) / 256, 256, 0, st>>>(w.seed_s, w.seed_id, nq, K, w.gthr);
      PQ_LAUNCH_CHECK("i8_seed_kernel");
    }
    CUtensorMap mraw;
    if ((rc = make_map_u8(&mraw, packed + f * ldb, r.rows[pass], ldb, ldb, kQBK * bits / 8, kQNh,
                          false)))
      return rc;
    BatArgs a;
    a.packed = packed + f * ldb; a.ldb = ldb; a.norms = norms + f; a.n = r.rows[pass];
    a.d = d; a.nk = b.nk; a.shift = bits - precision; a.nq = nq; a.qtiles = b.qtiles;
    a.rchunks = b.rchunks; a.rows_per_chunk = b.rpc; a.K = K; a.cap = b.cap; a.qinv = w.qscale;
    a.cscale = w.cscale; a.lut = w.lut; a.lut_size = lut_size; a.buf_s = w.buf_s;
    a.buf_i = w.buf_i; a.out_s = w.out_s; a.out_id = w.out_id; a.row_offset = row_offset + f;
    a.gthr = w.gthr; a.qdig = w.qdig; a.out_parts = r.parts; a.part_base = part_base;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute at[1];
    i8_config(&cfg, at, b.grid, b.smem, st);
    switch (bits) {
#define PQ_I8_CASE(BB)                                                                          \
  case BB: {                                                                                    \
    auto kern = pair_i8_kernel<BB>;                                                             \
    PQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,        \
                                     (int)b.smem));                                             \
    PQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, mhi, mlo, mraw, a));                             \
  } break;
      PQ_I8_CASE(2)
      PQ_I8_CASE(4)
      PQ_I8_CASE(8)
#undef PQ_I8_CASE
      default:
        return fail(PQ_ERR_INVALID,
                    "the int8 batched kernel takes 2-, 4- or 8-bit codes (got %d)", bits);
    }
    PQ_LAUNCH_CHECK("pair_i8_kernel");
    part_base += 2 * b.rchunks;
  }
  *parts_s = w.out_s;
  *parts_id = w.out_id;
  *nparts = r.parts;
  return PQ_OK;
}

static size_t batched_i8_ws(int64_t n, int d, int nq, int k) {
  if (k + kI8Margin > kBatMaxK || n < kQN || d < kI8MinDim) return 256;
  const int slots = i8_slots();
  if (slots < 1) return 256;
  const I8Run r = i8_run_plan(n, d, nq, k + kI8Margin, slots, 4);
  I8Ws w;
  return i8_ws_carve(r, nq, k + kI8Margin, nullptr, 0, &w);
}
