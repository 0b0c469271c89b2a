// Batched ADC on CTA pairs (tcgen05 .cta_group::2): the same scores, operands
// and fused top-k as batched_adc_kernel, with each MMA spanning the two SMs of
// a cluster.  One pair MMA computes 256 queries x 256 rows x 16: the even CTA
// holds queries [0, 128) and rows [0, 128) of the tile in its shared memory,
// the odd CTA queries [128, 256) and rows [128, 256); each CTA's TMEM receives
// its 128 queries x all 256 rows.  Per SM this halves the shared-memory
// operand traffic of an MMA and the decoding work of a tile (each CTA decodes
// only its 128 rows), which bounded the one-CTA kernel.
//
// Roles per CTA (448 threads): warp 0 loads this CTA's query planes by TMA
// (each CTA its own copy); in the even CTA warp 1 issues the pair MMAs and in the odd
// CTA it relays "query tile landed" to the even CTA; warps 2-5 run the top-k
// epilogue of this CTA's 128 queries; warps 6.. decode this CTA's half of the
// corpus tile.  The even CTA's MMA issuer waits on its own barriers, which the
// odd CTA's decoders, relay and epilogue reach by remote arrivals (mapa);
// tcgen05.commit with a CTA mask tells both CTAs when a stage or an
// accumulator is free or full.  Every wait is bounded (tc::mbar_wait*).
#include "tc.cuh"
#include "topk.cuh"

namespace pqb {

constexpr int kPM = 128;       // queries per CTA (256 per pair)
constexpr int kPN = 256;       // rows per pair tile
constexpr int kPNh = 128;      // rows per CTA
constexpr int kPStages = 3;
constexpr int kPThreads = 15 * 32;
constexpr int kPRawBytes = 16384;  // ring of raw code tiles (TMA), per CTA

// Decoder geometry for B-bit codes: one K block (64 codes) of a row is RB
// bytes, read as PER_ROW segments of SEG bytes (the one-CTA kernel's
// segments); DW decoder warps, UPT segments per thread per stage.
template <int B>
struct PairDec {
  static constexpr int DW = (B >= 4) ? 8 : 4;
  static constexpr int SEG = DecSeg<B>::SEG;
  static constexpr int PER_ROW = DecSeg<B>::PER_ROW;
  static constexpr int WORDS = DecSeg<B>::WORDS;
  static constexpr int CODES = DecSeg<B>::CODES;
  static constexpr int RB = DecSeg<B>::RB;
  static constexpr int UPT = kPNh * PER_ROW / (DW * 32);
  static_assert(UPT >= 1 && UPT * DW * 32 == kPNh * PER_ROW, "decoder split");
  static constexpr int RAWSTAGE = kPNh * RB;   // one K block of this CTA's 128 rows
  static constexpr int RAW = kPRawBytes / RAWSTAGE;
};

struct PairWalk {
  int t, tile, kb, tiles;
  int64_t r0, r1;
};

__device__ __forceinline__ void pair_task(PairWalk& w, const BatArgs& p) {
  const int rc = w.t / p.qtiles;
  w.r0 = (int64_t)rc * p.rows_per_chunk;
  w.r1 = min(p.n, w.r0 + p.rows_per_chunk);
  w.tiles = (int)((w.r1 - w.r0 + kPN - 1) / kPN);
}

__device__ __forceinline__ void pair_next(PairWalk& w, const BatArgs& p, int ntasks, int npairs) {
  if (++w.kb == p.nk) {
    w.kb = 0;
    if (++w.tile == w.tiles) {
      w.tile = 0;
      w.t += npairs;
      if (w.t < ntasks) pair_task(w, p);
    }
  }
}

template <int B>
__global__ void __launch_bounds__(kPThreads, 1)
pair_adc_kernel(const __grid_constant__ CUtensorMap tmQhi, const __grid_constant__ CUtensorMap tmQlo,
                const __grid_constant__ CUtensorMap tmRaw, const BatArgs p) {
  using S = PairDec<B>;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t raw = tc::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  constexpr uint32_t QPLANE = kPM * 128;   // 16 KB: 128 queries x 64 fp16
  constexpr uint32_t XPLANE = kPNh * 128;  // 16 KB: 128 rows x 64 fp16
  constexpr uint32_t STAGE = 2 * QPLANE + 2 * XPLANE;
  const uint32_t meta = base + kPStages * STAGE;
  uint8_t* gmeta = gbase + kPStages * STAGE;
  auto bar = [&](int i) { return meta + 8u * (uint32_t)i; };
  constexpr int FULLA = 0, FULLB = kPStages, PEER = 2 * kPStages, EMPTY = 3 * kPStages,
                TFULL = 4 * kPStages, TEMPTY = 4 * kPStages + 2, DRAIN = 4 * kPStages + 4,
                RAWFULL = 4 * kPStages + 5, RAWEMPTY = RAWFULL + S::RAW,
                NBAR = RAWEMPTY + S::RAW;
  constexpr int NBAR_MAX = 4 * kPStages + 5 + 2 * 8;  // layout is the same for every B
  static_assert(NBAR <= NBAR_MAX, "barrier area");
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(gmeta + 8 * NBAR_MAX);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gmeta + 8 * NBAR_MAX + 4);
  uint32_t* slut = reinterpret_cast<uint32_t*>(gmeta + 8 * NBAR_MAX + 16);       // 256 entries
  float* scratch_s = reinterpret_cast<float*>(gmeta + 8 * NBAR_MAX + 16 + 1024);  // 4 x 512
  int* scratch_i = reinterpret_cast<int*>(gmeta + 8 * NBAR_MAX + 16 + 1024 + 4 * kBatScratch * 4);
  const uint32_t raw_ring =
      (meta + 8 * NBAR_MAX + 16 + 1024 + 4 * kBatScratch * 8 + 127u) & ~127u;
  const uint8_t* graw = smem_raw + (raw_ring - raw);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) {
      tc::mbar_init(bar(FULLA + s), 1);
      tc::mbar_init(bar(FULLB + s), S::DW);
      tc::mbar_init(bar(PEER + s), 1);
      tc::mbar_init(bar(EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(bar(TFULL + b), 1);
      tc::mbar_init(bar(TEMPTY + b), 8);
    }
    tc::mbar_init(bar(DRAIN), 1);
    for (int r = 0; r < S::RAW; ++r) {
      tc::mbar_init(bar(RAWFULL + r), 1);
      tc::mbar_init(bar(RAWEMPTY + r), S::DW);
    }
    *abort_flag = 0;
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmQhi);
    tc::prefetch_tmap(&tmQlo);
    tc::prefetch_tmap(&tmRaw);
  }
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
        const int tiles = (int)((r1 - r0 + kPN - 1) / kPN);
        const int qrow = qt * 2 * kPM + (int)rank * kPM;
        for (int tile = 0; tile < tiles && ok; ++tile) {
          for (int kb = 0; kb < p.nk; ++kb, ++it) {
            const int s = it % kPStages;
            const uint32_t ph = (uint32_t)(it / kPStages) & 1u;
            if (!tc::mbar_wait(bar(EMPTY + s), ph ^ 1u, abort_flag, tc::kErrWaitStageEmpty)) {
              ok = false;
              break;
            }
            const uint32_t st = base + (uint32_t)s * STAGE;
            tc::mbar_arrive_expect_tx(bar(FULLA + s), 2 * QPLANE);
            tc::tma_load_2d(st, &tmQhi, kb * kBatBK, qrow, bar(FULLA + s));
            tc::tma_load_2d(st + QPLANE, &tmQlo, kb * kBatBK, qrow, bar(FULLA + s));
          }
        }
      }
      for (int j = it - kPStages; j < it; ++j) {
        if (j < 0) continue;
        volatile int never = 0;
        tc::mbar_wait(bar(FULLA + j % kPStages), (uint32_t)(j / kPStages) & 1u, &never,
                      tc::kErrWaitTmaFull);
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
        const int tiles = (int)((r1 - r0 + kPN - 1) / kPN);
        for (int tile = 0; tile < tiles && ok; ++tile) {
          for (int kb = 0; kb < p.nk; ++kb, ++it) {
            const int s = it % kPStages;
            const uint32_t ph = (uint32_t)(it / kPStages) & 1u;
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
      const uint32_t idesc = tc::idesc_f16_f32(2 * kPM, kPN);
      int it = 0, tcount = 0;
      bool ok = true;
      for (int t = pair; t < ntasks && ok; t += npairs) {
        const int rc = t / p.qtiles;
        const int64_t r0 = (int64_t)rc * p.rows_per_chunk;
        const int64_t r1 = min(p.n, r0 + p.rows_per_chunk);
        const int tiles = (int)((r1 - r0 + kPN - 1) / kPN);
        for (int tile = 0; tile < tiles && ok; ++tile, ++tcount) {
          const int buf = tcount & 1;
          const uint32_t tph = (uint32_t)(tcount >> 1) & 1u;
          if (!tc::mbar_wait_cluster(bar(TEMPTY + buf), tph ^ 1u, abort_flag,
                                     tc::kErrWaitAccEmpty)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)(buf * kPN);
          for (int kb = 0; kb < p.nk; ++kb, ++it) {
            const int s = it % kPStages;
            const uint32_t ph = (uint32_t)(it / kPStages) & 1u;
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
            for (int kk = 0; kk < kBatBK / 16; ++kk) {
              const uint32_t off = (uint32_t)kk * 32u;
              tc::mma_f16_pair(d_tmem, tc::sw128_desc(q_hi + off), tc::sw128_desc(x_hi + off),
                               idesc, (kb | kk) != 0);
              tc::mma_f16_pair(d_tmem, tc::sw128_desc(q_hi + off), tc::sw128_desc(x_lo + off),
                               idesc, 1);
              tc::mma_f16_pair(d_tmem, tc::sw128_desc(q_lo + off), tc::sw128_desc(x_hi + off),
                               idesc, 1);
            }
            tc::mma_commit_pair(bar(EMPTY + s), 3);
          }
          if (ok) tc::mma_commit_pair(bar(TFULL + buf), 3);
        }
      }
      tc::mma_commit_pair(bar(DRAIN), 1);
      volatile int never = 0;
      tc::mbar_wait(bar(DRAIN), 0, &never, tc::kErrWaitAccFull);
    }
  } else if (warp == 14) {
    if (lane == 0) {
      // ---------------- TMA producer: raw code tiles of this CTA's 128 rows ----------------
      const int half = (int)rank * kPNh;
      int it = 0;
      bool ok = true;
      for (int t = pair; t < ntasks && ok; t += npairs) {
        const int rc = t / p.qtiles;
        const int64_t r0 = (int64_t)rc * p.rows_per_chunk;
        const int64_t r1 = min(p.n, r0 + p.rows_per_chunk);
        const int tiles = (int)((r1 - r0 + kPN - 1) / kPN);
        for (int tile = 0; tile < tiles && ok; ++tile) {
          const int y = (int)(r0 + (int64_t)tile * kPN + half);
          for (int kb = 0; kb < p.nk; ++kb, ++it) {
            const int r = it % S::RAW;
            const uint32_t ph = (uint32_t)(it / S::RAW) & 1u;
            if (!tc::mbar_wait(bar(RAWEMPTY + r), ph ^ 1u, abort_flag, tc::kErrWaitStageEmpty)) {
              ok = false;
              break;
            }
            tc::mbar_arrive_expect_tx(bar(RAWFULL + r), (uint32_t)S::RAWSTAGE);
            tc::tma_load_2d(raw_ring + (uint32_t)(r * S::RAWSTAGE), &tmRaw, kb * S::RB, y,
                            bar(RAWFULL + r));
          }
        }
      }
      for (int j = it - S::RAW; j < it; ++j) {
        if (j < 0) continue;
        volatile int never = 0;
        tc::mbar_wait(bar(RAWFULL + j % S::RAW), (uint32_t)(j / S::RAW) & 1u, &never,
                      tc::kErrWaitTmaFull);
      }
    }
  } else if (warp >= 6) {
    if (warp < 6 + S::DW) {
      // ---------------- decoder: this CTA's 128 rows of each tile ----------------
      // Raw codes arrive by TMA in a ring several K blocks ahead; each thread
      // decodes UPT segments (rows r, byte segments sg) of the current block.
      const int dt = threadIdx.x - 6 * 32;
      const int half = (int)rank * kPNh;
      PairWalk w;
      w.t = pair;
      w.tile = 0;
      w.kb = 0;
      if (w.t < ntasks) pair_task(w, p);
      for (int it = 0; w.t < ntasks; ++it) {
        const int rr = it % S::RAW;
        const uint32_t rph = (uint32_t)(it / S::RAW) & 1u;
        const PairWalk here = w;
        pair_next(w, p, ntasks, npairs);
        const int s = it % kPStages;
        const uint32_t ph = (uint32_t)(it / kPStages) & 1u;
        if (!tc::mbar_wait(bar(RAWFULL + rr), rph, abort_flag, tc::kErrWaitTmaFull) ||
            !tc::mbar_wait(bar(EMPTY + s), ph ^ 1u, abort_flag, tc::kErrWaitStageEmpty))
          break;
        uint32_t cur[S::UPT][S::WORDS];
        const uint8_t* rawp = graw + rr * S::RAWSTAGE;
#pragma unroll
        for (int i = 0; i < S::UPT; ++i) {
          const int u = dt + i * S::DW * 32;  // = r * PER_ROW + sg: byte offset u * SEG
          if constexpr (S::SEG == 16) {
            const uint4 v = *reinterpret_cast<const uint4*>(rawp + u * 16);
            cur[i][0] = v.x; cur[i][1] = v.y; cur[i][2] = v.z; cur[i][3] = v.w;
          } else {
#pragma unroll
            for (int j = 0; j < S::WORDS; ++j)
              cur[i][j] = *reinterpret_cast<const uint32_t*>(rawp + u * S::SEG + 4 * j);
          }
        }
        uint8_t* xh = gbase + (size_t)s * STAGE + 2 * QPLANE;
        uint8_t* xl = xh + XPLANE;
        const int64_t tr0 = here.r0 + (int64_t)here.tile * kPN + half;
#pragma unroll
        for (int i = 0; i < S::UPT; ++i) {
          const int u = dt + i * S::DW * 32;
          const int r = u / S::PER_ROW, sg = u % S::PER_ROW;
          const bool live = tr0 + r < here.r1;
#pragma unroll
          for (int cc = 0; cc < S::CODES / 8; ++cc) {
            uint4 vh = make_uint4(0, 0, 0, 0), vl = make_uint4(0, 0, 0, 0);
            if (live) {
              uint32_t e[8];
#pragma unroll
              for (int t2 = 0; t2 < 8; ++t2)
                e[t2] = slut[seg_code<B>(cur[i], cc * 8 + t2) >> p.shift];
              vh.x = __byte_perm(e[0], e[1], 0x5410);
              vh.y = __byte_perm(e[2], e[3], 0x5410);
              vh.z = __byte_perm(e[4], e[5], 0x5410);
              vh.w = __byte_perm(e[6], e[7], 0x5410);
              vl.x = __byte_perm(e[0], e[1], 0x7632);
              vl.y = __byte_perm(e[2], e[3], 0x7632);
              vl.z = __byte_perm(e[4], e[5], 0x7632);
              vl.w = __byte_perm(e[6], e[7], 0x7632);
            }
            const int c = sg * (S::CODES / 8) + cc;
            const uint32_t off = (uint32_t)r * 128u + ((uint32_t)(c ^ (r & 7)) << 4);
            *reinterpret_cast<uint4*>(xh + off) = vh;
            *reinterpret_cast<uint4*>(xl + off) = vl;
          }
        }
        // Generic-proxy stores become visible to the tensor core (async proxy);
        // the odd CTA's relay forwards completion to the even CTA.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          tc::mbar_arrive(bar(FULLB + s));
          tc::mbar_arrive(bar(RAWEMPTY + rr));  // the raw codes were consumed by the stores
        }
      }
    }
  } else {
    // ---------------- epilogue: warps 2..5, thread = query ----------------
    const int ew = warp - 2;
    const int q_lane = 32 * (warp & 3) + lane;
    float* ss = scratch_s + ew * kBatScratch;
    int* si = scratch_i + ew * kBatScratch;
    const float csc = p.cscale[0];
    const size_t slot = (size_t)blockIdx.x * kPM;
    int tcount = 0;
    for (int t = pair; t < ntasks; t += npairs) {
      const int rc = t / p.qtiles, qt = t % p.qtiles;
      const int64_t r0 = (int64_t)rc * p.rows_per_chunk;
      const int64_t r1 = min(p.n, r0 + p.rows_per_chunk);
      const int tiles = (int)((r1 - r0 + kPN - 1) / kPN);
      const int qbase = qt * 2 * kPM + (int)rank * kPM;
      const int qg = qbase + q_lane;
      const bool qv = qg < p.nq;
      const float qs = qv ? p.qinv[qg] * csc : 0.f;
      float* bs = p.buf_s + (slot + q_lane) * p.cap;
      int* bi = p.buf_i + (slot + q_lane) * p.cap;
      int cnt = 0;
      float thr = -INFINITY;
      bool ok = true;
      for (int tile = 0; tile < tiles; ++tile, ++tcount) {
        const int buf = tcount & 1;
        const uint32_t tph = (uint32_t)(tcount >> 1) & 1u;
        if (!tc::mbar_wait(bar(TFULL + buf), tph, abort_flag, tc::kErrWaitAccFull)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        // A query's shared threshold: the best K-th score any chunk's buffer
        // of this launch has reached.  Rows below it cannot enter the
        // query's overall top K (each published value is the K-th best of K
        // real candidates).
        if (p.gthr != nullptr && qv) {
          const unsigned gk = __ldcg(p.gthr + qg);
          if (gk != 0u) thr = fmaxf(thr, key_to_float(gk));
        }
        const int64_t tr0 = r0 + (int64_t)tile * kPN;
        const uint32_t taddr =
            tmem_base + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(buf * kPN);
        for (int c0 = 0; c0 < kPN; c0 += 32) {
          uint32_t v[32];
          __syncwarp();
          tc::tmem_ld16(taddr + (uint32_t)c0, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
          tc::tmem_ld16(taddr + (uint32_t)c0 + 16u, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
          tc::tmem_ld_wait(v);
          uint32_t need = __ballot_sync(0xffffffffu, qv && cnt + 32 > p.cap);
          while (need) {
            const int src = __ffs(need) - 1;
            need &= need - 1;
            float* sbs = p.buf_s + (slot + 32 * (warp & 3) + src) * p.cap;
            int* sbi = p.buf_i + (slot + 32 * (warp & 3) + src) * p.cap;
            const float before = thr;
            warp_select(src, lane, cnt, sbs, sbi, p.K, cnt, thr);
            if (lane == src) {
              thr = fmaxf(thr, before);  // never below a threshold already adopted
              if (p.gthr != nullptr) atomicMax(p.gthr + qg, ordered_key(thr));  // publish
            }
          }
          const int64_t rb = tr0 + c0;
          // The 32 rows' norms: one coalesced load, broadcast by shuffles.
          const float my_norm = (rb + lane < r1) ? __ldg(p.norms + rb + lane) : 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float nr = __shfl_sync(0xffffffffu, my_norm, i);
            const int64_t row = rb + i;
            if (qv && row < r1) {
              const float sc = __uint_as_float(v[i]) * qs * nr;
              if (sc > thr) {
                bs[cnt] = sc;
                bi[cnt] = (int)row;
                ++cnt;
              }
            }
          }
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader) tc::mbar_arrive(bar(TEMPTY + buf));
          else tc::mbar_arrive_cluster(lead_bar(TEMPTY + buf));
        }
      }
      if (!ok) break;
      __syncwarp();
      uint32_t pend = __ballot_sync(0xffffffffu, qv);
      while (pend) {
        const int src = __ffs(pend) - 1;
        pend &= pend - 1;
        const int sq = qbase + 32 * (warp & 3) + src;
        float* sbs = p.buf_s + (slot + 32 * (warp & 3) + src) * p.cap;
        int* sbi = p.buf_i + (slot + 32 * (warp & 3) + src) * p.cap;
        const size_t o = ((size_t)sq * p.rchunks + rc) * p.K;
        warp_compact(src, lane, cnt, sbs, sbi, p.K, ss, si, cnt, thr, p.out_s + o, p.out_id + o,
                     p.row_offset);
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

struct PairPlan {
  int ldk, nk, nq_pad, qtiles, rchunks, grid, cap;
  int64_t rpc;
  size_t smem;
};

static size_t pair_smem() {
  return 1024 + (size_t)kPStages * (2 * kPM * 128 + 2 * kPNh * 128) + 8 * (4 * kPStages + 5 + 16) +
         16 + 1024 + (size_t)4 * kBatScratch * 8 + 128 + kPRawBytes;
}

// The pair kernel covers 2-, 4- and 8-bit codes (raw K blocks of 16, 32 and
// 64 bytes per row, a whole number of 16-byte TMA units) and corpora of at
// least one pair tile.
static bool pair_covers(int64_t n, int bits) {
  return (bits == 2 || bits == 4 || bits == 8) && n >= kPN;
}

static void pair_config(cudaLaunchConfig_t* cfg, cudaLaunchAttribute* at, int grid,
                        cudaStream_t st) {
  *cfg = cudaLaunchConfig_t{};
  cfg->gridDim = dim3(grid);
  cfg->blockDim = dim3(kPThreads);
  cfg->dynamicSmemBytes = pair_smem();
  cfg->stream = st;
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg->attrs = at;
  cfg->numAttrs = 1;
}

// CTA pairs that fit on the GPU at once (one pair per two SMs of a cluster);
// 0 when pair launches are unavailable.
static int pair_slots() {
  static int slots = -1;
  if (slots < 0) {
    int c = 0;
    auto kern = pair_adc_kernel<4>;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute at[1];
    pair_config(&cfg, at, 2 * (num_sms() / 2), 0);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)pair_smem()) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&c, (void*)kern, &cfg) != cudaSuccess) {
      cudaGetLastError();
      c = 0;
    }
    slots = c < num_sms() / 2 ? c : num_sms() / 2;
  }
  return slots;
}

static PairPlan pair_plan(int64_t n, int d, int nq, int k, int slots) {
  PairPlan b;
  b.ldk = (d + kBatBK - 1) / kBatBK * kBatBK;
  b.nk = b.ldk / kBatBK;
  b.qtiles = (nq + 2 * kPM - 1) / (2 * kPM);
  b.nq_pad = b.qtiles * 2 * kPM;
  // Row chunks per query tile: the smallest count whose task total fills the
  // pair slots in whole waves (>= 97% of the last wave busy); tasks stay >= 4
  // row tiles long.
  const int64_t min_rows = 4 * kPN;
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
  b.rpc = ((n + rc - 1) / rc + kPN - 1) / kPN * kPN;
  if (b.rpc < kPN) b.rpc = kPN;
  b.rchunks = (int)((n + b.rpc - 1) / b.rpc);
  if (b.rchunks < 1) b.rchunks = 1;
  const int tasks = b.qtiles * b.rchunks;
  b.grid = 2 * (tasks < slots ? tasks : slots);
  b.cap = 2 * k;
  if (b.cap < 64) b.cap = 64;
  b.smem = pair_smem();
  return b;
}

static size_t pair_ws_carve(const PairPlan& b, int nq, int K, void* ws, size_t ws_bytes,
                            BatWs* w) {
  Carve cv(ws, ws_bytes);
  w->qhi = cv.take<__half>((size_t)b.nq_pad * b.ldk);
  w->qlo = cv.take<__half>((size_t)b.nq_pad * b.ldk);
  w->qinv = cv.take<float>((size_t)b.nq_pad);
  w->cscale = cv.take<float>(4);
  w->lut = cv.take<uint32_t>(256);
  w->buf_s = cv.take<float>((size_t)b.grid * kPM * b.cap);
  w->buf_i = cv.take<int>((size_t)b.grid * kPM * b.cap);
  w->out_s = cv.take<float>((size_t)nq * b.rchunks * K);
  w->out_id = cv.take<long long>((size_t)nq * b.rchunks * K);
  w->gthr = cv.take<unsigned int>((size_t)b.nq_pad);
  return cv.off + 256;
}

}  // namespace pqb

using namespace pqb;

// Batched ADC: the CTA-pair kernel when pair launches are available, else the
// one-CTA kernel.  Leaves per-(query, row chunk) top-K lists in ws (layout
// [nq][rchunks][K]) and returns their location.
static int run_batched(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                       int bits, int precision, const float* qrot, int nq, const float* cent, int K,
                       int64_t row_offset, void* ws, size_t ws_bytes, cudaStream_t st,
                       float** parts_s, long long** parts_id, int* nparts, int* kpart) {
  *kpart = K;
  if (i8_eligible(n, d, ldb, bits, K) &&
      rerank_smem(d, precision, K + kI8Margin, K) <= 227 * 1024) {
    const int s8 = i8_slots();
    if (s8 >= 1) {
      *kpart = K + kI8Margin;
      return run_batched_i8(packed, ldb, norms, n, d, bits, precision, qrot, nq, cent,
                            K + kI8Margin, row_offset, ws, ws_bytes, st, s8, parts_s, parts_id,
                            nparts);
    }
  }
  const int slots = pair_covers(n, bits) ? pair_slots() : 0;
  if (slots < 1)
    return run_batched_1cta(packed, ldb, norms, n, d, bits, precision, qrot, nq, cent, K,
                            row_offset, ws, ws_bytes, st, parts_s, parts_id, nparts);
  const PairPlan b = pair_plan(n, d, nq, K, slots);
  BatWs w;
  const size_t need = pair_ws_carve(b, nq, K, ws, (size_t)-1 / 2, &w);
  if (ws_bytes < need) return fail(PQ_ERR_WORKSPACE, "batched ADC needs %zu workspace bytes", need);
  pair_ws_carve(b, nq, K, ws, ws_bytes, &w);
  PQ_CUDA_TRY(cudaMemsetAsync(w.qhi, 0, (size_t)b.nq_pad * b.ldk * 2, st));
  PQ_CUDA_TRY(cudaMemsetAsync(w.qlo, 0, (size_t)b.nq_pad * b.ldk * 2, st));
  PQ_CUDA_TRY(cudaMemsetAsync(w.gthr, 0, (size_t)b.nq_pad * sizeof(unsigned int), st));
  {
    const int pg = (nq + 7) / 8 < num_sms() * 16 ? (nq + 7) / 8 : num_sms() * 16;
    encode_prep_kernel<false><<<pg, 256, 0, st>>>(qrot, nq, d, b.ldk, w.qhi, w.qlo, w.qinv,
                                                  nullptr);
    PQ_LAUNCH_CHECK("encode_prep_kernel");
  }
  const int lut_size = 1 << precision;
  batch_lut_kernel<<<1, 256, 0, st>>>(cent, lut_size, w.lut, w.cscale);
  PQ_LAUNCH_CHECK("batch_lut_kernel");
  CUtensorMap mhi, mlo;
  int rc;
  if ((rc = make_map(&mhi, w.qhi, b.nq_pad, b.ldk, kPM))) return rc;
  if ((rc = make_map(&mlo, w.qlo, b.nq_pad, b.ldk, kPM))) return rc;
  CUtensorMap mraw;
  {
    auto fn = get_encode_fn();
    if (!fn) return fail(PQ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)ldb, (cuuint64_t)n};
    cuuint64_t strides[1] = {(cuuint64_t)ldb};
    cuuint32_t box[2] = {(cuuint32_t)(8 * bits), (cuuint32_t)kPNh};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(&mraw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(packed), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return fail(PQ_ERR_CUDA, "cuTensorMapEncodeTiled (code tiles) failed (%d)", (int)r);
  }
  BatArgs a;
  a.packed = packed; a.ldb = ldb; a.norms = norms; a.n = n; a.d = d; a.nk = b.nk;
  a.shift = bits - precision; a.nq = nq; a.qtiles = b.qtiles; a.rchunks = b.rchunks;
  a.rows_per_chunk = b.rpc; a.K = K; a.cap = b.cap; a.qinv = w.qinv; a.cscale = w.cscale;
  a.lut = w.lut; a.lut_size = lut_size; a.buf_s = w.buf_s; a.buf_i = w.buf_i;
  a.out_s = w.out_s; a.out_id = w.out_id; a.row_offset = row_offset; a.gthr = w.gthr; a.qdig = nullptr;
  a.out_parts = b.rchunks; a.part_base = 0;
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute at[1];
  pair_config(&cfg, at, b.grid, st);
  switch (bits) {
#define PQ_PAIR_CASE(BB)                                                                        \
  case BB: {                                                                                    \
    auto kern = pair_adc_kernel<BB>;                                                            \
    PQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,        \
                                     (int)b.smem));                                             \
    PQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, mhi, mlo, mraw, a));                                   \
  } break;
    PQ_PAIR_CASE(2)
    PQ_PAIR_CASE(4)
    PQ_PAIR_CASE(8)
#undef PQ_PAIR_CASE
    default:
      return fail(PQ_ERR_INVALID, "bits must be one of 1,2,3,4,8 (got %d)", bits);
  }
  PQ_LAUNCH_CHECK("pair_adc_kernel");
  *parts_s = w.out_s;
  *parts_id = w.out_id;
  *nparts = b.rchunks;
  return PQ_OK;
}

extern "C" int pq_adc_batch_kernel(int64_t n, int d, int bits, int precision, int k,
                                   int64_t ldb) {
  if (i8_eligible(n, d, ldb, bits, k) &&
      rerank_smem(d, precision, k + kI8Margin, k) <= 227 * 1024 && i8_slots() >= 1)
    return 1;
  return (pair_covers(n, bits) && pair_slots() >= 1) ? 2 : 3;
}

static size_t batched_ws(int64_t n, int d, int nq, int k) {
  if (n <= 0 || nq <= 0 || k <= 0 || d <= 0) return 256;
  const size_t one = batched_ws_1cta(n, d, nq, k);
  const int slots = pair_slots();  // any width: the workspace does not depend on it
  if (slots < 1) return one;
  const PairPlan b = pair_plan(n, d, nq, k, slots);
  BatWs w;
  const size_t two = pair_ws_carve(b, nq, k, nullptr, 0, &w);
  const size_t three = batched_i8_ws(n, d, nq, k);
  const size_t m = one > two ? one : two;
  return m > three ? m : three;
}
