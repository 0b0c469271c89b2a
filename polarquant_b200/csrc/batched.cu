// Batched ADC on the tensor cores: scores S[q, r] = norm_r * sum_j
// q_rot[q, j] * cent[code_rj >> shift] for a batch of queries against packed
// rows, with an exact per-query top-k fused into the epilogue.  Replaces
// Quantizer.search_batch (remex/core.py:721-778: Q_rot @ X_hat_rot^T * norms,
// per-row argpartition/argsort) and serves the coarse stage of two-stage
// search for query batches.
//
// Operands.  A = the rotated queries, split into fp16 hi/lo planes with a
// per-query power-of-two scale (the encode prep kernel), loaded by TMA as
// 128 x 64 tiles with 128-byte swizzle.  B = the corpus rows: four decoder
// warps read packed codes, shift out the Matryoshka precision, look up the
// centroid (fp16 hi/lo pair of cent * 2^ec) in a shared table and write
// 256 x 64 tiles in the same swizzled layout.  Three kind::f16 MMAs per K step
// (hi*hi + hi*lo + lo*hi) accumulate 128 queries x 256 rows in TMEM (two
// buffers).  Accuracy: ~22-bit operands, f32 accumulation, scores within
// ~1e-6 relative of the f32 reference.
//
// Epilogue.  Thread = query (TMEM lane).  Each score above the query's
// current k-th best is appended to that query's buffer in global memory; when
// a buffer could overflow, the warp sorts it in shared memory and keeps the
// best k, which raises the threshold.  Rows are visited in increasing order,
// so a later row that ties the k-th score is correctly rejected and the
// result is the exact top-k under (score desc, row asc).
//
// Work split.  A task is (row chunk, 128-query tile); persistent CTAs walk the
// tasks row-chunk-major so concurrent CTAs share corpus rows in L2.  Each task
// writes its top-k lists; a merge over row chunks gives the final top-k.
#include "tc.cuh"
#include "topk.cuh"

namespace pqb {

constexpr int kBatM = 128;
constexpr int kBatN = 256;
constexpr int kBatBK = 64;
constexpr int kBatStages = 2;
constexpr int kBatDecWarps = 8;
constexpr int kBatThreads = (6 + kBatDecWarps) * 32;  // w0 TMA(Q), w1 MMA + TMEM, w2-5 epilogue, w6.. decoder
constexpr int kBatMaxK = 256;
constexpr int kBatScratch = 512;  // per-warp sort scratch entries (power of two >= 2*kBatMaxK)

struct BatArgs {
  const uint8_t* packed;
  int64_t ldb;
  const float* norms;
  int64_t n;
  int d, nk, shift;
  int nq, qtiles, rchunks;
  int64_t rows_per_chunk;
  int K, cap;
  const float* qinv;      // per query 2^-(e_q + 14)
  const float* cscale;    // [0] = 2^(14 - ec)
  const uint32_t* lut;    // 2^P entries: fp16 hi | fp16 lo << 16 of cent * 2^ec
  int lut_size;
  float* buf_s;           // [grid][128][cap]
  int* buf_i;
  float* out_s;           // [nq][rchunks][K]
  long long* out_id;
  long long row_offset;
  unsigned int* gthr;     // int8 kernel: per-query running threshold (ordered key, 0 = none)
  const int* qdig;        // int8 kernel: per query {sum |hi digit|, sum |lo digit|}
  int out_parts;          // int8 kernel: lists per query in out_s / out_id
  int part_base;          // int8 kernel: this launch's first list
};

// Loads the 8 codes k0..k0+7 (k0 % 8 == 0) of a row as the low bits of c[].
template <int B>
__device__ __forceinline__ void load8(const uint8_t* row, int k0, uint32_t (&c)[8]) {
  if constexpr (B == 8) {
    const uint2 v = *reinterpret_cast<const uint2*>(row + k0);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      c[t] = (v.x >> (8 * t)) & 255u;
      c[4 + t] = (v.y >> (8 * t)) & 255u;
    }
  } else if constexpr (B == 4) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(row + k0 / 2);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      c[2 * t] = (w >> (8 * t + 4)) & 15u;
      c[2 * t + 1] = (w >> (8 * t)) & 15u;
    }
  } else if constexpr (B == 2) {
    const uint32_t w = *reinterpret_cast<const uint16_t*>(row + k0 / 4);
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int u = 0; u < 4; ++u) c[4 * t + u] = (w >> (8 * t + 6 - 2 * u)) & 3u;
  } else if constexpr (B == 1) {
    const uint32_t w = row[k0 / 8];
#pragma unroll
    for (int u = 0; u < 8; ++u) c[u] = (w >> (7 - u)) & 1u;
  } else {  // 3 bits: one 3-byte group, big-endian 24-bit value
    const uint8_t* g = row + (k0 / 8) * 3;
    const uint32_t v = ((uint32_t)g[0] << 16) | ((uint32_t)g[1] << 8) | (uint32_t)g[2];
#pragma unroll
    for (int u = 0; u < 8; ++u) c[u] = (v >> (21 - 3 * u)) & 7u;
  }
}

// Decoder geometry for B-bit codes: one K block (64 codes) of a row is RB
// bytes, read as PER_ROW segments of SEG bytes; every decoder thread owns UPT
// segments of each stage.
template <int B>
struct DecSeg {
  static constexpr int RB = 8 * B;
  static constexpr int SEG = (B == 3) ? 24 : (RB < 16 ? RB : 16);
  static constexpr int PER_ROW = RB / SEG;
  static constexpr int UPT = kBatN * PER_ROW / (kBatDecWarps * 32);
  static constexpr int WORDS = SEG / 4;
  static constexpr int CODES = SEG * 8 / B;
};

template <int B>
__device__ __forceinline__ void load_seg(const uint8_t* p, uint32_t (&w)[DecSeg<B>::WORDS]) {
  if constexpr (DecSeg<B>::SEG == 16) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else {
#pragma unroll
    for (int i = 0; i < DecSeg<B>::WORDS / 2; ++i) {
      const uint2 v = __ldg(reinterpret_cast<const uint2*>(p) + i);
      w[2 * i] = v.x;
      w[2 * i + 1] = v.y;
    }
  }
}

// Code t of a segment (MSB-first stream starting at the segment's first byte).
template <int B>
__device__ __forceinline__ uint32_t seg_code(const uint32_t* w, int t) {
  if constexpr (B == 3) {
    const int g = t >> 3, u = t & 7;
    auto byte = [&](int i) { return (w[i >> 2] >> (8 * (i & 3))) & 255u; };
    const uint32_t v = (byte(3 * g) << 16) | (byte(3 * g + 1) << 8) | byte(3 * g + 2);
    return (v >> (21 - 3 * u)) & 7u;
  } else {
    const int p = t * B;
    const int byte = p >> 3, sh = 8 - B - (p & 7);
    return (w[byte >> 2] >> (8 * (byte & 3) + sh)) & ((1u << B) - 1u);
  }
}

// The (task, tile, k-block) sequence every role of the batched kernel walks.
struct BatWalk {
  int t, tile, kb, tiles;
  int64_t r0, r1;
};

__device__ __forceinline__ void walk_task(BatWalk& w, const BatArgs& p) {
  const int rc = w.t / p.qtiles;
  w.r0 = (int64_t)rc * p.rows_per_chunk;
  w.r1 = min(p.n, w.r0 + p.rows_per_chunk);
  w.tiles = (int)((w.r1 - w.r0 + kBatN - 1) / kBatN);
}

__device__ __forceinline__ void walk_next(BatWalk& w, const BatArgs& p, int ntasks) {
  if (++w.kb == p.nk) {
    w.kb = 0;
    if (++w.tile == w.tiles) {
      w.tile = 0;
      w.t += gridDim.x;
      if (w.t < ntasks) walk_task(w, p);
    }
  }
}

template <int B>
__device__ __forceinline__ void dec_load(const BatArgs& p, const BatWalk& w, int dt,
                                         uint32_t (&seg)[DecSeg<B>::UPT][DecSeg<B>::WORDS]) {
  using S = DecSeg<B>;
  const int64_t tr0 = w.r0 + (int64_t)w.tile * kBatN;
#pragma unroll
  for (int i = 0; i < S::UPT; ++i) {
    const int u = dt + i * kBatDecWarps * 32;
    const int r = u / S::PER_ROW, sg = u % S::PER_ROW;
    const int64_t row = tr0 + r;
    if (row < w.r1) {
      load_seg<B>(p.packed + row * p.ldb + (int64_t)w.kb * S::RB + sg * S::SEG, seg[i]);
    } else {
#pragma unroll
      for (int j = 0; j < S::WORDS; ++j) seg[i][j] = 0xFFFFFFFFu;  // marks a padding row
    }
  }
}

__device__ __forceinline__ uint32_t ordered_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Warp-cooperative selection on lane `src`'s candidate buffer (n <= 512
// entries, appended in increasing row order): finds the K-th largest score by
// a 32-step radix search on order-preserving keys, then compacts in place to
// the entries above it plus the earliest (lowest-row) entries equal to it, so
// exactly K remain.  Lane src receives the new count and threshold.  About a
// fifth of the cost of sorting the buffer.
__device__ __forceinline__ void warp_select(int src, int lane, int n_src, float* bs, int* bi, int K,
                                            int& cnt, float& thr) {
  __syncwarp();
  const int n = __shfl_sync(0xffffffffu, n_src, src);
  if (n <= K) return;
  constexpr int PER = kBatScratch / 32;  // 16 entries per lane
  uint32_t key[PER];
  float sv[PER];
  int iv[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = j * 32 + lane;
    sv[j] = (e < n) ? bs[e] : -INFINITY;
    iv[j] = (e < n) ? bi[e] : 0;
    key[j] = (e < n) ? ordered_key(sv[j]) : 0u;
  }
  uint32_t prefix = 0;
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t cand = prefix | (1u << bit);
    int c = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) c += key[j] >= cand;
    c = (int)__reduce_add_sync(0xffffffffu, (unsigned)c);
    if (c >= K) prefix = cand;
  }
  // prefix = K-th largest key.  Keep key > prefix, then ties in buffer order.
  int above = 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) above += key[j] > prefix;
  above = (int)__reduce_add_sync(0xffffffffu, (unsigned)above);
  int ties_left = K - above;
  int out = 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const bool gt = key[j] > prefix;
    const bool eq = key[j] == prefix && (j * 32 + lane) < n;
    const uint32_t eqm = __ballot_sync(0xffffffffu, eq);
    const int eq_rank = __popc(eqm & ((1u << lane) - 1u));
    const bool keep = gt || (eq && eq_rank < ties_left);
    const uint32_t km = __ballot_sync(0xffffffffu, keep);
    if (keep) {
      const int pos = out + __popc(km & ((1u << lane) - 1u));
      bs[pos] = sv[j];
      bi[pos] = iv[j];
    }
    out += __popc(km);
    ties_left -= min(ties_left, __popc(eqm));
  }
  // Scores equal to the threshold arriving later have larger rows: rejected.
  uint32_t tk = prefix;
  const float t = __uint_as_float((tk & 0x80000000u) ? (tk & 0x7FFFFFFFu) : ~tk);
  __syncwarp();
  if (lane == src) {
    cnt = K;
    thr = t;
  }
}

// Warp-cooperative: sort lane `src`'s candidate buffer (n entries) and keep
// the best K; lane src receives the new count and threshold.  When `out_s`
// is non-null the best K (padded with -inf / -1) are also written there.
__device__ __forceinline__ void warp_compact(int src, int lane, int n_src, float* bs, int* bi,
                                             int K, float* ss, int* si, int& cnt, float& thr,
                                             float* out_s, long long* out_id, long long id_off) {
  __syncwarp();  // lane src's appends to its buffer are visible to the warp
  const int n = __shfl_sync(0xffffffffu, n_src, src);
  int NP = 32;
  while (NP < n) NP <<= 1;
  if (NP < K) {
    NP = 32;
    while (NP < K) NP <<= 1;
  }
  for (int j = lane; j < NP; j += 32) {
    ss[j] = (j < n) ? bs[j] : -INFINITY;
    si[j] = (j < n) ? bi[j] : 0x7fffffff;
  }
  __syncwarp();
  for (int k = 2; k <= NP; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = lane; i < NP; i += 32) {
        const int l = i ^ j;
        if (l > i) {
          const bool desc = (i & k) == 0;
          const float a = ss[i], b = ss[l];
          const int ia = si[i], ib = si[l];
          const bool l_better = b > a || (b == a && ib < ia);
          const bool i_better = a > b || (a == b && ia < ib);
          if (desc ? l_better : i_better) {
            ss[i] = b; ss[l] = a;
            si[i] = ib; si[l] = ia;
          }
        }
      }
      __syncwarp();
    }
  }
  const int m = n < K ? n : K;
  for (int j = lane; j < m; j += 32) {
    bs[j] = ss[j];
    bi[j] = si[j];
  }
  if (out_s) {
    for (int j = lane; j < K; j += 32) {
      out_s[j] = (j < m) ? ss[j] : -INFINITY;
      out_id[j] = (j < m) ? (long long)si[j] + id_off : -1ll;
    }
  }
  const float nt = (n >= K) ? ss[K - 1] : -INFINITY;
  __syncwarp();
  if (lane == src) {
    cnt = m;
    thr = nt;
  }
}

template <int B>
__global__ void __launch_bounds__(kBatThreads, 1)
batched_adc_kernel(const __grid_constant__ CUtensorMap tmQhi, const __grid_constant__ CUtensorMap tmQlo,
                   const BatArgs p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t raw = tc::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  constexpr uint32_t QPLANE = kBatM * 128;   // 16 KB
  constexpr uint32_t XPLANE = kBatN * 128;   // 32 KB
  constexpr uint32_t STAGE = 2 * QPLANE + 2 * XPLANE;
  const uint32_t meta = base + kBatStages * STAGE;
  uint8_t* gmeta = gbase + kBatStages * STAGE;
  auto bar = [&](int i) { return meta + 8u * (uint32_t)i; };
  constexpr int FULLA = 0, FULLB = kBatStages, EMPTY = 2 * kBatStages, TFULL = 3 * kBatStages,
                TEMPTY = 3 * kBatStages + 2, DRAIN = 3 * kBatStages + 4, NBAR = 3 * kBatStages + 5;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(gmeta + 8 * NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gmeta + 8 * NBAR + 4);
  uint32_t* slut = reinterpret_cast<uint32_t*>(gmeta + 8 * NBAR + 16);       // 256 entries
  float* scratch_s = reinterpret_cast<float*>(gmeta + 8 * NBAR + 16 + 1024);  // 4 x 512
  int* scratch_i = reinterpret_cast<int*>(gmeta + 8 * NBAR + 16 + 1024 + 4 * kBatScratch * 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBatStages; ++s) {
      tc::mbar_init(bar(FULLA + s), 1);
      tc::mbar_init(bar(FULLB + s), kBatDecWarps);
      tc::mbar_init(bar(EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(bar(TFULL + b), 1);
      tc::mbar_init(bar(TEMPTY + b), 4);
    }
    tc::mbar_init(bar(DRAIN), 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmQhi);
    tc::prefetch_tmap(&tmQlo);
  }
  for (int i = threadIdx.x; i < p.lut_size; i += blockDim.x) slut[i] = p.lut[i];
  if (warp == 1) tc::tmem_alloc(tc::smem_u32(tmem_holder), 512u);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  const int ntasks = p.qtiles * p.rchunks;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: query tiles ----------------
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntasks && ok; t += gridDim.x) {
        const int rc = t / p.qtiles, qt = t % p.qtiles;
        const int64_t r0 = (int64_t)rc * p.rows_per_chunk;
        const int64_t r1 = min(p.n, r0 + p.rows_per_chunk);
        const int tiles = (int)((r1 - r0 + kBatN - 1) / kBatN);
        for (int tile = 0; tile < tiles && ok; ++tile) {
          for (int kb = 0; kb < p.nk; ++kb, ++it) {
            const int s = it % kBatStages;
            const uint32_t ph = (uint32_t)(it / kBatStages) & 1u;
            if (!tc::mbar_wait(bar(EMPTY + s), ph ^ 1u, abort_flag, tc::kErrWaitStageEmpty)) {
              ok = false;
              break;
            }
            const uint32_t st = base + (uint32_t)s * STAGE;
            tc::mbar_arrive_expect_tx(bar(FULLA + s), 2 * QPLANE);
            tc::tma_load_2d(st, &tmQhi, kb * kBatBK, qt * kBatM, bar(FULLA + s));
            tc::tma_load_2d(st + QPLANE, &tmQlo, kb * kBatBK, qt * kBatM, bar(FULLA + s));
          }
        }
      }
      for (int j = it - kBatStages; j < it; ++j) {
        if (j < 0) continue;
        volatile int never = 0;
        tc::mbar_wait(bar(FULLA + j % kBatStages), (uint32_t)(j / kBatStages) & 1u, &never,
                      tc::kErrWaitTmaFull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = tc::idesc_f16_f32(kBatM, kBatN);
      int it = 0, tcount = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntasks && ok; t += gridDim.x) {
        const int rc = t / p.qtiles;
        const int64_t r0 = (int64_t)rc * p.rows_per_chunk;
        const int64_t r1 = min(p.n, r0 + p.rows_per_chunk);
        const int tiles = (int)((r1 - r0 + kBatN - 1) / kBatN);
        for (int tile = 0; tile < tiles && ok; ++tile, ++tcount) {
          const int buf = tcount & 1;
          const uint32_t tph = (uint32_t)(tcount >> 1) & 1u;
          if (!tc::mbar_wait(bar(TEMPTY + buf), tph ^ 1u, abort_flag, tc::kErrWaitAccEmpty)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)(buf * kBatN);
          for (int kb = 0; kb < p.nk; ++kb, ++it) {
            const int s = it % kBatStages;
            const uint32_t ph = (uint32_t)(it / kBatStages) & 1u;
            if (!tc::mbar_wait(bar(FULLA + s), ph, abort_flag, tc::kErrWaitTmaFull) ||
                !tc::mbar_wait(bar(FULLB + s), ph, abort_flag, tc::kErrWaitTmaFull)) {
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
              tc::mma_f16(d_tmem, tc::sw128_desc(q_hi + off), tc::sw128_desc(x_hi + off), idesc,
                          (kb | kk) != 0);
              tc::mma_f16(d_tmem, tc::sw128_desc(q_hi + off), tc::sw128_desc(x_lo + off), idesc, 1);
              tc::mma_f16(d_tmem, tc::sw128_desc(q_lo + off), tc::sw128_desc(x_hi + off), idesc, 1);
            }
            tc::mma_commit(bar(EMPTY + s));
          }
          if (ok) tc::mma_commit(bar(TFULL + buf));
        }
      }
      tc::mma_commit(bar(DRAIN));
      volatile int never = 0;
      tc::mbar_wait(bar(DRAIN), 0, &never, tc::kErrWaitAccFull);
    }
  } else if (warp >= 6) {
    // ---------------- decoder: corpus tiles ----------------
    // Each thread owns UPT row segments per stage.  The segments of the next
    // stage are loaded into registers before waiting for the current stage's
    // buffer, so HBM latency overlaps the MMAs of the stages in flight.
    using S = DecSeg<B>;
    const int dt = threadIdx.x - 6 * 32;
    BatWalk w;
    w.t = blockIdx.x;
    w.tile = 0;
    w.kb = 0;
    if (w.t < ntasks) walk_task(w, p);
    uint32_t cur[S::UPT][S::WORDS], nxt[S::UPT][S::WORDS];
    if (w.t < ntasks) dec_load<B>(p, w, dt, cur);
    for (int it = 0; w.t < ntasks; ++it) {
      const BatWalk here = w;
      walk_next(w, p, ntasks);
      if (w.t < ntasks) dec_load<B>(p, w, dt, nxt);
      const int s = it % kBatStages;
      const uint32_t ph = (uint32_t)(it / kBatStages) & 1u;
      if (!tc::mbar_wait(bar(EMPTY + s), ph ^ 1u, abort_flag, tc::kErrWaitStageEmpty)) break;
      uint8_t* xh = gbase + (size_t)s * STAGE + 2 * QPLANE;
      uint8_t* xl = xh + XPLANE;
      const int64_t tr0 = here.r0 + (int64_t)here.tile * kBatN;
#pragma unroll
      for (int i = 0; i < S::UPT; ++i) {
        const int u = dt + i * kBatDecWarps * 32;
        const int r = u / S::PER_ROW, sg = u % S::PER_ROW;
        const bool live = tr0 + r < here.r1;
#pragma unroll
        for (int cc = 0; cc < S::CODES / 8; ++cc) {
          uint4 vh = make_uint4(0, 0, 0, 0), vl = make_uint4(0, 0, 0, 0);
          if (live) {
            uint32_t e[8];
#pragma unroll
            for (int t2 = 0; t2 < 8; ++t2) e[t2] = slut[seg_code<B>(cur[i], cc * 8 + t2) >> p.shift];
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
      // Make the generic-proxy stores visible to the tensor core (async proxy).
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar(FULLB + s));
#pragma unroll
      for (int i = 0; i < S::UPT; ++i)
#pragma unroll
        for (int j = 0; j < S::WORDS; ++j) cur[i][j] = nxt[i][j];
    }
  } else {
    // ---------------- epilogue: warps 2..5, thread = query ----------------
    const int ew = warp - 2;
    const int q_lane = 32 * (warp & 3) + lane;
    float* ss = scratch_s + ew * kBatScratch;
    int* si = scratch_i + ew * kBatScratch;
    const float csc = p.cscale[0];
    int tcount = 0;
    for (int t = blockIdx.x; t < ntasks; t += gridDim.x) {
      const int rc = t / p.qtiles, qt = t % p.qtiles;
      const int64_t r0 = (int64_t)rc * p.rows_per_chunk;
      const int64_t r1 = min(p.n, r0 + p.rows_per_chunk);
      const int tiles = (int)((r1 - r0 + kBatN - 1) / kBatN);
      const int qg = qt * kBatM + q_lane;
      const bool qv = qg < p.nq;
      const float qs = qv ? p.qinv[qg] * csc : 0.f;
      float* bs = p.buf_s + ((size_t)blockIdx.x * kBatM + q_lane) * p.cap;
      int* bi = p.buf_i + ((size_t)blockIdx.x * kBatM + q_lane) * p.cap;
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
        const int64_t tr0 = r0 + (int64_t)tile * kBatN;
        const uint32_t taddr = tmem_base + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(buf * kBatN);
        for (int c0 = 0; c0 < kBatN; c0 += 32) {
          uint32_t v[32];
          __syncwarp();
          tc::tmem_ld16(taddr + (uint32_t)c0, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
          tc::tmem_ld16(taddr + (uint32_t)c0 + 16u, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
          tc::tmem_ld_wait(v);
          uint32_t need = __ballot_sync(0xffffffffu, qv && cnt + 32 > p.cap);
          while (need) {
            const int src = __ffs(need) - 1;
            need &= need - 1;
            float* sbs = p.buf_s + ((size_t)blockIdx.x * kBatM + 32 * (warp & 3) + src) * p.cap;
            int* sbi = p.buf_i + ((size_t)blockIdx.x * kBatM + 32 * (warp & 3) + src) * p.cap;
            warp_select(src, lane, cnt, sbs, sbi, p.K, cnt, thr);
          }
          const int64_t rb = tr0 + c0;
          if (qv && rb < r1) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int64_t row = rb + i;
              if (row < r1) {
                const float sc = __uint_as_float(v[i]) * qs * __ldg(p.norms + row);
                if (sc > thr) {
                  bs[cnt] = sc;
                  bi[cnt] = (int)row;
                  ++cnt;
                }
              }
            }
          }
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(bar(TEMPTY + buf));
      }
      if (!ok) break;
      // Task end: final top-K of every query of the tile.
      __syncwarp();
      uint32_t pend = __ballot_sync(0xffffffffu, qv);
      while (pend) {
        const int src = __ffs(pend) - 1;
        pend &= pend - 1;
        const int sq = qt * kBatM + 32 * (warp & 3) + src;
        float* sbs = p.buf_s + ((size_t)blockIdx.x * kBatM + 32 * (warp & 3) + src) * p.cap;
        int* sbi = p.buf_i + ((size_t)blockIdx.x * kBatM + 32 * (warp & 3) + src) * p.cap;
        const size_t o = ((size_t)sq * p.rchunks + rc) * p.K;
        warp_compact(src, lane, cnt, sbs, sbi, p.K, ss, si, cnt, thr, p.out_s + o, p.out_id + o,
                     p.row_offset);
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, 512u);
  }
}

// Centroid table for the decoder: cent[c] * 2^ec split into fp16 hi/lo,
// with ec chosen so the largest |centroid| lands in [2^14, 2^15).
__global__ void batch_lut_kernel(const float* __restrict__ cent, int size, uint32_t* __restrict__ lut,
                                 float* __restrict__ cscale) {
  __shared__ float mx;
  if (threadIdx.x == 0) {
    float m = 0.f;
    for (int i = 0; i < size; ++i) m = fmaxf(m, fabsf(cent[i]));
    mx = m;
  }
  __syncthreads();
  int ec = 0;
  if (mx > 0.f) ec = max(-100, min(100, 14 - ilogbf(mx)));
  const float sc = __int_as_float((127 + ec) << 23);
  for (int i = threadIdx.x; i < size; i += blockDim.x) {
    const float v = cent[i] * sc;
    const __half h = __float2half_rn(v);
    const __half l = __float2half_rn(v - __half2float(h));
    lut[i] = (uint32_t)__half_as_ushort(h) | ((uint32_t)__half_as_ushort(l) << 16);
  }
  if (threadIdx.x == 0) cscale[0] = __int_as_float((127 + 14 - ec) << 23);
}

struct BatPlan {
  int ldk, nk, nq_pad, qtiles, rchunks, grid, cap;
  int64_t rpc;
  size_t smem;
};

static BatPlan bat_plan(int64_t n, int d, int nq, int k) {
  BatPlan b;
  b.ldk = (d + kBatBK - 1) / kBatBK * kBatBK;
  b.nk = b.ldk / kBatBK;
  b.qtiles = (nq + kBatM - 1) / kBatM;
  b.nq_pad = b.qtiles * kBatM;
  // Row chunks per query tile: the smallest count whose task total fills the
  // SMs in whole waves (>= 97% of the last wave busy), so no SM idles at the
  // end; tasks stay >= 4 row tiles long.
  const int sms = num_sms();
  const int64_t min_rows = 4 * kBatN;
  const int64_t max_rc = (n + min_rows - 1) / min_rows < 1 ? 1 : (n + min_rows - 1) / min_rows;
  int rc = 1;
  double best = -1.0;
  const int lo = (sms + b.qtiles - 1) / b.qtiles;
  for (int c = lo < 1 ? 1 : lo; c <= 16 * lo + 16 && c <= max_rc; ++c) {
    const int64_t tasks = (int64_t)c * b.qtiles;
    const double eff = (double)tasks / (double)(((tasks + sms - 1) / sms) * sms);
    if (eff > best + 1e-9) {
      best = eff;
      rc = c;
    }
    if (eff >= 0.97) break;
  }
  if (best < 0) rc = (int)(max_rc < lo ? max_rc : lo);
  b.rpc = ((n + rc - 1) / rc + kBatN - 1) / kBatN * kBatN;
  if (b.rpc < kBatN) b.rpc = kBatN;
  b.rchunks = (int)((n + b.rpc - 1) / b.rpc);
  if (b.rchunks < 1) b.rchunks = 1;
  const int tasks = b.qtiles * b.rchunks;
  b.grid = tasks < num_sms() ? tasks : num_sms();
  b.cap = 2 * k;
  if (b.cap < 64) b.cap = 64;
  b.smem = 1024 + (size_t)kBatStages * (2 * kBatM * 128 + 2 * kBatN * 128) + 8 * 32 + 16 + 1024 +
           (size_t)4 * kBatScratch * 8 + 256;
  return b;
}

struct BatWs {
  __half *qhi, *qlo;
  float *qinv, *qrot_unused, *cscale, *buf_s, *out_s;
  int* buf_i;
  uint32_t* lut;
  long long* out_id;
  unsigned int* gthr;  // per-query shared threshold keys (pair kernel)
};

static size_t bat_ws_carve(const BatPlan& b, int nq, int K, void* ws, size_t ws_bytes, BatWs* w) {
  Carve cv(ws, ws_bytes);
  w->qhi = cv.take<__half>((size_t)b.nq_pad * b.ldk);
  w->qlo = cv.take<__half>((size_t)b.nq_pad * b.ldk);
  w->qinv = cv.take<float>((size_t)b.nq_pad);
  w->cscale = cv.take<float>(4);
  w->lut = cv.take<uint32_t>(256);
  w->buf_s = cv.take<float>((size_t)b.grid * kBatM * b.cap);
  w->buf_i = cv.take<int>((size_t)b.grid * kBatM * b.cap);
  w->out_s = cv.take<float>((size_t)nq * b.rchunks * K);
  w->out_id = cv.take<long long>((size_t)nq * b.rchunks * K);
  return cv.off + 256;
}

}  // namespace pqb

using namespace pqb;

// Runs the one-CTA batched kernel; leaves per-(query, row chunk) top-K lists
// in ws (layout [nq][rchunks][K]) and returns their location.
static int run_batched_1cta(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                       int bits, int precision, const float* qrot, int nq, const float* cent, int K,
                       int64_t row_offset, void* ws, size_t ws_bytes, cudaStream_t st,
                       float** parts_s, long long** parts_id, int* nparts) {
  const BatPlan b = bat_plan(n, d, nq, K);
  BatWs w;
  const size_t need = bat_ws_carve(b, nq, K, ws, (size_t)-1 / 2, &w);
  if (ws_bytes < need) return fail(PQ_ERR_WORKSPACE, "batched ADC needs %zu workspace bytes", need);
  bat_ws_carve(b, nq, K, ws, ws_bytes, &w);
  // Query planes (hi/lo fp16 with per-query scale), zero rows up to nq_pad.
  PQ_CUDA_TRY(cudaMemsetAsync(w.qhi, 0, (size_t)b.nq_pad * b.ldk * 2, st));
  PQ_CUDA_TRY(cudaMemsetAsync(w.qlo, 0, (size_t)b.nq_pad * b.ldk * 2, st));
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
  if ((rc = make_map(&mhi, w.qhi, b.nq_pad, b.ldk, kBatM))) return rc;
  if ((rc = make_map(&mlo, w.qlo, b.nq_pad, b.ldk, kBatM))) return rc;
  BatArgs a;
  a.packed = packed; a.ldb = ldb; a.norms = norms; a.n = n; a.d = d; a.nk = b.nk;
  a.shift = bits - precision; a.nq = nq; a.qtiles = b.qtiles; a.rchunks = b.rchunks;
  a.rows_per_chunk = b.rpc; a.K = K; a.cap = b.cap; a.qinv = w.qinv; a.cscale = w.cscale;
  a.lut = w.lut; a.lut_size = lut_size; a.buf_s = w.buf_s; a.buf_i = w.buf_i;
  a.out_s = w.out_s; a.out_id = w.out_id; a.row_offset = row_offset; a.gthr = nullptr; a.qdig = nullptr;
  a.out_parts = b.rchunks; a.part_base = 0;
  if (b.smem > 227 * 1024) return fail(PQ_ERR_UNSUPPORTED, "batched smem %zu too large", b.smem);
  switch (bits) {
#define PQ_BAT_CASE(BB)                                                                         \
  case BB: {                                                                                    \
    auto kern = batched_adc_kernel<BB>;                                                         \
    PQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,        \
                                     (int)b.smem));                                             \
    kern<<<b.grid, kBatThreads, b.smem, st>>>(mhi, mlo, a);                                     \
  } break;
    PQ_BAT_CASE(1)
    PQ_BAT_CASE(2)
    PQ_BAT_CASE(3)
    PQ_BAT_CASE(4)
    PQ_BAT_CASE(8)
#undef PQ_BAT_CASE
    default:
      return fail(PQ_ERR_INVALID, "bits must be one of 1,2,3,4,8 (got %d)", bits);
  }
  PQ_LAUNCH_CHECK("batched_adc_kernel");
  *parts_s = w.out_s;
  *parts_id = w.out_id;
  *nparts = b.rchunks;
  return PQ_OK;
}

static size_t batched_ws_1cta(int64_t n, int d, int nq, int k) {
  if (n <= 0 || nq <= 0 || k <= 0 || d <= 0) return 256;
  const BatPlan b = bat_plan(n, d, nq, k);
  BatWs w;
  return bat_ws_carve(b, nq, k, nullptr, 0, &w);
}

extern "C" {

size_t pq_adc_batch_workspace_bytes(int64_t n, int d, int nq, int k) {
  return batched_ws(n, d, nq, k);
}

int pq_adc_batch(const uint8_t* packed, int64_t ldb, const float* norms, int64_t n, int d,
                 int bits, int precision, const float* qrot, int nq, const float* cent, int k,
                 int64_t row_offset, float* out_scores, int64_t* out_ids, void* ws,
                 size_t ws_bytes, void* stream) {
  int rc = check_corpus(packed, ldb, norms, n, d, bits);
  if (rc) return rc;
  PQ_CHECK_ARG(precision >= 1 && precision <= bits, "precision must be 1-%d, got %d", bits,
               precision);
  PQ_CHECK_ARG(k >= 1 && k <= kBatMaxK && k <= n, "k must be in [1, min(n, %d)] (got %d)",
               kBatMaxK, k);
  PQ_CHECK_ARG(n < (1ll << 31), "n=%lld rows exceed one launch; shard the corpus", (long long)n);
  if (nq == 0) return PQ_OK;
  PQ_CHECK_ARG(qrot && cent && out_scores && out_ids && ws, "null pointer argument");
  cudaStream_t st = (cudaStream_t)stream;
  float* ps;
  long long* pi;
  int parts, kpart = k;
  rc = run_batched(packed, ldb, norms, n, d, bits, precision, qrot, nq, cent, k, 0, ws, ws_bytes,
                   st, &ps, &pi, &parts, &kpart);
  if (rc) return rc;
  if (kpart != k)
    return rescore_candidates(packed, ldb, norms, n, d, bits, precision, qrot, nq, cent, ps, pi,
                              parts, kpart, k, row_offset, out_scores, (long long*)out_ids, st);
  // The batched kernels write each list sorted best first (warp_compact).
  return launch_merge_sorted(ps, pi, parts, k, (long long)parts * k, k, nq, k, row_offset,
                             out_scores, (long long*)out_ids, st);
}

}  // extern "C"
