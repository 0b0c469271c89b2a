// Encode: norm -> normalise -> rotate (X_unit @ R^T) -> Lloyd-Max code ->
// bit-pack (remex/core.py:484-511, remex/packing.py:18-75).
//
// Two kernels per row chunk:
//  1. encode_prep_kernel (HBM-bound): per row, the f64 sum of squares and the
//     f32 norm exactly as remex/core.py:504-505, x_unit = x / max(norm, 1e-8)
//     with IEEE f32 division (core.py:506), then a per-row power-of-two scale
//     2^e (max |x_unit| * 2^e in [2^14, 2^15)) and a split of x_unit*2^e into
//     fp16 hi + fp16 lo planes.
//  2. encode_gemm_kernel (tensor-bound): a persistent warp-specialised
//     tcgen05 GEMM.  TMA streams 128x64 tiles of the A planes and BNx64 tiles
//     of the R planes (R*2^14, split the same way) into 128B-swizzled shared
//     memory; one thread issues three kind::f16 MMAs per 16-wide K step,
//     A_hi*R_hi + A_hi*R_lo + A_lo*R_hi, accumulating in f32 in TMEM (two
//     accumulator buffers so the epilogue of one tile overlaps the MMAs of the
//     next); four epilogue warps read the accumulators with tcgen05.ld, scale
//     by 2^-(e+14) (exact), count the boundaries below each value
//     (np.searchsorted side='left', core.py:509) and write packed rows.
//     Values within 1e-6 of a boundary are recomputed by the warp in f64
//     before packing, because the tensor core's f32 accumulation rounds
//     toward zero and would otherwise move ~1e-4 of 8-bit codes across a
//     boundary.
// The split carries 22 significant bits of each operand, so the rotated
// coordinates agree with an exact product to ~1e-7 relative and code flips
// against the reference's f32 sgemm stay at the reference's own rounding
// floor (flips only occur within ~1e-7 of a boundary).
#include <cudaTypedefs.h>

#include <mutex>

#include "tc.cuh"

namespace pqb {

constexpr int kEncBM = 128;     // rows per tile (TMEM lanes)
constexpr int kEncBK = 64;      // K per stage: one 128-byte swizzle atom of fp16
constexpr int kEncThreads = 320;  // warp 0 TMA, warp 1 MMA + TMEM, warps 2-9 epilogue
constexpr int kScaleBias = 14;  // R planes hold R * 2^14
constexpr int kGuideCells = 2048;  // uniform cells of the 8-bit guide table
constexpr int kFixPerRow = 16;     // near-boundary columns listed per row for the fix-up
// Shared memory after the stages: barriers, TMEM address, abort flag, the
// boundaries (255 f32) and the 8-bit guide table (kGuideCells + 1 bytes).
constexpr size_t kEncMetaBytes = 4096;

struct EncShape {
  int d, ntn, BN, ldn, ldk, nk, stages, tmem_cols;
  size_t stage_bytes, smem_bytes;
};

static EncShape enc_shape(int d) {
  EncShape s;
  s.d = d;
  s.ntn = (d + 255) / 256;
  // A multiple of 32: the epilogue packs 32 codes at a time, and a chunk
  // must not run into the next column tile's bytes.
  s.BN = ((d + s.ntn - 1) / s.ntn + 31) / 32 * 32;
  s.ldn = s.ntn * s.BN;
  s.ldk = (d + kEncBK - 1) / kEncBK * kEncBK;
  s.nk = s.ldk / kEncBK;
  s.stage_bytes = (size_t)2 * kEncBM * 128 + (size_t)2 * s.BN * 128;
  s.stages = (s.BN > 128) ? 2 : 3;
  s.tmem_cols = 32;
  while (s.tmem_cols < 2 * s.BN) s.tmem_cols <<= 1;
  s.smem_bytes = 1024 + (size_t)s.stages * s.stage_bytes + kEncMetaBytes;
  return s;
}

// ---------------------------------------------------------------------------
// 1. Normalise + split
// ---------------------------------------------------------------------------

__device__ __forceinline__ float pow2f(int e) { return __int_as_float((127 + e) << 23); }

template <bool NORMALIZE>
__global__ void __launch_bounds__(256)
encode_prep_kernel(const float* __restrict__ X, int64_t m, int d, int ldk, __half* __restrict__ Ahi,
                   __half* __restrict__ Alo, float* __restrict__ inv_scale,
                   float* __restrict__ norms_out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < m;
       r += warps) {
    const float* x = X + r * d;
    double ss = 0.0;
    float mx = 0.f;
    for (int j = lane; j < d; j += 32) {
      const float v = __ldg(x + j);
      ss = fma((double)v, (double)v, ss);
      mx = fmaxf(mx, fabsf(v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ss += __shfl_xor_sync(0xffffffffu, ss, o);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const float nrm = __double2float_rn(__dsqrt_rn(ss));
    const float den = fmaxf(nrm, 1e-8f);
    if (NORMALIZE) mx = __fdiv_rn(mx, den);
    int e = 0;
    if (mx > 0.f) {
      e = kScaleBias - ilogbf(mx);
      e = max(-100, min(100, e));
    }
    const float sc = pow2f(e);
    __half2* hp = reinterpret_cast<__half2*>(Ahi + r * ldk);
    __half2* lp = reinterpret_cast<__half2*>(Alo + r * ldk);
    for (int j = 2 * lane; j < ldk; j += 64) {
      float v0 = (j < d) ? __ldg(x + j) : 0.f;
      float v1 = (j + 1 < d) ? __ldg(x + j + 1) : 0.f;
      if (NORMALIZE) {
        v0 = __fdiv_rn(v0, den);
        v1 = __fdiv_rn(v1, den);
      }
      v0 *= sc;
      v1 *= sc;
      const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
      const __half l0 = __float2half_rn(v0 - __half2float(h0));
      const __half l1 = __float2half_rn(v1 - __half2float(h1));
      hp[j >> 1] = __halves2half2(h0, h1);
      lp[j >> 1] = __halves2half2(l0, l1);
    }
    if (lane == 0) {
      inv_scale[r] = pow2f(-e - kScaleBias);
      if (norms_out) norms_out[r] = nrm;
    }
  }
}

// The same, one warp per row with the whole row held in registers: T float4
// per lane (T = ldk / 128 rounded up, ldk <= 2048), all loads issued before
// the first use, so a few warps per SM keep enough bytes in flight to stream
// at HBM rate while the encode GEMM of the previous chunk occupies the SMs.
// Requires d % 4 == 0 and 16-byte aligned rows.  The f64 sum of squares runs
// in another order than encode_prep_kernel's; both round to the same f32 norm
// except in the rare case that an f64 sum lands within an ulp of an f32
// rounding boundary (the tests check norms bit for bit).
template <bool NORMALIZE, int T>
__global__ void __launch_bounds__(128)
encode_prep4_kernel(const float* __restrict__ X, int64_t m, int d, int ldk,
                    __half* __restrict__ Ahi, __half* __restrict__ Alo,
                    float* __restrict__ inv_scale, float* __restrict__ norms_out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int nv = d >> 2, nk = ldk >> 2;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < m;
       r += warps) {
    const float4* x4 = reinterpret_cast<const float4*>(X + r * d);
    float4 v[T];
#pragma unroll
    for (int t = 0; t < T; ++t) {
      const int i = lane + 32 * t;
      v[t] = i < nv ? __ldg(x4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    double ss = 0.0;
    float mx = 0.f;
#pragma unroll
    for (int t = 0; t < T; ++t) {
      ss = fma((double)v[t].x, (double)v[t].x, ss);
      ss = fma((double)v[t].y, (double)v[t].y, ss);
      ss = fma((double)v[t].z, (double)v[t].z, ss);
      ss = fma((double)v[t].w, (double)v[t].w, ss);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[t].x), fabsf(v[t].y)), fmaxf(fabsf(v[t].z), fabsf(v[t].w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ss += __shfl_xor_sync(0xffffffffu, ss, o);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const float nrm = __double2float_rn(__dsqrt_rn(ss));
    const float den = fmaxf(nrm, 1e-8f);
    if (NORMALIZE) mx = __fdiv_rn(mx, den);
    int e = 0;
    if (mx > 0.f) {
      e = kScaleBias - ilogbf(mx);
      e = max(-100, min(100, e));
    }
    const float sc = pow2f(e);
    uint2* hp = reinterpret_cast<uint2*>(Ahi + r * ldk);
    uint2* lp = reinterpret_cast<uint2*>(Alo + r * ldk);
#pragma unroll
    for (int t = 0; t < T; ++t) {
      const int i = lane + 32 * t;
      if (i < nk) {
        float a[4] = {v[t].x, v[t].y, v[t].z, v[t].w};
        __half h[4], l[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float x = a[u];
          if (NORMALIZE) x = __fdiv_rn(x, den);
          x *= sc;
          h[u] = __float2half_rn(x);
          l[u] = __float2half_rn(x - __half2float(h[u]));
        }
        const __half2 h01 = __halves2half2(h[0], h[1]), h23 = __halves2half2(h[2], h[3]);
        const __half2 l01 = __halves2half2(l[0], l[1]), l23 = __halves2half2(l[2], l[3]);
        hp[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&h01),
                           *reinterpret_cast<const uint32_t*>(&h23));
        lp[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&l01),
                           *reinterpret_cast<const uint32_t*>(&l23));
      }
    }
    if (lane == 0) {
      inv_scale[r] = pow2f(-e - kScaleBias);
      if (norms_out) norms_out[r] = nrm;
    }
  }
}

// R (d x d f32) -> R*2^14 split into fp16 hi/lo planes of ldn x ldk, zero padded.
__global__ void rot_planes_kernel(const float* __restrict__ R, int d, int ldn, int ldk,
                                  __half* __restrict__ Rhi, __half* __restrict__ Rlo) {
  const int64_t total = (int64_t)ldn * ldk;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(t / ldk), k = (int)(t % ldk);
    const float v = (i < d && k < d) ? R[(int64_t)i * d + k] * pow2f(kScaleBias) : 0.f;
    const __half h = __float2half_rn(v);
    Rhi[t] = h;
    Rlo[t] = __float2half_rn(v - __half2float(h));
  }
}

// ---------------------------------------------------------------------------
// 2. tcgen05 GEMM + quantise/pack epilogue
// ---------------------------------------------------------------------------

// Number of boundaries strictly below x (np.searchsorted side='left'); NaN
// sorts last as in NumPy.
template <int BITS>
__device__ __forceinline__ uint32_t code_of(float x, const float* sb) {
  uint32_t idx = 0;
#pragma unroll
  for (int step = 1 << (BITS - 1); step > 0; step >>= 1)
    if (x > sb[idx + step - 1]) idx += step;
  if (isnan(x)) idx = (1u << BITS) - 1u;
  return idx;
}

// 8-bit codes: a guide table over kGuideCells uniform cells between the first
// and last boundary gives each value a starting level -- the number of
// boundaries below its cell's left edge.  Cells are narrower than the
// smallest gap between boundaries, so a cell holds at most one and a single
// step up (x > sb[c]) lands on #{boundaries < x} (searchsorted side='left').
// The epilogue then checks the boundaries on both sides (which also gives
// the near-boundary test) and sends any value that fails -- float rounding
// of the cell index, NaN -- to the binary search.
struct Guide {
  float lo, scale;  // cell of x = (x - lo) * scale
};

__device__ __forceinline__ uint32_t guide_start(float x, const uint8_t* guide, Guide g) {
  float t = (x - g.lo) * g.scale;
  t = fminf(fmaxf(t, 0.f), (float)(kGuideCells - 1));
  return guide[(int)t];
}

// Builds the guide table: guide[i] = #{boundaries < lo + i / scale}.
__device__ __forceinline__ Guide build_guide(const float* sb, uint8_t* guide) {
  Guide g;
  g.lo = sb[0];
  g.scale = (float)kGuideCells / (sb[254] - sb[0]);
  for (int i = threadIdx.x; i <= kGuideCells; i += blockDim.x) {
    const float e = g.lo + (float)i / g.scale;
    uint32_t idx = 0;
#pragma unroll
    for (int step = 128; step > 0; step >>= 1)
      if (e > sb[idx + step - 1]) idx += step;
    guide[i] = (uint8_t)idx;
  }
  return g;
}

// Half-width of the band around each boundary inside which a coordinate is
// recomputed exactly (rotated-coordinate units; the GEMM's own error is
// ~1e-8, the reference's f32 sgemm error similar).
constexpr float kFixBand = 1e-6f;

template <int BITS>
__device__ __forceinline__ bool near_boundary(float x, uint32_t c, const float* sb) {
  const float lo = (c > 0) ? sb[c - 1] : -INFINITY;
  const float hi = (c < (1u << BITS) - 1u) ? sb[c] : INFINITY;
  return (x - lo < kFixBand) || (hi - x < kFixBand);
}

// Packs 32 codes (MSB-first stream) into 4*BITS bytes held as BITS words.
template <int BITS>
__device__ __forceinline__ void pack32(const uint32_t (&c)[32], uint32_t (&w)[8]) {
  uint8_t b[32];
  if constexpr (BITS == 8) {
#pragma unroll
    for (int t = 0; t < 32; ++t) b[t] = (uint8_t)c[t];
  } else if constexpr (BITS == 4) {
#pragma unroll
    for (int t = 0; t < 16; ++t) b[t] = (uint8_t)((c[2 * t] << 4) | c[2 * t + 1]);
  } else if constexpr (BITS == 2) {
#pragma unroll
    for (int t = 0; t < 8; ++t)
      b[t] = (uint8_t)((c[4 * t] << 6) | (c[4 * t + 1] << 4) | (c[4 * t + 2] << 2) | c[4 * t + 3]);
  } else if constexpr (BITS == 1) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      uint32_t v = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) v |= c[8 * t + i] << (7 - i);
      b[t] = (uint8_t)v;
    }
  } else {  // 3 bits: 8 codes -> 24-bit big-endian group
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      uint32_t v = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) v |= c[8 * g + i] << (21 - 3 * i);
      b[3 * g] = (uint8_t)(v >> 16);
      b[3 * g + 1] = (uint8_t)(v >> 8);
      b[3 * g + 2] = (uint8_t)v;
    }
  }
#pragma unroll
  for (int i = 0; i < BITS; ++i)
    w[i] = (uint32_t)b[4 * i] | ((uint32_t)b[4 * i + 1] << 8) | ((uint32_t)b[4 * i + 2] << 16) |
           ((uint32_t)b[4 * i + 3] << 24);
}

// BITS = 0: write the rotated f32 values (Y = X @ R^T) instead of codes.
template <int BITS>
__global__ void __launch_bounds__(kEncThreads, 1)
encode_gemm_kernel(const __grid_constant__ CUtensorMap tmAhi, const __grid_constant__ CUtensorMap tmAlo,
                   const __grid_constant__ CUtensorMap tmBhi, const __grid_constant__ CUtensorMap tmBlo,
                   int m, int d, int BN, int ntn, int nk, int stages, int tmem_cols,
                   const float* __restrict__ inv_scale, const float* __restrict__ bounds,
                   uint8_t* __restrict__ packed, int64_t ldb, int64_t rb, float* __restrict__ Y,
                   const __half* __restrict__ Ahi, const __half* __restrict__ Alo, int ldk,
                   const float* __restrict__ R, int* __restrict__ fix_cnt,
                   uint16_t* __restrict__ fix_cols) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t raw = tc::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t stage_bytes = 2u * kEncBM * 128u + 2u * (uint32_t)BN * 128u;
  const uint32_t meta = base + (uint32_t)stages * stage_bytes;
  uint8_t* gmeta = gbase + (size_t)stages * stage_bytes;
  // meta layout: full[S] empty[S] tfull[2] tempty[2] drain (8 B each), tmem addr, abort, bounds
  auto bar = [&](int i) { return meta + 8u * (uint32_t)i; };
  const int FULL = 0, EMPTY = stages, TFULL = 2 * stages, TEMPTY = 2 * stages + 2,
            DRAIN = 2 * stages + 4;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(gmeta + 8 * (2 * stages + 5));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gmeta + 8 * (2 * stages + 5) + 4);
  float* sb = reinterpret_cast<float*>(gmeta + 8 * (2 * stages + 5) + 8);
  uint8_t* guide = gmeta + 8 * (2 * stages + 5) + 8 + 1024;  // 8-bit codes only

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      tc::mbar_init(bar(FULL + s), 1);
      tc::mbar_init(bar(EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(bar(TFULL + b), 1);
      tc::mbar_init(bar(TEMPTY + b), 8);
    }
    tc::mbar_init(bar(DRAIN), 1);
    *abort_flag = 0;
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmAhi);
    tc::prefetch_tmap(&tmAlo);
    tc::prefetch_tmap(&tmBhi);
    tc::prefetch_tmap(&tmBlo);
  }
  if (BITS > 0)
    for (int i = threadIdx.x; i < (1 << BITS) - 1; i += blockDim.x) sb[i] = bounds[i];
  if (warp == 1) tc::tmem_alloc(tc::smem_u32(tmem_holder), (uint32_t)tmem_cols);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  Guide gd{0.f, 0.f};
  if constexpr (BITS == 8) {
    gd = build_guide(sb, guide);
    __syncthreads();
  }

  const int mt = (m + kEncBM - 1) / kEncBM;
  const int ntiles = mt * ntn;
  const uint32_t tx_bytes = stage_bytes;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int mb = tile / ntn, nb = tile % ntn;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % stages;
          const uint32_t ph = (uint32_t)(it / stages) & 1u;
          if (!tc::mbar_wait(bar(EMPTY + s), ph ^ 1u, abort_flag, tc::kErrWaitStageEmpty)) {
            ok = false;
            break;
          }
          const uint32_t st = base + (uint32_t)s * stage_bytes;
          tc::mbar_arrive_expect_tx(bar(FULL + s), tx_bytes);
          tc::tma_load_2d(st, &tmAhi, kb * kEncBK, mb * kEncBM, bar(FULL + s));
          tc::tma_load_2d(st + kEncBM * 128, &tmAlo, kb * kEncBK, mb * kEncBM, bar(FULL + s));
          tc::tma_load_2d(st + 2 * kEncBM * 128, &tmBhi, kb * kEncBK, nb * BN, bar(FULL + s));
          tc::tma_load_2d(st + 2 * kEncBM * 128 + BN * 128, &tmBlo, kb * kEncBK, nb * BN,
                          bar(FULL + s));
        }
      }
      // Before the CTA can exit, every issued copy must have landed.
      for (int j = it - stages; j < it; ++j) {
        if (j < 0) continue;
        const int s = j % stages;
        const uint32_t ph = (uint32_t)(j / stages) & 1u;
        volatile int never = 0;
        tc::mbar_wait(bar(FULL + s), ph, &never, tc::kErrWaitTmaFull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = tc::idesc_f16_f32(kEncBM, BN);
      int it = 0, tcount = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++tcount) {
        const int buf = tcount & 1;
        const uint32_t tph = (uint32_t)(tcount >> 1) & 1u;
        if (!tc::mbar_wait(bar(TEMPTY + buf), tph ^ 1u, abort_flag, tc::kErrWaitAccEmpty)) break;
        tc::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % stages;
          const uint32_t ph = (uint32_t)(it / stages) & 1u;
          if (!tc::mbar_wait(bar(FULL + s), ph, abort_flag, tc::kErrWaitTmaFull)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t st = base + (uint32_t)s * stage_bytes;
          const uint32_t a_hi = st, a_lo = st + kEncBM * 128;
          const uint32_t b_hi = st + 2 * kEncBM * 128, b_lo = b_hi + (uint32_t)BN * 128;
#pragma unroll
          for (int kk = 0; kk < kEncBK / 16; ++kk) {
            const uint32_t off = (uint32_t)kk * 32u;
            tc::mma_f16(d_tmem, tc::sw128_desc(a_hi + off), tc::sw128_desc(b_hi + off), idesc,
                        (kb | kk) != 0);
            tc::mma_f16(d_tmem, tc::sw128_desc(a_hi + off), tc::sw128_desc(b_lo + off), idesc, 1);
            tc::mma_f16(d_tmem, tc::sw128_desc(a_lo + off), tc::sw128_desc(b_hi + off), idesc, 1);
          }
          tc::mma_commit(bar(EMPTY + s));
        }
        if (ok) tc::mma_commit(bar(TFULL + buf));
      }
      // Drain: wait until every MMA this thread issued has completed.
      tc::mma_commit(bar(DRAIN));
      volatile int never = 0;
      tc::mbar_wait(bar(DRAIN), 0, &never, tc::kErrWaitAccFull);
    }
  } else {
    // ---------------- epilogue (warps 2..9) ----------------
    // Warps w and w + 4 read the same TMEM lanes (rows), w the first half of
    // the tile's BN columns and w + 4 the second.  Thread = row.
    const int q = warp & 3, half = (warp - 2) >> 2;
    const int nch = BN / 32, nch0 = (nch + 1) / 2;  // 32-column chunks, first half's share
    const int cbeg = half ? 32 * nch0 : 0, cend = half ? BN : 32 * nch0;
    int tcount = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++tcount) {
      const int mb = tile / ntn, nb = tile % ntn;
      const int buf = tcount & 1;
      const uint32_t tph = (uint32_t)(tcount >> 1) & 1u;
      if (!tc::mbar_wait(bar(TFULL + buf), tph, abort_flag, tc::kErrWaitAccFull)) break;
      tc::tc_fence_after();
      const int row = mb * kEncBM + 32 * q + lane;
      const bool rv = row < m;
      const float inv = rv ? __ldg(inv_scale + row) : 0.f;
      const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * BN);
      for (int c0 = cbeg; c0 < cend; c0 += 32) {
        uint32_t v[32];
        __syncwarp();
        tc::tmem_ld16(taddr + (uint32_t)c0, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
        tc::tmem_ld16(taddr + (uint32_t)c0 + 16u, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
        tc::tmem_ld_wait(v);
        const int col0 = nb * BN + c0;
        if (col0 >= d) continue;  // warp-uniform
        if constexpr (BITS == 0) {
          if (rv) {
            float* yr = Y + (int64_t)row * d;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i < d) yr[col0 + i] = __uint_as_float(v[i]) * inv;
          }
        } else {
          // np.searchsorted(boundaries, x, side='left') for the 32 values:
          // 8-bit codes through the guide table, narrower ones by a binary
          // search, step-major so the 32 table lookups of a step are
          // independent.
          float x[32];
          uint32_t c[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            x[i] = __uint_as_float(v[i]) * inv;
            c[i] = 0;
          }
          uint32_t near8 = 0, bad8 = 0;
          if constexpr (BITS == 8) {
            // Step-major: each round's 32 lookups are independent.
#pragma unroll
            for (int i = 0; i < 32; ++i) c[i] = guide_start(x[i], guide, gd);
#pragma unroll
            for (int i = 0; i < 32; ++i) c[i] += (c[i] < 255u && x[i] > sb[c[i]]) ? 1u : 0u;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float lo = c[i] > 0u ? sb[c[i] - 1u] : -INFINITY;
              const float hi = c[i] < 255u ? sb[c[i]] : INFINITY;
              if (!(x[i] > lo) || x[i] > hi) bad8 |= 1u << i;
              if (x[i] - lo < kFixBand || hi - x[i] < kFixBand) near8 |= 1u << i;
            }
            if (__any_sync(0xffffffffu, bad8 != 0u)) {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if ((bad8 >> i) & 1u) c[i] = code_of<8>(x[i], sb);
            }
          } else {
#pragma unroll
            for (int step = 1 << (BITS - 1); step > 0; step >>= 1) {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (x[i] > sb[c[i] + step - 1]) c[i] += step;
            }
          }
          uint32_t near = 0;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (isnan(x[i])) c[i] = (1u << BITS) - 1u;  // NaN sorts last, as in NumPy
            const bool valid = rv && col0 + i < d;
            if (!valid) {
              c[i] = 0;
            } else if (BITS == 8 && !((bad8 >> i) & 1u)) {
              if ((near8 >> i) & 1u) near |= 1u << i;
            } else if (near_boundary<BITS>(x[i], c[i], sb)) {
              near |= 1u << i;
            }
          }
          // Coordinates within kFixBand of a boundary are recomputed in f64
          // from the exact f32 R and the 22-bit x planes, so the side of the
          // boundary does not depend on the tensor core's f32 accumulation
          // order.  They go to the row's fix-up list (encode_fix_kernel
          // recomputes all listed coordinates after this kernel, a warp per
          // row, and patches the packed codes); only coordinates past the
          // list's kFixPerRow slots are recomputed here.
          if (near && fix_cnt) {
            const int cnt = __popc(near);
            const int base = atomicAdd(fix_cnt + row, cnt);
            uint32_t msk = near;
            for (int k = base; msk && k < kFixPerRow; ++k) {
              const int i = __ffs(msk) - 1;
              msk &= msk - 1;
              fix_cols[(size_t)row * kFixPerRow + k] = (uint16_t)(col0 + i);
            }
            near = msk;
          }
          uint32_t pend = __ballot_sync(0xffffffffu, near != 0);
          while (pend) {
            const int src = __ffs(pend) - 1;
            pend &= pend - 1;
            uint32_t msk = __shfl_sync(0xffffffffu, near, src);
            const int srow = __shfl_sync(0xffffffffu, row, src);
            const float sinv = __shfl_sync(0xffffffffu, inv, src);
            const __half* ah = Ahi + (int64_t)srow * ldk;
            const __half* al = Alo + (int64_t)srow * ldk;
            while (msk) {
              const int i = __ffs(msk) - 1;
              msk &= msk - 1;
              const float* rr = R + (int64_t)(col0 + i) * d;
              double acc = 0.0;
              for (int k = lane; k < d; k += 32)
                acc = fma((double)(__half2float(ah[k]) + __half2float(al[k])), (double)__ldg(rr + k),
                          acc);
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
              const float xr = (float)(acc * ((double)sinv * (double)(1 << kScaleBias)));
              const uint32_t code = code_of<BITS>(xr, sb);
              if (lane == src) {
#pragma unroll
                for (int t = 0; t < 32; ++t)
                  if (t == i) c[t] = code;
              }
            }
          }
          if (!rv) continue;
          uint32_t w[8];
          pack32<BITS>(c, w);
          uint8_t* dst = packed + (int64_t)row * ldb + (int64_t)col0 * BITS / 8;
          const int64_t off0 = (int64_t)col0 * BITS / 8;
          if (off0 + 4 * BITS <= rb) {
            // 4*BITS bytes at a multiple of 4*BITS (col0 % 32 == 0, ldb % 16 == 0).
            if constexpr (BITS == 4 || BITS == 8) {
              uint4* dq = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int i = 0; i < BITS / 4; ++i)
                dq[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
            } else if constexpr (BITS == 2) {
              *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
            } else {
              uint32_t* dw = reinterpret_cast<uint32_t*>(dst);
#pragma unroll
              for (int i = 0; i < BITS; ++i) dw[i] = w[i];
            }
          } else {
            for (int i = 0; i < 4 * BITS && off0 + i < rb; ++i)
              dst[i] = (uint8_t)(w[i >> 2] >> (8 * (i & 3)));
          }
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar(TEMPTY + buf));
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, (uint32_t)tmem_cols);
  }
}

// Recomputes the coordinates the GEMM epilogue listed (within kFixBand of a
// boundary) as its inline path does -- an f64 dot product of the 22-bit x
// planes with the f32 R, scaled -- and writes their codes into the packed
// rows.  One warp per row with listed columns: the row's x (hi + lo, exact
// in f32, kept in L1 across the row's entries) is dotted with each listed
// column of R, with coalesced loads.  A row's codes may share a 32-bit word, so
// each code is written with an atomic AND (clear its bits) and OR (set
// them): codes occupy disjoint bits, so the order of the updates does not
// matter.
template <int BITS>
__global__ void __launch_bounds__(128)
encode_fix_kernel(const int* __restrict__ fix_cnt, const uint16_t* __restrict__ fix_cols,
                  int64_t m, const __half* __restrict__ Ahi, const __half* __restrict__ Alo,
                  int ldk, const float* __restrict__ inv_scale, const float* __restrict__ R,
                  int d, const float* __restrict__ bounds, uint8_t* __restrict__ packed,
                  int64_t ldb) {
  __shared__ float sb[256];
  for (int i = threadIdx.x; i < (1 << BITS) - 1; i += blockDim.x) sb[i] = bounds[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); row < m;
       row += warps) {
    const int cnt = min(__ldg(fix_cnt + row), kFixPerRow);
    if (cnt == 0) continue;  // warp-uniform
    // The row's planes stay in L1 across its listed columns.
    const uint2* ah = reinterpret_cast<const uint2*>(Ahi + row * ldk);
    const uint2* al = reinterpret_cast<const uint2*>(Alo + row * ldk);
    const float sinv = __ldg(inv_scale + row);
    uint32_t* rowp = reinterpret_cast<uint32_t*>(packed + row * ldb);
    // d <= 1024 (d % 4 == 0): the row's x is converted to f64 once and kept in
    // registers (elements 4m .. 4m+3 of lane l, m = l + 32 t); each listed
    // column then costs one pass over its R row with all loads in flight.
    const bool regx = (d & 3) == 0 && d <= 1024;
    double xd[32];
    if (regx) {
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int m = lane + 32 * t;
        uint2 hv = make_uint2(0u, 0u), lv = make_uint2(0u, 0u);
        if (4 * m < d) {
          hv = __ldg(ah + m);
          lv = __ldg(al + m);
        }
        const __half* hh = reinterpret_cast<const __half*>(&hv);
        const __half* ll = reinterpret_cast<const __half*>(&lv);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          xd[4 * t + u] = (double)(__half2float(hh[u]) + __half2float(ll[u]));
      }
    }
    for (int k = 0; k < cnt; ++k) {
      const int col = fix_cols[(size_t)row * kFixPerRow + k];
      const float* rr = R + (int64_t)col * d;
      double acc = 0.0;
      if (regx) {
        const float4* r4 = reinterpret_cast<const float4*>(rr);
        float4 rv[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const int m = lane + 32 * t;
          rv[t] = 4 * m < d ? __ldg(r4 + m) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          acc = fma(xd[4 * t + 0], (double)rv[t].x, acc);
          acc = fma(xd[4 * t + 1], (double)rv[t].y, acc);
          acc = fma(xd[4 * t + 2], (double)rv[t].z, acc);
          acc = fma(xd[4 * t + 3], (double)rv[t].w, acc);
        }
      } else if ((d & 3) == 0) {
        // Lane l takes elements 4m .. 4m+3, m = l + 32 t: the warp's R loads
        // (16 B a lane) and plane loads (8 B a lane) are contiguous; two
        // steps' loads are in flight before the first FMA of the pair.
        const float4* r4 = reinterpret_cast<const float4*>(rr);
        for (int m0 = 0; 4 * m0 < d; m0 += 64) {
          float4 rv[2];
          uint2 hv[2], lv[2];
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int m = m0 + lane + 32 * t;
            if (4 * m < d) {
              rv[t] = __ldg(r4 + m);
              hv[t] = __ldg(ah + m);
              lv[t] = __ldg(al + m);
            } else {
              rv[t] = make_float4(0.f, 0.f, 0.f, 0.f);
              hv[t] = lv[t] = make_uint2(0u, 0u);
            }
          }
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const __half* hh = reinterpret_cast<const __half*>(&hv[t]);
            const __half* ll = reinterpret_cast<const __half*>(&lv[t]);
            const float r4v[4] = {rv[t].x, rv[t].y, rv[t].z, rv[t].w};
#pragma unroll
            for (int u = 0; u < 4; ++u)
              acc = fma((double)(__half2float(hh[u]) + __half2float(ll[u])), (double)r4v[u], acc);
          }
        }
      } else {
        const __half* hs = Ahi + row * ldk;
        const __half* ls = Alo + row * ldk;
        for (int j = lane; j < d; j += 32)
          acc = fma((double)(__half2float(hs[j]) + __half2float(ls[j])), (double)__ldg(rr + j),
                    acc);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane != 0) continue;
      const float xr = (float)(acc * ((double)sinv * (double)(1 << kScaleBias)));
      const uint32_t code = code_of<BITS>(xr, sb);
      // Stream bit p + i (MSB-first) holds code bit BITS - 1 - i; at most two
      // 32-bit words of the row are touched (3-bit codes may straddle bytes).
      const int p = col * BITS;
      int w0 = -1, w1 = -1;
      uint32_t m0 = 0, m1 = 0, v0 = 0, v1 = 0;
#pragma unroll
      for (int i = 0; i < BITS; ++i) {
        const int bit = p + i, byte = bit >> 3;
        const int sh = 8 * (byte & 3) + 7 - (bit & 7);
        const uint32_t b = (code >> (BITS - 1 - i)) & 1u;
        if (w0 < 0 || w0 == (byte >> 2)) {
          w0 = byte >> 2;
          m0 |= 1u << sh;
          v0 |= b << sh;
        } else {
          w1 = byte >> 2;
          m1 |= 1u << sh;
          v1 |= b << sh;
        }
      }
      atomicAnd(rowp + w0, ~m0);
      atomicOr(rowp + w0, v0);
      if (w1 >= 0) {
        atomicAnd(rowp + w1, ~m1);
        atomicOr(rowp + w1, v1);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// fp16 matrix (rows x ldk, row-major) tiled as {64 (K), box_rows} with 128B swizzle.
static int make_map(CUtensorMap* map, const void* ptr, int64_t rows, int ldk, int box_rows) {
  auto fn = get_encode_fn();
  if (!fn) return fail(PQ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  PQ_CHECK_ARG(((uintptr_t)ptr & 15) == 0, "TMA base must be 16-byte aligned");
  cuuint64_t dims[2] = {(cuuint64_t)ldk, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ldk * 2};
  cuuint32_t box[2] = {(cuuint32_t)kEncBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return PQ_OK;
}

// Rows per chunk (>= one M tile, so a TMA box never exceeds the tensor).
static int64_t enc_chunk_rows(int64_t n) {
  const int64_t cap = 131072;
  const int64_t c = n < cap ? n : cap;
  return c < kEncBM ? kEncBM : c;
}

}  // namespace pqb

using namespace pqb;

// Per device: the side stream and events of the encode pipeline (created on
// first use; the pipeline's enqueue runs under a mutex, so concurrent encode
// calls from several host threads do not interleave their event records).
// Streams of the chunk pipeline: the GEMMs on s1 (the device's highest
// priority, so that as an SM frees up the block scheduler places the next
// GEMM's CTA before more side-kernel blocks), prep and fix-up on s2.
struct EncSide {
  cudaStream_t s1, s2;
  cudaEvent_t start, prep[2], gemm[2], end1, end2;
  bool ok;
};
static EncSide g_enc_side[64];
static std::mutex g_enc_mu;

static int enc_side(EncSide** out) {
  int dev = 0;
  PQ_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(PQ_ERR_CUDA, "device ordinal %d out of range", dev);
  EncSide& e = g_enc_side[dev];
  if (!e.ok) {
    int least = 0, greatest = 0;
    PQ_CUDA_TRY(cudaDeviceGetStreamPriorityRange(&least, &greatest));
    PQ_CUDA_TRY(cudaStreamCreateWithPriority(&e.s1, cudaStreamNonBlocking, greatest));
    PQ_CUDA_TRY(cudaStreamCreateWithPriority(&e.s2, cudaStreamNonBlocking, least));
    PQ_CUDA_TRY(cudaEventCreateWithFlags(&e.start, cudaEventDisableTiming));
    PQ_CUDA_TRY(cudaEventCreateWithFlags(&e.end1, cudaEventDisableTiming));
    PQ_CUDA_TRY(cudaEventCreateWithFlags(&e.end2, cudaEventDisableTiming));
    for (int i = 0; i < 2; ++i) {
      PQ_CUDA_TRY(cudaEventCreateWithFlags(&e.prep[i], cudaEventDisableTiming));
      PQ_CUDA_TRY(cudaEventCreateWithFlags(&e.gemm[i], cudaEventDisableTiming));
    }
    e.ok = true;
  }
  *out = &e;
  return PQ_OK;
}

// Kernels that run beside the encode GEMM (which keeps ~200 KB of shared
// memory per SM) ask for the same maximal shared-memory carveout: an SM runs
// blocks of different kernels at once only under one L1 / shared-memory
// split, so with the default preference their blocks would wait for the GEMM
// to leave the SM.
static void enc_side_carveout(const void* kern) {
  cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                       (int)cudaSharedmemCarveoutMaxShared);
}

static int launch_prep(const float* X, int64_t m, int d, int ldk, __half* Ahi, __half* Alo,
                       float* inv, float* norms, bool normalize, cudaStream_t st) {
  const int T = (ldk + 127) / 128;
  if (d % 4 == 0 && ((uintptr_t)X & 15) == 0 && T <= 16) {
    int g = (int)((m + 3) / 4);
    if (g > num_sms() * 32) g = num_sms() * 32;
    switch (T) {
#define PQ_PREP4(TT)                                                                         \
  case TT:                                                                                   \
    if (normalize) {                                                                         \
      enc_side_carveout((const void*)encode_prep4_kernel<true, TT>);                         \
      encode_prep4_kernel<true, TT><<<g, 128, 0, st>>>(X, m, d, ldk, Ahi, Alo, inv, norms);  \
    } else {                                                                                 \
      enc_side_carveout((const void*)encode_prep4_kernel<false, TT>);                        \
      encode_prep4_kernel<false, TT><<<g, 128, 0, st>>>(X, m, d, ldk, Ahi, Alo, inv, norms); \
    }                                                                                        \
    break;
      PQ_PREP4(1) PQ_PREP4(2) PQ_PREP4(3) PQ_PREP4(4) PQ_PREP4(5) PQ_PREP4(6) PQ_PREP4(7)
      PQ_PREP4(8) PQ_PREP4(9) PQ_PREP4(10) PQ_PREP4(11) PQ_PREP4(12) PQ_PREP4(13)
      PQ_PREP4(14) PQ_PREP4(15) PQ_PREP4(16)
#undef PQ_PREP4
    }
    PQ_LAUNCH_CHECK("encode_prep4_kernel");
    return PQ_OK;
  }
  const int pg = (int)((m + 7) / 8 < (int64_t)num_sms() * 16 ? (m + 7) / 8 : num_sms() * 16);
  if (normalize)
    encode_prep_kernel<true><<<pg, 256, 0, st>>>(X, m, d, ldk, Ahi, Alo, inv, norms);
  else
    encode_prep_kernel<false><<<pg, 256, 0, st>>>(X, m, d, ldk, Ahi, Alo, inv, norms);
  PQ_LAUNCH_CHECK("encode_prep_kernel");
  return PQ_OK;
}

// Plane buffers of a call: two (ping-pong) when it spans several chunks.
static int enc_buffers(int64_t n) { return n > enc_chunk_rows(n) ? 2 : 1; }

// Encode in row chunks.  With several chunks the work runs as a pipeline on
// the caller's stream `st` and a side stream s2, ordered by events only (no
// host synchronisation):
//   s2: prep(0) prep(1) | fix(0) prep(2) | fix(1) prep(3) | ...
//   st:                 | gemm(0)        | gemm(1)        | ...
// so the HBM-bound normalise/split of chunk i+1 and the f64 fix-ups of chunk
// i-1 run while the tensor-bound GEMM of chunk i occupies the SMs.  Chunk i
// uses plane buffer i % 2; prep(i + 2) is enqueued on s2 after fix(i), which
// waits for gemm(i): the buffer is free by then.  `st` waits for s2's last
// work before the call returns its work to the caller.
static int run_encode(const float* X, int64_t n, int d, const void* planes, const float* R,
                      const float* bounds, int bits, uint8_t* packed, int64_t ldb, float* norms,
                      float* Y, void* ws, size_t ws_bytes, cudaStream_t st) {
  const EncShape s = enc_shape(d);
  const int64_t ch = enc_chunk_rows(n);
  const int nbuf = enc_buffers(n);
  Carve cv(ws, ws_bytes);
  __half *Ahi[2], *Alo[2];
  float* inv[2];
  int* fix_cnt[2];
  uint16_t* fix_cols[2];
  // The listed fix-ups need d <= 2048 (the fix kernel keeps the row in
  // registers; columns fit 16 bits); wider rows recompute inline.
  const bool deferred = bits > 0 && d <= 2048;
  for (int b = 0; b < nbuf; ++b) {
    Ahi[b] = cv.take<__half>((size_t)ch * s.ldk);
    Alo[b] = cv.take<__half>((size_t)ch * s.ldk);
    inv[b] = cv.take<float>((size_t)ch);
    fix_cnt[b] = cv.take<int>((size_t)ch);
    fix_cols[b] = cv.take<uint16_t>((size_t)ch * kFixPerRow);
  }
  if (!cv.ok()) return fail(PQ_ERR_WORKSPACE, "encode workspace too small (%zu bytes)", ws_bytes);
  const __half* Rhi = (const __half*)planes;
  const __half* Rlo = Rhi + (size_t)s.ldn * s.ldk;
  CUtensorMap mAhi[2], mAlo[2], mBhi, mBlo;
  int rc;
  for (int b = 0; b < nbuf; ++b) {
    if ((rc = make_map(&mAhi[b], Ahi[b], ch, s.ldk, kEncBM))) return rc;
    if ((rc = make_map(&mAlo[b], Alo[b], ch, s.ldk, kEncBM))) return rc;
  }
  if ((rc = make_map(&mBhi, Rhi, s.ldn, s.ldk, s.BN))) return rc;
  if ((rc = make_map(&mBlo, Rlo, s.ldn, s.ldk, s.BN))) return rc;

  const size_t sm = s.smem_bytes;
  if (sm > 227 * 1024) return fail(PQ_ERR_UNSUPPORTED, "encode tile needs %zu bytes of smem", sm);
  const int64_t rb = row_bytes(d, bits > 0 ? bits : 8);
  const int nch = (int)((n + ch - 1) / ch);

  std::unique_lock<std::mutex> lock(g_enc_mu, std::defer_lock);
  EncSide* side = nullptr;
  cudaStream_t s1 = st, s2 = st;  // one chunk: everything on the caller's stream
  if (nbuf == 2) {
    lock.lock();
    if ((rc = enc_side(&side))) return rc;
    s1 = side->s1;
    s2 = side->s2;
    PQ_CUDA_TRY(cudaEventRecord(side->start, st));
    PQ_CUDA_TRY(cudaStreamWaitEvent(s1, side->start, 0));
    PQ_CUDA_TRY(cudaStreamWaitEvent(s2, side->start, 0));
  }
  auto chunk_rows = [&](int i) { return (n - (int64_t)i * ch < ch) ? n - (int64_t)i * ch : ch; };
  auto prep = [&](int i) -> int {
    const int b = i % nbuf;
    const int64_t r0 = (int64_t)i * ch;
    int r = launch_prep(X + r0 * d, chunk_rows(i), d, s.ldk, Ahi[b], Alo[b], inv[b],
                        (bits > 0 && norms) ? norms + r0 : nullptr, bits > 0, s2);
    if (r) return r;
    if (side) PQ_CUDA_TRY(cudaEventRecord(side->prep[b], s2));
    return PQ_OK;
  };
  auto fix = [&](int i) -> int {
    if (!deferred) return PQ_OK;
    const int b = i % nbuf;
    const int64_t r0 = (int64_t)i * ch;
    const int64_t m = chunk_rows(i);
    uint8_t* pk = packed + r0 * ldb;
    const int g = num_sms() * 4;  // the resident blocks (128 registers a thread)
    switch (bits) {
#define PQ_FIX_CASE(B)                                                                      \
  case B:                                                                                   \
    encode_fix_kernel<B><<<g, 128, 0, s2>>>(fix_cnt[b], fix_cols[b], m, Ahi[b], Alo[b],     \
                                            s.ldk, inv[b], R, d, bounds, pk, ldb);          \
    break;
      PQ_FIX_CASE(1)
      PQ_FIX_CASE(2)
      PQ_FIX_CASE(3)
      PQ_FIX_CASE(4)
      PQ_FIX_CASE(8)
#undef PQ_FIX_CASE
    }
    PQ_LAUNCH_CHECK("encode_fix_kernel");
    return PQ_OK;
  };

  if ((rc = prep(0))) return rc;
  if (nch > 1 && (rc = prep(1))) return rc;
  for (int i = 0; i < nch; ++i) {
    const int b = i % nbuf;
    const int64_t r0 = (int64_t)i * ch;
    const int64_t m = chunk_rows(i);
    if (side) PQ_CUDA_TRY(cudaStreamWaitEvent(s1, side->prep[b], 0));
    const int ntiles = (int)((m + kEncBM - 1) / kEncBM) * s.ntn;
    const int grid = ntiles < num_sms() ? ntiles : num_sms();
    uint8_t* pk = packed ? packed + r0 * ldb : nullptr;
    float* yk = Y ? Y + r0 * d : nullptr;
    if (deferred) PQ_CUDA_TRY(cudaMemsetAsync(fix_cnt[b], 0, sizeof(int) * (size_t)m, s1));
    switch (bits) {
#define PQ_ENC_CASE(B)                                                                        \
  case B: {                                                                                   \
    auto kern = encode_gemm_kernel<B>;                                                        \
    PQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm)); \
    kern<<<grid, kEncThreads, sm, s1>>>(mAhi[b], mAlo[b], mBhi, mBlo, (int)m, d, s.BN, s.ntn,  \
                                        s.nk, s.stages, s.tmem_cols, inv[b], bounds, pk, ldb, \
                                        rb, yk, Ahi[b], Alo[b], s.ldk, R,                      \
                                        deferred ? fix_cnt[b] : nullptr, fix_cols[b]);         \
  } break;
      PQ_ENC_CASE(0)
      PQ_ENC_CASE(1)
      PQ_ENC_CASE(2)
      PQ_ENC_CASE(3)
      PQ_ENC_CASE(4)
      PQ_ENC_CASE(8)
#undef PQ_ENC_CASE
      default:
        return fail(PQ_ERR_INVALID, "bits must be one of 1,2,3,4,8 (got %d)", bits);
    }
    PQ_LAUNCH_CHECK("encode_gemm_kernel");
    if (side) {
      PQ_CUDA_TRY(cudaEventRecord(side->gemm[b], s1));
      PQ_CUDA_TRY(cudaStreamWaitEvent(s2, side->gemm[b], 0));
    }
    if ((rc = fix(i))) return rc;
    if (i + 2 < nch && (rc = prep(i + 2))) return rc;
  }
  if (side) {
    PQ_CUDA_TRY(cudaEventRecord(side->end1, s1));
    PQ_CUDA_TRY(cudaEventRecord(side->end2, s2));
    PQ_CUDA_TRY(cudaStreamWaitEvent(st, side->end1, 0));
    PQ_CUDA_TRY(cudaStreamWaitEvent(st, side->end2, 0));
  }
  return PQ_OK;
}

extern "C" {

size_t pq_rotation_planes_bytes(int d) {
  if (d <= 0) return 0;
  const EncShape s = enc_shape(d);
  return (size_t)2 * s.ldn * s.ldk * sizeof(__half);
}

int pq_prepare_rotation(const float* R, int d, void* planes, size_t planes_bytes, void* stream) {
  PQ_CHECK_ARG(d > 0, "d must be positive (got %d)", d);
  PQ_CHECK_ARG(R && planes, "null pointer argument");
  PQ_CHECK_ARG(planes_bytes >= pq_rotation_planes_bytes(d), "planes buffer too small");
  PQ_CHECK_ARG(((uintptr_t)planes & 15) == 0, "planes must be 16-byte aligned");
  const EncShape s = enc_shape(d);
  __half* hi = (__half*)planes;
  __half* lo = hi + (size_t)s.ldn * s.ldk;
  const int64_t total = (int64_t)s.ldn * s.ldk;
  int g = (int)((total + 255) / 256);
  if (g > num_sms() * 16) g = num_sms() * 16;
  rot_planes_kernel<<<g, 256, 0, (cudaStream_t)stream>>>(R, d, s.ldn, s.ldk, hi, lo);
  PQ_LAUNCH_CHECK("rot_planes_kernel");
  return PQ_OK;
}

size_t pq_encode_workspace_bytes(int64_t n, int d) {
  if (d <= 0) return 256;
  const EncShape s = enc_shape(d);
  const size_t ch = (size_t)enc_chunk_rows(n);
  const size_t one = align_up(ch * s.ldk * 2, 256) * 2 + align_up(ch * 4, 256) * 2 +
                     align_up(ch * kFixPerRow * 2, 256);
  return one * enc_buffers(n) + 1024;
}

int pq_encode(const float* X, int64_t n, int d, const float* R, const void* planes,
              const float* boundaries, int bits, uint8_t* packed, int64_t ldb, float* norms,
              void* ws, size_t ws_bytes, void* stream) {
  PQ_CHECK_ARG(supported_bits(bits), "bits must be one of 1,2,3,4,8 (got %d)", bits);
  PQ_CHECK_ARG(d > 0, "d must be positive (got %d)", d);
  PQ_CHECK_ARG(n >= 0, "n must be >= 0");
  PQ_CHECK_ARG(ldb >= row_bytes(d, bits) && ldb % 16 == 0,
               "row stride ldb=%lld must be a multiple of 16 and >= %lld", (long long)ldb,
               (long long)row_bytes(d, bits));
  if (n == 0) return PQ_OK;
  PQ_CHECK_ARG(X && R && planes && boundaries && packed && norms && ws, "null pointer argument");
  PQ_CHECK_ARG(((uintptr_t)packed & 15) == 0, "packed rows must be 16-byte aligned");
  const size_t need = pq_encode_workspace_bytes(n, d);
  if (ws_bytes < need)
    return fail(PQ_ERR_WORKSPACE, "pq_encode needs %zu workspace bytes, got %zu", need, ws_bytes);
  return run_encode(X, n, d, planes, R, boundaries, bits, packed, ldb, norms, nullptr, ws,
                    ws_bytes, (cudaStream_t)stream);
}

int pq_rotate_tc(const float* X, int64_t n, int d, const void* planes, float* Y, void* ws,
                 size_t ws_bytes, void* stream) {
  PQ_CHECK_ARG(d > 0, "d must be positive (got %d)", d);
  PQ_CHECK_ARG(n >= 0, "n must be >= 0");
  if (n == 0) return PQ_OK;
  PQ_CHECK_ARG(X && planes && Y && ws, "null pointer argument");
  const size_t need = pq_encode_workspace_bytes(n, d);
  if (ws_bytes < need)
    return fail(PQ_ERR_WORKSPACE, "pq_rotate_tc needs %zu workspace bytes, got %zu", need,
                ws_bytes);
  return run_encode(X, n, d, planes, nullptr, nullptr, 0, nullptr, 0, nullptr, Y, ws, ws_bytes,
                    (cudaStream_t)stream);
}

}  // extern "C"
