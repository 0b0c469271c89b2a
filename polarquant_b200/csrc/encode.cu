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

#include "tc.cuh"

namespace pqb {

constexpr int kEncBM = 128;     // rows per tile (TMEM lanes)
constexpr int kEncBK = 64;      // K per stage: one 128-byte swizzle atom of fp16
constexpr int kEncThreads = 320;  // warp 0 TMA, warp 1 MMA + TMEM, warps 2-9 epilogue
constexpr int kScaleBias = 14;  // R planes hold R * 2^14
constexpr int kGuideCells = 1024;  // uniform cells of the 8-bit guide table
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
// and last boundary gives each value a starting level (the number of
// boundaries below its cell's left edge); a walk of one or two steps then
// lands on #{boundaries < x} (searchsorted side='left').  The walk checks the
// boundaries on both sides, so the result is exact whatever cell the float
// arithmetic picks; the last line falls back to the binary search in the
// (never observed) case that two steps were not enough.
struct Guide {
  float lo, scale;  // cell of x = (x - lo) * scale
};

__device__ __forceinline__ uint32_t code_guided(float x, const float* sb, const uint8_t* guide,
                                                Guide g) {
  constexpr uint32_t L1 = 255u;  // number of boundaries
  float t = (x - g.lo) * g.scale;
  t = fminf(fmaxf(t, 0.f), (float)(kGuideCells - 1));
  uint32_t c = guide[(int)t];
  // Up to two steps up, then one down; each compares against a boundary.
  if (c < L1 && x > sb[c]) ++c;
  if (c < L1 && x > sb[c]) ++c;
  if (c > 0 && !(x > sb[c - 1])) --c;
  const bool ok = (c == 0 || x > sb[c - 1]) && (c == L1 || !(x > sb[c]));
  return ok ? c : code_of<8>(x, sb);
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
                   const float* __restrict__ R, unsigned long long* __restrict__ fix_list,
                   unsigned int* __restrict__ fix_count, int fix_cap) {
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
          if constexpr (BITS == 8) {
#pragma unroll
            for (int i = 0; i < 32; ++i) c[i] = code_guided(x[i], sb, guide, gd);
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
            if (!valid) c[i] = 0;
            else if (near_boundary<BITS>(x[i], c[i], sb)) near |= 1u << i;
          }
          // Coordinates within kFixBand of a boundary are recomputed in f64
          // from the exact f32 R and the 22-bit x planes, so the side of the
          // boundary does not depend on the tensor core's f32 accumulation
          // order.  They go to the fix-up list (encode_fix_kernel recomputes
          // them all after this kernel, many warps at once, and patches the
          // packed codes); only when the list is full does the warp
          // recompute them here.
          if (near && fix_list) {
            const uint32_t cnt = (uint32_t)__popc(near);
            const uint32_t base = atomicAdd(fix_count, cnt);
            if (base + cnt <= (uint32_t)fix_cap) {
              uint32_t msk = near, k = 0;
              while (msk) {
                const int i = __ffs(msk) - 1;
                msk &= msk - 1;
                fix_list[base + k++] =
                    ((unsigned long long)row << 32) | (unsigned)(col0 + i);
              }
              near = 0;
            } else {
              // Slots reserved below the capacity stay unused: mark them.
              for (uint32_t k = base; k < (uint32_t)fix_cap && k < base + cnt; ++k)
                fix_list[k] = ~0ull;
            }
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
// boundary) exactly as its inline path does -- f64 dot product of the 22-bit
// x planes with the f32 R, scaled -- and writes their codes into the packed
// rows.  One warp per entry; entries of one row may share a 32-bit word, so
// each code is written with an atomic AND (clear its bits) and OR (set
// them): codes occupy disjoint bits, so the order of the updates does not
// matter.  Entries ~0 are slots reserved but left unused.
template <int BITS>
__global__ void __launch_bounds__(256)
encode_fix_kernel(const unsigned long long* __restrict__ fix_list,
                  const unsigned int* __restrict__ fix_count, int fix_cap,
                  const __half* __restrict__ Ahi, const __half* __restrict__ Alo, int ldk,
                  const float* __restrict__ inv_scale, const float* __restrict__ R, int d,
                  const float* __restrict__ bounds, uint8_t* __restrict__ packed, int64_t ldb) {
  __shared__ float sb[256];
  for (int i = threadIdx.x; i < (1 << BITS) - 1; i += blockDim.x) sb[i] = bounds[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const unsigned total = min(*fix_count, (unsigned)fix_cap);
  const unsigned warps = gridDim.x * (blockDim.x >> 5);
  for (unsigned e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); e < total; e += warps) {
    const unsigned long long ent = fix_list[e];
    if (ent == ~0ull) continue;  // warp-uniform
    const int row = (int)(ent >> 32), col = (int)(ent & 0xFFFFFFFFu);
    const __half* ah = Ahi + (int64_t)row * ldk;
    const __half* al = Alo + (int64_t)row * ldk;
    const float* rr = R + (int64_t)col * d;
    double acc = 0.0;
    for (int k = lane; k < d; k += 32)
      acc = fma((double)(__half2float(ah[k]) + __half2float(al[k])), (double)__ldg(rr + k), acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane != 0) continue;
    const float sinv = __ldg(inv_scale + row);
    const float xr = (float)(acc * ((double)sinv * (double)(1 << kScaleBias)));
    const uint32_t code = code_of<BITS>(xr, sb);
    // Stream bit p + i (MSB-first) holds code bit BITS - 1 - i; at most two
    // 32-bit words of the row are touched (3-bit codes may straddle bytes).
    uint32_t* rowp = reinterpret_cast<uint32_t*>(packed + (int64_t)row * ldb);
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

// Entries of the near-boundary fix-up list per chunk: ~2x the share of 8-bit
// coordinates that land within kFixBand of a boundary (~0.2%); calls that
// overflow it recompute the rest inline.
static int enc_fix_cap(int64_t chunk_rows, int d) {
  const int64_t c = chunk_rows * d / 256;
  return (int)(c < 65536 ? 65536 : (c > (1 << 26) ? (1 << 26) : c));
}

// Rows per chunk (>= one M tile, so a TMA box never exceeds the tensor).
static int64_t enc_chunk_rows(int64_t n) {
  const int64_t cap = 131072;
  const int64_t c = n < cap ? n : cap;
  return c < kEncBM ? kEncBM : c;
}

}  // namespace pqb

using namespace pqb;

static int run_encode(const float* X, int64_t n, int d, const void* planes, const float* R,
                      const float* bounds, int bits, uint8_t* packed, int64_t ldb, float* norms,
                      float* Y, void* ws, size_t ws_bytes, cudaStream_t st) {
  const EncShape s = enc_shape(d);
  const int64_t ch = enc_chunk_rows(n);
  Carve cv(ws, ws_bytes);
  __half* Ahi = cv.take<__half>((size_t)ch * s.ldk);
  __half* Alo = cv.take<__half>((size_t)ch * s.ldk);
  float* inv = cv.take<float>((size_t)ch);
  const int fix_cap = enc_fix_cap(ch, d);
  unsigned int* fix_count = cv.take<unsigned int>(1);
  unsigned long long* fix_list = cv.take<unsigned long long>((size_t)fix_cap);
  if (!cv.ok()) return fail(PQ_ERR_WORKSPACE, "encode workspace too small (%zu bytes)", ws_bytes);
  const __half* Rhi = (const __half*)planes;
  const __half* Rlo = Rhi + (size_t)s.ldn * s.ldk;
  CUtensorMap mAhi, mAlo, mBhi, mBlo;
  int rc;
  if ((rc = make_map(&mAhi, Ahi, ch, s.ldk, kEncBM))) return rc;
  if ((rc = make_map(&mAlo, Alo, ch, s.ldk, kEncBM))) return rc;
  if ((rc = make_map(&mBhi, Rhi, s.ldn, s.ldk, s.BN))) return rc;
  if ((rc = make_map(&mBlo, Rlo, s.ldn, s.ldk, s.BN))) return rc;

  const size_t sm = s.smem_bytes;
  if (sm > 227 * 1024) return fail(PQ_ERR_UNSUPPORTED, "encode tile needs %zu bytes of smem", sm);
  const int64_t rb = row_bytes(d, bits > 0 ? bits : 8);
  for (int64_t r0 = 0; r0 < n; r0 += ch) {
    const int64_t m = (n - r0 < ch) ? n - r0 : ch;
    const int pg = (int)((m + 7) / 8 < (int64_t)num_sms() * 16 ? (m + 7) / 8 : num_sms() * 16);
    if (bits > 0)
      encode_prep_kernel<true><<<pg, 256, 0, st>>>(X + r0 * d, m, d, s.ldk, Ahi, Alo, inv,
                                                   norms ? norms + r0 : nullptr);
    else
      encode_prep_kernel<false><<<pg, 256, 0, st>>>(X + r0 * d, m, d, s.ldk, Ahi, Alo, inv,
                                                    nullptr);
    PQ_LAUNCH_CHECK("encode_prep_kernel");
    const int ntiles = (int)((m + kEncBM - 1) / kEncBM) * s.ntn;
    const int grid = ntiles < num_sms() ? ntiles : num_sms();
    uint8_t* pk = packed ? packed + r0 * ldb : nullptr;
    float* yk = Y ? Y + r0 * d : nullptr;
    if (bits > 0) PQ_CUDA_TRY(cudaMemsetAsync(fix_count, 0, sizeof(unsigned int), st));
    switch (bits) {
#define PQ_ENC_CASE(B)                                                                        \
  case B: {                                                                                   \
    auto kern = encode_gemm_kernel<B>;                                                        \
    PQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm)); \
    kern<<<grid, kEncThreads, sm, st>>>(mAhi, mAlo, mBhi, mBlo, (int)m, d, s.BN, s.ntn, s.nk,   \
                                        s.stages, s.tmem_cols, inv, bounds, pk, ldb, rb, yk,  \
                                        Ahi, Alo, s.ldk, R, B > 0 ? fix_list : nullptr,       \
                                        fix_count, fix_cap);                                  \
    PQ_LAUNCH_CHECK("encode_gemm_kernel");                                                    \
    if (B > 0) {                                                                              \
      encode_fix_kernel<(B > 0 ? B : 1)><<<num_sms() * 4, 256, 0, st>>>(                       \
          fix_list, fix_count, fix_cap, Ahi, Alo, s.ldk, inv, R, d, bounds, pk, ldb);          \
      PQ_LAUNCH_CHECK("encode_fix_kernel");                                                   \
    }                                                                                         \
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
  return align_up(ch * s.ldk * 2, 256) * 2 + align_up(ch * 4, 256) + 256 +
         (size_t)enc_fix_cap((int64_t)ch, d) * 8 + 1024;
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
