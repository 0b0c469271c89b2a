// Packed-code readers and per-row ADC scoring shared by the scan, rerank,
// IVF and unpack kernels.
//
// Storage format (remex/packing.py:18-75): every width is an MSB-first
// bitstream of b-bit codes, one row per packed_nbytes(1, d, b) bytes
// (the row-padded PackedVectors layout, remex/core.py:203-223).  On the device
// each row is padded further to a stride `ldb` that is a multiple of 16 bytes
// so a row can be streamed with 128-bit loads; buffers carry 64 bytes of slack
// past the last row because the 3-bit reader fetches whole 12-byte groups.
#pragma once
#include "common.cuh"

namespace pqb {

// Number of bytes one "unit" of the per-row loop reads, and the codes in it.
template <int B> struct Unit {
  static constexpr int BYTES = (B == 3) ? 12 : 16;
  static constexpr int CODES = BYTES * 8 / B;
};

// Loads one unit of row bytes as 32-bit little-endian words.
template <int B>
__device__ __forceinline__ void load_unit(const uint8_t* p, uint32_t w[4]) {
  if constexpr (B == 3) {
    const uint32_t* q = reinterpret_cast<const uint32_t*>(p);
    w[0] = __ldg(q);
    w[1] = __ldg(q + 1);
    w[2] = __ldg(q + 2);
    w[3] = 0;
  } else {
    uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  }
}

// Byte t (0..BYTES-1, memory order) of a unit.
__device__ __forceinline__ uint32_t unit_byte(const uint32_t w[4], int t) {
  return (w[t >> 2] >> (8 * (t & 3))) & 0xFFu;
}

// Code u (0..CODES-1) of a unit, MSB-first within the bitstream.
template <int B>
__device__ __forceinline__ uint32_t unit_code(const uint32_t w[4], int u) {
  if constexpr (B == 3) {
    const int g = u >> 3, t = u & 7;  // 3-byte group, position in group
    const uint32_t v = (unit_byte(w, 3 * g) << 16) | (unit_byte(w, 3 * g + 1) << 8) |
                       unit_byte(w, 3 * g + 2);
    return (v >> (21 - 3 * t)) & 7u;
  } else {
    constexpr int PER = 8 / B;
    const int byte = u / PER, pos = u % PER;
    const int word = byte >> 2, sh = 8 * (byte & 3) + 8 - B * (pos + 1);
    return (w[word] >> sh) & ((1u << B) - 1u);
  }
}

// Score of one row: sum_j q[j] * cent[code_j >> (B - P)].
//
// TABLE mode (P <= 4): `tab` is the per-query lookup table
// T[j*16 + c] = fl(q_rot[j] * cent[c]) -- the f32 products of the reference's
// `np.outer(q_rot, centroids)` (remex/core.py:618) -- so the sum adds the same
// rounded terms the reference gathers (core.py:823), in a different order.
// All lanes of a warp read the same j at once, so the 16-entry row of T is
// bank-conflict free.
//
// DIRECT mode (P > 4): `qs` holds q_rot (broadcast reads) and `crep` the
// centroid table replicated per lane (crep[c*32 + lane]) so the 2^P-entry
// lookups never collide on a bank; products are fused into the sum.
template <int B, int P>
__device__ __forceinline__ float score_row(const uint8_t* __restrict__ row, int d,
                                           const float* __restrict__ tab,
                                           const float* __restrict__ qs,
                                           const float* __restrict__ crep, int lane) {
  constexpr int SHIFT = B - P;
  constexpr int CU = Unit<B>::CODES;
  float acc0 = 0.f, acc1 = 0.f;
  const int full = d / CU;
  int u = 0;
  for (; u < full; ++u) {
    uint32_t w[4];
    load_unit<B>(row + u * Unit<B>::BYTES, w);
    const int j0 = u * CU;
#pragma unroll
    for (int t = 0; t < CU; ++t) {
      const uint32_t c = unit_code<B>(w, t) >> SHIFT;
      float v;
      if constexpr (P <= 4) {
        v = tab[(j0 + t) * 16 + c];
        if (t & 1) acc1 += v; else acc0 += v;
      } else {
        if (t & 1) acc1 = fmaf(qs[j0 + t], crep[c * 32 + lane], acc1);
        else acc0 = fmaf(qs[j0 + t], crep[c * 32 + lane], acc0);
      }
    }
  }
  const int rem = d - full * CU;
  if (rem > 0) {
    uint32_t w[4];
    load_unit<B>(row + u * Unit<B>::BYTES, w);
    const int j0 = u * CU;
    for (int t = 0; t < rem; ++t) {
      const uint32_t c = unit_code<B>(w, t) >> SHIFT;
      if constexpr (P <= 4) acc0 += tab[(j0 + t) * 16 + c];
      else acc0 = fmaf(qs[j0 + t], crep[c * 32 + lane], acc0);
    }
  }
  return acc0 + acc1;
}

// Pair tables for 4-bit codes at precision P <= 2: a byte's two codes keep 2P
// bits after the shift, so one 16-entry table per byte position p covers
// both: T2[p*16 + (hi << P | lo)] = fl(q[2p] * cent[hi]) + fl(q[2p+1] * cent[lo])
// (the reference's f32 table entries, remex/core.py:618, added in another
// order; a missing odd coordinate contributes 0).  One lookup per byte
// instead of one per code, and half the table.
template <int B, int P>
struct PairTab {
  static constexpr bool on = (B == 4 && P <= 2);
};

template <int P>
__device__ __forceinline__ void build_pair_tables(const float* __restrict__ q, int d,
                                                  const float* __restrict__ cent, float* tab) {
  const int nb = (d + 1) / 2;
  for (int i = threadIdx.x; i < nb * 16; i += blockDim.x) {
    const int p = i >> 4, idx = i & 15;
    const int hi = idx >> P, lo = idx & ((1 << P) - 1);
    float v = 0.f;
    if (hi < (1 << P)) {
      v = __fmul_rn(q[2 * p], cent[hi]);
      if (2 * p + 1 < d) v = __fadd_rn(v, __fmul_rn(q[2 * p + 1], cent[lo]));
    }
    tab[i] = v;
  }
}

// score_row for 4-bit codes at precision P <= 2 through the pair tables.
template <int P>
__device__ __forceinline__ float score_row_pair(const uint8_t* __restrict__ row, int d,
                                                const float* __restrict__ tab) {
  constexpr int SHIFT = 4 - P;
  constexpr uint32_t LO = (1u << P) - 1u;
  const int nb = (d + 1) / 2;  // bytes of the row
  float acc0 = 0.f, acc1 = 0.f;
  const int full = nb / 16;
  int u = 0;
  // The four bytes of a word give their four table indices at once: byte i
  // of ((w >> (4 + SHIFT - P)) & MHI) | ((w >> SHIFT) & MLO) is byte i's
  // (hi << P | lo).
  constexpr uint32_t MLO = LO * 0x01010101u;
  constexpr uint32_t MHI = (LO << P) * 0x01010101u;
  auto unit = [&](const uint32_t (&w)[4], const float* t0) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t ix = ((w[k] >> (4 + SHIFT - P)) & MHI) | ((w[k] >> SHIFT) & MLO);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float v = t0[(4 * k + i) * 16 + ((ix >> (8 * i)) & 15u)];
        if (i & 1) acc1 += v; else acc0 += v;
      }
    }
  };
  // Four units' loads (64 bytes of the row) in flight before their lookups.
  for (; u + 4 <= full; u += 4) {
    uint32_t w[4][4];
#pragma unroll
    for (int v = 0; v < 4; ++v) load_unit<4>(row + (u + v) * 16, w[v]);
#pragma unroll
    for (int v = 0; v < 4; ++v) unit(w[v], tab + (u + v) * 256);
  }
  for (; u < full; ++u) {
    uint32_t w[4];
    load_unit<4>(row + u * 16, w);
    unit(w, tab + u * 256);
  }
  const int rem = nb - full * 16;
  if (rem > 0) {
    uint32_t w[4];
    load_unit<4>(row + u * 16, w);
    const float* t0 = tab + u * 256;
    for (int t = 0; t < rem; ++t) {
      const uint32_t b = unit_byte(w, t);
      acc0 += t0[t * 16 + (((b >> (4 + SHIFT)) << P) | ((b >> SHIFT) & LO))];
    }
  }
  return acc0 + acc1;
}

// Builds the per-query scoring state in shared memory.
// TABLE mode: tab[j*16 + c] = q[j] * cent[c] for c < 2^P (rest zero).
// DIRECT mode: qs[j] = q[j]; crep[c*32 + l] = cent[c].
template <int P>
__device__ __forceinline__ void build_query_state(const float* __restrict__ q, int d,
                                                  const float* __restrict__ cent,
                                                  float* tab, float* qs, float* crep) {
  if constexpr (P <= 4) {
    for (int i = threadIdx.x; i < d * 16; i += blockDim.x) {
      const int j = i >> 4, c = i & 15;
      tab[i] = (c < (1 << P)) ? __fmul_rn(q[j], cent[c]) : 0.f;
    }
  } else {
    for (int i = threadIdx.x; i < d; i += blockDim.x) qs[i] = q[i];
    for (int i = threadIdx.x; i < (1 << P) * 32; i += blockDim.x) crep[i] = cent[i >> 5];
  }
}

template <int P>
__host__ __device__ constexpr size_t query_state_floats(int d) {
  return (P <= 4) ? (size_t)d * 16 : (size_t)d + (size_t)(1 << P) * 32;
}

}  // namespace pqb
