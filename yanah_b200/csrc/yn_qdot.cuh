// Row dot products over MLX-affine quantised rows staged in shared memory.
//
// Lane mapping (shared by every kernel and restated by the oracle): a row of
// `rowbytes` bytes is split into 16-byte chunks. LPR = gcd(32, chunks) lanes
// work on one row, lane l of the row owns chunks ci = l + LPR*c for
// c = 0..CPL-1, and a warp covers 32/LPR rows per step. Per-lane partial sums
// are reduced with a butterfly over the LPR lanes.
//
// Two arithmetic paths:
//  * fp32 (8-bit matrices: routers, shared expert). Canonical order, bit-exact
//    against the oracle: per chunk segment d = fma(x_k, q_k, d) in k order,
//    acc = fma(scale, d, acc); acc = fma(bias, xsum_segment, acc).
//  * packed fp16 (2- and 4-bit routed experts). Codes are turned into fp16
//    pairs with one LOP3 per pair (magic exponent 0x6400 = 1024.0, codes left
//    in place and compensated by pre-dividing x by the position multiplier),
//    then HSUB2 removes the 1024 offset exactly and HFMA2 accumulates a chunk
//    segment in fp16. The segment sum is converted to fp32, unscaled and
//    combined with scale/bias in fp32. x is pre-multiplied by a power of two so
//    that max|x| lands in [64, 128): partial sums stay far from fp16 overflow.
#pragma once
#include "yn_common.cuh"

namespace ynb {

template <int BITS>
struct CodeFmt {
  static constexpr int CPC = 128 / BITS;   // codes per 16-byte chunk
  static constexpr int CPW = 32 / BITS;    // codes per uint32 word
  static constexpr uint32_t MASK = (1u << BITS) - 1u;
  static constexpr int PPW = CPW / 2;      // fp16 pairs per word (fp16 path)
};

// ------------------------------------------------------------ fp32 path
template <int BITS, int CPL, int NSEG>
struct XF32 {
  static constexpr int CPC = CodeFmt<BITS>::CPC;
  float v[CPL][CPC];
  float xs[CPL][NSEG];
};

// Load the lane's x values (from a bf16 vector in shared memory) and their
// per-segment sums (fp32, ascending k).
template <int BITS, int CPL, int NSEG>
YN_DEV void load_x_f32(XF32<BITS, CPL, NSEG>& X, const uint16_t* xs_bf16, int l, int lpr) {
  constexpr int CPC = CodeFmt<BITS>::CPC;
  constexpr int SEG = CPC / NSEG;
#pragma unroll
  for (int c = 0; c < CPL; ++c) {
    const int k0 = (l + lpr * c) * CPC;
    if (CPC % 8 == 0) {
#pragma unroll
      for (int q = 0; q < CPC / 8; ++q) {
        const uint4 w = *reinterpret_cast<const uint4*>(xs_bf16 + k0 + 8 * q);
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          X.v[c][8 * q + 2 * i] = bf16_to_f32((uint16_t)(ww[i] & 0xFFFFu));
          X.v[c][8 * q + 2 * i + 1] = bf16_to_f32((uint16_t)(ww[i] >> 16));
        }
      }
    } else {
#pragma unroll
      for (int e = 0; e < CPC; ++e) X.v[c][e] = bf16_to_f32(xs_bf16[k0 + e]);
    }
#pragma unroll
    for (int s = 0; s < NSEG; ++s) {
      float a = 0.0f;
#pragma unroll
      for (int e = 0; e < SEG; ++e) a = __fadd_rn(a, X.v[c][s * SEG + e]);
      X.xs[c][s] = a;
    }
  }
}

template <int BITS, int CPL, int NSEG>
YN_DEV float row_dot_f32(const uint8_t* codes_row, const uint16_t* s_row, const uint16_t* b_row,
                         const XF32<BITS, CPL, NSEG>& X, int l, int lpr, int gs) {
  constexpr int CPC = CodeFmt<BITS>::CPC;
  constexpr int CPW = CodeFmt<BITS>::CPW;
  constexpr uint32_t MASK = CodeFmt<BITS>::MASK;
  constexpr int SEG = CPC / NSEG;
  float acc = 0.0f;
#pragma unroll
  for (int c = 0; c < CPL; ++c) {
    const int ci = l + lpr * c;
    const uint4 w = *reinterpret_cast<const uint4*>(codes_row + 16 * ci);
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int s = 0; s < NSEG; ++s) {
      float d = 0.0f;
#pragma unroll
      for (int e = 0; e < SEG; ++e) {
        const int kk = s * SEG + e;
        uint32_t qb;
        if constexpr (BITS == 8)  // byte kk % 4 under the exponent of 2^23 in one PRMT
          qb = __byte_perm(wv[kk / CPW], 0x4B000000u, 0x7540u + (unsigned)(kk % CPW));
        else
          qb = ((wv[kk / CPW] >> (BITS * (kk % CPW))) & MASK) | 0x4B000000u;
        const float qf = __fsub_rn(__uint_as_float(qb), 8388608.0f);
        d = __fmaf_rn(X.v[c][kk], qf, d);
      }
      const int g = (ci * CPC + s * SEG) / gs;
      acc = __fmaf_rn(f16_to_f32(s_row[g]), d, acc);
      acc = __fmaf_rn(f16_to_f32(b_row[g]), X.xs[c][s], acc);
    }
  }
  return acc;
}

// ------------------------------------------------------------ fp16 path
template <int BITS>
struct PairMap;
template <>
struct PairMap<4> {  // word i: pair p covers codes (8i+a, 8i+a+4), a = p; multiplier 1 or 16
  YN_DEV static int lo(int i, int p) { return 8 * i + p; }
  YN_DEV static int hi(int i, int p) { return 8 * i + p + 4; }
  YN_DEV static float inv_mult(int p) { return (p & 1) ? 0.0625f : 1.0f; }
};
template <>
struct PairMap<2> {  // word i: pair p covers codes (16i+p, 16i+p+8); multiplier 4^p (p<5), 4^(p-5)
  YN_DEV static int lo(int i, int p) { return 16 * i + p; }
  YN_DEV static int hi(int i, int p) { return 16 * i + p + 8; }
  YN_DEV static float inv_mult(int p) {
    const int e = (p < 5) ? p : p - 5;
    return __int_as_float((127 - 2 * e) << 23);
  }
};

template <int BITS, int CPL, int NSEG>
struct XF16 {
  static constexpr int NP = CodeFmt<BITS>::CPC / 2;  // pairs per chunk
  __half2 h[CPL][NP];
  float xs[CPL][NSEG];
};

template <int BITS, int CPL, int NSEG>
YN_DEV void load_x_f16(XF16<BITS, CPL, NSEG>& X, const uint16_t* xs_bf16, float scale, int l, int lpr) {
  constexpr int CPC = CodeFmt<BITS>::CPC;
  constexpr int PPW = CodeFmt<BITS>::PPW;
  constexpr int SEG = CPC / NSEG;
#pragma unroll
  for (int c = 0; c < CPL; ++c) {
    const int k0 = (l + lpr * c) * CPC;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int p = 0; p < PPW; ++p) {
        const float m = __fmul_rn(scale, PairMap<BITS>::inv_mult(p));
        const float a = __fmul_rn(bf16_to_f32(xs_bf16[k0 + PairMap<BITS>::lo(i, p)]), m);
        const float b = __fmul_rn(bf16_to_f32(xs_bf16[k0 + PairMap<BITS>::hi(i, p)]), m);
        X.h[c][i * PPW + p] = __floats2half2_rn(a, b);
      }
    }
#pragma unroll
    for (int s = 0; s < NSEG; ++s) {
      float a = 0.0f;
#pragma unroll
      for (int e = 0; e < SEG; ++e) a = __fadd_rn(a, bf16_to_f32(xs_bf16[k0 + s * SEG + e]));
      X.xs[c][s] = a;
    }
  }
}

// Unpack one word into PPW fp16 pairs holding mult*q exactly.
template <int BITS>
YN_DEV void unpack_word(uint32_t w, __half2 (&h)[CodeFmt<BITS>::PPW]);

template <>
YN_DEV void unpack_word<4>(uint32_t w, __half2 (&h)[4]) {
  const uint32_t MAGIC = 0x64006400u;
  const uint32_t w8 = w >> 8;
  const uint32_t u0 = (w & 0x000F000Fu) | MAGIC;
  const uint32_t u1 = (w & 0x00F000F0u) | MAGIC;
  const uint32_t u2 = (w8 & 0x000F000Fu) | MAGIC;
  const uint32_t u3 = (w8 & 0x00F000F0u) | MAGIC;
  const __half2 off = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
  h[0] = __hsub2(*reinterpret_cast<const __half2*>(&u0), off);
  h[1] = __hsub2(*reinterpret_cast<const __half2*>(&u1), off);
  h[2] = __hsub2(*reinterpret_cast<const __half2*>(&u2), off);
  h[3] = __hsub2(*reinterpret_cast<const __half2*>(&u3), off);
}

template <>
YN_DEV void unpack_word<2>(uint32_t w, __half2 (&h)[8]) {
  const uint32_t MAGIC = 0x64006400u;
  const uint32_t w10 = w >> 10;
  uint32_t u[8];
  u[0] = (w & 0x00030003u) | MAGIC;
  u[1] = (w & 0x000C000Cu) | MAGIC;
  u[2] = (w & 0x00300030u) | MAGIC;
  u[3] = (w & 0x00C000C0u) | MAGIC;
  u[4] = (w & 0x03000300u) | MAGIC;
  u[5] = (w10 & 0x00030003u) | MAGIC;
  u[6] = (w10 & 0x000C000Cu) | MAGIC;
  u[7] = (w10 & 0x00300030u) | MAGIC;
  const __half2 off = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
#pragma unroll
  for (int p = 0; p < 8; ++p) h[p] = __hsub2(*reinterpret_cast<const __half2*>(&u[p]), off);
}

template <int BITS, int CPL, int NSEG>
YN_DEV float row_dot_f16(const uint8_t* codes_row, const uint16_t* s_row, const uint16_t* b_row,
                         const XF16<BITS, CPL, NSEG>& X, float inv_scale, int l, int lpr, int gs) {
  constexpr int CPC = CodeFmt<BITS>::CPC;
  constexpr int PPW = CodeFmt<BITS>::PPW;
  constexpr int SEG = CPC / NSEG;
  constexpr int WPS = 4 / NSEG;  // words per segment
  float acc = 0.0f;
#pragma unroll
  for (int c = 0; c < CPL; ++c) {
    const int ci = l + lpr * c;
    const uint4 w = *reinterpret_cast<const uint4*>(codes_row + 16 * ci);
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int s = 0; s < NSEG; ++s) {
      __half2 hacc = __float2half2_rn(0.0f);
#pragma unroll
      for (int iw = 0; iw < WPS; ++iw) {
        const int i = s * WPS + iw;
        __half2 h[PPW];
        unpack_word<BITS>(wv[i], h);
#pragma unroll
        for (int p = 0; p < PPW; ++p) hacc = __hfma2(X.h[c][i * PPW + p], h[p], hacc);
      }
      const float d = __fmul_rn(__fadd_rn(__low2float(hacc), __high2float(hacc)), inv_scale);
      const int g = (ci * CPC + s * SEG) / gs;
      acc = __fmaf_rn(f16_to_f32(s_row[g]), d, acc);
      acc = __fmaf_rn(f16_to_f32(b_row[g]), X.xs[c][s], acc);
    }
  }
  return acc;
}

// Lanes per row for a row of `rowbytes` bytes: gcd(32, rowbytes/16).
__host__ __device__ inline int lanes_per_row(int rowbytes) {
  int chunks = rowbytes / 16;
  int l = 1;
  while (l < 32 && (chunks % (2 * l)) == 0) l *= 2;
  return l;
}

}  // namespace ynb
