// Tensor-core pieces of the quantised GEMV: the m16n8k16 MMA and the
// unpacking of MLX-affine code words into fp16 A fragments.
//
// Unpack: one LOP3 puts two codes of a word under the fp16 exponent of 1024
// (0x6400) at their bit position, so the fp16 pair holds
// (1024 + mult*q_lo, 1024 + mult*q_hi) exactly (mult = the power of two of
// the code's bit position inside its half-word). No subtraction follows: the
// activation fed to the same k-slots is x / mult (fp16), so a dot over a set
// of k-slots comes out as
//     sum(q * x) + 1024 * sum(x / mult)
// and the second term, which does not depend on the weight row, is removed
// once per group after the MMAs (see sb_apply in yn_decode.cuh).
#pragma once
#include "yn_common.cuh"

namespace ynb {

YN_DEV void mma16816(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Codes per bit width: one "unit" is 16 codes of a lane (WORDS words), giving
// 8 fp16 pairs; pair p holds unit-local codes lo(p) and hi(p) times
// 1 / inv_mult(p).
//  2-bit: one word (codes 0..15 at bits 2i): pair p = (code p, code p+8),
//         multiplier 4^p for p<5, 4^(p-5) for p>=5 (pairs 5..7 use w >> 10).
//  4-bit: two words (codes 0..7, 8..15): pairs 4i..4i+3 from word i:
//         (q0,q4) x1, (q1,q5) x16, (q2,q6) x1, (q3,q7) x16.
//  8-bit: four words (codes 4i..4i+3): pairs 2i = (q0,q2), 2i+1 = (q1,q3), x1.
template <int BITS>
struct MmaFmt;

template <>
struct MmaFmt<2> {
  static constexpr int WORDS = 1;
  YN_DEV static int lo(int p) { return p; }
  YN_DEV static int hi(int p) { return p + 8; }
  YN_DEV static float inv_mult(int p) {
    const int e = (p < 5) ? p : p - 5;
    return __int_as_float((127 - 2 * e) << 23);
  }
  // pair index of unit-local code j
  YN_DEV static int pair_of(int j) { return j & 7; }
  YN_DEV static void unpack_raw(const uint32_t* w, uint32_t (&pr)[8]) {
    const uint32_t M = 0x64006400u, a = w[0], a10 = w[0] >> 10;
    pr[0] = (a & 0x00030003u) | M;
    pr[1] = (a & 0x000C000Cu) | M;
    pr[2] = (a & 0x00300030u) | M;
    pr[3] = (a & 0x00C000C0u) | M;
    pr[4] = (a & 0x03000300u) | M;
    pr[5] = (a10 & 0x00030003u) | M;
    pr[6] = (a10 & 0x000C000Cu) | M;
    pr[7] = (a10 & 0x00300030u) | M;
  }
};

template <>
struct MmaFmt<4> {
  static constexpr int WORDS = 2;
  YN_DEV static int lo(int p) { return (p >> 2) * 8 + (p & 3); }
  YN_DEV static int hi(int p) { return (p >> 2) * 8 + (p & 3) + 4; }
  YN_DEV static float inv_mult(int p) { return (p & 1) ? 0.0625f : 1.0f; }
  YN_DEV static int pair_of(int j) { return (j >> 3) * 4 + (j & 3); }
  YN_DEV static void unpack_raw(const uint32_t* w, uint32_t (&pr)[8]) {
    const uint32_t M = 0x64006400u;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t a = w[i], a8 = w[i] >> 8;
      pr[4 * i + 0] = (a & 0x000F000Fu) | M;
      pr[4 * i + 1] = (a & 0x00F000F0u) | M;
      pr[4 * i + 2] = (a8 & 0x000F000Fu) | M;
      pr[4 * i + 3] = (a8 & 0x00F000F0u) | M;
    }
  }
};

template <>
struct MmaFmt<8> {
  static constexpr int WORDS = 4;
  YN_DEV static int lo(int p) { return (p >> 1) * 4 + (p & 1); }
  YN_DEV static int hi(int p) { return (p >> 1) * 4 + (p & 1) + 2; }
  YN_DEV static float inv_mult(int) { return 1.0f; }
  YN_DEV static int pair_of(int j) { return (j >> 2) * 2 + (j & 1); }
  YN_DEV static void unpack_raw(const uint32_t* w, uint32_t (&pr)[8]) {
    const uint32_t M = 0x64006400u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      pr[2 * i] = (w[i] & 0x00FF00FFu) | M;
      pr[2 * i + 1] = ((w[i] >> 8) & 0x00FF00FFu) | M;
    }
  }
};

}  // namespace ynb
