// Tensor-core GEMV engine for MLX-affine quantised rows (bs1..small T).
//
// A warp computes dot products of 16 weight rows with one activation vector
// over a range of 64-code blocks with mma.sync m16n8k16 (f16 x f16 -> f32):
//   A (16 rows x 16 k) = integer codes, unpacked in registers without any
//     conversion instruction: one LOP3 puts two codes under the fp16 exponent
//     of 1024 (0x6400) at their bit position, one HSUB2 removes the 1024 so
//     the pair holds (mult*q_lo, mult*q_hi) exactly;
//   B (16 k x 8 n) = the activation pairs divided by the same power-of-two
//     multiplier (all 8 columns equal), pre-scaled by a power of two so
//     max|x| sits in [64, 128);
//   D (16 x 8 f32) = per-row partial dot of one block (columns identical).
// Per block and row the group scale and bias are applied in fp32:
//   acc += scale * D / x_scale + bias * sum(x over the block's codes).
// Lane (g = lane/4, c = lane%4) owns rows g and g+8 of the tile and codes
// [16c, 16c+16) of every block; the pair p (0..7) of those 16 codes feeds
// MMA p/2 at k-slots 2c..2c+1 (p even) or 2c+8..2c+9 (p odd).
// Rows live in shared memory with a stride of (row bytes + 16) so that the
// eight rows of a fragment fall in different banks.
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

YN_DEV uint32_t h2_sub_1024(uint32_t u) {
  const __half2 off = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
  __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&u), off);
  return *reinterpret_cast<uint32_t*>(&r);
}

// 16-byte asynchronous global -> shared copy (LSU path; used where rows are
// placed at a padded stride that a bulk copy cannot produce).
YN_DEV void cp_async16(void* dst_smem, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
YN_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
YN_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Codes per bit width: a lane's 16 codes of a block and their 8 fp16 pairs.
//  2-bit: one word w (codes 0..15 at bits 2i): pair p = (code p, code p+8),
//         multiplier 4^p for p<5, 4^(p-5) for p>=5.
//  4-bit: two words (codes 0..7, 8..15): pairs 0..3 from word 0, 4..7 from
//         word 1, each word (q0,q4)x1, (q1,q5)x16, (q2,q6)x1, (q3,q7)x16.
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
  YN_DEV static void unpack(const uint32_t* w, uint32_t (&pr)[8]) {
    const uint32_t M = 0x64006400u, a = w[0], a10 = w[0] >> 10;
    pr[0] = h2_sub_1024((a & 0x00030003u) | M);
    pr[1] = h2_sub_1024((a & 0x000C000Cu) | M);
    pr[2] = h2_sub_1024((a & 0x00300030u) | M);
    pr[3] = h2_sub_1024((a & 0x00C000C0u) | M);
    pr[4] = h2_sub_1024((a & 0x03000300u) | M);
    pr[5] = h2_sub_1024((a10 & 0x00030003u) | M);
    pr[6] = h2_sub_1024((a10 & 0x000C000Cu) | M);
    pr[7] = h2_sub_1024((a10 & 0x00300030u) | M);
  }
};

template <>
struct MmaFmt<4> {
  static constexpr int WORDS = 2;
  YN_DEV static int lo(int p) { return (p >> 2) * 8 + (p & 3); }
  YN_DEV static int hi(int p) { return (p >> 2) * 8 + (p & 3) + 4; }
  YN_DEV static float inv_mult(int p) { return (p & 1) ? 0.0625f : 1.0f; }
  YN_DEV static void unpack(const uint32_t* w, uint32_t (&pr)[8]) {
    const uint32_t M = 0x64006400u;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t a = w[i], a8 = w[i] >> 8;
      pr[4 * i + 0] = h2_sub_1024((a & 0x000F000Fu) | M);
      pr[4 * i + 1] = h2_sub_1024((a & 0x00F000F0u) | M);
      pr[4 * i + 2] = h2_sub_1024((a8 & 0x000F000Fu) | M);
      pr[4 * i + 3] = h2_sub_1024((a8 & 0x00F000F0u) | M);
    }
  }
};

template <>
struct MmaFmt<8> {
  static constexpr int WORDS = 4;
  YN_DEV static int lo(int p) { return (p >> 1) * 4 + (p & 1); }
  YN_DEV static int hi(int p) { return (p >> 1) * 4 + (p & 1) + 2; }
  YN_DEV static float inv_mult(int) { return 1.0f; }
  YN_DEV static void unpack(const uint32_t* w, uint32_t (&pr)[8]) {
    const uint32_t M = 0x64006400u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      pr[2 * i] = h2_sub_1024((w[i] & 0x00FF00FFu) | M);
      pr[2 * i + 1] = h2_sub_1024(((w[i] >> 8) & 0x00FF00FFu) | M);
    }
  }
};

// Activation fragments of one block for lane c: 8 half2 pairs (as uint32)
// and the true sums of x over the block's two 32-code halves.
struct XBlock {
  uint32_t b[8];
  float xs_lo, xs_hi;   // sums over codes [0,32) and [32,64) of the block
};

// Build lane c's fragment of block `blk` (codes 64*blk ..) from a bf16 vector
// in shared memory; the two half sums are full-block sums shared by all lanes.
template <int BITS>
YN_DEV void build_xblock(XBlock& X, const uint16_t* x, int blk, float scale, int c) {
  const int base = blk * 64 + 16 * c;
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    const float m = __fmul_rn(scale, MmaFmt<BITS>::inv_mult(p));
    const float a = __fmul_rn(bf16_to_f32(x[base + MmaFmt<BITS>::lo(p)]), m);
    const float b = __fmul_rn(bf16_to_f32(x[base + MmaFmt<BITS>::hi(p)]), m);
    __half2 h = __floats2half2_rn(a, b);
    X.b[p] = *reinterpret_cast<uint32_t*>(&h);
  }
  float s = 0.0f;
#pragma unroll
  for (int e = 0; e < 16; ++e) s = __fadd_rn(s, bf16_to_f32(x[base + e]));
  // lanes c=0,1 hold the first half, c=2,3 the second: combine with shuffles
  const float s1 = __shfl_xor_sync(0xffffffffu, s, 1);
  const float s01 = __fadd_rn(s, s1);                      // (c0+c1) or (c2+c3)
  const float s23 = __shfl_xor_sync(0xffffffffu, s01, 2);
  X.xs_lo = (c < 2) ? s01 : s23;
  X.xs_hi = (c < 2) ? s23 : s01;
}

// Load one block's codes for rows g and g+8 of a tile (row pointers in
// shared memory, may be null for padding rows).
template <int BITS>
YN_DEV void load_codes(const uint8_t* row_g, const uint8_t* row_g8, int blk, int c, uint32_t (&wg)[4],
                       uint32_t (&wg8)[4]) {
  constexpr int W = MmaFmt<BITS>::WORDS;
  const int off = blk * 8 * BITS + c * 4 * W;  // a block is 8*BITS bytes; a lane 4*W of them
  if (W == 1) {
    wg[0] = row_g ? *reinterpret_cast<const uint32_t*>(row_g + off) : 0u;
    wg8[0] = row_g8 ? *reinterpret_cast<const uint32_t*>(row_g8 + off) : 0u;
  } else if (W == 2) {
    uint2 a = row_g ? *reinterpret_cast<const uint2*>(row_g + off) : make_uint2(0, 0);
    uint2 b = row_g8 ? *reinterpret_cast<const uint2*>(row_g8 + off) : make_uint2(0, 0);
    wg[0] = a.x; wg[1] = a.y; wg8[0] = b.x; wg8[1] = b.y;
  } else {
    uint4 a = row_g ? *reinterpret_cast<const uint4*>(row_g + off) : make_uint4(0, 0, 0, 0);
    uint4 b = row_g8 ? *reinterpret_cast<const uint4*>(row_g8 + off) : make_uint4(0, 0, 0, 0);
    wg[0] = a.x; wg[1] = a.y; wg[2] = a.z; wg[3] = a.w;
    wg8[0] = b.x; wg8[1] = b.y; wg8[2] = b.z; wg8[3] = b.w;
  }
}

// One block of one tile: returns the raw block dots of rows g and g+8 (f32,
// scaled by x_scale), for NSEG=1 (one scale group covers the block) or
// NSEG=2 (two 32-code groups: d_lo/d_hi separately).
template <int BITS, int NSEG>
YN_DEV void mma_block(const uint32_t (&wg)[4], const uint32_t (&wg8)[4], const XBlock& X, int c, float (&dg)[2],
                      float (&dg8)[2]) {
  uint32_t pg[8], pg8[8];
  MmaFmt<BITS>::unpack(wg, pg);
  MmaFmt<BITS>::unpack(wg8, pg8);
  if (NSEG == 1) {
    float d[4][4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      d[m][0] = d[m][1] = d[m][2] = d[m][3] = 0.f;
      const uint32_t a[4] = {pg[2 * m], pg8[2 * m], pg[2 * m + 1], pg8[2 * m + 1]};
      const uint32_t b[2] = {X.b[2 * m], X.b[2 * m + 1]};
      mma16816(d[m], a, b);
    }
    dg[0] = __fadd_rn(__fadd_rn(d[0][0], d[1][0]), __fadd_rn(d[2][0], d[3][0]));
    dg8[0] = __fadd_rn(__fadd_rn(d[0][2], d[1][2]), __fadd_rn(d[2][2], d[3][2]));
  } else {
    // lanes c<2 hold codes 0..31 (first group), c>=2 codes 32..63 (second)
    float dl[4][4], dh[4][4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      dl[m][0] = dl[m][1] = dl[m][2] = dl[m][3] = 0.f;
      dh[m][0] = dh[m][1] = dh[m][2] = dh[m][3] = 0.f;
      const uint32_t a[4] = {pg[2 * m], pg8[2 * m], pg[2 * m + 1], pg8[2 * m + 1]};
      const uint32_t blo[2] = {c < 2 ? X.b[2 * m] : 0u, c < 2 ? X.b[2 * m + 1] : 0u};
      const uint32_t bhi[2] = {c >= 2 ? X.b[2 * m] : 0u, c >= 2 ? X.b[2 * m + 1] : 0u};
      mma16816(dl[m], a, blo);
      mma16816(dh[m], a, bhi);
    }
    dg[0] = __fadd_rn(__fadd_rn(dl[0][0], dl[1][0]), __fadd_rn(dl[2][0], dl[3][0]));
    dg[1] = __fadd_rn(__fadd_rn(dh[0][0], dh[1][0]), __fadd_rn(dh[2][0], dh[3][0]));
    dg8[0] = __fadd_rn(__fadd_rn(dl[0][2], dl[1][2]), __fadd_rn(dl[2][2], dl[3][2]));
    dg8[1] = __fadd_rn(__fadd_rn(dh[0][2], dh[1][2]), __fadd_rn(dh[2][2], dh[3][2]));
  }
}

}  // namespace ynb
