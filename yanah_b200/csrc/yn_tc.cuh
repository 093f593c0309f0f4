// Grouped expert GEMM on the 5th-generation tensor cores (tcgen05) for
// many rows per expert: prompt prefill (sweep.py:80-138, the prompt pass of
// mlx_backend.py:421-433 `moe` with `_gather_sort`).
//
// One CTA computes one tile D[m][n] = sum_k W[m][k] * X[n][k]:
//  * A = 128 weight rows of one expert, dequantised from MLX 4-bit g64 codes
//    by the CTA's producer warps (TC_PW / 4 threads per tile row): for gate/up
//    the rows interleave gate unit u (row 2i) and up unit u (row 2i + 1) for
//    64 units, so SwiGLU fuses into the epilogue; for down they are 128
//    output rows;
//  * B = up to 256 rows of this expert's tokens (prefill x in fp16, or the
//    SwiGLU activations in bf16 for the down projection, whose weights are
//    then dequantised to bf16), copied by TMA;
//  * both operands are K-major in the 128-byte swizzled layout (row r of an
//    8-row atom at r * 128 bytes, 16-byte chunk c at (c ^ r) * 16); K moves
//    in stages of 64 codes = one quantisation group, 4 stages in flight;
//  * one thread issues tcgen05.mma (M 128, N = tokens rounded up to 16,
//    K 16 x 4 per stage) into a TMEM accumulator and commits each stage to
//    its mbarrier, which frees the stage's buffers for the producers;
//  * the epilogue reads TMEM with tcgen05.ld (warp w: lanes 32(w % 4)..+31).
//
// The codes of a word unpack into fp16 pairs (q0,q4), (q1,q5), (q2,q6),
// (q3,q7) (one LOP3 per pair, yn_mma.cuh), so the K order inside each block of
// 8 is permuted; the activations are stored in the same permuted order
// ("K-permuted": element 8j + p at 8j + 2p for p < 4, at 8j + 2(p-4) + 1 for
// p >= 4), which leaves every dot product unchanged.
//
// Warp-specialised and persistent: producer warps, an MMA warp and epilogue
// warps hand stages and accumulators to each other through mbarriers (see
// k_tc_experts). Every wait is bounded; on timeout the error word is set,
// each role leaves its loop, the MMA warp waits (bounded) for its last
// commit, and TMEM is released.
#pragma once
#include <cuda.h>

#include "yn_common.cuh"
#include "yn_moe.cuh"
#include "yn_mma.cuh"

namespace ynb {

constexpr int TC_THREADS = 128;
constexpr int TC_S = 4;          // pipeline stages
constexpr int TC_M = 128;        // weight rows per tile
constexpr int TC_NMAX = 256;     // token rows per tile
constexpr int TC_A_BYTES = TC_M * 128;       // one stage of A: 128 rows x 64 fp16
constexpr int TC_B_BYTES = TC_NMAX * 128;    // one stage of B: 256 rows x 64 fp16
constexpr int TC_C_BYTES = TC_M * 32;        // one stage of staged codes: 128 rows x 32 bytes
constexpr int TC_CR = 8;                     // code ring slots
constexpr int TC_PC = 6;                     // stages whose code words are in flight ahead of the dequantiser

struct TcTile {
  int e;       // expert
  int p0;      // first pair of the tile (pairs of one expert are contiguous)
  int n;       // pairs in the tile (1..256)
  int u0;      // gate/up: first unit (64 per tile); down: first output row (128 per tile)
};

// Tensor maps of the B rows (rows of the batch in pair order, 64-element x
// box-row boxes, 128-byte swizzle): box heights 16, 32, 64, 128, 256.
constexpr int TC_NMAPS = 5;
struct TcMaps {
  CUtensorMap m[TC_NMAPS];
};

struct TcArgs {
  const TcTile* tiles;
  int n_tiles;                 // capacity of `tiles` (grid size)
  const int* n_tiles_dev;      // tiles actually planned (device), or null for n_tiles
  // B rows (K-permuted, by pair: gate/up fp16 x, down bf16 SwiGLU activations) come through the tensor maps
  const uint8_t* base;         // expert arena
  long long stride;
  const int32_t* slot_of;      // expert -> slot or null (slot = expert)
  int n_slots;
  RecGeom rg;
  int H, I;
  uint16_t* act_out;           // mode 0: (P, I) bf16 K-permuted SwiGLU activations
  uint16_t* y_out;             // mode 1: (P, H) bf16 expert outputs
  int* err;
};

// One 4-bit code word -> fp16 pairs (q0,q4) x1, (q1,q5) x16, (q2,q6) x1,
// (q3,q7) x16, each value 1024 + mult * q exactly.
YN_DEV void tc_unpack4(uint32_t w, uint32_t (&pr)[4]) {
  const uint32_t M = 0x64006400u, a8 = w >> 8;
  pr[0] = (w & 0x000F000Fu) | M;
  pr[1] = (w & 0x00F000F0u) | M;
  pr[2] = (a8 & 0x000F000Fu) | M;
  pr[3] = (a8 & 0x00F000F0u) | M;
}

YN_DEV int kperm(int k) { const int p = k & 7; return (k & ~7) | (p < 4 ? 2 * p : 2 * (p - 4) + 1); }

// K order of the A tile for BITS-bit codes: inside every unit of 16 codes,
// pair p of the unpack (MmaFmt<BITS>: codes lo(p), hi(p)) sits at positions
// 2p, 2p+1. For 4-bit this is kperm above.
template <int BITS>
YN_DEV int kperm_fmt(int k) {
  const int j = k & 15, p = MmaFmt<BITS>::pair_of(j);
  return (k & ~15) | (2 * p + (j == MmaFmt<BITS>::hi(p) ? 1 : 0));
}

YN_DEV uint64_t tc_desc(uint32_t smem_addr) {
  // K-major, 128-byte swizzle: start address (>>4), leading offset 1 (unused
  // for swizzled K-major), stride offset 1024 bytes between 8-row atoms,
  // version 1, layout type 2 (SWIZZLE_128B)
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

YN_DEV uint32_t tc_idesc(int n, bool bf16) {
  // f32 accumulate (bits 4-5 = 1), A and B fp16 (format 0) or bf16 (format 1),
  // both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28
  const uint32_t f = bf16 ? 1u : 0u;
  return (1u << 4) | (f << 7) | (f << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(TC_M >> 4) << 24);
}

YN_DEV void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

YN_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

YN_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
YN_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
YN_DEV void tc_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

YN_DEV void tc_cpa16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
YN_DEV void tc_cpa8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
YN_DEV void tc_cpa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
YN_DEV void tc_cpa_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Bounded wait on an mbarrier phase by every thread; block-uniform result.
YN_DEV bool tc_wait(uint64_t* bar, uint32_t parity, int* err) {
  return mbar_wait_block(bar, parity, err);
}

// Producer-side dequantisation of NW code words (8 codes each) of one 64-code
// stage of a weight row, words i0 .. i0+NW-1 of the stage, into the swizzled
// A tile (fp16 for MODE 0, bf16 for MODE 1). t: the tile row (swizzle phase).
// `codes`: the thread's first 16-byte piece of code words; piece v at codes + v * PS.
template <int MODE, int NW, int PS>
YN_DEV void tc_dequant_row(const uint8_t* codes, uint16_t sc_bits, uint16_t bi_bits, uint8_t* Arow, int t, int i0) {
  uint32_t words[NW];
#pragma unroll
  for (int v = 0; v < NW / 4; ++v) {
    const uint4 c = *reinterpret_cast<const uint4*>(codes + v * PS);
    words[4 * v] = c.x;
    words[4 * v + 1] = c.y;
    words[4 * v + 2] = c.z;
    words[4 * v + 3] = c.w;
  }
  const __half sc = __ushort_as_half(sc_bits), bi = __ushort_as_half(bi_bits);
  const __half2 k1024 = __float2half2_rn(1024.0f);
  if constexpr (MODE == 0) {  // w = fp16(s * q + b): one HFMA2 per pair
    const __half2 s1 = __halves2half2(sc, sc);
    const __half sc16 = __float2half_rn(__fmul_rn(__half2float(sc), 0.0625f));
    const __half2 s16 = __halves2half2(sc16, sc16);
    const __half2 b2 = __halves2half2(bi, bi);
#pragma unroll
    for (int i = 0; i < NW; ++i) {
      uint32_t pr[4];
      tc_unpack4(words[i], pr);
      uint32_t o[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        __half2 h = *reinterpret_cast<__half2*>(&pr[p]);
        h = __hsub2(h, k1024);
        h = __hfma2(h, (p & 1) ? s16 : s1, b2);
        o[p] = *reinterpret_cast<uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(Arow + (((i0 + i) ^ (t & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  } else {  // w = bf16(s * q + b) from an fp32 FMA
    const float s1 = __half2float(sc), s16 = __fmul_rn(s1, 0.0625f), bf = __half2float(bi);
#pragma unroll
    for (int i = 0; i < NW; ++i) {
      uint32_t pr[4];
      tc_unpack4(words[i], pr);
      uint32_t o[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        __half2 h = *reinterpret_cast<__half2*>(&pr[p]);
        h = __hsub2(h, k1024);  // mult * q, exact
        const float2 q = __half22float2(h);
        const float m = (p & 1) ? s16 : s1;
        __nv_bfloat162 w = __floats2bfloat162_rn(__fmaf_rn(q.x, m, bf), __fmaf_rn(q.y, m, bf));
        o[p] = *reinterpret_cast<uint32_t*>(&w);
      }
      *reinterpret_cast<uint4*>(Arow + (((i0 + i) ^ (t & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Generic producer dequantisation (2- and 8-bit codes; 4-bit uses
// tc_dequant_row): this thread's 32 codes of one 64-code stage of a weight row
// (two units of 16 codes, MmaFmt<BITS>::WORDS words each) into 4 chunks of
// the swizzled A tile from chunk i0. w = s * q + b as one fp32 FMA of the
// unpacked (mult * q) and s / mult (exact: a power of two), rounded to fp16
// (MODE 0) or bf16 (MODE 1). The thread's code words come in pieces of at
// most 16 bytes, piece v at codes + v * PS.
template <int MODE, int BITS, int PS>
YN_DEV void tc_dequant_gen(const uint8_t* codes, uint16_t sc_bits, uint16_t bi_bits, uint8_t* Arow, int t, int i0) {
  using F = MmaFmt<BITS>;
  constexpr int PB = 2 * F::WORDS * 4 < 16 ? 2 * F::WORDS * 4 : 16;   // piece bytes (the thread's bytes, at most 16)
  uint32_t words[2 * F::WORDS];
#pragma unroll
  for (int v = 0; v < 2 * F::WORDS; v += 2) {
    const uint2 c = *reinterpret_cast<const uint2*>(codes + (4 * v / PB) * PS + (4 * v) % PB);
    words[v] = c.x;
    words[v + 1] = c.y;
  }
  const float s = f16_to_f32(sc_bits), b = f16_to_f32(bi_bits);
  const __half2 k1024 = __float2half2_rn(1024.0f);
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    uint32_t pr[8];
    F::unpack_raw(words + u * F::WORDS, pr);
    uint32_t o[8];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      __half2 h = *reinterpret_cast<__half2*>(&pr[p]);
      h = __hsub2(h, k1024);  // mult * q, exact
      const float2 q = __half22float2(h);
      const float m = __fmul_rn(s, F::inv_mult(p));
      const float w0 = __fmaf_rn(q.x, m, b), w1 = __fmaf_rn(q.y, m, b);
      if (MODE == 0) {
        __half2 hw = __floats2half2_rn(w0, w1);
        o[p] = *reinterpret_cast<uint32_t*>(&hw);
      } else {
        __nv_bfloat162 bw = __floats2bfloat162_rn(w0, w1);
        o[p] = *reinterpret_cast<uint32_t*>(&bw);
      }
    }
#pragma unroll
    for (int c = 0; c < 2; ++c)
      *reinterpret_cast<uint4*>(Arow + (((i0 + 2 * u + c) ^ (t & 7)) << 4)) =
          make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
  }
}

// SwiGLU with the same bf16 rounding points as swiglu_bf16, but the sigmoid
// from the hardware exponential and an approximate divide: these outputs are
// held to the bf16 output tolerance, not to bit equality, and the epilogue
// evaluates one per (row, unit).
YN_DEV float swiglu_bf16_fast(float g, float u) {
  const float sg = bf16r(__fdividef(1.0f, 1.0f + __expf(-g)));
  return bf16r(__fmul_rn(bf16r(__fmul_rn(g, sg)), u));
}

YN_DEV void tc_tma_rows(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

YN_DEV void mbar_arrive1(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Warp-specialised persistent form. 32 * (TC_PW + TC_EPW + 2) threads: warps
// 0..TC_PW-1 produce A (TC_PW / 4 threads per tile row, each dequantising
// 8 / (TC_PW / 4) code words of the row's stage), the next TC_EPW warps drain
// the accumulator (epilogue warp e reads TMEM lanes 32(e % 4)..+31, 32-column
// chunks e / 4, e / 4 + TC_EPW / 4, ...), then the MMA warp and the loader
// warp (one TMA copy of the B rows per stage). A stage's
// A and B are both written as soon as the MMA that last read the stage has
// committed, so the whole ring is in flight. Stage ring: full[s]
// (32 * TC_PW producer arrivals + the loader's expect_tx), empty[s] (MMA commit);
// accumulator ring of 2 x 256 TMEM columns: acc_full[b] (MMA commit),
// acc_empty[b] (one arrival per epilogue thread). The CTAs walk the planned tiles with
// stride gridDim.x, so one tile's epilogue overlaps the next tile's main loop.
// MODE 0: gate/up + SwiGLU, fp16 operands (normalised rows are small);
// MODE 1: down, bf16 operands (SwiGLU activations have bf16's range, as the
// reference's bf16 arrays do; fp16 would overflow on them).
#ifndef TC_PW
#define TC_PW 8
#endif
static_assert(TC_PW == 4 || TC_PW == 8, "producer warps: 4 or 8");
constexpr int TC_PT = 32 * TC_PW;            // producer threads
constexpr int TC_NH = TC_PW / 4;             // producer threads per tile row
constexpr int TC_NW = 8 / TC_NH;             // code words per producer thread and stage
#ifndef TC_EPW
#define TC_EPW 8
#endif
static_assert(TC_EPW == 4 || TC_EPW == 8, "epilogue warps: 4 or 8");
// Code staging per format: bytes of one row per 64-code stage, bytes per
// producer thread, ring slots (fewer for 8-bit, whose slots are twice as
// large) and stages in flight ahead of the dequantiser.
template <int BITS>
struct TcFmt {
  static constexpr int ROWB = 8 * BITS;
  static constexpr int TB = ROWB / TC_NH;
  static constexpr int CR = BITS == 8 ? 4 : TC_CR;
  static constexpr int PC = CR - 2;
  static constexpr int SLOT = TC_M * ROWB;
  // A slot holds each producer thread's TB bytes as pieces of min(TB, 16) bytes laid out
  // [part h][piece][tile row t]: the 32 threads of a warp (consecutive rows, one part) touch
  // consecutive pieces, so their copies and reads are free of bank conflicts.
  static constexpr int PB = TB < 16 ? TB : 16;   // piece bytes
  static constexpr int PS = TC_M * PB;            // bytes between a thread's pieces
  YN_DEV static uint8_t* at(uint8_t* ring, int slot, int t, int h) {
    return ring + slot * SLOT + h * (TC_M * TB) + t * PB;
  }
};
constexpr int TC_EW = TC_PW;                 // first epilogue warp (a multiple of 4: warp % 4 = TMEM lane quadrant)
constexpr int TC_MW = TC_PW + TC_EPW;        // the MMA warp
constexpr int TC_LW = TC_MW + 1;             // the B-row loader warp
constexpr int TCW_THREADS = 32 * (TC_MW + 2);

template <int MODE, int BITS, int GS>
__global__ void __launch_bounds__(TCW_THREADS, 1) k_tc_experts(const TcArgs a, const __grid_constant__ TcMaps maps) {
  using FT = TcFmt<BITS>;
  constexpr int GPS = 64 / GS;   // quantisation groups per 64-code stage
  constexpr int SPB = 8 / GPS;   // stages per 8-group block of scales
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + (((smem_u32(smem_raw) + 1023u) & ~1023u) - smem_u32(smem_raw));
  uint8_t* Abuf = smem;
  uint8_t* Bbuf = Abuf + TC_S * TC_A_BYTES;
  uint8_t* Cbuf = Bbuf + TC_S * TC_B_BYTES;
  const int Kd = MODE == 0 ? a.H : a.I;
  const int NG = Kd / GS, NK = Kd / 64;
  uint64_t* full = reinterpret_cast<uint64_t*>(Cbuf + FT::CR * FT::SLOT);
  uint64_t* empty = full + TC_S;
  uint64_t* acc_full = empty + TC_S;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_tiles = a.n_tiles_dev ? min(a.n_tiles, *a.n_tiles_dev) : a.n_tiles;
  if (tid == 0) {
    for (int s = 0; s < TC_S; ++s) {
      mbar_init(&full[s], TC_PT + 1);  // dequantising threads + the TMA transaction's expect_tx
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 32 * TC_EPW);
    }
    fence_mbar_init();
  }
  if (warp == TC_MW) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp < TC_PW) {
    // ------------------------------------------------------------ producers
    const int t = tid & (TC_M - 1), h = tid / TC_M;  // tile row, part of the row's stage
    // Where this thread's row of a tile lives: its code words and its scale / bias blocks.
    struct RowSrc {
      const uint8_t* w;
      const uint4* s;
      const uint4* b;
      bool good;
    };
    auto row_src = [&](const TcTile& tl, int slot) -> RowSrc {
      const bool good = tl.n >= 1 && tl.n <= TC_NMAX && slot >= 0 && slot < a.n_slots;
      const uint8_t* rec = a.base + (size_t)(good ? slot : 0) * (size_t)a.stride;
      const bool up = (MODE == 0) && (t & 1);
      const int wrow = MODE == 0 ? tl.u0 + (t >> 1) : tl.u0 + t;
      const int pw = MODE == 0 ? (up ? 3 : 0) : 6;
      return {rec + a.rg.off[pw] + (size_t)wrow * (Kd * BITS / 8),
              reinterpret_cast<const uint4*>(rec + a.rg.off[pw + 1] + (size_t)wrow * NG * 2),
              reinterpret_cast<const uint4*>(rec + a.rg.off[pw + 2] + (size_t)wrow * NG * 2), good};
    };
    // The next tile is prepared while the current one runs: its descriptor at
    // the start, its slot one block later, its first scale block and its first
    // TC_PC stages of code words in the last stages, so a tile starts without
    // a chain of dependent global loads.
    int g = 0;  // stages produced by this CTA so far
    TcTile ntl = {0, 0, 0, 0};
    int nslot = -1;
    if ((int)blockIdx.x < n_tiles) {
      ntl = a.tiles[blockIdx.x];
      nslot = a.slot_of ? a.slot_of[ntl.e] : ntl.e;
    }
    RowSrc nsrc = row_src(ntl, nslot);
    uint4 ns8 = make_uint4(0, 0, 0, 0), nb8 = ns8;
    if (nsrc.good) {
      ns8 = nsrc.s[0];
      nb8 = nsrc.b[0];
    }
    // this thread's code words of stage kc of a tile into its slot of the code
    // ring (TC_CR slots, read back only by this thread); one group per stage
    auto issue_codes = [&](const RowSrc& r, int ring, int kc) {
      if (r.good) {
        uint8_t* cd = FT::at(Cbuf, ring % FT::CR, t, h);
        const uint8_t* sw = r.w + FT::ROWB * kc + h * FT::TB;
        if (FT::TB == 8) {
          tc_cpa8(cd, sw);
        } else {
#pragma unroll
          for (int v = 0; v < FT::TB / 16; ++v) tc_cpa16(cd + FT::PS * v, sw + 16 * v);
        }
      }
      tc_cpa_commit();
    };
    for (int kc = 0; kc < FT::PC; ++kc) issue_codes(nsrc, kc, kc);  // NK >= 8 > PC
    for (int ti = blockIdx.x; ti < n_tiles && ok; ti += gridDim.x) {
      const RowSrc src = nsrc;
      const bool good = src.good;
      if (!good && t == 0) raise_error(a.err, YN_ERR_BAD_SLOT);
      const int tn = ti + gridDim.x;
      const bool more = tn < n_tiles;
      if (more) ntl = a.tiles[tn];
      // scales and biases of this row in blocks of 8 groups (16-byte loads, one block ahead)
      uint4 s8 = make_uint4(0, 0, 0, 0), b8 = s8, s8n = ns8, b8n = nb8;
      for (int kc0 = 0; kc0 < NK && ok; kc0 += SPB) {
        s8 = s8n;
        b8 = b8n;
        if (good && kc0 + SPB < NK) {
          s8n = src.s[(kc0 + SPB) / SPB];
          b8n = src.b[(kc0 + SPB) / SPB];
        }
        // the next tile's code words are issued from stage NK - PC on: its sources are known from the
        // block holding that stage (its slot one block earlier when there is one)
        const int ns_blk = ((NK - FT::PC) / SPB) * SPB, slot_blk = ns_blk >= SPB ? SPB : 0;
        if (more && kc0 == slot_blk) nslot = a.slot_of ? a.slot_of[ntl.e] : ntl.e;
        if (more && kc0 == ns_blk) {  // the next tile's sources and first scale block
          nsrc = row_src(ntl, nslot);
          if (nsrc.good) {
            ns8 = nsrc.s[0];
            nb8 = nsrc.b[0];
          }
        }
#pragma unroll
        for (int jj = 0; jj < SPB; ++jj) {
          const int kc = kc0 + jj;
          const int s = (g + kc) % TC_S;
          if (kc + FT::PC < NK) issue_codes(src, g + kc + FT::PC, kc + FT::PC);
          else if (more) issue_codes(nsrc, g + kc + FT::PC, kc + FT::PC - NK);
          else tc_cpa_commit();  // keep one group per stage
          // the stage's A buffer is free once the MMA of TC_S stages back has committed
          if (g + kc >= TC_S) ok = mbar_wait_bounded(&empty[s], (((g + kc) / TC_S) - 1) & 1, a.err);
          tc_cpa_wait<FT::PC>();  // this stage's code words have landed
          if (!ok) break;
          if (good) {
            const int gi = jj * GPS + (GPS == 2 ? h : 0);   // this thread's group inside the 8-group block
            const uint32_t sw = gi < 2 ? s8.x : gi < 4 ? s8.y : gi < 6 ? s8.z : s8.w;
            const uint32_t bw = gi < 2 ? b8.x : gi < 4 ? b8.y : gi < 6 ? b8.z : b8.w;
            const uint8_t* cd = FT::at(Cbuf, (g + kc) % FT::CR, t, h);
            uint8_t* arow = Abuf + s * TC_A_BYTES + (t >> 3) * 1024 + (t & 7) * 128;
            const uint16_t sb16 = (uint16_t)(sw >> (16 * (gi & 1))), bb16 = (uint16_t)(bw >> (16 * (gi & 1)));
            if (BITS == 4) tc_dequant_row<MODE, TC_NW, FT::PS>(cd, sb16, bb16, arow, t, h * TC_NW);
            else tc_dequant_gen<MODE, BITS, FT::PS>(cd, sb16, bb16, arow, t, 4 * h);
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          mbar_arrive1(&full[s]);
        }
      }
      g += NK;
    }
    tc_cpa_wait<0>();
  } else if (warp < TC_MW) {
    // ------------------------------------------------------------ epilogue
    const int q = (warp - TC_EW) & 3, m = 32 * q + lane;  // tile row of this thread
    const int hc = (warp - TC_EW) >> 2;                    // first 32-column chunk of this warp
    int j = 0;
    for (int ti = blockIdx.x; ti < n_tiles && ok; ti += gridDim.x, ++j) {
      const TcTile tl = a.tiles[ti];
      const int n = tl.n, nmma = (n + 15) & ~15, b = j & 1;
      ok = mbar_wait_bounded(&acc_full[b], (j >> 1) & 1, a.err);
      ok = __all_sync(0xffffffffu, ok) != 0;
      if (!ok) break;
      tc_fence_after();
      const uint32_t base = tmem + (uint32_t)(b * 256) + ((uint32_t)(32 * q) << 16);
      const bool good = n >= 1 && n <= TC_NMAX;
      for (int c0 = 32 * hc; c0 < nmma; c0 += 32 * (TC_EPW / 4)) {
        float v[32];
        tc_ld32(base + (uint32_t)c0, v);
        if (!good) continue;
        if (MODE == 0) {
          // lanes 2i (gate of unit u) and 2i+1 (up of unit u) share the columns:
          // of each column pair the gate lane takes the even column, the up lane
          // the odd one, after one exchange
          const int ku = kperm_fmt<BITS>(tl.u0 + (m >> 1));
          const bool is_up = m & 1;
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float recv = __shfl_xor_sync(0xffffffffu, is_up ? v[2 * k] : v[2 * k + 1], 1);
            const int col = c0 + 2 * k + (is_up ? 1 : 0);
            const float gv = bf16r(is_up ? recv : v[2 * k]), uv = bf16r(is_up ? v[2 * k + 1] : recv);
            if (col < n) a.act_out[(size_t)(tl.p0 + col) * a.I + ku] = f32_to_bf16(swiglu_bf16_fast(gv, uv));
          }
        } else {
          const int row = tl.u0 + m;
#pragma unroll
          for (int jj = 0; jj < 32; ++jj)
            if (c0 + jj < n) a.y_out[(size_t)(tl.p0 + c0 + jj) * a.H + row] = f32_to_bf16(v[jj]);
        }
      }
      tc_fence_before();
      mbar_arrive1(&acc_empty[b]);
    }
  } else if (warp == TC_MW) {
    // ------------------------------------------------------------------ MMA
    int g = 0, j = 0;
    for (int ti = blockIdx.x; ti < n_tiles && ok; ti += gridDim.x, ++j) {
      const TcTile tl = a.tiles[ti];
      const int nmma = ((tl.n >= 1 && tl.n <= TC_NMAX ? tl.n : 16) + 15) & ~15, b = j & 1;
      if (j >= 2) ok = mbar_wait_bounded(&acc_empty[b], ((j >> 1) - 1) & 1, a.err);
      ok = __all_sync(0xffffffffu, ok) != 0;
      if (!ok) break;
      tc_fence_after();
      const uint32_t idesc = tc_idesc(nmma, MODE == 1), dcol = tmem + (uint32_t)(b * 256);
      for (int kc = 0; kc < NK && ok; ++kc, ++g) {
        const int s = g % TC_S;
        ok = mbar_wait_bounded(&full[s], (g / TC_S) & 1, a.err);
        ok = __all_sync(0xffffffffu, ok) != 0;
        if (!ok) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t abase = smem_u32(Abuf + s * TC_A_BYTES), bbase = smem_u32(Bbuf + s * TC_B_BYTES);
#pragma unroll
          for (int k16 = 0; k16 < 4; ++k16)
            tc_mma(dcol, tc_desc(abase + 32 * k16), tc_desc(bbase + 32 * k16), idesc, (kc > 0 || k16 > 0) ? 1u : 0u);
          tc_commit(&empty[s]);
          if (kc == NK - 1) tc_commit(&acc_full[b]);
        }
        __syncwarp();
      }
    }
    // the last commits must land before TMEM is released (bounded)
    if (lane == 0 && j > 0) (void)mbar_wait_bounded(&acc_full[(j - 1) & 1], ((j - 1) >> 1) & 1, a.err);
    __syncwarp();
  } else if (warp == TC_LW) {
    // ------------------------------------------------------- B-row loader
    // one TMA copy per stage (rows past the batch read as zeros), as soon as
    // the stage's buffers are free
    int g = 0;
    for (int ti = blockIdx.x; ti < n_tiles && ok; ti += gridDim.x) {
      const TcTile tl = a.tiles[ti];
      const int n = tl.n;
      const int slot = a.slot_of ? a.slot_of[tl.e] : tl.e;
      const bool good = n >= 1 && n <= TC_NMAX && slot >= 0 && slot < a.n_slots;
      // B box: the smallest map whose height covers the tile's MMA width
      const int nmma = ((good ? n : 16) + 15) & ~15;
      const int mi = nmma <= 16 ? 0 : nmma <= 32 ? 1 : nmma <= 64 ? 2 : nmma <= 128 ? 3 : 4;
      const uint32_t box_bytes = (16u << mi) * 128u;
      for (int kc = 0; kc < NK && ok; ++kc) {
        const int gg = g + kc, s = gg % TC_S;
        if (gg >= TC_S) ok = mbar_wait_bounded(&empty[s], ((gg / TC_S) - 1) & 1, a.err);
        ok = __all_sync(0xffffffffu, ok) != 0;
        if (!ok) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[s], good ? box_bytes : 0u);
          if (good) tc_tma_rows(Bbuf + s * TC_B_BYTES, &maps.m[mi], 64 * kc, tl.p0, &full[s]);
        }
        __syncwarp();
      }
      g += NK;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == TC_MW) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

}  // namespace ynb

namespace ynb {

// bf16 rows -> fp16 rows in the K-permuted order of the tensor-core path.
__global__ void k_to_f16_kperm(const uint16_t* x, long long n, int cols, uint16_t* out) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / cols;
    const int k = (int)(i - r * cols);
    out[r * cols + kperm(k)] = __half_as_ushort(__float2half_rn(bf16_to_f32(x[i])));
  }
}

// out[p] = fp16 K-permuted copy of row row_of[p] of x (bf16): one 8-element
// block (16-byte load, 16-byte store) per thread step.
__global__ void k_gather_f16_kperm(const uint16_t* x, const int32_t* row_of, long long rows, int cols, uint16_t* out) {
  const long long nb = rows * (cols / 8);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nb; i += (long long)gridDim.x * blockDim.x) {
    const long long p = i / (cols / 8);
    const int blk = (int)(i - p * (cols / 8));
    const uint4 v = reinterpret_cast<const uint4*>(x + (size_t)row_of[p] * cols)[blk];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float f[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      f[2 * e] = bf16_to_f32((uint16_t)(w[e] & 0xFFFFu));
      f[2 * e + 1] = bf16_to_f32((uint16_t)(w[e] >> 16));
    }
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // positions 2q, 2q+1 hold elements q, q+4
      __half2 h = __floats2half2_rn(f[q], f[q + 4]);
      o[q] = *reinterpret_cast<uint32_t*>(&h);
    }
    reinterpret_cast<uint4*>(out + (size_t)p * cols)[blk] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// out[p] = row (row_of ? row_of[p] : p) of x (bf16) in the K order of
// BITS-bit codes (kperm_fmt), as fp16 (F16) or bf16: one unit of 16 elements
// (two 16-byte loads and stores) per thread step.
template <int BITS, bool F16>
__global__ void k_perm_rows(const uint16_t* x, const int32_t* row_of, long long rows, int cols, uint16_t* out) {
  using F = MmaFmt<BITS>;
  const long long nu = rows * (cols / 16);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nu; i += (long long)gridDim.x * blockDim.x) {
    const long long p = i / (cols / 16);
    const int u = (int)(i - p * (cols / 16));
    const uint16_t* src = x + (size_t)(row_of ? row_of[p] : p) * cols + 16 * u;
    const uint4 v0 = reinterpret_cast<const uint4*>(src)[0], v1 = reinterpret_cast<const uint4*>(src)[1];
    const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    uint32_t o[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {  // output positions 2q, 2q+1: the codes of pair q
      const int lo = F::lo(q), hi = F::hi(q);
      const uint16_t a = (uint16_t)(w[lo >> 1] >> (16 * (lo & 1))), b = (uint16_t)(w[hi >> 1] >> (16 * (hi & 1)));
      if (F16) {
        __half2 h = __floats2half2_rn(bf16_to_f32(a), bf16_to_f32(b));
        o[q] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        o[q] = (uint32_t)a | ((uint32_t)b << 16);
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(out + (size_t)p * cols + 16 * u);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// out[t][c] = bf16(scale[t] * y[t][c]) (y bf16): the gated shared-expert term
// sigmoid(g) * y_shared of every row, rounded as the single-row path rounds it.
__global__ void k_scale_rows(const uint16_t* y, const float* scale, long long rows, int cols, uint16_t* out) {
  const long long n = rows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    out[i] = f32_to_bf16(__fmul_rn(scale[i / cols], bf16_to_f32(y[i])));
}

// out[t] = h_res[t] + (sum_j bf16(y[pair_of[t][j]] * w[t][j]) in column order [+ ysh[t]]),
// rounded as the single-row combine.
// The same combine with 8 columns per thread (16-byte loads and stores);
// every element's arithmetic is that of k_pairs_combine. H % 8 == 0 and
// 16-byte aligned rows.
__global__ void k_pairs_combine8(const uint16_t* y, const int32_t* pair_of, const float* w, const uint16_t* ysh,
                                 const uint16_t* h_res, int H, int K, uint16_t* out) {
  const int t = blockIdx.y, r0 = 8 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (r0 >= H) return;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
  for (int j = 0; j < K; ++j) {
    const int p = pair_of[(size_t)t * K + j];
    if (p < 0) continue;  // column outside the computed pairs (a staging group)
    const float wj = w[(size_t)t * K + j];
    const uint4 q = *reinterpret_cast<const uint4*>(y + (size_t)p * H + r0);
    const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float v = bf16_to_f32((uint16_t)(u[i >> 1] >> (16 * (i & 1))));
      acc[i] = __fadd_rn(acc[i], bf16r(__fmul_rn(v, wj)));
    }
  }
  uint32_t sh[4] = {0, 0, 0, 0}, hr[4] = {0, 0, 0, 0};
  if (ysh) {
    const uint4 q = *reinterpret_cast<const uint4*>(ysh + (size_t)t * H + r0);
    sh[0] = q.x; sh[1] = q.y; sh[2] = q.z; sh[3] = q.w;
  }
  if (h_res) {
    const uint4 q = *reinterpret_cast<const uint4*>(h_res + (size_t)t * H + r0);
    hr[0] = q.x; hr[1] = q.y; hr[2] = q.z; hr[3] = q.w;
  }
  uint32_t o4[4];
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    uint32_t pk = 0;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      float o = bf16r(acc[i + k]);
      if (ysh) o = bf16r(__fadd_rn(o, bf16_to_f32((uint16_t)(sh[i >> 1] >> (16 * k)))));
      if (h_res) o = bf16r(__fadd_rn(bf16_to_f32((uint16_t)(hr[i >> 1] >> (16 * k))), o));
      pk |= (uint32_t)f32_to_bf16(o) << (16 * k);
    }
    o4[i >> 1] = pk;
  }
  *reinterpret_cast<uint4*>(out + (size_t)t * H + r0) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
}

__global__ void k_pairs_combine(const uint16_t* y, const int32_t* pair_of, const float* w, const uint16_t* ysh,
                                const uint16_t* h_res, int H, int K, uint16_t* out) {
  const int t = blockIdx.y, r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= H) return;
  float acc = 0.0f;
  for (int j = 0; j < K; ++j) {
    const int p = pair_of[(size_t)t * K + j];
    if (p < 0) continue;  // column outside the computed pairs (a staging group)
    const float v = bf16_to_f32(y[(size_t)p * H + r]);
    acc = __fadd_rn(acc, bf16r(__fmul_rn(v, w[(size_t)t * K + j])));
  }
  float o = bf16r(acc);
  if (ysh) o = bf16r(__fadd_rn(o, bf16_to_f32(ysh[(size_t)t * H + r])));
  if (h_res) o = bf16r(__fadd_rn(bf16_to_f32(h_res[(size_t)t * H + r]), o));
  out[(size_t)t * H + r] = f32_to_bf16(o);
}

}  // namespace ynb

namespace ynb {

// Expert groups and GEMM tiles of a prefill batch, on the device (one CTA of
// 1024 threads): counts per expert, a block scan over experts (ascending id),
// pair placement (pairs of one expert contiguous; their order inside an
// expert does not change any pair's result), then per expert ceil(n / 256)
// row chunks x (I / 64) gate/up tiles and x (H / 128) down tiles.
// n_tiles[0], n_tiles[1] = gate/up and down tiles written.
constexpr int PLAN_THREADS = 1024;

struct PrefillPlanArgs {
  const int32_t* ids;  // (T, K)
  int T, K, E, H, I;
  int32_t* pair_row;   // (T * K) pair -> row
  int32_t* pair_of;    // (T * K) t * K + j -> pair
  TcTile* up;
  int max_up;
  TcTile* dn;
  int max_dn;
  int* n_tiles;        // [2]
  int* err;
};

YN_DEV int2 block_scan2(int2 v, int2* total) {
  __shared__ int2 ws[PLAN_THREADS / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int2 inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int x = __shfl_up_sync(0xffffffffu, inc.x, o), y = __shfl_up_sync(0xffffffffu, inc.y, o);
    if (lane >= o) { inc.x += x; inc.y += y; }
  }
  if (lane == 31) ws[warp] = inc;
  __syncthreads();
  int2 base = make_int2(0, 0), tot = make_int2(0, 0);
  for (int w = 0; w < PLAN_THREADS / 32; ++w) {
    const int2 q = ws[w];
    if (w < warp) { base.x += q.x; base.y += q.y; }
    tot.x += q.x; tot.y += q.y;
  }
  *total = tot;
  __syncthreads();
  return make_int2(base.x + inc.x - v.x, base.y + inc.y - v.y);
}

// Warp-aggregated increment of ctr[e]: lanes with the same e take
// consecutive values from one atomicAdd (popular experts would otherwise
// serialise one shared-memory atomic per pair). Returns this lane's value.
YN_DEV int agg_atomic_add(int* ctr, int e, bool active) {
  const unsigned act = __ballot_sync(0xffffffffu, active);
  if (!active) return 0;
  const unsigned peers = __match_any_sync(act, e);
  const int lane = threadIdx.x & 31, leader = __ffs(peers) - 1;
  int base = 0;
  if (lane == leader) base = atomicAdd(&ctr[e], __popc(peers));
  base = __shfl_sync(peers, base, leader);
  return base + __popc(peers & ((1u << lane) - 1u));
}

constexpr int PLAN_MAX_CHUNKS = 1024 + 65536 / TC_NMAX;  // experts + pairs / rows per tile

__global__ void __launch_bounds__(PLAN_THREADS) k_prefill_plan(const PrefillPlanArgs a) {
  __shared__ int cnt[1024], start[1024], cursor[1024], toff[1024];
  __shared__ int chunk_e[PLAN_MAX_CHUNKS], chunk_p0[PLAN_MAX_CHUNKS], chunk_n[PLAN_MAX_CHUNKS], order[PLAN_MAX_CHUNKS];
  const int P = a.T * a.K, tid = threadIdx.x;
  for (int e = tid; e < 1024; e += PLAN_THREADS) cnt[e] = cursor[e] = 0;
  __syncthreads();
  // loop bounds rounded up to whole warps: the aggregated atomics are warp-collective
  const int Pw = (P + 31) & ~31;
  for (int i = tid; i < Pw; i += PLAN_THREADS) {
    const int e = i < P ? a.ids[i] : -1;
    const bool valid = e >= 0 && e < a.E;
    if (i < P && !valid) raise_error(a.err, YN_ERR_BAD_EXPERT);
    agg_atomic_add(cnt, valid ? e : 0, valid);
  }
  __syncthreads();
  const int c = tid < a.E ? cnt[tid] : 0;
  int2 tot;
  const int2 ex = block_scan2(make_int2(c, (c + TC_NMAX - 1) / TC_NMAX), &tot);
  if (tid < a.E) {
    start[tid] = ex.x;
    toff[tid] = ex.y;
  }
  __syncthreads();
  for (int i = tid; i < Pw; i += PLAN_THREADS) {
    const int e = i < P ? a.ids[i] : -1;
    const bool valid = e >= 0 && e < a.E;
    const int pos = agg_atomic_add(cursor, valid ? e : 0, valid);
    if (valid) {
      a.pair_row[start[e] + pos] = i / a.K;
      a.pair_of[i] = start[e] + pos;
    }
  }
  // chunks of at most TC_NMAX pairs per expert, then every tile in parallel
  if (tid < a.E && c) {
    for (int k = 0; k * TC_NMAX < c; ++k) {
      const int chunk = toff[tid] + k;
      if (chunk < PLAN_MAX_CHUNKS) {
        chunk_e[chunk] = tid;
        chunk_p0[chunk] = start[tid] + k * TC_NMAX;
        chunk_n[chunk] = min(TC_NMAX, c - k * TC_NMAX);
      }
    }
  }
  __syncthreads();
  const int UT = a.I / 64, DT = a.H / 128, nch = min(tot.y, PLAN_MAX_CHUNKS);
  // Tiles of the largest chunks first: the persistent GEMM CTAs take the
  // tiles round-robin, so descending rows per tile evens out their work. A
  // counting sort on TC_NMAX - rows (cnt / cursor / start are free again).
  for (int k = tid; k <= TC_NMAX; k += PLAN_THREADS) cnt[k] = cursor[k] = 0;
  __syncthreads();
  for (int ch = tid; ch < nch; ch += PLAN_THREADS) atomicAdd(&cnt[TC_NMAX - chunk_n[ch]], 1);
  __syncthreads();
  int2 btot;
  const int2 bex = block_scan2(make_int2(tid <= TC_NMAX ? cnt[tid] : 0, 0), &btot);
  if (tid <= TC_NMAX) start[tid] = bex.x;
  __syncthreads();
  for (int ch = tid; ch < nch; ch += PLAN_THREADS) {
    const int key = TC_NMAX - chunk_n[ch];
    order[start[key] + atomicAdd(&cursor[key], 1)] = ch;
  }
  __syncthreads();
  for (int q = tid; q < nch * UT && q < a.max_up; q += PLAN_THREADS) {
    const int ch = order[q / UT];
    a.up[q] = TcTile{chunk_e[ch], chunk_p0[ch], chunk_n[ch], 64 * (q % UT)};
  }
  for (int q = tid; q < nch * DT && q < a.max_dn; q += PLAN_THREADS) {
    const int ch = order[q / DT];
    a.dn[q] = TcTile{chunk_e[ch], chunk_p0[ch], chunk_n[ch], 128 * (q % DT)};
  }
  if (tid == 0) {
    a.n_tiles[0] = min(nch * UT, a.max_up);
    a.n_tiles[1] = min(nch * DT, a.max_dn);
    if (tot.y * UT > a.max_up || tot.y * DT > a.max_dn || tot.y > PLAN_MAX_CHUNKS) raise_error(a.err, YN_ERR_BAD_SLOT);
  }
}

}  // namespace ynb
