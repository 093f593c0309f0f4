// Persistent data-flow decode of a batch of T <= 8 rows through every layer
// of an all-resident stack, in one cooperative launch: the speculative-verify
// pass (speculative.py:121-193 runs the 1 + d rows of a draft through one
// forward and compares) and small decode batches. No grid barrier and no
// host round trip between layers.
//
// Compiled shape (the LFM2-24B-A2B-shaped stack): hidden 2048, 64 routed
// experts, top-k <= 8, SwiGLU intermediate 1536, routed experts 4-bit with
// groups of 64, router 8-bit with groups of 64, no shared expert.
//
// Grid = one CTA per SM (cooperative launch), 512 threads. Per layer:
//   In  every CTA reads the T input rows (the batch rows at the first layer,
//       else the previous layer's output rows, as flagged words) and
//       normalises them (canonical RMSNorm, bit-identical to the oracle).
//   R   CTA b < 64 computes router row b for the T rows (canonical fp32 dot
//       of the row copied during the previous layer) and publishes the
//       logits.
//   Rt  every CTA routes the T rows (warp t: row t; softmax with the
//       deterministic exp, top-k by (bf16 probability desc, id asc),
//       renormalisation; bit-identical to the single-row path) and derives
//       the plan: the D distinct experts in ascending id order, the rows of
//       each in ascending order; pair slot of (row t, expert e) = the rows
//       of the experts below e + the rows of e before t. CTAs
//       [G d / D, G (d+1) / D) take expert d.
//   GU  the CTA's share of its expert's 8-unit groups (8 gate + 8 up rows:
//       16 MMA rows) is split over its warps; each warp streams its rows
//       over the whole K through a private ring of 4 stage slots (16-byte
//       cp.async of 128 code bytes per row, chunks swizzled by row & 7, plus
//       the stage's scales and biases; cp.async groups, no block sync) and
//       keeps the GEMV accumulators in registers: tensor-core MMAs whose
//       n = 8 columns are the expert's rows, in the batch path's arithmetic.
//       Gate and up of a unit end in the same lane: SwiGLU there, and the
//       activations go out as flagged words, two units per word.
//   Dn  the warp's 16-row groups of the expert's down rows follow in the
//       same ring (their first stages are fetched during the gate/up tail);
//       once all of the expert's activations have arrived (published by its
//       CTAs), fragments, the same GEMV, and the expert outputs y go out as
//       flagged words, two rows per word.
//   C   CTA b owns a slice of the T x H/2 output words: the k routed y in
//       column order times the routing weights, then the residual; the
//       words are the next layer's input (or the outputs after the last
//       layer).
// A flagged word is {32-bit payload, epoch = layer + 1}, one relaxed 64-bit
// store; every buffer is double-buffered by layer parity. Every CTA reads
// all of layer l's output words before anything of layer l+1 and writes
// some of them, so a buffer of parity p, rewritten at layer l+2, is past
// every read of layer l. Every wait has a wall-clock limit and watches the
// error word; on an error each CTA lets its copies in flight land and
// returns. Reference behaviour: moe_prefetch/orchestrator.py:308-343 with
// every expert resident (mlx_backend.py:302-316 routing, :411-436 moe over
// the union of a batch's experts, :442-459 the expert MLP).
#pragma once
#include "yn_batch.cuh"
#include "yn_decode.cuh"

namespace ynb {

constexpr int RF_THREADS = 512;
constexpr int RF_WARPS = RF_THREADS / 32;
constexpr int RF_H = 2048, RF_E = 64, RF_I = 1536;
constexpr int RF_TMAX = 8, RF_KMAX = 8;
constexpr int RF_BITS = 4, RF_GS = 64;
constexpr int RF_GU_UNITS = 8;                // gate/up work group: 8 units = 8 gate + 8 up rows (16 MMA rows)
constexpr int RF_DN_ROWS = 16;                // down work group: 16 output rows
constexpr int RF_NGU = RF_I / RF_GU_UNITS;    // 192 gate/up groups per expert
constexpr int RF_NGD_R = RF_H / RF_DN_ROWS;   // 128 down groups per expert
constexpr int RF_RB = RF_H * RF_BITS / 8;     // 1024 code bytes per gate/up row
constexpr int RF_RBD = RF_I * RF_BITS / 8;    // 768 per down row
constexpr int RF_NG = RF_H / RF_GS;           // 32 groups per gate/up row
constexpr int RF_NGD = RF_I / RF_GS;          // 24 per down row
constexpr int RF_RNG = RF_H / DEC_DGS;        // 32 groups per router row
constexpr int RF_KSTAGE = 128;                // code bytes of a row per K stage (256 codes, 4 groups)
constexpr int RF_NKU = RF_RB / RF_KSTAGE;     // 8 stages per gate/up row
constexpr int RF_NKD = RF_RBD / RF_KSTAGE;    // 6 stages per down row
constexpr int RF_GPS = RF_KSTAGE * 8 / RF_BITS / RF_GS;   // 4 groups per stage
constexpr int RF_CSLOT = 16 * RF_KSTAGE;      // 2,048 B: a stage's 16 code rows
constexpr int RF_SSLOT = 2 * 16 * RF_GPS * 2; // 256 B: their scales and biases
constexpr int RF_NST = 4;                     // ring stages per warp (3 in flight while one is computed)
constexpr int RF_XSU = RF_H / 2 + 16;   // fragment words per row (frag_stride_words), gate/up
constexpr int RF_XSD = RF_I / 2 + 16;   // down
constexpr int RF_GSU = RF_NG + 2;       // group-data entries per row (gdata_stride), gate/up
constexpr int RF_GSD = RF_NGD + 2;      // down
constexpr int RF_MAX_CW = 64;           // output words per CTA
static_assert(RF_GPS == 4 && RF_NKU * RF_KSTAGE == RF_RB && RF_NKD * RF_KSTAGE == RF_RBD, "whole stages");
static_assert(RF_CSLOT % 128 == 0, "code slots stay 128-byte aligned");
static_assert(RF_E == 64, "every router row has a CTA of its own");
static_assert(RF_XSU == RF_H / 2 + 16 && RF_XSD == RF_I / 2 + 16, "batch-path fragment strides (4-bit)");

// Fixed shared-memory header (byte offsets).
constexpr int RF_OFF_BARR = 0;       // router / norm tile barrier
constexpr int RF_OFF_ZERO = 64;      // 16 zero bytes: the B fragment of batch columns past the rows
constexpr int RF_OFF_RED = 128;      // 32 floats
constexpr int RF_OFF_IDS = 256;      // (T, K) routed ids
constexpr int RF_OFF_W = 512;        // (T, K) routing weights
constexpr int RF_OFF_RMASK = 768;    // (E) rows of each expert (bit t)
constexpr int RF_OFF_PBASE = 1024;   // (E) first pair slot of each expert
constexpr int RF_OFF_ELIST = 1280;   // (D) experts in ascending id order
constexpr int RF_OFF_MISC = 1536;    // ints: [0] D, [8..16) local row -> row, [16..24) identity
constexpr int RF_OFF_ROWF = 1664;    // floats: [0..8) 1/rms, [8..16) fragment scales
constexpr int RF_OFF_HRES = 1792;    // (<= 64) residual words of this CTA's output slice
constexpr int RF_OFF_LAY = 2048;     // 2 layer descriptors
constexpr int RF_OFF_NORM = 2816;    // post-attention norm weight (H bf16)
constexpr int RF_OFF_RC = 6912;      // router row codes (H bytes)
constexpr int RF_OFF_RS = 8960;      // router row scales
constexpr int RF_OFF_RBI = 9024;     // router row biases
constexpr int RF_FIXED = 9216;
static_assert(RF_OFF_LAY + 2 * (int)sizeof(DecLayer) <= RF_OFF_NORM, "layer descriptors fit");
static_assert(RF_OFF_RC == RF_OFF_NORM + RF_H * 2 && RF_OFF_RS == RF_OFF_RC + RF_H &&
              RF_OFF_RBI == RF_OFF_RS + RF_RNG * 2 && RF_OFF_RBI + RF_RNG * 2 <= RF_FIXED, "router tile fits");

struct RowsArgs {
  int T, K, norm_topk;
  float eps;
  const DecLayer* layers;
  int n_layers;
  const uint16_t* inputs;   // (T, H)
  uint16_t* outputs;        // (T, H)
  u64* f_logits;            // (2, T, E) router logits (fp32)
  u64* f_act;               // (2, P, I/2) SwiGLU activations of each pair slot, two bf16 per word
  u64* f_y;                 // (2, P, H/2) expert outputs of each pair slot, two bf16 per word
  u64* f_h;                 // (2, T, H/2) layer outputs, two bf16 per word
  int P;                    // pair slots = T * K
  int32_t* trace_ids;       // (L, T, K) or null
  uint16_t* trace_h;        // (L, T, H) each layer's input rows, or null
  float* trace_w;           // (L, T, K) or null
  int* err;
  long long* timing;        // (L, RF_STAMPS, G) global-timer stamps, or null
  int off_x, off_xf, off_xg, off_ring, off_rsc;
};

YN_DEV void rf_stamp(const RowsArgs& a, int layer, int slot) {
  if (a.timing) stamp_at(a.timing, layer, slot);
}

// Wait for n flagged words (epoch ep) and store their payloads: each thread
// issues the loads of up to 8 words before it checks any, so the words of a
// thread are one round trip, not n / 512.
YN_DEV void rf_wait_words(const u64* src, uint32_t* dst, int n, uint32_t ep, int* err, bool& fail) {
  for (int i0 = threadIdx.x; i0 < n; i0 += 8 * RF_THREADS) {
    u64 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * RF_THREADS;
      v[u] = i < n ? get_flag(src + i) : 0ull;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * RF_THREADS;
      if (i < n) dst[i] = (uint32_t)(v[u] >> 32) == ep ? (uint32_t)v[u] : wait_flag(src + i, ep, err, fail);
    }
  }
}

// Post-attention norm weight of every CTA and router row b of the router
// CTAs, as bulk copies completing on `bar` (one thread).
YN_DEV void rf_issue_rtile(const DecLayer& L, int b, bool router, uint8_t* smem, uint64_t* bar) {
  const uint32_t nb = RF_H * 2, rb = router ? RF_H : 0u, sb = router ? RF_RNG * 2 : 0u;
  mbar_arrive_expect_tx(bar, nb + rb + 2 * sb);
  bulk_g2s(smem + RF_OFF_NORM, L.norm, nb, bar);
  if (router) {
    bulk_g2s(smem + RF_OFF_RC, L.router.w + (size_t)b * RF_H, rb, bar);
    bulk_g2s(smem + RF_OFF_RS, reinterpret_cast<const uint8_t*>(L.router.s) + (size_t)b * sb, sb, bar);
    bulk_g2s(smem + RF_OFF_RBI, reinterpret_cast<const uint8_t*>(L.router.b) + (size_t)b * sb, sb, bar);
  }
}

// RMSNorm of T rows in place, each in the canonical 128-thread order:
// x = bf16(w * bf16(h * r)), r = 1 / sqrt(sum(h^2) / H + eps), thread i of a
// row summing h[i + 128 m] in ascending m, a butterfly inside each warp and
// the four warp partials summed in warp order. Thread (q, i) takes rows q and
// q + 4 as two independent chains. Ends with a block sync.
YN_DEV void rf_rmsnorm_rows(uint16_t* x, const uint16_t* w, int T, float eps, float* red, float* rinv) {
  static_assert(RF_TMAX <= 8 && RF_THREADS == 512, "four rows of 128 threads per pass, two passes per thread");
  const int tid = threadIdx.x, q = tid >> 7, i = tid & 127;
  const int t0 = q, t1 = q + 4;
  float s0 = 0.0f, s1 = 0.0f;
  const uint16_t* x0 = x + (size_t)t0 * RF_H;
  const uint16_t* x1 = x + (size_t)t1 * RF_H;
  const bool h0 = t0 < T, h1 = t1 < T;
#pragma unroll
  for (int m = 0; m < RF_H / 128; ++m) {
    const int j = i + 128 * m;
    if (h0) {
      const float v = bf16_to_f32(x0[j]);
      s0 = __fmaf_rn(v, v, s0);
    }
    if (h1) {
      const float v = bf16_to_f32(x1[j]);
      s1 = __fmaf_rn(v, v, s1);
    }
  }
  s0 = group_sum_bfly(s0, 32);
  s1 = group_sum_bfly(s1, 32);
  if ((tid & 31) == 0) {
    red[tid >> 5] = s0;          // row q: red[4 q + warp of the row]
    red[16 + (tid >> 5)] = s1;   // row q + 4
  }
  __syncthreads();
  if (tid < T) {
    const float* r4 = red + 4 * tid;
    const float tot = __fadd_rn(__fadd_rn(__fadd_rn(r4[0], r4[1]), r4[2]), r4[3]);
    rinv[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(tot, 1.0f / (float)RF_H), eps)));
  }
  __syncthreads();
  for (int k = tid; k < T * RF_H / 8; k += RF_THREADS) {   // 8 elements per step
    const int t = k / (RF_H / 8), j8 = k % (RF_H / 8);
    const float r = rinv[t];
    uint4 hv = reinterpret_cast<const uint4*>(x)[k];
    const uint4 wv = reinterpret_cast<const uint4*>(w)[j8];
    uint32_t* hp = reinterpret_cast<uint32_t*>(&hv);
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(&wv);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float lo = __fmul_rn(bf16_to_f32((uint16_t)(wp[e] & 0xFFFFu)),
                                 bf16r(__fmul_rn(bf16_to_f32((uint16_t)(hp[e] & 0xFFFFu)), r)));
      const float hi = __fmul_rn(bf16_to_f32((uint16_t)(wp[e] >> 16)),
                                 bf16r(__fmul_rn(bf16_to_f32((uint16_t)(hp[e] >> 16)), r)));
      hp[e] = (uint32_t)f32_to_bf16(lo) | ((uint32_t)f32_to_bf16(hi) << 16);
    }
    reinterpret_cast<uint4*>(x)[k] = hv;
  }
  __syncthreads();
}

// Batch-path fragments (the layout k_batch_frags writes) of n rows of Kd bf16
// values, rows[i] the source row of fragment row i: per row a power-of-two
// scale from max|x|, the fp16 pair words, and per group {-1024 * sum of the
// fragment values, scale * sum(x)}, then {1 / scale, 0}. Group sums: eight
// threads per group, 8 consecutive values each, then a butterfly. Ends with a
// block sync.
template <int BITS, int GS, int Kd>
YN_DEV void rf_frags(const uint16_t* src, const int* rows, int n, uint32_t* XF, int xs_w, float2* XG, int gsd,
                     float* rsc) {
  using F = BFmt<BITS, GS>;
  static_assert(GS == 64 && F::WPL == 8, "eight threads of 8 codes (one code word) per group");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (warp < n) {
    const uint4* x = reinterpret_cast<const uint4*>(src + (size_t)rows[warp] * Kd);
    float mx = 0.0f;
    for (int k = lane; k < Kd / 8; k += 32) {
      const uint4 v = x[k];
      const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e)   // |x| as the magnitude bits of bf16: the order of the floats
        mx = fmaxf(mx, fmaxf(bf16_to_f32((uint16_t)(vv[e] & 0x7FFFu)), bf16_to_f32((uint16_t)((vv[e] >> 16) & 0x7FFFu))));
    }
    mx = warp_max(mx);
    if (lane == 0) rsc[warp] = fp16_input_scale(mx);
  }
  __syncthreads();
  constexpr int hw = Kd / 2;
  for (int i = tid; i < n * hw; i += RF_THREADS) {
    const int r = i / hw, w = i - r * hw;
    const uint16_t* x = src + (size_t)rows[r] * Kd;
    const int p = w % F::PPW, wc = w / F::PPW;   // wc = chunk * 4 + word of the chunk
    const int base = (wc >> 2) * F::CPCH + (wc & 3) * F::WPL;
    const float m = __fmul_rn(rsc[r], BW<BITS>::inv_mult(p));
    __half2 h = __floats2half2_rn(__fmul_rn(bf16_to_f32(x[base + BW<BITS>::lo(p)]), m),
                                  __fmul_rn(bf16_to_f32(x[base + BW<BITS>::hi(p)]), m));
    XF[(size_t)r * xs_w + w] = *reinterpret_cast<uint32_t*>(&h);
  }
  constexpr int NG = Kd / GS;
  for (int i = tid; i < n * NG * 8; i += RF_THREADS) {   // every lane of a warp takes part (butterflies)
    const int sub = i & 7, gq = i >> 3, r = gq / NG, g = gq - r * NG;
    const bool ok = r < n;
    float sx = 0.0f, o = 0.0f;
    if (ok) {
      const float scale = rsc[r];
      const uint4 v = *reinterpret_cast<const uint4*>(src + (size_t)rows[r] * Kd + g * GS + 8 * sub);
      const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float f = bf16_to_f32((uint16_t)((e & 1) ? vv[e >> 1] >> 16 : vv[e >> 1] & 0xFFFFu));
        sx = __fadd_rn(sx, f);
        const float m = __fmul_rn(scale, BW<BITS>::inv_mult(BW<BITS>::pair_of(e)));
        o = __fadd_rn(o, __half2float(__float2half_rn(__fmul_rn(f, m))));
      }
    }
    sx = group_sum_bfly(sx, 8);
    o = group_sum_bfly(o, 8);
    if (ok && sub == 0) XG[(size_t)r * gsd + g] = make_float2(__fmul_rn(-1024.0f, o), __fmul_rn(rsc[r], sx));
  }
  if (tid < n) {
    XG[(size_t)tid * gsd + NG] = make_float2(__fdiv_rn(1.0f, rsc[tid]), 0.0f);
    XG[(size_t)tid * gsd + NG + 1] = make_float2(0.0f, 0.0f);
  }
  __syncthreads();
}

// The MMAs of this kernel as plain (non-volatile) asm: pure register
// functions, so the compiler may interleave the independent group chains of
// a stage (volatile asm keeps every MMA in program order). The shared-memory
// reads (ldmatrix) stay volatile, ordered after the stage waits.
YN_DEV void rf_mma(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
YN_DEV void rf_mmac(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2], const float (&c)[4]) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}

YN_DEV void cp8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
YN_DEV void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
YN_DEV void cp_wait_prefetched() { asm volatile("cp.async.wait_group %0;" ::"n"(RF_NST - 2) : "memory"); }

// One K stage of a warp's 16 weight rows into its ring slots: the rows' 128
// code bytes of stage k (16-byte chunks swizzled by row & 7, so the ldmatrix
// rows of a chunk fall in different banks) and the 4 groups' scales and
// biases (8 bytes a row each), issued by the warp's lanes (4 + 1 copies
// each), not committed. Gate/up group (gu): rows 0..7 are the gate rows of
// units row0..row0+7, rows 8..15 their up rows; down group: output rows
// row0..row0+15.
template <bool gu>
YN_DEV void rf_issue_stage(uint8_t* cslot, uint8_t* sslot, const uint8_t* rec, const RecGeom& rg, int row0, int k,
                           int lane) {
  const int ch = lane & 7, rq = lane >> 3;
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const int row = rq + 4 * m;
    const uint8_t* src = gu ? rec + rg.off[m < 2 ? 0 : 3] + (size_t)(row0 + (row & 7)) * RF_RB
                            : rec + rg.off[6] + (size_t)(row0 + row) * RF_RBD;
    cp16(cslot + row * RF_KSTAGE + ((ch ^ (row & 7)) << 4), src + k * RF_KSTAGE + 16 * ch);
  }
  const int row = lane & 15, which = lane >> 4;   // scales (0) or biases (1) of row
  const int sb = gu ? RF_NG * 2 : RF_NGD * 2;
  const int piece = gu ? (row < 8 ? (which ? 2 : 1) : (which ? 5 : 4)) : (which ? 8 : 7);
  const int srow = gu ? row0 + (row & 7) : row0 + row;
  cp8(sslot + which * (16 * RF_GPS * 2) + row * (RF_GPS * 2), rec + rg.off[piece] + (size_t)srow * sb + k * (RF_GPS * 2));
}

// The MMAs of one stage (4 groups of 2 chunks) for the warp's 16 rows and up
// to 8 batch rows (the n = 8 columns), accumulated into acc (lane (g, c):
// weight rows g and g+8, batch rows 2c and 2c+1), in the batch path's
// arithmetic (warp_tile): each group's tile starts at the group's unpack
// offset, and its scale and bias are applied in fp32.
template <int xs, int gsd>
YN_DEV void rf_stage_mma(const uint8_t* slot, const uint8_t* sslot, int k, const uint32_t* XF, const float2* XG, int ntok,
                         float (&acc)[4]) {
  using F = BFmt<RF_BITS, RF_GS>;
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int mrow = ((lane >> 3) & 1) * 8 + (lane & 7), mch = lane >> 4;
  const uint16_t* Ss = reinterpret_cast<const uint16_t*>(sslot);
  const uint16_t* Bs = Ss + 16 * RF_GPS;
  const int t0 = 2 * c;
#pragma unroll
  for (int gi = 0; gi < RF_GPS; ++gi) {
    uint32_t wr[4];
    ldsm_x4(wr, slot + mrow * RF_KSTAGE + (((2 * gi + mch) ^ (mrow & 7)) << 4));
    const int grp = RF_GPS * k + gi;
    float d[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int ch = 8 * k + 2 * gi + h;
      uint32_t pa[F::PPW], pb[F::PPW], xb[F::PPW];
      BW<RF_BITS>::unpack(wr[2 * h], pa);
      BW<RF_BITS>::unpack(wr[2 * h + 1], pb);
      {   // batch columns past the expert's rows read the zero block (an address choice, no branch)
        extern __shared__ __align__(128) uint8_t smem_z[];
        const uint4* src = g < ntok ? reinterpret_cast<const uint4*>(XF + (size_t)g * xs + (size_t)(ch * 4 + c) * F::PPW)
                                    : reinterpret_cast<const uint4*>(smem_z + RF_OFF_ZERO);
        const uint4 v = *src;
        xb[0] = v.x; xb[1] = v.y; xb[2] = v.z; xb[3] = v.w;
      }
      const uint32_t A0[4] = {pa[0], pb[0], pa[1], pb[1]}, B0[2] = {xb[0], xb[1]};
      if (h == 0) {
        const float n0 = XG[(size_t)t0 * gsd + grp].x, n1 = XG[(size_t)(t0 + 1) * gsd + grp].x;
        const float ci[4] = {n0, n1, n0, n1};
        rf_mmac(d, A0, B0, ci);
      } else {
        rf_mma(d, A0, B0);
      }
      const uint32_t A1[4] = {pa[2], pb[2], pa[3], pb[3]}, B1[2] = {xb[2], xb[3]};
      rf_mma(d, A1, B1);
    }
    const float x0 = XG[(size_t)t0 * gsd + grp].y, x1 = XG[(size_t)(t0 + 1) * gsd + grp].y;
    const float s0 = f16_to_f32(Ss[g * RF_GPS + gi]), s1 = f16_to_f32(Ss[(g + 8) * RF_GPS + gi]);
    const float b0 = f16_to_f32(Bs[g * RF_GPS + gi]), b1 = f16_to_f32(Bs[(g + 8) * RF_GPS + gi]);
    acc[0] = __fmaf_rn(s0, d[0], __fmaf_rn(b0, x0, acc[0]));
    acc[1] = __fmaf_rn(s0, d[1], __fmaf_rn(b0, x1, acc[1]));
    acc[2] = __fmaf_rn(s1, d[2], __fmaf_rn(b1, x0, acc[2]));
    acc[3] = __fmaf_rn(s1, d[3], __fmaf_rn(b1, x1, acc[3]));
  }
}

// A finished gate/up group: lane (g, c) holds gate (acc 0, 1) and up (acc 2, 3)
// of unit u0 + g for batch rows 2c, 2c+1; SwiGLU, and units g, g+1 go out as
// one flagged word per row.
YN_DEV void rf_gu_out(const float (&acc)[4], const float2* XG, int Td, u64* f_act_rows, int u0, uint32_t ep) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3, t0 = 2 * c;
  uint32_t v[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const float inv = XG[(size_t)(t0 + h) * RF_GSU + RF_NG].x;
    v[h] = (uint32_t)f32_to_bf16(swiglu_bf16(bf16r(__fmul_rn(acc[h], inv)), bf16r(__fmul_rn(acc[2 + h], inv))));
  }
  const uint32_t n0 = __shfl_down_sync(0xffffffffu, v[0], 4), n1 = __shfl_down_sync(0xffffffffu, v[1], 4);
  if (!(g & 1)) {
    if (t0 < Td) put_flag(f_act_rows + (size_t)t0 * (RF_I / 2) + (u0 + g) / 2, v[0] | (n0 << 16), ep);
    if (t0 + 1 < Td) put_flag(f_act_rows + (size_t)(t0 + 1) * (RF_I / 2) + (u0 + g) / 2, v[1] | (n1 << 16), ep);
  }
}

// A finished down group: lane (g, c) holds output rows r0 + g (acc 0, 1) and
// r0 + g + 8 (acc 2, 3) for batch rows 2c, 2c+1; rows g, g+1 go out as one
// flagged word.
YN_DEV void rf_dn_out(const float (&acc)[4], const float2* XG, int Td, u64* f_y_rows, int r0, uint32_t ep) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3, t0 = 2 * c;
  uint32_t v[4];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const float inv = XG[(size_t)(t0 + h) * RF_GSD + RF_NGD].x;
    v[h] = (uint32_t)f32_to_bf16(__fmul_rn(acc[h], inv));
    v[2 + h] = (uint32_t)f32_to_bf16(__fmul_rn(acc[2 + h], inv));
  }
  uint32_t n[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) n[q] = __shfl_down_sync(0xffffffffu, v[q], 4);
  if (!(g & 1)) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (t0 + h >= Td) continue;
      u64* fr = f_y_rows + (size_t)(t0 + h) * (RF_H / 2);
      put_flag(fr + (r0 + g) / 2, v[h] | (n[h] << 16), ep);
      put_flag(fr + (r0 + g + 8) / 2, v[2 + h] | (n[2 + h] << 16), ep);
    }
  }
}

__global__ void __launch_bounds__(RF_THREADS, 1) k_rows_flow(const RowsArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* barR = reinterpret_cast<uint64_t*>(smem + RF_OFF_BARR);
  float* red = reinterpret_cast<float*>(smem + RF_OFF_RED);
  int32_t* ids_s = reinterpret_cast<int32_t*>(smem + RF_OFF_IDS);
  float* w_s = reinterpret_cast<float*>(smem + RF_OFF_W);
  uint32_t* rowmask = reinterpret_cast<uint32_t*>(smem + RF_OFF_RMASK);
  int* pbase = reinterpret_cast<int*>(smem + RF_OFF_PBASE);
  int* elist = reinterpret_cast<int*>(smem + RF_OFF_ELIST);
  int* misc = reinterpret_cast<int*>(smem + RF_OFF_MISC);
  float* rowf = reinterpret_cast<float*>(smem + RF_OFF_ROWF);
  uint32_t* hres = reinterpret_cast<uint32_t*>(smem + RF_OFF_HRES);
  DecLayer* lay = reinterpret_cast<DecLayer*>(smem + RF_OFF_LAY);
  const uint16_t* normw = reinterpret_cast<const uint16_t*>(smem + RF_OFF_NORM);
  const uint8_t* rcode = smem + RF_OFF_RC;
  const uint16_t* rsc = reinterpret_cast<const uint16_t*>(smem + RF_OFF_RS);
  const uint16_t* rbi = reinterpret_cast<const uint16_t*>(smem + RF_OFF_RBI);
  uint16_t* xb = reinterpret_cast<uint16_t*>(smem + a.off_x);
  uint32_t* XF = reinterpret_cast<uint32_t*>(smem + a.off_xf);
  float2* XG = reinterpret_cast<float2*>(smem + a.off_xg);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // this warp's stage slots (code rows, scales)
  uint8_t* cring = smem + a.off_ring + (size_t)warp * RF_NST * RF_CSLOT;
  uint8_t* sring = smem + a.off_rsc + (size_t)warp * RF_NST * RF_SSLOT;
  const int G = gridDim.x, b = blockIdx.x, T = a.T, K = a.K;
  const int W = T * (RF_H / 2);
  const int cw0 = (int)((long long)W * b / G), ncw = (int)((long long)W * (b + 1) / G) - cw0;
  const bool router_cta = b < RF_E;

  if (tid == 0) {
    mbar_init(barR, 1);
    fence_mbar_init();
  }
  if (tid < 8) misc[16 + tid] = tid;
  if (tid < 4) reinterpret_cast<uint32_t*>(smem + RF_OFF_ZERO)[tid] = 0u;
  load_layer(&lay[0], a.layers, 0);
  __syncthreads();
  if (tid == 0) rf_issue_rtile(lay[0], b, router_cta, smem, barR);
  uint32_t phR = 0;
  bool pendR = true;
  // diagnostics (timing only, thread 0): ns waiting on its warp's ring stages (gate/up, down)
  unsigned long long dg_wait_gu = 0, dg_wait_dn = 0, dg_t = 0;
  const bool diag = a.timing != nullptr && tid == 0;
  auto dg_now = [&]() { return diag ? globaltimer_ns() : 0ull; };
  auto drain = [&]() {   // block-uniform: every copy in flight lands before the CTA returns
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (pendR) mbar_wait_block(barR, phR, nullptr);
  };

  for (int layer = 0; layer < a.n_layers; ++layer) {
    const DecLayer& L = lay[layer & 1];
    const int par = layer & 1;
    const uint32_t ep = (uint32_t)layer + 1;
    const bool more = layer + 1 < a.n_layers;
    rf_stamp(a, layer, 0);
    if (more) load_layer(&lay[(layer + 1) & 1], a.layers, layer + 1);
    if (tid < RF_E) rowmask[tid] = 0u;
    // -------- In: the T input rows
    bool fail = false;
    if (layer == 0) {
      for (int i = tid; i < T * RF_H / 8; i += RF_THREADS)
        reinterpret_cast<uint4*>(xb)[i] = __ldcg(reinterpret_cast<const uint4*>(a.inputs) + i);
    } else {
      rf_wait_words(a.f_h + (size_t)((layer - 1) & 1) * W, reinterpret_cast<uint32_t*>(xb), W, (uint32_t)layer,
                    a.err, fail);
    }
    if (__syncthreads_or(fail)) { drain(); return; }
    if (tid < ncw) hres[tid] = reinterpret_cast<const uint32_t*>(xb)[cw0 + tid];
    if (a.trace_h && b == 0)
      for (int i = tid; i < T * RF_H / 8; i += RF_THREADS)
        reinterpret_cast<uint4*>(a.trace_h + (size_t)layer * T * RF_H)[i] = reinterpret_cast<const uint4*>(xb)[i];
    rf_stamp(a, layer, 1);
    if (!mbar_wait_block(barR, phR, a.err)) { drain(); return; }
    phR ^= 1;
    pendR = false;
    rf_rmsnorm_rows(xb, normw, T, a.eps, red, rowf);
    rf_stamp(a, layer, 2);
    // -------- R: router row b for every row
    if (router_cta && warp < T) {
      XF32<8, DEC_H / 16 / 32, 1> X;
      load_x_f32<8, DEC_H / 16 / 32, 1>(X, xb + (size_t)warp * RF_H, lane, 32);
      float v = row_dot_f32<8, DEC_H / 16 / 32, 1>(rcode, rsc, rbi, X, lane, 32, DEC_DGS);
      v = group_sum_bfly(v, 32);
      if (lane == 0) {
        const float bias = L.rbias ? __ldcg(L.rbias + b) : 0.0f;
        put_flag(a.f_logits + ((size_t)par * T + warp) * RF_E + b, __float_as_uint(bf16r(__fadd_rn(v, bias))), ep);
      }
    }
    __syncthreads();   // the norm weight and router row are read: the next layer's may come in
    if (more && tid == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      rf_issue_rtile(lay[(layer + 1) & 1], b, router_cta, smem, barR);
    }
    pendR = more;
    rf_stamp(a, layer, 3);
    // -------- Rt: routing of every row (warp t: row t)
    if (warp < T) {
      const u64* lg = a.f_logits + ((size_t)par * T + warp) * RF_E;
      const u64 v0 = get_flag(lg + lane), v1 = get_flag(lg + lane + 32);
      const float x0 = __uint_as_float((uint32_t)(v0 >> 32) == ep ? (uint32_t)v0 : wait_flag(lg + lane, ep, a.err, fail));
      const float x1 =
          __uint_as_float((uint32_t)(v1 >> 32) == ep ? (uint32_t)v1 : wait_flag(lg + lane + 32, ep, a.err, fail));
      const float m = warp_max_redux(fmaxf(x0, x1));
      const float p0 = yn_expf(__fsub_rn(x0, m)), p1 = yn_expf(__fsub_rn(x1, m));
      const float s = group_sum_bfly(__fadd_rn(p0, p1), 32);   // lane sum over e = lane, lane + 32, in that order
      uint32_t k0 = ((uint32_t)f32_to_bf16(bf16r(__fdiv_rn(p0, s))) << 16) | (0xFFFFu - (uint32_t)lane);
      uint32_t k1 = ((uint32_t)f32_to_bf16(bf16r(__fdiv_rn(p1, s))) << 16) | (0xFFFFu - (uint32_t)(lane + 32));
      float wsum = 0.0f, myp = 0.0f;
      int myid = 0;
      for (int j = 0; j < K; ++j) {
        const uint32_t top = __reduce_max_sync(0xffffffffu, max(k0, k1));
        if (k0 == top) k0 = 0u;
        if (k1 == top) k1 = 0u;
        const float pj = bf16_to_f32((uint16_t)(top >> 16));
        wsum = __fadd_rn(wsum, pj);
        if (lane == j) {
          myp = pj;
          myid = 0xFFFF - (int)(top & 0xFFFFu);
        }
      }
      const float sb = bf16r(wsum);
      if (lane < K) {
        ids_s[warp * K + lane] = myid;
        w_s[warp * K + lane] = a.norm_topk ? bf16r(__fdiv_rn(myp, sb)) : myp;
      }
    }
    if (__syncthreads_or(fail)) { drain(); return; }
    rf_stamp(a, layer, 4);
    if (tid < T * K) atomicOr(&rowmask[ids_s[tid]], 1u << (tid / K));
    if (b == 0 && tid < T * K) {
      if (a.trace_ids) a.trace_ids[(size_t)layer * T * K + tid] = ids_s[tid];
      if (a.trace_w) a.trace_w[(size_t)layer * T * K + tid] = w_s[tid];
    }
    __syncthreads();
    if (warp == 0) {   // experts in id order: pair-slot bases, dense index, count
      const uint32_t m0 = rowmask[2 * lane], m1 = rowmask[2 * lane + 1];
      const int c0 = __popc(m0), c1 = __popc(m1), pr = (m0 != 0u) + (m1 != 0u);
      int incP = c0 + c1, incD = pr;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int up = __shfl_up_sync(0xffffffffu, incP, o), ud = __shfl_up_sync(0xffffffffu, incD, o);
        if (lane >= o) {
          incP += up;
          incD += ud;
        }
      }
      const int exP = incP - c0 - c1, exD = incD - pr;
      pbase[2 * lane] = exP;
      pbase[2 * lane + 1] = exP + c0;
      if (m0) elist[exD] = 2 * lane;
      if (m1) elist[exD + (m0 != 0u ? 1 : 0)] = 2 * lane + 1;
      if (lane == 31) misc[0] = incD;
    }
    __syncthreads();
    const int D = misc[0];
    bool bad = false;
    if (tid < D) {
      const int e = elist[tid];
      const int sl = L.slot_of ? L.slot_of[e] : e;
      bad = sl < 0 || sl >= L.n_slots;
    }
    if (__syncthreads_or(bad)) {
      if (tid == 0) raise_error(a.err, YN_ERR_BAD_SLOT);
      drain();
      return;
    }
    // this CTA's expert, its rows, and this warp's work groups
    const int d = ((b + 1) * D - 1) / G;   // (b + 1) * D <= 148 * 64: 32-bit
    const int lo = d * G / D, hi = (d + 1) * G / D;
    const int r = b - lo, nd = hi - lo;
    const int e = elist[d];
    const uint32_t rm = rowmask[e];
    const int Td = __popc(rm), ps0 = pbase[e];
    const int gu0 = RF_NGU * r / nd, ngu = RF_NGU * (r + 1) / nd - gu0;        // 8-unit groups of the CTA
    const int dn0 = RF_NGD_R * r / nd, ndn = RF_NGD_R * (r + 1) / nd - dn0;    // 16-row groups
    const int my_gu = warp < ngu ? (ngu - warp + RF_WARPS - 1) / RF_WARPS : 0;    // groups w, w + 16, ...
    const int my_dn = warp < ndn ? (ndn - warp + RF_WARPS - 1) / RF_WARPS : 0;
    const int n_gu_items = my_gu * RF_NKU, n_items = n_gu_items + my_dn * RF_NKD;
    const uint8_t* rec = expert_record(L, e);
    if (tid < RF_TMAX) {   // local row tid -> its row: the position of set bit number tid of rm
      int pos = 0, cnt = 0;
      for (int bit = 0; bit < RF_TMAX; ++bit)
        if ((rm >> bit) & 1u) {
          if (cnt == tid) pos = bit;
          ++cnt;
        }
      misc[8 + tid] = pos;
    }
    // the warp's ring: item j = stage j % NK of its group j / NK (gate/up items first, then down) in slot
    // j % RF_NST; RF_NST - 1 items in flight; one cp.async commit group per item and lane, empty past the end
    auto issue_item = [&](int j) {
      if (j < n_items) {
        const int sl = j % RF_NST;
        const bool gu = j < n_gu_items;
        const int row0 = gu ? (gu0 + warp + RF_WARPS * (j / RF_NKU)) * RF_GU_UNITS
                            : (dn0 + warp + RF_WARPS * ((j - n_gu_items) / RF_NKD)) * RF_DN_ROWS;
        const int k = gu ? j % RF_NKU : (j - n_gu_items) % RF_NKD;
        if (gu) rf_issue_stage<true>(cring + (size_t)sl * RF_CSLOT, sring + (size_t)sl * RF_SSLOT, rec, L.rg, row0, k, lane);
        else rf_issue_stage<false>(cring + (size_t)sl * RF_CSLOT, sring + (size_t)sl * RF_SSLOT, rec, L.rg, row0, k, lane);
      }
      cp_commit();
    };
    // item j's stage in shared memory: this lane's copies landed, then every lane's (and every lane is done
    // with item j - 1, whose slot the next issue refills)
    auto wait_item = [&]() {
      cp_wait_prefetched();
      __syncwarp();
    };
    // the first stage before the fragments, the next two after them: a warp's copy issue stalls once the
    // SM's outstanding copies fill up, and the fragment build needs no copy
    issue_item(0);
    __syncthreads();   // misc[8..16)
    rf_stamp(a, layer, 5);
    rf_frags<RF_BITS, RF_GS, RF_H>(xb, misc + 8, Td, XF, RF_XSU, XG, RF_GSU, rowf + 8);
#pragma unroll
    for (int j = 1; j < RF_NST - 1; ++j) issue_item(j);
    rf_stamp(a, layer, 6);
    // -------- GU: the warp's gate/up groups, SwiGLU, activations out
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    u64* fa = a.f_act + ((size_t)par * a.P + ps0) * (RF_I / 2);
    for (int j = 0; j < n_gu_items; ++j) {
      dg_t = dg_now();
      wait_item();
      if (diag) dg_wait_gu += dg_now() - dg_t;
      issue_item(j + RF_NST - 1);   // into the slot of item j - 1
      const int sl = j % RF_NST;
      rf_stage_mma<RF_XSU, RF_GSU>(cring + (size_t)sl * RF_CSLOT, sring + (size_t)sl * RF_SSLOT, j % RF_NKU, XF, XG, Td,
                                   acc);
      if (j % RF_NKU == RF_NKU - 1) {
        rf_gu_out(acc, XG, Td, fa, (gu0 + warp + RF_WARPS * (j / RF_NKU)) * RF_GU_UNITS, ep);
        acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
      }
    }
    rf_stamp(a, layer, 7);
    // -------- Dn: the expert's activations of all its rows, fragments, the warp's down groups
    __syncthreads();   // warps without gate/up groups wait here in the barrier, not in polls beside the working warps
    rf_wait_words(fa, reinterpret_cast<uint32_t*>(xb), Td * (RF_I / 2), ep, a.err, fail);
    if (__syncthreads_or(fail)) { drain(); return; }
    rf_stamp(a, layer, 8);
    rf_frags<RF_BITS, RF_GS, RF_I>(xb, misc + 16, Td, XF, RF_XSD, XG, RF_GSD, rowf + 8);
    rf_stamp(a, layer, 9);
    u64* fy = a.f_y + ((size_t)par * a.P + ps0) * (RF_H / 2);
    for (int j = n_gu_items; j < n_items; ++j) {
      dg_t = dg_now();
      wait_item();
      if (diag) dg_wait_dn += dg_now() - dg_t;
      issue_item(j + RF_NST - 1);
      const int jd = j - n_gu_items;
      const int sl = j % RF_NST;
      rf_stage_mma<RF_XSD, RF_GSD>(cring + (size_t)sl * RF_CSLOT, sring + (size_t)sl * RF_SSLOT, jd % RF_NKD, XF, XG, Td,
                                   acc);
      if (jd % RF_NKD == RF_NKD - 1) {
        rf_dn_out(acc, XG, Td, fy, (dn0 + warp + RF_WARPS * (jd / RF_NKD)) * RF_DN_ROWS, ep);
        acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
      }
    }
    __syncthreads();   // likewise for warps without down groups
    rf_stamp(a, layer, 10);
    // -------- C: this CTA's output words (column order, then the residual)
    if (tid < ncw) {
      const int w = cw0 + tid, t = w / (RF_H / 2), p = w % (RF_H / 2);
      const u64* fy = a.f_y + (size_t)par * a.P * (RF_H / 2) + p;
      int ps[RF_KMAX];
      u64 v[RF_KMAX];
#pragma unroll
      for (int j = 0; j < RF_KMAX; ++j) {
        if (j < K) {
          const int ej = ids_s[t * K + j];
          ps[j] = pbase[ej] + __popc(rowmask[ej] & ((1u << t) - 1u));
          v[j] = get_flag(fy + (size_t)ps[j] * (RF_H / 2));
        }
      }
      float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
      for (int j = 0; j < RF_KMAX; ++j) {
        if (j < K) {
          const uint32_t y = (uint32_t)(v[j] >> 32) == ep ? (uint32_t)v[j]
                                                           : wait_flag(fy + (size_t)ps[j] * (RF_H / 2), ep, a.err, fail);
          const float wj = w_s[t * K + j];
          acc0 = __fadd_rn(acc0, bf16r(__fmul_rn(bf16_to_f32((uint16_t)(y & 0xFFFFu)), wj)));
          acc1 = __fadd_rn(acc1, bf16r(__fmul_rn(bf16_to_f32((uint16_t)(y >> 16)), wj)));
        }
      }
      const uint32_t hw = hres[tid];
      const float o0 = bf16r(__fadd_rn(bf16_to_f32((uint16_t)(hw & 0xFFFFu)), bf16r(acc0)));
      const float o1 = bf16r(__fadd_rn(bf16_to_f32((uint16_t)(hw >> 16)), bf16r(acc1)));
      const uint32_t pk = (uint32_t)f32_to_bf16(o0) | ((uint32_t)f32_to_bf16(o1) << 16);
      if (more) put_flag(a.f_h + (size_t)par * W + w, pk, ep);
      else reinterpret_cast<uint32_t*>(a.outputs)[w] = pk;
    }
    if (__syncthreads_or(fail)) { drain(); return; }
    rf_stamp(a, layer, 11);
    if (diag) {   // per-layer durations (ns) in stamp slots 12..14
      long long* tm = a.timing + ((size_t)layer * DEC_STAMPS) * gridDim.x + blockIdx.x;
      tm[12 * (size_t)gridDim.x] = (long long)dg_wait_gu;
      tm[13 * (size_t)gridDim.x] = (long long)dg_wait_dn;
      tm[14 * (size_t)gridDim.x] = (long long)(ngu * 1000 + ndn);
      dg_wait_gu = dg_wait_dn = 0;
    }
  }
  drain();
}

}  // namespace ynb
