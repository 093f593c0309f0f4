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
//   GU  the CTA's share of its expert's 96 gate/up tiles (16 units: 16 gate
//       and 16 up rows) streams through a ring of shared-memory slots
//       (16-byte cp.async, 16-byte chunks of a row swizzled by row & 7);
//       per tile the 16 warps split gate/up x 8 K slices of the tensor-core
//       GEMV whose n = 8 MMA columns are the expert's rows (warp_tile of the
//       batch path), the slices are summed in slice order, SwiGLU, and the
//       activations go out as flagged words, two units per word.
//   Dn  the CTA's down tiles (32 output rows) follow in the same ring, so
//       their copies start while gate/up tiles are computed; once all of
//       its expert's activations have arrived (published by the expert's
//       CTAs), fragments, GEMV, and the expert outputs y go out as flagged
//       words, two rows per word.
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
constexpr int RF_UR = 16;                     // gate/up units per tile
constexpr int RF_DR = 32;                     // down output rows per tile
constexpr int RF_NUT = RF_I / RF_UR;          // 96 gate/up tiles per expert
constexpr int RF_NDT = RF_H / RF_DR;          // 64 down tiles per expert
constexpr int RF_RB = RF_H * RF_BITS / 8;     // 1024 code bytes per gate/up row
constexpr int RF_RBD = RF_I * RF_BITS / 8;    // 768 per down row
constexpr int RF_NG = RF_H / RF_GS;           // 32 groups per gate/up row
constexpr int RF_NGD = RF_I / RF_GS;          // 24 per down row
constexpr int RF_RNG = RF_H / DEC_DGS;        // 32 groups per router row
constexpr int RF_SRB = 80;    // shared-memory bytes per gate/up scale row (64 + 16: consecutive rows change bank)
constexpr int RF_SRBD = 64;   // per down scale row (48 + 16)
constexpr int RF_XSU = RF_H / 2 + 16;   // fragment words per row (frag_stride_words), gate/up
constexpr int RF_XSD = RF_I / 2 + 16;   // down
constexpr int RF_GSU = RF_NG + 2;       // group-data entries per row (gdata_stride), gate/up
constexpr int RF_GSD = RF_NGD + 2;      // down
constexpr int RF_SLOT = 2 * RF_UR * RF_RB + 4 * RF_UR * RF_SRB;   // 37,888 B: one gate/up tile
constexpr int RF_MAX_SLOTS = 6;
constexpr int RF_MAX_CW = 64;           // output words per CTA
constexpr int RF_STAMPS = 16;
static_assert(RF_DR * RF_RBD + 2 * RF_DR * RF_SRBD <= RF_SLOT, "a down tile fits a slot");
static_assert(RF_SLOT % 128 == 0, "slots stay 128-byte aligned");
static_assert(RF_E == 64, "every router row has a CTA of its own");
static_assert(RF_XSU == RF_H / 2 + 16 && RF_XSD == RF_I / 2 + 16, "batch-path fragment strides (4-bit)");

// Fixed shared-memory header (byte offsets).
constexpr int RF_OFF_BARR = 0;       // router / norm tile barrier
constexpr int RF_OFF_BARS = 64;      // ring slot barriers (<= 8)
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
  int nslot;
  int off_x, off_xf, off_xg, off_red, off_slots;
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

// RMSNorm of T rows in place, each in the canonical 128-thread order (four
// rows per pass): x = bf16(w * bf16(h * r)), r = 1 / sqrt(sum(h^2) / H + eps)
// with the warp partials summed in warp order. Ends with a block sync.
YN_DEV void rf_rmsnorm_rows(uint16_t* x, const uint16_t* w, int T, float eps, float* red, float* rinv) {
  const int tid = threadIdx.x, q = tid >> 7, i = tid & 127;
  for (int t0 = 0; t0 < T; t0 += 4) {
    const int t = t0 + q;
    float ss = 0.0f;
    if (t < T)
      for (int j = i; j < RF_H; j += 128) {
        const float v = bf16_to_f32(x[(size_t)t * RF_H + j]);
        ss = __fmaf_rn(v, v, ss);
      }
    ss = group_sum_bfly(ss, 32);
    if ((tid & 31) == 0) red[tid >> 5] = ss;   // red[4 q + warp of the row]
    __syncthreads();
    if (tid < 4 && t0 + tid < T) {
      const float* r4 = red + 4 * tid;
      const float tot = __fadd_rn(__fadd_rn(__fadd_rn(r4[0], r4[1]), r4[2]), r4[3]);
      rinv[t0 + tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(tot, 1.0f / (float)RF_H), eps)));
    }
    __syncthreads();
  }
  for (int k = tid; k < T * RF_H; k += RF_THREADS) {
    const int t = k / RF_H, j = k % RF_H;
    x[k] = f32_to_bf16(__fmul_rn(bf16_to_f32(w[j]), bf16r(__fmul_rn(bf16_to_f32(x[k]), rinv[t]))));
  }
  __syncthreads();
}

// Batch-path fragments (the layout k_batch_frags writes) of n rows of Kd bf16
// values, rows[i] the source row of fragment row i: per row a power-of-two
// scale from max|x|, the fp16 pair words, and per group {-1024 * sum of the
// fragment values, scale * sum(x)}, then {1 / scale, 0}. Ends with a block
// sync.
template <int BITS, int GS>
YN_DEV void rf_frags(const uint16_t* src, int Kd, const int* rows, int n, uint32_t* XF, int xs_w, float2* XG,
                     int gsd, float* rsc) {
  using F = BFmt<BITS, GS>;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (warp < n) {
    const uint16_t* x = src + (size_t)rows[warp] * Kd;
    float mx = 0.0f;
    for (int k = lane; k < Kd; k += 32) mx = fmaxf(mx, fabsf(bf16_to_f32(x[k])));
    mx = warp_max(mx);
    if (lane == 0) rsc[warp] = fp16_input_scale(mx);
  }
  __syncthreads();
  const int hw = Kd / 2;
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
  const int NG = Kd / GS;
  for (int q = warp; q < n * NG; q += RF_WARPS) {
    const int r = q / NG, g = q - r * NG;
    const uint16_t* x = src + (size_t)rows[r] * Kd;
    const float scale = rsc[r];
    float sx = 0.0f, o = 0.0f;
    for (int k = g * GS + lane; k < (g + 1) * GS; k += 32) {
      const float v = bf16_to_f32(x[k]);
      sx = __fadd_rn(sx, v);
      const float m = __fmul_rn(scale, BW<BITS>::inv_mult(BW<BITS>::pair_of(k % F::WPL)));
      o = __fadd_rn(o, __half2float(__float2half_rn(__fmul_rn(v, m))));
    }
    sx = group_sum_bfly(sx, 32);
    o = group_sum_bfly(o, 32);
    if (lane == 0) XG[(size_t)r * gsd + g] = make_float2(__fmul_rn(-1024.0f, o), __fmul_rn(scale, sx));
  }
  if (tid < n) {
    XG[(size_t)tid * gsd + NG] = make_float2(__fdiv_rn(1.0f, rsc[tid]), 0.0f);
    XG[(size_t)tid * gsd + NG + 1] = make_float2(0.0f, 0.0f);
  }
  __syncthreads();
}

// Copies of ring item i of this CTA (gate/up tile u_t0 + i for i < n_up, else
// down tile d_t0 + i - n_up of the expert record `rec`) into slot S: every
// thread issues its 16-byte pieces and arrives (no-increment) on `bar`,
// which therefore completes when every piece has landed (count = threads).
YN_DEV void rf_issue(const uint8_t* rec, const RecGeom& rg, int i, int n_up, int u_t0, int d_t0, uint8_t* S,
                     uint64_t* bar) {
  const int tid = threadIdx.x;
  if (i < n_up) {
    const int u0 = (u_t0 + i) * RF_UR;
    constexpr int CPR = RF_RB / 16;   // 64 chunks per row
    for (int q = tid; q < 2 * RF_UR * CPR; q += RF_THREADS) {
      const int row = q / CPR, ch = q % CPR, mat = row / RF_UR, rr = row % RF_UR;
      cp16(S + (size_t)row * RF_RB + ((ch ^ (row & 7)) << 4),
           rec + rg.off[mat ? 3 : 0] + (size_t)(u0 + rr) * RF_RB + 16 * ch);
    }
    uint8_t* Sc = S + 2 * RF_UR * RF_RB;
    constexpr int SPR = RF_NG * 2 / 16;   // 4 chunks per scale row
    for (int q = tid; q < 4 * RF_UR * SPR; q += RF_THREADS) {
      const int pc = q / (RF_UR * SPR), rem = q % (RF_UR * SPR), rr = rem / SPR, ch = rem % SPR;
      const int piece = pc == 0 ? 1 : pc == 1 ? 2 : pc == 2 ? 4 : 5;   // gate s, gate b, up s, up b
      cp16(Sc + (size_t)(pc * RF_UR + rr) * RF_SRB + 16 * ch,
           rec + rg.off[piece] + (size_t)(u0 + rr) * (RF_NG * 2) + 16 * ch);
    }
  } else {
    const int r0 = (d_t0 + i - n_up) * RF_DR;
    constexpr int CPR = RF_RBD / 16;   // 48 chunks per row (a multiple of 8: the XOR stays in the row)
    for (int q = tid; q < RF_DR * CPR; q += RF_THREADS) {
      const int row = q / CPR, ch = q % CPR;
      cp16(S + (size_t)row * RF_RBD + ((ch ^ (row & 7)) << 4), rec + rg.off[6] + (size_t)(r0 + row) * RF_RBD + 16 * ch);
    }
    uint8_t* Sc = S + RF_DR * RF_RBD;
    constexpr int SPR = RF_NGD * 2 / 16;   // 3 chunks per scale row
    for (int q = tid; q < 2 * RF_DR * SPR; q += RF_THREADS) {
      const int pc = q / (RF_DR * SPR), rem = q % (RF_DR * SPR), rr = rem / SPR, ch = rem % SPR;
      cp16(Sc + (size_t)(pc * RF_DR + rr) * RF_SRBD + 16 * ch,
           rec + rg.off[pc ? 8 : 7] + (size_t)(r0 + rr) * (RF_NGD * 2) + 16 * ch);
    }
  }
  cp_arrive(bar);
}

__global__ void __launch_bounds__(RF_THREADS, 1) k_rows_flow(const RowsArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* barR = reinterpret_cast<uint64_t*>(smem + RF_OFF_BARR);
  uint64_t* barS = reinterpret_cast<uint64_t*>(smem + RF_OFF_BARS);
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
  float* RED = reinterpret_cast<float*>(smem + a.off_red);
  uint8_t* slots = smem + a.off_slots;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, c = lane & 3;
  const int G = gridDim.x, b = blockIdx.x, T = a.T, K = a.K, NS = a.nslot;
  const int W = T * (RF_H / 2);
  const int cw0 = (int)((long long)W * b / G), ncw = (int)((long long)W * (b + 1) / G) - cw0;
  const bool router_cta = b < RF_E;

  if (tid == 0) {
    mbar_init(barR, 1);
    for (int s = 0; s < NS; ++s) mbar_init(&barS[s], RF_THREADS);
    fence_mbar_init();
  }
  if (tid < 8) misc[16 + tid] = tid;
  load_layer(&lay[0], a.layers, 0);
  __syncthreads();
  if (tid == 0) rf_issue_rtile(lay[0], b, router_cta, smem, barR);
  uint32_t phR = 0, seq = 0;
  bool pendR = true;
  auto drain = [&]() {
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
    // this CTA's expert, its rows and its tiles
    const int d = (int)(((long long)(b + 1) * D - 1) / G);
    const int lo = (int)((long long)d * G / D), hi = (int)((long long)(d + 1) * G / D);
    const int r = b - lo, nd = hi - lo;
    const int e = elist[d];
    const uint32_t rm = rowmask[e];
    const int Td = __popc(rm), ps0 = pbase[e];
    const int u_t0 = RF_NUT * r / nd, n_up = RF_NUT * (r + 1) / nd - u_t0;
    const int d_t0 = RF_NDT * r / nd, n_dn = RF_NDT * (r + 1) / nd - d_t0;
    const int n_items = n_up + n_dn;
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
    const uint32_t base = seq;
    for (int i = 0; i < n_items && i < NS; ++i)
      rf_issue(rec, L.rg, i, n_up, u_t0, d_t0, slots + (size_t)((base + i) % NS) * RF_SLOT, &barS[(base + i) % NS]);
    __syncthreads();   // misc[8..16)
    rf_stamp(a, layer, 4);
    rf_frags<RF_BITS, RF_GS>(xb, RF_H, misc + 8, Td, XF, RF_XSU, XG, RF_GSU, rowf + 8);
    rf_stamp(a, layer, 5);
    // -------- GU: gate/up tiles, SwiGLU, activations out
    for (int i = 0; i < n_up; ++i) {
      const uint32_t q = base + i;
      uint8_t* S = slots + (size_t)(q % NS) * RF_SLOT;
      if (!mbar_wait_block(&barS[q % NS], (q / NS) & 1u, a.err)) { drain(); return; }
      const int mat = warp >> 3, ks = warp & 7;
      const uint16_t* Sc = reinterpret_cast<const uint16_t*>(S + 2 * RF_UR * RF_RB);
      constexpr int SH = RF_SRB / 2;
      // warp_tile reads the scale row of weight row r0 + g at S[(r0 + g) * SH]: gate rows are 0..15, up rows 16..31
      const uint16_t* Sm = Sc + (size_t)(mat ? 2 * RF_UR - RF_UR : 0) * SH;
      const uint16_t* Bm = Sc + (size_t)(mat ? 3 * RF_UR - RF_UR : RF_UR) * SH;
      float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
      warp_tile<RF_BITS, RF_GS, 1>(S, RF_RB, RF_UR * mat, Sm, Bm, SH, ks * 8, 8, XF, RF_XSU, XG, RF_GSU, Td, acc);
      float* rd = RED + (size_t)(mat * 8 + ks) * RF_UR * 8;
      rd[g * 8 + 2 * c] = acc[0][0];
      rd[g * 8 + 2 * c + 1] = acc[0][1];
      rd[(g + 8) * 8 + 2 * c] = acc[0][2];
      rd[(g + 8) * 8 + 2 * c + 1] = acc[0][3];
      __syncthreads();   // the slot is read: refill it
      if (i + NS < n_items) rf_issue(rec, L.rg, i + NS, n_up, u_t0, d_t0, S, &barS[q % NS]);
      if (tid < 8 * Td) {
        const int tl = tid >> 3, up = tid & 7;
        const float inv = XG[(size_t)tl * RF_GSU + RF_NG].x;
        uint32_t pk = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int u = 2 * up + h;
          float gs = 0.0f, us = 0.0f;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            gs = __fadd_rn(gs, RED[((size_t)k * RF_UR + u) * 8 + tl]);
            us = __fadd_rn(us, RED[((size_t)(8 + k) * RF_UR + u) * 8 + tl]);
          }
          const float gv = bf16r(__fmul_rn(gs, inv)), uv = bf16r(__fmul_rn(us, inv));
          pk |= (uint32_t)f32_to_bf16(swiglu_bf16(gv, uv)) << (16 * h);
        }
        put_flag(a.f_act + ((size_t)par * a.P + ps0 + tl) * (RF_I / 2) + ((u_t0 + i) * RF_UR) / 2 + up, pk, ep);
      }
      // the next wait's block sync orders these RED reads before the next tile's writes
    }
    rf_stamp(a, layer, 6);
    // -------- Dn: the expert's activations of all its rows, fragments, down tiles
    rf_wait_words(a.f_act + ((size_t)par * a.P + ps0) * (RF_I / 2), reinterpret_cast<uint32_t*>(xb), Td * (RF_I / 2),
                  ep, a.err, fail);
    if (__syncthreads_or(fail)) { drain(); return; }
    rf_stamp(a, layer, 7);
    rf_frags<RF_BITS, RF_GS>(xb, RF_I, misc + 16, Td, XF, RF_XSD, XG, RF_GSD, rowf + 8);
    rf_stamp(a, layer, 8);
    for (int i = n_up; i < n_items; ++i) {
      const uint32_t q = base + i;
      uint8_t* S = slots + (size_t)(q % NS) * RF_SLOT;
      if (!mbar_wait_block(&barS[q % NS], (q / NS) & 1u, a.err)) { drain(); return; }
      const int rs = warp & 1, ks = warp >> 1;
      const uint16_t* Sd = reinterpret_cast<const uint16_t*>(S + RF_DR * RF_RBD);
      constexpr int SH = RF_SRBD / 2;
      float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
      warp_tile<RF_BITS, RF_GS, 1>(S, RF_RBD, 16 * rs, Sd, Sd + (size_t)RF_DR * SH, SH, ks * 6, 6, XF, RF_XSD, XG,
                                   RF_GSD, Td, acc);
      float* rd = RED + (size_t)ks * RF_DR * 8;
      const int ra = 16 * rs + g;
      rd[ra * 8 + 2 * c] = acc[0][0];
      rd[ra * 8 + 2 * c + 1] = acc[0][1];
      rd[(ra + 8) * 8 + 2 * c] = acc[0][2];
      rd[(ra + 8) * 8 + 2 * c + 1] = acc[0][3];
      __syncthreads();
      if (i + NS < n_items) rf_issue(rec, L.rg, i + NS, n_up, u_t0, d_t0, S, &barS[q % NS]);
      if (tid < 16 * Td) {
        const int tl = tid >> 4, rp = tid & 15;
        const float inv = XG[(size_t)tl * RF_GSD + RF_NGD].x;
        uint32_t pk = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = 2 * rp + h;
          float y = 0.0f;
#pragma unroll
          for (int k = 0; k < 8; ++k) y = __fadd_rn(y, RED[((size_t)k * RF_DR + row) * 8 + tl]);
          pk |= (uint32_t)f32_to_bf16(__fmul_rn(y, inv)) << (16 * h);
        }
        const int r0 = (d_t0 + i - n_up) * RF_DR;
        put_flag(a.f_y + ((size_t)par * a.P + ps0 + tl) * (RF_H / 2) + r0 / 2 + rp, pk, ep);
      }
    }
    seq = base + (uint32_t)n_items;
    rf_stamp(a, layer, 9);
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
    rf_stamp(a, layer, 10);
  }
  drain();
}

}  // namespace ynb
