// Persistent whole-stack bs1 decode in data-flow form: no grid barriers.
//
// Same compiled shape, same arithmetic and the same building blocks as
// k_stack_decode (yn_decode.cuh), with the work of a layer split by expert
// instead of by output row, so that every exchange between CTAs is a small
// set of flagged words that each consumer reads directly:
//
//   P1  (every CTA) h -> RMSNorm -> its slice of the router rows (logits
//       published as flagged words, as in k_stack_decode) and of the shared
//       expert's gate/up rows (its SwiGLU activations published one unit per
//       flagged word; the shared_expert_gate published as one more word).
//   R   (every CTA) routing of the 512 logits, redundantly.
//   P2r (K groups of `nr` CTAs; group j owns routed column j) CTA r of group
//       j copies the gate/up rows of its units of expert ids[j] and, at the
//       same time, its own 16-row blocks of the expert's down rows; computes
//       its units' SwiGLU activations and publishes them (two units per
//       word); then reads the expert's 512 activations back (256 words,
//       published by the group's CTAs), builds the down-projection
//       fragments and computes its down rows: y_j published as flagged words,
//       two rows per word.
//   P2s (the remaining `ns` CTAs) read the shared expert's 512 activations
//       and gate, compute their blocks of the shared down rows (weights
//       copied during the previous layer) and publish sigmoid(g) * y_shared.
//   P3  (every CTA) its 6-7 words of output rows: the K routed y and the
//       shared term of those rows, the weighted combine in column order and
//       the residual; published as flagged words (the next layer's input),
//       or written to `outputs` after the last layer.
//
// A flagged word is {32-bit payload, epoch}, epoch = step + 1, stored with
// one relaxed 64-bit store; a consumer polls the word until its epoch shows
// (the data read is the synchronisation). Every buffer is double-buffered by
// step parity. A buffer of parity p is written again only two steps later,
// and every writer of step s+2 has, through the routing of step s+2, waited
// for every CTA's router slice of step s+2, which each CTA computes after it
// has finished reading step s's words. Every wait has a wall-clock limit and
// watches the error word; on an error each CTA lets its copies in flight land
// and returns.
//
// Each routed y and each output row is computed by the same fp32 operations
// in the same order as in k_stack_decode, so the two kernels give identical
// outputs. Reference behaviour: moe_prefetch/orchestrator.py:308-343 with
// every expert resident (mlx_backend.py:302-316, :442-459, :438-440).
#pragma once
#include "yn_decode.cuh"

namespace ynb {

constexpr int FL_MAX_DT = 16;   // 16-row down blocks per CTA
constexpr int FL_MAX_CW = 16;   // combine words per CTA
constexpr int FL_HW = DEC_H / 2;  // words of a hidden row
constexpr int FL_AW = DEC_I / 2;  // words of a routed activation vector

struct FlowArgs {
  int K, Ish, norm_topk;
  float eps;
  const DecLayer* layers;
  int n_layers;
  const uint16_t* inputs;
  int n_tokens;
  uint16_t* outputs;
  u64* f_logits;  // (2, E) router logits (fp32)
  u64* f_act;     // (2, K, I/2) routed SwiGLU activations, two bf16 per word
  u64* f_ash;     // (2, Ish + 1) shared-expert activations (one bf16 per word), then the shared gate (fp32)
  u64* f_y;       // (2, K + 1, H/2) routed bf16(y_j) and the gated shared term, two rows per word
  u64* f_h;       // (2, H/2) layer outputs, two bf16 per word
  int32_t* trace_ids;
  uint16_t* trace_h;
  float* trace_w;
  int* err;
  long long* timing;
  int nr, ns;  // CTAs per routed column, shared-down CTAs
  int off_hs, off_xs, off_route, off_xf2, off_xf3, off_part, off_stage, off_A, off_C, off_D;
  int c_rows, c_rb, c_sb;  // gate/up tile: rows reserved per block, bytes per code / scale row (largest format)
  int d_rows, d_rb, d_sb;  // down tile: rows reserved, bytes per code / scale row (largest format)
};

YN_DEV void stamp(const FlowArgs& a, int tok, int layer, int slot) {
  if (a.timing && tok == a.n_tokens - 1) stamp_at(a.timing, layer, slot);
}

// P1 compute of the data-flow kernel: k_stack_decode's p1_compute with the
// shared activations and gate published as flagged words.
YN_DEV void p1_compute_flow(const FlowArgs& a, const P1Range& r, const P1Tile& t, const uint16_t* xs,
                            const float* rbias_s, float* gu, int par, uint32_t ep) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int LPR = 32, CPL = DEC_H / 16 / LPR;
  constexpr int NGD = DEC_H / DEC_DGS;
  XF32<8, CPL, 1> X;
  load_x_f32<8, CPL, 1>(X, xs, lane, LPR);
  const int nr = r.r1 - r.r0, np = r.p1 - r.p0;
  const int ntask = nr + 2 * np + r.sg;
  u64* ash = a.f_ash + (size_t)par * (a.Ish + 1);
  for (int k = warp; k < ntask; k += DEC_WARPS) {
    const uint8_t* cr;
    const uint16_t* sr;
    const uint16_t* br;
    if (k < nr) {
      cr = t.rc + (size_t)k * DEC_H; sr = t.rs + k * NGD; br = t.rbv + k * NGD;
    } else if (k < nr + 2 * np) {
      const int q = k - nr, p = q >> 1;
      if (q & 1) { cr = t.uc + (size_t)p * DEC_H; sr = t.usc + p * NGD; br = t.ubi + p * NGD; }
      else { cr = t.gc + (size_t)p * DEC_H; sr = t.gsc + p * NGD; br = t.gbi + p * NGD; }
    } else {
      cr = t.sc; sr = t.ssc; br = t.sbi;
    }
    float v = row_dot_f32<8, CPL, 1>(cr, sr, br, X, lane, LPR, DEC_DGS);
    v = group_sum_bfly(v, LPR);
    if (lane == 0) {
      if (k < nr) put_flag(a.f_logits + par * DEC_E + r.r0 + k, __float_as_uint(bf16r(__fadd_rn(v, rbias_s[k]))), ep);
      else if (k < nr + 2 * np) gu[k - nr] = bf16r(v);
      else put_flag(ash + a.Ish, __float_as_uint(bf16r(sigmoid_f32(bf16r(v)))), ep);
    }
  }
  __syncthreads();
  for (int p = threadIdx.x; p < np; p += DEC_THREADS)
    put_flag(ash + r.p0 + p, (uint32_t)f32_to_bf16(swiglu_bf16(gu[2 * p], gu[2 * p + 1])), ep);
}

// Fragments, group sums and the power-of-two scale of one 512-element bf16
// vector in shared memory, built by the whole block (identical values to
// k_stack_decode's per-warp p3_frags). Ends with a block sync.
template <int BITS, int GS>
YN_DEV void vec_frags(const uint16_t* x, uint32_t* xf, float* xsum, float* off, float* xsc, float* red) {
  using S = Sb<BITS>;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float m = 0.0f;
  if (tid < DEC_I / 2) {
    const uint32_t w = reinterpret_cast<const uint32_t*>(x)[tid];
    m = fmaxf(fabsf(bf16_to_f32((uint16_t)(w & 0xFFFFu))), fabsf(bf16_to_f32((uint16_t)(w >> 16))));
  }
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  const float scale = fp16_input_scale(warp_max(red[lane & 15]));
  if (tid < DEC_I / 2) {
    const int sb = tid / (4 * S::FRAG), rem = tid % (4 * S::FRAG);
    xf[tid] = frag_word<BITS>(x, scale, sb, rem / S::FRAG, rem % S::FRAG);
  }
  if (warp == 0) group_sums16<BITS, GS>(x, lane, true, scale, xsum, off);
  if (tid == 0) *xsc = scale;
  __syncthreads();
}

// Down-projection dots of `ndt` 16-row blocks (codes [rows][RBI], scales and
// biases [rows][SBI]) against one vector's fragments: part[row * NSB + sb].
template <int BITS, int GS>
YN_DEV void down_blocks(const uint8_t* D, const uint8_t* Ds, const uint8_t* Db, int ndt, const uint32_t* xf,
                        const float* xsum, const float* off, float inv, float* part) {
  constexpr int RBI = DEC_I * BITS / 8, SBI = DEC_I / GS * 2, NSB = RBI / 64, NG = DEC_I / GS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  for (int it = warp; it < ndt * NSB; it += DEC_WARPS) {
    const int q = it / NSB, sb = it % NSB;
    const int row = 16 * q + g;
    float d[4];
    sb_mma<BITS, GS>(D + (size_t)row * RBI + sb * 64 + c * 16, D + (size_t)(row + 8) * RBI + sb * 64 + c * 16,
                     xf + (sb * 4 + c) * Sb<BITS>::FRAG, g, c, d);
    const uint16_t* s0 = reinterpret_cast<const uint16_t*>(Ds + (size_t)row * SBI);
    const uint16_t* b0 = reinterpret_cast<const uint16_t*>(Db + (size_t)row * SBI);
    const float v0 = sb_apply<BITS, GS>(d[0], d[1], s0, b0, xsum, off, sb, c, inv);
    const float v1 = sb_apply<BITS, GS>(d[2], d[3], s0 + 8 * NG, b0 + 8 * NG, xsum, off, sb, c, inv);
    if (c == 0) {
      part[row * NSB + sb] = v0;
      part[(row + 8) * NSB + sb] = v1;
    }
  }
}

// Row sums of `down_blocks` (super-blocks in order) for rows 2i, 2i+1 of the
// CTA's blocks, as one word of two bf16: bf16(y) (routed) or
// bf16(gate * bf16(y)) (shared, gate given).
template <int NSB>
YN_DEV uint32_t y_word(const float* part, int i, bool shared, float gate) {
  uint32_t pk = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float y = 0.0f;
#pragma unroll
    for (int q = 0; q < NSB; ++q) y = __fadd_rn(y, part[(2 * i + h) * NSB + q]);
    const float o = shared ? bf16r(__fmul_rn(gate, bf16r(y))) : bf16r(y);
    pk |= (uint32_t)f32_to_bf16(o) << (16 * h);
  }
  return pk;
}

// Bulk copies of `rows` rows (from row `r0`) of a down piece triple (codes
// of `rb` bytes per row, scales and biases of `sb` bytes per row) into
// D / Ds / Db, completing on `bar` (count 1). One thread.
YN_DEV void issue_down(const uint8_t* w, const uint8_t* s, const uint8_t* b, int r0, int rows, int rb, int sb,
                       uint8_t* D, uint8_t* Ds, uint8_t* Db, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, (uint32_t)rows * (uint32_t)(rb + 2 * sb));
  if (rows <= 0) return;
  bulk_g2s(D, w + (size_t)r0 * rb, (uint32_t)rows * rb, bar);
  bulk_g2s(Ds, s + (size_t)r0 * sb, (uint32_t)rows * sb, bar);
  bulk_g2s(Db, b + (size_t)r0 * sb, (uint32_t)rows * sb, bar);
}

__global__ void __launch_bounds__(DEC_THREADS, 1) k_stack_flow(const FlowArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* barA = reinterpret_cast<uint64_t*>(smem);        // P1 tile (+ layer descriptor)
  uint64_t* barD = barA + 1;                                  // routed down rows
  uint64_t* barS = barA + 2;                                  // shared down rows
  float* red = reinterpret_cast<float*>(smem + 32);           // 24 floats
  int* ids_ok_s = reinterpret_cast<int*>(smem + 132);
  uint64_t* barT = reinterpret_cast<uint64_t*>(smem + 136);  // DEC_MAX_OCT gate/up tile barriers
  uint16_t* hs = reinterpret_cast<uint16_t*>(smem + a.off_hs);
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem + a.off_xs);
  uint8_t* rt = smem + a.off_route;
  float* rv = reinterpret_cast<float*>(rt);                               // E
  uint32_t* cand = reinterpret_cast<uint32_t*>(rt + 4 * DEC_E);           // 16 * 16
  int32_t* ids = reinterpret_cast<int32_t*>(cand + DEC_WARPS * DEC_MAX_K);
  float* wts = reinterpret_cast<float*>(ids + DEC_MAX_K);
  float* misc = wts + DEC_MAX_K;                                          // [0] vector scale, [1] shared gate
  float* rbias_s = misc + DEC_MAX_K + 4;                                  // 64
  float* gu = rbias_s + 64;                                               // 256
  DecLayer* lay = reinterpret_cast<DecLayer*>(gu + 256);                  // 3 slots
  uint32_t* xf2 = reinterpret_cast<uint32_t*>(smem + a.off_xf2);          // H / 2 words
  float* xsum2 = reinterpret_cast<float*>(xf2 + DEC_H / 2);               // H / 32 sums + H / 32 offsets
  uint32_t* xf3 = reinterpret_cast<uint32_t*>(smem + a.off_xf3);          // I / 2 words
  float* xsum3 = reinterpret_cast<float*>(xf3 + DEC_I / 2);               // 16 sums
  float* off3 = xsum3 + 16;                                               // 16 offsets
  float* part = reinterpret_cast<float*>(smem + a.off_part);
  uint16_t* stage = reinterpret_cast<uint16_t*>(smem + a.off_stage);      // I bf16
  uint32_t* ys = reinterpret_cast<uint32_t*>(stage + DEC_I);              // (K + 1) * FL_MAX_CW words
  uint8_t* Abuf = smem + a.off_A;
  uint8_t* C = smem + a.off_C;
  uint8_t* D = smem + a.off_D;

  const int tid = threadIdx.x, warp = tid >> 5;
  const int G = gridDim.x, b = blockIdx.x, K = a.K;
  const int nrt = K * a.nr;
  const bool routed = b < nrt;
  const int col = routed ? b / a.nr : K;               // routed column, or K: the shared expert
  const int part_i = routed ? b % a.nr : b - nrt;
  const int nparts = routed ? a.nr : a.ns;
  const int t0 = routed ? (DEC_I / 8) * part_i / nparts : 0;
  const int ntile = routed ? (DEC_I / 8) * (part_i + 1) / nparts - t0 : 0;
  const int q0 = (DEC_H / 16) * part_i / nparts;
  const int ndt = (DEC_H / 16) * (part_i + 1) / nparts - q0;   // 16-row down blocks
  CSeg sg;
  sg.n = ntile ? 1 : 0;
  sg.j[0] = sg.j[1] = col;
  sg.n0[0] = sg.n0[1] = 8 * t0;
  sg.rows[0] = 8 * ntile;
  sg.rows[1] = 0;
  const int cw0 = FL_HW * b / G, ncw = FL_HW * (b + 1) / G - cw0;   // combine words
  const int nsrc = K + (a.Ish ? 1 : 0);
  const P1Range r1 = p1_range(b, G, a.Ish);
  const int nr1 = r1.r1 - r1.r0;
  const int total_steps = a.n_tokens * a.n_layers;
  // down tile pieces (routed: codes / scales / biases of up to d_rows rows; shared: 8-bit rows over C and D)
  uint8_t* Dw = routed ? D : C;
  uint8_t* Dsc = routed ? D + (size_t)a.d_rows * a.d_rb : C + (size_t)ndt * 16 * DEC_I;
  uint8_t* Dbi = routed ? Dsc + (size_t)a.d_rows * a.d_sb : Dsc + (size_t)ndt * 16 * DEC_DSBI;

  if (tid == 0) {
    mbar_init(barA, DEC_THREADS);
    mbar_init(barD, 1);
    mbar_init(barS, 1);
    for (int t = 0; t < DEC_MAX_OCT; ++t) mbar_init(&barT[t], 1);
    fence_mbar_init();
  }
  if (tid < 8) reinterpret_cast<uint32_t*>(smem + DEC_ZERO_OFF)[tid] = 0u;
  load_layer(&lay[0], a.layers, 0);
  load_layer(&lay[1], a.layers, a.n_layers > 1 ? 1 : 0);
  __syncthreads();
  issue_p1(lay[0], r1, p1_tile(Abuf, r1), barA, 0);
  const bool sh_work = !routed && a.Ish && ndt > 0;
  if (sh_work && tid == 0) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    issue_down(lay[0].sd.w, reinterpret_cast<const uint8_t*>(lay[0].sd.s), reinterpret_cast<const uint8_t*>(lay[0].sd.b),
               16 * q0, 16 * ndt, DEC_I, DEC_DSBI, Dw, Dsc, Dbi, barS);
  }
  uint32_t phA = 0, phT = 0, phD = 0, phS = 0;
  bool pendA = true, pendT = false, pendD = false, pendS = sh_work;
  auto drain = [&]() {
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (pendA) mbar_wait_block(barA, phA, nullptr);
    if (pendT)
      for (int t = 0; t < ntile; ++t) mbar_wait_block(&barT[t], phT, nullptr);
    if (pendD) mbar_wait_block(barD, phD, nullptr);
    if (pendS) mbar_wait_block(barS, phS, nullptr);
  };

  for (int step = 0; step < total_steps; ++step) {
    const int tok = step / a.n_layers, layer = step % a.n_layers;
    const DecLayer& L = lay[step % 3];
    const DecLayer& Ln = lay[(step + 1) % 3];
    const bool more = step + 1 < total_steps;
    const int fmt = fmt_of(L);
    const int par = step & 1;
    const uint32_t ep = (uint32_t)step + 1;
    stamp(a, tok, layer, 0);
    // -------- P1 input: the token row, or the previous layer's published output
    bool fail = false;
    if (layer == 0) {
      if (tid < DEC_H / 8)
        reinterpret_cast<uint4*>(hs)[tid] = __ldcg(reinterpret_cast<const uint4*>(a.inputs + (size_t)tok * DEC_H) + tid);
    } else {
      const u64* fh = a.f_h + (size_t)((step - 1) & 1) * FL_HW;
      reinterpret_cast<uint32_t*>(hs)[tid] = wait_flag(fh + tid, (uint32_t)step, a.err, fail);
      reinterpret_cast<uint32_t*>(hs)[tid + DEC_THREADS] = wait_flag(fh + tid + DEC_THREADS, (uint32_t)step, a.err, fail);
    }
    if (tid < 64) rbias_s[tid] = (tid < nr1 && L.rbias) ? __ldcg(L.rbias + r1.r0 + tid) : 0.0f;
    if (__syncthreads_or(fail)) { drain(); return; }
    if (a.trace_h && b == 0 && tid < DEC_H / 8)
      reinterpret_cast<uint4*>(a.trace_h + ((size_t)tok * a.n_layers + layer) * DEC_H)[tid] =
          reinterpret_cast<const uint4*>(hs)[tid];
    const P1Tile t1 = p1_tile(Abuf, r1);
    stamp(a, tok, layer, 1);
    if (!mbar_wait_block(barA, phA, a.err)) { drain(); return; }
    phA ^= 1;
    pendA = false;
    stamp(a, tok, layer, 2);
    const float xscale2 = fp16_input_scale(rmsnorm_smem(hs, t1.norm, a.eps, xs, red));
    stamp(a, tok, layer, 3);
    p1_compute_flow(a, r1, t1, xs, rbias_s, gu, par, ep);
    if (routed) {
      switch (fmt) {
        case 0: p2_frags<2, 64>(xs, xscale2, xf2, xsum2); break;
        case 1: p2_frags<2, 32>(xs, xscale2, xf2, xsum2); break;
        case 2: p2_frags<4, 64>(xs, xscale2, xf2, xsum2); break;
        default: p2_frags<4, 32>(xs, xscale2, xf2, xsum2); break;
      }
    }
    stamp(a, tok, layer, 4);
    // -------- routing (every CTA: the combine needs the weights)
    if (!route_block(a.f_logits + par * DEC_E, ep, a.err, K, a.norm_topk, rv, cand, red, ids, wts, L, ids_ok_s)) {
      drain();
      return;
    }
    if (b == 0 && tid < K) {
      if (a.trace_ids) a.trace_ids[((size_t)tok * a.n_layers + layer) * K + tid] = ids[tid];
      if (a.trace_w) a.trace_w[((size_t)tok * a.n_layers + layer) * K + tid] = wts[tid];
    }
    if (*ids_ok_s == 0) {   // block-uniform (set before routing's last sync)
      if (tid == 0) raise_error(a.err, YN_ERR_BAD_SLOT);
      drain();
      return;
    }
    stamp(a, tok, layer, 5);
    if (routed) {
      // -------- P2r: gate/up rows (tile by tile) and this CTA's down rows, issued together
      const int RBI = DEC_I * L.rg.bits / 8, SBI = DEC_I / L.rg.gs * 2;
      // one warp per tile (warp DEC_WARPS - 1 - t issues tile t), so the issue is not one warp's serial chain
      if (warp >= DEC_WARPS - DEC_MAX_OCT) {
        const int tw = DEC_WARPS - 1 - warp;
        switch (fmt) {
          case 0: copy_c<2, 64>(a, L, ids, sg, ntile, C, barT, tw, DEC_MAX_OCT); break;
          case 1: copy_c<2, 32>(a, L, ids, sg, ntile, C, barT, tw, DEC_MAX_OCT); break;
          case 2: copy_c<4, 64>(a, L, ids, sg, ntile, C, barT, tw, DEC_MAX_OCT); break;
          default: copy_c<4, 32>(a, L, ids, sg, ntile, C, barT, tw, DEC_MAX_OCT); break;
        }
      } else if (tid == 32 * (DEC_WARPS - DEC_MAX_OCT - 1)) {
        const uint8_t* rec = expert_record(L, ids[col]);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue_down(rec + L.rg.off[6], rec + L.rg.off[7], rec + L.rg.off[8], 16 * q0, 16 * ndt, RBI, SBI, Dw, Dsc, Dbi,
                   barD);
      }
      pendT = pendD = true;
    }
    stamp(a, tok, layer, 6);
    if (routed) {
      const float inv2 = __frcp_rn(xscale2);
      switch (fmt) {
        case 0: p2_tiles<2, 64>(a, ntile, C, xf2, xsum2, inv2, part, barT, phT); break;
        case 1: p2_tiles<2, 32>(a, ntile, C, xf2, xsum2, inv2, part, barT, phT); break;
        case 2: p2_tiles<4, 64>(a, ntile, C, xf2, xsum2, inv2, part, barT, phT); break;
        default: p2_tiles<4, 32>(a, ntile, C, xf2, xsum2, inv2, part, barT, phT); break;
      }
      phT ^= 1;
      pendT = false;
      __syncthreads();
      // SwiGLU of this CTA's units, one unit per thread (gate/up sums over the super-blocks in
      // order), published two units per word by the even thread
      if (warp < DEC_MAX_OCT * 8 / 32) {
        const int NSB = DEC_H * L.rg.bits / 8 / 64, u = tid;
        uint32_t v = 0;
        if (u < 8 * ntile) {
          float gsum = 0.0f, usum = 0.0f;
          for (int q = 0; q < NSB; ++q) {
            gsum = __fadd_rn(gsum, part[(u * 2 + 0) * NSB + q]);
            usum = __fadd_rn(usum, part[(u * 2 + 1) * NSB + q]);
          }
          v = (uint32_t)f32_to_bf16(swiglu_bf16(bf16r(gsum), bf16r(usum)));
        }
        const uint32_t hi = __shfl_down_sync(0xffffffffu, v, 1);
        if (u < 8 * ntile && !(u & 1))
          put_flag(a.f_act + ((size_t)par * K + col) * FL_AW + 4 * t0 + (u >> 1), v | (hi << 16), ep);
      }
    }
    stamp(a, tok, layer, 7);
    float gate = 0.0f;
    if (routed) {
      // -------- P2r: the expert's 512 activations back, down rows
      if (tid < FL_AW)
        reinterpret_cast<uint32_t*>(stage)[tid] = wait_flag(a.f_act + ((size_t)par * K + col) * FL_AW + tid, ep, a.err, fail);
      if (__syncthreads_or(fail)) { drain(); return; }
      switch (fmt) {
        case 0: vec_frags<2, 64>(stage, xf3, xsum3, off3, misc, red); break;
        case 1: vec_frags<2, 32>(stage, xf3, xsum3, off3, misc, red); break;
        case 2: vec_frags<4, 64>(stage, xf3, xsum3, off3, misc, red); break;
        default: vec_frags<4, 32>(stage, xf3, xsum3, off3, misc, red); break;
      }
      if (!mbar_wait_block(barD, phD, a.err)) { drain(); return; }
      phD ^= 1;
      pendD = false;
      const float inv3 = __frcp_rn(misc[0]);
      switch (fmt) {
        case 0: down_blocks<2, 64>(Dw, Dsc, Dbi, ndt, xf3, xsum3, off3, inv3, part); break;
        case 1: down_blocks<2, 32>(Dw, Dsc, Dbi, ndt, xf3, xsum3, off3, inv3, part); break;
        case 2: down_blocks<4, 64>(Dw, Dsc, Dbi, ndt, xf3, xsum3, off3, inv3, part); break;
        default: down_blocks<4, 32>(Dw, Dsc, Dbi, ndt, xf3, xsum3, off3, inv3, part); break;
      }
      __syncthreads();
    } else if (sh_work) {
      // -------- P2s: the shared expert's activations and gate, its down rows
      const u64* ash = a.f_ash + (size_t)par * (a.Ish + 1);
      for (int u = tid; u < a.Ish; u += DEC_THREADS) stage[u] = (uint16_t)wait_flag(ash + u, ep, a.err, fail);
      if (tid == 0) misc[1] = __uint_as_float(wait_flag(ash + a.Ish, ep, a.err, fail));
      if (__syncthreads_or(fail)) { drain(); return; }
      vec_frags<8, DEC_DGS>(stage, xf3, xsum3, off3, misc, red);
      if (!mbar_wait_block(barS, phS, a.err)) { drain(); return; }
      phS ^= 1;
      pendS = false;
      down_blocks<8, DEC_DGS>(Dw, Dsc, Dbi, ndt, xf3, xsum3, off3, __frcp_rn(misc[0]), part);
      __syncthreads();
      gate = misc[1];
    }
    stamp(a, tok, layer, 8);
    if (routed || sh_work) {
      // y words of this CTA's down rows (8 per 16-row block)
      const int NSBv = routed ? DEC_I * L.rg.bits / 8 / 64 : DEC_I / 64;
      u64* fy = a.f_y + ((size_t)par * (K + 1) + col) * FL_HW + 8 * q0;
      for (int i = tid; i < 8 * ndt; i += DEC_THREADS) {
        const uint32_t pk = NSBv == 2 ? y_word<2>(part, i, false, 0.0f)
                            : NSBv == 4 ? y_word<4>(part, i, false, 0.0f)
                                        : y_word<8>(part, i, !routed, gate);
        put_flag(fy + i, pk, ep);
      }
      if (!routed && more) {   // the next layer's shared down rows, once every read of this layer's has run
        __syncthreads();
        if (tid == 0) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          issue_down(Ln.sd.w, reinterpret_cast<const uint8_t*>(Ln.sd.s), reinterpret_cast<const uint8_t*>(Ln.sd.b),
                     16 * q0, 16 * ndt, DEC_I, DEC_DSBI, Dw, Dsc, Dbi, barS);
        }
        pendS = true;
      }
    }
    // next layer's P1 tile (and the descriptor of layer step + 2) while the row exchange runs
    if (step + 2 < total_steps) load_layer_async(&lay[(step + 2) % 3], a.layers, (step + 2) % a.n_layers);
    if (more) issue_p1(Ln, r1, p1_tile(Abuf, r1), barA, 0);
    pendA = more;
    stamp(a, tok, layer, 9);
    // -------- P3: this CTA's output rows: routed y, shared term, combine, residual
    for (int i = tid; i < nsrc * ncw; i += DEC_THREADS) {
      const int s = i / ncw, w = i % ncw;
      ys[s * FL_MAX_CW + w] = wait_flag(a.f_y + ((size_t)par * (K + 1) + s) * FL_HW + cw0 + w, ep, a.err, fail);
    }
    if (__syncthreads_or(fail)) { drain(); return; }
    stamp(a, tok, layer, 10);
    if (tid < ncw) {
      const bool last = layer == a.n_layers - 1;
      uint32_t pk = 0;
      for (int h = 0; h < 2; ++h) {
        const int row = 2 * (cw0 + tid) + h;
        float acc = 0.0f;
        for (int j = 0; j < K; ++j) {
          const float y = bf16_to_f32((uint16_t)(ys[j * FL_MAX_CW + tid] >> (16 * h)));
          acc = __fadd_rn(acc, bf16r(__fmul_rn(y, wts[j])));
        }
        float o = bf16r(acc);
        if (a.Ish) o = bf16r(__fadd_rn(o, bf16_to_f32((uint16_t)(ys[K * FL_MAX_CW + tid] >> (16 * h)))));
        o = bf16r(__fadd_rn(bf16_to_f32(hs[row]), o));
        pk |= (uint32_t)f32_to_bf16(o) << (16 * h);
      }
      if (last) reinterpret_cast<uint32_t*>(a.outputs + (size_t)tok * DEC_H)[cw0 + tid] = pk;
      else put_flag(a.f_h + (size_t)par * FL_HW + cw0 + tid, pk, ep);
    }
    stamp(a, tok, layer, 11);
    stamp(a, tok, layer, 12);
    stamp(a, tok, layer, 13);
    stamp(a, tok, layer, 14);
    stamp(a, tok, layer, 15);
    // hs (the residual), ys and the routing weights are read above; the next
    // step overwrites them (a token's first layer without waiting for anything)
    __syncthreads();
  }
  // copies issued for a step that does not come (none with `more` false) are none; let the last land
  drain();
}

}  // namespace ynb
