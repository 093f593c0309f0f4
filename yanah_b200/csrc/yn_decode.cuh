// Persistent whole-stack bs1 decode kernel (one cooperative launch decodes
// n_tokens tokens sequentially through every layer).
//
// Grid = one CTA per SM (co-resident, cooperative launch), 256 threads.
// Per layer three phases separated by grid barriers:
//   P1  RMSNorm(h) -> router logits, shared-expert gate/up/SwiGLU, shared gate
//       (each CTA owns a byte-balanced slice of those rows; the tiles were
//       prefetched into shared memory one whole layer earlier)
//   P2  routing (every CTA, redundantly, from the 512 logits) -> each CTA
//       issues bulk copies for its slice of routed gate/up rows (C tiles) and
//       of the down rows it will need in P3 (D tiles), then computes its
//       gate/up rows -> SwiGLU activations
//   P3  each CTA owns a contiguous block of output rows: routed + shared down
//       projections for those rows, the weighted combine in column order and
//       the residual -> next h
// Grid barriers are a global counter (release add / acquire poll) with a
// wall-clock limit; on any error every CTA skips work and leaves at the next
// barrier. Reference behaviour: orchestrator.py:308-343 layer loop with
// every expert resident; arithmetic as in the separate layer kernels.
#pragma once
#include "yn_common.cuh"
#include "yn_moe.cuh"
#include "yn_qdot.cuh"

namespace ynb {

constexpr int DEC_THREADS = 256;
constexpr int DEC_WARPS = DEC_THREADS / 32;
constexpr int DEC_MAX_K = 16;
constexpr int DEC_MAX_DROWS = 32;  // output rows per CTA in P3

struct DecLayer {
  const uint16_t* norm;
  QM router;
  const float* rbias;
  QM sg, su, sd, sgt;  // shared gate_proj, up_proj, down_proj, shared_expert_gate
  const uint8_t* ebase;
  long long stride;
  const int32_t* slot_of;
  int n_slots;
  RecGeom rg;
};

struct DecodeArgs {
  int H, E, K, I, Ish, norm_topk;
  float eps;
  const DecLayer* layers;
  int n_layers;
  const uint16_t* inputs;
  int n_tokens;
  uint16_t* outputs;
  uint16_t* hbuf;      // (2, H)
  float* logits;       // (E)
  uint16_t* act;       // (K, I)
  uint16_t* act_sh;    // (Ish)
  float* sgate;        // (1)
  int32_t* trace_ids;  // (n_tokens, n_layers, K) or null
  unsigned* bar;
  int* err;
  long long* timing;   // (n_layers, 8) for token 0, or null
  // shared-memory carve (byte offsets)
  int off_hs, off_xs, off_act, off_actsh, off_route, off_y, off_A0, off_A1, off_C, off_D;
};

// ---------------------------------------------------------------- barrier
// Returns true (block-uniform) when the error word is set after the barrier.
YN_DEV bool grid_barrier(const DecodeArgs& a, unsigned& gen, int* flag) {
  __syncthreads();
  gen += 1;
  if (threadIdx.x == 0) {
    const unsigned target = gen * gridDim.x;
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar) : "memory");
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.bar) : "memory");
    if (v < target) {
      const uint64_t t0 = globaltimer_ns();
      while (true) {
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.bar) : "memory");
        if (v >= target) break;
        if (globaltimer_ns() - t0 > 2000000000ull) {
          raise_error(a.err, YN_ERR_BULK_TIMEOUT);
          break;
        }
      }
    }
    *flag = *reinterpret_cast<volatile int*>(a.err);
  }
  __syncthreads();
  return *flag != 0;
}

YN_DEV void proxy_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// --------------------------------------------------------------- partition
// P1 units: router rows (cost 1), shared gate/up row pairs (cost 2), the
// shared_expert_gate row (cost 1); CTA b takes the units whose cumulative
// cost starts in [b*C/G, (b+1)*C/G).
struct P1Range {
  int r0, r1;   // router rows
  int p0, p1;   // shared pairs
  int sg;       // 1 if this CTA owns the shared_expert_gate row
};
YN_DEV int p1_unit_at(int c, int E, int Ish) {
  if (c <= E) return c;
  if (c <= E + 2 * Ish) return E + (c - E + 1) / 2;
  return E + Ish + (c - E - 2 * Ish);
}
YN_DEV P1Range p1_range(int b, int G, int E, int Ish) {
  const int C = E + 2 * Ish + (Ish ? 1 : 0);
  const int lo = (int)((long long)b * C / G), hi = (int)((long long)(b + 1) * C / G);
  const int u0 = p1_unit_at(lo, E, Ish), u1 = p1_unit_at(hi, E, Ish);
  P1Range r;
  r.r0 = min(u0, E);
  r.r1 = min(u1, E);
  r.p0 = min(max(u0 - E, 0), Ish);
  r.p1 = min(max(u1 - E, 0), Ish);
  r.sg = (Ish > 0 && u0 <= E + Ish && u1 > E + Ish) ? 1 : 0;
  return r;
}

// Shared-memory layout of one P1 tile (router rows, shared gate rows, shared
// up rows, shared_expert_gate row), each as codes | scales | biases.
struct P1Tile {
  uint8_t* rc; uint16_t* rs; uint16_t* rbv;
  uint8_t* gc; uint16_t* gsc; uint16_t* gbi;
  uint8_t* uc; uint16_t* usc; uint16_t* ubi;
  uint8_t* sc; uint16_t* ssc; uint16_t* sbi;
};

YN_DEV size_t a16d(size_t v) { return (v + 15) & ~size_t(15); }

YN_DEV P1Tile p1_tile(uint8_t* base, const P1Range& r, int H, int gs_r, int gs_s) {
  P1Tile t;
  size_t o = 0;
  const size_t nr = r.r1 - r.r0, np = r.p1 - r.p0;
  const size_t sbr = (size_t)(H / gs_r) * 2, sbs = (size_t)(H / gs_s) * 2;
  t.rc = base + o; o += a16d(nr * H);
  t.rs = (uint16_t*)(base + o); o += a16d(nr * sbr);
  t.rbv = (uint16_t*)(base + o); o += a16d(nr * sbr);
  t.gc = base + o; o += a16d(np * H);
  t.gsc = (uint16_t*)(base + o); o += a16d(np * sbs);
  t.gbi = (uint16_t*)(base + o); o += a16d(np * sbs);
  t.uc = base + o; o += a16d(np * H);
  t.usc = (uint16_t*)(base + o); o += a16d(np * sbs);
  t.ubi = (uint16_t*)(base + o); o += a16d(np * sbs);
  t.sc = base + o; o += a16d(r.sg ? (size_t)H : 0);
  t.ssc = (uint16_t*)(base + o); o += a16d(r.sg ? sbs : 0);
  t.sbi = (uint16_t*)(base + o); o += a16d(r.sg ? sbs : 0);
  return t;
}

// Thread 0 only: arm `bar` and issue the bulk copies of one layer's P1 tile.
YN_DEV void issue_p1(const DecLayer& L, const P1Range& r, const P1Tile& t, int H, uint64_t* bar) {
  const uint32_t sbr = (uint32_t)(H / L.router.gs) * 2;
  const uint32_t nr = r.r1 - r.r0, np = r.p1 - r.p0;
  const uint32_t sbs = L.sg.gs ? (uint32_t)(H / L.sg.gs) * 2 : 0;
  uint32_t tx = nr * (H + 2 * sbr) + np * 2 * (H + 2 * sbs) + (r.sg ? H + 2 * sbs : 0);
  mbar_arrive_expect_tx(bar, tx);
  if (nr) {
    bulk_g2s(t.rc, L.router.w + (size_t)r.r0 * H, nr * H, bar);
    bulk_g2s(t.rs, reinterpret_cast<const uint8_t*>(L.router.s) + (size_t)r.r0 * sbr, nr * sbr, bar);
    bulk_g2s(t.rbv, reinterpret_cast<const uint8_t*>(L.router.b) + (size_t)r.r0 * sbr, nr * sbr, bar);
  }
  if (np) {
    bulk_g2s(t.gc, L.sg.w + (size_t)r.p0 * H, np * H, bar);
    bulk_g2s(t.gsc, reinterpret_cast<const uint8_t*>(L.sg.s) + (size_t)r.p0 * sbs, np * sbs, bar);
    bulk_g2s(t.gbi, reinterpret_cast<const uint8_t*>(L.sg.b) + (size_t)r.p0 * sbs, np * sbs, bar);
    bulk_g2s(t.uc, L.su.w + (size_t)r.p0 * H, np * H, bar);
    bulk_g2s(t.usc, reinterpret_cast<const uint8_t*>(L.su.s) + (size_t)r.p0 * sbs, np * sbs, bar);
    bulk_g2s(t.ubi, reinterpret_cast<const uint8_t*>(L.su.b) + (size_t)r.p0 * sbs, np * sbs, bar);
  }
  if (r.sg) {
    bulk_g2s(t.sc, L.sgt.w, H, bar);
    bulk_g2s(t.ssc, L.sgt.s, sbs, bar);
    bulk_g2s(t.sbi, L.sgt.b, sbs, bar);
  }
}

// ------------------------------------------------------------------ routing
// Block-wide routing of one row of logits (global, E <= 1024) with the
// canonical order of the oracle: max (order-free), exp per element, sum per
// lane over e = lane + 32 i then a butterfly (warp 0), bf16 probabilities,
// then top-k by the unique key (bf16 prob << 16 | 0xFFFF - id): per-warp
// top-k over a slice, merged by warp 0. Results in shared memory.
YN_DEV void route_block(const float* logits_g, int E, int K, int norm, float* v /* E */, uint32_t* keys /* E */,
                        uint32_t* cand /* DEC_WARPS*K */, float* red, int32_t* ids_out, float* w_out) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float m = -INFINITY;
  for (int e = tid; e < E; e += DEC_THREADS) {
    const float x = __ldcg(logits_g + e);
    v[e] = x;
    m = fmaxf(m, x);
  }
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int w = 1; w < DEC_WARPS; ++w) m = fmaxf(m, red[w]);
  for (int e = tid; e < E; e += DEC_THREADS) v[e] = yn_expf(__fsub_rn(v[e], m));
  __syncthreads();
  if (warp == 0) {
    float s = 0.0f;
    for (int e = lane; e < E; e += 32) s = __fadd_rn(s, v[e]);
    s = group_sum_bfly(s, 32);
    if (lane == 0) red[8] = s;
  }
  __syncthreads();
  const float S = red[8];
  for (int e = tid; e < E; e += DEC_THREADS) {
    const float p = bf16r(__fdiv_rn(v[e], S));
    v[e] = p;
    keys[e] = ((uint32_t)f32_to_bf16(p) << 16) | (uint32_t)(0xFFFF - e);
  }
  __syncthreads();
  // per-warp top-K over slice [w*E/8, (w+1)*E/8)
  {
    const int lo = warp * E / DEC_WARPS, hi = (warp + 1) * E / DEC_WARPS;
    uint32_t mine[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = lo + lane + 32 * i;
      mine[i] = (e < hi) ? keys[e] : 0u;
    }
    for (int j = 0; j < K; ++j) {
      uint32_t best = 0;
      int bi = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (mine[i] > best) { best = mine[i]; bi = i; }
      const uint32_t top = __reduce_max_sync(0xffffffffu, best);
      if (best == top && top != 0u) mine[bi] = 0u;
      if (lane == 0) cand[warp * K + j] = top;
    }
  }
  __syncthreads();
  if (warp == 0) {
    uint32_t mine[(DEC_WARPS * DEC_MAX_K + 31) / 32];
    const int nc = DEC_WARPS * K;
#pragma unroll
    for (int i = 0; i < (DEC_WARPS * DEC_MAX_K + 31) / 32; ++i) {
      const int c = lane + 32 * i;
      mine[i] = (c < nc) ? cand[c] : 0u;
    }
    float wsum = 0.0f, myp = 0.0f;
    int myid = 0;
    for (int j = 0; j < K; ++j) {
      uint32_t best = 0;
      int bi = 0;
#pragma unroll
      for (int i = 0; i < (DEC_WARPS * DEC_MAX_K + 31) / 32; ++i)
        if (mine[i] > best) { best = mine[i]; bi = i; }
      const uint32_t top = __reduce_max_sync(0xffffffffu, best);
      if (best == top) mine[bi] = 0u;
      const float p = bf16_to_f32((uint16_t)(top >> 16));
      wsum = __fadd_rn(wsum, p);
      if (lane == j) {
        myp = p;
        myid = 0xFFFF - (int)(top & 0xFFFFu);
      }
    }
    const float sb = bf16r(wsum);
    if (lane < K) {
      ids_out[lane] = myid;
      w_out[lane] = norm ? bf16r(__fdiv_rn(myp, sb)) : myp;
    }
  }
  __syncthreads();
}

// RMSNorm in the canonical 128-thread order (threads 128.. idle in the sum).
YN_DEV void rmsnorm_smem(const uint16_t* h, const uint16_t* w_g, int H, float eps, uint16_t* out, float* red) {
  const int tid = threadIdx.x;
  float ss = 0.0f;
  if (tid < 128)
    for (int i = tid; i < H; i += 128) {
      const float v = bf16_to_f32(h[i]);
      ss = __fmaf_rn(v, v, ss);
    }
  ss = group_sum_bfly(ss, 32);
  __syncthreads();
  if ((tid & 31) == 0 && tid < 128) red[tid >> 5] = ss;
  __syncthreads();
  const float tot = __fadd_rn(__fadd_rn(__fadd_rn(red[0], red[1]), red[2]), red[3]);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)H), eps)));
  for (int i = tid; i < H; i += DEC_THREADS)
    out[i] = f32_to_bf16(__fmul_rn(bf16_to_f32(w_g[i]), bf16r(__fmul_rn(bf16_to_f32(h[i]), r))));
  __syncthreads();
}

// ------------------------------------------------------------ P2 / P3 tiles
struct CSeg {       // one expert's share of this CTA's gate/up rows
  int j, n0, n1;
  uint8_t* gc; uint16_t* gsc; uint16_t* gbi;
  uint8_t* uc; uint16_t* usc; uint16_t* ubi;
};

template <int BITS>
struct DecCfgC {    // routed gate/up rows (K = H)
};

// Issue C (gate/up) and D (down) copies for this CTA. Thread 0 only.
YN_DEV void issue_cd(const DecodeArgs& a, const DecLayer& L, const int32_t* ids, int u0, int u1, int d0, int d1,
                     uint8_t* cbuf, uint8_t* dbuf, CSeg* seg, int& nseg, uint64_t* barC, uint64_t* barD,
                     uint8_t** dptr /* per piece pointers, 3*(K+1) */) {
  const int H = a.H, I = a.I, K = a.K;
  const int bits = L.rg.bits, gs = L.rg.gs;
  const uint32_t rbH = (uint32_t)(H * bits / 8), sbH = (uint32_t)(H / gs) * 2;
  const uint32_t rbI = (uint32_t)(I * bits / 8), sbI = (uint32_t)(I / gs) * 2;
  // segments of [u0, u1) in (j, n) space
  nseg = 0;
  size_t o = 0;
  uint32_t txc = 0;
  for (int u = u0; u < u1;) {
    const int j = u / I, n0 = u % I;
    const int n1 = min(I, n0 + (u1 - u));
    CSeg& s = seg[nseg++];
    s.j = j; s.n0 = n0; s.n1 = n1;
    const size_t nr = n1 - n0;
    s.gc = cbuf + o; o += a16d(nr * rbH);
    s.gsc = (uint16_t*)(cbuf + o); o += a16d(nr * sbH);
    s.gbi = (uint16_t*)(cbuf + o); o += a16d(nr * sbH);
    s.uc = cbuf + o; o += a16d(nr * rbH);
    s.usc = (uint16_t*)(cbuf + o); o += a16d(nr * sbH);
    s.ubi = (uint16_t*)(cbuf + o); o += a16d(nr * sbH);
    txc += 2 * (uint32_t)nr * (rbH + 2 * sbH);
    u += n1 - n0;
  }
  mbar_arrive_expect_tx(barC, txc);
  for (int i = 0; i < nseg; ++i) {
    const CSeg& s = seg[i];
    const int e = ids[s.j];
    const int slot = L.slot_of ? L.slot_of[e] : e;
    const uint8_t* rec = L.ebase + (size_t)slot * (size_t)L.stride;
    const uint32_t nr = s.n1 - s.n0;
    bulk_g2s(s.gc, rec + L.rg.off[0] + (size_t)s.n0 * rbH, nr * rbH, barC);
    bulk_g2s(s.gsc, rec + L.rg.off[1] + (size_t)s.n0 * sbH, nr * sbH, barC);
    bulk_g2s(s.gbi, rec + L.rg.off[2] + (size_t)s.n0 * sbH, nr * sbH, barC);
    bulk_g2s(s.uc, rec + L.rg.off[3] + (size_t)s.n0 * rbH, nr * rbH, barC);
    bulk_g2s(s.usc, rec + L.rg.off[4] + (size_t)s.n0 * sbH, nr * sbH, barC);
    bulk_g2s(s.ubi, rec + L.rg.off[5] + (size_t)s.n0 * sbH, nr * sbH, barC);
  }
  // D: rows [d0, d1) of every routed expert's down_proj and of the shared down_proj
  const uint32_t nd = d1 - d0;
  const uint32_t sbS = a.Ish ? (uint32_t)(a.Ish / L.sd.gs) * 2 : 0;
  uint32_t txd = K * nd * (rbI + 2 * sbI) + (a.Ish ? nd * (a.Ish + 2 * sbS) : 0);
  mbar_arrive_expect_tx(barD, txd);
  o = 0;
  for (int j = 0; j < K; ++j) {
    const int e = ids[j];
    const int slot = L.slot_of ? L.slot_of[e] : e;
    const uint8_t* rec = L.ebase + (size_t)slot * (size_t)L.stride;
    uint8_t* c = dbuf + o; o += a16d((size_t)nd * rbI);
    uint8_t* sc = dbuf + o; o += a16d((size_t)nd * sbI);
    uint8_t* bi = dbuf + o; o += a16d((size_t)nd * sbI);
    dptr[3 * j] = c; dptr[3 * j + 1] = sc; dptr[3 * j + 2] = bi;
    bulk_g2s(c, rec + L.rg.off[6] + (size_t)d0 * rbI, nd * rbI, barD);
    bulk_g2s(sc, rec + L.rg.off[7] + (size_t)d0 * sbI, nd * sbI, barD);
    bulk_g2s(bi, rec + L.rg.off[8] + (size_t)d0 * sbI, nd * sbI, barD);
  }
  if (a.Ish) {
    uint8_t* c = dbuf + o; o += a16d((size_t)nd * a.Ish);
    uint8_t* sc = dbuf + o; o += a16d((size_t)nd * sbS);
    uint8_t* bi = dbuf + o; o += a16d((size_t)nd * sbS);
    dptr[3 * K] = c; dptr[3 * K + 1] = sc; dptr[3 * K + 2] = bi;
    bulk_g2s(c, L.sd.w + (size_t)d0 * a.Ish, nd * a.Ish, barD);
    bulk_g2s(sc, reinterpret_cast<const uint8_t*>(L.sd.s) + (size_t)d0 * sbS, nd * sbS, barD);
    bulk_g2s(bi, reinterpret_cast<const uint8_t*>(L.sd.b) + (size_t)d0 * sbS, nd * sbS, barD);
  }
}

// P2 gate/up compute for one bit width. x registers come from the normed row.
template <int BITS, int CPL, int NSEG>
YN_DEV void p2_compute(const DecodeArgs& a, const CSeg* seg, int nseg, const uint16_t* xs, float xscale, int gs) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rb = a.H * BITS / 8, ng = a.H / gs;
  const int lpr = lanes_per_row(rb), rpi = 32 / lpr, l = lane % lpr, u = lane / lpr;
  XF16<BITS, CPL, NSEG> X;
  load_x_f16<BITS, CPL, NSEG>(X, xs, xscale, l, lpr);
  const float inv = __fdiv_rn(1.0f, xscale);
  // flatten (segment, row) over warps; rpi rows per warp step
  int total = 0;
  for (int i = 0; i < nseg; ++i) total += seg[i].n1 - seg[i].n0;
  for (int base = warp * rpi; base < total; base += DEC_WARPS * rpi) {
    int r = base + u;
    const bool valid = r < total;
    if (!valid) r = 0;
    int si = 0;
    while (r >= seg[si].n1 - seg[si].n0) { r -= seg[si].n1 - seg[si].n0; ++si; }
    const CSeg& s = seg[si];
    float g = row_dot_f16<BITS, CPL, NSEG>(s.gc + (size_t)r * rb, s.gsc + (size_t)r * ng, s.gbi + (size_t)r * ng, X,
                                           inv, l, lpr, gs);
    float up = row_dot_f16<BITS, CPL, NSEG>(s.uc + (size_t)r * rb, s.usc + (size_t)r * ng, s.ubi + (size_t)r * ng, X,
                                            inv, l, lpr, gs);
    g = group_sum_bfly(g, lpr);
    up = group_sum_bfly(up, lpr);
    if (valid && l == 0) a.act[(size_t)s.j * a.I + s.n0 + r] = f32_to_bf16(swiglu_bf16(bf16r(g), bf16r(up)));
  }
}

// P3 routed down rows for one bit width: ybuf[j][r - d0] = bf16(dot).
template <int BITS, int CPL, int NSEG>
YN_DEV void p3_routed(const DecodeArgs& a, uint8_t* const* dptr, int nd, const uint16_t* acts, const float* ascale,
                      float* ybuf, int gs) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rb = a.I * BITS / 8, ng = a.I / gs;
  const int lpr = lanes_per_row(rb), rpi = 32 / lpr, l = lane % lpr, u = lane / lpr;
  const int groups = (nd + rpi - 1) / rpi;
  const int ntask = a.K * groups;
  const int t0 = warp * ntask / DEC_WARPS, t1 = (warp + 1) * ntask / DEC_WARPS;
  int cur_j = -1;
  XF16<BITS, CPL, NSEG> X;
  float inv = 1.0f;
  for (int t = t0; t < t1; ++t) {
    const int j = t / groups, g = t % groups;
    if (j != cur_j) {
      load_x_f16<BITS, CPL, NSEG>(X, acts + (size_t)j * a.I, ascale[j], l, lpr);
      inv = __fdiv_rn(1.0f, ascale[j]);
      cur_j = j;
    }
    int r = g * rpi + u;
    const bool valid = r < nd;
    if (!valid) r = 0;
    float v = row_dot_f16<BITS, CPL, NSEG>(dptr[3 * j] + (size_t)r * rb,
                                           reinterpret_cast<const uint16_t*>(dptr[3 * j + 1]) + (size_t)r * ng,
                                           reinterpret_cast<const uint16_t*>(dptr[3 * j + 2]) + (size_t)r * ng, X, inv,
                                           l, lpr, gs);
    v = group_sum_bfly(v, lpr);
    if (valid && l == 0) ybuf[j * DEC_MAX_DROWS + r] = bf16r(v);
  }
}

template <int CPLS>
YN_DEV void p3_shared(const DecodeArgs& a, uint8_t* const* dptr, int nd, const uint16_t* actsh, float sg, float* ybuf,
                      int gs) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rb = a.Ish, ng = a.Ish / gs;
  const int lpr = lanes_per_row(rb), rpi = 32 / lpr, l = lane % lpr, u = lane / lpr;
  XF32<8, CPLS, 1> X;
  load_x_f32<8, CPLS, 1>(X, actsh, l, lpr);
  const uint8_t* c = dptr[3 * a.K];
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(dptr[3 * a.K + 1]);
  const uint16_t* bi = reinterpret_cast<const uint16_t*>(dptr[3 * a.K + 2]);
  for (int base = warp * rpi; base < nd; base += DEC_WARPS * rpi) {
    int r = base + u;
    const bool valid = r < nd;
    if (!valid) r = 0;
    float v = row_dot_f32<8, CPLS, 1>(c + (size_t)r * rb, sc + (size_t)r * ng, bi + (size_t)r * ng, X, l, lpr, gs);
    v = group_sum_bfly(v, lpr);
    if (valid && l == 0) ybuf[a.K * DEC_MAX_DROWS + r] = bf16r(__fmul_rn(sg, bf16r(v)));
  }
}

// P1 compute: router rows, shared pairs, shared_expert_gate (fp32 path, 8-bit).
template <int CPL8>
YN_DEV void p1_compute(const DecodeArgs& a, const DecLayer& L, const P1Range& r, const P1Tile& t, const uint16_t* xs) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int H = a.H, rb = H;
  const int lpr = lanes_per_row(rb), rpi = 32 / lpr, l = lane % lpr, u = lane / lpr;
  XF32<8, CPL8, 1> X;
  load_x_f32<8, CPL8, 1>(X, xs, l, lpr);
  const int nr = r.r1 - r.r0, np = r.p1 - r.p0;
  const int ntask = nr + np + r.sg;  // rows of work; pairs count once (two dots)
  const int ngr = H / L.router.gs, ngs = L.sg.gs ? H / L.sg.gs : 1;
  for (int base = warp * rpi; base < ntask; base += DEC_WARPS * rpi) {
    int k = base + u;
    const bool valid = k < ntask;
    if (!valid) k = 0;
    if (k < nr) {
      float v = row_dot_f32<8, CPL8, 1>(t.rc + (size_t)k * rb, t.rs + (size_t)k * ngr, t.rbv + (size_t)k * ngr, X, l,
                                        lpr, L.router.gs);
      v = group_sum_bfly(v, lpr);
      if (valid && l == 0) {
        const int e = r.r0 + k;
        a.logits[e] = bf16r(__fadd_rn(v, L.rbias ? L.rbias[e] : 0.0f));
      }
    } else if (k < nr + np) {
      const int p = k - nr;
      float g = row_dot_f32<8, CPL8, 1>(t.gc + (size_t)p * rb, t.gsc + (size_t)p * ngs, t.gbi + (size_t)p * ngs, X, l,
                                        lpr, L.sg.gs);
      float up = row_dot_f32<8, CPL8, 1>(t.uc + (size_t)p * rb, t.usc + (size_t)p * ngs, t.ubi + (size_t)p * ngs, X, l,
                                         lpr, L.su.gs);
      g = group_sum_bfly(g, lpr);
      up = group_sum_bfly(up, lpr);
      if (valid && l == 0) a.act_sh[r.p0 + p] = f32_to_bf16(swiglu_bf16(bf16r(g), bf16r(up)));
    } else {
      float v = row_dot_f32<8, CPL8, 1>(t.sc, t.ssc, t.sbi, X, l, lpr, L.sgt.gs);
      v = group_sum_bfly(v, lpr);
      if (valid && l == 0) a.sgate[0] = bf16r(sigmoid_f32(bf16r(v)));
    }
  }
}

YN_DEV void stamp(const DecodeArgs& a, int tok, int layer, int slot) {
  if (a.timing && tok == 0 && blockIdx.x == 0 && threadIdx.x == 0)
    a.timing[(size_t)layer * 8 + slot] = (long long)globaltimer_ns();
}

template <int CPL8, int CPLS>
__global__ void __launch_bounds__(DEC_THREADS, 1) k_stack_decode(const DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* barA = reinterpret_cast<uint64_t*>(smem);        // [2]
  uint64_t* barC = reinterpret_cast<uint64_t*>(smem + 16);
  uint64_t* barD = reinterpret_cast<uint64_t*>(smem + 24);
  float* red = reinterpret_cast<float*>(smem + 32);           // 16 floats
  int* eflag = reinterpret_cast<int*>(smem + 128);
  uint16_t* hs = reinterpret_cast<uint16_t*>(smem + a.off_hs);
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem + a.off_xs);
  uint16_t* acts = reinterpret_cast<uint16_t*>(smem + a.off_act);   // (K, I)
  uint16_t* actsh = reinterpret_cast<uint16_t*>(smem + a.off_actsh);
  uint8_t* rt = smem + a.off_route;
  float* rv = reinterpret_cast<float*>(rt);                             // E
  uint32_t* keys = reinterpret_cast<uint32_t*>(rt + 4 * a.E);           // E
  uint32_t* cand = keys + a.E;                                          // 8*K
  int32_t* ids = reinterpret_cast<int32_t*>(cand + DEC_WARPS * DEC_MAX_K);
  float* wts = reinterpret_cast<float*>(ids + DEC_MAX_K);
  float* ascale = wts + DEC_MAX_K;                                      // K
  CSeg* seg = reinterpret_cast<CSeg*>(ascale + DEC_MAX_K + 8);          // 4
  uint8_t** dptr = reinterpret_cast<uint8_t**>(reinterpret_cast<uint8_t*>(seg) + 4 * sizeof(CSeg));
  int* nseg_s = reinterpret_cast<int*>(dptr + 3 * (DEC_MAX_K + 1));
  float* ybuf = reinterpret_cast<float*>(smem + a.off_y);               // (K+1, DEC_MAX_DROWS)
  uint8_t* Abuf[2] = {smem + a.off_A0, smem + a.off_A1};
  uint8_t* cbuf = smem + a.off_C;
  uint8_t* dbuf = smem + a.off_D;

  const int tid = threadIdx.x;
  const int G = gridDim.x, b = blockIdx.x;
  const int H = a.H, E = a.E, K = a.K, I = a.I;
  const P1Range r1 = p1_range(b, G, E, a.Ish);
  const int U = K * I;
  const int u0 = (int)((long long)b * U / G), u1 = (int)((long long)(b + 1) * U / G);
  const int d0 = (int)((long long)b * H / G), d1 = (int)((long long)(b + 1) * H / G);
  const int nd = d1 - d0;

  if (tid == 0) {
    mbar_init(&barA[0], 1);
    mbar_init(&barA[1], 1);
    mbar_init(barC, 1);
    mbar_init(barD, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    const DecLayer& L0 = a.layers[0];
    issue_p1(L0, r1, p1_tile(Abuf[0], r1, H, L0.router.gs, L0.sg.gs ? L0.sg.gs : 64), H, &barA[0]);
  }
  unsigned gen = 0;
  uint32_t phA[2] = {0, 0}, phC = 0, phD = 0;
  bool pendA[2] = {true, false}, pendC = false, pendD = false;  // armed, not yet waited on
  int step = 0;  // global layer step counter (selects the A buffer)
  // Error exit: wait (bounded) for every bulk copy still landing in this
  // CTA's shared memory, then leave.
  auto drain = [&]() {
    for (int i = 0; i < 2; ++i)
      if (pendA[i]) mbar_wait_block(&barA[i], phA[i], nullptr);
    if (pendC) mbar_wait_block(barC, phC, nullptr);
    if (pendD) mbar_wait_block(barD, phD, nullptr);
  };

  for (int tok = 0; tok < a.n_tokens; ++tok) {
    for (int layer = 0; layer < a.n_layers; ++layer, ++step) {
      const DecLayer& L = a.layers[layer];
      const int ab = step & 1;
      stamp(a, tok, layer, 0);
      // -------- P1: prefetch next layer's tile, norm, router + shared rows
      if (tid == 0) {
        const int nl = (layer + 1 < a.n_layers) ? layer + 1 : 0;
        const bool more = (layer + 1 < a.n_layers) || (tok + 1 < a.n_tokens);
        if (more) {
          const DecLayer& N = a.layers[nl];
          proxy_fence();
          issue_p1(N, r1, p1_tile(Abuf[ab ^ 1], r1, H, N.router.gs, N.sg.gs ? N.sg.gs : 64), H, &barA[ab ^ 1]);
        }
      }
      pendA[ab ^ 1] = (layer + 1 < a.n_layers) || (tok + 1 < a.n_tokens);
      const uint16_t* hin = (layer == 0) ? a.inputs + (size_t)tok * H : a.hbuf + (size_t)(step & 1) * H;
      for (int i = tid; i < H / 8; i += DEC_THREADS)
        reinterpret_cast<uint4*>(hs)[i] = __ldcg(reinterpret_cast<const uint4*>(hin) + i);
      __syncthreads();
      rmsnorm_smem(hs, L.norm, H, a.eps, xs, red);
      const bool a_ok = mbar_wait_block(&barA[ab], phA[ab], a.err);
      if (a_ok) {
        phA[ab] ^= 1;
        pendA[ab] = false;
      }
      if (a_ok) p1_compute<CPL8>(a, L, r1, p1_tile(Abuf[ab], r1, H, L.router.gs, L.sg.gs ? L.sg.gs : 64), xs);
      stamp(a, tok, layer, 1);
      if (grid_barrier(a, gen, eflag)) { drain(); return; }
      stamp(a, tok, layer, 2);
      // -------- P2: routing, issue C and D tiles, gate/up rows
      route_block(a.logits, E, K, a.norm_topk, rv, keys, cand, red, ids, wts);
      if (a.trace_ids && b == 0 && tid < K) a.trace_ids[((size_t)tok * a.n_layers + layer) * K + tid] = ids[tid];
      if (tid == 0) {
        bool ok = true;
        for (int j = 0; j < K; ++j) {
          const int e = ids[j];
          const int s = (e >= 0 && e < E) ? (L.slot_of ? L.slot_of[e] : e) : -1;
          if (s < 0 || s >= L.n_slots) ok = false;
        }
        if (!ok) {
          raise_error(a.err, YN_ERR_BAD_SLOT);
          *nseg_s = -1;
        } else {
          int nseg = 0;
          proxy_fence();
          issue_cd(a, L, ids, u0, u1, d0, d1, cbuf, dbuf, seg, nseg, barC, barD, dptr);
          *nseg_s = nseg;
        }
      }
      // x max for the fp16 path (normed row in xs)
      float mx = 0.0f;
      for (int i = tid; i < H; i += DEC_THREADS) mx = fmaxf(mx, fabsf(bf16_to_f32(xs[i])));
      mx = warp_max(mx);
      if ((tid & 31) == 0) red[tid >> 5] = mx;
      __syncthreads();
      mx = red[0];
#pragma unroll
      for (int w = 1; w < DEC_WARPS; ++w) mx = fmaxf(mx, red[w]);
      const float xscale = fp16_input_scale(mx);
      const bool cd_ok = (*nseg_s >= 0);  // uniform: written by thread 0 before the sync above
      pendC = pendD = cd_ok;
      const bool c_ok = cd_ok && mbar_wait_block(barC, phC, a.err);
      if (c_ok) {
        phC ^= 1;
        pendC = false;
        const int bits = L.rg.bits, gs = L.rg.gs;
        const int nseg = *nseg_s;
        if (bits == 2) {
          if (gs == 32) p2_compute<2, 1, 2>(a, seg, nseg, xs, xscale, gs);
          else p2_compute<2, 1, 1>(a, seg, nseg, xs, xscale, gs);
        } else {
          p2_compute<4, 2, 1>(a, seg, nseg, xs, xscale, gs);
        }
      }
      stamp(a, tok, layer, 3);
      if (grid_barrier(a, gen, eflag)) { drain(); return; }
      stamp(a, tok, layer, 4);
      // -------- P3: down rows [d0, d1) of every expert + shared, combine, residual
      for (int i = tid; i < K * I / 8; i += DEC_THREADS)
        reinterpret_cast<uint4*>(acts)[i] = __ldcg(reinterpret_cast<const uint4*>(a.act) + i);
      for (int i = tid; i < a.Ish / 8; i += DEC_THREADS)
        reinterpret_cast<uint4*>(actsh)[i] = __ldcg(reinterpret_cast<const uint4*>(a.act_sh) + i);
      __syncthreads();
      {
        const int warp = tid >> 5, lane = tid & 31;
        for (int j = warp; j < K; j += DEC_WARPS) {
          float m = 0.0f;
          for (int i = lane; i < I; i += 32) m = fmaxf(m, fabsf(bf16_to_f32(acts[(size_t)j * I + i])));
          m = warp_max(m);
          if (lane == 0) ascale[j] = fp16_input_scale(m);
        }
      }
      __syncthreads();
      const bool d_ok = mbar_wait_block(barD, phD, a.err);
      if (d_ok) {
        phD ^= 1;
        pendD = false;
      }
      if (d_ok) {
        const int bits = L.rg.bits, gs = L.rg.gs;
        if (bits == 2) {
          if (gs == 32) p3_routed<2, 1, 2>(a, dptr, nd, acts, ascale, ybuf, gs);
          else p3_routed<2, 1, 1>(a, dptr, nd, acts, ascale, ybuf, gs);
        } else {
          p3_routed<4, 1, 1>(a, dptr, nd, acts, ascale, ybuf, gs);
        }
        if (a.Ish) p3_shared<CPLS>(a, dptr, nd, actsh, __ldcg(a.sgate), ybuf, L.sd.gs);
      }
      __syncthreads();
      {
        uint16_t* hout = (layer == a.n_layers - 1) ? a.outputs + (size_t)tok * H : a.hbuf + (size_t)((step + 1) & 1) * H;
        for (int t = tid; t < nd; t += DEC_THREADS) {
          float acc = 0.0f;
          for (int j = 0; j < K; ++j) acc = __fadd_rn(acc, bf16r(__fmul_rn(ybuf[j * DEC_MAX_DROWS + t], wts[j])));
          float o = bf16r(acc);
          if (a.Ish) o = bf16r(__fadd_rn(o, ybuf[K * DEC_MAX_DROWS + t]));
          o = bf16r(__fadd_rn(bf16_to_f32(hs[d0 + t]), o));
          hout[d0 + t] = f32_to_bf16(o);
        }
      }
      stamp(a, tok, layer, 5);
      if (grid_barrier(a, gen, eflag)) { drain(); return; }
    }
  }
}

}  // namespace ynb
