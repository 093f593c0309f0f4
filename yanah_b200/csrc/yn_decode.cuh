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
#include "yn_mma.cuh"

namespace ynb {

constexpr int DEC_THREADS = 512;
constexpr int DEC_WARPS = DEC_THREADS / 32;
constexpr int DEC_MAX_K = 16;
constexpr int DEC_MAX_DROWS = 16;  // output rows per CTA in P3 (one MMA tile)

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
  int off_hs, off_xs, off_xf, off_route, off_part, off_A, off_C, off_D;
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

// Shared-memory layout of one P1 tile: norm weight, router rows, shared gate
// rows, shared up rows, shared_expert_gate row (codes | scales | biases each).
struct P1Tile {
  uint16_t* norm;
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
  t.norm = (uint16_t*)(base + o); o += a16d((size_t)H * 2);
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

YN_DEV int shared_gs(const DecLayer& L) { return L.sg.gs ? L.sg.gs : 64; }

// One warp: issue the bulk copies of one layer's P1 tile (every CTA also
// takes the whole norm weight); lane i issues piece i.
YN_DEV void issue_p1(const DecLayer& L, const P1Range& r, const P1Tile& t, int H, uint64_t* bar) {
  const int lane = threadIdx.x & 31;
  const uint32_t sbr = (uint32_t)(H / L.router.gs) * 2;
  const uint32_t nr = r.r1 - r.r0, np = r.p1 - r.p0;
  const uint32_t sbs = L.sg.gs ? (uint32_t)(H / L.sg.gs) * 2 : 0;
  const uint32_t tx = (uint32_t)H * 2 + nr * (H + 2 * sbr) + np * 2 * (H + 2 * sbs) + (r.sg ? H + 2 * sbs : 0);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (lane == 0) mbar_arrive_expect_tx(bar, tx);
  __syncwarp();
  void* dst = nullptr;
  const void* src = nullptr;
  uint32_t bytes = 0;
  const uint8_t* rs = reinterpret_cast<const uint8_t*>(L.router.s);
  const uint8_t* rb = reinterpret_cast<const uint8_t*>(L.router.b);
  switch (lane) {
    case 0: dst = t.norm; src = L.norm; bytes = (uint32_t)H * 2; break;
    case 1: dst = t.rc; src = L.router.w + (size_t)r.r0 * H; bytes = nr * H; break;
    case 2: dst = t.rs; src = rs + (size_t)r.r0 * sbr; bytes = nr * sbr; break;
    case 3: dst = t.rbv; src = rb + (size_t)r.r0 * sbr; bytes = nr * sbr; break;
    case 4: dst = t.gc; src = L.sg.w + (size_t)r.p0 * H; bytes = np * H; break;
    case 5: dst = t.gsc; src = reinterpret_cast<const uint8_t*>(L.sg.s) + (size_t)r.p0 * sbs; bytes = np * sbs; break;
    case 6: dst = t.gbi; src = reinterpret_cast<const uint8_t*>(L.sg.b) + (size_t)r.p0 * sbs; bytes = np * sbs; break;
    case 7: dst = t.uc; src = L.su.w + (size_t)r.p0 * H; bytes = np * H; break;
    case 8: dst = t.usc; src = reinterpret_cast<const uint8_t*>(L.su.s) + (size_t)r.p0 * sbs; bytes = np * sbs; break;
    case 9: dst = t.ubi; src = reinterpret_cast<const uint8_t*>(L.su.b) + (size_t)r.p0 * sbs; bytes = np * sbs; break;
    case 10: dst = t.sc; src = L.sgt.w; bytes = r.sg ? (uint32_t)H : 0u; break;
    case 11: dst = t.ssc; src = L.sgt.s; bytes = r.sg ? sbs : 0u; break;
    case 12: dst = t.sbi; src = L.sgt.b; bytes = r.sg ? sbs : 0u; break;
    default: break;
  }
  if (bytes) bulk_g2s(dst, src, bytes, bar);
  __syncwarp();
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
// Shared-memory layout of this CTA's routed gate/up rows ("C rows"): the
// rows of at most two (column, row-range) segments, ordered seg0 gate, seg0
// up, seg1 gate, seg1 up; codes with a padded stride, scales and biases dense.
struct CPlan {
  int nseg;
  int j[2], n0[2], nr[2];   // column, first row, rows
  int R;                    // total C rows (2 * sum nr)
  int rs;                   // padded code-row stride
};

YN_DEV CPlan c_plan(int u0, int u1, int I, int rbH) {
  CPlan p;
  p.nseg = 0;
  p.R = 0;
  p.rs = rbH + 16;
  for (int u = u0; u < u1 && p.nseg < 2;) {
    const int j = u / I, n0 = u % I, n1 = min(I, n0 + (u1 - u));
    p.j[p.nseg] = j; p.n0[p.nseg] = n0; p.nr[p.nseg] = n1 - n0;
    p.R += 2 * (n1 - n0);
    ++p.nseg;
    u += n1 - n0;
  }
  return p;
}
// C row r -> (segment, up?, row inside the segment)
YN_DEV void c_row(const CPlan& p, int r, int& s, int& up, int& n) {
  const int r0 = 2 * p.nr[0];
  s = (r >= r0) ? 1 : 0;
  const int rr = s ? r - r0 : r;
  up = rr >= p.nr[s] ? 1 : 0;
  n = up ? rr - p.nr[s] : rr;
}

// All warps: 16-byte asynchronous copies of this CTA's C rows (one commit
// group) then D rows (a second group). A warp takes a row at a time; its
// lanes take the row's 16-byte chunks, so rows land at a padded stride.
struct DLayout {  // D tile: per column a 16-row block at stride rsI, then the shared tile
  uint32_t rbI, sbI, rsI, rsS, sbS;
  size_t dsh, dsc, dbi, ssc, sbi;
};
YN_DEV DLayout d_layout(const DecodeArgs& a, const DecLayer& L) {
  DLayout d;
  const int bits = L.rg.bits, gs = L.rg.gs, K = a.K, Ish = a.Ish;
  d.rbI = (uint32_t)(a.I * bits / 8);
  d.sbI = (uint32_t)(a.I / gs) * 2;
  d.rsI = d.rbI + 16;
  d.rsS = (uint32_t)Ish + 16;
  d.sbS = Ish ? (uint32_t)(Ish / L.sd.gs) * 2 : 0;
  d.dsh = (size_t)K * DEC_MAX_DROWS * d.rsI;
  d.dsc = d.dsh + (size_t)DEC_MAX_DROWS * d.rsS;
  d.dbi = d.dsc + (size_t)K * DEC_MAX_DROWS * d.sbI;
  d.ssc = d.dbi + (size_t)K * DEC_MAX_DROWS * d.sbI;
  d.sbi = d.ssc + (size_t)DEC_MAX_DROWS * d.sbS;
  return d;
}

// One warp: pull this CTA's D pieces (rows [d0, d0+nd) of every column's
// down_proj codes/scales/biases and of the shared down_proj) into L2 with
// bulk prefetches, so the P3 register loads hit L2.
YN_DEV void prefetch_d(const DecodeArgs& a, const DecLayer& L, const int32_t* ids, int d0, int nd) {
  const int lane = threadIdx.x & 31, K = a.K;
  const DLayout dl = d_layout(a, L);
  for (int i = lane; i < 3 * K + (a.Ish ? 3 : 0); i += 32) {
    const int j = i / 3, piece = i % 3;
    const uint8_t* src;
    uint32_t bytes;
    if (j < K) {
      const int e = ids[j];
      const uint8_t* rec = L.ebase + (size_t)(L.slot_of ? L.slot_of[e] : e) * (size_t)L.stride;
      const uint32_t rb = piece == 0 ? dl.rbI : dl.sbI;
      src = rec + L.rg.off[6 + piece] + (size_t)d0 * rb;
      bytes = (uint32_t)nd * rb;
    } else {
      const uint8_t* base = piece == 0 ? L.sd.w : reinterpret_cast<const uint8_t*>(piece == 1 ? L.sd.s : L.sd.b);
      const uint32_t rb = piece == 0 ? (uint32_t)a.Ish : dl.sbS;
      src = base + (size_t)d0 * rb;
      bytes = (uint32_t)nd * rb;
    }
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
  }
}

// Scale/bias contribution of one block for one row.
YN_DEV float block_contrib(const uint16_t* srow, const uint16_t* brow, int blk, int gs, const float (&d)[2],
                           const XBlock& X, float inv_scale, int nseg) {
  if (nseg == 1) {
    const int g = blk * 64 / gs;
    return __fmaf_rn(f16_to_f32(srow[g]), __fmul_rn(d[0], inv_scale),
                     __fmul_rn(f16_to_f32(brow[g]), __fadd_rn(X.xs_lo, X.xs_hi)));
  }
  const int g = blk * 2;
  const float lo = __fmaf_rn(f16_to_f32(srow[g]), __fmul_rn(d[0], inv_scale), __fmul_rn(f16_to_f32(brow[g]), X.xs_lo));
  const float hi = __fmaf_rn(f16_to_f32(srow[g + 1]), __fmul_rn(d[1], inv_scale),
                             __fmul_rn(f16_to_f32(brow[g + 1]), X.xs_hi));
  return __fadd_rn(lo, hi);
}

// Global address of one lane's code words for (row of the C list, block).
YN_DEV const uint8_t* c_row_ptr(const DecLayer& L, const int32_t* ids, const CPlan& cp, int r, uint32_t rbH) {
  int sgi, up, n;
  c_row(cp, r, sgi, up, n);
  const int e = ids[cp.j[sgi]];
  const uint8_t* rec = L.ebase + (size_t)(L.slot_of ? L.slot_of[e] : e) * (size_t)L.stride;
  return rec + L.rg.off[up ? 3 : 0] + (size_t)(cp.n0[sgi] + n) * rbH;
}
YN_DEV const uint16_t* c_scale_ptr(const DecLayer& L, const int32_t* ids, const CPlan& cp, int r, uint32_t sbH,
                                   int bias) {
  int sgi, up, n;
  c_row(cp, r, sgi, up, n);
  const int e = ids[cp.j[sgi]];
  const uint8_t* rec = L.ebase + (size_t)(L.slot_of ? L.slot_of[e] : e) * (size_t)L.stride;
  return reinterpret_cast<const uint16_t*>(rec + L.rg.off[(up ? 4 : 1) + bias] + (size_t)(cp.n0[sgi] + n) * sbH);
}

template <int BITS>
YN_DEV void ldg_codes(const uint8_t* p, uint32_t (&w)[4]) {
  constexpr int W = MmaFmt<BITS>::WORDS;
  if (W == 1) {
    w[0] = __ldg(reinterpret_cast<const unsigned int*>(p));
  } else if (W == 2) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
    w[0] = v.x; w[1] = v.y;
  } else {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  }
}

// P2: warp w owns blocks [NBW*w, NBW*w + NBW) of the hidden dimension for
// every C row. All code words and scales a lane needs are loaded from global
// memory into registers up front (one memory round trip), then unpacked and
// multiplied. Contributions go to part[blk * R + row].
template <int BITS, int NSEG, int NBW, int MAXT>
YN_DEV void p2_regs(const DecodeArgs& a, const DecLayer& L, const int32_t* ids, const CPlan& cp, int gs,
                    const uint16_t* xs, float xscale, float* part) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  constexpr int W = MmaFmt<BITS>::WORDS;
  const int H = a.H, R = cp.R;
  const uint32_t rbH = (uint32_t)(H * BITS / 8), sbH = (uint32_t)(H / gs) * 2;
  const int ntile = (R + 15) / 16;
  const int blk0 = warp * NBW;
  uint32_t w[MAXT][2][NBW][4];
  uint2 sc[MAXT][2][2];      // scales / biases of an aligned 4-group window (fp16) for rows g, g+8
  const int grp0 = (blk0 * 64 / gs) & ~3;
#pragma unroll
  for (int t = 0; t < MAXT; ++t) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = t * 16 + g + 8 * h;
      const bool ok = (t < ntile) && (r < R);
      if (ok) {
        const uint8_t* rp = c_row_ptr(L, ids, cp, r, rbH);
#pragma unroll
        for (int q = 0; q < NBW; ++q) ldg_codes<BITS>(rp + (blk0 + q) * 8 * BITS + c * 4 * W, w[t][h][q]);
        const uint16_t* sp = c_scale_ptr(L, ids, cp, r, sbH, 0);
        const uint16_t* bp = c_scale_ptr(L, ids, cp, r, sbH, 1);
        sc[t][h][0] = __ldg(reinterpret_cast<const uint2*>(sp + grp0));
        sc[t][h][1] = __ldg(reinterpret_cast<const uint2*>(bp + grp0));
      } else {
#pragma unroll
        for (int q = 0; q < NBW; ++q) w[t][h][q][0] = w[t][h][q][1] = w[t][h][q][2] = w[t][h][q][3] = 0u;
        sc[t][h][0] = sc[t][h][1] = make_uint2(0u, 0u);
      }
    }
  }
  const float inv = __fdiv_rn(1.0f, xscale);
#pragma unroll
  for (int q = 0; q < NBW; ++q) {
    const int blk = blk0 + q;
    XBlock X;
    build_xblock<BITS>(X, xs, blk, xscale, c);
    float* pb = part + (size_t)blk * R;
#pragma unroll
    for (int t = 0; t < MAXT; ++t) {
      if (t >= ntile) break;
      float da[2], db[2];
      mma_block<BITS, NSEG>(w[t][0][q], w[t][1][q], X, c, da, db);
      if (c == 0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = t * 16 + g + 8 * h;
          if (r < R) {
            // scales of group index blk*64/gs inside the loaded 4-group window
            const uint2 s4 = sc[t][h][0], b4 = sc[t][h][1];
            auto pick = [](uint2 v, int i) -> float {
              const uint32_t wv = (i < 2) ? v.x : v.y;
              return f16_to_f32((uint16_t)((i & 1) ? wv >> 16 : wv & 0xFFFFu));
            };
            const float* dd = h ? db : da;
            float v;
            if (NSEG == 1) {
              const int gi = blk * 64 / gs - grp0;
              v = __fmaf_rn(pick(s4, gi), __fmul_rn(dd[0], inv), __fmul_rn(pick(b4, gi), __fadd_rn(X.xs_lo, X.xs_hi)));
            } else {
              const int gi = 2 * blk - grp0;
              v = __fadd_rn(__fmaf_rn(pick(s4, gi), __fmul_rn(dd[0], inv), __fmul_rn(pick(b4, gi), X.xs_lo)),
                            __fmaf_rn(pick(s4, gi + 1), __fmul_rn(dd[1], inv), __fmul_rn(pick(b4, gi + 1), X.xs_hi)));
            }
            pb[r] = v;
          }
        }
      }
    }
  }
}

// P3 prologue: warp j < K builds the fragments of routed column j's
// activations (from global), warp K those of the shared expert's; each lane
// (blk = lane/4, c = lane%4) owns one block fragment.
template <int BITS>
YN_DEV void p3_frags(const DecodeArgs& a, XBlock* xf, float* xscale) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, blk = lane >> 2, c = lane & 3;
  const int K = a.K;
  if (warp > K || (warp == K && !a.Ish)) return;
  const int n = (warp < K) ? a.I : a.Ish;
  if (n != 512) return;  // one warp covers 8 blocks of 64 codes (checked on the host)
  const uint16_t* src = (warp < K) ? a.act + (size_t)warp * a.I : a.act_sh;
  uint16_t v[16];
  {
    const uint4 q0 = __ldcg(reinterpret_cast<const uint4*>(src + blk * 64 + 16 * c));
    const uint4 q1 = __ldcg(reinterpret_cast<const uint4*>(src + blk * 64 + 16 * c + 8));
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[2 * i] = (uint16_t)(w[i] & 0xFFFFu);
      v[2 * i + 1] = (uint16_t)(w[i] >> 16);
    }
  }
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(bf16_to_f32(v[i])));
  m = warp_max(m);
  const float scale = fp16_input_scale(m);
  // fragment from registers (same construction as build_xblock)
  XBlock X;
  const bool eight = (warp == K);
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    const int lo = eight ? MmaFmt<8>::lo(p) : MmaFmt<BITS>::lo(p);
    const int hi = eight ? MmaFmt<8>::hi(p) : MmaFmt<BITS>::hi(p);
    const float im = eight ? MmaFmt<8>::inv_mult(p) : MmaFmt<BITS>::inv_mult(p);
    const float mm = __fmul_rn(scale, im);
    float va = 0.f, vb = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (i == lo) va = bf16_to_f32(v[i]);
      if (i == hi) vb = bf16_to_f32(v[i]);
    }
    __half2 h = __floats2half2_rn(__fmul_rn(va, mm), __fmul_rn(vb, mm));
    X.b[p] = *reinterpret_cast<uint32_t*>(&h);
  }
  float s = 0.0f;
#pragma unroll
  for (int e = 0; e < 16; ++e) s = __fadd_rn(s, bf16_to_f32(v[e]));
  const float s1 = __shfl_xor_sync(0xffffffffu, s, 1);
  const float s01 = __fadd_rn(s, s1);
  const float s23 = __shfl_xor_sync(0xffffffffu, s01, 2);
  X.xs_lo = (c < 2) ? s01 : s23;
  X.xs_hi = (c < 2) ? s23 : s01;
  xf[(size_t)(warp * 8 + blk) * 4 + c] = X;
  if (lane == 0) xscale[warp] = scale;
}

// P3: (tile, block) items over all warps; tiles 0..K-1 routed (BITS), tile K
// the shared expert (8-bit). Code words and scales come straight from global
// memory (prefetched into L2 during P2), all items' loads issued up front.
// Contributions to part[(tile * 8 + blk) * 16 + row].
template <int BITS, int NSEG, int MAXI>
YN_DEV void p3_regs(const DecodeArgs& a, const DecLayer& L, const int32_t* ids, int d0, int nd, const XBlock* xf,
                    const float* xscale, float* part) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int K = a.K, I = a.I, Ish = a.Ish, gs = L.rg.gs;
  const DLayout dl = d_layout(a, L);
  const int nblk = 8;  // I = Ish = 512
  const int ntile = K + (Ish ? 1 : 0);
  const int nitems = ntile * nblk;
  uint32_t w[MAXI][2][4];
  uint32_t sc[MAXI][2][2];
#pragma unroll
  for (int k = 0; k < MAXI; ++k) {
    const int item = warp + k * DEC_WARPS;
    const int t = item / nblk, blk = item % nblk;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = g + 8 * h;
      w[k][h][0] = w[k][h][1] = w[k][h][2] = w[k][h][3] = 0u;
      sc[k][h][0] = sc[k][h][1] = 0u;
      if (item < nitems && r < nd) {
        if (t < K) {
          const int e = ids[t];
          const uint8_t* rec = L.ebase + (size_t)(L.slot_of ? L.slot_of[e] : e) * (size_t)L.stride;
          const uint8_t* rp = rec + L.rg.off[6] + (size_t)(d0 + r) * dl.rbI;
          ldg_codes<BITS>(rp + blk * 8 * BITS + c * 4 * MmaFmt<BITS>::WORDS, w[k][h]);
          const int gi = (blk * 64 / gs) & ~1;
          sc[k][h][0] = __ldg(reinterpret_cast<const unsigned int*>(rec + L.rg.off[7] + (size_t)(d0 + r) * dl.sbI) + gi / 2);
          sc[k][h][1] = __ldg(reinterpret_cast<const unsigned int*>(rec + L.rg.off[8] + (size_t)(d0 + r) * dl.sbI) + gi / 2);
        } else {
          const uint8_t* rp = L.sd.w + (size_t)(d0 + r) * Ish;
          ldg_codes<8>(rp + blk * 64 + c * 16, w[k][h]);
          const int gi = (blk * 64 / L.sd.gs) & ~1;
          sc[k][h][0] = __ldg(reinterpret_cast<const unsigned int*>(L.sd.s + (size_t)(d0 + r) * (Ish / L.sd.gs)) + gi / 2);
          sc[k][h][1] = __ldg(reinterpret_cast<const unsigned int*>(L.sd.b + (size_t)(d0 + r) * (Ish / L.sd.gs)) + gi / 2);
        }
      }
    }
  }
#pragma unroll
  for (int k = 0; k < MAXI; ++k) {
    const int item = warp + k * DEC_WARPS;
    if (item >= nitems) break;
    const int t = item / nblk, blk = item % nblk;
    const XBlock& X = xf[(size_t)(t * 8 + blk) * 4 + c];
    const float inv = __fdiv_rn(1.0f, xscale[t]);
    const bool routed = t < K;
    float da[2], db[2];
    if (routed) mma_block<BITS, NSEG>(w[k][0], w[k][1], X, c, da, db);
    else mma_block<8, 1>(w[k][0], w[k][1], X, c, da, db);
    if (c == 0) {
      const int gsx = routed ? gs : L.sd.gs;
      const int nsx = routed ? NSEG : 1;
      float* pp = part + (size_t)(t * nblk + blk) * DEC_MAX_DROWS;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = g + 8 * h;
        if (r < nd) {
          const uint32_t s2 = sc[k][h][0], b2 = sc[k][h][1];
          const float* dd = h ? db : da;
          float v;
          if (nsx == 1) {
            const int gi = (blk * 64 / gsx) & 1;
            const float sv = f16_to_f32((uint16_t)(gi ? s2 >> 16 : s2 & 0xFFFFu));
            const float bv = f16_to_f32((uint16_t)(gi ? b2 >> 16 : b2 & 0xFFFFu));
            v = __fmaf_rn(sv, __fmul_rn(dd[0], inv), __fmul_rn(bv, __fadd_rn(X.xs_lo, X.xs_hi)));
          } else {
            const float s0 = f16_to_f32((uint16_t)(s2 & 0xFFFFu)), s1 = f16_to_f32((uint16_t)(s2 >> 16));
            const float b0 = f16_to_f32((uint16_t)(b2 & 0xFFFFu)), b1 = f16_to_f32((uint16_t)(b2 >> 16));
            v = __fadd_rn(__fmaf_rn(s0, __fmul_rn(dd[0], inv), __fmul_rn(b0, X.xs_lo)),
                          __fmaf_rn(s1, __fmul_rn(dd[1], inv), __fmul_rn(b1, X.xs_hi)));
          }
          pp[r] = v;
        }
      }
    }
  }
  (void)I;
}

// P1 compute: router rows, shared pairs, shared_expert_gate (fp32 path, 8-bit).
template <int CPL8>
YN_DEV void p1_compute(const DecodeArgs& a, const DecLayer& L, const P1Range& r, const P1Tile& t, const uint16_t* xs,
                       const float* rbias_s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int H = a.H, rb = H;
  const int lpr = lanes_per_row(rb), rpi = 32 / lpr, l = lane % lpr, u = lane / lpr;
  XF32<8, CPL8, 1> X;
  load_x_f32<8, CPL8, 1>(X, xs, l, lpr);
  const int nr = r.r1 - r.r0, np = r.p1 - r.p0;
  const int ntask = nr + 2 * np + r.sg;  // shared pairs as two rows (gate, up)
  const int ngr = H / L.router.gs, ngs = L.sg.gs ? H / L.sg.gs : 1;
  float* gu = const_cast<float*>(rbias_s) + 64;  // shared gate/up dots (bf16-rounded) [2][np]
  for (int base = warp * rpi; base < ntask; base += DEC_WARPS * rpi) {
    int k = base + u;
    const bool valid = k < ntask;
    if (!valid) k = 0;
    float v;
    if (k < nr) {
      v = row_dot_f32<8, CPL8, 1>(t.rc + (size_t)k * rb, t.rs + (size_t)k * ngr, t.rbv + (size_t)k * ngr, X, l, lpr,
                                  L.router.gs);
    } else if (k < nr + 2 * np) {
      const int q = k - nr, p = q >> 1, up = q & 1;
      v = up ? row_dot_f32<8, CPL8, 1>(t.uc + (size_t)p * rb, t.usc + (size_t)p * ngs, t.ubi + (size_t)p * ngs, X, l,
                                       lpr, L.su.gs)
             : row_dot_f32<8, CPL8, 1>(t.gc + (size_t)p * rb, t.gsc + (size_t)p * ngs, t.gbi + (size_t)p * ngs, X, l,
                                       lpr, L.sg.gs);
    } else {
      v = row_dot_f32<8, CPL8, 1>(t.sc, t.ssc, t.sbi, X, l, lpr, L.sgt.gs);
    }
    v = group_sum_bfly(v, lpr);
    if (valid && l == 0) {
      if (k < nr) {
        a.logits[r.r0 + k] = bf16r(__fadd_rn(v, rbias_s[k]));
      } else if (k < nr + 2 * np) {
        const int q = k - nr;
        gu[q] = bf16r(v);
      } else {
        a.sgate[0] = bf16r(sigmoid_f32(bf16r(v)));
      }
    }
  }
  __syncthreads();
  for (int p = threadIdx.x; p < np; p += DEC_THREADS)
    a.act_sh[r.p0 + p] = f32_to_bf16(swiglu_bf16(gu[2 * p], gu[2 * p + 1]));
}

// Diagnostics: SM-cycle stamps of CTA 0 for one token (the last one decoded),
// 16 per layer; a block-wide sync before each stamp attributes the time of the
// slowest warp of the CTA.
constexpr int DEC_STAMPS = 16;
YN_DEV void stamp(const DecodeArgs& a, int tok, int layer, int slot) {
  if (a.timing && blockIdx.x == 0 && tok == a.n_tokens - 1) {
    __syncthreads();
    if (threadIdx.x == 0) a.timing[(size_t)layer * DEC_STAMPS + slot] = (long long)clock64();
  }
}

// Copy descriptor of layer `idx` into a shared-memory slot (threads 0..20).
YN_DEV void load_layer(DecLayer* slot, const DecLayer* table, int idx) {
  constexpr int NW = sizeof(DecLayer) / 16;
  static_assert(sizeof(DecLayer) % 16 == 0, "DecLayer must be a multiple of 16 bytes");
  if (threadIdx.x < NW)
    reinterpret_cast<uint4*>(slot)[threadIdx.x] = __ldcg(reinterpret_cast<const uint4*>(table + idx) + threadIdx.x);
}

template <int CPL8, int CPLS>
__global__ void __launch_bounds__(DEC_THREADS, 1) k_stack_decode(const DecodeArgs a) {
  constexpr int NBW = (CPL8 + 1) / 2;  // 64-code blocks of the hidden dimension per warp in P2
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* barA = reinterpret_cast<uint64_t*>(smem);
  uint64_t* barC = reinterpret_cast<uint64_t*>(smem + 16);
  uint64_t* barD = reinterpret_cast<uint64_t*>(smem + 24);
  float* red = reinterpret_cast<float*>(smem + 32);           // 16 floats
  int* eflag = reinterpret_cast<int*>(smem + 128);
  uint16_t* hs = reinterpret_cast<uint16_t*>(smem + a.off_hs);
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem + a.off_xs);
  XBlock* xf = reinterpret_cast<XBlock*>(smem + a.off_xf);           // [(K+1) * 8 blocks * 4 lanes]
  uint8_t* rt = smem + a.off_route;
  float* rv = reinterpret_cast<float*>(rt);                             // E
  uint32_t* keys = reinterpret_cast<uint32_t*>(rt + 4 * a.E);           // E
  uint32_t* cand = keys + a.E;                                          // WARPS*K
  int32_t* ids = reinterpret_cast<int32_t*>(cand + DEC_WARPS * DEC_MAX_K);
  float* wts = reinterpret_cast<float*>(ids + DEC_MAX_K);
  float* xsc = wts + DEC_MAX_K;                                         // K+1 fragment scales
  float* rbias_s = xsc + DEC_MAX_K + 4;                                 // 64 + shared gate/up scratch
  DecLayer* lay = reinterpret_cast<DecLayer*>(rbias_s + 64 + 256);      // 3 slots
  float* part = reinterpret_cast<float*>(smem + a.off_part);
  uint8_t* Abuf = smem + a.off_A;
  uint8_t* cbuf = smem + a.off_C;
  uint8_t* dbuf = smem + a.off_D;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, b = blockIdx.x;
  const int H = a.H, E = a.E, K = a.K, I = a.I;
  const P1Range r1 = p1_range(b, G, E, a.Ish);
  const int nr1 = r1.r1 - r1.r0;
  const int U = K * I;
  const int u0 = (int)((long long)b * U / G), u1 = (int)((long long)(b + 1) * U / G);
  const int d0 = (int)((long long)b * H / G), d1 = (int)((long long)(b + 1) * H / G);
  const int nd = d1 - d0;
  const int total_steps = a.n_tokens * a.n_layers;

  if (tid == 0) {
    mbar_init(barA, 1);
    mbar_init(barC, 1);
    mbar_init(barD, 1);
    fence_mbar_init();
  }
  load_layer(&lay[0], a.layers, 0);
  load_layer(&lay[1], a.layers, a.n_layers > 1 ? 1 : 0);
  __syncthreads();
  if (warp == 0) issue_p1(lay[0], r1, p1_tile(Abuf, r1, H, lay[0].router.gs, shared_gs(lay[0])), H, barA);
  unsigned gen = 0;
  uint32_t phA = 0;
  bool pendA = true;
  auto drain = [&]() {
    if (pendA) mbar_wait_block(barA, phA, nullptr);
  };

  for (int step = 0; step < total_steps; ++step) {
    const int tok = step / a.n_layers, layer = step % a.n_layers;
    const DecLayer& L = lay[step % 3];
    const DecLayer& Ln = lay[(step + 1) % 3];
    const bool more = step + 1 < total_steps;
    stamp(a, tok, layer, 0);
    // -------- P1: norm; router + shared rows (tile prefetched during the previous layer)
    {
      const uint16_t* hin = (layer == 0) ? a.inputs + (size_t)tok * H : a.hbuf + (size_t)(step & 1) * H;
      const float bv = (tid < nr1 && L.rbias) ? __ldcg(L.rbias + r1.r0 + tid) : 0.0f;
      if (tid < H / 8) reinterpret_cast<uint4*>(hs)[tid] = __ldcg(reinterpret_cast<const uint4*>(hin) + tid);
      if (tid < 64) rbias_s[tid] = bv;
    }
    const P1Tile t1 = p1_tile(Abuf, r1, H, L.router.gs, shared_gs(L));
    stamp(a, tok, layer, 1);
    const bool a_ok = mbar_wait_block(barA, phA, a.err);
    stamp(a, tok, layer, 2);
    if (a_ok) {
      phA ^= 1;
      pendA = false;
      rmsnorm_smem(hs, t1.norm, H, a.eps, xs, red);
      stamp(a, tok, layer, 3);
      p1_compute<CPL8>(a, L, r1, t1, xs, rbias_s);
    }
    stamp(a, tok, layer, 4);
    if (grid_barrier(a, gen, eflag)) { drain(); return; }
    stamp(a, tok, layer, 5);
    // -------- P2: prefetch next layer's P1 tile, route, C/D tiles, gate/up rows
    if (warp == 2 && more)
      issue_p1(Ln, r1, p1_tile(Abuf, r1, H, Ln.router.gs, shared_gs(Ln)), H, barA);
    pendA = more;
    if (step + 2 < total_steps) load_layer(&lay[(step + 2) % 3], a.layers, (step + 2) % a.n_layers);
    route_block(a.logits, E, K, a.norm_topk, rv, keys, cand, red, ids, wts);
    if (a.trace_ids && b == 0 && tid < K) a.trace_ids[((size_t)tok * a.n_layers + layer) * K + tid] = ids[tid];
    stamp(a, tok, layer, 6);
    bool ids_ok = true;
    for (int j = 0; j < K; ++j) {
      const int e = ids[j];
      const int sl = (e >= 0 && e < E) ? (L.slot_of ? L.slot_of[e] : e) : -1;
      if (sl < 0 || sl >= L.n_slots) ids_ok = false;
    }
    if (!ids_ok && tid == 0) raise_error(a.err, YN_ERR_BAD_SLOT);
    const int bits = L.rg.bits, gs = L.rg.gs;
    const CPlan cp = c_plan(u0, u1, I, H * bits / 8);
    if (ids_ok && warp == DEC_WARPS - 1) prefetch_d(a, L, ids, d0, nd);
    // max |x| of the normed row (power-of-two scale for the fp16 fragments)
    float mx = 0.0f;
    for (int i = tid; i < H; i += DEC_THREADS) mx = fmaxf(mx, fabsf(bf16_to_f32(xs[i])));
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < DEC_WARPS; ++w) mx = fmaxf(mx, red[w]);
    const float xscale = fp16_input_scale(mx);
    stamp(a, tok, layer, 7);
    stamp(a, tok, layer, 8);
    const bool c_ok = ids_ok;
    if (c_ok) {
      if (bits == 2) {
        if (gs == 32) p2_regs<2, 2, NBW, 5>(a, L, ids, cp, gs, xs, xscale, part);
        else p2_regs<2, 1, NBW, 5>(a, L, ids, cp, gs, xs, xscale, part);
      } else {
        if (gs == 32) p2_regs<4, 2, NBW, 5>(a, L, ids, cp, gs, xs, xscale, part);
        else p2_regs<4, 1, NBW, 5>(a, L, ids, cp, gs, xs, xscale, part);
      }
      __syncthreads();
      // gate/up rows of each n: sum the per-block contributions in block order
      const int nblk = H / 64;
      int off = 0;
      for (int s = 0; s < cp.nseg; ++s) {
        for (int i = tid; i < cp.nr[s]; i += DEC_THREADS) {
          float gsum = 0.0f, usum = 0.0f;
          for (int q = 0; q < nblk; ++q) {
            gsum = __fadd_rn(gsum, part[(size_t)q * cp.R + off + i]);
            usum = __fadd_rn(usum, part[(size_t)q * cp.R + off + cp.nr[s] + i]);
          }
          a.act[(size_t)cp.j[s] * I + cp.n0[s] + i] = f32_to_bf16(swiglu_bf16(bf16r(gsum), bf16r(usum)));
        }
        off += 2 * cp.nr[s];
      }
    }
    stamp(a, tok, layer, 9);
    if (grid_barrier(a, gen, eflag)) { drain(); return; }
    stamp(a, tok, layer, 10);
    // -------- P3: fragments of every column's activations, down rows, combine
    if (bits == 2) p3_frags<2>(a, xf, xsc);
    else p3_frags<4>(a, xf, xsc);
    __syncthreads();
    stamp(a, tok, layer, 11);
    const float sgv = a.Ish ? __ldcg(a.sgate) : 0.0f;
    stamp(a, tok, layer, 12);
    stamp(a, tok, layer, 13);
    const bool d_ok = ids_ok;
    if (d_ok) {
      if (bits == 2) {
        if (gs == 32) p3_regs<2, 2, 6>(a, L, ids, d0, nd, xf, xsc, part);
        else p3_regs<2, 1, 6>(a, L, ids, d0, nd, xf, xsc, part);
      } else {
        if (gs == 32) p3_regs<4, 2, 6>(a, L, ids, d0, nd, xf, xsc, part);
        else p3_regs<4, 1, 6>(a, L, ids, d0, nd, xf, xsc, part);
      }
    }
    __syncthreads();
    stamp(a, tok, layer, 14);
    if (d_ok) {
      uint16_t* hout = (layer == a.n_layers - 1) ? a.outputs + (size_t)tok * H : a.hbuf + (size_t)((step + 1) & 1) * H;
      for (int t = tid; t < nd; t += DEC_THREADS) {
        float acc = 0.0f;
        for (int j = 0; j < K; ++j) {
          float y = 0.0f;
#pragma unroll
          for (int q = 0; q < 8; ++q) y = __fadd_rn(y, part[(size_t)(j * 8 + q) * DEC_MAX_DROWS + t]);
          acc = __fadd_rn(acc, bf16r(__fmul_rn(bf16r(y), wts[j])));
        }
        float o = bf16r(acc);
        if (a.Ish) {
          float y = 0.0f;
#pragma unroll
          for (int q = 0; q < 8; ++q) y = __fadd_rn(y, part[(size_t)(K * 8 + q) * DEC_MAX_DROWS + t]);
          o = bf16r(__fadd_rn(o, bf16r(__fmul_rn(sgv, bf16r(y)))));
        }
        o = bf16r(__fadd_rn(bf16_to_f32(hs[d0 + t]), o));
        hout[d0 + t] = f32_to_bf16(o);
      }
    }
    stamp(a, tok, layer, 15);
    if (grid_barrier(a, gen, eflag)) { drain(); return; }
  }
}

}  // namespace ynb
