// Persistent whole-stack bs1 decode kernel (one cooperative launch decodes
// n_tokens tokens sequentially through every layer).
//
// Compiled shape: hidden 2048, 512 experts, expert and shared-expert
// intermediate 512, top-k <= 16, routed experts 2- or 4-bit with groups of 32
// or 64, dense matrices (router, shared expert) 8-bit with groups of 64. All
// index arithmetic uses these constants, and every phase is a short rolled
// loop, so the hot code of a layer stays small.
//
// Grid = one CTA per SM (co-resident, cooperative launch), 512 threads.
// Per layer three phases; P1 -> P2 passes the router logits as "flagged
// words" (below), P2 -> P3 and P3 -> next P1 are grid barriers:
//   P1  RMSNorm(h) -> router logits, shared-expert gate/up/SwiGLU, shared gate
//       (each CTA owns a cost-balanced slice of those rows; its tile was
//       copied into shared memory during the previous layer). The
//       tensor-core fragments of the normed row are built here too.
//   P2  routing (every CTA, redundantly, from the 512 logits); each CTA then
//       copies its gate/up rows (tiles of 8 units: 8 gate rows + 8 up
//       rows of one expert) and the down rows it needs in P3, and computes its
//       units' SwiGLU activations.
//   P3  each CTA owns <= 16 consecutive output rows: routed + shared down
//       projections of those rows, the weighted combine and the residual.
// Flagged words: each router logit is stored as one aligned 64-bit word
// {fp32 payload, epoch} with a relaxed gpu-scope store, epoch = decode step
// + 1; in routing every thread polls its expert's word with relaxed gpu-scope
// loads until the epoch matches, so the data read is the synchronisation (no
// fence, no counter, one load in flight per thread). The words are
// double-buffered by step parity: at a token boundary a CTA may start the next
// token's first layer while others still route the last one.
// Grid barriers are a global counter (release add / acquire poll; the poll
// also watches the error word). Every wait has a wall-clock limit; on any
// error each CTA waits for its copies in flight and returns. Reference
// behaviour: moe_prefetch/orchestrator.py:308-343 layer
// loop with every expert resident (mlx_backend.py:302-316 post-attention and
// routing, :442-459 routed experts, :438-440 shared expert and combine).
//
// Tensor-core GEMV ("super-block" form). A lane owns 16 contiguous bytes of a
// weight row per super-block (4 lanes = 64 bytes of a row); a 16-row tile of
// one super-block is a chain of m16n8k16 MMAs in which the 8 N columns of B
// carry the activation masked to one quantisation group each: column n is
// nonzero only at the k-slots whose codes belong to group n. D then holds the
// per-group dot products of each row in separate columns, and the group scale
// and bias are applied in fp32 afterwards (y = s*D/x_scale + b*sum(x_group)).
#pragma once
#include "yn_common.cuh"
#include "yn_moe.cuh"
#include "yn_qdot.cuh"
#include "yn_mma.cuh"

namespace ynb {

constexpr int DEC_THREADS = 512;
constexpr int DEC_WARPS = DEC_THREADS / 32;
constexpr int DEC_H = 2048, DEC_E = 512, DEC_I = 512;
constexpr int DEC_MAX_K = 16;
constexpr int DEC_MAX_OCT = 8;       // gate/up tiles (8 units each) per CTA
constexpr int DEC_MAX_DROWS = 16;    // output rows per CTA in P3 (one MMA tile)
constexpr int DEC_DGS = 64;          // group size of the 8-bit dense matrices
constexpr int DEC_STAMPS = 16;

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
  int K, Ish, norm_topk;
  float eps;
  const DecLayer* layers;
  int n_layers;
  const uint16_t* inputs;
  int n_tokens;
  uint16_t* outputs;
  // flagged router logits {fp32 (low 32 bits), epoch (high 32 bits)},
  // two buffers (step parity); zeroed before every launch
  unsigned long long* f_logits;  // (2, E)
  uint16_t* hbuf;      // (2, H) hidden row between layers
  uint16_t* act;       // (K, I) routed SwiGLU activations
  uint16_t* act_sh;    // (Ish) shared-expert SwiGLU activations
  float* sgate;        // (1) shared-expert gate
  int32_t* trace_ids;  // (n_tokens, n_layers, K) or null
  uint16_t* trace_h;   // (n_tokens, n_layers, H) each layer's input row, or null
  float* trace_w;      // (n_tokens, n_layers, K) routed weights, or null
  unsigned* bar;       // grid barrier counter (zeroed before every launch)
  int* err;
  long long* timing;   // (n_layers, DEC_STAMPS, grid) for the last token, or null
  // shared-memory carve (byte offsets)
  int off_hs, off_xs, off_route, off_xf2, off_xf3, off_part, off_A, off_C, off_D;
  int c_rows;          // rows reserved per code / scale block of the C tile (8 * max tiles)
  int c_rb, c_sb;      // bytes reserved per C code row / scale row
  int d_rb, d_sb;      // bytes reserved per D code row / scale row (routed)
};

// ------------------------------------------------------------ flagged words
using u64 = unsigned long long;
YN_DEV void put_flag(u64* p, uint32_t payload, uint32_t epoch) {
  const u64 v = ((u64)epoch << 32) | payload;
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
YN_DEV u64 get_flag(const u64* p) {
  u64 v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Payload of *p once it carries `epoch`. On an error raised elsewhere, or
// after 2 s (then the error is raised here), sets `fail` and returns 0.
YN_DEV uint32_t wait_flag(const u64* p, uint32_t epoch, int* err, bool& fail) {
  u64 v = get_flag(p);
  if ((uint32_t)(v >> 32) == epoch) return (uint32_t)v;
  const uint64_t t0 = globaltimer_ns();
  for (unsigned it = 1;; ++it) {
    v = get_flag(p);
    if ((uint32_t)(v >> 32) == epoch) return (uint32_t)v;
    if ((it & 63) == 0) {
      if (*reinterpret_cast<volatile int*>(err)) break;
      if (globaltimer_ns() - t0 > 2000000000ull) {
        raise_error(err, YN_ERR_BULK_TIMEOUT);
        break;
      }
    }
  }
  fail = true;
  return 0;
}

// ---------------------------------------------------------------- barrier
// Grid barrier in two halves so that a CTA can issue copies for the next
// phase between its arrival and the release. Arrival: block sync, then one
// release add on the counter. Wait: thread 0 polls the counter with acquire
// loads (watching the error word every 64 polls and a 2 s limit), then a
// block sync. Returns true (block-uniform) when the decode must stop.
YN_DEV void grid_arrive(const DecodeArgs& a) {
  __syncthreads();
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar) : "memory");
}
YN_DEV bool grid_wait(const DecodeArgs& a, unsigned target, int* flag) {
  if (threadIdx.x == 0) {
    int stop = 0;
    const uint64_t t0 = globaltimer_ns();
    for (unsigned it = 0;; ++it) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.bar) : "memory");
      if (v >= target) break;
      if ((it & 63) == 63) {
        if (*reinterpret_cast<volatile int*>(a.err)) { stop = 1; break; }
        if (globaltimer_ns() - t0 > 2000000000ull) {
          raise_error(a.err, YN_ERR_BULK_TIMEOUT);
          stop = 1;
          break;
        }
      }
    }
    *flag = stop;
  }
  __syncthreads();
  return *flag != 0;
}

// --------------------------------------------------------------- P1 slices
// P1 units: router rows (cost 1), shared gate/up row pairs (cost 2), the
// shared_expert_gate row (cost 1); CTA b takes the units whose cumulative
// cost starts in [b*C/G, (b+1)*C/G).
struct P1Range {
  int r0, r1;   // router rows
  int p0, p1;   // shared pairs
  int sg;       // 1 if this CTA owns the shared_expert_gate row
};
YN_DEV int p1_unit_at(int c, int Ish) {
  if (c <= DEC_E) return c;
  if (c <= DEC_E + 2 * Ish) return DEC_E + (c - DEC_E + 1) / 2;
  return DEC_E + Ish + (c - DEC_E - 2 * Ish);
}
YN_DEV P1Range p1_range(int b, int G, int Ish) {
  const int C = DEC_E + 2 * Ish + (Ish ? 1 : 0);
  const int lo = (int)((long long)b * C / G), hi = (int)((long long)(b + 1) * C / G);
  const int u0 = p1_unit_at(lo, Ish), u1 = p1_unit_at(hi, Ish);
  P1Range r;
  r.r0 = min(u0, DEC_E);
  r.r1 = min(u1, DEC_E);
  r.p0 = min(max(u0 - DEC_E, 0), Ish);
  r.p1 = min(max(u1 - DEC_E, 0), Ish);
  r.sg = (Ish > 0 && u0 <= DEC_E + Ish && u1 > DEC_E + Ish) ? 1 : 0;
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

// Tiles move with 16-byte cp.async (L2 -> shared, no L1 allocation): every
// thread issues a few, then arrives on the tile's mbarrier with
// cp.async.mbarrier.arrive.noinc, which fires when all of that thread's
// earlier copies have landed (barrier count = DEC_THREADS).
YN_DEV void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
YN_DEV void cp_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
YN_DEV void warp_copy(uint8_t* dst, const uint8_t* src, uint32_t bytes, int lane) {
  for (uint32_t o = (uint32_t)lane * 16; o < bytes; o += 512) cp16(dst + o, src + o);
}
constexpr int DEC_DSB = DEC_H / DEC_DGS * 2;   // scale-row bytes of a dense 2048-column matrix

YN_DEV P1Tile p1_tile(uint8_t* base, const P1Range& r) {
  P1Tile t;
  size_t o = 0;
  const size_t nr = r.r1 - r.r0, np = r.p1 - r.p0;
  t.norm = (uint16_t*)(base + o); o += a16d((size_t)DEC_H * 2);
  t.rc = base + o; o += a16d(nr * DEC_H);
  t.rs = (uint16_t*)(base + o); o += a16d(nr * DEC_DSB);
  t.rbv = (uint16_t*)(base + o); o += a16d(nr * DEC_DSB);
  t.gc = base + o; o += a16d(np * DEC_H);
  t.gsc = (uint16_t*)(base + o); o += a16d(np * DEC_DSB);
  t.gbi = (uint16_t*)(base + o); o += a16d(np * DEC_DSB);
  t.uc = base + o; o += a16d(np * DEC_H);
  t.usc = (uint16_t*)(base + o); o += a16d(np * DEC_DSB);
  t.ubi = (uint16_t*)(base + o); o += a16d(np * DEC_DSB);
  t.sc = base + o; o += a16d(r.sg ? (size_t)DEC_H : 0);
  t.ssc = (uint16_t*)(base + o); o += a16d(r.sg ? DEC_DSB : 0);
  t.sbi = (uint16_t*)(base + o); o += a16d(r.sg ? DEC_DSB : 0);
  return t;
}

// Copies of one layer's P1 tile (every CTA also takes the whole norm
// weight): warps w0.. copy the 13 pieces round-robin; then every thread of
// the CTA arrives on `bar` (once per layer).
YN_DEV void issue_p1(const DecLayer& L, const P1Range& r, const P1Tile& t, uint64_t* bar, int w0) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t nr = r.r1 - r.r0, np = r.p1 - r.p0;
  const uint8_t* rs = reinterpret_cast<const uint8_t*>(L.router.s);
  const uint8_t* rb = reinterpret_cast<const uint8_t*>(L.router.b);
  for (int piece = warp - w0; warp >= w0 && piece < 13; piece += DEC_WARPS - w0) {
  void* dst = nullptr;
  const void* src = nullptr;
  uint32_t bytes = 0;
  switch (piece) {
    case 0: dst = t.norm; src = L.norm; bytes = (uint32_t)DEC_H * 2; break;
    case 1: dst = t.rc; src = L.router.w + (size_t)r.r0 * DEC_H; bytes = nr * DEC_H; break;
    case 2: dst = t.rs; src = rs + (size_t)r.r0 * DEC_DSB; bytes = nr * DEC_DSB; break;
    case 3: dst = t.rbv; src = rb + (size_t)r.r0 * DEC_DSB; bytes = nr * DEC_DSB; break;
    case 4: dst = t.gc; src = L.sg.w + (size_t)r.p0 * DEC_H; bytes = np * DEC_H; break;
    case 5: dst = t.gsc; src = reinterpret_cast<const uint8_t*>(L.sg.s) + (size_t)r.p0 * DEC_DSB; bytes = np * DEC_DSB; break;
    case 6: dst = t.gbi; src = reinterpret_cast<const uint8_t*>(L.sg.b) + (size_t)r.p0 * DEC_DSB; bytes = np * DEC_DSB; break;
    case 7: dst = t.uc; src = L.su.w + (size_t)r.p0 * DEC_H; bytes = np * DEC_H; break;
    case 8: dst = t.usc; src = reinterpret_cast<const uint8_t*>(L.su.s) + (size_t)r.p0 * DEC_DSB; bytes = np * DEC_DSB; break;
    case 9: dst = t.ubi; src = reinterpret_cast<const uint8_t*>(L.su.b) + (size_t)r.p0 * DEC_DSB; bytes = np * DEC_DSB; break;
    case 10: dst = t.sc; src = L.sgt.w; bytes = r.sg ? (uint32_t)DEC_H : 0u; break;
    case 11: dst = t.ssc; src = L.sgt.s; bytes = r.sg ? (uint32_t)DEC_DSB : 0u; break;
    case 12: dst = t.sbi; src = L.sgt.b; bytes = r.sg ? (uint32_t)DEC_DSB : 0u; break;
    default: break;
  }
  warp_copy(reinterpret_cast<uint8_t*>(dst), reinterpret_cast<const uint8_t*>(src), bytes, lane);
  }
  cp_arrive(bar);
}

// RMSNorm in the canonical 128-thread order (threads 128.. idle in the sum);
// returns max |x| of the normed row (every thread).
YN_DEV float rmsnorm_smem(const uint16_t* h, const uint16_t* w_g, float eps, uint16_t* out, float* red) {
  const int tid = threadIdx.x;
  float ss = 0.0f;
  if (tid < 128)
    for (int i = tid; i < DEC_H; i += 128) {
      const float v = bf16_to_f32(h[i]);
      ss = __fmaf_rn(v, v, ss);
    }
  if (tid < 128) {
    ss = group_sum_bfly(ss, 32);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
  }
  __syncthreads();
  // warp partials in warp order and r = 1 / sqrt(.) with two roundings, as the
  // canonical RMSNorm defines them (a fused rsqrt rounds once and can differ
  // in the last bit)
  const float tot = __fadd_rn(__fadd_rn(__fadd_rn(red[0], red[1]), red[2]), red[3]);
  // DEC_H is a power of two, so tot * (1 / H) is tot / H exactly
  static_assert((DEC_H & (DEC_H - 1)) == 0, "hidden size: a power of two");
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(tot, 1.0f / (float)DEC_H), eps)));
  float mx = 0.0f;
#pragma unroll
  for (int i = tid; i < DEC_H; i += DEC_THREADS) {
    const uint16_t o = f32_to_bf16(__fmul_rn(bf16_to_f32(w_g[i]), bf16r(__fmul_rn(bf16_to_f32(h[i]), r))));
    out[i] = o;
    mx = fmaxf(mx, fabsf(bf16_to_f32(o)));
  }
  // mx >= 0: the unsigned order of the bits is the float order
  mx = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(mx)));
  if ((tid & 31) == 0) red[8 + (tid >> 5)] = mx;
  __syncthreads();
  return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(red[8 + (tid & 15)])));
}

// P1 compute: router rows, shared pairs, shared_expert_gate (canonical fp32
// row dot, one row per warp step, bit-exact with the oracle).
YN_DEV void p1_compute(const DecodeArgs& a, const P1Range& r, const P1Tile& t, const uint16_t* xs,
                       const float* rbias_s, float* gu, int par, uint32_t ep) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int LPR = 32, CPL = DEC_H / 16 / LPR;
  constexpr int NGD = DEC_H / DEC_DGS;
  XF32<8, CPL, 1> X;
  load_x_f32<8, CPL, 1>(X, xs, lane, LPR);
  const int nr = r.r1 - r.r0, np = r.p1 - r.p0;
  const int ntask = nr + 2 * np + r.sg;
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
      else a.sgate[0] = bf16r(sigmoid_f32(bf16r(v)));
    }
  }
  __syncthreads();
  for (int p = threadIdx.x; p < np; p += DEC_THREADS)
    a.act_sh[r.p0 + p] = f32_to_bf16(swiglu_bf16(gu[2 * p], gu[2 * p + 1]));
}

// ------------------------------------------------------------------ routing
// Block-wide routing of the 512 logits (thread t <-> expert t; each thread
// waits for its flagged logit; false when that wait failed; *ids_ok = whether
// every routed expert has a slot in layer L) in the
// canonical order of the oracle: max (order-free), exp per element, sum per
// lane over e = lane + 32 i then a butterfly (warp 0), bf16 probabilities,
// then top-k by the unique key (bf16 prob << 16 | 0xFFFF - id): per-warp
// top-k over its 32 experts, merged by warp 0. Results in shared memory.
YN_DEV bool route_block(const u64* f_logits, uint32_t ep, int* err, int K, int norm, float* v /* E */,
                        uint32_t* cand /* 16*16 */, float* red, int32_t* ids_out, float* w_out,
                        const DecLayer& L, int* ids_ok) {
  static_assert(DEC_E == DEC_THREADS, "one expert per thread");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  bool fail = false;
  const float x = __uint_as_float(wait_flag(f_logits + tid, ep, err, fail));
  if (__syncthreads_or(fail)) return false;
  float m = warp_max_redux(x);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = warp_max_redux(red[lane & 15]);
  v[tid] = yn_expf(__fsub_rn(x, m));
  __syncthreads();
  if (warp == 0) {
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < DEC_E / 32; ++i) s = __fadd_rn(s, v[lane + 32 * i]);
    s = group_sum_bfly(s, 32);
    if (lane == 0) red[16] = s;
  }
  __syncthreads();
  const float p = bf16r(__fdiv_rn(v[tid], red[16]));
  uint32_t key = ((uint32_t)f32_to_bf16(p) << 16) | (uint32_t)(0xFFFF - tid);
  for (int j = 0; j < K; ++j) {
    const uint32_t top = __reduce_max_sync(0xffffffffu, key);
    if (key == top) key = 0u;
    if (lane == 0) cand[warp * DEC_MAX_K + j] = top;
  }
  __syncthreads();
  if (warp == 0) {
    constexpr int NC = DEC_WARPS * DEC_MAX_K / 32;
    uint32_t mine[NC];
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int cix = lane + 32 * i;
      mine[i] = ((cix % DEC_MAX_K) < K) ? cand[cix] : 0u;
    }
    float wsum = 0.0f, myp = 0.0f;
    int myid = 0;
    for (int j = 0; j < K; ++j) {
      uint32_t best = 0;
#pragma unroll
      for (int i = 0; i < NC; ++i) best = max(best, mine[i]);
      const uint32_t top = __reduce_max_sync(0xffffffffu, best);
#pragma unroll
      for (int i = 0; i < NC; ++i)
        if (mine[i] == top) mine[i] = 0u;
      const float pj = bf16_to_f32((uint16_t)(top >> 16));
      wsum = __fadd_rn(wsum, pj);
      if (lane == j) {
        myp = pj;
        myid = 0xFFFF - (int)(top & 0xFFFFu);
      }
    }
    const float sb = bf16r(wsum);
    bool bad = false;
    if (lane < K) {
      ids_out[lane] = myid;
      w_out[lane] = norm ? bf16r(__fdiv_rn(myp, sb)) : myp;
      const int sl = L.slot_of ? L.slot_of[myid] : myid;   // the expert's slot must exist
      bad = sl < 0 || sl >= L.n_slots;
    }
    const unsigned anybad = __ballot_sync(0xffffffffu, bad);
    if (lane == 0) *ids_ok = anybad == 0u;
  }
  __syncthreads();
  return true;
}

// ------------------------------------------------------- super-block GEMV
template <int BITS>
struct Sb {
  static constexpr int W = MmaFmt<BITS>::WORDS;  // code words per 8-pair unpack unit
  static constexpr int U = 4 / W;                 // units per lane per super-block
  static constexpr int CPL = 16 * U;              // codes per lane
  static constexpr int CODES = 4 * CPL;           // codes per row per super-block (64 bytes)
  static constexpr int FRAG = 8 * U;              // activation fragment words per lane
};

// Fragment word w of lane c of super-block sb of a bf16 vector x: the pair
// (x[lo], x[hi]) of unpack pair p = w % 8 of unit u = w / 8, pre-scaled by
// `scale` and divided by the pair's code multiplier, as fp16.
template <int BITS>
YN_DEV uint32_t frag_word(const uint16_t* x, float scale, int sb, int c, int w) {
  using S = Sb<BITS>;
  const int u = w >> 3, p = w & 7;
  const int base = sb * S::CODES + c * S::CPL + 16 * u;
  const float m = __fmul_rn(scale, MmaFmt<BITS>::inv_mult(p));
  __half2 h = __floats2half2_rn(__fmul_rn(bf16_to_f32(x[base + MmaFmt<BITS>::lo(p)]), m),
                                __fmul_rn(bf16_to_f32(x[base + MmaFmt<BITS>::hi(p)]), m));
  return *reinterpret_cast<uint32_t*>(&h);
}

// Fragments of an n-code vector: word index i = ((sb * 4 + c) * FRAG + w).
template <int BITS>
YN_DEV void build_frags(const uint16_t* x, int n, float scale, uint32_t* out, int t0, int nthreads) {
  using S = Sb<BITS>;
  for (int i = t0; i < n / 2; i += nthreads) {
    const int sb = i / (4 * S::FRAG), rem = i % (4 * S::FRAG);
    out[i] = frag_word<BITS>(x, scale, sb, rem / S::FRAG, rem % S::FRAG);
  }
}

// One 16-row tile x one super-block. rg / rg8: this lane's 16 bytes of rows g
// and g+8; xf: lane c's fragment words. d = D[g][2c], D[g][2c+1],
// D[g+8][2c], D[g+8][2c+1]; column n = dot over group n of the super-block
// (times the activation scale) plus the group's unpack offset.
// 32 bytes of zeros in the decode kernels' shared-memory header (written at
// kernel start): the B fragments of lanes outside a unit's group.
constexpr int DEC_ZERO_OFF = 224;
YN_DEV const uint4* dec_zero_block() {
  extern __shared__ __align__(128) uint8_t smem[];
  return reinterpret_cast<const uint4*>(smem + DEC_ZERO_OFF);
}

template <int BITS, int GS>
YN_DEV void sb_mma(const uint8_t* rg, const uint8_t* rg8, const uint32_t* xf, int g, int c, float (&d)[4]) {
  using S = Sb<BITS>;
  const uint4 va = *reinterpret_cast<const uint4*>(rg);
  const uint4 vb = *reinterpret_cast<const uint4*>(rg8);
  const uint32_t wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
  const uint4* zero = dec_zero_block();
  float acc[S::U][4];
#pragma unroll
  for (int u = 0; u < S::U; ++u) {
    acc[u][0] = acc[u][1] = acc[u][2] = acc[u][3] = 0.f;
    uint32_t pa[8], pb[8];
    MmaFmt<BITS>::unpack_raw(wa + u * S::W, pa);
    MmaFmt<BITS>::unpack_raw(wb + u * S::W, pb);
    // The unit's fragment words in the lanes of its group, zeros elsewhere, both
    // as plain shared-memory loads: choosing the address keeps the B operands
    // straight out of the loads, which lets the mma chains of the units overlap
    // (a branch or a select of the values here measured 2.1x slower per item).
    const uint4* src = (c * S::CPL + 16 * u) / GS == g ? reinterpret_cast<const uint4*>(xf) + 2 * u : zero;
    const uint4 x0 = src[0], x1 = src[1];
    const uint32_t xb[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const uint32_t A[4] = {pa[2 * m], pb[2 * m], pa[2 * m + 1], pb[2 * m + 1]};
      const uint32_t B[2] = {xb[2 * m], xb[2 * m + 1]};
      mma16816(acc[u], A, B);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float s = acc[0][i];
#pragma unroll
    for (int u = 1; u < S::U; ++u) s = __fadd_rn(s, acc[u][i]);
    d[i] = s;
  }
}

// Scale and bias of one row's two groups (columns 2c, 2c+1 of super-block sb),
// summed over the lane quad: every lane of the quad returns the row's
// super-block partial. s_row / b_row: fp16 scale / bias rows; xsum: group sums
// of x; off: group unpack offsets (removed from D first).
template <int BITS, int GS>
YN_DEV float sb_apply(float d0, float d1, const uint16_t* s_row, const uint16_t* b_row, const float* xsum,
                      const float* off, int sb, int c, float inv) {
  constexpr int NG = Sb<BITS>::CODES / GS;
  float v = 0.0f;
  if (2 * c < NG) {
    const int gi = sb * NG + 2 * c;
    d0 = __fsub_rn(d0, off[gi]);
    if (NG >= 2) d1 = __fsub_rn(d1, off[gi + 1]);
    if (NG >= 2) {
      const uint32_t s2 = *reinterpret_cast<const uint32_t*>(s_row + gi);
      const uint32_t b2 = *reinterpret_cast<const uint32_t*>(b_row + gi);
      v = __fmaf_rn(f16_to_f32((uint16_t)(s2 & 0xFFFFu)), __fmul_rn(d0, inv),
                    __fmul_rn(f16_to_f32((uint16_t)(b2 & 0xFFFFu)), xsum[gi]));
      v = __fadd_rn(v, __fmaf_rn(f16_to_f32((uint16_t)(s2 >> 16)), __fmul_rn(d1, inv),
                                 __fmul_rn(f16_to_f32((uint16_t)(b2 >> 16)), xsum[gi + 1])));
    } else {
      v = __fmaf_rn(f16_to_f32(s_row[gi]), __fmul_rn(d0, inv), __fmul_rn(f16_to_f32(b_row[gi]), xsum[gi]));
    }
  }
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
  return v;
}

// Per group of GS codes: the sum of x (fp32) and the unpack offset
// 1024 * sum(fp16(x * scale / mult)) of the fragment values fed to the MMA.
// Thread i takes codes [16i, 16i+16) (one unpack unit of one lane), then a
// butterfly over the GS/16 consecutive threads of a group; the first of them
// writes entry i / (GS/16). Every lane of the calling warp takes part.
template <int BITS, int GS>
YN_DEV void group_sums16(const uint16_t* x, int i, bool valid, float scale, float* xsum, float* off) {
  float s = 0.0f, o = 0.0f;
  if (valid) {
    const uint4 q0 = reinterpret_cast<const uint4*>(x + 16 * i)[0];
    const uint4 q1 = reinterpret_cast<const uint4*>(x + 16 * i)[1];
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float v = bf16_to_f32((uint16_t)((k & 1) ? w[k >> 1] >> 16 : w[k >> 1] & 0xFFFFu));
      s = __fadd_rn(s, v);
      const float m = __fmul_rn(scale, MmaFmt<BITS>::inv_mult(MmaFmt<BITS>::pair_of(k)));
      o = __fadd_rn(o, __half2float(__float2half_rn(__fmul_rn(v, m))));
    }
    o = __fmul_rn(o, 1024.0f);
  }
  s = group_sum_bfly(s, GS / 16);
  o = group_sum_bfly(o, GS / 16);
  if (valid && i % (GS / 16) == 0) {
    xsum[i / (GS / 16)] = s;
    off[i / (GS / 16)] = o;
  }
}

// Warp-level bounded wait (the result is warp-uniform).
YN_DEV bool mbar_wait_warp(uint64_t* bar, uint32_t phase, int* err) {
  const bool ok = mbar_wait_bounded(bar, phase, err);
  return __all_sync(0xffffffffu, ok ? 1 : 0) != 0;
}

// ------------------------------------------------------------ P2 / P3 tiles
// C tile (gate/up rows of this CTA's units), in shared memory:
//   codes: gate rows [c_rows][c_rb] then up rows [c_rows][c_rb];
//   scales/biases: gate scales, gate biases, up scales, up biases [c_rows][c_sb].
// Tile t (8 units) = C rows 8t..8t+7; a CTA's tiles span at most two experts
// ("segments"), whose rows are copied back to back.
struct CSeg {
  int n;       // segments (0..2)
  int j[2];    // routed column of each segment
  int n0[2];   // first unit row inside the expert
  int rows[2]; // units in the segment
};
YN_DEV CSeg c_segments(int o0, int o1) {
  CSeg s;
  s.n = 0;
  for (int o = o0; o < o1 && s.n < 2;) {
    const int j = o / (DEC_I / 8), oe = min(o1, (j + 1) * (DEC_I / 8));
    s.j[s.n] = j;
    s.n0[s.n] = (o % (DEC_I / 8)) * 8;
    s.rows[s.n] = (oe - o) * 8;
    ++s.n;
    o = oe;
  }
  return s;
}

YN_DEV const uint8_t* expert_record(const DecLayer& L, int e) {
  return L.ebase + (size_t)(L.slot_of ? L.slot_of[e] : e) * (size_t)L.stride;
}

// Copies of this CTA's C tile, issued by one warp tile by tile; tile t
// completes on its own mbarrier (count 1: lane 0 posts the tile's bytes), so
// P2 starts on tile 0 while later tiles are in flight. Per tile, six bulk
// copies from six lanes: the gate and up codes of its 8 rows and the four
// 8-row scale/bias pieces (each a contiguous run of whole 16-byte units).
// A tile (8 units) never crosses an expert boundary.
template <int BITS, int GS, class Args>
YN_DEV void copy_c(const Args& a, const DecLayer& L, const int32_t* ids, const CSeg& sg, int ntile, uint8_t* C,
                   uint64_t* barT, int t0, int tstep) {
  constexpr int RB = DEC_H * BITS / 8, SBH = DEC_H / GS * 2;
  static_assert(SBH % 16 == 0 && RB % 16 == 0, "bulk copies move whole 16-byte units");
  const int lane = threadIdx.x & 31;
  if (!ntile) return;
  const uint8_t* rec0 = expert_record(L, ids[sg.j[0]]);
  const uint8_t* rec1 = sg.n > 1 ? expert_record(L, ids[sg.j[1]]) : rec0;
  const size_t sbase = (size_t)2 * a.c_rows * a.c_rb;
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  for (int t = t0; t < ntile; t += tstep) {
    const int row = 8 * t, seg = row >= sg.rows[0] ? 1 : 0;
    const int n = sg.n0[seg] + (seg ? row - sg.rows[0] : row);
    const uint8_t* rec = seg ? rec1 : rec0;
    if (lane == 0) mbar_arrive_expect_tx(&barT[t], 16u * RB + 32u * SBH);
    __syncwarp();
    if (lane < 2) {   // gate and up codes: 8 rows each
      bulk_g2s(C + (size_t)lane * a.c_rows * a.c_rb + (size_t)row * RB, rec + L.rg.off[3 * lane] + (size_t)n * RB,
               8u * RB, &barT[t]);
    } else if (lane < 6) {   // gate s, gate b, up s, up b: 8 rows x SBH bytes each
      const int q = lane - 2;
      bulk_g2s(C + sbase + (size_t)q * a.c_rows * a.c_sb + (size_t)row * SBH,
               rec + L.rg.off[3 * (q >> 1) + 1 + (q & 1)] + (size_t)n * SBH, 8u * SBH, &barT[t]);
    }
  }
}

#ifndef YN_DEC_CW
#define YN_DEC_CW 1
#endif
constexpr int DEC_CW = YN_DEC_CW;  // warps that issue the C-tile copies (tile t by warp t % DEC_CW)


// D tile (down rows [d0, d0+nd) of every routed column and of the shared
// expert): codes [K][16][RBI] then shared [16][Ish]; scales / biases
// [K][16][SBI] each, then shared scales / biases [16][DEC_DSBI].
constexpr int DEC_DSBI = DEC_I / DEC_DGS * 2;  // scale-row bytes of the shared down_proj
struct DOff {
  size_t sh, rs, rb, ss, sb;
};
YN_DEV DOff d_offsets(const DecodeArgs& a) {
  DOff o;
  o.sh = (size_t)a.K * DEC_MAX_DROWS * a.d_rb;
  o.rs = o.sh + (size_t)DEC_MAX_DROWS * DEC_I;
  o.rb = o.rs + (size_t)a.K * DEC_MAX_DROWS * a.d_sb;
  o.ss = o.rb + (size_t)a.K * DEC_MAX_DROWS * a.d_sb;
  o.sb = o.ss + (size_t)DEC_MAX_DROWS * DEC_DSBI;
  return o;
}

// Copies of the D tile by one warp: column j < K (three pieces), or the
// shared expert's pieces for j == K.
template <int BITS, int GS>
YN_DEV void copy_d(const DecodeArgs& a, const DecLayer& L, const int32_t* ids, int d0, int nd, uint8_t* D, int j) {
  constexpr int RBI = DEC_I * BITS / 8, SBI = DEC_I / GS * 2;
  const int lane = threadIdx.x & 31, K = a.K;
  const DOff o = d_offsets(a);
  if (j < K) {
    const uint8_t* rec = expert_record(L, ids[j]);
    warp_copy(D + (size_t)j * DEC_MAX_DROWS * a.d_rb, rec + L.rg.off[6] + (size_t)d0 * RBI, (uint32_t)nd * RBI, lane);
    warp_copy(D + o.rs + (size_t)j * DEC_MAX_DROWS * a.d_sb, rec + L.rg.off[7] + (size_t)d0 * SBI, (uint32_t)nd * SBI,
              lane);
    warp_copy(D + o.rb + (size_t)j * DEC_MAX_DROWS * a.d_sb, rec + L.rg.off[8] + (size_t)d0 * SBI, (uint32_t)nd * SBI,
              lane);
  } else if (j == K && a.Ish) {
    warp_copy(D + o.sh, L.sd.w + (size_t)d0 * DEC_I, (uint32_t)nd * DEC_I, lane);
    warp_copy(D + o.ss, reinterpret_cast<const uint8_t*>(L.sd.s) + (size_t)d0 * DEC_DSBI, (uint32_t)nd * DEC_DSBI, lane);
    warp_copy(D + o.sb, reinterpret_cast<const uint8_t*>(L.sd.b) + (size_t)d0 * DEC_DSBI, (uint32_t)nd * DEC_DSBI, lane);
  }
}

// P2: gate/up dots of this CTA's tiles. Items (tile t, super-block sb) go
// round-robin over the warps; partial sums land in
// part[((t * 8 + row) * 2 + up) * NSB + sb].
template <int BITS, int GS, class Args>
YN_DEV void p2_tiles(const Args& a, int ntile, const uint8_t* C, const uint32_t* xf, const float* xsum,
                     float inv, float* part, uint64_t* barT, uint32_t phT) {
  using S = Sb<BITS>;
  constexpr int RB = DEC_H * BITS / 8, SBH = DEC_H / GS * 2, NSB = RB / 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const float* xoff = xsum + DEC_H / 32;
  const uint8_t* cg = C;
  const uint8_t* cu = C + (size_t)a.c_rows * a.c_rb;
  const uint8_t* sc = C + (size_t)2 * a.c_rows * a.c_rb;
  int waited = -1;
  bool ok = true;
  for (int it = warp; it < ntile * NSB; it += DEC_WARPS) {
    const int t = it / NSB, sb = it % NSB;
    if (t != waited) {
      ok = mbar_wait_warp(&barT[t], phT, a.err);
      waited = t;
    }
    if (!ok) continue;  // error raised; the grid barrier ends the decode
    const int row = t * 8 + g;
    float d[4];
    sb_mma<BITS, GS>(cg + (size_t)row * RB + sb * 64 + c * 16, cu + (size_t)row * RB + sb * 64 + c * 16,
                     xf + (sb * 4 + c) * S::FRAG, g, c, d);
    const uint16_t* gs_ = reinterpret_cast<const uint16_t*>(sc + (size_t)row * SBH);
    const uint16_t* gb_ = reinterpret_cast<const uint16_t*>(sc + (size_t)a.c_rows * a.c_sb + (size_t)row * SBH);
    const uint16_t* us_ = reinterpret_cast<const uint16_t*>(sc + (size_t)2 * a.c_rows * a.c_sb + (size_t)row * SBH);
    const uint16_t* ub_ = reinterpret_cast<const uint16_t*>(sc + (size_t)3 * a.c_rows * a.c_sb + (size_t)row * SBH);
    const float vg = sb_apply<BITS, GS>(d[0], d[1], gs_, gb_, xsum, xoff, sb, c, inv);
    const float vu = sb_apply<BITS, GS>(d[2], d[3], us_, ub_, xsum, xoff, sb, c, inv);
    if (c == 0) {
      part[(row * 2 + 0) * NSB + sb] = vg;
      part[(row * 2 + 1) * NSB + sb] = vu;
    }
  }
}

// P3: down dots of rows [d0, d0+16) for every routed column (BITS, GS) and
// the shared expert (8-bit, DEC_DGS). part[(j * 16 + row) * 8 + sb].
template <int BITS, int GS>
YN_DEV void p3_tiles(const DecodeArgs& a, const uint8_t* D, const uint32_t* xf3, const float* xsum3,
                     const float* xsc3, float* part) {
  constexpr int RBI = DEC_I * BITS / 8, SBI = DEC_I / GS * 2, NSBR = RBI / 64, NSBS = DEC_I / 64;
  constexpr int NGR = DEC_I / GS, NGS = DEC_I / DEC_DGS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int K = a.K;
  const DOff o = d_offsets(a);
  const float* off3 = xsum3 + (DEC_MAX_K + 1) * 16;
  const int nr = K * NSBR, nitems = nr + (a.Ish ? NSBS : 0);
  for (int it = warp; it < nitems; it += DEC_WARPS) {
    float d[4];
    int j, sb;
    if (it < nr) {
      j = it / NSBR;
      sb = it % NSBR;
      const uint8_t* cb = D + (size_t)j * DEC_MAX_DROWS * a.d_rb + sb * 64 + c * 16;
      sb_mma<BITS, GS>(cb + (size_t)g * RBI, cb + (size_t)(g + 8) * RBI, xf3 + j * (DEC_I / 2) + (sb * 4 + c) * Sb<BITS>::FRAG,
                       g, c, d);
      const size_t srow = (size_t)j * DEC_MAX_DROWS * a.d_sb + (size_t)g * SBI;
      const uint16_t* s0 = reinterpret_cast<const uint16_t*>(D + o.rs + srow);
      const uint16_t* b0 = reinterpret_cast<const uint16_t*>(D + o.rb + srow);
      const float inv = __frcp_rn(xsc3[j]);
      const float v0 = sb_apply<BITS, GS>(d[0], d[1], s0, b0, xsum3 + j * 16, off3 + j * 16, sb, c, inv);
      const float v1 = sb_apply<BITS, GS>(d[2], d[3], s0 + 8 * NGR, b0 + 8 * NGR, xsum3 + j * 16, off3 + j * 16, sb, c,
                                          inv);
      if (c == 0) {
        part[(j * 16 + g) * 8 + sb] = v0;
        part[(j * 16 + g + 8) * 8 + sb] = v1;
      }
    } else {
      j = K;
      sb = it - nr;
      const uint8_t* cb = D + o.sh + sb * 64 + c * 16;
      sb_mma<8, DEC_DGS>(cb + (size_t)g * DEC_I, cb + (size_t)(g + 8) * DEC_I,
                         xf3 + K * (DEC_I / 2) + (sb * 4 + c) * Sb<8>::FRAG, g, c, d);
      const uint16_t* s0 = reinterpret_cast<const uint16_t*>(D + o.ss + (size_t)g * DEC_DSBI);
      const uint16_t* b0 = reinterpret_cast<const uint16_t*>(D + o.sb + (size_t)g * DEC_DSBI);
      const float inv = __frcp_rn(xsc3[K]);
      const float v0 = sb_apply<8, DEC_DGS>(d[0], d[1], s0, b0, xsum3 + K * 16, off3 + K * 16, sb, c, inv);
      const float v1 = sb_apply<8, DEC_DGS>(d[2], d[3], s0 + 8 * NGS, b0 + 8 * NGS, xsum3 + K * 16, off3 + K * 16, sb,
                                            c, inv);
      if (c == 0) {
        part[(K * 16 + g) * 8 + sb] = v0;
        part[(K * 16 + g + 8) * 8 + sb] = v1;
      }
    }
  }
}

// Activation fragments for P3: routed columns (BITS) from act, the shared
// expert (8-bit) from act_sh. Warp j takes vector j: lane l holds values
// [16l, 16l+16), takes the vector's power-of-two scale (warp max) and its
// group sums, stages the values in shared memory and builds 8 fragment words.
// stage: (K+1) x 512 bf16 in shared memory.
template <int BITS, int GS>
YN_DEV void p3_frags(const DecodeArgs& a, uint16_t* stage, uint32_t* xf3, float* xsum3, float* xsc3) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, K = a.K;
  const int nvec = K + (a.Ish ? 1 : 0);
  float* off3 = xsum3 + (DEC_MAX_K + 1) * 16;
  for (int j = warp; j < nvec; j += DEC_WARPS) {
    const uint16_t* src = j < K ? a.act + (size_t)j * DEC_I : a.act_sh;
    uint16_t* x = stage + j * DEC_I;
    const uint4 q0 = __ldcg(reinterpret_cast<const uint4*>(src) + 2 * lane);
    const uint4 q1 = __ldcg(reinterpret_cast<const uint4*>(src) + 2 * lane + 1);
    reinterpret_cast<uint4*>(x)[2 * lane] = q0;
    reinterpret_cast<uint4*>(x)[2 * lane + 1] = q1;
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      m = fmaxf(m, fmaxf(fabsf(bf16_to_f32((uint16_t)(w[k] & 0xFFFFu))), fabsf(bf16_to_f32((uint16_t)(w[k] >> 16)))));
    const float scale = fp16_input_scale(warp_max(m));
    __syncwarp();
    uint32_t* out = xf3 + j * (DEC_I / 2);
    if (j < K) {
      using S = Sb<BITS>;
      group_sums16<BITS, GS>(x, lane, true, scale, xsum3 + j * 16, off3 + j * 16);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int wd = lane + 32 * i, sb = wd / (4 * S::FRAG), rem = wd % (4 * S::FRAG);
        out[wd] = frag_word<BITS>(x, scale, sb, rem / S::FRAG, rem % S::FRAG);
      }
    } else {
      using S = Sb<8>;
      group_sums16<8, DEC_DGS>(x, lane, true, scale, xsum3 + j * 16, off3 + j * 16);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int wd = lane + 32 * i, sb = wd / (4 * S::FRAG), rem = wd % (4 * S::FRAG);
        out[wd] = frag_word<8>(x, scale, sb, rem / S::FRAG, rem % S::FRAG);
      }
    }
    if (lane == 0) xsc3[j] = scale;
    if (lane == 0 && j == K) xsc3[DEC_MAX_K + 2] = __ldcg(a.sgate);  // shared-expert gate for the combine
  }
  __syncthreads();
}

// Diagnostics: global-timer stamps (ns) of every CTA for one token (the last
// one decoded), DEC_STAMPS per layer, at timing[(layer * DEC_STAMPS + slot) *
// gridDim.x + blockIdx.x]; a block-wide sync before each stamp attributes the
// time of the slowest warp of the CTA. Out of line: off the hot code path.
static __device__ __noinline__ void stamp_at(long long* timing, int layer, int slot) {
  __syncthreads();
  if (threadIdx.x == 0)
    timing[((size_t)layer * DEC_STAMPS + slot) * gridDim.x + blockIdx.x] = (long long)globaltimer_ns();
}
YN_DEV void stamp(const DecodeArgs& a, int tok, int layer, int slot) {
  if (a.timing && tok == a.n_tokens - 1) stamp_at(a.timing, layer, slot);
}

// Asynchronous copy of the descriptor of layer `idx` into a shared-memory
// slot (tracked by the next cp_arrive of the copying threads).
YN_DEV void load_layer_async(DecLayer* slot, const DecLayer* table, int idx) {
  constexpr int NW = sizeof(DecLayer) / 16;
  if (threadIdx.x < NW)
    cp16(reinterpret_cast<uint4*>(slot) + threadIdx.x, reinterpret_cast<const uint4*>(table + idx) + threadIdx.x);
}

// Copy descriptor of layer `idx` into a shared-memory slot.
YN_DEV void load_layer(DecLayer* slot, const DecLayer* table, int idx) {
  constexpr int NW = sizeof(DecLayer) / 16;
  static_assert(sizeof(DecLayer) % 16 == 0, "DecLayer must be a multiple of 16 bytes");
  if (threadIdx.x < NW)
    reinterpret_cast<uint4*>(slot)[threadIdx.x] = __ldcg(reinterpret_cast<const uint4*>(table + idx) + threadIdx.x);
}

// Layer format index: bits 2/4 x group 32/64.
YN_DEV int fmt_of(const DecLayer& L) { return (L.rg.bits == 4 ? 2 : 0) + (L.rg.gs == 32 ? 1 : 0); }

// Fragments and group sums of the normed row for P2 (format of layer L).
template <int BITS, int GS>
YN_DEV void p2_frags(const uint16_t* xs, float scale, uint32_t* xf2, float* xsum2) {
  float* off2 = xsum2 + DEC_H / 32;
  build_frags<BITS>(xs, DEC_H, scale, xf2, threadIdx.x, DEC_THREADS);
  if (threadIdx.x < DEC_H / 16) group_sums16<BITS, GS>(xs, threadIdx.x, true, scale, xsum2, off2);
}

// P2 after the tile dots: thread v takes units 2v and 2v+1 (same tile, so
// the same expert): gate/up sums over the super-blocks in order, SwiGLU, both
// bf16 activations in one 32-bit store.
template <int BITS>
YN_DEV void p2_swiglu(const DecodeArgs& a, const CSeg& sg, int ntile, const float* part, int v) {
  constexpr int NSB = DEC_H * BITS / 8 / 64;
  if (v >= ntile * 4) return;
  uint32_t pk = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int u = 2 * v + h;
    float gsum = 0.0f, usum = 0.0f;
#pragma unroll
    for (int q = 0; q < NSB; ++q) {
      gsum = __fadd_rn(gsum, part[(u * 2 + 0) * NSB + q]);
      usum = __fadd_rn(usum, part[(u * 2 + 1) * NSB + q]);
    }
    pk |= (uint32_t)f32_to_bf16(swiglu_bf16(bf16r(gsum), bf16r(usum))) << (16 * h);
  }
  const int u = 2 * v;
  const int s = (sg.n > 1 && u >= sg.rows[0]) ? 1 : 0;
  const int n = sg.n0[s] + (s ? u - sg.rows[0] : u);
  reinterpret_cast<uint32_t*>(a.act)[((size_t)sg.j[s] * DEC_I + n) / 2] = pk;
}

// Translation units that only need the building blocks above define
// YN_NO_STACK_DECODE_KERNEL (the kernel has external linkage: one definition).
#ifndef YN_NO_STACK_DECODE_KERNEL
__global__ void __launch_bounds__(DEC_THREADS, 1) k_stack_decode(const DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* barA = reinterpret_cast<uint64_t*>(smem);
  uint64_t* barT = reinterpret_cast<uint64_t*>(smem + 136);   // DEC_MAX_OCT tile barriers
  uint64_t* barD = reinterpret_cast<uint64_t*>(smem + 24);
  float* red = reinterpret_cast<float*>(smem + 32);           // 24 floats
  int* eflag = reinterpret_cast<int*>(smem + 128);
  int* ids_ok_s = reinterpret_cast<int*>(smem + 200);                  // routed experts all have slots
  uint16_t* hs = reinterpret_cast<uint16_t*>(smem + a.off_hs);
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem + a.off_xs);
  uint8_t* rt = smem + a.off_route;
  float* rv = reinterpret_cast<float*>(rt);                              // E
  uint32_t* cand = reinterpret_cast<uint32_t*>(rt + 4 * DEC_E);          // 16 * 16
  int32_t* ids = reinterpret_cast<int32_t*>(cand + DEC_WARPS * DEC_MAX_K);
  float* wts = reinterpret_cast<float*>(ids + DEC_MAX_K);
  float* xsc3 = wts + DEC_MAX_K;                                         // K + 1
  float* rbias_s = xsc3 + DEC_MAX_K + 4;                                 // 64
  float* gu = rbias_s + 64;                                              // 256
  DecLayer* lay = reinterpret_cast<DecLayer*>(gu + 256);                 // 3 slots
  uint32_t* xf2 = reinterpret_cast<uint32_t*>(smem + a.off_xf2);         // H / 2 words
  float* xsum2 = reinterpret_cast<float*>(xf2 + DEC_H / 2);              // H / 32
  uint32_t* xf3 = reinterpret_cast<uint32_t*>(smem + a.off_xf3);         // (K+1) * I / 2 words
  float* xsum3 = reinterpret_cast<float*>(xf3 + (DEC_MAX_K + 1) * (DEC_I / 2));  // (K+1) * 16
  float* part = reinterpret_cast<float*>(smem + a.off_part);
  uint8_t* Abuf = smem + a.off_A;
  uint8_t* C = smem + a.off_C;
  uint8_t* D = smem + a.off_D;

  const int tid = threadIdx.x, warp = tid >> 5;
  const int G = gridDim.x, b = blockIdx.x, K = a.K;
  const P1Range r1 = p1_range(b, G, a.Ish);
  const int nr1 = r1.r1 - r1.r0;
  const int noct = K * (DEC_I / 8);
  const int o0 = (int)((long long)b * noct / G), o1 = (int)((long long)(b + 1) * noct / G);
  const int ntile = o1 - o0;
  const CSeg sg = c_segments(o0, o1);
  const int d0 = (int)((long long)b * DEC_H / G), d1 = (int)((long long)(b + 1) * DEC_H / G);
  const int nd = d1 - d0;
  const int total_steps = a.n_tokens * a.n_layers;

  if (tid == 0) {
    mbar_init(barA, DEC_THREADS);
    for (int t = 0; t < DEC_MAX_OCT; ++t) mbar_init(&barT[t], 1);  // the issuing lane's expect_tx
    mbar_init(barD, DEC_THREADS);
    fence_mbar_init();
  }
  if (tid < 8) reinterpret_cast<uint32_t*>(smem + DEC_ZERO_OFF)[tid] = 0u;
  load_layer(&lay[0], a.layers, 0);
  load_layer(&lay[1], a.layers, a.n_layers > 1 ? 1 : 0);
  __syncthreads();
  issue_p1(lay[0], r1, p1_tile(Abuf, r1), barA, 0);
  uint32_t phA = 0, phT = 0, phD = 0;
  bool pendA = true, pendT = false, pendD = false;
  // before leaving on an error: let every copy in flight land (bounded)
  auto drain = [&]() {
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (pendA) mbar_wait_block(barA, phA, nullptr);
    if (pendT)
      for (int t = 0; t < ntile; ++t) mbar_wait_block(&barT[t], phT, nullptr);
    if (pendD) mbar_wait_block(barD, phD, nullptr);
  };

  unsigned gen = 0;
  for (int step = 0; step < total_steps; ++step) {
    const int tok = step / a.n_layers, layer = step % a.n_layers;
    const DecLayer& L = lay[step % 3];
    const DecLayer& Ln = lay[(step + 1) % 3];
    const bool more = step + 1 < total_steps;
    const int fmt = fmt_of(L);
    const int par = step & 1;
    const uint32_t ep = (uint32_t)step + 1;  // epoch of the words this step produces
    stamp(a, tok, layer, 0);
    // -------- P1: norm; router + shared rows (tile prefetched during the previous layer)
    {
      const uint16_t* hin = (layer == 0) ? a.inputs + (size_t)tok * DEC_H : a.hbuf + (size_t)par * DEC_H;
      const float bv = (tid < nr1 && L.rbias) ? __ldcg(L.rbias + r1.r0 + tid) : 0.0f;
      if (tid < DEC_H / 8) {
        const uint4 hv = __ldcg(reinterpret_cast<const uint4*>(hin) + tid);
        reinterpret_cast<uint4*>(hs)[tid] = hv;
        if (a.trace_h && b == 0)
          reinterpret_cast<uint4*>(a.trace_h + ((size_t)tok * a.n_layers + layer) * DEC_H)[tid] = hv;
      }
      if (tid < 64) rbias_s[tid] = bv;
    }
    const P1Tile t1 = p1_tile(Abuf, r1);
    stamp(a, tok, layer, 1);
    const bool a_ok = mbar_wait_block(barA, phA, a.err);
    stamp(a, tok, layer, 2);
    float xscale2 = 1.0f;
    if (a_ok) {
      phA ^= 1;
      pendA = false;
      // power-of-two scale of the normed row; the router logits go out first,
      // then the fragments and group sums for P2 are built while the other
      // CTAs' logits arrive (routing's block syncs order them before P2)
      xscale2 = fp16_input_scale(rmsnorm_smem(hs, t1.norm, a.eps, xs, red));
      stamp(a, tok, layer, 3);
      p1_compute(a, r1, t1, xs, rbias_s, gu, par, ep);
      switch (fmt) {
        case 0: p2_frags<2, 64>(xs, xscale2, xf2, xsum2); break;
        case 1: p2_frags<2, 32>(xs, xscale2, xf2, xsum2); break;
        case 2: p2_frags<4, 64>(xs, xscale2, xf2, xsum2); break;
        default: p2_frags<4, 32>(xs, xscale2, xf2, xsum2); break;
      }
    }
    stamp(a, tok, layer, 4);
    if (!a_ok) { drain(); return; }
    stamp(a, tok, layer, 5);
    // -------- P2: route; C / D copies; next layer's P1 tile; gate/up rows
    if (!route_block(a.f_logits + par * DEC_E, ep, a.err, K, a.norm_topk, rv, cand, red, ids, wts, L, ids_ok_s)) {
      drain();
      return;
    }
    if (b == 0 && tid < K) {
      if (a.trace_ids) a.trace_ids[((size_t)tok * a.n_layers + layer) * K + tid] = ids[tid];
      if (a.trace_w) a.trace_w[((size_t)tok * a.n_layers + layer) * K + tid] = wts[tid];
    }
    stamp(a, tok, layer, 6);
    const bool ids_ok = *ids_ok_s != 0;   // block-uniform (set before routing's last sync)
    if (!ids_ok && tid == 0) raise_error(a.err, YN_ERR_BAD_SLOT);
    if (ids_ok) {
      if (warp >= DEC_WARPS - DEC_CW) {  // the last DEC_CW warps issue the C-tile copies
        const int t0 = warp - (DEC_WARPS - DEC_CW);
        switch (fmt) {
          case 0: copy_c<2, 64>(a, L, ids, sg, ntile, C, barT, t0, DEC_CW); break;
          case 1: copy_c<2, 32>(a, L, ids, sg, ntile, C, barT, t0, DEC_CW); break;
          case 2: copy_c<4, 64>(a, L, ids, sg, ntile, C, barT, t0, DEC_CW); break;
          default: copy_c<4, 32>(a, L, ids, sg, ntile, C, barT, t0, DEC_CW); break;
        }
      }
      pendT = true;
    }
    stamp(a, tok, layer, 7);
    if (ids_ok) {
      const float inv = __frcp_rn(xscale2);
      switch (fmt) {
        case 0: p2_tiles<2, 64>(a, ntile, C, xf2, xsum2, inv, part, barT, phT); break;
        case 1: p2_tiles<2, 32>(a, ntile, C, xf2, xsum2, inv, part, barT, phT); break;
        case 2: p2_tiles<4, 64>(a, ntile, C, xf2, xsum2, inv, part, barT, phT); break;
        default: p2_tiles<4, 32>(a, ntile, C, xf2, xsum2, inv, part, barT, phT); break;
      }
      phT ^= 1;
      pendT = false;
    }
    __syncthreads();
    stamp(a, tok, layer, 8);
    if (ids_ok && warp < 2) {  // SwiGLU of this CTA's units
      if (L.rg.bits == 2) p2_swiglu<2>(a, sg, ntile, part, tid);
      else p2_swiglu<4>(a, sg, ntile, part, tid);
    }
    stamp(a, tok, layer, 9);
    grid_arrive(a);
    if (ids_ok) {
      // the D-tile copies for P3 go out while the grid barrier is pending
      for (int j = warp; j <= K; j += DEC_WARPS) {
        switch (fmt) {
          case 0: copy_d<2, 64>(a, L, ids, d0, nd, D, j); break;
          case 1: copy_d<2, 32>(a, L, ids, d0, nd, D, j); break;
          case 2: copy_d<4, 64>(a, L, ids, d0, nd, D, j); break;
          default: copy_d<4, 32>(a, L, ids, d0, nd, D, j); break;
        }
      }
      cp_arrive(barD);
      pendD = true;
    }
    gen += 1;
    if (grid_wait(a, gen * (unsigned)G, eflag)) { drain(); return; }
    stamp(a, tok, layer, 10);
    // -------- P3: next layer's P1 tile (idle warps), activation fragments
    // (staged in the free C tile), down rows, combine
    // descriptor of layer step+2: its copy completes with this P1-tile phase,
    // which step+1 waits for before using anything of step+2
    if (step + 2 < total_steps) load_layer_async(&lay[(step + 2) % 3], a.layers, (step + 2) % a.n_layers);
    if (more) issue_p1(Ln, r1, p1_tile(Abuf, r1), barA, min(K + 1, DEC_WARPS - 4));
    pendA = more;
    uint16_t* stage = reinterpret_cast<uint16_t*>(C);
    switch (fmt) {
      case 0: p3_frags<2, 64>(a, stage, xf3, xsum3, xsc3); break;
      case 1: p3_frags<2, 32>(a, stage, xf3, xsum3, xsc3); break;
      case 2: p3_frags<4, 64>(a, stage, xf3, xsum3, xsc3); break;
      default: p3_frags<4, 32>(a, stage, xf3, xsum3, xsc3); break;
    }
    stamp(a, tok, layer, 11);
    const bool d_ok = ids_ok && mbar_wait_block(barD, phD, a.err);
    stamp(a, tok, layer, 12);
    if (d_ok) {
      phD ^= 1;
      pendD = false;
      switch (fmt) {
        case 0: p3_tiles<2, 64>(a, D, xf3, xsum3, xsc3, part); break;
        case 1: p3_tiles<2, 32>(a, D, xf3, xsum3, xsc3, part); break;
        case 2: p3_tiles<4, 64>(a, D, xf3, xsum3, xsc3, part); break;
        default: p3_tiles<4, 32>(a, D, xf3, xsum3, xsc3, part); break;
      }
    }
    __syncthreads();
    stamp(a, tok, layer, 13);
    if (d_ok) {
      // warp t combines output row d0 + t: lane j < K holds routed column j's
      // weighted term, lane K the gated shared term; sums in column order.
      const int nsbr = (L.rg.bits * DEC_I / 8) / 64;
      const int lane = tid & 31;
      const bool last = layer == a.n_layers - 1;
      for (int t = warp; t < nd; t += DEC_WARPS) {
        float term = 0.0f;
        if (lane < K) {
          float y = 0.0f;
          for (int q = 0; q < nsbr; ++q) y = __fadd_rn(y, part[(lane * 16 + t) * 8 + q]);
          term = bf16r(__fmul_rn(bf16r(y), wts[lane]));
        } else if (lane == K && a.Ish) {
          float y = 0.0f;
#pragma unroll
          for (int q = 0; q < DEC_I / 64; ++q) y = __fadd_rn(y, part[(K * 16 + t) * 8 + q]);
          term = bf16r(__fmul_rn(xsc3[DEC_MAX_K + 2], bf16r(y)));
        }
        float acc = 0.0f;
        for (int j = 0; j < K; ++j) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, term, j));
        const float sh = __shfl_sync(0xffffffffu, term, K);
        if (lane == 0) {
          float o = bf16r(acc);
          if (a.Ish) o = bf16r(__fadd_rn(o, sh));
          o = bf16r(__fadd_rn(bf16_to_f32(hs[d0 + t]), o));
          (last ? a.outputs + (size_t)tok * DEC_H : a.hbuf + (size_t)(par ^ 1) * DEC_H)[d0 + t] = f32_to_bf16(o);
        }
      }
    }
    // the C tile held generic-proxy writes (activation staging): order them
    // before the next layer's bulk copies into it
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    stamp(a, tok, layer, 14);
    stamp(a, tok, layer, 15);
    grid_arrive(a);
    gen += 1;
    if (grid_wait(a, gen * (unsigned)G, eflag)) { drain(); return; }
  }
}
#endif  // YN_NO_STACK_DECODE_KERNEL

}  // namespace ynb
