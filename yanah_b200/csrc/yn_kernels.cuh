// Decode-path kernels for one MoE layer on B200 (sm_100a).
//
//  k_post_attention : RMSNorm + router logits + shared-expert gate/up/SwiGLU +
//                     shared_expert_gate + lookahead routers; the last CTA to
//                     finish runs routing (softmax -> top-k -> renormalise) and
//                     the lookahead softmax. (mlx_backend.py:302-316, 326-348)
//  k_expert_up      : routed gate/up projections + SwiGLU, one tile of n-rows
//                     of one (row, column) task per CTA. (mlx_backend.py:447-456)
//  k_expert_down    : routed and shared down projections; the last CTA to
//                     finish a 256-row block combines sum_j w_j y_j + shared and
//                     the residual in a fixed column order. (mlx_backend.py:
//                     409, 420, 438-440; orchestrator.py:287)
//
// Every CTA stages its whole weight tile into shared memory with bulk copies
// (cp.async.bulk, mbarrier completion) at launch, so a phase keeps all of its
// bytes in flight at once; the compute then reads the tile from shared memory.
// No kernel spins on another CTA: cross-CTA completion uses a counter and the
// last arriving CTA does the follow-up work.
#pragma once
#include "yn_common.cuh"
#include "yn_moe.cuh"
#include "yn_qdot.cuh"

namespace ynb {

constexpr int SMEM_HDR = 256;  // mbarrier, flags, reduction scratch

YN_DEV size_t a16(size_t v) { return (v + 15) & ~size_t(15); }

YN_DEV bool bulk_ok(const void* dst, const void* src, uint32_t bytes) {
  return ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | bytes) & 15u) == 0;
}

// Cooperative byte copy for pieces that cannot use the bulk engine.
YN_DEV void coop_copy(uint8_t* dst, const uint8_t* src, uint32_t bytes) {
  for (uint32_t i = threadIdx.x; i < bytes; i += blockDim.x) dst[i] = src[i];
}

struct Piece {
  uint8_t* dst;
  const uint8_t* src;
  uint32_t bytes;
};

// Issue up to 6 pieces: bulk where possible (thread 0), cooperative otherwise.
// Must be called by all threads. Leaves the mbarrier armed with the bulk bytes.
YN_DEV void stage_pieces(const Piece* pc, int n, uint64_t* bar) {
  if (threadIdx.x == 0) {
    uint32_t tx = 0;
    for (int i = 0; i < n; ++i)
      if (bulk_ok(pc[i].dst, pc[i].src, pc[i].bytes)) tx += pc[i].bytes;
    mbar_arrive_expect_tx(bar, tx);
    for (int i = 0; i < n; ++i)
      if (pc[i].bytes && bulk_ok(pc[i].dst, pc[i].src, pc[i].bytes)) bulk_g2s(pc[i].dst, pc[i].src, pc[i].bytes, bar);
  }
  for (int i = 0; i < n; ++i)
    if (!bulk_ok(pc[i].dst, pc[i].src, pc[i].bytes)) coop_copy(pc[i].dst, pc[i].src, pc[i].bytes);
}

// Shared-memory header: [0] weight barrier, [8] activation barrier,
// [16] last-CTA flag, [32..64) reduction scratch.
YN_DEV void init_bars(uint64_t* bar_w, uint64_t* bar_a) {
  if (threadIdx.x == 0) {
    mbar_init(bar_w, 1);
    mbar_init(bar_a, 1);
    fence_mbar_init();
  }
  __syncthreads();
}

// Block-wide sum with a fixed tree: butterfly inside each warp, then the four
// warp partials summed in warp order. Every thread returns the same value.
YN_DEV float block_sum4(float v, float* red) {
  v = group_sum_bfly(v, 32);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  return __fadd_rn(__fadd_rn(__fadd_rn(red[0], red[1]), red[2]), red[3]);
}
YN_DEV float block_max4(float v, float* red) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  return fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
}

// RMSNorm (canonical order, 128 threads): out = bf16(w * bf16(x * r)),
// r = 1/sqrt(mean(x^2) + eps), sum of squares per thread over i = tid + 128 j.
YN_DEV void rmsnorm_row(const uint16_t* h, const uint16_t* w, int H, float eps, uint16_t* out_smem,
                        uint16_t* out_global, float* red) {  // h, w in shared memory
  float ss = 0.0f;
  for (int i = threadIdx.x; i < H; i += THREADS) {
    const float v = bf16_to_f32(h[i]);
    ss = __fmaf_rn(v, v, ss);
  }
  const float tot = block_sum4(ss, red);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)H), eps)));
  for (int i = threadIdx.x; i < H; i += THREADS) {
    const float v = bf16_to_f32(h[i]);
    const uint16_t o = f32_to_bf16(__fmul_rn(bf16_to_f32(w[i]), bf16r(__fmul_rn(v, r))));
    out_smem[i] = o;
    if (out_global) out_global[i] = o;
  }
}

// ------------------------------------------------------------- routing
// One warp routes one row of E logits (E <= 1024): softmax in fp32 with the
// deterministic exp, probabilities rounded to bf16, top-k by (prob desc, id
// asc), weights renormalised as bf16(p / bf16(sum p)) when norm != 0.
YN_DEV void route_row(const float* logits, int E, int K, int norm, int32_t* ids_out, float* w_out) {
  const int lane = threadIdx.x & 31;
  const int nv = (E + 31) >> 5;
  float v[32];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int e = lane + 32 * i;
    v[i] = (i < nv && e < E) ? __ldcg(logits + e) : -INFINITY;
    m = fmaxf(m, v[i]);
  }
  m = warp_max(m);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int e = lane + 32 * i;
    const float p = (i < nv && e < E) ? yn_expf(__fsub_rn(v[i], m)) : 0.0f;
    v[i] = p;
    s = __fadd_rn(s, p);
  }
  s = group_sum_bfly(s, 32);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int e = lane + 32 * i;
    v[i] = (i < nv && e < E) ? bf16r(__fdiv_rn(v[i], s)) : -1.0f;
  }
  float wsum = 0.0f, mine = 0.0f;
  int mine_id = 0;
  for (int j = 0; j < K; ++j) {
    float bp = -2.0f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int e = lane + 32 * i;
      if (v[i] > bp) {
        bp = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int mk = 16; mk > 0; mk >>= 1) {
      const float op = __shfl_xor_sync(0xffffffffu, bp, mk);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, mk);
      if (op > bp || (op == bp && oi < bi)) {
        bp = op;
        bi = oi;
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (lane + 32 * i == bi) v[i] = -2.0f;
    wsum = __fadd_rn(wsum, bp);
    if (lane == j) {
      mine = bp;
      mine_id = bi;
    }
  }
  const float sb = bf16r(wsum);
  if (lane < K) {
    ids_out[lane] = mine_id;
    w_out[lane] = norm ? bf16r(__fdiv_rn(mine, sb)) : mine;
  }
}

// fp32 softmax of one row (lookahead forecast), folded into a running max.
YN_DEV void softmax_max_row(const float* logits, int E, float* run_max, bool first) {
  const int lane = threadIdx.x & 31;
  const int nv = (E + 31) >> 5;
  float v[32];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int e = lane + 32 * i;
    v[i] = (i < nv && e < E) ? __ldcg(logits + e) : -INFINITY;
    m = fmaxf(m, v[i]);
  }
  m = warp_max(m);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int e = lane + 32 * i;
    const float p = (i < nv && e < E) ? yn_expf(__fsub_rn(v[i], m)) : 0.0f;
    v[i] = p;
    s = __fadd_rn(s, p);
  }
  s = group_sum_bfly(s, 32);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int e = lane + 32 * i;
    if (i < nv && e < E) {
      const float p = __fdiv_rn(v[i], s);
      run_max[e] = first ? p : fmaxf(run_max[e], p);
    }
  }
}

__global__ void k_route(const float* logits, int T, int E, int K, int norm, int32_t* ids, float* w) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= T) return;
  route_row(logits + (size_t)row * E, E, K, norm, ids + (size_t)row * K, w + (size_t)row * K);
}

// ------------------------------------------------------- post attention
template <int CPL>
__global__ void __launch_bounds__(THREADS) k_post_attention(const PostAttnArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  uint64_t* bar_a = reinterpret_cast<uint64_t*>(smem + 8);
  int* flag = reinterpret_cast<int*>(smem + 16);
  float* red = reinterpret_cast<float*>(smem + 32);
  uint16_t* hs = reinterpret_cast<uint16_t*>(smem + SMEM_HDR);                 // (T, H) h1 rows
  uint16_t* ns = hs + a16((size_t)a.T * a.H * 2) / 2;                           // (H) norm weight
  uint16_t* xs = ns + a16((size_t)a.H * 2) / 2;                                 // (T, H) normed rows
  uint8_t* tile = reinterpret_cast<uint8_t*>(xs) + a16((size_t)a.T * a.H * 2);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int t = blockIdx.x;
  int kind, tgt = 0, row0, nrows;
  const uint16_t* normw = a.norm;
  QM m0 = a.router, m1 = a.router;
  if (t < a.nt_router) {
    kind = 0; row0 = t * a.r_router; nrows = a.r_router; m0 = a.router;
  } else if ((t -= a.nt_router) < a.nt_shared) {
    kind = 1; row0 = t * a.r_shared; nrows = a.r_shared; m0 = a.sh_gate; m1 = a.sh_up;
  } else if ((t -= a.nt_shared) < a.nt_sg) {
    kind = 2; row0 = 0; nrows = 1; m0 = a.sg;
  } else {
    t -= a.nt_sg;
    kind = 3; tgt = t / a.nt_target; row0 = (t % a.nt_target) * a.r_target; nrows = a.r_target;
    m0 = a.trouter[tgt]; normw = a.tnorm[tgt];
  }
  const int H = a.H;
  const uint32_t rb = (uint32_t)H;              // 8-bit rows: one byte per code
  const uint32_t ng = (uint32_t)(H / m0.gs);
  const uint32_t sb = ng * 2u;
  const int nparts = (kind == 1) ? 2 : 1;
  uint8_t* pc_codes[2];
  uint16_t* pc_s[2];
  uint16_t* pc_b[2];
  {
    size_t o = 0;
    for (int p = 0; p < nparts; ++p) {
      pc_codes[p] = tile + o; o += a16((size_t)nrows * rb);
      pc_s[p] = reinterpret_cast<uint16_t*>(tile + o); o += a16((size_t)nrows * sb);
      pc_b[p] = reinterpret_cast<uint16_t*>(tile + o); o += a16((size_t)nrows * sb);
    }
  }
  init_bars(bar, bar_a);
  {
    Piece act[2] = {{reinterpret_cast<uint8_t*>(hs), reinterpret_cast<const uint8_t*>(a.h1), (uint32_t)(a.T * H * 2)},
                    {reinterpret_cast<uint8_t*>(ns), reinterpret_cast<const uint8_t*>(normw), (uint32_t)(H * 2)}};
    stage_pieces(act, 2, bar_a);
    Piece pc[6];
    int n = 0;
    for (int p = 0; p < nparts; ++p) {
      const QM& m = (p == 0) ? m0 : m1;
      pc[n++] = {pc_codes[p], m.w + (size_t)row0 * rb, (uint32_t)(nrows * rb)};
      pc[n++] = {reinterpret_cast<uint8_t*>(pc_s[p]), reinterpret_cast<const uint8_t*>(m.s + (size_t)row0 * ng),
                 (uint32_t)(nrows * sb)};
      pc[n++] = {reinterpret_cast<uint8_t*>(pc_b[p]), reinterpret_cast<const uint8_t*>(m.b + (size_t)row0 * ng),
                 (uint32_t)(nrows * sb)};
    }
    stage_pieces(pc, n, bar);
  }
  // RMSNorm of every row while the weights are in flight.
  __syncthreads();
  const bool act_ok = mbar_wait_block(bar_a, 0, a.err);
  if (act_ok)
    for (int tt = 0; tt < a.T; ++tt)
      rmsnorm_row(hs + (size_t)tt * H, ns, H, a.eps, xs + (size_t)tt * H,
                  (blockIdx.x == 0) ? a.x + (size_t)tt * H : nullptr, red);
  __syncthreads();
  const bool ok = mbar_wait_block(bar, 0, a.err) && act_ok;

  if (ok) {
    const int lpr = lanes_per_row((int)rb), rpi = 32 / lpr, l = lane % lpr, u = lane / lpr;
    for (int tt = 0; tt < a.T; ++tt) {
      XF32<8, CPL, 1> X;
      load_x_f32<8, CPL, 1>(X, xs + (size_t)tt * H, l, lpr);
      for (int rbase = warp * rpi; rbase < nrows; rbase += 4 * rpi) {
        const int r = rbase + u;
        const int rr = (r < nrows) ? r : 0;
        float v0 = row_dot_f32<8, CPL, 1>(pc_codes[0] + (size_t)rr * rb, pc_s[0] + (size_t)rr * ng,
                                          pc_b[0] + (size_t)rr * ng, X, l, lpr, m0.gs);
        v0 = group_sum_bfly(v0, lpr);
        float v1 = 0.0f;
        if (kind == 1) {
          v1 = row_dot_f32<8, CPL, 1>(pc_codes[1] + (size_t)rr * rb, pc_s[1] + (size_t)rr * ng,
                                      pc_b[1] + (size_t)rr * ng, X, l, lpr, m1.gs);
          v1 = group_sum_bfly(v1, lpr);
        }
        if (l == 0 && r < nrows) {
          const int row = row0 + r;
          if (kind == 0) {
            const float bias = a.rbias ? a.rbias[row] : 0.0f;
            a.logits[(size_t)tt * a.E + row] = bf16r(__fadd_rn(v0, bias));
          } else if (kind == 1) {
            a.act_sh[(size_t)tt * a.Ish + row] = f32_to_bf16(swiglu_bf16(bf16r(v0), bf16r(v1)));
          } else if (kind == 2) {
            a.sgate[tt] = bf16r(sigmoid_f32(bf16r(v0)));
          } else {
            const float bias = a.tbias[tgt] ? a.tbias[tgt][row] : 0.0f;
            a.flogits[((size_t)tgt * a.T + tt) * a.E + row] = bf16r(__fadd_rn(v0, bias));
          }
        }
      }
    }
  }

  // Last CTA to finish: routing for every row and the lookahead softmax.
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const int prev = atomicAdd(a.counter, 1);
    *flag = (prev == a.n_tiles - 1);
  }
  __syncthreads();
  if (*flag) {
    __threadfence();
    for (int tt = warp; tt < a.T; tt += 4)
      route_row(a.logits + (size_t)tt * a.E, a.E, a.K, a.norm_topk, a.ids + (size_t)tt * a.K,
                a.wts + (size_t)tt * a.K);
    for (int g = warp; g < a.n_targets; g += 4)
      for (int tt = 0; tt < a.T; ++tt)
        softmax_max_row(a.flogits + ((size_t)g * a.T + tt) * a.E, a.E, a.fprobs + (size_t)g * a.E, tt == 0);
    __syncthreads();
    if (tid == 0) *a.counter = 0;
  }
}

// ---------------------------------------------------------- expert up
YN_DEV bool expert_record(const int32_t* ids, int idx, const int32_t* slot_of, int E, int n_slots,
                          const uint8_t* base, long long stride, int* err, const uint8_t** rec) {
  const int e = ids[idx];
  if (e < 0 || e >= E) {
    raise_error(err, YN_ERR_BAD_EXPERT);
    return false;
  }
  const int s = slot_of ? slot_of[e] : e;
  if (s < 0 || s >= n_slots) {
    raise_error(err, YN_ERR_BAD_SLOT);
    return false;
  }
  *rec = base + (size_t)s * (size_t)stride;
  return true;
}

template <int BITS, int CPL, int NSEG>
__global__ void __launch_bounds__(THREADS) k_expert_up(const ExpertUpArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  uint64_t* bar_a = reinterpret_cast<uint64_t*>(smem + 8);
  float* red = reinterpret_cast<float*>(smem + 32);
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem + SMEM_HDR);
  uint8_t* tile = smem + SMEM_HDR + a16((size_t)a.H * 2);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int task = blockIdx.x / a.tiles_per_task;
  const int n0 = (blockIdx.x % a.tiles_per_task) * a.rows;
  const int tt = task / a.ncols;
  const int j = a.cols[task % a.ncols];
  const uint8_t* rec;
  if (!expert_record(a.ids, tt * a.K + j, a.slot_of, a.E, a.n_slots, a.base, a.stride, a.err, &rec)) return;

  const int H = a.H, R = a.rows;
  const uint32_t rb = (uint32_t)(H * BITS / 8);
  const uint32_t ng = (uint32_t)(H / a.rg.gs);
  const uint32_t sb = ng * 2u;
  uint8_t* gc = tile;
  uint16_t* gsc = reinterpret_cast<uint16_t*>(gc + a16((size_t)R * rb));
  uint16_t* gbi = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(gsc) + a16((size_t)R * sb));
  uint8_t* uc = reinterpret_cast<uint8_t*>(gbi) + a16((size_t)R * sb);
  uint16_t* usc = reinterpret_cast<uint16_t*>(uc + a16((size_t)R * rb));
  uint16_t* ubi = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(usc) + a16((size_t)R * sb));

  init_bars(bar, bar_a);
  {
    Piece act[1] = {{reinterpret_cast<uint8_t*>(xs), reinterpret_cast<const uint8_t*>(a.x + (size_t)tt * H),
                     (uint32_t)(H * 2)}};
    stage_pieces(act, 1, bar_a);
    Piece pc[6] = {
        {gc, rec + a.rg.off[0] + (size_t)n0 * rb, (uint32_t)(R * rb)},
        {reinterpret_cast<uint8_t*>(gsc), rec + a.rg.off[1] + (size_t)n0 * sb, (uint32_t)(R * sb)},
        {reinterpret_cast<uint8_t*>(gbi), rec + a.rg.off[2] + (size_t)n0 * sb, (uint32_t)(R * sb)},
        {uc, rec + a.rg.off[3] + (size_t)n0 * rb, (uint32_t)(R * rb)},
        {reinterpret_cast<uint8_t*>(usc), rec + a.rg.off[4] + (size_t)n0 * sb, (uint32_t)(R * sb)},
        {reinterpret_cast<uint8_t*>(ubi), rec + a.rg.off[5] + (size_t)n0 * sb, (uint32_t)(R * sb)},
    };
    stage_pieces(pc, 6, bar);
  }
  // max |x| of the staged row (power-of-two scale for the fp16 path).
  __syncthreads();
  if (!mbar_wait_block(bar_a, 0, a.err)) return;
  float mx = 0.0f;
  for (int i = tid; i < H; i += THREADS) mx = fmaxf(mx, fabsf(bf16_to_f32(xs[i])));
  mx = block_max4(mx, red);
  const float scale = fp16_input_scale(mx);
  const float inv_scale = __fdiv_rn(1.0f, scale);
  __syncthreads();
  if (!mbar_wait_block(bar, 0, a.err)) return;

  const int lpr = lanes_per_row((int)rb), rpi = 32 / lpr, l = lane % lpr, u = lane / lpr;
  XF16<BITS, CPL, NSEG> X;
  load_x_f16<BITS, CPL, NSEG>(X, xs, scale, l, lpr);
  uint16_t* act = a.act + ((size_t)tt * a.K + j) * a.I + n0;
  for (int rbase = warp * rpi; rbase < R; rbase += 4 * rpi) {
    const int r = rbase + u;
    const int rr = (r < R) ? r : 0;
    float g = row_dot_f16<BITS, CPL, NSEG>(gc + (size_t)rr * rb, gsc + (size_t)rr * ng, gbi + (size_t)rr * ng, X,
                                           inv_scale, l, lpr, a.rg.gs);
    float up = row_dot_f16<BITS, CPL, NSEG>(uc + (size_t)rr * rb, usc + (size_t)rr * ng, ubi + (size_t)rr * ng, X,
                                            inv_scale, l, lpr, a.rg.gs);
    g = group_sum_bfly(g, lpr);
    up = group_sum_bfly(up, lpr);
    if (l == 0 && r < R) act[r] = f32_to_bf16(swiglu_bf16(bf16r(g), bf16r(up)));
  }
}

// -------------------------------------------------------- expert down
template <int BITS, int CPL, int NSEG, int CPLS>
__global__ void __launch_bounds__(THREADS) k_expert_down(const ExpertDownArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  uint64_t* bar_a = reinterpret_cast<uint64_t*>(smem + 8);
  int* flag = reinterpret_cast<int*>(smem + 16);
  float* red = reinterpret_cast<float*>(smem + 32);
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem + SMEM_HDR);
  const int Kx = (a.I > a.Ish) ? a.I : a.Ish;
  uint8_t* tile = smem + SMEM_HDR + a16((size_t)Kx * 2);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = a.H;
  const bool routed = (int)blockIdx.x < a.n_routed_tiles;
  int tt, j = 0, r0, R;
  const uint8_t* wsrc;
  const uint8_t* ssrc;
  const uint8_t* bsrc;
  uint32_t rb, ng, gs;
  const uint16_t* xg;
  int Kin;
  if (routed) {
    const int task = blockIdx.x / a.tiles_routed_per_task;
    tt = task / a.K;
    j = task % a.K;
    R = a.rows_routed;
    r0 = (blockIdx.x % a.tiles_routed_per_task) * R;
    const uint8_t* rec;
    if (!expert_record(a.ids, tt * a.K + j, a.slot_of, a.E, a.n_slots, a.base, a.stride, a.err, &rec)) {
      rec = nullptr;
    }
    Kin = a.I;
    rb = (uint32_t)(a.I * BITS / 8);
    gs = (uint32_t)a.rg.gs;
    ng = (uint32_t)(a.I / a.rg.gs);
    wsrc = rec ? rec + a.rg.off[6] + (size_t)r0 * rb : nullptr;
    ssrc = rec ? rec + a.rg.off[7] + (size_t)r0 * ng * 2 : nullptr;
    bsrc = rec ? rec + a.rg.off[8] + (size_t)r0 * ng * 2 : nullptr;
    xg = a.act + ((size_t)tt * a.K + j) * a.I;
  } else {
    const int s = blockIdx.x - a.n_routed_tiles;
    tt = s / a.tiles_shared_per_token;
    R = a.rows_shared;
    r0 = (s % a.tiles_shared_per_token) * R;
    Kin = a.Ish;
    rb = (uint32_t)a.Ish;  // 8-bit
    gs = (uint32_t)a.sh_down.gs;
    ng = (uint32_t)(a.Ish / a.sh_down.gs);
    wsrc = a.sh_down.w + (size_t)r0 * rb;
    ssrc = reinterpret_cast<const uint8_t*>(a.sh_down.s + (size_t)r0 * ng);
    bsrc = reinterpret_cast<const uint8_t*>(a.sh_down.b + (size_t)r0 * ng);
    xg = a.act_sh + (size_t)tt * a.Ish;
  }
  const uint32_t sb = ng * 2u;
  uint8_t* wc = tile;
  uint16_t* wsc = reinterpret_cast<uint16_t*>(wc + a16((size_t)R * rb));
  uint16_t* wbi = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(wsc) + a16((size_t)R * sb));

  init_bars(bar, bar_a);
  const bool have = (wsrc != nullptr);
  {
    Piece act[1] = {{reinterpret_cast<uint8_t*>(xs), reinterpret_cast<const uint8_t*>(xg), (uint32_t)(Kin * 2)}};
    stage_pieces(act, 1, bar_a);
  }
  if (have) {
    Piece pc[3] = {{wc, wsrc, R * rb}, {reinterpret_cast<uint8_t*>(wsc), ssrc, R * sb},
                   {reinterpret_cast<uint8_t*>(wbi), bsrc, R * sb}};
    stage_pieces(pc, 3, bar);
  }
  __syncthreads();
  const bool act_ok = mbar_wait_block(bar_a, 0, a.err);
  float mx = 0.0f;
  if (act_ok)
    for (int i = tid; i < Kin; i += THREADS) mx = fmaxf(mx, fabsf(bf16_to_f32(xs[i])));
  mx = block_max4(mx, red);
  __syncthreads();
  const bool wok = have ? mbar_wait_block(bar, 0, a.err) : false;
  const bool ok = have && act_ok && wok;

  if (ok) {
    const int lpr = lanes_per_row((int)rb), rpi = 32 / lpr, l = lane % lpr, u = lane / lpr;
    if (routed) {
      const float scale = fp16_input_scale(mx);
      const float inv_scale = __fdiv_rn(1.0f, scale);
      XF16<BITS, CPL, NSEG> X;
      load_x_f16<BITS, CPL, NSEG>(X, xs, scale, l, lpr);
      uint16_t* yo = a.y + ((size_t)tt * a.K + j) * H + r0;
      for (int rbase = warp * rpi; rbase < R; rbase += 4 * rpi) {
        const int r = rbase + u;
        const int rr = (r < R) ? r : 0;
        float v = row_dot_f16<BITS, CPL, NSEG>(wc + (size_t)rr * rb, wsc + (size_t)rr * ng, wbi + (size_t)rr * ng,
                                               X, inv_scale, l, lpr, (int)gs);
        v = group_sum_bfly(v, lpr);
        if (l == 0 && r < R) yo[r] = f32_to_bf16(v);
      }
    } else {
      XF32<8, CPLS, 1> X;
      load_x_f32<8, CPLS, 1>(X, xs, l, lpr);
      const float sg = a.sgate[tt];
      uint16_t* yo = a.ysh + (size_t)tt * H + r0;
      for (int rbase = warp * rpi; rbase < R; rbase += 4 * rpi) {
        const int r = rbase + u;
        const int rr = (r < R) ? r : 0;
        float v = row_dot_f32<8, CPLS, 1>(wc + (size_t)rr * rb, wsc + (size_t)rr * ng, wbi + (size_t)rr * ng, X, l,
                                          lpr, (int)gs);
        v = group_sum_bfly(v, lpr);
        if (l == 0 && r < R) yo[r] = f32_to_bf16(__fmul_rn(sg, bf16r(v)));
      }
    }
  }

  // Completion count per (row, 256-row block); the last arrival combines.
  const int cbr = (H < CB_ROWS) ? H : CB_ROWS;
  const int cb = r0 / cbr;
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const int expect = a.K * (cbr / a.rows_routed) + (a.has_shared ? cbr / a.rows_shared : 0);
    const int prev = atomicAdd(&a.counters[tt * a.n_cb + cb], 1);
    *flag = (prev == expect - 1);
  }
  __syncthreads();
  if (*flag) {
    __threadfence();
    const float* wrow = a.wts + (size_t)tt * a.K;
    float wv[16];
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) wv[jj] = (jj < a.K) ? __ldcg(wrow + jj) : 0.0f;
    for (int r = cb * cbr + tid; r < (cb + 1) * cbr; r += THREADS) {
      uint16_t yv[16];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) yv[jj] = (jj < a.K) ? __ldcg(a.y + ((size_t)tt * a.K + jj) * H + r) : 0;
      const uint16_t sh = (a.mode >= 1 && a.has_shared) ? __ldcg(a.ysh + (size_t)tt * H + r) : 0;
      const uint16_t hr = (a.mode == 2) ? a.h_res[(size_t)tt * H + r] : 0;
      float acc = 0.0f;
#pragma unroll
      for (int jj = 0; jj < 16; ++jj)
        if (jj < a.K) acc = __fadd_rn(acc, bf16r(__fmul_rn(bf16_to_f32(yv[jj]), wv[jj])));
      float o = bf16r(acc);
      if (a.mode >= 1 && a.has_shared) o = bf16r(__fadd_rn(o, bf16_to_f32(sh)));
      if (a.mode == 2) o = bf16r(__fadd_rn(bf16_to_f32(hr), o));
      a.out[(size_t)tt * H + r] = f32_to_bf16(o);
    }
    __syncthreads();
    if (tid == 0) a.counters[tt * a.n_cb + cb] = 0;
  }
}

// ---------------------------------------------------------- standalone
// fp32 dequantisation: out[r][k] = fma(scale, q, bias).
template <int BITS>
__global__ void k_dequant(const uint32_t* w, const uint16_t* s, const uint16_t* b, int rows, int cols, int gs,
                          float* out) {
  const size_t n = (size_t)rows * cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), k = (int)(i % cols);
    constexpr int CPW = 32 / BITS;
    const uint32_t word = w[(size_t)r * (cols / CPW) + k / CPW];
    const uint32_t q = (word >> (BITS * (k % CPW))) & ((1u << BITS) - 1u);
    const int g = k / gs;
    const size_t gi = (size_t)r * (cols / gs) + g;
    out[i] = __fmaf_rn(f16_to_f32(s[gi]), (float)q, f16_to_f32(b[gi]));
  }
}

// Canonical fp32-path linear over T rows for 8-bit matrices; x from global.
template <int CPL>
__global__ void __launch_bounds__(THREADS) k_qlinear8(QM m, const uint16_t* x, int T, float* y) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem);
  const int H = m.cols;
  for (int i = threadIdx.x; i < T * H; i += THREADS) xs[i] = x[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rb = H, ng = H / m.gs;
  const int lpr = lanes_per_row(rb), rpi = 32 / lpr, l = lane % lpr, u = lane / lpr;
  const int rows_per_cta = 4 * rpi;
  const int rbase = blockIdx.x * rows_per_cta + warp * rpi;
  const int r = rbase + u;
  const int rr = (r < m.rows) ? r : 0;
  for (int tt = 0; tt < T; ++tt) {
    XF32<8, CPL, 1> X;
    load_x_f32<8, CPL, 1>(X, xs + (size_t)tt * H, l, lpr);
    float v = row_dot_f32<8, CPL, 1>(m.w + (size_t)rr * rb, m.s + (size_t)rr * ng, m.b + (size_t)rr * ng, X, l, lpr,
                                     m.gs);
    v = group_sum_bfly(v, lpr);
    if (l == 0 && r < m.rows) y[(size_t)tt * m.rows + r] = bf16r(v);
  }
}

}  // namespace ynb
