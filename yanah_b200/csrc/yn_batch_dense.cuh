// Post-attention of a batch of up to 64 rows: RMSNorm, router logits,
// shared-expert gate/up + SwiGLU and the shared-expert gate, then routing of
// each group of 8 rows by the group's last CTA (mlx_backend.py:302-316 for T
// rows). The arithmetic of every
// (row, token) dot product is the canonical fp32 order of k_post_attention
// (the same lane mapping and reduction tree), so logits, ids and weights are
// bit-identical to the single-row path; only the work split differs: a CTA
// takes 8 router rows (or 8 shared units, or the gate row) for a group of at
// most 8 tokens, so a batch spreads over hundreds of CTAs.
#pragma once
#include "yn_kernels.cuh"

namespace ynb {

constexpr int BD_ROWS = 8;   // router rows / shared units per CTA
constexpr int BD_TOK = 8;    // tokens per CTA

struct BatchDenseArgs {
  int T, H, E, K, Ish, norm_topk;
  float eps;
  const uint16_t* h;        // (T, H) input rows
  const uint16_t* norm;     // (H)
  QM router;
  const float* rbias;
  QM sh_gate, sh_up, sg;
  int has_shared;
  int nt_router, nt_shared, nt_sg;
  uint16_t* x;              // (T, H) normalised rows
  float* logits;            // (T, E)
  uint16_t* act_sh;         // (T, Ish)
  float* sgate;             // (T)
  int32_t* ids;             // (T, K)
  float* wts;               // (T, K)
  unsigned* counter;        // (8) CTA arrivals per token group (monotonic; the last one routes)
  int* err;
};

template <int CPL>
__global__ void __launch_bounds__(THREADS) k_batch_dense(const BatchDenseArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  uint64_t* bar_a = reinterpret_cast<uint64_t*>(smem + 8);
  int* flag = reinterpret_cast<int*>(smem + 16);
  float* red = reinterpret_cast<float*>(smem + 32);
  const int H = a.H;
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem + SMEM_HDR);               // (BD_TOK, H) rows, normalised in place
  uint16_t* ns = xs + (size_t)BD_TOK * H;                                    // (H) norm weight
  uint8_t* tile = reinterpret_cast<uint8_t*>(ns + H);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t0 = blockIdx.y * BD_TOK, nt = min(BD_TOK, a.T - t0);
  int t = blockIdx.x, kind, row0, nrows;
  QM m0 = a.router, m1 = a.router;
  if (t < a.nt_router) {
    kind = 0; row0 = t * BD_ROWS; nrows = BD_ROWS; m0 = a.router;
  } else if ((t -= a.nt_router) < a.nt_shared) {
    kind = 1; row0 = t * BD_ROWS; nrows = BD_ROWS; m0 = a.sh_gate; m1 = a.sh_up;
  } else {
    kind = 2; row0 = 0; nrows = 1; m0 = a.sg;
  }
  const uint32_t rb = (uint32_t)H, ng = (uint32_t)(H / m0.gs), sb = ng * 2u;
  const int nparts = kind == 1 ? 2 : 1;
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
    Piece act[2] = {{reinterpret_cast<uint8_t*>(xs), reinterpret_cast<const uint8_t*>(a.h + (size_t)t0 * H),
                     (uint32_t)(nt * H * 2)},
                    {reinterpret_cast<uint8_t*>(ns), reinterpret_cast<const uint8_t*>(a.norm), (uint32_t)(H * 2)}};
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
  __syncthreads();
  const bool act_ok = mbar_wait_block(bar_a, 0, a.err);
  if (act_ok)
    for (int tt = 0; tt < nt; ++tt)
      rmsnorm_row(xs + (size_t)tt * H, ns, H, a.eps, xs + (size_t)tt * H,
                  (blockIdx.x == 0) ? a.x + (size_t)(t0 + tt) * H : nullptr, red);
  __syncthreads();
  const bool ok = mbar_wait_block(bar, 0, a.err) && act_ok;
  if (ok) {
    const int lpr = lanes_per_row((int)rb), rpi = 32 / lpr, l = lane % lpr, u = lane / lpr;
    for (int tt = 0; tt < nt; ++tt) {
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
          const int row = row0 + r, tg = t0 + tt;
          if (kind == 0) {
            const float bias = a.rbias ? a.rbias[row] : 0.0f;
            a.logits[(size_t)tg * a.E + row] = bf16r(__fadd_rn(v0, bias));
          } else if (kind == 1) {
            a.act_sh[(size_t)tg * a.Ish + row] = f32_to_bf16(swiglu_bf16(bf16r(v0), bf16r(v1)));
          } else {
            a.sgate[tg] = bf16r(sigmoid_f32(bf16r(v0)));
          }
        }
      }
    }
  }
  // the last CTA of each token group routes that group's rows
  __syncthreads();
  const unsigned n_cta = gridDim.x;
  if (tid == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(a.counter + blockIdx.y, 1u);
    *flag = ((prev + 1u) % n_cta) == 0u;
  }
  __syncthreads();
  if (*flag) {
    __threadfence();
    for (int tt = t0 + warp; tt < t0 + nt; tt += 4)
      route_row(a.logits + (size_t)tt * a.E, a.E, a.K, a.norm_topk, a.ids + (size_t)tt * a.K,
                a.wts + (size_t)tt * a.K);
  }
}

}  // namespace ynb
