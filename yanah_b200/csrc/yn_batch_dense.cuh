// Post-attention of a batch of up to 64 rows: RMSNorm, router logits,
// shared-expert gate/up + SwiGLU and the shared-expert gate, then routing of
// each group of 8 rows by the group's last CTA (mlx_backend.py:302-316 for T
// rows). The arithmetic of every
// (row, token) dot product is the canonical fp32 order of k_post_attention
// (the same lane mapping and reduction tree), so logits, ids and weights are
// bit-identical to the single-row path; only the work split differs: a CTA
// takes 16 router rows (or 8 shared units, or the gate row) for a group of at
// most 8 tokens, so a batch spreads over hundreds of CTAs.
#pragma once
#include "yn_kernels.cuh"

namespace ynb {

constexpr int BD_THREADS = 256;
constexpr int BD_RROWS = 16;  // router rows per CTA (two per warp)
constexpr int BD_SUNITS = 8;  // shared-expert units per CTA (gate and up row: one unit per warp)
constexpr int BD_TOK = 8;     // tokens per CTA

struct BatchDenseArgs {
  int T, H, E, K, Ish, norm_topk;
  float eps;
  const float4* xf;         // (T, H / 4) normalised rows, fp32 lane-interleaved (k_rmsnorm_rows)
  const float* xsum;        // (T, H / 16) chunk sums
  QM router;
  const float* rbias;
  QM sh_gate, sh_up, sg;
  int has_shared;
  int nt_router, nt_shared, nt_sg;
  float* logits;            // (T, E)
  uint16_t* act_sh;         // (T, Ish)
  float* sgate;             // (T)
  int32_t* ids;             // (T, K)
  float* wts;               // (T, K)
  unsigned* counter;        // (8) CTA arrivals per token group (monotonic; the last one routes)
  int* err;
};

// RMSNorm of T rows (one 128-thread CTA per row, the canonical order of
// rmsnorm_row): x = bf16(w * bf16(h * r)).
// The normalised row is also written in the dot kernel's fp32 layout:
// element 16 ci + 4 v + e (ci = l + 32 c) at float4 (c * 4 + v) * 32 + l,
// component e, plus the sum of each 16-element chunk in ascending order (the
// order of load_x_f32).
__global__ void __launch_bounds__(THREADS) k_rmsnorm_rows(const uint16_t* h, const uint16_t* norm, int H, float eps,
                                                          uint16_t* x, float4* xf, float* xsum) {
  extern __shared__ __align__(16) uint16_t rs[];
  __shared__ float red[32];
  uint16_t* hs = rs;
  uint16_t* ws = rs + H;
  const uint4* hg = reinterpret_cast<const uint4*>(h + (size_t)blockIdx.x * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) {
    reinterpret_cast<uint4*>(hs)[i] = hg[i];
    reinterpret_cast<uint4*>(ws)[i] = reinterpret_cast<const uint4*>(norm)[i];
  }
  __syncthreads();
  rmsnorm_row(hs, ws, H, eps, hs, x + (size_t)blockIdx.x * H, red);
  __syncthreads();
  float4* xr = xf + (size_t)blockIdx.x * (H / 4);
  for (int ci = threadIdx.x; ci < H / 16; ci += blockDim.x) {
    const int c = ci >> 5, l = ci & 31;
    float sum = 0.0f;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      float4 f;
      f.x = bf16_to_f32(hs[16 * ci + 4 * v]);
      f.y = bf16_to_f32(hs[16 * ci + 4 * v + 1]);
      f.z = bf16_to_f32(hs[16 * ci + 4 * v + 2]);
      f.w = bf16_to_f32(hs[16 * ci + 4 * v + 3]);
      sum = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sum, f.x), f.y), f.z), f.w);
      xr[(c * 4 + v) * 32 + l] = f;
    }
    xsum[(size_t)blockIdx.x * (H / 16) + ci] = sum;
  }
}

// Canonical 8-bit dot products of two rows (codes / scales / biases in
// shared memory) with the nt token rows of the CTA: lane l owns 16-code
// chunks ci = l + 32 c (c < CPL); per chunk d = fma chain over the 16 codes in
// order, acc = fma(s, d, acc), acc = fma(b, sum(x over the chunk), acc); then
// a butterfly over the 32 lanes -- the exact arithmetic of row_dot_f32 for
// every (row, token). The codes of a chunk are turned into floats once for
// all tokens. X: per token, float4 v of lane l's chunk c at
// ((c * 4 + v) * 32 + l); XS: per token, the chunk sums by chunk index.
template <int CPL>
YN_DEV void dense_rows2(const uint8_t* ca, const uint16_t* sa, const uint16_t* ba, const uint8_t* cb,
                        const uint16_t* sb, const uint16_t* bb, const float4* X, const float* XS, int H, int nt,
                        int gs, float (&oa)[BD_TOK], float (&ob)[BD_TOK]) {
  const int l = threadIdx.x & 31;
  float acca[BD_TOK], accb[BD_TOK];
#pragma unroll
  for (int t = 0; t < BD_TOK; ++t) acca[t] = accb[t] = 0.0f;
  // the chunk loop stays rolled: a batch launch is short and starts with a cold instruction cache, and the
  // unrolled body (tokens x rows x 16 FMAs per chunk) is large
#pragma unroll 1
  for (int c = 0; c < CPL; ++c) {
    const int ci = l + 32 * c;
    const uint4 wa = *reinterpret_cast<const uint4*>(ca + 16 * ci);
    const uint4 wb = *reinterpret_cast<const uint4*>(cb + 16 * ci);
    const uint32_t wva[4] = {wa.x, wa.y, wa.z, wa.w}, wvb[4] = {wb.x, wb.y, wb.z, wb.w};
    float qa[16], qb[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      qa[k] = __fsub_rn(__uint_as_float(__byte_perm(wva[k >> 2], 0x4B000000u, 0x7540u + (unsigned)(k & 3))),
                        8388608.0f);
      qb[k] = __fsub_rn(__uint_as_float(__byte_perm(wvb[k >> 2], 0x4B000000u, 0x7540u + (unsigned)(k & 3))),
                        8388608.0f);
    }
    const int g = ci * 16 / gs;
    const float s_a = f16_to_f32(sa[g]), b_a = f16_to_f32(ba[g]);
    const float s_b = f16_to_f32(sb[g]), b_b = f16_to_f32(bb[g]);
#pragma unroll
    for (int t = 0; t < BD_TOK; ++t) {
      if (t < nt) {
        const float4* xt = X + (size_t)t * (H / 4);
        float xv[16];
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const float4 f = xt[(c * 4 + v) * 32 + l];
          xv[4 * v] = f.x; xv[4 * v + 1] = f.y; xv[4 * v + 2] = f.z; xv[4 * v + 3] = f.w;
        }
        float da = 0.0f, db = 0.0f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          da = __fmaf_rn(xv[k], qa[k], da);
          db = __fmaf_rn(xv[k], qb[k], db);
        }
        const float xs = XS[(size_t)t * (H / 16) + ci];
        acca[t] = __fmaf_rn(b_a, xs, __fmaf_rn(s_a, da, acca[t]));
        accb[t] = __fmaf_rn(b_b, xs, __fmaf_rn(s_b, db, accb[t]));
      }
    }
  }
#pragma unroll
  for (int t = 0; t < BD_TOK; ++t) {
    oa[t] = group_sum_bfly(acca[t], 32);
    ob[t] = group_sum_bfly(accb[t], 32);
  }
}

template <int CPL>
__global__ void __launch_bounds__(BD_THREADS) k_batch_dense(const BatchDenseArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  int* flag = reinterpret_cast<int*>(smem + 16);
  const int H = a.H;
  float4* X = reinterpret_cast<float4*>(smem + SMEM_HDR);                        // (BD_TOK, H) fp32, lane-interleaved
  float* XS = reinterpret_cast<float*>(X + (size_t)BD_TOK * (H / 4));            // (BD_TOK, H / 16) chunk sums
  uint8_t* tile = reinterpret_cast<uint8_t*>(XS + (size_t)BD_TOK * (H / 16));

  const int tid = threadIdx.x, warp = tid >> 5;
  const int t0 = blockIdx.y * BD_TOK, nt = min(BD_TOK, a.T - t0);
  int t = blockIdx.x, kind, row0, nrows;
  QM m0 = a.router, m1 = a.router;
  if (t < a.nt_router) {
    kind = 0; row0 = t * BD_RROWS; nrows = BD_RROWS; m0 = a.router;
  } else if ((t -= a.nt_router) < a.nt_shared) {
    kind = 1; row0 = t * BD_SUNITS; nrows = BD_SUNITS; m0 = a.sh_gate; m1 = a.sh_up;
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
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  {
    Piece pc[8];
    int n = 0;
    pc[n++] = {reinterpret_cast<uint8_t*>(X), reinterpret_cast<const uint8_t*>(a.xf + (size_t)t0 * (H / 4)),
               (uint32_t)(nt * H * 4)};
    pc[n++] = {reinterpret_cast<uint8_t*>(XS), reinterpret_cast<const uint8_t*>(a.xsum + (size_t)t0 * (H / 16)),
               (uint32_t)(nt * (H / 16) * 4)};
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
  const bool ok = mbar_wait_block(bar, 0, a.err);
  if (ok) {
    // router: warp w takes rows w and w + 8; shared: unit w (gate and up rows
    // as the pair); gate row: warp 0
    float oa[BD_TOK], ob[BD_TOK];
    if (kind == 0) {
      const int rA = warp, rB = warp + 8;
      dense_rows2<CPL>(pc_codes[0] + (size_t)rA * rb, pc_s[0] + (size_t)rA * ng, pc_b[0] + (size_t)rA * ng,
                       pc_codes[0] + (size_t)rB * rb, pc_s[0] + (size_t)rB * ng, pc_b[0] + (size_t)rB * ng, X, XS,
                       H, nt, m0.gs, oa, ob);
      if ((tid & 31) == 0) {
        const float bA = a.rbias ? a.rbias[row0 + rA] : 0.0f, bB = a.rbias ? a.rbias[row0 + rB] : 0.0f;
        for (int tt = 0; tt < nt; ++tt) {
          a.logits[(size_t)(t0 + tt) * a.E + row0 + rA] = bf16r(__fadd_rn(oa[tt], bA));
          a.logits[(size_t)(t0 + tt) * a.E + row0 + rB] = bf16r(__fadd_rn(ob[tt], bB));
        }
      }
    } else if (kind == 1) {
      const int r = warp;
      dense_rows2<CPL>(pc_codes[0] + (size_t)r * rb, pc_s[0] + (size_t)r * ng, pc_b[0] + (size_t)r * ng,
                       pc_codes[1] + (size_t)r * rb, pc_s[1] + (size_t)r * ng, pc_b[1] + (size_t)r * ng, X, XS, H,
                       nt, m0.gs, oa, ob);
      if ((tid & 31) == 0)
        for (int tt = 0; tt < nt; ++tt)
          a.act_sh[(size_t)(t0 + tt) * a.Ish + row0 + r] = f32_to_bf16(swiglu_bf16(bf16r(oa[tt]), bf16r(ob[tt])));
    } else if (warp == 0) {
      dense_rows2<CPL>(pc_codes[0], pc_s[0], pc_b[0], pc_codes[0], pc_s[0], pc_b[0], X, XS, H, nt, m0.gs, oa, ob);
      if ((tid & 31) == 0)
        for (int tt = 0; tt < nt; ++tt) a.sgate[t0 + tt] = bf16r(sigmoid_f32(bf16r(oa[tt])));
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
    for (int tt = t0 + warp; tt < t0 + nt; tt += BD_THREADS / 32)
      route_row(a.logits + (size_t)tt * a.E, a.E, a.K, a.norm_topk, a.ids + (size_t)tt * a.K,
                a.wts + (size_t)tt * a.K);
  }
}

}  // namespace ynb
