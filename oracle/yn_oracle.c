/*
 * CPU oracle for the sparse-MoE decode path. TEST INFRASTRUCTURE ONLY: the
 * checker that tests, the smoke check and the benchmark's CPU-baseline leg
 * compare the CUDA library against. Nothing in the product links or calls it.
 *
 * It restates, in plain C, the arithmetic of the reference engine's MLX
 * path (moe_prefetch/mlx_backend.py) with every unpinned detail fixed:
 *   - MLX affine dequantisation w = scale*q + bias (mlx_backend.py:442-445,
 *     quantize_2bit.py:158-160), codes little-endian inside uint32 words.
 *   - QuantizedLinear / gather_qmm as per-group  scale*sum(x*q) + bias*sum(x)
 *     in fp32, summed in the canonical lane/chunk order of the CUDA kernels
 *     (16-byte chunks, LPR lanes per row, butterfly over the lanes).
 *   - Routing (mlx_backend.py:308-316): softmax in fp32 with a deterministic
 *     exp (Cody-Waite reduction + degree-7 Taylor), probabilities rounded to
 *     bf16, top-k by (probability desc, expert id asc), weights
 *     bf16(p / bf16(sum p)).
 *   - Lookahead forecast (mlx_backend.py:340-346): fp32 softmax of each target
 *     router applied to RMSNorm_t(h_res), max over rows.
 *   - SwiGLU experts (mlx_backend.py:447-459) with bf16 rounding after every
 *     elementwise op, shared expert sigmoid(gate(x)) * mlp(x) (:305), combine
 *     (y*w).sum over the k columns in column order (:420), routed + shared
 *     (:440), residual (orchestrator.py:287).
 * Routing, RMSNorm and the 8-bit GEMVs are bit-exact with the kernels; the
 * 2/4-bit expert GEMVs here are exact fp32 while the kernels use packed fp16
 * partial sums, so those are compared within a relative tolerance.
 *
 * Build: oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ----------------------------------------------------------- conversions */
static inline float bf16_to_f32(uint16_t b) {
  uint32_t u = ((uint32_t)b) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint16_t f32_to_bf16(float f) { /* round to nearest even; NaN kept quiet */
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}
static inline float bf16r(float f) { return bf16_to_f32(f32_to_bf16(f)); }

static inline float f16_to_f32(uint16_t h) {
  uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1f, m = h & 0x3ff, u;
  if (e == 0) {
    if (m == 0) {
      u = s;
    } else { /* subnormal: normalise */
      int sh = 0;
      while (!(m & 0x400)) { m <<= 1; ++sh; }
      m &= 0x3ff;
      u = s | ((uint32_t)(127 - 15 - sh + 1) << 23) | (m << 13);
    }
  } else if (e == 31) {
    u = s | 0x7f800000u | (m << 13);
  } else {
    u = s | ((e + 112) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint16_t f32_to_f16(float f) { /* round to nearest even */
  uint32_t u;
  memcpy(&u, &f, 4);
  uint32_t s = (u >> 16) & 0x8000u;
  uint32_t a = u & 0x7fffffffu;
  if (a > 0x7f800000u) return (uint16_t)(s | 0x7e00u);
  if (a >= 0x477ff000u) return (uint16_t)(s | 0x7c00u); /* >= 65520 rounds to inf */
  if (a < 0x38800000u) {                                 /* below 2^-14: subnormal or zero */
    if (a < 0x33000000u) return (uint16_t)s;             /* < 2^-25 rounds to 0 */
    uint32_t e = a >> 23, m = (a & 0x7fffffu) | 0x800000u;
    uint32_t shift = 126 - e; /* 14 - (e - 127) + 13 - 1 ... mantissa shift */
    /* value = m * 2^(e-150); half subnormal unit = 2^-24 -> q = m * 2^(e-126) */
    uint32_t sh = 126 - e;
    uint32_t q = m >> sh;
    uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    (void)shift;
    return (uint16_t)(s | q);
  }
  uint32_t e = (a >> 23) - 112, m = a & 0x7fffffu;
  uint32_t q = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;
  return (uint16_t)(s | q);
}

/* --------------------------------------------------- synthetic generator */
static inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static inline uint64_t stream_key(uint64_t seed, uint64_t sid) { return mix64(seed ^ mix64(sid + 0x632BE59BD9B4E019ull)); }
static inline float irwin_hall(uint64_t key, int64_t i) {
  uint64_t h = mix64(key + (uint64_t)i);
  int u = (int)(h & 0xFFFF) + (int)((h >> 16) & 0xFFFF) + (int)((h >> 32) & 0xFFFF) + (int)(h >> 48);
  return (float)(u - 131070);
}

/* Elements [start, start + n) of stream (seed, sid). */
void yo_synth_u32(uint32_t* dst, int64_t n, uint64_t seed, uint64_t sid, int64_t start) {
  uint64_t key = stream_key(seed, sid);
  for (int64_t i = 0; i < n; ++i) dst[i] = (uint32_t)(mix64(key + (uint64_t)(start + i)) >> 32);
}
void yo_synth_f16(uint16_t* dst, int64_t n, uint64_t seed, uint64_t sid, float std, int absolute, int64_t start) {
  uint64_t key = stream_key(seed, sid);
  const float c = std / 37837.227f;
  for (int64_t i = 0; i < n; ++i) {
    float v = irwin_hall(key, start + i) * c;
    if (absolute) v = fabsf(v);
    dst[i] = f32_to_f16(v);
  }
}
void yo_synth_bf16(uint16_t* dst, int64_t n, uint64_t seed, uint64_t sid, float std, float mean, int64_t start) {
  uint64_t key = stream_key(seed, sid);
  const float c = std / 37837.227f;
  for (int64_t i = 0; i < n; ++i) dst[i] = f32_to_bf16(irwin_hall(key, start + i) * c + mean);
}
/* Conversions exposed for tests. */
void yo_f32_to_bf16(const float* x, int64_t n, uint16_t* out) { for (int64_t i = 0; i < n; ++i) out[i] = f32_to_bf16(x[i]); }
void yo_f32_to_f16(const float* x, int64_t n, uint16_t* out) { for (int64_t i = 0; i < n; ++i) out[i] = f32_to_f16(x[i]); }
void yo_f16_to_f32(const uint16_t* x, int64_t n, float* out) { for (int64_t i = 0; i < n; ++i) out[i] = f16_to_f32(x[i]); }

/* -------------------------------------------------------- deterministic exp */
static inline float pow2i(int n) {
  uint32_t u = (uint32_t)(n + 127) << 23;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
float yo_expf(float x) {
  if (!(x > -87.33654f)) return 0.0f;
  if (x > 88.72283f) return INFINITY;
  float n = rintf(x * 1.44269504f);
  float r = fmaf(-n, 0.693145751953125f, x);
  r = fmaf(-n, 1.428606820309417e-06f, r);
  float p = 1.984126984e-4f;
  p = fmaf(p, r, 1.388888889e-3f);
  p = fmaf(p, r, 8.333333333e-3f);
  p = fmaf(p, r, 4.166666667e-2f);
  p = fmaf(p, r, 1.666666667e-1f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int ni = (int)n;
  int a = ni >> 1, b = ni - a;
  return (p * pow2i(a)) * pow2i(b);
}
static inline float sigmoid_f32(float g) { return 1.0f / (1.0f + yo_expf(-g)); }
static inline float swiglu_bf16(float g, float u) {
  float s = bf16r(sigmoid_f32(g));
  float silu = bf16r(g * s);
  return bf16r(silu * u);
}

/* --------------------------------------------------------- quantised rows */
typedef struct yo_qmat {
  const uint32_t* w;
  const uint16_t* s;
  const uint16_t* b;
  int32_t rows, cols, bits, gs;
} yo_qmat;

static int lanes_per_row(int rowbytes) {
  int chunks = rowbytes / 16, l = 1;
  while (l < 32 && (chunks % (2 * l)) == 0) l *= 2;
  return l;
}

/* Canonical fp32 dot of one quantised row with x (bf16 bits, K values). */
static float row_dot(const uint8_t* codes, const uint16_t* sc, const uint16_t* bi, const uint16_t* x, int K, int bits,
                     int gs) {
  const int rowbytes = K * bits / 8;
  const int lpr = lanes_per_row(rowbytes);
  const int cpl = (rowbytes / 16) / lpr;
  const int cpc = 128 / bits, cpw = 32 / bits;
  const uint32_t mask = (1u << bits) - 1u;
  const int seg = cpc < gs ? cpc : gs;
  const int nseg = cpc / seg;
  float lane[32];
  for (int l = 0; l < lpr; ++l) {
    float acc = 0.0f;
    for (int c = 0; c < cpl; ++c) {
      const int ci = l + lpr * c;
      const uint8_t* ch = codes + 16 * ci;
      uint32_t wv[4];
      memcpy(wv, ch, 16);
      const int k0 = ci * cpc;
      for (int s = 0; s < nseg; ++s) {
        float d = 0.0f, xs = 0.0f;
        for (int e = 0; e < seg; ++e) {
          const int kk = s * seg + e;
          const uint32_t q = (wv[kk / cpw] >> (bits * (kk % cpw))) & mask;
          const float xv = bf16_to_f32(x[k0 + kk]);
          d = fmaf(xv, (float)q, d);
          xs = xs + xv;
        }
        const int g = (k0 + s * seg) / gs;
        acc = fmaf(f16_to_f32(sc[g]), d, acc);
        acc = fmaf(f16_to_f32(bi[g]), xs, acc);
      }
    }
    lane[l] = acc;
  }
  for (int m = lpr >> 1; m > 0; m >>= 1) {
    float nv[32];
    for (int l = 0; l < lpr; ++l) nv[l] = lane[l] + lane[l ^ m];
    memcpy(lane, nv, sizeof(float) * lpr);
  }
  return lane[0];
}

static inline const uint8_t* qrow_codes(const yo_qmat* m, int r) { return (const uint8_t*)m->w + (size_t)r * m->cols * m->bits / 8; }
static inline const uint16_t* qrow_s(const yo_qmat* m, int r) { return m->s + (size_t)r * (m->cols / m->gs); }
static inline const uint16_t* qrow_b(const yo_qmat* m, int r) { return m->b + (size_t)r * (m->cols / m->gs); }

/* y[t][r] = bf16(dot(x[t], row r)) held in fp32. */
void yo_qlinear(const yo_qmat* m, const uint16_t* x, int T, float* y) {
  for (int t = 0; t < T; ++t) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < m->rows; ++r)
      y[(size_t)t * m->rows + r] =
          bf16r(row_dot(qrow_codes(m, r), qrow_s(m, r), qrow_b(m, r), x + (size_t)t * m->cols, m->cols, m->bits, m->gs));
  }
}

/* out[r][k] = fmaf(scale, q, bias) */
void yo_dequantize(const yo_qmat* m, float* out) {
  const int cpw = 32 / m->bits, ng = m->cols / m->gs;
  const uint32_t mask = (1u << m->bits) - 1u;
  for (int r = 0; r < m->rows; ++r)
    for (int k = 0; k < m->cols; ++k) {
      const uint32_t word = m->w[(size_t)r * (m->cols / cpw) + k / cpw];
      const uint32_t q = (word >> (m->bits * (k % cpw))) & mask;
      const int g = k / m->gs;
      out[(size_t)r * m->cols + k] = fmaf(f16_to_f32(m->s[(size_t)r * ng + g]), (float)q, f16_to_f32(m->b[(size_t)r * ng + g]));
    }
}

/* ------------------------------------------------------------- RMSNorm */
/* Canonical 128-thread order: thread i sums x^2 over i + 128 j, butterfly
 * inside each 32-lane warp, warp partials summed in warp order. */
void yo_rmsnorm(const uint16_t* h, const uint16_t* w, int H, float eps, uint16_t* out) {
  float th[128];
  for (int i = 0; i < 128; ++i) {
    float ss = 0.0f;
    for (int j = i; j < H; j += 128) {
      const float v = bf16_to_f32(h[j]);
      ss = fmaf(v, v, ss);
    }
    th[i] = ss;
  }
  float wsum[4];
  for (int wp = 0; wp < 4; ++wp) {
    float lane[32];
    memcpy(lane, th + 32 * wp, sizeof(lane));
    for (int m = 16; m > 0; m >>= 1) {
      float nv[32];
      for (int l = 0; l < 32; ++l) nv[l] = lane[l] + lane[l ^ m];
      memcpy(lane, nv, sizeof(lane));
    }
    wsum[wp] = lane[0];
  }
  const float tot = ((wsum[0] + wsum[1]) + wsum[2]) + wsum[3];
  const float r = 1.0f / sqrtf(tot / (float)H + eps);
  for (int i = 0; i < H; ++i) out[i] = f32_to_bf16(bf16_to_f32(w[i]) * bf16r(bf16_to_f32(h[i]) * r));
}

/* ------------------------------------------------------------- routing */
static void softmax_canonical(const float* logits, int E, float* p_out /* unnormalised exp */, float* s_out) {
  float m = -INFINITY;
  for (int e = 0; e < E; ++e) m = fmaxf(m, logits[e]);
  float lane[32];
  for (int l = 0; l < 32; ++l) {
    float s = 0.0f;
    for (int e = l; e < E; e += 32) {
      const float p = yo_expf(logits[e] - m);
      p_out[e] = p;
      s = s + p;
    }
    lane[l] = s;
  }
  for (int mk = 16; mk > 0; mk >>= 1) {
    float nv[32];
    for (int l = 0; l < 32; ++l) nv[l] = lane[l] + lane[l ^ mk];
    memcpy(lane, nv, sizeof(lane));
  }
  *s_out = lane[0];
}

/* ids (k) in descending bf16 probability, ties to the lower id; weights as
 * bf16 values in fp32. probs_out (E, optional): bf16 probabilities. */
void yo_route_row(const float* logits, int E, int K, int norm, int32_t* ids, float* w, float* probs_out) {
  float* p = (float*)malloc(sizeof(float) * E);
  float s;
  softmax_canonical(logits, E, p, &s);
  for (int e = 0; e < E; ++e) p[e] = bf16r(p[e] / s);
  if (probs_out) memcpy(probs_out, p, sizeof(float) * E);
  float wsum = 0.0f;
  float sel[64];
  for (int j = 0; j < K; ++j) {
    int bi = -1;
    float bp = -2.0f;
    for (int e = 0; e < E; ++e)
      if (p[e] > bp) { bp = p[e]; bi = e; }
    ids[j] = bi;
    sel[j] = bp;
    p[bi] = -2.0f;
    wsum = wsum + bp;
  }
  const float sb = bf16r(wsum);
  for (int j = 0; j < K; ++j) w[j] = norm ? bf16r(sel[j] / sb) : sel[j];
  free(p);
}

void yo_route(const float* logits, int T, int E, int K, int norm, int32_t* ids, float* w) {
  for (int t = 0; t < T; ++t) yo_route_row(logits + (size_t)t * E, E, K, norm, ids + (size_t)t * K, w + (size_t)t * K, NULL);
}

/* fp32 softmax probabilities of one row (lookahead forecast). */
void yo_softmax_f32(const float* logits, int E, float* probs) {
  float s;
  softmax_canonical(logits, E, probs, &s);
  for (int e = 0; e < E; ++e) probs[e] = probs[e] / s;
}

/* ------------------------------------------------------------ layer math */
typedef struct yo_dense {
  const uint16_t* norm;    /* (H) bf16 post_attention_layernorm */
  yo_qmat router;          /* (E, H) */
  const float* rbias;      /* (E) or NULL */
  yo_qmat sh_gate, sh_up;  /* (Ish, H) */
  yo_qmat sh_down;         /* (H, Ish) */
  yo_qmat sgate;           /* (1, H) */
  int32_t has_shared;
} yo_dense;

typedef struct yo_dims {
  int32_t H, E, K, I, Ish, norm_topk;
  float eps;
} yo_dims;

/* Post-attention block for T rows: x, logits, shared activations, sigmoid
 * gate, routing, lookahead probabilities. Outputs mirror the workspace view. */
void yo_post_attention(const yo_dims* d, const yo_dense* L, const uint16_t* h1, int T, const yo_dense* targets,
                       int NT, uint16_t* x, float* logits, uint16_t* act_sh, float* sgate, int32_t* ids, float* w,
                       float* fprobs) {
  const int H = d->H, E = d->E;
  for (int t = 0; t < T; ++t) {
    const uint16_t* ht = h1 + (size_t)t * H;
    uint16_t* xt = x + (size_t)t * H;
    yo_rmsnorm(ht, L->norm, H, d->eps, xt);
#pragma omp parallel for schedule(static)
    for (int e = 0; e < E; ++e) {
      const float v = row_dot(qrow_codes(&L->router, e), qrow_s(&L->router, e), qrow_b(&L->router, e), xt, H, 8, L->router.gs);
      logits[(size_t)t * E + e] = bf16r(v + (L->rbias ? L->rbias[e] : 0.0f));
    }
    if (L->has_shared) {
#pragma omp parallel for schedule(static)
      for (int n = 0; n < d->Ish; ++n) {
        const float g = row_dot(qrow_codes(&L->sh_gate, n), qrow_s(&L->sh_gate, n), qrow_b(&L->sh_gate, n), xt, H, 8, L->sh_gate.gs);
        const float u = row_dot(qrow_codes(&L->sh_up, n), qrow_s(&L->sh_up, n), qrow_b(&L->sh_up, n), xt, H, 8, L->sh_up.gs);
        act_sh[(size_t)t * d->Ish + n] = f32_to_bf16(swiglu_bf16(bf16r(g), bf16r(u)));
      }
      const float sv = row_dot(qrow_codes(&L->sgate, 0), qrow_s(&L->sgate, 0), qrow_b(&L->sgate, 0), xt, H, 8, L->sgate.gs);
      sgate[t] = bf16r(sigmoid_f32(bf16r(sv)));
    }
    yo_route_row(logits + (size_t)t * E, E, d->K, d->norm_topk, ids + (size_t)t * d->K, w + (size_t)t * d->K, NULL);
  }
  uint16_t* xt = (uint16_t*)malloc(sizeof(uint16_t) * H);
  float* lg = (float*)malloc(sizeof(float) * E);
  float* pr = (float*)malloc(sizeof(float) * E);
  for (int g = 0; g < NT; ++g) {
    const yo_dense* Tg = &targets[g];
    for (int t = 0; t < T; ++t) {
      yo_rmsnorm(h1 + (size_t)t * H, Tg->norm, H, d->eps, xt);
#pragma omp parallel for schedule(static)
      for (int e = 0; e < E; ++e) {
        const float v = row_dot(qrow_codes(&Tg->router, e), qrow_s(&Tg->router, e), qrow_b(&Tg->router, e), xt, H, 8, Tg->router.gs);
        lg[e] = bf16r(v + (Tg->rbias ? Tg->rbias[e] : 0.0f));
      }
      yo_softmax_f32(lg, E, pr);
      for (int e = 0; e < E; ++e) fprobs[(size_t)g * E + e] = (t == 0) ? pr[e] : fmaxf(fprobs[(size_t)g * E + e], pr[e]);
    }
  }
  free(xt);
  free(lg);
  free(pr);
}

typedef struct yo_record {
  int32_t bits, gs;
  int64_t off[9];
} yo_record;

static void piece_qmat(const uint8_t* rec, const yo_record* rg, int which /*0 gate,1 up,2 down*/, int rows, int cols,
                       yo_qmat* m) {
  m->w = (const uint32_t*)(rec + rg->off[3 * which + 0]);
  m->s = (const uint16_t*)(rec + rg->off[3 * which + 1]);
  m->b = (const uint16_t*)(rec + rg->off[3 * which + 2]);
  m->rows = rows;
  m->cols = cols;
  m->bits = rg->bits;
  m->gs = rg->gs;
}

/* One routed expert on one row: act (I) bf16 and y (H) bf16. */
void yo_expert(const yo_dims* d, const uint8_t* rec, const yo_record* rg, const uint16_t* x, uint16_t* act, uint16_t* y) {
  yo_qmat g, u, dn;
  piece_qmat(rec, rg, 0, d->I, d->H, &g);
  piece_qmat(rec, rg, 1, d->I, d->H, &u);
  piece_qmat(rec, rg, 2, d->H, d->I, &dn);
#pragma omp parallel for schedule(static)
  for (int n = 0; n < d->I; ++n) {
    const float gv = row_dot(qrow_codes(&g, n), qrow_s(&g, n), qrow_b(&g, n), x, d->H, g.bits, g.gs);
    const float uv = row_dot(qrow_codes(&u, n), qrow_s(&u, n), qrow_b(&u, n), x, d->H, u.bits, u.gs);
    act[n] = f32_to_bf16(swiglu_bf16(bf16r(gv), bf16r(uv)));
  }
#pragma omp parallel for schedule(static)
  for (int r = 0; r < d->H; ++r)
    y[r] = f32_to_bf16(row_dot(qrow_codes(&dn, r), qrow_s(&dn, r), qrow_b(&dn, r), act, d->I, dn.bits, dn.gs));
}

/* Shared expert down projection of one row: bf16(sg * bf16(down(act_sh))). */
void yo_shared_down(const yo_dims* d, const yo_dense* L, const uint16_t* act_sh, float sg, uint16_t* ysh) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < d->H; ++r) {
    const float v = row_dot(qrow_codes(&L->sh_down, r), qrow_s(&L->sh_down, r), qrow_b(&L->sh_down, r), act_sh, d->Ish, 8,
                            L->sh_down.gs);
    ysh[r] = f32_to_bf16(sg * bf16r(v));
  }
}

/* Combine one row: mode 0 routed, 1 + shared, 2 + residual. y: (K, H). */
void yo_combine(const yo_dims* d, const uint16_t* y, const float* w, const uint16_t* ysh, const uint16_t* h_res, int mode,
                uint16_t* out) {
  for (int r = 0; r < d->H; ++r) {
    float acc = 0.0f;
    for (int j = 0; j < d->K; ++j) acc = acc + bf16r(bf16_to_f32(y[(size_t)j * d->H + r]) * w[j]);
    float o = bf16r(acc);
    if (mode >= 1 && ysh) o = bf16r(o + bf16_to_f32(ysh[r]));
    if (mode == 2) o = bf16r(bf16_to_f32(h_res[r]) + o);
    out[r] = f32_to_bf16(o);
  }
}

/* One whole MoE layer for T rows (pool path, every expert resident).
 * records[t*K + j] points at the record of ids[t*K + j] (the caller resolves
 * the expert -> record mapping after routing; see yo_post_attention). */
void yo_moe_experts(const yo_dims* d, const yo_dense* L, const yo_record* rg, const uint8_t* const* records,
                    const uint16_t* x, const uint16_t* act_sh, const float* sgate, const float* w, const uint16_t* h_res,
                    int T, int mode, uint16_t* act_out, uint16_t* y_out, uint16_t* ysh_out, uint16_t* out) {
  for (int t = 0; t < T; ++t) {
    for (int j = 0; j < d->K; ++j)
      yo_expert(d, records[t * d->K + j], rg, x + (size_t)t * d->H, act_out + ((size_t)t * d->K + j) * d->I,
                y_out + ((size_t)t * d->K + j) * d->H);
    const int sh = mode >= 1 && L->has_shared;
    if (sh) yo_shared_down(d, L, act_sh + (size_t)t * d->Ish, sgate[t], ysh_out + (size_t)t * d->H);
    yo_combine(d, y_out + (size_t)t * d->K * d->H, w + (size_t)t * d->K, sh ? ysh_out + (size_t)t * d->H : NULL,
               h_res ? h_res + (size_t)t * d->H : NULL, mode, out + (size_t)t * d->H);
  }
}

int yo_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
void yo_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
