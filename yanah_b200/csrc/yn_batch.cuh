// Union-of-experts kernels for a batch of token rows and the expert-parallel
// exchange between ranks over peer memory.
//
// A batch of T rows routes T*K (token, column) pairs. The pairs of the
// experts a rank holds are grouped by expert ("segments", ascending expert
// id), so every expert record is read from HBM once per layer however many
// rows chose it (mlx_backend.py:111-123 `_gather_sort`, :411-436 `moe`;
// orchestrator.py:361-405 `generate_batch` reads the union of the batch's
// experts).
//
// Tensor-core GEMV (mma.sync m16n8k16, fp16 in, fp32 accumulate) with the
// token rows as the n = 8 columns:
//  * weights: the 16-byte chunk ch of a row holds 128/BITS codes; lane
//    (g, c) of the warp reads word c of chunk ch of rows g and g+8 with one
//    ldmatrix (the tile is stored with chunk index XOR (row & 7) so the eight
//    rows of a matrix fall in different banks) and turns each word into fp16
//    pairs with one LOP3 per pair (1024 + mult*q exactly, yn_mma.cuh);
//  * activations: per row vector a "fragment" copy is built once per layer
//    (k_batch_frags): word (ch*4 + c)*PPW + p holds the pair of x values
//    under unpack pair p of word c of chunk ch, times the vector's power-of-
//    two scale and divided by the pair's code multiplier, as fp16;
//  * a group of GS codes covers whole chunks (GS*BITS/128 of them, at least
//    one), so one accumulator tile holds one group's dot products. It starts
//    at -1024 * sum(fragment values of the group) (the unpack offset) and the
//    group's scale and bias are applied in fp32 afterwards:
//        acc += s * D + b * scale * sum(x over the group);
//    the row result is acc / scale. 2-bit codes with 32-code groups (a group
//    is half a chunk) are not handled here.
//
// Expert parallelism (no counterpart in the reference, which runs on one
// device): rank r holds experts [e_lo, e_hi) of every layer and T_h home
// rows. Per layer each rank writes its home rows (normalised x, routed ids)
// into every rank's gather buffer with peer stores and raises a flag there;
// each rank computes the pairs of its experts for all rows and stores every
// output row y(t, j) straight into the home rank's (T_h, K, H) buffer, then
// adds the number of finished (pair, row tile) units to the home rank's
// counter; the home rank waits for its count and combines in column order,
// so the result is bit-identical for every number of ranks. Flags and
// counters are monotonic (targets derive from a per-rank step epoch), so a
// captured graph replays without resets. Every wait is bounded: on timeout
// the error word is set and the kernel skips its work.
#pragma once
#include "yn_common.cuh"
#include "yn_moe.cuh"
#include "yn_mma.cuh"

#ifndef YN_HOST_DEV
#define YN_HOST_DEV __host__ __device__
#endif

// Translation units that use only the device building blocks define
// YN_NO_BATCH_EP_KERNELS: the non-template kernels below (external linkage)
// are then left to yn_batch.cu.
namespace ynb {

constexpr int BT_MAX_TOK = 64;                       // rows of one batch (all ranks)
constexpr int BT_MAX_K = 16;
constexpr int BT_MAX_PAIRS = BT_MAX_TOK * BT_MAX_K;  // 1024
constexpr int BT_THREADS = 256;
constexpr int BT_MAX_RANKS = 8;
constexpr int BT_MAX_DISPATCH = 16;                  // dispatch CTAs per destination

enum : int { YN_ERR_PEER_TIMEOUT = 6, YN_ERR_BATCH_ID = 7 };

struct BatchPlan {
  int n_seg, n_pairs, n_up, n_dn;  // segments, pairs, up passes (8 rows), down passes (32 pairs)
  int seg_e[BT_MAX_PAIRS];         // expert id of segment s (ascending)
  int seg_off[BT_MAX_PAIRS + 1];   // pair range of segment s
  int seg_up0[BT_MAX_PAIRS + 1];   // first up pass of segment s
  int seg_dn0[BT_MAX_PAIRS + 1];   // first down pass of segment s
  int pair_tj[BT_MAX_PAIRS];       // t * K + j, by (expert, t, j)
};
constexpr int BT_UP_PASS = 8;      // token rows per up work item
constexpr int BT_DN_PASS = 32;     // pairs per down work item

// The plan's segment tables in shared memory (16-bit: every entry < 2^16),
// copied once per CTA so that work-item lookups do not chain global loads.
struct PlanSmem {
  uint16_t first[BT_MAX_PAIRS + 1];  // first pass of each segment (up or down passes)
  uint16_t seg_e[BT_MAX_PAIRS];
  uint16_t off[BT_MAX_PAIRS + 1];
  uint16_t tj[BT_MAX_PAIRS];
  int n_seg, n_pass;
};
YN_DEV void load_plan(const BatchPlan* p, bool up, PlanSmem* sm) {
  const int ns = p->n_seg, np = p->n_pairs;
  const int* first = up ? p->seg_up0 : p->seg_dn0;
  for (int i = threadIdx.x; i <= ns; i += blockDim.x) {
    sm->first[i] = (uint16_t)first[i];
    sm->off[i] = (uint16_t)p->seg_off[i];
    if (i < ns) sm->seg_e[i] = (uint16_t)p->seg_e[i];
  }
  for (int i = threadIdx.x; i < np; i += blockDim.x) sm->tj[i] = (uint16_t)p->pair_tj[i];
  if (threadIdx.x == 0) {
    sm->n_seg = ns;
    sm->n_pass = up ? p->n_up : p->n_dn;
  }
  __syncthreads();
}

// Segment of global pass index gp: the last s with first[s] <= gp.
YN_DEV int seg_of_pass(const uint16_t* first, int n_seg, int gp) {
  int lo = 0, hi = n_seg - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (first[mid] <= gp) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// ------------------------------------------------------------ code words
// Per-word unpack of one code word into PPW fp16 pairs; pair p holds word-
// local codes lo(p), hi(p) times the multiplier 1 / inv_mult(p).
template <int BITS>
struct BW;
template <>
struct BW<2> {
  static constexpr int PPW = 8;
  YN_DEV static int lo(int p) { return p; }
  YN_DEV static int hi(int p) { return p + 8; }
  YN_DEV static int pair_of(int j) { return j & 7; }
  YN_DEV static float inv_mult(int p) { return MmaFmt<2>::inv_mult(p); }
  YN_DEV static void unpack(uint32_t w, uint32_t (&pr)[8]) { MmaFmt<2>::unpack_raw(&w, pr); }
};
template <>
struct BW<4> {
  static constexpr int PPW = 4;
  YN_DEV static int lo(int p) { return p; }
  YN_DEV static int hi(int p) { return p + 4; }
  YN_DEV static int pair_of(int j) { return j & 3; }
  YN_DEV static float inv_mult(int p) { return (p & 1) ? 0.0625f : 1.0f; }
  YN_DEV static void unpack(uint32_t w, uint32_t (&pr)[4]) {
    const uint32_t M = 0x64006400u, a8 = w >> 8;
    pr[0] = (w & 0x000F000Fu) | M;
    pr[1] = (w & 0x00F000F0u) | M;
    pr[2] = (a8 & 0x000F000Fu) | M;
    pr[3] = (a8 & 0x00F000F0u) | M;
  }
};
template <>
struct BW<8> {
  static constexpr int PPW = 2;
  YN_DEV static int lo(int p) { return p; }
  YN_DEV static int hi(int p) { return p + 2; }
  YN_DEV static int pair_of(int j) { return j & 1; }
  YN_DEV static float inv_mult(int) { return 1.0f; }
  YN_DEV static void unpack(uint32_t w, uint32_t (&pr)[2]) {
    const uint32_t M = 0x64006400u;
    pr[0] = (w & 0x00FF00FFu) | M;
    pr[1] = ((w >> 8) & 0x00FF00FFu) | M;
  }
};

// Host/device geometry of one (BITS, GS) format over vectors of Kd codes.
template <int BITS, int GS>
struct BFmt {
  static constexpr int CPCH = 128 / BITS;        // codes per 16-byte chunk
  static constexpr int WPL = 32 / BITS;          // codes per word
  static constexpr int PPW = BW<BITS>::PPW;      // fp16 pairs per word
  static constexpr int MPC = PPW / 2;            // MMAs per chunk
  static constexpr int CPG = GS / CPCH;          // chunks per group
  static_assert(GS % CPCH == 0, "a group must cover whole 16-byte chunks");
  // fragment row padding (words) that spreads the 8 token rows of a B load
  // over distinct banks
  static constexpr int PADW = BITS == 2 ? 4 : (BITS == 4 ? 16 : 8);
};

YN_HOST_DEV inline int frag_stride_words(int Kd, int bits) {
  return Kd / 2 + (bits == 2 ? 4 : (bits == 4 ? 16 : 8));
}
// Group-data row: NG x {-1024 * sum(fragment values), scale * sum(x)}, then
// {1 / scale, 0}, padded to a multiple of 16 bytes.
YN_HOST_DEV inline int gdata_stride(int Kd, int gs) { return Kd / gs + 2; }

YN_DEV void mma16816c(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2], const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}

YN_DEV void ldsm_x4(uint32_t (&r)[4], const void* row_addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(row_addr)));
}

YN_DEV void cpa16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
YN_DEV void cpa_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Contiguous global -> shared copy by the whole block (16-byte pieces).
YN_DEV void cpa_block(void* dst, const void* src, int bytes) {
  uint8_t* d = reinterpret_cast<uint8_t*>(dst);
  const uint8_t* s = reinterpret_cast<const uint8_t*>(src);
  for (int i = threadIdx.x; i < bytes / 16; i += blockDim.x) cpa16(d + 16 * i, s + 16 * i);
}

// Rows of RB bytes from global into a swizzled shared tile: chunk ch of row r
// lands at r * RB + ((ch ^ (r & 7)) * 16). RB / 16 must be a multiple of 8.
// Row index of piece i for cpr pieces per row: a shift when cpr is a power
// of two, a division otherwise.
YN_DEV int piece_row(int i, int cpr, int sh) { return sh >= 0 ? i >> sh : i / cpr; }
YN_DEV int pow2_shift(int cpr) { return (cpr & (cpr - 1)) == 0 ? __ffs(cpr) - 1 : -1; }

// RB / 16 must be a multiple of 8 (the XOR stays inside the row).
YN_DEV void cpa_rows_swz(uint8_t* dst, int row0, const uint8_t* src, int rows, int RB) {
  const int cpr = RB >> 4, sh = pow2_shift(cpr);
  for (int i = threadIdx.x; i < rows * cpr; i += blockDim.x) {
    const int r = piece_row(i, cpr, sh), ch = i - r * cpr, rr = row0 + r;
    cpa16(dst + (size_t)rr * RB + ((ch ^ (rr & 7)) << 4), src + ((size_t)i << 4));
  }
}

// Rows of `bytes` bytes into rows of `stride` bytes (both multiples of 16).
YN_DEV void cpa_rows(uint8_t* dst, int stride, const uint8_t* src, int rows, int bytes) {
  const int cpr = bytes >> 4, sh = pow2_shift(cpr);
  for (int i = threadIdx.x; i < rows * cpr; i += blockDim.x) {
    const int r = piece_row(i, cpr, sh), ch = i - r * cpr;
    cpa16(dst + (size_t)r * stride + (ch << 4), src + ((size_t)i << 4));
  }
}

// -------------------------------------------------------- peer signalling
YN_DEV void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
YN_DEV unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
YN_DEV void red_release_sys_add_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Thread 0 waits until *p >= target (2 s limit), then the block syncs. Returns
// false (block-uniform) on timeout or when another kernel already failed.
YN_DEV bool wait_geq_block(const unsigned long long* p, unsigned long long target, int* err) {
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    int ok = 1;
    if (ld_acquire_sys_u64(p) < target) {
      const uint64_t t0 = globaltimer_ns();
      unsigned n = 0;
      while (ld_acquire_sys_u64(p) < target) {
        if ((++n & 63u) == 0) {
          if (*(volatile int*)err != 0 || globaltimer_ns() - t0 > 2000000000ull) {
            raise_error(err, YN_ERR_PEER_TIMEOUT);
            ok = 0;
            break;
          }
        }
      }
    }
    ok_s = ok;
  }
  __syncthreads();
  const bool ok = ok_s != 0;
  __syncthreads();
  return ok;
}

// ------------------------------------------------------------------ args
struct EpPeers {
  uint16_t* x_all[BT_MAX_RANKS];               // (G*T_h, H) gather buffer of rank d
  int32_t* ids_all[BT_MAX_RANKS];              // (G*T_h, K)
  unsigned long long* flag[BT_MAX_RANKS];      // (G, BT_MAX_DISPATCH) arrival flags of rank d: [writer][cta]
  uint16_t* y[BT_MAX_RANKS];                   // (T_h, K, H) routed outputs of rank d's rows
  unsigned long long* cnt[BT_MAX_RANKS];       // finished-unit counter of rank d
};

struct EpStep {      // what every EP kernel of one layer knows
  int rank, G, T_h, L, layer;
  const unsigned long long* epoch;  // this rank's step counter (device)
  int* err;
};

YN_DEV unsigned long long ep_stamp(const EpStep& s) {
  return (*s.epoch) * (unsigned long long)s.L + (unsigned long long)s.layer + 1ull;
}

struct DispatchArgs {
  EpStep st;
  EpPeers peers;
  const uint16_t* x_home;   // (T_h, H)
  const int32_t* ids_home;  // (T_h, K)
  int H, K;
};

struct FragArgs {
  const uint16_t* src;      // rows of Kd bf16 values
  long long src_stride;     // elements between rows
  int n_rows, Kd;
  const int* n_rows_dev;    // optional device row count (at most n_rows)
  uint32_t* xf;             // (n_rows, frag_stride_words) fp16-pair words
  float2* xg;               // (n_rows, gdata_stride)
  // k_batch_prep only: wait for every rank's rows, then block 0 plans
  EpStep st;
  const unsigned long long* flags;  // this rank's arrival flags (G, BT_MAX_DISPATCH)
  int n_dispatch;           // dispatch CTAs per source rank
  const int32_t* ids;       // (n_rows, K) routed ids of every row
  int K, E, e_lo, e_hi;
  BatchPlan* plan;
};

struct BatchUpArgs {
  const BatchPlan* plan;
  const uint32_t* xf;
  const float2* xg;
  int xf_stride, xg_stride;
  const uint8_t* base;
  long long stride;
  const int32_t* slot_of;   // expert -> slot, or null for slot = e - e_lo
  int n_slots, e_lo;
  RecGeom rg;
  int H, I, K;
  uint16_t* act;            // (n_pairs, I) bf16, plan order
  int* err;
};

struct BatchDownArgs {
  // routed: the down passes of `plan`, pairs in plan order; shared: n_shared
  // rows (pair p = home row p) through the shared expert's down matrix
  const BatchPlan* plan;
  int shared, n_shared;
  const uint32_t* af;
  const float2* ag;
  int af_stride, ag_stride;
  const uint8_t* base;
  long long stride;
  const int32_t* slot_of;
  int n_slots, e_lo;
  RecGeom rg;
  QM sh_down;
  int H, I, K;
  EpStep st;
  EpPeers peers;
  uint16_t* ysh;            // (n_shared, H) shared outputs
  const float* sgate;       // (n_shared)
  int* err;
};

struct CombineArgs {
  EpStep st;
  const unsigned long long* cnt;  // this rank's counter
  unsigned long long per_layer;   // units expected per layer
  const uint16_t* y;        // (T_h, K, H)
  const float* w;           // (T_h, K)
  const uint16_t* ysh;      // (T_h, H) or null
  const uint16_t* h_res;    // (T_h, H) or null
  uint16_t* out;            // (T_h, H)
  int H, K, mode;
};

// ------------------------------------------------------------- dispatch
// Grid (G, NB): the NB CTAs of destination d copy slices of this rank's home
// rows (and CTA 0 the ids) into rank d's gather buffer; each CTA then raises
// its own flag there, flag[rank][cta] (a release at system scope, after the
// block barrier, so it covers every store of the CTA).
#ifndef YN_NO_BATCH_EP_KERNELS
__global__ void __launch_bounds__(BT_THREADS) k_ep_dispatch(const DispatchArgs a) {
  const int d = blockIdx.x, nb = gridDim.y;
  const EpStep& s = a.st;
  const size_t row0 = (size_t)s.rank * s.T_h;
  uint4* xd = reinterpret_cast<uint4*>(a.peers.x_all[d] + row0 * a.H);
  const uint4* xs = reinterpret_cast<const uint4*>(a.x_home);
  const int nx = s.T_h * a.H / 8;
  constexpr int U = 4;
  for (int i0 = (blockIdx.y * BT_THREADS + threadIdx.x) * U; i0 < nx; i0 += nb * BT_THREADS * U) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i0 + u < nx) v[u] = xs[i0 + u];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i0 + u < nx) xd[i0 + u] = v[u];
  }
  if (blockIdx.y == 0) {
    int32_t* id = a.peers.ids_all[d] + row0 * a.K;
    for (int i = threadIdx.x; i < s.T_h * a.K; i += blockDim.x) id[i] = a.ids_home[i];
  }
  __syncthreads();  // the CTA's stores, then its flag (a release covers them)
  if (threadIdx.x == 0) st_release_sys_u64(a.peers.flag[d] + s.rank * BT_MAX_DISPATCH + blockIdx.y, ep_stamp(s));
}
#endif  // YN_NO_BATCH_EP_KERNELS

// ------------------------------------------------------------ fragments
// One row per block: stage the row in shared memory, power-of-two scale from
// max|x|, fragment words, then per group {-1024 * sum(fragment values),
// scale * sum(x)} (butterfly over one warp per group) and {1 / scale, 0}.
template <int BITS, int GS>
YN_DEV void frag_row_block(const uint16_t* x_g, int Kd, uint32_t* xf, float2* xg, uint16_t* xs, float* red) {
  using F = BFmt<BITS, GS>;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  for (int i = tid; i < Kd / 8; i += blockDim.x)
    reinterpret_cast<uint4*>(xs)[i] = reinterpret_cast<const uint4*>(x_g)[i];
  __syncthreads();
  float mx = 0.0f;
  for (int k = tid; k < Kd; k += blockDim.x) mx = fmaxf(mx, fabsf(bf16_to_f32(xs[k])));
  mx = warp_max(mx);
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < nw; ++w) mx = fmaxf(mx, red[w]);
  const float scale = fp16_input_scale(mx);
  for (int w = tid; w < Kd / 2; w += blockDim.x) {
    const int p = w % F::PPW, wc = w / F::PPW;  // wc = ch * 4 + c
    const int base = (wc >> 2) * F::CPCH + (wc & 3) * F::WPL;
    const float m = __fmul_rn(scale, BW<BITS>::inv_mult(p));
    __half2 h = __floats2half2_rn(__fmul_rn(bf16_to_f32(xs[base + BW<BITS>::lo(p)]), m),
                                  __fmul_rn(bf16_to_f32(xs[base + BW<BITS>::hi(p)]), m));
    xf[w] = *reinterpret_cast<uint32_t*>(&h);
  }
  const int NG = Kd / GS;
  for (int g = warp; g < NG; g += nw) {
    float sx = 0.0f, o = 0.0f;
    for (int k = g * GS + lane; k < (g + 1) * GS; k += 32) {
      const float v = bf16_to_f32(xs[k]);
      sx = __fadd_rn(sx, v);
      const float m = __fmul_rn(scale, BW<BITS>::inv_mult(BW<BITS>::pair_of(k % F::WPL)));
      o = __fadd_rn(o, __half2float(__float2half_rn(__fmul_rn(v, m))));
    }
    sx = group_sum_bfly(sx, 32);
    o = group_sum_bfly(o, 32);
    if (lane == 0) xg[g] = make_float2(__fmul_rn(-1024.0f, o), __fmul_rn(scale, sx));
  }
  if (tid == 0) {
    xg[NG] = make_float2(__fdiv_rn(1.0f, scale), 0.0f);
    xg[NG + 1] = make_float2(0.0f, 0.0f);
  }
  __syncthreads();
}

// Block-wide exclusive scan of int4 (256 threads); returns the total.
YN_DEV int4 block_scan4(int4 v, int4* out_excl) {
  __shared__ int4 wsum[BT_THREADS / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int4 inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int x = __shfl_up_sync(0xffffffffu, inc.x, o), y = __shfl_up_sync(0xffffffffu, inc.y, o);
    const int z = __shfl_up_sync(0xffffffffu, inc.z, o), w = __shfl_up_sync(0xffffffffu, inc.w, o);
    if (lane >= o) { inc.x += x; inc.y += y; inc.z += z; inc.w += w; }
  }
  if (lane == 31) wsum[warp] = inc;
  __syncthreads();
  int4 base = make_int4(0, 0, 0, 0), tot = make_int4(0, 0, 0, 0);
  for (int w = 0; w < BT_THREADS / 32; ++w) {
    const int4 ws = wsum[w];
    if (w < warp) { base.x += ws.x; base.y += ws.y; base.z += ws.z; base.w += ws.w; }
    tot.x += ws.x; tot.y += ws.y; tot.z += ws.z; tot.w += ws.w;
  }
  *out_excl = make_int4(base.x + inc.x - v.x, base.y + inc.y - v.y, base.z + inc.z - v.z, base.w + inc.w - v.w);
  __syncthreads();
  return tot;
}

// Segments of the local experts: counting by expert in shared memory, a
// block scan over experts (ascending id), then each pair's rank among the
// earlier pairs of its expert (stable: (t, j) order).
YN_DEV void build_plan(const FragArgs& a) {
  __shared__ int ids_s[BT_MAX_PAIRS];
  __shared__ int cnt[1024];
  __shared__ int segof[1024];
  const int P = a.n_rows * a.K, El = a.e_hi - a.e_lo;
  for (int e = threadIdx.x; e < 1024; e += blockDim.x) cnt[e] = 0;
  for (int i = threadIdx.x; i < P; i += blockDim.x) ids_s[i] = a.ids[i];
  __syncthreads();
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    const int e = ids_s[i];
    if (e < 0 || e >= a.E) raise_error(a.st.err, YN_ERR_BATCH_ID);
    else if (e >= a.e_lo && e < a.e_hi) atomicAdd(&cnt[e - a.e_lo], 1);
  }
  __syncthreads();
  // thread i owns experts 4i..4i+3
  int c[4];
  int4 v = make_int4(0, 0, 0, 0);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int e = 4 * threadIdx.x + k;
    c[k] = e < El ? cnt[e] : 0;
    if (c[k]) {
      v.x += 1;
      v.y += c[k];
      v.z += (c[k] + BT_UP_PASS - 1) / BT_UP_PASS;
      v.w += (c[k] + BT_DN_PASS - 1) / BT_DN_PASS;
    }
  }
  int4 ex;
  const int4 tot = block_scan4(v, &ex);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (!c[k]) continue;
    const int e = 4 * threadIdx.x + k;
    a.plan->seg_e[ex.x] = a.e_lo + e;
    a.plan->seg_off[ex.x] = ex.y;
    a.plan->seg_up0[ex.x] = ex.z;
    a.plan->seg_dn0[ex.x] = ex.w;
    segof[e] = ex.x;
    ex.x += 1;
    ex.y += c[k];
    ex.z += (c[k] + BT_UP_PASS - 1) / BT_UP_PASS;
    ex.w += (c[k] + BT_DN_PASS - 1) / BT_DN_PASS;
  }
  if (threadIdx.x == 0) {
    a.plan->n_seg = tot.x;
    a.plan->n_pairs = tot.y;
    a.plan->n_up = tot.z;
    a.plan->n_dn = tot.w;
    a.plan->seg_off[tot.x] = tot.y;
    a.plan->seg_up0[tot.x] = tot.z;
    a.plan->seg_dn0[tot.x] = tot.w;
  }
  __syncthreads();
  // warp 0 places the pairs in index order, 32 at a time: a pair's position
  // is its segment start + the pairs of its expert placed before it
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    for (int e = lane; e < El; e += 32) cnt[e] = 0;
    __syncwarp();
    for (int i0 = 0; i0 < P; i0 += 32) {
      const int i = i0 + lane;
      const int e = i < P ? ids_s[i] : -1;
      const bool mine = e >= a.e_lo && e < a.e_hi;
      const int key = mine ? e : -1 - lane;  // non-local lanes match nobody
      const unsigned same = __match_any_sync(0xffffffffu, key);
      if (mine) {
        const int el = e - a.e_lo;
        const int before = __popc(same & ((1u << lane) - 1u));
        a.plan->pair_tj[a.plan->seg_off[segof[el]] + cnt[el] + before] = i;
      }
      __syncwarp();
      if (mine && (same >> lane) == 1u) cnt[e - a.e_lo] += __popc(same);  // highest lane of the group
      __syncwarp();
    }
  }
}

// After every rank's rows have arrived: block 0 builds the plan, block 1 + r
// the fragments of row r.
template <int BITS, int GS>
__global__ void __launch_bounds__(BT_THREADS) k_batch_prep(const FragArgs a) {
  __shared__ __align__(16) uint16_t xs[8192];
  __shared__ float red[BT_THREADS / 32];
  bool ok = true;
  for (int r = 0; r < a.st.G && ok; ++r)
    for (int q = 0; q < a.n_dispatch && ok; ++q)
      ok = wait_geq_block(a.flags + r * BT_MAX_DISPATCH + q, ep_stamp(a.st), a.st.err);
  if (!ok) return;
  if (blockIdx.x == 0) {
    build_plan(a);
    return;
  }
  const int xs_w = frag_stride_words(a.Kd, BITS), gsd = gdata_stride(a.Kd, GS);
  for (int r = blockIdx.x - 1; r < a.n_rows; r += gridDim.x - 1)
    frag_row_block<BITS, GS>(a.src + (size_t)r * a.src_stride, a.Kd, a.xf + (size_t)r * xs_w,
                             a.xg + (size_t)r * gsd, xs, red);
}

// Fragments of rows without waiting (activations of the pairs, shared rows).
template <int BITS, int GS>
__global__ void __launch_bounds__(BT_THREADS) k_batch_frags(const FragArgs a) {
  __shared__ __align__(16) uint16_t xs[8192];
  __shared__ float red[BT_THREADS / 32];
  if (*(volatile const int*)a.st.err) return;
  const int n = a.n_rows_dev ? min(a.n_rows, *a.n_rows_dev) : a.n_rows;
  const int xs_w = frag_stride_words(a.Kd, BITS), gsd = gdata_stride(a.Kd, GS);
  for (int r = blockIdx.x; r < n; r += gridDim.x)
    frag_row_block<BITS, GS>(a.src + (size_t)r * a.src_stride, a.Kd, a.xf + (size_t)r * xs_w,
                             a.xg + (size_t)r * gsd, xs, red);
}

// ------------------------------------------------------------- MMA core
// One warp: 16 rows (rows r0..r0+15 of the swizzled tile W, RB bytes per row)
// x chunks [c0, c0 + nch) x NCH token blocks of 8. XF: fragment rows of the
// pass (stride xs words), XG: group data rows (stride gsd). ntok: valid
// tokens of the pass. acc[t][i]: token block t, the lane's D layout
// (rows g, g+8; tokens 2c, 2c+1), in scaled units.
template <int BITS, int GS, int NCH>
YN_DEV void warp_tile(const uint8_t* W, int RB, int r0, const uint16_t* S, const uint16_t* Bs, int srow_h,
                      int c0, int nch, const uint32_t* XF, int xs, const float2* XG, int gsd, int ntok,
                      float (&acc)[NCH][4]) {
  using F = BFmt<BITS, GS>;
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  // ldmatrix row addresses: matrix i = lane >> 3 -> (row half i & 1, chunk +(i >> 1))
  const int mrow = r0 + ((lane >> 3) & 1) * 8 + (lane & 7);
  const int mch = lane >> 4;
  float d[NCH][4];
#pragma unroll 1
  for (int cp = 0; cp < nch; cp += 2) {
    uint32_t wr[4];
    {
      const int ch = c0 + cp + mch;
      ldsm_x4(wr, W + (size_t)mrow * RB + ((ch ^ (mrow & 7)) << 4));
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int ch = c0 + cp + h;
      const int grp = ch / F::CPG;
      const bool first = (ch % F::CPG) == 0, last = (ch % F::CPG) == F::CPG - 1;
      uint32_t pa[F::PPW], pb[F::PPW];
      BW<BITS>::unpack(wr[2 * h], pa);
      BW<BITS>::unpack(wr[2 * h + 1], pb);
#pragma unroll
      for (int t = 0; t < NCH; ++t) {
        const int n = 8 * t + g;  // token row of this lane's B fragment
        uint32_t xb[F::PPW];
        const uint32_t* src = XF + (size_t)n * xs + (size_t)(ch * 4 + c) * F::PPW;
        if (n < ntok) {
          if constexpr (F::PPW >= 4) {
#pragma unroll
            for (int q = 0; q < F::PPW; q += 4) {
              const uint4 v = *reinterpret_cast<const uint4*>(src + q);
              xb[q] = v.x; xb[q + 1] = v.y; xb[q + 2] = v.z; xb[q + 3] = v.w;
            }
          } else {
            const uint2 v = *reinterpret_cast<const uint2*>(src);
            xb[0] = v.x; xb[1] = v.y;
          }
        } else {
#pragma unroll
          for (int q = 0; q < F::PPW; ++q) xb[q] = 0u;
        }
        if (first) {
          const int t0 = 8 * t + 2 * c;
          const float n0 = XG[(size_t)t0 * gsd + grp].x, n1 = XG[(size_t)(t0 + 1) * gsd + grp].x;
          const float ci[4] = {n0, n1, n0, n1};
          const uint32_t A[4] = {pa[0], pb[0], pa[1], pb[1]};
          const uint32_t B[2] = {xb[0], xb[1]};
          mma16816c(d[t], A, B, ci);
        } else {
          const uint32_t A[4] = {pa[0], pb[0], pa[1], pb[1]};
          const uint32_t B[2] = {xb[0], xb[1]};
          mma16816(d[t], A, B);
        }
#pragma unroll
        for (int m = 1; m < F::MPC; ++m) {
          const uint32_t A[4] = {pa[2 * m], pb[2 * m], pa[2 * m + 1], pb[2 * m + 1]};
          const uint32_t B[2] = {xb[2 * m], xb[2 * m + 1]};
          mma16816(d[t], A, B);
        }
        if (last) {
          const int t0 = 8 * t + 2 * c;
          const float x0 = XG[(size_t)t0 * gsd + grp].y, x1 = XG[(size_t)(t0 + 1) * gsd + grp].y;
          const float s0 = f16_to_f32(S[(size_t)(r0 + g) * srow_h + grp]);
          const float s1 = f16_to_f32(S[(size_t)(r0 + g + 8) * srow_h + grp]);
          const float b0 = f16_to_f32(Bs[(size_t)(r0 + g) * srow_h + grp]);
          const float b1 = f16_to_f32(Bs[(size_t)(r0 + g + 8) * srow_h + grp]);
          acc[t][0] = __fmaf_rn(s0, d[t][0], __fmaf_rn(b0, x0, acc[t][0]));
          acc[t][1] = __fmaf_rn(s0, d[t][1], __fmaf_rn(b0, x1, acc[t][1]));
          acc[t][2] = __fmaf_rn(s1, d[t][2], __fmaf_rn(b1, x0, acc[t][2]));
          acc[t][3] = __fmaf_rn(s1, d[t][3], __fmaf_rn(b1, x1, acc[t][3]));
        }
      }
    }
  }
}

YN_DEV size_t al16(size_t v) { return (v + 15) & ~size_t(15); }

// ---------------------------------------------------------- gate / up
// Work item = (up pass, tile of 16*NUT units): the pass's at most 8 token
// rows of one expert. Warp w: unit subtile w % NUT, K slice w / NUT of
// H / (8 / NUT) codes; the slices' partials are summed in slice order.
template <int BITS, int GS, int NUT>
__global__ void __launch_bounds__(BT_THREADS) k_batch_up(const BatchUpArgs a) {
  using F = BFmt<BITS, GS>;
  constexpr int NKS = 8 / NUT, UR = 16 * NUT;
  extern __shared__ __align__(128) uint8_t smem[];
  if (*(volatile const int*)a.err) return;
  const int H = a.H, RB = H * BITS / 8, NG = H / GS;
  const int srow_b = (int)al16((size_t)NG * 2) + 16, srow_h = srow_b / 2;
  const int xs = a.xf_stride, gsd = a.xg_stride;
  uint8_t* Wt = smem;                                          // 2*UR rows (gate, up) x RB, swizzled
  uint16_t* Sg = reinterpret_cast<uint16_t*>(Wt + (size_t)2 * UR * RB);  // 4 x UR rows x srow_b
  uint16_t* Bg = Sg + (size_t)UR * srow_h;
  uint16_t* Su = Bg + (size_t)UR * srow_h;
  uint16_t* Bu = Su + (size_t)UR * srow_h;
  uint32_t* XF = reinterpret_cast<uint32_t*>(Bu + (size_t)UR * srow_h);  // 8 rows x xs
  float2* XG = reinterpret_cast<float2*>(XF + (size_t)8 * xs);           // 8 rows x gsd
  float* RED = reinterpret_cast<float*>(XG + (size_t)8 * gsd);           // NKS x 2 x UR x 8
  __shared__ int tok_s[8];
  __shared__ PlanSmem pl;
  load_plan(a.plan, true, &pl);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int ut = warp % NUT, ks = warp / NUT;
  const int tiles = a.I / UR;
  const int n_seg = pl.n_seg;
  const int n_items = pl.n_pass * tiles;
  const int nchunk = H / F::CPCH, cpw = nchunk / NKS;
  for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
    const int gp = it / tiles, u0 = (it % tiles) * UR;
    const int sidx = seg_of_pass(pl.first, n_seg, gp);
    const int e = pl.seg_e[sidx];
    const int p0 = pl.off[sidx] + (gp - pl.first[sidx]) * BT_UP_PASS;
    const int ntok = min(BT_UP_PASS, (int)pl.off[sidx + 1] - p0);
    const int slot = a.slot_of ? a.slot_of[e] : e - a.e_lo;
    if (slot < 0 || slot >= a.n_slots) {
      if (threadIdx.x == 0) raise_error(a.err, YN_ERR_BAD_SLOT);
      continue;
    }
    const uint8_t* rec = a.base + (size_t)slot * (size_t)a.stride;
    __syncthreads();  // the previous item is done with every buffer
    if (threadIdx.x < 8) tok_s[threadIdx.x] = threadIdx.x < ntok ? pl.tj[p0 + threadIdx.x] / a.K : 0;
    cpa_rows_swz(Wt, 0, rec + a.rg.off[0] + (size_t)u0 * RB, UR, RB);
    cpa_rows_swz(Wt, UR, rec + a.rg.off[3] + (size_t)u0 * RB, UR, RB);
    cpa_rows(reinterpret_cast<uint8_t*>(Sg), srow_b, rec + a.rg.off[1] + (size_t)u0 * NG * 2, UR, NG * 2);
    cpa_rows(reinterpret_cast<uint8_t*>(Bg), srow_b, rec + a.rg.off[2] + (size_t)u0 * NG * 2, UR, NG * 2);
    cpa_rows(reinterpret_cast<uint8_t*>(Su), srow_b, rec + a.rg.off[4] + (size_t)u0 * NG * 2, UR, NG * 2);
    cpa_rows(reinterpret_cast<uint8_t*>(Bu), srow_b, rec + a.rg.off[5] + (size_t)u0 * NG * 2, UR, NG * 2);
    __syncthreads();  // tok_s
    for (int r = 0; r < ntok; ++r) {
      const uint32_t* xr = a.xf + (size_t)tok_s[r] * xs;
      for (int q = threadIdx.x; q < xs / 4; q += blockDim.x) cpa16(XF + (size_t)r * xs + 4 * q, xr + 4 * q);
      const float2* gr = a.xg + (size_t)tok_s[r] * gsd;
      for (int q = threadIdx.x; q < gsd / 2; q += blockDim.x) cpa16(XG + (size_t)r * gsd + 2 * q, gr + 2 * q);
    }
    cpa_wait_all();
    __syncthreads();
    float ag[1][4] = {{0.f, 0.f, 0.f, 0.f}}, au[1][4] = {{0.f, 0.f, 0.f, 0.f}};
    warp_tile<BITS, GS, 1>(Wt, RB, 16 * ut, Sg, Bg, srow_h, ks * cpw, cpw, XF, xs, XG, gsd, ntok, ag);
    warp_tile<BITS, GS, 1>(Wt, RB, UR + 16 * ut, Su - (size_t)UR * srow_h, Bu - (size_t)UR * srow_h, srow_h,
                           ks * cpw, cpw, XF, xs, XG, gsd, ntok, au);
    // RED[ks][gu][unit][tok]
    float* rg_ = RED + ((size_t)(ks * 2 + 0) * UR) * 8;
    float* ru_ = RED + ((size_t)(ks * 2 + 1) * UR) * 8;
    const int u_a = 16 * ut + g, u_b = u_a + 8;
    rg_[u_a * 8 + 2 * c] = ag[0][0];
    rg_[u_a * 8 + 2 * c + 1] = ag[0][1];
    rg_[u_b * 8 + 2 * c] = ag[0][2];
    rg_[u_b * 8 + 2 * c + 1] = ag[0][3];
    ru_[u_a * 8 + 2 * c] = au[0][0];
    ru_[u_a * 8 + 2 * c + 1] = au[0][1];
    ru_[u_b * 8 + 2 * c] = au[0][2];
    ru_[u_b * 8 + 2 * c + 1] = au[0][3];
    __syncthreads();
    for (int i = threadIdx.x; i < UR * 8; i += blockDim.x) {
      const int tok = i / UR, u = i % UR;
      if (tok >= ntok) continue;
      float gs_ = 0.0f, us_ = 0.0f;
#pragma unroll
      for (int k = 0; k < NKS; ++k) {
        gs_ = __fadd_rn(gs_, RED[((size_t)(k * 2 + 0) * UR + u) * 8 + tok]);
        us_ = __fadd_rn(us_, RED[((size_t)(k * 2 + 1) * UR + u) * 8 + tok]);
      }
      const float inv = XG[(size_t)tok * gsd + NG].x;
      const float gv = bf16r(__fmul_rn(gs_, inv)), uv = bf16r(__fmul_rn(us_, inv));
      a.act[(size_t)(p0 + tok) * a.I + u0 + u] = f32_to_bf16(swiglu_bf16(gv, uv));
    }
  }
}

// --------------------------------------------------------------- down
// Work item = (down pass, tile of 64 output rows): the pass's at most 32
// pairs of one expert. Warp w: row subtile w & 3, K half w >> 2. Routed
// outputs go to the home rank's buffer (peer stores), then the home counter
// is raised by the item's pairs of that rank; shared outputs go to ysh
// (times the shared gate).
template <int BITS, int GS, int NCH>
__global__ void __launch_bounds__(BT_THREADS) k_batch_down(const BatchDownArgs a) {
  using F = BFmt<BITS, GS>;
  constexpr int RT = 64, PP = 8 * NCH;
  static_assert(PP == BT_DN_PASS, "a down item is one plan pass");
  extern __shared__ __align__(128) uint8_t smem[];
  if (*(volatile const int*)a.st.err) return;
  const int Kd = a.shared ? a.sh_down.cols : a.I;
  const int RB = Kd * BITS / 8, NG = Kd / GS, H = a.H;
  const int srow_b = (int)al16((size_t)NG * 2) + 16, srow_h = srow_b / 2;
  const int xs = a.af_stride, gsd = a.ag_stride;
  uint8_t* Wt = smem;
  uint16_t* Ss = reinterpret_cast<uint16_t*>(Wt + (size_t)RT * RB);
  uint16_t* Bs = Ss + (size_t)RT * srow_h;
  uint32_t* XF = reinterpret_cast<uint32_t*>(Bs + (size_t)RT * srow_h);
  float2* XG = reinterpret_cast<float2*>(XF + (size_t)PP * xs);
  float* RED = reinterpret_cast<float*>(XG + (size_t)PP * gsd);  // 2 x RT x PP
  __shared__ int home_cnt[BT_MAX_RANKS];
  __shared__ PlanSmem pl;
  if (!a.shared) load_plan(a.plan, false, &pl);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int rs = warp & 3, kh = warp >> 2;
  const int tiles = H / RT;
  const int n_pass = a.shared ? (a.n_shared + PP - 1) / PP : pl.n_pass;
  const int n_items = n_pass * tiles;
  const int nchunk = Kd / F::CPCH, cpw = nchunk / 2;
  const int T_h = a.st.T_h, K = a.K;
  if (threadIdx.x < BT_MAX_RANKS) home_cnt[threadIdx.x] = 0;  // units per home rank, over all items
  for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
    const int gp = it / tiles, r0 = (it % tiles) * RT;
    int p0, ntok;
    const uint8_t *wsrc, *ssrc, *bsrc;
    if (a.shared) {
      p0 = gp * PP;
      ntok = min(PP, a.n_shared - p0);
      wsrc = a.sh_down.w + (size_t)r0 * RB;
      ssrc = reinterpret_cast<const uint8_t*>(a.sh_down.s + (size_t)r0 * NG);
      bsrc = reinterpret_cast<const uint8_t*>(a.sh_down.b + (size_t)r0 * NG);
    } else {
      const int sidx = seg_of_pass(pl.first, pl.n_seg, gp);
      const int e = pl.seg_e[sidx];
      p0 = pl.off[sidx] + (gp - pl.first[sidx]) * PP;
      ntok = min(PP, (int)pl.off[sidx + 1] - p0);
      const int slot = a.slot_of ? a.slot_of[e] : e - a.e_lo;
      if (slot < 0 || slot >= a.n_slots) {
        if (threadIdx.x == 0) raise_error(a.err, YN_ERR_BAD_SLOT);
        continue;
      }
      const uint8_t* rec = a.base + (size_t)slot * (size_t)a.stride;
      wsrc = rec + a.rg.off[6] + (size_t)r0 * RB;
      ssrc = rec + a.rg.off[7] + (size_t)r0 * NG * 2;
      bsrc = rec + a.rg.off[8] + (size_t)r0 * NG * 2;
    }
    __syncthreads();
    cpa_rows_swz(Wt, 0, wsrc, RT, RB);
    cpa_rows(reinterpret_cast<uint8_t*>(Ss), srow_b, ssrc, RT, NG * 2);
    cpa_rows(reinterpret_cast<uint8_t*>(Bs), srow_b, bsrc, RT, NG * 2);
    cpa_block(XF, a.af + (size_t)p0 * xs, ntok * xs * 4);
    cpa_block(XG, a.ag + (size_t)p0 * gsd, ntok * gsd * 8);
    cpa_wait_all();
    __syncthreads();
    float acc[NCH][4];
#pragma unroll
    for (int t = 0; t < NCH; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
    warp_tile<BITS, GS, NCH>(Wt, RB, 16 * rs, Ss, Bs, srow_h, kh * cpw, cpw, XF, xs, XG, gsd, ntok, acc);
    float* rd = RED + (size_t)kh * RT * PP;
#pragma unroll
    for (int t = 0; t < NCH; ++t) {
      const int ra = 16 * rs + g, rb = ra + 8, tk = 8 * t + 2 * c;
      rd[ra * PP + tk] = acc[t][0];
      rd[ra * PP + tk + 1] = acc[t][1];
      rd[rb * PP + tk] = acc[t][2];
      rd[rb * PP + tk + 1] = acc[t][3];
    }
    __syncthreads();
    // 8 consecutive rows of one pair per thread (one 16-byte store)
    for (int i = threadIdx.x; i < ntok * (RT / 8); i += blockDim.x) {
      const int tok = i / (RT / 8), rr = (i % (RT / 8)) * 8;
      const float inv = XG[(size_t)tok * gsd + NG].x;
      uint32_t pk[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float v2[2];
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int r = rr + 2 * q + h2;
          const float v = __fmul_rn(__fadd_rn(RED[(size_t)r * PP + tok], RED[((size_t)RT + r) * PP + tok]), inv);
          v2[h2] = a.shared ? __fmul_rn(a.sgate[p0 + tok], bf16r(v)) : v;
        }
        pk[q] = (uint32_t)f32_to_bf16(v2[0]) | ((uint32_t)f32_to_bf16(v2[1]) << 16);
      }
      uint16_t* dst;
      if (a.shared) {
        dst = a.ysh + (size_t)(p0 + tok) * H + r0 + rr;
      } else {
        const int tj = pl.tj[p0 + tok], t = tj / K, j = tj % K;
        const int home = t / T_h, tl = t % T_h;
        dst = a.peers.y[home] + ((size_t)tl * K + j) * H + r0 + rr;
        if (rr == 0) atomicAdd(&home_cnt[home], 1);
      }
      *reinterpret_cast<uint4*>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  }
  // one release per CTA and home rank, after every item's stores
  if (!a.shared) {
    __syncthreads();  // every store of the CTA, then the releases (which cover them)
    if (threadIdx.x == 0)
      for (int h = 0; h < a.st.G; ++h)
        if (home_cnt[h]) red_release_sys_add_u64(a.peers.cnt[h], (unsigned long long)home_cnt[h]);
  }
}

// ------------------------------------------------------------ combine
// out = sum_j bf16(y_j * w_j) in column order (+ shared, + residual), as the
// single-row combine; starts once the rank's counter shows every (pair,
// row tile) unit of this layer.
#ifndef YN_NO_BATCH_EP_KERNELS
__global__ void __launch_bounds__(BT_THREADS) k_batch_combine(const CombineArgs a) {
  const unsigned long long target = ep_stamp(a.st) * a.per_layer;
  if (!wait_geq_block(a.cnt, target, a.st.err)) return;
  const int t = blockIdx.y;
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= a.H) return;
  const float* wr = a.w + (size_t)t * a.K;
  float acc = 0.0f;
  for (int j = 0; j < a.K; ++j) {
    const float y = bf16_to_f32(__ldcg(a.y + ((size_t)t * a.K + j) * a.H + r));
    acc = __fadd_rn(acc, bf16r(__fmul_rn(y, wr[j])));
  }
  float o = bf16r(acc);
  if (a.mode >= 1 && a.ysh) o = bf16r(__fadd_rn(o, bf16_to_f32(a.ysh[(size_t)t * a.H + r])));
  if (a.mode == 2) o = bf16r(__fadd_rn(bf16_to_f32(a.h_res[(size_t)t * a.H + r]), o));
  a.out[(size_t)t * a.H + r] = f32_to_bf16(o);
}
#endif  // YN_NO_BATCH_EP_KERNELS

#ifndef YN_NO_BATCH_EP_KERNELS
__global__ void k_ep_step_end(unsigned long long* epoch) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *epoch += 1ull;
}
#endif  // YN_NO_BATCH_EP_KERNELS

}  // namespace ynb
