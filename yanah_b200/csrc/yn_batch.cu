// C ABI of the union-of-experts batch path and of expert parallelism over
// peer memory (kernels in yn_batch.cuh).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>

#include "yanah_b200.h"
#include "yn_batch.cuh"
#include "yn_internal.h"

using namespace ynb;

#define YN_CUDA_B(call)                                                                              \
  do {                                                                                               \
    cudaError_t e_ = (call);                                                                         \
    if (e_ != cudaSuccess) return host_fail(YN_E_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

namespace {

cudaStream_t as_st(void* s) { return reinterpret_cast<cudaStream_t>(s); }
size_t a256(size_t v) { return (v + 255) / 256 * 256; }

// Largest sizes over the routed formats this path takes (2-bit g64, 4-bit
// g64 / g32) and the 8-bit dense format (g64 / g32).
int xs_max(int Kd) { return frag_stride_words(Kd, 4); }
int gsd_max(int Kd) { return gdata_stride(Kd, 32); }

struct SymLayout {
  size_t x_all, ids_all, flags, cnt, y, total;
};
struct LocalLayout {
  size_t err, counter, epoch, xf32, xsum, x_home, logits, ids, w, act_sh, sgate, plan, xf, xg, act, af, ag, sf, sg, ysh, total;
};

SymLayout sym_layout(const yn_dims& d, const yn_ep_config& c) {
  SymLayout L{};
  size_t o = 0;
  auto take = [&](size_t b) { size_t at = o; o = a256(o + b); return at; };
  const size_t R = (size_t)c.n_ranks * c.rows_per_rank;
  L.x_all = take(R * d.hidden * 2);
  L.ids_all = take(R * d.top_k * 4);
  L.flags = take((size_t)BT_MAX_RANKS * BT_MAX_DISPATCH * 8);
  L.cnt = take(8);
  L.y = take((size_t)c.rows_per_rank * d.top_k * d.hidden * 2);
  L.total = o;
  return L;
}

LocalLayout local_layout(const yn_dims& d, const yn_ep_config& c) {
  LocalLayout L{};
  size_t o = 0;
  auto take = [&](size_t b) { size_t at = o; o = a256(o + b); return at; };
  const size_t T = c.rows_per_rank, R = (size_t)c.n_ranks * c.rows_per_rank, P = R * d.top_k;
  const size_t H = d.hidden, E = d.n_experts, K = d.top_k, I = d.moe_inter;
  const size_t Ish = d.shared_inter ? d.shared_inter : 64;
  L.err = take(4);
  L.counter = take(8 * 4);
  L.epoch = take(8);
  L.xf32 = take(T * H * 4);
  L.xsum = take(T * (H / 16) * 4);
  L.x_home = take(T * H * 2);
  L.logits = take(T * E * 4);
  L.ids = take(T * K * 4);
  L.w = take(T * K * 4);
  L.act_sh = take(T * Ish * 2);
  L.sgate = take(T * 4);
  L.plan = take(sizeof(BatchPlan));
  L.xf = take(R * xs_max((int)H) * 4);
  L.xg = take(R * gsd_max((int)H) * 8);
  L.act = take(P * I * 2);
  L.af = take(P * xs_max((int)I) * 4);
  L.ag = take(P * gsd_max((int)I) * 8);
  L.sf = take(T * frag_stride_words((int)Ish, 8) * 4);
  L.sg = take(T * gdata_stride((int)Ish, 32) * 8);
  L.ysh = take(T * H * 2);
  L.total = o;
  return L;
}

int check_cfg(const yn_dims* d, const yn_ep_config* c) {
  if (!d || !c) return host_fail(YN_E_INVALID, "null dims or config");
  if (c->n_ranks < 1 || c->n_ranks > BT_MAX_RANKS) return host_fail(YN_E_UNSUPPORTED, "n_ranks must be in [1, 8]");
  if (c->rank < 0 || c->rank >= c->n_ranks) return host_fail(YN_E_INVALID, "rank outside [0, n_ranks)");
  if (c->rows_per_rank < 1 || c->rows_per_rank * c->n_ranks > BT_MAX_TOK)
    return host_fail(YN_E_UNSUPPORTED, "n_ranks * rows_per_rank must be in [1, 64]");
  if (c->n_layers < 1) return host_fail(YN_E_INVALID, "n_layers must be positive");
  if (d->top_k < 1 || d->top_k > BT_MAX_K) return host_fail(YN_E_UNSUPPORTED, "top_k must be in [1, 16]");
  if (d->hidden % 512 || d->hidden < 512 || d->hidden > 8192)
    return host_fail(YN_E_UNSUPPORTED, "hidden must be a multiple of 512 in [512, 8192]");
  if (d->moe_inter % 64 || d->moe_inter < 128) return host_fail(YN_E_UNSUPPORTED, "moe_inter must be a multiple of 64");
  if (d->shared_inter && (d->shared_inter % 128 || d->shared_inter < 256))
    return host_fail(YN_E_UNSUPPORTED, "shared_inter must be a multiple of 128 (>= 256)");
  if (d->n_experts < 1 || d->n_experts > 1024) return host_fail(YN_E_UNSUPPORTED, "n_experts must be in [1, 1024]");
  if (c->expert_lo < 0 || c->expert_hi > d->n_experts || c->expert_lo >= c->expert_hi)
    return host_fail(YN_E_INVALID, "expert range outside [0, n_experts)");
  return YN_OK;
}

template <typename K>
int occupancy_grid(K kernel, size_t smem, int* grid) {
  int dev = 0, sms = 0, per = 0;
  YN_CUDA_B(cudaGetDevice(&dev));
  YN_CUDA_B(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  YN_CUDA_B(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kernel, BT_THREADS, smem));
  *grid = sms * std::max(per, 1);
  return YN_OK;
}

size_t al16h(size_t v) { return (v + 15) / 16 * 16; }

// A vector of Kd codes split into `nks` warp slices: every slice must hold an
// even number of 16-byte chunks made of whole groups, and a row must span at
// least 8 chunks (the shared tile's XOR swizzle stays inside the row).
int check_split(int bits, int gs, int Kd, int nks, const char* what) {
  const int cpch = 128 / bits, nchunk = Kd / cpch;
  const bool ok = Kd % cpch == 0 && gs % cpch == 0 && nchunk % 8 == 0 && nchunk % (2 * nks) == 0 &&
                  (nchunk / nks) % (gs / cpch) == 0;
  if (!ok)
    return host_fail(YN_E_UNSUPPORTED, std::string("batch path: ") + what + " of " + std::to_string(Kd) + " " +
                                           std::to_string(bits) + "-bit codes (group " + std::to_string(gs) +
                                           ") does not split into the kernel's tiles");
  return YN_OK;
}

size_t up_smem(int bits, int gs, int nut, int H) {
  const size_t UR = 16 * nut, RB = (size_t)H * bits / 8, NG = H / gs;
  const size_t srow_b = al16h(NG * 2) + 16, NKS = 8 / nut;
  return 2 * UR * RB + 4 * UR * srow_b + 8 * (size_t)frag_stride_words(H, bits) * 4 + 8 * (size_t)gdata_stride(H, gs) * 8 +
         NKS * 2 * UR * 8 * 4;
}
size_t down_smem(int bits, int gs, int nch, int Kd) {
  const size_t RT = 64, RB = (size_t)Kd * bits / 8, NG = Kd / gs, PP = 8 * nch;
  const size_t srow_b = al16h(NG * 2) + 16;
  return RT * RB + 2 * RT * srow_b + PP * (size_t)frag_stride_words(Kd, bits) * 4 + PP * (size_t)gdata_stride(Kd, gs) * 8 +
         2 * RT * PP * 4;
}

constexpr int DOWN_NCH = 4;

template <int BITS, int GS>
int launch_frags(const FragArgs& a, int grid, cudaStream_t st) {
  k_batch_frags<BITS, GS><<<grid, BT_THREADS, 0, st>>>(a);
  YN_CUDA_B(cudaGetLastError());
  return YN_OK;
}

int frags(int bits, int gs, const FragArgs& a, int grid, cudaStream_t st) {
  if (bits == 2 && gs == 64) return launch_frags<2, 64>(a, grid, st);
  if (bits == 4 && gs == 64) return launch_frags<4, 64>(a, grid, st);
  if (bits == 4 && gs == 32) return launch_frags<4, 32>(a, grid, st);
  if (bits == 8 && gs == 64) return launch_frags<8, 64>(a, grid, st);
  if (bits == 8 && gs == 32) return launch_frags<8, 32>(a, grid, st);
  return host_fail(YN_E_UNSUPPORTED, "batch path: " + std::to_string(bits) + "-bit group " + std::to_string(gs));
}

template <int BITS, int GS>
int launch_prep(const FragArgs& a, int grid, cudaStream_t st) {
  k_batch_prep<BITS, GS><<<grid, BT_THREADS, 0, st>>>(a);
  YN_CUDA_B(cudaGetLastError());
  return YN_OK;
}

int prep(int bits, int gs, const FragArgs& a, int grid, cudaStream_t st) {
  if (bits == 2 && gs == 64) return launch_prep<2, 64>(a, grid, st);
  if (bits == 4 && gs == 64) return launch_prep<4, 64>(a, grid, st);
  if (bits == 4 && gs == 32) return launch_prep<4, 32>(a, grid, st);
  return host_fail(YN_E_UNSUPPORTED, "batch path: routed " + std::to_string(bits) + "-bit group " + std::to_string(gs));
}

template <int BITS, int GS, int NUT>
int launch_up(const BatchUpArgs& a, cudaStream_t st) {
  const size_t smem = up_smem(BITS, GS, NUT, a.H);
  int rc = host_set_smem(reinterpret_cast<const void*>(k_batch_up<BITS, GS, NUT>), smem);
  if (rc) return rc;
  int grid = 0;
  if ((rc = occupancy_grid(k_batch_up<BITS, GS, NUT>, smem, &grid))) return rc;
  k_batch_up<BITS, GS, NUT><<<grid, BT_THREADS, smem, st>>>(a);
  YN_CUDA_B(cudaGetLastError());
  return YN_OK;
}

int up(int bits, int gs, const BatchUpArgs& a, cudaStream_t st) {
  if (bits == 2 && gs == 64) return launch_up<2, 64, 2>(a, st);
  if (bits == 4 && gs == 64) return launch_up<4, 64, 1>(a, st);
  if (bits == 4 && gs == 32) return launch_up<4, 32, 1>(a, st);
  return host_fail(YN_E_UNSUPPORTED, "batch path: routed " + std::to_string(bits) + "-bit group " + std::to_string(gs));
}

template <int BITS, int GS>
int launch_down(const BatchDownArgs& a, int Kd, int max_items, cudaStream_t st) {
  const size_t smem = down_smem(BITS, GS, DOWN_NCH, Kd);
  int rc = host_set_smem(reinterpret_cast<const void*>(k_batch_down<BITS, GS, DOWN_NCH>), smem);
  if (rc) return rc;
  int grid = 0;
  if ((rc = occupancy_grid(k_batch_down<BITS, GS, DOWN_NCH>, smem, &grid))) return rc;
  grid = std::max(1, std::min(grid, max_items));
  k_batch_down<BITS, GS, DOWN_NCH><<<grid, BT_THREADS, smem, st>>>(a);
  YN_CUDA_B(cudaGetLastError());
  return YN_OK;
}

int down(int bits, int gs, const BatchDownArgs& a, int Kd, int max_items, cudaStream_t st) {
  if (bits == 2 && gs == 64) return launch_down<2, 64>(a, Kd, max_items, st);
  if (bits == 4 && gs == 64) return launch_down<4, 64>(a, Kd, max_items, st);
  if (bits == 4 && gs == 32) return launch_down<4, 32>(a, Kd, max_items, st);
  if (bits == 8 && gs == 64) return launch_down<8, 64>(a, Kd, max_items, st);
  if (bits == 8 && gs == 32) return launch_down<8, 32>(a, Kd, max_items, st);
  return host_fail(YN_E_UNSUPPORTED, "batch path: down " + std::to_string(bits) + "-bit group " + std::to_string(gs));
}

RecGeom to_rg(const yn_record& r) {
  RecGeom g;
  for (int i = 0; i < 9; ++i) g.off[i] = r.piece_offset[i];
  g.bytes = r.record_bytes;
  g.bits = r.bits;
  g.gs = r.group_size;
  return g;
}

QM to_q(const yn_qmat& m) {
  QM q;
  q.w = reinterpret_cast<const uint8_t*>(m.weight);
  q.s = reinterpret_cast<const uint16_t*>(m.scales);
  q.b = reinterpret_cast<const uint16_t*>(m.biases);
  q.rows = m.rows;
  q.cols = m.cols;
  q.bits = m.bits;
  q.gs = m.group_size;
  return q;
}

}  // namespace

// ---------------------------------------------------------------- sizes
extern "C" size_t yn_ep_sym_bytes(const yn_dims* dims, const yn_ep_config* cfg) {
  if (check_cfg(dims, cfg)) return 0;
  return sym_layout(*dims, *cfg).total;
}

extern "C" size_t yn_ep_local_bytes(const yn_dims* dims, const yn_ep_config* cfg) {
  if (check_cfg(dims, cfg)) return 0;
  return local_layout(*dims, *cfg).total;
}

extern "C" int yn_ep_init(void* sym, void* local, const yn_dims* dims, const yn_ep_config* cfg, void* stream) {
  int rc = check_cfg(dims, cfg);
  if (rc) return rc;
  if (!sym || !local) return host_fail(YN_E_INVALID, "null buffer");
  YN_CUDA_B(cudaMemsetAsync(sym, 0, sym_layout(*dims, *cfg).total, as_st(stream)));
  YN_CUDA_B(cudaMemsetAsync(local, 0, local_layout(*dims, *cfg).total, as_st(stream)));
  return YN_OK;
}

extern "C" int yn_ep_view(void* local, const yn_dims* dims, const yn_ep_config* cfg, yn_ep_local_ptrs* out) {
  int rc = check_cfg(dims, cfg);
  if (rc) return rc;
  if (!local || !out) return host_fail(YN_E_INVALID, "null argument");
  const LocalLayout L = local_layout(*dims, *cfg);
  uint8_t* b = reinterpret_cast<uint8_t*>(local);
  out->x = b + L.x_home;
  out->ids = reinterpret_cast<int32_t*>(b + L.ids);
  out->weights = reinterpret_cast<float*>(b + L.w);
  out->act_sh = b + L.act_sh;
  out->sgate = reinterpret_cast<float*>(b + L.sgate);
  out->y_shared = b + L.ysh;
  out->error = reinterpret_cast<int32_t*>(b + L.err);
  out->epoch = reinterpret_cast<uint64_t*>(b + L.epoch);
  return YN_OK;
}

extern "C" int yn_ep_sym_view(void* sym, const yn_dims* dims, const yn_ep_config* cfg, yn_ep_sym_ptrs* out) {
  int rc = check_cfg(dims, cfg);
  if (rc) return rc;
  if (!sym || !out) return host_fail(YN_E_INVALID, "null argument");
  const SymLayout S = sym_layout(*dims, *cfg);
  uint8_t* b = reinterpret_cast<uint8_t*>(sym);
  out->x_all = b + S.x_all;
  out->ids_all = reinterpret_cast<int32_t*>(b + S.ids_all);
  out->y = b + S.y;
  out->flags = reinterpret_cast<uint64_t*>(b + S.flags);
  out->counter = reinterpret_cast<uint64_t*>(b + S.cnt);
  return YN_OK;
}

// ---------------------------------------------------------------- layer
extern "C" int yn_ep_layer(const yn_dims* dims, const yn_layer* layer, int32_t layer_index, const yn_ep_config* cfg,
                           const void* h_in, void* h_out, void* const* peer_sym, void* local, void* stream) {
  int rc = check_cfg(dims, cfg);
  if (rc) return rc;
  if (!layer || !h_in || !h_out || !peer_sym || !local) return host_fail(YN_E_INVALID, "null argument");
  if (layer_index < 0 || layer_index >= cfg->n_layers) return host_fail(YN_E_INVALID, "layer_index outside [0, n_layers)");
  const yn_dims& d = *dims;
  const yn_layer& Ly = *layer;
  const yn_record& rec = Ly.record;
  const int G = cfg->n_ranks, T_h = cfg->rows_per_rank, R = G * T_h, H = d.hidden, K = d.top_k, I = d.moe_inter;
  const int bits = rec.bits, gs = rec.group_size;
  if (!((bits == 2 && gs == 64) || (bits == 4 && (gs == 64 || gs == 32))))
    return host_fail(YN_E_UNSUPPORTED, "batch path: routed experts must be 2-bit g64 or 4-bit g64/g32");
  if (!Ly.expert_base) return host_fail(YN_E_INVALID, "expert_base is null");
  if (reinterpret_cast<uintptr_t>(Ly.expert_base) % 16 || Ly.slot_stride % 16)
    return host_fail(YN_E_INVALID, "expert arena and slot stride must be 16-byte aligned");
  for (int i = 0; i < 9; ++i)
    if (rec.piece_offset[i] % 16) return host_fail(YN_E_INVALID, "record pieces must be 16-byte aligned");
  const bool sh = d.shared_inter > 0;
  if (sh) {
    if ((rc = host_check_qmat(Ly.shared_down, H, d.shared_inter, 8, "shared_down"))) return rc;
    if (Ly.shared_down.group_size != 64 && Ly.shared_down.group_size != 32)
      return host_fail(YN_E_UNSUPPORTED, "shared_down group size must be 32 or 64");
    if ((rc = check_split(8, Ly.shared_down.group_size, d.shared_inter, 2, "shared down input"))) return rc;
  }
  if ((rc = check_split(bits, gs, H, bits == 2 ? 4 : 8, "gate/up input"))) return rc;
  if ((rc = check_split(bits, gs, I, 2, "down input"))) return rc;
  if (I % (bits == 2 ? 32 : 16)) return host_fail(YN_E_UNSUPPORTED, "moe_inter must be a multiple of 32");
  for (int r = 0; r < G; ++r)
    if (!peer_sym[r]) return host_fail(YN_E_INVALID, "peer buffer " + std::to_string(r) + " is null");
  cudaStream_t st = as_st(stream);
  const SymLayout S = sym_layout(d, *cfg);
  const LocalLayout L = local_layout(d, *cfg);
  uint8_t* lb = reinterpret_cast<uint8_t*>(local);
  int* err = reinterpret_cast<int*>(lb + L.err);

  EpStep es{};
  es.rank = cfg->rank;
  es.G = G;
  es.T_h = T_h;
  es.L = cfg->n_layers;
  es.layer = layer_index;
  es.epoch = reinterpret_cast<const unsigned long long*>(lb + L.epoch);
  es.err = err;
  EpPeers peers{};
  for (int r = 0; r < G; ++r) {
    uint8_t* b = reinterpret_cast<uint8_t*>(peer_sym[r]);
    peers.x_all[r] = reinterpret_cast<uint16_t*>(b + S.x_all);
    peers.ids_all[r] = reinterpret_cast<int32_t*>(b + S.ids_all);
    peers.flag[r] = reinterpret_cast<unsigned long long*>(b + S.flags);
    peers.y[r] = reinterpret_cast<uint16_t*>(b + S.y);
    peers.cnt[r] = reinterpret_cast<unsigned long long*>(b + S.cnt);
  }

  // dispatch CTAs per destination (the same on every rank: same T_h and H)
  const int n_disp = std::max(1, std::min(BT_MAX_DISPATCH, (T_h * H / 8 + BT_THREADS * 4 - 1) / (BT_THREADS * 4)));

  // 1. post-attention + routing of the home rows
  PostAttnOut pa{};
  pa.x = reinterpret_cast<uint16_t*>(lb + L.x_home);
  pa.logits = reinterpret_cast<float*>(lb + L.logits);
  pa.act_sh = reinterpret_cast<uint16_t*>(lb + L.act_sh);
  pa.sgate = reinterpret_cast<float*>(lb + L.sgate);
  pa.ids = reinterpret_cast<int32_t*>(lb + L.ids);
  pa.wts = reinterpret_cast<float*>(lb + L.w);
  pa.err = err;
  pa.xf32 = reinterpret_cast<float*>(lb + L.xf32);
  pa.xsum = reinterpret_cast<float*>(lb + L.xsum);
  if ((rc = host_batch_dense(d, Ly, h_in, T_h, pa, reinterpret_cast<unsigned*>(lb + L.counter), st))) return rc;

  // 2. home rows -> every rank's gather buffer
  {
    DispatchArgs a{};
    a.st = es;
    a.peers = peers;
    a.x_home = pa.x;
    a.ids_home = pa.ids;
    a.H = H;
    a.K = K;
    k_ep_dispatch<<<dim3(G, n_disp), BT_THREADS, 0, st>>>(a);
    YN_CUDA_B(cudaGetLastError());
  }

  // 3. shared expert down projection of the home rows (local)
  uint16_t* ysh = reinterpret_cast<uint16_t*>(lb + L.ysh);
  if (sh) {
    const int dgs = Ly.shared_down.group_size;
    FragArgs f{};
    f.src = pa.act_sh;
    f.src_stride = d.shared_inter;
    f.n_rows = T_h;
    f.Kd = d.shared_inter;
    f.xf = reinterpret_cast<uint32_t*>(lb + L.sf);
    f.xg = reinterpret_cast<float2*>(lb + L.sg);
    f.st = es;
    if ((rc = frags(8, dgs, f, T_h, st))) return rc;
    BatchDownArgs a{};
    a.shared = 1;
    a.n_shared = T_h;
    a.af = f.xf;
    a.ag = f.xg;
    a.af_stride = frag_stride_words(d.shared_inter, 8);
    a.ag_stride = gdata_stride(d.shared_inter, dgs);
    a.sh_down = to_q(Ly.shared_down);
    a.H = H;
    a.I = I;
    a.K = K;
    a.st = es;
    a.ysh = ysh;
    a.sgate = pa.sgate;
    a.err = err;
    if ((rc = down(8, dgs, a, d.shared_inter, ((T_h + BT_DN_PASS - 1) / BT_DN_PASS) * (H / 64), st))) return rc;
  }

  // 4. wait for every rank's rows, plan the local experts, x fragments
  BatchPlan* plan = reinterpret_cast<BatchPlan*>(lb + L.plan);
  const int xs = frag_stride_words(H, bits), gsd = gdata_stride(H, gs);
  {
    FragArgs f{};
    f.src = peers.x_all[cfg->rank];
    f.src_stride = H;
    f.n_rows = R;
    f.Kd = H;
    f.xf = reinterpret_cast<uint32_t*>(lb + L.xf);
    f.xg = reinterpret_cast<float2*>(lb + L.xg);
    f.st = es;
    f.flags = peers.flag[cfg->rank];
    f.n_dispatch = n_disp;
    f.ids = peers.ids_all[cfg->rank];
    f.K = K;
    f.E = d.n_experts;
    f.e_lo = cfg->expert_lo;
    f.e_hi = cfg->expert_hi;
    f.plan = plan;
    if ((rc = prep(bits, gs, f, 1 + R, st))) return rc;
  }

  // 5. gate/up + SwiGLU of the local pairs
  uint16_t* act = reinterpret_cast<uint16_t*>(lb + L.act);
  {
    BatchUpArgs a{};
    a.plan = plan;
    a.xf = reinterpret_cast<const uint32_t*>(lb + L.xf);
    a.xg = reinterpret_cast<const float2*>(lb + L.xg);
    a.xf_stride = xs;
    a.xg_stride = gsd;
    a.base = reinterpret_cast<const uint8_t*>(Ly.expert_base);
    a.stride = Ly.slot_stride;
    a.slot_of = Ly.expert_slot;
    a.n_slots = Ly.n_slots;
    a.e_lo = cfg->expert_lo;
    a.rg = to_rg(rec);
    a.H = H;
    a.I = I;
    a.K = K;
    a.act = act;
    a.err = err;
    if ((rc = up(bits, gs, a, st))) return rc;
  }

  // 6. activation fragments, down projections into the home ranks' buffers
  {
    FragArgs f{};
    f.src = act;
    f.src_stride = I;
    f.n_rows = R * K;
    f.n_rows_dev = &plan->n_pairs;
    f.Kd = I;
    f.xf = reinterpret_cast<uint32_t*>(lb + L.af);
    f.xg = reinterpret_cast<float2*>(lb + L.ag);
    f.st = es;
    if ((rc = frags(bits, gs, f, R * K, st))) return rc;
    BatchDownArgs a{};
    a.plan = plan;
    a.af = f.xf;
    a.ag = f.xg;
    a.af_stride = frag_stride_words(I, bits);
    a.ag_stride = gdata_stride(I, gs);
    a.base = reinterpret_cast<const uint8_t*>(Ly.expert_base);
    a.stride = Ly.slot_stride;
    a.slot_of = Ly.expert_slot;
    a.n_slots = Ly.n_slots;
    a.e_lo = cfg->expert_lo;
    a.rg = to_rg(rec);
    a.H = H;
    a.I = I;
    a.K = K;
    a.st = es;
    a.peers = peers;
    a.err = err;
    const int max_pass = std::min(cfg->expert_hi - cfg->expert_lo, R * K) + (R * K) / BT_DN_PASS;
    if ((rc = down(bits, gs, a, I, max_pass * (H / 64), st))) return rc;
  }

  // 7. combine of the home rows once every unit has landed
  {
    CombineArgs a{};
    a.st = es;
    a.cnt = peers.cnt[cfg->rank];
    a.per_layer = (unsigned long long)T_h * K * (H / 64);
    a.y = peers.y[cfg->rank];
    a.w = pa.wts;
    a.ysh = sh ? ysh : nullptr;
    a.h_res = reinterpret_cast<const uint16_t*>(h_in);
    a.out = reinterpret_cast<uint16_t*>(h_out);
    a.H = H;
    a.K = K;
    a.mode = 2;
    dim3 grid((H + BT_THREADS - 1) / BT_THREADS, T_h);
    k_batch_combine<<<grid, BT_THREADS, 0, st>>>(a);
    YN_CUDA_B(cudaGetLastError());
  }
  return YN_OK;
}

extern "C" int yn_ep_step_end(void* local, const yn_dims* dims, const yn_ep_config* cfg, void* stream) {
  int rc = check_cfg(dims, cfg);
  if (rc) return rc;
  if (!local) return host_fail(YN_E_INVALID, "null buffer");
  const LocalLayout L = local_layout(*dims, *cfg);
  k_ep_step_end<<<1, 32, 0, as_st(stream)>>>(
      reinterpret_cast<unsigned long long*>(reinterpret_cast<uint8_t*>(local) + L.epoch));
  YN_CUDA_B(cudaGetLastError());
  return YN_OK;
}

extern "C" int yn_ep_error(void* local, const yn_dims* dims, const yn_ep_config* cfg, void* stream, int32_t* code_out) {
  int rc = check_cfg(dims, cfg);
  if (rc) return rc;
  if (!local || !code_out) return host_fail(YN_E_INVALID, "null argument");
  const LocalLayout L = local_layout(*dims, *cfg);
  int32_t* e = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(local) + L.err);
  YN_CUDA_B(cudaMemcpyAsync(code_out, e, 4, cudaMemcpyDeviceToHost, as_st(stream)));
  YN_CUDA_B(cudaStreamSynchronize(as_st(stream)));
  YN_CUDA_B(cudaMemsetAsync(e, 0, 4, as_st(stream)));
  YN_CUDA_B(cudaStreamSynchronize(as_st(stream)));
  return YN_OK;
}

// ----------------------------------------------------------- peer memory
extern "C" int yn_device_alloc(size_t bytes, void** ptr) {
  if (!ptr || !bytes) return host_fail(YN_E_INVALID, "null pointer or zero size");
  YN_CUDA_B(cudaMalloc(ptr, bytes));
  return YN_OK;
}

extern "C" int yn_device_free(void* ptr) {
  if (ptr) YN_CUDA_B(cudaFree(ptr));
  return YN_OK;
}

extern "C" int yn_ipc_export(const void* dev_ptr, void* handle_out) {
  if (!dev_ptr || !handle_out) return host_fail(YN_E_INVALID, "null argument");
  cudaIpcMemHandle_t h;
  YN_CUDA_B(cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)));
  static_assert(sizeof(h) == YN_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  return YN_OK;
}

extern "C" int yn_ipc_import(const void* handle, void** dev_ptr_out) {
  if (!handle || !dev_ptr_out) return host_fail(YN_E_INVALID, "null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  YN_CUDA_B(cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess));
  return YN_OK;
}

extern "C" int yn_ipc_close(void* dev_ptr) {
  if (dev_ptr) YN_CUDA_B(cudaIpcCloseMemHandle(dev_ptr));
  return YN_OK;
}

extern "C" int yn_memcpy(void* dst, const void* src, size_t bytes, void* stream) {
  if (!bytes) return YN_OK;
  if (!dst || !src) return host_fail(YN_E_INVALID, "null argument");
  YN_CUDA_B(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, as_st(stream)));
  YN_CUDA_B(cudaStreamSynchronize(as_st(stream)));
  return YN_OK;
}

extern "C" int yn_memcpy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (!bytes) return YN_OK;
  if (!dst || !src) return host_fail(YN_E_INVALID, "null argument");
  YN_CUDA_B(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, as_st(stream)));
  return YN_OK;
}
