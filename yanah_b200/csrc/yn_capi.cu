// extern "C" entry points of libyanah_b200.so (declared in include/yanah_b200.h).
//
// Host-side responsibilities: validate shapes and alignment, choose tile
// sizes (about 40 KB of weights per CTA so every phase keeps its bytes in
// flight), dispatch the template instantiation that matches the layer's bit
// widths and row lengths, and carve the caller's workspace. Nothing here
// allocates device memory.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <string>
#include <utility>
#include <vector>
#include <algorithm>

#include "yn_common.cuh"
#include "yn_moe.cuh"
#include "yn_qdot.cuh"
#include "yn_kernels.cuh"
#include "yn_flow.cuh"
#include "yn_batch_dense.cuh"
#include "yn_internal.h"


using namespace ynb;

// ------------------------------------------------------------------ errors
static thread_local std::string g_err;
static int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}
int ynb::host_fail(int code, const std::string& msg) { return fail(code, msg); }
#define YN_CUDA(call)                                                                         \
  do {                                                                                        \
    cudaError_t e_ = (call);                                                                  \
    if (e_ != cudaSuccess) return fail(YN_E_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

extern "C" const char* yn_last_error(void) { return g_err.c_str(); }
extern "C" const char* yn_version(void) { return "yanah_b200 0.1 (sm_100a)"; }

// --------------------------------------------------------------- helpers
static cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

static QM to_qm(const yn_qmat& m) {
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

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int check_qmat(const yn_qmat& m, int rows, int cols, int bits, const char* what) {
  if (!m.weight || !m.scales || !m.biases) return fail(YN_E_INVALID, std::string(what) + ": null pointer");
  if (m.rows != rows || m.cols != cols)
    return fail(YN_E_INVALID, std::string(what) + ": shape " + std::to_string(m.rows) + "x" + std::to_string(m.cols) +
                                  ", expected " + std::to_string(rows) + "x" + std::to_string(cols));
  if (bits && m.bits != bits)
    return fail(YN_E_UNSUPPORTED, std::string(what) + ": " + std::to_string(m.bits) + "-bit not supported here");
  if (m.group_size < 16 || (m.group_size & (m.group_size - 1)) || cols % m.group_size)
    return fail(YN_E_UNSUPPORTED, std::string(what) + ": group size " + std::to_string(m.group_size));
  if ((cols * m.bits / 8) % 16) return fail(YN_E_UNSUPPORTED, std::string(what) + ": row bytes not a multiple of 16");
  if (!aligned16(m.weight) || !aligned16(m.scales) || !aligned16(m.biases))
    return fail(YN_E_INVALID, std::string(what) + ": pointers must be 16-byte aligned");
  return YN_OK;
}

static int lanes(int rowbytes) { return lanes_per_row(rowbytes); }
static int cpl_of(int rowbytes) { return (rowbytes / 16) / lanes(rowbytes); }

// Rows per tile: the largest power of two R <= limit dividing n whose tile
// stays under the budget, preferring R whose scale block (R * scale_row_bytes)
// is a multiple of 16 bytes so that every piece can use the bulk engine.
static int pick_rows(int n, int limit, size_t row_bytes, size_t scale_row_bytes) {
  const size_t budget = 40 * 1024;
  int best_aligned = 0, best_any = 1;
  for (int R = 1; R <= limit && R <= n; R *= 2) {
    if (n % R) continue;
    if (R > 1 && (size_t)R * row_bytes > budget) break;
    best_any = R;
    if (((size_t)R * scale_row_bytes) % 16 == 0) best_aligned = R;
  }
  return best_aligned ? best_aligned : best_any;
}

// Raise the dynamic shared-memory limit of a kernel once per device (the
// first call must come before any stream capture that launches it).
template <typename K>
static int set_smem(K kernel, size_t bytes);
static int set_smem_ptr(const void* kernel, size_t bytes);
template <typename K>
static int set_smem(K kernel, size_t bytes) { return set_smem_ptr(reinterpret_cast<const void*>(kernel), bytes); }
static int set_smem_ptr(const void* kernel, size_t bytes) {
  if (bytes > 227 * 1024) return fail(YN_E_UNSUPPORTED, "tile needs " + std::to_string(bytes) + " B of shared memory");
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(kernel, dev);
  if (done.count(key)) return YN_OK;
  int optin = 0;
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
  if (e != cudaSuccess) return fail(YN_E_CUDA, std::string("cudaFuncGetAttributes: ") + cudaGetErrorString(e));
  const int avail = optin - (int)fa.sharedSizeBytes;
  if ((int)bytes > avail) return fail(YN_E_UNSUPPORTED, "kernel needs " + std::to_string(bytes) + " B of shared memory, " +
                                                            std::to_string(avail) + " available");
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, avail);
  if (e != cudaSuccess) return fail(YN_E_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  done.insert(key);
  return YN_OK;
}

int ynb::host_check_qmat(const yn_qmat& m, int rows, int cols, int bits, const char* what) {
  return check_qmat(m, rows, cols, bits, what);
}
int ynb::host_set_smem(const void* kernel, size_t bytes) { return set_smem_ptr(kernel, bytes); }

static RecGeom rec_geom(const yn_record& r) {
  RecGeom g;
  for (int i = 0; i < 9; ++i) g.off[i] = r.piece_offset[i];
  g.bytes = r.record_bytes;
  g.bits = r.bits;
  g.gs = r.group_size;
  return g;
}

static int check_dims(const yn_dims* d, int T) {
  if (!d) return fail(YN_E_INVALID, "dims is null");
  if (T < 1 || T > YN_MAX_ROWS) return fail(YN_E_UNSUPPORTED, "rows T must be in [1, " + std::to_string(YN_MAX_ROWS) + "]");
  if (d->hidden < 128 || d->hidden % 128) return fail(YN_E_UNSUPPORTED, "hidden must be a multiple of 128");
  if (d->n_experts < 1 || d->n_experts > 1024) return fail(YN_E_UNSUPPORTED, "n_experts must be in [1, 1024]");
  if (d->top_k < 1 || d->top_k > 16 || d->top_k > d->n_experts) return fail(YN_E_UNSUPPORTED, "top_k must be in [1, 16]");
  if (d->moe_inter < 64 || d->moe_inter % 64) return fail(YN_E_UNSUPPORTED, "moe_inter must be a multiple of 64");
  if (d->shared_inter < 0 || d->shared_inter % 64) return fail(YN_E_UNSUPPORTED, "shared_inter must be a multiple of 64");
  int cbr = d->hidden < CB_ROWS ? d->hidden : CB_ROWS;
  if (d->hidden % cbr) return fail(YN_E_UNSUPPORTED, "hidden must be a multiple of 256 (or below 256)");
  return YN_OK;
}

// ------------------------------------------------------------- workspace
extern "C" size_t yn_workspace_bytes(const yn_dims* dims) {
  if (!dims) return 0;
  return ws_layout(*dims).total;
}

extern "C" int yn_workspace_init(void* ws, size_t ws_bytes, const yn_dims* dims, void* stream) {
  int rc = check_dims(dims, 1);
  if (rc) return rc;
  WsLayout L = ws_layout(*dims);
  if (!ws || ws_bytes < L.total) return fail(YN_E_INVALID, "workspace too small");
  YN_CUDA(cudaMemsetAsync(ws, 0, L.total, as_stream(stream)));
  return YN_OK;
}

extern "C" int yn_workspace_view(void* ws, const yn_dims* dims, yn_ws_view* out) {
  int rc = check_dims(dims, 1);
  if (rc) return rc;
  if (!ws || !out) return fail(YN_E_INVALID, "null workspace or view");
  WsLayout L = ws_layout(*dims);
  uint8_t* b = reinterpret_cast<uint8_t*>(ws);
  out->x = b + L.x;
  out->logits = reinterpret_cast<float*>(b + L.logits);
  out->ids = reinterpret_cast<int32_t*>(b + L.ids);
  out->weights = reinterpret_cast<float*>(b + L.w);
  out->fprobs = reinterpret_cast<float*>(b + L.fprobs);
  out->act = b + L.act;
  out->act_sh = b + L.act_sh;
  out->sgate = reinterpret_cast<float*>(b + L.sgate);
  out->y = b + L.y;
  out->y_shared = b + L.y + (size_t)YN_MAX_ROWS * dims->top_k * dims->hidden * 2;
  out->flogits = reinterpret_cast<float*>(b + L.flogits);
  out->error = reinterpret_cast<int32_t*>(b + L.err);
  return YN_OK;
}

extern "C" int yn_workspace_error(void* ws, const yn_dims* dims, void* stream, int32_t* code_out) {
  if (!ws || !dims) return fail(YN_E_INVALID, "null argument");
  WsLayout L = ws_layout(*dims);
  int32_t code = 0;
  uint8_t* b = reinterpret_cast<uint8_t*>(ws);
  YN_CUDA(cudaMemcpyAsync(&code, b + L.err, 4, cudaMemcpyDeviceToHost, as_stream(stream)));
  YN_CUDA(cudaStreamSynchronize(as_stream(stream)));
  if (code) YN_CUDA(cudaMemsetAsync(b + L.err, 0, 4, as_stream(stream)));
  if (code_out) *code_out = code;
  return code ? fail(YN_E_DEVICE, "kernel error code " + std::to_string(code)) : YN_OK;
}

// ----------------------------------------------------------- standalone
extern "C" int yn_dequantize(const yn_qmat* m, float* out, void* stream) {
  if (!m || !out) return fail(YN_E_INVALID, "null argument");
  int rc = check_qmat(*m, m->rows, m->cols, 0, "yn_dequantize");
  if (rc) return rc;
  const size_t n = (size_t)m->rows * m->cols;
  const int threads = 256;
  const int blocks = (int)((n + threads - 1) / threads < 148 * 16 ? (n + threads - 1) / threads : 148 * 16);
  auto w = reinterpret_cast<const uint32_t*>(m->weight);
  auto s = reinterpret_cast<const uint16_t*>(m->scales);
  auto b = reinterpret_cast<const uint16_t*>(m->biases);
  switch (m->bits) {
    case 2: k_dequant<2><<<blocks, threads, 0, as_stream(stream)>>>(w, s, b, m->rows, m->cols, m->group_size, out); break;
    case 4: k_dequant<4><<<blocks, threads, 0, as_stream(stream)>>>(w, s, b, m->rows, m->cols, m->group_size, out); break;
    case 8: k_dequant<8><<<blocks, threads, 0, as_stream(stream)>>>(w, s, b, m->rows, m->cols, m->group_size, out); break;
    default: return fail(YN_E_UNSUPPORTED, "bits must be 2, 4 or 8");
  }
  YN_CUDA(cudaGetLastError());
  return YN_OK;
}

extern "C" int yn_qlinear(const yn_qmat* m, const void* x, int32_t T, float* y, void* stream) {
  if (!m || !x || !y) return fail(YN_E_INVALID, "null argument");
  if (T < 1 || T > YN_MAX_ROWS) return fail(YN_E_UNSUPPORTED, "T out of range");
  int rc = check_qmat(*m, m->rows, m->cols, 8, "yn_qlinear");
  if (rc) return rc;
  const int rb = m->cols;
  const int lpr = lanes(rb), rpi = 32 / lpr, cpl = cpl_of(rb);
  const int rows_per_cta = 4 * rpi;
  const int grid = (m->rows + rows_per_cta - 1) / rows_per_cta;
  const size_t smem = (size_t)T * m->cols * 2;
  QM q = to_qm(*m);
  auto xx = reinterpret_cast<const uint16_t*>(x);
  switch (cpl) {
#define QL(C)                                                                       \
  case C:                                                                           \
    if ((rc = set_smem(k_qlinear8<C>, smem))) return rc;                            \
    k_qlinear8<C><<<grid, THREADS, smem, as_stream(stream)>>>(q, xx, T, y);         \
    break;
    QL(1) QL(2) QL(3) QL(4) QL(8)
#undef QL
    default: return fail(YN_E_UNSUPPORTED, "row length not supported");
  }
  YN_CUDA(cudaGetLastError());
  return YN_OK;
}

extern "C" int yn_route(const float* logits, int32_t T, const yn_dims* dims, int32_t* ids, float* weights,
                        void* stream) {
  if (!logits || !dims || !ids || !weights) return fail(YN_E_INVALID, "null argument");
  if (dims->n_experts < 1 || dims->n_experts > 1024) return fail(YN_E_UNSUPPORTED, "n_experts must be in [1, 1024]");
  if (dims->top_k < 1 || dims->top_k > 16 || dims->top_k > dims->n_experts) return fail(YN_E_UNSUPPORTED, "top_k out of range");
  if (T < 1) return fail(YN_E_INVALID, "T must be >= 1");
  const int warps = 4;
  k_route<<<(T + warps - 1) / warps, warps * 32, 0, as_stream(stream)>>>(logits, T, dims->n_experts, dims->top_k,
                                                                           dims->norm_topk, ids, weights);
  YN_CUDA(cudaGetLastError());
  return YN_OK;
}

// -------------------------------------------------------- layer kernels
static int launch_post_attention_out(const yn_dims& d, const yn_layer& L, const void* h1, int T, const yn_layer* tg,
                                     int NT, const PostAttnOut& o, cudaStream_t st) {
  int rc;
  const int H = d.hidden, E = d.n_experts;
  if (!h1 || !L.post_norm) return fail(YN_E_INVALID, "post_attention: null input or norm");
  if ((rc = check_qmat(L.router, E, H, 8, "router"))) return rc;
  const bool sh = d.shared_inter > 0;
  if (sh) {
    if ((rc = check_qmat(L.shared_gate, d.shared_inter, H, 8, "shared_gate"))) return rc;
    if ((rc = check_qmat(L.shared_up, d.shared_inter, H, 8, "shared_up"))) return rc;
    if ((rc = check_qmat(L.shared_expert_gate, 1, H, 8, "shared_expert_gate"))) return rc;
  }
  if (NT < 0 || NT > YN_MAX_TARGETS) return fail(YN_E_UNSUPPORTED, "at most 2 lookahead targets");
  PostAttnArgs a{};
  a.T = T; a.H = H; a.E = E; a.K = d.top_k; a.Ish = d.shared_inter; a.norm_topk = d.norm_topk; a.eps = d.rms_eps;
  a.h1 = reinterpret_cast<const uint16_t*>(h1);
  a.norm = reinterpret_cast<const uint16_t*>(L.post_norm);
  a.router = to_qm(L.router);
  a.rbias = L.router_bias;
  a.has_shared = sh;
  if (sh) {
    a.sh_gate = to_qm(L.shared_gate);
    a.sh_up = to_qm(L.shared_up);
    a.sg = to_qm(L.shared_expert_gate);
  }
  a.n_targets = NT;
  for (int g = 0; g < NT; ++g) {
    if ((rc = check_qmat(tg[g].router, E, H, 8, "target router"))) return rc;
    if (!tg[g].post_norm) return fail(YN_E_INVALID, "target norm is null");
    a.tnorm[g] = reinterpret_cast<const uint16_t*>(tg[g].post_norm);
    a.trouter[g] = to_qm(tg[g].router);
    a.tbias[g] = tg[g].router_bias;
  }
  const size_t rowb = (size_t)H + 2 * (size_t)(H / L.router.group_size) * 2;
  const size_t srow = (size_t)(H / L.router.group_size) * 2;
  a.r_router = pick_rows(E, 64, rowb, srow);
  a.nt_router = E / a.r_router;
  if (sh) {
    const size_t srow_s = (size_t)(H / L.shared_gate.group_size) * 2;
    a.r_shared = pick_rows(d.shared_inter, 64, 2 * ((size_t)H + 2 * srow_s), srow_s);
    a.nt_shared = d.shared_inter / a.r_shared;
    a.nt_sg = 1;
  }
  a.r_target = a.r_router;
  a.nt_target = NT ? E / a.r_target : 0;
  a.n_tiles = a.nt_router + a.nt_shared + a.nt_sg + NT * a.nt_target;
  auto part = [](size_t R, size_t rb, size_t sb) { return (R * rb + 15) / 16 * 16 + 2 * ((R * sb + 15) / 16 * 16); };
  size_t tile = part(a.r_router, H, srow);
  if (sh) {
    const size_t srow_s = (size_t)(H / L.shared_gate.group_size) * 2;
    const size_t ts = 2 * part(a.r_shared, H, srow_s);
    const size_t tsg = part(1, H, (size_t)(H / L.shared_expert_gate.group_size) * 2);
    if (ts > tile) tile = ts;
    if (tsg > tile) tile = tsg;
  }
  for (int g = 0; g < NT; ++g) {
    const size_t tt = part(a.r_target, H, (size_t)(H / tg[g].router.group_size) * 2);
    if (tt > tile) tile = tt;
  }
  a.tile_bytes = tile;
  a.x = o.x;
  a.logits = o.logits;
  a.act_sh = o.act_sh;
  a.sgate = o.sgate;
  a.ids = o.ids;
  a.wts = o.wts;
  a.flogits = o.flogits;
  a.fprobs = o.fprobs;
  a.counter = o.counter;
  a.err = o.err;
  const size_t rows_b = ((size_t)T * H * 2 + 15) / 16 * 16;
  const size_t smem = 256 + 2 * rows_b + ((size_t)H * 2 + 15) / 16 * 16 + tile;
  const int cpl = cpl_of(H);
  switch (cpl) {
#define PA(C)                                                                        \
  case C:                                                                            \
    if ((rc = set_smem(k_post_attention<C>, smem))) return rc;                       \
    k_post_attention<C><<<a.n_tiles, THREADS, smem, st>>>(a);                        \
    break;
    PA(1) PA(2) PA(3) PA(4) PA(8)
#undef PA
    default: return fail(YN_E_UNSUPPORTED, "hidden size not supported by the router kernel");
  }
  YN_CUDA(cudaGetLastError());
  return YN_OK;
}

static int launch_post_attention(const yn_dims& d, const yn_layer& L, const void* h1, int T, const yn_layer* tg,
                                 int NT, uint8_t* ws, const WsLayout& W, cudaStream_t st) {
  PostAttnOut o{};
  o.x = reinterpret_cast<uint16_t*>(ws + W.x);
  o.logits = reinterpret_cast<float*>(ws + W.logits);
  o.act_sh = reinterpret_cast<uint16_t*>(ws + W.act_sh);
  o.sgate = reinterpret_cast<float*>(ws + W.sgate);
  o.ids = reinterpret_cast<int32_t*>(ws + W.ids);
  o.wts = reinterpret_cast<float*>(ws + W.w);
  o.flogits = reinterpret_cast<float*>(ws + W.flogits);
  o.fprobs = reinterpret_cast<float*>(ws + W.fprobs);
  o.counter = reinterpret_cast<int*>(ws + W.counters);
  o.err = reinterpret_cast<int*>(ws + W.err);
  return launch_post_attention_out(d, L, h1, T, tg, NT, o, st);
}

int ynb::host_post_attention_rows(const yn_dims& d, const yn_layer& L, const void* h1, int T, const PostAttnOut& o,
                                  cudaStream_t st) {
  for (int t0 = 0; t0 < T; t0 += YN_MAX_ROWS) {
    const int n = std::min(YN_MAX_ROWS, T - t0);
    PostAttnOut c = o;
    c.x = o.x + (size_t)t0 * d.hidden;
    c.logits = o.logits + (size_t)t0 * d.n_experts;
    c.act_sh = o.act_sh + (size_t)t0 * (d.shared_inter ? d.shared_inter : 1);
    c.sgate = o.sgate + t0;
    c.ids = o.ids + (size_t)t0 * d.top_k;
    c.wts = o.wts + (size_t)t0 * d.top_k;
    const int rc = launch_post_attention_out(d, L, reinterpret_cast<const uint16_t*>(h1) + (size_t)t0 * d.hidden, n,
                                             nullptr, 0, c, st);
    if (rc) return rc;
  }
  return YN_OK;
}

int ynb::host_batch_dense(const yn_dims& d, const yn_layer& L, const void* h, int T, const PostAttnOut& o,
                          unsigned* counter, cudaStream_t st) {
  int rc;
  const int H = d.hidden, E = d.n_experts;
  if (!h || !L.post_norm || !counter) return fail(YN_E_INVALID, "batch post-attention: null argument");
  if (T < 1 || T > 4096) return fail(YN_E_UNSUPPORTED, "batch post-attention: rows must be in [1, 4096]");
  if ((rc = check_qmat(L.router, E, H, 8, "router"))) return rc;
  if (E % BD_RROWS) return fail(YN_E_UNSUPPORTED, "batch post-attention: n_experts must be a multiple of 16");
  if (!o.xf32 || !o.xsum) return fail(YN_E_INVALID, "batch post-attention: null fp32 row buffers");
  const bool sh = d.shared_inter > 0;
  if (sh) {
    if ((rc = check_qmat(L.shared_gate, d.shared_inter, H, 8, "shared_gate"))) return rc;
    if ((rc = check_qmat(L.shared_up, d.shared_inter, H, 8, "shared_up"))) return rc;
    if ((rc = check_qmat(L.shared_expert_gate, 1, H, 8, "shared_expert_gate"))) return rc;
    if (d.shared_inter % BD_SUNITS) return fail(YN_E_UNSUPPORTED, "batch post-attention: shared_inter % 8");
  }
  BatchDenseArgs a{};
  a.T = T; a.H = H; a.E = E; a.K = d.top_k; a.Ish = d.shared_inter; a.norm_topk = d.norm_topk; a.eps = d.rms_eps;
  a.xf = reinterpret_cast<const float4*>(o.xf32);
  a.xsum = o.xsum;
  a.router = to_qm(L.router);
  a.rbias = L.router_bias;
  a.has_shared = sh;
  if (sh) {
    a.sh_gate = to_qm(L.shared_gate);
    a.sh_up = to_qm(L.shared_up);
    a.sg = to_qm(L.shared_expert_gate);
  }
  a.nt_router = E / BD_RROWS;
  a.nt_shared = sh ? d.shared_inter / BD_SUNITS : 0;
  a.nt_sg = sh ? 1 : 0;
  a.logits = o.logits; a.act_sh = o.act_sh; a.sgate = o.sgate; a.ids = o.ids; a.wts = o.wts;
  a.counter = counter;
  a.err = o.err;
  auto part = [](size_t R, size_t rb, size_t sb) { return (R * rb + 15) / 16 * 16 + 2 * ((R * sb + 15) / 16 * 16); };
  size_t tile = part(BD_RROWS, H, (size_t)(H / L.router.group_size) * 2);
  if (sh) tile = std::max(tile, 2 * part(BD_SUNITS, H, (size_t)(H / L.shared_gate.group_size) * 2));
  const size_t smem = SMEM_HDR + (size_t)BD_TOK * H * 4 + (size_t)BD_TOK * (H / 16) * 4 + tile;
  dim3 grid(a.nt_router + a.nt_shared + a.nt_sg, (T + BD_TOK - 1) / BD_TOK);
  // RMSNorm once per row, then the dot products of every tile
  if ((rc = set_smem(k_rmsnorm_rows, (size_t)H * 4))) return rc;
  k_rmsnorm_rows<<<T, THREADS, (size_t)H * 4, st>>>(reinterpret_cast<const uint16_t*>(h),
                                                   reinterpret_cast<const uint16_t*>(L.post_norm), H, d.rms_eps, o.x,
                                                   reinterpret_cast<float4*>(o.xf32), o.xsum);
  YN_CUDA(cudaGetLastError());
  switch (H / 512) {
#define BDK(C)                                                                      \
  case C:                                                                           \
    if ((rc = set_smem(k_batch_dense<C>, smem))) return rc;                         \
    k_batch_dense<C><<<grid, BD_THREADS, smem, st>>>(a);                            \
    break;
    BDK(1) BDK(2) BDK(4) BDK(8)
#undef BDK
    default: return fail(YN_E_UNSUPPORTED, "batch post-attention: hidden must be 512, 1024, 2048 or 4096");
  }
  YN_CUDA(cudaGetLastError());
  return YN_OK;
}

static int check_layer_experts(const yn_dims& d, const yn_layer& L) {
  const yn_record& r = L.record;
  if (!L.expert_base) return fail(YN_E_INVALID, "expert_base is null");
  if (r.bits != 2 && r.bits != 4) return fail(YN_E_UNSUPPORTED, "routed experts must be 2- or 4-bit");
  if (r.group_size != 32 && r.group_size != 64 && r.group_size != 128)
    return fail(YN_E_UNSUPPORTED, "routed expert group size must be 32, 64 or 128");
  if (d.hidden % r.group_size || d.moe_inter % r.group_size) return fail(YN_E_INVALID, "group size must divide H and I");
  if (!aligned16(L.expert_base) || L.slot_stride % 16) return fail(YN_E_INVALID, "slot arena must be 16-byte aligned");
  for (int i = 0; i < 9; ++i)
    if (r.piece_offset[i] % 16) return fail(YN_E_INVALID, "record piece offsets must be multiples of 16");
  if (L.n_slots < 1) return fail(YN_E_INVALID, "n_slots must be >= 1");
  if (!L.expert_slot && L.n_slots < d.n_experts) return fail(YN_E_INVALID, "identity slot map needs n_slots >= n_experts");
  return YN_OK;
}

static int launch_expert_up(const yn_dims& d, const yn_layer& L, const void* x, const int32_t* ids, int T,
                            const int32_t* cols, int ncols, uint8_t* ws, const WsLayout& W, cudaStream_t st) {
  int rc;
  if ((rc = check_layer_experts(d, L))) return rc;
  ExpertUpArgs a{};
  a.T = T; a.H = d.hidden; a.I = d.moe_inter; a.K = d.top_k; a.E = d.n_experts; a.n_slots = L.n_slots;
  a.x = reinterpret_cast<const uint16_t*>(x ? x : ws + W.x);
  a.ids = ids ? ids : reinterpret_cast<const int32_t*>(ws + W.ids);
  a.slot_of = L.expert_slot;
  a.base = reinterpret_cast<const uint8_t*>(L.expert_base);
  a.stride = L.slot_stride;
  a.rg = rec_geom(L.record);
  if (!cols) ncols = d.top_k;
  if (ncols < 0 || ncols > 16) return fail(YN_E_INVALID, "n_cols must be in [0, 16]");
  if (ncols == 0) return YN_OK;
  a.ncols = ncols;
  for (int i = 0; i < ncols; ++i) {
    a.cols[i] = cols ? cols[i] : i;
    if (a.cols[i] < 0 || a.cols[i] >= d.top_k) return fail(YN_E_INVALID, "column index out of range");
  }
  const int bits = L.record.bits, gs = L.record.group_size;
  const int rb = d.hidden * bits / 8;
  const size_t srow = (size_t)(d.hidden / gs) * 2;
  a.rows = pick_rows(d.moe_inter, 64, 2 * ((size_t)rb + 2 * srow), srow);
  a.tiles_per_task = d.moe_inter / a.rows;
  a.act = reinterpret_cast<uint16_t*>(ws + W.act);
  a.err = reinterpret_cast<int*>(ws + W.err);
  const size_t tile = 2 * ((((size_t)a.rows * rb + 15) / 16 * 16) + 2 * (((size_t)a.rows * srow + 15) / 16 * 16));
  const size_t smem = 256 + ((size_t)d.hidden * 2 + 15) / 16 * 16 + tile;
  const int grid = T * ncols * a.tiles_per_task;
  const int cpl = cpl_of(rb);
  const int nseg = (bits == 2 && gs == 32) ? 2 : 1;
  bool done = false;
#define EU(B, C, S)                                                              \
  if (!done && bits == B && cpl == C && nseg == S) {                             \
    if ((rc = set_smem(k_expert_up<B, C, S>, smem))) return rc;                  \
    k_expert_up<B, C, S><<<grid, THREADS, smem, st>>>(a);                        \
    done = true;                                                                 \
  }
  EU(4, 1, 1) EU(4, 2, 1) EU(4, 3, 1) EU(4, 4, 1)
  EU(2, 1, 1) EU(2, 2, 1) EU(2, 3, 1) EU(2, 1, 2) EU(2, 2, 2) EU(2, 3, 2)
#undef EU
  if (!done) return fail(YN_E_UNSUPPORTED, "expert up: no kernel for this bit width / hidden size");
  YN_CUDA(cudaGetLastError());
  return YN_OK;
}

static int launch_expert_down(const yn_dims& d, const yn_layer& L, const int32_t* ids, const float* wts, int T,
                              const void* h_res, int mode, void* out, uint8_t* ws, const WsLayout& W,
                              cudaStream_t st) {
  int rc;
  if ((rc = check_layer_experts(d, L))) return rc;
  if (!out) return fail(YN_E_INVALID, "out is null");
  if (mode < 0 || mode > 2) return fail(YN_E_INVALID, "mode must be 0, 1 or 2");
  if (mode == 2 && !h_res) return fail(YN_E_INVALID, "mode 2 needs h_res");
  const bool sh = (mode >= 1) && d.shared_inter > 0;
  if (sh && (rc = check_qmat(L.shared_down, d.hidden, d.shared_inter, 8, "shared_down"))) return rc;
  ExpertDownArgs a{};
  a.T = T; a.H = d.hidden; a.I = d.moe_inter; a.K = d.top_k; a.E = d.n_experts; a.n_slots = L.n_slots;
  a.Ish = sh ? d.shared_inter : 0;
  a.has_shared = sh;
  a.mode = mode;
  a.act = reinterpret_cast<const uint16_t*>(ws + W.act);
  a.ids = ids ? ids : reinterpret_cast<const int32_t*>(ws + W.ids);
  a.wts = wts ? wts : reinterpret_cast<const float*>(ws + W.w);
  a.slot_of = L.expert_slot;
  a.base = reinterpret_cast<const uint8_t*>(L.expert_base);
  a.stride = L.slot_stride;
  a.rg = rec_geom(L.record);
  if (sh) a.sh_down = to_qm(L.shared_down);
  a.act_sh = reinterpret_cast<const uint16_t*>(ws + W.act_sh);
  a.sgate = reinterpret_cast<const float*>(ws + W.sgate);
  a.h_res = reinterpret_cast<const uint16_t*>(h_res);
  a.y = reinterpret_cast<uint16_t*>(ws + W.y);
  a.ysh = a.y + (size_t)YN_MAX_ROWS * d.top_k * d.hidden;
  a.out = reinterpret_cast<uint16_t*>(out);
  a.counters = reinterpret_cast<int*>(ws + W.counters) + 1;
  a.n_cb = W.n_cb;
  a.err = reinterpret_cast<int*>(ws + W.err);
  const int bits = L.record.bits, gs = L.record.group_size;
  const int cbr = d.hidden < CB_ROWS ? d.hidden : CB_ROWS;
  const int rb = d.moe_inter * bits / 8;
  const size_t srow = (size_t)(d.moe_inter / gs) * 2;
  a.rows_routed = pick_rows(cbr, cbr, (size_t)rb + 2 * srow, srow);
  a.tiles_routed_per_task = d.hidden / a.rows_routed;
  a.n_routed_tiles = T * d.top_k * a.tiles_routed_per_task;
  size_t tile = ((size_t)a.rows_routed * rb + 15) / 16 * 16 + 2 * (((size_t)a.rows_routed * srow + 15) / 16 * 16);
  int cpls = 1;
  if (sh) {
    const size_t srow_s = (size_t)(d.shared_inter / L.shared_down.group_size) * 2;
    a.rows_shared = pick_rows(cbr, cbr, (size_t)d.shared_inter + 2 * srow_s, srow_s);
    a.tiles_shared_per_token = d.hidden / a.rows_shared;
    const size_t ts = ((size_t)a.rows_shared * d.shared_inter + 15) / 16 * 16 + 2 * (((size_t)a.rows_shared * srow_s + 15) / 16 * 16);
    if (ts > tile) tile = ts;
    cpls = cpl_of(d.shared_inter);
  } else {
    a.rows_shared = 1;
  }
  const int kx = d.moe_inter > d.shared_inter ? d.moe_inter : d.shared_inter;
  const size_t smem = 256 + ((size_t)kx * 2 + 15) / 16 * 16 + tile;
  const int grid = a.n_routed_tiles + (sh ? T * a.tiles_shared_per_token : 0);
  const int cpl = cpl_of(rb);
  const int nseg = (bits == 2 && gs == 32) ? 2 : 1;
  bool done = false;
#define ED(B, C, S, CS)                                                          \
  if (!done && bits == B && cpl == C && nseg == S && cpls == CS) {               \
    if ((rc = set_smem(k_expert_down<B, C, S, CS>, smem))) return rc;            \
    k_expert_down<B, C, S, CS><<<grid, THREADS, smem, st>>>(a);                  \
    done = true;                                                                 \
  }
  ED(4, 1, 1, 1) ED(4, 2, 1, 1) ED(4, 3, 1, 1) ED(4, 1, 1, 2) ED(4, 2, 1, 2) ED(4, 3, 1, 2)
  ED(2, 1, 1, 1) ED(2, 2, 1, 1) ED(2, 3, 1, 1) ED(2, 1, 1, 2) ED(2, 3, 1, 2)
  ED(2, 1, 2, 1) ED(2, 3, 2, 1) ED(2, 1, 2, 2)
#undef ED
  if (!done) return fail(YN_E_UNSUPPORTED, "expert down: no kernel for this bit width / intermediate size");
  YN_CUDA(cudaGetLastError());
  return YN_OK;
}

extern "C" int yn_post_attention(const yn_dims* dims, const yn_layer* layer, const void* h1, int32_t T,
                                 const yn_layer* targets, int32_t n_targets, void* ws, void* stream) {
  int rc = check_dims(dims, T);
  if (rc) return rc;
  if (!layer || !ws) return fail(YN_E_INVALID, "null layer or workspace");
  if (n_targets && !targets) return fail(YN_E_INVALID, "targets is null");
  WsLayout W = ws_layout(*dims);
  return launch_post_attention(*dims, *layer, h1, T, targets, n_targets, reinterpret_cast<uint8_t*>(ws), W,
                               as_stream(stream));
}

extern "C" int yn_moe_up(const yn_dims* dims, const yn_layer* layer, const void* x, const int32_t* ids, int32_t T,
                         const int32_t* cols, int32_t n_cols, void* ws, void* stream) {
  int rc = check_dims(dims, T);
  if (rc) return rc;
  if (!layer || !ws) return fail(YN_E_INVALID, "null layer or workspace");
  WsLayout W = ws_layout(*dims);
  return launch_expert_up(*dims, *layer, x, ids, T, cols, n_cols, reinterpret_cast<uint8_t*>(ws), W,
                          as_stream(stream));
}

extern "C" int yn_moe_down(const yn_dims* dims, const yn_layer* layer, const int32_t* ids, const float* weights,
                           int32_t T, const void* h_res, int32_t mode, void* out, void* ws, void* stream) {
  int rc = check_dims(dims, T);
  if (rc) return rc;
  if (!layer || !ws) return fail(YN_E_INVALID, "null layer or workspace");
  WsLayout W = ws_layout(*dims);
  return launch_expert_down(*dims, *layer, ids, weights, T, h_res, mode, out, reinterpret_cast<uint8_t*>(ws), W,
                            as_stream(stream));
}

extern "C" int yn_moe_layer(const yn_dims* dims, const yn_layer* layer, const void* h_in, int32_t T,
                            const yn_layer* targets, int32_t n_targets, void* h_out, void* ws, void* stream) {
  int rc = check_dims(dims, T);
  if (rc) return rc;
  if (!layer || !ws || !h_in || !h_out) return fail(YN_E_INVALID, "null argument");
  if (h_in == h_out) return fail(YN_E_INVALID, "h_in and h_out must not alias");
  WsLayout W = ws_layout(*dims);
  uint8_t* b = reinterpret_cast<uint8_t*>(ws);
  cudaStream_t st = as_stream(stream);
  if ((rc = launch_post_attention(*dims, *layer, h_in, T, targets, n_targets, b, W, st))) return rc;
  if ((rc = launch_expert_up(*dims, *layer, nullptr, nullptr, T, nullptr, 0, b, W, st))) return rc;
  return launch_expert_down(*dims, *layer, nullptr, nullptr, T, h_in, 2, h_out, b, W, st);
}

// ------------------------------------------------- no-allocation variant
// One workspace per device in static device memory (zero at module load,
// zeroed again explicitly at set-up). g_na_clean[dev] is the byte offset up
// to which the front of the array is known to hold zero counters: the
// counters reset themselves at the end of each call, the bytes behind them
// may hold a previous call's activations.
static __device__ __align__(256) uint8_t g_noalloc_scratch[YN_NOALLOC_SCRATCH_BYTES];
static constexpr int kNaMaxDevices = 64;
static std::mutex g_na_mu;
static uint8_t* g_na_ptr[kNaMaxDevices];
static size_t g_na_clean[kNaMaxDevices];

extern "C" int yn_moe_layer_noalloc(const yn_dims* dims, const yn_layer* layer, const void* h_in, int32_t T,
                                    const yn_layer* targets, int32_t n_targets, void* h_out, void* stream,
                                    void** scratch_out) {
  int rc = check_dims(dims, T);
  if (rc) return rc;
  if (!layer || !h_in || !h_out) return fail(YN_E_INVALID, "null argument");
  if (h_in == h_out) return fail(YN_E_INVALID, "h_in and h_out must not alias");
  if (n_targets && !targets) return fail(YN_E_INVALID, "targets is null");
  WsLayout W = ws_layout(*dims);
  if (W.total > YN_NOALLOC_SCRATCH_BYTES)
    return fail(YN_E_UNSUPPORTED, "yn_moe_layer_noalloc: workspace of " + std::to_string(W.total) +
                                      " bytes exceeds the static scratch of " +
                                      std::to_string((size_t)YN_NOALLOC_SCRATCH_BYTES) + " bytes");
  int dev = 0;
  YN_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNaMaxDevices) return fail(YN_E_UNSUPPORTED, "device ordinal out of range");
  cudaStream_t st = as_stream(stream);
  const size_t counters_end = W.counters + (size_t)(1 + YN_MAX_ROWS * W.n_cb) * 4;
  uint8_t* b = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_na_mu);
    if (!g_na_ptr[dev]) {
      void* p = nullptr;
      YN_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
      YN_CUDA(cudaMemsetAsync(p, 0, YN_NOALLOC_SCRATCH_BYTES, st));
      g_na_ptr[dev] = reinterpret_cast<uint8_t*>(p);
      g_na_clean[dev] = counters_end;
    } else if (counters_end > g_na_clean[dev]) {
      YN_CUDA(cudaMemsetAsync(g_na_ptr[dev] + g_na_clean[dev], 0, counters_end - g_na_clean[dev], st));
    }
    g_na_clean[dev] = counters_end;
    b = g_na_ptr[dev];
  }
  if (scratch_out) *scratch_out = b;
  if ((rc = launch_post_attention(*dims, *layer, h_in, T, targets, n_targets, b, W, st))) return rc;
  if ((rc = launch_expert_up(*dims, *layer, nullptr, nullptr, T, nullptr, 0, b, W, st))) return rc;
  return launch_expert_down(*dims, *layer, nullptr, nullptr, T, h_in, 2, h_out, b, W, st);
}

// ------------------------------------------------------------ slot copy
extern "C" int yn_slot_copy(void* arena, int64_t slot_stride, const int32_t* slots, const void* const* host_src,
                            int32_t n, int64_t record_bytes, void* stream) {
  if (n < 0) return fail(YN_E_INVALID, "n < 0");
  if (n && (!arena || !slots || !host_src)) return fail(YN_E_INVALID, "null argument");
  if (record_bytes > slot_stride) return fail(YN_E_INVALID, "record larger than a slot");
  for (int i = 0; i < n; ++i) {
    if (slots[i] < 0) return fail(YN_E_INVALID, "negative slot index");
    uint8_t* dst = reinterpret_cast<uint8_t*>(arena) + (size_t)slots[i] * (size_t)slot_stride;
    YN_CUDA(cudaMemcpyAsync(dst, host_src[i], (size_t)record_bytes, cudaMemcpyHostToDevice, as_stream(stream)));
  }
  return YN_OK;
}

// ---------------------------------------------------------------- timing
// Record a timing event on `stream`; inside a stream capture the record
// becomes an external event node, so per-kernel durations can be read after
// each replay of the graph.
extern "C" int yn_record_event(void* event, void* stream) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  YN_CUDA(cudaStreamIsCapturing(as_stream(stream), &cs));
  if (cs == cudaStreamCaptureStatusActive)
    YN_CUDA(cudaEventRecordWithFlags(reinterpret_cast<cudaEvent_t>(event), as_stream(stream), cudaEventRecordExternal));
  else
    YN_CUDA(cudaEventRecord(reinterpret_cast<cudaEvent_t>(event), as_stream(stream)));
  return YN_OK;
}

extern "C" int yn_event_create(void** event) {
  if (!event) return fail(YN_E_INVALID, "null argument");
  cudaEvent_t e;
  YN_CUDA(cudaEventCreate(&e));
  *event = reinterpret_cast<void*>(e);
  return YN_OK;
}
extern "C" int yn_event_destroy(void* event) {
  YN_CUDA(cudaEventDestroy(reinterpret_cast<cudaEvent_t>(event)));
  return YN_OK;
}
extern "C" int yn_event_elapsed_ms(void* start, void* end, float* ms) {
  if (!ms) return fail(YN_E_INVALID, "null argument");
  YN_CUDA(cudaEventElapsedTime(ms, reinterpret_cast<cudaEvent_t>(start), reinterpret_cast<cudaEvent_t>(end)));
  return YN_OK;
}

// ------------------------------------------------- persistent stack decode
static size_t a16h(size_t v) { return (v + 15) / 16 * 16; }

extern "C" size_t yn_stack_table_bytes(int32_t n_layers) { return (size_t)(n_layers > 0 ? n_layers : 0) * sizeof(DecLayer); }

struct StackScratch {
  size_t err, bar, f_logits, zero_end, hbuf, act, act_sh, sgate, total;
};
// Error word; barrier counter and flagged logits (zeroed before every launch);
// buffers passed between phases.
static StackScratch stack_scratch(const yn_dims& d) {
  StackScratch S{};
  size_t o = 0;
  auto take = [&](size_t b) { size_t at = o; o = (o + b + 255) / 256 * 256; return at; };
  S.err = take(4);
  S.bar = take(4);
  S.f_logits = take(2 * (size_t)d.n_experts * 8);
  S.zero_end = o;
  S.hbuf = take(2 * (size_t)d.hidden * 2);
  S.act = take((size_t)d.top_k * d.moe_inter * 2);
  S.act_sh = take((size_t)(d.shared_inter ? d.shared_inter : 8) * 2);
  S.sgate = take(4);
  S.total = o;
  return S;
}
extern "C" size_t yn_stack_scratch_bytes(const yn_dims* dims) { return dims ? stack_scratch(*dims).total : 0; }

extern "C" int yn_stack_prepare(const yn_dims* dims, const yn_layer* layers, int32_t n_layers, void* table,
                                size_t table_bytes) {
  int rc = check_dims(dims, 1);
  if (rc) return rc;
  if (!layers || n_layers < 1 || !table) return fail(YN_E_INVALID, "null layers/table or n_layers < 1");
  if (table_bytes < yn_stack_table_bytes(n_layers)) return fail(YN_E_INVALID, "layer table too small");
  std::vector<DecLayer> t(n_layers);
  for (int l = 0; l < n_layers; ++l) {
    const yn_layer& L = layers[l];
    if ((rc = check_qmat(L.router, dims->n_experts, dims->hidden, 8, "router"))) return rc;
    if (dims->shared_inter) {
      if ((rc = check_qmat(L.shared_gate, dims->shared_inter, dims->hidden, 8, "shared_gate"))) return rc;
      if ((rc = check_qmat(L.shared_up, dims->shared_inter, dims->hidden, 8, "shared_up"))) return rc;
      if ((rc = check_qmat(L.shared_down, dims->hidden, dims->shared_inter, 8, "shared_down"))) return rc;
      if ((rc = check_qmat(L.shared_expert_gate, 1, dims->hidden, 8, "shared_expert_gate"))) return rc;
    }
    if ((rc = check_layer_experts(*dims, L))) return rc;
    if (!L.post_norm) return fail(YN_E_INVALID, "post_norm is null");
    DecLayer& D = t[l];
    memset(&D, 0, sizeof(D));
    D.norm = reinterpret_cast<const uint16_t*>(L.post_norm);
    D.router = to_qm(L.router);
    D.rbias = L.router_bias;
    if (dims->shared_inter) {
      D.sg = to_qm(L.shared_gate);
      D.su = to_qm(L.shared_up);
      D.sd = to_qm(L.shared_down);
      D.sgt = to_qm(L.shared_expert_gate);
    }
    D.ebase = reinterpret_cast<const uint8_t*>(L.expert_base);
    D.stride = L.slot_stride;
    D.slot_of = L.expert_slot;
    D.n_slots = L.n_slots;
    D.rg = rec_geom(L.record);
  }
  YN_CUDA(cudaMemcpy(table, t.data(), t.size() * sizeof(DecLayer), cudaMemcpyHostToDevice));
  return YN_OK;
}

// Host mirror of the device P1 partition, for buffer sizing.
static size_t p1_tile_bytes_max(int Ish, int G) {
  size_t best = 0;
  const int E = DEC_E, H = DEC_H;
  auto unit_at = [&](int c) {
    if (c <= E) return c;
    if (c <= E + 2 * Ish) return E + (c - E + 1) / 2;
    return E + Ish + (c - E - 2 * Ish);
  };
  const int C = E + 2 * Ish + (Ish ? 1 : 0);
  for (int b = 0; b < G; ++b) {
    const int lo = (int)((long long)b * C / G), hi = (int)((long long)(b + 1) * C / G);
    const int u0 = unit_at(lo), u1 = unit_at(hi);
    const size_t nr = std::min(u1, E) - std::min(u0, E);
    const size_t np = std::min(std::max(u1 - E, 0), Ish) - std::min(std::max(u0 - E, 0), Ish);
    const int sg = (Ish > 0 && u0 <= E + Ish && u1 > E + Ish) ? 1 : 0;
    const size_t sb = DEC_DSB;
    size_t o = a16h((size_t)H * 2) + a16h(nr * H) + 2 * a16h(nr * sb) + 2 * (a16h(np * H) + 2 * a16h(np * sb)) +
               (sg ? a16h(H) + 2 * a16h(sb) : 0);
    best = std::max(best, o);
  }
  return best;
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" int yn_stack_decode(const yn_dims* dims, const void* table, const yn_layer* layers, int32_t n_layers,
                               const void* inputs, int32_t n_tokens, void* outputs, void* scratch,
                               size_t scratch_bytes, int32_t* trace_ids, void* trace_hidden, float* trace_weights,
                               int64_t* timing, void* stream) {
  int rc = check_dims(dims, 1);
  if (rc) return rc;
  const yn_dims& d = *dims;
  if (!table || !inputs || !outputs || !scratch || !layers) return fail(YN_E_INVALID, "null argument");
  if (n_layers < 1 || n_tokens < 1) return fail(YN_E_INVALID, "n_layers and n_tokens must be >= 1");
  StackScratch S = stack_scratch(d);
  if (scratch_bytes < S.total) return fail(YN_E_INVALID, "scratch too small");
  const int K = d.top_k, Ish = d.shared_inter;
  // The persistent kernel is compiled for one shape (index arithmetic on constants).
  if (d.hidden != DEC_H || d.n_experts != DEC_E || d.moe_inter != DEC_I || (Ish != 0 && Ish != DEC_I) ||
      K > DEC_MAX_K)
    return fail(YN_E_UNSUPPORTED, "stack decode is compiled for hidden 2048, 512 experts, intermediate 512 "
                                  "(shared 0 or 512), top_k <= 16");
  int rb_max = 0, sb_max = 0, rbi_max = 0, sbi_max = 0;
  for (int l = 0; l < n_layers; ++l) {
    const yn_layer& L = layers[l];
    const int bits = L.record.bits, gs = L.record.group_size;
    if ((bits != 2 && bits != 4) || (gs != 32 && gs != 64))
      return fail(YN_E_UNSUPPORTED, "stack decode: routed experts must be 2- or 4-bit with groups of 32 or 64");
    if (L.router.group_size != DEC_DGS ||
        (Ish && (L.shared_gate.group_size != DEC_DGS || L.shared_up.group_size != DEC_DGS ||
                 L.shared_down.group_size != DEC_DGS || L.shared_expert_gate.group_size != DEC_DGS)))
      return fail(YN_E_UNSUPPORTED, "stack decode: dense 8-bit matrices must use groups of 64");
    for (int i = 0; i < 9; ++i)
      if (L.record.piece_offset[i] % 16) return fail(YN_E_UNSUPPORTED, "stack decode: record pieces must be 16-byte aligned");
    if (!al16(L.expert_base) || L.slot_stride % 16)
      return fail(YN_E_UNSUPPORTED, "stack decode: slot arena and stride must be 16-byte aligned");
    if (!al16(L.router.weight) || !al16(L.router.scales) || !al16(L.router.biases) || !al16(L.post_norm))
      return fail(YN_E_UNSUPPORTED, "stack decode: router pieces must be 16-byte aligned");
    if (Ish && (!al16(L.shared_gate.weight) || !al16(L.shared_gate.scales) || !al16(L.shared_gate.biases) ||
                !al16(L.shared_up.weight) || !al16(L.shared_up.scales) || !al16(L.shared_up.biases) ||
                !al16(L.shared_down.weight) || !al16(L.shared_down.scales) || !al16(L.shared_down.biases) ||
                !al16(L.shared_expert_gate.weight) || !al16(L.shared_expert_gate.scales) ||
                !al16(L.shared_expert_gate.biases)))
      return fail(YN_E_UNSUPPORTED, "stack decode: shared-expert pieces must be 16-byte aligned");
    rb_max = std::max(rb_max, DEC_H * bits / 8);
    sb_max = std::max(sb_max, DEC_H / gs * 2);
    rbi_max = std::max(rbi_max, DEC_I * bits / 8);
    sbi_max = std::max(sbi_max, DEC_I / gs * 2);
  }
  int dev = 0, sms = 0;
  YN_CUDA(cudaGetDevice(&dev));
  YN_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int G = sms;
  const int noct = K * (DEC_I / 8);
  const int oct_max = (noct + G - 1) / G;
  if (oct_max > DEC_MAX_OCT) return fail(YN_E_UNSUPPORTED, "stack decode: too many gate/up tiles per CTA");
  if ((DEC_H + G - 1) / G > DEC_MAX_DROWS) return fail(YN_E_UNSUPPORTED, "stack decode: more than 16 output rows per CTA");
  // shared-memory carve (mirrors the pointer layout at the top of k_stack_decode)
  DecodeArgs a{};
  size_t o = 256;
  a.off_hs = (int)o; o += a16h((size_t)DEC_H * 2);
  a.off_xs = (int)o; o += a16h((size_t)DEC_H * 2);
  a.off_route = (int)o;
  o += a16h(4 * (size_t)DEC_E + 4 * DEC_WARPS * DEC_MAX_K + 4 * DEC_MAX_K + 4 * DEC_MAX_K + 4 * (DEC_MAX_K + 4) +
            4 * 64 + 4 * 256 + 3 * sizeof(DecLayer));
  // fragments + group sums + group unpack offsets
  a.off_xf2 = (int)o; o += a16h((size_t)DEC_H / 2 * 4 + 2 * (size_t)DEC_H / 32 * 4);
  a.off_xf3 = (int)o; o += a16h((size_t)(DEC_MAX_K + 1) * (DEC_I / 2) * 4 + 2 * (size_t)(DEC_MAX_K + 1) * 16 * 4);
  const size_t part_p2 = (size_t)oct_max * 8 * 2 * 16 * 4, part_p3 = (size_t)(K + 1) * 16 * 8 * 4;
  a.off_part = (int)o; o += a16h(std::max(part_p2, part_p3));
  a.off_A = (int)o; o += a16h(p1_tile_bytes_max(Ish, G));
  a.c_rows = 8 * oct_max;
  a.c_rb = rb_max;
  a.c_sb = sb_max;
  a.d_rb = rbi_max;
  a.d_sb = sbi_max;
  const size_t d_bytes = (size_t)K * DEC_MAX_DROWS * a.d_rb + (size_t)DEC_MAX_DROWS * DEC_I +
                         2 * (size_t)K * DEC_MAX_DROWS * a.d_sb + 2 * (size_t)DEC_MAX_DROWS * DEC_DSBI;
  // The C tile (gate/up rows) is dead once P2's dots are done; P3's
  // activation staging and the D tile (down rows, copied after P2) share its
  // space, staging first.
  const size_t stage_bytes = a16h((size_t)(K + 1) * DEC_I * 2);
  const size_t c_bytes = std::max((size_t)2 * a.c_rows * a.c_rb + (size_t)4 * a.c_rows * a.c_sb,
                                  stage_bytes + d_bytes);
  a.off_C = (int)o;
  a.off_D = (int)(o + stage_bytes);
  o += a16h(c_bytes);
  const size_t smem = o;
  int optin = 0;
  YN_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  if (smem > (size_t)optin)
    return fail(YN_E_UNSUPPORTED, "stack decode needs " + std::to_string(smem) + " B of shared memory (" +
                                      std::to_string(optin) + " available)");

  uint8_t* sc = reinterpret_cast<uint8_t*>(scratch);
  a.K = K; a.Ish = Ish; a.norm_topk = d.norm_topk; a.eps = d.rms_eps;
  a.layers = reinterpret_cast<const DecLayer*>(table);
  a.n_layers = n_layers;
  a.inputs = reinterpret_cast<const uint16_t*>(inputs);
  a.n_tokens = n_tokens;
  a.outputs = reinterpret_cast<uint16_t*>(outputs);
  a.f_logits = reinterpret_cast<unsigned long long*>(sc + S.f_logits);
  a.hbuf = reinterpret_cast<uint16_t*>(sc + S.hbuf);
  a.act = reinterpret_cast<uint16_t*>(sc + S.act);
  a.act_sh = reinterpret_cast<uint16_t*>(sc + S.act_sh);
  a.sgate = reinterpret_cast<float*>(sc + S.sgate);
  a.trace_ids = trace_ids;
  a.trace_h = reinterpret_cast<uint16_t*>(trace_hidden);
  a.trace_w = trace_weights;
  if (trace_hidden && !al16(trace_hidden)) return fail(YN_E_INVALID, "stack decode: trace_hidden must be 16-byte aligned");
  a.bar = reinterpret_cast<unsigned*>(sc + S.bar);
  a.err = reinterpret_cast<int*>(sc + S.err);
  a.timing = reinterpret_cast<long long*>(timing);
  if (!al16(inputs) || !al16(outputs) || !al16(scratch))
    return fail(YN_E_INVALID, "stack decode: inputs, outputs and scratch must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  // barrier counter, and stale logit epochs of an earlier launch that must not
  // match this launch's steps
  YN_CUDA(cudaMemsetAsync(sc + S.bar, 0, S.zero_end - S.bar, st));
  const void* kernel = reinterpret_cast<const void*>(&k_stack_decode);
  if ((rc = set_smem_ptr(kernel, smem))) return rc;
  int per_sm = 0;
  YN_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, DEC_THREADS, smem));
  if (per_sm < 1) return fail(YN_E_UNSUPPORTED, "stack decode kernel does not fit on an SM");
  void* args[] = {&a};
  YN_CUDA(cudaLaunchCooperativeKernel(kernel, dim3(G), dim3(DEC_THREADS), args, smem, st));
  return YN_OK;
}

// ------------------------------------------ persistent decode, data-flow form
struct FlowScratch {
  size_t err, f_logits, f_act, f_ash, f_y, f_h, total;
};
// Error word first (as in the barrier form, so yn_stack_error reads both),
// then the flagged-word buffers, zeroed before every launch.
static FlowScratch flow_scratch(const yn_dims& d) {
  FlowScratch S{};
  size_t o = 0;
  auto take = [&](size_t b) { size_t at = o; o = (o + b + 255) / 256 * 256; return at; };
  S.err = take(4);
  S.f_logits = take(2 * (size_t)d.n_experts * 8);
  S.f_act = take(2 * (size_t)d.top_k * (d.moe_inter / 2) * 8);
  S.f_ash = take(2 * ((size_t)d.shared_inter + 1) * 8);
  S.f_y = take(2 * ((size_t)d.top_k + 1) * (d.hidden / 2) * 8);
  S.f_h = take(2 * (size_t)(d.hidden / 2) * 8);
  S.total = o;
  return S;
}
extern "C" size_t yn_stack_flow_scratch_bytes(const yn_dims* dims) { return dims ? flow_scratch(*dims).total : 0; }

extern "C" int yn_stack_flow_decode(const yn_dims* dims, const void* table, const yn_layer* layers, int32_t n_layers,
                                    const void* inputs, int32_t n_tokens, void* outputs, void* scratch,
                                    size_t scratch_bytes, int32_t* trace_ids, void* trace_hidden,
                                    float* trace_weights, int64_t* timing, void* stream) {
  int rc = check_dims(dims, 1);
  if (rc) return rc;
  const yn_dims& d = *dims;
  if (!table || !inputs || !outputs || !scratch || !layers) return fail(YN_E_INVALID, "null argument");
  if (n_layers < 1 || n_tokens < 1) return fail(YN_E_INVALID, "n_layers and n_tokens must be >= 1");
  const FlowScratch S = flow_scratch(d);
  if (scratch_bytes < S.total) return fail(YN_E_INVALID, "scratch too small");
  const int K = d.top_k, Ish = d.shared_inter;
  if (d.hidden != DEC_H || d.n_experts != DEC_E || d.moe_inter != DEC_I || (Ish != 0 && Ish != DEC_I) ||
      K > DEC_MAX_K)
    return fail(YN_E_UNSUPPORTED, "stack decode is compiled for hidden 2048, 512 experts, intermediate 512 "
                                  "(shared 0 or 512), top_k <= 16");
  int rb_max = 0, sb_max = 0, rbi_max = 0, sbi_max = 0;
  for (int l = 0; l < n_layers; ++l) {
    const yn_layer& L = layers[l];
    const int bits = L.record.bits, gs = L.record.group_size;
    if ((bits != 2 && bits != 4) || (gs != 32 && gs != 64))
      return fail(YN_E_UNSUPPORTED, "stack decode: routed experts must be 2- or 4-bit with groups of 32 or 64");
    if (L.router.group_size != DEC_DGS ||
        (Ish && (L.shared_gate.group_size != DEC_DGS || L.shared_up.group_size != DEC_DGS ||
                 L.shared_down.group_size != DEC_DGS || L.shared_expert_gate.group_size != DEC_DGS)))
      return fail(YN_E_UNSUPPORTED, "stack decode: dense 8-bit matrices must use groups of 64");
    for (int i = 0; i < 9; ++i)
      if (L.record.piece_offset[i] % 16) return fail(YN_E_UNSUPPORTED, "stack decode: record pieces must be 16-byte aligned");
    if (!al16(L.expert_base) || L.slot_stride % 16)
      return fail(YN_E_UNSUPPORTED, "stack decode: slot arena and stride must be 16-byte aligned");
    if (!al16(L.router.weight) || !al16(L.router.scales) || !al16(L.router.biases) || !al16(L.post_norm))
      return fail(YN_E_UNSUPPORTED, "stack decode: router pieces must be 16-byte aligned");
    if (Ish && (!al16(L.shared_gate.weight) || !al16(L.shared_gate.scales) || !al16(L.shared_gate.biases) ||
                !al16(L.shared_up.weight) || !al16(L.shared_up.scales) || !al16(L.shared_up.biases) ||
                !al16(L.shared_down.weight) || !al16(L.shared_down.scales) || !al16(L.shared_down.biases) ||
                !al16(L.shared_expert_gate.weight) || !al16(L.shared_expert_gate.scales) ||
                !al16(L.shared_expert_gate.biases)))
      return fail(YN_E_UNSUPPORTED, "stack decode: shared-expert pieces must be 16-byte aligned");
    rb_max = std::max(rb_max, DEC_H * bits / 8);
    sb_max = std::max(sb_max, DEC_H / gs * 2);
    rbi_max = std::max(rbi_max, DEC_I * bits / 8);
    sbi_max = std::max(sbi_max, DEC_I / gs * 2);
  }
  int dev = 0, sms = 0;
  YN_CUDA(cudaGetDevice(&dev));
  YN_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int G = sms;
  // K groups of nr CTAs (routed columns), the rest (ns >= 18 where the SMs allow, else >= 8) for the shared
  // expert's down rows: 8-bit rows cost ~4x a 2-bit routed row, so the shared blocks are spread wider
  const int nr = std::max((G - 18) / K, std::min(8, (G - 8) / K)), ns = G - K * nr;
  const int oct_max = (DEC_I / 8 + nr - 1) / std::max(nr, 1), dt_max = (DEC_H / 16 + nr - 1) / std::max(nr, 1);
  const int dts_max = (DEC_H / 16 + ns - 1) / ns;
  if (nr < 1 || ns < 8 || oct_max > DEC_MAX_OCT || dt_max > FL_MAX_DT || dts_max > FL_MAX_DT ||
      (FL_HW + G - 1) / G > FL_MAX_CW)
    return fail(YN_E_UNSUPPORTED, "data-flow decode: " + std::to_string(G) + " SMs cannot hold " +
                                      std::to_string(K) + " routed columns of at least 8 CTAs plus 8 shared CTAs");
  FlowArgs a{};
  size_t o = 256;
  auto put = [&](int& off, size_t bytes) { off = (int)o; o += (bytes + 127) / 128 * 128; };
  put(a.off_hs, (size_t)DEC_H * 2);
  put(a.off_xs, (size_t)DEC_H * 2);
  put(a.off_route, 4 * (size_t)DEC_E + 4 * DEC_WARPS * DEC_MAX_K + 4 * DEC_MAX_K + 4 * DEC_MAX_K + 4 * (DEC_MAX_K + 4) +
                       4 * 64 + 4 * 256 + 3 * sizeof(DecLayer));
  put(a.off_xf2, (size_t)DEC_H / 2 * 4 + 2 * (size_t)DEC_H / 32 * 4);
  put(a.off_xf3, (size_t)DEC_I / 2 * 4 + 2 * 16 * 4);
  const size_t part_up = (size_t)oct_max * 8 * 2 * (DEC_H * 4 / 8 / 64) * 4;
  const size_t part_dn = (size_t)16 * std::max(dt_max, dts_max) * (DEC_I / 64) * 4;
  put(a.off_part, std::max(part_up, part_dn));
  put(a.off_stage, (size_t)DEC_I * 2 + (size_t)(K + 1) * FL_MAX_CW * 4);
  put(a.off_A, p1_tile_bytes_max(Ish, G));
  a.c_rows = 8 * oct_max;
  a.c_rb = rb_max;
  a.c_sb = sb_max;
  a.d_rows = 16 * dt_max;
  a.d_rb = rbi_max;
  a.d_sb = sbi_max;
  const size_t c_bytes = (size_t)2 * a.c_rows * a.c_rb + (size_t)4 * a.c_rows * a.c_sb;
  const size_t d_bytes = (size_t)a.d_rows * (a.d_rb + 2 * a.d_sb);
  const size_t sd_bytes = Ish ? (size_t)16 * dts_max * (DEC_I + 2 * DEC_DSBI) : 0;
  a.off_C = (int)o;
  a.off_D = (int)(o + (c_bytes + 127) / 128 * 128);
  o += std::max((c_bytes + 127) / 128 * 128 + d_bytes, sd_bytes);
  const size_t smem = (o + 127) / 128 * 128;
  int optin = 0;
  YN_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  if (smem > (size_t)optin)
    return fail(YN_E_UNSUPPORTED, "data-flow decode needs " + std::to_string(smem) + " B of shared memory (" +
                                      std::to_string(optin) + " available)");
  uint8_t* sc = reinterpret_cast<uint8_t*>(scratch);
  a.K = K; a.Ish = Ish; a.norm_topk = d.norm_topk; a.eps = d.rms_eps;
  a.layers = reinterpret_cast<const DecLayer*>(table);
  a.n_layers = n_layers;
  a.inputs = reinterpret_cast<const uint16_t*>(inputs);
  a.n_tokens = n_tokens;
  a.outputs = reinterpret_cast<uint16_t*>(outputs);
  a.f_logits = reinterpret_cast<unsigned long long*>(sc + S.f_logits);
  a.f_act = reinterpret_cast<unsigned long long*>(sc + S.f_act);
  a.f_ash = reinterpret_cast<unsigned long long*>(sc + S.f_ash);
  a.f_y = reinterpret_cast<unsigned long long*>(sc + S.f_y);
  a.f_h = reinterpret_cast<unsigned long long*>(sc + S.f_h);
  a.trace_ids = trace_ids;
  a.trace_h = reinterpret_cast<uint16_t*>(trace_hidden);
  a.trace_w = trace_weights;
  a.err = reinterpret_cast<int*>(sc + S.err);
  a.timing = reinterpret_cast<long long*>(timing);
  a.nr = nr;
  a.ns = ns;
  if (!al16(inputs) || !al16(outputs) || !al16(scratch) || (trace_hidden && !al16(trace_hidden)))
    return fail(YN_E_INVALID, "stack decode: inputs, outputs, scratch and trace_hidden must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  // stale epochs of an earlier launch must not match this launch's steps
  YN_CUDA(cudaMemsetAsync(sc + S.f_logits, 0, S.total - S.f_logits, st));
  const void* kernel = reinterpret_cast<const void*>(&k_stack_flow);
  if ((rc = set_smem_ptr(kernel, smem))) return rc;
  int per_sm = 0;
  YN_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, DEC_THREADS, smem));
  if (per_sm < 1) return fail(YN_E_UNSUPPORTED, "data-flow decode kernel does not fit on an SM");
  void* args[] = {&a};
  YN_CUDA(cudaLaunchCooperativeKernel(kernel, dim3(G), dim3(DEC_THREADS), args, smem, st));
  return YN_OK;
}

extern "C" int yn_stack_error(void* scratch, const yn_dims* dims, void* stream, int32_t* code_out) {
  if (!scratch || !dims) return fail(YN_E_INVALID, "null argument");
  StackScratch S = stack_scratch(*dims);
  int32_t code = 0;
  uint8_t* b = reinterpret_cast<uint8_t*>(scratch);
  YN_CUDA(cudaMemcpyAsync(&code, b + S.err, 4, cudaMemcpyDeviceToHost, as_stream(stream)));
  YN_CUDA(cudaStreamSynchronize(as_stream(stream)));
  if (code) YN_CUDA(cudaMemsetAsync(b + S.err, 0, 4, as_stream(stream)));
  if (code_out) *code_out = code;
  return code ? fail(YN_E_DEVICE, "stack decode kernel error code " + std::to_string(code)) : YN_OK;
}
