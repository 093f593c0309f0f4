// C ABI of the tensor-core grouped expert GEMM (prefill) and its helpers:
// routing of many rows, fp16 K-permuted activations, the pair combine.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "yanah_b200.h"
#include "yn_internal.h"
#include "yn_tc.cuh"

using namespace ynb;

#define YN_CUDA_T(call)                                                                              \
  do {                                                                                               \
    cudaError_t e_ = (call);                                                                         \
    if (e_ != cudaSuccess) return host_fail(YN_E_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

namespace {
cudaStream_t as_st(void* s) { return reinterpret_cast<cudaStream_t>(s); }
size_t a256(size_t v) { return (v + 255) / 256 * 256; }

constexpr int ROUTE_MAX_ROWS = 4096;

// Route workspace: error word and the per-group counters first (fixed
// offsets, so calls with different row counts share them), then the
// row-sized arrays.
struct RouteWs {
  size_t err, counter, logits, xf32, xsum, act_sh, sgate, total;
};
RouteWs route_ws(const yn_dims& d, int rows) {
  RouteWs L{};
  size_t o = 0;
  auto take = [&](size_t b) { size_t at = o; o = a256(o + b); return at; };
  const size_t C = rows;
  L.err = take(4);
  L.counter = take((ROUTE_MAX_ROWS / 8) * 4);
  L.logits = take(C * d.n_experts * 4);
  L.xf32 = take(C * d.hidden * 4);
  L.xsum = take(C * (d.hidden / 16) * 4);
  L.act_sh = take(C * (d.shared_inter ? d.shared_inter : 1) * 2);
  L.sgate = take(C * 4);
  L.total = o;
  return L;
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library).
int encode_fn(EncodeTiled* out) {
  static std::mutex mu;
  static EncodeTiled fn = nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    YN_CUDA_T(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (!p || q != cudaDriverEntryPointSuccess)
      return host_fail(YN_E_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    fn = reinterpret_cast<EncodeTiled>(p);
  }
  *out = fn;
  return YN_OK;
}

// Row maps over `rows` rows of `cols` 16-bit elements: boxes of 64 elements x
// 16 << i rows, 128-byte swizzle (the UMMA K-major layout), zero fill.
int make_row_maps(const void* base, long long rows, int cols, bool bf16, TcMaps* maps) {
  EncodeTiled fn;
  int rc = encode_fn(&fn);
  if (rc) return rc;
  if (reinterpret_cast<uintptr_t>(base) % 16 || (cols * 2) % 16)
    return host_fail(YN_E_INVALID, "tensor-map rows must be 16-byte aligned");
  for (int i = 0; i < TC_NMAPS; ++i) {
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {64u, (cuuint32_t)(16 << i)};
    const cuuint32_t elem[2] = {1u, 1u};
    const CUresult r = fn(&maps->m[i], bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                          const_cast<void*>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return host_fail(YN_E_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  }
  return YN_OK;
}

size_t tc_smem(int Kd, int bits) {
  (void)Kd;
  const size_t ring = bits == 2 ? (size_t)TcFmt<2>::CR * TcFmt<2>::SLOT
                     : bits == 8 ? (size_t)TcFmt<8>::CR * TcFmt<8>::SLOT : (size_t)TcFmt<4>::CR * TcFmt<4>::SLOT;
  return 1024 + (size_t)TC_S * (TC_A_BYTES + TC_B_BYTES) + ring + (2 * TC_S + 4) * 8 + 16;
}
}  // namespace

extern "C" size_t yn_rows_route_bytes(const yn_dims* dims, int32_t max_rows) {
  if (!dims || max_rows < 1 || max_rows > ROUTE_MAX_ROWS) return 0;
  return route_ws(*dims, max_rows).total;
}

extern "C" int yn_rows_route(const yn_dims* dims, const yn_layer* layer, const void* h, int32_t T, void* x_out,
                             int32_t* ids_out, float* w_out, void* ws, size_t ws_bytes, void* stream) {
  if (!dims || !layer || !h || !x_out || !ids_out || !w_out || !ws) return host_fail(YN_E_INVALID, "null argument");
  if (T < 1 || T > ROUTE_MAX_ROWS) return host_fail(YN_E_UNSUPPORTED, "rows must be in [1, 4096]");
  const RouteWs L = route_ws(*dims, T);
  if (ws_bytes < L.total) return host_fail(YN_E_INVALID, "route workspace too small for this many rows");
  uint8_t* b = reinterpret_cast<uint8_t*>(ws);
  PostAttnOut o{};
  o.x = reinterpret_cast<uint16_t*>(x_out);
  o.logits = reinterpret_cast<float*>(b + L.logits);
  o.act_sh = reinterpret_cast<uint16_t*>(b + L.act_sh);
  o.sgate = reinterpret_cast<float*>(b + L.sgate);
  o.ids = ids_out;
  o.wts = w_out;
  o.err = reinterpret_cast<int*>(b + L.err);
  o.xf32 = reinterpret_cast<float*>(b + L.xf32);
  o.xsum = reinterpret_cast<float*>(b + L.xsum);
  return host_batch_dense(*dims, *layer, h, T, o, reinterpret_cast<unsigned*>(b + L.counter), as_st(stream));
}

extern "C" int yn_route_error(void* ws, const yn_dims* dims, void* stream, int32_t* code_out) {
  if (!ws || !dims || !code_out) return host_fail(YN_E_INVALID, "null argument");
  int32_t* e = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(ws) + route_ws(*dims, 1).err);
  YN_CUDA_T(cudaMemcpyAsync(code_out, e, 4, cudaMemcpyDeviceToHost, as_st(stream)));
  YN_CUDA_T(cudaStreamSynchronize(as_st(stream)));
  YN_CUDA_T(cudaMemsetAsync(e, 0, 4, as_st(stream)));
  return YN_OK;
}

extern "C" int yn_gather_f16_kperm(const void* x, const int32_t* row_of, int64_t rows, int32_t cols, void* out,
                                   void* stream) {
  if (!x || !row_of || !out || rows < 1 || cols < 8 || cols % 8) return host_fail(YN_E_INVALID, "bad rows/cols or null");
  const long long n = rows * (long long)cols;
  const int grid = (int)std::min<long long>((n / 8 + 255) / 256, 8192);
  k_gather_f16_kperm<<<grid, 256, 0, as_st(stream)>>>(reinterpret_cast<const uint16_t*>(x), row_of, rows, cols,
                                                      reinterpret_cast<uint16_t*>(out));
  YN_CUDA_T(cudaGetLastError());
  return YN_OK;
}

extern "C" int yn_gather_kperm(const void* x, const int32_t* row_of, int64_t rows, int32_t cols, int32_t bits,
                               int32_t f16, void* out, void* stream) {
  if (!x || !out || rows < 1 || cols < 16 || cols % 16) return host_fail(YN_E_INVALID, "bad rows/cols or null");
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!a16(x) || !a16(out)) return host_fail(YN_E_INVALID, "rows must be 16-byte aligned");
  const long long nu = rows * (long long)(cols / 16);
  const int grid = (int)std::min<long long>((nu + 255) / 256, 8192);
  auto xx = reinterpret_cast<const uint16_t*>(x);
  auto oo = reinterpret_cast<uint16_t*>(out);
  cudaStream_t st = as_st(stream);
  if (bits == 2) {
    if (f16) k_perm_rows<2, true><<<grid, 256, 0, st>>>(xx, row_of, rows, cols, oo);
    else k_perm_rows<2, false><<<grid, 256, 0, st>>>(xx, row_of, rows, cols, oo);
  } else if (bits == 4) {
    if (f16) k_perm_rows<4, true><<<grid, 256, 0, st>>>(xx, row_of, rows, cols, oo);
    else k_perm_rows<4, false><<<grid, 256, 0, st>>>(xx, row_of, rows, cols, oo);
  } else if (bits == 8) {
    if (f16) k_perm_rows<8, true><<<grid, 256, 0, st>>>(xx, row_of, rows, cols, oo);
    else k_perm_rows<8, false><<<grid, 256, 0, st>>>(xx, row_of, rows, cols, oo);
  } else {
    return host_fail(YN_E_UNSUPPORTED, "bits must be 2, 4 or 8");
  }
  YN_CUDA_T(cudaGetLastError());
  return YN_OK;
}

extern "C" int yn_scale_rows(const void* y, const float* scale, int64_t rows, int32_t cols, void* out, void* stream) {
  if (!y || !scale || !out || rows < 1 || cols < 1) return host_fail(YN_E_INVALID, "bad rows/cols or null");
  const long long n = rows * (long long)cols;
  const int grid = (int)std::min<long long>((n + 255) / 256, 8192);
  k_scale_rows<<<grid, 256, 0, as_st(stream)>>>(reinterpret_cast<const uint16_t*>(y), scale, rows, cols,
                                                reinterpret_cast<uint16_t*>(out));
  YN_CUDA_T(cudaGetLastError());
  return YN_OK;
}

extern "C" int yn_rows_route_shared(const yn_dims* dims, int32_t T, void* ws, void** act_sh, float** sgate) {
  if (!dims || !ws || !act_sh || !sgate) return host_fail(YN_E_INVALID, "null argument");
  if (T < 1 || T > ROUTE_MAX_ROWS) return host_fail(YN_E_UNSUPPORTED, "rows must be in [1, 4096]");
  const RouteWs L = route_ws(*dims, T);
  *act_sh = reinterpret_cast<uint8_t*>(ws) + L.act_sh;
  *sgate = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + L.sgate);
  return YN_OK;
}

extern "C" int yn_to_f16_kperm(const void* x, int64_t rows, int32_t cols, void* out, void* stream) {
  if (!x || !out || rows < 1 || cols < 8 || cols % 8) return host_fail(YN_E_INVALID, "bad rows/cols or null");
  const long long n = rows * (long long)cols;
  const int grid = (int)std::min<long long>((n + 255) / 256, 4096);
  k_to_f16_kperm<<<grid, 256, 0, as_st(stream)>>>(reinterpret_cast<const uint16_t*>(x), n, cols,
                                                  reinterpret_cast<uint16_t*>(out));
  YN_CUDA_T(cudaGetLastError());
  return YN_OK;
}

extern "C" int yn_tc_experts(const yn_dims* dims, const yn_layer* layer, int32_t mode, const yn_tc_tile* tiles,
                             int32_t n_tiles, const int32_t* n_tiles_dev, const void* b_rows, int64_t n_rows,
                             void* act_out, void* y_out, int32_t* err, void* stream) {
  if (!dims || !layer || !tiles || !b_rows || !err) return host_fail(YN_E_INVALID, "null argument");
  if (n_rows < 1) return host_fail(YN_E_INVALID, "n_rows must be positive");
  if (mode != 0 && mode != 1) return host_fail(YN_E_INVALID, "mode must be 0 (gate/up) or 1 (down)");
  if (mode == 0 && !act_out) return host_fail(YN_E_INVALID, "gate/up needs act_out");
  if (mode == 1 && !y_out) return host_fail(YN_E_INVALID, "down needs y_out");
  const yn_record& r = layer->record;
  const bool fmt_ok = (r.bits == 4 && r.group_size == 64) || (r.bits == 2 && (r.group_size == 64 || r.group_size == 32)) ||
                      (mode == 1 && r.bits == 8 && r.group_size == 64);
  if (!fmt_ok)
    return host_fail(YN_E_UNSUPPORTED, "tensor-core expert GEMM: records must be 4-bit g64 or 2-bit g64/g32 "
                                       "(8-bit g64 for the down projection)");
  const int H = dims->hidden, I = dims->moe_inter;
  if (H % 512 || I % 512)  // whole 128-row down tiles, 64-unit gate/up tiles, scale rows in 8-group blocks
    return host_fail(YN_E_UNSUPPORTED, "tensor-core expert GEMM: hidden and moe_inter must be multiples of 512");
  if (!layer->expert_base || reinterpret_cast<uintptr_t>(layer->expert_base) % 16 || layer->slot_stride % 16)
    return host_fail(YN_E_INVALID, "expert arena and slot stride must be 16-byte aligned");
  for (int i = 0; i < 9; ++i)
    if (r.piece_offset[i] % 16) return host_fail(YN_E_INVALID, "record pieces must be 16-byte aligned");
  if (n_tiles < 1) return YN_OK;
  TcArgs a{};
  a.tiles = reinterpret_cast<const TcTile*>(tiles);
  a.n_tiles = n_tiles;
  a.n_tiles_dev = n_tiles_dev;
  a.base = reinterpret_cast<const uint8_t*>(layer->expert_base);
  a.stride = layer->slot_stride;
  a.slot_of = layer->expert_slot;
  a.n_slots = layer->n_slots;
  for (int i = 0; i < 9; ++i) a.rg.off[i] = r.piece_offset[i];
  a.rg.bytes = r.record_bytes;
  a.rg.bits = r.bits;
  a.rg.gs = r.group_size;
  a.H = H;
  a.I = I;
  a.act_out = reinterpret_cast<uint16_t*>(act_out);
  a.y_out = reinterpret_cast<uint16_t*>(y_out);
  a.err = err;
  const size_t smem = tc_smem(mode == 0 ? H : I, r.bits);
  const int fi = r.bits == 8 ? 3 : r.bits == 4 ? 0 : r.group_size == 64 ? 1 : 2;
  const void* kern0[3] = {reinterpret_cast<const void*>(k_tc_experts<0, 4, 64>),
                          reinterpret_cast<const void*>(k_tc_experts<0, 2, 64>),
                          reinterpret_cast<const void*>(k_tc_experts<0, 2, 32>)};
  const void* kern1[4] = {reinterpret_cast<const void*>(k_tc_experts<1, 4, 64>),
                          reinterpret_cast<const void*>(k_tc_experts<1, 2, 64>),
                          reinterpret_cast<const void*>(k_tc_experts<1, 2, 32>),
                          reinterpret_cast<const void*>(k_tc_experts<1, 8, 64>)};
  const void* kern = mode == 0 ? kern0[fi] : kern1[fi];
  int rc = host_set_smem(kern, smem);
  if (rc) return rc;
  int dev = 0, sms = 0;
  YN_CUDA_T(cudaGetDevice(&dev));
  YN_CUDA_T(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int grid = std::max(1, std::min(n_tiles, sms));  // persistent: one CTA per SM walks the tiles
  TcMaps maps;
  if ((rc = make_row_maps(b_rows, n_rows, mode == 0 ? H : I, mode == 1, &maps))) return rc;
  void* args[] = {&a, &maps};
  YN_CUDA_T(cudaLaunchKernel(kern, dim3(grid), dim3(TCW_THREADS), args, smem, as_st(stream)));
  YN_CUDA_T(cudaGetLastError());
  return YN_OK;
}

extern "C" int yn_pairs_combine(const yn_dims* dims, const void* y, const int32_t* pair_of, const float* weights,
                                const void* y_shared, const void* h_res, int32_t T, void* out, void* stream) {
  if (!dims || !y || !pair_of || !weights || !out || T < 1) return host_fail(YN_E_INVALID, "null argument or T < 1");
  const int H = dims->hidden;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (H % 8 == 0 && a16(y) && a16(out) && (!y_shared || a16(y_shared)) && (!h_res || a16(h_res))) {
    dim3 grid((H / 8 + 255) / 256, T);
    k_pairs_combine8<<<grid, 256, 0, as_st(stream)>>>(
        reinterpret_cast<const uint16_t*>(y), pair_of, weights, reinterpret_cast<const uint16_t*>(y_shared),
        reinterpret_cast<const uint16_t*>(h_res), H, dims->top_k, reinterpret_cast<uint16_t*>(out));
    YN_CUDA_T(cudaGetLastError());
    return YN_OK;
  }
  dim3 grid((H + 255) / 256, T);
  k_pairs_combine<<<grid, 256, 0, as_st(stream)>>>(
      reinterpret_cast<const uint16_t*>(y), pair_of, weights, reinterpret_cast<const uint16_t*>(y_shared),
      reinterpret_cast<const uint16_t*>(h_res), H, dims->top_k, reinterpret_cast<uint16_t*>(out));
  YN_CUDA_T(cudaGetLastError());
  return YN_OK;
}

extern "C" int yn_prefill_max_tiles(const yn_dims* dims, int32_t T, int32_t* max_up, int32_t* max_dn) {
  if (!dims || !max_up || !max_dn || T < 1) return host_fail(YN_E_INVALID, "null argument or T < 1");
  const long long chunks = (long long)dims->n_experts + ((long long)T * dims->top_k + TC_NMAX - 1) / TC_NMAX;
  *max_up = (int32_t)(chunks * (dims->moe_inter / 64));
  *max_dn = (int32_t)(chunks * (dims->hidden / 128));
  return YN_OK;
}

extern "C" int yn_prefill_plan(const yn_dims* dims, const int32_t* ids, int32_t T, int32_t* pair_row, int32_t* pair_of,
                               yn_tc_tile* tiles_up, int32_t max_up, yn_tc_tile* tiles_dn, int32_t max_dn,
                               int32_t* n_tiles, int32_t* err, void* stream) {
  if (!dims || !ids || !pair_row || !pair_of || !tiles_up || !tiles_dn || !n_tiles || !err)
    return host_fail(YN_E_INVALID, "null argument");
  if (T < 1 || (long long)T * dims->top_k > 65536) return host_fail(YN_E_UNSUPPORTED, "T * top_k must be in [1, 65536]");
  if (dims->n_experts > 1024) return host_fail(YN_E_UNSUPPORTED, "at most 1024 experts");
  PrefillPlanArgs a{};
  a.ids = ids;
  a.T = T;
  a.K = dims->top_k;
  a.E = dims->n_experts;
  a.H = dims->hidden;
  a.I = dims->moe_inter;
  a.pair_row = pair_row;
  a.pair_of = pair_of;
  a.up = reinterpret_cast<TcTile*>(tiles_up);
  a.max_up = max_up;
  a.dn = reinterpret_cast<TcTile*>(tiles_dn);
  a.max_dn = max_dn;
  a.n_tiles = n_tiles;
  a.err = err;
  k_prefill_plan<<<1, PLAN_THREADS, 0, as_st(stream)>>>(a);
  YN_CUDA_T(cudaGetLastError());
  return YN_OK;
}
