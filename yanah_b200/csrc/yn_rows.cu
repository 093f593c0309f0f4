// C ABI of the persistent multi-row decode (kernel in yn_rows.cuh).
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "yanah_b200.h"
#include "yn_internal.h"
// the stack decode and expert-parallel kernels live in yn_capi.cu / yn_batch.cu
#define YN_NO_STACK_DECODE_KERNEL
#define YN_NO_BATCH_EP_KERNELS
#include "yn_rows.cuh"

using namespace ynb;

#define YN_CUDA_R(call)                                                                              \
  do {                                                                                               \
    cudaError_t e_ = (call);                                                                         \
    if (e_ != cudaSuccess) return host_fail(YN_E_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

namespace {

struct RowsScratch {
  size_t err, f_logits, f_act, f_y, f_h, total;
};
// Error word first (the stack decodes' layout, so yn_stack_error reads it),
// then the flagged-word buffers of a batch of T rows, zeroed before every
// launch.
RowsScratch rows_scratch(const yn_dims& d, int T) {
  RowsScratch S{};
  size_t o = 0;
  auto take = [&](size_t b) { size_t at = o; o = (o + b + 255) / 256 * 256; return at; };
  const size_t P = (size_t)T * d.top_k;
  S.err = take(4);
  S.f_logits = take(2 * (size_t)T * d.n_experts * 8);
  S.f_act = take(2 * P * (d.moe_inter / 2) * 8);
  S.f_y = take(2 * P * (d.hidden / 2) * 8);
  S.f_h = take(2 * (size_t)T * (d.hidden / 2) * 8);
  S.total = o;
  return S;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

size_t r128(size_t v) { return (v + 127) / 128 * 128; }

}  // namespace

extern "C" size_t yn_rows_flow_scratch_bytes(const yn_dims* dims, int32_t max_rows) {
  if (!dims || max_rows < 1 || max_rows > RF_TMAX || dims->top_k < 1) return 0;
  return rows_scratch(*dims, max_rows).total;
}

extern "C" int yn_rows_flow_decode(const yn_dims* dims, const void* table, const yn_layer* layers, int32_t n_layers,
                                   const void* inputs, int32_t n_rows, void* outputs, void* scratch,
                                   size_t scratch_bytes, int32_t* trace_ids, void* trace_hidden, float* trace_weights,
                                   int64_t* timing, void* stream) {
  if (!dims || !table || !layers || !inputs || !outputs || !scratch) return host_fail(YN_E_INVALID, "null argument");
  const yn_dims& d = *dims;
  if (n_layers < 1) return host_fail(YN_E_INVALID, "n_layers must be >= 1");

  if (n_rows < 1 || n_rows > RF_TMAX)
    return host_fail(YN_E_UNSUPPORTED, "rows decode: n_rows must be in [1, " + std::to_string(RF_TMAX) + "]");
  if (d.hidden != RF_H || d.n_experts != RF_E || d.moe_inter != RF_I || d.shared_inter != 0 || d.top_k < 1 ||
      d.top_k > RF_KMAX)
    return host_fail(YN_E_UNSUPPORTED, "rows decode is compiled for hidden 2048, 64 experts, intermediate 1536, "
                                       "no shared expert, top_k <= 8");
  const RowsScratch S = rows_scratch(d, n_rows);
  if (scratch_bytes < S.total) return host_fail(YN_E_INVALID, "scratch too small");
  for (int l = 0; l < n_layers; ++l) {
    const yn_layer& L = layers[l];
    if (L.record.bits != RF_BITS || L.record.group_size != RF_GS)
      return host_fail(YN_E_UNSUPPORTED, "rows decode: routed experts must be 4-bit with groups of 64");
    if (L.router.bits != 8 || L.router.group_size != DEC_DGS || L.router.rows != RF_E || L.router.cols != RF_H)
      return host_fail(YN_E_UNSUPPORTED, "rows decode: the router must be 8-bit (64 x 2048) with groups of 64");
    for (int i = 0; i < 9; ++i)
      if (L.record.piece_offset[i] % 16) return host_fail(YN_E_UNSUPPORTED, "rows decode: record pieces must be 16-byte aligned");
    if (!al16(L.expert_base) || L.slot_stride % 16 || L.n_slots < 1)
      return host_fail(YN_E_UNSUPPORTED, "rows decode: slot arena and stride must be 16-byte aligned");
    if (!al16(L.router.weight) || !al16(L.router.scales) || !al16(L.router.biases) || !al16(L.post_norm))
      return host_fail(YN_E_UNSUPPORTED, "rows decode: router pieces and norm must be 16-byte aligned");
  }
  if (!al16(inputs) || !al16(outputs) || !al16(scratch) || (trace_hidden && !al16(trace_hidden)))
    return host_fail(YN_E_INVALID, "rows decode: inputs, outputs, scratch and trace_hidden must be 16-byte aligned");
  int dev = 0, sms = 0, optin = 0;
  YN_CUDA_R(cudaGetDevice(&dev));
  YN_CUDA_R(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  YN_CUDA_R(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  const int G = sms;
  const int W = n_rows * (RF_H / 2);
  if (G < RF_E || (W + G - 1) / G > RF_MAX_CW)
    return host_fail(YN_E_UNSUPPORTED, "rows decode: needs at least 128 SMs (one CTA per router row, <= 64 output "
                                       "words per CTA)");
  RowsArgs a{};
  size_t o = RF_FIXED;
  a.off_x = (int)o;
  o = r128(o + (size_t)n_rows * RF_H * 2);
  a.off_xf = (int)o;
  o = r128(o + (size_t)n_rows * RF_XSU * 4);
  a.off_xg = (int)o;
  o = r128(o + (size_t)8 * RF_GSU * 8);   // eight rows always: the MMA reads the group data of all 8 columns
  a.off_ring = (int)o;
  o += (size_t)RF_WARPS * RF_NST * RF_CSLOT;
  a.off_rsc = (int)o;
  o = r128(o + (size_t)RF_WARPS * RF_NST * RF_SSLOT);
  if (o > (size_t)optin)
    return host_fail(YN_E_UNSUPPORTED, "rows decode needs " + std::to_string(o) + " B of shared memory (" +
                                           std::to_string(optin) + " available)");
  const size_t smem = o;
  uint8_t* sc = reinterpret_cast<uint8_t*>(scratch);
  a.T = n_rows;
  a.K = d.top_k;
  a.norm_topk = d.norm_topk;
  a.eps = d.rms_eps;
  a.layers = reinterpret_cast<const DecLayer*>(table);
  a.n_layers = n_layers;
  a.inputs = reinterpret_cast<const uint16_t*>(inputs);
  a.outputs = reinterpret_cast<uint16_t*>(outputs);
  a.f_logits = reinterpret_cast<u64*>(sc + S.f_logits);
  a.f_act = reinterpret_cast<u64*>(sc + S.f_act);
  a.f_y = reinterpret_cast<u64*>(sc + S.f_y);
  a.f_h = reinterpret_cast<u64*>(sc + S.f_h);
  a.P = n_rows * d.top_k;
  a.trace_ids = trace_ids;
  a.trace_h = reinterpret_cast<uint16_t*>(trace_hidden);
  a.trace_w = trace_weights;
  a.err = reinterpret_cast<int*>(sc + S.err);
  a.timing = reinterpret_cast<long long*>(timing);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // stale epochs of an earlier launch must not match this launch's layers
  YN_CUDA_R(cudaMemsetAsync(sc + S.f_logits, 0, S.total - S.f_logits, st));
  const void* kernel = reinterpret_cast<const void*>(&k_rows_flow);
  int rc = host_set_smem(kernel, smem);
  if (rc) return rc;
  int per_sm = 0;
  YN_CUDA_R(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, RF_THREADS, smem));
  if (per_sm < 1) return host_fail(YN_E_UNSUPPORTED, "rows decode kernel does not fit on an SM");
  void* args[] = {&a};
  YN_CUDA_R(cudaLaunchCooperativeKernel(kernel, dim3(G), dim3(RF_THREADS), args, smem, st));
  return YN_OK;
}
