// Kernel argument structs and workspace layout shared by the kernels and the
// C-ABI launchers.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include "yanah_b200.h"

namespace ynb {

struct QM {  // device view of a quantised matrix
  const uint8_t* w;
  const uint16_t* s;
  const uint16_t* b;
  int rows, cols, bits, gs;
};

// Routed expert record: byte offsets of the nine pieces.
struct RecGeom {
  long long off[9];
  long long bytes;
  int bits, gs;
};

struct WsLayout {
  size_t x, logits, act_sh, sgate, ids, w, act, y, flogits, fprobs, counters, err, total;
  int n_cb;  // combine blocks per row of H
};

constexpr int CB_ROWS = 256;        // rows per combine block of the down kernel
constexpr int THREADS = 128;        // threads per CTA of every layer kernel

inline size_t align_up_sz(size_t v, size_t a) { return (v + a - 1) / a * a; }

// The workspace is laid out for the largest call (YN_MAX_ROWS rows and
// YN_MAX_TARGETS lookahead routers), so one workspace serves every call of a
// model regardless of its row count.
inline WsLayout ws_layout(const yn_dims& d) {
  WsLayout L{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o = align_up_sz(o + bytes, 256);
    return at;
  };
  const size_t T = YN_MAX_ROWS, NT = YN_MAX_TARGETS;
  const size_t H = d.hidden, E = d.n_experts, K = d.top_k, I = d.moe_inter, Ish = d.shared_inter;
  L.n_cb = (int)((H + CB_ROWS - 1) / CB_ROWS);
  // The error word and the combine counters come first, in this order, for
  // every dims: yn_moe_layer_noalloc keeps them zero across calls of
  // different shapes by zeroing only [counters, counters + size) growth.
  L.err = take(4);
  L.counters = take((1 + T * L.n_cb) * 4);
  L.x = take(T * H * 2);
  L.logits = take(T * E * 4);
  L.act_sh = take(T * (Ish ? Ish : 1) * 2);
  L.sgate = take(T * 4);
  L.ids = take(T * K * 4);
  L.w = take(T * K * 4);
  L.act = take(T * K * I * 2);
  L.y = take((T * K + T) * H * 2);
  L.flogits = take(NT * T * E * 4);
  L.fprobs = take(NT * E * 4);
  L.total = o;
  return L;
}

struct PostAttnArgs {
  int T, H, E, K, Ish, norm_topk;
  float eps;
  const uint16_t* h1;
  const uint16_t* norm;
  QM router;
  const float* rbias;
  QM sh_gate, sh_up, sg;
  int has_shared;
  int n_targets;
  const uint16_t* tnorm[YN_MAX_TARGETS];
  QM trouter[YN_MAX_TARGETS];
  const float* tbias[YN_MAX_TARGETS];
  int r_router, r_shared, r_target;
  int nt_router, nt_shared, nt_sg, nt_target, n_tiles;
  size_t tile_bytes;  // max weight bytes of one tile
  uint16_t* x;
  float* logits;
  uint16_t* act_sh;
  float* sgate;
  int32_t* ids;
  float* wts;
  float* flogits;
  float* fprobs;
  int* counter;
  int* err;
};

struct ExpertUpArgs {
  int T, H, I, K, E, n_slots;
  const uint16_t* x;       // (T, H) bf16
  const int32_t* ids;      // (T, K)
  const int32_t* slot_of;  // (E) or null
  const uint8_t* base;
  long long stride;
  RecGeom rg;
  int ncols;
  int cols[16];
  int rows;                // n-rows per tile
  int tiles_per_task;
  uint16_t* act;           // (T, K, I) bf16
  int* err;
};

struct ExpertDownArgs {
  int T, H, I, K, E, n_slots, Ish, has_shared, mode;
  const uint16_t* act;     // (T, K, I)
  const int32_t* ids;
  const float* wts;
  const int32_t* slot_of;
  const uint8_t* base;
  long long stride;
  RecGeom rg;
  QM sh_down;
  const uint16_t* act_sh;  // (T, Ish)
  const float* sgate;      // (T)
  const uint16_t* h_res;   // (T, H) or null
  uint16_t* y;             // (YN_MAX_ROWS*K, H) routed outputs [t*K + j]
  uint16_t* ysh;           // (YN_MAX_ROWS, H) shared outputs [t]
  uint16_t* out;           // (T, H)
  int* counters;           // (T, n_cb)
  int n_cb;
  int rows_routed, rows_shared;
  int tiles_routed_per_task, tiles_shared_per_token;
  int n_routed_tiles;      // T*K*tiles_routed_per_task
  int* err;
};

}  // namespace ynb
