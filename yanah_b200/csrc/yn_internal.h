// Host-side helpers shared by the C-ABI translation units.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "yanah_b200.h"

namespace ynb {

// Record the message for yn_last_error and return `code`.
int host_fail(int code, const std::string& msg);

// Validation of one quantised matrix (shape, bit width, group size, alignment).
int host_check_qmat(const yn_qmat& m, int rows, int cols, int bits, const char* what);

// Raise a kernel's dynamic shared-memory limit (once per device).
int host_set_smem(const void* kernel, size_t bytes);

// Output arrays of the post-attention kernel (rows 0..T-1 of each).
struct PostAttnOut {
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
  float* xf32;   // batch path only: (T, H) normalised rows in fp32 (dot-kernel layout)
  float* xsum;   // batch path only: (T, H / 16) chunk sums
};

// Post-attention + routing for any number of rows, in launches of at most
// YN_MAX_ROWS rows (no lookahead routers).
int host_post_attention_rows(const yn_dims& d, const yn_layer& L, const void* h1, int T, const PostAttnOut& o,
                             cudaStream_t st);

// Post-attention + routing of up to 4096 rows (k_batch_dense): bit-identical
// to the single-row path, spread over (router rows x 8 tokens) tiles.
// `counter`: ceil(T / 8) device words that only this call sequence uses
// (monotonic; zero before the first call).
int host_batch_dense(const yn_dims& d, const yn_layer& L, const void* h, int T, const PostAttnOut& o,
                     unsigned* counter, cudaStream_t st);

}  // namespace ynb
