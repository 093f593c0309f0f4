// Seeded synthetic weights and activations generated directly in HBM.
//
// A counter-based generator (SplitMix64 finaliser over seed, stream id and
// element index) makes every element a pure function of (seed, stream, i), so
// the CPU oracle regenerates any record it needs bit for bit without holding
// the whole 27 GB expert set. Normal samples use the Irwin-Hall sum of four
// 16-bit uniforms (mean 131070, standard deviation 37837.227), converted with
// one exact int->float conversion, one multiply and one rounding.
#include <cuda_runtime.h>

#include "yanah_b200.h"
#include "yn_common.cuh"

namespace ynb {

__host__ __device__ inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__host__ __device__ inline uint64_t stream_key(uint64_t seed, uint64_t sid) {
  return mix64(seed ^ mix64(sid + 0x632BE59BD9B4E019ull));
}

__global__ void k_synth_u32(uint32_t* dst, int64_t n, uint64_t key) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = (uint32_t)(mix64(key + (uint64_t)i) >> 32);
}

YN_DEV float irwin_hall(uint64_t key, int64_t i) {
  const uint64_t h = mix64(key + (uint64_t)i);
  const int u = (int)(h & 0xFFFF) + (int)((h >> 16) & 0xFFFF) + (int)((h >> 32) & 0xFFFF) + (int)(h >> 48);
  return (float)(u - 131070);
}

__global__ void k_synth_f16(uint16_t* dst, int64_t n, uint64_t key, float c, int absolute) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = __fmul_rn(irwin_hall(key, i), c);
    if (absolute) v = fabsf(v);
    dst[i] = __half_as_ushort(__float2half_rn(v));
  }
}

__global__ void k_synth_bf16(uint16_t* dst, int64_t n, uint64_t key, float c, float mean) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = __fadd_rn(__fmul_rn(irwin_hall(key, i), c), mean);
    dst[i] = f32_to_bf16(v);
  }
}

}  // namespace ynb

using namespace ynb;

static int launch_grid(int64_t n) {
  int64_t b = (n + 255) / 256;
  return (int)(b < 148 * 32 ? (b > 0 ? b : 1) : 148 * 32);
}

extern "C" int yn_synth_u32(void* dst, int64_t n_words, uint64_t seed, uint64_t stream_id, void* stream) {
  if (n_words < 0 || (n_words && !dst)) return YN_E_INVALID;
  if (!n_words) return YN_OK;
  k_synth_u32<<<launch_grid(n_words), 256, 0, (cudaStream_t)stream>>>((uint32_t*)dst, n_words,
                                                                       stream_key(seed, stream_id));
  return cudaGetLastError() == cudaSuccess ? YN_OK : YN_E_CUDA;
}

extern "C" int yn_synth_f16(void* dst, int64_t n, uint64_t seed, uint64_t stream_id, float std, int32_t absolute,
                            void* stream) {
  if (n < 0 || (n && !dst)) return YN_E_INVALID;
  if (!n) return YN_OK;
  const float c = std / 37837.227f;
  k_synth_f16<<<launch_grid(n), 256, 0, (cudaStream_t)stream>>>((uint16_t*)dst, n, stream_key(seed, stream_id), c,
                                                                 absolute);
  return cudaGetLastError() == cudaSuccess ? YN_OK : YN_E_CUDA;
}

extern "C" int yn_synth_bf16(void* dst, int64_t n, uint64_t seed, uint64_t stream_id, float std, float mean,
                             void* stream) {
  if (n < 0 || (n && !dst)) return YN_E_INVALID;
  if (!n) return YN_OK;
  const float c = std / 37837.227f;
  k_synth_bf16<<<launch_grid(n), 256, 0, (cudaStream_t)stream>>>((uint16_t*)dst, n, stream_key(seed, stream_id), c,
                                                                  mean);
  return cudaGetLastError() == cudaSuccess ? YN_OK : YN_E_CUDA;
}
