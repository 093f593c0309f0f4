// Shared device helpers for the sparse-MoE decode kernels (sm_100a only).
//
// Contents: bf16/fp16 rounding helpers, a deterministic exp written from the
// Cody-Waite range reduction plus a degree-7 Taylor polynomial (so the CPU
// oracle can reproduce it bit for bit), warp butterfly reductions, and thin
// PTX wrappers for mbarriers and the non-tensor bulk copy engine
// (cp.async.bulk, every copy to this CTA alone).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "yanah_b200 kernels are written for sm_100a (B200) only"
#endif

#define YN_DEV __device__ __forceinline__

namespace ynb {

// ------------------------------------------------------------------ numbers
YN_DEV float bf16_to_f32(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }
YN_DEV uint16_t f32_to_bf16(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
// Round an fp32 value through bf16 (round-to-nearest-even), back to fp32.
YN_DEV float bf16r(float f) { return bf16_to_f32(f32_to_bf16(f)); }
YN_DEV float f16_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// 2^n for n in [-126, 127] built from the exponent field (exact).
YN_DEV float pow2i(int n) { return __int_as_float((n + 127) << 23); }

// exp(x) in fp32, deterministic and identical to the oracle's restatement.
// Method: Cody-Waite reduction x = n*ln2 + r (ln2 split into a 12-trailing-
// zero head and a tail), then the Taylor series of e^r to degree 7 in Horner
// form with explicit fmaf, then scaling by 2^n as two exact power-of-two
// factors. |r| <= ln2/2 keeps the truncation error below 6e-9 relative.
YN_DEV float yn_expf(float x) {
  if (!(x > -87.33654f)) return 0.0f;            // also maps NaN to 0
  if (x > 88.72283f) return __int_as_float(0x7f800000);
  float n = rintf(__fmul_rn(x, 1.44269504f));
  float r = __fmaf_rn(-n, 0.693145751953125f, x);
  r = __fmaf_rn(-n, 1.428606820309417e-06f, r);
  float p = 1.984126984e-4f;                      // 1/7!
  p = __fmaf_rn(p, r, 1.388888889e-3f);           // 1/6!
  p = __fmaf_rn(p, r, 8.333333333e-3f);           // 1/5!
  p = __fmaf_rn(p, r, 4.166666667e-2f);           // 1/4!
  p = __fmaf_rn(p, r, 1.666666667e-1f);           // 1/3!
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int ni = (int)n;
  int a = ni >> 1;
  int b = ni - a;
  return __fmul_rn(__fmul_rn(p, pow2i(a)), pow2i(b));
}

// sigmoid with the reference's bf16 rounding point (mx.sigmoid on bf16).
YN_DEV float sigmoid_f32(float g) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, yn_expf(-g))); }

// swiglu(gate, up) = silu(gate) * up, rounded to bf16 after each op as the
// reference's bf16 elementwise ops do: s = sigmoid(g), silu = g*s, out = silu*up.
YN_DEV float swiglu_bf16(float g_bf16, float u_bf16) {
  float s = bf16r(sigmoid_f32(g_bf16));
  float silu = bf16r(__fmul_rn(g_bf16, s));
  return bf16r(__fmul_rn(silu, u_bf16));
}

// Power-of-two scale that maps max|x| into [64, 128) for fp16 partial sums.
YN_DEV float fp16_input_scale(float maxabs) {
  if (!(maxabs > 0.0f)) return 1.0f;
  int e;
  frexpf(maxabs, &e);                  // maxabs = f * 2^e, f in [0.5, 1)
  int s = 7 - e;                       // maxabs * 2^s in [64, 128)
  if (s > 100) s = 100;
  if (s < -100) s = -100;
  return ldexpf(1.0f, s);
}

// ------------------------------------------------------------ reductions
// Butterfly sum over groups of `width` consecutive lanes (width = power of 2).
// With commutative fp32 addition every lane of a group ends with the same
// bits, so the oracle reproduces the result by simulating the same tree.
YN_DEV float group_sum_bfly(float v, int width) {
  for (int m = width >> 1; m > 0; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}
YN_DEV float warp_max(float v) {
  for (int m = 16; m > 0; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}
// Integer key of a finite float whose signed order is the float order (-0 below +0), and back.
YN_DEV int f32_order_key(float f) {
  const int b = __float_as_int(f);
  return b ^ ((b >> 31) & 0x7FFFFFFF);
}
YN_DEV float f32_from_order_key(int k) { return __int_as_float(k ^ ((k >> 31) & 0x7FFFFFFF)); }
// Warp maximum of finite floats as one redux instruction (the value warp_max returns; of +0 and -0, +0).
YN_DEV float warp_max_redux(float v) {
  return f32_from_order_key(__reduce_max_sync(0xffffffffu, f32_order_key(v)));
}

// ----------------------------------------------------------- time & flags
YN_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Error codes written to the workspace error word (first error wins).
enum : int {
  YN_ERR_NONE = 0,
  YN_ERR_BULK_TIMEOUT = 1,   // a bulk copy did not land within the wait limit
  YN_ERR_BAD_EXPERT = 2,     // routed expert id outside [0, n_experts)
  YN_ERR_BAD_SLOT = 3,       // slot table entry outside [0, n_slots)
};
YN_DEV void raise_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ------------------------------------------------------ mbarrier + bulk copy
YN_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

YN_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
YN_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
YN_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
YN_DEV bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
// Wait for phase completion with a wall-clock limit (1 s). On timeout the
// error word is set and false is returned; callers then skip their compute.
YN_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t phase, int* err) {
  if (mbar_try_wait(bar, phase)) return true;
  uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, phase)) return true;
    if (globaltimer_ns() - t0 > 1000000000ull) {
      raise_error(err, YN_ERR_BULK_TIMEOUT);
      return false;
    }
  }
}

// Every thread of the block waits; the result is made block-uniform so that
// no thread skips work (or returns) while others continue.
YN_DEV bool mbar_wait_block(uint64_t* bar, uint32_t phase, int* err) {
  const bool ok = mbar_wait_bounded(bar, phase, err);
  return __syncthreads_and(ok ? 1 : 0) != 0;
}

// Global -> shared bulk copy (non-tensor TMA path). dst/src 16-byte aligned,
// bytes a multiple of 16. Completion is signalled as transaction bytes on bar.
YN_DEV void bulk_g2s(void* dst_smem, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Read-only 16-byte global load that does not allocate in L1.
YN_DEV uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

}  // namespace ynb
