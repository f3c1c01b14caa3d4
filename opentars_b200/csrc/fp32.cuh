// The tars_mini fp32 numeric contract as CUDA device functions.
//
// Each function restates one function of the reference's tars_mini/numerics.py (cited per
// function). Contract: one round-to-nearest-even per step, operands and results flushed to a
// signed zero when denormal, no fused multiply-add, every NaN a step produces is 0x7FC00000.
// The library is compiled with -ftz=false -fmad=false: products use __fmul_rn (IEEE with gradual
// underflow, never contracted) and are flushed explicitly afterwards, which is what numpy's
// float32 multiply followed by the reference's ftz() computes, including products that round up
// to the smallest normal; sums use the hardware's flush-to-zero add, exact for sums (see fadd). exp/recip/rsqrt are the contract's own published sequences
// (magic-constant seeds, Newton steps in correction form, a degree-6 Horner polynomial); CUDA's
// math library is not used for them.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace tc {

__device__ __forceinline__ uint32_t fb(float x) { return __float_as_uint(x); }
__device__ __forceinline__ float bf(uint32_t b) { return __uint_as_float(b); }
__device__ __forceinline__ bool is_nan(float x) { return (fb(x) & 0x7FFFFFFFu) > 0x7F800000u; }

// numerics.py:26-31
__device__ __forceinline__ float ftz(float x) {
  const uint32_t b = fb(x);
  return (b & 0x7F800000u) ? x : bf(b & 0x80000000u);
}
// numerics.py:34-37
__device__ __forceinline__ float canon(float x) { return is_nan(x) ? bf(0x7FC00000u) : x; }
// numerics.py:40-47. fmul: IEEE product with gradual underflow, then the flush (a product just
// below 2^-126 may round up to the smallest normal, so the hardware's flush-to-zero multiply,
// which judges tininess on the 24-bit rounded value, could differ). fadd: the hardware's
// flush-to-zero add is exact here: both operands are multiples of 2^-149, so a sum below 2^-126
// is exactly representable, is never rounded, and is flushed with its sign either way.
__device__ __forceinline__ float fmul(float a, float b) { return canon(ftz(__fmul_rn(ftz(a), ftz(b)))); }
// The product of operands already flushed (values this library stored): only the result's
// flush remains; a NaN it returns is canonicalised by the caller where the value is kept.
__device__ __forceinline__ float fmul_ff(float a, float b) { return ftz(__fmul_rn(a, b)); }
__device__ __forceinline__ float fadd_nc(float a, float b) {   // without canonicalising NaN
  float r;
  asm("add.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float fadd(float a, float b) { return canon(fadd_nc(a, b)); }
// numerics.py:50-52
__device__ __forceinline__ float i2f(int v) { return __int2float_rn(v); }
// numerics.py:111-113
__device__ __forceinline__ float neg(float x) { return bf(fb(x) ^ 0x80000000u); }
// numerics.py:265-267
__device__ __forceinline__ float fabs_c(float x) { return bf(fb(ftz(x)) & 0x7FFFFFFFu); }

// numerics.py:126-132: e added to the biased exponent of a positive normal y (>= 255: +inf, <= 0: +0)
__device__ __forceinline__ float add_exp(float y, int e) {
  const uint32_t b = fb(y);
  const int ne = (int)((b >> 23) & 0xFF) + e;
  if (ne >= 255) return bf(0x7F800000u);
  if (ne <= 0) return 0.0f;
  return bf(((uint32_t)ne << 23) | (b & 0x7FFFFFu));
}

// numerics.py:135-150
__device__ __forceinline__ float exp_f(float x) {
  x = ftz(x);
  float n = rintf(fmul(x, bf(0x3FB8AA3Bu)));
  n = fminf(fmaxf(n, -200.0f), 200.0f);
  const float r = fadd(fadd(x, fmul(n, bf(0xBF317200u))), fmul(n, bf(0xB5BFBE8Eu)));
  float p = bf(0x3AB60B61u);
  p = fadd(fmul(p, r), bf(0x3C088889u));
  p = fadd(fmul(p, r), bf(0x3D2AAAABu));
  p = fadd(fmul(p, r), bf(0x3E2AAAABu));
  p = fadd(fmul(p, r), bf(0x3F000000u));
  p = fadd(fmul(p, r), bf(0x3F800000u));
  p = fadd(fmul(p, r), bf(0x3F800000u));
  float y = add_exp(p, is_nan(n) ? 0 : (int)n);
  if (x >= 89.0f) y = bf(0x7F800000u);
  else if (x <= -104.0f) y = 0.0f;
  if (is_nan(x)) y = bf(0x7FC00000u);
  return canon(y);
}

// numerics.py:153-168
__device__ __forceinline__ float recip_f(float x) {
  x = ftz(x);
  const uint32_t b = fb(x), sgn = b & 0x80000000u, a = b & 0x7FFFFFFFu;
  const uint32_t mb = (a & 0x7FFFFFu) | (127u << 23);
  const float m = bf(mb);
  float y = bf(0x7EF311C7u - mb);
  const float one = 1.0f;
#pragma unroll
  for (int i = 0; i < 3; ++i) y = fadd(y, fmul(y, fadd(one, neg(fmul(m, y)))));
  y = bf(fb(add_exp(y, -((int)(a >> 23) - 127))) | sgn);
  if (a == 0) y = bf(sgn | 0x7F800000u);
  if (a == 0x7F800000u) y = bf(sgn);
  if (is_nan(x)) y = bf(0x7FC00000u);
  return canon(y);
}

// numerics.py:171-191
__device__ __forceinline__ float rsqrt_f(float x) {
  x = ftz(x);
  const uint32_t b = fb(x);
  const int E = (int)((b >> 23) & 0xFF) - 127;
  const int j = E & 1;
  const int k = (E - j) / 2;  // floor(E / 2)
  const uint32_t mb = (b & 0x7FFFFFu) | ((uint32_t)(127 + j) << 23);
  const float m = bf(mb);
  float y = bf(0x5F3759DFu - (mb >> 1));
  const float half = 0.5f;
#pragma unroll
  for (int i = 0; i < 3; ++i) y = fadd(y, fmul(y, fadd(half, neg(fmul(half, fmul(fmul(m, y), y))))));
  y = add_exp(y, -k);
  if ((b & 0x7FFFFFFFu) == 0) y = bf((b & 0x80000000u) | 0x7F800000u);
  if (b == 0x7F800000u) y = 0.0f;
  if (is_nan(x) || x < 0.0f) y = bf(0x7FC00000u);
  return canon(y);
}

// numerics.py:194-201
__device__ __forceinline__ float gelu_f(float x) {
  x = ftz(x);
  const float x3 = fmul(fmul(x, x), x);
  const float u = fmul(bf(0x3F4C422Au), fadd(x, fmul(bf(0x3D372713u), x3)));
  const float t = fadd(1.0f, neg(fmul(2.0f, recip_f(fadd(exp_f(fmul(2.0f, u)), 1.0f)))));
  return fmul(fmul(0.5f, x), fadd(1.0f, t));
}
// numerics.py:204-207
__device__ __forceinline__ float silu_f(float x) {
  x = ftz(x);
  return fmul(x, recip_f(fadd(1.0f, exp_f(neg(x)))));
}
// numerics.py:241-244
__device__ __forceinline__ float sigmoid_f(float x) {
  x = ftz(x);
  return recip_f(fadd(1.0f, exp_f(neg(x))));
}
// numerics.py:247-262
__device__ __forceinline__ float softplus_f(float x) {
  x = ftz(x);
  const float t = exp_f(neg(fabs_c(x)));
  const float s = fmul(t, recip_f(fadd(t, 2.0f)));
  const float z = fmul(s, s);
  float p = bf(0x3D70F0F1u);
  p = fadd(fmul(p, z), bf(0x3D888889u));
  p = fadd(fmul(p, z), bf(0x3D9D89D9u));
  p = fadd(fmul(p, z), bf(0x3DBA2E8Cu));
  p = fadd(fmul(p, z), bf(0x3DE38E39u));
  p = fadd(fmul(p, z), bf(0x3E124925u));
  p = fadd(fmul(p, z), bf(0x3E4CCCCDu));
  p = fadd(fmul(p, z), bf(0x3EAAAAABu));
  p = fadd(fmul(p, z), 1.0f);
  float y = fadd(x > 0.0f ? x : 0.0f, fmul(fmul(2.0f, s), p));
  if (x > 20.0f) y = x;
  if (is_nan(x)) y = bf(0x7FC00000u);
  return canon(y);
}

// numerics.py:210-230: 0 none, 1 relu, 2 relu6, 3 gelu, 4 silu, 5 sigmoid, 6 softplus, 7 exp
__device__ __forceinline__ float act_fn(float x, int act) {
  x = ftz(x);
  switch (act) {
    case 0: return x;
    case 1: return x > 0.0f ? x : 0.0f;
    case 2: { const float r = x > 0.0f ? x : 0.0f; return r > 6.0f ? 6.0f : r; }
    case 3: return gelu_f(x);
    case 4: return silu_f(x);
    case 5: return sigmoid_f(x);
    case 6: return softplus_f(x);
    default: return exp_f(x);
  }
}

// act_fn with the transcendental cases (3-7) in one out-of-line function: for epilogues that run
// the activation inside long per-element loops, whose body must stay small in the instruction
// cache. The same results as act_fn.
static __device__ __noinline__ float act_transcendental(float x, int act) {
  switch (act) {
    case 3: return gelu_f(x);
    case 4: return silu_f(x);
    case 5: return sigmoid_f(x);
    case 6: return softplus_f(x);
    default: return exp_f(x);
  }
}
__device__ __forceinline__ float act_fn_lean(float x, int act) {
  x = ftz(x);
  if (act == 0) return x;
  if (act == 1) return x > 0.0f ? x : 0.0f;
  if (act == 2) { const float r = x > 0.0f ? x : 0.0f; return r > 6.0f ? 6.0f : r; }
  return act_transcendental(x, act);
}

// numerics.py:293-303: NaN wins; equal values (+0 / -0 included) give the AND of the sign bits
__device__ __forceinline__ float fmax_c(float a, float b) {
  a = ftz(a);
  b = ftz(b);
  if (is_nan(a) || is_nan(b)) return bf(0x7FC00000u);
  if (a == b) return bf((fb(a) & fb(b) & 0x80000000u) | (fb(a) & 0x7FFFFFFFu));
  return a > b ? a : b;
}

// numerics.py:270-275
__device__ __forceinline__ uint16_t to_bf16(float y) {
  const uint32_t b = fb(ftz(y));
  if ((b & 0x7F800000u) == 0x7F800000u && (b & 0x7FFFFFu)) return 0x7FC0;
  return (uint16_t)((b + 0x7FFFu + ((b >> 16) & 1u)) >> 16);
}
// numerics.py:14-18
__device__ __forceinline__ uint16_t to_fp16(float y) {
  if (is_nan(y)) return 0x7E00;
  return __half_as_ushort(__float2half_rn(y));
}
// numerics.py:21-23
__device__ __forceinline__ float from_fp16(uint16_t h) { return canon(__half2float(__ushort_as_half(h))); }
// numerics.py:278-279
__device__ __forceinline__ float from_bf16(uint16_t h) { return bf((uint32_t)h << 16); }

// numerics.py:282-286
__device__ __forceinline__ int8_t q8(float x, float inv) {
  float y = fmul(x, inv);
  if (is_nan(y)) y = 0.0f;
  y = rintf(y);
  y = fminf(fmaxf(y, -127.0f), 127.0f);
  return (int8_t)(int)y;
}

// --------------------------------------------------------------------------- memory helpers
// Loads at addresses that may be only byte aligned (a BASE_ADDR that is not a multiple of 16
// makes every tensor of the descriptor unaligned; the contract allows it).
__device__ __forceinline__ uint32_t ld_u32(const uint8_t* p) {
  if (((uintptr_t)p & 3) == 0) return *reinterpret_cast<const uint32_t*>(p);
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
__device__ __forceinline__ uint16_t ld_u16(const uint8_t* p) {
  if (((uintptr_t)p & 1) == 0) return *reinterpret_cast<const uint16_t*>(p);
  return (uint16_t)(p[0] | (p[1] << 8));
}
__device__ __forceinline__ float ld_f32(const uint8_t* p) { return bf(ld_u32(p)); }
__device__ __forceinline__ void st_u32(uint8_t* p, uint32_t v) {
  if (((uintptr_t)p & 3) == 0) { *reinterpret_cast<uint32_t*>(p) = v; return; }
  p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); p[2] = (uint8_t)(v >> 16); p[3] = (uint8_t)(v >> 24);
}
__device__ __forceinline__ void st_u16(uint8_t* p, uint16_t v) {
  if (((uintptr_t)p & 1) == 0) { *reinterpret_cast<uint16_t*>(p) = v; return; }
  p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8);
}

// Asynchronous 16-byte global -> shared copies (both addresses 16-byte aligned): a staging loop
// issues all of its copies before waiting once, instead of one dependent load per iteration.
__device__ __forceinline__ void cp16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// golden.py:273-280: one output element in the descriptor's format (fp32 flushed, bf16 RNE,
// int8 via q8 with OUT_SCALE, fp16 IEEE RNE)
__device__ __forceinline__ void store_out(uint8_t* row, int n, float y, int out, float out_scale) {
  switch (out) {
    case 0: st_u32(row + 4 * n, fb(ftz(y))); break;
    case 1: st_u16(row + 2 * n, to_bf16(y)); break;
    case 2: row[n] = (uint8_t)q8(y, out_scale); break;
    default: st_u16(row + 2 * n, to_fp16(y)); break;
  }
}

}  // namespace tc
