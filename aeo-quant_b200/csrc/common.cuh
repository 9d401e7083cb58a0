// Shared device numerics for the quantized MoE expert path (sm_100a).
//
// Formats (aeo_quant src/aeo_quant/gpu/quant.py:15-27):
//   * FP4 E2M1 nibble: bit 3 = sign, bits 0-2 = magnitude index into
//     {0, .5, 1, 1.5, 2, 3, 4, 6}; two nibbles per byte, HIGH nibble = even k.
//   * e4m3fn block scale per 16 elements along K.
//   * per-tensor scale in the input dtype (bf16 for activations).
// All arithmetic that decides a quantized bit is IEEE round-to-nearest: the
// library is built without fast-math, and divisions are correctly rounded
// (div_rn below).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/aeoq.h"

namespace aeoq {

// ---------------------------------------------------------------------------
// host-side error plumbing
// ---------------------------------------------------------------------------
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);

// Per-device launch set-up. Function attributes belong to the context of the
// device that is current when they are set, and the SM count is a property of
// that device, so both are cached per (device, function) under a mutex: a
// process that drives several GPUs sets each attribute once on each of them.
// func_smem_attr raises the function's dynamic shared-memory limit to at
// least `bytes` on the current device (and, with carveout >= 0, its preferred
// shared-memory carveout); returns AEOQ_OK or an AEOQ error code.
int func_smem_attr(const void* func, size_t bytes, int carveout, const char* what);
// Multiprocessor count of the current device (148 on B200).
int device_sm_count();

#define AEOQ_REQUIRE(cond, code, ...)                     \
  do {                                                    \
    if (!(cond)) return ::aeoq::set_error((code), __VA_ARGS__); \
  } while (0)

constexpr float kFp4Max = 6.0f;
constexpr float kFp8Max = 448.0f;
constexpr float kNvfp4Denom = 2688.0f;  // 6 * 448

// ---------------------------------------------------------------------------
// input dtypes
// ---------------------------------------------------------------------------
template <int DT> struct In;
template <> struct In<AEOQ_BF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float load(const T* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ float to_f(T v) { return __bfloat162float(v); }
  static __device__ __forceinline__ float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
  static __device__ __forceinline__ void store(void* p, float v) { *reinterpret_cast<T*>(p) = __float2bfloat16_rn(v); }
  // |x| as an order-preserving integer; NaN patterns sort above infinity.
  static __device__ __forceinline__ uint32_t abs_key(T v) { return __bfloat16_as_ushort(v) & 0x7FFFu; }
  static __device__ __forceinline__ float key_to_f(uint32_t k) { return __bfloat162float(__ushort_as_bfloat16((unsigned short)k)); }
};
template <> struct In<AEOQ_F16> {
  using T = __half;
  static __device__ __forceinline__ float load(const T* p) { return __half2float(*p); }
  static __device__ __forceinline__ float to_f(T v) { return __half2float(v); }
  static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
  static __device__ __forceinline__ void store(void* p, float v) { *reinterpret_cast<T*>(p) = __float2half_rn(v); }
  static __device__ __forceinline__ uint32_t abs_key(T v) { return __half_as_ushort(v) & 0x7FFFu; }
  static __device__ __forceinline__ float key_to_f(uint32_t k) { return __half2float(__ushort_as_half((unsigned short)k)); }
};
template <> struct In<AEOQ_F32> {
  using T = float;
  static __device__ __forceinline__ float load(const T* p) { return *p; }
  static __device__ __forceinline__ float to_f(T v) { return v; }
  static __device__ __forceinline__ float round(float v) { return v; }
  static __device__ __forceinline__ void store(void* p, float v) { *reinterpret_cast<T*>(p) = v; }
  static __device__ __forceinline__ uint32_t abs_key(T v) { return __float_as_uint(v) & 0x7FFFFFFFu; }
  static __device__ __forceinline__ float key_to_f(uint32_t k) { return __uint_as_float(k); }
};

__device__ __forceinline__ float nan_max(float a, float b) {
  // max that propagates NaN like torch.amax / clamp
  return (a != a || b != b) ? __int_as_float(0x7FC00000) : fmaxf(a, b);
}

// ---------------------------------------------------------------------------
// float -> e4m3fn code, round-to-nearest-even; values that round past 448,
// infinities and NaN map to the NaN code 0x7F (sign kept). This is torch's
// float8_e4m3fn conversion rule, written from the format definition.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t e4m3_encode(float x) {
  uint32_t b = __float_as_uint(x);
  uint32_t sign = (b >> 24) & 0x80u;
  uint32_t a = b & 0x7FFFFFFFu;
  uint32_t code;
  if (a >= 0x7F800000u) {
    code = 0x7Fu;
  } else if (a >= 0x3C800000u) {            // >= 2^-6: normal
    code = ((a + 0x7FFFFu + ((a >> 20) & 1u)) >> 20) - (120u << 3);
    if (code > 0x7Eu) code = 0x7Fu;
  } else {                                  // subnormal: k * 2^-9, k in [0, 8]
    code = __float2uint_rn(__uint_as_float(a) * 512.0f);
  }
  return sign | code;
}

__device__ __forceinline__ float e4m3_decode(uint32_t c) {
  uint32_t e = (c >> 3) & 0xFu, m = c & 7u;
  float v;
  if (e == 0) v = (float)m * (1.0f / 512.0f);
  else v = __uint_as_float(((e + 120u) << 23) | (m << 20));
  if ((c & 0x7Fu) == 0x7Fu) v = __int_as_float(0x7FC00000);
  return (c & 0x80u) ? -v : v;
}

// two e4m3 codes (low byte first) -> half2 (exact; e4m3 is a subset of fp16)
__device__ __forceinline__ __half2 e4m3x2_to_half2(uint16_t two) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(two));
  return *reinterpret_cast<__half2*>(&r);
}

// ---------------------------------------------------------------------------
// FP4 E2M1 binning: count of midpoints {.25,.75,1.25,1.75,2.5,3.5,5} strictly
// below |q| (ties go to the smaller magnitude), NaN -> 7, sign = (q < 0).
// Restates _round_to_fp4_e2m1 (quant.py:121-130) incl. its clamp (:177).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t fp4_nibble(float q) {
  if (q != q) return 7u;
  float m = fabsf(q);
  uint32_t idx = (m > 0.25f) + (m > 0.75f) + (m > 1.25f) + (m > 1.75f) +
                 (m > 2.5f) + (m > 3.5f) + (m > 5.0f);
  return ((q < 0.0f) ? 8u : 0u) | idx;
}

// Exact FP4 magnitude of a nibble as float (for building exact operands).
__device__ __forceinline__ float fp4_value(uint32_t nib) {
  const uint32_t m = nib & 7u;
  // 0, .5, 1, 1.5, 2, 3, 4, 6  == (m<2 ? m*.5 : (2+(m&1)) * 2^((m>>1)-2))
  float v = (m < 2u) ? 0.5f * (float)m : (float)(2u + (m & 1u)) * __uint_as_float((127u + (m >> 1) - 2u) << 23);
  return (nib & 8u) ? -v : v;
}

// ---------------------------------------------------------------------------
// Correctly rounded float division (IEEE round-to-nearest-even), the rounding
// every quantized bit of the reference depends on.
//
// div_rn_core: one Newton-Raphson step on an approximate reciprocal
// (q = a*y, r = a - q*b, q += r*y; Markstein, IBM J. Res. Dev. 34(1), 1990)
// leaves q within about half an ulp of a/b, so the rounded quotient is q or
// its neighbour toward a/b. Both remainders a - q*b are exact in one fma
// (each candidate is within an ulp of a/b and nothing underflows in the
// operand range below), and |a - q*b| = |b| * |a/b - q| orders the candidates
// by distance: the smaller remainder wins, equal remainders are a tie and go
// to the even significand. Valid for a == 0 or 2^-80 <= |a| <= 2^80, and
// 2^-40 <= |b| <= 2^40; div_rn checks that and otherwise calls the
// compiler's __fdiv_rn (out of line, so the common path carries no trace of
// it). Tested bit for bit against __fdiv_rn over every significand pair of
// the quantizers' operand domains.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float div_rn_core(float a, float b) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(b));
  float q = a * y;
  float r = fmaf(-q, b, a);
  q = (r != 0.0f) ? fmaf(r, y, q) : q;   // keeps the sign of a zero quotient
  r = fmaf(-q, b, a);
  const uint32_t qb = __float_as_uint(q);
  const bool up = (r > 0.0f) == (b > 0.0f);              // a/b lies above q
  const uint32_t nb = (up == (q > 0.0f)) ? qb + 1u : qb - 1u;
  const float q2 = __uint_as_float(nb);
  const float d1 = fabsf(r), d2 = fabsf(fmaf(-q2, b, a));
  const bool take = (r != 0.0f) && (d2 < d1 || (d2 == d1 && (nb & 1u) == 0u));
  return take ? q2 : q;
}

static __device__ __noinline__ float div_rn_slow(float a, float b) { return __fdiv_rn(a, b); }

__device__ __forceinline__ float div_rn(float a, float b) {
  const float aa = fabsf(a), ab = fabsf(b);
  const bool in_range = (aa == 0.0f || (aa >= 0x1p-80f && aa <= 0x1p80f)) && ab >= 0x1p-40f && ab <= 0x1p40f;
  if (__builtin_expect(in_range, 1)) return div_rn_core(a, b);
  return div_rn_slow(a, b);
}

// Tensor scale from the (abs) amax, in the input dtype: quant.py:167-168.
template <int DT>
__device__ __forceinline__ float nvfp4_tensor_scale(float amax) {
  float t = In<DT>::round(div_rn(amax, kNvfp4Denom));
  float floor_v = In<DT>::round(1e-12f);
  return nan_max(t, floor_v);
}

// Elements of a block whose operands leave div_rn_core's range: the same
// steps with the compiler's division, out of line.
static __device__ __noinline__ void nvfp4_block_nibbles_slow(float4 a, float4 b, float4 c, float4 d, float ts,
                                                             float bs, uint32_t& w0, uint32_t& w1) {
  const float v[16] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
  uint32_t words[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 16; ++i)
    words[i >> 3] |= fp4_nibble(__fdiv_rn(__fdiv_rn(v[i], ts), bs)) << (4 * ((i & 7) ^ 1));
  w0 = words[0];
  w1 = words[1];
}

// E2M1 bin thresholds of one block, in the input's own float domain.
//
// The nibble magnitude of x is the number of midpoints m in
// {.25, .75, 1.25, 1.75, 2.5, 3.5, 5} with q = RN(RN(|x|/ts)/bs) > m. Both
// roundings are monotone, so each test is |x| > W for one float W per
// midpoint and block:
//  * q > m  <=>  q1 = RN(|x|/ts) > m' * bs, m' the midpoint between m and
//    its float successor (a tie at m' rounds to m, whose significand is
//    even). m' * bs is exact in double; q1 is a float, so q1 > m' * bs
//    <=> q1 > Tf = RD_float(m' * bs).
//  * q1 > Tf  <=>  q1 >= S = succ(Tf)  <=>  |x|/ts > M, or = M when S is
//    even (M the midpoint of Tf and S). M * ts is exact in double (M has 25
//    significant bits, ts at most 24), so |x| > M*ts <=> |x| > RD_float(M*ts)
//    and |x| >= M*ts <=> |x| > pred(RU_float(M*ts)).
// Valid when ts, bs, every nonzero |x| and the quotients are finite normal
// floats (the fast-path range of nvfp4_quant_block).
__device__ __forceinline__ void nvfp4_block_thresholds(float ts, float bs, float (&w)[7]) {
  const float mids[7] = {0.25f, 0.75f, 1.25f, 1.75f, 2.5f, 3.5f, 5.0f};
#pragma unroll
  for (int j = 0; j < 7; ++j) {
    const double mp = (double)mids[j] + 0.5 * ((double)__uint_as_float(__float_as_uint(mids[j]) + 1u) - mids[j]);
    const float tf = __double2float_rd(mp * (double)bs);
    const uint32_t sb = __float_as_uint(tf) + 1u;
    const double M = 0.5 * ((double)tf + (double)__uint_as_float(sb));
    const double U = M * (double)ts;
    w[j] = (sb & 1u) ? __double2float_rd(U) : __uint_as_float(__float_as_uint(__double2float_ru(U)) - 1u);
  }
}

// Quantize one 16-element block given the tensor scale (quant.py:169-183).
// v[16] holds the input values as float. Returns the e4m3 code and the 8
// packed bytes (high nibble = even k) in w0 (elements 0-7) / w1 (8-15).
// The reference's steps: bmax = RN(max|x| / ts) (division by a positive
// scale is monotone, so the block maximum of RN(|x|/ts) is this one
// quotient), the e4m3 scale bs of RN(max(bmax, 1e-8) / 6), and per element
// q = RN(RN(x / ts) / bs) binned to E2M1 (ties toward the smaller
// magnitude). The per-element bins come from nvfp4_block_thresholds when
// every nonzero |x| is in [2^-30, 2^30], ts in [2^-40, 2^40] and bs in
// [2^-9, 448] (all quotients then stay finite normal floats); any other
// block runs the two divisions per element.
// The block's binning once its thresholds w[7] are known (fast path) or
// with the two divisions per element (any other block).
template <class GetThresholds>
__device__ __forceinline__ uint32_t nvfp4_quant_block_core(const float (&v)[16], float ts, uint32_t& w0,
                                                           uint32_t& w1, GetThresholds get_w) {
  float amax = 0.0f, amin = 0x1p30f;
  bool anynan = false;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float a = fabsf(v[i]);
    anynan |= (a != a);
    amax = fmaxf(amax, a);
    amin = fminf(amin, a == 0.0f ? 0x1p30f : a);
  }
  const float bmax = anynan ? __int_as_float(0x7FC00000) : div_rn(amax, ts);
  const float bm = (bmax != bmax) ? bmax : fmaxf(bmax, 1e-8f);
  const uint32_t sf = e4m3_encode(div_rn(bm, kFp4Max));
  const float bs = e4m3_decode(sf);
  const bool fast = !anynan && amax <= 0x1p30f && amin >= 0x1p-30f && ts >= 0x1p-40f && ts <= 0x1p40f &&
                    bs >= 0x1p-9f && bs <= 448.0f;
  if (__builtin_expect(fast, 1)) {
    float w[7];
    get_w(sf, bs, w);
    uint32_t words[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float a = fabsf(v[i]);
      const uint32_t nib = (v[i] < 0.0f ? 8u : 0u) | (uint32_t)((a > w[0]) + (a > w[1]) + (a > w[2]) + (a > w[3]) +
                                                                (a > w[4]) + (a > w[5]) + (a > w[6]));
      words[i >> 3] |= nib << (4 * ((i & 7) ^ 1));
    }
    w0 = words[0];
    w1 = words[1];
  } else {
    nvfp4_block_nibbles_slow(make_float4(v[0], v[1], v[2], v[3]), make_float4(v[4], v[5], v[6], v[7]),
                             make_float4(v[8], v[9], v[10], v[11]), make_float4(v[12], v[13], v[14], v[15]), ts,
                             bs, w0, w1);
  }
  return sf;
}

__device__ __forceinline__ uint32_t nvfp4_quant_block(const float (&v)[16], float ts,
                                                      uint32_t& w0, uint32_t& w1) {
  return nvfp4_quant_block_core(v, ts, w0, w1, [&](uint32_t, float bs, float (&w)[7]) {
    nvfp4_block_thresholds(ts, bs, w);
  });
}

// Thresholds of every positive e4m3 block scale for one tensor scale ts:
// tab[8 * code + j], j < 7 (codes whose scale leaves the fast-path range
// are never read). Filled cooperatively by the threads of a block
// (nthreads of them, this one being `t`); the caller synchronises before use.
__device__ __forceinline__ void nvfp4_threshold_table(float ts, float* tab, int t, int nthreads) {
  for (int c = t; c < 127; c += nthreads) {
    const float bs = e4m3_decode((uint32_t)c);
    float w[7] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (bs >= 0x1p-9f && bs <= 448.0f && ts >= 0x1p-40f && ts <= 0x1p40f) nvfp4_block_thresholds(ts, bs, w);
#pragma unroll
    for (int j = 0; j < 7; ++j) tab[8 * c + j] = w[j];
    tab[8 * c + 7] = 0.0f;
  }
}

// nvfp4_quant_block with the block thresholds read from a table made by
// nvfp4_threshold_table for the same ts (shared memory, 4 KB): the same bits,
// without the per-block double-precision threshold arithmetic.
__device__ __forceinline__ uint32_t nvfp4_quant_block_tab(const float (&v)[16], float ts, const float* tab,
                                                          uint32_t& w0, uint32_t& w1) {
  return nvfp4_quant_block_core(v, ts, w0, w1, [&](uint32_t code, float, float (&w)[7]) {
    const float4 a = *reinterpret_cast<const float4*>(tab + 8 * code);
    const float4 b = *reinterpret_cast<const float4*>(tab + 8 * code + 4);
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z;
  });
}

// ---------------------------------------------------------------------------
// FP4 -> fp16 decode for the CUDA-core dot products.
// A 32-bit word holds 8 nibbles; byte b has element 2b in its high nibble and
// 2b+1 in its low nibble. Each output half2 pairs the nibbles 16 bits apart.
// Placing the 3 magnitude bits at fp16 bits [11:9] and the sign at bit 15
// yields exactly value * 2^-14 (code 001 lands on the fp16 subnormal 2^-15).
//   h[0] = (e1, e5)   h[1] = (e0, e4)   h[2] = (e3, e7)   h[3] = (e2, e6)
// Any operand decoded with this routine pairs with any other decoded with it.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void fp4x8_to_half2x4_scaled(uint32_t w, __half2 (&h)[4]) {
  uint32_t r0 = ((w << 9) & 0x0E000E00u) | ((w << 12) & 0x80008000u);
  uint32_t r1 = ((w << 5) & 0x0E000E00u) | ((w << 8) & 0x80008000u);
  uint32_t r2 = ((w << 1) & 0x0E000E00u) | ((w << 4) & 0x80008000u);
  uint32_t r3 = ((w >> 3) & 0x0E000E00u) | (w & 0x80008000u);
  h[0] = *reinterpret_cast<__half2*>(&r0);
  h[1] = *reinterpret_cast<__half2*>(&r1);
  h[2] = *reinterpret_cast<__half2*>(&r2);
  h[3] = *reinterpret_cast<__half2*>(&r3);
}

// Exact (unscaled) FP4 values in the same pairing, for the activation side.
__device__ __forceinline__ void fp4x8_to_half2x4_exact(uint32_t w, __half2 (&h)[4]) {
  fp4x8_to_half2x4_scaled(w, h);
  const __half2 k = __floats2half2_rn(16384.0f, 16384.0f);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __hmul2(h[i], k);
}

// ---------------------------------------------------------------------------
// warp helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}
__device__ __forceinline__ uint32_t warp_umax(uint32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ float gelu_tanh(float x) {
  // tanh-approximated GELU in float32, as torch's gelu(approximate="tanh")
  const float kBeta = 0.7978845608028654f;   // sqrt(2/pi)
  const float kKappa = 0.044715f;
  float inner = kBeta * (x + kKappa * (x * x * x));
  return 0.5f * x * (1.0f + tanhf(inner));
}

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

}  // namespace aeoq

namespace aeoq {

// Scalar loads of a 0-d device tensor of a given dtype code.
__device__ __forceinline__ float load_scalar_f(const void* p, int dt) {
  if (dt == AEOQ_BF16) return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(p));
  if (dt == AEOQ_F16) return __half2float(*reinterpret_cast<const __half*>(p));
  return *reinterpret_cast<const float*>(p);
}
__device__ __forceinline__ int64_t load_index(const void* p, int dt, int64_t i) {
  if (dt == AEOQ_I64) return reinterpret_cast<const int64_t*>(p)[i];
  return reinterpret_cast<const int32_t*>(p)[i];
}

// Dot product of one 16-byte chunk (32 FP4 values = 2 blocks of 16) of an
// activation already decoded to exact halves `a[16]` with a packed weight
// chunk `w`, given the activation block scales pre-multiplied by 2^14 and the
// two weight e4m3 codes. Each block's 16 products are accumulated in fp16,
// where they are exact (|sum| < 2^-5 at a 2^-16 grid), then scaled exactly
// and added to the float accumulator.
__device__ __forceinline__ float chunk_dot(const __half2 (&a)[16], const float (&sa16k)[2], uint4 w,
                                           uint16_t wsf, float acc) {
  const float2 sw = __half22float2(e4m3x2_to_half2(wsf));
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int b = 0; b < 2; ++b) {
    __half2 h = __float2half2_rn(0.0f);
    __half2 d[4];
    fp4x8_to_half2x4_scaled(words[2 * b], d);
#pragma unroll
    for (int i = 0; i < 4; ++i) h = __hfma2(a[8 * b + i], d[i], h);
    fp4x8_to_half2x4_scaled(words[2 * b + 1], d);
#pragma unroll
    for (int i = 0; i < 4; ++i) h = __hfma2(a[8 * b + 4 + i], d[i], h);
    const float2 f = __half22float2(h);
    acc = fmaf(f.x + f.y, sa16k[b] * (b ? sw.y : sw.x), acc);
  }
  return acc;
}

// Decode a packed activation chunk (uint4 + two e4m3 codes) into exact
// halves and 2^14-scaled block scales for chunk_dot.
__device__ __forceinline__ void decode_act_chunk(uint4 p, uint16_t sf2, __half2 (&a)[16],
                                                 float (&sa16k)[2]) {
  const uint32_t words[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 t[4];
    fp4x8_to_half2x4_exact(words[i], t);
#pragma unroll
    for (int j = 0; j < 4; ++j) a[4 * i + j] = t[j];
  }
  const float2 s = __half22float2(e4m3x2_to_half2(sf2));
  sa16k[0] = s.x * 16384.0f;
  sa16k[1] = s.y * 16384.0f;
}

// Quantize 32 consecutive bf16 values (one chunk) with tensor scale ts and
// return the chunk in chunk_dot's activation form.
__device__ __forceinline__ void quant_act_chunk_bf16(const __nv_bfloat16* src, float ts,
                                                     __half2 (&a)[16], float (&sa16k)[2]) {
  float v[2][16];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 u = *reinterpret_cast<const uint4*>(src + 8 * q);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[q >> 1][8 * (q & 1) + j] = __bfloat162float(e[j]);
  }
  uint32_t w[4];
  const uint32_t s0 = nvfp4_quant_block(v[0], ts, w[0], w[1]);
  const uint32_t s1 = nvfp4_quant_block(v[1], ts, w[2], w[3]);
  decode_act_chunk(make_uint4(w[0], w[1], w[2], w[3]), (uint16_t)(s0 | (s1 << 8)), a, sa16k);
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace aeoq

namespace aeoq {

// ---------------------------------------------------------------------------
// FP4 -> exact fp16 via the hardware converter (cvt.rn.f16x2.e2m1x2): byte b
// of w becomes h[b] = (low nibble, high nibble) = (element 2b+1, element 2b).
// Activations and weights decoded with this routine pair element-for-element.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void fp4x8_to_half2x4(uint32_t w, __half2 (&h)[4]) {
  uint32_t r0, r1, r2, r3;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(w));
  h[0] = *reinterpret_cast<__half2*>(&r0);
  h[1] = *reinterpret_cast<__half2*>(&r1);
  h[2] = *reinterpret_cast<__half2*>(&r2);
  h[3] = *reinterpret_cast<__half2*>(&r3);
}

// One 16-byte chunk (two 16-value blocks) of exact activation halves `a`
// (with per-block scales sa) against a packed weight chunk. Within a block,
// each fp16 lane sums 8 products of E2M1 values (multiples of 1/4, |sum| <=
// 288): exact in fp16. The block sum times the two e4m3 scales is exact in
// fp32; only the running sum across blocks rounds.
__device__ __forceinline__ float chunk_dot_x(const __half2 (&a)[16], const float (&sa)[2], uint4 w,
                                             uint16_t wsf, float acc) {
  const float2 sw = __half22float2(e4m3x2_to_half2(wsf));
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int b = 0; b < 2; ++b) {
    __half2 h = __float2half2_rn(0.0f);
    __half2 d[4];
    fp4x8_to_half2x4(words[2 * b], d);
#pragma unroll
    for (int i = 0; i < 4; ++i) h = __hfma2(a[8 * b + i], d[i], h);
    fp4x8_to_half2x4(words[2 * b + 1], d);
#pragma unroll
    for (int i = 0; i < 4; ++i) h = __hfma2(a[8 * b + 4 + i], d[i], h);
    const float2 f = __half22float2(h);
    acc = fmaf(f.x + f.y, sa[b] * (b ? sw.y : sw.x), acc);
  }
  return acc;
}

// Packed activation chunk -> exact halves + block scales for chunk_dot_x.
__device__ __forceinline__ void decode_act_chunk_x(uint4 p, uint16_t sf2, __half2 (&a)[16], float (&sa)[2]) {
  const uint32_t words[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 t[4];
    fp4x8_to_half2x4(words[i], t);
#pragma unroll
    for (int j = 0; j < 4; ++j) a[4 * i + j] = t[j];
  }
  const float2 s = __half22float2(e4m3x2_to_half2(sf2));
  sa[0] = s.x;
  sa[1] = s.y;
}

// ---------------------------------------------------------------- bulk copy
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          (uint32_t)__cvta_generic_to_shared(dst)),
      "l"(src), "r"(bytes), "r"((uint32_t)__cvta_generic_to_shared(bar))
      : "memory");
}

}  // namespace aeoq
