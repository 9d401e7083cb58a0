// Device self-tests of the numerics every quantized bit depends on.
//
// aeoq_selftest_div_rn compares div_rn (common.cuh) with the compiler's
// __fdiv_rn bit for bit over whole operand domains, enumerated on the GPU:
//   domain 0: every float significand of the dividend (a in [1, 2), both
//             signs) against every bf16 significand of the divisor. Covers
//             max|x| / ts, x / ts (ts is bf16), q / bs (bs is e4m3, a subset
//             of bf16) and bm / 6, amax / 448, amax / 2688.
//   domain 1: every bf16 significand of the dividend against every float
//             significand of the divisor: x / s with the f32 activation
//             scale s of the FP8 path.
//   domain 2: 2^28 pseudo-random pairs with exponents spread over div_rn's
//             whole fast-path range, zeros and the range edges included.
//   domain 3: nvfp4_quant_block (scale and packed nibbles) against the
//             reference's formula computed with __fdiv_rn, over 2^22 blocks:
//             random values over many scales, bf16 and f32 tensor scales,
//             zeros, and values placed exactly on, one float below and one
//             float above each of the block's bin thresholds.
// Only significands matter inside the fast path's range (no overflow,
// underflow or subnormal is reachable there), so domains 0 and 1 are
// exhaustive for the quantizers' divisions.
#include "common.cuh"

namespace aeoq {
namespace {

__device__ __forceinline__ void check(float a, float b, unsigned long long* mism, float* ex) {
  const float got = div_rn(a, b), want = __fdiv_rn(a, b);
  if (__float_as_uint(got) != __float_as_uint(want) && !(got != got && want != want)) {
    if (atomicAdd(mism, 1ull) == 0ull) {
      ex[0] = a; ex[1] = b; ex[2] = got; ex[3] = want;
    }
  }
}

__device__ __forceinline__ uint32_t mix32(uint64_t x) {
  x ^= x >> 33; x *= 0xff51afd7ed558ccdull; x ^= x >> 33; x *= 0xc4ceb9fe1a85ec53ull; x ^= x >> 33;
  return (uint32_t)x;
}

__global__ void selftest_div_kernel(int domain, unsigned long long* mism, float* ex) {
  const uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (domain == 0) {
    if (t >= (1ull << 24)) return;
    const float a = __uint_as_float(((uint32_t)(t & 1) << 31) | 0x3F800000u | (uint32_t)(t >> 1));
    for (uint32_t m = 0; m < 128; ++m) check(a, __uint_as_float(0x3F800000u | (m << 16)), mism, ex);
  } else if (domain == 1) {
    if (t >= (1ull << 23)) return;
    const float b = __uint_as_float(0x3F800000u | (uint32_t)t);
    for (uint32_t m = 0; m < 256; ++m)
      check(__uint_as_float(((m & 1u) << 31) | 0x3F800000u | ((m >> 1) << 16)), b, mism, ex);
  } else {
    if (t >= (1ull << 22)) return;
    for (int i = 0; i < 64; ++i) {
      const uint32_t r0 = mix32(t * 64 + i), r1 = mix32((t * 64 + i) ^ 0x9E3779B97F4A7C15ull);
      // a: exponent in [-82, 82], b: exponent in [-42, 42], so both sides of
      // every range edge are exercised (the outer ones take __fdiv_rn).
      const uint32_t ea = 127u - 82u + (r0 >> 24) % 165u, eb = 127u - 42u + (r1 >> 24) % 85u;
      float a = __uint_as_float((r0 & 0x80000000u) | (ea << 23) | (r0 & 0x7FFFFFu));
      const float b = __uint_as_float((r1 & 0x80000000u) | (eb << 23) | (r1 & 0x7FFFFFu));
      if ((r0 & 0xFFu) == 0u) a = (r0 & 0x100u) ? -0.0f : 0.0f;
      check(a, b, mism, ex);
    }
  }
}

// The reference's block quantization, division by division (quant.py:169-183).
__device__ uint32_t quant_block_direct(const float (&v)[16], float ts, uint32_t& w0, uint32_t& w1) {
  float amax = 0.0f;
  bool anynan = false;
  for (int i = 0; i < 16; ++i) {
    anynan |= v[i] != v[i];
    amax = fmaxf(amax, fabsf(v[i]));
  }
  const float bmax = anynan ? __int_as_float(0x7FC00000) : __fdiv_rn(amax, ts);
  const float bm = (bmax != bmax) ? bmax : fmaxf(bmax, 1e-8f);
  const uint32_t sf = e4m3_encode(__fdiv_rn(bm, kFp4Max));
  const float bs = e4m3_decode(sf);
  w0 = w1 = 0u;
  for (int i = 0; i < 16; ++i) {
    const uint32_t nib = fp4_nibble(__fdiv_rn(__fdiv_rn(v[i], ts), bs));
    (i < 8 ? w0 : w1) |= nib << (4 * ((i & 7) ^ 1));
  }
  return sf;
}

__global__ void selftest_quant_kernel(unsigned long long* mism, float* ex) {
  const uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  uint64_t ctr = t * 97;
  auto rnd = [&]() { return mix32(ctr++ ^ 0x5851F42D4C957F2Dull); };
  auto unif = [&]() { return (float)(rnd() >> 8) * 0x1p-24f; };
  const float scale = __uint_as_float((127u - 24u + rnd() % 40u) << 23);   // 2^-24 .. 2^15
  float v[16];
  for (int i = 0; i < 16; ++i) {
    const uint32_t r = rnd();
    float x = (unif() * 2.0f - 1.0f) * scale * (1.0f + 7.0f * unif());
    if ((r & 15u) == 0u) x = 0.0f;
    if ((r & 15u) == 1u) x = __uint_as_float(__float_as_uint(x) & 0xFFFF0000u);   // bf16-exact
    v[i] = x;
  }
  float ts;
  {
    float gmax = 0.0f;
    for (int i = 0; i < 16; ++i) gmax = fmaxf(gmax, fabsf(v[i]));
    gmax *= 1.0f + 3.0f * unif();                    // the tensor max is at least the block's
    ts = __fdiv_rn(gmax, kNvfp4Denom);
    if (rnd() & 1u) ts = bf16r(ts);
    ts = fmaxf(ts, 1e-12f);
  }
  if (t & 1) {
    // probes on the block's own thresholds (the block max stays in v[0..7])
    float amax = 0.0f;
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const float bs = e4m3_decode(e4m3_encode(__fdiv_rn(fmaxf(__fdiv_rn(amax, ts), 1e-8f), kFp4Max)));
    if (bs >= 0x1p-9f && bs <= 448.0f && ts >= 0x1p-40f) {
      float w[7];
      nvfp4_block_thresholds(ts, bs, w);
      for (int i = 8; i < 16; ++i) {
        const uint32_t r = rnd();
        float x = w[r % 7u];
        const int d = (int)((r >> 8) % 3u) - 1;
        x = __uint_as_float(__float_as_uint(x) + d);
        if (fabsf(x) > amax) x = amax;
        v[i] = (r >> 16) & 1u ? -x : x;
      }
    }
  }
  uint32_t a0, a1, b0, b1;
  const uint32_t sa = nvfp4_quant_block(v, ts, a0, a1);
  const uint32_t sb = quant_block_direct(v, ts, b0, b1);
  if (sa != sb || a0 != b0 || a1 != b1) {
    if (atomicAdd(mism, 1ull) == 0ull) {
      ex[0] = ts;
      for (int i = 0; i < 16; ++i) ex[1 + i] = v[i];
    }
  }
}

}  // namespace
}  // namespace aeoq

extern "C" int aeoq_selftest_div_rn(int domain, unsigned long long* mismatches, float* example, void* stream) {
  AEOQ_REQUIRE(domain >= 0 && domain <= 3, AEOQ_ERR_INVALID, "selftest_div_rn: domain 0 to 3");
  AEOQ_REQUIRE(mismatches && example, AEOQ_ERR_INVALID, "selftest_div_rn: null pointer");
  if (domain == 3) {
    aeoq::selftest_quant_kernel<<<(1u << 22) / 256, 256, 0, (cudaStream_t)stream>>>(mismatches, example);
    return aeoq::check_launch("selftest_quant_kernel");
  }
  const unsigned threads = domain == 0 ? (1u << 24) : domain == 1 ? (1u << 23) : (1u << 22);
  aeoq::selftest_div_kernel<<<threads / 256, 256, 0, (cudaStream_t)stream>>>(domain, mismatches, example);
  return aeoq::check_launch("selftest_div_kernel");
}
