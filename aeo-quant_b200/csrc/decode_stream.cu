// One-token NVFP4 MoE expert forward, streamed: one launch, one grid barrier.
//
// Restates Gemma4TextExpertsNVFP4._forward_decode_3d (aeo_quant
// src/aeo_quant/bridges/gemma4/modeling_nvfp4.py:132-186) for one token:
// quantize the hidden vector (:150-153), gate_up GEMV of the k routed
// experts (:155-160), GeGLU in bf16 (:161-162), re-quantize the k GeGLU rows
// with ONE shared tensor scale (:164-172), down GEMV (:174-179), weighted
// sum over the k experts (:181-186).
//
// At one token the layer is a pure stream of the k experts' packed weights
// (26.8 MB for Gemma-4-26B-A4B), so the kernel is laid out for HBM:
//
// * Work split by bytes into few, large copies. HBM serves a CTA's bulk
//   copies at full rate when they are large; many small copies from
//   scattered addresses (a few KB each) run at a third of it. So CTA c
//   (one per SM) owns ONE down block: `rows` consecutive down rows (a
//   multiple of 4, so its 44-byte scale rows start on 16-byte boundaries)
//   of ONE expert slot (two copies, ~63 KB), and a contiguous range of the
//   k*I gate/up row pairs (gate rows, up rows and their scales: four copies
//   per slot segment, split in groups of kGroup pairs for early compute).
//   The host plan balances the CTAs' bytes.
// * Everything the CTA will read from HBM is requested at entry (L2
//   evict-first): every warp loads the expert ids itself and issues its
//   share of the copies. Meanwhile the hidden vector is staged in shared
//   memory and quantized (global amax, bf16 tensor scale, e4m3 block scales,
//   E2M1 codes) into exact fp16 operands.
// * gate/up dot products run per pair group as soon as its barrier flips;
//   h = bf16(bf16(gelu(g)) * u) goes to the workspace.
// * One grid barrier (an arrival counter with a bounded spin; the launch is
//   cooperative, so every CTA is resident); the grid's max |h| is one word
//   updated with atomicMax before the arrival.
// * Each CTA then reads its slot's GeGLU row (I values), quantizes it with
//   the shared tensor scale and runs its down dot products from shared
//   memory. The weighted products bf16(bf16(a*d_j) * w_j) of the k slots
//   meet in an f64 accumulator per output row (atomic adds: a sum of k bf16
//   values in f64 is exact, so the order does not matter); the CTA that
//   brings a row block's arrival count to k rounds it once to f32 then bf16,
//   as the reference's sum does, and clears the accumulator and the count.
// * The last CTA to leave zeroes the grid counters, so a zeroed workspace
//   stays valid for every call on one stream.
//
// An expert id outside [0, E) reads no weights and contributes zeros.
#include "common.cuh"
#include "sm100.cuh"

namespace aeoq {
namespace dst {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxK = 16;
constexpr int kMaxCtas = 160;
constexpr int kGroup = 20;            // gate/up pairs per arrival barrier
constexpr int kMaxGroups = 8;
constexpr int kMaxRows = 512;         // down rows per CTA
constexpr int kMaxChunks = 4;         // 32-value chunks per lane of a hidden row (H <= 4096)
constexpr size_t kSmemCap = 227 * 1024;

// Host-side plan (passed by value).
struct Plan {
  int H, I, k, G;
  int rows;                    // down rows per block (multiple of 4)
  int nb;                      // down blocks per expert slot; CTA c < k*nb owns slot c/nb, block c%nb
  int max_pairs;               // largest pair range of any CTA
  size_t bytes;                // dynamic shared memory
  int pair0[kMaxCtas + 1];     // CTA c owns pairs [pair0[c], pair0[c+1])
};

struct Args {
  const __nv_bfloat16* hidden;
  const void* ids; int ids_dt;
  const __nv_bfloat16* topw;
  const uint8_t* gu; const uint8_t* gu_sf; const void* gu_ts; int gu_ts_dt;
  const uint8_t* dw; const uint8_t* dw_sf; const void* d_ts; int d_ts_dt;
  int64_t E;
  __nv_bfloat16* out;
  __nv_bfloat16* h;      // k*I bf16 GeGLU rows
  uint32_t* sync;        // [0] arrivals, [1] departures, [2] max |h| key over the grid
  uint32_t* cnt;         // [nb] slots folded into each down row block
  double* acc;           // [H] f64 sums of the weighted down products
  int* err;              // error word (bounded waits)
};

__host__ __device__ inline size_t a16(size_t v) { return (v + 15) / 16 * 16; }

// Shared-memory carve-up of one CTA (np pairs, nr down rows).
struct Carve {
  size_t gate, up, gsf, usf, dn, dsf, hid, act, asa, hrow, end;
};
__host__ __device__ inline Carve carve(int H, int I, int k, int np, int nr) {
  Carve c{};
  const size_t rb = H / 2, sb = H / 16, rb2 = I / 2, sb2 = I / 16;
  size_t o = 0;
  c.gate = o; o = a16(o + (size_t)np * rb);
  c.up = o;   o = a16(o + (size_t)np * rb);
  c.gsf = o;  o = a16(o + (size_t)np * sb);
  c.usf = o;  o = a16(o + (size_t)np * sb);
  c.dn = o;   o = a16(o + (size_t)nr * rb2);
  c.dsf = o;  o = a16(o + (size_t)nr * sb2);
  c.hid = o;  o = a16(o + (size_t)H * 2);
  c.act = o;  o = a16(o + (size_t)(H / 16) * 8 * sizeof(__half2));
  c.asa = o;  o = a16(o + (size_t)(H / 16) * sizeof(float));
  c.hrow = o; o = a16(o + (size_t)I * 2);
  c.end = o;
  return c;
}

// Down rows of CTA c (0 when it owns no down block).
__host__ __device__ inline int down_rows(const Plan& p, int c, int* slot, int* r0) {
  if (c >= p.k * p.nb) { *slot = 0; *r0 = 0; return 0; }
  *slot = c / p.nb;
  *r0 = (c % p.nb) * p.rows;
  return min(p.rows, p.H - *r0);
}

static bool make_plan(int64_t k, int64_t H, int64_t I, int G, Plan& p) {
  if (k < 1 || k > kMaxK || G < 1 || G > kMaxCtas) return false;
  if (H <= 0 || I <= 0 || H % 256 != 0 || I % 64 != 0) return false;
  if (H / 32 > 32 * kMaxChunks || I / 32 > 32) return false;
  p.H = (int)H; p.I = (int)I; p.k = (int)k; p.G = G;
  // smallest multiple of 4 rows whose k * ceil(H / rows) blocks fit the grid
  int rows = (int)((H * k + G - 1) / G + 3) / 4 * 4;
  while (rows <= kMaxRows && k * ((H + rows - 1) / rows) > G) rows += 4;
  if (rows > kMaxRows) return false;
  p.rows = rows;
  p.nb = (int)((H + rows - 1) / rows);
  const double pair_b = 2.0 * (H / 2 + H / 16);
  const double row_b = (double)(I / 2 + I / 16);
  const int64_t pairs = k * I;
  const double total = pairs * pair_b + (double)k * H * row_b;
  const double target = total / G;
  double down_before = 0.0;
  for (int c = 0; c <= G; ++c) {
    int64_t q = (int64_t)((c * target - down_before) / pair_b + 0.5);
    q = q < 0 ? 0 : (q > pairs ? pairs : q);
    if (c == G) q = pairs;
    if (c > 0 && q < p.pair0[c - 1]) q = p.pair0[c - 1];
    p.pair0[c] = (int)q;
    if (c < G) {
      int j, r0;
      down_before += down_rows(p, c, &j, &r0) * row_b;
    }
  }
  size_t need = 0;
  p.max_pairs = 0;
  for (int c = 0; c < G; ++c) {
    const int np = p.pair0[c + 1] - p.pair0[c];
    p.max_pairs = np > p.max_pairs ? np : p.max_pairs;
    int j, r0;
    const int nr = down_rows(p, c, &j, &r0);
    const size_t b = carve(p.H, p.I, p.k, np, nr).end;
    need = b > need ? b : need;
  }
  if ((p.max_pairs + kGroup - 1) / kGroup > kMaxGroups) return false;
  p.bytes = need + 1024;
  return p.bytes <= kSmemCap;
}

__device__ __forceinline__ void complete_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" ::"r"(sm100::smem_u32(bar)), "r"(bytes) : "memory");
}

// Eight E2M1 values (one 32-bit word, two per byte) to four f16x2 with the
// hardware conversion (cvt.rn.f16x2.e2m1x2, exact). Activations and weights
// go through the same conversion, so both operands pair their elements the
// same way and the dot product is unchanged.
__device__ __forceinline__ void e2m1x8_to_h2x4(uint32_t w, __half2 (&h)[4]) {
  uint32_t r0, r1, r2, r3;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(w));
  h[0] = *reinterpret_cast<__half2*>(&r0);
  h[1] = *reinterpret_cast<__half2*>(&r1);
  h[2] = *reinterpret_cast<__half2*>(&r2);
  h[3] = *reinterpret_cast<__half2*>(&r3);
}

// Quantize 16 bf16 values (shared memory) with tensor scale ts
// (quant.py:169-183) and store them as 8 exact f16x2 plus the block scale.
__device__ __forceinline__ void quant16_h2(const __nv_bfloat16* src, float ts, __half2* dst, float* scale) {
  float v[16];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const uint4 u = reinterpret_cast<const uint4*>(src)[q];
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[8 * q + j] = __bfloat162float(e[j]);
  }
  uint32_t w0, w1;
  const uint32_t sf = nvfp4_quant_block(v, ts, w0, w1);
  __half2 t[4];
  e2m1x8_to_h2x4(w0, t);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = t[i];
  e2m1x8_to_h2x4(w1, t);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[4 + i] = t[i];
  *scale = e4m3_decode(sf);
}

// 32-value chunk dot product: a[16] the activation's f16x2 (two 16-blocks),
// sa[2] their block scales, w 16 packed weight bytes, wsf the weight's two
// e4m3 block scales. Within a block every product of two E2M1 values is a
// multiple of 1/4 at most 36, so each f16 half sums 8 of them exactly
// (|sum| <= 288); the block sum is exact in f32 and is scaled and added to
// the f32 accumulator once per block, as the tensor core's block16 MMA does.
__device__ __forceinline__ float dot32(const __half2 (&a)[16], const float (&sa)[2], uint4 w, uint16_t wsf,
                                       float acc) {
  const float2 sw = __half22float2(e4m3x2_to_half2(wsf));
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int b = 0; b < 2; ++b) {
    __half2 h = __float2half2_rn(0.0f);
    __half2 d[4];
    e2m1x8_to_h2x4(words[2 * b], d);
#pragma unroll
    for (int i = 0; i < 4; ++i) h = __hfma2(a[8 * b + i], d[i], h);
    e2m1x8_to_h2x4(words[2 * b + 1], d);
#pragma unroll
    for (int i = 0; i < 4; ++i) h = __hfma2(a[8 * b + 4 + i], d[i], h);
    const float2 f = __half22float2(h);
    acc = fmaf(f.x + f.y, sa[b] * (b ? sw.y : sw.x), acc);
  }
  return acc;
}

// Fire-and-forget f64 add at L2 (no value returned, so the issuing warp does
// not wait for the round trip).
__device__ __forceinline__ void red_add_f64(double* p, double v) {
  asm volatile("red.relaxed.gpu.global.add.f64 [%0], %1;" ::"l"(p), "d"(v) : "memory");
}

// L2 policy for data read once: evict first.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Bulk global -> shared copy with an L2 cache policy.
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"((uint32_t)__cvta_generic_to_shared(dst)),
      "l"(src), "r"(bytes), "r"((uint32_t)__cvta_generic_to_shared(bar)), "l"(pol)
      : "memory");
}

__global__ void __launch_bounds__(kThreads, 1) decode_stream_kernel(const Args a, const Plan pl) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bars[kMaxGroups + 1];
  __shared__ int64_t ids_w[kWarps][kMaxK];
  __shared__ uint32_t red[kWarps];
  __shared__ float topw_s[kMaxK];
  __shared__ uint32_t hmax_s;
  __shared__ int last_s;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = pl.H, I = pl.I, k = pl.k;
  const size_t rb = H / 2, sb = H / 16, rb2 = I / 2, sb2 = I / 16;
  const int p0 = pl.pair0[blockIdx.x], np = pl.pair0[blockIdx.x + 1] - p0;
  const int ngroups = (np + kGroup - 1) / kGroup;
  int dslot, r0;
  const int nr = down_rows(pl, (int)blockIdx.x, &dslot, &r0);
  const Carve cv = carve(H, I, k, np, nr);
  uint64_t* bdown = &bars[kMaxGroups];

  // The hidden vector and the small operands are requested before the weight
  // copies: issued after them, they would queue behind ~27 MB of traffic.
  uint4 hid_u[(4096 / 8 + kThreads - 1) / kThreads];
#pragma unroll
  for (int q = 0; q < (4096 / 8 + kThreads - 1) / kThreads; ++q) {
    const int i = tid + q * kThreads;
    if (i < H / 8) hid_u[q] = __ldg(reinterpret_cast<const uint4*>(a.hidden) + i);
  }
  const float gu_ts = load_scalar_f(a.gu_ts, a.gu_ts_dt);
  const float d_ts = load_scalar_f(a.d_ts, a.d_ts_dt);
  const float topw_r = tid < k ? __bfloat162float(a.topw[tid]) : 0.0f;

  // ---- every warp: its barriers, the expert ids, its share of the copies ----
  // Warp w owns pair groups g = w, w + 16, ...; the last warp owns the down
  // block. Every warp loads the k ids itself (one L2 line), so no warp waits
  // for another before issuing. The copies carry an L2 evict-first hint: the
  // streamed weights are read once and must not push the kernel's code and
  // small operands out of L2.
  if (lane == 0) {
    for (int g = warp; g < ngroups; g += kWarps) sm100::mbar_init(&bars[g], 1);
    if (warp == kWarps - 1) sm100::mbar_init(bdown, 1);
    sm100::fence_barrier_init();
  }
  if (lane < k) {
    const int64_t e = load_index(a.ids, a.ids_dt, lane);
    ids_w[warp][lane] = (e < 0 || e >= a.E) ? -1 : e;
  }
  __syncwarp();
  if (lane == 0) {
    const uint64_t pol = l2_evict_first();
    for (int g = warp; g < ngroups; g += kWarps) {
      const int i0 = g * kGroup, i1 = min(np, i0 + kGroup);
      sm100::mbar_arrive_expect_tx(&bars[g], (uint32_t)((i1 - i0) * (2 * rb + 2 * sb)));
      int i = i0;
      while (i < i1) {   // split at slot boundaries
        const int p = p0 + i, j = p / I, n = p - j * I;
        const int len = min(i1 - i, I - n);
        const int64_t e = ids_w[warp][j];
        if (e >= 0) {
          const uint8_t* g0 = a.gu + ((size_t)e * 2 * I + n) * rb;
          const uint8_t* s0 = a.gu_sf + ((size_t)e * 2 * I + n) * sb;
          bulk_g2s_hint(smem + cv.gate + i * rb, g0, (uint32_t)(len * rb), &bars[g], pol);
          bulk_g2s_hint(smem + cv.up + i * rb, g0 + (size_t)I * rb, (uint32_t)(len * rb), &bars[g], pol);
          bulk_g2s_hint(smem + cv.gsf + i * sb, s0, (uint32_t)(len * sb), &bars[g], pol);
          bulk_g2s_hint(smem + cv.usf + i * sb, s0 + (size_t)I * sb, (uint32_t)(len * sb), &bars[g], pol);
        } else {
          complete_tx(&bars[g], (uint32_t)(len * (2 * rb + 2 * sb)));
        }
        i += len;
      }
    }
    if (warp == kWarps - 1) {
      const int64_t e = ids_w[warp][dslot];
      sm100::mbar_arrive_expect_tx(bdown, (uint32_t)(nr * (rb2 + sb2)));
      if (e >= 0 && nr > 0) {
        bulk_g2s_hint(smem + cv.dn, a.dw + ((size_t)e * H + r0) * rb2, (uint32_t)(nr * rb2), bdown, pol);
        bulk_g2s_hint(smem + cv.dsf, a.dw_sf + ((size_t)e * H + r0) * sb2, (uint32_t)(nr * sb2), bdown, pol);
      } else if (nr > 0) {
        complete_tx(bdown, (uint32_t)(nr * (rb2 + sb2)));
      }
    }
  }
  __syncwarp();

  // ---- hidden vector: stage in shared memory, amax, quantize ---------------
  __nv_bfloat16* hid_s = reinterpret_cast<__nv_bfloat16*>(smem + cv.hid);
  uint32_t key = 0;
#pragma unroll
  for (int q = 0; q < (4096 / 8 + kThreads - 1) / kThreads; ++q) {
    const int i = tid + q * kThreads;
    if (i < H / 8) {
      const uint4 u = hid_u[q];
      reinterpret_cast<uint4*>(hid_s)[i] = u;
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) key = max(key, In<AEOQ_BF16>::abs_key(e[j]));
    }
  }
  if (tid < k) topw_s[tid] = topw_r;
  key = warp_umax(key);
  if (lane == 0) red[warp] = key;
  __syncthreads();   // hid_s, red, topw_s, ids_w, barrier inits
  key = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) key = max(key, red[w]);
  const float ts = nvfp4_tensor_scale<AEOQ_BF16>(In<AEOQ_BF16>::key_to_f(key));
  const float alpha = ts * gu_ts;
  __half2* act_s = reinterpret_cast<__half2*>(smem + cv.act);
  float* asa_s = reinterpret_cast<float*>(smem + cv.asa);
  for (int b = tid; b < H / 16; b += kThreads) quant16_h2(hid_s + 16 * b, ts, act_s + 8 * b, asa_s + b);
  __syncthreads();

  // ---- gate/up GEMV + GeGLU, pair groups as they land ----------------------
  const int nchunk = H / 32;
  __half2 act[kMaxChunks][16];
  float sa[kMaxChunks][2];
#pragma unroll
  for (int q = 0; q < kMaxChunks; ++q) {
    const int c = lane + 32 * q;
    if (c < nchunk) {
      const uint4* ap = reinterpret_cast<const uint4*>(act_s + 16 * c);
#pragma unroll
      for (int z = 0; z < 4; ++z) *reinterpret_cast<uint4*>(&act[q][4 * z]) = ap[z];
      sa[q][0] = asa_s[2 * c];
      sa[q][1] = asa_s[2 * c + 1];
    }
  }
  const uint8_t* gate_s = smem + cv.gate;
  const uint8_t* up_s = smem + cv.up;
  const uint8_t* gsf_s = smem + cv.gsf;
  const uint8_t* usf_s = smem + cv.usf;
  uint32_t hkey = 0;
  bool ok = true;
  // Two pairs per warp iteration (i and i + kWarps): four independent dot
  // product chains and one interleaved reduction, for latency hiding.
  for (int i = warp; i < np; i += 2 * kWarps) {
    const int i2 = i + kWarps;
    const bool two = i2 < np;
    // pair i lies in group i / kGroup, whose copies another warp may own
    ok &= sm100::mbar_wait(&bars[i / kGroup], 0, a.err, 31);
    if (two) ok &= sm100::mbar_wait(&bars[i2 / kGroup], 0, a.err, 31);
    const int p = p0 + i, pb = p0 + i2;
    const bool v1 = ok && ids_w[0][p / I] >= 0;
    const bool v2 = two && ok && ids_w[0][pb / I] >= 0;
    float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int q = 0; q < kMaxChunks; ++q) {
      const int c = lane + 32 * q;
      if (c < nchunk) {
        if (v1) {
          const uint4 gw = *reinterpret_cast<const uint4*>(gate_s + i * rb + 16 * c);
          const uint4 uw = *reinterpret_cast<const uint4*>(up_s + i * rb + 16 * c);
          s[0] = dot32(act[q], sa[q], gw, *reinterpret_cast<const uint16_t*>(gsf_s + i * sb + 2 * c), s[0]);
          s[1] = dot32(act[q], sa[q], uw, *reinterpret_cast<const uint16_t*>(usf_s + i * sb + 2 * c), s[1]);
        }
        if (v2) {
          const uint4 gw = *reinterpret_cast<const uint4*>(gate_s + i2 * rb + 16 * c);
          const uint4 uw = *reinterpret_cast<const uint4*>(up_s + i2 * rb + 16 * c);
          s[2] = dot32(act[q], sa[q], gw, *reinterpret_cast<const uint16_t*>(gsf_s + i2 * sb + 2 * c), s[2]);
          s[3] = dot32(act[q], sa[q], uw, *reinterpret_cast<const uint16_t*>(usf_s + i2 * sb + 2 * c), s[3]);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int z = 0; z < 4; ++z) s[z] += __shfl_xor_sync(0xffffffffu, s[z], o);
    }
    if (lane == 0) {
      const float gv = bf16r(s[0] * alpha), uv = bf16r(s[1] * alpha);
      const __nv_bfloat16 hv = __float2bfloat16_rn(bf16r(gelu_tanh(gv)) * uv);
      a.h[p] = hv;
      hkey = max(hkey, In<AEOQ_BF16>::abs_key(hv));
      if (two) {
        const float gv2 = bf16r(s[2] * alpha), uv2 = bf16r(s[3] * alpha);
        const __nv_bfloat16 hv2 = __float2bfloat16_rn(bf16r(gelu_tanh(gv2)) * uv2);
        a.h[pb] = hv2;
        hkey = max(hkey, In<AEOQ_BF16>::abs_key(hv2));
      }
    }
  }
  // every group barrier completes before the CTA exits (the copies land)
  for (int g = warp; g < ngroups; g += kWarps) sm100::mbar_wait(&bars[g], 0, a.err, 31);
  hkey = warp_umax(hkey);
  if (lane == 0) red[warp] = hkey;
  __syncthreads();

  // ---- grid barrier ----------------------------------------------------------
  // One word holds the grid's max |h| key (atomicMax before the arrival), so
  // after the barrier each CTA reads one word, not every CTA's maximum: all
  // CTAs reading the same few L2 lines at once serialise there. The pollers
  // back off after a short spin for the same reason.
  if (tid == 0) {
    uint32_t m = 0;
    for (int w = 0; w < kWarps; ++w) m = max(m, red[w]);
    if (m) atomicMax(a.sync + 2, m);
    __threadfence();   // h and the maximum ordered before the arrival
    atomicAdd(a.sync + 0, 1u);
    bool done = false;
    for (uint32_t it = 0; it < sm100::kSpinLimit; ++it) {
      uint32_t v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.sync + 0) : "memory");
      if (v >= (uint32_t)pl.G) { done = true; break; }
      if (it >= 32) __nanosleep(40);
    }
    if (!done) atomicCAS(a.err, 0, 32);
    hmax_s = __ldcg(a.sync + 2);
  }
  __syncthreads();

  // ---- this CTA's down block: its slot's GeGLU row, dot products ------------
  if (nr > 0) {
    __nv_bfloat16* hrow_s = reinterpret_cast<__nv_bfloat16*>(smem + cv.hrow);
    for (int i = tid; i < I / 8; i += kThreads)
      reinterpret_cast<uint4*>(hrow_s)[i] = __ldcg(reinterpret_cast<const uint4*>(a.h + (size_t)dslot * I) + i);
    const float hts = nvfp4_tensor_scale<AEOQ_BF16>(In<AEOQ_BF16>::key_to_f(hmax_s));
    const float alpha_d = hts * d_ts;
    __syncthreads();
    // the slot's GeGLU row quantized once per CTA (one 16-block per thread)
    __half2* hact_s = act_s;          // the hidden vector's operand is no longer read
    float* hsa_s = asa_s;
    for (int b = tid; b < I / 16; b += kThreads) quant16_h2(hrow_s + 16 * b, hts, hact_s + 8 * b, hsa_s + b);
    __syncthreads();
    const bool ok_dn = sm100::mbar_wait(bdown, 0, a.err, 33);
    const bool valid = ok_dn && ids_w[0][dslot] >= 0;
    const float wj = topw_s[dslot];
    const int nchunk2 = I / 32;            // <= 32: one chunk per lane
    __half2 hv[16];
    float hs[2] = {0.f, 0.f};
    if (lane < nchunk2) {
      const uint4* hp = reinterpret_cast<const uint4*>(hact_s + 16 * lane);
#pragma unroll
      for (int z = 0; z < 4; ++z) *reinterpret_cast<uint4*>(&hv[4 * z]) = hp[z];
      hs[0] = hsa_s[2 * lane];
      hs[1] = hsa_s[2 * lane + 1];
    }
    const uint8_t* dn_s = smem + cv.dn;
    const uint8_t* dsf_s = smem + cv.dsf;
    if (valid) {
      // two rows per warp iteration (r and r + kWarps) for latency hiding
      for (int r = warp; r < nr; r += 2 * kWarps) {
        const int r2 = r + kWarps;
        float s0 = 0.f, s1 = 0.f;
        if (lane < nchunk2) {
          s0 = dot32(hv, hs, *reinterpret_cast<const uint4*>(dn_s + r * rb2 + 16 * lane),
                     *reinterpret_cast<const uint16_t*>(dsf_s + r * sb2 + 2 * lane), s0);
          if (r2 < nr)
            s1 = dot32(hv, hs, *reinterpret_cast<const uint4*>(dn_s + r2 * rb2 + 16 * lane),
                       *reinterpret_cast<const uint16_t*>(dsf_s + r2 * sb2 + 2 * lane), s1);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          s0 += __shfl_xor_sync(0xffffffffu, s0, o);
          s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        }
        if (lane == 0) {
          red_add_f64(a.acc + r0 + r, (double)bf16r(bf16r(s0 * alpha_d) * wj));
          if (r2 < nr) red_add_f64(a.acc + r0 + r2, (double)bf16r(bf16r(s1 * alpha_d) * wj));
        }
      }
    }
    // arrival on the row block; the k-th arrival rounds and clears it
    __threadfence();   // this thread's adds ordered before the CTA's arrival
    __syncthreads();
    if (tid == 0) {
      const uint32_t old = atomicAdd(a.cnt + r0 / pl.rows, 1u);
      last_s = (old == (uint32_t)k - 1);
      __threadfence();   // every arrival's adds visible to the reads below
    }
    __syncthreads();
    if (last_s) {
      for (int r = tid; r < nr; r += kThreads) {
        a.out[r0 + r] = __float2bfloat16_rn((float)__ldcg(a.acc + r0 + r));
        a.acc[r0 + r] = 0.0;
      }
      if (tid == 0) a.cnt[r0 / pl.rows] = 0;
    }
  } else {
    sm100::mbar_wait(bdown, 0, a.err, 33);   // nothing in flight; the phase is complete
  }

  // ---- departure: the last CTA out resets the counters ----------------------
  if (tid == 0) {
    const uint32_t d = atomicAdd(a.sync + 1, 1u);
    if (d == (uint32_t)pl.G - 1) {
      a.sync[0] = 0;
      a.sync[1] = 0;
      a.sync[2] = 0;
      __threadfence();
    }
  }
}

}  // namespace dst
}  // namespace aeoq

using namespace aeoq;

static bool stream_plan(int64_t k, int64_t H, int64_t I, dst::Plan& p) {
  return dst::make_plan(k, H, I, device_sm_count(), p);
}

extern "C" int aeoq_moe_nvfp4_decode_stream_supported(int64_t top_k, int64_t hidden, int64_t inter) {
  dst::Plan p;
  return stream_plan(top_k, hidden, inter, p) ? 1 : 0;
}

static size_t al256(size_t v) { return (v + 255) / 256 * 256; }

// Workspace: [grid counters 256 B][row-block counters nb u32][f64 row sums H]
// [k*I bf16 GeGLU rows], each part 256-aligned. Everything but the GeGLU
// rows must be zero before the first call; every call leaves it zero.
extern "C" size_t aeoq_moe_nvfp4_decode_stream_workspace_size(int64_t top_k, int64_t hidden, int64_t inter) {
  dst::Plan p;
  if (!stream_plan(top_k, hidden, inter, p)) return 0;
  return 256 + al256((size_t)p.nb * 4) + al256((size_t)hidden * 8) + al256((size_t)(top_k * inter) * 2);
}

extern "C" int aeoq_moe_nvfp4_decode_stream(const void* hidden, const void* top_k_index, int idx_dtype,
                                            const void* top_k_weights, int64_t top_k, const uint8_t* gate_up,
                                            const uint8_t* gate_up_sf, const void* gate_up_ts, int gate_up_ts_dtype,
                                            const uint8_t* down, const uint8_t* down_sf, const void* down_ts,
                                            int down_ts_dtype, int64_t num_experts, int64_t hidden_dim,
                                            int64_t inter_dim, void* out, void* workspace, size_t workspace_bytes,
                                            int* err_word, void* stream) {
  dst::Plan pl;
  AEOQ_REQUIRE(stream_plan(top_k, hidden_dim, inter_dim, pl), AEOQ_ERR_INVALID,
               "moe_decode_stream: unsupported shape (top_k=%lld hidden=%lld inter=%lld)", (long long)top_k,
               (long long)hidden_dim, (long long)inter_dim);
  AEOQ_REQUIRE(idx_dtype == AEOQ_I32 || idx_dtype == AEOQ_I64, AEOQ_ERR_INVALID,
               "moe_decode_stream: top_k_index must be int32 or int64");
  AEOQ_REQUIRE(hidden && top_k_index && top_k_weights && gate_up && gate_up_sf && gate_up_ts && down && down_sf &&
                   down_ts && out && err_word,
               AEOQ_ERR_INVALID, "moe_decode_stream: null pointer");
  AEOQ_REQUIRE(((uintptr_t)hidden % 16 == 0) && ((uintptr_t)gate_up % 16 == 0) && ((uintptr_t)down % 16 == 0) &&
                   ((uintptr_t)gate_up_sf % 16 == 0) && ((uintptr_t)down_sf % 16 == 0),
               AEOQ_ERR_INVALID, "moe_decode_stream: hidden, weights and scales must be 16-byte aligned");
  const size_t need = aeoq_moe_nvfp4_decode_stream_workspace_size(top_k, hidden_dim, inter_dim);
  AEOQ_REQUIRE(workspace && workspace_bytes >= need && (uintptr_t)workspace % 256 == 0, AEOQ_ERR_WORKSPACE,
               "moe_decode_stream: workspace of %zu bytes (256-aligned, zeroed before first use) needed, %zu given", need,
               workspace_bytes);
  char* w = reinterpret_cast<char*>(workspace);
  dst::Args a{};
  a.hidden = reinterpret_cast<const __nv_bfloat16*>(hidden);
  a.ids = top_k_index; a.ids_dt = idx_dtype;
  a.topw = reinterpret_cast<const __nv_bfloat16*>(top_k_weights);
  a.gu = gate_up; a.gu_sf = gate_up_sf; a.gu_ts = gate_up_ts; a.gu_ts_dt = gate_up_ts_dtype;
  a.dw = down; a.dw_sf = down_sf; a.d_ts = down_ts; a.d_ts_dt = down_ts_dtype;
  a.E = num_experts;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.sync = reinterpret_cast<uint32_t*>(w);
  a.cnt = reinterpret_cast<uint32_t*>(w + 256);
  a.acc = reinterpret_cast<double*>(w + 256 + al256((size_t)pl.nb * 4));
  a.h = reinterpret_cast<__nv_bfloat16*>(w + 256 + al256((size_t)pl.nb * 4) + al256((size_t)hidden_dim * 8));
  a.err = err_word;
  {
    const int rc = func_smem_attr((const void*)dst::decode_stream_kernel, pl.bytes, -1, "moe_decode_stream");
    if (rc) return rc;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)pl.G);
  cfg.blockDim = dim3(dst::kThreads);
  cfg.dynamicSmemBytes = pl.bytes;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, dst::decode_stream_kernel, a, pl);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(AEOQ_ERR_CUDA, "decode_stream_kernel: %s", cudaGetErrorString(e));
  }
  return check_launch("decode_stream_kernel");
}
