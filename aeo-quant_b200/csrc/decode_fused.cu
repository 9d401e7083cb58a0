// One-token NVFP4 MoE expert forward as ONE persistent cooperative kernel.
//
// Restates Gemma4TextExpertsNVFP4._forward_decode_3d (aeo_quant
// src/aeo_quant/bridges/gemma4/modeling_nvfp4.py:132-186). At one token the
// cost is streaming the k selected experts' packed weights (26.8 MB for
// Gemma-4-26B-A4B: k=8, H=2816, I=704), so the kernel is organised around
// HBM, not arithmetic:
//
//  1. Each of the G = #SM CTAs owns a contiguous slice of the k*I gate/up
//     row pairs and a slice of the H down rows (for all k slots). At entry
//     one thread issues cp.async.bulk copies of the whole slice into shared
//     memory (~180 KB per CTA), so every SM streams from HBM from t = 0.
//  2. Meanwhile the CTA quantizes the hidden vector (global amax, bf16 tensor
//     scale, per-16 e4m3 scales, E2M1 nibbles: quantize_2d_to_nvfp4, :150-153)
//     into exact fp16 operands in shared memory.
//  3. gate/up dot products from shared memory (fp16 exact per 16-block, f32
//     across blocks), GeGLU in bf16 (:155-162); h goes to global memory and
//     the CTA's |h| maximum to a per-CTA slot.
//  4. One grid barrier (bounded spin on an arrival counter; cooperative launch
//     guarantees co-residency). Every CTA then reduces the G maxima to the
//     shared tensor scale (:164-172) and re-quantizes all of h itself.
//  5. down dot products from shared memory, bf16(bf16(a*d_j) * w_j), summed
//     over the k slots and rounded once (:174-186).
// The counters self-reset: the last CTA to leave zeroes them, so a zeroed
// workspace stays valid call after call on one stream.
#include <cstdlib>

#include "common.cuh"
#include "sm100.cuh"

namespace aeoq {

constexpr int kFThreads = 512;
constexpr int kFWarps = kFThreads / 32;
constexpr int kFMaxTopK = 16;
constexpr int kFMaxDownRows = 32;
constexpr int kSmemCap = 232448 - 1024;   // opt-in shared memory per CTA less static use

struct FusedShape {
  int64_t E, H, I;
  int k, G;
  int ppc;      // gate/up row pairs per CTA
  int rpc;      // down rows per CTA
  size_t off_gate, off_up, off_gsf, off_usf, off_dn, off_dsf, off_act, off_asa, off_hact, off_hsa, off_prod,
      bytes;
};

__host__ __device__ inline size_t al128(size_t v) { return (v + 127) / 128 * 128; }

__host__ __device__ inline FusedShape fused_shape(int64_t E, int64_t H, int64_t I, int k, int G) {
  FusedShape s{};
  s.E = E; s.H = H; s.I = I; s.k = k; s.G = G;
  s.ppc = (int)((k * I + G - 1) / G);
  s.rpc = (int)((H + G - 1) / G);
  const size_t rb = H / 2, sb = H / 16, rb2 = I / 2, sb2 = I / 16;
  size_t o = 0;
  s.off_gate = o; o = al128(o + s.ppc * rb);
  s.off_up = o;   o = al128(o + s.ppc * rb);
  s.off_gsf = o;  o = al128(o + s.ppc * sb);
  s.off_usf = o;  o = al128(o + s.ppc * sb);
  s.off_dn = o;   o = al128(o + (size_t)s.rpc * k * rb2);
  s.off_dsf = o;  o = al128(o + (size_t)s.rpc * k * sb2);
  s.off_act = o;  o = al128(o + (H / 16) * 8 * sizeof(__half2));
  s.off_asa = o;  o = al128(o + (H / 16) * sizeof(float));
  s.off_hact = o; o = al128(o + (k * I / 16) * 8 * sizeof(__half2));
  s.off_hsa = o;  o = al128(o + (k * I / 16) * sizeof(float));
  s.off_prod = o; o = al128(o + (size_t)kFMaxTopK * kFMaxDownRows * sizeof(float));
  s.bytes = o + 128;   // two mbarriers
  return s;
}

struct FusedArgs {
  const __nv_bfloat16* hidden;
  const void* ids; int ids_dt;
  const __nv_bfloat16* topw;
  const uint8_t* gu; const uint8_t* gu_sf; const void* gu_ts; int gu_ts_dt;
  const uint8_t* dw; const uint8_t* dw_sf; const void* d_ts; int d_ts_dt;
  __nv_bfloat16* out;
  __nv_bfloat16* h;      // k*I bf16 intermediate
  uint32_t* parts;       // G amax keys
  uint32_t* sync;        // [0] arrivals, [1] departures, [2] error code
};

// Phase timestamps for development builds (-DAEOQ_DECODE_TRACE): thread 0 of
// each CTA records %globaltimer at each phase boundary into the workspace.
#ifdef AEOQ_DECODE_TRACE
#define TRACE(i)                                                                               \
  do {                                                                                         \
    if (tid == 0) {                                                                            \
      uint64_t t_;                                                                             \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                   \
      reinterpret_cast<uint64_t*>(a.h + (size_t)s.k * s.I)[blockIdx.x * 16 + (i)] = t_;      \
    }                                                                                          \
  } while (0)
#else
#define TRACE(i) do {} while (0)
#endif

// Quantize 16 bf16 values (global; read L2-coherently when another CTA of
// this grid wrote them) and store exact halves + 2^14-scaled block scale.
template <bool kCoherent>
__device__ __forceinline__ void quant_block_to_smem(const __nv_bfloat16* src, float ts, __half2* dst, float* sa16k) {
  float v[16];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const uint4 u = kCoherent ? __ldcg(reinterpret_cast<const uint4*>(src + 8 * q))
                              : *reinterpret_cast<const uint4*>(src + 8 * q);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[8 * q + j] = __bfloat162float(e[j]);
  }
  uint32_t w0, w1;
  const uint32_t sf = nvfp4_quant_block(v, ts, w0, w1);
  __half2 t[4];
  fp4x8_to_half2x4_exact(w0, t);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = t[i];
  fp4x8_to_half2x4_exact(w1, t);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[4 + i] = t[i];
  *sa16k = e4m3_decode(sf) * 16384.0f;
}

constexpr int kPairsPerBar = 16;   // gate/up pairs per arrival barrier
constexpr int kMaxGuBars = 8;

__global__ void __launch_bounds__(kFThreads, 1) moe_decode_fused_kernel(FusedArgs a, FusedShape s) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint32_t red[kFWarps];
  __shared__ int64_t ids_s[kFMaxTopK];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + s.bytes - 128);   // [0..kMaxGuBars) gate/up, [kMaxGuBars] down
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t H = s.H, I = s.I;
  const int k = s.k;
  const size_t rb = H / 2, sb = H / 16, rb2 = I / 2, sb2 = I / 16;
  const int64_t p0 = (int64_t)blockIdx.x * s.ppc;
  const int64_t p1 = min((int64_t)k * I, p0 + s.ppc);
  const int np = (int)max((int64_t)0, p1 - p0);
  const int nbar = (np + kPairsPerBar - 1) / kPairsPerBar;
  const int64_t r0 = (int64_t)blockIdx.x * s.rpc;
  const int nr = (int)max((int64_t)0, min(H, r0 + s.rpc) - r0);
  uint8_t* gate_s = smem + s.off_gate;
  uint8_t* up_s = smem + s.off_up;
  uint8_t* gsf_s = smem + s.off_gsf;
  uint8_t* usf_s = smem + s.off_usf;
  uint8_t* dn_s = smem + s.off_dn;
  uint8_t* dsf_s = smem + s.off_dsf;
  __half2* act_s = reinterpret_cast<__half2*>(smem + s.off_act);
  float* asa_s = reinterpret_cast<float*>(smem + s.off_asa);
  __half2* hact_s = reinterpret_cast<__half2*>(smem + s.off_hact);
  float* hsa_s = reinterpret_cast<float*>(smem + s.off_hsa);
  float* prod_s = reinterpret_cast<float*>(smem + s.off_prod);
  int* err = reinterpret_cast<int*>(a.sync + 2);
  TRACE(0);

  // ---- 1. expert ids (one load latency), then every weight copy -----------
  if (warp == 0) {
    int64_t myid = -1;
    if (lane < k) myid = load_index(a.ids, a.ids_dt, lane);
    if (lane < k) ids_s[lane] = myid;
    if (lane == 0) {
      for (int b = 0; b <= kMaxGuBars; ++b) sm100::mbar_init(bars + b, 1);
      sm100::fence_barrier_init();
    }
    __syncwarp();
    if (lane == 0) {
      // gate/up: kPairsPerBar pairs per barrier, split at slot boundaries
      for (int b = 0; b < nbar; ++b) {
        const int i0 = b * kPairsPerBar, i1 = min(np, i0 + kPairsPerBar);
        sm100::mbar_arrive_expect_tx(bars + b, (uint32_t)((i1 - i0) * (2 * rb + 2 * sb)));
        int64_t p = p0 + i0;
        int dst = i0;
        while (p < p0 + i1) {
          const int64_t slot = p / I, n = p - slot * I;
          const int64_t len = min(p0 + i1 - p, I - n);
          const int64_t e = ids_s[slot];
          if (e >= 0 && e < s.E) {
            const uint8_t* g = a.gu + (e * 2 * I + n) * rb;
            const uint8_t* gs = a.gu_sf + (e * 2 * I + n) * sb;
            bulk_g2s(gate_s + dst * rb, g, (uint32_t)(len * rb), bars + b);
            bulk_g2s(up_s + dst * rb, g + I * rb, (uint32_t)(len * rb), bars + b);
            bulk_g2s(gsf_s + dst * sb, gs, (uint32_t)(len * sb), bars + b);
            bulk_g2s(usf_s + dst * sb, gs + I * sb, (uint32_t)(len * sb), bars + b);
          } else {
            asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" ::"r"(sm100::smem_u32(bars + b)),
                         "r"((uint32_t)(len * (2 * rb + 2 * sb)))
                         : "memory");
          }
          dst += (int)len;
          p += len;
        }
      }
      uint64_t* bdn = bars + kMaxGuBars;
      sm100::mbar_arrive_expect_tx(bdn, (uint32_t)((size_t)nr * k * rb2));
      for (int j = 0; j < k && nr > 0; ++j) {
        const int64_t e = ids_s[j];
        if (e >= 0 && e < s.E) {
          bulk_g2s(dn_s + (size_t)j * nr * rb2, a.dw + (e * H + r0) * rb2, (uint32_t)(nr * rb2), bdn);
        } else {
          asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" ::"r"(sm100::smem_u32(bdn)),
                       "r"((uint32_t)(nr * rb2))
                       : "memory");
        }
      }
    }
  }
  TRACE(1);
  // hidden amax (independent of the ids)
  uint32_t key = 0;
  for (int64_t i = tid; i < H / 8; i += kFThreads) {
    const uint4 u = *reinterpret_cast<const uint4*>(a.hidden + 8 * i);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) key = max(key, In<AEOQ_BF16>::abs_key(e[j]));
  }
  key = warp_umax(key);
  if (lane == 0) red[warp] = key;
  __syncthreads();   // publishes ids_s, the barrier inits and red
  key = 0;
#pragma unroll
  for (int w = 0; w < kFWarps; ++w) key = max(key, red[w]);
  const float ts = nvfp4_tensor_scale<AEOQ_BF16>(In<AEOQ_BF16>::key_to_f(key));
  const float alpha = ts * load_scalar_f(a.gu_ts, a.gu_ts_dt);
  for (int64_t b = tid; b < H / 16; b += kFThreads)
    quant_block_to_smem<false>(a.hidden + 16 * b, ts, act_s + 8 * b, asa_s + b);
  // down scale rows (44 B per row: not bulk-copy aligned) with plain loads
  {
    const int words = (int)(nr * sb2 / 4);   // per slot
    for (int idx = tid; idx < k * words; idx += kFThreads) {
      const int j = idx / words, wdx = idx - j * words;
      const int64_t e = ids_s[j];
      uint32_t v = 0;
      if (e >= 0 && e < s.E) v = *reinterpret_cast<const uint32_t*>(a.dw_sf + (e * H + r0) * sb2 + 4 * wdx);
      reinterpret_cast<uint32_t*>(dsf_s + (size_t)j * nr * sb2)[wdx] = v;
    }
  }
  __syncthreads();
  TRACE(2);

  // ---- 3. gate/up GEMV + GeGLU, pair groups consumed as they land ---------
  constexpr int kCPL = 4;   // 16-byte chunks per lane per row (H <= 4096)
  const int nchunk = (int)(H / 32);
  __half2 act[kCPL][16];
  float sa[kCPL][2];
#pragma unroll
  for (int q = 0; q < kCPL; ++q) {
    const int c = lane + 32 * q;
    if (c < nchunk) {
      const uint4* ap = reinterpret_cast<const uint4*>(act_s + 16 * c);
#pragma unroll
      for (int z = 0; z < 4; ++z) *reinterpret_cast<uint4*>(&act[q][4 * z]) = ap[z];
      sa[q][0] = asa_s[2 * c];
      sa[q][1] = asa_s[2 * c + 1];
    }
  }
  uint32_t hkey = 0;
  bool ok = true;
  int waited_bar = -1;
  for (int i = warp; i < np; i += kFWarps) {
    const int b = i / kPairsPerBar;
    if (b > waited_bar) {
      for (int bb = waited_bar + 1; bb <= b; ++bb) ok &= sm100::mbar_wait(bars + bb, 0, err, 1);
      waited_bar = b;
    }
    const int64_t slot = (p0 + i) / I;
    const int64_t e = ids_s[slot];
    const bool valid = ok && e >= 0 && e < s.E;   // an invalid id contributes zeros
    float ag = 0.f, au = 0.f;
    if (valid) {
#pragma unroll
      for (int q = 0; q < kCPL; ++q) {
        const int c = lane + 32 * q;
        if (c < nchunk) {
          const uint4 gw = *reinterpret_cast<const uint4*>(gate_s + i * rb + 16 * c);
          const uint4 uw = *reinterpret_cast<const uint4*>(up_s + i * rb + 16 * c);
          const uint16_t gs = *reinterpret_cast<const uint16_t*>(gsf_s + i * sb + 2 * c);
          const uint16_t us = *reinterpret_cast<const uint16_t*>(usf_s + i * sb + 2 * c);
          ag = chunk_dot(act[q], sa[q], gw, gs, ag);
          au = chunk_dot(act[q], sa[q], uw, us, au);
        }
      }
    }
    ag = warp_sum(ag);
    au = warp_sum(au);
    if (lane == 0) {
      const float g = bf16r(ag * alpha), u = bf16r(au * alpha);
      const __nv_bfloat16 hv = __float2bfloat16_rn(bf16r(gelu_tanh(g)) * u);
      a.h[p0 + i] = hv;
      hkey = max(hkey, In<AEOQ_BF16>::abs_key(hv));
    }
  }
  // barriers this warp never waited on still have to complete before exit
  for (int bb = waited_bar + 1; bb < nbar; ++bb) sm100::mbar_wait(bars + bb, 0, err, 1);
  TRACE(3);
  hkey = warp_umax(hkey);
  __threadfence();   // h stores of every writer ordered before the arrival below
  __syncthreads();
  if (lane == 0) red[warp] = hkey;
  __syncthreads();
  TRACE(4);

  // ---- 4. grid barrier ----------------------------------------------------
  if (tid == 0) {
    uint32_t m = 0;
    for (int w = 0; w < kFWarps; ++w) m = max(m, red[w]);
    a.parts[blockIdx.x] = m;
    __threadfence();
    atomicAdd(a.sync + 0, 1u);
    bool done = false;
    for (uint32_t it = 0; it < sm100::kSpinLimit; ++it) {
      uint32_t v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.sync + 0) : "memory");
      if (v >= (uint32_t)s.G) { done = true; break; }
      __nanosleep(32);
    }
    if (!done) atomicCAS(err, 0, 2);
  }
  __syncthreads();
  TRACE(5);

  // shared tensor scale of h over all CTAs, then re-quantize all of h here
  uint32_t hk = 0;
  for (int i = tid; i < s.G; i += kFThreads) hk = max(hk, __ldcg(a.parts + i));
  hk = warp_umax(hk);
  if (lane == 0) red[warp] = hk;
  __syncthreads();
  hk = 0;
#pragma unroll
  for (int w = 0; w < kFWarps; ++w) hk = max(hk, red[w]);
  const float hts = nvfp4_tensor_scale<AEOQ_BF16>(In<AEOQ_BF16>::key_to_f(hk));
  const float alpha_d = hts * load_scalar_f(a.d_ts, a.d_ts_dt);
  for (int64_t b = tid; b < (int64_t)k * I / 16; b += kFThreads)
    quant_block_to_smem<true>(a.h + 16 * b, hts, hact_s + 8 * b, hsa_s + b);
  __syncthreads();
  TRACE(6);

  // ---- 5. down GEMV + weighted combine: warps own one slot each ------------
  const bool ok_dn = sm100::mbar_wait(bars + kMaxGuBars, 0, err, 3);
  TRACE(7);
  const int nchunk2 = (int)(I / 32);
  const int wpj = kFWarps / k;   // warps per slot (k <= 16)
  if (ok_dn && warp < wpj * k) {
    const int j = warp / wpj;
    const int64_t e = ids_s[j];
    const bool valid = e >= 0 && e < s.E;
    const float wj = __bfloat162float(a.topw[j]);
    // the intermediate dimension is at most 2048: at most two chunks per lane
    __half2 hv0[16], hv1[16];
    float hs0[2] = {0.f, 0.f}, hs1[2] = {0.f, 0.f};
    const int c0 = lane, c1 = lane + 32;
    if (c0 < nchunk2) {
      const int hb = (int)(j * (I / 16) + 2 * c0);
      const uint4* ap = reinterpret_cast<const uint4*>(hact_s + hb * 8);
#pragma unroll
      for (int z = 0; z < 4; ++z) *reinterpret_cast<uint4*>(&hv0[4 * z]) = ap[z];
      hs0[0] = hsa_s[hb];
      hs0[1] = hsa_s[hb + 1];
    }
    if (c1 < nchunk2) {
      const int hb = (int)(j * (I / 16) + 2 * c1);
      const uint4* ap = reinterpret_cast<const uint4*>(hact_s + hb * 8);
#pragma unroll
      for (int z = 0; z < 4; ++z) *reinterpret_cast<uint4*>(&hv1[4 * z]) = ap[z];
      hs1[0] = hsa_s[hb];
      hs1[1] = hsa_s[hb + 1];
    }
    for (int r = warp % wpj; r < nr; r += wpj) {
      float acc = 0.f;
      if (valid) {
        const size_t row = (size_t)j * nr + r;
        if (c0 < nchunk2)
          acc = chunk_dot(hv0, hs0, *reinterpret_cast<const uint4*>(dn_s + row * rb2 + 16 * c0),
                          *reinterpret_cast<const uint16_t*>(dsf_s + row * sb2 + 2 * c0), acc);
        if (c1 < nchunk2)
          acc = chunk_dot(hv1, hs1, *reinterpret_cast<const uint4*>(dn_s + row * rb2 + 16 * c1),
                          *reinterpret_cast<const uint16_t*>(dsf_s + row * sb2 + 2 * c1), acc);
      }
      acc = warp_sum(acc);
      if (lane == 0) prod_s[j * kFMaxDownRows + r] = bf16r(bf16r(acc * alpha_d) * wj);
    }
  }
  __syncthreads();
  if (tid < nr) {
    float acc = 0.f;
    for (int j = 0; j < k; ++j) acc += prod_s[j * kFMaxDownRows + tid];
    a.out[r0 + tid] = __float2bfloat16_rn(acc);
  }
  TRACE(8);

  // ---- departure: the last CTA out resets the counters ------------------
  if (tid == 0) {
    const uint32_t d = atomicAdd(a.sync + 1, 1u);
    if (d == (uint32_t)s.G - 1) {
      a.sync[0] = 0;
      a.sync[1] = 0;
      __threadfence();
    }
  }
}

static int fused_grid() { return device_sm_count(); }

}  // namespace aeoq

using namespace aeoq;

// Workspace: [sync 256 B][parts G*4][h k*I bf16], all 256-aligned.
extern "C" size_t aeoq_moe_nvfp4_decode_fused_workspace_size(int64_t top_k, int64_t hidden, int64_t inter) {
  (void)hidden;
  const size_t G = (size_t)fused_grid();
  return 256 + (G * 4 + 255) / 256 * 256 + ((size_t)(top_k * inter) * 2 + 255) / 256 * 256;
}

extern "C" int aeoq_moe_nvfp4_decode_fused_supported(int64_t top_k, int64_t hidden, int64_t inter) {
  if (top_k < 1 || top_k > kFMaxTopK) return 0;
  if (hidden % 256 != 0 || inter % 64 != 0 || hidden <= 0 || inter <= 0) return 0;
  if (hidden > 4096 || inter > 2048) return 0;
  const FusedShape s = fused_shape(0, hidden, inter, (int)top_k, fused_grid());
  if (s.rpc > kFMaxDownRows) return 0;
  if ((s.ppc + kPairsPerBar - 1) / kPairsPerBar > kMaxGuBars) return 0;
  return s.bytes <= (size_t)kSmemCap ? 1 : 0;
}

extern "C" int aeoq_moe_nvfp4_decode_fused(const void* hidden, const void* top_k_index, int idx_dtype,
                                           const void* top_k_weights, int64_t top_k, const uint8_t* gate_up,
                                           const uint8_t* gate_up_sf, const void* gate_up_ts, int gate_up_ts_dtype,
                                           const uint8_t* down, const uint8_t* down_sf, const void* down_ts,
                                           int down_ts_dtype, int64_t num_experts, int64_t hidden_dim,
                                           int64_t inter_dim, void* out, void* workspace, size_t workspace_bytes,
                                           void* stream) {
  AEOQ_REQUIRE(aeoq_moe_nvfp4_decode_fused_supported(top_k, hidden_dim, inter_dim), AEOQ_ERR_INVALID,
               "moe_decode_fused: unsupported shape (top_k=%lld hidden=%lld inter=%lld)", (long long)top_k,
               (long long)hidden_dim, (long long)inter_dim);
  AEOQ_REQUIRE(idx_dtype == AEOQ_I32 || idx_dtype == AEOQ_I64, AEOQ_ERR_INVALID,
               "moe_decode_fused: top_k_index must be int32 or int64");
  AEOQ_REQUIRE(hidden && top_k_index && top_k_weights && gate_up && gate_up_sf && gate_up_ts && down && down_sf &&
                   down_ts && out,
               AEOQ_ERR_INVALID, "moe_decode_fused: null pointer");
  AEOQ_REQUIRE(((uintptr_t)hidden % 16 == 0) && ((uintptr_t)gate_up % 16 == 0) && ((uintptr_t)down % 16 == 0) &&
                   ((uintptr_t)gate_up_sf % 16 == 0) && ((uintptr_t)down_sf % 4 == 0),
               AEOQ_ERR_INVALID, "moe_decode_fused: weights must be 16-byte aligned (down scales 4-byte)");
  const size_t need = aeoq_moe_nvfp4_decode_fused_workspace_size(top_k, hidden_dim, inter_dim);
  AEOQ_REQUIRE(workspace && workspace_bytes >= need && (uintptr_t)workspace % 256 == 0, AEOQ_ERR_WORKSPACE,
               "moe_decode_fused: workspace of %zu bytes (256-aligned, first 256 B zero) needed, %zu given", need,
               workspace_bytes);
  const int G = fused_grid();
  const FusedShape s = fused_shape(num_experts, hidden_dim, inter_dim, (int)top_k, G);
  char* w = reinterpret_cast<char*>(workspace);
  FusedArgs a{};
  a.hidden = reinterpret_cast<const __nv_bfloat16*>(hidden);
  a.ids = top_k_index; a.ids_dt = idx_dtype;
  a.topw = reinterpret_cast<const __nv_bfloat16*>(top_k_weights);
  a.gu = gate_up; a.gu_sf = gate_up_sf; a.gu_ts = gate_up_ts; a.gu_ts_dt = gate_up_ts_dtype;
  a.dw = down; a.dw_sf = down_sf; a.d_ts = down_ts; a.d_ts_dt = down_ts_dtype;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.sync = reinterpret_cast<uint32_t*>(w);
  a.parts = reinterpret_cast<uint32_t*>(w + 256);
  a.h = reinterpret_cast<__nv_bfloat16*>(w + 256 + ((size_t)G * 4 + 255) / 256 * 256);
  {
    const int rc = func_smem_attr((const void*)moe_decode_fused_kernel, s.bytes, -1, "moe_decode_fused");
    if (rc) return rc;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)G);
  cfg.blockDim = dim3(kFThreads);
  cfg.dynamicSmemBytes = s.bytes;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, moe_decode_fused_kernel, a, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(AEOQ_ERR_CUDA, "moe_decode_fused_kernel: %s", cudaGetErrorString(e));
  }
  return check_launch("moe_decode_fused_kernel");
}

// ---------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot allocate device memory at the point where they run the
// expert forward: a serving runtime that reserves every byte of device memory
// at start-up and forbids allocation on its request path, or a plugin hosted
// by a framework whose allocator it cannot reach. For them this entry point
// takes the same inputs and outputs as aeoq_moe_nvfp4_decode_fused but no
// workspace: its scratch (arrival counters, per-CTA maxima, the bf16
// intermediate) lives in the file-scope device array below, kNoAllocScratch
// bytes per GPU, held by every GPU that loads the library until the process
// exits.
//
// * Host code only names the array through a host-side stand-in, so its
//   device address is looked up with cudaGetSymbolAddress, once per device,
//   with that device current. The first call on a device performs this
//   lookup; make that first call before any stream capture.
// * All calls on a device share the array and it keeps the last call's
//   contents. Each call clears the counters that must start at zero
//   (cudaMemsetAsync on its stream). Calls whose kernels overlap on the GPU
//   (different streams without ordering) race on the array.
// * Shapes whose scratch exceeds kNoAllocScratch are rejected.
// ---------------------------------------------------------------------------
#include <mutex>

namespace aeoq {
constexpr size_t kNoAllocScratch = 128 * 1024;
constexpr int kNoAllocMaxDevices = 64;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratch];
static void* g_noalloc_ptr[kNoAllocMaxDevices] = {};
static std::mutex g_noalloc_mu;

static int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(AEOQ_ERR_CUDA, "moe_decode_fused_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  }
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return set_error(AEOQ_ERR_UNSUPPORTED, "moe_decode_fused_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      return set_error(AEOQ_ERR_CUDA, "moe_decode_fused_noalloc: cudaGetSymbolAddress: %s",
                       cudaGetErrorString(e));
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return AEOQ_OK;
}
}  // namespace aeoq

extern "C" size_t aeoq_moe_nvfp4_decode_fused_noalloc_max_scratch(void) { return aeoq::kNoAllocScratch; }

extern "C" int aeoq_moe_nvfp4_decode_fused_noalloc(const void* hidden, const void* top_k_index, int idx_dtype,
                                                   const void* top_k_weights, int64_t top_k,
                                                   const uint8_t* gate_up, const uint8_t* gate_up_sf,
                                                   const void* gate_up_ts, int gate_up_ts_dtype,
                                                   const uint8_t* down, const uint8_t* down_sf,
                                                   const void* down_ts, int down_ts_dtype, int64_t num_experts,
                                                   int64_t hidden_dim, int64_t inter_dim, void* out,
                                                   void* stream) {
  const size_t need = aeoq_moe_nvfp4_decode_fused_workspace_size(top_k, hidden_dim, inter_dim);
  AEOQ_REQUIRE(need <= kNoAllocScratch, AEOQ_ERR_INVALID,
               "moe_decode_fused_noalloc: needs %zu bytes of scratch, the static array holds %zu "
               "(top_k * inter too large); use aeoq_moe_nvfp4_decode_fused with a workspace",
               need, kNoAllocScratch);
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  cudaError_t e = cudaMemsetAsync(scratch, 0, 256, (cudaStream_t)stream);   // arrival/departure counters
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(AEOQ_ERR_CUDA, "moe_decode_fused_noalloc: clearing counters: %s", cudaGetErrorString(e));
  }
  return aeoq_moe_nvfp4_decode_fused(hidden, top_k_index, idx_dtype, top_k_weights, top_k, gate_up, gate_up_sf,
                                     gate_up_ts, gate_up_ts_dtype, down, down_sf, down_ts, down_ts_dtype,
                                     num_experts, hidden_dim, inter_dim, out, scratch, kNoAllocScratch, stream);
}
