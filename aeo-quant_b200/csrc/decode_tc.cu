// One-token NVFP4 MoE expert forward on the tensor cores (two launches).
//
// Restates Gemma4TextExpertsNVFP4._forward_decode_3d (aeo_quant
// src/aeo_quant/bridges/gemma4/modeling_nvfp4.py:132-186). At one token the
// work is a stream of the k selected experts' packed weights; the FP4 x FP4
// products, their e4m3 scaling and the f32 sums are left to tcgen05.mma
// (kind::mxf4nvf4, M = 128 weight rows, N = 8 with the token in column 0),
// so the SMs only move bytes and run the small quantizations.
//
//  launch 1  gate_up + GeGLU. CTA (m, j): 64 gate rows 64m.. and the 64
//            matching up rows of expert ids[j], K streamed through an 8-deep
//            TMA ring. Meanwhile four warps quantize the hidden vector
//            (quantize_2d_to_nvfp4 semantics, :150-153) straight into the
//            MMA's B tile and scale atoms. Epilogue: h = bf16(bf16(gelu(g))*u)
//            (:155-162) to global memory, the CTA's max |h| to a slot.
//  launch 2  down + combine, launched early (programmatic dependent launch):
//            CTA (m, j) copies its 128 x I down rows of expert ids[j] into
//            shared memory while launch 1 still runs, then waits, reduces
//            the maxima to the shared tensor scale (:164-172), quantizes its
//            slot's h row into the B tile, runs the MMAs, and writes
//            bf16(bf16(a*d) * w_j) (:183). The last of the k CTAs of a row
//            tile (arrival counter) sums the k rows in f32 and rounds once
//            (:184-186). Counters reset themselves.
//
// Every wait is bounded (sm100::mbar_wait); TMEM is freed on every path.
#include <cuda.h>

#include <cstdlib>

#include "common.cuh"
#include "sm100.cuh"

namespace aeoq {

int make_tmap(CUtensorMap* m, const void* ptr, int64_t rows, int64_t row_bytes, int64_t ld, int box_rows);

namespace dtc {

#ifdef AEOQ_TC_TRACE
__device__ uint64_t* g_dtrace = nullptr;
#define DT(slot)                                                                                     \
  do {                                                                                               \
    if (g_dtrace) {                                                                                  \
      uint64_t t_;                                                                                   \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                         \
      g_dtrace[(kTraceBase + blockIdx.y * gridDim.x + blockIdx.x) * 32 + (slot)] = t_;                \
    }                                                                                                \
  } while (0)
#define DC(slot, v) do { if (g_dtrace) g_dtrace[(kTraceBase + blockIdx.y * gridDim.x + blockIdx.x) * 32 + (slot)] = (v); } while (0)
#else
#define DT(slot) do {} while (0)
#define DC(slot, v) do {} while (0)
#endif

constexpr int kThreads = 192;
constexpr int kRing = 8;            // launch-1 ring depth (16 KB A tiles)
constexpr int kN = 8;               // MMA N: the token plus 7 zero columns
constexpr uint32_t kAccCol = 0, kSfaCol = 8, kSfbCol = 24;   // launch-1 TMEM columns
constexpr int kMaxKB = 64;          // K / 64 for the hidden size (H <= 4096)
constexpr int kMaxKB2 = 32;         // K / 64 for the intermediate size (I <= 2048)

struct Args {
  const __nv_bfloat16* hidden;
  const void* ids; int ids_dt;
  const __nv_bfloat16* topw;
  const uint8_t* gu_atoms;  const void* gu_ts; int gu_ts_dt;
  const uint8_t* dw_atoms;  const void* d_ts;  int d_ts_dt;
  int64_t E, H, I;
  int k;
  __nv_bfloat16* h;        // [k][I]
  uint32_t* parts;          // [k * I / 64] maxima of launch 1
  __nv_bfloat16* c;         // [k][H] weighted expert outputs
  uint32_t* counters;       // [H / 128] arrival counters (self-resetting)
  __nv_bfloat16* out;       // [H]
  int* err;
};

struct Smem1 {
  uint64_t full[kRing], empty[kRing], bready, accum;
  uint32_t tmem;
  uint32_t red[4];
  float xchg[64];
};

// Quantize one 16-value block of bf16 (src) into row 0 of a B tile set:
// packed bytes at btile + (b / 16) * 1024 + (b % 16) * 8 (row 0 of a
// 128-byte-swizzled 8-row tile is unpermuted) and its scale at byte b % 4 of
// row 0 in atom b / 4.
template <bool kCoherent>
__device__ __forceinline__ void quant_to_btile(const __nv_bfloat16* src, float ts, int64_t b, uint8_t* btile,
                                               uint8_t* sfb) {
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
  *reinterpret_cast<uint2*>(btile + (b >> 4) * 1024 + (b & 15) * 8) = make_uint2(w0, w1);
  sfb[(b >> 2) * 512 + (b & 3)] = (uint8_t)sf;
}

// Max |x| key over n bf16 values by the 128 threads of warps 2-5.
__device__ __forceinline__ uint32_t amax_key128(const __nv_bfloat16* x, int64_t n, int t, uint32_t* red) {
  uint32_t key = 0;
  for (int64_t i = t; i < n / 8; i += 128) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + 8 * i);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) key = max(key, In<AEOQ_BF16>::abs_key(e[j]));
  }
  key = warp_umax(key);
  if ((t & 31) == 0) red[t >> 5] = key;
  asm volatile("bar.sync 2, 128;" ::: "memory");
  key = max(max(red[0], red[1]), max(red[2], red[3]));
  asm volatile("bar.sync 2, 128;" ::: "memory");
  return key;
}

__device__ __forceinline__ void zero_smem128(uint8_t* p, int bytes, int t) {
  for (int i = t; i < bytes / 16; i += 128) reinterpret_cast<uint4*>(p)[i] = make_uint4(0, 0, 0, 0);
}

// ------------------------------------------------------------------ launch 1
__global__ void __launch_bounds__(kThreads, 1) decode_gateup_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                       const Args a) {
  constexpr int kTraceBase = 0;
  if (threadIdx.x == 0) DT(0);
  extern __shared__ __align__(1024) uint8_t dsm[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  const int H = (int)a.H, I = (int)a.I;
  const int kb_total = H / 64, num_kt = (H + 255) / 256;
  uint8_t* ringA = base;                                   // kRing x 16 KB
  uint8_t* ringSFA = ringA + kRing * 16384;                // kRing x 2 KB
  uint8_t* btile = ringSFA + kRing * 2048;                 // num_kt x 1 KB
  uint8_t* sfb = btile + num_kt * 1024;                    // kb_total x 512 B
  Smem1* sh = reinterpret_cast<Smem1*>(sfb + kb_total * 512);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m = blockIdx.x, j = blockIdx.y;

  if (tid == 0) {
    for (int s = 0; s < kRing; ++s) {
      sm100::mbar_init(&sh->full[s], 1);
      sm100::mbar_init(&sh->empty[s], 1);
    }
    sm100::mbar_init(&sh->bready, 4);
    sm100::mbar_init(&sh->accum, 1);
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tmA);
  }
  if (warp == 1) sm100::tmem_alloc(&sh->tmem, 64);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = sh->tmem;
  pdl_wait();        // inputs may come from the preceding kernel
  pdl_trigger();     // the down launch may start its weight prefetch
  const int64_t e = load_index(a.ids, a.ids_dt, j);
  const bool valid = e >= 0 && e < a.E;

  if (warp == 0) {
    const bool leader = sm100::elect_one();
    const uint8_t* sfa_src = a.gu_atoms + ((valid ? e : 0) * (I / 64) + m) * (int64_t)kb_total * 512;
    const int32_t row_g = (int32_t)((valid ? e : 0) * 2 * I + 64 * m);
    for (int kt = 0; kt < num_kt && valid; ++kt) {
      const int s = kt % kRing;
      const uint32_t ph = (kt / kRing) & 1;
      if (!sm100::mbar_wait(&sh->empty[s], ph ^ 1, a.err, 21)) break;
      const int nkb = min(4, kb_total - kt * 4);
      if (leader) {
        sm100::mbar_arrive_expect_tx(&sh->full[s], 16384u + (uint32_t)nkb * 512u);
        bulk_g2s(ringSFA + s * 2048, sfa_src + (size_t)kt * 4 * 512, (uint32_t)nkb * 512, &sh->full[s]);
        sm100::tma_load_2d(ringA + s * 16384, &tmA, kt * 128, row_g, &sh->full[s]);
        sm100::tma_load_2d(ringA + s * 16384 + 8192, &tmA, kt * 128, row_g + I, &sh->full[s]);
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    const bool leader = sm100::elect_one();
    const uint32_t idesc = sm100::idesc_nvf4(kN);
    bool ok = sm100::mbar_wait(&sh->bready, 0, a.err, 22);
    if (sm100::elect_one()) DT(5);
    for (int kt = 0; kt < num_kt && ok && valid; ++kt) {
      const int s = kt % kRing;
      const uint32_t ph = (kt / kRing) & 1;
      if (!sm100::mbar_wait(&sh->full[s], ph, a.err, 23)) { ok = false; break; }
      if (kt < 11 && sm100::elect_one()) DT(6 + kt);
      const long long c0_ = clock64();
      sm100::tc_fence_after();
      const int nkb = min(4, kb_total - kt * 4);
      if (leader) {
        for (int kb = 0; kb < nkb; ++kb) {
          sm100::tc_cp_32x128b_warpx4(tmem + kSfaCol + 4 * kb,
                                      sm100::sdesc_sf_atom(sm100::smem_u32(ringSFA + s * 2048 + kb * 512)));
          sm100::tc_cp_32x128b_warpx4(tmem + kSfbCol + 4 * kb,
                                      sm100::sdesc_sf_atom(sm100::smem_u32(sfb + (kt * 4 + kb) * 512)));
        }
        for (int kb = 0; kb < nkb; ++kb) {
          const uint64_t ad = sm100::sdesc_k_sw128(sm100::smem_u32(ringA + s * 16384) + kb * 32);
          const uint64_t bd = sm100::sdesc_k_sw128(sm100::smem_u32(btile + kt * 1024) + kb * 32);
          sm100::tc_mma_nvf4(tmem + kAccCol, ad, bd, idesc, tmem + kSfaCol + 4 * kb, tmem + kSfbCol + 4 * kb,
                             (kt | kb) ? 1u : 0u);
        }
        sm100::tc_commit(&sh->empty[s]);
        if (kt < 11) DC(17 + kt, clock64() - c0_);
      }
      __syncwarp();
    }
    if (leader) sm100::tc_commit(&sh->accum);
    __syncwarp();
  } else {
    // ---- warps 2-5: hidden quant into the B tile, then the epilogue
    const int t = tid - 64;
    zero_smem128(btile, num_kt * 1024, t);
    zero_smem128(sfb, kb_total * 512, t);
    const uint32_t key = amax_key128(a.hidden, H, t, sh->red);   // (its barriers order the zeroing too)
    if (t == 0) DT(4);
    const float ts = nvfp4_tensor_scale<AEOQ_BF16>(In<AEOQ_BF16>::key_to_f(key));
    for (int64_t b = t; b < H / 16; b += 128) quant_to_btile<false>(a.hidden + 16 * b, ts, b, btile, sfb);
    sm100::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) sm100::mbar_arrive(&sh->bready);
    if (t == 0) DT(1);
    const float alpha = ts * load_scalar_f(a.gu_ts, a.gu_ts_dt);
    const bool ok = sm100::mbar_wait(&sh->accum, 0, a.err, 24);
    if (t == 0) DT(2);
    sm100::tc_fence_after();
    const int q = warp & 3, row = 32 * q + lane;
    float v[16];
    sm100::tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + kAccCol, v);
    const float y = (ok && valid) ? bf16r(v[0] * alpha) : 0.0f;
    if (row >= 64) sh->xchg[row - 64] = y;
    asm volatile("bar.sync 2, 128;" ::: "memory");
    uint32_t hkey = 0;
    if (row < 64) {
      const __nv_bfloat16 hv = __float2bfloat16_rn(bf16r(gelu_tanh(y)) * sh->xchg[row]);
      a.h[(int64_t)j * I + 64 * m + row] = hv;
      hkey = In<AEOQ_BF16>::abs_key(hv);
    }
    hkey = warp_umax(hkey);
    if (lane == 0) sh->red[warp & 3] = hkey;
    asm volatile("bar.sync 2, 128;" ::: "memory");
    if (t == 0) {
      a.parts[(int64_t)j * gridDim.x + m] = max(max(sh->red[0], sh->red[1]), max(sh->red[2], sh->red[3]));
      DT(3);
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 64);
  }
}

// ------------------------------------------------------------------ launch 2
struct Smem2 {
  uint64_t full, bready, accum;
  uint32_t tmem;
  uint32_t red[4];
  int last;
};

__global__ void __launch_bounds__(kThreads, 1) decode_down_tc_kernel(const __grid_constant__ CUtensorMap tmD,
                                                                     const Args a, int n_parts) {
  constexpr int kTraceBase = 4096;
  if (threadIdx.x == 0) DT(0);
  extern __shared__ __align__(1024) uint8_t dsm[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  const int H = (int)a.H, I = (int)a.I;
  const int kb_total = I / 64, num_kt = (I + 255) / 256;
  // swizzled tiles first: both must start on 1024-byte boundaries
  uint8_t* tileA = base;                         // num_kt x 16 KB
  uint8_t* btile = tileA + num_kt * 16384;       // num_kt x 1 KB
  uint8_t* sfa = btile + num_kt * 1024;          // kb_total x 512 B
  uint8_t* sfb = sfa + kb_total * 512;           // kb_total x 512 B
  Smem2* sh = reinterpret_cast<Smem2*>(sfb + kb_total * 512);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m = blockIdx.x, j = blockIdx.y;
  // TMEM: accumulator (8 columns) + all K steps' scale atoms of A and B;
  // sized to the shape so several CTAs of this kernel share an SM.
  const uint32_t acc_col = 0, sfa_col = 8, sfb_col = 8 + 4 * kb_total;
  uint32_t tcols = 32;
  while (tcols < 8u + 8u * kb_total) tcols <<= 1;

  if (tid == 0) {
    sm100::mbar_init(&sh->full, 1);
    sm100::mbar_init(&sh->bready, 4);
    sm100::mbar_init(&sh->accum, 1);
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tmD);
  }
  if (warp == 1) sm100::tmem_alloc(&sh->tmem, tcols);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = sh->tmem;
  // The ids and the down weights do not depend on launch 1: fetch them now.
  const int64_t e = load_index(a.ids, a.ids_dt, j);
  const bool valid = e >= 0 && e < a.E;

  if (warp == 0) {
    if (sm100::elect_one() && valid) {
#ifdef AEOQ_TC_TRACE
      DT(5);
#endif
      sm100::mbar_arrive_expect_tx(&sh->full, (uint32_t)(num_kt * 16384 + kb_total * 512));
      bulk_g2s(sfa, a.dw_atoms + (e * (H / 128) + m) * (int64_t)kb_total * 512, (uint32_t)kb_total * 512,
               &sh->full);
      for (int kt = 0; kt < num_kt; ++kt)
        sm100::tma_load_2d(tileA + kt * 16384, &tmD, kt * 128, (int32_t)(e * H + 128 * m), &sh->full);
    }
    __syncwarp();
  } else if (warp == 1) {
    const bool leader = sm100::elect_one();
    bool ok = valid && sm100::mbar_wait(&sh->full, 0, a.err, 31);
    if (sm100::elect_one()) DT(8);
    ok = ok && sm100::mbar_wait(&sh->bready, 0, a.err, 32);
    if (sm100::elect_one()) DT(6);
    const long long c0_ = clock64();
    sm100::tc_fence_after();
    if (ok && leader) {
      const uint32_t idesc = sm100::idesc_nvf4(kN);
      for (int kb = 0; kb < kb_total; ++kb) {
        sm100::tc_cp_32x128b_warpx4(tmem + sfa_col + 4 * kb, sm100::sdesc_sf_atom(sm100::smem_u32(sfa + kb * 512)));
        sm100::tc_cp_32x128b_warpx4(tmem + sfb_col + 4 * kb, sm100::sdesc_sf_atom(sm100::smem_u32(sfb + kb * 512)));
      }
      for (int kb = 0; kb < kb_total; ++kb) {
        const int kt = kb >> 2, r = kb & 3;
        const uint64_t ad = sm100::sdesc_k_sw128(sm100::smem_u32(tileA + kt * 16384) + r * 32);
        const uint64_t bd = sm100::sdesc_k_sw128(sm100::smem_u32(btile + kt * 1024) + r * 32);
        sm100::tc_mma_nvf4(tmem + acc_col, ad, bd, idesc, tmem + sfa_col + 4 * kb, tmem + sfb_col + 4 * kb,
                           kb ? 1u : 0u);
      }
      DC(9, clock64() - c0_);
    }
    if (leader) sm100::tc_commit(&sh->accum);
    __syncwarp();
  } else {
    const int t = tid - 64;
    zero_smem128(btile, num_kt * 1024, t);
    zero_smem128(sfb, kb_total * 512, t);
    pdl_wait();   // launch 1 complete: h and the maxima are visible
    if (t == 0) DT(1);
    uint32_t key = 0;
    for (int i = t; i < n_parts; i += 128) key = max(key, __ldcg(a.parts + i));
    key = warp_umax(key);
    if (lane == 0) sh->red[t >> 5] = key;
    asm volatile("bar.sync 2, 128;" ::: "memory");
    key = max(max(sh->red[0], sh->red[1]), max(sh->red[2], sh->red[3]));
    if (t == 0) DT(7);
    const float ts = nvfp4_tensor_scale<AEOQ_BF16>(In<AEOQ_BF16>::key_to_f(key));
    for (int64_t b = t; b < I / 16; b += 128)
      quant_to_btile<true>(a.h + (int64_t)j * I + 16 * b, ts, b, btile, sfb);
    sm100::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) sm100::mbar_arrive(&sh->bready);
    const float alpha = ts * load_scalar_f(a.d_ts, a.d_ts_dt);
    const float wj = __bfloat162float(a.topw[j]);
    if (t == 0) DT(2);
    const bool ok = sm100::mbar_wait(&sh->accum, 0, a.err, 33);
    if (t == 0) DT(3);
    sm100::tc_fence_after();
    const int q = warp & 3, row = 32 * q + lane;
    float v[16];
    sm100::tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + acc_col, v);
    const float y = (ok && valid) ? bf16r(bf16r(v[0] * alpha) * wj) : 0.0f;
    a.c[(int64_t)j * H + 128 * m + row] = __float2bfloat16_rn(y);
    __threadfence();
    asm volatile("bar.sync 2, 128;" ::: "memory");
    if (t == 0) {
      sh->last = (atomicAdd(a.counters + m, 1u) == (uint32_t)a.k - 1) ? 1 : 0;
      __threadfence();
    }
    asm volatile("bar.sync 2, 128;" ::: "memory");
    if (sh->last) {
      // the last expert of this row tile: f32 sum over the k slots, one rounding
      float s = 0.f;
      for (int jj = 0; jj < a.k; ++jj) s += __bfloat162float(__ldcg(a.c + (int64_t)jj * H + 128 * m + row));
      a.out[128 * m + row] = __float2bfloat16_rn(s);
      if (t == 0) a.counters[m] = 0;
    }
    if (t == 0) DT(4);
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, tcols);
  }
}

size_t smem1_bytes(int64_t H) {
  return 1024 + kRing * (16384 + 2048) + (size_t)((H + 255) / 256) * 1024 + (size_t)(H / 64) * 512 + sizeof(Smem1);
}
size_t smem2_bytes(int64_t I) {
  return 1024 + (size_t)((I + 255) / 256) * (16384 + 1024) + (size_t)(I / 64) * 1024 + sizeof(Smem2);
}

struct Ws {
  uint32_t* counters;
  uint32_t* parts;
  __nv_bfloat16* h;
  __nv_bfloat16* c;
  size_t bytes;
};

Ws layout(void* base, int64_t k, int64_t H, int64_t I) {
  char* p = reinterpret_cast<char*>(base);
  auto al = [](size_t v) { return (v + 255) / 256 * 256; };
  Ws w{};
  size_t o = 0;
  w.counters = reinterpret_cast<uint32_t*>(p + o); o += al((size_t)(H / 128) * 4);
  w.parts = reinterpret_cast<uint32_t*>(p + o);    o += al((size_t)(k * I / 64) * 4);
  w.h = reinterpret_cast<__nv_bfloat16*>(p + o);   o += al((size_t)(k * I) * 2);
  w.c = reinterpret_cast<__nv_bfloat16*>(p + o);   o += al((size_t)(k * H) * 2);
  w.bytes = o;
  return w;
}

}  // namespace dtc
}  // namespace aeoq

using namespace aeoq;

#ifdef AEOQ_TC_TRACE
extern "C" int aeoq_debug_set_decode_trace(void* p) {
  return cudaMemcpyToSymbol(dtc::g_dtrace, &p, sizeof(p)) == cudaSuccess ? 0 : -2;
}
#endif

extern "C" int aeoq_moe_nvfp4_decode_tc_supported(int64_t top_k, int64_t hidden, int64_t inter) {
  if (top_k < 1 || top_k > 16 || hidden <= 0 || inter <= 0) return 0;
  if (hidden % 128 != 0 || hidden > 64 * dtc::kMaxKB || inter % 64 != 0 || inter > 64 * dtc::kMaxKB2) return 0;
  return (dtc::smem1_bytes(hidden) <= 232448 - 1024 && dtc::smem2_bytes(inter) <= 232448 - 1024) ? 1 : 0;
}

extern "C" size_t aeoq_moe_nvfp4_decode_tc_workspace_size(int64_t top_k, int64_t hidden, int64_t inter) {
  return dtc::layout(nullptr, top_k, hidden, inter).bytes;
}

extern "C" int aeoq_moe_nvfp4_decode_tc(const void* hidden, const void* top_k_index, int idx_dtype,
                                        const void* top_k_weights, int64_t top_k, const uint8_t* gate_up,
                                        const uint8_t* gate_up_atoms, const void* gate_up_ts, int gate_up_ts_dtype,
                                        const uint8_t* down, const uint8_t* down_atoms, const void* down_ts,
                                        int down_ts_dtype, int64_t num_experts, int64_t hidden_dim, int64_t inter_dim,
                                        void* out, void* workspace, size_t workspace_bytes, int* err_word,
                                        void* stream) {
  AEOQ_REQUIRE(aeoq_moe_nvfp4_decode_tc_supported(top_k, hidden_dim, inter_dim), AEOQ_ERR_INVALID,
               "moe_decode_tc: unsupported shape (top_k=%lld hidden=%lld inter=%lld)", (long long)top_k,
               (long long)hidden_dim, (long long)inter_dim);
  AEOQ_REQUIRE(idx_dtype == AEOQ_I32 || idx_dtype == AEOQ_I64, AEOQ_ERR_INVALID, "moe_decode_tc: int32/int64 ids");
  AEOQ_REQUIRE(hidden && top_k_index && top_k_weights && gate_up && gate_up_atoms && gate_up_ts && down &&
                   down_atoms && down_ts && out && err_word,
               AEOQ_ERR_INVALID, "moe_decode_tc: null pointer");
  AEOQ_REQUIRE((uintptr_t)hidden % 16 == 0 && (uintptr_t)gate_up % 16 == 0 && (uintptr_t)down % 16 == 0 &&
                   (uintptr_t)gate_up_atoms % 16 == 0 && (uintptr_t)down_atoms % 16 == 0,
               AEOQ_ERR_INVALID, "moe_decode_tc: operands must be 16-byte aligned");
  const size_t need = aeoq_moe_nvfp4_decode_tc_workspace_size(top_k, hidden_dim, inter_dim);
  AEOQ_REQUIRE(workspace && workspace_bytes >= need && (uintptr_t)workspace % 256 == 0, AEOQ_ERR_WORKSPACE,
               "moe_decode_tc: workspace of %zu bytes (256-aligned, counters zero) needed, %zu given", need,
               workspace_bytes);
  const int64_t E = num_experts, H = hidden_dim, I = inter_dim;
  cudaStream_t st = (cudaStream_t)stream;
  CUtensorMap tg, td;
  int rc = make_tmap(&tg, gate_up, E * 2 * I, H / 2, H / 2, 64);
  if (rc) return rc;
  rc = make_tmap(&td, down, E * H, I / 2, I / 2, 128);
  if (rc) return rc;
  dtc::Ws w = dtc::layout(workspace, top_k, H, I);
  dtc::Args a{};
  a.hidden = reinterpret_cast<const __nv_bfloat16*>(hidden);
  a.ids = top_k_index; a.ids_dt = idx_dtype;
  a.topw = reinterpret_cast<const __nv_bfloat16*>(top_k_weights);
  a.gu_atoms = gate_up_atoms; a.gu_ts = gate_up_ts; a.gu_ts_dt = gate_up_ts_dtype;
  a.dw_atoms = down_atoms; a.d_ts = down_ts; a.d_ts_dt = down_ts_dtype;
  a.E = E; a.H = H; a.I = I; a.k = (int)top_k;
  a.h = w.h; a.parts = w.parts; a.c = w.c; a.counters = w.counters;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.err = err_word;
  const size_t s1 = dtc::smem1_bytes(H), s2 = dtc::smem2_bytes(I);
  static size_t set1 = 0, set2 = 0;
  if (set1 < s1) {
    if (cudaFuncSetAttribute(dtc::decode_gateup_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s1) !=
        cudaSuccess) {
      cudaGetLastError();
      return set_error(AEOQ_ERR_CUDA, "moe_decode_tc: shared memory attribute (launch 1)");
    }
    set1 = s1;
  }
  if (set2 < s2) {
    if (cudaFuncSetAttribute(dtc::decode_down_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s2) !=
        cudaSuccess) {
      cudaGetLastError();
      return set_error(AEOQ_ERR_CUDA, "moe_decode_tc: shared memory attribute (launch 2)");
    }
    set2 = s2;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t c1 = {};
  c1.gridDim = dim3((unsigned)(I / 64), (unsigned)top_k);
  c1.blockDim = dim3(dtc::kThreads);
  c1.dynamicSmemBytes = s1;
  c1.stream = st;
  c1.attrs = attr;
  c1.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&c1, dtc::decode_gateup_tc_kernel, tg, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(AEOQ_ERR_CUDA, "decode_gateup_tc_kernel: %s", cudaGetErrorString(e));
  }
  cudaLaunchConfig_t c2 = c1;
  c2.gridDim = dim3((unsigned)(H / 128), (unsigned)top_k);
  c2.dynamicSmemBytes = s2;
  e = cudaLaunchKernelEx(&c2, dtc::decode_down_tc_kernel, td, a, (int)(top_k * I / 64));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(AEOQ_ERR_CUDA, "decode_down_tc_kernel: %s", cudaGetErrorString(e));
  }
  return check_launch("decode_down_tc_kernel");
}
