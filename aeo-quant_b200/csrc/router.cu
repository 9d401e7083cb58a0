// Gemma-4 router for a few tokens in one launch: RMS norm, scale, the
// hidden -> experts projection, softmax, top-k, renormalisation and the
// per-expert scale. Replaces HF transformers' Gemma4TextRouter.forward
// (transformers 5.5.0, models/gemma4/modeling_gemma4.py:1296-1316) with
// Gemma4RMSNorm (:166-175, with_scale=False), whose eager form is about ten
// launches per call.
//
// Rounding points follow the eager ops:
//   r   = rsqrt(sum(x^2)/H + eps)                 f32 (torch pow(., -0.5) on
//                                                 CUDA is rsqrt)
//   n   = bf16(x * r)                             (type_as, :175)
//   y   = bf16(bf16(n * scale) * f32(H^-0.5))     (:1300, bf16 tensor ops)
//   l_e = bf16(sum_h y[h] * W[e][h])              (nn.Linear, f32 accumulate)
//   p_e = bf16(exp(l_e - max) / sum)              (softmax, f32 inside)
//   top-k of p (descending; equal values: lower expert id first)
//   w_j = bf16(bf16(p_j / bf16(sum_j p_j)) * per_expert_scale[i_j])
// The reduction orders of the sums differ from cuBLAS / ATen, so logits can
// differ from the eager ones in the last bf16 place.
//
// Layout: one 8-CTA cluster per tile of 16 tokens (1 for a single token).
// Every CTA copies the tile's token rows into shared memory with cp.async,
// all pieces in flight at once. CTA rank r computes the logits of experts
// [r*E/8, (r+1)*E/8) for the tile's tokens: a warp takes two expert rows at
// a time, reads them once with 16-byte loads (twelve per row and lane in
// flight for one token, the first of them issued before the copy) and dots
// them with every token's normalised row in shared memory; the 0.7 MB
// projection is read once per tile and stays in L2. Warp w of every CTA
// normalises tokens w, w + 8 of the tile. Token q is finished by warp q / 8
// of rank q % 8, which gathers its E logits through distributed shared
// memory; top-k is k rounds of a warp argmax.
#include "common.cuh"
#include "sm100.cuh"

namespace aeoq {
namespace {

constexpr int kRouterCluster = 8;
constexpr int kRouterThreads = 256;
constexpr int kRouterMaxE = 256;
constexpr int kRouterMaxK = 32;
constexpr int kTok = 16;   // tokens per cluster tile (one for a single token)

struct RouterArgs {
  const __nv_bfloat16* x;
  int64_t ldx;
  const __nv_bfloat16* scale;   // (H,)
  const __nv_bfloat16* w;       // (E, H) row-major
  const __nv_bfloat16* pes;     // (E,) per-expert scale
  int H, E, k;
  float eps, root;
  __nv_bfloat16* probs;         // (T, E)
  __nv_bfloat16* topw;          // (T, k)
  int64_t* topi;                // (T, k)
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sm100::smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// NT tokens per cluster; U 16-byte loads per expert row and lane in flight
// (U = 12 covers H <= 3072 in one round trip).
template <int NT, int U>
__global__ void __launch_bounds__(kRouterThreads) gemma4_router_kernel(const RouterArgs a, int64_t T) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int kRows = kRouterMaxE / kRouterCluster;
  __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(smem);                   // NT x H
  __nv_bfloat16* scs = y + (size_t)NT * a.H;                                   // H
  float* logit = reinterpret_cast<float*>(smem + (size_t)2 * (NT + 1) * a.H);  // NT x kRows
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = sm100::cluster_ctarank();
  const int H = a.H, E = a.E, rows = E / kRouterCluster, h8 = H / 8;
  const int64_t t0 = (int64_t)blockIdx.y * NT;
  const int nt = T - t0 < NT ? (int)(T - t0) : NT;
  const uint4* wbase = reinterpret_cast<const uint4*>(a.w + (int64_t)rank * rows * H);

  // The first chunk of this warp's two expert rows is in flight while the
  // tokens are normalised.
  uint4 wa[U], wb[U];
  {
    const int ea = 2 * warp, eb = ea + 1;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = lane + 32 * u;
      wa[u] = ea < rows && i < h8 ? __ldg(wbase + (int64_t)ea * h8 + i) : make_uint4(0u, 0u, 0u, 0u);
      wb[u] = eb < rows && i < h8 ? __ldg(wbase + (int64_t)eb * h8 + i) : make_uint4(0u, 0u, 0u, 0u);
    }
  }
  // 0. the tile's token rows and the norm scale into shared memory, every
  //    16-byte piece in flight at once (cp.async); rows past T are zero
  for (int i = tid; i < h8; i += kRouterThreads) cp_async16(reinterpret_cast<uint4*>(scs) + i,
                                                           reinterpret_cast<const uint4*>(a.scale) + i);
  for (int j = tid; j < NT * h8; j += kRouterThreads) {
    const int q = j / h8, i = j - q * h8;
    uint4* dst = reinterpret_cast<uint4*>(y + (size_t)q * H) + i;
    if (q < nt)
      cp_async16(dst, reinterpret_cast<const uint4*>(a.x + (t0 + q) * a.ldx) + i);
    else
      *dst = make_uint4(0u, 0u, 0u, 0u);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  // 1. warp w: tokens t0 + w, t0 + w + 8, ... r = rsqrt(mean(x^2) + eps);
  //    y = bf16(bf16(bf16(x * r) * scale) * root), in place
  for (int q = warp; q < nt; q += kRouterThreads / 32) {
    uint4* yw = reinterpret_cast<uint4*>(y + (size_t)q * H);
    const uint4* s8 = reinterpret_cast<const uint4*>(scs);
    float ss = 0.0f;
    for (int i = lane; i < h8; i += 32) {
      float f[8];
      unpack8(yw[i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
    }
    const float r = rsqrtf(warp_sum(ss) / (float)H + a.eps);
    for (int i = lane; i < h8; i += 32) {
      float f[8], sc[8];
      unpack8(yw[i], f);
      unpack8(s8[i], sc);
      __align__(16) __nv_bfloat16 o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = __float2bfloat16_rn(bf16r(bf16r(f[j] * r) * sc[j]) * a.root);
      yw[i] = *reinterpret_cast<const uint4*>(o);
    }
  }
  __syncthreads();
  // 2. this CTA's logits: each warp two expert rows per pass, every token
  //    of the tile, U 16-byte loads per row in flight
  for (int base = 0; base < rows; base += 2 * (kRouterThreads / 32)) {
    const int ea = base + 2 * warp, eb = ea + 1;
    float acca[NT], accb[NT];
#pragma unroll
    for (int q = 0; q < NT; ++q) acca[q] = accb[q] = 0.0f;
    for (int i0 = 0; i0 < h8; i0 += 32 * U) {
      if (base != 0 || i0 != 0) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = i0 + lane + 32 * u;
          wa[u] = ea < rows && i < h8 ? __ldg(wbase + (int64_t)ea * h8 + i) : make_uint4(0u, 0u, 0u, 0u);
          wb[u] = eb < rows && i < h8 ? __ldg(wbase + (int64_t)eb * h8 + i) : make_uint4(0u, 0u, 0u, 0u);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + lane + 32 * u;
        if (i < h8) {
          float fa[8], fb[8];
          unpack8(wa[u], fa);
          unpack8(wb[u], fb);
#pragma unroll
          for (int q = 0; q < NT; ++q) {
            float yf[8];
            unpack8(reinterpret_cast<const uint4*>(y + (size_t)q * H)[i], yf);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              acca[q] = fmaf(fa[j], yf[j], acca[q]);
              accb[q] = fmaf(fb[j], yf[j], accb[q]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < NT; ++q) {
      const float va = warp_sum(acca[q]);
      const float vb = warp_sum(accb[q]);
      if (lane == 0 && ea < rows) logit[q * kRows + ea] = bf16r(va);
      if (lane == 0 && eb < rows) logit[q * kRows + eb] = bf16r(vb);
    }
  }
  sm100::cluster_sync();
  // 3. token q is finished by warp q / 8 of cluster rank q % 8: softmax,
  //    top-k, renormalisation, per-expert scale. Top-k is k rounds of a
  //    warp argmax over 64-bit keys (probability bits above the inverted
  //    expert id): probabilities are >= +0, so the key order is descending
  //    probability, equal values by lower expert id.
  for (int q = (int)rank + kRouterCluster * warp; q < nt; q += kRouterCluster * (kRouterThreads / 32)) {
    const int64_t t = t0 + q;
    constexpr int kPer = kRouterMaxE / 32;
    float l[kPer], p[kPer];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = lane + 32 * i;
      l[i] = e < E ? sm100::ld_dsmem_f32(sm100::dsmem_addr(logit + q * kRows + e % rows, (uint32_t)(e / rows)))
                   : -INFINITY;
      mx = fmaxf(mx, l[i]);
    }
    mx = warp_max(mx);
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      p[i] = lane + 32 * i < E ? expf(l[i] - mx) : 0.0f;
      sum += p[i];
    }
    sum = warp_sum(sum);
    unsigned long long key[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = lane + 32 * i;
      p[i] = bf16r(p[i] / sum);
      key[i] = 0ull;
      if (e < E) {
        a.probs[t * E + e] = __float2bfloat16_rn(p[i]);
        key[i] = ((unsigned long long)__float_as_uint(p[i]) << 32) | (0xFFFFFFFFu - (uint32_t)e);
      }
    }
    float tot = 0.0f, myval = 0.0f;
    int myidx = 0;
    for (int j = 0; j < a.k; ++j) {
      unsigned long long m = key[0];
#pragma unroll
      for (int i = 1; i < kPer; ++i) m = key[i] > m ? key[i] : m;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long v = __shfl_xor_sync(0xFFFFFFFFu, m, o);
        m = v > m ? v : m;
      }
      const int e = (int)(0xFFFFFFFFu - (uint32_t)m);
      const float v = __uint_as_float((uint32_t)(m >> 32));
#pragma unroll
      for (int i = 0; i < kPer; ++i)
        if (key[i] == m) key[i] = 0ull;
      tot += v;
      if (lane == j) {
        myidx = e;
        myval = v;
      }
    }
    const float den = bf16r(tot);
    if (lane < a.k) {
      const float wj = bf16r(myval / den);
      a.topw[t * a.k + lane] = __float2bfloat16_rn(wj * __bfloat162float(a.pes[myidx]));
      a.topi[t * a.k + lane] = myidx;
    }
  }
  sm100::cluster_sync();   // every CTA's logits have been read
}

}  // namespace
}  // namespace aeoq

using namespace aeoq;

extern "C" int aeoq_gemma4_router(const void* x, int64_t ldx, const void* scale, const void* proj_w,
                                  const void* per_expert_scale, int64_t T, int64_t H, int64_t E, int64_t top_k,
                                  float eps, float root_scale, void* probs, void* top_w, int64_t* top_i,
                                  void* stream) {
  AEOQ_REQUIRE(T >= 0 && H > 0 && E > 0 && top_k > 0, AEOQ_ERR_INVALID, "gemma4_router: bad shape");
  AEOQ_REQUIRE(H % 8 == 0 && ldx % 8 == 0 && ldx >= H, AEOQ_ERR_INVALID,
               "gemma4_router: hidden size and row stride must be multiples of 8");
  AEOQ_REQUIRE(H <= 6144, AEOQ_ERR_INVALID, "gemma4_router: hidden size above 6144");
  AEOQ_REQUIRE(H >= 2 * E + 128, AEOQ_ERR_INVALID, "gemma4_router: hidden size below 2 * num_experts + 128");
  AEOQ_REQUIRE(E % kRouterCluster == 0 && E <= kRouterMaxE, AEOQ_ERR_INVALID,
               "gemma4_router: num_experts must be a multiple of 8 and at most 256");
  AEOQ_REQUIRE(top_k <= E && top_k <= kRouterMaxK, AEOQ_ERR_INVALID, "gemma4_router: top_k above min(E, 32)");
  AEOQ_REQUIRE(T <= 65535LL * kTok, AEOQ_ERR_INVALID, "gemma4_router: too many tokens");
  if (T == 0) return AEOQ_OK;
  AEOQ_REQUIRE(x && scale && proj_w && per_expert_scale && probs && top_w && top_i, AEOQ_ERR_INVALID,
               "gemma4_router: null pointer");
  AEOQ_REQUIRE((uintptr_t)x % 16 == 0 && (uintptr_t)scale % 16 == 0 && (uintptr_t)proj_w % 16 == 0,
               AEOQ_ERR_INVALID, "gemma4_router: x, scale and proj_w must be 16-byte aligned");
  RouterArgs a;
  a.x = (const __nv_bfloat16*)x;
  a.ldx = ldx;
  a.scale = (const __nv_bfloat16*)scale;
  a.w = (const __nv_bfloat16*)proj_w;
  a.pes = (const __nv_bfloat16*)per_expert_scale;
  a.H = (int)H;
  a.E = (int)E;
  a.k = (int)top_k;
  a.eps = eps;
  a.root = root_scale;
  a.probs = (__nv_bfloat16*)probs;
  a.topw = (__nv_bfloat16*)top_w;
  a.topi = top_i;
  const int nt = T == 1 ? 1 : kTok;
  auto kern = nt == 1 ? gemma4_router_kernel<1, 12> : gemma4_router_kernel<kTok, 4>;
  const size_t smem = (size_t)2 * (nt + 1) * H + sizeof(float) * nt * (kRouterMaxE / kRouterCluster);
  if (smem > 48 * 1024) {
    const int rc = func_smem_attr((const void*)kern, smem, -1, "gemma4_router_kernel");
    if (rc) return rc;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kRouterCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t c = {};
  c.gridDim = dim3(kRouterCluster, (unsigned)((T + nt - 1) / nt));
  c.blockDim = dim3(kRouterThreads);
  c.dynamicSmemBytes = smem;
  c.stream = (cudaStream_t)stream;
  c.attrs = attr;
  c.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&c, kern, a, T);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(AEOQ_ERR_CUDA, "gemma4_router_kernel: %s", cudaGetErrorString(e));
  }
  return check_launch("gemma4_router_kernel");
}
