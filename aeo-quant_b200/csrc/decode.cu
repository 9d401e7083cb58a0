// Fused one-token NVFP4 MoE expert forward (two launches).
//
// Restates Gemma4TextExpertsNVFP4._forward_decode_3d (aeo_quant
// src/aeo_quant/bridges/gemma4/modeling_nvfp4.py:132-186) as a stream over
// the k selected experts' packed weights, which is the whole cost at one
// token: k * (2I*H + H*I) / 2 bytes of FP4 plus 1/8 of that in scales.
//
//   launch 1 (gate_up):  persistent CTAs, one warp per (slot, n) row pair
//     gate row n and up row n+I of expert ids[slot]. Every CTA quantizes the
//     hidden vector itself (global amax, tensor scale, block scales: the same
//     bits as quantize_2d_to_nvfp4, :150-153), keeps its lanes' activation
//     chunks in registers, streams the rows with 16-byte coalesced loads
//     (one row pair in flight ahead of the math), reduces by warp shuffles,
//     and writes h = bf16(bf16(gelu(bf16(a*g))) * bf16(a*u)) (:155-162) plus
//     one amax key per CTA into the workspace.
//   launch 2 (down + combine): CTA per R output rows, one warp per slot.
//     Launched with programmatic dependent launch, so it streams its weight
//     rows while launch 1 drains; after griddepcontrol.wait it reduces the
//     amax keys to the shared tensor scale of (:164-172), quantizes its
//     chunk of h, finishes the GEMV, and combines the k slots as
//     bf16(sum_j bf16(bf16(a*d_j) * w_j)) (:174-186).
#include <cstdlib>

#include "common.cuh"

namespace aeoq {

constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDownRows = 8;     // output rows per CTA in launch 3
constexpr int kMaxTopK = 16;
constexpr int kMaxHidden = 4096;
constexpr int kQuantThreadsH = 512;

template <int CPL>
struct RowPair {
  uint4 g[CPL], u[CPL];
  uint16_t gs[CPL], us[CPL];
};

template <int CPL>
__device__ __forceinline__ void load_row_pair(RowPair<CPL>& b, const uint8_t* gu, const uint8_t* gu_sf,
                                              int64_t e, bool valid, int64_t n, int64_t I, int64_t H,
                                              int lane) {
  const int64_t rb = H / 2, sb = H / 16, nchunk = H / 32;
  const uint8_t* rg = gu + (e * 2 * I + n) * rb;
  const uint8_t* ru = rg + I * rb;
  const uint8_t* sg = gu_sf + (e * 2 * I + n) * sb;
  const uint8_t* su = sg + I * sb;
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int64_t c = lane + 32 * j;
    if (valid && c < nchunk) {
      b.g[j] = ldg_stream(rg + 16 * c);
      b.u[j] = ldg_stream(ru + 16 * c);
      b.gs[j] = *reinterpret_cast<const uint16_t*>(sg + 2 * c);
      b.us[j] = *reinterpret_cast<const uint16_t*>(su + 2 * c);
    } else {
      b.g[j] = b.u[j] = make_uint4(0, 0, 0, 0);
      b.gs[j] = b.us[j] = 0;
    }
  }
}

template <int CPL>
__global__ void __launch_bounds__(kDecThreads, 2) moe_decode_gateup_kernel(
    const __nv_bfloat16* __restrict__ hidden, const void* __restrict__ ids, int ids_dt, int k,
    const uint8_t* __restrict__ gu, const uint8_t* __restrict__ gu_sf, const void* gu_ts, int gu_ts_dt,
    int64_t E, int64_t H, int64_t I, __nv_bfloat16* __restrict__ h_out, uint32_t* __restrict__ parts) {
  __shared__ uint32_t red[32];
  __shared__ __align__(16) __half2 act_s[kMaxHidden / 16 * 8];
  __shared__ float sa_s[kMaxHidden / 16];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t total = (int64_t)k * I;
  const int64_t per = (total + gridDim.x - 1) / gridDim.x;
  const int64_t p_begin = blockIdx.x * per;
  const int64_t p_end = min(total, p_begin + per);
  const int64_t nchunk = H / 32;

  // Issue the first row pair's loads before the activation prologue.
  int64_t p = p_begin + warp;
  RowPair<CPL> cur;
  int64_t cur_e = 0;
  bool cur_valid = false;
  if (p < p_end) {
    const int64_t slot = p / I;
    cur_e = load_index(ids, ids_dt, slot);
    cur_valid = cur_e >= 0 && cur_e < E;
    load_row_pair<CPL>(cur, gu, gu_sf, cur_e, cur_valid, p - slot * I, I, H, lane);
  }

  // Activation quant, once per CTA: global amax -> bf16 tensor scale ->
  // one 16-element block per thread, decoded to exact halves in shared memory.
  uint32_t key = 0;
  for (int64_t i = threadIdx.x; i < H / 8; i += blockDim.x) {
    const uint4 u = *reinterpret_cast<const uint4*>(hidden + 8 * i);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) key = max(key, In<AEOQ_BF16>::abs_key(e[j]));
  }
  key = warp_umax(key);
  if (lane == 0) red[warp] = key;
  __syncthreads();
  key = 0;
#pragma unroll
  for (int w = 0; w < kDecWarps; ++w) key = max(key, red[w]);
  const float ts = nvfp4_tensor_scale<AEOQ_BF16>(In<AEOQ_BF16>::key_to_f(key));
  const float alpha = ts * load_scalar_f(gu_ts, gu_ts_dt);
  for (int64_t b = threadIdx.x; b < H / 16; b += blockDim.x) {
    float v[16];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const uint4 u = *reinterpret_cast<const uint4*>(hidden + 16 * b + 8 * q);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[8 * q + j] = __bfloat162float(e[j]);
    }
    uint32_t w0, w1;
    const uint32_t sf = nvfp4_quant_block(v, ts, w0, w1);
    __half2 t[4];
    fp4x8_to_half2x4_exact(w0, t);
#pragma unroll
    for (int i = 0; i < 4; ++i) act_s[8 * b + i] = t[i];
    fp4x8_to_half2x4_exact(w1, t);
#pragma unroll
    for (int i = 0; i < 4; ++i) act_s[8 * b + 4 + i] = t[i];
    sa_s[b] = e4m3_decode(sf) * 16384.0f;
  }
  __syncthreads();
  __half2 act[CPL][16];
  float sa[CPL][2];
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int64_t c = lane + 32 * j;
    if (c < nchunk) {
#pragma unroll
      for (int i = 0; i < 16; ++i) act[j][i] = act_s[16 * c + i];
      sa[j][0] = sa_s[2 * c];
      sa[j][1] = sa_s[2 * c + 1];
    }
  }
  pdl_trigger();

  uint32_t hkey = 0;
  while (p < p_end) {
    const int64_t pn = p + kDecWarps;
    RowPair<CPL> nxt;
    int64_t nxt_e = 0;
    bool nxt_valid = false;
    if (pn < p_end) {
      const int64_t slot = pn / I;
      nxt_e = load_index(ids, ids_dt, slot);
      nxt_valid = nxt_e >= 0 && nxt_e < E;
      load_row_pair<CPL>(nxt, gu, gu_sf, nxt_e, nxt_valid, pn - slot * I, I, H, lane);
    }
    float ag = 0.0f, au = 0.0f;
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      if (lane + 32 * j < nchunk) {
        ag = chunk_dot(act[j], sa[j], cur.g[j], cur.gs[j], ag);
        au = chunk_dot(act[j], sa[j], cur.u[j], cur.us[j], au);
      }
    }
    ag = warp_sum(ag);
    au = warp_sum(au);
    if (lane == 0) {
      const float g = bf16r(ag * alpha), u = bf16r(au * alpha);
      const __nv_bfloat16 hv = __float2bfloat16_rn(bf16r(gelu_tanh(g)) * u);
      h_out[p] = hv;  // p == slot * I + n
      hkey = max(hkey, In<AEOQ_BF16>::abs_key(hv));
    }
    cur = nxt;
    p = pn;
  }
  __syncthreads();
  if (lane == 0) red[warp] = hkey;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t m = 0;
    for (int w = 0; w < kDecWarps; ++w) m = max(m, red[w]);
    parts[blockIdx.x] = m;
  }
}

// Launch 2: the shared-scale re-quant of the k x I GeGLU output
// (modeling_nvfp4.py:164-172). One CTA: reduce the per-CTA amax keys of
// launch 1, then one 16-element block per thread into the workspace.
__global__ void __launch_bounds__(kQuantThreadsH) moe_decode_hquant_kernel(
    const __nv_bfloat16* h, const uint32_t* parts, int nparts, int64_t n,
    uint8_t* __restrict__ hq, uint8_t* __restrict__ hsf, float* __restrict__ hts) {
  __shared__ uint32_t red[kQuantThreadsH / 32];
  pdl_trigger();
  pdl_wait();
  // Data written by the preceding grid is read with L2-coherent loads
  // (ld.global.cg): this grid may have started before those writes.
  uint32_t key = 0;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) key = max(key, __ldcg(parts + i));
  key = warp_umax(key);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = key;
  __syncthreads();
  key = 0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) key = max(key, red[w]);
  const float ts = nvfp4_tensor_scale<AEOQ_BF16>(In<AEOQ_BF16>::key_to_f(key));
  if (threadIdx.x == 0) *hts = ts;
  for (int64_t b = threadIdx.x; b < n / 16; b += blockDim.x) {
    float v[16];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const uint4 u = __ldcg(reinterpret_cast<const uint4*>(h + 16 * b + 8 * q));
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[8 * q + j] = __bfloat162float(e[j]);
    }
    uint32_t w0, w1;
    hsf[b] = (uint8_t)nvfp4_quant_block(v, ts, w0, w1);
    *reinterpret_cast<uint2*>(hq + 8 * b) = make_uint2(w0, w1);
  }
}

// Launch 3: down GEMV + weighted combine. CTA per kDownRows output rows,
// warp per slot; weight rows are prefetched before the dependency wait.
template <int CPL2>
__global__ void __launch_bounds__(kDecThreads, 2) moe_decode_down_kernel(
    const uint8_t* hq, const uint8_t* hsf, const float* hts,
    const void* __restrict__ ids, int ids_dt, const __nv_bfloat16* __restrict__ topw, int k,
    const uint8_t* __restrict__ dw, const uint8_t* __restrict__ dw_sf, const void* d_ts, int d_ts_dt,
    int64_t E, int64_t H, int64_t I, __nv_bfloat16* __restrict__ out) {
  __shared__ float prod[kMaxTopK][kDownRows];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t n0 = blockIdx.x * (int64_t)kDownRows;
  const int rows = (int)min((int64_t)kDownRows, H - n0);
  const int64_t rb = I / 2, sb = I / 16, nchunk = I / 32;
  bool waited = false;

  for (int j = warp; j < k; j += kDecWarps) {
    const int64_t e = load_index(ids, ids_dt, j);
    const bool valid = e >= 0 && e < E;
    uint4 wv[kDownRows][CPL2];
    uint16_t ws[kDownRows][CPL2];
#pragma unroll
    for (int r = 0; r < kDownRows; ++r) {
#pragma unroll
      for (int q = 0; q < CPL2; ++q) {
        const int64_t c = lane + 32 * q;
        if (valid && r < rows && c < nchunk) {
          const int64_t row = e * H + n0 + r;
          wv[r][q] = ldg_stream(dw + row * rb + 16 * c);
          ws[r][q] = *reinterpret_cast<const uint16_t*>(dw_sf + row * sb + 2 * c);
        } else {
          wv[r][q] = make_uint4(0, 0, 0, 0);
          ws[r][q] = 0;
        }
      }
    }
    if (!waited) {
      pdl_wait();
      waited = true;
    }
    const float alpha = __ldcg(hts) * load_scalar_f(d_ts, d_ts_dt);
    const float wj = __bfloat162float(topw[j]);
    __half2 act[CPL2][16];
    float sa[CPL2][2];
#pragma unroll
    for (int q = 0; q < CPL2; ++q) {
      const int64_t c = lane + 32 * q;
      if (c < nchunk)
        decode_act_chunk(__ldcg(reinterpret_cast<const uint4*>(hq + j * rb + 16 * c)),
                         __ldcg(reinterpret_cast<const unsigned short*>(hsf + j * sb + 2 * c)), act[q], sa[q]);
    }
#pragma unroll
    for (int r = 0; r < kDownRows; ++r) {
      float acc = 0.0f;
#pragma unroll
      for (int q = 0; q < CPL2; ++q)
        if (lane + 32 * q < nchunk) acc = chunk_dot(act[q], sa[q], wv[r][q], ws[r][q], acc);
      acc = warp_sum(acc);
      if (lane == 0 && r < rows) prod[j][r] = bf16r(bf16r(acc * alpha) * wj);
    }
  }
  if (!waited) pdl_wait();
  __syncthreads();
  if (threadIdx.x < rows) {
    float s = 0.0f;
    for (int j = 0; j < k; ++j) s += prod[j][threadIdx.x];
    out[n0 + threadIdx.x] = __float2bfloat16_rn(s);
  }
}

static int num_sms() { return device_sm_count(); }

static int gateup_grid(int64_t k, int64_t I) {
  const int64_t pairs = k * I;
  const int64_t want = (pairs + kDecWarps - 1) / kDecWarps;
  const int64_t cap = 2 * (int64_t)num_sms();
  return (int)(want < cap ? want : cap);
}

struct DecodeWs {
  __nv_bfloat16* h;
  uint32_t* parts;
  uint8_t* hq;
  uint8_t* hsf;
  float* hts;
  size_t bytes;
};

static size_t align256(size_t v) { return (v + 255) / 256 * 256; }

static DecodeWs decode_ws(void* base, int64_t k, int64_t I) {
  char* p = reinterpret_cast<char*>(base);
  DecodeWs w{};
  size_t off = 0;
  w.h = reinterpret_cast<__nv_bfloat16*>(p + off); off += align256((size_t)(k * I) * 2);
  w.parts = reinterpret_cast<uint32_t*>(p + off); off += align256((size_t)gateup_grid(k, I) * 4);
  w.hq = reinterpret_cast<uint8_t*>(p + off); off += align256((size_t)(k * I) / 2);
  w.hsf = reinterpret_cast<uint8_t*>(p + off); off += align256((size_t)(k * I) / 16);
  w.hts = reinterpret_cast<float*>(p + off); off += 256;
  w.bytes = off;
  return w;
}

}  // namespace aeoq

using namespace aeoq;

extern "C" size_t aeoq_moe_nvfp4_decode_workspace_size(int64_t top_k, int64_t hidden, int64_t inter) {
  (void)hidden;
  return decode_ws(nullptr, top_k, inter).bytes;
}

template <typename... KArgs, typename... Args>
static int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, const char* name,
                      Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(AEOQ_ERR_CUDA, "%s: %s", name, cudaGetErrorString(e));
  }
  return check_launch(name);
}

// stages: bit 0 = gate_up launch, bit 1 = re-quant + down launches
template <int CPL, int CPL2>
static int launch_decode(int stages, const void* hidden, const void* ids, int ids_dt, const void* topw, int k,
                         const uint8_t* gu, const uint8_t* gu_sf, const void* gu_ts, int gu_ts_dt,
                         const uint8_t* dw, const uint8_t* dw_sf, const void* d_ts, int d_ts_dt,
                         int64_t E, int64_t H, int64_t I, void* out, void* wsp, cudaStream_t st) {
  const int g1 = gateup_grid(k, I);
  DecodeWs ws = decode_ws(wsp, k, I);
  if (stages & 1) {
    moe_decode_gateup_kernel<CPL><<<g1, kDecThreads, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(hidden), ids, ids_dt, k, gu, gu_sf, gu_ts, gu_ts_dt, E, H, I,
        ws.h, ws.parts);
    int rc = check_launch("moe_decode_gateup_kernel");
    if (rc) return rc;
  }
  if (!(stages & 2)) return AEOQ_OK;
  int rc = launch_pdl(moe_decode_hquant_kernel, dim3(1), dim3(kQuantThreadsH), st, "moe_decode_hquant_kernel",
                      (const __nv_bfloat16*)ws.h, (const uint32_t*)ws.parts, g1, (int64_t)(k * I), ws.hq, ws.hsf,
                      ws.hts);
  if (rc) return rc;
  return launch_pdl(moe_decode_down_kernel<CPL2>, dim3((unsigned)((H + kDownRows - 1) / kDownRows)),
                    dim3(kDecThreads), st, "moe_decode_down_kernel", (const uint8_t*)ws.hq,
                    (const uint8_t*)ws.hsf, (const float*)ws.hts, ids, ids_dt,
                    reinterpret_cast<const __nv_bfloat16*>(topw), k, dw, dw_sf, d_ts, d_ts_dt, E, H, I,
                    reinterpret_cast<__nv_bfloat16*>(out));
}

static int decode_entry(int stages, const void* hidden, const void* top_k_index, int idx_dtype,
                                     const void* top_k_weights, int64_t top_k, const uint8_t* gate_up,
                                     const uint8_t* gate_up_sf, const void* gate_up_ts, int gate_up_ts_dtype,
                                     const uint8_t* down, const uint8_t* down_sf, const void* down_ts,
                                     int down_ts_dtype, int64_t num_experts, int64_t hidden_dim,
                                     int64_t inter_dim, void* out, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  AEOQ_REQUIRE(top_k >= 1 && top_k <= kMaxTopK, AEOQ_ERR_INVALID, "moe_decode: top_k must be in [1, %d]",
               kMaxTopK);
  AEOQ_REQUIRE(hidden_dim % 64 == 0 && inter_dim % 64 == 0 && hidden_dim > 0 && inter_dim > 0,
               AEOQ_ERR_INVALID, "moe_decode: hidden and intermediate sizes must be multiples of 64");
  AEOQ_REQUIRE(hidden_dim <= 4096 && inter_dim <= 2048, AEOQ_ERR_INVALID,
               "moe_decode: hidden <= 4096 and intermediate <= 2048 supported");
  AEOQ_REQUIRE(idx_dtype == AEOQ_I32 || idx_dtype == AEOQ_I64, AEOQ_ERR_INVALID,
               "moe_decode: top_k_index must be int32 or int64");
  AEOQ_REQUIRE(hidden && top_k_index && top_k_weights && gate_up && gate_up_sf && gate_up_ts && down &&
                   down_sf && down_ts && out,
               AEOQ_ERR_INVALID, "moe_decode: null pointer");
  AEOQ_REQUIRE(((uintptr_t)hidden % 16 == 0) && ((uintptr_t)gate_up % 16 == 0) && ((uintptr_t)down % 16 == 0) &&
                   ((uintptr_t)gate_up_sf % 2 == 0) && ((uintptr_t)down_sf % 2 == 0),
               AEOQ_ERR_INVALID, "moe_decode: hidden/weights must be 16-byte aligned, scales 2-byte aligned");
  const size_t need = aeoq_moe_nvfp4_decode_workspace_size(top_k, hidden_dim, inter_dim);
  AEOQ_REQUIRE(workspace && workspace_bytes >= need && (uintptr_t)workspace % 256 == 0, AEOQ_ERR_WORKSPACE,
               "moe_decode: workspace of %zu bytes (256-aligned) needed, %zu given", need, workspace_bytes);
  cudaStream_t st = (cudaStream_t)stream;
  const int cpl = (int)((hidden_dim / 32 + 31) / 32);
  const int cpl2 = (int)((inter_dim / 32 + 31) / 32);
#define AEOQ_DEC(A, B)                                                                                    \
  if (cpl == A && cpl2 == B)                                                                              \
  return launch_decode<A, B>(stages, hidden, top_k_index, idx_dtype, top_k_weights, (int)top_k, gate_up, gate_up_sf, \
                             gate_up_ts, gate_up_ts_dtype, down, down_sf, down_ts, down_ts_dtype, num_experts,  \
                             hidden_dim, inter_dim, out, workspace, st)
  AEOQ_DEC(1, 1); AEOQ_DEC(2, 1); AEOQ_DEC(3, 1); AEOQ_DEC(4, 1);
  AEOQ_DEC(1, 2); AEOQ_DEC(2, 2); AEOQ_DEC(3, 2); AEOQ_DEC(4, 2);
#undef AEOQ_DEC
  return set_error(AEOQ_ERR_INVALID, "moe_decode: unsupported shape");
}

#define AEOQ_DECODE_ARGS                                                                                     \
  const void *hidden, const void *top_k_index, int idx_dtype, const void *top_k_weights, int64_t top_k,    \
      const uint8_t *gate_up, const uint8_t *gate_up_sf, const void *gate_up_ts, int gate_up_ts_dtype,     \
      const uint8_t *down, const uint8_t *down_sf, const void *down_ts, int down_ts_dtype,                 \
      int64_t num_experts, int64_t hidden_dim, int64_t inter_dim, void *out, void *workspace,              \
      size_t workspace_bytes, void *stream
#define AEOQ_DECODE_PASS                                                                                    \
  hidden, top_k_index, idx_dtype, top_k_weights, top_k, gate_up, gate_up_sf, gate_up_ts, gate_up_ts_dtype, \
      down, down_sf, down_ts, down_ts_dtype, num_experts, hidden_dim, inter_dim, out, workspace,           \
      workspace_bytes, stream

extern "C" int aeoq_moe_nvfp4_decode(AEOQ_DECODE_ARGS) { return decode_entry(3, AEOQ_DECODE_PASS); }
extern "C" int aeoq_moe_nvfp4_decode_gate_up(AEOQ_DECODE_ARGS) { return decode_entry(1, AEOQ_DECODE_PASS); }
extern "C" int aeoq_moe_nvfp4_decode_down(AEOQ_DECODE_ARGS) { return decode_entry(2, AEOQ_DECODE_PASS); }
