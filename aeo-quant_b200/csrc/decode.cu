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
#include "common.cuh"

namespace aeoq {

constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDownRows = 16;    // output rows per CTA in launch 2
constexpr int kMaxTopK = 16;

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

  // Activation quant: global amax -> tensor scale (bf16) -> lane chunks.
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
  __half2 act[CPL][16];
  float sa[CPL][2];
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int64_t c = lane + 32 * j;
    if (c < nchunk) quant_act_chunk_bf16(hidden + 32 * c, ts, act[j], sa[j]);
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

template <int CPL2>
__global__ void __launch_bounds__(kDecThreads) moe_decode_down_kernel(
    const __nv_bfloat16* __restrict__ h, const uint32_t* __restrict__ parts, int nparts,
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
    // shared tensor scale of the k x I intermediate (one amax key per launch-1 CTA)
    uint32_t key = 0;
    for (int i = lane; i < nparts; i += 32) key = max(key, parts[i]);
    key = warp_umax(key);
    const float ts = nvfp4_tensor_scale<AEOQ_BF16>(In<AEOQ_BF16>::key_to_f(key));
    const float alpha = ts * load_scalar_f(d_ts, d_ts_dt);
    const float wj = __bfloat162float(topw[j]);
    __half2 act[CPL2][16];
    float sa[CPL2][2];
#pragma unroll
    for (int q = 0; q < CPL2; ++q) {
      const int64_t c = lane + 32 * q;
      if (c < nchunk) quant_act_chunk_bf16(h + j * I + 32 * c, ts, act[q], sa[q]);
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

static int g_num_sms = 0;

static int num_sms() {
  if (!g_num_sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

static int gateup_grid(int64_t k, int64_t I) {
  const int64_t pairs = k * I;
  const int64_t want = (pairs + kDecWarps - 1) / kDecWarps;
  const int64_t cap = 2 * (int64_t)num_sms();
  return (int)(want < cap ? want : cap);
}

}  // namespace aeoq

using namespace aeoq;

extern "C" size_t aeoq_moe_nvfp4_decode_workspace_size(int64_t top_k, int64_t hidden, int64_t inter) {
  (void)hidden;
  const size_t h_bytes = ((size_t)(top_k * inter) * 2 + 255) / 256 * 256;
  return h_bytes + (size_t)gateup_grid(top_k, inter) * sizeof(uint32_t);
}

// stages: bit 0 = gate_up launch, bit 1 = down launch (both for the fused op)
template <int CPL, int CPL2>
static int launch_decode(int stages, const void* hidden, const void* ids, int ids_dt, const void* topw, int k,
                         const uint8_t* gu, const uint8_t* gu_sf, const void* gu_ts, int gu_ts_dt,
                         const uint8_t* dw, const uint8_t* dw_sf, const void* d_ts, int d_ts_dt,
                         int64_t E, int64_t H, int64_t I, void* out, void* ws, cudaStream_t st) {
  const int g1 = gateup_grid(k, I);
  const size_t h_bytes = ((size_t)(k * I) * 2 + 255) / 256 * 256;
  __nv_bfloat16* hbuf = reinterpret_cast<__nv_bfloat16*>(ws);
  uint32_t* parts = reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(ws) + h_bytes);
  if (stages & 1) {
    moe_decode_gateup_kernel<CPL><<<g1, kDecThreads, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(hidden), ids, ids_dt, k, gu, gu_sf, gu_ts, gu_ts_dt, E, H, I,
        hbuf, parts);
    int rc = check_launch("moe_decode_gateup_kernel");
    if (rc) return rc;
  }
  if (!(stages & 2)) return AEOQ_OK;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((H + kDownRows - 1) / kDownRows));
  cfg.blockDim = dim3(kDecThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, moe_decode_down_kernel<CPL2>, (const __nv_bfloat16*)hbuf,
                                     (const uint32_t*)parts, g1, ids, ids_dt,
                                     reinterpret_cast<const __nv_bfloat16*>(topw), k, dw, dw_sf, d_ts,
                                     d_ts_dt, E, H, I, reinterpret_cast<__nv_bfloat16*>(out));
  if (e != cudaSuccess) return set_error(AEOQ_ERR_CUDA, "moe_decode_down_kernel: %s", cudaGetErrorString(e));
  return check_launch("moe_decode_down_kernel");
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
