// NVFP4 and FP8 quantizers, bit-exact with aeo_quant src/aeo_quant/gpu/quant.py.
//
// NVFP4 (quant.py:138-185) needs the global amax before any element can be
// binned, so large tensors take two launches: a grid-wide partial amax that
// writes one key per CTA into the workspace, then the quantize pass whose
// CTAs each re-reduce those few hundred keys. Small tensors (<= 64K elements:
// every activation quant on the decode path) run both phases in one CTA.
// Each thread owns one 16-element block: 2-4 x 16-byte loads, 8 packed bytes
// and one e4m3 code out. HBM-bound: 2 B read twice + 0.5625 B written per
// bf16 element.
#include "common.cuh"

namespace aeoq {

constexpr int kQuantThreads = 256;
constexpr int64_t kSmallElems = 1 << 16;
constexpr int kMaxParts = 148 * 8;

template <int DT, bool VEC>
__device__ __forceinline__ void load_group(const typename In<DT>::T* p, float (&v)[16]) {
  using T = typename In<DT>::T;
  if constexpr (VEC) {
    constexpr int kVec = 16 / sizeof(T);
#pragma unroll
    for (int i = 0; i < 16; i += kVec) {
      uint4 u = *reinterpret_cast<const uint4*>(p + i);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < kVec; ++j) v[i + j] = In<DT>::to_f(e[j]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = In<DT>::load(p + i);
  }
}

template <int DT, bool VEC>
__device__ __forceinline__ uint32_t group_key(const typename In<DT>::T* p) {
  using T = typename In<DT>::T;
  uint32_t k = 0;
  if constexpr (VEC) {
    constexpr int kVec = 16 / sizeof(T);
#pragma unroll
    for (int i = 0; i < 16; i += kVec) {
      uint4 u = *reinterpret_cast<const uint4*>(p + i);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < kVec; ++j) k = max(k, In<DT>::abs_key(e[j]));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) k = max(k, In<DT>::abs_key(p[i]));
  }
  return k;
}

__device__ __forceinline__ uint32_t block_umax(uint32_t v, uint32_t* sm) {
  v = warp_umax(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sm[w] = v;
  __syncthreads();
  if (w == 0) {
    v = (l < (int)(blockDim.x >> 5)) ? sm[l] : 0u;
    v = warp_umax(v);
    if (l == 0) sm[0] = v;
  }
  __syncthreads();
  v = sm[0];
  __syncthreads();
  return v;
}

template <int DT, bool VEC>
__device__ __forceinline__ void quant_group(const typename In<DT>::T* x, int64_t g, int64_t gpr,
                                            int64_t ld, float ts, const float* tab, uint8_t* packed, uint8_t* sf) {
  const int64_t r = g / gpr, c = g - r * gpr;
  float v[16];
  load_group<DT, VEC>(x + r * ld + c * 16, v);
  uint32_t w0, w1;
  uint32_t code = nvfp4_quant_block_tab(v, ts, tab, w0, w1);
  *reinterpret_cast<uint2*>(packed + g * 8) = make_uint2(w0, w1);
  sf[g] = (uint8_t)code;
}

template <int DT, bool VEC>
__global__ void __launch_bounds__(1024) nvfp4_quant_small_kernel(
    const typename In<DT>::T* __restrict__ x, int64_t rows, int64_t gpr, int64_t ld,
    uint8_t* __restrict__ packed, uint8_t* __restrict__ sf, void* ts_out) {
  __shared__ uint32_t sm[32];
  __shared__ __align__(16) float tab[128 * 8];
  const int64_t ng = rows * gpr;
  uint32_t key = 0;
  for (int64_t g = threadIdx.x; g < ng; g += blockDim.x) {
    const int64_t r = g / gpr, c = g - r * gpr;
    key = max(key, group_key<DT, VEC>(x + r * ld + c * 16));
  }
  key = block_umax(key, sm);
  const float ts = nvfp4_tensor_scale<DT>(ng ? In<DT>::key_to_f(key) : 0.0f);
  if (threadIdx.x == 0) In<DT>::store(ts_out, ts);
  nvfp4_threshold_table(ts, tab, threadIdx.x, blockDim.x);
  __syncthreads();
  for (int64_t g = threadIdx.x; g < ng; g += blockDim.x)
    quant_group<DT, VEC>(x, g, gpr, ld, ts, tab, packed, sf);
}

template <int DT, bool VEC>
__global__ void __launch_bounds__(kQuantThreads) amax_partial_kernel(
    const typename In<DT>::T* __restrict__ x, int64_t rows, int64_t gpr, int64_t ld,
    uint32_t* __restrict__ parts) {
  __shared__ uint32_t sm[32];
  const int64_t ng = rows * gpr;
  uint32_t key = 0;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < ng;
       g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = g / gpr, c = g - r * gpr;
    key = max(key, group_key<DT, VEC>(x + r * ld + c * 16));
  }
  key = block_umax(key, sm);
  if (threadIdx.x == 0) parts[blockIdx.x] = key;
}

template <int DT, bool VEC>
__global__ void __launch_bounds__(kQuantThreads) nvfp4_quant_kernel(
    const typename In<DT>::T* __restrict__ x, int64_t rows, int64_t gpr, int64_t ld,
    const uint32_t* __restrict__ parts, int nparts, const void* ts_in,
    uint8_t* __restrict__ packed, uint8_t* __restrict__ sf, void* ts_out) {
  __shared__ uint32_t sm[32];
  __shared__ __align__(16) float tab[128 * 8];
  float ts;
  if (ts_in) {
    ts = In<DT>::load(reinterpret_cast<const typename In<DT>::T*>(ts_in));
  } else {
    uint32_t key = 0;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) key = max(key, parts[i]);
    key = block_umax(key, sm);
    ts = nvfp4_tensor_scale<DT>(In<DT>::key_to_f(key));
    if (blockIdx.x == 0 && threadIdx.x == 0 && ts_out) In<DT>::store(ts_out, ts);
  }
  nvfp4_threshold_table(ts, tab, threadIdx.x, blockDim.x);
  __syncthreads();
  const int64_t ng = rows * gpr;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < ng;
       g += (int64_t)gridDim.x * blockDim.x)
    quant_group<DT, VEC>(x, g, gpr, ld, ts, tab, packed, sf);
}

static int dtype_size(int dt) { return dt == AEOQ_F32 ? 4 : 2; }

static int nparts_for(int64_t ng) {
  int64_t b = (ng + kQuantThreads - 1) / kQuantThreads;
  return (int)(b < kMaxParts ? (b < 1 ? 1 : b) : kMaxParts);
}

template <int DT, bool VEC>
static int launch_quant(const void* xv, int64_t rows, int64_t K, int64_t ld, uint8_t* packed,
                        uint8_t* sf, void* ts_out, const void* ts_in, uint32_t* parts,
                        cudaStream_t st) {
  using T = typename In<DT>::T;
  const T* x = reinterpret_cast<const T*>(xv);
  const int64_t gpr = K / 16, ng = rows * gpr;
  if (!ts_in && rows * K <= kSmallElems) {
    nvfp4_quant_small_kernel<DT, VEC><<<1, 1024, 0, st>>>(x, rows, gpr, ld, packed, sf, ts_out);
    return check_launch("nvfp4_quant_small_kernel");
  }
  const int np = nparts_for(ng);
  if (!ts_in) {
    amax_partial_kernel<DT, VEC><<<np, kQuantThreads, 0, st>>>(x, rows, gpr, ld, parts);
    int rc = check_launch("amax_partial_kernel");
    if (rc) return rc;
  }
  nvfp4_quant_kernel<DT, VEC><<<np, kQuantThreads, 0, st>>>(x, rows, gpr, ld, parts, np, ts_in,
                                                            packed, sf, ts_out);
  return check_launch("nvfp4_quant_kernel");
}

static int dispatch_quant(const void* x, int dtype, int64_t rows, int64_t K, int64_t ld,
                          uint8_t* packed, uint8_t* sf, void* ts_out, const void* ts_in,
                          uint32_t* parts, cudaStream_t st) {
  const int es = dtype_size(dtype);
  const bool vec = ((uintptr_t)x % 16 == 0) && ((ld * es) % 16 == 0);
#define AEOQ_Q(DT)                                                                          \
  return vec ? launch_quant<DT, true>(x, rows, K, ld, packed, sf, ts_out, ts_in, parts, st) \
             : launch_quant<DT, false>(x, rows, K, ld, packed, sf, ts_out, ts_in, parts, st)
  switch (dtype) {
    case AEOQ_BF16: AEOQ_Q(AEOQ_BF16);
    case AEOQ_F16: AEOQ_Q(AEOQ_F16);
    case AEOQ_F32: AEOQ_Q(AEOQ_F32);
  }
#undef AEOQ_Q
  return set_error(AEOQ_ERR_INVALID, "nvfp4_quantize: unsupported dtype %d", dtype);
}

static int check_quant_args(const void* x, int dtype, int64_t rows, int64_t K, int64_t ld,
                            const uint8_t* packed, const uint8_t* sf) {
  AEOQ_REQUIRE(dtype == AEOQ_BF16 || dtype == AEOQ_F16 || dtype == AEOQ_F32, AEOQ_ERR_INVALID,
               "nvfp4_quantize: dtype must be bf16, f16 or f32 (got %d)", dtype);
  AEOQ_REQUIRE(rows >= 0 && K >= 0, AEOQ_ERR_INVALID, "nvfp4_quantize: negative shape");
  AEOQ_REQUIRE(K % 16 == 0, AEOQ_ERR_INVALID,
               "in_dim (%lld) must be divisible by block_size (16)", (long long)K);
  AEOQ_REQUIRE(ld >= K, AEOQ_ERR_INVALID, "nvfp4_quantize: ld (%lld) < K (%lld)", (long long)ld,
               (long long)K);
  AEOQ_REQUIRE(((uintptr_t)packed % 8) == 0, AEOQ_ERR_INVALID,
               "nvfp4_quantize: packed output must be 8-byte aligned");
  AEOQ_REQUIRE(rows * K == 0 || (x && packed && sf), AEOQ_ERR_INVALID, "nvfp4_quantize: null pointer");
  return AEOQ_OK;
}

}  // namespace aeoq

using namespace aeoq;

extern "C" size_t aeoq_nvfp4_quantize_workspace_size(int64_t rows, int64_t K) {
  if (rows * K <= kSmallElems) return 0;
  return (size_t)nparts_for(rows * (K / 16)) * sizeof(uint32_t);
}

extern "C" int aeoq_nvfp4_quantize(const void* x, int dtype, int64_t rows, int64_t K, int64_t ld,
                                   uint8_t* packed, uint8_t* sf, void* ts_out, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  int rc = check_quant_args(x, dtype, rows, K, ld, packed, sf);
  if (rc) return rc;
  AEOQ_REQUIRE(ts_out, AEOQ_ERR_INVALID, "nvfp4_quantize: ts_out is null");
  const size_t need = aeoq_nvfp4_quantize_workspace_size(rows, K);
  AEOQ_REQUIRE(workspace_bytes >= need && (need == 0 || workspace), AEOQ_ERR_WORKSPACE,
               "nvfp4_quantize: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  return dispatch_quant(x, dtype, rows, K, ld, packed, sf, ts_out, nullptr,
                        reinterpret_cast<uint32_t*>(workspace), (cudaStream_t)stream);
}

extern "C" int aeoq_nvfp4_quantize_with_scale(const void* x, int dtype, int64_t rows, int64_t K,
                                              int64_t ld, const void* ts_in, uint8_t* packed,
                                              uint8_t* sf, void* stream) {
  int rc = check_quant_args(x, dtype, rows, K, ld, packed, sf);
  if (rc) return rc;
  AEOQ_REQUIRE(ts_in, AEOQ_ERR_INVALID, "nvfp4_quantize_with_scale: ts_in is null");
  if (rows * K == 0) return AEOQ_OK;
  return dispatch_quant(x, dtype, rows, K, ld, packed, sf, nullptr, ts_in, nullptr,
                        (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// FP8 per-row quantizer: one warp per row.
// ---------------------------------------------------------------------------
namespace aeoq {

template <int DT>
__global__ void __launch_bounds__(256) fp8_rows_kernel(const typename In<DT>::T* __restrict__ x,
                                                       int64_t rows, int64_t K, int64_t ld,
                                                       uint8_t* __restrict__ q, int64_t q_ld,
                                                       void* __restrict__ scale_out, int mode) {
  const int64_t row = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const typename In<DT>::T* xr = x + row * ld;
  uint32_t key = 0;
  for (int64_t i = lane; i < K; i += 32) key = max(key, In<DT>::abs_key(xr[i]));
  key = warp_umax(key);
  const float amax = K ? In<DT>::key_to_f(key) : 0.0f;
  float s;
  if (mode == AEOQ_FP8_WEIGHT) {
    // (max_abs / 448).clamp(min=1e-8) in the input dtype, then to bf16 (quant.py:101-102)
    float t = In<DT>::round(div_rn(amax, kFp8Max));
    t = nan_max(t, In<DT>::round(1e-8f));
    s = bf16r(t);
    if (lane == 0) reinterpret_cast<__nv_bfloat16*>(scale_out)[row] = __float2bfloat16_rn(s);
  } else {
    // amax.clamp(min=1e-4) in the input dtype -> f32, / 448 (modeling.py:102-103)
    float a = nan_max(amax, In<DT>::round(1e-4f));
    s = div_rn(a, kFp8Max);
    if (lane == 0) reinterpret_cast<float*>(scale_out)[row] = s;
  }
  uint8_t* qr = q + row * q_ld;
  for (int64_t i = lane; i < K; i += 32) qr[i] = (uint8_t)e4m3_encode(div_rn(In<DT>::load(xr + i), s));
}

}  // namespace aeoq

extern "C" int aeoq_fp8_quantize_rows(const void* x, int dtype, int64_t rows, int64_t K, int64_t ld,
                                      uint8_t* q, int64_t q_ld, void* scale_out, int mode,
                                      void* stream) {
  AEOQ_REQUIRE(mode == AEOQ_FP8_WEIGHT || mode == AEOQ_FP8_ACTIVATION, AEOQ_ERR_INVALID,
               "fp8_quantize_rows: bad mode %d", mode);
  AEOQ_REQUIRE(rows >= 0 && K >= 0 && ld >= K && q_ld >= K, AEOQ_ERR_INVALID,
               "fp8_quantize_rows: bad shape");
  if (rows == 0) return AEOQ_OK;
  AEOQ_REQUIRE(x && q && scale_out, AEOQ_ERR_INVALID, "fp8_quantize_rows: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t blocks = (rows + 7) / 8;
  switch (dtype) {
    case AEOQ_BF16:
      fp8_rows_kernel<AEOQ_BF16><<<blocks, 256, 0, st>>>((const __nv_bfloat16*)x, rows, K, ld, q, q_ld, scale_out, mode);
      break;
    case AEOQ_F16:
      fp8_rows_kernel<AEOQ_F16><<<blocks, 256, 0, st>>>((const __half*)x, rows, K, ld, q, q_ld, scale_out, mode);
      break;
    case AEOQ_F32:
      fp8_rows_kernel<AEOQ_F32><<<blocks, 256, 0, st>>>((const float*)x, rows, K, ld, q, q_ld, scale_out, mode);
      break;
    default:
      return set_error(AEOQ_ERR_INVALID, "fp8_quantize_rows: unsupported dtype %d", dtype);
  }
  return check_launch("fp8_rows_kernel");
}

// ---------------------------------------------------------------------------
// FP8 per-row activation quantizer over gathered rows: output row r is input
// row idx[r] (identity without idx), r < *n_rows (or max_rows). bf16 input,
// K % 8 == 0; one warp per row, 16-byte loads. Semantics of _fp8_linear's
// input quantization (modeling.py:101-104), as AEOQ_FP8_ACTIVATION above.
// ---------------------------------------------------------------------------
namespace aeoq {

__global__ void __launch_bounds__(256) fp8_rows_gather_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld,
                                                              const int* __restrict__ idx,
                                                              const int* __restrict__ n_rows, int64_t max_rows,
                                                              int64_t K, uint8_t* __restrict__ q, int64_t q_ld,
                                                              float* __restrict__ scale_out) {
  const int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t nr = n_rows ? (int64_t)*n_rows : max_rows;
  if (r >= nr || r >= max_rows) return;
  const int64_t src = idx ? (int64_t)idx[r] : r;
  const uint4* xr = reinterpret_cast<const uint4*>(x + src * ld);
  uint32_t key = 0;
  for (int64_t i = lane; i < K / 8; i += 32) {
    const uint4 u = xr[i];
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) key = max(key, In<AEOQ_BF16>::abs_key(e[j]));
  }
  key = warp_umax(key);
  const float a = nan_max(K ? In<AEOQ_BF16>::key_to_f(key) : 0.0f, In<AEOQ_BF16>::round(1e-4f));
  const float s = div_rn(a, kFp8Max);
  if (lane == 0) scale_out[r] = s;
  uint2* qr = reinterpret_cast<uint2*>(q + r * q_ld);
  for (int64_t i = lane; i < K / 8; i += 32) {
    const uint4 u = xr[i];
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j >> 2] |= e4m3_encode(div_rn(__bfloat162float(e[j]), s)) << (8 * (j & 3));
    qr[i] = make_uint2(w[0], w[1]);
  }
}

}  // namespace aeoq

extern "C" int aeoq_fp8_quantize_rows_gather(const void* x, int64_t ld, const int* row_idx, const int* n_rows,
                                             int64_t max_rows, int64_t K, uint8_t* q, int64_t q_ld,
                                             float* scale_out, void* stream) {
  AEOQ_REQUIRE(max_rows >= 0 && K >= 0 && ld >= K && q_ld >= K, AEOQ_ERR_INVALID,
               "fp8_quantize_rows_gather: bad shape");
  AEOQ_REQUIRE(K % 8 == 0 && ld % 8 == 0 && q_ld % 8 == 0, AEOQ_ERR_INVALID,
               "fp8_quantize_rows_gather: K and strides must be multiples of 8");
  if (max_rows == 0 || K == 0) return AEOQ_OK;
  AEOQ_REQUIRE(x && q && scale_out, AEOQ_ERR_INVALID, "fp8_quantize_rows_gather: null pointer");
  AEOQ_REQUIRE((uintptr_t)x % 16 == 0 && (uintptr_t)q % 8 == 0, AEOQ_ERR_INVALID,
               "fp8_quantize_rows_gather: x 16-byte and q 8-byte alignment required");
  fp8_rows_gather_kernel<<<(unsigned)((max_rows + 7) / 8), 256, 0, (cudaStream_t)stream>>>(
      (const __nv_bfloat16*)x, ld, row_idx, n_rows, max_rows, K, q, q_ld, scale_out);
  return check_launch("fp8_rows_gather_kernel");
}

// ---------------------------------------------------------------------------
// NVFP4 dequantizer (quant.py:188-212): bf16(value * block_scale * ts),
// evaluated left to right in float32. One thread per 16-element block.
// ---------------------------------------------------------------------------
namespace aeoq {

__global__ void __launch_bounds__(256) nvfp4_dequant_kernel(const uint8_t* __restrict__ packed,
                                                            const uint8_t* __restrict__ sf,
                                                            const void* ts_p, int ts_dt, int64_t ngroups,
                                                            __nv_bfloat16* __restrict__ out) {
  const float ts = load_scalar_f(ts_p, ts_dt);
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < ngroups;
       g += (int64_t)gridDim.x * blockDim.x) {
    const uint2 p = *reinterpret_cast<const uint2*>(packed + 8 * g);
    const float bs = e4m3_decode(sf[g]);
    const uint32_t words[2] = {p.x, p.y};
    __align__(16) __nv_bfloat16 o[16];
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      const uint32_t byte = (words[i >> 3] >> (8 * ((i >> 1) & 3))) & 0xFFu;
      o[i] = __float2bfloat16_rn(fp4_value(byte >> 4) * bs * ts);
      o[i + 1] = __float2bfloat16_rn(fp4_value(byte & 0xFu) * bs * ts);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + 16 * g);
    dst[0] = *reinterpret_cast<uint4*>(&o[0]);
    dst[1] = *reinterpret_cast<uint4*>(&o[8]);
  }
}

}  // namespace aeoq

extern "C" int aeoq_nvfp4_dequantize(const uint8_t* packed, const uint8_t* sf, const void* ts, int ts_dtype,
                                     int64_t rows, int64_t K, void* out, void* stream) {
  AEOQ_REQUIRE(rows >= 0 && K >= 0 && K % 16 == 0, AEOQ_ERR_INVALID,
               "nvfp4_dequantize: K (%lld) must be a multiple of 16", (long long)K);
  if (rows * K == 0) return AEOQ_OK;
  AEOQ_REQUIRE(packed && sf && ts && out && (uintptr_t)packed % 8 == 0 && (uintptr_t)out % 16 == 0,
               AEOQ_ERR_INVALID, "nvfp4_dequantize: null or misaligned pointer");
  const int64_t ng = rows * (K / 16);
  const int64_t blocks = (ng + 255) / 256 < 148 * 16 ? (ng + 255) / 256 : 148 * 16;
  nvfp4_dequant_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(packed, sf, ts, ts_dtype, ng,
                                                                  reinterpret_cast<__nv_bfloat16*>(out));
  return check_launch("nvfp4_dequant_kernel");
}
