// CUDA-core block-scaled NVFP4 GEMM for small M, with optional expert gather.
//
// Serves nvfp4_linear_prequantized / nvfp4_linear_3d_prequantized /
// nvfp4_linear_3d_gather (aeo_quant src/aeo_quant/gpu/nvfp4_matmul.py:399-864)
// when M is small: the work is then a stream over the selected experts'
// packed weights (HBM-bound), so each warp owns one weight row (slot s,
// output n), keeps the row's chunks in registers (one 16-byte coalesced load
// per lane per 32 K-values) and sweeps the M activation rows against it.
// Per 16-value block the FP4 x FP4 products are summed exactly in fp16, then
// scaled by the two e4m3 block scales in fp32; alpha = f32(a_ts)*f32(w_ts)
// and the output cast close the epilogue as in the reference kernel
// (nvfp4_matmul.py:315-325).
#include "common.cuh"

namespace aeoq {

constexpr int kGemvWarps = 4;
constexpr int kGemvChunksPerLane = 4;  // K up to 4096 per register tile

struct GemvArgs {
  const uint8_t* a; const uint8_t* a_sf; const void* a_ts; int a_ts_dt;
  int64_t a_ss, a_rs, a_sfss, a_sfrs;
  const uint8_t* w; const uint8_t* w_sf; const void* w_ts; int w_ts_dt;
  int64_t w_es, w_rs, w_sfes, w_sfrs;
  const void* ids; int ids_dt; int64_t num_experts;
  int64_t slots, M, N, K;
  void* c; int c_dt; int64_t c_ss, c_rs;
};

__global__ void __launch_bounds__(kGemvWarps * 32) nvfp4_gemv_kernel(GemvArgs g) {
  const int lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x * (int64_t)kGemvWarps + (threadIdx.x >> 5);  // (slot, n)
  if (row >= g.slots * g.N) return;
  const int64_t s = row / g.N, n = row - s * g.N;
  const int64_t e = g.ids ? load_index(g.ids, g.ids_dt, s) : s;
  const bool valid = (e >= 0 && e < g.num_experts);
  const float alpha = load_scalar_f(g.a_ts, g.a_ts_dt) * load_scalar_f(g.w_ts, g.w_ts_dt);
  const int64_t nchunk = g.K / 32;
  const uint8_t* wrow = g.w + e * g.w_es + n * g.w_rs;
  const uint8_t* wsrow = g.w_sf + e * g.w_sfes + n * g.w_sfrs;
  const uint8_t* arow0 = g.a + s * g.a_ss;
  const uint8_t* asrow0 = g.a_sf + s * g.a_sfss;

  for (int64_t m0 = 0; m0 < g.M; m0 += 1) {
    float acc = 0.0f;
    if (valid) {
      const uint8_t* arow = arow0 + m0 * g.a_rs;
      const uint8_t* asrow = asrow0 + m0 * g.a_sfrs;
      for (int64_t c0 = 0; c0 < nchunk; c0 += 32 * kGemvChunksPerLane) {
#pragma unroll
        for (int j = 0; j < kGemvChunksPerLane; ++j) {
          const int64_t c = c0 + lane + 32 * j;
          if (c < nchunk) {
            const uint4 wv = ldg_stream(wrow + 16 * c);
            const uint16_t wsf = *reinterpret_cast<const uint16_t*>(wsrow + 2 * c);
            const uint4 av = *reinterpret_cast<const uint4*>(arow + 16 * c);
            const uint16_t asf = *reinterpret_cast<const uint16_t*>(asrow + 2 * c);
            __half2 ah[16];
            float sa16k[2];
            decode_act_chunk(av, asf, ah, sa16k);
            acc = chunk_dot(ah, sa16k, wv, wsf, acc);
          }
        }
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) {
      char* cp = reinterpret_cast<char*>(g.c) + s * g.c_ss + m0 * g.c_rs;
      const float v = acc * alpha;
      if (g.c_dt == AEOQ_BF16) reinterpret_cast<__nv_bfloat16*>(cp)[n] = __float2bfloat16_rn(v);
      else reinterpret_cast<float*>(cp)[n] = v;
    }
  }
}

}  // namespace aeoq

using namespace aeoq;

extern "C" int aeoq_nvfp4_gemm(const uint8_t* a, const uint8_t* a_sf, const void* a_ts, int a_ts_dtype,
                               int64_t a_slot_stride, int64_t a_row_stride,
                               int64_t a_sf_slot_stride, int64_t a_sf_row_stride,
                               const uint8_t* w, const uint8_t* w_sf, const void* w_ts, int w_ts_dtype,
                               int64_t w_expert_stride, int64_t w_row_stride,
                               int64_t w_sf_expert_stride, int64_t w_sf_row_stride,
                               const void* expert_ids, int ids_dtype, int64_t num_experts,
                               int64_t slots, int64_t M, int64_t N, int64_t K,
                               void* c, int c_dtype, int64_t c_slot_stride, int64_t c_row_stride,
                               void* stream) {
  AEOQ_REQUIRE(slots >= 0 && M >= 0 && N >= 0 && K >= 0, AEOQ_ERR_INVALID, "nvfp4_gemm: negative shape");
  AEOQ_REQUIRE(K % 32 == 0, AEOQ_ERR_INVALID, "nvfp4_gemm: K (%lld) must be a multiple of 32", (long long)K);
  AEOQ_REQUIRE(c_dtype == AEOQ_BF16 || c_dtype == AEOQ_F32, AEOQ_ERR_INVALID,
               "nvfp4_gemm: output dtype must be bf16 or f32");
  AEOQ_REQUIRE(!expert_ids || ids_dtype == AEOQ_I32 || ids_dtype == AEOQ_I64, AEOQ_ERR_INVALID,
               "nvfp4_gemm: expert ids must be int32 or int64");
  if (slots * M * N == 0) return AEOQ_OK;
  AEOQ_REQUIRE(a && a_sf && a_ts && w && w_sf && w_ts && c, AEOQ_ERR_INVALID, "nvfp4_gemm: null pointer");
  const bool aligned = ((uintptr_t)a % 16 == 0) && ((uintptr_t)w % 16 == 0) && (a_row_stride % 16 == 0) &&
                       (a_slot_stride % 16 == 0) && (w_row_stride % 16 == 0) && (w_expert_stride % 16 == 0) &&
                       ((uintptr_t)a_sf % 2 == 0) && ((uintptr_t)w_sf % 2 == 0) && (a_sf_row_stride % 2 == 0) &&
                       (a_sf_slot_stride % 2 == 0) && (w_sf_row_stride % 2 == 0) && (w_sf_expert_stride % 2 == 0);
  AEOQ_REQUIRE(aligned, AEOQ_ERR_INVALID,
               "nvfp4_gemm: packed rows must be 16-byte aligned and scale rows 2-byte aligned");
  GemvArgs g{a, a_sf, a_ts, a_ts_dtype, a_slot_stride, a_row_stride, a_sf_slot_stride, a_sf_row_stride,
             w, w_sf, w_ts, w_ts_dtype, w_expert_stride, w_row_stride, w_sf_expert_stride, w_sf_row_stride,
             expert_ids, ids_dtype, expert_ids ? num_experts : slots, slots, M, N, K,
             c, c_dtype, c_slot_stride, c_row_stride};
  const int64_t rows = slots * N;
  const int64_t blocks = (rows + kGemvWarps - 1) / kGemvWarps;
  nvfp4_gemv_kernel<<<blocks, kGemvWarps * 32, 0, (cudaStream_t)stream>>>(g);
  return check_launch("nvfp4_gemv_kernel");
}
