// Whole expert-layer forwards behind one C call each, for hosts that bind the
// library without the Python package: the launch sequence of the Python
// layer (bridges/gemma4/moe_ops.py) in C++, over one caller-provided
// workspace.
//
//   aeoq_moe_nvfp4_forward: Gemma4TextExpertsNVFP4._forward_prefill
//     (aeo_quant src/aeo_quant/bridges/gemma4/modeling_nvfp4.py:188-255), or
//     with one_token_semantics the rounding of _forward_decode_3d (:132-186)
//     over any number of tokens. route -> NVFP4 quantization of the hidden
//     rows (global tensor scale) -> gather by expert -> grouped gate_up GEMM
//     with the GeGLU epilogue -> NVFP4 re-quantization (per-expert or shared
//     tensor scale) -> grouped down GEMM weighted by the routing weights ->
//     combine in ascending expert order.
//   aeoq_moe_fp8_forward: Gemma4TextExpertsFP8.forward
//     (src/aeo_quant/bridges/gemma4/modeling.py:110-146). route -> gathered
//     per-row e4m3 quantization -> grouped gate_up GEMM with GeGLU -> per-row
//     re-quantization -> grouped down GEMM weighted -> bf16 index_add_ fold.
//
// Neither allocates: every intermediate lives in the workspace, carved in a
// fixed order at 256-byte boundaries (sizes from the *_workspace_size
// functions). Nothing synchronises with the host; all work is stream-ordered
// on `stream`.
#include <algorithm>

#include "common.cuh"

namespace aeoq {
namespace {

// Token-tile width of the grouped GEMMs from the mean rows per expert (the
// same rule as the Python layer's pick_tile_n).
int pick_tile_n(int64_t pairs, int64_t experts) {
  const int64_t avg = std::max<int64_t>(1, pairs / std::max<int64_t>(1, std::min(experts, pairs)));
  for (int bn : {8, 16, 32, 64})
    if (avg <= bn) return bn;
  return avg < 160 ? 128 : 224;
}

struct Carver {
  uint8_t* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<uint8_t*>(b)) {}
  template <class T>
  T* take(size_t bytes) {
    T* p = reinterpret_cast<T*>(base ? base + off : nullptr);
    off += (std::max<size_t>(bytes, 1) + 255) / 256 * 256;
    return p;
  }
};

struct RouteBufs {
  int *cnt, *fill, *grp_off, *tile_off, *pair_row, *row_tok, *row_exp;
  __nv_bfloat16* row_w;
};

RouteBufs carve_route(Carver& c, int64_t P, int64_t E) {
  RouteBufs r;
  r.cnt = c.take<int>(4 * E);
  r.fill = c.take<int>(4 * E);
  r.grp_off = c.take<int>(4 * (E + 1));
  r.tile_off = c.take<int>(4 * (E + 1));
  r.pair_row = c.take<int>(4 * P);
  r.row_tok = c.take<int>(4 * P);
  r.row_exp = c.take<int>(4 * P);
  r.row_w = c.take<__nv_bfloat16>(2 * P);
  return r;
}

struct Nvfp4Bufs {
  RouteBufs r;
  uint8_t *hp, *hs, *qws, *a_sorted, *a_sorted_sf, *hq, *hq_sf;
  __nv_bfloat16 *hts, *h_sorted, *c_sorted;
  uint32_t* amax;
  float* ts_e;
  size_t qws_bytes;
};

Nvfp4Bufs carve_nvfp4(Carver& c, int64_t T, int64_t k, int64_t E, int64_t H, int64_t I, int tile_n) {
  const int64_t P = T * k;
  const int64_t max_tiles = (P + tile_n - 1) / tile_n + E;
  Nvfp4Bufs b;
  b.r = carve_route(c, P, E);
  b.hp = c.take<uint8_t>((size_t)T * H / 2);
  b.hs = c.take<uint8_t>((size_t)T * H / 16);
  b.hts = c.take<__nv_bfloat16>(2);
  b.qws_bytes = aeoq_nvfp4_quantize_workspace_size(T, H);
  b.qws = c.take<uint8_t>(b.qws_bytes);
  b.a_sorted = c.take<uint8_t>((size_t)P * H / 2);
  b.a_sorted_sf = c.take<uint8_t>(aeoq_nvfp4_act_atoms_size(max_tiles, H, tile_n));
  b.amax = c.take<uint32_t>(4 * E);
  b.h_sorted = c.take<__nv_bfloat16>((size_t)P * I * 2);
  b.hq = c.take<uint8_t>((size_t)P * I / 2);
  b.hq_sf = c.take<uint8_t>(aeoq_nvfp4_act_atoms_size(max_tiles, I, tile_n));
  b.ts_e = c.take<float>(4 * E);
  b.c_sorted = c.take<__nv_bfloat16>((size_t)P * H * 2);
  return b;
}

// The buffers of the grouped pipeline over rows that arrive already
// quantized (the expert-parallel experts step): the same as carve_nvfp4
// without the activation quantizer's.
Nvfp4Bufs carve_nvfp4_rows(Carver& c, int64_t n, int64_t k, int64_t E, int64_t H, int64_t I, int tile_n) {
  const int64_t P = n * k;
  const int64_t max_tiles = (P + tile_n - 1) / tile_n + E;
  Nvfp4Bufs b{};
  b.r = carve_route(c, P, E);
  b.a_sorted = c.take<uint8_t>((size_t)P * H / 2);
  b.a_sorted_sf = c.take<uint8_t>(aeoq_nvfp4_act_atoms_size(max_tiles, H, tile_n));
  b.amax = c.take<uint32_t>(4 * E);
  b.h_sorted = c.take<__nv_bfloat16>((size_t)P * I * 2);
  b.hq = c.take<uint8_t>((size_t)P * I / 2);
  b.hq_sf = c.take<uint8_t>(aeoq_nvfp4_act_atoms_size(max_tiles, I, tile_n));
  b.ts_e = c.take<float>(4 * E);
  b.c_sorted = c.take<__nv_bfloat16>((size_t)P * H * 2);
  return b;
}

struct Fp8Bufs {
  RouteBufs r;
  uint8_t *xq, *hq;
  float *sa, *sh;
  __nv_bfloat16 *h, *c;
};

Fp8Bufs carve_fp8(Carver& c, int64_t T, int64_t k, int64_t E, int64_t H, int64_t I) {
  const int64_t P = T * k;
  Fp8Bufs b;
  b.r = carve_route(c, P, E);
  b.xq = c.take<uint8_t>((size_t)P * H);
  b.sa = c.take<float>(4 * P);
  b.h = c.take<__nv_bfloat16>((size_t)P * I * 2);
  b.hq = c.take<uint8_t>((size_t)P * I);
  b.sh = c.take<float>(4 * P);
  b.c = c.take<__nv_bfloat16>((size_t)P * H * 2);
  return b;
}

int check_shape(int64_t T, int64_t k, int64_t E, int64_t H, int64_t I, const char* who) {
  AEOQ_REQUIRE(T >= 0 && k >= 1 && k <= 16 && E >= 1 && H > 0 && I > 0, AEOQ_ERR_INVALID,
               "%s: bad shape (T=%lld, top_k=%lld, experts=%lld, hidden=%lld, inter=%lld)", who, (long long)T,
               (long long)k, (long long)E, (long long)H, (long long)I);
  AEOQ_REQUIRE(T * k <= INT32_MAX, AEOQ_ERR_INVALID, "%s: more than 2^31 (token, slot) pairs", who);
  return AEOQ_OK;
}

#define AEOQ_TRY(expr)             \
  do {                             \
    const int rc_ = (expr);        \
    if (rc_ != AEOQ_OK) return rc_; \
  } while (0)

}  // namespace
}  // namespace aeoq

using namespace aeoq;

extern "C" size_t aeoq_moe_nvfp4_forward_workspace_size(int64_t T, int64_t top_k, int64_t num_experts,
                                                        int64_t hidden, int64_t inter) {
  if (T <= 0 || top_k <= 0 || num_experts <= 0 || hidden <= 0 || inter <= 0) return 0;
  Carver c(nullptr);
  carve_nvfp4(c, T, top_k, num_experts, hidden, inter, pick_tile_n(T * top_k, num_experts));
  return c.off;
}

extern "C" int aeoq_moe_nvfp4_forward(const void* hidden, int64_t T, const void* top_k_index, int idx_dtype,
                                      const void* top_k_weights, int64_t top_k, const uint8_t* gate_up,
                                      const uint8_t* gate_up_atoms, const void* gate_up_ts, int gate_up_ts_dtype,
                                      const uint8_t* down, const uint8_t* down_atoms, const void* down_ts,
                                      int down_ts_dtype, int64_t num_experts, int64_t hidden_size, int64_t inter,
                                      int one_token_semantics, void* out, void* workspace, size_t workspace_bytes,
                                      int* err_word, void* stream) {
  const int64_t E = num_experts, H = hidden_size, I = inter, k = top_k;
  AEOQ_TRY(check_shape(T, k, E, H, I, "moe_nvfp4_forward"));
  if (T == 0) return AEOQ_OK;
  AEOQ_REQUIRE(hidden && top_k_index && top_k_weights && gate_up && gate_up_atoms && gate_up_ts && down &&
                   down_atoms && down_ts && out && err_word,
               AEOQ_ERR_INVALID, "moe_nvfp4_forward: null pointer");
  const size_t need = aeoq_moe_nvfp4_forward_workspace_size(T, k, E, H, I);
  AEOQ_REQUIRE(workspace && workspace_bytes >= need, AEOQ_ERR_WORKSPACE,
               "moe_nvfp4_forward: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  AEOQ_REQUIRE((uintptr_t)workspace % 256 == 0, AEOQ_ERR_INVALID, "moe_nvfp4_forward: workspace not 256-byte aligned");
  const int64_t P = T * k;
  const int tile_n = pick_tile_n(P, E);
  Carver c(workspace);
  const Nvfp4Bufs b = carve_nvfp4(c, T, k, E, H, I, tile_n);
  const int* n_rows = b.r.grp_off + E;
  cudaStream_t st = (cudaStream_t)stream;

  AEOQ_TRY(aeoq_moe_route(top_k_index, idx_dtype, top_k_weights, T, k, E, tile_n, b.r.cnt, b.r.fill, b.r.grp_off,
                          b.r.tile_off, b.r.pair_row, b.r.row_tok, b.r.row_w, b.r.row_exp, stream));
  // the hidden rows with one global tensor scale (modeling_nvfp4.py:203-206)
  AEOQ_TRY(aeoq_nvfp4_quantize(hidden, AEOQ_BF16, T, H, H, b.hp, b.hs, b.hts, b.qws, b.qws_bytes, stream));
  AEOQ_TRY(aeoq_gather_rows(b.hp, b.hs, b.r.row_tok, b.r.row_exp, b.r.grp_off, b.r.tile_off, tile_n, n_rows, P, H / 2,
                            H / 16, b.a_sorted, b.a_sorted_sf, stream));
  if (cudaMemsetAsync(b.amax, 0, sizeof(uint32_t) * E, st) != cudaSuccess) return check_launch("moe_nvfp4_forward");
  AEOQ_TRY(aeoq_nvfp4_gemm_grouped(b.a_sorted, b.a_sorted_sf, P, b.r.grp_off, b.r.tile_off, tile_n, gate_up,
                                   gate_up_atoms, E, 2 * I, H, 1, b.hts, AEOQ_BF16, gate_up_ts, gate_up_ts_dtype,
                                   nullptr, nullptr, b.amax, b.h_sorted, I * 2, err_word, stream));
  AEOQ_TRY(aeoq_requant_rows(b.h_sorted, I, b.r.row_exp, b.r.grp_off, b.r.tile_off, tile_n, n_rows, P, b.amax, E,
                             one_token_semantics ? 1 : 0, b.hq, b.hq_sf, b.ts_e, stream));
  AEOQ_TRY(aeoq_nvfp4_gemm_grouped(b.hq, b.hq_sf, P, b.r.grp_off, b.r.tile_off, tile_n, down, down_atoms, E, H, I, 2,
                                   nullptr, 0, down_ts, down_ts_dtype, b.ts_e, b.r.row_w, nullptr, b.c_sorted, H * 2,
                                   err_word, stream));
  return aeoq_moe_combine(b.c_sorted, b.r.pair_row, top_k_index, idx_dtype, T, k, H, one_token_semantics ? 1 : 0,
                          out, stream);
}

extern "C" size_t aeoq_moe_fp8_forward_workspace_size(int64_t T, int64_t top_k, int64_t num_experts, int64_t hidden,
                                                      int64_t inter) {
  if (T <= 0 || top_k <= 0 || num_experts <= 0 || hidden <= 0 || inter <= 0) return 0;
  Carver c(nullptr);
  carve_fp8(c, T, top_k, num_experts, hidden, inter);
  return c.off;
}

extern "C" int aeoq_moe_fp8_forward(const void* hidden, int64_t T, const void* top_k_index, int idx_dtype,
                                    const void* top_k_weights, int64_t top_k, const uint8_t* gate_up,
                                    const float* gate_up_scale, const uint8_t* down, const float* down_scale,
                                    int64_t num_experts, int64_t hidden_size, int64_t inter, void* out,
                                    void* workspace, size_t workspace_bytes, int* err_word, void* stream) {
  const int64_t E = num_experts, H = hidden_size, I = inter, k = top_k;
  AEOQ_TRY(check_shape(T, k, E, H, I, "moe_fp8_forward"));
  if (T == 0) return AEOQ_OK;
  AEOQ_REQUIRE(hidden && top_k_index && top_k_weights && gate_up && gate_up_scale && down && down_scale && out &&
                   err_word,
               AEOQ_ERR_INVALID, "moe_fp8_forward: null pointer");
  const size_t need = aeoq_moe_fp8_forward_workspace_size(T, k, E, H, I);
  AEOQ_REQUIRE(workspace && workspace_bytes >= need, AEOQ_ERR_WORKSPACE,
               "moe_fp8_forward: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  AEOQ_REQUIRE((uintptr_t)workspace % 256 == 0, AEOQ_ERR_INVALID, "moe_fp8_forward: workspace not 256-byte aligned");
  const int64_t P = T * k;
  const int tile_n = pick_tile_n(P, E);
  Carver c(workspace);
  const Fp8Bufs b = carve_fp8(c, T, k, E, H, I);
  const int* n_rows = b.r.grp_off + E;

  AEOQ_TRY(aeoq_moe_route(top_k_index, idx_dtype, top_k_weights, T, k, E, tile_n, b.r.cnt, b.r.fill, b.r.grp_off,
                          b.r.tile_off, b.r.pair_row, b.r.row_tok, b.r.row_w, b.r.row_exp, stream));
  AEOQ_TRY(aeoq_fp8_quantize_rows_gather(hidden, H, b.r.row_tok, n_rows, P, H, b.xq, H, b.sa, stream));
  AEOQ_TRY(aeoq_fp8_gemm_grouped(b.xq, b.sa, P, b.r.grp_off, b.r.tile_off, tile_n, gate_up, gate_up_scale, E, 2 * I,
                                 H, 1, nullptr, b.h, I * 2, err_word, stream));
  AEOQ_TRY(aeoq_fp8_quantize_rows_gather(b.h, I, nullptr, n_rows, P, I, b.hq, I, b.sh, stream));
  AEOQ_TRY(aeoq_fp8_gemm_grouped(b.hq, b.sh, P, b.r.grp_off, b.r.tile_off, tile_n, down, down_scale, E, H, I, 2,
                                 b.r.row_w, b.c, H * 2, err_word, stream));
  return aeoq_moe_combine(b.c, b.r.pair_row, top_k_index, idx_dtype, T, k, H, 0, out, stream);
}

// ---------------------------------------------------------------------------
// Expert-parallel experts step: the grouped forward of rows that arrived
// NVFP4-quantized (aeoq_ep_dispatch) over this rank's experts, each row's
// local experts folded in ascending id with bf16 rounding after every add.
// The launch sequence of NVFP4EpOps.experts
// (aeo_quant_b200/bridges/gemma4/expert_parallel.py).
// ---------------------------------------------------------------------------
extern "C" size_t aeoq_ep_experts_nvfp4_workspace_size(int64_t n_rows, int64_t top_k, int64_t pairs_hint,
                                                       int64_t local_experts, int64_t hidden, int64_t inter) {
  if (n_rows <= 0 || top_k <= 0 || local_experts <= 0 || hidden <= 0 || inter <= 0) return 0;
  Carver c(nullptr);
  carve_nvfp4_rows(c, n_rows, top_k, local_experts, hidden, inter,
                   pick_tile_n(pairs_hint > 0 ? pairs_hint : n_rows * top_k / 2, local_experts));
  return c.off;
}

extern "C" int aeoq_ep_experts_nvfp4(const uint8_t* packed, const uint8_t* sf, const void* ts, int64_t n_rows,
                                     const int32_t* local_ids, const void* weights, int64_t top_k,
                                     int64_t pairs_hint, const uint8_t* gate_up, const uint8_t* gate_up_atoms,
                                     const void* gate_up_ts, int gate_up_ts_dtype, const uint8_t* down,
                                     const uint8_t* down_atoms, const void* down_ts, int down_ts_dtype,
                                     int64_t local_experts, int64_t hidden_size, int64_t inter, void* out,
                                     void* workspace, size_t workspace_bytes, int* err_word, void* stream) {
  const int64_t E = local_experts, H = hidden_size, I = inter, k = top_k, n = n_rows;
  AEOQ_TRY(check_shape(n, k, E, H, I, "ep_experts_nvfp4"));
  if (n == 0) return AEOQ_OK;
  AEOQ_REQUIRE(packed && sf && ts && local_ids && weights && gate_up && gate_up_atoms && gate_up_ts && down &&
                   down_atoms && down_ts && out && err_word,
               AEOQ_ERR_INVALID, "ep_experts_nvfp4: null pointer");
  const size_t need = aeoq_ep_experts_nvfp4_workspace_size(n, k, pairs_hint, E, H, I);
  AEOQ_REQUIRE(workspace && workspace_bytes >= need, AEOQ_ERR_WORKSPACE,
               "ep_experts_nvfp4: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  AEOQ_REQUIRE((uintptr_t)workspace % 256 == 0, AEOQ_ERR_INVALID, "ep_experts_nvfp4: workspace not 256-byte aligned");
  const int64_t P = n * k;
  const int tile_n = pick_tile_n(pairs_hint > 0 ? pairs_hint : P / 2, E);
  Carver c(workspace);
  const Nvfp4Bufs b = carve_nvfp4_rows(c, n, k, E, H, I, tile_n);
  const int* n_rows_dev = b.r.grp_off + E;
  cudaStream_t st = (cudaStream_t)stream;
  AEOQ_TRY(aeoq_moe_route(local_ids, AEOQ_I32, weights, n, k, E, tile_n, b.r.cnt, b.r.fill, b.r.grp_off, b.r.tile_off,
                          b.r.pair_row, b.r.row_tok, b.r.row_w, b.r.row_exp, stream));
  AEOQ_TRY(aeoq_gather_rows(packed, sf, b.r.row_tok, b.r.row_exp, b.r.grp_off, b.r.tile_off, tile_n, n_rows_dev, P,
                            H / 2, H / 16, b.a_sorted, b.a_sorted_sf, stream));
  if (cudaMemsetAsync(b.amax, 0, sizeof(uint32_t) * E, st) != cudaSuccess) return check_launch("ep_experts_nvfp4");
  AEOQ_TRY(aeoq_nvfp4_gemm_grouped(b.a_sorted, b.a_sorted_sf, P, b.r.grp_off, b.r.tile_off, tile_n, gate_up,
                                   gate_up_atoms, E, 2 * I, H, 1, ts, AEOQ_BF16, gate_up_ts, gate_up_ts_dtype,
                                   nullptr, nullptr, b.amax, b.h_sorted, I * 2, err_word, stream));
  AEOQ_TRY(aeoq_requant_rows(b.h_sorted, I, b.r.row_exp, b.r.grp_off, b.r.tile_off, tile_n, n_rows_dev, P, b.amax, E,
                             0, b.hq, b.hq_sf, b.ts_e, stream));
  AEOQ_TRY(aeoq_nvfp4_gemm_grouped(b.hq, b.hq_sf, P, b.r.grp_off, b.r.tile_off, tile_n, down, down_atoms, E, H, I, 2,
                                   nullptr, 0, down_ts, down_ts_dtype, b.ts_e, b.r.row_w, nullptr, b.c_sorted, H * 2,
                                   err_word, stream));
  return aeoq_moe_combine(b.c_sorted, b.r.pair_row, local_ids, AEOQ_I32, n, k, H, 0, out, stream);
}
