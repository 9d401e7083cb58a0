/*
 * aeoq.h — C ABI of the B200 (sm_100a) quantized MoE expert library.
 *
 * Every entry point takes plain device pointers, element counts, byte strides
 * and a cudaStream_t passed as void*. None allocates device memory: callers
 * pass outputs and, where a kernel needs scratch, a workspace whose size the
 * matching *_workspace_size() function returns. All calls are asynchronous
 * on the given stream, never synchronize the host, and never abort: they
 * return AEOQ_OK (0) or a negative status, with a message available from
 * aeoq_last_error() (thread-local).
 *
 * The Python package aeo_quant_b200 binds these with ctypes and mirrors the
 * aeo_quant Python API that each entry point replaces; citations below are
 * path:line inside the aeo_quant project.
 */
#ifndef AEOQ_H_
#define AEOQ_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define AEOQ_API __attribute__((visibility("default")))
#else
#define AEOQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* element type codes */
#define AEOQ_BF16 0
#define AEOQ_F16 1
#define AEOQ_F32 2
#define AEOQ_I32 3
#define AEOQ_I64 4

/* status codes */
#define AEOQ_OK 0
#define AEOQ_ERR_INVALID (-1)     /* bad shape, stride, dtype or alignment */
#define AEOQ_ERR_CUDA (-2)        /* a CUDA launch or runtime call failed */
#define AEOQ_ERR_WORKSPACE (-3)   /* workspace missing or too small */
#define AEOQ_ERR_UNSUPPORTED (-4) /* device is not sm_100 */

/* FP8 row-quantizer modes */
#define AEOQ_FP8_WEIGHT 0     /* quant.py:51-106 — bf16 scale per row */
#define AEOQ_FP8_ACTIVATION 1 /* bridges/gemma4/modeling.py:101-104 — f32 scale */

/* Library version (major*10000 + minor*100 + patch). */
AEOQ_API int aeoq_version(void);

/* Message for the last failing call on this host thread ("" if none). */
AEOQ_API const char* aeoq_last_error(void);

/* ------------------------------------------------------------------------
 * NVFP4 two-level quantizer.
 * Replaces quantize_2d_to_nvfp4 / quantize_3d_to_nvfp4
 * (src/aeo_quant/gpu/quant.py:138-185, :215-230) and the activation alias
 * _quantize_bf16_activation_to_nvfp4 (src/aeo_quant/gpu/nvfp4_matmul.py:338-354).
 *
 * x        rows x K elements of `dtype` (AEOQ_BF16/F16/F32), row stride `ld`
 *          elements; leading dims of the reference tensor are flattened.
 * packed   rows x K/2 bytes, contiguous (high nibble = even k).
 * sf       rows x K/16 e4m3fn codes, contiguous.
 * ts_out   one element of `dtype`: clamp(amax/2688, 1e-12) in that dtype.
 * Bit-exact with the reference. K % 16 == 0 required (quant.py:161-164).
 * ------------------------------------------------------------------------ */
AEOQ_API size_t aeoq_nvfp4_quantize_workspace_size(int64_t rows, int64_t K);
AEOQ_API int aeoq_nvfp4_quantize(const void* x, int dtype, int64_t rows, int64_t K, int64_t ld,
                        uint8_t* packed, uint8_t* sf, void* ts_out,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Same, with a caller-provided tensor scale (`ts_in`, one `dtype` element on
 * the device) instead of the global amax. Used where one scale is shared
 * across a batch that is quantized in pieces. */
AEOQ_API int aeoq_nvfp4_quantize_with_scale(const void* x, int dtype, int64_t rows, int64_t K, int64_t ld,
                                   const void* ts_in, uint8_t* packed, uint8_t* sf, void* stream);

/* NVFP4 dequantizer: bf16(value * block_scale * ts), rows x K out, contiguous.
 * Replaces dequant_2d_from_nvfp4 / dequant_3d_from_nvfp4 (quant.py:188-212,
 * :233-246). `ts` is one element of ts_dtype on the device. */
AEOQ_API int aeoq_nvfp4_dequantize(const uint8_t* packed, const uint8_t* sf, const void* ts, int ts_dtype,
                          int64_t rows, int64_t K, void* out, void* stream);

/* ------------------------------------------------------------------------
 * FP8 e4m3fn per-row quantizer.
 * mode AEOQ_FP8_WEIGHT replaces quantize_2d_to_fp8 / quantize_3d_to_fp8
 * (src/aeo_quant/gpu/quant.py:51-106): scale_out is rows bf16 values.
 * mode AEOQ_FP8_ACTIVATION replaces the per-row dynamic input quant of
 * Gemma4TextExpertsFP8._fp8_linear (src/aeo_quant/bridges/gemma4/modeling.py:101-104):
 * scale_out is rows f32 values. Bit-exact with the reference.
 * ------------------------------------------------------------------------ */
AEOQ_API int aeoq_fp8_quantize_rows(const void* x, int dtype, int64_t rows, int64_t K, int64_t ld,
                           uint8_t* q, int64_t q_ld, void* scale_out, int mode, void* stream);

/* ------------------------------------------------------------------------
 * Block-scaled NVFP4 GEMM with optional expert gather.
 * Replaces nvfp4_linear_prequantized, nvfp4_linear_3d_prequantized and
 * nvfp4_linear_3d_gather (src/aeo_quant/gpu/nvfp4_matmul.py:399-519,
 * :522-686, :689-864), i.e. the Triton kernels _nvfp4_matmul_kernel,
 * _nvfp4_matmul_kernel_3d and _nvfp4_matmul_kernel_3d_gather (:51-325).
 *
 *   C[s][m][n] = out( alpha * sum_k A[s][m][k] * W[e(s)][n][k] )
 *   e(s) = expert_ids ? expert_ids[s] : s;   alpha = f32(*a_ts) * f32(*w_ts)
 *
 * Operands are packed FP4 bytes with e4m3 block scales (16 along K). All
 * strides are in BYTES; a_slot_stride == 0 shares one activation across the
 * slots (the reference's stride_ae = 0). Packed rows must be 16-byte aligned.
 * An expert id outside [0, num_experts) contributes zeros (the reference's
 * forward skips id == num_experts, modeling_nvfp4.py:220).
 * c_dtype is AEOQ_BF16 or AEOQ_F32.
 * ------------------------------------------------------------------------ */
AEOQ_API int aeoq_nvfp4_gemm(const uint8_t* a, const uint8_t* a_sf, const void* a_ts, int a_ts_dtype,
                    int64_t a_slot_stride, int64_t a_row_stride,
                    int64_t a_sf_slot_stride, int64_t a_sf_row_stride,
                    const uint8_t* w, const uint8_t* w_sf, const void* w_ts, int w_ts_dtype,
                    int64_t w_expert_stride, int64_t w_row_stride,
                    int64_t w_sf_expert_stride, int64_t w_sf_row_stride,
                    const void* expert_ids, int ids_dtype, int64_t num_experts,
                    int64_t slots, int64_t M, int64_t N, int64_t K,
                    void* c, int c_dtype, int64_t c_slot_stride, int64_t c_row_stride,
                    void* stream);

/* Tensor-core (tcgen05, kind::mxf4nvf4) path of aeoq_nvfp4_gemm for
 * contiguous operands: activation rows of K/2 bytes (a_slot_rows != 0: each
 * slot has its own M rows; 0: one M-row activation shared by every slot),
 * weights [num_experts, N, K/2], scales [.., K/16], C [slots, M, N].
 * N % 128 == 0, K % 64 == 0. `err_word` is a device int that a bounded wait
 * sets non-zero if the pipeline stalls (never expected). Same replaced
 * reference functions as aeoq_nvfp4_gemm (nvfp4_matmul.py:399-864). */
AEOQ_API int aeoq_nvfp4_gemm_tc(const uint8_t* a, const uint8_t* a_sf_atoms, const void* a_ts, int a_ts_dtype,
                                int64_t a_slot_rows, const uint8_t* w, const uint8_t* w_sf_atoms, const void* w_ts,
                                int w_ts_dtype, int64_t num_experts, const void* expert_ids, int ids_dtype,
                                int64_t slots, int64_t M, int64_t N, int64_t K, int tile_n, void* c, int c_dtype,
                                int* err_word, void* stream);

/* Token-tile width for M activation rows against N weight rows in `slots`
 * problems (the activation atoms must be built for the same width). */
AEOQ_API int aeoq_nvfp4_tile_n(int64_t M, int64_t N, int64_t slots);

/* Scale-factor atoms (the order tcgen05.cp loads into tensor memory: 128
 * rows x 4 scales per 512 B, row r at byte (r%32)*16 + (r/32)*4).
 * Weights: [groups][rows_per_group/128][K/64][512 B]; with geglu_inter = I
 * each 128-row tile holds gate rows 64t.. and up rows I+64t.. of a group.
 * Activations: [tile][K/64][ceil(tile_n/128)][512 B], rows r of slot r/M in
 * tiles of tile_n. Sizes in bytes from the *_size functions. */
AEOQ_API size_t aeoq_nvfp4_weight_atoms_size(int64_t rows, int64_t K);
AEOQ_API size_t aeoq_nvfp4_act_atoms_size(int64_t tiles, int64_t K, int tile_n);
AEOQ_API int aeoq_nvfp4_sf_to_atoms(const uint8_t* sf, int64_t groups, int64_t rows_per_group, int64_t K,
                                    int64_t geglu_inter, uint8_t* out, void* stream);
AEOQ_API int aeoq_nvfp4_rows_to_tile_atoms(const uint8_t* sf, int64_t rows, int64_t M, int64_t K, int tile_n,
                                           uint8_t* out, void* stream);

/* Grouped tensor-core GEMM over expert-sorted activation rows (the MoE
 * prefill path). Expert e owns sorted rows [grp_off[e], grp_off[e+1]) and
 * token tiles [tile_off[e], tile_off[e+1]) of tile_n rows (as produced by
 * aeoq_moe_route). epi 0: C = bf16(f32(*a_ts) * f32(*w_ts) * acc);
 * epi 1 (gate_up, N = 2I): C[r][0..I) = bf16(bf16(gelu(g)) * u), with the
 * per-expert max |C| accumulated into grp_amax keys (zero them first);
 * epi 2 (down): C = bf16(bf16(grp_ts[e] * f32(*w_ts) * acc) * row_w[r]).
 * Scales as atoms: b_sf_atoms token-tile atoms, w_sf weight atoms (GeGLU
 * layout for epi 1, plain otherwise).
 * Replaces the per-expert nvfp4_linear_prequantized / nvfp4_linear calls,
 * GeGLU and weighting of _forward_prefill (modeling_nvfp4.py:218-249). */
AEOQ_API int aeoq_nvfp4_gemm_grouped(const uint8_t* b, const uint8_t* b_sf_atoms, int64_t max_rows, const int* grp_off,
                                     const int* tile_off, int tile_n, const uint8_t* w, const uint8_t* w_sf,
                                     int64_t num_experts, int64_t N, int64_t K, int epi, const void* a_ts,
                                     int a_ts_dtype, const void* w_ts, int w_ts_dtype, const float* grp_ts,
                                     const void* row_w, uint32_t* grp_amax, void* c, int64_t ldc, int* err_word,
                                     void* stream);

/* FP8 tensor-core GEMMs (tcgen05.mma kind::f8f6f4, e4m3 x e4m3 -> f32) with
 * the rowwise scaling of torch._scaled_mm as _fp8_linear calls it
 * (bridges/gemma4/modeling.py:89-108).
 * aeoq_fp8_gemm: a (M, K) e4m3 rows, sa (M) f32; w (N, K) e4m3, sb (N) f32;
 *   C (M, N) bf16 = bf16((acc * sa[m]) * sb[n]). N % 128 == 0, K % 32 == 0.
 * aeoq_fp8_gemm_grouped: expert-sorted rows b (max_rows, K) with sa_rows;
 *   w (E, N, K), sb_rows (E * N) f32; epi 0 plain, 1 GeGLU (N = 2I, output
 *   I wide, bf16(bf16(gelu(g)) * u)), 2 down weighted by row_w (bf16). */
AEOQ_API int aeoq_fp8_gemm(const uint8_t* a, const float* sa, int64_t M, const uint8_t* w, const float* sb,
                           int64_t N, int64_t K, void* c, int* err_word, void* stream);
AEOQ_API int aeoq_fp8_gemm_grouped(const uint8_t* b, const float* sa_rows, int64_t max_rows, const int* grp_off,
                                   const int* tile_off, int tile_n, const uint8_t* w, const float* sb_rows,
                                   int64_t num_experts, int64_t N, int64_t K, int epi, const void* row_w, void* c,
                                   int64_t ldc, int* err_word, void* stream);

/* FP8 per-row activation quantization (_fp8_linear, modeling.py:101-104) of
 * gathered bf16 rows: q[r] = e4m3(x[idx[r]] / sa[r]), sa[r] = max(amax, 1e-4)
 * / 448 (f32), for r < *n_rows (device count; max_rows bounds the launch).
 * idx = NULL reads row r. K, ld, q_ld multiples of 8. */
AEOQ_API int aeoq_fp8_quantize_rows_gather(const void* x, int64_t ld, const int* row_idx, const int* n_rows,
                                           int64_t max_rows, int64_t K, uint8_t* q, int64_t q_ld,
                                           float* scale_out, void* stream);

/* Gemma-4 router for T tokens (HF transformers 5.5.0 Gemma4TextRouter.forward,
 * models/gemma4/modeling_gemma4.py:1296-1316): probs = softmax(proj(
 * bf16(bf16(rmsnorm(x)) * scale) * root_scale)), top_k of probs (descending,
 * equal values by lower expert id), renormalised and multiplied by
 * per_expert_scale. x (T, H) bf16 with row stride ldx; scale (H,), proj_w
 * (E, H), per_expert_scale (E,) bf16. Outputs probs (T, E) bf16, top_w
 * (T, top_k) bf16, top_i (T, top_k) int64. H and ldx multiples of 8, H <=
 * 6144 and >= 2 E + 128, E a multiple of 8 and <= 256, top_k <= min(E, 32). One launch,
 * one 8-CTA cluster per 16 tokens. */
AEOQ_API int aeoq_gemma4_router(const void* x, int64_t ldx, const void* scale, const void* proj_w,
                                const void* per_expert_scale, int64_t T, int64_t H, int64_t E, int64_t top_k,
                                float eps, float root_scale, void* probs, void* top_w, int64_t* top_i,
                                void* stream);

/* Device-side grouping of (token, slot) pairs by expert (replaces the
 * one_hot / nonzero / where scaffolding, modeling_nvfp4.py:208-222, and
 * modeling.py:111-121): counts, row offsets, token-tile offsets for tile_n,
 * pair -> sorted row, and per sorted row its token, routing weight and
 * expert. Arrays: cnt/fill [E] (scratch), grp_off/tile_off [E+1],
 * pair_row [T*k] (-1 for ids outside [0,E)), row_tok/row_w(bf16)/row_exp [T*k]. */
AEOQ_API int aeoq_moe_route(const void* top_k_index, int idx_dtype, const void* top_k_weights, int64_t T,
                            int64_t k, int64_t num_experts, int tile_n, int* cnt, int* fill, int* grp_off,
                            int* tile_off, int* pair_row, int* row_tok, void* row_w, int* row_exp, void* stream);

/* dst[r] = src[row_tok[r]] for r < *n_rows; the scale rows go to the
 * grouped GEMM's token-tile atoms (expert of row r: row_exp[r]). */
AEOQ_API int aeoq_gather_rows(const uint8_t* src, const uint8_t* src_sf, const int* row_tok, const int* row_exp,
                              const int* grp_off, const int* tile_off, int tile_n, const int* n_rows,
                              int64_t max_rows, int64_t row_bytes, int64_t sf_bytes, uint8_t* dst,
                              uint8_t* dst_atoms, void* stream);

/* NVFP4 re-quantization of the sorted GeGLU rows: one tensor scale per
 * expert from amax_key[e] (shared_scale = 0; per-expert nvfp4_linear in the
 * prefill path, nvfp4_matmul.py:386) or one for all rows (shared_scale = 1;
 * the one-token path, modeling_nvfp4.py:164-172). ts_out[e] gets the scales. */
AEOQ_API int aeoq_requant_rows(const void* h, int64_t I, const int* row_exp, const int* grp_off, const int* tile_off,
                               int tile_n, const int* n_rows, int64_t max_rows, const uint32_t* amax_key,
                               int64_t num_experts, int shared_scale, uint8_t* hq, uint8_t* hsf_atoms,
                               float* ts_out, void* stream);

/* out[t] = fold over token t's expert outputs in ascending expert order:
 * mode 0 bf16 rounding after every add (index_add_, modeling_nvfp4.py:250-253);
 * mode 1 f32 sum rounded once (modeling_nvfp4.py:181-186). */
AEOQ_API int aeoq_moe_combine(const void* c_sorted, const int* pair_row, const void* top_k_index, int idx_dtype,
                              int64_t T, int64_t k, int64_t H, int mode, void* out, void* stream);

/* ------------------------------------------------------------------------
 * Whole expert-layer forwards, one call each (the launch sequence of the
 * Python layer over one caller-provided workspace; nothing is allocated,
 * nothing synchronises with the host). hidden (T, H) bf16 contiguous;
 * top_k_index (T, k) int32/int64 (idx_dtype), ids outside [0, E) dropped;
 * top_k_weights (T, k) bf16; out (T, H) bf16. err_word: device int that a
 * tensor-core wait which times out sets nonzero.
 *
 * aeoq_moe_nvfp4_forward replaces Gemma4TextExpertsNVFP4._forward_prefill
 * (src/aeo_quant/bridges/gemma4/modeling_nvfp4.py:188-255): one global
 * activation tensor scale, per-expert re-quantized down input, bf16
 * index_add_ fold. one_token_semantics = 1 gives the rounding of
 * _forward_decode_3d (:132-186): one shared down-input scale, f32 combine.
 * gate_up (E, 2I, H/2) / down (E, H, I/2) packed E2M1; their scales as
 * weight atoms from aeoq_nvfp4_sf_to_atoms (gate_up with geglu_inter = I,
 * down with 0); *_ts 0-d tensor scales (f32 or bf16 per *_ts_dtype).
 *
 * aeoq_moe_fp8_forward replaces Gemma4TextExpertsFP8.forward
 * (src/aeo_quant/bridges/gemma4/modeling.py:110-146): gate_up (E, 2I, H) and
 * down (E, H, I) e4m3, per-output-channel scales flat f32 (E * 2I), (E * H).
 * ------------------------------------------------------------------------ */
AEOQ_API size_t aeoq_moe_nvfp4_forward_workspace_size(int64_t T, int64_t top_k, int64_t num_experts,
                                                      int64_t hidden, int64_t inter);
AEOQ_API int aeoq_moe_nvfp4_forward(const void* hidden, int64_t T, const void* top_k_index, int idx_dtype,
                                    const void* top_k_weights, int64_t top_k, const uint8_t* gate_up,
                                    const uint8_t* gate_up_atoms, const void* gate_up_ts, int gate_up_ts_dtype,
                                    const uint8_t* down, const uint8_t* down_atoms, const void* down_ts,
                                    int down_ts_dtype, int64_t num_experts, int64_t hidden_size, int64_t inter,
                                    int one_token_semantics, void* out, void* workspace, size_t workspace_bytes,
                                    int* err_word, void* stream);
AEOQ_API size_t aeoq_moe_fp8_forward_workspace_size(int64_t T, int64_t top_k, int64_t num_experts, int64_t hidden,
                                                    int64_t inter);
AEOQ_API int aeoq_moe_fp8_forward(const void* hidden, int64_t T, const void* top_k_index, int idx_dtype,
                                  const void* top_k_weights, int64_t top_k, const uint8_t* gate_up,
                                  const float* gate_up_scale, const uint8_t* down, const float* down_scale,
                                  int64_t num_experts, int64_t hidden_size, int64_t inter, void* out,
                                  void* workspace, size_t workspace_bytes, int* err_word, void* stream);

/* ------------------------------------------------------------------------
 * Expert-parallel NVFP4 layer over NCCL (config 4), one rank per GPU, every
 * rank with the same T tokens (sequence-sharded prefill). Replaces, for a
 * host without Python, the layer's three phases in
 * aeo_quant_b200/bridges/gemma4/expert_parallel.py (_ep_dense); the
 * reference runs its experts on one GPU (modeling_nvfp4.py:188-255), and
 * this layer's output is within the bf16 re-association of the rank fold
 * of that forward (bit-identical to the Python layer).
 *
 *   aeoq_ep_dispatch        (comm, ...) -> recv_packed (world*T, H/2) u8,
 *                           recv_sf (world*T, H/16) e4m3 rows,
 *                           recv_local_ids (world*T, k) i32,
 *                           recv_weights (world*T, k) bf16, ts_out bf16 0-d,
 *                           slot_row (T, world) i32 for the combine
 *   aeoq_ep_experts_nvfp4   the received rows through this rank's E/world
 *                           experts (weights of those experts only, scale
 *                           atoms as for aeoq_moe_nvfp4_forward; pairs_hint
 *                           = T*k picks the tile width, any gives the same
 *                           bits) -> out (world*T, H) bf16
 *   aeoq_ep_combine         those rows back to their home ranks and each
 *                           token's partials folded in rank order -> out (T, H)
 *
 * comm is an ncclComm_t: the host's own, or one from aeoq_ep_nccl_comm_init
 * (unique id from aeoq_ep_nccl_unique_id on one rank, passed to the others
 * by the host). placement: null = experts [r*E/world, (r+1)*E/world) on rank
 * r; else device int32 [2E]: owner rank of expert e, then its index among
 * that rank's experts (ascending id). libnccl.so.2 is opened at the first
 * call; AEOQ_ERR_UNSUPPORTED if it is absent. Workspaces 256-byte aligned.
 * ------------------------------------------------------------------------ */
AEOQ_API size_t aeoq_ep_nccl_unique_id_bytes(void);
AEOQ_API int aeoq_ep_nccl_unique_id(void* out, size_t out_bytes);
AEOQ_API int aeoq_ep_nccl_comm_init(void** comm, int world, int rank, const void* unique_id);
AEOQ_API int aeoq_ep_nccl_comm_destroy(void* comm);
AEOQ_API size_t aeoq_ep_dispatch_workspace_size(int world, int64_t T, int64_t top_k, int64_t hidden);
AEOQ_API int aeoq_ep_dispatch(void* comm, int world, int rank, const void* hidden, int64_t T, int64_t H,
                              const void* top_k_index, int idx_dtype, const void* top_k_weights, int64_t top_k,
                              int64_t num_experts, const int32_t* placement, uint8_t* recv_packed, uint8_t* recv_sf,
                              int32_t* recv_local_ids, void* recv_weights, void* ts_out, int32_t* slot_row,
                              void* workspace, size_t workspace_bytes, void* stream);
AEOQ_API size_t aeoq_ep_experts_nvfp4_workspace_size(int64_t n_rows, int64_t top_k, int64_t pairs_hint,
                                                     int64_t local_experts, int64_t hidden, int64_t inter);
AEOQ_API int aeoq_ep_experts_nvfp4(const uint8_t* packed, const uint8_t* sf, const void* ts, int64_t n_rows,
                                   const int32_t* local_ids, const void* weights, int64_t top_k, int64_t pairs_hint,
                                   const uint8_t* gate_up, const uint8_t* gate_up_atoms, const void* gate_up_ts,
                                   int gate_up_ts_dtype, const uint8_t* down, const uint8_t* down_atoms,
                                   const void* down_ts, int down_ts_dtype, int64_t local_experts, int64_t hidden_size,
                                   int64_t inter, void* out, void* workspace, size_t workspace_bytes, int* err_word,
                                   void* stream);
AEOQ_API size_t aeoq_ep_combine_workspace_size(int world, int64_t T, int64_t hidden);
AEOQ_API int aeoq_ep_combine(void* comm, int world, int rank, const void* rows, const int32_t* slot_row, int64_t T,
                             int64_t H, void* out, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * One-token NVFP4 MoE expert forward, fully fused (two launches).
 * Replaces Gemma4TextExpertsNVFP4._forward_decode_3d
 * (src/aeo_quant/bridges/gemma4/modeling_nvfp4.py:132-186): hidden quant ->
 * gathered gate_up GEMV -> GeGLU (bf16) -> shared-scale re-quant -> gathered
 * down GEMV -> bf16 weighted combine. Same bf16 rounding points.
 *
 * hidden      [1, H] bf16        top_k_index [1, k] int32/int64 (idx_dtype)
 * top_k_w     [1, k] bf16        out         [1, H] bf16
 * gate_up     [E, 2I, H/2] u8 contiguous, gate_up_sf [E, 2I, H/16] e4m3
 * down        [E, H, I/2]  u8 contiguous, down_sf    [E, H, I/16]  e4m3
 * *_ts        0-d tensor scale (f32 or bf16, *_ts_dtype)
 * Requires H % 64 == 0, I % 64 == 0, 1 <= k <= 16.
 * ------------------------------------------------------------------------ */
AEOQ_API size_t aeoq_moe_nvfp4_decode_workspace_size(int64_t top_k, int64_t hidden, int64_t inter);
AEOQ_API int aeoq_moe_nvfp4_decode(const void* hidden, const void* top_k_index, int idx_dtype,
                          const void* top_k_weights, int64_t top_k,
                          const uint8_t* gate_up, const uint8_t* gate_up_sf,
                          const void* gate_up_ts, int gate_up_ts_dtype,
                          const uint8_t* down, const uint8_t* down_sf,
                          const void* down_ts, int down_ts_dtype,
                          int64_t num_experts, int64_t hidden_dim, int64_t inter_dim,
                          void* out, void* workspace, size_t workspace_bytes, void* stream);

/* The two launches of aeoq_moe_nvfp4_decode issued one at a time, same
 * arguments. gate_up leaves the GeGLU output and its amax in the workspace;
 * down consumes them. Used to time and profile each stage on its own. */
AEOQ_API int aeoq_moe_nvfp4_decode_gate_up(const void* hidden, const void* top_k_index, int idx_dtype,
                                           const void* top_k_weights, int64_t top_k,
                                           const uint8_t* gate_up, const uint8_t* gate_up_sf,
                                           const void* gate_up_ts, int gate_up_ts_dtype,
                                           const uint8_t* down, const uint8_t* down_sf,
                                           const void* down_ts, int down_ts_dtype,
                                           int64_t num_experts, int64_t hidden_dim, int64_t inter_dim,
                                           void* out, void* workspace, size_t workspace_bytes, void* stream);
AEOQ_API int aeoq_moe_nvfp4_decode_down(const void* hidden, const void* top_k_index, int idx_dtype,
                                        const void* top_k_weights, int64_t top_k,
                                        const uint8_t* gate_up, const uint8_t* gate_up_sf,
                                        const void* gate_up_ts, int gate_up_ts_dtype,
                                        const uint8_t* down, const uint8_t* down_sf,
                                        const void* down_ts, int down_ts_dtype,
                                        int64_t num_experts, int64_t hidden_dim, int64_t inter_dim,
                                        void* out, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * One-token NVFP4 MoE expert forward as ONE persistent cooperative kernel
 * (same math and arguments as aeoq_moe_nvfp4_decode; replaces the same
 * reference function, modeling_nvfp4.py:132-186). Each SM copies its whole
 * weight slice to shared memory at launch; one grid barrier separates the
 * gate/up and down halves.
 * Workspace contract: aeoq_moe_nvfp4_decode_fused_workspace_size() bytes,
 * 256-aligned, whose first 256 bytes are zero before the first call; each
 * call leaves them zero again, so one workspace serves successive calls on
 * one stream (calls that overlap on the device must not share it).
 * aeoq_moe_nvfp4_decode_fused_supported() tells whether a shape fits
 * (hidden % 256 == 0, inter % 64 == 0, top_k <= 16, shared memory budget).
 * ------------------------------------------------------------------------ */
AEOQ_API int aeoq_moe_nvfp4_decode_fused_supported(int64_t top_k, int64_t hidden, int64_t inter);
AEOQ_API size_t aeoq_moe_nvfp4_decode_fused_workspace_size(int64_t top_k, int64_t hidden, int64_t inter);
AEOQ_API int aeoq_moe_nvfp4_decode_fused(const void* hidden, const void* top_k_index, int idx_dtype,
                                         const void* top_k_weights, int64_t top_k,
                                         const uint8_t* gate_up, const uint8_t* gate_up_sf,
                                         const void* gate_up_ts, int gate_up_ts_dtype,
                                         const uint8_t* down, const uint8_t* down_sf,
                                         const void* down_ts, int down_ts_dtype,
                                         int64_t num_experts, int64_t hidden_dim, int64_t inter_dim,
                                         void* out, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * One-token NVFP4 MoE expert forward on the tensor cores (two launches,
 * the second programmatically dependent on the first). Same math and
 * rounding points as aeoq_moe_nvfp4_decode (modeling_nvfp4.py:132-186) and
 * the same arguments (weight scales in the reference's [E][rows][K/16]
 * layout) plus an error word: a bounded wait that times out records a
 * nonzero code there. Workspace: *_tc_workspace_size() bytes, 256-aligned,
 * no initialization (calls that overlap on the device must not share it).
 * hidden % 256 == 0, inter % 64 == 0, top_k <= 8 (see *_supported).
 * ------------------------------------------------------------------------ */
AEOQ_API int aeoq_moe_nvfp4_decode_tc_supported(int64_t top_k, int64_t hidden, int64_t inter);
AEOQ_API size_t aeoq_moe_nvfp4_decode_tc_workspace_size(int64_t top_k, int64_t hidden, int64_t inter);
AEOQ_API int aeoq_moe_nvfp4_decode_tc(const void* hidden, const void* top_k_index, int idx_dtype,
                                      const void* top_k_weights, int64_t top_k, const uint8_t* gate_up,
                                      const uint8_t* gate_up_sf, const void* gate_up_ts, int gate_up_ts_dtype,
                                      const uint8_t* down, const uint8_t* down_sf, const void* down_ts,
                                      int down_ts_dtype, int64_t num_experts, int64_t hidden_dim, int64_t inter_dim,
                                      void* out, void* workspace, size_t workspace_bytes, int* err_word,
                                      void* stream);

/* ------------------------------------------------------------------------
 * One-token NVFP4 MoE expert forward streamed through ONE cooperative
 * launch (the module's one-token path where the tensor-core pair does not
 * cover the shape). Same math, rounding points and
 * arguments as aeoq_moe_nvfp4_decode (replaces the same reference function,
 * modeling_nvfp4.py:132-186) plus an error word. Work is split across the
 * SMs by bytes; each CTA requests every weight, scale and down row it needs
 * from HBM at entry (about 181 KB of shared memory per CTA at Gemma-4
 * shapes) and computes as the copies land; one grid barrier separates the
 * gate/up and down halves. The down scales are bulk-copied too, so the
 * weight scales must be 16-byte aligned.
 * Workspace contract: aeoq_moe_nvfp4_decode_stream_workspace_size() bytes,
 * 256-aligned, whose first 256 bytes are zero before the first call; each
 * call leaves them zero again, so one workspace serves successive calls on
 * one stream (calls that overlap on the device must not share it). A bounded
 * wait that times out records a nonzero code in *err_word.
 * aeoq_moe_nvfp4_decode_stream_supported(): hidden % 256 == 0, inter % 64
 * == 0, inter <= 1024, top_k <= 16, shared-memory budget.
 * ------------------------------------------------------------------------ */
AEOQ_API int aeoq_moe_nvfp4_decode_stream_supported(int64_t top_k, int64_t hidden, int64_t inter);
AEOQ_API size_t aeoq_moe_nvfp4_decode_stream_workspace_size(int64_t top_k, int64_t hidden, int64_t inter);
AEOQ_API int aeoq_moe_nvfp4_decode_stream(const void* hidden, const void* top_k_index, int idx_dtype,
                                          const void* top_k_weights, int64_t top_k, const uint8_t* gate_up,
                                          const uint8_t* gate_up_sf, const void* gate_up_ts, int gate_up_ts_dtype,
                                          const uint8_t* down, const uint8_t* down_sf, const void* down_ts,
                                          int down_ts_dtype, int64_t num_experts, int64_t hidden_dim,
                                          int64_t inter_dim, void* out, void* workspace, size_t workspace_bytes,
                                          int* err_word, void* stream);

/* ------------------------------------------------------------------------
 * Allocation-free one-token decode. No counterpart in the reference: it
 * exists for callers that cannot allocate device memory where they run the
 * expert forward (a serving runtime that pre-reserves all device memory, a
 * plugin without access to its host's allocator). Same arguments as
 * aeoq_moe_nvfp4_decode_fused minus the workspace; the scratch is a static
 * device array of aeoq_moe_nvfp4_decode_fused_noalloc_max_scratch() bytes
 * (128 KiB) per GPU, kept for the life of the process. Shapes needing more
 * are rejected with AEOQ_ERR_INVALID. The first call on a device looks the
 * array up (cudaGetSymbolAddress) and should precede any stream capture.
 * Calls that overlap on the device share the array and race. Allocates
 * nothing: no cudaMalloc/cudaFree, only a 256-byte cudaMemsetAsync of the
 * counters on the given stream.
 * ------------------------------------------------------------------------ */
AEOQ_API size_t aeoq_moe_nvfp4_decode_fused_noalloc_max_scratch(void);
AEOQ_API int aeoq_moe_nvfp4_decode_fused_noalloc(const void* hidden, const void* top_k_index, int idx_dtype,
                                                 const void* top_k_weights, int64_t top_k,
                                                 const uint8_t* gate_up, const uint8_t* gate_up_sf,
                                                 const void* gate_up_ts, int gate_up_ts_dtype,
                                                 const uint8_t* down, const uint8_t* down_sf,
                                                 const void* down_ts, int down_ts_dtype,
                                                 int64_t num_experts, int64_t hidden_dim, int64_t inter_dim,
                                                 void* out, void* stream);

/* ------------------------------------------------------------------------
 * Self-test of the device division every quantized bit depends on: counts
 * (into *mismatches, device memory, accumulated) the operand pairs of a
 * domain where the library's correctly rounded division differs from the
 * compiler's __fdiv_rn, and stores the first such (a, b, got, want) in
 * example[0..3] (device memory). Domains: 0 = every float dividend
 * significand x every bf16 divisor significand; 1 = every bf16 dividend
 * significand x every float divisor significand; 2 = 2^28 random pairs over
 * the full exponent range of the fast path; 3 = the NVFP4 block quantizer
 * (threshold form) against the reference's division-by-division formula on
 * 2^22 random and boundary-probing blocks (example holds ts and the 16
 * inputs of the first mismatching block, 17 floats). No counterpart in the
 * reference.
 * ------------------------------------------------------------------------ */
AEOQ_API int aeoq_selftest_div_rn(int domain, unsigned long long* mismatches, float* example, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* AEOQ_H_ */
