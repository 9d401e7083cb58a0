// Device-side MoE plumbing around the grouped tensor-core GEMMs.
//
// The reference builds per-expert token lists with one_hot / nonzero /
// torch.where in a Python loop over the hit experts (aeo_quant
// src/aeo_quant/bridges/gemma4/modeling_nvfp4.py:208-253, and
// bridges/gemma4/modeling.py:111-144 for FP8), which synchronizes the host
// once per layer. Here the same grouping is a counting sort on the device:
//
//   route_hist      per-expert pair counts (global atomics)
//   route_scatter   every CTA re-scans the E counts (cheap), then places each
//                   (token, slot) pair at grp_off[e] + atomic rank: rows of
//                   one expert become contiguous. The order inside an expert
//                   is arbitrary, which changes nothing: each row of a GEMM
//                   is computed independently and the combine sorts by id.
//   gather_rows     copies the quantized activation row of each pair's token
//                   into the expert-sorted buffer (packed FP4 + scales)
//   requant_rows    re-quantizes the GeGLU output rows with a per-expert
//                   tensor scale (prefill semantics, :239-244) or one shared
//                   scale (one-token semantics, :164-172)
//   combine         per token: its k weighted expert outputs, ordered by
//                   expert id and folded with a bf16 rounding after every add
//                   (index_add_ in expert order, :246-253), or summed in f32
//                   and rounded once (the one-token path, :181-186)
#include <algorithm>

#include "common.cuh"

namespace aeoq {

constexpr int kRouteThreads = 256;

__global__ void route_hist_kernel(const void* ids, int ids_dt, int64_t n_pairs, int E, int* cnt) {
  extern __shared__ int sh_cnt[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) sh_cnt[e] = 0;
  __syncthreads();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_pairs; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = load_index(ids, ids_dt, i);
    if (e >= 0 && e < E) atomicAdd(&sh_cnt[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    if (sh_cnt[e]) atomicAdd(&cnt[e], sh_cnt[e]);
}

// Exclusive scans of the counts (rows) and of the token tiles of size bn.
__device__ void scan_counts(const int* cnt, int E, int bn, int* grp_off, int* tile_off) {
  // E <= 1024: one thread per expert, block-wide scan through shared memory
  __shared__ int s_rows[1024 + 1], s_tiles[1024 + 1];
  const int t = threadIdx.x;
  for (int e = t; e < E; e += blockDim.x) {
    const int c = cnt[e];
    s_rows[e] = c;
    s_tiles[e] = (c + bn - 1) / bn;
  }
  __syncthreads();
  if (t == 0) {
    int r = 0, q = 0;
    for (int e = 0; e < E; ++e) {
      const int c = s_rows[e], d = s_tiles[e];
      s_rows[e] = r;
      s_tiles[e] = q;
      r += c;
      q += d;
    }
    s_rows[E] = r;
    s_tiles[E] = q;
  }
  __syncthreads();
  for (int e = t; e <= E; e += blockDim.x) {
    grp_off[e] = s_rows[e];
    tile_off[e] = s_tiles[e];
  }
  __syncthreads();
}

// pair i = t*k + j  ->  sorted row r; row_tok[r] = t, row_w[r] = w[t][j].
__global__ void route_scatter_kernel(const void* ids, int ids_dt, const __nv_bfloat16* topw, int64_t n_pairs, int k,
                                     int E, int bn, const int* cnt, int* fill, int* grp_off_out, int* tile_off_out,
                                     int* pair_row, int* row_tok, __nv_bfloat16* row_w, int* row_exp) {
  __shared__ int s_off[1024 + 1];
  __shared__ int s_dummy[1024 + 1];
  scan_counts(cnt, E, bn, s_off, s_dummy);
  if (blockIdx.x == 0) {
    for (int e = threadIdx.x; e <= E; e += blockDim.x) {
      grp_off_out[e] = s_off[e];
      tile_off_out[e] = s_dummy[e];
    }
  }
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_pairs; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = load_index(ids, ids_dt, i);
    if (e < 0 || e >= E) {
      pair_row[i] = -1;
      continue;
    }
    const int r = s_off[e] + atomicAdd(&fill[e], 1);
    pair_row[i] = r;
    row_tok[r] = (int)(i / k);
    row_w[r] = topw[i];
    row_exp[r] = (int)e;
  }
}

// Byte offset of (sorted row r, K-step kb) in the token-tile scale atoms of
// the grouped GEMM (tiles of tile_n rows per expert, see sf_atoms.cu).
__device__ __forceinline__ int64_t tile_atom_offset(int r, int64_t kb, int64_t kbc, const int* row_exp,
                                                    const int* grp_off, const int* tile_off, int tile_n) {
  const int e = row_exp[r];
  const int q = r - grp_off[e];
  const int64_t tile = tile_off[e] + q / tile_n;
  const int rit = q % tile_n;
  const int natoms = (tile_n + 127) / 128;
  const int rr = rit & 127;
  return ((tile * kbc + kb) * natoms + (rit >> 7)) * 512 + (rr & 31) * 16 + (rr >> 5) * 4;
}

// Copy packed rows of src (indexed by token) into sorted order; their scales
// go straight into the grouped GEMM's token-tile atoms.
__global__ void gather_rows_kernel(const uint8_t* __restrict__ src, const uint8_t* __restrict__ src_sf,
                                   const int* __restrict__ row_tok, const int* __restrict__ row_exp,
                                   const int* __restrict__ grp_off, const int* __restrict__ tile_off, int tile_n,
                                   const int* __restrict__ n_rows_ptr, int64_t row_bytes, int64_t sf_bytes,
                                   uint8_t* __restrict__ dst, uint8_t* __restrict__ dst_atoms) {
  const int n_rows = *n_rows_ptr;
  const int64_t v_row = row_bytes / 16;
  const int64_t kbc = sf_bytes / 4;
  for (int64_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
    const int t = row_tok[r];
    const uint4* s = reinterpret_cast<const uint4*>(src + (int64_t)t * row_bytes);
    uint4* d = reinterpret_cast<uint4*>(dst + r * row_bytes);
    for (int64_t i = threadIdx.x; i < v_row; i += blockDim.x) d[i] = s[i];
    const uint32_t* ss = reinterpret_cast<const uint32_t*>(src_sf + (int64_t)t * sf_bytes);
    for (int64_t kb = threadIdx.x; kb < kbc; kb += blockDim.x)
      *reinterpret_cast<uint32_t*>(dst_atoms + tile_atom_offset((int)r, kb, kbc, row_exp, grp_off, tile_off, tile_n)) =
          ss[kb];
  }
}

// Per-expert (or one shared) tensor scale from amax keys, then one 16-value
// block per thread. amax_key[e] holds the max |h| key of expert e's rows.
__global__ void requant_rows_kernel(const __nv_bfloat16* __restrict__ h, int64_t I, const int* __restrict__ row_exp,
                                    const int* __restrict__ grp_off, const int* __restrict__ tile_off, int tile_n,
                                    const int* __restrict__ n_rows_ptr, const uint32_t* __restrict__ amax_key, int E,
                                    int shared_scale, uint8_t* __restrict__ hq, uint8_t* __restrict__ hsf_atoms,
                                    float* __restrict__ ts_out) {
  const int n_rows = *n_rows_ptr;
  const int64_t bpr = I / 16;
  const int64_t nb = (int64_t)n_rows * bpr;
  uint32_t gkey = 0;
  if (shared_scale)
    for (int e = 0; e < E; ++e) gkey = max(gkey, amax_key[e]);
  if (blockIdx.x == 0)
    for (int e = threadIdx.x; e < E; e += blockDim.x)
      ts_out[e] = nvfp4_tensor_scale<AEOQ_BF16>(In<AEOQ_BF16>::key_to_f(shared_scale ? gkey : amax_key[e]));
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nb; b += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = b / bpr;
    const int e = row_exp[r];
    const float ts = nvfp4_tensor_scale<AEOQ_BF16>(In<AEOQ_BF16>::key_to_f(shared_scale ? gkey : amax_key[e]));
    float v[16];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const uint4 u = *reinterpret_cast<const uint4*>(h + 16 * b + 8 * q);
      const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[8 * q + j] = __bfloat162float(x[j]);
    }
    uint32_t w0, w1;
    const uint32_t sf = nvfp4_quant_block(v, ts, w0, w1);
    *reinterpret_cast<uint2*>(hq + 8 * b) = make_uint2(w0, w1);
    // block b of row r is scale column c = b % bpr: byte c % 4 of K-step c / 4
    const int64_t c = b - r * bpr;
    hsf_atoms[tile_atom_offset((int)r, c >> 2, bpr / 4, row_exp, grp_off, tile_off, tile_n) + (c & 3)] = (uint8_t)sf;
  }
}

// out[t][n]: fold the k expert outputs of token t in ascending expert order.
//   mode 0 (prefill / index_add_): acc = bf16(acc + c_j), starting from 0
//   mode 1 (one token):            bf16(sum_j c_j) in f32
__global__ void combine_kernel(const __nv_bfloat16* __restrict__ c_sorted, const int* __restrict__ pair_row,
                               const void* ids, int ids_dt, int64_t T, int k, int64_t H, int mode,
                               __nv_bfloat16* __restrict__ out) {
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    int rows[16];
    int64_t eids[16];
    int n = 0;
    for (int j = 0; j < k; ++j) {
      const int r = pair_row[t * k + j];
      if (r < 0) continue;
      const int64_t e = load_index(ids, ids_dt, t * k + j);
      int pos = n++;
      while (pos > 0 && eids[pos - 1] > e) {   // insertion sort by expert id
        eids[pos] = eids[pos - 1];
        rows[pos] = rows[pos - 1];
        --pos;
      }
      eids[pos] = e;
      rows[pos] = r;
    }
    for (int64_t c = threadIdx.x; c < H / 2; c += blockDim.x) {
      float a0 = 0.f, a1 = 0.f;
      for (int i = 0; i < n; ++i) {
        const __nv_bfloat162 v = reinterpret_cast<const __nv_bfloat162*>(c_sorted + (int64_t)rows[i] * H)[c];
        if (mode == 0) {
          a0 = bf16r(a0 + __bfloat162float(v.x));
          a1 = bf16r(a1 + __bfloat162float(v.y));
        } else {
          a0 += __bfloat162float(v.x);
          a1 += __bfloat162float(v.y);
        }
      }
      reinterpret_cast<__nv_bfloat162*>(out + t * H)[c] = __floats2bfloat162_rn(a0, a1);
    }
  }
}

}  // namespace aeoq

using namespace aeoq;

extern "C" int aeoq_moe_route(const void* top_k_index, int idx_dtype, const void* top_k_weights, int64_t T, int64_t k,
                              int64_t num_experts, int tile_n, int* cnt, int* fill, int* grp_off, int* tile_off,
                              int* pair_row, int* row_tok, void* row_w, int* row_exp, void* stream) {
  AEOQ_REQUIRE(num_experts >= 1 && num_experts <= 1024, AEOQ_ERR_INVALID, "moe_route: 1 <= num_experts <= 1024");
  AEOQ_REQUIRE(k >= 1 && k <= 16, AEOQ_ERR_INVALID, "moe_route: 1 <= top_k <= 16");
  AEOQ_REQUIRE(tile_n >= 1, AEOQ_ERR_INVALID, "moe_route: tile_n >= 1");
  AEOQ_REQUIRE(idx_dtype == AEOQ_I32 || idx_dtype == AEOQ_I64, AEOQ_ERR_INVALID, "moe_route: int32/int64 ids");
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t P = T * k;
  cudaError_t e = cudaMemsetAsync(cnt, 0, sizeof(int) * num_experts, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(fill, 0, sizeof(int) * num_experts, st);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(AEOQ_ERR_CUDA, "moe_route: memset: %s", cudaGetErrorString(e));
  }
  const int blocks = (int)std::min<int64_t>(std::max<int64_t>((P + kRouteThreads - 1) / kRouteThreads, 1), 148 * 4);
  route_hist_kernel<<<blocks, kRouteThreads, num_experts * sizeof(int), st>>>(top_k_index, idx_dtype, P,
                                                                               (int)num_experts, cnt);
  int rc = check_launch("route_hist_kernel");
  if (rc) return rc;
  route_scatter_kernel<<<blocks, kRouteThreads, 0, st>>>(top_k_index, idx_dtype,
                                                         reinterpret_cast<const __nv_bfloat16*>(top_k_weights), P,
                                                         (int)k, (int)num_experts, tile_n, cnt, fill, grp_off,
                                                         tile_off, pair_row, row_tok,
                                                         reinterpret_cast<__nv_bfloat16*>(row_w), row_exp);
  return check_launch("route_scatter_kernel");
}

extern "C" int aeoq_gather_rows(const uint8_t* src, const uint8_t* src_sf, const int* row_tok, const int* row_exp,
                                const int* grp_off, const int* tile_off, int tile_n, const int* n_rows,
                                int64_t max_rows, int64_t row_bytes, int64_t sf_bytes, uint8_t* dst,
                                uint8_t* dst_atoms, void* stream) {
  AEOQ_REQUIRE(row_bytes % 16 == 0 && sf_bytes % 4 == 0, AEOQ_ERR_INVALID,
               "gather_rows: row bytes must be a multiple of 16, scale bytes of 4");
  if (max_rows <= 0) return AEOQ_OK;
  const int blocks = (int)std::min<int64_t>(max_rows, 148 * 8);
  gather_rows_kernel<<<blocks, 128, 0, (cudaStream_t)stream>>>(src, src_sf, row_tok, row_exp, grp_off, tile_off,
                                                                tile_n, n_rows, row_bytes, sf_bytes, dst, dst_atoms);
  return check_launch("gather_rows_kernel");
}

extern "C" int aeoq_requant_rows(const void* h, int64_t I, const int* row_exp, const int* grp_off, const int* tile_off,
                                 int tile_n, const int* n_rows, int64_t max_rows, const uint32_t* amax_key,
                                 int64_t num_experts, int shared_scale, uint8_t* hq, uint8_t* hsf_atoms,
                                 float* ts_out, void* stream) {
  AEOQ_REQUIRE(I % 64 == 0, AEOQ_ERR_INVALID, "requant_rows: I must be a multiple of 64");
  const int64_t nb = std::max<int64_t>(max_rows * (I / 16), 1);
  const int blocks = (int)std::min<int64_t>((nb + 255) / 256, 148 * 8);
  requant_rows_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(reinterpret_cast<const __nv_bfloat16*>(h), I, row_exp,
                                                                 grp_off, tile_off, tile_n, n_rows, amax_key,
                                                                 (int)num_experts, shared_scale, hq, hsf_atoms, ts_out);
  return check_launch("requant_rows_kernel");
}

extern "C" int aeoq_moe_combine(const void* c_sorted, const int* pair_row, const void* top_k_index, int idx_dtype,
                                int64_t T, int64_t k, int64_t H, int mode, void* out, void* stream) {
  AEOQ_REQUIRE(k >= 1 && k <= 16 && H % 2 == 0, AEOQ_ERR_INVALID, "moe_combine: 1 <= k <= 16, even H");
  if (T <= 0) return AEOQ_OK;
  const int blocks = (int)std::min<int64_t>(T, 148 * 8);
  combine_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(reinterpret_cast<const __nv_bfloat16*>(c_sorted), pair_row,
                                                            top_k_index, idx_dtype, T, (int)k, H, mode,
                                                            reinterpret_cast<__nv_bfloat16*>(out));
  return check_launch("combine_kernel");
}
