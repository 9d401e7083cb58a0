// Scale-factor atoms for the tensor-core GEMMs.
//
// tcgen05.cp .32x128b.warpx4 moves one 512-byte "atom" into TMEM: the four
// UE4M3 scales (one K = 64 step) of 128 rows, row r at byte
// (r % 32) * 16 + (r / 32) * 4. The reference keeps scales row-major
// ([rows, K/16], src/aeo_quant/gpu/quant.py:174), which a TMA tile cannot
// turn into that order, so this file re-arranges them:
//
//  * weights, once per tensor: [group][tile of 128 rows][K/64][512 B], where
//    a tile is 128 consecutive rows, or for the fused GeGLU tiles 64 gate
//    rows n0.. and the 64 matching up rows I + n0.. of one expert;
//  * activations, per call: [token tile][K/64][ceil(BN/128)][512 B] for
//    token tiles of BN rows (rows past the end of a tile's rows are unused).
#include <algorithm>

#include "common.cuh"

namespace aeoq {

__device__ __forceinline__ uint32_t atom_byte(int rr) { return (uint32_t)((rr & 31) * 16 + (rr >> 5) * 4); }

// One thread per (group, tile, k-step, row-in-tile): copies 4 scale bytes.
__global__ void sf_to_atoms_kernel(const uint8_t* __restrict__ sf, int64_t groups, int64_t rows_per_group,
                                   int64_t kbc, int64_t geglu_inter, uint8_t* __restrict__ out) {
  const int64_t tiles = rows_per_group / 128;
  const int64_t total = groups * tiles * kbc * 128;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int rr = (int)(i & 127);
    const int64_t rest = i >> 7;
    const int64_t kb = rest % kbc;
    const int64_t gt = rest / kbc;   // group * tiles + tile
    const int64_t g = gt / tiles, t = gt - g * tiles;
    int64_t srow;
    if (geglu_inter) srow = rr < 64 ? 64 * t + rr : geglu_inter + 64 * t + (rr - 64);
    else srow = 128 * t + rr;
    const uint32_t v =
        *reinterpret_cast<const uint32_t*>(sf + (g * rows_per_group + srow) * (kbc * 4) + kb * 4);
    *reinterpret_cast<uint32_t*>(out + (gt * kbc + kb) * 512 + atom_byte(rr)) = v;
  }
}

// Activation rows (slot s = r / M, j = r % M) -> token-tile atoms. One warp
// per output atom (token tile, K step, 128-row group): lane l gathers the
// four scale words of rows l, l+32, l+64, l+96 of the group (zero past the
// slot's M rows) and writes its 16 bytes, so each atom is one contiguous
// 512-byte store.
__global__ void rows_to_tile_atoms_kernel(const uint8_t* __restrict__ sf, int64_t slots, int64_t M, int64_t kbc,
                                          int tile_n, uint8_t* __restrict__ out) {
  const int natoms = (tile_n + 127) / 128;
  const int64_t tps = (M + tile_n - 1) / tile_n;
  const int64_t total = slots * tps * kbc * natoms;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t w = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); w < total; w += warps) {
    const int a = (int)(w % natoms);
    const int64_t tk = w / natoms;              // tile * kbc + kb
    const int64_t kb = tk % kbc, tile = tk / kbc;
    const int64_t s = tile / tps, jt = tile - s * tps;
    uint32_t v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rit = 128 * a + 32 * i + lane;   // row in the token tile
      const int64_t j = jt * tile_n + rit;
      v[i] = (rit < tile_n && j < M) ? *reinterpret_cast<const uint32_t*>(sf + (s * M + j) * (kbc * 4) + kb * 4) : 0u;
    }
    *reinterpret_cast<uint4*>(out + w * 512 + 16 * lane) = make_uint4(v[0], v[1], v[2], v[3]);
  }
}

}  // namespace aeoq

using namespace aeoq;

extern "C" size_t aeoq_nvfp4_weight_atoms_size(int64_t rows, int64_t K) {
  return (size_t)((rows + 127) / 128) * (size_t)(K / 64) * 512;
}

extern "C" size_t aeoq_nvfp4_act_atoms_size(int64_t tiles, int64_t K, int tile_n) {
  return (size_t)tiles * (size_t)(K / 64) * (size_t)((tile_n + 127) / 128) * 512;
}

extern "C" int aeoq_nvfp4_sf_to_atoms(const uint8_t* sf, int64_t groups, int64_t rows_per_group, int64_t K,
                                      int64_t geglu_inter, uint8_t* out, void* stream) {
  AEOQ_REQUIRE(K % 64 == 0 && K > 0, AEOQ_ERR_INVALID, "sf_to_atoms: K must be a positive multiple of 64");
  AEOQ_REQUIRE(rows_per_group % 128 == 0, AEOQ_ERR_INVALID, "sf_to_atoms: rows per group must be a multiple of 128");
  AEOQ_REQUIRE(!geglu_inter || (2 * geglu_inter == rows_per_group && geglu_inter % 64 == 0), AEOQ_ERR_INVALID,
               "sf_to_atoms: GeGLU layout needs rows = 2 * I with I a multiple of 64");
  AEOQ_REQUIRE(sf && out && (uintptr_t)sf % 4 == 0 && (uintptr_t)out % 16 == 0, AEOQ_ERR_INVALID,
               "sf_to_atoms: null or misaligned pointer");
  const int64_t total = groups * (rows_per_group / 128) * (K / 64) * 128;
  if (total == 0) return AEOQ_OK;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  sf_to_atoms_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(sf, groups, rows_per_group, K / 64, geglu_inter,
                                                                out);
  return check_launch("sf_to_atoms_kernel");
}

extern "C" int aeoq_nvfp4_rows_to_tile_atoms(const uint8_t* sf, int64_t rows, int64_t M, int64_t K, int tile_n,
                                             uint8_t* out, void* stream) {
  AEOQ_REQUIRE(K % 64 == 0 && K > 0 && M > 0 && tile_n > 0, AEOQ_ERR_INVALID, "rows_to_tile_atoms: bad shape");
  AEOQ_REQUIRE(sf && out && (uintptr_t)sf % 4 == 0 && (uintptr_t)out % 16 == 0, AEOQ_ERR_INVALID,
               "rows_to_tile_atoms: null or misaligned pointer");
  const int64_t total = rows * (K / 64);
  if (total == 0) return AEOQ_OK;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  rows_to_tile_atoms_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(sf, rows / M, M, K / 64, tile_n, out);
  return check_launch("rows_to_tile_atoms_kernel");
}
