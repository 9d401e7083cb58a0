// Block-scaled NVFP4 GEMM on the 5th-generation tensor cores (tcgen05).
//
// Computes, for a set of (weight matrix, activation rows) problems,
//   C[row][n] = epilogue( sum_k A[n][k] * B[row][k] )      (A = weights)
// with A and B packed E2M1 (two per byte, high nibble = even k, the aeo_quant
// layout: src/aeo_quant/gpu/quant.py:180-183) and one UE4M3 scale per 16
// values along k, i.e. the contract of the reference's tl.dot_scaled kernels
// (src/aeo_quant/gpu/nvfp4_matmul.py:51-325). Both operands share the
// in-byte nibble order, so the hardware's (low nibble = even k) convention
// only permutes k inside each 16-value scale block, identically for A and B:
// the dot product is unchanged.
//
// Weight-stationary "swap AB" tiling: the MMA's M = 128 rows are weight
// rows (output features), its N = BN columns are activation rows (tokens),
// so one to a few hundred tokens per expert map onto N = 8..256 without
// padding M. Per CTA: one 128 x BN output tile, K in steps of 256 values
// (128 B rows, four MMAs of K = 64), a STAGES-deep shared-memory ring.
//
//   warp 0      producer: per stage one TMA tile of A and of B (128-byte
//               swizzle) and one bulk copy of each operand's scale atoms
//   warp 1      TMEM owner + MMA issuer (one thread): tcgen05.cp of the
//               stage's scale atoms, four tcgen05.mma, tcgen05.commit
//   warps 2-5   epilogue (tcgen05.ld -> alpha, GeGLU / weighting, cast, store)
//
// Scale factors travel pre-arranged in "atoms": 128 rows x 4 scales (one
// K = 64 step) = 512 B, row r at byte (r % 32) * 16 + (r / 32) * 4, the
// layout tcgen05.cp .32x128b.warpx4 broadcasts into TMEM. Weights' atoms are
// derived once per weight tensor (aeoq_nvfp4_sf_to_atoms); activations'
// atoms are written by the kernels that produce them, tile by tile.
//
// FP8 instance (kF8 = true): A and B are e4m3 codes (one per byte, K = 128
// values per 128-byte stage row, four tcgen05.mma kind::f8f6f4 of K = 32),
// no scale atoms; the epilogue applies the rowwise scales of the reference's
// torch._scaled_mm call (bridges/gemma4/modeling.py:101-108):
// y = (acc * sa[token]) * sb[weight row], f32.
//
// Every CTA loads its own operand tiles; no tile is shared across CTAs.
#include <cuda.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "sm100.cuh"

namespace aeoq {

constexpr int kEpiWarps = 8;                       // two per TMEM lane quadrant
constexpr int kTcThreads = 64 + 32 * kEpiWarps;    // producer, MMA issuer, epilogue
constexpr int kTcStages = 4;
constexpr int kKT = 256;            // K values per stage
constexpr int kKTBytes = kKT / 2;   // 128 B per row per stage

enum TcEpilogue : int { kEpiStore = 0, kEpiGeglu = 1, kEpiScaleRow = 2 };

struct TcParams {
  // problem
  int64_t n_out;        // weight rows per expert (N of the reference, multiple of 128)
  int64_t K;            // reduction length (multiple of 64)
  int64_t num_experts;
  // A (weights): tensor map over (num_experts * n_out) rows; scale atoms
  // [expert][n_out / 128][K / 64][512 B]
  const uint8_t* sfa;
  // B (activations): tensor map over b_rows rows; scale atoms
  // [token tile][K / 64][ceil(BN / 128)][512 B]
  const uint8_t* sfb;
  int64_t b_rows;       // rows addressable through the tensor map
  int64_t tiles_per_slot;   // mode 0 with per-slot activations
  // tiling of B rows into problems
  int mode;             // 0: slots (blockIdx.z = slot), 1: grouped by expert (device offsets)
  int64_t M;            // rows per slot (mode 0)
  int64_t b_slot_rows;  // row offset between slots' activations (0 = shared)
  const void* ids; int ids_dt;   // mode 0: slot -> expert (null = identity)
  const int* grp_off;   // mode 1: [E+1] row offsets of each expert's rows
  const int* tile_off;  // mode 1: [E+1] first token tile of each expert
  // epilogue
  int epi;
  const void* a_ts; int a_ts_dt;          // alpha = f32(*a_ts) * f32(*w_ts) (kEpiStore / kEpiGeglu)
  const void* w_ts; int w_ts_dt;
  const float* grp_alpha_ts;              // kEpiScaleRow: per-expert activation scale (f32), times w_ts
  const __nv_bfloat16* row_w;             // kEpiScaleRow: per-row weight (bf16)
  void* c; int c_dt;                      // output
  int64_t ldc;                            // bytes per output row
  int64_t c_slot_stride;                  // bytes between slots (mode 0)
  uint32_t* grp_amax;                     // kEpiGeglu: per-expert |h| max key (atomicMax)
  const float* sa_rows;                   // FP8: per activation (B) row scale, f32
  const float* sb_rows;                   // FP8: per weight row scale, f32 [num_experts * n_out]
  int tiles_x, tiles_y, tiles_z;          // persistent kernel: tile grid (mode 1: tiles_y read on device)
  int* err;                               // device error word (bounded waits)
};


constexpr int kTcMaxStages = 8;
struct TcSmem {
  uint64_t full[kTcMaxStages];
  uint64_t empty[kTcMaxStages];
  uint64_t accum;
  uint32_t tmem_base;
  float colscale[256];   // FP8: the tile's activation row scales
};

template <int BN, bool kF8 = false>
struct TcLayout {
  static constexpr int kSfbAtoms = (BN + 127) / 128;
  static constexpr size_t kA = 128 * kKTBytes;             // 16 KB
  static constexpr size_t kB = (size_t)BN * kKTBytes;
  static constexpr size_t kSfa = kF8 ? 0 : 4 * 512;
  static constexpr size_t kSfb = kF8 ? 0 : (size_t)4 * 512 * kSfbAtoms;
  static constexpr size_t kStage = kA + kB + kSfa + kSfb;
  // Tiles up to 128 tokens wide run two CTAs per SM (half the shared memory
  // and at most 256 TMEM columns each), so one CTA's epilogue overlaps the
  // other's main loop; wider tiles take the whole SM.
  static constexpr int kCtasPerSm = (BN <= 128) ? 2 : 1;
  // two CTAs: 2 x (kBytes + 1 KB reserved) within the SM's 228 KB
  static constexpr size_t kBudget =
      kCtasPerSm == 2 ? (113 * 1024 - 1024 - sizeof(TcSmem) - 64) : (220 * 1024 - 1280 - sizeof(TcSmem));
  // as many stages as the budget holds (at most 8)
  static constexpr int kStages = (int)(kBudget / kStage) < kTcMaxStages ? (int)(kBudget / kStage) : kTcMaxStages;
  // The epilogue reuses the stage ring, idle once the accumulator is
  // complete, for the GeGLU exchange of the up half (64 x BN f32).
  // row pitch BN + 1 words: the 32 lanes of a warp (32 rows) hit 32 banks
  static constexpr size_t kXchg = 64 * (size_t)(BN + 1) * 4;
  static_assert(kXchg <= kStages * kStage, "the GeGLU exchange must fit in the stage ring");
  static constexpr size_t kBytes = 1024 + kStages * kStage + sizeof(TcSmem) + 64;
  static constexpr uint32_t kTmemCols =
      kF8 ? (BN <= 32 ? 32u : (uint32_t)BN) : ((BN + 32 * kSfbAtoms + 16 <= 256) ? 256u : 512u);
  static_assert(kCtasPerSm == 1 || kTmemCols <= 256, "two CTAs per SM need at most 256 TMEM columns each");
  static constexpr uint32_t kSfaCol = BN;                  // 16 columns
  static constexpr uint32_t kSfbCol = BN + 16;             // 16 * kSfbAtoms columns
};

// Resolve this CTA's problem: expert, first activation row, valid rows.
struct TileInfo {
  int64_t expert, b_row0, c_row0, tile;
  int n_valid;
  int64_t slot;
  bool active;
};

template <int BN>
__device__ __forceinline__ TileInfo resolve_tile_at(const TcParams& p, int y_tile, int z_slot,
                                                    const int* tile_off = nullptr, const int* grp_off = nullptr) {
  TileInfo t{};
  if (p.mode == 0) {
    const int64_t s = z_slot;
    const int64_t tb = (int64_t)y_tile * BN;
    t.slot = s;
    t.expert = p.ids ? load_index(p.ids, p.ids_dt, s) : s;
    t.b_row0 = s * p.b_slot_rows + tb;
    t.c_row0 = tb;
    t.tile = (p.b_slot_rows ? s * p.tiles_per_slot : 0) + y_tile;
    t.n_valid = (int)min((int64_t)BN, p.M - tb);
    t.active = t.n_valid > 0;
  } else {
    const int y = y_tile;
    const int* toff = tile_off ? tile_off : p.tile_off;
    const int* goff = grp_off ? grp_off : p.grp_off;
    const int E = (int)p.num_experts;
    if (y >= toff[E]) {
      t.active = false;
      return t;
    }
    int lo = 0, hi = E;   // largest e with tile_off[e] <= y
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (toff[mid] <= y) lo = mid; else hi = mid;
    }
    while (lo < E - 1 && toff[lo + 1] <= y) ++lo;
    t.expert = lo;
    t.tile = y;
    const int64_t tb = (int64_t)(y - toff[lo]) * BN;
    t.b_row0 = goff[lo] + tb;
    t.c_row0 = t.b_row0;
    t.n_valid = (int)min((int64_t)BN, (int64_t)(goff[lo + 1] - goff[lo]) - tb);
    t.slot = 0;
    t.active = t.n_valid > 0;
  }
  if (t.expert < 0 || t.expert >= p.num_experts) t.active = false;
  return t;
}

template <int BN>
__device__ __forceinline__ TileInfo resolve_tile(const TcParams& p) {
  return resolve_tile_at<BN>(p, (int)blockIdx.y, (int)blockIdx.z);
}

// min(BN, 32) accumulator columns of this thread's TMEM lane, one wait.
template <int BN>
__device__ __forceinline__ void tmem_cols(uint32_t taddr, float (&v)[32]) {
  if constexpr (BN >= 32) {
    uint32_t r[32];
    sm100::tmem_ld32_nowait(taddr, r);
    sm100::tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
  } else {
    float w[16];
    sm100::tmem_ld16(taddr, w);   // reads 16 columns; only BN of them are used
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = w[i];
  }
}

// Stores 8 tokens x the warp's 32 output columns as bf16. On entry lane L
// holds column L's values for the 8 tokens in y[]; an 8x8 transpose inside
// each group of 8 lanes (three butterfly stages of shuffles) leaves lane
// 8g + i with token i's values for columns 8g .. 8g+7, written as one
// 16-byte store. row0 = output of token 0, column 0 of the warp; tokens >=
// n_ok are not written.
__device__ __forceinline__ void store_8tok_bf16(float (&y)[8], char* row0, int64_t ldc, int n_ok, int lane) {
#pragma unroll
  for (int s = 4; s >= 1; s >>= 1) {
    const bool up = (lane & s) != 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j & s) continue;
      const float send = up ? y[j] : y[j | s];
      const float recv = __shfl_xor_sync(0xffffffffu, send, s);
      if (up) y[j] = recv; else y[j | s] = recv;
    }
  }
  const int i = lane & 7, g = lane >> 3;
  if (i < n_ok) {
    __align__(16) __nv_bfloat16 o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = __float2bfloat16_rn(y[j]);
    *reinterpret_cast<uint4*>(row0 + i * ldc + 16 * g) = *reinterpret_cast<const uint4*>(o);
  }
}

// N (8, 16, 32 or 64) accumulator columns of this thread's TMEM lane, one wait.
template <int N, int VN>
__device__ __forceinline__ void tmem_chunk(uint32_t taddr, float (&v)[VN]) {
  if constexpr (N == 64) {
    uint32_t r0[32], r1[32];
    sm100::tmem_ld32_nowait(taddr, r0);
    sm100::tmem_ld32_nowait(taddr + 32, r1);
    sm100::tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      v[i] = __uint_as_float(r0[i]);
      v[32 + i] = __uint_as_float(r1[i]);
    }
  } else if constexpr (N == 32) {
    uint32_t r[32];
    sm100::tmem_ld32_nowait(taddr, r);
    sm100::tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
  } else {
    float w[16];
    sm100::tmem_ld16(taddr, w);   // reads 16 columns; only N of them are used
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = w[i];
  }
}

template <int BN, bool kF8>
__global__ void __launch_bounds__(kTcThreads, (BN <= 128) ? 2 : 1) nvfp4_tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                      const __grid_constant__ CUtensorMap tmB,
                                                                      const TcParams p) {
  using L = TcLayout<BN, kF8>;
  constexpr int kStepK = kF8 ? 32 : 64;      // K values per MMA (32 bytes of a row)
  extern __shared__ __align__(1024) uint8_t dsmem[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~uintptr_t(1023));
  uint8_t* stage0 = base;
  float* xchg = reinterpret_cast<float*>(base);   // epilogue only (stage ring idle by then)
  TcSmem* sh = reinterpret_cast<TcSmem*>(base + L::kStages * L::kStage);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const TileInfo ti = resolve_tile<BN>(p);
  if (!ti.active) return;   // whole CTA exits together before any sync
  const int64_t m_tile = blockIdx.x;
  const bool geglu = (p.epi == kEpiGeglu);
  // A rows of this tile: 128 consecutive weight rows, or for GeGLU 64 gate
  // rows (n0..n0+63) and the matching 64 up rows (n0 + n_out/2 ...).
  const int64_t a_row_base = ti.expert * p.n_out;
  const int num_kt = (int)((p.K + 4 * kStepK - 1) / (4 * kStepK));
  const int kb_total = (int)(p.K / kStepK);

  auto stA = [&](int s) { return stage0 + s * L::kStage; };
  auto stB = [&](int s) { return stage0 + s * L::kStage + L::kA; };
  auto stSFA = [&](int s) { return stage0 + s * L::kStage + L::kA + L::kB; };
  auto stSFB = [&](int s) { return stage0 + s * L::kStage + L::kA + L::kB + L::kSfa; };

  if (tid == 0) {
    for (int s = 0; s < L::kStages; ++s) {
      sm100::mbar_init(&sh->full[s], 1);       // producer arrival + transaction bytes
      sm100::mbar_init(&sh->empty[s], 1);      // tcgen05.commit
    }
    sm100::mbar_init(&sh->accum, 1);
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tmA);
    sm100::prefetch_tmap(&tmB);
  }
  if (warp == 1) sm100::tmem_alloc(&sh->tmem_base, L::kTmemCols);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  // ------------------------------------------------------------ producers
  // Each ring slot's copies are split by operand: request r = 4 * slot + op
  // (op 0 the A tile, which also posts the stage's expected bytes, 1 the B
  // tile, 2 and 3 the two scale-atom blocks; FP8 has ops 0 and 1) is issued
  // by producer r % kProducers (warp 0 and the epilogue warps, idle until
  // the accumulator is complete). A producer issues every use of its
  // requests in order, so each parity wait on a slot's empty barrier refers
  // to the previous use of that slot. One warp's copies complete one after
  // another, so spreading them over many warps multiplies the fill rate.
  // (A copy may complete before the stage's expected bytes are posted; the
  // barrier's transaction count then dips below zero until they are.)
  constexpr int kProducers = 1 + kEpiWarps;
  constexpr int kOps = kF8 ? 2 : 4;
  const int pidx = warp == 0 ? 0 : warp - 1;   // warps 2.. -> 1..
  if (warp != 1) {
    const bool leader = sm100::elect_one();
    const int64_t m_tiles = p.n_out / 128;
    const uint8_t* sfa_base = p.sfa + ((ti.expert * m_tiles + m_tile) * kb_total) * 512;
    const uint8_t* sfb_base = p.sfb + (ti.tile * kb_total) * (size_t)L::kSfbAtoms * 512;
    for (int kt = 0; kt < num_kt; ++kt) {
      const int s = kt % L::kStages;
      const uint32_t ph = (kt / L::kStages) & 1;
      const int nkb = min(4, kb_total - kt * 4);
      const uint32_t sfa_bytes = kF8 ? 0u : (uint32_t)nkb * 512;
      const uint32_t sfb_bytes = kF8 ? 0u : (uint32_t)nkb * L::kSfbAtoms * 512;
      const int32_t x = kt * kKTBytes;
      for (int op = 0; op < kOps; ++op) {
        if ((kOps * s + op) % kProducers != pidx) continue;
        if (!sm100::mbar_wait(&sh->empty[s], ph ^ 1, p.err, 11)) { kt = num_kt; break; }
        if (leader) {
          if (op == 0) {
            sm100::mbar_arrive_expect_tx(&sh->full[s], (uint32_t)(L::kA + L::kB) + sfa_bytes + sfb_bytes);
            if (geglu) {
              const int64_t n0 = m_tile * 64;
              sm100::tma_load_2d(stA(s), &tmA, x, (int32_t)(a_row_base + n0), &sh->full[s]);
              sm100::tma_load_2d(stA(s) + 64 * kKTBytes, &tmA, x, (int32_t)(a_row_base + p.n_out / 2 + n0),
                                 &sh->full[s]);
            } else {
              sm100::tma_load_2d(stA(s), &tmA, x, (int32_t)(a_row_base + m_tile * 128), &sh->full[s]);
            }
          } else if (op == 1) {
            sm100::tma_load_2d(stB(s), &tmB, x, (int32_t)ti.b_row0, &sh->full[s]);
          } else if constexpr (!kF8) {
            if (op == 2) bulk_g2s(stSFA(s), sfa_base + (size_t)kt * 4 * 512, sfa_bytes, &sh->full[s]);
            else bulk_g2s(stSFB(s), sfb_base + (size_t)kt * 4 * L::kSfbAtoms * 512, sfb_bytes, &sh->full[s]);
          }
        }
        __syncwarp();
      }
    }
  }
  if (warp == 0) {
    // producer only
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    {
      const bool leader = sm100::elect_one();
      const uint32_t idesc = kF8 ? sm100::idesc_f8(BN) : sm100::idesc_nvf4(BN);
      for (int kt = 0; kt < num_kt; ++kt) {
        const int s = kt % L::kStages;
        const uint32_t ph = (kt / L::kStages) & 1;
        if (!sm100::mbar_wait(&sh->full[s], ph, p.err, 12)) break;
        sm100::tc_fence_after();
        const int nkb = min(4, kb_total - kt * 4);
        if (!kF8 && leader)
        for (int kb = 0; kb < nkb; ++kb) {
          sm100::tc_cp_32x128b_warpx4(tmem + L::kSfaCol + 4 * kb, sm100::sdesc_sf_atom(sm100::smem_u32(stSFA(s) + kb * 512)));
#pragma unroll
          for (int a = 0; a < L::kSfbAtoms; ++a)
            sm100::tc_cp_32x128b_warpx4(tmem + L::kSfbCol + 4 * (kb * L::kSfbAtoms + a),
                                        sm100::sdesc_sf_atom(sm100::smem_u32(stSFB(s) + (kb * L::kSfbAtoms + a) * 512)));
        }
        if (leader)
        for (int kb = 0; kb < nkb; ++kb) {
          const uint64_t ad = sm100::sdesc_k_sw128(sm100::smem_u32(stA(s)) + kb * 32);
          const uint64_t bd = sm100::sdesc_k_sw128(sm100::smem_u32(stB(s)) + kb * 32);
          if constexpr (kF8)
            sm100::tc_mma_f8(tmem, ad, bd, idesc, (kt | kb) ? 1u : 0u);
          else
            sm100::tc_mma_nvf4(tmem, ad, bd, idesc, tmem + L::kSfaCol + 4 * kb,
                               tmem + L::kSfbCol + 4 * kb * L::kSfbAtoms, (kt | kb) ? 1u : 0u);
        }
        if (leader) sm100::tc_commit(&sh->empty[s]);
        __syncwarp();
      }
      if (leader) sm100::tc_commit(&sh->accum);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;            // TMEM lane quadrant this warp may access
    const int row = 32 * q + lane;     // accumulator row = weight row in the tile
    // the two warps of a quadrant split the tile's tokens
    constexpr int kHalf = BN >= 16 ? BN / 2 : BN;
    const int hseg = (warp - 2) >> 2;
    const int tbeg = hseg * kHalf, tend = min(BN, tbeg + kHalf);
    // Scales, read while the main loop runs. NVFP4: one alpha per tile.
    // FP8: this row's weight scale (GeGLU tiles: gate rows n0.., up rows
    // n_out/2 + n0..) and the tile's activation row scales in shared memory.
    float alpha = 1.0f;
    float* colscale = sh->colscale;
    if constexpr (kF8) {
      const int64_t wrow = geglu ? (row < 64 ? m_tile * 64 + row : p.n_out / 2 + m_tile * 64 + (row - 64))
                                 : m_tile * 128 + row;
      alpha = p.sb_rows[ti.expert * p.n_out + wrow];
      for (int t = tid - 64; t < BN; t += 32 * kEpiWarps) colscale[t] = t < ti.n_valid ? p.sa_rows[ti.b_row0 + t] : 0.0f;
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory");
    } else {
      if (p.epi == kEpiScaleRow) alpha = p.grp_alpha_ts[ti.expert] * load_scalar_f(p.w_ts, p.w_ts_dt);
      else alpha = load_scalar_f(p.a_ts, p.a_ts_dt) * load_scalar_f(p.w_ts, p.w_ts_dt);
    }
    // accumulator -> f32 value of output (row, token t)
    auto scaled = [&](float acc, int t) { return kF8 ? (acc * colscale[t]) * alpha : acc * alpha; };
    const bool ok = sm100::mbar_wait(&sh->accum, 0, p.err, 14);
    sm100::tc_fence_after();
    char* cbase = reinterpret_cast<char*>(p.c) + ti.slot * p.c_slot_stride;
    uint32_t hkey = 0;
    const int ncol = geglu ? 64 : 128;
    const int es = (p.epi == kEpiStore && p.c_dt == AEOQ_F32) ? 4 : 2;
    // Stores go straight from registers. A thread owns one output column
    // (its weight row); bf16 outputs are transposed in 8-token groups so each
    // lane writes 8 consecutive columns of one token (16 bytes); f32 outputs
    // are written per element (a warp covers 128 contiguous bytes).
    const int64_t col_w = (int64_t)m_tile * ncol + 32 * (q & (geglu ? 1 : 3));   // warp's first column
    char* cwarp = cbase + ti.c_row0 * p.ldc + col_w * es;
    constexpr int kChunk = kHalf < 32 ? kHalf : 32;   // columns per TMEM wait
    const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
    if (p.epi != kEpiGeglu) {
      for (int c0 = tbeg; c0 < tend; c0 += kChunk) {
        float v[kChunk < 16 ? 16 : kChunk];
        tmem_chunk<kChunk>(tq + (uint32_t)c0, v);
#pragma unroll
        for (int g8 = 0; g8 < kChunk; g8 += 8) {
          const int t0 = c0 + g8;
          float y[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int t = t0 + j;
            float val = (t < ti.n_valid) ? scaled(v[g8 + j], t) : 0.0f;
            if (p.epi == kEpiScaleRow && t < ti.n_valid) val = bf16r(val) * __bfloat162float(p.row_w[ti.c_row0 + t]);
            y[j] = val;
          }
          if (!ok) continue;
          if (es == 2) {
            store_8tok_bf16(y, cwarp + t0 * p.ldc, p.ldc, ti.n_valid - t0, lane);
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              if (t0 + j < ti.n_valid) *reinterpret_cast<float*>(cwarp + (t0 + j) * p.ldc + 4 * lane) = y[j];
          }
        }
      }
    } else {
      // GeGLU: rows 64..127 (up) hand bf16(alpha*acc) to rows 0..63 (gate)
      if (row >= 64) {
        for (int c0 = tbeg; c0 < tend; c0 += kChunk) {
          float v[kChunk < 16 ? 16 : kChunk];
          tmem_chunk<kChunk>(tq + (uint32_t)c0, v);
#pragma unroll
          for (int j = 0; j < kChunk; ++j) xchg[(row - 64) * (BN + 1) + c0 + j] = bf16r(scaled(v[j], c0 + j));
        }
      }
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory");
      if (q < 2) {
        for (int c0 = tbeg; c0 < tend; c0 += kChunk) {
          float v[kChunk < 16 ? 16 : kChunk];
          tmem_chunk<kChunk>(tq + (uint32_t)c0, v);
#pragma unroll
          for (int g8 = 0; g8 < kChunk; g8 += 8) {
            const int t0 = c0 + g8;
            float y[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int t = t0 + j;
              float hvf = 0.0f;
              if (t < ti.n_valid) {
                const float gv = bf16r(scaled(v[g8 + j], t));
                const float u = xchg[row * (BN + 1) + t];
                const __nv_bfloat16 hv = __float2bfloat16_rn(bf16r(gelu_tanh(gv)) * u);
                hkey = max(hkey, In<AEOQ_BF16>::abs_key(hv));
                hvf = __bfloat162float(hv);
              }
              y[j] = hvf;
            }
            if (ok) store_8tok_bf16(y, cwarp + t0 * p.ldc, p.ldc, ti.n_valid - t0, lane);
          }
        }
      }
    }
    if (p.epi == kEpiGeglu && p.grp_amax) {
      hkey = warp_umax(hkey);
      if (lane == 0 && hkey) atomicMax(p.grp_amax + ti.expert, hkey);
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, L::kTmemCols);
  }
}


int make_tmap(CUtensorMap* m, const void* ptr, int64_t rows, int64_t row_bytes, int64_t ld, int box_rows);

// ---------------------------------------------------------------- persistent
// Persistent variant: one CTA per SM walks a static tile schedule (weight
// tiles fastest, so the CTAs working at the same time share token tiles in
// L2). The producers run ahead across tile boundaries, and the accumulator
// is double-buffered in TMEM: the epilogue of tile i (eight warps, two per
// lane quadrant) overlaps the main loop of tile i + 1.
//   warps 0, 2, 3   producers (ring slot s is filled by producer s % 3)
//   warp 1          TMEM owner + MMA issuer
//   warps 4 .. 19   epilogue (four per TMEM lane quadrant)
constexpr int kPEpiWarps = 16;
constexpr int kPMaxExperts = 256;   // grouped offsets held in shared memory up to this many experts
constexpr int kPThreads = 128 + 32 * kPEpiWarps;
constexpr int kPProducers = 3;

template <int BN, bool kF8>
struct PLayout {
  static constexpr int kSfbAtoms = (BN + 127) / 128;
  static constexpr size_t kA = 128 * kKTBytes;
  static constexpr size_t kB = (size_t)BN * kKTBytes;
  static constexpr size_t kSfa = kF8 ? 0 : 4 * 512;
  static constexpr size_t kSfb = kF8 ? 0 : (size_t)4 * 512 * kSfbAtoms;
  static constexpr size_t kStage = kA + kB + kSfa + kSfb;
  // GeGLU up half, bf16, row pitch BN + 2 (an odd number of words: the 32
  // lanes of a warp, 32 rows, hit 32 banks)
  static constexpr int kXs = BN + 2;
  static constexpr size_t kXchg = 64 * (size_t)kXs * 2;
  struct Smem {
    uint64_t full[kTcMaxStages], empty[kTcMaxStages], acc_full[2], acc_empty[2];
    uint32_t tmem_base;
    float colscale[256];
    float roww[256];       // kEpiScaleRow: the tile's per-row weights
    // grouped mode: the expert tile and row offsets, so every role resolves
    // a tile from shared memory instead of a chain of dependent L2 loads
    int tile_off[kPMaxExperts + 1];
    int grp_off[kPMaxExperts + 1];
  };
  static constexpr size_t kFixed = 1024 + kXchg + sizeof(Smem) + 64;
  static constexpr int kStages =
      (int)((227 * 1024 - kFixed) / kStage) < kTcMaxStages ? (int)((227 * 1024 - kFixed) / kStage) : kTcMaxStages;
  static_assert(kStages >= 2, "persistent tile too wide for the shared-memory ring");
  static constexpr size_t kBytes = 1024 + kStages * kStage + kXchg + sizeof(Smem) + 64;
  static constexpr uint32_t kAccStride = (uint32_t)((BN + 31) / 32 * 32);
  static constexpr uint32_t kSfaCol = 2 * kAccStride;
  static constexpr uint32_t kSfbCol = kSfaCol + 16;
  static_assert(kSfbCol + 16 * kSfbAtoms <= 512, "two accumulators and the scale columns must fit in TMEM");
  static constexpr uint32_t kTmemCols = (kF8 ? 2 * kAccStride : kSfbCol + 16 * kSfbAtoms) <= 256 ? 256u : 512u;
};

template <int BN, bool kF8>
__global__ void __launch_bounds__(kPThreads, 1) tc_gemm_persistent_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                          const __grid_constant__ CUtensorMap tmB,
                                                                          const TcParams p) {
  using L = PLayout<BN, kF8>;
  using Smem = typename L::Smem;
  constexpr int kStepK = kF8 ? 32 : 64;
  extern __shared__ __align__(1024) uint8_t dsmem[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~uintptr_t(1023));
  uint8_t* stage0 = base;
  __nv_bfloat16* xchg = reinterpret_cast<__nv_bfloat16*>(base + L::kStages * L::kStage);
  Smem* sh = reinterpret_cast<Smem*>(base + L::kStages * L::kStage + L::kXchg);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool geglu = (p.epi == kEpiGeglu);
  const int num_kt = (int)((p.K + 4 * kStepK - 1) / (4 * kStepK));
  const int kb_total = (int)(p.K / kStepK);
  auto stA = [&](int s) { return stage0 + s * L::kStage; };
  auto stB = [&](int s) { return stage0 + s * L::kStage + L::kA; };
  auto stSFA = [&](int s) { return stage0 + s * L::kStage + L::kA + L::kB; };
  auto stSFB = [&](int s) { return stage0 + s * L::kStage + L::kA + L::kB + L::kSfa; };

  // the tile schedule: tile t -> (weight tile t % tiles_x, token tile, slot)
  const bool offs_smem = p.mode == 1 && p.num_experts <= kPMaxExperts;
  if (offs_smem) {
    for (int i = tid; i <= (int)p.num_experts; i += kPThreads) {
      sh->tile_off[i] = p.tile_off[i];
      sh->grp_off[i] = p.grp_off[i];
    }
    __syncthreads();
  }
  const int* toff = offs_smem ? sh->tile_off : nullptr;
  const int* goff = offs_smem ? sh->grp_off : nullptr;
  const int tx = p.tiles_x;
  const int ty = p.mode == 1 ? (offs_smem ? sh->tile_off[p.num_experts] : p.tile_off[p.num_experts]) : p.tiles_y;
  const int64_t total = (int64_t)tx * ty * (p.mode == 1 ? 1 : p.tiles_z);
  auto tile_of = [&](int64_t t, int64_t& m_tile) {
    m_tile = t % tx;
    const int64_t r = t / tx;
    return p.mode == 1 ? resolve_tile_at<BN>(p, (int)r, 0, toff, goff)
                       : resolve_tile_at<BN>(p, (int)(r % ty), (int)(r / ty));
  };

  if (tid == 0) {
    for (int s = 0; s < L::kStages; ++s) {
      sm100::mbar_init(&sh->full[s], 1);
      sm100::mbar_init(&sh->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&sh->acc_full[b], 1);
      sm100::mbar_init(&sh->acc_empty[b], kPEpiWarps);
    }
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tmA);
    sm100::prefetch_tmap(&tmB);
  }
  if (warp == 1) sm100::tmem_alloc(&sh->tmem_base, L::kTmemCols);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (warp == 0 || warp == 2 || warp == 3) {
    // ------------------------------------------------------------ producers
    const int pidx = warp == 0 ? 0 : warp - 1;
    const bool leader = sm100::elect_one();
    int64_t g = 0;   // stage counter over all of this CTA's tiles
    bool alive = true;
    for (int64_t t = blockIdx.x; t < total && alive; t += gridDim.x) {
      int64_t m_tile;
      const TileInfo ti = tile_of(t, m_tile);
      if (!ti.active) continue;
      const int64_t a_row_base = ti.expert * p.n_out;
      const int64_t m_tiles = p.n_out / 128;
      const uint8_t* sfa_base = kF8 ? nullptr : p.sfa + ((ti.expert * m_tiles + m_tile) * kb_total) * 512;
      const uint8_t* sfb_base = kF8 ? nullptr : p.sfb + (ti.tile * kb_total) * (size_t)L::kSfbAtoms * 512;
      for (int kt = 0; kt < num_kt; ++kt, ++g) {
        const int s = (int)(g % L::kStages);
        if (s % kPProducers != pidx) continue;
        const uint32_t ph = (uint32_t)((g / L::kStages) & 1);
        if (!sm100::mbar_wait(&sh->empty[s], ph ^ 1, p.err, 61)) { alive = false; break; }
        const int nkb = min(4, kb_total - kt * 4);
        const uint32_t sfa_bytes = kF8 ? 0u : (uint32_t)nkb * 512;
        const uint32_t sfb_bytes = kF8 ? 0u : (uint32_t)nkb * L::kSfbAtoms * 512;
        const int32_t x = kt * kKTBytes;
        if (leader) {
          sm100::mbar_arrive_expect_tx(&sh->full[s], (uint32_t)(L::kA + L::kB) + sfa_bytes + sfb_bytes);
          if constexpr (!kF8) {
            bulk_g2s(stSFA(s), sfa_base + (size_t)kt * 4 * 512, sfa_bytes, &sh->full[s]);
            bulk_g2s(stSFB(s), sfb_base + (size_t)kt * 4 * L::kSfbAtoms * 512, sfb_bytes, &sh->full[s]);
          }
          if (geglu) {
            const int64_t n0 = m_tile * 64;
            sm100::tma_load_2d(stA(s), &tmA, x, (int32_t)(a_row_base + n0), &sh->full[s]);
            sm100::tma_load_2d(stA(s) + 64 * kKTBytes, &tmA, x, (int32_t)(a_row_base + p.n_out / 2 + n0),
                               &sh->full[s]);
          } else {
            sm100::tma_load_2d(stA(s), &tmA, x, (int32_t)(a_row_base + m_tile * 128), &sh->full[s]);
          }
          sm100::tma_load_2d(stB(s), &tmB, x, (int32_t)ti.b_row0, &sh->full[s]);
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const bool leader = sm100::elect_one();
    const uint32_t idesc = kF8 ? sm100::idesc_f8(BN) : sm100::idesc_nvf4(BN);
    int64_t g = 0;
    int it = 0;
    bool alive = true;
    for (int64_t t = blockIdx.x; t < total && alive; t += gridDim.x) {
      int64_t m_tile;
      const TileInfo ti = tile_of(t, m_tile);
      if (!ti.active) continue;
      const int b = it & 1;
      const uint32_t accp = (uint32_t)((it >> 1) & 1);
      if (!sm100::mbar_wait(&sh->acc_empty[b], accp ^ 1, p.err, 62)) break;
      sm100::tc_fence_after();
      const uint32_t dcol = tmem + (uint32_t)b * L::kAccStride;
      for (int kt = 0; kt < num_kt; ++kt, ++g) {
        const int s = (int)(g % L::kStages);
        const uint32_t ph = (uint32_t)((g / L::kStages) & 1);
        if (!sm100::mbar_wait(&sh->full[s], ph, p.err, 63)) { alive = false; break; }
        sm100::tc_fence_after();
        const int nkb = min(4, kb_total - kt * 4);
        if (leader) {
          if constexpr (!kF8) {
            for (int kb = 0; kb < nkb; ++kb) {
              sm100::tc_cp_32x128b_warpx4(tmem + L::kSfaCol + 4 * kb,
                                          sm100::sdesc_sf_atom(sm100::smem_u32(stSFA(s) + kb * 512)));
#pragma unroll
              for (int a = 0; a < L::kSfbAtoms; ++a)
                sm100::tc_cp_32x128b_warpx4(
                    tmem + L::kSfbCol + 4 * (kb * L::kSfbAtoms + a),
                    sm100::sdesc_sf_atom(sm100::smem_u32(stSFB(s) + (kb * L::kSfbAtoms + a) * 512)));
            }
          }
          for (int kb = 0; kb < nkb; ++kb) {
            const uint64_t ad = sm100::sdesc_k_sw128(sm100::smem_u32(stA(s)) + kb * 32);
            const uint64_t bd = sm100::sdesc_k_sw128(sm100::smem_u32(stB(s)) + kb * 32);
            if constexpr (kF8)
              sm100::tc_mma_f8(dcol, ad, bd, idesc, (kt | kb) ? 1u : 0u);
            else
              sm100::tc_mma_nvf4(dcol, ad, bd, idesc, tmem + L::kSfaCol + 4 * kb,
                                 tmem + L::kSfbCol + 4 * kb * L::kSfbAtoms, (kt | kb) ? 1u : 0u);
          }
          sm100::tc_commit(&sh->empty[s]);
        }
        __syncwarp();
      }
      if (leader) sm100::tc_commit(&sh->acc_full[b]);
      __syncwarp();
      ++it;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = 32 * q + lane;
    // the four warps of a quadrant split the tile's tokens (segments of a
    // multiple of 8 tokens)
    constexpr int kSegs = kPEpiWarps / 4;
    constexpr int kSeg = ((BN + 8 * kSegs - 1) / (8 * kSegs)) * 8;
    const int hseg = (warp - 4) >> 2;
    const int tbeg = hseg * kSeg, tend = min(BN, tbeg + kSeg);
    constexpr int kChunk = kSeg < 32 ? kSeg : 32;
    const int ncol = geglu ? 64 : 128;
    const int es = (p.epi == kEpiStore && p.c_dt == AEOQ_F32) ? 4 : 2;
    float* colscale = sh->colscale;
    int it = 0;
    for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
      int64_t m_tile;
      const TileInfo ti = tile_of(t, m_tile);
      if (!ti.active) continue;
      const int b = it & 1;
      const uint32_t accp = (uint32_t)((it >> 1) & 1);
      ++it;
      // the previous tile's exchange and column scales are no longer read
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kPEpiWarps) : "memory");
      float alpha = 1.0f;
      if constexpr (kF8) {
        const int64_t wrow = geglu ? (row < 64 ? m_tile * 64 + row : p.n_out / 2 + m_tile * 64 + (row - 64))
                                   : m_tile * 128 + row;
        alpha = p.sb_rows[ti.expert * p.n_out + wrow];
        for (int c = tid - 128; c < BN; c += 32 * kPEpiWarps)
          colscale[c] = c < ti.n_valid ? p.sa_rows[ti.b_row0 + c] : 0.0f;
      } else {
        if (p.epi == kEpiScaleRow) alpha = p.grp_alpha_ts[ti.expert] * load_scalar_f(p.w_ts, p.w_ts_dt);
        else alpha = load_scalar_f(p.a_ts, p.a_ts_dt) * load_scalar_f(p.w_ts, p.w_ts_dt);
      }
      // the tile's row weights in shared memory: one load per row, not one
      // per (row, output column)
      float* roww = sh->roww;
      if (p.epi == kEpiScaleRow)
        for (int c = tid - 128; c < BN; c += 32 * kPEpiWarps)
          roww[c] = c < ti.n_valid ? __bfloat162float(p.row_w[ti.c_row0 + c]) : 0.0f;
      if (kF8 || p.epi == kEpiScaleRow) asm volatile("bar.sync 1, %0;" ::"n"(32 * kPEpiWarps) : "memory");
      auto scaled = [&](float acc, int c) { return kF8 ? (acc * colscale[c]) * alpha : acc * alpha; };
      const bool ok = sm100::mbar_wait(&sh->acc_full[b], accp, p.err, 64);
      sm100::tc_fence_after();
      const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)b * L::kAccStride;
      char* cbase = reinterpret_cast<char*>(p.c) + ti.slot * p.c_slot_stride;
      const int64_t col_w = (int64_t)m_tile * ncol + 32 * (q & (geglu ? 1 : 3));
      char* cwarp = cbase + ti.c_row0 * p.ldc + col_w * es;
      uint32_t hkey = 0;
      if (!geglu) {
        for (int c0 = tbeg; c0 < tend; c0 += kChunk) {
          float v[kChunk < 16 ? 16 : kChunk];
          tmem_chunk<kChunk>(tq + (uint32_t)c0, v);
#pragma unroll
          for (int g8 = 0; g8 < kChunk; g8 += 8) {
            const int t0 = c0 + g8;
            if (t0 >= tend) break;
            float y[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int c = t0 + j;
              float val = (c < ti.n_valid) ? scaled(v[g8 + j], c) : 0.0f;
              if (p.epi == kEpiScaleRow && c < ti.n_valid) val = bf16r(val) * roww[c];
              y[j] = val;
            }
            if (!ok) continue;
            if (es == 2) {
              store_8tok_bf16(y, cwarp + t0 * p.ldc, p.ldc, ti.n_valid - t0, lane);
            } else {
#pragma unroll
              for (int j = 0; j < 8; ++j)
                if (t0 + j < ti.n_valid) *reinterpret_cast<float*>(cwarp + (t0 + j) * p.ldc + 4 * lane) = y[j];
            }
          }
        }
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&sh->acc_empty[b]);
      } else {
        if (row >= 64) {
          for (int c0 = tbeg; c0 < tend; c0 += kChunk) {
            float v[kChunk < 16 ? 16 : kChunk];
            tmem_chunk<kChunk>(tq + (uint32_t)c0, v);
#pragma unroll
            for (int j = 0; j < kChunk; ++j)
              if (c0 + j < tend) xchg[(row - 64) * L::kXs + c0 + j] = __float2bfloat16_rn(scaled(v[j], c0 + j));
          }
          sm100::tc_fence_before();
          __syncwarp();
          if (lane == 0) sm100::mbar_arrive(&sh->acc_empty[b]);
        }
        asm volatile("bar.sync 1, %0;" ::"n"(32 * kPEpiWarps) : "memory");
        if (q < 2) {
          for (int c0 = tbeg; c0 < tend; c0 += kChunk) {
            float v[kChunk < 16 ? 16 : kChunk];
            tmem_chunk<kChunk>(tq + (uint32_t)c0, v);
#pragma unroll
            for (int g8 = 0; g8 < kChunk; g8 += 8) {
              const int t0 = c0 + g8;
              if (t0 >= tend) break;
              float y[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const int c = t0 + j;
                float hvf = 0.0f;
                if (c < ti.n_valid) {
                  const float gv = bf16r(scaled(v[g8 + j], c));
                  const float u = __bfloat162float(xchg[row * L::kXs + c]);
                  const __nv_bfloat16 hv = __float2bfloat16_rn(bf16r(gelu_tanh(gv)) * u);
                  hkey = max(hkey, In<AEOQ_BF16>::abs_key(hv));
                  hvf = __bfloat162float(hv);
                }
                y[j] = hvf;
              }
              if (ok) store_8tok_bf16(y, cwarp + t0 * p.ldc, p.ldc, ti.n_valid - t0, lane);
            }
          }
          sm100::tc_fence_before();
          __syncwarp();
          if (lane == 0) sm100::mbar_arrive(&sh->acc_empty[b]);
        }
        if (p.grp_amax) {
          hkey = warp_umax(hkey);
          if (lane == 0 && hkey) atomicMax(p.grp_amax + ti.expert, hkey);
        }
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, L::kTmemCols);
  }
}

template <int BN, bool kF8>
static int launch_persistent(const uint8_t* a, int64_t a_rows, const uint8_t* b, TcParams p, int grid_ctas,
                             cudaStream_t st) {
  using L = PLayout<BN, kF8>;
  CUtensorMap ta, tb;
  const int64_t row_bytes = kF8 ? p.K : p.K / 2;
  int rc = make_tmap(&ta, a, a_rows, row_bytes, row_bytes, p.epi == kEpiGeglu ? 64 : 128);
  if (rc) return rc;
  rc = make_tmap(&tb, b, p.b_rows, row_bytes, row_bytes, BN);
  if (rc) return rc;
  {
    const int rc = func_smem_attr((const void*)tc_gemm_persistent_kernel<BN, kF8>, L::kBytes, -1,
                                  "tc_gemm_persistent");
    if (rc) return rc;
  }
  tc_gemm_persistent_kernel<BN, kF8><<<grid_ctas, kPThreads, L::kBytes, st>>>(ta, tb, p);
  return check_launch(kF8 ? "tc_gemm_persistent_kernel<fp8>" : "tc_gemm_persistent_kernel");
}

static int sm_count() { return device_sm_count(); }

// ---------------------------------------------------------------- host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    cudaGetLastError();
  });
  return fn;
}

// 2D uint8 tensor map: rows x row_bytes (row stride ld), box 128 B x box_rows, 128-byte swizzle.
// 2D byte tensor map: rows x row_bytes with a row pitch of ld bytes; boxes of
// box_rows x box_bytes, 128-byte swizzled (operand tiles, box_bytes = 128)
// or plain (row-major staging of scale rows).
int make_tmap_bytes(CUtensorMap* m, const void* ptr, int64_t rows, int64_t row_bytes, int64_t ld, int box_bytes,
                    int box_rows, bool swizzle128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(AEOQ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld};
  cuuint32_t box[2] = {(cuuint32_t)box_bytes, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(AEOQ_ERR_INVALID, "tensor map encode failed (%d)", (int)r);
  return AEOQ_OK;
}

int make_tmap(CUtensorMap* m, const void* ptr, int64_t rows, int64_t row_bytes, int64_t ld, int box_rows) {
  return make_tmap_bytes(m, ptr, rows, row_bytes, ld, kKTBytes, box_rows, true);
}

// Byte tensor map of rank 2..5: dims[0] innermost (bytes), strides[i] the
// byte pitch of dims[i + 1], box[] the tile extents.
int make_tmap_nd(CUtensorMap* m, const void* ptr, int rank, const int64_t* dims, const int64_t* strides,
                 const int* box, bool swizzle128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(AEOQ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = (cuuint64_t)dims[i];
    b[i] = (cuuint32_t)box[i];
    e[i] = 1;
    if (i + 1 < rank) st[i] = (cuuint64_t)strides[i];
  }
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, (cuuint32_t)rank, const_cast<void*>(ptr), d, st, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(AEOQ_ERR_INVALID, "tensor map (rank %d) encode failed (%d)", rank, (int)r);
  return AEOQ_OK;
}

template <int BN, bool kF8>
static int launch_tc(const uint8_t* a, int64_t a_rows, const uint8_t* b, const TcParams& p, dim3 grid,
                     cudaStream_t st) {
  using L = TcLayout<BN, kF8>;
  CUtensorMap ta, tb;
  const int64_t row_bytes = kF8 ? p.K : p.K / 2;
  int rc = make_tmap(&ta, a, a_rows, row_bytes, row_bytes, p.epi == kEpiGeglu ? 64 : 128);
  if (rc) return rc;
  rc = make_tmap(&tb, b, p.b_rows, row_bytes, row_bytes, BN);
  if (rc) return rc;
  {
    const int rc = func_smem_attr((const void*)nvfp4_tc_gemm_kernel<BN, kF8>, L::kBytes, -1, "tc_gemm");
    if (rc) return rc;
  }
  nvfp4_tc_gemm_kernel<BN, kF8><<<grid, kTcThreads, L::kBytes, st>>>(ta, tb, p);
  return check_launch(kF8 ? "fp8_tc_gemm_kernel" : "nvfp4_tc_gemm_kernel");
}

template <bool kF8>
int tc_gemm_dispatch_kind(int bn, const uint8_t* a, int64_t a_rows, const uint8_t* b, const TcParams& p, dim3 grid,
                          cudaStream_t st) {
  switch (bn) {
    case 8: return launch_tc<8, kF8>(a, a_rows, b, p, grid, st);
    case 16: return launch_tc<16, kF8>(a, a_rows, b, p, grid, st);
    case 32: return launch_tc<32, kF8>(a, a_rows, b, p, grid, st);
    case 64: return launch_tc<64, kF8>(a, a_rows, b, p, grid, st);
    case 128: return launch_tc<128, kF8>(a, a_rows, b, p, grid, st);
    case 256: return launch_tc<256, kF8>(a, a_rows, b, p, grid, st);
  }
  return set_error(AEOQ_ERR_INVALID, "tc_gemm: unsupported tile N %d", bn);
}

int tc_gemm_dispatch(int bn, const uint8_t* a, int64_t a_rows, const uint8_t* b, const TcParams& p, dim3 grid,
                     cudaStream_t st) {
  return tc_gemm_dispatch_kind<false>(bn, a, a_rows, b, p, grid, st);
}

// Persistent launch over the tile grid `grid` (x: weight tiles, y: token
// tiles, z: slots; mode 1 reads the token-tile count on the device).
template <bool kF8>
int tc_gemm_persistent(int bn, const uint8_t* a, int64_t a_rows, const uint8_t* b, TcParams p, dim3 grid,
                       cudaStream_t st) {
  p.tiles_x = (int)grid.x;
  p.tiles_y = (int)grid.y;
  p.tiles_z = (int)grid.z;
  const int64_t total = (int64_t)grid.x * grid.y * grid.z;
  const int ctas = (int)std::min<int64_t>(sm_count(), std::max<int64_t>(1, total));
  if (bn == 224) return launch_persistent<224, kF8>(a, a_rows, b, p, ctas, st);
  if (bn == 128) return launch_persistent<128, kF8>(a, a_rows, b, p, ctas, st);
  return set_error(AEOQ_ERR_INVALID, "tc_gemm_persistent: unsupported tile N %d", bn);
}

int pick_bn(int64_t M) {
  if (M <= 8) return 8;
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

}  // namespace aeoq

using namespace aeoq;

// Token-tile width: the smallest tile covering M, halved while the grid
// would leave SMs idle (each halving adds CTAs that re-read the weight tile
// from L2, which is cheaper than idle HBM bandwidth).
extern "C" int aeoq_nvfp4_tile_n(int64_t M, int64_t N, int64_t slots) {
  // Problems of two or more waves of 224-token tiles take the persistent
  // kernel (double-buffered accumulator, epilogue under the next main loop).
  if ((N / 128) * (slots > 0 ? slots : 1) * ((M + 223) / 224) >= 2 * 148) return 224;
  int bn = pick_bn(M);
  const int64_t base = (N / 128) * (slots > 0 ? slots : 1);
  while (bn > 8 && base * ((M + bn - 1) / bn) < 148) bn >>= 1;
  return bn;
}

// Tensor-core path of aeoq_nvfp4_gemm for contiguous operands: A/B packed rows
// of K/2 bytes, scale rows of K/16 bytes (the reference tensors' layouts).
extern "C" int aeoq_nvfp4_gemm_tc(const uint8_t* a, const uint8_t* a_sf_atoms, const void* a_ts, int a_ts_dtype,
                                  int64_t a_slot_rows, const uint8_t* w, const uint8_t* w_sf_atoms, const void* w_ts,
                                  int w_ts_dtype, int64_t num_experts, const void* expert_ids, int ids_dtype,
                                  int64_t slots, int64_t M, int64_t N, int64_t K, int tile_n, void* c, int c_dtype,
                                  int* err_word, void* stream) {
  AEOQ_REQUIRE(slots >= 0 && M >= 0 && N >= 0 && K >= 0, AEOQ_ERR_INVALID, "nvfp4_gemm_tc: negative shape");
  AEOQ_REQUIRE(N % 128 == 0, AEOQ_ERR_INVALID, "nvfp4_gemm_tc: N (%lld) must be a multiple of 128", (long long)N);
  AEOQ_REQUIRE(K % 64 == 0 && K > 0, AEOQ_ERR_INVALID, "nvfp4_gemm_tc: K (%lld) must be a multiple of 64",
               (long long)K);
  AEOQ_REQUIRE((K / 2) % 16 == 0, AEOQ_ERR_INVALID, "nvfp4_gemm_tc: K/2 must be a multiple of 16");
  AEOQ_REQUIRE(c_dtype == AEOQ_BF16 || c_dtype == AEOQ_F32, AEOQ_ERR_INVALID, "nvfp4_gemm_tc: bad output dtype");
  AEOQ_REQUIRE(tile_n == 8 || tile_n == 16 || tile_n == 32 || tile_n == 64 || tile_n == 128 || tile_n == 224 ||
                   tile_n == 256,
               AEOQ_ERR_INVALID, "nvfp4_gemm_tc: tile_n %d must be 224 or a power of two in [8, 256]", tile_n);
  if (slots * M * N == 0) return AEOQ_OK;
  AEOQ_REQUIRE(a && a_sf_atoms && a_ts && w && w_sf_atoms && w_ts && c && err_word, AEOQ_ERR_INVALID,
               "nvfp4_gemm_tc: null pointer");
  AEOQ_REQUIRE((uintptr_t)a % 16 == 0 && (uintptr_t)w % 16 == 0 && (uintptr_t)a_sf_atoms % 16 == 0 &&
                   (uintptr_t)w_sf_atoms % 16 == 0,
               AEOQ_ERR_INVALID, "nvfp4_gemm_tc: operands and scale atoms must be 16-byte aligned");
  TcParams p{};
  p.n_out = N;
  p.K = K;
  p.num_experts = num_experts;
  p.sfa = w_sf_atoms;
  p.sfb = a_sf_atoms;
  p.b_rows = a_slot_rows ? slots * M : M;
  p.tiles_per_slot = (M + tile_n - 1) / tile_n;
  p.mode = 0;
  p.M = M;
  p.b_slot_rows = a_slot_rows ? M : 0;
  p.ids = expert_ids;
  p.ids_dt = ids_dtype;
  p.epi = kEpiStore;
  p.a_ts = a_ts; p.a_ts_dt = a_ts_dtype;
  p.w_ts = w_ts; p.w_ts_dt = w_ts_dtype;
  p.c = c;
  p.c_dt = c_dtype;
  const int es = c_dtype == AEOQ_BF16 ? 2 : 4;
  p.ldc = N * es;
  p.c_slot_stride = M * N * es;
  p.err = err_word;
  dim3 grid((unsigned)(N / 128), (unsigned)((M + tile_n - 1) / tile_n), (unsigned)slots);
  if (tile_n == 224) return tc_gemm_persistent<false>(tile_n, w, num_experts * N, a, p, grid, (cudaStream_t)stream);
  return tc_gemm_dispatch(tile_n, w, num_experts * N, a, p, grid, (cudaStream_t)stream);
}

// Grouped (MoE) path: B rows are sorted by expert; expert e owns rows
// [grp_off[e], grp_off[e+1]) and token tiles [tile_off[e], tile_off[e+1]) of
// tile_n rows. epi: 0 store alpha*acc (bf16), 1 GeGLU over the gate/up halves
// (N = 2I weight rows, output I wide, per-expert amax keys), 2 down with
// bf16(bf16(grp_ts[e]*w_ts*acc) * row_w[r]).
extern "C" int aeoq_nvfp4_gemm_grouped(const uint8_t* b, const uint8_t* b_sf, int64_t max_rows, const int* grp_off,
                                       const int* tile_off, int tile_n, const uint8_t* w, const uint8_t* w_sf,
                                       int64_t num_experts, int64_t N, int64_t K, int epi, const void* a_ts,
                                       int a_ts_dtype, const void* w_ts, int w_ts_dtype, const float* grp_ts,
                                       const void* row_w, uint32_t* grp_amax, void* c, int64_t ldc, int* err_word,
                                       void* stream) {
  AEOQ_REQUIRE(N % 128 == 0 && K % 64 == 0 && K > 0 && (K / 2) % 16 == 0, AEOQ_ERR_INVALID,
               "nvfp4_gemm_grouped: N %% 128 == 0 and K %% 64 == 0 required");
  AEOQ_REQUIRE(epi >= 0 && epi <= 2, AEOQ_ERR_INVALID, "nvfp4_gemm_grouped: bad epilogue %d", epi);
  AEOQ_REQUIRE(tile_n == 8 || tile_n == 16 || tile_n == 32 || tile_n == 64 || tile_n == 128 || tile_n == 224 ||
                   tile_n == 256,
               AEOQ_ERR_INVALID, "nvfp4_gemm_grouped: tile_n must be 224 or a power of two in [8, 256]");
  AEOQ_REQUIRE(num_experts >= 1 && num_experts <= 1024, AEOQ_ERR_INVALID, "nvfp4_gemm_grouped: bad expert count");
  if (max_rows <= 0) return AEOQ_OK;
  AEOQ_REQUIRE(b && b_sf && grp_off && tile_off && w && w_sf && w_ts && c && err_word, AEOQ_ERR_INVALID,
               "nvfp4_gemm_grouped: null pointer");
  AEOQ_REQUIRE(epi != 2 || (grp_ts && row_w), AEOQ_ERR_INVALID, "nvfp4_gemm_grouped: down epilogue needs scales");
  AEOQ_REQUIRE(epi == 2 || a_ts, AEOQ_ERR_INVALID, "nvfp4_gemm_grouped: activation scale missing");
  TcParams p{};
  p.n_out = N;
  p.K = K;
  p.num_experts = num_experts;
  p.sfa = w_sf;
  p.sfb = b_sf;
  p.b_rows = max_rows;
  p.mode = 1;
  p.grp_off = grp_off;
  p.tile_off = tile_off;
  p.epi = epi;
  p.a_ts = a_ts; p.a_ts_dt = a_ts_dtype;
  p.w_ts = w_ts; p.w_ts_dt = w_ts_dtype;
  p.grp_alpha_ts = grp_ts;
  p.row_w = reinterpret_cast<const __nv_bfloat16*>(row_w);
  p.c = c;
  p.c_dt = AEOQ_BF16;
  p.ldc = ldc;
  p.grp_amax = grp_amax;
  p.err = err_word;
  const int64_t max_tiles = (max_rows + tile_n - 1) / tile_n + num_experts;
  const unsigned gx = (unsigned)(epi == kEpiGeglu ? (N / 2) / 64 : N / 128);
  dim3 grid(gx, (unsigned)max_tiles, 1);
  if (tile_n == 128 || tile_n == 224)
    return tc_gemm_persistent<false>(tile_n, w, num_experts * N, b, p, grid, (cudaStream_t)stream);
  return tc_gemm_dispatch(tile_n, w, num_experts * N, b, p, grid, (cudaStream_t)stream);
}

// ---------------------------------------------------------------- FP8
// torch._scaled_mm(x_fp8, w_fp8.t(), scale_a, scale_b, out_dtype=bf16) of
// _fp8_linear (modeling.py:105-108): C[m][n] = bf16((acc * sa[m]) * sb[n]).
extern "C" int aeoq_fp8_gemm(const uint8_t* a, const float* sa, int64_t M, const uint8_t* w, const float* sb,
                             int64_t N, int64_t K, void* c, int* err_word, void* stream) {
  AEOQ_REQUIRE(M >= 0 && N >= 0 && K >= 0, AEOQ_ERR_INVALID, "fp8_gemm: negative shape");
  AEOQ_REQUIRE(N % 128 == 0, AEOQ_ERR_INVALID, "fp8_gemm: N (%lld) must be a multiple of 128", (long long)N);
  AEOQ_REQUIRE(K % 32 == 0 && K > 0, AEOQ_ERR_INVALID, "fp8_gemm: K (%lld) must be a multiple of 32", (long long)K);
  if (M * N == 0) return AEOQ_OK;
  AEOQ_REQUIRE(a && sa && w && sb && c && err_word, AEOQ_ERR_INVALID, "fp8_gemm: null pointer");
  AEOQ_REQUIRE((uintptr_t)a % 16 == 0 && (uintptr_t)w % 16 == 0, AEOQ_ERR_INVALID,
               "fp8_gemm: operands must be 16-byte aligned");
  const int tile_n = aeoq_nvfp4_tile_n(M, N, 1);
  TcParams p{};
  p.n_out = N;
  p.K = K;
  p.num_experts = 1;
  p.b_rows = M;
  p.tiles_per_slot = (M + tile_n - 1) / tile_n;
  p.mode = 0;
  p.M = M;
  p.epi = kEpiStore;
  p.c = c;
  p.c_dt = AEOQ_BF16;
  p.ldc = N * 2;
  p.sa_rows = sa;
  p.sb_rows = sb;
  p.err = err_word;
  dim3 grid((unsigned)(N / 128), (unsigned)((M + tile_n - 1) / tile_n), 1);
  if (tile_n == 224) return tc_gemm_persistent<true>(tile_n, w, N, a, p, grid, (cudaStream_t)stream);
  return tc_gemm_dispatch_kind<true>(tile_n, w, N, a, p, grid, (cudaStream_t)stream);
}

// Grouped FP8 expert GEMM over expert-sorted rows (aeoq_moe_route layout).
// epi 0: C = bf16((acc * sa[r]) * sb[e][n]); 1: GeGLU over the gate/up halves
// (N = 2I rows, output I wide): h = bf16(bf16(gelu(bf16(g))) * bf16(u));
// 2: down, bf16(bf16(y) * row_w[r]) (modeling.py:122-146).
extern "C" int aeoq_fp8_gemm_grouped(const uint8_t* b, const float* sa_rows, int64_t max_rows, const int* grp_off,
                                     const int* tile_off, int tile_n, const uint8_t* w, const float* sb_rows,
                                     int64_t num_experts, int64_t N, int64_t K, int epi, const void* row_w, void* c,
                                     int64_t ldc, int* err_word, void* stream) {
  AEOQ_REQUIRE(N % 128 == 0 && K % 32 == 0 && K > 0, AEOQ_ERR_INVALID,
               "fp8_gemm_grouped: N %% 128 == 0 and K %% 32 == 0 required");
  AEOQ_REQUIRE(epi >= 0 && epi <= 2, AEOQ_ERR_INVALID, "fp8_gemm_grouped: bad epilogue %d", epi);
  AEOQ_REQUIRE(tile_n == 8 || tile_n == 16 || tile_n == 32 || tile_n == 64 || tile_n == 128 || tile_n == 224 ||
                   tile_n == 256,
               AEOQ_ERR_INVALID, "fp8_gemm_grouped: tile_n must be 224 or a power of two in [8, 256]");
  AEOQ_REQUIRE(num_experts >= 1 && num_experts <= 1024, AEOQ_ERR_INVALID, "fp8_gemm_grouped: bad expert count");
  if (max_rows <= 0) return AEOQ_OK;
  AEOQ_REQUIRE(b && sa_rows && grp_off && tile_off && w && sb_rows && c && err_word, AEOQ_ERR_INVALID,
               "fp8_gemm_grouped: null pointer");
  AEOQ_REQUIRE(epi != 2 || row_w, AEOQ_ERR_INVALID, "fp8_gemm_grouped: down epilogue needs row weights");
  AEOQ_REQUIRE((uintptr_t)b % 16 == 0 && (uintptr_t)w % 16 == 0, AEOQ_ERR_INVALID,
               "fp8_gemm_grouped: operands must be 16-byte aligned");
  TcParams p{};
  p.n_out = N;
  p.K = K;
  p.num_experts = num_experts;
  p.b_rows = max_rows;
  p.mode = 1;
  p.grp_off = grp_off;
  p.tile_off = tile_off;
  p.epi = epi;
  p.row_w = reinterpret_cast<const __nv_bfloat16*>(row_w);
  p.c = c;
  p.c_dt = AEOQ_BF16;
  p.ldc = ldc;
  p.sa_rows = sa_rows;
  p.sb_rows = sb_rows;
  p.err = err_word;
  const int64_t max_tiles = (max_rows + tile_n - 1) / tile_n + num_experts;
  const unsigned gx = (unsigned)(epi == kEpiGeglu ? (N / 2) / 64 : N / 128);
  dim3 grid(gx, (unsigned)max_tiles, 1);
  if (tile_n == 128 || tile_n == 224)
    return tc_gemm_persistent<true>(tile_n, w, num_experts * N, b, p, grid, (cudaStream_t)stream);
  return tc_gemm_dispatch_kind<true>(tile_n, w, num_experts * N, b, p, grid, (cudaStream_t)stream);
}
