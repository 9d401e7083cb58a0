// One-token NVFP4 MoE expert forward on the tensor cores (two launches).
//
// Restates Gemma4TextExpertsNVFP4._forward_decode_3d (aeo_quant
// src/aeo_quant/bridges/gemma4/modeling_nvfp4.py:132-186). At one token the
// work is a stream of the k selected experts' packed weights through
// tcgen05.mma (kind::mxf4nvf4, block16 e4m3 scales, f32 accumulate in TMEM).
//
// Orientation: the weights are the MMA's N side (B operand, up to 256 rows
// per instruction) and the token is the M = 128 side (A operand) with the
// token in row 0. Only accumulator row 0 is read, so A rows 1-127 may hold
// anything: each 1 KB token tile (8 swizzled rows of 128 B) is followed in
// shared memory by other buffers that serve as those rows. One instruction
// thus covers 64 K-values of up to 256 weight rows.
//
// Scale factors are taken in the reference's own row layout ([rows][K/16]
// e4m3 bytes) and written into TMEM by the four epilogue warps with
// tcgen05.st, in the arrangement tcgen05.cp.32x128b.warpx4 would produce
// from a 512-byte atom (matrix row r of a 128-row group at lane r % 32 of
// every lane quadrant, column (r / 32) % 4, byte k of the 64-value step).
// No precomputed weight layout is needed.
//
//  launch 1  gate_up + GeGLU. CTA (m, p, j): T gate rows T*m.. and the T
//            matching up rows of expert ids[j] (N = 2T), K range p of the
//            hidden size. TMA streams the weight tiles through a ring while
//            the epilogue warps quantize the hidden vector
//            (quantize_2d_to_nvfp4 semantics, :150-153) into the token tile
//            and both scale sets into TMEM. The K parts of a tile form a
//            thread-block cluster: rank 0 adds the parts' f32 accumulator
//            rows in part order from their shared memory (distributed shared
//            memory), then computes h = bf16(bf16(gelu(bf16(g*a))) *
//            bf16(u*a)) (:155-162) and the tile's max |h|.
//  launch 2  down + combine, launched early (programmatic dependent launch):
//            CTA (t, j) prefetches its N2 down rows of expert ids[j] and
//            their scales and writes the weight scales into TMEM while
//            launch 1 still runs; then waits, reduces the maxima to the
//            shared tensor scale (:164-172), quantizes h[j] into its token
//            tile, runs the MMAs and writes bf16(bf16(a*d) * w_j) (:183).
//            The k CTAs of a row tile form a cluster; each sums a slice of
//            the rows over the k CTAs' shared memory in f32 in expert order
//            and rounds once (:184-186).
// Every mbarrier wait is bounded (sm100::mbar_wait); TMEM is freed on every
// path, and before any wait on another CTA (a cluster barrier), so that no
// CTA blocked in tcgen05.alloc can be part of a wait cycle.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"

namespace aeoq {

int make_tmap_bytes(CUtensorMap* m, const void* ptr, int64_t rows, int64_t row_bytes, int64_t ld, int box_bytes,
                    int box_rows, bool swizzle128);
int make_tmap_nd(CUtensorMap* m, const void* ptr, int rank, const int64_t* dims, const int64_t* strides,
                 const int* box, bool swizzle128);

namespace dtc {

__device__ __forceinline__ int cta_linear() {
  return (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
}


constexpr int kThreads = 192;      // launch 2
constexpr int kThreads1 = 256;     // launch 1: two more producer warps (6, 7)
constexpr int kRing = 6;           // launch-1 weight ring: every K stage of a CTA in flight at once
constexpr int kProducers1 = 3;     // launch-1 producer warps 0, 6, 7 (slot s -> producer s % 3)

__host__ __device__ constexpr int rup(int v, int m) { return (v + m - 1) / m * m; }

// Shape plan, computed once on the host (plan_for) and passed by value.
struct Plan {
  int H, I, k;
  int64_t E;
  int T;                // launch 1: gate rows (= up rows) per tile, N1 = 2T
  int tiles;            // I / T
  int parts;            // K parts of launch 1
  int Q;                // 64-value K steps per part (multiple of 4)
  int sfa1, sfb1, cols1;
  int N2;               // launch 2: down rows per tile
  int sfa2, sfb2, cols2;
};

struct Args {
  const __nv_bfloat16* hidden;
  const void* ids; int ids_dt;
  const __nv_bfloat16* topw;
  const void* gu_ts; int gu_ts_dt;
  const uint8_t* d_sf;  const void* d_ts; int d_ts_dt;
  uint32_t* hmax;        // [k * tiles]   max |h| key per tile
  __nv_bfloat16* h;      // [k][I]
  __nv_bfloat16* out;    // [H]
  int* err;
};

// ---- shared-memory layouts (offsets from a 1024-aligned base)
struct L1 {
  int a, ring, stage, hid, sf, sfrow, tok, dv, bars, bytes;
  __host__ __device__ explicit L1(const Plan& p) {
    const int nt = p.Q / 4;
    a = 0;                                   // nt token tiles of 1 KB
    ring = 1024 * nt;
    stage = 2 * p.T * 128;
    hid = ring + kRing * stage;
    sfrow = 4 * p.Q;                         // scale rows: gate rows, then up rows, 4Q bytes each
    sf = rup(hid + 2 * p.H, 128);
    tok = rup(sf + 2 * p.T * sfrow, 16);     // token scale bytes, 4 per K step
    dv = rup(tok + 4 * p.Q, 16);             // 2T f32 accumulator row
    bars = rup(dv + 8 * p.T, 16);
    bytes = bars + 256;
    if (bytes < ring + 16384) bytes = ring + 16384;   // token tiles' rows 8-127 stay inside
  }
};
struct L2 {
  int a, b, sf, sfrow, tok, dv, bars, bytes;
  __host__ __device__ explicit L2(const Plan& p) {
    const int nt = (p.I / 64 + 3) / 4;
    a = 0;
    b = 1024 * nt;                           // nt weight tiles of N2 x 128 B
    sfrow = p.I / 16;
    sf = b + nt * p.N2 * 128;
    tok = rup(sf + p.N2 * sfrow, 16);
    dv = rup(tok + p.I / 16, 16);
    bars = rup(dv + 4 * p.N2, 16);
    bytes = bars + 256;
    if (bytes < b + 16384) bytes = b + 16384;
  }
};

struct Bars1 {
  uint64_t full[kRing], empty[kRing], hid, sf, bready, accum;
  uint32_t tmem;
  uint32_t red[4];
};
struct Bars2 {
  uint64_t full, bready, accum;
  uint32_t tmem;
  uint32_t red[4];
};

// One 16-value block quantized into row 0 of a token tile set (packed bytes
// at (bl / 16) * 1024 + (bl % 16) * 8; row 0 of a 128-byte-swizzled tile is
// unpermuted) with its scale byte at tok[bl].
__device__ __forceinline__ void quant_block_row0(const float (&v)[16], float ts, int bl, uint8_t* tiles,
                                                 uint8_t* tok) {
  uint32_t w0, w1;
  const uint32_t sf = nvfp4_quant_block(v, ts, w0, w1);
  *reinterpret_cast<uint2*>(tiles + (bl >> 4) * 1024 + (bl & 15) * 8) = make_uint2(w0, w1);
  tok[bl] = (uint8_t)sf;
}

__device__ __forceinline__ void unpack16(uint4 u0, uint4 u1, float (&v)[16]) {
  const __nv_bfloat16* e0 = reinterpret_cast<const __nv_bfloat16*>(&u0);
  const __nv_bfloat16* e1 = reinterpret_cast<const __nv_bfloat16*>(&u1);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[i] = __bfloat162float(e0[i]);
    v[8 + i] = __bfloat162float(e1[i]);
  }
}

// Token scales into TMEM, column 4 * kb of the warp's quadrant (lane 0 holds
// row 0's four bytes; the other lanes' values belong to rows whose results
// are never read).
__device__ __forceinline__ void st_token_scales(uint32_t taddr, const uint8_t* tok, int nkb, int lane) {
  for (int kb = 0; kb < nkb; ++kb)
    sm100::tmem_st1(taddr + 4 * kb, lane == 0 ? *reinterpret_cast<const uint32_t*>(tok + 4 * kb) : 0u);
}

// Weight scales into TMEM for the N-row B operand: 8 columns per K step,
// column 4a + i of lane l = matrix row 128a + 32i + l (rows >= n_rows zero).
// Launch-1 layout: chunk c (4 K steps) holds each of the N rows' 16 scale
// bytes contiguously (row r at c * chunk_bytes + 16 r), so every lane reads a
// row's four steps with one conflict-free 16-byte load.
__device__ __forceinline__ void st_weight_scales_chunked(uint32_t taddr, const uint8_t* sf, int chunk_bytes,
                                                         int n_rows, int nkb, int lane) {
  for (int c = 0; c < (nkb + 3) / 4; ++c) {
    uint4 v[2][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = 128 * a + 32 * i + lane;
        v[a][i] = *reinterpret_cast<const uint4*>(sf + c * chunk_bytes + 16 * (row < n_rows ? row : 0));
        if (row >= n_rows) v[a][i] = make_uint4(0u, 0u, 0u, 0u);
      }
    uint32_t r[32];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        r[0 * 8 + 4 * a + i] = v[a][i].x;
        r[1 * 8 + 4 * a + i] = v[a][i].y;
        r[2 * 8 + 4 * a + i] = v[a][i].z;
        r[3 * 8 + 4 * a + i] = v[a][i].w;
      }
    sm100::tmem_st32(taddr + 32 * c, r);
  }
}

// Same, from row-major scale rows of row_bytes (a multiple of 16): each lane
// reads a row's four steps with one 16-byte load.
__device__ __forceinline__ void st_weight_scales_rows16(uint32_t taddr, const uint8_t* sf, int row_bytes, int n_rows,
                                                        int nkb, int lane) {
  for (int c = 0; c < (nkb + 3) / 4; ++c) {
    uint4 v[2][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = 128 * a + 32 * i + lane;
        v[a][i] = *reinterpret_cast<const uint4*>(sf + (row < n_rows ? row : 0) * row_bytes + 16 * c);
        if (row >= n_rows) v[a][i] = make_uint4(0u, 0u, 0u, 0u);
      }
    uint32_t r[32];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        r[0 * 8 + 4 * a + i] = v[a][i].x;
        r[1 * 8 + 4 * a + i] = v[a][i].y;
        r[2 * 8 + 4 * a + i] = v[a][i].z;
        r[3 * 8 + 4 * a + i] = v[a][i].w;
      }
    sm100::tmem_st32(taddr + 32 * c, r);
  }
}

// Same, from row-major scale rows of sfrow bytes (a multiple of 4; words
// past a row's last K step are read but not used by any MMA), for an N-row
// operand of kAtoms 128-row groups: 4 * kAtoms columns per K step.
template <int kAtoms>
__device__ __forceinline__ void st_weight_scales_rows(uint32_t taddr, const uint8_t* sf, int sfrow, int n_rows,
                                                      int nkb, int lane) {
  constexpr int kPer = 8 / kAtoms;   // K steps per 32-column store
  for (int c = 0; c < (nkb + kPer - 1) / kPer; ++c) {
    uint32_t r[32];
#pragma unroll
    for (int a = 0; a < kAtoms; ++a)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = 128 * a + 32 * i + lane;
        const uint32_t* src = reinterpret_cast<const uint32_t*>(sf + (row < n_rows ? row : 0) * sfrow) + kPer * c;
#pragma unroll
        for (int kbi = 0; kbi < kPer; ++kbi) r[4 * kAtoms * kbi + 4 * a + i] = row < n_rows ? src[kbi] : 0u;
      }
    sm100::tmem_st32(taddr + 32 * c, r);
  }
}

// Accumulator row 0 (lane 0 of quadrant 0) -> dv[0..n) in shared memory;
// run by the warp whose lane quadrant is 0.
__device__ __forceinline__ void read_row0(uint32_t tmem, int n, bool keep, float* dv, int lane) {
  for (int c = 0; c < (n + 63) / 64; ++c) {
    uint32_t r0[32], r1[32];
    sm100::tmem_ld32_nowait(tmem + 64 * c, r0);
    sm100::tmem_ld32_nowait(tmem + 64 * c + 32, r1);
    sm100::tmem_ld_wait();
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (64 * c + i < n) dv[64 * c + i] = keep ? __uint_as_float(r0[i]) : 0.0f;
        if (64 * c + 32 + i < n) dv[64 * c + 32 + i] = keep ? __uint_as_float(r1[i]) : 0.0f;
      }
    }
  }
  __syncwarp();
}

__device__ __forceinline__ uint32_t block_max128(uint32_t key, int t, uint32_t* red) {
  key = warp_umax(key);
  if ((t & 31) == 0) red[t >> 5] = key;
  asm volatile("bar.sync 2, 128;" ::: "memory");
  key = max(max(red[0], red[1]), max(red[2], red[3]));
  asm volatile("bar.sync 2, 128;" ::: "memory");
  return key;
}

// ------------------------------------------------------------------ launch 1
__global__ void __launch_bounds__(kThreads1, 1)
    decode_gateup_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmS,
                            const Args a, const Plan pl) {
  extern __shared__ __align__(1024) uint8_t dsm[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  const L1 L(pl);
  uint8_t* tokA = base + L.a;
  uint8_t* ring = base + L.ring;
  const __nv_bfloat16* hid = reinterpret_cast<const __nv_bfloat16*>(base + L.hid);
  uint8_t* sfs = base + L.sf;
  uint8_t* tok = base + L.tok;
  float* dv = reinterpret_cast<float*>(base + L.dv);
  Bars1* sh = reinterpret_cast<Bars1*>(base + L.bars);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m = blockIdx.x, p = blockIdx.y, j = blockIdx.z;
  const int T = pl.T, N1 = 2 * T, H = pl.H, I = pl.I;
  const int kb0 = p * pl.Q, nkb = min(pl.Q, H / 64 - kb0), nt = (nkb + 3) / 4;

  if (tid == 0) {
    for (int s = 0; s < kRing; ++s) {
      sm100::mbar_init(&sh->full[s], 1);
      sm100::mbar_init(&sh->empty[s], 1);
    }
    sm100::mbar_init(&sh->hid, 1);
    sm100::mbar_init(&sh->sf, 1);
    sm100::mbar_init(&sh->bready, 5);
    sm100::mbar_init(&sh->accum, 1);
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tmW);
    sm100::prefetch_tmap(&tmS);
  }
  if (warp == 1) sm100::tmem_alloc(&sh->tmem, (uint32_t)pl.cols1);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = sh->tmem;
  pdl_wait();        // inputs may come from the preceding kernel
  const int64_t e = load_index(a.ids, a.ids_dt, j);
  const bool valid = e >= 0 && e < pl.E;
  float alpha = 0.0f;

  if (warp == 0 || warp >= 6) {
    // ---- producers: warp 0 (ring slot 0, plus the hidden vector, the
    // scales and the weight scales' TMEM copy), warps 6 and 7 (slots 1, 2).
    // One warp's copies complete one after another, so the slots go to
    // different warps. Tensor maps: weights (H/2, I, gate|up, E) and scales
    // (H/16, I, gate|up, E), so one box brings a stage's gate and up rows.
    const int pidx = warp == 0 ? 0 : warp - 5;
    const bool leader = sm100::elect_one();
    if (warp == 0 && leader) {
      // the hidden vector and the scales first: the quantization and the
      // scale copy into TMEM wait on them, the MMAs on those
      sm100::mbar_arrive_expect_tx(&sh->hid, (uint32_t)(2 * H));
      bulk_g2s(base + L.hid, a.hidden, (uint32_t)(2 * H), &sh->hid);
      if (valid) {
        sm100::mbar_arrive_expect_tx(&sh->sf, (uint32_t)(2 * T * L.sfrow));
        sm100::tma_load_4d(sfs, &tmS, 4 * kb0, T * m, 0, (int32_t)e, &sh->sf);
      }
    }
    __syncwarp();
    // Every stage of the CTA's K range is issued at once (the ring holds
    // them all for the configured shapes; a slot's later uses wait for its
    // empty barrier).
    for (int kt = 0; kt < nt && valid; ++kt) {
      const int s = kt % kRing;
      if (s % kProducers1 != pidx) continue;
      const uint32_t ph = (kt / kRing) & 1;
      if (!sm100::mbar_wait(&sh->empty[s], ph ^ 1, a.err, 41)) break;
      if (leader) {
        sm100::mbar_arrive_expect_tx(&sh->full[s], (uint32_t)L.stage);
        sm100::tma_load_4d(ring + s * L.stage, &tmW, 32 * kb0 + 128 * kt, T * m, 0, (int32_t)e, &sh->full[s]);
      }
      __syncwarp();
    }
    if (warp == 0) {
      pdl_trigger();   // the down launch may start its prefetch now
      // The weight scales into TMEM (lane quadrant 0, the only one
      // accumulator row 0 reads), in parallel with the quantization of the
      // hidden vector by the epilogue warps.
      if (valid && sm100::mbar_wait(&sh->sf, 0, a.err, 48))
        st_weight_scales_rows16(tmem + pl.sfb1, sfs, L.sfrow, N1, nkb, lane);
      sm100::tmem_st_wait();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&sh->bready);
    }
  } else if (warp == 1) {
    const bool leader = sm100::elect_one();
    const uint32_t idesc = sm100::idesc_nvf4((uint32_t)N1);
    bool ok = sm100::mbar_wait(&sh->bready, 0, a.err, 42);
    sm100::tc_fence_after();
    for (int kt = 0; kt < nt && ok && valid; ++kt) {
      const int s = kt % kRing;
      const uint32_t ph = (kt / kRing) & 1;
      if (!sm100::mbar_wait(&sh->full[s], ph, a.err, 43)) { ok = false; break; }
      sm100::tc_fence_after();
      const int n4 = min(4, nkb - 4 * kt);
      if (leader) {
        for (int kb = 0; kb < n4; ++kb) {
          const int kk = 4 * kt + kb;
          const uint64_t ad = sm100::sdesc_k_sw128(sm100::smem_u32(tokA + kt * 1024) + kb * 32);
          const uint64_t bd = sm100::sdesc_k_sw128(sm100::smem_u32(ring + s * L.stage) + kb * 32);
          sm100::tc_mma_nvf4(tmem, ad, bd, idesc, tmem + pl.sfa1 + 4 * kk, tmem + pl.sfb1 + 8 * kk, kk ? 1u : 0u);
        }
        sm100::tc_commit(&sh->empty[s]);
      }
      __syncwarp();
    }
    if (leader) sm100::tc_commit(&sh->accum);
    __syncwarp();
  } else {
    // ---- warps 2-5: quantize, token scales into TMEM, then the epilogue
    const int t = tid - 64;
    const uint32_t qaddr = (uint32_t)(32 * (warp & 3)) << 16;
    const bool hid_ok = sm100::mbar_wait(&sh->hid, 0, a.err, 44);
    uint32_t key = 0;
    if (hid_ok) {
      for (int i = t; i < H / 8; i += 128) {
        const uint4 u = reinterpret_cast<const uint4*>(hid)[i];
        const __nv_bfloat16* v8 = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
        for (int q = 0; q < 8; ++q) key = max(key, In<AEOQ_BF16>::abs_key(v8[q]));
      }
    }
    key = block_max128(key, t, sh->red);
    const float ts = nvfp4_tensor_scale<AEOQ_BF16>(In<AEOQ_BF16>::key_to_f(key));
    for (int bl = t; bl < 4 * nkb; bl += 128) {
      const uint4* src = reinterpret_cast<const uint4*>(hid + 16 * (4 * kb0 + bl));
      float v[16];
      unpack16(src[0], src[1], v);
      quant_block_row0(v, ts, bl, tokA, tok);
    }
    sm100::fence_proxy_async_smem();   // token tiles: generic writes -> MMA reads
    asm volatile("bar.sync 2, 128;" ::: "memory");
    if (warp == 4) st_token_scales(tmem + qaddr + pl.sfa1, tok, nkb, lane);
    sm100::tmem_st_wait();
    sm100::tc_fence_before();
    __syncwarp();
    if (lane == 0) sm100::mbar_arrive(&sh->bready);
    alpha = ts * load_scalar_f(a.gu_ts, a.gu_ts_dt);
    const bool ok = sm100::mbar_wait(&sh->accum, 0, a.err, 46);
    sm100::tc_fence_after();
    if (warp == 4) read_row0(tmem, N1, ok && valid, dv, lane);
  }
  // TMEM is released before any wait on another CTA: a CTA blocked in
  // tcgen05.alloc behind this one must never be what this one waits for.
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, (uint32_t)pl.cols1);
  }
  // The K parts of a tile form one cluster: rank 0 adds the parts' rows (in
  // part order, from each CTA's shared memory) and finishes the tile.
  sm100::cluster_sync();
  if (warp >= 2 && warp < 6 && sm100::cluster_ctarank() == 0) {   // the four epilogue warps
    const int t = tid - 64;
    uint32_t hkey = 0;
    if (t < T) {
      float g = 0.0f, u = 0.0f;
      for (int pp = 0; pp < pl.parts; ++pp) {
        const float gp = sm100::ld_dsmem_f32(sm100::dsmem_addr(dv + t, (uint32_t)pp));
        const float up = sm100::ld_dsmem_f32(sm100::dsmem_addr(dv + T + t, (uint32_t)pp));
        g = pp ? g + gp : gp;
        u = pp ? u + up : up;
      }
      const float yg = bf16r(g * alpha), yu = bf16r(u * alpha);
      const __nv_bfloat16 hv = __float2bfloat16_rn(bf16r(gelu_tanh(yg)) * yu);
      a.h[(int64_t)j * I + (int64_t)T * m + t] = hv;
      hkey = In<AEOQ_BF16>::abs_key(hv);
    }
    hkey = block_max128(hkey, t, sh->red);
    if (t == 0) {
      a.hmax[(int64_t)j * pl.tiles + m] = hkey;
    }
  }
  sm100::cluster_sync();   // every part's row has been read
}

// ------------------------------------------------------------------ launch 2
__global__ void __launch_bounds__(kThreads, 1)
    decode_down_tc_kernel(const __grid_constant__ CUtensorMap tmD, const Args a, const Plan pl) {
  extern __shared__ __align__(1024) uint8_t dsm[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  const L2 L(pl);
  uint8_t* tokA = base + L.a;
  uint8_t* btile = base + L.b;
  uint8_t* sfs = base + L.sf;
  uint8_t* tok = base + L.tok;
  float* dv = reinterpret_cast<float*>(base + L.dv);
  Bars2* sh = reinterpret_cast<Bars2*>(base + L.bars);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t2 = blockIdx.x, j = blockIdx.y;
  const int H = pl.H, I = pl.I, N2 = pl.N2, kb2 = I / 64, nt = (kb2 + 3) / 4;

  if (tid == 0) {
    sm100::mbar_init(&sh->full, 1);
    sm100::mbar_init(&sh->bready, 4);   // the four epilogue warps
    sm100::mbar_init(&sh->accum, 1);
    sm100::fence_barrier_init();
    sm100::prefetch_tmap(&tmD);
  }
  __syncthreads();
  // The ids, the down weights and their scales do not depend on launch 1.
  const int64_t e = load_index(a.ids, a.ids_dt, j);
  const bool valid = e >= 0 && e < pl.E;
  // Loads spread over warps 0, 2, 3, 4, 5 (one warp's copies complete one
  // after another); warp 0 posts the expected bytes. A copy that completes
  // first leaves the transaction count below zero until then.
  if (valid && warp != 1) {
    const int pw = warp == 0 ? 0 : warp - 1;   // 0..4
    const int32_t row0 = (int32_t)(e * H + (int64_t)N2 * t2);
    if (sm100::elect_one()) {
      if (pw == 0) {
        sm100::mbar_arrive_expect_tx(&sh->full, (uint32_t)(nt * N2 * 128 + N2 * L.sfrow));
        bulk_g2s(sfs, a.d_sf + (int64_t)row0 * L.sfrow, (uint32_t)(N2 * L.sfrow), &sh->full);
      }
      for (int kt = 0; kt < nt; ++kt)
        if ((kt + 1) % 5 == pw) sm100::tma_load_2d(btile + kt * N2 * 128, &tmD, 128 * kt, row0, &sh->full);
    }
    __syncwarp();
  }
  // May wait until a launch-1 CTA on this SM releases its columns.
  if (warp == 1) sm100::tmem_alloc(&sh->tmem, (uint32_t)pl.cols2);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = sh->tmem;

  if (warp == 1) {
    const bool leader = sm100::elect_one();
    bool ok = sm100::mbar_wait(&sh->bready, 0, a.err, 51);
    if (valid) ok = ok && sm100::mbar_wait(&sh->full, 0, a.err, 52);
    sm100::tc_fence_after();
    if (ok && valid && leader) {
      const uint32_t idesc = sm100::idesc_nvf4((uint32_t)N2);
      for (int kb = 0; kb < kb2; ++kb) {
        const uint64_t ad = sm100::sdesc_k_sw128(sm100::smem_u32(tokA + (kb >> 2) * 1024) + (kb & 3) * 32);
        const uint64_t bd = sm100::sdesc_k_sw128(sm100::smem_u32(btile + (kb >> 2) * N2 * 128) + (kb & 3) * 32);
        sm100::tc_mma_nvf4(tmem, ad, bd, idesc, tmem + pl.sfa2 + 4 * kb, tmem + pl.sfb2 + (N2 > 128 ? 8 : 4) * kb,
                           kb ? 1u : 0u);
      }
    }
    if (leader) sm100::tc_commit(&sh->accum);
    __syncwarp();
  } else if (warp >= 2) {
    const int t = tid - 64;
    const uint32_t qaddr = (uint32_t)(32 * (warp & 3)) << 16;
    if (valid && sm100::mbar_wait(&sh->full, 0, a.err, 53)) {
      if (warp == 4) {
        if (pl.N2 > 128) st_weight_scales_rows<2>(tmem + qaddr + pl.sfb2, sfs, L.sfrow, N2, kb2, lane);
        else st_weight_scales_rows<1>(tmem + qaddr + pl.sfb2, sfs, L.sfrow, N2, kb2, lane);
      }
    }
    pdl_wait();   // launch 1 complete: h and the maxima are visible
    // this thread's first h block is loaded alongside the maxima (one round trip)
    uint4 h0 = make_uint4(0u, 0u, 0u, 0u), h1 = h0;
    if (t < I / 16) {
      const uint4* src = reinterpret_cast<const uint4*>(a.h + (int64_t)j * I + 16 * t);
      h0 = __ldcg(src);
      h1 = __ldcg(src + 1);
    }
    uint32_t key = 0;
    const int n_parts = pl.k * pl.tiles;
    for (int i = t; i < n_parts; i += 128) key = max(key, __ldcg(a.hmax + i));
    key = block_max128(key, t, sh->red);
    const float ts = nvfp4_tensor_scale<AEOQ_BF16>(In<AEOQ_BF16>::key_to_f(key));
    for (int bl = t; bl < I / 16; bl += 128) {
      if (bl != t) {
        const uint4* src = reinterpret_cast<const uint4*>(a.h + (int64_t)j * I + 16 * bl);
        h0 = __ldcg(src);
        h1 = __ldcg(src + 1);
      }
      float v[16];
      unpack16(h0, h1, v);
      quant_block_row0(v, ts, bl, tokA, tok);
    }
    sm100::fence_proxy_async_smem();
    asm volatile("bar.sync 2, 128;" ::: "memory");
    if (warp == 4) st_token_scales(tmem + qaddr + pl.sfa2, tok, kb2, lane);
    sm100::tmem_st_wait();
    sm100::tc_fence_before();
    __syncwarp();
    if (lane == 0) sm100::mbar_arrive(&sh->bready);
    const float alpha = ts * load_scalar_f(a.d_ts, a.d_ts_dt);
    const float wj = __bfloat162float(a.topw[j]);
    const bool ok = sm100::mbar_wait(&sh->accum, 0, a.err, 54);
    sm100::tc_fence_after();
    if (warp == 4) read_row0(tmem, N2, ok && valid, dv, lane);
    asm volatile("bar.sync 2, 128;" ::: "memory");
    for (int i = t; i < N2; i += 128) dv[i] = bf16r(bf16r(dv[i] * alpha) * wj);
  }
  // TMEM is released before any wait on another CTA (see launch 1).
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, (uint32_t)pl.cols2);
  }
  // The k experts of a row tile form one cluster: CTA rank r sums rows
  // [r*R, r*R + R) over the k CTAs' shared memory in expert order (f32, one
  // rounding) and writes them.
  sm100::cluster_sync();
  if (warp >= 2) {
    const int t = tid - 64;
    const int R = (N2 + pl.k - 1) / pl.k, r0 = (int)sm100::cluster_ctarank() * R;
    for (int i = r0 + t; i < min(N2, r0 + R); i += 128) {
      float s = 0.0f;
      for (int jj = 0; jj < pl.k; ++jj) s += sm100::ld_dsmem_f32(sm100::dsmem_addr(dv + i, (uint32_t)jj));
      a.out[(int64_t)N2 * t2 + i] = __float2bfloat16_rn(s);
    }
  }
  sm100::cluster_sync();   // every CTA's rows have been read
}

constexpr int kSmemLimit = 232448 - 1024;

bool plan_for(int64_t k, int64_t H, int64_t I, Plan& p) {
  // H % 256: the gate_up scale rows (H/16 bytes) are a TMA pitch, a multiple of 16
  // k <= 8 and parts <= 8: both are cluster extents (portable cluster size)
  if (k < 1 || k > 8 || H <= 0 || I <= 0 || H % 256 || I % 64 || H > 8192 || I > 4096) return false;
  p = Plan{};
  p.H = (int)H; p.I = (int)I; p.k = (int)k;
  for (int t = 128; t >= 8; t -= 8)
    if (I % t == 0) { p.T = t; break; }
  p.tiles = (int)(I / p.T);
  const int kbt = (int)(H / 64);
  // K parts: enough CTAs to cover the SMs once, each part a multiple of 4 steps
  int parts = (int)std::max<int64_t>(1, std::min<int64_t>(std::min<int64_t>(148 / (k * p.tiles), kbt / 4), 8));
  for (;; ++parts) {
    p.Q = rup((kbt + parts - 1) / parts, 4);
    p.parts = (kbt + p.Q - 1) / p.Q;
    p.sfa1 = rup(2 * p.T, 32);
    p.sfb1 = p.sfa1 + rup(4 * p.Q, 32);
    if (p.sfb1 + 8 * p.Q <= 512) break;
    if (p.Q <= 4 || parts >= 8) return false;
  }
  p.cols1 = (p.sfb1 + 8 * p.Q <= 256) ? 256 : 512;
  const int kb2 = (int)(I / 64);
  // 128-row down tiles: a launch-2 CTA (about 58 KB of shared memory, at
  // most 256 TMEM columns) fits beside a launch-1 CTA and prefetches its
  // weights while launch 1 runs; two of them share an SM afterwards.
  p.N2 = 128;
  auto need2 = [&](int n2) {
    return n2 + rup(4 * kb2, 32) + (n2 > 128 ? 8 * rup(kb2, 4) : 4 * rup(kb2, 8));
  };
  if (need2(p.N2) > 512) return false;
  p.sfa2 = p.N2;
  p.sfb2 = p.sfa2 + rup(4 * kb2, 32);
  p.cols2 = need2(p.N2) <= 256 ? 256 : 512;
  return L1(p).bytes + 1024 <= kSmemLimit && L2(p).bytes + 1024 <= kSmemLimit;
}

struct Ws {
  uint32_t* hmax;
  __nv_bfloat16* h;
  size_t bytes;
};

Ws layout(void* base, const Plan& p) {
  char* b = reinterpret_cast<char*>(base);
  auto al = [](size_t v) { return (v + 255) / 256 * 256; };
  Ws w{};
  size_t o = 0;
  w.hmax = reinterpret_cast<uint32_t*>(b + o); o += al((size_t)p.k * p.tiles * 4);
  w.h = reinterpret_cast<__nv_bfloat16*>(b + o); o += al((size_t)p.k * p.I * 2);
  w.bytes = o;
  return w;
}

}  // namespace dtc
}  // namespace aeoq

using namespace aeoq;


extern "C" int aeoq_moe_nvfp4_decode_tc_supported(int64_t top_k, int64_t hidden, int64_t inter) {
  dtc::Plan p;
  return dtc::plan_for(top_k, hidden, inter, p) ? 1 : 0;
}

extern "C" size_t aeoq_moe_nvfp4_decode_tc_workspace_size(int64_t top_k, int64_t hidden, int64_t inter) {
  dtc::Plan p;
  if (!dtc::plan_for(top_k, hidden, inter, p)) return 0;
  return dtc::layout(nullptr, p).bytes;
}

extern "C" int aeoq_moe_nvfp4_decode_tc(const void* hidden, const void* top_k_index, int idx_dtype,
                                        const void* top_k_weights, int64_t top_k, const uint8_t* gate_up,
                                        const uint8_t* gate_up_sf, const void* gate_up_ts, int gate_up_ts_dtype,
                                        const uint8_t* down, const uint8_t* down_sf, const void* down_ts,
                                        int down_ts_dtype, int64_t num_experts, int64_t hidden_dim, int64_t inter_dim,
                                        void* out, void* workspace, size_t workspace_bytes, int* err_word,
                                        void* stream) {
  dtc::Plan pl;
  AEOQ_REQUIRE(dtc::plan_for(top_k, hidden_dim, inter_dim, pl), AEOQ_ERR_INVALID,
               "moe_decode_tc: unsupported shape (top_k=%lld hidden=%lld inter=%lld)", (long long)top_k,
               (long long)hidden_dim, (long long)inter_dim);
  AEOQ_REQUIRE(num_experts > 0, AEOQ_ERR_INVALID, "moe_decode_tc: num_experts must be positive");
  AEOQ_REQUIRE(idx_dtype == AEOQ_I32 || idx_dtype == AEOQ_I64, AEOQ_ERR_INVALID, "moe_decode_tc: int32/int64 ids");
  AEOQ_REQUIRE(hidden && top_k_index && top_k_weights && gate_up && gate_up_sf && gate_up_ts && down && down_sf &&
                   down_ts && out && err_word,
               AEOQ_ERR_INVALID, "moe_decode_tc: null pointer");
  AEOQ_REQUIRE((uintptr_t)hidden % 16 == 0 && (uintptr_t)gate_up % 16 == 0 && (uintptr_t)down % 16 == 0 &&
                   (uintptr_t)gate_up_sf % 16 == 0 && (uintptr_t)down_sf % 16 == 0,
               AEOQ_ERR_INVALID, "moe_decode_tc: operands must be 16-byte aligned");
  pl.E = num_experts;
  const size_t need = dtc::layout(nullptr, pl).bytes;
  AEOQ_REQUIRE(workspace && workspace_bytes >= need && (uintptr_t)workspace % 256 == 0, AEOQ_ERR_WORKSPACE,
               "moe_decode_tc: workspace of %zu bytes (256-aligned) needed, %zu given",
               need, workspace_bytes);
  const int64_t E = num_experts, H = hidden_dim, I = inter_dim;
  cudaStream_t st = (cudaStream_t)stream;
  CUtensorMap tw, ts, td;
  {
    const int64_t dw[4] = {H / 2, I, 2, E}, sw[3] = {H / 2, I * (H / 2), 2 * I * (H / 2)};
    const int bw[4] = {128, pl.T, 2, 1};
    int rc = make_tmap_nd(&tw, gate_up, 4, dw, sw, bw, true);
    if (rc) return rc;
    const int64_t ds[4] = {H / 16, I, 2, E}, ss[3] = {H / 16, I * (H / 16), 2 * I * (H / 16)};
    const int bs[4] = {4 * pl.Q, pl.T, 2, 1};
    rc = make_tmap_nd(&ts, gate_up_sf, 4, ds, ss, bs, false);
    if (rc) return rc;
  }
  int rc = 0;
  rc = make_tmap_bytes(&td, down, E * H, I / 2, I / 2, 128, pl.N2, true);
  if (rc) return rc;
  dtc::Ws w = dtc::layout(workspace, pl);
  dtc::Args a{};
  a.hidden = reinterpret_cast<const __nv_bfloat16*>(hidden);
  a.ids = top_k_index; a.ids_dt = idx_dtype;
  a.topw = reinterpret_cast<const __nv_bfloat16*>(top_k_weights);
  a.gu_ts = gate_up_ts; a.gu_ts_dt = gate_up_ts_dtype;
  a.d_sf = down_sf; a.d_ts = down_ts; a.d_ts_dt = down_ts_dtype;
  a.hmax = w.hmax; a.h = w.h;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.err = err_word;
  const size_t s1 = dtc::L1(pl).bytes + 1024, s2 = dtc::L2(pl).bytes + 1024;
  // the whole carveout as shared memory, so a launch-2 CTA fits beside a launch-1 CTA
  {
    int rc = func_smem_attr((const void*)dtc::decode_gateup_tc_kernel, s1, 100, "moe_decode_tc (launch 1)");
    if (!rc) rc = func_smem_attr((const void*)dtc::decode_down_tc_kernel, s2, 100, "moe_decode_tc (launch 2)");
    if (rc) return rc;
  }
  cudaLaunchAttribute attr1[2], attr2[2];
  attr1[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr1[0].val.programmaticStreamSerializationAllowed = 1;
  attr1[1].id = cudaLaunchAttributeClusterDimension;   // the K parts of a tile
  attr1[1].val.clusterDim.x = 1;
  attr1[1].val.clusterDim.y = (unsigned)pl.parts;
  attr1[1].val.clusterDim.z = 1;
  attr2[0] = attr1[0];
  attr2[1].id = cudaLaunchAttributeClusterDimension;   // the k experts of a row tile
  attr2[1].val.clusterDim.x = 1;
  attr2[1].val.clusterDim.y = (unsigned)top_k;
  attr2[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t c1 = {};
  c1.gridDim = dim3((unsigned)pl.tiles, (unsigned)pl.parts, (unsigned)top_k);
  c1.blockDim = dim3(dtc::kThreads1);
  c1.dynamicSmemBytes = s1;
  c1.stream = st;
  c1.attrs = attr1;
  c1.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&c1, dtc::decode_gateup_tc_kernel, tw, ts, a, pl);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(AEOQ_ERR_CUDA, "decode_gateup_tc_kernel: %s", cudaGetErrorString(e));
  }
  cudaLaunchConfig_t c2 = c1;
  c2.gridDim = dim3((unsigned)(H / pl.N2), (unsigned)top_k);
  c2.blockDim = dim3(dtc::kThreads);
  c2.dynamicSmemBytes = s2;
  c2.attrs = attr2;
  e = cudaLaunchKernelEx(&c2, dtc::decode_down_tc_kernel, td, a, pl);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(AEOQ_ERR_CUDA, "decode_down_tc_kernel: %s", cudaGetErrorString(e));
  }
  return check_launch("decode_down_tc_kernel");
}
