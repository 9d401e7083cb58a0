// Expert-parallel dispatch and combine over NCCL, for hosts that bind the
// library without the Python package: the equal-token ("dense") form of
// ep_moe_forward (aeo_quant_b200/bridges/gemma4/expert_parallel.py,
// _ep_dense) in C++.
//
//   aeoq_ep_dispatch   global |hidden| max (all-reduce max) -> the one-GPU
//                      tensor scale -> NVFP4 rows with that scale -> every
//                      rank's rows to every rank (all-gather), the routing
//                      weights likewise, and per destination rank the local
//                      expert ids of each token (all-to-all)
//   aeoq_ep_experts_nvfp4 (moe_forward.cu) the received rows through this
//                      rank's experts
//   aeoq_ep_combine    the partial rows back to their home ranks
//                      (all-to-all) and each token's partials folded in rank
//                      order, bf16 after each add
//
// NCCL is not linked: libnccl.so.2 is opened at the first call (the copy a
// host already loaded, e.g. PyTorch's, when there is one). Only NCCL's
// public, stable C ABI is used: ncclGetUniqueId, ncclCommInitRank,
// ncclCommDestroy, ncclAllReduce, ncclAllGather, ncclSend, ncclRecv,
// ncclGroupStart/End and ncclGetErrorString. Every call is stream-ordered
// on `stream` and nothing synchronises with the host; every rank must pass
// the same T (tokens per rank), as in sequence-sharded prefill.
#include <dlfcn.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace aeoq {
namespace {

// NCCL's public ABI (nccl.h): the unique id is 128 bytes passed by value;
// data types and reduction ops are C enums.
struct NcclUniqueId {
  char internal[128];
};
constexpr int kNcclUint8 = 1, kNcclInt32 = 2, kNcclFloat32 = 7, kNcclBfloat16 = 9;
constexpr int kNcclMax = 2;

struct Nccl {
  int (*get_unique_id)(NcclUniqueId*) = nullptr;
  int (*comm_init_rank)(void**, int, NcclUniqueId, int) = nullptr;
  int (*comm_destroy)(void*) = nullptr;
  int (*all_reduce)(const void*, void*, size_t, int, int, void*, cudaStream_t) = nullptr;
  int (*all_gather)(const void*, void*, size_t, int, void*, cudaStream_t) = nullptr;
  int (*send)(const void*, size_t, int, int, void*, cudaStream_t) = nullptr;
  int (*recv)(void*, size_t, int, int, void*, cudaStream_t) = nullptr;
  int (*group_start)() = nullptr;
  int (*group_end)() = nullptr;
  const char* (*error_string)(int) = nullptr;
  bool ok = false;
};

const Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      return fn != nullptr;
    };
    n.ok = sym(n.get_unique_id, "ncclGetUniqueId") && sym(n.comm_init_rank, "ncclCommInitRank") &&
           sym(n.comm_destroy, "ncclCommDestroy") && sym(n.all_reduce, "ncclAllReduce") &&
           sym(n.all_gather, "ncclAllGather") && sym(n.send, "ncclSend") && sym(n.recv, "ncclRecv") &&
           sym(n.group_start, "ncclGroupStart") && sym(n.group_end, "ncclGroupEnd") &&
           sym(n.error_string, "ncclGetErrorString");
  });
  return n;
}

int nccl_check(int r, const char* what) {
  if (r == 0) return AEOQ_OK;
  const Nccl& n = nccl();
  return set_error(AEOQ_ERR_CUDA, "%s: NCCL error %d (%s)", what, r, n.error_string ? n.error_string(r) : "?");
}

#define AEOQ_NCCL(expr, what)                       \
  do {                                              \
    const int rc_ = nccl_check((expr), (what));      \
    if (rc_ != AEOQ_OK) return rc_;                 \
  } while (0)

size_t al256(size_t b) { return (std::max<size_t>(b, 1) + 255) / 256 * 256; }

// max |x| over n bf16 values as the bits of a non-negative f32 (ordered like
// the floats), one atomicMax per warp.
__global__ void amax_bf16_kernel(const __nv_bfloat16* x, int64_t n, uint32_t* out) {
  float m = 0.0f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(__bfloat162float(x[i])));
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

// The one-GPU tensor scale from the all-reduced amax in bf16, as the Python
// layer computes it (NVFP4EpOps.tensor_scale: bf16(amax) / 2688 clamped at
// 1e-12, where PyTorch divides a GPU tensor by a Python number as a multiply
// by the f32 reciprocal).
__global__ void tensor_scale_kernel(const uint32_t* amax_bits, __nv_bfloat16* ts) {
  const float a = __bfloat162float(__float2bfloat16_rn(__uint_as_float(*amax_bits)));
  const float q = __bfloat162float(__float2bfloat16_rn(a * (1.0f / 2688.0f)));
  *ts = __float2bfloat16_rn(fmaxf(q, 1e-12f));
}

// Per destination rank r and token t: the local id of each of t's experts
// that r owns, else e_loc (dropped by the grouped forward); slot_row[t][r] =
// r * T + t when r owns any of t's experts, else -1 (plan_dense_dispatch).
// placement: null = contiguous blocks of e_loc experts per rank; else
// placement[e] = owning rank, placement[E + e] = local index there.
template <typename Idx>
__global__ void plan_dense_kernel(const Idx* ids, int64_t T, int k, int64_t E, int world, const int32_t* placement,
                                  int32_t* lid, int32_t* slot_row) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const int64_t e_loc = E / world;
  for (int r = 0; r < world; ++r) {
    bool any = false;
    for (int j = 0; j < k; ++j) {
      const int64_t e = (int64_t)ids[t * k + j];
      int32_t v = (int32_t)e_loc;
      if (e >= 0 && e < E) {
        const int dest = placement ? placement[e] : (int)(e / e_loc);
        const int32_t local = placement ? placement[E + e] : (int32_t)(e % e_loc);
        if (dest == r) {
          v = local;
          any = true;
        }
      }
      lid[((int64_t)r * T + t) * k + j] = v;
    }
    slot_row[t * world + r] = any ? (int32_t)(r * T + t) : -1;
  }
}

__global__ void rank_ids_kernel(int32_t* ranks, int64_t T, int world) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < T * world) ranks[i] = (int32_t)(i % world);
}

}  // namespace
}  // namespace aeoq

using namespace aeoq;

extern "C" size_t aeoq_ep_nccl_unique_id_bytes(void) { return sizeof(NcclUniqueId); }

extern "C" int aeoq_ep_nccl_unique_id(void* out, size_t out_bytes) {
  AEOQ_REQUIRE(out && out_bytes >= sizeof(NcclUniqueId), AEOQ_ERR_INVALID, "ep_nccl_unique_id: need %zu bytes",
               sizeof(NcclUniqueId));
  const Nccl& n = nccl();
  AEOQ_REQUIRE(n.ok, AEOQ_ERR_UNSUPPORTED, "ep: libnccl.so.2 not found or incomplete");
  AEOQ_NCCL(n.get_unique_id(static_cast<NcclUniqueId*>(out)), "ep_nccl_unique_id");
  return AEOQ_OK;
}

extern "C" int aeoq_ep_nccl_comm_init(void** comm, int world, int rank, const void* unique_id) {
  AEOQ_REQUIRE(comm && unique_id && world >= 1 && rank >= 0 && rank < world, AEOQ_ERR_INVALID,
               "ep_nccl_comm_init: bad arguments (world %d, rank %d)", world, rank);
  const Nccl& n = nccl();
  AEOQ_REQUIRE(n.ok, AEOQ_ERR_UNSUPPORTED, "ep: libnccl.so.2 not found or incomplete");
  NcclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  AEOQ_NCCL(n.comm_init_rank(comm, world, id, rank), "ep_nccl_comm_init");
  return AEOQ_OK;
}

extern "C" int aeoq_ep_nccl_comm_destroy(void* comm) {
  if (!comm) return AEOQ_OK;
  const Nccl& n = nccl();
  AEOQ_REQUIRE(n.ok, AEOQ_ERR_UNSUPPORTED, "ep: libnccl.so.2 not found or incomplete");
  AEOQ_NCCL(n.comm_destroy(comm), "ep_nccl_comm_destroy");
  return AEOQ_OK;
}

extern "C" size_t aeoq_ep_dispatch_workspace_size(int world, int64_t T, int64_t top_k, int64_t hidden) {
  if (world < 1 || T <= 0 || top_k <= 0 || hidden <= 0) return 0;
  return al256(4) + al256((size_t)T * hidden / 2) + al256((size_t)T * hidden / 16) +
         al256((size_t)world * T * top_k * 4);
}

extern "C" int aeoq_ep_dispatch(void* comm, int world, int rank, const void* hidden, int64_t T, int64_t H,
                                const void* top_k_index, int idx_dtype, const void* top_k_weights, int64_t top_k,
                                int64_t num_experts, const int32_t* placement, uint8_t* recv_packed,
                                uint8_t* recv_sf, int32_t* recv_local_ids, void* recv_weights, void* ts_out,
                                int32_t* slot_row, void* workspace, size_t workspace_bytes, void* stream) {
  const int64_t k = top_k, E = num_experts;
  AEOQ_REQUIRE(comm && world >= 1 && rank >= 0 && rank < world && T >= 0 && H > 0 && H % 16 == 0 && k >= 1 &&
                   k <= 16 && E >= world && E % world == 0,
               AEOQ_ERR_INVALID,
               "ep_dispatch: bad arguments (world %d, rank %d, T %lld, H %lld, top_k %lld, experts %lld; "
               "H a multiple of 16, experts a multiple of world)",
               world, rank, (long long)T, (long long)H, (long long)k, (long long)E);
  AEOQ_REQUIRE(idx_dtype == AEOQ_I32 || idx_dtype == AEOQ_I64, AEOQ_ERR_INVALID, "ep_dispatch: ids must be i32 or i64");
  if (T == 0) return AEOQ_OK;   // every rank holds the same T: none of them joins a collective
  AEOQ_REQUIRE(hidden && top_k_index && top_k_weights && recv_packed && recv_sf && recv_local_ids && recv_weights &&
                   ts_out && slot_row,
               AEOQ_ERR_INVALID, "ep_dispatch: null pointer");
  const size_t need = aeoq_ep_dispatch_workspace_size(world, T, k, H);
  AEOQ_REQUIRE(workspace && workspace_bytes >= need, AEOQ_ERR_WORKSPACE,
               "ep_dispatch: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  AEOQ_REQUIRE((uintptr_t)workspace % 256 == 0, AEOQ_ERR_INVALID, "ep_dispatch: workspace not 256-byte aligned");
  const Nccl& n = nccl();
  AEOQ_REQUIRE(n.ok, AEOQ_ERR_UNSUPPORTED, "ep: libnccl.so.2 not found or incomplete");
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* w = static_cast<uint8_t*>(workspace);
  uint32_t* amax = reinterpret_cast<uint32_t*>(w);
  w += al256(4);
  uint8_t* send_packed = w;
  w += al256((size_t)T * H / 2);
  uint8_t* send_sf = w;
  w += al256((size_t)T * H / 16);
  int32_t* send_lid = reinterpret_cast<int32_t*>(w);

  // the one-GPU tensor scale: max over every rank's tokens
  if (cudaMemsetAsync(amax, 0, 4, st) != cudaSuccess) return check_launch("ep_dispatch");
  const int64_t nel = T * H;
  const int blocks = (int)std::min<int64_t>((nel + 255) / 256, 4 * 148);
  amax_bf16_kernel<<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(hidden), nel, amax);
  AEOQ_NCCL(n.all_reduce(amax, amax, 1, kNcclFloat32, kNcclMax, comm, st), "ep_dispatch (amax all-reduce)");
  tensor_scale_kernel<<<1, 1, 0, st>>>(amax, static_cast<__nv_bfloat16*>(ts_out));
  {
    const int rc = check_launch("ep_dispatch (tensor scale)");
    if (rc) return rc;
  }
  {
    const int rc = aeoq_nvfp4_quantize_with_scale(hidden, AEOQ_BF16, T, H, H, ts_out, send_packed, send_sf, stream);
    if (rc) return rc;
  }
  const int pb = (int)((T + 127) / 128);
  if (idx_dtype == AEOQ_I64)
    plan_dense_kernel<int64_t><<<pb, 128, 0, st>>>(static_cast<const int64_t*>(top_k_index), T, (int)k, E, world,
                                                   placement, send_lid, slot_row);
  else
    plan_dense_kernel<int32_t><<<pb, 128, 0, st>>>(static_cast<const int32_t*>(top_k_index), T, (int)k, E, world,
                                                   placement, send_lid, slot_row);
  {
    const int rc = check_launch("ep_dispatch (plan)");
    if (rc) return rc;
  }
  // every rank's rows and routing weights to every rank; the local ids per
  // destination
  AEOQ_NCCL(n.all_gather(send_packed, recv_packed, (size_t)T * H / 2, kNcclUint8, comm, st), "ep_dispatch (rows)");
  AEOQ_NCCL(n.all_gather(send_sf, recv_sf, (size_t)T * H / 16, kNcclUint8, comm, st), "ep_dispatch (scales)");
  AEOQ_NCCL(n.all_gather(top_k_weights, recv_weights, (size_t)T * k, kNcclBfloat16, comm, st),
            "ep_dispatch (weights)");
  const size_t chunk = (size_t)T * k;
  AEOQ_NCCL(n.group_start(), "ep_dispatch (ids)");
  for (int r = 0; r < world; ++r) {
    const int s1 = n.send(send_lid + r * chunk, chunk, kNcclInt32, r, comm, st);
    const int s2 = n.recv(recv_local_ids + r * chunk, chunk, kNcclInt32, r, comm, st);
    if (s1 || s2) {
      n.group_end();
      return nccl_check(s1 ? s1 : s2, "ep_dispatch (ids)");
    }
  }
  AEOQ_NCCL(n.group_end(), "ep_dispatch (ids)");
  return AEOQ_OK;
}

extern "C" size_t aeoq_ep_combine_workspace_size(int world, int64_t T, int64_t hidden) {
  if (world < 1 || T <= 0 || hidden <= 0) return 0;
  return al256((size_t)world * T * hidden * 2) + al256((size_t)T * world * 4);
}

extern "C" int aeoq_ep_combine(void* comm, int world, int rank, const void* rows, const int32_t* slot_row, int64_t T,
                               int64_t H, void* out, void* workspace, size_t workspace_bytes, void* stream) {
  AEOQ_REQUIRE(comm && world >= 1 && rank >= 0 && rank < world && T >= 0 && H > 0, AEOQ_ERR_INVALID,
               "ep_combine: bad arguments (world %d, rank %d, T %lld, H %lld)", world, rank, (long long)T,
               (long long)H);
  if (T == 0) return AEOQ_OK;
  AEOQ_REQUIRE(rows && slot_row && out, AEOQ_ERR_INVALID, "ep_combine: null pointer");
  const size_t need = aeoq_ep_combine_workspace_size(world, T, H);
  AEOQ_REQUIRE(workspace && workspace_bytes >= need, AEOQ_ERR_WORKSPACE,
               "ep_combine: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  AEOQ_REQUIRE((uintptr_t)workspace % 256 == 0, AEOQ_ERR_INVALID, "ep_combine: workspace not 256-byte aligned");
  const Nccl& n = nccl();
  AEOQ_REQUIRE(n.ok, AEOQ_ERR_UNSUPPORTED, "ep: libnccl.so.2 not found or incomplete");
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* w = static_cast<uint8_t*>(workspace);
  __nv_bfloat16* back = reinterpret_cast<__nv_bfloat16*>(w);
  w += al256((size_t)world * T * H * 2);
  int32_t* ranks = reinterpret_cast<int32_t*>(w);
  // block r of `rows` goes back to rank r; block r of `back` is this rank's
  // tokens as rank r folded them
  const size_t chunk = (size_t)T * H;
  const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(rows);
  AEOQ_NCCL(n.group_start(), "ep_combine");
  for (int r = 0; r < world; ++r) {
    const int s1 = n.send(src + r * chunk, chunk, kNcclBfloat16, r, comm, st);
    const int s2 = n.recv(back + r * chunk, chunk, kNcclBfloat16, r, comm, st);
    if (s1 || s2) {
      n.group_end();
      return nccl_check(s1 ? s1 : s2, "ep_combine");
    }
  }
  AEOQ_NCCL(n.group_end(), "ep_combine");
  rank_ids_kernel<<<(int)((T * world + 255) / 256), 256, 0, st>>>(ranks, T, world);
  {
    const int rc = check_launch("ep_combine");
    if (rc) return rc;
  }
  return aeoq_moe_combine(back, slot_row, ranks, AEOQ_I32, T, world, H, 0, out, stream);
}
