// The vocab-parallel certified head screen over NCCL, as one C-ABI call a C++ host can make.
//
// Rank r holds rows row0.. of the head (its int4 screen copy, bf16p rows and exceptions, optionally
// the unpacked copy).  The single-device screen (screen_task :460-538, eval_row :1453-1474,
// resc_task :540-571) has exactly two global reductions, so one call is, on the caller's stream:
//   broadcast H from root -> shard bound -> all-reduce max (bound L) -> shard survivors and rescoring
//   (or the shard's full exact head) -> all-reduce max (candidate value) -> shard pick -> all-reduce
//   min (global index; none = -1).
// Every step is an ordinary stream operation, so the whole call can be recorded in a CUDA graph.
// NCCL is loaded on first use (dlopen of libnccl.so.2: in a process that already has NCCL loaded,
// e.g. through PyTorch, that copy is the one used), so the library does not depend on it otherwise.
#include "g4_api.h"
#include "g4_common.cuh"
#include <climits>
#include <cstring>
#include <dlfcn.h>
#include <mutex>
#include <nccl.h>

namespace g4 {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclBroadcast) broadcast = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  bool ok = false;
};

static const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.broadcast = reinterpret_cast<decltype(api.broadcast)>(dlsym(h, "ncclBroadcast"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.broadcast && api.all_reduce && api.error_string;
  });
  return api;
}

static int nccl_check(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return G4_OK;
  return set_error(G4_ERR_CUDA, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
}

// The winners' sentinel (no candidate on any shard) to -1.
__global__ void k_idx_none(int* idx, int M) {
  pdl_wait();
  pdl_trigger();
  const int m = threadIdx.x;
  if (m < M && idx[m] == INT_MAX) idx[m] = -1;
}

}  // namespace g4

using namespace g4;

extern "C" int g4_nccl_get_unique_id(void* id128) {
  G4_REQUIRE(id128, "g4_nccl_get_unique_id: null pointer");
  if (!nccl().ok) return set_error(G4_ERR_UNSUPPORTED, "g4_nccl_get_unique_id: libnccl.so.2 not available");
  ncclUniqueId id;
  if (int rc = nccl_check(nccl().get_unique_id(&id), "ncclGetUniqueId")) return rc;
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(id128, &id, sizeof id);
  return G4_OK;
}

extern "C" int g4_nccl_comm_init(const void* id128, int nranks, int rank, void** comm) {
  G4_REQUIRE(id128 && comm && nranks >= 1 && rank >= 0 && rank < nranks, "g4_nccl_comm_init: bad arguments");
  if (!nccl().ok) return set_error(G4_ERR_UNSUPPORTED, "g4_nccl_comm_init: libnccl.so.2 not available");
  ncclUniqueId id;
  std::memcpy(&id, id128, sizeof id);
  ncclComm_t c = nullptr;
  if (int rc = nccl_check(nccl().comm_init_rank(&c, nranks, id, rank), "ncclCommInitRank")) return rc;
  *comm = c;
  return G4_OK;
}

extern "C" int g4_nccl_comm_destroy(void* comm) {
  G4_REQUIRE(comm, "g4_nccl_comm_destroy: null communicator");
  if (!nccl().ok) return set_error(G4_ERR_UNSUPPORTED, "g4_nccl_comm_destroy: libnccl.so.2 not available");
  return nccl_check(nccl().comm_destroy(static_cast<ncclComm_t>(comm)), "ncclCommDestroy");
}

static size_t round256(size_t b) { return (b + 255) / 256 * 256; }

extern "C" size_t g4_head_screen_dist_ws_bytes(int M, int N, int lim) {
  return round256(g4_head_screen_ws_bytes(M, N, lim)) + 3 * round256(sizeof(float) * (size_t)M);
}

extern "C" int g4_head_screen_dist(void* comm, int root, const uint8_t* W4p, const uint16_t* S4, const float* coef,
                                   const uint8_t* data, const uint8_t* unp, const uint8_t* cb8, const long long* exc_ptr,
                                   const uint16_t* exc_col, const float* exc_delta, int N, int K, int row0, float* H, int M,
                                   int lim, int* out_idx, void* ws, size_t ws_bytes, void* stream) {
  G4_REQUIRE(comm && H && out_idx && ws && M >= 1 && M <= 4, "g4_head_screen_dist: bad arguments");
  G4_REQUIRE(ws_bytes >= g4_head_screen_dist_ws_bytes(M, N, lim), "g4_head_screen_dist: workspace too small");
  G4_REQUIRE(aligned(ws, 256), "g4_head_screen_dist: workspace must be 256-byte aligned");
  if (!nccl().ok) return set_error(G4_ERR_UNSUPPORTED, "g4_head_screen_dist: libnccl.so.2 not available");
  cudaStream_t st = as_stream(stream);
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  const size_t sws = round256(g4_head_screen_ws_bytes(M, N, lim));
  float* L = reinterpret_cast<float*>(static_cast<char*>(ws) + sws);
  float* vmax = reinterpret_cast<float*>(static_cast<char*>(ws) + sws + round256(sizeof(float) * M));
  int* ns = reinterpret_cast<int*>(static_cast<char*>(ws) + sws + 2 * round256(sizeof(float) * M));
  if (int rc = nccl_check(nccl().broadcast(H, H, (size_t)M * K, ncclFloat32, root, c, st), "ncclBroadcast")) return rc;
  if (int rc = g4_head_screen_shard_bound(W4p, S4, coef, N, K, H, M, lim, L, ws, sws, st)) return rc;
  if (int rc = nccl_check(nccl().all_reduce(L, L, M, ncclFloat32, ncclMax, c, st), "ncclAllReduce(bound)")) return rc;
  if (int rc = g4_head_screen_shard_select(coef, data, unp, cb8, exc_ptr, exc_col, exc_delta, N, K, H, M, lim, L, vmax, ns, ws,
                                           sws, st))
    return rc;
  if (int rc = nccl_check(nccl().all_reduce(vmax, vmax, M, ncclFloat32, ncclMax, c, st), "ncclAllReduce(candidate)")) return rc;
  if (int rc = g4_head_screen_shard_pick(N, M, lim, row0, vmax, out_idx, ws, sws, st)) return rc;
  if (int rc = nccl_check(nccl().all_reduce(out_idx, out_idx, M, ncclInt32, ncclMin, c, st), "ncclAllReduce(index)")) return rc;
  if (int rc = launch("k_idx_none", k_idx_none, dim3(1), dim3(32), 0, st, out_idx, M)) return rc;
  return check_launch("g4_head_screen_dist");
}
