// fms_shard.cu -- the multi-GPU paths of the C ABI: galleries sharded by
// document id over the GPUs of one node, one process (or Julia task) per GPU,
// NCCL over NVLink for the only exchanges.  The reference is single-device, so
// none of this has a counterpart there; each sharded call reproduces what the
// single-device layout driver returns for the whole gallery.
//
//  * Candidates: a compaction kernel reads the (C, B) idxs once, lists the slots
//    whose document this shard holds (in order within 8192-slot ranges) and
//    writes -Inf into every other slot; the
//    scan walks only the list (per-rank work independent of the number of
//    ranks); ncclAllReduce(max) merges the owner-disjoint scores in place and
//    the `neg` fill of globally invalid slots follows.
//  * Packed: every rank scans its contiguous document range; ncclAllGather of
//    the (B_max, nq) score blocks into a staging buffer, then one kernel places
//    every block into the (B_total, nq) result.
//  * INT8 exhaustive top-k: local scan + top-k with global ids; ncclAllGather of
//    the (k, nq) lists; the device merge (score descending, id ascending).
//
// NCCL is loaded at run time (dlopen): the process's already loaded libnccl.so.2
// (torch's, NCCL.jl's) when there is one, so a communicator the caller created
// can be used directly (fms_comm_from_nccl); FMS_NCCL_LIBRARY overrides the
// file.  Nothing here allocates: staging buffers come from the caller's
// workspace, sized by the *_workspace_size queries.
#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>

#include <mutex>

#include "fms_common.cuh"
#include "fms_int8.cuh"
#include "fms_internal.h"

namespace fms {

// ------------------------------------------------------------------ NCCL loader

struct NcclApi {
  ncclResult_t (*getUniqueId)(ncclUniqueId*);
  ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*commDestroy)(ncclComm_t);
  ncclResult_t (*commCount)(const ncclComm_t, int*);
  ncclResult_t (*commUserRank)(const ncclComm_t, int*);
  ncclResult_t (*allReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t);
  ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*groupStart)();
  ncclResult_t (*groupEnd)();
  const char* (*getErrorString)(ncclResult_t);
  bool ok;
};

static NcclApi g_nccl;
static std::once_flag g_nccl_once;
static thread_local ncclResult_t g_last_nccl = ncclSuccess;

static void load_nccl() {
  memset(&g_nccl, 0, sizeof(g_nccl));
  void* h = nullptr;
  const char* env = getenv("FMS_NCCL_LIBRARY");
  if (env && *env) {
    h = dlopen(env, RTLD_NOW | RTLD_LOCAL);
  } else {
    h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the process's own NCCL first
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
  }
  if (!h) return;
#define FMS_SYM(field, name) \
  *reinterpret_cast<void**>(&g_nccl.field) = dlsym(h, name); \
  if (!g_nccl.field) return;
  FMS_SYM(getUniqueId, "ncclGetUniqueId")
  FMS_SYM(commInitRank, "ncclCommInitRank")
  FMS_SYM(commDestroy, "ncclCommDestroy")
  FMS_SYM(commCount, "ncclCommCount")
  FMS_SYM(commUserRank, "ncclCommUserRank")
  FMS_SYM(allReduce, "ncclAllReduce")
  FMS_SYM(allGather, "ncclAllGather")
  FMS_SYM(groupStart, "ncclGroupStart")
  FMS_SYM(groupEnd, "ncclGroupEnd")
  FMS_SYM(getErrorString, "ncclGetErrorString")
#undef FMS_SYM
  g_nccl.ok = true;
}

static const NcclApi* nccl() {
  std::call_once(g_nccl_once, load_nccl);
  return g_nccl.ok ? &g_nccl : nullptr;
}

static int nccl_status(ncclResult_t r) {
  if (r == ncclSuccess) return FMS_OK;
  g_last_nccl = r;
  return FMS_ERR_NCCL;
}

// ------------------------------------------------------------------ kernels

// Candidate slots of this shard: unit u (= b * C + c) is owned when idxs[u] is
// one of the shard's documents id_lo .. id_lo + n_local - 1.  A block takes a
// contiguous range of COMPACT_TILE units, lists its owned units in order into
// one reserved output range (one atomic per block), so the list keeps runs of
// the same query together (the scan reloads its query tile only when the
// query changes); blocks land in any order, which changes nothing in the
// results (every unit's output is independent).  The other units get -Inf,
// which loses the max-merge.
constexpr int COMPACT_THREADS = 1024;
constexpr int COMPACT_ITEMS = 8;
constexpr int COMPACT_TILE = COMPACT_THREADS * COMPACT_ITEMS;

__global__ void __launch_bounds__(COMPACT_THREADS)
shard_compact_kernel(const int32_t* __restrict__ idxs, int64_t n, int64_t id_lo, int64_t n_local,
                     int32_t* __restrict__ list, int32_t* __restrict__ count, float* __restrict__ S) {
  __shared__ int32_t warp_tot[COMPACT_THREADS / 32];
  __shared__ int32_t base_s;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int64_t t0 = (int64_t)blockIdx.x * COMPACT_TILE; t0 < n; t0 += (int64_t)gridDim.x * COMPACT_TILE) {
    // thread k holds units t0 + k*ITEMS .. + ITEMS-1 (consecutive, in order)
    const int64_t u0 = t0 + (int64_t)threadIdx.x * COMPACT_ITEMS;
    uint32_t own = 0u;
#pragma unroll
    for (int j = 0; j < COMPACT_ITEMS; ++j) {
      const int64_t u = u0 + j;
      if (u < n) {
        const int64_t d = (int64_t)idxs[u] - (id_lo - 1);
        if (d >= 1 && d <= n_local) own |= 1u << j;
        else S[u] = -INFINITY;
      }
    }
    const int cnt = __popc(own);
    // block-wide exclusive scan of the per-thread counts
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_tot[w] = incl;
    __syncthreads();
    if (w == 0) {
      const int t = warp_tot[lane];
      int wi = t;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, wi, o);
        if (lane >= o) wi += v;
      }
      warp_tot[lane] = wi - t;  // exclusive offset of each warp
      if (lane == 31) base_s = wi > 0 ? atomicAdd(count, wi) : 0;
    }
    __syncthreads();
    int pos = base_s + warp_tot[w] + incl - cnt;
#pragma unroll
    for (int j = 0; j < COMPACT_ITEMS; ++j)
      if ((own >> j) & 1u) list[pos++] = (int32_t)(u0 + j);
    __syncthreads();  // warp_tot / base_s are rewritten by the next tile
  }
}

// First document of every rank's block (rank r: v[r] .. v[r+1]-1), passed by
// value so that no host-to-device copy is needed.
constexpr int MAX_RANKS = 128;
struct RankOffsets {
  int32_t v[MAX_RANKS + 1];
};

// Staging (nranks, nq, Bmax) of all-gathered packed score blocks -> S (nq, B_total)
// (torch order; Julia (B_total, nq)).
__global__ void packed_place_kernel(const float* __restrict__ stage, int nranks, int nq, int Bmax,
                                    const RankOffsets offs, int64_t B_total,
                                    float* __restrict__ S) {
  const int64_t n = (int64_t)nq * B_total;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t qi = i / B_total, b = i - qi * B_total;
    int r = 0;  // owning rank: offsets ascending, few ranks
    while (r + 1 < nranks && b >= offs.v[r + 1]) ++r;
    S[i] = stage[((int64_t)r * nq + qi) * Bmax + (b - offs.v[r])];
  }
}

static unsigned grid_for(int64_t work, int per_block) {
  int64_t g = (work + per_block - 1) / per_block;
  const int64_t cap = (int64_t)device_sm_count() * 8;
  if (g > cap) g = cap;
  return (unsigned)(g < 1 ? 1 : g);
}

static size_t al256(size_t x) { return (x + 255) / 256 * 256; }

size_t shard_list_bytes(int64_t nslots) { return al256(4) + al256((size_t)nslots * 4 + 4); }

cudaError_t launch_shard_compact(const int32_t* idxs, int64_t nslots, int64_t id_lo, int64_t n_local,
                                 void* ws, float* S, const int32_t** list, const int32_t** count,
                                 cudaStream_t s) {
  int32_t* cnt = static_cast<int32_t*>(ws);
  int32_t* lst = reinterpret_cast<int32_t*>(static_cast<char*>(ws) + al256(4));
  cudaError_t e = cudaMemsetAsync(cnt, 0, 4, s);
  if (e != cudaSuccess) return e;
  if (nslots > 0) {
    int64_t blocks = (nslots + COMPACT_TILE - 1) / COMPACT_TILE;
    const int64_t cap = (int64_t)device_sm_count() * 2;
    if (blocks > cap) blocks = cap;
    shard_compact_kernel<<<(unsigned)blocks, COMPACT_THREADS, 0, s>>>(idxs, nslots, id_lo, n_local,
                                                                       lst, cnt, S);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  *list = lst;
  *count = cnt;
  return cudaSuccess;
}

}  // namespace fms

using namespace fms;

struct fms_comm {
  ncclComm_t nc;
  int owned;  // created here (destroyed by fms_comm_destroy) or borrowed
  int nranks, rank;
};

extern "C" {

int fms_nccl_available(void) { return nccl() != nullptr ? 1 : 0; }

const char* fms_last_nccl_error(void) {
  const NcclApi* a = nccl();
  if (!a) return "NCCL library not found (libnccl.so.2; FMS_NCCL_LIBRARY overrides)";
  return a->getErrorString(g_last_nccl);
}

int fms_comm_unique_id(void* id) {
  const NcclApi* a = nccl();
  if (!a) return FMS_ERR_UNSUPPORTED;
  if (!id) return FMS_ERR_INVALID;
  ncclUniqueId u;
  const int st = nccl_status(a->getUniqueId(&u));
  if (st == FMS_OK) memcpy(id, &u, sizeof(u));
  return st;
}

int fms_comm_init(fms_comm_t* comm, int nranks, int rank, const void* id) {
  const NcclApi* a = nccl();
  if (!a) return FMS_ERR_UNSUPPORTED;
  if (!comm || !id || nranks < 1 || rank < 0 || rank >= nranks) return FMS_ERR_INVALID;
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclComm_t nc = nullptr;
  const int st = nccl_status(a->commInitRank(&nc, nranks, u, rank));
  if (st != FMS_OK) return st;
  fms_comm* c = new (std::nothrow) fms_comm;
  if (!c) {
    a->commDestroy(nc);
    return FMS_ERR_INVALID;
  }
  c->nc = nc;
  c->owned = 1;
  c->nranks = nranks;
  c->rank = rank;
  *comm = c;
  return FMS_OK;
}

int fms_comm_from_nccl(fms_comm_t* comm, void* nccl_comm) {
  const NcclApi* a = nccl();
  if (!a) return FMS_ERR_UNSUPPORTED;
  if (!comm || !nccl_comm) return FMS_ERR_INVALID;
  ncclComm_t nc = static_cast<ncclComm_t>(nccl_comm);
  int n = 0, r = 0;
  int st = nccl_status(a->commCount(nc, &n));
  if (st == FMS_OK) st = nccl_status(a->commUserRank(nc, &r));
  if (st != FMS_OK) return st;
  fms_comm* c = new (std::nothrow) fms_comm;
  if (!c) return FMS_ERR_INVALID;
  c->nc = nc;
  c->owned = 0;
  c->nranks = n;
  c->rank = r;
  *comm = c;
  return FMS_OK;
}

int fms_comm_destroy(fms_comm_t comm) {
  if (!comm) return FMS_OK;
  int st = FMS_OK;
  if (comm->owned) {
    const NcclApi* a = nccl();
    if (a) st = nccl_status(a->commDestroy(comm->nc));
  }
  delete comm;
  return st;
}

int fms_comm_size(fms_comm_t comm, int* nranks, int* rank) {
  if (!comm) return FMS_ERR_INVALID;
  if (nranks) *nranks = comm->nranks;
  if (rank) *rank = comm->rank;
  return FMS_OK;
}

// --------------------------------------------------------------- candidates

size_t fms_candidates_shard_workspace_size(int B, int C) {
  if (B < 0 || C < 0) return 0;
  return shard_list_bytes((int64_t)B * C);
}

size_t fms_sharded_candidates_workspace_size(int B, int C) {
  return fms_candidates_shard_workspace_size(B, C);
}

int fms_sharded_candidates_fwd(fms_comm_t comm, int dtype, const void* Q, const void* gallery_shard,
                               const int32_t* idxs, const uint8_t* qmask,
                               const uint8_t* dmask_shard, int dim, int Tq, int B, int Td,
                               int64_t N_local, int C, int64_t id_lo, int64_t N_global, double neg,
                               int normalize, float* S, void* workspace, size_t ws_bytes,
                               fms_stream_t stream) {
  const NcclApi* a = nccl();
  if (!a) return FMS_ERR_UNSUPPORTED;
  if (!comm) return FMS_ERR_INVALID;
  if (dtype != FMS_F32 && dtype != FMS_F16 && dtype != FMS_BF16) return FMS_ERR_DTYPE;
  if (N_global < N_local || id_lo < 1 || id_lo - 1 + N_local > N_global) return FMS_ERR_INVALID;
  int st = fms_candidates_shard_fwd(dtype, Q, gallery_shard, idxs, qmask, dmask_shard, dim, Tq, B,
                                    Td, N_local, C, id_lo, normalize, S, workspace, ws_bytes, stream);
  if (st != FMS_OK) return st;
  const int64_t n = (int64_t)B * C;
  if (n == 0) return FMS_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (comm->nranks > 1) {
    st = nccl_status(a->allReduce(S, S, (size_t)n, ncclFloat32, ncclMax, comm->nc, s));
    if (st != FMS_OK) return st;
  }
  // MaxSim{T} stores T(neg) (types.jl:34-37); the caller passes it already in T
  return fms_candidates_finalize_neg(idxs, N_global, C, B, neg, S, stream);
}

// ------------------------------------------------------------------ packed

size_t fms_sharded_packed_workspace_size(int nranks, int nq, int B_max) {
  if (nranks < 1 || nq < 0 || B_max < 0) return 0;
  const size_t blk = (size_t)nq * (size_t)B_max * 4;
  return al256(blk) + al256(blk * (size_t)nranks);
}

int fms_sharded_packed_fwd(fms_comm_t comm, int dtype, const void* Qs, const void* tokens_shard,
                           const int32_t* cu_shard, const uint8_t* qmask, int dim, int Tq, int nq,
                           const int32_t* counts, int64_t ntok_local, int normalize, float* S,
                           void* workspace, size_t ws_bytes, fms_stream_t stream) {
  const NcclApi* a = nccl();
  if (!a) return FMS_ERR_UNSUPPORTED;
  if (!comm || !counts) return FMS_ERR_INVALID;
  if (dtype != FMS_F32 && dtype != FMS_F16 && dtype != FMS_BF16) return FMS_ERR_DTYPE;
  const int R = comm->nranks;
  if (R > MAX_RANKS) return FMS_ERR_INVALID;
  int Bmax = 0;
  int64_t Btot = 0;
  for (int r = 0; r < R; ++r) {
    if (counts[r] < 0) return FMS_ERR_INVALID;
    Bmax = counts[r] > Bmax ? counts[r] : Bmax;
    Btot += counts[r];
  }
  const int Bl = counts[comm->rank];
  if ((int64_t)nq * Btot > 0 && !S) return FMS_ERR_INVALID;
  const size_t need = fms_sharded_packed_workspace_size(R, nq, Bmax);
  if (!workspace || ws_bytes < need) return FMS_ERR_WORKSPACE;
  const size_t blk = (size_t)nq * (size_t)Bmax * 4;
  float* local = static_cast<float*>(workspace);
  float* stage = reinterpret_cast<float*>(static_cast<char*>(workspace) + al256(blk));
  cudaStream_t s = (cudaStream_t)stream;
  // the local block (nq, Bmax), columns past this rank's count unused
  int st = FMS_OK;
  if (Bl > 0) {
    // scan straight into a (nq, Bl) block, then widen the rows to Bmax in place
    st = fms_packed_fwd(dtype, Qs, tokens_shard, cu_shard, qmask, dim, Tq, nq, Bl, ntok_local,
                        normalize, local, nullptr, stream);
    if (st != FMS_OK) return st;
    if (Bl != Bmax && nq > 1) {
      cudaError_t e = cudaMemcpy2DAsync(stage, (size_t)Bmax * 4, local, (size_t)Bl * 4,
                                        (size_t)Bl * 4, (size_t)nq, cudaMemcpyDeviceToDevice, s);
      if (e != cudaSuccess) return (int)e;
      e = cudaMemcpyAsync(local, stage, blk, cudaMemcpyDeviceToDevice, s);
      if (e != cudaSuccess) return (int)e;
    }
  }
  if ((int64_t)nq * Bmax == 0) return FMS_OK;
  st = nccl_status(a->allGather(local, stage, (size_t)nq * Bmax, ncclFloat32, comm->nc, s));
  if (st != FMS_OK) return st;
  RankOffsets offs;
  offs.v[0] = 0;
  for (int r = 0; r < R; ++r) offs.v[r + 1] = offs.v[r] + counts[r];
  packed_place_kernel<<<grid_for((int64_t)nq * Btot, 256), 256, 0, s>>>(stage, R, nq, Bmax, offs,
                                                                          Btot, S);
  return (int)cudaGetLastError();
}

// ---------------------------------------------------------------- INT8 top-k

size_t fms_sharded_int8_topk_workspace_size(int nranks, int nq, int64_t N_local, int k) {
  if (nranks < 1 || nq < 0 || N_local < 0 || k < 0) return 0;
  const size_t lst = (size_t)k * (size_t)nq;
  return al256(fms_int8_topk_workspace_size(nq, N_local, k)) + 2 * al256(lst * 4) +
         2 * al256(lst * 4 * (size_t)nranks);
}

int fms_sharded_int8_topk(fms_comm_t comm, int qs_dtype, int ds_dtype, const int8_t* Qc,
                          const void* Qs, const int8_t* Gc_shard, const void* Gs_shard,
                          const uint8_t* qmask, const uint8_t* dmask_shard, int dim, int Tq, int nq,
                          int Td, int64_t N_local, int64_t id_lo, int normalize, int k,
                          float* topk_vals, int32_t* topk_ids, void* workspace, size_t ws_bytes,
                          fms_stream_t stream) {
  const NcclApi* a = nccl();
  if (!a) return FMS_ERR_UNSUPPORTED;
  if (!comm || k < 1 || nq < 0 || id_lo < 1) return FMS_ERR_INVALID;
  const int R = comm->nranks;
  const size_t need = fms_sharded_int8_topk_workspace_size(R, nq, N_local, k);
  if (!workspace || ws_bytes < need) return FMS_ERR_WORKSPACE;
  const size_t lst = (size_t)k * (size_t)nq;
  char* w = static_cast<char*>(workspace);
  void* scan_ws = w;
  const size_t scan_bytes = al256(fms_int8_topk_workspace_size(nq, N_local, k));
  w += scan_bytes;
  float* lv = reinterpret_cast<float*>(w);
  w += al256(lst * 4);
  int32_t* li = reinterpret_cast<int32_t*>(w);
  w += al256(lst * 4);
  float* gv = reinterpret_cast<float*>(w);
  w += al256(lst * 4 * (size_t)R);
  int32_t* gi = reinterpret_cast<int32_t*>(w);
  int st = fms_int8_exhaustive_fwd(qs_dtype, ds_dtype, Qc, Qs, Gc_shard, Gs_shard, qmask,
                                   dmask_shard, dim, Tq, nq, Td, N_local, normalize, nullptr, k, lv,
                                   li, id_lo - 1, scan_ws, scan_bytes, stream);
  if (st != FMS_OK || nq == 0) return st;
  cudaStream_t s = (cudaStream_t)stream;
  if ((st = nccl_status(a->groupStart())) != FMS_OK) return st;
  a->allGather(lv, gv, lst, ncclFloat32, comm->nc, s);
  a->allGather(li, gi, lst, ncclInt32, comm->nc, s);
  if ((st = nccl_status(a->groupEnd())) != FMS_OK) return st;
  return fms_topk_merge(gv, gi, k, nq, R, topk_vals, topk_ids, stream);
}

}  // extern "C"
