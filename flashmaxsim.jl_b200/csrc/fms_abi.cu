// fms_abi.cu -- the extern "C" entry points declared in include/fms.h.
//
// Each entry point checks its arguments the way the reference's layout drivers
// do (require_*_shapes raise DimensionMismatch / ArgumentError; here they return
// FMS_ERR_INVALID), builds the shared ScanParams geometry and dispatches:
// 16-bit features go to a tcgen05 + TMA engine when its constraints hold (the
// short-query gallery engine for paired / candidate layouts with Tq <= 32 and
// dim <= 256, else the general engine), everything else (and Float32 /
// Float64) to the CUDA-core scan.  No entry
// point allocates, synchronizes, prints or aborts.
#include <cuda.h>
#include <mutex>

#include "fms_common.cuh"
#include "fms_internal.h"
#include "fms_int8.cuh"

namespace fms {

static int g_sms[64];
static int g_cc[64];
static std::once_flag g_once[64];

static int cur_dev() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 64) d = 0;
  return d;
}

static void fill_dev(int d) {
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, d) == cudaSuccess) {
    g_sms[d] = prop.multiProcessorCount;
    g_cc[d] = prop.major * 10 + prop.minor;
  } else {
    g_sms[d] = 148;
    g_cc[d] = 0;
  }
}

int device_sm_count() {
  int d = cur_dev();
  std::call_once(g_once[d], fill_dev, d);
  return g_sms[d] > 0 ? g_sms[d] : 148;
}

int device_cc() {
  int d = cur_dev();
  std::call_once(g_once[d], fill_dev, d);
  return g_cc[d];
}

static int status_of(cudaError_t e) { return e == cudaSuccess ? FMS_OK : (int)e; }

static bool dtype_ok(int dtype) {
  return dtype == FMS_F32 || dtype == FMS_F16 || dtype == FMS_BF16 || dtype == FMS_F64;
}

static size_t elem_size(int dtype) {
  return dtype == FMS_F64 ? 8 : (dtype == FMS_F32 ? 4 : 2);
}

static int run_scan(int dtype, ScanParams& p, cudaStream_t s) {
  p.nunits = num_units(p);
  if (p.nunits == 0) return FMS_OK;
  if ((dtype == FMS_F16 || dtype == FMS_BF16) && scan_gallery_supported(dtype, p)) {
    cudaError_t e = launch_scan_gallery(dtype, p, s);
    if (e != cudaErrorNotSupported) return status_of(e);
  }
  if ((dtype == FMS_F16 || dtype == FMS_BF16) && scan_tc_supported(dtype, p)) {
    cudaError_t e = launch_scan_tc(dtype, p, s);
    if (e != cudaErrorNotSupported) return status_of(e);
  }
  return status_of(launch_scan_simt(dtype, p, s));
}

static ScanParams base_params() {
  ScanParams p;
  memset(&p, 0, sizeof(p));
  return p;
}

}  // namespace fms

using namespace fms;

extern "C" {

const char* fms_status_string(int status) {
  switch (status) {
    case FMS_OK: return "ok";
    case FMS_ERR_INVALID: return "invalid argument or shape mismatch";
    case FMS_ERR_DTYPE: return "unsupported dtype";
    case FMS_ERR_ALIGN: return "pointer alignment requirement not met";
    case FMS_ERR_WORKSPACE: return "workspace missing or too small";
    case FMS_ERR_UNSUPPORTED: return "unsupported device or feature";
    case FMS_ERR_TOO_LARGE: return "input too large for the fixed scratch of a no-allocation entry point";
    case FMS_ERR_NCCL: return "an NCCL call failed (fms_last_nccl_error)";
    default: return status > 0 ? cudaGetErrorString((cudaError_t)status) : "unknown error";
  }
}

int fms_version(void) { return 10100; }

int fms_device_error(int reset) {
  const int a = read_device_error(reset);
  const int b = read_i8tc_device_error(reset);
  const int c = read_gal_device_error(reset);
  return a != 0 ? a : (b != 0 ? b : c);
}

int fms_pair_fwd(int dtype, const void* q, const void* d, const uint8_t* qmask,
                 const uint8_t* dmask, int dim, int Tq, int Td, int normalize, void* score,
                 int32_t* args, fms_stream_t stream) {
  return fms_paired_fwd(dtype, q, d, qmask, dmask, dim, Tq, Td, 1, normalize, score, args, stream);
}

int fms_paired_fwd(int dtype, const void* Q, const void* D, const uint8_t* qmask,
                   const uint8_t* dmask, int dim, int Tq, int Td, int B, int normalize,
                   void* scores, int32_t* args, fms_stream_t stream) {
  if (!dtype_ok(dtype)) return FMS_ERR_DTYPE;
  if (dim < 0 || Tq < 0 || Td < 0 || B < 0) return FMS_ERR_INVALID;
  if (B > 0 && (!scores || (Tq > 0 && dim > 0 && !Q) || (Td > 0 && dim > 0 && !D)))
    return FMS_ERR_INVALID;
  ScanParams p = base_params();
  p.layout = L_PAIRED;
  p.Q = Q; p.D = D; p.qmask = qmask; p.dmask = dmask;
  p.dim = dim; p.Tq = Tq; p.Td = Td; p.B = B;
  p.nq_tok = (int64_t)Tq * B; p.nd_tok = (int64_t)Td * B;
  p.normalize = normalize; p.scores = scores; p.args = args;
  return run_scan(dtype, p, (cudaStream_t)stream);
}

int fms_inbatch_fwd(int dtype, const void* Q, const void* D, const uint8_t* qmask,
                    const uint8_t* dmask, int dim, int Tq, int Bq, int Td, int Bd, int normalize,
                    void* S, int32_t* args, fms_stream_t stream) {
  if (!dtype_ok(dtype)) return FMS_ERR_DTYPE;
  if (dim < 0 || Tq < 0 || Bq < 0 || Td < 0 || Bd < 0) return FMS_ERR_INVALID;
  if ((int64_t)Bq * Bd > 0 && !S) return FMS_ERR_INVALID;
  ScanParams p = base_params();
  p.layout = L_INBATCH;
  p.Q = Q; p.D = D; p.qmask = qmask; p.dmask = dmask;
  p.dim = dim; p.Tq = Tq; p.Td = Td; p.Bq = Bq; p.Bd = Bd;
  p.nq_tok = (int64_t)Tq * Bq; p.nd_tok = (int64_t)Td * Bd;
  p.normalize = normalize; p.scores = S; p.args = args;
  return run_scan(dtype, p, (cudaStream_t)stream);
}

int fms_candidates_fwd(int dtype, const void* Q, const void* gallery, const int32_t* idxs,
                       const uint8_t* qmask, const uint8_t* dmask, int dim, int Tq, int B,
                       int Td, int64_t N, int C, double neg, int normalize, void* S,
                       int32_t* args, fms_stream_t stream) {
  if (!dtype_ok(dtype)) return FMS_ERR_DTYPE;
  if (dim < 0 || Tq < 0 || B < 0 || Td < 0 || N < 0 || C < 0) return FMS_ERR_INVALID;
  if ((int64_t)C * B > 0 && (!S || !idxs)) return FMS_ERR_INVALID;
  ScanParams p = base_params();
  p.layout = L_CANDIDATES;
  p.Q = Q; p.D = gallery; p.qmask = qmask; p.dmask = dmask; p.idxs = idxs;
  p.dim = dim; p.Tq = Tq; p.Td = Td; p.B = B; p.C = C; p.Ngal = N;
  p.nq_tok = (int64_t)Tq * B; p.nd_tok = (int64_t)Td * N;
  p.neg = neg; p.normalize = normalize; p.scores = S; p.args = args;
  return run_scan(dtype, p, (cudaStream_t)stream);
}

int fms_candidates_shard_fwd(int dtype, const void* Q, const void* gallery_shard,
                             const int32_t* idxs, const uint8_t* qmask,
                             const uint8_t* dmask_shard, int dim, int Tq, int B, int Td,
                             int64_t N_local, int C, int64_t id_lo, int normalize, void* S,
                             void* workspace, size_t ws_bytes, fms_stream_t stream) {
  if (!dtype_ok(dtype)) return FMS_ERR_DTYPE;
  if (dim < 0 || Tq < 0 || B < 0 || Td < 0 || N_local < 0 || C < 0 || id_lo < 1)
    return FMS_ERR_INVALID;
  if ((int64_t)C * B > 0 && (!S || !idxs)) return FMS_ERR_INVALID;
  if (workspace && ws_bytes < shard_list_bytes((int64_t)C * B)) return FMS_ERR_WORKSPACE;
  if (workspace && dtype == FMS_F64) return FMS_ERR_DTYPE;  // the list path writes float32 -Inf
  ScanParams p = base_params();
  if (workspace && (int64_t)C * B > 0) {
    cudaError_t e = launch_shard_compact(idxs, (int64_t)C * B, id_lo, N_local, workspace,
                                         static_cast<float*>(S), &p.unit_list, &p.unit_count,
                                         (cudaStream_t)stream);
    if (e != cudaSuccess) return (int)e;
  }
  p.layout = L_CANDIDATES;
  p.Q = Q; p.D = gallery_shard; p.qmask = qmask; p.dmask = dmask_shard; p.idxs = idxs;
  p.dim = dim; p.Tq = Tq; p.Td = Td; p.B = B; p.C = C; p.Ngal = N_local;
  p.id_base = id_lo - 1;
  p.nq_tok = (int64_t)Tq * B; p.nd_tok = (int64_t)Td * N_local;
  p.neg = -INFINITY;  // slots owned by other shards lose the max-merge
  p.normalize = normalize; p.scores = S; p.args = nullptr;
  return run_scan(dtype, p, (cudaStream_t)stream);
}

int fms_packed_fwd(int dtype, const void* Qs, const void* tokens, const int32_t* cu,
                   const uint8_t* qmask, int dim, int Tq, int nq, int B, int64_t ntok,
                   int normalize, void* S, int32_t* args, fms_stream_t stream) {
  if (!dtype_ok(dtype)) return FMS_ERR_DTYPE;
  if (dim < 0 || Tq < 0 || nq < 0 || B < 0 || ntok < 0) return FMS_ERR_INVALID;
  if ((int64_t)B * nq > 0 && (!S || !cu)) return FMS_ERR_INVALID;
  ScanParams p = base_params();
  p.layout = L_PACKED;
  p.Q = Qs; p.D = tokens; p.qmask = qmask; p.cu_d = cu;
  p.dim = dim; p.Tq = Tq; p.B = B; p.nq = nq;
  p.nq_tok = (int64_t)Tq * nq; p.nd_tok = ntok;
  p.normalize = normalize; p.scores = S; p.args = args;
  return run_scan(dtype, p, (cudaStream_t)stream);
}

int fms_varlen_fwd(int dtype, const void* Qp, const void* Dp, const int32_t* cu_q,
                   const int32_t* cu_d, int dim, int N, int max_q, int64_t nq_tok,
                   int64_t nd_tok, int normalize, void* S, int32_t* args, fms_stream_t stream) {
  if (!dtype_ok(dtype)) return FMS_ERR_DTYPE;
  if (dim < 0 || N < 0 || max_q < 0 || nq_tok < 0 || nd_tok < 0) return FMS_ERR_INVALID;
  if (N > 0 && (!S || !cu_q || !cu_d)) return FMS_ERR_INVALID;
  ScanParams p = base_params();
  p.layout = L_VARLEN;
  p.Q = Qp; p.D = Dp; p.cu_q = cu_q; p.cu_d = cu_d;
  p.dim = dim; p.Tq = max_q; p.N = N;
  p.nq_tok = nq_tok; p.nd_tok = nd_tok;
  p.normalize = normalize; p.scores = S; p.args = args;
  return run_scan(dtype, p, (cudaStream_t)stream);
}

int fms_inv_counts(int dtype, const uint8_t* qmask, int Tq, int B, void* inv_n,
                   fms_stream_t stream) {
  if (!dtype_ok(dtype)) return FMS_ERR_DTYPE;
  if (Tq < 0 || B < 0 || (B > 0 && !inv_n)) return FMS_ERR_INVALID;
  return status_of(launch_inv_counts(dtype, qmask, Tq, B, inv_n, (cudaStream_t)stream));
}

// ------------------------------------------------------------------ backward

size_t fms_bwd_workspace_size(int strategy, int dtype, int64_t n_src, int64_t n_dest,
                              int64_t grad_d_numel) {
  return bwd_workspace_bytes(strategy, dtype, n_src, n_dest, grad_d_numel);
}

static int run_bwd(int dtype, int strategy, BwdParams& b, void* ws, size_t ws_bytes,
                   cudaStream_t s) {
  if (!dtype_ok(dtype)) return FMS_ERR_DTYPE;
  if (strategy != FMS_ATOMIC_UNIFIED && strategy != FMS_INVGRID) return FMS_ERR_INVALID;
  b.g.nunits = num_units(b.g);
  const size_t es = elem_size(dtype);
  // the outputs are fully overwritten: clear them first (rows no source reaches)
  if (b.nq_rows * b.g.dim > 0) {
    if (!b.dQ) return FMS_ERR_INVALID;
    cudaError_t e = cudaMemsetAsync(b.dQ, 0, (size_t)b.nq_rows * b.g.dim * es, s);
    if (e != cudaSuccess) return (int)e;
  }
  if (b.nd_rows * b.g.dim > 0 && !b.dD) return FMS_ERR_INVALID;
  if (b.g.nunits > 0 && (!b.g.args || !b.Delta)) return FMS_ERR_INVALID;
  const int64_t n_src = b.g.nunits * (int64_t)b.g.Tq;
  const size_t need = bwd_workspace_bytes(strategy, dtype, n_src, b.nd_rows, b.nd_rows * b.g.dim);
  if (need > 0 && (ws == nullptr || ws_bytes < need)) return FMS_ERR_WORKSPACE;
  if (n_src >= (int64_t)INT32_MAX) return FMS_ERR_INVALID;
  if (b.g.dim == 0) return FMS_OK;
  if (b.g.nunits == 0 || b.g.Tq == 0) {
    if (b.nd_rows > 0) {
      cudaError_t e = cudaMemsetAsync(b.dD, 0, (size_t)b.nd_rows * b.g.dim * es, s);
      if (e != cudaSuccess) return (int)e;
    }
    return FMS_OK;
  }
  return status_of(launch_backward(dtype, strategy, b, ws, ws_bytes, s));
}

int fms_pair_bwd(int dtype, int strategy, const void* delta, const void* q, const void* d,
                 const uint8_t* qmask, const int32_t* args, int dim, int Tq, int Td, void* dq,
                 void* dd, void* workspace, size_t ws_bytes, fms_stream_t stream) {
  return fms_paired_bwd(dtype, strategy, delta, nullptr, q, d, qmask, args, dim, Tq, Td, 1, dq,
                        dd, workspace, ws_bytes, stream);
}

int fms_paired_bwd(int dtype, int strategy, const void* Delta, const void* inv_n, const void* Q,
                   const void* D, const uint8_t* qmask, const int32_t* args, int dim, int Tq,
                   int Td, int B, void* dQ, void* dD, void* workspace, size_t ws_bytes,
                   fms_stream_t stream) {
  if (dim < 0 || Tq < 0 || Td < 0 || B < 0) return FMS_ERR_INVALID;
  BwdParams b;
  memset(&b, 0, sizeof(b));
  b.g.layout = L_PAIRED;
  b.g.Q = Q; b.g.D = D; b.g.qmask = qmask; b.g.args = const_cast<int32_t*>(args);
  b.g.dim = dim; b.g.Tq = Tq; b.g.Td = Td; b.g.B = B;
  b.g.nq_tok = (int64_t)Tq * B; b.g.nd_tok = (int64_t)Td * B;
  b.Delta = Delta; b.inv_n = inv_n; b.dQ = dQ; b.dD = dD;
  b.nq_rows = (int64_t)Tq * B; b.nd_rows = (int64_t)Td * B;
  return run_bwd(dtype, strategy, b, workspace, ws_bytes, (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// No-allocation variant of the InvGrid paired backward.  Its CSR scratch lives in
// a fixed device array of this library instead of a caller workspace.
//
// FMS_STATIC_SCRATCH_BYTES (4 MiB) bounds the problem: the InvGrid CSR needs
// about 4 * (2 * B*Td + B*Tq) bytes plus alignment, i.e. up to roughly 340 k
// document tokens for Tq = 32 sources per 180-token document.
static __device__ __align__(256) unsigned char g_static_scratch[FMS_STATIC_SCRATCH_BYTES];

// The device address is cached per device together with the unique id of the
// context it was looked up in: a primary context that was torn down and created
// again (cudaDeviceReset, cuDevicePrimaryCtxReset) gets a new id, the module --
// and with it the array -- is loaded again, and the set-up runs again.
static void* g_scratch_addr[64];
static unsigned long long g_scratch_ctx[64];
static std::mutex g_scratch_mu;

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current context, 0 when there is none yet
// (or the driver does not offer the query: the address is then looked up anew).
static unsigned long long current_ctx_id() {
  static CtxGetCurrentFn get_cur = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<CtxGetCurrentFn>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  if (!get_cur || !get_id) return 0;
  CUcontext c = nullptr;
  unsigned long long id = 0;
  if (get_cur(&c) != CUDA_SUCCESS || c == nullptr || get_id(c, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Set-up of the scratch on the current device: its device address
// (cudaGetSymbolAddress, return code checked), looked up once per device and
// context and cached.
static cudaError_t static_scratch(void** out) {
  int d = 0;
  cudaError_t e = cudaGetDevice(&d);
  if (e != cudaSuccess) return e;
  if (d < 0 || d >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  const unsigned long long ctx = current_ctx_id();
  if (g_scratch_addr[d] == nullptr || ctx == 0 || ctx != g_scratch_ctx[d]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_addr[d] = p;
    g_scratch_ctx[d] = current_ctx_id();  // the lookup above made the context current
  }
  *out = g_scratch_addr[d];
  return cudaSuccess;
}

int fms_paired_bwd_invgrid_noalloc(int dtype, const void* Delta, const void* inv_n, const void* Q,
                                   const void* D, const uint8_t* qmask, const int32_t* args,
                                   int dim, int Tq, int Td, int B, void* dQ, void* dD,
                                   fms_stream_t stream) {
  if (dim < 0 || Tq < 0 || Td < 0 || B < 0) return FMS_ERR_INVALID;
  if (!dtype_ok(dtype)) return FMS_ERR_DTYPE;
  const int64_t n_src = (int64_t)Tq * B, n_dest = (int64_t)Td * B;
  if (bwd_workspace_bytes(FMS_INVGRID, dtype, n_src, n_dest, n_dest * dim) >
      (size_t)FMS_STATIC_SCRATCH_BYTES)
    return FMS_ERR_TOO_LARGE;
  void* ws = nullptr;
  cudaError_t e = static_scratch(&ws);
  if (e != cudaSuccess) return (int)e;
  // everything of the scratch that must start at zero (the CSR row counts) is
  // cleared on the stream by the InvGrid path itself before use
  return fms_paired_bwd(dtype, FMS_INVGRID, Delta, inv_n, Q, D, qmask, args, dim, Tq, Td, B, dQ,
                        dD, ws, (size_t)FMS_STATIC_SCRATCH_BYTES, stream);
}

int fms_inbatch_bwd(int dtype, int strategy, const void* Delta, const void* inv_n, const void* Q,
                    const void* D, const uint8_t* qmask, const int32_t* args, int dim, int Tq,
                    int Bq, int Td, int Bd, void* dQ, void* dD, void* workspace,
                    size_t ws_bytes, fms_stream_t stream) {
  if (dim < 0 || Tq < 0 || Bq < 0 || Td < 0 || Bd < 0) return FMS_ERR_INVALID;
  BwdParams b;
  memset(&b, 0, sizeof(b));
  b.g.layout = L_INBATCH;
  b.g.Q = Q; b.g.D = D; b.g.qmask = qmask; b.g.args = const_cast<int32_t*>(args);
  b.g.dim = dim; b.g.Tq = Tq; b.g.Td = Td; b.g.Bq = Bq; b.g.Bd = Bd;
  b.g.nq_tok = (int64_t)Tq * Bq; b.g.nd_tok = (int64_t)Td * Bd;
  b.Delta = Delta; b.inv_n = inv_n; b.dQ = dQ; b.dD = dD;
  b.nq_rows = (int64_t)Tq * Bq; b.nd_rows = (int64_t)Td * Bd;
  return run_bwd(dtype, strategy, b, workspace, ws_bytes, (cudaStream_t)stream);
}

int fms_candidates_bwd(int dtype, int strategy, const void* Delta, const void* inv_n,
                       const void* Q, const void* gallery, const int32_t* idxs,
                       const uint8_t* qmask, const int32_t* args, int dim, int Tq, int B, int Td,
                       int64_t N, int C, void* dQ, void* dG, void* workspace, size_t ws_bytes,
                       fms_stream_t stream) {
  if (dim < 0 || Tq < 0 || B < 0 || Td < 0 || N < 0 || C < 0) return FMS_ERR_INVALID;
  if ((int64_t)C * B > 0 && !idxs) return FMS_ERR_INVALID;
  BwdParams b;
  memset(&b, 0, sizeof(b));
  b.g.layout = L_CANDIDATES;
  b.g.Q = Q; b.g.D = gallery; b.g.qmask = qmask; b.g.idxs = idxs;
  b.g.args = const_cast<int32_t*>(args);
  b.g.dim = dim; b.g.Tq = Tq; b.g.Td = Td; b.g.B = B; b.g.C = C; b.g.Ngal = N;
  b.g.nq_tok = (int64_t)Tq * B; b.g.nd_tok = (int64_t)Td * N;
  b.Delta = Delta; b.inv_n = inv_n; b.dQ = dQ; b.dD = dG;
  b.nq_rows = (int64_t)Tq * B; b.nd_rows = (int64_t)Td * N;
  return run_bwd(dtype, strategy, b, workspace, ws_bytes, (cudaStream_t)stream);
}

int fms_packed_bwd(int dtype, int strategy, const void* Delta, const void* inv_n,
                   const void* Qs, const void* tokens, const int32_t* cu, const uint8_t* qmask,
                   const int32_t* args, int dim, int Tq, int nq, int B, int64_t ntok, void* dQ,
                   void* dP, void* workspace, size_t ws_bytes, fms_stream_t stream) {
  if (dim < 0 || Tq < 0 || nq < 0 || B < 0 || ntok < 0) return FMS_ERR_INVALID;
  if ((int64_t)B * nq > 0 && !cu) return FMS_ERR_INVALID;
  BwdParams b;
  memset(&b, 0, sizeof(b));
  b.g.layout = L_PACKED;
  b.g.Q = Qs; b.g.D = tokens; b.g.qmask = qmask; b.g.cu_d = cu;
  b.g.args = const_cast<int32_t*>(args);
  b.g.dim = dim; b.g.Tq = Tq; b.g.B = B; b.g.nq = nq;
  b.g.nq_tok = (int64_t)Tq * nq; b.g.nd_tok = ntok;
  b.Delta = Delta; b.inv_n = inv_n; b.dQ = dQ; b.dD = dP;
  b.nq_rows = (int64_t)Tq * nq; b.nd_rows = ntok;
  return run_bwd(dtype, strategy, b, workspace, ws_bytes, (cudaStream_t)stream);
}

int fms_varlen_bwd(int dtype, int strategy, const void* Delta, const void* inv_n,
                   const void* Qp, const void* Dp, const int32_t* cu_q, const int32_t* cu_d,
                   const int32_t* args, int dim, int N, int max_q, int64_t nq_tok,
                   int64_t nd_tok, void* dQ, void* dD, void* workspace, size_t ws_bytes,
                   fms_stream_t stream) {
  if (dim < 0 || N < 0 || max_q < 0 || nq_tok < 0 || nd_tok < 0) return FMS_ERR_INVALID;
  if (N > 0 && (!cu_q || !cu_d)) return FMS_ERR_INVALID;
  BwdParams b;
  memset(&b, 0, sizeof(b));
  b.g.layout = L_VARLEN;
  b.g.Q = Qp; b.g.D = Dp; b.g.cu_q = cu_q; b.g.cu_d = cu_d;
  b.g.args = const_cast<int32_t*>(args);
  b.g.dim = dim; b.g.Tq = max_q; b.g.N = N;
  b.g.nq_tok = nq_tok; b.g.nd_tok = nd_tok;
  b.Delta = Delta; b.inv_n = inv_n; b.dQ = dQ; b.dD = dD;
  b.nq_rows = nq_tok; b.nd_rows = nd_tok;
  return run_bwd(dtype, strategy, b, workspace, ws_bytes, (cudaStream_t)stream);
}

// ------------------------------------------------------------------ INT8

int fms_quantize_int8(int dtype, const void* x, int dim, int64_t ntok, int8_t* codes,
                      void* scales, fms_stream_t stream) {
  if (dtype != FMS_F32 && dtype != FMS_F16 && dtype != FMS_BF16) return FMS_ERR_DTYPE;
  if (dim < 0 || ntok < 0) return FMS_ERR_INVALID;
  if (ntok > 0 && (!scales || (dim > 0 && (!x || !codes)))) return FMS_ERR_INVALID;
  return status_of(launch_quantize(dtype, x, dim, ntok, codes, scales, (cudaStream_t)stream));
}

static bool scale_ok(int d) { return d == FMS_F32 || d == FMS_F16; }

int fms_int8_paired_fwd(int qs_dtype, int ds_dtype, const int8_t* Qc, const void* Qs,
                        const int8_t* Dc, const void* Ds, const uint8_t* qmask,
                        const uint8_t* dmask, int dim, int Tq, int Td, int B, int normalize,
                        float* scores, int32_t* args, fms_stream_t stream) {
  if (!scale_ok(qs_dtype) || !scale_ok(ds_dtype)) return FMS_ERR_DTYPE;
  if (dim < 0 || Tq < 0 || Td < 0 || B < 0) return FMS_ERR_INVALID;
  if (B > 0 && !scores) return FMS_ERR_INVALID;
  Int8ScanParams p;
  memset(&p, 0, sizeof(p));
  p.Qc = Qc; p.Qs = Qs; p.Dc = Dc; p.Ds = Ds; p.qmask = qmask; p.dmask = dmask;
  p.qs_dtype = qs_dtype; p.ds_dtype = ds_dtype;
  p.dim = dim; p.Tq = Tq; p.Td = Td; p.exhaustive = 0; p.N = B; p.nunits = B;
  p.normalize = normalize; p.scores = scores; p.args = args;
  // tensor cores (kind::i8) when the shape allows, else the dp4a scan
  cudaError_t e = launch_int8_paired_tc(p, (cudaStream_t)stream);
  if (e == cudaErrorNotSupported) e = launch_int8_scan(p, (cudaStream_t)stream);
  return status_of(e);
}

int fms_int8_pair_fwd(int qs_dtype, int ds_dtype, const int8_t* qc, const void* qs,
                      const int8_t* dc, const void* ds, const uint8_t* qmask,
                      const uint8_t* dmask, int dim, int Tq, int Td, int normalize, float* score,
                      int32_t* args, fms_stream_t stream) {
  return fms_int8_paired_fwd(qs_dtype, ds_dtype, qc, qs, dc, ds, qmask, dmask, dim, Tq, Td, 1,
                             normalize, score, args, stream);
}

size_t fms_int8_topk_workspace_size(int nq, int64_t N, int k) {
  // score matrix (N, nq) float32 + top-k candidate lists
  return ((size_t)N * (size_t)nq * 4 + 255) / 256 * 256 + topk_workspace_bytes(nq, N, k);
}

// The exhaustive scan + top-k for prepared parameters (quantised queries in
// Qc / Qs, or float queries in Qf for the tensor-core prologue).
static int exhaustive_run(Int8ScanParams& p, float* S, int k, float* topk_vals, int32_t* topk_ids,
                          int64_t id_offset, void* workspace, size_t ws_bytes, cudaStream_t s) {
  const int64_t N = p.N;
  const int nq = (int)(N > 0 ? p.nunits / N : 0);
  float* Sbuf = S;
  char* ws = static_cast<char*>(workspace);
  if (k > 0) {
    size_t need = fms_int8_topk_workspace_size(nq, N, k);
    if (!workspace || ws_bytes < need) return FMS_ERR_WORKSPACE;
    if (!Sbuf) Sbuf = reinterpret_cast<float*>(ws);
    ws += ((size_t)N * (size_t)nq * 4 + 255) / 256 * 256;
  } else if (!S) {
    return FMS_ERR_INVALID;
  }
  p.scores = Sbuf;
  cudaError_t e = launch_int8_exhaustive_tc(p, s);
  if (e == cudaErrorNotSupported && p.Qf == nullptr) e = launch_int8_scan(p, s);
  if (e != cudaSuccess) return (int)e;
  if (k > 0) {
    e = launch_topk(Sbuf, N, nq, k, id_offset, ws, topk_vals, topk_ids, s);
    if (e != cudaSuccess) return (int)e;
  }
  return FMS_OK;
}

int fms_int8_exhaustive_fwd(int qs_dtype, int ds_dtype, const int8_t* Qc, const void* Qs,
                            const int8_t* Gc, const void* Gs, const uint8_t* qmask,
                            const uint8_t* dmask, int dim, int Tq, int nq, int Td, int64_t N,
                            int normalize, float* S, int k, float* topk_vals,
                            int32_t* topk_ids, int64_t id_offset, void* workspace,
                            size_t ws_bytes, fms_stream_t stream) {
  if (!scale_ok(qs_dtype) || !scale_ok(ds_dtype)) return FMS_ERR_DTYPE;
  if (dim < 0 || Tq < 0 || nq < 0 || Td < 0 || N < 0 || k < 0) return FMS_ERR_INVALID;
  if (k > 4096) return FMS_ERR_INVALID;
  if (k > 0 && (!topk_vals || !topk_ids)) return FMS_ERR_INVALID;
  if (N + id_offset >= (int64_t)INT32_MAX) return FMS_ERR_INVALID;
  Int8ScanParams p;
  memset(&p, 0, sizeof(p));
  p.Qc = Qc; p.Qs = Qs; p.Dc = Gc; p.Ds = Gs; p.qmask = qmask; p.dmask = dmask;
  p.qs_dtype = qs_dtype; p.ds_dtype = ds_dtype;
  p.dim = dim; p.Tq = Tq; p.Td = Td; p.exhaustive = 1; p.N = N; p.nunits = N * nq;
  p.normalize = normalize; p.args = nullptr;
  return exhaustive_run(p, S, k, topk_vals, topk_ids, id_offset, workspace, ws_bytes,
                        (cudaStream_t)stream);
}

static size_t al256(size_t x) { return (x + 255) / 256 * 256; }

size_t fms_int8_exhaustive_float_workspace_size(int nq, int Tq, int dim, int64_t N, int k) {
  if (nq < 0 || Tq < 0 || dim < 0 || N < 0 || k < 0) return 0;
  const size_t ntok = (size_t)nq * (size_t)Tq;
  return al256(k > 0 ? fms_int8_topk_workspace_size(nq, N, k) : 0) + al256(ntok * (size_t)dim) +
         al256(ntok * 4);
}

int fms_int8_exhaustive_float_fwd(int q_dtype, const void* Q, int ds_dtype, const int8_t* Gc,
                                  const void* Gs, const uint8_t* qmask, const uint8_t* dmask,
                                  int dim, int Tq, int nq, int Td, int64_t N, int normalize,
                                  float* S, int k, float* topk_vals, int32_t* topk_ids,
                                  int64_t id_offset, void* workspace, size_t ws_bytes,
                                  fms_stream_t stream) {
  if (q_dtype != FMS_F32 && q_dtype != FMS_F16 && q_dtype != FMS_BF16) return FMS_ERR_DTYPE;
  if (!scale_ok(ds_dtype)) return FMS_ERR_DTYPE;
  if (dim < 0 || Tq < 0 || nq < 0 || Td < 0 || N < 0 || k < 0) return FMS_ERR_INVALID;
  if (k > 4096) return FMS_ERR_INVALID;
  if (k > 0 && (!topk_vals || !topk_ids)) return FMS_ERR_INVALID;
  if (N + id_offset >= (int64_t)INT32_MAX) return FMS_ERR_INVALID;
  const size_t need = fms_int8_exhaustive_float_workspace_size(nq, Tq, dim, N, k);
  if (need > 0 && (!workspace || ws_bytes < need)) return FMS_ERR_WORKSPACE;
  cudaStream_t s = (cudaStream_t)stream;
  Int8ScanParams p;
  memset(&p, 0, sizeof(p));
  p.Dc = Gc; p.Ds = Gs; p.qmask = qmask; p.dmask = dmask;
  p.qs_dtype = FMS_F32; p.ds_dtype = ds_dtype;
  p.dim = dim; p.Tq = Tq; p.Td = Td; p.exhaustive = 1; p.N = N; p.nunits = N * nq;
  p.normalize = normalize; p.args = nullptr;
  p.Qf = Q; p.qf_dtype = q_dtype;
  const size_t topk_part = al256(k > 0 ? fms_int8_topk_workspace_size(nq, N, k) : 0);
  if (int8_exhaustive_tc_supported(p))
    return exhaustive_run(p, S, k, topk_vals, topk_ids, id_offset, workspace, topk_part, s);
  // shapes the tensor-core scan does not take: quantise into the workspace,
  // then the scan of quantised queries
  if (q_dtype == FMS_BF16) return FMS_ERR_DTYPE;  // the CUDA-core scan reads f32 / f16 scales
  char* w = static_cast<char*>(workspace) + topk_part;
  int8_t* qc = reinterpret_cast<int8_t*>(w);
  void* qs = w + al256((size_t)nq * Tq * dim);
  cudaError_t e = launch_quantize(q_dtype, Q, dim, (int64_t)nq * Tq, qc, qs, s);
  if (e != cudaSuccess) return (int)e;
  p.Qf = nullptr;
  p.Qc = qc; p.Qs = qs; p.qs_dtype = q_dtype;
  return exhaustive_run(p, S, k, topk_vals, topk_ids, id_offset, workspace, topk_part, s);
}

int fms_topk_merge(const float* vals, const int32_t* ids, int k, int nq, int nshard,
                   float* out_vals, int32_t* out_ids, fms_stream_t stream) {
  if (k < 0 || nq < 0 || nshard < 0 || k > 4096 || (int64_t)k * nshard > (1 << 16))
    return FMS_ERR_INVALID;
  if (k > 0 && nq > 0 && (!vals || !ids || !out_vals || !out_ids)) return FMS_ERR_INVALID;
  return status_of(launch_topk_merge(vals, ids, k, nq, nshard, out_vals, out_ids,
                                     (cudaStream_t)stream));
}

int fms_candidates_finalize_neg(const int32_t* idxs, int64_t N, int C, int B, double neg,
                                float* S, fms_stream_t stream) {
  if (C < 0 || B < 0 || N < 0) return FMS_ERR_INVALID;
  if ((int64_t)C * B > 0 && (!idxs || !S)) return FMS_ERR_INVALID;
  return status_of(launch_cand_neg(idxs, N, (int64_t)C * B, (float)neg, S, (cudaStream_t)stream));
}

}  // extern "C"
