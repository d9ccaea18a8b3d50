/*
 * fms.h -- C ABI of libflashmaxsim_sm100.so, the B200 (sm_100a) MaxSim engine.
 *
 * This is the drop-in boundary for FlashMaxSim.jl's CUDA path.  Each entry point
 * replaces one layout driver of the reference (file:line in FlashMaxSim.jl
 * v0.1.2 given beside it); the Julia package binds them with `ccall` from a
 * package extension, Python binds them with ctypes.
 *
 * Conventions (the reference's own, so Julia arrays pass straight through):
 *  - All arrays are device pointers, contiguous and column-major with tokens as
 *    columns: q (dim,Tq), Q (dim,Tq,B), gallery (dim,Td,N), packed (dim,ntok).
 *    Token t of a (dim,T,...) array starts at element t*dim.
 *  - Masks are 1-byte Bool (uint8, 0/1).  A NULL mask means "all true"
 *    (what `true_mask` builds, colocation.jl:4-6).
 *  - idxs, cu, cu_q, cu_d and args are Int32 and 1-based; args 0 = "no valid
 *    document token" (kernels_forward.jl:30-60).
 *  - dtype selects the feature eltype T; scores are score_eltype(T): float32 for
 *    FMS_F32/F16/BF16, float64 for FMS_F64 (kernels_forward.jl:16-21).
 *  - Every output is caller-owned and fully written by the call (scores are the
 *    finished values: Sigma_t, `neg` fill and `normalize` are fused, replacing
 *    the reference's separate sum/ifelse/normalize kernels).
 *  - `args` may be NULL: the kernels then skip the argmax tape (scores-only
 *    mode, for the non-AD calls that discard it, dispatch.jl:44,201,229,261,287).
 *  - Calls are asynchronous on `stream`, never synchronize, never allocate
 *    device memory, and are re-entrant; the caller's current device must own
 *    every pointer.
 *  - Return value: 0 on success; a negative FMS_ERR_* for a rejected argument
 *    (the reference's DimensionMismatch / ArgumentError); a positive
 *    cudaError_t if a launch failed.  Nothing aborts or prints.
 */
#ifndef FMS_H
#define FMS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* fms_stream_t; /* identical to cudaStream_t */

enum fms_dtype { FMS_F32 = 0, FMS_F16 = 1, FMS_BF16 = 2, FMS_F64 = 3 };

/* BackwardStrategy (types.jl:8-17) */
enum fms_backward { FMS_ATOMIC_UNIFIED = 0, FMS_INVGRID = 1 };

#define FMS_OK 0
#define FMS_ERR_INVALID (-1)     /* shape / argument rejected */
#define FMS_ERR_DTYPE (-2)       /* dtype not supported by this entry point */
#define FMS_ERR_ALIGN (-3)       /* pointer alignment not met */
#define FMS_ERR_WORKSPACE (-4)   /* workspace missing or too small */
#define FMS_ERR_UNSUPPORTED (-5) /* no sm_100 device, or feature unavailable */
#define FMS_ERR_TOO_LARGE (-6)   /* input exceeds a no-allocation entry point's scratch */
#define FMS_ERR_NCCL (-7)        /* an NCCL call failed (fms_last_nccl_error) */

/* Fixed device scratch of fms_paired_bwd_invgrid_noalloc (bytes). */
#define FMS_STATIC_SCRATCH_BYTES (4u << 20)

/* Human-readable text for a status code (static storage). */
const char* fms_status_string(int status);
/* Library ABI version: major*10000 + minor*100 + patch. */
int fms_version(void);

/* Device-side health flag of the current device: 1 if a kernel's bounded wait
   timed out since the last reset (that launch stopped early and its outputs are
   invalid), else 0; negative / positive status codes on failure.  Synchronizes
   the device.  reset != 0 clears the flag.  (No reference counterpart: the
   reference's kernels have no device-side waits.) */
int fms_device_error(int reset);

/* ------------------------------------------------------------------ forward */

/* Pair: score (1,) = maxsim(q, d, qmask, dmask), args (Tq,).
   Replaces pair_forward(::Backend) + pair_finalize (forward_pair.jl:104-116,
   146-173); normalize multiplies by one(T)/max(count(qmask),1). */
int fms_pair_fwd(int dtype, const void* q, const void* d, const uint8_t* qmask,
                 const uint8_t* dmask, int dim, int Tq, int Td, int normalize,
                 void* score, int32_t* args, fms_stream_t stream);

/* Paired batch: scores (B,), args (Tq,B).  Replaces paired_forward(::Backend)
   (forward_layouts.jl:105-124) + length_normalize (normalize.jl:13-25). */
int fms_paired_fwd(int dtype, const void* Q, const void* D, const uint8_t* qmask,
                   const uint8_t* dmask, int dim, int Tq, int Td, int B,
                   int normalize, void* scores, int32_t* args, fms_stream_t stream);

/* In-batch: S (Bd,Bq) with S[j,i] = MaxSim(Q_i, D_j), args (Tq,Bd,Bq).
   Replaces inbatch_forward(::Backend) (forward_layouts.jl:181-225). */
int fms_inbatch_fwd(int dtype, const void* Q, const void* D, const uint8_t* qmask,
                    const uint8_t* dmask, int dim, int Tq, int Bq, int Td, int Bd,
                    int normalize, void* S, int32_t* args, fms_stream_t stream);

/* Candidates: S (C,B) with S[c,b] = MaxSim(Q_b, gallery_{idxs[c,b]}); slots with
   idxs outside 1:N hold `neg` (also under normalize) and zero args (Tq,C,B).
   Replaces candidates_forward(::Backend) (forward_layouts.jl:263-290) +
   length_normalize_candidates (normalize.jl:37-46). */
int fms_candidates_fwd(int dtype, const void* Q, const void* gallery, const int32_t* idxs,
                       const uint8_t* qmask, const uint8_t* dmask, int dim, int Tq,
                       int B, int Td, int64_t N, int C, double neg, int normalize,
                       void* S, int32_t* args, fms_stream_t stream);

/* Candidates against one shard of a gallery sharded by doc id (multi-GPU; no
   reference counterpart -- the reference is single-device).  The shard holds
   global docs id_lo .. id_lo+N_local-1; slots whose idxs fall outside it get
   -Inf so an all-reduce(max) over shards yields the full S, after which
   fms_candidates_finalize_neg writes `neg` into globally invalid slots.
   Scores only (float32 / float64 per dtype).  With a workspace of
   fms_candidates_shard_workspace_size(B, C) bytes the call first lists the
   slots this shard owns (one pass over idxs, which also writes the -Inf) and
   scans only those, so its cost does not grow with the number of shards;
   with workspace NULL every slot is decoded by the scan itself. */
size_t fms_candidates_shard_workspace_size(int B, int C);
int fms_candidates_shard_fwd(int dtype, const void* Q, const void* gallery_shard,
                             const int32_t* idxs, const uint8_t* qmask,
                             const uint8_t* dmask_shard, int dim, int Tq, int B, int Td,
                             int64_t N_local, int C, int64_t id_lo, int normalize, void* S,
                             void* workspace, size_t ws_bytes, fms_stream_t stream);

/* Packed cu_seqlens: nq queries Qs (dim,Tq,nq) against the B ragged documents of
   tokens (dim,ntok), doc b = tokens[:, cu[b]:cu[b+1]-1].  S (B,nq), args
   (Tq,B,nq) local 1-based.  nq = 1 is the reference's maxsim(q, P::PackedSeq)
   (packed.jl:178-217, packed_finalize :333-337); nq > 1 is the batched
   multi-query form (one pass over the packed gallery for all queries). */
int fms_packed_fwd(int dtype, const void* Qs, const void* tokens, const int32_t* cu,
                   const uint8_t* qmask, int dim, int Tq, int nq, int B, int64_t ntok,
                   int normalize, void* S, int32_t* args, fms_stream_t stream);

/* Varlen pairs: S (N,), args (max_q,N); rows t >= Tq_n are written 0.
   Replaces varlen_forward(::Backend) + varlen_finalize (packed.jl:262-354). */
int fms_varlen_fwd(int dtype, const void* Qp, const void* Dp, const int32_t* cu_q,
                   const int32_t* cu_d, int dim, int N, int max_q, int64_t nq_tok,
                   int64_t nd_tok, int normalize, void* S, int32_t* args,
                   fms_stream_t stream);

/* inv_n[b] = T(one(S)/max(count(qmask[:,b]),1)) for B columns of qmask (Tq,B),
   written in dtype T (inv_token_counts + convert_scores, normalize.jl:4-10,
   rrule.jl:77).  qmask NULL counts Tq. */
int fms_inv_counts(int dtype, const uint8_t* qmask, int Tq, int B, void* inv_n,
                   fms_stream_t stream);

/* ----------------------------------------------------------------- backward */
/* Delta is the score cotangent already converted to T (rrule.jl:77,94,112);
   inv_n the per-query scale in T (NULL = ones).  delta = Delta*inv_n is formed
   in T, then dQ_t = delta * D_{u*} and dD_u = sum_{t: u*=t} delta * Q_t
   (Eqs. 2-3) accumulate in float32 and are written once, in T.  dQ and dD
   are fully overwritten.  FMS_ATOMIC_UNIFIED: one fused launch, float32 atomics
   (kernels_backward.jl:69-138).  FMS_INVGRID: inverse-grid CSR (parallel
   counting sort) + destination-owned scatter summing each destination's
   sources in ascending source order (deterministic; invgrid.jl:16-65,
   kernels_backward.jl:146-354).  Workspace: see fms_bwd_workspace_size. */

/* Bytes of workspace a backward call needs.  n_src = query-token sources
   (Tq*units), n_dest = destination doc tokens, grad_d_numel = numel(dD). */
size_t fms_bwd_workspace_size(int strategy, int dtype, int64_t n_src, int64_t n_dest,
                              int64_t grad_d_numel);

/* backward_pair.jl:38-87 (pair_pullback / pair_apply_pullback!). delta (1,) in T. */
int fms_pair_bwd(int dtype, int strategy, const void* delta, const void* q, const void* d,
                 const uint8_t* qmask, const int32_t* args, int dim, int Tq, int Td,
                 void* dq, void* dd, void* workspace, size_t ws_bytes, fms_stream_t stream);

/* backward_layouts.jl:28-60 (paired_pullback_ka). Delta (B,), inv_n (B,). */
int fms_paired_bwd(int dtype, int strategy, const void* Delta, const void* inv_n,
                   const void* Q, const void* D, const uint8_t* qmask, const int32_t* args,
                   int dim, int Tq, int Td, int B, void* dQ, void* dD, void* workspace,
                   size_t ws_bytes, fms_stream_t stream);

/* No counterpart in the reference: fms_paired_bwd with FMS_INVGRID for callers
   that cannot pass a workspace and must not allocate device memory on the call
   path (cudaMalloc / cudaFree synchronise the device and can fail under memory
   pressure, which a latency-bound serving loop or a caller holding only a
   fixed memory budget cannot afford).  The CSR scratch is a fixed array of
   FMS_STATIC_SCRATCH_BYTES inside this library; the call allocates nothing.
   - Inputs whose InvGrid scratch (fms_bwd_workspace_size(FMS_INVGRID, ...))
     exceeds FMS_STATIC_SCRATCH_BYTES return FMS_ERR_TOO_LARGE before any work.
   - The scratch address is looked up (cudaGetSymbolAddress) on the first call
     on a device and again on the first call after that device's primary context
     was torn down and created anew (cudaDeviceReset reloads the library's
     device code, so the array may move); make that first call before any
     stream capture begins.
   - One scratch per device: calls that overlap in time on the same device (other
     streams, other host threads) race on it and corrupt each other's results.
     Serialise them.
   Results are identical to fms_paired_bwd(dtype, FMS_INVGRID, ...). */
int fms_paired_bwd_invgrid_noalloc(int dtype, const void* Delta, const void* inv_n,
                                   const void* Q, const void* D, const uint8_t* qmask,
                                   const int32_t* args, int dim, int Tq, int Td, int B,
                                   void* dQ, void* dD, fms_stream_t stream);

/* backward_layouts.jl:96-128 (inbatch_pullback_ka). Delta (Bd,Bq), inv_n (Bq,). */
int fms_inbatch_bwd(int dtype, int strategy, const void* Delta, const void* inv_n,
                    const void* Q, const void* D, const uint8_t* qmask, const int32_t* args,
                    int dim, int Tq, int Bq, int Td, int Bd, void* dQ, void* dD,
                    void* workspace, size_t ws_bytes, fms_stream_t stream);

/* backward_layouts.jl:167-202 (candidates_pullback_ka). Delta (C,B), inv_n (B,). */
int fms_candidates_bwd(int dtype, int strategy, const void* Delta, const void* inv_n,
                       const void* Q, const void* gallery, const int32_t* idxs,
                       const uint8_t* qmask, const int32_t* args, int dim, int Tq, int B,
                       int Td, int64_t N, int C, void* dQ, void* dG, void* workspace,
                       size_t ws_bytes, fms_stream_t stream);

/* packed.jl:379-417 (packed_pullback_ka / _invgrid), nq queries.
   Delta (B,nq), inv_n (nq,), args (Tq,B,nq). */
int fms_packed_bwd(int dtype, int strategy, const void* Delta, const void* inv_n,
                   const void* Qs, const void* tokens, const int32_t* cu,
                   const uint8_t* qmask, const int32_t* args, int dim, int Tq, int nq,
                   int B, int64_t ntok, void* dQ, void* dP, void* workspace,
                   size_t ws_bytes, fms_stream_t stream);

/* packed.jl:445-485 (varlen_pullback_ka / _invgrid). Delta (N,), inv_n (N,). */
int fms_varlen_bwd(int dtype, int strategy, const void* Delta, const void* inv_n,
                   const void* Qp, const void* Dp, const int32_t* cu_q, const int32_t* cu_d,
                   const int32_t* args, int dim, int N, int max_q, int64_t nq_tok,
                   int64_t nd_tok, void* dQ, void* dD, void* workspace, size_t ws_bytes,
                   fms_stream_t stream);

/* --------------------------------------------------------------------- INT8 */

/* quantize_int8_symmetric (quant.jl:42-49) per token of x (dim,ntok) in T:
   codes (dim,ntok) int8, scales (ntok,) in T; every op rounded to T. */
int fms_quantize_int8(int dtype, const void* x, int dim, int64_t ntok, int8_t* codes,
                      void* scales, fms_stream_t stream);

/* int8_pair_forward / int8_paired_forward (quant.jl:127-197, 156-168, 220-231):
   s = (f32(qs_t) * f32(ds_u)) * f32(acc), acc the exact int32 dot product.
   qs_dtype / ds_dtype: FMS_F32 or FMS_F16 scale arrays.  score/scores float32. */
int fms_int8_pair_fwd(int qs_dtype, int ds_dtype, const int8_t* qc, const void* qs,
                      const int8_t* dc, const void* ds, const uint8_t* qmask,
                      const uint8_t* dmask, int dim, int Tq, int Td, int normalize,
                      float* score, int32_t* args, fms_stream_t stream);
int fms_int8_paired_fwd(int qs_dtype, int ds_dtype, const int8_t* Qc, const void* Qs,
                        const int8_t* Dc, const void* Ds, const uint8_t* qmask,
                        const uint8_t* dmask, int dim, int Tq, int Td, int B,
                        int normalize, float* scores, int32_t* args, fms_stream_t stream);

/* Exhaustive INT8 index search (new layout: the reference has pair/paired only,
   quant.jl:96-197).  Scores all N docs of an index (dim,Td,N) + scales (Td,N)
   for nq quantized queries (dim,Tq,nq) + scales (Tq,nq) with the pair formula.
   S (N,nq) is written when non-NULL.  When k > 0, the k best docs per query
   (score descending, doc id ascending on ties) go to topk_vals (k,nq) and
   topk_ids (k,nq) as 1-based ids plus id_offset (a shard's first global id - 1).
   Workspace: fms_int8_topk_workspace_size(nq, N, k). */
size_t fms_int8_topk_workspace_size(int nq, int64_t N, int k);
int fms_int8_exhaustive_fwd(int qs_dtype, int ds_dtype, const int8_t* Qc, const void* Qs,
                            const int8_t* Gc, const void* Gs, const uint8_t* qmask,
                            const uint8_t* dmask, int dim, int Tq, int nq, int Td, int64_t N,
                            int normalize, float* S, int k, float* topk_vals,
                            int32_t* topk_ids, int64_t id_offset, void* workspace,
                            size_t ws_bytes, fms_stream_t stream);

/* The same search for float queries Q (dim,Tq,nq) in q_dtype (FMS_F32, FMS_F16 or
   FMS_BF16): quantize_int8_symmetric (quant.jl:42-49, every op in q_dtype) runs
   inside the tensor-core scan's prologue, as the reference quantises queries on
   every call (quant.jl:159), so no quantised copy of the queries is written;
   shapes the tensor-core scan does not take quantise into the workspace first
   (f32 / f16 queries).  Workspace: fms_int8_exhaustive_float_workspace_size. */
size_t fms_int8_exhaustive_float_workspace_size(int nq, int Tq, int dim, int64_t N, int k);
int fms_int8_exhaustive_float_fwd(int q_dtype, const void* Q, int ds_dtype, const int8_t* Gc,
                                  const void* Gs, const uint8_t* qmask, const uint8_t* dmask,
                                  int dim, int Tq, int nq, int Td, int64_t N, int normalize,
                                  float* S, int k, float* topk_vals, int32_t* topk_ids,
                                  int64_t id_offset, void* workspace, size_t ws_bytes,
                                  fms_stream_t stream);

/* Merge per-shard top-k lists: vals/ids (k,nq,nshard) -> out (k,nq), same order
   rule.  Used after an all-gather of shard results. */
int fms_topk_merge(const float* vals, const int32_t* ids, int k, int nq, int nshard,
                   float* out_vals, int32_t* out_ids, fms_stream_t stream);

/* Element-wise max-merge of owner-disjoint sharded candidate scores: for slots
   whose idxs fall outside this shard the shard wrote -Inf / arg 0.  After an
   all-reduce(max) of S the slots that are invalid globally get `neg`. */
int fms_candidates_finalize_neg(const int32_t* idxs, int64_t N, int C, int B, double neg,
                                float* S, fms_stream_t stream);

/* ------------------------------------------------------------ multi-GPU (NCCL)
   No reference counterpart (the reference is single-device): galleries sharded
   by document id over the GPUs of one node, one process or task per GPU, each
   call on the caller's stream doing the local scan, the NCCL exchange and the
   finalisation, and returning on every rank what the single-device entry point
   returns for the whole gallery.  NCCL is loaded at run time: the process's
   own libnccl.so.2 when one is loaded (torch's, NCCL.jl's), else the system's;
   FMS_NCCL_LIBRARY names another file.  Every rank makes the same calls in the
   same order (NCCL collectives). */
typedef struct fms_comm* fms_comm_t;
#define FMS_UNIQUE_ID_BYTES 128

/* 1 when an NCCL library could be loaded, else 0. */
int fms_nccl_available(void);
/* Text of the last NCCL error seen by this thread (static storage). */
const char* fms_last_nccl_error(void);
/* An NCCL unique id (FMS_UNIQUE_ID_BYTES bytes): made on one rank and sent to
   the others by the caller (a file, MPI, a torch.distributed broadcast...). */
int fms_comm_unique_id(void* id);
/* Collective over nranks callers: a communicator on the current device. */
int fms_comm_init(fms_comm_t* comm, int nranks, int rank, const void* id);
/* Wrap an ncclComm_t the caller created (e.g. NCCL.jl's); not destroyed by
   fms_comm_destroy. */
int fms_comm_from_nccl(fms_comm_t* comm, void* nccl_comm);
int fms_comm_destroy(fms_comm_t comm);
int fms_comm_size(fms_comm_t comm, int* nranks, int* rank);

/* candidates_forward (forward_layouts.jl:263-290, normalize.jl:37-46) over a
   gallery sharded by doc id: this rank holds docs id_lo .. id_lo+N_local-1 of
   N_global.  Lists and scans the slots this rank owns, ncclAllReduce(max) of S
   (C,B) float32 in place, then `neg` (already T(neg)) in slots outside
   1:N_global.  Scores only.  Workspace: fms_sharded_candidates_workspace_size. */
size_t fms_sharded_candidates_workspace_size(int B, int C);
int fms_sharded_candidates_fwd(fms_comm_t comm, int dtype, const void* Q, const void* gallery_shard,
                               const int32_t* idxs, const uint8_t* qmask,
                               const uint8_t* dmask_shard, int dim, int Tq, int B, int Td,
                               int64_t N_local, int C, int64_t id_lo, int64_t N_global, double neg,
                               int normalize, float* S, void* workspace, size_t ws_bytes,
                               fms_stream_t stream);

/* packed_forward (packed.jl:178-217) for nq queries over a packed gallery split
   into contiguous document ranges: rank r holds counts[r] documents (host array
   of nranks entries, the same on every rank) with its own 1-based cu_shard.
   S (B_total, nq) float32 on every rank (ncclAllGather of the score blocks).
   Workspace: fms_sharded_packed_workspace_size(nranks, nq, max(counts)). */
size_t fms_sharded_packed_workspace_size(int nranks, int nq, int B_max);
int fms_sharded_packed_fwd(fms_comm_t comm, int dtype, const void* Qs, const void* tokens_shard,
                           const int32_t* cu_shard, const uint8_t* qmask, int dim, int Tq, int nq,
                           const int32_t* counts, int64_t ntok_local, int normalize, float* S,
                           void* workspace, size_t ws_bytes, fms_stream_t stream);

/* Exhaustive INT8 top-k (the layout of fms_int8_exhaustive_fwd) over an index
   sharded by doc id (this rank: docs id_lo .. id_lo+N_local-1): local scan and
   top-k with global ids, ncclAllGather of the (k,nq) lists, device merge (score
   descending, id ascending).  Workspace: fms_sharded_int8_topk_workspace_size. */
size_t fms_sharded_int8_topk_workspace_size(int nranks, int nq, int64_t N_local, int k);
int fms_sharded_int8_topk(fms_comm_t comm, int qs_dtype, int ds_dtype, const int8_t* Qc,
                          const void* Qs, const int8_t* Gc_shard, const void* Gs_shard,
                          const uint8_t* qmask, const uint8_t* dmask_shard, int dim, int Tq, int nq,
                          int Td, int64_t N_local, int64_t id_lo, int normalize, int k,
                          float* topk_vals, int32_t* topk_ids, void* workspace, size_t ws_bytes,
                          fms_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FMS_H */
