// fms_common.cuh -- shared device helpers for the sm_100a MaxSim kernels.
//
// Every MaxSim layout of FlashMaxSim.jl (pair, paired, in-batch, candidates,
// packed cu_seqlens, varlen pairs) is a set of independent "units": one query
// token run scored against one document token run.  Both runs are rows of a
// token-major (dim, ntok) matrix, exactly the reference's column-major
// (dim, T, B) arrays.  decode_unit() maps a unit id to its runs, masks and
// output slots; all kernels (SIMT, tcgen05, backward) share it.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>

#include "fms.h"

namespace fms {

enum Layout : int {
  L_PAIRED = 0,      // pair == paired with B = 1
  L_CANDIDATES = 1,
  L_INBATCH = 2,
  L_PACKED = 3,
  L_VARLEN = 4,
};

struct ScanParams {
  int layout;
  const void* Q;            // query tokens (dim, nq_tok)
  const void* D;            // document tokens (dim, nd_tok)
  const uint8_t* qmask;     // NULL = all true
  const uint8_t* dmask;     // NULL = all true
  const int32_t* idxs;      // candidates (C,B), 1-based
  const int32_t* cu_q;      // varlen query CSR, 1-based
  const int32_t* cu_d;      // packed / varlen doc CSR, 1-based
  int dim;
  int Tq;                   // query tokens per unit (max_q for varlen)
  int Td;                   // doc tokens per doc (dense layouts)
  int B, C, Bq, Bd, nq, N;  // layout counts (N = varlen pairs)
  int64_t Ngal;             // gallery docs (candidates)
  int64_t id_base;          // candidates: idxs value of local doc 1, minus 1 (shards)
  int64_t nq_tok, nd_tok;   // token rows of Q and D (bounds for CSR layouts)
  int64_t nunits;
  int normalize;
  double neg;
  void* scores;             // score_eltype(T)
  int32_t* args;            // NULL = scores only
  // Optional device list of the unit ids to scan (a sharded candidate scan
  // scans only the slots its shard owns) and its device-resident length; the
  // scans then walk list entries 0 .. *unit_count - 1 instead of 0 .. nunits-1.
  const int32_t* unit_list;
  const int32_t* unit_count;
};

// Units a scan walks (device side) and the unit id of walk position v.
__device__ __forceinline__ int64_t units_to_scan(const ScanParams& p) {
  return p.unit_count ? (int64_t)*p.unit_count : p.nunits;
}
__device__ __forceinline__ int64_t unit_at(const ScanParams& p, int64_t v) {
  return p.unit_list ? (int64_t)p.unit_list[v] : v;
}

// Backward geometry: the forward's ScanParams plus cotangents and outputs.
struct BwdParams {
  ScanParams g;           // geometry; g.args is the input argmax tape
  const void* Delta;      // (nunits,) in T, unit order of decode_unit
  const void* inv_n;      // (nqcols,) in T, NULL = ones
  void* dQ;               // (dim, nq_rows) in T
  void* dD;               // (dim, nd_rows) in T
  int64_t nq_rows;
  int64_t nd_rows;
};

struct Unit {
  int64_t q0;               // first query token row
  int Tq;                   // query tokens in this unit
  const uint8_t* qmask;     // per-token mask of this unit's query (NULL = all)
  int64_t d0;               // first doc token row
  int Td;                   // doc tokens in this unit
  const uint8_t* dmask;     // per-token mask of this unit's doc (NULL = all)
  int64_t out;              // score slot
  int64_t arg0;             // args[arg0 + t]
  int arg_rows;             // args rows owned by the unit (max_q for varlen)
  int qidx;                 // query column (for inv_n)
  bool valid;               // false: candidate slot whose idx is outside 1:N
};

__host__ __device__ inline int64_t num_units(const ScanParams& p) {
  switch (p.layout) {
    case L_PAIRED: return p.B;
    case L_CANDIDATES: return (int64_t)p.C * p.B;
    case L_INBATCH: return (int64_t)p.Bd * p.Bq;
    case L_PACKED: return (int64_t)p.B * p.nq;
    default: return p.N;
  }
}

// Clamp a CSR run [a, a+len) into [0, ntok): malformed device CSR cannot fault.
__device__ inline void clamp_run(int64_t& a, int& len, int64_t ntok) {
  if (len < 0) len = 0;
  if (a < 0) { len = 0; a = 0; }
  if (a > ntok) { a = ntok; len = 0; }
  if (a + len > ntok) len = (int)(ntok - a);
}

__device__ inline Unit decode_unit(const ScanParams& p, int64_t u) {
  Unit U;
  U.valid = true;
  U.out = u;
  U.arg_rows = p.Tq;
  switch (p.layout) {
    case L_PAIRED: {
      U.q0 = u * p.Tq; U.Tq = p.Tq; U.qmask = p.qmask ? p.qmask + u * p.Tq : nullptr;
      U.d0 = u * p.Td; U.Td = p.Td; U.dmask = p.dmask ? p.dmask + u * p.Td : nullptr;
      U.arg0 = u * p.Tq; U.qidx = (int)u;
      break;
    }
    case L_CANDIDATES: {
      int64_t b = u / p.C;
      int64_t j = (int64_t)p.idxs[u] - p.id_base;
      U.valid = (j >= 1 && j <= p.Ngal);
      if (!U.valid) j = 1;
      U.q0 = b * p.Tq; U.Tq = p.Tq; U.qmask = p.qmask ? p.qmask + b * p.Tq : nullptr;
      U.d0 = (j - 1) * p.Td; U.Td = p.Td; U.dmask = p.dmask ? p.dmask + (j - 1) * p.Td : nullptr;
      U.arg0 = u * p.Tq; U.qidx = (int)b;
      break;
    }
    case L_INBATCH: {
      int64_t j = u % p.Bd, i = u / p.Bd;
      U.q0 = i * p.Tq; U.Tq = p.Tq; U.qmask = p.qmask ? p.qmask + i * p.Tq : nullptr;
      U.d0 = j * p.Td; U.Td = p.Td; U.dmask = p.dmask ? p.dmask + j * p.Td : nullptr;
      U.arg0 = u * p.Tq; U.qidx = (int)i;
      break;
    }
    case L_PACKED: {
      int64_t b = u % p.B, qi = u / p.B;
      U.q0 = qi * p.Tq; U.Tq = p.Tq; U.qmask = p.qmask ? p.qmask + qi * p.Tq : nullptr;
      U.d0 = (int64_t)p.cu_d[b] - 1; U.Td = p.cu_d[b + 1] - p.cu_d[b];
      clamp_run(U.d0, U.Td, p.nd_tok);
      U.dmask = nullptr;
      U.arg0 = u * p.Tq; U.qidx = (int)qi;
      break;
    }
    default: {  // L_VARLEN
      U.q0 = (int64_t)p.cu_q[u] - 1; U.Tq = p.cu_q[u + 1] - p.cu_q[u];
      clamp_run(U.q0, U.Tq, p.nq_tok);
      if (U.Tq > p.Tq) U.Tq = p.Tq;   // never past the args rows (max_q)
      U.qmask = nullptr;
      U.d0 = (int64_t)p.cu_d[u] - 1; U.Td = p.cu_d[u + 1] - p.cu_d[u];
      clamp_run(U.d0, U.Td, p.nd_tok);
      U.dmask = nullptr;
      U.arg0 = u * p.Tq; U.qidx = (int)u;
      break;
    }
  }
  return U;
}

// ------------------------------------------------------------------ dtype traits

template <typename T> struct Tr;
template <> struct Tr<float> {
  using Acc = float;
  static __device__ __forceinline__ float to(float x) { return x; }
  static __device__ __forceinline__ float from(float x) { return x; }
  static __device__ __forceinline__ float floatmin() { return 1.17549435e-38f; }
};
template <> struct Tr<double> {
  using Acc = double;
  static __device__ __forceinline__ double to(double x) { return x; }
  static __device__ __forceinline__ double from(double x) { return x; }
  static __device__ __forceinline__ double floatmin() { return 2.2250738585072014e-308; }
};
template <> struct Tr<__half> {
  using Acc = float;
  static __device__ __forceinline__ float to(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from(float x) { return __float2half_rn(x); }
  static __device__ __forceinline__ float floatmin() { return 6.103515625e-05f; }
};
template <> struct Tr<__nv_bfloat16> {
  using Acc = float;
  static __device__ __forceinline__ float to(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ float floatmin() { return 1.17549435e-38f; }
};

// Product rounded to T, as Julia evaluates `a * b` for T-typed operands
// (Float16/BFloat16 arithmetic = Float32 op then one rounding, exact here).
template <typename T>
__device__ __forceinline__ typename Tr<T>::Acc tmul(typename Tr<T>::Acc a, typename Tr<T>::Acc b) {
  return Tr<T>::to(Tr<T>::from(a * b));
}

template <typename A> __device__ __forceinline__ A neg_inf();
template <> __device__ __forceinline__ float neg_inf<float>() { return -INFINITY; }
template <> __device__ __forceinline__ double neg_inf<double>() { return -(double)INFINITY; }

// ------------------------------------------------------------------ argmax states
//
// Per-thread partial states use `s > mx` from (-inf, 0): NaN and -inf never
// enter a state.  Partials over disjoint column sets merge by value, then by
// smaller index.  The final fixup restores the reference's exact sequential
// rule `arg == 0 || s > mx` (forward_pair.jl:83): the first valid column u_f
// always enters, so if S[t,u_f] is NaN (sticky) or no column beat -inf, the
// result is (S[t,u_f], u_f).
template <typename A>
__device__ __forceinline__ void merge_state(A& m1, int& a1, A m2, int a2) {
  if (a2 == 0) return;
  if (a1 == 0 || m2 > m1 || (m2 == m1 && a2 < a1)) { m1 = m2; a1 = a2; }
}

template <typename A>
__device__ __forceinline__ void final_fixup(A& mx, int& arg, int ufirst, A s_first) {
  if (ufirst >= 0 && (arg == 0 || s_first != s_first)) { mx = s_first; arg = ufirst + 1; }
}

__device__ __forceinline__ bool mask_ok(const uint8_t* m, int64_t i) {
  return m == nullptr || m[i] != 0;
}

}  // namespace fms
