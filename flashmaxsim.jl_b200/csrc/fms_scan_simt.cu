// fms_scan_simt.cu -- CUDA-core MaxSim scan for every layout and feature type.
//
// This is the Float32 / Float64 production path (the 1e-5 tolerance rules out
// TF32 tensor cores) and the path for 16-bit inputs whose shape the tcgen05 +
// TMA engine cannot take (row stride not a multiple of 16 bytes).  It follows
// the reference's SRAM-tiled scan (kernels_forward.jl:125-356): query tokens in
// tiles of 32, document tokens streamed in tiles of 32, the embedding split in
// K-chunks of 32 so shared memory does not grow with dim (split-d, §F.9), and
// the max / argmax kept in registers -- but each thread owns a 2 x 4 register
// micro-tile of (query token, doc token) dot products instead of a full row,
// and the per-query-token states of 8 threads are merged with warp shuffles.
// The Sigma_t reduction, normalisation and `neg` fill are fused into the same
// kernel (no separate sum / broadcast launches).
#include "fms_common.cuh"
#include "fms_internal.h"

namespace fms {

constexpr int ST_Q = 32;       // query tokens per tile
constexpr int ST_D = 32;       // doc tokens per tile
constexpr int ST_K = 32;       // embedding chunk
constexpr int ST_THREADS = 128;

template <typename T, bool ARGS>
__global__ void __launch_bounds__(ST_THREADS)
simt_scan_kernel(ScanParams p) {
  using A = typename Tr<T>::Acc;
  __shared__ A Qs[ST_K][ST_Q + 1];
  __shared__ A Ds[ST_K][ST_D + 1];
  __shared__ uint8_t dm_s[ST_D];
  __shared__ int ufirst_s;
  extern __shared__ unsigned char dyn_raw[];
  A* red = reinterpret_cast<A*>(dyn_raw);   // per-query-token contribution (Tq)

  const int tid = threadIdx.x;
  const int tx = tid & 7;          // doc-token lane group: columns tx + 8*j
  const int ty = tid >> 3;         // query tokens 2*ty, 2*ty+1
  const T* Q = static_cast<const T*>(p.Q);
  const T* D = static_cast<const T*>(p.D);
  const int dim = p.dim;
  A* scores = static_cast<A*>(p.scores);

  const int64_t nwalk = units_to_scan(p);
  for (int64_t v = blockIdx.x; v < nwalk; v += gridDim.x) {
    const int64_t unit = unit_at(p, v);
    const Unit U = decode_unit(p, unit);
    if (!U.valid) {
      if (tid == 0) scores[U.out] = (A)p.neg;
      if (ARGS)
        for (int t = tid; t < U.arg_rows; t += ST_THREADS) p.args[U.arg0 + t] = 0;
      continue;
    }
    // First valid document token (the one the sequential rule always takes).
    if (tid == 0) ufirst_s = INT32_MAX;
    __syncthreads();
    for (int u = tid; u < U.Td; u += ST_THREADS) {
      if (mask_ok(U.dmask, u)) { atomicMin(&ufirst_s, u); break; }
    }
    __syncthreads();
    const int ufirst = (ufirst_s == INT32_MAX) ? -1 : ufirst_s;

    for (int qt0 = 0; qt0 < U.Tq; qt0 += ST_Q) {
      A mx[2], sf[2];
      int ag[2];
      bool tv[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        int t = qt0 + 2 * ty + i;
        tv[i] = t < U.Tq && mask_ok(U.qmask, t);
        mx[i] = neg_inf<A>(); ag[i] = 0; sf[i] = (A)0;
      }
      for (int u0 = 0; u0 < U.Td; u0 += ST_D) {
        A acc[2][4];
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = (A)0;
        if (tid < ST_D) {
          int u = u0 + tid;
          dm_s[tid] = (u < U.Td && mask_ok(U.dmask, u)) ? 1 : 0;
        }
        __syncthreads();
        for (int k0 = 0; k0 < dim; k0 += ST_K) {
          // stage: consecutive threads read consecutive k of one token (coalesced)
#pragma unroll
          for (int r = 0; r < (ST_K * ST_Q) / ST_THREADS; ++r) {
            int e = tid + r * ST_THREADS;
            int kk = e & (ST_K - 1), tt = e / ST_K;
            int k = k0 + kk;
            int t = qt0 + tt, u = u0 + tt;
            Qs[kk][tt] = (k < dim && t < U.Tq) ? Tr<T>::to(Q[(U.q0 + t) * dim + k]) : (A)0;
            Ds[kk][tt] = (k < dim && u < U.Td) ? Tr<T>::to(D[(U.d0 + u) * dim + k]) : (A)0;
          }
          __syncthreads();
#pragma unroll 8
          for (int kk = 0; kk < ST_K; ++kk) {
            A qv0 = Qs[kk][2 * ty], qv1 = Qs[kk][2 * ty + 1];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              A dv = Ds[kk][tx + 8 * j];
              acc[0][j] += qv0 * dv;
              acc[1][j] += qv1 * dv;
            }
          }
          __syncthreads();
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          int uu = tx + 8 * j;
          int u = u0 + uu;
          if (dm_s[uu]) {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              A s = acc[i][j];
              if (u == ufirst) sf[i] = s;
              if (s > mx[i]) { mx[i] = s; ag[i] = u + 1; }
            }
          }
        }
        __syncthreads();  // dm_s reuse
      }
      // merge the 8 column groups of each query token
#pragma unroll
      for (int i = 0; i < 2; ++i) {
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) {
          A m2 = __shfl_xor_sync(0xffffffffu, mx[i], off);
          int a2 = __shfl_xor_sync(0xffffffffu, ag[i], off);
          merge_state(mx[i], ag[i], m2, a2);
        }
        // value at the first valid column lives in group (ufirst % 8)
        int src = (tid & 31 & ~7) | ((ufirst >= 0 ? ufirst : 0) & 7);
        A s0 = __shfl_sync(0xffffffffu, sf[i], src);
        final_fixup(mx[i], ag[i], ufirst, s0);
      }
      if (tx == 0) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          int t = qt0 + 2 * ty + i;
          if (t < U.Tq) {
            bool ok = tv[i] && ag[i] > 0;
            red[t] = ok ? mx[i] : (A)0;
            if (ARGS) p.args[U.arg0 + t] = ok ? ag[i] : 0;
          }
        }
      }
    }
    __syncthreads();
    if (tid == 0) {
      // Sigma_t in t order, as forward_pair.jl:92-95 does
      A score = (A)0;
      int nvalid = 0;
      for (int t = 0; t < U.Tq; ++t) {
        score += red[t];
        nvalid += mask_ok(U.qmask, t) ? 1 : 0;
      }
      if (p.normalize) score = score * ((A)1 / (A)(nvalid > 1 ? nvalid : 1));
      scores[U.out] = score;
    }
    if (ARGS)
      for (int t = U.Tq + tid; t < U.arg_rows; t += ST_THREADS) p.args[U.arg0 + t] = 0;
    __syncthreads();
  }
}

template <typename T>
static cudaError_t launch_simt_t(const ScanParams& p, cudaStream_t s, int num_sms) {
  using A = typename Tr<T>::Acc;
  if (p.nunits == 0) return cudaSuccess;
  int64_t grid = p.nunits;
  int64_t cap = (int64_t)num_sms * 16;
  if (grid > cap) grid = cap;
  size_t dyn = sizeof(A) * (size_t)(p.Tq > 0 ? p.Tq : 1);
  if (dyn > 48 * 1024) {
    auto k = p.args ? simt_scan_kernel<T, true> : simt_scan_kernel<T, false>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
    if (e != cudaSuccess) return e;
  }
  if (p.args)
    simt_scan_kernel<T, true><<<(unsigned)grid, ST_THREADS, dyn, s>>>(p);
  else
    simt_scan_kernel<T, false><<<(unsigned)grid, ST_THREADS, dyn, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_scan_simt(int dtype, const ScanParams& p, cudaStream_t s) {
  int sms = device_sm_count();
  switch (dtype) {
    case FMS_F32: return launch_simt_t<float>(p, s, sms);
    case FMS_F16: return launch_simt_t<__half>(p, s, sms);
    case FMS_BF16: return launch_simt_t<__nv_bfloat16>(p, s, sms);
    case FMS_F64: return launch_simt_t<double>(p, s, sms);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace fms
