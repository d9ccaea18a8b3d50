// fms_int8.cu -- INT8 index path (quant.jl, kernels_int8.jl): on-device
// per-token symmetric quantization, the deferred-dequant INT8 MaxSim scan
// (s = (qs_t * ds_u) * float(acc), acc the exact int32 dot product), the
// exhaustive index scan with per-query top-k, and the top-k merge used after
// sharded scans.
#include "fms_common.cuh"
#include "fms_internal.h"
#include "fms_int8.cuh"
#include "fms_quant.cuh"

namespace fms {

// ------------------------------------------------------------------ quantize

// quantize_int8_symmetric (quant.jl:42-49), one warp per token (fms_quant.cuh).
template <typename T>
__global__ void quantize_kernel(const T* __restrict__ x, int dim, int64_t ntok,
                                int8_t* __restrict__ codes, T* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t t = w; t < ntok; t += nw) {
    int8_t* ct = codes + t * dim;
    const auto sc = quantize_token<T>(x + t * dim, dim, lane, [&](int k, int8_t c) { ct[k] = c; });
    if (lane == 0) scales[t] = Tr<T>::from(sc);
  }
}

cudaError_t launch_quantize(int dtype, const void* x, int dim, int64_t ntok, int8_t* codes,
                            void* scales, cudaStream_t s) {
  if (ntok == 0) return cudaSuccess;
  int64_t blocks = (ntok + 7) / 8;
  int64_t cap = (int64_t)device_sm_count() * 32;
  if (blocks > cap) blocks = cap;
  switch (dtype) {
    case FMS_F32:
      quantize_kernel<float><<<(unsigned)blocks, 256, 0, s>>>((const float*)x, dim, ntok, codes, (float*)scales);
      break;
    case FMS_F16:
      quantize_kernel<__half><<<(unsigned)blocks, 256, 0, s>>>((const __half*)x, dim, ntok, codes, (__half*)scales);
      break;
    case FMS_BF16:
      quantize_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, s>>>((const __nv_bfloat16*)x, dim, ntok, codes,
                                                                      (__nv_bfloat16*)scales);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ------------------------------------------------------------------ INT8 scan

__device__ __forceinline__ float load_scale(const void* p, int dtype, int64_t i) {
  return dtype == FMS_F16 ? __half2float(static_cast<const __half*>(p)[i])
                          : static_cast<const float*>(p)[i];
}

constexpr int I8_Q = 32, I8_D = 32, I8_K = 128, I8_THREADS = 128;

// SIMT INT8 scan (dp4a), same tiling and merge as the float SIMT scan.  Layout:
// paired units (B = pairs) or exhaustive units (unit = doc j + N*qi).
template <bool ARGS>
__global__ void __launch_bounds__(I8_THREADS) int8_scan_kernel(Int8ScanParams p) {
  __shared__ int32_t Qs[I8_K / 4][I8_Q + 1];
  __shared__ int32_t Ds[I8_K / 4][I8_D + 1];
  __shared__ float qs_s[I8_Q], ds_s[I8_D];
  __shared__ uint8_t dm_s[I8_D];
  __shared__ int ufirst_s;
  __shared__ float red[I8_Q];
  const int tid = threadIdx.x, tx = tid & 7, ty = tid >> 3;
  const int dim = p.dim;
  for (int64_t unit = blockIdx.x; unit < p.nunits; unit += gridDim.x) {
    int64_t qi, dj, out;
    if (p.exhaustive) { dj = unit % p.N; qi = unit / p.N; out = dj + p.N * qi; }
    else { dj = unit; qi = unit; out = unit; }
    const int8_t* qc = p.Qc + qi * (int64_t)p.Tq * dim;
    const int8_t* dc = p.Dc + dj * (int64_t)p.Td * dim;
    const uint8_t* qm = p.qmask ? p.qmask + qi * p.Tq : nullptr;
    const uint8_t* dm = p.dmask ? p.dmask + dj * p.Td : nullptr;
    if (tid == 0) ufirst_s = INT32_MAX;
    __syncthreads();
    for (int u = tid; u < p.Td; u += I8_THREADS)
      if (mask_ok(dm, u)) { atomicMin(&ufirst_s, u); break; }
    __syncthreads();
    const int ufirst = ufirst_s == INT32_MAX ? -1 : ufirst_s;
    float total = 0.f;
    for (int qt0 = 0; qt0 < p.Tq; qt0 += I8_Q) {
      float mx[2], sf[2];
      int ag[2];
      bool tv[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        int t = qt0 + 2 * ty + i;
        tv[i] = t < p.Tq && mask_ok(qm, t);
        mx[i] = -INFINITY; ag[i] = 0; sf[i] = 0.f;
      }
      if (tid < I8_Q) {
        int t = qt0 + tid;
        qs_s[tid] = t < p.Tq ? load_scale(p.Qs, p.qs_dtype, qi * p.Tq + t) : 0.f;
      }
      for (int u0 = 0; u0 < p.Td; u0 += I8_D) {
        int32_t acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
        if (tid < I8_D) {
          int u = u0 + tid;
          dm_s[tid] = (u < p.Td && mask_ok(dm, u)) ? 1 : 0;
          ds_s[tid] = u < p.Td ? load_scale(p.Ds, p.ds_dtype, dj * p.Td + u) : 0.f;
        }
        __syncthreads();
        for (int k0 = 0; k0 < dim; k0 += I8_K) {
          // stage 4 codes per int32 word: e -> (word kk, token tt)
          for (int e = tid; e < (I8_K / 4) * I8_Q; e += I8_THREADS) {
            int kk = e % (I8_K / 4), tt = e / (I8_K / 4);
            int t = qt0 + tt, u = u0 + tt;
            int32_t qw = 0, dw = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              int k = k0 + kk * 4 + b;
              if (k < dim) {
                if (t < p.Tq) qw |= ((int32_t)(uint8_t)qc[(int64_t)t * dim + k]) << (8 * b);
                if (u < p.Td) dw |= ((int32_t)(uint8_t)dc[(int64_t)u * dim + k]) << (8 * b);
              }
            }
            Qs[kk][tt] = qw;
            Ds[kk][tt] = dw;
          }
          __syncthreads();
#pragma unroll 4
          for (int kk = 0; kk < I8_K / 4; ++kk) {
            int32_t q0 = Qs[kk][2 * ty], q1 = Qs[kk][2 * ty + 1];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              int32_t dv = Ds[kk][tx + 8 * j];
              acc[0][j] = __dp4a(q0, dv, acc[0][j]);
              acc[1][j] = __dp4a(q1, dv, acc[1][j]);
            }
          }
          __syncthreads();
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          int uu = tx + 8 * j, u = u0 + uu;
          if (dm_s[uu]) {
            float dsc = ds_s[uu];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              float s = qs_s[2 * ty + i] * dsc * (float)acc[i][j];
              if (u == ufirst) sf[i] = s;
              if (s > mx[i]) { mx[i] = s; ag[i] = u + 1; }
            }
          }
        }
        __syncthreads();
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) {
          float m2 = __shfl_xor_sync(0xffffffffu, mx[i], off);
          int a2 = __shfl_xor_sync(0xffffffffu, ag[i], off);
          merge_state(mx[i], ag[i], m2, a2);
        }
        int src = (tid & 31 & ~7) | ((ufirst >= 0 ? ufirst : 0) & 7);
        float s0 = __shfl_sync(0xffffffffu, sf[i], src);
        final_fixup(mx[i], ag[i], ufirst, s0);
      }
      if (tx == 0) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          int t = qt0 + 2 * ty + i;
          bool ok = t < p.Tq && tv[i] && ag[i] > 0;
          red[2 * ty + i] = ok ? mx[i] : 0.f;
          if (ARGS && t < p.Tq) p.args[out * p.Tq + t] = ok ? ag[i] : 0;
        }
      }
      __syncthreads();
      if (tid == 0) {  // Sigma_t in t order (quant.jl:121-123)
        int lim = p.Tq - qt0 < I8_Q ? p.Tq - qt0 : I8_Q;
        for (int t = 0; t < lim; ++t) total += red[t];
      }
      __syncthreads();
    }
    if (tid == 0) {
      if (p.normalize) {
        int n = 0;
        for (int t = 0; t < p.Tq; ++t) n += mask_ok(qm, t) ? 1 : 0;
        total = total * (1.0f / (float)(n > 1 ? n : 1));
      }
      p.scores[out] = total;
    }
    __syncthreads();
  }
}

cudaError_t launch_int8_scan(const Int8ScanParams& p, cudaStream_t s) {
  if (p.nunits == 0) return cudaSuccess;
  int64_t grid = p.nunits;
  int64_t cap = (int64_t)device_sm_count() * 16;
  if (grid > cap) grid = cap;
  if (p.args)
    int8_scan_kernel<true><<<(unsigned)grid, I8_THREADS, 0, s>>>(p);
  else
    int8_scan_kernel<false><<<(unsigned)grid, I8_THREADS, 0, s>>>(p);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ top-k

// Order key: larger score first, then smaller doc id.  Float bits are mapped
// to an unsigned order; ids are complemented so that ascending id sorts first
// in a descending sort.
__device__ __forceinline__ uint64_t topk_key(float v, uint32_t id) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((uint64_t)b << 32) | (uint64_t)(0xffffffffu - id);
}
__device__ __forceinline__ float key_val(uint64_t k) {
  uint32_t b = (uint32_t)(k >> 32);
  b = (b & 0x80000000u) ? (b & 0x7fffffffu) : ~b;
  return __uint_as_float(b);
}
__device__ __forceinline__ uint32_t key_id(uint64_t k) { return 0xffffffffu - (uint32_t)k; }

// Block-wide descending bitonic sort of n (power of two) keys in shared memory.
__device__ void bitonic_desc(uint64_t* a, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
        int lo = 2 * i - (i & (stride - 1));
        int hi = lo + stride;
        bool desc = ((lo & size) == 0);
        uint64_t x = a[lo], y = a[hi];
        if ((x < y) == desc) { a[lo] = y; a[hi] = x; }
      }
    }
  }
  __syncthreads();
}

constexpr int TOPK_CHUNK = 8192;  // keys per block and round (64 KB shared memory)
constexpr int TOPK_THREADS = 1024;
constexpr int TOPK_PER = TOPK_CHUNK / TOPK_THREADS;  // keys per thread
constexpr int TOPK_PRUNE_K = TOPK_THREADS / TOPK_PER;  // k up to which a chunk is pruned first

// One reduction round: every chunk of TOPK_CHUNK keys of a query's list keeps its
// best k.  From S (first round, keys built from scores and ids) or from keys.
// Keys are unique (the id is part of the key) and 0 only as padding.
//
// For k <= TOPK_PRUNE_K the chunk is pruned before it is sorted: with t the
// k-th largest of the threads' maxima, at least k keys are >= t, so every key
// of the chunk's best k is >= t; and only a thread whose maximum is >= t can
// hold such a key, so at most TOPK_PER * k <= TOPK_THREADS nonzero keys
// survive (if fewer than k threads hold a nonzero key, t = 0 and the
// survivors are all the nonzero keys, fewer still).  Sorting the 1024 maxima
// and the 1024 survivors replaces the sort of all 8192 keys; the result is the
// same best k in the same order.
__global__ void __launch_bounds__(TOPK_THREADS) topk_round_kernel(const float* __restrict__ S,
                                                                 const uint64_t* __restrict__ kin,
                                                                 int64_t L, int nq, int k,
                                                                 int64_t id_offset,
                                                                 uint64_t* __restrict__ kout) {
  extern __shared__ uint64_t keys[];
  __shared__ int nsurv;
  const int64_t nchunks = (L + TOPK_CHUNK - 1) / TOPK_CHUNK;
  for (int64_t job = blockIdx.x; job < nchunks * nq; job += gridDim.x) {
    const int64_t c = job % nchunks, qi = job / nchunks;
    const int64_t j0 = c * TOPK_CHUNK;
    __syncthreads();
    if (k <= TOPK_PRUNE_K) {
      uint64_t kv[TOPK_PER];
      uint64_t mx = 0ull;
#pragma unroll
      for (int r = 0; r < TOPK_PER; ++r) {
        const int64_t j = j0 + threadIdx.x + (int64_t)r * TOPK_THREADS;
        uint64_t key = 0ull;
        if (j < L) key = S ? topk_key(S[j + L * qi], (uint32_t)(j + 1 + id_offset)) : kin[qi * L + j];
        kv[r] = key;
        mx = key > mx ? key : mx;
      }
      keys[threadIdx.x] = mx;
      if (threadIdx.x == 0) nsurv = 0;
      bitonic_desc(keys, TOPK_THREADS);  // ends with a block barrier
      const uint64_t t = keys[k - 1];
      __syncthreads();
#pragma unroll
      for (int r = 0; r < TOPK_PER; ++r)
        if (kv[r] != 0ull && kv[r] >= t) {
          const int pos = atomicAdd(&nsurv, 1);
          if (pos < TOPK_THREADS) keys[pos] = kv[r];  // always, by the bound above
        }
      __syncthreads();
      for (int i = min(nsurv, TOPK_THREADS) + threadIdx.x; i < TOPK_THREADS; i += TOPK_THREADS) keys[i] = 0ull;
      bitonic_desc(keys, TOPK_THREADS);
    } else {
      for (int i = threadIdx.x; i < TOPK_CHUNK; i += blockDim.x) {
        int64_t j = j0 + i;
        uint64_t key = 0ull;
        if (j < L) key = S ? topk_key(S[j + L * qi], (uint32_t)(j + 1 + id_offset)) : kin[qi * L + j];
        keys[i] = key;
      }
      bitonic_desc(keys, TOPK_CHUNK);
    }
    for (int i = threadIdx.x; i < k; i += blockDim.x)
      kout[(qi * nchunks + c) * k + i] = keys[i];
  }
}

// Final write-out of the first k keys of each query's (sorted) list.
__global__ void topk_write_kernel(const uint64_t* __restrict__ kin, int64_t L, int nq, int k,
                                  float* __restrict__ vals, int32_t* __restrict__ ids) {
  int64_t n = (int64_t)nq * k;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t qi = i / k, r = i % k;
    uint64_t key = r < L ? kin[qi * L + r] : 0ull;
    vals[i] = key ? key_val(key) : -INFINITY;
    ids[i] = key ? (int32_t)key_id(key) : 0;
  }
}

static int64_t topk_round_len(int64_t L, int k) {
  return ((L + TOPK_CHUNK - 1) / TOPK_CHUNK) * k;
}

size_t topk_workspace_bytes(int nq, int64_t N, int k) {
  int64_t L1 = topk_round_len(N, k);
  return 2 * ((size_t)nq * (size_t)L1 * 8 + 256);
}

cudaError_t launch_topk(const float* S, int64_t N, int nq, int k, int64_t id_offset, void* ws,
                        float* vals, int32_t* ids, cudaStream_t s) {
  if (nq == 0 || k == 0) return cudaSuccess;
  const size_t smem = (size_t)TOPK_CHUNK * 8;
  cudaError_t e = cudaFuncSetAttribute(topk_round_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  int64_t L1 = topk_round_len(N, k);
  uint64_t* bufA = static_cast<uint64_t*>(ws);
  uint64_t* bufB = reinterpret_cast<uint64_t*>(static_cast<char*>(ws) + (size_t)nq * (size_t)L1 * 8 + 256);
  const int64_t cap = (int64_t)device_sm_count() * 2;
  int64_t L = N;
  const uint64_t* in = nullptr;
  uint64_t* out = bufA;
  bool first = true;
  // Rounds until a single chunk remains; each round shrinks L by TOPK_CHUNK/k >= 2.
  while (true) {
    int64_t jobs = ((L + TOPK_CHUNK - 1) / TOPK_CHUNK) * nq;
    topk_round_kernel<<<(unsigned)(jobs < cap ? jobs : cap), TOPK_THREADS, smem, s>>>(
        first ? S : nullptr, in, L, nq, k, id_offset, out);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    int64_t Ln = topk_round_len(L, k);
    bool done = L <= TOPK_CHUNK;
    first = false;
    in = out;
    out = (out == bufA) ? bufB : bufA;
    L = Ln;
    if (done) break;
  }
  int64_t n = (int64_t)nq * k;
  topk_write_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(in, L, nq, k, vals, ids);
  return cudaGetLastError();
}

// Merge nshard lists (k,nq,nshard) of already-ranked (value, id) pairs.
__global__ void __launch_bounds__(1024) topk_merge_kernel(const float* __restrict__ vals,
                                                          const int32_t* __restrict__ ids, int k,
                                                          int nq, int nshard, float* __restrict__ ov,
                                                          int32_t* __restrict__ oi) {
  extern __shared__ uint64_t mk[];
  const int qi = blockIdx.x;
  const int n_in = k * nshard;
  int n = 1;
  while (n < n_in) n <<= 1;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    uint64_t key = 0ull;
    if (i < n_in) {
      int sh = i / k, r = i % k;
      int64_t src = ((int64_t)sh * nq + qi) * k + r;
      int32_t id = ids[src];
      key = id > 0 ? topk_key(vals[src], (uint32_t)id) : 0ull;
    }
    mk[i] = key;
  }
  bitonic_desc(mk, n);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    uint64_t key = mk[i];
    ov[(int64_t)qi * k + i] = key ? key_val(key) : -INFINITY;
    oi[(int64_t)qi * k + i] = key ? (int32_t)key_id(key) : 0;
  }
}

cudaError_t launch_topk_merge(const float* vals, const int32_t* ids, int k, int nq, int nshard,
                              float* ov, int32_t* oi, cudaStream_t s) {
  if (nq == 0 || k == 0) return cudaSuccess;
  int64_t n_in = (int64_t)k * nshard, n = 1;
  while (n < n_in) n <<= 1;
  size_t smem = (size_t)n * 8;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(topk_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  topk_merge_kernel<<<nq, 1024, smem, s>>>(vals, ids, k, nq, nshard, ov, oi);
  return cudaGetLastError();
}

// Slots whose idx is outside 1:N get `neg` after a sharded max-merge.
__global__ void cand_neg_kernel(const int32_t* __restrict__ idxs, int64_t N, int64_t n, float neg,
                                float* __restrict__ S) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t j = idxs[i];
    if (!(j >= 1 && j <= N)) S[i] = neg;
  }
}

cudaError_t launch_cand_neg(const int32_t* idxs, int64_t N, int64_t n, float neg, float* S,
                            cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  int64_t g = (n + 255) / 256;
  if (g > 4096) g = 4096;
  cand_neg_kernel<<<(unsigned)g, 256, 0, s>>>(idxs, N, n, neg, S);
  return cudaGetLastError();
}

}  // namespace fms
