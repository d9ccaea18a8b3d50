// fms_backward.cu -- sparse MaxSim backward from the argmax tape (Eqs. 2-3):
//   dQ[:,t] = sum over units using query token t of  delta_u * D[:, u*]
//   dD[:,u] = sum over (unit, t) whose argmax is u of delta_u * Q[:, t]
// with delta_u = T(Delta[u] * inv_n[q(u)]) formed in T (rrule.jl:77,94,112;
// backward_layouts.jl:19,79,146).  Two strategies, as the reference's
// BackwardStrategy (types.jl:8-17):
//  * AtomicUnified (kernels_backward.jl:69-138): one fused launch; a warp per
//    query token walks the units that use it, gathers dQ in registers and
//    scatters dD with float32 atomics (into dD directly for f32/f64, into a
//    float32 workspace then one conversion pass for 16-bit T).
//  * InvGrid (kernels_backward.jl:146-354, csr_ka.jl): inverse-grid CSR built
//    by a parallel counting sort (atomic count -> block-parallel exclusive scan,
//    replacing the reference's one-thread serial prefix -> atomic fill), then a
//    destination-owned scatter: a warp per document token sums its sources in
//    ascending source order (segments up to 1024 sources are ranked in shared
//    memory by the scatter warp; longer segments are sorted in place first, one
//    block each), so dD is deterministic run to run whatever the segment
//    lengths, unlike the reference's atomic-order fill.  The dQ gather is the
//    same warp-per-token kernel.
// Accumulation is float32 (float64 for T = Float64) and each gradient element
// is rounded to T once.
#include "fms_common.cuh"
#include "fms_internal.h"

namespace fms {

// Units that read query-token row r: a contiguous id range [u0, u0+cnt).
__device__ inline void units_of_row(const ScanParams& p, int64_t r, int64_t& u0, int64_t& cnt,
                                    int& t) {
  switch (p.layout) {
    case L_PAIRED: t = (int)(r % p.Tq); u0 = r / p.Tq; cnt = 1; break;
    case L_CANDIDATES: t = (int)(r % p.Tq); u0 = (r / p.Tq) * p.C; cnt = p.C; break;
    case L_INBATCH: t = (int)(r % p.Tq); u0 = (r / p.Tq) * p.Bd; cnt = p.Bd; break;
    case L_PACKED: t = (int)(r % p.Tq); u0 = (r / p.Tq) * p.B; cnt = p.B; break;
    default: {  // varlen: binary search cu_q for the pair owning token row r
      int lo = 0, hi = p.N;  // find n with cu_q[n]-1 <= r < cu_q[n+1]-1
      while (hi - lo > 1) {
        int mid = (lo + hi) >> 1;
        if ((int64_t)p.cu_q[mid] - 1 <= r) lo = mid; else hi = mid;
      }
      u0 = lo; cnt = (p.N > 0) ? 1 : 0;
      t = (int)(r - ((int64_t)p.cu_q[lo] - 1));
      break;
    }
  }
}

template <typename T>
__device__ __forceinline__ typename Tr<T>::Acc unit_delta(const BwdParams& b, int64_t u, int qidx) {
  using A = typename Tr<T>::Acc;
  const T* Dl = static_cast<const T*>(b.Delta);
  A d = Tr<T>::to(Dl[u]);
  if (b.inv_n) d = tmul<T>(d, Tr<T>::to(static_cast<const T*>(b.inv_n)[qidx]));
  return d;
}

constexpr int BW_VEC = 8;              // dim elements per lane per chunk
constexpr int BW_CHUNK = 32 * BW_VEC;  // dim elements per warp chunk

// Warp per query-token row: dQ gather (+ dD atomics when ATOMIC).
template <typename T, bool ATOMIC>
__global__ void __launch_bounds__(256) bwd_gather_kernel(BwdParams b, typename Tr<T>::Acc* dD_acc) {
  using A = typename Tr<T>::Acc;
  const ScanParams& p = b.g;
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const T* Q = static_cast<const T*>(p.Q);
  const T* D = static_cast<const T*>(p.D);
  T* dQ = static_cast<T*>(b.dQ);
  const int dim = p.dim;
  for (int64_t r = warp; r < b.nq_rows; r += nwarps) {
    int64_t u0, cnt;
    int t;
    units_of_row(p, r, u0, cnt, t);
    for (int k0 = 0; k0 < dim; k0 += BW_CHUNK) {
      A acc[BW_VEC];
      A qv[BW_VEC];
#pragma unroll
      for (int v = 0; v < BW_VEC; ++v) {
        acc[v] = (A)0;
        int k = k0 + lane + 32 * v;
        qv[v] = (ATOMIC && k < dim) ? Tr<T>::to(Q[r * dim + k]) : (A)0;
      }
      for (int64_t i = 0; i < cnt; ++i) {
        int64_t u = u0 + i;
        Unit U = decode_unit(p, u);
        if (!U.valid || t >= U.Tq || !mask_ok(U.qmask, t)) continue;
        int a = p.args[U.arg0 + t];
        if (a < 1 || a > U.Td) continue;
        A dl = unit_delta<T>(b, u, U.qidx);
        int64_t drow = U.d0 + a - 1;
#pragma unroll
        for (int v = 0; v < BW_VEC; ++v) {
          int k = k0 + lane + 32 * v;
          if (k < dim) {
            acc[v] += dl * Tr<T>::to(D[drow * dim + k]);
            if (ATOMIC) atomicAdd(&dD_acc[drow * dim + k], dl * qv[v]);
          }
        }
      }
#pragma unroll
      for (int v = 0; v < BW_VEC; ++v) {
        int k = k0 + lane + 32 * v;
        if (k < dim) dQ[r * dim + k] = Tr<T>::from(acc[v]);
      }
    }
  }
}

template <typename A, typename T>
__global__ void convert_kernel(const A* __restrict__ src, T* __restrict__ dst, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = Tr<T>::from(src[i]);
}

// ------------------------------------------------------------------ InvGrid CSR

// Sources are (unit, t) pairs, id = unit * Tq + t (Tq = max_q for varlen).
__device__ __forceinline__ bool source_dest(const ScanParams& p, int64_t s, int64_t& dest) {
  int64_t u = s / p.Tq;
  int t = (int)(s % p.Tq);
  Unit U = decode_unit(p, u);
  if (!U.valid || t >= U.Tq || !mask_ok(U.qmask, t)) return false;
  int a = p.args[U.arg0 + t];
  if (a < 1 || a > U.Td) return false;
  dest = U.d0 + a - 1;
  return true;
}

__global__ void csr_count_kernel(ScanParams p, int64_t n_src, int32_t* __restrict__ count) {
  for (int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; s < n_src;
       s += (int64_t)gridDim.x * blockDim.x) {
    int64_t dest;
    if (source_dest(p, s, dest)) atomicAdd(&count[dest], 1);
  }
}

constexpr int SCAN_BLOCK = 1024;
constexpr int SC_SEG = 1024;  // sources ranked per destination in shared memory

// In-place exclusive scan, phase 1: each block scans 1024 entries and records
// its total.  Destinations with more than SC_SEG sources (counts x[i]) are
// appended to long_list (long_cnt counts them) for the segment sort.
__global__ void __launch_bounds__(SCAN_BLOCK) scan_blocks_kernel(int32_t* __restrict__ x, int64_t n,
                                                                int32_t* __restrict__ block_sums,
                                                                int32_t* __restrict__ long_cnt,
                                                                int32_t* __restrict__ long_list) {
  __shared__ int32_t warp_sums[32];
  int64_t i = (int64_t)blockIdx.x * SCAN_BLOCK + threadIdx.x;
  int32_t v = (i < n) ? x[i] : 0;
  if (v > SC_SEG) long_list[atomicAdd(long_cnt, 1)] = (int32_t)i;
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int32_t incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    int32_t o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  if (lane == 31) warp_sums[w] = incl;
  __syncthreads();
  if (w == 0) {
    int32_t ws = warp_sums[lane];
    int32_t wi = ws;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      int32_t o = __shfl_up_sync(0xffffffffu, wi, off);
      if (lane >= off) wi += o;
    }
    warp_sums[lane] = wi - ws;  // exclusive warp offsets
    if (lane == 31) block_sums[blockIdx.x] = wi;
  }
  __syncthreads();
  if (i < n) x[i] = incl - v + warp_sums[w];
}

// Phase 2: one block scans the block totals sequentially in chunks of 1024.
__global__ void __launch_bounds__(SCAN_BLOCK) scan_sums_kernel(int32_t* __restrict__ sums, int64_t nb) {
  __shared__ int32_t warp_sums[32];
  __shared__ int32_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int64_t base = 0; base < nb; base += SCAN_BLOCK) {
    int64_t i = base + threadIdx.x;
    int32_t v = (i < nb) ? sums[i] : 0;
    int32_t incl = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      int32_t o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    if (lane == 31) warp_sums[w] = incl;
    __syncthreads();
    if (w == 0) {
      int32_t ws = warp_sums[lane];
      int32_t wi = ws;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        int32_t o = __shfl_up_sync(0xffffffffu, wi, off);
        if (lane >= off) wi += o;
      }
      warp_sums[lane] = wi - ws;
    }
    __syncthreads();
    int32_t c = carry;
    if (i < nb) sums[i] = incl - v + warp_sums[w] + c;
    __syncthreads();
    if (threadIdx.x == SCAN_BLOCK - 1) carry = c + incl + warp_sums[w];
    __syncthreads();
  }
}

// Phase 3: add block offsets; also seed the fill cursors.
__global__ void scan_add_kernel(int32_t* __restrict__ x, int64_t n, const int32_t* __restrict__ sums,
                                int32_t* __restrict__ cursor, int64_t n_dest) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int32_t v = x[i] + sums[i / SCAN_BLOCK];
    x[i] = v;
    if (i < n_dest) cursor[i] = v;
  }
}

__global__ void csr_fill_kernel(ScanParams p, int64_t n_src, int32_t* __restrict__ cursor,
                                int32_t* __restrict__ col_idx) {
  for (int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; s < n_src;
       s += (int64_t)gridDim.x * blockDim.x) {
    int64_t dest;
    if (source_dest(p, s, dest)) {
      int32_t pos = atomicAdd(&cursor[dest], 1);
      col_idx[pos] = (int32_t)s;
    }
  }
}

// Segments longer than SC_SEG: sorted ascending in place, one block per segment
// (block-stride over the list of long segments).  Tiles of SORT_TILE ids are
// bitonic-sorted in shared memory, then sorted runs are merged pairwise: the
// ids of a segment are distinct, so an id's place in the merged run is its
// index in its own run plus the number of smaller ids in the sibling run (a
// binary search).  Runs ping-pong between the segment and the same offsets of
// `tmp`, and end in the segment.
constexpr int SORT_TILE = 2048;
constexpr int SORT_THREADS = 1024;

__device__ __forceinline__ int lower_bound_i32(const int32_t* a, int n, int32_t x) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (a[mid] < x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

__global__ void __launch_bounds__(SORT_THREADS) csr_sort_long_kernel(const int32_t* __restrict__ row_ptr,
                                                                     int32_t* __restrict__ col_idx,
                                                                     int32_t* __restrict__ tmp,
                                                                     const int32_t* __restrict__ long_cnt,
                                                                     const int32_t* __restrict__ long_list) {
  __shared__ int32_t tile[SORT_TILE];
  const int nlong = *long_cnt;
  for (int li = blockIdx.x; li < nlong; li += gridDim.x) {
    const int32_t d = long_list[li];
    const int32_t a0 = row_ptr[d];
    const int n = row_ptr[d + 1] - a0;
    int32_t* seg = col_idx + a0;
    int32_t* alt = tmp + a0;
    // sorted tiles
    for (int t0 = 0; t0 < n; t0 += SORT_TILE) {
      const int len = min(SORT_TILE, n - t0);
      __syncthreads();
      for (int i = threadIdx.x; i < SORT_TILE; i += SORT_THREADS) tile[i] = i < len ? seg[t0 + i] : INT32_MAX;
      for (int size = 2; size <= SORT_TILE; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          __syncthreads();
          for (int i = threadIdx.x; i < SORT_TILE / 2; i += SORT_THREADS) {
            const int lo = 2 * i - (i & (stride - 1));
            const int hi = lo + stride;
            const bool asc = (lo & size) == 0;
            const int32_t x = tile[lo], y = tile[hi];
            if ((x > y) == asc) { tile[lo] = y; tile[hi] = x; }
          }
        }
      }
      __syncthreads();
      for (int i = threadIdx.x; i < len; i += SORT_THREADS) seg[t0 + i] = tile[i];
    }
    // pairwise merges of sorted runs of width w
    const int32_t* src = seg;
    int32_t* dst = alt;
    for (int w = SORT_TILE; w < n; w <<= 1) {
      __syncthreads();
      for (int p = threadIdx.x; p < n; p += SORT_THREADS) {
        const int r = p / w;
        const int base = (r & ~1) * w;
        const int32_t x = src[p];
        int pos;
        if ((r & 1) == 0) {
          const int lenb = min(w, max(0, n - (base + w)));
          pos = p + lower_bound_i32(src + base + w, lenb, x);
        } else {
          pos = base + (p - (base + w)) + lower_bound_i32(src + base, w, x);
        }
        dst[pos] = x;
      }
      const int32_t* t = src;
      src = dst;
      dst = const_cast<int32_t*>(t);
    }
    __syncthreads();
    if (src != seg)
      for (int p = threadIdx.x; p < n; p += SORT_THREADS) seg[p] = src[p];
    __syncthreads();
  }
}

constexpr int SC_WARPS = 8;

// ------------------------------------------------------------ in-batch CSR
// The in-batch sources of document j are the pairs (i, t) of the units
// u = i * Bd + j.  Their ids u * Tq + t ascend with e = i * Tq + t, which is
// also the query-token row the source reads.  So the CSR of one document is a
// stable counting sort of its Bq * Tq tape entries by argmax, done by one block
// in shared memory: the segments come out in ascending source order with no
// atomics on global memory and no ranking or sorting afterwards, and each
// entry is stored pre-decoded as (query row, delta) for the scatter.
constexpr int IB_THREADS = 512;
constexpr int IB_WARPS = IB_THREADS / 32;
constexpr int IB_TD_MAX = 1024;    // destinations per document
constexpr int IB_E_MAX = 16384;    // sources per document (Bq * Tq), keys staged in shared memory
constexpr int IB_BQ_MAX = 4096;    // deltas of a document's units staged in shared memory

// Destination token (argmax - 1) of source e of document j, or -1 when it
// contributes nothing (masked query token or no argmax); as source_dest().
__device__ __forceinline__ int inb_key(const ScanParams& p, int64_t j, int e) {
  const int i = e / p.Tq;
  const int t = e - i * p.Tq;
  const bool qok = p.qmask == nullptr || p.qmask[e] != 0;  // qmask row i, token t
  const int a = p.args[((int64_t)i * p.Bd + j) * p.Tq + t];
  return (qok && a >= 1 && a <= p.Td) ? a - 1 : -1;
}

// Sources of each document (one block per document).
__global__ void __launch_bounds__(IB_THREADS) inb_csr_total_kernel(ScanParams p, int32_t* __restrict__ doc_tot) {
  __shared__ int32_t ws[IB_WARPS];
  const int64_t j = blockIdx.x;
  const int E = p.Bq * p.Tq;
  int n = 0;
#pragma unroll 4
  for (int e = threadIdx.x; e < E; e += IB_THREADS) n += inb_key(p, j, e) >= 0 ? 1 : 0;
  n = __reduce_add_sync(0xffffffffu, n);
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = n;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < IB_WARPS; ++w) t += ws[w];
    doc_tot[j] = t;
  }
}

// Shared memory of inb_csr_build_kernel: per-warp counts [IB_WARPS][Td],
// segment starts [Td], unit deltas [Bq], source keys [Bq * Tq] (int16).
static size_t inb_csr_smem(int Td, int Bq, int Tq) {
  return (size_t)(IB_WARPS + 1) * Td * 4 + (size_t)Bq * 4 + (size_t)Bq * Tq * 2;
}

// One document per block: its segments (row_ptr) and its sources in
// ascending order as (query row, delta).  doc_base[j] = sources of the
// documents before j; the last block also writes row_ptr[Bd * Td].
template <typename T>
__global__ void __launch_bounds__(IB_THREADS)
inb_csr_build_kernel(BwdParams b, const int32_t* __restrict__ doc_base, int32_t* __restrict__ row_ptr,
                     int32_t* __restrict__ qrow, float* __restrict__ coef) {
  extern __shared__ int32_t ib_s[];
  __shared__ int32_t wsum[IB_WARPS];
  const ScanParams& p = b.g;
  const int64_t j = blockIdx.x;
  const int Td = p.Td;
  const int E = p.Bq * p.Tq;
  const int per = ((E + IB_WARPS - 1) / IB_WARPS + 31) & ~31;  // sources per warp, whole chunks
  int32_t* hist = ib_s;                                       // [IB_WARPS][Td]
  int32_t* bin = hist + IB_WARPS * Td;                        // [Td]
  float* cq = reinterpret_cast<float*>(bin + Td);             // [Bq]
  int16_t* key = reinterpret_cast<int16_t*>(cq + p.Bq);       // [E]
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  for (int x = tid; x < IB_WARPS * Td; x += IB_THREADS) hist[x] = 0;
  for (int i = tid; i < p.Bq; i += IB_THREADS) cq[i] = unit_delta<T>(b, (int64_t)i * p.Bd + j, i);
  __syncthreads();
  // pass 1: keys (the tape loads of a thread all in flight at once, no
  // atomics between them), then counted per owning warp (warp w owns sources
  // [w * per, (w + 1) * per))
#pragma unroll 8
  for (int e = tid; e < E; e += IB_THREADS) key[e] = (int16_t)inb_key(p, j, e);
  __syncthreads();
  for (int e = tid; e < E; e += IB_THREADS) {
    const int k = key[e];
    if (k >= 0) atomicAdd(&hist[(e / per) * Td + k], 1);
  }
  __syncthreads();
  // pass 2: per destination the warps' counts become running offsets; the
  // destination totals are scanned (contiguous destinations per thread)
  const int bpt = (Td + IB_THREADS - 1) / IB_THREADS;
  const int a0 = min(Td, tid * bpt), a1 = min(Td, a0 + bpt);
  int mysum = 0;
  for (int a = a0; a < a1; ++a) {
    int run = 0;
    for (int ww = 0; ww < IB_WARPS; ++ww) {
      const int h = hist[ww * Td + a];
      hist[ww * Td + a] = run;
      run += h;
    }
    bin[a] = run;
    mysum += run;
  }
  int incl = mysum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) wsum[w] = incl;
  __syncthreads();
  int before = 0, total = 0;
  for (int ww = 0; ww < IB_WARPS; ++ww) {
    before += ww < w ? wsum[ww] : 0;
    total += wsum[ww];
  }
  int off = before + incl - mysum;
  for (int a = a0; a < a1; ++a) {
    const int n = bin[a];
    bin[a] = off;
    off += n;
  }
  __syncthreads();
  const int32_t base = doc_base[j];
  for (int a = tid; a < Td; a += IB_THREADS) {
    const int st = bin[a];
    row_ptr[j * Td + a] = base + st;
    for (int ww = 0; ww < IB_WARPS; ++ww) hist[ww * Td + a] += st;
  }
  if (j == p.Bd - 1 && tid == 0) row_ptr[(int64_t)p.Bd * Td] = base + total;
  __syncthreads();
  // pass 3: each warp places its sources in order; lanes with the same
  // destination take consecutive places in lane order
  const int e_lo = w * per, e_hi = min(E, e_lo + per);
  for (int e0 = e_lo; e0 < e_hi; e0 += 32) {
    const int e = e0 + lane;
    const int k = e < e_hi ? (int)key[e] : -1;
    const uint32_t peers = __match_any_sync(0xffffffffu, k >= 0 ? k : 0x100000 + lane);
    if (k >= 0) {
      const int pos = base + hist[w * Td + k] + __popc(peers & ((1u << lane) - 1u));
      qrow[pos] = e;
      coef[pos] = cq[e / p.Tq];
    }
    __syncwarp();
    if (k >= 0 && lane == __ffs(peers) - 1) hist[w * Td + k] += __popc(peers);
    __syncwarp();
  }
}

// Warp per destination document token; sources summed in ascending id order.
template <typename T>
__global__ void __launch_bounds__(SC_WARPS * 32)
csr_scatter_kernel(BwdParams b, const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col_idx) {
  using A = typename Tr<T>::Acc;
  __shared__ int32_t seg_s[SC_WARPS][SC_SEG];
  const ScanParams& p = b.g;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int32_t* seg = seg_s[w];
  const T* Q = static_cast<const T*>(p.Q);
  T* dD = static_cast<T*>(b.dD);
  const int dim = p.dim;
  const int64_t warp = (int64_t)blockIdx.x * SC_WARPS + w;
  const int64_t nwarps = (int64_t)gridDim.x * SC_WARPS;
  for (int64_t d = warp; d < b.nd_rows; d += nwarps) {
    const int32_t a0 = row_ptr[d], n = row_ptr[d + 1] - a0;
    const bool ranked = n <= SC_SEG;
    if (ranked) {
      // rank each source id by counting smaller ids (ids are distinct)
      for (int i = lane; i < n; i += 32) {
        int32_t x = col_idx[a0 + i];
        int r = 0;
        for (int j = 0; j < n; ++j) r += (col_idx[a0 + j] < x) ? 1 : 0;
        seg[r] = x;
      }
      __syncwarp();
    }
    for (int k0 = 0; k0 < dim; k0 += BW_CHUNK) {
      A acc[BW_VEC];
#pragma unroll
      for (int v = 0; v < BW_VEC; ++v) acc[v] = (A)0;
      for (int i = 0; i < n; ++i) {
        int64_t s = ranked ? seg[i] : col_idx[a0 + i];
        int64_t u = s / p.Tq;
        int t = (int)(s % p.Tq);
        Unit U = decode_unit(p, u);
        A dl = unit_delta<T>(b, u, U.qidx);
        int64_t qrow = U.q0 + t;
#pragma unroll
        for (int v = 0; v < BW_VEC; ++v) {
          int k = k0 + lane + 32 * v;
          if (k < dim) acc[v] += dl * Tr<T>::to(Q[qrow * dim + k]);
        }
      }
#pragma unroll
      for (int v = 0; v < BW_VEC; ++v) {
        int k = k0 + lane + 32 * v;
        if (k < dim) dD[d * dim + k] = Tr<T>::from(acc[v]);
      }
    }
    __syncwarp();
  }
}

// ------------------------------------------------------------------ vector paths
//
// Rows of 16-bit or f32 features move as 16-byte vectors: lane l of a warp
// owns vectors l, l + 32, ... of a row (NV per lane), so one warp covers a
// whole row (dim <= 256 * NV * 16 / sizeof(T) bytes) in a single pass over its
// units or sources, with two rows in flight per warp and registers capped so
// that two 8-warp blocks share an SM.  The sums run in the same order as the
// scalar kernels (units ascending, sources ascending), so the results
// are identical.

template <typename T> struct V16 { static constexpr int E = 16 / (int)sizeof(T); };

__device__ __forceinline__ void unpack(const uint4& v, float (&x)[8], __nv_bfloat16*) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    x[2 * i] = f.x; x[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void unpack(const uint4& v, float (&x)[8], __half*) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    x[2 * i] = f.x; x[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void unpack(const uint4& v, float (&x)[4], float*) {
  x[0] = __uint_as_float(v.x); x[1] = __uint_as_float(v.y);
  x[2] = __uint_as_float(v.z); x[3] = __uint_as_float(v.w);
}
__device__ __forceinline__ uint4 pack(const float (&x)[8], __nv_bfloat16*) {
  uint4 v;
  uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return v;
}
__device__ __forceinline__ uint4 pack(const float (&x)[8], __half*) {
  uint4 v;
  uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 h = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return v;
}
__device__ __forceinline__ uint4 pack(const float (&x)[4], float*) {
  return make_uint4(__float_as_uint(x[0]), __float_as_uint(x[1]), __float_as_uint(x[2]), __float_as_uint(x[3]));
}

// Source row and delta of one (unit, token) pair, or false when it contributes
// nothing (masked token, invalid slot, no argmax).  In-batch units of query
// row r are u = i * Bd + j with i = r / Tq fixed, so the caller passes i and j.
template <typename T, bool INB>
__device__ __forceinline__ bool unit_row(const BwdParams& b, int64_t u, int64_t i, int64_t j, int t,
                                         int64_t& drow, float& dl) {
  const ScanParams& p = b.g;
  if constexpr (INB) {
    if (p.qmask && !p.qmask[i * p.Tq + t]) return false;
    const int a = p.args[u * p.Tq + t];
    if (a < 1 || a > p.Td) return false;
    drow = j * p.Td + a - 1;
    dl = unit_delta<T>(b, u, (int)i);
    return true;
  } else {
    Unit U = decode_unit(p, u);
    if (!U.valid || t >= U.Tq || !mask_ok(U.qmask, t)) return false;
    const int a = p.args[U.arg0 + t];
    if (a < 1 || a > U.Td) return false;
    drow = U.d0 + a - 1;
    dl = unit_delta<T>(b, u, U.qidx);
    return true;
  }
}

// Warp per query-token row: dQ gather (+ dD float32 atomics when ATOMIC).
constexpr int VEC_UNROLL = 2;  // rows in flight per warp

// Rows (documents or sources) in flight per warp: four for rows of up to 96 vectors, two for
// wider ones (register budget)
template <int NV> struct RowsInFlight { static constexpr int n = NV <= 3 ? 4 : 2; };

// In-batch dQ (no atomics): the tape entries and deltas of 32 documents are
// loaded at once, one per lane, and broadcast; RowsInFlight rows are in flight
// at a time.  Documents are still summed in ascending order with one
// fused multiply-add per element, so the result is the same as the generic
// kernel's.

template <typename T, int NV>
__device__ __forceinline__ void inb_gather_row(const BwdParams& b, int64_t r, int lane) {
  constexpr int E = V16<T>::E;
  constexpr int GB_ROWS = RowsInFlight<NV>::n;
  const ScanParams& p = b.g;
  const uint4* D = static_cast<const uint4*>(p.D);
  uint4* dQ = static_cast<uint4*>(b.dQ);
  const int nvec = p.dim / E;
  const int64_t qi = r / p.Tq;
  const int t = (int)(r - qi * p.Tq);
  const bool live = p.qmask == nullptr || p.qmask[qi * p.Tq + t];
  float acc[NV][E];
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int e = 0; e < E; ++e) acc[k][e] = 0.f;
  for (int64_t j0 = 0; live && j0 < p.Bd; j0 += 32) {
    // lane d: document j0 + d
    int my_a = 0;
    float my_dl = 0.f;
    if (j0 + lane < p.Bd) {
      const int64_t u = qi * p.Bd + j0 + lane;
      my_a = p.args[u * p.Tq + t];
      if (my_a >= 1 && my_a <= p.Td) my_dl = unit_delta<T>(b, u, (int)qi);
      else my_a = 0;
    }
    const int nd = (int)min((int64_t)32, p.Bd - j0);
    if (nd == 32 && __all_sync(0xffffffffu, my_a != 0)) {
      // every document of the batch contributes: no per-row tests (a branch
      // costs more here than the loads and FMAs it guards)
#pragma unroll 1
      for (int d0 = 0; d0 < 32; d0 += GB_ROWS) {
        float dl[GB_ROWS];
        uint4 dv[GB_ROWS][NV];
#pragma unroll
        for (int q = 0; q < GB_ROWS; ++q) {
          const int aq = __shfl_sync(0xffffffffu, my_a, d0 + q);
          dl[q] = __shfl_sync(0xffffffffu, my_dl, d0 + q);
          const int64_t drow = (j0 + d0 + q) * p.Td + aq - 1;
#pragma unroll
          for (int k = 0; k < NV; ++k) {
            const int v = lane + 32 * k;
            if (v < nvec) dv[q][k] = D[drow * nvec + v];
          }
        }
#pragma unroll
        for (int q = 0; q < GB_ROWS; ++q)
#pragma unroll
          for (int k = 0; k < NV; ++k) {
            const int v = lane + 32 * k;
            if (v < nvec) {
              float x[E];
              unpack(dv[q][k], x, (T*)nullptr);
#pragma unroll
              for (int e = 0; e < E; ++e) acc[k][e] += dl[q] * x[e];
            }
          }
      }
      continue;
    }
    // a partial batch (the last one, or invalid tape entries): one row at a time
    for (int d = 0; d < nd; ++d) {
      const int ad = __shfl_sync(0xffffffffu, my_a, d);
      const float dl = __shfl_sync(0xffffffffu, my_dl, d);
      if (!ad) continue;
      const int64_t drow = (j0 + d) * p.Td + ad - 1;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int v = lane + 32 * k;
        if (v < nvec) {
          float x[E];
          unpack(D[drow * nvec + v], x, (T*)nullptr);
#pragma unroll
          for (int e = 0; e < E; ++e) acc[k][e] += dl * x[e];
        }
      }
    }
  }
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int v = lane + 32 * k;
    if (v < nvec) dQ[r * nvec + v] = pack(acc[k], (T*)nullptr);
  }
}

// dQ of the other layouts (no atomics): the units of a row are decoded 32 at a
// time (one per lane: slot, validity, tape entry, delta), then their document
// rows are summed in ascending unit order with RowsInFlight rows in flight;
// units that contribute nothing read row 0 and are discarded by a select, so
// the sum is the one of the one-row-at-a-time kernel, bit for bit.
template <typename T, int NV>
__device__ __forceinline__ void gen_gather_row(const BwdParams& b, int64_t r, int lane) {
  constexpr int E = V16<T>::E;
  constexpr int R = RowsInFlight<NV>::n;
  const ScanParams& p = b.g;
  const uint4* D = static_cast<const uint4*>(p.D);
  uint4* dQ = static_cast<uint4*>(b.dQ);
  const int nvec = p.dim / E;
  int64_t u0, cnt;
  int t;
  units_of_row(p, r, u0, cnt, t);
  float acc[NV][E];
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int e = 0; e < E; ++e) acc[k][e] = 0.f;
  for (int64_t i0 = 0; i0 < cnt; i0 += 32) {
    int64_t my_row = -1;
    float my_dl = 0.f;
    if (i0 + lane < cnt) {
      int64_t dr;
      float dl;
      if (unit_row<T, false>(b, u0 + i0 + lane, 0, i0 + lane, t, dr, dl)) {
        my_row = dr;
        my_dl = dl;
      }
    }
    const int nd = (int)min((int64_t)32, cnt - i0);
#pragma unroll 1
    for (int c0 = 0; c0 < nd; c0 += R) {
      float dl[R];
      bool use[R];
      uint4 dv[R][NV];
#pragma unroll
      for (int q = 0; q < R; ++q) {
        int64_t dr = __shfl_sync(0xffffffffu, my_row, (c0 + q) & 31);
        dl[q] = __shfl_sync(0xffffffffu, my_dl, (c0 + q) & 31);
        use[q] = c0 + q < nd && dr >= 0;
        dr = use[q] ? dr : 0;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
          const int v = lane + 32 * k;
          if (v < nvec) dv[q][k] = D[dr * nvec + v];
        }
      }
#pragma unroll
      for (int q = 0; q < R; ++q)
#pragma unroll
        for (int k = 0; k < NV; ++k) {
          const int v = lane + 32 * k;
          if (v < nvec) {
            float x[E];
            unpack(dv[q][k], x, (T*)nullptr);
#pragma unroll
            for (int e = 0; e < E; ++e) {
              const float y = acc[k][e] + dl[q] * x[e];
              acc[k][e] = use[q] ? y : acc[k][e];
            }
          }
        }
    }
  }
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int v = lane + 32 * k;
    if (v < nvec) dQ[r * nvec + v] = pack(acc[k], (T*)nullptr);
  }
}

template <typename T, bool ATOMIC, int NV, bool INB>
__global__ void __launch_bounds__(256, 2) bwd_gather_vec_kernel(BwdParams b, float* dD_acc) {
  constexpr int E = V16<T>::E;
  const ScanParams& p = b.g;
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const uint4* Q = static_cast<const uint4*>(p.Q);
  const uint4* D = static_cast<const uint4*>(p.D);
  uint4* dQ = static_cast<uint4*>(b.dQ);
  const int nvec = p.dim / E;  // 16-byte vectors per row
  if constexpr (INB && !ATOMIC) {
    for (int64_t r = warp; r < b.nq_rows; r += nwarps) inb_gather_row<T, NV>(b, r, lane);
  } else if constexpr (!ATOMIC) {
    for (int64_t r = warp; r < b.nq_rows; r += nwarps) gen_gather_row<T, NV>(b, r, lane);
  } else {
    for (int64_t r = warp; r < b.nq_rows; r += nwarps) {
      int64_t u0, cnt;
      int t;
      units_of_row(p, r, u0, cnt, t);
      const int64_t qi = INB ? r / p.Tq : 0;
      float acc[NV][E];
      float qv[NV][E];
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int v = lane + 32 * k;
#pragma unroll
        for (int e = 0; e < E; ++e) { acc[k][e] = 0.f; qv[k][e] = 0.f; }
        if (ATOMIC && v < nvec) unpack(Q[r * nvec + v], qv[k], (T*)nullptr);
      }
      for (int64_t i0 = 0; i0 < cnt; i0 += VEC_UNROLL) {
        int64_t drow[VEC_UNROLL];
        float dl[VEC_UNROLL];
        bool ok[VEC_UNROLL];
#pragma unroll
        for (int q = 0; q < VEC_UNROLL; ++q) {
          ok[q] = i0 + q < cnt && unit_row<T, INB>(b, u0 + i0 + q, qi, i0 + q, t, drow[q], dl[q]);
        }
        uint4 dv[VEC_UNROLL][NV];
#pragma unroll
        for (int q = 0; q < VEC_UNROLL; ++q)
#pragma unroll
          for (int k = 0; k < NV; ++k) {
            const int v = lane + 32 * k;
            if (ok[q] && v < nvec) dv[q][k] = D[drow[q] * nvec + v];
          }
#pragma unroll
        for (int q = 0; q < VEC_UNROLL; ++q) {
          if (!ok[q]) continue;
#pragma unroll
          for (int k = 0; k < NV; ++k) {
            const int v = lane + 32 * k;
            if (v < nvec) {
              float x[E];
              unpack(dv[q][k], x, (T*)nullptr);
#pragma unroll
              for (int e = 0; e < E; ++e) acc[k][e] += dl[q] * x[e];
              if (ATOMIC) {
                float* dst = dD_acc + (drow[q] * nvec + v) * E;
#pragma unroll
                for (int e = 0; e < E; e += 4)
                  atomicAdd(reinterpret_cast<float4*>(dst + e),
                            make_float4(dl[q] * qv[k][e], dl[q] * qv[k][e + 1], dl[q] * qv[k][e + 2],
                                        dl[q] * qv[k][e + 3]));
              }
            }
          }
        }
      }
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int v = lane + 32 * k;
        if (v < nvec) dQ[r * nvec + v] = pack(acc[k], (T*)nullptr);
      }
    }
  }
}

// Warp per destination document token: sources summed in ascending id order.
// PRE: the segments are already in ascending order and hold (query row,
// delta) pairs (col_idx, coef) instead of source ids.

template <typename T, int NV, bool INB, bool PRE = false>
__global__ void __launch_bounds__(SC_WARPS * 32, NV <= 3 ? 3 : 2)
csr_scatter_vec_kernel(BwdParams b, const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col_idx,
                       const float* __restrict__ coef = nullptr) {
  constexpr int E = V16<T>::E;
  constexpr int SC_ROWS = 2;  // rows in flight (up to three blocks per SM share the registers)
  __shared__ int32_t seg_s[SC_WARPS][SC_SEG];
  const ScanParams& p = b.g;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int32_t* seg = seg_s[w];
  const uint4* Q = static_cast<const uint4*>(p.Q);
  uint4* dD = static_cast<uint4*>(b.dD);
  const int nvec = p.dim / E;
  const int64_t warp = (int64_t)blockIdx.x * SC_WARPS + w;
  const int64_t nwarps = (int64_t)gridDim.x * SC_WARPS;
  // one destination: its sources (col_idx[a0 .. a0 + n)) summed in ascending
  // id order into dD row d
  auto do_dest = [&](int64_t d, int32_t a0, int32_t n) {
    const bool ranked = !PRE && n <= SC_SEG;
    if (!PRE && n <= 128) {
      // up to 128 sources: four per lane in registers, each ranked by counting
      // the smaller ids among all of them, broadcast 32 at a time by shuffles
      // (no loads or branches in the count; ids are distinct, padding is
      // INT32_MAX and never smaller)
      int32_t v[4];
      int rk[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        v[c] = 32 * c + lane < n ? col_idx[a0 + 32 * c + lane] : INT32_MAX;
        rk[c] = 0;
      }
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        if (32 * cc >= n) break;  // warp-uniform
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int32_t y = __shfl_sync(0xffffffffu, v[cc], jj);
#pragma unroll
          for (int c = 0; c < 4; ++c) rk[c] += y < v[c] ? 1 : 0;
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (32 * c + lane < n) seg[rk[c]] = v[c];
      __syncwarp();
    } else if (ranked) {
      // rank each source id by counting smaller ids (ids are distinct)
      for (int i = lane; i < n; i += 32) {
        const int32_t x = col_idx[a0 + i];
        int rk = 0;
        for (int j = 0; j < n; ++j) rk += (col_idx[a0 + j] < x) ? 1 : 0;
        seg[rk] = x;
      }
      __syncwarp();
    }
    float acc[NV][E];
#pragma unroll
    for (int k = 0; k < NV; ++k)
#pragma unroll
      for (int e = 0; e < E; ++e) acc[k][e] = 0.f;
    for (int i0 = 0; i0 < n; i0 += 32) {
      // lane l decodes source i0 + l (its query row and delta) once; the
      // rows are then broadcast and summed in ascending order, SC_ROWS rows
      // in flight
      int64_t my_row = -1;
      float my_dl = 0.f;
      if (PRE) {
        if (i0 + lane < n) {
          my_row = col_idx[a0 + i0 + lane];
          my_dl = coef[a0 + i0 + lane];
        }
      } else if (i0 + lane < n) {
        // source ids are int32 (the CSR stores them so): 32-bit division
        const uint32_t s = (uint32_t)(ranked ? seg[i0 + lane] : col_idx[a0 + i0 + lane]);
        const uint32_t u = s / (uint32_t)p.Tq;
        const int t = (int)(s - u * (uint32_t)p.Tq);
        if constexpr (INB) {
          const int64_t qi = u / (uint32_t)p.Bd;
          my_row = qi * p.Tq + t;
          my_dl = unit_delta<T>(b, u, (int)qi);
        } else {
          const Unit U = decode_unit(p, u);
          my_row = U.q0 + t;
          my_dl = unit_delta<T>(b, u, U.qidx);
        }
      }
      const int ns = min(32, n - i0);
      // SC_ROWS rows in flight; rows past the batch end read row 0 and are
      // discarded by a select (a per-row branch costs more than the selects)
#pragma unroll 1
      for (int c0 = 0; c0 < ns; c0 += SC_ROWS) {
        float dl[SC_ROWS];
        bool use[SC_ROWS];
        uint4 qv[SC_ROWS][NV];
#pragma unroll
        for (int q = 0; q < SC_ROWS; ++q) {
          use[q] = c0 + q < ns;
          int64_t qr = __shfl_sync(0xffffffffu, my_row, (c0 + q) & 31);
          dl[q] = __shfl_sync(0xffffffffu, my_dl, (c0 + q) & 31);
          qr = use[q] ? qr : 0;
#pragma unroll
          for (int k = 0; k < NV; ++k) {
            const int v = lane + 32 * k;
            if (v < nvec) qv[q][k] = Q[qr * nvec + v];
          }
        }
#pragma unroll
        for (int q = 0; q < SC_ROWS; ++q)
#pragma unroll
          for (int k = 0; k < NV; ++k) {
            const int v = lane + 32 * k;
            if (v < nvec) {
              float x[E];
              unpack(qv[q][k], x, (T*)nullptr);
#pragma unroll
              for (int e = 0; e < E; ++e) {
                const float y = acc[k][e] + dl[q] * x[e];
                acc[k][e] = use[q] ? y : acc[k][e];
              }
            }
          }
      }
    }
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int v = lane + 32 * k;
      if (v < nvec) dD[d * nvec + v] = pack(acc[k], (T*)nullptr);
    }
    __syncwarp();
  };
  if (b.nd_rows >= 64 * nwarps) {
    // many destinations per warp (a whole gallery's gradient, mostly empty):
    // 32 consecutive destinations per step, their row_ptr entries loaded by
    // the lanes at once, the empty ones written as zero rows without their own
    // dependent loads, the others summed one by one
    for (int64_t d0 = warp * 32; d0 < b.nd_rows; d0 += nwarps * 32) {
      const int64_t dl = d0 + lane;
      int32_t my_a0 = 0, my_n = 0;
      if (dl < b.nd_rows) {
        my_a0 = row_ptr[dl];
        my_n = row_ptr[dl + 1] - my_a0;
      }
      const uint32_t inr = __ballot_sync(0xffffffffu, dl < b.nd_rows);
      const uint32_t ne = __ballot_sync(0xffffffffu, my_n > 0);
      uint32_t em = inr & ~ne;
      if (ne == 0u) {
        // no destination of the step has a source: its rows are one contiguous
        // block of zeros, written with every lane
        const int64_t nv = (int64_t)__popc(inr) * nvec;
        for (int64_t v = lane; v < nv; v += 32) dD[d0 * nvec + v] = make_uint4(0u, 0u, 0u, 0u);
        continue;
      }
      while (em) {
        const int j = __ffs(em) - 1;
        em &= em - 1;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
          const int v = lane + 32 * k;
          if (v < nvec) dD[(d0 + j) * nvec + v] = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      uint32_t nm = ne;
      while (nm) {
        const int j = __ffs(nm) - 1;
        nm &= nm - 1;
        do_dest(d0 + j, __shfl_sync(0xffffffffu, my_a0, j), __shfl_sync(0xffffffffu, my_n, j));
      }
    }
  } else {
    for (int64_t d = warp; d < b.nd_rows; d += nwarps) do_dest(d, row_ptr[d], row_ptr[d + 1] - row_ptr[d]);
  }
}

// 16-byte vectors per lane for a row of `dim` elements of T, or 0 when the
// vector paths do not apply (dim not a whole number of vectors, misaligned
// base pointers, rows over 32 * 5 vectors, or T = double).
template <typename T>
static int vec_lanes(const BwdParams& b) {
  if (sizeof(T) == 8) return 0;
  constexpr int E = V16<T>::E;
  const ScanParams& p = b.g;
  if (p.dim % E != 0) return 0;
  const uintptr_t m = reinterpret_cast<uintptr_t>(p.Q) | reinterpret_cast<uintptr_t>(p.D) |
                      reinterpret_cast<uintptr_t>(b.dQ) | reinterpret_cast<uintptr_t>(b.dD);
  if (m & 15) return 0;
  const int nvec = p.dim / E;
  const int nv = (nvec + 31) / 32;
  return nv <= 5 ? nv : 0;  // wider rows keep the scalar kernels (register budget)
}

// Launch the vector gather / scatter when vec_lanes() allows; false otherwise.
template <typename T, bool ATOMIC>
static bool launch_gather_vec(const BwdParams& b, float* acc, unsigned grid, cudaStream_t s) {
  if constexpr (sizeof(T) == 8) {
    return false;
  } else {
  switch (vec_lanes<T>(b)) {
#define FMS_GV(NV)                                                                           \
  case NV:                                                                                   \
    if (b.g.layout == L_INBATCH) bwd_gather_vec_kernel<T, ATOMIC, NV, true><<<grid, 256, 0, s>>>(b, acc); \
    else bwd_gather_vec_kernel<T, ATOMIC, NV, false><<<grid, 256, 0, s>>>(b, acc);           \
    return true;
    FMS_GV(1) FMS_GV(2) FMS_GV(3) FMS_GV(4) FMS_GV(5)
#undef FMS_GV
    default: return false;
  }
  }
}
// coef != nullptr: the in-batch CSR of inb_csr_build_kernel (pre-decoded).
template <typename T>
static bool launch_scatter_vec(const BwdParams& b, const int32_t* row_ptr, const int32_t* col_idx, unsigned grid,
                               cudaStream_t s, const float* coef = nullptr) {
  if constexpr (sizeof(T) == 8) {
    return false;
  } else {
  switch (vec_lanes<T>(b)) {
#define FMS_SV(NV)                                                                                   \
  case NV:                                                                                           \
    if (coef != nullptr)                                                                             \
      csr_scatter_vec_kernel<T, NV, true, true><<<grid, SC_WARPS * 32, 0, s>>>(b, row_ptr, col_idx, \
                                                                               coef);               \
    else if (b.g.layout == L_INBATCH)                                                                \
      csr_scatter_vec_kernel<T, NV, true><<<grid, SC_WARPS * 32, 0, s>>>(b, row_ptr, col_idx);      \
    else                                                                                             \
      csr_scatter_vec_kernel<T, NV, false><<<grid, SC_WARPS * 32, 0, s>>>(b, row_ptr, col_idx);     \
    return true;
    FMS_SV(1) FMS_SV(2) FMS_SV(3) FMS_SV(4) FMS_SV(5)
#undef FMS_SV
    default: return false;
  }
  }
}

static inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

size_t bwd_workspace_bytes(int strategy, int dtype, int64_t n_src, int64_t n_dest,
                           int64_t grad_d_numel) {
  if (strategy == FMS_ATOMIC_UNIFIED) {
    if (dtype == FMS_F16 || dtype == FMS_BF16) return align_up((size_t)grad_d_numel * 4, 256);
    return 0;
  }
  // row_ptr (+ the long-segment count), cursor, col_idx, scan partials, the
  // list of long segments and the segment sort's ping-pong buffer
  size_t nscan = (size_t)n_dest + 1;
  size_t nb = (nscan + SCAN_BLOCK - 1) / SCAN_BLOCK;
  size_t nlong = (size_t)n_src / (SC_SEG + 1) + 1;
  return align_up(nscan * 4 + 4, 256) + align_up((size_t)n_dest * 4 + 4, 256) +
         align_up((size_t)n_src * 4 + 4, 256) + align_up(nb * 4 + 4, 256) +
         align_up(nlong * 4, 256) + align_up((size_t)n_src * 4 + 4, 256);
}

template <typename T>
static cudaError_t run_backward(int strategy, const BwdParams& b, void* ws, size_t ws_bytes,
                                cudaStream_t s) {
  using A = typename Tr<T>::Acc;
  const ScanParams& p = b.g;
  const int sms = device_sm_count();
  const int64_t dim = p.dim;
  cudaError_t e;
  auto grid_for = [&](int64_t work, int per_block) -> unsigned {
    int64_t g = (work + per_block - 1) / per_block;
    int64_t cap = (int64_t)sms * 32;
    if (g > cap) g = cap;
    return (unsigned)(g < 1 ? 1 : g);
  };
  if (strategy == FMS_ATOMIC_UNIFIED) {
    A* acc = nullptr;
    const bool wide = sizeof(T) == sizeof(A);
    if (wide) {
      acc = reinterpret_cast<A*>(b.dD);
    } else {
      if (ws == nullptr || ws_bytes < (size_t)b.nd_rows * dim * sizeof(A)) return cudaErrorInvalidValue;
      acc = reinterpret_cast<A*>(ws);
    }
    e = cudaMemsetAsync(acc, 0, (size_t)b.nd_rows * dim * sizeof(A), s);
    if (e != cudaSuccess) return e;
    if (!launch_gather_vec<T, true>(b, reinterpret_cast<float*>(acc), grid_for(b.nq_rows, 8), s))
      bwd_gather_kernel<T, true><<<grid_for(b.nq_rows, 8), 256, 0, s>>>(b, acc);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if (!wide) {
      int64_t n = b.nd_rows * dim;
      convert_kernel<A, T><<<grid_for(n, 256), 256, 0, s>>>(acc, static_cast<T*>(b.dD), n);
      if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    return cudaSuccess;
  }
  // InvGrid
  const int64_t n_src = p.nunits * (int64_t)p.Tq;
  const int64_t n_dest = b.nd_rows;
  const size_t need = bwd_workspace_bytes(strategy, 0, n_src, n_dest, 0);
  if (ws == nullptr || ws_bytes < need) return cudaErrorInvalidValue;
  const int64_t nscan = n_dest + 1;
  const int64_t nb = (nscan + SCAN_BLOCK - 1) / SCAN_BLOCK;
  const size_t nlong = (size_t)n_src / (SC_SEG + 1) + 1;
  char* w = static_cast<char*>(ws);
  int32_t* row_ptr = reinterpret_cast<int32_t*>(w);
  int32_t* long_cnt = row_ptr + nscan;  // cleared with row_ptr
  w += align_up((size_t)nscan * 4 + 4, 256);
  int32_t* cursor = reinterpret_cast<int32_t*>(w);
  w += align_up((size_t)n_dest * 4 + 4, 256);
  int32_t* col_idx = reinterpret_cast<int32_t*>(w);
  w += align_up((size_t)n_src * 4 + 4, 256);
  int32_t* sums = reinterpret_cast<int32_t*>(w);
  w += align_up((size_t)nb * 4 + 4, 256);
  int32_t* long_list = reinterpret_cast<int32_t*>(w);
  w += align_up(nlong * 4, 256);
  int32_t* sort_tmp = reinterpret_cast<int32_t*>(w);

  // dQ gather (no atomics)
  if (!launch_gather_vec<T, false>(b, nullptr, grid_for(b.nq_rows, 8), s))
    bwd_gather_kernel<T, false><<<grid_for(b.nq_rows, 8), 256, 0, s>>>(b, nullptr);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  // in-batch with the vector scatter: per-document stable counting sort
  // (document totals -> their exclusive scan -> one block per document), the
  // sources stored as (query row, delta) in col_idx and sort_tmp
  if (p.layout == L_INBATCH && vec_lanes<T>(b) > 0 && p.Bd >= 1 && p.Td >= 1 && p.Td <= IB_TD_MAX &&
      p.Bq <= IB_BQ_MAX && (int64_t)p.Bq * p.Tq <= IB_E_MAX && n_dest > 0) {
    int32_t* doc_base = cursor;  // Bd <= n_dest entries
    float* coef = reinterpret_cast<float*>(sort_tmp);
    inb_csr_total_kernel<<<(unsigned)p.Bd, IB_THREADS, 0, s>>>(p, doc_base);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    scan_sums_kernel<<<1, SCAN_BLOCK, 0, s>>>(doc_base, p.Bd);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const size_t smem = inb_csr_smem(p.Td, p.Bq, p.Tq);
    if (smem > 48 * 1024 &&
        (e = cudaFuncSetAttribute(inb_csr_build_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem)) != cudaSuccess)
      return e;
    inb_csr_build_kernel<T><<<(unsigned)p.Bd, IB_THREADS, smem, s>>>(b, doc_base, row_ptr, col_idx, coef);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    launch_scatter_vec<T>(b, row_ptr, col_idx, grid_for(n_dest, SC_WARPS), s, coef);
    return cudaGetLastError();
  }
  // counting sort: counts land at row_ptr[dest], exclusive scan turns them into
  // segment starts, row_ptr[n_dest] = nnz.
  if ((e = cudaMemsetAsync(row_ptr, 0, (size_t)nscan * 4 + 4, s)) != cudaSuccess) return e;
  if (n_src > 0) {
    csr_count_kernel<<<grid_for(n_src, 256), 256, 0, s>>>(p, n_src, row_ptr);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  scan_blocks_kernel<<<(unsigned)nb, SCAN_BLOCK, 0, s>>>(row_ptr, nscan, sums, long_cnt, long_list);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  scan_sums_kernel<<<1, SCAN_BLOCK, 0, s>>>(sums, nb);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  scan_add_kernel<<<grid_for(nscan, 256), 256, 0, s>>>(row_ptr, nscan, sums, cursor, n_dest);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if (n_src > 0) {
    csr_fill_kernel<<<grid_for(n_src, 256), 256, 0, s>>>(p, n_src, cursor, col_idx);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // segments over SC_SEG sources: ascending order before the scatter (a
    // no-op launch when there are none)
    if (n_src > SC_SEG) {
      csr_sort_long_kernel<<<(unsigned)sms, SORT_THREADS, 0, s>>>(row_ptr, col_idx, sort_tmp, long_cnt,
                                                                  long_list);
      if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
  }
  if (n_dest > 0) {
    if (!launch_scatter_vec<T>(b, row_ptr, col_idx, grid_for(n_dest, SC_WARPS), s))
      csr_scatter_kernel<T><<<grid_for(n_dest, SC_WARPS), SC_WARPS * 32, 0, s>>>(b, row_ptr, col_idx);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_backward(int dtype, int strategy, const BwdParams& b, void* ws, size_t ws_bytes,
                            cudaStream_t s) {
  // zero-size outputs: nothing to do
  if (b.g.dim == 0) return cudaSuccess;
  switch (dtype) {
    case FMS_F32: return run_backward<float>(strategy, b, ws, ws_bytes, s);
    case FMS_F16: return run_backward<__half>(strategy, b, ws, ws_bytes, s);
    case FMS_BF16: return run_backward<__nv_bfloat16>(strategy, b, ws, ws_bytes, s);
    case FMS_F64: return run_backward<double>(strategy, b, ws, ws_bytes, s);
    default: return cudaErrorInvalidValue;
  }
}

// ------------------------------------------------------------------ inv counts

template <typename T>
__global__ void inv_counts_kernel(const uint8_t* __restrict__ qmask, int Tq, int B, T* inv_n) {
  using A = typename Tr<T>::Acc;
  int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  int n = 0;
  for (int t = 0; t < Tq; ++t) n += (qmask == nullptr || qmask[(int64_t)b * Tq + t]) ? 1 : 0;
  A c = (A)(n > 1 ? n : 1);
  inv_n[b] = Tr<T>::from((A)1 / c);
}

cudaError_t launch_inv_counts(int dtype, const uint8_t* qmask, int Tq, int B, void* inv_n,
                              cudaStream_t s) {
  if (B == 0) return cudaSuccess;
  unsigned g = (unsigned)((B + 127) / 128);
  switch (dtype) {
    case FMS_F32: inv_counts_kernel<float><<<g, 128, 0, s>>>(qmask, Tq, B, (float*)inv_n); break;
    case FMS_F16: inv_counts_kernel<__half><<<g, 128, 0, s>>>(qmask, Tq, B, (__half*)inv_n); break;
    case FMS_BF16:
      inv_counts_kernel<__nv_bfloat16><<<g, 128, 0, s>>>(qmask, Tq, B, (__nv_bfloat16*)inv_n);
      break;
    case FMS_F64: inv_counts_kernel<double><<<g, 128, 0, s>>>(qmask, Tq, B, (double*)inv_n); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace fms
