// fms_scan_gallery.cu -- the sm_100a MaxSim engine for short queries (Tq <= 32)
// against galleries of documents: the candidate layout (candidates_forward,
// forward_layouts.jl:229-290, normalize.jl:37-46) and the paired layout
// (forward_layouts.jl:78-124) for Float16 / BFloat16 features, dim 64..256.
// It replaces the reference's WMMA candidate / paired kernels
// (ext/FlashMaxSimCUDAExt.jl:298-359, 488-553) for these shapes.
//
// Orientation: DOCUMENT tokens on the MMA M side (128-row tiles), the query on
// N (32 rows, one resident tile).  A unit (one query x one document) is cut
// into chunks of up to slot_rows document rows; each chunk is one shared-memory
// slot of the TMA ring and one small TMEM accumulator (32 columns per 128-row
// tile), so a CTA's 256 TMEM columns hold up to eight 128-row chunks: the MMA
// runs as far ahead of the epilogue as the ring allows, and a slot is released
// as soon as its MMAs complete.  There is no query replication, so the tensor
// work is the useful work.
//
// Epilogue: one tcgen05.ld.32x32b.x32 gives a thread (one document token) its
// 32 similarities (one per query token); a five-round shuffle reduce-scatter
// over the warp leaves lane t with the masked max (and argmax) over the warp's
// 32 document tokens for query token t; the four warps of a group merge through
// shared memory, apply the first-valid-column rule (forward_pair.jl:83: a NaN
// in the first valid column sticks), and lane 0 writes Sigma_t (and the
// normalisation); the tape is one coalesced 32-lane store.
//
// Two CTAs per SM, each an independent pipeline (352 threads, persistent over a
// contiguous range of units or of unit-list entries); every ring between roles
// has one producer and one consumer, so parity waits never alias:
//   warp 0   TMA producer (one lane): the unit's query tile into a resident
//            slot when the query changes, document rows (stopping at the last
//            valid token) into the slot ring;
//   warp 1   MMA issuer (one lane): per chunk, per 128-row tile, dim/16 MMAs
//            of M = 128, N = 32, K = 16 into the chunk's accumulator;
//   warp 2   scheduler: decodes 32 units at a time into a shared-memory
//            metadata ring (first / last valid document token, mask words);
//            units with nothing to scan are written directly;
//   warps 3-10  epilogue, two groups of four (alternate units; a group has one
//            warp per TMEM subpartition).
// One issuing thread needs ~90 cycles per MMA (waits, descriptors) against the
// tensor pipe's ~55 at this shape, and ~1.4k cycles to hand a document's boxes
// to the TMA unit: two pipelines per SM overlap each other's issue.  Role
// waits spin (a sleeping mbarrier wait costs ~1k cycles per wake-up, measured).
// Every wait is bounded: on a timeout the CTA raises an error flag, stops,
// lets in-flight copies land, frees TMEM and returns.
#include <cuda.h>

#include "fms_common.cuh"
#include "fms_int8.cuh"
#include "fms_internal.h"
#include "fms_tc_ptx.cuh"

namespace fms {

__device__ int g_gal_error = 0;  // set when a wait of this engine timed out

namespace gal {

constexpr int KBLK = 64;     // K elements per block: one 128-byte swizzled row
constexpr int ROWB = 128;    // bytes per tile row per K block
constexpr int NQ = 32;       // MMA N: query rows
constexpr int QTILE = NQ * ROWB;  // one K block of the query tile
constexpr int PROD_WARP = 0, MMA_WARP = 1, SCHED_WARP = 2, EPI_WARP0 = 3;
constexpr int NGROUP = 2;    // epilogue groups (alternate units)
constexpr int NEPI = 4 * NGROUP;  // epilogue warps (a group: one per TMEM subpartition)
constexpr int NWARPS = EPI_WARP0 + NEPI;
constexpr int NTHREADS = NWARPS * 32;
// Per element kind: 16-bit features run two independent pipelines (CTAs) per
// SM; INT8 codes one (the dequantisation keeps 32 query scales in registers).
template <bool I8> struct Kind {
  static constexpr int CTAS_PER_SM = I8 ? 1 : 2;
  static constexpr int TMEM_COLS = 512 / CTAS_PER_SM;
  static constexpr int SMEM_BUDGET = I8 ? 212 * 1024 : 106 * 1024;  // dynamic, per CTA
};
constexpr int UQ = 16;       // metadata ring depth
constexpr int MW_MAX = 16;   // document mask words held per unit (32 * 16 = 512 tokens)
constexpr int SMAX = 4;      // document slots at most
constexpr int NACC_MAX = 512 / 32;  // accumulators at most

struct Params {
  ScanParams p;
  const void* qs;  // INT8: query token scales (Tq per query), f32 or f16
  const void* ds;  // INT8: document token scales (one per document row)
  int qs_f16, ds_f16;
  int KB;          // 128-byte K blocks per row (dim / 64 for 16-bit, dim / 128 for INT8)
  uint32_t fmt;    // 16-bit kinds: 0 = f16, 1 = bf16
  int slot_rows;   // document rows per chunk (256 or 128)
  int sr_log2;     // log2(slot_rows)
  int nslots;      // shared-memory slots
  int acc_cols;    // TMEM columns per chunk (slot_rows / 128 * 32)
  int nacc;        // accumulators (TMEM columns / acc_cols)
  int qslots;      // resident query tiles (1 or 2)
};

struct Meta {
  int64_t q_row0, d_row0, out0, arg0;
  const uint8_t* dmask;  // consulted for tokens past 32 * MW_MAX
  int Tq, leff, first, arg_rows, mw_ok, anew, valid;
  uint32_t qw;           // bit t: query token t valid
  uint32_t mw[MW_MAX];   // bit u: document token u valid
};

// Nonzero bytes of a 32-bit word -> 4 bits.
__device__ __forceinline__ uint32_t nz4(uint32_t w) {
  const uint32_t r = __vcmpne4(w, 0u);
  return (r & 1u) | ((r >> 7) & 2u) | ((r >> 14) & 4u) | ((r >> 21) & 8u);
}

// Bits of n mask bytes (0/1) starting at m (NULL = all valid) into W words.
template <int W>
__device__ __forceinline__ void mask_words(const uint8_t* m, int n, uint32_t (&w)[W]) {
#pragma unroll
  for (int i = 0; i < W; ++i) {
    const int lo = 32 * i;
    w[i] = m ? 0u : (n >= lo + 32 ? 0xffffffffu : (n > lo ? ((1u << (n - lo)) - 1u) : 0u));
  }
  if (m == nullptr) return;
  if ((reinterpret_cast<uintptr_t>(m) & 15) == 0) {
#pragma unroll
    for (int i = 0; i < 2 * W; ++i) {
      const int base = 16 * i;
      if (base < n) {
        uint32_t bits;
        if (base + 16 <= n) {
          const uint4 x = __ldg(reinterpret_cast<const uint4*>(m + base));
          bits = nz4(x.x) | (nz4(x.y) << 4) | (nz4(x.z) << 8) | (nz4(x.w) << 12);
        } else {
          bits = 0u;
          for (int b = 0; base + b < n; ++b) bits |= (m[base + b] != 0 ? 1u : 0u) << b;
        }
        w[i >> 1] |= bits << (16 * (i & 1));
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < W; ++i)
      for (int b = 0; b < 32 && 32 * i + b < n; ++b) w[i] |= (m[32 * i + b] != 0 ? 1u : 0u) << b;
  }
}

// Document rows [row, row + nr) of one K block (nr a multiple of 16).
__device__ __forceinline__ void load_rows(unsigned char* dst, const CUtensorMap* b128, const CUtensorMap* b64,
                                          const CUtensorMap* b32, const CUtensorMap* b16, int x, int64_t row,
                                          int nr, uint64_t* bar) {
  int r = 0;
  for (; nr - r >= 128; r += 128) ptx::tma_load_2d(dst + r * ROWB, b128, x, (int)(row + r), bar);
  if (nr - r >= 64) { ptx::tma_load_2d(dst + r * ROWB, b64, x, (int)(row + r), bar); r += 64; }
  if (nr - r >= 32) { ptx::tma_load_2d(dst + r * ROWB, b32, x, (int)(row + r), bar); r += 32; }
  if (nr - r >= 16) { ptx::tma_load_2d(dst + r * ROWB, b16, x, (int)(row + r), bar); r += 16; }
}

struct Maps {
  CUtensorMap q, b128, b64, b32, b16;
};

// Warp-wide bounded wait in which every lane polls the barrier itself (no
// broadcast from one lane: a completed phase costs one poll per lane); the
// verdict is warp-uniform and the warp re-converges.
__device__ __forceinline__ bool lane_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const bool ok = ptx::mbar_wait(bar, parity, abort);
  return __all_sync(0xffffffffu, ok);
}

// Reduce-scatter of 32 per-lane values over the warp: lane t ends with the max
// over the 32 lanes of value t.  Five rounds; in each, a lane keeps the half of
// its values whose index bit matches its own lane bit and takes the max with the
// partner's copy of that half.
__device__ __forceinline__ float rs_max(float (&v)[32], int lane) {
#pragma unroll
  for (int o = 16, n = 32; o > 0; o >>= 1, n >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = up ? v[i] : v[i + n / 2];
      const float keep = up ? v[i + n / 2] : v[i];
      v[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, o));
    }
  }
  return v[0];
}

// The same with (value, 1-based index) pairs merged by merge_state (larger value,
// then smaller index; index 0 = empty).
__device__ __forceinline__ void rs_argmax(float (&v)[32], int (&a)[32], int lane, float& mo, int& ao) {
#pragma unroll
  for (int o = 16, n = 32; o > 0; o >>= 1, n >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float sv = up ? v[i] : v[i + n / 2];
      const int sa = up ? a[i] : a[i + n / 2];
      float kv = up ? v[i + n / 2] : v[i];
      int ka = up ? a[i + n / 2] : a[i];
      const float rv = __shfl_xor_sync(0xffffffffu, sv, o);
      const int ra = __shfl_xor_sync(0xffffffffu, sa, o);
      merge_state(kv, ka, rv, ra);
      v[i] = kv;
      a[i] = ka;
    }
  }
  mo = v[0];
  ao = a[0];
}

__device__ __forceinline__ float ld_scale(const void* p, int f16, int64_t i) {
  return f16 ? __half2float(__ldg(static_cast<const __half*>(p) + i))
             : __ldg(static_cast<const float*>(p) + i);
}

template <bool ARGS, bool I8>
__global__ void __launch_bounds__(NTHREADS, Kind<I8>::CTAS_PER_SM)
gallery_kernel(const __grid_constant__ Maps maps, Params P) {
  extern __shared__ __align__(1024) unsigned char dsm[];
  __shared__ __align__(8) uint64_t full_bar[SMAX];
  __shared__ __align__(8) uint64_t empty_bar[SMAX];
  __shared__ __align__(8) uint64_t afull_bar[2];
  __shared__ __align__(8) uint64_t aempty_bar[2];
  __shared__ __align__(8) uint64_t accf_bar[NACC_MAX];
  __shared__ __align__(8) uint64_t acce_bar[NACC_MAX];
  __shared__ __align__(8) uint64_t metaf_bar[UQ];
  __shared__ __align__(8) uint64_t metae_bar[UQ];
  __shared__ __align__(8) uint64_t grp_bar[NGROUP];  // the four warps of a group
  __shared__ Meta meta[UQ];
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile int abort_s;
  // per group, double-buffered by the group's unit parity
  __shared__ float red_mx[NGROUP][2][3][32];
  __shared__ int red_ag[NGROUP][2][3][32];
  __shared__ float s0_s[NGROUP][2][32];  // similarities of the first valid document token

  unsigned char* tiles = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(dsm) + 1023) & ~(uintptr_t)1023);
  const int qslot_bytes = P.KB * QTILE;
  const int slot_bytes = P.KB * P.slot_rows * ROWB;
  unsigned char* qslots = tiles;
  unsigned char* ring = tiles + P.qslots * qslot_bytes;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const ScanParams& p = P.p;

  if (threadIdx.x == 0) {
    for (int i = 0; i < SMAX; ++i) {
      ptx::mbar_init(&full_bar[i], 1);
      ptx::mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&afull_bar[i], 1);
      ptx::mbar_init(&aempty_bar[i], 1);
    }
    for (int g = 0; g < NGROUP; ++g) ptx::mbar_init(&grp_bar[g], 4);
    for (int i = 0; i < NACC_MAX; ++i) {
      ptx::mbar_init(&accf_bar[i], 1);
      ptx::mbar_init(&acce_bar[i], 4);  // the four warps of the group that drains it
    }
    for (int i = 0; i < UQ; ++i) {
      ptx::mbar_init(&metaf_bar[i], 1);
      ptx::mbar_init(&metae_bar[i], 2 + NEPI);  // producer lane, MMA lane, epilogue warps
    }
    abort_s = 0;
    ptx::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&maps.q);
    ptx::prefetch_tmap(&maps.b128);
    ptx::prefetch_tmap(&maps.b64);
    ptx::prefetch_tmap(&maps.b32);
    ptx::prefetch_tmap(&maps.b16);
  }
  constexpr int TMEM_COLS = Kind<I8>::TMEM_COLS;
  constexpr int KBLK_E = I8 ? 128 : KBLK;  // elements per 128-byte K block
  if (warp == MMA_WARP) ptx::tmem_alloc(&tmem_base_s, TMEM_COLS);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;
  const int64_t nwalk = units_to_scan(p);
  const int64_t u_begin = nwalk * blockIdx.x / gridDim.x;
  const int64_t my_units = nwalk * (blockIdx.x + 1) / gridDim.x - u_begin;
  const int SR = P.slot_rows;

  if (warp == SCHED_WARP) {
    // ------------------------------------------------------------ scheduler
    int have_prev = 0;
    int64_t prev_q = -1;
    int64_t qn = 0;  // units queued so far (warp-uniform)
    float* scores_out = static_cast<float*>(p.scores);
    for (int64_t i0 = 0; i0 < my_units; i0 += 32) {
      if (__any_sync(0xffffffffu, abort_s != 0)) break;
      const int64_t i = i0 + lane;
      Meta m;
      int working = 0, direct = 0;
      if (i < my_units) {
        const Unit U = decode_unit(p, unit_at(p, u_begin + i));
        m.q_row0 = U.q0; m.d_row0 = U.d0; m.out0 = U.out; m.arg0 = U.arg0;
        m.dmask = U.dmask; m.Tq = U.Tq; m.arg_rows = U.arg_rows; m.valid = U.valid ? 1 : 0;
        uint32_t qw1[1];
        mask_words<1>(U.qmask, U.Tq, qw1);
        m.qw = qw1[0];
        m.mw_ok = U.Td <= 32 * MW_MAX;
        int first = -1, last = -1;
        if (U.valid) {
          mask_words<MW_MAX>(U.dmask, U.Td < 32 * MW_MAX ? U.Td : 32 * MW_MAX, m.mw);
#pragma unroll
          for (int w = MW_MAX - 1; w >= 0; --w)
            if (m.mw[w]) first = 32 * w + __ffs(m.mw[w]) - 1;
#pragma unroll
          for (int w = 0; w < MW_MAX; ++w)
            if (m.mw[w]) last = 32 * w + 31 - __clz(m.mw[w]);
          for (int u = 32 * MW_MAX; u < U.Td; ++u)  // long documents: the mask tail
            if (U.dmask == nullptr || U.dmask[u]) {
              if (first < 0) first = u;
              last = u;
              if (U.dmask == nullptr) { last = U.Td - 1; break; }
            }
        } else {
#pragma unroll
          for (int w = 0; w < MW_MAX; ++w) m.mw[w] = 0u;
        }
        m.first = first;
        m.leff = last + 1;
        working = (m.valid && U.Tq > 0 && m.leff > 0) ? 1 : 0;
        if (!working) {
          // nothing to scan (a slot outside 1:N or this shard, an empty or fully
          // masked document, an empty query): written here, never queued
          scores_out[U.out] = U.valid ? 0.f : (float)p.neg;
          if (ARGS)
            for (int t = 0; t < U.arg_rows; ++t) p.args[U.arg0 + t] = 0;
          direct = 1;
        }
      }
      // a new query tile is needed when a working unit's query differs from the
      // previous working unit's (in queue order)
      int anew = 0;
      for (int k = 0; k < 32; ++k) {
        const int wk = __shfl_sync(0xffffffffu, working, k);
        const long long qk = __shfl_sync(0xffffffffu, (long long)(working ? m.q_row0 : 0), k);
        if (wk) {
          if (lane == k) anew = (!have_prev || qk != prev_q) ? 1 : 0;
          have_prev = 1;
          prev_q = qk;
        }
      }
      m.anew = anew;
      uint32_t enq = __ballot_sync(0xffffffffu, i < my_units && !direct);
      while (enq) {
        const int k = __ffs(enq) - 1;
        enq &= enq - 1;
        if (lane == k) {
          const int slot = (int)(qn % UQ);
          const uint32_t par = (uint32_t)((qn / UQ) & 1);
          if (ptx::mbar_wait(&metae_bar[slot], par ^ 1, &abort_s)) {
            meta[slot] = m;
            ptx::mbar_arrive(&metaf_bar[slot]);
          }
        }
        ++qn;
        __syncwarp();
        if (__any_sync(0xffffffffu, abort_s != 0)) break;
      }
    }
    if (lane == 0 && !abort_s) {  // end marker
      const int slot = (int)(qn % UQ);
      if (ptx::mbar_wait(&metae_bar[slot], (uint32_t)(((qn / UQ) & 1) ^ 1), &abort_s)) {
        meta[slot].valid = -1;
        ptx::mbar_arrive(&metaf_bar[slot]);
      }
    }
    __syncwarp();
  } else if (warp == PROD_WARP) {
    // ------------------------------------------------------------ TMA producer
    // Lane 0 alone: the unit's query tile into a resident slot when the query
    // changes, then the document rows of every chunk into the slot ring.
    if (lane == 0) {
      int slot = 0;
      uint32_t sphase = 0;
      int qs = P.qslots - 1;
      uint32_t qphase = 1;
      for (int64_t i = 0;; ++i) {
        const int ms = (int)(i % UQ);
        if (!ptx::mbar_wait(&metaf_bar[ms], (uint32_t)((i / UQ) & 1), &abort_s)) goto prod_out;
        const Meta& m = meta[ms];
        if (m.valid < 0) break;
        const int64_t q_row0 = m.q_row0, d_row0 = m.d_row0;
        const int leff = m.leff, anew = m.anew;
        ptx::mbar_arrive(&metae_bar[ms]);
        if (anew) {
          if (++qs == P.qslots) { qs = 0; qphase ^= 1; }
          if (!ptx::mbar_wait(&aempty_bar[qs], qphase ^ 1, &abort_s)) goto prod_out;
          ptx::mbar_expect_tx(&afull_bar[qs], (uint32_t)qslot_bytes);
          for (int kb = 0; kb < P.KB; ++kb)
            ptx::tma_load_2d(qslots + qs * qslot_bytes + kb * QTILE, &maps.q, kb * KBLK_E, (int)q_row0,
                             &afull_bar[qs]);
        }
        const int nch = (leff + SR - 1) >> P.sr_log2;
        for (int c = 0; c < nch; ++c) {
          const int n = min(SR, leff - c * SR);
          const int nr = (n + 15) & ~15;
          if (!ptx::mbar_wait(&empty_bar[slot], sphase ^ 1u, &abort_s)) goto prod_out;
          unsigned char* st = ring + slot * slot_bytes;
          ptx::mbar_expect_tx(&full_bar[slot], (uint32_t)(P.KB * nr * ROWB));
          for (int kb = 0; kb < P.KB; ++kb)
            load_rows(st + kb * SR * ROWB, &maps.b128, &maps.b64, &maps.b32, &maps.b16, kb * KBLK_E,
                      d_row0 + (int64_t)c * SR, nr, &full_bar[slot]);
          if (++slot == P.nslots) { slot = 0; sphase ^= 1u; }
        }
      }
    }
  prod_out:
    __syncwarp();
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int qs = P.qslots - 1;
      uint32_t qphase = 1;
      bool holding = false;
      int slot = 0, acc = 0;           // slot and accumulator of the next chunk
      uint32_t sphase = 0, aphase = 0; // parities of their uses
      const uint32_t idesc = I8 ? ptx::idesc_i8(128, NQ) : ptx::idesc_f16(P.fmt, 128, NQ);
      for (int64_t i = 0;; ++i) {
        const int ms = (int)(i % UQ);
        if (!ptx::mbar_wait(&metaf_bar[ms], (uint32_t)((i / UQ) & 1), &abort_s)) goto mma_out;
        const Meta& m = meta[ms];
        if (m.valid < 0) break;
        const int leff = m.leff, anew = m.anew;
        ptx::mbar_arrive(&metae_bar[ms]);
        if (anew) {
          if (holding) ptx::mma_commit(&aempty_bar[qs]);  // after the previous query's last MMA
          if (++qs == P.qslots) { qs = 0; qphase ^= 1; }
          if (!ptx::mbar_wait(&afull_bar[qs], qphase, &abort_s)) goto mma_out;
          ptx::tc_fence_after();
          holding = true;
        }
        const uint32_t qbase = ptx::smem_u32(qslots + qs * qslot_bytes);
        const int nch = (leff + SR - 1) >> P.sr_log2;
        for (int c = 0; c < nch; ++c) {
          const int n = min(SR, leff - c * SR);
          const int ntile = (n + 127) >> 7;
          const uint32_t a = (uint32_t)acc;
          if (!ptx::mbar_wait(&acce_bar[a], aphase ^ 1u, &abort_s)) goto mma_out;
          ptx::tc_fence_after();
          if (!ptx::mbar_wait(&full_bar[slot], sphase, &abort_s)) goto mma_out;
          ptx::tc_fence_after();
          const uint32_t sbase = ptx::smem_u32(ring + slot * slot_bytes);
          for (int t = 0; t < ntile; ++t) {
            const uint32_t d = tmem_base + a * (uint32_t)P.acc_cols + (uint32_t)(t * NQ);
            for (int kb = 0; kb < P.KB; ++kb) {
              const uint64_t adesc = ptx::sw128_desc(sbase + (uint32_t)(kb * SR * ROWB + t * 128 * ROWB));
              const uint64_t bdesc = ptx::sw128_desc(qbase + (uint32_t)(kb * QTILE));
              // four 32-byte K steps per block (K = 16 f16 / bf16, K = 32 int8)
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                if (I8) ptx::mma_i8(d, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0);
                else ptx::mma_f16(d, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0);
              }
            }
          }
          ptx::mma_commit(&empty_bar[slot]);
          ptx::mma_commit(&accf_bar[a]);
          if (++slot == P.nslots) { slot = 0; sphase ^= 1u; }
          if (++acc == P.nacc) { acc = 0; aphase ^= 1u; }
        }
      }
    }
  mma_out:
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int g = (warp - EPI_WARP0) >> 2;  // group: takes the units of its parity
    const int sp = warp & 3;                // TMEM subpartition (lanes 32 sp .. 32 sp + 31)
    int acc = 0;             // accumulator of the next chunk (all groups)
    uint32_t aphase = 0;     // parity of its use
    uint32_t gphase = 0;
    int par = 0;
    float* scores = static_cast<float*>(p.scores);
    for (int64_t i = 0;; ++i) {
      const int ms = (int)(i % UQ);
      if (!lane_wait(&metaf_bar[ms], (uint32_t)((i / UQ) & 1), &abort_s)) goto done;
      const Meta& m = meta[ms];
      if (m.valid < 0) break;
      const int leff = m.leff;
      const int nch = (leff + SR - 1) >> P.sr_log2;
      if ((int)(i % NGROUP) != g) {
        for (int c = 0; c < nch; ++c)
          if (++acc == P.nacc) { acc = 0; aphase ^= 1u; }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&metae_bar[ms]);
        continue;
      }
      const int first = m.first;
      float mx = -INFINITY;
      int ag = 0;
      // INT8: the unit's 32 query-token scales, one per lane, then in every lane
      float qsr[I8 ? 32 : 1];
      if (I8) {
        const float q_own = lane < m.Tq ? ld_scale(P.qs, P.qs_f16, m.q_row0 + lane) : 0.f;
#pragma unroll
        for (int j = 0; j < (I8 ? 32 : 1); ++j) qsr[j] = __shfl_sync(0xffffffffu, q_own, j);
      }
      for (int c = 0; c < nch; ++c) {
        const int n = min(SR, leff - c * SR);
        const int ntile = (n + 127) >> 7;
        const uint32_t a = (uint32_t)acc;
        const uint32_t ap = aphase;
        if (++acc == P.nacc) { acc = 0; aphase ^= 1u; }
        if (!lane_wait(&accf_bar[a], ap, &abort_s)) goto done;
        ptx::tc_fence_after();
        for (int t = 0; t < ntile; ++t) {
          const int u = c * SR + t * 128 + sp * 32 + lane;  // this lane's document token
          bool ok = u < leff;
          if (ok) {
            if (m.mw_ok || u < 32 * MW_MAX) ok = (m.mw[u >> 5] >> (u & 31)) & 1u;
            else ok = m.dmask == nullptr || m.dmask[u] != 0;
          }
          // no early exit for 32 rows without a valid token: they are rare, and
          // on this part a branch costs about as much as the selects below
          const bool has_first = __any_sync(0xffffffffu, u == first);
          uint32_t r[32];
          ptx::tmem_ld32(tmem_base + ((uint32_t)(sp * 32) << 16) + a * (uint32_t)P.acc_cols +
                             (uint32_t)(t * NQ),
                         r);
          ptx::tmem_wait_ld();
          if (I8) {
            // s = (qs_t * ds_u) * float(acc): acc is the exact int32 dot product
            // (quant.jl:113), exactly representable (|acc| < 2^24 for dim <= 1024)
            const float dsu = (u < leff) ? ld_scale(P.ds, P.ds_f16, m.d_row0 + u) : 0.f;
#pragma unroll
            for (int j = 0; j < (I8 ? 32 : 1); ++j)
              r[j] = __float_as_uint((qsr[j] * dsu) * __int2float_rn((int)r[j]));
          }
          if (has_first && u == first) {
#pragma unroll
            for (int j = 0; j < 32; ++j) s0_s[g][par][j] = __uint_as_float(r[j]);
          }
          float v[32];
          if (ARGS) {
            int ai[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float s = __uint_as_float(r[j]);
              const bool take = ok && s > -INFINITY;  // strict > from -Inf: no NaN, no -Inf
              v[j] = take ? s : -INFINITY;
              ai[j] = take ? u + 1 : 0;
            }
            float tm;
            int ta;
            rs_argmax(v, ai, lane, tm, ta);
            merge_state(mx, ag, tm, ta);
          } else {
            const bool all = __all_sync(0xffffffffu, ok);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = (all || ok) ? __uint_as_float(r[j]) : -INFINITY;
            mx = fmaxf(mx, rs_max(v, lane));
          }
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&acce_bar[a]);
      }
      // the group's four partial states per query token meet in warp sp == 0
      if (sp != 0) {
        red_mx[g][par][sp - 1][lane] = mx;
        red_ag[g][par][sp - 1][lane] = ag;
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&grp_bar[g]);
      if (!lane_wait(&grp_bar[g], gphase, &abort_s)) goto done;
      gphase ^= 1;
      if (sp == 0) {
#pragma unroll
        for (int q = 0; q < 3; ++q) {
          if (ARGS) merge_state(mx, ag, red_mx[g][par][q][lane], red_ag[g][par][q][lane]);
          else mx = fmaxf(mx, red_mx[g][par][q][lane]);
        }
        const float s0 = s0_s[g][par][lane];
        const int t = lane;
        const bool tv = t < m.Tq && ((m.qw >> t) & 1u);
        float val = mx;
        bool okr;
        if (ARGS) {
          int aa = ag;
          final_fixup(val, aa, first, s0);
          okr = tv && aa > 0;
          if (t < m.arg_rows) p.args[m.arg0 + t] = okr ? aa : 0;
        } else {
          // a NaN in the first valid column sticks; otherwise the max of the
          // non-NaN values (>= that column's value) is the result
          if (s0 != s0) val = s0;
          okr = tv;
        }
        const float rowv = okr ? val : 0.f;
        float sum = 0.f;
        if (I8) {
          // Sigma_t in t order (quant.jl:121-123), so INT8 scores are the
          // reference's bit for bit
          for (int tt = 0; tt < m.Tq; ++tt) sum += __shfl_sync(0xffffffffu, rowv, tt);
        } else {
          sum = rowv;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        }
        if (lane == 0) {
          if (p.normalize) {
            const int nvalid = __popc(m.qw & (m.Tq >= 32 ? 0xffffffffu : ((1u << m.Tq) - 1u)));
            sum = sum * (1.0f / (float)(nvalid > 1 ? nvalid : 1));
          }
          scores[m.out0] = sum;
        }
        if (ARGS)
          for (int tt = 32 + lane; tt < m.arg_rows; tt += 32) p.args[m.arg0 + tt] = 0;
      }
      par ^= 1;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&metae_bar[ms]);
    }
  }
done:
  if (abort_s && threadIdx.x == 0) {
    atomicExch(&g_gal_error, 1);
    const uint64_t t0 = ptx::globaltimer_ns();
    while (ptx::globaltimer_ns() - t0 < 50000ull) {
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace gal

int read_gal_device_error(int reset) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_gal_error, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  if (reset) {
    int z = 0;
    e = cudaMemcpyToSymbol(g_gal_error, &z, sizeof(int));
    if (e != cudaSuccess) return (int)e;
  }
  return v;
}

// Slot rows, accumulators, resident query tiles and slots of one CTA: two
// query tiles when three document slots still fit beside them, else one (a
// query change then waits for the previous query's last MMA).  16-bit kinds
// share the SM with a second CTA (106 KB, 256 TMEM columns each).
template <bool I8>
static void gal_plan(int dim, gal::Params& P) {
  using K = gal::Kind<I8>;
  P.KB = I8 ? dim / 128 : dim / gal::KBLK;
  P.slot_rows = (I8 || P.KB == 1) ? 256 : 128;
  P.sr_log2 = P.slot_rows == 256 ? 8 : 7;
  P.acc_cols = (P.slot_rows / 128) * gal::NQ;
  P.nacc = K::TMEM_COLS / P.acc_cols;
  if (P.nacc > gal::NACC_MAX) P.nacc = gal::NACC_MAX;
  const int slot_bytes = P.KB * P.slot_rows * gal::ROWB;
  for (P.qslots = 2; P.qslots >= 1; --P.qslots) {
    P.nslots = (K::SMEM_BUDGET - 1024 - P.qslots * P.KB * gal::QTILE) / slot_bytes;
    if (P.nslots >= 3 || P.qslots == 1) break;
  }
  if (P.nslots > gal::SMAX) P.nslots = gal::SMAX;
}

// Shapes both kinds take: paired / candidate units of at most 32 query tokens,
// token rows addressable by TMA, at most nacc - 1 chunks per unit (an epilogue
// group then never waits on an accumulator whose previous use, by the other
// group, is still uncommitted -- a parity wait could not tell the two apart).
template <bool I8>
static bool gal_shape_ok(const ScanParams& p) {
  if (device_cc() != 100) return false;
  if (p.layout != L_PAIRED && p.layout != L_CANDIDATES) return false;
  if (p.Tq < 1 || p.Tq > gal::NQ) return false;
  if (p.nq_tok <= 0 || p.nd_tok <= 0 || p.nq_tok >= INT32_MAX || p.nd_tok >= INT32_MAX) return false;
  if ((reinterpret_cast<uintptr_t>(p.Q) & 15) || (reinterpret_cast<uintptr_t>(p.D) & 15)) return false;
  gal::Params P;
  gal_plan<I8>(p.dim, P);
  if (p.Td > (P.nacc - 1) * P.slot_rows) return false;
  return P.nslots >= 2;
}

bool scan_gallery_supported(int dtype, const ScanParams& p) {
  if (dtype != FMS_F16 && dtype != FMS_BF16) return false;
  if (p.dim < 64 || p.dim > 256 || p.dim % gal::KBLK != 0) return false;
  return gal_shape_ok<false>(p);
}

template <bool I8>
static cudaError_t gal_launch(gal::Params& P, const gal::Maps& maps, cudaStream_t s) {
  const ScanParams& p = P.p;
  const int dyn = P.qslots * P.KB * gal::QTILE + P.nslots * P.KB * P.slot_rows * gal::ROWB + 1024;
  auto k = p.args ? gal::gallery_kernel<true, I8> : gal::gallery_kernel<false, I8>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
  if (e != cudaSuccess) return e;
  int64_t grid = (int64_t)device_sm_count() * gal::Kind<I8>::CTAS_PER_SM;
  if (grid > p.nunits) grid = p.nunits;
  if (grid < 1) grid = 1;
  k<<<(unsigned)grid, gal::NTHREADS, dyn, s>>>(maps, P);
  return cudaGetLastError();
}

cudaError_t launch_scan_gallery(int dtype, const ScanParams& p, cudaStream_t s) {
  if (!scan_gallery_supported(dtype, p)) return cudaErrorNotSupported;
  gal::Params P;
  memset(&P, 0, sizeof(P));
  P.p = p;
  P.fmt = dtype == FMS_BF16 ? 1u : 0u;
  gal_plan<false>(p.dim, P);
  if (p.nunits == 0) return cudaSuccess;
  gal::Maps maps;
  if (!make_tmap_16(&maps.q, p.Q, P.fmt, p.dim, p.nq_tok, gal::NQ) ||
      !make_tmap_16(&maps.b128, p.D, P.fmt, p.dim, p.nd_tok, 128) ||
      !make_tmap_16(&maps.b64, p.D, P.fmt, p.dim, p.nd_tok, 64) ||
      !make_tmap_16(&maps.b32, p.D, P.fmt, p.dim, p.nd_tok, 32) ||
      !make_tmap_16(&maps.b16, p.D, P.fmt, p.dim, p.nd_tok, 16))
    return cudaErrorNotSupported;
  return gal_launch<false>(P, maps, s);
}

// INT8 pair / paired (int8_pair_forward_host, quant.jl:96-125; the reference's
// GPU path is the s8 WMMA kernel at ext/FlashMaxSimCUDAExt.jl:621-746): codes
// on the tensor cores (kind::i8), the pair formula in the epilogue.
static ScanParams i8_scan_params(const Int8ScanParams& ip) {
  ScanParams p;
  memset(&p, 0, sizeof(p));
  p.layout = L_PAIRED;
  p.Q = ip.Qc; p.D = ip.Dc; p.qmask = ip.qmask; p.dmask = ip.dmask;
  p.dim = ip.dim; p.Tq = ip.Tq; p.Td = ip.Td; p.B = (int)ip.N;
  p.nq_tok = (int64_t)ip.Tq * ip.N; p.nd_tok = (int64_t)ip.Td * ip.N;
  p.nunits = ip.N;
  p.normalize = ip.normalize; p.scores = ip.scores; p.args = ip.args;
  return p;
}

bool int8_paired_tc_supported(const Int8ScanParams& ip) {
  if (ip.exhaustive) return false;
  if (ip.dim % 128 != 0 || ip.dim < 128 || ip.dim > 256) return false;
  if (ip.N < 1 || ip.N >= INT32_MAX) return false;
  return gal_shape_ok<true>(i8_scan_params(ip));
}

cudaError_t launch_int8_paired_tc(const Int8ScanParams& ip, cudaStream_t s) {
  if (!int8_paired_tc_supported(ip)) return cudaErrorNotSupported;
  gal::Params P;
  memset(&P, 0, sizeof(P));
  P.p = i8_scan_params(ip);
  P.qs = ip.Qs; P.ds = ip.Ds;
  P.qs_f16 = ip.qs_dtype == FMS_F16; P.ds_f16 = ip.ds_dtype == FMS_F16;
  gal_plan<true>(ip.dim, P);
  gal::Maps maps;
  const ScanParams& p = P.p;
  if (!make_tmap_i8(&maps.q, p.Q, p.dim, p.nq_tok, gal::NQ) ||
      !make_tmap_i8(&maps.b128, p.D, p.dim, p.nd_tok, 128) ||
      !make_tmap_i8(&maps.b64, p.D, p.dim, p.nd_tok, 64) ||
      !make_tmap_i8(&maps.b32, p.D, p.dim, p.nd_tok, 32) ||
      !make_tmap_i8(&maps.b16, p.D, p.dim, p.nd_tok, 16))
    return cudaErrorNotSupported;
  return gal_launch<true>(P, maps, s);
}

}  // namespace fms
