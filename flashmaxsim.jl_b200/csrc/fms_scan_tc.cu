// fms_scan_tc.cu -- the sm_100a MaxSim engine for Float16 / BFloat16 features:
// TMA-staged tiles, tcgen05 MMAs accumulating in TMEM, and the fused
// max / argmax / Sigma_t epilogue read straight out of TMEM (the similarity
// matrix never reaches HBM).  Replaces the reference's WMMA m16n16k16 scans
// (ext/FlashMaxSimCUDAExt.jl:236-617) and its KA SRAM-tiled scans
// (kernels_forward.jl:125-356, kernels_packed.jl:35-227) for 16-bit inputs.
//
// Orientation: query tokens on the MMA M side (64 or 128 rows per tile, up to
// MAXMT tiles), document tokens on N (chunks of NT).  Each epilogue thread owns
// one query-token row of the accumulator, so the per-token max over document
// tokens is a register loop over TMEM columns -- no cross-thread reduction.
// For queries of <= 32 tokens a 128-row tile holds the query four times (R = 4):
// every TMEM subpartition (every epilogue warp) then holds all 32 rows and takes
// a quarter of the chunk's columns; the four partial (max, argmax) states meet
// in shared memory.  With 256-column chunks a whole document is one MMA chain
// (per-instruction issue cost, not tensor throughput, bounds small MMAs).
//
// Persistent CTAs walk contiguous ranges of units (one query run x one document
// run; the query tile then changes rarely along a CTA's range); a unit may
// stack several queries (in-batch, multi-query packed; up to 256 rows in two
// tiles and at most 128 queries) so one document tile
// feeds all of them.  Warp roles (224 threads):
//   warp 6  scheduler: decodes 32 upcoming units at once (one per lane: candidate
//           index, CSR bounds, first / last valid document token, document and
//           query mask bits) into a 16-entry shared-memory metadata ring, so the
//           dependent index -> mask global loads are off the other roles' paths;
//           single-query units with nothing to scan (slots outside 1:N or outside
//           this shard, empty documents) get their outputs written here and are
//           not queued; an end marker closes the queue;
//   warp 0  TMA producer: loads the document rows of a chunk (128/64/32/16-row
//           boxes, stopping at the last valid token, so masked padding is not
//           read) into an S-stage ring, with the query tile either resident
//           (re-loaded only when the unit's query changes) or carried per stage;
//   warp 1 (+ warps 7, 8)  MMA issuers, one per query tile (one elected lane
//           each): 4 K=16 MMAs per K block into the tile's columns of one of
//           NACC TMEM accumulator buffers, tcgen05.commit to the ring slot and,
//           after the chunk's last K block, to the accumulator barrier.  A single
//           thread that waits on a barrier between MMA groups leaves the tensor
//           pipe idle while it waits (a 128x128x16 MMA lasts 64 cycles, about
//           what one completed-barrier check costs the issuer); with one issuer
//           per tile the others keep the pipe fed;
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time, masked running
//           (max, argmax) per row -- a plain max when no tape is wanted -- then
//           Sigma_t per query in t order, the normalisation and the `neg` fill;
//           every output written once.
// Every wait is bounded: on a timeout the CTA raises an error flag, stops
// issuing, lets in-flight copies land, frees TMEM and returns.
#include <cuda.h>
#include <stdlib.h>
#include <mutex>

#include "fms_common.cuh"
#include "fms_internal.h"
#include "fms_tc_ptx.cuh"

namespace fms {

__device__ int g_tc_error = 0;  // set when an engine wait timed out (diagnostic)

namespace tc {

constexpr int KBLK = 64;    // K elements per block: one 128-byte swizzled row
constexpr int ROWB = 128;   // bytes per tile row
constexpr int SCHED_WARP = 6;
constexpr int UQ = 16;      // metadata ring depth (units)
constexpr int MW_MAX = 16;  // document-mask words carried per unit (Td <= 512)
constexpr int QW_MAX = 12;  // query-row valid words (rows <= 384)

struct TcParams {
  ScanParams p;
  int G;          // queries stacked per unit (in-batch / packed), else 1
  int ngroups;    // query groups
  int64_t nunits;
  int KB;         // K blocks (dim / 64)
  uint32_t fmt;   // 0 = f16, 1 = bf16
};

struct TcUnit {
  bool valid;
  int64_t q_row0;
  int nq;                 // queries in the unit
  int Tq;                 // tokens per query
  const uint8_t* qmask;   // mask of the unit's first query (stride Tq)
  int64_t d_row0;
  int Td;
  const uint8_t* dmask;
  int64_t out0, out_stride;
  int64_t arg0, arg_stride;
  int arg_rows;
};

// One unit as the other roles see it (written by the scheduler warp).
struct UnitMeta {
  int64_t q_row0, d_row0, out0, out_stride, arg0, arg_stride;
  const uint8_t* dmask;   // kept for documents longer than 32*MW_MAX tokens
  int nq, Tq, leff, first, valid, arg_rows, mw_ok, aflags;  // aflags bit0: load a new query tile
  uint32_t mw[MW_MAX];    // bit u: document token u valid (u < 32*MW_MAX)
  uint32_t qw[QW_MAX];    // bit r: query row r valid
};

__device__ __forceinline__ TcUnit tc_decode(const TcParams& P, int64_t v) {
  const ScanParams& p = P.p;
  TcUnit U;
  if (p.layout == L_INBATCH || p.layout == L_PACKED) {
    // query-group major: consecutive units share their query tile
    const int64_t ndocs = (p.layout == L_INBATCH) ? p.Bd : p.B;
    const int g = (int)(v / ndocs);
    const int64_t j = v - (int64_t)g * ndocs;  // document: in-batch j, packed b
    const int qi0 = g * P.G;
    const int nqt = (p.layout == L_INBATCH) ? p.Bq : p.nq;
    U.valid = true;
    U.nq = min(P.G, nqt - qi0);
    U.Tq = p.Tq;
    U.q_row0 = (int64_t)qi0 * p.Tq;
    U.qmask = p.qmask ? p.qmask + (int64_t)qi0 * p.Tq : nullptr;
    U.arg_rows = p.Tq;
    if (p.layout == L_INBATCH) {
      U.d_row0 = j * p.Td;
      U.Td = p.Td;
      U.dmask = p.dmask ? p.dmask + j * p.Td : nullptr;
      U.out0 = j + (int64_t)p.Bd * qi0;
      U.out_stride = p.Bd;
    } else {
      U.d_row0 = (int64_t)p.cu_d[j] - 1;
      U.Td = p.cu_d[j + 1] - p.cu_d[j];
      clamp_run(U.d_row0, U.Td, p.nd_tok);
      U.dmask = nullptr;
      U.out0 = j + (int64_t)p.B * qi0;
      U.out_stride = p.B;
    }
    U.arg0 = U.out0 * p.Tq;
    U.arg_stride = U.out_stride * p.Tq;
  } else {
    const Unit u1 = decode_unit(p, v);
    U.valid = u1.valid;
    U.q_row0 = u1.q0;
    U.nq = 1;
    U.Tq = u1.Tq;
    U.qmask = u1.qmask;
    U.d_row0 = u1.d0;
    U.Td = u1.Td;
    U.dmask = u1.dmask;
    U.out0 = u1.out;
    U.out_stride = 0;
    U.arg0 = u1.arg0;
    U.arg_stride = 0;
    U.arg_rows = u1.arg_rows;
  }
  return U;
}

// Nonzero bytes of a 32-bit word -> 4 bits.
__device__ __forceinline__ uint32_t nz4(uint32_t w) {
  const uint32_t r = __vcmpne4(w, 0u);
  return (r & 1u) | ((r >> 7) & 2u) | ((r >> 14) & 4u) | ((r >> 21) & 8u);
}

// Bits of n mask bytes (0/1) starting at m into words (per thread, sequential
// loads; 16-byte vector loads when aligned).  Bits past n are zero.
template <int W>
__device__ __forceinline__ void mask_bits(const uint8_t* m, int n, uint32_t (&w)[W]) {
#pragma unroll
  for (int i = 0; i < W; ++i) w[i] = 0u;
  if (m == nullptr) {
#pragma unroll
    for (int i = 0; i < W; ++i) {
      const int lo = 32 * i;
      w[i] = n >= lo + 32 ? 0xffffffffu : (n > lo ? ((1u << (n - lo)) - 1u) : 0u);
    }
    return;
  }
  if ((reinterpret_cast<uintptr_t>(m) & 15) == 0) {
#pragma unroll
    for (int i = 0; i < 2 * W; ++i) {  // 16 bytes per step
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


// Shared-memory / TMEM plan of one engine configuration.
//  NT     document rows per chunk (one MMA N), NACC accumulator buffers in TMEM
//         (the MMA may run NACC chunks ahead of the epilogue).
//  ARES   the query tile of a unit (all K blocks) stays resident in one of two
//         slots, re-loaded only when the unit's query differs from the previous
//         unit's; a ring stage then carries one chunk of document rows for all
//         K blocks (one barrier round trip per chunk).  Without ARES (large dim)
//         a stage carries one K block of both operands.
//  SMAX   ring stages available (the launch uses as many as fit its budget).
//  MAXMT = 3 (384 query rows, resident, one CTA per SM): the single
//         accumulator is handed over tile by tile -- the MMA issuer fills tile m
//         of the next chunk as soon as the epilogue has read tile m of this one,
//         so the MMAs of one tile overlap the epilogue of the previous tile.
template <int M, int NT, int MAXMT, int R, int NACC, int SMAX, int ARES>
struct Cfg {
  static constexpr bool TP = MAXMT == 3;            // tile-by-tile accumulator hand-off
  static constexpr int NISS = MAXMT;                // MMA issuer warps: 1, then 7, 8
  static constexpr int NTHR = (6 + NISS) * 32;      // producer, issuers, 4 epilogue, scheduler
  static constexpr int MINB = NACC * MAXMT * NT > 256 ? 1 : 2;  // CTAs per SM (TMEM: 512 columns)
  static constexpr int NBAR = TP ? MAXMT : NACC;    // accumulator barrier pairs
  static constexpr int A_BYTES = MAXMT * M * ROWB;  // one K block of all M tiles
  static constexpr int B_BYTES = NT * ROWB;         // one K block of a chunk
  static constexpr int ACC_COLS = MAXMT * NT;       // TMEM columns per accumulator buffer
  static constexpr int TMEM_COLS = NACC * ACC_COLS;
  // allocation: a power of two of at least 32 columns (three 128-column tiles use 512)
  static constexpr int TMEM_ALLOC = TMEM_COLS <= 128 ? 128 : TMEM_COLS <= 256 ? 256 : 512;
  static constexpr int HALF = NT / R;               // columns per epilogue thread per chunk
  static __host__ __device__ int stage_bytes(int KB) { return ARES ? KB * B_BYTES : A_BYTES + B_BYTES; }
  static __host__ __device__ int aslot_bytes(int KB) { return ARES ? KB * A_BYTES : 0; }
  static_assert(R == 1 || (R == 2 && M == 64 && MAXMT == 1) || (R == 4 && M == 128 && MAXMT == 1),
                "replication: 2 copies of 32 rows in a 64-row tile, or 4 in a 128-row tile");
  static_assert(TMEM_COLS % 128 == 0 && TMEM_COLS <= 512, "TMEM columns");
  static_assert(HALF % 32 == 0, "epilogue reads 32-column groups");
  static_assert(!TP || (NACC == 1 && ARES == 1 && R == 1 && M == 128),
                "tile hand-off: one accumulator, resident query, 128-row tiles");
};

struct BMaps {
  CUtensorMap b128, b64, b32, b16;  // document rows, boxes of 128 / 64 / 32 / 16 rows
};

// Document rows [row, row + nr) of one K block (nr a multiple of 16, <= NT):
// 128-row boxes, then at most one box each of 64, 32 and 16 rows.
__device__ __forceinline__ void load_doc_rows(unsigned char* sB, const BMaps& bm, int x, int64_t row,
                                              int nr, uint64_t* bar) {
  int r = 0;
  for (; nr - r >= 128; r += 128) ptx::tma_load_2d(sB + r * ROWB, &bm.b128, x, (int)(row + r), bar);
  if (nr - r >= 64) { ptx::tma_load_2d(sB + r * ROWB, &bm.b64, x, (int)(row + r), bar); r += 64; }
  if (nr - r >= 32) { ptx::tma_load_2d(sB + r * ROWB, &bm.b32, x, (int)(row + r), bar); r += 32; }
  if (nr - r >= 16) { ptx::tma_load_2d(sB + r * ROWB, &bm.b16, x, (int)(row + r), bar); r += 16; }
}

// Registers are capped for two co-resident CTAs, except for the three-tile
// configuration (one CTA per SM).
template <int M, int NT, int MAXMT, int R, int NACC, int SMAX, int ARES, bool ARGS>
__global__ void __launch_bounds__(Cfg<M, NT, MAXMT, R, NACC, SMAX, ARES>::NTHR,
                                  Cfg<M, NT, MAXMT, R, NACC, SMAX, ARES>::MINB)
tc_scan_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ BMaps bm, TcParams P,
               int S) {
  using L = Cfg<M, NT, MAXMT, R, NACC, SMAX, ARES>;
  extern __shared__ __align__(1024) unsigned char dsm[];
  __shared__ __align__(8) uint64_t full_bar[SMAX];
  __shared__ __align__(8) uint64_t empty_bar[SMAX];
  __shared__ __align__(8) uint64_t afull_bar[2];
  __shared__ __align__(8) uint64_t aempty_bar[2];
  __shared__ __align__(8) uint64_t accf_bar[L::NBAR];
  __shared__ __align__(8) uint64_t acce_bar[L::NBAR];
  __shared__ __align__(8) uint64_t metaf_bar[UQ];
  __shared__ __align__(8) uint64_t metae_bar[UQ];
  __shared__ __align__(8) uint64_t epi_bar;  // epilogue-wide barrier (bounded, unlike bar.sync);
                                             // one arrival per epilogue warp
  __shared__ UnitMeta meta[UQ];
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile int abort_s;
  // per-row results and the copies' states, double-buffered by unit parity so that
  // the next unit may write while the current one is still being read
  __shared__ __align__(16) float red_s[2][MAXMT * M];
  __shared__ float half_mx[2][3][32];  // states of the copies 1..R-1, handed to copy 0
  __shared__ int half_ag[2][3][32];
  __shared__ float half_s0[2][3][32];

  unsigned char* tiles = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(dsm) + 1023) & ~(uintptr_t)1023);
  unsigned char* aslots = tiles;  // ARES only
  const int abytes = L::aslot_bytes(P.KB);
  const int sbytes = L::stage_bytes(P.KB);
  unsigned char* ring = tiles + ARES * abytes;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const ScanParams& p = P.p;

  if (threadIdx.x == 0) {
    // every issuer commits to each ring slot, query slot and (without the tile
    // hand-off) accumulator it uses
    for (int i = 0; i < SMAX; ++i) {
      ptx::mbar_init(&full_bar[i], 1);
      ptx::mbar_init(&empty_bar[i], L::NISS);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&afull_bar[i], 1);
      ptx::mbar_init(&aempty_bar[i], L::NISS);
    }
    for (int i = 0; i < L::NBAR; ++i) {
      ptx::mbar_init(&accf_bar[i], L::TP ? 1 : L::NISS);
      ptx::mbar_init(&acce_bar[i], 4);  // one arrival per epilogue warp
    }
    for (int i = 0; i < UQ; ++i) {
      ptx::mbar_init(&metaf_bar[i], 1);
      ptx::mbar_init(&metae_bar[i], 5 + L::NISS);  // producer + issuers + 4 epilogue warps
    }
    ptx::mbar_init(&epi_bar, 4);
    abort_s = 0;
    ptx::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmA);
    ptx::prefetch_tmap(&bm.b128);
    ptx::prefetch_tmap(&bm.b64);
    ptx::prefetch_tmap(&bm.b32);
    ptx::prefetch_tmap(&bm.b16);
  }
  if (warp == 1) ptx::tmem_alloc(&tmem_base_s, L::TMEM_ALLOC);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;
  // a contiguous range of units (or of unit-list entries) per CTA (query tiles
  // change rarely along it)
  const int64_t nwalk = p.unit_count ? (int64_t)*p.unit_count : P.nunits;
  const int64_t u_begin = nwalk * blockIdx.x / gridDim.x;
  const int64_t my_units = nwalk * (blockIdx.x + 1) / gridDim.x - u_begin;
  // K blocks per ring stage and stages per chunk
  const int kbs = ARES ? P.KB : 1;
  const int spc = ARES ? 1 : P.KB;

  if (warp == SCHED_WARP) {
    // ------------------------------------------------------------ scheduler
    int have_prev = 0;       // warp-uniform: last working unit's query run
    int64_t prev_q = -1;
    int64_t qn = 0;          // warp-uniform: units queued so far
    float* scores_out = static_cast<float*>(p.scores);
    for (int64_t i0 = 0; i0 < my_units; i0 += 32) {
      if (__any_sync(0xffffffffu, abort_s != 0)) break;  // warp-uniform exit
      const int64_t i = i0 + lane;
      UnitMeta m;
      int working = 0, direct = 0;
      if (i < my_units) {
        const TcUnit U = tc_decode(P, unit_at(p, u_begin + i));
        m.q_row0 = U.q_row0; m.d_row0 = U.d_row0;
        m.out0 = U.out0; m.out_stride = U.out_stride;
        m.arg0 = U.arg0; m.arg_stride = U.arg_stride;
        m.dmask = U.dmask;
        m.nq = U.nq; m.Tq = U.Tq; m.valid = U.valid ? 1 : 0; m.arg_rows = U.arg_rows;
        const int rows = U.nq * U.Tq;
        mask_bits<QW_MAX>(U.qmask, rows < 32 * QW_MAX ? rows : 32 * QW_MAX, m.qw);
        m.mw_ok = U.Td <= 32 * MW_MAX;
        int first = -1, last = -1;
        if (U.valid) {
          mask_bits<MW_MAX>(U.dmask, U.Td < 32 * MW_MAX ? U.Td : 32 * MW_MAX, m.mw);
#pragma unroll
          for (int w = MW_MAX - 1; w >= 0; --w)
            if (m.mw[w]) { first = 32 * w + __ffs(m.mw[w]) - 1; }
#pragma unroll
          for (int w = 0; w < MW_MAX; ++w)
            if (m.mw[w]) { last = 32 * w + 31 - __clz(m.mw[w]); }
          for (int u = 32 * MW_MAX; u < U.Td; ++u)  // long documents: mask tail scanned here
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
        working = (m.valid && rows > 0 && m.leff > 0) ? 1 : 0;
        if (!working && U.nq == 1) {
          // nothing to scan (a slot outside 1:N or this shard, an empty or
          // fully masked document, no query rows): the unit's outputs are
          // written here and it never enters the pipeline
          scores_out[U.out0] = U.valid ? 0.f : (float)p.neg;
          if (ARGS)
            for (int t = 0; t < U.arg_rows; ++t) p.args[U.arg0 + t] = 0;
          direct = 1;
        }
      }
      // a new query tile is needed when a working unit's query run differs from
      // the previous working unit's (scanned in unit order across the warp)
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
      m.aflags = anew;
      // queue the other units in order (entry index qn counts queued units)
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
    // end marker: the other roles stop at an entry with valid < 0
    if (lane == 0 && !abort_s) {
      const int slot = (int)(qn % UQ);
      if (ptx::mbar_wait(&metae_bar[slot], (uint32_t)(((qn / UQ) & 1) ^ 1), &abort_s)) {
        meta[slot].valid = -1;
        ptx::mbar_arrive(&metaf_bar[slot]);
      }
    }
    __syncwarp();
  } else if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    int stage = 0;
    uint32_t phase = 0;
    int aslot = ARES - 1;    // ARES: slot of the current query tile
    uint32_t aphase = 1;     // flips when aslot wraps to 0
    for (int64_t i = 0;; ++i) {  // queued units, up to the end marker
      const int slot = (int)(i % UQ);
      if (!ptx::all_wait(&metaf_bar[slot], (uint32_t)((i / UQ) & 1), &abort_s)) goto done;
      const UnitMeta& m = meta[slot];
      if (m.valid < 0) break;
      const int rows = m.nq * m.Tq;
      const int nmt = (rows + M - 1) / M;
      const int nch = (m.valid && rows > 0) ? (m.leff + NT - 1) / NT : 0;
      const int64_t q_row0 = m.q_row0, d_row0 = m.d_row0;
      const int leff = m.leff;
      const int anew = m.aflags & 1;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&metae_bar[slot]);
      if (ARES && anew) {
        if (++aslot == ARES) { aslot = 0; aphase ^= 1; }
        if (!ptx::all_wait(&aempty_bar[aslot], aphase ^ 1, &abort_s)) goto done;
        if (lane == 0) {
          unsigned char* sA = aslots + aslot * abytes;
          ptx::mbar_expect_tx(&afull_bar[aslot], (uint32_t)(P.KB * nmt * M * ROWB));
          for (int kb = 0; kb < P.KB; ++kb) {
            unsigned char* sAk = sA + kb * L::A_BYTES;
            if (R > 1) {  // R copies of the 32-row query: rows 0-31, 32-63, ...
              for (int q = 0; q < R; ++q)
                ptx::tma_load_2d(sAk + q * 32 * ROWB, &tmA, kb * KBLK, (int)q_row0, &afull_bar[aslot]);
            } else {
              for (int mt = 0; mt < nmt; ++mt)
                ptx::tma_load_2d(sAk + mt * M * ROWB, &tmA, kb * KBLK, (int)(q_row0 + mt * M),
                                 &afull_bar[aslot]);
            }
          }
        }
        __syncwarp();
      }
      for (int c = 0; c < nch; ++c) {
        const int u0 = c * NT;
        const int n = min(NT, leff - u0);
        const int nr = (n + 15) & ~15;
        for (int ks = 0; ks < spc; ++ks) {
          if (!ptx::all_wait(&empty_bar[stage], phase ^ 1, &abort_s)) goto done;
          if (lane == 0) {
            unsigned char* st = ring + stage * sbytes;
            if (ARES) {
              ptx::mbar_expect_tx(&full_bar[stage], (uint32_t)(kbs * nr * ROWB));
              for (int kb = 0; kb < kbs; ++kb)
                load_doc_rows(st + kb * L::B_BYTES, bm, kb * KBLK, d_row0 + u0, nr, &full_bar[stage]);
            } else {
              ptx::mbar_expect_tx(&full_bar[stage], (uint32_t)(nmt * M * ROWB + nr * ROWB));
              if (R > 1) {
                for (int q = 0; q < R; ++q)
                  ptx::tma_load_2d(st + q * 32 * ROWB, &tmA, ks * KBLK, (int)q_row0, &full_bar[stage]);
              } else {
                for (int mt = 0; mt < nmt; ++mt)
                  ptx::tma_load_2d(st + mt * M * ROWB, &tmA, ks * KBLK, (int)(q_row0 + mt * M),
                                   &full_bar[stage]);
              }
              load_doc_rows(st + L::A_BYTES, bm, ks * KBLK, d_row0 + u0, nr, &full_bar[stage]);
            }
          }
          __syncwarp();
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1 || warp > SCHED_WARP) {
    // ------------------------------------------------------------ MMA issuers
    const int mo = warp == 1 ? 0 : warp - SCHED_WARP;  // this issuer's query tile
    int stage = 0;
    uint32_t phase = 0;
    int as = 0;
    uint32_t aphase = 0;
    int aslot = ARES - 1;
    uint32_t aslot_phase = 1;
    bool holding = false;    // ARES: an A slot is in use (released on the next switch)
    uint32_t tph = 0;        // TP: phase of this tile's accumulator barriers
    for (int64_t i = 0;; ++i) {  // queued units, up to the end marker
      const int slot = (int)(i % UQ);
      if (!ptx::all_wait(&metaf_bar[slot], (uint32_t)((i / UQ) & 1), &abort_s)) goto done;
      const UnitMeta& m = meta[slot];
      if (m.valid < 0) break;
      const int rows = m.nq * m.Tq;
      const int nmt = (rows + M - 1) / M;
      const int nch = (m.valid && rows > 0) ? (m.leff + NT - 1) / NT : 0;
      const int leff = m.leff;
      const int anew = m.aflags & 1;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&metae_bar[slot]);
      if (ARES && anew) {
        if (holding && lane == 0) ptx::mma_commit(&aempty_bar[aslot]);  // after its last MMA
        if (++aslot == ARES) { aslot = 0; aslot_phase ^= 1; }
        if (!ptx::all_wait(&afull_bar[aslot], aslot_phase, &abort_s)) goto done;
        ptx::tc_fence_after();
        holding = true;
      }
      const bool mine = mo < nmt;  // this unit has a tile for this issuer
      for (int c = 0; c < nch; ++c) {
        const int n = min(NT, leff - c * NT);
        const int nr = (n + 15) & ~15;
        const uint32_t idesc = ptx::idesc_f16(P.fmt, M, nr);
        if (!L::TP) {
          if (!ptx::all_wait(&acce_bar[as], aphase ^ 1, &abort_s)) goto done;
          ptx::tc_fence_after();
        }
        for (int ks = 0; ks < spc; ++ks) {
          if (!ptx::all_wait(&full_bar[stage], phase, &abort_s)) goto done;
          ptx::tc_fence_after();
          if (L::TP && mine) {
            // tile hand-off: the epilogue has released this tile's columns
            if (!ptx::all_wait(&acce_bar[mo], tph ^ 1u, &abort_s)) goto done;
            ptx::tc_fence_after();
          }
          if (lane == 0) {
            if (mine) {
              const uint32_t st = ptx::smem_u32(ring + stage * sbytes);
              const uint32_t d = tmem_base + (uint32_t)(as * L::ACC_COLS + mo * NT);
              for (int kk = 0; kk < kbs; ++kk) {
                const int kb = ARES ? kk : ks;
                const uint32_t sA = ARES ? ptx::smem_u32(aslots + aslot * abytes + kb * L::A_BYTES) : st;
                const uint32_t sB = ARES ? st + kk * L::B_BYTES : st + L::A_BYTES;
                const uint64_t adesc = ptx::sw128_desc(sA + mo * M * ROWB);
                const uint64_t bdesc = ptx::sw128_desc(sB);
#pragma unroll
                for (int k = 0; k < KBLK / 16; ++k)
                  ptx::mma_f16(d, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0);
              }
              if (L::TP) ptx::mma_commit(&accf_bar[mo]);
            }
            ptx::mma_commit(&empty_bar[stage]);
          }
          __syncwarp();
          if (L::TP && mine) tph ^= 1u;
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!L::TP) {
          if (lane == 0) ptx::mma_commit(&accf_bar[as]);
          __syncwarp();
          if (++as == NACC) { as = 0; aphase ^= 1; }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int sp = warp & 3;   // TMEM subpartition of this warp
    const int et = threadIdx.x - 64;  // 0..127
    // row of the accumulator this thread reads, and its column half
    //  R = 4: every subpartition holds rows 0-31 (one copy each) -> column quarter sp
    //  R = 2: subpartitions {0,1} and {2,3} hold the two copies -> column half sp/2
    const int lr = (R == 4) ? lane
                 : (M == 128) ? sp * 32 + lane
                 : (lane < 16 ? (R == 2 ? (sp & 1) * 16 : sp * 16) + lane : -1);
    const int h = (R == 4) ? sp : (R == 2) ? (sp >> 1) : 0;
    int as = 0;
    uint32_t aphase = 0;
    uint32_t ephase = 0;
    uint32_t tph = 0;  // TP: bit mt = phase of tile mt's accumulator barriers
    float* scores = static_cast<float*>(p.scores);
    for (int64_t i = 0;; ++i) {  // queued units, up to the end marker
      const int slot = (int)(i % UQ);
      if (!ptx::all_wait(&metaf_bar[slot], (uint32_t)((i / UQ) & 1), &abort_s)) goto done;
      const UnitMeta& m = meta[slot];
      if (m.valid < 0) break;
      const int ub = (int)(i & 1);  // buffer of this unit (red_s, half_*)
      if (!m.valid) {
        if (et == 0) scores[m.out0] = (float)p.neg;
        if (ARGS)
          for (int t = et; t < m.arg_rows; t += 128) p.args[m.arg0 + t] = 0;
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&metae_bar[slot]);
        continue;
      }
      const int rows = m.nq * m.Tq;
      const int nmt = (rows + M - 1) / M;
      const int nch = rows == 0 ? 0 : (m.leff + NT - 1) / NT;
      const int first = m.first, leff = m.leff;
      float mx[MAXMT], s0[MAXMT];
      int ag[MAXMT];
      bool has_s0 = false;
#pragma unroll
      for (int mt = 0; mt < MAXMT; ++mt) { mx[mt] = -INFINITY; ag[mt] = 0; s0[mt] = 0.f; }
      for (int c = 0; c < nch; ++c) {
        const int u0 = c * NT;
        const int n = min(NT, leff - u0);
        uint32_t mw[L::HALF / 32];
#pragma unroll
        for (int g = 0; g < L::HALF / 32; ++g) {
          const int col0 = h * L::HALF + 32 * g;  // chunk column of this group
          uint32_t w;
          if (m.mw_ok) {
            w = (u0 + col0) < 32 * MW_MAX ? m.mw[(u0 + col0) >> 5] : 0u;
          } else {
            const int cc = col0 + lane;
            const bool ok = cc < n && (m.dmask == nullptr || m.dmask[u0 + cc] != 0);
            w = __ballot_sync(0xffffffffu, ok);
          }
          const int lim = n - col0;
          mw[g] = lim >= 32 ? w : (lim > 0 ? w & ((1u << lim) - 1u) : 0u);
        }
        if (!L::TP) {
          if (!ptx::all_wait(&accf_bar[as], aphase, &abort_s)) goto done;
          ptx::tc_fence_after();
        }
        const uint32_t tb = tmem_base + ((uint32_t)(sp * 32) << 16) + (uint32_t)(as * L::ACC_COLS);
        const int fc = first - u0 - h * L::HALF;  // first valid column, in my half?
        const bool s0_here = fc >= 0 && fc < L::HALF && first - u0 < n;
        bool chunk_full = true;  // every column of the chunk valid (warp-uniform)
#pragma unroll
        for (int g = 0; g < L::HALF / 32; ++g) chunk_full = chunk_full && mw[g] == 0xffffffffu;
        // one copy of the tile body (the running states of the tiles are
        // selected in and out of registers): unrolling it per tile multiplies
        // the epilogue's code, and instruction fetch then stalls it
#pragma unroll 1
        for (int mt = 0; mt < nmt; ++mt) {
          float cmx = mx[0];
          int cag = ag[0];
#pragma unroll
          for (int q = 1; q < MAXMT; ++q)
            if (mt == q) { cmx = mx[q]; cag = ag[q]; }
          if (L::TP) {
            if (!ptx::all_wait(&accf_bar[mt], (tph >> mt) & 1u, &abort_s)) goto done;
            ptx::tc_fence_after();
          }
          // GB 32-column groups are loaded before one wait (three or four with
          // one CTA per SM; two when registers are shared).  The
          // group code is branch-free apart from one warp-uniform test per tile
          // (are all the chunk's columns valid?) and, with the tape, one vote
          // per group: on this part a branch costs more than the dozens of
          // selects it would skip.
          constexpr int NG = L::HALF / 32;
          constexpr int GB = L::MINB == 1 ? (NG % 3 == 0 ? 3 : (NG < 4 ? NG : 4)) : (NG < 2 ? NG : 2);
#pragma unroll
          for (int g0 = 0; g0 < NG; g0 += GB) {
            uint32_t r[GB][32];
            // columns past the chunk's end are read too (they lie inside this
            // tile's accumulator) and masked out below
#pragma unroll
            for (int gg = 0; gg < GB; ++gg) ptx::tmem_ld32(tb + mt * NT + h * L::HALF + 32 * (g0 + gg), r[gg]);
            ptx::tmem_wait_ld();
            if (!chunk_full) {
#pragma unroll
              for (int gg = 0; gg < GB; ++gg) {
                const uint32_t mm = mw[g0 + gg];
#pragma unroll
                for (int cc = 0; cc < 32; ++cc)
                  r[gg][cc] = ((mm >> cc) & 1u) ? r[gg][cc] : __float_as_uint(-INFINITY);
              }
            }
#pragma unroll
            for (int gg = 0; gg < GB; ++gg) {
              // max of the group's valid non-NaN entries: four interleaved
              // chains of three-input maxima (NaN inputs are dropped, so the
              // order does not matter); masked columns hold -inf
              float t4[4] = {ARGS ? -INFINITY : cmx, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
              for (int cc = 0; cc < 32; cc += 2)
                t4[(cc >> 1) & 3] = ptx::fmax3(t4[(cc >> 1) & 3], __uint_as_float(r[gg][cc]),
                                               __uint_as_float(r[gg][cc + 1]));
              const float gmax = fmaxf(fmaxf(t4[0], t4[1]), fmaxf(t4[2], t4[3]));
              if (ARGS) {
                // the running (max, argmax) of a strict `>` scan in column
                // order: the group wins only with a strictly larger value, and
                // its argmax is the first column holding that value (a masked
                // column holds -inf, which never wins)
                if (__any_sync(0xffffffffu, gmax > cmx)) {
                  int idx = 31;
#pragma unroll
                  for (int cc = 30; cc >= 0; --cc) idx = (__uint_as_float(r[gg][cc]) == gmax) ? cc : idx;
                  const bool take = gmax > cmx;
                  cag = take ? u0 + h * L::HALF + 32 * (g0 + gg) + idx + 1 : cag;
                  cmx = take ? gmax : cmx;
                }
              } else {
                // values only; the first-valid rule is applied at the end
                cmx = gmax;
              }
            }
          }
          float cs0 = 0.f;
          if (s0_here) {
            cs0 = __uint_as_float(ptx::tmem_ld1(tb + mt * NT + (first - u0)));
            ptx::tmem_wait_ld();
            has_s0 = true;
          }
#pragma unroll
          for (int q = 0; q < MAXMT; ++q)
            if (mt == q) {
              mx[q] = cmx;
              ag[q] = cag;
              if (s0_here) s0[q] = cs0;
            }
          if (L::TP) {
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&acce_bar[mt]);
            tph ^= 1u << mt;
          }
        }
        if (!L::TP) {
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&acce_bar[as]);
          if (++as == NACC) { as = 0; aphase ^= 1; }
        }
      }
      if (R > 1) {
        // copies 1..R-1 of rows 0-31 (the other column slices) hand their states over
        if (h > 0 && lr >= 0) {
          half_mx[ub][h - 1][lr] = mx[0];
          half_ag[ub][h - 1][lr] = ag[0] | (has_s0 ? (1 << 30) : 0);  // flag: this slice read column `first`
          half_s0[ub][h - 1][lr] = has_s0 ? s0[0] : 0.f;
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&epi_bar);
        if (!ptx::all_wait(&epi_bar, ephase, &abort_s)) goto done;
        ephase ^= 1;
        if (h == 0 && lr >= 0) {
#pragma unroll
          for (int q = 0; q < R - 1; ++q) {
            const int a2 = half_ag[ub][q][lr];
            if (ARGS)
              merge_state(mx[0], ag[0], half_mx[ub][q][lr], a2 & ~(1 << 30));
            else
              mx[0] = fmaxf(mx[0], half_mx[ub][q][lr]);
            if (!has_s0 && (a2 & (1 << 30))) { s0[0] = half_s0[ub][q][lr]; has_s0 = true; }
          }
        }
      }
      // finish the rows: exact first-valid rule, tape, per-row contribution.
      // One query of <= 32 rows with R = 4: the rows are the lanes of the copy-0
      // warp, which sums them itself (butterfly; no shared-memory round trip and
      // no second epilogue barrier).  Otherwise rows go through red_s and one
      // thread per query sums them in t order.
      const bool one_warp = (R == 4) && (m.nq == 1);
      float rowv[MAXMT];
#pragma unroll
      for (int mt = 0; mt < MAXMT; ++mt) {
        rowv[mt] = 0.f;
        const int r = mt * M + lr;
        if (mt < nmt && lr >= 0 && h == 0 && r < rows) {
          const int qi = r / m.Tq, t = r - qi * m.Tq;
          const bool tv = (m.qw[r >> 5] >> (r & 31)) & 1u;
          float v = mx[mt];
          int a = ag[mt];
          bool ok;
          if (ARGS) {
            final_fixup(v, a, first, s0[mt]);
            ok = tv && a > 0;
          } else {
            // a NaN in the first valid column sticks; otherwise the max of the
            // non-NaN values (>= that column's value) is the result
            if (first >= 0 && s0[mt] != s0[mt]) v = s0[mt];
            ok = tv && first >= 0;
          }
          rowv[mt] = ok ? v : 0.f;
          if (!one_warp) red_s[ub][r] = rowv[mt];
          if (ARGS) p.args[m.arg0 + qi * m.arg_stride + t] = ok ? a : 0;
        }
      }
      if (one_warp) {
        if (h == 0) {
          float sum = rowv[0];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
          if (lane == 0) {
            if (p.normalize) {
              const uint32_t vm = m.Tq >= 32 ? 0xffffffffu : ((1u << m.Tq) - 1u);
              const int nvalid = __popc(m.qw[0] & vm);
              sum = sum * (1.0f / (float)(nvalid > 1 ? nvalid : 1));
            }
            scores[m.out0] = sum;
          }
        }
      } else {
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&epi_bar);
        if (!ptx::all_wait(&epi_bar, ephase, &abort_s)) goto done;
        ephase ^= 1;
        if (et < m.nq) {
          const int qi = et;
          const float* rs = red_s[ub] + qi * m.Tq;
          float score = 0.f;
          // Sigma_t in t order (forward_pair.jl:92-95)
          if ((m.Tq & 3) == 0) {
            for (int t = 0; t < m.Tq; t += 4) {
              const float4 v4 = *reinterpret_cast<const float4*>(rs + t);
              score += v4.x;
              score += v4.y;
              score += v4.z;
              score += v4.w;
            }
          } else {
            for (int t = 0; t < m.Tq; ++t) score += rs[t];
          }
          if (p.normalize) {
            int nvalid = 0;
            for (int t = 0; t < m.Tq; ++t) {
              const int r = qi * m.Tq + t;
              nvalid += (m.qw[r >> 5] >> (r & 31)) & 1u;
            }
            score = score * (1.0f / (float)(nvalid > 1 ? nvalid : 1));
          }
          scores[m.out0 + qi * m.out_stride] = score;
        }
      }
      if (ARGS)
        for (int t = m.Tq + et; t < m.arg_rows; t += 128) p.args[m.arg0 + t] = 0;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&metae_bar[slot]);
    }
  }
done:
  if (abort_s && threadIdx.x == 0) {
    atomicExch(&g_tc_error, 1);
    // let copies and MMAs already in flight land before shared memory and TMEM go away
    const uint64_t t0 = ptx::globaltimer_ns();
    while (ptx::globaltimer_ns() - t0 < 50000ull) {
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, L::TMEM_ALLOC);
  }
}

// ---------------------------------------------------------------- host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 2-D map over a token matrix (dim, rows) of 16-bit elements: box 64 x box_rows,
// 128-byte swizzle, zero fill out of bounds.
static bool make_map(CUtensorMap* m, const void* base, uint32_t fmt, int dim, int64_t rows, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[2] = {(cuuint64_t)dim, (cuuint64_t)rows};
  cuuint64_t gstride[1] = {(cuuint64_t)dim * 2};
  cuuint32_t box[2] = {(cuuint32_t)KBLK, (cuuint32_t)box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = enc(m, fmt == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                   const_cast<void*>(base), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static int queries_total(const ScanParams& p) {
  return p.layout == L_INBATCH ? p.Bq : (p.layout == L_PACKED ? p.nq : 1);
}

// Largest stacked row count: three resident 128-row tiles when the query's K
// blocks fit (dim <= 128: 96 KB of query tile), else two tiles carried per stage.
static int max_rows(const ScanParams& p) { return p.dim <= 2 * KBLK ? 384 : 256; }

// Queries stacked per unit and the resulting row count (up to max_rows(); at
// most 128 queries, one epilogue thread sums each).
static void plan(const ScanParams& p, int& G, int& rows) {
  const int Tq = p.Tq;
  G = 1;
  if ((p.layout == L_INBATCH || p.layout == L_PACKED) && Tq > 0) {
    const int nq = queries_total(p);
    G = max_rows(p) / Tq;
    if (G < 1) G = 1;
    if (G > 128) G = 128;
    if (G > nq) G = nq > 0 ? nq : 1;
  }
  rows = G * Tq;
}

// Launch one configuration.  budget: dynamic shared memory per CTA (bytes) for
// the query slots and the ring; ctas_per_sm: CTAs that share an SM (TMEM is
// sized for it; every configuration stays at or under 128 registers per thread,
// the per-SMSP limit for two 7-warp CTAs).
template <int M, int NT, int MAXMT, int R, int NACC, int SMAX, int ARES>
static cudaError_t launch_cfg(const TcParams& P, const CUtensorMap& a, const BMaps& bm, cudaStream_t s,
                              int ctas_per_sm, int budget) {
  using L = Cfg<M, NT, MAXMT, R, NACC, SMAX, ARES>;
  const int sb = L::stage_bytes(P.KB);
  int S = (budget - ARES * L::aslot_bytes(P.KB)) / sb;
  if (S > SMAX) S = SMAX;
  if (S < 2) return cudaErrorNotSupported;
  const int dyn = ARES * L::aslot_bytes(P.KB) + S * sb + 1024;
  auto k = P.p.args ? tc_scan_kernel<M, NT, MAXMT, R, NACC, SMAX, ARES, true>
                    : tc_scan_kernel<M, NT, MAXMT, R, NACC, SMAX, ARES, false>;
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn)) != cudaSuccess)
    return e;
  int64_t grid = (int64_t)device_sm_count() * ctas_per_sm;
  if (grid > P.nunits) grid = P.nunits;
  if (grid < 1) grid = 1;
  k<<<(unsigned)grid, L::NTHR, dyn, s>>>(a, bm, P, S);
  return cudaGetLastError();
}

// Resident query tiles: two slots (a new query loads while the previous one is
// in use) when they leave room for three ring stages, else one slot and two
// stages, else none (every stage carries its own query K block).
template <int M, int NT, int MAXMT, int R, int NACC, int SMAX>
static cudaError_t launch_auto(const TcParams& P, const CUtensorMap& a, const BMaps& bm, cudaStream_t s,
                               int ctas_per_sm, int budget) {
  using LA = Cfg<M, NT, MAXMT, R, NACC, SMAX, 1>;
  const int ab = LA::aslot_bytes(P.KB), sb = LA::stage_bytes(P.KB);
  if (2 * ab + 3 * sb <= budget) return launch_cfg<M, NT, MAXMT, R, NACC, SMAX, 2>(P, a, bm, s, ctas_per_sm, budget);
  if (ab + 2 * sb <= budget) return launch_cfg<M, NT, MAXMT, R, NACC, SMAX, 1>(P, a, bm, s, ctas_per_sm, budget);
  return launch_cfg<M, NT, MAXMT, R, NACC, SMAX, 0>(P, a, bm, s, ctas_per_sm, budget);
}

}  // namespace tc

bool make_tmap_16(CUtensorMap* m, const void* base, uint32_t fmt, int dim, int64_t rows, int box_rows) {
  return tc::make_map(m, base, fmt, dim, rows, box_rows);
}

bool make_tmap_i8(CUtensorMap* m, const void* base, int dim, int64_t rows, int box_rows) {
  tc::EncodeTiledFn enc = tc::encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[2] = {(cuuint64_t)dim, (cuuint64_t)rows};
  cuuint64_t gstride[1] = {(cuuint64_t)dim};
  cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
  cuuint32_t estride[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), gdim, gstride, box, estride,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int read_device_error(int reset) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  if (reset) {
    int z = 0;
    e = cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int));
    if (e != cudaSuccess) return (int)e;
  }
  return v;
}

bool scan_tc_supported(int dtype, const ScanParams& p) {
  if (dtype != FMS_F16 && dtype != FMS_BF16) return false;
  if (device_cc() != 100) return false;
  if (tc::encode_fn() == nullptr) return false;
  if (p.dim <= 0 || p.dim % tc::KBLK != 0) return false;
  if (p.nq_tok <= 0 || p.nd_tok <= 0 || p.nq_tok >= INT32_MAX || p.nd_tok >= INT32_MAX) return false;
  if ((reinterpret_cast<uintptr_t>(p.Q) & 15) || (reinterpret_cast<uintptr_t>(p.D) & 15)) return false;
  if (p.Tq <= 0) return false;
  int G, rows;
  tc::plan(p, G, rows);
  return rows <= tc::max_rows(p);
}

cudaError_t launch_scan_tc(int dtype, const ScanParams& p, cudaStream_t s) {
  if (!scan_tc_supported(dtype, p)) return cudaErrorNotSupported;
  tc::TcParams P;
  P.p = p;
  int G, rows;
  tc::plan(p, G, rows);
  P.G = G;
  const int nqt = tc::queries_total(p);
  P.ngroups = (p.layout == L_INBATCH || p.layout == L_PACKED) ? (nqt + G - 1) / G : 1;
  if (p.layout == L_INBATCH)
    P.nunits = (int64_t)p.Bd * P.ngroups;
  else if (p.layout == L_PACKED)
    P.nunits = (int64_t)p.B * P.ngroups;
  else
    P.nunits = p.nunits;
  P.KB = p.dim / tc::KBLK;
  P.fmt = dtype == FMS_BF16 ? 1u : 0u;
  if (P.nunits == 0) return cudaSuccess;
  const bool rep = rows <= 32;
  const int M = rows <= 64 ? 64 : 128;
  CUtensorMap a;
  tc::BMaps bm;
  if (!tc::make_map(&a, p.Q, P.fmt, p.dim, p.nq_tok, rep ? 32 : M)) return cudaErrorNotSupported;
  if (!tc::make_map(&bm.b128, p.D, P.fmt, p.dim, p.nd_tok, 128) ||
      !tc::make_map(&bm.b64, p.D, P.fmt, p.dim, p.nd_tok, 64) ||
      !tc::make_map(&bm.b32, p.D, P.fmt, p.dim, p.nd_tok, 32) ||
      !tc::make_map(&bm.b16, p.D, P.fmt, p.dim, p.nd_tok, 16))
    return cudaErrorNotSupported;
  // Two CTAs per SM get ~100 KB of dynamic shared memory each.
  constexpr int B2 = 100 * 1024;
  if (rep)  // one 32-row query, 4 copies in a 128-row tile: a whole document per MMA chain
    return tc::launch_cfg<128, 256, 1, 4, 1, 2, 0>(P, a, bm, s, 2, B2);
  if (rows <= 64) return tc::launch_auto<64, 64, 1, 1, 4, 8>(P, a, bm, s, 2, B2);
  if (rows <= 128) return tc::launch_auto<128, 64, 1, 1, 4, 8>(P, a, bm, s, 2, B2);
  if (rows > 256)  // three resident tiles, one CTA per SM, tile-by-tile accumulator hand-off
    return tc::launch_cfg<128, 128, 3, 1, 1, 4, 1>(P, a, bm, s, 1, 200 * 1024);
  // two 128-row tiles: two CTAs per SM, one 256-column accumulator each (two
  // CTAs' issuers and epilogues per SM beat one CTA with wider 192-row chunks,
  // which would bring the stacked query once per 192 document rows but leaves
  // no accumulator for the MMAs to run ahead into)
  return tc::launch_auto<128, 128, 2, 1, 1, 12>(P, a, bm, s, 2, B2);
}

}  // namespace fms
