// fms_int8_tc.cu -- the sm_100a INT8 exhaustive index scan: every document of
// an Int8Index scored against a batch of INT8 queries with tcgen05.mma
// kind::i8 (exact int32 dot products accumulated in TMEM) and the deferred
// per-token dequantisation s = (qs_t * ds_u) * float(acc) applied in the
// epilogue (quant.jl:96-125, the formula of int8_pair_forward_host at
// quant.jl:113; the reference's GPU counterpart is the s8 WMMA kernel at
// ext/FlashMaxSimCUDAExt.jl:621-746, which has no exhaustive layout).
//
// Orientation: query tokens on the MMA M side, document tokens on N.  Every
// query owns one 32-row slot (one TMEM subpartition), so a 128-row M tile holds
// four queries and a query's Sigma_t is a butterfly over the 32 lanes of one
// warp.  All queries of a launch (up to 8 M tiles = 32 queries) stay resident
// in shared memory; the index streams through a two-stage ring once per launch,
// each stage up to 256 document rows (two 128-token documents).
//
// Warp roles (576 threads, one CTA per SM, persistent over a contiguous range
// of stages; the producer sleeps in its waits, the MMA lane spins on the
// accumulators (sleeps on the stages), every epilogue lane polls its barriers):
//   warp 0  producer: TMA loads of the document rows, plus the stage's
//           document scales and mask words written to shared memory by all 32
//           lanes (every lane arrives on the stage barrier after its stores);
//   warp 1  MMA issuer (one lane): per unit (one M tile x the documents of one
//           accumulator) a bias MMA and dim/32 MMAs of K = 32 into one of four
//           128-column TMEM accumulators (two of 256 for documents over 128
//           tokens), so up to four units are in flight;
//   warps 2-17 epilogue, four groups of four (group g drains accumulator g, one
//           warp per subpartition = per query): tcgen05.ld 32 columns at a time
//           with the next load in flight, the dequantised masked max per query
//           token, the first-valid-column rule, Sigma_t (butterfly),
//           `normalize`, one score write per (query, document).
// The exact int32 -> float conversion is folded into the accumulator: a first
// f16 MMA of each chain writes 12582912.0f (bits 0x4B400000 = 1.5 * 2^23) into
// every entry, the s32 MMAs then add the exact dot products to that bit
// pattern, so the result read as a float is 12582912 + acc exactly
// (|acc| <= 127 * 127 * dim < 2^22 for dim <= 256) and one subtraction
// recovers float(acc).  Paired f32x2 arithmetic and three-input max keep the
// epilogue at about two instructions per cell.  Every wait is bounded (error
// flag, then a clean exit freeing TMEM).
#include <cuda.h>
#include <mutex>

#include "fms_common.cuh"
#include "fms_internal.h"
#include "fms_int8.cuh"
#include "fms_quant.cuh"
#include "fms_tc_ptx.cuh"

namespace fms {

__device__ int g_i8tc_error = 0;  // set when a wait of this engine timed out

namespace i8tc {

constexpr int ROWB = 128;             // bytes per tile row: 128 int8 = one K block
constexpr int NEPI = 16;              // epilogue warps (four per SM sub-partition)
constexpr int NWARPS = 2 + NEPI;
constexpr int NTHREADS = NWARPS * 32;
constexpr int MT_MAX = 8;             // resident M tiles (4 queries each)
constexpr int NMAX = 256;             // document rows per stage (MMA N)
constexpr int STAGES = 2;
constexpr int NBUF_MAX = 4;           // TMEM accumulators (4 x 128 or 2 x 256 columns)
constexpr int DPS_MAX = 8;            // documents per stage (>= 32 rows each)
constexpr int MWS = 16;               // mask words per stage
constexpr int A_TILE = 128 * ROWB;    // one K block of one M tile
constexpr int B_STAGE_KB = NMAX * ROWB;
constexpr float MAGIC_F = 12582912.0f;  // 1.5 * 2^23, bits 0x4B400000
// f16 bias operands of the accumulator-initialising MMA: A rows (3072, 0, ...)
// and B rows (4096, 0, ...), so every entry of A * B^T is 3072 * 4096 = 12582912.0f
constexpr uint16_t BIAS_A_F16 = 0x6A00u;  // 3072 = 1.5 * 2^11
constexpr uint16_t BIAS_B_F16 = 0x6C00u;  // 4096 = 2^12
constexpr int BIAS_BYTES = 512;           // two 8-row x 32-byte tiles (K = 16 f16)

struct Params {
  const void* Qs;         // query scales (nq_total, Tq): f32 or f16
  const void* Qf;         // float queries (nq_total, Tq, dim) quantised in the prologue, or NULL
  int qf_dtype;           // FMS_F32 / FMS_F16 / FMS_BF16 of Qf
  const void* Gs;         // document scales (N, Td): f32 or f16
  const uint8_t* qmask;   // (nq_total, Tq) or NULL
  const uint8_t* dmask;   // (N, Td) or NULL
  float* S;               // (nq_total, N)
  int64_t N;
  int64_t nstages;
  int qs_f16, ds_f16;
  int Tq, Td, Tdp, dps, W;  // W: mask words per document slot
  int UW, dpu;            // accumulator width (128 or 256 columns), documents per accumulator
  int KB;                 // dim / 128
  int q0, nq;             // queries of this launch
  int MT;                 // M tiles of this launch
  int normalize;
};

__device__ __forceinline__ float ld_scale(const void* p, int f16, int64_t i) {
  return f16 ? __half2float(__ldg(static_cast<const __half*>(p) + i))
             : __ldg(static_cast<const float*>(p) + i);
}

__device__ __forceinline__ void mbar_expect_tx_only(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(ptx::smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// tcgen05.wait::ld tied to the loaded registers, so that no use of them can be
// scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
        "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
        "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
        "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
        "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// One column of this warp's lanes, loaded and waited for in one statement.
__device__ __forceinline__ uint32_t tmem_ld1_sync(uint32_t taddr) {
  uint32_t r;
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r)
      : "r"(taddr)
      : "memory");
  return r;
}

// Max of the dequantised scores of 32 columns (one thread = one query token):
// s = (qs * ds_u) * (acc_bits - 12582912), paired f32x2, three-input maxima
// into four independent running maxima (two chains of maxima would serialise
// on the max latency).
// FULL: every column valid; otherwise the mask word selects (-inf elsewhere).
// Branch-free: on this part a branch costs more than the selects it skips.
template <bool FULL>
__device__ __forceinline__ void reduce32(const uint32_t (&r)[32], uint32_t mm, const float* ds, float2 qs2,
                                         float (&mx)[4]) {
  const float2 negm = make_float2(-MAGIC_F, -MAGIC_F);
  const float4* dsp = reinterpret_cast<const float4*>(ds);
#pragma unroll
  for (int q4 = 0; q4 < 8; ++q4) {
    const float4 dv = dsp[q4];
    const float2 a0 = __fadd2_rn(make_float2(__uint_as_float(r[4 * q4]), __uint_as_float(r[4 * q4 + 1])), negm);
    const float2 a1 = __fadd2_rn(make_float2(__uint_as_float(r[4 * q4 + 2]), __uint_as_float(r[4 * q4 + 3])), negm);
    const float2 s0 = __fmul2_rn(__fmul2_rn(qs2, make_float2(dv.x, dv.y)), a0);
    const float2 s1 = __fmul2_rn(__fmul2_rn(qs2, make_float2(dv.z, dv.w)), a1);
    float& m0 = mx[2 * (q4 & 1)];
    float& m1 = mx[2 * (q4 & 1) + 1];
    if (FULL) {
      m0 = max3(m0, s0.x, s0.y);
      m1 = max3(m1, s1.x, s1.y);
    } else {
      const uint32_t b4 = mm >> (4 * q4);
      m0 = max3(m0, (b4 & 1u) ? s0.x : -INFINITY, (b4 & 2u) ? s0.y : -INFINITY);
      m1 = max3(m1, (b4 & 4u) ? s1.x : -INFINITY, (b4 & 8u) ? s1.y : -INFINITY);
    }
  }
}

// Masked max over one document slot of W 32-column groups (W compile-time, so
// the loop has no runtime bounds).  One 32-register buffer: a TMEM load
// completes in a few dozen cycles, and a second buffer would not fit the 96
// registers that 18 warps per SM leave each thread.
template <int W, bool FULL>
__device__ __forceinline__ void reduce_doc(uint32_t tcol, const uint32_t* mw, const float* ds, float2 qs2,
                                           float (&mx)[4]) {
#pragma unroll 1
  for (int w = 0; w < W; ++w) {
    uint32_t r[32];
    ptx::tmem_ld32(tcol + 32 * w, r);
    tmem_wait_ld_regs(r);
    reduce32<FULL>(r, FULL ? 0u : mw[w], ds + 32 * w, qs2, mx);
  }
}

// W: 32-column groups per document slot (Td rounded up to 32, / 32), a
// template parameter so that the epilogue's per-document loop is unrolled.
template <int W>
__global__ void __launch_bounds__(NTHREADS, 1)
i8_exhaustive_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmG,
                     Params P) {
  extern __shared__ __align__(1024) unsigned char dsm[];
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t afull_bar;
  __shared__ __align__(8) uint64_t accf_bar[NBUF_MAX];
  __shared__ __align__(8) uint64_t acce_bar[NBUF_MAX];
  __shared__ __align__(16) float ds_s[STAGES][NMAX];
  __shared__ uint32_t mw_s[STAGES][MWS];
  __shared__ int first_s[STAGES][DPS_MAX];
  __shared__ float qs_s[MT_MAX * 4][32];   // query scales of the launch (0 past Tq)
  __shared__ uint32_t qv_s[MT_MAX * 4];    // valid query tokens (bit t)
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile int abort_s;

  unsigned char* tiles = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(dsm) + 1023) & ~(uintptr_t)1023);
  unsigned char* aregion = tiles;
  unsigned char* ring = tiles + P.MT * P.KB * A_TILE;
  const int stage_bytes = P.KB * B_STAGE_KB;
  unsigned char* bias = ring + STAGES * stage_bytes;  // A tile, then B tile
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nbl = P.UW == 128 ? 2 : 1;  // log2 of the TMEM accumulators (512 / UW)

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      ptx::mbar_init(&full_bar[i], 32);            // every producer lane
      ptx::mbar_init(&empty_bar[i], 1 + NEPI);     // MMA commit + every epilogue warp
    }
    ptx::mbar_init(&afull_bar, 1);
    for (int i = 0; i < NBUF_MAX; ++i) {
      ptx::mbar_init(&accf_bar[i], 1);
      ptx::mbar_init(&acce_bar[i], 4);             // the four warps of a group
    }
    abort_s = 0;
    ptx::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    if (P.Qf == nullptr) ptx::prefetch_tmap(&tmQ);
    ptx::prefetch_tmap(&tmG);
  }
  if (warp == 2) {
    // bias tiles: 8 rows x (K 0-7 | K 8-15), 16 bytes per row and core matrix;
    // only element K = 0 of every row is nonzero
    uint16_t* bh = reinterpret_cast<uint16_t*>(bias);
    for (int e = lane; e < BIAS_BYTES / 2; e += 32) {
      const int tile = e >> 7, within = e & 127;  // 128 halves per tile
      const bool k0 = within < 64 && (within & 7) == 0;
      bh[e] = k0 ? (tile == 0 ? BIAS_A_F16 : BIAS_B_F16) : (uint16_t)0;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp >= 2) {
    // query scales and valid-token words of the launch, one warp per query
    for (int qi = warp - 2; qi < P.MT * 4; qi += NEPI) {
      bool tv = false;
      float qsv = 0.f;
      const bool real = qi < P.nq && lane < P.Tq;
      if (real) {
        const int64_t qr = (int64_t)(P.q0 + qi) * P.Tq + lane;
        tv = P.qmask == nullptr || P.qmask[qr] != 0;
        if (P.Qf == nullptr) qsv = ld_scale(P.Qs, P.qs_f16, qr);
      }
      if (P.Qf == nullptr || !real) qs_s[qi][lane] = qsv;  // fused: written by the quantiser
      const uint32_t vw = __ballot_sync(0xffffffffu, tv);
      if (lane == 0) qv_s[qi] = vw;
    }
    if (P.Qf != nullptr) {
      // Fused query quantisation (quant.jl:42-49, as the reference quantises on
      // every call, quant.jl:159): one warp per query token writes its codes
      // straight into the resident A tiles in the 128-byte swizzled layout the
      // MMA reads (16-byte chunk c of row r stored at chunk c ^ (r & 7)), and
      // its scale into qs_s.
      const int ntok = P.nq * P.Tq;
      for (int tk = warp - 2; tk < ntok; tk += NEPI) {
        const int qi = tk / P.Tq, t = tk - qi * P.Tq;
        const int row = (qi & 3) * 32 + t;
        unsigned char* tile0 = aregion + (qi >> 2) * P.KB * A_TILE + row * ROWB;
        auto emit = [&](int k, int8_t c) {
          const int kb = k >> 7, b = k & 127;
          tile0[kb * A_TILE + ((((b >> 4) ^ (row & 7)) << 4) | (b & 15))] = (unsigned char)c;
        };
        const int64_t off = ((int64_t)(P.q0 + qi) * P.Tq + t) * P.KB * 128;
        float sc;
        if (P.qf_dtype == FMS_F16)
          sc = quantize_token<__half>(static_cast<const __half*>(P.Qf) + off, P.KB * 128, lane, emit);
        else if (P.qf_dtype == FMS_BF16)
          sc = quantize_token<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(P.Qf) + off, P.KB * 128,
                                             lane, emit);
        else
          sc = quantize_token<float>(static_cast<const float*>(P.Qf) + off, P.KB * 128, lane, emit);
        if (lane == 0) qs_s[qi][t] = sc;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> MMA reads
    }
  }
  if (warp == 1) ptx::tmem_alloc(&tmem_base_s, 512);
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;
  const int64_t st_begin = P.nstages * blockIdx.x / gridDim.x;
  const int64_t my_st = P.nstages * (blockIdx.x + 1) / gridDim.x - st_begin;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      if (P.Qf != nullptr) {
        ptx::mbar_arrive(&afull_bar);  // the prologue wrote the tiles before the block barrier
      } else {
        // resident queries: query qi -> rows [32 (qi % 4), +32) of M tile qi / 4
        ptx::mbar_expect_tx(&afull_bar, (uint32_t)(P.nq * P.KB * 32 * ROWB));
        for (int qi = 0; qi < P.nq; ++qi)
          for (int kb = 0; kb < P.KB; ++kb)
            ptx::tma_load_2d(aregion + ((qi >> 2) * P.KB + kb) * A_TILE + (qi & 3) * 32 * ROWB, &tmQ,
                             kb * 128, (P.q0 + qi) * P.Tq, &afull_bar);
      }
    }
    __syncwarp();
    for (int64_t i = 0; i < my_st; ++i) {
      const int s = (int)(i & (STAGES - 1));
      const uint32_t ph = (uint32_t)((i / STAGES) & 1);
      if (!ptx::warp_wait<true>(&empty_bar[s], ph ^ 1, &abort_s)) goto done;
      const int64_t j0 = (st_begin + i) * P.dps;
      int ndoc = P.dps;
      if (j0 + ndoc > P.N) ndoc = (int)(P.N - j0);
      unsigned char* st = ring + s * stage_bytes;
      if (lane == 0) {
        mbar_expect_tx_only(&full_bar[s], (uint32_t)(ndoc * P.KB * P.Tdp * ROWB));
        for (int d = 0; d < ndoc; ++d)
          for (int kb = 0; kb < P.KB; ++kb)
            ptx::tma_load_2d(st + kb * B_STAGE_KB + d * P.Tdp * ROWB, &tmG, kb * 128,
                             (int)((j0 + d) * P.Td), &full_bar[s]);
      }
      // scales, mask words and first valid column of every document slot
      for (int d = 0; d < P.dps; ++d) {
        const int64_t j = j0 + d;
        int first = -2;  // -2: no document in this slot
        if (d < ndoc) {
          for (int c = lane; c < P.Tdp; c += 32)
            ds_s[s][d * P.Tdp + c] = c < P.Td ? ld_scale(P.Gs, P.ds_f16, j * P.Td + c) : 0.f;
          first = -1;
#pragma unroll 1
          for (int w = 0; w < W; ++w) {
            const int c = 32 * w + lane;
            const bool ok = c < P.Td && (P.dmask == nullptr || P.dmask[j * P.Td + c] != 0);
            const uint32_t word = __ballot_sync(0xffffffffu, ok);
            if (lane == 0) mw_s[s][d * W + w] = word;
            if (first < 0 && word != 0u) first = 32 * w + __ffs(word) - 1;
          }
        }
        if (lane == 0) first_s[s][d] = first;
      }
      ptx::mbar_arrive(&full_bar[s]);  // each lane, after its own stores
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // One unit = one M tile x the documents of one accumulator (UW columns).
    // Lane 0 alone runs this role (no per-unit warp synchronisation).
    if (lane == 0) {
      if (!ptx::mbar_wait(&afull_bar, 0, &abort_s)) goto mma_out;
      ptx::tc_fence_after();
      const uint64_t abias = ptx::plain_desc(ptx::smem_u32(bias), 128, 0);
      const uint64_t bbias = ptx::plain_desc(ptx::smem_u32(bias + BIAS_BYTES / 2), 128, 0);
      uint32_t c = 0;  // units so far
      for (int64_t i = 0; i < my_st; ++i) {
        const int s = (int)(i & (STAGES - 1));
        const uint32_t ph = (uint32_t)((i / STAGES) & 1);
        if (!ptx::mbar_wait<true>(&full_bar[s], ph, &abort_s)) goto mma_out;
        ptx::tc_fence_after();
        const int64_t j0 = (st_begin + i) * P.dps;
        int ndoc = P.dps;
        if (j0 + ndoc > P.N) ndoc = (int)(P.N - j0);
        const int nunit = (ndoc + P.dpu - 1) / P.dpu;
        const uint32_t sB = ptx::smem_u32(ring + s * stage_bytes);
        for (int mt = 0; mt < P.MT; ++mt) {
          const uint64_t adesc0 = ptx::sw128_desc(ptx::smem_u32(aregion + mt * P.KB * A_TILE));
          for (int u = 0; u < nunit; ++u, ++c) {
            const uint32_t b = c & ((1u << nbl) - 1u);
            const uint32_t use = c >> nbl;
            const int nd = min(P.dpu, ndoc - u * P.dpu);
            const int n = nd * P.Tdp;  // MMA N: a multiple of 32, at most UW
            // the first use of each buffer passes at once (parity of the phase before)
            if (!ptx::mbar_wait(&acce_bar[b], (use & 1u) ^ 1u, &abort_s)) goto mma_out;
            ptx::tc_fence_after();
            const uint32_t d = tmem_base + b * (uint32_t)P.UW;
            // every accumulator entry <- 12582912.0f (bits 0x4B400000), then the
            // s32 MMAs add the exact dot products to that bit pattern
            ptx::mma_f16(d, abias, bbias, ptx::idesc_f16(0u, 128, n), 0u);
            const uint32_t idesc = ptx::idesc_i8(128, n);
            const uint64_t bdesc0 = ptx::sw128_desc(sB + u * P.dpu * P.Tdp * ROWB);
            for (int kb = 0; kb < P.KB; ++kb) {
              const uint64_t adesc = adesc0 + (uint64_t)((kb * A_TILE) >> 4);
              const uint64_t bdesc = bdesc0 + (uint64_t)((kb * B_STAGE_KB) >> 4);
#pragma unroll
              for (int k = 0; k < 4; ++k) ptx::mma_i8(d, adesc + 2 * k, bdesc + 2 * k, idesc, 1u);
            }
            ptx::mma_commit(&accf_bar[b]);
          }
        }
        ptx::mma_commit(&empty_bar[s]);
      }
    }
  mma_out:
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // warp e = warp - 2: group g = e / 4 drains accumulator g (groups beyond
    // the accumulator count only follow the stages); warp % 4 is the TMEM
    // subpartition it may read, i.e. the query of the M tile.
    const int g = (warp - 2) >> 2;
    const int sp = warp & 3;
    const uint32_t tacc = tmem_base + ((uint32_t)(sp * 32) << 16) + (uint32_t)(g * P.UW);
    uint32_t c = 0;  // units of the stages before this one (all groups)
    for (int64_t i = 0; i < my_st; ++i) {
      const int s = (int)(i & (STAGES - 1));
      const uint32_t ph = (uint32_t)((i / STAGES) & 1);
      if (!ptx::all_wait(&full_bar[s], ph, &abort_s)) goto done;
      const int64_t j0 = (st_begin + i) * P.dps;
      int ndoc = P.dps;
      if (j0 + ndoc > P.N) ndoc = (int)(P.N - j0);
      const int nunit = (ndoc + P.dpu - 1) / P.dpu;
      const uint32_t nus = (uint32_t)(P.MT * nunit);  // units of this stage, (M tile, unit) order
      // this group's units: unit c + k goes to accumulator (c + k) mod 2^nbl
      // (groups beyond the accumulator count take none)
      const uint32_t k0 = g < (1 << nbl) ? (((uint32_t)g - c) & ((1u << nbl) - 1u)) : nus;
      for (uint32_t k = k0; k < nus; k += 1u << nbl) {
        const int mt = nunit == 2 ? (int)(k >> 1) : (int)(k / (uint32_t)nunit);
        const int u = (int)k - mt * nunit;
        const int qi = mt * 4 + sp;  // query of this warp within the launch
        const uint32_t use = (c + k) >> nbl;
        if (!ptx::all_wait(&accf_bar[g], use & 1u, &abort_s)) goto done;
        ptx::tc_fence_after();
        const float qsv = qs_s[qi][lane];
        const uint32_t qv = qv_s[qi];
        const bool tv = (qv >> lane) & 1u;
        const float2 qs2 = make_float2(qsv, qsv);
        const int d1 = min((u + 1) * P.dpu, ndoc);
        for (int d = u * P.dpu; d < d1; ++d) {
          const int first = first_s[s][d];
          const int cbase = (d - u * P.dpu) * P.Tdp;  // column within the accumulator
          const int sbase = d * P.Tdp;                // column within the stage
          float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
          // one warp-uniform test per document: all its columns valid?
          const uint32_t* mwd = &mw_s[s][d * W];
          bool full = true;
#pragma unroll
          for (int w = 0; w < W; ++w) full = full && mwd[w] == 0xffffffffu;
          if (full) reduce_doc<W, true>(tacc + cbase, mwd, &ds_s[s][sbase], qs2, mx4);
          else reduce_doc<W, false>(tacc + cbase, mwd, &ds_s[s][sbase], qs2, mx4);
          const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
          float v = 0.f;
          if (first >= 0) {
            // the first valid column is taken unconditionally (a NaN there sticks);
            // every later column replaces it only when strictly greater.  With
            // float(acc) finite, that score is NaN only if qs * ds is not finite,
            // so the accumulator is read back only then.
            v = mx;
            const float pf = qsv * ds_s[s][sbase + first];
            if (__any_sync(0xffffffffu, !isfinite(pf))) {  // warp-uniform: the load is .sync.aligned
              const uint32_t r0 = tmem_ld1_sync(tacc + cbase + first);
              const float sf = pf * (__uint_as_float(r0) - MAGIC_F);
              if (sf != sf) v = sf;
            }
          }
          float sum = (tv && first >= 0) ? v : 0.f;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
          if (lane == 0 && qi < P.nq) {
            if (P.normalize) {
              const int nvalid = __popc(qv);
              sum = sum * (1.0f / (float)(nvalid > 1 ? nvalid : 1));
            }
            P.S[(int64_t)(P.q0 + qi) * P.N + j0 + d] = sum;
          }
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&acce_bar[g]);
      }
      c += nus;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&empty_bar[s]);
    }
  }
done:
  if (abort_s && threadIdx.x == 0) {
    atomicExch(&g_i8tc_error, 1);
    const uint64_t t0 = ptx::globaltimer_ns();
    while (ptx::globaltimer_ns() - t0 < 50000ull) {
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, 512);
  }
}

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

// 2-D map over int8 token rows (dim, rows): box 128 x box_rows, 128-byte swizzle.
static bool make_map_i8(CUtensorMap* m, const void* base, int dim, int64_t rows, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[2] = {(cuuint64_t)dim, (cuuint64_t)rows};
  cuuint64_t gstride[1] = {(cuuint64_t)dim};
  cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
  cuuint32_t estride[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), gdim, gstride, box, estride,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr int SMEM_BUDGET = 216 * 1024;  // dynamic shared memory per CTA (one CTA per SM; + 7 KB static)

static int max_mtiles(int KB) {
  const int ring = STAGES * KB * B_STAGE_KB;
  const int mt = (SMEM_BUDGET - 1024 - BIAS_BYTES - ring) / (KB * A_TILE);
  return mt > MT_MAX ? MT_MAX : mt;
}

}  // namespace i8tc

bool int8_exhaustive_tc_supported(const Int8ScanParams& p) {
  using namespace i8tc;
  if (device_cc() != 100 || encode_fn() == nullptr) return false;
  if (!p.exhaustive || p.args != nullptr) return false;
  if (p.dim <= 0 || p.dim % 128 != 0 || p.dim > 256) return false;  // |acc| < 2^22 needs dim <= 256
  if (p.Tq < 1 || p.Tq > 32 || p.Td < 1 || p.Td > NMAX) return false;
  if (p.N < 1 || p.N * (int64_t)p.Td >= INT32_MAX) return false;
  const int64_t nq = p.nunits / p.N;
  if (nq < 1 || nq * (int64_t)p.Tq >= INT32_MAX) return false;
  if ((reinterpret_cast<uintptr_t>(p.Qc) & 15) || (reinterpret_cast<uintptr_t>(p.Dc) & 15)) return false;
  return max_mtiles(p.dim / 128) >= 1;
}

cudaError_t launch_int8_exhaustive_tc(const Int8ScanParams& p, cudaStream_t s) {
  using namespace i8tc;
  if (!int8_exhaustive_tc_supported(p)) return cudaErrorNotSupported;
  const int nq_total = (int)(p.nunits / p.N);
  Params P;
  P.Qs = p.Qs; P.Gs = p.Ds; P.qmask = p.qmask; P.dmask = p.dmask; P.S = p.scores;
  P.Qf = p.Qf; P.qf_dtype = p.qf_dtype;
  P.N = p.N;
  P.qs_f16 = p.qs_dtype == FMS_F16; P.ds_f16 = p.ds_dtype == FMS_F16;
  P.Tq = p.Tq; P.Td = p.Td;
  P.Tdp = (p.Td + 31) & ~31;  // document slot: whole 32-column groups
  P.dps = NMAX / P.Tdp;
  if (P.dps > DPS_MAX) P.dps = DPS_MAX;
  P.W = (P.Tdp + 31) / 32;
  P.UW = P.Tdp <= 128 ? 128 : 256;
  P.dpu = P.UW / P.Tdp;
  P.KB = p.dim / 128;
  P.nstages = (p.N + P.dps - 1) / P.dps;
  P.normalize = p.normalize;
  CUtensorMap tq, tg;
  memset(&tq, 0, sizeof(tq));  // unused when the queries are quantised in the prologue
  if (p.Qf == nullptr && !make_map_i8(&tq, p.Qc, p.dim, (int64_t)nq_total * p.Tq, 32))
    return cudaErrorNotSupported;
  if (!make_map_i8(&tg, p.Dc, p.dim, p.N * (int64_t)p.Td, P.Tdp)) return cudaErrorNotSupported;
  const int mt_max = max_mtiles(P.KB);
  const int qpp = 4 * mt_max;  // queries per pass over the index
  int64_t grid = device_sm_count();
  if (grid > P.nstages) grid = P.nstages;
  for (int q0 = 0; q0 < nq_total; q0 += qpp) {
    P.q0 = q0;
    P.nq = nq_total - q0 < qpp ? nq_total - q0 : qpp;
    P.MT = (P.nq + 3) / 4;
    // the whole budget, whatever this pass needs: one CTA per SM, so that the
    // 512-column TMEM allocation never waits for a co-resident CTA
    const int dyn = SMEM_BUDGET;
    void (*k)(const CUtensorMap, const CUtensorMap, Params) = nullptr;
    switch (P.W) {
      case 1: k = i8_exhaustive_kernel<1>; break;
      case 2: k = i8_exhaustive_kernel<2>; break;
      case 3: k = i8_exhaustive_kernel<3>; break;
      case 4: k = i8_exhaustive_kernel<4>; break;
      case 5: k = i8_exhaustive_kernel<5>; break;
      case 6: k = i8_exhaustive_kernel<6>; break;
      case 7: k = i8_exhaustive_kernel<7>; break;
      case 8: k = i8_exhaustive_kernel<8>; break;
      default: return cudaErrorNotSupported;
    }
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
    if (e != cudaSuccess) return e;
    k<<<(unsigned)grid, NTHREADS, dyn, s>>>(tq, tg, P);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

int read_i8tc_device_error(int reset) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_i8tc_error, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  if (reset) {
    int z = 0;
    e = cudaMemcpyToSymbol(g_i8tc_error, &z, sizeof(int));
    if (e != cudaSuccess) return (int)e;
  }
  return v;
}

}  // namespace fms
