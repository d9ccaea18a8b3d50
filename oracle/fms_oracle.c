/*
 * fms_oracle.c -- CPU restatement of FlashMaxSim.jl's host (`Array`) path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA library: only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may
 * load it.  The product path (libflashmaxsim_sm100.so) never links or calls it.
 *
 * Parity pinning: FlashMaxSim.jl is pure Julia and Julia is not installed, so the
 * reference cannot be run here.  This restatement is pinned against the
 * reference's seed-independent known-answer tests (tests/test_oracle_pins.py
 * ports each one, with the reference file:line it comes from) and against an
 * independent float64 dense restatement (maxsim_dense, dense.jl:26-109) on
 * seeded inputs.  Parity is therefore "pinned to known answers", not to
 * reference-generated vectors.
 *
 * Conventions (identical to the reference's Julia column-major arrays):
 *   q (dim,Tq) -> q[k + dim*t];  Q (dim,Tq,B) -> Q[k + dim*(t + Tq*b)]
 *   masks are 1-byte Bool, args / idxs / cu are Int32 and 1-based (0 = none).
 * Feature inputs arrive already widened to the accumulate type (f32 or f64); the
 * Python wrapper widens f16/bf16 exactly, which is what `dot_accum(Float16) =
 * Float32` does in the reference (kernels_forward.jl:16-17, forward_pair.jl:25-39).
 *
 * Inner products are formed per 64-token document tile (DOC_TILE,
 * forward_pair.jl:12) as a GEMM whose k-sum runs in order; the reference hands
 * that GEMM to BLAS (`mul!`, forward_pair.jl:79), whose summation order is
 * unspecified, so results match the reference to rounding, not bit for bit.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define DOC_TILE 64

/* ------------------------------------------------------------------------- */
/* Pair scan (forward_pair.jl:59-95, pair_forward_host!)                      */
/* ------------------------------------------------------------------------- */

/* Generic over accumulate type via macro so f32 and f64 share one text. */
#define DEFINE_PAIR(SUF, A)                                                        \
static void pair_scan_##SUF(const A* q, const A* d, const uint8_t* qmask,          \
                            const uint8_t* dmask, int dim, int Tq, int Td,         \
                            A* mx, int32_t* arg, A* qT, A* Stile)                   \
{                                                                                  \
    for (int t = 0; t < Tq; ++t) { mx[t] = (A)0; arg[t] = 0; }                    \
    /* qT[k*Tq + t] = q[k + dim*t]: lets the tile GEMM run over t innermost */   \
    for (int t = 0; t < Tq; ++t)                                                   \
        for (int k = 0; k < dim; ++k) qT[(int64_t)k * Tq + t] = q[(int64_t)k + (int64_t)dim * t]; \
    for (int u = 0; u < Td; u += DOC_TILE) {                                       \
        int w = (Td - u < DOC_TILE) ? Td - u : DOC_TILE;                           \
        /* Stile[uu][t] = sum_k d[k, u+uu] * q[k, t]   (mul!, forward_pair.jl:79) */ \
        for (int uu = 0; uu < w; ++uu) {                                           \
            A* srow = Stile + (int64_t)uu * Tq;                                    \
            for (int t = 0; t < Tq; ++t) srow[t] = (A)0;                           \
            const A* dc = d + (int64_t)dim * (u + uu);                             \
            for (int k = 0; k < dim; ++k) {                                        \
                const A dk = dc[k];                                                \
                const A* qk = qT + (int64_t)k * Tq;                                \
                for (int t = 0; t < Tq; ++t) srow[t] += dk * qk[t];                \
            }                                                                      \
        }                                                                          \
        /* scan: first valid wins, strict > (forward_pair.jl:80-91) */             \
        for (int t = 0; t < Tq; ++t) {                                             \
            if (qmask && !qmask[t]) continue;                                      \
            for (int uu = 0; uu < w; ++uu) {                                       \
                if (dmask && !dmask[u + uu]) continue;                             \
                A s = Stile[(int64_t)uu * Tq + t];                                 \
                if (arg[t] == 0 || s > mx[t]) { mx[t] = s; arg[t] = u + uu + 1; }  \
            }                                                                      \
        }                                                                          \
    }                                                                              \
}                                                                                  \
static A pair_sum_##SUF(const uint8_t* qmask, int Tq, const A* mx, const int32_t* arg) \
{                                                                                  \
    /* forward_pair.jl:92-95: sum in t order over valid tokens with arg > 0 */    \
    A score = (A)0;                                                                \
    for (int t = 0; t < Tq; ++t)                                                   \
        if ((!qmask || qmask[t]) && arg[t] > 0) score += mx[t];                    \
    return score;                                                                  \
}

DEFINE_PAIR(f32, float)
DEFINE_PAIR(f64, double)

static int count_true(const uint8_t* m, int n)
{
    int c = 0;
    if (!m) return n;
    for (int i = 0; i < n; ++i) c += m[i] ? 1 : 0;
    return c;
}

/* One macro instantiates every forward layout for an accumulate type A. */
#define DEFINE_LAYOUTS(SUF, A)                                                     \
/* pair: maxsim(q,d,qmask,dmask) = pair_forward + pair_finalize                  \
   (dispatch.jl:46-56, forward_pair.jl:153-173).  normalize multiplies by        \
   one(T)/T(query_count) (forward_pair.jl:156-159). */                           \
A fmso_pair_##SUF(const A* q, const A* d, const uint8_t* qmask,                    \
                  const uint8_t* dmask, int dim, int Tq, int Td, int normalize,    \
                  int32_t* args)                                                   \
{                                                                                  \
    A* mx = (A*)malloc(sizeof(A) * (Tq > 0 ? Tq : 1));                             \
    A* qT = (A*)malloc(sizeof(A) * ((int64_t)dim * Tq + 1));                       \
    A* St = (A*)malloc(sizeof(A) * ((int64_t)DOC_TILE * Tq + 1));                  \
    pair_scan_##SUF(q, d, qmask, dmask, dim, Tq, Td, mx, args, qT, St);            \
    A s = pair_sum_##SUF(qmask, Tq, mx, args);                                     \
    if (normalize) {                                                               \
        int n = count_true(qmask, Tq); if (n < 1) n = 1;                           \
        s = s * ((A)1 / (A)n);                                                     \
    }                                                                              \
    free(mx); free(qT); free(St);                                                  \
    return s;                                                                      \
}                                                                                  \
/* paired (forward_layouts.jl:86-103); normalize = length_normalize             \
   (normalize.jl:4-25): scores .* (1 ./ max.(n,1)). nthreads>1 runs pairs in      \
   parallel (a labelled speed-up of the same per-pair loop). */                   \
void fmso_paired_##SUF(const A* Q, const A* D, const uint8_t* qmask,               \
                       const uint8_t* dmask, int dim, int Tq, int Td, int B,       \
                       int normalize, A* scores, int32_t* args, int nthreads)      \
{                                                                                  \
    _Pragma("omp parallel for schedule(dynamic,1) num_threads(nthreads) if(nthreads > 1)") \
    for (int b = 0; b < B; ++b) {                                                  \
        const uint8_t* qm = qmask ? qmask + (int64_t)Tq * b : NULL;                \
        const uint8_t* dm = dmask ? dmask + (int64_t)Td * b : NULL;                \
        scores[b] = fmso_pair_##SUF(Q + (int64_t)dim * Tq * b, D + (int64_t)dim * Td * b, \
                                    qm, dm, dim, Tq, Td, normalize, args + (int64_t)Tq * b); \
    }                                                                              \
}                                                                                  \
/* candidates (forward_layouts.jl:239-261): S prefilled with neg; invalid idx   \
   keeps neg and zero args.  normalize = length_normalize_candidates            \
   (normalize.jl:37-46): valid slots scaled, invalid slots stay neg. */          \
void fmso_candidates_##SUF(const A* Q, const A* G, const int32_t* idxs,            \
                           const uint8_t* qmask, const uint8_t* dmask, int dim,    \
                           int Tq, int B, int Td, int N, int C, A neg,             \
                           int normalize, A* S, int32_t* args, int nthreads)       \
{                                                                                  \
    _Pragma("omp parallel for schedule(dynamic,4) num_threads(nthreads) if(nthreads > 1)") \
    for (int64_t cb = 0; cb < (int64_t)C * B; ++cb) {                              \
        int b = (int)(cb / C);                                                     \
        int32_t j = idxs[cb];                                                      \
        int32_t* a = args + cb * Tq;                                               \
        if (!(j >= 1 && j <= N)) {                                                 \
            S[cb] = neg;                                                           \
            for (int t = 0; t < Tq; ++t) a[t] = 0;                                 \
            continue;                                                              \
        }                                                                          \
        const uint8_t* qm = qmask ? qmask + (int64_t)Tq * b : NULL;                \
        const uint8_t* dm = dmask ? dmask + (int64_t)Td * (j - 1) : NULL;          \
        S[cb] = fmso_pair_##SUF(Q + (int64_t)dim * Tq * b, G + (int64_t)dim * Td * (j - 1), \
                                qm, dm, dim, Tq, Td, normalize, a);                \
    }                                                                              \
}                                                                                  \
/* in-batch (forward_layouts.jl:155-179 + inbatch_accumulate_host! :49-74):      \
   S[j,i] = MaxSim(Q_i, D_j) -> S[j + Bd*i]; args (Tq,Bd,Bq). */                  \
void fmso_inbatch_##SUF(const A* Q, const A* D, const uint8_t* qmask,              \
                        const uint8_t* dmask, int dim, int Tq, int Bq, int Td,     \
                        int Bd, int normalize, A* S, int32_t* args, int nthreads)  \
{                                                                                  \
    _Pragma("omp parallel for schedule(dynamic,4) num_threads(nthreads) if(nthreads > 1)") \
    for (int64_t ji = 0; ji < (int64_t)Bd * Bq; ++ji) {                            \
        int j = (int)(ji % Bd), i = (int)(ji / Bd);                                \
        const uint8_t* qm = qmask ? qmask + (int64_t)Tq * i : NULL;                \
        const uint8_t* dm = dmask ? dmask + (int64_t)Td * j : NULL;                \
        S[ji] = fmso_pair_##SUF(Q + (int64_t)dim * Tq * i, D + (int64_t)dim * Td * j, \
                                qm, dm, dim, Tq, Td, normalize, args + ji * Tq);   \
    }                                                                              \
}                                                                                  \
/* packed, nq queries stacked (packed.jl:153-176 per query; the multi-query     \
   form is hcat of per-query calls): S (B,nq), args (Tq,B,nq).  The reference   \
   passes an all-true dmask of the doc length (packed.jl:161,171). */           \
void fmso_packed_##SUF(const A* Qs, const A* tokens, const int32_t* cu,            \
                       const uint8_t* qmask, int dim, int Tq, int nq, int B,       \
                       int normalize, A* S, int32_t* args, int nthreads)           \
{                                                                                  \
    _Pragma("omp parallel for schedule(dynamic,4) num_threads(nthreads) if(nthreads > 1)") \
    for (int64_t bq = 0; bq < (int64_t)B * nq; ++bq) {                             \
        int b = (int)(bq % B), qi = (int)(bq / B);                                 \
        int a0 = cu[b] - 1, z = cu[b + 1] - 1;                                     \
        int Td = z - a0; if (Td < 0) Td = 0;                                       \
        const uint8_t* qm = qmask ? qmask + (int64_t)Tq * qi : NULL;               \
        S[bq] = fmso_pair_##SUF(Qs + (int64_t)dim * Tq * qi, tokens + (int64_t)dim * a0, \
                                qm, NULL, dim, Tq, Td, normalize, args + bq * Tq); \
    }                                                                              \
}                                                                                  \
/* varlen pairs (packed.jl:236-260): args (max_q, N), rows t >= Tq_n stay 0.     \
   normalize: inv_n[n] = 1/max(Tq_n,1) (kernels_packed.jl:277-282). */            \
void fmso_varlen_##SUF(const A* Qp, const A* Dp, const int32_t* cu_q,              \
                       const int32_t* cu_d, int dim, int N, int max_q,             \
                       int normalize, A* S, int32_t* args, int nthreads)           \
{                                                                                  \
    _Pragma("omp parallel for schedule(dynamic,4) num_threads(nthreads) if(nthreads > 1)") \
    for (int n = 0; n < N; ++n) {                                                  \
        int qa = cu_q[n] - 1, Tq = cu_q[n + 1] - cu_q[n];                          \
        int da = cu_d[n] - 1, Td = cu_d[n + 1] - cu_d[n];                          \
        if (Td < 0) Td = 0;                                                        \
        int32_t* a = args + (int64_t)n * max_q;                                    \
        for (int t = 0; t < max_q; ++t) a[t] = 0;                                  \
        S[n] = fmso_pair_##SUF(Qp + (int64_t)dim * qa, Dp + (int64_t)dim * da,     \
                               NULL, NULL, dim, Tq, Td, normalize, a);             \
    }                                                                              \
}

DEFINE_LAYOUTS(f32, float)
DEFINE_LAYOUTS(f64, double)

/* ------------------------------------------------------------------------- */
/* Dense oracle in float64 (dense.jl:26-56): materialises S = d'q, same       */
/* first-valid-wins max.  Used to pin the tiled scan above.                   */
/* ------------------------------------------------------------------------- */
double fmso_dense_pair_f64(const double* q, const double* d, const uint8_t* qmask,
                           const uint8_t* dmask, int dim, int Tq, int Td, int normalize)
{
    double score = 0.0;
    int nq = 0;
    for (int t = 0; t < Tq; ++t) {
        if (qmask && !qmask[t]) continue;
        double mx = 0.0;
        int hit = 0;
        for (int u = 0; u < Td; ++u) {
            if (dmask && !dmask[u]) continue;
            double s = 0.0;
            for (int k = 0; k < dim; ++k) s += d[(int64_t)dim * u + k] * q[(int64_t)dim * t + k];
            if (!hit || s > mx) { mx = s; hit = 1; }
        }
        if (!hit) continue;
        score += mx;
        nq += 1;
    }
    return normalize ? score / (double)(nq > 1 ? nq : 1) : score;
}

/* ------------------------------------------------------------------------- */
/* INT8 (quant.jl)                                                            */
/* ------------------------------------------------------------------------- */

/* IEEE binary16 / bfloat16 round-to-nearest-even from float32.  Used to
   restate Julia's Float16 / BFloat16 arithmetic, which computes each op in
   Float32 and rounds the result back (exact for + - * / at these widths). */
static uint16_t f32_to_f16_bits(float f)
{
    uint32_t x; memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) {                       /* inf or nan */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 -> inf */
    if (ax < 0x38800000u) {                        /* below min normal 2^-14 */
        if (ax < 0x33000000u) return (uint16_t)sign;  /* < 2^-25 -> 0 (ties at 2^-25 go to 0) */
        uint32_t e = ax >> 23;                      /* biased f32 exponent */
        uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        /* value = m * 2^(e-150); count of f16 subnormal units (2^-24) = m >> (126-e) */
        int sh = 126 - (int)e;                     /* 14..24 */
        uint32_t r = m >> sh;
        uint32_t rem = m & ((1u << sh) - 1u);
        uint32_t half = 1u << (sh - 1);
        if (rem > half || (rem == half && (r & 1u))) r += 1;
        return (uint16_t)(sign | r);
    }
    uint32_t r = ((ax - 0x38000000u) >> 13);       /* rebias 127->15, drop 13 bits */
    uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r += 1;
    return (uint16_t)(sign | r);
}

static float f16_bits_to_f32(uint16_t h)
{
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) x = sign;
        else {                                      /* subnormal */
            float v = ldexpf((float)m, -24);
            memcpy(&x, &v, 4);
            x |= sign;
        }
    } else if (e == 31) x = sign | 0x7f800000u | (m << 13);
    else x = sign | ((e + 112u) << 23) | (m << 13);
    float f; memcpy(&f, &x, 4);
    return f;
}

static uint16_t f32_to_bf16_bits(float f)
{
    uint32_t x; memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
    uint32_t lsb = (x >> 16) & 1u;
    x += 0x7fffu + lsb;
    return (uint16_t)(x >> 16);
}

static float bf16_bits_to_f32(uint16_t h)
{
    uint32_t x = (uint32_t)h << 16;
    float f; memcpy(&f, &x, 4);
    return f;
}

float fmso_round_f16(float x) { return f16_bits_to_f32(f32_to_f16_bits(x)); }
float fmso_round_bf16(float x) { return bf16_bits_to_f32(f32_to_bf16_bits(x)); }

/* quantize_int8_symmetric (quant.jl:42-49), per token of x (dim, ntok).
   dtype: 0 = Float32, 1 = Float16, 2 = BFloat16.  x holds the values widened
   to float32; scales_out receives them widened too (exact).
     am     = maximum(abs, x[:,t])               (0 when dim == 0, quant.jl:27-30)
     raw    = max(am, T(1f-8)) / T(127)          (quant.jl:44; int8_scale_eps)
     scale  = max(raw, floatmin(T))              (quant.jl:45; int8_scale_floor)
     code   = round(Int8, clamp(x / scale, -127, 127))   ties to even
   Every op is rounded to T, as Julia does for Float16 / BFloat16. */
void fmso_quantize_int8(const float* x, int dtype, int dim, int64_t ntok,
                        int8_t* codes, float* scales)
{
    float (*rt)(float) = NULL;
    float eps, fmin;
    if (dtype == 1) { rt = fmso_round_f16; eps = fmso_round_f16(1e-8f); fmin = 6.103515625e-05f; }
    else if (dtype == 2) { rt = fmso_round_bf16; eps = fmso_round_bf16(1e-8f); fmin = 1.17549435e-38f; }
    else { eps = 1e-8f; fmin = 1.17549435e-38f; }
    for (int64_t t = 0; t < ntok; ++t) {
        const float* xt = x + (int64_t)dim * t;
        float am = 0.0f;                       /* maximum(abs, x[:,t]); NaN propagates */
        for (int k = 0; k < dim; ++k) {
            float a = fabsf(xt[k]);
            if (k == 0 || a > am || isnan(a)) { if (!isnan(am) || k == 0) am = a; }
        }
        float raw = (isnan(am) || am > eps ? am : eps) / 127.0f;
        if (rt) raw = rt(raw);
        float sc = raw > fmin ? raw : fmin;
        scales[t] = sc;
        for (int k = 0; k < dim; ++k) {
            float v = xt[k] / sc;
            if (rt) v = rt(v);
            if (v < -127.0f) v = -127.0f;
            if (v > 127.0f) v = 127.0f;
            if (isnan(v)) v = 0.0f;            /* Julia throws InexactError here */
            codes[(int64_t)dim * t + k] = (int8_t)nearbyintf(v);
        }
    }
}

/* int8_pair_forward_host (quant.jl:96-125): s = (qt * ds[u]) * Float32(acc),
   acc the exact Int32 dot product.  Scales arrive widened to float32. */
float fmso_int8_pair(const int8_t* qc, const float* qs, const int8_t* dc, const float* ds,
                     const uint8_t* qmask, const uint8_t* dmask, int dim, int Tq, int Td,
                     int normalize, int32_t* args, float* mx_out)
{
    float* mx = mx_out ? mx_out : (float*)malloc(sizeof(float) * (Tq > 0 ? Tq : 1));
    for (int t = 0; t < Tq; ++t) { mx[t] = 0.0f; args[t] = 0; }
    for (int t = 0; t < Tq; ++t) {
        if (qmask && !qmask[t]) continue;
        float qt = qs[t];
        const int8_t* qk = qc + (int64_t)dim * t;
        for (int u = 0; u < Td; ++u) {
            if (dmask && !dmask[u]) continue;
            const int8_t* dk = dc + (int64_t)dim * u;
            int32_t acc = 0;
            for (int k = 0; k < dim; ++k) acc += (int32_t)qk[k] * (int32_t)dk[k];
            float s = qt * ds[u] * (float)acc;
            if (args[t] == 0 || s > mx[t]) { mx[t] = s; args[t] = u + 1; }
        }
    }
    float score = 0.0f;
    for (int t = 0; t < Tq; ++t)
        if ((!qmask || qmask[t]) && args[t] > 0) score += mx[t];
    if (normalize) {
        int n = count_true(qmask, Tq); if (n < 1) n = 1;
        score = score * (1.0f / (float)n);
    }
    if (!mx_out) free(mx);
    return score;
}

/* int8_paired_forward_host (quant.jl:172-185) */
void fmso_int8_paired(const int8_t* Qc, const float* Qs, const int8_t* Dc, const float* Ds,
                      const uint8_t* qmask, const uint8_t* dmask, int dim, int Tq, int Td,
                      int B, int normalize, float* scores, int32_t* args, int nthreads)
{
    #pragma omp parallel for schedule(dynamic,1) num_threads(nthreads) if(nthreads > 1)
    for (int b = 0; b < B; ++b)
        scores[b] = fmso_int8_pair(Qc + (int64_t)dim * Tq * b, Qs + (int64_t)Tq * b,
                                   Dc + (int64_t)dim * Td * b, Ds + (int64_t)Td * b,
                                   qmask ? qmask + (int64_t)Tq * b : NULL,
                                   dmask ? dmask + (int64_t)Td * b : NULL,
                                   dim, Tq, Td, normalize, args + (int64_t)Tq * b, NULL);
}

/* Exhaustive INT8 index scan (no reference entry point: the reference has only
   pair / paired, quant.jl:96-185; a caller loops pairs).  Scores every doc of
   an index (dim,Td,N) for nq queries (dim,Tq,nq) with the pair formula above:
   S (N, nq) -> S[j + N*qi].  docs [j0, j1) only, for sampled CPU timing. */
void fmso_int8_exhaustive(const int8_t* Qc, const float* Qs, const int8_t* Gc,
                          const float* Gs, const uint8_t* qmask, const uint8_t* dmask,
                          int dim, int Tq, int nq, int Td, int64_t N, int64_t j0, int64_t j1,
                          int normalize, float* S, int nthreads)
{
    #pragma omp parallel for schedule(dynamic,16) num_threads(nthreads) if(nthreads > 1)
    for (int64_t j = j0; j < j1; ++j) {
        int32_t args[4096];
        for (int qi = 0; qi < nq; ++qi) {
            S[j + N * qi] = fmso_int8_pair(Qc + (int64_t)dim * Tq * qi, Qs + (int64_t)Tq * qi,
                                           Gc + (int64_t)dim * Td * j, Gs + (int64_t)Td * j,
                                           qmask ? qmask + (int64_t)Tq * qi : NULL,
                                           dmask ? dmask + (int64_t)Td * j : NULL,
                                           dim, Tq, Td, normalize, args, NULL);
        }
    }
}

/* ------------------------------------------------------------------------- */
/* Backward (backward_pair.jl:14-37, accumulate.jl:12-39, invgrid.jl:16-65)   */
/* Gradients are computed in float32 for every feature type: the caller      */
/* passes delta already rounded to T as the rrule does (rrule.jl:77,94).      */
/* ------------------------------------------------------------------------- */

/* build_inverse_csr (invgrid.jl:16-38): row_ptr (n_dest+1), 0-based exclusive
   ends; col_idx 1-based sources in source order; returns nnz. */
int fmso_build_inverse_csr(const int32_t* arg, int n_src, int n_dest,
                           int32_t* row_ptr, int32_t* col_idx)
{
    for (int u = 0; u <= n_dest; ++u) row_ptr[u] = 0;
    for (int s = 0; s < n_src; ++s) {
        int u = arg[s];
        if (u >= 1 && u <= n_dest) row_ptr[u] += 1;
    }
    for (int u = 0; u < n_dest; ++u) row_ptr[u + 1] += row_ptr[u];
    int nnz = row_ptr[n_dest];
    int32_t* cursor = (int32_t*)malloc(sizeof(int32_t) * (n_dest + 1));
    memcpy(cursor, row_ptr, sizeof(int32_t) * (n_dest + 1));
    for (int s = 0; s < n_src; ++s) {
        int u = arg[s];
        if (!(u >= 1 && u <= n_dest)) continue;
        cursor[u - 1] += 1;                    /* cursor[u] += 1 (1-based u) */
        col_idx[cursor[u - 1] - 1] = s + 1;
    }
    free(cursor);
    return nnz;
}

/* pair_pullback(::CPU) + accumulate_doc!(mode): dq, dd are ACCUMULATED into
   (callers zero them), matching `dQ[:,:,b] .+= dq` in the layout loops.
   mode 0 = AtomicUnified (accumulate.jl:12-29), 1 = InvGrid (accumulate.jl:32-39
   via build_inverse_csr + invgrid_accumulate_doc!, invgrid.jl:46-65). */
void fmso_pair_pullback(float delta, const float* q, const float* d, const uint8_t* qmask,
                        const int32_t* argmax, int dim, int Tq, int Td, int mode,
                        float* dq, float* dd)
{
    if (delta == 0.0f) return;                 /* backward_pair.jl:20 */
    float* dsrc = (float*)calloc(Tq > 0 ? Tq : 1, sizeof(float));
    for (int t = 0; t < Tq; ++t) {
        if (qmask && !qmask[t]) continue;
        int u = argmax[t];
        if (!(u >= 1 && u <= Td)) continue;
        dsrc[t] = delta;
        for (int k = 0; k < dim; ++k)
            dq[(int64_t)dim * t + k] += delta * d[(int64_t)dim * (u - 1) + k];
    }
    if (mode == 0) {
        for (int t = 0; t < Tq; ++t) {
            float dt = dsrc[t];
            if (dt == 0.0f) continue;
            int u = argmax[t];
            if (!(u >= 1 && u <= Td)) continue;
            for (int k = 0; k < dim; ++k)
                dd[(int64_t)dim * (u - 1) + k] += dt * q[(int64_t)dim * t + k];
        }
    } else {
        int32_t* rp = (int32_t*)malloc(sizeof(int32_t) * (Td + 1));
        int32_t* ci = (int32_t*)malloc(sizeof(int32_t) * (Tq > 0 ? Tq : 1));
        fmso_build_inverse_csr(argmax, Tq, Td, rp, ci);
        for (int u = 0; u < Td; ++u)
            for (int p = rp[u]; p < rp[u + 1]; ++p) {
                int t = ci[p] - 1;
                float dt = dsrc[t];
                if (dt == 0.0f) continue;
                for (int k = 0; k < dim; ++k)
                    dd[(int64_t)dim * u + k] += dt * q[(int64_t)dim * t + k];
            }
        free(rp); free(ci);
    }
    free(dsrc);
}

/* T-arithmetic delta = T(Delta) * inv_n_T (backward_layouts.jl:19, 79, 146). */
static float tmul(float a, float b, int dtype)
{
    float r = a * b;
    if (dtype == 1) r = fmso_round_f16(r);
    else if (dtype == 2) r = fmso_round_bf16(r);
    return r;
}

/* paired_pullback(::CPU) (backward_layouts.jl:13-26); Delta, inv_n already in T
   (widened); dtype gives T for the delta product. */
void fmso_paired_pullback(const float* Delta, const float* inv_n, const float* Q,
                          const float* D, const uint8_t* qmask, const int32_t* args,
                          int dim, int Tq, int Td, int B, int mode, int dtype,
                          float* dQ, float* dD)
{
    memset(dQ, 0, sizeof(float) * (int64_t)dim * Tq * B);
    memset(dD, 0, sizeof(float) * (int64_t)dim * Td * B);
    for (int b = 0; b < B; ++b) {
        float delta = tmul(Delta[b], inv_n ? inv_n[b] : 1.0f, dtype);
        fmso_pair_pullback(delta, Q + (int64_t)dim * Tq * b, D + (int64_t)dim * Td * b,
                           qmask ? qmask + (int64_t)Tq * b : NULL, args + (int64_t)Tq * b,
                           dim, Tq, Td, mode, dQ + (int64_t)dim * Tq * b, dD + (int64_t)dim * Td * b);
    }
}

/* inbatch_pullback(::CPU) (backward_layouts.jl:69-94): loop j outer, i inner. */
void fmso_inbatch_pullback(const float* Delta, const float* inv_n, const float* Q,
                           const float* D, const uint8_t* qmask, const int32_t* args,
                           int dim, int Tq, int Bq, int Td, int Bd, int mode, int dtype,
                           float* dQ, float* dD)
{
    memset(dQ, 0, sizeof(float) * (int64_t)dim * Tq * Bq);
    memset(dD, 0, sizeof(float) * (int64_t)dim * Td * Bd);
    for (int j = 0; j < Bd; ++j)
        for (int i = 0; i < Bq; ++i) {
            float delta = tmul(Delta[j + (int64_t)Bd * i], inv_n ? inv_n[i] : 1.0f, dtype);
            fmso_pair_pullback(delta, Q + (int64_t)dim * Tq * i, D + (int64_t)dim * Td * j,
                               qmask ? qmask + (int64_t)Tq * i : NULL,
                               args + ((int64_t)j + (int64_t)Bd * i) * Tq,
                               dim, Tq, Td, mode, dQ + (int64_t)dim * Tq * i, dD + (int64_t)dim * Td * j);
        }
}

/* candidates_pullback(::CPU) (backward_layouts.jl:137-165): b outer, c inner. */
void fmso_candidates_pullback(const float* Delta, const float* inv_n, const float* Q,
                              const float* G, const int32_t* idxs, const uint8_t* qmask,
                              const int32_t* args, int dim, int Tq, int B, int Td, int N,
                              int C, int mode, int dtype, float* dQ, float* dG)
{
    memset(dQ, 0, sizeof(float) * (int64_t)dim * Tq * B);
    memset(dG, 0, sizeof(float) * (int64_t)dim * Td * N);
    for (int b = 0; b < B; ++b)
        for (int c = 0; c < C; ++c) {
            int64_t cb = c + (int64_t)C * b;
            int j = idxs[cb];
            if (!(j >= 1 && j <= N)) continue;
            float delta = tmul(Delta[cb], inv_n ? inv_n[b] : 1.0f, dtype);
            fmso_pair_pullback(delta, Q + (int64_t)dim * Tq * b, G + (int64_t)dim * Td * (j - 1),
                               qmask ? qmask + (int64_t)Tq * b : NULL, args + cb * Tq,
                               dim, Tq, Td, mode, dQ + (int64_t)dim * Tq * b,
                               dG + (int64_t)dim * Td * (j - 1));
        }
}

/* packed_pullback(::CPU) (packed.jl:361-377), nq queries: Delta (B,nq). */
void fmso_packed_pullback(const float* Delta, const float* inv_n, const float* Qs,
                          const float* tokens, const int32_t* cu, const uint8_t* qmask,
                          const int32_t* args, int dim, int Tq, int nq, int B, int mode,
                          int dtype, float* dQ, float* dP, int64_t ntok)
{
    memset(dQ, 0, sizeof(float) * (int64_t)dim * Tq * nq);
    memset(dP, 0, sizeof(float) * (int64_t)dim * ntok);
    for (int qi = 0; qi < nq; ++qi)
        for (int b = 0; b < B; ++b) {
            int a0 = cu[b] - 1, Td = cu[b + 1] - cu[b];
            if (Td < 0) Td = 0;
            int64_t bq = b + (int64_t)B * qi;
            float delta = tmul(Delta[bq], inv_n ? inv_n[qi] : 1.0f, dtype);
            fmso_pair_pullback(delta, Qs + (int64_t)dim * Tq * qi, tokens + (int64_t)dim * a0,
                               qmask ? qmask + (int64_t)Tq * qi : NULL, args + bq * Tq,
                               dim, Tq, Td, mode, dQ + (int64_t)dim * Tq * qi, dP + (int64_t)dim * a0);
        }
}

/* varlen_pullback(::CPU) (packed.jl:424-443). */
void fmso_varlen_pullback(const float* Delta, const float* inv_n, const float* Qp,
                          const float* Dp, const int32_t* cu_q, const int32_t* cu_d,
                          const int32_t* args, int dim, int N, int max_q, int mode,
                          int dtype, float* dQ, float* dD, int64_t nq_tok, int64_t nd_tok)
{
    memset(dQ, 0, sizeof(float) * (int64_t)dim * nq_tok);
    memset(dD, 0, sizeof(float) * (int64_t)dim * nd_tok);
    for (int n = 0; n < N; ++n) {
        int qa = cu_q[n] - 1, Tq = cu_q[n + 1] - cu_q[n];
        int da = cu_d[n] - 1, Td = cu_d[n + 1] - cu_d[n];
        float delta = tmul(Delta[n], inv_n ? inv_n[n] : 1.0f, dtype);
        fmso_pair_pullback(delta, Qp + (int64_t)dim * qa, Dp + (int64_t)dim * da, NULL,
                           args + (int64_t)n * max_q, dim, Tq, Td, mode,
                           dQ + (int64_t)dim * qa, dD + (int64_t)dim * da);
    }
}

int fmso_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
