// fms_int8.cuh -- INT8 scan parameters and launchers (internal).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace fms {

struct Int8ScanParams {
  const int8_t* Qc;       // (dim, Tq, nq|B)
  const void* Qs;         // (Tq, nq|B) scales, f32 or f16
  const int8_t* Dc;       // (dim, Td, N|B)
  const void* Ds;         // (Td, N|B)
  const uint8_t* qmask;   // (Tq, nq|B) or NULL
  const uint8_t* dmask;   // (Td, N|B) or NULL
  int qs_dtype, ds_dtype;
  int dim, Tq, Td;
  int exhaustive;         // 0: paired units (doc b with query b); 1: all docs x all queries
  int64_t N;              // docs in the index (exhaustive)
  int64_t nunits;
  int normalize;
  float* scores;          // paired (B,), exhaustive (N, nq)
  int32_t* args;          // (Tq, units) or NULL
  const void* Qf;         // exhaustive tensor-core scan only: float queries quantised
  int qf_dtype;           //   in its prologue instead of Qc / Qs (NULL = use Qc / Qs)
};

cudaError_t launch_quantize(int dtype, const void* x, int dim, int64_t ntok, int8_t* codes,
                            void* scales, cudaStream_t s);
cudaError_t launch_int8_scan(const Int8ScanParams& p, cudaStream_t s);
// tcgen05 kind::i8 engine for the exhaustive layout (fms_int8_tc.cu).  Returns
// cudaErrorNotSupported for shapes it does not take (dim not a multiple of 128
// or above 256, Tq > 32, Td > 256, unaligned codes, no tape); the caller then
// runs the SIMT scan, which is also a GPU kernel.
bool int8_exhaustive_tc_supported(const Int8ScanParams& p);
// The short-query gallery engine's INT8 kind for the paired layout (pair is B = 1):
// Tq <= 32, dim 128 or 256, codes 16-byte aligned (fms_scan_gallery.cu).
bool int8_paired_tc_supported(const Int8ScanParams& p);
cudaError_t launch_int8_paired_tc(const Int8ScanParams& p, cudaStream_t s);
cudaError_t launch_int8_exhaustive_tc(const Int8ScanParams& p, cudaStream_t s);
int read_i8tc_device_error(int reset);
size_t topk_workspace_bytes(int nq, int64_t N, int k);
cudaError_t launch_topk(const float* S, int64_t N, int nq, int k, int64_t id_offset, void* ws,
                        float* vals, int32_t* ids, cudaStream_t s);
cudaError_t launch_topk_merge(const float* vals, const int32_t* ids, int k, int nq, int nshard,
                              float* ov, int32_t* oi, cudaStream_t s);
cudaError_t launch_cand_neg(const int32_t* idxs, int64_t N, int64_t n, float neg, float* S,
                            cudaStream_t s);

}  // namespace fms
