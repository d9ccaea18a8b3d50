// fms_internal.h -- launcher declarations shared between the kernel files and
// the C-ABI layer (fms_abi.cu).  Not part of the public ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fms {

struct ScanParams;

// Number of SMs of the current device (cached per device).
int device_sm_count();
// Compute capability major*10+minor of the current device (cached per device).
int device_cc();

// Forward scans.  dtype is an fms_dtype.
cudaError_t launch_scan_simt(int dtype, const ScanParams& p, cudaStream_t s);
// tcgen05 + TMA engine for 16-bit features.  Returns cudaErrorNotSupported when
// the shape or pointers do not meet its TMA constraints (caller falls back to
// the SIMT scan, which is also a GPU kernel).
cudaError_t launch_scan_tc(int dtype, const ScanParams& p, cudaStream_t s);
bool scan_tc_supported(int dtype, const ScanParams& p);
// Device health flag set by engine waits that timed out (0 = healthy).
int read_device_error(int reset);
// 2-D TMA map over a token matrix (dim, rows) of 16-bit elements (fmt 0 = f16,
// 1 = bf16): boxes of 64 elements x box_rows rows, 128-byte swizzle.
bool make_tmap_16(CUtensorMap* m, const void* base, uint32_t fmt, int dim, int64_t rows, int box_rows);
// The same over int8 token rows: boxes of 128 elements (128 bytes) x box_rows.
bool make_tmap_i8(CUtensorMap* m, const void* base, int dim, int64_t rows, int box_rows);
// The short-query gallery engine (fms_scan_gallery.cu): paired and candidate
// layouts with Tq <= 32, document tokens on the MMA M side.
bool scan_gallery_supported(int dtype, const ScanParams& p);
cudaError_t launch_scan_gallery(int dtype, const ScanParams& p, cudaStream_t s);
int read_gal_device_error(int reset);

cudaError_t launch_inv_counts(int dtype, const uint8_t* qmask, int Tq, int B, void* inv_n,
                              cudaStream_t s);

// Backward (all layouts share ScanParams for the geometry).
struct BwdParams;
size_t bwd_workspace_bytes(int strategy, int dtype, int64_t n_src, int64_t n_dest,
                           int64_t grad_d_numel);
cudaError_t launch_backward(int dtype, int strategy, const BwdParams& b, void* ws,
                            size_t ws_bytes, cudaStream_t s);

// Sharded candidates: list the slots of idxs (nslots) whose doc is one of this
// shard's n_local docs starting at id_lo into the workspace (shard_list_bytes),
// writing -Inf into S for every other slot; *list / *count point into it.
size_t shard_list_bytes(int64_t nslots);
cudaError_t launch_shard_compact(const int32_t* idxs, int64_t nslots, int64_t id_lo, int64_t n_local,
                                 void* ws, float* S, const int32_t** list, const int32_t** count,
                                 cudaStream_t s);

}  // namespace fms
