// fms_scan_tc.cu -- tcgen05 + TMA MaxSim engine for 16-bit features (placeholder
// until the engine lands: reports "not supported" so run_scan uses the CUDA-core
// scan, which is also a GPU kernel).
#include "fms_common.cuh"
#include "fms_internal.h"

namespace fms {

bool scan_tc_supported(int, const ScanParams&) { return false; }

cudaError_t launch_scan_tc(int, const ScanParams&, cudaStream_t) { return cudaErrorNotSupported; }

}  // namespace fms
