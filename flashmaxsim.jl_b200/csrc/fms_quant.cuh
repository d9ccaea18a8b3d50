// fms_quant.cuh -- quantize_int8_symmetric (quant.jl:42-49) of one token by one
// warp, shared by the quantization kernel (fms_int8.cu) and the INT8 exhaustive
// scan's fused query prologue (fms_int8_tc.cu).
//
// scale = max(max(absmax, T(1f-8)) / T(127), floatmin(T)) and
// code  = round(clamp(x / scale, -127, 127)) with ties to even, every operation
// rounded to T as Julia's Float16 / BFloat16 arithmetic does (an f32 op then
// one rounding, which is exact double rounding for these types).  A NaN
// element gives a NaN scale and code 0 (the reference throws InexactError).
#pragma once
#include "fms_common.cuh"

namespace fms {

// Lane `lane` handles elements lane, lane + 32, ...; emit(k, code) receives
// every code; returns the scale widened to the accumulate type.
template <typename T, typename Emit>
__device__ __forceinline__ typename Tr<T>::Acc quantize_token(const T* __restrict__ xt, int dim, int lane,
                                                             Emit emit) {
  using A = typename Tr<T>::Acc;
  const A eps = Tr<T>::to(Tr<T>::from((A)1e-8f));  // T(1f-8) (quant.jl:21)
  const A fmin = Tr<T>::floatmin();                // floatmin(T) (quant.jl:22)
  A am = (A)0;
  bool nan = false;
  for (int k = lane; k < dim; k += 32) {
    const A a = fabs(Tr<T>::to(xt[k]));
    if (a != a) nan = true;
    am = a > am ? a : am;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const A o = __shfl_xor_sync(0xffffffffu, am, off);
    am = o > am ? o : am;
  }
  nan = __any_sync(0xffffffffu, nan);
  if (nan) am = (A)NAN;
  const A raw = Tr<T>::to(Tr<T>::from(((am != am || am > eps) ? am : eps) / (A)127));
  const A sc = (raw != raw || raw > fmin) ? raw : fmin;
  for (int k = lane; k < dim; k += 32) {
    A v = Tr<T>::to(Tr<T>::from(Tr<T>::to(xt[k]) / sc));
    v = v < (A)-127 ? (A)-127 : (v > (A)127 ? (A)127 : v);
    if (v != v) v = (A)0;
    emit(k, (int8_t)rint(v));
  }
  return Tr<T>::to(Tr<T>::from(sc));
}

}  // namespace fms
