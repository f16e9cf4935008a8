// Specialisations of the 2-CTA tcgen05 GEMM with a MN-major A operand
// (one translation unit per layout, so they compile in parallel).
#include "gemm_sm100.cuh"

namespace tb {
namespace g2 {

template <>
void launch_gemm2<true, true, STORE>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, STORE>(mp, x, st);
}
template <>
void launch_gemm2<true, true, PARTIAL>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, PARTIAL>(mp, x, st);
}
template <>
void launch_gemm2<true, false, STORE>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, false, STORE>(mp, x, st);
}
template <>
void launch_gemm2<true, false, PARTIAL>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, false, PARTIAL>(mp, x, st);
}

}  // namespace g2
}  // namespace tb
