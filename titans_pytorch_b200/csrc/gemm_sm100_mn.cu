// Specialisations of the 2-CTA tcgen05 GEMM with an MN-major A operand (both tile widths)
// (one translation unit per group, so they compile in parallel).
#include "gemm_sm100.cuh"

namespace tb {
namespace g2 {

template <>
void launch_gemm2<true, true, STORE, 256>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, STORE, 256>(mp, x, st);
}
template <>
void launch_gemm2<true, true, PARTIAL, 256>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, PARTIAL, 256>(mp, x, st);
}
template <>
void launch_gemm2<true, false, STORE, 256>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, false, STORE, 256>(mp, x, st);
}
template <>
void launch_gemm2<true, false, PARTIAL, 256>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, false, PARTIAL, 256>(mp, x, st);
}
template <>
void launch_gemm2<true, true, STORE, 128>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, STORE, 128>(mp, x, st);
}
template <>
void launch_gemm2<true, true, PARTIAL, 128>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, PARTIAL, 128>(mp, x, st);
}
template <>
void launch_gemm2<true, false, STORE, 128>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, false, STORE, 128>(mp, x, st);
}
template <>
void launch_gemm2<true, false, PARTIAL, 128>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, false, PARTIAL, 128>(mp, x, st);
}

}  // namespace g2
}  // namespace tb
