// Specialisations of the 2-CTA tcgen05 GEMM with a K-major A operand
// (one translation unit per layout, so they compile in parallel).
#include "gemm_sm100.cuh"

namespace tb {
namespace g2 {

template <>
void launch_gemm2<false, false, STORE>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, STORE>(mp, x, st);
}
template <>
void launch_gemm2<false, false, RESID>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, RESID>(mp, x, st);
}
template <>
void launch_gemm2<false, false, ACT>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, ACT>(mp, x, st);
}
template <>
void launch_gemm2<false, false, ERR>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, ERR>(mp, x, st);
}
template <>
void launch_gemm2<false, false, SWIGLU>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, SWIGLU>(mp, x, st);
}
template <>
void launch_gemm2<false, false, PARTIAL>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, PARTIAL>(mp, x, st);
}
template <>
void launch_gemm2<false, true, STORE>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, true, STORE>(mp, x, st);
}
template <>
void launch_gemm2<false, true, ACT_GRAD>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, true, ACT_GRAD>(mp, x, st);
}
template <>
void launch_gemm2<false, true, SWIGLU_BWD>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, true, SWIGLU_BWD>(mp, x, st);
}
template <>
void launch_gemm2<false, true, PARTIAL>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, true, PARTIAL>(mp, x, st);
}

}  // namespace g2
}  // namespace tb
