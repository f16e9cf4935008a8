// Specialisations of the tcgen05 GEMM with a K-major A operand on single CTAs (128 x 128 tiles)
// (one translation unit per group, so they compile in parallel).
#include "gemm_sm100.cuh"

namespace tb {
namespace g2 {

template <>
void launch_gemm2<false, false, STORE, 128, 1>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, STORE, 128, 1>(mp, x, st);
}
template <>
void launch_gemm2<false, false, RESID, 128, 1>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, RESID, 128, 1>(mp, x, st);
}
template <>
void launch_gemm2<false, false, ACT, 128, 1>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, ACT, 128, 1>(mp, x, st);
}
template <>
void launch_gemm2<false, false, ERR, 128, 1>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, ERR, 128, 1>(mp, x, st);
}
template <>
void launch_gemm2<false, false, SWIGLU, 128, 1>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, SWIGLU, 128, 1>(mp, x, st);
}
template <>
void launch_gemm2<false, false, PARTIAL, 128, 1>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, PARTIAL, 128, 1>(mp, x, st);
}
template <>
void launch_gemm2<false, true, STORE, 128, 1>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, true, STORE, 128, 1>(mp, x, st);
}
template <>
void launch_gemm2<false, true, ACT_GRAD, 128, 1>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, true, ACT_GRAD, 128, 1>(mp, x, st);
}
template <>
void launch_gemm2<false, true, SWIGLU_BWD, 128, 1>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, true, SWIGLU_BWD, 128, 1>(mp, x, st);
}
template <>
void launch_gemm2<false, true, PARTIAL, 128, 1>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, true, PARTIAL, 128, 1>(mp, x, st);
}

}  // namespace g2
}  // namespace tb
