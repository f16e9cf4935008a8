// Specialisations of the tcgen05 GEMM with a K-major A operand on CTA pairs (256 x 256 tiles)
// (one translation unit per group, so they compile in parallel).
#include "gemm_sm100.cuh"

namespace tb {
namespace g2 {

template <>
void launch_gemm2<false, false, STORE, 256, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, STORE, 256, 2>(mp, x, st);
}
template <>
void launch_gemm2<false, false, RESID, 256, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, RESID, 256, 2>(mp, x, st);
}
template <>
void launch_gemm2<false, false, ACT, 256, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, ACT, 256, 2>(mp, x, st);
}
template <>
void launch_gemm2<false, false, ERR, 256, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, ERR, 256, 2>(mp, x, st);
}
template <>
void launch_gemm2<false, false, SWIGLU, 256, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, SWIGLU, 256, 2>(mp, x, st);
}
template <>
void launch_gemm2<false, false, PARTIAL, 256, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, false, PARTIAL, 256, 2>(mp, x, st);
}
template <>
void launch_gemm2<false, true, STORE, 256, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, true, STORE, 256, 2>(mp, x, st);
}
template <>
void launch_gemm2<false, true, ACT_GRAD, 256, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, true, ACT_GRAD, 256, 2>(mp, x, st);
}
template <>
void launch_gemm2<false, true, SWIGLU_BWD, 256, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, true, SWIGLU_BWD, 256, 2>(mp, x, st);
}
template <>
void launch_gemm2<false, true, PARTIAL, 256, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<false, true, PARTIAL, 256, 2>(mp, x, st);
}

}  // namespace g2
}  // namespace tb
