// Specialisations of the tcgen05 GEMM with an MN-major A operand (every tile shape)
// (one translation unit per group, so they compile in parallel).
#include "gemm_sm100.cuh"

namespace tb {
namespace g2 {

template <>
void launch_gemm2<true, true, STORE, 256, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, STORE, 256, 2>(mp, x, st);
}
template <>
void launch_gemm2<true, true, ACCUM, 256, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, ACCUM, 256, 2>(mp, x, st);
}
template <>
void launch_gemm2<true, true, MEM_UPDATE, 256, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, MEM_UPDATE, 256, 2>(mp, x, st);
}
template <>
void launch_gemm2<true, true, PARTIAL, 256, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, PARTIAL, 256, 2>(mp, x, st);
}
template <>
void launch_gemm2<true, false, STORE, 256, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, false, STORE, 256, 2>(mp, x, st);
}
template <>
void launch_gemm2<true, false, PARTIAL, 256, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, false, PARTIAL, 256, 2>(mp, x, st);
}
template <>
void launch_gemm2<true, true, STORE, 128, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, STORE, 128, 2>(mp, x, st);
}
template <>
void launch_gemm2<true, true, ACCUM, 128, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, ACCUM, 128, 2>(mp, x, st);
}
template <>
void launch_gemm2<true, true, MEM_UPDATE, 128, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, MEM_UPDATE, 128, 2>(mp, x, st);
}
template <>
void launch_gemm2<true, true, PARTIAL, 128, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, PARTIAL, 128, 2>(mp, x, st);
}
template <>
void launch_gemm2<true, false, STORE, 128, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, false, STORE, 128, 2>(mp, x, st);
}
template <>
void launch_gemm2<true, false, PARTIAL, 128, 2>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, false, PARTIAL, 128, 2>(mp, x, st);
}
template <>
void launch_gemm2<true, true, STORE, 128, 1>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, STORE, 128, 1>(mp, x, st);
}
template <>
void launch_gemm2<true, true, ACCUM, 128, 1>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, ACCUM, 128, 1>(mp, x, st);
}
template <>
void launch_gemm2<true, true, MEM_UPDATE, 128, 1>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, MEM_UPDATE, 128, 1>(mp, x, st);
}
template <>
void launch_gemm2<true, true, PARTIAL, 128, 1>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, true, PARTIAL, 128, 1>(mp, x, st);
}
template <>
void launch_gemm2<true, false, STORE, 128, 1>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, false, STORE, 128, 1>(mp, x, st);
}
template <>
void launch_gemm2<true, false, PARTIAL, 128, 1>(const Maps& mp, const Args& x, cudaStream_t st) {
  launch_gemm2_impl<true, false, PARTIAL, 128, 1>(mp, x, st);
}

}  // namespace g2
}  // namespace tb
