// Descriptor staging: copies one flush's packed descriptors (problem records, tile prefixes,
// TMA tensor maps) from the pinned host ring into the device ring with the SMs reading host
// memory directly.
//
// A copy-engine transfer (cudaMemcpyAsync) would do the same work, but host-to-device copies are
// served in submission order: a descriptor copy submitted after a multi-gigabyte input upload on
// another stream waits for that whole upload, and the attention launches behind it stall. A
// kernel only shares the host link with such an upload.
#include "kernels.h"

namespace supra {
namespace {

__global__ void __launch_bounds__(256) stage_copy_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                         int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = __ldcv(src + i);  // the host rewrites the ring between launches: never a cached line
}

}  // namespace

cudaError_t launch_stage_copy(const void* src, void* dst, size_t bytes, cudaStream_t s) {
  if (bytes == 0) return cudaSuccess;
  if ((bytes & 15) || (reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 15))
    return cudaErrorInvalidValue;
  const int64_t n = (int64_t)(bytes / 16);
  const int64_t blocks = (n + 255) / 256;
  stage_copy_kernel<<<(unsigned)(blocks < 128 ? blocks : 128), 256, 0, s>>>(static_cast<const uint4*>(src),
                                                                          static_cast<uint4*>(dst), n);
  return cudaGetLastError();
}

}  // namespace supra
