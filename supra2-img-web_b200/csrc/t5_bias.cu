// T5 relative-position bias on the device: T5Encoder.positionBias (app/models/t5.js:55-65),
//   out[(h*L + i)*L + j] = table[bucket(j - i)*H + h],
// with bucket() supplied as a lookup table over rel = -(L-1) .. L-1 that the host computes with
// the reference's float32 rounding (relativeBucket, app/models/t5.js:14-23). The reference
// builds this [H, L, L] array on the CPU and uploads it per encode (app/models/t5.js:73); here
// it is written straight into HBM with coalesced stores. HBM-write bound.
#include "common.cuh"

namespace supra {
namespace {

__global__ void __launch_bounds__(256) position_bias_kernel(const float* __restrict__ table,
                                                            const int32_t* __restrict__ lut, int32_t H, int32_t L,
                                                            float* __restrict__ out) {
  const int64_t total = (int64_t)H * L * L;
  const int64_t LL = (int64_t)L * L;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int h = (int)(e / LL);
    const int64_t rem = e - (int64_t)h * LL;
    const int i = (int)(rem / L);
    const int j = (int)(rem - (int64_t)i * L);
    out[e] = __ldg(table + (int64_t)__ldg(lut + (j - i + L - 1)) * H + h);
  }
}

// The bias as a function of the relative position alone: out[h*R + d] = table[lut[d]*H + h],
// d = rel + rel_max over R = 2 rel_max + 1 positions (past +-rel_max the bucket no longer
// changes). The FP32 attention kernel reads a T5 table bias from this array, one load per score.
__global__ void __launch_bounds__(256) rel_bias_kernel(const float* __restrict__ table, const int32_t* __restrict__ lut,
                                                       int32_t H, int32_t R, float* __restrict__ out) {
  const int total = H * R;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
    const int h = e / R;
    out[e] = __ldg(table + (int64_t)__ldg(lut + (e - h * R)) * H + h);
  }
}

}  // namespace

cudaError_t launch_rel_bias(const float* table, const int32_t* lut, int32_t H, int32_t rel_max, float* out,
                            cudaStream_t s) {
  const int64_t total = (int64_t)H * (2 * (int64_t)rel_max + 1);
  if (H <= 0 || rel_max < 0 || total > (int64_t(1) << 30)) return cudaErrorInvalidValue;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148) blocks = 148;
  rel_bias_kernel<<<(unsigned)blocks, 256, 0, s>>>(table, lut, H, (int32_t)(2 * rel_max + 1), out);
  return cudaGetLastError();
}

cudaError_t launch_position_bias(const float* table, const int32_t* lut, int32_t H, int32_t L, float* out,
                                 cudaStream_t s) {
  if (H <= 0 || L <= 0) return cudaSuccess;
  const int64_t total = (int64_t)H * L * L;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  position_bias_kernel<<<(unsigned)blocks, 256, 0, s>>>(table, lut, H, L, out);
  return cudaGetLastError();
}

}  // namespace supra
