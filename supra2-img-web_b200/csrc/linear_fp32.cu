// FP32 linear layer y = x W^T (+ bias): the projections on either side of the attention path
// (ops.linear, app/gpu/ops.js:35-43; the cross-attention K/V preparation of
// app/models/dit.js:137-144 runs ctx_proj and then the 14 blocks' kv projections).
//
// One grouped launch per flush over every recorded problem: 128x128 output tiles over 256
// threads, each thread an 8x8 register block (rows rg + 16i, columns cg + 16j), x and W both
// read along K (W is [N, K] row-major, the reference's weight layout) and staged 16 deep through
// double-buffered padded shared memory by cp.async, zero-filled past every edge. FFMA only, fp32
// throughout. Two CTAs per SM (128 registers per thread): with the compiler's 242 registers one
// CTA, 2 warps per scheduler, left the FMA pipe waiting (K/V preparation 75.9 -> 67.7 ms). Within a problem the row tiles are outer and the column tiles inner, so CTAs that
// run together share x rows and sweep W, which stays in L2 (the 14 stacked kv weights are
// 37 MB).
// Optional fusions: GroupNorm of x applied to each staged x tile in shared memory before it is
// used (statistics from gn_stats_kernel, an earlier launch in the same flush; the VAE mid-block
// attention, app/models/vae.js:77-94), and a residual, optionally gated per column, added in the
// epilogue (app/gpu/gemm.js:10,135; in place for the DiT blocks' projections).
#include "common.cuh"

namespace supra {
namespace {

constexpr int kT = 256;   // threads
constexpr int kBM = 128;  // rows per tile
constexpr int kBN = 128;  // columns per tile
constexpr int kBK = 16;   // reduction depth per stage
constexpr int kS = kBK + 4;  // row stride of the stage buffers (conflict-free float4 reads)

template <bool BIAS, bool ALIGNED>
__global__ void __launch_bounds__(kT, 2) linear_fp32_kernel(const LinLaunch L) {
  __shared__ __align__(16) float As[2][kBM * kS];
  __shared__ __align__(16) float Bs[2][kBN * kS];
  const int t = blockIdx.x;
  if (t >= L.total) {
    if (threadIdx.x == 0) report_error(L.status, DEV_BAD_TILE, 30);
    return;
  }
  const int pi = find_problem(L.begin, L.n, t);
  const LinProb& P = L.probs[pi];
  const int local = t - __ldg(L.begin + pi);
  const int rt = local / P.n_tiles;
  const int r0 = rt * kBM;
  const int c0 = (local - rt * P.n_tiles) * kBN;
  const int K = P.K;
  const float* abase = P.x + (int64_t)r0 * P.ldx;
  const float* bbase = P.w + (int64_t)c0 * P.ldw;
  const int nr = min(kBM, P.M - r0);
  const int nc = min(kBN, P.N - c0);

  const int tid = threadIdx.x;
  const int rg = tid >> 4, cg = tid & 15;

  auto load_stage = [&](int buf, int k0) {
    if (ALIGNED) {
#pragma unroll
      for (int it = 0; it < 2; ++it) {  // 512 float4 per operand
        const int idx = tid + it * kT;
        const int r = idx >> 2, c4 = idx & 3;
        const int k = k0 + c4 * 4;
        const bool okA = (r < nr) && (k < K);
        cp_async16(&As[buf][r * kS + c4 * 4], okA ? (const void*)(abase + (int64_t)r * P.ldx + k) : (const void*)abase,
                   okA ? 16u : 0u);
        const bool okB = (r < nc) && (k < K);
        cp_async16(&Bs[buf][r * kS + c4 * 4], okB ? (const void*)(bbase + (int64_t)r * P.ldw + k) : (const void*)bbase,
                   okB ? 16u : 0u);
      }
    } else {
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int idx = tid + it * kT;
        const int r = idx >> 4, c = idx & 15;
        const int k = k0 + c;
        const bool okA = (r < nr) && (k < K);
        cp_async4(&As[buf][r * kS + c], okA ? (const void*)(abase + (int64_t)r * P.ldx + k) : (const void*)abase,
                  okA ? 4u : 0u);
        const bool okB = (r < nc) && (k < K);
        cp_async4(&Bs[buf][r * kS + c], okB ? (const void*)(bbase + (int64_t)r * P.ldw + k) : (const void*)bbase,
                  okB ? 4u : 0u);
      }
    }
    cp_async_commit();
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int nstage = (K + kBK - 1) / kBK;
  load_stage(0, 0);
  for (int st = 0; st < nstage; ++st) {
    if (st + 1 < nstage) {
      load_stage((st + 1) & 1, (st + 1) * kBK);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (P.gn_stats) {
      // GroupNorm (+ SiLU) or LayerNorm (+ modulation) of the staged x tile, per element of a
      // valid row and column (padding stays zero): (x - mean) * rstd * g + b with g, b = gamma,
      // beta (app/gpu/kernels.js:141-162), 1 + scale, shift (app/gpu/kernels.js:111) or 1, 0
      float* a = As[st & 1];
      const int k0 = st * kBK;
#pragma unroll
      for (int it = 0; it < kBM * kBK / kT; ++it) {
        const int idx = tid + it * kT;
        const int r = idx >> 4, kk = idx & 15;
        const int k = k0 + kk;
        if (r < nr && k < K) {
          const float2 ms = __ldg(P.gn_stats + (int64_t)((r0 + r) / P.gn_rows) * P.gn_groups + k / P.gn_cg);
          float g = 1.f, b = 0.f;
          if (P.gn_mode != kNormPlain) {
            g = __ldg(P.gamma + k);
            b = __ldg(P.beta + k);
            if (P.gn_mode == kNormModulated) g = 1.f + g;
          }
          float v = (a[r * kS + kk] - ms.x) * ms.y * g + b;
          if (P.gn_silu) v = v / (1.f + __expf(-v));
          a[r * kS + kk] = v;
        }
      }
      __syncthreads();
    }
    const float4* A4 = reinterpret_cast<const float4*>(As[st & 1]) + rg * (kS / 4);
    const float4* B4 = reinterpret_cast<const float4*>(Bs[st & 1]) + cg * (kS / 4);
#pragma unroll
    for (int k4 = 0; k4 < kBK / 4; ++k4) {
      float4 bf[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) bf[j] = B4[j * 16 * (kS / 4) + k4];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 af = A4[i * 16 * (kS / 4) + k4];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          acc[i][j] = fmaf(af.x, bf[j].x, acc[i][j]);
          acc[i][j] = fmaf(af.y, bf[j].y, acc[i][j]);
          acc[i][j] = fmaf(af.z, bf[j].z, acc[i][j]);
          acc[i][j] = fmaf(af.w, bf[j].w, acc[i][j]);
        }
      }
    }
    __syncthreads();
  }

  // y rows r0 + rg + 16i, columns c0 + cg + 16j: each store instruction writes two 64-byte row runs
  float bias[8], gate[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    bias[j] = (BIAS && cg + 16 * j < nc) ? __ldg(P.bias + c0 + cg + 16 * j) : 0.f;
    gate[j] = (P.gate && cg + 16 * j < nc) ? __ldg(P.gate + c0 + cg + 16 * j) : 1.f;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = rg + 16 * i;
    if (r >= nr) continue;
    float* yrow = P.y + (int64_t)(r0 + r) * P.ldy + c0;
    // resid may be y itself (in place): each element is read and then written by this thread only
    const float* rrow = P.resid ? P.resid + (int64_t)(r0 + r) * P.ldr + c0 : nullptr;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = cg + 16 * j;
      if (c < nc) {
        float v = acc[i][j] + bias[j];
        if (P.act != kActNone) v = linear_act(P.act, v);
        if (P.gate) v *= gate[j];
        yrow[c] = rrow ? rrow[c] + v : v;
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------
// One CTA per (image, group): mean, then the variance around it (two passes for accuracy, as the
// reference's groupnormStatsShader), over rows_per_image rows x cg channels.
__global__ void __launch_bounds__(256) gn_stats_kernel(const float* __restrict__ x, int32_t K, int32_t rows,
                                                       int32_t groups, float eps, float2* __restrict__ stats) {
  __shared__ float red[8];
  const int img = blockIdx.x / groups;
  const int g = blockIdx.x - img * groups;
  const int cg = K / groups;
  const int64_t n = (int64_t)rows * cg;
  const float* base = x + (int64_t)img * rows * K + (int64_t)g * cg;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  auto block_sum = [&](float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w];
    __syncthreads();
    return t;
  };
  float s = 0.f;
  for (int64_t i = tid; i < n; i += 256) s += __ldg(base + (i / cg) * K + i % cg);
  const float mean = block_sum(s) / (float)n;
  float v = 0.f;
  for (int64_t i = tid; i < n; i += 256) {
    const float d = __ldg(base + (i / cg) * K + i % cg) - mean;
    v = fmaf(d, d, v);
  }
  const float var = block_sum(v) / (float)n;
  if (tid == 0) stats[blockIdx.x] = make_float2(mean, rsqrtf(var + eps));
}

// One warp per row: LayerNorm statistics over the row's K channels, mean then the variance
// around it, as the reference's layernormShader (app/gpu/kernels.js:104-110).
__global__ void __launch_bounds__(256) ln_stats_kernel(const float* __restrict__ x, int32_t K, int32_t rows,
                                                       float eps, float2* __restrict__ stats) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* base = x + (int64_t)row * K;
  float s = 0.f;
  for (int i = lane; i < K; i += 32) s += __ldg(base + i);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / (float)K;
  float v = 0.f;
  for (int i = lane; i < K; i += 32) {
    const float d = __ldg(base + i) - mean;
    v = fmaf(d, d, v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) stats[row] = make_float2(mean, rsqrtf(v / (float)K + eps));
}

}  // namespace

cudaError_t launch_ln_stats(const float* x, int32_t K, int32_t rows, float eps, float2* stats, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  ln_stats_kernel<<<(rows + 7) / 8, 256, 0, s>>>(x, K, rows, eps, stats);
  return cudaGetLastError();
}

cudaError_t launch_gn_stats(const float* x, int32_t K, int32_t rows_per_image, int32_t images, int32_t groups,
                            float eps, float2* stats, cudaStream_t s) {
  if (images <= 0) return cudaSuccess;
  gn_stats_kernel<<<images * groups, 256, 0, s>>>(x, K, rows_per_image, groups, eps, stats);
  return cudaGetLastError();
}

cudaError_t launch_linear_fp32(bool bias, bool aligned, const LinLaunch& L, cudaStream_t s) {
  if (L.total <= 0) return cudaSuccess;
  if (bias) {
    if (aligned) linear_fp32_kernel<true, true><<<L.total, kT, 0, s>>>(L);
    else linear_fp32_kernel<true, false><<<L.total, kT, 0, s>>>(L);
  } else {
    if (aligned) linear_fp32_kernel<false, true><<<L.total, kT, 0, s>>>(L);
    else linear_fp32_kernel<false, false><<<L.total, kT, 0, s>>>(L);
  }
  return cudaGetLastError();
}

}  // namespace supra
