// Score-materialising FP32 attention for head dims above 128 (the VAE's single 512-wide head).
//
// The same three steps as the reference's unfused path (app/gpu/ops.js:119-147):
//   attn.qk       S = Q K^T * scale (+ bias)          batched GEMM, K read row-major
//   attn.softmax  P = softmax(S) per row, in place     (app/gpu/kernels.js:27-63)
//   attn.pv       O = P V, written with row stride H*D (app/gpu/ops.js:139-144)
// with the scores of a chunk of (problem, head, rows) units held in a scratch buffer that the
// host sizes so that a chunk's scores stay resident in the 126 MB L2 between the three kernels.
//
// Both GEMMs are 128x128 tiles over 256 threads with 8x8 register blocks (thread (rg, cg) in
// 16x16 owns rows rg + 16*i and columns cg + 16*j / float4 groups cg, cg + 16), operands staged
// 16-deep through double-buffered padded shared memory by cp.async (zero-filled past every edge).
#include <type_traits>

#include "common.cuh"

namespace supra {
namespace {

constexpr int kGT = 256;  // threads
constexpr int kBN = 128;  // columns per tile
constexpr int kBK = 16;   // reduction depth per stage
constexpr int kAS = kBK + 4;   // row stride of the [rows][k] stage buffers
constexpr int kVS = kBN + 4;   // row stride of the [k][cols] V stage buffer

__device__ __forceinline__ int find_unit(const int32_t* begin, int n, int t) { return find_problem(begin, n, t); }

// ------------------------------------------------------------------------------------------------
// S[r][c] = scale * sum_d Q[row0 + r][d] K[c][d] (+ bias[h][row0 + r][c]). BM query rows per tile
// (128, or 64 / 32 for launches with fewer 128-row tiles than SMs: one VAE image has 64), thread
// (rg, cg) owning rows rg + 16i (i < BM / 16) and columns cg + 16j (j < 8).
template <bool BIAS, bool ALIGNED, int BM>
__global__ void __launch_bounds__(kGT, 2) gemm_qk_kernel(const GemmLaunch L) {
  constexpr int MI = BM / 16;
  __shared__ __align__(16) float As[2][BM * kAS];
  __shared__ __align__(16) float Bs[2][kBN * kAS];
  const int t = blockIdx.x;
  if (t >= L.qk_total) return;
  const int ui = find_unit(L.qk_begin, L.n_units, t);
  const GemmUnit u = L.units[ui];
  const AttnProb& P = L.probs[u.prob];
  const int local = t - u.qk_begin;
  const int ktiles = (P.Lk + kBN - 1) / kBN;
  const int rt = local / ktiles;
  const int kt = local - rt * ktiles;
  const int r0 = rt * BM;  // within the unit
  const int c0 = kt * kBN;
  const int D = P.D;
  const float* qbase = P.q + P.q_off + (int64_t)(u.row0 + r0) * P.ldq + (int64_t)u.h * D;
  const float* kbase = P.k + P.k_off + (int64_t)c0 * P.ldk + (int64_t)u.h * D;
  const int nr = min(BM, u.rows - r0);
  const int nc = min(kBN, P.Lk - c0);

  const int tid = threadIdx.x;
  const int rg = tid >> 4, cg = tid & 15;

  auto load_stage = [&](int buf, int d0) {
    if (ALIGNED) {
#pragma unroll
      for (int it = 0; it < 2; ++it) {  // 512 float4 of K, BM * 4 of Q
        const int idx = tid + it * kGT;
        const int r = idx >> 2, c4 = idx & 3;
        const int d = d0 + c4 * 4;
        if (idx < BM * 4) {
          const bool okA = (r < nr) && (d < D);
          cp_async16(&As[buf][r * kAS + c4 * 4], okA ? (const void*)(qbase + (int64_t)r * P.ldq + d) : (const void*)qbase,
                     okA ? 16u : 0u);
        }
        const bool okB = (r < nc) && (d < D);
        cp_async16(&Bs[buf][r * kAS + c4 * 4], okB ? (const void*)(kbase + (int64_t)r * P.ldk + d) : (const void*)kbase,
                   okB ? 16u : 0u);
      }
    } else {
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int idx = tid + it * kGT;
        const int r = idx >> 4, c = idx & 15;
        const int d = d0 + c;
        if (idx < BM * 16) {
          const bool okA = (r < nr) && (d < D);
          cp_async4(&As[buf][r * kAS + c], okA ? (const void*)(qbase + (int64_t)r * P.ldq + d) : (const void*)qbase,
                    okA ? 4u : 0u);
        }
        const bool okB = (r < nc) && (d < D);
        cp_async4(&Bs[buf][r * kAS + c], okB ? (const void*)(kbase + (int64_t)r * P.ldk + d) : (const void*)kbase,
                  okB ? 4u : 0u);
      }
    }
    cp_async_commit();
  };

  float acc[MI][8];
#pragma unroll
  for (int i = 0; i < MI; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int nstage = (D + kBK - 1) / kBK;
  load_stage(0, 0);
  for (int st = 0; st < nstage; ++st) {
    if (st + 1 < nstage) {
      load_stage((st + 1) & 1, (st + 1) * kBK);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float4* A4 = reinterpret_cast<const float4*>(As[st & 1]) + rg * (kAS / 4);
    const float4* B4 = reinterpret_cast<const float4*>(Bs[st & 1]) + cg * (kAS / 4);
#pragma unroll
    for (int d4 = 0; d4 < kBK / 4; ++d4) {
      float4 bf[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) bf[j] = B4[j * 16 * (kAS / 4) + d4];
#pragma unroll
      for (int i = 0; i < MI; ++i) {
        const float4 af = A4[i * 16 * (kAS / 4) + d4];
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

  float* S = L.scratch + u.s_off;
  const float scale = P.scale;
#pragma unroll
  for (int i = 0; i < MI; ++i) {
    const int r = rg + 16 * i;
    if (r >= nr) continue;
    const int grow = u.row0 + r0 + r;  // query row within the problem
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = cg + 16 * j;
      if (c >= nc) continue;
      float x = acc[i][j] * scale;
      if (BIAS)
        x += P.rel_lut ? t5_table_bias(P.bias + u.h, P.rel_lut + P.rel_max, P.rel_max, (uint32_t)P.H, c0 + c - grow)
                       : __ldg(P.bias + ((int64_t)u.h * P.Lq + grow) * P.Lk + c0 + c);
      S[(int64_t)(r0 + r) * u.ldS + c0 + c] = x;
    }
  }
}

// ------------------------------------------------------------------------------------------------
// In-place row softmax of the unit's scores, one warp per row: max, exp and sum, normalise
// (app/gpu/kernels.js:53-62). For the tensor-core products (L.sm_scale) the scores come unscaled
// and the problem's scale is applied here, exp(scale s - max(scale s)); with L.lo set each
// probability p leaves split, hi (p with its 13 low mantissa bits cleared) in place and p - hi at
// the same offset from L.lo. Columns Lk .. ldS - 1 are zeroed.
// A row of at most 128 NV keys (ldS floats, a multiple of 4, 16-byte aligned) held in registers:
// lane l owns the float4 chunks l, l + 32, ..., so the row is read once and written once (P, and
// its lo part for the split tensor-core product) instead of three passes over memory. Same
// arithmetic per score as the loop form below (scale, max, expf(s - max), one reciprocal); the
// sum is formed in another order.
template <int NV>
__device__ __forceinline__ void softmax_row_regs(float* __restrict__ row, float* __restrict__ lrow, int Lk, int ldS,
                                                 float sc, int lane) {
  float4 x[NV];
  float mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int c = 4 * (lane + 32 * k);
    x[k] = c < ldS ? *reinterpret_cast<const float4*>(row + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    x[k].x = c + 0 < Lk ? x[k].x * sc : -INFINITY;
    x[k].y = c + 1 < Lk ? x[k].y * sc : -INFINITY;
    x[k].z = c + 2 < Lk ? x[k].z * sc : -INFINITY;
    x[k].w = c + 3 < Lk ? x[k].w * sc : -INFINITY;
    mx = fmaxf(mx, fmaxf(fmaxf(x[k].x, x[k].y), fmaxf(x[k].z, x[k].w)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sm = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {  // (expf(-inf) = 0 past Lk)
    x[k] = make_float4(expf(x[k].x - mx), expf(x[k].y - mx), expf(x[k].z - mx), expf(x[k].w - mx));
    sm += (x[k].x + x[k].y) + (x[k].z + x[k].w);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
  const float inv = 1.0f / sm;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int c = 4 * (lane + 32 * k);
    if (c >= ldS) continue;
    float4 p = make_float4(x[k].x * inv, x[k].y * inv, x[k].z * inv, x[k].w * inv);
    if (lrow) {
      const float4 h = make_float4(__uint_as_float(__float_as_uint(p.x) & 0xffffe000u),
                                   __uint_as_float(__float_as_uint(p.y) & 0xffffe000u),
                                   __uint_as_float(__float_as_uint(p.z) & 0xffffe000u),
                                   __uint_as_float(__float_as_uint(p.w) & 0xffffe000u));
      *reinterpret_cast<float4*>(lrow + c) = make_float4(p.x - h.x, p.y - h.y, p.z - h.z, p.w - h.w);
      p = h;
    }
    *reinterpret_cast<float4*>(row + c) = p;
  }
}

__global__ void __launch_bounds__(256) softmax_rows_kernel(const GemmLaunch L) {
  const int wid = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (wid >= L.row_total) return;
  const int ui = find_unit(L.row_begin, L.n_units, wid);
  const GemmUnit u = L.units[ui];
  const int Lk = L.probs[u.prob].Lk;
  const float sc = L.sm_scale ? L.probs[u.prob].scale : 1.f;
  const int64_t off = u.s_off + (int64_t)(wid - u.row_begin) * u.ldS;
  float* row = L.scratch + off;
  // rows of up to 1024 keys in registers (the VAE's 32 x 32 latents): one pass each way
  switch ((u.ldS + 127) >> 7) {
    case 1: return softmax_row_regs<1>(row, L.lo ? L.lo + off : nullptr, Lk, u.ldS, sc, lane);
    case 2: return softmax_row_regs<2>(row, L.lo ? L.lo + off : nullptr, Lk, u.ldS, sc, lane);
    case 3: return softmax_row_regs<3>(row, L.lo ? L.lo + off : nullptr, Lk, u.ldS, sc, lane);
    case 4: return softmax_row_regs<4>(row, L.lo ? L.lo + off : nullptr, Lk, u.ldS, sc, lane);
    case 5: return softmax_row_regs<5>(row, L.lo ? L.lo + off : nullptr, Lk, u.ldS, sc, lane);
    case 6: return softmax_row_regs<6>(row, L.lo ? L.lo + off : nullptr, Lk, u.ldS, sc, lane);
    case 7: return softmax_row_regs<7>(row, L.lo ? L.lo + off : nullptr, Lk, u.ldS, sc, lane);
    case 8: return softmax_row_regs<8>(row, L.lo ? L.lo + off : nullptr, Lk, u.ldS, sc, lane);
    default: break;
  }
  float mx = -INFINITY;
  for (int c = lane; c < Lk; c += 32) mx = fmaxf(mx, row[c] * sc);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sm = 0.f;
  for (int c = lane; c < Lk; c += 32) {
    const float e = expf(row[c] * sc - mx);
    row[c] = e;
    sm += e;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
  const float inv = 1.0f / sm;
  if (L.lo) {
    float* lrow = L.lo + off;
    for (int c = lane; c < u.ldS; c += 32) {
      const float p = c < Lk ? row[c] * inv : 0.f;
      const float h = __uint_as_float(__float_as_uint(p) & 0xffffe000u);
      row[c] = h;
      lrow[c] = p - h;
    }
  } else {
    for (int c = lane; c < u.ldS; c += 32) row[c] = c < Lk ? row[c] * inv : 0.f;
  }
}

// ------------------------------------------------------------------------------------------------
// O[row0 + r][c] = sum_k P[r][k] V[k][c], BM rows per tile as gemm_qk_kernel
template <bool ALIGNED, int BM>
__global__ void __launch_bounds__(kGT) gemm_pv_kernel(const GemmLaunch L) {
  constexpr int MI = BM / 16;
  __shared__ __align__(16) float As[2][BM * kAS];
  __shared__ __align__(16) float Vt[2][kBK * kVS];
  const int t = blockIdx.x;
  if (t >= L.pv_total) return;
  const int ui = find_unit(L.pv_begin, L.n_units, t);
  const GemmUnit u = L.units[ui];
  const AttnProb& P = L.probs[u.prob];
  const int local = t - u.pv_begin;
  const int D = P.D;
  const int ctiles = (D + kBN - 1) / kBN;
  const int rt = local / ctiles;
  const int ct = local - rt * ctiles;
  const int r0 = rt * BM;
  const int c0 = ct * kBN;
  const int Lk = P.Lk;
  const int nr = min(BM, u.rows - r0);
  const int nc = min(kBN, D - c0);
  const float* pbase = L.scratch + u.s_off + (int64_t)r0 * u.ldS;
  const float* vbase = P.v + P.v_off + (int64_t)u.h * D + c0;

  const int tid = threadIdx.x;
  const int rg = tid >> 4, cg = tid & 15;

  auto load_stage = [&](int buf, int k0) {
#pragma unroll
    for (int it = 0; it < (BM * 4 + kGT - 1) / kGT; ++it) {  // P tile [BM][16]: scratch rows are 16-byte aligned
      const int idx = tid + it * kGT;
      const int r = idx >> 2, c4 = idx & 3;
      const int k = k0 + c4 * 4;
      if (idx < BM * 4) {
        const bool ok = (r < nr) && (k < u.ldS);
        cp_async16(&As[buf][r * kAS + c4 * 4], ok ? (const void*)(pbase + (int64_t)r * u.ldS + k) : (const void*)pbase,
                   ok ? 16u : 0u);
      }
    }
    if (ALIGNED) {
#pragma unroll
      for (int it = 0; it < 2; ++it) {  // V tile [16][128]
        const int idx = tid + it * kGT;
        const int k = idx >> 5, c4 = idx & 31;
        const bool ok = (k0 + k < Lk) && (c4 * 4 < nc);
        cp_async16(&Vt[buf][k * kVS + c4 * 4],
                   ok ? (const void*)(vbase + (int64_t)(k0 + k) * P.ldv + c4 * 4) : (const void*)vbase, ok ? 16u : 0u);
      }
    } else {
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int idx = tid + it * kGT;
        const int k = idx >> 7, c = idx & 127;
        const bool ok = (k0 + k < Lk) && (c < nc);
        cp_async4(&Vt[buf][k * kVS + c], ok ? (const void*)(vbase + (int64_t)(k0 + k) * P.ldv + c) : (const void*)vbase,
                  ok ? 4u : 0u);
      }
    }
    cp_async_commit();
  };

  float4 acc[MI][2];
#pragma unroll
  for (int i = 0; i < MI; ++i) acc[i][0] = acc[i][1] = make_float4(0.f, 0.f, 0.f, 0.f);

  const int nstage = (Lk + kBK - 1) / kBK;
  load_stage(0, 0);
  for (int st = 0; st < nstage; ++st) {
    if (st + 1 < nstage) {
      load_stage((st + 1) & 1, (st + 1) * kBK);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float4* A4 = reinterpret_cast<const float4*>(As[st & 1]) + rg * (kAS / 4);
    const float4* V4 = reinterpret_cast<const float4*>(Vt[st & 1]) + cg;
#pragma unroll
    for (int k4 = 0; k4 < kBK / 4; ++k4) {
      float4 af[MI];
#pragma unroll
      for (int i = 0; i < MI; ++i) af[i] = A4[i * 16 * (kAS / 4) + k4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float4 v0 = V4[(k4 * 4 + e) * (kVS / 4)];
        const float4 v1 = V4[(k4 * 4 + e) * (kVS / 4) + 16];
#pragma unroll
        for (int i = 0; i < MI; ++i) {
          const float pe = e == 0 ? af[i].x : e == 1 ? af[i].y : e == 2 ? af[i].z : af[i].w;
          acc[i][0].x = fmaf(pe, v0.x, acc[i][0].x);
          acc[i][0].y = fmaf(pe, v0.y, acc[i][0].y);
          acc[i][0].z = fmaf(pe, v0.z, acc[i][0].z);
          acc[i][0].w = fmaf(pe, v0.w, acc[i][0].w);
          acc[i][1].x = fmaf(pe, v1.x, acc[i][1].x);
          acc[i][1].y = fmaf(pe, v1.y, acc[i][1].y);
          acc[i][1].z = fmaf(pe, v1.z, acc[i][1].z);
          acc[i][1].w = fmaf(pe, v1.w, acc[i][1].w);
        }
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < MI; ++i) {
    const int r = rg + 16 * i;
    if (r >= nr) continue;
    float* dst = P.o + P.o_off + (int64_t)(u.row0 + r0 + r) * P.ldo + (int64_t)u.h * D + c0;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int c = 4 * cg + 64 * hf;
      const float4 v = acc[i][hf];
      if (ALIGNED) {
        if (c < nc) *reinterpret_cast<float4*>(dst + c) = v;
      } else {
        if (c + 0 < nc) dst[c + 0] = v.x;
        if (c + 1 < nc) dst[c + 1] = v.y;
        if (c + 2 < nc) dst[c + 2] = v.z;
        if (c + 3 < nc) dst[c + 3] = v.w;
      }
    }
  }
}

}  // namespace

cudaError_t launch_gemm_qk(bool bias, bool aligned, const GemmLaunch& L, cudaStream_t s) {
  if (L.qk_total <= 0) return cudaSuccess;
  auto go = [&](auto bm) {
    constexpr int BM = decltype(bm)::value;
    if (bias) {
      if (aligned) gemm_qk_kernel<true, true, BM><<<L.qk_total, kGT, 0, s>>>(L);
      else gemm_qk_kernel<true, false, BM><<<L.qk_total, kGT, 0, s>>>(L);
    } else {
      if (aligned) gemm_qk_kernel<false, true, BM><<<L.qk_total, kGT, 0, s>>>(L);
      else gemm_qk_kernel<false, false, BM><<<L.qk_total, kGT, 0, s>>>(L);
    }
  };
  if (L.bm == 32) go(std::integral_constant<int, 32>{});
  else if (L.bm == 64) go(std::integral_constant<int, 64>{});
  else go(std::integral_constant<int, 128>{});
  return cudaGetLastError();
}

cudaError_t launch_softmax_rows(const GemmLaunch& L, cudaStream_t s) {
  if (L.row_total <= 0) return cudaSuccess;
  softmax_rows_kernel<<<(L.row_total + 7) / 8, 256, 0, s>>>(L);
  return cudaGetLastError();
}

cudaError_t launch_gemm_pv(bool aligned, const GemmLaunch& L, cudaStream_t s) {
  if (L.pv_total <= 0) return cudaSuccess;
  auto go = [&](auto bm) {
    constexpr int BM = decltype(bm)::value;
    if (aligned) gemm_pv_kernel<true, BM><<<L.pv_total, kGT, 0, s>>>(L);
    else gemm_pv_kernel<false, BM><<<L.pv_total, kGT, 0, s>>>(L);
  };
  if (L.bm == 32) go(std::integral_constant<int, 32>{});
  else if (L.bm == 64) go(std::integral_constant<int, 64>{});
  else go(std::integral_constant<int, 128>{});
  return cudaGetLastError();
}

}  // namespace supra
