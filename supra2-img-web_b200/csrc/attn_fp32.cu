// Fused FP32 attention for sm_100a (FFMA pipe), head dim D <= 128.
//
// Computes, per (problem, head, tile of MQ query rows), O = softmax(Q K^T * scale + bias) V with
// an online softmax over key blocks of 64 — the algorithm of the reference's fused WGSL kernel
// (app/gpu/kernels.js:164-316: S = Q K^T per key block, masked keys at -inf, running row max
// m and sum l, O rescaled by exp(m_old - m_new), O / l at the end) extended with the optional
// additive [H, Lq, Lk] bias that the reference only supports on its unfused path
// (app/gpu/kernels.js:34, app/gpu/ops.js:135-137).
//
// B200 design:
//  * 128 threads; thread (rg = 0..15, cg = 0..7) owns query rows rg + 16*i (i < MQ/16), keys
//    cg + 8*j (j < 8) of the 64-key score tile, and output columns 4*(cg + 8*u) .. +3.
//    Both products are register-blocked (MQ/16 x 8 accumulators per thread per product) with
//    float4 shared-memory fragments: 16 LDS.128 per 256 FFMA for MQ = 128.
//  * Q, K and V tiles are staged by the bulk-copy (TMA) engine: one cp.async.bulk per row into a
//    padded shared-memory row (stride D+4 floats keeps the float4 fragment loads conflict-free),
//    completion on mbarriers with bounded waits. K for block j+1 streams in during PV of block j
//    and V for block j+1 during QK^T/softmax of block j+1. No tensor map; each CTA loads only into its own shared memory.
//  * Scores are exponentiated with exp2 and scale*log2(e) folded into one multiply.
//  * Row max is reduced with three xor-shuffles across the 8 lanes that share a row; row sums
//    stay per thread and are reduced once at the end.
//  * Ragged key lengths: keys >= Lk in the last block are masked to -inf and PV stops at the
//    last valid group of 4 keys.
//  * Many problems per launch: blockIdx.x indexes a tile list the host sorts longest-first.
#include "common.cuh"

namespace supra {
namespace {

constexpr int kThreads = 128;
constexpr int kNK = 64;       // keys per block
constexpr int kPS = kNK + 8;  // P row stride in floats (scalar writes and float4 reads conflict-free)
constexpr float kLog2e = 1.4426950408889634f;

template <int DT, int MQ>
struct Geom {
  static constexpr int TM = MQ / 16;  // query rows per thread
  static constexpr int U = DT / 32;   // float4 output column groups per thread
  static constexpr int QS = DT + 4;   // Q row stride (floats)
  static constexpr int KS = DT + 4;   // K row stride
  static constexpr int VS = DT;       // V row stride
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + MQ * QS;
  static constexpr int V_OFF = K_OFF + kNK * KS;
  static constexpr int P_OFF = V_OFF + kNK * VS;
  static constexpr int FLOATS = P_OFF + MQ * kPS;
  static constexpr int BYTES = FLOATS * 4 + 4 * 8;  // + 3 mbarriers (8-byte aligned)
};

// BM: bias mode, 0 none, 1 an expanded [H, Lq, Lk] bias, 2 a T5 relative-bias table.
template <int DT, int MQ, int BM, bool ALIGNED>
__global__ void __launch_bounds__(kThreads) attn_fp32_kernel(const AttnLaunch L) {
  constexpr bool BIAS = BM != 0;
  using G = Geom<DT, MQ>;
  constexpr int TM = G::TM;
  constexpr int U = G::U;
  extern __shared__ __align__(128) float smem[];
  float* Qs = smem + G::Q_OFF;
  float* Ks = smem + G::K_OFF;
  float* Vs = smem + G::V_OFF;
  float* Ps = smem + G::P_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::FLOATS);  // [0] Q, [1] K, [2] V

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int rg = warp * 4 + (lane >> 3);
  const int cg = lane & 7;

  const int t = blockIdx.x;
  if (t >= L.total) {
    if (tid == 0) report_error(L.status, DEV_BAD_TILE, 0);
    return;
  }
  const int pidx = find_problem(L.begin, L.n, t);
  const AttnProb* __restrict__ pp = L.probs + pidx;
  const int local = t - __ldg(L.begin + pidx);
  const int q_tiles = pp->q_tiles;
  const int h = local / q_tiles;
  const int q0 = (local - h * q_tiles) * MQ;
  const int Lq = pp->Lq, Lk = pp->Lk, D = pp->D;
  const int rows_q = min(MQ, Lq - q0);
  const int nblk = (Lk + kNK - 1) / kNK;
  const int64_t ldq = pp->ldq, ldk = pp->ldk, ldv = pp->ldv;
  const float* qsrc = pp->q + pp->q_off + (int64_t)q0 * ldq + (int64_t)h * D;
  const float* ksrc = pp->k + pp->k_off + (int64_t)h * D;
  const float* vsrc = pp->v + pp->v_off + (int64_t)h * D;
  // bias: the expanded [H, Lq, Lk] array (staged per block), or a T5 table read per score
  const float* bsrc = BM == 1 ? pp->bias + ((int64_t)h * Lq + q0) * Lk : nullptr;
  const float* tab_h = BM == 2 ? pp->bias + h : nullptr;
  const int32_t* lut_c = BM == 2 ? pp->rel_lut + pp->rel_max : nullptr;
  const int32_t rel_max = BM == 2 ? pp->rel_max : 0;
  const float sl2 = pp->scale_log2;

  // ---- set-up: barriers and the zero padding the bulk copies never write -------------------------
  if (ALIGNED && tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_init(&bars[2], 1);
    mbar_fence_init();
  }
  if (D < DT) {  // head-dim padding columns of Q and K must be zero for the padded dot products
    for (int idx = tid; idx < MQ * (DT - D); idx += kThreads) {
      const int r = idx / (DT - D);
      Qs[r * G::QS + D + (idx - r * (DT - D))] = 0.f;
    }
    for (int idx = tid; idx < kNK * (DT - D); idx += kThreads) {
      const int r = idx / (DT - D);
      Ks[r * G::KS + D + (idx - r * (DT - D))] = 0.f;
    }
  }
  if (rows_q < MQ) {  // query rows past Lq: zeros keep their (never stored) scores finite
    for (int idx = tid; idx < (MQ - rows_q) * DT; idx += kThreads) {
      const int r = rows_q + idx / DT;
      Qs[r * G::QS + (idx % DT)] = 0.f;
    }
  }
  if (Lk % kNK != 0) {  // V rows past Lk meet P == 0 and must hold finite values
    float4* V4 = reinterpret_cast<float4*>(Vs);
    for (int idx = tid; idx < kNK * G::VS / 4; idx += kThreads) V4[idx] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (ALIGNED) fence_proxy_async_smem();
  __syncthreads();

  const uint32_t row_bytes = (uint32_t)D * 4u;
  auto issue_rows = [&](float* dst, int stride, const float* src, int64_t ld, int nrows, uint64_t* bar) {
    // called by warp 0 only
    if (lane == 0) mbar_arrive_expect_tx(bar, row_bytes * (uint32_t)nrows);
    __syncwarp();
    for (int r = lane; r < nrows; r += 32) bulk_g2s(dst + r * stride, src + (int64_t)r * ld, row_bytes, bar);
  };
  auto load_rows_sync = [&](float* dst, int stride, const float* src, int64_t ld, int nrows) {
    for (int idx = tid; idx < nrows * D; idx += kThreads) {
      const int r = idx / D;
      const int c = idx - r * D;
      dst[r * stride + c] = __ldg(src + (int64_t)r * ld + c);
    }
  };
  auto issue_bias = [&](int k0) {
    // each thread stages the bias of exactly the score slots it owns into its own P slots
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int r = rg + 16 * i;
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int key = k0 + cg + 8 * jj;
        const bool ok = (r < rows_q) && (key < Lk);
        cp_async4(&Ps[r * kPS + cg + 8 * jj], ok ? (const void*)(bsrc + (int64_t)r * Lk + key) : (const void*)bsrc,
                  ok ? 4u : 0u);
      }
    }
    cp_async_commit();
  };
  auto fail = [&](int stage, uint64_t* bar, uint32_t parity) {
    if (tid == 0) report_error(L.status, DEV_TIMEOUT, stage);
    // drain the copies that may still target this CTA's shared memory (bounded again)
    mbar_wait_bounded(bar, parity);
    if (BM == 1) cp_async_wait<0>();
  };

  if (ALIGNED && warp == 0) {
    issue_rows(Qs, G::QS, qsrc, ldq, rows_q, &bars[0]);
    issue_rows(Ks, G::KS, ksrc, ldk, min(kNK, Lk), &bars[1]);
    issue_rows(Vs, G::VS, vsrc, ldv, min(kNK, Lk), &bars[2]);
  }
  if (BM == 1) issue_bias(0);

  float4 o[TM][U];
  float m[TM], l[TM];
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int u = 0; u < U; ++u) o[i][u] = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  for (int j = 0; j < nblk; ++j) {
    const int k0 = j * kNK;
    const int nk = min(kNK, Lk - k0);
    const uint32_t par = (uint32_t)(j & 1);

    // ---- K_j (and Q) resident ----------------------------------------------------------------
    if (ALIGNED) {
      bool ok = true;
      if (j == 0) ok = mbar_wait_bounded(&bars[0], 0);
      ok = ok && mbar_wait_bounded(&bars[1], par);
      if (__syncthreads_or(!ok)) {
        fail(1, &bars[1], par);
        return;
      }
    } else {
      if (j == 0) load_rows_sync(Qs, G::QS, qsrc, ldq, rows_q);
      load_rows_sync(Ks, G::KS, ksrc + (int64_t)k0 * ldk, ldk, nk);
      __syncthreads();
    }

    // ---- S = Q K^T (64 keys) -----------------------------------------------------------------
    float s[TM][8];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) s[i][jj] = 0.f;
    {
      const float4* Q4 = reinterpret_cast<const float4*>(Qs) + rg * (G::QS / 4);
      const float4* K4 = reinterpret_cast<const float4*>(Ks) + cg * (G::KS / 4);
#pragma unroll 2
      for (int d4 = 0; d4 < DT / 4; ++d4) {
        float4 kf[8];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) kf[jj] = K4[jj * 8 * (G::KS / 4) + d4];
#pragma unroll
        for (int i = 0; i < TM; ++i) {
          const float4 qf = Q4[i * 16 * (G::QS / 4) + d4];
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            s[i][jj] = fmaf(qf.x, kf[jj].x, s[i][jj]);
            s[i][jj] = fmaf(qf.y, kf[jj].y, s[i][jj]);
            s[i][jj] = fmaf(qf.z, kf[jj].z, s[i][jj]);
            s[i][jj] = fmaf(qf.w, kf[jj].w, s[i][jj]);
          }
        }
      }
    }

    // ---- online softmax (exp2 domain) --------------------------------------------------------
    if (BM == 1) cp_async_wait<0>();  // this thread's own staged bias slots
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int r = rg + 16 * i;
      float mx = -INFINITY;
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        float x = s[i][jj] * sl2;
        if (BIAS) {
          const float b = BM == 2 ? t5_table_bias(tab_h, lut_c, rel_max, (uint32_t)pp->H, k0 + cg + 8 * jj - (q0 + r))
                                  : Ps[r * kPS + cg + 8 * jj];
          x = fmaf(b, kLog2e, x);
        }
        x = (cg + 8 * jj < nk) ? x : -INFINITY;
        s[i][jj] = x;
        mx = fmaxf(mx, x);
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      const float mn = fmaxf(m[i], mx);
      const float alpha = exp2f(m[i] - mn);
      m[i] = mn;
      float ls = 0.f;
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const float pe = exp2f(s[i][jj] - mn);
        ls += pe;
        Ps[r * kPS + cg + 8 * jj] = pe;
      }
      l[i] = l[i] * alpha + ls;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        o[i][u].x *= alpha;
        o[i][u].y *= alpha;
        o[i][u].z *= alpha;
        o[i][u].w *= alpha;
      }
    }
    __syncthreads();  // P complete; K_j no longer read

    if (ALIGNED && warp == 0 && j + 1 < nblk) {
      fence_proxy_async_smem();
      issue_rows(Ks, G::KS, ksrc + (int64_t)(k0 + kNK) * ldk, ldk, min(kNK, Lk - k0 - kNK), &bars[1]);
    }

    // ---- V_j resident ------------------------------------------------------------------------
    if (ALIGNED) {
      const bool ok = mbar_wait_bounded(&bars[2], par);
      if (__syncthreads_or(!ok)) {
        fail(2, &bars[2], par);
        return;
      }
    } else {
      load_rows_sync(Vs, G::VS, vsrc + (int64_t)k0 * ldv, ldv, nk);
      __syncthreads();
    }

    // ---- O += P V ----------------------------------------------------------------------------
    {
      const int k4end = (nk + 3) >> 2;
      const float4* P4 = reinterpret_cast<const float4*>(Ps) + rg * (kPS / 4);
      const float4* V4 = reinterpret_cast<const float4*>(Vs) + cg;
#pragma unroll 2
      for (int k4 = 0; k4 < k4end; ++k4) {
        float4 pf[TM];
#pragma unroll
        for (int i = 0; i < TM; ++i) pf[i] = P4[i * 16 * (kPS / 4) + k4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float4 vf[U];
#pragma unroll
          for (int u = 0; u < U; ++u) vf[u] = V4[(k4 * 4 + e) * (G::VS / 4) + 8 * u];
#pragma unroll
          for (int i = 0; i < TM; ++i) {
            const float pe = e == 0 ? pf[i].x : e == 1 ? pf[i].y : e == 2 ? pf[i].z : pf[i].w;
#pragma unroll
            for (int u = 0; u < U; ++u) {
              o[i][u].x = fmaf(pe, vf[u].x, o[i][u].x);
              o[i][u].y = fmaf(pe, vf[u].y, o[i][u].y);
              o[i][u].z = fmaf(pe, vf[u].z, o[i][u].z);
              o[i][u].w = fmaf(pe, vf[u].w, o[i][u].w);
            }
          }
        }
      }
    }
    __syncthreads();  // V_j and P no longer read

    if (j + 1 < nblk) {
      if (ALIGNED && warp == 0) {
        fence_proxy_async_smem();
        issue_rows(Vs, G::VS, vsrc + (int64_t)(k0 + kNK) * ldv, ldv, min(kNK, Lk - k0 - kNK), &bars[2]);
      }
      if (BM == 1) issue_bias(k0 + kNK);
    }
  }

  // ---- O / l, store rows < Lq ------------------------------------------------------------------
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    float ls = l[i];
    ls += __shfl_xor_sync(0xffffffffu, ls, 1);
    ls += __shfl_xor_sync(0xffffffffu, ls, 2);
    ls += __shfl_xor_sync(0xffffffffu, ls, 4);
    const float inv = 1.0f / ls;
    const int r = rg + 16 * i;
    if (r < rows_q) {
      float* dst = pp->o + pp->o_off + (int64_t)(q0 + r) * pp->ldo + (int64_t)h * D;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = 4 * (cg + 8 * u);
        const float4 v = make_float4(o[i][u].x * inv, o[i][u].y * inv, o[i][u].z * inv, o[i][u].w * inv);
        if (ALIGNED) {
          if (c < D) *reinterpret_cast<float4*>(dst + c) = v;
        } else {
          if (c + 0 < D) dst[c + 0] = v.x;
          if (c + 1 < D) dst[c + 1] = v.y;
          if (c + 2 < D) dst[c + 2] = v.z;
          if (c + 3 < D) dst[c + 3] = v.w;
        }
      }
    }
  }
}

template <int DT, int MQ, int BM, bool ALIGNED>
cudaError_t launch_one(const AttnLaunch& L, cudaStream_t s) {
  using G = Geom<DT, MQ>;
  auto k = attn_fp32_kernel<DT, MQ, BM, ALIGNED>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, G::BYTES);
  if (e != cudaSuccess) return e;
  k<<<L.total, kThreads, G::BYTES, s>>>(L);
  return cudaGetLastError();
}

template <int DT, int MQ>
cudaError_t launch_cfg(int bm, bool aligned, const AttnLaunch& L, cudaStream_t s) {
  if (bm == 2) return aligned ? launch_one<DT, MQ, 2, true>(L, s) : launch_one<DT, MQ, 2, false>(L, s);
  if (bm == 1) return aligned ? launch_one<DT, MQ, 1, true>(L, s) : launch_one<DT, MQ, 1, false>(L, s);
  return aligned ? launch_one<DT, MQ, 0, true>(L, s) : launch_one<DT, MQ, 0, false>(L, s);
}

}  // namespace

int fused_cfg_tile_rows(int cfg) {
  return cfg == CFG_D64_Q128 ? 128 : 64;
}
int fused_cfg_head_dim(int cfg) { return cfg == CFG_D128_Q64 ? 128 : 64; }

cudaError_t launch_attn_fp32(int cfg, int bias_mode, bool aligned, const AttnLaunch& L, cudaStream_t s) {
  if (L.total <= 0) return cudaSuccess;
  if (bias_mode < 0 || bias_mode > 2) return cudaErrorInvalidValue;
  switch (cfg) {
    case CFG_D64_Q128: return launch_cfg<64, 128>(bias_mode, aligned, L, s);
    case CFG_D64_Q64: return launch_cfg<64, 64>(bias_mode, aligned, L, s);
    case CFG_D128_Q64: return launch_cfg<128, 64>(bias_mode, aligned, L, s);
    default: return cudaErrorInvalidValue;
  }
}

const char* attn_fp32_name(int cfg, int bias_mode, bool aligned) {
  static const char* names[CFG_COUNT][3][2] = {
      {{"attn_fp32_d64_q128_u", "attn_fp32_d64_q128"},
       {"attn_fp32_d64_q128_bias_u", "attn_fp32_d64_q128_bias"},
       {"attn_fp32_d64_q128_t5_u", "attn_fp32_d64_q128_t5"}},
      {{"attn_fp32_d64_q64_u", "attn_fp32_d64_q64"},
       {"attn_fp32_d64_q64_bias_u", "attn_fp32_d64_q64_bias"},
       {"attn_fp32_d64_q64_t5_u", "attn_fp32_d64_q64_t5"}},
      {{"attn_fp32_d128_q64_u", "attn_fp32_d128_q64"},
       {"attn_fp32_d128_q64_bias_u", "attn_fp32_d128_q64_bias"},
       {"attn_fp32_d128_q64_t5_u", "attn_fp32_d128_q64_t5"}},
  };
  if (cfg < 0 || cfg >= CFG_COUNT || bias_mode < 0 || bias_mode > 2) return "attn_fp32_?";
  return names[cfg][bias_mode][aligned ? 1 : 0];
}

}  // namespace supra
