// Fused FP32 attention, warp-independent pipeline (sm_100a): D <= 64, no bias, 16-byte aligned rows.
// The DiT self/cross-attention kernel (app/models/dit.js:172,184).
//
// Same algorithm as attn_fp32.cu (online softmax over key blocks, app/gpu/kernels.js:164-316),
// reorganised so that the main loop has no block-wide barrier:
//  * 4 warps x 32 query rows (128-row tile). Lane (rg = lane/8, cg = lane%8) of warp w owns rows
//    32w + rg + 4i (i < 8), keys cg + 8j (j < 4) of each 32-key block and output columns
//    4*(cg + 8u) .. +3 (u < 2): 8x4 score and 8x8 output register blocks.
//  * Each warp stages its own 32 Q rows (bulk copies, its own mbarrier) and keeps its own P tile,
//    so softmax -> PV needs only __syncwarp.
//  * K/V blocks flow through a 3-stage ring of shared-memory stages filled by the bulk-copy (TMA)
//    engine with one "full" mbarrier per stage (expect_tx). A warp that has finished a stage
//    counts itself out on the stage's counter; the last warp out issues the refill for the block
//    three ahead, so no warp ever waits for a producer and warps drift freely.
//  * Lazy rescaling: the running row maximum used as the exp2 offset is only moved when a block
//    exceeds it by more than 8 (a factor 256), so the O/l rescale is skipped on almost every block;
//    the result is the same softmax (O and l always share one offset).
//  * exp2 via ex2.approx.ftz (relative error ~2^-22), scale*log2(e) folded into the scores.
//  * Ragged last blocks: whole 8-key groups past Lk are skipped in QK^T and PV; the rest are masked.
//  * All waits are bounded (2 s); a timeout sets the device status word and the warp leaves.
#include "common.cuh"

namespace supra {
namespace {

constexpr int kW = 4;           // consumer warps per CTA
constexpr int kRows = 32 * kW;  // query rows per tile
constexpr int kNK = 32;         // keys per block
constexpr int kNS = 3;          // K/V stages
constexpr int kD = 64;          // head-dim capacity
constexpr int kQS = kD + 4;     // Q row stride (floats)
constexpr int kKS = kD + 4;     // K row stride
constexpr int kVS = kD;         // V row stride
constexpr int kPS = kNK + 8;    // P row stride: conflict-free scalar writes and float4 reads

constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + kRows * kQS;
constexpr int OFF_V = OFF_K + kNS * kNK * kKS;
constexpr int OFF_P = OFF_V + kNS * kNK * kVS;
constexpr int FLOATS = OFF_P + kW * 32 * kPS;
// barriers: qbar[kW], full[kNS] (8 B each), then the stage counters cnt[kNS] (4 B each)
constexpr int BYTES = FLOATS * 4 + (kW + kNS) * 8 + kNS * 4 + 4;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(kW * 32, 2) attn_fp32_w4_kernel(const AttnLaunch L) {
  extern __shared__ __align__(128) float smem[];
  float* Qs = smem + OFF_Q;
  float* Ks = smem + OFF_K;
  float* Vs = smem + OFF_V;
  uint64_t* qbar = reinterpret_cast<uint64_t*>(smem + FLOATS);
  uint64_t* full = qbar + kW;
  int* cnt = reinterpret_cast<int*>(full + kNS);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int w = tid >> 5;
  const int rg = lane >> 3;
  const int cg = lane & 7;
  float* Pw = smem + OFF_P + w * 32 * kPS;

  const int t = blockIdx.x;
  if (t >= L.total) {
    if (tid == 0) report_error(L.status, DEV_BAD_TILE, 0);
    return;
  }
  const int pidx = L.uniform > 0 ? t / L.uniform : find_problem(L.begin, L.n, t);
  const AttnProb* __restrict__ pp = L.probs + pidx;
  const int local = t - (L.uniform > 0 ? pidx * L.uniform : __ldg(L.begin + pidx));
  const int q_tiles = pp->q_tiles;
  const int h = local / q_tiles;
  const int q0 = (local - h * q_tiles) * kRows;
  const int Lq = pp->Lq, Lk = pp->Lk, D = pp->D;
  const int rows_q = min(kRows, Lq - q0);
  const int nwa = (rows_q + 31) >> 5;  // warps with at least one valid row
  const int nblk = (Lk + kNK - 1) / kNK;
  const int64_t ldq = pp->ldq, ldk = pp->ldk, ldv = pp->ldv;
  const float* qsrc = pp->q + pp->q_off + (int64_t)q0 * ldq + (int64_t)h * D;
  const float* ksrc = pp->k + pp->k_off + (int64_t)h * D;
  const float* vsrc = pp->v + pp->v_off + (int64_t)h * D;
  const float sl2 = pp->scale_log2;
  const uint32_t row_bytes = (uint32_t)D * 4u;

  // ---- set-up (the kernel's only block-wide barrier) ------------------------------------------------
  if (tid == 0) {
    for (int i = 0; i < kW; ++i) mbar_init(&qbar[i], 1);
    for (int s = 0; s < kNS; ++s) {
      mbar_init(&full[s], 1);
      cnt[s] = 0;
    }
    mbar_fence_init();
  }
  if (D < kD) {  // padding columns of Q and K take part in the dot products: zero them
    for (int idx = tid; idx < kRows * (kD - D); idx += kW * 32) {
      const int r = idx / (kD - D);
      Qs[r * kQS + D + (idx - r * (kD - D))] = 0.f;
    }
    for (int idx = tid; idx < kNS * kNK * (kD - D); idx += kW * 32) {
      const int r = idx / (kD - D);
      Ks[r * kKS + D + (idx - r * (kD - D))] = 0.f;
    }
  }
  if (rows_q < kRows) {  // query rows past Lq: keep their (never stored) scores finite
    for (int idx = tid; idx < (kRows - rows_q) * kD; idx += kW * 32) {
      const int r = rows_q + idx / kD;
      Qs[r * kQS + (idx % kD)] = 0.f;
    }
  }
  if (Lk % kNK != 0) {  // V rows past Lk meet P == 0 and must hold finite values
    float4* V4 = reinterpret_cast<float4*>(Vs);
    for (int idx = tid; idx < kNS * kNK * kVS / 4; idx += kW * 32) V4[idx] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (w >= nwa) return;  // no valid rows: this warp takes no part (nwa counts the stage users)

  // K and V rows of block b into stage s, issued by one warp
  auto issue_block = [&](int b, int s) {
    const int k0 = b * kNK;
    const int nk = min(kNK, Lk - k0);
    if (lane == 0) mbar_arrive_expect_tx(&full[s], 2u * row_bytes * (uint32_t)nk);
    __syncwarp();
    float* kd = Ks + s * kNK * kKS;
    float* vd = Vs + s * kNK * kVS;
    for (int r = lane; r < nk; r += 32) {
      bulk_g2s(kd + r * kKS, ksrc + (int64_t)(k0 + r) * ldk, row_bytes, &full[s]);
      bulk_g2s(vd + r * kVS, vsrc + (int64_t)(k0 + r) * ldv, row_bytes, &full[s]);
    }
  };

  // own Q rows
  const int my_rows = min(32, rows_q - 32 * w);
  if (lane == 0) mbar_arrive_expect_tx(&qbar[w], row_bytes * (uint32_t)my_rows);
  __syncwarp();
  for (int r = lane; r < my_rows; r += 32)
    bulk_g2s(Qs + (32 * w + r) * kQS, qsrc + (int64_t)(32 * w + r) * ldq, row_bytes, &qbar[w]);
  if (w == 0)
    for (int b = 0; b < min(kNS, nblk); ++b) issue_block(b, b);

  float4 o[8][2];
  float mo[8], l[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    mo[i] = -INFINITY;
    l[i] = 0.f;
    o[i][0] = o[i][1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  if (!mbar_wait_bounded(&qbar[w], 0)) {
    if (lane == 0) report_error(L.status, DEV_TIMEOUT, 10);
    return;
  }
  const float4* Q4 = reinterpret_cast<const float4*>(Qs) + (32 * w + rg) * (kQS / 4);

  for (int j = 0; j < nblk; ++j) {
    const int s = j % kNS;
    const uint32_t par = (uint32_t)((j / kNS) & 1);
    const int nk = min(kNK, Lk - j * kNK);
    if (!mbar_wait_bounded(&full[s], par)) {
      if (lane == 0) report_error(L.status, DEV_TIMEOUT, 11);
      return;
    }
    const float4* K4 = reinterpret_cast<const float4*>(Ks + s * kNK * kKS) + cg * (kKS / 4);
    const float4* V4 = reinterpret_cast<const float4*>(Vs + s * kNK * kVS) + cg;

    // ---- S = Q K^T. Component-major order: for each 4-deep slice of the head dim, the 32
    // products of one component are independent FFMAs, so no accumulator waits on its previous
    // update. Keys past Lk in a partial block are computed from stale rows and masked below.
    float sc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) sc[i][jj] = 0.f;
#pragma unroll 2
    for (int d4 = 0; d4 < kD / 4; ++d4) {
      float4 kf[4], qf[8];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) kf[jj] = K4[jj * 8 * (kKS / 4) + d4];
#pragma unroll
      for (int i = 0; i < 8; ++i) qf[i] = Q4[i * 4 * (kQS / 4) + d4];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) sc[i][jj] = fmaf(qf[i].x, kf[jj].x, sc[i][jj]);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) sc[i][jj] = fmaf(qf[i].y, kf[jj].y, sc[i][jj]);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) sc[i][jj] = fmaf(qf[i].z, kf[jj].z, sc[i][jj]);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) sc[i][jj] = fmaf(qf[i].w, kf[jj].w, sc[i][jj]);
    }
    if (nk < kNK) {  // partial block (warp-uniform): mask the keys past Lk
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) sc[i][jj] = (cg + 8 * jj < nk) ? sc[i][jj] : -INFINITY;
    }

    // ---- softmax with a lazily moved offset (exp2 domain). scale > 0 (host-checked), so the
    // maximum of the raw scores times scale*log2(e) is the maximum of the scaled scores.
    bool any_move = false;
    float mprev[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float mr = fmaxf(fmaxf(sc[i][0], sc[i][1]), fmaxf(sc[i][2], sc[i][3]));
      mr = fmaxf(mr, __shfl_xor_sync(0xffffffffu, mr, 1));
      mr = fmaxf(mr, __shfl_xor_sync(0xffffffffu, mr, 2));
      mr = fmaxf(mr, __shfl_xor_sync(0xffffffffu, mr, 4));
      const float mx = mr * sl2;
      mprev[i] = mo[i];
      if (mx > mo[i] + 8.f) {
        mo[i] = mx;
        any_move = true;
      }
    }
    if (__any_sync(0xffffffffu, any_move)) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float alpha = ex2(mprev[i] - mo[i]);
        l[i] *= alpha;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          o[i][u].x *= alpha;
          o[i][u].y *= alpha;
          o[i][u].z *= alpha;
          o[i][u].w *= alpha;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const float pe = ex2(fmaf(sc[i][jj], sl2, -mo[i]));
        l[i] += pe;
        Pw[(rg + 4 * i) * kPS + cg + 8 * jj] = pe;
      }
    }
    __syncwarp();

    // ---- O += P V ----------------------------------------------------------------------------
    {
      const float4* P4 = reinterpret_cast<const float4*>(Pw) + rg * (kPS / 4);
      const int k4end = (nk + 3) >> 2;  // groups of 4 keys with a valid key (8 in full blocks)
#pragma unroll 2
      for (int k4 = 0; k4 < k4end; ++k4) {
        float4 pf[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pf[i] = P4[i * 4 * (kPS / 4) + k4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float4 v0 = V4[(k4 * 4 + e) * (kVS / 4)];
          const float4 v1 = V4[(k4 * 4 + e) * (kVS / 4) + 8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float pe = e == 0 ? pf[i].x : e == 1 ? pf[i].y : e == 2 ? pf[i].z : pf[i].w;
            o[i][0].x = fmaf(pe, v0.x, o[i][0].x);
            o[i][0].y = fmaf(pe, v0.y, o[i][0].y);
            o[i][0].z = fmaf(pe, v0.z, o[i][0].z);
            o[i][0].w = fmaf(pe, v0.w, o[i][0].w);
            o[i][1].x = fmaf(pe, v1.x, o[i][1].x);
            o[i][1].y = fmaf(pe, v1.y, o[i][1].y);
            o[i][1].z = fmaf(pe, v1.z, o[i][1].z);
            o[i][1].w = fmaf(pe, v1.w, o[i][1].w);
          }
        }
      }
    }
    __syncwarp();  // every lane is done with P and with stage s

    // ---- release stage s; the last warp out refills it with block j + kNS ------------------------
    int last = 0;
    if (lane == 0) {
      __threadfence_block();
      last = (atomicAdd(&cnt[s], 1) == nwa - 1);
      if (last) {
        atomicExch(&cnt[s], 0);
        __threadfence_block();
      }
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last && j + kNS < nblk) {
      fence_proxy_async_smem();
      issue_block(j + kNS, s);
    }
  }

  // ---- O / l, rows < Lq ----------------------------------------------------------------------
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float ls = l[i];
    ls += __shfl_xor_sync(0xffffffffu, ls, 1);
    ls += __shfl_xor_sync(0xffffffffu, ls, 2);
    ls += __shfl_xor_sync(0xffffffffu, ls, 4);
    const float inv = 1.0f / ls;
    const int r = 32 * w + rg + 4 * i;
    if (r < rows_q) {
      float* dst = pp->o + pp->o_off + (int64_t)(q0 + r) * pp->ldo + (int64_t)h * D;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int c = 4 * (cg + 8 * u);
        if (c < D)
          *reinterpret_cast<float4*>(dst + c) =
              make_float4(o[i][u].x * inv, o[i][u].y * inv, o[i][u].z * inv, o[i][u].w * inv);
      }
    }
  }
}

}  // namespace

int attn_fp32_w4_tile_rows() { return kRows; }

cudaError_t launch_attn_fp32_w4(const AttnLaunch& L, cudaStream_t s) {
  if (L.total <= 0) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(attn_fp32_w4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BYTES);
  if (e != cudaSuccess) return e;
  attn_fp32_w4_kernel<<<L.total, kW * 32, BYTES, s>>>(L);
  return cudaGetLastError();
}

}  // namespace supra
