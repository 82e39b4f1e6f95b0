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
#include <type_traits>

#include "common.cuh"
#include "tcgen05.cuh"

namespace supra {
namespace {

constexpr int kT = 256;   // threads
constexpr int kBM = 128;  // rows per tile
constexpr int kBK = 16;   // reduction depth per stage
constexpr int kS = kBK + 4;  // row stride of the stage buffers (conflict-free float4 reads)
// k stages in flight: the load of stage s + stages - 1 is issued while stage s is computed. With
// two (one load ahead) a 128 x 64 tile's stage compute, about 1 us, did not cover its load's
// latency from L2, and such a tile took as long as a 128 x 128 one; four stages for the 64-column
// tiles, two for the 128-column tiles (whose 64 accumulators leave no registers for deeper
// address bookkeeping under the two-CTA bound: four stages spilled ~1 KB there).
template <int BN>
constexpr int stages_of() { return BN == 64 ? 4 : 2; }
// dynamic shared memory of the form (the two-stage form's arrays are static)
template <int BN>
constexpr int smem_bytes() { return stages_of<BN>() == 2 ? 0 : stages_of<BN>() * (kBM + BN) * kS * 4; }
// the TMA-staged form: 32-deep stages (one pair of barriers per 32 k), two in flight (a stage's
// products take several microseconds, well over a copy's latency from L2), 128-byte aligned boxes
// of kLinBoxCols columns, one mbarrier per stage
constexpr int kTmaStages = 2;
constexpr int kBKT = kLinBoxCols - 4;  // reduction depth per stage
constexpr int kST = kLinBoxCols;       // row stride of the stage buffers
// x^T of the stage being computed: [kBKT][kTS], row r of x at position 8 (r % 16) + r / 16, so a
// thread's 8 rows (rg + 16i) are two float4 at 8rg
constexpr int kTS = kBM + 4;
// a stage's W tile: [BN][kST] (W as [N, K]) or [kBKT][BN] (W as [K, N], w_kn)
template <int BN, bool WKN>
constexpr int w_stage_floats() { return WKN ? kBKT * BN : BN * kST; }
template <int BN, bool WKN>
constexpr int tma_smem_bytes() {
  return 128 + (kTmaStages * (kBM * kST + w_stage_floats<BN, WKN>()) + kBKT * kTS) * 4 + kTmaStages * 8;
}

// GroupNorm (+ SiLU) or LayerNorm (+ modulation) of a staged x tile `a` (stage st of the tile at
// rows r0.., nr of them valid), per element of a valid row and column (padding stays zero):
// (x - mean) * rstd * g + b with g, b = gamma, beta (app/gpu/kernels.js:141-162), 1 + scale, shift
// (app/gpu/kernels.js:111) or 1, 0. Thread tid normalises column kk = tid % 16 of the stage in rows
// tid / 16 + 16 i: its column's g, b and group are one lookup per stage, its rows' images one per
// tile. (Per element, with two integer divisions and three global loads, it cost as much as the
// stage's FMAs.)
template <int BK = kBK, int S = kS>
__device__ __forceinline__ void norm_stage(const LinProb& P, float* a, int st, int r0, int nr, int tid) {
  const int kk = tid % BK, rb = tid / BK;
  const int k = st * BK + kk;
  if (k >= P.K) return;
  float g = 1.f, b = 0.f;
  if (P.gn_mode != kNormPlain) {
    g = __ldg(P.gamma + k);
    b = __ldg(P.beta + k);
    if (P.gn_mode == kNormModulated) g = 1.f + g;
  }
  const float2* st_k = P.gn_stats + k / P.gn_cg;  // the column's group
  // a row's image: one for the whole tile when images are whole tiles (the VAE's 1024-row
  // images), the row itself for a LayerNorm
  const bool one_img = P.gn_rows % kBM == 0;
  const int img0 = one_img ? r0 / P.gn_rows : 0;
#pragma unroll
  for (int it = 0; it < kBM * BK / kT; ++it) {
    const int r = rb + (kT / BK) * it;
    if (r < nr) {
      const int img = one_img ? img0 : (P.gn_rows == 1 ? r0 + r : (r0 + r) / P.gn_rows);
      const float2 ms = __ldg(st_k + (int64_t)img * P.gn_groups);
      float v = (a[r * S + kk] - ms.x) * (ms.y * g) + b;
      if (P.gn_silu) v = v / (1.f + __expf(-v));
      a[r * S + kk] = v;
    }
  }
}

// acc += the stage's x tile (rows rg + 16i) times its W tile (rows cg + 16j), kBK deep
template <int NJ>
__device__ __forceinline__ void mma_stage(const float* a, const float* b, int rg, int cg, float (&acc)[8][NJ]) {
  const float4* A4 = reinterpret_cast<const float4*>(a) + rg * (kS / 4);
  const float4* B4 = reinterpret_cast<const float4*>(b) + cg * (kS / 4);
#pragma unroll
  for (int k4 = 0; k4 < kBK / 4; ++k4) {
    float4 bf[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) bf[j] = B4[j * 16 * (kS / 4) + k4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 af = A4[i * 16 * (kS / 4) + k4];
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        acc[i][j] = fmaf(af.x, bf[j].x, acc[i][j]);
        acc[i][j] = fmaf(af.y, bf[j].y, acc[i][j]);
        acc[i][j] = fmaf(af.z, bf[j].z, acc[i][j]);
        acc[i][j] = fmaf(af.w, bf[j].w, acc[i][j]);
      }
    }
  }
}

// The stage's x tile `a` ([kBM][kS], row-major) into x^T `at`: thread tid moves rows rg + 16 (2ip)
// and rg + 16 (2ip + 1) (rg = tid % 16, ip = tid / 16 % 4) of k4 group tid / 64, two float4 loads
// and four float2 stores (the two rows sit side by side in x^T).
__device__ __forceinline__ void transpose_stage(const float* __restrict__ a, float* __restrict__ at, int tid) {
  const int rg = tid & 15, ip = (tid >> 4) & 3;
  const int r = rg + 32 * ip;
#pragma unroll
  for (int k4 = tid >> 6; k4 < kBKT / 4; k4 += kT / 64) {
    const float4 x0 = *reinterpret_cast<const float4*>(a + r * kST + 4 * k4);
    const float4 x1 = *reinterpret_cast<const float4*>(a + (r + 16) * kST + 4 * k4);
    float* d = at + (4 * k4) * kTS + 8 * rg + 2 * ip;
    *reinterpret_cast<float2*>(d) = make_float2(x0.x, x1.x);
    *reinterpret_cast<float2*>(d + kTS) = make_float2(x0.y, x1.y);
    *reinterpret_cast<float2*>(d + 2 * kTS) = make_float2(x0.z, x1.z);
    *reinterpret_cast<float2*>(d + 3 * kTS) = make_float2(x0.w, x1.w);
  }
}

// acc += the stage's x^T (rows rg + 16i in pairs: acc[p][j] holds rows rg + 32p (x) and
// rg + 32p + 16 (y)) times its W tile (rows cg + 16j), kBK deep, with packed f32x2 FMAs: one W
// value (broadcast) times the x values of two rows
template <int NJ, bool WKN>
__device__ __forceinline__ void mma_stage_t(const float* at, const float* b, int rg, int cg, float2 (&acc)[4][NJ]) {
  const float4* A4 = reinterpret_cast<const float4*>(at) + 2 * rg;
  const float4* B4 = reinterpret_cast<const float4*>(b) + (WKN ? cg : cg * (kST / 4));
#pragma unroll
  for (int k4 = 0; k4 < kBKT / 4; ++k4) {
    // W as [N, K]: column cg + 16j's 4 values of k (one float4 each); as [K, N] (w_kn): row k's
    // columns 4cg .. 4cg + 3 and 64 + 4cg .. + 3 (one or two float4 per k)
    float4 bf[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j)
      bf[j] = WKN ? B4[(4 * k4 + (j & 3)) * (NJ * 4) + 16 * (j >> 2)] : B4[j * 16 * (kST / 4) + k4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float4 q0 = A4[(4 * k4 + e) * (kTS / 4)];
      const float4 q1 = A4[(4 * k4 + e) * (kTS / 4) + 1];
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        // W as [K, N]: bf[(j & 4) | e] holds row k = 4 k4 + e; column j is its component j & 3
        const float4 bw = WKN ? bf[(j & 4) | e] : bf[j];
        const int comp = WKN ? (j & 3) : e;
        const float w = comp == 0 ? bw.x : comp == 1 ? bw.y : comp == 2 ? bw.z : bw.w;
        const float2 w2 = make_float2(w, w);
        acc[0][j] = __ffma2_rn(make_float2(q0.x, q0.y), w2, acc[0][j]);
        acc[1][j] = __ffma2_rn(make_float2(q0.z, q0.w), w2, acc[1][j]);
        acc[2][j] = __ffma2_rn(make_float2(q1.x, q1.y), w2, acc[2][j]);
        acc[3][j] = __ffma2_rn(make_float2(q1.z, q1.w), w2, acc[3][j]);
      }
    }
  }
}

// y rows r0 + rg + 16i, columns c0 + cg + 16j: each store instruction writes two 64-byte row runs
// the tile column of a thread's column j: cg + 16j, or (WKN, the form that reads W as [K, N])
// 4cg + j for j < 4 and 64 + 4cg + j - 4 above
template <bool WKN>
__device__ __forceinline__ int col_of(int cg, int j) {
  return WKN ? 4 * cg + (j & 3) + 64 * (j >> 2) : cg + 16 * j;
}

template <bool BIAS, int NJ, bool WKN = false>
__device__ __forceinline__ void linear_epilogue(const LinProb& P, const float (&acc)[8][NJ], int r0, int c0, int nr,
                                                int nc, int rg, int cg) {
  float bias[NJ], gate[NJ];
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int c = col_of<WKN>(cg, j);
    bias[j] = (BIAS && c < nc) ? __ldg(P.bias + c0 + c) : 0.f;
    gate[j] = (P.gate && c < nc) ? __ldg(P.gate + c0 + c) : 1.f;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = rg + 16 * i;
    if (r >= nr) continue;
    float* yrow = P.y + (int64_t)(r0 + r) * P.ldy + c0;
    // resid may be y itself (in place): each element is read and then written by this thread only.
    // The row's residuals are all loaded before any of its stores (with y and resid possibly the
    // same array, a load after a store would wait for it: one memory round trip per element).
    const float* rrow = P.resid ? P.resid + (int64_t)(r0 + r) * P.ldr + c0 : nullptr;
    float rv[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int c = col_of<WKN>(cg, j);
      rv[j] = (rrow && c < nc) ? rrow[c] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int c = col_of<WKN>(cg, j);
      if (c < nc) {
        float v = acc[i][j] + bias[j];
        if (P.act != kActNone) v = linear_act(P.act, v);
        if (P.gate) v *= gate[j];
        yrow[c] = rv[j] + v;
      }
    }
  }
}

// BN: columns per tile, 128 or 64 (the host picks per launch the width that fills the last wave
// of tiles best: the DiT blocks' N = 576 products are 320 tiles of 128 x 128, 1.08 waves of the
// 296 CTA slots, against 576 tiles of 128 x 64). Thread (rg, cg) owns rows rg + 16i (i < 8) and
// columns cg + 16j (j < BN / 16).

// Tiles staged by TMA (x and W 16-byte aligned with row strides of a multiple of 4 floats): per
// stage thread 0 issues two tensor copies, a [128 x 36] box of x and a [BN x 36] box of W (the 4
// columns past the stage's 32 pad the shared-memory rows against bank conflicts and are never
// read; past K and past the last row the copies read zeros), completing on the stage's mbarrier,
// one stage ahead. The 256 threads only compute: the per-thread cp.async form spent a third of
// its issue slots on copy addresses and predicates. Each stage's x tile is first transposed in
// shared memory (x^T, 8 values per thread), so that the products run as packed f32x2 FMAs of two
// rows' x values by one W value: half the FMA instructions of the scalar form (which, with its
// 16 fragment loads per 256 FMAs, kept the schedulers near their issue limit), as the 256-row
// attention kernel's Q^T K does. Two barriers per stage: after the wait for the stage's copies
// (every thread is also done with the previous stage, whose buffers thread 0 then refills) and
// after the transposition.
template <bool BIAS, int BN, bool WKN>
__global__ void __launch_bounds__(kT, 2) linear_fp32_tma_kernel(const __grid_constant__ LinLaunch L) {
  constexpr int NJ = BN / 16;
  constexpr int WS = w_stage_floats<BN, WKN>();
  extern __shared__ uint8_t lin_raw[];
  const uint32_t raw = smem_u32(lin_raw);
  float* const As = reinterpret_cast<float*>(lin_raw + (((raw + 127u) & ~127u) - raw));  // [kTmaStages][kBM * kST]
  float* const Bs = As + kTmaStages * kBM * kST;                                                 // [kTmaStages][WS]
  float* const At = Bs + kTmaStages * WS;                                                        // [kBKT][kTS]
  uint64_t* const full = reinterpret_cast<uint64_t*>(At + kBKT * kTS);                           // [kTmaStages]
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
  const int c0 = (local - rt * P.n_tiles) * BN;
  const int nr = min(kBM, P.M - r0);
  const int nc = min(BN, P.N - c0);
  const int nstage = (P.K + kBKT - 1) / kBKT;
  const CUtensorMap* mx = L.maps + P.mx;
  const CUtensorMap* mw = L.maps + P.mw;
  const int tid = threadIdx.x;
  const int rg = tid >> 4, cg = tid & 15;
  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kTmaStages; ++s) mbar_init(&full[s], 1);
    mbar_fence_init();
  }
  __syncthreads();
  auto issue = [&](int st) {  // (thread 0)
    if (st < nstage) {
      const int buf = st % kTmaStages;
      mbar_arrive_expect_tx(&full[buf], (uint32_t)((kBM * kST + WS) * 4));
      tc::tma_load_2d(As + buf * kBM * kST, mx, st * kBKT, r0, &full[buf]);
      if (WKN) tc::tma_load_2d(Bs + buf * WS, mw, c0, st * kBKT, &full[buf]);  // [32 k][BN] of W as [K, N]
      else tc::tma_load_2d(Bs + buf * WS, mw, st * kBKT, c0, &full[buf]);
    }
  };
  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kTmaStages; ++s) issue(s);
  }
  float2 acc[4][NJ];
#pragma unroll
  for (int p = 0; p < 4; ++p)
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc[p][j] = make_float2(0.f, 0.f);
  for (int st = 0; st < nstage; ++st) {
    const int buf = st % kTmaStages;
    // every thread waits for the stage (bounded); a vote keeps the CTA together if a wait runs
    // out. Past it every thread is done with stage st - 1, whose buffers take stage st + 1.
    const bool ok = mbar_wait_bounded(&full[buf], (uint32_t)((st / kTmaStages) & 1));
    if (!__syncthreads_and(ok)) {
      if (tid == 0) report_error(L.status, DEV_TIMEOUT, 31, st);
      return;
    }
    if (tid == 0 && st > 0) issue(st + kTmaStages - 1);
    float* a = As + buf * kBM * kST;
    if (P.gn_stats) {
      norm_stage<kBKT, kST>(P, a, st, r0, nr, tid);
      __syncthreads();
    }
    transpose_stage(a, At, tid);
    __syncthreads();  // x^T complete
    mma_stage_t<NJ, WKN>(At, Bs + buf * WS, rg, cg, acc);
    fence_proxy_async_smem();  // this thread's reads (and norm writes) of the buffers before they are refilled
  }
  float accf[8][NJ];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < NJ; ++j) accf[i][j] = (i & 1) ? acc[i >> 1][j].y : acc[i >> 1][j].x;
  linear_epilogue<BIAS, NJ, WKN>(P, accf, r0, c0, nr, nc, rg, cg);
}

// The same product with the tiles staged by per-thread cp.async (any alignment: 4-byte copies
// when rows are not 16-byte aligned).
template <bool BIAS, bool ALIGNED, int BN>
__global__ void __launch_bounds__(kT, BN == 64 ? 3 : 2) linear_fp32_kernel(const LinLaunch L) {
  constexpr int NJ = BN / 16;
  constexpr int kStages = stages_of<BN>();
  float* As;  // [kStages][kBM * kS]
  float* Bs;  // [kStages][BN * kS]
  if constexpr (kStages == 2) {  // static arrays (40 KB), as the two-stage form always had
    __shared__ __align__(16) float sA[2 * kBM * kS];
    __shared__ __align__(16) float sB[2 * BN * kS];
    As = sA;
    Bs = sB;
  } else {
    extern __shared__ __align__(16) float lin_smem[];
    As = lin_smem;
    Bs = lin_smem + kStages * kBM * kS;
  }
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
  const int c0 = (local - rt * P.n_tiles) * BN;
  const int K = P.K;
  const float* abase = P.x + (int64_t)r0 * P.ldx;
  const float* bbase = P.w + (int64_t)c0 * P.ldw;
  const int nr = min(kBM, P.M - r0);
  const int nc = min(BN, P.N - c0);

  const int tid = threadIdx.x;
  const int rg = tid >> 4, cg = tid & 15;

  auto load_stage = [&](int buf, int k0) {
    if (ALIGNED) {
#pragma unroll
      for (int it = 0; it < 2; ++it) {  // 512 float4 of x, BN * 4 of W
        const int idx = tid + it * kT;
        const int r = idx >> 2, c4 = idx & 3;
        const int k = k0 + c4 * 4;
        const bool okA = (r < nr) && (k < K);
        cp_async16(&As[buf * kBM * kS + r * kS + c4 * 4], okA ? (const void*)(abase + (int64_t)r * P.ldx + k) : (const void*)abase,
                   okA ? 16u : 0u);
        if (it * kT < BN * 4) {
          const bool okB = (r < nc) && (k < K);
          cp_async16(&Bs[buf * BN * kS + r * kS + c4 * 4], okB ? (const void*)(bbase + (int64_t)r * P.ldw + k) : (const void*)bbase,
                     okB ? 16u : 0u);
        }
      }
    } else {
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int idx = tid + it * kT;
        const int r = idx >> 4, c = idx & 15;
        const int k = k0 + c;
        const bool okA = (r < nr) && (k < K);
        cp_async4(&As[buf * kBM * kS + r * kS + c], okA ? (const void*)(abase + (int64_t)r * P.ldx + k) : (const void*)abase,
                  okA ? 4u : 0u);
        if (it * kT < BN * 16) {
          const bool okB = (r < nc) && (k < K);
          cp_async4(&Bs[buf * BN * kS + r * kS + c], okB ? (const void*)(bbase + (int64_t)r * P.ldw + k) : (const void*)bbase,
                    okB ? 4u : 0u);
        }
      }
    }
    cp_async_commit();
  };

  float acc[8][NJ];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc[i][j] = 0.f;

  const int nstage = (K + kBK - 1) / kBK;
  if constexpr (kStages == 2) {
    load_stage(0, 0);
  } else {
#pragma unroll
    for (int s0 = 0; s0 < kStages - 1; ++s0) {  // the first kStages - 1 stages (empty groups past K)
      if (s0 < nstage) load_stage(s0, s0 * kBK);
      else cp_async_commit();
    }
  }
  for (int st = 0; st < nstage; ++st) {
    const int buf = st % kStages;
    if constexpr (kStages == 2) {  // next stage's load first, then wait for this one
      if (st + 1 < nstage) {
        load_stage((st + 1) & 1, (st + 1) * kBK);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
    } else {
      cp_async_wait<kStages - 2>();  // stage st has landed (one commit group per stage)
      __syncthreads();               // ... for every thread; and every thread is done with stage st - 1
      if (st + kStages - 1 < nstage) load_stage((st + kStages - 1) % kStages, (st + kStages - 1) * kBK);
      else cp_async_commit();
    }
    if (P.gn_stats) {
      norm_stage(P, As + buf * kBM * kS, st, r0, nr, tid);
      __syncthreads();
    }
    mma_stage<NJ>(As + buf * kBM * kS, Bs + buf * BN * kS, rg, cg, acc);
    if constexpr (kStages == 2) __syncthreads();  // the next iteration's load overwrites this buffer
  }
  linear_epilogue<BIAS, NJ>(P, acc, r0, c0, nr, nc, rg, cg);
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

// x normalised once into dst ([M, K] dense), for products whose x tiles would otherwise be
// normalised again by every column tile: the same arithmetic as norm_stage, one float4 per thread.
__global__ void __launch_bounds__(256) norm_apply_kernel(const LinProb P, float* __restrict__ dst) {
  const int64_t k4n = P.K / 4;
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (i >= (int64_t)P.M * k4n) return;
  const int r = (int)(i / k4n);
  const int k = (int)(i - (int64_t)r * k4n) * 4;
  const int img = P.gn_rows == 1 ? r : r / P.gn_rows;
  const float4 x = __ldg(reinterpret_cast<const float4*>(P.x + (int64_t)r * P.ldx + k));
  float v[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    float g = 1.f, b = 0.f;
    if (P.gn_mode != kNormPlain) {
      g = __ldg(P.gamma + k + u);
      b = __ldg(P.beta + k + u);
      if (P.gn_mode == kNormModulated) g = 1.f + g;
    }
    const float2 ms = __ldg(P.gn_stats + (int64_t)img * P.gn_groups + (k + u) / P.gn_cg);
    float y = (v[u] - ms.x) * (ms.y * g) + b;
    if (P.gn_silu) y = y / (1.f + __expf(-y));
    v[u] = y;
  }
  *reinterpret_cast<float4*>(dst + (int64_t)r * P.K + k) = make_float4(v[0], v[1], v[2], v[3]);
}

}  // namespace

cudaError_t launch_norm_apply(const LinProb& P, float* dst, cudaStream_t s) {
  const int64_t n = (int64_t)P.M * (P.K / 4);
  if (n <= 0) return cudaSuccess;
  norm_apply_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(P, dst);
  return cudaGetLastError();
}

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

cudaError_t launch_linear_fp32(bool bias, bool aligned, int tile_cols, const LinLaunch& L, cudaStream_t s) {
  if (L.total <= 0) return cudaSuccess;
  cudaError_t e = cudaSuccess;
  auto go = [&](auto kern, int bytes) {
    if (bytes > 0) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) kern<<<L.total, kT, bytes, s>>>(L);
  };
  auto pick = [&](auto bn) {
    constexpr int BN = decltype(bn)::value;
    constexpr int bytes = smem_bytes<BN>();
    if (bias) {
      if (aligned) go(linear_fp32_kernel<true, true, BN>, bytes);
      else go(linear_fp32_kernel<true, false, BN>, bytes);
    } else {
      if (aligned) go(linear_fp32_kernel<false, true, BN>, bytes);
      else go(linear_fp32_kernel<false, false, BN>, bytes);
    }
  };
  if (tile_cols == 64) pick(std::integral_constant<int, 64>{});
  else pick(std::integral_constant<int, 128>{});
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_linear_fp32_tma(bool bias, int tile_cols, bool w_kn, const LinLaunch& L, cudaStream_t s) {
  if (L.total <= 0) return cudaSuccess;
  cudaError_t e = cudaSuccess;
  auto go = [&](auto kern, int bytes) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) kern<<<L.total, kT, bytes, s>>>(L);
  };
  if (w_kn) {  // (the score path's O = P V: no bias)
    if (tile_cols == 64) go(linear_fp32_tma_kernel<false, 64, true>, tma_smem_bytes<64, true>());
    else go(linear_fp32_tma_kernel<false, 128, true>, tma_smem_bytes<128, true>());
  } else if (tile_cols == 64) {
    if (bias) go(linear_fp32_tma_kernel<true, 64, false>, tma_smem_bytes<64, false>());
    else go(linear_fp32_tma_kernel<false, 64, false>, tma_smem_bytes<64, false>());
  } else {
    if (bias) go(linear_fp32_tma_kernel<true, 128, false>, tma_smem_bytes<128, false>());
    else go(linear_fp32_tma_kernel<false, 128, false>, tma_smem_bytes<128, false>());
  }
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace supra
