// Fused FP32 attention, persistent kernel for large unbiased launches (sm_100a): D = 64, scale > 0,
// no score bias. The DiT self- and cross-attention launches (app/models/dit.js:172,184) when they
// hold enough 256-row tiles to fill the device; smaller launches, and the T5 encoder's biased
// ones, run on attn_fp32_warp.cu.
//
// Same algorithm as attn_fp32_warp.cu (online softmax over key blocks, app/gpu/kernels.js:164-316,
// persistent CTAs claiming tiles from a counter, a K/V ring that runs across tiles, lazy exp2
// offsets), with a larger register block per lane for Q K^T:
//  * One CTA per SM, 8 warps x 32 query rows: a tile is 256 query rows of one head, so the DiT's
//    K/V blocks are read once per (sequence, head).
//  * 64-key blocks. Lane (rg = lane/8, cg = lane%8) of warp w owns rows 32w + rg + 4i (i < 8),
//    keys cg + 8j (j < 8) of each block, and output columns 4cg .. +3, 32 + 4cg .. +3: 8x8 score
//    and 8x8 output register blocks. With 8 keys per lane instead of 4, each Q fragment load feeds
//    twice the products: per four head-dim steps a lane loads 8 Q and 8 K float4 fragments for
//    128 packed FMAs (attn_fp32_warp.cu: 12 loads for 64), and the Q K^T loop runs at about the
//    rate of the P V loop (80 % of the FMA pipe in isolation at two warps per scheduler, against
//    71 % for the 8x4 block).
//  * Row-pair packing: a packed f32x2 FMA multiplies the Q values of two of the lane's rows by one
//    K value (broadcast) into the two rows' scores of that key, so a score needs one register.
//    For that the warp transposes its 32 Q rows in place once per tile (Q^T [64 d][32]): the two
//    rows of a pair must sit side by side. Position 8rg + i of a Q^T row holds row rg + 4i, so a
//    lane's 8 rows are two float4 loads and pairs (i, i+1) are the halves of a float4.
//  * Operands by TMA tensor copies with the same tensor maps as attn_fp32_warp.cu: a warp's Q rows
//    as one [32 x 68] box, a K/V block as two [32 x 68] K and two [32 x 64] V boxes (the second
//    pair only if the block has keys past 32). Two stages (211 KB of shared memory with the P
//    rows); the last of the 8 warps to finish a stage issues the block two ahead into it.
//  * Softmax on the row pairs (f32x2 FMA for the exp2 arguments, f32x2 adds for the sums); P goes
//    to shared memory transposed (P^T [key][position], two float4 stores per key), and the
//    probabilities of keys 32..63 are formed inside the P V of keys 0..31, so that their exp2 (on
//    the SFU) overlap the products (on the FMA pipe).
//  * Ragged last blocks: keys past Lk take -inf scores (a select), Q^T K runs over the 16-key
//    groups that hold a key below Lk, and P V skips the 4-key groups past Lk (V rows past Lk are
//    never read).
//  * Whole 32-row output blocks are staged in the warp's P^T buffer and leave by TMA store.
//  * All waits are bounded (2 s); a timeout sets the device status word and the warp leaves.
#include "common.cuh"
#include "tcgen05.cuh"

namespace supra {
namespace {

constexpr int kW = 8;              // warps per CTA
constexpr int kRI = 8;             // query rows per lane
constexpr int kRowsW = 4 * kRI;    // query rows per warp
constexpr int kRows = kW * kRowsW; // query rows per tile
constexpr int kNK = 64;            // keys per block
constexpr int kBox = kFwBoxRows;   // rows per TMA box (32): a block is two K and two V boxes
constexpr int kNS = 2;             // K/V stages
constexpr int kD = 64;             // head dim
constexpr int kQS = kFwBoxWide;    // Q box row stride in shared memory (floats)
constexpr int kKS = kFwBoxWide;    // K row stride
constexpr int kVS = kFwBoxNarrow;  // V row stride
constexpr int kTS = kRowsW;        // Q^T row stride: 32 positions (conflict-free float4 reads)
constexpr int kPT = kRowsW + 4;    // P^T row stride: conflict-free float4 writes and reads
static_assert(kRowsW == kBox, "one Q box per warp");
static_assert(kD * kTS <= kRowsW * kQS, "Q^T fits in the warp's Q box");

constexpr uint32_t kQBytes = kRowsW * kQS * 4;
constexpr uint32_t kKBoxBytes = kBox * kKS * 4;
constexpr uint32_t kVBoxBytes = kBox * kVS * 4;

constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + kW * kRowsW * kQS;
constexpr int OFF_V = OFF_K + kNS * kNK * kKS;
constexpr int OFF_P = OFF_V + kNS * kNK * kVS;
constexpr int FLOATS = OFF_P + kW * kNK * kPT;
static_assert((OFF_K * 4) % 128 == 0 && (OFF_V * 4) % 128 == 0 && (OFF_P * 4) % 128 == 0 && kQBytes % 128 == 0 &&
                  kKBoxBytes % 128 == 0 && kVBoxBytes % 128 == 0,
              "TMA destinations are 128-byte aligned");

struct Cursor {
  int32_t t, b, nblk, Lk, mk, mv, kx, ky, vx, vy;
  int32_t k;  // the tile's position in the CTA's tile sequence
};
constexpr int kTileSlots = 8;
struct Ctl {
  uint64_t qbar[kW];
  uint64_t full[kNS];
  int32_t cnt[kNS];
  Cursor cur;
  int32_t tiles[kTileSlots];
};
constexpr int BYTES = FLOATS * 4 + (int)sizeof(Ctl) + 128;
static_assert(BYTES <= 232448, "shared memory per CTA");

struct Tile {
  const TmaProb* p;
  int h, q0;
};
// Within a problem, tile local = h * q_tiles + query tile (TmaProb::q_tiles counts 256-row tiles).
__device__ __forceinline__ Tile tile_of(const TmaLaunch& L, int t) {
  const int pidx = L.uniform > 0 ? t / L.uniform : find_problem(L.begin, L.n, t);
  const int local = t - (L.uniform > 0 ? pidx * L.uniform : __ldg(L.begin + pidx));
  Tile r;
  r.p = L.probs + pidx;
  const int qt = r.p->q_tiles;
  r.h = local / qt;
  r.q0 = (local - r.h * qt) * kRows;
  return r;
}

__device__ __forceinline__ void cursor_at(const TmaLaunch& L, Cursor& c, int t) {
  const Tile T = tile_of(L, t);
  c.t = t;
  c.b = 0;
  c.Lk = T.p->Lk;
  c.nblk = (c.Lk + kNK - 1) / kNK;
  c.mk = T.p->mk;
  c.mv = T.p->mv;
  c.kx = T.p->kx + T.h * kD;
  c.ky = T.p->ky;
  c.vx = T.p->vx + T.h * kD;
  c.vy = T.p->vy;
}

// Issues the cursor's block into stage s and advances the cursor (one thread); with a tile's last
// block it first claims and publishes the CTA's next tile (as attn_fp32_warp.cu).
__device__ __forceinline__ void issue_next(const TmaLaunch& L, Ctl* C, float* Ks, float* Vs, int s) {
  Cursor& c = C->cur;
  if (c.t >= L.total) return;
  int tn = 0;
  if (c.b + 1 == c.nblk) {
    tn = (int)gridDim.x + atomicAdd(L.next_tile, 1);
    C->tiles[(c.k + 1) % kTileSlots] = tn;
  }
  const int y0 = c.b * kNK;
  const bool two = c.Lk - y0 > kBox;  // keys past the first 32 of the block
  uint64_t* bar = &C->full[s];
  mbar_arrive_expect_tx(bar, (kKBoxBytes + kVBoxBytes) * (two ? 2u : 1u));
  float* kd = Ks + s * kNK * kKS;
  float* vd = Vs + s * kNK * kVS;
  tc::tma_load_2d(kd, L.maps + c.mk, c.kx, c.ky + y0, bar);
  tc::tma_load_2d(vd, L.maps + c.mv, c.vx, c.vy + y0, bar);
  if (two) {
    tc::tma_load_2d(kd + kBox * kKS, L.maps + c.mk, c.kx, c.ky + y0 + kBox, bar);
    tc::tma_load_2d(vd + kBox * kVS, L.maps + c.mv, c.vx, c.vy + y0 + kBox, bar);
  }
  if (++c.b == c.nblk) {
    ++c.k;
    if (tn < L.total) cursor_at(L, c, tn);
    else c.t = tn;
  }
}

__device__ __forceinline__ void issue_q(const TmaLaunch& L, const Tile& T, int w, float* dst, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, kQBytes);
  tc::tma_load_2d(dst, L.maps + T.p->mq, T.p->qx + T.h * kD, T.p->qy + T.q0 + w * kRowsW, bar);
}

// The warp's Q box [32 rows][68] -> Q^T [64 d][32] in place, in 4x4 blocks: row r goes to
// position 8 (r % 4) + r / 4, so rows a + 4 (b + t), t < 4, fill positions 8a + b + t. Lane (a =
// lane % 4, x = lane / 4) moves four blocks (columns 4c .. 4c + 3 of those rows): all 16 float4
// loads before any store, then 16 float4 stores. The choice of c and b per lane keeps the loads
// and the stores of each quarter-warp on 8 distinct 16-byte bank groups.
__device__ __forceinline__ void transpose_q(float* Qw, int lane) {
  const int a = lane & 3, x = lane >> 2;
  float4 f[4][4];
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const int c = 4 * (x & 1) + (x >> 1) + 8 * (m & 1);
    const int b = 4 * (((m >> 1) ^ x) & 1);
#pragma unroll
    for (int t = 0; t < 4; ++t) f[m][t] = *reinterpret_cast<const float4*>(Qw + (a + 4 * (b + t)) * kQS + 4 * c);
  }
  __syncwarp();
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const int c = 4 * (x & 1) + (x >> 1) + 8 * (m & 1);
    const int b = 4 * (((m >> 1) ^ x) & 1);
    float* dst = Qw + 4 * c * kTS + 8 * a + b;
    *reinterpret_cast<float4*>(dst) = make_float4(f[m][0].x, f[m][1].x, f[m][2].x, f[m][3].x);
    *reinterpret_cast<float4*>(dst + kTS) = make_float4(f[m][0].y, f[m][1].y, f[m][2].y, f[m][3].y);
    *reinterpret_cast<float4*>(dst + 2 * kTS) = make_float4(f[m][0].z, f[m][1].z, f[m][2].z, f[m][3].z);
    *reinterpret_cast<float4*>(dst + 3 * kTS) = make_float4(f[m][0].w, f[m][1].w, f[m][2].w, f[m][3].w);
  }
  __syncwarp();
}

// S = Q K^T for keys cg + 8j (j < NJ) of one block: acc[p][j] holds the scores of rows rg + 8p
// (x) and rg + 8p + 4 (y) for key cg + 8j.
template <int NJ>
__device__ __forceinline__ void qk_block(const float4* __restrict__ QT4, const float4* __restrict__ K4,
                                         float2 (&acc)[4][8]) {
#pragma unroll
  for (int p = 0; p < 4; ++p)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[p][j] = make_float2(0.f, 0.f);
#pragma unroll 2
  for (int d4 = 0; d4 < kD / 4; ++d4) {
    float4 kf[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) kf[j] = K4[j * 8 * (kKS / 4) + d4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float4 q0 = QT4[(4 * d4 + e) * (kTS / 4)];
      const float4 q1 = QT4[(4 * d4 + e) * (kTS / 4) + 1];
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const float kv = e == 0 ? kf[j].x : e == 1 ? kf[j].y : e == 2 ? kf[j].z : kf[j].w;
        const float2 k2 = make_float2(kv, kv);
        acc[0][j] = __ffma2_rn(make_float2(q0.x, q0.y), k2, acc[0][j]);
        acc[1][j] = __ffma2_rn(make_float2(q0.z, q0.w), k2, acc[1][j]);
        acc[2][j] = __ffma2_rn(make_float2(q1.x, q1.y), k2, acc[2][j]);
        acc[3][j] = __ffma2_rn(make_float2(q1.z, q1.w), k2, acc[3][j]);
      }
    }
  }
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float score(const float2 (&acc)[4][8], int i, int j) {
  return (i & 1) ? acc[i >> 1][j].y : acc[i >> 1][j].x;
}
// row i of a row-pair array (x: even rows, y: odd rows)
__device__ __forceinline__ float pick(const float2 (&a)[4], int i) { return (i & 1) ? a[i >> 1].y : a[i >> 1].x; }
__device__ __forceinline__ void set(float2 (&a)[4], int i, float v) {
  if (i & 1) a[i >> 1].y = v;
  else a[i >> 1].x = v;
}

__global__ void __launch_bounds__(kW * 32, 1) attn_fp32_wide_kernel(const __grid_constant__ TmaLaunch L) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  float* smem = reinterpret_cast<float*>(smem_raw + (((raw + 127u) & ~127u) - raw));
  float* Ks = smem + OFF_K;
  float* Vs = smem + OFF_V;
  Ctl* C = reinterpret_cast<Ctl*>(smem + FLOATS);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int w = tid >> 5;
  const int rg = lane >> 3;
  const int cg = lane & 7;
  float* Qw = smem + OFF_Q + w * kRowsW * kQS;
  float* Pw = smem + OFF_P + w * kNK * kPT;

  const int t0 = blockIdx.x;
  if (t0 >= L.total) {  // the host sizes the grid to at most one CTA per tile
    if (tid == 0) report_error(L.status, DEV_BAD_TILE, 60);
    return;
  }
  if (tid == 0) {
    for (int i = 0; i < kW; ++i) mbar_init(&C->qbar[i], 1);
    for (int s = 0; s < kNS; ++s) {
      mbar_init(&C->full[s], 1);
      C->cnt[s] = 0;
    }
    mbar_fence_init();
    C->tiles[0] = t0;
    C->cur.k = 0;
  }
  __syncthreads();  // the kernel's only block-wide barrier
  if (tid == 0) {
    cursor_at(L, C->cur, t0);
    for (int s = 0; s < kNS; ++s) issue_next(L, C, Ks, Vs, s);
  }
  Tile T = tile_of(L, t0);
  if (lane == 0) issue_q(L, T, w, Qw, &C->qbar[w]);

  const float4* QT4 = reinterpret_cast<const float4*>(Qw) + 2 * rg;
  const float4* PT4 = reinterpret_cast<const float4*>(Pw) + 2 * rg;
  uint32_t g = 0;  // position in the CTA's K/V block sequence
  uint32_t k = 0;  // position in the CTA's tile sequence
  for (int t = t0; t < L.total; ++k) {
    const TmaProb* __restrict__ pp = T.p;
    int Lk = pp->Lk;
    float sl2 = pp->scale_log2;
    asm volatile("" : "+r"(Lk), "+f"(sl2));
    const int nb = (Lk + kNK - 1) / kNK;
    const int64_t ldo = pp->ldo;
    const int rows_q = min(kRows, pp->Lq - T.q0) - (kRowsW * w + rg);  // rows r with r - (32w + rg) < rows_q
    const bool active = kRowsW * w < pp->Lq - T.q0;  // (warp-uniform) the warp holds a row below Lq
    float* const orow = pp->o + pp->o_off + ((int64_t)T.q0 + kRowsW * w + rg) * ldo + (int64_t)T.h * kD + 4 * cg;
    int tn = L.total;
    Tile Tn = T;

    // per row: the negated exp2 offset and the running sum, in row pairs (i = 2p, 2p + 1) as the
    // scores are
    float2 o[kRI][4];
    float2 nm2[4], l2[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      nm2[p] = make_float2(INFINITY, INFINITY);
      l2[p] = make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < kRI; ++i)
#pragma unroll
      for (int u = 0; u < 4; ++u) o[i][u] = make_float2(0.f, 0.f);
    if (!mbar_wait_bounded(&C->qbar[w], k & 1u)) {
      if (lane == 0) {
        report_error(L.status, DEV_TIMEOUT, 61, (int32_t)k);
        tc::bulk_wait_group_all();
      }
      return;
    }
    if (active) transpose_q(Qw, lane);

    for (int j = 0; j < nb; ++j, ++g) {
      const int s = (int)(g % kNS);
      const uint32_t par = (g / kNS) & 1u;
      const int nk = min(kNK, Lk - j * kNK);
      if (!mbar_wait_bounded(&C->full[s], par)) {
        if (lane == 0) {
          report_error(L.status, DEV_TIMEOUT, 62, (int32_t)g);
          tc::bulk_wait_group_all();
        }
        return;
      }
      if (j == nb - 1) {
        tn = *reinterpret_cast<volatile const int32_t*>(&C->tiles[(k + 1) % kTileSlots]);
        if (tn < L.total) Tn = tile_of(L, tn);
      }
      const float4* K4 = reinterpret_cast<const float4*>(Ks + s * kNK * kKS) + cg * (kKS / 4);
      const float4* V4 = reinterpret_cast<const float4*>(Vs + s * kNK * kVS) + cg;

      // ---- S = Q K^T over the block's 16-key groups that hold a key below Lk
      float2 acc[4][8];
      if (active) {
        if (nk > 48) qk_block<8>(QT4, K4, acc);
        else if (nk > 32) qk_block<6>(QT4, K4, acc);
        else if (nk > 16) qk_block<4>(QT4, K4, acc);
        else qk_block<2>(QT4, K4, acc);
      }
      if (j == nb - 1 && tn < L.total) {  // this warp's Q^T is done: fetch its next Q rows
        __syncwarp();
        if (lane == 0) {
          fence_proxy_async_smem();
          issue_q(L, Tn, w, Qw, &C->qbar[w]);
        }
      }
      if (active) {
        if (nk < kNK) {  // ragged block (warp-uniform): keys past Lk get -inf (a select, not a product)
#pragma unroll
          for (int p = 0; p < 4; ++p)
#pragma unroll
            for (int jj = 0; jj < 8; ++jj)
              if (cg + 8 * jj >= nk) acc[p][jj] = make_float2(-INFINITY, -INFINITY);
        }
        // ---- softmax with a lazily moved exp2 offset (as attn_fp32_warp.cu): the row maxima are
        // reduced across the row's 8 lanes only when some score exceeds its row's offset by 8
        float lmax[kRI];
        bool need = false;
#pragma unroll
        for (int i = 0; i < kRI; ++i) {
          float m = score(acc, i, 0);
#pragma unroll
          for (int jj = 1; jj < 8; ++jj) m = fmaxf(m, score(acc, i, jj));
          lmax[i] = m;
          need |= fmaf(m, sl2, pick(nm2, i)) > 8.f;
        }
        if (__any_sync(0xffffffffu, need)) {
          bool moved = false;
          float2 nprev[4];
#pragma unroll
          for (int p = 0; p < 4; ++p) nprev[p] = nm2[p];
#pragma unroll
          for (int i = 0; i < kRI; ++i) {
            float mr = lmax[i];
            mr = fmaxf(mr, __shfl_xor_sync(0xffffffffu, mr, 1));
            mr = fmaxf(mr, __shfl_xor_sync(0xffffffffu, mr, 2));
            mr = fmaxf(mr, __shfl_xor_sync(0xffffffffu, mr, 4));
            const float mx = mr * sl2;  // the same value in all 8 lanes of the row
            if (mx + pick(nm2, i) > 8.f) {
              set(nm2, i, -mx);
              moved = true;
            }
          }
          if (j > 0 && __any_sync(0xffffffffu, moved)) {
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              const float2 alpha = make_float2(ex2(nm2[p].x - nprev[p].x), ex2(nm2[p].y - nprev[p].y));
              l2[p] = __fmul2_rn(l2[p], alpha);
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                o[2 * p][u] = __fmul2_rn(o[2 * p][u], make_float2(alpha.x, alpha.x));
                o[2 * p + 1][u] = __fmul2_rn(o[2 * p + 1][u], make_float2(alpha.y, alpha.y));
              }
            }
          }
        }
        if (j == 0) {  // the previous tile's output copy has read the P^T buffer
          if (lane == 0) tc::bulk_wait_group_read<0>();
          __syncwarp();
        }
        // P^T [key][position]: a lane's 8 rows of one key are two float4 stores (positions 8rg..)
        auto pv_group = [&](int k4, int valid) {  // O += P V over keys 4 k4 .. + 3
          float4 pa[4], pb[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            pa[e] = PT4[(k4 * 4 + e) * (kPT / 4)];
            pb[e] = PT4[(k4 * 4 + e) * (kPT / 4) + 1];
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v0;
            if (e < valid) {  // V rows past Lk are replaced by zeros (they may hold anything; 0 * inf is not 0)
              v0 = V4[(k4 * 4 + e) * (kVS / 4)];
              v1 = V4[(k4 * 4 + e) * (kVS / 4) + 8];
            }
#pragma unroll
            for (int i = 0; i < kRI; ++i) {
              const float4& pq = i < 4 ? pa[e] : pb[e];
              const int c = i & 3;
              const float pv = c == 0 ? pq.x : c == 1 ? pq.y : c == 2 ? pq.z : pq.w;
              const float2 p2 = make_float2(pv, pv);
              o[i][0] = __ffma2_rn(p2, make_float2(v0.x, v0.y), o[i][0]);
              o[i][1] = __ffma2_rn(p2, make_float2(v0.z, v0.w), o[i][1]);
              o[i][2] = __ffma2_rn(p2, make_float2(v1.x, v1.y), o[i][2]);
              o[i][3] = __ffma2_rn(p2, make_float2(v1.z, v1.w), o[i][3]);
            }
          }
        };
        // probabilities of key group jj (key cg + 8 jj), row pairs 2h and 2h + 1 (rows 4h .. 4h + 3):
        // one float4 of P^T, and the rows' sums
        auto p_half = [&](int jj, int h) {
          const float2 a0 = __ffma2_rn(acc[2 * h][jj], make_float2(sl2, sl2), nm2[2 * h]);
          const float2 a1 = __ffma2_rn(acc[2 * h + 1][jj], make_float2(sl2, sl2), nm2[2 * h + 1]);
          const float2 p0 = make_float2(ex2(a0.x), ex2(a0.y));
          const float2 p1 = make_float2(ex2(a1.x), ex2(a1.y));
          l2[2 * h] = __fadd2_rn(l2[2 * h], p0);
          l2[2 * h + 1] = __fadd2_rn(l2[2 * h + 1], p1);
          *reinterpret_cast<float4*>(Pw + (cg + 8 * jj) * kPT + 8 * rg + 4 * h) = make_float4(p0.x, p0.y, p1.x, p1.y);
        };
        if (nk > kBox) {
          // keys past 32: their probabilities are formed inside the P V of keys 0..31, so that
          // their exp2 (on the SFU) overlap the products (on the FMA pipe)
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            p_half(jj, 0);
            p_half(jj, 1);
          }
          __syncwarp();
#pragma unroll
          for (int k4 = 0; k4 < 8; ++k4) {
            pv_group(k4, 4);
            p_half(4 + (k4 >> 1), k4 & 1);
          }
          __syncwarp();
          if (nk == kNK) {
#pragma unroll 2
            for (int k4 = 8; k4 < kNK / 4; ++k4) pv_group(k4, 4);
          } else {
#pragma unroll 2
            for (int k4 = 8; 4 * k4 < nk; ++k4) pv_group(k4, min(4, nk - 4 * k4));
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            p_half(jj, 0);
            p_half(jj, 1);
          }
          __syncwarp();
#pragma unroll 2
          for (int k4 = 0; 4 * k4 < nk; ++k4) pv_group(k4, min(4, nk - 4 * k4));
        }
      }  // active
      __syncwarp();  // every lane is done with P and with stage s

      // ---- release stage s; the last warp out loads the block two ahead into it
      if (lane == 0) {
        __threadfence_block();
        if (atomicAdd(&C->cnt[s], 1) == kW - 1) {
          atomicExch(&C->cnt[s], 0);
          __threadfence_block();
          fence_proxy_async_smem();
          issue_next(L, C, Ks, Vs, s);
        }
      }
    }

    // ---- O / l, rows < Lq. A warp whose 32 rows all lie below Lq stages them in its P^T buffer
    // ([32][64]) and stores them with one TMA copy, which runs on while the next tile starts (the
    // next write to the buffer, in the next tile's first block, first waits for the copy to have
    // read it); other warps store their rows below Lq directly.
    if (active) {
      const bool tma_o = pp->mo >= 0 && pp->Lq - T.q0 >= kRowsW * (w + 1);  // (warp-uniform)
#pragma unroll
      for (int i = 0; i < kRI; ++i) {
        float ls = pick(l2, i);
        ls += __shfl_xor_sync(0xffffffffu, ls, 1);
        ls += __shfl_xor_sync(0xffffffffu, ls, 2);
        ls += __shfl_xor_sync(0xffffffffu, ls, 4);
        float inv;
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(inv) : "f"(ls));  // within 1 ulp; l >= 1 here
        const float4 lo = make_float4(o[i][0].x * inv, o[i][0].y * inv, o[i][1].x * inv, o[i][1].y * inv);
        const float4 hi = make_float4(o[i][2].x * inv, o[i][2].y * inv, o[i][3].x * inv, o[i][3].y * inv);
        if (tma_o) {
          float* st = Pw + (rg + 4 * i) * kD + 4 * cg;
          *reinterpret_cast<float4*>(st) = lo;
          *reinterpret_cast<float4*>(st + 32) = hi;
        } else if (4 * i < rows_q) {
          float* dst = orow + (int64_t)(4 * i) * ldo;
          *reinterpret_cast<float4*>(dst) = lo;
          *reinterpret_cast<float4*>(dst + 32) = hi;
        }
      }
      if (tma_o) {
        fence_proxy_async_smem();  // this lane's staged rows, before the copy reads them
        __syncwarp();
        if (lane == 0) {
          tc::tma_store_2d(L.maps + pp->mo, Pw, T.h * kD, pp->oy + T.q0 + kRowsW * w);
          tc::bulk_commit_group();
        }
      }
    }
    T = Tn;
    t = tn;
  }
  if (lane == 0) tc::bulk_wait_group_all();  // the output copies are complete
}

}  // namespace

int attn_fp32_wide_tile_rows() { return kRows; }

int attn_fp32_wide_ctas() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

cudaError_t launch_attn_fp32_wide(const TmaLaunch& L, cudaStream_t s) {
  if (L.total <= 0) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(attn_fp32_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BYTES);
  if (e != cudaSuccess) return e;
  const int ctas = attn_fp32_wide_ctas();
  const int grid = L.total < ctas ? L.total : ctas;  // persistent: one CTA per SM
  attn_fp32_wide_kernel<<<grid, kW * 32, BYTES, s>>>(L);
  return cudaGetLastError();
}

}  // namespace supra
