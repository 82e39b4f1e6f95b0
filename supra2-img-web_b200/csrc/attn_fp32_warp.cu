// Fused FP32 attention, persistent warp-pipelined kernel (sm_100a): D = 64, scale > 0, with or
// without a score bias (expanded [H, Lq, Lk], or the T5 [buckets, H] table, which the host
// turns into a bias by relative position with one small launch before this one).
// The DiT self/cross-attention kernel (app/models/dit.js:172,184) and, with the bias, the T5
// encoder's (app/models/t5.js:80).
//
// Same algorithm as attn_fp32.cu (online softmax over key blocks, app/gpu/kernels.js:164-316),
// organised so that the main loop has no block-wide barrier and no start-up gap between tiles:
//  * Persistent CTAs (two per SM): CTA c starts with tile c and then claims tiles one at a time
//    from the launch's counter (grid, grid + 1, ... in claim order). A tile is 128 query rows of
//    one head of one problem; the host orders problems longest-Lk first. (With a fixed stride
//    c, c + grid, ... the two CTAs of an SM progressed at different rates, about 4.8 against
//    7.0 ms over a DiT self-attention launch, and the slower one finished alone on the SM.)
//  * 4 warps x 32 query rows. Lane (rg = lane/8, cg = lane%8) of warp w owns rows 32w + rg + 4i
//    (i < 8), keys cg + 8j (j < 4) of each 32-key block and output columns 4*(cg + 8u) .. +3
//    (u < 2): 8x4 score and 8x8 output register blocks (fp32 throughout). The products use the
//    packed f32x2 FMA (two FMAs per issued instruction), which leaves issue slots for the
//    fragment loads and the softmax: with scalar FFMA the kernel was issue-bound.
//  * All operands arrive by TMA tensor copies (fp32 tensor maps, no rounding): one box per warp
//    for its Q rows, one box each for the K and V rows of a 32-key block. Q and K boxes are 68
//    columns wide, so their shared-memory rows are 68 floats apart and the fragment reads are
//    free of bank conflicts; the 4 extra columns (the next head, or zero fill past the buffer)
//    are never read.
//  * The K/V blocks of all of a CTA's tiles form one sequence flowing through a 3-stage ring
//    (one "full" mbarrier per stage, expect_tx). A warp that has finished a stage counts itself
//    out on the stage's counter; the last warp out issues the block three ahead, which may
//    belong to the CTA's next tile, through a cursor kept in shared memory. No warp waits for
//    a producer, warps drift freely, and the next tile's first blocks are already in flight
//    while the current tile finishes. The cursor claims the next tile when it issues a tile's
//    last block and publishes it in a small shared table before that block's barrier arrive,
//    so every warp finds it there once it has waited for the block.
//  * Each warp fetches its Q rows of the next tile as soon as it has finished the last QK^T of
//    the current tile (its own Q rows are read by no other warp).
//  * Lazy rescaling: the running row maximum used as the exp2 offset is only moved when a block
//    exceeds it by more than 8 (a factor 256), so the O/l rescale is skipped on almost every
//    block; the result is the same softmax (O and l always share one offset).
//  * exp2 via ex2.approx.ftz (relative error ~2^-22), scale*log2(e) folded into the scores.
//  * Boxes are always whole (32 rows). Rows past Lq or Lk hold other rows of the buffer or zero
//    fill: scores of keys past Lk are replaced (not multiplied) by -inf, V rows past Lk are not
//    read, and rows past Lq are never stored, so no value there can reach a stored output. In a
//    ragged last block the 4-key groups wholly past Lk are skipped in PV.
//  * With a bias, each lane copies (cp.async) the 32 bias values of its scores of the next key
//    block into its own places of the warp's P block as soon as that block's P V is done, so
//    the loads overlap the next block's wait and Q K^T (they used to sit in front of the
//    softmax, one L2 round trip per block with one or two warps per scheduler).
//  * Key splits, for launches with fewer tiles than CTAs (the DiT self-attention of one image
//    pair, 36 tiles): a tile then covers a range of key blocks of its (head, query tile) group,
//    writes its unnormalised O rows with their exp2 offset and sum to a partial array, and the last
//    split of each warp's 32 rows to arrive (a counter per group and warp) combines the group's
//    partials: O = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s, M = max_s m_s.
//  * All waits are bounded (2 s); a timeout sets the device status word and the CTA leaves.
#include "common.cuh"
#include "tcgen05.cuh"

namespace supra {
namespace {

constexpr int kW = 4;             // warps per CTA
constexpr int kRI = 8;            // query rows per lane
constexpr int kRowsW = 4 * kRI;   // query rows per warp
constexpr int kRows = kW * kRowsW;
constexpr int kNK = kFwBoxRows;   // keys per block
constexpr int kNS = 3;            // K/V stages
constexpr int kD = 64;            // head dim
constexpr int kQS = kFwBoxWide;   // Q row stride in shared memory (floats)
constexpr int kKS = kFwBoxWide;   // K row stride
constexpr int kVS = kFwBoxNarrow; // V row stride
constexpr int kPS = kNK + 8;      // P row stride: conflict-free scalar writes and float4 reads
static_assert(kRowsW == kFwBoxRows, "one Q box per warp");
static_assert(kVS == kD && kQS >= kD, "box widths");

constexpr uint32_t kQBytes = kRowsW * kQS * 4;
constexpr uint32_t kKBytes = kNK * kKS * 4;
constexpr uint32_t kVBytes = kNK * kVS * 4;

constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + kRows * kQS;
constexpr int OFF_V = OFF_K + kNS * kNK * kKS;
constexpr int OFF_P = OFF_V + kNS * kNK * kVS;
constexpr int FLOATS = OFF_P + kW * kRowsW * kPS;
static_assert((OFF_K * 4) % 128 == 0 && (OFF_V * 4) % 128 == 0 && kQBytes % 128 == 0 && kKBytes % 128 == 0 &&
                  kVBytes % 128 == 0,
              "TMA destinations are 128-byte aligned");

// Next K/V block of this CTA's block sequence: tile t, block b (the tile's blocks end before
// block nblk), and the tile's TMA coordinates (head column already added).
struct Cursor {
  int32_t t, b, nblk, mk, mv, kx, ky, vx, vy;
  int32_t k;  // the tile's position in the CTA's tile sequence
};
constexpr int kMaxSplits = 8;  // key splits per (head, query tile) group at most (the host caps them)
constexpr int kTileSlots = 8;  // claimed tiles in flight: the cursor runs at most 3 blocks ahead
struct Ctl {
  uint64_t qbar[kW];
  uint64_t full[kNS];
  int32_t cnt[kNS];
  int32_t pad;
  Cursor cur;
  int32_t tiles[kTileSlots];  // tile k of this CTA at tiles[k % kTileSlots]
};
constexpr int BYTES = FLOATS * 4 + (int)sizeof(Ctl) + 128;  // + slack for the 128-byte alignment

// A tile: query rows q0 .. q0 + 127 of head h, key blocks b0 .. b1 - 1 (all of them unless the
// problem's groups are split).
struct Tile {
  const TmaProb* p;
  int h, q0, b0, b1;
};

struct TileIdx {
  int pidx, local;
};
__device__ __forceinline__ TileIdx tile_idx(const TmaLaunch& L, int t) {
  const int pidx = L.uniform > 0 ? t / L.uniform : find_problem(L.begin, L.n, t);
  return TileIdx{pidx, t - (L.uniform > 0 ? pidx * L.uniform : __ldg(L.begin + pidx))};
}

// Within a problem, tile local = (h * q_tiles + query tile) * splits + split. SPLIT: the launch
// may split groups (a separate kernel form, so that the unsplit form keeps its registers).
template <bool SPLIT>
__device__ __forceinline__ Tile tile_of(const TmaLaunch& L, int t) {
  Tile r;
  const TileIdx ix = tile_idx(L, t);
  r.p = L.probs + ix.pidx;
  const int qt = r.p->q_tiles;
  const int nb = (r.p->Lk + kNK - 1) / kNK;
  if (SPLIT) {
    const int ns = r.p->splits;
    const int grp = ix.local / ns;
    r.h = grp / qt;
    r.q0 = (grp - r.h * qt) * kRows;
    r.b0 = (ix.local - grp * ns) * r.p->bps;
    r.b1 = min(nb, r.b0 + r.p->bps);
  } else {
    r.h = ix.local / qt;
    r.q0 = (ix.local - r.h * qt) * kRows;
    r.b0 = 0;
    r.b1 = nb;
  }
  return r;
}

template <bool SPLIT>
__device__ __forceinline__ void cursor_at(const TmaLaunch& L, Cursor& c, int t) {
  const Tile T = tile_of<SPLIT>(L, t);
  c.t = t;
  c.b = T.b0;
  c.nblk = T.b1;
  c.mk = T.p->mk;
  c.mv = T.p->mv;
  c.kx = T.p->kx + T.h * kD;
  c.ky = T.p->ky;
  c.vx = T.p->vx + T.h * kD;
  c.vy = T.p->vy;
}

// Issues the cursor's block into stage s and advances the cursor (one thread). With a tile's
// last block it first claims the CTA's next tile and publishes it in C->tiles; the barrier
// arrive below releases that store to every warp that later waits for this block. Past the
// CTA's last tile it issues nothing: no warp will wait for that stage again.
template <bool SPLIT>
__device__ __forceinline__ void issue_next(const TmaLaunch& L, Ctl* C, float* Ks, float* Vs, int s) {
  Cursor& c = C->cur;
  if (c.t >= L.total) return;
  int tn = 0;
  if (c.b + 1 == c.nblk) {
    tn = (int)gridDim.x + atomicAdd(L.next_tile, 1);
    C->tiles[(c.k + 1) % kTileSlots] = tn;
  }
  uint64_t* bar = &C->full[s];
  mbar_arrive_expect_tx(bar, kKBytes + kVBytes);
  tc::tma_load_2d(Ks + s * kNK * kKS, L.maps + c.mk, c.kx, c.ky + c.b * kNK, bar);
  tc::tma_load_2d(Vs + s * kNK * kVS, L.maps + c.mv, c.vx, c.vy + c.b * kNK, bar);
  if (++c.b == c.nblk) {
    ++c.k;
    if (tn < L.total) cursor_at<SPLIT>(L, c, tn);
    else c.t = tn;
  }
}

// A warp's 32 Q rows of a tile: tensor map and TMA coordinates.
struct QBox {
  int32_t m, x, y;
};
__device__ __forceinline__ QBox qbox_of(const Tile& T, int w) {
  return QBox{T.p->mq, T.p->qx + T.h * kD, T.p->qy + T.q0 + w * kRowsW};
}
__device__ __forceinline__ void issue_q(const TmaLaunch& L, const QBox& q, float* dst, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, kQBytes);
  tc::tma_load_2d(dst, L.maps + q.m, q.x, q.y, bar);
}

// S = Q K^T for keys cg + 8jj (jj < 4) of one block. Packed FFMA (f32x2, two FMAs per issued
// instruction): each score accumulates the head dim's even and odd components in the two halves
// of one float2 ((x, y) and (z, w) of a float4 fragment are register pairs already), summed at the
// end.
__device__ __forceinline__ void qk_block(const float4* __restrict__ Q4, const float4* __restrict__ K4,
                                         float (&sc)[kRI][4]) {
  float2 acc[kRI][4];
#pragma unroll
  for (int i = 0; i < kRI; ++i)
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) acc[i][jj] = make_float2(0.f, 0.f);
#pragma unroll 2
  for (int d4 = 0; d4 < kD / 4; ++d4) {
    float4 kf[4], qf[kRI];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) kf[jj] = K4[jj * 8 * (kKS / 4) + d4];
#pragma unroll
    for (int i = 0; i < kRI; ++i) qf[i] = Q4[i * 4 * (kQS / 4) + d4];
#pragma unroll
    for (int i = 0; i < kRI; ++i)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj)
        acc[i][jj] = __ffma2_rn(make_float2(qf[i].x, qf[i].y), make_float2(kf[jj].x, kf[jj].y), acc[i][jj]);
#pragma unroll
    for (int i = 0; i < kRI; ++i)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj)
        acc[i][jj] = __ffma2_rn(make_float2(qf[i].z, qf[i].w), make_float2(kf[jj].z, kf[jj].w), acc[i][jj]);
  }
#pragma unroll
  for (int i = 0; i < kRI; ++i)
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) sc[i][jj] = acc[i][jj].x + acc[i][jj].y;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Key-split epilogue of warp w for tile t (TmaProb::splits > 1). Lane (rg, cg) holds rows
// 32w + rg + 4i, output columns 4cg .. 4cg + 3 and 32 + 4cg .. + 3 (o, unnormalised), the rows'
// exp2 offsets mo (equal in the row's 8 lanes) and its share of the row sums l. The warp writes
// its rows to the partial arrays; the last split of (group, w) to arrive reads every split's
// rows back from L2 and stores O / l for rows < Lq.
__device__ __forceinline__ void split_epilogue(const TmaLaunch& L, int t, int w, int lane, int rg, int cg, int rows_q,
                                            float* orow, int64_t ldo, const float2 (&o)[kRI][4],
                                            const float (&mo)[kRI], const float (&l)[kRI]) {
  const TileIdx ix = tile_idx(L, t);
  const TmaProb* p = L.probs + ix.pidx;
  const int ns = p->splits;
  const int grp_local = ix.local / ns;
  const int split = ix.local - grp_local * ns;
  const int64_t group = (int64_t)p->group0 + grp_local;
  const int64_t base = (group * L.part_splits) * kRows;  // row index of split 0's first row
  const int r0 = kRowsW * w + rg;
#pragma unroll
  for (int i = 0; i < kRI; ++i) {
    float ls = l[i];
    ls += __shfl_xor_sync(0xffffffffu, ls, 1);
    ls += __shfl_xor_sync(0xffffffffu, ls, 2);
    ls += __shfl_xor_sync(0xffffffffu, ls, 4);
    const int64_t row = base + (int64_t)split * kRows + r0 + 4 * i;
    float* dst = L.part_o + row * kD + 4 * cg;
    *reinterpret_cast<float4*>(dst) = make_float4(o[i][0].x, o[i][0].y, o[i][1].x, o[i][1].y);
    *reinterpret_cast<float4*>(dst + 32) = make_float4(o[i][2].x, o[i][2].y, o[i][3].x, o[i][3].y);
    if (cg == 0) L.part_ml[row] = make_float2(mo[i], ls);
  }
  __syncwarp();
  int last = 0;
  if (lane == 0) {
    __threadfence();  // this warp's partial rows before its count
    last = atomicAdd(L.part_cnt + group * kW + w, 1) == ns - 1;
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return;
  __threadfence();  // every split's partial rows after the count that saw them all
  // The row's 8 lanes share its offsets and sums: lane cg reads split cg's (offset, sum) of each
  // of its 8 rows (all loads before any use), the row maximum M and the denominator come from
  // shuffles across the 8 lanes, and each lane keeps the weight 2^(m_cg - M) of its split.
  float wgt[kRI], inv[kRI];
#pragma unroll
  for (int i = 0; i < kRI; ++i) {
    const float2 ml =
        cg < ns ? __ldcg(&L.part_ml[base + (int64_t)cg * kRows + r0 + 4 * i]) : make_float2(-INFINITY, 0.f);
    wgt[i] = ml.x;
    inv[i] = ml.y;
  }
#pragma unroll
  for (int i = 0; i < kRI; ++i) {
    float M = wgt[i];
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 1));
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 2));
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 4));
    const float f = cg < ns ? ex2(wgt[i] - M) : 0.f;
    float den = f * inv[i];
    den += __shfl_xor_sync(0xffffffffu, den, 1);
    den += __shfl_xor_sync(0xffffffffu, den, 2);
    den += __shfl_xor_sync(0xffffffffu, den, 4);
    wgt[i] = f;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(inv[i]) : "f"(den));  // den >= 1: the split holding M adds >= 1
  }
  // per row: the row's O fragments of up to four splits loaded together, then summed with the
  // weights (about one wait for L2 per row; splits-outer loops hold twice the registers and spill)
#pragma unroll 1
  for (int i = 0; i < kRI; ++i) {
    float f[kMaxSplits];
#pragma unroll
    for (int s = 0; s < kMaxSplits; ++s) f[s] = __shfl_sync(0xffffffffu, wgt[i], (lane & ~7) | s);
    if (4 * i < rows_q) {
      const int64_t row0 = base + r0 + 4 * i;
      float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
#pragma unroll
      for (int s0 = 0; s0 < kMaxSplits; s0 += 4) {
        if (s0 < ns) {
          float4 x0[4], x1[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (s0 + u < ns) {
              const float* src = L.part_o + (row0 + (int64_t)(s0 + u) * kRows) * kD + 4 * cg;
              x0[u] = __ldcg(reinterpret_cast<const float4*>(src));
              x1[u] = __ldcg(reinterpret_cast<const float4*>(src + 32));
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (s0 + u < ns) {
              const float w = f[s0 + u];
              a0 = make_float4(fmaf(w, x0[u].x, a0.x), fmaf(w, x0[u].y, a0.y), fmaf(w, x0[u].z, a0.z),
                               fmaf(w, x0[u].w, a0.w));
              a1 = make_float4(fmaf(w, x1[u].x, a1.x), fmaf(w, x1[u].y, a1.y), fmaf(w, x1[u].z, a1.z),
                               fmaf(w, x1[u].w, a1.w));
            }
          }
        }
      }
      float* dst = orow + (int64_t)(4 * i) * ldo;
      const float v = inv[i];
      *reinterpret_cast<float4*>(dst) = make_float4(a0.x * v, a0.y * v, a0.z * v, a0.w * v);
      *reinterpret_cast<float4*>(dst + 32) = make_float4(a1.x * v, a1.y * v, a1.z * v, a1.w * v);
    }
  }
}

template <bool BIAS, bool SPLIT>
__global__ void __launch_bounds__(kW * 32, 2) attn_fp32_warp_kernel(const __grid_constant__ TmaLaunch L) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  float* smem = reinterpret_cast<float*>(smem_raw + (((raw + 127u) & ~127u) - raw));
  float* Qs = smem + OFF_Q;
  float* Ks = smem + OFF_K;
  float* Vs = smem + OFF_V;
  Ctl* C = reinterpret_cast<Ctl*>(smem + FLOATS);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int w = tid >> 5;
  const int rg = lane >> 3;
  const int cg = lane & 7;
  float* Pw = smem + OFF_P + w * kRowsW * kPS;
  float* Qw = Qs + w * kRowsW * kQS;

  const int t0 = blockIdx.x;
  if (t0 >= L.total) {  // the host sizes the grid to at most one CTA per tile
    if (tid == 0) report_error(L.status, DEV_BAD_TILE, 20);
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
    cursor_at<SPLIT>(L, C->cur, t0);
    for (int s = 0; s < kNS; ++s) issue_next<SPLIT>(L, C, Ks, Vs, s);
  }
  Tile T = tile_of<SPLIT>(L, t0);
  if (lane == 0) issue_q(L, qbox_of(T, w), Qw, &C->qbar[w]);

  // Expanded bias ([H, Lq, Lk]): the lane's 32 bias values of a key block are copied (cp.async,
  // zero fill for rows past Lq and keys past Lk) into the places of the warp's P block that the
  // lane itself writes, so the loads run behind the block's wait and Q K^T instead of in front
  // of its softmax. Issued once the previous block's P V is done (the tile's first block: at the
  // end of the previous tile, or here), waited for by the same lane before the scores take them.
  auto warp_active = [&](const Tile& X) { return !BIAS || kRowsW * w < X.p->Lq - X.q0; };
  // The T5 form reads the bias by relative position, [H, 2 rel_max + 1] (formed from the table
  // before the launch), at clamp(c - r, -rel_max, rel_max).
  auto issue_bias = [&](const Tile& X, int jx) {
    const TmaProb* __restrict__ xp = X.p;
    const int Lqx = xp->Lq, Lkx = xp->Lk;
    const int r0 = X.q0 + kRowsW * w + rg, c0 = jx * kNK + cg;
    if (xp->rel_lut == nullptr) {
      const float* bh = xp->bias + (int64_t)X.h * Lqx * Lkx;
#pragma unroll
      for (int i = 0; i < kRI; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int r = r0 + 4 * i, c = c0 + 8 * jj;
          const bool ok = r < Lqx && c < Lkx;
          cp_async4(Pw + (rg + 4 * i) * kPS + cg + 8 * jj, ok ? bh + (int64_t)r * Lkx + c : bh, ok ? 4u : 0u);
        }
    } else {
      const int rm = xp->rel_max;
      const float* bh = xp->bias + (int64_t)X.h * (2 * rm + 1) + rm;
#pragma unroll
      for (int i = 0; i < kRI; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int r = r0 + 4 * i, c = c0 + 8 * jj;
          const bool ok = r < Lqx && c < Lkx;
          cp_async4(Pw + (rg + 4 * i) * kPS + cg + 8 * jj, bh + (ok ? max(-rm, min(rm, c - r)) : 0), ok ? 4u : 0u);
        }
    }
    cp_async_commit();
  };
  if (BIAS && warp_active(T)) issue_bias(T, T.b0);

  const float4* Q4 = reinterpret_cast<const float4*>(Qw) + rg * (kQS / 4);
  const float4* P4 = reinterpret_cast<const float4*>(Pw) + rg * (kPS / 4);
  uint32_t g = 0;  // position in the CTA's K/V block sequence
  uint32_t k = 0;  // position in the CTA's tile sequence
  for (int t = t0; t < L.total; ++k) {
    const TmaProb* __restrict__ pp = T.p;
    int Lk = pp->Lk;
    float sl2 = pp->scale_log2;
    asm volatile("" : "+r"(Lk), "+f"(sl2));  // kept in registers, not re-loaded from the descriptor
    const int b0 = T.b0, b1 = T.b1;
    // this lane's first output row, read now rather than behind the last block
    const int64_t ldo = pp->ldo;
    const int rows_q = min(kRows, pp->Lq - T.q0) - (kRowsW * w + rg);  // rows r with r - (32w + rg) < rows_q
    // With a bias (the T5 encoder: Lq = Lk, often below 128) a warp whose rows all lie past Lq
    // skips the arithmetic; it still waits for its Q rows and releases every K/V stage.
    const bool active = warp_active(T);
    float* const orow = pp->o + pp->o_off + ((int64_t)T.q0 + kRowsW * w + rg) * ldo + (int64_t)T.h * kD + 4 * cg;
    // the next tile: known once the wait for this tile's last block has returned (it was claimed
    // and published before that block was issued); its Q rows are requested right after this
    // tile's last QK^T
    int tn = L.total;
    Tile Tn = T;

    // output columns 4cg + (0,1), (2,3), 32 + 4cg + (0,1), (2,3): packed pairs
    float2 o[kRI][4];
    float mo[kRI], l[kRI];
#pragma unroll
    for (int i = 0; i < kRI; ++i) {
      mo[i] = -INFINITY;
      l[i] = 0.f;
#pragma unroll
      for (int u = 0; u < 4; ++u) o[i][u] = make_float2(0.f, 0.f);
    }
    if (!mbar_wait_bounded(&C->qbar[w], k & 1u)) {
      if (lane == 0) report_error(L.status, DEV_TIMEOUT, 21, (int32_t)k);
      return;
    }

    for (int j = b0; j < b1; ++j, ++g) {
      const int s = (int)(g % kNS);
      const uint32_t par = (g / kNS) & 1u;
      const int nk = min(kNK, Lk - j * kNK);
      if (!mbar_wait_bounded(&C->full[s], par)) {
        if (lane == 0) report_error(L.status, DEV_TIMEOUT, 22, (int32_t)g);
        return;
      }
      if (j == b1 - 1) {
        tn = *reinterpret_cast<volatile const int32_t*>(&C->tiles[(k + 1) % kTileSlots]);
        if (tn < L.total) Tn = tile_of<SPLIT>(L, tn);
      }
      const float4* K4 = reinterpret_cast<const float4*>(Ks + s * kNK * kKS) + cg * (kKS / 4);
      const float4* V4 = reinterpret_cast<const float4*>(Vs + s * kNK * kVS) + cg;

      // ---- S = Q K^T
      float sc[kRI][4];
      if (active) {
        // (ragged blocks too: scores of keys past Lk are replaced below; forms that skipped the
        // 8-key groups past Lk measured 0.2 % slower over the DiT step, their code being larger)
        qk_block(Q4, K4, sc);
      }
      if (j == b1 - 1 && tn < L.total) {  // this warp's Q rows are done: fetch its next ones
        __syncwarp();
        if (lane == 0) {
          fence_proxy_async_smem();
          issue_q(L, qbox_of(Tn, w), Qw, &C->qbar[w]);
        }
      }
      if (active) {
        if (nk < kNK) {  // ragged block (warp-uniform): keys past Lk get -inf (a select, not a product)
  #pragma unroll
          for (int i = 0; i < kRI; ++i)
  #pragma unroll
            for (int jj = 0; jj < 4; ++jj) sc[i][jj] = (cg + 8 * jj < nk) ? sc[i][jj] : -INFINITY;
        }
        if constexpr (BIAS) {
          // scores into the exp2 domain with the bias added, s scale log2 e + b log2 e (the
          // reference adds the bias to the scaled scores, app/gpu/kernels.js:53-62); rows past Lq
          // and keys past Lk take none (zero-filled copies)
          cp_async_wait<0>();  // this lane's bias values of the block, copied into its P places
  #pragma unroll
          for (int i = 0; i < kRI; ++i)
  #pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              const float b = Pw[(rg + 4 * i) * kPS + cg + 8 * jj];
              sc[i][jj] = fmaf(b, 1.4426950408889634f, sc[i][jj] * sl2);
            }
        }
        // exponent factor: the raw scores times scale log2 e, or the biased scores as they are
        const float f = BIAS ? 1.f : sl2;

        // ---- softmax with a lazily moved offset (exp2 domain). scale > 0 (host-checked), so the
        // maximum of the raw scores times scale*log2(e) is the maximum of the scaled scores.
        // Cheap test first: does any lane hold a score more than 8 above its row's offset? Only
        // then (every tile's first block, rarely afterwards) are the row maxima reduced across
        // the row's 8 lanes and the offsets moved.
        float lmax[kRI];
        bool need = false;
  #pragma unroll
        for (int i = 0; i < kRI; ++i) {
          lmax[i] = fmaxf(fmaxf(sc[i][0], sc[i][1]), fmaxf(sc[i][2], sc[i][3]));
          need |= fmaf(lmax[i], f, -mo[i]) > 8.f;
        }
        if (__any_sync(0xffffffffu, need)) {
          bool moved = false;
          float mprev[kRI];
  #pragma unroll
          for (int i = 0; i < kRI; ++i) {
            float mr = lmax[i];
            mr = fmaxf(mr, __shfl_xor_sync(0xffffffffu, mr, 1));
            mr = fmaxf(mr, __shfl_xor_sync(0xffffffffu, mr, 2));
            mr = fmaxf(mr, __shfl_xor_sync(0xffffffffu, mr, 4));
            const float mx = mr * f;  // the same value in all 8 lanes of the row
            mprev[i] = mo[i];
            if (mx > mo[i] + 8.f) {
              mo[i] = mx;
              moved = true;
            }
          }
          if (j > b0 && __any_sync(0xffffffffu, moved)) {  // (first block: O and l are still zero)
  #pragma unroll
            for (int i = 0; i < kRI; ++i) {
              const float alpha = ex2(mprev[i] - mo[i]);
              l[i] *= alpha;
  #pragma unroll
              for (int u = 0; u < 4; ++u) o[i][u] = __fmul2_rn(o[i][u], make_float2(alpha, alpha));
            }
          }
        }
  #pragma unroll
        for (int i = 0; i < kRI; ++i) {
  #pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const float pe = ex2(fmaf(sc[i][jj], f, -mo[i]));
            l[i] += pe;
            Pw[(rg + 4 * i) * kPS + cg + 8 * jj] = pe;
          }
        }
        __syncwarp();

        // ---- O += P V: whole groups of 4 valid keys, then the ragged group, whose V rows past
        // Lk are replaced by zeros (they may hold anything, and 0 * inf is not 0).
        auto pv_group = [&](int k4, int valid) {
          float4 pf[kRI];
  #pragma unroll
          for (int i = 0; i < kRI; ++i) pf[i] = P4[i * 4 * (kPS / 4) + k4];
  #pragma unroll
          for (int e = 0; e < 4; ++e) {
            float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v0;
            if (e < valid) {
              v0 = V4[(k4 * 4 + e) * (kVS / 4)];
              v1 = V4[(k4 * 4 + e) * (kVS / 4) + 8];
            }
  #pragma unroll
            for (int i = 0; i < kRI; ++i) {
              const float pe = e == 0 ? pf[i].x : e == 1 ? pf[i].y : e == 2 ? pf[i].z : pf[i].w;
              const float2 pp = make_float2(pe, pe);
              o[i][0] = __ffma2_rn(pp, make_float2(v0.x, v0.y), o[i][0]);
              o[i][1] = __ffma2_rn(pp, make_float2(v0.z, v0.w), o[i][1]);
              o[i][2] = __ffma2_rn(pp, make_float2(v1.x, v1.y), o[i][2]);
              o[i][3] = __ffma2_rn(pp, make_float2(v1.z, v1.w), o[i][3]);
            }
          }
        };
        const int nfull = nk >> 2;
  #pragma unroll 2
        for (int k4 = 0; k4 < nfull; ++k4) pv_group(k4, 4);
        if (nk & 3) pv_group(nfull, nk & 3);
      }  // active
      __syncwarp();  // every lane is done with P and with stage s
      if constexpr (BIAS) {  // the next block's bias values into P
        if (j + 1 < b1) {
          if (active) issue_bias(T, j + 1);
        } else if (tn < L.total && warp_active(Tn)) {
          issue_bias(Tn, Tn.b0);
        }
      }

      // ---- release stage s; the last warp out loads the block three ahead into it -----------
      if (lane == 0) {
        __threadfence_block();
        if (atomicAdd(&C->cnt[s], 1) == kW - 1) {
          atomicExch(&C->cnt[s], 0);
          __threadfence_block();
          fence_proxy_async_smem();
          issue_next<SPLIT>(L, C, Ks, Vs, s);
        }
      }
    }

    if (SPLIT && pp->splits > 1) {
      // ---- key split: this split's unnormalised rows, then the last split of this warp's rows
      // combines the group (every split of a group has the same active warps)
      if (active) split_epilogue(L, t, w, lane, rg, cg, rows_q, orow, ldo, o, mo, l);
    } else {
      // ---- O / l, rows < Lq ----------------------------------------------------------------
#pragma unroll
      for (int i = 0; i < kRI; ++i) {
        float ls = l[i];
        ls += __shfl_xor_sync(0xffffffffu, ls, 1);
        ls += __shfl_xor_sync(0xffffffffu, ls, 2);
        ls += __shfl_xor_sync(0xffffffffu, ls, 4);
        float inv;
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(inv) : "f"(ls));  // within 1 ulp; l >= 1 here
        if (4 * i < rows_q) {
          float* dst = orow + (int64_t)(4 * i) * ldo;
#pragma unroll
          for (int u = 0; u < 2; ++u)
            *reinterpret_cast<float4*>(dst + 32 * u) = make_float4(o[i][2 * u].x * inv, o[i][2 * u].y * inv,
                                                                   o[i][2 * u + 1].x * inv, o[i][2 * u + 1].y * inv);
        }
      }
    }
    T = Tn;
    t = tn;
  }
}

}  // namespace

int attn_fp32_warp_tile_rows() { return kRows; }

// SMs of the current device (the persistent grid is two CTAs per SM).
static int fp32_warp_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

cudaError_t launch_attn_fp32_warp(const TmaLaunch& L, bool bias, cudaStream_t s) {
  if (L.total <= 0) return cudaSuccess;
  const bool split = L.part_splits > 1;
  auto kern = bias ? (split ? attn_fp32_warp_kernel<true, true> : attn_fp32_warp_kernel<true, false>)
                   : (split ? attn_fp32_warp_kernel<false, true> : attn_fp32_warp_kernel<false, false>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, BYTES);
  if (e != cudaSuccess) return e;
  const int grid = L.total < 2 * fp32_warp_sms() ? L.total : 2 * fp32_warp_sms();  // persistent: two CTAs per SM
  kern<<<grid, kW * 32, BYTES, s>>>(L);
  return cudaGetLastError();
}

int attn_fp32_warp_cta_slots() { return 2 * fp32_warp_sms(); }

}  // namespace supra
