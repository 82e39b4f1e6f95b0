// ops.linear (app/gpu/ops.js:35-43, app/gpu/gemm.js:116-223) on the tensor cores, sm_100a: the
// TF32 and split-precision (TF32X3) variants of supra_attn_enqueue_linear.
//
//   split_kernel         every operand of a flush that is not read in place (x normalised
//                        first when asked: GroupNorm / LayerNorm with the statistics of the
//                        stats kernels, app/gpu/kernels.js:87-162; w times a folded gate; a w
//                        stored [K, N] transposed) into dense hi / lo arrays: hi = value with
//                        its 13 low mantissa bits cleared (a TF32 value), lo = value - hi
//                        (exact). One launch, HBM-bound.
//   linear_tc_kernel     C[128 x 128 tile] = X W^T with tcgen05.mma kind::tf32: per 32-deep
//                        k-block the TMA brings hi(X), hi(W) (and lo(X), lo(W)) tiles
//                        (SWIZZLE_128B, K-major), the MMA warp issues per 8-deep step one
//                        product (TF32) or three, lo*hi + hi*lo + hi*hi (TF32X3, the small terms
//                        first), into a TMEM accumulator. Every kFlush k-blocks the partial sum
//                        goes to a fresh accumulator (four in turn) and the epilogue warps add
//                        it to the row they hold in registers, in fp32 rounded to nearest, so the
//                        error does not grow with K as it would in one TMEM accumulator. The
//                        epilogue then applies bias, activation, gate and residual (the
//                        reference's order, app/gpu/gemm.js:130-135) and each thread stores its
//                        row (float4 stores when the rows are 16-byte aligned).
// Persistent: CTA c takes tiles c, c + grid, ... of the launch's (problem, row tile, column tile)
// list, in groups of 16 row tiles with the row tile innermost. 6 warps: TMA producer, MMA issuer, 4 epilogue warps (warp w owns
// TMEM lanes 32*(w%4) .. +31, i.e. output rows). One CTA per SM (three 64 KB stages). Every wait
// is bounded; on a timeout the CTA records the failure, drains its MMAs, frees TMEM and leaves.
#include <type_traits>

#include "tcgen05.cuh"

namespace supra {
namespace {

constexpr int kBM = 128, kBN = 128, kBK = 32;
constexpr int kStages = 3;
constexpr int kFlush = 4;                        // k-blocks per TMEM partial sum
constexpr uint32_t kTile = kBM * kBK * 4;        // one operand tile: 128 rows x 128 bytes = 16 KB
constexpr uint32_t kStage = 4 * kTile;           // hi(X), hi(W), lo(X), lo(W)
constexpr uint32_t kSlot = 32 * 32 * 4;          // epilogue: one 32 x 32 block, 128-byte rows, swizzled
constexpr uint32_t OFF_EPI = kStages * kStage;   // two slots per epilogue warp (TMA stores)
constexpr uint32_t OFF_BAR = OFF_EPI + 4 * 2 * kSlot;
constexpr uint32_t SMEM_BYTES = OFF_BAR + 256 + 1024;
constexpr int kAcc = 4;                          // TMEM accumulators (partial sums in flight)
constexpr uint32_t kTmemCols = kAcc * 128;       // 512: four 128-column accumulators
constexpr int kThreads = 192;

struct Bars {
  uint64_t full[kStages], empty[kStages], accf[kAcc], acce[kAcc], drain;
  int32_t abort;
  uint32_t tmem;
};
static_assert(sizeof(Bars) <= 256, "barrier block");
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");

enum WaitId : int32_t { W_EMPTY = 51, W_FULL = 52, W_ACCE = 53, W_ACCF = 54 };

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int32_t* abort,
                                              int32_t* status, int32_t id, int32_t detail) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0u) {
      if (*abort) return false;
      if (global_ns() - t0 > kWaitLimitNs) {
        report_error(status, DEV_TIMEOUT, id, detail);
        *abort = 1;
        return false;
      }
    }
  }
}

struct TileRef {
  const LinTcProb* p;
  int mt, nt;
};
// Tiles walk a problem in groups of kGroup row tiles: within a group the row tile is innermost,
// so the CTAs running at one time share a few weight column tiles (each read from memory once per
// group) and the group's rows of x stay in L2. (Column tiles innermost over all rows made every
// row tile read all of w again: for a [131K, 576] x [16128, 576]^T product that is 74 GB.)
constexpr int kGroup = 16;
__device__ __forceinline__ TileRef tile_ref(const LinTcLaunch& L, int t) {
  TileRef r;
  const int pi = find_problem(L.begin, L.n, t);
  r.p = L.probs + pi;
  const int local = t - __ldg(L.begin + pi);
  const int nt_all = r.p->n_tiles, mt_all = r.p->m_tiles;
  const int g = local / (kGroup * nt_all);       // row-tile group
  const int rem = local - g * (kGroup * nt_all);
  const int gs = min(kGroup, mt_all - g * kGroup);  // row tiles in this group
  r.nt = rem / gs;
  r.mt = g * kGroup + (rem - r.nt * gs);
  return r;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* m, int x, int y, uint64_t* bar) {
  tc::tma_load_2d(dst, m, x, y, bar);
}

template <bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1) linear_tc_kernel(const __grid_constant__ LinTcLaunch L) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);  // 1024-B aligned for the swizzle atoms
  Bars* B = reinterpret_cast<Bars*>(base + OFF_BAR);
  volatile int32_t* abort = &B->abort;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&B->full[s], 1);
      mbar_init(&B->empty[s], 1);
    }
    for (int b = 0; b < kAcc; ++b) {
      mbar_init(&B->accf[b], 1);
      mbar_init(&B->acce[b], 128);
    }
    mbar_init(&B->drain, 1);
    B->abort = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(&B->tmem, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = B->tmem;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < L.total; t += gridDim.x) {
        // the tile's fields in registers: each TMA issue below is an asm statement that clobbers
        // memory, after which fields read through P would be loaded from global memory again
        const TileRef T = tile_ref(L, t);
        const LinTcProb* P = T.p;
        const int nkb = P->nkb;
        const CUtensorMap* mxh = L.maps + P->mxh;
        const CUtensorMap* mwh = L.maps + P->mwh;
        const CUtensorMap* mxl = L.maps + P->mxl;
        const CUtensorMap* mwl = L.maps + P->mwl;
        const int ym = T.mt * kBM, yn = T.nt * kBN;
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % kStages;
          if (g >= kStages &&
              !(ok = wait_or_abort(&B->empty[s], (uint32_t)(((g / kStages) - 1) & 1), abort, L.status, W_EMPTY, g)))
            break;
          uint8_t* st = base + s * kStage;
          mbar_arrive_expect_tx(&B->full[s], SPLIT ? 4 * kTile : 2 * kTile);
          tma_load_2d(st, mxh, kb * kBK, ym, &B->full[s]);
          tma_load_2d(st + kTile, mwh, kb * kBK, yn, &B->full[s]);
          if (SPLIT) {
            tma_load_2d(st + 2 * kTile, mxl, kb * kBK, ym, &B->full[s]);
            tma_load_2d(st + 3 * kTile, mwl, kb * kBK, yn, &B->full[s]);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = tc::idesc_tf32(kBM, kBN, false, false);
    int g = 0, f = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < L.total; t += gridDim.x) {
      const TileRef T = tile_ref(L, t);
      const int nkb = T.p->nkb;
      for (int kb = 0; ok && kb < nkb; ++kb, ++g) {
        const int s = g % kStages;
        const bool start = (kb % kFlush) == 0;
        const bool end = (kb % kFlush) == kFlush - 1 || kb == nkb - 1;
        if (start && f >= kAcc)  // the epilogue has read this accumulator's previous partial sum
          ok = __all_sync(0xffffffffu, wait_or_abort(&B->acce[f % kAcc], (uint32_t)(((f / kAcc) - 1) & 1), abort,
                                                     L.status, W_ACCE, f));
        if (!ok) break;
        ok = __all_sync(0xffffffffu, wait_or_abort(&B->full[s], (uint32_t)((g / kStages) & 1), abort, L.status, W_FULL, g));
        if (!ok) break;
        tc::fence_after_sync();
        if (lane == 0) {
          const uint8_t* st = base + s * kStage;
          const uint32_t d = tmem + (uint32_t)(f % kAcc) * kBN;
          auto desc = [&](const uint8_t* tile, int k8) {
            return tc::smem_desc(tile + k8 * 32, 16, 1024, tc::kLayoutSW128);
          };
#pragma unroll
          for (int k8 = 0; k8 < kBK / 8; ++k8) {
            const uint32_t acc = (start && k8 == 0) ? 0u : 1u;
            if (SPLIT) {
              tc::mma_tf32_ss(d, desc(st + 2 * kTile, k8), desc(st + kTile, k8), idesc, acc);  // lo(X) hi(W)
              tc::mma_tf32_ss(d, desc(st, k8), desc(st + 3 * kTile, k8), idesc, 1u);           // hi(X) lo(W)
              tc::mma_tf32_ss(d, desc(st, k8), desc(st + kTile, k8), idesc, 1u);               // hi(X) hi(W)
            } else {
              tc::mma_tf32_ss(d, desc(st, k8), desc(st + kTile, k8), idesc, acc);
            }
          }
          tc::commit(&B->empty[s]);
          if (end) tc::commit(&B->accf[f % kAcc]);
        }
        __syncwarp();
        if (end) ++f;
      }
    }
    if (!ok && lane == 0) report_error(L.status, DEV_TIMEOUT, 55, g);
  } else {
    // ---------------- epilogue (warps 2..5): one output row per thread ----------------
    const int q4 = warp & 3;  // this warp's 32 rows of the tile (its TMEM lanes); lane = row
    const uint32_t tl = tmem + ((uint32_t)(32 * q4) << 16);
    int f = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < L.total; t += gridDim.x) {
      const TileRef T = tile_ref(L, t);
      const int nkb = T.p->nkb;
      // the problem's epilogue fields in registers (the stores below would otherwise make the
      // compiler reload them from global memory for every column)
      // (the empty asm statements make the values opaque: at this register pressure the
      // compiler would otherwise re-load them from the descriptor in global memory at each use,
      // a dependent load per output column)
      const LinProb& P = T.p->p;
      const float* bias = P.bias;
      const float* gate = P.gate;
      const float* resid = P.resid;
      float* y = P.y;
      int64_t ldy = P.ldy, ldr = P.ldr;
      int act = P.act, M = P.M, N = P.N;
      asm volatile("" : "+l"(bias), "+l"(gate), "+l"(resid), "+l"(y), "+l"(ldy), "+l"(ldr));
      asm volatile("" : "+r"(act), "+r"(M), "+r"(N));
      const int c0 = T.nt * kBN;
      const int nc = min(kBN, N - c0);
      // the row starts at the bias: its loads are issued here, ahead of the wait for the first
      // partial sum (at this register pressure, loads in the epilogue loop would run one by one)
      float o[kBN];
#pragma unroll
      for (int c = 0; c < kBN; ++c) o[c] = (bias && c < nc) ? __ldg(bias + c0 + c) : 0.f;
      int flast = f;  // the partial sum whose accumulator ends up holding the finished row
      for (int kb0 = 0; kb0 < nkb; kb0 += kFlush, ++f) {
        ok = __all_sync(0xffffffffu, wait_or_abort(&B->accf[f % kAcc], (uint32_t)((f / kAcc) & 1), abort, L.status,
                                                   W_ACCF, f));
        if (!ok) break;
        tc::fence_after_sync();
        const uint32_t acc = tl + (uint32_t)(f % kAcc) * kBN;
#pragma unroll
        for (int c32 = 0; c32 < kBN / 32; ++c32) {
          float ad[32];
          tc::tmem_ld32(acc + 32 * c32, ad);
          tc::tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const float2 x = __fadd2_rn(make_float2(o[32 * c32 + c], o[32 * c32 + c + 1]), make_float2(ad[c], ad[c + 1]));
            o[32 * c32 + c] = x.x;
            o[32 * c32 + c + 1] = x.y;
          }
        }
        if (kb0 + kFlush < nkb) {
          tc::fence_before_sync();
          mbar_arrive(&B->acce[f % kAcc]);
        } else {
          // the finished row goes back into this accumulator, which the epilogue below reads in
          // 32-column chunks (with the row no longer held in registers) and then releases
#pragma unroll
          for (int c32 = 0; c32 < kBN / 32; ++c32) {
            float t32[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) t32[c] = o[32 * c32 + c];
            tc::tmem_st32(acc + 32 * c32, t32);
          }
          tc::tmem_wait_st();
          flast = f;
        }
      }
      if (!ok) break;
      // y = resid + gate * act(o + bias), the reference's epilogue order, in 32-column chunks read
      // back from TMEM (the row started at the bias; gate is the same column for every thread:
      // broadcast loads). y leaves through TMA stores, or each thread stores its own row (float4
      // when the rows are 16-byte aligned). (Staging through shared memory for coalesced rows and
      // reading it back was slower: shared loads wait about a thousand cycles while the tensor
      // core streams the next tile's operands.)
      const uint32_t accl = tl + (uint32_t)(flast % kAcc) * kBN;
      const int r = T.mt * kBM + 32 * q4 + lane;
      int my = T.p->my;
      asm volatile("" : "+r"(my));
      const CUtensorMap* ymap = L.maps + (my >= 0 ? my : 0);
      uint8_t* slots = base + OFF_EPI + q4 * 2 * kSlot;
      const float* rrow = (resid && r < M) ? resid + (int64_t)r * ldr + c0 : nullptr;
      float* yrow = y + (int64_t)r * ldy + c0;
      const bool rvec = rrow && (reinterpret_cast<uintptr_t>(rrow) & 15u) == 0 && (nc & 3) == 0;
      const bool yvec = (reinterpret_cast<uintptr_t>(yrow) & 15u) == 0 && (nc & 3) == 0;
      // Without gate and activation each 32-column block is read and written whole; with either,
      // in a loop over 4-column groups that is not unrolled (unrolled 32-wide with the three
      // activations' code ran about three times slower than the whole product without them).
      const bool plain = !gate && act == kActNone;
#pragma unroll
      for (int cb = 0; cb < kBN / 32; ++cb) {
        // blocks wholly past N are skipped altogether (every block written to a slot is stored,
        // which is what keeps "at most one store still reading" on the other slot)
        if (32 * cb >= nc) break;
        uint8_t* slot = slots + (cb & 1) * kSlot;
        if (my >= 0) {
          if (lane == 0) tc::bulk_wait_group_read<1>();
          __syncwarp();
        }
        if (plain) {
          float v[32];
          tc::tmem_ld32(accl + 32 * cb, v);
          tc::tmem_wait_ld();
          if (rrow) {
            if (rvec) {
#pragma unroll
              for (int c = 0; c < 32; c += 4)
                if (32 * cb + c < nc) {
                  const float4 rv = *reinterpret_cast<const float4*>(rrow + 32 * cb + c);
                  v[c] += rv.x, v[c + 1] += rv.y, v[c + 2] += rv.z, v[c + 3] += rv.w;
                }
            } else {
#pragma unroll
              for (int c = 0; c < 32; ++c)
                if (32 * cb + c < nc) v[c] += rrow[32 * cb + c];
            }
          }
          if (my >= 0) {
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4)
              *reinterpret_cast<float4*>(slot + lane * 128 + ((c4 ^ (lane & 7)) << 4)) =
                  make_float4(v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
          } else if (r < M) {
            if (yvec) {
#pragma unroll
              for (int c = 0; c < 32; c += 4)
                if (32 * cb + c < nc)
                  *reinterpret_cast<float4*>(yrow + 32 * cb + c) = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
            } else {
#pragma unroll
              for (int c = 0; c < 32; ++c)
                if (32 * cb + c < nc) yrow[32 * cb + c] = v[c];
            }
          }
        } else {
          // one loop per activation, chosen outside it (the activation known at compile time
          // keeps each loop's code small)
          auto groups = [&](auto actc) {
            constexpr int A = decltype(actc)::value;
#pragma unroll 2
            for (int c4 = 0; c4 < 8; ++c4) {
              const int cc = 32 * cb + 4 * c4;  // first of the group's 4 columns in the tile
              const float4 q = tc::tmem_ld4(accl + cc);
              tc::tmem_wait_ld();
              float e[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                if (cc + u < nc) {
                  if constexpr (A != kActNone) e[u] = linear_act(A, e[u]);
                  if (gate) e[u] *= __ldg(gate + c0 + cc + u);
                  if (rrow) e[u] += rrow[cc + u];
                }
              }
              if (my >= 0) {
                *reinterpret_cast<float4*>(slot + lane * 128 + ((c4 ^ (lane & 7)) << 4)) =
                    make_float4(e[0], e[1], e[2], e[3]);
              } else if (r < M) {
                if (yvec && cc < nc) {
                  *reinterpret_cast<float4*>(yrow + cc) = make_float4(e[0], e[1], e[2], e[3]);
                } else {
#pragma unroll
                  for (int u = 0; u < 4; ++u)
                    if (cc + u < nc) yrow[cc + u] = e[u];
                }
              }
            }
          };
          switch (act) {
            case kActGelu: groups(std::integral_constant<int, kActGelu>{}); break;
            case kActGeluTanh: groups(std::integral_constant<int, kActGeluTanh>{}); break;
            case kActSilu: groups(std::integral_constant<int, kActSilu>{}); break;
            default: groups(std::integral_constant<int, kActNone>{}); break;
          }
        }
        if (my >= 0) {
          // TMA store of the 32 x 32 block (16-byte chunks swizzled by row, SWIZZLE_128B); the TMA
          // clips rows past M and columns past N. A slot is rewritten once at most one store (the
          // other slot's) is still reading.
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tc::tma_store_2d(ymap, slot, c0 + 32 * cb, T.mt * kBM + 32 * q4);
            tc::bulk_commit_group();
          }
        }
      }
      tc::fence_before_sync();
      mbar_arrive(&B->acce[flast % kAcc]);  // the finished row's accumulator is free again
    }
    if (!ok && lane == 0) report_error(L.status, DEV_TIMEOUT, 56, f);
    if (lane == 0) tc::bulk_wait_group_all();  // this warp's TMA stores are complete
  }

  tc::fence_before_sync();
  __syncthreads();
  if (*abort && warp == 1) {
    if (lane == 0) {
      tc::commit(&B->drain);
      mbar_wait_bounded(&B->drain, 0);
    }
    __syncwarp();
  }
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------------------------------------
// hi / lo split of every job of a flush, one 32-row x 128-column tile per block iteration. Value
// order: x * xscale, times rowscale[r] when set (a gate folded into w, with the bias scaled
// alongside), normalised when gn_stats is set: (x - mean) * rstd * g + b (then SiLU if asked) with
// g, b = gamma, beta (GroupNorm), 1 + scale, shift (modulated LayerNorm) or 1, 0 (plain
// LayerNorm), as the linear_fp32 prologue applies them. Lanes run along k: a job whose rows are
// 16-byte aligned moves 16 bytes per lane (512-byte rows per warp, a warp's 4 rows loaded before
// any is stored), others 4 bytes per lane; a transposed job ([K, rows] source) goes through a
// shared-memory tile so that its loads run along r.
constexpr int kSplitRows = kSplitTileRows, kSplitCols = kSplitTileCols;

__device__ __forceinline__ void split_store(const SplitJob& J, int32_t r, int32_t k, float x) {
  const float h = __uint_as_float(__float_as_uint(x) & 0xffffe000u);
  if (J.hi) J.hi[(int64_t)r * J.ldd + k] = h;
  if (J.lo) J.lo[(int64_t)r * J.ldd + k] = x - h;
}

// TRANS: the launch has transposed jobs (the form without them keeps fewer registers and no
// transposition tile)
template <bool TRANS>
__global__ void __launch_bounds__(256) split_kernel(const SplitLaunch L) {
  static_assert(kSplitRows == 32, "the transposition tile's swizzle spans 32 columns");
  __shared__ float t[TRANS ? kSplitCols : 1][kSplitRows];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int tile = blockIdx.x; tile < L.total; tile += gridDim.x) {
    const int ji = find_problem(L.begin, L.n, tile);
    const SplitJob J = L.jobs[ji];
    const int local = tile - __ldg(L.begin + ji);
    const int rt = local / J.ktiles, kt = local - rt * J.ktiles;
    const int32_t r0 = rt * kSplitRows, k0 = kt * kSplitCols;
    if (TRANS && J.trans) {  // (uniform over the block: one job per tile)
      // element (r, k) of the tile at t[k][r ^ ((k >> 2) & 31)]: the loads (one k, lanes along r)
      // and the 16-byte stores' reads (one r, lane l reading k = 4l .. 4l + 3) both hit 32
      // distinct banks
#pragma unroll 4
      for (int kk = ty; kk < kSplitCols; kk += 8) {
        const int32_t k = k0 + kk, r = r0 + tx;
        t[kk][tx ^ ((kk >> 2) & 31)] =
            (k < J.K && r < J.rows) ? __ldg(J.src + (int64_t)k * J.ld + r) * J.xscale : 0.f;
      }
      __syncthreads();
      const bool vec = ((J.K | J.ldd) & 3) == 0 &&
                       ((reinterpret_cast<uintptr_t>(J.hi) | reinterpret_cast<uintptr_t>(J.lo)) & 15u) == 0;
      for (int rr = ty; rr < kSplitRows; rr += 8) {
        const int32_t r = r0 + rr;
        if (r >= J.rows) break;
        if (vec) {  // lane tx: columns k0 + 4 tx .. +3 of row r, one 16-byte store per array
          const int32_t k = k0 + 4 * tx;
          if (k >= J.K) continue;
          float v[4], h[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            v[e] = t[4 * tx + e][rr ^ tx];
            h[e] = __uint_as_float(__float_as_uint(v[e]) & 0xffffe000u);
          }
          const int64_t o = (int64_t)r * J.ldd + k;
          if (J.hi) *reinterpret_cast<float4*>(J.hi + o) = make_float4(h[0], h[1], h[2], h[3]);
          if (J.lo) *reinterpret_cast<float4*>(J.lo + o) = make_float4(v[0] - h[0], v[1] - h[1], v[2] - h[2], v[3] - h[3]);
        } else {
#pragma unroll
          for (int c = 0; c < kSplitCols / 32; ++c) {
            const int kl = 32 * c + tx;
            if (k0 + kl < J.K) split_store(J, r, k0 + kl, t[kl][rr ^ ((kl >> 2) & 31)]);
          }
        }
      }
      __syncthreads();  // the tile buffer is rewritten by the next iteration
      continue;
    }
    // 16-byte rows (every job's copy, and sources whose rows are 16-byte aligned): lane tx owns
    // columns k0 + 4 tx .. +3, and the 4 rows of a warp are loaded before any is stored
    const bool vec = ((J.ld | J.K | J.ldd) & 3) == 0 && ((reinterpret_cast<uintptr_t>(J.src) |
                                                         reinterpret_cast<uintptr_t>(J.hi) |
                                                         reinterpret_cast<uintptr_t>(J.lo)) & 15u) == 0;
    if (vec) {
      constexpr int kRw = kSplitRows / 8;  // rows per warp
      const int32_t k = k0 + 4 * tx;
      float4 xv[kRw];
#pragma unroll
      for (int i = 0; i < kRw; ++i) {
        const int32_t r = r0 + ty + 8 * i;
        xv[i] = (r < J.rows && k < J.K) ? __ldg(reinterpret_cast<const float4*>(J.src + (int64_t)r * J.ld + k))
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < kRw; ++i) {
        const int32_t r = r0 + ty + 8 * i;
        if (r >= J.rows) break;
        float g = J.xscale;
        if (J.rowscale) {
          const float rs = __ldg(J.rowscale + r);
          g *= rs;
          if (J.bias_out && kt == 0 && tx == 0) J.bias_out[r] = J.bias_in ? __ldg(J.bias_in + r) * rs : 0.f;
        }
        if (k >= J.K) continue;
        float v[4] = {xv[i].x * g, xv[i].y * g, xv[i].z * g, xv[i].w * g};
        if (J.gn_stats) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 ms = __ldg(J.gn_stats + (int64_t)(r / J.gn_rows) * J.gn_groups + (k + e) / J.gn_cg);
            float ga = 1.f, b = 0.f;
            if (J.gn_mode != kNormPlain) {
              ga = __ldg(J.gamma + k + e);
              b = __ldg(J.beta + k + e);
              if (J.gn_mode == kNormModulated) ga = 1.f + ga;
            }
            v[e] = (v[e] - ms.x) * ms.y * ga + b;
            if (J.gn_silu) v[e] = v[e] / (1.f + __expf(-v[e]));
          }
        }
        float h[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) h[e] = __uint_as_float(__float_as_uint(v[e]) & 0xffffe000u);
        const int64_t o = (int64_t)r * J.ldd + k;
        if (J.hi) *reinterpret_cast<float4*>(J.hi + o) = make_float4(h[0], h[1], h[2], h[3]);
        if (J.lo) *reinterpret_cast<float4*>(J.lo + o) = make_float4(v[0] - h[0], v[1] - h[1], v[2] - h[2], v[3] - h[3]);
      }
      continue;
    }
    for (int rr = ty; rr < kSplitRows; rr += 8) {
      const int32_t r = r0 + rr;
      if (r >= J.rows) break;
      const float* src = J.src + (int64_t)r * J.ld;
      float g = J.xscale;
      if (J.rowscale) {
        const float rs = __ldg(J.rowscale + r);
        g *= rs;
        if (J.bias_out && kt == 0 && tx == 0) J.bias_out[r] = J.bias_in ? __ldg(J.bias_in + r) * rs : 0.f;
      }
      float x[kSplitCols / 32];
#pragma unroll
      for (int c = 0; c < kSplitCols / 32; ++c) {
        const int32_t k = k0 + 32 * c + tx;
        x[c] = k < J.K ? __ldg(src + k) : 0.f;
      }
#pragma unroll
      for (int c = 0; c < kSplitCols / 32; ++c) {
        const int32_t k = k0 + 32 * c + tx;
        if (k >= J.K) continue;
        float v = x[c] * g;
        if (J.gn_stats) {
          const float2 ms = __ldg(J.gn_stats + (int64_t)(r / J.gn_rows) * J.gn_groups + k / J.gn_cg);
          float ga = 1.f, b = 0.f;
          if (J.gn_mode != kNormPlain) {
            ga = __ldg(J.gamma + k);
            b = __ldg(J.beta + k);
            if (J.gn_mode == kNormModulated) ga = 1.f + ga;
          }
          v = (v - ms.x) * ms.y * ga + b;
          if (J.gn_silu) v = v / (1.f + __expf(-v));
        }
        split_store(J, r, k, v);
      }
    }
  }
}

}  // namespace

cudaError_t launch_split(const SplitLaunch& L, cudaStream_t s) {
  if (L.total <= 0) return cudaSuccess;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = L.total < 8 * sms ? L.total : 8 * sms;
  if (L.trans_jobs == 0) split_kernel<false><<<grid, 256, 0, s>>>(L);
  else split_kernel<true><<<grid, 256, 0, s>>>(L);
  return cudaGetLastError();
}

cudaError_t launch_linear_tc(const LinTcLaunch& L, bool split, cudaStream_t s) {
  if (L.total <= 0) return cudaSuccess;
  auto k = split ? linear_tc_kernel<true> : linear_tc_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = L.total < sms ? L.total : sms;
  k<<<grid, kThreads, SMEM_BYTES, s>>>(L);
  return cudaGetLastError();
}

}  // namespace supra
