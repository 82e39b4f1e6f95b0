// TF32 tensor-core attention for sm_100a: tcgen05.mma with TMEM accumulators, TMA-staged tiles.
// Head dim 64 (the DiT self/cross-attention call sites, app/models/dit.js:172,184, and the T5
// encoder attention, app/models/t5.js:80, whose [H, Lq, Lk] relative-position bias the softmax
// warps add to the scores read from TMEM).
//
// Same math as the reference's fused kernel (app/gpu/kernels.js:164-316: online softmax over key
// blocks, O / l at the end), with both contractions on the 5th-generation tensor cores:
//   S_n = Q K_n^T   tcgen05.mma kind::tf32, A = Q (TMEM), B = K_n (smem, K-major),
//                   D = S_n in TMEM (128 lanes = query rows x 64 columns = keys), fp32
//   P_n            softmax warps read S_n from TMEM (one row per thread), compute
//                   exp2(s*scale*log2e - m), round to TF32 and write P_n over S_n in TMEM
//   O += P_n V_n   tcgen05.mma kind::tf32, A = P_n from TMEM, B = V_n (smem, MN-major), D = O in TMEM
// Persistent CTAs: CTA b takes tiles b, b + grid, b + 2*grid, ... of the launch's list of
// (problem, head, 128-row query tile); the key blocks of all its tiles form one stream n = 0, 1, ...
// that flows through separate K and V rings (2 stages each; a K stage is released once its S
// product is done, a V stage once its PV product is) and a double-buffered S/P in TMEM without
// draining at tile boundaries. 6 warps:
//   warp 0     TMA producer: lane 0 per tile the Q tile (as soon as the softmax threads have
//              copied the previous one into TMEM, so it lands while the previous tile runs),
//              then the K blocks of 64 keys; lane 1 the V blocks, so K runs ahead of the V stages
//   warp 1     TMEM allocation and the single-thread MMA issuer; S_n is issued before PV_{n-1}
//              so the tensor core computes S_n while the softmax warps work on P_{n-1}
//   warps 2-5  softmax and epilogue; warp w owns TMEM lanes 32*(w%4) .. +31 (query rows)
// TMEM: S/P double buffer (2 x 64 columns), O (64 columns) and Q (64 columns, the softmax threads
// copy each tile's Q rows there from the landed tile: at the start of the CTA's first tile, and
// for later tiles right after the previous tile's last P, once its last S product is done):
// 256 columns, two CTAs per SM. The MMA warp issues a tile's last PV before it waits for the next
// tile's Q in TMEM.
// The running maximum moves lazily (only when a block exceeds it by more than 8 in log2 units),
// so O is rarely rescaled; when it is, the softmax warps wait for the previous PV product and
// rescale O in TMEM. The first PV of a tile overwrites O once the previous tile's epilogue has
// read it.
// Q and K tiles are loaded with the 128-byte swizzle (K-major operands), V tiles with the
// 128-byte / 32-byte-atom swizzle (the MN-major TF32 operand layout); every CTA loads only its own tiles.
// Every wait is bounded; on a timeout the CTA records the failure, drains the MMAs it issued,
// frees its TMEM and leaves.
//
// Split precision (SPLIT = true, variant TF32X3): fp32-class accuracy from the same tensor cores.
// The TMA copies the operands exactly (fp32 tensor maps). hi is x with its 13 low mantissa bits
// cleared: the tensor core ignores those bits of a TF32 operand, so the landed K and V tiles
// serve as their own hi parts, and two converter warps (6: K, 7: V) write lo = x - hi (exact)
// into a second copy. The softmax threads split their Q rows into hi(Q) / lo(Q) in TMEM (the A
// operand of S) and P the same way. K and V have separate rings, so the next K blocks land
// while a V stage waits for its PV product. Every product is formed as
// lo*hi + hi*lo + hi*hi (three TF32 MMAs, the small terms first), which leaves an error of about
// 2^-21 relative per product. Each block's PV product goes into a fresh TMEM accumulator and the
// softmax threads add it to O in fp32 registers (rounded to nearest), so the error does not grow
// with the number of key blocks. Q is double-buffered in TMEM: the next tile's Q rows are split
// right after the current tile's last P, so the tensor core starts the next tile while the
// epilogue runs (the MMA warp issues a tile's last PV before waiting for the next Q). One CTA
// per SM (the tiles take twice the shared memory).
#include "tcgen05.cuh"

namespace supra {
namespace {

constexpr int kM = 128;  // query rows per tile (MMA M)
constexpr int kN = 64;   // keys per block (MMA N of S)
constexpr int kD = 64;   // head dim (MMA N of O)
constexpr int kNS = 2;   // K stages
constexpr int kNSV = 3;  // V stages of the split kernel (a V stage is held until its PV product is done)
constexpr uint32_t kQSlab = kM * 128;   // one 32-column slab of the Q tile: 16 KB
constexpr uint32_t kKVSlab = kN * 128;  // one 32-column slab of a K or V block: 8 KB
constexpr uint32_t kQBytes = 2 * kQSlab;
constexpr uint32_t kKVBytes = 2 * kKVSlab;  // one K (or V) block
constexpr uint32_t kOStage = 16 * 32 * 4;   // epilogue staging: 16 rows x 32 columns of O per softmax warp

// Shared memory, TMEM and threads of the plain (SPLIT = false) and split-precision kernels. The
// split kernel keeps K and V tiles twice, hi (x with its low mantissa bits cleared) in place of
// x and lo = x - hi beside it, in separate K and V rings: one CTA per SM, 512 TMEM columns
// (S/hi(P) double buffer, lo(P), the per-block PV accumulator and two hi(Q) | lo(Q) buffers),
// and a fourth role, the converter warps.
template <bool SPLIT>
struct Lay {
  static constexpr uint32_t Q = 0;
  static constexpr uint32_t K = Q + kQBytes;
  static constexpr uint32_t KL = K + kNS * kKVBytes;
  static constexpr uint32_t V = SPLIT ? KL + kNS * kKVBytes : K + kNS * kKVBytes;
  static constexpr uint32_t VL = V + kNSV * kKVBytes;
  static constexpr uint32_t O = SPLIT ? VL + kNSV * kKVBytes : V + kNS * kKVBytes;
  static constexpr uint32_t BAR = O + 4 * kOStage;
  static constexpr uint32_t TILES = BAR + 256;         // the CTA's claimed tiles (TileSlot table)
  static constexpr uint32_t SMEM = TILES + 64 + 1024;  // + alignment slack for the 1024-B base
  static constexpr uint32_t TMEM_COLS = SPLIT ? 512 : 256;
  static constexpr int THREADS = SPLIT ? 256 : 192;  // 8 warps: two per SM sub-partition, up to 255 registers
  static constexpr int CTAS_PER_SM = SPLIT ? 1 : 2;
  static constexpr int NSV = SPLIT ? kNSV : kNS;  // V stages
};
static_assert(Lay<true>::SMEM <= 227 * 1024 && 2 * Lay<false>::SMEM <= 228 * 1024, "shared memory");
constexpr uint32_t COL_S0 = 0, COL_S1 = 64, COL_O = 128;
// plain kernel: the tile's Q rows, the A operand of S, copied from the landed smem tile by the
// softmax threads so that the smem tile is free for the next tile's Q at once
constexpr uint32_t COL_QP = 192;
// split kernel: lo(P), a fresh per-block PV accumulator (O itself lives in the softmax threads'
// registers), and two buffers of hi(Q) | lo(Q) (64 + 64 columns), the A operand of S, so the
// next tile's Q is split before the current tile's epilogue
constexpr uint32_t COL_PL = 128, COL_OB = 192, COL_Q0 = 256, COL_Q1 = 384;
constexpr int kBatch = 8;  // converter: 16-byte chunks per lane loaded before any is stored
constexpr int kConv = 32;  // threads per converter warp (split kernel: warp 6 for K, warp 7 for V)

// pv_done is double-buffered by block parity so that a waiter for PV_n never sees a barrier
// that is two phases ahead or behind (PV_{n-2} is always complete when PV_n is awaited).
struct Bars {
  uint64_t q_full, q_empty, kv_full[kNS], kv_empty[kNS], s_full[2], p_full[2], pv_done[2], o_empty, drain;
  // K and V flow through separate rings (kv_full / kv_empty serve K, released once S is done;
  // v_full / v_empty serve V, released once PV is done); in the split kernel each landed tile
  // is released to the MMA warp once its lo part is in place (kv_conv, v_conv)
  uint64_t q_conv, kv_conv[kNS], v_full[kNSV], v_empty[kNSV], v_conv[kNSV];
  uint32_t tmem;
  int32_t abort;
};
static_assert(sizeof(Bars) <= 256, "barrier block");

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Wait ids reported with a timeout (status[2]); status[3] carries the waiter's block counter.
enum WaitId : int32_t {
  W_Q_EMPTY = 31, W_KV_EMPTY = 32, W_Q_FULL = 33, W_KV_FULL = 34, W_P_FULL = 35, W_O_EMPTY = 36,
  W_S_FULL = 37, W_PV_RESCALE = 38, W_PV_EPILOGUE = 39, W_CONV_Q = 40, W_CONV_KV = 41, W_TILE = 42,
};

// The split of the 3xTF32 scheme, x*y ~ hi(x)hi(y) + hi(x)lo(y) + lo(x)hi(y): hi = x with the
// 13 low mantissa bits cleared (a TF32 value, so the tensor core takes it exactly) and
// lo = x - hi, exact in fp32 and below 2^-10 |x|; the tensor core keeps 11 significant bits of
// lo, so what is lost is below 2^-21 |x|. (Clearing bits is one logic op; a rounding convert
// costs several instructions per element.)
__device__ __forceinline__ float hi_of(float x) { return __uint_as_float(__float_as_uint(x) & 0xffffe000u); }
__device__ __forceinline__ void split4(float4& x, float4& lo) {
  const float4 h = make_float4(hi_of(x.x), hi_of(x.y), hi_of(x.z), hi_of(x.w));
  const float2 neg1 = make_float2(-1.f, -1.f);  // x - hi as packed f32x2 FFMAs (exact)
  const float2 a = __ffma2_rn(make_float2(h.x, h.y), neg1, make_float2(x.x, x.y));
  const float2 b = __ffma2_rn(make_float2(h.z, h.w), neg1, make_float2(x.z, x.w));
  lo = make_float4(a.x, a.y, b.x, b.y);
  x = h;
}

// Bounded wait that also gives up as soon as another warp of the CTA has aborted. The thread
// whose own wait runs out reports which barrier it was and the block counter it waited for.
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

// The CTA's tiles in claim order: tile k (k = 0, 1, ...) sits in slot k % kTileSlots with
// seq = k + 1. Tile 0 is blockIdx.x; the Q/K producer claims each later one from the launch's
// counter (L.next_tile) as it starts it and publishes it here, and every other role reads it
// before working on it. (With a fixed stride blockIdx.x, + gridDim.x, ... the two CTAs that
// share an SM progress at different rates and the slower one finishes alone.) The producer runs
// at most a few tiles ahead of the slowest role, well inside the 8 slots; a slot that does not
// hold the awaited tile within the wait limit is reported like any other wait.
constexpr int kTileSlots = 8;
struct TileSlot {
  int32_t seq, t;
};
static_assert(sizeof(TileSlot) * kTileSlots <= 64, "tile table");

__device__ __forceinline__ void publish_tile(TileSlot* tab, int k, int t) {
  volatile TileSlot* s = tab + (k % kTileSlots);
  s->t = t;
  __threadfence_block();
  s->seq = k + 1;
}

__device__ __forceinline__ bool tile_at(TileSlot* tab, int k, int* t, volatile int32_t* abort, int32_t* status) {
  volatile TileSlot* s = tab + (k % kTileSlots);
  if (s->seq != k + 1) {
    const uint64_t t0 = global_ns();
    for (uint32_t it = 1;; ++it) {
      if (s->seq == k + 1) break;
      if ((it & 63u) == 0u) {
        if (*abort) return false;
        if (global_ns() - t0 > kWaitLimitNs) {
          report_error(status, DEV_TIMEOUT, W_TILE, k);
          *abort = 1;
          return false;
        }
      }
    }
  }
  __threadfence_block();
  *t = s->t;
  return true;
}

// A tile of the launch: problem, head and first query row.
struct Tile {
  const TmaProb* p;
  int h, q0, nblk;
};
__device__ __forceinline__ Tile tile_of(const TmaLaunch& L, int t) {
  Tile r;
  const int pidx = L.uniform > 0 ? t / L.uniform : find_problem(L.begin, L.n, t);
  r.p = L.probs + pidx;
  const int local = t - (L.uniform > 0 ? pidx * L.uniform : __ldg(L.begin + pidx));
  const int q_tiles = r.p->q_tiles;
  r.h = local / q_tiles;
  r.q0 = (local - r.h * q_tiles) * kM;
  r.nblk = (r.p->Lk + kN - 1) / kN;
  return r;
}

// Split kernel, softmax threads: this thread's row of the landed Q tile (row r of a 32-column
// slab is 128 bytes at r * 128, its 16-byte chunks swizzled by r % 8: SWIZZLE_128B) into hi(Q)
// at column qh and lo(Q) at qh + 64 of its TMEM lane.
__device__ __forceinline__ void split_q_row(const uint8_t* Qs, int row, uint32_t taddr_qh) {
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    float hi[32], lo[32];
    const uint8_t* qrow = Qs + hf * kQSlab + row * 128;
#pragma unroll
    for (int c4 = 0; c4 < 8; ++c4) {
      float4 x = *reinterpret_cast<const float4*>(qrow + ((c4 ^ (row & 7)) << 4)), l4;
      split4(x, l4);
      hi[4 * c4] = x.x, hi[4 * c4 + 1] = x.y, hi[4 * c4 + 2] = x.z, hi[4 * c4 + 3] = x.w;
      lo[4 * c4] = l4.x, lo[4 * c4 + 1] = l4.y, lo[4 * c4 + 2] = l4.z, lo[4 * c4 + 3] = l4.w;
    }
    tc::tmem_st32(taddr_qh + 32 * hf, hi);
    tc::tmem_st32(taddr_qh + 64 + 32 * hf, lo);
    tc::tmem_wait_st();
  }
}

// Maximum of a row's 64 scores through eight partial maxima (one 64-long chain of dependent max
// operations cost ~256 cycles per block).
__device__ __forceinline__ float max64(const float (&v)[64]) {
  float rp[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) rp[u] = v[u];
#pragma unroll
  for (int c = 8; c < 64; ++c) rp[c & 7] = fmaxf(rp[c & 7], v[c]);
  return fmaxf(fmaxf(fmaxf(rp[0], rp[1]), fmaxf(rp[2], rp[3])), fmaxf(fmaxf(rp[4], rp[5]), fmaxf(rp[6], rp[7])));
}

// Plain kernel, softmax threads: this thread's row of the landed Q tile into TMEM at column qc of
// its lane, unchanged (the tensor core reads it as TF32).
__device__ __forceinline__ void copy_q_row(const uint8_t* Qs, int row, uint32_t taddr_q) {
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    float q[32];
    const uint8_t* qrow = Qs + hf * kQSlab + row * 128;
#pragma unroll
    for (int c4 = 0; c4 < 8; ++c4) {
      const float4 x = *reinterpret_cast<const float4*>(qrow + ((c4 ^ (row & 7)) << 4));
      q[4 * c4] = x.x, q[4 * c4 + 1] = x.y, q[4 * c4 + 2] = x.z, q[4 * c4 + 3] = x.w;
    }
    tc::tmem_st32(taddr_q + 32 * hf, q);
  }
  tc::tmem_wait_st();
}

template <bool BIAS, bool SPLIT>
__global__ void __launch_bounds__(Lay<SPLIT>::THREADS, Lay<SPLIT>::CTAS_PER_SM)
    attn_tf32_kernel(const __grid_constant__ TmaLaunch L) {
  using Y = Lay<SPLIT>;
  constexpr uint32_t kTmemCols = Y::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);  // 1024-B aligned for the swizzle atoms
  uint8_t* Qs = base + Y::Q;
  uint8_t* Ks = base + Y::K;
  uint8_t* Vs = base + Y::V;
  uint8_t* KLs = base + Y::KL;
  uint8_t* VLs = base + Y::VL;
  float* Os = reinterpret_cast<float*>(base + Y::O);
  Bars* B = reinterpret_cast<Bars*>(base + Y::BAR);
  volatile int32_t* abort = &B->abort;
  TileSlot* tab = reinterpret_cast<TileSlot*>(base + Y::TILES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&B->q_full, 1);
    mbar_init(&B->q_empty, 128);  // the softmax threads release the Q tile once it is in TMEM
    for (int s = 0; s < kNS; ++s) {
      mbar_init(&B->kv_full[s], 1);
      mbar_init(&B->kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&B->s_full[b], 1);
      mbar_init(&B->p_full[b], 128);
    }
    mbar_init(&B->pv_done[0], 1);
    mbar_init(&B->pv_done[1], 1);
    mbar_init(&B->o_empty, 128);
    mbar_init(&B->drain, 1);
    mbar_init(&B->q_conv, 128);  // split kernel: the softmax threads, one Q row each
    for (int s = 0; s < kNS; ++s) mbar_init(&B->kv_conv[s], kConv);
    for (int s = 0; s < Y::NSV; ++s) {
      mbar_init(&B->v_full[s], 1);
      mbar_init(&B->v_empty[s], 1);
      mbar_init(&B->v_conv[s], kConv);
    }
    B->abort = 0;
    TileSlot* tab0 = reinterpret_cast<TileSlot*>(base + Y::TILES);
    for (int i = 0; i < kTileSlots; ++i) tab0[i].seq = 0;
    tab0[0].t = (int32_t)blockIdx.x;
    tab0[0].seq = 1;
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
    if (lane == 1) {
      // the V ring, on its own lane so that K blocks run ahead of the V stages, which stay busy
      // until their PV products are done
      int n = 0;
      for (int k = 0;; ++k) {
        int t = 0;
        if (!tile_at(tab, k, &t, abort, L.status) || t >= L.total) break;
        const Tile T = tile_of(L, t);
        const TmaProb* pp = T.p;
        const CUtensorMap* mv = L.maps + pp->mv;
        const int vx = pp->vx + T.h * kD, vy = pp->vy;  // in registers (the TMA asm clobbers memory)
        bool ok = true;
        for (int j = 0; j < T.nblk; ++j, ++n) {
          const int s = n % Y::NSV;
          if (n >= Y::NSV && !(ok = wait_or_abort(&B->v_empty[s], (uint32_t)(((n / Y::NSV) - 1) & 1), abort, L.status, W_KV_EMPTY, n))) break;
          mbar_arrive_expect_tx(&B->v_full[s], kKVBytes);
          uint8_t* vd = Vs + s * kKVBytes;
          tc::tma_load_2d(vd, mv, vx, vy + j * kN, &B->v_full[s]);
          tc::tma_load_2d(vd + kKVSlab, mv, vx + 32, vy + j * kN, &B->v_full[s]);
        }
        if (!ok) break;
      }
    } else if (lane == 0) {
      int n = 0;
      for (int k = 0;; ++k) {
        int t = (int)blockIdx.x;
        if (k > 0) {  // claim and publish the CTA's next tile (past the end: every role stops)
          t = (int)gridDim.x + atomicAdd(L.next_tile, 1);
          publish_tile(tab, k, t);
        }
        if (t >= L.total) break;
        const Tile T = tile_of(L, t);
        const TmaProb* pp = T.p;
        const CUtensorMap* mq = L.maps + pp->mq;
        const CUtensorMap* mk = L.maps + pp->mk;
        const int hx = T.h * kD;
        const int kx = pp->kx + hx, ky = pp->ky;  // in registers (the TMA asm clobbers memory)
        if (k > 0 && !wait_or_abort(&B->q_empty, (uint32_t)((k - 1) & 1), abort, L.status, W_Q_EMPTY, n)) break;
        mbar_arrive_expect_tx(&B->q_full, kQBytes);
        tc::tma_load_2d(Qs, mq, pp->qx + hx, pp->qy + T.q0, &B->q_full);
        tc::tma_load_2d(Qs + kQSlab, mq, pp->qx + hx + 32, pp->qy + T.q0, &B->q_full);
        bool ok = true;
        for (int j = 0; j < T.nblk; ++j, ++n) {
          const int s = n % kNS;
          if (n >= kNS && !(ok = wait_or_abort(&B->kv_empty[s], (uint32_t)(((n / kNS) - 1) & 1), abort, L.status, W_KV_EMPTY, n))) break;
          mbar_arrive_expect_tx(&B->kv_full[s], kKVBytes);
          uint8_t* kd = Ks + s * kKVBytes;
          tc::tma_load_2d(kd, mk, kx, ky + j * kN, &B->kv_full[s]);
          tc::tma_load_2d(kd + kKVSlab, mk, kx + 32, ky + j * kN, &B->kv_full[s]);
        }
        if (!ok) break;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    const uint32_t idS = tc::idesc_tf32(kM, kN, false, false);
    const uint32_t idPV = tc::idesc_tf32(kM, kD, false, true);
    bool ok = true;
    int n = 0, k = 0;
    // the block whose PV product is still to be issued
    int pend_n = -1, pend_nk = 0, pend_k = 0;
    bool pend_first = false;
    auto issue_pv = [&]() -> bool {
      const int m = pend_n;
      const int sp = m % Y::NSV;
      const int bp = m & 1;
      if (!__all_sync(0xffffffffu, wait_or_abort(&B->p_full[bp], (uint32_t)((m >> 1) & 1), abort, L.status, W_P_FULL, m))) return false;
      if (!__all_sync(0xffffffffu, wait_or_abort(SPLIT ? &B->v_conv[sp] : &B->v_full[sp], (uint32_t)((m / Y::NSV) & 1),
                                                 abort, L.status, W_KV_FULL, m)))
        return false;
      if (!SPLIT && pend_first && pend_k > 0 &&
          !__all_sync(0xffffffffu, wait_or_abort(&B->o_empty, (uint32_t)((pend_k - 1) & 1), abort, L.status, W_O_EMPTY, m)))
        return false;
      uint8_t* vb = Vs + sp * kKVBytes;
      if (!SPLIT && pend_nk < kN) {  // (the split kernel's converter zeroes these rows)
        // V rows past Lk meet P == 0; make them zeros (they may hold another sequence's data).
        // Whole 128-byte rows, so the swizzle inside a row does not matter.
        for (int idx = lane; idx < (kN - pend_nk) * 16; idx += 32) {
          const int r = pend_nk + (idx >> 4);
          const int c = idx & 15;  // 16-byte chunk over both slabs
          *reinterpret_cast<float4*>(vb + (c >> 3) * kKVSlab + r * 128 + (c & 7) * 16) =
              make_float4(0.f, 0.f, 0.f, 0.f);
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      tc::fence_after_sync();
      if (lane == 0) {
        const uint32_t pcol = bp ? COL_S1 : COL_S0;
        // V is MN-major: 32-column atoms kKVSlab apart (LBO), 4-key groups 512 B apart (SBO)
        auto vdesc = [&](const uint8_t* v, int kk) {
          return tc::smem_desc(v + kk * 1024, kKVSlab, 512, tc::kLayoutSW128Base32B);
        };
        if (SPLIT) {
          // this block's P V into its own accumulator (the softmax threads add it to O in fp32):
          // lo(P) hi(V) + hi(P) lo(V) + hi(P) hi(V), the small terms first
          const uint32_t plcol = COL_PL;
          const uint32_t ob = tmem + COL_OB;
          const uint8_t* vl = VLs + sp * kKVBytes;
#pragma unroll
          for (int kk = 0; kk < kN / 8; ++kk)
            tc::mma_tf32_ts(ob, tmem + plcol + 8 * kk, vdesc(vb, kk), idPV, kk > 0 ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < kN / 8; ++kk) tc::mma_tf32_ts(ob, tmem + pcol + 8 * kk, vdesc(vl, kk), idPV, 1u);
#pragma unroll
          for (int kk = 0; kk < kN / 8; ++kk) tc::mma_tf32_ts(ob, tmem + pcol + 8 * kk, vdesc(vb, kk), idPV, 1u);
        } else {
#pragma unroll
          for (int kk = 0; kk < kN / 8; ++kk)
            tc::mma_tf32_ts(tmem + COL_O, tmem + pcol + 8 * kk, vdesc(vb, kk), idPV, (!pend_first || kk > 0) ? 1u : 0u);
        }
        tc::commit(&B->v_empty[sp]);
        tc::commit(&B->pv_done[m & 1]);
      }
      __syncwarp();
      pend_n = -1;
      return true;
    };
    for (; ok; ++k) {
      int t = 0;
      ok = __all_sync(0xffffffffu, tile_at(tab, k, &t, abort, L.status));
      if (!ok || t >= L.total) break;
      const Tile T = tile_of(L, t);
      int Lk = T.p->Lk;
      asm volatile("" : "+r"(Lk));  // kept in a register (see the softmax warps)
      // split kernel: the softmax threads split this tile's Q only after the previous tile's
      // epilogue, which waits for that tile's last PV product: issue it first
      if (pend_n >= 0) ok = issue_pv();
      if (!ok) break;
      ok = __all_sync(0xffffffffu, wait_or_abort(&B->q_conv, (uint32_t)(k & 1), abort, L.status,
                                                 W_Q_FULL, n));
      for (int j = 0; ok && j < T.nblk; ++j, ++n) {
        const int s = n % kNS;
        const int b = n & 1;
        ok = __all_sync(0xffffffffu, wait_or_abort(SPLIT ? &B->kv_conv[s] : &B->kv_full[s], (uint32_t)((n / kNS) & 1),
                                                   abort, L.status, W_KV_FULL, n));
        if (!ok) break;
        tc::fence_after_sync();
        if (lane == 0) {
          const uint8_t* kb = Ks + s * kKVBytes;
          const uint32_t scol = tmem + (b ? COL_S1 : COL_S0);
          // S = Q K^T with Q from TMEM (the split kernel: lo(Q) hi(K) + hi(Q) lo(K) + hi(Q) hi(K),
          // the small terms first)
          auto s_product_t = [&](uint32_t qcol, const uint8_t* kk, bool first) {
#pragma unroll
            for (int k8 = 0; k8 < kD / 8; ++k8) {
              const uint32_t offk = (uint32_t)(k8 >> 2) * kKVSlab + (uint32_t)(k8 & 3) * 32u;
              tc::mma_tf32_ts(scol, tmem + qcol + 8 * k8, tc::smem_desc(kk + offk, 16, 1024, tc::kLayoutSW128), idS,
                              (!first || k8 > 0) ? 1u : 0u);
            }
          };
          if (SPLIT) {
            const uint8_t* kl = KLs + s * kKVBytes;
            const uint32_t qh = (k & 1) ? COL_Q1 : COL_Q0, ql = qh + 64;
            s_product_t(ql, kb, true);
            s_product_t(qh, kl, false);
            s_product_t(qh, kb, false);
          } else {
            s_product_t(COL_QP, kb, true);
          }
          tc::commit(&B->kv_empty[s]);  // the K stage is free once S is done
          tc::commit(&B->s_full[b]);
        }
        __syncwarp();
        if (pend_n >= 0) ok = issue_pv();
        pend_n = n;
        pend_nk = min(kN, Lk - j * kN);
        pend_k = k;
        pend_first = (j == 0);
      }
    }
    if (ok && pend_n >= 0) ok = issue_pv();
    if (!ok && lane == 0) report_error(L.status, DEV_TIMEOUT, 21, n);
  } else if (warp < 6) {
    // ---------------- softmax + epilogue (warps 2..5) ----------------
    const int q4 = warp & 3;
    const int row = 32 * q4 + lane;
    const uint32_t tl = tmem + ((uint32_t)(32 * q4) << 16);
    bool ok = true;
    int n = 0;
    float v[64];
    float o[SPLIT ? 64 : 1];  // split kernel: this thread's row of O
    int kt = 0;               // this CTA's tile count
    // The CTA's first tile; each later one is looked up during the previous tile's last block
    // (its descriptor's loads then overlap that tile's epilogue).
    int t = 0;
    ok = __all_sync(0xffffffffu, tile_at(tab, 0, &t, abort, L.status));
    Tile Tn = ok && t < L.total ? tile_of(L, t) : Tile{};
    int Lkn = 0, Lqn = 0;
    float sl2n = 0.f;
    if (ok && t < L.total) {
      Lkn = Tn.p->Lk;
      Lqn = Tn.p->Lq;
      sl2n = Tn.p->scale_log2;
    }
    for (; ok && t < L.total; ++kt) {
      const Tile T = Tn;
      const TmaProb* pp = T.p;
      int Lk = Lkn, Lq = Lqn;
      float sl2 = sl2n;
      // opaque: kept in registers rather than re-loaded from the descriptor at each block
      asm volatile("" : "+r"(Lk), "+r"(Lq), "+f"(sl2));
      int tnext = L.total;
      float m = -INFINITY, l = 0.f;
      if constexpr (SPLIT) {
#pragma unroll
        for (int c = 0; c < 64; ++c) o[c] = 0.f;
      }
      if (kt == 0) {
        // the first tile's Q into TMEM; later tiles' Q rows go there during the previous tile's
        // last block (split kernel: into the other Q buffer), and the smem tile is released
        // right after, so the next tile's Q copy is in flight while this tile runs
        ok = __all_sync(0xffffffffu, wait_or_abort(&B->q_full, 0u, abort, L.status, W_CONV_Q, n));
        if (!ok) break;
        if constexpr (SPLIT) split_q_row(Qs, row, tl + COL_Q0);
        else copy_q_row(Qs, row, tl + COL_QP);
        tc::fence_before_sync();
        mbar_arrive(&B->q_conv);
        mbar_arrive(&B->q_empty);
      }
      for (int j = 0; j < T.nblk; ++j, ++n) {
        const int b = n & 1;
        ok = __all_sync(0xffffffffu, wait_or_abort(&B->s_full[b], (uint32_t)((n >> 1) & 1), abort, L.status, W_S_FULL, n));
        if (!ok) break;
        tc::fence_after_sync();
        const uint32_t scol = b ? COL_S1 : COL_S0;
        tc::tmem_ld64(tl + scol, v);
        tc::tmem_wait_ld();
        const int nk = min(kN, Lk - j * kN);
        float mx = -INFINITY;
        if (BIAS && T.q0 + row < Lq && pp->rel_lut) {
          // T5 table bias: this thread's query row, keys j*64 .. j*64 + nk (exp2 domain)
          const float* tab_h = pp->bias + T.h;
          const int32_t* lut_c = pp->rel_lut + pp->rel_max;
          const int32_t rel_max = pp->rel_max;
          const uint32_t Hu = (uint32_t)pp->H;
          const int32_t rel0 = j * kN - (T.q0 + row);
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            const float b = t5_table_bias(tab_h, lut_c, rel_max, Hu, rel0 + c);
            v[c] = (c < nk) ? fmaf(b, 1.4426950408889634f, v[c] * sl2) : -INFINITY;
          }
          mx = max64(v);
        } else if (BIAS && T.q0 + row < Lq) {
          // this thread's query row of the bias, keys j*64 .. j*64 + nk (exp2 domain: times log2 e)
          const float* brow = pp->bias + ((int64_t)T.h * Lq + T.q0 + row) * Lk + (int64_t)j * kN;
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            v[c] = (c < nk) ? fmaf(__ldg(brow + c), 1.4426950408889634f, v[c] * sl2) : -INFINITY;
          }
          mx = max64(v);
        } else if constexpr (!BIAS) {
          // no bias: the scores stay raw and the scale goes into the exponent's FFMA below; with
          // scale > 0 the raw row maximum times the scale is the scaled maximum. Keys past Lk
          // only in a ragged block (warp-uniform test).
          if (nk < kN) {
#pragma unroll
            for (int c = 0; c < 64; ++c) v[c] = (c < nk) ? v[c] : -INFINITY;
          }
          mx = max64(v) * sl2;
        } else {
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            v[c] = (c < nk) ? v[c] * sl2 : -INFINITY;
          }
          mx = max64(v);
        }
        const float vs = BIAS ? 1.f : sl2;  // exponent = v * vs - m
        const bool move = mx > m + 8.f;
        if constexpr (SPLIT) {
          // O stays in registers: hi(P_n) goes over S_n; then the previous block's accumulator
          // (its PV product is done once lo(P) may be overwritten) is added in fp32 and the sum
          // moved to the new offset, O = (O + OB_{n-1}) * 2^(m_old - m_new); then lo(P_n).
          // (pairs of columns go through the packed f32x2 FFMA / FADD / FMUL, same rounding)
          const float alpha = move ? ex2(m - mx) : 1.f;  // 0 on a tile's first block (m = -inf)
          if (move) m = mx;
          const float2 vs2 = make_float2(vs, vs), nm2 = make_float2(-m, -m);
          float2 ps2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
          for (int c = 0; c < 64; c += 2) {
            float2 a = __ffma2_rn(make_float2(v[c], v[c + 1]), vs2, nm2);
            a.x = ex2(a.x);
            a.y = ex2(a.y);
            v[c] = a.x;
            v[c + 1] = a.y;
            ps2[(c >> 1) & 3] = __fadd2_rn(ps2[(c >> 1) & 3], a);
          }
          const float2 pt = __fadd2_rn(__fadd2_rn(ps2[0], ps2[1]), __fadd2_rn(ps2[2], ps2[3]));
          l = l * alpha + (pt.x + pt.y);
          const float2 neg1 = make_float2(-1.f, -1.f);
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            float hi[32];
#pragma unroll
            for (int c = 0; c < 32; c += 2) {
              const float2 x = make_float2(v[32 * hf + c], v[32 * hf + c + 1]);
              const float2 h = make_float2(hi_of(x.x), hi_of(x.y));
              const float2 lo = __ffma2_rn(h, neg1, x);  // x - hi, exact
              hi[c] = h.x;
              hi[c + 1] = h.y;
              v[32 * hf + c] = lo.x;
              v[32 * hf + c + 1] = lo.y;
            }
            tc::tmem_st32(tl + scol + 32 * hf, hi);
            tc::tmem_wait_st();
          }
          if (j > 0) {
            ok = __all_sync(0xffffffffu, wait_or_abort(&B->pv_done[(n - 1) & 1], (uint32_t)(((n - 1) >> 1) & 1), abort,
                                                       L.status, W_PV_RESCALE, n));
            if (!ok) break;
            tc::fence_after_sync();
            const uint32_t ob = tl + COL_OB;
            const bool moved = !__all_sync(0xffffffffu, alpha == 1.f);
            const float2 al2 = make_float2(alpha, alpha);
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              float ad[32];
              tc::tmem_ld32(ob + 32 * hf, ad);
              tc::tmem_wait_ld();
#pragma unroll
              for (int c = 0; c < 32; c += 2) {
                float2 x = __fadd2_rn(make_float2(o[32 * hf + c], o[32 * hf + c + 1]), make_float2(ad[c], ad[c + 1]));
                if (moved) x = __fmul2_rn(x, al2);
                o[32 * hf + c] = x.x;
                o[32 * hf + c + 1] = x.y;
              }
            }
          }
          tc::tmem_st64(tl + COL_PL, v);
          tc::tmem_wait_st();
          tc::fence_before_sync();
          mbar_arrive(&B->p_full[b]);
          int tn = L.total;
          if (j == T.nblk - 1) {  // the CTA's next tile, once the producer has claimed it
            ok = __all_sync(0xffffffffu, tile_at(tab, kt + 1, &tn, abort, L.status));
            if (!ok) break;
            tnext = tn;
            if (tn < L.total) {
              Tn = tile_of(L, tn);
              Lkn = Tn.p->Lk;
              Lqn = Tn.p->Lq;
              sl2n = Tn.p->scale_log2;
            }
          }
          if (j == T.nblk - 1 && tn < L.total) {
            // the next tile's Q, into the other buffer, before this tile's epilogue: the tensor
            // core can start the next tile while the epilogue runs
            ok = __all_sync(0xffffffffu, wait_or_abort(&B->q_full, (uint32_t)((kt + 1) & 1), abort, L.status, W_CONV_Q, n));
            if (!ok) break;
            split_q_row(Qs, row, tl + (((kt + 1) & 1) ? COL_Q1 : COL_Q0));
            tc::fence_before_sync();
            mbar_arrive(&B->q_conv);
            mbar_arrive(&B->q_empty);
          }
          continue;
        }
        if (j > 0 && __any_sync(0xffffffffu, move)) {
          // O holds this tile's PV products up to block n-1: wait for it, rescale the moved rows
          ok = __all_sync(0xffffffffu, wait_or_abort(&B->pv_done[(n - 1) & 1], (uint32_t)(((n - 1) >> 1) & 1), abort,
                                                     L.status, W_PV_RESCALE, n));
          if (!ok) break;
          tc::fence_after_sync();
          const float alpha = move ? ex2(m - mx) : 1.f;
          float o[64];
          tc::tmem_ld64(tl + COL_O, o);
          tc::tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 64; ++c) o[c] *= alpha;
          tc::tmem_st64(tl + COL_O, o);
          tc::tmem_wait_st();
          l *= alpha;
        }
        if (move) m = mx;
        // (four packed partial sums rather than one 64-long chain of dependent adds)
        float2 ps2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        const float2 vs2 = make_float2(vs, vs), nm2 = make_float2(-m, -m);
#pragma unroll
        for (int c = 0; c < 64; c += 2) {
          const float2 a = __ffma2_rn(make_float2(v[c], v[c + 1]), vs2, nm2);
          const float2 p = make_float2(tc::to_tf32(ex2(a.x)), tc::to_tf32(ex2(a.y)));
          ps2[(c >> 1) & 3] = __fadd2_rn(ps2[(c >> 1) & 3], p);
          v[c] = p.x;
          v[c + 1] = p.y;
        }
        const float2 pt = __fadd2_rn(__fadd2_rn(ps2[0], ps2[1]), __fadd2_rn(ps2[2], ps2[3]));
        l += pt.x + pt.y;
        tc::tmem_st64(tl + scol, v);
        tc::tmem_wait_st();
        tc::fence_before_sync();
        mbar_arrive(&B->p_full[b]);
        if (j == T.nblk - 1) {
          // this tile's last S product is done: the CTA's next tile's Q rows into TMEM
          int tn = L.total;
          ok = __all_sync(0xffffffffu, tile_at(tab, kt + 1, &tn, abort, L.status));
          if (!ok) break;
          tnext = tn;
          if (tn < L.total) {
            Tn = tile_of(L, tn);
            Lkn = Tn.p->Lk;
            Lqn = Tn.p->Lq;
            sl2n = Tn.p->scale_log2;
            ok = __all_sync(0xffffffffu, wait_or_abort(&B->q_full, (uint32_t)((kt + 1) & 1), abort, L.status, W_CONV_Q, n));
            if (!ok) break;
            copy_q_row(Qs, row, tl + COL_QP);
            tc::fence_before_sync();
            mbar_arrive(&B->q_conv);
            mbar_arrive(&B->q_empty);
          }
        }
      }
      if (!ok) break;
      // epilogue: O of this tile is complete after its last PV product
      ok = __all_sync(0xffffffffu, wait_or_abort(&B->pv_done[(n - 1) & 1], (uint32_t)(((n - 1) >> 1) & 1), abort,
                                                 L.status, W_PV_EPILOGUE, n));
      if (!ok) break;
      tc::fence_after_sync();
      if constexpr (SPLIT) {
        const uint32_t ob = tl + COL_OB;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          float ad[32];
          tc::tmem_ld32(ob + 32 * hf, ad);
          tc::tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) v[32 * hf + c] = o[32 * hf + c] + ad[c];
        }
      } else {
        tc::tmem_ld64(tl + COL_O, v);
        tc::tmem_wait_ld();
        tc::fence_before_sync();
        mbar_arrive(&B->o_empty);  // the next tile's first PV may overwrite O
      }
      // O / l, stored coalesced: each thread holds its own row, so the warp's 32 x 64 block goes
      // through a 32 x 16 shared-memory slot in four rounds of 16 columns: every lane writes its
      // row's 4 chunks of 16 bytes (chunk c at position (c + r / 2) % 4 of row r: the 8 lanes of a
      // quarter-warp on distinct bank groups), then each store instruction writes eight 64-byte
      // row segments.
      const float inv = 1.0f / l;
      const int64_t ldo = pp->ldo;
      float* orow0 = pp->o + pp->o_off + (int64_t)(T.q0 + 32 * q4) * ldo + (int64_t)T.h * kD;
      const int vrows = Lq - (T.q0 + 32 * q4);  // rows of this warp's 32 that exist
      float* stg = Os + q4 * (kOStage / 4);
#pragma unroll
      for (int hc = 0; hc < 4; ++hc) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int col = 16 * hc + 4 * c;
          *reinterpret_cast<float4*>(stg + lane * 16 + 4 * ((c + (lane >> 1)) & 3)) =
              make_float4(v[col] * inv, v[col + 1] * inv, v[col + 2] * inv, v[col + 3] * inv);
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = 8 * i + (lane >> 2);
          const int c = lane & 3;
          const float4 val = *reinterpret_cast<const float4*>(stg + r * 16 + 4 * ((c + (r >> 1)) & 3));
          if (r < vrows) *reinterpret_cast<float4*>(orow0 + (int64_t)r * ldo + 16 * hc + 4 * c) = val;
        }
        __syncwarp();
      }
      t = tnext;
    }
    if (!ok && lane == 0) report_error(L.status, DEV_TIMEOUT, 22, n);
  } else if (SPLIT) {
    // ---------------- converters (split kernel): warp 6 for K, warp 7 for V ----------------
    // Each landed tile x is its own hi part; lo = x - hi goes into the lo copy (same offsets, so
    // the same swizzled layout). V rows past Lk become zeros in both parts: they meet P == 0 but
    // may hold another sequence's data. Then the generic-proxy writes are made visible to the
    // tensor core and the MMA warp is released.
    const bool vconv = warp == 7;
    bool ok = true;
    int n = 0, k = 0;
    for (; ok; ++k) {
      int t = 0;
      ok = __all_sync(0xffffffffu, tile_at(tab, k, &t, abort, L.status));
      if (!ok || t >= L.total) break;
      const Tile T = tile_of(L, t);
      int Lk = T.p->Lk;
      asm volatile("" : "+r"(Lk));  // kept in a register (see the softmax warps)
      for (int j = 0; ok && j < T.nblk; ++j, ++n) {
        const int ns = vconv ? kNSV : kNS;
        const int s = n % ns;
        const uint32_t par = (uint32_t)((n / ns) & 1);
        ok = __all_sync(0xffffffffu, wait_or_abort(vconv ? &B->v_full[s] : &B->kv_full[s], par, abort, L.status,
                                                   W_CONV_KV, n));
        if (!ok) break;
        const int nk = min(kN, Lk - j * kN);
        float4* xb = reinterpret_cast<float4*>((vconv ? Vs : Ks) + s * kKVBytes);
        float4* xl = reinterpret_cast<float4*>((vconv ? VLs : KLs) + s * kKVBytes);
        // Batches of kBatch chunks per lane, every load of a batch ahead of its stores (the
        // stores write the same array, so the compiler would not move later loads above them).
        // (One batch of all 32 chunks was slower overall.) The tensor core reads a TF32 operand
        // from the high 19 bits of its 32-bit container and ignores the 13 low mantissa bits,
        // so the landed x already serves as hi; only lo = x - hi is written (and rows of V past
        // Lk are zeroed in both copies).
        constexpr int kPer = (int)(kKVBytes / 16) / kConv;  // 32 chunks per lane
#pragma unroll 1
        for (int b0 = 0; b0 < kPer; b0 += kBatch) {
          float4 x[kBatch], lo[kBatch];
#pragma unroll
          for (int r = 0; r < kBatch; ++r) x[r] = xb[lane + kConv * (b0 + r)];
#pragma unroll
          for (int r = 0; r < kBatch; ++r) {
            const int i = lane + kConv * (b0 + r);
            // a 16-byte chunk of V: slab i / 512, key row (i % 512) / 8 (128-byte rows)
            if (!vconv || ((i & 511) >> 3) < nk) {
              split4(x[r], lo[r]);
            } else {
              x[r] = lo[r] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
          }
#pragma unroll
          for (int r = 0; r < kBatch; ++r) {
            if (vconv && ((lane + kConv * (b0 + r)) & 511) >> 3 >= nk) xb[lane + kConv * (b0 + r)] = x[r];
            xl[lane + kConv * (b0 + r)] = lo[r];
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(vconv ? &B->v_conv[s] : &B->kv_conv[s]);
      }
    }
    if (!ok && lane == 0) report_error(L.status, DEV_TIMEOUT, 23, n);
  }

  tc::fence_before_sync();
  __syncthreads();
  if (*abort && warp == 1) {
    // drain: every MMA this CTA issued must finish (bounded wait) before its TMEM is freed
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

}  // namespace

int attn_tf32_tile_rows() { return kM; }

template <bool SPLIT>
cudaError_t launch_tf32(const TmaLaunch& L, bool bias, cudaStream_t s) {
  using Y = Lay<SPLIT>;
  auto k = bias ? attn_tf32_kernel<true, SPLIT> : attn_tf32_kernel<false, SPLIT>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, Y::SMEM);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int slots = Y::CTAS_PER_SM * sms;  // persistent
  const int grid = L.total < slots ? L.total : slots;
  k<<<grid, Y::THREADS, Y::SMEM, s>>>(L);
  return cudaGetLastError();
}

cudaError_t launch_attn_tf32(const TmaLaunch& L, bool bias, bool split, cudaStream_t s) {
  if (L.total <= 0) return cudaSuccess;
  return split ? launch_tf32<true>(L, bias, s) : launch_tf32<false>(L, bias, s);
}

}  // namespace supra
