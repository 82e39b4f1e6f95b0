// TF32 tensor-core attention for sm_100a: tcgen05.mma with TMEM accumulators, TMA-staged tiles.
// Head dim 64 (the DiT self/cross-attention call sites, app/models/dit.js:172,184, and the T5
// encoder attention, app/models/t5.js:80, whose [H, Lq, Lk] relative-position bias the softmax
// warps add to the scores read from TMEM).
//
// Same math as the reference's fused kernel (app/gpu/kernels.js:164-316: online softmax over key
// blocks, O / l at the end), with both contractions on the 5th-generation tensor cores:
//   S_n = Q K_n^T   tcgen05.mma kind::tf32, A = Q (smem, K-major), B = K_n (smem, K-major),
//                   D = S_n in TMEM (128 lanes = query rows x 64 columns = keys), fp32
//   P_n            softmax warps read S_n from TMEM (one row per thread), compute
//                   exp2(s*scale*log2e - m), round to TF32 and write P_n over S_n in TMEM
//   O += P_n V_n   tcgen05.mma kind::tf32, A = P_n from TMEM, B = V_n (smem, MN-major), D = O in TMEM
// Persistent CTAs: CTA b takes tiles b, b + grid, b + 2*grid, ... of the launch's list of
// (problem, head, 128-row query tile); the key blocks of all its tiles form one stream n = 0, 1, ...
// that flows through a 2-stage K/V ring and a double-buffered S/P in TMEM without draining at
// tile boundaries. 6 warps:
//   warp 0     TMA producer: per tile the Q tile (once the previous tile's last S product has
//              read the old one), then K/V blocks of 64 keys into the ring
//   warp 1     TMEM allocation and the single-thread MMA issuer; S_n is issued before PV_{n-1}
//              so the tensor core computes S_n while the softmax warps work on P_{n-1}
//   warps 2-5  softmax and epilogue; warp w owns TMEM lanes 32*(w%4) .. +31 (query rows)
// TMEM: S/P double buffer (2 x 64 columns) and O (64 columns): 256 columns, two CTAs per SM.
// The running maximum moves lazily (only when a block exceeds it by more than 8 in log2 units),
// so O is rarely rescaled; when it is, the softmax warps wait for the previous PV product and
// rescale O in TMEM. The first PV of a tile overwrites O once the previous tile's epilogue has
// read it.
// Q and K tiles are loaded with the 128-byte swizzle (K-major operands), V tiles with the
// 128-byte / 32-byte-atom swizzle (the MN-major TF32 operand layout); every CTA loads only its own tiles.
// Every wait is bounded; on a timeout the CTA records the failure, drains the MMAs it issued,
// frees its TMEM and leaves.
#include "tcgen05.cuh"

namespace supra {
namespace {

constexpr int kM = 128;  // query rows per tile (MMA M)
constexpr int kN = 64;   // keys per block (MMA N of S)
constexpr int kD = 64;   // head dim (MMA N of O)
constexpr int kNS = 2;   // K/V stages
constexpr uint32_t kQSlab = kM * 128;   // one 32-column slab of the Q tile: 16 KB
constexpr uint32_t kKVSlab = kN * 128;  // one 32-column slab of a K or V block: 8 KB
constexpr uint32_t kQBytes = 2 * kQSlab;
constexpr uint32_t kKVBytes = 2 * kKVSlab;  // one K (or V) block
constexpr uint32_t OFF_Q = 0;
constexpr uint32_t OFF_K = OFF_Q + kQBytes;
constexpr uint32_t OFF_V = OFF_K + kNS * kKVBytes;
constexpr uint32_t OFF_O = OFF_V + kNS * kKVBytes;  // epilogue staging: 2 KB per softmax warp
constexpr uint32_t kOStage = 16 * 32 * 4;            // 16 rows x 32 columns of O
constexpr uint32_t OFF_BAR = OFF_O + 4 * kOStage;
constexpr uint32_t SMEM_BYTES = OFF_BAR + 256 + 1024;  // barriers + alignment slack for the 1024-B base
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t COL_S0 = 0, COL_S1 = 64, COL_O = 128;
constexpr int kThreads = 192;

// pv_done is double-buffered by block parity so that a waiter for PV_n never sees a barrier
// that is two phases ahead or behind (PV_{n-2} is always complete when PV_n is awaited).
struct Bars {
  uint64_t q_full, q_empty, kv_full[kNS], kv_empty[kNS], s_full[2], p_full[2], pv_done[2], o_empty, drain;
  uint32_t tmem;
  int32_t abort;
};
static_assert(sizeof(Bars) <= 256, "barrier block");

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Wait ids reported with a timeout (status[2]); status[3] carries the waiter's block counter.
enum WaitId : int32_t {
  W_Q_EMPTY = 31, W_KV_EMPTY = 32, W_Q_FULL = 33, W_KV_FULL = 34, W_P_FULL = 35, W_O_EMPTY = 36,
  W_S_FULL = 37, W_PV_RESCALE = 38, W_PV_EPILOGUE = 39,
};

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

template <bool BIAS>
__global__ void __launch_bounds__(kThreads, 2) attn_tf32_kernel(const __grid_constant__ TmaLaunch L) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);  // 1024-B aligned for the swizzle atoms
  uint8_t* Qs = base + OFF_Q;
  uint8_t* Ks = base + OFF_K;
  uint8_t* Vs = base + OFF_V;
  float* Os = reinterpret_cast<float*>(base + OFF_O);
  Bars* B = reinterpret_cast<Bars*>(base + OFF_BAR);
  volatile int32_t* abort = &B->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&B->q_full, 1);
    mbar_init(&B->q_empty, 1);
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
      int n = 0, k = 0;
      for (int t = blockIdx.x; t < L.total; t += gridDim.x, ++k) {
        const Tile T = tile_of(L, t);
        const TmaProb* pp = T.p;
        const CUtensorMap* mq = L.maps + pp->mq;
        const CUtensorMap* mk = L.maps + pp->mk;
        const CUtensorMap* mv = L.maps + pp->mv;
        const int hx = T.h * kD;
        if (k > 0 && !wait_or_abort(&B->q_empty, (uint32_t)((k - 1) & 1), abort, L.status, W_Q_EMPTY, n)) break;
        mbar_arrive_expect_tx(&B->q_full, kQBytes);
        tc::tma_load_2d(Qs, mq, pp->qx + hx, pp->qy + T.q0, &B->q_full);
        tc::tma_load_2d(Qs + kQSlab, mq, pp->qx + hx + 32, pp->qy + T.q0, &B->q_full);
        bool ok = true;
        for (int j = 0; j < T.nblk; ++j, ++n) {
          const int s = n % kNS;
          if (n >= kNS && !(ok = wait_or_abort(&B->kv_empty[s], (uint32_t)(((n / kNS) - 1) & 1), abort, L.status, W_KV_EMPTY, n))) break;
          mbar_arrive_expect_tx(&B->kv_full[s], 2 * kKVBytes);
          uint8_t* kd = Ks + s * kKVBytes;
          uint8_t* vd = Vs + s * kKVBytes;
          tc::tma_load_2d(kd, mk, pp->kx + hx, pp->ky + j * kN, &B->kv_full[s]);
          tc::tma_load_2d(kd + kKVSlab, mk, pp->kx + hx + 32, pp->ky + j * kN, &B->kv_full[s]);
          tc::tma_load_2d(vd, mv, pp->vx + hx, pp->vy + j * kN, &B->kv_full[s]);
          tc::tma_load_2d(vd + kKVSlab, mv, pp->vx + hx + 32, pp->vy + j * kN, &B->kv_full[s]);
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
      const int sp = m % kNS;
      const int bp = m & 1;
      if (!__all_sync(0xffffffffu, wait_or_abort(&B->p_full[bp], (uint32_t)((m >> 1) & 1), abort, L.status, W_P_FULL, m))) return false;
      if (pend_first && pend_k > 0 &&
          !__all_sync(0xffffffffu, wait_or_abort(&B->o_empty, (uint32_t)((pend_k - 1) & 1), abort, L.status, W_O_EMPTY, m)))
        return false;
      uint8_t* vb = Vs + sp * kKVBytes;
      if (pend_nk < kN) {
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
#pragma unroll
        for (int kk = 0; kk < kN / 8; ++kk)
          // V is MN-major: 32-column atoms kKVSlab apart (LBO), 4-key groups 512 B apart (SBO)
          tc::mma_tf32_ts(tmem + COL_O, tmem + pcol + 8 * kk,
                          tc::smem_desc(vb + kk * 1024, kKVSlab, 512, tc::kLayoutSW128Base32B), idPV,
                          (!pend_first || kk > 0) ? 1u : 0u);
        tc::commit(&B->kv_empty[sp]);
        tc::commit(&B->pv_done[m & 1]);
      }
      __syncwarp();
      pend_n = -1;
      return true;
    };
    for (int t = blockIdx.x; ok && t < L.total; t += gridDim.x, ++k) {
      const Tile T = tile_of(L, t);
      const int Lk = T.p->Lk;
      ok = __all_sync(0xffffffffu, wait_or_abort(&B->q_full, (uint32_t)(k & 1), abort, L.status, W_Q_FULL, n));
      for (int j = 0; ok && j < T.nblk; ++j, ++n) {
        const int s = n % kNS;
        const int b = n & 1;
        ok = __all_sync(0xffffffffu, wait_or_abort(&B->kv_full[s], (uint32_t)((n / kNS) & 1), abort, L.status, W_KV_FULL, n));
        if (!ok) break;
        tc::fence_after_sync();
        if (lane == 0) {
          const uint8_t* kb = Ks + s * kKVBytes;
#pragma unroll
          for (int k8 = 0; k8 < kD / 8; ++k8) {
            const uint32_t off = (uint32_t)(k8 >> 2) * kQSlab + (uint32_t)(k8 & 3) * 32u;
            const uint32_t offk = (uint32_t)(k8 >> 2) * kKVSlab + (uint32_t)(k8 & 3) * 32u;
            tc::mma_tf32_ss(tmem + (b ? COL_S1 : COL_S0), tc::smem_desc(Qs + off, 16, 1024, tc::kLayoutSW128),
                            tc::smem_desc(kb + offk, 16, 1024, tc::kLayoutSW128), idS, k8 > 0 ? 1u : 0u);
          }
          tc::commit(&B->s_full[b]);
          if (j == T.nblk - 1) tc::commit(&B->q_empty);  // the Q tile is no longer read
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
  } else {
    // ---------------- softmax + epilogue (warps 2..5) ----------------
    const int q4 = warp & 3;
    const int row = 32 * q4 + lane;
    const uint32_t tl = tmem + ((uint32_t)(32 * q4) << 16);
    bool ok = true;
    int n = 0;
    float v[64];
    for (int t = blockIdx.x; ok && t < L.total; t += gridDim.x) {
      const Tile T = tile_of(L, t);
      const TmaProb* pp = T.p;
      const int Lk = pp->Lk, Lq = pp->Lq;
      const float sl2 = pp->scale_log2;
      float m = -INFINITY, l = 0.f;
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
            const float x = (c < nk) ? fmaf(b, 1.4426950408889634f, v[c] * sl2) : -INFINITY;
            v[c] = x;
            mx = fmaxf(mx, x);
          }
        } else if (BIAS && T.q0 + row < Lq) {
          // this thread's query row of the bias, keys j*64 .. j*64 + nk (exp2 domain: times log2 e)
          const float* brow = pp->bias + ((int64_t)T.h * Lq + T.q0 + row) * Lk + (int64_t)j * kN;
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            const float x = (c < nk) ? fmaf(__ldg(brow + c), 1.4426950408889634f, v[c] * sl2) : -INFINITY;
            v[c] = x;
            mx = fmaxf(mx, x);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            const float x = (c < nk) ? v[c] * sl2 : -INFINITY;
            v[c] = x;
            mx = fmaxf(mx, x);
          }
        }
        const bool move = mx > m + 8.f;
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
        float ps = 0.f;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float p = tc::to_tf32(ex2(v[c] - m));
          ps += p;
          v[c] = p;
        }
        l += ps;
        tc::tmem_st64(tl + scol, v);
        tc::tmem_wait_st();
        tc::fence_before_sync();
        mbar_arrive(&B->p_full[b]);
      }
      if (!ok) break;
      // epilogue: O of this tile is complete after its last PV product
      ok = __all_sync(0xffffffffu, wait_or_abort(&B->pv_done[(n - 1) & 1], (uint32_t)(((n - 1) >> 1) & 1), abort,
                                                 L.status, W_PV_EPILOGUE, n));
      if (!ok) break;
      tc::fence_after_sync();
      tc::tmem_ld64(tl + COL_O, v);
      tc::tmem_wait_ld();
      tc::fence_before_sync();
      mbar_arrive(&B->o_empty);  // the next tile's first PV may overwrite O
      // O / l, stored coalesced: each thread holds its own row, so the warp's 32 x 64 block goes
      // through a 16 x 32 shared-memory slot (16-byte chunks swizzled by row) in four rounds and
      // every store instruction writes four whole 128-byte row segments.
      const float inv = 1.0f / l;
      const int64_t ldo = pp->ldo;
      float* orow0 = pp->o + pp->o_off + (int64_t)(T.q0 + 32 * q4) * ldo + (int64_t)T.h * kD;
      const int vrows = Lq - (T.q0 + 32 * q4);  // rows of this warp's 32 that exist
      float* stg = Os + q4 * (kOStage / 4);
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          if ((lane >> 4) == hr) {
            const int r = lane & 15;
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4) {
              const int c = 32 * hc + 4 * c4;
              *reinterpret_cast<float4*>(stg + r * 32 + ((c4 ^ (r & 7)) << 2)) =
                  make_float4(v[c] * inv, v[c + 1] * inv, v[c + 2] * inv, v[c + 3] * inv);
            }
          }
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = 4 * i + (lane >> 3);
            const int c4 = lane & 7;
            const float4 val = *reinterpret_cast<const float4*>(stg + r * 32 + ((c4 ^ (r & 7)) << 2));
            if (16 * hr + r < vrows)
              *reinterpret_cast<float4*>(orow0 + (int64_t)(16 * hr + r) * ldo + 32 * hc + 4 * c4) = val;
          }
          __syncwarp();
        }
      }
    }
    if (!ok && lane == 0) report_error(L.status, DEV_TIMEOUT, 22, n);
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

cudaError_t launch_attn_tf32(const TmaLaunch& L, bool bias, cudaStream_t s) {
  if (L.total <= 0) return cudaSuccess;
  auto k = bias ? attn_tf32_kernel<true> : attn_tf32_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = L.total < 2 * sms ? L.total : 2 * sms;  // persistent: two CTAs per SM
  k<<<grid, kThreads, SMEM_BYTES, s>>>(L);
  return cudaGetLastError();
}

}  // namespace supra
