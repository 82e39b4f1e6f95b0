// TF32 tensor-core attention for sm_100a: tcgen05.mma with TMEM accumulators, TMA-staged tiles.
// Head dim 64, no bias (the DiT self/cross-attention call sites, app/models/dit.js:172,184).
//
// Same math as the reference's fused kernel (app/gpu/kernels.js:164-316: online softmax over key
// blocks, O / l at the end), with both contractions on the 5th-generation tensor cores:
//   S_j = Q K_j^T   tcgen05.mma kind::tf32, A = Q (smem, K-major), B = K_j (smem, K-major),
//                   D = S_j in TMEM (128 lanes = query rows x 64 columns = keys), fp32
//   P_j            softmax warps read S_j from TMEM (one row per thread), compute
//                   exp2(s*scale*log2e - m), round to TF32 and write P_j over S_j in TMEM
//   O += P_j V_j   tcgen05.mma kind::tf32, A = P_j from TMEM, B = V_j (smem, MN-major), D = O in TMEM
// One CTA = one (problem, head, 128-row query tile); 6 warps:
//   warp 0     TMA producer: Q once, then K/V blocks of 64 keys into a 2-stage ring
//   warp 1     TMEM allocation and the single-thread MMA issuer (S_{j+1} overlaps softmax of j)
//   warps 2-5  softmax and epilogue; warp w owns TMEM lanes 32*(w%4) .. +31 (query rows)
// S is double-buffered in TMEM (2 x 64 columns) next to O (64 columns): 256 columns per CTA,
// two CTAs per SM. The running maximum moves lazily (only when a block exceeds it by more than
// 8 in log2 units), so O is rarely rescaled; when it is, the softmax warps wait for the
// previous PV product and rescale O in TMEM.
// Q and K tiles are loaded with the 128-byte swizzle (K-major operands), V tiles with the
// 128-byte / 32-byte-atom swizzle (the MN-major TF32 operand layout); no multicast. Every wait is bounded; on a timeout the
// CTA records the failure, drains what it can, frees its TMEM and leaves.
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
constexpr uint32_t OFF_BAR = OFF_V + kNS * kKVBytes;
// barriers: q, kv_full[2], kv_empty[2], s_full[2], p_full[2], pv_done, then tmem slot + abort flag
constexpr uint32_t SMEM_BYTES = OFF_BAR + 16 * 8 + 1024;  // + alignment slack for the 1024-B base
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t COL_S0 = 0, COL_S1 = 64, COL_O = 128;
constexpr int kThreads = 192;

struct Bars {
  uint64_t q, kv_full[kNS], kv_empty[kNS], s_full[2], p_full[2], pv_done, drain;
  uint32_t tmem;
  int32_t abort;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait that also gives up as soon as another warp of the CTA has aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int32_t* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0u) {
      if (*abort) return false;
      if (global_ns() - t0 > kWaitLimitNs) {
        *abort = 1;
        return false;
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads, 2) attn_tf32_kernel(const __grid_constant__ Tf32Launch L) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);  // 1024-B aligned for the swizzle atoms
  uint8_t* Qs = base + OFF_Q;
  uint8_t* Ks = base + OFF_K;
  uint8_t* Vs = base + OFF_V;
  Bars* B = reinterpret_cast<Bars*>(base + OFF_BAR);
  volatile int32_t* abort = &B->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int t = blockIdx.x;
  if (t >= L.total) {
    if (threadIdx.x == 0) report_error(L.status, DEV_BAD_TILE, 20);
    return;
  }
  const int pidx = L.uniform > 0 ? t / L.uniform : find_problem(L.begin, L.n, t);
  const Tf32Prob* __restrict__ pp = L.probs + pidx;
  const int local = t - (L.uniform > 0 ? pidx * L.uniform : __ldg(L.begin + pidx));
  const int q_tiles = pp->q_tiles;
  const int h = local / q_tiles;
  const int q0 = (local - h * q_tiles) * kM;
  const int Lq = pp->Lq, Lk = pp->Lk;
  const int nblk = (Lk + kN - 1) / kN;

  if (threadIdx.x == 0) {
    mbar_init(&B->q, 1);
    for (int s = 0; s < kNS; ++s) {
      mbar_init(&B->kv_full[s], 1);
      mbar_init(&B->kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&B->s_full[b], 1);
      mbar_init(&B->p_full[b], 128);
    }
    mbar_init(&B->pv_done, 1);
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
      const CUtensorMap* mq = L.maps + pp->mq;
      const CUtensorMap* mk = L.maps + pp->mk;
      const CUtensorMap* mv = L.maps + pp->mv;
      const int hx = h * kD;
      mbar_arrive_expect_tx(&B->q, kQBytes);
      tc::tma_load_2d(Qs, mq, pp->qx + hx, pp->qy + q0, &B->q);
      tc::tma_load_2d(Qs + kQSlab, mq, pp->qx + hx + 32, pp->qy + q0, &B->q);
      for (int j = 0; j < nblk; ++j) {
        const int s = j % kNS;
        if (j >= kNS && !wait_or_abort(&B->kv_empty[s], (uint32_t)(((j / kNS) - 1) & 1), abort)) break;
        mbar_arrive_expect_tx(&B->kv_full[s], 2 * kKVBytes);
        uint8_t* kd = Ks + s * kKVBytes;
        uint8_t* vd = Vs + s * kKVBytes;
        tc::tma_load_2d(kd, mk, pp->kx + hx, pp->ky + j * kN, &B->kv_full[s]);
        tc::tma_load_2d(kd + kKVSlab, mk, pp->kx + hx + 32, pp->ky + j * kN, &B->kv_full[s]);
        tc::tma_load_2d(vd, mv, pp->vx + hx, pp->vy + j * kN, &B->kv_full[s]);
        tc::tma_load_2d(vd + kKVSlab, mv, pp->vx + hx + 32, pp->vy + j * kN, &B->kv_full[s]);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    const uint32_t idS = tc::idesc_tf32(kM, kN, false, false);
    const uint32_t idPV = tc::idesc_tf32(kM, kD, false, true);
    bool ok = __all_sync(0xffffffffu, wait_or_abort(&B->q, 0, abort));
    for (int j = 0; ok && j <= nblk; ++j) {
      if (j < nblk) {
        const int s = j % kNS;
        const int b = j & 1;
        ok = __all_sync(0xffffffffu, wait_or_abort(&B->kv_full[s], (uint32_t)((j / kNS) & 1), abort));
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
        }
        __syncwarp();
      }
      if (j > 0) {
        const int jp = j - 1;
        const int sp = jp % kNS;
        const int bp = jp & 1;
        ok = __all_sync(0xffffffffu, wait_or_abort(&B->p_full[bp], (uint32_t)((jp >> 1) & 1), abort));
        if (!ok) break;
        const int nkp = min(kN, Lk - jp * kN);
        uint8_t* vb = Vs + sp * kKVBytes;
        if (nkp < kN) {
          // V rows past Lk meet P == 0; make them zeros (they may hold another sequence's data).
          // Whole 128-byte rows, so the swizzle inside a row does not matter.
          for (int idx = lane; idx < (kN - nkp) * 16; idx += 32) {
            const int r = nkp + (idx >> 4);
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
                            (jp > 0 || kk > 0) ? 1u : 0u);
          tc::commit(&B->kv_empty[sp]);
          tc::commit(&B->pv_done);
        }
        __syncwarp();
      }
    }
    if (!ok && lane == 0) report_error(L.status, DEV_TIMEOUT, 21);
  } else {
    // ---------------- softmax + epilogue (warps 2..5) ----------------
    const int q4 = warp & 3;
    const int row = 32 * q4 + lane;
    const uint32_t tl = tmem + ((uint32_t)(32 * q4) << 16);
    const float sl2 = pp->scale_log2;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    float v[64];
    for (int j = 0; j < nblk; ++j) {
      const int b = j & 1;
      ok = wait_or_abort(&B->s_full[b], (uint32_t)((j >> 1) & 1), abort);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const uint32_t scol = b ? COL_S1 : COL_S0;
      tc::tmem_ld64(tl + scol, v);
      tc::tmem_wait_ld();
      const int nk = min(kN, Lk - j * kN);
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float x = (c < nk) ? v[c] * sl2 : -INFINITY;
        v[c] = x;
        mx = fmaxf(mx, x);
      }
      const bool move = mx > m + 8.f;
      if (j > 0 && __any_sync(0xffffffffu, move)) {
        // O holds PV_0 .. PV_{j-1}: wait for the last one, then rescale the moved rows
        ok = wait_or_abort(&B->pv_done, (uint32_t)((j - 1) & 1), abort);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
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
    if (ok) {
      ok = wait_or_abort(&B->pv_done, (uint32_t)((nblk - 1) & 1), abort);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc::fence_after_sync();
      tc::tmem_ld64(tl + COL_O, v);
      tc::tmem_wait_ld();
      const float inv = 1.0f / l;
      if (q0 + row < Lq) {
        float* dst = pp->o + pp->o_off + (int64_t)(q0 + row) * pp->ldo + (int64_t)h * kD;
#pragma unroll
        for (int c = 0; c < 64; c += 4)
          *reinterpret_cast<float4*>(dst + c) = make_float4(v[c] * inv, v[c + 1] * inv, v[c + 2] * inv, v[c + 3] * inv);
      }
    } else if (lane == 0) {
      report_error(L.status, DEV_TIMEOUT, 22);
    }
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

cudaError_t launch_attn_tf32(const Tf32Launch& L, cudaStream_t s) {
  if (L.total <= 0) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(attn_tf32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return e;
  attn_tf32_kernel<<<L.total, kThreads, SMEM_BYTES, s>>>(L);
  return cudaGetLastError();
}

}  // namespace supra
