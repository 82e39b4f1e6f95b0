// supra_attn_attention_noalloc: attention that allocates no memory, for callers that cannot
// allocate device memory at the point where they need attention.
//
// Who needs it: a host whose device memory is handed out up front by its own allocator
// (an engine that reserves the GPU's memory at start-up and sub-allocates from that pool,
// leaving nothing for cudaMalloc), and code on a latency-critical path that must not call
// cudaMalloc/cudaFree because those calls can synchronise the whole device. Such callers
// still pass their own input and output buffers, but the score scratch this path needs
// cannot come from them.
//
// What it runs: the score-materialising path of attn_gemm_fp32.cu (QK^T GEMM -> row softmax
// -> PV GEMM) for ONE problem per call, for any head dim, with two kinds of memory that live
// in this file instead of being allocated:
//   - g_scratch: a file-scope static __device__ array of kScratchBytes (16 MiB) holding the
//     scores of one chunk of (head, row-range) units; a problem larger than that is processed
//     chunk by chunk, so the only limit is that one score row (round_up(Lk, 4) floats) must fit;
//   - g_desc: the problem descriptor, its units and tile prefix arrays (about 123 KB).
// Every GPU on which this library's kernels are loaded holds both arrays until the process exits.
// In host code the arrays' names are host-side stand-ins, not device addresses, so their
// device addresses are looked up once per device with cudaGetSymbolAddress (see dev_state)
// and passed to the kernels.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <mutex>

#include "kernels.h"
#include "supra_attn.h"

namespace {

constexpr size_t kScratchBytes = size_t(16) << 20;
constexpr size_t kScratchFloats = kScratchBytes / 4;
constexpr int kMaxUnits = 2048;
constexpr int kMaxDevices = 64;

struct alignas(256) NoAllocDesc {
  supra::AttnProb prob;
  supra::GemmUnit units[kMaxUnits];
  int32_t qk[kMaxUnits + 1];
  int32_t pv[kMaxUnits + 1];
  int32_t rows[kMaxUnits + 1];
  int32_t status[4];
};

static __device__ __align__(256) float g_scratch[kScratchFloats];
static __device__ __align__(256) NoAllocDesc g_desc;

struct DevState {
  bool ready = false;
  float* scratch = nullptr;
  NoAllocDesc* desc = nullptr;
};
DevState g_state[kMaxDevices];
std::mutex g_mu;

// Looks up the device addresses of the static arrays for the current device, once.
int dev_state(DevState** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SUPRA_ATTN_ECUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  DevState& s = g_state[dev];
  if (!s.ready) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || !p) {
      cudaGetLastError();
      return SUPRA_ATTN_ECUDA;
    }
    s.scratch = static_cast<float*>(p);
    p = nullptr;
    if (cudaGetSymbolAddress(&p, g_desc) != cudaSuccess || !p) {
      cudaGetLastError();
      return SUPRA_ATTN_ECUDA;
    }
    s.desc = static_cast<NoAllocDesc*>(p);
    s.ready = true;
  }
  *out = &s;
  return SUPRA_ATTN_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Copies the used part of the host staging descriptor to the device and runs the three
// kernels over `nu` units. Stream-ordered: the copy runs after earlier work on the stream.
int run_chunk(DevState* s, NoAllocDesc& h, int nu, bool bias, bool aligned, cudaStream_t st) {
  int64_t tq = 0, tp = 0, tr = 0;
  const supra::AttnProb& P = h.prob;
  for (int i = 0; i < nu; ++i) {
    supra::GemmUnit& u = h.units[i];
    u.qk_begin = (int32_t)tq;
    u.pv_begin = (int32_t)tp;
    u.row_begin = (int32_t)tr;
    h.qk[i] = u.qk_begin;
    h.pv[i] = u.pv_begin;
    h.rows[i] = u.row_begin;
    const int rt = (u.rows + 127) / 128;
    tq += (int64_t)rt * ((P.Lk + 127) / 128);
    tp += (int64_t)rt * ((P.D + 127) / 128);
    tr += u.rows;
  }
  if (tq > INT32_MAX || tp > INT32_MAX || tr > INT32_MAX) return SUPRA_ATTN_EINVAL;
  h.qk[nu] = (int32_t)tq;
  h.pv[nu] = (int32_t)tp;
  h.rows[nu] = (int32_t)tr;
  std::memset(h.status, 0, sizeof h.status);
  // the whole struct up to the used prefix entries is copied (pageable source: the copy is
  // staged before cudaMemcpyAsync returns, so the host staging may be reused right after)
  if (cudaMemcpyAsync(s->desc, &h, sizeof(NoAllocDesc), cudaMemcpyHostToDevice, st) != cudaSuccess) {
    cudaGetLastError();
    return SUPRA_ATTN_ECUDA;
  }
  supra::GemmLaunch L;
  L.probs = &s->desc->prob;
  L.units = s->desc->units;
  L.qk_begin = s->desc->qk;
  L.pv_begin = s->desc->pv;
  L.row_begin = s->desc->rows;
  L.scratch = s->scratch;
  L.n_units = nu;
  L.qk_total = (int32_t)tq;
  L.pv_total = (int32_t)tp;
  L.row_total = (int32_t)tr;
  L.status = s->desc->status;
  if (supra::launch_gemm_qk(bias, aligned, L, st) != cudaSuccess) return SUPRA_ATTN_ECUDA;
  if (supra::launch_softmax_rows(L, st) != cudaSuccess) return SUPRA_ATTN_ECUDA;
  if (supra::launch_gemm_pv(aligned, L, st) != cudaSuccess) return SUPRA_ATTN_ECUDA;
  return SUPRA_ATTN_OK;
}

}  // namespace

extern "C" int supra_attn_attention_noalloc(const supra_attn_desc* d, void* stream, char* msg, int32_t cap) {
  auto fail = [&](int code, const char* text) {
    if (msg && cap > 0) std::snprintf(msg, (size_t)cap, "%s", text);
    return code;
  };
  int rc = supra_attn_check_desc(d, msg, cap);  // same checks as supra_attn_enqueue
  if (rc) return rc;
  if (d->flags & SUPRA_ATTN_F_T5_TABLE)
    return fail(SUPRA_ATTN_EINVAL, "the no-alloc entry point takes an expanded [H, Lq, Lk] bias, not a T5 table");
  if (msg && cap > 0) msg[0] = 0;
  if (d->Lq == 0) return SUPRA_ATTN_OK;
  const int ldS = (d->Lk + 3) & ~3;
  if ((size_t)ldS > kScratchFloats)
    return fail(SUPRA_ATTN_EINVAL, "Lk too large for the 16 MiB no-alloc scratch: one score row must fit "
                                   "(Lk <= 4194304)");
  DevState* s = nullptr;
  rc = dev_state(&s);
  if (rc) return fail(rc, "cudaGetSymbolAddress failed for the no-alloc scratch");
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  static thread_local NoAllocDesc h;  // host staging (static storage, not allocated per call)
  std::memset(&h.prob, 0, sizeof h.prob);
  supra::AttnProb& P = h.prob;
  P.q = d->q;
  P.k = d->k;
  P.v = d->v;
  P.o = d->out;
  P.bias = d->bias;
  P.q_off = d->q_off;
  P.k_off = d->k_off;
  P.v_off = d->v_off;
  P.o_off = d->o_off;
  P.ldq = d->ldq;
  P.ldk = d->ldk;
  P.ldv = d->ldv;
  P.ldo = (int64_t)d->H * d->D;
  P.Lq = d->Lq;
  P.Lk = d->Lk;
  P.H = d->H;
  P.D = d->D;
  P.scale = (d->flags & SUPRA_ATTN_F_DEFAULT_SCALE) ? (float)(1.0 / std::sqrt((double)d->D)) : d->scale;
  P.scale_log2 = P.scale * 1.4426950408889634f;
  const bool bias = d->bias != nullptr;
  const bool aligned = (d->D % 4 == 0) && (d->ldq % 4 == 0) && (d->ldk % 4 == 0) && (d->ldv % 4 == 0) &&
                       aligned16(d->q + d->q_off) && aligned16(d->k + d->k_off) && aligned16(d->v + d->v_off) &&
                       aligned16(d->out + d->o_off);

  // units of (head, row range) whose scores fit the scratch; chunks of units fill it
  int64_t rows_max = (int64_t)(kScratchFloats / (size_t)ldS);
  if (rows_max >= 128) rows_max = rows_max / 128 * 128;
  if (rows_max > d->Lq) rows_max = d->Lq;
  int nu = 0;
  size_t used = 0;  // floats
  for (int hh = 0; hh < d->H; ++hh) {
    for (int r0 = 0; r0 < d->Lq; r0 += (int)rows_max) {
      const int rows = (int)std::min<int64_t>(rows_max, d->Lq - r0);
      const size_t uf = ((size_t)rows * ldS + 3) & ~size_t(3);
      if (nu == kMaxUnits || used + uf > kScratchFloats) {
        rc = run_chunk(s, h, nu, bias, aligned, st);
        if (rc) return fail(rc, "launch failed");
        nu = 0;
        used = 0;
      }
      supra::GemmUnit& u = h.units[nu++];
      std::memset(&u, 0, sizeof u);
      u.s_off = (int64_t)used;
      u.prob = 0;
      u.h = hh;
      u.row0 = r0;
      u.rows = rows;
      u.ldS = ldS;
      used += uf;
    }
  }
  rc = run_chunk(s, h, nu, bias, aligned, st);
  return rc ? fail(rc, "launch failed") : SUPRA_ATTN_OK;
}
