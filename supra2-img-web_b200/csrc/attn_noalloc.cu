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
// -> PV GEMM) for ONE problem per call, for any head dim, always in FP32 (a TF32 / TF32X3
// request gets the FP32 result, which is inside their tolerances), with two kinds of memory
// that live in this file instead of being allocated:
//   - g_scratch: a file-scope static __device__ array of kScratchBytes (16 MiB) holding the
//     scores of one chunk of (head, row-range) units; a problem larger than that is processed
//     chunk by chunk, so the only limit is that one score row (round_up(Lk, 4) floats) must fit;
//   - g_units: the problem descriptor and one chunk's units and tile prefix arrays (about
//     57 KB). It is written on the device by noalloc_units_kernel from values passed as kernel
//     arguments, so no host buffer is read after the call returns and nothing is copied from
//     the host: the units of a chunk follow from (H, Lq, rows per unit, first unit) in closed
//     form.
// Every GPU on which this library's kernels are loaded holds both arrays until the process exits.
// In host code the arrays' names are host-side stand-ins, not device addresses, so their
// device addresses are looked up once per device with cudaGetSymbolAddress (see dev_state)
// and passed to the kernels.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "kernels.h"
#include "supra_attn.h"

namespace {

constexpr size_t kScratchBytes = size_t(16) << 20;
constexpr size_t kScratchFloats = kScratchBytes / 4;
constexpr int kMaxUnits = 1024;
constexpr int kMaxDevices = 64;

struct alignas(256) NoAllocUnits {
  supra::AttnProb prob;
  supra::GemmUnit units[kMaxUnits];
  int32_t qk[kMaxUnits + 1];
  int32_t pv[kMaxUnits + 1];
  int32_t rows[kMaxUnits + 1];
};

static __device__ __align__(256) float g_scratch[kScratchFloats];
static __device__ __align__(256) NoAllocUnits g_units;

// The regular grid of (head, row range) units of one problem: unit g covers head g / per_head,
// rows [j * rows_max, min(Lq, (j + 1) * rows_max)) with j = g % per_head. Only the last unit of a
// head can be shorter. pre_* give the sums over units 0 .. g-1, so a chunk's prefixes are
// differences of them; the host uses the same functions to size each chunk's launch grid.
struct UnitGrid {
  int64_t Lq, rows_max, per_head, ldS, ctiles, dtiles;

  __host__ __device__ int64_t rows_of(int64_t j) const {
    return j + 1 < per_head ? rows_max : Lq - (per_head - 1) * rows_max;
  }
  // sum over units before g of f(rows), f(rows) = a * rows + b * ceil(rows / 128) + c * floats(rows)
  __host__ __device__ int64_t pre(int64_t g, int64_t a, int64_t b, int64_t c) const {
    auto f = [&](int64_t r) { return a * r + b * ((r + 127) / 128) + c * r * ldS; };
    const int64_t head = g / per_head, j = g - head * per_head;
    const int64_t per_head_sum = (per_head - 1) * f(rows_max) + f(rows_of(per_head - 1));
    return head * per_head_sum + j * f(rows_max);
  }
  __host__ __device__ int64_t pre_qk(int64_t g) const { return pre(g, 0, ctiles, 0); }
  __host__ __device__ int64_t pre_pv(int64_t g) const { return pre(g, 0, dtiles, 0); }
  __host__ __device__ int64_t pre_rows(int64_t g) const { return pre(g, 1, 0, 0); }
  // scores: rows * ldS floats per unit (ldS is a multiple of 4, so every unit starts 16-byte aligned)
  __host__ __device__ int64_t pre_floats(int64_t g) const { return pre(g, 0, 0, 1); }
};

// Writes the descriptor, the units g0 .. g0+nu-1 and their prefix arrays (relative to unit g0)
// into g_units. One thread per unit plus one for the closing prefix entries.
__global__ void noalloc_units_kernel(const supra::AttnProb prob, const UnitGrid grid, const int64_t g0, const int nu) {
  NoAllocUnits& d = g_units;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i == 0) d.prob = prob;
  if (i > nu) return;
  const int64_t g = g0 + i;
  const int32_t qk = (int32_t)(grid.pre_qk(g) - grid.pre_qk(g0));
  const int32_t pv = (int32_t)(grid.pre_pv(g) - grid.pre_pv(g0));
  const int32_t rows = (int32_t)(grid.pre_rows(g) - grid.pre_rows(g0));
  d.qk[i] = qk;
  d.pv[i] = pv;
  d.rows[i] = rows;
  if (i == nu) return;
  const int64_t head = g / grid.per_head, j = g - head * grid.per_head;
  supra::GemmUnit u;
  u.s_off = grid.pre_floats(g) - grid.pre_floats(g0);
  u.prob = 0;
  u.h = (int32_t)head;
  u.row0 = (int32_t)(j * grid.rows_max);
  u.rows = (int32_t)grid.rows_of(j);
  u.ldS = (int32_t)grid.ldS;
  u.qk_begin = qk;
  u.pv_begin = pv;
  u.row_begin = rows;
  d.units[i] = u;
}

struct DevState {
  bool ready = false;
  float* scratch = nullptr;
  NoAllocUnits* units = nullptr;
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
    if (cudaGetSymbolAddress(&p, g_units) != cudaSuccess || !p) {
      cudaGetLastError();
      return SUPRA_ATTN_ECUDA;
    }
    s.units = static_cast<NoAllocUnits*>(p);
    s.ready = true;
  }
  *out = &s;
  return SUPRA_ATTN_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Builds units g0 .. g0+nu-1 on the device and runs the three kernels over them, all on st.
int run_chunk(const DevState* s, const supra::AttnProb& prob, const UnitGrid& grid, int64_t g0, int nu, bool bias,
              bool aligned, cudaStream_t st) {
  const int64_t tq = grid.pre_qk(g0 + nu) - grid.pre_qk(g0);
  const int64_t tp = grid.pre_pv(g0 + nu) - grid.pre_pv(g0);
  const int64_t tr = grid.pre_rows(g0 + nu) - grid.pre_rows(g0);
  if (tq > INT32_MAX || tp > INT32_MAX || tr > INT32_MAX) return SUPRA_ATTN_EINVAL;
  noalloc_units_kernel<<<(nu + 1 + 255) / 256, 256, 0, st>>>(prob, grid, g0, nu);
  if (cudaGetLastError() != cudaSuccess) return SUPRA_ATTN_ECUDA;
  supra::GemmLaunch L;
  L.probs = &s->units->prob;
  L.units = s->units->units;
  L.qk_begin = s->units->qk;
  L.pv_begin = s->units->pv;
  L.row_begin = s->units->rows;
  L.scratch = s->scratch;
  L.n_units = nu;
  L.qk_total = (int32_t)tq;
  L.pv_total = (int32_t)tp;
  L.row_total = (int32_t)tr;
  L.status = nullptr;  // the score kernels have no bounded waits and report nothing
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
  const int64_t ldS = (d->Lk + 3) & ~3;
  if ((size_t)ldS > kScratchFloats)
    return fail(SUPRA_ATTN_EINVAL, "Lk too large for the 16 MiB no-alloc scratch: one score row must fit "
                                   "(Lk <= 4194304)");
  DevState* s = nullptr;
  rc = dev_state(&s);
  if (rc) return fail(rc, "cudaGetSymbolAddress failed for the no-alloc scratch");
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  supra::AttnProb P;
  std::memset(&P, 0, sizeof P);
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

  // (head, row range) units whose scores fit the scratch; consecutive units fill it chunk by chunk
  UnitGrid grid;
  int64_t rows_max = (int64_t)(kScratchFloats / (size_t)ldS);
  if (rows_max >= 128) rows_max = rows_max / 128 * 128;
  grid.rows_max = std::min<int64_t>(rows_max, d->Lq);
  grid.Lq = d->Lq;
  grid.per_head = (d->Lq + grid.rows_max - 1) / grid.rows_max;
  grid.ldS = ldS;
  grid.ctiles = (d->Lk + 127) / 128;
  grid.dtiles = (d->D + 127) / 128;
  const int64_t n_units = (int64_t)d->H * grid.per_head;
  int64_t g0 = 0;
  while (g0 < n_units) {
    int64_t g1 = g0;
    while (g1 < n_units && g1 - g0 < kMaxUnits &&
           grid.pre_floats(g1 + 1) - grid.pre_floats(g0) <= (int64_t)kScratchFloats)
      ++g1;
    rc = run_chunk(s, P, grid, g0, (int)(g1 - g0), bias, aligned, st);
    if (rc) return fail(rc, "launch failed");
    g0 = g1;
  }
  return SUPRA_ATTN_OK;
}
