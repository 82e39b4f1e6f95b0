// libsupra_attn host runtime: the C ABI declared in include/supra_attn.h.
//
// It replaces, for the attention operator, the reference's WebGPU runtime (app/gpu/device.js):
//   - GPU/Tensor/BufferPool  -> context, pooled device buffers with the same size bucketing
//                               (BufferPool.round, app/gpu/device.js:64-70)
//   - dispatch + flush       -> enqueue records validated problems; flush issues one grouped
//                               launch per kernel configuration (app/gpu/device.js:207-253)
//   - uniform ring           -> a pinned/device descriptor ring, two halves fenced by events
//                               (app/gpu/device.js:7-8,128-130,210-218)
//   - checkErrors / lost     -> a device status word read at sync/download
//                               (app/gpu/device.js:134,186,258,262-268)
//   - Profiler               -> CUDA events per grouped launch, aggregated by kernel name with
//                               FLOPs and bytes (app/gpu/device.js:272-325, app/gpu/ops.js:116)
// and the operator itself (app/gpu/ops.js:103-149): the same arguments, the same defaults,
// and synchronous errors for invalid calls.
#include "supra_attn.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "kernels.h"

using supra::AttnLaunch;
using supra::AttnProb;
using supra::GemmLaunch;
using supra::GemmUnit;

namespace {

constexpr float kLog2e = 1.4426950408889634f;

// Disjoint, merged [begin, end) byte ranges.
class IntervalSet {
 public:
  void clear() { m_.clear(); }
  bool empty() const { return m_.empty(); }
  bool overlaps(uintptr_t b, uintptr_t e) const {
    if (b >= e || m_.empty()) return false;
    auto it = m_.upper_bound(b);
    if (it != m_.end() && it->first < e) return true;
    if (it != m_.begin()) {
      --it;
      if (it->second > b) return true;
    }
    return false;
  }
  void add(uintptr_t b, uintptr_t e) {
    if (b >= e) return;
    auto it = m_.upper_bound(b);
    if (it != m_.begin()) {
      auto pv = std::prev(it);
      if (pv->second >= b) {
        b = pv->first;
        e = std::max(e, pv->second);
        it = m_.erase(pv);
      }
    }
    while (it != m_.end() && it->first <= e) {
      e = std::max(e, it->second);
      it = m_.erase(it);
    }
    m_.emplace(b, e);
  }

 private:
  std::map<uintptr_t, uintptr_t> m_;
};

struct ByteRange {
  uintptr_t b = 0, e = 0;
};

enum Path : int { PATH_FUSED = 0, PATH_GEMM = 1, PATH_TF32 = 2, PATH_FP32_TMA = 3, PATH_LINEAR = 4 };

struct Queued {
  AttnProb p;
  int path;
  int cfg;
  bool bias;
  bool aligned;
  double flops;
  double bytes;
  int64_t rows_q, rows_k, rows_v;  // whole rows of each operand buffer (TMA tensor maps)
  int32_t t5_buckets, t5_maxd;      // T5 table bias (SUPRA_ATTN_F_T5_TABLE), else 0
  supra::LinProb lin;               // PATH_LINEAR: the linear problem (p unused)
  float gn_eps;                     // PATH_LINEAR with GroupNorm of x
};

// A tensor map over a whole operand buffer: [rows, ld] fp32, boxes of box_cols columns x
// box_rows rows. tf32: the TMA unit may round to TF32 on the way in (tensor-core operands);
// otherwise the values arrive unchanged (FP32 kernel).
struct MapKey {
  uintptr_t base;
  int64_t ld, rows;
  int64_t cols;  // the inner extent: boxes reaching past it read zeros
  int32_t box_cols, box_rows;
  int32_t swz;  // CUtensorMapSwizzle
  int32_t tf32;
  bool operator==(const MapKey& o) const {
    return base == o.base && ld == o.ld && rows == o.rows && cols == o.cols && box_cols == o.box_cols &&
           box_rows == o.box_rows && swz == o.swz && tf32 == o.tf32;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<uintptr_t>()(k.base);
    h ^= std::hash<int64_t>()(k.ld) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    h ^= std::hash<int64_t>()(k.rows) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    h ^= std::hash<int64_t>()(k.cols) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    h ^= std::hash<int64_t>()(((int64_t)k.box_cols << 32) ^ (k.box_rows * 16 + k.swz * 2 + k.tf32)) +
         0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    return h;
  }
};

struct ProfStat {
  int64_t launches = 0;
  double ms = 0, flops = 0, bytes = 0;
};

struct PendingEvt {
  std::string name;
  double flops, bytes;
  cudaEvent_t a, b;
};

size_t pool_round(size_t bytes) {  // BufferPool.round (app/gpu/device.js:64-70)
  size_t b = std::max<size_t>(256, bytes);
  size_t p = 1;
  while (p * 2 <= b) p *= 2;
  const size_t step = std::max<size_t>(256, p / 8);
  return (b + step - 1) / step * step;
}

size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

}  // namespace

struct supra_attn_ctx {
  int device = 0;
  cudaStream_t own = nullptr;
  cudaStream_t stream = nullptr;
  int32_t* d_status = nullptr;
  int32_t* h_status = nullptr;

  // descriptor ring: two halves of pinned staging + device memory
  char* ring_h = nullptr;
  char* ring_hd = nullptr;  // ring_h as the device addresses it (pinned, mapped)
  char* ring_d = nullptr;
  size_t ring_half = 0;
  int ring_cur = 0;
  size_t ring_head = 0;
  cudaEvent_t ring_ev[2] = {nullptr, nullptr};
  bool ring_ev_used[2] = {false, false};

  std::vector<Queued> queue;
  IntervalSet qreads, qwrites;

  float2* gn_stats = nullptr;  // GroupNorm statistics of the linear problems of a flush
  size_t gn_cap = 0;             // in float2
  float* lin_split = nullptr;    // tensor-core linears: hi / lo copies of x and w of a flush
  size_t lin_split_cap = 0;      // in floats
  std::map<size_t, std::vector<void*>> pool_free;
  std::unordered_map<void*, size_t> pool_live;
  std::unordered_set<void*> host_live;

  float* scratch = nullptr;
  size_t scratch_cap = 0;
  size_t scratch_budget = size_t(64) << 20;  // per chunk of score-materialising units

  bool profile = false;
  std::vector<PendingEvt> pend;
  std::vector<cudaEvent_t> evt_free;
  std::map<std::string, ProfStat> stats;

  // encoded TMA tensor maps, reused across flushes (keyed by buffer, box and element handling)
  std::unordered_map<MapKey, CUtensorMap, MapKeyHash> map_cache;

  int64_t launches = 0;
  std::string err;
};

namespace {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link-time libcuda dependency).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    else
      cudaGetLastError();
  }
  return fn;
}

// [rows, ld] fp32 buffer, boxes of box_cols x box_rows with the key's swizzle, zero fill outside.
// The TF32 kernel uses 32-column (128-byte) boxes with SWIZZLE_128B for K-major operands and
// SWIZZLE_128B_ATOM_32B for the MN-major V operand, and lets the TMA unit round to TF32 when the
// driver accepts that type; the FP32 kernel uses unswizzled FLOAT32 boxes (exact copies).
bool encode_map(CUtensorMap* m, const MapKey& k) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)k.cols, (cuuint64_t)k.rows};
  const cuuint64_t strides[1] = {(cuuint64_t)k.ld * 4};
  const cuuint32_t box[2] = {(cuuint32_t)k.box_cols, (cuuint32_t)k.box_rows};
  const cuuint32_t estr[2] = {1, 1};
  for (CUtensorMapDataType t : {CU_TENSOR_MAP_DATA_TYPE_TFLOAT32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32}) {
    if (t == CU_TENSOR_MAP_DATA_TYPE_TFLOAT32 && !k.tf32) continue;
    if (fn(m, t, 2, reinterpret_cast<void*>(k.base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           static_cast<CUtensorMapSwizzle>(k.swz), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
      return true;
  }
  return false;
}

class DeviceGuard {
 public:
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev_) != cudaSuccess) prev_ = -1;
    if (prev_ != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev_ >= 0) {
      int cur = -1;
      if (cudaGetDevice(&cur) == cudaSuccess && cur != prev_) cudaSetDevice(prev_);
    }
  }

 private:
  int prev_ = -1;
};

int set_err(supra_attn_ctx* c, int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (c) c->err = buf;
  return code;
}

int cuda_err(supra_attn_ctx* c, cudaError_t e, const char* what) {
  return set_err(c, SUPRA_ATTN_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

// ---- descriptor ring ---------------------------------------------------------------------------
int ring_reserve(supra_attn_ctx* c, size_t bytes, char** host, char** dev) {
  bytes = align16(bytes);
  if (bytes > c->ring_half) {
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return cuda_err(c, e, "ring grow: stream sync");
    size_t half = std::max<size_t>(c->ring_half * 2, align16(bytes));
    char *nh = nullptr, *nd = nullptr;
    if (cudaMallocHost(&nh, 2 * half) != cudaSuccess) return set_err(c, SUPRA_ATTN_ENOMEM, "ring: pinned alloc");
    if (cudaMalloc(&nd, 2 * half) != cudaSuccess) {
      cudaFreeHost(nh);
      return set_err(c, SUPRA_ATTN_ENOMEM, "ring: device alloc");
    }
    void* nhd = nullptr;
    if (cudaHostGetDevicePointer(&nhd, nh, 0) != cudaSuccess) {
      cudaGetLastError();
      cudaFreeHost(nh);
      cudaFree(nd);
      return set_err(c, SUPRA_ATTN_ENOMEM, "ring: pinned buffer not addressable by the device");
    }
    cudaFreeHost(c->ring_h);
    cudaFree(c->ring_d);
    c->ring_h = nh;
    c->ring_hd = static_cast<char*>(nhd);
    c->ring_d = nd;
    c->ring_half = half;
    c->ring_cur = 0;
    c->ring_head = 0;
    c->ring_ev_used[0] = c->ring_ev_used[1] = false;
  }
  if (c->ring_head + bytes > c->ring_half) {
    c->ring_cur ^= 1;
    c->ring_head = 0;
    if (c->ring_ev_used[c->ring_cur]) {
      cudaError_t e = cudaEventSynchronize(c->ring_ev[c->ring_cur]);
      if (e != cudaSuccess) return cuda_err(c, e, "ring: event sync");
    }
  }
  const size_t off = c->ring_cur * c->ring_half + c->ring_head;
  *host = c->ring_h + off;
  *dev = c->ring_d + off;
  c->ring_head += bytes;
  return SUPRA_ATTN_OK;
}

// Copies bytes staged at host (inside the ring) to dev, stream-ordered, with the staging kernel
// (stage.cu) rather than the copy engine, so that large uploads on other streams cannot hold
// the descriptors back.
int ring_commit(supra_attn_ctx* c, char* host, char* dev, size_t bytes) {
  cudaError_t e = supra::launch_stage_copy(c->ring_hd + (host - c->ring_h), dev, align16(bytes), c->stream);
  if (e != cudaSuccess) return cuda_err(c, e, "ring: stage");
  c->launches += 1;
  e = cudaEventRecord(c->ring_ev[c->ring_cur], c->stream);
  if (e != cudaSuccess) return cuda_err(c, e, "ring: event record");
  c->ring_ev_used[c->ring_cur] = true;
  return SUPRA_ATTN_OK;
}

// ---- profiling -------------------------------------------------------------------------------
cudaEvent_t take_event(supra_attn_ctx* c) {
  if (!c->evt_free.empty()) {
    cudaEvent_t e = c->evt_free.back();
    c->evt_free.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

struct ProfScope {
  supra_attn_ctx* c;
  PendingEvt pe;
  bool on;
  ProfScope(supra_attn_ctx* ctx, const char* name, double flops, double bytes) : c(ctx), on(ctx->profile) {
    if (!on) return;
    pe.name = name;
    pe.flops = flops;
    pe.bytes = bytes;
    pe.a = take_event(c);
    pe.b = take_event(c);
    if (!pe.a || !pe.b) {
      on = false;
      return;
    }
    cudaEventRecord(pe.a, c->stream);
  }
  ~ProfScope() {
    if (!on) return;
    cudaEventRecord(pe.b, c->stream);
    c->pend.push_back(pe);
  }
};

int collect_profile(supra_attn_ctx* c) {
  for (auto& pe : c->pend) {
    float ms = 0.f;
    cudaError_t e = cudaEventSynchronize(pe.b);
    if (e != cudaSuccess) return cuda_err(c, e, "profile: event sync");
    cudaEventElapsedTime(&ms, pe.a, pe.b);
    ProfStat& s = c->stats[pe.name];
    s.launches += 1;
    s.ms += ms;
    s.flops += pe.flops;
    s.bytes += pe.bytes;
    c->evt_free.push_back(pe.a);
    c->evt_free.push_back(pe.b);
  }
  c->pend.clear();
  return SUPRA_ATTN_OK;
}

// ---- validation --------------------------------------------------------------------------------
struct Checked {
  Queued q;
  ByteRange reads[8];
  int nreads = 0;
  ByteRange write;
  bool empty = false;  // Lq == 0: nothing to do
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int validate(supra_attn_ctx* c, const supra_attn_desc* d, Checked* out) {
  if (!d) return set_err(c, SUPRA_ATTN_EINVAL, "descriptor is NULL");
  if (d->flags & ~(SUPRA_ATTN_F_DEFAULT_SCALE | SUPRA_ATTN_F_T5_TABLE))
    return set_err(c, SUPRA_ATTN_EINVAL, "unknown flag bits 0x%x", d->flags);
  if (d->variant != SUPRA_ATTN_FP32 && d->variant != SUPRA_ATTN_TF32 && d->variant != SUPRA_ATTN_TF32X3)
    return set_err(c, SUPRA_ATTN_EINVAL, "unknown variant %d", d->variant);
  if (d->Lq < 0 || d->Lq > (1 << 30)) return set_err(c, SUPRA_ATTN_EINVAL, "Lq=%d out of range [0, 2^30]", d->Lq);
  if (d->Lk < 1 || d->Lk > (1 << 30)) return set_err(c, SUPRA_ATTN_EINVAL, "Lk=%d out of range [1, 2^30]", d->Lk);
  if (d->H < 1 || d->H > 65536) return set_err(c, SUPRA_ATTN_EINVAL, "H=%d out of range [1, 65536]", d->H);
  if (d->D < 1 || d->D > 65536) return set_err(c, SUPRA_ATTN_EINVAL, "D=%d out of range [1, 65536]", d->D);
  if ((int64_t)d->H * d->D > (int64_t(1) << 24)) return set_err(c, SUPRA_ATTN_EINVAL, "H*D too large");
  const int64_t lim = int64_t(1) << 46;
  const int64_t lds[3] = {d->ldq, d->ldk, d->ldv};
  const int64_t offs[4] = {d->q_off, d->k_off, d->v_off, d->o_off};
  for (int i = 0; i < 3; ++i)
    if (lds[i] < 0 || lds[i] > lim) return set_err(c, SUPRA_ATTN_EINVAL, "leading dimension out of range");
  for (int i = 0; i < 4; ++i)
    if (offs[i] < 0 || offs[i] > lim) return set_err(c, SUPRA_ATTN_EINVAL, "offset out of range (negative?)");
  if (!d->q || !d->k || !d->v || !d->out) return set_err(c, SUPRA_ATTN_EINVAL, "q, k, v and out must be non-NULL");
  const void* ptrs[5] = {d->q, d->k, d->v, d->out, d->bias};
  for (int i = 0; i < 5; ++i)
    if (ptrs[i] && (reinterpret_cast<uintptr_t>(ptrs[i]) & 3u))
      return set_err(c, SUPRA_ATTN_EINVAL, "pointers must be 4-byte aligned float arrays");
  float scale = d->scale;
  if (d->flags & SUPRA_ATTN_F_DEFAULT_SCALE) scale = (float)(1.0 / std::sqrt((double)d->D));  // ops.js:109
  if (!std::isfinite(scale)) return set_err(c, SUPRA_ATTN_EINVAL, "scale must be finite");

  const int64_t HD = (int64_t)d->H * d->D;
  out->empty = (d->Lq == 0);
  // bounds: the last element each operand touches (app/gpu/ops.js:104-105)
  auto last = [&](int64_t off, int64_t rows, int64_t ld) { return off + (rows - 1) * ld + HD - 1; };
  if (!out->empty && last(d->q_off, d->Lq, d->ldq) >= d->q_size)
    return set_err(c, SUPRA_ATTN_EINVAL, "q out of bounds: needs %lld floats, q_size=%lld",
                   (long long)(last(d->q_off, d->Lq, d->ldq) + 1), (long long)d->q_size);
  if (last(d->k_off, d->Lk, d->ldk) >= d->k_size)
    return set_err(c, SUPRA_ATTN_EINVAL, "k out of bounds: needs %lld floats, k_size=%lld",
                   (long long)(last(d->k_off, d->Lk, d->ldk) + 1), (long long)d->k_size);
  if (last(d->v_off, d->Lk, d->ldv) >= d->v_size)
    return set_err(c, SUPRA_ATTN_EINVAL, "v out of bounds: needs %lld floats, v_size=%lld",
                   (long long)(last(d->v_off, d->Lk, d->ldv) + 1), (long long)d->v_size);
  if (d->o_off + (int64_t)d->Lq * HD > d->out_size)
    return set_err(c, SUPRA_ATTN_EINVAL, "out out of bounds: needs %lld floats, out_size=%lld",
                   (long long)(d->o_off + (int64_t)d->Lq * HD), (long long)d->out_size);
  const bool t5 = (d->flags & SUPRA_ATTN_F_T5_TABLE) != 0;
  const int32_t t5_buckets = t5 ? (int32_t)(d->bias_param & 0xffffu) : 0;
  const int32_t t5_maxd = t5 ? (int32_t)(d->bias_param >> 16) : 0;
  if (t5) {
    if (!d->bias) return set_err(c, SUPRA_ATTN_EINVAL, "SUPRA_ATTN_F_T5_TABLE: bias must point at the table");
    if (supra_attn_relative_bucket(0, t5_buckets, t5_maxd) < 0)
      return set_err(c, SUPRA_ATTN_EINVAL,
                     "T5 table: buckets (bias_param bits 0-15) must be even and >= 4 and max_distance "
                     "(bits 16-31) > buckets/4; got buckets=%d max_distance=%d", t5_buckets, t5_maxd);
  } else if (d->bias_param != 0) {
    return set_err(c, SUPRA_ATTN_EINVAL, "bias_param must be 0 without SUPRA_ATTN_F_T5_TABLE");
  }
  const int64_t nbias = t5 ? (int64_t)t5_buckets * d->H : (int64_t)d->H * d->Lq * d->Lk;
  if (d->bias && nbias > d->bias_size)
    return set_err(c, SUPRA_ATTN_EINVAL, t5 ? "T5 table must hold buckets*H=%lld floats, bias_size=%lld"
                                            : "bias must hold H*Lq*Lk=%lld floats, bias_size=%lld",
                   (long long)nbias, (long long)d->bias_size);

  // byte ranges for hazard tracking; the output may not alias an input of the same problem
  // (a writable binding may not alias a read-only one in one WebGPU dispatch)
  auto rng = [](const float* base, int64_t first, int64_t lastidx) {
    ByteRange r;
    r.b = reinterpret_cast<uintptr_t>(base + first);
    r.e = reinterpret_cast<uintptr_t>(base + lastidx + 1);
    return r;
  };
  out->nreads = 0;
  if (!out->empty) {
    out->reads[out->nreads++] = rng(d->q, d->q_off, last(d->q_off, d->Lq, d->ldq));
    out->reads[out->nreads++] = rng(d->k, d->k_off, last(d->k_off, d->Lk, d->ldk));
    out->reads[out->nreads++] = rng(d->v, d->v_off, last(d->v_off, d->Lk, d->ldv));
    if (d->bias) out->reads[out->nreads++] = rng(d->bias, 0, nbias - 1);
    out->write = rng(d->out, d->o_off, d->o_off + (int64_t)d->Lq * HD - 1);
    for (int i = 0; i < out->nreads; ++i)
      if (out->reads[i].b < out->write.e && out->write.b < out->reads[i].e)
        return set_err(c, SUPRA_ATTN_EINVAL, "out overlaps an input of the same call");
  }

  Queued& q = out->q;
  std::memset(&q.p, 0, sizeof(q.p));
  q.p.q = d->q;
  q.p.k = d->k;
  q.p.v = d->v;
  q.p.o = d->out;
  q.p.bias = d->bias;
  q.p.q_off = d->q_off;
  q.p.k_off = d->k_off;
  q.p.v_off = d->v_off;
  q.p.o_off = d->o_off;
  q.p.ldq = d->ldq;
  q.p.ldk = d->ldk;
  q.p.ldv = d->ldv;
  q.p.ldo = HD;
  q.p.Lq = d->Lq;
  q.p.Lk = d->Lk;
  q.p.H = d->H;
  q.p.D = d->D;
  q.p.scale = scale;
  q.p.scale_log2 = scale * kLog2e;
  q.bias = d->bias != nullptr;
  q.t5_buckets = t5_buckets;
  q.t5_maxd = t5_maxd;
  q.p.rel_max = t5_maxd;
  // 16-byte aligned rows for the bulk-copy engine (the reference's fused path needs the same
  // %4 alignment of every stride and offset, app/gpu/ops.js:111)
  q.aligned = (d->D % 4 == 0) && (d->ldq % 4 == 0) && (d->ldk % 4 == 0) && (d->ldv % 4 == 0) &&
              aligned16(d->q + d->q_off) && aligned16(d->k + d->k_off) && aligned16(d->v + d->v_off) &&
              aligned16(d->out + d->o_off);
  if (d->D <= 64) {
    q.path = PATH_FUSED;
    q.cfg = d->Lq <= 64 ? supra::CFG_D64_Q64 : supra::CFG_D64_Q128;
  } else if (d->D <= 128) {
    q.path = PATH_FUSED;
    q.cfg = supra::CFG_D128_Q64;
  } else {
    q.path = PATH_GEMM;
    // TF32 / TF32X3 requests without a bias and with at least 32 keys run the score path's two
    // products (Q K^T and P V) on the tensor-core linear (cfg 1 / 2); the row softmax between them
    // stays as it is
    const bool tc = d->variant != SUPRA_ATTN_FP32 && !q.bias && d->Lk >= 32;
    q.cfg = tc ? (d->variant == SUPRA_ATTN_TF32X3 ? 2 : 1) : 0;
  }
  q.rows_q = d->ldq > 0 ? d->q_size / d->ldq : 0;
  q.rows_k = d->ldk > 0 ? d->k_size / d->ldk : 0;
  q.rows_v = d->ldv > 0 ? d->v_size / d->ldv : 0;
  // The TMA kernels read whole boxes of full buffer rows through tensor maps: head dim 64,
  // 16-byte aligned rows, every row of the problem a whole row of its buffer, and the heads
  // inside one row.
  auto rows_ok = [](int64_t off, int64_t ld, int64_t rows, int64_t nrows, int64_t HDc) {
    return ld >= 32 && ld <= (int64_t(1) << 30) && (off % ld) + HDc <= ld && off / ld + nrows <= rows &&
           rows <= (int64_t(1) << 31) - 1;
  };
  const bool tma_ok = d->D == 64 && q.aligned && d->Lq > 0 && aligned16(d->q) && aligned16(d->k) &&
                      aligned16(d->v) && d->q_off % 4 == 0 && d->k_off % 4 == 0 && d->v_off % 4 == 0 &&
                      rows_ok(d->q_off, d->ldq, q.rows_q, d->Lq, HD) && rows_ok(d->k_off, d->ldk, q.rows_k, d->Lk, HD) &&
                      rows_ok(d->v_off, d->ldv, q.rows_v, d->Lk, HD);
  if (d->variant == SUPRA_ATTN_TF32 || d->variant == SUPRA_ATTN_TF32X3) {
    // Other tensor-core requests run the FP32 kernels, which are at least as accurate (a bias is
    // read directly by the tensor-core kernel). cfg 1: the split-precision form.
    if (tma_ok) {
      q.path = PATH_TF32;
      q.cfg = d->variant == SUPRA_ATTN_TF32X3 ? 1 : 0;
    }
  } else if (tma_ok && scale > 0.f && (d->Lq > 64 || q.bias) && d->ldq >= supra::kFwBoxWide &&
             d->ldk >= supra::kFwBoxWide) {
    // persistent FP32 kernel (with or without a bias): its Q/K boxes are kFwBoxWide columns wide
    q.path = PATH_FP32_TMA;
    q.cfg = 0;
  }
  q.flops = 4.0 * d->Lq * (double)d->Lk * d->D * d->H;  // app/gpu/ops.js:116
  q.bytes = 4.0 * ((double)d->Lq * HD * 2 + (double)d->Lk * HD * 2 + (d->bias ? (double)nbias : 0.0));
  return SUPRA_ATTN_OK;
}

int validate_linear(supra_attn_ctx* c, const supra_attn_linear_desc* d, Checked* out) {
  if (!d) return set_err(c, SUPRA_ATTN_EINVAL, "linear descriptor is NULL");
  if (d->flags) return set_err(c, SUPRA_ATTN_EINVAL, "linear: flags must be 0");
  if (d->act > SUPRA_ATTN_ACT_SILU) return set_err(c, SUPRA_ATTN_EINVAL, "linear: act=%u unknown", d->act);
  if (d->variant != SUPRA_ATTN_FP32 && d->variant != SUPRA_ATTN_TF32 && d->variant != SUPRA_ATTN_TF32X3)
    return set_err(c, SUPRA_ATTN_EINVAL, "linear: unknown variant %d", d->variant);
  if (d->M < 0 || d->M > (1 << 30)) return set_err(c, SUPRA_ATTN_EINVAL, "linear: M=%d out of range [0, 2^30]", d->M);
  if (d->N < 1 || d->N > (1 << 30)) return set_err(c, SUPRA_ATTN_EINVAL, "linear: N=%d out of range [1, 2^30]", d->N);
  if (d->K < 1 || d->K > (1 << 30)) return set_err(c, SUPRA_ATTN_EINVAL, "linear: K=%d out of range [1, 2^30]", d->K);
  const int64_t lim = int64_t(1) << 46;
  if (d->ldx < d->K || d->ldw < d->K || d->ldy < d->N || d->ldx > lim || d->ldw > lim || d->ldy > lim)
    return set_err(c, SUPRA_ATTN_EINVAL, "linear: need ldx >= K, ldw >= K, ldy >= N");
  if (d->x_off < 0 || d->y_off < 0 || d->x_off > lim || d->y_off > lim)
    return set_err(c, SUPRA_ATTN_EINVAL, "linear: offset out of range (negative?)");
  if (!d->x || !d->w || !d->y) return set_err(c, SUPRA_ATTN_EINVAL, "linear: x, w and y must be non-NULL");
  const void* ptrs[4] = {d->x, d->w, d->y, d->bias};
  for (int i = 0; i < 4; ++i)
    if (ptrs[i] && (reinterpret_cast<uintptr_t>(ptrs[i]) & 3u))
      return set_err(c, SUPRA_ATTN_EINVAL, "linear: pointers must be 4-byte aligned float arrays");
  out->empty = (d->M == 0);
  const int64_t x_last = d->x_off + (int64_t)(d->M - 1) * d->ldx + d->K - 1;
  const int64_t w_last = (int64_t)(d->N - 1) * d->ldw + d->K - 1;
  const int64_t y_last = d->y_off + (int64_t)(d->M - 1) * d->ldy + d->N - 1;
  if (!out->empty && x_last >= d->x_size)
    return set_err(c, SUPRA_ATTN_EINVAL, "linear: x out of bounds: needs %lld floats, x_size=%lld",
                   (long long)(x_last + 1), (long long)d->x_size);
  if (w_last >= d->w_size)
    return set_err(c, SUPRA_ATTN_EINVAL, "linear: w out of bounds: needs %lld floats, w_size=%lld",
                   (long long)(w_last + 1), (long long)d->w_size);
  if (d->bias && d->N > d->bias_size)
    return set_err(c, SUPRA_ATTN_EINVAL, "linear: bias must hold N=%d floats, bias_size=%lld", d->N,
                   (long long)d->bias_size);
  if (!out->empty && y_last >= d->y_size)
    return set_err(c, SUPRA_ATTN_EINVAL, "linear: y out of bounds: needs %lld floats, y_size=%lld",
                   (long long)(y_last + 1), (long long)d->y_size);
  const int64_t tiles = ((int64_t)d->M + 127) / 128 * (((int64_t)d->N + 127) / 128);
  if (tiles > INT32_MAX) return set_err(c, SUPRA_ATTN_EINVAL, "linear: too many 128x128 tiles");
  const supra_attn_groupnorm* gn = d->gn;
  if (gn) {
    if (!gn->gamma || !gn->beta || (reinterpret_cast<uintptr_t>(gn->gamma) & 3u) ||
        (reinterpret_cast<uintptr_t>(gn->beta) & 3u))
      return set_err(c, SUPRA_ATTN_EINVAL, "linear: groupnorm gamma and beta must be non-NULL float arrays");
    if (gn->groups < 1 || d->K % gn->groups)
      return set_err(c, SUPRA_ATTN_EINVAL, "linear: groupnorm groups=%d must divide K=%d", gn->groups, d->K);
    if (gn->rows_per_image < 1 || (d->M % gn->rows_per_image))
      return set_err(c, SUPRA_ATTN_EINVAL, "linear: groupnorm rows_per_image=%d must divide M=%d", gn->rows_per_image,
                     d->M);
    if (!std::isfinite(gn->eps) || gn->eps < 0.f) return set_err(c, SUPRA_ATTN_EINVAL, "linear: groupnorm eps");
    if (d->x_off != 0 || d->ldx != d->K)
      return set_err(c, SUPRA_ATTN_EINVAL, "linear: groupnorm needs contiguous x rows (x_off == 0, ldx == K)");
    if ((int64_t)(d->M / gn->rows_per_image) * gn->groups > INT32_MAX)
      return set_err(c, SUPRA_ATTN_EINVAL, "linear: too many groupnorm groups");
  }
  const supra_attn_layernorm* ln = d->ln;
  if (ln) {
    if (gn) return set_err(c, SUPRA_ATTN_EINVAL, "linear: groupnorm and layernorm are exclusive");
    if (ln->reserved) return set_err(c, SUPRA_ATTN_EINVAL, "linear: layernorm reserved must be 0");
    if (!std::isfinite(ln->eps) || ln->eps < 0.f) return set_err(c, SUPRA_ATTN_EINVAL, "linear: layernorm eps");
    if (d->x_off != 0 || d->ldx != d->K)
      return set_err(c, SUPRA_ATTN_EINVAL, "linear: layernorm needs contiguous x rows (x_off == 0, ldx == K)");
    if (ln->mod) {
      if (reinterpret_cast<uintptr_t>(ln->mod) & 3u)
        return set_err(c, SUPRA_ATTN_EINVAL, "linear: layernorm mod must be a 4-byte aligned float array");
      if (ln->shift_off < 0 || ln->scale_off < 0 || ln->shift_off > lim || ln->scale_off > lim ||
          ln->shift_off + d->K > ln->mod_size || ln->scale_off + d->K > ln->mod_size)
        return set_err(c, SUPRA_ATTN_EINVAL,
                       "linear: layernorm mod out of bounds: needs shift_off + K and scale_off + K <= mod_size=%lld",
                       (long long)ln->mod_size);
    }
  }
  // in place: resid is y itself, element for element (the reference's out: x, resid: true)
  const bool in_place = d->resid && d->resid == d->y && d->r_off == d->y_off && d->ldr == d->ldy;
  if (d->resid) {
    if (reinterpret_cast<uintptr_t>(d->resid) & 3u)
      return set_err(c, SUPRA_ATTN_EINVAL, "linear: resid must be a 4-byte aligned float array");
    if (d->ldr < d->N || d->ldr > lim || d->r_off < 0 || d->r_off > lim)
      return set_err(c, SUPRA_ATTN_EINVAL, "linear: resid needs ldr >= N and a non-negative r_off");
    if (!out->empty && d->r_off + (int64_t)(d->M - 1) * d->ldr + d->N - 1 >= d->resid_size)
      return set_err(c, SUPRA_ATTN_EINVAL, "linear: resid out of bounds: resid_size=%lld", (long long)d->resid_size);
  }
  if (d->gate) {
    if (!d->resid) return set_err(c, SUPRA_ATTN_EINVAL, "linear: gate needs resid (the gated residual)");
    if (reinterpret_cast<uintptr_t>(d->gate) & 3u)
      return set_err(c, SUPRA_ATTN_EINVAL, "linear: gate must be a 4-byte aligned float array");
    if (d->g_off < 0 || d->g_off > lim || d->g_off + d->N > d->gate_size)
      return set_err(c, SUPRA_ATTN_EINVAL, "linear: gate out of bounds: needs g_off + N <= gate_size");
  }
  auto rng = [](const float* base, int64_t first, int64_t lastidx) {
    ByteRange r;
    r.b = reinterpret_cast<uintptr_t>(base + first);
    r.e = reinterpret_cast<uintptr_t>(base + lastidx + 1);
    return r;
  };
  out->nreads = 0;
  if (!out->empty) {
    out->reads[out->nreads++] = rng(d->x, d->x_off, x_last);
    out->reads[out->nreads++] = rng(d->w, 0, w_last);
    if (d->bias) out->reads[out->nreads++] = rng(d->bias, 0, d->N - 1);
    if (gn) {
      out->reads[out->nreads++] = rng(gn->gamma, 0, d->K - 1);
      out->reads[out->nreads++] = rng(gn->beta, 0, d->K - 1);
    }
    if (ln && ln->mod) {
      out->reads[out->nreads++] = rng(ln->mod, ln->shift_off, ln->shift_off + d->K - 1);
      out->reads[out->nreads++] = rng(ln->mod, ln->scale_off, ln->scale_off + d->K - 1);
    }
    if (d->resid && !in_place)
      out->reads[out->nreads++] = rng(d->resid, d->r_off, d->r_off + (int64_t)(d->M - 1) * d->ldr + d->N - 1);
    if (d->gate) out->reads[out->nreads++] = rng(d->gate, d->g_off, d->g_off + d->N - 1);
    out->write = rng(d->y, d->y_off, y_last);
    for (int i = 0; i < out->nreads; ++i)
      if (out->reads[i].b < out->write.e && out->write.b < out->reads[i].e)
        return set_err(c, SUPRA_ATTN_EINVAL, "linear: y overlaps an input of the same call");
  }
  Queued& q = out->q;
  std::memset(&q.p, 0, sizeof(q.p));
  std::memset(&q.lin, 0, sizeof(q.lin));
  q.lin.x = d->x + d->x_off;
  q.lin.w = d->w;
  q.lin.bias = d->bias;
  q.lin.y = d->y + d->y_off;
  q.lin.ldx = d->ldx;
  q.lin.ldw = d->ldw;
  q.lin.ldy = d->ldy;
  q.lin.M = d->M;
  q.lin.N = d->N;
  q.lin.K = d->K;
  q.lin.n_tiles = (d->N + 127) / 128;
  q.lin.resid = d->resid ? d->resid + d->r_off : nullptr;
  q.lin.ldr = d->resid ? d->ldr : 0;
  q.lin.gate = d->gate ? d->gate + d->g_off : nullptr;
  q.lin.act = (int32_t)d->act;
  q.gn_eps = 0.f;
  if (gn) {
    q.lin.gamma = gn->gamma;
    q.lin.beta = gn->beta;
    q.lin.gn_groups = gn->groups;
    q.lin.gn_cg = d->K / gn->groups;
    q.lin.gn_rows = gn->rows_per_image;
    q.lin.gn_silu = gn->silu ? 1 : 0;
    q.lin.gn_mode = supra::kNormAffine;
    q.gn_eps = gn->eps;
  }
  if (ln) {  // one image per row, one group of K channels (app/gpu/kernels.js:101-113)
    q.lin.gamma = ln->mod ? ln->mod + ln->scale_off : nullptr;
    q.lin.beta = ln->mod ? ln->mod + ln->shift_off : nullptr;
    q.lin.gn_groups = 1;
    q.lin.gn_cg = d->K;
    q.lin.gn_rows = 1;
    q.lin.gn_mode = ln->mod ? supra::kNormModulated : supra::kNormPlain;
    q.gn_eps = ln->eps;
  }
  q.path = PATH_LINEAR;
  // TF32 / TF32X3 requests with at least one 32-deep k-block run on the tensor cores (cfg 1 / 2);
  // FP32 requests and shallower products run the FFMA kernel
  q.cfg = (d->variant != SUPRA_ATTN_FP32 && d->K >= 32) ? (d->variant == SUPRA_ATTN_TF32X3 ? 2 : 1) : 0;
  q.bias = d->bias != nullptr;
  q.aligned = (d->K % 4 == 0) && (d->ldx % 4 == 0) && (d->ldw % 4 == 0) && aligned16(d->x + d->x_off) &&
              aligned16(d->w);
  q.t5_buckets = q.t5_maxd = 0;
  q.rows_q = q.rows_k = q.rows_v = 0;
  q.flops = 2.0 * d->M * (double)d->N * d->K;
  q.bytes = 4.0 * ((double)d->M * d->K + (double)d->N * d->K + (double)d->M * d->N + (d->bias ? d->N : 0) +
                   (d->resid ? (double)d->M * d->N : 0.0) + ((gn || (ln && ln->mod)) ? 2.0 * d->K : 0.0) +
                   (d->gate ? d->N : 0));
  return SUPRA_ATTN_OK;
}

// ---- flush ---------------------------------------------------------------------------------------
// T5 table bias: one bucket table per distinct (buckets, max_distance) among a launch's
// problems, over relative positions [-max_distance, max_distance] (app/models/t5.js:14-23; the
// bucket saturates at max_distance, so the kernels clamp beyond it). off[i] is problem i's
// table offset in ints within blob, or -1 (no T5 table). Returns the blob's bytes, 16-aligned.
size_t t5_luts(const std::vector<const Queued*>& g, std::vector<int32_t>& blob, std::vector<int64_t>& off) {
  blob.clear();
  off.assign(g.size(), -1);
  std::vector<std::pair<int64_t, int64_t>> seen;  // (buckets | maxd << 32, offset)
  for (size_t i = 0; i < g.size(); ++i) {
    const Queued& q = *g[i];
    if (q.t5_buckets == 0) continue;
    const int64_t key = (int64_t)q.t5_buckets | ((int64_t)q.t5_maxd << 32);
    int64_t at = -1;
    for (auto& kv : seen)
      if (kv.first == key) at = kv.second;
    if (at < 0) {
      at = (int64_t)blob.size();
      seen.emplace_back(key, at);
      for (int32_t r = -q.t5_maxd; r <= q.t5_maxd; ++r)
        blob.push_back(supra_attn_relative_bucket(r, q.t5_buckets, q.t5_maxd));
    }
    off[i] = at;
  }
  return align16(blob.size() * sizeof(int32_t));
}

int flush_fused(supra_attn_ctx* c, std::vector<const Queued*>& g) {
  const Queued& first = *g[0];
  const int mq = supra::fused_cfg_tile_rows(first.cfg);
  // longest-first (work per tile grows with the number of key blocks)
  std::stable_sort(g.begin(), g.end(), [](const Queued* a, const Queued* b) { return a->p.Lk > b->p.Lk; });
  const int n = (int)g.size();
  int64_t total = 0;
  double flops = 0, bytes = 0;
  std::vector<int32_t> begin(n + 1);
  for (int i = 0; i < n; ++i) {
    begin[i] = (int32_t)total;
    const int qt = (g[i]->p.Lq + mq - 1) / mq;
    total += (int64_t)qt * g[i]->p.H;
    flops += g[i]->flops;
    bytes += g[i]->bytes;
  }
  if (total > INT32_MAX) return set_err(c, SUPRA_ATTN_EINVAL, "too many tiles in one flush (%lld)", (long long)total);
  begin[n] = (int32_t)total;
  std::vector<int32_t> lut;
  std::vector<int64_t> loff;
  const size_t pbytes = align16(sizeof(AttnProb) * n);
  const size_t lbytes = t5_luts(g, lut, loff);
  const size_t bbytes = sizeof(int32_t) * (n + 1);
  char *h = nullptr, *dv = nullptr;
  int rc = ring_reserve(c, pbytes + lbytes + bbytes, &h, &dv);
  if (rc) return rc;
  AttnProb* hp = reinterpret_cast<AttnProb*>(h);
  for (int i = 0; i < n; ++i) {
    hp[i] = g[i]->p;
    hp[i].q_tiles = (g[i]->p.Lq + mq - 1) / mq;
    hp[i].rel_lut = loff[i] < 0 ? nullptr : reinterpret_cast<const int32_t*>(dv + pbytes) + loff[i];
  }
  if (!lut.empty()) std::memcpy(h + pbytes, lut.data(), lut.size() * sizeof(int32_t));
  std::memcpy(h + pbytes + lbytes, begin.data(), bbytes);
  rc = ring_commit(c, h, dv, pbytes + lbytes + bbytes);
  if (rc) return rc;
  AttnLaunch L;
  L.probs = reinterpret_cast<const AttnProb*>(dv);
  L.begin = reinterpret_cast<const int32_t*>(dv + pbytes + lbytes);
  L.n = n;
  L.total = (int32_t)total;
  L.status = c->d_status;
  L.uniform = 0;
  L.pad = 0;
  {
    const int64_t t0 = begin[1] - begin[0];
    bool uni = t0 > 0;
    for (int i = 1; i < n && uni; ++i) uni = (begin[i + 1] - begin[i]) == t0;
    if (uni) L.uniform = (int32_t)t0;
  }
  const int bias_mode = first.t5_buckets ? 2 : first.bias ? 1 : 0;
  const char* name = supra::attn_fp32_name(first.cfg, bias_mode, first.aligned);
  cudaError_t e;
  {
    ProfScope ps(c, name, flops, bytes);
    e = supra::launch_attn_fp32(first.cfg, bias_mode, first.aligned, L, c->stream);
  }
  if (e != cudaSuccess) return cuda_err(c, e, name);
  c->launches += 1;
  return SUPRA_ATTN_OK;
}

int ensure_scratch(supra_attn_ctx* c, size_t bytes) {
  if (bytes <= c->scratch_cap) return SUPRA_ATTN_OK;
  cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return cuda_err(c, e, "scratch: stream sync");
  if (c->scratch) cudaFree(c->scratch);
  c->scratch = nullptr;
  c->scratch_cap = 0;
  if (cudaMalloc(&c->scratch, bytes) != cudaSuccess) {
    cudaGetLastError();
    return set_err(c, SUPRA_ATTN_ENOMEM, "scratch: cudaMalloc(%zu) failed", bytes);
  }
  c->scratch_cap = bytes;
  return SUPRA_ATTN_OK;
}

// A tensor-core linear job: the problem, a factor applied to x before its split (with the gate
// folding, the only prologue the split applies to the attention operands), whether w is read as
// [K, N] (w[k * ldw + n]: V of an attention as the weights of P V) instead of [N, K], and x given
// ready (xh non-null: the TF32 part at xh, the remainder at xl in the split form, row stride
// ldxs, both 16-byte aligned) instead of from p.x.
struct TcJob {
  supra::LinProb p;
  float xscale;
  bool wtrans;
  const float* xh;
  const float* xl;
  int64_t ldxs;
};

int run_linear_tc(supra_attn_ctx* c, std::vector<TcJob>& jobs, bool split, double flops, double bytes);

int run_gemm_chunk(supra_attn_ctx* c, const std::vector<const Queued*>& g, std::vector<GemmUnit>& units,
                   size_t scratch_bytes, bool bias, bool aligned) {
  if (units.empty()) return SUPRA_ATTN_OK;
  // cfg 1 / 2: both products on the tensor-core linear, TF32 / split form; the split form keeps
  // the probabilities' remainders in a second region of the scratch of the same layout
  const int tc = g[0]->cfg;
  int rc = ensure_scratch(c, tc == 2 ? 2 * scratch_bytes : scratch_bytes);
  if (rc) return rc;
  const int np = (int)g.size();
  const int nu = (int)units.size();
  std::vector<int32_t> qk(nu + 1), pv(nu + 1), rw(nu + 1);
  int64_t tq = 0, tp = 0, tr = 0;
  double fl = 0, by_qk = 0, by_sm = 0, by_pv = 0;
  for (int i = 0; i < nu; ++i) {
    GemmUnit& u = units[i];
    const AttnProb& P = g[u.prob]->p;
    u.qk_begin = (int32_t)tq;
    u.pv_begin = (int32_t)tp;
    u.row_begin = (int32_t)tr;
    qk[i] = u.qk_begin;
    pv[i] = u.pv_begin;
    rw[i] = u.row_begin;
    const int rt = (u.rows + 127) / 128;
    tq += (int64_t)rt * ((P.Lk + 127) / 128);
    tp += (int64_t)rt * ((P.D + 127) / 128);
    tr += u.rows;
    fl += 2.0 * u.rows * (double)P.Lk * P.D;
    const double s = 4.0 * u.rows * (double)P.Lk;
    by_qk += 4.0 * ((double)u.rows * P.D + (double)P.Lk * P.D) + s + (P.bias ? s : 0.0);
    by_sm += 2 * s;
    by_pv += s + 4.0 * ((double)P.Lk * P.D + (double)u.rows * P.D);
  }
  if (tq > INT32_MAX || tp > INT32_MAX || tr > INT32_MAX) return set_err(c, SUPRA_ATTN_EINVAL, "chunk too large");
  qk[nu] = (int32_t)tq;
  pv[nu] = (int32_t)tp;
  rw[nu] = (int32_t)tr;
  std::vector<int32_t> lut;
  std::vector<int64_t> loff;
  const size_t lbytes = t5_luts(g, lut, loff);
  const size_t pbytes = align16(sizeof(AttnProb) * np) + lbytes;  // problems, then T5 bucket tables
  const size_t ubytes = align16(sizeof(GemmUnit) * nu);
  const size_t ibytes = align16(sizeof(int32_t) * (nu + 1));
  char *h = nullptr, *dv = nullptr;
  rc = ring_reserve(c, pbytes + ubytes + 3 * ibytes, &h, &dv);
  if (rc) return rc;
  AttnProb* hp = reinterpret_cast<AttnProb*>(h);
  const size_t lut_at = pbytes - lbytes;
  for (int i = 0; i < np; ++i) {
    hp[i] = g[i]->p;
    hp[i].rel_lut = loff[i] < 0 ? nullptr : reinterpret_cast<const int32_t*>(dv + lut_at) + loff[i];
  }
  if (!lut.empty()) std::memcpy(h + lut_at, lut.data(), lut.size() * sizeof(int32_t));
  std::memcpy(h + pbytes, units.data(), sizeof(GemmUnit) * nu);
  std::memcpy(h + pbytes + ubytes, qk.data(), sizeof(int32_t) * (nu + 1));
  std::memcpy(h + pbytes + ubytes + ibytes, pv.data(), sizeof(int32_t) * (nu + 1));
  std::memcpy(h + pbytes + ubytes + 2 * ibytes, rw.data(), sizeof(int32_t) * (nu + 1));
  rc = ring_commit(c, h, dv, pbytes + ubytes + 3 * ibytes);
  if (rc) return rc;
  GemmLaunch L;
  L.probs = reinterpret_cast<const AttnProb*>(dv);
  L.units = reinterpret_cast<const GemmUnit*>(dv + pbytes);
  L.qk_begin = reinterpret_cast<const int32_t*>(dv + pbytes + ubytes);
  L.pv_begin = reinterpret_cast<const int32_t*>(dv + pbytes + ubytes + ibytes);
  L.row_begin = reinterpret_cast<const int32_t*>(dv + pbytes + ubytes + 2 * ibytes);
  L.scratch = c->scratch;
  L.n_units = nu;
  L.qk_total = (int32_t)tq;
  L.pv_total = (int32_t)tp;
  L.row_total = (int32_t)tr;
  L.status = c->d_status;
  L.lo = tc == 2 ? c->scratch + scratch_bytes / 4 : nullptr;
  L.sm_scale = tc ? 1 : 0;
  cudaError_t e;
  if (tc) {
    // S = Q_h K_h^T (unscaled: the softmax applies the scale) for each unit's rows into its
    // scores: a linear with x = the unit's Q rows and w = K_h, both [rows, D]
    std::vector<TcJob> jobs((size_t)nu);
    for (int i = 0; i < nu; ++i) {
      const GemmUnit& u = units[i];
      const AttnProb& P = g[u.prob]->p;
      supra::LinProb lp;
      std::memset(&lp, 0, sizeof lp);
      lp.x = P.q + P.q_off + (int64_t)u.row0 * P.ldq + (int64_t)u.h * P.D;
      lp.ldx = P.ldq;
      lp.w = P.k + P.k_off + (int64_t)u.h * P.D;
      lp.ldw = P.ldk;
      lp.y = c->scratch + u.s_off;
      lp.ldy = u.ldS;
      lp.M = u.rows;
      lp.N = P.Lk;
      lp.K = P.D;
      lp.n_tiles = (P.Lk + 127) / 128;
      jobs[i] = TcJob{lp, 1.f, false, nullptr, nullptr, 0};
    }
    rc = run_linear_tc(c, jobs, tc == 2, fl, by_qk);
    if (rc) return rc;
  } else {
    {
      ProfScope ps(c, bias ? "attn_gemm_qk_bias" : "attn_gemm_qk", fl, by_qk);
      e = supra::launch_gemm_qk(bias, aligned, L, c->stream);
    }
    if (e != cudaSuccess) return cuda_err(c, e, "attn_gemm_qk");
    c->launches += 1;
  }
  {
    ProfScope ps(c, "attn_softmax_rows", 0.0, by_sm);
    e = supra::launch_softmax_rows(L, c->stream);
  }
  if (e != cudaSuccess) return cuda_err(c, e, "attn_softmax_rows");
  c->launches += 1;
  if (tc) {
    // O_h rows = P V_h: a linear with x = the unit's probabilities, as the softmax left them (in
    // place, or split into the scratch's two regions), and w = V_h read as [Lk, D]
    std::vector<TcJob> jobs((size_t)nu);
    for (int i = 0; i < nu; ++i) {
      const GemmUnit& u = units[i];
      const AttnProb& P = g[u.prob]->p;
      supra::LinProb lp;
      std::memset(&lp, 0, sizeof lp);
      lp.x = c->scratch + u.s_off;
      lp.ldx = u.ldS;
      lp.w = P.v + P.v_off + (int64_t)u.h * P.D;
      lp.ldw = P.ldv;
      lp.y = P.o + P.o_off + (int64_t)u.row0 * P.ldo + (int64_t)u.h * P.D;
      lp.ldy = P.ldo;
      lp.M = u.rows;
      lp.N = P.D;
      lp.K = P.Lk;
      lp.n_tiles = (P.D + 127) / 128;
      jobs[i] = TcJob{lp, 1.f, true, c->scratch + u.s_off, L.lo ? L.lo + u.s_off : nullptr, u.ldS};
    }
    rc = run_linear_tc(c, jobs, tc == 2, fl, by_pv);
    if (rc) return rc;
  } else {
    {
      ProfScope ps(c, "attn_gemm_pv", fl, by_pv);
      e = supra::launch_gemm_pv(aligned, L, c->stream);
    }
    if (e != cudaSuccess) return cuda_err(c, e, "attn_gemm_pv");
    c->launches += 1;
  }
  return SUPRA_ATTN_OK;
}

int flush_gemm(supra_attn_ctx* c, std::vector<const Queued*>& g) {
  const bool bias = g[0]->bias, aligned = g[0]->aligned;
  std::vector<GemmUnit> units;
  size_t used = 0;
  for (int pi = 0; pi < (int)g.size(); ++pi) {
    const AttnProb& P = g[pi]->p;
    const int ldS = (P.Lk + 3) & ~3;
    const size_t row_bytes = (size_t)ldS * 4;
    // rows per unit: the whole problem when it fits the budget, else multiples of 128 rows
    int64_t rows_max = (int64_t)(c->scratch_budget / row_bytes);
    if (rows_max >= 128) rows_max = rows_max / 128 * 128;
    if (rows_max < 1) rows_max = 1;
    for (int h = 0; h < P.H; ++h) {
      for (int r0 = 0; r0 < P.Lq; r0 += (int)std::min<int64_t>(rows_max, P.Lq)) {
        const int rows = (int)std::min<int64_t>(rows_max, P.Lq - r0);
        const size_t ub = align16((size_t)rows * row_bytes);
        if (used + ub > c->scratch_budget && !units.empty()) {
          int rc = run_gemm_chunk(c, g, units, used, bias, aligned);
          if (rc) return rc;
          units.clear();
          used = 0;
        }
        GemmUnit u;
        std::memset(&u, 0, sizeof u);
        u.s_off = (int64_t)(used / 4);
        u.prob = pi;
        u.h = h;
        u.row0 = r0;
        u.rows = rows;
        u.ldS = ldS;
        units.push_back(u);
        used += ub;
      }
    }
  }
  return run_gemm_chunk(c, g, units, used, bias, aligned);
}

// A group read through TMA tensor maps (the TF32 tensor-core kernel or the persistent FP32
// kernel): one tensor map per distinct (buffer, ld, rows, box) in the flush, encoded once per
// context and cached; problems refer to maps by index.
int flush_tma(supra_attn_ctx* c, std::vector<const Queued*>& g, bool tf32) {
  const int mrows = tf32 ? supra::attn_tf32_tile_rows() : supra::attn_fp32_warp_tile_rows();
  // the split kernel needs the operands exactly: fp32 maps with the tensor-core swizzles
  const bool split = tf32 && g[0]->cfg == 1;
  std::stable_sort(g.begin(), g.end(), [](const Queued* a, const Queued* b) { return a->p.Lk > b->p.Lk; });
  const int n = (int)g.size();
  std::vector<supra::TmaProb> probs((size_t)n);
  std::vector<CUtensorMap> maps;
  std::unordered_map<MapKey, int32_t, MapKeyHash> index;
  MapKey last_key{0, 0, 0, 0, 0, 0, 0, 0};
  int32_t last_idx = -1;
  auto map_index = [&](const float* base, int64_t ld, int64_t rows, int32_t box_cols, int32_t box_rows,
                       CUtensorMapSwizzle swz, int32_t* out) -> int {
    const MapKey k{reinterpret_cast<uintptr_t>(base), ld, rows, ld, box_cols, box_rows, (int32_t)swz,
                   (tf32 && !split) ? 1 : 0};
    if (last_idx >= 0 && k == last_key) {
      *out = last_idx;
      return SUPRA_ATTN_OK;
    }
    auto it = index.find(k);
    if (it == index.end()) {
      auto ct = c->map_cache.find(k);
      if (ct == c->map_cache.end()) {
        CUtensorMap m;
        if (!encode_map(&m, k)) return set_err(c, SUPRA_ATTN_ECUDA, "cuTensorMapEncodeTiled failed");
        if (c->map_cache.size() > 65536) c->map_cache.clear();
        ct = c->map_cache.emplace(k, m).first;
      }
      it = index.emplace(k, (int32_t)maps.size()).first;
      maps.push_back(ct->second);
    }
    last_key = k;
    last_idx = it->second;
    *out = it->second;
    return SUPRA_ATTN_OK;
  };
  std::vector<int32_t> begin(n + 1);
  int64_t total = 0;
  double flops = 0, bytes = 0;
  for (int i = 0; i < n; ++i) {
    const Queued& q = *g[i];
    const AttnProb& P = q.p;
    supra::TmaProb& t = probs[i];
    std::memset(&t, 0, sizeof t);
    t.o = P.o;
    t.o_off = P.o_off;
    t.ldo = P.ldo;
    t.bias = P.bias;
    t.rel_max = P.rel_max;
    t.Lq = P.Lq;
    t.Lk = P.Lk;
    t.H = P.H;
    t.D = P.D;
    int rc;
    if (tf32) {
      rc = map_index(P.q, P.ldq, q.rows_q, 32, mrows, CU_TENSOR_MAP_SWIZZLE_128B, &t.mq);
      if (!rc) rc = map_index(P.k, P.ldk, q.rows_k, 32, 64, CU_TENSOR_MAP_SWIZZLE_128B, &t.mk);
      if (!rc) rc = map_index(P.v, P.ldv, q.rows_v, 32, 64, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, &t.mv);
    } else {
      rc = map_index(P.q, P.ldq, q.rows_q, supra::kFwBoxWide, supra::kFwBoxRows, CU_TENSOR_MAP_SWIZZLE_NONE,
                     &t.mq);
      if (!rc)
        rc = map_index(P.k, P.ldk, q.rows_k, supra::kFwBoxWide, supra::kFwBoxRows, CU_TENSOR_MAP_SWIZZLE_NONE,
                       &t.mk);
      if (!rc)
        rc = map_index(P.v, P.ldv, q.rows_v, supra::kFwBoxNarrow, supra::kFwBoxRows, CU_TENSOR_MAP_SWIZZLE_NONE,
                       &t.mv);
    }
    if (rc) return rc;
    t.qx = (int32_t)(P.q_off % P.ldq);
    t.qy = (int32_t)(P.q_off / P.ldq);
    t.kx = (int32_t)(P.k_off % P.ldk);
    t.ky = (int32_t)(P.k_off / P.ldk);
    t.vx = (int32_t)(P.v_off % P.ldv);
    t.vy = (int32_t)(P.v_off / P.ldv);
    t.scale_log2 = P.scale_log2;
    t.q_tiles = (P.Lq + mrows - 1) / mrows;
    begin[i] = (int32_t)total;
    total += (int64_t)t.q_tiles * P.H;
    flops += q.flops;
    bytes += q.bytes;
  }
  // (headroom: claimed tile indices run up to total + 2 x the grid)
  if (total > INT32_MAX - (int64_t(1) << 20))
    return set_err(c, SUPRA_ATTN_EINVAL, "too many tiles in one flush (%lld)", (long long)total);
  begin[n] = (int32_t)total;
  std::vector<int32_t> lut;
  std::vector<int64_t> loff;
  const size_t pbytes = align16(sizeof(supra::TmaProb) * n);
  const size_t lbytes = t5_luts(g, lut, loff);
  const size_t mbytes = sizeof(CUtensorMap) * maps.size();
  const size_t bbytes = align16(sizeof(int32_t) * (n + 1));
  const size_t cbytes = 16;  // the launch's tile counter, staged as zero
  char *h = nullptr, *dv = nullptr;
  int rc = ring_reserve(c, 64 + pbytes + mbytes + lbytes + bbytes + cbytes, &h, &dv);
  if (rc) return rc;
  // tensor maps must sit on a 64-byte boundary in device memory
  const size_t pad = (64 - (reinterpret_cast<uintptr_t>(dv) & 63)) & 63;
  char* hm = h + pad;
  char* dm = dv + pad;
  for (int i = 0; i < n; ++i)
    probs[i].rel_lut = loff[i] < 0 ? nullptr : reinterpret_cast<const int32_t*>(dm + mbytes + pbytes) + loff[i];
  std::memcpy(hm, maps.data(), mbytes);
  std::memcpy(hm + mbytes, probs.data(), sizeof(supra::TmaProb) * n);
  if (!lut.empty()) std::memcpy(hm + mbytes + pbytes, lut.data(), lut.size() * sizeof(int32_t));
  std::memcpy(hm + mbytes + pbytes + lbytes, begin.data(), sizeof(int32_t) * (n + 1));
  std::memset(hm + mbytes + pbytes + lbytes + bbytes, 0, cbytes);
  rc = ring_commit(c, h, dv, pad + mbytes + pbytes + lbytes + bbytes + cbytes);
  if (rc) return rc;
  supra::TmaLaunch L;
  L.next_tile = reinterpret_cast<int32_t*>(dm + mbytes + pbytes + lbytes + bbytes);
  L.maps = reinterpret_cast<const CUtensorMap*>(dm);
  L.probs = reinterpret_cast<const supra::TmaProb*>(dm + mbytes);
  L.begin = reinterpret_cast<const int32_t*>(dm + mbytes + pbytes + lbytes);
  L.n = n;
  L.total = (int32_t)total;
  L.uniform = 0;
  {
    const int64_t t0 = begin[1] - begin[0];
    bool uni = t0 > 0;
    for (int i = 1; i < n && uni; ++i) uni = (begin[i + 1] - begin[i]) == t0;
    if (uni) L.uniform = (int32_t)t0;
  }
  L.status = c->d_status;
  const char* name = !tf32  ? (g[0]->bias ? "attn_fp32_d64_tma_bias" : "attn_fp32_d64_tma")
                     : split ? (g[0]->bias ? "attn_tf32x3_d64_bias" : "attn_tf32x3_d64")
                             : (g[0]->bias ? "attn_tf32_d64_bias" : "attn_tf32_d64");
  cudaError_t e;
  {
    ProfScope ps(c, name, flops, bytes);
    e = tf32 ? supra::launch_attn_tf32(L, g[0]->bias, split, c->stream) : supra::launch_attn_fp32_warp(L, g[0]->bias, c->stream);
  }
  if (e != cudaSuccess) return cuda_err(c, e, name);
  c->launches += 1;
  return SUPRA_ATTN_OK;
}

// Linear group: one launch over the 128x128 output tiles of every recorded problem.
// Grows a context-owned device buffer to at least `need` elements of `esize` bytes (the stream
// is drained first: earlier launches may still read the old buffer).
int grow_buffer(supra_attn_ctx* c, void** buf, size_t* cap, size_t need, size_t esize, const char* what) {
  if (need <= *cap) return SUPRA_ATTN_OK;
  cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return cuda_err(c, e, what);
  if (*buf) cudaFree(*buf);
  *buf = nullptr;
  *cap = 0;
  if (cudaMalloc(buf, need * esize) != cudaSuccess) {
    cudaGetLastError();
    return set_err(c, SUPRA_ATTN_ENOMEM, "%s: cudaMalloc of %zu bytes failed", what, need * esize);
  }
  *cap = need;
  return SUPRA_ATTN_OK;
}

// GroupNorm / LayerNorm statistics of the linear problems that normalise x, into the context's
// statistics buffer, one launch each; sets lp[i].gn_stats (lp[i] starts as g[i]->lin).
int norm_stats(supra_attn_ctx* c, const std::vector<const Queued*>& g, supra::LinProb* lp) {
  const int n = (int)g.size();
  size_t nstats = 0;
  for (int i = 0; i < n; ++i)
    if (lp[i].gn_rows > 0) nstats += (size_t)(lp[i].M / lp[i].gn_rows) * lp[i].gn_groups;
  int rc = grow_buffer(c, reinterpret_cast<void**>(&c->gn_stats), &c->gn_cap, nstats, sizeof(float2), "norm stats");
  if (rc) return rc;
  size_t at = 0;
  for (int i = 0; i < n; ++i) {
    if (lp[i].gn_rows <= 0) continue;
    const int32_t images = lp[i].M / lp[i].gn_rows;
    lp[i].gn_stats = c->gn_stats + at;
    cudaError_t e;
    const bool ln = lp[i].gn_mode != supra::kNormAffine;
    {
      ProfScope ps(c, ln ? "layernorm_stats" : "groupnorm_stats", 0.0, 4.0 * (double)lp[i].M * lp[i].K);
      e = ln ? supra::launch_ln_stats(lp[i].x, lp[i].K, lp[i].M, g[i]->gn_eps, c->gn_stats + at, c->stream)
             : supra::launch_gn_stats(lp[i].x, lp[i].K, lp[i].gn_rows, images, lp[i].gn_groups, g[i]->gn_eps,
                                      c->gn_stats + at, c->stream);
    }
    if (e != cudaSuccess) return cuda_err(c, e, ln ? "layernorm_stats" : "groupnorm_stats");
    c->launches += 1;
    at += (size_t)images * lp[i].gn_groups;
  }
  return SUPRA_ATTN_OK;
}

int flush_linear(supra_attn_ctx* c, std::vector<const Queued*>& g) {
  const int n = (int)g.size();
  std::vector<int32_t> begin(n + 1);
  int64_t total = 0;
  double flops = 0, bytes = 0;
  for (int i = 0; i < n; ++i) {
    begin[i] = (int32_t)total;
    total += (int64_t)((g[i]->lin.M + 127) / 128) * g[i]->lin.n_tiles;
    flops += g[i]->flops;
    bytes += g[i]->bytes;
    if (total > INT32_MAX) return set_err(c, SUPRA_ATTN_EINVAL, "too many linear tiles in one flush");
  }
  begin[n] = (int32_t)total;
  const size_t pbytes = align16(sizeof(supra::LinProb) * n);
  const size_t bbytes = sizeof(int32_t) * (n + 1);
  char *h = nullptr, *dv = nullptr;
  int rc = ring_reserve(c, pbytes + bbytes, &h, &dv);
  if (rc) return rc;
  supra::LinProb* hp = reinterpret_cast<supra::LinProb*>(h);
  for (int i = 0; i < n; ++i) hp[i] = g[i]->lin;
  rc = norm_stats(c, g, hp);
  if (rc) return rc;
  std::memcpy(h + pbytes, begin.data(), bbytes);
  rc = ring_commit(c, h, dv, pbytes + bbytes);
  if (rc) return rc;
  supra::LinLaunch L;
  L.probs = reinterpret_cast<const supra::LinProb*>(dv);
  L.begin = reinterpret_cast<const int32_t*>(dv + pbytes);
  L.n = n;
  L.total = (int32_t)total;
  L.status = c->d_status;
  const char* name = g[0]->bias ? "linear_fp32_bias" : "linear_fp32";
  cudaError_t e;
  {
    ProfScope ps(c, name, flops, bytes);
    e = supra::launch_linear_fp32(g[0]->bias, g[0]->aligned, L, c->stream);
  }
  if (e != cudaSuccess) return cuda_err(c, e, name);
  c->launches += 1;
  return SUPRA_ATTN_OK;
}

// Tensor-core linear group (variants TF32 / TF32X3, cfg 1 / 2): the norm statistics, then the
// hi / lo split of each problem's x (normalised) and of each distinct weight matrix into the
// context's split buffer (dense rows of ldk = K rounded up to 4 floats), then one launch over the
// 128x128 output tiles of every problem.
int flush_linear_tc(supra_attn_ctx* c, std::vector<const Queued*>& g) {
  const int n = (int)g.size();
  std::vector<TcJob> jobs((size_t)n);
  for (int i = 0; i < n; ++i) jobs[i] = TcJob{g[i]->lin, 1.f, false, nullptr, nullptr, 0};
  std::vector<supra::LinProb> lp((size_t)n);
  for (int i = 0; i < n; ++i) lp[i] = g[i]->lin;
  int rc = norm_stats(c, g, lp.data());
  if (rc) return rc;
  double flops = 0, bytes = 0;
  for (int i = 0; i < n; ++i) {
    jobs[i].p = lp[i];
    flops += g[i]->flops;
    bytes += g[i]->bytes;
  }
  return run_linear_tc(c, jobs, g[0]->cfg == 2, flops, bytes);
}

int run_linear_tc(supra_attn_ctx* c, std::vector<TcJob>& jobs, bool split, double flops, double bytes) {
  const int n = (int)jobs.size();
  if (n == 0) return SUPRA_ATTN_OK;
  const size_t parts = split ? 2 : 1;  // hi (and lo)
  std::vector<supra::LinProb> lp((size_t)n);
  for (int i = 0; i < n; ++i) lp[i] = jobs[i].p;
  int rc = SUPRA_ATTN_OK;
  // A gate without an activation folds into the split of w: gate[n] * (x w[n] + b[n]) =
  // x (gate[n] w[n]) + gate[n] b[n], so the product runs the plain epilogue (one extra rounding
  // of gate * w, far inside the FP32 bar). Such a w is split per gate, with a gated bias copy.
  std::vector<char> fold((size_t)n, 0);
  for (int i = 0; i < n; ++i) fold[i] = lp[i].gate != nullptr && lp[i].act == supra::kActNone;
  // Operands read in place: a 16-byte aligned fp32 operand with a row stride of a multiple of 4
  // floats, not to be normalised, scaled, gated or transposed first, is its own TF32 part (the
  // tensor core ignores the 13 low mantissa bits): the TF32 form reads it as it is and the split
  // form copies only its remainder x - hi. Every other operand is copied whole (hi, and lo in the
  // split form) into lin_split: x per job, w once per distinct (w, shape, gate) in the flush.
  // x: 0 = given split by the caller (TcJob::xh), 1 = in place, 2 = copied; w: 1 or 2.
  std::vector<char> xmode((size_t)n, 2), wmode((size_t)n, 2), wfirst((size_t)n, 0);
  std::vector<size_t> xoff((size_t)n, 0), woff((size_t)n, 0), boff((size_t)n, 0);
  size_t need = 0;
  for (int i = 0; i < n; ++i) {
    const size_t kp = (size_t)((lp[i].K + 3) & ~3);
    if (jobs[i].xh) xmode[i] = 0;
    else if (!lp[i].gn_stats && jobs[i].xscale == 1.f && aligned16(lp[i].x) && (lp[i].ldx & 3) == 0) xmode[i] = 1;
    if (!fold[i] && !jobs[i].wtrans && aligned16(lp[i].w) && (lp[i].ldw & 3) == 0) wmode[i] = 1;
    // floats copied per row: none (TF32 in place), the remainder (split form in place), or all
    const size_t xparts = xmode[i] == 0 ? 0 : xmode[i] == 1 ? (split ? 1 : 0) : parts;
    const size_t wparts = wmode[i] == 1 ? (split ? 1 : 0) : parts;
    xoff[i] = need;
    need += xparts * (size_t)lp[i].M * kp;
    if (!wparts) continue;
    const float* gi = fold[i] ? lp[i].gate : nullptr;
    int j = 0;
    for (; j < i; ++j)
      if (wmode[j] == wmode[i] && lp[j].w == lp[i].w && lp[j].ldw == lp[i].ldw && lp[j].N == lp[i].N &&
          lp[j].K == lp[i].K && jobs[j].wtrans == jobs[i].wtrans && (fold[j] ? lp[j].gate : nullptr) == gi &&
          (!gi || lp[j].bias == lp[i].bias))
        break;
    if (j < i) {
      woff[i] = woff[j];
      boff[i] = boff[j];
    } else {
      woff[i] = need;
      wfirst[i] = 1;
      need += wparts * (size_t)lp[i].N * kp;
      if (gi) {  // the gated bias, 16-byte aligned
        boff[i] = need;
        need += ((size_t)lp[i].N + 3) & ~(size_t)3;
      }
    }
  }
  if (need) {
    rc = grow_buffer(c, reinterpret_cast<void**>(&c->lin_split), &c->lin_split_cap, need, sizeof(float),
                     "linear split");
    if (rc) return rc;
  }
  // the split jobs
  std::vector<supra::SplitJob> sj;
  std::vector<int32_t> sbegin;
  int64_t stotal = 0;
  double sbytes = 0;
  // a copy job: hi and lo (either may be null: remainder only, or TF32 part only)
  auto add_split = [&](const float* src, int64_t ld, int32_t rows, int32_t K, float* hi, float* lo, bool trans,
                       float xscale, const supra::LinProb* norm, const float* rowscale, const float* bias_in,
                       float* bias_out) {
    supra::SplitJob J;
    std::memset(&J, 0, sizeof J);
    const int32_t kp = (K + 3) & ~3;
    J.src = src;
    J.hi = hi;
    J.lo = lo;
    J.rowscale = rowscale;
    J.bias_in = bias_in;
    J.bias_out = bias_out;
    if (norm && norm->gn_stats) {
      J.gn_stats = norm->gn_stats;
      J.gamma = norm->gamma;
      J.beta = norm->beta;
      J.gn_mode = norm->gn_mode;
      J.gn_cg = norm->gn_cg;
      J.gn_rows = norm->gn_rows;
      J.gn_groups = norm->gn_groups;
      J.gn_silu = norm->gn_silu;
    }
    J.ld = ld;
    J.rows = rows;
    J.K = K;
    J.ldd = kp;
    J.trans = trans ? 1 : 0;
    J.xscale = xscale;
    J.ktiles = (K + supra::kSplitTileCols - 1) / supra::kSplitTileCols;
    sbegin.push_back((int32_t)stotal);
    stotal += (int64_t)((rows + supra::kSplitTileRows - 1) / supra::kSplitTileRows) * J.ktiles;
    sbytes += 4.0 * (1.0 + (hi ? 1.0 : 0.0) + (lo ? 1.0 : 0.0)) * rows * (double)K;
    sj.push_back(J);
  };
  for (int i = 0; i < n; ++i) {
    const size_t kp = (size_t)((lp[i].K + 3) & ~3);
    float* xb = c->lin_split + xoff[i];
    if (xmode[i] == 2)
      add_split(lp[i].x, lp[i].ldx, lp[i].M, lp[i].K, xb, split ? xb + (size_t)lp[i].M * kp : nullptr, false,
                jobs[i].xscale, &lp[i], nullptr, nullptr, nullptr);
    else if (xmode[i] == 1 && split)
      add_split(lp[i].x, lp[i].ldx, lp[i].M, lp[i].K, nullptr, xb, false, 1.f, nullptr, nullptr, nullptr, nullptr);
    if (!wfirst[i]) continue;
    float* wb = c->lin_split + woff[i];
    if (wmode[i] == 2)
      add_split(lp[i].w, lp[i].ldw, lp[i].N, lp[i].K, wb, split ? wb + (size_t)lp[i].N * kp : nullptr, jobs[i].wtrans,
                1.f, nullptr, fold[i] ? lp[i].gate : nullptr, lp[i].bias, fold[i] ? c->lin_split + boff[i] : nullptr);
    else
      add_split(lp[i].w, lp[i].ldw, lp[i].N, lp[i].K, nullptr, wb, false, 1.f, nullptr, nullptr, nullptr, nullptr);
  }
  if (stotal > INT32_MAX) return set_err(c, SUPRA_ATTN_EINVAL, "too many split tiles in one flush");
  sbegin.push_back((int32_t)stotal);
  // tensor maps: [rows, K] with row stride ld (the split arrays' kp, or the operand's own), 32 x
  // 128 boxes, SWIZZLE_128B, exact fp32 (the tensor core takes them as TF32 values)
  std::vector<CUtensorMap> maps;
  std::unordered_map<MapKey, int32_t, MapKeyHash> index;
  auto map_of = [&](const float* b, int64_t ld, int64_t rows, int64_t cols, int32_t* out, int32_t box_rows = 128) -> int {
    const MapKey k{reinterpret_cast<uintptr_t>(b), ld, rows, cols, 32, box_rows, (int32_t)CU_TENSOR_MAP_SWIZZLE_128B, 0};
    auto it = index.find(k);
    if (it == index.end()) {
      auto ct = c->map_cache.find(k);
      if (ct == c->map_cache.end()) {
        CUtensorMap m;
        if (!encode_map(&m, k)) return set_err(c, SUPRA_ATTN_ECUDA, "cuTensorMapEncodeTiled failed (linear)");
        if (c->map_cache.size() > 65536) c->map_cache.clear();
        ct = c->map_cache.emplace(k, m).first;
      }
      it = index.emplace(k, (int32_t)maps.size()).first;
      maps.push_back(ct->second);
    }
    *out = it->second;
    return SUPRA_ATTN_OK;
  };
  std::vector<supra::LinTcProb> probs((size_t)n);
  std::vector<int32_t> begin((size_t)n + 1);
  int64_t total = 0;
  for (int i = 0; i < n; ++i) {
    supra::LinTcProb& t = probs[i];
    std::memset(&t, 0, sizeof t);
    t.p = lp[i];
    if (fold[i]) {  // the gate lives in the split w and the gated bias
      t.p.gate = nullptr;
      t.p.bias = c->lin_split + boff[i];
    }
    const int64_t kp = (lp[i].K + 3) & ~3;
    const int64_t M = lp[i].M, N = lp[i].N, K = lp[i].K;
    const float* xb = c->lin_split + xoff[i];
    const float* wb = c->lin_split + woff[i];
    if (xmode[i] == 0) {
      rc = map_of(jobs[i].xh, jobs[i].ldxs, M, K, &t.mxh);
      if (!rc && split) rc = map_of(jobs[i].xl, jobs[i].ldxs, M, K, &t.mxl);
    } else if (xmode[i] == 1) {
      rc = map_of(lp[i].x, lp[i].ldx, M, K, &t.mxh);
      if (!rc && split) rc = map_of(xb, kp, M, K, &t.mxl);
    } else {
      rc = map_of(xb, kp, M, K, &t.mxh);
      if (!rc && split) rc = map_of(xb + (size_t)M * kp, kp, M, K, &t.mxl);
    }
    if (!rc && wmode[i] == 1) {
      rc = map_of(lp[i].w, lp[i].ldw, N, K, &t.mwh);
      if (!rc && split) rc = map_of(wb, kp, N, K, &t.mwl);
    } else if (!rc) {
      rc = map_of(wb, kp, N, K, &t.mwh);
      if (!rc && split) rc = map_of(wb + (size_t)N * kp, kp, N, K, &t.mwl);
    }
    // y through TMA stores (32 x 32 boxes) when its rows are 16-byte aligned and N is a multiple
    // of 4 columns; else per-row stores. (A store box clipped at an inner extent that ends inside a
    // 16-byte chunk overwrote the chunk's elements past the extent with zeros on B200: the first
    // columns of a neighbouring head, written by another tile, came out 0.)
    t.my = -1;
    if (!rc && aligned16(lp[i].y) && (lp[i].ldy & 3) == 0 && (N & 3) == 0) rc = map_of(lp[i].y, lp[i].ldy, M, N, &t.my, 32);
    if (rc) return rc;
    t.m_tiles = (lp[i].M + 127) / 128;
    t.n_tiles = (lp[i].N + 127) / 128;
    t.nkb = (lp[i].K + 31) / 32;
    begin[i] = (int32_t)total;
    total += (int64_t)t.m_tiles * t.n_tiles;
    if (total > INT32_MAX) return set_err(c, SUPRA_ATTN_EINVAL, "too many linear tiles in one flush");
  }
  begin[n] = (int32_t)total;
  // one descriptor staging for both launches: tensor maps (64-byte aligned), problems, tile
  // starts, split jobs, split tile starts
  const size_t mbytes = sizeof(CUtensorMap) * maps.size();
  const size_t pbytes = align16(sizeof(supra::LinTcProb) * n);
  const size_t bbytes = align16(sizeof(int32_t) * (n + 1));
  const size_t jbytes = sizeof(supra::SplitJob) * sj.size();
  const size_t sbbytes = sj.empty() ? 0 : sizeof(int32_t) * sbegin.size();
  const size_t body = mbytes + pbytes + bbytes + jbytes + sbbytes;
  char *h = nullptr, *dv = nullptr;
  rc = ring_reserve(c, 64 + body, &h, &dv);
  if (rc) return rc;
  const size_t pad = (64 - (reinterpret_cast<uintptr_t>(dv) & 63)) & 63;
  std::memcpy(h + pad, maps.data(), mbytes);
  std::memcpy(h + pad + mbytes, probs.data(), sizeof(supra::LinTcProb) * n);
  std::memcpy(h + pad + mbytes + pbytes, begin.data(), sizeof(int32_t) * (n + 1));
  if (!sj.empty()) {
    std::memcpy(h + pad + mbytes + pbytes + bbytes, sj.data(), jbytes);
    std::memcpy(h + pad + mbytes + pbytes + bbytes + jbytes, sbegin.data(), sbbytes);
  }
  rc = ring_commit(c, h, dv, pad + body);
  if (rc) return rc;
  cudaError_t e;
  if (!sj.empty()) {
    supra::SplitLaunch S;
    S.jobs = reinterpret_cast<const supra::SplitJob*>(dv + pad + mbytes + pbytes + bbytes);
    S.begin = reinterpret_cast<const int32_t*>(dv + pad + mbytes + pbytes + bbytes + jbytes);
    S.n = (int32_t)sj.size();
    S.total = (int32_t)stotal;
    {
      ProfScope ps(c, "linear_split", 0.0, sbytes);
      e = supra::launch_split(S, c->stream);
    }
    if (e != cudaSuccess) return cuda_err(c, e, "linear_split");
    c->launches += 1;
  }
  supra::LinTcLaunch L;
  L.maps = reinterpret_cast<const CUtensorMap*>(dv + pad);
  L.probs = reinterpret_cast<const supra::LinTcProb*>(dv + pad + mbytes);
  L.begin = reinterpret_cast<const int32_t*>(dv + pad + mbytes + pbytes);
  L.n = n;
  L.total = (int32_t)total;
  L.status = c->d_status;
  const char* name = split ? "linear_tc_tf32x3" : "linear_tc_tf32";
  {
    ProfScope ps(c, name, flops, bytes);
    e = supra::launch_linear_tc(L, split, c->stream);
  }
  if (e != cudaSuccess) return cuda_err(c, e, name);
  c->launches += 1;
  return SUPRA_ATTN_OK;
}

int do_flush(supra_attn_ctx* c) {
  if (c->queue.empty()) return SUPRA_ATTN_OK;
  std::map<int, std::vector<const Queued*>> groups;
  for (const Queued& q : c->queue) {
    // (a T5 table and an expanded bias run as different kernel forms)
    const int key = q.path * 1024 + q.cfg * 8 + (q.t5_buckets ? 4 : 0) + (q.bias ? 2 : 0) + (q.aligned ? 1 : 0);
    groups[key].push_back(&q);
  }
  int rc = SUPRA_ATTN_OK;
  for (auto& kv : groups) {
    const int path = kv.second[0]->path;
    rc = path == PATH_FUSED ? flush_fused(c, kv.second)
         : path == PATH_TF32 ? flush_tma(c, kv.second, true)
         : path == PATH_FP32_TMA ? flush_tma(c, kv.second, false)
         : path == PATH_LINEAR ? (kv.second[0]->cfg ? flush_linear_tc(c, kv.second) : flush_linear(c, kv.second))
                             : flush_gemm(c, kv.second);
    if (rc) break;
  }
  c->queue.clear();
  c->qreads.clear();
  c->qwrites.clear();
  return rc;
}

int check_device_status(supra_attn_ctx* c, int32_t* device_status) {
  cudaError_t e = cudaMemcpyAsync(c->h_status, c->d_status, 4 * sizeof(int32_t), cudaMemcpyDeviceToHost, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return cuda_err(c, e, "sync");
  const int32_t code = c->h_status[0];
  if (device_status) *device_status = code;
  if (code == 0) return SUPRA_ATTN_OK;
  const int32_t blk = c->h_status[1], stage = c->h_status[2], detail = c->h_status[3];
  cudaMemsetAsync(c->d_status, 0, 4 * sizeof(int32_t), c->stream);
  cudaStreamSynchronize(c->stream);
  if (code == supra::DEV_TIMEOUT)
    return set_err(c, SUPRA_ATTN_ETIMEOUT, "device wait timed out (block %d, stage %d, detail %d)", blk, stage,
                   detail);
  return set_err(c, SUPRA_ATTN_EDEVICE, "device status %d (block %d, stage %d, detail %d)", code, blk, stage, detail);
}

int do_sync(supra_attn_ctx* c, int32_t* device_status) {
  int rc = do_flush(c);
  if (rc) return rc;
  cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return cuda_err(c, e, "stream sync");
  return check_device_status(c, device_status);
}

int record(supra_attn_ctx* c, const Checked& ck) {
  if (ck.empty) return SUPRA_ATTN_OK;
  bool hazard = c->qwrites.overlaps(ck.write.b, ck.write.e) || c->qreads.overlaps(ck.write.b, ck.write.e);
  for (int i = 0; i < ck.nreads && !hazard; ++i) hazard = c->qwrites.overlaps(ck.reads[i].b, ck.reads[i].e);
  if (hazard) {
    int rc = do_flush(c);
    if (rc) return rc;
  }
  for (int i = 0; i < ck.nreads; ++i) c->qreads.add(ck.reads[i].b, ck.reads[i].e);
  c->qwrites.add(ck.write.b, ck.write.e);
  c->queue.push_back(ck.q);
  return SUPRA_ATTN_OK;
}

}  // namespace

// ==================================================================================================
extern "C" {

const char* supra_attn_status_string(int status) {
  switch (status) {
    case SUPRA_ATTN_OK: return "ok";
    case SUPRA_ATTN_EINVAL: return "invalid argument";
    case SUPRA_ATTN_ENOMEM: return "out of memory";
    case SUPRA_ATTN_ECUDA: return "CUDA error";
    case SUPRA_ATTN_ETIMEOUT: return "device wait timed out";
    case SUPRA_ATTN_EDEVICE: return "device error";
    case SUPRA_ATTN_ESTATE: return "invalid state";
    default: return "unknown status";
  }
}

const char* supra_attn_last_error(const supra_attn_ctx* ctx) { return ctx ? ctx->err.c_str() : "NULL context"; }

int supra_attn_create(int device, supra_attn_ctx** out) {
  if (!out) return SUPRA_ATTN_EINVAL;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return SUPRA_ATTN_ECUDA;
  }
  if (device < 0 || device >= n) return SUPRA_ATTN_EINVAL;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return SUPRA_ATTN_ECUDA;
  if (prop.major != 10) return SUPRA_ATTN_ECUDA;  // kernels are built for sm_100a only
  DeviceGuard g(device);
  supra_attn_ctx* c = new supra_attn_ctx();
  c->device = device;
  bool ok = cudaStreamCreateWithFlags(&c->own, cudaStreamNonBlocking) == cudaSuccess;
  c->stream = c->own;
  ok = ok && cudaMalloc(&c->d_status, 4 * sizeof(int32_t)) == cudaSuccess;
  ok = ok && cudaMemset(c->d_status, 0, 4 * sizeof(int32_t)) == cudaSuccess;
  ok = ok && cudaMallocHost(&c->h_status, 4 * sizeof(int32_t)) == cudaSuccess;
  ok = ok && cudaEventCreateWithFlags(&c->ring_ev[0], cudaEventDisableTiming) == cudaSuccess;
  ok = ok && cudaEventCreateWithFlags(&c->ring_ev[1], cudaEventDisableTiming) == cudaSuccess;
  if (ok) {
    // 8 MiB halves: the host may record about one DiT step (28 flushes of 2048 problems) ahead
    c->ring_half = size_t(8) << 20;
    void* hd = nullptr;
    ok = cudaMallocHost(&c->ring_h, 2 * c->ring_half) == cudaSuccess &&
         cudaMalloc(&c->ring_d, 2 * c->ring_half) == cudaSuccess &&
         cudaHostGetDevicePointer(&hd, c->ring_h, 0) == cudaSuccess;
    c->ring_hd = static_cast<char*>(hd);
  }
  if (!ok) {
    cudaGetLastError();
    supra_attn_destroy(c);
    return SUPRA_ATTN_ENOMEM;
  }
  *out = c;
  return SUPRA_ATTN_OK;
}

int supra_attn_destroy(supra_attn_ctx* c) {
  if (!c) return SUPRA_ATTN_OK;
  DeviceGuard g(c->device);
  if (c->stream) {
    do_flush(c);
    cudaStreamSynchronize(c->stream);
  }
  for (auto& pe : c->pend) {
    cudaEventDestroy(pe.a);
    cudaEventDestroy(pe.b);
  }
  for (cudaEvent_t e : c->evt_free) cudaEventDestroy(e);
  for (auto& kv : c->pool_free)
    for (void* p : kv.second) cudaFree(p);
  for (auto& kv : c->pool_live) cudaFree(kv.first);
  for (void* p : c->host_live) cudaFreeHost(p);
  if (c->scratch) cudaFree(c->scratch);
  if (c->gn_stats) cudaFree(c->gn_stats);
  if (c->lin_split) cudaFree(c->lin_split);
  if (c->ring_h) cudaFreeHost(c->ring_h);
  if (c->ring_d) cudaFree(c->ring_d);
  for (int i = 0; i < 2; ++i)
    if (c->ring_ev[i]) cudaEventDestroy(c->ring_ev[i]);
  if (c->d_status) cudaFree(c->d_status);
  if (c->h_status) cudaFreeHost(c->h_status);
  if (c->own) cudaStreamDestroy(c->own);
  delete c;
  return SUPRA_ATTN_OK;
}

int supra_attn_set_stream(supra_attn_ctx* c, void* s) {
  if (!c) return SUPRA_ATTN_EINVAL;
  DeviceGuard g(c->device);
  int rc = do_sync(c, nullptr);
  if (rc) return rc;
  c->stream = s ? static_cast<cudaStream_t>(s) : c->own;
  return SUPRA_ATTN_OK;
}

int supra_attn_tensor_alloc(supra_attn_ctx* c, int64_t n, float** dptr) {
  if (!c || !dptr || n < 0) return c ? set_err(c, SUPRA_ATTN_EINVAL, "tensor_alloc: bad arguments") : SUPRA_ATTN_EINVAL;
  DeviceGuard g(c->device);
  const size_t size = pool_round((size_t)n * 4);
  auto it = c->pool_free.find(size);
  void* p = nullptr;
  if (it != c->pool_free.end() && !it->second.empty()) {
    p = it->second.back();
    it->second.pop_back();
  } else if (cudaMalloc(&p, size) != cudaSuccess) {
    cudaGetLastError();
    return set_err(c, SUPRA_ATTN_ENOMEM, "tensor_alloc: cudaMalloc(%zu) failed", size);
  }
  c->pool_live[p] = size;
  *dptr = static_cast<float*>(p);
  return SUPRA_ATTN_OK;
}

int supra_attn_tensor_free(supra_attn_ctx* c, float* dptr) {
  if (!c) return SUPRA_ATTN_EINVAL;
  if (!dptr) return SUPRA_ATTN_OK;
  auto it = c->pool_live.find(dptr);
  if (it == c->pool_live.end()) return set_err(c, SUPRA_ATTN_EINVAL, "tensor_free: pointer not from this context");
  DeviceGuard g(c->device);
  int rc = do_flush(c);  // recorded work may still read it; later reuse is stream-ordered after it
  c->pool_free[it->second].push_back(dptr);
  c->pool_live.erase(it);
  return rc;
}

int supra_attn_upload(supra_attn_ctx* c, float* dst, const float* src, int64_t n) {
  if (!c || n < 0 || (n > 0 && (!dst || !src))) return c ? set_err(c, SUPRA_ATTN_EINVAL, "upload: bad arguments") : 1;
  DeviceGuard g(c->device);
  int rc = do_flush(c);  // as fromArray: recorded work that reads dst runs first (app/gpu/device.js:150-157)
  if (rc) return rc;
  if (n == 0) return SUPRA_ATTN_OK;
  cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)n * 4, cudaMemcpyHostToDevice, c->stream);
  return e == cudaSuccess ? SUPRA_ATTN_OK : cuda_err(c, e, "upload");
}

int supra_attn_download(supra_attn_ctx* c, float* dst, const float* src, int64_t n) {
  if (!c || n < 0 || (n > 0 && (!dst || !src))) return c ? set_err(c, SUPRA_ATTN_EINVAL, "download: bad arguments") : 1;
  DeviceGuard g(c->device);
  int rc = do_flush(c);
  if (rc) return rc;
  if (n > 0) {
    cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)n * 4, cudaMemcpyDeviceToHost, c->stream);
    if (e != cudaSuccess) return cuda_err(c, e, "download");
  }
  cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return cuda_err(c, e, "download: sync");
  return check_device_status(c, nullptr);  // read() surfaces pending errors (app/gpu/device.js:186)
}

int supra_attn_host_alloc(supra_attn_ctx* c, int64_t n, float** hptr) {
  if (!c || !hptr || n < 0) return c ? set_err(c, SUPRA_ATTN_EINVAL, "host_alloc: bad arguments") : 1;
  DeviceGuard g(c->device);
  void* p = nullptr;
  if (cudaMallocHost(&p, std::max<size_t>(16, (size_t)n * 4)) != cudaSuccess) {
    cudaGetLastError();
    return set_err(c, SUPRA_ATTN_ENOMEM, "host_alloc failed");
  }
  c->host_live.insert(p);
  *hptr = static_cast<float*>(p);
  return SUPRA_ATTN_OK;
}

int supra_attn_host_free(supra_attn_ctx* c, float* hptr) {
  if (!c) return SUPRA_ATTN_EINVAL;
  if (!hptr) return SUPRA_ATTN_OK;
  auto it = c->host_live.find(hptr);
  if (it == c->host_live.end()) return set_err(c, SUPRA_ATTN_EINVAL, "host_free: pointer not from this context");
  DeviceGuard g(c->device);
  int rc = do_sync(c, nullptr);
  cudaFreeHost(hptr);
  c->host_live.erase(it);
  return rc;
}

int supra_attn_enqueue(supra_attn_ctx* c, const supra_attn_desc* d) {
  if (!c) return SUPRA_ATTN_EINVAL;
  Checked ck;
  int rc = validate(c, d, &ck);
  if (rc) return rc;
  DeviceGuard g(c->device);
  return record(c, ck);
}

int supra_attn_check_desc(const supra_attn_desc* d, char* msg, int32_t cap) {
  supra_attn_ctx tmp;  // only its message field is used; no device state is touched
  Checked ck;
  const int rc = validate(&tmp, d, &ck);
  if (msg && cap > 0) std::snprintf(msg, (size_t)cap, "%s", rc ? tmp.err.c_str() : "");
  return rc;
}

int supra_attn_enqueue_linear(supra_attn_ctx* c, const supra_attn_linear_desc* d) {
  if (!c) return SUPRA_ATTN_EINVAL;
  Checked ck;
  int rc = validate_linear(c, d, &ck);
  if (rc) return rc;
  DeviceGuard g(c->device);
  return record(c, ck);
}

int supra_attn_check_linear_desc(const supra_attn_linear_desc* d, char* msg, int32_t cap) {
  supra_attn_ctx tmp;  // only its message field is used; no device state is touched
  Checked ck;
  const int rc = validate_linear(&tmp, d, &ck);
  if (msg && cap > 0) std::snprintf(msg, (size_t)cap, "%s", rc ? tmp.err.c_str() : "");
  return rc;
}

int supra_attn_enqueue_batch(supra_attn_ctx* c, const supra_attn_desc* descs, int32_t n) {
  if (!c) return SUPRA_ATTN_EINVAL;
  if (n < 0 || (n > 0 && !descs)) return set_err(c, SUPRA_ATTN_EINVAL, "enqueue_batch: bad arguments");
  std::vector<Checked> cks((size_t)n);
  for (int32_t i = 0; i < n; ++i) {
    int rc = validate(c, descs + i, &cks[i]);
    if (rc) {
      c->err = "problem " + std::to_string(i) + ": " + c->err;
      return rc;
    }
  }
  DeviceGuard g(c->device);
  for (int32_t i = 0; i < n; ++i) {
    int rc = record(c, cks[i]);
    if (rc) return rc;
  }
  return SUPRA_ATTN_OK;
}

int supra_attn_flush(supra_attn_ctx* c) {
  if (!c) return SUPRA_ATTN_EINVAL;
  DeviceGuard g(c->device);
  return do_flush(c);
}

int supra_attn_sync(supra_attn_ctx* c, int32_t* device_status) {
  if (!c) return SUPRA_ATTN_EINVAL;
  DeviceGuard g(c->device);
  return do_sync(c, device_status);
}

int supra_attn_pending(const supra_attn_ctx* c, int32_t* n) {
  if (!c || !n) return SUPRA_ATTN_EINVAL;
  *n = (int32_t)c->queue.size();
  return SUPRA_ATTN_OK;
}

int32_t supra_attn_relative_bucket(int32_t rel, int32_t buckets, int32_t max_distance) {
  // relativeBucket (app/models/t5.js:14-23), float32 rounding at every step like Math.fround
  if (buckets < 4 || (buckets & 1)) return -1;
  const int32_t nb = buckets / 2;
  const int32_t max_exact = nb / 2;
  if (max_distance <= max_exact) return -1;
  int32_t bucket = rel > 0 ? nb : 0;
  const int64_t n = rel < 0 ? -(int64_t)rel : (int64_t)rel;
  if (n < max_exact) return bucket + (int32_t)n;
  const float a = (float)((double)n / (double)max_exact);
  const float b = (float)std::log((double)a);
  const float cc = (float)std::log((double)max_distance / (double)max_exact);
  const float dd = (float)((double)b / (double)cc);
  const float e = (float)((double)dd * (double)(nb - max_exact));
  const int64_t large = (int64_t)max_exact + (int64_t)std::trunc((double)e);
  return bucket + (int32_t)std::min<int64_t>(large, nb - 1);
}

int supra_attn_position_bias(supra_attn_ctx* c, const float* table, int64_t table_size, int32_t buckets,
                             int32_t max_distance, int32_t H, int32_t L, float* out, int64_t out_size) {
  if (!c) return SUPRA_ATTN_EINVAL;
  if (!table || !out) return set_err(c, SUPRA_ATTN_EINVAL, "position_bias: table and out must be non-NULL");
  if (H < 1 || H > 65536 || L < 1 || L > (1 << 14)) return set_err(c, SUPRA_ATTN_EINVAL, "position_bias: bad H or L");
  if (supra_attn_relative_bucket(0, buckets, max_distance) < 0)
    return set_err(c, SUPRA_ATTN_EINVAL, "position_bias: buckets must be even and >= 4, max_distance > buckets/4");
  if ((int64_t)buckets * H > table_size)
    return set_err(c, SUPRA_ATTN_EINVAL, "position_bias: table holds fewer than buckets*H floats");
  if ((int64_t)H * L * L > out_size) return set_err(c, SUPRA_ATTN_EINVAL, "position_bias: out holds fewer than H*L*L");
  if (reinterpret_cast<uintptr_t>(out) < reinterpret_cast<uintptr_t>(table + table_size) &&
      reinterpret_cast<uintptr_t>(table) < reinterpret_cast<uintptr_t>(out + (int64_t)H * L * L))
    return set_err(c, SUPRA_ATTN_EINVAL, "position_bias: out overlaps table");
  DeviceGuard g(c->device);
  int rc = do_flush(c);
  if (rc) return rc;
  const size_t n = 2 * (size_t)L - 1;
  char *h = nullptr, *dv = nullptr;
  rc = ring_reserve(c, n * sizeof(int32_t), &h, &dv);
  if (rc) return rc;
  int32_t* lut = reinterpret_cast<int32_t*>(h);
  for (int32_t r = -(L - 1); r <= L - 1; ++r) lut[r + L - 1] = supra_attn_relative_bucket(r, buckets, max_distance);
  rc = ring_commit(c, h, dv, n * sizeof(int32_t));
  if (rc) return rc;
  cudaError_t e;
  {
    ProfScope ps(c, "position_bias", 0.0, 4.0 * (double)H * L * L);
    e = supra::launch_position_bias(table, reinterpret_cast<const int32_t*>(dv), H, L, out, c->stream);
  }
  if (e != cudaSuccess) return cuda_err(c, e, "position_bias");
  c->launches += 1;
  return SUPRA_ATTN_OK;
}

int supra_attn_profile_enable(supra_attn_ctx* c, int32_t on) {
  if (!c) return SUPRA_ATTN_EINVAL;
  c->profile = on != 0;
  return SUPRA_ATTN_OK;
}

int supra_attn_profile_report(supra_attn_ctx* c, supra_attn_profile_entry* entries, int32_t cap, int32_t* n) {
  if (!c || !n || cap < 0 || (cap > 0 && !entries)) return SUPRA_ATTN_EINVAL;
  DeviceGuard g(c->device);
  int rc = do_sync(c, nullptr);
  if (rc) return rc;
  rc = collect_profile(c);
  if (rc) return rc;
  std::vector<std::pair<std::string, ProfStat>> v(c->stats.begin(), c->stats.end());
  std::sort(v.begin(), v.end(), [](const auto& a, const auto& b) { return a.second.ms > b.second.ms; });
  int32_t k = 0;
  for (auto& kv : v) {
    if (k >= cap) break;
    supra_attn_profile_entry& e = entries[k++];
    std::memset(&e, 0, sizeof e);
    std::snprintf(e.name, sizeof e.name, "%s", kv.first.c_str());
    e.launches = kv.second.launches;
    e.ms = kv.second.ms;
    e.flops = kv.second.flops;
    e.bytes = kv.second.bytes;
  }
  *n = k;
  return SUPRA_ATTN_OK;
}

int supra_attn_profile_reset(supra_attn_ctx* c) {
  if (!c) return SUPRA_ATTN_EINVAL;
  DeviceGuard g(c->device);
  int rc = do_sync(c, nullptr);
  if (rc) return rc;
  rc = collect_profile(c);
  c->stats.clear();
  return rc;
}

int supra_attn_launch_count(const supra_attn_ctx* c, int64_t* n) {
  if (!c || !n) return SUPRA_ATTN_EINVAL;
  *n = c->launches;
  return SUPRA_ATTN_OK;
}

}  // extern "C"
