// Internal interface of the libsupra_attn host runtime (not installed; the public C ABI is
// include/supra_attn.h). The context, the recorded problems and the helpers shared by the runtime's
// translation units:
//   runtime.cpp       tensor maps, errors, the descriptor ring, profiling, context-owned buffers
//   validate.cpp      argument checks of the attention and linear descriptors (ops.js:103-149)
//   flush_attn.cpp    the attention groups of a flush: block, score-materialising and TMA kernels
//   flush_linear.cpp  the linear groups of a flush: FFMA and tensor-core kernels
//   supra_attn.cpp    recording, flush/sync and the C ABI entry points
#pragma once

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

namespace supra {
namespace rt {

using supra::AttnLaunch;
using supra::AttnProb;
using supra::GemmLaunch;
using supra::GemmUnit;

constexpr float kLog2e = 1.4426950408889634f;

struct ByteRange {
  uintptr_t b = 0, e = 0;
};

// Disjoint, merged [begin, end) byte ranges, kept sorted in a flat vector: an overlap test is one
// binary search, an add merges in place (no allocation per range: recording 256 separate T5
// prompts took ~0.15 ms with a node-based map). Ranges added as a batch wait unsorted until the
// set is next queried, so a batch that is flushed before the next recording is never sorted.
class IntervalSet {
 public:
  void clear() {
    v_.clear();
    pend_.clear();
  }
  bool empty() const { return v_.empty() && pend_.empty(); }
  bool overlaps(uintptr_t b, uintptr_t e) const {
    settle();
    if (b >= e || v_.empty()) return false;
    // the first range ending after b is the only one that can start before e
    auto it = std::upper_bound(v_.begin(), v_.end(), b, [](uintptr_t x, const ByteRange& r) { return x < r.e; });
    return it != v_.end() && it->b < e;
  }
  void add(uintptr_t b, uintptr_t e) {
    settle();
    if (b >= e) return;
    // ranges touching [b, e] (end >= b and begin <= e) merge with it
    auto lo = std::lower_bound(v_.begin(), v_.end(), b, [](const ByteRange& r, uintptr_t x) { return r.e < x; });
    auto hi = lo;
    while (hi != v_.end() && hi->b <= e) {
      b = std::min(b, hi->b);
      e = std::max(e, hi->e);
      ++hi;
    }
    if (lo == hi) {
      v_.insert(lo, ByteRange{b, e});
    } else {
      lo->b = b;
      lo->e = e;
      v_.erase(lo + 1, hi);
    }
  }
  // Adds ranges in any order (they may overlap or touch each other).
  void add_batch(const std::vector<ByteRange>& in) { pend_.insert(pend_.end(), in.begin(), in.end()); }

 private:
  // sorts the pending ranges and merges them into v_ in one pass
  void settle() const {
    if (pend_.empty()) return;
    auto by_begin = [](const ByteRange& a, const ByteRange& b) { return a.b < b.b; };
    if (!std::is_sorted(pend_.begin(), pend_.end(), by_begin)) std::sort(pend_.begin(), pend_.end(), by_begin);
    tmp_.clear();
    tmp_.reserve(v_.size() + pend_.size());
    size_t i = 0, j = 0;
    while (i < v_.size() || j < pend_.size()) {
      const ByteRange r = (j == pend_.size() || (i < v_.size() && v_[i].b <= pend_[j].b)) ? v_[i++] : pend_[j++];
      if (r.b >= r.e) continue;
      if (!tmp_.empty() && r.b <= tmp_.back().e) tmp_.back().e = std::max(tmp_.back().e, r.e);
      else tmp_.push_back(r);
    }
    v_.swap(tmp_);
    pend_.clear();
  }
  mutable std::vector<ByteRange> v_, pend_, tmp_;
};

enum Path : int { PATH_FUSED = 0, PATH_GEMM = 1, PATH_TF32 = 2, PATH_FP32_TMA = 3, PATH_LINEAR = 4 };

struct Queued {
  union {
    AttnProb p;          // attention problems
    supra::LinProb lin;  // PATH_LINEAR: the linear problem
  };
  int path;
  int cfg;
  bool bias;
  bool aligned;
  double flops;
  double bytes;
  int64_t rows_q, rows_k, rows_v;  // whole rows of each operand buffer (TMA tensor maps)
  int64_t rows_o;                  // whole H*D-float rows of the output buffer
  int32_t t5_buckets, t5_maxd;      // T5 table bias (SUPRA_ATTN_F_T5_TABLE), else 0
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

inline size_t pool_round(size_t bytes) {  // BufferPool.round (app/gpu/device.js:64-70)
  size_t b = std::max<size_t>(256, bytes);
  size_t p = 1;
  while (p * 2 <= b) p *= 2;
  const size_t step = std::max<size_t>(256, p / 8);
  return (b + step - 1) / step * step;
}

inline size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

// An encoded tensor map, and its slot in the launch being packed when it was last used there.
struct CachedMap {
  CUtensorMap map;
  uint64_t epoch = 0;  // map_slot: the launch this map was last packed into, and its slot there
  int32_t slot = -1;
  int32_t dslot = -1;   // map_table_slot: its slot in the context's device table ...
  uint64_t depoch = 0;  // ... valid while this equals the table's epoch
};

// A validated problem with the byte ranges it reads and writes (hazard tracking).
struct Checked {
  Queued q;
  ByteRange reads[8];
  int nreads = 0;
  ByteRange write;
  bool empty = false;  // Lq == 0: nothing to do
};

}  // namespace rt
}  // namespace supra

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

  std::vector<supra::rt::Queued> queue;
  supra::rt::IntervalSet qreads, qwrites;
  // enqueue_batch's working storage, kept across calls
  std::vector<supra::rt::Checked> batch_checked;
  std::vector<supra::rt::ByteRange> batch_reads, batch_writes;

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
  std::vector<supra::rt::PendingEvt> pend;
  std::vector<cudaEvent_t> evt_free;
  std::map<std::string, supra::rt::ProfStat> stats;

  // encoded TMA tensor maps, reused across flushes (keyed by buffer, box and element handling)
  std::unordered_map<supra::rt::MapKey, supra::rt::CachedMap, supra::rt::MapKeyHash> map_cache;
  uint64_t map_epoch = 0;  // one per launch being packed (map_slot)
  // the attention launches' tensor maps: a device table that persists across flushes, each cached
  // map given a slot at its first use (only maps new to the table are staged); a new epoch
  // empties it
  CUtensorMap* map_table = nullptr;
  int32_t map_table_cap = 0, map_table_used = 0;
  uint64_t map_table_epoch = 1;

  int64_t launches = 0;
  std::string err;
};

namespace supra {
namespace rt {

// ---- runtime.cpp ----
bool encode_map(CUtensorMap* m, const MapKey& k);
// The slot in `maps` (the tensor maps of the launch being packed, map epoch c->map_epoch) of the
// map for k: encoded once per context and cached, appended to maps at its first use in the epoch.
int map_slot(supra_attn_ctx* c, const MapKey& k, std::vector<CUtensorMap>& maps, int32_t* out);
// Makes room for `need` more maps in the device table (a new epoch when it is full: launches
// already on the stream finish before the slots are written again; a larger table when one
// launch needs more than it holds), trimming the host cache alongside.
int map_table_reserve(supra_attn_ctx* c, size_t need);
// The device-table slot of the map for k; a map new to the table is appended to `fresh` (the
// slots of a flush's fresh maps are consecutive, from the table's fill level before the flush).
int map_table_slot(supra_attn_ctx* c, const MapKey& k, std::vector<const CUtensorMap*>& fresh, int32_t* out);
int set_err(supra_attn_ctx* c, int code, const char* fmt, ...);
int cuda_err(supra_attn_ctx* c, cudaError_t e, const char* what);
int ring_reserve(supra_attn_ctx* c, size_t bytes, char** host, char** dev);
int ring_commit(supra_attn_ctx* c, char* host, char* dev, size_t bytes);
cudaEvent_t take_event(supra_attn_ctx* c);
int collect_profile(supra_attn_ctx* c);
int ensure_scratch(supra_attn_ctx* c, size_t bytes);
int grow_buffer(supra_attn_ctx* c, void** buf, size_t* cap, size_t need, size_t esize, const char* what);

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

// ---- validate.cpp ----

bool aligned16(const void* p);
int validate(supra_attn_ctx* c, const supra_attn_desc* d, Checked* out);
int validate_linear(supra_attn_ctx* c, const supra_attn_linear_desc* d, Checked* out);

// ---- flush_attn.cpp / flush_linear.cpp ----
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

int flush_fused(supra_attn_ctx* c, std::vector<const Queued*>& g);
int flush_gemm(supra_attn_ctx* c, std::vector<const Queued*>& g);
int flush_tma(supra_attn_ctx* c, std::vector<const Queued*>& g, bool tf32);
int flush_linear(supra_attn_ctx* c, std::vector<const Queued*>& g);
int run_linear_fp32(supra_attn_ctx* c, std::vector<supra::LinProb>& lp, bool bias, bool aligned, double flops,
                    double bytes, const char* name, bool w_kn = false);
int flush_linear_tc(supra_attn_ctx* c, std::vector<const Queued*>& g);
int run_linear_tc(supra_attn_ctx* c, std::vector<TcJob>& jobs, bool split, double flops, double bytes);

}  // namespace rt
}  // namespace supra
