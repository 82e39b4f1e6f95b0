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
//
// This file: recording (validation, hazard tracking), flush/sync and the C ABI entry points; the
// rest of the runtime is declared in runtime.h.
#include "runtime.h"

using namespace supra::rt;

namespace {

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

// Merges r into the last few runs it overlaps or touches (reads), or appends it. Batches list
// their problems in memory order, so runs stay few (the DiT self-attention's 2048 q/k/v reads of
// one buffer become one run) and a batch of separate buffers (T5 prompts) keeps one run each.
void add_run(std::vector<ByteRange>& runs, const ByteRange& r) {
  if (r.b >= r.e) return;
  const size_t n = runs.size();
  for (size_t k = n; k-- > (n > 4 ? n - 4 : 0);) {
    ByteRange& x = runs[k];
    if (r.b <= x.e && x.b <= r.e) {
      x.b = std::min(x.b, r.b);
      x.e = std::max(x.e, r.e);
      return;
    }
  }
  runs.push_back(r);
}

// A batch none of whose problems writes memory that another of its problems, or a recorded
// problem, reads or writes, and that reads nothing a recorded problem writes, is hazard-free in
// any order: it is recorded with one merge of its ranges into the hazard sets. Returns false
// (nothing recorded) for any other batch, which is then recorded problem by problem.
bool record_batch_fast(supra_attn_ctx* c, const std::vector<Checked>& cks, int32_t n) {
  std::vector<ByteRange>& W = c->batch_writes;
  std::vector<ByteRange>& R = c->batch_reads;
  W.clear();
  R.clear();
  for (int32_t i = 0; i < n; ++i) {
    const Checked& ck = cks[i];
    if (ck.empty) continue;
    const ByteRange& w = ck.write;
    if (w.b < w.e) {  // writes may touch (adjacent outputs) but not overlap
      bool merged = false;
      const size_t m = W.size();
      for (size_t k = m; k-- > (m > 4 ? m - 4 : 0);) {
        ByteRange& x = W[k];
        if (w.b < x.e && x.b < w.e) return false;
        if (w.b == x.e || w.e == x.b) {
          x.b = std::min(x.b, w.b);
          x.e = std::max(x.e, w.e);
          merged = true;
          break;
        }
      }
      if (!merged) W.push_back(w);
    }
    for (int k = 0; k < ck.nreads; ++k) add_run(R, ck.reads[k]);
  }
  auto by_begin = [](const ByteRange& a, const ByteRange& b) { return a.b < b.b; };
  if (!std::is_sorted(W.begin(), W.end(), by_begin)) std::sort(W.begin(), W.end(), by_begin);
  if (!std::is_sorted(R.begin(), R.end(), by_begin)) std::sort(R.begin(), R.end(), by_begin);
  for (size_t i = 1; i < W.size(); ++i)
    if (W[i].b < W[i - 1].e) return false;  // two writes of the batch overlap
  // reads against the batch's writes: both sorted by begin, the writes disjoint
  size_t j = 0;
  for (const ByteRange& r : R) {
    while (j < W.size() && W[j].e <= r.b) ++j;
    if (j < W.size() && W[j].b < r.e) return false;
  }
  if (!c->qwrites.empty() || !c->qreads.empty()) {  // (empty after a flush)
    for (const ByteRange& w : W)
      if (c->qwrites.overlaps(w.b, w.e) || c->qreads.overlaps(w.b, w.e)) return false;
    for (const ByteRange& r : R)
      if (c->qwrites.overlaps(r.b, r.e)) return false;
  }
  c->qreads.add_batch(R);
  c->qwrites.add_batch(W);
  c->queue.reserve(c->queue.size() + (size_t)n);
  for (int32_t i = 0; i < n; ++i)
    if (!cks[i].empty) c->queue.push_back(cks[i].q);
  return true;
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
  if (c->map_table) cudaFree(c->map_table);
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
  std::vector<Checked>& cks = c->batch_checked;  // reused across calls: no allocation per batch
  if (cks.size() < (size_t)n) cks.resize((size_t)n);
  for (int32_t i = 0; i < n; ++i) {
    int rc = validate(c, descs + i, &cks[i]);
    if (rc) {
      c->err = "problem " + std::to_string(i) + ": " + c->err;
      return rc;
    }
  }
  DeviceGuard g(c->device);
  if (record_batch_fast(c, cks, n)) return SUPRA_ATTN_OK;
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
