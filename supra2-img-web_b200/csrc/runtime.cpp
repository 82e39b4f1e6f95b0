// libsupra_attn host runtime: tensor maps, errors, the descriptor ring, profiling and the
// context-owned device buffers.
#include "runtime.h"

namespace supra {
namespace rt {

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

int map_table_reserve(supra_attn_ctx* c, size_t need) {
  if (c->map_cache.size() + need > 65536) {  // (every map is encoded and staged again as it is used)
    c->map_cache.clear();
    ++c->map_table_epoch;
    c->map_table_used = 0;
  }
  if (need > (size_t)c->map_table_cap) {
    size_t cap = 16384;
    while (cap < need) cap *= 2;
    if (cap > (size_t(1) << 24)) return set_err(c, SUPRA_ATTN_EINVAL, "too many tensor maps in one flush");
    if (c->map_table) {  // earlier launches may still read the old table
      cudaError_t e = cudaStreamSynchronize(c->stream);
      if (e != cudaSuccess) return cuda_err(c, e, "map table: stream sync");
      cudaFree(c->map_table);
      c->map_table = nullptr;
      c->map_table_cap = 0;
    }
    if (cudaMalloc(&c->map_table, cap * sizeof(CUtensorMap)) != cudaSuccess) {
      cudaGetLastError();
      return set_err(c, SUPRA_ATTN_ENOMEM, "map table: cudaMalloc failed");
    }
    c->map_table_cap = (int32_t)cap;
    ++c->map_table_epoch;
    c->map_table_used = 0;
  } else if ((size_t)c->map_table_used + need > (size_t)c->map_table_cap) {
    ++c->map_table_epoch;  // (launches already on the stream read their slots before they are rewritten)
    c->map_table_used = 0;
  }
  return SUPRA_ATTN_OK;
}

int map_table_slot(supra_attn_ctx* c, const MapKey& k, std::vector<const CUtensorMap*>& fresh, int32_t* out) {
  auto ct = c->map_cache.find(k);
  if (ct == c->map_cache.end()) {
    CachedMap e;
    if (!encode_map(&e.map, k)) return set_err(c, SUPRA_ATTN_ECUDA, "cuTensorMapEncodeTiled failed");
    ct = c->map_cache.emplace(k, e).first;  // (references to entries stay valid: no trim here)
  }
  CachedMap& m = ct->second;
  if (m.depoch != c->map_table_epoch) {
    m.depoch = c->map_table_epoch;
    m.dslot = c->map_table_used++;
    fresh.push_back(&m.map);
  }
  *out = m.dslot;
  return SUPRA_ATTN_OK;
}

int map_slot(supra_attn_ctx* c, const MapKey& k, std::vector<CUtensorMap>& maps, int32_t* out) {
  auto ct = c->map_cache.find(k);
  if (ct == c->map_cache.end()) {
    CachedMap e;
    if (!encode_map(&e.map, k)) return set_err(c, SUPRA_ATTN_ECUDA, "cuTensorMapEncodeTiled failed");
    if (c->map_cache.size() > 65536) c->map_cache.clear();  // (entries of this epoch are re-added)
    ct = c->map_cache.emplace(k, e).first;
  }
  CachedMap& m = ct->second;
  if (m.epoch != c->map_epoch) {
    m.epoch = c->map_epoch;
    m.slot = (int32_t)maps.size();
    maps.push_back(m.map);
  }
  *out = m.slot;
  return SUPRA_ATTN_OK;
}



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

}  // namespace rt
}  // namespace supra
