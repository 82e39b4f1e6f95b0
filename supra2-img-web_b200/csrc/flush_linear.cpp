// libsupra_attn host runtime: the linear groups of a flush (ops.linear, app/gpu/ops.js:35-43) on the
// FFMA kernel and on the tensor cores.
#include "runtime.h"

namespace supra {
namespace rt {

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

// Column tile width of an FFMA linear launch: 128 x 64 tiles cost about 0.55 of a 128 x 128 tile
// (a smaller register block reads more shared memory per FMA); take the width whose whole waves of
// the grid's CTA slots (two per SM) cost less. The DiT blocks' N = 576 products: 2 waves either
// way, 1.1 against 2.0 in tile costs; the stacked K/V preparation (N = 16128) keeps 128.
static int linear_tile_cols(const std::vector<supra::LinProb>& lp) {
  int64_t t128 = 0, t64 = 0;
  for (const supra::LinProb& q : lp) {
    const int64_t mt = (q.M + 127) / 128;
    t128 += mt * ((q.N + 127) / 128);
    t64 += mt * ((q.N + 63) / 64);
  }
  const int64_t slots = supra::attn_fp32_warp_cta_slots();
  return 0.55 * (double)((t64 + slots - 1) / slots) < (double)((t128 + slots - 1) / slots) ? 64 : 128;
}

// One grouped FFMA linear launch over problems whose x is ready to be read as it is (any norm
// prologue still set in gn_stats runs per staged tile). 16-byte aligned groups (`aligned`) stage
// their tiles by TMA: a tensor map of x [M, K] with kLinBoxCols x 128 boxes and of W [N, K] with
// kLinBoxCols x (tile columns) boxes per problem, cached per context like the attention kernels'
// maps; a shape the driver's encoder refuses, or a misaligned group, takes the per-thread copy form.
int run_linear_fp32(supra_attn_ctx* c, std::vector<supra::LinProb>& lp, bool bias, bool aligned, double flops,
                    double bytes, const char* name, bool w_kn) {
  const int n = (int)lp.size();
  const int cols = linear_tile_cols(lp);
  std::vector<int32_t> begin(n + 1);
  int64_t total = 0;
  for (int i = 0; i < n; ++i) {
    lp[i].n_tiles = (lp[i].N + cols - 1) / cols;
    begin[i] = (int32_t)total;
    total += (int64_t)((lp[i].M + 127) / 128) * lp[i].n_tiles;
    if (total > INT32_MAX) return set_err(c, SUPRA_ATTN_EINVAL, "too many linear tiles in one flush");
  }
  begin[n] = (int32_t)total;
  bool tma = aligned;
  std::vector<CUtensorMap> maps;
  ++c->map_epoch;
  for (int i = 0; i < n && tma; ++i) {
    const supra::LinProb& q = lp[i];
    int rc0 = map_slot(c, MapKey{reinterpret_cast<uintptr_t>(q.x), q.ldx, q.M, q.K, supra::kLinBoxCols, 128, 0, 0},
                       maps, &lp[i].mx);
    if (!rc0)
      rc0 = w_kn ? map_slot(c, MapKey{reinterpret_cast<uintptr_t>(q.w), q.ldw, q.K, q.N, cols, 32, 0, 0}, maps, &lp[i].mw)
                 : map_slot(c, MapKey{reinterpret_cast<uintptr_t>(q.w), q.ldw, q.N, q.K, supra::kLinBoxCols, cols, 0, 0},
                            maps, &lp[i].mw);
    if (rc0) {
      tma = false;
      maps.clear();
      c->err.clear();
    }
    lp[i].w_kn = w_kn ? 1 : 0;
  }
  // W as [K, N] has only the TMA-staged form (callers pass aligned operands)
  if (w_kn && !tma) return set_err(c, SUPRA_ATTN_EINVAL, "%s: W as [K, N] needs 16-byte aligned operands", name);
  const size_t mbytes = sizeof(CUtensorMap) * maps.size();
  const size_t pbytes = align16(sizeof(supra::LinProb) * n);
  const size_t bbytes = sizeof(int32_t) * (n + 1);
  char *h = nullptr, *dv = nullptr;
  int rc = ring_reserve(c, 64 + mbytes + pbytes + bbytes, &h, &dv);
  if (rc) return rc;
  // tensor maps first, on a 64-byte boundary in device memory
  const size_t pad = (64 - (reinterpret_cast<uintptr_t>(dv) & 63)) & 63;
  char* hm = h + pad;
  char* dm = dv + pad;
  if (mbytes) std::memcpy(hm, maps.data(), mbytes);
  std::memcpy(hm + mbytes, lp.data(), sizeof(supra::LinProb) * n);
  std::memcpy(hm + mbytes + pbytes, begin.data(), bbytes);
  rc = ring_commit(c, h, dv, pad + mbytes + pbytes + bbytes);
  if (rc) return rc;
  supra::LinLaunch L;
  L.maps = reinterpret_cast<const CUtensorMap*>(dm);
  L.probs = reinterpret_cast<const supra::LinProb*>(dm + mbytes);
  L.begin = reinterpret_cast<const int32_t*>(dm + mbytes + pbytes);
  L.n = n;
  L.total = (int32_t)total;
  L.status = c->d_status;
  cudaError_t e;
  {
    ProfScope ps(c, name, flops, bytes);
    e = tma ? supra::launch_linear_fp32_tma(bias, cols, w_kn, L, c->stream)
            : supra::launch_linear_fp32(bias, false, cols, L, c->stream);
  }
  if (e != cudaSuccess) return cuda_err(c, e, name);
  c->launches += 1;
  return SUPRA_ATTN_OK;
}

int flush_linear(supra_attn_ctx* c, std::vector<const Queued*>& g) {
  const int n = (int)g.size();
  std::vector<supra::LinProb> lp((size_t)n);
  double flops = 0, bytes = 0;
  for (int i = 0; i < n; ++i) {
    lp[i] = g[i]->lin;
    flops += g[i]->flops;
    bytes += g[i]->bytes;
  }
  const int cols = linear_tile_cols(lp);
  // A normalised x read by two or more column tiles is normalised once, into the context's split
  // buffer ([M, K] dense), by a launch between its statistics and the product (which then reads it
  // plainly): the prologue would normalise every x tile again for every column tile (the DiT
  // block's qkv, N = 1728: 27 times). x of such problems is 16-byte aligned with K % 4 == 0.
  std::vector<int64_t> xn((size_t)n, -1);  // offset of the normalised x in lin_split, or -1
  size_t xn_need = 0;
  for (int i = 0; i < n; ++i) {
    const int n_tiles = (lp[i].N + cols - 1) / cols;
    if (lp[i].gn_rows > 0 && n_tiles >= 2 && lp[i].K % 4 == 0 && (lp[i].ldx & 3) == 0 && aligned16(lp[i].x)) {
      xn[i] = (int64_t)xn_need;
      xn_need += align16((size_t)lp[i].M * lp[i].K * sizeof(float)) / sizeof(float);
    }
  }
  if (xn_need) {
    const int rc0 = grow_buffer(c, reinterpret_cast<void**>(&c->lin_split), &c->lin_split_cap, xn_need, sizeof(float),
                                "normalised x");
    if (rc0) return rc0;
  }
  int rc = norm_stats(c, g, lp.data());
  if (rc) return rc;
  for (int i = 0; i < n; ++i) {
    if (xn[i] < 0) continue;
    float* dst = c->lin_split + xn[i];
    cudaError_t e;
    {
      ProfScope ps(c, "norm_apply", 0.0, 8.0 * (double)lp[i].M * lp[i].K);
      e = supra::launch_norm_apply(lp[i], dst, c->stream);
    }
    if (e != cudaSuccess) return cuda_err(c, e, "norm_apply");
    c->launches += 1;
    lp[i].x = dst;
    lp[i].ldx = lp[i].K;
    lp[i].gn_stats = nullptr;  // the product reads x as it is
  }
  return run_linear_fp32(c, lp, g[0]->bias, g[0]->aligned, flops, bytes, g[0]->bias ? "linear_fp32_bias" : "linear_fp32");
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
  ++c->map_epoch;
  auto map_of = [&](const float* b, int64_t ld, int64_t rows, int64_t cols, int32_t* out, int32_t box_rows = 128) -> int {
    const MapKey k{reinterpret_cast<uintptr_t>(b), ld, rows, cols, 32, box_rows, (int32_t)CU_TENSOR_MAP_SWIZZLE_128B, 0};
    return map_slot(c, k, maps, out);
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
    S.trans_jobs = 0;
    for (const supra::SplitJob& J : sj) S.trans_jobs += J.trans ? 1 : 0;
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

}  // namespace rt
}  // namespace supra
