// libsupra_attn host runtime: the attention groups of a flush (block kernels, the score-materialising
// path for head dims above 128, and the TMA-fed persistent FP32 and tensor-core kernels).
#include "runtime.h"

namespace supra {
namespace rt {

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
  // FFMA score kernels: query rows per tile. A chunk with fewer Q K^T tiles of 128 rows than SMs
  // (one VAE image: 8 x 8) takes 64- or 32-row tiles, so that every SM has work.
  int bm = 128;
  if (!tc) {
    const int sms = supra::attn_fp32_warp_cta_slots() / 2;
    auto qk_tiles = [&](int rows_per_tile) {
      int64_t n = 0;
      for (const GemmUnit& u : units)
        n += (int64_t)((u.rows + rows_per_tile - 1) / rows_per_tile) * ((g[u.prob]->p.Lk + 127) / 128);
      return n;
    };
    while (bm > 32 && qk_tiles(bm) < sms) bm /= 2;
  }
  // FFMA path: with enough 128 x 128 score tiles to fill two CTAs per SM, S = Q K^T runs on the
  // FFMA linear (TMA-staged, packed FMAs; the VAE at 8 or more images) rather than the score kernel
  // and O = P V too (W = V read as [Lk, D]) when its 128 x 64 tiles fill them
  bool lin_qk = false, lin_pv = false;
  if (!tc && !bias && aligned) {
    int64_t t = 0, tv = 0;
    for (const GemmUnit& u : units) {
      t += (int64_t)((u.rows + 127) / 128) * ((g[u.prob]->p.Lk + 127) / 128);
      tv += (int64_t)((u.rows + 127) / 128) * ((g[u.prob]->p.D + 63) / 64);
    }
    lin_qk = t >= supra::attn_fp32_warp_cta_slots();
    lin_pv = tv >= supra::attn_fp32_warp_cta_slots();
  }
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
    const int rt = (u.rows + bm - 1) / bm;
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
  L.sm_scale = (tc || lin_qk) ? 1 : 0;
  L.bm = bm;
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
  } else if (lin_qk) {
    // the same products on the FFMA linear, unscaled (the softmax applies the scale)
    std::vector<supra::LinProb> lps((size_t)nu);
    for (int i = 0; i < nu; ++i) {
      const GemmUnit& u = units[i];
      const AttnProb& P = g[u.prob]->p;
      supra::LinProb& lp = lps[i];
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
    }
    rc = run_linear_fp32(c, lps, false, true, fl, by_qk, "attn_gemm_qk_lin");
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
  } else if (lin_pv) {
    // O_h rows = P V_h on the FFMA linear with W = V_h as [Lk, D] (read in place)
    std::vector<supra::LinProb> lps((size_t)nu);
    for (int i = 0; i < nu; ++i) {
      const GemmUnit& u = units[i];
      const AttnProb& P = g[u.prob]->p;
      supra::LinProb& lp = lps[i];
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
    }
    rc = run_linear_fp32(c, lps, false, true, fl, by_pv, "attn_gemm_pv_lin", true);
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
// kernels): one tensor map per distinct (buffer, ld, rows, box), encoded once per context and
// kept in the context's device table of maps; problems refer to maps by their slot there, and
// a flush stages only the maps that are new to the table (a batch of separate per-prompt
// buffers reuses its maps call after call).
int flush_tma(supra_attn_ctx* c, std::vector<const Queued*>& g, bool tf32) {
  // Unbiased FP32 launches with at least one 256-row tile per SM that lose little to the larger
  // tile (query rows rounded up to 256 at most 1/8 more than rounded up to 128) run on the
  // 256-row kernel (8x8 register blocks, one CTA per SM); the others on the 128-row kernel. (Past
  // one tile per SM both kernels quantise alike: n 256-row tiles on 148 CTAs against 2n 128-row
  // tiles on 296.)
  bool wide = false;
  if (!tf32 && !g[0]->bias) {
    const int64_t wr = supra::attn_fp32_wide_tile_rows(), nr = supra::attn_fp32_warp_tile_rows();
    int64_t tiles = 0, rows_w = 0, rows_n = 0;
    for (const Queued* q : g) {
      const int64_t tw = (q->p.Lq + wr - 1) / wr;
      tiles += tw * q->p.H;
      rows_w += tw * wr * q->p.H;
      rows_n += (q->p.Lq + nr - 1) / nr * nr * q->p.H;
    }
    wide = tiles >= (int64_t)supra::attn_fp32_wide_ctas() && 8 * rows_w <= 9 * rows_n;
  }
  const int mrows = tf32 ? supra::attn_tf32_tile_rows()
                    : wide ? supra::attn_fp32_wide_tile_rows()
                           : supra::attn_fp32_warp_tile_rows();
  // the split kernel needs the operands exactly: fp32 maps with the tensor-core swizzles
  const bool split = tf32 && g[0]->cfg == 1;
  std::stable_sort(g.begin(), g.end(), [](const Queued* a, const Queued* b) { return a->p.Lk > b->p.Lk; });
  const int n = (int)g.size();
  std::vector<supra::TmaProb> probs((size_t)n);
  {
    const int rm = map_table_reserve(c, 4 * (size_t)n);  // (at most four maps per problem)
    if (rm) return rm;
  }
  const int32_t fresh0 = c->map_table_used;
  std::vector<const CUtensorMap*> fresh;  // maps new to the table, slots fresh0, fresh0 + 1, ...
  // Slots handed out below hold their maps only once the staging copy is on the stream: a return
  // before that starts the table over, so no later launch reads a slot that was never written.
  struct TableGuard {
    supra_attn_ctx* c;
    bool armed;
    ~TableGuard() {
      if (armed) {
        ++c->map_table_epoch;
        c->map_table_used = 0;
      }
    }
  } table_guard{c, true};
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
    const int rc = map_table_slot(c, k, fresh, out);
    if (rc) return rc;
    last_key = k;
    last_idx = *out;
    return SUPRA_ATTN_OK;
  };
  // Key splits (persistent FP32 kernel): a launch with at most half as many (head, query tile)
  // groups as the device has SMs (the DiT self-attention of one image pair: 36 groups) splits
  // each group's key blocks over up to 8 tiles, about one tile per SM; the splits' partial rows
  // are combined in the kernel. (One tile per SM runs each tile's warps alone on their
  // schedulers, and fewer splits leave fewer partial rows to combine.)
  int ns_max = 1;
  int64_t groups = 0;
  if (!tf32 && !wide) {
    for (int i = 0; i < n; ++i) groups += (int64_t)((g[i]->p.Lq + mrows - 1) / mrows) * g[i]->p.H;
    const int sms = supra::attn_fp32_warp_cta_slots() / 2;
    if (groups > 0 && 2 * groups <= sms) ns_max = (int)std::min<int64_t>(8, sms / groups);
  }
  std::vector<int32_t> begin(n + 1);
  int64_t total = 0, group0 = 0;
  int used_splits = 1;
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
    // output rows by TMA stores (256-row kernel): one map over the whole output buffer, when the
    // problem's rows are whole rows of it
    t.mo = -1;
    if (!rc && wide && aligned16(P.o) && P.o_off % P.ldo == 0 && P.o_off / P.ldo + P.Lq <= q.rows_o &&
        q.rows_o <= INT32_MAX) {
      rc = map_index(P.o, P.ldo, q.rows_o, 64, 32, CU_TENSOR_MAP_SWIZZLE_NONE, &t.mo);
      t.oy = (int32_t)(P.o_off / P.ldo);
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
    const int nb = (P.Lk + supra::kFwBoxRows - 1) / supra::kFwBoxRows;
    t.bps = std::max(1, (nb + ns_max - 1) / ns_max);
    t.splits = (nb + t.bps - 1) / t.bps;  // every split has at least one key block
    t.group0 = (int32_t)group0;
    used_splits = std::max(used_splits, (int)t.splits);
    begin[i] = (int32_t)total;
    group0 += (int64_t)t.q_tiles * P.H;
    total += (int64_t)t.q_tiles * P.H * t.splits;
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
  const size_t fbytes = sizeof(CUtensorMap) * fresh.size();
  const size_t bbytes = align16(sizeof(int32_t) * (n + 1));
  // the launch's tile counter and, with key splits, one counter per (group, warp), staged as zero
  const size_t cbytes = 16 + (used_splits > 1 ? align16(sizeof(int32_t) * 4 * (size_t)group0) : 0);
  if (used_splits > 1) {  // partial rows: 128 rows x (64 O columns + offset and sum) per split
    const int rc0 = ensure_scratch(c, (size_t)group0 * used_splits * mrows * (64 + 2) * sizeof(float));
    if (rc0) return rc0;
  }
  // The FP32 kernel with a T5 table reads the bias by relative position: per distinct (table,
  // bucket LUT, H) one [H, 2 rel_max + 1] array, formed on the device (rel_bias_kernel) in the
  // ring space past the staged bytes, before the launch.
  struct RelBias {
    const float* table;
    int64_t loff;
    int32_t H, rel_max;
    size_t off;
  };
  std::vector<RelBias> rb;
  std::vector<int32_t> rb_of((size_t)n, -1);
  size_t rbytes = 0;
  if (!tf32) {
    for (int i = 0; i < n; ++i) {
      if (loff[i] < 0) continue;
      const AttnProb& P = g[i]->p;
      int k = 0;
      for (; k < (int)rb.size(); ++k)
        if (rb[k].table == P.bias && rb[k].loff == loff[i] && rb[k].H == P.H && rb[k].rel_max == P.rel_max) break;
      if (k == (int)rb.size()) {
        rb.push_back(RelBias{P.bias, loff[i], P.H, P.rel_max, rbytes});
        rbytes += align16(sizeof(float) * (size_t)P.H * (2 * (size_t)P.rel_max + 1));
      }
      rb_of[i] = k;
    }
  }
  // ring: problems | bucket LUTs | tile prefixes | counters (staged), then the relative-bias
  // arrays (device only) and the new maps (host only: staged into their table slots)
  const size_t staged = pbytes + lbytes + bbytes + cbytes;
  char *h = nullptr, *dv = nullptr;
  int rc = ring_reserve(c, staged + rbytes + fbytes, &h, &dv);
  if (rc) return rc;
  for (int i = 0; i < n; ++i) {
    probs[i].rel_lut = loff[i] < 0 ? nullptr : reinterpret_cast<const int32_t*>(dv + pbytes) + loff[i];
    if (rb_of[i] >= 0) probs[i].bias = reinterpret_cast<const float*>(dv + staged + rb[rb_of[i]].off);
  }
  std::memcpy(h, probs.data(), sizeof(supra::TmaProb) * n);
  if (!lut.empty()) std::memcpy(h + pbytes, lut.data(), lut.size() * sizeof(int32_t));
  std::memcpy(h + pbytes + lbytes, begin.data(), sizeof(int32_t) * (n + 1));
  std::memset(h + pbytes + lbytes + bbytes, 0, cbytes);
  if (fbytes) {  // the new maps into their table slots (ordered before the launch by the stream)
    char* hf = h + staged + rbytes;
    for (size_t i = 0; i < fresh.size(); ++i) std::memcpy(hf + i * sizeof(CUtensorMap), fresh[i], sizeof(CUtensorMap));
    const cudaError_t ef = supra::launch_stage_copy(c->ring_hd + (hf - c->ring_h), c->map_table + fresh0, fbytes,
                                                    c->stream);
    if (ef != cudaSuccess) return cuda_err(c, ef, "map table: stage");
    c->launches += 1;
  }
  table_guard.armed = false;
  rc = ring_commit(c, h, dv, staged);  // (its event, recorded after both copies, frees the ring half)
  if (rc) return rc;
  for (const RelBias& r : rb) {
    const cudaError_t e0 = supra::launch_rel_bias(r.table, reinterpret_cast<const int32_t*>(dv + pbytes) + r.loff,
                                                  r.H, r.rel_max, reinterpret_cast<float*>(dv + staged + r.off), c->stream);
    if (e0 != cudaSuccess) return cuda_err(c, e0, "rel_bias");
    c->launches += 1;
  }
  supra::TmaLaunch L;
  L.next_tile = reinterpret_cast<int32_t*>(dv + pbytes + lbytes + bbytes);
  L.maps = c->map_table;
  L.probs = reinterpret_cast<const supra::TmaProb*>(dv);
  L.begin = reinterpret_cast<const int32_t*>(dv + pbytes + lbytes);
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
  if (used_splits > 1) {
    L.part_splits = used_splits;
    L.part_o = c->scratch;
    L.part_ml = reinterpret_cast<float2*>(c->scratch + (size_t)group0 * used_splits * mrows * 64);
    L.part_cnt = L.next_tile + 4;  // (16 bytes past the tile counter)
  }
  const char* name = wide    ? "attn_fp32_d64_wide"
                     : !tf32  ? (g[0]->bias ? "attn_fp32_d64_tma_bias" : "attn_fp32_d64_tma")
                     : split ? (g[0]->bias ? "attn_tf32x3_d64_bias" : "attn_tf32x3_d64")
                             : (g[0]->bias ? "attn_tf32_d64_bias" : "attn_tf32_d64");
  cudaError_t e;
  {
    ProfScope ps(c, name, flops, bytes);
    e = tf32   ? supra::launch_attn_tf32(L, g[0]->bias, split, c->stream)
        : wide ? supra::launch_attn_fp32_wide(L, c->stream)
               : supra::launch_attn_fp32_warp(L, g[0]->bias, c->stream);
  }
  if (e != cudaSuccess) return cuda_err(c, e, name);
  c->launches += 1;
  return SUPRA_ATTN_OK;
}

}  // namespace rt
}  // namespace supra
