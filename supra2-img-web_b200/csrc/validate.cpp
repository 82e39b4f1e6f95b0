// libsupra_attn host runtime: argument checks of the attention descriptor (the operator surface of
// app/gpu/ops.js:103-149) and of the linear descriptor (ops.linear, app/gpu/ops.js:35-43).
#include "runtime.h"

namespace supra {
namespace rt {

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
  q.rows_o = HD > 0 ? d->out_size / HD : 0;
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
  q.rows_q = q.rows_k = q.rows_v = q.rows_o = 0;
  q.flops = 2.0 * d->M * (double)d->N * d->K;
  q.bytes = 4.0 * ((double)d->M * d->K + (double)d->N * d->K + (double)d->M * d->N + (d->bias ? d->N : 0) +
                   (d->resid ? (double)d->M * d->N : 0.0) + ((gn || (ln && ln->mod)) ? 2.0 * d->K : 0.0) +
                   (d->gate ? d->N : 0));
  return SUPRA_ATTN_OK;
}

}  // namespace rt
}  // namespace supra
