// Internal interface between the host runtime (supra_attn.cpp) and the CUDA kernels.
// Plain structs that the host packs into the descriptor ring and the kernels read from HBM.
#pragma once

#include <cuda.h>  // CUtensorMap (the library calls the driver only through cudaGetDriverEntryPoint)
#include <cuda_runtime.h>
#include <stdint.h>

namespace supra {

// Device status codes written to the context's status word (status[0]).
enum DevStatus : int32_t {
  DEV_OK = 0,
  DEV_TIMEOUT = 1,   // a bounded mbarrier / copy wait ran out
  DEV_BAD_TILE = 2,  // a tile index outside the launch's problem list
};

// One attention problem (all heads of one ops.attention call) as the fused kernels see it.
// Element offsets already include the caller's qOff/kOff/vOff/oOff; head h adds h*D.
struct alignas(16) AttnProb {
  const float* q;
  const float* k;
  const float* v;
  float* o;
  const float* bias;  // [H, Lq, Lk] or nullptr
  int64_t q_off, k_off, v_off, o_off;
  int64_t ldq, ldk, ldv, ldo;
  int32_t Lq, Lk, H, D;
  float scale;       // score multiplier
  float scale_log2;  // scale * log2(e): scores are exponentiated with exp2
  int32_t q_tiles;   // ceil(Lq / tile rows)
  int32_t rel_max;   // T5 table bias: relative positions are clamped to [-rel_max, rel_max]
  const int32_t* rel_lut;  // T5 table bias: bucket of relative position r at rel_lut[r + rel_max]
                           // (bias is then the [buckets, H] table); nullptr: bias is [H, Lq, Lk]
};
static_assert(sizeof(AttnProb) % 16 == 0, "AttnProb is packed into the descriptor ring");

// A grouped launch: `n` problems, tile t belongs to the problem p with begin[p] <= t < begin[p+1].
struct AttnLaunch {
  const AttnProb* probs;
  const int32_t* begin;  // n + 1 entries, begin[n] = total tiles
  int32_t n;
  int32_t total;
  int32_t* status;
  int32_t uniform;  // > 0: every problem has this many tiles (tile -> problem by division)
  int32_t pad;
};

// One (problem, head, row chunk) unit of the score-materialising path used for D > 128: the
// scores of `rows` query rows starting at row0 live in scratch at s_off with row stride ldS.
struct alignas(16) GemmUnit {
  int64_t s_off;
  int32_t prob, h, row0, rows;
  int32_t ldS;
  int32_t qk_begin;  // prefix of QK^T tiles
  int32_t pv_begin;  // prefix of PV tiles
  int32_t row_begin; // prefix of softmax rows
};
static_assert(sizeof(GemmUnit) % 16 == 0, "GemmUnit is packed into the descriptor ring");

struct GemmLaunch {
  const AttnProb* probs;
  const GemmUnit* units;
  const int32_t* qk_begin;  // n_units + 1
  const int32_t* pv_begin;  // n_units + 1
  const int32_t* row_begin; // n_units + 1
  float* scratch;
  // The row softmax for the tensor-core products: with sm_scale it applies each problem's scale
  // (the scores come unscaled); with lo set it writes the probabilities split, hi in place and
  // lo at the same offset from lo (the operand of the split-precision P V).
  float* lo = nullptr;
  int32_t sm_scale = 0;
  int32_t bm = 128;  // query rows per tile of the FFMA score kernels: 128, 64 or 32 (qk/pv prefixes count those)
  int32_t n_units;
  int32_t qk_total, pv_total, row_total;
  int32_t* status;
};

// Fused FP32 kernel configurations (head-dim capacity DT, query rows per CTA MQ).
enum FusedCfg : int32_t {
  CFG_D64_Q128 = 0,
  CFG_D64_Q64 = 1,
  CFG_D128_Q64 = 2,
  CFG_COUNT = 3,
};
int fused_cfg_tile_rows(int cfg);
int fused_cfg_head_dim(int cfg);

// Launchers. Each returns the cudaError_t of the launch (cudaSuccess on success).
// bias_mode: 0 none, 1 an expanded [H, Lq, Lk] bias, 2 a T5 relative-bias table (AttnProb::rel_lut)
cudaError_t launch_attn_fp32(int cfg, int bias_mode, bool aligned, const AttnLaunch& L, cudaStream_t s);
const char* attn_fp32_name(int cfg, int bias_mode, bool aligned);

cudaError_t launch_gemm_qk(bool bias, bool aligned, const GemmLaunch& L, cudaStream_t s);
cudaError_t launch_softmax_rows(const GemmLaunch& L, cudaStream_t s);
cudaError_t launch_gemm_pv(bool aligned, const GemmLaunch& L, cudaStream_t s);

// Problems read through TMA tensor maps (the TF32 tensor-core kernel, attn_tf32.cu, and the
// persistent FP32 kernel, attn_fp32_warp.cu): one problem with its tensor-map indices and the
// TMA coordinates (x = column, y = row) of head 0 / row 0 of each operand.
struct alignas(16) TmaProb {
  float* o;
  int64_t o_off;
  int64_t ldo;
  // [H, Lq, Lk] additive score bias, or nullptr; with rel_lut set, the T5 [buckets, H] table (the
  // TF32 kernels) or the [H, 2 rel_max + 1] bias by relative position (the 128-row FP32 kernel)
  const float* bias;
  int32_t Lq, Lk, H, D;
  int32_t mq, mk, mv;
  int32_t qx, qy, kx, ky, vx, vy;
  float scale_log2;
  int32_t q_tiles;
  const int32_t* rel_lut;  // T5 table bias (as AttnProb): bias is then the [buckets, H] table
  int32_t rel_max;
  // Key splits (persistent FP32 kernel only; 1 elsewhere): each (head, query tile) group of the
  // problem is `splits` tiles, split s covering key blocks [s * bps, min((s + 1) * bps, blocks)),
  // every split at least one block. The group's partial results meet in TmaLaunch::part_o /
  // part_ml at group index group0 + h * q_tiles + query tile.
  int32_t splits;
  int32_t bps;
  int32_t group0;
  // The 256-row FP32 kernel: tensor map of the whole output buffer as [rows, H*D] (boxes of 64
  // columns x 32 rows) and the problem's first output row in it, for TMA stores of whole 32-row
  // blocks; mo = -1: plain stores only.
  int32_t mo;
  int32_t oy;
};
static_assert(sizeof(TmaProb) % 16 == 0, "TmaProb is packed into the descriptor ring");

struct TmaLaunch {
  const TmaProb* probs;
  const CUtensorMap* maps;
  const int32_t* begin;
  int32_t n, total, uniform;
  int32_t* status;
  // Tiles past the first gridDim.x are handed out by this counter (zero at launch, one per
  // launch, in the staged descriptor block): the persistent FP32 kernel's CTAs claim them one at
  // a time, so CTAs that share an SM and progress at different rates finish together.
  int32_t* next_tile = nullptr;
  // Key splits (TmaProb::splits > 1), persistent FP32 kernel: split s of group g writes its
  // unnormalised O rows to part_o[((g * part_splits + s) * tile rows + row) * 64 + col] and the
  // row's (exp2 offset, sum) to part_ml[(g * part_splits + s) * tile rows + row]; part_cnt holds one
  // counter per (group, warp), zero at launch, and the last split of a warp's rows to arrive
  // combines them.
  float* part_o = nullptr;
  float2* part_ml = nullptr;
  int32_t* part_cnt = nullptr;
  int32_t part_splits = 0;
};

cudaError_t launch_attn_tf32(const TmaLaunch& L, bool bias, bool split, cudaStream_t s);
int attn_tf32_tile_rows();

// Persistent FP32 kernel (attn_fp32_warp.cu): D = 64, scale > 0, optional score bias (expanded
// or the T5 table, as TmaProb describes it). Q and K tensor maps
// have boxes of kFwBoxWide columns x 32 rows, V maps kFwBoxNarrow columns x 32 rows (fp32, no
// swizzle): the 4 extra Q/K columns pad the shared-memory rows against bank conflicts.
constexpr int kFwBoxWide = 68;
constexpr int kFwBoxNarrow = 64;
constexpr int kFwBoxRows = 32;
cudaError_t launch_attn_fp32_warp(const TmaLaunch& L, bool bias, cudaStream_t s);
int attn_fp32_warp_tile_rows();
int attn_fp32_warp_cta_slots();  // CTAs the persistent grid holds at most (two per SM)

// Persistent FP32 kernel for large unbiased launches (attn_fp32_wide.cu): D = 64, scale > 0, no
// bias; 256-row tiles (TmaProb::q_tiles counts those), no key splits, the same tensor maps as
// attn_fp32_warp.cu. One CTA per SM.
cudaError_t launch_attn_fp32_wide(const TmaLaunch& L, cudaStream_t s);
int attn_fp32_wide_tile_rows();
int attn_fp32_wide_ctas();

// Normalisation of x in the linear prologue (LinProb::gn_mode): GroupNorm with gamma/beta,
// LayerNorm with adaLN modulation (gamma = scale, beta = shift, applied as 1 + scale), plain
// LayerNorm.
constexpr int kNormAffine = 0, kNormModulated = 1, kNormPlain = 2;
// Activation in the linear epilogue (LinProb::act), the values of SUPRA_ATTN_ACT_*.
constexpr int kActNone = 0, kActGelu = 1, kActGeluTanh = 2, kActSilu = 3;

// Columns of the x and W tensor-map boxes of the TMA-staged FFMA linear: 32 of K per stage plus 4
// that pad the shared-memory rows.
constexpr int kLinBoxCols = 36;

// y = x W^T (+ bias) for one ops.linear call (app/gpu/ops.js:35-43), linear_fp32.cu. x rows of
// stride ldx (the caller's x offset already applied), W [N, K] row-major with row stride ldw,
// y rows of stride ldy (offset applied).
struct alignas(16) LinProb {
  const float* x;
  const float* w;
  const float* bias;  // [N] or nullptr
  float* y;
  int64_t ldx, ldw, ldy;
  int32_t M, N, K;
  int32_t n_tiles;  // column tiles: ceil(N / tile columns) (128 or 64, the FFMA kernel; 128 elsewhere)
  const float* resid;  // y = resid[row * ldr + col] + ..., or nullptr (may be y itself)
  int64_t ldr;
  const float* gate;   // the product is scaled by gate[col] (offset applied), or nullptr
  int32_t gn_mode;     // normalisation of x: kNormAffine, kNormModulated or kNormPlain
  int32_t act;         // activation of x W^T + bias: kActNone, kActGelu, kActGeluTanh, kActSilu
  // normalisation of x on the way in (gn_stats != nullptr): stats[image * groups + g] = (mean,
  // rstd); a LayerNorm is one image per row and one group
  const float2* gn_stats;
  const float* gamma;
  const float* beta;
  int32_t gn_cg;     // channels per group
  int32_t gn_rows;   // rows per image
  int32_t gn_groups;
  int32_t gn_silu;
  int32_t mx, mw;    // the TMA-staged FFMA kernel: tensor maps of x ([M, K], boxes kLinBoxCols x 128)
                     // and W ([N, K], boxes kLinBoxCols x tile columns; with w_kn, [K, N] in boxes
                     // of tile columns x 32) in LinLaunch::maps; unused elsewhere
  int32_t w_kn;      // the TMA-staged FFMA kernel: W is stored [K, N] (row stride ldw along N), as
                     // V is for O = P V; every problem of a launch alike
  int32_t pad_;
};
static_assert(sizeof(LinProb) % 16 == 0, "LinProb is packed into the descriptor ring");

// A grouped linear launch: tile t (a 128x128 block of one problem's y) belongs to the problem p
// with begin[p] <= t < begin[p+1]; within a problem, row tiles outer, column tiles inner.
struct LinLaunch {
  const LinProb* probs;
  const int32_t* begin;
  int32_t n, total;
  int32_t* status;
  const CUtensorMap* maps = nullptr;  // the TMA-staged form's tensor maps
};
// tile_cols: 128 or 64 columns per 128-row tile (LinProb::n_tiles counts tiles of that width)
cudaError_t launch_linear_fp32(bool bias, bool aligned, int tile_cols, const LinLaunch& L, cudaStream_t s);
// The same with the x and W tiles staged by TMA tensor copies (x and W 16-byte aligned, row strides
// of a multiple of 4 floats; LinProb::mx / mw index L.maps).
cudaError_t launch_linear_fp32_tma(bool bias, int tile_cols, bool w_kn, const LinLaunch& L, cudaStream_t s);
// GroupNorm statistics of x [images * rows_per_image, K] (contiguous rows): for every image and
// group of K / groups channels, (mean, 1 / sqrt(var + eps)) with the variance taken around the
// mean in a second pass (app/gpu/kernels.js:117-139).
// Linear on the tensor cores (linear_tc.cu) for the TF32 / TF32X3 variants: x and w are read
// through tensor maps, either in place (TF32: the tensor core ignores the 13 low mantissa bits, so
// a 16-byte aligned fp32 operand is its own TF32 part) or from dense [rows, ldk] arrays (ldk = K
// rounded up to 4) written by launch_split, hi = the value with its 13 low mantissa bits cleared
// and lo = value - hi; the product is then hi(x) hi(w) (TF32) or lo(x) hi(w) + hi(x) lo(w) +
// hi(x) hi(w) (TF32X3) on tcgen05, with p's epilogue (bias, activation, gate, residual). x and w
// in p are unused.
struct alignas(16) LinTcProb {
  LinProb p;
  int32_t mxh, mxl, mwh, mwl;  // tensor maps of hi(x), lo(x), hi(w), lo(w) (lo: split form only)
  int32_t m_tiles, n_tiles;    // 128-row and 128-column output tiles
  int32_t nkb;                 // 32-deep k-blocks: ceil(K / 32)
  int32_t my;                  // tensor map of y (32 x 32 boxes, TMA stores), or -1: per-row stores
};
static_assert(sizeof(LinTcProb) % 16 == 0, "LinTcProb is packed into the descriptor ring");
struct LinTcLaunch {
  const LinTcProb* probs;
  const CUtensorMap* maps;
  const int32_t* begin;  // first tile of each problem
  int32_t n, total;
  int32_t* status;
};
cudaError_t launch_linear_tc(const LinTcLaunch& L, bool split, cudaStream_t s);
constexpr int kSplitTileRows = 32, kSplitTileCols = 128;  // launch_split's tile
// One split job: rows x K floats of src (row stride ld; with trans read as [K, rows], element
// (r, k) at src[k * ld + r]) -> hi and lo, each written when non-null (an operand read in place
// as its own TF32 part needs only lo), dense with row stride ldd. Every value
// is multiplied by xscale, then by rowscale[r] when rowscale is set (w rows times a gate; then
// bias_out[r] = bias_in[r] * rowscale[r] too when bias_out is set), then normalised when gn_stats
// is set (LinProb's GroupNorm / LayerNorm fields of x rows). trans excludes rowscale and gn_stats.
struct alignas(16) SplitJob {
  const float* src;
  float* hi;
  float* lo;
  const float* rowscale;
  const float* bias_in;
  float* bias_out;
  const float2* gn_stats;
  const float* gamma;
  const float* beta;
  int64_t ld;
  int32_t rows, K, ldd, trans;
  int32_t gn_mode, gn_cg, gn_rows, gn_groups;
  int32_t gn_silu;
  float xscale;
  int32_t ktiles;  // k tiles: ceil(K / kSplitTileCols); the job has ceil(rows / kSplitTileRows) * ktiles
  int32_t pad_;
};
static_assert(sizeof(SplitJob) % 16 == 0, "SplitJob is packed into the descriptor ring");
struct SplitLaunch {
  const SplitJob* jobs;
  const int32_t* begin;  // first tile of each job
  int32_t n, total;
  int32_t trans_jobs;  // how many of the jobs are transposed (none: the kernel form without them)
};
// All jobs of one flush in one launch (32 x 128 tiles, HBM-bound).
cudaError_t launch_split(const SplitLaunch& L, cudaStream_t s);
cudaError_t launch_ln_stats(const float* x, int32_t K, int32_t rows, float eps, float2* stats, cudaStream_t s);
// P.x (rows of stride P.ldx) normalised as the linear's prologue would (P.gn_stats set, K % 4 == 0,
// 16-byte aligned rows) into dst as [M, K] dense.
cudaError_t launch_norm_apply(const LinProb& P, float* dst, cudaStream_t s);
cudaError_t launch_gn_stats(const float* x, int32_t K, int32_t rows_per_image, int32_t images, int32_t groups,
                            float eps, float2* stats, cudaStream_t s);

// Copies bytes (a multiple of 16, both addresses 16-byte aligned) from src, which may be pinned
// host memory addressable by the device, to device memory dst (stage.cu).
cudaError_t launch_stage_copy(const void* src, void* dst, size_t bytes, cudaStream_t s);

cudaError_t launch_position_bias(const float* table, const int32_t* lut, int32_t H, int32_t L,
                                 float* out, cudaStream_t s);
// [H, 2 rel_max + 1]: the T5 table bias by relative position (lut over rel = -rel_max .. rel_max)
cudaError_t launch_rel_bias(const float* table, const int32_t* lut, int32_t H, int32_t rel_max, float* out,
                            cudaStream_t s);

}  // namespace supra
