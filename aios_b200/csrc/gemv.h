// Decode-width linears on register-operand MMAs (gemv.cu), dispatched from the C-ABI
// linear entry points in gemm.cu for at most kMaxGemvRows token rows.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace aiosb {

// Token rows: up to 16 in one row group (decode), more as 16-row groups along
// grid y (prefill widths), up to kMaxGemvRows; rows above kGemvDefaultRows go to
// the tcgen05 GEMM unless AIOSB_GEMV_MAX_ROWS says otherwise. Measured per S10
// linear (us, GEMV / tcgen05): 32 rows 2.9 / 6.4-7.3, 64 rows 4.1 / 8.0-8.7,
// 128 rows 6.1 / 11.4-13.3, 512 rows 19.9 / 16.1-21.4, 2048 rows 78.9 / 27-35.
constexpr int kMaxGemvRows = 4096;
constexpr int kGemvDefaultRows = 512;
constexpr int kMaxGemvK = 2048;

struct GemvArgs {
  const __nv_bfloat16* x;  // [rows, k] bf16 operand rows (row stride x_stride), or NULL:
  int64_t x_stride;
  const float* stat_x;      // statistics mode: rows = bf16(stat_x * rcp * nw), rcp from the row itself
  const __nv_bfloat16* nw;
  float eps;
  const __nv_bfloat16* w;   // [n, k] weights
  int64_t n;                // weight rows
  int64_t n_out;            // output features (n, or n / 2 for SwiGLU)
  int64_t k;
  int rows;
  __nv_bfloat16* y;
  int64_t y_stride;
  int epilogue;
  const __nv_bfloat16* residual;
  int64_t residual_stride;
  float* out_stat_x;        // ADD: fp32 s [rows, n_out] and per-8-column sums of squares
  float* out_stat_ss;       // out_stat_ss[group * out_ss_stride + row], group = column / 8
  int64_t out_ss_stride;
  // mixer mode (mix_bank != NULL): the operand rows are rmsnorm(AttnRes mix of the
  // bank sources and the partial) * nw with eps, for rows <= 8 and k == 768
  const __nv_bfloat16* mix_bank;     // [mix_sources, mix_tokens, k]
  const __nv_bfloat16* mix_partial;  // [rows, k] or NULL
  const float* mix_wq;               // [k] fp32 routing query (key-norm weight folded in)
  float mix_eps;                     // the mixer's key-norm epsilon
  int mix_sources;                   // bank sources
  int mix_stable;                    // bank sources written before the previous kernel began
  int64_t mix_tokens;                // rows of one bank source
  // statistics operand and store epilogue, optional (tile_stats_eligible()): per
  // 16-column tile and row, (max, sum of exp(v - max), min, 1 if any NaN) of the
  // stored bf16 values, at tile_stats[tile * rows + row]
  float4* tile_stats;
  int early_dependents;  // launch the next kernel before the wait (as an ADD epilogue does)
};

// Mixer mode: at most this many sources (bank + partial), k of exactly kMixMaxK,
// and staged bank rows padded by kMixRowPad elements.
constexpr int kMixMaxSources = 10;
constexpr int kMixMaxK = 768;
constexpr int kMixRowPad = 32;
constexpr int kGemvPlain = 0, kGemvStat = 1, kGemvMix = 2, kGemvStatTiles = 3, kGemvPlainTiles = 4;  // operand modes
inline size_t mix_smem_bytes(int64_t stable, int64_t k) {
  return (size_t)stable * 8 * (size_t)(k + kMixRowPad) * 2 + (size_t)8 * 8 * kMixMaxSources * 2 * 4 +
         (size_t)8 * kMixMaxSources * 4;
}

// Columns per sum-of-squares part written by the GEMV residual epilogue.
constexpr int kGemvStatGroup = 8;

bool gemv_eligible(int64_t rows, int64_t k, int64_t n_out);
bool tile_stats_eligible(int64_t rows, int64_t k, int64_t n_out);  // GEMV, rows <= 16, k <= 768
bool mix_eligible(int64_t rows, int64_t k, int64_t n_out, int64_t sources, int64_t stable, bool partial);
int gemv_launch(const GemvArgs& a, cudaStream_t stream);

}  // namespace aiosb
