// Quantisation prologue: argument block and launchers.
#pragma once

#include "internal.cuh"

namespace scmp {

enum QuantRecipe {
  Q_TENSOR_BIP = 0,   // fused_quant_kernel flat bipolar         (quant/fused.py:86-112)
  Q_TENSOR_UNI = 1,   // fused_quant_kernel per-row unipolar     (quant/fused.py:82-84, 113-121)
  Q_GROUP_SYM = 2,    // _grouped_symmetric_quant + boundary     (quant/grouped.py:13-75, sc/kernels.py:1679)
  Q_GROUP_ASYM = 3,   // _grouped_asymmetric_quant + boundary    (quant/grouped.py:78-133, sc/kernels.py:1685)
  Q_BATCH_SYM = 4,    // _grouped_symmetric_quant_batched        (quant/grouped.py:136-163, sc/kernels.py:1864)
  Q_ROWCHUNK_BIP = 5, // fused_quantize_bipolar_perrow per chunk (quant/fused.py:134-159, sc/kernels.py:1342-1347)
  Q_HEAD_BIP = 6      // fused_quant_bipolar_batched_kernel      (quant/fused.py:237-283)
};

enum GroupRecipe { GP_SYM = 0, GP_ASYM = 1, GP_HEAD = 2 };

// Grid of one row level: boundary scale, grid, table (operand a's k-table).
struct LevelQ {
  float ratio;          // fl32(G / q) of the multiply-form boundary
  int G;                // grid levels of the divide-form boundary
  int vcap;
  const int16_t* ktab;  // operand a: boundary -> k, or NULL
  const int32_t* amap;
};

struct QuantArgs {
  const float* x;  // (rows, d) float32, rows = batch * rows_per_batch
  int rows, d, rows_per_batch;
  int vec;         // x is 16-byte aligned and d % 4 == 0 (rows read as float4)
  const float* smooth;  // (d,) or NULL
  int smooth_div;       // 1: x / s (operand a), 0: x * s (operand b)
  int q;                // q_max
  float qmin;           // lower clamp of the bipolar recipes (-q, or -(q+1) per head)
  float ratio;          // fl32(G / q) of the multiply-form boundary
  int G;                // grid levels of the divide-form boundary
  // per-row parameters
  int self_stats;       // G == 1 row recipes compute their own scale
  float* row_scale;     // (rows,)  written when self_stats, else read
  float* row_zp;        // (rows,)
  const float* params;  // Q_TENSOR_*: scalar block; Q_HEAD_BIP: per-batch inverse scale
  int param_off;        // Q_TENSOR_*: index of this operand's inverse scale in params
  int chunk_d;          // Q_ROWCHUNK_BIP
  float* chunk_scale;   // (nchunks, rows)
  // outputs
  int16_t* out16;       // blocked [ceil(d/8)][rows][8] (internal.cuh: blk_idx)
  const int16_t* ktab;  // non-NULL for operand a: map boundary -> k
  const int32_t* amap;
  int vcap;
  float* row_sum;       // (rows,) unipolar, or NULL
  // Row levels (operand a): row i of the output is row row_of[i] of x (-1:
  // padding, written as zeros), quantised on the grid of its level, the level
  // whose rows [256 * lev_tile0[l], 256 * lev_tile0[l + 1]) hold i.
  const int* row_of;
  const int* lev_tile0;
  int nlev;
  LevelQ lq[kMaxLevels];
};

cudaError_t launch_row_stats(const QuantArgs& q, float* stats, cudaStream_t st);
cudaError_t launch_group_params(const float* stats, int batch, int rpb, int G, int q, int recipe,
                                float* scale, float* zp, cudaStream_t st);
// Per batch entry (rows_per_batch rows of q.x): scale and its inverse of the
// per_head recipe, in one pass.
cudaError_t launch_head_params(const QuantArgs& q, int batch, int q_max, float* scale, float* inv,
                               cudaStream_t st);
cudaError_t launch_tensor_params(const float* sa, int ra, const float* sb, int rb, int d, int q,
                                 int unipolar, const double* ranges, float* scal, cudaStream_t st);
cudaError_t launch_quant_rows(int recipe, const QuantArgs& q, cudaStream_t st);
// Permutation of a's rows by level (rows of one level in increasing order,
// every level padded to whole 256-row tiles): row_of (n_pad entries) and
// lev_tile0 (nlev + 1 entries) on the device, from row_level (n,).
cudaError_t launch_level_perm(const int32_t* row_level, int n, int nlev, int n_pad, int* row_of, int* lev_tile0,
                              cudaStream_t st);

}  // namespace scmp
