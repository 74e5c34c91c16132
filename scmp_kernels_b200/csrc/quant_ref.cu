// Quantisers with the reference's own output formats, for callers of the
// scmp_kernels.quant API (quant/fused.py, quant/grouped.py), and the
// enable-signal matmul on already-quantised operands (sc/kernels.py:798-868).
#include "quant.cuh"

namespace scmp {

// fused_quant_kernel, flat bipolar variant (quant/fused.py:86-112), optional
// transposed store of fused_quant_bipolar_batched_kernel (fused.py:275-283).
__global__ void ref_bipolar_kernel(const float* __restrict__ x, size_t slice, int rows, int cols,
                                   const float* __restrict__ inv_dev, float inv_host, int q,
                                   float qmin, float ratio, int transpose,
                                   int16_t* __restrict__ boundary, int8_t* __restrict__ sign) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= slice) return;
  const int bh = blockIdx.y;
  const float inv = inv_dev ? __ldg(inv_dev + bh) : inv_host;
  const float xc = fclamp(frint(fmul(__ldg(x + bh * slice + i), inv)), qmin, (float)q);
  const int8_t s = xc > 0.f ? 1 : (xc < 0.f ? -1 : 0);
  const int16_t b = (int16_t)frint(fmul(fabsf(xc), ratio));
  size_t o = i;
  if (transpose) o = (size_t)(i % cols) * rows + i / cols;
  boundary[bh * slice + o] = b;
  sign[bh * slice + o] = s;
}

// fused_quant_kernel per-row bipolar (fused.py:65-81): one warp per row.
__global__ void ref_bipolar_perrow_kernel(const float* __restrict__ x, int rows, int cols, int q,
                                          float ratio, int16_t* __restrict__ boundary,
                                          int8_t* __restrict__ sign, float* __restrict__ scale_row) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + (size_t)row * cols;
  float am = 0.f;
  for (int j = lane; j < cols; j += 32) am = fmaxf(am, fabsf(xr[j]));
  am = fmaxf(warp_max(am), 1e-5f);
  const float sc = fdiv(am, (float)q), inv = fdiv(1.0f, sc);
  if (lane == 0) scale_row[row] = sc;
  for (int j = lane; j < cols; j += 32) {
    const float xc = fclamp(frint(fmul(xr[j], inv)), -(float)q, (float)q);
    boundary[(size_t)row * cols + j] = (int16_t)frint(fmul(fabsf(xc), ratio));
    sign[(size_t)row * cols + j] = xc > 0.f ? 1 : (xc < 0.f ? -1 : 0);
  }
}

// fused_quant_kernel unipolar (fused.py:82-84, 96, 113-123): one warp per row.
__global__ void ref_unipolar_kernel(const float* __restrict__ x, int rows, int cols, float inv,
                                    float zp, int q, float ratio, int32_t* __restrict__ boundary,
                                    float* __restrict__ row_sum) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (row >= rows) return;
  float s = 0.f;
  for (int j = lane; j < cols; j += 32) {
    const float xc =
        fclamp(frint(fadd(fmul(x[(size_t)row * cols + j], inv), zp)), 0.f, (float)q);
    boundary[(size_t)row * cols + j] = (int32_t)frint(fmul(xc, ratio));
    s = fadd(s, xc);
  }
  if (row_sum) {
    s = warp_sum(s);
    if (lane == 0) row_sum[row] = s;
  }
}

// _grouped_*_quant elementwise stage with the per-row scale (and zero point)
// from group_params_kernel (quant/grouped.py:51-53, 131).
__global__ void ref_grouped_kernel(const float* __restrict__ x, size_t total, int cols, int q,
                                   int asym, const float* __restrict__ scale,
                                   const float* __restrict__ zp, float* __restrict__ xint,
                                   int8_t* __restrict__ sign) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const size_t r = i / cols;
  const float qf = (float)q;
  if (asym) {
    xint[i] = fclamp(frint(fadd(fdiv(x[i], scale[r]), zp[r])), 0.f, qf);
  } else {
    const float xi = fclamp(frint(fdiv(x[i], scale[r])), -qf, qf);
    xint[i] = xi;
    sign[i] = xi < 0.f ? -1 : 1;  // torch.sign with 0 -> +1
  }
}

// Reference-format (boundary, sign) -> signed thermometer length / boundary,
// written in the GEMM's blocked layout.
__global__ void encode_kernel(const int16_t* __restrict__ bnd, const int8_t* __restrict__ sgn,
                              size_t total, int rows, int d, const int16_t* __restrict__ ktab,
                              const int32_t* __restrict__ map, int vcap,
                              int16_t* __restrict__ out) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int j = (int)(i % d);
  const int row = (int)(i / d);
  int v = bnd[i];
  v = v < 0 ? 0 : (v < vcap ? v : vcap);
  if (ktab) v = ktab[(size_t)map[j] * (vcap + 1) + v];
  out[blk_idx(rows, row, j)] = (int16_t)(sgn && sgn[i] < 0 ? -v : v);
}

}  // namespace scmp

using namespace scmp;

extern "C" {

int scmp_fused_quantize_bipolar(const float* x, int rows, int cols, double abs_max, int sc_prec,
                                int rng_levels, int16_t* boundary, int8_t* sign, double* scale_out,
                                void* stream) {
  if (rows < 0 || cols < 0 || sc_prec < 2 || rng_levels < 1) return scmp::fail(SCMP_ERR_INVALID_ARG, "fused_quantize_bipolar: bad arguments");
  const int q = (1 << (sc_prec - 1)) - 1;
  abs_max = abs_max > 1e-5 ? abs_max : 1e-5;
  const double scale = abs_max / q;
  if (scale_out) *scale_out = scale;
  const size_t total = (size_t)rows * cols;
  if (total == 0) return SCMP_OK;
  dim3 grid((unsigned)((total + 255) / 256), 1);
  ref_bipolar_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
      x, total, rows, cols, nullptr, (float)(1.0 / scale), q, -(float)q,
      (float)rng_levels / (float)q, 0, boundary, sign);
  count_launch();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SCMP_OK : scmp::fail(SCMP_ERR_CUDA, cudaGetErrorString(e));
}

int scmp_fused_quantize_bipolar_perrow(const float* x, int rows, int cols, int sc_prec,
                                       int rng_levels, int16_t* boundary, int8_t* sign,
                                       float* scale_row, void* stream) {
  if (rows < 0 || cols < 0 || sc_prec < 2 || rng_levels < 1) return scmp::fail(SCMP_ERR_INVALID_ARG, "fused_quantize_bipolar_perrow: bad arguments");
  if (rows == 0) return SCMP_OK;
  const int q = (1 << (sc_prec - 1)) - 1;
  ref_bipolar_perrow_kernel<<<cdiv(rows, 8), 256, 0, (cudaStream_t)stream>>>(
      x, rows, cols, q, (float)rng_levels / (float)q, boundary, sign, scale_row);
  count_launch();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SCMP_OK : scmp::fail(SCMP_ERR_CUDA, cudaGetErrorString(e));
}

int scmp_fused_quantize_unipolar(const float* x, int rows, int cols, double fp_max, double fp_min,
                                 int sc_prec, int rng_levels, int32_t* boundary, float* row_sum,
                                 double* scale_out, double* zp_out, void* stream) {
  if (rows < 0 || cols < 0 || sc_prec < 1 || rng_levels < 1) return scmp::fail(SCMP_ERR_INVALID_ARG, "fused_quantize_unipolar: bad arguments");
  const int q = (1 << sc_prec) - 1;
  double range = fp_max - fp_min;
  range = range > 1e-5 ? range : 1e-5;
  const double scale = range / q;
  double zp = rint(-fp_min / scale);  // Python round(): half to even
  zp = zp < 0 ? 0 : (zp > q ? q : zp);
  if (scale_out) *scale_out = scale;
  if (zp_out) *zp_out = zp;
  if (rows == 0) return SCMP_OK;
  ref_unipolar_kernel<<<cdiv(rows, 8), 256, 0, (cudaStream_t)stream>>>(
      x, rows, cols, (float)(1.0 / scale), (float)zp, q, (float)rng_levels / (float)q, boundary,
      row_sum);
  count_launch();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SCMP_OK : scmp::fail(SCMP_ERR_CUDA, cudaGetErrorString(e));
}

int scmp_fused_quant_bipolar_batched(const float* x, int bh, int rows, int cols,
                                     const float* inv_scale, int sc_prec, int rng_levels,
                                     int16_t* boundary, int8_t* sign, void* stream) {
  if (bh < 0 || rows < 0 || cols < 0 || sc_prec < 2 || rng_levels < 1 || !inv_scale) return scmp::fail(SCMP_ERR_INVALID_ARG, "fused_quant_bipolar_batched: bad arguments");
  const size_t slice = (size_t)rows * cols;
  if (slice == 0 || bh == 0) return SCMP_OK;
  const int q = (1 << (sc_prec - 1)) - 1;
  dim3 grid((unsigned)((slice + 255) / 256), bh);
  ref_bipolar_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
      x, slice, rows, cols, inv_scale, 0.f, q, -(float)(q + 1), (float)rng_levels / (float)q, 1,
      boundary, sign);
  count_launch();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SCMP_OK : scmp::fail(SCMP_ERR_CUDA, cudaGetErrorString(e));
}

int scmp_grouped_symmetric_quant(const float* x, int batch, int rows, int cols, int group,
                                 int q_max, float* scale_row, float* x_int, int8_t* sign,
                                 float* group_stats, void* stream) {
  if (batch < 1 || rows < 0 || cols < 1 || group < 1 || q_max < 1) return scmp::fail(SCMP_ERR_INVALID_ARG, "grouped_symmetric_quant: bad arguments");
  if (batch > 1 && !(group == 1 || group >= rows))
    return scmp::fail(SCMP_ERR_UNSUPPORTED, "_grouped_symmetric_quant_batched: G not supported (use G=1 or G>=rows)");
  if (rows == 0) return SCMP_OK;
  cudaStream_t st = (cudaStream_t)stream;
  QuantArgs a{};
  a.x = x;
  a.rows = batch * rows;
  a.rows_per_batch = rows;
  a.d = cols;
  cudaError_t e = launch_row_stats(a, group_stats, st);
  if (e == cudaSuccess) e = launch_group_params(group_stats, batch, rows, group, q_max, GP_SYM, scale_row, nullptr, st);
  const size_t total = (size_t)a.rows * cols;
  if (e == cudaSuccess) {
    ref_grouped_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(x, total, cols, q_max, 0, scale_row, nullptr, x_int, sign);
    count_launch();
    e = cudaGetLastError();
  }
  return e == cudaSuccess ? SCMP_OK : scmp::fail(SCMP_ERR_CUDA, cudaGetErrorString(e));
}

int scmp_grouped_asymmetric_quant(const float* x, int rows, int cols, int group, int q_max,
                                  float* scale_row, float* zp_row, float* x_int,
                                  float* group_stats, void* stream) {
  if (rows < 0 || cols < 1 || group < 1 || q_max < 1) return scmp::fail(SCMP_ERR_INVALID_ARG, "grouped_asymmetric_quant: bad arguments");
  if (rows == 0) return SCMP_OK;
  cudaStream_t st = (cudaStream_t)stream;
  QuantArgs a{};
  a.x = x;
  a.rows = rows;
  a.rows_per_batch = rows;
  a.d = cols;
  cudaError_t e = launch_row_stats(a, group_stats, st);
  if (e == cudaSuccess) e = launch_group_params(group_stats, 1, rows, group, q_max, GP_ASYM, scale_row, zp_row, st);
  const size_t total = (size_t)rows * cols;
  if (e == cudaSuccess) {
    ref_grouped_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(x, total, cols, q_max, 1, scale_row, zp_row, x_int, nullptr);
    count_launch();
    e = cudaGetLastError();
  }
  return e == cudaSuccess ? SCMP_OK : scmp::fail(SCMP_ERR_CUDA, cudaGetErrorString(e));
}

static void carve_enable(int n, int m, int d, scmp::Carver& c, int16_t** ka, int16_t** vb,
                         int32_t** bmap) {
  const size_t dd = (size_t)scmp::d8(d) * 8;
  *ka = c.take<int16_t>((size_t)n * dd);
  *vb = c.take<int16_t>((size_t)m * dd);
  *bmap = c.take<int32_t>(dd);
}

int scmp_enable_matmul_workspace_size(int n, int m, int d, size_t* bytes) {
  if (n < 0 || m < 0 || d < 1 || !bytes) return scmp::fail(SCMP_ERR_INVALID_ARG, "enable_matmul_workspace_size: bad arguments");
  scmp::Carver c;
  int16_t *ka, *vb;
  int32_t* bm;
  carve_enable(n, m, d, c, &ka, &vb, &bm);
  *bytes = c.off;
  return SCMP_OK;
}

int scmp_enable_matmul(const int16_t* ktab, const uint32_t* pattern, const int32_t* amap,
                       const int32_t* bmap, int vcap, int L, int lp, const int16_t* boundary_a,
                       const int16_t* boundary_b, const int8_t* sign_a, const int8_t* sign_b,
                       int n, int m, int d, float q_max_sq, int is_bipolar, float* out,
                       void* workspace, size_t workspace_bytes, int flags, void* stream) {
  size_t need = 0;
  if (scmp_enable_matmul_workspace_size(n, m, d, &need)) return SCMP_ERR_INVALID_ARG;
  if (L < 1 || lp < L || lp % 32 || vcap < 1 || vcap > 32767) return scmp::fail(SCMP_ERR_INVALID_ARG, "enable_matmul: bad table sizes");
  if (n == 0 || m == 0) return SCMP_OK;
  if (!workspace || workspace_bytes < need) return scmp::fail(SCMP_ERR_WORKSPACE, "enable_matmul: workspace missing or too small");
  cudaStream_t st = (cudaStream_t)stream;
  scmp::Carver c{static_cast<char*>(workspace), 0};
  int16_t *ka, *vb;
  int32_t* bm;
  carve_enable(n, m, d, c, &ka, &vb, &bm);
  const size_t ta = (size_t)n * d, tb = (size_t)m * d;
  encode_kernel<<<(unsigned)((ta + 255) / 256), 256, 0, st>>>(boundary_a, is_bipolar ? sign_a : nullptr, ta, n, d, ktab, amap, vcap, ka);
  count_launch();
  encode_kernel<<<(unsigned)((tb + 255) / 256), 256, 0, st>>>(boundary_b, is_bipolar ? sign_b : nullptr, tb, m, d, nullptr, bmap, vcap, vb);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = scmp::launch_pad_map(bmap, d, bm, st);
  GemmArgs g{};
  g.batch = 1;
  g.n = n;
  g.m = m;
  g.d = d;
  g.L = L;
  g.lp = lp;
  g.vcap = vcap;
  g.bipolar = is_bipolar;
  g.ka = ka;
  g.vb = vb;
  g.pattern = pattern;
  g.bmap = bm;
  g.unit_d = d;
  g.outs[0] = out;
  g.nouts = 1;
  g.out_off = 0;
  g.out_ld = m;
  g.out_vec = m % 4 == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  g.epi.kind = EPI_RAW;
  g.epi.inner = q_max_sq / (float)L;
  if (e == cudaSuccess) e = scmp::launch_gemm(g, flags, st);
  return e == cudaSuccess ? SCMP_OK : scmp::fail(SCMP_ERR_CUDA, cudaGetErrorString(e));
}

}  // extern "C"
