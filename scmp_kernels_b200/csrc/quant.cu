// Quantisation prologue of the fused sc_matmul path (HBM-bound).
//
// Each kernel restates one of the reference's float32 quantisation recipes
// bit for bit and writes the operands in the form the SC-GEMM consumes:
//   operand a -> int16 sa * k, k = ktab[amap[j]][min(boundary, vcap)]
//   operand b -> int16 sb * v, v = min(boundary, vcap)
// (the reference keeps (boundary, sign) and looks k up inside the GEMM,
// sc/kernels.py:229-231). SmoothQuant's a / s and b * s
// (quant/smoothquant.py:124-126) are applied on the fly.
#include "quant.cuh"

namespace scmp {

__device__ __forceinline__ float load_x(const QuantArgs& q, size_t row, int j) {
  float x = __ldg(q.x + row * (size_t)q.d + j);
  if (q.smooth) x = q.smooth_div ? fdiv(x, __ldg(q.smooth + j)) : fmul(x, __ldg(q.smooth + j));
  return x;
}

__device__ __forceinline__ int16_t encode(const LevelQ& lq, int j, int boundary, float sgn) {
  int v = boundary < lq.vcap ? boundary : lq.vcap;
  if (lq.ktab) v = __ldg(lq.ktab + (size_t)__ldg(lq.amap + j) * (lq.vcap + 1) + v);
  return (int16_t)(sgn < 0.f ? -v : v);
}

// --------------------------------------------------------------------------
// statistics
// --------------------------------------------------------------------------

// {absmax, max, min} of (smoothed) row `row`, reduced over the warp. With
// q.vec the row is read as float4, four loads in flight per lane.
__device__ __forceinline__ void row_minmax(const QuantArgs& q, int row, int lane, float& am, float& mx, float& mn) {
  am = 0.f;
  mx = -INFINITY;
  mn = INFINITY;
  if (q.vec) {
    const float4* src = reinterpret_cast<const float4*>(q.x + (size_t)row * q.d);
    const int n4 = q.d >> 2;
#pragma unroll 4
    for (int k = lane; k < n4; k += 32) {
      const float4 v = __ldg(src + k);
      float xs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = xs[e];
        if (q.smooth) {
          const float sv = __ldg(q.smooth + 4 * k + e);
          x = q.smooth_div ? fdiv(x, sv) : fmul(x, sv);
        }
        am = fmaxf(am, fabsf(x));
        mx = fmaxf(mx, x);
        mn = fminf(mn, x);
      }
    }
  } else {
    for (int j = lane; j < q.d; j += 32) {
      const float x = load_x(q, row, j);
      am = fmaxf(am, fabsf(x));
      mx = fmaxf(mx, x);
      mn = fminf(mn, x);
    }
  }
  am = warp_max(am);
  mx = warp_max(mx);
  mn = warp_min(mn);
}

// stats[r] = {absmax, max, min} of (smoothed) row r; one warp per row.
__global__ void row_stats_kernel(QuantArgs q, float* __restrict__ stats) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= q.rows) return;
  float am, mx, mn;
  row_minmax(q, warp, lane, am, mx, mn);
  if (lane == 0) {
    stats[3 * (size_t)warp + 0] = am;
    stats[3 * (size_t)warp + 1] = mx;
    stats[3 * (size_t)warp + 2] = mn;
  }
}

// Reduce stats over the rows of one group: blockIdx.x = group.
__device__ void group_reduce(const float* stats, int r0, int r1, float& am, float& mx, float& mn) {
  __shared__ float sh[3][32];
  __syncthreads();  // a previous call may still be reading sh
  am = 0.f;
  mx = -INFINITY;
  mn = INFINITY;
  for (int r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
    am = fmaxf(am, stats[3 * (size_t)r]);
    mx = fmaxf(mx, stats[3 * (size_t)r + 1]);
    mn = fminf(mn, stats[3 * (size_t)r + 2]);
  }
  am = warp_max(am);
  mx = warp_max(mx);
  mn = warp_min(mn);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (l == 0) {
    sh[0][w] = am;
    sh[1][w] = mx;
    sh[2][w] = mn;
  }
  __syncthreads();
  if (w == 0) {
    am = l < nw ? sh[0][l] : 0.f;
    mx = l < nw ? sh[1][l] : -INFINITY;
    mn = l < nw ? sh[2][l] : INFINITY;
    am = warp_max(am);
    mx = warp_max(mx);
    mn = warp_min(mn);
    if (l == 0) {
      sh[0][0] = am;
      sh[1][0] = mx;
      sh[2][0] = mn;
    }
  }
  __syncthreads();
  am = sh[0][0];
  mx = sh[1][0];
  mn = sh[2][0];
}

// Group id layout: rows are (batch, rows_per_batch); inside a batch, full
// groups of G rows and one remainder group; G >= rows_per_batch is one group
// (quant/grouped.py:28-75).
__device__ __forceinline__ void group_bounds(int g, int rpb, int G, int& r0, int& r1) {
  const int gpb = G >= rpb ? 1 : cdiv(rpb, G);
  const int b = g / gpb, gl = g % gpb;
  if (G >= rpb) {
    r0 = b * rpb;
    r1 = r0 + rpb;
  } else {
    r0 = b * rpb + gl * G;
    r1 = min(r0 + G, (b + 1) * rpb);
  }
}

// Per-group scale (and zero point) written to every row of the group.
//   symmetric  (grouped.py:46-47): scale = max(absmax, 1e-5) / q
//   asymmetric (grouped.py:111-115): scale = max(max - min, 1e-5) / q,
//              zp = clamp(round(-min / scale), 0, q)
//   head       (kernels.py:490-495): scale = max(|max|, |min|, 1e-5) / q and
//              inv = 1 / scale, one value per batch entry
__global__ void group_params_kernel(const float* __restrict__ stats, int rpb, int G, int q,
                                    int recipe, float* __restrict__ scale, float* __restrict__ zp) {
  int r0, r1;
  group_bounds(blockIdx.x, rpb, G, r0, r1);
  float am, mx, mn;
  group_reduce(stats, r0, r1, am, mx, mn);
  const float qf = (float)q;
  float sc = 0.f, z = 0.f;
  if (recipe == GP_SYM) {
    sc = fdiv(fmaxf(am, 1e-5f), qf);
  } else if (recipe == GP_ASYM) {
    sc = fdiv(fmaxf(fsub(mx, mn), 1e-5f), qf);
    z = fclamp(frint(fdiv(-mn, sc)), 0.f, qf);
  } else {  // GP_HEAD: per batch entry, scale in `scale`, inverse in `zp`
    sc = fdiv(fmaxf(fmaxf(fabsf(mx), fabsf(mn)), 1e-5f), qf);
    if (threadIdx.x == 0) {
      scale[blockIdx.x] = sc;
      zp[blockIdx.x] = fdiv(1.0f, sc);
    }
    return;
  }
  for (int r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
    scale[r] = sc;
    if (zp) zp[r] = z;
  }
}

// Per-head parameters in one pass (the GP_HEAD recipe of group_params_kernel
// over row_stats_kernel's statistics, sc/kernels.py:490-495): one block per
// batch entry reads the entry's
// rows_per_batch * d (smoothed) values as one contiguous range — 16-byte
// loads on its aligned middle, several in flight per thread — reduces max and
// min (order-free, so the bits equal the two-kernel path's, NaN and empty
// entries included) and writes scale = max(|max|, |min|, 1e-5) / q and its
// inverse.
__global__ void __launch_bounds__(512) head_params_kernel(QuantArgs q, int q_max, float* __restrict__ scale,
                                                          float* __restrict__ inv) {
  __shared__ float sh[2][16];
  const size_t n = (size_t)q.rows_per_batch * q.d;
  const float* x = q.x + (size_t)blockIdx.x * n;
  float mx = -INFINITY, mn = INFINITY;
  auto take = [&](size_t i, float v) {
    if (q.smooth) {
      const float s = __ldg(q.smooth + (int)(i % (size_t)q.d));
      v = q.smooth_div ? fdiv(v, s) : fmul(v, s);
    }
    mx = fmaxf(mx, v);
    mn = fminf(mn, v);
  };
  // elements before the first 16-byte boundary (x is 4-byte aligned), the
  // float4 body, the tail
  const size_t lead = ((16u - (uint32_t)(reinterpret_cast<uintptr_t>(x) & 15u)) & 15u) / 4u;
  const size_t h0 = lead < n ? lead : n;
  for (size_t i = threadIdx.x; i < h0; i += blockDim.x) take(i, __ldg(x + i));
  const size_t n4 = (n - h0) / 4;
  const float4* x4 = reinterpret_cast<const float4*>(x + h0);
#pragma unroll 4
  for (size_t k = threadIdx.x; k < n4; k += blockDim.x) {
    const float4 v = __ldg(x4 + k);
    const size_t i = h0 + 4 * k;
    take(i, v.x);
    take(i + 1, v.y);
    take(i + 2, v.z);
    take(i + 3, v.w);
  }
  for (size_t i = h0 + 4 * n4 + threadIdx.x; i < n; i += blockDim.x) take(i, __ldg(x + i));
  mx = warp_max(mx);
  mn = warp_min(mn);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sh[0][w] = mx;
    sh[1][w] = mn;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k) {
      mx = fmaxf(mx, sh[0][k]);
      mn = fminf(mn, sh[1][k]);
    }
    const float sc = fdiv(fmaxf(fmaxf(fabsf(mx), fabsf(mn)), 1e-5f), (float)q_max);
    scale[blockIdx.x] = sc;
    inv[blockIdx.x] = fdiv(1.0f, sc);
  }
}

// Per-tensor parameters for both operands, computed in double like the
// reference's host code (kernels.py:1173-1186, quant/fused.py:172-174, 204-209,
// and the scale product of kernels.py:1204). One block of 1024 threads.
//   scal[0] = fl32(scale_a * scale_b)        scal[4] = fl32(inv_scale_a)
//   scal[1] = fl32(-zp_b)                    scal[5] = fl32(inv_scale_b)
//   scal[2] = fl32(zp_a)                     scal[6] = fl32(zp_a)  (quant offset)
//   scal[3] = fl32(D * zp_a * zp_b)          scal[7] = fl32(zp_b)
// `ranges` (optional) = {a_max, a_min, b_max, b_min} given by the caller.
__global__ void tensor_params_kernel(const float* __restrict__ stats_a, int rows_a,
                                     const float* __restrict__ stats_b, int rows_b, int d, int q,
                                     int unipolar, const double* __restrict__ ranges,
                                     float* __restrict__ scal) {
  double mx_a, mn_a, mx_b, mn_b;
  if (ranges) {
    mx_a = ranges[0];
    mn_a = ranges[1];
    mx_b = ranges[2];
    mn_b = ranges[3];
  } else {
    float am, x, n;
    group_reduce(stats_a, 0, rows_a, am, x, n);
    mx_a = x;
    mn_a = n;
    group_reduce(stats_b, 0, rows_b, am, x, n);
    mx_b = x;
    mn_b = n;
  }
  if (threadIdx.x != 0) return;
  const double qd = (double)q;
  if (!unipolar) {
    // abs_max = max(|max|, |min|, 1e-5); scale = abs_max / q; inv = 1 / scale
    const double aa = fmax(fmax(fabs(mx_a), fabs(mn_a)), 1e-5);
    const double ab = fmax(fmax(fabs(mx_b), fabs(mn_b)), 1e-5);
    const double sa = aa / qd, sb = ab / qd;
    scal[0] = (float)(sa * sb);
    scal[4] = (float)(1.0 / sa);
    scal[5] = (float)(1.0 / sb);
    scal[1] = scal[2] = scal[3] = scal[6] = scal[7] = 0.f;
  } else {
    // range = max(max - min, 1e-5); scale = range / q; inv = 1 / scale;
    // zp = clamp(round(-min / scale), 0, q)
    const double ra = fmax(mx_a - mn_a, 1e-5);
    const double rb = fmax(mx_b - mn_b, 1e-5);
    const double sa = ra / qd, sb = rb / qd;
    const double za = fmax(0.0, fmin(qd, rint(-mn_a / sa)));
    const double zb = fmax(0.0, fmin(qd, rint(-mn_b / sb)));
    scal[0] = (float)(sa * sb);
    scal[1] = (float)(-zb);
    scal[2] = (float)za;
    scal[3] = (float)((double)d * za * zb);
    scal[4] = (float)(1.0 / sa);
    scal[5] = (float)(1.0 / sb);
    scal[6] = (float)za;
    scal[7] = (float)zb;
  }
}

// --------------------------------------------------------------------------
// quantisers: one warp per row
// --------------------------------------------------------------------------

// One element of the non-chunked recipes: the quantised value's boundary
// (through the k-table for operand a) with its sign, as the GEMM operand.
// Boundary of a quantised magnitude m (an integer held in a float) on the grid
// of lq: the divide form of the grouped recipes, round(m * G / q)
// (kernels.py:1679, 1685), or the multiply form round(m * fl32(G / q)) of the
// others (quant/fused.py:98-106, kernels.py:1864).
template <int R>
__device__ __forceinline__ int bnd_of(const LevelQ& lq, float m, float qf) {
  if (R == Q_GROUP_SYM || R == Q_GROUP_ASYM) return (int)frint(fdiv(fmul(m, (float)lq.G), qf));
  return (int)frint(fmul(m, lq.ratio));
}

// Magnitudes 0 .. kBndTab - 1 whose boundaries quant_rows_kernel tabulates in
// shared memory (q_max + 1 < kBndTab; the magnitude of a clamped value is an
// integer in [0, q_max + 1]), so that an element costs one table read instead
// of the boundary's multiply, divide and rounding. The table holds bnd_of's
// own results, so the boundaries are the same.
constexpr int kBndTab = 258;  // q_max <= 256: sc_prec up to 8 (4 KB of shared memory for four grids)

// tab: the boundary table of lq's grid, or NULL to compute the boundary.
template <int R>
__device__ __forceinline__ int16_t quant_one(const QuantArgs& q, const LevelQ& lq, int j, float x, float sc, float inv,
                                            float zp, float qf, float& rsum, const int* tab = nullptr) {
  {
    float mag;
    float sgn = 1.f;
    if (R == Q_TENSOR_BIP || R == Q_HEAD_BIP) {
      // fused.py:94-106 / 265-273: clamp(rint(x * inv), [qmin, q]); rint(|xc| * G/q)
      const float xc = fclamp(frint(fmul(x, inv)), q.qmin, qf);
      mag = fabsf(xc);
      sgn = xc;
    } else if (R == Q_TENSOR_UNI) {
      // fused.py:84, 98, 114-121: clamp(rint(x * inv + zp), 0, q)
      const float xc = fclamp(frint(fadd(fmul(x, inv), zp)), 0.f, qf);
      mag = xc;
      rsum = fadd(rsum, xc);
    } else if (R == Q_GROUP_SYM) {
      // grouped.py:51 + kernels.py:1679: clamp(round(x / s), +-q); round(|xi| * G / q)
      const float xi = fclamp(frint(fdiv(x, sc)), -qf, qf);
      mag = fabsf(xi);
      sgn = xi;
    } else if (R == Q_BATCH_SYM) {
      // grouped.py:148/156 + kernels.py:1864: round(|xi| * fl32(G / q))
      const float xi = fclamp(frint(fdiv(x, sc)), -qf, qf);
      mag = fabsf(xi);
      sgn = xi;
    } else {  // Q_GROUP_ASYM: grouped.py:131 + kernels.py:1685
      const float xi = fclamp(frint(fadd(fdiv(x, sc), zp)), 0.f, qf);
      mag = xi;
      rsum = fadd(rsum, xi);
    }
    const int bnd = tab ? tab[(int)mag] : bnd_of<R>(lq, mag, qf);
    return encode(lq, j, bnd, sgn);
  }
}

template <int R>
__global__ void quant_rows_kernel(QuantArgs q) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const float qf = (float)q.q;
  // boundary tables of the grids (one, or one per row level), see kBndTab
  __shared__ int s_bnd[kMaxLevels][kBndTab];
  const bool use_tab = q.q + 1 < kBndTab;
  if (use_tab) {
    const int nt = q.row_of ? q.nlev : 1;
    for (int l = 0; l < nt; ++l) {
      const LevelQ L = q.row_of ? q.lq[l] : LevelQ{q.ratio, q.G, q.vcap, q.ktab, q.amap};
      for (int i = threadIdx.x; i <= q.q + 1; i += blockDim.x) s_bnd[l][i] = bnd_of<R>(L, (float)i, qf);
    }
    __syncthreads();
  }
  if (row >= q.rows) return;
  int16_t* out = q.out16;  // blocked [d/8][rows][8] layout (blk_idx)
  // the source row and the grid it is quantised on (row levels: its level's)
  int src = row;
  LevelQ lq{q.ratio, q.G, q.vcap, q.ktab, q.amap};
  const int* tab = use_tab ? s_bnd[0] : nullptr;
  if (q.row_of) {
    src = __ldg(q.row_of + row);
    int lv = q.nlev - 1;
    for (int l = 0; l < q.nlev; ++l)
      if ((row >> 8) < __ldg(q.lev_tile0 + l + 1)) {
        lv = l;
        break;
      }
    lq = q.lq[lv];
    if (use_tab) tab = s_bnd[lv];
    if (src < 0) {  // padding row of a level's last tile: a zero operand
      const int nch = R == Q_ROWCHUNK_BIP ? cdiv(q.d, q.chunk_d) : 0;
      for (int c = lane; c < nch; c += 32) q.chunk_scale[(size_t)c * q.rows + row] = 0.f;
      for (int jb = lane; jb < d8(q.d); jb += 32)
        *reinterpret_cast<uint4*>(out + blk_idx(q.rows, row, 8 * jb)) = make_uint4(0, 0, 0, 0);
      if (lane == 0) {
        if (q.row_scale) q.row_scale[row] = 0.f;
        if (q.row_zp) q.row_zp[row] = 0.f;
        if (q.row_sum) q.row_sum[row] = 0.f;
      }
      return;
    }
  }

  if (R == Q_ROWCHUNK_BIP) {
    // fused_quant_kernel PER_ROW bipolar on every chunk (fused.py:65-81, 98-112)
    const int nch = cdiv(q.d, q.chunk_d);
    for (int c = 0; c < nch; ++c) {
      const int j0 = c * q.chunk_d, j1 = min(j0 + q.chunk_d, q.d);
      float am = 0.f;
      for (int j = j0 + lane; j < j1; j += 32) am = fmaxf(am, fabsf(load_x(q, src, j)));
      am = fmaxf(warp_max(am), 1e-5f);
      const float sc = fdiv(am, qf);
      const float inv = fdiv(1.0f, sc);
      if (lane == 0) q.chunk_scale[(size_t)c * q.rows + row] = sc;
      for (int j = j0 + lane; j < j1; j += 32) {
        const float xc = fclamp(frint(fmul(load_x(q, src, j), inv)), -qf, qf);
        const int bnd = tab ? tab[(int)fabsf(xc)] : bnd_of<R>(lq, fabsf(xc), qf);
        out[blk_idx(q.rows, row, j)] = encode(lq, j, bnd, xc);
      }
    }
    return;
  }

  float inv = 0.f, sc = 0.f, zp = 0.f;
  if (R == Q_TENSOR_BIP || R == Q_TENSOR_UNI) {
    inv = __ldg(q.params + q.param_off);
    zp = R == Q_TENSOR_UNI ? __ldg(q.params + q.param_off + 2) : 0.f;
  } else if (R == Q_HEAD_BIP) {
    inv = __ldg(q.params + row / q.rows_per_batch);
  } else if (q.self_stats) {
    // G == 1: the row is its own group (grouped.py:46-47, 111-115)
    float am, mx, mn;
    row_minmax(q, src, lane, am, mx, mn);
    if (R == Q_GROUP_ASYM) {
      sc = fdiv(fmaxf(fsub(mx, mn), 1e-5f), qf);
      zp = fclamp(frint(fdiv(-mn, sc)), 0.f, qf);
    } else {
      sc = fdiv(fmaxf(am, 1e-5f), qf);
    }
    if (lane == 0) {
      q.row_scale[row] = sc;
      if (R == Q_GROUP_ASYM) q.row_zp[row] = zp;
    }
  } else {
    sc = __ldg(q.row_scale + row);
    if (R == Q_GROUP_ASYM) zp = __ldg(q.row_zp + row);
  }

  float rsum = 0.f;
  // Each lane quantises whole blocks of eight dimensions (blocked output: one
  // 16-byte store per block; with q.vec, two 16-byte loads per block).
  const int nb = d8(q.d);
#pragma unroll 2
  for (int jb = lane; jb < nb; jb += 32) {
    const int j0 = 8 * jb;
    float xs[8];
    if (q.vec && j0 + 8 <= q.d) {
      const float4* sp = reinterpret_cast<const float4*>(q.x + (size_t)src * q.d + j0);
      const float4 u = __ldg(sp), w = __ldg(sp + 1);
      xs[0] = u.x; xs[1] = u.y; xs[2] = u.z; xs[3] = u.w;
      xs[4] = w.x; xs[5] = w.y; xs[6] = w.z; xs[7] = w.w;
      if (q.smooth) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float sv = __ldg(q.smooth + j0 + e);
          xs[e] = q.smooth_div ? fdiv(xs[e], sv) : fmul(xs[e], sv);
        }
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) xs[e] = j0 + e < q.d ? load_x(q, src, j0 + e) : 0.f;
    }
    uint32_t packed[4];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int j = j0 + e;
      const float x = xs[e];
      int16_t code = 0;
      if (j < q.d) code = quant_one<R>(q, lq, j, x, sc, inv, zp, qf, rsum, tab);
      if (e & 1)
        packed[e >> 1] |= (uint32_t)(uint16_t)code << 16;
      else
        packed[e >> 1] = (uint16_t)code;
    }
    *reinterpret_cast<uint4*>(out + blk_idx(q.rows, row, j0)) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
  if (q.row_sum) {
    rsum = warp_sum(rsum);
    if (lane == 0) q.row_sum[row] = rsum;
  }
}

// --------------------------------------------------------------------------
// quantisers: one block of 256 threads per row, the row held in registers
// --------------------------------------------------------------------------

// The non-chunked recipes of quant_rows_kernel, a row per TPR threads: each
// thread loads its NB blocks of eight dimensions (blocks t, t + TPR, ...; two
// 16-byte loads each, all in flight at once), smooths them once, reduces the
// row statistics over the row's threads and quantises from its registers.
// One pass over HBM, the smoothing division done once per element. Rows of
// more than 32 blocks take a whole block (TPR = 256); shorter rows 8, 16 or
// 32 threads and one block of eight dimensions each (NB = 1), 256 / TPR rows
// per block, so that the block's boundary table serves all of them and no
// thread idles on a 64-long row (the rows of one block lie in one 256-row
// tile, hence in one row level). Results are identical to quant_rows_kernel
// (same per-element recipe; the row sums add exact integers, so their order
// does not matter).
template <int R, int NB, int TPR>
__global__ void __launch_bounds__(256) quant_row_cta_kernel(QuantArgs q) {
  static_assert(TPR == 256 || (NB == 1 && TPR >= 8 && TPR <= 32), "short rows: 8 to 32 threads, one block each");
  constexpr int RPB = 256 / TPR;  // rows per block
  __shared__ int s_bnd[kBndTab];
  __shared__ float s_red[3][8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int sub = tid % TPR;  // the thread's place in its row
  const int row = blockIdx.x * RPB + tid / TPR;
  const bool in_range = row < q.rows;
  const float qf = (float)q.q;
  int src = in_range ? row : -1;
  LevelQ lq{q.ratio, q.G, q.vcap, q.ktab, q.amap};
  if (q.row_of) {
    src = in_range ? __ldg(q.row_of + row) : -1;
    const int tile = (blockIdx.x * RPB) >> 8;  // the block's rows' tile
    int lv = q.nlev - 1;
    for (int l = 0; l < q.nlev; ++l)
      if (tile < __ldg(q.lev_tile0 + l + 1)) {
        lv = l;
        break;
      }
    lq = q.lq[lv];
  }
  const bool use_tab = q.q + 1 < kBndTab;
  if (use_tab)
    for (int i = tid; i <= q.q + 1; i += 256) s_bnd[i] = bnd_of<R>(lq, (float)i, qf);
  __syncthreads();  // the boundary table is complete
  const int nb = d8(q.d);
  int16_t* out = q.out16;
  if (in_range && src < 0) {  // padding row of a level's last tile: a zero operand
    for (int jb = sub; jb < nb; jb += TPR)
      *reinterpret_cast<uint4*>(out + blk_idx(q.rows, row, 8 * jb)) = make_uint4(0, 0, 0, 0);
    if (sub == 0) {
      if (q.row_scale) q.row_scale[row] = 0.f;
      if (q.row_zp) q.row_zp[row] = 0.f;
      if (q.row_sum) q.row_sum[row] = 0.f;
    }
  }
  // a thread of a padding or out-of-range row takes part in its row group's
  // shuffles with zeros and stores nothing; a whole-block row leaves at once
  // (uniform over the block: no barrier follows for it)
  const bool active = in_range && src >= 0;
  if (TPR == 256 && !active) return;
  float xs[NB][8];
#pragma unroll
  for (int k = 0; k < NB; ++k) {
    const int j0 = 8 * (sub + TPR * k);
    if (active && q.vec && j0 + 8 <= q.d) {
      const float4* sp = reinterpret_cast<const float4*>(q.x + (size_t)src * q.d + j0);
      const float4 u = __ldg(sp), w = __ldg(sp + 1);
      xs[k][0] = u.x; xs[k][1] = u.y; xs[k][2] = u.z; xs[k][3] = u.w;
      xs[k][4] = w.x; xs[k][5] = w.y; xs[k][6] = w.z; xs[k][7] = w.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        xs[k][e] = active && j0 + e < q.d ? __ldg(q.x + (size_t)src * q.d + j0 + e) : 0.f;
    }
  }
  if (q.smooth && active) {
#pragma unroll
    for (int k = 0; k < NB; ++k)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = 8 * (sub + TPR * k) + e;
        if (j < q.d) {
          const float sv = __ldg(q.smooth + j);
          xs[k][e] = q.smooth_div ? fdiv(xs[k][e], sv) : fmul(xs[k][e], sv);
        }
      }
  }
  const bool self = (R == Q_GROUP_SYM || R == Q_GROUP_ASYM || R == Q_BATCH_SYM) && q.self_stats;
  float sc = 0.f, inv = 0.f, zp = 0.f;
  if (self) {
    float am = 0.f, mx = -INFINITY, mn = INFINITY;
#pragma unroll
    for (int k = 0; k < NB; ++k)
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (8 * (sub + TPR * k) + e < q.d) {
          const float x = xs[k][e];
          am = fmaxf(am, fabsf(x));
          mx = fmaxf(mx, x);
          mn = fminf(mn, x);
        }
    if constexpr (TPR == 256) {
      am = warp_max(am);
      mx = warp_max(mx);
      mn = warp_min(mn);
      if (lane == 0) {
        s_red[0][warp] = am;
        s_red[1][warp] = mx;
        s_red[2][warp] = mn;
      }
      __syncthreads();
      am = s_red[0][0];
      mx = s_red[1][0];
      mn = s_red[2][0];
#pragma unroll
      for (int w = 1; w < 8; ++w) {
        am = fmaxf(am, s_red[0][w]);
        mx = fmaxf(mx, s_red[1][w]);
        mn = fminf(mn, s_red[2][w]);
      }
    } else {
      // the row's TPR lanes (an aligned group of the warp): xor offsets below
      // TPR stay inside it
#pragma unroll
      for (int o = TPR / 2; o > 0; o >>= 1) {
        am = fmaxf(am, __shfl_xor_sync(0xFFFFFFFFu, am, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
        mn = fminf(mn, __shfl_xor_sync(0xFFFFFFFFu, mn, o));
      }
    }
    if (R == Q_GROUP_ASYM) {
      sc = fdiv(fmaxf(fsub(mx, mn), 1e-5f), qf);
      zp = fclamp(frint(fdiv(-mn, sc)), 0.f, qf);
    } else {
      sc = fdiv(fmaxf(am, 1e-5f), qf);
    }
    if (sub == 0 && active) {
      q.row_scale[row] = sc;
      if (R == Q_GROUP_ASYM) q.row_zp[row] = zp;
    }
  } else if (active) {
    if (R == Q_TENSOR_BIP || R == Q_TENSOR_UNI) {
      inv = __ldg(q.params + q.param_off);
      zp = R == Q_TENSOR_UNI ? __ldg(q.params + q.param_off + 2) : 0.f;
    } else if (R == Q_HEAD_BIP) {
      inv = __ldg(q.params + row / q.rows_per_batch);
    } else {
      sc = __ldg(q.row_scale + row);
      if (R == Q_GROUP_ASYM) zp = __ldg(q.row_zp + row);
    }
  }
  const int* tab = use_tab ? s_bnd : nullptr;
  float rsum = 0.f;
  if (active) {
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      const int jb = sub + TPR * k;
      if (jb >= nb) break;
      const int j0 = 8 * jb;
      uint32_t packed[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = j0 + e;
        int16_t code = 0;
        if (j < q.d) code = quant_one<R>(q, lq, j, xs[k][e], sc, inv, zp, qf, rsum, tab);
        packed[e >> 1] |= (uint32_t)(uint16_t)code << (16 * (e & 1));
      }
      *reinterpret_cast<uint4*>(out + blk_idx(q.rows, row, j0)) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
  }
  if (q.row_sum) {
    if constexpr (TPR == 256) {
      rsum = warp_sum(rsum);
      __syncthreads();  // every thread has read s_red
      if (lane == 0) s_red[0][warp] = rsum;
      __syncthreads();
      if (tid == 0) {
        float t = 0.f;
        for (int w = 0; w < 8; ++w) t = fadd(t, s_red[0][w]);
        q.row_sum[row] = t;
      }
    } else {
#pragma unroll
      for (int o = TPR / 2; o > 0; o >>= 1) rsum = fadd(rsum, __shfl_xor_sync(0xFFFFFFFFu, rsum, o));
      if (sub == 0 && active) q.row_sum[row] = rsum;
    }
  }
}

// Blocks of eight dimensions per thread of a whole-block row of
// quant_row_cta_kernel for d (0: rows too long, quant_rows_kernel instead).
static int row_cta_blocks(int d) {
  const int nb = d8(d);
  for (int k = 1; k <= 8; k *= 2)
    if (nb <= 256 * k) return k;
  return 0;
}

template <int R>
static cudaError_t launch_row_cta(const QuantArgs& q, cudaStream_t st) {
  const int nb = d8(q.d);
  if (nb <= 8) {
    quant_row_cta_kernel<R, 1, 8><<<cdiv(q.rows, 32), 256, 0, st>>>(q);
  } else if (nb <= 16) {
    quant_row_cta_kernel<R, 1, 16><<<cdiv(q.rows, 16), 256, 0, st>>>(q);
  } else if (nb <= 32) {
    quant_row_cta_kernel<R, 1, 32><<<cdiv(q.rows, 8), 256, 0, st>>>(q);
  } else {
    switch (row_cta_blocks(q.d)) {
      case 1: quant_row_cta_kernel<R, 1, 256><<<q.rows, 256, 0, st>>>(q); break;
      case 2: quant_row_cta_kernel<R, 2, 256><<<q.rows, 256, 0, st>>>(q); break;
      case 4: quant_row_cta_kernel<R, 4, 256><<<q.rows, 256, 0, st>>>(q); break;
      default: quant_row_cta_kernel<R, 8, 256><<<q.rows, 256, 0, st>>>(q); break;
    }
  }
  count_launch();
  return cudaGetLastError();
}

// --------------------------------------------------------------------------
// row levels: a's rows grouped by level, each level padded to whole tiles
// --------------------------------------------------------------------------

// One block. Counts the rows of every level, lays the levels out in tiles of
// 256 rows (level l from tile lev_tile0[l]) and scatters the row indices
// stably: within a level, rows keep their order (the order in which a
// caller's a[rows] would gather them). Rows whose level is out of range are
// left out and recorded as a device error.
__global__ void level_perm_kernel(const int32_t* __restrict__ row_level, int n, int nlev, int n_pad,
                                  int* __restrict__ row_of, int* __restrict__ lev_tile0) {
  __shared__ int cnt[kMaxLevels], base[kMaxLevels], wcnt[32][kMaxLevels];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  for (int i = tid; i < n_pad; i += blockDim.x) row_of[i] = -1;
  if (tid < kMaxLevels) cnt[tid] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x) {
    const int l = __ldg(row_level + i);
    if (l >= 0 && l < nlev) atomicAdd(&cnt[l], 1);
    else record_error(SCMP_ERR_INVALID_ARG, 40);
  }
  __syncthreads();
  if (tid == 0) {
    int t = 0;
    for (int l = 0; l < nlev; ++l) {
      lev_tile0[l] = t;
      base[l] = 256 * t;
      t += cdiv(cnt[l], 256);
    }
    lev_tile0[nlev] = t;
  }
  __syncthreads();
  for (int c0 = 0; c0 < n; c0 += blockDim.x) {
    const int i = c0 + tid;
    const int l = i < n ? __ldg(row_level + i) : -1;
    const bool ok = l >= 0 && l < nlev;
    int rank = 0;
#pragma unroll
    for (int k = 0; k < kMaxLevels; ++k) {
      const unsigned bal = __ballot_sync(0xFFFFFFFFu, ok && l == k);
      if (l == k) rank = __popc(bal & ((1u << lane) - 1u));
      if (lane == 0) wcnt[warp][k] = __popc(bal);
    }
    __syncthreads();
    if (ok) {
      int off = 0;
      for (int w = 0; w < warp; ++w) off += wcnt[w][l];
      row_of[base[l] + off + rank] = i;
    }
    __syncthreads();
    if (tid < nlev) {
      int tot = 0;
      for (int w = 0; w < nw; ++w) tot += wcnt[w][tid];
      base[tid] += tot;
    }
    __syncthreads();
  }
}

// --------------------------------------------------------------------------
// host launchers
// --------------------------------------------------------------------------

cudaError_t launch_level_perm(const int32_t* row_level, int n, int nlev, int n_pad, int* row_of, int* lev_tile0,
                              cudaStream_t st) {
  level_perm_kernel<<<1, 1024, 0, st>>>(row_level, n, nlev, n_pad, row_of, lev_tile0);
  count_launch();
  return cudaGetLastError();
}

static inline dim3 warp_grid(int rows) { return dim3(cdiv(rows, 8)); }

cudaError_t launch_row_stats(const QuantArgs& q, float* stats, cudaStream_t st) {
  if (q.rows > 0) {
    row_stats_kernel<<<warp_grid(q.rows), 256, 0, st>>>(q, stats);
    count_launch();
  }
  return cudaGetLastError();
}

cudaError_t launch_group_params(const float* stats, int batch, int rpb, int G, int q, int recipe,
                                float* scale, float* zp, cudaStream_t st) {
  const int gpb = G >= rpb ? 1 : cdiv(rpb, G);
  const int ng = recipe == GP_HEAD ? batch : batch * gpb;
  if (ng > 0) {
    group_params_kernel<<<ng, 256, 0, st>>>(stats, rpb, recipe == GP_HEAD ? rpb : G, q,
                                                       recipe, scale, zp);
    count_launch();
  }
  return cudaGetLastError();
}

cudaError_t launch_head_params(const QuantArgs& q, int batch, int q_max, float* scale, float* inv,
                               cudaStream_t st) {
  if (batch > 0) {
    head_params_kernel<<<batch, 512, 0, st>>>(q, q_max, scale, inv);
    count_launch();
  }
  return cudaGetLastError();
}

cudaError_t launch_tensor_params(const float* sa, int ra, const float* sb, int rb, int d, int q,
                                 int unipolar, const double* ranges, float* scal, cudaStream_t st) {
  tensor_params_kernel<<<1, 1024, 0, st>>>(sa, ra, sb, rb, d, q, unipolar, ranges, scal);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_quant_rows(int recipe, const QuantArgs& q, cudaStream_t st) {
  if (q.rows <= 0) return cudaSuccess;
  // one block per row for every recipe but the chunked one, while a row fits
  // its registers (SCMP_QUANT_WARP=1 in the environment: one warp per row)
  const char* ew = getenv("SCMP_QUANT_WARP");
  if (recipe != Q_ROWCHUNK_BIP && row_cta_blocks(q.d) > 0 && !(ew && ew[0] == '1')) {
    switch (recipe) {
      case Q_TENSOR_BIP: return launch_row_cta<Q_TENSOR_BIP>(q, st);
      case Q_TENSOR_UNI: return launch_row_cta<Q_TENSOR_UNI>(q, st);
      case Q_GROUP_SYM: return launch_row_cta<Q_GROUP_SYM>(q, st);
      case Q_GROUP_ASYM: return launch_row_cta<Q_GROUP_ASYM>(q, st);
      case Q_BATCH_SYM: return launch_row_cta<Q_BATCH_SYM>(q, st);
      case Q_HEAD_BIP: return launch_row_cta<Q_HEAD_BIP>(q, st);
      default: return cudaErrorInvalidValue;
    }
  }
  const dim3 g = warp_grid(q.rows);
  switch (recipe) {
    case Q_TENSOR_BIP: { quant_rows_kernel<Q_TENSOR_BIP><<<g, 256, 0, st>>>(q); count_launch(); } break;
    case Q_TENSOR_UNI: { quant_rows_kernel<Q_TENSOR_UNI><<<g, 256, 0, st>>>(q); count_launch(); } break;
    case Q_GROUP_SYM: { quant_rows_kernel<Q_GROUP_SYM><<<g, 256, 0, st>>>(q); count_launch(); } break;
    case Q_GROUP_ASYM: { quant_rows_kernel<Q_GROUP_ASYM><<<g, 256, 0, st>>>(q); count_launch(); } break;
    case Q_BATCH_SYM: { quant_rows_kernel<Q_BATCH_SYM><<<g, 256, 0, st>>>(q); count_launch(); } break;
    case Q_ROWCHUNK_BIP: { quant_rows_kernel<Q_ROWCHUNK_BIP><<<g, 256, 0, st>>>(q); count_launch(); } break;
    case Q_HEAD_BIP: { quant_rows_kernel<Q_HEAD_BIP><<<g, 256, 0, st>>>(q); count_launch(); } break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace scmp
