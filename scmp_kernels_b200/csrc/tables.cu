// Enable-signal tables: the k-table of operand a and the bit-packed comparator
// streams of operand b, built once per (config, sc_prec, stoc_len, grid) and
// kept resident in HBM.
//
// Restates build_cum_indicator_kernel / compute_k_table_kernel
// (scmp_kernels/sc/kernels.py:102-169). The reference materialises
// cum[d][k][v] = #{i < k : rb[d][i] < v} as an int16 (D, L+1, V_PAD) table
// (1.08 GB at D=4096, L=256); here each (row, v) keeps only its L-bit stream
// [rb[i] < v], from which cum is a prefix popcount, and distinct rows are
// stored once (all dimensions share one row under the default Sobol config).
#include "internal.cuh"

namespace scmp {

// ktab[r][v] = #{t < L : ra[r][t] < v}, v in [0, vcap]
__global__ void k_table_kernel(const int32_t* __restrict__ ra, int L, int vcap,
                               int16_t* __restrict__ ktab) {
  extern __shared__ int32_t srow[];
  const int r = blockIdx.x;
  for (int t = threadIdx.x; t < L; t += blockDim.x) srow[t] = ra[(size_t)r * L + t];
  __syncthreads();
  for (int v = threadIdx.x; v <= vcap; v += blockDim.x) {
    int c = 0;
    for (int t = 0; t < L; ++t) c += srow[t] < v;
    ktab[(size_t)r * (vcap + 1) + v] = (int16_t)c;
  }
}

// pattern[r][v][w] bit slice_bit(i) = (32w + i < L) && rb[r][32w + i] < v,
// and the same bit at slice4_bit(i) in pattern4 (when given)
__global__ void pattern_kernel(const int32_t* __restrict__ rb, int L, int lp, int vcap,
                               uint32_t* __restrict__ pat, uint32_t* __restrict__ pat4) {
  extern __shared__ int32_t srow[];
  const int r = blockIdx.x;
  const int lw = lp / 32;
  for (int t = threadIdx.x; t < L; t += blockDim.x) srow[t] = rb[(size_t)r * L + t];
  __syncthreads();
  const int total = (vcap + 1) * lw;
  for (int idx = blockIdx.y * blockDim.x + threadIdx.x; idx < total; idx += gridDim.y * blockDim.x) {
    const int v = idx / lw, w = idx % lw;
    uint32_t bits = 0, bits4 = 0;
    for (int i = 0; i < 32; ++i) {
      const int t = 32 * w + i;
      if (t < L && srow[t] < v) {
        bits |= 1u << slice_bit(i);
        bits4 |= 1u << slice4_bit(i);
      }
    }
    pat[((size_t)r * (vcap + 1) + v) * lw + w] = bits;
    if (pat4) pat4[((size_t)r * (vcap + 1) + v) * lw + w] = bits4;
  }
}

cudaError_t launch_build_tables(const int32_t* ra, int n_ra, const int32_t* rb, int n_rb, int L,
                                int lp, int vcap, int16_t* ktab, uint32_t* pattern, uint32_t* pattern4,
                                cudaStream_t st) {
  const size_t sm = (size_t)L * sizeof(int32_t);
  if (sm > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k_table_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(pattern_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
  }
  if (n_ra > 0) {
    k_table_kernel<<<n_ra, 256, sm, st>>>(ra, L, vcap, ktab);
    count_launch();
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (n_rb > 0) {
    const int lw = lp / 32;
    const int ys = cdiv((vcap + 1) * lw, 256);
    dim3 grid(n_rb, ys < 64 ? ys : 64);
    pattern_kernel<<<grid, 256, sm, st>>>(rb, L, lp, vcap, pattern, pattern4);
    count_launch();
  }
  return cudaGetLastError();
}

}  // namespace scmp
