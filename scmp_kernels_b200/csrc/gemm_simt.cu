// CUDA-core SC-GEMM: the general, bit-exact baseline kernel.
//
// S[i][j] = sum_d sa*sb * popcount(pattern[bmap[d]][v[j][d]] & (2^k[i][d] - 1))
// i.e. the reference's cum_indicator[d][k][v] lookup (sc/kernels.py:229-236)
// evaluated as a prefix popcount of b's bit-packed comparator stream (words
// put back in position order when staged). Each
// 64x64 output tile stages, per dimension, every b row's stream words and
// their running popcounts in shared memory, so one popc serves one MAC.
// Used for shapes the tcgen05 kernel does not take and as its cross-check.
#include "internal.cuh"

namespace scmp {

namespace {
constexpr int TA = 64, TB = 64, DB = 4, THREADS = 256;
}

__global__ void __launch_bounds__(THREADS) gemm_simt_kernel(GemmArgs g) {
  extern __shared__ uint32_t sm[];
  const int lw = g.lp / 32;
  const int lw1 = lw + 1;
  int16_t* sk = reinterpret_cast<int16_t*>(sm);                       // [DB][TA]
  uint32_t* pw = sm + (DB * TA) / 2;                                  // [DB][TB][lw1]
  uint32_t* pre = pw + DB * TB * lw1;                                 // [DB][TB][lw1]
  int8_t* sgnb = reinterpret_cast<int8_t*>(pre + DB * TB * lw1);      // [DB][TB]

  const int tid = threadIdx.x;
  const int ty = tid / 16, tx = tid % 16;
  const int bh = blockIdx.z;
  const int a0 = blockIdx.y * TA, b0 = blockIdx.x * TB;
  const int Ra = g.batch * g.n, Rb = g.batch * g.m;  // rows of the blocked operands

  float run[4][4];
  int S[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) run[i][j] = 0.f;

  const int unit_d = g.unit_d > 0 ? g.unit_d : g.d;
  const int nunits = cdiv(g.d, unit_d);
  for (int u = 0; u < nunits; ++u) {
    const int d0 = u * unit_d, d1 = min(d0 + unit_d, g.d);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) S[i][j] = 0;

    for (int dd = d0; dd < d1; dd += DB) {
      __syncthreads();
      // stage a: signed thermometer lengths
      for (int e = tid; e < DB * TA; e += THREADS) {
        const int dl = e / TA, r = e % TA, d = dd + dl;
        int16_t v = 0;
        if (d < d1 && a0 + r < g.n) v = g.ka[blk_idx(Ra, bh * g.n + a0 + r, d)];
        sk[dl * TA + r] = v;
      }
      // stage b: stream words and their prefix popcounts
      {
        const int dl = tid / TB, r = tid % TB, d = dd + dl;
        int vv = 0;
        if (d < d1 && b0 + r < g.m) vv = g.vb[blk_idx(Rb, bh * g.m + b0 + r, d)];
        const int v = vv < 0 ? -vv : vv;
        uint32_t* w = pw + (dl * TB + r) * lw1;
        uint32_t* p = pre + (dl * TB + r) * lw1;
        sgnb[dl * TB + r] = vv < 0 ? -1 : 1;
        uint32_t acc = 0;
        if (d < d1) {
          const uint32_t* src =
              g.pattern + ((size_t)__ldg(g.bmap + d) * (g.vcap + 1) + v) * lw;
          for (int x = 0; x < lw; ++x) {
            const uint32_t bits = unslice(__ldg(src + x));
            w[x] = bits;
            p[x] = acc;
            acc += __popc(bits);
          }
        } else {
          for (int x = 0; x < lw; ++x) {
            w[x] = 0;
            p[x] = 0;
          }
        }
        w[lw] = 0;
        p[lw] = acc;
      }
      __syncthreads();
      const int nd = min(DB, d1 - dd);
      for (int dl = 0; dl < nd; ++dl) {
        int kk[4], sa[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int kv = sk[dl * TA + ty * 4 + i];
          kk[i] = kv < 0 ? -kv : kv;
          sa[i] = kv < 0 ? -1 : 1;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = tx * 4 + j;
          const uint32_t* w = pw + (dl * TB + r) * lw1;
          const uint32_t* p = pre + (dl * TB + r) * lw1;
          const int sb = sgnb[dl * TB + r];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int q = kk[i] >> 5, rr = kk[i] & 31;
            const int c = (int)p[q] + __popc(w[q] & ((1u << rr) - 1u));
            S[i][j] += g.bipolar ? sa[i] * sb * c : c;
          }
        }
      }
    }
    // epilogue of this accumulation unit
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int ia = a0 + ty * 4 + i;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int ib = b0 + tx * 4 + j;
        if (ia < g.n && ib < g.m) {
          const float val = epi_value(g.epi, S[i][j], bh * g.n + ia, bh * g.m + ib, bh, u, g.n, g.m);
          run[i][j] = g.epi.kind == EPI_CHUNK ? fadd(run[i][j], val) : val;
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int ia = a0 + ty * 4 + i;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int ib = b0 + tx * 4 + j;
      if (ia < g.n && ib < g.m) store_out(g, bh, ia, ib, run[i][j]);
    }
  }
}

cudaError_t launch_gemm_simt(const GemmArgs& g, cudaStream_t st) {
  const int lw1 = g.lp / 32 + 1;
  const size_t smem = (size_t)DB * TA * 2 + (size_t)2 * DB * TB * lw1 * 4 + DB * TB;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(gemm_simt_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  dim3 grid(cdiv(g.m, TB), cdiv(g.n, TA), g.batch);
  gemm_simt_kernel<<<grid, THREADS, smem, st>>>(g);
  count_launch();
  return cudaGetLastError();
}

}  // namespace scmp
