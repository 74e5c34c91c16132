/* CPU oracle -- TEST INFRASTRUCTURE ONLY (checker and CPU baseline, never the
 * product). C restatement of the integer accumulator of the reference's
 * enable_matmul_tiled_kernel (scmp_kernels/sc/kernels.py:216-245):
 *
 *   S[m][n] = sum_d sa[m][d] * sb[n][d] * cum_{row(d)}[k[m][d]][bb[n][d]]
 *
 * where k[m][d] = k_table[d][boundary_a[m][d]] (looked up by the caller) and
 * cum_r[k][v] = #{i < k : rb_r[i] < v} is the reference's cum_indicator row
 * (kernels.py:102-137) for the distinct prepared sequence r of dimension d.
 * Signs are NULL for unipolar. Rows of S are split over OpenMP threads.
 */
#include <stdint.h>
#include <omp.h>

void sc_enable_sum(int N, int M, int D, const int32_t* kk, const int32_t* bb, const int8_t* sa,
                   const int8_t* sb, const int32_t* cum, const int32_t* rowmap, int L1, int V,
                   int64_t* S, int threads) {
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(dynamic, 1)
  for (int m = 0; m < N; ++m) {
    const int32_t* km = kk + (int64_t)m * D;
    const int8_t* sam = sa ? sa + (int64_t)m * D : 0;
    for (int n = 0; n < M; ++n) {
      const int32_t* bn = bb + (int64_t)n * D;
      const int8_t* sbn = sb ? sb + (int64_t)n * D : 0;
      int64_t s = 0;
      for (int d = 0; d < D; ++d) {
        const int32_t c = cum[((int64_t)rowmap[d] * L1 + km[d]) * V + bn[d]];
        s += sam ? (int64_t)(sam[d] * sbn[d]) * c : c;
      }
      S[(int64_t)m * M + n] = s;
    }
  }
}
