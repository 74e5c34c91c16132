// tcgen05 SC-GEMM for sm_100a.
//
// The reference's integer accumulator (sc/kernels.py:216-245)
//   S[i][j] = sum_d sa*sb * #{t < k[i][d] : rb_d[t] < v[j][d]}
// is an int8 GEMM over K = D * L:
//   A'[i][(d,t)] = sa[i][d] * [t < k[i][d]]          (thermometer of a)
//   B'[j][(d,t)] = sb[j][d] * [rb_d[t] < v[j][d]]    (comparator stream of b)
// with every entry in {-1, 0, 1}. Neither operand exists in memory: producer
// warps expand them per pipeline stage straight into shared memory, in the
// canonical K-major 128-byte-swizzled layout, from the int16 operands of the
// quantiser (signed k, signed v) and the bit-packed streams of the table
// builder. One thread issues tcgen05.mma.kind::i8 (M=128, N=256, K=32) into
// an int32 accumulator in tensor memory; epilogue warps read it back with
// tcgen05.ld and apply the path's float32 recipe. The accumulation is exact.
//
// CTA: warps 0-3 expand A' (one a row per thread), warps 4-11 expand B' (one
// b row per thread), warp 12 allocates tensor memory and issues the MMAs,
// warps 13-16 run the epilogue. Persistent grid over output tiles. Every
// mbarrier wait is bounded (common.cuh): on timeout the kernel records
// SCMP_ERR_TIMEOUT, all roles leave their loops, outstanding MMAs are drained
// and tensor memory is freed before the CTA exits.
#include "internal.cuh"

namespace scmp {
namespace tc {

constexpr int BM = 128;                    // a rows per tile (UMMA M)
constexpr int BN = 256;                    // b rows per tile (UMMA N)
constexpr int KS = 256;                    // K bytes per stage
constexpr int NST = 2;                     // pipeline stages
constexpr int A_BYTES = BM * KS;           // 32 KB
constexpr int B_BYTES = BN * KS;           // 64 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int A_ATOM = BM * 128;           // one 128-byte-wide K atom of A
constexpr int B_ATOM = BN * 128;
constexpr int PROD_A_WARPS = 4, PROD_B_WARPS = 8;
constexpr int PROD_THREADS = (PROD_A_WARPS + PROD_B_WARPS) * 32;
constexpr int MMA_WARP = 12;
constexpr int EPI_WARP0 = 13;
constexpr int NWARPS = 17;
constexpr int THREADS = NWARPS * 32;
constexpr int TMEM_COLS = 512;             // [0,256) accumulator, [256,512) running chunk sum
constexpr int SMEM_BYTES = NST * STAGE_BYTES + 1024 + 256;

// Instruction descriptor: kind::i8, D = s32, A = B = s8, both K-major,
// N = 256 (n_dim = N >> 3), M = 128 (m_dim = M >> 4).
constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                           ((uint32_t)(BM >> 4) << 24);

// Shared-memory matrix descriptor, K-major with 128-byte swizzle: rows at a
// 128-byte pitch, 8-row groups 1024 bytes apart (SBO), version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

#define TMEM_LD32(taddr, r)                                                                        \
  asm volatile(                                                                                    \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14," \
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"               \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),       \
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),   \
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),             \
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),             \
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])              \
      : "r"(taddr))
#define TMEM_ST32(taddr, r)                                                                        \
  asm volatile(                                                                                    \
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13," \
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr), \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),     \
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),           \
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),         \
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),         \
      "r"(r[29]), "r"(r[30]), "r"(r[31]))

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Byte address of 16-byte chunk `kc` (0..15 within the stage's 256 K bytes)
// of row `r` in a K-major SW128 tile with `atom_bytes` per 128-byte K atom.
__device__ __forceinline__ uint32_t swz(uint32_t base, int atom_bytes, int r, int kc) {
  return base + (kc >> 3) * atom_bytes + r * 128 + ((((kc & 7) ^ (r & 7))) << 4);
}

struct Sched {
  int tiles, tiles_a, tiles_b, nunits, unit_d, spu_full;  // spu_full: stages of a full unit
};

__device__ __forceinline__ void tile_coords(const GemmArgs& g, const Sched& s, int tile, int& bh,
                                            int& a0, int& b0) {
  const int per = s.tiles_a * s.tiles_b;
  bh = tile / per;
  const int r = tile % per;
  a0 = (r / s.tiles_b) * BM;
  b0 = (r % s.tiles_b) * BN;
}

template <int TLEN>
__device__ __forceinline__ int stages_of_unit(int len) {
  if (TLEN < 256) return cdiv(len, 256 / TLEN);
  return len * (TLEN / 256);
}

// TLEN: padded stream length lp when lp <= 256 (256/lp dimensions per stage),
// or 256*k for lp = 256*k (k stages per dimension); here TLEN = min(lp, 256)
// and SPD = lp / TLEN stages per dimension.
template <int TLEN>
__global__ void __launch_bounds__(THREADS, 1) gemm_tc_kernel(GemmArgs g, Sched sc, int spd) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;          // SW128 tiles need 1024-B alignment
  uint8_t* gbase = smem_raw + (sbase - raw);
  const uint32_t bar_base = sbase + NST * STAGE_BYTES;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (NST + s); };
  const uint32_t accf_bar = bar_base + 8u * (2 * NST);
  const uint32_t acce_bar = bar_base + 8u * (2 * NST + 1);
  const uint32_t drain_bar = bar_base + 8u * (2 * NST + 2);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + NST * STAGE_BYTES + 128);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + NST * STAGE_BYTES + 136);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int DPS = TLEN < 256 ? 256 / TLEN : 1;  // dimensions per stage

  if (warp == MMA_WARP) {
    if (lane == 0) {
      for (int s = 0; s < NST; ++s) {
        mbar_init(full_bar(s), PROD_THREADS);
        mbar_init(empty_bar(s), 1);
      }
      mbar_init(accf_bar, 1);
      mbar_init(acce_bar, 128);
      mbar_init(drain_bar, 1);
      *abort_flag = 0;
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32((const void*)tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < PROD_A_WARPS + PROD_B_WARPS) {
    // ------------------------------------------------------------ producers
    const bool side_a = warp < PROD_A_WARPS;
    const int r = side_a ? threadIdx.x : threadIdx.x - PROD_A_WARPS * 32;
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < sc.tiles; tile += gridDim.x) {
      int bh, a0, b0;
      tile_coords(g, sc, tile, bh, a0, b0);
      const int row = side_a ? a0 + r : b0 + r;
      const bool valid = side_a ? row < g.n : row < g.m;
      const int16_t* src = side_a ? g.ka + ((size_t)bh * g.n + (valid ? row : 0)) * g.d
                                  : g.vb + ((size_t)bh * g.m + (valid ? row : 0)) * g.d;
      for (int u = 0; u < sc.nunits; ++u) {
        const int d0 = u * sc.unit_d, d1 = min(d0 + sc.unit_d, g.d);
        const int nst = stages_of_unit<TLEN>(d1 - d0) * spd;
        for (int st = 0; st < nst; ++st, ++it) {
          const int s = it % NST;
          if (!mbar_wait(empty_bar(s), ((it / NST) & 1) ^ 1, abort_flag, side_a ? 1 : 2)) goto done;
          const uint32_t stage = sbase + s * STAGE_BYTES;
          const int dfirst = d0 + (st / spd) * DPS;
          const int tbase = (st % spd) * TLEN;
#pragma unroll
          for (int dl = 0; dl < DPS; ++dl) {
            const int d = dfirst + dl;
            const int kv = (valid && d < d1) ? (int)__ldg(src + d) : 0;
            const int mag = kv < 0 ? -kv : kv;
            if (side_a) {
              const uint32_t fill = kv < 0 ? 0xFFFFFFFFu : 0x01010101u;
#pragma unroll
              for (int c = 0; c < TLEN / 16; ++c) {
                const int r8 = 8 * (mag - tbase - 16 * c);
                uint32_t w[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const int sh = max(r8 - 32 * j, 0);
                  w[j] = fill & __funnelshift_lc(0xFFFFFFFFu, 0u, (uint32_t)sh);
                }
                st_shared_v4(swz(stage, A_ATOM, r, dl * (TLEN / 16) + c), w[0], w[1], w[2], w[3]);
              }
            } else {
              const uint32_t mult = kv < 0 ? 0xFFu : 1u;
              uint32_t pw[TLEN / 32];
              if (valid && d < d1 && mag != 0) {
                const uint32_t* p = g.pattern +
                                    ((size_t)__ldg(g.bmap + d) * (g.vcap + 1) + mag) * (g.lp / 32) + tbase / 32;
#pragma unroll
                for (int x = 0; x < TLEN / 32; ++x) pw[x] = __ldg(p + x);
              } else {
#pragma unroll
                for (int x = 0; x < TLEN / 32; ++x) pw[x] = 0u;
              }
#pragma unroll
              for (int c = 0; c < TLEN / 16; ++c) {
                const uint32_t bits = (pw[c >> 1] >> (16 * (c & 1))) & 0xFFFFu;
                uint32_t w[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const uint32_t nib = (bits >> (4 * j)) & 0xFu;
                  w[j] = ((nib * 0x00204081u) & 0x01010101u) * mult;
                }
                st_shared_v4(swz(stage + A_BYTES, B_ATOM, r, dl * (TLEN / 16) + c), w[0], w[1], w[2], w[3]);
              }
            }
          }
          fence_proxy_async();
          mbar_arrive(full_bar(s));
        }
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t it = 0, uc = 0;
      for (int tile = blockIdx.x; tile < sc.tiles; tile += gridDim.x) {
        for (int u = 0; u < sc.nunits; ++u, ++uc) {
          if (!mbar_wait(acce_bar, (uc & 1) ^ 1, abort_flag, 4)) goto mma_done;
          tc_fence_after();
          const int d0 = u * sc.unit_d, d1 = min(d0 + sc.unit_d, g.d);
          const int nst = stages_of_unit<TLEN>(d1 - d0) * spd;
          for (int st = 0; st < nst; ++st, ++it) {
            const int s = it % NST;
            if (!mbar_wait(full_bar(s), (it / NST) & 1, abort_flag, 3)) goto mma_done;
            tc_fence_after();
            const uint32_t a_base = sbase + s * STAGE_BYTES, b_base = a_base + A_BYTES;
#pragma unroll
            for (int kk = 0; kk < KS / 32; ++kk) {
              const uint32_t off = (kk & 3) * 32;
              mma_i8(tmem, smem_desc(a_base + (kk >> 2) * A_ATOM + off),
                     smem_desc(b_base + (kk >> 2) * B_ATOM + off), (st > 0 || kk > 0) ? 1u : 0u);
            }
            mma_commit(empty_bar(s));
          }
          mma_commit(accf_bar);
        }
      }
    mma_done:
      // drain: completes once every MMA issued above has finished; waited on
      // even after an abort, so tensor memory is never freed under a live MMA
      mma_commit(drain_bar);
      {
        int zero = 0;
        mbar_wait(drain_bar, 0, &zero, 6);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16);
    uint32_t uc = 0;
    for (int tile = blockIdx.x; tile < sc.tiles; tile += gridDim.x) {
      int bh, a0, b0;
      tile_coords(g, sc, tile, bh, a0, b0);
      const int ia = a0 + 32 * q + lane;
      const bool chunked = g.epi.kind == EPI_CHUNK;
      for (int u = 0; u < sc.nunits; ++u, ++uc) {
        if (!mbar_wait(accf_bar, uc & 1, abort_flag, 5)) goto done;
        tc_fence_after();
        const bool last = u == sc.nunits - 1;
#pragma unroll 1
        for (int cb = 0; cb < BN / 32; ++cb) {
          uint32_t acc[32], run[32];
          TMEM_LD32(lane_addr + cb * 32, acc);
          if (chunked && u > 0) TMEM_LD32(lane_addr + 256 + cb * 32, run);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int ib = b0 + cb * 32 + j;
            float v = 0.f;
            if (ia < g.n && ib < g.m)
              v = epi_value(g.epi, (int)acc[j], bh * g.n + ia, bh * g.m + ib, bh, u, g.n, g.m);
            if (chunked) v = fadd(u > 0 ? __uint_as_float(run[j]) : 0.f, v);
            run[j] = __float_as_uint(v);
          }
          if (!chunked || last) {
            if (ia < g.n) {
              float* o = g.out + ((size_t)bh * g.n + ia) * g.m;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int ib = b0 + cb * 32 + j;
                if (ib < g.m) o[ib] = __uint_as_float(run[j]);
              }
            }
          } else {
            TMEM_ST32(lane_addr + 256 + cb * 32, run);
          }
        }
        if (chunked && !last) tmem_wait_st();
        tc_fence_before();
        mbar_arrive(acce_bar);
      }
    }
  }
done:
  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS)
                 : "memory");
  }
}

template <int TLEN>
static cudaError_t launch_t(const GemmArgs& g, const Sched& s, int spd, int grid, cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    cudaError_t e =
        cudaFuncSetAttribute(gemm_tc_kernel<TLEN>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  gemm_tc_kernel<TLEN><<<grid, THREADS, SMEM_BYTES, st>>>(g, s, spd);
  return cudaGetLastError();
}

}  // namespace tc

bool gemm_tc_supported(const GemmArgs& g) {
  if (g.n <= 0 || g.m <= 0 || g.d <= 0) return false;
  if (g.lp < 32 || (g.lp & (g.lp - 1))) return false;  // power of two >= 32
  if ((long long)g.d * g.L >= (1LL << 31)) return false;
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return major == 10 && minor == 0;
}

cudaError_t launch_gemm_tc(const GemmArgs& g, cudaStream_t st) {
  using namespace tc;
  Sched s{};
  s.tiles_a = cdiv(g.n, BM);
  s.tiles_b = cdiv(g.m, BN);
  s.tiles = g.batch * s.tiles_a * s.tiles_b;
  s.unit_d = g.unit_d > 0 ? g.unit_d : g.d;
  s.nunits = cdiv(g.d, s.unit_d);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = s.tiles < sms ? s.tiles : sms;
  const int tlen = g.lp < 256 ? g.lp : 256;
  const int spd = g.lp / tlen;
  switch (tlen) {
    case 32: return launch_t<32>(g, s, spd, grid, st);
    case 64: return launch_t<64>(g, s, spd, grid, st);
    case 128: return launch_t<128>(g, s, spd, grid, st);
    default: return launch_t<256>(g, s, spd, grid, st);
  }
}

}  // namespace scmp
