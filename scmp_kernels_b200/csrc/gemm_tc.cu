// tcgen05 SC-GEMM for sm_100a.
//
// The reference's integer accumulator (sc/kernels.py:216-245)
//   S[i][j] = sum_d sa*sb * #{t < k[i][d] : rb_d[t] < v[j][d]}
// is a GEMM over K = D * L:
//   A'[i][(d,t)] = sa[i][d] * [t < k[i][d]]          (thermometer of a)
//   B'[j][(d,t)] = sb[j][d] * [rb_d[t] < v[j][d]]    (comparator stream of b)
// with every entry in {-1, 0, 1}. Neither operand exists in memory: producer
// warps expand them per pipeline stage straight into shared memory, in the
// canonical K-major 128-byte-swizzled layout, from the int16 operands of the
// quantiser (signed k, signed v) and the bit-packed streams of the table
// builder. One thread issues the MMAs into an accumulator in tensor memory;
// epilogue warps read it back with tcgen05.ld and apply the path's float32
// recipe. The accumulation is exact.
//
// Operand types: e2m1 (4-bit floats 0, +1, -1; tcgen05.mma.kind::mxf4 with
// every block scale 1.0, float32 accumulator holding integers below 2^24)
// on SM pairs for streams of 64 to 512 positions, the default; int8
// (kind::i8, int32 accumulator) otherwise. e2m1 halves the shared-memory
// bytes and the producer work per K position and runs at twice the int8 MMA
// rate.
//
// Two variants share this code (template parameter PAIR):
//  - 1 SM per tile (cta_group::1): 128 a rows x 256 b rows per CTA; warps 0-3
//    expand A' (one a row per thread), warps 4-11 expand B', warp 12 issues
//    the MMAs, warps 13-16 run the epilogue;
//  - 2 SMs per tile (cta_group::2, a cluster of two CTAs): 256 a rows per
//    pair; each CTA expands its 128 a rows and its half of B'. The leader CTA
//    (rank 0) issues M=256 MMAs that read both CTAs' shared memory; producers
//    of both CTAs signal the leader's "full" barriers, the leader's commits
//    are multicast to both CTAs, and each CTA's epilogue reads its own 128
//    rows of the accumulator.
// Persistent grid over output tiles. Every mbarrier wait is bounded
// (common.cuh): on timeout the kernel records SCMP_ERR_TIMEOUT, all roles
// leave their loops, outstanding MMAs are drained and tensor memory is freed
// before the CTA exits.
#include "internal.cuh"

namespace scmp {
namespace tc {

constexpr int KS = 256;                    // K bytes per stage
constexpr int PROD_A_WARPS = 4;            // 128 a rows per CTA
// Tensor memory (512 columns): the accumulator from column 0; after it, the
// running chunk sum (chunked path, [256,512)), a second accumulator (short
// tiles, [256,512)) or, with a in tensor memory, a's stages (64 columns each).
constexpr int TMEM_COLS = 512;

// ATMEM (2-SM variant, one accumulation unit per tile): a's stages live in
// tensor memory, written by the producers with tcgen05.st and read by the
// MMA from there, so shared memory carries only b. WIDE (with ATMEM, for
// streams shorter than 256): up to 320 b rows per tile, computed as two MMAs
// of half the width per K step (the MMA's N is at most 256), so that each
// expanded a stage serves 320 columns; the accumulator takes columns [0,320)
// and a's three stages [320,512). (With 256-long streams the fifth b warp on
// one SM sub-partition costs more than the wider tile gains.)
template <int TLEN>
__host__ __device__ constexpr bool wide_tiles() { return TLEN < 256; }

// WIDE without ATMEM (SM pairs, a in shared memory): up to 512 b rows per
// tile as two MMAs of width 256 that share every a stage; the accumulator
// takes all 512 tensor-memory columns and two shared-memory stages of
// 32 + 64 KB are used.
//
// F4 (SM pairs, a in shared memory): the operands are e2m1 (4-bit) values
// 0, +1, -1 and the MMA is tcgen05.mma.kind::mxf4 with every block scale 1.0
// (E8M0 0x7F), twice the int8 MMA rate; its float32 accumulator holds the
// integer sums exactly (|S| <= D * L < 2^24). A 256-byte stage carries 512 K
// positions. The scale factors sit in tensor-memory columns
// [F4_SF_COL, F4_SF_COL + 16), so the accumulator takes at most 480 columns:
// tiles of at most 480 (wide) or 240 b rows, while shared memory and the
// producer warps stay sized for 512 / 256 rows (rows past the tile are not
// read by the MMA).
constexpr int F4_SF_COL = 480;
template <bool PAIR, bool ATMEM = false, bool WIDE_ = false, bool F4_ = false>
struct Cfg {
  static_assert(PAIR || !ATMEM, "a in tensor memory is implemented for SM pairs");
  static_assert(PAIR || !WIDE_, "wide tiles are implemented for SM pairs");
  static_assert(!F4_ || (PAIR && !ATMEM), "e2m1 operands are implemented for SM pairs with a in shared memory");
  static constexpr bool WIDE = WIDE_;                     // two half-width MMAs per K step
  static constexpr bool F4 = F4_;                         // e2m1 operands, kind::mxf4
  static constexpr int BM = 128;                          // a rows per CTA
  static constexpr int TILE_A = PAIR ? 256 : 128;         // a rows per tile
  static constexpr int TILE_B = WIDE ? (ATMEM ? 320 : 512) : 256;  // b rows per tile the shared
                                                          // memory and producers are sized for
  static constexpr int TILE_MAX = F4 ? (WIDE ? 480 : 240) : TILE_B;  // most b rows per tile; the
                                                          // schedule's tile_b <= TILE_MAX is used
  static constexpr int ACC_STRIDE = F4 ? 240 : 256;       // columns between accumulator buffers
  static constexpr int BNL = TILE_B / (PAIR ? 2 : 1);     // b rows per CTA
  static constexpr int TMEM_A = TILE_B;                   // first tensor-memory column of a's stages
  static constexpr int NST = WIDE ? (ATMEM ? 3 : 2) : ATMEM ? 4 : PAIR ? 3 : 2;  // pipeline stages
  static constexpr int A_BYTES = ATMEM ? 0 : BM * KS;     // a's bytes of a smem stage
  static constexpr int B_BYTES = BNL * KS;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int A_ATOM = BM * 128;                 // one 128-byte-wide K atom
  static constexpr int B_ATOM = BNL * 128;
  static constexpr int PROD_B_WARPS = BNL / 32;
  static constexpr int PROD_WARPS = PROD_A_WARPS + PROD_B_WARPS;
  // With one accumulator (wide tiles) the MMAs and the epilogue of a tile never
  // overlap, so the first epilogue warp's lane 0 (leader CTA) issues the MMAs:
  // one warp fewer leaves more registers per thread (the block's warps are
  // allocated registers in groups of four).
  static constexpr bool MERGED = WIDE;
  static constexpr int MMA_WARP = PROD_WARPS;
  static constexpr int EPI_WARP0 = MERGED ? MMA_WARP : MMA_WARP + 1;
  static constexpr int NWARPS = EPI_WARP0 + 4;
  static constexpr int THREADS = NWARPS * 32;
  // epilogue staging: 4 warps x 32 rows x 32 result columns (float32)
  static constexpr int STG_BYTES = 4 * 32 * 32 * 4;
  static constexpr int SB_BYTES = TILE_B * 4;            // a chunk's column scales (chunked path)
  static constexpr int SMEM_BYTES = NST * STAGE_BYTES + STG_BYTES + SB_BYTES + 1024 + 256;
  static constexpr int NCTA = PAIR ? 2 : 1;
  // kind::i8, D = s32, A = B = s8, K-major, M = 128 per SM; N from idesc_n().
  // kind::mxf4: A = B = E2M1, scale factors E8M0, K-major, K = 64, scale
  // factor ids 0; N from idesc_n().
  static constexpr uint32_t IDESC_M =
      F4 ? ((1u << 7) | (1u << 10) | (1u << 23) | ((uint32_t)((PAIR ? 256 : 128) >> 4) << 24))
         : ((2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)((PAIR ? 256 : 128) >> 4) << 24));
  __device__ static uint32_t idesc_n(int n) { return IDESC_M | ((uint32_t)(n >> 3) << 17); }
};

// Positions of the stream per 256-byte stage (one byte per int8 value, half a
// byte per e2m1 value) and the dimensions a stage covers for padded stream
// length TLEN (TLEN = 256 * SPD covers one dimension in SPD stages).
template <bool F4>
__host__ __device__ constexpr int stage_positions() { return F4 ? 512 : 256; }
template <int TLEN, bool F4>
__host__ __device__ constexpr int dims_per_stage() {
  return TLEN < stage_positions<F4>() ? stage_positions<F4>() / TLEN : 1;
}

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
template <bool PAIR>
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t acc) {
  if constexpr (PAIR) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
  }
}
// M=256 N=256 K=32 pair MMA with a read from tensor memory (column a_tmem of
// lanes 0..127 in both CTAs) and b from shared memory.
__device__ __forceinline__ void mma_i8_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                          uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// kind::mxf4 MMA (M = 256 over the pair or 128, N from idesc, K = 64) with
// both operands in shared memory and the scale factors of a and b at
// tensor-memory address sf (all 1.0).
template <bool PAIR>
__device__ __forceinline__ void mma_f4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t acc, uint32_t sf) {
  if constexpr (PAIR) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%5], p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(sf)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%5], p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(sf)
        : "memory");
  }
}
// Arrive on `bar` (same offset) in every CTA of the tile once all MMAs issued
// so far by this thread have completed.
template <bool PAIR>
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  if constexpr (PAIR) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
        "h"((uint16_t)0x3)
        : "memory");
  } else {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
  }
}
// Arrive on the barrier at smem offset `bar` of the tile's leader CTA (rank 0):
// a local arrive in the leader, a remote one (through mapa) from the peer.
template <bool PAIR>
__device__ __forceinline__ void mbar_arrive_leader(uint32_t bar, uint32_t rank) {
  if (PAIR && rank != 0) {
    asm volatile(
        "{\n\t.reg .b32 ra;\n\t"
        "mapa.shared::cluster.u32 ra, %0, 0;\n\t"
        "mbarrier.arrive.shared::cluster.b64 _, [ra];\n\t}" ::"r"(bar)
        : "memory");
  } else {
    mbar_arrive(bar);
  }
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

#define TMEM_LD16(taddr, r)                                                                        \
  asm volatile(                                                                                    \
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14," \
      "%15}, [%16];"                                                                               \
      : "=r"((r)[0]), "=r"((r)[1]), "=r"((r)[2]), "=r"((r)[3]), "=r"((r)[4]), "=r"((r)[5]),      \
        "=r"((r)[6]), "=r"((r)[7]), "=r"((r)[8]), "=r"((r)[9]), "=r"((r)[10]), "=r"((r)[11]),      \
        "=r"((r)[12]), "=r"((r)[13]), "=r"((r)[14]), "=r"((r)[15])                                 \
      : "r"(taddr))
#define TMEM_ST16(taddr, r)                                                                        \
  asm volatile(                                                                                    \
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13," \
      "%14,%15,%16};" ::"r"(taddr),                                                                \
      "r"((r)[0]), "r"((r)[1]), "r"((r)[2]), "r"((r)[3]), "r"((r)[4]), "r"((r)[5]), "r"((r)[6]),  \
      "r"((r)[7]), "r"((r)[8]), "r"((r)[9]), "r"((r)[10]), "r"((r)[11]), "r"((r)[12]),             \
      "r"((r)[13]), "r"((r)[14]), "r"((r)[15]))

#define TMEM_LD8(taddr, r)                                                                         \
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"            \
               : "=r"((r)[0]), "=r"((r)[1]), "=r"((r)[2]), "=r"((r)[3]), "=r"((r)[4]), "=r"((r)[5]), \
                 "=r"((r)[6]), "=r"((r)[7])                                                         \
               : "r"(taddr))
#define TMEM_ST8(taddr, r)                                                                         \
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), \
               "r"((r)[0]), "r"((r)[1]), "r"((r)[2]), "r"((r)[3]), "r"((r)[4]), "r"((r)[5]), "r"((r)[6]), \
               "r"((r)[7]))

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}

// Result rows ia0 .. ia0+31 (lane l holds row ia0 + l in v), columns
// ib0 .. ib0+31, to every destination of the result (the columns < m_end, the
// end of the tile's columns, of the rows < n). The warp transposes through its 4 KB staging area `stg` so that
// each store instruction writes four 128-byte row segments (16 bytes per
// lane) instead of 32 scattered words: full lines for local HBM and for a
// peer's memory over NVLink alike. Chunks are XOR-swizzled by row, so both
// the row-wise writes and the segment-wise reads are free of bank conflicts.
// only >= 0: store to destination `only` alone (the tile's peer copies are
// made later by copy_rows_to_peers).
__device__ __forceinline__ void store_rows32(const GemmArgs& g, uint32_t stg, int bh, int ia0, int ib0, int m_end,
                                             const uint32_t (&v)[32], int lane, int only = -1) {
#pragma unroll
  for (int k = 0; k < 8; ++k)
    st_shared_v4(stg + lane * 128 + ((k ^ (lane & 7)) << 4), v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
  __syncwarp();
  const int c = lane & 7;  // 16-byte chunk of the row segment this lane writes
  const int ib = ib0 + 4 * c;
#pragma unroll 1
  for (int rr = 0; rr < 8; ++rr) {
    const int r = 4 * rr + (lane >> 3);
    const uint4 x = ld_shared_v4(stg + r * 128 + ((c ^ (r & 7)) << 4));
    const int ia = ia0 + r;
    // result row (with row levels, the permuted row's place in the result)
    int orow = ia < g.n ? ia : -1;
    if (g.row_of && orow >= 0) orow = __ldg(g.row_of + ia);
    if (orow >= 0 && ib < m_end) {
      const long long idx = g.out_off + ((long long)bh * (g.row_of ? g.n_out : g.n) + orow) * g.out_ld + ib;
      const bool whole = g.out_vec && ib + 3 < m_end;
#pragma unroll 1
      for (int k = only < 0 ? 0 : only; k < (only < 0 ? g.nouts : only + 1); ++k) {
        float* o = g.outs[k] + idx;
        if (whole) {
          *reinterpret_cast<uint4*>(o) = x;
        } else {
          o[0] = __uint_as_float(x.x);
          if (ib + 1 < m_end) o[1] = __uint_as_float(x.y);
          if (ib + 2 < m_end) o[2] = __uint_as_float(x.z);
          if (ib + 3 < m_end) o[3] = __uint_as_float(x.w);
        }
      }
    }
  }
  __syncwarp();
}

// Copies the tile block rows [ia0, ia0 + nrows) x columns [ib0, m_end) of
// batch entry bh from destination `self` (this device's memory, where the
// epilogue stored it) to every other destination, one warp over the rows
// r0, r0 + rstep, ...: 16 bytes per lane, a row segment per instruction.
// Reads bypass L1 (the rows were written by other warps of the CTA).
__device__ __forceinline__ void copy_rows_to_peers(const GemmArgs& g, int self, int bh, int ia0, int nrows, int ib0,
                                                   int m_end, int r0, int rstep, int lane) {
  const int ncol = m_end - ib0;
  const long long rows_base = (long long)bh * (g.row_of ? g.n_out : g.n);
#pragma unroll 1
  for (int r = r0; r < nrows; r += rstep) {
    const int ia = ia0 + r;
    int orow = ia < g.n ? ia : -1;
    if (g.row_of && orow >= 0) orow = __ldg(g.row_of + ia);
    if (orow < 0) continue;
    const long long base = g.out_off + (rows_base + orow) * g.out_ld + ib0;
    const float* src = g.outs[self] + base;
    if (g.out_vec) {
#pragma unroll 1
      for (int c = 4 * lane; c < ncol; c += 128) {
        if (c + 3 < ncol) {
          const float4 x = __ldcg(reinterpret_cast<const float4*>(src + c));
#pragma unroll 1
          for (int k = 0; k < g.nouts; ++k)
            if (k != self) *reinterpret_cast<float4*>(g.outs[k] + base + c) = x;
        } else {
          for (int e = c; e < ncol; ++e) {
            const float x = __ldcg(src + e);
            for (int k = 0; k < g.nouts; ++k)
              if (k != self) g.outs[k][base + e] = x;
          }
        }
      }
    } else {
#pragma unroll 1
      for (int c = lane; c < ncol; c += 32) {
        const float x = __ldcg(src + c);
#pragma unroll 1
        for (int k = 0; k < g.nouts; ++k)
          if (k != self) g.outs[k][base + c] = x;
      }
    }
  }
}

// Integer value of an accumulator word: int32 for kind::i8, a float32 holding
// an integer below 2^24 in magnitude for kind::mxf4 (exact conversion).
template <bool F4>
__device__ __forceinline__ int acc_int(uint32_t w) {
  if constexpr (F4) return __float2int_rz(__uint_as_float(w));
  return (int)w;
}

struct Sched {
  int tiles, tiles_a, tiles_b, nunits, unit_d, tile_a, tile_b;
  int full;     // whole tiles, taken round-robin by the workers (a multiple of `workers` with a tail)
  int workers;  // workers of the persistent grid (SM pairs or SMs)
  int tail_w;   // workers sharing the tail tiles' K range (0: no tail)
  int tail_blk; // blocks of eight dimensions in the tail: (tiles - full) * nblk
  int nwork, nblk;
  int band_group;  // bands of a per group of the tile order (tile_coords)
};

// Work items of a worker: whole tiles w = worker, worker + workers, ... < full,
// then (with a tail) its two tail pieces w = full + worker + j * workers. The
// tail is the last `tiles - full` tiles' K ranges laid end to end (tile after
// tile, blocks of eight dimensions) and cut into tail_w equal ranges, one per
// worker ("stream-K"), so every worker ends at the same time; a range spans at
// most two tiles, piece j of the worker being its part in the j-th of them.
struct Work {
  int tile;  // output tile
  int part;  // slot of a tail piece (2 * worker + j), -1 for a whole tile
  int d0, d1;  // dimension range of a piece (d0 == d1: no work)
};

__host__ __device__ __forceinline__ int tail_lo(const Sched& s, int u) {  // first block of worker u's range
  return (int)((long long)u * s.tail_blk / s.tail_w);
}
// Worker whose range holds tail block x: the largest u with tail_lo(u) <= x.
__host__ __device__ __forceinline__ int tail_worker(const Sched& s, int x) {
  return (int)(((long long)(x + 1) * s.tail_w - 1) / s.tail_blk);
}

__device__ __forceinline__ Work work_of(const Sched& s, int w, int d) {
  Work k;
  k.tile = w;
  k.part = -1;
  k.d0 = 0;
  k.d1 = d;
  if (w >= s.full) {
    const int v = w - s.full;
    const int u = v % s.workers, j = v / s.workers;
    k.part = 2 * u + j;
    k.tile = s.full;
    k.d0 = k.d1 = 0;
    if (u < s.tail_w) {
      const int lo = tail_lo(s, u), hi = tail_lo(s, u + 1);
      const int t = lo / s.nblk + j;  // tail tile of piece j
      const int b0 = j == 0 ? lo : t * s.nblk;
      const int b1 = min(hi, (t + 1) * s.nblk);
      if (b1 > b0) {
        k.tile = s.full + t;
        k.d0 = 8 * (b0 - t * s.nblk);
        k.d1 = min(8 * (b1 - t * s.nblk), d);
      }
    }
  }
  return k;
}
// Accumulation units of a work item and the dimension range of unit u.
__device__ __forceinline__ int units_of(const Sched& s, const Work& k) {
  return k.part < 0 ? s.nunits : (k.d1 > k.d0 ? 1 : 0);
}
__device__ __forceinline__ void unit_range(const Sched& s, const Work& k, int u, int d, int& d0, int& d1) {
  if (k.part < 0) {
    d0 = u * s.unit_d;
    d1 = min(d0 + s.unit_d, d);
  } else {
    d0 = k.d0;
    d1 = k.d1;
  }
}

// Tile order: bands of a (tile_a rows) in groups of `band_group`; inside a
// group, b's tiles one after another, each for every band of the group, so
// that the tiles running at the same time share b's operand rows and the
// group's a rows in L2.
__device__ __forceinline__ void tile_coords(const Sched& s, int tile, int& bh, int& a0, int& b0) {
  const int per = s.tiles_a * s.tiles_b;
  bh = tile / per;
  const int r = tile % per;
  const int G = s.band_group;
  const int grp = r / (G * s.tiles_b), j = r % (G * s.tiles_b);
  const int gb = min(G, s.tiles_a - grp * G);  // bands in this group (the last may have fewer)
  a0 = (grp * G + j % gb) * s.tile_a;
  b0 = (j / gb) * s.tile_b;
}

template <int TLEN, int SPD, bool F4 = false>
__host__ __device__ constexpr int SPB() {  // stages per block of eight dimensions
  return (8 / dims_per_stage<TLEN, F4>()) * SPD;
}

// Signed value of dimension e (0..7, compile-time after unrolling) of a block.
__device__ __forceinline__ int kv_at(const uint4& v, int e) {
  const uint32_t w = e < 2 ? v.x : e < 4 ? v.y : e < 6 ? v.z : v.w;
  return (int)(int16_t)((e & 1) ? (w >> 16) : (w & 0xFFFFu));
}
__device__ __forceinline__ int bm_at(const int4& lo, const int4& hi, int e) {
  return e == 0 ? lo.x : e == 1 ? lo.y : e == 2 ? lo.z : e == 3 ? lo.w
       : e == 4 ? hi.x : e == 5 ? hi.y : e == 6 ? hi.z : hi.w;
}

// The stream words that stage j of a block expands (8 for int8 operands, 16
// for e2m1): for each of its DPS dimensions, TLEN bits of the row (bmap, |v|)
// of `pat`, starting at bit (j % SPD) * TLEN. Dimensions past d1, rows past
// the tile (`valid` false, their values zero) and v == 0 give zeros. With
// streams of at most 64 positions, v == 0 and rows past the tile read the
// table's entry 0 (all zeros) instead, so that the test that selects the load
// is the same for every lane of the warp (config 5: 2% faster; with longer
// streams, 32-byte loads, skipping them is 1% faster).
template <int TLEN, int SPD, bool F4 = false>
__device__ __forceinline__ void load_stream_words(int vcap1, const uint32_t* __restrict__ pat,
                                                  const uint4& kv, const int4& bl, const int4& bh, int j,
                                                  int dbase, int d1, bool valid, uint32_t LW,
                                                  uint32_t (&pw)[F4 ? 16 : 8]) {
  constexpr int DPS = dims_per_stage<TLEN, F4>();
  constexpr int NW = TLEN / 32 < 16 ? TLEN / 32 : 16;  // words of one dimension in the stage
  static_assert(DPS * NW == (F4 ? 16 : 8), "a stage is 8 (int8) or 16 (e2m1) stream words");
#pragma unroll
  for (int dl = 0; dl < DPS; ++dl) {
    const int e = (j / SPD) * DPS + dl;
    const int v = kv_at(kv, e);
    const int mag = v < 0 ? -v : v;
    if (TLEN <= 64 ? dbase + e < d1 : (valid && dbase + e < d1 && mag != 0)) {
      const uint32_t* p = pat + ((size_t)bm_at(bl, bh, e) * vcap1 + mag) * LW + (j % SPD) * NW;
      if constexpr (NW >= 4) {
#pragma unroll
        for (int x = 0; x < NW / 4; ++x) {
          const uint4 y = __ldg(reinterpret_cast<const uint4*>(p) + x);
          pw[dl * NW + 4 * x] = y.x;
          pw[dl * NW + 4 * x + 1] = y.y;
          pw[dl * NW + 4 * x + 2] = y.z;
          pw[dl * NW + 4 * x + 3] = y.w;
        }
      } else if constexpr (NW == 2) {
        const uint2 x = __ldg(reinterpret_cast<const uint2*>(p));
        pw[dl * 2] = x.x;
        pw[dl * 2 + 1] = x.y;
      } else {
        pw[dl] = __ldg(p);
      }
    } else {
#pragma unroll
      for (int x = 0; x < NW; ++x) pw[dl * NW + x] = 0u;
    }
  }
}

template <int TLEN, bool F4 = false>
__device__ __forceinline__ int stages_of_unit(int len) {
  if (TLEN < stage_positions<F4>()) return cdiv(len, dims_per_stage<TLEN, F4>());
  return len * (TLEN / stage_positions<F4>());
}

// Producer loop of one operand side. Operands arrive in blocks of eight
// dimensions: one 16-byte load per thread (its row's signed k or v values,
// blocked layout) and, for b, two 16-byte loads of the block's table rows.
// Blocks are fetched one block ahead and b's stream words one stage ahead, so
// the loads are in flight while the producer waits for its shared-memory
// slot. Stages are not unrolled (the instruction cache holds both sides'
// loops); the chunks of a stage are. Returns false after an abort.
// With ATMEM, side a writes its row's 64 columns of each stage to tensor
// memory at tmem_a (this thread's lane, first stage column) instead.
// With F4 the words are e2m1: eight 4-bit values (0, +1 = 0x2, -1 = 0xA) per
// 32-bit word, so a 16-byte chunk covers 32 positions instead of 16.
// b's side of one work item: its quantised operand, stream table and row map
// (one set per call, or the level's with row levels).
struct BSide {
  const uint32_t* pat;
  const uint4* kv;
  const int4* bm;
  uint32_t LW;
  int vcap1;
};

// Level of the a tile starting at permuted row a0, -1 for a tile past the
// last level (row levels only).
__device__ __forceinline__ int level_of(const GemmArgs& g, int a0) {
  const int t = a0 >> 8;
  for (int l = 0; l < g.nlev; ++l)
    if (t < __ldg(g.lev_tile0 + l + 1)) return l;
  return -1;
}

// Stages of an accumulation unit of `len` dimensions for padded stream
// length lp (runtime form of stages_of_unit for the row-level kernel).
__device__ __forceinline__ int stages_rt(int lp, bool f4, int len) {
  const int sp = f4 ? 512 : 256;
  return lp < sp ? cdiv(len, sp / lp) : len * (lp / sp);
}

// The stages of one work item (all its accumulation units).
template <bool SIDE_A, int TLEN, int SPD, bool PAIR, bool ATMEM, bool WIDE, bool F4, bool UNR>
__device__ __forceinline__ bool produce_item(const GemmArgs& g, const Sched& sc, const Work& wk, const BSide& bs,
                                             uint32_t sbase, uint32_t bar_base, volatile int* abort_flag,
                                             uint32_t rank, int r, int lane, uint32_t tmem_a,
                                             const uint32_t (&xo)[8], uint32_t& it) {
  using C = Cfg<PAIR, ATMEM, WIDE, F4>;
  constexpr int NST = C::NST;
  constexpr int DPS = dims_per_stage<TLEN, F4>();
  constexpr int NSPB = SPB<TLEN, SPD, F4>();
  constexpr int NPW = F4 ? 16 : 8;  // stream words per stage
  // 16-byte chunks of one dimension in a stage
  constexpr int CPDS = (TLEN < stage_positions<F4>() ? TLEN : stage_positions<F4>()) / (F4 ? 32 : 16);
  const int R = SIDE_A ? g.batch * g.n : g.batch * g.m;
  const uint4* kvsrc = SIDE_A ? reinterpret_cast<const uint4*>(g.ka) : bs.kv;
  const int4* bmsrc = bs.bm;
  const uint32_t LW = bs.LW;
  {
    int bh, a0, b0;
    tile_coords(sc, wk.tile, bh, a0, b0);
    // b: the tile's tile_b rows, tile_b / NCTA per CTA (rows past them are not
    // read). A pair MMA of width N takes its first N/2 columns from CTA 0's
    // rows and the rest from CTA 1's; wide tiles stack two such MMAs of width
    // nh = tile_b / 2, so smem row r of CTA c is column h*nh + c*nh/2 + r' of
    // the tile (h = r / (nh/2), r' = r % (nh/2)).
    const int bnl = sc.tile_b / C::NCTA;
    int bcol = (int)rank * bnl + r;
    if constexpr (C::WIDE) {
      const int hh = sc.tile_b / 4;
      bcol = (r / hh) * (2 * hh) + (int)rank * hh + r % hh;
    }
    const int row = SIDE_A ? a0 + (int)rank * C::BM + r : b0 + bcol;
    const bool valid = SIDE_A ? row < g.n : (r < bnl && row < g.m);
    const int grow = bh * (SIDE_A ? g.n : g.m) + (valid ? row : 0);
    const int nu = units_of(sc, wk);
    for (int u = 0; u < nu; ++u) {
      int d0, d1;
      unit_range(sc, wk, u, g.d, d0, d1);
      const int nst = stages_of_unit<TLEN, F4>(d1 - d0) * SPD;
      const int nblk = cdiv(d1 - d0, 8);
      const int blk0 = d0 >> 3;
      uint4 kv_cur = valid ? __ldg(kvsrc + (size_t)blk0 * R + grow) : make_uint4(0, 0, 0, 0);
      int4 bm_lo = make_int4(0, 0, 0, 0), bm_hi = make_int4(0, 0, 0, 0);
      uint32_t pw[NPW];
      if (!SIDE_A) {
        bm_lo = __ldg(bmsrc + 2 * blk0);
        bm_hi = __ldg(bmsrc + 2 * blk0 + 1);
        load_stream_words<TLEN, SPD, F4>(bs.vcap1, bs.pat, kv_cur, bm_lo, bm_hi, 0, d0, d1, valid, LW, pw);
      }
      // Blocks of one stage (64-long e2m1 streams): the next block's operand
      // values (and table rows) are loaded two blocks ahead, so that a whole
      // stage hides their latency; longer blocks load one block ahead.
      uint4 kv_ahead = make_uint4(0, 0, 0, 0);
      int4 ab_lo = make_int4(0, 0, 0, 0), ab_hi = make_int4(0, 0, 0, 0);
      if constexpr (NSPB == 1) {
        if (nblk > 1) {
          if (valid) kv_ahead = __ldg(kvsrc + (size_t)(blk0 + 1) * R + grow);
          if (!SIDE_A) {
            ab_lo = __ldg(bmsrc + 2 * (blk0 + 1));
            ab_hi = __ldg(bmsrc + 2 * (blk0 + 1) + 1);
          }
        }
      }
      for (int blk = 0; blk < nblk; ++blk) {
        const int dbase = d0 + 8 * blk;
        const bool more = blk + 1 < nblk;
        uint4 kv_nxt = make_uint4(0, 0, 0, 0);
        int4 nb_lo = make_int4(0, 0, 0, 0), nb_hi = make_int4(0, 0, 0, 0);
        if constexpr (NSPB == 1) {
          kv_nxt = kv_ahead;  // block blk + 1 (zeros past the last)
          nb_lo = ab_lo;
          nb_hi = ab_hi;
          kv_ahead = make_uint4(0, 0, 0, 0);
          if (blk + 2 < nblk) {
            if (valid) kv_ahead = __ldg(kvsrc + (size_t)(blk0 + blk + 2) * R + grow);
            if (!SIDE_A) {
              ab_lo = __ldg(bmsrc + 2 * (blk0 + blk + 2));
              ab_hi = __ldg(bmsrc + 2 * (blk0 + blk + 2) + 1);
            }
          }
        } else if (more) {
          if (valid) kv_nxt = __ldg(kvsrc + (size_t)(blk0 + blk + 1) * R + grow);
          if (!SIDE_A) {
            nb_lo = __ldg(bmsrc + 2 * (blk0 + blk + 1));
            nb_hi = __ldg(bmsrc + 2 * (blk0 + blk + 1) + 1);
          }
        }
        if constexpr (NSPB <= 2) {
          // short streams: a block is one or two stages, so the operand load
          // one block ahead has little time to arrive; the row's block
          // PF blocks ahead is fetched into L2 now
          constexpr int PF = NSPB == 1 ? 4 : 2;
          if (valid && blk + PF < nblk)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(kvsrc + (size_t)(blk0 + blk + PF) * R + grow));
        }
        const int jmax = min(NSPB, nst - blk * NSPB);
        // UNR (e2m1 long tiles and the chunked path): the block's stages are
        // unrolled, so every dimension index below is a compile-time constant
        // (no selects on kv, bm); measured 6.7% faster on config 2 and 4.5%
        // on config 4. int8 (twice the stages per block) keeps the loop
        // rolled so that it stays in the instruction cache, and so do the
        // short-tile kernels (slower unrolled).
        constexpr int UNROLL = UNR ? NSPB : 1;
#pragma unroll UNROLL
        for (int j = 0; j < NSPB; ++j) {
          if (j >= jmax) break;
          uint32_t pn[NPW];
          if (!SIDE_A) {
            if (j + 1 < NSPB)
              load_stream_words<TLEN, SPD, F4>(bs.vcap1, bs.pat, kv_cur, bm_lo, bm_hi, j + 1, dbase, d1, valid, LW, pn);
            else
              load_stream_words<TLEN, SPD, F4>(bs.vcap1, bs.pat, kv_nxt, nb_lo, nb_hi, 0, dbase + 8, more ? d1 : dbase, valid,
                                               LW, pn);
          }
          const int s = it % NST;
          if (!mbar_wait(bar_base + 8u * (NST + s), ((it / NST) & 1) ^ 1, abort_flag, SIDE_A ? 1 : 2))
            return false;
          const uint32_t stage = sbase + s * C::STAGE_BYTES + (SIDE_A ? 0 : C::A_BYTES);
          const int tbase = (j % SPD) * TLEN;
          if constexpr (SIDE_A && ATMEM) {
            // stage s of a in tensor memory: K bytes 4x..4x+3 in column x of
            // this row's lane, 16 columns (four 16-byte chunks) per store;
            // the MMAs that read the slot before have completed (empty barrier)
            tc_fence_after();
            constexpr int CPD = TLEN / 16;  // chunks per dimension piece
            uint32_t fillv[DPS];
            int shv[DPS];
#pragma unroll
            for (int dl = 0; dl < DPS; ++dl) {
              const int e = (j / SPD) * DPS + dl;
              const int kv = (dbase + e < d1) ? kv_at(kv_cur, e) : 0;
              fillv[dl] = kv < 0 ? 0xFFFFFFFFu : 0x01010101u;
              shv[dl] = 8 * ((kv < 0 ? -kv : kv) - tbase);
            }
#pragma unroll
            for (int grp = 0; grp < 4; ++grp) {
              uint32_t wv[16];
#pragma unroll
              for (int x = 0; x < 4; ++x) {
                const int kc = 4 * grp + x, dl = kc / CPD, c = kc % CPD;
#pragma unroll
                for (int q = 0; q < 4; ++q)
                  wv[4 * x + q] = __funnelshift_lc(fillv[dl], 0u, (uint32_t)max(shv[dl] - 32 * (4 * c + q), 0));
              }
              TMEM_ST16(tmem_a + (uint32_t)(s * 64 + 16 * grp), wv);
            }
            tmem_wait_st();
            tc_fence_before();  // the stores precede the arrive for the MMA
          } else {
#pragma unroll
            for (int dl = 0; dl < DPS; ++dl) {
              const int e = (j / SPD) * DPS + dl;  // dimension inside the block
              const int kv = (dbase + e < d1) ? kv_at(kv_cur, e) : 0;
              const int mag = kv < 0 ? -kv : kv;
              if (SIDE_A) {
                // word x of the piece holds positions PW*x .. PW*x+PW-1 (PW =
                // 4 int8 or 8 e2m1 values): its low clamp(mag - tbase - PW*x,
                // 0, PW) values are `fill`, i.e. the top bits of
                // (0:fill) << max(VB*(mag - tbase) - 32x, 0) (VB bits per
                // value), the shift clamped at 32
                const uint32_t fill = F4 ? (kv < 0 ? 0xAAAAAAAAu : 0x22222222u) : (kv < 0 ? 0xFFFFFFFFu : 0x01010101u);
                const int sh = (F4 ? 4 : 8) * (mag - tbase);
#pragma unroll
                for (int c = 0; c < CPDS; ++c) {
                  uint32_t w[4];
#pragma unroll
                  for (int q = 0; q < 4; ++q)
                    w[q] = __funnelshift_lc(fill, 0u, (uint32_t)max(sh - 32 * (4 * c + q), 0));
                  const int kc = dl * CPDS + c;
                  st_shared_v4(stage + (kc >> 3) * C::A_ATOM + xo[kc & 7], w[0], w[1], w[2], w[3]);
                }
              } else if constexpr (F4) {
                // e2m1 sliced stream words: chunk c is stream word c of the
                // dimension; its word q holds nibble-spaced bits q, q+4, ...
                // (positions 8q .. 8q+7), times 0x2 (+1) or 0xA (-1)
                const uint32_t mult = kv < 0 ? 0xAu : 0x2u;
#pragma unroll
                for (int c = 0; c < CPDS; ++c) {
                  const uint32_t sw = pw[dl * CPDS + c];
                  uint32_t w[4];
#pragma unroll
                  for (int q = 0; q < 4; ++q) w[q] = ((sw >> q) & 0x11111111u) * mult;
                  const int kc = dl * CPDS + c;
                  st_shared_v4(stage + (kc >> 3) * C::B_ATOM + xo[kc & 7], w[0], w[1], w[2], w[3]);
                }
              } else {
                // sliced stream words: chunk c's four words are the bytes'
                // bit 0 of (word >> (4*(c&1) + q)), negated for v < 0
                const uint32_t mult = kv < 0 ? 0xFFu : 1u;
#pragma unroll
                for (int c = 0; c < CPDS; ++c) {
                  const uint32_t sw = pw[dl * (TLEN / 32) + (c >> 1)];
                  uint32_t w[4];
#pragma unroll
                  for (int q = 0; q < 4; ++q) w[q] = ((sw >> (4 * (c & 1) + q)) & 0x01010101u) * mult;
                  const int kc = dl * CPDS + c;
                  st_shared_v4(stage + (kc >> 3) * C::B_ATOM + xo[kc & 7], w[0], w[1], w[2], w[3]);
                }
              }
            }
            // every lane's stores become visible to the tensor core, then one
            // lane signals the tile's leader CTA for the whole warp
            fence_proxy_async();
          }
          __syncwarp();
          if (lane == 0) mbar_arrive_leader<PAIR>(bar_base + 8u * s, rank);
          ++it;
          if (!SIDE_A) {
#pragma unroll
            for (int x = 0; x < NPW; ++x) pw[x] = pn[x];
          }
        }
        kv_cur = kv_nxt;
        bm_lo = nb_lo;
        bm_hi = nb_hi;
      }
    }
  }
  return true;
}

// Producer loop of one operand side over the worker's items. LEV (row
// levels): each item's stream length is its level's, dispatched at run time.
template <bool SIDE_A, int TLEN, int SPD, bool PAIR, bool ATMEM, bool WIDE, bool F4, bool UNR, bool LEV>
__device__ __forceinline__ bool produce(const GemmArgs& g, const Sched& sc, uint32_t sbase, uint32_t bar_base,
                                        volatile int* abort_flag, uint32_t rank, int tile0, int tstep, int r,
                                        int lane, uint32_t tmem_a) {
  // byte offset of 16-byte chunk k (0..7) of row r in a 128-byte-swizzled atom
  uint32_t xo[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) xo[k] = (uint32_t)r * 128u + (uint32_t)((k ^ (r & 7)) << 4);
  uint32_t it = 0;
  for (int w = tile0; w < sc.nwork; w += tstep) {
    const Work wk = work_of(sc, w, g.d);
    if constexpr (LEV) {
      int bh, a0, b0;
      tile_coords(sc, wk.tile, bh, a0, b0);
      const int lv = level_of(g, a0);
      if (lv < 0) continue;
      const LevelB& L = g.lev[lv];
      const BSide bs{L.pattern4, reinterpret_cast<const uint4*>(L.vb), reinterpret_cast<const int4*>(L.bmap),
                     (uint32_t)L.lp / 32, L.vcap + 1};
      bool ok;
      switch (L.lp) {
        case 64:
          ok = produce_item<SIDE_A, 64, 1, PAIR, ATMEM, WIDE, F4, UNR>(g, sc, wk, bs, sbase, bar_base, abort_flag,
                                                                      rank, r, lane, tmem_a, xo, it);
          break;
        case 128:
          ok = produce_item<SIDE_A, 128, 1, PAIR, ATMEM, WIDE, F4, UNR>(g, sc, wk, bs, sbase, bar_base, abort_flag,
                                                                       rank, r, lane, tmem_a, xo, it);
          break;
        case 256:
          ok = produce_item<SIDE_A, 256, 1, PAIR, ATMEM, WIDE, F4, UNR>(g, sc, wk, bs, sbase, bar_base, abort_flag,
                                                                       rank, r, lane, tmem_a, xo, it);
          break;
        default:
          ok = produce_item<SIDE_A, 512, 1, PAIR, ATMEM, WIDE, F4, UNR>(g, sc, wk, bs, sbase, bar_base, abort_flag,
                                                                       rank, r, lane, tmem_a, xo, it);
          break;
      }
      if (!ok) return false;
    } else {
      const BSide bs{F4 ? g.pattern4 : g.pattern, reinterpret_cast<const uint4*>(g.vb),
                     reinterpret_cast<const int4*>(g.bmap), (uint32_t)g.lp / 32, g.vcap + 1};
      if (!produce_item<SIDE_A, TLEN, SPD, PAIR, ATMEM, WIDE, F4, UNR>(g, sc, wk, bs, sbase, bar_base, abort_flag,
                                                                      rank, r, lane, tmem_a, xo, it))
        return false;
    }
  }
  return true;
}


// TLEN: padded stream length lp when lp <= 256 (256/lp dimensions per stage),
// or 256 when lp = 256*SPD (SPD stages per dimension, SPD = 1 or 2).
// LEV: row levels (GemmArgs.nlev > 0): every a tile belongs to one level,
// whose stream length (TLEN is then unused), b operand, tables and epilogue
// scale the item uses; tiles past the last level are skipped by every role.
// TAIL = false: the launch has no stream-K tail (Sched.tail_w == 0), so the
// tail pieces' epilogue is not compiled in.
template <int TLEN, int SPD, bool PAIR, bool ATMEM, bool WIDE, bool F4, bool UNR, bool LEV = false, bool TAIL = true>
__global__ void __launch_bounds__(Cfg<PAIR, ATMEM, WIDE, F4>::THREADS, 1) gemm_tc_kernel(GemmArgs g, Sched sc) {
  using C = Cfg<PAIR, ATMEM, WIDE, F4>;
  constexpr int NST = C::NST;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;  // SW128 tiles need 1024-B alignment; the
  uint8_t* gbase = smem_raw + (sbase - raw);      // offset is the same in both CTAs of a pair
  const uint32_t stg_base = sbase + NST * C::STAGE_BYTES;   // epilogue staging
  float* sbs = reinterpret_cast<float*>(gbase + NST * C::STAGE_BYTES + C::STG_BYTES);  // chunk column scales
  const uint32_t bar_base = stg_base + C::STG_BYTES + C::SB_BYTES;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (NST + s); };
  // accumulator buffers: two (tensor-memory columns [0,256) and [256,512))
  // when those columns are free (a in shared memory, one accumulation unit per
  // tile), so that a tile's epilogue overlaps the next tile's MMAs; else one
  const int nbuf = (!ATMEM && !WIDE && sc.nunits == 1) ? 2 : 1;
  auto accf_bar = [&](int b) { return bar_base + 8u * (2 * NST + b); };
  auto acce_bar = [&](int b) { return bar_base + 8u * (2 * NST + 2 + b); };
  const uint32_t drain_bar = bar_base + 8u * (2 * NST + 4);
  // wide tiles with the result's peer copies deferred (GemmArgs.out_self):
  // the epilogue warps' local stores of a tile are complete
  const uint32_t cpy_bar = bar_base + 8u * (2 * NST + 5);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + NST * C::STAGE_BYTES + C::STG_BYTES + C::SB_BYTES + 128);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + NST * C::STAGE_BYTES + C::STG_BYTES + C::SB_BYTES + 136);
  volatile int* split_flag = reinterpret_cast<volatile int*>(gbase + NST * C::STAGE_BYTES + C::STG_BYTES + C::SB_BYTES + 144);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_rank() : 0u;   // CTA rank inside the pair
  const bool leader = rank == 0;
  const int tile0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tstep = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (warp == C::MMA_WARP) {
    if (lane == 0) {
      for (int s = 0; s < NST; ++s) {
        mbar_init(full_bar(s), C::NCTA * C::PROD_WARPS);  // one arrival per producer warp of the tile
        mbar_init(empty_bar(s), 1);
      }
      for (int b = 0; b < 2; ++b) {
        mbar_init(accf_bar(b), 1);
        mbar_init(acce_bar(b), C::NCTA * 4);  // one arrival per epilogue warp of the tile
      }
      mbar_init(drain_bar, 1);
      mbar_init(cpy_bar, 4);  // one arrival per epilogue warp of the CTA
      *abort_flag = 0;
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    if constexpr (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32((const void*)tmem_slot)), "r"(TMEM_COLS) : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32((const void*)tmem_slot)), "r"(TMEM_COLS) : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the peer's barriers exist before anyone arrives on them
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if constexpr (F4) {
    // block scale factors of every MMA: E8M0 0x7F (2^0) in columns
    // [F4_SF_COL, F4_SF_COL + 16) of all 128 lanes, in both CTAs of a pair
    // (an MMA of N <= 256 reads 4 columns for a and 8 for b)
    if (warp < 4) {
      const uint32_t one[8] = {0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu,
                               0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu};
      TMEM_ST8(tmem + ((uint32_t)(32 * warp) << 16) + F4_SF_COL, one);
      TMEM_ST8(tmem + ((uint32_t)(32 * warp) << 16) + F4_SF_COL + 8, one);
      tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) cluster_sync();
    tc_fence_after();
  }

  // MMAs of accumulation unit u of work item wk into accumulator buffer uc % nbuf
  // (leader CTA, one thread); it counts the K stages consumed. False on abort.
  auto issue_unit = [&](const Work& wk, int u, uint32_t& it, uint32_t uc, int lp) -> bool {
    const int nmma = C::WIDE ? 2 : 1;  // MMAs per K step
    const int nw = sc.tile_b / nmma;   // width of each
    const uint32_t idesc = C::idesc_n(nw);
    const int buf = (int)(uc % nbuf);
    if (!mbar_wait(acce_bar(buf), ((uc / nbuf) & 1) ^ 1, abort_flag, 4)) return false;
    const uint32_t tacc = tmem + (uint32_t)(buf * C::ACC_STRIDE);
    tc_fence_after();
    int d0, d1;
    unit_range(sc, wk, u, g.d, d0, d1);
    const int nst = LEV ? stages_rt(lp, F4, d1 - d0) : stages_of_unit<TLEN, F4>(d1 - d0) * SPD;
    for (int st = 0; st < nst; ++st, ++it) {
      const int s = it % NST;
      if (!mbar_wait(full_bar(s), (it / NST) & 1, abort_flag, 3)) return false;
      tc_fence_after();
      const uint32_t a_base = sbase + s * C::STAGE_BYTES, b_base = a_base + C::A_BYTES;
#pragma unroll
      for (int kk = 0; kk < KS / 32; ++kk) {
        const uint32_t off = (kk & 3) * 32;
        const uint32_t acc = (st > 0 || kk > 0) ? 1u : 0u;
        if constexpr (ATMEM) {
#pragma unroll
          for (int h = 0; h < nmma; ++h)  // half h: columns [h*nw, (h+1)*nw), smem rows from h*nw/2
            mma_i8_ts(tacc + h * nw, tmem + C::TMEM_A + s * 64 + kk * 8,
                      smem_desc(b_base + (kk >> 2) * C::B_ATOM + h * (nw / 2) * 128 + off), idesc, acc);
        } else if constexpr (F4) {
#pragma unroll
          for (int h = 0; h < nmma; ++h)
            mma_f4<PAIR>(tacc + h * nw, smem_desc(a_base + (kk >> 2) * C::A_ATOM + off),
                         smem_desc(b_base + (kk >> 2) * C::B_ATOM + h * (nw / 2) * 128 + off), idesc, acc,
                         tmem + F4_SF_COL);
        } else {
#pragma unroll
          for (int h = 0; h < nmma; ++h)
            mma_i8<PAIR>(tacc + h * nw, smem_desc(a_base + (kk >> 2) * C::A_ATOM + off),
                         smem_desc(b_base + (kk >> 2) * C::B_ATOM + h * (nw / 2) * 128 + off), idesc, acc);
        }
      }
      mma_commit<PAIR>(empty_bar(s));
    }
    mma_commit<PAIR>(accf_bar(buf));
    return true;
  };
  // Completes once every MMA issued before has finished; waited on even after
  // an abort, so tensor memory is never freed under a live MMA.
  auto drain = [&]() {
    if constexpr (PAIR) {
      asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(drain_bar)
                   : "memory");
    } else {
      mma_commit<false>(drain_bar);
    }
    int zero = 0;
    mbar_wait(drain_bar, 0, &zero, 6);
  };

  if (warp < C::PROD_WARPS) {
    // ------------------------------------------------------------ producers
    // a's warp w writes tensor-memory lanes 32w..32w+31 (its rows)
    if (warp < PROD_A_WARPS)
      produce<true, TLEN, SPD, PAIR, ATMEM, WIDE, F4, UNR, LEV>(g, sc, sbase, bar_base, abort_flag, rank, tile0, tstep, threadIdx.x,
                                            lane, tmem + ((uint32_t)(32 * warp) << 16) + C::TMEM_A);
    else
      produce<false, TLEN, SPD, PAIR, ATMEM, WIDE, F4, UNR, LEV>(g, sc, sbase, bar_base, abort_flag, rank, tile0, tstep,
                                             threadIdx.x - PROD_A_WARPS * 32, lane, 0u);
  } else if (!C::MERGED && warp == C::MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    if (lane == 0 && leader) {
      uint32_t it = 0, uc = 0;
      for (int w = tile0; w < sc.nwork; w += tstep) {
        const Work wk = work_of(sc, w, g.d);
        int lp = g.lp;
        if constexpr (LEV) {
          int bh, a0, b0;
          tile_coords(sc, wk.tile, bh, a0, b0);
          const int lv = level_of(g, a0);
          if (lv < 0) continue;
          lp = g.lev[lv].lp;
        }
        const int nu = units_of(sc, wk);
        for (int u = 0; u < nu; ++u, ++uc)
          if (!issue_unit(wk, u, it, uc, lp)) goto mma_done;
      }
    mma_done:
      drain();
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // (MERGED: the first epilogue warp's lane 0 in the leader CTA issues each
    // work item's MMAs before the warp turns to that item's epilogue)
    const bool issuer = C::MERGED && warp == C::MMA_WARP && leader;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16);
    const uint32_t stg = stg_base + (uint32_t)q * (32 * 32 * 4);  // this warp's staging area
    uint32_t uc = 0, mit = 0, cpy_phase = 0;
    const bool deferred = C::MERGED && g.out_self > 0;
    for (int w = tile0; w < sc.nwork; w += tstep) {
      const Work wk = work_of(sc, w, g.d);
      if (units_of(sc, wk) == 0) continue;  // empty tail piece
      int bh, a0, b0;
      tile_coords(sc, wk.tile, bh, a0, b0);
      // the item's epilogue recipe (with row levels, its level's scale)
      Epilogue ep = g.epi;
      int lp = g.lp;
      if constexpr (LEV) {
        const int lv = level_of(g, a0);
        if (lv < 0) continue;
        ep.inner = g.lev[lv].inner;
        lp = g.lev[lv].lp;
      }
      if (issuer) {  // one accumulation unit per item with wide tiles
        int ok = 1;
        if (lane == 0) ok = issue_unit(wk, 0, mit, uc, lp) ? 1 : 0;
        if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) goto epi_out;
      }
      const int ia = a0 + (int)rank * C::BM + 32 * q + lane;
      const int m_end = min(g.m, b0 + sc.tile_b);  // end of this tile's columns
      // Tail pieces (stream-K) come only to kernels that can receive them: the
      // row-level launcher runs whole tiles, and the unrolled two-buffer e2m1
      // kernel runs the chunked path (several accumulation units, no tail)
      // and the opt-in narrow long tiles (no tail either); without this code
      // those kernels do not spill (76 and 72 bytes with it)
      constexpr bool TAIL_CODE = TAIL && !LEV && !(C::F4 && !C::WIDE && UNR);
      if (TAIL_CODE && wk.part >= 0) {
        // ---- one K piece of a tail tile
        const int buf = (int)(uc % nbuf);
        if (!mbar_wait(accf_bar(buf), (uc / nbuf) & 1, abort_flag, 5)) goto epi_out;
        ++uc;
        tc_fence_after();
        const uint32_t acc_addr = lane_addr + (uint32_t)(buf * C::ACC_STRIDE);
        const int st = wk.tile - sc.full;
        const size_t slot_ints = (size_t)C::BM * C::TILE_MAX;
        const int rowq = 32 * q + lane;
        int* mine = g.split_acc + ((size_t)wk.part * C::NCTA + rank) * slot_ints;
        // the tile's pieces: those of the workers whose ranges meet its blocks
        const int u_first = tail_worker(sc, st * sc.nblk), u_last = tail_worker(sc, (st + 1) * sc.nblk - 1);
#pragma unroll 1
        for (int cb = 0; cb < cdiv(sc.tile_b, 16); ++cb) {
          uint32_t acc[16];
          TMEM_LD16(acc_addr + cb * 16, acc);
          tmem_wait_ld();
          int4* dst = reinterpret_cast<int4*>(mine + ((size_t)cb * C::BM + rowq) * 16);
#pragma unroll
          for (int x = 0; x < 4; ++x)
            dst[x] = make_int4(acc_int<F4>(acc[4 * x]), acc_int<F4>(acc[4 * x + 1]), acc_int<F4>(acc[4 * x + 2]),
                               acc_int<F4>(acc[4 * x + 3]));
        }
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
        if (warp == C::EPI_WARP0 && lane == 0)
          *split_flag = atomicAdd(g.split_cnt + st * C::NCTA + rank, 1) == u_last - u_first;
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const bool tile_done = *split_flag;  // read once: the next item's piece may overwrite it
        if (tile_done) {
          // last part to finish: the other parts' accumulators are complete
          __threadfence();
#pragma unroll 1
          for (int cp = 0; cp < cdiv(sc.tile_b, 32); ++cp) {
            uint32_t fin[32];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int cb = 2 * cp + h;
              uint32_t acc[16];
              TMEM_LD16(acc_addr + cb * 16, acc);
              tmem_wait_ld();
#pragma unroll
              for (int j = 0; j < 16; ++j) acc[j] = (uint32_t)acc_int<F4>(acc[j]);
              for (int u = u_first; u <= u_last; ++u) {
                // a worker that starts in an earlier tile has its second piece here
                const int p = 2 * u + (tail_lo(sc, u) < st * sc.nblk ? 1 : 0);
                if (p == wk.part) continue;
                const int4* src = reinterpret_cast<const int4*>(
                    g.split_acc + ((size_t)p * C::NCTA + rank) * slot_ints + ((size_t)cb * C::BM + rowq) * 16);
#pragma unroll
                for (int x = 0; x < 4; ++x) {
                  const int4 v = __ldcg(src + x);
                  acc[4 * x] += (uint32_t)v.x;
                  acc[4 * x + 1] += (uint32_t)v.y;
                  acc[4 * x + 2] += (uint32_t)v.z;
                  acc[4 * x + 3] += (uint32_t)v.w;
                }
              }
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int ib = b0 + cb * 16 + j;
                fin[16 * h + j] =
                    (ia < g.n && ib < m_end)
                        ? __float_as_uint(epi_value(ep, (int)acc[j], bh * g.n + ia, bh * g.m + ib, bh, 0, g.n, g.m))
                        : 0u;
              }
            }
            // tail tiles end together at the end of the kernel: their stores go
            // to every destination at once (deferring them measured slower)
            store_rows32(g, stg, bh, ia - lane, b0 + 32 * cp, m_end, fin, lane);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_leader<PAIR>(acce_bar(buf), rank);
        continue;
      }
      // The chunk epilogue is compiled only into the kernels that can run it:
      // wide tiles always have one accumulation unit, and with e2m1 operands
      // the chunked path runs on the unrolled two-buffer kernel (UNR), the
      // short tiles on the rolled one. Without it the default wide kernel
      // spills 8 bytes of registers instead of 24 and the short-tile kernel
      // none instead of 68 (the 128-register limit of 512 / 416 threads). The
      // row-level kernels keep it (the wide one compiles without spills with
      // it, with spills without it)
      const bool chunked = (LEV || (!C::WIDE && (!C::F4 || UNR))) && ep.kind == EPI_CHUNK;
      for (int u = 0; u < sc.nunits; ++u, ++uc) {
        const int buf = (int)(uc % nbuf);
        if (!mbar_wait(accf_bar(buf), (uc / nbuf) & 1, abort_flag, 5)) goto epi_out;
        tc_fence_after();
        const uint32_t acc_addr = lane_addr + (uint32_t)(buf * C::ACC_STRIDE);  // running sum: lane_addr + ACC_STRIDE
        const bool last = u == sc.nunits - 1;
        if (chunked && !last) {
          // Chunk u of several: add its scaled values to the running sum in
          // tensor-memory columns 256+. The chunk's column scales are staged
          // in shared memory, and slice cb+1 is loaded while cb is processed.
          const int et = (warp - C::EPI_WARP0) * 32 + lane;
          asm volatile("bar.sync 1, 128;" ::: "memory");  // the previous chunk's readers are done
          for (int c = et; c < sc.tile_b; c += 128)
            sbs[c] = b0 + c < g.m ? __ldg(ep.sb + (size_t)u * g.m + b0 + c) : 0.f;
          asm volatile("bar.sync 1, 128;" ::: "memory");
          const float sar = ia < g.n ? __ldg(ep.sa + (size_t)u * g.n + ia) : 0.f;
          const int ns = cdiv(sc.tile_b, 8);  // slices of eight columns
          uint32_t acc0[8], run0[8], acc1[8], run1[8];
          // result of slice cb into acc (in place), stored to the running sum
          auto chunk_slice = [&](int cb, uint32_t (&acc)[8], const uint32_t (&run)[8]) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int ib = b0 + cb * 8 + j;
              float x = 0.f;
              if (ia < g.n && ib < m_end)
                x = fmul(fmul((float)acc_int<F4>(acc[j]), ep.inner), fmul(sar, sbs[cb * 8 + j]));
              acc[j] = __float_as_uint(fadd(u > 0 ? __uint_as_float(run[j]) : 0.f, x));
            }
            TMEM_ST8(lane_addr + C::ACC_STRIDE + cb * 8, acc);
          };
          TMEM_LD8(acc_addr, acc0);
          if (u > 0) TMEM_LD8(lane_addr + C::ACC_STRIDE, run0);
#pragma unroll 1
          for (int cb = 0; cb < ns; cb += 2) {
            tmem_wait_ld();
            if (cb + 1 < ns) {
              TMEM_LD8(acc_addr + (cb + 1) * 8, acc1);
              if (u > 0) TMEM_LD8(lane_addr + C::ACC_STRIDE + (cb + 1) * 8, run1);
            }
            chunk_slice(cb, acc0, run0);
            if (cb + 1 < ns) {
              tmem_wait_ld();
              tmem_wait_st();  // acc0 is about to be reloaded; its store has read it
              if (cb + 2 < ns) {
                TMEM_LD8(acc_addr + (cb + 2) * 8, acc0);
                if (u > 0) TMEM_LD8(lane_addr + C::ACC_STRIDE + (cb + 2) * 8, run0);
              }
              chunk_slice(cb + 1, acc1, run1);
              tmem_wait_st();  // likewise acc1
            }
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_leader<PAIR>(acce_bar(buf), rank);
          continue;
        }
#pragma unroll 1
        for (int cp = 0; cp < cdiv(sc.tile_b, 32); ++cp) {
          uint32_t fin[32];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int cb = 2 * cp + h;
            uint32_t acc[16], run[16];
            TMEM_LD16(acc_addr + cb * 16, acc);
            if (chunked && u > 0) TMEM_LD16(lane_addr + C::ACC_STRIDE + cb * 16, run);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int ib = b0 + cb * 16 + j;
              float v = 0.f;
              if (ia < g.n && ib < m_end)
                v = epi_value(ep, acc_int<F4>(acc[j]), bh * g.n + ia, bh * g.m + ib, bh, u, g.n, g.m);
              if (chunked) v = fadd(u > 0 ? __uint_as_float(run[j]) : 0.f, v);
              fin[16 * h + j] = __float_as_uint(v);
            }
          }
          store_rows32(g, stg, bh, ia - lane, b0 + 32 * cp, m_end, fin, lane, deferred ? g.out_self - 1 : -1);
        }
        if (deferred) {  // this warp's rows are in this device's destination
          __threadfence_block();
          __syncwarp();
          if (lane == 0) mbar_arrive(cpy_bar);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_leader<PAIR>(acce_bar(buf), rank);
        if (deferred) {
          // The accumulator is free and the next tile's MMAs can start; the
          // other epilogue warps copy the CTA's 128 rows of this tile to the
          // other destinations (over NVLink) meanwhile, once all four warps
          // have stored their rows. The first warp (the MMA issuer in the
          // leader CTA) goes straight on.
          if (q != 0) {
            if (!mbar_wait(cpy_bar, cpy_phase & 1, abort_flag, 7)) goto epi_out;
            // (spreading the copy over the next tile with pauses between rows
            // measured slower at 8 devices than copying at full speed)
            copy_rows_to_peers(g, g.out_self - 1, bh, a0 + (int)rank * C::BM, C::BM, b0, m_end, q - 1, 3, lane);
          }
          ++cpy_phase;
        }
      }
    }
  epi_out:
    if (issuer && lane == 0) drain();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // no CTA leaves while its peer may still touch it
  if (warp == C::MMA_WARP) {
    tc_fence_after();
    if constexpr (PAIR) {
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS)
                   : "memory");
    } else {
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS)
                   : "memory");
    }
  }
}

template <int TLEN, int SPD, bool PAIR, bool ATMEM = false, bool WIDE = ATMEM && wide_tiles<TLEN>(), bool F4 = false,
          bool UNR = F4 && WIDE, bool LEV = false, bool TAIL = true>
static cudaError_t launch_t(const GemmArgs& g, const Sched& s, int sms, cudaStream_t st) {
  using C = Cfg<PAIR, ATMEM, WIDE, F4>;
  auto kern = gemm_tc_kernel<TLEN, SPD, PAIR, ATMEM, WIDE, F4, UNR, LEV, TAIL>;
  // The attribute belongs to the current device's context, so it is set on
  // every launch (a host call; a process may drive several devices).
  {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return e;
  }
  if constexpr (!PAIR) {
    const int grid = s.workers;
    kern<<<grid, C::THREADS, C::SMEM_BYTES, st>>>(g, s);
    count_launch();
    return cudaGetLastError();
  } else {
    const int pairs = s.workers;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    cfg.blockDim = dim3(C::THREADS, 1, 1);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, g, s);
    count_launch();
    return e;
  }
}

}  // namespace tc

bool gemm_tc_supported(const GemmArgs& g) {
  if (g.n <= 0 || g.m <= 0 || g.d <= 0) return false;
  if (g.lp < 32 || g.lp > 512 || (g.lp & (g.lp - 1))) return false;  // power of two in [32, 512]
  if ((long long)g.d * g.L >= (1LL << 31)) return false;
  // accumulation units (chunks) must start on a block of eight dimensions
  if (g.unit_d > 0 && g.unit_d < g.d && g.unit_d % 8 != 0) return false;
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return major == 10 && minor == 0;
}

// The 2-SM variant is the default; SCMP_TC_SINGLE=1 in the environment selects
// the 1-SM variant (kept for comparison and as a fallback).
static bool use_pair() {
  const char* e = getenv("SCMP_TC_SINGLE");
  return !(e && e[0] == '1');
}

// Tiles with fewer K stages than this use two accumulators rather than a in
// tensor memory (the epilogue is then a visible share of a tile).
constexpr int kShortTileStages = 512;

// Which kernel a call runs. SM pairs (single SMs with SCMP_TC_SINGLE=1);
// on pairs, with one accumulation unit per tile and long tiles, 512-wide
// tiles with a in shared memory (SCMP_TC_ATMEM=1 selects a in tensor memory
// instead, 256- or 320-wide tiles); short tiles use two 256-wide accumulators
// and the chunked path one accumulator plus the running sum.
static bool env_on(const char* name) {
  const char* e = getenv(name);
  return e && e[0] == '1';
}
struct Variant {
  bool pair, atmem, wide;  // wide without atmem: 512-wide tiles, a in shared memory
  bool f4;                 // e2m1 operands (kind::mxf4)
  bool long_tiles;         // one accumulation unit of at least kShortTileStages stages
};
// f4_table: the call carries the e2m1-sliced stream table. e2m1 operands are
// used on SM pairs with a in shared memory for streams of 64 to 512
// positions (a stage then covers at most one block of eight dimensions);
// SCMP_TC_INT8=1 in the environment keeps int8 operands.
static Variant choose_variant(int d, int unit_d, int lp, bool f4_table) {
  Variant v;
  v.pair = use_pair();
  const int nunits = cdiv(d, unit_d > 0 ? unit_d : d);
  const int tlen = lp < 256 ? lp : 256;
  const int stages = (tlen < 256 ? cdiv(d, 256 / tlen) : d) * (lp / tlen);
  const bool long_tiles = v.pair && nunits == 1 && stages >= kShortTileStages;
  v.long_tiles = long_tiles;
  v.atmem = long_tiles && env_on("SCMP_TC_ATMEM");
  // SCMP_TC_NARROW=1: long tiles on the two-accumulator kernel (tiles of at
  // most 240 / 256 b rows, a tile's epilogue under the next tile's MMAs)
  v.wide = long_tiles && (!v.atmem || lp < 256) && !(env_on("SCMP_TC_NARROW") && !v.atmem);
  v.f4 = f4_table && v.pair && !v.atmem && lp >= 64 && lp <= 512 && !env_on("SCMP_TC_INT8");
  return v;
}

static int device_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    sms = 148;
  return sms;
}

namespace tc {
// Columns of a split part's accumulator slot (the variant's most b rows per tile).
static int tile_cols(const Variant& v) {
  if (v.f4) return v.wide ? Cfg<true, false, true, true>::TILE_MAX : Cfg<true, false, false, true>::TILE_MAX;
  return v.wide ? (v.atmem ? Cfg<true, true, true>::TILE_B : Cfg<true, false, true>::TILE_B) : 256;
}
constexpr int kMaxSplit = 8;              // tail pieces per tile, about, at most
constexpr int kMinSplitBlocks = 8;        // blocks of eight dimensions per tail range, at least
constexpr size_t kSplitBudget = 128u << 20;  // bytes of tail-piece accumulators, at most

// Schedule of the persistent grid: the workers (SM pairs or SMs) take whole
// tiles round-robin; when that leaves a last wave of rem < workers tiles (and
// d is one accumulation unit), the rem tiles' K ranges are shared evenly by
// tail_w workers (work_of), so the last wave takes rem / tail_w of a tile
// instead of a whole one. tail_w is the number of workers, within the limits
// above (SCMP_TC_NO_SPLIT=1 in the environment turns the tail off).
static Sched make_sched(int batch, int n, int m, int d, int unit_d, Variant v, int sms) {
  const bool pair = v.pair;
  Sched s{};
  s.tile_a = pair ? Cfg<true>::TILE_A : Cfg<false>::TILE_A;
  // columns per tile: b's rows in equal tiles of at most TILE_B, a multiple of
  // 16 per MMA (N), so that a small or ragged m does not pay for a full tile
  const int tmax = tile_cols(v);
  const int gran = v.wide ? 32 : 16;
  s.tiles_b = cdiv(m, tmax);
  s.tile_b = cdiv(cdiv(m, s.tiles_b), gran) * gran;
  s.tiles_a = cdiv(n, s.tile_a);
  s.tiles = batch * s.tiles_a * s.tiles_b;
  s.unit_d = unit_d > 0 ? unit_d : d;
  s.nunits = cdiv(d, s.unit_d);
  s.nblk = cdiv(d, 8);
  s.full = s.tiles;
  const int units = pair ? sms / 2 : sms;
  s.workers = s.tiles < units ? s.tiles : units;
  const int rem = s.tiles % units;
  const char* off = getenv("SCMP_TC_NO_SPLIT");
  // (e2m1 narrow long tiles, an opt-in comparison mode, run on the unrolled
  // two-buffer kernel, which is compiled without the tail; so do row levels)
  const bool narrow_long = v.f4 && !v.wide && v.long_tiles;
  // A last wave at least 90% full is run as whole tiles: sharing it saves at
  // most a tenth of a tile and its fix-ups cost more (config 2, 72 tiles on
  // 74 pairs: GEMM 11.31 ms split, 11.23 ms whole; config 5, 70 on 74:
  // 34.07 / 34.02 ms)
  const bool worth = (long long)rem * 10 <= (long long)units * 9;
  if (s.nunits == 1 && rem > 0 && worth && !(off && off[0] == '1') && !narrow_long) {
    const size_t part_bytes = (size_t)(pair ? 2 : 1) * 128 * tmax * sizeof(int);
    const long long tblk = (long long)rem * s.nblk;
    long long tw = units;
    if (tw > (long long)rem * kMaxSplit) tw = (long long)rem * kMaxSplit;
    if (tw > tblk / kMinSplitBlocks) tw = tblk / kMinSplitBlocks;
    if (tw > (long long)(kSplitBudget / (2 * part_bytes))) tw = (long long)(kSplitBudget / (2 * part_bytes));
    if (tw > rem) {  // each worker's share is less than one tile
      s.full = s.tiles - rem;
      s.workers = units;
      s.tail_w = (int)tw;
      s.tail_blk = (int)tblk;
    }
  }
  s.nwork = s.full + (s.tail_w > 0 ? 2 * s.workers : 0);
  // Tile order: for wide tiles, groups of eight 256-row bands of a
  // (SCMP_TC_BAND_GROUP=g in the environment selects g; 1 is band after
  // band). With eight bands the tiles in flight share about nine b tiles'
  // operand rows and the group's a rows in L2 (config 5, whose b operand is
  // 470 MB: GEMM 37.7 -> 36.0 ms). Narrow tiles keep the band order (config
  // 4's row-level call was slower grouped: 2.92 -> 3.28 ms).
  const char* bg = getenv("SCMP_TC_BAND_GROUP");
  s.band_group = bg ? atoi(bg) : (v.wide ? 8 : 1);
  if (s.band_group < 1) s.band_group = 1;
  return s;
}
}  // namespace tc

// Workspace of the tail: 2 * tail_w piece accumulators (slot 2u + j: worker u's
// piece j), then one arrival counter per tail tile and CTA.
size_t gemm_tc_split_cnt_offset(int batch, int n, int m, int d, int unit_d, int lp, bool f4_table) {
  const Variant v = choose_variant(d, unit_d, lp, f4_table);
  const tc::Sched s = tc::make_sched(batch, n, m, d, unit_d, v, device_sms());
  return (size_t)2 * s.tail_w * (v.pair ? 2 : 1) * 128 * tc::tile_cols(v) * sizeof(int);
}

size_t gemm_tc_split_bytes(int batch, int n, int m, int d, int unit_d, int lp, bool f4_table) {
  const Variant v = choose_variant(d, unit_d, lp, f4_table);
  const tc::Sched s = tc::make_sched(batch, n, m, d, unit_d, v, device_sms());
  if (s.tail_w == 0) return 0;
  return gemm_tc_split_cnt_offset(batch, n, m, d, unit_d, lp, f4_table) +
         (size_t)(s.tiles - s.full) * (v.pair ? 2 : 1) * sizeof(int);
}

cudaError_t launch_gemm_tc(const GemmArgs& g, cudaStream_t st) {
  using namespace tc;
  const Variant v = choose_variant(g.d, g.unit_d, g.lp, g.pattern4 != nullptr);
  const bool pair = v.pair;
  const int sms = device_sms();
  Sched s = make_sched(g.batch, g.n, g.m, g.d, g.unit_d, v, sms);
  if (s.tail_w > 0) {
    if (!g.split_acc || !g.split_cnt) {  // no workspace for the pieces: whole tiles only
      s.full = s.tiles;
      s.tail_w = 0;
      s.nwork = s.tiles;
    } else {
      const cudaError_t e = cudaMemsetAsync(g.split_cnt, 0, (size_t)(s.tiles - s.full) * (pair ? 2 : 1) * sizeof(int), st);
      if (e != cudaSuccess) return e;
    }
  }
  if (v.f4) {  // e2m1 operands: TLEN is the padded stream length, 64 .. 512
    if (v.wide && s.tail_w == 0) {  // whole tiles only: the kernel without the tail's code
      switch (g.lp) {
        case 64: return launch_t<64, 1, true, false, true, true, true, false, false>(g, s, sms, st);
        case 128: return launch_t<128, 1, true, false, true, true, true, false, false>(g, s, sms, st);
        case 256: return launch_t<256, 1, true, false, true, true, true, false, false>(g, s, sms, st);
        default: return launch_t<512, 1, true, false, true, true, true, false, false>(g, s, sms, st);
      }
    }
    if (v.wide) {
      switch (g.lp) {
        case 64: return launch_t<64, 1, true, false, true, true>(g, s, sms, st);
        case 128: return launch_t<128, 1, true, false, true, true>(g, s, sms, st);
        case 256: return launch_t<256, 1, true, false, true, true>(g, s, sms, st);
        default: return launch_t<512, 1, true, false, true, true>(g, s, sms, st);
      }
    }
    if (s.nunits > 1 || v.long_tiles) {  // chunked path and narrow long tiles: stages unrolled
      switch (g.lp) {
        case 64: return launch_t<64, 1, true, false, false, true, true>(g, s, sms, st);
        case 128: return launch_t<128, 1, true, false, false, true, true>(g, s, sms, st);
        case 256: return launch_t<256, 1, true, false, false, true, true>(g, s, sms, st);
        default: return launch_t<512, 1, true, false, false, true, true>(g, s, sms, st);
      }
    }
    switch (g.lp) {
      case 64: return launch_t<64, 1, true, false, false, true>(g, s, sms, st);
      case 128: return launch_t<128, 1, true, false, false, true>(g, s, sms, st);
      case 256: return launch_t<256, 1, true, false, false, true>(g, s, sms, st);
      default: return launch_t<512, 1, true, false, false, true>(g, s, sms, st);
    }
  }
  const int tlen = g.lp < 256 ? g.lp : 256;
  const int spd = g.lp / tlen;
  if (v.wide && !v.atmem) {  // 512-wide tiles, a in shared memory (default for long tiles)
    switch (tlen) {
      case 32: return launch_t<32, 1, true, false, true>(g, s, sms, st);
      case 64: return launch_t<64, 1, true, false, true>(g, s, sms, st);
      case 128: return launch_t<128, 1, true, false, true>(g, s, sms, st);
      default:
        return spd == 2 ? launch_t<256, 2, true, false, true>(g, s, sms, st)
                        : launch_t<256, 1, true, false, true>(g, s, sms, st);
    }
  }
  if (v.atmem) {
    switch (tlen) {
      case 32: return launch_t<32, 1, true, true>(g, s, sms, st);
      case 64: return launch_t<64, 1, true, true>(g, s, sms, st);
      case 128: return launch_t<128, 1, true, true>(g, s, sms, st);
      default:
        return spd == 2 ? launch_t<256, 2, true, true>(g, s, sms, st) : launch_t<256, 1, true, true>(g, s, sms, st);
    }
  }
  if (pair) {
    switch (tlen) {
      case 32: return launch_t<32, 1, true>(g, s, sms, st);
      case 64: return launch_t<64, 1, true>(g, s, sms, st);
      case 128: return launch_t<128, 1, true>(g, s, sms, st);
      default: return spd == 2 ? launch_t<256, 2, true>(g, s, sms, st) : launch_t<256, 1, true>(g, s, sms, st);
    }
  }
  switch (tlen) {
    case 32: return launch_t<32, 1, false>(g, s, sms, st);
    case 64: return launch_t<64, 1, false>(g, s, sms, st);
    case 128: return launch_t<128, 1, false>(g, s, sms, st);
    default: return spd == 2 ? launch_t<256, 2, false>(g, s, sms, st) : launch_t<256, 1, false>(g, s, sms, st);
  }
}

// Row levels: one launch on SM pairs with e2m1 operands; every level's
// padded stream length in [64, 512]. a's permuted rows (g.n, whole 256-row
// tiles) bound the schedule; tiles past the last level's end are skipped.
// Whole tiles only (the tail is not shared over K).
bool gemm_tc_levels_supported(const GemmArgs& g) {
  if (g.nlev < 1 || g.nlev > kMaxLevels || g.n % 256 != 0 || g.m <= 0 || g.d <= 0 || g.batch != 1) return false;
  if (g.unit_d > 0 && g.unit_d < g.d && g.unit_d % 8 != 0) return false;
  for (int l = 0; l < g.nlev; ++l) {
    const int lp = g.lev[l].lp;
    if (lp < 64 || lp > 512 || (lp & (lp - 1)) || !g.lev[l].pattern4) return false;
    if ((long long)g.d * g.lev[l].L >= (1LL << 31)) return false;
  }
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return major == 10 && minor == 0;
}

cudaError_t launch_gemm_tc_levels(const GemmArgs& g, cudaStream_t st) {
  using namespace tc;
  const int sms = device_sms();
  int min_lp = 512;
  for (int l = 0; l < g.nlev; ++l) min_lp = g.lev[l].lp < min_lp ? g.lev[l].lp : min_lp;
  // wide tiles when every level's tiles are long (one accumulation unit)
  Variant v = choose_variant(g.d, g.unit_d, min_lp, true);
  v.f4 = true;
  v.pair = true;
  v.atmem = false;
  Sched s = make_sched(g.batch, g.n, g.m, g.d, g.unit_d, v, sms);
  s.full = s.tiles;
  s.tail_w = 0;
  s.nwork = s.tiles;
  s.workers = s.tiles < sms / 2 ? s.tiles : sms / 2;
  if (v.wide) return launch_t<256, 1, true, false, true, true, true, true>(g, s, sms, st);
  return launch_t<256, 1, true, false, false, true, true, true>(g, s, sms, st);
}

}  // namespace scmp
