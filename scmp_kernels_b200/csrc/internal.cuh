// Internal argument blocks shared by the quantisers, the GEMM kernels and the
// C-ABI layer.
#pragma once

#include "common.cuh"

namespace scmp {

// Float32 epilogue recipes of the reference's path orchestrators. `raw` below
// is fl32(S * inner) with inner = fl32(q_max^2 / L), the in-kernel scale of
// enable_matmul_tiled_kernel (sc/kernels.py:212, 248).
enum EpiKind {
  EPI_RAW = 0,         // out = raw                               (enable_matmul_triton)
  EPI_SCALAR = 1,      // out = raw * c0                          (per_tensor bipolar, kernels.py:1204)
  EPI_SCALAR_UNI = 2,  // zero-point correction with host scalars (per_tensor unipolar, 1198-1204)
  EPI_ROW = 3,         // out = raw * fl32(sa[r] * sb[c])         (per_row bipolar, 1707 / 1894)
  EPI_ROW_UNI = 4,     // per-row zero-point correction           (per_row unipolar, 1699-1707)
  EPI_HEAD = 5,        // out = S * fl32(inner * fl32(sa[bh]*sb[bh])) (per_head, 430-432, 550)
  EPI_CHUNK = 6        // out += raw_c * fl32(sa_c[r] * sb_c[c])  (chunked, 1380-1381)
};

struct Epilogue {
  int kind;
  float inner;
  const float* scal;  // EPI_SCALAR*: [0] c0 = fl32(scale_a*scale_b), [1] -zp_b, [2] zp_a, [3] fl32(D*zp_a*zp_b)
  const float* sa;    // EPI_ROW*: (batch*n); EPI_CHUNK: (nchunks, n); EPI_HEAD: (batch)
  const float* sb;    // EPI_ROW*: (batch*m); EPI_CHUNK: (nchunks, m); EPI_HEAD: (batch)
  const float* zpa;   // EPI_ROW_UNI: (batch*n)
  const float* zpb;   // EPI_ROW_UNI: (batch*m)
  const float* asum;  // EPI_*_UNI: row sums of the quantised a (batch*n)
  const float* bsum;  // EPI_*_UNI: row sums of the quantised b (batch*m)
  float fd;           // EPI_ROW_UNI: float(D)
};

// Value of one output element for accumulation unit `unit` (chunk index for
// EPI_CHUNK). ia / ib are row indices including the batch offset.
__device__ __forceinline__ float epi_value(const Epilogue& e, int S, int ia, int ib, int bh,
                                           int unit, int n, int m) {
  const float Sf = (float)S;  // exact: |S| <= D * L < 2^24
  if (e.kind == EPI_HEAD) return fmul(Sf, fmul(e.inner, fmul(e.sa[bh], e.sb[bh])));
  const float raw = fmul(Sf, e.inner);
  switch (e.kind) {
    case EPI_SCALAR:
      return fmul(raw, e.scal[0]);
    case EPI_SCALAR_UNI: {
      const float t1 = fmul(e.scal[1], e.asum[ia]);
      const float t2 = fmul(e.scal[2], e.bsum[ib]);
      const float t5 = fadd(fsub(t1, t2), e.scal[3]);
      return fmul(fadd(raw, t5), e.scal[0]);
    }
    case EPI_ROW:
      return fmul(raw, fmul(e.sa[ia], e.sb[ib]));
    case EPI_ROW_UNI: {
      const float zb = e.zpb[ib], za = e.zpa[ia];
      const float t1 = fmul(-zb, e.asum[ia]);
      const float t2 = fmul(za, e.bsum[ib]);
      const float t4 = fmul(fmul(e.fd, za), zb);
      const float t5 = fadd(fsub(t1, t2), t4);
      return fmul(fadd(raw, t5), fmul(e.sa[ia], e.sb[ib]));
    }
    case EPI_CHUNK:
      return fmul(raw, fmul(e.sa[(size_t)unit * n + ia], e.sb[(size_t)unit * m + ib]));
    default:
      return raw;
  }
}

// Operand layout of the quantised operands: int16 [ceil(d/8)][R][8] with
// R = batch * rows, so that one aligned 16-byte load gives a thread eight
// consecutive dimensions of its row and a warp's 32 consecutive rows are one
// contiguous 512-byte segment. Entries past d are padding (never read as data).
__host__ __device__ __forceinline__ int d8(int d) { return (d + 7) >> 3; }
__host__ __device__ __forceinline__ size_t blk_idx(int R, int row, int j) {
  return ((size_t)(j >> 3) * R + row) * 8 + (j & 7);
}

// Bit order of the e2m1-sliced stream words: position 8q + i of a word
// (q < 4, i < 8) sits at bit 4i + q, so (word >> q) & 0x11111111 has the eight
// positions 8q .. 8q+7 as the low bits of its nibbles (one e2m1 operand word
// after a multiply by 0x2 or 0xA).
__host__ __device__ constexpr int slice4_bit(int l) { return 4 * (l & 7) + (l >> 3); }

// Bit order of the 32-bit comparator-stream words ("sliced"): stream
// position 16h + 4q + i of a word (h < 2, q < 4, i < 4) sits at bit
// 8i + 4h + q, so the four positions 16h+4q .. 16h+4q+3 are bit 0 of the four
// bytes of (word >> (4h + q)): one shift and one mask give four int8 stream
// values. slice_bit(l) is the bit of position l; unslice() restores position
// order (bit l = position l).
__host__ __device__ constexpr int slice_bit(int l) { return 8 * (l & 3) + 4 * (l >> 4) + ((l >> 2) & 3); }
__device__ __forceinline__ uint32_t unslice(uint32_t w) {
  uint32_t lin = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {  // k = 4h + q: positions 4k .. 4k+3
    const uint32_t x = (w >> k) & 0x01010101u;
    // bytes' bit 0 (bits 0, 8, 16, 24) gathered into bits 24..27 by one
    // multiply: partial products land on distinct bits, so nothing carries
    lin |= (((x * 0x01020408u) >> 24) & 0xFu) << (4 * k);
  }
  return lin;
}

// SC-GEMM operands and epilogue.
//   ka: signed thermometer length sa * k of operand a, blocked (R = batch*n);
//   vb: signed boundary sb * v of operand b, blocked (R = batch*m);
//   bmap: table row of every dimension, padded with zeros to 8*ceil(d/8);
//   pattern/bmap: comparator streams of b, bit t of row (bmap[j], v);
//   the d range is split into accumulation units of unit_d dimensions (the
//   chunks of the chunked path; one unit of d otherwise).
constexpr int kMaxOuts = SCMP_MAX_OUT_PEERS;  // destinations of one result

// Row groups of a with their own stream lengths in one GEMM (the caller's
// mixed precision, scmp_kernels/mp/config.py:154-191): a's rows are permuted
// so that every level occupies whole 256-row tiles, level l holding permuted
// rows [256 * tile0[l], 256 * tile0[l + 1]); b is quantised once per level.
constexpr int kMaxLevels = 4;
struct LevelB {
  const int16_t* vb;         // b's operand quantised on this level's grid (blocked layout)
  const uint32_t* pattern4;  // this level's e2m1-sliced stream table
  const int32_t* bmap;       // padded dimension -> table row map
  int vcap, lp, L;
  float inner;               // fl32(q_max^2 / L)
};

// Writes v to element (h, i, j) of every destination of the result.
struct GemmArgs;
__device__ __forceinline__ void store_out(const GemmArgs& g, int h, int i, int j, float v);

struct GemmArgs {
  int batch, n, m, d;
  int L, lp, vcap;
  int bipolar;
  const int16_t* ka;
  const int16_t* vb;
  const uint32_t* pattern;
  const uint32_t* pattern4;  // the same streams in e2m1-sliced order, or NULL
  const int32_t* bmap;
  int unit_d;
  Epilogue epi;
  // Result destinations: element (h, i, j) goes to outs[k][out_off + (h*n + i)*out_ld + j]
  // for every k < nouts (the local output, or every device's all-gather buffer).
  float* outs[kMaxOuts];
  int nouts;
  long long out_off;
  int out_ld;
  int out_vec;  // every destination row is 16-byte aligned (whole 4-float stores)
  int out_self; // 1 + index of the destination in this device's memory (0: none); see store_rows32
  int* split_acc;  // tcgen05 GEMM, split last wave: per-part integer accumulators
  int* split_cnt;  //   and per-tile arrival counters (see gemm_tc_split_bytes)
  // Row levels (nlev > 0): n counts a's permuted rows (whole tiles per level),
  // row_of[i] is the result row of permuted row i (-1: padding), n_out the
  // result's rows; lev_tile0 (device, nlev + 1 entries) the first 256-row
  // tile of every level and the end of the last.
  int nlev;
  LevelB lev[kMaxLevels];
  const int* lev_tile0;
  const int* row_of;
  int n_out;
};

__device__ __forceinline__ void store_out(const GemmArgs& g, int h, int i, int j, float v) {
  const long long idx = g.out_off + ((long long)h * g.n + i) * g.out_ld + j;
#pragma unroll 1
  for (int k = 0; k < g.nouts; ++k) g.outs[k][idx] = v;
}

// Host launchers (return cudaError_t of the launch).
cudaError_t launch_build_tables(const int32_t* ra, int n_ra, const int32_t* rb, int n_rb, int L,
                                int lp, int vcap, int16_t* ktab, uint32_t* pattern, uint32_t* pattern4,
                                cudaStream_t st);
cudaError_t launch_gemm_simt(const GemmArgs& g, cudaStream_t st);
cudaError_t launch_gemm_tc(const GemmArgs& g, cudaStream_t st);
bool gemm_tc_supported(const GemmArgs& g);
// The row-level GEMM (GemmArgs.nlev > 0).
cudaError_t launch_gemm_tc_levels(const GemmArgs& g, cudaStream_t st);
bool gemm_tc_levels_supported(const GemmArgs& g);
// Workspace of the tcgen05 GEMM's split last wave for this shape on the
// current device (0 when the last wave is not split); the counters sit at
// byte offset gemm_tc_split_cnt_offset of that block.
// f4_table: the call carries the e2m1-sliced stream table (pattern4).
size_t gemm_tc_split_bytes(int batch, int n, int m, int d, int unit_d, int lp, bool f4_table);
size_t gemm_tc_split_cnt_offset(int batch, int n, int m, int d, int unit_d, int lp, bool f4_table);

}  // namespace scmp
