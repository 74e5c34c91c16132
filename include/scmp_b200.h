/*
 * scmp_b200.h -- C ABI of the B200 (sm_100a) stochastic-computing matmul.
 *
 * Drop-in native boundary for the reference package scmp_kernels
 * (swalther06/scmp_kernels). The reference is Python + Triton; its path
 * orchestrators and Triton launchers are what the functions below replace.
 * Each declaration names the reference function it stands in for
 * (file:line relative to the reference repository root).
 *
 * Conventions
 *   - every function returns an int status (SCMP_OK or an SCMP_ERR_* code) and
 *     never throws or aborts; scmp_last_error() gives a message for the
 *     calling thread;
 *   - all array pointers are device pointers owned by the caller unless the
 *     parameter says "host"; the compute entry points allocate no device
 *     memory (scratch comes from the caller's workspace, or from the fixed
 *     array of scmp_sc_matmul_noalloc); scmp_peer_alloc is the one function
 *     that allocates (with cudaMalloc), and scmp_peer_free releases it;
 *   - work is enqueued on the given CUDA stream (a cudaStream_t passed as
 *     void*; NULL is the legacy default stream) on the current device;
 *   - float arithmetic follows the reference bit for bit: IEEE float32 with
 *     round-to-nearest-even per operation and no contraction into FMA.
 */
#ifndef SCMP_B200_H
#define SCMP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SCMP_ABI_VERSION 4

enum scmp_status {
  SCMP_OK = 0,
  SCMP_ERR_INVALID_ARG = 1, /* maps to ValueError in the Python layer          */
  SCMP_ERR_CUDA = 2,        /* a CUDA runtime call failed                      */
  SCMP_ERR_TIMEOUT = 3,     /* a bounded device-side wait gave up             */
  SCMP_ERR_UNSUPPORTED = 4, /* maps to NotImplementedError                     */
  SCMP_ERR_WORKSPACE = 5    /* workspace missing or smaller than required      */
};

enum scmp_granularity { SCMP_PER_TENSOR = 0, SCMP_PER_ROW = 1, SCMP_PER_HEAD = 2 };
enum scmp_mode { SCMP_BIPOLAR = 0, SCMP_UNIPOLAR = 1 };

/* scmp_matmul_desc.flags */
#define SCMP_FLAG_FORCE_SIMT 0x1 /* use the CUDA-core GEMM instead of tcgen05  */
#define SCMP_FLAG_NO_SPLIT 0x2   /* do not split the last wave of output tiles
                                    over K (smaller workspace, longer tail)     */
/* SCMP_FLAG_B_READY: per_row calls without chunking only. b's quantised
 * operand and row parameters are already in the workspace, left there by an
 * earlier scmp_sc_matmul call on the same workspace with the same b and the
 * same b-side arguments (m, d, batch, mode, sc_prec, stoc_len, rng_levels,
 * group_b, smooth_scales, tables); b's quantisation is skipped and `b` is not
 * read (it may be NULL). b's part of the workspace sits at its start and does
 * not depend on n, so one workspace serves calls with any a that fits it: a
 * static weight is quantised once (no counterpart in the reference, which
 * quantises both operands on every call; its SmoothQuant offline helper,
 * quant/smoothquant.py:129-147, is the analogue for the smoothing step). */
#define SCMP_FLAG_B_READY 0x4

/*
 * Enable-signal tables (the "RNG cache" kept resident in HBM).
 *
 * Replaces build_enable_tables / build_k_table_only and their kernels
 * build_cum_indicator_kernel + compute_k_table_kernel
 * (scmp_kernels/sc/kernels.py:712-759, 871-894, 102-169).
 *
 * Inputs are the prepared comparator sequences (prefix / Owen scramble /
 * rescale already applied, kernels.py:673-704), deduplicated to distinct rows:
 *   ra: (n_ra, L) int32   sequences of operand a ("q" side)
 *   rb: (n_rb, L) int32   sequences of operand b ("k" side)
 * Outputs, for v in [0, vcap]:
 *   ktab:    (n_ra, vcap+1) int16   ktab[r][v] = #{t < L : ra[r][t] < v}
 *   pattern: (n_rb, vcap+1, lp/32) uint32, the comparator stream of b,
 *            bit-packed: position t of row (r, v) is set iff t < L and
 *            rb[r][t] < v. Word w holds positions 32w..32w+31 in "sliced"
 *            order: position 32w + 16h + 4q + i at bit 8i + 4h + q (h < 2,
 *            q, i < 4), so that one shift and one mask of a word yield four
 *            consecutive positions as the bytes of an int8 operand word.
 *   pattern4: NULL, or the same streams with position 32w + 8q + i (q < 4,
 *            i < 8) at bit 4i + q of word w ("e2m1-sliced"), so that one
 *            shift and one mask yield eight consecutive positions as the
 *            nibbles of a 4-bit (e2m1) operand word. Passing it to
 *            scmp_sc_matmul lets the GEMM run on e2m1 operands
 *            (tcgen05.mma.kind::mxf4, twice the int8 rate; same results).
 * lp >= L is the padded stream length (a multiple of 32). Every sequence value
 * must be < vcap, so that boundaries >= vcap saturate (ktab = L, all bits set).
 * The reference's cum_indicator[d][k][v] equals the number of set positions t < k of
 * pattern[d][v].
 */
int scmp_build_tables(const int32_t* ra, int n_ra, const int32_t* rb, int n_rb, int L, int lp,
                      int vcap, int16_t* ktab, uint32_t* pattern, uint32_t* pattern4, void* stream);

/*
 * One sc_matmul call: quantise both operands, run the integer SC-GEMM and the
 * path's float32 epilogue into `out`.
 *
 * Replaces the dispatch of _sc_matmul_impl (scmp_kernels/sc/matmul.py:224-279)
 * and the five path orchestrators it calls:
 *   per_tensor            _sc_matmul_per_tensor + _sc_matmul_enable_triton
 *                         (kernels.py:1053-1204; 3D: 1207-1226)
 *   per_row               _sc_matmul_per_row + _sc_matmul_grouped_enable
 *                         (kernels.py:1573-1707)
 *   per_row, chunk_d > 0  _sc_matmul_per_row_mlp + _sc_matmul_bipolar_mlp_chunked
 *                         (kernels.py:1443-1566, 1274-1383)
 *   per_row, 3D           _sc_matmul_per_row_batched (kernels.py:1778-1895)
 *   per_head              _sc_matmul_per_head_bipolar (kernels.py:440-585)
 * with apply_smoothing (scmp_kernels/quant/smoothquant.py:96-126) fused into
 * the quantisation when smooth_scales is non-NULL. No host synchronisation:
 * the per-tensor ranges that the reference reads back with .item()
 * (matmul.py:227-230) are reduced and turned into scales on the device.
 */
typedef struct scmp_matmul_desc {
  int granularity;      /* enum scmp_granularity                                   */
  int mode;             /* enum scmp_mode                                          */
  int sc_prec;          /* p: q_max = 2^(p-1)-1 (bipolar) or 2^p-1 (unipolar)       */
  int stoc_len;         /* L                                                       */
  int rng_levels;       /* G, the resolved enable grid (2^p when rng_levels=None)  */
  int chunk_d;          /* > 0 selects the chunked per_row path (2D bipolar, D > chunk_d) */
  int group_a, group_b; /* per_row row-group sizes                                 */
  int batch;            /* BH; 1 for 2D inputs                                     */
  int n, m, d;          /* a: (batch, n, d), b: (batch, m, d), out: (batch, n, m)  */
  const float* a;
  const float* b;
  const float* smooth_scales; /* (d,) or NULL                                      */
  float* out;
  const int16_t* ktab;     /* from scmp_build_tables                               */
  const uint32_t* pattern; /* from scmp_build_tables                               */
  const int32_t* amap;     /* (d,) table row of dimension j for operand a           */
  const int32_t* bmap;     /* (d,) table row of dimension j for operand b           */
  int vcap;                /* as passed to scmp_build_tables                       */
  int lp;                  /* as passed to scmp_build_tables                       */
  int flags;               /* SCMP_FLAG_*                                          */
  const double* tensor_ranges; /* per_tensor only, may be NULL: device {a_max, a_min,
                                  b_max, b_min} used instead of reducing a and b on the
                                  device; the max_fp_* / min_fp_* arguments of
                                  _sc_matmul_per_tensor (kernels.py:1053-1066), e.g.
                                  global ranges when b is sharded over devices       */
  /* Result written to several buffers, e.g. this rank's column block into every
   * rank's full output (an all-gather fused into the GEMM's epilogue; no
   * reference counterpart). When n_out_peers > 0, `out` is ignored and element
   * (h, i, j) of the (batch, n, m) result is stored at
   *   out_peers[k][out_offset + (h*n + i) * out_ld + j]   for k < n_out_peers,
   * out_peers being a HOST array of device pointers (this device's memory or
   * peers' memory mapped with scmp_peer_open). */
  float* const* out_peers;
  int n_out_peers;         /* 0 .. SCMP_MAX_OUT_PEERS                              */
  int out_ld;              /* row stride of the destinations, >= m                */
  long long out_offset;    /* element offset of (0, 0, 0) in every destination    */
  const uint32_t* pattern4; /* from scmp_build_tables, or NULL (int8 operands)     */
  /* With n_out_peers > 1: 1 + the index in out_peers of the destination in this
   * device's own memory, or 0 if none is. When set, the wide-tile GEMM stores
   * each finished tile there first, frees the tile's accumulator, and copies
   * the tile to the other destinations while the next tile's MMAs run. */
  int out_self;
} scmp_matmul_desc;

#define SCMP_MAX_OUT_PEERS 8

/*
 * Device buffers shared between the processes of one node (CUDA IPC), the
 * destinations of a fused all-gather. scmp_peer_alloc allocates `bytes` on
 * the current device and returns the pointer and a 64-byte handle that other
 * processes pass to scmp_peer_open to map the same memory (peer access
 * enabled); scmp_peer_close unmaps a mapped buffer, scmp_peer_free frees an
 * allocated one.
 */
int scmp_peer_alloc(size_t bytes, void** ptr, void* handle64);
int scmp_peer_open(const void* handle64, void** ptr);
int scmp_peer_close(void* ptr);
int scmp_peer_free(void* ptr);

/* Bytes of device workspace scmp_sc_matmul needs for `desc` (host-only call). */
int scmp_sc_matmul_workspace_size(const scmp_matmul_desc* desc, size_t* bytes);

int scmp_sc_matmul(const scmp_matmul_desc* desc, void* workspace, size_t workspace_bytes,
                   void* stream);

/*
 * Row levels: rows of a in groups with their own stream lengths, in one call
 * (one quantisation pass over a, one SC-GEMM launch).
 *
 * Replaces the caller-side mixed precision of the reference: rows classified
 * into levels (classify_rows_by_metric, scmp_kernels/mp/config.py:154-191,
 * and the range classifier of :924-1007) and one sc_matmul per level on the
 * gathered rows, scattered back (the per-level calls of the chunked MLP path,
 * sc/kernels.py:1443-1566). The result equals that composition bit for bit:
 * row i of a is computed with the stream length, grid and tables of level
 * row_level[i].
 *
 * desc: as for scmp_sc_matmul with granularity SCMP_PER_ROW, batch 1 and
 * either chunk_d > 0 (bipolar, chunked path; group sizes are ignored there,
 * as in the reference) or group_a == 1; its stoc_len, rng_levels, ktab,
 * pattern, pattern4, amap, bmap, vcap and lp are not used (the levels carry
 * them) and neither is SCMP_FLAG_B_READY. levels: n_levels (1..4) HOST
 * descriptors with each level's tables from scmp_build_tables (pattern4
 * required; padded stream lengths 64..512). row_level: DEVICE int32 (n,),
 * the level of every row of a; a row with a level outside [0, n_levels) is
 * left out of the result and recorded as a device error. Runs on SM pairs of
 * an sm_100 device only (SCMP_ERR_UNSUPPORTED otherwise).
 */
typedef struct scmp_level_desc {
  int stoc_len;             /* L of this level                                  */
  int rng_levels;           /* G of this level                                  */
  int vcap, lp;             /* as passed to scmp_build_tables for this level    */
  const int16_t* ktab;      /* this level's tables (scmp_build_tables)          */
  const uint32_t* pattern4;
  const int32_t* amap;      /* (d,) table row of every dimension, as for scmp_matmul_desc */
  const int32_t* bmap;
} scmp_level_desc;

int scmp_sc_matmul_levels_workspace_size(const scmp_matmul_desc* desc, const scmp_level_desc* levels,
                                         int n_levels, size_t* bytes);
int scmp_sc_matmul_levels(const scmp_matmul_desc* desc, const scmp_level_desc* levels, int n_levels,
                          const int32_t* row_level, void* workspace, size_t workspace_bytes, void* stream);

/*
 * scmp_sc_matmul without a caller workspace. No counterpart in the reference.
 * For callers that cannot allocate device memory (a host reaching this
 * library through a plain C FFI with no device allocator, or a process that
 * reserved all its device memory up front and must not call cudaMalloc,
 * which can also synchronise the device). Runs the same pipeline on a fixed
 * 16 MiB scratch array inside the library's device image (present on every
 * GPU that loads the library until exit); allocates and frees nothing. The
 * first call on a device looks up that array's address, so make it before
 * any stream capture. Calls needing more than 16 MiB of scratch (see
 * scmp_sc_matmul_workspace_size) return SCMP_ERR_INVALID_ARG. All calls on a
 * device share the array: calls that overlap on the GPU race.
 */
int scmp_sc_matmul_noalloc(const scmp_matmul_desc* desc, void* stream);

/*
 * Enable-signal matmul on already-quantised operands.
 * Replaces enable_matmul_triton + enable_matmul_tiled_kernel
 * (scmp_kernels/sc/kernels.py:798-868, 176-252).
 *   boundary_a (n, d) int16, boundary_b (m, d) int16, sign_a (n, d) int8 and
 *   sign_b (m, d) int8 (signs ignored when is_bipolar == 0);
 *   out (n, m) = fl32(S * fl32(q_max_sq / L)) with S the integer accumulator.
 * Tables and maps as in scmp_matmul_desc. The workspace holds the signed
 * thermometer lengths; scmp_enable_matmul_workspace_size gives its size.
 */
int scmp_enable_matmul_workspace_size(int n, int m, int d, size_t* bytes);
int scmp_enable_matmul(const int16_t* ktab, const uint32_t* pattern, const int32_t* amap,
                       const int32_t* bmap, int vcap, int L, int lp, const int16_t* boundary_a,
                       const int16_t* boundary_b, const int8_t* sign_a, const int8_t* sign_b,
                       int n, int m, int d, float q_max_sq, int is_bipolar, float* out,
                       void* workspace, size_t workspace_bytes, int flags, void* stream);

/*
 * Quantisers with the reference's output formats (scmp_kernels/quant/).
 *
 * scmp_fused_quantize_bipolar        fused_quantize_bipolar, fused.py:162-189
 *   boundary (rows, cols) int16, sign int8; *scale_out = (host double) the
 *   scale max(abs_max, 1e-5) / q_max.
 * scmp_fused_quantize_bipolar_perrow fused_quantize_bipolar_perrow, fused.py:134-159
 *   per-row on-device scale written to scale_row (rows,) float32.
 * scmp_fused_quantize_unipolar       fused_quantize_unipolar, fused.py:192-234
 *   boundary int32; row_sum (rows,) float32 written when non-NULL
 *   (compute_sum=True); *scale_out and *zp_out are host doubles.
 * scmp_fused_quant_bipolar_batched   fused_quant_bipolar_batched_kernel, fused.py:237-283
 *   x (bh, rows, cols); inv_scale (bh,) float32 device; outputs transposed
 *   to (bh, cols, rows).
 * scmp_grouped_symmetric_quant       _grouped_symmetric_quant, grouped.py:13-75
 * scmp_grouped_asymmetric_quant      _grouped_asymmetric_quant, grouped.py:78-133
 * scmp_grouped_symmetric_quant_batched  _grouped_symmetric_quant_batched, grouped.py:136-163
 *   (group == 1 or group >= rows; any other group returns SCMP_ERR_UNSUPPORTED)
 *   x_int is float32 like the reference's; sign int8 with 0 -> +1.
 * The grouped quantisers need scratch: group_stats holds 3 floats per group.
 */
int scmp_fused_quantize_bipolar(const float* x, int rows, int cols, double abs_max, int sc_prec,
                                int rng_levels, int16_t* boundary, int8_t* sign, double* scale_out,
                                void* stream);
int scmp_fused_quantize_bipolar_perrow(const float* x, int rows, int cols, int sc_prec,
                                       int rng_levels, int16_t* boundary, int8_t* sign,
                                       float* scale_row, void* stream);
int scmp_fused_quantize_unipolar(const float* x, int rows, int cols, double fp_max, double fp_min,
                                 int sc_prec, int rng_levels, int32_t* boundary, float* row_sum,
                                 double* scale_out, double* zp_out, void* stream);
int scmp_fused_quant_bipolar_batched(const float* x, int bh, int rows, int cols,
                                     const float* inv_scale, int sc_prec, int rng_levels,
                                     int16_t* boundary, int8_t* sign, void* stream);
int scmp_grouped_symmetric_quant(const float* x, int batch, int rows, int cols, int group,
                                 int q_max, float* scale_row, float* x_int, int8_t* sign,
                                 float* group_stats, void* stream);
int scmp_grouped_asymmetric_quant(const float* x, int rows, int cols, int group, int q_max,
                                  float* scale_row, float* zp_row, float* x_int,
                                  float* group_stats, void* stream);

/* Profiling hook (no reference counterpart; the reference has no native
 * timing). While set, scmp_sc_matmul and scmp_enable_matmul record the CUDA
 * event gemm_start on their stream right before the SC-GEMM launch and
 * gemm_stop right after it, so a caller can time the GEMM kernel alone. Both
 * are cudaEvent_t passed as void*; NULL, NULL turns the hook off. Process-wide. */
int scmp_set_profile_events(void* gemm_start, void* gemm_stop);
/* The same for the operand preparation of scmp_sc_matmul: quant_start is
 * recorded before its first kernel (row statistics, quantisers, the padded
 * row map) and quant_stop after its last, before the SC-GEMM; NULL, NULL
 * turns it off. Process-wide. */
int scmp_set_quant_profile_events(void* quant_start, void* quant_stop);

/* Diagnostics. scmp_device_error synchronises the device, returns in *code
 * the first error a kernel recorded since the last call (SCMP_OK if none)
 * and clears it. */
int scmp_device_error(int* code);
const char* scmp_last_error(void);
int scmp_abi_version(void);
/* Number of CUDA kernels this library has launched in the process so far
 * (every entry point counts its own launches). */
unsigned long long scmp_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* SCMP_B200_H */
