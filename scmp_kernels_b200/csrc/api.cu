// extern "C" entry points declared in include/scmp_b200.h.
#include <stdio.h>
#include <string.h>

#include <string>

#include "quant.cuh"

namespace scmp {

static thread_local std::string t_last_error;
static cudaEvent_t g_prof_start = nullptr, g_prof_stop = nullptr;
static cudaEvent_t g_qprof_start = nullptr, g_qprof_stop = nullptr;

// Copy of the dimension -> table-row map padded with zeros to 8*ceil(d/8),
// so the GEMM can read it in aligned blocks of eight.
__global__ void pad_map_kernel(const int32_t* __restrict__ src, int d, int32_t* __restrict__ dst) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < d8(d) * 8) dst[i] = i < d ? src[i] : 0;
}
static cudaError_t launch_pad_map(const int32_t* src, int d, int32_t* dst, cudaStream_t st) {
  pad_map_kernel<<<cdiv(d8(d) * 8, 256), 256, 0, st>>>(src, d, dst);
  count_launch();
  return cudaGetLastError();
}

// SC-GEMM launch bracketed by the optional profiling events.
static cudaError_t launch_gemm(const GemmArgs& g, int flags, cudaStream_t st) {
  if (g_prof_start) cudaEventRecord(g_prof_start, st);
  const bool tc = !(flags & SCMP_FLAG_FORCE_SIMT) && gemm_tc_supported(g);
  cudaError_t e = tc ? launch_gemm_tc(g, st) : launch_gemm_simt(g, st);
  if (g_prof_stop) cudaEventRecord(g_prof_stop, st);
  return e;
}

static int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}
static int cuda_fail(cudaError_t e, const char* what) {
  return fail(SCMP_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}
#define SCMP_CUDA(call, what)                  \
  do {                                         \
    cudaError_t e_ = (call);                   \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

// Bump allocator over the caller's workspace; a dry run only measures.
struct Carver {
  char* base = nullptr;
  size_t off = 0;
  template <class T>
  T* take(size_t count) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
};

struct Plan {
  int16_t* ka = nullptr;
  int16_t* vb = nullptr;
  int32_t* bmap = nullptr;
  float* stats_a = nullptr;
  float* stats_b = nullptr;
  float* scale_a = nullptr;
  float* scale_b = nullptr;
  float* zp_a = nullptr;
  float* zp_b = nullptr;
  float* sum_a = nullptr;
  float* sum_b = nullptr;
  float* scal = nullptr;
  bool chunked = false;
  int nchunks = 1;
  int* split_acc = nullptr;  // tcgen05 GEMM: accumulators and counters of the split last wave
  int* split_cnt = nullptr;
};

static bool is_chunked(const scmp_matmul_desc* d) {
  return d->granularity == SCMP_PER_ROW && d->chunk_d > 0 && d->mode == SCMP_BIPOLAR &&
         d->batch == 1 && d->d > d->chunk_d;
}

static int validate(const scmp_matmul_desc* d) {
  if (!d) return fail(SCMP_ERR_INVALID_ARG, "sc_matmul: null descriptor");
  if (d->granularity < SCMP_PER_TENSOR || d->granularity > SCMP_PER_HEAD)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul: unknown granularity");
  if (d->mode != SCMP_BIPOLAR && d->mode != SCMP_UNIPOLAR)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul: unknown mode");
  if (d->granularity == SCMP_PER_HEAD && d->mode != SCMP_BIPOLAR)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul: granularity='per_head' currently only supports mode='bipolar'");
  if ((d->flags & SCMP_FLAG_B_READY) && (d->granularity != SCMP_PER_ROW || is_chunked(d)))
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul: SCMP_FLAG_B_READY applies to per_row calls without chunk_d");
  const int pmin = d->mode == SCMP_BIPOLAR ? 2 : 1;
  if (d->sc_prec < pmin || d->sc_prec > 15)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul: sc_prec out of range (bipolar 2..15, unipolar 1..15)");
  if (d->stoc_len < 1 || d->stoc_len > 32767)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul: stoc_len must be in [1, 32767]");
  if (d->lp < d->stoc_len || d->lp % 32 != 0)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul: lp must be a multiple of 32 and >= stoc_len");
  if (d->rng_levels < 1) return fail(SCMP_ERR_INVALID_ARG, "sc_matmul: rng_levels must be >= 1");
  if (d->vcap < 1 || d->vcap > 32767) return fail(SCMP_ERR_INVALID_ARG, "sc_matmul: vcap must be in [1, 32767]");
  if (d->batch < 1 || d->n < 0 || d->m < 0 || d->d < 1)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul: bad shape (batch >= 1, n, m >= 0, d >= 1)");
  if (d->group_a < 1 || d->group_b < 1)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul: group sizes must be >= 1");
  if (d->n_out_peers < 0 || d->n_out_peers > SCMP_MAX_OUT_PEERS)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul: n_out_peers must be in [0, SCMP_MAX_OUT_PEERS]");
  if (d->n_out_peers > 0 && (d->out_ld < d->m || d->out_offset < 0 || !d->out_peers))
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul: out_peers needs out_ld >= m, out_offset >= 0 and the pointer array");
  if (d->granularity == SCMP_PER_ROW && d->batch > 1 && d->mode == SCMP_BIPOLAR) {
    auto ok = [&](int g, int rows) { return g == 1 || g >= rows; };
    if (!ok(d->group_a, d->n) || !ok(d->group_b, d->m))
      return fail(SCMP_ERR_UNSUPPORTED,
                  "_grouped_symmetric_quant_batched: group size not supported (use G=1 or G>=rows)");
  }
  return SCMP_OK;
}


static void carve(const scmp_matmul_desc* d, Carver& c, Plan& p) {
  const size_t na = (size_t)d->batch * d->n, nb = (size_t)d->batch * d->m;
  const size_t dd = (size_t)d8(d->d) * 8;
  p.chunked = is_chunked(d);
  p.nchunks = p.chunked ? cdiv(d->d, d->chunk_d) : 1;
  const size_t rows_a = p.chunked ? na * p.nchunks : na, rows_b = p.chunked ? nb * p.nchunks : nb;
  // b's buffers first: their offsets do not depend on n (SCMP_FLAG_B_READY)
  p.vb = c.take<int16_t>(nb * dd);
  p.stats_b = c.take<float>(3 * nb);
  p.scale_b = c.take<float>(rows_b > (size_t)d->batch ? rows_b : d->batch);
  p.zp_b = c.take<float>(nb > (size_t)d->batch ? nb : d->batch);
  p.sum_b = c.take<float>(nb);
  p.ka = c.take<int16_t>(na * dd);
  p.bmap = c.take<int32_t>(dd);
  p.stats_a = c.take<float>(3 * na);
  p.scale_a = c.take<float>(rows_a > (size_t)d->batch ? rows_a : d->batch);
  p.zp_a = c.take<float>(na > (size_t)d->batch ? na : d->batch);
  p.sum_a = c.take<float>(na);
  p.scal = c.take<float>(8);
  if (!(d->flags & (SCMP_FLAG_FORCE_SIMT | SCMP_FLAG_NO_SPLIT))) {
    const int unit_d = p.chunked ? d->chunk_d : d->d;
    const bool f4 = d->pattern4 != nullptr;
    const size_t bytes = gemm_tc_split_bytes(d->batch, d->n, d->m, d->d, unit_d, d->lp, f4);
    if (bytes) {
      char* blk = c.take<char>(bytes);
      if (blk) {
        p.split_acc = reinterpret_cast<int*>(blk);
        p.split_cnt =
            reinterpret_cast<int*>(blk + gemm_tc_split_cnt_offset(d->batch, d->n, d->m, d->d, unit_d, d->lp, f4));
      }
    }
  }
}

static QuantArgs base_quant(const scmp_matmul_desc* d, bool side_a, int q) {
  QuantArgs a{};
  a.x = side_a ? d->a : d->b;
  a.vec = (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && d->d % 4 == 0;
  a.rows_per_batch = side_a ? d->n : d->m;
  a.rows = d->batch * a.rows_per_batch;
  a.d = d->d;
  a.smooth = d->smooth_scales;
  a.smooth_div = side_a ? 1 : 0;
  a.q = q;
  a.qmin = -(float)q;
  a.G = d->rng_levels;
  a.ratio = (float)d->rng_levels / (float)q;
  a.vcap = d->vcap;
  a.ktab = side_a ? d->ktab : nullptr;
  a.amap = d->amap;
  return a;
}

}  // namespace scmp

using namespace scmp;

extern "C" {

int scmp_abi_version(void) { return SCMP_ABI_VERSION; }

unsigned long long scmp_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int scmp_set_profile_events(void* gemm_start, void* gemm_stop) {
  g_prof_start = (cudaEvent_t)gemm_start;
  g_prof_stop = (cudaEvent_t)gemm_stop;
  return SCMP_OK;
}

int scmp_set_quant_profile_events(void* quant_start, void* quant_stop) {
  g_qprof_start = (cudaEvent_t)quant_start;
  g_qprof_stop = (cudaEvent_t)quant_stop;
  return SCMP_OK;
}

const char* scmp_last_error(void) { return t_last_error.c_str(); }

int scmp_device_error(int* code) {
  SCMP_CUDA(cudaDeviceSynchronize(), "scmp_device_error: synchronize");
  DeviceError h{0, 0}, z{0, 0};
  SCMP_CUDA(cudaMemcpyFromSymbol(&h, g_device_error, sizeof(h)), "scmp_device_error: read");
  SCMP_CUDA(cudaMemcpyToSymbol(g_device_error, &z, sizeof(z)), "scmp_device_error: clear");
  if (code) *code = h.code;
  if (h.code) {
    char buf[96];
    snprintf(buf, sizeof buf, "device error %d recorded at site %d", h.code, h.where);
    t_last_error = buf;
  }
  return SCMP_OK;
}

int scmp_build_tables(const int32_t* ra, int n_ra, const int32_t* rb, int n_rb, int L, int lp,
                      int vcap, int16_t* ktab, uint32_t* pattern, uint32_t* pattern4, void* stream) {
  if (L < 1 || lp < L || lp % 32 || vcap < 1 || vcap > 32767 || n_ra < 0 || n_rb < 0)
    return fail(SCMP_ERR_INVALID_ARG, "build_tables: bad sizes");
  if ((n_ra && (!ra || !ktab)) || (n_rb && (!rb || !pattern)))
    return fail(SCMP_ERR_INVALID_ARG, "build_tables: null pointer");
  SCMP_CUDA(launch_build_tables(ra, n_ra, rb, n_rb, L, lp, vcap, ktab, pattern, pattern4,
                                (cudaStream_t)stream),
            "build_tables");
  return SCMP_OK;
}

int scmp_peer_alloc(size_t bytes, void** ptr, void* handle64) {
  if (!ptr || !handle64 || bytes == 0) return fail(SCMP_ERR_INVALID_ARG, "peer_alloc: bad arguments");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  void* p = nullptr;
  SCMP_CUDA(cudaMalloc(&p, bytes), "peer_alloc: cudaMalloc");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "peer_alloc: cudaIpcGetMemHandle");
  }
  memcpy(handle64, &h, sizeof h);
  *ptr = p;
  return SCMP_OK;
}

int scmp_peer_open(const void* handle64, void** ptr) {
  if (!ptr || !handle64) return fail(SCMP_ERR_INVALID_ARG, "peer_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof h);
  SCMP_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "peer_open: cudaIpcOpenMemHandle");
  return SCMP_OK;
}

int scmp_peer_close(void* ptr) {
  SCMP_CUDA(cudaIpcCloseMemHandle(ptr), "peer_close");
  return SCMP_OK;
}

int scmp_peer_free(void* ptr) {
  SCMP_CUDA(cudaFree(ptr), "peer_free");
  return SCMP_OK;
}

int scmp_sc_matmul_workspace_size(const scmp_matmul_desc* desc, size_t* bytes) {
  int s = validate(desc);
  if (s) return s;
  if (!bytes) return fail(SCMP_ERR_INVALID_ARG, "workspace_size: null output");
  Carver c;
  Plan p;
  carve(desc, c, p);
  *bytes = c.off;
  return SCMP_OK;
}

int scmp_sc_matmul(const scmp_matmul_desc* d, void* workspace, size_t workspace_bytes,
                   void* stream) {
  int s = validate(d);
  if (s) return s;
  if (d->n == 0 || d->m == 0) return SCMP_OK;
  const bool b_ready = (d->flags & SCMP_FLAG_B_READY) != 0;
  if (!d->a || (!d->b && !b_ready) || (!d->out && d->n_out_peers == 0) || !d->ktab || !d->pattern || !d->amap ||
      !d->bmap)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul: null operand, output or table pointer");
  for (int k = 0; k < d->n_out_peers; ++k)
    if (!d->out_peers[k]) return fail(SCMP_ERR_INVALID_ARG, "sc_matmul: null out_peers entry");
  Carver c;
  Plan p;
  carve(d, c, p);
  if (!workspace || workspace_bytes < c.off)
    return fail(SCMP_ERR_WORKSPACE, "sc_matmul: workspace missing or too small");
  c = Carver{static_cast<char*>(workspace), 0};
  carve(d, c, p);
  cudaStream_t st = (cudaStream_t)stream;

  const bool bip = d->mode == SCMP_BIPOLAR;
  const int q = bip ? (1 << (d->sc_prec - 1)) - 1 : (1 << d->sc_prec) - 1;
  QuantArgs qa = base_quant(d, true, q), qb = base_quant(d, false, q);
  qa.out16 = p.ka;
  qb.out16 = p.vb;

  GemmArgs g{};
  g.batch = d->batch;
  g.n = d->n;
  g.m = d->m;
  g.d = d->d;
  g.L = d->stoc_len;
  g.lp = d->lp;
  g.vcap = d->vcap;
  g.bipolar = bip;
  g.ka = p.ka;
  g.vb = p.vb;
  g.pattern = d->pattern;
  g.pattern4 = d->pattern4;
  g.bmap = p.bmap;
  if (g_qprof_start) cudaEventRecord(g_qprof_start, st);
  SCMP_CUDA(launch_pad_map(d->bmap, d->d, p.bmap, st), "pad bmap");
  g.unit_d = d->d;
  if (d->n_out_peers > 0) {
    for (int k = 0; k < d->n_out_peers; ++k) g.outs[k] = d->out_peers[k];
    g.nouts = d->n_out_peers;
    g.out_off = d->out_offset;
    g.out_ld = d->out_ld;
  } else {
    g.outs[0] = d->out;
    g.nouts = 1;
    g.out_off = 0;
    g.out_ld = d->m;
  }
  g.out_vec = g.out_off % 4 == 0 && g.out_ld % 4 == 0;
  g.out_self = d->n_out_peers > 1 && d->out_self >= 1 && d->out_self <= d->n_out_peers ? d->out_self : 0;
  for (int k = 0; k < g.nouts; ++k) g.out_vec &= (reinterpret_cast<uintptr_t>(g.outs[k]) & 15) == 0;
  g.split_acc = p.split_acc;
  g.split_cnt = p.split_cnt;
  g.epi.inner = (float)(q * q) / (float)d->stoc_len;
  g.epi.fd = (float)d->d;

  if (d->granularity == SCMP_PER_TENSOR) {
    if (!d->tensor_ranges) {
      SCMP_CUDA(launch_row_stats(qa, p.stats_a, st), "per_tensor stats a");
      SCMP_CUDA(launch_row_stats(qb, p.stats_b, st), "per_tensor stats b");
    }
    SCMP_CUDA(launch_tensor_params(p.stats_a, qa.rows, p.stats_b, qb.rows, d->d, q, !bip,
                                   d->tensor_ranges, p.scal, st),
              "per_tensor params");
    qa.params = qb.params = p.scal;
    qa.param_off = 4;
    qb.param_off = 5;
    g.epi.scal = p.scal;
    if (bip) {
      SCMP_CUDA(launch_quant_rows(Q_TENSOR_BIP, qa, st), "per_tensor quant a");
      SCMP_CUDA(launch_quant_rows(Q_TENSOR_BIP, qb, st), "per_tensor quant b");
      g.epi.kind = EPI_SCALAR;
    } else {
      qa.row_sum = p.sum_a;
      qb.row_sum = p.sum_b;
      SCMP_CUDA(launch_quant_rows(Q_TENSOR_UNI, qa, st), "per_tensor quant a");
      SCMP_CUDA(launch_quant_rows(Q_TENSOR_UNI, qb, st), "per_tensor quant b");
      g.epi.kind = EPI_SCALAR_UNI;
      g.epi.asum = p.sum_a;
      g.epi.bsum = p.sum_b;
    }
  } else if (d->granularity == SCMP_PER_HEAD) {
    SCMP_CUDA(launch_head_params(qa, d->batch, q, p.scale_a, p.zp_a, st), "per_head params a");
    SCMP_CUDA(launch_head_params(qb, d->batch, q, p.scale_b, p.zp_b, st), "per_head params b");
    qa.params = p.zp_a;
    qb.params = p.zp_b;
    qa.qmin = qb.qmin = -(float)(q + 1);
    SCMP_CUDA(launch_quant_rows(Q_HEAD_BIP, qa, st), "per_head quant a");
    SCMP_CUDA(launch_quant_rows(Q_HEAD_BIP, qb, st), "per_head quant b");
    g.epi.kind = EPI_HEAD;
    g.epi.sa = p.scale_a;
    g.epi.sb = p.scale_b;
  } else if (p.chunked) {
    qa.chunk_d = qb.chunk_d = d->chunk_d;
    qa.chunk_scale = p.scale_a;
    qb.chunk_scale = p.scale_b;
    SCMP_CUDA(launch_quant_rows(Q_ROWCHUNK_BIP, qa, st), "chunked quant a");
    SCMP_CUDA(launch_quant_rows(Q_ROWCHUNK_BIP, qb, st), "chunked quant b");
    g.unit_d = d->chunk_d;
    g.epi.kind = EPI_CHUNK;
    g.epi.sa = p.scale_a;
    g.epi.sb = p.scale_b;
  } else {
    // per_row: row groups inside every batch entry
    const int recipe = bip ? (d->batch > 1 ? Q_BATCH_SYM : Q_GROUP_SYM) : Q_GROUP_ASYM;
    const int gp = bip ? GP_SYM : GP_ASYM;
    QuantArgs* ops[2] = {&qa, &qb};
    const int groups[2] = {d->group_a, d->group_b};
    float* stats[2] = {p.stats_a, p.stats_b};
    float* scales[2] = {p.scale_a, p.scale_b};
    float* zps[2] = {p.zp_a, p.zp_b};
    float* sums[2] = {p.sum_a, p.sum_b};
    for (int i = 0; i < 2; ++i) {
      if (i == 1 && b_ready) break;  // b's operand, scales, zero points, sums: in the workspace
      QuantArgs& o = *ops[i];
      o.row_scale = scales[i];
      o.row_zp = zps[i];
      if (!bip) o.row_sum = sums[i];
      if (groups[i] == 1 || o.rows_per_batch == 1) {
        o.self_stats = 1;
      } else {
        SCMP_CUDA(launch_row_stats(o, stats[i], st), "per_row stats");
        SCMP_CUDA(launch_group_params(stats[i], d->batch, o.rows_per_batch, groups[i], q, gp,
                                      scales[i], bip ? nullptr : zps[i], st),
                  "per_row group params");
      }
      SCMP_CUDA(launch_quant_rows(recipe, o, st), "per_row quant");
    }
    g.epi.kind = bip ? EPI_ROW : EPI_ROW_UNI;
    g.epi.sa = p.scale_a;
    g.epi.sb = p.scale_b;
    g.epi.zpa = p.zp_a;
    g.epi.zpb = p.zp_b;
    g.epi.asum = p.sum_a;
    g.epi.bsum = p.sum_b;
  }

  if (g_qprof_stop) cudaEventRecord(g_qprof_stop, st);
  SCMP_CUDA(launch_gemm(g, d->flags, st), "sc_gemm");
  return SCMP_OK;
}

}  // extern "C"
