// scmp_sc_matmul_levels: row groups of a with their own stream lengths, in one
// quantisation pass over a and one SC-GEMM launch.
//
// The reference leaves mixed precision to its caller: rows are classified into
// levels (scmp_kernels/mp/config.py:154-191) and sc_matmul runs once per level
// on the gathered rows. Here a's rows are permuted on the device so that each
// level fills whole 256-row tiles (level_perm_kernel), a is quantised once with
// every row on its level's grid and tables, b once per level (its grid, and so
// its operand, depends on the level), and one GEMM launch takes every tile's
// stream length, b operand and epilogue scale from its level; the epilogue
// writes each permuted row to its place in the result. Per-row quantisation is
// row-local, so every row's bits equal those of the per-level call.

namespace scmp {

struct LevelPlan {
  int16_t* ka = nullptr;
  int16_t* vb[kMaxLevels] = {};
  int32_t* bmap[kMaxLevels] = {};
  float* stats_b = nullptr;
  float* scale_b = nullptr;
  float* zp_b = nullptr;
  float* sum_b = nullptr;
  float* scale_a = nullptr;
  float* zp_a = nullptr;
  float* sum_a = nullptr;
  int* row_of = nullptr;
  int* lev_tile0 = nullptr;
  int n_pad = 0, nchunks = 1;
  bool chunked = false;
};

// a's permuted rows: every level padded to whole tiles of 256 rows.
static int levels_rows(int n, int nlev) { return 256 * (cdiv(n, 256) + nlev - 1); }

static void carve_levels(const scmp_matmul_desc* d, int nlev, Carver& c, LevelPlan& p) {
  const size_t dd = (size_t)d8(d->d) * 8, m = (size_t)d->m;
  p.chunked = d->chunk_d > 0 && d->d > d->chunk_d;
  p.nchunks = p.chunked ? cdiv(d->d, d->chunk_d) : 1;
  p.n_pad = levels_rows(d->n, nlev);
  const size_t na = (size_t)p.n_pad;
  for (int l = 0; l < nlev; ++l) {
    p.vb[l] = c.take<int16_t>(m * dd);
    p.bmap[l] = c.take<int32_t>(dd);
  }
  p.stats_b = c.take<float>(3 * m);
  p.scale_b = c.take<float>(p.nchunks * m);
  p.zp_b = c.take<float>(m);
  p.sum_b = c.take<float>(m);
  p.ka = c.take<int16_t>(na * dd);
  p.scale_a = c.take<float>(p.nchunks * na);
  p.zp_a = c.take<float>(na);
  p.sum_a = c.take<float>(na);
  p.row_of = c.take<int>(na);
  p.lev_tile0 = c.take<int>(kMaxLevels + 1);
}

static int validate_levels(const scmp_matmul_desc* d, const scmp_level_desc* lv, int nlev) {
  if (!d) return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_levels: null descriptor");
  if (d->granularity != SCMP_PER_ROW)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_levels: row levels apply to granularity='per_row'");
  if (d->mode != SCMP_BIPOLAR && d->mode != SCMP_UNIPOLAR) return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_levels: unknown mode");
  const int pmin = d->mode == SCMP_BIPOLAR ? 2 : 1;
  if (d->sc_prec < pmin || d->sc_prec > 15)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_levels: sc_prec out of range (bipolar 2..15, unipolar 1..15)");
  if (d->batch != 1 || d->n < 0 || d->m < 0 || d->d < 1)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_levels: bad shape (2D operands: batch 1, n, m >= 0, d >= 1)");
  if (d->group_a < 1 || d->group_b < 1) return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_levels: group sizes must be >= 1");
  const bool chunked = d->chunk_d > 0 && d->d > d->chunk_d;
  if (chunked && d->mode != SCMP_BIPOLAR)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_levels: chunk_d > 0 requires mode='bipolar'");
  if (chunked && d->chunk_d % 8 != 0)
    return fail(SCMP_ERR_UNSUPPORTED, "sc_matmul_levels: chunk_d must be a multiple of 8");
  if (!chunked && d->group_a != 1)
    return fail(SCMP_ERR_UNSUPPORTED, "sc_matmul_levels: row groups of a (group_a > 1) are not supported");
  if (d->flags & (SCMP_FLAG_B_READY | SCMP_FLAG_FORCE_SIMT))
    return fail(SCMP_ERR_UNSUPPORTED, "sc_matmul_levels: SCMP_FLAG_B_READY and SCMP_FLAG_FORCE_SIMT do not apply");
  if (d->n_out_peers < 0 || d->n_out_peers > SCMP_MAX_OUT_PEERS)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_levels: n_out_peers must be in [0, SCMP_MAX_OUT_PEERS]");
  if (d->n_out_peers > 0 && (d->out_ld < d->m || d->out_offset < 0 || !d->out_peers))
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_levels: out_peers needs out_ld >= m, out_offset >= 0 and the pointer array");
  if (!lv || nlev < 1 || nlev > kMaxLevels)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_levels: 1 to 4 levels");
  for (int l = 0; l < nlev; ++l) {
    const scmp_level_desc& x = lv[l];
    if (x.stoc_len < 1 || x.rng_levels < 1 || x.vcap < 1 || x.vcap > 32767 || x.lp < x.stoc_len)
      return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_levels: bad level (stoc_len, rng_levels, vcap or lp)");
    if (x.lp < 64 || x.lp > 512 || (x.lp & (x.lp - 1)))
      return fail(SCMP_ERR_UNSUPPORTED, "sc_matmul_levels: padded stream lengths of 64 to 512 only");
    if (!x.ktab || !x.pattern4 || !x.amap || !x.bmap)
      return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_levels: null level table pointer");
  }
  return SCMP_OK;
}

}  // namespace scmp

using namespace scmp;

extern "C" {

int scmp_sc_matmul_levels_workspace_size(const scmp_matmul_desc* desc, const scmp_level_desc* levels,
                                         int n_levels, size_t* bytes) {
  int s = validate_levels(desc, levels, n_levels);
  if (s) return s;
  if (!bytes) return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_levels_workspace_size: null output");
  Carver c;
  LevelPlan p;
  carve_levels(desc, n_levels, c, p);
  *bytes = c.off;
  return SCMP_OK;
}

int scmp_sc_matmul_levels(const scmp_matmul_desc* d, const scmp_level_desc* lv, int nlev,
                          const int32_t* row_level, void* workspace, size_t workspace_bytes, void* stream) {
  int s = validate_levels(d, lv, nlev);
  if (s) return s;
  if (d->n == 0 || d->m == 0) return SCMP_OK;
  if (!d->a || !d->b || (!d->out && d->n_out_peers == 0) || !row_level)
    return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_levels: null operand, output or row_level pointer");
  for (int k = 0; k < d->n_out_peers; ++k)
    if (!d->out_peers[k]) return fail(SCMP_ERR_INVALID_ARG, "sc_matmul_levels: null out_peers entry");
  Carver c;
  LevelPlan p;
  carve_levels(d, nlev, c, p);
  if (!workspace || workspace_bytes < c.off)
    return fail(SCMP_ERR_WORKSPACE, "sc_matmul_levels: workspace missing or too small");
  c = Carver{static_cast<char*>(workspace), 0};
  carve_levels(d, nlev, c, p);
  cudaStream_t st = (cudaStream_t)stream;

  const bool bip = d->mode == SCMP_BIPOLAR;
  const int q = bip ? (1 << (d->sc_prec - 1)) - 1 : (1 << d->sc_prec) - 1;

  GemmArgs g{};
  g.batch = 1;
  g.n = p.n_pad;
  g.m = d->m;
  g.d = d->d;
  g.L = lv[0].stoc_len;
  g.lp = lv[0].lp;
  g.vcap = lv[0].vcap;
  g.bipolar = bip;
  g.ka = p.ka;
  g.unit_d = p.chunked ? d->chunk_d : d->d;
  g.nlev = nlev;
  g.lev_tile0 = p.lev_tile0;
  g.row_of = p.row_of;
  g.n_out = d->n;
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
  for (int l = 0; l < nlev; ++l) {
    g.lev[l].vb = p.vb[l];
    g.lev[l].pattern4 = lv[l].pattern4;
    g.lev[l].bmap = p.bmap[l];
    g.lev[l].vcap = lv[l].vcap;
    g.lev[l].lp = lv[l].lp;
    g.lev[l].L = lv[l].stoc_len;
    g.lev[l].inner = (float)(q * q) / (float)lv[l].stoc_len;
  }
  if (!gemm_tc_levels_supported(g))
    return fail(SCMP_ERR_UNSUPPORTED, "sc_matmul_levels: needs an sm_100 device (SM pairs, e2m1 tables)");

  if (g_qprof_start) cudaEventRecord(g_qprof_start, st);
  // a's rows grouped by level
  SCMP_CUDA(launch_level_perm(row_level, d->n, nlev, p.n_pad, p.row_of, p.lev_tile0, st), "level permutation");

  // b, once per level (its boundaries depend on the level's grid)
  for (int l = 0; l < nlev; ++l) {
    QuantArgs qb = base_quant(d, false, q);
    qb.G = lv[l].rng_levels;
    qb.ratio = (float)lv[l].rng_levels / (float)q;
    qb.vcap = lv[l].vcap;
    qb.out16 = p.vb[l];
    if (p.chunked) {
      qb.chunk_d = d->chunk_d;
      qb.chunk_scale = p.scale_b;
      SCMP_CUDA(launch_quant_rows(Q_ROWCHUNK_BIP, qb, st), "levels: chunked quant b");
    } else {
      qb.row_scale = p.scale_b;
      qb.row_zp = p.zp_b;
      if (!bip) qb.row_sum = p.sum_b;
      if (d->group_b == 1 || d->m == 1) {
        qb.self_stats = 1;
      } else if (l == 0) {
        SCMP_CUDA(launch_row_stats(qb, p.stats_b, st), "levels: stats b");
        SCMP_CUDA(launch_group_params(p.stats_b, 1, d->m, d->group_b, q, bip ? GP_SYM : GP_ASYM, p.scale_b,
                                      bip ? nullptr : p.zp_b, st),
                  "levels: group params b");
      }
      SCMP_CUDA(launch_quant_rows(bip ? Q_GROUP_SYM : Q_GROUP_ASYM, qb, st), "levels: quant b");
    }
    SCMP_CUDA(launch_pad_map(lv[l].bmap, d->d, p.bmap[l], st), "levels: pad bmap");
  }

  // a, one pass over the permuted rows, each on its level's grid and tables
  QuantArgs qa = base_quant(d, true, q);
  qa.rows = qa.rows_per_batch = p.n_pad;
  qa.out16 = p.ka;
  qa.row_of = p.row_of;
  qa.lev_tile0 = p.lev_tile0;
  qa.nlev = nlev;
  for (int l = 0; l < nlev; ++l)
    qa.lq[l] = LevelQ{(float)lv[l].rng_levels / (float)q, lv[l].rng_levels, lv[l].vcap, lv[l].ktab, lv[l].amap};
  if (p.chunked) {
    qa.chunk_d = d->chunk_d;
    qa.chunk_scale = p.scale_a;
    SCMP_CUDA(launch_quant_rows(Q_ROWCHUNK_BIP, qa, st), "levels: chunked quant a");
    g.epi.kind = EPI_CHUNK;
  } else {
    qa.self_stats = 1;
    qa.row_scale = p.scale_a;
    qa.row_zp = p.zp_a;
    if (!bip) qa.row_sum = p.sum_a;
    SCMP_CUDA(launch_quant_rows(bip ? Q_GROUP_SYM : Q_GROUP_ASYM, qa, st), "levels: quant a");
    g.epi.kind = bip ? EPI_ROW : EPI_ROW_UNI;
    g.epi.zpa = p.zp_a;
    g.epi.zpb = p.zp_b;
    g.epi.asum = p.sum_a;
    g.epi.bsum = p.sum_b;
  }
  g.epi.sa = p.scale_a;
  g.epi.sb = p.scale_b;
  g.epi.inner = g.lev[0].inner;
  g.epi.fd = (float)d->d;
  if (g_qprof_stop) cudaEventRecord(g_qprof_stop, st);

  if (g_prof_start) cudaEventRecord(g_prof_start, st);
  const cudaError_t e = launch_gemm_tc_levels(g, st);
  if (g_prof_stop) cudaEventRecord(g_prof_stop, st);
  SCMP_CUDA(e, "levels: sc_gemm");
  return SCMP_OK;
}

}  // extern "C"
