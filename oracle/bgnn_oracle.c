/*
 * bgnn_oracle.c -- CPU restatement of BrowserGNN's message-passing path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product): the CUDA library
 * is compared against these functions in tests/, in __graft_entry__.smoke()
 * and in bench.py's CPU-baseline / reference arm.  Nothing in
 * browsergnn_b200/ links or loads this file.
 *
 * Each function cites the reference (TypeScript) function it restates.
 * Arithmetic model: JS locals are doubles; a store into a Float32Array rounds
 * once to float.  Every `(float)` cast below marks such a store; every other
 * intermediate is `double`.  Build flags: -O2 -ffp-contract=off (no FMA
 * contraction), no -ffast-math.
 *
 * Parity pinned by the reference's own known-answer tests (tests/wasm.test.ts,
 * tests/graph.test.ts), transcribed under tests/golden/.
 */
#include "bgnn_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int pick_threads(int threads) {
#ifdef _OPENMP
  return threads > 0 ? threads : omp_get_max_threads();
#else
  (void)threads;
  return 1;
#endif
}

/* wasmMatmul, src/backend/wasm/index.ts:18-63.  The reference tiles i/j/k by
 * 32, but for a fixed output (i,j) the k index still runs 0..k-1 in ascending
 * order (k0 tiles ascend inside each j0 tile), and each step is
 * result = f32(result + a*b) evaluated in double.  An i/k/j loop nest keeps
 * that per-output sequence, so it produces the same bits. */
void orc_matmul(const float* a, const float* b, int64_t m, int64_t k, int64_t n, float* out) {
  memset(out, 0, sizeof(float) * (size_t)(m * n));
  for (int64_t i = 0; i < m; i++) {
    float* orow = out + i * n;
    for (int64_t kk = 0; kk < k; kk++) {
      const double av = (double)a[i * k + kk];
      const float* brow = b + kk * n;
      for (int64_t j = 0; j < n; j++) orow[j] = (float)((double)orow[j] + av * (double)brow[j]);
    }
  }
}

void orc_matmul_par(const float* a, const float* b, int64_t m, int64_t k, int64_t n,
                    int threads, float* out) {
  const int nt = pick_threads(threads);
#pragma omp parallel for schedule(static) num_threads(nt)
  for (int64_t i = 0; i < m; i++) {
    float* orow = out + i * n;
    for (int64_t j = 0; j < n; j++) orow[j] = 0.0f;
    for (int64_t kk = 0; kk < k; kk++) {
      const double av = (double)a[i * k + kk];
      const float* brow = b + kk * n;
      for (int64_t j = 0; j < n; j++) orow[j] = (float)((double)orow[j] + av * (double)brow[j]);
    }
  }
}

/* wasmScatterAdd, src/backend/wasm/index.ts:70-105: edge order, one f32
 * rounding per add. */
void orc_scatter_add(const float* src, const uint32_t* index, int64_t num_msgs,
                     int64_t num_nodes, int64_t nf, float* out) {
  memset(out, 0, sizeof(float) * (size_t)(num_nodes * nf));
  for (int64_t e = 0; e < num_msgs; e++) {
    float* d = out + (int64_t)index[e] * nf;
    const float* s = src + e * nf;
    for (int64_t f = 0; f < nf; f++) d[f] = (float)((double)d[f] + (double)s[f]);
  }
}

/* wasmScatterMean, src/backend/wasm/index.ts:112-151: sum as above, u32
 * counts, then sum * (1/count) with 1/count held as a double. */
void orc_scatter_mean(const float* src, const uint32_t* index, int64_t num_msgs,
                      int64_t num_nodes, int64_t nf, float* out) {
  orc_scatter_add(src, index, num_msgs, num_nodes, nf, out);
  uint32_t* counts = (uint32_t*)calloc((size_t)num_nodes + 1, sizeof(uint32_t));
  for (int64_t e = 0; e < num_msgs; e++) counts[index[e]] += 1u;
  for (int64_t i = 0; i < num_nodes; i++) {
    if (counts[i] > 0) {
      const double inv = 1.0 / (double)counts[i];
      float* d = out + i * nf;
      for (int64_t f = 0; f < nf; f++) d[f] = (float)((double)d[f] * inv);
    }
  }
  free(counts);
}

/* wasmScatterMax, src/backend/wasm/index.ts:158-206: init -Infinity, replace
 * when strictly greater (NaN never wins, the first of +0/-0 stays), then every
 * remaining -Infinity becomes 0. */
void orc_scatter_max(const float* src, const uint32_t* index, int64_t num_msgs,
                     int64_t num_nodes, int64_t nf, float* out) {
  const int64_t total = num_nodes * nf;
  for (int64_t i = 0; i < total; i++) out[i] = -INFINITY;
  for (int64_t e = 0; e < num_msgs; e++) {
    float* d = out + (int64_t)index[e] * nf;
    const float* s = src + e * nf;
    for (int64_t f = 0; f < nf; f++)
      if (s[f] > d[f]) d[f] = s[f];
  }
  for (int64_t i = 0; i < total; i++)
    if (out[i] == -INFINITY) out[i] = 0.0f;
}

/* wasmGather, src/backend/wasm/index.ts:213-245. */
void orc_gather(const float* src, const uint32_t* index, int64_t num_idx, int64_t nf,
                float* out) {
  for (int64_t i = 0; i < num_idx; i++)
    memcpy(out + i * nf, src + (int64_t)index[i] * nf, sizeof(float) * (size_t)nf);
}

/* wasmRelu, src/backend/wasm/index.ts:250-271: x > 0 ? x : 0 (NaN -> 0). */
void orc_relu(const float* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = x[i] > 0.0f ? x[i] : 0.0f;
}

/* wasmAdd, src/backend/wasm/index.ts:276-297. */
void orc_add(const float* a, const float* b, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = (float)((double)a[i] + (double)b[i]);
}

/* wasmSpmv, src/backend/wasm/index.ts:304-335: double accumulator, one
 * rounding at the store. */
void orc_spmv(const uint32_t* row_ptr, const uint32_t* col, const float* val, const float* x,
              int64_t num_rows, float* out) {
  for (int64_t i = 0; i < num_rows; i++) {
    double sum = 0.0;
    for (uint32_t j = row_ptr[i]; j < row_ptr[i + 1]; j++)
      sum += (double)val[j] * (double)x[col[j]];
    out[i] = (float)sum;
  }
}

/* wasmSpmm, src/backend/wasm/index.ts:342-383: per row, CSR order,
 * result = f32(result + val*dense) in double. */
void orc_spmm(const uint32_t* row_ptr, const uint32_t* col, const float* val, const float* dense,
              int64_t num_rows, int64_t nf, float* out) {
  memset(out, 0, sizeof(float) * (size_t)(num_rows * nf));
  for (int64_t i = 0; i < num_rows; i++) {
    float* o = out + i * nf;
    for (uint32_t j = row_ptr[i]; j < row_ptr[i + 1]; j++) {
      const double v = (double)val[j];
      const float* d = dense + (int64_t)col[j] * nf;
      for (int64_t f = 0; f < nf; f++) o[f] = (float)((double)o[f] + v * (double)d[f]);
    }
  }
}

/* wasmSpmm (src/backend/wasm/index.ts:342-383) for a list of rows, row-parallel:
 * every row is computed exactly as in orc_spmm (CSR order, f32 store after
 * each double step), so the bits are the same.  rows NULL: rows 0..nrows-1.
 * out is [nrows, nf] in the order of the list. */
void orc_spmm_rows(const uint32_t* row_ptr, const uint32_t* col, const float* val,
                   const float* dense, int64_t nf, const uint32_t* rows, int64_t nrows,
                   int threads, float* out) {
  const int nt = pick_threads(threads);
#pragma omp parallel for schedule(dynamic, 64) num_threads(nt)
  for (int64_t q = 0; q < nrows; q++) {
    const int64_t i = rows ? (int64_t)rows[q] : q;
    float* o = out + q * nf;
    for (int64_t f = 0; f < nf; f++) o[f] = 0.0f;
    for (uint32_t j = row_ptr[i]; j < row_ptr[i + 1]; j++) {
      const double v = (double)val[j];
      const float* d = dense + (int64_t)col[j] * nf;
      for (int64_t f = 0; f < nf; f++) o[f] = (float)((double)o[f] + v * (double)d[f]);
    }
  }
}

/* SparseCOO.matmul, src/core/sparse.ts:138-159: COO (edge) order. */
void orc_coo_spmm(const uint32_t* rows, const uint32_t* cols, const float* vals, int64_t nnz,
                  int64_t m, const float* dense, int64_t k, float* out) {
  memset(out, 0, sizeof(float) * (size_t)(m * k));
  for (int64_t i = 0; i < nnz; i++) {
    float* o = out + (int64_t)rows[i] * k;
    const float* d = dense + (int64_t)cols[i] * k;
    const double v = (double)vals[i];
    for (int64_t j = 0; j < k; j++) o[j] = (float)((double)o[j] + v * (double)d[j]);
  }
}

/* SparseCSR.fromCOO, src/core/sparse.ts:259-296: a permutation sorted by
 * (row, col) with ties in original order (Array.prototype.sort is stable),
 * rowPtr[r] = first sorted position whose row >= r.  Restated as two stable
 * counting sorts (by col, then by row), which yields the same permutation. */
int orc_coo_to_csr(const uint32_t* rows, const uint32_t* cols, const float* vals, int64_t nnz,
                   int64_t num_rows, uint32_t* row_ptr, uint32_t* col_out, float* val_out) {
  uint32_t max_col = 0;
  for (int64_t i = 0; i < nnz; i++) {
    if ((int64_t)rows[i] >= num_rows) return -2;
    if (cols[i] > max_col) max_col = cols[i];
  }
  const int64_t ncols = (int64_t)max_col + 1;
  uint32_t* perm = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(nnz ? nnz : 1));
  uint32_t* perm2 = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(nnz ? nnz : 1));
  int64_t* cnt = (int64_t*)calloc((size_t)(ncols > num_rows ? ncols : num_rows) + 1, sizeof(int64_t));
  if (!perm || !perm2 || !cnt) {
    free(perm); free(perm2); free(cnt);
    return -1;
  }
  /* pass 1: stable by col */
  for (int64_t i = 0; i < nnz; i++) cnt[cols[i] + 1]++;
  for (int64_t c = 0; c < ncols; c++) cnt[c + 1] += cnt[c];
  for (int64_t i = 0; i < nnz; i++) perm[cnt[cols[i]]++] = (uint32_t)i;
  /* pass 2: stable by row */
  memset(cnt, 0, sizeof(int64_t) * (size_t)((ncols > num_rows ? ncols : num_rows) + 1));
  for (int64_t i = 0; i < nnz; i++) cnt[rows[i] + 1]++;
  for (int64_t r = 0; r < num_rows; r++) cnt[r + 1] += cnt[r];
  for (int64_t r = 0; r <= num_rows; r++) row_ptr[r] = (uint32_t)cnt[r];
  for (int64_t t = 0; t < nnz; t++) {
    const uint32_t i = perm[t];
    perm2[cnt[rows[i]]++] = i;
  }
  for (int64_t t = 0; t < nnz; t++) {
    col_out[t] = cols[perm2[t]];
    if (val_out) val_out[t] = vals ? vals[perm2[t]] : 1.0f;
  }
  free(perm); free(perm2); free(cnt);
  return 0;
}

/* GraphData constructor bounds check, src/core/graph.ts:88-92. */
int64_t orc_validate_edges(const uint32_t* ei, int64_t num_edges, int64_t num_nodes) {
  for (int64_t i = 0; i < 2 * num_edges; i++)
    if ((int64_t)ei[i] >= num_nodes) return i;
  return -1;
}

/* getInDegrees / getOutDegrees, src/core/graph.ts:172-195. */
void orc_in_degree(const uint32_t* ei, int64_t num_edges, int64_t num_nodes, uint32_t* out) {
  memset(out, 0, sizeof(uint32_t) * (size_t)num_nodes);
  for (int64_t i = 0; i < num_edges; i++) out[ei[num_edges + i]] += 1u;
}
void orc_out_degree(const uint32_t* ei, int64_t num_edges, int64_t num_nodes, uint32_t* out) {
  memset(out, 0, sizeof(uint32_t) * (size_t)num_nodes);
  for (int64_t i = 0; i < num_edges; i++) out[ei[i]] += 1u;
}

/* hasSelfLoops, src/core/graph.ts:220-227. */
int orc_has_self_loops(const uint32_t* ei, int64_t num_edges) {
  for (int64_t i = 0; i < num_edges; i++)
    if (ei[i] == ei[num_edges + i]) return 1;
  return 0;
}

/* addSelfLoops, src/core/graph.ts:232-272: original edges first, then a loop
 * (i,i) for every node without one, in node order. */
int64_t orc_add_self_loops(const uint32_t* ei, int64_t num_edges, int64_t num_nodes,
                           uint32_t* out) {
  unsigned char* has = (unsigned char*)calloc((size_t)num_nodes + 1, 1);
  int64_t have = 0;
  for (int64_t i = 0; i < num_edges; i++)
    if (ei[i] == ei[num_edges + i] && !has[ei[i]]) {
      has[ei[i]] = 1;
      have++;
    }
  const int64_t ne = num_edges + (num_nodes - have);
  memmove(out, ei, sizeof(uint32_t) * (size_t)num_edges);
  memcpy(out + ne, ei + num_edges, sizeof(uint32_t) * (size_t)num_edges);
  int64_t idx = num_edges;
  for (int64_t i = 0; i < num_nodes; i++)
    if (!has[i]) {
      out[idx] = (uint32_t)i;
      out[ne + idx] = (uint32_t)i;
      idx++;
    }
  free(has);
  return ne;
}

/* computeGCNNorm, src/core/sparse.ts:480-513: degree counted in a
 * Float32Array, dinv = f32(1/sqrt(deg)) in double, w = f32(dinv[s]*dinv[t]). */
static void gcn_dinv(const uint32_t* ei, int64_t num_edges, int64_t num_nodes, int add_loops,
                     float* dinv) {
  float* deg = (float*)malloc(sizeof(float) * (size_t)(num_nodes ? num_nodes : 1));
  for (int64_t i = 0; i < num_nodes; i++) deg[i] = add_loops ? 1.0f : 0.0f;
  for (int64_t i = 0; i < num_edges; i++) {
    const uint32_t t = ei[num_edges + i];
    deg[t] = (float)((double)deg[t] + 1.0);
  }
  for (int64_t i = 0; i < num_nodes; i++)
    dinv[i] = deg[i] > 0.0f ? (float)(1.0 / sqrt((double)deg[i])) : 0.0f;
  free(deg);
}

void orc_gcn_norm(const uint32_t* ei, int64_t num_edges, int64_t num_nodes, int add_self_loops,
                  float* out) {
  float* dinv = (float*)malloc(sizeof(float) * (size_t)(num_nodes ? num_nodes : 1));
  gcn_dinv(ei, num_edges, num_nodes, add_self_loops, dinv);
  for (int64_t i = 0; i < num_edges; i++)
    out[i] = (float)((double)dinv[ei[i]] * (double)dinv[ei[num_edges + i]]);
  free(dinv);
}

/* ELU, src/nn/activation.ts:56-65: x > 0 ? x : alpha*(exp(x)-1). */
void orc_elu(const float* x, int64_t n, double alpha, float* out) {
  for (int64_t i = 0; i < n; i++) {
    const double v = (double)x[i];
    out[i] = v > 0.0 ? (float)v : (float)(alpha * (exp(v) - 1.0));
  }
}

/* Tensor.leakyRelu, src/core/tensor.ts:401-408. */
void orc_leaky_relu(const float* x, int64_t n, double slope, float* out) {
  for (int64_t i = 0; i < n; i++) {
    const double v = (double)x[i];
    out[i] = v > 0.0 ? (float)v : (float)(slope * v);
  }
}

/* JS Math.max(0, v) as used by GINConv.relu (src/layers/gin.ts:106-112):
 * NaN propagates, -0 becomes +0. */
static inline double js_max0(double v) {
  if (v != v) return v;
  return v > 0.0 ? v : 0.0;
}
void orc_relu_max(const float* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = (float)js_max0((double)x[i]);
}

static uint32_t* maybe_self_loops(const uint32_t* ei, int64_t e, int64_t n, int add_cfg,
                                  int64_t* e_out) {
  uint32_t* buf = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(2 * (e + n) + 2));
  if (!buf) return NULL;
  if (add_cfg && !orc_has_self_loops(ei, e)) {
    *e_out = orc_add_self_loops(ei, e, n, buf);
  } else {
    memcpy(buf, ei, sizeof(uint32_t) * (size_t)(2 * e));
    *e_out = e;
  }
  return buf;
}

/* GCNConv.forward, src/layers/gcn.ts:78-160. */
int orc_gcn_forward(const float* x, int64_t n, int64_t fin, const uint32_t* ei, int64_t e,
                    const float* weight, const float* bias, int64_t fout, int add_self_loops,
                    int normalize, float* out) {
  int64_t ep;
  uint32_t* pe = maybe_self_loops(ei, e, n, add_self_loops, &ep);
  float* h = (float*)malloc(sizeof(float) * (size_t)(n * fout + 1));
  float* msg = (float*)malloc(sizeof(float) * (size_t)(ep * fout + 1));
  float* norm = (float*)malloc(sizeof(float) * (size_t)(ep + 1));
  if (!pe || !h || !msg || !norm) {
    free(pe); free(h); free(msg); free(norm);
    return -1;
  }
  orc_matmul(x, weight, n, fin, fout, h);
  orc_gather(h, pe, ep, fout, msg);
  if (normalize) {
    orc_gcn_norm(pe, ep, n, 0, norm);
    for (int64_t i = 0; i < ep; i++)
      for (int64_t f = 0; f < fout; f++)
        msg[i * fout + f] = (float)((double)msg[i * fout + f] * (double)norm[i]);
  }
  orc_scatter_add(msg, pe + ep, ep, n, fout, out);
  if (bias)
    for (int64_t i = 0; i < n; i++)
      for (int64_t f = 0; f < fout; f++)
        out[i * fout + f] = (float)((double)out[i * fout + f] + (double)bias[f]);
  free(pe); free(h); free(msg); free(norm);
  return 0;
}

/* GATConv.forward, src/layers/gat.ts:107-258 (dropout off: inference). */
int orc_gat_forward(const float* x, int64_t n, int64_t fin, const uint32_t* ei, int64_t e,
                    const float* weight, const float* att_src, const float* att_dst,
                    const float* bias, int64_t heads, int64_t c, double slope, int concat,
                    int add_self_loops, float* out) {
  return orc_gat_forward_train(x, n, fin, ei, e, weight, att_src, att_dst, bias, heads, c, slope,
                               concat, add_self_loops, 0.0, 0, out);
}

/* GATConv.forward in training mode: the attention dropout of gat.ts:194-203
 * applied to alphaExp in index order, Math.random() replaced by the
 * counter-based draw orc_uniform(seed, i). */
int orc_gat_forward_train(const float* x, int64_t n, int64_t fin, const uint32_t* ei, int64_t e,
                          const float* weight, const float* att_src, const float* att_dst,
                          const float* bias, int64_t heads, int64_t c, double slope, int concat,
                          int add_self_loops, double drop_p, uint64_t seed, float* out) {
  int64_t ep;
  uint32_t* pe = maybe_self_loops(ei, e, n, add_self_loops, &ep);
  const int64_t hc = heads * c;
  float* h = (float*)malloc(sizeof(float) * (size_t)(n * hc + 1));
  float* alpha = (float*)malloc(sizeof(float) * (size_t)(ep * heads + 1));
  float* aexp = (float*)malloc(sizeof(float) * (size_t)(ep * heads + 1));
  float* asum = (float*)calloc((size_t)(n * heads + 1), sizeof(float));
  if (!pe || !h || !alpha || !aexp || !asum) {
    free(pe); free(h); free(alpha); free(aexp); free(asum);
    return -1;
  }
  const uint32_t* src = pe;
  const uint32_t* dst = pe + ep;
  orc_matmul(x, weight, n, fin, hc, h);
  /* scores, :138-164 */
  for (int64_t i = 0; i < ep; i++) {
    const int64_t s = src[i], t = dst[i];
    for (int64_t hh = 0; hh < heads; hh++) {
      double score = 0.0;
      for (int64_t f = 0; f < c; f++) {
        const double hs = (double)h[s * hc + hh * c + f];
        const double hd = (double)h[t * hc + hh * c + f];
        score += (double)att_src[hh * c + f] * hs + (double)att_dst[hh * c + f] * hd;
      }
      if (score < 0) score *= slope;
      alpha[i * heads + hh] = (float)score;
    }
  }
  /* exp(score - 10) and per-destination sum, :172-180 */
  for (int64_t i = 0; i < ep; i++) {
    const int64_t t = dst[i];
    for (int64_t hh = 0; hh < heads; hh++) {
      const double ev = exp((double)alpha[i * heads + hh] - 10.0);
      aexp[i * heads + hh] = (float)ev;
      asum[t * heads + hh] = (float)((double)asum[t * heads + hh] + ev);
    }
  }
  /* normalise, :183-192 */
  for (int64_t i = 0; i < ep; i++) {
    const int64_t t = dst[i];
    for (int64_t hh = 0; hh < heads; hh++) {
      const float sm = asum[t * heads + hh];
      if (sm > 0.0f)
        aexp[i * heads + hh] = (float)((double)aexp[i * heads + hh] / (double)sm);
    }
  }
  if (drop_p > 0.0)
    for (int64_t i = 0; i < ep * heads; i++)
      aexp[i] = orc_uniform(seed, (uint64_t)i) < drop_p
                    ? 0.0f
                    : (float)((double)aexp[i] / (1.0 - drop_p));
  /* weighted aggregation, :209-243 */
  const int64_t od = concat ? hc : c;
  memset(out, 0, sizeof(float) * (size_t)(n * od));
  for (int64_t i = 0; i < ep; i++) {
    const int64_t s = src[i], t = dst[i];
    for (int64_t hh = 0; hh < heads; hh++) {
      const double at = (double)aexp[i * heads + hh];
      for (int64_t f = 0; f < c; f++) {
        const double sv = (double)h[s * hc + hh * c + f];
        if (concat) {
          float* o = &out[t * od + hh * c + f];
          *o = (float)((double)*o + at * sv);
        } else {
          float* o = &out[t * od + f];
          *o = (float)((double)*o + at * sv / (double)heads);
        }
      }
    }
  }
  if (bias)
    for (int64_t i = 0; i < n; i++)
      for (int64_t f = 0; f < od; f++)
        out[i * od + f] = (float)((double)out[i * od + f] + (double)bias[f]);
  free(pe); free(h); free(alpha); free(aexp); free(asum);
  return 0;
}

/* SAGEConv.forward, src/layers/sage.ts:113-217. */
int orc_sage_forward(const float* x, int64_t n, int64_t fin, const uint32_t* ei, int64_t e,
                     int aggr, const float* lin_neighbor, const float* lin_self,
                     const float* bias, const float* pool_weight, const float* pool_bias,
                     int64_t fout, int normalize, float* out) {
  float* g = (float*)malloc(sizeof(float) * (size_t)(e * fin + 1));
  float* agg = (float*)malloc(sizeof(float) * (size_t)(n * fin + 1));
  float* nt = (float*)malloc(sizeof(float) * (size_t)(n * fout + 1));
  float* st = (float*)malloc(sizeof(float) * (size_t)(n * fout + 1));
  if (!g || !agg || !nt || !st) {
    free(g); free(agg); free(nt); free(st);
    return -1;
  }
  const uint32_t* dst = ei + e;
  orc_gather(x, ei, e, fin, g);
  if (aggr == 0) {
    orc_scatter_mean(g, dst, e, n, fin, agg);
  } else if (aggr == 1) {
    orc_scatter_max(g, dst, e, n, fin, agg);
  } else if (aggr == 2) {
    orc_scatter_add(g, dst, e, n, fin, agg);
  } else {
    /* pool: relu(src @ pool_weight + pool_bias) in a double accumulator,
     * :149-163, then scatterMax */
    float* proj = (float*)malloc(sizeof(float) * (size_t)(e * fin + 1));
    if (!proj) {
      free(g); free(agg); free(nt); free(st);
      return -1;
    }
    for (int64_t i = 0; i < e; i++)
      for (int64_t j = 0; j < fin; j++) {
        double sum = (double)pool_bias[j];
        for (int64_t k = 0; k < fin; k++)
          sum += (double)g[i * fin + k] * (double)pool_weight[k * fin + j];
        proj[i * fin + j] = (float)js_max0(sum);
      }
    orc_scatter_max(proj, dst, e, n, fin, agg);
    free(proj);
  }
  orc_matmul(agg, lin_neighbor, n, fin, fout, nt);
  if (lin_self) {
    orc_matmul(x, lin_self, n, fin, fout, st);
    orc_add(st, nt, n * fout, out);
  } else {
    memcpy(out, nt, sizeof(float) * (size_t)(n * fout));
  }
  if (bias)
    for (int64_t i = 0; i < n; i++)
      for (int64_t f = 0; f < fout; f++)
        out[i * fout + f] = (float)((double)out[i * fout + f] + (double)bias[f]);
  if (normalize) {
    for (int64_t i = 0; i < n; i++) {
      double nrm = 0.0;
      for (int64_t f = 0; f < fout; f++) {
        const double v = (double)out[i * fout + f];
        nrm += v * v;
      }
      nrm = sqrt(nrm);
      if (nrm > 0)
        for (int64_t f = 0; f < fout; f++)
          out[i * fout + f] = (float)((double)out[i * fout + f] / nrm);
    }
  }
  free(g); free(agg); free(nt); free(st);
  return 0;
}

/* GINConv.forward, src/layers/gin.ts:120-192. */
int orc_gin_forward(const float* x, int64_t n, int64_t fin, const uint32_t* ei, int64_t e,
                    float eps, const float* w1, const float* b1, int64_t hidden,
                    const float* w2, const float* b2, int64_t fout, float* out) {
  float* g = (float*)malloc(sizeof(float) * (size_t)(e * fin + 1));
  float* agg = (float*)malloc(sizeof(float) * (size_t)(n * fin + 1));
  float* comb = (float*)malloc(sizeof(float) * (size_t)(n * fin + 1));
  float* hid = (float*)malloc(sizeof(float) * (size_t)(n * hidden + 1));
  if (!g || !agg || !comb || !hid) {
    free(g); free(agg); free(comb); free(hid);
    return -1;
  }
  orc_gather(x, ei, e, fin, g);
  orc_scatter_add(g, ei + e, e, n, fin, agg);
  const double ope = 1.0 + (double)eps;
  for (int64_t i = 0; i < n * fin; i++) comb[i] = (float)(ope * (double)x[i] + (double)agg[i]);
  orc_matmul(comb, w1, n, fin, hidden, hid);
  if (b1)
    for (int64_t i = 0; i < n; i++)
      for (int64_t f = 0; f < hidden; f++)
        hid[i * hidden + f] = (float)((double)hid[i * hidden + f] + (double)b1[f]);
  orc_relu_max(hid, n * hidden, hid);
  orc_matmul(hid, w2, n, hidden, fout, out);
  if (b2)
    for (int64_t i = 0; i < n; i++)
      for (int64_t f = 0; f < fout; f++)
        out[i * fout + f] = (float)((double)out[i * fout + f] + (double)b2[f]);
  free(g); free(agg); free(comb); free(hid);
  return 0;
}

/* Global sum pool (no counterpart in the reference: it has no readout op);
 * defined here as f32 adds in node order. */
void orc_sum_pool(const float* x, int64_t n, int64_t f, const uint32_t* batch,
                  int64_t num_graphs, float* out) {
  memset(out, 0, sizeof(float) * (size_t)(num_graphs * f));
  for (int64_t i = 0; i < n; i++) {
    float* o = out + (int64_t)batch[i] * f;
    for (int64_t j = 0; j < f; j++) o[j] = (float)((double)o[j] + (double)x[i * f + j]);
  }
}

/* ---- streamed, row-parallel restatement ---------------------------------
 * Each destination row visits its incoming edges in COO order, which is the
 * order in which the reference's edge-ordered scatters touch that row, so the
 * per-element rounding sequence (and the bits) are the same as above. */
int orc_dst_csr(const uint32_t* ei, int64_t e, int64_t n, uint32_t* row_ptr, uint32_t* src_of,
                uint32_t* eid) {
  int64_t* cur = (int64_t*)calloc((size_t)n + 1, sizeof(int64_t));
  if (!cur) return -1;
  for (int64_t i = 0; i < e; i++) cur[ei[e + i] + 1]++;
  for (int64_t r = 0; r < n; r++) cur[r + 1] += cur[r];
  for (int64_t r = 0; r <= n; r++) row_ptr[r] = (uint32_t)cur[r];
  for (int64_t i = 0; i < e; i++) {
    const int64_t p = cur[ei[e + i]]++;
    src_of[p] = ei[i];
    if (eid) eid[p] = (uint32_t)i;
  }
  free(cur);
  return 0;
}

static void row_aggregate(const uint32_t* row_ptr, const uint32_t* src_of, int64_t r,
                          const float* x, int64_t f, int op, int tail, const float* dinv,
                          float* o) {
  const uint32_t b = row_ptr[r], en = row_ptr[r + 1];
  const int64_t cnt = (int64_t)(en - b) + (tail ? 1 : 0);
  if (op == 2) {
    for (int64_t j = 0; j < f; j++) o[j] = -INFINITY;
  } else {
    for (int64_t j = 0; j < f; j++) o[j] = 0.0f;
  }
  for (int64_t q = 0; q < cnt; q++) {
    const int64_t s = (q < (int64_t)(en - b)) ? (int64_t)src_of[b + q] : r;
    const float* xs = x + s * f;
    if (op == 2) {
      for (int64_t j = 0; j < f; j++)
        if (xs[j] > o[j]) o[j] = xs[j];
    } else if (op == 3) {
      const double w = (double)(float)((double)dinv[s] * (double)dinv[r]);
      for (int64_t j = 0; j < f; j++) {
        const float m = (float)((double)xs[j] * w);
        o[j] = (float)((double)o[j] + (double)m);
      }
    } else {
      for (int64_t j = 0; j < f; j++) o[j] = (float)((double)o[j] + (double)xs[j]);
    }
  }
  if (op == 1 && cnt > 0) {
    const double inv = 1.0 / (double)cnt;
    for (int64_t j = 0; j < f; j++) o[j] = (float)((double)o[j] * inv);
  }
  if (op == 2)
    for (int64_t j = 0; j < f; j++)
      if (o[j] == -INFINITY) o[j] = 0.0f;
}

void orc_csr_aggregate(const uint32_t* row_ptr, const uint32_t* src_of, int64_t num_rows,
                       const float* x, int64_t f, int op, int tail, int threads, float* out) {
  float* dinv = NULL;
  if (op == 3) {
    dinv = (float*)malloc(sizeof(float) * (size_t)(num_rows ? num_rows : 1));
    for (int64_t r = 0; r < num_rows; r++) {
      const uint32_t d = row_ptr[r + 1] - row_ptr[r] + (tail ? 1u : 0u);
      /* f32 counting saturates at 2^24, as the Float32Array degree does */
      const float deg = d >= 16777216u ? 16777216.0f : (float)d;
      dinv[r] = deg > 0.0f ? (float)(1.0 / sqrt((double)deg)) : 0.0f;
    }
  }
  const int nt = pick_threads(threads);
#pragma omp parallel for schedule(dynamic, 256) num_threads(nt)
  for (int64_t r = 0; r < num_rows; r++)
    row_aggregate(row_ptr, src_of, r, x, f, op, tail, dinv, out + r * f);
  free(dinv);
}

int orc_sage_forward_csr(const uint32_t* row_ptr, const uint32_t* src_of, int64_t n,
                         const float* x, int64_t fin, int aggr, const float* lin_neighbor,
                         const float* lin_self, const float* bias, int64_t fout, int relu,
                         int threads, float* out) {
  float* agg = (float*)malloc(sizeof(float) * (size_t)(n * fin + 1));
  float* nt = (float*)malloc(sizeof(float) * (size_t)(n * fout + 1));
  if (!agg || !nt) {
    free(agg); free(nt);
    return -1;
  }
  const int op = aggr == 0 ? 1 : (aggr == 1 ? 2 : 0);
  orc_csr_aggregate(row_ptr, src_of, n, x, fin, op, 0, threads, agg);
  orc_matmul_par(agg, lin_neighbor, n, fin, fout, threads, nt);
  if (lin_self) {
    orc_matmul_par(x, lin_self, n, fin, fout, threads, out);
    const int ntd = pick_threads(threads);
#pragma omp parallel for schedule(static) num_threads(ntd)
    for (int64_t i = 0; i < n * fout; i++) out[i] = (float)((double)out[i] + (double)nt[i]);
  } else {
    memcpy(out, nt, sizeof(float) * (size_t)(n * fout));
  }
  const int ntd = pick_threads(threads);
#pragma omp parallel for schedule(static) num_threads(ntd)
  for (int64_t i = 0; i < n; i++)
    for (int64_t f = 0; f < fout; f++) {
      float v = out[i * fout + f];
      if (bias) v = (float)((double)v + (double)bias[f]);
      if (relu) v = v > 0.0f ? v : 0.0f;
      out[i * fout + f] = v;
    }
  free(agg); free(nt);
  return 0;
}

/* ---- backward of the message passing and of X*W ------------------------
 * The reference's autograd (src/autograd/variable.ts) has a matmul backward
 * (variable.ts:213-235: gradA = grad @ B^T, gradB = A^T @ grad through
 * Tensor.transpose and wasmMatmul) and a broadcast bias reduction
 * (variable.ts:665-688), but never differentiates through MessagePassing.
 * The message-passing adjoint below is what it would compute if its
 * gather / scatter were autograd ops: edge e carries a message m_e derived
 * from grad[dst(e)], and the messages are scatter-added over the sources in
 * COO edge order (wasmScatterAdd, src/backend/wasm/index.ts:70-105):
 *   op 0 sum   m_e = grad[dst]
 *   op 1 mean  m_e = f32(grad[dst] * (1 / cnt(dst))), 1/cnt in double
 *   op 2 max   m_e = grad[dst] where src(e) supplied the forward maximum of
 *              that feature (the edge that last raised it: x > acc in COO
 *              order from -inf), else 0
 *   op 3 gcn   m_e = f32(grad[dst] * w_e), w_e the computeGCNNorm weight;
 *              tail != 0 appends the self-loop edges (i, i) after the edges
 * out [n, f] (zeros first). */
void orc_aggregate_backward(const uint32_t* ei, int64_t e, int64_t n, const float* x,
                            const float* grad, int64_t f, int op, int tail, float* out) {
  const uint32_t* src = ei;
  const uint32_t* dst = ei + e;
  for (int64_t i = 0; i < n * f; i++) out[i] = 0.0f;
  int64_t* arg = NULL;
  uint32_t* cnt = NULL;
  float* dinv = NULL;
  if (op == 2) {
    float* acc = (float*)malloc(sizeof(float) * (size_t)(n * f + 1));
    arg = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n * f + 1));
    for (int64_t i = 0; i < n * f; i++) {
      acc[i] = -INFINITY;
      arg[i] = -1;
    }
    for (int64_t q = 0; q < e; q++) {
      const float* xs = x + (int64_t)src[q] * f;
      float* a = acc + (int64_t)dst[q] * f;
      int64_t* g = arg + (int64_t)dst[q] * f;
      for (int64_t j = 0; j < f; j++)
        if (xs[j] > a[j]) {
          a[j] = xs[j];
          g[j] = q;
        }
    }
    free(acc);
  } else if (op == 1) {
    cnt = (uint32_t*)calloc((size_t)n + 1, sizeof(uint32_t));
    for (int64_t q = 0; q < e; q++) cnt[dst[q]]++;
  } else if (op == 3) {
    dinv = (float*)malloc(sizeof(float) * (size_t)(n + 1));
    gcn_dinv(ei, e, n, tail, dinv);
  }
  const int64_t total = e + ((op == 3 && tail) ? n : 0);
  for (int64_t q = 0; q < total; q++) {
    const int64_t s = q < e ? (int64_t)src[q] : q - e;
    const int64_t d = q < e ? (int64_t)dst[q] : q - e;
    const float* gd = grad + d * f;
    float* o = out + s * f;
    if (op == 0) {
      for (int64_t j = 0; j < f; j++) o[j] = (float)((double)o[j] + (double)gd[j]);
    } else if (op == 1) {
      const double inv = 1.0 / (double)cnt[d];
      for (int64_t j = 0; j < f; j++) {
        const float m = (float)((double)gd[j] * inv);
        o[j] = (float)((double)o[j] + (double)m);
      }
    } else if (op == 2) {
      const int64_t* g = arg + d * f;
      for (int64_t j = 0; j < f; j++) {
        const float m = g[j] == q ? gd[j] : 0.0f;
        o[j] = (float)((double)o[j] + (double)m);
      }
    } else {
      const double w = (double)(float)((double)dinv[s] * (double)dinv[d]);
      for (int64_t j = 0; j < f; j++) {
        const float m = (float)((double)gd[j] * w);
        o[j] = (float)((double)o[j] + (double)m);
      }
    }
  }
  free(arg);
  free(cnt);
  free(dinv);
}

/* Tensor.transpose, src/core/tensor.ts:131-144 */
static float* transpose_new(const float* a, int64_t rows, int64_t cols) {
  float* t = (float*)malloc(sizeof(float) * (size_t)(rows * cols + 1));
  for (int64_t i = 0; i < rows; i++)
    for (int64_t j = 0; j < cols; j++) t[j * rows + i] = a[i * cols + j];
  return t;
}

/* Variable.matmul backward, src/autograd/variable.ts:213-235:
 * grad_a [m, k] = grad [m, n] @ transpose(b); grad_b [k, n] = transpose(a) @ grad.
 * Either output may be NULL. */
void orc_matmul_backward(const float* a, const float* b, const float* grad, int64_t m, int64_t k,
                         int64_t n, float* grad_a, float* grad_b) {
  if (grad_a) {
    float* bt = transpose_new(b, k, n);
    orc_matmul(grad, bt, m, n, k, grad_a);
    free(bt);
  }
  if (grad_b) {
    float* at = transpose_new(a, m, k);
    orc_matmul(at, grad, k, m, n, grad_b);
    free(at);
  }
}

/* The bias gradient of a broadcast add, Variable._reduceBroadcast
 * (src/autograd/variable.ts:675-685): out[j] = sum over rows, in row order,
 * stored to a Float32Array after every step. */
void orc_bias_backward(const float* grad, int64_t rows, int64_t cols, float* out) {
  for (int64_t j = 0; j < cols; j++) out[j] = 0.0f;
  for (int64_t i = 0; i < rows; i++)
    for (int64_t j = 0; j < cols; j++) out[j] = (float)((double)out[j] + (double)grad[i * cols + j]);
}

/* ======================================================================= */
/* model zoo                                                               */
/* ======================================================================= */

/* Linear.forward, src/nn/linear.ts:50-111 (the 2-D branch; the 1-D branch is
 * the same sum for one row): `let sum = 0; sum += x*w` in double, stored to a
 * Float32Array, then the bias loop adds b[j] in double and stores again. */
void orc_linear(const float* x, int64_t m, int64_t k, const float* w, const float* b, int64_t n,
                float* out) {
  for (int64_t r = 0; r < m; r++) {
    for (int64_t j = 0; j < n; j++) {
      double sum = 0.0;
      for (int64_t i = 0; i < k; i++) sum += (double)x[r * k + i] * (double)w[j * k + i];
      float y = (float)sum;
      if (b) y = (float)((double)y + (double)b[j]);
      out[r * n + j] = y;
    }
  }
}

/* Tensor.sigmoid, src/core/tensor.ts:413-419: 1 / (1 + Math.exp(-x)). */
void orc_sigmoid(const float* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = (float)(1.0 / (1.0 + exp(-(double)x[i])));
}

/* Tensor.tanh, src/core/tensor.ts:424-430. */
void orc_tanh(const float* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = (float)tanh((double)x[i]);
}

/* GELU (tanh form), src/nn/activation.ts:129-147, left-to-right in double. */
void orc_gelu(const float* x, int64_t n, float* out) {
  const double s2p = sqrt(2.0 / 3.141592653589793);
  for (int64_t i = 0; i < n; i++) {
    const double v = (double)x[i];
    const double inner = s2p * (v + 0.044715 * v * v * v);
    out[i] = (float)(0.5 * v * (1.0 + tanh(inner)));
  }
}

/* SiLU, src/nn/activation.ts:153-168: x / (1 + Math.exp(-x)). */
void orc_silu(const float* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) {
    const double v = (double)x[i];
    out[i] = (float)(v / (1.0 + exp(-v)));
  }
}

/* PReLU, src/nn/activation.ts:175-200: one slope, or slope i % numParams. */
void orc_prelu(const float* x, int64_t n, const float* w, int64_t nw, float* out) {
  for (int64_t i = 0; i < n; i++) {
    const double v = (double)x[i];
    const double a = (double)(nw == 1 ? w[0] : w[i % nw]);
    out[i] = v > 0.0 ? (float)v : (float)(a * v);
  }
}

/* Math.max: NaN if either is NaN; +0 beats -0. */
static inline double js_max(double a, double b) {
  if (a != a || b != b) return NAN;
  if (a == 0.0 && b == 0.0) return signbit(a) ? b : a;
  return a > b ? a : b;
}

/* Tensor.softmax / logSoftmax, src/core/tensor.ts:435-499.  softmax stores
 * f32(exp) first and divides the stored value by the double sum of the
 * unrounded exps; logSoftmax subtracts max + log(sum) from x. */
void orc_softmax_rows(const float* x, int64_t rows, int64_t cols, const uint8_t* col_mask,
                      float mask_value, int log_softmax, float* out) {
  for (int64_t r = 0; r < rows; r++) {
    const float* xr = x + r * cols;
    float* o = out + r * cols;
#define XV(c) ((col_mask && col_mask[c]) ? (double)mask_value : (double)xr[c])
    double mx = -INFINITY;
    for (int64_t c = 0; c < cols; c++) mx = js_max(mx, XV(c));
    double sum = 0.0;
    if (log_softmax) {
      for (int64_t c = 0; c < cols; c++) sum += exp(XV(c) - mx);
      const double lse = mx + log(sum);
      for (int64_t c = 0; c < cols; c++) o[c] = (float)(XV(c) - lse);
    } else {
      for (int64_t c = 0; c < cols; c++) {
        const double e = exp(XV(c) - mx);
        o[c] = (float)e;
        sum += e;
      }
      for (int64_t c = 0; c < cols; c++) o[c] = (float)((double)o[c] / sum);
    }
#undef XV
  }
}

double orc_uniform(uint64_t seed, uint64_t i) {
  uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (double)(z >> 11) * (1.0 / 9007199254740992.0);
}

void orc_dropout(const float* x, int64_t n, double p, uint64_t seed, float* out) {
  const double scale = 1.0 / (1.0 - p);
  for (int64_t i = 0; i < n; i++)
    out[i] = orc_uniform(seed, (uint64_t)i) > p ? (float)((double)x[i] * scale) : 0.0f;
}

/* ConceptPrerequisiteMapper.predictLinks, ConceptPrerequisiteMapper.ts:224-295.
 * The embeddings are copied into Float32Arrays (no rounding); dot and
 * bilinear sums are JS doubles, the bilinear W*tgt vector is stored to a
 * Float32Array, the mlp input holds f32(src*tgt) in its last third. */
void orc_link_scores(const float* emb, int64_t d, const uint32_t* src, const uint32_t* tgt,
                     int64_t num_pairs, int mode, const float* w_bilinear, const float* w1,
                     const float* b1, const float* w2, const float* b2, double* out) {
  float* tmp = (float*)malloc(sizeof(float) * (size_t)(4 * d + 1));
  for (int64_t q = 0; q < num_pairs; q++) {
    const float* s = emb + (int64_t)src[q] * d;
    const float* t = emb + (int64_t)tgt[q] * d;
    double score = 0.0;
    if (mode == 0) {
      for (int64_t i = 0; i < d; i++) score += (double)s[i] * (double)t[i];
    } else if (mode == 1) {
      for (int64_t i = 0; i < d; i++) {
        double sum = 0.0;
        for (int64_t j = 0; j < d; j++) sum += (double)w_bilinear[i * d + j] * (double)t[j];
        tmp[i] = (float)sum;
      }
      for (int64_t i = 0; i < d; i++) score += (double)s[i] * (double)tmp[i];
    } else {
      float* in = tmp;          /* [3d] */
      float* hid = tmp + 3 * d; /* [d]  */
      for (int64_t i = 0; i < d; i++) {
        in[i] = s[i];
        in[d + i] = t[i];
        in[2 * d + i] = (float)((double)s[i] * (double)t[i]);
      }
      orc_linear(in, 1, 3 * d, w1, b1, d, hid);
      orc_relu(hid, d, hid);
      float o;
      orc_linear(hid, 1, d, w2, b2, 1, &o);
      score = (double)o;
    }
    out[q] = 1.0 / (1.0 + exp(-score));
  }
  free(tmp);
}
