/*
 * bgnn_oracle.h -- CPU restatement of BrowserGNN's message-passing path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the oracle that the CUDA library is
 * checked against; nothing in the product library links, loads or calls it.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
 * arm may use it.
 *
 * Arithmetic model (the reference is TypeScript): every JS local is an IEEE
 * double, every store into a Float32Array rounds once to float.  The
 * restatement keeps every local as `double` and casts to `float` exactly
 * where the reference stores into a Float32Array.  Compile with
 * -ffp-contract=off and without -ffast-math so no FMA contraction or
 * reassociation changes the rounding sequence.
 *
 * Parity pins: the reference's own known-answer tests (tests/wasm.test.ts,
 * tests/graph.test.ts) are transcribed as fixtures under tests/golden/ and
 * checked against these functions.
 */
#ifndef BGNN_ORACLE_H
#define BGNN_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- src/backend/wasm/index.ts kernels ---------------------------------- */
void orc_matmul(const float* a, const float* b, int64_t m, int64_t k, int64_t n, float* out);
void orc_scatter_add(const float* src, const uint32_t* index, int64_t num_msgs,
                     int64_t num_nodes, int64_t num_features, float* out);
void orc_scatter_mean(const float* src, const uint32_t* index, int64_t num_msgs,
                      int64_t num_nodes, int64_t num_features, float* out);
void orc_scatter_max(const float* src, const uint32_t* index, int64_t num_msgs,
                     int64_t num_nodes, int64_t num_features, float* out);
void orc_gather(const float* src, const uint32_t* index, int64_t num_idx,
                int64_t num_features, float* out);
void orc_relu(const float* x, int64_t n, float* out);
void orc_add(const float* a, const float* b, int64_t n, float* out);
void orc_spmv(const uint32_t* row_ptr, const uint32_t* col, const float* val,
              const float* x, int64_t num_rows, float* out);
void orc_spmm(const uint32_t* row_ptr, const uint32_t* col, const float* val,
              const float* dense, int64_t num_rows, int64_t num_features, float* out);

/* ---- src/core/sparse.ts ------------------------------------------------- */
void orc_coo_spmm(const uint32_t* rows, const uint32_t* cols, const float* vals,
                  int64_t nnz, int64_t m, const float* dense, int64_t k, float* out);
/* SparseCSR.fromCOO: stable sort by (row, col); returns 0 or -1 on OOM. */
int orc_coo_to_csr(const uint32_t* rows, const uint32_t* cols, const float* vals,
                   int64_t nnz, int64_t num_rows, uint32_t* row_ptr,
                   uint32_t* col_out, float* val_out);
void orc_gcn_norm(const uint32_t* edge_index, int64_t num_edges, int64_t num_nodes,
                  int add_self_loops, float* out);

/* ---- src/core/graph.ts -------------------------------------------------- */
/* returns -1 if valid, else the position of the first out-of-range index */
int64_t orc_validate_edges(const uint32_t* edge_index, int64_t num_edges, int64_t num_nodes);
void orc_in_degree(const uint32_t* edge_index, int64_t num_edges, int64_t num_nodes, uint32_t* out);
void orc_out_degree(const uint32_t* edge_index, int64_t num_edges, int64_t num_nodes, uint32_t* out);
int orc_has_self_loops(const uint32_t* edge_index, int64_t num_edges);
/* out has room for 2*(num_edges+num_nodes); returns the new edge count */
int64_t orc_add_self_loops(const uint32_t* edge_index, int64_t num_edges, int64_t num_nodes,
                           uint32_t* out);

/* ---- activations (src/core/tensor.ts, src/nn/activation.ts, gin.ts) ---- */
void orc_elu(const float* x, int64_t n, double alpha, float* out);
void orc_leaky_relu(const float* x, int64_t n, double slope, float* out);
void orc_relu_max(const float* x, int64_t n, float* out); /* Math.max(0, x) */

/* ---- layer forwards (src/layers/{gcn,gat,sage,gin}.ts), reference data layout ----------- */
/* weight [fin, fout]; bias may be NULL.  add_self_loops / normalize follow
 * GCNConvConfig.  out [N, fout]. */
int orc_gcn_forward(const float* x, int64_t n, int64_t fin, const uint32_t* edge_index,
                    int64_t num_edges, const float* weight, const float* bias, int64_t fout,
                    int add_self_loops, int normalize, float* out);
/* weight [fin, heads*c]; att_src/att_dst [heads, c]; bias [heads*c or c] or NULL */
int orc_gat_forward(const float* x, int64_t n, int64_t fin, const uint32_t* edge_index,
                    int64_t num_edges, const float* weight, const float* att_src,
                    const float* att_dst, const float* bias, int64_t heads, int64_t c,
                    double negative_slope, int concat, int add_self_loops, float* out);
/* training mode: attention dropout p with the counter-based draw (seed) */
int orc_gat_forward_train(const float* x, int64_t n, int64_t fin, const uint32_t* edge_index,
                          int64_t num_edges, const float* weight, const float* att_src,
                          const float* att_dst, const float* bias, int64_t heads, int64_t c,
                          double negative_slope, int concat, int add_self_loops, double drop_p,
                          uint64_t seed, float* out);
/* aggr: 0 mean, 1 max, 2 sum, 3 pool.  lin_self NULL => rootWeight=false. */
int orc_sage_forward(const float* x, int64_t n, int64_t fin, const uint32_t* edge_index,
                     int64_t num_edges, int aggr, const float* lin_neighbor,
                     const float* lin_self, const float* bias, const float* pool_weight,
                     const float* pool_bias, int64_t fout, int normalize, float* out);
int orc_gin_forward(const float* x, int64_t n, int64_t fin, const uint32_t* edge_index,
                    int64_t num_edges, float eps, const float* w1, const float* b1,
                    int64_t hidden, const float* w2, const float* b2, int64_t fout,
                    float* out);
/* global sum pool over a batch vector (nodes visited in node order) */
void orc_sum_pool(const float* x, int64_t n, int64_t f, const uint32_t* batch,
                  int64_t num_graphs, float* out);

/* ---- streamed / row-parallel restatement (same per-row order) ---------- */
/* Destination-keyed CSR with each row's edges in COO order (stable counting
 * sort).  row_ptr [N+1], src_of [E] (source node), eid [E] (edge id). */
int orc_dst_csr(const uint32_t* edge_index, int64_t num_edges, int64_t num_nodes,
                uint32_t* row_ptr, uint32_t* src_of, uint32_t* eid);
/* op: 0 sum, 1 mean, 2 max, 3 gcn (norm from in-degree of the given graph),
 * self_loop_tail: treat every row as having one extra edge (i -> i) after its
 * own edges (the GCN/GAT self-loop insertion).  threads <= 0: all cores. */
void orc_csr_aggregate(const uint32_t* row_ptr, const uint32_t* src_of, int64_t num_rows,
                       const float* x, int64_t f, int op, int self_loop_tail,
                       int threads, float* out);
/* SAGE layer forward over a destination CSR, row-parallel, same bits as
 * orc_sage_forward (mean/max/sum aggregators). */
int orc_sage_forward_csr(const uint32_t* row_ptr, const uint32_t* src_of, int64_t n,
                         const float* x, int64_t fin, int aggr, const float* lin_neighbor,
                         const float* lin_self, const float* bias, int64_t fout,
                         int relu, int threads, float* out);
void orc_matmul_par(const float* a, const float* b, int64_t m, int64_t k, int64_t n,
                    int threads, float* out);
/* wasmSpmm for a list of rows (NULL: rows 0..nrows-1), row-parallel, same
 * bits as orc_spmm; out is [nrows, nf] in list order. */
void orc_spmm_rows(const uint32_t* row_ptr, const uint32_t* col, const float* val,
                   const float* dense, int64_t nf, const uint32_t* rows, int64_t nrows,
                   int threads, float* out);

/* ---- backward (no reference counterpart for the message passing; the
 *      matmul backward and bias reduction follow src/autograd/variable.ts) */
/* op: 0 sum, 1 mean, 2 max (x = the forward's input), 3 gcn (tail: appended
 * self-loops); out [n, f] = the gradient for the source rows. */
void orc_aggregate_backward(const uint32_t* edge_index, int64_t num_edges, int64_t num_nodes,
                            const float* x, const float* grad, int64_t f, int op, int tail,
                            float* out);
void orc_matmul_backward(const float* a, const float* b, const float* grad, int64_t m, int64_t k,
                         int64_t n, float* grad_a, float* grad_b);
void orc_bias_backward(const float* grad, int64_t rows, int64_t cols, float* out);

/* ---- model zoo: src/nn/linear.ts, src/nn/activation.ts, src/core/tensor.ts,
 *      and the three models under src/models/ ------------------------------ */
/* Linear.forward (src/nn/linear.ts:50-111): y[r,j] = f32(sum_i x[r,i]*w[j,i])
 * with the sum in double over i ascending, then f32(y + b[j]).  w is
 * [n, k] ([outFeatures, inFeatures]); b may be NULL. */
void orc_linear(const float* x, int64_t m, int64_t k, const float* w, const float* b, int64_t n,
                float* out);
void orc_sigmoid(const float* x, int64_t n, float* out); /* tensor.ts:413-419 */
void orc_tanh(const float* x, int64_t n, float* out);    /* tensor.ts:424-430 */
void orc_gelu(const float* x, int64_t n, float* out);    /* activation.ts:129-147 */
void orc_silu(const float* x, int64_t n, float* out);    /* activation.ts:153-168 */
void orc_prelu(const float* x, int64_t n, const float* w, int64_t nw, float* out); /* :175-200 */
/* Tensor.softmax / logSoftmax along the last axis (tensor.ts:435-499).
 * col_mask (may be NULL): column c with col_mask[c] != 0 reads mask_value
 * instead of x (the -1e9 mastery mask of LearningPathRecommender.ts:190-203). */
void orc_softmax_rows(const float* x, int64_t rows, int64_t cols, const uint8_t* col_mask,
                      float mask_value, int log_softmax, float* out);
/* The uniform draw that stands in for Math.random() at element i: the
 * SplitMix64 output of state seed + (i+1)*0x9E3779B97F4A7C15, top 53 bits
 * scaled to [0, 1). */
double orc_uniform(uint64_t seed, uint64_t i);
/* Dropout.forward in training mode (activation.ts:207-245): keep element i
 * when u_i > p and scale it by 1/(1-p) in double; else 0. */
void orc_dropout(const float* x, int64_t n, double p, uint64_t seed, float* out);
/* ConceptPrerequisiteMapper.predictLinks (ConceptPrerequisiteMapper.ts:224-295)
 * for pairs (src[q], tgt[q]) of node embeddings emb [num_nodes, d]; scores in
 * double.  mode 0 dot, 1 bilinear (w_bilinear [d, d]), 2 mlp (w1 [d, 3d],
 * b1 [d], w2 [1, d], b2 [1]; Dropout between them is the identity in eval). */
void orc_link_scores(const float* emb, int64_t d, const uint32_t* src, const uint32_t* tgt,
                     int64_t num_pairs, int mode, const float* w_bilinear, const float* w1,
                     const float* b1, const float* w2, const float* b2, double* out);

#ifdef __cplusplus
}
#endif
#endif
