/*
 * bgnn.h -- C ABI of libbgnn_cuda.so, the sm_100a (B200) backend for
 * BrowserGNN's message-passing path.
 *
 * The reference's device boundary is the GPUSparse / GPUTensor facade over
 * WebGPUComputeManager (src/core/gpu-sparse.ts:19-285,
 * src/backend/webgpu/compute-pipeline.ts:140-644).  Each entry point below
 * names the reference method it replaces.  Two families:
 *
 *   *_host  the reference's ownership model: the caller keeps its host
 *           buffers, the library copies inputs in, computes, copies the result
 *           into a caller-allocated host buffer and returns when it is there
 *           (WebGPUComputeManager uploads, dispatches and reads back per op).
 *   *_dev   device pointers, asynchronous on the context's stream, for
 *           device-resident multi-layer pipelines.  Results are ready after
 *           bgnn_ctx_synchronize (or any later operation on the same stream).
 *
 * Conventions: every call returns a bgnn_status; no exception or abort
 * crosses the ABI; bgnn_last_error() describes the last failure on a context.
 * A context is used by one host thread at a time.  Outputs are always
 * caller-allocated.  Feature matrices are row-major float32 [rows, features];
 * indices are uint32 node ids; edge_index is the reference's flat layout
 * [sources(E) | targets(E)] (src/core/graph.ts:14-35).
 *
 * Arithmetic: the reference evaluates in IEEE double and rounds once to f32
 * at every Float32Array store; the kernels reproduce that rounding sequence.
 * Sum/mean/max aggregation, GCN propagation, scatter/gather, CSR/degree/norm
 * construction are bit-exact with the reference in both math modes.  With
 * BGNN_MATH_EXACT the dense X*W transform and the SpMM/GAT accumulations are
 * bit-exact too (f64 emulation of each JS step); BGNN_MATH_FAST (default)
 * uses f32 FMA in the same order, which differs only where the reference's
 * double rounding lands on an f32 tie (well inside 1e-5 rel / 1e-6 abs).
 */
#ifndef BGNN_H
#define BGNN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BGNN_ABI_VERSION 1

#if defined(__GNUC__)
#define BGNN_API __attribute__((visibility("default")))
#else
#define BGNN_API
#endif

typedef enum bgnn_status {
  BGNN_OK = 0,
  BGNN_ERR_INVALID_ARG = 1,   /* bad size, null pointer, shape mismatch      */
  BGNN_ERR_OUT_OF_RANGE = 2,  /* an index >= its bound (graph.ts:88-92)      */
  BGNN_ERR_CUDA = 3,          /* a CUDA runtime call failed                  */
  BGNN_ERR_NO_MEMORY = 4,     /* device allocation failed                    */
  BGNN_ERR_TIMEOUT = 5,       /* a bounded device wait gave up               */
  BGNN_ERR_UNSUPPORTED = 6,   /* configuration the backend does not provide  */
  BGNN_ERR_DEVICE = 7         /* a kernel raised its error flag              */
} bgnn_status;

/* BGNN_MATH_TENSOR: as BGNN_MATH_FAST, except that the dense X*W products
 * (bgnn_linear, bgnn_sage_linear, bgnn_linear_add, matmul) run on the
 * tcgen05 tensor cores with a 3xTF32 split: f32-level accuracy but not the
 * reference's k-ascending f32 rounding sequence, so an element whose
 * reference value is a near-cancellation can fall outside the element-wise
 * 1e-6 + 1e-5|ref| bar.  Operands whose row length is not a multiple of 4
 * fall back to the FAST kernel. */
typedef enum bgnn_math_mode {
  BGNN_MATH_FAST = 0,
  BGNN_MATH_EXACT = 1,
  BGNN_MATH_TENSOR = 2
} bgnn_math_mode;

typedef enum bgnn_aggr {
  BGNN_AGGR_SUM = 0,  /* wasmScatterAdd  src/backend/wasm/index.ts:70-105  */
  BGNN_AGGR_MEAN = 1, /* wasmScatterMean src/backend/wasm/index.ts:112-151 */
  BGNN_AGGR_MAX = 2,  /* wasmScatterMax  src/backend/wasm/index.ts:158-206 */
  BGNN_AGGR_SPMM = 3  /* per-entry values, wasmSpmm src/backend/wasm/index.ts:342-383 */
} bgnn_aggr;

typedef enum bgnn_act {
  BGNN_ACT_NONE = 0,
  BGNN_ACT_RELU = 1,       /* wasmRelu: x > 0 ? x : 0   (index.ts:250-271)  */
  BGNN_ACT_RELU_MAX = 2,   /* Math.max(0, x): NaN kept  (gin.ts:106-112)    */
  BGNN_ACT_ELU = 3,        /* x > 0 ? x : a*(exp(x)-1)  (activation.ts:56-65) */
  BGNN_ACT_LEAKY_RELU = 4, /* x > 0 ? x : s*x           (tensor.ts:401-408) */
  BGNN_ACT_SIGMOID = 5,    /* 1/(1+exp(-x)) in f64      (tensor.ts:413-419) */
  BGNN_ACT_TANH = 6,       /* Math.tanh(x)              (tensor.ts:424-430) */
  BGNN_ACT_GELU = 7,       /* tanh-form GELU in f64     (activation.ts:129-147) */
  BGNN_ACT_SILU = 8        /* x/(1+exp(-x)) in f64      (activation.ts:153-168) */
} bgnn_act;

/* link scorers of ConceptPrerequisiteMapper (ConceptPrerequisiteMapper.ts:224-295) */
typedef enum bgnn_link_mode {
  BGNN_LINK_DOT = 0,      /* sigmoid(sum_i s[i]*t[i])                 */
  BGNN_LINK_BILINEAR = 1, /* sigmoid(sum_i s[i]*f32(W t)[i])          */
  BGNN_LINK_MLP = 2       /* sigmoid(Linear(ReLU(Linear([s,t,s*t]))))   */
} bgnn_link_mode;

typedef struct bgnn_ctx bgnn_ctx;
typedef struct bgnn_graph bgnn_graph;

/* ---- context ------------------------------------------------------------ */
BGNN_API int bgnn_abi_version(void);
/* Replaces BackendManager.initialize / initWebGPU (src/backend/index.ts:102-182). */
BGNN_API int bgnn_ctx_create(int device, bgnn_ctx** out);
BGNN_API int bgnn_ctx_destroy(bgnn_ctx* ctx);
/* Run subsequent work on an existing cudaStream_t (NULL: the legacy default
 * stream).  A new context starts on a non-blocking stream of its own. */
BGNN_API int bgnn_ctx_set_stream(bgnn_ctx* ctx, void* cuda_stream);
BGNN_API int bgnn_ctx_set_math(bgnn_ctx* ctx, int math_mode);
/* Persistent launches (the streaming aggregation, the tensor-core X*W) size
 * their grids for at most `sms` SMs, leaving the others to work the caller
 * runs beside them on another stream (0 or >= the GPU's SMs: all).  No
 * counterpart in the reference, which runs one kernel at a time. */
BGNN_API int bgnn_ctx_set_sm_budget(bgnn_ctx* ctx, uint32_t sms);
/* Waits for the context's stream and reports any kernel-raised error. */
BGNN_API int bgnn_ctx_synchronize(bgnn_ctx* ctx);
BGNN_API const char* bgnn_last_error(const bgnn_ctx* ctx);
/* Count of this library's kernel launches on the context (for accounting). */
BGNN_API uint64_t bgnn_ctx_launch_count(const bgnn_ctx* ctx);

/* Copies between caller host memory and device memory, returning when the
 * data is in place (the reference uploads each operand from a typed array
 * and reads a fresh one back, compute-pipeline.ts:182-190).  They first wait
 * for the work already queued on the context's stream.  Page-locked host
 * memory is copied directly; pageable memory (JS typed arrays, numpy) is
 * staged through pinned chunks the library owns, each filled or drained by a
 * pool of host threads while the DMA of the next chunk runs.  Safe to call
 * from two host threads at once (two staging rings per device). */
BGNN_API int bgnn_memcpy_h2d(bgnn_ctx* ctx, void* dst_dev, const void* src_host, uint64_t bytes);
BGNN_API int bgnn_memcpy_d2h(bgnn_ctx* ctx, void* dst_host, const void* src_dev, uint64_t bytes);

/* ---- facade mirror: WebGPUComputeManager methods, host buffers ---------- */
/* spmm: compute-pipeline.ts:140-232 / wasmSpmm index.ts:342-383 */
BGNN_API int bgnn_spmm_host(bgnn_ctx* ctx, const uint32_t* row_ptr, const uint32_t* col_indices,
                   const float* values, const float* dense, uint32_t num_rows,
                   uint32_t num_cols, uint32_t num_features, float* out);
/* scatterAdd: compute-pipeline.ts:237-305 / wasmScatterAdd index.ts:70-105 */
BGNN_API int bgnn_scatter_add_host(bgnn_ctx* ctx, const float* src, const uint32_t* index,
                          uint64_t num_msgs, uint32_t num_nodes, uint32_t num_features,
                          float* out);
/* scatterMean: gpu-sparse.ts:113-122 (CPU-only there) / index.ts:112-151 */
BGNN_API int bgnn_scatter_mean_host(bgnn_ctx* ctx, const float* src, const uint32_t* index,
                           uint64_t num_msgs, uint32_t num_nodes, uint32_t num_features,
                           float* out);
/* scatterMax: compute-pipeline.ts:310-385 / index.ts:158-206 */
BGNN_API int bgnn_scatter_max_host(bgnn_ctx* ctx, const float* src, const uint32_t* index,
                          uint64_t num_msgs, uint32_t num_nodes, uint32_t num_features,
                          float* out);
/* gather: compute-pipeline.ts:390-453 / index.ts:213-245 */
BGNN_API int bgnn_gather_host(bgnn_ctx* ctx, const float* src, uint32_t num_src_rows,
                     const uint32_t* index, uint64_t num_idx, uint32_t num_features,
                     float* out);
/* matmul: compute-pipeline.ts:458-521 / wasmMatmul index.ts:18-63 */
BGNN_API int bgnn_matmul_host(bgnn_ctx* ctx, const float* a, const float* b, uint32_t m, uint32_t k,
                     uint32_t n, float* out);
/* relu: compute-pipeline.ts:526-576 / index.ts:250-271 */
BGNN_API int bgnn_relu_host(bgnn_ctx* ctx, const float* x, uint64_t n, float* out);
/* add: compute-pipeline.ts:581-644 / index.ts:276-297 */
BGNN_API int bgnn_add_host(bgnn_ctx* ctx, const float* a, const float* b, uint64_t n, float* out);
/* wasmSpmv index.ts:304-335 (SparseCSR.matvec sparse.ts:301-317) */
BGNN_API int bgnn_spmv_host(bgnn_ctx* ctx, const uint32_t* row_ptr, const uint32_t* col_indices,
                   const float* values, const float* x, uint32_t num_rows, uint32_t num_cols,
                   float* out);

/* ---- the same ops on device pointers (async on the context stream) ------ */
BGNN_API int bgnn_spmm_dev(bgnn_ctx* ctx, const uint32_t* row_ptr, const uint32_t* col_indices,
                  const float* values, const float* dense, uint32_t num_rows,
                  uint32_t num_cols, uint32_t num_features, float* out);
BGNN_API int bgnn_scatter_dev(bgnn_ctx* ctx, int aggr, const float* src, const uint32_t* index,
                     uint64_t num_msgs, uint32_t num_nodes, uint32_t num_features, float* out);
BGNN_API int bgnn_gather_dev(bgnn_ctx* ctx, const float* src, uint32_t num_src_rows,
                    const uint32_t* index, uint64_t num_idx, uint32_t num_features, float* out);
BGNN_API int bgnn_matmul_dev(bgnn_ctx* ctx, const float* a, const float* b, uint32_t m, uint32_t k,
                    uint32_t n, float* out);
/* out[i] = act(x[i]); param = ELU alpha or LeakyReLU slope */
BGNN_API int bgnn_activation_dev(bgnn_ctx* ctx, int act, double param, const float* x, uint64_t n,
                        float* out);
BGNN_API int bgnn_add_dev(bgnn_ctx* ctx, const float* a, const float* b, uint64_t n, float* out);
BGNN_API int bgnn_spmv_dev(bgnn_ctx* ctx, const uint32_t* row_ptr, const uint32_t* col_indices,
                  const float* values, const float* x, uint32_t num_rows, uint32_t num_cols,
                  float* out);

/* ---- COO -> CSR, degrees, normalisation (device pointers) -------------- */
/* SparseCSR.fromCOO (src/core/sparse.ts:259-296): stable sort by (row, col),
 * bit-exact.  values may be NULL (all ones, SparseCOO.fromEdgeIndex
 * sparse.ts:81-92); val_out may be NULL. */
BGNN_API int bgnn_coo_to_csr_dev(bgnn_ctx* ctx, const uint32_t* rows, const uint32_t* cols,
                        const float* values, uint64_t nnz, uint32_t num_rows, uint32_t num_cols,
                        uint32_t* row_ptr, uint32_t* col_out, float* val_out);
BGNN_API int bgnn_coo_to_csr_host(bgnn_ctx* ctx, const uint32_t* rows, const uint32_t* cols,
                         const float* values, uint64_t nnz, uint32_t num_rows,
                         uint32_t num_cols, uint32_t* row_ptr, uint32_t* col_out,
                         float* val_out);
/* computeGCNNorm (src/core/sparse.ts:480-513): per-edge f32 weights. */
BGNN_API int bgnn_gcn_norm_dev(bgnn_ctx* ctx, const uint32_t* edge_index, uint64_t num_edges,
                      uint32_t num_nodes, int add_self_loops, float* out);

/* ---- device-resident graph (cached destination CSR) -------------------- */
/* Validates indices like the GraphData constructor (src/core/graph.ts:88-92),
 * then builds once: the destination-keyed CSR with each row's edges in COO
 * order (stable), in/out degrees, the self-loop flag (graph.ts:220-227) and
 * the row schedule.  edge_index is [src(E) | dst(E)], on the host when
 * edge_index_on_host != 0, else on the device.  num_src == num_dst for an
 * ordinary graph; a partition's local graph has num_dst owned rows and
 * num_src = owned + halo columns. */
BGNN_API int bgnn_graph_create(bgnn_ctx* ctx, const uint32_t* edge_index, uint64_t num_edges,
                      uint32_t num_src, uint32_t num_dst, int edge_index_on_host,
                      bgnn_graph** out);
/* A graph over an existing CSR (device buffers, copied): row r's entries are
 * col[row_ptr[r] .. row_ptr[r+1]).  For the standalone SpMM built by
 * bgnn_coo_to_csr_dev (SparseCSR, sparse.ts:236-383). */
BGNN_API int bgnn_graph_create_csr(bgnn_ctx* ctx, const uint32_t* row_ptr, const uint32_t* col,
                          uint32_t num_rows, uint32_t num_cols, bgnn_graph** out);
BGNN_API int bgnn_graph_destroy(bgnn_graph* g);
BGNN_API int bgnn_graph_info(const bgnn_graph* g, uint32_t* num_src, uint32_t* num_dst,
                    uint64_t* num_edges, int* has_self_loops);
/* getInDegrees / getOutDegrees (graph.ts:172-195) into device buffers */
BGNN_API int bgnn_graph_degrees(bgnn_ctx* ctx, const bgnn_graph* g, uint32_t* in_deg, uint32_t* out_deg);
/* copy the cached CSR out (device buffers; any may be NULL) */
BGNN_API int bgnn_graph_csr(bgnn_ctx* ctx, const bgnn_graph* g, uint32_t* row_ptr, uint32_t* src_of,
                   uint32_t* edge_id);

/* ---- fused layer message passing on a graph (device pointers) ---------- */
/* MessagePassing.gather + scatter{Add,Mean,Max} fused, no [E,F] message
 * tensor (sparse.ts:400-473): out[N_dst,F] from x[N_src,F]. */
BGNN_API int bgnn_aggregate(bgnn_ctx* ctx, const bgnn_graph* g, int aggr, const float* x,
                   uint32_t num_features, float* out);
/* GCNConv.forward after X*W (gcn.ts:88-156): the self-loop rule (loops
 * appended only if the graph has none and add_self_loops != 0), symmetric
 * norm (normalize != 0), edge-order sum, + bias (may be NULL), then act. */
BGNN_API int bgnn_gcn_propagate(bgnn_ctx* ctx, const bgnn_graph* g, const float* h,
                       uint32_t num_features, int add_self_loops, int normalize,
                       const float* bias, int act, double act_param, float* out);
/* GATConv.forward after X*W (gat.ts:115-254): LeakyReLU edge scores,
 * exp(s-10) softmax per destination, weighted sum (concat or head mean),
 * + bias, then act.  h [N, heads*c]; att_src/att_dst [heads, c]. */
BGNN_API int bgnn_gat(bgnn_ctx* ctx, const bgnn_graph* g, const float* h, uint32_t heads, uint32_t c,
             const float* att_src, const float* att_dst, double negative_slope, int concat,
             int add_self_loops, const float* bias, int act, double act_param, float* out);
/* GATConv.forward in training mode (gat.ts:107-258 with :194-203): bgnn_gat
 * plus attention dropout.  Entry (edge e, head h) of the normalised attention
 * (e counts the appended self-loops after the edges) is zeroed when u < p and
 * otherwise divided by (1 - p) in double, with u = the counter-based draw of
 * bgnn_dropout at position e*heads + h standing in for Math.random().
 * dropout in [0, 1). */
BGNN_API int bgnn_gat_train(bgnn_ctx* ctx, const bgnn_graph* g, const float* h, uint32_t heads,
                            uint32_t c, const float* att_src, const float* att_dst,
                            double negative_slope, int concat, int add_self_loops,
                            const float* bias, int act, double act_param, double dropout,
                            uint64_t seed, float* out);
/* bgnn_gat without any device allocation (no counterpart in the reference).
 * For callers that must not allocate once running -- an inference server
 * that reserves its memory budget at start-up, or a host application (such as
 * a Node-API addon inside a JavaScript runtime) whose device memory belongs to
 * someone else.  Same arguments and results as bgnn_gat; its per-edge
 * attention scratch and its slot -> row map live in a fixed 16 MiB device
 * array that every GPU loading this library keeps until exit, so
 * (edges + appended self-loops) * heads + edges must not exceed 4,194,304
 * (larger graphs get BGNN_ERR_INVALID_ARG).
 * The first call on a device looks up the array's device address; make that
 * first call before any stream capture begins.  All calls share the array:
 * calls that overlap on the GPU race on it. */
BGNN_API int bgnn_gat_noalloc(bgnn_ctx* ctx, const bgnn_graph* g, const float* h, uint32_t heads,
                              uint32_t c, const float* att_src, const float* att_dst,
                              double negative_slope, int concat, int add_self_loops,
                              const float* bias, int act, double act_param, float* out);
/* GINConv step 1-3 (gin.ts:131-157): out = f32((1+eps)*x + sum_j x_j). */
BGNN_API int bgnn_gin_aggregate(bgnn_ctx* ctx, const bgnn_graph* g, const float* x,
                       uint32_t num_features, float eps, float* out);
/* SpMM with per-edge values over the cached CSR (values in CSR order). */
BGNN_API int bgnn_graph_spmm(bgnn_ctx* ctx, const bgnn_graph* g, const float* values, const float* x,
                    uint32_t num_features, float* out);

/* ---- dense transforms with fused epilogues ------------------------------ */
/* out = act(a[m,k] * w[k,n] + bias)   (Tensor.matmul + bias loop + act) */
BGNN_API int bgnn_linear(bgnn_ctx* ctx, const float* a, const float* w, uint32_t m, uint32_t k,
                uint32_t n, const float* bias, int act, double act_param, float* out);
/* SAGEConv steps 3-5 (sage.ts:171-196):
 * out = act(f32(x*w_self + agg*w_neigh) + bias); w_self may be NULL
 * (rootWeight = false). */
BGNN_API int bgnn_sage_linear(bgnn_ctx* ctx, const float* agg, const float* x, const float* w_neigh,
                     const float* w_self, uint32_t m, uint32_t k, uint32_t n,
                     const float* bias, int act, double act_param, float* out);
/* The second half of bgnn_sage_linear as its own call: out = act(f32(f32(
 * addend + a*w) + bias)), a*w accumulated k-ascending per output exactly as
 * bgnn_linear.  With addend = x*w_self from bgnn_linear this is
 * bgnn_sage_linear split in two (SAGEConv.forward, sage.ts:171-196), so the
 * self product can run while the neighbour rows are still being exchanged.
 * addend may alias out. */
BGNN_API int bgnn_linear_add(bgnn_ctx* ctx, const float* a, const float* w, uint32_t m,
                             uint32_t k, uint32_t n, const float* addend, const float* bias,
                             int act, double act_param, float* out);
/* SAGE 'pool' aggregator projection (sage.ts:149-159) applied per node:
 * out[i,j] = f32(Math.max(0, bias[j] + sum_q x[i,q]*w[q,j])) with a double
 * accumulator; w is [k, k].  An edge's projected message depends only on its
 * source node, so max-aggregating these rows equals the reference. */
BGNN_API int bgnn_pool_projection(bgnn_ctx* ctx, const float* x, const float* w,
                                  const float* bias, uint32_t m, uint32_t k, float* out);
/* SAGE L2 normalise (sage.ts:199-214), in place on [m, n]. */
BGNN_API int bgnn_l2_normalize_rows(bgnn_ctx* ctx, float* x, uint32_t m, uint32_t n);
/* Global sum pool: g[b,:] = sum over nodes i with batch[i] == b, node order. */
BGNN_API int bgnn_sum_pool(bgnn_ctx* ctx, const float* x, uint32_t num_nodes, uint32_t num_features,
                  const uint32_t* batch, uint32_t num_graphs, float* out);
/* The same pool when every graph's nodes are contiguous (batchGraphs lays
 * them out so, graph.ts:439-492): graph b owns rows seg_ptr[b] ..
 * seg_ptr[b+1]-1 (device array, num_graphs+1 entries, non-decreasing,
 * seg_ptr[num_graphs] <= num rows of x).  No temporary structures, so it can
 * be captured in a CUDA graph. */
BGNN_API int bgnn_segment_sum(bgnn_ctx* ctx, const float* x, uint32_t num_features,
                              const uint32_t* seg_ptr, uint32_t num_graphs, float* out);

/* ---- partitioning support (node-partitioned multi-GPU) ------------------ */
/* out[i,:] = x[rows[i],:]  (halo pack; same kernel as gather) */
BGNN_API int bgnn_pack_rows(bgnn_ctx* ctx, const float* x, uint32_t num_x_rows, const uint32_t* rows,
                   uint32_t num_rows, uint32_t num_features, float* out);

/* ---- backward ----------------------------------------------------------
 * The reference's autograd differentiates X*W (Variable.matmul,
 * src/autograd/variable.ts:213-235), ReLU (variable.ts:358-373) and the
 * broadcast bias add (variable.ts:665-688) but not the message passing.  The
 * message-passing gradients below are the adjoint of the forward as that
 * autograd would compute it if gather and scatter were autograd ops: edge e
 * carries a message from grad[dst(e)], scatter-added over the sources in COO
 * edge order with an f32 store after every add (wasmScatterAdd,
 * src/backend/wasm/index.ts:70-105).  They run on the graph's transpose,
 * built on first use and kept with the graph (graphs from an edge list). */
/* grad_x [N_src, F] of bgnn_aggregate: sum: m_e = grad[dst]; mean:
 * m_e = f32(grad[dst] * (1/cnt(dst))), 1/cnt in double; max: m_e = grad[dst]
 * for the edge that last raised the forward maximum of that feature (x > acc
 * in edge order from -inf; x = the forward input), else 0. */
BGNN_API int bgnn_aggregate_backward(bgnn_ctx* ctx, const bgnn_graph* g, int aggr,
                                     const float* x, const float* grad, uint32_t num_features,
                                     float* grad_x);
/* grad_h [N, F] of bgnn_gcn_propagate before its bias and activation:
 * m_e = f32(grad[dst] * w_e) with the forward's norm w_e, the appended
 * self-loop edges (when the forward appended them) last. */
BGNN_API int bgnn_gcn_propagate_backward(bgnn_ctx* ctx, const bgnn_graph* g, const float* grad,
                                         uint32_t num_features, int add_self_loops,
                                         int normalize, float* grad_h);
/* Variable.matmul backward (variable.ts:213-235), out = a[m,k] * b[k,n]:
 * grad_a [m, k] = grad @ transpose(b), grad_b [k, n] = transpose(a) @ grad,
 * each output one k-ascending chain as wasmMatmul computes it (either may be
 * NULL). */
BGNN_API int bgnn_matmul_backward(bgnn_ctx* ctx, const float* a, const float* b,
                                  const float* grad, uint32_t m, uint32_t k, uint32_t n,
                                  float* grad_a, float* grad_b);
/* The bias gradient of a broadcast add (variable.ts:675-685): out[j] = the
 * row-ordered f32 sum of grad[:, j]. */
BGNN_API int bgnn_bias_backward(bgnn_ctx* ctx, const float* grad, uint64_t rows, uint32_t cols,
                                float* out);
/* ReLU backward (variable.ts:358-373): grad where the forward output > 0. */
BGNN_API int bgnn_relu_backward(bgnn_ctx* ctx, const float* grad, const float* out, uint64_t n,
                                float* grad_in);

/* ---- row partition of a graph across the GPUs of one node ---------------
 * No counterpart in the reference, which is single-device: these run the
 * message passing of SAGEConv.forward (src/layers/sage.ts:113-217) and
 * SparseCSR.matmul (src/core/sparse.ts:322-344) on several GPUs, one process
 * per GPU.  Rank r owns the contiguous rows [lo, hi) of a square graph (about
 * (E + N) / world entries plus rows each) and keeps their entries in the
 * global order, so each row is reduced on one GPU exactly as on a single GPU.
 * Every rank passes the same graph and derives the same plan on its device:
 * no communication.  The local graph has n_own = hi - lo rows and
 * n_own + n_halo columns: owned nodes first, then the halo nodes (the
 * sorted unique remote columns the local rows read, grouped by owner).  A
 * layer's input therefore lives in an [owned | halo] buffer of
 * n_own + n_halo rows whose first n_own rows are this rank's. */
typedef struct bgnn_part bgnn_part;
/* From a graph's edge list ([src(E) | dst(E)], host or device): rows are
 * destinations, each row's edges in COO order (the aggregation's order). */
BGNN_API int bgnn_part_create(bgnn_ctx* ctx, const uint32_t* edge_index, uint64_t num_edges,
                              uint32_t num_nodes, uint32_t world, uint32_t rank,
                              int edge_index_on_host, bgnn_part** out);
/* From a square device CSR (SparseCSR.fromCOO output): rows keep their
 * entries in CSR order; the local entries are the global entries
 * [entry_lo, entry_lo + num_local_entries), so per-entry values are the
 * caller's value array offset by entry_lo. */
BGNN_API int bgnn_part_create_csr(bgnn_ctx* ctx, const uint32_t* row_ptr, const uint32_t* col,
                                  uint32_t num_rows, uint32_t world, uint32_t rank,
                                  bgnn_part** out);
BGNN_API int bgnn_part_destroy(bgnn_part* p);
BGNN_API int bgnn_part_info(const bgnn_part* p, uint32_t* row_lo, uint32_t* row_hi,
                            uint32_t* num_halo, uint64_t* entry_lo, uint64_t* num_local_entries,
                            uint64_t* num_send);
/* bounds: world + 1 row boundaries (host array) */
BGNN_API int bgnn_part_bounds(const bgnn_part* p, uint32_t* bounds);
/* rows this rank sends to / receives from each rank (host arrays of world) */
BGNN_API int bgnn_part_counts(const bgnn_part* p, uint64_t* send_rows, uint64_t* recv_rows);
/* Row blocks (the early halo sends of bgnn_dist_sage_layer_ex): every
 * rank's owned rows cut into `blocks` blocks, block c of n rows being rows
 * [c*n/blocks, (c+1)*n/blocks).  Host arrays of world * (blocks + 1), either
 * may be NULL: send_first[q*(blocks+1) + c] = the first entry of peer q's
 * send list in this rank's block c (entry indices as in bgnn_part_lists),
 * recv_first[q*(blocks+1) + c] = the first halo slot of owner q's block c. */
BGNN_API int bgnn_part_row_blocks(bgnn_ctx* ctx, const bgnn_part* p, uint32_t blocks,
                                  uint64_t* send_first, uint64_t* recv_first);
/* the local graph (owned by the partition; valid until bgnn_part_destroy) */
BGNN_API int bgnn_part_graph(const bgnn_part* p, const bgnn_graph** out);
/* copies of the plan's lists (device buffers; either may be NULL): the
 * global id of each halo slot [num_halo], and the owned rows (local ids)
 * sent to the peers in peer order [num_send] */
BGNN_API int bgnn_part_lists(bgnn_ctx* ctx, const bgnn_part* p, uint32_t* halo_ids,
                             uint32_t* send_rows);
/* out[i, :] = x[send_row[i], col0 : col0 + width] (x row stride ld_x) */
BGNN_API int bgnn_part_pack(bgnn_ctx* ctx, const bgnn_part* p, const float* x, uint64_t ld_x,
                            uint32_t col0, uint32_t width, float* out);
/* x[n_own + i, col0 : col0 + width] = halo[i, :] for every halo row i */
BGNN_API int bgnn_part_unpack(bgnn_ctx* ctx, const bgnn_part* p, const float* halo,
                              uint32_t width, float* x, uint64_t ld_x, uint32_t col0);
/* bgnn_aggregate / bgnn_graph_spmm (aggr BGNN_AGGR_SPMM, values per entry)
 * over a column slice: x rows of stride ld_x, out rows of stride ld_out. */
BGNN_API int bgnn_aggregate_strided(bgnn_ctx* ctx, const bgnn_graph* g, int aggr,
                                    const float* values, const float* x, uint64_t ld_x,
                                    uint32_t width, float* out, uint64_t ld_out);

/* ---- NCCL halo exchange and distributed layers (one process per GPU) ----
 * A bgnn_dist is one rank's NCCL communicator plus its streams.  Rank 0
 * makes the unique id (bgnn_dist_unique_id) and the caller shares it with
 * the other ranks by its own means.  Every call is asynchronous on the
 * context's stream.  timeout_ms bounds every piece of NCCL work: when it is
 * not done in time (a peer failed or never joined) the communicator is
 * aborted and this and every later call on the object return
 * BGNN_ERR_TIMEOUT.  max_ctas caps the CTAs NCCL uses (0: NCCL's default);
 * the aggregation leaves that many SMs free while later chunks are in
 * flight.  NCCL is loaded at run time (the copy already in the process, else
 * libnccl.so.2 or $BGNN_NCCL_LIBRARY); without it these return
 * BGNN_ERR_UNSUPPORTED. */
#define BGNN_UNIQUE_ID_BYTES 128
typedef struct bgnn_dist bgnn_dist;
BGNN_API int bgnn_dist_unique_id(uint8_t* id_out);
BGNN_API int bgnn_dist_create(bgnn_ctx* ctx, const uint8_t* unique_id, uint32_t world,
                              uint32_t rank, uint32_t timeout_ms, uint32_t max_ctas,
                              bgnn_dist** out);
BGNN_API int bgnn_dist_destroy(bgnn_dist* d);
/* Abort the communicator (a rank that learned on the host that a peer is
 * gone): pending NCCL work ends, later calls return BGNN_ERR_DEVICE, and
 * bgnn_dist_destroy then needs no peer. */
BGNN_API int bgnn_dist_abort(bgnn_dist* d);
/* column chunks of the exchange (0 or 1: one; a column slice re-walks every
 * edge, so more chunks pay only when the exchange outlasts x*W_self) and
 * SMs left to NCCL while later chunks fly */
BGNN_API int bgnn_dist_set_pipeline(bgnn_dist* d, uint32_t chunks, uint32_t reserve_sms);
/* Fill the halo rows of x_ext ([n_own + n_halo, F], owned rows present)
 * with their owners' rows. */
BGNN_API int bgnn_dist_exchange(bgnn_dist* d, const bgnn_part* p, float* x_ext,
                                uint32_t num_features);
/* Halo exchange + fused gather/scatter (MessagePassing.scatter{Add,Mean,Max},
 * sparse.ts:400-451) of the local rows: out [n_own, F].  With several column
 * chunks (bgnn_dist_set_pipeline) each chunk's columns are aggregated as soon
 * as it has landed; the halo rows of x_ext are filled as a side effect. */
BGNN_API int bgnn_dist_aggregate(bgnn_dist* d, const bgnn_part* p, int aggr, float* x_ext,
                                 uint32_t num_features, float* out);
/* The same with per-entry values: the row-partitioned SparseCSR.matmul
 * (sparse.ts:322-344 / wasmSpmm index.ts:342-383); values are the local
 * entries' values (global values + entry_lo). */
BGNN_API int bgnn_dist_spmm(bgnn_dist* d, const bgnn_part* p, const float* values, float* x_ext,
                            uint32_t num_features, float* out);
/* One SAGEConv layer (sage.ts:113-217) on the partition: x_ext [n_own +
 * n_halo, k] with owned rows present; agg [n_own, k] scratch for the
 * aggregation; out [n_own, n] = act(f32(f32(x*w_self + agg*w_neigh) + bias))
 * (the roundings of bgnn_sage_linear; w_self NULL: rootWeight = false).
 * x*w_self runs on a side stream while the halo rows are exchanged.  out may
 * be the owned rows of the next layer's [owned | halo] buffer. */
BGNN_API int bgnn_dist_sage_layer(bgnn_dist* d, const bgnn_part* p, int aggr, float* x_ext,
                                  uint32_t k, uint32_t n, const float* w_neigh,
                                  const float* w_self, const float* bias, int act,
                                  double act_param, float* agg, float* out);
/* bgnn_dist_sage_layer with flags.  BGNN_DIST_SEND_OUT: out is the owned
 * rows of the next layer's [n_own + n_halo, n] buffer, and its halo exchange
 * starts while the layer's last product is still running: the product runs
 * in row blocks (bgnn_dist_set_row_blocks) and each block's rows go to the
 * peers as soon as it is written.  The next bgnn_dist_sage_layer /
 * _aggregate / _exchange on that buffer (same partition, width n) finds its
 * halo in flight and only waits for it.  Every rank passes the same flags
 * (the sends pair up across ranks). */
#define BGNN_DIST_SEND_OUT 1u
BGNN_API int bgnn_dist_sage_layer_ex(bgnn_dist* d, const bgnn_part* p, int aggr, float* x_ext,
                                     uint32_t k, uint32_t n, const float* w_neigh,
                                     const float* w_self, const float* bias, int act,
                                     double act_param, float* agg, float* out, uint32_t flags);
/* row blocks of BGNN_DIST_SEND_OUT (1..8; default 4) */
BGNN_API int bgnn_dist_set_row_blocks(bgnn_dist* d, uint32_t blocks);
/* Element-wise maximum over the ranks of count host doubles, in place
 * (timing); synchronises. */
BGNN_API int bgnn_dist_allreduce_max(bgnn_dist* d, double* values, uint32_t count);
/* Wait for the context's stream, or for the timeout to abort the NCCL work
 * it depends on (BGNN_ERR_TIMEOUT). */
BGNN_API int bgnn_dist_synchronize(bgnn_dist* d);

/* ---- benchmark inputs ------------------------------------------------------ */
/* Seeded R-MAT edge list [src(E) | dst(E)] on the device (no reference
 * counterpart: the reference's randomGraph is Erdos-Renyi on Math.random).
 * Quadrant probabilities a, b, c (d = 1-a-b-c), 2^scale id space, ids >=
 * num_nodes rejected, optional seeded relabelling of node ids.  Produces the
 * same list as the numpy generator in browsergnn_b200/synth.py. */
BGNN_API int bgnn_synth_rmat(bgnn_ctx* ctx, uint64_t seed, int scale, uint32_t num_nodes,
                             uint64_t num_edges, double a, double b, double c, int permute,
                             uint32_t* edge_index);

/* ---- model zoo building blocks (src/nn/, src/core/tensor.ts, src/models/) ----
 * Device pointers, asynchronous on the context stream; index errors surface
 * at the next synchronising call (bgnn_ctx_synchronize or a *_host call). */

/* Linear.forward (src/nn/linear.ts:50-111): out[m, n] = act(f32(f32(x w^T) + b))
 * where the sum over k is one double per output, ascending, w is
 * [n, k] ([outFeatures, inFeatures]) and bias may be NULL.  act applies the
 * activation module that follows in a Sequential. */
BGNN_API int bgnn_dense(bgnn_ctx* ctx, const float* x, const float* w, uint32_t m, uint32_t k,
                        uint32_t n, const float* bias, int act, double act_param, float* out);
/* Tensor.softmax (log_softmax = 0) / Tensor.logSoftmax (1) along the rows of
 * [rows, cols] (src/core/tensor.ts:435-499).  col_mask may be NULL; where
 * col_mask[c] != 0 the input reads mask_value (LearningPathRecommender.ts:
 * 190-203 masks mastered concepts with -1e9 before its softmax). */
BGNN_API int bgnn_softmax_rows(bgnn_ctx* ctx, const float* x, uint32_t rows, uint32_t cols,
                               const uint8_t* col_mask, float mask_value, int log_softmax,
                               float* out);
/* Dropout.forward in training mode (src/nn/activation.ts:207-245): keeps
 * element i when u_i > p and scales it by 1/(1-p).  u_i is a counter-based
 * draw in [0, 1) (SplitMix64 of seed + (i+1)*0x9E3779B97F4A7C15, top 53 bits)
 * standing in for Math.random(); in eval mode Dropout is the identity and
 * needs no call.  p outside [0, 1] -> BGNN_ERR_INVALID_ARG. */
BGNN_API int bgnn_dropout(bgnn_ctx* ctx, const float* x, uint64_t n, double p, uint64_t seed,
                          float* out);
/* PReLU (src/nn/activation.ts:175-200): x > 0 ? x : a*x, a = weight[0] when
 * num_params == 1, else weight[i % num_params]. */
BGNN_API int bgnn_prelu(bgnn_ctx* ctx, const float* x, uint64_t n, const float* weight,
                        uint32_t num_params, float* out);
/* ConceptPrerequisiteMapper.predictLinks (ConceptPrerequisiteMapper.ts:224-295):
 * out[q] (double) scores the pair (src[q], tgt[q]) of rows of emb
 * [num_nodes, dim].  mode: bgnn_link_mode.  bilinear: w_bilinear [dim, dim];
 * mlp: w1 [dim, 3*dim], b1 [dim] (or NULL), w2 [1, dim], b2 [1] (or NULL),
 * the eval-mode network (its Dropout is the identity).  dim <= 1600 for mlp.
 * An out-of-range node id is reported as BGNN_ERR_OUT_OF_RANGE. */
BGNN_API int bgnn_link_scores(bgnn_ctx* ctx, const float* emb, uint32_t num_nodes, uint32_t dim,
                              const uint32_t* src, const uint32_t* tgt, uint64_t num_pairs,
                              int mode, const float* w_bilinear, const float* w1, const float* b1,
                              const float* w2, const float* b2, double* out);

#ifdef __cplusplus
}
#endif
#endif /* BGNN_H */
