// extern "C" entry points of libbgnn_cuda.so: context lifetime, the
// WebGPUComputeManager-shaped facade (host and device variants) and the fused
// layer operations on cached graphs.  See include/bgnn.h for the contract.
#include <cstring>

#include "bgnn_internal.cuh"

namespace {

int ctx_ok(bgnn_ctx* ctx) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess)
    return bgnn_set_error(ctx, BGNN_ERR_CUDA, "cudaSetDevice(%d): %s", ctx->device,
                          cudaGetErrorString(e));
  return BGNN_OK;
}

// copy host -> fresh device buffer
int to_dev(bgnn_ctx* ctx, DevTmp& t, const void* h, size_t bytes) {
  BGNN_TRY(bgnn_tmp_alloc(ctx, t, bytes));
  if (bytes && h)
    BGNN_CUDA(ctx, cudaMemcpyAsync(t.p, h, bytes, cudaMemcpyHostToDevice, ctx->stream));
  return BGNN_OK;
}

int finish_host(bgnn_ctx* ctx, void* host_out, const void* dev_out, size_t bytes) {
  if (bytes)
    BGNN_CUDA(ctx, cudaMemcpyAsync(host_out, dev_out, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  return bgnn_check_device_error(ctx);  // synchronises
}

AggArgs graph_args(const bgnn_graph* g, const float* x, uint32_t f, float* out) {
  AggArgs a;
  std::memset(&a, 0, sizeof(a));
  a.row_ptr = g->row_ptr;
  a.src_of = g->src_of;
  a.x = x;
  a.ld_x = f;
  a.n_rows = g->n_dst;
  a.num_features = (int)f;
  a.out = out;
  a.ld_out = f;
  a.heavy_rows = g->heavy_rows;
  a.n_heavy = g->n_heavy;
  a.heavy_threshold = g->heavy_threshold;
  a.items = g->items;
  a.n_items = g->n_items;
  a.n_heavy_items = g->n_heavy_items;
  a.heavy_deg = g->heavy_deg.empty() ? nullptr : g->heavy_deg.data();
  a.num_edges = g->num_edges;
  a.gin_ope = 1.0;
  a.act = BGNN_ACT_NONE;
  return a;
}

int check_act(bgnn_ctx* ctx, int act) {
  if (act < BGNN_ACT_NONE || act > BGNN_ACT_SILU)
    return bgnn_set_error(ctx, BGNN_ERR_INVALID_ARG, "unknown activation %d", act);
  return BGNN_OK;
}

// temporary graph over a caller's (msg -> node) index list: the scatter ops
int scatter_graph(bgnn_ctx* ctx, const uint32_t* index, uint64_t m, uint32_t num_nodes,
                  bgnn_graph* g) {
  if (m >= 0xffffffffull)
    return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED, "message count exceeds 2^32-2");
  DevTmp iota;
  BGNN_TRY(bgnn_tmp_alloc(ctx, iota, (m ? m : 1) * 4));
  BGNN_TRY(bgnn_iota(ctx, iota.as<uint32_t>(), m));
  return bgnn_graph_build(ctx, iota.as<uint32_t>(), index, m, (uint32_t)m, num_nodes, g);
}

struct GraphGuard {
  bgnn_graph g;
  ~GraphGuard() { bgnn_graph_free(&g); }
};

}  // namespace

// ---- context ---------------------------------------------------------------
extern "C" int bgnn_abi_version(void) { return BGNN_ABI_VERSION; }

extern "C" int bgnn_ctx_create(int device, bgnn_ctx** out) {
  if (!out) return BGNN_ERR_INVALID_ARG;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
    cudaGetLastError();
    return BGNN_ERR_CUDA;
  }
  bgnn_ctx* c = new bgnn_ctx();
  c->device = device;
  bool ok = cudaSetDevice(device) == cudaSuccess;
  ok = ok && cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device) == cudaSuccess;
  ok = ok && cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking) == cudaSuccess;
  int lo_prio = 0, hi_prio = 0;
  ok = ok && cudaDeviceGetStreamPriorityRange(&lo_prio, &hi_prio) == cudaSuccess;
  // the aux stream runs work that gates the main stream (heavy rows, hub slices)
  ok = ok && cudaStreamCreateWithPriority(&c->aux_stream, cudaStreamNonBlocking, hi_prio) == cudaSuccess;
  ok = ok && cudaEventCreateWithFlags(&c->ev_fork, cudaEventDisableTiming) == cudaSuccess;
  ok = ok && cudaEventCreateWithFlags(&c->ev_join, cudaEventDisableTiming) == cudaSuccess;
  ok = ok && cudaMalloc(&c->d_err, 4 * sizeof(int)) == cudaSuccess;
  ok = ok && cudaMalloc(&c->d_small, 64) == cudaSuccess;
  ok = ok && cudaMemset(c->d_err, 0, 4 * sizeof(int)) == cudaSuccess;
  if (ok) {
    // keep freed stream-ordered allocations cached in this process's pool
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
      uint64_t thr = ~0ull;
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
    }
  }
  if (!ok) {
    cudaGetLastError();
    bgnn_ctx_destroy(c);
    return BGNN_ERR_CUDA;
  }
  c->stream = c->own_stream;
  *out = c;
  return BGNN_OK;
}

extern "C" int bgnn_ctx_destroy(bgnn_ctx* c) {
  if (!c) return BGNN_OK;
  cudaSetDevice(c->device);
  if (c->own_stream) cudaStreamSynchronize(c->own_stream);
  if (c->stream && c->stream != c->own_stream) cudaStreamSynchronize(c->stream);
  if (c->aux_stream) cudaStreamSynchronize(c->aux_stream);
  cudaFree(c->d_err);
  cudaFree(c->d_small);
  if (c->ev_fork) cudaEventDestroy(c->ev_fork);
  if (c->ev_join) cudaEventDestroy(c->ev_join);
  if (c->aux_stream) cudaStreamDestroy(c->aux_stream);
  if (c->own_stream) cudaStreamDestroy(c->own_stream);
  delete c;
  return BGNN_OK;
}

extern "C" int bgnn_ctx_set_stream(bgnn_ctx* ctx, void* s) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  ctx->stream = static_cast<cudaStream_t>(s);  // NULL: the legacy default stream
  return BGNN_OK;
}

extern "C" int bgnn_ctx_set_sm_budget(bgnn_ctx* ctx, uint32_t sms) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  ctx->grid_sms = sms >= (uint32_t)ctx->num_sms ? 0 : (int)sms;
  return BGNN_OK;
}

extern "C" int bgnn_ctx_set_math(bgnn_ctx* ctx, int mode) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  if (mode != BGNN_MATH_FAST && mode != BGNN_MATH_EXACT && mode != BGNN_MATH_TENSOR)
    return bgnn_set_error(ctx, BGNN_ERR_INVALID_ARG, "unknown math mode %d", mode);
  ctx->math = mode;
  return BGNN_OK;
}

extern "C" int bgnn_ctx_synchronize(bgnn_ctx* ctx) {
  BGNN_TRY(ctx_ok(ctx));
  return bgnn_check_device_error(ctx);
}

extern "C" const char* bgnn_last_error(const bgnn_ctx* ctx) {
  return ctx ? ctx->last_error.c_str() : "null context";
}

extern "C" uint64_t bgnn_ctx_launch_count(const bgnn_ctx* ctx) { return ctx ? ctx->launches : 0; }

// ---- device-pointer facade ---------------------------------------------------
extern "C" int bgnn_scatter_dev(bgnn_ctx* ctx, int aggr, const float* src, const uint32_t* index,
                                uint64_t m, uint32_t num_nodes, uint32_t f, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, aggr >= BGNN_AGGR_SUM && aggr <= BGNN_AGGR_MAX, "unknown aggregation %d", aggr);
  BGNN_REQUIRE(ctx, (src && index) || m == 0, "NULL src/index");
  BGNN_REQUIRE(ctx, out || (uint64_t)num_nodes * f == 0, "NULL out");
  GraphGuard gg;
  BGNN_TRY(scatter_graph(ctx, index, m, num_nodes, &gg.g));
  AggArgs a = graph_args(&gg.g, src, f, out);
  a.mean = aggr == BGNN_AGGR_MEAN;
  a.max_fix = aggr == BGNN_AGGR_MAX;
  BGNN_TRY(bgnn_run_aggregate(ctx, aggr == BGNN_AGGR_MAX ? OP_MAX : OP_SUM, a));
  // the temporary graph is freed on return: wait for the kernels that read it
  BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return BGNN_OK;
}

extern "C" int bgnn_gather_dev(bgnn_ctx* ctx, const float* src, uint32_t num_src_rows,
                               const uint32_t* index, uint64_t n, uint32_t f, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, (src && index && out) || n * f == 0, "NULL argument");
  return bgnn_run_gather_rows(ctx, src, num_src_rows, index, n, f, out);
}

extern "C" int bgnn_pack_rows(bgnn_ctx* ctx, const float* x, uint32_t num_x_rows,
                              const uint32_t* rows, uint32_t num_rows, uint32_t f, float* out) {
  return bgnn_gather_dev(ctx, x, num_x_rows, rows, num_rows, f, out);
}

extern "C" int bgnn_matmul_dev(bgnn_ctx* ctx, const float* a, const float* b, uint32_t m,
                               uint32_t k, uint32_t n, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, (a && b) || (uint64_t)m * k * n == 0, "NULL operand");
  BGNN_REQUIRE(ctx, out || (uint64_t)m * n == 0, "NULL out");
  return bgnn_run_linear(ctx, a, b, nullptr, nullptr, m, k, n, nullptr, BGNN_ACT_NONE, 0.0, out);
}

extern "C" int bgnn_activation_dev(bgnn_ctx* ctx, int act, double param, const float* x,
                                   uint64_t n, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_TRY(check_act(ctx, act));
  BGNN_REQUIRE(ctx, (x && out) || n == 0, "NULL argument");
  return bgnn_run_activation(ctx, act, param, x, n, out);
}

extern "C" int bgnn_add_dev(bgnn_ctx* ctx, const float* a, const float* b, uint64_t n, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, (a && b && out) || n == 0, "NULL argument");
  return bgnn_run_add(ctx, a, b, n, out);
}

extern "C" int bgnn_spmm_dev(bgnn_ctx* ctx, const uint32_t* row_ptr, const uint32_t* col,
                             const float* values, const float* dense, uint32_t num_rows,
                             uint32_t num_cols, uint32_t f, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, row_ptr && out, "NULL row_ptr/out");
  GraphGuard gg;
  BGNN_TRY(bgnn_graph_from_csr(ctx, row_ptr, col, num_rows, num_cols, &gg.g, false));
  BGNN_REQUIRE(ctx, (values && dense) || gg.g.num_edges == 0 || f == 0, "NULL values/dense");
  AggArgs a = graph_args(&gg.g, dense, f, out);
  a.val = values;
  a.exact = ctx->math == BGNN_MATH_EXACT;
  BGNN_TRY(bgnn_run_aggregate(ctx, OP_SPMM, a));
  BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return BGNN_OK;
}

extern "C" int bgnn_spmv_dev(bgnn_ctx* ctx, const uint32_t* row_ptr, const uint32_t* col,
                             const float* values, const float* x, uint32_t num_rows,
                             uint32_t num_cols, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, row_ptr && out, "NULL row_ptr/out");
  {
    GraphGuard gg;  // validates row_ptr monotonicity and column bounds
    BGNN_TRY(bgnn_graph_from_csr(ctx, row_ptr, col, num_rows, num_cols, &gg.g, false));
  }
  return bgnn_run_spmv(ctx, row_ptr, col, values, x, num_rows, out);
}

// ---- host facade (WebGPUComputeManager ownership model) ----------------------
extern "C" int bgnn_spmm_host(bgnn_ctx* ctx, const uint32_t* row_ptr, const uint32_t* col,
                              const float* values, const float* dense, uint32_t num_rows,
                              uint32_t num_cols, uint32_t f, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, row_ptr && out, "NULL row_ptr/out");
  const uint64_t nnz = (uint64_t)row_ptr[num_rows];
  DevTmp drp, dcol, dval, dx, dout;
  BGNN_TRY(to_dev(ctx, drp, row_ptr, ((size_t)num_rows + 1) * 4));
  BGNN_TRY(to_dev(ctx, dcol, col, nnz * 4));
  BGNN_TRY(to_dev(ctx, dval, values, nnz * 4));
  BGNN_TRY(to_dev(ctx, dx, dense, (size_t)num_cols * f * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, dout, (size_t)num_rows * f * 4));
  BGNN_TRY(bgnn_spmm_dev(ctx, drp.as<uint32_t>(), dcol.as<uint32_t>(), dval.as<float>(),
                         dx.as<float>(), num_rows, num_cols, f, dout.as<float>()));
  return finish_host(ctx, out, dout.p, (size_t)num_rows * f * 4);
}

static int scatter_host(bgnn_ctx* ctx, int aggr, const float* src, const uint32_t* index,
                        uint64_t m, uint32_t num_nodes, uint32_t f, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, out || (uint64_t)num_nodes * f == 0, "NULL out");
  DevTmp dsrc, didx, dout;
  BGNN_TRY(to_dev(ctx, dsrc, src, m * f * 4));
  BGNN_TRY(to_dev(ctx, didx, index, m * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, dout, (size_t)num_nodes * f * 4));
  BGNN_TRY(bgnn_scatter_dev(ctx, aggr, dsrc.as<float>(), didx.as<uint32_t>(), m, num_nodes, f,
                            dout.as<float>()));
  return finish_host(ctx, out, dout.p, (size_t)num_nodes * f * 4);
}

extern "C" int bgnn_scatter_add_host(bgnn_ctx* ctx, const float* src, const uint32_t* index,
                                     uint64_t m, uint32_t num_nodes, uint32_t f, float* out) {
  return scatter_host(ctx, BGNN_AGGR_SUM, src, index, m, num_nodes, f, out);
}
extern "C" int bgnn_scatter_mean_host(bgnn_ctx* ctx, const float* src, const uint32_t* index,
                                      uint64_t m, uint32_t num_nodes, uint32_t f, float* out) {
  return scatter_host(ctx, BGNN_AGGR_MEAN, src, index, m, num_nodes, f, out);
}
extern "C" int bgnn_scatter_max_host(bgnn_ctx* ctx, const float* src, const uint32_t* index,
                                     uint64_t m, uint32_t num_nodes, uint32_t f, float* out) {
  return scatter_host(ctx, BGNN_AGGR_MAX, src, index, m, num_nodes, f, out);
}

extern "C" int bgnn_gather_host(bgnn_ctx* ctx, const float* src, uint32_t num_src_rows,
                                const uint32_t* index, uint64_t n, uint32_t f, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, out || n * f == 0, "NULL out");
  DevTmp dsrc, didx, dout;
  BGNN_TRY(to_dev(ctx, dsrc, src, (size_t)num_src_rows * f * 4));
  BGNN_TRY(to_dev(ctx, didx, index, n * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, dout, n * f * 4));
  BGNN_TRY(bgnn_gather_dev(ctx, dsrc.as<float>(), num_src_rows, didx.as<uint32_t>(), n, f,
                           dout.as<float>()));
  return finish_host(ctx, out, dout.p, n * f * 4);
}

extern "C" int bgnn_matmul_host(bgnn_ctx* ctx, const float* a, const float* b, uint32_t m,
                                uint32_t k, uint32_t n, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, out || (uint64_t)m * n == 0, "NULL out");
  DevTmp da, db, dout;
  BGNN_TRY(to_dev(ctx, da, a, (size_t)m * k * 4));
  BGNN_TRY(to_dev(ctx, db, b, (size_t)k * n * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, dout, (size_t)m * n * 4));
  BGNN_TRY(bgnn_matmul_dev(ctx, da.as<float>(), db.as<float>(), m, k, n, dout.as<float>()));
  return finish_host(ctx, out, dout.p, (size_t)m * n * 4);
}

extern "C" int bgnn_relu_host(bgnn_ctx* ctx, const float* x, uint64_t n, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  DevTmp dx, dout;
  BGNN_TRY(to_dev(ctx, dx, x, n * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, dout, n * 4));
  BGNN_TRY(bgnn_activation_dev(ctx, BGNN_ACT_RELU, 0.0, dx.as<float>(), n, dout.as<float>()));
  return finish_host(ctx, out, dout.p, n * 4);
}

extern "C" int bgnn_add_host(bgnn_ctx* ctx, const float* a, const float* b, uint64_t n,
                             float* out) {
  BGNN_TRY(ctx_ok(ctx));
  DevTmp da, db, dout;
  BGNN_TRY(to_dev(ctx, da, a, n * 4));
  BGNN_TRY(to_dev(ctx, db, b, n * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, dout, n * 4));
  BGNN_TRY(bgnn_add_dev(ctx, da.as<float>(), db.as<float>(), n, dout.as<float>()));
  return finish_host(ctx, out, dout.p, n * 4);
}

extern "C" int bgnn_spmv_host(bgnn_ctx* ctx, const uint32_t* row_ptr, const uint32_t* col,
                              const float* values, const float* x, uint32_t num_rows,
                              uint32_t num_cols, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, row_ptr && out, "NULL row_ptr/out");
  const uint64_t nnz = (uint64_t)row_ptr[num_rows];
  DevTmp drp, dcol, dval, dx, dout;
  BGNN_TRY(to_dev(ctx, drp, row_ptr, ((size_t)num_rows + 1) * 4));
  BGNN_TRY(to_dev(ctx, dcol, col, nnz * 4));
  BGNN_TRY(to_dev(ctx, dval, values, nnz * 4));
  BGNN_TRY(to_dev(ctx, dx, x, (size_t)num_cols * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, dout, (size_t)num_rows * 4));
  BGNN_TRY(bgnn_spmv_dev(ctx, drp.as<uint32_t>(), dcol.as<uint32_t>(), dval.as<float>(),
                         dx.as<float>(), num_rows, num_cols, dout.as<float>()));
  return finish_host(ctx, out, dout.p, (size_t)num_rows * 4);
}

extern "C" int bgnn_coo_to_csr_host(bgnn_ctx* ctx, const uint32_t* rows, const uint32_t* cols,
                                    const float* values, uint64_t nnz, uint32_t num_rows,
                                    uint32_t num_cols, uint32_t* row_ptr, uint32_t* col_out,
                                    float* val_out) {
  BGNN_TRY(ctx_ok(ctx));
  DevTmp dr, dc, dv, drp, dco, dvo;
  BGNN_TRY(to_dev(ctx, dr, rows, nnz * 4));
  BGNN_TRY(to_dev(ctx, dc, cols, nnz * 4));
  if (values) BGNN_TRY(to_dev(ctx, dv, values, nnz * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, drp, ((size_t)num_rows + 1) * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, dco, nnz * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, dvo, nnz * 4));
  BGNN_TRY(bgnn_coo_to_csr_dev(ctx, dr.as<uint32_t>(), dc.as<uint32_t>(),
                               values ? dv.as<float>() : nullptr, nnz, num_rows, num_cols,
                               drp.as<uint32_t>(), dco.as<uint32_t>(),
                               val_out ? dvo.as<float>() : nullptr));
  BGNN_CUDA(ctx, cudaMemcpyAsync(row_ptr, drp.p, ((size_t)num_rows + 1) * 4,
                                 cudaMemcpyDeviceToHost, ctx->stream));
  if (col_out && nnz)
    BGNN_CUDA(ctx, cudaMemcpyAsync(col_out, dco.p, nnz * 4, cudaMemcpyDeviceToHost, ctx->stream));
  if (val_out && nnz)
    BGNN_CUDA(ctx, cudaMemcpyAsync(val_out, dvo.p, nnz * 4, cudaMemcpyDeviceToHost, ctx->stream));
  return bgnn_check_device_error(ctx);
}

// ---- fused layer ops on graphs ----------------------------------------------
extern "C" int bgnn_aggregate(bgnn_ctx* ctx, const bgnn_graph* g, int aggr, const float* x,
                              uint32_t f, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, g != nullptr, "NULL graph");
  BGNN_REQUIRE(ctx, aggr >= BGNN_AGGR_SUM && aggr <= BGNN_AGGR_MAX, "unknown aggregation %d", aggr);
  BGNN_REQUIRE(ctx, (x && out) || (uint64_t)g->n_dst * f == 0, "NULL x/out");
  AggArgs a = graph_args(g, x, f, out);
  a.mean = aggr == BGNN_AGGR_MEAN;
  a.max_fix = aggr == BGNN_AGGR_MAX;
  return bgnn_run_aggregate(ctx, aggr == BGNN_AGGR_MAX ? OP_MAX : OP_SUM, a);
}

int bgnn_run_aggregate_cols(bgnn_ctx* ctx, const bgnn_graph* g, int aggr, const float* values,
                            const float* x, uint64_t ld_x, uint32_t width, float* out,
                            uint64_t ld_out) {
  AggArgs a = graph_args(g, x, width, out);
  a.ld_x = (int64_t)ld_x;
  a.ld_out = (int64_t)ld_out;
  if (aggr == BGNN_AGGR_SPMM) {
    a.val = values;
    a.exact = ctx->math == BGNN_MATH_EXACT;
    return bgnn_run_aggregate(ctx, OP_SPMM, a);
  }
  a.mean = aggr == BGNN_AGGR_MEAN;
  a.max_fix = aggr == BGNN_AGGR_MAX;
  return bgnn_run_aggregate(ctx, aggr == BGNN_AGGR_MAX ? OP_MAX : OP_SUM, a);
}

extern "C" int bgnn_aggregate_strided(bgnn_ctx* ctx, const bgnn_graph* g, int aggr,
                                      const float* values, const float* x, uint64_t ld_x,
                                      uint32_t width, float* out, uint64_t ld_out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, g != nullptr, "NULL graph");
  BGNN_REQUIRE(ctx, aggr >= BGNN_AGGR_SUM && aggr <= BGNN_AGGR_SPMM, "unknown aggregation %d",
               aggr);
  BGNN_REQUIRE(ctx, ld_x >= width && ld_out >= width, "row strides must cover the width");
  BGNN_REQUIRE(ctx, (x && out) || (uint64_t)g->n_dst * width == 0, "NULL x/out");
  BGNN_REQUIRE(ctx, aggr != BGNN_AGGR_SPMM || values || g->num_edges == 0, "NULL values");
  return bgnn_run_aggregate_cols(ctx, g, aggr, values, x, ld_x, width, out, ld_out);
}

extern "C" int bgnn_gcn_propagate(bgnn_ctx* ctx, const bgnn_graph* g, const float* h, uint32_t f,
                                  int add_self_loops, int normalize, const float* bias, int act,
                                  double act_param, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, g != nullptr, "NULL graph");
  BGNN_TRY(check_act(ctx, act));
  BGNN_REQUIRE(ctx, (h && out) || (uint64_t)g->n_dst * f == 0, "NULL h/out");
  // gcn.ts:90-92: loops are appended only when the graph has none at all
  const int tail = (add_self_loops && !g->has_self_loops) ? 1 : 0;
  BGNN_REQUIRE(ctx, !tail || g->n_src == g->n_dst, "self-loops need a square graph");
  AggArgs a = graph_args(g, h, f, out);
  a.tail = tail;
  a.bias = bias;
  a.act = act;
  a.act_param = act_param;
  if (normalize) {
    const float* dinv = nullptr;
    BGNN_TRY(bgnn_graph_dinv(ctx, const_cast<bgnn_graph*>(g), tail, &dinv));
    a.dinv = dinv;
    return bgnn_run_aggregate(ctx, OP_GCN, a);
  }
  return bgnn_run_aggregate(ctx, OP_SUM, a);
}

extern "C" int bgnn_gat(bgnn_ctx* ctx, const bgnn_graph* g, const float* h, uint32_t heads,
                        uint32_t c, const float* att_src, const float* att_dst,
                        double negative_slope, int concat, int add_self_loops, const float* bias,
                        int act, double act_param, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, g != nullptr, "NULL graph");
  BGNN_TRY(check_act(ctx, act));
  BGNN_REQUIRE(ctx, h && att_src && att_dst && out, "NULL argument");
  const int tail = (add_self_loops && !g->has_self_loops) ? 1 : 0;  // gat.ts:116-118
  return bgnn_run_gat(ctx, g, h, heads, c, att_src, att_dst, negative_slope, concat, tail, bias,
                      act, act_param, out);
}

extern "C" int bgnn_gat_train(bgnn_ctx* ctx, const bgnn_graph* g, const float* h, uint32_t heads,
                              uint32_t c, const float* att_src, const float* att_dst,
                              double negative_slope, int concat, int add_self_loops,
                              const float* bias, int act, double act_param, double dropout,
                              uint64_t seed, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, g != nullptr, "NULL graph");
  BGNN_TRY(check_act(ctx, act));
  BGNN_REQUIRE(ctx, h && att_src && att_dst && out, "NULL argument");
  BGNN_REQUIRE(ctx, dropout >= 0.0 && dropout < 1.0, "attention dropout must be in [0, 1)");
  const int tail = (add_self_loops && !g->has_self_loops) ? 1 : 0;
  return bgnn_run_gat(ctx, g, h, heads, c, att_src, att_dst, negative_slope, concat, tail, bias,
                      act, act_param, out, dropout, seed);
}

extern "C" int bgnn_gin_aggregate(bgnn_ctx* ctx, const bgnn_graph* g, const float* x, uint32_t f,
                                  float eps, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, g != nullptr, "NULL graph");
  BGNN_REQUIRE(ctx, g->n_src == g->n_dst, "GIN needs a square graph");
  BGNN_REQUIRE(ctx, (x && out) || (uint64_t)g->n_dst * f == 0, "NULL x/out");
  AggArgs a = graph_args(g, x, f, out);
  a.gin_x = x;
  a.ld_gin = f;
  a.gin_ope = 1.0 + (double)eps;  // JS: (1 + eps) with eps read from a Float32Array
  return bgnn_run_aggregate(ctx, OP_SUM, a);
}

extern "C" int bgnn_graph_spmm(bgnn_ctx* ctx, const bgnn_graph* g, const float* values,
                               const float* x, uint32_t f, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, g != nullptr, "NULL graph");
  BGNN_REQUIRE(ctx, (values && x && out) || (uint64_t)g->n_dst * f == 0 || g->num_edges == 0,
               "NULL argument");
  AggArgs a = graph_args(g, x, f, out);
  a.val = values;
  a.exact = ctx->math == BGNN_MATH_EXACT;
  return bgnn_run_aggregate(ctx, OP_SPMM, a);
}

extern "C" int bgnn_linear(bgnn_ctx* ctx, const float* a, const float* w, uint32_t m, uint32_t k,
                           uint32_t n, const float* bias, int act, double act_param, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_TRY(check_act(ctx, act));
  BGNN_REQUIRE(ctx, (a && w) || (uint64_t)m * k * n == 0, "NULL operand");
  BGNN_REQUIRE(ctx, out || (uint64_t)m * n == 0, "NULL out");
  return bgnn_run_linear(ctx, a, w, nullptr, nullptr, m, k, n, bias, act, act_param, out);
}

extern "C" int bgnn_sage_linear(bgnn_ctx* ctx, const float* agg, const float* x,
                                const float* w_neigh, const float* w_self, uint32_t m, uint32_t k,
                                uint32_t n, const float* bias, int act, double act_param,
                                float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_TRY(check_act(ctx, act));
  BGNN_REQUIRE(ctx, (agg && w_neigh) || (uint64_t)m * k * n == 0, "NULL operand");
  BGNN_REQUIRE(ctx, !w_self || x, "w_self without x");
  BGNN_REQUIRE(ctx, out || (uint64_t)m * n == 0, "NULL out");
  return bgnn_run_linear(ctx, agg, w_neigh, w_self ? x : nullptr, w_self, m, k, n, bias, act,
                         act_param, out);
}

extern "C" int bgnn_linear_add(bgnn_ctx* ctx, const float* a, const float* w, uint32_t m,
                               uint32_t k, uint32_t n, const float* addend, const float* bias,
                               int act, double act_param, float* out) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_TRY(check_act(ctx, act));
  BGNN_REQUIRE(ctx, (a && w) || (uint64_t)m * k * n == 0, "NULL operand");
  BGNN_REQUIRE(ctx, (addend && out) || (uint64_t)m * n == 0, "NULL addend/out");
  return bgnn_run_linear_add(ctx, a, w, m, k, n, addend, bias, act, act_param, out);
}


extern "C" int bgnn_l2_normalize_rows(bgnn_ctx* ctx, float* x, uint32_t m, uint32_t n) {
  BGNN_TRY(ctx_ok(ctx));
  BGNN_REQUIRE(ctx, x || (uint64_t)m * n == 0, "NULL x");
  return bgnn_run_l2norm(ctx, x, m, n);
}

extern "C" int bgnn_sum_pool(bgnn_ctx* ctx, const float* x, uint32_t num_nodes, uint32_t f,
                             const uint32_t* batch, uint32_t num_graphs, float* out) {
  // g[b,:] = sum of x[i,:] over batch[i] == b, in node order: a scatter-add
  // of the node rows keyed by the batch vector
  return bgnn_scatter_dev(ctx, BGNN_AGGR_SUM, x, batch, num_nodes, num_graphs, f, out);
}
