// Backward of the message passing and of X*W.
//
// The reference's autograd differentiates X*W (Variable.matmul,
// src/autograd/variable.ts:213-235: grad @ B^T and A^T @ grad through
// Tensor.transpose and wasmMatmul), ReLU (variable.ts:358-373) and the
// broadcast bias add (variable.ts:665-688), but never the message passing.
// The message-passing adjoint here is what it would compute if gather and
// scatter were autograd ops: edge e carries a message from grad[dst(e)] and
// the messages are scatter-added over the sources in COO edge order, an f32
// store after every add (wasmScatterAdd, src/backend/wasm/index.ts:70-105).
//
// The scatter over sources in edge order is an aggregation over the
// transposed graph (rows = sources, each row's edges in COO order), so the
// sum, mean and GCN adjoints run the forward's streaming aggregation on a
// transpose built once per graph; mean pre-scales the gradient rows
// (f32(grad * (1/cnt)), 1/cnt in double, a function of the destination
// only); max routes each (destination, feature) gradient to the edge that
// last raised the forward maximum, recorded by replaying the forward.
#include <cstring>

#include "bgnn_internal.cuh"

namespace {

inline unsigned grid_for(bgnn_ctx* ctx, uint64_t n, int tpb) {
  uint64_t b = (n + tpb - 1) / tpb;
  const uint64_t cap = (uint64_t)ctx->num_sms * 16;
  if (b > cap) b = cap;
  if (b == 0) b = 1;
  return (unsigned)b;
}

// the COO edge list back from the CSR: src and dst of edge eid[j]
__global__ void k_coo_from_csr(const uint32_t* __restrict__ src_of,
                               const uint32_t* __restrict__ dst_of,
                               const uint32_t* __restrict__ eid, uint64_t E,
                               uint32_t* __restrict__ coo_src, uint32_t* __restrict__ coo_dst) {
  for (uint64_t j = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; j < E;
       j += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t e = eid[j];
    coo_src[e] = src_of[j];
    coo_dst[e] = dst_of[j];
  }
}

// mean adjoint: the message of every edge into d is f32(grad[d] * (1/cnt(d)))
__global__ void k_scale_rows_by_inv_count(const float* __restrict__ g,
                                          const uint32_t* __restrict__ rp, uint32_t n,
                                          uint32_t f, float* __restrict__ out) {
  const uint64_t total = (uint64_t)n * f;
  for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t d = (uint32_t)(t / f);
    const uint32_t c = rp[d + 1] - rp[d];
    out[t] = c ? __double2float_rn(__dmul_rn((double)g[t], __ddiv_rn(1.0, (double)c))) : 0.0f;
  }
}

// max: for every (destination row, feature) the COO id of the edge that
// last raised the running maximum (x > acc in edge order from -inf), or
// ~0 when none did.  Warp per row, lanes over features.
__global__ void k_argmax(const uint32_t* __restrict__ rp, const uint32_t* __restrict__ src_of,
                         const uint32_t* __restrict__ eid, uint32_t n, const float* __restrict__ x,
                         uint32_t f, uint32_t* __restrict__ arg) {
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
  for (uint32_t r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < n; r += warps) {
    const uint32_t b = rp[r], en = rp[r + 1];
    for (uint32_t c0 = 0; c0 < f; c0 += 32) {
      const uint32_t c = c0 + lane;
      float acc = -INFINITY;
      uint32_t best = 0xffffffffu;
      for (uint32_t j = b; j < en; j++) {
        const uint32_t s = src_of[j];
        const float v = c < f ? __ldg(x + (uint64_t)s * f + c) : 0.0f;
        if (v > acc) {
          acc = v;
          best = eid[j];
        }
      }
      if (c < f) arg[(uint64_t)r * f + c] = best;
    }
  }
}

// max adjoint over the transpose: out[s, c] = edge-ordered sum of grad[d, c]
// over the edges (s -> d) that supplied d's maximum of feature c.  Adding the
// +0 messages of the other edges changes nothing (the running sum is never
// -0), so they are skipped.  Warp per source row, lanes over features.
__global__ void k_max_backward(const uint32_t* __restrict__ trp, const uint32_t* __restrict__ tdst,
                               const uint32_t* __restrict__ teid, uint32_t n_src,
                               const uint32_t* __restrict__ arg, const float* __restrict__ g,
                               uint32_t f, float* __restrict__ out) {
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
  for (uint32_t s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; s < n_src; s += warps) {
    const uint32_t b = trp[s], en = trp[s + 1];
    for (uint32_t c0 = 0; c0 < f; c0 += 32) {
      const uint32_t c = c0 + lane;
      float acc = 0.0f;
      if (c < f) {
        for (uint32_t j = b; j < en; j++) {
          const uint32_t d = tdst[j];
          const uint64_t at = (uint64_t)d * f + c;
          if (__ldg(arg + at) == teid[j]) acc = __fadd_rn(acc, __ldg(g + at));
        }
        out[(uint64_t)s * f + c] = acc;
      }
    }
  }
}

// C[i, j] = sum_r A[r, i] * B[r, j], r ascending, one chain per output (the
// k-ascending wasmMatmul order of transpose(A) @ B).  ones: A is a column of
// ones (the bias reduction of variable.ts:675-685), n_a must be 1.
// 16 x 16 outputs per CTA, rows streamed through shared memory 64 at a time.
template <bool EXACT>
__global__ void __launch_bounds__(256) k_matmul_tn(const float* __restrict__ A,
                                                  const float* __restrict__ B, uint64_t m,
                                                  uint32_t n_a, uint32_t n_b, int ones,
                                                  float* __restrict__ C) {
  __shared__ float sa[64][17];
  __shared__ float sb[64][17];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const uint32_t i0 = blockIdx.x * 16, j0 = blockIdx.y * 16;
  float acc = 0.0f;
  for (uint64_t r0 = 0; r0 < m; r0 += 64) {
    for (int q = threadIdx.x; q < 64 * 16; q += 256) {
      const int rr = q >> 4, cc = q & 15;
      const uint64_t r = r0 + rr;
      const uint32_t ia = i0 + cc, jb = j0 + cc;
      sa[rr][cc] = (r < m && ia < n_a) ? (ones ? 1.0f : A[r * n_a + ia]) : 0.0f;
      sb[rr][cc] = (r < m && jb < n_b) ? B[r * n_b + jb] : 0.0f;
    }
    __syncthreads();
    const int cnt = (int)(m - r0 < 64 ? m - r0 : 64);
    for (int rr = 0; rr < cnt; rr++) {
      if (EXACT)
        acc = __double2float_rn(__fma_rn((double)sa[rr][ty], (double)sb[rr][tx], (double)acc));
      else
        acc = __fmaf_rn(sa[rr][ty], sb[rr][tx], acc);
    }
    __syncthreads();
  }
  const uint32_t i = i0 + ty, j = j0 + tx;
  if (i < n_a && j < n_b) C[(uint64_t)i * n_b + j] = acc;
}

__global__ void k_transpose(const float* __restrict__ a, uint64_t rows, uint32_t cols,
                            float* __restrict__ t) {
  const uint64_t total = rows * cols;
  for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < total;
       q += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t i = q / cols;
    const uint32_t j = (uint32_t)(q - i * cols);
    t[(uint64_t)j * rows + i] = a[q];
  }
}

AggArgs graph_args_t(const bgnn_graph* g, const float* x, uint32_t f, float* out) {
  AggArgs a;
  memset(&a, 0, sizeof(a));
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

__global__ void k_relu_mask(const float* __restrict__ g, const float* __restrict__ y, uint64_t n,
                            float* __restrict__ out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = y[i] > 0.0f ? g[i] : 0.0f;
}

int run_tn(bgnn_ctx* ctx, const float* a, const float* b, uint64_t m, uint32_t n_a, uint32_t n_b,
           int ones, float* out) {
  if (n_a == 0 || n_b == 0) return BGNN_OK;
  dim3 grid((n_a + 15) / 16, (n_b + 15) / 16);
  if (ctx->math == BGNN_MATH_EXACT)
    k_matmul_tn<true><<<grid, 256, 0, ctx->stream>>>(a, b, m, n_a, n_b, ones, out);
  else
    k_matmul_tn<false><<<grid, 256, 0, ctx->stream>>>(a, b, m, n_a, n_b, ones, out);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

}  // namespace

// The transpose of a graph (rows = sources, each row's edges in COO order,
// columns = destinations), built on first use and kept with the graph.
int bgnn_graph_transpose(bgnn_ctx* ctx, bgnn_graph* g, const bgnn_graph** out) {
  if (g->transpose) {
    *out = g->transpose;
    return BGNN_OK;
  }
  if (g->csr_only || !g->eid || !g->out_deg)
    return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED,
                          "the backward needs a graph built from an edge list");
  const uint64_t E = g->num_edges;
  const uint32_t* dst_of = nullptr;
  BGNN_TRY(bgnn_graph_dst_of(ctx, g, &dst_of));
  bgnn_graph* t = new bgnn_graph();
  uint32_t* trp = nullptr;
  uint32_t* tdst = nullptr;
  int rc = BGNN_OK;
  do {
    DevTmp csrc, cdst;
    if ((rc = bgnn_tmp_alloc(ctx, csrc, (E ? E : 1) * 4)) != BGNN_OK) break;
    if ((rc = bgnn_tmp_alloc(ctx, cdst, (E ? E : 1) * 4)) != BGNN_OK) break;
    if (cudaMalloc(&trp, ((size_t)g->n_src + 1) * 4) != cudaSuccess ||
        cudaMalloc(&tdst, (E ? E : 1) * 4) != cudaSuccess ||
        cudaMalloc(&t->eid, (E ? E : 1) * 4) != cudaSuccess) {
      cudaGetLastError();
      rc = bgnn_set_error(ctx, BGNN_ERR_NO_MEMORY, "transpose allocation failed");
      break;
    }
    if (E) {
      k_coo_from_csr<<<grid_for(ctx, E, 256), 256, 0, ctx->stream>>>(
          g->src_of, dst_of, g->eid, E, csrc.as<uint32_t>(), cdst.as<uint32_t>());
      if (cudaGetLastError() != cudaSuccess) {
        rc = bgnn_set_error(ctx, BGNN_ERR_CUDA, "transpose kernel launch failed");
        break;
      }
      ctx->launches++;
    }
    // stable by source: each row keeps its edges in COO order
    const int bits = g->n_src > 1 ? bgnn_bits_for(g->n_src - 1) : 0;
    if ((rc = bgnn_radix_sort(ctx, csrc.as<uint32_t>(), E, bits, nullptr, 1, cdst.as<uint32_t>(),
                              nullptr, t->eid, tdst)) != BGNN_OK)
      break;
    // row offsets: the out-degrees (one spare zero entry) scanned
    if (cudaMemcpyAsync(trp, g->out_deg, ((size_t)g->n_src + 1) * 4, cudaMemcpyDeviceToDevice,
                        ctx->stream) != cudaSuccess) {
      rc = bgnn_set_error(ctx, BGNN_ERR_CUDA, "transpose copy failed");
      break;
    }
    if ((rc = bgnn_exclusive_scan(ctx, trp, trp, (uint64_t)g->n_src + 1)) != BGNN_OK) break;
    rc = bgnn_graph_adopt_csr(ctx, trp, tdst, g->n_src, g->n_dst, E, t);
    trp = tdst = nullptr;  // owned by t now (freed with it on failure)
  } while (false);
  if (rc != BGNN_OK) {
    cudaFree(trp);
    cudaFree(tdst);
    bgnn_graph_free(t);
    delete t;
    return rc;
  }
  t->csr_only = false;  // keeps eid (the COO id of each slot)
  t->has_self_loops = g->has_self_loops;
  g->transpose = t;
  *out = t;
  return BGNN_OK;
}

extern "C" int bgnn_aggregate_backward(bgnn_ctx* ctx, const bgnn_graph* g, int aggr,
                                       const float* x, const float* grad,
                                       uint32_t num_features, float* out) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  BGNN_REQUIRE(ctx, g != nullptr, "NULL graph");
  BGNN_REQUIRE(ctx, aggr >= BGNN_AGGR_SUM && aggr <= BGNN_AGGR_MAX, "unknown aggregation %d", aggr);
  const uint32_t f = num_features;
  BGNN_REQUIRE(ctx, (grad && out) || (uint64_t)g->n_src * f == 0, "NULL grad/out");
  BGNN_REQUIRE(ctx, aggr != BGNN_AGGR_MAX || x || (uint64_t)g->n_src * f == 0,
               "max needs the forward input x");
  if ((uint64_t)g->n_src * f == 0) return BGNN_OK;
  const bgnn_graph* t = nullptr;
  BGNN_TRY(bgnn_graph_transpose(ctx, const_cast<bgnn_graph*>(g), &t));
  if (aggr == BGNN_AGGR_MAX) {
    DevTmp arg;
    BGNN_TRY(bgnn_tmp_alloc(ctx, arg, ((uint64_t)g->n_dst * f + 1) * 4));
    if (g->n_dst) {
      k_argmax<<<grid_for(ctx, (uint64_t)g->n_dst * 32, 256), 256, 0, ctx->stream>>>(
          g->row_ptr, g->src_of, g->eid, g->n_dst, x, f, arg.as<uint32_t>());
      BGNN_LAUNCHED(ctx);
    }
    k_max_backward<<<grid_for(ctx, (uint64_t)g->n_src * 32, 256), 256, 0, ctx->stream>>>(
        t->row_ptr, t->src_of, t->eid, g->n_src, arg.as<uint32_t>(), grad, f, out);
    BGNN_LAUNCHED(ctx);
    return BGNN_OK;
  }
  const float* msg = grad;
  DevTmp scaled;
  if (aggr == BGNN_AGGR_MEAN) {
    BGNN_TRY(bgnn_tmp_alloc(ctx, scaled, ((uint64_t)g->n_dst * f + 1) * 4));
    k_scale_rows_by_inv_count<<<grid_for(ctx, (uint64_t)g->n_dst * f, 256), 256, 0,
                                ctx->stream>>>(grad, g->row_ptr, g->n_dst, f,
                                               scaled.as<float>());
    BGNN_LAUNCHED(ctx);
    msg = scaled.as<float>();
  }
  AggArgs a = graph_args_t(t, msg, f, out);
  return bgnn_run_aggregate(ctx, OP_SUM, a);
}

extern "C" int bgnn_gcn_propagate_backward(bgnn_ctx* ctx, const bgnn_graph* g, const float* grad,
                                           uint32_t num_features, int add_self_loops,
                                           int normalize, float* out) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  BGNN_REQUIRE(ctx, g != nullptr, "NULL graph");
  const uint32_t f = num_features;
  BGNN_REQUIRE(ctx, (grad && out) || (uint64_t)g->n_src * f == 0, "NULL grad/out");
  if ((uint64_t)g->n_src * f == 0) return BGNN_OK;
  const int tail = (add_self_loops && !g->has_self_loops) ? 1 : 0;  // gcn.ts:90-92
  BGNN_REQUIRE(ctx, !tail || g->n_src == g->n_dst, "self-loops need a square graph");
  const bgnn_graph* t = nullptr;
  BGNN_TRY(bgnn_graph_transpose(ctx, const_cast<bgnn_graph*>(g), &t));
  AggArgs a = graph_args_t(t, grad, f, out);
  a.tail = tail;
  if (normalize) {
    // the forward's D^-1/2 (in-degrees of g, + 1 with the appended loops);
    // f32(dinv[d] * dinv[s]) is the forward's f32(dinv[s] * dinv[d])
    const float* dinv = nullptr;
    BGNN_TRY(bgnn_graph_dinv(ctx, const_cast<bgnn_graph*>(g), tail, &dinv));
    a.dinv = dinv;
    return bgnn_run_aggregate(ctx, OP_GCN, a);
  }
  return bgnn_run_aggregate(ctx, OP_SUM, a);
}

extern "C" int bgnn_matmul_backward(bgnn_ctx* ctx, const float* a, const float* b,
                                    const float* grad, uint32_t m, uint32_t k, uint32_t n,
                                    float* grad_a, float* grad_b) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  BGNN_REQUIRE(ctx, grad || (uint64_t)m * n == 0, "NULL grad");
  if (grad_a && (uint64_t)m * k) {
    BGNN_REQUIRE(ctx, b != nullptr, "grad_a needs b");
    // grad @ transpose(b): b^T [n, k] then the k-ascending product
    DevTmp bt;
    BGNN_TRY(bgnn_tmp_alloc(ctx, bt, ((uint64_t)k * n + 1) * 4));
    if ((uint64_t)k * n) {
      k_transpose<<<grid_for(ctx, (uint64_t)k * n, 256), 256, 0, ctx->stream>>>(b, k, n,
                                                                                bt.as<float>());
      BGNN_LAUNCHED(ctx);
    }
    BGNN_TRY(bgnn_run_linear(ctx, grad, bt.as<float>(), nullptr, nullptr, m, n, k, nullptr,
                             BGNN_ACT_NONE, 0.0, grad_a));
  }
  if (grad_b && (uint64_t)k * n) {
    BGNN_REQUIRE(ctx, a != nullptr, "grad_b needs a");
    BGNN_TRY(run_tn(ctx, a, grad, m, k, n, 0, grad_b));
  }
  return BGNN_OK;
}

extern "C" int bgnn_bias_backward(bgnn_ctx* ctx, const float* grad, uint64_t rows, uint32_t cols,
                                  float* out) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  BGNN_REQUIRE(ctx, (grad && out) || cols == 0, "NULL argument");
  if (cols == 0) return BGNN_OK;
  return run_tn(ctx, nullptr, grad, rows, 1, cols, 1, out);
}

extern "C" int bgnn_relu_backward(bgnn_ctx* ctx, const float* grad, const float* out, uint64_t n,
                                  float* grad_in) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  BGNN_REQUIRE(ctx, (grad && out && grad_in) || n == 0, "NULL argument");
  if (n == 0) return BGNN_OK;
  // variable.ts:358-373: the input gradient where the input was > 0, which
  // for ReLU is where its output is > 0
  k_relu_mask<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(grad, out, n, grad_in);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}
