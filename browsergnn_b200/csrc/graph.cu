// Graph construction on the device: index validation, degrees, self-loop
// detection, the stable destination-keyed CSR, SparseCSR.fromCOO and
// computeGCNNorm.
//
// Reference semantics followed here:
//   GraphData ctor bounds check        src/core/graph.ts:88-92
//   getInDegrees / getOutDegrees       src/core/graph.ts:172-195
//   hasSelfLoops                       src/core/graph.ts:220-227
//   SparseCSR.fromCOO (stable sort)    src/core/sparse.ts:259-296
//   computeGCNNorm                     src/core/sparse.ts:480-513
#include <algorithm>
#include <vector>

#include "bgnn_internal.cuh"

namespace {

constexpr unsigned FULL = 0xffffffffu;

inline unsigned grid_for(bgnn_ctx* ctx, uint64_t n, int tpb) {
  uint64_t b = (n + tpb - 1) / tpb;
  const uint64_t cap = (uint64_t)ctx->num_sms * 16;
  if (b > cap) b = cap;
  if (b == 0) b = 1;
  return (unsigned)b;
}

// warp-aggregated increment: lanes hitting the same counter add once
__device__ __forceinline__ void agg_inc(uint32_t* base, uint32_t idx, bool active) {
  const unsigned act = __ballot_sync(FULL, active);
  if (!active) return;
  const unsigned peers = __match_any_sync(act, idx);
  if ((threadIdx.x & 31) == (unsigned)(__ffs(peers) - 1)) atomicAdd(&base[idx], (uint32_t)__popc(peers));
}

// Count degrees and detect self-loops; record the first out-of-range position
// in the reference's flat [src | dst] order.
__global__ void k_count_validate(const uint32_t* __restrict__ src, const uint32_t* __restrict__ dst,
                                 uint64_t E, uint32_t n_src, uint32_t n_dst,
                                 uint32_t* __restrict__ in_deg, uint32_t* __restrict__ out_deg,
                                 int check_loops, uint32_t* __restrict__ flags,
                                 unsigned long long* __restrict__ first_bad) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t start = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  // uniform trip count per warp so the warp-collective increments stay converged
  const uint64_t warp0 = start - (threadIdx.x & 31);
  for (uint64_t wb = warp0; wb < E; wb += stride) {
    const uint64_t e = wb + (threadIdx.x & 31);
    const bool in = e < E;
    const uint32_t s = in ? src[e] : 0u;
    const uint32_t d = in ? dst[e] : 0u;
    const bool sb = in && s >= n_src;
    const bool db = in && d >= n_dst;
    if (sb) atomicMin(first_bad, (unsigned long long)e);
    if (db) atomicMin(first_bad, (unsigned long long)(E + e));
    const bool ok = in && !sb && !db;
    agg_inc(in_deg, d, ok);
    if (out_deg) agg_inc(out_deg, s, ok);
    if (check_loops && ok && s == d) flags[0] = 1u;
  }
}

// D^-1/2 from the CSR degree: the reference counts degrees in a Float32Array
// (+1 per edge, saturating at 2^24) and stores f32(1/Math.sqrt(deg)).
__global__ void k_dinv_from_rowptr(const uint32_t* __restrict__ row_ptr, uint32_t n, int tail,
                                   float* __restrict__ dinv) {
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < n; r += gridDim.x * blockDim.x) {
    const uint32_t d = row_ptr[r + 1] - row_ptr[r] + (tail ? 1u : 0u);
    const float deg = d >= 16777216u ? 16777216.0f : (float)d;
    dinv[r] = deg > 0.0f ? __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn((double)deg))) : 0.0f;
  }
}

__global__ void k_dinv_from_deg(const uint32_t* __restrict__ deg_u, uint32_t n, int loops,
                                float* __restrict__ dinv) {
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < n; r += gridDim.x * blockDim.x) {
    const uint32_t d = deg_u[r] + (loops ? 1u : 0u);
    const float deg = d >= 16777216u ? 16777216.0f : (float)d;
    dinv[r] = deg > 0.0f ? __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn((double)deg))) : 0.0f;
  }
}

__global__ void k_edge_norm(const uint32_t* __restrict__ ei, uint64_t E,
                            const float* __restrict__ dinv, float* __restrict__ out) {
  for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < E;
       e += (uint64_t)gridDim.x * blockDim.x)
    out[e] = __fmul_rn(dinv[ei[e]], dinv[ei[E + e]]);
}

__global__ void k_validate_cols(const uint32_t* __restrict__ col, uint64_t nnz, uint32_t bound,
                                unsigned long long* __restrict__ first_bad) {
  for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nnz;
       e += (uint64_t)gridDim.x * blockDim.x)
    if (col[e] >= bound) atomicMin(first_bad, (unsigned long long)e);
}

// a caller-supplied CSR must be non-decreasing or the row loops would read
// outside col[]; record the first offending row
__global__ void k_validate_rowptr(const uint32_t* __restrict__ rp, uint32_t n,
                                  unsigned long long* __restrict__ first_bad) {
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < n; r += gridDim.x * blockDim.x)
    if (rp[r + 1] < rp[r]) atomicMin(first_bad, (unsigned long long)r);
}

__global__ void k_fill_ones(float* out, uint64_t n) {
  for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (uint64_t)gridDim.x * blockDim.x)
    out[e] = 1.0f;
}

// row_ptr[r] = number of entries with row < r, from a zeroed histogram
int counts_to_rowptr(bgnn_ctx* ctx, uint32_t* counts_then_rowptr, uint32_t n_rows) {
  // counts has n_rows+1 entries with the last one zero; scanning gives E at the end
  return bgnn_exclusive_scan(ctx, counts_then_rowptr, counts_then_rowptr, (uint64_t)n_rows + 1);
}

// Row schedule, built once per graph on the host from a copy of row_ptr:
//  * heavy rows (degree >= 256), largest first, for the CTA-per-row kernel;
//  * streaming work items: every heavy row alone (largest first), then runs
//    of consecutive light rows holding up to kItemEdges edges and
//    kItemRows rows.  Items never split a row, so each row is still reduced
//    by one pipe in edge order.
constexpr uint32_t kHeavyThreshold = 256;
constexpr uint32_t kItemEdges = 1024;
constexpr uint32_t kItemRows = 256;  // must equal the streaming kernel's row buffer

int build_schedule(bgnn_ctx* ctx, bgnn_graph* g) {
  g->heavy_threshold = kHeavyThreshold;
  g->n_heavy = 0;
  g->n_items = 0;
  g->n_heavy_items = 0;
  g->heavy_deg.clear();
  const uint32_t n = g->n_dst;
  if (n == 0) return BGNN_OK;
  std::vector<uint32_t> rp((size_t)n + 1);
  BGNN_CUDA(ctx, cudaMemcpyAsync(rp.data(), g->row_ptr, ((size_t)n + 1) * 4,
                                 cudaMemcpyDeviceToHost, ctx->stream));
  BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  std::vector<uint32_t> heavy;
  for (uint32_t r = 0; r < n; r++)
    if (rp[r + 1] - rp[r] >= kHeavyThreshold) heavy.push_back(r);
  std::sort(heavy.begin(), heavy.end(), [&](uint32_t a, uint32_t b) {
    const uint32_t da = rp[a + 1] - rp[a], db = rp[b + 1] - rp[b];
    return da != db ? da > db : a < b;
  });
  std::vector<uint2> items;
  items.reserve(heavy.size() + n / 64 + 16);
  for (uint32_t r : heavy) items.push_back(make_uint2(r, r + 1));
  uint32_t begin = 0, edges = 0;
  bool open = false;
  for (uint32_t r = 0; r < n; r++) {
    const uint32_t d = rp[r + 1] - rp[r];
    if (d >= kHeavyThreshold) {
      if (open) items.push_back(make_uint2(begin, r));
      open = false;
      continue;
    }
    if (!open) {
      begin = r;
      edges = 0;
      open = true;
    }
    edges += d;
    if (edges >= kItemEdges || r + 1 - begin >= kItemRows) {
      items.push_back(make_uint2(begin, r + 1));
      open = false;
    }
  }
  if (open) items.push_back(make_uint2(begin, n));
  if (!heavy.empty()) {
    BGNN_CUDA(ctx, cudaMalloc(&g->heavy_rows, heavy.size() * 4));
    BGNN_CUDA(ctx, cudaMemcpy(g->heavy_rows, heavy.data(), heavy.size() * 4,
                              cudaMemcpyHostToDevice));
    g->n_heavy = (uint32_t)heavy.size();
  }
  BGNN_CUDA(ctx, cudaMalloc(&g->items, items.size() * sizeof(uint2)));
  BGNN_CUDA(ctx, cudaMemcpy(g->items, items.data(), items.size() * sizeof(uint2),
                            cudaMemcpyHostToDevice));
  g->n_items = (uint32_t)items.size();
  g->n_heavy_items = (uint32_t)heavy.size();
  g->heavy_deg.resize(heavy.size());
  for (size_t i = 0; i < heavy.size(); i++) g->heavy_deg[i] = rp[heavy[i] + 1] - rp[heavy[i]];
  return BGNN_OK;
}

}  // namespace

void bgnn_graph_free(bgnn_graph* g) {
  if (!g) return;
  cudaFree(g->row_ptr);
  cudaFree(g->src_of);
  cudaFree(g->eid);
  cudaFree(g->out_deg);
  cudaFree(g->heavy_rows);
  cudaFree(g->items);
  cudaFree(g->dinv[0]);
  cudaFree(g->dinv[1]);
  cudaFree(g->dst_of);
  if (g->transpose) {
    bgnn_graph_free(g->transpose);
    delete g->transpose;
  }
  *g = bgnn_graph();
}

int bgnn_graph_build(bgnn_ctx* ctx, const uint32_t* src, const uint32_t* dst, uint64_t E,
                     uint32_t n_src, uint32_t n_dst, bgnn_graph* g) {
  if (E >= 0xffffffffull)
    return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED, "edge count %llu exceeds 2^32-2",
                          (unsigned long long)E);
  g->device = ctx->device;
  g->n_src = n_src;
  g->n_dst = n_dst;
  g->num_edges = E;
  BGNN_CUDA(ctx, cudaMalloc(&g->row_ptr, ((size_t)n_dst + 1) * 4));
  BGNN_CUDA(ctx, cudaMalloc(&g->out_deg, ((size_t)n_src + 1) * 4));
  BGNN_CUDA(ctx, cudaMalloc(&g->src_of, (size_t)(E ? E : 1) * 4));
  BGNN_CUDA(ctx, cudaMalloc(&g->eid, (size_t)(E ? E : 1) * 4));
  BGNN_CUDA(ctx, cudaMemsetAsync(g->row_ptr, 0, ((size_t)n_dst + 1) * 4, ctx->stream));
  BGNN_CUDA(ctx, cudaMemsetAsync(g->out_deg, 0, ((size_t)n_src + 1) * 4, ctx->stream));
  DevTmp flagbuf;
  BGNN_TRY(bgnn_tmp_alloc(ctx, flagbuf, 16));
  BGNN_CUDA(ctx, cudaMemsetAsync(flagbuf.p, 0, 4, ctx->stream));
  BGNN_CUDA(ctx, cudaMemsetAsync((char*)flagbuf.p + 8, 0xff, 8, ctx->stream));
  uint32_t* flags = flagbuf.as<uint32_t>();
  unsigned long long* first_bad = reinterpret_cast<unsigned long long*>((char*)flagbuf.p + 8);
  if (E) {
    k_count_validate<<<grid_for(ctx, E, 256), 256, 0, ctx->stream>>>(
        src, dst, E, n_src, n_dst, g->row_ptr, g->out_deg, n_src == n_dst, flags, first_bad);
    BGNN_LAUNCHED(ctx);
  }
  unsigned long long hbuf[2] = {0, 0};
  BGNN_CUDA(ctx, cudaMemcpyAsync(hbuf, flagbuf.p, 16, cudaMemcpyDeviceToHost, ctx->stream));
  BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if (hbuf[1] != ~0ull) {
    const unsigned long long pos = hbuf[1];
    uint32_t val = 0;
    const uint32_t* where = pos < E ? src + pos : dst + (pos - E);
    cudaMemcpy(&val, where, 4, cudaMemcpyDeviceToHost);
    return bgnn_set_error(ctx, BGNN_ERR_OUT_OF_RANGE,
                          "Edge index %u out of bounds for %u nodes (position %llu)", val,
                          pos < E ? n_src : n_dst, pos);
  }
  g->has_self_loops = (int)(hbuf[0] & 0xffffffffull) != 0;
  BGNN_TRY(counts_to_rowptr(ctx, g->row_ptr, n_dst));
  // stable sort by destination carrying each edge's id and source: every row
  // keeps its edges in COO order
  const int bits = n_dst > 1 ? bgnn_bits_for(n_dst - 1) : 0;
  BGNN_TRY(bgnn_radix_sort(ctx, dst, E, bits, nullptr, 1, src, nullptr, g->eid, g->src_of));
  BGNN_TRY(build_schedule(ctx, g));
  return BGNN_OK;
}

int bgnn_graph_from_csr(bgnn_ctx* ctx, const uint32_t* row_ptr, const uint32_t* col,
                        uint32_t num_rows, uint32_t num_cols, bgnn_graph* g, bool /*copy*/) {
  uint32_t nnz = 0;
  BGNN_CUDA(ctx, cudaMemcpyAsync(&nnz, row_ptr + num_rows, 4, cudaMemcpyDeviceToHost, ctx->stream));
  BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  g->device = ctx->device;
  g->n_src = num_cols;
  g->n_dst = num_rows;
  g->num_edges = nnz;
  g->csr_only = true;
  BGNN_CUDA(ctx, cudaMalloc(&g->row_ptr, ((size_t)num_rows + 1) * 4));
  BGNN_CUDA(ctx, cudaMalloc(&g->src_of, (size_t)(nnz ? nnz : 1) * 4));
  BGNN_CUDA(ctx, cudaMemcpyAsync(g->row_ptr, row_ptr, ((size_t)num_rows + 1) * 4,
                                 cudaMemcpyDeviceToDevice, ctx->stream));
  if (nnz)
    BGNN_CUDA(ctx, cudaMemcpyAsync(g->src_of, col, (size_t)nnz * 4, cudaMemcpyDeviceToDevice,
                                   ctx->stream));
  DevTmp bad;
  BGNN_TRY(bgnn_tmp_alloc(ctx, bad, 16));
  BGNN_CUDA(ctx, cudaMemsetAsync(bad.p, 0xff, 16, ctx->stream));
  unsigned long long* bad_col = bad.as<unsigned long long>();
  unsigned long long* bad_row = bad_col + 1;
  if (num_rows) {
    k_validate_rowptr<<<grid_for(ctx, num_rows, 256), 256, 0, ctx->stream>>>(g->row_ptr, num_rows,
                                                                            bad_row);
    BGNN_LAUNCHED(ctx);
  }
  if (nnz) {
    k_validate_cols<<<grid_for(ctx, nnz, 256), 256, 0, ctx->stream>>>(g->src_of, nnz, num_cols,
                                                                      bad_col);
    BGNN_LAUNCHED(ctx);
  }
  unsigned long long hb[2] = {0, 0};
  BGNN_CUDA(ctx, cudaMemcpyAsync(hb, bad.p, 16, cudaMemcpyDeviceToHost, ctx->stream));
  BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if (hb[1] != ~0ull)
    return bgnn_set_error(ctx, BGNN_ERR_INVALID_ARG, "row_ptr decreases at row %llu", hb[1]);
  if (hb[0] != ~0ull)
    return bgnn_set_error(ctx, BGNN_ERR_OUT_OF_RANGE,
                          "column index out of bounds for %u columns (position %llu)", num_cols,
                          hb[0]);
  BGNN_TRY(build_schedule(ctx, g));
  return BGNN_OK;
}

int bgnn_graph_adopt_csr(bgnn_ctx* ctx, uint32_t* row_ptr, uint32_t* col, uint32_t n_rows,
                         uint32_t n_cols, uint64_t nnz, bgnn_graph* g) {
  g->device = ctx->device;
  g->n_src = n_cols;
  g->n_dst = n_rows;
  g->num_edges = nnz;
  g->csr_only = true;
  g->row_ptr = row_ptr;
  g->src_of = col;
  return build_schedule(ctx, g);
}

int bgnn_graph_dinv(bgnn_ctx* ctx, bgnn_graph* g, int tail, const float** out) {
  float*& d = g->dinv[tail ? 1 : 0];
  if (!d) {
    BGNN_CUDA(ctx, cudaMalloc(&d, ((size_t)g->n_dst + 1) * 4));
    k_dinv_from_rowptr<<<grid_for(ctx, g->n_dst, 256), 256, 0, ctx->stream>>>(g->row_ptr, g->n_dst,
                                                                             tail, d);
    BGNN_LAUNCHED(ctx);
  }
  *out = d;
  return BGNN_OK;
}

// warp per row: every slot of the row gets the row's id
__global__ void k_dst_of(const uint32_t* __restrict__ rp, uint32_t n, uint32_t* __restrict__ out) {
  const uint32_t lane = threadIdx.x & 31;
  for (uint32_t r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < n;
       r += (gridDim.x * blockDim.x) >> 5)
    for (uint32_t s = rp[r] + lane; s < rp[r + 1]; s += 32) out[s] = r;
}

// the same map written into a caller's buffer of num_edges words (no allocation)
int bgnn_graph_dst_of_into(bgnn_ctx* ctx, const bgnn_graph* g, uint32_t* out) {
  if (g->num_edges == 0) return BGNN_OK;
  k_dst_of<<<grid_for(ctx, (uint64_t)g->n_dst * 32, 256), 256, 0, ctx->stream>>>(g->row_ptr,
                                                                                 g->n_dst, out);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

int bgnn_graph_dst_of(bgnn_ctx* ctx, bgnn_graph* g, const uint32_t** out) {
  if (!g->dst_of) {
    BGNN_CUDA(ctx, cudaMalloc(&g->dst_of, (g->num_edges ? g->num_edges : 1) * 4));
    k_dst_of<<<grid_for(ctx, (uint64_t)g->n_dst * 32, 256), 256, 0, ctx->stream>>>(
        g->row_ptr, g->n_dst, g->dst_of);
    BGNN_LAUNCHED(ctx);
  }
  *out = g->dst_of;
  return BGNN_OK;
}

// ---- C ABI: graph handles and standalone builders --------------------------

extern "C" int bgnn_graph_create(bgnn_ctx* ctx, const uint32_t* edge_index, uint64_t num_edges,
                                 uint32_t num_src, uint32_t num_dst, int on_host,
                                 bgnn_graph** out) {
  if (!ctx || !out) return BGNN_ERR_INVALID_ARG;
  BGNN_REQUIRE(ctx, edge_index || num_edges == 0, "edge_index is NULL");
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  bgnn_graph* g = new bgnn_graph();
  DevTmp staged;
  const uint32_t* ei = edge_index;
  int rc = BGNN_OK;
  if (on_host && num_edges) {
    // pageable host memory is staged through the library's pinned chunks
    rc = bgnn_tmp_alloc(ctx, staged, num_edges * 8);
    if (rc == BGNN_OK) rc = bgnn_copy_h2d(ctx, staged.p, edge_index, num_edges * 8);
    ei = staged.as<uint32_t>();
  }
  if (rc == BGNN_OK) rc = bgnn_graph_build(ctx, ei, ei + num_edges, num_edges, num_src, num_dst, g);
  if (rc == BGNN_OK) {
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) rc = bgnn_set_error(ctx, BGNN_ERR_CUDA, "graph build: %s",
                                              cudaGetErrorString(e));
  }
  if (rc != BGNN_OK) {
    bgnn_graph_free(g);
    delete g;
    return rc;
  }
  *out = g;
  return BGNN_OK;
}

extern "C" int bgnn_graph_create_csr(bgnn_ctx* ctx, const uint32_t* row_ptr, const uint32_t* col,
                                     uint32_t num_rows, uint32_t num_cols, bgnn_graph** out) {
  if (!ctx || !out || !row_ptr) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  bgnn_graph* g = new bgnn_graph();
  int rc = bgnn_graph_from_csr(ctx, row_ptr, col, num_rows, num_cols, g, true);
  if (rc != BGNN_OK) {
    bgnn_graph_free(g);
    delete g;
    return rc;
  }
  *out = g;
  return BGNN_OK;
}

extern "C" int bgnn_graph_destroy(bgnn_graph* g) {
  if (!g) return BGNN_OK;
  cudaSetDevice(g->device);
  bgnn_graph_free(g);
  delete g;
  return BGNN_OK;
}

extern "C" int bgnn_graph_info(const bgnn_graph* g, uint32_t* num_src, uint32_t* num_dst,
                               uint64_t* num_edges, int* has_self_loops) {
  if (!g) return BGNN_ERR_INVALID_ARG;
  if (num_src) *num_src = g->n_src;
  if (num_dst) *num_dst = g->n_dst;
  if (num_edges) *num_edges = g->num_edges;
  if (has_self_loops) *has_self_loops = g->has_self_loops;
  return BGNN_OK;
}

namespace {
__global__ void k_rowptr_diff(const uint32_t* __restrict__ rp, uint32_t n, uint32_t* __restrict__ out) {
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < n; r += gridDim.x * blockDim.x)
    out[r] = rp[r + 1] - rp[r];
}
}  // namespace

extern "C" int bgnn_graph_degrees(bgnn_ctx* ctx, const bgnn_graph* g, uint32_t* in_deg,
                                  uint32_t* out_deg) {
  if (!ctx || !g) return BGNN_ERR_INVALID_ARG;
  if (in_deg && g->n_dst) {
    k_rowptr_diff<<<grid_for(ctx, g->n_dst, 256), 256, 0, ctx->stream>>>(g->row_ptr, g->n_dst, in_deg);
    BGNN_LAUNCHED(ctx);
  }
  if (out_deg) {
    BGNN_REQUIRE(ctx, g->out_deg != nullptr, "graph built from a CSR has no out-degree");
    BGNN_CUDA(ctx, cudaMemcpyAsync(out_deg, g->out_deg, (size_t)g->n_src * 4,
                                   cudaMemcpyDeviceToDevice, ctx->stream));
  }
  return BGNN_OK;
}

extern "C" int bgnn_graph_csr(bgnn_ctx* ctx, const bgnn_graph* g, uint32_t* row_ptr,
                              uint32_t* src_of, uint32_t* edge_id) {
  if (!ctx || !g) return BGNN_ERR_INVALID_ARG;
  if (row_ptr)
    BGNN_CUDA(ctx, cudaMemcpyAsync(row_ptr, g->row_ptr, ((size_t)g->n_dst + 1) * 4,
                                   cudaMemcpyDeviceToDevice, ctx->stream));
  if (src_of && g->num_edges)
    BGNN_CUDA(ctx, cudaMemcpyAsync(src_of, g->src_of, (size_t)g->num_edges * 4,
                                   cudaMemcpyDeviceToDevice, ctx->stream));
  if (edge_id && g->num_edges) {
    BGNN_REQUIRE(ctx, g->eid != nullptr, "graph built from a CSR has no edge ids");
    BGNN_CUDA(ctx, cudaMemcpyAsync(edge_id, g->eid, (size_t)g->num_edges * 4,
                                   cudaMemcpyDeviceToDevice, ctx->stream));
  }
  return BGNN_OK;
}

// SparseCSR.fromCOO: stable sort by (row, col), as two stable LSD radix
// sorts (col first, then row) carrying the original entry index.
extern "C" int bgnn_coo_to_csr_dev(bgnn_ctx* ctx, const uint32_t* rows, const uint32_t* cols,
                                   const float* values, uint64_t nnz, uint32_t num_rows,
                                   uint32_t num_cols, uint32_t* row_ptr, uint32_t* col_out,
                                   float* val_out) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  BGNN_REQUIRE(ctx, row_ptr != nullptr, "row_ptr is NULL");
  BGNN_REQUIRE(ctx, nnz == 0 || (rows && cols && col_out), "NULL COO arrays");
  if (nnz >= 0xffffffffull)
    return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED, "nnz exceeds 2^32-2");
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  BGNN_CUDA(ctx, cudaMemsetAsync(row_ptr, 0, ((size_t)num_rows + 1) * 4, ctx->stream));
  DevTmp flagbuf;
  BGNN_TRY(bgnn_tmp_alloc(ctx, flagbuf, 16));
  BGNN_CUDA(ctx, cudaMemsetAsync(flagbuf.p, 0, 8, ctx->stream));
  BGNN_CUDA(ctx, cudaMemsetAsync((char*)flagbuf.p + 8, 0xff, 8, ctx->stream));
  if (nnz) {
    // row histogram + bounds (rows < num_rows, cols < num_cols)
    k_count_validate<<<grid_for(ctx, nnz, 256), 256, 0, ctx->stream>>>(
        cols, rows, nnz, num_cols, num_rows, row_ptr, nullptr, 0, flagbuf.as<uint32_t>(),
        reinterpret_cast<unsigned long long*>((char*)flagbuf.p + 8));
    BGNN_LAUNCHED(ctx);
  }
  unsigned long long hb = 0;
  BGNN_CUDA(ctx, cudaMemcpyAsync(&hb, (char*)flagbuf.p + 8, 8, cudaMemcpyDeviceToHost, ctx->stream));
  BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if (hb != ~0ull)
    return bgnn_set_error(ctx, BGNN_ERR_OUT_OF_RANGE, "COO %s index out of bounds (entry %llu)",
                          hb < nnz ? "column" : "row", hb < nnz ? hb : hb - nnz);
  BGNN_TRY(counts_to_rowptr(ctx, row_ptr, num_rows));
  if (nnz == 0) return BGNN_OK;
  // column pass: stable sort by column carrying each entry's row (and value);
  // row pass: stable sort of that order by row carrying the columns (and
  // values).  The result is sorted by (row, col) with ties in input order.
  const bool want_vals = values != nullptr && val_out != nullptr;
  const uint32_t* vbits = reinterpret_cast<const uint32_t*>(values);
  DevTmp cols_c, rows_c, vals_c;
  BGNN_TRY(bgnn_tmp_alloc(ctx, cols_c, nnz * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, rows_c, nnz * 4));
  if (want_vals) BGNN_TRY(bgnn_tmp_alloc(ctx, vals_c, nnz * 4));
  const int cbits = num_cols > 1 ? bgnn_bits_for(num_cols - 1) : 0;
  const int rbits = num_rows > 1 ? bgnn_bits_for(num_rows - 1) : 0;
  BGNN_TRY(bgnn_radix_sort(ctx, cols, nnz, cbits, rows, 0, want_vals ? vbits : nullptr,
                           cols_c.as<uint32_t>(), rows_c.as<uint32_t>(),
                           want_vals ? vals_c.as<uint32_t>() : nullptr));
  BGNN_TRY(bgnn_radix_sort(ctx, rows_c.as<uint32_t>(), nnz, rbits, cols_c.as<uint32_t>(), 0,
                           want_vals ? vals_c.as<uint32_t>() : nullptr, nullptr, col_out,
                           want_vals ? reinterpret_cast<uint32_t*>(val_out) : nullptr));
  if (val_out && !values) {
    k_fill_ones<<<grid_for(ctx, nnz, 256), 256, 0, ctx->stream>>>(val_out, nnz);
    BGNN_LAUNCHED(ctx);
  }
  return BGNN_OK;
}

extern "C" int bgnn_gcn_norm_dev(bgnn_ctx* ctx, const uint32_t* edge_index, uint64_t E,
                                 uint32_t num_nodes, int add_self_loops, float* out) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  BGNN_REQUIRE(ctx, (edge_index && out) || E == 0, "NULL argument");
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  DevTmp deg, dinv, flagbuf;
  BGNN_TRY(bgnn_tmp_alloc(ctx, deg, ((size_t)num_nodes + 1) * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, dinv, ((size_t)num_nodes + 1) * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, flagbuf, 16));
  BGNN_CUDA(ctx, cudaMemsetAsync(deg.p, 0, ((size_t)num_nodes + 1) * 4, ctx->stream));
  BGNN_CUDA(ctx, cudaMemsetAsync((char*)flagbuf.p + 8, 0xff, 8, ctx->stream));
  if (E) {
    k_count_validate<<<grid_for(ctx, E, 256), 256, 0, ctx->stream>>>(
        edge_index, edge_index + E, E, num_nodes, num_nodes, deg.as<uint32_t>(), nullptr, 0,
        flagbuf.as<uint32_t>(), reinterpret_cast<unsigned long long*>((char*)flagbuf.p + 8));
    BGNN_LAUNCHED(ctx);
  }
  unsigned long long hb = 0;
  BGNN_CUDA(ctx, cudaMemcpyAsync(&hb, (char*)flagbuf.p + 8, 8, cudaMemcpyDeviceToHost, ctx->stream));
  BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if (hb != ~0ull)
    return bgnn_set_error(ctx, BGNN_ERR_OUT_OF_RANGE, "Edge index out of bounds (position %llu)", hb);
  if (num_nodes) {
    k_dinv_from_deg<<<grid_for(ctx, num_nodes, 256), 256, 0, ctx->stream>>>(
        deg.as<uint32_t>(), num_nodes, add_self_loops, dinv.as<float>());
    BGNN_LAUNCHED(ctx);
  }
  if (E) {
    k_edge_norm<<<grid_for(ctx, E, 256), 256, 0, ctx->stream>>>(edge_index, E, dinv.as<float>(), out);
    BGNN_LAUNCHED(ctx);
  }
  return BGNN_OK;
}
