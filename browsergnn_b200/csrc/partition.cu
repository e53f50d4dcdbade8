// Row partition of a graph across the GPUs of one node, built on the device
// with no communication.
//
// The reference has no multi-device code: this is how the B200 backend runs
// one layer's message passing (SAGEConv.forward, src/layers/sage.ts:113-217)
// or one SpMM (SparseCSR.matmul, src/core/sparse.ts:322-344) over several
// GPUs.  Rank r owns the contiguous rows [lo, hi) of a square CSR (a graph's
// destination-keyed CSR, or a SparseCSR) and keeps their entries in the
// global order, so every row is still reduced on one GPU in the reference's
// order and the result does not depend on the number of GPUs.
//
// Every rank is given the same global CSR and derives the same plan, so the
// plan needs no exchange of requests:
//   bounds     rank r's first row is the first row j with
//              row_ptr[j] + j >= r (E + N) / world (entries plus one per
//              row, so empty graphs still balance rows);
//   halo       the sorted unique columns of the local entries outside
//              [lo, hi): a flag per global node, then an exclusive scan gives
//              each its halo slot.  Sorted by id means grouped by owner, in
//              rank order, which is the order the owners send them in;
//   send list  for each peer p, the sorted owned rows some entry of p's rows
//              reads: a flag per (peer, owned row), scanned.  This is exactly
//              p's halo segment from this rank.
// The local CSR keeps the global entry order with columns relabelled to
// [0, n_own) for owned nodes and n_own + slot for halo nodes.
#include <algorithm>

#include "bgnn_internal.cuh"

namespace {

inline unsigned grid_for(bgnn_ctx* ctx, uint64_t n, int tpb) {
  uint64_t b = (n + tpb - 1) / tpb;
  const uint64_t cap = (uint64_t)ctx->num_sms * 16;
  if (b > cap) b = cap;
  if (b == 0) b = 1;
  return (unsigned)b;
}

// bounds[r] for r = 0..world: the first row j with row_ptr[j] + j >= target(r)
__global__ void k_part_bounds(const uint32_t* __restrict__ rp, uint32_t n, uint32_t world,
                              uint32_t* __restrict__ bounds) {
  const uint32_t r = threadIdx.x;
  if (r > world) return;
  if (n == 0) {
    bounds[r] = 0;
    return;
  }
  if (r == 0) {
    bounds[0] = 0;
    return;
  }
  if (r == world) {
    bounds[world] = n;
    return;
  }
  const uint64_t total = (uint64_t)rp[n] + n;
  const uint64_t target = total * r / world;
  uint32_t lo = 1, hi = n;  // answer in [1, n]
  while (lo < hi) {
    const uint32_t mid = lo + (hi - lo) / 2;
    if ((uint64_t)rp[mid] + mid >= target)
      hi = mid;
    else
      lo = mid + 1;
  }
  bounds[r] = lo;
}

// a caller's CSR: row_ptr[0] == 0 and non-decreasing, so every entry index
// below row_ptr[n] is one the caller provided; records the first bad row
__global__ void k_check_rowptr(const uint32_t* __restrict__ rp, uint32_t n,
                               unsigned long long* __restrict__ first_bad) {
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < n; r += gridDim.x * blockDim.x)
    if (rp[r + 1] < rp[r] || (r == 0 && rp[0] != 0)) atomicMin(first_bad, (unsigned long long)r);
}

__global__ void k_local_rowptr(const uint32_t* __restrict__ rp, uint32_t lo, uint32_t n_own,
                               uint32_t* __restrict__ out) {
  const uint32_t base = rp[lo];
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i <= n_own; i += gridDim.x * blockDim.x)
    out[i] = rp[lo + i] - base;
}

__global__ void k_halo_mark(const uint32_t* __restrict__ col, uint64_t e0, uint64_t e1,
                            uint32_t lo, uint32_t hi, uint32_t n, uint32_t* __restrict__ flag,
                            int* err) {
  for (uint64_t e = e0 + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < e1;
       e += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t c = col[e];
    if (c >= n) {
      dev_raise(err, DEVERR_INDEX, e, 40);
      continue;
    }
    if (c < lo || c >= hi) flag[c] = 1u;
  }
}

__global__ void k_halo_ids(const uint32_t* __restrict__ flag, const uint32_t* __restrict__ slot,
                           uint32_t n, uint32_t* __restrict__ ids) {
  for (uint32_t c = blockIdx.x * blockDim.x + threadIdx.x; c < n; c += gridDim.x * blockDim.x)
    if (flag[c]) ids[slot[c]] = c;
}

__global__ void k_relabel(const uint32_t* __restrict__ col, uint64_t e0, uint64_t ne, uint32_t lo,
                          uint32_t hi, uint32_t n_own, const uint32_t* __restrict__ slot,
                          uint32_t* __restrict__ out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < ne;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t c = col[e0 + i];
    out[i] = (c >= lo && c < hi) ? c - lo : n_own + slot[c];
  }
}

// warp per foreign row: mark (owner of the row, owned column) pairs
__global__ void k_send_mark(const uint32_t* __restrict__ rp, const uint32_t* __restrict__ col,
                            uint32_t n, const uint32_t* __restrict__ bounds, uint32_t world,
                            uint32_t rank, uint32_t* __restrict__ sflag) {
  __shared__ uint32_t sb[65];
  for (uint32_t i = threadIdx.x; i <= world; i += blockDim.x) sb[i] = bounds[i];
  __syncthreads();
  const uint32_t lo = sb[rank], hi = sb[rank + 1], n_own = hi - lo;
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
  for (uint32_t r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < n; r += warps) {
    if (r >= lo && r < hi) continue;
    uint32_t p = 0;
    while (p + 1 < world && r >= sb[p + 1]) p++;
    uint32_t* f = sflag + (uint64_t)p * n_own;
    const uint32_t b = rp[r], en = rp[r + 1];
    for (uint32_t e = b + lane; e < en; e += 32) {
      const uint32_t c = col[e];
      if (c >= lo && c < hi) f[c - lo] = 1u;
    }
  }
}

__global__ void k_send_list(const uint32_t* __restrict__ sflag, const uint32_t* __restrict__ pos,
                            uint64_t total, uint32_t n_own, uint32_t* __restrict__ rows) {
  for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < total;
       q += (uint64_t)gridDim.x * blockDim.x)
    if (sflag[q]) rows[pos[q]] = (uint32_t)(q % n_own);
}

// out[w] = a[idx[w]] for a few positions (the scans read at the bounds)
__global__ void k_pick(const uint32_t* __restrict__ a, const uint64_t* __restrict__ idx,
                       uint32_t m, uint32_t* __restrict__ out) {
  const uint32_t w = threadIdx.x;
  if (w < m) out[w] = a[idx[w]];
}

// out[i, :] = x[rows[i], col0 : col0 + width]  (vector path when aligned)
template <int V>
__global__ void k_pack_cols(const float* __restrict__ x, uint64_t ld_x, uint32_t col0,
                            uint32_t width, const uint32_t* __restrict__ rows, uint64_t n,
                            float* __restrict__ out) {
  const uint32_t wv = width / V;
  const uint64_t total = n * wv;
  for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t i = t / wv;
    const uint32_t j = (uint32_t)(t - i * wv) * V;
    const float* src = x + (uint64_t)rows[i] * ld_x + col0 + j;
    float* dst = out + i * width + j;
    if constexpr (V == 4)
      *reinterpret_cast<float4*>(dst) = __ldg(reinterpret_cast<const float4*>(src));
    else
      *dst = __ldg(src);
  }
}

// x[i, col0 : col0 + width] = src[i, :]
template <int V>
__global__ void k_unpack_cols(const float* __restrict__ src, uint64_t n, uint32_t width,
                              float* __restrict__ x, uint64_t ld_x, uint32_t col0) {
  const uint32_t wv = width / V;
  const uint64_t total = n * wv;
  for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t i = t / wv;
    const uint32_t j = (uint32_t)(t - i * wv) * V;
    float* dst = x + i * ld_x + col0 + j;
    if constexpr (V == 4)
      *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(src + i * width + j);
    else
      *dst = src[i * width + j];
  }
}

// first index i in [0, len) with a[i] >= key (len when none)
__device__ __forceinline__ uint64_t lower_bound_u32(const uint32_t* a, uint64_t len, uint32_t key) {
  uint64_t lo = 0, hi = len;
  while (lo < hi) {
    const uint64_t mid = (lo + hi) >> 1;
    if (a[mid] < key)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

// one thread per (peer q, block boundary c): where block c starts in peer q's
// send list (owned local ids, ascending) and in owner q's halo slots (global
// ids, ascending)
__global__ void k_row_blocks(const uint32_t* __restrict__ send_rows,
                             const uint32_t* __restrict__ halo_ids,
                             const uint64_t* __restrict__ offs,  // send_off [w+1], recv_off [w+1]
                             const uint32_t* __restrict__ bounds, uint32_t world, uint32_t rank,
                             uint32_t blocks, uint64_t* __restrict__ out_send,
                             uint64_t* __restrict__ out_recv) {
  const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= world * (blocks + 1)) return;
  const uint32_t q = t / (blocks + 1), c = t % (blocks + 1);
  const uint64_t* send_off = offs;
  const uint64_t* recv_off = offs + world + 1;
  const uint32_t n_own = bounds[rank + 1] - bounds[rank];
  const uint32_t key = (uint32_t)((uint64_t)c * n_own / blocks);
  out_send[t] = send_off[q] + lower_bound_u32(send_rows + send_off[q],
                                              send_off[q + 1] - send_off[q], key);
  const uint32_t nq = bounds[q + 1] - bounds[q];
  const uint32_t gkey = bounds[q] + (uint32_t)((uint64_t)c * nq / blocks);
  out_recv[t] = recv_off[q] + lower_bound_u32(halo_ids + recv_off[q],
                                              recv_off[q + 1] - recv_off[q], gkey);
}

// out[i, :] = x[rows[i], :] for the entries of block c of every peer
// (blockIdx.y = peer)
template <int V>
__global__ void k_pack_block(const float* __restrict__ x, uint32_t width,
                             const uint32_t* __restrict__ rows, const uint64_t* __restrict__ blk,
                             uint32_t blocks, uint32_t c, float* __restrict__ out) {
  const uint32_t q = blockIdx.y;
  const uint64_t b = blk[q * (blocks + 1) + c], e = blk[q * (blocks + 1) + c + 1];
  const uint32_t wv = width / V;
  const uint64_t total = (e - b) * wv;
  for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t i = b + t / wv;
    const uint32_t j = (uint32_t)(t % wv) * V;
    const float* src = x + (uint64_t)rows[i] * width + j;
    float* dst = out + i * width + j;
    if constexpr (V == 4)
      *reinterpret_cast<float4*>(dst) = __ldg(reinterpret_cast<const float4*>(src));
    else
      *dst = __ldg(src);
  }
}

// The plan from a square device CSR (row_ptr [n+1], col [nnz]).
int build_part(bgnn_ctx* ctx, const uint32_t* rp, const uint32_t* col, uint32_t n,
               uint32_t world, uint32_t rank, bgnn_part* p) {
  p->device = ctx->device;
  p->world = world;
  p->rank = rank;
  p->n_global = n;
  DevTmp d_bounds;
  BGNN_TRY(bgnn_tmp_alloc(ctx, d_bounds, (world + 1) * 4));
  k_part_bounds<<<1, 128, 0, ctx->stream>>>(rp, n, world, d_bounds.as<uint32_t>());
  BGNN_LAUNCHED(ctx);
  p->bounds.assign(world + 1, 0);
  BGNN_CUDA(ctx, cudaMemcpyAsync(p->bounds.data(), d_bounds.p, (world + 1) * 4,
                                 cudaMemcpyDeviceToHost, ctx->stream));
  uint32_t rp_lohi[2] = {0, 0};
  BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  for (uint32_t r = 1; r <= world; r++) p->bounds[r] = std::max(p->bounds[r], p->bounds[r - 1]);
  p->lo = p->bounds[rank];
  p->hi = p->bounds[rank + 1];
  p->n_own = p->hi - p->lo;
  BGNN_CUDA(ctx, cudaMemcpyAsync(&rp_lohi[0], rp + p->lo, 4, cudaMemcpyDeviceToHost, ctx->stream));
  BGNN_CUDA(ctx, cudaMemcpyAsync(&rp_lohi[1], rp + p->hi, 4, cudaMemcpyDeviceToHost, ctx->stream));
  BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if (rp_lohi[1] < rp_lohi[0])
    return bgnn_set_error(ctx, BGNN_ERR_INVALID_ARG, "row_ptr decreases inside rows [%u, %u)",
                          p->lo, p->hi);
  p->entry_lo = rp_lohi[0];
  p->n_local_entries = (uint64_t)rp_lohi[1] - rp_lohi[0];
  const uint64_t e0 = p->entry_lo, e1 = e0 + p->n_local_entries;

  // halo: flag every foreign column the local rows read, scan to slots
  DevTmp flag, slot;
  BGNN_TRY(bgnn_tmp_alloc(ctx, flag, ((uint64_t)n + 1) * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, slot, ((uint64_t)n + 1) * 4));
  BGNN_CUDA(ctx, cudaMemsetAsync(flag.p, 0, ((uint64_t)n + 1) * 4, ctx->stream));
  if (e1 > e0) {
    k_halo_mark<<<grid_for(ctx, e1 - e0, 256), 256, 0, ctx->stream>>>(
        col, e0, e1, p->lo, p->hi, n, flag.as<uint32_t>(), ctx->d_err);
    BGNN_LAUNCHED(ctx);
  }
  BGNN_TRY(bgnn_check_device_error(ctx));
  BGNN_TRY(bgnn_exclusive_scan(ctx, flag.as<uint32_t>(), slot.as<uint32_t>(), (uint64_t)n + 1));
  // halo count and per-owner receive counts: the slot scan at the bounds
  std::vector<uint64_t> at(world + 1);
  for (uint32_t r = 0; r <= world; r++) at[r] = p->bounds[r];
  DevTmp d_at, d_picked;
  BGNN_TRY(bgnn_tmp_alloc(ctx, d_at, (world + 1) * 8));
  BGNN_TRY(bgnn_tmp_alloc(ctx, d_picked, (world + 1) * 4));
  std::vector<uint32_t> picked(world + 1);
  BGNN_CUDA(ctx, cudaMemcpyAsync(d_at.p, at.data(), (world + 1) * 8, cudaMemcpyHostToDevice,
                                 ctx->stream));
  k_pick<<<1, 128, 0, ctx->stream>>>(slot.as<uint32_t>(), d_at.as<uint64_t>(), world + 1,
                                     d_picked.as<uint32_t>());
  BGNN_LAUNCHED(ctx);
  BGNN_CUDA(ctx, cudaMemcpyAsync(picked.data(), d_picked.p, (world + 1) * 4,
                                 cudaMemcpyDeviceToHost, ctx->stream));
  BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  p->n_halo = picked[world];
  p->recv_counts.assign(world, 0);
  for (uint32_t r = 0; r < world; r++) p->recv_counts[r] = (uint64_t)picked[r + 1] - picked[r];
  BGNN_CUDA(ctx, cudaMalloc(&p->halo_ids, ((uint64_t)p->n_halo + 1) * 4));
  k_halo_ids<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(flag.as<uint32_t>(),
                                                             slot.as<uint32_t>(), n, p->halo_ids);
  BGNN_LAUNCHED(ctx);

  // local CSR: the rows' entries in global order, columns relabelled
  uint32_t* lrp = nullptr;
  uint32_t* lcol = nullptr;
  BGNN_CUDA(ctx, cudaMalloc(&lrp, ((uint64_t)p->n_own + 1) * 4));
  cudaError_t ce = cudaMalloc(&lcol, (p->n_local_entries ? p->n_local_entries : 1) * 4);
  if (ce != cudaSuccess) {
    cudaFree(lrp);
    return bgnn_set_error(ctx, BGNN_ERR_NO_MEMORY, "local CSR allocation failed");
  }
  k_local_rowptr<<<grid_for(ctx, (uint64_t)p->n_own + 1, 256), 256, 0, ctx->stream>>>(
      rp, p->lo, p->n_own, lrp);
  cudaError_t le = cudaGetLastError();
  if (le == cudaSuccess && p->n_local_entries) {
    k_relabel<<<grid_for(ctx, p->n_local_entries, 256), 256, 0, ctx->stream>>>(
        col, e0, p->n_local_entries, p->lo, p->hi, p->n_own, slot.as<uint32_t>(), lcol);
    le = cudaGetLastError();
  }
  if (le != cudaSuccess) {
    cudaFree(lrp);
    cudaFree(lcol);
    return bgnn_set_error(ctx, BGNN_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(le));
  }
  ctx->launches += p->n_local_entries ? 2 : 1;
  BGNN_TRY(bgnn_graph_adopt_csr(ctx, lrp, lcol, p->n_own, p->n_own + p->n_halo,
                                p->n_local_entries, &p->local));

  // send lists: flag (peer, owned row) pairs read by the other ranks' rows
  const uint64_t total = (uint64_t)world * p->n_own;
  DevTmp sflag, pos;
  BGNN_TRY(bgnn_tmp_alloc(ctx, sflag, (total + 1) * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, pos, (total + 1) * 4));
  BGNN_CUDA(ctx, cudaMemsetAsync(sflag.p, 0, (total + 1) * 4, ctx->stream));
  if (world > 1 && p->n_own > 0 && n > p->n_own) {
    k_send_mark<<<grid_for(ctx, (uint64_t)n * 32, 256), 256, 0, ctx->stream>>>(
        rp, col, n, d_bounds.as<uint32_t>(), world, rank, sflag.as<uint32_t>());
    BGNN_LAUNCHED(ctx);
  }
  BGNN_TRY(bgnn_exclusive_scan(ctx, sflag.as<uint32_t>(), pos.as<uint32_t>(), total + 1));
  for (uint32_t r = 0; r <= world; r++) at[r] = (uint64_t)r * p->n_own;
  BGNN_CUDA(ctx, cudaMemcpyAsync(d_at.p, at.data(), (world + 1) * 8, cudaMemcpyHostToDevice,
                                 ctx->stream));
  k_pick<<<1, 128, 0, ctx->stream>>>(pos.as<uint32_t>(), d_at.as<uint64_t>(), world + 1,
                                     d_picked.as<uint32_t>());
  BGNN_LAUNCHED(ctx);
  BGNN_CUDA(ctx, cudaMemcpyAsync(picked.data(), d_picked.p, (world + 1) * 4,
                                 cudaMemcpyDeviceToHost, ctx->stream));
  BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  p->n_send = picked[world];
  p->send_counts.assign(world, 0);
  for (uint32_t r = 0; r < world; r++) p->send_counts[r] = (uint64_t)picked[r + 1] - picked[r];
  BGNN_CUDA(ctx, cudaMalloc(&p->send_rows, (p->n_send + 1) * 4));
  if (total) {
    k_send_list<<<grid_for(ctx, total, 256), 256, 0, ctx->stream>>>(
        sflag.as<uint32_t>(), pos.as<uint32_t>(), total, p->n_own, p->send_rows);
    BGNN_LAUNCHED(ctx);
  }
  p->send_off.assign(world + 1, 0);
  p->recv_off.assign(world + 1, 0);
  for (uint32_t r = 0; r < world; r++) {
    p->send_off[r + 1] = p->send_off[r] + p->send_counts[r];
    p->recv_off[r + 1] = p->recv_off[r] + p->recv_counts[r];
  }
  BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return BGNN_OK;
}

int part_args_ok(bgnn_ctx* ctx, uint32_t world, uint32_t rank) {
  if (world == 0 || world > 64)
    return bgnn_set_error(ctx, BGNN_ERR_INVALID_ARG, "world size %u outside [1, 64]", world);
  if (rank >= world)
    return bgnn_set_error(ctx, BGNN_ERR_INVALID_ARG, "rank %u outside [0, %u)", rank, world);
  return BGNN_OK;
}

}  // namespace

void bgnn_part_free(bgnn_part* p) {
  if (!p) return;
  bgnn_graph_free(&p->local);
  cudaFree(p->halo_ids);
  cudaFree(p->send_rows);
  cudaFree(p->d_blk_send);
  p->halo_ids = nullptr;
  p->send_rows = nullptr;
  p->d_blk_send = nullptr;
  p->blk_count = 0;
}

int bgnn_part_row_blocks(bgnn_ctx* ctx, const bgnn_part* p, uint32_t blocks) {
  if (blocks == 0) return bgnn_set_error(ctx, BGNN_ERR_INVALID_ARG, "zero row blocks");
  if (p->blk_count == blocks) return BGNN_OK;
  const uint32_t w = p->world;
  const uint64_t cells = (uint64_t)w * (blocks + 1);
  cudaFree(p->d_blk_send);
  p->d_blk_send = nullptr;
  p->blk_count = 0;
  BGNN_CUDA(ctx, cudaMalloc(&p->d_blk_send, cells * 8));
  DevTmp recv, offs, bnd;
  BGNN_TRY(bgnn_tmp_alloc(ctx, recv, cells * 8));
  BGNN_TRY(bgnn_tmp_alloc(ctx, offs, (uint64_t)(w + 1) * 16));
  BGNN_TRY(bgnn_tmp_alloc(ctx, bnd, (uint64_t)(w + 1) * 4));
  std::vector<uint64_t> h_offs(2 * (w + 1));
  std::copy(p->send_off.begin(), p->send_off.end(), h_offs.begin());
  std::copy(p->recv_off.begin(), p->recv_off.end(), h_offs.begin() + w + 1);
  BGNN_CUDA(ctx, cudaMemcpyAsync(offs.p, h_offs.data(), h_offs.size() * 8, cudaMemcpyHostToDevice,
                                 ctx->stream));
  BGNN_CUDA(ctx, cudaMemcpyAsync(bnd.p, p->bounds.data(), (w + 1) * 4, cudaMemcpyHostToDevice,
                                 ctx->stream));
  k_row_blocks<<<(unsigned)((cells + 127) / 128), 128, 0, ctx->stream>>>(
      p->send_rows, p->halo_ids, offs.as<uint64_t>(), bnd.as<uint32_t>(), w, p->rank, blocks,
      p->d_blk_send, recv.as<uint64_t>());
  BGNN_LAUNCHED(ctx);
  p->blk_send.assign(cells, 0);
  p->blk_recv.assign(cells, 0);
  BGNN_CUDA(ctx, cudaMemcpyAsync(p->blk_send.data(), p->d_blk_send, cells * 8,
                                 cudaMemcpyDeviceToHost, ctx->stream));
  BGNN_CUDA(ctx, cudaMemcpyAsync(p->blk_recv.data(), recv.p, cells * 8, cudaMemcpyDeviceToHost,
                                 ctx->stream));
  BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  p->blk_count = blocks;
  return BGNN_OK;
}

int bgnn_run_pack_block(bgnn_ctx* ctx, const float* x, uint32_t width, const bgnn_part* p,
                        uint32_t c, float* out) {
  const uint32_t C = p->blk_count;
  if (C == 0 || c >= C) return bgnn_set_error(ctx, BGNN_ERR_INVALID_ARG, "row block %u of %u", c, C);
  if (width == 0 || p->n_send == 0 || p->world < 2) return BGNN_OK;
  const bool v4 = width % 4 == 0 && (uintptr_t)x % 16 == 0 && (uintptr_t)out % 16 == 0;
  const uint64_t per_peer = p->n_send / C / (p->world - 1) + 1;
  const uint64_t work = per_peer * (v4 ? width / 4 : width);
  uint64_t gx = (work + 255) / 256;
  const uint64_t cap = (uint64_t)ctx->num_sms * 8 / p->world + 1;
  if (gx > cap) gx = cap;
  dim3 grid((unsigned)gx, p->world);
  if (v4)
    k_pack_block<4><<<grid, 256, 0, ctx->stream>>>(x, width, p->send_rows, p->d_blk_send, C, c,
                                                   out);
  else
    k_pack_block<1><<<grid, 256, 0, ctx->stream>>>(x, width, p->send_rows, p->d_blk_send, C, c,
                                                   out);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

int bgnn_run_pack_cols(bgnn_ctx* ctx, const float* x, uint64_t ld_x, uint32_t col0,
                       uint32_t width, const uint32_t* rows, uint64_t n, float* out) {
  if (n == 0 || width == 0) return BGNN_OK;
  const bool v4 = width % 4 == 0 && col0 % 4 == 0 && ld_x % 4 == 0 &&
                  (uintptr_t)x % 16 == 0 && (uintptr_t)out % 16 == 0;
  if (v4)
    k_pack_cols<4><<<grid_for(ctx, n * width / 4, 256), 256, 0, ctx->stream>>>(x, ld_x, col0,
                                                                               width, rows, n, out);
  else
    k_pack_cols<1><<<grid_for(ctx, n * width, 256), 256, 0, ctx->stream>>>(x, ld_x, col0, width,
                                                                           rows, n, out);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

int bgnn_run_unpack_cols(bgnn_ctx* ctx, const float* src, uint64_t n, uint32_t width, float* x,
                         uint64_t ld_x, uint32_t col0) {
  if (n == 0 || width == 0) return BGNN_OK;
  const bool v4 = width % 4 == 0 && col0 % 4 == 0 && ld_x % 4 == 0 &&
                  (uintptr_t)x % 16 == 0 && (uintptr_t)src % 16 == 0;
  if (v4)
    k_unpack_cols<4><<<grid_for(ctx, n * width / 4, 256), 256, 0, ctx->stream>>>(src, n, width, x,
                                                                                 ld_x, col0);
  else
    k_unpack_cols<1><<<grid_for(ctx, n * width, 256), 256, 0, ctx->stream>>>(src, n, width, x,
                                                                             ld_x, col0);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

// ---- C ABI -----------------------------------------------------------------

extern "C" int bgnn_part_create_csr(bgnn_ctx* ctx, const uint32_t* row_ptr, const uint32_t* col,
                                    uint32_t num_rows, uint32_t world, uint32_t rank,
                                    bgnn_part** out) {
  if (!ctx || !out) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  BGNN_TRY(part_args_ok(ctx, world, rank));
  BGNN_REQUIRE(ctx, row_ptr != nullptr, "row_ptr is NULL");
  if (num_rows) {
    DevTmp bad;
    BGNN_TRY(bgnn_tmp_alloc(ctx, bad, 8));
    BGNN_CUDA(ctx, cudaMemsetAsync(bad.p, 0xff, 8, ctx->stream));
    k_check_rowptr<<<grid_for(ctx, num_rows, 256), 256, 0, ctx->stream>>>(
        row_ptr, num_rows, bad.as<unsigned long long>());
    BGNN_LAUNCHED(ctx);
    unsigned long long hb = 0;
    BGNN_CUDA(ctx, cudaMemcpyAsync(&hb, bad.p, 8, cudaMemcpyDeviceToHost, ctx->stream));
    BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    if (hb != ~0ull)
      return bgnn_set_error(ctx, BGNN_ERR_INVALID_ARG,
                            "row_ptr must start at 0 and not decrease (row %llu)", hb);
  }
  BGNN_REQUIRE(ctx, col != nullptr || num_rows == 0, "col is NULL");
  bgnn_part* p = new bgnn_part();
  int rc = build_part(ctx, row_ptr, col, num_rows, world, rank, p);
  if (rc != BGNN_OK) {
    bgnn_part_free(p);
    delete p;
    return rc;
  }
  *out = p;
  return BGNN_OK;
}

extern "C" int bgnn_part_create(bgnn_ctx* ctx, const uint32_t* edge_index, uint64_t num_edges,
                                uint32_t num_nodes, uint32_t world, uint32_t rank, int on_host,
                                bgnn_part** out) {
  if (!ctx || !out) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  BGNN_TRY(part_args_ok(ctx, world, rank));
  BGNN_REQUIRE(ctx, edge_index || num_edges == 0, "edge_index is NULL");
  // the destination-keyed CSR of the whole graph (each row's edges in COO
  // order), partitioned by rows, then dropped
  bgnn_graph* g = nullptr;
  BGNN_TRY(bgnn_graph_create(ctx, edge_index, num_edges, num_nodes, num_nodes, on_host, &g));
  bgnn_part* p = new bgnn_part();
  int rc = build_part(ctx, g->row_ptr, g->src_of, num_nodes, world, rank, p);
  bgnn_graph_destroy(g);
  if (rc != BGNN_OK) {
    bgnn_part_free(p);
    delete p;
    return rc;
  }
  *out = p;
  return BGNN_OK;
}

extern "C" int bgnn_part_destroy(bgnn_part* p) {
  if (!p) return BGNN_OK;
  cudaSetDevice(p->device);
  bgnn_part_free(p);
  delete p;
  return BGNN_OK;
}

extern "C" int bgnn_part_info(const bgnn_part* p, uint32_t* row_lo, uint32_t* row_hi,
                              uint32_t* num_halo, uint64_t* entry_lo, uint64_t* num_local_entries,
                              uint64_t* num_send) {
  if (!p) return BGNN_ERR_INVALID_ARG;
  if (row_lo) *row_lo = p->lo;
  if (row_hi) *row_hi = p->hi;
  if (num_halo) *num_halo = p->n_halo;
  if (entry_lo) *entry_lo = p->entry_lo;
  if (num_local_entries) *num_local_entries = p->n_local_entries;
  if (num_send) *num_send = p->n_send;
  return BGNN_OK;
}

extern "C" int bgnn_part_bounds(const bgnn_part* p, uint32_t* bounds) {
  if (!p || !bounds) return BGNN_ERR_INVALID_ARG;
  std::copy(p->bounds.begin(), p->bounds.end(), bounds);
  return BGNN_OK;
}

extern "C" int bgnn_part_counts(const bgnn_part* p, uint64_t* send_rows, uint64_t* recv_rows) {
  if (!p) return BGNN_ERR_INVALID_ARG;
  if (send_rows) std::copy(p->send_counts.begin(), p->send_counts.end(), send_rows);
  if (recv_rows) std::copy(p->recv_counts.begin(), p->recv_counts.end(), recv_rows);
  return BGNN_OK;
}

extern "C" int bgnn_part_row_blocks(bgnn_ctx* ctx, const bgnn_part* p, uint32_t blocks,
                                    uint64_t* send_first, uint64_t* recv_first) {
  if (!ctx || !p) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(p->device));
  BGNN_REQUIRE(ctx, blocks >= 1 && blocks <= 64, "row blocks %u outside [1, 64]", blocks);
  BGNN_TRY(bgnn_part_row_blocks(ctx, p, blocks));
  if (send_first) std::copy(p->blk_send.begin(), p->blk_send.end(), send_first);
  if (recv_first) std::copy(p->blk_recv.begin(), p->blk_recv.end(), recv_first);
  return BGNN_OK;
}

extern "C" int bgnn_part_graph(const bgnn_part* p, const bgnn_graph** out) {
  if (!p || !out) return BGNN_ERR_INVALID_ARG;
  *out = &p->local;
  return BGNN_OK;
}

extern "C" int bgnn_part_lists(bgnn_ctx* ctx, const bgnn_part* p, uint32_t* halo_ids,
                               uint32_t* send_rows) {
  if (!ctx || !p) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  if (halo_ids && p->n_halo)
    BGNN_CUDA(ctx, cudaMemcpyAsync(halo_ids, p->halo_ids, (uint64_t)p->n_halo * 4,
                                   cudaMemcpyDeviceToDevice, ctx->stream));
  if (send_rows && p->n_send)
    BGNN_CUDA(ctx, cudaMemcpyAsync(send_rows, p->send_rows, p->n_send * 4,
                                   cudaMemcpyDeviceToDevice, ctx->stream));
  return BGNN_OK;
}

extern "C" int bgnn_part_pack(bgnn_ctx* ctx, const bgnn_part* p, const float* x, uint64_t ld_x,
                              uint32_t col0, uint32_t width, float* out) {
  if (!ctx || !p) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  BGNN_REQUIRE(ctx, (x && out) || p->n_send == 0 || width == 0, "NULL argument");
  BGNN_REQUIRE(ctx, (uint64_t)col0 + width <= ld_x, "columns [%u, %u) exceed the row stride %llu",
               col0, col0 + width, (unsigned long long)ld_x);
  return bgnn_run_pack_cols(ctx, x, ld_x, col0, width, p->send_rows, p->n_send, out);
}

extern "C" int bgnn_part_unpack(bgnn_ctx* ctx, const bgnn_part* p, const float* halo,
                                uint32_t width, float* x, uint64_t ld_x, uint32_t col0) {
  if (!ctx || !p) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  BGNN_REQUIRE(ctx, (x && halo) || p->n_halo == 0 || width == 0, "NULL argument");
  BGNN_REQUIRE(ctx, (uint64_t)col0 + width <= ld_x, "columns [%u, %u) exceed the row stride %llu",
               col0, col0 + width, (unsigned long long)ld_x);
  return bgnn_run_unpack_cols(ctx, halo, p->n_halo, width, x + (uint64_t)p->n_own * ld_x, ld_x,
                              col0);
}
