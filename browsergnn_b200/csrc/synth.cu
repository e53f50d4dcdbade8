// Seeded synthetic graph generator for benchmark inputs (R-MAT).  Not part of
// the reference's path: it produces the same edge list as the numpy generator
// in browsergnn_b200/synth.py (identical integer hashing and double compares),
// fast enough for the 62M- and 268M-edge graphs.
//
// Edge attempt t draws one uniform per recursion level from a counter-based
// hash; the quadrant thresholds a, a+b, a+b+c pick one bit of the source and
// one of the destination.  Attempts with an id >= num_nodes are rejected; the
// first num_edges accepted attempts (in attempt order) form the graph.  Node
// ids are then relabelled by a seeded bijection of [0, num_nodes).
#include "bgnn_internal.cuh"

namespace {

__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  uint64_t z = x;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

struct Perm {
  uint64_t mul[4];
  uint64_t add[4];
  uint64_t mask;
  int shift;
};

__host__ __device__ __forceinline__ uint64_t perm_round(uint64_t x, const Perm& p) {
#pragma unroll
  for (int r = 0; r < 4; r++) {
    x = (x * p.mul[r]) & p.mask;
    x ^= x >> p.shift;
    x = (x + p.add[r]) & p.mask;
  }
  return x;
}

__host__ __device__ __forceinline__ uint32_t perm_apply(uint32_t v, uint32_t n, const Perm& p) {
  uint64_t y = perm_round(v, p);
  while (y >= n) y = perm_round(y, p);  // cycle walking: a bijection of [0, n)
  return (uint32_t)y;
}

Perm make_perm(uint64_t seed, int bits) {
  Perm p;
  uint64_t s = splitmix64(seed ^ 0x5045524D5045524Dull);
  for (int r = 0; r < 4; r++) {
    s = splitmix64(s);
    p.mul[r] = s | 1ull;
    s = splitmix64(s);
    p.add[r] = s;
  }
  p.mask = bits >= 64 ? ~0ull : ((1ull << bits) - 1ull);
  p.shift = (bits + 1) / 2;
  if (p.shift == 0) p.shift = 1;
  return p;
}

__global__ void k_rmat_attempts(uint64_t key0, uint64_t t0, uint32_t count, int scale, double a,
                                double ab, double abc, uint32_t n, uint32_t* __restrict__ src,
                                uint32_t* __restrict__ dst, uint32_t* __restrict__ ok) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
    const uint64_t t = t0 + i;
    uint32_t s = 0, d = 0;
    for (int l = 0; l < scale; l++) {
      const uint64_t h = splitmix64(key0 + t * (uint64_t)scale + (uint64_t)l);
      const double u = (double)(h >> 11) * 0x1p-53;
      const uint32_t rb = (u >= ab) ? 1u : 0u;                          // quadrants c, d
      const uint32_t cb = (u >= a && u < ab) || (u >= abc) ? 1u : 0u;   // quadrants b, d
      s = (s << 1) | rb;
      d = (d << 1) | cb;
    }
    src[i] = s;
    dst[i] = d;
    ok[i] = (s < n && d < n) ? 1u : 0u;
  }
}

__global__ void k_rmat_compact(const uint32_t* __restrict__ src, const uint32_t* __restrict__ dst,
                               const uint32_t* __restrict__ ok, const uint32_t* __restrict__ pos,
                               uint32_t count, uint64_t base, uint64_t limit, uint64_t num_edges,
                               uint32_t* __restrict__ out) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
    if (!ok[i]) continue;
    const uint64_t p = base + pos[i];
    if (p < limit) {
      out[p] = src[i];
      out[num_edges + p] = dst[i];
    }
  }
}

__global__ void k_permute(uint32_t* __restrict__ ids, uint64_t n_ids, uint32_t n, Perm p) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_ids;
       i += (uint64_t)gridDim.x * blockDim.x)
    ids[i] = perm_apply(ids[i], n, p);
}

inline unsigned grid_for(bgnn_ctx* ctx, uint64_t n, int tpb) {
  uint64_t b = (n + tpb - 1) / tpb;
  const uint64_t cap = (uint64_t)ctx->num_sms * 16;
  if (b > cap) b = cap;
  if (b == 0) b = 1;
  return (unsigned)b;
}

}  // namespace

extern "C" BGNN_API int bgnn_synth_rmat(bgnn_ctx* ctx, uint64_t seed, int scale, uint32_t num_nodes,
                                        uint64_t num_edges, double a, double b, double c,
                                        int permute, uint32_t* edge_index) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  BGNN_REQUIRE(ctx, scale >= 1 && scale <= 31, "scale must be in [1, 31]");
  BGNN_REQUIRE(ctx, num_nodes >= 1 && (uint64_t)num_nodes <= (1ull << scale),
               "num_nodes must be in [1, 2^scale]");
  BGNN_REQUIRE(ctx, edge_index != nullptr || num_edges == 0, "NULL edge_index");
  const uint32_t CHUNK = 1u << 24;
  DevTmp s, d, ok, pos;
  BGNN_TRY(bgnn_tmp_alloc(ctx, s, (size_t)CHUNK * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, d, (size_t)CHUNK * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, ok, ((size_t)CHUNK + 1) * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, pos, ((size_t)CHUNK + 1) * 4));
  const uint64_t key0 = splitmix64(seed);
  uint64_t have = 0, t0 = 0;
  int guard = 0;
  while (have < num_edges) {
    if (++guard > 1 << 20)
      return bgnn_set_error(ctx, BGNN_ERR_DEVICE, "R-MAT acceptance too low");
    k_rmat_attempts<<<grid_for(ctx, CHUNK, 256), 256, 0, ctx->stream>>>(
        key0, t0, CHUNK, scale, a, a + b, a + b + c, num_nodes, s.as<uint32_t>(), d.as<uint32_t>(),
        ok.as<uint32_t>());
    BGNN_LAUNCHED(ctx);
    BGNN_CUDA(ctx, cudaMemsetAsync(ok.as<uint32_t>() + CHUNK, 0, 4, ctx->stream));
    BGNN_TRY(bgnn_exclusive_scan(ctx, ok.as<uint32_t>(), pos.as<uint32_t>(), (uint64_t)CHUNK + 1));
    k_rmat_compact<<<grid_for(ctx, CHUNK, 256), 256, 0, ctx->stream>>>(
        s.as<uint32_t>(), d.as<uint32_t>(), ok.as<uint32_t>(), pos.as<uint32_t>(), CHUNK, have,
        num_edges, num_edges, edge_index);
    BGNN_LAUNCHED(ctx);
    uint32_t got = 0;
    BGNN_CUDA(ctx, cudaMemcpyAsync(&got, pos.as<uint32_t>() + CHUNK, 4, cudaMemcpyDeviceToHost,
                                   ctx->stream));
    BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    have += got;
    t0 += CHUNK;
  }
  if (permute && num_edges) {
    int bits = 0;
    while (bits < 32 && ((uint64_t)1 << bits) < num_nodes) bits++;
    if (bits == 0) bits = 1;
    const Perm p = make_perm(seed, bits);
    k_permute<<<grid_for(ctx, 2 * num_edges, 256), 256, 0, ctx->stream>>>(edge_index, 2 * num_edges,
                                                                         num_nodes, p);
    BGNN_LAUNCHED(ctx);
  }
  return BGNN_OK;
}
