// Device primitives: exclusive scan, stable LSD radix sort, gathers.
//
// The CSR builds need a *stable* ordering (each destination row keeps its
// edges in COO order, SparseCSR.fromCOO keeps ties in input order), so the
// sort is an LSD radix sort whose per-pass ranking is stable by construction:
// tiles are ranked in input order with warp match/popc, offsets come from a
// digit-major scan of per-tile histograms, never from atomic arrival order.
#include <cstdarg>

#include "bgnn_internal.cuh"

namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr int TPB = 256;          // threads per block for scan / sort tiles
constexpr int WARPS = TPB / 32;
constexpr int ROUNDS = 16;        // 32-item rounds per warp
constexpr int TILE = TPB * ROUNDS;  // 4096 items per tile
constexpr int RADIX = 256;

__device__ __forceinline__ uint32_t warp_incl_scan(uint32_t v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t t = __shfl_up_sync(FULL, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// --- exclusive scan --------------------------------------------------------
__global__ void __launch_bounds__(TPB) k_scan_reduce(const uint32_t* __restrict__ in, uint64_t n,
                                                     uint32_t* __restrict__ sums) {
  __shared__ uint32_t ws[WARPS];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const uint64_t base = (uint64_t)blockIdx.x * TILE + (uint64_t)w * (32 * ROUNDS);
  uint32_t s = 0;
#pragma unroll
  for (int r = 0; r < ROUNDS; r++) {
    const uint64_t i = base + (uint64_t)r * 32 + lane;
    if (i < n) s += in[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(FULL, s, o);
  if (lane == 0) ws[w] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t t = 0;
    for (int i = 0; i < WARPS; i++) t += ws[i];
    sums[blockIdx.x] = t;
  }
}

__global__ void __launch_bounds__(TPB) k_scan_down(const uint32_t* in, uint64_t n,
                                                   const uint32_t* __restrict__ offs,
                                                   uint32_t* out) {
  __shared__ uint32_t ws[WARPS];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const uint64_t base = (uint64_t)blockIdx.x * TILE + (uint64_t)w * (32 * ROUNDS);
  uint32_t v[ROUNDS];
  uint32_t run = 0;
#pragma unroll
  for (int r = 0; r < ROUNDS; r++) {
    const uint64_t i = base + (uint64_t)r * 32 + lane;
    const uint32_t x = i < n ? in[i] : 0u;
    const uint32_t inc = warp_incl_scan(x, lane);
    v[r] = run + inc - x;
    run += __shfl_sync(FULL, inc, 31);
  }
  if (lane == 0) ws[w] = run;
  __syncthreads();
  uint32_t wb = offs ? offs[blockIdx.x] : 0u;
  for (int i = 0; i < w; i++) wb += ws[i];
#pragma unroll
  for (int r = 0; r < ROUNDS; r++) {
    const uint64_t i = base + (uint64_t)r * 32 + lane;
    if (i < n) out[i] = wb + v[r];
  }
}

// --- radix sort -------------------------------------------------------------
__global__ void __launch_bounds__(TPB) k_radix_hist(const uint32_t* __restrict__ keys, uint64_t n,
                                                    int shift, uint32_t num_tiles,
                                                    uint32_t* __restrict__ hist) {
  __shared__ uint32_t h[RADIX];
  h[threadIdx.x] = 0;
  __syncthreads();
  const uint64_t base = (uint64_t)blockIdx.x * TILE;
#pragma unroll 4
  for (int r = 0; r < ROUNDS; r++) {
    const uint64_t i = base + (uint64_t)r * TPB + threadIdx.x;
    if (i < n) atomicAdd(&h[(keys[i] >> shift) & (RADIX - 1)], 1u);
  }
  __syncthreads();
  hist[(uint64_t)threadIdx.x * num_tiles + blockIdx.x] = h[threadIdx.x];
}

// One stable counting pass over 8 key bits.  Warp w of a tile owns items
// [w*512, w*512+512) in input order and ranks them 32 at a time; the ranks
// plus per-(warp,digit) running counts give every item its position among
// the tile's items of the same digit, in input order.
__global__ void __launch_bounds__(TPB) k_radix_scatter(const uint32_t* __restrict__ keys_in,
                                                       const uint32_t* __restrict__ vals_in,
                                                       uint64_t n, int shift, uint32_t num_tiles,
                                                       const uint32_t* __restrict__ offs,
                                                       uint32_t* __restrict__ keys_out,
                                                       uint32_t* __restrict__ vals_out) {
  __shared__ uint32_t whist[WARPS][RADIX];
  __shared__ uint32_t tile_off[RADIX];
  __shared__ uint32_t wsum[WARPS];
  __shared__ uint32_t sk[TILE];
  __shared__ uint32_t sv[TILE];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < WARPS * RADIX; i += TPB) (&whist[0][0])[i] = 0;
  __syncthreads();

  const uint64_t tile_base = (uint64_t)blockIdx.x * TILE;
  const uint64_t wbase = tile_base + (uint64_t)w * (32 * ROUNDS);
  const unsigned lt_mask = (1u << lane) - 1u;
  uint32_t key[ROUNDS], val[ROUNDS], loc[ROUNDS];
#pragma unroll
  for (int r = 0; r < ROUNDS; r++) {
    const uint64_t i = wbase + (uint64_t)r * 32 + lane;
    const bool valid = i < n;
    const uint32_t k = valid ? keys_in[i] : 0u;
    const uint32_t v = valid ? (vals_in ? vals_in[i] : (uint32_t)i) : 0u;
    const uint32_t d = valid ? ((k >> shift) & (RADIX - 1)) : (uint32_t)RADIX;
    const unsigned peers = __match_any_sync(FULL, d);
    const int leader = __ffs(peers) - 1;
    uint32_t b = 0;
    if (valid && lane == leader) {
      b = whist[w][d];
      whist[w][d] = b + (uint32_t)__popc(peers);
    }
    b = __shfl_sync(FULL, b, leader);
    __syncwarp();
    key[r] = k;
    val[r] = v;
    loc[r] = valid ? (b + (uint32_t)__popc(peers & lt_mask)) : 0xffffffffu;
  }
  __syncthreads();
  // per digit: exclusive prefix over warps, and the tile's digit count
  {
    const int d = threadIdx.x;
    uint32_t run = 0;
#pragma unroll
    for (int ww = 0; ww < WARPS; ww++) {
      const uint32_t c = whist[ww][d];
      whist[ww][d] = run;
      run += c;
    }
    // block-wide exclusive scan of the 256 digit counts
    const uint32_t inc = warp_incl_scan(run, lane);
    if (lane == 31) wsum[w] = inc;
    __syncthreads();
    uint32_t wb = 0;
    for (int ww = 0; ww < w; ww++) wb += wsum[ww];
    tile_off[d] = wb + inc - run;
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < ROUNDS; r++) {
    if (loc[r] != 0xffffffffu) {
      const uint32_t d = (key[r] >> shift) & (RADIX - 1);
      const uint32_t p = tile_off[d] + whist[w][d] + loc[r];
      sk[p] = key[r];
      sv[p] = val[r];
    }
  }
  __syncthreads();
  const uint64_t rem = n - tile_base;
  const uint32_t count = rem < (uint64_t)TILE ? (uint32_t)rem : (uint32_t)TILE;
  for (uint32_t p = threadIdx.x; p < count; p += TPB) {
    const uint32_t k = sk[p];
    const uint32_t d = (k >> shift) & (RADIX - 1);
    const uint64_t g = (uint64_t)offs[(uint64_t)d * num_tiles + blockIdx.x] + (p - tile_off[d]);
    if (keys_out) keys_out[g] = k;
    vals_out[g] = sv[p];
  }
}

__global__ void k_gather_u32(const uint32_t* __restrict__ src, const uint32_t* __restrict__ idx,
                             uint64_t n, uint32_t* __restrict__ out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = src[idx[i]];
}

__global__ void k_gather_f32(const float* __restrict__ src, const uint32_t* __restrict__ idx,
                             uint64_t n, float* __restrict__ out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = src[idx[i]];
}

__global__ void k_iota(uint32_t* out, uint64_t n) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = (uint32_t)i;
}

inline unsigned grid_for(bgnn_ctx* ctx, uint64_t n, int tpb) {
  uint64_t b = (n + tpb - 1) / tpb;
  const uint64_t cap = (uint64_t)ctx->num_sms * 16;
  if (b > cap) b = cap;
  if (b == 0) b = 1;
  return (unsigned)b;
}

}  // namespace

int bgnn_set_error(bgnn_ctx* ctx, int code, const char* fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    ctx->last_error = buf;
  }
  return code;
}

int bgnn_tmp_alloc(bgnn_ctx* ctx, DevTmp& t, size_t bytes) {
  t.s = ctx->stream;
  if (bytes == 0) bytes = 16;
  cudaError_t e = cudaMallocAsync(&t.p, bytes, ctx->stream);
  if (e != cudaSuccess) {
    t.p = nullptr;
    cudaGetLastError();
    return bgnn_set_error(ctx, BGNN_ERR_NO_MEMORY, "device allocation of %zu bytes failed: %s",
                          bytes, cudaGetErrorString(e));
  }
  return BGNN_OK;
}

int bgnn_exclusive_scan(bgnn_ctx* ctx, const uint32_t* in, uint32_t* out, uint64_t n) {
  if (n == 0) return BGNN_OK;
  const uint64_t tiles = (n + TILE - 1) / TILE;
  if (tiles == 1) {
    k_scan_down<<<1, TPB, 0, ctx->stream>>>(in, n, nullptr, out);
    BGNN_LAUNCHED(ctx);
    return BGNN_OK;
  }
  DevTmp sums;
  BGNN_TRY(bgnn_tmp_alloc(ctx, sums, tiles * sizeof(uint32_t)));
  k_scan_reduce<<<(unsigned)tiles, TPB, 0, ctx->stream>>>(in, n, sums.as<uint32_t>());
  BGNN_LAUNCHED(ctx);
  BGNN_TRY(bgnn_exclusive_scan(ctx, sums.as<uint32_t>(), sums.as<uint32_t>(), tiles));
  k_scan_down<<<(unsigned)tiles, TPB, 0, ctx->stream>>>(in, n, sums.as<uint32_t>(), out);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

int bgnn_bits_for(uint64_t max_value) {
  int b = 0;
  while (b < 64 && (max_value >> b) != 0) b++;
  return b;
}

int bgnn_radix_sort_pairs(bgnn_ctx* ctx, const uint32_t* keys_in, const uint32_t* vals_in,
                          uint64_t n, int key_bits, uint32_t* keys_out, uint32_t* vals_out) {
  if (n == 0) return BGNN_OK;
  if (n > 0xffffffffull)
    return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED, "radix sort limited to 2^32-1 items");
  const int passes = (key_bits + 7) / 8;
  if (passes == 0) {
    if (vals_in)
      BGNN_CUDA(ctx, cudaMemcpyAsync(vals_out, vals_in, n * 4, cudaMemcpyDeviceToDevice,
                                     ctx->stream));
    else {
      k_iota<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(vals_out, n);
      BGNN_LAUNCHED(ctx);
    }
    if (keys_out)
      BGNN_CUDA(ctx, cudaMemcpyAsync(keys_out, keys_in, n * 4, cudaMemcpyDeviceToDevice,
                                     ctx->stream));
    return BGNN_OK;
  }
  const uint64_t tiles = (n + TILE - 1) / TILE;
  DevTmp hist, kb0, kb1, vb0, vb1;
  BGNN_TRY(bgnn_tmp_alloc(ctx, hist, tiles * RADIX * sizeof(uint32_t)));
  BGNN_TRY(bgnn_tmp_alloc(ctx, kb0, n * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, kb1, n * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, vb0, n * 4));
  BGNN_TRY(bgnn_tmp_alloc(ctx, vb1, n * 4));
  const uint32_t* kin = keys_in;
  const uint32_t* vin = vals_in;
  uint32_t* kbuf[2] = {kb0.as<uint32_t>(), kb1.as<uint32_t>()};
  uint32_t* vbuf[2] = {vb0.as<uint32_t>(), vb1.as<uint32_t>()};
  for (int p = 0; p < passes; p++) {
    const int shift = 8 * p;
    const bool last = p == passes - 1;
    uint32_t* kout = last ? keys_out : kbuf[p & 1];
    uint32_t* vout = last ? vals_out : vbuf[p & 1];
    k_radix_hist<<<(unsigned)tiles, TPB, 0, ctx->stream>>>(kin, n, shift, (uint32_t)tiles,
                                                            hist.as<uint32_t>());
    BGNN_LAUNCHED(ctx);
    BGNN_TRY(bgnn_exclusive_scan(ctx, hist.as<uint32_t>(), hist.as<uint32_t>(), tiles * RADIX));
    // the last pass may skip writing keys when the caller does not want them
    k_radix_scatter<<<(unsigned)tiles, TPB, 0, ctx->stream>>>(
        kin, vin, n, shift, (uint32_t)tiles, hist.as<uint32_t>(), kout, vout);
    BGNN_LAUNCHED(ctx);
    kin = kout ? kout : kin;  // (kout is only null on the last pass)
    vin = vout;
  }
  return BGNN_OK;
}

int bgnn_gather_u32(bgnn_ctx* ctx, const uint32_t* src, const uint32_t* idx, uint64_t n,
                    uint32_t* out) {
  if (n == 0) return BGNN_OK;
  k_gather_u32<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(src, idx, n, out);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

int bgnn_gather_f32(bgnn_ctx* ctx, const float* src, const uint32_t* idx, uint64_t n,
                    float* out) {
  if (n == 0) return BGNN_OK;
  k_gather_f32<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(src, idx, n, out);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

int bgnn_iota(bgnn_ctx* ctx, uint32_t* out, uint64_t n) {
  if (n == 0) return BGNN_OK;
  k_iota<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(out, n);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

int bgnn_check_device_error(bgnn_ctx* ctx) {
  int h[4] = {0, 0, 0, 0};
  BGNN_CUDA(ctx, cudaMemcpyAsync(h, ctx->d_err, sizeof(h), cudaMemcpyDeviceToHost, ctx->stream));
  BGNN_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if (h[0] == DEVERR_NONE) return BGNN_OK;
  BGNN_CUDA(ctx, cudaMemsetAsync(ctx->d_err, 0, 4 * sizeof(int), ctx->stream));
  const uint64_t info = (uint64_t)(uint32_t)h[1] | ((uint64_t)(uint32_t)h[2] << 32);
  if (h[0] == DEVERR_INDEX)
    return bgnn_set_error(ctx, BGNN_ERR_OUT_OF_RANGE,
                          "index out of range at position %llu (check site %d)",
                          (unsigned long long)info, h[3]);
  if (h[0] == DEVERR_TIMEOUT)
    return bgnn_set_error(ctx, BGNN_ERR_TIMEOUT, "a bounded device wait gave up (site %d)", h[3]);
  return bgnn_set_error(ctx, BGNN_ERR_DEVICE, "device error %d (site %d)", h[0], h[3]);
}
