// Device primitives: exclusive scan, stable LSD radix sort.
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

// One stable counting pass over 8 key bits, carrying NP payload words per
// item.  Warp w of a tile owns items [w*512, w*512+512) in input order and
// ranks them 32 at a time; the ranks plus per-(warp,digit) running counts give
// every item its position among the tile's items of the same digit, in input
// order.  The tile is then regrouped by digit in shared memory (keys and
// payloads, the payloads read from global memory only at that point, in
// input order), and each digit's run is written to its global position,
// consecutive threads on consecutive positions.  The tile's 256 global digit
// offsets are read once into shared memory: reading them per item from the
// digit-major table (one cache line per digit, 256 lines per tile) missed L1
// and cost a random L2 read per item.
// ident0: payload 0 is the item's input index (p0_in unused).
template <int NP>
__global__ void __launch_bounds__(TPB) k_radix_scatter(
    const uint32_t* __restrict__ keys_in, const uint32_t* __restrict__ p0_in,
    const uint32_t* __restrict__ p1_in, int ident0, uint64_t n, int shift, uint32_t num_tiles,
    const uint32_t* __restrict__ offs, uint32_t* __restrict__ keys_out,
    uint32_t* __restrict__ p0_out, uint32_t* __restrict__ p1_out) {
  __shared__ uint32_t whist[WARPS][RADIX];
  __shared__ uint32_t tile_off[RADIX];
  __shared__ uint32_t gbase[RADIX];  // global position of the tile's digit-d run, minus tile_off[d]
  __shared__ uint32_t wsum[WARPS];
  extern __shared__ uint32_t rs_dyn[];
  uint32_t* sk = rs_dyn;             // [TILE] keys grouped by digit
  uint32_t* sp0 = rs_dyn + TILE;     // [TILE] payload 0 (NP >= 1)
  uint32_t* sp1 = rs_dyn + 2 * TILE; // [TILE] payload 1 (NP == 2)
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < WARPS * RADIX; i += TPB) (&whist[0][0])[i] = 0;
  __syncthreads();

  const uint64_t tile_base = (uint64_t)blockIdx.x * TILE;
  const uint64_t wbase = tile_base + (uint64_t)w * (32 * ROUNDS);
  const unsigned lt_mask = (1u << lane) - 1u;
  uint32_t key[ROUNDS], loc[ROUNDS];
#pragma unroll
  for (int r = 0; r < ROUNDS; r++) {
    const uint64_t i = wbase + (uint64_t)r * 32 + lane;
    const bool valid = i < n;
    const uint32_t k = valid ? keys_in[i] : 0u;
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
    const uint32_t toff = wb + inc - run;
    tile_off[d] = toff;
    gbase[d] = offs[(uint64_t)d * num_tiles + blockIdx.x] - toff;
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < ROUNDS; r++) {
    if (loc[r] != 0xffffffffu) {
      const uint32_t d = (key[r] >> shift) & (RADIX - 1);
      const uint32_t p = tile_off[d] + whist[w][d] + loc[r];
      const uint64_t i = wbase + (uint64_t)r * 32 + lane;
      sk[p] = key[r];
      if (NP >= 1) sp0[p] = ident0 ? (uint32_t)i : p0_in[i];
      if (NP >= 2) sp1[p] = p1_in[i];
    }
  }
  __syncthreads();
  const uint64_t rem = n - tile_base;
  const uint32_t count = rem < (uint64_t)TILE ? (uint32_t)rem : (uint32_t)TILE;
  for (uint32_t p = threadIdx.x; p < count; p += TPB) {
    const uint32_t k = sk[p];
    const uint64_t g = (uint64_t)gbase[(k >> shift) & (RADIX - 1)] + p;
    if (keys_out) keys_out[g] = k;
    if (NP >= 1) p0_out[g] = sp0[p];
    if (NP >= 2) p1_out[g] = sp1[p];
  }
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

int bgnn_radix_sort(bgnn_ctx* ctx, const uint32_t* keys_in, uint64_t n, int key_bits,
                    const uint32_t* p0_in, int ident0, const uint32_t* p1_in, uint32_t* keys_out,
                    uint32_t* p0_out, uint32_t* p1_out) {
  if (n == 0) return BGNN_OK;
  if (n > 0xffffffffull)
    return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED, "radix sort limited to 2^32-1 items");
  const bool has0 = p0_in != nullptr || ident0;
  const bool has1 = p1_in != nullptr;
  if (has1 && !has0)
    return bgnn_set_error(ctx, BGNN_ERR_INVALID_ARG, "radix sort: payload 1 without payload 0");
  const int np = (has0 ? 1 : 0) + (has1 ? 1 : 0);
  const int passes = (key_bits + 7) / 8;
  if (passes == 0) {  // every key equal: the input order is the sorted order
    if (ident0) {
      k_iota<<<grid_for(ctx, n, 256), 256, 0, ctx->stream>>>(p0_out, n);
      BGNN_LAUNCHED(ctx);
    } else if (p0_in) {
      BGNN_CUDA(ctx, cudaMemcpyAsync(p0_out, p0_in, n * 4, cudaMemcpyDeviceToDevice, ctx->stream));
    }
    if (p1_in)
      BGNN_CUDA(ctx, cudaMemcpyAsync(p1_out, p1_in, n * 4, cudaMemcpyDeviceToDevice, ctx->stream));
    if (keys_out)
      BGNN_CUDA(ctx, cudaMemcpyAsync(keys_out, keys_in, n * 4, cudaMemcpyDeviceToDevice,
                                     ctx->stream));
    return BGNN_OK;
  }
  const uint64_t tiles = (n + TILE - 1) / TILE;
  DevTmp hist, kb[2], pb0[2], pb1[2];
  BGNN_TRY(bgnn_tmp_alloc(ctx, hist, tiles * RADIX * sizeof(uint32_t)));
  if (passes > 1) {
    for (int b = 0; b < 2 && b < passes - 1; b++) {
      BGNN_TRY(bgnn_tmp_alloc(ctx, kb[b], n * 4));
      if (has0) BGNN_TRY(bgnn_tmp_alloc(ctx, pb0[b], n * 4));
      if (has1) BGNN_TRY(bgnn_tmp_alloc(ctx, pb1[b], n * 4));
    }
  }
  const size_t dyn = (size_t)(1 + np) * TILE * sizeof(uint32_t);
  static_assert(TILE * 4 * 3 + (WARPS * RADIX + 2 * RADIX + WARPS) * 4 <= 227 * 1024,
                "radix tile fits in shared memory");
  const uint32_t* kin = keys_in;
  const uint32_t* pin0 = p0_in;
  const uint32_t* pin1 = p1_in;
  int ident = ident0;
  for (int p = 0; p < passes; p++) {
    const int shift = 8 * p;
    const bool last = p == passes - 1;
    uint32_t* kout = last ? keys_out : kb[p & 1].as<uint32_t>();
    uint32_t* pout0 = last ? p0_out : pb0[p & 1].as<uint32_t>();
    uint32_t* pout1 = last ? p1_out : pb1[p & 1].as<uint32_t>();
    k_radix_hist<<<(unsigned)tiles, TPB, 0, ctx->stream>>>(kin, n, shift, (uint32_t)tiles,
                                                            hist.as<uint32_t>());
    BGNN_LAUNCHED(ctx);
    BGNN_TRY(bgnn_exclusive_scan(ctx, hist.as<uint32_t>(), hist.as<uint32_t>(), tiles * RADIX));
    // the last pass skips writing keys when the caller does not want them
    switch (np) {
      case 0:
        k_radix_scatter<0><<<(unsigned)tiles, TPB, dyn, ctx->stream>>>(
            kin, nullptr, nullptr, 0, n, shift, (uint32_t)tiles, hist.as<uint32_t>(), kout,
            nullptr, nullptr);
        break;
      case 1:
        k_radix_scatter<1><<<(unsigned)tiles, TPB, dyn, ctx->stream>>>(
            kin, pin0, nullptr, ident, n, shift, (uint32_t)tiles, hist.as<uint32_t>(), kout,
            pout0, nullptr);
        break;
      default:
        BGNN_CUDA(ctx, cudaFuncSetAttribute(k_radix_scatter<2>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn));
        k_radix_scatter<2><<<(unsigned)tiles, TPB, dyn, ctx->stream>>>(
            kin, pin0, pin1, ident, n, shift, (uint32_t)tiles, hist.as<uint32_t>(), kout, pout0,
            pout1);
        break;
    }
    BGNN_LAUNCHED(ctx);
    kin = kout;  // (kout is only null on the last pass)
    pin0 = pout0;
    pin1 = pout1;
    ident = 0;
  }
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
