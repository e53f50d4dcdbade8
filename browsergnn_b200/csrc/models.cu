// Kernels behind the model zoo (src/models/*.ts) and the nn building blocks
// they use: Linear (src/nn/linear.ts), the softmax / log-softmax row ops
// (src/core/tensor.ts), training-mode Dropout and PReLU
// (src/nn/activation.ts), and the link scorers of ConceptPrerequisiteMapper.
//
// Arithmetic follows the reference's JS: a running sum in a local is a
// double; a value stored into a Float32Array is rounded to f32 once.  The
// f32 x f32 product is exact in double, so a double FMA reproduces
// `sum += a * b` bit for bit.
#include "bgnn_internal.cuh"

namespace {

// ---------------------------------------------------------------------------
// Linear.forward (src/nn/linear.ts:50-111): y[r, j] = f32(sum_i x[r, i] *
// w[j, i]) with the sum in double over i ascending, then f32(y + b[j]), then
// an optional activation (the next module of a Sequential, applied to the
// stored f32 value).  w is [n, k] ([outFeatures, inFeatures]).
//
// 64 x 64 output tile per 256-thread block, k staged through shared memory
// 16 at a time (both operands are k-contiguous, so each tile row is one
// coalesced 64-byte run), 4 x 4 double accumulators per thread.
// ---------------------------------------------------------------------------
constexpr int DN_T = 64;
constexpr int DN_K = 16;

__global__ void __launch_bounds__(256) k_dense(const float* __restrict__ x,
                                               const float* __restrict__ w, uint32_t m,
                                               uint32_t k, uint32_t n,
                                               const float* __restrict__ bias, int act,
                                               double act_param, float* __restrict__ out) {
  __shared__ float xs[DN_K][DN_T + 1];
  __shared__ float ws[DN_K][DN_T + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const uint64_t r0 = (uint64_t)blockIdx.y * DN_T;
  const uint64_t c0 = (uint64_t)blockIdx.x * DN_T;
  double acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0.0;
  for (uint32_t k0 = 0; k0 < k; k0 += DN_K) {
#pragma unroll
    for (int t = 0; t < (DN_T * DN_K) / 256; t++) {
      const int e = threadIdx.x + t * 256;
      const int row = e / DN_K, kk = e % DN_K;
      const uint64_t gr = r0 + row, gc = c0 + row;
      const uint32_t gk = k0 + kk;
      xs[kk][row] = (gr < m && gk < k) ? x[gr * k + gk] : 0.0f;
      ws[kk][row] = (gc < n && gk < k) ? w[gc * k + gk] : 0.0f;
    }
    __syncthreads();
    const int kn = (int)min((uint32_t)DN_K, k - k0);
    for (int kk = 0; kk < kn; kk++) {
      double xv[4], wv[4];
#pragma unroll
      for (int i = 0; i < 4; i++) xv[i] = (double)xs[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; j++) wv[j] = (double)ws[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = __fma_rn(xv[i], wv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint64_t r = r0 + ty + 16 * i;
    if (r >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint64_t c = c0 + tx + 16 * j;
      if (c >= n) continue;
      float y = __double2float_rn(acc[i][j]);
      if (bias) y = __fadd_rn(y, bias[c]);
      out[r * n + c] = apply_act(y, act, act_param);
    }
  }
}

// ---------------------------------------------------------------------------
// Tensor.softmax / logSoftmax along the last axis (src/core/tensor.ts:435-499),
// one block per row.  The max follows Math.max (NaN wins, +0 beats -0; both
// are order-free).  softmax stores f32(exp(x - max)) and divides the stored
// value by the double sum of the unrounded exps; logSoftmax subtracts
// max + log(sum).  The double sum is a fixed-shape block reduction instead of
// the reference's left-to-right loop; the two differ by a few ulps of a
// double, below the f32 rounding of the results.
// col_mask[c] != 0 replaces x[r, c] by mask_value first
// (LearningPathRecommender.ts:190-203 sets mastered scores to -1e9).
// ---------------------------------------------------------------------------
constexpr int SM_THREADS = 1024;

__device__ __forceinline__ double js_max(double a, double b) {
  if (a != a || b != b) return __longlong_as_double(0x7ff8000000000000LL);
  if (a == 0.0 && b == 0.0) return signbit(a) ? b : a;
  return a > b ? a : b;
}

__global__ void __launch_bounds__(SM_THREADS) k_softmax_rows(const float* __restrict__ x,
                                                             uint32_t cols,
                                                             const uint8_t* __restrict__ mask,
                                                             float mask_value, int log_sm,
                                                             float* __restrict__ out) {
  __shared__ double red[SM_THREADS / 32];
  __shared__ double bcast;
  const uint64_t base = (uint64_t)blockIdx.x * cols;
  auto xv = [&](uint32_t c) -> double {
    return (mask && mask[c]) ? (double)mask_value : (double)x[base + c];
  };
  const int lane = threadIdx.x % 32, wid = threadIdx.x / 32;
  // 1. max
  double mx = -INFINITY;
  for (uint32_t c = threadIdx.x; c < cols; c += SM_THREADS) mx = js_max(mx, xv(c));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = js_max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[wid] = mx;
  __syncthreads();
  if (wid == 0) {
    double v = lane < SM_THREADS / 32 ? red[lane] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = js_max(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) bcast = v;
  }
  __syncthreads();
  mx = bcast;
  __syncthreads();
  // 2. exps and their double sum
  double sum = 0.0;
  for (uint32_t c = threadIdx.x; c < cols; c += SM_THREADS) {
    const double e = exp(__dsub_rn(xv(c), mx));
    if (!log_sm) out[base + c] = __double2float_rn(e);
    sum = __dadd_rn(sum, e);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum = __dadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
  if (lane == 0) red[wid] = sum;
  __syncthreads();
  if (wid == 0) {
    double v = lane < SM_THREADS / 32 ? red[lane] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) bcast = v;
  }
  __syncthreads();
  sum = bcast;
  // 3. normalise
  if (log_sm) {
    const double lse = __dadd_rn(mx, log(sum));
    for (uint32_t c = threadIdx.x; c < cols; c += SM_THREADS)
      out[base + c] = __double2float_rn(__dsub_rn(xv(c), lse));
  } else {
    for (uint32_t c = threadIdx.x; c < cols; c += SM_THREADS)
      out[base + c] = __double2float_rn(__ddiv_rn((double)out[base + c], sum));
  }
}

// ---------------------------------------------------------------------------
// Training-mode Dropout (src/nn/activation.ts:207-245).  Math.random() is
// replaced by a counter-based draw: u_i = top 53 bits of the SplitMix64
// output for state seed + (i+1) * 0x9E3779B97F4A7C15, scaled to [0, 1).
// Element i is kept when u_i > p and scaled by 1/(1-p) in double.
// ---------------------------------------------------------------------------
__global__ void k_dropout(const float* __restrict__ x, uint64_t n, double p, double scale,
                          uint64_t seed, float* __restrict__ out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = bgnn_uniform(seed, i) > p ? __double2float_rn(__dmul_rn((double)x[i], scale)) : 0.0f;
}

// PReLU (src/nn/activation.ts:175-200): x > 0 ? x : a * x, with a = w[0]
// when there is one parameter, else w[i % numParams].
__global__ void k_prelu(const float* __restrict__ x, uint64_t n, const float* __restrict__ w,
                        uint32_t nw, float* __restrict__ out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    const float a = nw == 1 ? w[0] : w[i % nw];
    out[i] = v > 0.0f ? v : __fmul_rn(a, v);
  }
}

// ---------------------------------------------------------------------------
// ConceptPrerequisiteMapper.predictLinks (ConceptPrerequisiteMapper.ts:224-295)
// ---------------------------------------------------------------------------
// dot and bilinear: one thread per pair walks i ascending with a double sum
// of s[i] * t[i].  For bilinear, t is row tgt of wt = emb W^T, computed once
// per node by k_dense (each W*tgt vector depends only on the target node,
// and k_dense produces exactly the reference's f32(sum_j W[i,j] * tgt[j])).
__global__ void k_link_dot(const float* __restrict__ emb, const float* __restrict__ rhs,
                           uint32_t num_nodes, uint32_t d, const uint32_t* __restrict__ src,
                           const uint32_t* __restrict__ tgt, uint64_t pairs,
                           double* __restrict__ out, int* err) {
  for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < pairs;
       q += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t s = src[q], t = tgt[q];
    if (s >= num_nodes || t >= num_nodes) {
      dev_raise(err, DEVERR_INDEX, q, 20);
      out[q] = 0.0;
      continue;
    }
    const float* a = emb + (uint64_t)s * d;
    const float* b = rhs + (uint64_t)t * d;
    double score = 0.0;
    for (uint32_t i = 0; i < d; i++) score = __fma_rn((double)a[i], (double)b[i], score);
    out[q] = __ddiv_rn(1.0, __dadd_rn(1.0, exp(-score)));
  }
}

// mlp: one warp per pair.  The [src | tgt | f32(src*tgt)] input row goes to
// shared memory; lane l computes hidden units l, l+32, ... as double sums over
// the 3d inputs in order, stores f32, adds b1 in f32 and applies ReLU; lane 0
// then sums the hidden row against w2 in order, adds b2 and takes the sigmoid
// in double.  The Dropout between the two Linears is the identity in eval.
constexpr int LK_WARPS = 8;

__global__ void __launch_bounds__(LK_WARPS * 32) k_link_mlp(
    const float* __restrict__ emb, uint32_t num_nodes, uint32_t d,
    const uint32_t* __restrict__ src, const uint32_t* __restrict__ tgt, uint64_t pairs,
    const float* __restrict__ w1, const float* __restrict__ b1, const float* __restrict__ w2,
    const float* __restrict__ b2, double* __restrict__ out, int* err) {
  extern __shared__ float lk_smem[];
  const int lane = threadIdx.x % 32, wid = threadIdx.x / 32;
  float* in = lk_smem + (size_t)wid * 4 * d;  // [3d] input, then [d] hidden
  float* hid = in + 3 * d;
  for (uint64_t q = (uint64_t)blockIdx.x * LK_WARPS + wid; q < pairs;
       q += (uint64_t)gridDim.x * LK_WARPS) {
    const uint32_t s = src[q], t = tgt[q];
    if (s >= num_nodes || t >= num_nodes) {  // uniform over the warp
      if (lane == 0) {
        dev_raise(err, DEVERR_INDEX, q, 21);
        out[q] = 0.0;
      }
      continue;
    }
    for (uint32_t i = lane; i < d; i += 32) {
      const float a = emb[(uint64_t)s * d + i], b = emb[(uint64_t)t * d + i];
      in[i] = a;
      in[d + i] = b;
      in[2 * d + i] = __fmul_rn(a, b);
    }
    __syncwarp();
    const uint32_t k3 = 3 * d;
    for (uint32_t j = lane; j < d; j += 32) {
      const float* wr = w1 + (uint64_t)j * k3;
      double acc = 0.0;
      for (uint32_t i = 0; i < k3; i++) acc = __fma_rn((double)in[i], (double)wr[i], acc);
      float h = __double2float_rn(acc);
      if (b1) h = __fadd_rn(h, b1[j]);
      hid[j] = h > 0.0f ? h : 0.0f;
    }
    __syncwarp();
    if (lane == 0) {
      double acc = 0.0;
      for (uint32_t j = 0; j < d; j++) acc = __fma_rn((double)hid[j], (double)w2[j], acc);
      float o = __double2float_rn(acc);
      if (b2) o = __fadd_rn(o, b2[0]);
      out[q] = __ddiv_rn(1.0, __dadd_rn(1.0, exp(-(double)o)));
    }
    __syncwarp();
  }
}

unsigned grid_1d(bgnn_ctx* ctx, uint64_t n, int tpb) {
  uint64_t b = (n + tpb - 1) / tpb;
  const uint64_t cap = (uint64_t)ctx->num_sms * 16;
  if (b > cap) b = cap;
  return (unsigned)(b ? b : 1);
}

int check_ctx(bgnn_ctx* ctx) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess)
    return bgnn_set_error(ctx, BGNN_ERR_CUDA, "cudaSetDevice(%d): %s", ctx->device,
                          cudaGetErrorString(e));
  return BGNN_OK;
}

int run_dense(bgnn_ctx* ctx, const float* x, const float* w, uint32_t m, uint32_t k, uint32_t n,
              const float* bias, int act, double act_param, float* out) {
  if ((uint64_t)m * n == 0) return BGNN_OK;
  dim3 grid((n + DN_T - 1) / DN_T, (m + DN_T - 1) / DN_T);
  BGNN_REQUIRE(ctx, grid.y <= 65535u, "too many rows for one launch (%u)", m);
  k_dense<<<grid, 256, 0, ctx->stream>>>(x, w, m, k, n, bias, act, act_param, out);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

}  // namespace

// g[b, f] = sum of x[i, f] over the rows i of segment b, rows in order (one
// CTA per segment, a thread per feature; the same f32 adds in the same order
// as the scatter-add over a sorted batch vector)
__global__ void k_segment_sum(const float* __restrict__ x, uint32_t f,
                              const uint32_t* __restrict__ seg, float* __restrict__ out) {
  const uint32_t b = blockIdx.x;
  const uint32_t r0 = seg[b], r1 = seg[b + 1];
  for (uint32_t c = threadIdx.x; c < f; c += blockDim.x) {
    float acc = 0.0f;
    for (uint32_t r = r0; r < r1; r++) acc = __fadd_rn(acc, x[(uint64_t)r * f + c]);
    out[(uint64_t)b * f + c] = acc;
  }
}

extern "C" int bgnn_segment_sum(bgnn_ctx* ctx, const float* x, uint32_t f,
                                const uint32_t* seg_ptr, uint32_t num_graphs, float* out) {
  BGNN_TRY(check_ctx(ctx));
  if ((uint64_t)num_graphs * f == 0) return BGNN_OK;
  BGNN_REQUIRE(ctx, x && seg_ptr && out, "NULL argument");
  const unsigned threads = f >= 256 ? 256u : ((f + 31) / 32) * 32;
  k_segment_sum<<<num_graphs, threads, 0, ctx->stream>>>(x, f, seg_ptr, out);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

extern "C" int bgnn_dense(bgnn_ctx* ctx, const float* x, const float* w, uint32_t m, uint32_t k,
                          uint32_t n, const float* bias, int act, double act_param, float* out) {
  BGNN_TRY(check_ctx(ctx));
  BGNN_REQUIRE(ctx, act >= BGNN_ACT_NONE && act <= BGNN_ACT_SILU, "unknown activation %d", act);
  BGNN_REQUIRE(ctx, (x && w) || (uint64_t)m * k * n == 0, "NULL operand");
  BGNN_REQUIRE(ctx, out || (uint64_t)m * n == 0, "NULL out");
  return run_dense(ctx, x, w, m, k, n, bias, act, act_param, out);
}

extern "C" int bgnn_softmax_rows(bgnn_ctx* ctx, const float* x, uint32_t rows, uint32_t cols,
                                 const uint8_t* col_mask, float mask_value, int log_softmax,
                                 float* out) {
  BGNN_TRY(check_ctx(ctx));
  if ((uint64_t)rows * cols == 0) return BGNN_OK;
  BGNN_REQUIRE(ctx, x && out, "NULL argument");
  BGNN_REQUIRE(ctx, rows <= 0x7fffffffu, "too many rows");
  k_softmax_rows<<<rows, SM_THREADS, 0, ctx->stream>>>(x, cols, col_mask, mask_value,
                                                       log_softmax ? 1 : 0, out);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

extern "C" int bgnn_dropout(bgnn_ctx* ctx, const float* x, uint64_t n, double p, uint64_t seed,
                            float* out) {
  BGNN_TRY(check_ctx(ctx));
  // the reference's constructor rejects p outside [0, 1]; p = 1 divides by
  // zero in the scale but drops every element (u > 1 never holds)
  BGNN_REQUIRE(ctx, p >= 0.0 && p <= 1.0, "Dropout probability must be between 0 and 1");
  if (n == 0) return BGNN_OK;
  BGNN_REQUIRE(ctx, x && out, "NULL argument");
  const double scale = 1.0 / (1.0 - p);
  k_dropout<<<grid_1d(ctx, n, 256), 256, 0, ctx->stream>>>(x, n, p, scale, seed, out);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

extern "C" int bgnn_prelu(bgnn_ctx* ctx, const float* x, uint64_t n, const float* weight,
                          uint32_t num_params, float* out) {
  BGNN_TRY(check_ctx(ctx));
  if (n == 0) return BGNN_OK;
  BGNN_REQUIRE(ctx, x && out && weight && num_params > 0, "NULL argument or no parameters");
  k_prelu<<<grid_1d(ctx, n, 256), 256, 0, ctx->stream>>>(x, n, weight, num_params, out);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

extern "C" int bgnn_link_scores(bgnn_ctx* ctx, const float* emb, uint32_t num_nodes, uint32_t dim,
                                const uint32_t* src, const uint32_t* tgt, uint64_t num_pairs,
                                int mode, const float* w_bilinear, const float* w1,
                                const float* b1, const float* w2, const float* b2, double* out) {
  BGNN_TRY(check_ctx(ctx));
  BGNN_REQUIRE(ctx, mode >= BGNN_LINK_DOT && mode <= BGNN_LINK_MLP, "unknown link mode %d", mode);
  if (num_pairs == 0) return BGNN_OK;
  BGNN_REQUIRE(ctx, emb && src && tgt && out, "NULL argument");
  BGNN_REQUIRE(ctx, dim > 0, "zero embedding width");
  if (mode == BGNN_LINK_DOT) {
    k_link_dot<<<grid_1d(ctx, num_pairs, 256), 256, 0, ctx->stream>>>(
        emb, emb, num_nodes, dim, src, tgt, num_pairs, out, ctx->d_err);
    BGNN_LAUNCHED(ctx);
    return BGNN_OK;
  }
  if (mode == BGNN_LINK_BILINEAR) {
    BGNN_REQUIRE(ctx, w_bilinear, "NULL bilinear weight");
    DevTmp wt;
    BGNN_TRY(bgnn_tmp_alloc(ctx, wt, (size_t)num_nodes * dim * 4));
    BGNN_TRY(run_dense(ctx, emb, w_bilinear, num_nodes, dim, dim, nullptr, BGNN_ACT_NONE, 0.0,
                       wt.as<float>()));
    k_link_dot<<<grid_1d(ctx, num_pairs, 256), 256, 0, ctx->stream>>>(
        emb, wt.as<float>(), num_nodes, dim, src, tgt, num_pairs, out, ctx->d_err);
    BGNN_LAUNCHED(ctx);
    return BGNN_OK;
  }
  BGNN_REQUIRE(ctx, w1 && w2, "NULL mlp weight");
  const size_t smem = (size_t)LK_WARPS * 4 * dim * sizeof(float);
  BGNN_REQUIRE(ctx, smem <= 200u * 1024u, "embedding width %u too large for the mlp scorer", dim);
  BGNN_CUDA(ctx, cudaFuncSetAttribute(k_link_mlp, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
  const uint64_t blocks = (num_pairs + LK_WARPS - 1) / LK_WARPS;
  const unsigned grid = (unsigned)(blocks < (uint64_t)ctx->num_sms * 8 ? blocks
                                                                       : (uint64_t)ctx->num_sms * 8);
  k_link_mlp<<<grid, LK_WARPS * 32, smem, ctx->stream>>>(emb, num_nodes, dim, src, tgt, num_pairs,
                                                         w1, b1, w2, b2, out, ctx->d_err);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}
