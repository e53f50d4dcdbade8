// GATConv message passing after the X*W transform (src/layers/gat.ts:115-254),
// fused per destination row: edge scores with LeakyReLU, exp(score - 10),
// the per-destination softmax denominator, normalisation and the weighted
// aggregation (concat or head mean), + bias and the following activation.
//
// One warp owns one destination row and walks its incoming edges in COO
// order (destination CSR), so every per-(row, head) and per-(row, feature)
// reduction runs in the reference's edge order.  All JS arithmetic is
// reproduced in double with the reference's f32 store points:
//   score   = sum_f (as*hs + ad*hd)   f64, sequential over f      (:147-155)
//   score  *= slope if score < 0      f64                          (:158-160)
//   alpha   = f32(score)                                           (:162)
//   ex      = exp(f64(alpha) - 10);  alphaExp = f32(ex)            (:175-176)
//   sum     = f32(sum + ex)           edge order                   (:178)
//   alpha'  = f32(alphaExp / sum) if sum > 0                       (:187-190)
//   concat: out = f32(out + alpha'*h)          (:222)
//   mean:   out = f32(out + alpha'*h / heads)  (:239)
// Dropout is a training-time op (Math.random) and is not offered here.
// The softmax keeps the reference's constant shift of 10 rather than a max
// shift, so exp overflows exactly where the reference's does.
#include <mutex>

#include "bgnn_internal.cuh"

namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr int GAT_WARPS = 8;

struct GatArgs {
  const uint32_t* row_ptr;
  const uint32_t* src_of;
  const float* h;
  const float* att_src;
  const float* att_dst;
  const float* bias;
  float* out;
  float* scratch;      // [E_slots, heads]: exp values, then normalised weights
  uint64_t num_edges;  // tail slots live at num_edges + row
  uint32_t n_rows;
  int heads, c, lpe;
  double slope;
  int concat, tail, act;
  double act_param;
  // training-mode attention dropout (gat.ts:194-203): drop_p == 0 disables
  const uint32_t* eid;  // COO edge id of each CSR slot (NULL: the slot itself)
  double drop_p;
  uint64_t seed;
};

__device__ __forceinline__ double shfl_d(double v, int src) {
  int lo = __double2loint(v), hi = __double2hiint(v);
  lo = __shfl_sync(FULL, lo, src);
  hi = __shfl_sync(FULL, hi, src);
  return __hiloint2double(hi, lo);
}

template <int KO>
__global__ void __launch_bounds__(GAT_WARPS * 32) k_gat(const GatArgs a) {
  __shared__ float s_sum[GAT_WARPS][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const uint32_t row = blockIdx.x * GAT_WARPS + w;
  if (row >= a.n_rows) return;  // warp-uniform
  const int H = a.heads, C = a.c, HC = H * C;
  const int lpe = a.lpe, epr = 32 / lpe;
  const int slot = lane / lpe, hl = lane % lpe;
  const bool has_head = hl < H;
  const uint32_t b = a.row_ptr[row];
  const uint32_t deg = a.row_ptr[row + 1] - b;
  const uint32_t total = deg + (a.tail ? 1u : 0u);
  const float* hd_row = a.h + (int64_t)row * HC;

  // ---- pass 1: scores, exp, per-head running sum in edge order ----
  float sum = 0.0f;
  for (uint32_t j0 = 0; j0 < total; j0 += epr) {
    const uint32_t j = j0 + slot;
    double ex = 0.0;
    if (j < total && has_head) {
      const uint32_t s = j < deg ? a.src_of[b + j] : row;
      const float* hs_row = a.h + (int64_t)s * HC + hl * C;
      const float* hdr = hd_row + hl * C;
      const float* as = a.att_src + hl * C;
      const float* ad = a.att_dst + hl * C;
      double score = 0.0;
      for (int f = 0; f < C; f++) {
        const double t = __dadd_rn(__dmul_rn((double)__ldg(as + f), (double)__ldg(hs_row + f)),
                                   __dmul_rn((double)__ldg(ad + f), (double)__ldg(hdr + f)));
        score = __dadd_rn(score, t);
      }
      if (score < 0.0) score = __dmul_rn(score, a.slope);
      const float alpha = __double2float_rn(score);
      ex = exp(__dsub_rn((double)alpha, 10.0));
      const uint64_t slot_idx = j < deg ? (uint64_t)b + j : a.num_edges + row;
      a.scratch[slot_idx * H + hl] = __double2float_rn(ex);
    }
    for (int s2 = 0; s2 < epr; s2++) {
      const double e2 = shfl_d(ex, s2 * lpe + hl);
      if (j0 + (uint32_t)s2 < total) sum = __double2float_rn(__dadd_rn((double)sum, e2));
    }
  }
  if (slot == 0 && has_head) s_sum[w][hl] = sum;
  __syncwarp();

  // ---- pass 1.5: alpha' = f32(alphaExp / sum) when sum > 0 ----
  for (uint32_t j0 = 0; j0 < total; j0 += epr) {
    const uint32_t j = j0 + slot;
    if (j < total && has_head) {
      const uint64_t slot_idx = j < deg ? (uint64_t)b + j : a.num_edges + row;
      const float sm = s_sum[w][hl];
      float* p = a.scratch + slot_idx * H + hl;
      if (sm > 0.0f) *p = __fdiv_rn(*p, sm);
      if (a.drop_p > 0.0) {
        // entry (edge e, head h) of alphaExp sits at e*heads + h in the
        // reference, with the appended self-loops numbered after the edges
        const uint64_t e = j < deg ? (a.eid ? (uint64_t)a.eid[b + j] : (uint64_t)b + j)
                                   : a.num_edges + row;
        const double u = bgnn_uniform(a.seed, e * (uint64_t)H + (uint64_t)hl);
        *p = u < a.drop_p ? 0.0f : __double2float_rn(__ddiv_rn((double)*p, 1.0 - a.drop_p));
      }
    }
  }
  __syncwarp();

  // ---- pass 2: weighted aggregation in edge order ----
  const int OD = a.concat ? HC : C;
  float accf[KO];
#pragma unroll
  for (int k = 0; k < KO; k++) accf[k] = 0.0f;
  for (uint32_t j0 = 0; j0 < total; j0 += 32) {
    const uint32_t jj = j0 + lane;
    const uint32_t my_s = jj < deg ? a.src_of[b + jj] : row;
    const uint32_t cnt = min(32u, total - j0);
    for (uint32_t t = 0; t < cnt; t++) {
      const uint32_t j = j0 + t;
      const uint32_t s = __shfl_sync(FULL, my_s, (int)t);
      const uint64_t slot_idx = j < deg ? (uint64_t)b + j : a.num_edges + row;
      const float* al = a.scratch + slot_idx * H;
      const float* hs = a.h + (int64_t)s * HC;
#pragma unroll
      for (int k = 0; k < KO; k++) {
        const int o = lane + 32 * k;
        if (o < OD) {
          if (a.concat) {
            const int hh = o / C;
            accf[k] = __double2float_rn(
                __fma_rn((double)__ldg(al + hh), (double)__ldg(hs + o), (double)accf[k]));
          } else {
            for (int hh = 0; hh < H; hh++) {
              const double p = __dmul_rn((double)__ldg(al + hh), (double)__ldg(hs + hh * C + o));
              accf[k] = __double2float_rn(__dadd_rn((double)accf[k], __ddiv_rn(p, (double)H)));
            }
          }
        }
      }
    }
  }
  float* orow = a.out + (int64_t)row * OD;
#pragma unroll
  for (int k = 0; k < KO; k++) {
    const int o = lane + 32 * k;
    if (o < OD) {
      float v = accf[k];
      if (a.bias) v = __fadd_rn(v, a.bias[o]);
      orow[o] = apply_act(v, a.act, a.act_param);
    }
  }
}

template <int KO>
int launch_gat(bgnn_ctx* ctx, const GatArgs& a) {
  const unsigned blocks = (a.n_rows + GAT_WARPS - 1) / GAT_WARPS;
  k_gat<KO><<<blocks, GAT_WARPS * 32, 0, ctx->stream>>>(a);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

}  // namespace

int bgnn_run_gat(bgnn_ctx* ctx, const bgnn_graph* g, const float* h, uint32_t heads, uint32_t c,
                 const float* att_src, const float* att_dst, double slope, int concat, int tail,
                 const float* bias, int act, double act_param, float* out, double drop_p,
                 uint64_t seed) {
  if (heads == 0 || c == 0)
    return bgnn_set_error(ctx, BGNN_ERR_INVALID_ARG, "heads and channels must be positive");
  if (heads > 32)
    return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED, "GAT supports up to 32 heads (got %u)", heads);
  const uint32_t od = concat ? heads * c : c;
  if (od > 256)
    return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED, "GAT output width %u exceeds 256", od);
  if (g->n_dst == 0) return BGNN_OK;
  if (g->n_src != g->n_dst)
    return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED, "GAT needs a square graph");
  const uint64_t slots = g->num_edges + (tail ? g->n_dst : 0);
  DevTmp scratch;
  BGNN_TRY(bgnn_tmp_alloc(ctx, scratch, (slots ? slots : 1) * heads * sizeof(float)));
  GatArgs a;
  a.row_ptr = g->row_ptr;
  a.src_of = g->src_of;
  a.h = h;
  a.att_src = att_src;
  a.att_dst = att_dst;
  a.bias = bias;
  a.out = out;
  a.scratch = scratch.as<float>();
  a.num_edges = g->num_edges;
  a.n_rows = g->n_dst;
  a.heads = (int)heads;
  a.c = (int)c;
  int lpe = 1;
  while (lpe < (int)heads) lpe <<= 1;
  a.lpe = lpe;
  a.slope = slope;
  a.concat = concat;
  a.tail = tail;
  a.act = act;
  a.act_param = act_param;
  a.eid = g->eid;
  a.drop_p = drop_p;
  a.seed = seed;
  const int ko = (int)((od + 31) / 32);
  if (ko <= 1) return launch_gat<1>(ctx, a);
  if (ko <= 2) return launch_gat<2>(ctx, a);
  if (ko <= 4) return launch_gat<4>(ctx, a);
  return launch_gat<8>(ctx, a);
}

// ---------------------------------------------------------------------------
// Allocation-free GAT: the same kernel, with its per-edge attention scratch
// in a fixed device array instead of a stream-ordered allocation.
//
// For callers that must not allocate device memory once they are running:
// an inference server that reserves its whole memory budget at start-up and
// forbids allocation afterwards, or a host application (a Node-API addon
// embedded in a JavaScript runtime, for instance) whose device memory is
// owned by someone else.  The caller still provides every input and output.
//
// The array holds BGNN_GAT_NOALLOC_MAX_FLOATS floats (16 MiB); every GPU that
// loads this library keeps it until the process exits.  A call needs
// (edges + appended self-loops) * heads floats.  All calls share the one
// array, so calls whose kernels overlap on the GPU race on it; the kernel
// writes each slot before reading it, so nothing needs clearing between calls.
// ---------------------------------------------------------------------------
#define BGNN_GAT_NOALLOC_MAX_FLOATS (4u << 20)

static __device__ __align__(256) float g_gat_noalloc_scratch[BGNN_GAT_NOALLOC_MAX_FLOATS];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kMaxDevices] = {};

// The array's name in host code is only a host-side stand-in; the device
// address comes from cudaGetSymbolAddress, looked up once per device with
// that device current (on the first call on the device).
int noalloc_scratch(bgnn_ctx* ctx, float** out) {
  if (ctx->device < 0 || ctx->device >= kMaxDevices)
    return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED, "device ordinal %d out of range", ctx->device);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[ctx->device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_gat_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return bgnn_set_error(ctx, BGNN_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed: %s",
                            cudaGetErrorString(e));
    g_noalloc_ptr[ctx->device] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[ctx->device];
  return BGNN_OK;
}
}  // namespace

extern "C" int bgnn_gat_noalloc(bgnn_ctx* ctx, const bgnn_graph* g, const float* h,
                                uint32_t heads, uint32_t c, const float* att_src,
                                const float* att_dst, double negative_slope, int concat,
                                int add_self_loops, const float* bias, int act,
                                double act_param, float* out) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  BGNN_REQUIRE(ctx, g != nullptr, "NULL graph");
  BGNN_REQUIRE(ctx, h && att_src && att_dst && out, "NULL argument");
  BGNN_REQUIRE(ctx, act >= BGNN_ACT_NONE && act <= BGNN_ACT_SILU, "unknown activation %d", act);
  BGNN_REQUIRE(ctx, heads > 0 && c > 0, "heads and channels must be positive");
  if (heads > 32)
    return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED, "GAT supports up to 32 heads (got %u)", heads);
  const uint32_t od = concat ? heads * c : c;
  if (od > 256)
    return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED, "GAT output width %u exceeds 256", od);
  BGNN_REQUIRE(ctx, g->n_src == g->n_dst, "GAT needs a square graph");
  const int tail = (add_self_loops && !g->has_self_loops) ? 1 : 0;  // gat.ts:116-118
  const uint64_t need = (g->num_edges + (tail ? g->n_dst : 0)) * (uint64_t)heads;
  if (need > BGNN_GAT_NOALLOC_MAX_FLOATS)
    return bgnn_set_error(ctx, BGNN_ERR_INVALID_ARG,
                          "allocation-free GAT needs %llu scratch floats; the limit is %u "
                          "((edges + self-loops) * heads)",
                          (unsigned long long)need, BGNN_GAT_NOALLOC_MAX_FLOATS);
  if (g->n_dst == 0) return BGNN_OK;
  float* scratch = nullptr;
  BGNN_TRY(noalloc_scratch(ctx, &scratch));
  GatArgs a;
  a.row_ptr = g->row_ptr;
  a.src_of = g->src_of;
  a.h = h;
  a.att_src = att_src;
  a.att_dst = att_dst;
  a.bias = bias;
  a.out = out;
  a.scratch = scratch;
  a.num_edges = g->num_edges;
  a.n_rows = g->n_dst;
  a.heads = (int)heads;
  a.c = (int)c;
  int lpe = 1;
  while (lpe < (int)heads) lpe <<= 1;
  a.lpe = lpe;
  a.slope = negative_slope;
  a.concat = concat;
  a.tail = tail;
  a.act = act;
  a.act_param = act_param;
  a.eid = g->eid;
  a.drop_p = 0.0;
  a.seed = 0;
  const int ko = (int)((od + 31) / 32);
  if (ko <= 1) return launch_gat<1>(ctx, a);
  if (ko <= 2) return launch_gat<2>(ctx, a);
  if (ko <= 4) return launch_gat<4>(ctx, a);
  return launch_gat<8>(ctx, a);
}
