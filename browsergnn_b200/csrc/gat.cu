// GATConv message passing after the X*W transform (src/layers/gat.ts:115-254),
// fused per destination row: edge scores with LeakyReLU, exp(score - 10),
// the per-destination softmax denominator, normalisation and the weighted
// aggregation (concat or head mean), + bias and the following activation.
//
// Scores are computed edge-parallel (k_gat_alpha); then one warp owns one
// destination row and walks its incoming edges in COO order (destination
// CSR), so every per-(row, head) and per-(row, feature) reduction runs in the
// reference's edge order.  All JS arithmetic is
// reproduced in double with the reference's f32 store points:
//   score   = sum_f (as*hs + ad*hd)   f64, sequential over f      (:147-155)
//   score  *= slope if score < 0      f64                          (:158-160)
//   alpha   = f32(score)                                           (:162)
//   ex      = exp(f64(alpha) - 10);  alphaExp = f32(ex)            (:175-176)
//   sum     = f32(sum + ex)           edge order                   (:178)
//   alpha'  = f32(alphaExp / sum) if sum > 0                       (:187-190)
//   concat: out = f32(out + alpha'*h)          (:222)
//   mean:   out = f32(out + alpha'*h / heads)  (:239)
// Training-mode attention dropout (:194-203) draws from a counter-based
// generator instead of Math.random (bgnn_gat_train).
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
  const bgnn_graph* graph;  // for the lazily built slot -> row map
  // rows of at least heavy_threshold edges go to k_gat_heavy (a CTA each)
  const uint32_t* heavy_rows;
  uint32_t n_heavy, heavy_threshold;
};

__device__ __forceinline__ double shfl_d(double v, int src) {
  int lo = __double2loint(v), hi = __double2hiint(v);
  lo = __shfl_sync(FULL, lo, src);
  hi = __shfl_sync(FULL, hi, src);
  return __hiloint2double(hi, lo);
}

// Edge scores, one thread per (CSR slot, head), appended self-loop slots
// after the graph's edges: alpha = f32(LeakyReLU(score)) into the scratch.
// Consecutive threads take consecutive heads of one slot, so the H rows are
// read as contiguous runs.  Computing every score here, spread over the whole
// GPU, keeps a hub row's thousands of scores off its one warp below.
__global__ void k_gat_alpha(const GatArgs a, const uint32_t* __restrict__ dst_of) {
  const int H = a.heads, C = a.c, HC = H * C;
  const uint64_t slots = a.num_edges + (a.tail ? a.n_rows : 0u);
  const uint64_t total = slots * (uint64_t)H;
  for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t slot = idx / H;
    const int hl = (int)(idx - slot * H);
    uint32_t s, d;
    if (slot < a.num_edges) {
      s = a.src_of[slot];
      d = dst_of[slot];
    } else {
      s = d = (uint32_t)(slot - a.num_edges);
    }
    const float* hs_row = a.h + (int64_t)s * HC + hl * C;
    const float* hd_row = a.h + (int64_t)d * HC + hl * C;
    const float* as = a.att_src + hl * C;
    const float* ad = a.att_dst + hl * C;
    double score = 0.0;
#pragma unroll 4
    for (int f = 0; f < C; f++) {
      const double t = __dadd_rn(__dmul_rn((double)__ldg(as + f), (double)__ldg(hs_row + f)),
                                 __dmul_rn((double)__ldg(ad + f), (double)__ldg(hd_row + f)));
      score = __dadd_rn(score, t);
    }
    if (score < 0.0) score = __dmul_rn(score, a.slope);
    a.scratch[idx] = __double2float_rn(score);
  }
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
  if (a.n_heavy && deg >= a.heavy_threshold) return;  // k_gat_heavy's row (warp-uniform)
  const uint32_t total = deg + (a.tail ? 1u : 0u);
  auto slot_of = [&](uint32_t j) -> uint64_t {
    return j < deg ? (uint64_t)b + j : a.num_edges + row;
  };

  // ---- pass 1: exp(alpha - 10), stored f32, and the per-head running sum in
  // edge order.  The alphas of U rounds are loaded before any is used, so a
  // long row waits on memory once per U rounds.
  constexpr int U = 8;
  float sum = 0.0f;
  for (uint32_t j0 = 0; j0 < total; j0 += (uint32_t)(epr * U)) {
    float al[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const uint32_t j = j0 + (uint32_t)(u * epr + slot);
      al[u] = (j < total && has_head) ? a.scratch[slot_of(j) * H + hl] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const uint32_t jb = j0 + (uint32_t)(u * epr);
      if (jb >= total) break;  // warp-uniform
      const uint32_t j = jb + slot;
      double ex = 0.0;
      if (j < total && has_head) {
        ex = exp(__dsub_rn((double)al[u], 10.0));
        a.scratch[slot_of(j) * H + hl] = __double2float_rn(ex);
      }
      for (int s2 = 0; s2 < epr; s2++) {
        const double e2 = shfl_d(ex, s2 * lpe + hl);
        if (jb + (uint32_t)s2 < total) sum = __double2float_rn(__dadd_rn((double)sum, e2));
      }
    }
  }
  if (slot == 0 && has_head) s_sum[w][hl] = sum;
  __syncwarp();

  // ---- pass 1.5: alpha' = f32(alphaExp / sum) when sum > 0 (:187-190),
  // then the training dropout of entry (edge e, head h), which sits at
  // e*heads + h in the reference with the appended self-loops numbered after
  // the edges (:194-203) ----
  for (uint32_t j0 = 0; j0 < total; j0 += (uint32_t)(epr * U)) {
    float ev[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const uint32_t j = j0 + (uint32_t)(u * epr + slot);
      ev[u] = (j < total && has_head) ? a.scratch[slot_of(j) * H + hl] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const uint32_t j = j0 + (uint32_t)(u * epr + slot);
      if (j < total && has_head) {
        const float sm = s_sum[w][hl];
        float v = sm > 0.0f ? __fdiv_rn(ev[u], sm) : ev[u];
        if (a.drop_p > 0.0) {
          const uint64_t e = j < deg ? (a.eid ? (uint64_t)a.eid[b + j] : (uint64_t)b + j)
                                     : a.num_edges + row;
          const double r = bgnn_uniform(a.seed, e * (uint64_t)H + (uint64_t)hl);
          v = r < a.drop_p ? 0.0f : __double2float_rn(__ddiv_rn((double)v, 1.0 - a.drop_p));
        }
        a.scratch[slot_of(j) * H + hl] = v;
      }
    }
  }
  __syncwarp();

  // ---- pass 2: weighted aggregation in edge order.  Per block of V edges
  // the lane loads every weight and H value it needs first, then runs its
  // add chains over them in order. ----
  const int OD = a.concat ? HC : C;
  constexpr int V = KO <= 2 ? 8 : (KO == 4 ? 4 : 2);
  float accf[KO];
#pragma unroll
  for (int k = 0; k < KO; k++) accf[k] = 0.0f;
  for (uint32_t j0 = 0; j0 < total; j0 += 32) {
    const uint32_t jj = j0 + lane;
    const uint32_t my_s = jj < deg ? a.src_of[b + jj] : row;
    const uint32_t cnt = min(32u, total - j0);
    for (uint32_t t0 = 0; t0 < cnt; t0 += V) {
      if (a.concat) {
        float hv[V][KO], av[V][KO];
#pragma unroll
        for (int u = 0; u < V; u++) {
          const uint32_t t = t0 + (uint32_t)u;
          const uint32_t s = __shfl_sync(FULL, my_s, (int)(t < cnt ? t : 0));
          const float* al = a.scratch + slot_of(j0 + t) * H;
          const float* hs = a.h + (int64_t)s * HC;
#pragma unroll
          for (int k = 0; k < KO; k++) {
            const int o = lane + 32 * k;
            const bool live = t < cnt && o < OD;
            hv[u][k] = live ? __ldg(hs + o) : 0.0f;
            av[u][k] = live ? al[o / C] : 0.0f;
          }
        }
#pragma unroll
        for (int u = 0; u < V; u++) {
          if (t0 + (uint32_t)u >= cnt) break;  // warp-uniform
#pragma unroll
          for (int k = 0; k < KO; k++) {
            const int o = lane + 32 * k;
            if (o < OD)
              accf[k] = __double2float_rn(
                  __fma_rn((double)av[u][k], (double)hv[u][k], (double)accf[k]));
          }
        }
      } else {
        for (uint32_t t = t0; t < min(cnt, t0 + (uint32_t)V); t++) {
          const uint32_t s = __shfl_sync(FULL, my_s, (int)t);
          const float* al = a.scratch + slot_of(j0 + t) * H;
          const float* hs = a.h + (int64_t)s * HC;
#pragma unroll
          for (int k = 0; k < KO; k++) {
            const int o = lane + 32 * k;
            if (o < OD) {
              for (int hh = 0; hh < H; hh++) {
                const double p = __dmul_rn((double)al[hh], (double)__ldg(hs + hh * C + o));
                accf[k] = __double2float_rn(__dadd_rn((double)accf[k], __ddiv_rn(p, (double)H)));
              }
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

// ---------------------------------------------------------------------------
// One CTA per heavy row (the graph's rows of >= 256 edges).  A warp walking a
// hub row alone spends milliseconds on its serial chains; here the row's
// exps, normalisation and row staging are spread over the CTA, and only the
// chains that must run in edge order stay serial, each on one thread reading
// shared memory:
//   A  ex = exp(alpha - 10) for (edge, head) items of a chunk, in parallel;
//      thread h then adds its head's chunk into the running sum in order
//   B  alpha' = f32(ex / sum) (+ training dropout), in parallel
//   C  the chunk's H rows and weights staged in shared memory; thread o adds
//      its feature's terms in edge order
// ---------------------------------------------------------------------------
constexpr int GH_THREADS = 256;
constexpr int GH_ITEMS = 2048;    // (edge, head) items per chunk in pass A
constexpr int GH_STAGE = 16384;   // floats of H rows per chunk in pass C
constexpr int GH_MAXE = 64;       // edges per chunk in pass C

inline size_t gat_heavy_smem() {
  return (size_t)GH_ITEMS * 8 + 32 * 4 + (size_t)GH_MAXE * 32 * 4 + (size_t)GH_STAGE * 4;
}

__global__ void __launch_bounds__(GH_THREADS) k_gat_heavy(const GatArgs a) {
  extern __shared__ double gh_smem[];
  double* exs = gh_smem;                                         // [GH_ITEMS]
  float* sums = reinterpret_cast<float*>(exs + GH_ITEMS);        // [32]
  float* wst = sums + 32;                                        // [GH_MAXE * H]
  float* hst = wst + GH_MAXE * 32;                               // [ae * HC]
  const int tid = threadIdx.x;
  const int H = a.heads, C = a.c, HC = H * C;
  const int OD = a.concat ? HC : C;
  const uint32_t row = a.heavy_rows[blockIdx.x];
  const uint32_t b = a.row_ptr[row];
  const uint32_t deg = a.row_ptr[row + 1] - b;
  const uint32_t total = deg + (a.tail ? 1u : 0u);
  auto slot_of = [&](uint32_t j) -> uint64_t {
    return j < deg ? (uint64_t)b + j : a.num_edges + row;
  };

  // A: exps and the per-head running sums, chunk by chunk in edge order
  const uint32_t ch = (uint32_t)(GH_ITEMS / H);
  float sum = 0.0f;
  for (uint32_t c0 = 0; c0 < total; c0 += ch) {
    const uint32_t cnt = min(ch, total - c0);
    for (uint32_t i = tid; i < cnt * (uint32_t)H; i += GH_THREADS) {
      const uint32_t j = c0 + i / (uint32_t)H, h = i % (uint32_t)H;
      float* p = a.scratch + slot_of(j) * H + h;
      const double ex = exp(__dsub_rn((double)*p, 10.0));
      *p = __double2float_rn(ex);
      exs[i] = ex;
    }
    __syncthreads();
    if (tid < H) {
      uint32_t jj = 0;
      for (; jj + 8 <= cnt; jj += 8) {
        double v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) v[u] = exs[(jj + u) * H + tid];
#pragma unroll
        for (int u = 0; u < 8; u++) sum = __double2float_rn(__dadd_rn((double)sum, v[u]));
      }
      for (; jj < cnt; jj++) sum = __double2float_rn(__dadd_rn((double)sum, exs[jj * H + tid]));
    }
    __syncthreads();
  }
  if (tid < H) sums[tid] = sum;
  __syncthreads();

  // B: normalise (+ dropout) every (edge, head) entry of the row
  for (uint32_t i = tid; i < total * (uint32_t)H; i += GH_THREADS) {
    const uint32_t j = i / (uint32_t)H, h = i % (uint32_t)H;
    float* p = a.scratch + slot_of(j) * H + h;
    const float sm = sums[h];
    float v = sm > 0.0f ? __fdiv_rn(*p, sm) : *p;
    if (a.drop_p > 0.0) {
      const uint64_t e = j < deg ? (a.eid ? (uint64_t)a.eid[b + j] : (uint64_t)b + j)
                                 : a.num_edges + row;
      const double r = bgnn_uniform(a.seed, e * (uint64_t)H + (uint64_t)h);
      v = r < a.drop_p ? 0.0f : __double2float_rn(__ddiv_rn((double)v, 1.0 - a.drop_p));
    }
    *p = v;
  }
  __syncthreads();

  // C: weighted aggregation, chunks of ae edges staged in shared memory
  const uint32_t ae = (uint32_t)min(GH_MAXE, GH_STAGE / HC);
  float acc = 0.0f;
  for (uint32_t c0 = 0; c0 < total; c0 += ae) {
    const uint32_t cnt = min(ae, total - c0);
    for (uint32_t i = tid; i < cnt * (uint32_t)HC; i += GH_THREADS) {
      const uint32_t j = i / (uint32_t)HC, f = i % (uint32_t)HC;
      const uint32_t s = c0 + j < deg ? a.src_of[b + c0 + j] : row;
      hst[i] = a.h[(int64_t)s * HC + f];
    }
    for (uint32_t i = tid; i < cnt * (uint32_t)H; i += GH_THREADS)
      wst[i] = a.scratch[slot_of(c0 + i / (uint32_t)H) * H + i % (uint32_t)H];
    __syncthreads();
    if (tid < OD) {
      if (a.concat) {
        const int hh = tid / C;
        for (uint32_t jj = 0; jj < cnt; jj++)
          acc = __double2float_rn(__fma_rn((double)wst[jj * H + hh], (double)hst[jj * HC + tid],
                                           (double)acc));
      } else {
        for (uint32_t jj = 0; jj < cnt; jj++)
          for (int hh = 0; hh < H; hh++) {
            const double p = __dmul_rn((double)wst[jj * H + hh], (double)hst[jj * HC + hh * C + tid]);
            acc = __double2float_rn(__dadd_rn((double)acc, __ddiv_rn(p, (double)H)));
          }
      }
    }
    __syncthreads();
  }
  if (tid < OD) {
    float v = acc;
    if (a.bias) v = __fadd_rn(v, a.bias[tid]);
    a.out[(int64_t)row * OD + tid] = apply_act(v, a.act, a.act_param);
  }
}

// dst_given: a slot -> destination row map the caller already built (the
// allocation-free entry point); otherwise the graph's own, built on first use
template <int KO>
int launch_gat(bgnn_ctx* ctx, const GatArgs& a, const uint32_t* dst_given = nullptr) {
  const uint32_t* dst_of = dst_given;
  if (dst_of == nullptr)
    BGNN_TRY(bgnn_graph_dst_of(ctx, const_cast<bgnn_graph*>(a.graph), &dst_of));
  const uint64_t items = (a.num_edges + (a.tail ? a.n_rows : 0u)) * (uint64_t)a.heads;
  uint64_t ab = (items + 255) / 256;
  if (ab > (uint64_t)ctx->num_sms * 32) ab = (uint64_t)ctx->num_sms * 32;
  k_gat_alpha<<<(unsigned)(ab ? ab : 1), 256, 0, ctx->stream>>>(a, dst_of);
  BGNN_LAUNCHED(ctx);
  const unsigned blocks = (a.n_rows + GAT_WARPS - 1) / GAT_WARPS;
  if (a.n_heavy) {
    // heavy rows on the aux stream, next to the warp-per-row launch
    const size_t hs = gat_heavy_smem();
    BGNN_CUDA(ctx, cudaFuncSetAttribute(k_gat_heavy, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)hs));
    BGNN_CUDA(ctx, cudaEventRecord(ctx->ev_fork, ctx->stream));
    BGNN_CUDA(ctx, cudaStreamWaitEvent(ctx->aux_stream, ctx->ev_fork, 0));
    k_gat_heavy<<<a.n_heavy, GH_THREADS, hs, ctx->aux_stream>>>(a);
    BGNN_LAUNCHED(ctx);
    BGNN_CUDA(ctx, cudaEventRecord(ctx->ev_join, ctx->aux_stream));
  }
  k_gat<KO><<<blocks, GAT_WARPS * 32, 0, ctx->stream>>>(a);
  BGNN_LAUNCHED(ctx);
  if (a.n_heavy) BGNN_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, ctx->ev_join, 0));
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
  a.graph = g;
  a.heavy_rows = g->heavy_rows;
  a.n_heavy = g->heavy_rows ? g->n_heavy : 0u;
  a.heavy_threshold = g->heavy_threshold;
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
// The array holds BGNN_GAT_NOALLOC_MAX_FLOATS 4-byte words (16 MiB); every
// GPU that loads this library keeps it until the process exits.  A call
// needs (edges + appended self-loops) * heads words for the attention values
// plus one word per edge for the slot -> destination map (rebuilt in the array
// on every call, so the graph's own lazily allocated map is never touched).
// All calls share the one array, so calls whose kernels overlap on the GPU
// race on it; every word a call reads it has written first, so nothing needs
// clearing between calls.
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
  const uint64_t n_alpha = (g->num_edges + (tail ? g->n_dst : 0)) * (uint64_t)heads;
  const uint64_t need = n_alpha + g->num_edges;
  if (need > BGNN_GAT_NOALLOC_MAX_FLOATS)
    return bgnn_set_error(ctx, BGNN_ERR_INVALID_ARG,
                          "allocation-free GAT needs %llu scratch words; the limit is %u "
                          "((edges + self-loops) * heads + edges)",
                          (unsigned long long)need, BGNN_GAT_NOALLOC_MAX_FLOATS);
  if (g->n_dst == 0) return BGNN_OK;
  float* scratch = nullptr;
  BGNN_TRY(noalloc_scratch(ctx, &scratch));
  // the slot -> destination map goes after the attention values
  uint32_t* dst_of = reinterpret_cast<uint32_t*>(scratch + n_alpha);
  BGNN_TRY(bgnn_graph_dst_of_into(ctx, g, dst_of));
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
  a.graph = g;
  a.heavy_rows = g->heavy_rows;
  a.n_heavy = g->heavy_rows ? g->n_heavy : 0u;
  a.heavy_threshold = g->heavy_threshold;
  const int ko = (int)((od + 31) / 32);
  if (ko <= 1) return launch_gat<1>(ctx, a, dst_of);
  if (ko <= 2) return launch_gat<2>(ctx, a, dst_of);
  if (ko <= 4) return launch_gat<4>(ctx, a, dst_of);
  return launch_gat<8>(ctx, a, dst_of);
}
