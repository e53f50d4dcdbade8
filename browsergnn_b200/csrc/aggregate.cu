// Fused gather + aggregate over a destination-keyed CSR: sum / mean / max,
// GCN-normalised sum, and SpMM with per-edge values.  No [E, F] message
// tensor is ever materialised (the reference builds one per layer with
// MessagePassing.gather, src/core/sparse.ts:462-473).
//
// Bit-exactness: each output element is accumulated by ONE thread, visiting
// the row's edges in CSR order, which for a graph CSR is the COO edge order
// the reference's scatters use (src/backend/wasm/index.ts:80-102).  Each step
// rounds exactly where the reference stores into a Float32Array:
//   sum   f32(acc + x)                       == __fadd_rn
//   gcn   f32(acc + f32(x * f32(ds * dd)))   == __fadd_rn(acc, __fmul_rn(x, w))
//   spmm  f32(acc + v*x) in double           == f64 fma then one rounding
//   max   x > acc ? x : acc, -inf -> 0 after (index.ts:158-206)
//   mean  f32(sum * (1/count as double))     (index.ts:128-148)
// No float atomics, no tree reductions, no FMA contraction (-fmad=false and
// explicit _rn intrinsics).
//
// Schedules:
//   streaming (k_agg_stream, the default): a persistent kernel pulls work
//               items (each heavy row alone, largest first, then runs of light
//               rows) from a queue; a pipe of threads streams an item's source
//               rows into a 3-stage shared-memory ring with 16-byte cp.async
//               copies and reduces them in edge order (see below).
//   light/heavy pair (k_agg_light + k_agg_heavy): only for the appended
//               self-loop edge of GCN/GAT loop insertion.  Light rows: a group
//               of G lanes per row, lanes over features; heavy rows: one CTA per
//               (row, 32-feature slice) with a cp.async ring, on a second
//               stream concurrently with the light rows.
#include "bgnn_internal.cuh"

namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr int OP_SPMM_X = 4;  // SpMM with f64 emulation of each JS step

template <int OP>
__device__ __forceinline__ float step(float acc, float x, float w) {
  if constexpr (OP == OP_SUM) {
    return __fadd_rn(acc, x);
  } else if constexpr (OP == OP_MAX) {
    return x > acc ? x : acc;
  } else if constexpr (OP == OP_GCN) {
    return __fadd_rn(acc, __fmul_rn(x, w));
  } else if constexpr (OP == OP_SPMM) {
    return __fmaf_rn(w, x, acc);
  } else {
    // the JS product of two f32 values is exact in double; fma rounds the sum once
    return __double2float_rn(__fma_rn((double)w, (double)x, (double)acc));
  }
}

template <int OP>
__device__ __forceinline__ float init_acc() {
  return OP == OP_MAX ? -INFINITY : 0.0f;
}

// rinv: 1/cnt already computed (the streaming pipes compute it once per row
// into shared memory rather than in every warp of the row)
__device__ __forceinline__ float epilogue(float v, const AggArgs& a, uint32_t row, int f,
                                          uint32_t cnt, const double* rinv = nullptr) {
  if (a.mean && cnt > 0)
    v = __double2float_rn(__dmul_rn((double)v, rinv ? *rinv : __ddiv_rn(1.0, (double)cnt)));
  if (a.max_fix && v == -INFINITY) v = 0.0f;
  if (a.gin_x) {
    // GINConv: combined = (1 + eps) * x + aggregated, in double (gin.ts:150-157)
    const double xs = (double)a.gin_x[(int64_t)row * a.ld_gin + f];
    v = __double2float_rn(__dadd_rn(__dmul_rn(a.gin_ope, xs), (double)v));
  }
  if (a.bias) v = __fadd_rn(v, a.bias[f]);
  return apply_act(v, a.act, a.act_param);
}

// Epilogue chosen at compile time by the streaming kernel: the generic one
// above (runtime flags), a mean alone, or nothing (a plain sum / SpMM).  The
// runtime checks of the generic one, run by every warp of every row, cost
// 1.5 ms of an 11 ms F = 256 mean aggregation.
enum : int { EPI_ANY = 0, EPI_MEAN = 1, EPI_NONE = 2 };

template <int EPI>
__device__ __forceinline__ float epilogue_t(float v, const AggArgs& a, uint32_t row, int f,
                                            uint32_t cnt, const double* rinv) {
  if constexpr (EPI == EPI_NONE) {
    return v;
  } else if constexpr (EPI == EPI_MEAN) {
    if (cnt > 0)
      v = __double2float_rn(__dmul_rn((double)v, rinv ? *rinv : __ddiv_rn(1.0, (double)cnt)));
    return v;
  } else {
    return epilogue(v, a, row, f, cnt, rinv);
  }
}

template <int V>
struct VecT;
template <>
struct VecT<4> {
  using T = float4;
  static __device__ __forceinline__ T load(const float* p) {
    return __ldg(reinterpret_cast<const float4*>(p));
  }
  static __device__ __forceinline__ float get(const T& v, int k) {
    return k == 0 ? v.x : (k == 1 ? v.y : (k == 2 ? v.z : v.w));
  }
};
template <>
struct VecT<1> {
  using T = float;
  static __device__ __forceinline__ T load(const float* p) { return __ldg(p); }
  static __device__ __forceinline__ float get(const T& v, int) { return v; }
};

// ---------------------------------------------------------------------------
// light rows: G lanes per row
// ---------------------------------------------------------------------------
template <int OP, int V, int CH>
__global__ void __launch_bounds__(256) k_agg_light(const AggArgs a, int G, int slice_w) {
  // edges whose row data is in flight per lane: ~32 registers of staging
  constexpr int U = (32 / (V * CH)) > 8 ? 8 : ((32 / (V * CH)) < 1 ? 1 : 32 / (V * CH));
  using VT = typename VecT<V>::T;
  const int lane = threadIdx.x & 31;
  const int gl = lane & (G - 1);
  const unsigned gmask = (G == 32) ? FULL : (((1u << G) - 1u) << (lane & ~(G - 1)));
  const uint64_t gid = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) / (uint64_t)G;
  if (gid >= a.n_rows) return;
  const uint32_t row = (uint32_t)gid;
  const uint32_t b = a.row_ptr[row];
  const uint32_t deg = a.row_ptr[row + 1] - b;
  if (deg >= a.heavy_threshold) return;  // the heavy-row kernel owns this row
  const uint32_t total = deg + (a.tail ? 1u : 0u);
  const int f_off = blockIdx.y * slice_w;
  const int f_end = min(a.num_features, f_off + slice_w);
  const int f0 = f_off + gl * V;

  float acc[CH][V];
#pragma unroll
  for (int c = 0; c < CH; c++)
#pragma unroll
    for (int k = 0; k < V; k++) acc[c][k] = init_acc<OP>();
  const float dinv_r = (OP == OP_GCN) ? a.dinv[row] : 0.0f;

  for (uint32_t j0 = 0; j0 < total; j0 += G) {
    const uint32_t jj = j0 + gl;
    uint32_t my_s = row;
    float my_w = 0.0f;
    if (jj < deg) {
      my_s = a.src_of[b + jj];
      if (OP == OP_SPMM || OP == OP_SPMM_X) my_w = a.val[b + jj];
    }
    if (OP == OP_GCN && jj < total) my_w = __fmul_rn(a.dinv[my_s], dinv_r);
    const int cnt = (int)min((uint32_t)G, total - j0);
    for (int t = 0; t < cnt; t += U) {
      VT buf[U][CH];
#pragma unroll
      for (int u = 0; u < U; u++) {
        const uint32_t s = __shfl_sync(gmask, my_s, (t + u) & (G - 1), G);
        const float* xr = a.x + (int64_t)s * a.ld_x;
#pragma unroll
        for (int c = 0; c < CH; c++) {
          const int f = f0 + c * G * V;
          if (t + u < cnt && f < f_end) buf[u][c] = VecT<V>::load(xr + f);
        }
      }
#pragma unroll
      for (int u = 0; u < U; u++) {
        const float w = __shfl_sync(gmask, my_w, (t + u) & (G - 1), G);
        if (t + u < cnt) {
#pragma unroll
          for (int c = 0; c < CH; c++)
#pragma unroll
            for (int k = 0; k < V; k++) acc[c][k] = step<OP>(acc[c][k], VecT<V>::get(buf[u][c], k), w);
        }
      }
    }
  }
  float* orow = a.out + (int64_t)row * a.ld_out;
#pragma unroll
  for (int c = 0; c < CH; c++) {
    const int f = f0 + c * G * V;
    if (f < f_end) {
      if constexpr (V == 4) {
        float4 o;
        o.x = epilogue(acc[c][0], a, row, f + 0, total);
        o.y = epilogue(acc[c][1], a, row, f + 1, total);
        o.z = epilogue(acc[c][2], a, row, f + 2, total);
        o.w = epilogue(acc[c][3], a, row, f + 3, total);
        *reinterpret_cast<float4*>(orow + f) = o;
      } else {
        orow[f] = epilogue(acc[c][0], a, row, f, total);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// heavy rows: CTA per (row, 32-feature slice), cp.async ring
// ---------------------------------------------------------------------------
constexpr int HV_THREADS = 256;
constexpr int HV_EPS = 128;    // edges per stage
constexpr int HV_STAGES = 4;
constexpr int HV_SW = 32;      // features per slice
constexpr size_t HV_SMEM = (size_t)HV_STAGES * HV_EPS * (HV_SW + 1) * sizeof(float);

__device__ __forceinline__ void cp_async16(void* s, const void* g) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(s);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(g) : "memory");
}
// 32-bit shared-memory addresses for the streaming pipes' hot loops: the
// ring is walked with stepped addresses instead of 64-bit index arithmetic
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ float lds_f32(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];\n" : "=f"(v) : "r"(a));
  return v;
}
template <int OFF>
__device__ __forceinline__ float lds_f32_off(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1+%2];\n" : "=f"(v) : "r"(a), "n"(OFF));
  return v;
}
__device__ __forceinline__ void cp_async16_sa(uint32_t sa, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(g) : "memory");
}
// the same at both addresses plus a constant byte offset
template <int OFF>
__device__ __forceinline__ void cp_async16_off(uint32_t sa, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0+%2], [%1+%2], 16;\n" ::"r"(sa), "l"(g), "n"(OFF)
               : "memory");
}
// Source-row slices of QPT x 64 floats (16-byte copies): 16 lanes per row,
// lane c copying chunks c, c+16, c+32, ... at constant 256-byte offsets, so
// one index load and one address computation serve QPT copies (one copy per
// lane per row cost 20 of an F = 256 aggregation's 106 warp instructions per
// edge).  Rows j0, j0 + jstep, ... < cnt of the stage; da / src already
// include the lane's first chunk.
template <int QPT>
__device__ __forceinline__ void copy_rows16(uint32_t da, uint32_t dstep, const float* src,
                                            const uint32_t* sid, int j0, int jstep, int cnt,
                                            int64_t ld_x) {
  for (int j = j0; j < cnt; j += jstep, da += dstep) {
    const float* g = src + (int64_t)sid[j] * ld_x;
    cp_async16_off<0>(da, g);
    if (QPT > 1) cp_async16_off<256>(da, g);
    if (QPT > 2) cp_async16_off<512>(da, g);
    if (QPT > 3) cp_async16_off<768>(da, g);
  }
}
__device__ __forceinline__ void cp_async4(void* s, const void* g) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(s);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(sa), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

template <int OP>
__global__ void __launch_bounds__(HV_THREADS) k_agg_heavy(const AggArgs a, int vec4) {
  extern __shared__ float4 hv_smem[];
  float* buf = reinterpret_cast<float*>(hv_smem);          // [STAGES][EPS][SW]
  float* wbuf = buf + (size_t)HV_STAGES * HV_EPS * HV_SW;  // [STAGES][EPS]
  const uint32_t row = a.heavy_rows[blockIdx.x];
  const int f0 = blockIdx.y * HV_SW;
  if (f0 >= a.num_features) return;
  const int fw = min(HV_SW, a.num_features - f0);
  const uint32_t b = a.row_ptr[row];
  const uint32_t deg = a.row_ptr[row + 1] - b;
  const uint32_t total = deg + (a.tail ? 1u : 0u);
  const uint32_t nst = (total + HV_EPS - 1) / HV_EPS;
  const bool v4 = vec4 && (fw % 4 == 0);
  const int per_edge = v4 ? fw / 4 : fw;
  const int copies = HV_EPS * per_edge;
  const float dinv_r = (OP == OP_GCN) ? a.dinv[row] : 0.0f;

  auto issue = [&](uint32_t k) {
    if (k < nst) {
      const int st = (int)(k % HV_STAGES);
      float* sb = buf + (size_t)st * HV_EPS * HV_SW;
      float* wb = wbuf + (size_t)st * HV_EPS;
      for (int c = threadIdx.x; c < copies; c += HV_THREADS) {
        const int j = c / per_edge;
        const int q = c - j * per_edge;
        const uint32_t jj = k * HV_EPS + (uint32_t)j;
        if (jj < total) {
          const uint32_t s = jj < deg ? a.src_of[b + jj] : row;
          const float* gp = a.x + (int64_t)s * a.ld_x + f0;
          if (v4)
            cp_async16(sb + j * HV_SW + 4 * q, gp + 4 * q);
          else
            cp_async4(sb + j * HV_SW + q, gp + q);
          if (q == 0) {
            if (OP == OP_GCN) cp_async4(wb + j, a.dinv + s);
            if ((OP == OP_SPMM || OP == OP_SPMM_X) && jj < deg) cp_async4(wb + j, a.val + b + jj);
          }
        }
      }
    }
    cp_async_commit();
  };

#pragma unroll
  for (int k = 0; k < HV_STAGES - 1; k++) issue((uint32_t)k);
  float acc = init_acc<OP>();
  for (uint32_t k = 0; k < nst; k++) {
    cp_async_wait<HV_STAGES - 2>();
    __syncthreads();
    issue(k + HV_STAGES - 1);
    if (threadIdx.x < (unsigned)fw) {
      const int st = (int)(k % HV_STAGES);
      const float* sb = buf + (size_t)st * HV_EPS * HV_SW + threadIdx.x;
      const float* wb = wbuf + (size_t)st * HV_EPS;
      const uint32_t cnt = min((uint32_t)HV_EPS, total - k * HV_EPS);
      for (uint32_t j = 0; j < cnt; j++) {
        float w = 0.0f;
        if (OP == OP_GCN) w = __fmul_rn(wb[j], dinv_r);
        if (OP == OP_SPMM || OP == OP_SPMM_X) w = wb[j];
        acc = step<OP>(acc, sb[j * HV_SW], w);
      }
    }
  }
  cp_async_wait<0>();
  if (threadIdx.x < (unsigned)fw) {
    const int f = f0 + threadIdx.x;
    a.out[(int64_t)row * a.ld_out + f] = epilogue(acc, a, row, f, total);
  }
}

// ---------------------------------------------------------------------------
// streaming schedule: a persistent kernel over the graph's work items.
//
// A "pipe" is a group of threads that streams one item (a heavy row, or a run
// of consecutive light rows) through a 3-stage cp.async ring in shared
// memory: every thread of the pipe copies the source-row slices of its edge,
// and thread f (f < slice width) accumulates feature f over the item's edges
// in CSR order, writing a row out when the edge stream crosses the row's end.
// Phase 1 runs the heavy items (largest first) with the whole CTA as one pipe;
// phase 2 splits the CTA into P pipes (P = 256 / padded width) that pull light
// items from a queue.  Items are fetched with one atomic per item.
// ---------------------------------------------------------------------------
constexpr int ST_THREADS = 256;
constexpr int ST_S = 3;       // ring stages
constexpr int ST_EPS = 32;    // edges per stage per light pipe
constexpr int ST_RMAX = 256;  // rows per light item (the graph's schedule builder cuts at this)
constexpr int ST_SW = 256;    // features per slice
constexpr int ST_GSTAGE = ST_EPS * ST_THREADS;  // floats per stage of a giant-row slice
constexpr int ST_GSW = ST_GSTAGE / ST_THREADS;    // narrowest giant slice (ST_THREADS edges)

// Source-id ring slots for an S-stage ring.  The prologue issues stages
// 0..S-2 back to back with no barrier between them, each issue reading its
// stage's ids and fetching (asynchronously) the ids of stage k + S - 1, so
// the slots read (stages 0..S-2) and written (stages S-1..2S-3) there must
// all differ: 2S - 2 slots.  Fewer (S + 1 for S = 5) let a fast thread's
// fetch land in a slot a slower thread was still reading.
__host__ __device__ constexpr int ids_slots(int S) { return 2 * S - 2 > S + 1 ? 2 * S - 2 : S + 1; }

// shared-memory regions, large enough for both the pipe layout and the
// giant-slice layout (ST_GSTAGE floats per stage, any slice width)
__host__ __device__ constexpr size_t stream_data_floats(int P, int swp) {
  return (size_t)P * ST_S * ST_EPS * swp > (size_t)ST_S * ST_GSTAGE
             ? (size_t)P * ST_S * ST_EPS * swp
             : (size_t)ST_S * ST_GSTAGE;
}
__host__ __device__ constexpr size_t stream_w_floats(int P) {
  return (size_t)P * ST_S * ST_EPS > (size_t)ST_S * ST_THREADS ? (size_t)P * ST_S * ST_EPS
                                                                 : (size_t)ST_S * ST_THREADS;
}
__host__ __device__ constexpr size_t stream_sidx_words(int P) {
  return (size_t)P * ids_slots(ST_S) * ST_EPS > (size_t)ids_slots(ST_S) * ST_THREADS
             ? (size_t)P * ids_slots(ST_S) * ST_EPS
             : (size_t)ids_slots(ST_S) * ST_THREADS;
}

// Both forms are volatile asm, like the shared-memory loads of the hot loops
// (lds_f32): volatile asm keeps its order, so no load of a stage can be
// scheduled above the barrier that publishes the stage.
__device__ __forceinline__ void pipe_bar(int id, int count) {
  if (id == 0)
    asm volatile("bar.sync 0;\n" ::: "memory");
  else
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}

// how a stage's source rows reach shared memory.  (One bulk copy per edge
// through the TMA engine, completing on an mbarrier, measured slower at every
// width: 14.0 vs 13.4 ms at F = 256, 8.0 vs 7.1 ms at F = 100, 18.6 vs
// 17.3 ms for the F = 32 SpMM.  A bulk L2 prefetch per row four stages
// ahead of the copies was slower still: 18.8 vs 13.9 ms at F = 256.)
enum : int {
  CP_A16 = 0,  // 16-byte cp.async copies spread over the pipe
  CP_A4 = 1,   // 4-byte cp.async copies (rows not 16-byte aligned)
};

template <int OP, int CP, int S = ST_S, bool ONE_ROW = false, int EPI = EPI_ANY>
__device__ __forceinline__ void stream_range(const AggArgs& a, uint32_t rb, uint32_t re, int f0,
                                             int fw, int swp, int tp, int ptid, int eps,
                                             float* buf, float* wbuf, uint32_t* sidx, uint32_t* rps,
                                             float* rdv, double* rinv, uint32_t& kg,
                                             int bar_id) {
  const uint32_t e0 = a.row_ptr[rb];
  const uint32_t ne = a.row_ptr[re] - e0;
  const uint32_t nrows = re - rb;
  for (uint32_t i = ptid; i <= nrows; i += tp) rps[i] = a.row_ptr[rb + i] - e0;
  if (OP == OP_GCN)
    for (uint32_t i = ptid; i < nrows; i += tp) rdv[i] = a.dinv[rb + i];
  if (rinv != nullptr)  // mean: 1/count in double, one division per row
    for (uint32_t i = ptid; i < nrows; i += tp)
      rinv[i] = __ddiv_rn(1.0, (double)(a.row_ptr[rb + i + 1] - a.row_ptr[rb + i]));

  const uint32_t nst = (ne + eps - 1) / eps;
  // Source ids: sidx slot m % IDS holds stage m's ids.  Stages 0..S-2 are
  // loaded before the ring starts; issue(m) fetches stage m+S-1's ids with
  // cp.async in the same group as stage m's rows.  issue(m+S-1) runs at
  // iteration m, after the wait that completes stage m's group and the
  // barrier that publishes it, so no copy ever waits on an index load.
  constexpr int IDS = ids_slots(S);
  auto fetch_ids = [&](uint32_t m) {
    const uint32_t e = m * (uint32_t)eps + (uint32_t)ptid;
    if (ptid < eps && m < nst && e < ne)
      cp_async4(sidx + (m % IDS) * eps + ptid, a.src_of + e0 + e);
  };
  // Row slices move as cp.async copies of 16 (CP_A16) or 4 bytes spread over
  // the pipe, consecutive threads on consecutive chunks of one row; per-edge
  // weights (GCN dinv, SpMM values) as 4-byte cp.async by the edge's thread.
  // Copy c of a stage (c = ptid, ptid + tp, ...) is chunk q = c % ch of
  // edge j = c / ch; the thread walks (j, q) incrementally (ch <= tp always),
  // so the copy loop has no integer division.
  // ONE_ROW (a giant slice, fw <= 128): the consumer warps only reduce and
  // the other warps copy (consumer warps that also issued copies ran the
  // chain at about 6 ns per edge, 5 without)
  const int cons = ONE_ROW ? ((fw + 31) & ~31) : 0;
  const int ctp = tp - cons, cpt = ptid - cons;  // copying threads, this one's rank
  const int ch = CP == CP_A16 ? fw >> 2 : fw;  // chunks per edge (16 or 4 bytes)
  const int cdj = ctp / ch, cdq = ctp - cdj * ch;
  const int cj0 = cpt / ch, cq0 = cpt - cj0 * ch;
  // widths of 128, 192 or 256 floats: 16 lanes per row (copy_rows16; at 64
  // floats the one-chunk-per-lane copy below is as cheap)
  const int q16 = (CP == CP_A16 && (ch & 15) == 0 && ch >= 32) ? ch >> 4 : 0;
  const int g_lane = cpt & 15, g_j0 = cpt >> 4, g_js = ctp >> 4;
  auto issue = [&](uint32_t k) {
    if (k < nst) {
      const int slot = (int)((kg + k) % S);
      const uint32_t* sid = sidx + (k % IDS) * eps;
      const int cnt = (int)min((uint32_t)eps, ne - k * (uint32_t)eps);  // edges in this stage
      float* sb = buf + (size_t)slot * eps * swp;
      constexpr int QB = CP == CP_A16 ? 4 : 1;  // floats per chunk
      if (cpt < 0) {
        // a consumer warp of a giant slice: no row copies
      } else if (q16) {
        const uint32_t da = smem_u32(sb + 4 * g_lane + (size_t)g_j0 * swp);
        const uint32_t dstep = (uint32_t)(g_js * swp) * 4u;
        const float* src = a.x + f0 + 4 * g_lane;
        switch (q16) {
            case 2: copy_rows16<2>(da, dstep, src, sid, g_j0, g_js, cnt, a.ld_x); break;
          case 3: copy_rows16<3>(da, dstep, src, sid, g_j0, g_js, cnt, a.ld_x); break;
          default: copy_rows16<4>(da, dstep, src, sid, g_j0, g_js, cnt, a.ld_x); break;
        }
      } else if (cdq == 0) {
        // ch divides the pipe width: the thread's chunk q never changes
        const float* src = a.x + f0 + QB * cq0;
        float* dst = sb + QB * cq0;
        if (CP == CP_A16) {
          uint32_t da = smem_u32(dst + (size_t)cj0 * swp);
          const uint32_t dstep = (uint32_t)(cdj * swp) * 4u;
          for (int j = cj0; j < cnt; j += cdj, da += dstep)
            cp_async16_sa(da, src + (int64_t)sid[j] * a.ld_x);
        } else {
          for (int j = cj0; j < cnt; j += cdj)
            cp_async4(dst + (size_t)j * swp, src + (int64_t)sid[j] * a.ld_x);
        }
      } else {
        int j = cj0, q = cq0;
        for (; j < cnt; j += cdj) {
          if (CP == CP_A16)
            cp_async16(sb + (size_t)j * swp + 4 * q, a.x + (int64_t)sid[j] * a.ld_x + f0 + 4 * q);
          else
            cp_async4(sb + (size_t)j * swp + q, a.x + (int64_t)sid[j] * a.ld_x + f0 + q);
          q += cdq;
          if (q >= ch) {
            q -= ch;
            j++;
          }
        }
      }
      if (ptid < cnt) {
        float* w = wbuf + slot * eps + ptid;
        if (OP == OP_GCN) cp_async4(w, a.dinv + sid[ptid]);
        if (OP == OP_SPMM || OP == OP_SPMM_X) cp_async4(w, a.val + e0 + k * (uint32_t)eps + ptid);
      }
    }
    fetch_ids(k + S - 1);
    cp_async_commit();
  };

  if (ptid < eps) {
#pragma unroll
    for (uint32_t m = 0; m < S - 1; m++) {
      const uint32_t e = m * (uint32_t)eps + (uint32_t)ptid;
      if (m < nst && e < ne) sidx[m * eps + ptid] = a.src_of[e0 + e];
    }
  }
  pipe_bar(bar_id, tp);
#pragma unroll
  for (int k = 0; k < S - 1; k++) issue((uint32_t)k);
  // Consumers: thread ptid reduces feature f0 + ptid, one serial chain in
  // edge order.  (Four features per thread, with one 16-byte shared load per
  // edge and a quarter of the warps paying the per-edge bookkeeping, measured
  // slower: 21.0 vs 11.0 ms at F = 256.  A consumer warp then stalls on each
  // load with no other consumer warp on its scheduler to cover it.)
  const bool consumer = ptid < fw;
  const int fv = f0 + ptid;
  float acc = init_acc<OP>();
  uint32_t r = 0;
  uint32_t nxt = rps[1];
  float dinv_r = (OP == OP_GCN && nrows) ? rdv[0] : 0.0f;
  auto finalize = [&]() {
    const uint32_t row = rb + r;
    const uint32_t cnt_r = rps[r + 1] - rps[r];
    const double* ri = rinv ? rinv + r : nullptr;
    a.out[(int64_t)row * a.ld_out + fv] = epilogue_t<EPI>(acc, a, row, fv, cnt_r, ri);
    acc = init_acc<OP>();
    r++;
    if (r < nrows) {
      nxt = rps[r + 1];
      if (OP == OP_GCN) dinv_r = rdv[r];
    }
  };
  constexpr bool HAS_W = OP == OP_GCN || OP == OP_SPMM || OP == OP_SPMM_X;
  for (uint32_t k = 0; k < nst; k++) {
    const int slot = (int)((kg + k) % S);
    cp_async_wait<S - 2>();  // this thread's copies of stage k have landed
    pipe_bar(bar_id, tp);       // ... and everyone's; stage k-1's slot is free
    issue(k + S - 1);
    if (ONE_ROW && consumer) {
      // a single row (a giant slice): no row ends inside the stream, and the
      // add chain is the critical path, so the shared-memory reads run R
      // edges ahead of the adds in a rolling register window.  32-bit shared
      // addresses throughout (generic 64-bit indexing here made the giant
      // launch slower per edge than a giant slice inside the main launch).
      const uint32_t swp4 = (uint32_t)swp * 4u;
      uint32_t ra = smem_u32(buf + (size_t)slot * eps * swp + ptid);
      const uint32_t w32 = smem_u32(wbuf + slot * eps);
      const uint32_t cnt = min((uint32_t)eps, ne - k * (uint32_t)eps);
      constexpr int R = 16;
      float v[R], wr[R];
#pragma unroll
      for (int u = 0; u < R; u++, ra += swp4) {
        v[u] = (uint32_t)u < cnt ? lds_f32(ra) : 0.0f;
        wr[u] = (HAS_W && (uint32_t)u < cnt) ? lds_f32(w32 + 4u * u) : 0.0f;
      }
      // ra: edge R's address
      uint32_t j = 0;
      for (; j + 2 * R <= cnt; j += R) {
        const uint32_t wa = w32 + (j + R) * 4u;
#pragma unroll
        for (int u = 0; u < R; u++) {
          const float w = (OP == OP_GCN) ? __fmul_rn(wr[u], dinv_r) : wr[u];
          acc = step<OP>(acc, v[u], w);
          v[u] = lds_f32(ra);
          ra += swp4;
          if (HAS_W) wr[u] = lds_f32(wa + 4u * u);
        }
      }
#pragma unroll
      for (int u = 0; u < R; u++) {  // the window's last R (or fewer) edges
        if (j + u < cnt) {
          const float w = (OP == OP_GCN) ? __fmul_rn(wr[u], dinv_r) : wr[u];
          acc = step<OP>(acc, v[u], w);
        }
      }
      for (j += R; j < cnt; j++, ra += swp4) {
        float w = 0.0f;
        if (OP == OP_GCN) w = __fmul_rn(lds_f32(w32 + j * 4u), dinv_r);
        if (OP == OP_SPMM || OP == OP_SPMM_X) w = lds_f32(w32 + j * 4u);
        acc = step<OP>(acc, lds_f32(ra), w);
      }
    } else if (consumer) {
      const uint32_t b32 = smem_u32(buf + (size_t)slot * eps * swp + ptid);
      const uint32_t swp4 = (uint32_t)swp * 4u;
      const uint32_t w32 = smem_u32(wbuf + slot * eps);
      const uint32_t base = k * (uint32_t)eps;
      const uint32_t cnt = min((uint32_t)eps, ne - base);
      // 16-edge blocks with the lean epilogues; the generic one keeps 8 (its
      // row-end path inlines the whole epilogue once per edge of the block)
      constexpr int UB = EPI == EPI_ANY ? 8 : 16;
      uint32_t j = 0;
      for (; j + UB <= cnt; j += UB) {
        // issue the block's shared-memory reads first, then reduce in order
        float v[UB], wr[UB];
        uint32_t ra = b32 + j * swp4;
#pragma unroll
        for (int u = 0; u < UB; u++, ra += swp4) {
          v[u] = lds_f32(ra);
          wr[u] = HAS_W ? lds_f32(w32 + (j + u) * 4u) : 0.0f;
        }
        if (nxt >= base + j + UB) {  // no row ends inside this block
#pragma unroll
          for (int u = 0; u < UB; u++) {
            const float w = (OP == OP_GCN) ? __fmul_rn(wr[u], dinv_r) : wr[u];
            acc = step<OP>(acc, v[u], w);
          }
        } else {
          // d: edges of the block before the next row end (one compare with a
          // constant per edge)
          int d = (int)(nxt - (base + j));
#pragma unroll
          for (int u = 0; u < UB; u++) {
            while (d == u) {
              finalize();
              d = (int)(nxt - (base + j));
            }
            const float w = (OP == OP_GCN) ? __fmul_rn(wr[u], dinv_r) : wr[u];
            acc = step<OP>(acc, v[u], w);
          }
        }
      }
      for (; j < cnt; j++) {
        while (base + j == nxt) finalize();
        float w = 0.0f;
        if (OP == OP_GCN) w = __fmul_rn(lds_f32(w32 + j * 4u), dinv_r);
        if (OP == OP_SPMM || OP == OP_SPMM_X) w = lds_f32(w32 + j * 4u);
        acc = step<OP>(acc, lds_f32(b32 + j * swp4), w);
      }
    }
  }
  cp_async_wait<0>();
  kg += nst;
  if (consumer)
    while (r < nrows) finalize();
  pipe_bar(bar_id, tp);  // the ring and row buffer are reused by the next item
}

template <int OP, bool A16, int EPI>
__global__ void __launch_bounds__(ST_THREADS, 2)
    k_agg_stream(const AggArgs a, int P, int swp, int n_slices, uint32_t n_giant, int gsw,
                 int eps_g, int mode, uint32_t n_ex, uint32_t* queue, int mean_rinv) {
  extern __shared__ float4 st_smem4[];
  float* data = reinterpret_cast<float*>(st_smem4);
  const size_t data_f = stream_data_floats(P, swp);
  // after the ring: per-edge weights, source ids, row offsets, fetched
  // items, GCN row dinv
  float* wb = data + data_f;
  uint32_t* sidx = reinterpret_cast<uint32_t*>(wb + stream_w_floats(P));
  uint32_t* rps = sidx + stream_sidx_words(P);
  int* slots = reinterpret_cast<int*>(rps + P * (ST_RMAX + 1));  // [0..P] fetched items
  float* rdv = reinterpret_cast<float*>(slots + 16);  // present for OP_GCN only
  // present for a mean with P <= 2 only: 8-byte aligned after slots
  double* rinv = mean_rinv ? reinterpret_cast<double*>(
                                 (reinterpret_cast<uintptr_t>(slots + 16) + 7) & ~uintptr_t(7))
                           : nullptr;
  const int F = a.num_features;
  const uint32_t gs = (uint32_t)((F + gsw - 1) / gsw);
  const uint32_t giant_work = n_giant * gs;
  // With several pipes per CTA (slices of at most 128 features), a heavy row
  // streamed by the whole CTA would have no more consumer threads than one
  // pipe (one per feature either way) and would restart the ring for a few
  // stages: the pipes take those rows instead, at the front of their queue
  // (largest first).  Phase 1 then runs only the giant-row slices.
  const uint32_t first_light = P > 1 ? n_giant : a.n_heavy_items;
  const uint32_t heavy_work = giant_work + (first_light - n_giant) * (uint32_t)n_slices;
  const uint32_t light_work = (a.n_items - first_light) * (uint32_t)n_slices;
  const int tp = ST_THREADS / P;
  constexpr int CP = A16 ? CP_A16 : CP_A4;  // rows 16-byte aligned: 16-byte copies
  auto run = [&](uint32_t rb, uint32_t re, int f0, int fw, int width, int tpp, int pt, int eps,
                 float* d, float* w_, uint32_t* si, uint32_t* rp, float* dv, double* ri,
                 uint32_t& kgr, int bar) {
    stream_range<OP, CP, ST_S, false, EPI>(a, rb, re, f0, fw, width, tpp, pt, eps, d, w_, si, rp,
                                           dv, ri, kgr, bar);
  };

  // Giant rows (the first n_giant heavy items, chosen at launch) are cut into
  // gsw-feature slices with eps_g edges per stage, so several CTAs stream one
  // hub row at once; each slice is still reduced in edge order by one thread
  // per feature.  mode 2: the slices of the first n_ex giant rows run in
  // their own launch (k_agg_giant), skip them; mode 0: everything here.
  uint32_t kg = 0;  // stages run so far (ring slot)
  const uint32_t w0 = mode == 2 ? n_ex * gs : 0u;
  // phase 1: heavy rows with the whole CTA as one pipe
  for (;;) {
    if (threadIdx.x == 0) slots[P] = (int)(w0 + atomicAdd(&queue[0], 1u));
    __syncthreads();
    const uint32_t w = (uint32_t)slots[P];
    if (w >= heavy_work) break;
    if (w < giant_work) {
      const uint2 item = a.items[w / gs];
      const int f0 = (int)(w % gs) * gsw;
      run(item.x, item.y, f0, min(gsw, F - f0), gsw, ST_THREADS, threadIdx.x, eps_g, data, wb, sidx,
          rps, rdv, rinv, kg, 0);
    } else {
      const uint32_t w2 = w - giant_work;
      const uint2 item = a.items[n_giant + w2 / (uint32_t)n_slices];
      const int f0 = (int)(w2 % (uint32_t)n_slices) * ST_SW;
      run(item.x, item.y, f0, min(ST_SW, F - f0), swp, ST_THREADS, threadIdx.x, ST_EPS * P, data, wb,
          sidx, rps, rdv, rinv, kg, 0);
    }
  }
  // phase 2: light items (with P > 1 also the non-giant heavy rows), P pipes
  const int pipe = threadIdx.x / tp, ptid = threadIdx.x % tp;
  const int bar_id = P == 1 ? 0 : pipe + 1;
  float* pdata = data + (size_t)pipe * ST_S * ST_EPS * swp;
  float* pwb = wb + pipe * ST_S * ST_EPS;
  uint32_t* psidx = sidx + pipe * ids_slots(ST_S) * ST_EPS;
  uint32_t* prps = rps + pipe * (ST_RMAX + 1);
  float* prdv = rdv + pipe * ST_RMAX;
  double* prinv = rinv ? rinv + pipe * ST_RMAX : nullptr;
  uint32_t kgp = 0;
  for (;;) {
    if (ptid == 0) slots[pipe] = (int)atomicAdd(&queue[1], 1u);
    pipe_bar(bar_id, tp);
    const uint32_t w = (uint32_t)slots[pipe];
    if (w >= light_work) break;
    const uint2 item = a.items[first_light + w / (uint32_t)n_slices];
    const int f0 = (int)(w % (uint32_t)n_slices) * ST_SW;
    run(item.x, item.y, f0, min(ST_SW, F - f0), swp, tp, ptid, ST_EPS, pdata, pwb, psidx, prps, prdv,
        prinv, kgp, bar_id);
  }
}

// Giant-row slices in their own launch: one CTA per slice, alone on its SM
// (its shared memory request leaves no room for a second CTA), with a deeper
// ring than the shared-SM pipes since the whole SM's shared memory is its.
constexpr int GS_S = 6;  // ring stages of a giant-slice CTA (208 KB of shared memory)
constexpr size_t giant_smem_bytes() {
  return ((size_t)GS_S * ST_GSTAGE + (size_t)GS_S * ST_THREADS + (size_t)ids_slots(GS_S) * ST_THREADS +
          16) * 4;
}

template <int OP, bool A16>
__global__ void __launch_bounds__(ST_THREADS, 1)
    k_agg_giant(const AggArgs a, uint32_t n_ex, int gsw, int eps_g) {
  extern __shared__ float4 gt_smem4[];
  float* data = reinterpret_cast<float*>(gt_smem4);
  float* wb = data + (size_t)GS_S * ST_GSTAGE;
  uint32_t* sidx = reinterpret_cast<uint32_t*>(wb + GS_S * ST_THREADS);
  uint32_t* rps = sidx + ids_slots(GS_S) * ST_THREADS;  // one row per item: 2 offsets
  float* rdv = reinterpret_cast<float*>(rps + 4);
  const int F = a.num_features;
  const uint32_t gs = (uint32_t)((F + gsw - 1) / gsw);
  constexpr int CP = A16 ? CP_A16 : CP_A4;
  uint32_t kg = 0;
  for (uint32_t w = blockIdx.x; w < n_ex * gs; w += gridDim.x) {
    const uint2 item = a.items[w / gs];
    const int f0 = (int)(w % gs) * gsw;
    stream_range<OP, CP, GS_S, true>(a, item.x, item.y, f0, min(gsw, F - f0), gsw, ST_THREADS,
                                     threadIdx.x, eps_g, data, wb, sidx, rps, rdv, nullptr, kg, 0);
  }
}

template <int OP, bool A16, int EPI>
int launch_stream_t(bgnn_ctx* ctx, const AggArgs& a, int P, int swp, int n_slices) {
  size_t smem = (stream_data_floats(P, swp) + stream_w_floats(P) + stream_sidx_words(P) +
                 (size_t)P * (ST_RMAX + 1) + 16) * 4;
  if (OP == OP_GCN) smem += (size_t)P * ST_RMAX * 4;
  const int mean_rinv = (OP == OP_SUM && a.mean && P <= 2) ? 1 : 0;
  if (mean_rinv) smem += (size_t)P * ST_RMAX * 8 + 8;
  BGNN_CUDA(ctx, cudaFuncSetAttribute(k_agg_stream<OP, A16, EPI>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0;
  BGNN_CUDA(ctx, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_agg_stream<OP, A16, EPI>,
                                                               ST_THREADS, smem));
  if (per_sm < 1) per_sm = 1;
  const uint64_t work = (uint64_t)a.n_items * n_slices;
  const int sms = ctx->grid_sms > 0 && ctx->grid_sms < ctx->num_sms ? ctx->grid_sms : ctx->num_sms;
  uint64_t grid = (uint64_t)sms * per_sm;
  if (grid > work) grid = work ? work : 1;
  // Giant rows: a heavy row whose bytes exceed one pipe's fair share of the
  // launch would finish long after the rest, so it is cut into feature slices
  // that separate CTAs stream (a single slice when F <= ST_GSW: the row then
  // still gets a whole CTA and its larger stages).  The slice is the widest power of two from 128
  // down to ST_GSW features that keeps the largest row's slice within the
  // share (ST_GSW at least), with ST_GSTAGE floats per stage (eps_g edges x
  // gsw features).
  const int F = a.num_features;
  uint32_t n_giant = 0;
  int gsw = ST_GSW;
  if (a.heavy_deg != nullptr && grid > 1) {
    // a heavy row otherwise runs in one pipe (1/P of a CTA): it is giant once
    // its bytes exceed a pipe's share; its slices then get whole CTAs
    const double share = (double)a.num_edges * (double)F * 4.0 / (double)grid;
    const double pipe_share = share / (double)P;
    while (n_giant < a.n_heavy_items && (double)a.heavy_deg[n_giant] * F * 4.0 > pipe_share)
      n_giant++;
    if (n_giant) {
      gsw = 128;
      while (gsw > ST_GSW && (gsw >= F || (double)a.heavy_deg[0] * gsw * 4.0 > share)) gsw >>= 1;
    }
  }
  const int eps_g = ST_GSTAGE / gsw;  // edges per giant stage (at most ST_THREADS)
  uint32_t* queue = ctx->d_small;
  BGNN_CUDA(ctx, cudaMemsetAsync(queue, 0, 2 * sizeof(uint32_t), ctx->stream));
  // rows long enough (four CTA shares or more) to finish last even when cut
  // into slices get their own launch, up to a quarter of the SMs
  uint32_t n_ex = 0;
  if (n_giant > 0) {
    const double share = (double)a.num_edges * (double)F * 4.0 / (double)grid;
    const uint32_t gs = (uint32_t)((F + gsw - 1) / gsw);
    const uint32_t cap = (uint32_t)sms / 4 / gs;
    while (n_ex < n_giant && n_ex < cap && (double)a.heavy_deg[n_ex] * F * 4.0 > 4.0 * share) n_ex++;
  }
  int mode = 0;
  if (n_ex > 0) {
    // The giant slices go first, in their own launch on the (high-priority)
    // aux stream, one CTA per slice with enough shared memory that nothing
    // else shares its SM: a slice is one serial add chain per feature, and on
    // a shared SM its single consumer warp gets a fraction of the issue slots
    // and its two stages in flight leave it waiting on memory.
    // The main launch skips them; its persistent CTAs that find no room
    // start as the slices finish and pull from the same work queue.
    constexpr size_t gsmem = giant_smem_bytes();
    static_assert(gsmem > 228 * 1024 - 106 * 1024, "a giant-slice CTA must fill its SM");
    BGNN_CUDA(ctx, cudaFuncSetAttribute(k_agg_giant<OP, A16>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gsmem));
    BGNN_CUDA(ctx, cudaEventRecord(ctx->ev_fork, ctx->stream));
    BGNN_CUDA(ctx, cudaStreamWaitEvent(ctx->aux_stream, ctx->ev_fork, 0));
    const uint32_t gs = (uint32_t)((F + gsw - 1) / gsw);
    k_agg_giant<OP, A16><<<n_ex * gs, ST_THREADS, gsmem, ctx->aux_stream>>>(a, n_ex, gsw, eps_g);
    BGNN_LAUNCHED(ctx);
    BGNN_CUDA(ctx, cudaEventRecord(ctx->ev_join, ctx->aux_stream));
    mode = 2;
  }
  k_agg_stream<OP, A16, EPI><<<(unsigned)grid, ST_THREADS, smem, ctx->stream>>>(
      a, P, swp, n_slices, n_giant, gsw, eps_g, mode, n_ex, queue, mean_rinv);
  BGNN_LAUNCHED(ctx);
  if (n_ex > 0) BGNN_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, ctx->ev_join, 0));
  return BGNN_OK;
}

template <int OP>
int launch_stream(bgnn_ctx* ctx, const AggArgs& a0) {
  AggArgs a = a0;
  a.err = ctx->d_err;
  const int F = a.num_features;
  const int fs = F < ST_SW ? F : ST_SW;
  const int swp = (fs + 3) & ~3;
  int pw = 32;
  while (pw < swp) pw <<= 1;
  const int P = ST_THREADS / pw;  // 1, 2, 4 or 8
  const int n_slices = (F + ST_SW - 1) / ST_SW;
  // 16-byte copies need 16-byte aligned rows: F % 4 == 0 covers every slice
  const bool a16 = (F % 4 == 0) && ((uintptr_t)a.x % 16 == 0) && (a.ld_x % 4 == 0);
  // compile-time epilogue when no bias, activation, GIN term or max fix-up
  const bool bare = !a.max_fix && a.gin_x == nullptr && a.bias == nullptr && a.act == BGNN_ACT_NONE;
  if constexpr (OP == OP_SUM) {
    if (bare && a.mean)
      return a16 ? launch_stream_t<OP, true, EPI_MEAN>(ctx, a, P, swp, n_slices)
                 : launch_stream_t<OP, false, EPI_MEAN>(ctx, a, P, swp, n_slices);
  }
  if constexpr (OP == OP_SUM || OP == OP_SPMM || OP == OP_SPMM_X) {
    if (bare && !a.mean)
      return a16 ? launch_stream_t<OP, true, EPI_NONE>(ctx, a, P, swp, n_slices)
                 : launch_stream_t<OP, false, EPI_NONE>(ctx, a, P, swp, n_slices);
  }
  return a16 ? launch_stream_t<OP, true, EPI_ANY>(ctx, a, P, swp, n_slices)
             : launch_stream_t<OP, false, EPI_ANY>(ctx, a, P, swp, n_slices);
}

// ---------------------------------------------------------------------------
// host dispatch
// ---------------------------------------------------------------------------
template <int OP, int V, int CH>
int launch_light(bgnn_ctx* ctx, const AggArgs& a, int G, int slices, int slice_w) {
  const uint64_t threads = (uint64_t)a.n_rows * (uint64_t)G;
  const uint64_t blocks = (threads + 255) / 256;
  dim3 grid((unsigned)blocks, (unsigned)slices);
  k_agg_light<OP, V, CH><<<grid, 256, 0, ctx->stream>>>(a, G, slice_w);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

template <int OP, int V>
int launch_light_ch(bgnn_ctx* ctx, const AggArgs& a, int G, int CH, int slices, int slice_w) {
  switch (CH) {
    case 1: return launch_light<OP, V, 1>(ctx, a, G, slices, slice_w);
    case 2: return launch_light<OP, V, 2>(ctx, a, G, slices, slice_w);
    case 4: return launch_light<OP, V, 4>(ctx, a, G, slices, slice_w);
    default: return launch_light<OP, V, 8>(ctx, a, G, slices, slice_w);
  }
}

template <int OP>
int launch_heavy(bgnn_ctx* ctx, const AggArgs& a, int vec4, cudaStream_t s) {
  BGNN_CUDA(ctx, cudaFuncSetAttribute(k_agg_heavy<OP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)HV_SMEM));
  dim3 grid(a.n_heavy, (unsigned)((a.num_features + HV_SW - 1) / HV_SW));
  k_agg_heavy<OP><<<grid, HV_THREADS, HV_SMEM, s>>>(a, vec4);
  BGNN_LAUNCHED(ctx);
  return BGNN_OK;
}

template <int OP>
int run_op(bgnn_ctx* ctx, const AggArgs& a0) {
  AggArgs a = a0;
  const int F = a.num_features;
  // the streaming schedule covers every case except the appended self-loop
  // edge (GCN/GAT loop insertion), which the light/heavy pair handles
  if (!a.tail && a.items != nullptr && a.n_items > 0) return launch_stream<OP>(ctx, a);
  const bool al_x = ((uintptr_t)a.x % 16 == 0) && (a.ld_x % 4 == 0);
  const bool al_o = ((uintptr_t)a.out % 16 == 0) && (a.ld_out % 4 == 0);
  const int V = (F % 4 == 0 && al_x && al_o) ? 4 : 1;
  const int nv = (F + V - 1) / V;
  int G, CH, slices = 1, slice_w = F;
  if (nv <= 32) {
    G = 1;
    while (G < nv) G <<= 1;
    CH = 1;
  } else if (nv <= 256) {
    G = 32;
    const int need = (nv + 31) / 32;
    CH = need <= 2 ? 2 : (need <= 4 ? 4 : 8);
  } else {
    G = 32;
    CH = 8;
    slice_w = 256 * V;
    slices = (F + slice_w - 1) / slice_w;
  }
  const bool heavy = a.n_heavy > 0 && a.heavy_rows != nullptr;
  if (!heavy) a.heavy_threshold = 0xffffffffu;
  if (heavy) {
    BGNN_CUDA(ctx, cudaEventRecord(ctx->ev_fork, ctx->stream));
    BGNN_CUDA(ctx, cudaStreamWaitEvent(ctx->aux_stream, ctx->ev_fork, 0));
    BGNN_TRY(launch_heavy<OP>(ctx, a, al_x ? 1 : 0, ctx->aux_stream));
    BGNN_CUDA(ctx, cudaEventRecord(ctx->ev_join, ctx->aux_stream));
  }
  int rc = (V == 4) ? launch_light_ch<OP, 4>(ctx, a, G, CH, slices, slice_w)
                    : launch_light_ch<OP, 1>(ctx, a, G, CH, slices, slice_w);
  if (heavy) BGNN_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, ctx->ev_join, 0));
  return rc;
}

}  // namespace

int bgnn_run_aggregate(bgnn_ctx* ctx, int op, const AggArgs& a) {
  if (a.n_rows == 0 || a.num_features == 0) return BGNN_OK;
  switch (op) {
    case OP_SUM: return run_op<OP_SUM>(ctx, a);
    case OP_MAX: return run_op<OP_MAX>(ctx, a);
    case OP_GCN: return run_op<OP_GCN>(ctx, a);
    case OP_SPMM: return a.exact ? run_op<OP_SPMM_X>(ctx, a) : run_op<OP_SPMM>(ctx, a);
    default: return bgnn_set_error(ctx, BGNN_ERR_INVALID_ARG, "unknown aggregation op %d", op);
  }
}
