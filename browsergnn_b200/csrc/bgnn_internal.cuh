// Internal declarations shared by the translation units of libbgnn_cuda.so.
#pragma once

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

#include "bgnn.h"

// ---------------------------------------------------------------------------
// context and graph handles
// ---------------------------------------------------------------------------
struct bgnn_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;      // stream all work is ordered on
  cudaStream_t own_stream = nullptr;  // created by the context
  cudaStream_t aux_stream = nullptr;  // heavy-row kernels run here, joined back
  cudaEvent_t ev_fork = nullptr;
  cudaEvent_t ev_join = nullptr;
  int math = BGNN_MATH_FAST;
  int* d_err = nullptr;      // [0]=code, [1]=info lo, [2]=info hi, [3]=where
  uint32_t* d_small = nullptr;  // small device counters (heavy-row count etc.)
  int grid_sms = 0;  // SMs the persistent aggregation may fill (0: all); the multi-GPU
                     // pipeline leaves the rest to the collectives running beside it
  uint64_t launches = 0;
  std::string last_error;
};

struct bgnn_graph {
  int device = 0;
  uint32_t n_src = 0, n_dst = 0;
  uint64_t num_edges = 0;
  uint32_t* row_ptr = nullptr;     // [n_dst+1] destination-keyed CSR
  uint32_t* src_of = nullptr;      // [E] source node of each CSR slot
  uint32_t* eid = nullptr;         // [E] COO edge id of each CSR slot
  uint32_t* out_deg = nullptr;     // [n_src]
  uint32_t* heavy_rows = nullptr;  // rows handled CTA-per-row, largest first
  uint32_t n_heavy = 0;
  uint32_t heavy_threshold = 0;
  // streaming schedule: work items [row_begin, row_end): first every heavy
  // row on its own (largest first), then runs of consecutive light rows
  uint2* items = nullptr;
  uint32_t n_items = 0;
  uint32_t n_heavy_items = 0;
  std::vector<uint32_t> heavy_deg;  // degrees of the heavy items, host copy (largest first)
  int has_self_loops = 0;
  bool csr_only = false;           // built from an existing CSR (no eid/out_deg)
  float* dinv[2] = {nullptr, nullptr};  // GCN D^-1/2 without / with loop tail
  uint32_t* dst_of = nullptr;      // [E] destination row of each CSR slot (built on first use)
  bgnn_graph* transpose = nullptr; // rows = sources, edges in COO order (built for the backward)
};

// Row partition of a square graph / CSR for one rank (partition.cu): rank r
// owns rows [lo, hi); its local CSR holds those rows' entries in the global
// order with columns relabelled to [0, n_own) for owned nodes and
// n_own + k for the k-th halo node (sorted global id, hence grouped by owner).
struct bgnn_part {
  int device = 0;
  uint32_t world = 1, rank = 0;
  uint32_t n_global = 0;
  std::vector<uint32_t> bounds;       // [world+1]
  uint32_t lo = 0, hi = 0, n_own = 0, n_halo = 0;
  uint64_t entry_lo = 0, n_local_entries = 0;  // the local rows' entries in the global CSR
  bgnn_graph local;                   // [n_own rows, n_own + n_halo columns]
  uint32_t* halo_ids = nullptr;       // [n_halo] global id of each halo slot
  uint32_t* send_rows = nullptr;      // [n_send] owned rows (local ids) other ranks read, by peer
  uint64_t n_send = 0;
  std::vector<uint64_t> send_counts, recv_counts;  // rows per peer
  std::vector<uint64_t> send_off, recv_off;        // exclusive prefix of the counts
  // Row blocks, for halo sends that start as each block of a layer's output
  // is written: every rank's owned rows cut into blk_count blocks (block c of
  // n rows: [c n / C, (c+1) n / C)); blk_send[q (C+1) + c] is the first entry
  // of peer q's send list in block c, blk_recv[q (C+1) + c] the first halo
  // slot of owner q's block c (host copies; blk_send also on the device).
  // Derived on first use and kept.
  mutable uint32_t blk_count = 0;
  mutable std::vector<uint64_t> blk_send, blk_recv;
  mutable uint64_t* d_blk_send = nullptr;
};
// the first owned row of block c of `blocks` over n rows
inline uint32_t bgnn_block_row(uint32_t n, uint32_t blocks, uint32_t c) {
  return (uint32_t)((uint64_t)c * n / blocks);
}
int bgnn_part_row_blocks(bgnn_ctx* ctx, const bgnn_part* p, uint32_t blocks);
// pack block c's send rows (every peer's) of x ([n_own, width] rows at
// stride width) into out at their send-list positions
int bgnn_run_pack_block(bgnn_ctx* ctx, const float* x, uint32_t width, const bgnn_part* p,
                        uint32_t c, float* out);
void bgnn_part_free(bgnn_part* p);
int bgnn_run_pack_cols(bgnn_ctx* ctx, const float* x, uint64_t ld_x, uint32_t col0,
                       uint32_t width, const uint32_t* rows, uint64_t n, float* out);
int bgnn_run_unpack_cols(bgnn_ctx* ctx, const float* src, uint64_t n, uint32_t width, float* x,
                         uint64_t ld_x, uint32_t col0);

// ---------------------------------------------------------------------------
// error plumbing: every internal call returns a bgnn_status
// ---------------------------------------------------------------------------
int bgnn_set_error(bgnn_ctx* ctx, int code, const char* fmt, ...);

#define BGNN_CUDA(ctx, call)                                                       \
  do {                                                                             \
    cudaError_t _e = (call);                                                       \
    if (_e != cudaSuccess) {                                                       \
      return bgnn_set_error((ctx), _e == cudaErrorMemoryAllocation ? BGNN_ERR_NO_MEMORY \
                                                                   : BGNN_ERR_CUDA, \
                            "%s failed: %s (%s:%d)", #call, cudaGetErrorString(_e),  \
                            __FILE__, __LINE__);                                   \
    }                                                                              \
  } while (0)

#define BGNN_LAUNCHED(ctx)                                                         \
  do {                                                                             \
    cudaError_t _e = cudaGetLastError();                                           \
    if (_e != cudaSuccess)                                                         \
      return bgnn_set_error((ctx), BGNN_ERR_CUDA, "kernel launch failed: %s (%s:%d)", \
                            cudaGetErrorString(_e), __FILE__, __LINE__);           \
    (ctx)->launches++;                                                             \
  } while (0)

#define BGNN_TRY(x)              \
  do {                           \
    int _s = (x);                \
    if (_s != BGNN_OK) return _s; \
  } while (0)

#define BGNN_REQUIRE(ctx, cond, ...)                                   \
  do {                                                                 \
    if (!(cond)) return bgnn_set_error((ctx), BGNN_ERR_INVALID_ARG, __VA_ARGS__); \
  } while (0)

// Stream-ordered temporary device buffer (cudaMallocAsync on the ctx stream).
struct DevTmp {
  void* p = nullptr;
  cudaStream_t s = nullptr;
  DevTmp() = default;
  DevTmp(const DevTmp&) = delete;
  DevTmp& operator=(const DevTmp&) = delete;
  ~DevTmp() {
    if (p) cudaFreeAsync(p, s);
  }
  template <class T>
  T* as() const {
    return static_cast<T*>(p);
  }
};
int bgnn_tmp_alloc(bgnn_ctx* ctx, DevTmp& t, size_t bytes);

// device error word codes (written by kernels, read at synchronisation)
enum : int { DEVERR_NONE = 0, DEVERR_INDEX = 1, DEVERR_TIMEOUT = 2 };

__device__ __forceinline__ void dev_raise(int* err, int code, uint64_t info, int where) {
  if (atomicCAS(err, 0, code) == 0) {
    err[1] = (int)(uint32_t)(info & 0xffffffffu);
    err[2] = (int)(uint32_t)(info >> 32);
    err[3] = where;
  }
}

// ---------------------------------------------------------------------------
// primitives (util.cu)
// ---------------------------------------------------------------------------
// exclusive prefix sum of n uint32 values (in may equal out)
int bgnn_exclusive_scan(bgnn_ctx* ctx, const uint32_t* in, uint32_t* out, uint64_t n);
// Stable LSD radix sort (8-bit digits) of 32-bit keys carrying up to two
// 32-bit payload streams.  Payload 0 is p0_in, or the item's input index
// when ident0 != 0 (p0_in NULL); payload 1 is p1_in (NULL: none; needs
// payload 0).  key_bits: number of low key bits to sort.  keys_out may be
// NULL when the sorted keys are not wanted.
int bgnn_radix_sort(bgnn_ctx* ctx, const uint32_t* keys_in, uint64_t n, int key_bits,
                    const uint32_t* p0_in, int ident0, const uint32_t* p1_in, uint32_t* keys_out,
                    uint32_t* p0_out, uint32_t* p1_out);
int bgnn_bits_for(uint64_t max_value);
int bgnn_iota(bgnn_ctx* ctx, uint32_t* out, uint64_t n);
// synchronous copies of caller host memory (hostcopy.cu): page-locked memory
// directly, pageable memory staged through library-owned pinned chunks
int bgnn_copy_h2d(bgnn_ctx* ctx, void* dst, const void* src, uint64_t bytes);
int bgnn_copy_d2h(bgnn_ctx* ctx, void* dst, const void* src, uint64_t bytes);
int bgnn_check_device_error(bgnn_ctx* ctx);

// ---------------------------------------------------------------------------
// graph construction (graph.cu)
// ---------------------------------------------------------------------------
int bgnn_graph_build(bgnn_ctx* ctx, const uint32_t* src_dev, const uint32_t* dst_dev,
                     uint64_t num_edges, uint32_t num_src, uint32_t num_dst, bgnn_graph* g);
int bgnn_graph_from_csr(bgnn_ctx* ctx, const uint32_t* row_ptr, const uint32_t* col,
                        uint32_t num_rows, uint32_t num_cols, bgnn_graph* g, bool copy);
// Takes ownership of a device CSR (cudaMalloc'd row_ptr [n_rows+1] and col
// [nnz], already validated) and builds the row schedule.
int bgnn_graph_adopt_csr(bgnn_ctx* ctx, uint32_t* row_ptr, uint32_t* col, uint32_t n_rows,
                         uint32_t n_cols, uint64_t nnz, bgnn_graph* g);
void bgnn_graph_free(bgnn_graph* g);
int bgnn_graph_dinv(bgnn_ctx* ctx, bgnn_graph* g, int tail, const float** out);
int bgnn_graph_dst_of(bgnn_ctx* ctx, bgnn_graph* g, const uint32_t** out);
int bgnn_graph_dst_of_into(bgnn_ctx* ctx, const bgnn_graph* g, uint32_t* out);
// the source-keyed transpose of an edge-list graph (backward.cu), built on
// first use and freed with the graph
int bgnn_graph_transpose(bgnn_ctx* ctx, bgnn_graph* g, const bgnn_graph** out);

// ---------------------------------------------------------------------------
// aggregation (aggregate.cu)
// ---------------------------------------------------------------------------
enum AggOp : int { OP_SUM = 0, OP_MAX = 1, OP_GCN = 2, OP_SPMM = 3 };

struct AggArgs {
  const uint32_t* row_ptr;
  const uint32_t* src_of;
  const float* x;
  int64_t ld_x;
  const float* val;       // OP_SPMM: per-slot values
  const float* dinv;      // OP_GCN: per-node D^-1/2
  uint32_t n_rows;
  int num_features;
  float* out;
  int64_t ld_out;
  const uint32_t* heavy_rows;
  uint32_t n_heavy;
  uint32_t heavy_threshold;
  const uint2* items;     // streaming schedule (NULL: use the light/heavy pair)
  uint32_t n_items;
  uint32_t n_heavy_items;
  const uint32_t* heavy_deg;   // host pointer: degrees of the heavy items (launch-time split)
  uint64_t num_edges;
  int tail;               // virtual self-loop edge after each row's edges
  int mean;               // sum * (1/count)
  int max_fix;            // -inf -> 0
  const float* bias;
  const float* gin_x;     // GIN combine: out = (1+eps)*x_self + agg
  int64_t ld_gin;
  double gin_ope;
  int act;
  double act_param;
  int exact;              // OP_SPMM rounding mode
  int* err;               // device error word (set by the launcher)
};
int bgnn_run_aggregate(bgnn_ctx* ctx, int op, const AggArgs& a);
// bgnn_aggregate / bgnn_graph_spmm (aggr BGNN_AGGR_SPMM) over a column slice
// of x (row stride ld_x) into a column slice of out (row stride ld_out)
int bgnn_run_aggregate_cols(bgnn_ctx* ctx, const bgnn_graph* g, int aggr, const float* values,
                            const float* x, uint64_t ld_x, uint32_t width, float* out,
                            uint64_t ld_out);

// ---------------------------------------------------------------------------
// GAT (gat.cu)
// ---------------------------------------------------------------------------
int bgnn_run_gat(bgnn_ctx* ctx, const bgnn_graph* g, const float* h, uint32_t heads, uint32_t c,
                 const float* att_src, const float* att_dst, double slope, int concat, int tail,
                 const float* bias, int act, double act_param, float* out, double drop_p = 0.0,
                 uint64_t seed = 0);

// ---------------------------------------------------------------------------
// dense (gemm.cu)
// ---------------------------------------------------------------------------
int bgnn_run_linear(bgnn_ctx* ctx, const float* a, const float* w, const float* a2,
                    const float* w2, uint32_t m, uint32_t k, uint32_t n, const float* bias,
                    int act, double act_param, float* out);
// out = act(f32(f32(addend + a*w) + bias)), the a*w chain k-ascending per output
int bgnn_run_linear_add(bgnn_ctx* ctx, const float* a, const float* w, uint32_t m, uint32_t k,
                        uint32_t n, const float* addend, const float* bias, int act,
                        double act_param, float* out);
// out = act(f32(f32(addend + a1*w1 + a2*w2) + bias)) on the tcgen05 tensor
// cores (3xTF32, one f32 accumulator per output); a2/w2 optional (k2 = 0).
// BGNN_ERR_UNSUPPORTED (no error recorded) when the operands do not suit
// TMA (row lengths not a multiple of 4, unaligned bases): use the FP32 path.
int bgnn_run_linear_tc(bgnn_ctx* ctx, const float* a1, const float* w1, uint32_t k1,
                       const float* a2, const float* w2, uint32_t k2, uint32_t m, uint32_t n,
                       const float* addend, const float* bias, int act, double act_param,
                       float* out);
int bgnn_run_activation(bgnn_ctx* ctx, int act, double param, const float* x, uint64_t n,
                        float* out);
int bgnn_run_add(bgnn_ctx* ctx, const float* a, const float* b, uint64_t n, float* out);
int bgnn_run_l2norm(bgnn_ctx* ctx, float* x, uint32_t m, uint32_t n);
int bgnn_run_gather_rows(bgnn_ctx* ctx, const float* x, uint32_t num_x_rows,
                         const uint32_t* idx, uint64_t n, uint32_t f, float* out);
int bgnn_run_spmv(bgnn_ctx* ctx, const uint32_t* row_ptr, const uint32_t* col,
                  const float* val, const float* x, uint32_t num_rows, float* out);

// Counter-based uniform draw in [0, 1) standing in for Math.random() at
// position i of a training-mode dropout: the SplitMix64 output for state
// seed + (i+1) * 0x9E3779B97F4A7C15, top 53 bits scaled by 2^-53.
__host__ __device__ __forceinline__ double bgnn_uniform(uint64_t seed, uint64_t i) {
  uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (double)(z >> 11) * (1.0 / 9007199254740992.0);
}

// ---------------------------------------------------------------------------
// shared device helpers: the reference's activations and f32 store points
// ---------------------------------------------------------------------------
__device__ __forceinline__ float apply_act(float v, int act, double p) {
  switch (act) {
    case BGNN_ACT_RELU:  // wasmRelu: x > 0 ? x : 0 (NaN -> 0)
      return v > 0.0f ? v : 0.0f;
    case BGNN_ACT_RELU_MAX:  // Math.max(0, x): NaN propagates, -0 -> +0
      return (v != v) ? v : (v > 0.0f ? v : 0.0f);
    case BGNN_ACT_ELU:  // x > 0 ? x : alpha*(exp(x)-1), evaluated in double
      return v > 0.0f ? v : __double2float_rn(__dmul_rn(p, __dsub_rn(exp((double)v), 1.0)));
    case BGNN_ACT_LEAKY_RELU:
      return v > 0.0f ? v : __double2float_rn(__dmul_rn(p, (double)v));
    case BGNN_ACT_SIGMOID:  // 1 / (1 + Math.exp(-x))
      return __double2float_rn(__ddiv_rn(1.0, __dadd_rn(1.0, exp(-(double)v))));
    case BGNN_ACT_TANH:
      return __double2float_rn(tanh((double)v));
    case BGNN_ACT_GELU: {  // 0.5*x*(1 + tanh(sqrt(2/pi)*(x + 0.044715*x*x*x))), left to right
      const double x = (double)v;
      const double s2p = __dsqrt_rn(__ddiv_rn(2.0, 3.141592653589793));
      const double cube = __dmul_rn(__dmul_rn(__dmul_rn(0.044715, x), x), x);
      const double inner = __dmul_rn(s2p, __dadd_rn(x, cube));
      return __double2float_rn(__dmul_rn(__dmul_rn(0.5, x), __dadd_rn(1.0, tanh(inner))));
    }
    case BGNN_ACT_SILU: {  // x / (1 + Math.exp(-x))
      const double x = (double)v;
      return __double2float_rn(__ddiv_rn(x, __dadd_rn(1.0, exp(-x))));
    }
    default:
      return v;
  }
}
