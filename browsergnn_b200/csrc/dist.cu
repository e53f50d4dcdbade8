// Multi-GPU message passing over NCCL: one process per GPU, a row partition
// (partition.cu) per rank, and the halo rows moved by grouped NCCL
// send/receive over NVLink into local memory before the local aggregation
// reads them.  The reference has no multi-device code; these entry points run
// SAGEConv.forward (src/layers/sage.ts:113-217) and SparseCSR.matmul
// (src/core/sparse.ts:322-344) on a partitioned graph with the same per-row
// order and roundings as on one GPU, so the result is the same bits.
//
// Overlap: the halo exchange starts on a high-priority stream at the start of
// the layer, while the root-weight product x * W_self (owned rows only) runs
// on a side stream; the aggregation starts when the halo rows have landed.
// On request (bgnn_dist_set_pipeline) the exchange runs in column chunks and
// the aggregation of chunk c (its columns of every row, each row still summed
// in edge order) starts as soon as chunk c has landed, leaving `reserve` SMs
// to the NCCL kernels while later chunks are in flight.
//
// Early sends (BGNN_DIST_SEND_OUT): when a layer's output is the next
// layer's [owned | halo] buffer, the layer's last product runs in row blocks
// and each block's rows are packed and sent as soon as the block is written,
// so the next layer's exchange overlaps this layer's product; the next layer
// then finds its halo in flight and only waits for it.
//
// Timeouts: the communicator is created non-blocking and every piece of NCCL
// work is watched by a thread that aborts the communicator when the work is
// not done by its deadline (timeout_ms after it was enqueued) or NCCL reports
// an asynchronous error; from then on every call on the object returns
// BGNN_ERR_TIMEOUT (or BGNN_ERR_CUDA).  Aborting ends the NCCL kernels, so
// the streams drain instead of waiting for a peer that is gone.
//
// NCCL is resolved at run time (dlopen): the copy already loaded into the
// process (PyTorch's, for instance) when there is one, else libnccl.so.2 from
// the loader path or BGNN_NCCL_LIBRARY.  The library therefore links no NCCL
// and loads without it; only these entry points need it.
#include <dlfcn.h>
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <deque>
#include <mutex>
#include <thread>

#include "bgnn_internal.cuh"

namespace {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  ncclResult_t (*GetVersion)(int*) = nullptr;
  bool ok = false;
  std::string why;
};

template <class F>
bool sym(void* h, const char* name, F& f) {
  f = reinterpret_cast<F>(dlsym(h, name));
  return f != nullptr;
}

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) {
      const char* path = std::getenv("BGNN_NCCL_LIBRARY");
      h = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    }
    if (!h) {
      const char* e = dlerror();
      api.why = std::string("cannot load NCCL: ") + (e ? e : "unknown");
      return;
    }
    bool ok = sym(h, "ncclGetUniqueId", api.GetUniqueId) &&
              sym(h, "ncclCommInitRankConfig", api.CommInitRankConfig) &&
              sym(h, "ncclCommDestroy", api.CommDestroy) && sym(h, "ncclCommAbort", api.CommAbort) &&
              sym(h, "ncclCommGetAsyncError", api.CommGetAsyncError) &&
              sym(h, "ncclSend", api.Send) && sym(h, "ncclRecv", api.Recv) &&
              sym(h, "ncclGroupStart", api.GroupStart) && sym(h, "ncclGroupEnd", api.GroupEnd) &&
              sym(h, "ncclAllReduce", api.AllReduce) &&
              sym(h, "ncclGetErrorString", api.GetErrorString) &&
              sym(h, "ncclGetVersion", api.GetVersion);
    if (!ok) {
      api.why = "NCCL library lacks an expected symbol";
      return;
    }
    api.ok = true;
  });
  return api;
}

constexpr int kMaxChunks = 8;

using Clock = std::chrono::steady_clock;

}  // namespace

struct bgnn_dist {
  bgnn_ctx* ctx = nullptr;
  int device = 0;
  uint32_t world = 1, rank = 0;
  uint32_t timeout_ms = 0;
  ncclComm_t comm = nullptr;
  cudaStream_t nccl_stream = nullptr;  // high priority: its CTAs are placed first
  cudaStream_t side_stream = nullptr;  // the root-weight product
  cudaEvent_t ev_start = nullptr, ev_side = nullptr, ev_chunk[kMaxChunks] = {};
  // staging for packed send rows and received halo chunks
  float* send_buf = nullptr;
  float* recv_buf = nullptr;
  uint64_t send_cap = 0, recv_cap = 0;  // floats
  float* st_buf = nullptr;              // x * W_self of the SAGE layer
  uint64_t st_cap = 0;
  uint32_t chunks = 0;                  // 0: chosen per call from the width
  uint32_t reserve_sms = 16;            // SMs the aggregation leaves to NCCL while chunks fly
  // early sends: row blocks of the last product, their events, and the
  // buffer whose exchange is in flight (landed at ev_early)
  uint32_t row_blocks = 4;
  cudaEvent_t ev_rows[kMaxChunks] = {};
  cudaEvent_t ev_early = nullptr;
  const float* early_buf = nullptr;
  const bgnn_part* early_part = nullptr;
  uint32_t early_f = 0;
  // watchdog
  std::mutex mu;
  std::condition_variable cv;
  std::deque<std::pair<cudaEvent_t, Clock::time_point>> pending;
  std::vector<cudaEvent_t> spare;
  std::thread watchdog;
  bool stop = false;
  std::atomic<int> failed{BGNN_OK};
  std::string fail_msg;
  bool aborted = false;
};

namespace {

int dist_fail(bgnn_dist* d) {
  const int f = d->failed.load();
  if (f == BGNN_OK) return BGNN_OK;
  return bgnn_set_error(d->ctx, f, "distributed context failed: %s", d->fail_msg.c_str());
}

// (mu held) abort the communicator once; later calls report `code`
void abort_locked(bgnn_dist* d, int code, const std::string& why) {
  if (!d->aborted && d->comm) {
    nccl().CommAbort(d->comm);
    d->aborted = true;
  }
  int expect = BGNN_OK;
  if (d->failed.compare_exchange_strong(expect, code)) d->fail_msg = why;
  // (destroying an event whose work is pending is allowed: it is released
  // when the work ends, which the abort makes happen)
  for (auto& pe : d->pending) cudaEventDestroy(pe.first);
  d->pending.clear();
}

void watchdog_loop(bgnn_dist* d) {
  cudaSetDevice(d->device);
  std::unique_lock<std::mutex> lk(d->mu);
  while (!d->stop) {
    d->cv.wait_for(lk, std::chrono::milliseconds(2));
    if (d->stop || d->aborted) continue;
    while (!d->pending.empty()) {
      auto& f = d->pending.front();
      const cudaError_t q = cudaEventQuery(f.first);
      if (q == cudaSuccess) {
        d->spare.push_back(f.first);
        d->pending.pop_front();
        continue;
      }
      if (q != cudaErrorNotReady) {
        abort_locked(d, BGNN_ERR_CUDA, std::string("CUDA error while waiting for NCCL: ") +
                                           cudaGetErrorString(q));
        break;
      }
      ncclResult_t st = ncclSuccess;
      nccl().CommGetAsyncError(d->comm, &st);
      if (st != ncclSuccess && st != ncclInProgress) {
        abort_locked(d, BGNN_ERR_CUDA, std::string("NCCL: ") + nccl().GetErrorString(st));
        break;
      }
      if (Clock::now() > f.second) {
        abort_locked(d, BGNN_ERR_TIMEOUT, "NCCL work not done within the timeout (a peer failed "
                                          "or never joined); communicator aborted");
      }
      break;
    }
  }
}

// (mu held) wait until non-blocking NCCL calls have been enqueued
int wait_enqueued_locked(bgnn_dist* d, Clock::time_point deadline) {
  for (;;) {
    ncclResult_t st = ncclSuccess;
    nccl().CommGetAsyncError(d->comm, &st);
    if (st == ncclSuccess) return BGNN_OK;
    if (st != ncclInProgress) {
      abort_locked(d, BGNN_ERR_CUDA, std::string("NCCL: ") + nccl().GetErrorString(st));
      return dist_fail(d);
    }
    if (Clock::now() > deadline) {
      abort_locked(d, BGNN_ERR_TIMEOUT, "NCCL call not enqueued within the timeout");
      return dist_fail(d);
    }
    std::this_thread::yield();
  }
}

// (mu held) record an event on the NCCL stream and give it to the watchdog;
// `marker` (owned by the caller, never recycled) is recorded at the same
// point for the caller's streams to wait on
int watch_locked(bgnn_dist* d, cudaEvent_t marker) {
  cudaEvent_t ev = nullptr;
  if (!d->spare.empty()) {
    ev = d->spare.back();
    d->spare.pop_back();
  } else {
    BGNN_CUDA(d->ctx, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  }
  BGNN_CUDA(d->ctx, cudaEventRecord(ev, d->nccl_stream));
  d->pending.emplace_back(ev, Clock::now() + std::chrono::milliseconds(d->timeout_ms));
  if (marker) BGNN_CUDA(d->ctx, cudaEventRecord(marker, d->nccl_stream));
  d->cv.notify_one();
  return BGNN_OK;
}

int ensure(bgnn_dist* d, float** buf, uint64_t* cap, uint64_t floats) {
  if (floats <= *cap) return BGNN_OK;
  // the old buffer may still be read by queued work: cudaFree waits for the device
  if (*buf) BGNN_CUDA(d->ctx, cudaFree(*buf));
  *buf = nullptr;
  *cap = 0;
  BGNN_CUDA(d->ctx, cudaMalloc(buf, floats * sizeof(float)));
  *cap = floats;
  return BGNN_OK;
}

struct StreamSwap {
  bgnn_ctx* ctx;
  cudaStream_t saved;
  StreamSwap(bgnn_ctx* c, cudaStream_t s) : ctx(c), saved(c->stream) { c->stream = s; }
  ~StreamSwap() { ctx->stream = saved; }
};

struct GridBudget {
  bgnn_ctx* ctx;
  int saved;
  GridBudget(bgnn_ctx* c, int sms) : ctx(c), saved(c->grid_sms) { c->grid_sms = sms; }
  ~GridBudget() { ctx->grid_sms = saved; }
};

// One chunk unless the caller asks for more: a column slice re-walks every
// edge's index and row bookkeeping, so four 64-column aggregations of a
// 256-column layer took 6.67 ms against 4.68 ms for one (2 GPUs), more than
// the 1.2 ms exchange they would hide -- which x * W_self already covers
// (2-GPU step 26.4 ms with one chunk, 31.4 ms with four).
uint32_t pick_chunks(const bgnn_dist* d, uint32_t f) {
  if (d->world == 1) return 1;
  uint32_t c = d->chunks ? d->chunks : 1u;
  if (c > kMaxChunks) c = kMaxChunks;
  while (c > 1 && f / c < 8) c--;
  return c;
}

// chunk c covers columns [c0, c0 + w): widths rounded to multiples of 4 so
// every chunk starts 16-byte aligned
void chunk_cols(uint32_t f, uint32_t chunks, uint32_t c, uint32_t* c0, uint32_t* w) {
  uint32_t step = (f + chunks - 1) / chunks;
  step = (step + 3) & ~3u;
  *c0 = c * step < f ? c * step : f;
  const uint32_t end = (c + 1) * step < f ? (c + 1) * step : f;
  *w = end - *c0;
}

// Enqueue the halo exchange of columns [c0, c0 + w) of x_ext on the NCCL
// stream (after ev_start): pack the rows the peers read, then one group of
// sends and receives.  direct: receive straight into x_ext's halo rows (the
// whole width in one chunk); else into the staging buffer's chunk.
int enqueue_chunk(bgnn_dist* d, const bgnn_part* p, float* x_ext, uint32_t f, uint32_t c0,
                  uint32_t w, bool direct, cudaEvent_t done) {
  bgnn_ctx* ctx = d->ctx;
  const NcclApi& api = nccl();
  float* send = d->send_buf + p->n_send * (uint64_t)c0;
  {
    StreamSwap sw(ctx, d->nccl_stream);
    BGNN_TRY(bgnn_run_pack_cols(ctx, x_ext, f, c0, w, p->send_rows, p->n_send, send));
  }
  float* recv = direct ? x_ext + (uint64_t)p->n_own * f : d->recv_buf + p->n_halo * (uint64_t)c0;
  std::lock_guard<std::mutex> lk(d->mu);
  BGNN_TRY(dist_fail(d));
  const auto deadline = Clock::now() + std::chrono::milliseconds(d->timeout_ms);
  ncclResult_t r = api.GroupStart();
  for (uint32_t q = 0; q < d->world && (r == ncclSuccess || r == ncclInProgress); q++) {
    if (q == d->rank) continue;
    if (p->send_counts[q])
      r = api.Send(send + p->send_off[q] * w, p->send_counts[q] * w, ncclFloat32, (int)q, d->comm,
                   d->nccl_stream);
    if ((r == ncclSuccess || r == ncclInProgress) && p->recv_counts[q])
      r = api.Recv(recv + p->recv_off[q] * w, p->recv_counts[q] * w, ncclFloat32, (int)q, d->comm,
                   d->nccl_stream);
  }
  const ncclResult_t r2 = api.GroupEnd();
  if (r == ncclSuccess || r == ncclInProgress) r = r2;
  if (r != ncclSuccess && r != ncclInProgress) {
    abort_locked(d, BGNN_ERR_CUDA, std::string("NCCL send/recv: ") + api.GetErrorString(r));
    return dist_fail(d);
  }
  BGNN_TRY(wait_enqueued_locked(d, deadline));
  return watch_locked(d, done);
}

// x_ext's halo exchange already in flight (started by the layer that wrote
// it, BGNN_DIST_SEND_OUT): the caller's stream waits for it, and true
bool take_early(bgnn_dist* d, const bgnn_part* p, const float* x_ext, uint32_t f) {
  if (!x_ext || d->early_buf != x_ext || d->early_part != p || d->early_f != f) return false;
  d->early_buf = nullptr;
  d->early_part = nullptr;
  d->early_f = 0;
  return cudaStreamWaitEvent(d->ctx->stream, d->ev_early, 0) == cudaSuccess;
}

// The layer's last product, out[r] = act(f32(f32(st[r] + agg[r] * w) + bias))
// (st NULL: act(f32(agg[r] * w + bias))), in row blocks; each block's send
// rows are packed and sent to the peers as soon as the block is written,
// and the peers' blocks land in out's halo rows.  out: the next layer's
// [n_own + n_halo, n] buffer.
int product_and_send(bgnn_dist* d, const bgnn_part* p, const float* agg, const float* w,
                     uint32_t k, uint32_t n, const float* st, const float* bias, int act,
                     double act_param, float* out) {
  bgnn_ctx* ctx = d->ctx;
  const uint32_t C = d->row_blocks;
  BGNN_TRY(bgnn_part_row_blocks(ctx, p, C));
  BGNN_TRY(ensure(d, &d->send_buf, &d->send_cap, p->n_send * (uint64_t)n + 4));
  const NcclApi& api = nccl();
  const uint32_t m = p->n_own;
  for (uint32_t c = 0; c < C; c++) {
    const uint32_t r0 = bgnn_block_row(m, C, c), r1 = bgnn_block_row(m, C, c + 1);
    if (r1 > r0) {
      const uint64_t o = r0;
      if (st)
        BGNN_TRY(bgnn_run_linear_add(ctx, agg + o * k, w, r1 - r0, k, n, st + o * n, bias, act,
                                     act_param, out + o * n));
      else
        BGNN_TRY(bgnn_run_linear(ctx, agg + o * k, w, nullptr, nullptr, r1 - r0, k, n, bias, act,
                                 act_param, out + o * n));
    }
    BGNN_CUDA(ctx, cudaEventRecord(d->ev_rows[c], ctx->stream));
    BGNN_CUDA(ctx, cudaStreamWaitEvent(d->nccl_stream, d->ev_rows[c], 0));
    {
      StreamSwap sw(ctx, d->nccl_stream);
      BGNN_TRY(bgnn_run_pack_block(ctx, out, n, p, c, d->send_buf));
    }
    std::lock_guard<std::mutex> lk(d->mu);
    BGNN_TRY(dist_fail(d));
    const auto deadline = Clock::now() + std::chrono::milliseconds(d->timeout_ms);
    ncclResult_t r = api.GroupStart();
    for (uint32_t q = 0; q < d->world && (r == ncclSuccess || r == ncclInProgress); q++) {
      if (q == d->rank) continue;
      const uint64_t* bs = p->blk_send.data() + (uint64_t)q * (C + 1);
      const uint64_t* br = p->blk_recv.data() + (uint64_t)q * (C + 1);
      if (bs[c + 1] > bs[c])
        r = api.Send(d->send_buf + bs[c] * n, (bs[c + 1] - bs[c]) * n, ncclFloat32, (int)q, d->comm,
                     d->nccl_stream);
      if ((r == ncclSuccess || r == ncclInProgress) && br[c + 1] > br[c])
        r = api.Recv(out + (m + br[c]) * (uint64_t)n, (br[c + 1] - br[c]) * n, ncclFloat32, (int)q,
                     d->comm, d->nccl_stream);
    }
    const ncclResult_t r2 = api.GroupEnd();
    if (r == ncclSuccess || r == ncclInProgress) r = r2;
    if (r != ncclSuccess && r != ncclInProgress) {
      abort_locked(d, BGNN_ERR_CUDA, std::string("NCCL send/recv: ") + api.GetErrorString(r));
      return dist_fail(d);
    }
    BGNN_TRY(wait_enqueued_locked(d, deadline));
    if (c + 1 == C) BGNN_TRY(watch_locked(d, d->ev_early));
  }
  d->early_buf = out;
  d->early_part = p;
  d->early_f = n;
  return BGNN_OK;
}

// exchange + per-chunk aggregation of x_ext ([n_own + n_halo, f], owned rows
// present) into out ([n_own, f]); aggr as bgnn_aggregate_strided
int exchange_aggregate(bgnn_dist* d, const bgnn_part* p, int aggr, const float* values,
                       float* x_ext, uint32_t f, float* out) {
  bgnn_ctx* ctx = d->ctx;
  const bgnn_graph* g = &p->local;
  if (d->world == 1 || f == 0 || take_early(d, p, x_ext, f))
    return bgnn_run_aggregate_cols(ctx, g, aggr, values, x_ext, f, f, out, f);
  const uint32_t chunks = pick_chunks(d, f);
  BGNN_TRY(ensure(d, &d->send_buf, &d->send_cap, p->n_send * (uint64_t)f + 4));
  if (chunks > 1) BGNN_TRY(ensure(d, &d->recv_buf, &d->recv_cap, p->n_halo * (uint64_t)f + 4));
  // the owned rows of x_ext are written on the caller's stream
  BGNN_CUDA(ctx, cudaEventRecord(d->ev_start, ctx->stream));
  BGNN_CUDA(ctx, cudaStreamWaitEvent(d->nccl_stream, d->ev_start, 0));
  for (uint32_t c = 0; c < chunks; c++) {
    uint32_t c0, w;
    chunk_cols(f, chunks, c, &c0, &w);
    if (w == 0) continue;
    BGNN_TRY(enqueue_chunk(d, p, x_ext, f, c0, w, chunks == 1, d->ev_chunk[c]));
  }
  for (uint32_t c = 0; c < chunks; c++) {
    uint32_t c0, w;
    chunk_cols(f, chunks, c, &c0, &w);
    if (w == 0) continue;
    BGNN_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, d->ev_chunk[c], 0));
    if (chunks > 1)
      BGNN_TRY(bgnn_run_unpack_cols(ctx, d->recv_buf + p->n_halo * (uint64_t)c0, p->n_halo, w,
                                    x_ext + (uint64_t)p->n_own * f, f, c0));
    // while later chunks are in flight, leave SMs to the NCCL kernels
    const bool more = c + 1 < chunks;
    GridBudget gb(ctx, more && ctx->num_sms > (int)d->reserve_sms + 8
                           ? ctx->num_sms - (int)d->reserve_sms : 0);
    BGNN_TRY(bgnn_run_aggregate_cols(ctx, g, aggr, values, x_ext + c0, f, w, out + c0, f));
  }
  return BGNN_OK;
}

int dist_ok(bgnn_dist* d) {
  if (!d) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(d->ctx, cudaSetDevice(d->device));
  return dist_fail(d);
}

int part_matches(bgnn_dist* d, const bgnn_part* p) {
  if (!p) return bgnn_set_error(d->ctx, BGNN_ERR_INVALID_ARG, "NULL partition");
  if (p->world != d->world || p->rank != d->rank)
    return bgnn_set_error(d->ctx, BGNN_ERR_INVALID_ARG,
                          "partition is rank %u of %u, the context rank %u of %u", p->rank,
                          p->world, d->rank, d->world);
  return BGNN_OK;
}

}  // namespace

// ---- C ABI -----------------------------------------------------------------

extern "C" int bgnn_dist_unique_id(uint8_t* id_out) {
  if (!id_out) return BGNN_ERR_INVALID_ARG;
  const NcclApi& api = nccl();
  if (!api.ok) return BGNN_ERR_UNSUPPORTED;
  ncclUniqueId id;
  if (api.GetUniqueId(&id) != ncclSuccess) return BGNN_ERR_CUDA;
  static_assert(sizeof(id) == BGNN_UNIQUE_ID_BYTES, "NCCL unique id size");
  memcpy(id_out, &id, sizeof(id));
  return BGNN_OK;
}

extern "C" int bgnn_dist_create(bgnn_ctx* ctx, const uint8_t* unique_id, uint32_t world,
                                uint32_t rank, uint32_t timeout_ms, uint32_t max_ctas,
                                bgnn_dist** out) {
  if (!ctx || !out || !unique_id) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  BGNN_REQUIRE(ctx, world >= 1 && rank < world, "rank %u outside [0, %u)", rank, world);
  BGNN_REQUIRE(ctx, timeout_ms > 0, "timeout must be positive");
  const NcclApi& api = nccl();
  if (!api.ok) return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED, "%s", api.why.c_str());
  bgnn_dist* d = new bgnn_dist();
  d->ctx = ctx;
  d->device = ctx->device;
  d->world = world;
  d->rank = rank;
  d->timeout_ms = timeout_ms;
  int lo_prio = 0, hi_prio = 0;
  bool ok = cudaDeviceGetStreamPriorityRange(&lo_prio, &hi_prio) == cudaSuccess;
  ok = ok && cudaStreamCreateWithPriority(&d->nccl_stream, cudaStreamNonBlocking, hi_prio) ==
                 cudaSuccess;
  ok = ok && cudaStreamCreateWithFlags(&d->side_stream, cudaStreamNonBlocking) == cudaSuccess;
  ok = ok && cudaEventCreateWithFlags(&d->ev_start, cudaEventDisableTiming) == cudaSuccess;
  ok = ok && cudaEventCreateWithFlags(&d->ev_side, cudaEventDisableTiming) == cudaSuccess;
  for (int c = 0; c < kMaxChunks; c++) {
    ok = ok && cudaEventCreateWithFlags(&d->ev_chunk[c], cudaEventDisableTiming) == cudaSuccess;
    ok = ok && cudaEventCreateWithFlags(&d->ev_rows[c], cudaEventDisableTiming) == cudaSuccess;
  }
  ok = ok && cudaEventCreateWithFlags(&d->ev_early, cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    bgnn_dist_destroy(d);
    return bgnn_set_error(ctx, BGNN_ERR_CUDA, "stream/event creation failed");
  }
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // init and enqueue return at once; progress is polled with a deadline
  if (max_ctas) {
    cfg.maxCTAs = (int)max_ctas;
    cfg.minCTAs = 1;
    d->reserve_sms = max_ctas;
  }
  ncclResult_t r = api.CommInitRankConfig(&d->comm, (int)world, id, (int)rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    const char* why = api.GetErrorString(r);
    d->comm = nullptr;
    bgnn_dist_destroy(d);
    return bgnn_set_error(ctx, BGNN_ERR_CUDA, "ncclCommInitRankConfig: %s", why);
  }
  {
    std::lock_guard<std::mutex> lk(d->mu);
    const int rc = wait_enqueued_locked(d, Clock::now() + std::chrono::milliseconds(timeout_ms));
    if (rc != BGNN_OK) {
      const std::string msg = d->fail_msg;
      d->comm = nullptr;  // aborted, which also freed it
      bgnn_dist_destroy(d);
      return bgnn_set_error(ctx, rc, "communicator init: %s", msg.c_str());
    }
  }
  d->watchdog = std::thread(watchdog_loop, d);
  *out = d;
  return BGNN_OK;
}

extern "C" int bgnn_dist_destroy(bgnn_dist* d) {
  if (!d) return BGNN_OK;
  cudaSetDevice(d->device);
  if (d->watchdog.joinable()) {
    {
      std::lock_guard<std::mutex> lk(d->mu);
      d->stop = true;
    }
    d->cv.notify_all();
    d->watchdog.join();
  }
  if (d->nccl_stream) cudaStreamSynchronize(d->nccl_stream);
  if (d->side_stream) cudaStreamSynchronize(d->side_stream);
  if (d->comm) {
    if (d->aborted || d->failed.load() != BGNN_OK) {
      if (!d->aborted) nccl().CommAbort(d->comm);
    } else {
      nccl().CommDestroy(d->comm);
    }
  }
  for (auto& pe : d->pending) cudaEventDestroy(pe.first);
  for (auto ev : d->spare) cudaEventDestroy(ev);
  if (d->ev_start) cudaEventDestroy(d->ev_start);
  if (d->ev_side) cudaEventDestroy(d->ev_side);
  for (int c = 0; c < kMaxChunks; c++) {
    if (d->ev_chunk[c]) cudaEventDestroy(d->ev_chunk[c]);
    if (d->ev_rows[c]) cudaEventDestroy(d->ev_rows[c]);
  }
  if (d->ev_early) cudaEventDestroy(d->ev_early);
  cudaFree(d->send_buf);
  cudaFree(d->recv_buf);
  cudaFree(d->st_buf);
  if (d->nccl_stream) cudaStreamDestroy(d->nccl_stream);
  if (d->side_stream) cudaStreamDestroy(d->side_stream);
  delete d;
  return BGNN_OK;
}

extern "C" int bgnn_dist_abort(bgnn_dist* d) {
  if (!d) return BGNN_ERR_INVALID_ARG;
  cudaSetDevice(d->device);
  std::lock_guard<std::mutex> lk(d->mu);
  abort_locked(d, BGNN_ERR_DEVICE, "aborted by the caller");
  return BGNN_OK;
}

extern "C" int bgnn_dist_set_pipeline(bgnn_dist* d, uint32_t chunks, uint32_t reserve_sms) {
  BGNN_TRY(dist_ok(d));
  BGNN_REQUIRE(d->ctx, chunks <= kMaxChunks, "at most %d chunks", kMaxChunks);
  d->chunks = chunks;
  d->reserve_sms = reserve_sms;
  return BGNN_OK;
}

extern "C" int bgnn_dist_exchange(bgnn_dist* d, const bgnn_part* p, float* x_ext,
                                  uint32_t num_features) {
  BGNN_TRY(dist_ok(d));
  BGNN_TRY(part_matches(d, p));
  BGNN_REQUIRE(d->ctx, x_ext || (uint64_t)(p->n_own + p->n_halo) * num_features == 0, "NULL x_ext");
  if (d->world == 1 || num_features == 0 || take_early(d, p, x_ext, num_features))
    return BGNN_OK;
  bgnn_ctx* ctx = d->ctx;
  BGNN_TRY(ensure(d, &d->send_buf, &d->send_cap, p->n_send * (uint64_t)num_features + 4));
  BGNN_CUDA(ctx, cudaEventRecord(d->ev_start, ctx->stream));
  BGNN_CUDA(ctx, cudaStreamWaitEvent(d->nccl_stream, d->ev_start, 0));
  BGNN_TRY(enqueue_chunk(d, p, x_ext, num_features, 0, num_features, true, d->ev_chunk[0]));
  BGNN_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, d->ev_chunk[0], 0));
  return BGNN_OK;
}

extern "C" int bgnn_dist_aggregate(bgnn_dist* d, const bgnn_part* p, int aggr, float* x_ext,
                                   uint32_t num_features, float* out) {
  BGNN_TRY(dist_ok(d));
  BGNN_TRY(part_matches(d, p));
  BGNN_REQUIRE(d->ctx, aggr >= BGNN_AGGR_SUM && aggr <= BGNN_AGGR_MAX, "unknown aggregation %d",
               aggr);
  BGNN_REQUIRE(d->ctx, (x_ext && out) || (uint64_t)p->n_own * num_features == 0,
               "NULL x_ext/out");
  return exchange_aggregate(d, p, aggr, nullptr, x_ext, num_features, out);
}

extern "C" int bgnn_dist_spmm(bgnn_dist* d, const bgnn_part* p, const float* values,
                              float* x_ext, uint32_t num_features, float* out) {
  BGNN_TRY(dist_ok(d));
  BGNN_TRY(part_matches(d, p));
  BGNN_REQUIRE(d->ctx, (x_ext && out) || (uint64_t)p->n_own * num_features == 0,
               "NULL x_ext/out");
  BGNN_REQUIRE(d->ctx, values || p->n_local_entries == 0, "NULL values");
  return exchange_aggregate(d, p, BGNN_AGGR_SPMM, values, x_ext, num_features, out);
}

extern "C" int bgnn_dist_sage_layer(bgnn_dist* d, const bgnn_part* p, int aggr, float* x_ext,
                                    uint32_t k, uint32_t n, const float* w_neigh,
                                    const float* w_self, const float* bias, int act,
                                    double act_param, float* agg, float* out) {
  return bgnn_dist_sage_layer_ex(d, p, aggr, x_ext, k, n, w_neigh, w_self, bias, act, act_param,
                                 agg, out, 0u);
}

extern "C" int bgnn_dist_set_row_blocks(bgnn_dist* d, uint32_t blocks) {
  BGNN_TRY(dist_ok(d));
  BGNN_REQUIRE(d->ctx, blocks >= 1 && blocks <= (uint32_t)kMaxChunks, "row blocks %u outside [1, %d]",
               blocks, kMaxChunks);
  d->row_blocks = blocks;
  return BGNN_OK;
}

extern "C" int bgnn_dist_sage_layer_ex(bgnn_dist* d, const bgnn_part* p, int aggr, float* x_ext,
                                       uint32_t k, uint32_t n, const float* w_neigh,
                                       const float* w_self, const float* bias, int act,
                                       double act_param, float* agg, float* out, uint32_t flags) {
  BGNN_TRY(dist_ok(d));
  BGNN_TRY(part_matches(d, p));
  bgnn_ctx* ctx = d->ctx;
  BGNN_REQUIRE(ctx, aggr >= BGNN_AGGR_SUM && aggr <= BGNN_AGGR_MAX, "unknown aggregation %d", aggr);
  BGNN_REQUIRE(ctx, act >= BGNN_ACT_NONE && act <= BGNN_ACT_SILU, "unknown activation %d", act);
  BGNN_REQUIRE(ctx, (flags & ~BGNN_DIST_SEND_OUT) == 0, "unknown flags 0x%x", flags);
  const uint64_t m = p->n_own;
  BGNN_REQUIRE(ctx, (x_ext && agg && out && w_neigh) || m * k * n == 0, "NULL argument");
  const bool send_out = (flags & BGNN_DIST_SEND_OUT) && d->world > 1;
  if (m == 0 || n == 0) {
    // a rank without rows still takes part in the exchanges its peers wait for
    if (k) BGNN_TRY(exchange_aggregate(d, p, aggr, nullptr, x_ext, k, agg));
    return send_out && n ? product_and_send(d, p, agg, w_neigh, k, n, nullptr, bias, act,
                                            act_param, out)
                         : BGNN_OK;
  }
  const bool root = w_self != nullptr;
  if (root) {
    // x * W_self (owned rows only) on the side stream from the start of the layer
    BGNN_TRY(ensure(d, &d->st_buf, &d->st_cap, m * n + 4));
    BGNN_CUDA(ctx, cudaEventRecord(d->ev_start, ctx->stream));
    BGNN_CUDA(ctx, cudaStreamWaitEvent(d->side_stream, d->ev_start, 0));
    {
      StreamSwap sw(ctx, d->side_stream);
      BGNN_TRY(bgnn_run_linear(ctx, x_ext, w_self, nullptr, nullptr, (uint32_t)m, k, n, nullptr,
                               BGNN_ACT_NONE, 0.0, d->st_buf));
    }
    BGNN_CUDA(ctx, cudaEventRecord(d->ev_side, d->side_stream));
  }
  BGNN_TRY(exchange_aggregate(d, p, aggr, nullptr, x_ext, k, agg));
  if (root) BGNN_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, d->ev_side, 0));
  if (send_out)
    return product_and_send(d, p, agg, w_neigh, k, n, root ? d->st_buf : nullptr, bias, act,
                            act_param, out);
  if (root) {
    // out = act(f32(f32(St + agg * W_neigh) + bias)): the two f32 products and
    // the final rounding of bgnn_sage_linear
    return bgnn_run_linear_add(ctx, agg, w_neigh, (uint32_t)m, k, n, d->st_buf, bias, act,
                               act_param, out);
  }
  return bgnn_run_linear(ctx, agg, w_neigh, nullptr, nullptr, (uint32_t)m, k, n, bias, act,
                         act_param, out);
}

extern "C" int bgnn_dist_allreduce_max(bgnn_dist* d, double* values, uint32_t count) {
  BGNN_TRY(dist_ok(d));
  bgnn_ctx* ctx = d->ctx;
  BGNN_REQUIRE(ctx, values || count == 0, "NULL values");
  if (count == 0) return BGNN_OK;
  DevTmp buf;
  BGNN_TRY(bgnn_tmp_alloc(ctx, buf, count * sizeof(double)));
  BGNN_CUDA(ctx, cudaMemcpyAsync(buf.p, values, count * sizeof(double), cudaMemcpyHostToDevice,
                                 ctx->stream));
  BGNN_CUDA(ctx, cudaEventRecord(d->ev_start, ctx->stream));
  BGNN_CUDA(ctx, cudaStreamWaitEvent(d->nccl_stream, d->ev_start, 0));
  {
    std::lock_guard<std::mutex> lk(d->mu);
    BGNN_TRY(dist_fail(d));
    const auto deadline = Clock::now() + std::chrono::milliseconds(d->timeout_ms);
    const ncclResult_t r = nccl().AllReduce(buf.p, buf.p, count, ncclFloat64, ncclMax, d->comm,
                                            d->nccl_stream);
    if (r != ncclSuccess && r != ncclInProgress) {
      abort_locked(d, BGNN_ERR_CUDA, std::string("NCCL all-reduce: ") + nccl().GetErrorString(r));
      return dist_fail(d);
    }
    BGNN_TRY(wait_enqueued_locked(d, deadline));
    BGNN_TRY(watch_locked(d, d->ev_chunk[0]));
  }
  BGNN_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, d->ev_chunk[0], 0));
  BGNN_CUDA(ctx, cudaMemcpyAsync(values, buf.p, count * sizeof(double), cudaMemcpyDeviceToHost,
                                 ctx->stream));
  return bgnn_dist_synchronize(d);
}

extern "C" int bgnn_dist_synchronize(bgnn_dist* d) {
  BGNN_TRY(dist_ok(d));
  bgnn_ctx* ctx = d->ctx;
  // wait for the caller's stream, giving up (and aborting) when the NCCL work
  // it depends on misses its deadline
  cudaEvent_t ev = nullptr;
  BGNN_CUDA(ctx, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  cudaError_t e = cudaEventRecord(ev, ctx->stream);
  while (e == cudaSuccess) {
    e = cudaEventQuery(ev);
    if (e == cudaErrorNotReady) {
      if (d->failed.load() != BGNN_OK) break;
      std::this_thread::sleep_for(std::chrono::microseconds(200));
      e = cudaSuccess;
      continue;
    }
    break;
  }
  if (d->failed.load() != BGNN_OK) {
    // the aborted NCCL kernels have exited; let the stream drain
    cudaStreamSynchronize(ctx->stream);
    cudaGetLastError();
    cudaEventDestroy(ev);
    return dist_fail(d);
  }
  cudaEventDestroy(ev);
  if (e != cudaSuccess)
    return bgnn_set_error(ctx, BGNN_ERR_CUDA, "synchronize: %s", cudaGetErrorString(e));
  return bgnn_check_device_error(ctx);
}
