// Host <-> device copies of caller-owned host memory.
//
// The reference's WebGPU manager uploads each operand from a JS typed array
// and reads a fresh one back (src/backend/webgpu/compute-pipeline.ts:182-190);
// typed arrays are ordinary pageable memory.  A DMA engine can only read or
// write page-locked memory, so a pageable copy is staged: here through a
// ring of library-owned pinned chunks, each filled (or drained) by a pool of
// host threads while the DMA of the neighbouring chunk runs on a copy stream
// of the library's own.  Page-locked caller memory is copied directly.
// Every copy is synchronous for the caller (the data is in place when the
// call returns) and waits first for the work already queued on the
// context's stream.  Two rings per device let two copies (say the edge list
// and the features) proceed at once from two host threads.
#include <condition_variable>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>

#include "bgnn_internal.cuh"

namespace {

constexpr size_t kChunk = 32u << 20;  // bytes per staging chunk
constexpr int kBufs = 3;              // chunks in flight per ring
constexpr int kRings = 2;
constexpr int kMaxDevices = 64;

// a fixed pool of threads that split one memcpy between them
class CopyPool {
 public:
  explicit CopyPool(int n) : n_(n) {
    for (int i = 0; i < n_; i++) threads_.emplace_back([this, i] { worker(i); });
  }
  ~CopyPool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
      gen_++;
    }
    cv_.notify_all();
    for (auto& t : threads_) t.join();
  }
  // dst[0, len) = src[0, len), split into n_ + 1 parts (the caller does one)
  void copy(void* dst, const void* src, size_t len) {
    const size_t parts = (size_t)n_ + 1;
    const size_t step = ((len + parts - 1) / parts + 63) & ~(size_t)63;
    std::unique_lock<std::mutex> lk(mu_);
    dst_ = static_cast<char*>(dst);
    src_ = static_cast<const char*>(src);
    len_ = len;
    step_ = step;
    pending_ = n_;
    gen_++;
    lk.unlock();
    cv_.notify_all();
    part(n_);
    lk.lock();
    done_.wait(lk, [this] { return pending_ == 0; });
  }

 private:
  void part(int i) {
    const size_t a = (size_t)i * step_;
    if (a >= len_) return;
    const size_t b = a + step_ < len_ ? a + step_ : len_;
    memcpy(dst_ + a, src_ + a, b - a);
  }
  void worker(int i) {
    uint64_t seen = 0;
    for (;;) {
      std::unique_lock<std::mutex> lk(mu_);
      cv_.wait(lk, [&] { return gen_ != seen; });
      seen = gen_;
      if (stop_) return;
      lk.unlock();
      part(i);
      lk.lock();
      if (--pending_ == 0) done_.notify_one();
    }
  }
  int n_;
  std::vector<std::thread> threads_;
  std::mutex mu_;
  std::condition_variable cv_, done_;
  uint64_t gen_ = 0;
  bool stop_ = false;
  int pending_ = 0;
  char* dst_ = nullptr;
  const char* src_ = nullptr;
  size_t len_ = 0, step_ = 0;
};

struct Ring {
  std::mutex busy;
  void* buf[kBufs] = {};
  cudaEvent_t ev[kBufs] = {};
  cudaStream_t stream = nullptr;
  bool ready = false;
  std::unique_ptr<CopyPool> pool;
};

struct DeviceRings {
  Ring ring[kRings];
};

std::mutex g_rings_mu;
DeviceRings* g_rings[kMaxDevices] = {};

int ring_init(bgnn_ctx* ctx, Ring& r) {
  if (r.ready) return BGNN_OK;
  for (int b = 0; b < kBufs; b++) {
    BGNN_CUDA(ctx, cudaHostAlloc(&r.buf[b], kChunk, cudaHostAllocDefault));
    BGNN_CUDA(ctx, cudaEventCreateWithFlags(&r.ev[b], cudaEventDisableTiming));
  }
  BGNN_CUDA(ctx, cudaStreamCreateWithFlags(&r.stream, cudaStreamNonBlocking));
  unsigned hw = std::thread::hardware_concurrency();
  int threads = hw >= 16 ? 7 : (hw >= 4 ? (int)hw / 2 - 1 : 0);
  r.pool.reset(new CopyPool(threads));
  r.ready = true;
  return BGNN_OK;
}

// a free ring of this device (blocks until one is)
Ring* take_ring(bgnn_ctx* ctx, std::unique_lock<std::mutex>* hold) {
  if (ctx->device < 0 || ctx->device >= kMaxDevices) return nullptr;
  DeviceRings* dr;
  {
    std::lock_guard<std::mutex> lk(g_rings_mu);
    if (!g_rings[ctx->device]) g_rings[ctx->device] = new DeviceRings();
    dr = g_rings[ctx->device];
  }
  for (;;) {
    for (int i = 0; i < kRings; i++) {
      std::unique_lock<std::mutex> lk(dr->ring[i].busy, std::try_to_lock);
      if (lk.owns_lock()) {
        *hold = std::move(lk);
        return &dr->ring[i];
      }
    }
    std::this_thread::yield();
  }
}

bool pinned(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

// the copy stream waits for the work queued so far on the context's stream
int after_ctx_stream(bgnn_ctx* ctx, cudaStream_t s) {
  cudaEvent_t ev;
  BGNN_CUDA(ctx, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  cudaError_t e = cudaEventRecord(ev, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s, ev, 0);
  cudaEventDestroy(ev);
  if (e != cudaSuccess)
    return bgnn_set_error(ctx, BGNN_ERR_CUDA, "stream ordering failed: %s", cudaGetErrorString(e));
  return BGNN_OK;
}

}  // namespace

int bgnn_copy_h2d(bgnn_ctx* ctx, void* dst, const void* src, uint64_t bytes) {
  if (bytes == 0) return BGNN_OK;
  std::unique_lock<std::mutex> hold;
  Ring* r = take_ring(ctx, &hold);
  if (!r) return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED, "device ordinal out of range");
  BGNN_TRY(ring_init(ctx, *r));
  BGNN_TRY(after_ctx_stream(ctx, r->stream));
  if (pinned(src)) {
    BGNN_CUDA(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, r->stream));
    BGNN_CUDA(ctx, cudaStreamSynchronize(r->stream));
    return BGNN_OK;
  }
  const char* s = static_cast<const char*>(src);
  char* d = static_cast<char*>(dst);
  uint64_t off = 0;
  for (uint64_t i = 0; off < bytes; i++, off += kChunk) {
    const int b = (int)(i % kBufs);
    const size_t len = bytes - off < kChunk ? (size_t)(bytes - off) : kChunk;
    // the DMA that last read this chunk has finished
    if (i >= (uint64_t)kBufs) BGNN_CUDA(ctx, cudaEventSynchronize(r->ev[b]));
    r->pool->copy(r->buf[b], s + off, len);
    BGNN_CUDA(ctx, cudaMemcpyAsync(d + off, r->buf[b], len, cudaMemcpyHostToDevice, r->stream));
    BGNN_CUDA(ctx, cudaEventRecord(r->ev[b], r->stream));
  }
  BGNN_CUDA(ctx, cudaStreamSynchronize(r->stream));
  return BGNN_OK;
}

int bgnn_copy_d2h(bgnn_ctx* ctx, void* dst, const void* src, uint64_t bytes) {
  if (bytes == 0) return BGNN_OK;
  std::unique_lock<std::mutex> hold;
  Ring* r = take_ring(ctx, &hold);
  if (!r) return bgnn_set_error(ctx, BGNN_ERR_UNSUPPORTED, "device ordinal out of range");
  BGNN_TRY(ring_init(ctx, *r));
  BGNN_TRY(after_ctx_stream(ctx, r->stream));
  if (pinned(dst)) {
    BGNN_CUDA(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, r->stream));
    BGNN_CUDA(ctx, cudaStreamSynchronize(r->stream));
    return BGNN_OK;
  }
  const char* s = static_cast<const char*>(src);
  char* d = static_cast<char*>(dst);
  const uint64_t n = (bytes + kChunk - 1) / kChunk;
  auto issue = [&](uint64_t i) -> int {
    const int b = (int)(i % kBufs);
    const uint64_t off = i * kChunk;
    const size_t len = bytes - off < kChunk ? (size_t)(bytes - off) : kChunk;
    BGNN_CUDA(ctx, cudaMemcpyAsync(r->buf[b], s + off, len, cudaMemcpyDeviceToHost, r->stream));
    BGNN_CUDA(ctx, cudaEventRecord(r->ev[b], r->stream));
    return BGNN_OK;
  };
  for (uint64_t i = 0; i < n && i < (uint64_t)kBufs; i++) BGNN_TRY(issue(i));
  for (uint64_t i = 0; i < n; i++) {
    const int b = (int)(i % kBufs);
    const uint64_t off = i * kChunk;
    const size_t len = bytes - off < kChunk ? (size_t)(bytes - off) : kChunk;
    BGNN_CUDA(ctx, cudaEventSynchronize(r->ev[b]));
    r->pool->copy(d + off, r->buf[b], len);
    if (i + kBufs < n) BGNN_TRY(issue(i + kBufs));
  }
  return BGNN_OK;
}

extern "C" int bgnn_memcpy_h2d(bgnn_ctx* ctx, void* dst_dev, const void* src_host,
                               uint64_t bytes) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  BGNN_REQUIRE(ctx, (dst_dev && src_host) || bytes == 0, "NULL argument");
  return bgnn_copy_h2d(ctx, dst_dev, src_host, bytes);
}

extern "C" int bgnn_memcpy_d2h(bgnn_ctx* ctx, void* dst_host, const void* src_dev,
                               uint64_t bytes) {
  if (!ctx) return BGNN_ERR_INVALID_ARG;
  BGNN_CUDA(ctx, cudaSetDevice(ctx->device));
  BGNN_REQUIRE(ctx, (dst_host && src_dev) || bytes == 0, "NULL argument");
  return bgnn_copy_d2h(ctx, dst_host, src_dev, bytes);
}
