// The host -> device half of the streamed weight mode: a ring of device
// slots fed from host memory on a copy stream, in lock step with a compute
// stream. It backs DoubleBufferRuntime's streamed mode
// (layer_streaming/runtime.py:137-268 of the reference) and the chunked LM
// head (layer_streaming/vocab.py:207-266), which both move a list of host
// spans through the same device slots.
//
// Protocol for one pass over n spans (n transfer units, or n vocab chunks):
//   begin    both streams are ordered after the coordinator's queued work;
//            the copies of spans 0 .. slots-1 are started;
//   acquire  (span i) the compute stream waits for span i's copy; returns
//            the device slot it landed in (slot i % slots);
//   release  (span i) the compute stream is done with the slot: span
//            i + slots is started into it once that point of the compute
//            stream is reached (the copy stream waits on an event);
//   end      the coordinator waits for the last release; the host waits for
//            the coordinator; timing figures are read.
// Nothing allocates device memory; events are created once per ring and
// reused by every pass.
//
// Pinned sources are copied straight from the host arena. With staging
// buffers (the pinned-staging store: a pageable arena plus one pinned buffer
// per slot) a native stager thread runs ahead of the compute loop: for span
// i it waits until the DMA that last read staging buffer i % slots has
// finished, copies the span pageable -> pinned on `copy_threads` native
// threads, and only then starts the H2D copy, so the Python loop never runs
// a memcpy itself. acquire blocks on the host until span i's copy has been
// issued (the "source wait" of the reference's profile).
#include <condition_variable>
#include <chrono>
#include <deque>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "cascade_b200.h"
#include "internal.h"

namespace cb {

int host_copy_parallel(void* dst, const void* src, int64_t bytes, int threads);  // host_io.cu

namespace {

using Clock = std::chrono::steady_clock;

double ms_since(Clock::time_point t0) {
  return std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
}

struct Ring {
  // fixed at creation
  int nslots = 0;
  std::vector<char*> dslots;
  int64_t slot_bytes = 0;
  cudaStream_t copy = nullptr;
  std::vector<char*> staging;  // empty: sources are pinned
  int64_t staging_bytes = 0;
  int copy_threads = 0;
  int device = 0;

  // events, grown to the longest pass
  std::vector<cudaEvent_t> ready, freed;                    // no timing
  std::vector<cudaEvent_t> copy0, copy1, comp0, comp1;      // timing (profile)
  cudaEvent_t pass0 = nullptr, pass1 = nullptr;

  // the current pass
  int n = 0;
  std::vector<const char*> src;
  std::vector<int64_t> bytes;
  cudaStream_t compute = nullptr, coordinator = nullptr;
  bool profile = false;
  bool active = false;
  int64_t moved = 0;
  double source_wait_ms = 0.0;

  // stager thread (staging mode) and the issue state shared with it
  std::mutex mu;
  std::condition_variable cv;
  std::deque<int> jobs;
  std::vector<char> issued;
  std::vector<double> stage_ms;
  std::string failure;
  bool stop = false;
  bool skip = false;  // abort: drop queued jobs
  bool running = false;  // the stager is inside a job
  std::thread stager;

  ~Ring() {
    {
      std::lock_guard<std::mutex> lock(mu);
      stop = true;
    }
    cv.notify_all();
    if (stager.joinable()) stager.join();
    auto destroy = [](std::vector<cudaEvent_t>& v) {
      for (cudaEvent_t e : v)
        if (e) cudaEventDestroy(e);
      v.clear();
    };
    destroy(ready);
    destroy(freed);
    destroy(copy0);
    destroy(copy1);
    destroy(comp0);
    destroy(comp1);
    if (pass0) cudaEventDestroy(pass0);
    if (pass1) cudaEventDestroy(pass1);
  }

  int grow_events(int count) {
    auto grow = [count](std::vector<cudaEvent_t>& v, unsigned flags) -> cudaError_t {
      while (int(v.size()) < count) {
        cudaEvent_t e = nullptr;
        cudaError_t rc = cudaEventCreateWithFlags(&e, flags);
        if (rc != cudaSuccess) return rc;
        v.push_back(e);
      }
      return cudaSuccess;
    };
    cudaError_t rc = grow(ready, cudaEventDisableTiming);
    if (rc == cudaSuccess) rc = grow(freed, cudaEventDisableTiming);
    if (rc == cudaSuccess) rc = grow(copy0, cudaEventDefault);
    if (rc == cudaSuccess) rc = grow(copy1, cudaEventDefault);
    if (rc == cudaSuccess) rc = grow(comp0, cudaEventDefault);
    if (rc == cudaSuccess) rc = grow(comp1, cudaEventDefault);
    if (rc == cudaSuccess && !pass0) rc = cudaEventCreate(&pass0);
    if (rc == cudaSuccess && !pass1) rc = cudaEventCreate(&pass1);
    if (rc != cudaSuccess) return fail(kErrCuda, "cb_ring: event creation failed: %s", cudaGetErrorString(rc));
    return kOk;
  }

  // Start span u's H2D copy from `from` into its slot (any host thread).
  cudaError_t issue_copy(int u, const char* from) {
    cudaError_t rc = cudaSuccess;
    if (u >= nslots) rc = cudaStreamWaitEvent(copy, freed[u - nslots], 0);
    if (rc == cudaSuccess && profile) rc = cudaEventRecord(copy0[u], copy);
    if (rc == cudaSuccess)
      rc = cudaMemcpyAsync(dslots[u % nslots], from, size_t(bytes[u]), cudaMemcpyHostToDevice, copy);
    if (rc == cudaSuccess && profile) rc = cudaEventRecord(copy1[u], copy);
    if (rc == cudaSuccess) rc = cudaEventRecord(ready[u], copy);
    return rc;
  }

  void mark_issued(int u, const std::string& error) {
    {
      std::lock_guard<std::mutex> lock(mu);
      issued[u] = 1;
      if (!error.empty() && failure.empty()) failure = error;
    }
    cv.notify_all();
  }

  // Staging job of span u (stager thread).
  void stage(int u) {
    const Clock::time_point t0 = Clock::now();
    std::string error;
    cudaError_t rc = cudaSetDevice(device);
    // the H2D copy that last read this staging buffer must have finished
    if (rc == cudaSuccess && u >= nslots) rc = cudaEventSynchronize(ready[u - nslots]);
    char* buf = staging[u % nslots];
    if (rc == cudaSuccess) {
      if (host_copy_parallel(buf, src[u], bytes[u], copy_threads) != kOk) error = "cb_ring: staging copy failed";
    }
    const double ms = ms_since(t0);
    if (rc == cudaSuccess && error.empty()) rc = issue_copy(u, buf);
    if (rc != cudaSuccess && error.empty()) error = std::string("cb_ring: ") + cudaGetErrorString(rc);
    {
      std::lock_guard<std::mutex> lock(mu);
      stage_ms.push_back(ms);
    }
    mark_issued(u, error);
  }

  void stager_loop() {
    for (;;) {
      int u = -1;
      {
        std::unique_lock<std::mutex> lock(mu);
        cv.wait(lock, [this] { return stop || !jobs.empty(); });
        if (stop) return;
        u = jobs.front();
        jobs.pop_front();
        if (skip) {
          issued[u] = 1;
          cv.notify_all();
          continue;
        }
        running = true;
      }
      stage(u);
      {
        std::lock_guard<std::mutex> lock(mu);
        running = false;
      }
      cv.notify_all();
    }
  }

  // Start span u: directly (pinned sources) or through the stager.
  int start(int u) {
    if (staging.empty()) {
      cudaError_t rc = issue_copy(u, src[u]);
      {
        std::lock_guard<std::mutex> lock(mu);
        issued[u] = 1;
      }
      if (rc != cudaSuccess) return fail(kErrCuda, "cb_ring: copy of span %d failed: %s", u, cudaGetErrorString(rc));
      return kOk;
    }
    {
      std::lock_guard<std::mutex> lock(mu);
      jobs.push_back(u);
    }
    cv.notify_all();
    return kOk;
  }
};

Ring* as_ring(void* handle) { return static_cast<Ring*>(handle); }

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" int cb_ring_create(int slots, void* const* device_slots, int64_t slot_bytes, void* copy_stream,
                              void* const* staging, int64_t staging_bytes, int copy_threads, void** ring_out) {
  CB_REQUIRE(ring_out, "cb_ring_create: ring_out is null");
  *ring_out = nullptr;
  CB_REQUIRE(slots >= 1 && slots <= 8 && device_slots, "cb_ring_create: 1..8 device slots required");
  CB_REQUIRE(slot_bytes > 0, "cb_ring_create: slot_bytes must be positive");
  for (int i = 0; i < slots; ++i) CB_REQUIRE(device_slots[i], "cb_ring_create: device slot %d is null", i);
  if (staging) {
    CB_REQUIRE(staging_bytes > 0, "cb_ring_create: staging_bytes must be positive");
    for (int i = 0; i < slots; ++i) CB_REQUIRE(staging[i], "cb_ring_create: staging buffer %d is null", i);
  }
  Ring* r = new Ring();
  r->nslots = slots;
  for (int i = 0; i < slots; ++i) r->dslots.push_back(static_cast<char*>(device_slots[i]));
  r->slot_bytes = slot_bytes;
  r->copy = static_cast<cudaStream_t>(copy_stream);
  r->copy_threads = copy_threads;
  cudaGetDevice(&r->device);
  if (staging) {
    for (int i = 0; i < slots; ++i) r->staging.push_back(static_cast<char*>(staging[i]));
    r->staging_bytes = staging_bytes;
    r->stager = std::thread([r] { r->stager_loop(); });
  }
  *ring_out = r;
  return kOk;
}

extern "C" int cb_ring_destroy(void* ring) {
  delete as_ring(ring);
  return kOk;
}

extern "C" int cb_ring_begin(void* ring, int spans, const void* const* sources, const int64_t* bytes,
                             void* compute_stream, void* coordinator_stream, int profile) {
  Ring* r = as_ring(ring);
  CB_REQUIRE(r, "cb_ring_begin: null ring");
  CB_REQUIRE(!r->active, "cb_ring_begin: the previous pass has not ended");
  CB_REQUIRE(spans >= 1 && sources && bytes, "cb_ring_begin: need at least one span");
  for (int i = 0; i < spans; ++i) {
    CB_REQUIRE(sources[i], "cb_ring_begin: source of span %d is null", i);
    CB_REQUIRE(bytes[i] > 0 && bytes[i] <= r->slot_bytes, "cb_ring_begin: span %d has %lld bytes (slot %lld)", i,
               (long long)bytes[i], (long long)r->slot_bytes);
    CB_REQUIRE(r->staging.empty() || bytes[i] <= r->staging_bytes,
               "cb_ring_begin: span %d exceeds the staging buffers", i);
  }
  int rc = r->grow_events(spans);
  if (rc != kOk) return rc;
  r->n = spans;
  r->src.assign(reinterpret_cast<const char* const*>(sources), reinterpret_cast<const char* const*>(sources) + spans);
  r->bytes.assign(bytes, bytes + spans);
  r->compute = static_cast<cudaStream_t>(compute_stream);
  r->coordinator = static_cast<cudaStream_t>(coordinator_stream);
  r->profile = profile != 0;
  r->moved = 0;
  for (int i = 0; i < spans; ++i) r->moved += bytes[i];
  r->source_wait_ms = 0.0;
  {
    std::lock_guard<std::mutex> lock(r->mu);
    r->issued.assign(spans, 0);
    r->stage_ms.clear();
    r->failure.clear();
    r->skip = false;
  }
  // both streams start after the work the caller has queued so far
  cudaError_t e = cudaEventRecord(r->pass0, r->coordinator);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(r->copy, r->pass0, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(r->compute, r->pass0, 0);
  if (e != cudaSuccess) return fail(kErrCuda, "cb_ring_begin: %s", cudaGetErrorString(e));
  r->active = true;
  for (int u = 0; u < spans && u < r->nslots; ++u) {
    rc = r->start(u);
    if (rc != kOk) return rc;
  }
  return kOk;
}

extern "C" int cb_ring_acquire(void* ring, int span, void** device_ptr) {
  Ring* r = as_ring(ring);
  CB_REQUIRE(r && r->active && device_ptr, "cb_ring_acquire: no active pass");
  CB_REQUIRE(span >= 0 && span < r->n, "cb_ring_acquire: span %d of %d", span, r->n);
  const Clock::time_point t0 = Clock::now();
  std::string failure;
  {
    std::unique_lock<std::mutex> lock(r->mu);
    r->cv.wait(lock, [r, span] { return r->issued[span] != 0; });
    failure = r->failure;
  }
  r->source_wait_ms += ms_since(t0);
  if (!failure.empty()) return fail(kErrCuda, "%s", failure.c_str());
  cudaError_t e = cudaStreamWaitEvent(r->compute, r->ready[span], 0);
  if (e == cudaSuccess && r->profile) e = cudaEventRecord(r->comp0[span], r->compute);
  if (e != cudaSuccess) return fail(kErrCuda, "cb_ring_acquire: %s", cudaGetErrorString(e));
  *device_ptr = r->dslots[span % r->nslots];
  return kOk;
}

extern "C" int cb_ring_release(void* ring, int span) {
  Ring* r = as_ring(ring);
  CB_REQUIRE(r && r->active, "cb_ring_release: no active pass");
  CB_REQUIRE(span >= 0 && span < r->n, "cb_ring_release: span %d of %d", span, r->n);
  cudaError_t e = cudaSuccess;
  if (r->profile) e = cudaEventRecord(r->comp1[span], r->compute);
  if (e == cudaSuccess) e = cudaEventRecord(r->freed[span], r->compute);
  if (e != cudaSuccess) return fail(kErrCuda, "cb_ring_release: %s", cudaGetErrorString(e));
  const int next = span + r->nslots;
  return next < r->n ? r->start(next) : kOk;
}

// stats[0..7]: gpu_pipeline_ms, h2d_event_sum_ms, compute_event_sum_ms,
// source_wait_ms, staging copies, staging ms sum, staging ms max, bytes moved.
// Timing entries are 0 unless the pass was begun with profile = 1.
extern "C" int cb_ring_end(void* ring, int last_span, double* stats) {
  Ring* r = as_ring(ring);
  CB_REQUIRE(r && r->active, "cb_ring_end: no active pass");
  CB_REQUIRE(last_span >= 0 && last_span < r->n, "cb_ring_end: span %d of %d", last_span, r->n);
  cudaError_t e = cudaStreamWaitEvent(r->coordinator, r->freed[last_span], 0);
  if (e == cudaSuccess && r->profile) e = cudaEventRecord(r->pass1, r->coordinator);
  if (e == cudaSuccess) e = cudaStreamSynchronize(r->coordinator);
  r->active = false;
  if (e != cudaSuccess) return fail(kErrCuda, "cb_ring_end: %s", cudaGetErrorString(e));
  double pipe = 0, h2d = 0, comp = 0;
  if (r->profile) {
    float ms = 0;
    if (cudaEventElapsedTime(&ms, r->pass0, r->pass1) == cudaSuccess) pipe = ms;
    for (int u = 0; u < r->n; ++u) {
      if (cudaEventElapsedTime(&ms, r->copy0[u], r->copy1[u]) == cudaSuccess) h2d += ms;
      if (cudaEventElapsedTime(&ms, r->comp0[u], r->comp1[u]) == cudaSuccess) comp += ms;
    }
  }
  double sum = 0, mx = 0;
  size_t count = 0;
  {
    std::lock_guard<std::mutex> lock(r->mu);
    count = r->stage_ms.size();
    for (double v : r->stage_ms) {
      sum += v;
      mx = v > mx ? v : mx;
    }
  }
  if (stats) {
    stats[0] = pipe;
    stats[1] = h2d;
    stats[2] = comp;
    stats[3] = r->source_wait_ms;
    stats[4] = double(count);
    stats[5] = sum;
    stats[6] = mx;
    stats[7] = double(r->moved);
  }
  return kOk;
}

// Ends a pass that stopped early (the compute callback raised): queued
// staging jobs are dropped, every copy already started is waited for, and
// the ring is ready for the next pass.
extern "C" int cb_ring_abort(void* ring) {
  Ring* r = as_ring(ring);
  CB_REQUIRE(r, "cb_ring_abort: null ring");
  if (!r->active) return kOk;
  {
    // drop the queued jobs; a job already running finishes and issues its copy
    std::unique_lock<std::mutex> lock(r->mu);
    r->skip = true;
    r->cv.notify_all();
    r->cv.wait(lock, [r] { return r->jobs.empty() && !r->running; });
  }
  cudaError_t e = cudaStreamSynchronize(r->copy);
  if (e == cudaSuccess) e = cudaStreamSynchronize(r->compute);
  r->active = false;
  if (e != cudaSuccess) return fail(kErrCuda, "cb_ring_abort: %s", cudaGetErrorString(e));
  return kOk;
}
