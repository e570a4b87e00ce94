// memory_manager.cpp — native weight/activation transfer engine behind the C ABI.
//
// Same responsibilities and method set as the reference's LemaMemoryManager
// (src/lema/_csrc/memory_manager.h:25-92, .cpp:9-199): registered pinned RAM
// buffers and VRAM slots, host memcpy packing, H2D copies on a dedicated copy
// stream tracked by a ring of 1024 events, and a 2-thread prefetch job pool.
// Differences, all additive:
//   * buffers are registered as (pointer, bytes); the Python side owns memory;
//   * every copy into a VRAM slot first waits (on the device) for the slot's
//     "free" event, recorded by the compute stream when it stops reading the
//     slot — the cross-stream write-after-read the reference leaves open;
//   * compute streams can wait for a transfer on the device
//     (lema_mm_stream_wait_transfer) instead of blocking the host;
//   * bounded waits (…_timeout) return LEMA_ERR_TIMEOUT instead of spinning;
//   * an aligned pack lays int8 weight segments out on 128-byte boundaries.
#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <memory>
#include <mutex>
#include <queue>
#include <thread>
#include <unordered_map>
#include <vector>

#include "internal.h"

namespace {

constexpr int64_t kMaxEvents = 1024;
constexpr int64_t kStreamingOffset = 1000;

struct Buf {
  void* ptr = nullptr;
  size_t bytes = 0;
};

struct Job {
  lema_job_fn fn = nullptr;
  void* user = nullptr;
  std::shared_ptr<std::atomic<bool>> done;
};

}  // namespace

struct lema_mm {
  int64_t num_layers_hint = 0;
  int64_t max_layer_size = 0;
  int device = 0;
  cudaStream_t h2d = nullptr;
  std::vector<cudaEvent_t> events;
  std::atomic<int64_t> next_event{0};

  std::mutex buf_mu;
  std::unordered_map<int64_t, Buf> ram;
  std::vector<Buf> vram;
  std::vector<cudaEvent_t> slot_free;
  std::vector<bool> slot_free_recorded;

  std::unique_ptr<std::atomic<bool>[]> in_ram;
  int64_t in_ram_size = 0;

  std::vector<std::thread> workers;
  std::queue<Job> jobs;
  std::mutex q_mu;
  std::condition_variable cv;
  std::atomic<bool> stop{false};
  std::mutex st_mu;
  std::unordered_map<int64_t, std::shared_ptr<std::atomic<bool>>> status;
  std::atomic<int64_t> next_job{1};

  int64_t status_index(int64_t layer_id) const {
    return layer_id >= kStreamingOffset ? layer_id - kStreamingOffset + num_layers_hint
                                        : layer_id;
  }
  void mark_in_ram(int64_t layer_id) {
    const int64_t i = status_index(layer_id);
    if (i >= 0 && i < in_ram_size) in_ram[i].store(true, std::memory_order_release);
  }

  void worker_loop() {
    while (true) {
      Job job;
      {
        std::unique_lock<std::mutex> lk(q_mu);
        cv.wait(lk, [this] { return stop.load() || !jobs.empty(); });
        if (stop.load() && jobs.empty()) return;
        job = std::move(jobs.front());
        jobs.pop();
      }
      if (job.fn) job.fn(job.user);
      job.done->store(true, std::memory_order_release);
    }
  }
};

using lema::set_error;

namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    int cur = -1;
    if (dev >= 0 && cudaGetDevice(&cur) == cudaSuccess) {
      prev = cur;
      if (cur != dev) cudaSetDevice(dev);
    }
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

cudaEvent_t event_for(lema_mm* mm, int64_t id) {
  if (id < 0 || id >= static_cast<int64_t>(mm->events.size())) return nullptr;
  return mm->events[static_cast<size_t>(id)];
}

int pack_impl(lema_mm* mm, int64_t layer_id, const void* const* srcs, const size_t* sizes,
              int64_t n, size_t align, size_t* offsets_out) {
  lema::clear_error();
  if (!mm) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null manager");
  if (n < 0 || (n > 0 && (!srcs || !sizes)))
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "bad tensor list");
  Buf dst;
  {
    std::lock_guard<std::mutex> lk(mm->buf_mu);
    auto it = mm->ram.find(layer_id);
    if (it == mm->ram.end())
      return set_error(LEMA_ERR_NOT_REGISTERED,
                       "RAM buffer not registered for layer " + std::to_string(layer_id));
    dst = it->second;
  }
  if (!dst.ptr)
    return set_error(LEMA_ERR_NOT_REGISTERED,
                     "RAM buffer not defined for layer " + std::to_string(layer_id));
  size_t off = 0;
  for (int64_t i = 0; i < n; ++i) {
    if (align > 1) off = (off + align - 1) / align * align;
    if (off + sizes[i] > dst.bytes)
      return set_error(LEMA_ERR_OVERFLOW, "Pack overflow for layer " + std::to_string(layer_id));
    if (sizes[i]) std::memcpy(static_cast<char*>(dst.ptr) + off, srcs[i], sizes[i]);
    if (offsets_out) offsets_out[i] = off;
    off += sizes[i];
  }
  mm->mark_in_ram(layer_id);
  return LEMA_OK;
}

}  // namespace

extern "C" int lema_mm_create(int64_t num_layers_hint, int64_t max_layer_size, int32_t device,
                              lema_mm** out) {
  lema::clear_error();
  if (!out || num_layers_hint < 0) return set_error(LEMA_ERR_INVALID_ARGUMENT, "bad arguments");
  std::unique_ptr<lema_mm> mm(new lema_mm());
  mm->num_layers_hint = num_layers_hint;
  mm->max_layer_size = max_layer_size;
  mm->device = device;
  if (device >= 0) {  // device < 0: host-only manager (packing and jobs, no transfers)
    DeviceGuard g(device);
    LEMA_CUDA_TRY(cudaStreamCreateWithFlags(&mm->h2d, cudaStreamNonBlocking));
    mm->events.resize(kMaxEvents, nullptr);
    for (auto& e : mm->events) LEMA_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  mm->in_ram_size = num_layers_hint + 2;
  mm->in_ram.reset(new std::atomic<bool>[static_cast<size_t>(mm->in_ram_size)]);
  for (int64_t i = 0; i < mm->in_ram_size; ++i) mm->in_ram[i].store(false);
  const unsigned hw = std::thread::hardware_concurrency();
  const int nworkers = static_cast<int>(std::min<unsigned>(2u, hw ? hw : 2u));
  lema_mm* raw = mm.get();
  for (int i = 0; i < nworkers; ++i) mm->workers.emplace_back([raw] { raw->worker_loop(); });
  *out = mm.release();
  return LEMA_OK;
}

extern "C" int lema_mm_destroy(lema_mm* mm) {
  lema::clear_error();
  if (!mm) return LEMA_OK;
  mm->stop.store(true);
  mm->cv.notify_all();
  for (auto& w : mm->workers)
    if (w.joinable()) w.join();
  if (mm->device >= 0) {
    DeviceGuard g(mm->device);
    if (mm->h2d) cudaStreamSynchronize(mm->h2d);
    for (auto e : mm->events)
      if (e) cudaEventDestroy(e);
    for (auto e : mm->slot_free)
      if (e) cudaEventDestroy(e);
    if (mm->h2d) cudaStreamDestroy(mm->h2d);
  }
  delete mm;
  return LEMA_OK;
}

extern "C" int lema_mm_register_ram_buffer(lema_mm* mm, int64_t layer_id, void* host_ptr,
                                           size_t bytes) {
  lema::clear_error();
  if (!mm) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null manager");
  {
    std::lock_guard<std::mutex> lk(mm->buf_mu);
    mm->ram[layer_id] = Buf{host_ptr, bytes};
  }
  mm->mark_in_ram(layer_id);
  return LEMA_OK;
}

extern "C" int lema_mm_register_vram_slot(lema_mm* mm, int64_t slot, void* dev_ptr, size_t bytes) {
  lema::clear_error();
  if (!mm || slot < 0) return set_error(LEMA_ERR_INVALID_ARGUMENT, "bad manager or slot");
  std::lock_guard<std::mutex> lk(mm->buf_mu);
  if (slot >= static_cast<int64_t>(mm->vram.size())) {
    mm->vram.resize(static_cast<size_t>(slot) + 1);
    mm->slot_free.resize(static_cast<size_t>(slot) + 1, nullptr);
    mm->slot_free_recorded.resize(static_cast<size_t>(slot) + 1, false);
  }
  mm->vram[static_cast<size_t>(slot)] = Buf{dev_ptr, bytes};
  if (!mm->slot_free[static_cast<size_t>(slot)] && mm->device >= 0) {
    DeviceGuard g(mm->device);
    LEMA_CUDA_TRY(
        cudaEventCreateWithFlags(&mm->slot_free[static_cast<size_t>(slot)], cudaEventDisableTiming));
  }
  mm->slot_free_recorded[static_cast<size_t>(slot)] = false;
  return LEMA_OK;
}

extern "C" int lema_mm_pack_layer_to_ram(lema_mm* mm, int64_t layer_id, const void* const* srcs,
                                         const size_t* sizes, int64_t n) {
  return pack_impl(mm, layer_id, srcs, sizes, n, 1, nullptr);
}

extern "C" int lema_mm_pack_layer_to_ram_aligned(lema_mm* mm, int64_t layer_id,
                                                 const void* const* srcs, const size_t* sizes,
                                                 int64_t n, size_t align, size_t* offsets_out) {
  if (align == 0 || (align & (align - 1)) != 0)
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "align must be a power of two");
  return pack_impl(mm, layer_id, srcs, sizes, n, align, offsets_out);
}

extern "C" int lema_mm_async_transfer_to_vram(lema_mm* mm, int64_t layer_id, int64_t vram_slot,
                                              size_t bytes, int64_t* event_id_out) {
  lema::clear_error();
  if (!mm || !event_id_out) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null argument");
  Buf src, dst;
  cudaEvent_t free_ev = nullptr;
  {
    std::lock_guard<std::mutex> lk(mm->buf_mu);
    auto it = mm->ram.find(layer_id);
    if (it == mm->ram.end())
      return set_error(LEMA_ERR_NOT_REGISTERED,
                       "Source RAM buffer not registered for layer " + std::to_string(layer_id));
    src = it->second;
    if (vram_slot < 0 || vram_slot >= static_cast<int64_t>(mm->vram.size()) ||
        !mm->vram[static_cast<size_t>(vram_slot)].ptr)
      return set_error(LEMA_ERR_NOT_REGISTERED, "Invalid VRAM slot: " + std::to_string(vram_slot));
    dst = mm->vram[static_cast<size_t>(vram_slot)];
    if (mm->slot_free_recorded[static_cast<size_t>(vram_slot)])
      free_ev = mm->slot_free[static_cast<size_t>(vram_slot)];
  }
  const size_t n = bytes ? bytes : src.bytes;
  if (n > src.bytes || n > dst.bytes)
    return set_error(LEMA_ERR_OVERFLOW, "transfer larger than the RAM buffer or VRAM slot");
  if (!mm->h2d) return set_error(LEMA_ERR_INVALID_ARGUMENT, "manager was created without a device");
  const int64_t id = mm->next_event.fetch_add(1) % kMaxEvents;
  DeviceGuard g(mm->device);
  if (free_ev) LEMA_CUDA_TRY(cudaStreamWaitEvent(mm->h2d, free_ev, 0));
  if (n) LEMA_CUDA_TRY(cudaMemcpyAsync(dst.ptr, src.ptr, n, cudaMemcpyHostToDevice, mm->h2d));
  LEMA_CUDA_TRY(cudaEventRecord(mm->events[static_cast<size_t>(id)], mm->h2d));
  *event_id_out = id;
  return LEMA_OK;
}

extern "C" int lema_mm_stream_wait_transfer(lema_mm* mm, int64_t event_id, void* stream) {
  lema::clear_error();
  if (!mm) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null manager");
  cudaEvent_t e = event_for(mm, event_id);
  if (!e) return LEMA_OK;  // invalid ids are no-ops, as in the reference
  LEMA_CUDA_TRY(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), e, 0));
  return LEMA_OK;
}

extern "C" int lema_mm_release_vram_slot(lema_mm* mm, int64_t vram_slot, void* stream) {
  lema::clear_error();
  if (!mm) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null manager");
  std::lock_guard<std::mutex> lk(mm->buf_mu);
  if (vram_slot < 0 || vram_slot >= static_cast<int64_t>(mm->vram.size()))
    return set_error(LEMA_ERR_NOT_REGISTERED, "Invalid VRAM slot: " + std::to_string(vram_slot));
  if (!mm->slot_free[static_cast<size_t>(vram_slot)])
    return set_error(LEMA_ERR_INVALID_ARGUMENT, "manager was created without a device");
  DeviceGuard g(mm->device);
  LEMA_CUDA_TRY(cudaEventRecord(mm->slot_free[static_cast<size_t>(vram_slot)],
                                static_cast<cudaStream_t>(stream)));
  mm->slot_free_recorded[static_cast<size_t>(vram_slot)] = true;
  return LEMA_OK;
}

extern "C" int lema_mm_wait_vram_transfer(lema_mm* mm, int64_t event_id) {
  lema::clear_error();
  if (!mm) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null manager");
  cudaEvent_t e = event_for(mm, event_id);
  if (!e) return LEMA_OK;
  LEMA_CUDA_TRY(cudaEventSynchronize(e));
  return LEMA_OK;
}

extern "C" int lema_mm_wait_vram_transfer_timeout(lema_mm* mm, int64_t event_id,
                                                  int64_t timeout_ms) {
  lema::clear_error();
  if (!mm) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null manager");
  cudaEvent_t e = event_for(mm, event_id);
  if (!e) return LEMA_OK;
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  while (true) {
    cudaError_t r = cudaEventQuery(e);
    if (r == cudaSuccess) return LEMA_OK;
    if (r != cudaErrorNotReady) return lema::cuda_check(r, "cudaEventQuery");
    if (std::chrono::steady_clock::now() >= deadline)
      return set_error(LEMA_ERR_TIMEOUT, "transfer " + std::to_string(event_id) +
                                             " not complete after " +
                                             std::to_string(timeout_ms) + " ms");
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

extern "C" int lema_mm_is_transfer_complete(lema_mm* mm, int64_t event_id, int32_t* done_out) {
  lema::clear_error();
  if (!mm || !done_out) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null argument");
  cudaEvent_t e = event_for(mm, event_id);
  if (!e) {
    *done_out = 1;
    return LEMA_OK;
  }
  cudaError_t r = cudaEventQuery(e);
  if (r != cudaSuccess && r != cudaErrorNotReady) return lema::cuda_check(r, "cudaEventQuery");
  *done_out = (r == cudaSuccess) ? 1 : 0;
  return LEMA_OK;
}

extern "C" int lema_mm_synchronize_all(lema_mm* mm) {
  lema::clear_error();
  if (!mm) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null manager");
  if (!mm->h2d) return LEMA_OK;
  LEMA_CUDA_TRY(cudaStreamSynchronize(mm->h2d));
  return LEMA_OK;
}

extern "C" int lema_mm_submit_prefetch_job(lema_mm* mm, lema_job_fn fn, void* user,
                                           int64_t* job_id_out) {
  lema::clear_error();
  if (!mm || !fn || !job_id_out) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null argument");
  auto done = std::make_shared<std::atomic<bool>>(false);
  const int64_t id = mm->next_job.fetch_add(1);
  {
    std::lock_guard<std::mutex> lk(mm->st_mu);
    mm->status[id] = done;
  }
  {
    std::lock_guard<std::mutex> lk(mm->q_mu);
    mm->jobs.push(Job{fn, user, done});
  }
  mm->cv.notify_one();
  *job_id_out = id;
  return LEMA_OK;
}

std::shared_ptr<std::atomic<bool>> job_flag(lema_mm* mm, int64_t id) {
  std::lock_guard<std::mutex> lk(mm->st_mu);
  auto it = mm->status.find(id);
  return it == mm->status.end() ? nullptr : it->second;
}

extern "C" int lema_mm_is_prefetch_complete(lema_mm* mm, int64_t job_id, int32_t* done_out) {
  lema::clear_error();
  if (!mm || !done_out) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null argument");
  auto f = job_flag(mm, job_id);
  *done_out = (!f || f->load(std::memory_order_acquire)) ? 1 : 0;
  return LEMA_OK;
}

extern "C" int lema_mm_wait_for_prefetch_timeout(lema_mm* mm, int64_t job_id,
                                                 int64_t timeout_ms) {
  lema::clear_error();
  if (!mm) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null manager");
  auto f = job_flag(mm, job_id);
  if (!f) return LEMA_OK;
  const bool bounded = timeout_ms >= 0;
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  while (!f->load(std::memory_order_acquire)) {
    if (bounded && std::chrono::steady_clock::now() >= deadline)
      return set_error(LEMA_ERR_TIMEOUT, "prefetch job " + std::to_string(job_id) +
                                             " not complete after " +
                                             std::to_string(timeout_ms) + " ms");
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  return LEMA_OK;
}

extern "C" int lema_mm_wait_for_prefetch(lema_mm* mm, int64_t job_id) {
  return lema_mm_wait_for_prefetch_timeout(mm, job_id, -1);
}

extern "C" int lema_mm_is_layer_in_ram(lema_mm* mm, int64_t layer_id, int32_t* out) {
  lema::clear_error();
  if (!mm || !out) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null argument");
  const int64_t i = mm->status_index(layer_id);
  *out = (i >= 0 && i < mm->in_ram_size && mm->in_ram[i].load(std::memory_order_acquire)) ? 1 : 0;
  return LEMA_OK;
}

extern "C" int lema_mm_copy_stream(lema_mm* mm, void** stream_out) {
  lema::clear_error();
  if (!mm || !stream_out) return set_error(LEMA_ERR_INVALID_ARGUMENT, "null argument");
  *stream_out = mm->h2d;
  return LEMA_OK;
}
