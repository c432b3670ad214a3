#include "transfer/transfer.h"

#include <cuda_runtime.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <thread>

namespace lakeb {

namespace {
[[noreturn]] void fail(const std::string& m) { throw std::runtime_error(m); }

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(std::string(what) + ": " + cudaGetErrorString(e));
}

struct DeviceGuard {  // restores the calling thread's current device
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (dev >= 0 && cudaGetDevice(&prev) == cudaSuccess && prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};
}  // namespace

TransferEngine::TransferEngine(std::string node_id) : node_id_(std::move(node_id)) {}

TransferEngine::~TransferEngine() {
  std::vector<uint64_t> b, s;
  {
    std::lock_guard<std::mutex> g(mu_);
    for (auto& kv : batches_) b.push_back(kv.first);
    for (auto& kv : segs_) s.push_back(kv.first);
  }
  for (auto id : b) {
    try {
      wait_batch(id, 5000);
      free_batch_id(id);
    } catch (...) {
    }
  }
  for (auto id : s) {
    try {
      free_segment(id);
    } catch (...) {
    }
  }
}

uint64_t TransferEngine::open_segment(const std::string& name, uint64_t capacity, int kind, int device) {
  if (capacity == 0) fail("open_segment: capacity must be > 0");
  Segment s;
  s.name = name;
  s.capacity = capacity;
  s.kind = kind;
  s.owned = true;
  void* p = nullptr;
  if (kind == SEG_HOST) {
    p = std::aligned_alloc(256, (capacity + 255) / 256 * 256);
    if (!p) fail("open_segment: out of host memory");
    std::memset(p, 0, capacity);
  } else if (kind == SEG_PINNED) {
    cuda_check(cudaHostAlloc(&p, capacity, cudaHostAllocPortable), "cudaHostAlloc");
    std::memset(p, 0, capacity);
  } else if (kind == SEG_DEVICE) {
    if (device < 0) fail("open_segment: device segment needs a device ordinal");
    DeviceGuard dg(device);
    cuda_check(cudaMalloc(&p, capacity), "cudaMalloc");
    cuda_check(cudaMemset(p, 0, capacity), "cudaMemset");
    s.device = device;
  } else {
    fail("open_segment: unknown segment kind");
  }
  s.base = static_cast<uint8_t*>(p);
  std::lock_guard<std::mutex> g(mu_);
  uint64_t id = next_seg_++;
  segs_[id] = s;
  return id;
}

uint64_t TransferEngine::register_segment(const std::string& name, uintptr_t ptr, uint64_t capacity, int device) {
  if (!ptr || !capacity) fail("register_segment: null range");
  Segment s;
  s.name = name;
  s.base = reinterpret_cast<uint8_t*>(ptr);
  s.capacity = capacity;
  s.kind = SEG_EXTERNAL;
  s.device = device;
  s.owned = false;
  std::lock_guard<std::mutex> g(mu_);
  uint64_t id = next_seg_++;
  segs_[id] = s;
  return id;
}

// [offset, offset + length) inside a segment of `capacity` bytes, without the sum wrapping
static bool in_range(uint64_t offset, uint64_t length, uint64_t capacity) {
  return length <= capacity && offset <= capacity - length;
}

void TransferEngine::free_segment(uint64_t id) {
  Segment s;
  {
    std::lock_guard<std::mutex> g(mu_);
    auto it = segs_.find(id);
    if (it == segs_.end()) fail("unknown segment " + std::to_string(id));
    s = it->second;
    segs_.erase(it);
  }
  if (!s.owned) return;
  if (s.kind == SEG_HOST) {
    std::free(s.base);
  } else if (s.kind == SEG_PINNED) {
    cudaFreeHost(s.base);
  } else if (s.kind == SEG_DEVICE) {
    DeviceGuard dg(s.device);
    cudaFree(s.base);
  }
}

const Segment& TransferEngine::seg(uint64_t id) const {
  auto it = segs_.find(id);
  if (it == segs_.end()) fail("unknown segment " + std::to_string(id));
  return it->second;
}

uintptr_t TransferEngine::segment_ptr(uint64_t id) const {
  std::lock_guard<std::mutex> g(mu_);
  return reinterpret_cast<uintptr_t>(seg(id).base);
}

void TransferEngine::write_segment(uint64_t id, uint64_t offset, const std::string& data) {
  Segment s;
  {
    std::lock_guard<std::mutex> g(mu_);
    s = seg(id);
  }
  if (!in_range(offset, data.size(), s.capacity)) fail("write_segment: out of range");
  if (s.device >= 0) {
    DeviceGuard dg(s.device);
    cuda_check(cudaMemcpy(s.base + offset, data.data(), data.size(), cudaMemcpyHostToDevice), "cudaMemcpy");
  } else {
    std::memcpy(s.base + offset, data.data(), data.size());
  }
}

std::string TransferEngine::read_segment(uint64_t id, uint64_t offset, uint64_t length) {
  Segment s;
  {
    std::lock_guard<std::mutex> g(mu_);
    s = seg(id);
  }
  if (!in_range(offset, length, s.capacity)) fail("read_segment: out of range");
  std::string out(length, '\0');
  if (s.device >= 0) {
    DeviceGuard dg(s.device);
    cuda_check(cudaMemcpy(out.data(), s.base + offset, length, cudaMemcpyDeviceToHost), "cudaMemcpy");
  } else {
    std::memcpy(out.data(), s.base + offset, length);
  }
  return out;
}

uint64_t TransferEngine::allocate_batch_id(size_t batch_size) {
  if (batch_size == 0) fail("allocate_batch_id: empty batch");
  std::lock_guard<std::mutex> g(mu_);
  uint64_t id = next_batch_++;
  batches_[id].capacity = batch_size;
  return id;
}

void TransferEngine::submit_transfer(uint64_t batch_id, const std::vector<TransferOp>& ops) {
  if (ops.empty()) fail("submit_transfer: empty batch");
  std::lock_guard<std::mutex> g(mu_);
  auto bit = batches_.find(batch_id);
  if (bit == batches_.end()) fail("unknown batch " + std::to_string(batch_id));
  Batch& b = bit->second;
  if (b.tasks.size() + ops.size() > b.capacity) fail("submit_transfer: batch capacity exceeded");
  // validate everything first: a rejected batch moves no byte
  for (auto& op : ops) {
    if (op.src_tier < 1 || op.src_tier > 3) fail("invalid source tier " + std::to_string(op.src_tier));
    const Segment& s = seg(op.src_segment);
    const Segment& d = seg(op.dst_segment);
    if (!in_range(op.src_offset, op.length, s.capacity)) fail("submit_transfer: source range out of segment");
    if (!in_range(op.dst_offset, op.length, d.capacity)) fail("submit_transfer: target range out of segment");
  }
  for (auto& op : ops) {
    const Segment& s = seg(op.src_segment);
    const Segment& d = seg(op.dst_segment);
    Task t;
    t.bytes = op.length;
    if (s.device < 0 && d.device < 0) {
      std::memcpy(d.base + op.dst_offset, s.base + op.src_offset, op.length);
      t.state = TASK_DONE;
    } else {
      int dev = d.device >= 0 ? d.device : s.device;
      DeviceGuard dg(dev);
      if (!b.stream) {
        cudaStream_t st;
        cuda_check(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "cudaStreamCreate");
        b.stream = st;
        b.device = dev;
      }
      auto st = static_cast<cudaStream_t>(b.stream);
      cuda_check(cudaMemcpyAsync(d.base + op.dst_offset, s.base + op.src_offset, op.length, cudaMemcpyDefault, st),
                 "cudaMemcpyAsync");
      cudaEvent_t ev;
      cuda_check(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "cudaEventCreate");
      cuda_check(cudaEventRecord(ev, st), "cudaEventRecord");
      t.event = ev;
      t.state = TASK_IN_FLIGHT;
    }
    bytes_moved_ += op.length;
    b.tasks.push_back(t);
  }
}

void TransferEngine::poll(Task& t) {
  if (t.state != TASK_IN_FLIGHT || !t.event) return;
  cudaError_t e = cudaEventQuery(static_cast<cudaEvent_t>(t.event));
  if (e == cudaSuccess) {
    t.state = TASK_DONE;
  } else if (e != cudaErrorNotReady) {
    t.state = TASK_FAILED;
  }
}

TaskStatus TransferEngine::get_transfer_status(uint64_t batch_id, uint64_t task_id) {
  std::lock_guard<std::mutex> g(mu_);
  auto bit = batches_.find(batch_id);
  if (bit == batches_.end()) fail("unknown batch " + std::to_string(batch_id));
  auto& tasks = bit->second.tasks;
  if (task_id >= tasks.size()) {
    if (task_id < bit->second.capacity) return TaskStatus{TASK_PENDING, 0};
    fail("unknown task " + std::to_string(task_id));
  }
  poll(tasks[task_id]);
  auto& t = tasks[task_id];
  return TaskStatus{t.state, t.state == TASK_DONE ? t.bytes : 0};
}

bool TransferEngine::wait_batch(uint64_t batch_id, uint64_t timeout_ms) {
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    {
      std::lock_guard<std::mutex> g(mu_);
      auto bit = batches_.find(batch_id);
      if (bit == batches_.end()) fail("unknown batch " + std::to_string(batch_id));
      bool all = true;
      for (auto& t : bit->second.tasks) {
        poll(t);
        if (t.state == TASK_IN_FLIGHT || t.state == TASK_PENDING) all = false;
      }
      if (all) return true;
    }
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (uint64_t(ms) >= timeout_ms) return false;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

void TransferEngine::free_batch_id(uint64_t batch_id) {
  Batch b;
  {
    std::lock_guard<std::mutex> g(mu_);
    auto bit = batches_.find(batch_id);
    if (bit == batches_.end()) fail("unknown batch " + std::to_string(batch_id));
    b = std::move(bit->second);
    batches_.erase(bit);
  }
  DeviceGuard dg(b.device);
  if (b.stream) cudaStreamSynchronize(static_cast<cudaStream_t>(b.stream));  // copies must not outlive the ids
  for (auto& t : b.tasks)
    if (t.event) cudaEventDestroy(static_cast<cudaEvent_t>(t.event));
  if (b.stream) cudaStreamDestroy(static_cast<cudaStream_t>(b.stream));
}

size_t TransferEngine::segment_count() const {
  std::lock_guard<std::mutex> g(mu_);
  return segs_.size();
}
size_t TransferEngine::batch_count() const {
  std::lock_guard<std::mutex> g(mu_);
  return batches_.size();
}

// ------------------------------------------------------------------ byte store
std::string ByteStore::key(const std::string& model_id, const std::string& revision, int pool_kind,
                           const std::string& block_hash) {
  std::string k;
  k.reserve(model_id.size() + revision.size() + block_hash.size() + 8);
  k += model_id;
  k.push_back('\0');
  k += revision;
  k.push_back('\0');
  k += std::to_string(pool_kind);
  k.push_back('\0');
  k += block_hash;
  return k;
}

void ByteStore::put(const std::string& key, std::string data) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = map_.find(key);
  if (it != map_.end()) {
    used_ -= it->second.data.size();
    lru_.erase(it->second.lru);
    map_.erase(it);
  }
  used_ += data.size();
  lru_.push_front(key);
  map_[key] = Item{std::move(data), lru_.begin()};
  while (cap_ > 0 && used_ > cap_ && lru_.size() > 1) {
    auto& victim = lru_.back();
    auto v = map_.find(victim);
    used_ -= v->second.data.size();
    map_.erase(v);
    lru_.pop_back();
    evictions_++;
  }
}

bool ByteStore::get(const std::string& key, std::string* out) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = map_.find(key);
  if (it == map_.end()) return false;
  lru_.splice(lru_.begin(), lru_, it->second.lru);
  *out = it->second.data;
  return true;
}

bool ByteStore::contains(const std::string& key) const {
  std::lock_guard<std::mutex> g(mu_);
  return map_.count(key) != 0;
}

bool ByteStore::erase(const std::string& key) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = map_.find(key);
  if (it == map_.end()) return false;
  used_ -= it->second.data.size();
  lru_.erase(it->second.lru);
  map_.erase(it);
  return true;
}

size_t ByteStore::size() const {
  std::lock_guard<std::mutex> g(mu_);
  return map_.size();
}
uint64_t ByteStore::bytes() const {
  std::lock_guard<std::mutex> g(mu_);
  return used_;
}

}  // namespace lakeb
