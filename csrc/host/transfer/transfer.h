// Batch transfer engine over registered memory segments, and the
// content-addressed byte store behind Pull and the TCP data service.
//
// A segment is a byte range this process can address: host memory it owns
// (pageable or pinned), device memory it owns, or an external range it was
// given (a KV arena, or a peer GPU's arena mapped through CUDA IPC - inside
// one NVSwitch box every peer's memory is one cudaMemcpyAsync away).
//
// Lifecycle (same shape as a Mooncake-style transport):
//   open_segment / register_segment -> allocate_batch_id(n)
//   -> submit_transfer(batch, ops) -> get_transfer_status(batch, task)
//   -> free_batch_id(batch)
// Host-to-host ops complete inline (memcpy). Ops touching device memory are
// one cudaMemcpyAsync each on the batch's own non-blocking stream, followed by
// an event per task; the status is the event's state.
//
// Reference parity: rust/transfer/src/transport.rs:31-68 (Transport trait),
// tcp.rs (in-process segment copies), location.rs:9-18 (tier check: sources
// live in L0/L1/L2 only), bytes.rs:1-53 (byte store), kv-pool/src/lib.rs.
#pragma once

#include <cstdint>
#include <list>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

namespace lakeb {

enum SegKind : int { SEG_HOST = 0, SEG_PINNED = 1, SEG_DEVICE = 2, SEG_EXTERNAL = 3 };
enum TaskState : int { TASK_PENDING = 0, TASK_IN_FLIGHT = 1, TASK_DONE = 2, TASK_FAILED = 3 };

struct Segment {
  std::string name;
  uint8_t* base = nullptr;
  uint64_t capacity = 0;
  int kind = SEG_HOST;
  int device = -1;  // >= 0: device memory of that ordinal
  bool owned = false;
};

struct TransferOp {
  int src_tier = 0;
  std::string src_node;
  uint64_t src_segment = 0;
  uint64_t src_offset = 0;
  uint64_t dst_segment = 0;
  uint64_t dst_offset = 0;
  uint64_t length = 0;
};

struct TaskStatus {
  int state = TASK_PENDING;
  uint64_t bytes_done = 0;
};

class TransferEngine {
 public:
  explicit TransferEngine(std::string node_id = "node-0");
  ~TransferEngine();
  TransferEngine(const TransferEngine&) = delete;
  TransferEngine& operator=(const TransferEngine&) = delete;

  const std::string& node_id() const { return node_id_; }
  // kind SEG_HOST / SEG_PINNED / SEG_DEVICE; device is the ordinal for SEG_DEVICE
  uint64_t open_segment(const std::string& name, uint64_t capacity, int kind = SEG_HOST, int device = -1);
  // external memory: host (device = -1) or device / peer-mapped device memory (device >= 0)
  uint64_t register_segment(const std::string& name, uintptr_t ptr, uint64_t capacity, int device = -1);
  void free_segment(uint64_t id);
  void write_segment(uint64_t id, uint64_t offset, const std::string& data);
  std::string read_segment(uint64_t id, uint64_t offset, uint64_t length);
  uintptr_t segment_ptr(uint64_t id) const;

  uint64_t allocate_batch_id(size_t batch_size);
  void submit_transfer(uint64_t batch_id, const std::vector<TransferOp>& ops);
  TaskStatus get_transfer_status(uint64_t batch_id, uint64_t task_id);
  // true when every task of the batch finished within timeout_ms
  bool wait_batch(uint64_t batch_id, uint64_t timeout_ms);
  void free_batch_id(uint64_t batch_id);

  size_t segment_count() const;
  size_t batch_count() const;
  uint64_t bytes_moved() const { return bytes_moved_; }

 private:
  struct Task {
    int state = TASK_PENDING;
    uint64_t bytes = 0;
    void* event = nullptr;  // cudaEvent_t when the copy went to a stream
  };
  struct Batch {
    size_t capacity = 0;
    std::vector<Task> tasks;
    void* stream = nullptr;  // cudaStream_t, created on first device op
    int device = -1;
  };
  const Segment& seg(uint64_t id) const;
  void poll(Task& t);

  std::string node_id_;
  mutable std::mutex mu_;
  std::unordered_map<uint64_t, Segment> segs_;
  std::unordered_map<uint64_t, Batch> batches_;
  uint64_t next_seg_ = 1, next_batch_ = 1;
  uint64_t bytes_moved_ = 0;
};

// (model_id, revision, pool_kind, block_hash) -> bytes. capacity_bytes > 0
// bounds the store; the least recently used blocks are dropped first.
class ByteStore {
 public:
  explicit ByteStore(uint64_t capacity_bytes = 0) : cap_(capacity_bytes) {}
  static std::string key(const std::string& model_id, const std::string& revision, int pool_kind,
                         const std::string& block_hash);
  void put(const std::string& key, std::string data);
  bool get(const std::string& key, std::string* out);
  bool contains(const std::string& key) const;
  bool erase(const std::string& key);
  size_t size() const;
  uint64_t bytes() const;
  uint64_t evictions() const { return evictions_; }

 private:
  struct Item {
    std::string data;
    std::list<std::string>::iterator lru;
  };
  mutable std::mutex mu_;
  uint64_t cap_, used_ = 0, evictions_ = 0;
  std::unordered_map<std::string, Item> map_;
  std::list<std::string> lru_;  // front = most recent
};

}  // namespace lakeb
