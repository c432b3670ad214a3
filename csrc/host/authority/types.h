// Control-plane value types. Field names and enum values follow the wire
// schema (proto/schema.proto and proto/lake.proto of the reference, mirrored
// by lake_b200/api/protos/*.proto) so the gRPC layer maps them one to one.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace lakeb::cp {

enum Tier : int { TIER_UNSPECIFIED = 0, L0 = 1, L1 = 2, L2 = 3, L3 = 4 };
enum PoolKind : int { POOL_UNSPECIFIED = 0, TARGET = 1, DRAFT = 2 };
enum BlockKind : int { KIND_UNSPECIFIED = 0, T_TYPE = 1, R_TYPE_STATE = 2, R_TYPE_TRAILING = 3 };
enum RefKind : int { REF_KIND_UNSPECIFIED = 0, REQUEST = 1, IN_FLIGHT = 2, WRITEBACK = 3 };
enum EventKind : int { REGISTERED = 0, INVALIDATED = 1, MOVED = 2 };
enum DefragMode : int { DEFRAG_MODE_UNSPECIFIED = 0, COMPACT = 1, COLOCATE = 2, BOTH = 3 };

struct KVBlockID {
  std::string model_id;
  std::string block_hash;  // raw bytes
  int pool_kind = TARGET;
  std::string scope = "public";
  std::string revision;
};

struct Location {
  int tier = TIER_UNSPECIFIED;
  std::string node_id;
  uint64_t segment_id = 0;
  uint64_t offset = 0;
};

struct BlockMeta {
  KVBlockID id;
  int block_kind = T_TYPE;
  std::vector<Location> locations;
  bool l3_present = false;
  uint32_t ref_count = 0;
};

struct Quota {
  int64_t soft_bytes = 0;
  int64_t hard_bytes = 0;
  bool borrow_enabled = false;
};

struct BackpressureSignal {
  std::string model_id, revision;
  int64_t used_bytes = 0, soft_bytes = 0, hard_bytes = 0, deficit_bytes = 0;
  std::string reason;  // HARD_QUOTA | POOL_CAPACITY
};

struct ModelDescriptor {
  std::string model_id, revision;
  uint32_t num_layers = 0;
  uint32_t block_tokens = 16;
  uint64_t bytes_per_block = 0;
  int hash_algo = 1;
  Quota quota;
};

struct ViewEvent {
  int kind = REGISTERED;
  KVBlockID id;
  std::vector<Location> locations;
  bool l3_present = false;
  int block_kind = 0;
};

struct ViewUpdate {
  uint64_t seq = 0;
  std::vector<ViewEvent> events;
};

struct ReusableBlock {
  KVBlockID id;
  BlockMeta meta;
  bool local_hit = false;
};

struct LookupResult {
  std::vector<ReusableBlock> blocks;
  uint32_t hit_length = 0;
  bool all_local_hit = false;
};

struct RefDelta {
  KVBlockID id;
  int kind = REQUEST;
  int32_t delta = 0;
  std::string node_id;
};

struct RegisterResult {
  bool accepted = true;
  BackpressureSignal backpressure;
};

struct OrphanReport {
  std::string node_id;
  std::vector<KVBlockID> ids;
  uint64_t marked_at_ms = 0;
};

struct CheckpointBlock {
  BlockMeta meta;
  std::vector<std::string> prefix_chain;
};

struct CheckpointSnapshot {
  uint64_t seq = 0;
  std::vector<ModelDescriptor> models;
  std::vector<CheckpointBlock> blocks;
};

struct DefragMove {
  KVBlockID id;
  std::string node_id;
  uint64_t from_segment = 0, from_offset = 0, to_segment = 0, to_offset = 0;
  bool compact_segment = false;
  uint64_t segment_id = 0;
};

struct ShardEntry {
  std::string node_id;
  uint32_t vnode_count = 0;
  bool draining = false;
  std::vector<uint64_t> vnode_hashes;
};

struct ShardMap {
  uint64_t generation = 0;
  uint32_t default_vnode_count = 64;
  std::vector<ShardEntry> nodes;
};

struct ShardMigration {
  KVBlockID id;
  std::string from_node, to_node;
  bool push_l2_first = false;
};

struct PlacementPlan {
  std::string node_id;
  std::vector<KVBlockID> ids;
};

}  // namespace lakeb::cp
