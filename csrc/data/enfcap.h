// ENFCAP v1 capture files: memory-mapped reader with O(1) random frame access and
// multi-threaded batch decode, and an append-only writer.
//
// Layout (little endian, packed), the same bytes the reference's Rust crate reads and
// writes (rust/drivedit-data/src/enfcap.rs:61-79, :162-222, :562-680):
//   header (64 B): "ENFCAP01", u32 version = 1, u32 frame_count,
//                  f32 start_ts_lo, f32 start_ts_hi (ts = lo + hi * FLT_MAX), u32 flags,
//                  36 reserved bytes
//   frames:        u32 frame_id, f32 timestamp, f32 ego[12] (3x4), f32 vehicle[10],
//                  u16 n_entities, n x {u32 type, f32 x, y, z}, u16 n_road, n x f32[3],
//                  u16 flags                                   (102 B + variable)
//   index (end):   frame_count x u64 absolute frame offsets
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include "parallel.h"

namespace ddd {

constexpr char kEnfcapMagic[8] = {'E', 'N', 'F', 'C', 'A', 'P', '0', '1'};
constexpr uint32_t kEnfcapVersion = 1;
constexpr size_t kHeaderSize = 64;
constexpr size_t kFrameBaseSize = 102;
constexpr size_t kEntitySize = 16;
constexpr size_t kRoadPointSize = 12;

struct Entity {
  uint32_t type = 0;
  float pos[3] = {0, 0, 0};
};

struct Frame {
  uint32_t frame_id = 0;
  float timestamp = 0;
  float ego[12] = {};
  float vehicle[10] = {};
  std::vector<Entity> entities;
  std::vector<float> road;  // 3 floats per point
  uint16_t flags = 0;
};

// Struct-of-arrays result of a batch read.
struct FrameBatch {
  std::vector<uint32_t> frame_id;
  std::vector<float> timestamp;
  std::vector<float> ego;      // n x 12
  std::vector<float> vehicle;  // n x 10
  std::vector<uint16_t> flags;
  std::vector<int64_t> entity_offsets;  // n + 1 (prefix sums into entity arrays)
  std::vector<uint32_t> entity_type;
  std::vector<float> entity_pos;        // 3 per entity
  std::vector<int64_t> road_offsets;    // n + 1
  std::vector<float> road;              // 3 per point
};

class EnfcapReader {
 public:
  explicit EnfcapReader(const std::string& path);
  ~EnfcapReader();
  EnfcapReader(const EnfcapReader&) = delete;
  EnfcapReader& operator=(const EnfcapReader&) = delete;

  uint32_t frame_count() const { return frame_count_; }
  uint32_t flags() const { return flags_; }
  double start_timestamp() const { return start_ts_; }
  const std::string& path() const { return path_; }

  Frame read_frame(uint32_t i) const;
  // frames [start, end) decoded by `threads` worker threads (0 = hardware concurrency)
  FrameBatch read_frames(uint32_t start, uint32_t end, int threads) const;
  // (valid frames, first error message or "")
  std::pair<uint32_t, std::string> validate() const;

 private:
  void release();
  std::string path_;
  int fd_ = -1;
  const uint8_t* data_ = nullptr;
  size_t size_ = 0;
  uint32_t frame_count_ = 0;
  uint32_t flags_ = 0;
  double start_ts_ = 0;
  const uint8_t* index_ = nullptr;
};

class EnfcapWriter {
 public:
  EnfcapWriter(const std::string& path, double start_timestamp, uint32_t flags);
  ~EnfcapWriter();
  void write_frame(const Frame& f);
  void finalize();
  uint32_t frames_written() const { return static_cast<uint32_t>(offsets_.size()); }

 private:
  std::string path_;
  void* fp_ = nullptr;
  double start_ts_;
  uint32_t flags_;
  uint64_t pos_ = 0;
  std::vector<uint64_t> offsets_;
  bool finalized_ = false;
};

// Decode a frame record at `p` (at most `avail` bytes); returns the bytes consumed, or
// throws on a truncated record.
size_t decode_frame(const uint8_t* p, size_t avail, Frame& out);
std::vector<uint8_t> encode_frame(const Frame& f);

}  // namespace ddd
