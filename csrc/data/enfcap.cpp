#include "enfcap.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cfloat>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <stdexcept>

namespace ddd {

namespace {
template <class T>
T rd(const uint8_t* p) {
  T v;
  std::memcpy(&v, p, sizeof(T));
  return v;
}
template <class T>
void wr(std::vector<uint8_t>& b, T v) {
  const auto* p = reinterpret_cast<const uint8_t*>(&v);
  b.insert(b.end(), p, p + sizeof(T));
}
}  // namespace

size_t decode_frame(const uint8_t* p, size_t avail, Frame& f) {
  if (avail < kFrameBaseSize) throw std::runtime_error("ENFCAP: truncated frame record");
  size_t o = 0;
  f.frame_id = rd<uint32_t>(p + o);
  o += 4;
  f.timestamp = rd<float>(p + o);
  o += 4;
  std::memcpy(f.ego, p + o, 48);
  o += 48;
  std::memcpy(f.vehicle, p + o, 40);
  o += 40;
  const size_t ne = rd<uint16_t>(p + o);
  o += 2;
  if (avail < o + ne * kEntitySize + 4) throw std::runtime_error("ENFCAP: truncated entity list");
  f.entities.resize(ne);
  for (size_t i = 0; i < ne; ++i) {
    const uint8_t* q = p + o + i * kEntitySize;
    f.entities[i].type = rd<uint32_t>(q);
    std::memcpy(f.entities[i].pos, q + 4, 12);
  }
  o += ne * kEntitySize;
  const size_t nr = rd<uint16_t>(p + o);
  o += 2;
  if (avail < o + nr * kRoadPointSize + 2) throw std::runtime_error("ENFCAP: truncated road list");
  f.road.resize(nr * 3);
  if (nr) std::memcpy(f.road.data(), p + o, nr * kRoadPointSize);
  o += nr * kRoadPointSize;
  f.flags = rd<uint16_t>(p + o);
  o += 2;
  return o;
}

std::vector<uint8_t> encode_frame(const Frame& f) {
  std::vector<uint8_t> b;
  const size_t ne = std::min<size_t>(f.entities.size(), 65535);
  const size_t nr = std::min<size_t>(f.road.size() / 3, 65535);
  b.reserve(kFrameBaseSize + ne * kEntitySize + nr * kRoadPointSize);
  wr<uint32_t>(b, f.frame_id);
  wr<float>(b, f.timestamp);
  for (float v : f.ego) wr<float>(b, v);
  for (float v : f.vehicle) wr<float>(b, v);
  wr<uint16_t>(b, static_cast<uint16_t>(ne));
  for (size_t i = 0; i < ne; ++i) {
    wr<uint32_t>(b, f.entities[i].type);
    for (float v : f.entities[i].pos) wr<float>(b, v);
  }
  wr<uint16_t>(b, static_cast<uint16_t>(nr));
  for (size_t i = 0; i < nr * 3; ++i) wr<float>(b, f.road[i]);
  wr<uint16_t>(b, f.flags);
  return b;
}

// ------------------------------------------------------------------ reader
EnfcapReader::EnfcapReader(const std::string& path) : path_(path) {
  fd_ = ::open(path.c_str(), O_RDONLY);
  if (fd_ < 0) throw std::runtime_error("ENFCAP: cannot open " + path);
  struct stat st;
  if (fstat(fd_, &st) != 0) {
    ::close(fd_);
    throw std::runtime_error("ENFCAP: cannot stat " + path);
  }
  size_ = static_cast<size_t>(st.st_size);
  if (size_ < kHeaderSize) {
    ::close(fd_);
    throw std::runtime_error("ENFCAP: file too small: " + path);
  }
  void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
  if (m == MAP_FAILED) {
    ::close(fd_);
    throw std::runtime_error("ENFCAP: mmap failed: " + path);
  }
  data_ = static_cast<const uint8_t*>(m);
  if (std::memcmp(data_, kEnfcapMagic, 8) != 0) {
    release();
    throw std::runtime_error("ENFCAP: invalid magic (expected ENFCAP01): " + path);
  }
  const uint32_t ver = rd<uint32_t>(data_ + 8);
  if (ver != kEnfcapVersion) {
    release();
    throw std::runtime_error("ENFCAP: unsupported version " + std::to_string(ver));
  }
  frame_count_ = rd<uint32_t>(data_ + 12);
  const float lo = rd<float>(data_ + 16), hi = rd<float>(data_ + 20);
  // The format's writer stores lo = ts and hi = ts / FLT_MAX (the reference decodes
  // lo + hi * FLT_MAX, which is 2 ts for such files). When hi is exactly that redundant
  // copy of lo, lo is the timestamp; otherwise (a genuine split) lo + hi * FLT_MAX.
  const double hi_part = static_cast<double>(hi) * static_cast<double>(FLT_MAX);
  const double dl = static_cast<double>(lo);
  start_ts_ = (hi != 0.f && std::abs(hi_part - dl) <= 1e-3 * std::abs(dl) + 1e-3) ? dl : dl + hi_part;
  flags_ = rd<uint32_t>(data_ + 24);
  const size_t isz = static_cast<size_t>(frame_count_) * 8;
  if (size_ < kHeaderSize + isz) {
    release();
    throw std::runtime_error("ENFCAP: invalid index table");
  }
  index_ = data_ + size_ - isz;
}

void EnfcapReader::release() {
  if (data_) munmap(const_cast<uint8_t*>(data_), size_);
  data_ = nullptr;
  if (fd_ >= 0) ::close(fd_);
  fd_ = -1;
}

EnfcapReader::~EnfcapReader() { release(); }

Frame EnfcapReader::read_frame(uint32_t i) const {
  if (i >= frame_count_)
    throw std::out_of_range("ENFCAP: frame " + std::to_string(i) + " out of bounds (" +
                            std::to_string(frame_count_) + " frames)");
  const uint64_t off = rd<uint64_t>(index_ + 8 * i);
  const size_t end = static_cast<size_t>(index_ - data_);
  if (off < kHeaderSize || off >= end) throw std::runtime_error("ENFCAP: corrupt index entry");
  Frame f;
  decode_frame(data_ + off, end - off, f);
  return f;
}

FrameBatch EnfcapReader::read_frames(uint32_t start, uint32_t end, int threads) const {
  end = std::min(end, frame_count_);
  FrameBatch b;
  if (start >= end) {
    b.entity_offsets = {0};
    b.road_offsets = {0};
    return b;
  }
  const uint32_t n = end - start;
  std::vector<Frame> frames(n);
  parallel_for(n, threads, [&](int64_t i) { frames[i] = read_frame(start + static_cast<uint32_t>(i)); });
  b.frame_id.resize(n);
  b.timestamp.resize(n);
  b.ego.resize(n * 12);
  b.vehicle.resize(n * 10);
  b.flags.resize(n);
  b.entity_offsets.assign(n + 1, 0);
  b.road_offsets.assign(n + 1, 0);
  for (uint32_t i = 0; i < n; ++i) {
    b.entity_offsets[i + 1] = b.entity_offsets[i] + frames[i].entities.size();
    b.road_offsets[i + 1] = b.road_offsets[i] + frames[i].road.size() / 3;
  }
  b.entity_type.resize(b.entity_offsets[n]);
  b.entity_pos.resize(b.entity_offsets[n] * 3);
  b.road.resize(b.road_offsets[n] * 3);
  parallel_for(n, threads, [&](int64_t i) {
    const Frame& f = frames[i];
    b.frame_id[i] = f.frame_id;
    b.timestamp[i] = f.timestamp;
    std::memcpy(&b.ego[i * 12], f.ego, 48);
    std::memcpy(&b.vehicle[i * 10], f.vehicle, 40);
    b.flags[i] = f.flags;
    for (size_t e = 0; e < f.entities.size(); ++e) {
      const int64_t k = b.entity_offsets[i] + e;
      b.entity_type[k] = f.entities[e].type;
      std::memcpy(&b.entity_pos[k * 3], f.entities[e].pos, 12);
    }
    if (!f.road.empty())
      std::memcpy(&b.road[b.road_offsets[i] * 3], f.road.data(), f.road.size() * sizeof(float));
  });
  return b;
}

std::pair<uint32_t, std::string> EnfcapReader::validate() const {
  uint32_t ok = 0;
  std::string first;
  for (uint32_t i = 0; i < frame_count_; ++i) {
    try {
      read_frame(i);
      ++ok;
    } catch (const std::exception& e) {
      if (first.empty()) first = "frame " + std::to_string(i) + ": " + e.what();
    }
  }
  return {ok, first};
}

// ------------------------------------------------------------------ writer
EnfcapWriter::EnfcapWriter(const std::string& path, double start_timestamp, uint32_t flags)
    : path_(path), start_ts_(start_timestamp), flags_(flags) {
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) throw std::runtime_error("ENFCAP: cannot create " + path);
  fp_ = f;
  std::vector<uint8_t> hdr(kHeaderSize, 0);  // rewritten by finalize()
  if (std::fwrite(hdr.data(), 1, hdr.size(), f) != hdr.size())
    throw std::runtime_error("ENFCAP: write failed");
  pos_ = kHeaderSize;
}

EnfcapWriter::~EnfcapWriter() {
  if (fp_) std::fclose(static_cast<FILE*>(fp_));
}

void EnfcapWriter::write_frame(const Frame& fr) {
  if (finalized_) throw std::runtime_error("ENFCAP: writer already finalized");
  const auto bytes = encode_frame(fr);
  if (std::fwrite(bytes.data(), 1, bytes.size(), static_cast<FILE*>(fp_)) != bytes.size())
    throw std::runtime_error("ENFCAP: write failed");
  offsets_.push_back(pos_);
  pos_ += bytes.size();
}

void EnfcapWriter::finalize() {
  if (finalized_) return;
  FILE* f = static_cast<FILE*>(fp_);
  std::vector<uint8_t> idx;
  for (uint64_t o : offsets_) wr<uint64_t>(idx, o);
  if (!idx.empty() && std::fwrite(idx.data(), 1, idx.size(), f) != idx.size())
    throw std::runtime_error("ENFCAP: index write failed");
  std::vector<uint8_t> hdr;
  hdr.insert(hdr.end(), kEnfcapMagic, kEnfcapMagic + 8);
  wr<uint32_t>(hdr, kEnfcapVersion);
  wr<uint32_t>(hdr, static_cast<uint32_t>(offsets_.size()));
  wr<float>(hdr, static_cast<float>(start_ts_));
  wr<float>(hdr, static_cast<float>(start_ts_ / static_cast<double>(FLT_MAX)));
  wr<uint32_t>(hdr, flags_);
  hdr.resize(kHeaderSize, 0);
  std::fseek(f, 0, SEEK_SET);
  if (std::fwrite(hdr.data(), 1, hdr.size(), f) != hdr.size())
    throw std::runtime_error("ENFCAP: header write failed");
  std::fclose(f);
  fp_ = nullptr;
  finalized_ = true;
}

}  // namespace ddd
