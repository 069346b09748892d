// Background frame loading (the role of the reference's Rust FrameLoaderService and
// ImageCache, rust/drivedit-data/src/frame_loader.rs:28-290 and frames.rs:31): requests
// are split into per-frame jobs for a fixed worker pool; decoded, resized frames go into
// a byte-bounded-by-count LRU cache so frames shared by overlapping clips decode once.
#include "service.h"

#include <cstring>
#include <stdexcept>

#include "frames.h"

namespace ddd {

bool FrameCache::get(const std::string& key, uint8_t* out, size_t bytes) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = index_.find(key);
  if (it == index_.end() || it->second->second.size() != bytes) {
    ++misses_;
    return false;
  }
  lru_.splice(lru_.begin(), lru_, it->second);
  std::memcpy(out, it->second->second.data(), bytes);
  ++hits_;
  return true;
}

void FrameCache::put(const std::string& key, const uint8_t* data, size_t bytes) {
  if (capacity_ == 0) return;
  std::lock_guard<std::mutex> g(mu_);
  auto it = index_.find(key);
  if (it != index_.end()) {
    lru_.erase(it->second);
    index_.erase(it);
  }
  lru_.emplace_front(key, std::vector<uint8_t>(data, data + bytes));
  index_[key] = lru_.begin();
  while (lru_.size() > capacity_) {
    index_.erase(lru_.back().first);
    lru_.pop_back();
  }
}

size_t FrameCache::size() const {
  std::lock_guard<std::mutex> g(mu_);
  return lru_.size();
}

void FrameCache::clear() {
  std::lock_guard<std::mutex> g(mu_);
  lru_.clear();
  index_.clear();
}

FrameLoaderService::FrameLoaderService(int threads, size_t cache_frames) : cache_(cache_frames) {
  const int t = threads > 0 ? threads : static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
  for (int i = 0; i < t; ++i) workers_.emplace_back([this] { worker(); });
}

FrameLoaderService::~FrameLoaderService() {
  {
    std::lock_guard<std::mutex> g(mu_);
    stop_ = true;
  }
  cv_.notify_all();
  for (auto& w : workers_) w.join();
}

int64_t FrameLoaderService::submit(const std::vector<std::string>& paths, int H, int W, uint8_t* out) {
  std::lock_guard<std::mutex> g(mu_);
  const int64_t id = next_id_++;
  remaining_[id] = static_cast<int>(paths.size());
  const size_t plane = static_cast<size_t>(H) * W * 3;
  for (size_t i = 0; i < paths.size(); ++i) jobs_.push_back({id, paths[i], H, W, out + i * plane});
  if (paths.empty()) done_cv_.notify_all();
  cv_.notify_all();
  return id;
}

void FrameLoaderService::finish_one(int64_t id, const std::string& err) {
  std::lock_guard<std::mutex> g(mu_);
  if (!err.empty() && !errors_.count(id)) errors_[id] = err;
  if (--remaining_[id] == 0) done_cv_.notify_all();
}

void FrameLoaderService::worker() {
  for (;;) {
    Job j;
    {
      std::unique_lock<std::mutex> g(mu_);
      cv_.wait(g, [this] { return stop_ || !jobs_.empty(); });
      if (stop_ && jobs_.empty()) return;
      j = jobs_.front();
      jobs_.pop_front();
    }
    std::string err;
    try {
      const size_t bytes = static_cast<size_t>(j.H) * j.W * 3;
      const std::string key = j.path + "|" + std::to_string(j.H) + "x" + std::to_string(j.W);
      if (!cache_.get(key, j.out, bytes)) {
        const Image img = decode_png_file(j.path);
        if (img.h == j.H && img.w == j.W) std::memcpy(j.out, img.rgb.data(), bytes);
        else resize_bilinear(img, j.H, j.W, j.out);
        cache_.put(key, j.out, bytes);
      }
    } catch (const std::exception& e) {
      err = std::string(e.what()) + " (" + j.path + ")";
    }
    finish_one(j.id, err);
  }
}

void FrameLoaderService::wait(int64_t id) {
  std::unique_lock<std::mutex> g(mu_);
  if (!remaining_.count(id)) throw std::runtime_error("FrameLoaderService: unknown request");
  done_cv_.wait(g, [&] { return remaining_[id] <= 0; });
  remaining_.erase(id);
  auto e = errors_.find(id);
  if (e != errors_.end()) {
    const std::string msg = e->second;
    errors_.erase(e);
    throw std::runtime_error(msg);
  }
}

bool FrameLoaderService::done(int64_t id) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = remaining_.find(id);
  return it == remaining_.end() || it->second <= 0;
}

size_t FrameLoaderService::pending() const {
  std::lock_guard<std::mutex> g(mu_);
  return jobs_.size();
}

}  // namespace ddd
