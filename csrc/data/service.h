// Background frame loading: a bounded LRU cache of decoded frames and a worker pool that
// fills caller-owned uint8 [N, H, W, 3] buffers asynchronously (submit -> wait).
#pragma once
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <functional>
#include <list>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

namespace ddd {

// LRU cache of resized frames keyed by (path, H, W); thread-safe.
class FrameCache {
 public:
  explicit FrameCache(size_t capacity) : capacity_(capacity) {}
  bool get(const std::string& key, uint8_t* out, size_t bytes);
  void put(const std::string& key, const uint8_t* data, size_t bytes);
  size_t size() const;
  size_t hits() const { return hits_; }
  size_t misses() const { return misses_; }
  void clear();

 private:
  size_t capacity_;
  mutable std::mutex mu_;
  std::list<std::pair<std::string, std::vector<uint8_t>>> lru_;
  std::unordered_map<std::string, decltype(lru_)::iterator> index_;
  size_t hits_ = 0, misses_ = 0;
};

class FrameLoaderService {
 public:
  FrameLoaderService(int threads, size_t cache_frames);
  ~FrameLoaderService();
  // Decodes + resizes `paths` into out (paths.size() x H x W x 3) in the background.
  int64_t submit(const std::vector<std::string>& paths, int H, int W, uint8_t* out);
  // Blocks until request `id` is done; rethrows its error (message) if it failed.
  void wait(int64_t id);
  bool done(int64_t id);
  size_t pending() const;
  FrameCache& cache() { return cache_; }

 private:
  struct Job {
    int64_t id;
    std::string path;
    int H, W;
    uint8_t* out;
  };
  void worker();
  void finish_one(int64_t id, const std::string& err);

  FrameCache cache_;
  mutable std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  std::deque<Job> jobs_;
  std::unordered_map<int64_t, int> remaining_;
  std::unordered_map<int64_t, std::string> errors_;
  std::vector<std::thread> workers_;
  int64_t next_id_ = 1;
  bool stop_ = false;
};

}  // namespace ddd
