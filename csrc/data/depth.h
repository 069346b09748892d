// Depth maps: .npy / .npz (stored or deflated members) / 16-bit PNG -> float32, bilinear
// resize, min-max normalisation to [0, 1] (optional clip / inversion), batched parallel load.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace ddd {

struct DepthLoaderConfig {
  int target_width = 640, target_height = 360;  // 0 = keep the source size
  float min_depth = 0.f, max_depth = 0.f;       // both 0 = range from the finite values
  bool clip_depth = true;
  bool invert_depth = false;
  std::string npz_array_name = "depth";
};

struct DepthMap {
  int width = 0, height = 0;
  float original_min = 0.f, original_max = 0.f;
  std::vector<float> data;  // height x width, normalised
};

// Raw float32 array [h, w] from an .npy byte buffer (dtypes <f4 <f8 <f2 <u2 <u1 <i4, C order;
// shapes (h, w), (1, h, w) or (h, w, 1)).
std::vector<float> npy_to_float(const uint8_t* data, size_t size, int* h, int* w);
// The member "<name>.npy" of an .npz (zip) byte buffer; an empty name takes the first .npy member.
std::vector<uint8_t> npz_member(const uint8_t* data, size_t size, const std::string& name);

DepthMap process_depth(const std::vector<float>& src, int h, int w, const DepthLoaderConfig& cfg);
DepthMap load_depth(const std::string& path, const DepthLoaderConfig& cfg);
// out: paths.size() x target_height x target_width (all maps resized to the target)
void load_depth_batch(const std::vector<std::string>& paths, const DepthLoaderConfig& cfg, int threads,
                      float* out);

}  // namespace ddd
