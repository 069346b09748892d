// PNG decode, bilinear resize and batched parallel frame loading (uint8 RGB).
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace ddd {

struct Image {
  int w = 0, h = 0;
  std::vector<uint8_t> rgb;  // h x w x 3
};

// Unfiltered PNG samples: h x w x channels, 1 or 2 bytes per sample (16-bit big-endian).
struct PngPixels {
  int w = 0, h = 0, channels = 0, depth = 0;
  std::vector<uint8_t> px;
};
PngPixels decode_png_pixels(const uint8_t* data, size_t size);
Image decode_png(const uint8_t* data, size_t size);
Image decode_png_file(const std::string& path);
void resize_bilinear(const Image& src, int H, int W, uint8_t* out);
// out: paths.size() x H x W x 3 (resized when a frame's size differs)
void load_frames(const std::vector<std::string>& paths, int H, int W, int threads, uint8_t* out);

}  // namespace ddd
