// Native frame loading: PNG decode (zlib inflate + scanline unfiltering), bilinear resize
// (half-pixel centres, the convention of F.interpolate(align_corners=False)) and batched
// multi-threaded loading into one uint8 [N, H, W, 3] buffer.
//
// Replaces the reference's Rust FrameLoader (rust/drivedit-data/src/frames.rs:71-420,
// rayon decode + resize) for the PNG frames that Enfusion sessions store
// (data/enfusion_loader.py:6-30); 8- and 16-bit grey / grey+alpha / RGB / RGBA,
// non-interlaced. Other formats are decoded on the Python side.
#include "frames.h"

#include <zlib.h>

#include <cmath>
#include <cstring>
#include <fstream>
#include <sstream>
#include <stdexcept>

#include "parallel.h"

namespace ddd {

namespace {

uint32_t be32(const uint8_t* p) {
  return (uint32_t(p[0]) << 24) | (uint32_t(p[1]) << 16) | (uint32_t(p[2]) << 8) | uint32_t(p[3]);
}

int paeth(int a, int b, int c) {
  const int p = a + b - c;
  const int pa = std::abs(p - a), pb = std::abs(p - b), pc = std::abs(p - c);
  if (pa <= pb && pa <= pc) return a;
  if (pb <= pc) return b;
  return c;
}

std::vector<uint8_t> read_file(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("frames: cannot open " + path);
  return std::vector<uint8_t>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

}  // namespace

PngPixels decode_png_pixels(const uint8_t* data, size_t size) {
  static const uint8_t sig[8] = {0x89, 'P', 'N', 'G', '\r', '\n', 0x1a, '\n'};
  if (size < 8 || std::memcmp(data, sig, 8) != 0) throw std::runtime_error("PNG: bad signature");
  size_t o = 8;
  uint32_t w = 0, h = 0;
  int depth = 0, ctype = -1, interlace = 0;
  std::vector<uint8_t> z;
  while (o + 12 <= size) {
    const uint32_t len = be32(data + o);
    const uint8_t* type = data + o + 4;
    const uint8_t* body = data + o + 8;
    if (o + 12 + len > size) throw std::runtime_error("PNG: truncated chunk");
    if (!std::memcmp(type, "IHDR", 4)) {
      w = be32(body);
      h = be32(body + 4);
      depth = body[8];
      ctype = body[9];
      interlace = body[12];
    } else if (!std::memcmp(type, "IDAT", 4)) {
      z.insert(z.end(), body, body + len);
    } else if (!std::memcmp(type, "IEND", 4)) {
      break;
    }
    o += 12 + len;
  }
  if (w == 0 || h == 0) throw std::runtime_error("PNG: missing IHDR");
  if (interlace) throw std::runtime_error("PNG: interlaced images are not supported");
  if (depth != 8 && depth != 16) throw std::runtime_error("PNG: unsupported bit depth");
  int ch;
  switch (ctype) {
    case 0: ch = 1; break;
    case 2: ch = 3; break;
    case 4: ch = 2; break;
    case 6: ch = 4; break;
    default: throw std::runtime_error("PNG: unsupported colour type (palette?)");
  }
  const size_t bpp = static_cast<size_t>(ch) * (depth / 8);
  const size_t stride = bpp * w;
  std::vector<uint8_t> raw((stride + 1) * h);
  uLongf dlen = static_cast<uLongf>(raw.size());
  if (uncompress(raw.data(), &dlen, z.data(), static_cast<uLong>(z.size())) != Z_OK || dlen != raw.size())
    throw std::runtime_error("PNG: inflate failed");
  std::vector<uint8_t> px(stride * h);
  for (uint32_t y = 0; y < h; ++y) {
    const uint8_t ft = raw[y * (stride + 1)];
    const uint8_t* src = &raw[y * (stride + 1) + 1];
    uint8_t* dst = &px[y * stride];
    const uint8_t* up = y ? &px[(y - 1) * stride] : nullptr;
    for (size_t x = 0; x < stride; ++x) {
      const int a = x >= bpp ? dst[x - bpp] : 0;
      const int b = up ? up[x] : 0;
      const int c = (up && x >= bpp) ? up[x - bpp] : 0;
      int v = src[x];
      switch (ft) {
        case 0: break;
        case 1: v += a; break;
        case 2: v += b; break;
        case 3: v += (a + b) >> 1; break;
        case 4: v += paeth(a, b, c); break;
        default: throw std::runtime_error("PNG: bad filter type");
      }
      dst[x] = static_cast<uint8_t>(v);
    }
  }
  PngPixels out;
  out.w = static_cast<int>(w);
  out.h = static_cast<int>(h);
  out.channels = ch;
  out.depth = depth;
  out.px = std::move(px);
  return out;
}

Image decode_png(const uint8_t* data, size_t size) {
  const PngPixels pp = decode_png_pixels(data, size);
  const uint32_t w = pp.w, h = pp.h;
  const int ch = pp.channels, depth = pp.depth;
  const size_t bpp = static_cast<size_t>(ch) * (depth / 8);
  const std::vector<uint8_t>& px = pp.px;
  Image img;
  img.w = static_cast<int>(w);
  img.h = static_cast<int>(h);
  img.rgb.resize(static_cast<size_t>(w) * h * 3);
  const int step = depth / 8;  // 16-bit: the most significant byte comes first
  for (size_t i = 0; i < static_cast<size_t>(w) * h; ++i) {
    const uint8_t* p = &px[i * bpp];
    uint8_t r, g, b;
    if (ch >= 3) {
      r = p[0];
      g = p[step];
      b = p[2 * step];
    } else {
      r = g = b = p[0];
    }
    img.rgb[i * 3] = r;
    img.rgb[i * 3 + 1] = g;
    img.rgb[i * 3 + 2] = b;
  }
  return img;
}

Image decode_png_file(const std::string& path) {
  const auto bytes = read_file(path);
  return decode_png(bytes.data(), bytes.size());
}

void resize_bilinear(const Image& src, int H, int W, uint8_t* out) {
  const float sy = static_cast<float>(src.h) / H, sx = static_cast<float>(src.w) / W;
  for (int y = 0; y < H; ++y) {
    float fy = (y + 0.5f) * sy - 0.5f;
    if (fy < 0) fy = 0;
    int y0 = static_cast<int>(fy);
    if (y0 > src.h - 1) y0 = src.h - 1;
    const int y1 = std::min(y0 + 1, src.h - 1);
    const float wy = fy - y0;
    for (int x = 0; x < W; ++x) {
      float fx = (x + 0.5f) * sx - 0.5f;
      if (fx < 0) fx = 0;
      int x0 = static_cast<int>(fx);
      if (x0 > src.w - 1) x0 = src.w - 1;
      const int x1 = std::min(x0 + 1, src.w - 1);
      const float wx = fx - x0;
      for (int c = 0; c < 3; ++c) {
        const float v00 = src.rgb[(y0 * src.w + x0) * 3 + c], v01 = src.rgb[(y0 * src.w + x1) * 3 + c];
        const float v10 = src.rgb[(y1 * src.w + x0) * 3 + c], v11 = src.rgb[(y1 * src.w + x1) * 3 + c];
        const float v = (1 - wy) * ((1 - wx) * v00 + wx * v01) + wy * ((1 - wx) * v10 + wx * v11);
        out[(y * W + x) * 3 + c] = static_cast<uint8_t>(std::lround(std::min(255.f, std::max(0.f, v))));
      }
    }
  }
}

void load_frames(const std::vector<std::string>& paths, int H, int W, int threads, uint8_t* out) {
  const size_t per = static_cast<size_t>(H) * W * 3;
  parallel_for(static_cast<int64_t>(paths.size()), threads, [&](int64_t i) {
    const Image img = decode_png_file(paths[i]);
    if (img.h == H && img.w == W)
      std::memcpy(out + i * per, img.rgb.data(), per);
    else
      resize_bilinear(img, H, W, out + i * per);
  });
}

}  // namespace ddd
