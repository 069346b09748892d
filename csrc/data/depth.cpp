// Native depth-map loader, the C++ counterpart of the reference's Rust DepthLoader
// (rust/drivedit-data/src/depth.rs:59-505): same configuration (target size, depth range or
// automatic range from the finite samples, clipping, inversion, npz member name), same
// bilinear sampling (source coordinate = destination index x source/destination ratio,
// neighbours clamped at the border) and the same normalisation to [0, 1]. The .npy parser,
// the zip reader for .npz (stored or deflated members, zip64 sizes, zlib raw inflate) and the 16-bit PNG
// path are written here; EXR is not supported (the reference's EXR path is a placeholder too).
#include "depth.h"

#include <zlib.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <fstream>
#include <limits>
#include <stdexcept>

#include "frames.h"
#include "parallel.h"

namespace ddd {
namespace {

std::vector<uint8_t> read_all(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("depth: cannot open " + path);
  return std::vector<uint8_t>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

uint16_t le16(const uint8_t* p) { return static_cast<uint16_t>(p[0] | (p[1] << 8)); }
uint32_t le32(const uint8_t* p) { return p[0] | (p[1] << 8) | (p[2] << 16) | (uint32_t(p[3]) << 24); }

std::string ext_of(const std::string& path) {
  const auto dot = path.find_last_of('.');
  std::string e = dot == std::string::npos ? "" : path.substr(dot + 1);
  for (auto& c : e) c = static_cast<char>(std::tolower(c));
  return e;
}

float half_to_float(uint16_t h) {
  const uint32_t s = (h >> 15) & 1, e = (h >> 10) & 0x1f, m = h & 0x3ff;
  float v;
  if (e == 0) v = std::ldexp(static_cast<float>(m), -24);
  else if (e == 31) v = m ? std::numeric_limits<float>::quiet_NaN() : std::numeric_limits<float>::infinity();
  else v = std::ldexp(static_cast<float>(m | 0x400), static_cast<int>(e) - 25);
  return s ? -v : v;
}

}  // namespace

std::vector<float> npy_to_float(const uint8_t* data, size_t size, int* h, int* w) {
  if (size < 10 || std::memcmp(data, "\x93NUMPY", 6) != 0) throw std::runtime_error("npy: bad magic");
  const int major = data[6];
  size_t hlen, off;
  if (major == 1) {
    hlen = le16(data + 8);
    off = 10;
  } else {
    if (size < 12) throw std::runtime_error("npy: truncated header");
    hlen = le32(data + 8);
    off = 12;
  }
  if (off + hlen > size) throw std::runtime_error("npy: truncated header");
  const std::string hdr(reinterpret_cast<const char*>(data + off), hlen);
  auto field = [&](const char* key) {
    const auto k = hdr.find(key);
    if (k == std::string::npos) throw std::runtime_error(std::string("npy: header lacks ") + key);
    return k + std::strlen(key);
  };
  size_t p = hdr.find('\'', field("'descr':")) + 1;
  const std::string descr = hdr.substr(p, hdr.find('\'', p) - p);
  if (hdr.find("True", field("'fortran_order':")) < hdr.find(',', field("'fortran_order':")))
    throw std::runtime_error("npy: Fortran-ordered arrays are not supported");
  p = hdr.find('(', field("'shape':")) + 1;
  const std::string shp = hdr.substr(p, hdr.find(')', p) - p);
  std::vector<long> dims;
  for (size_t i = 0; i < shp.size();) {
    while (i < shp.size() && !std::isdigit(static_cast<unsigned char>(shp[i]))) ++i;
    size_t j = i;
    while (j < shp.size() && std::isdigit(static_cast<unsigned char>(shp[j]))) ++j;
    if (j > i) dims.push_back(std::stol(shp.substr(i, j - i)));
    i = j;
  }
  std::vector<long> hw;
  for (long d : dims)
    if (d != 1) hw.push_back(d);
  while (hw.size() < 2) hw.insert(hw.begin(), 1);
  if (hw.size() != 2) throw std::runtime_error("npy: expected a 2-D depth array");
  *h = static_cast<int>(hw[0]);
  *w = static_cast<int>(hw[1]);
  const size_t n = static_cast<size_t>(*h) * *w;
  const uint8_t* src = data + off + hlen;
  const size_t avail = size - off - hlen;
  std::vector<float> out(n);
  auto need = [&](size_t es) {
    if (avail < n * es) throw std::runtime_error("npy: truncated data");
  };
  if (descr == "<f4" || descr == "|f4") {
    need(4);
    std::memcpy(out.data(), src, n * 4);
  } else if (descr == "<f8") {
    need(8);
    for (size_t i = 0; i < n; ++i) {
      double d;
      std::memcpy(&d, src + 8 * i, 8);
      out[i] = static_cast<float>(d);
    }
  } else if (descr == "<f2") {
    need(2);
    for (size_t i = 0; i < n; ++i) out[i] = half_to_float(le16(src + 2 * i));
  } else if (descr == "<u2") {
    need(2);
    for (size_t i = 0; i < n; ++i) out[i] = le16(src + 2 * i);
  } else if (descr == "|u1" || descr == "<u1") {
    need(1);
    for (size_t i = 0; i < n; ++i) out[i] = src[i];
  } else if (descr == "<i4") {
    need(4);
    for (size_t i = 0; i < n; ++i) out[i] = static_cast<float>(static_cast<int32_t>(le32(src + 4 * i)));
  } else {
    throw std::runtime_error("npy: unsupported dtype " + descr);
  }
  return out;
}

std::vector<uint8_t> npz_member(const uint8_t* data, size_t size, const std::string& name) {
  const std::string want = name + ".npy";
  size_t o = 0;
  while (o + 30 <= size && le32(data + o) == 0x04034b50) {  // local file header
    const uint16_t flags = le16(data + o + 6), method = le16(data + o + 8);
    uint64_t csize = le32(data + o + 18);
    uint64_t usize = le32(data + o + 22);
    const uint16_t nlen = le16(data + o + 26), xlen = le16(data + o + 28);
    const std::string fname(reinterpret_cast<const char*>(data + o + 30), nlen);
    const size_t body = o + 30 + nlen + xlen;
    if (flags & 0x8) throw std::runtime_error("npz: streamed members (data descriptors) are not supported");
    if (csize == 0xffffffffu || usize == 0xffffffffu) {  // sizes in the zip64 extra field
      size_t e = o + 30 + nlen;
      const size_t end = e + xlen;
      bool found = false;
      while (e + 4 <= end) {
        const uint16_t id = le16(data + e), sz = le16(data + e + 2);
        if (id == 0x0001) {
          size_t q = e + 4;
          auto rd64 = [&](uint64_t* v) {
            if (q + 8 > e + 4 + sz) throw std::runtime_error("npz: bad zip64 field");
            *v = le32(data + q) | (static_cast<uint64_t>(le32(data + q + 4)) << 32);
            q += 8;
          };
          if (usize == 0xffffffffu) rd64(&usize);
          if (csize == 0xffffffffu) rd64(&csize);
          found = true;
          break;
        }
        e += 4 + sz;
      }
      if (!found) throw std::runtime_error("npz: zip64 sizes missing");
    }
    if (body + csize > size) throw std::runtime_error("npz: truncated member");
    const bool is_npy = fname.size() > 4 && fname.compare(fname.size() - 4, 4, ".npy") == 0;
    if (fname == want || (name.empty() && is_npy)) {
      if (method == 0) return std::vector<uint8_t>(data + body, data + body + csize);
      if (method != 8) throw std::runtime_error("npz: unsupported compression method");
      std::vector<uint8_t> out(static_cast<size_t>(usize));
      z_stream zs{};
      if (inflateInit2(&zs, -MAX_WBITS) != Z_OK) throw std::runtime_error("npz: inflate init failed");
      zs.next_in = const_cast<Bytef*>(data + body);
      zs.avail_in = static_cast<uInt>(csize);
      zs.next_out = out.data();
      zs.avail_out = static_cast<uInt>(usize);
      const int rc = inflate(&zs, Z_FINISH);
      inflateEnd(&zs);
      if (rc != Z_STREAM_END || zs.total_out != usize) throw std::runtime_error("npz: inflate failed");
      return out;
    }
    o = body + csize;
  }
  throw std::runtime_error(name.empty() ? std::string("npz: no .npy member") : "npz: no member named " + want);
}

DepthMap process_depth(const std::vector<float>& src, int h, int w, const DepthLoaderConfig& cfg) {
  float lo = cfg.min_depth, hi = cfg.max_depth;
  if (lo == 0.f && hi == 0.f) {
    lo = std::numeric_limits<float>::infinity();
    hi = -lo;
    for (float v : src)
      if (std::isfinite(v)) {
        lo = std::min(lo, v);
        hi = std::max(hi, v);
      }
    if (!std::isfinite(lo)) lo = 0.f;
    if (!std::isfinite(hi)) hi = 1.f;
  }
  DepthMap m;
  m.original_min = lo;
  m.original_max = hi;
  const bool resize = cfg.target_width > 0 && cfg.target_height > 0 &&
                      (cfg.target_width != w || cfg.target_height != h);
  m.width = resize ? cfg.target_width : w;
  m.height = resize ? cfg.target_height : h;
  m.data.resize(static_cast<size_t>(m.width) * m.height);
  const float range = hi - lo;
  const float inv = range > 1e-8f ? 1.f / range : 1.f;
  const float rx = static_cast<float>(w) / m.width, ry = static_cast<float>(h) / m.height;
  for (int y = 0; y < m.height; ++y) {
    float fy = 0.f;
    int y0 = y, y1 = y;
    if (resize) {
      const float sy = y * ry;
      y0 = static_cast<int>(std::floor(sy));
      y1 = std::min(y0 + 1, h - 1);
      fy = sy - y0;
    }
    for (int x = 0; x < m.width; ++x) {
      float v;
      if (resize) {
        const float sx = x * rx;
        const int x0 = static_cast<int>(std::floor(sx));
        const int x1 = std::min(x0 + 1, w - 1);
        const float fx = sx - x0;
        const float a = src[static_cast<size_t>(y0) * w + x0] * (1 - fx) + src[static_cast<size_t>(y0) * w + x1] * fx;
        const float b = src[static_cast<size_t>(y1) * w + x0] * (1 - fx) + src[static_cast<size_t>(y1) * w + x1] * fx;
        v = a * (1 - fy) + b * fy;
      } else {
        v = src[static_cast<size_t>(y) * w + x];
      }
      float n = cfg.clip_depth ? (std::min(std::max(v, lo), hi) - lo) * inv : (v - lo) * inv;
      if (cfg.invert_depth) n = 1.f - n;
      m.data[static_cast<size_t>(y) * m.width + x] = n;
    }
  }
  return m;
}

DepthMap load_depth(const std::string& path, const DepthLoaderConfig& cfg) {
  const std::string e = ext_of(path);
  const auto bytes = read_all(path);
  int h = 0, w = 0;
  std::vector<float> raw;
  if (e == "npy") {
    raw = npy_to_float(bytes.data(), bytes.size(), &h, &w);
  } else if (e == "npz") {
    const auto member = npz_member(bytes.data(), bytes.size(), cfg.npz_array_name);
    raw = npy_to_float(member.data(), member.size(), &h, &w);
  } else if (e == "png") {
    const PngPixels p = decode_png_pixels(bytes.data(), bytes.size());
    h = p.h;
    w = p.w;
    raw.resize(static_cast<size_t>(h) * w);
    const size_t bps = p.depth / 8, bpp = bps * p.channels;
    for (size_t i = 0; i < raw.size(); ++i) {  // first channel (grey / red), 16-bit big-endian
      const uint8_t* q = &p.px[i * bpp];
      raw[i] = bps == 2 ? static_cast<float>((q[0] << 8) | q[1]) : static_cast<float>(q[0]);
    }
  } else if (e == "exr") {
    throw std::runtime_error("depth: EXR is not supported (convert to .npy / .npz / 16-bit PNG)");
  } else {
    throw std::runtime_error("depth: unsupported format ." + e);
  }
  return process_depth(raw, h, w, cfg);
}

void load_depth_batch(const std::vector<std::string>& paths, const DepthLoaderConfig& cfg, int threads,
                      float* out) {
  if (cfg.target_width <= 0 || cfg.target_height <= 0)
    throw std::runtime_error("depth batch: a target size is required");
  const size_t plane = static_cast<size_t>(cfg.target_width) * cfg.target_height;
  parallel_for(static_cast<int64_t>(paths.size()), threads, [&](int64_t i) {
    const DepthMap m = load_depth(paths[i], cfg);
    std::memcpy(out + i * plane, m.data.data(), plane * sizeof(float));
  });
}

}  // namespace ddd
