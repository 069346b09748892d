// Telemetry CSV parsing and control normalisation (native).
//
// Columns are found by case-insensitive header name with the same alias lists as the
// reference parser (rust/drivedit-data/src/telemetry.rs:353-520, e.g. latitude|lat,
// steering|steer|steering_angle, throttle|gas|accel); unparsable cells leave the field at
// its default and malformed rows are skipped. Output is column-major (one float64 vector
// per field) so Python receives each field as one tensor. Files parse in parallel.
//
// `normalize_controls` produces the 6-D DriveDiT control vector of the reference
// Python normaliser (data/enfusion_preprocessing.py:262-345): [steering in [-1,1],
// throttle - brake, brake in [0,1], forward-velocity or speed proxy, lateral velocity,
// speed in [0,1]].
#include "telemetry.h"

#include <algorithm>
#include <cctype>
#include <cstdlib>
#include <fstream>
#include <sstream>
#include <stdexcept>
#include <unordered_map>

#include "parallel.h"

namespace ddd {

const std::vector<TelemetryField>& telemetry_fields() {
  static const std::vector<TelemetryField> f = {
      {"timestamp_ms", {"timestamp_ms", "timestamp", "time_ms", "time"}},
      {"frame_id", {"frame_id", "frame", "id"}},
      {"latitude", {"latitude", "lat"}},
      {"longitude", {"longitude", "lng", "lon"}},
      {"altitude", {"altitude", "alt"}},
      {"heading", {"heading", "yaw", "bearing"}},
      {"pitch", {"pitch"}},
      {"roll", {"roll"}},
      {"speed_kmh", {"speed_kmh", "speed", "velocity_kmh"}},
      {"speed_ms", {"speed_ms", "velocity_ms"}},
      {"steering", {"steering", "steer", "steering_angle"}},
      {"throttle", {"throttle", "gas", "accel"}},
      {"brake", {"brake", "braking"}},
      {"clutch", {"clutch"}},
      {"gear", {"gear"}},
      {"engine_rpm", {"engine_rpm", "rpm"}},
      {"acceleration_x", {"acceleration_x", "accel_x", "ax"}},
      {"acceleration_y", {"acceleration_y", "accel_y", "ay"}},
      {"acceleration_z", {"acceleration_z", "accel_z", "az"}},
      {"yaw_rate", {"yaw_rate", "gyro_z"}},
      {"velocity_x", {"velocity_x", "vel_x", "vx"}},
      {"velocity_y", {"velocity_y", "vel_y", "vy"}},
  };
  return f;
}

namespace {

std::string lower_trim(const std::string& s) {
  size_t a = 0, b = s.size();
  while (a < b && std::isspace(static_cast<unsigned char>(s[a]))) ++a;
  while (b > a && std::isspace(static_cast<unsigned char>(s[b - 1]))) --b;
  std::string o = s.substr(a, b - a);
  for (auto& c : o) c = static_cast<char>(std::tolower(static_cast<unsigned char>(c)));
  return o;
}

void split_csv(const std::string& line, std::vector<std::string>& out) {
  out.clear();
  std::string cur;
  bool q = false;
  for (size_t i = 0; i < line.size(); ++i) {
    const char c = line[i];
    if (q) {
      if (c == '"' && i + 1 < line.size() && line[i + 1] == '"') {
        cur += '"';
        ++i;
      } else if (c == '"') {
        q = false;
      } else {
        cur += c;
      }
    } else if (c == '"') {
      q = true;
    } else if (c == ',') {
      out.push_back(cur);
      cur.clear();
    } else if (c != '\r') {
      cur += c;
    }
  }
  out.push_back(cur);
}

bool parse_num(const std::string& s, double& v) {
  const std::string t = lower_trim(s);
  if (t.empty()) return false;
  char* end = nullptr;
  v = std::strtod(t.c_str(), &end);
  return end != t.c_str() && *end == '\0';
}

}  // namespace

TelemetryTable parse_telemetry_text(const std::string& text) {
  const auto& fields = telemetry_fields();
  TelemetryTable t;
  t.columns.resize(fields.size());
  t.present.assign(fields.size(), false);
  std::istringstream in(text);
  std::string line;
  if (!std::getline(in, line)) return t;
  std::vector<std::string> cells;
  split_csv(line, cells);
  std::unordered_map<std::string, int> hdr;
  for (size_t i = 0; i < cells.size(); ++i) hdr.emplace(lower_trim(cells[i]), static_cast<int>(i));
  std::vector<int> col(fields.size(), -1);
  for (size_t f = 0; f < fields.size(); ++f) {
    for (const auto& alias : fields[f].aliases) {
      auto it = hdr.find(alias);
      if (it != hdr.end()) {
        col[f] = it->second;
        t.present[f] = true;
        break;
      }
    }
  }
  while (std::getline(in, line)) {
    if (line.empty() || line == "\r") continue;
    split_csv(line, cells);
    std::vector<double> row(fields.size(), 0.0);
    bool any = false;
    for (size_t f = 0; f < fields.size(); ++f) {
      if (col[f] < 0 || col[f] >= static_cast<int>(cells.size())) continue;
      double v;
      if (parse_num(cells[col[f]], v)) {
        row[f] = v;
        any = true;
      }
    }
    if (!any) {
      ++t.skipped;
      continue;
    }
    for (size_t f = 0; f < fields.size(); ++f) t.columns[f].push_back(row[f]);
    ++t.rows;
  }
  // derived: speed in m/s from km/h when not given
  const int kmh = 8, ms = 9;
  if (t.present[kmh] && !t.present[ms]) {
    for (int64_t r = 0; r < t.rows; ++r) t.columns[ms][r] = t.columns[kmh][r] / 3.6;
    t.present[ms] = true;
  }
  return t;
}

TelemetryTable parse_telemetry_file(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("telemetry: cannot open " + path);
  std::stringstream ss;
  ss << f.rdbuf();
  return parse_telemetry_text(ss.str());
}

std::vector<TelemetryTable> parse_telemetry_files(const std::vector<std::string>& paths, int threads) {
  std::vector<TelemetryTable> out(paths.size());
  parallel_for(static_cast<int64_t>(paths.size()), threads,
               [&](int64_t i) { out[i] = parse_telemetry_file(paths[i]); });
  return out;
}

namespace {
double to_range(double v, double lo, double hi, double olo, double ohi) {
  v = std::min(std::max(v, lo), hi);
  const double n = (hi - lo) > 1e-8 ? (v - lo) / (hi - lo) : 0.0;
  return n * (ohi - olo) + olo;
}
}  // namespace

std::vector<float> normalize_controls(const TelemetryTable& t, const NormalizerConfig& c) {
  const auto& fields = telemetry_fields();
  auto idx = [&](const char* name) {
    for (size_t i = 0; i < fields.size(); ++i)
      if (fields[i].name == name) return static_cast<int>(i);
    return -1;
  };
  const int st = idx("steering"), th = idx("throttle"), br = idx("brake"), sp = idx("speed_kmh"),
            spm = idx("speed_ms"), vx = idx("velocity_x"), vy = idx("velocity_y");
  const bool has_speed = t.present[sp] || t.present[spm];
  const int64_t T = t.rows;
  std::vector<float> out(static_cast<size_t>(T) * 6, 0.f);
  const bool has_vel = t.present[vx] && t.present[vy];
  for (int64_t r = 0; r < T; ++r) {
    float* o = &out[r * 6];
    const double steer = t.present[st] ? t.columns[st][r] : 0.0;
    const double thr = t.present[th] ? t.columns[th][r] : 0.0;
    const double brk = t.present[br] ? t.columns[br][r] : 0.0;
    // speed in m/s: the m/s column (derived from km/h by the parser when absent), else
    // the km/h column scaled by speed_scale
    const double spd = t.present[spm] ? t.columns[spm][r]
                                      : (t.present[sp] ? t.columns[sp][r] * c.speed_scale : 0.0);
    if (t.present[st]) o[0] = static_cast<float>(to_range(steer, c.steering_lo, c.steering_hi, -1, 1));
    o[1] = static_cast<float>(thr - brk);
    if (t.present[br]) o[2] = static_cast<float>(to_range(brk, c.brake_lo, c.brake_hi, 0, 1));
    if (has_vel) {
      o[3] = static_cast<float>(to_range(t.columns[vx][r], -c.speed_hi, c.speed_hi, -1, 1));
      o[4] = static_cast<float>(to_range(t.columns[vy][r], -0.5 * c.speed_hi, 0.5 * c.speed_hi, -1, 1));
    } else if (has_speed) {
      o[3] = static_cast<float>(to_range(spd, c.speed_lo, c.speed_hi, 0, 1));
    }
    if (has_speed) o[5] = static_cast<float>(to_range(spd, c.speed_lo, c.speed_hi, 0, 1));
  }
  return out;
}

}  // namespace ddd
