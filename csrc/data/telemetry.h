// Telemetry CSV -> column table; control normalisation to the 6-D DriveDiT format.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace ddd {

struct TelemetryField {
  std::string name;
  std::vector<std::string> aliases;  // lower-case header names, first match wins
};
const std::vector<TelemetryField>& telemetry_fields();

struct TelemetryTable {
  int64_t rows = 0;
  int64_t skipped = 0;
  std::vector<std::vector<double>> columns;  // one per telemetry_fields() entry
  std::vector<bool> present;                 // column found in the header
};

TelemetryTable parse_telemetry_text(const std::string& text);
TelemetryTable parse_telemetry_file(const std::string& path);
std::vector<TelemetryTable> parse_telemetry_files(const std::vector<std::string>& paths, int threads);

struct NormalizerConfig {
  double steering_lo = -1.0, steering_hi = 1.0;
  double brake_lo = 0.0, brake_hi = 1.0;
  double speed_lo = 0.0, speed_hi = 50.0;  // m/s
  double speed_scale = 1.0 / 3.6;          // speed column (km/h) -> m/s
};
// [rows x 6] row-major
std::vector<float> normalize_controls(const TelemetryTable& t, const NormalizerConfig& c);

}  // namespace ddd
