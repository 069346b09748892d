// Python bindings of the native data runtime (module drivedit_b200._data): ENFCAP
// reader/writer, telemetry CSV parsing + control normalisation, PNG frame loading.
// Heavy calls release the GIL; results are returned as torch tensors.
#include <torch/extension.h>

#include <memory>

#include "enfcap.h"
#include "depth.h"
#include "frames.h"
#include "service.h"
#include "telemetry.h"

namespace py = pybind11;

namespace {

template <class T>
torch::Tensor to_tensor(const std::vector<T>& v, torch::ScalarType st, std::vector<int64_t> shape) {
  auto t = torch::empty(shape, torch::TensorOptions().dtype(st));
  if (!v.empty()) std::memcpy(t.data_ptr(), v.data(), v.size() * sizeof(T));
  return t;
}

py::dict frame_dict(const ddd::Frame& f) {
  py::dict d;
  const int64_t ne = f.entities.size(), nr = f.road.size() / 3;
  std::vector<int32_t> et(ne);
  std::vector<float> ep(ne * 3);
  for (int64_t i = 0; i < ne; ++i) {
    et[i] = static_cast<int32_t>(f.entities[i].type);
    std::memcpy(&ep[i * 3], f.entities[i].pos, 12);
  }
  d["frame_id"] = f.frame_id;
  d["timestamp"] = f.timestamp;
  d["ego_transform"] = to_tensor(std::vector<float>(f.ego, f.ego + 12), torch::kFloat32, {3, 4});
  d["vehicle_state"] = to_tensor(std::vector<float>(f.vehicle, f.vehicle + 10), torch::kFloat32, {10});
  d["entity_type"] = to_tensor(et, torch::kInt32, {ne});
  d["entity_pos"] = to_tensor(ep, torch::kFloat32, {ne, 3});
  d["road_points"] = to_tensor(f.road, torch::kFloat32, {nr, 3});
  d["flags"] = f.flags;
  return d;
}

ddd::Frame frame_from(uint32_t frame_id, float timestamp, torch::Tensor ego, torch::Tensor vehicle,
                      torch::Tensor entity_type, torch::Tensor entity_pos, torch::Tensor road,
                      int flags) {
  ddd::Frame f;
  f.frame_id = frame_id;
  f.timestamp = timestamp;
  auto e = ego.to(torch::kFloat32).contiguous().view(-1);
  auto v = vehicle.to(torch::kFloat32).contiguous().view(-1);
  TORCH_CHECK(e.numel() == 12 && v.numel() == 10, "ego must have 12 values, vehicle 10");
  std::memcpy(f.ego, e.data_ptr<float>(), 48);
  std::memcpy(f.vehicle, v.data_ptr<float>(), 40);
  auto et = entity_type.to(torch::kInt64).contiguous().view(-1);
  auto ep = entity_pos.to(torch::kFloat32).contiguous().view({-1, 3});
  TORCH_CHECK(et.numel() == ep.size(0), "entity_type / entity_pos length mismatch");
  f.entities.resize(et.numel());
  for (int64_t i = 0; i < et.numel(); ++i) {
    f.entities[i].type = static_cast<uint32_t>(et[i].item<int64_t>());
    std::memcpy(f.entities[i].pos, ep.data_ptr<float>() + i * 3, 12);
  }
  auto rp = road.to(torch::kFloat32).contiguous().view(-1);
  TORCH_CHECK(rp.numel() % 3 == 0, "road points must be [n, 3]");
  f.road.assign(rp.data_ptr<float>(), rp.data_ptr<float>() + rp.numel());
  f.flags = static_cast<uint16_t>(flags);
  return f;
}

py::dict table_dict(const ddd::TelemetryTable& t) {
  py::dict d;
  const auto& fields = ddd::telemetry_fields();
  for (size_t i = 0; i < fields.size(); ++i)
    if (t.present[i]) d[py::str(fields[i].name)] = to_tensor(t.columns[i], torch::kFloat64, {t.rows});
  d["_rows"] = t.rows;
  d["_skipped"] = t.skipped;
  return d;
}

ddd::TelemetryTable table_from(const py::dict& d) {
  const auto& fields = ddd::telemetry_fields();
  ddd::TelemetryTable t;
  t.columns.resize(fields.size());
  t.present.assign(fields.size(), false);
  t.rows = -1;
  for (size_t i = 0; i < fields.size(); ++i) {
    if (!d.contains(fields[i].name)) continue;
    auto col = d[py::str(fields[i].name)].cast<torch::Tensor>().to(torch::kFloat64).contiguous().view(-1);
    if (t.rows < 0) t.rows = col.numel();
    TORCH_CHECK(col.numel() == t.rows, "telemetry columns differ in length");
    t.columns[i].assign(col.data_ptr<double>(), col.data_ptr<double>() + col.numel());
    t.present[i] = true;
  }
  if (t.rows < 0) t.rows = 0;
  return t;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "native data runtime: ENFCAP, telemetry, frames";
  py::class_<ddd::EnfcapReader, std::shared_ptr<ddd::EnfcapReader>>(m, "ENFCAPReader")
      .def(py::init<const std::string&>())
      .def_property_readonly("frame_count", &ddd::EnfcapReader::frame_count)
      .def_property_readonly("flags", &ddd::EnfcapReader::flags)
      .def_property_readonly("start_timestamp", &ddd::EnfcapReader::start_timestamp)
      .def_property_readonly("path", &ddd::EnfcapReader::path)
      .def("__len__", &ddd::EnfcapReader::frame_count)
      .def("read_frame", [](const ddd::EnfcapReader& r, uint32_t i) { return frame_dict(r.read_frame(i)); })
      .def("read_frames",
           [](const ddd::EnfcapReader& r, uint32_t start, uint32_t end, int threads) {
             ddd::FrameBatch b;
             {
               py::gil_scoped_release nogil;
               b = r.read_frames(start, end, threads);
             }
             const int64_t n = b.frame_id.size(), ne = b.entity_type.size(), nr = b.road.size() / 3;
             py::dict d;
             std::vector<int64_t> ids(b.frame_id.begin(), b.frame_id.end());
             std::vector<int32_t> fl(b.flags.begin(), b.flags.end());
             std::vector<int32_t> et(b.entity_type.begin(), b.entity_type.end());
             d["frame_id"] = to_tensor(ids, torch::kInt64, {n});
             d["timestamp"] = to_tensor(b.timestamp, torch::kFloat32, {n});
             d["ego_transform"] = to_tensor(b.ego, torch::kFloat32, {n, 3, 4});
             d["vehicle_state"] = to_tensor(b.vehicle, torch::kFloat32, {n, 10});
             d["flags"] = to_tensor(fl, torch::kInt32, {n});
             d["entity_offsets"] = to_tensor(b.entity_offsets, torch::kInt64, {n + 1});
             d["entity_type"] = to_tensor(et, torch::kInt32, {ne});
             d["entity_pos"] = to_tensor(b.entity_pos, torch::kFloat32, {ne, 3});
             d["road_offsets"] = to_tensor(b.road_offsets, torch::kInt64, {n + 1});
             d["road_points"] = to_tensor(b.road, torch::kFloat32, {nr, 3});
             return d;
           },
           py::arg("start"), py::arg("end"), py::arg("threads") = 0)
      .def("validate", &ddd::EnfcapReader::validate);
  py::class_<ddd::EnfcapWriter>(m, "ENFCAPWriter")
      .def(py::init<const std::string&, double, uint32_t>(), py::arg("path"),
           py::arg("start_timestamp") = 0.0, py::arg("flags") = 16u)
      .def("write_frame",
           [](ddd::EnfcapWriter& w, uint32_t frame_id, float timestamp, torch::Tensor ego,
              torch::Tensor vehicle, torch::Tensor entity_type, torch::Tensor entity_pos,
              torch::Tensor road, int flags) {
             w.write_frame(frame_from(frame_id, timestamp, ego, vehicle, entity_type, entity_pos, road, flags));
           },
           py::arg("frame_id"), py::arg("timestamp"), py::arg("ego_transform"), py::arg("vehicle_state"),
           py::arg("entity_type"), py::arg("entity_pos"), py::arg("road_points"), py::arg("flags") = 0)
      .def("finalize", &ddd::EnfcapWriter::finalize)
      .def_property_readonly("frames_written", &ddd::EnfcapWriter::frames_written);

  m.def("telemetry_fields", [] {
    std::vector<std::string> n;
    for (const auto& f : ddd::telemetry_fields()) n.push_back(f.name);
    return n;
  });
  m.def("parse_telemetry_text", [](const std::string& s) { return table_dict(ddd::parse_telemetry_text(s)); });
  m.def("parse_telemetry", [](const std::string& p) {
    ddd::TelemetryTable t;
    {
      py::gil_scoped_release nogil;
      t = ddd::parse_telemetry_file(p);
    }
    return table_dict(t);
  });
  m.def("parse_telemetry_files", [](const std::vector<std::string>& paths, int threads) {
    std::vector<ddd::TelemetryTable> ts;
    {
      py::gil_scoped_release nogil;
      ts = ddd::parse_telemetry_files(paths, threads);
    }
    py::list out;
    for (const auto& t : ts) out.append(table_dict(t));
    return out;
  }, py::arg("paths"), py::arg("threads") = 0);
  m.def("normalize_controls",
        [](const py::dict& table, std::pair<double, double> steering, std::pair<double, double> brake,
           std::pair<double, double> speed, double speed_scale) {
          ddd::NormalizerConfig c;
          c.steering_lo = steering.first;
          c.steering_hi = steering.second;
          c.brake_lo = brake.first;
          c.brake_hi = brake.second;
          c.speed_lo = speed.first;
          c.speed_hi = speed.second;
          c.speed_scale = speed_scale;
          const auto t = table_from(table);
          return to_tensor(ddd::normalize_controls(t, c), torch::kFloat32, {t.rows, 6});
        },
        py::arg("table"), py::arg("steering_range") = std::make_pair(-1.0, 1.0),
        py::arg("brake_range") = std::make_pair(0.0, 1.0), py::arg("speed_range") = std::make_pair(0.0, 50.0),
        py::arg("speed_scale") = 1.0 / 3.6);
  m.def("decode_png", [](py::bytes b) {
    const std::string s = b;
    const auto img = ddd::decode_png(reinterpret_cast<const uint8_t*>(s.data()), s.size());
    return to_tensor(img.rgb, torch::kUInt8, {img.h, img.w, 3});
  });
  m.def("load_frames",
        [](const std::vector<std::string>& paths, int H, int W, int threads) {
          auto out = torch::empty({static_cast<int64_t>(paths.size()), H, W, 3}, torch::kUInt8);
          uint8_t* p = out.data_ptr<uint8_t>();
          {
            py::gil_scoped_release nogil;
            ddd::load_frames(paths, H, W, threads, p);
          }
          return out;
        },
        py::arg("paths"), py::arg("height"), py::arg("width"), py::arg("threads") = 0);

  // ---- depth maps
  auto depth_cfg = [](int tw, int th, float mn, float mx, bool clip, bool inv, const std::string& name) {
    ddd::DepthLoaderConfig c;
    c.target_width = tw; c.target_height = th; c.min_depth = mn; c.max_depth = mx;
    c.clip_depth = clip; c.invert_depth = inv; c.npz_array_name = name;
    return c;
  };
  m.def("load_depth",
        [depth_cfg](const std::string& path, int tw, int th, float mn, float mx, bool clip, bool inv,
                    const std::string& name) {
          ddd::DepthMap dm;
          {
            py::gil_scoped_release nogil;
            dm = ddd::load_depth(path, depth_cfg(tw, th, mn, mx, clip, inv, name));
          }
          return py::make_tuple(to_tensor(dm.data, torch::kFloat32, {dm.height, dm.width}), dm.original_min,
                                dm.original_max);
        },
        py::arg("path"), py::arg("target_width") = 640, py::arg("target_height") = 360, py::arg("min_depth") = 0.f,
        py::arg("max_depth") = 0.f, py::arg("clip_depth") = true, py::arg("invert_depth") = false,
        py::arg("npz_array_name") = "depth");
  m.def("load_depth_batch",
        [depth_cfg](const std::vector<std::string>& paths, int tw, int th, float mn, float mx, bool clip, bool inv,
                    const std::string& name, int threads) {
          auto out = torch::empty({static_cast<int64_t>(paths.size()), th, tw}, torch::kFloat32);
          float* p = out.data_ptr<float>();
          {
            py::gil_scoped_release nogil;
            ddd::load_depth_batch(paths, depth_cfg(tw, th, mn, mx, clip, inv, name), threads, p);
          }
          return out;
        },
        py::arg("paths"), py::arg("target_width") = 640, py::arg("target_height") = 360, py::arg("min_depth") = 0.f,
        py::arg("max_depth") = 0.f, py::arg("clip_depth") = true, py::arg("invert_depth") = false,
        py::arg("npz_array_name") = "depth", py::arg("threads") = 0);

  // ---- background frame loading
  py::class_<ddd::FrameLoaderService, std::shared_ptr<ddd::FrameLoaderService>>(m, "FrameLoaderService")
      .def(py::init<int, size_t>(), py::arg("threads") = 0, py::arg("cache_frames") = 256)
      .def("submit",
           [](ddd::FrameLoaderService& s, const std::vector<std::string>& paths, int H, int W) {
             auto out = torch::empty({static_cast<int64_t>(paths.size()), H, W, 3}, torch::kUInt8);
             const int64_t id = s.submit(paths, H, W, out.data_ptr<uint8_t>());
             return py::make_tuple(id, out);
           })
      .def("wait", [](ddd::FrameLoaderService& s, int64_t id) {
             py::gil_scoped_release nogil;
             s.wait(id);
           })
      .def("done", &ddd::FrameLoaderService::done)
      .def("pending", &ddd::FrameLoaderService::pending)
      .def("cache_stats", [](ddd::FrameLoaderService& s) {
             return py::dict(py::arg("size") = s.cache().size(), py::arg("hits") = s.cache().hits(),
                             py::arg("misses") = s.cache().misses());
           })
      .def("clear_cache", [](ddd::FrameLoaderService& s) { s.cache().clear(); });
}
