// Benchmark runner with the reference runner's command line and JSON contract
// (reference src/runner/main.cpp: flags :119-155, case loading :157-184, correctness rule
// :324-365, JSON :373-418, timing protocol :508-535, exit codes :505/:540/:549), so that the
// reference's scripts/eval_kernel.py drives it unchanged.  Built twice:
//   custom_runner  -> backend = matmul_optimizer::launch_bf16_gemm_v1 (libmo_gemm.so)
//   cublas_runner  -> backend = cuBLASLt (cublas_runner.cpp), the same-box baseline
//
// Additions over the reference contract (ignored by eval_kernel.py unless passed through
// --extra-runner-arg):
//   --gpus G       N-shard C over devices 0..G-1: A replicated, B column slab of width
//                  roundup16(ceil(N/G)) per device, copied contiguously into that device's
//                  memory before timing; per-iteration time = max over devices.
//   --allgather    after the sharded GEMM, an NCCL all-gather of the C slabs and a local
//                  column re-layout on every device; timed and reported separately.
//   --verify-shards  (correctness mode, G > 1) also runs the 1-GPU GEMM on device 0 and
//                  reports whether every slab is bit-identical to its columns.

#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <iostream>
#include <memory>
#include <optional>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/runner_contract.h"
#include "runner_common.h"

#ifndef MO_RUNNER_CUBLAS
#include "../../include/kernel_api.h"
#include "../../include/mo_gemm.h"
namespace mo_runner {
bool backend_gemm(const std::uint16_t* a, const std::uint16_t* b, std::uint16_t* c, int m,
                  int n, int k, cudaStream_t stream) {
  return matmul_optimizer::launch_bf16_gemm_v1(a, b, c, m, n, k, stream);
}
bool backend_gemm_shards(int g, const int* devices, const std::uint16_t* const* a,
                         const std::uint16_t* const* b, std::uint16_t* const* c, int m, int k,
                         const int* widths, cudaStream_t const* streams) {
  std::vector<void*> s(streams, streams + g);
  return mo_gemm_nshard(g, devices, a, b, c, m, k, widths, s.data()) == MO_OK;
}
const char* backend_name() { return "mo_sm100"; }
}  // namespace mo_runner
#endif

namespace fs = std::filesystem;
using matmul_optimizer::CorrectnessSummary;
using matmul_optimizer::RunnerMode;
using matmul_optimizer::RuntimeSummary;

namespace {

[[noreturn]] void fail(const std::string& msg) { throw std::runtime_error(msg); }

void cuda_ok(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(std::string(what) + ": " + cudaGetErrorString(e));
}

void nccl_ok(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) fail(std::string(what) + ": " + ncclGetErrorString(r));
}

struct Options {
  fs::path dataset_dir;
  std::string case_id;
  RunnerMode mode = RunnerMode::kCorrectness;
  int warmup = 0;
  int iters = 1;
  int flush_mb = 0;
  std::optional<fs::path> json_out;
  int gpus = 1;
  bool allgather = false;
  bool verify_shards = false;
};

const char* mode_name(RunnerMode m) { return m == RunnerMode::kPerf ? "perf" : "correctness"; }

int to_int(const std::string& flag, const std::string& v) {
  try {
    size_t used = 0;
    const int x = std::stoi(v, &used);
    if (used != v.size()) throw std::invalid_argument(v);
    return x;
  } catch (const std::exception&) {
    fail("invalid integer for " + flag + ": " + v);
  }
}

Options parse_options(int argc, char** argv) {
  Options o;
  for (int i = 1; i < argc; ++i) {
    const std::string flag = argv[i];
    auto value = [&]() -> std::string {
      if (i + 1 >= argc) fail("missing value for " + flag);
      return argv[++i];
    };
    if (flag == "--dataset-dir") o.dataset_dir = value();
    else if (flag == "--case-id") o.case_id = value();
    else if (flag == "--mode") {
      const std::string v = value();
      if (v == "correctness") o.mode = RunnerMode::kCorrectness;
      else if (v == "perf") o.mode = RunnerMode::kPerf;
      else fail("unsupported --mode value: " + v);
    } else if (flag == "--warmup") o.warmup = to_int(flag, value());
    else if (flag == "--iters") o.iters = to_int(flag, value());
    else if (flag == "--flush-cache-mb") o.flush_mb = to_int(flag, value());
    else if (flag == "--json-out") o.json_out = fs::path(value());
    else if (flag == "--gpus") o.gpus = to_int(flag, value());
    else if (flag == "--allgather") o.allgather = true;
    else if (flag == "--verify-shards") o.verify_shards = true;
    else fail("unknown argument: " + flag);
  }
  if (o.dataset_dir.empty()) fail("--dataset-dir is required");
  if (o.case_id.empty()) fail("--case-id is required");
  if (o.warmup < 0) fail("--warmup must be >= 0");
  if (o.iters <= 0) fail("--iters must be > 0");
  if (o.flush_mb < 0) fail("--flush-cache-mb must be >= 0");
  if (o.gpus <= 0 || o.gpus > 64) fail("--gpus must be in 1..64");
  return o;
}

std::string slurp(const fs::path& p) {
  std::ifstream in(p);
  if (!in) fail("failed to open text file: " + p.string());
  std::stringstream ss;
  ss << in.rdbuf();
  return ss.str();
}

// Value text following "key": in a flat JSON document (the generator's meta/manifest files).
std::optional<std::string> json_scalar(const std::string& text, const std::string& key) {
  const std::string quoted = "\"" + key + "\"";
  size_t pos = text.find(quoted);
  if (pos == std::string::npos) return std::nullopt;
  pos = text.find(':', pos + quoted.size());
  if (pos == std::string::npos) return std::nullopt;
  const size_t begin = text.find_first_not_of(" \t\r\n", pos + 1);
  if (begin == std::string::npos) return std::nullopt;
  const size_t end = text.find_first_of(",}\r\n", begin);
  return text.substr(begin, end == std::string::npos ? std::string::npos : end - begin);
}

struct CaseFiles {
  fs::path dir;
  int m = 0, n = 0, k = 0;
  double atol = 0.15, rtol = 0.01;
};

CaseFiles load_case(const Options& o) {
  CaseFiles c;
  c.dir = o.dataset_dir / "cases" / o.case_id;
  if (!fs::exists(c.dir)) fail("case directory not found: " + c.dir.string());
  const fs::path meta = c.dir / "meta.json";
  if (!fs::exists(meta)) fail("case meta.json not found: " + meta.string());
  const std::string text = slurp(meta);
  auto dim = [&](const char* key) {
    const auto v = json_scalar(text, key);
    if (!v) fail(std::string("missing integer key in JSON: ") + key);
    return to_int(key, *v);
  };
  c.m = dim("m");
  c.n = dim("n");
  c.k = dim("k");
  const fs::path manifest = o.dataset_dir / "manifest.json";
  if (fs::exists(manifest)) {
    const std::string mt = slurp(manifest);
    if (auto v = json_scalar(mt, "initial_atol")) c.atol = std::stod(*v);
    if (auto v = json_scalar(mt, "initial_rtol")) c.rtol = std::stod(*v);
  }
  return c;
}

template <typename T>
std::vector<T> read_raw(const fs::path& p, size_t count) {
  if (!fs::exists(p)) fail("binary file not found: " + p.string());
  if (fs::file_size(p) != count * sizeof(T)) fail("unexpected binary size for " + p.string());
  std::vector<T> v(count);
  std::ifstream in(p, std::ios::binary);
  in.read(reinterpret_cast<char*>(v.data()), static_cast<std::streamsize>(count * sizeof(T)));
  if (!in) fail("failed to read binary file: " + p.string());
  return v;
}

float bf16_to_float(std::uint16_t b) {
  const std::uint32_t u = static_cast<std::uint32_t>(b) << 16;
  float f;
  std::memcpy(&f, &u, sizeof f);
  return f;
}

// The reference's pass rule (main.cpp:324-365): every element within atol + rtol*|ref|; a NaN
// output counts as a failure here.
CorrectnessSummary check_result(const std::vector<std::uint16_t>& out,
                                const std::vector<float>& ref32,
                                const std::vector<std::uint16_t>& ref16, double atol,
                                double rtol, bool* passed) {
  CorrectnessSummary s;
  s.atol = atol;
  s.rtol = rtol;
  s.bf16_exact_match = true;
  *passed = true;
  double sum = 0.0;
  for (size_t i = 0; i < out.size(); ++i) {
    const double o = bf16_to_float(out[i]);
    const double r = ref32[i];
    const double e = std::fabs(o - r);
    s.max_abs_err = std::max(s.max_abs_err, e);
    s.max_rel_err = std::max(s.max_rel_err, e / std::max(std::fabs(r), 1.0e-12));
    sum += e;
    // !(e <= tol) so that a NaN output fails (the reference's `e > tol` lets NaN pass).
    if (!(e <= atol + rtol * std::fabs(r))) *passed = false;
    if (out[i] != ref16[i]) s.bf16_exact_match = false;
  }
  s.mean_abs_err = out.empty() ? 0.0 : sum / static_cast<double>(out.size());
  return s;
}

double percentile(std::vector<float> v, double q) {
  std::sort(v.begin(), v.end());
  if (v.size() == 1) return v[0];
  const double pos = q * static_cast<double>(v.size() - 1);
  const size_t lo = static_cast<size_t>(std::floor(pos)), hi = static_cast<size_t>(std::ceil(pos));
  return v[lo] + (v[hi] - v[lo]) * (pos - static_cast<double>(lo));
}

RuntimeSummary summarize(const std::vector<float>& t) {
  if (t.empty()) fail("no runtimes recorded");
  RuntimeSummary r;
  r.p10_ms = percentile(t, 0.10);
  r.median_ms = percentile(t, 0.50);
  r.p90_ms = percentile(t, 0.90);
  return r;
}

std::string num(double v) {
  std::ostringstream s;
  s.precision(10);
  s << v;
  return s.str();
}

std::string escape(const std::string& in) {
  std::string out;
  for (char ch : in) {
    if (ch == '"' || ch == '\\') out += '\\';
    if (ch == '\n') {
      out += "\\n";
      continue;
    }
    out += ch;
  }
  return out;
}

void write_json(const Options& o, const std::string& body) {
  if (!o.json_out) return;
  if (o.json_out->has_parent_path()) fs::create_directories(o.json_out->parent_path());
  std::ofstream out(*o.json_out);
  if (!out) fail("failed to open JSON output: " + o.json_out->string());
  out << body;
  if (!out) fail("failed to write JSON output: " + o.json_out->string());
}

// RAII device buffer on a given device.
struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  int dev = 0;
  DevBuf(int device, size_t nbytes) : bytes(nbytes), dev(device) {
    if (nbytes == 0) return;
    cuda_ok(cudaSetDevice(device), "cudaSetDevice");
    cuda_ok(cudaMalloc(&p, nbytes), "cudaMalloc");
  }
  ~DevBuf() {
    if (p != nullptr) {
      cudaSetDevice(dev);
      cudaFree(p);
    }
  }
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  template <typename T>
  T* as() const {
    return static_cast<T*>(p);
  }
};

struct Shard {
  int dev = 0;
  int begin = 0, width = 0;
  std::unique_ptr<DevBuf> a, b, c, flush, gathered, full;
  cudaStream_t stream = nullptr;
  cudaEvent_t start = nullptr, stop = nullptr;
};

int run(const Options& o) {
  const CaseFiles cf = load_case(o);
  const int m = cf.m, n = cf.n, k = cf.k;
  int device_count = 0;
  cuda_ok(cudaGetDeviceCount(&device_count), "cudaGetDeviceCount");
  if (o.gpus > device_count) fail("--gpus exceeds the visible device count");
  const int g = o.gpus;

  const size_t a_elems = static_cast<size_t>(m) * k;
  std::vector<std::uint16_t> a_host = read_raw<std::uint16_t>(cf.dir / "A.bf16.bin", a_elems);
  std::vector<std::uint16_t> b_host =
      read_raw<std::uint16_t>(cf.dir / "B.bf16.bin", static_cast<size_t>(k) * n);

  // Column partition: w = roundup16(ceil(n/g)).
  const int w = g == 1 ? n : ((n + g - 1) / g + 15) / 16 * 16;
  std::vector<Shard> shards(g);
  for (int i = 0; i < g; ++i) {
    Shard& s = shards[i];
    s.dev = i;
    s.begin = std::min(n, i * w);
    s.width = std::max(0, std::min(w, n - i * w));
    cuda_ok(cudaSetDevice(i), "cudaSetDevice");
    cuda_ok(cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking), "cudaStreamCreate");
    cuda_ok(cudaEventCreate(&s.start), "cudaEventCreate");
    cuda_ok(cudaEventCreate(&s.stop), "cudaEventCreate");
    s.a = std::make_unique<DevBuf>(i, a_elems * 2);
    s.b = std::make_unique<DevBuf>(i, static_cast<size_t>(k) * std::max(1, s.width) * 2);
    s.c = std::make_unique<DevBuf>(i, static_cast<size_t>(m) * w * 2);
    s.flush = std::make_unique<DevBuf>(i, static_cast<size_t>(o.flush_mb) << 20);
    cuda_ok(cudaMemcpy(s.a->p, a_host.data(), a_elems * 2, cudaMemcpyHostToDevice), "H2D A");
    if (s.width > 0) {
      // B slab [k, width] copied contiguously into this device's own memory.
      cuda_ok(cudaMemcpy2D(s.b->p, static_cast<size_t>(s.width) * 2, b_host.data() + s.begin,
                           static_cast<size_t>(n) * 2, static_cast<size_t>(s.width) * 2, k,
                           cudaMemcpyHostToDevice),
              "H2D B slab");
    }
  }
  std::vector<std::uint16_t>().swap(a_host);

  // Correctness runs and warm-up issue every slab in one multi-device call (mo_gemm_nshard for
  // custom_runner).  The timed loop below launches slab by slab instead, so that each device's
  // events bracket only its own launch and not the host time spent issuing the others.
  auto launch_all = [&]() {
    std::vector<int> devs(g), widths(g);
    std::vector<const std::uint16_t*> as(g), bs(g);
    std::vector<std::uint16_t*> cs(g);
    std::vector<cudaStream_t> streams(g);
    for (int i = 0; i < g; ++i) {
      const Shard& s = shards[i];
      devs[i] = s.dev;
      widths[i] = s.width;
      as[i] = s.a->as<std::uint16_t>();
      bs[i] = s.b->as<std::uint16_t>();
      cs[i] = s.c->as<std::uint16_t>();
      streams[i] = s.stream;
    }
    if (!mo_runner::backend_gemm_shards(g, devs.data(), as.data(), bs.data(), cs.data(), m, k,
                                        widths.data(), streams.data())) {
      fail("launch_bf16_gemm_v1 failed");
    }
  };
  auto sync_all = [&]() {
    for (Shard& s : shards) {
      cuda_ok(cudaSetDevice(s.dev), "cudaSetDevice");
      cuda_ok(cudaStreamSynchronize(s.stream), "cudaStreamSynchronize");
    }
  };
  auto flush_all = [&](int salt) {
    for (Shard& s : shards) {
      if (s.flush->bytes == 0) continue;
      cuda_ok(cudaSetDevice(s.dev), "cudaSetDevice");
      cuda_ok(cudaMemsetAsync(s.flush->p, salt & 0xFF, s.flush->bytes, s.stream), "cache flush");
    }
    sync_all();
  };

  // Optional NCCL all-gather of the C slabs (each padded to m*w elements) + re-layout.
  std::vector<ncclComm_t> comms;
  if (o.allgather && g > 1) {
    comms.resize(g);
    std::vector<int> devs(g);
    for (int i = 0; i < g; ++i) devs[i] = i;
    nccl_ok(ncclCommInitAll(comms.data(), g, devs.data()), "ncclCommInitAll");
    for (Shard& s : shards) {
      s.gathered = std::make_unique<DevBuf>(s.dev, static_cast<size_t>(g) * m * w * 2);
      s.full = std::make_unique<DevBuf>(s.dev, static_cast<size_t>(m) * n * 2);
    }
  }
  auto allgather_all = [&]() {
    nccl_ok(ncclGroupStart(), "ncclGroupStart");
    for (int i = 0; i < g; ++i) {
      Shard& s = shards[i];
      nccl_ok(ncclAllGather(s.c->p, s.gathered->p, static_cast<size_t>(m) * w * 2, ncclUint8,
                            comms[i], s.stream),
              "ncclAllGather");
    }
    nccl_ok(ncclGroupEnd(), "ncclGroupEnd");
    for (Shard& s : shards) {
      cuda_ok(cudaSetDevice(s.dev), "cudaSetDevice");
      for (const Shard& src : shards) {
        if (src.width == 0) continue;
        cuda_ok(cudaMemcpy2DAsync(s.full->as<std::uint16_t>() + src.begin,
                                  static_cast<size_t>(n) * 2,
                                  s.gathered->as<std::uint16_t>() +
                                      static_cast<size_t>(src.dev) * m * w,
                                  static_cast<size_t>(src.width) * 2,
                                  static_cast<size_t>(src.width) * 2, m,
                                  cudaMemcpyDeviceToDevice, s.stream),
                "re-layout copy");
      }
    }
  };

  std::ostringstream extra;
  extra << ",\n  \"backend\": \"" << mo_runner::backend_name() << "\",\n  \"n_gpus\": " << g
        << ",\n  \"shape\": [" << m << ", " << n << ", " << k << "]";

  if (o.mode == RunnerMode::kCorrectness) {
    launch_all();
    sync_all();
    std::vector<std::uint16_t> out(static_cast<size_t>(m) * n);
    if (o.allgather && g > 1) {
      allgather_all();
      sync_all();
      cuda_ok(cudaSetDevice(g - 1), "cudaSetDevice");
      cuda_ok(cudaMemcpy(out.data(), shards[g - 1].full->p, out.size() * 2, cudaMemcpyDeviceToHost),
              "D2H gathered C");
    } else {
      for (Shard& s : shards) {
        if (s.width == 0) continue;
        cuda_ok(cudaSetDevice(s.dev), "cudaSetDevice");
        cuda_ok(cudaMemcpy2D(out.data() + s.begin, static_cast<size_t>(n) * 2, s.c->p,
                             static_cast<size_t>(s.width) * 2, static_cast<size_t>(s.width) * 2,
                             m, cudaMemcpyDeviceToHost),
                "D2H C slab");
      }
    }
    if (o.verify_shards && g > 1) {
      // 1-GPU run on device 0 with the full B: every slab must match bit for bit.
      DevBuf full_b(0, static_cast<size_t>(k) * n * 2), full_c(0, static_cast<size_t>(m) * n * 2);
      cuda_ok(cudaMemcpy(full_b.p, b_host.data(), full_b.bytes, cudaMemcpyHostToDevice), "H2D B");
      if (!mo_runner::backend_gemm(shards[0].a->as<std::uint16_t>(), full_b.as<std::uint16_t>(),
                                   full_c.as<std::uint16_t>(), m, n, k, shards[0].stream)) {
        fail("launch_bf16_gemm_v1 failed (1-GPU reference run)");
      }
      cuda_ok(cudaStreamSynchronize(shards[0].stream), "sync");
      std::vector<std::uint16_t> single(static_cast<size_t>(m) * n);
      cuda_ok(cudaMemcpy(single.data(), full_c.p, single.size() * 2, cudaMemcpyDeviceToHost), "D2H");
      extra << ",\n  \"shards_bit_identical\": " << (single == out ? "true" : "false");
    }
    std::vector<std::uint16_t>().swap(b_host);
    const auto ref32 = read_raw<float>(cf.dir / "C_ref_fp32.bin", out.size());
    const auto ref16 = read_raw<std::uint16_t>(cf.dir / "C_ref_bf16.bin", out.size());
    bool passed = false;
    const CorrectnessSummary cs = check_result(out, ref32, ref16, cf.atol, cf.rtol, &passed);
    std::ostringstream js;
    js << "{\n  \"mode\": \"correctness\",\n  \"passed\": " << (passed ? "true" : "false")
       << ",\n  \"correctness\": {\n    \"max_abs_err\": " << num(cs.max_abs_err)
       << ",\n    \"max_rel_err\": " << num(cs.max_rel_err) << ",\n    \"mean_abs_err\": "
       << num(cs.mean_abs_err) << ",\n    \"bf16_exact_match\": "
       << (cs.bf16_exact_match ? "true" : "false") << ",\n    \"atol\": " << num(cs.atol)
       << ",\n    \"rtol\": " << num(cs.rtol) << "\n  }" << extra.str() << "\n}\n";
    write_json(o, js.str());
    return passed ? 0 : 1;
  }
  std::vector<std::uint16_t>().swap(b_host);

  for (int i = 0; i < o.warmup; ++i) {
    flush_all(i);
    launch_all();
  }
  sync_all();

  std::vector<float> times, gather_times;
  std::vector<std::vector<float>> per_gpu(g);
  for (int it = 0; it < o.iters; ++it) {
    flush_all(it + o.warmup);
    // Events bracket each device's own launch, so the host issuing the devices one after the
    // other does not count toward any device's time.
    for (Shard& s : shards) {
      if (s.width == 0) continue;
      cuda_ok(cudaSetDevice(s.dev), "cudaSetDevice");
      cuda_ok(cudaEventRecord(s.start, s.stream), "cudaEventRecord");
      if (!mo_runner::backend_gemm(s.a->as<std::uint16_t>(), s.b->as<std::uint16_t>(),
                                   s.c->as<std::uint16_t>(), m, s.width, k, s.stream)) {
        fail("launch_bf16_gemm_v1 failed");
      }
      cuda_ok(cudaEventRecord(s.stop, s.stream), "cudaEventRecord");
    }
    float worst = 0.0f;
    for (int i = 0; i < g; ++i) {
      Shard& s = shards[i];
      if (s.width == 0) continue;
      cuda_ok(cudaSetDevice(s.dev), "cudaSetDevice");
      cuda_ok(cudaEventSynchronize(s.stop), "cudaEventSynchronize");
      float ms = 0.0f;
      cuda_ok(cudaEventElapsedTime(&ms, s.start, s.stop), "cudaEventElapsedTime");
      per_gpu[i].push_back(ms);
      worst = std::max(worst, ms);
    }
    times.push_back(worst);
    if (o.allgather && g > 1) {
      for (Shard& s : shards) {
        cuda_ok(cudaSetDevice(s.dev), "cudaSetDevice");
        cuda_ok(cudaEventRecord(s.start, s.stream), "cudaEventRecord");
      }
      allgather_all();
      float gworst = 0.0f;
      for (Shard& s : shards) {
        cuda_ok(cudaSetDevice(s.dev), "cudaSetDevice");
        cuda_ok(cudaEventRecord(s.stop, s.stream), "cudaEventRecord");
      }
      for (Shard& s : shards) {
        cuda_ok(cudaSetDevice(s.dev), "cudaSetDevice");
        cuda_ok(cudaEventSynchronize(s.stop), "cudaEventSynchronize");
        float ms = 0.0f;
        cuda_ok(cudaEventElapsedTime(&ms, s.start, s.stop), "cudaEventElapsedTime");
        gworst = std::max(gworst, ms);
      }
      gather_times.push_back(gworst);
    }
  }
  const RuntimeSummary rs = summarize(times);
  const double tflops = 2.0 * m * static_cast<double>(n) * k / (rs.median_ms * 1.0e9);
  std::ostringstream js;
  js << "{\n  \"mode\": \"perf\",\n  \"passed\": true,\n  \"runtime_ms\": {\n    \"median\": "
     << num(rs.median_ms) << ",\n    \"p10\": " << num(rs.p10_ms) << ",\n    \"p90\": "
     << num(rs.p90_ms) << "\n  },\n  \"tflops\": " << num(tflops) << extra.str();
  js << ",\n  \"per_gpu_median_ms\": [";
  for (int i = 0; i < g; ++i) js << (i ? ", " : "") << num(percentile(per_gpu[i], 0.5));
  js << "]";
  if (!gather_times.empty()) {
    js << ",\n  \"allgather_ms\": {\"median\": " << num(percentile(gather_times, 0.5))
       << ", \"p10\": " << num(percentile(gather_times, 0.1))
       << ", \"p90\": " << num(percentile(gather_times, 0.9)) << "}";
  }
  js << "\n}\n";
  write_json(o, js.str());

  for (auto& c : comms) ncclCommDestroy(c);
  for (Shard& s : shards) {
    cudaSetDevice(s.dev);
    cudaEventDestroy(s.start);
    cudaEventDestroy(s.stop);
    cudaStreamDestroy(s.stream);
  }
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  std::optional<Options> opts;
  try {
    opts = parse_options(argc, argv);
    return run(*opts);
  } catch (const std::exception& ex) {
    std::cerr << "[runner-error] " << ex.what() << '\n';
    if (opts) {
      try {
        write_json(*opts, std::string("{\n  \"mode\": \"") + mode_name(opts->mode) +
                              "\",\n  \"passed\": false,\n  \"error\": \"" + escape(ex.what()) +
                              "\"\n}\n");
      } catch (...) {
      }
    }
    return 1;
  }
}
