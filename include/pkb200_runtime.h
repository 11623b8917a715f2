/* pkb200_runtime.h - C++ runtime over libpkb200: detect -> select -> load -> serve.
 *
 * The B200 counterpart of the reference's lib/Runtime (include/PolyKernel/
 * Runtime/Runtime.h, KernelCache.h, DeviceDetect.h), header-only C++17:
 *
 *   DeviceDetector  detects the device arch ("sm_100" on B200). The detector is
 *                   injected, so the whole flow is testable without a GPU
 *                   (FixedArchDetector), as the reference's runtime tests do.
 *   KernelCache     tuning-cache entries in the reference's tuning/schema.json
 *                   format (version 1), partitioned by gpu. Select serves only
 *                   validated entries; a miss or an unvalidated entry is a clear
 *                   error, never a wrong kernel (KernelCache.cpp:83-100). Loads are
 *                   all-or-nothing. Persist/LoadPersisted write and read
 *                   tuning_db.json + binaries.json in a cache directory; binaries
 *                   whose file hash changed are invalidated (KernelCache.h:80-131).
 *   Runtime         per-op launcher registry; Run = Resolve (detect + select) +
 *                   the registered launcher, with typed errors for every failure
 *                   (Runtime.cpp:20-57).
 *   RegisterLibraryLaunchers  the launchers that serve this library's GEMM ops
 *                   with the selected entry's tile config (block_n x stages).
 *
 * Error texts keep the reference's wording ("no tuned kernel for <key>; run the
 * autotuner ...") so callers that match on them keep working.
 */
#pragma once

#include <sys/stat.h>

#include <cerrno>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <functional>
#include <map>
#include <mutex>
#include <optional>
#include <sstream>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

#include "../polykernel_b200/csrc/tuning.h"
#include "pkb200.h"

#ifdef PKB200_RUNTIME_CUDA
#include <cuda_runtime_api.h>
#endif

namespace pkb200 {
namespace runtime {

// ------------------------------------------------------------------ device --
struct DeviceInfo {
  std::string arch;  // "sm_100"
  std::string name;
  bool operator==(const DeviceInfo& o) const { return arch == o.arch && name == o.name; }
};

class DeviceDetector {
 public:
  virtual ~DeviceDetector() = default;
  // std::nullopt when there is no usable device.
  virtual std::optional<DeviceInfo> Detect(int ordinal = 0) const = 0;
};

inline std::string SmArchFromComputeCapability(int major, int minor) {
  return "sm_" + std::to_string(major) + std::to_string(minor);
}

// Returns the injected arch for every ordinal (tests, offline cache tools).
class FixedArchDetector final : public DeviceDetector {
 public:
  explicit FixedArchDetector(std::string arch, std::string name = "mock-device")
      : arch_(std::move(arch)), name_(std::move(name)) {}
  std::optional<DeviceInfo> Detect(int = 0) const override { return DeviceInfo{arch_, name_}; }

 private:
  std::string arch_, name_;
};

// The arch of the current device as libpkb200 reports it (pkb200_device_arch).
class LibraryDeviceDetector final : public DeviceDetector {
 public:
  std::optional<DeviceInfo> Detect(int = 0) const override {
    char buf[32] = {};
    if (pkb200_device_arch(buf, sizeof(buf)) != 0 || buf[0] == 0) return std::nullopt;
    return DeviceInfo{buf, "cuda device"};
  }
};

#ifdef PKB200_RUNTIME_CUDA
class CudaDeviceDetector final : public DeviceDetector {
 public:
  std::optional<DeviceInfo> Detect(int ordinal = 0) const override {
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, ordinal) != cudaSuccess) return std::nullopt;
    return DeviceInfo{SmArchFromComputeCapability(prop.major, prop.minor), prop.name};
  }
};
#endif

// ------------------------------------------------------------------- cache --
using CacheEntry = tuning::Entry;

struct Shape {
  long long m = 0, n = 0, k = 0;
  std::string dtype = "bf16";
};

inline std::string FormatKey(std::string_view gpu, std::string_view op, const Shape& s) {
  return std::string(gpu) + "/" + std::string(op) + "/M=" + std::to_string(s.m) +
         ",N=" + std::to_string(s.n) + ",K=" + std::to_string(s.k) + "," + s.dtype;
}

inline Shape ShapeOf(const CacheEntry& e) { return Shape{e.M, e.N, e.K, e.dtype}; }

struct SelectionResult {
  std::optional<CacheEntry> entry;
  std::string error;
  bool ok() const { return entry.has_value(); }
};

struct CachedBinary {
  std::string so_path;      // compiled library backing the entry
  std::string kernel_hash;  // its file hash when it was recorded
  bool operator==(const CachedBinary& o) const {
    return so_path == o.so_path && kernel_hash == o.kernel_hash;
  }
};

// 64-bit FNV-1a over the file's bytes, as 16 hex digits.
inline bool HashFile(std::string_view path, std::string& hash_out, std::string& error) {
  std::ifstream f{std::string(path), std::ios::binary};
  if (!f) {
    error = "cannot read binary " + std::string(path) + ": " + std::strerror(errno);
    return false;
  }
  uint64_t h = 0xcbf29ce484222325ULL;
  char buf[1 << 16];
  while (f) {
    f.read(buf, sizeof(buf));
    for (std::streamsize i = 0; i < f.gcount(); ++i) {
      h ^= static_cast<unsigned char>(buf[i]);
      h *= 0x100000001b3ULL;
    }
  }
  char hex[17];
  std::snprintf(hex, sizeof(hex), "%016llx", static_cast<unsigned long long>(h));
  hash_out = hex;
  return true;
}

class KernelCache {
 public:
  static constexpr const char* kTuningFile = "/tuning_db.json";
  static constexpr const char* kBinariesFile = "/binaries.json";

  // Replace the cache with a tuning-cache document; on any schema error the
  // cache is left unchanged and `error` names the offending field.
  bool LoadTuningCache(std::string_view json, std::string& error) {
    std::vector<CacheEntry> parsed;
    if (!tuning::parse_cache(std::string(json), parsed, error)) return false;
    std::map<std::string, CacheEntry> next;
    for (auto& e : parsed) next[FormatKey(e.gpu, e.op, ShapeOf(e))] = e;
    entries_ = std::move(next);
    binaries_.clear();
    return true;
  }

  // Add (or replace) one entry; an entry without a gpu is refused.
  bool Put(CacheEntry e) {
    if (e.gpu.empty()) return false;
    const std::string key = FormatKey(e.gpu, e.op, ShapeOf(e));
    entries_[key] = std::move(e);
    return true;
  }

  SelectionResult Select(std::string_view gpu, std::string_view op, const Shape& shape) const {
    SelectionResult r;
    const std::string key = FormatKey(gpu, op, shape);
    auto it = entries_.find(key);
    if (it == entries_.end()) {
      r.error = "no tuned kernel for " + key +
                "; run the autotuner (polykernel_b200.tuning.autotune) to populate the cache";
      return r;
    }
    if (!it->second.validated) {
      r.error = "cached entry for " + key +
                " is not validated; run the autotuner to produce a correctness-gated variant";
      return r;
    }
    r.entry = it->second;
    return r;
  }

  std::vector<std::pair<std::string, SelectionResult>> SelectPerGpu(
      const std::vector<std::string>& gpus, std::string_view op, const Shape& shape) const {
    std::vector<std::pair<std::string, SelectionResult>> out;
    for (const auto& g : gpus) out.emplace_back(g, Select(g, op, shape));
    return out;
  }

  size_t Size() const { return entries_.size(); }

  // Record the compiled library behind an existing entry.
  bool PutBinary(std::string_view gpu, std::string_view op, const Shape& shape, CachedBinary b) {
    const std::string key = FormatKey(gpu, op, shape);
    if (gpu.empty() || !entries_.count(key)) return false;
    binaries_[key] = std::move(b);
    return true;
  }

  std::optional<CachedBinary> GetBinary(std::string_view gpu, std::string_view op,
                                        const Shape& shape) const {
    auto it = binaries_.find(FormatKey(gpu, op, shape));
    if (it == binaries_.end()) return std::nullopt;
    return it->second;
  }

  std::string SerializeTuning() const {
    std::vector<CacheEntry> v;
    for (const auto& kv : entries_) v.push_back(kv.second);
    return tuning::serialize_cache(v);
  }

  std::string SerializeBinaries() const {
    std::string o = "{\n  \"version\": 1,\n  \"binaries\": [";
    bool first = true;
    for (const auto& kv : binaries_) {
      const CacheEntry& e = entries_.at(kv.first);
      o += first ? "\n    {" : ",\n    {";
      first = false;
      o += "\"gpu\": " + tuning::json_string(e.gpu) + ", \"op\": " + tuning::json_string(e.op) +
           ", \"shape\": " + tuning::shape_json(e) + ", \"so_path\": " +
           tuning::json_string(kv.second.so_path) + ", \"kernel_hash\": " +
           tuning::json_string(kv.second.kernel_hash) + "}";
    }
    o += first ? "]\n}\n" : "\n  ]\n}\n";
    return o;
  }

  // Write tuning_db.json + binaries.json into `dir` (created if absent).
  bool Persist(std::string_view dir, std::string& error) const {
    const std::string d(dir);
    if (::mkdir(d.c_str(), 0755) != 0 && errno != EEXIST) {
      error = "cannot create cache dir " + d + ": " + std::strerror(errno);
      return false;
    }
    return WriteFile(d + kTuningFile, SerializeTuning(), error) &&
           WriteFile(d + kBinariesFile, SerializeBinaries(), error);
  }

  // Inverse of Persist. All-or-nothing: any unreadable file, schema error, or
  // binary record without a tuning entry leaves the cache unchanged.
  bool LoadPersisted(std::string_view dir, std::string& error) {
    const std::string d(dir);
    std::string tj, bj;
    if (!ReadFile(d + kTuningFile, tj, error) || !ReadFile(d + kBinariesFile, bj, error))
      return false;
    KernelCache next;
    if (!next.LoadTuningCache(tj, error)) {
      error = "tuning_db.json: " + error;
      return false;
    }
    if (!next.ParseBinaries(bj, error)) {
      error = "binaries.json: " + error;
      return false;
    }
    *this = std::move(next);
    return true;
  }

  // Drop every entry whose recorded binary is missing or no longer hashes to
  // the recorded value, so Select falls back to the miss. Returns the count.
  size_t InvalidateStale() {
    std::vector<std::string> stale;
    for (const auto& kv : binaries_) {
      std::string h, err;
      if (!HashFile(kv.second.so_path, h, err) || h != kv.second.kernel_hash)
        stale.push_back(kv.first);
    }
    for (const auto& k : stale) {
      binaries_.erase(k);
      entries_.erase(k);
    }
    return stale.size();
  }

 private:
  std::map<std::string, CacheEntry> entries_;   // keyed by FormatKey
  std::map<std::string, CachedBinary> binaries_;

  static bool WriteFile(const std::string& path, const std::string& text, std::string& error) {
    std::ofstream f(path, std::ios::binary | std::ios::trunc);
    if (!f || !(f << text) || !f.flush()) {
      error = "cannot write " + path;
      return false;
    }
    return true;
  }

  static bool ReadFile(const std::string& path, std::string& out, std::string& error) {
    std::ifstream f(path, std::ios::binary);
    if (!f) {
      error = "cannot read " + path + ": " + std::strerror(errno);
      return false;
    }
    std::ostringstream ss;
    ss << f.rdbuf();
    out = ss.str();
    return true;
  }

  bool ParseBinaries(const std::string& text, std::string& error) {
    using tuning::Json;
    Json root;
    if (!tuning::Parser(text).parse(root, error)) return false;
    if (!tuning::expect_keys(root, {"version", "binaries"}, "root", error)) return false;
    long long version = 0;
    if (!tuning::get_int(root, "version", version, "root", error)) return false;
    if (version != 1) {
      error = "root.version: unsupported binaries version " + std::to_string(version) +
              " (expected 1)";
      return false;
    }
    const Json* arr = root.get("binaries");
    if (arr->kind != Json::Arr) {
      error = "root.binaries: expected an array";
      return false;
    }
    for (size_t i = 0; i < arr->arr.size(); ++i) {
      const Json& o = arr->arr[i];
      const std::string w = "binaries[" + std::to_string(i) + "]";
      if (!tuning::expect_keys(o, {"gpu", "op", "shape", "so_path", "kernel_hash"}, w, error))
        return false;
      std::string gpu, op, so, hash;
      Shape s;
      if (!tuning::get_str(o, "gpu", gpu, w, error) || !tuning::get_str(o, "op", op, w, error) ||
          !tuning::get_str(o, "so_path", so, w, error) ||
          !tuning::get_str(o, "kernel_hash", hash, w, error))
        return false;
      const Json& sh = *o.get("shape");
      if (!tuning::expect_keys(sh, {"M", "N", "K", "dtype"}, w + ".shape", error) ||
          !tuning::get_int(sh, "M", s.m, w + ".shape", error) ||
          !tuning::get_int(sh, "N", s.n, w + ".shape", error) ||
          !tuning::get_int(sh, "K", s.k, w + ".shape", error) ||
          !tuning::get_str(sh, "dtype", s.dtype, w + ".shape", error))
        return false;
      if (!PutBinary(gpu, op, s, CachedBinary{so, hash})) {
        error = w + ": no tuning entry for " + FormatKey(gpu, op, s);
        return false;
      }
    }
    return true;
  }
};

// ----------------------------------------------------------------- runtime --
using LaunchFn = std::function<bool(const CacheEntry& entry, void* io, std::string& error)>;

struct ResolveResult {
  std::optional<DeviceInfo> device;
  std::optional<CacheEntry> entry;
  std::string error;
  bool ok() const { return entry.has_value(); }
};

class Runtime {
 public:
  Runtime(const DeviceDetector& detector, const KernelCache& cache)
      : detector_(detector), cache_(cache) {}

  // The launcher that serves `op` (last registration wins).
  void RegisterLauncher(std::string op, LaunchFn fn) { launchers_[std::move(op)] = std::move(fn); }

  // Detect + select, no launch.
  ResolveResult Resolve(std::string_view op, const Shape& shape) const {
    ResolveResult r;
    r.device = detector_.Detect();
    if (!r.device) {
      r.error = "device detection failed; no usable GPU to serve op " + std::string(op);
      return r;
    }
    SelectionResult s = cache_.Select(r.device->arch, op, shape);
    if (!s.ok()) {
      r.error = std::move(s.error);
      return r;
    }
    r.entry = std::move(s.entry);
    return r;
  }

  // Detect -> select -> load (the registered launcher) -> serve.
  bool Run(std::string_view op, const Shape& shape, void* io, std::string& error) {
    ResolveResult r = Resolve(op, shape);
    if (!r.ok()) {
      error = std::move(r.error);
      return false;
    }
    auto it = launchers_.find(std::string(op));
    if (it == launchers_.end()) {
      error = "no compiled launcher registered for op " + std::string(op) +
              "; load the compiled variant (register its launch entry) first";
      return false;
    }
    return it->second(*r.entry, io, error);
  }

 private:
  const DeviceDetector& detector_;
  const KernelCache& cache_;
  std::map<std::string, LaunchFn> launchers_;
};

// ------------------------------------------------- this library's launchers --
// I/O bundle of the GEMM-family launchers (bf16 device pointers; the shape
// comes from the selected entry: A [M,K], B [K,N], out [M,N]).
struct GemmIO {
  const void* a = nullptr;
  const void* b = nullptr;
  const void* bias = nullptr;   // fused_matmul_bias_gelu, matmul_bias_residual
  const void* resid = nullptr;  // matmul_bias_residual
  const void* gamma = nullptr;  // fused_rmsnorm_matmul (optional)
  void* out = nullptr;
  float eps = 1e-5f;
  void* stream = nullptr;
};

// Serve matmul, fused_rmsnorm_matmul, fused_matmul_bias_gelu and
// matmul_bias_residual with the entry's tile config. The library's forced
// config is process-wide, so launches through these launchers are serialised.
inline void RegisterLibraryLaunchers(Runtime& rt) {
  static std::mutex mu;
  auto make = [](std::string op) {
    return [op](const CacheEntry& e, void* io, std::string& error) -> bool {
      auto* g = static_cast<GemmIO*>(io);
      if (!g) {
        error = op + ": no I/O bundle";
        return false;
      }
      const int cfg[7] = {e.best.block_m, e.best.block_n, e.best.block_k, e.best.num_warps,
                          e.best.vector_width, e.best.unroll, e.best.shared_memory_stages};
      const int M = static_cast<int>(e.M), N = static_cast<int>(e.N), K = static_cast<int>(e.K);
      std::lock_guard<std::mutex> lk(mu);
      if (pkb200_set_gemm_config(cfg) != 0) {
        error = op + ": cached config block_n=" + std::to_string(e.best.block_n) + " stages=" +
                std::to_string(e.best.shared_memory_stages) + " has no compiled variant";
        return false;
      }
      int st;
      if (op == "matmul")
        st = pkb200_matmul(g->a, g->b, g->out, M, N, K, g->stream);
      else if (op == "fused_rmsnorm_matmul")
        st = pkb200_fused_rmsnorm_matmul(g->a, g->b, g->gamma, g->out, M, N, K, g->eps, g->stream);
      else if (op == "fused_matmul_bias_gelu")
        st = pkb200_fused_matmul_bias_gelu(g->a, g->b, g->bias, g->out, M, N, K, g->stream);
      else
        st = pkb200_matmul_bias_residual(g->a, g->b, g->bias, g->resid, g->out, M, N, K,
                                         g->stream);
      pkb200_set_gemm_config(nullptr);
      if (st != 0) {
        error = op + ": launch failed (status " + std::to_string(st) + ")";
        return false;
      }
      return true;
    };
  };
  for (const char* op :
       {"matmul", "fused_rmsnorm_matmul", "fused_matmul_bias_gelu", "matmul_bias_residual"})
    rt.RegisterLauncher(op, make(op));
}

}  // namespace runtime
}  // namespace pkb200
