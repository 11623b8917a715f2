// GPU-free tests of include/pkb200_runtime.h: the detect -> select -> load ->
// serve flow with an injected arch and recording launchers, the cache's
// all-or-nothing loads, persistence and stale-binary invalidation, and the
// library's own launchers rejecting a bad call with a typed error. They cover
// the cases of the reference's lib/Runtime/tests (runtime_test.cpp:81-271,
// kernel_cache_persist_test.cpp:76-260, device_detect_test.cpp:54-80).
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iterator>
#include <string>
#include <vector>

#include "pkb200_runtime.h"

using namespace pkb200::runtime;

static int g_failed = 0, g_checks = 0;
#define CHECK(cond)                                                          \
  do {                                                                       \
    ++g_checks;                                                              \
    if (!(cond)) {                                                           \
      ++g_failed;                                                            \
      std::fprintf(stderr, "%s:%d: CHECK failed: %s\n", __FILE__, __LINE__, #cond); \
    }                                                                        \
  } while (0)

static bool contains(const std::string& s, const std::string& sub) {
  return s.find(sub) != std::string::npos;
}

static CacheEntry entry(const std::string& gpu, const std::string& op, long long M, long long N,
                        long long K, int block_n, bool validated = true) {
  CacheEntry e;
  e.gpu = gpu;
  e.op = op;
  e.dtype = "bf16";
  e.M = M;
  e.N = N;
  e.K = K;
  e.best.block_n = block_n;
  e.validated = validated;
  e.time_ms = 0.25;
  e.cosine = 1.0;
  e.pcc = 1.0;
  return e;
}

static const char* kDoc = R"({"version": 1, "entries": [
  {"gpu": "sm_100", "op": "matmul", "shape": {"M": 256, "N": 512, "K": 1024, "dtype": "bf16"},
   "best": {"block_m": 128, "block_n": 128, "block_k": 64, "num_warps": 10, "vector_width": 8,
            "unroll": 2, "shared_memory_stages": 6},
   "scored_by": "measure", "time_ms": 0.01, "validated": true,
   "correctness": {"cosine": 1.0, "max_rel_err": 0.0, "pcc": 1.0}},
  {"gpu": "sm_90", "op": "matmul", "shape": {"M": 256, "N": 512, "K": 1024, "dtype": "bf16"},
   "best": {"block_m": 128, "block_n": 256, "block_k": 64, "num_warps": 10, "vector_width": 8,
            "unroll": 2, "shared_memory_stages": 4},
   "scored_by": "compile_time_model", "time_ms": null, "validated": true,
   "correctness": {"cosine": 1.0, "max_rel_err": 0.0, "pcc": 1.0}}]})";

class NoDevice final : public DeviceDetector {
 public:
  std::optional<DeviceInfo> Detect(int = 0) const override { return std::nullopt; }
};

static void test_detect() {
  CHECK(SmArchFromComputeCapability(10, 0) == "sm_100");
  CHECK(SmArchFromComputeCapability(9, 0) == "sm_90");
  FixedArchDetector d("sm_100");
  CHECK(d.Detect(0)->arch == "sm_100" && d.Detect(3)->arch == "sm_100");
}

static void test_selection_and_serve() {
  KernelCache cache;
  CHECK(cache.Put(entry("sm_100", "matmul", 256, 512, 1024, 128)));
  CHECK(cache.Put(entry("sm_90", "matmul", 256, 512, 1024, 256)));
  CHECK(!cache.Put(entry("", "matmul", 1, 1, 1, 128)));
  FixedArchDetector b200("sm_100");
  Runtime rt(b200, cache);
  std::vector<int> served;
  rt.RegisterLauncher("matmul", [&](const CacheEntry& e, void* io, std::string&) {
    served.push_back(e.best.block_n);
    *static_cast<int*>(io) += 1;
    return true;
  });
  ResolveResult r = rt.Resolve("matmul", Shape{256, 512, 1024});
  CHECK(r.ok() && r.device->arch == "sm_100" && r.entry->best.block_n == 128);
  int calls = 0;
  std::string err;
  CHECK(rt.Run("matmul", Shape{256, 512, 1024}, &calls, err));
  CHECK(calls == 1 && served.size() == 1 && served[0] == 128);
  // a miss never serves
  CHECK(!rt.Run("matmul", Shape{256, 512, 2048}, &calls, err));
  CHECK(contains(err, "no tuned kernel for sm_100/matmul/M=256,N=512,K=2048,bf16"));
  CHECK(contains(err, "run the autotuner"));
  CHECK(calls == 1);
  // another op with no entry
  CHECK(!rt.Run("fused_matmul_bias_gelu", Shape{256, 512, 1024}, &calls, err));
  CHECK(contains(err, "no tuned kernel"));
}

static void test_unvalidated_and_missing_launcher() {
  KernelCache cache;
  cache.Put(entry("sm_100", "matmul", 64, 64, 64, 128, /*validated=*/false));
  cache.Put(entry("sm_100", "fused_matmul_bias_gelu", 64, 64, 64, 128));
  FixedArchDetector b200("sm_100");
  Runtime rt(b200, cache);
  bool called = false;
  rt.RegisterLauncher("matmul", [&](const CacheEntry&, void*, std::string&) {
    called = true;
    return true;
  });
  std::string err;
  CHECK(!rt.Run("matmul", Shape{64, 64, 64}, nullptr, err));
  CHECK(contains(err, "not validated") && !called);
  CHECK(!rt.Run("fused_matmul_bias_gelu", Shape{64, 64, 64}, nullptr, err));
  CHECK(contains(err, "no compiled launcher registered for op fused_matmul_bias_gelu"));
  // a failing launcher's error reaches the caller
  rt.RegisterLauncher("fused_matmul_bias_gelu", [](const CacheEntry&, void*, std::string& e) {
    e = "launch failed: simulated";
    return false;
  });
  CHECK(!rt.Run("fused_matmul_bias_gelu", Shape{64, 64, 64}, nullptr, err));
  CHECK(err == "launch failed: simulated");
  // no device: a typed error, not a launch
  NoDevice none;
  Runtime rt2(none, cache);
  CHECK(!rt2.Run("matmul", Shape{64, 64, 64}, nullptr, err));
  CHECK(contains(err, "device detection failed"));
}

static void test_load_json() {
  KernelCache cache;
  std::string err;
  CHECK(cache.LoadTuningCache(kDoc, err));
  CHECK(cache.Size() == 2);
  SelectionResult s = cache.Select("sm_100", "matmul", Shape{256, 512, 1024});
  CHECK(s.ok() && s.entry->best.block_n == 128 && s.entry->best.shared_memory_stages == 6);
  CHECK(s.entry->scored_by == "measure" && s.entry->has_time);
  SelectionResult m = cache.Select("sm_90", "matmul", Shape{256, 512, 1024});
  CHECK(m.ok() && !m.entry->has_time);
  // malformed documents are rejected with a field path, and the cache is unchanged
  std::string bad = kDoc;
  bad.replace(bad.find("\"validated\": true"), 17, "\"validated\": 1");
  CHECK(!cache.LoadTuningCache(bad, err) && contains(err, "validated"));
  CHECK(cache.Size() == 2);
  CHECK(!cache.LoadTuningCache("{\"version\": 2, \"entries\": []}", err) &&
        contains(err, "version"));
  CHECK(!cache.LoadTuningCache("{\"version\": 1}", err) && contains(err, "entries"));
  CHECK(!cache.LoadTuningCache("not json", err));
  CHECK(cache.Size() == 2);
  // the serialiser writes what the parser reads
  KernelCache again;
  CHECK(again.LoadTuningCache(cache.SerializeTuning(), err));
  CHECK(again.Size() == 2);
  CHECK(again.Select("sm_100", "matmul", Shape{256, 512, 1024}).entry->best.shared_memory_stages == 6);
}

static void test_persist_and_invalidate(const std::string& tmp) {
  const std::string so = tmp + "/variant.so";
  { std::ofstream(so) << "compiled variant v1"; }
  std::string h1, err;
  CHECK(HashFile(so, h1, err) && h1.size() == 16);
  KernelCache cache;
  CHECK(cache.LoadTuningCache(kDoc, err));
  Shape s{256, 512, 1024};
  CHECK(cache.PutBinary("sm_100", "matmul", s, CachedBinary{so, h1}));
  CHECK(!cache.PutBinary("sm_100", "matmul", Shape{1, 2, 3}, CachedBinary{so, h1}));
  const std::string dir = tmp + "/cache";
  CHECK(cache.Persist(dir, err));
  KernelCache loaded;
  CHECK(loaded.LoadPersisted(dir, err));
  CHECK(loaded.Size() == 2 && loaded.GetBinary("sm_100", "matmul", s)->kernel_hash == h1);
  // per-gpu selection from the reloaded cache
  auto per = loaded.SelectPerGpu({"sm_100", "sm_90", "sm_80"}, "matmul", s);
  CHECK(per.size() == 3 && per[0].second.ok() && per[0].second.entry->best.block_n == 128);
  CHECK(per[1].second.ok() && per[1].second.entry->best.block_n == 256);
  CHECK(!per[2].second.ok() && contains(per[2].second.error, "no tuned kernel"));
  // an unchanged binary stays; a changed one is dropped and selection misses
  CHECK(loaded.InvalidateStale() == 0);
  { std::ofstream(so) << "compiled variant v2"; }
  CHECK(loaded.InvalidateStale() == 1);
  CHECK(!loaded.Select("sm_100", "matmul", s).ok());
  CHECK(loaded.Select("sm_90", "matmul", s).ok());  // no binary recorded: untouched
  // a missing binary is stale too
  KernelCache c2;
  c2.LoadTuningCache(kDoc, err);
  c2.PutBinary("sm_100", "matmul", s, CachedBinary{tmp + "/absent.so", h1});
  CHECK(c2.InvalidateStale() == 1);
  CHECK(!HashFile(tmp + "/absent.so", h1, err) && contains(err, "cannot read"));
  // a binaries.json naming an entry that does not exist is rejected, cache unchanged
  { std::ofstream(dir + "/binaries.json")
        << R"({"version": 1, "binaries": [{"gpu": "sm_100", "op": "matmul",
              "shape": {"M": 9, "N": 9, "K": 9, "dtype": "bf16"},
              "so_path": "x.so", "kernel_hash": "00"}]})"; }
  KernelCache c3;
  c3.Put(entry("sm_100", "matmul", 1, 1, 1, 128));
  CHECK(!c3.LoadPersisted(dir, err) && contains(err, "binaries.json"));
  CHECK(c3.Size() == 1);
  CHECK(!c3.LoadPersisted(tmp + "/no_such_dir", err) && contains(err, "cannot read"));
}

static void test_library_launchers() {
  KernelCache cache;
  cache.Put(entry("sm_100", "matmul", 128, 128, 128, 128));
  CacheEntry odd = entry("sm_100", "fused_matmul_bias_gelu", 128, 128, 128, 192);
  cache.Put(odd);
  FixedArchDetector b200("sm_100");
  Runtime rt(b200, cache);
  RegisterLibraryLaunchers(rt);
  GemmIO io;  // null operands: the library rejects the call before any launch
  std::string err;
  CHECK(!rt.Run("matmul", Shape{128, 128, 128}, &io, err));
  CHECK(contains(err, "matmul: launch failed (status"));
  // a cached config with no compiled variant is refused, not approximated
  CHECK(!rt.Run("fused_matmul_bias_gelu", Shape{128, 128, 128}, &io, err));
  CHECK(contains(err, "no compiled variant"));
  CHECK(!rt.Run("matmul", Shape{128, 128, 128}, nullptr, err) && contains(err, "no I/O bundle"));
}

// A cache written by the Python tuning module (polykernel_b200.tuning.save)
// loads here unchanged: one schema, two writers.
static void test_python_written_cache(const std::string& path) {
  std::ifstream f(path);
  CHECK(static_cast<bool>(f));
  std::string text((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  KernelCache cache;
  std::string err;
  CHECK(cache.LoadTuningCache(text, err));
  CHECK(cache.Size() == 2);
  SelectionResult s = cache.Select("sm_100", "fused_matmul_bias_gelu", Shape{2048, 16384, 4096});
  CHECK(s.ok() && s.entry->best.block_n == 128 && s.entry->best.shared_memory_stages == 6);
  CHECK(!cache.Select("sm_100", "matmul", Shape{64, 64, 64}).ok());  // validated: false
}

int main(int argc, char** argv) {
  const std::string tmp = argc > 1 ? argv[1] : "/tmp";
  if (argc > 2) test_python_written_cache(argv[2]);
  test_detect();
  test_selection_and_serve();
  test_unvalidated_and_missing_launcher();
  test_load_json();
  test_persist_and_invalidate(tmp);
  test_library_launchers();
  std::printf("%d checks, %d failed\n", g_checks, g_failed);
  if (g_failed == 0) std::printf("ALL PASSED\n");
  return g_failed ? 1 : 0;
}
