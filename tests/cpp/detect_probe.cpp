// Prints what the real device detectors of include/pkb200_runtime.h report
// ("none" when there is no usable device) and what Runtime::Run returns then.
#include <cstdio>
#include <string>

#include "pkb200_runtime.h"

using namespace pkb200::runtime;

int main() {
  CudaDeviceDetector cuda;
  LibraryDeviceDetector library;
  const auto a = cuda.Detect(0);
  const auto b = library.Detect(0);
  std::printf("cuda=%s library=%s\n", a ? a->arch.c_str() : "none", b ? b->arch.c_str() : "none");
  KernelCache cache;
  Runtime rt(cuda, cache);
  std::string err;
  const bool ok = rt.Run("matmul", Shape{8, 8, 8}, nullptr, err);
  std::printf("run=%d error=%s\n", ok ? 1 : 0, err.c_str());
  return 0;
}
