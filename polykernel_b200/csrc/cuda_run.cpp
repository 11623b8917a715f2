// cuda_run.cpp - the .npy launcher harness over libpkb200.so, with the command
// line of the reference's lib/Runtime/cuda_run_main.cpp:356 (`cuda_run <op> ...`):
// read bf16 .npy inputs, copy them to the device, call the library's entry
// point, copy the result back and write a bf16 .npy. Same op names, argument
// order, defaults (--epsilon 1e-5) and exit codes (0 ok, 1 runtime error,
// 2 usage), plus the ops this library adds (mlp_block, matmul_int8, fp8sim,
// attention_prefill, kv_cache_update, attention_append).
//
// bf16 arrays use NumPy's '<V2' void descr (raw 16-bit brain-float values), as
// the reference's kernels/cpu/npy_io.h:264-277 writes them; int8 uses '|i1' and
// fp32 '<f4'.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/pkb200.h"

namespace {

struct Npy {
  std::string descr;
  std::vector<int64_t> shape;
  std::vector<char> bytes;
  int64_t size() const {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    return n;
  }
};

int elem_size(const std::string& d) {
  if (d == "<V2" || d == "|V2" || d == "<u2" || d == "<i2") return 2;
  if (d == "|i1" || d == "<i1" || d == "|u1") return 1;
  if (d == "<f4") return 4;
  throw std::runtime_error("unsupported npy descr " + d);
}

Npy read_npy(const std::string& path, const char* want_descr) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("cannot open " + path);
  char magic[6];
  f.read(magic, 6);
  if (std::memcmp(magic, "\x93NUMPY", 6) != 0) throw std::runtime_error(path + ": not a .npy file");
  unsigned char ver[2];
  f.read(reinterpret_cast<char*>(ver), 2);
  uint32_t hlen = 0;
  if (ver[0] == 1) {
    unsigned char l[2];
    f.read(reinterpret_cast<char*>(l), 2);
    hlen = l[0] | (l[1] << 8);
  } else {
    unsigned char l[4];
    f.read(reinterpret_cast<char*>(l), 4);
    hlen = l[0] | (l[1] << 8) | (l[2] << 16) | (static_cast<uint32_t>(l[3]) << 24);
  }
  std::string h(hlen, ' ');
  f.read(&h[0], hlen);
  Npy a;
  auto q = h.find("'descr'");
  auto s1 = h.find('\'', h.find(':', q) + 1);
  auto s2 = h.find('\'', s1 + 1);
  a.descr = h.substr(s1 + 1, s2 - s1 - 1);
  if (h.find("'fortran_order': True") != std::string::npos)
    throw std::runtime_error(path + ": fortran order not supported");
  auto p1 = h.find('(', h.find("'shape'"));
  auto p2 = h.find(')', p1);
  std::string dims = h.substr(p1 + 1, p2 - p1 - 1);
  size_t pos = 0;
  while (pos < dims.size()) {
    while (pos < dims.size() && (dims[pos] == ' ' || dims[pos] == ',')) ++pos;
    if (pos >= dims.size()) break;
    size_t e = pos;
    while (e < dims.size() && dims[e] != ',') ++e;
    a.shape.push_back(std::stoll(dims.substr(pos, e - pos)));
    pos = e;
  }
  const std::string want = want_descr ? want_descr : "";
  const bool same = a.descr == want || (want == "|i1" && a.descr == "<i1") ||
                    (want == "<V2" && a.descr == "|V2");  // NumPy writes 2-byte voids as |V2
  if (want_descr && !same)
    throw std::runtime_error(path + ": dtype " + a.descr + ", expected " + want_descr);
  a.bytes.resize(static_cast<size_t>(a.size()) * elem_size(a.descr));
  f.read(a.bytes.data(), static_cast<std::streamsize>(a.bytes.size()));
  if (!f) throw std::runtime_error(path + ": truncated payload");
  return a;
}

void write_npy_bf16(const std::string& path, const std::vector<int64_t>& shape,
                    const std::vector<char>& bytes) {
  std::string dims;
  for (size_t i = 0; i < shape.size(); ++i) dims += std::to_string(shape[i]) + ",";
  if (shape.size() > 1) dims.pop_back();
  std::string h = "{'descr': '<V2', 'fortran_order': False, 'shape': (" + dims + "), }";
  while ((10 + h.size() + 1) % 64) h += ' ';
  h += '\n';
  std::ofstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("cannot write " + path);
  f.write("\x93NUMPY\x01\x00", 8);
  const uint16_t hl = static_cast<uint16_t>(h.size());
  f.put(static_cast<char>(hl & 0xFF));
  f.put(static_cast<char>(hl >> 8));
  f.write(h.data(), static_cast<std::streamsize>(h.size()));
  f.write(bytes.data(), static_cast<std::streamsize>(bytes.size()));
}

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    std::fprintf(stderr, "[pkb200-cuda_run] %s failed: %s\n", what, cudaGetErrorString(e));
    std::exit(EXIT_FAILURE);
  }
}

// Owning device buffer.
struct Dev {
  void* p = nullptr;
  size_t n = 0;
  explicit Dev(size_t bytes) : n(bytes) {
    if (bytes) ck(cudaMalloc(&p, bytes), "cudaMalloc");
  }
  explicit Dev(const Npy& a) : Dev(a.bytes.size()) {
    if (n) ck(cudaMemcpy(p, a.bytes.data(), n, cudaMemcpyHostToDevice), "cudaMemcpy H2D");
  }
  ~Dev() {
    if (p) cudaFree(p);
  }
  Dev(const Dev&) = delete;
  Dev& operator=(const Dev&) = delete;
};

void download(const Dev& d, const std::vector<int64_t>& shape, const std::string& path) {
  std::vector<char> host(d.n);
  if (d.n) ck(cudaMemcpy(host.data(), d.p, d.n, cudaMemcpyDeviceToHost), "cudaMemcpy D2H");
  write_npy_bf16(path, shape, host);
}

int finish(int status, const char* what) {
  if (status != 0) {
    std::fprintf(stderr, "[pkb200-cuda_run] %s returned %s\n", what,
                 cudaGetErrorString(static_cast<cudaError_t>(status)));
    return 1;
  }
  ck(cudaDeviceSynchronize(), what);
  int derr = 0;
  pkb200_device_error(&derr);
  if (derr) {
    std::fprintf(stderr, "[pkb200-cuda_run] %s: device error code %d\n", what, derr);
    return 1;
  }
  return 0;
}

int usage(const char* msg) {
  std::fprintf(stderr, "usage: cuda_run <op> ...\n  %s\n", msg);
  return 2;
}

std::vector<int64_t> with_last(std::vector<int64_t> s, int64_t last) {
  s.back() = last;
  return s;
}

// ------------------------------------------------------------ shape checks --
// Every operand is validated against the primary one before any device
// allocation, so a mismatched or short file is rejected (exit 1) and no kernel
// ever reads past a buffer.
int shape_error(const char* op, const std::string& msg) {
  std::fprintf(stderr, "[pkb200-cuda_run] %s: shape error: %s\n", op, msg.c_str());
  return 1;
}

std::string dims_str(const Npy& a) {
  std::string s = "(";
  for (size_t i = 0; i < a.shape.size(); ++i) s += (i ? "," : "") + std::to_string(a.shape[i]);
  return s + ")";
}

constexpr int64_t kIntMax = 2147483647;

// Rows x cols view of a matrix operand whose last axis is the contraction /
// feature axis: rank >= 1, last axis > 0, both fit in int.
bool rows_cols(const Npy& a, int64_t& rows, int64_t& cols) {
  if (a.shape.empty() || a.shape.back() <= 0) return false;
  cols = a.shape.back();
  rows = a.size() / cols;
  return rows <= kIntMax && cols <= kIntMax;
}

// A [K, N] weight: rank 2, K == k, N > 0.
bool is_kn(const Npy& w, int64_t k) {
  return w.shape.size() == 2 && w.shape[0] == k && w.shape[1] > 0 && w.shape[1] <= kIntMax;
}

// A vector of n elements (any rank, as the reference's harness accepts).
bool is_vec(const Npy& v, int64_t n) { return !v.shape.empty() && v.size() == n; }

bool is_4d(const Npy& a) {
  if (a.shape.size() != 4) return false;
  for (int64_t d : a.shape)
    if (d < 0 || d > kIntMax) return false;
  return a.shape[3] > 0;
}

// Optional "--flag value" arguments after the positional ones.
struct Opts {
  float epsilon = 1e-5f;
  std::string weight;
  int causal = 1;
  float scale = NAN;
  int s_cache = 0;
  bool ok = true;
};
Opts parse_opts(int argc, char** argv, int first) {
  Opts o;
  for (int i = first; i < argc; ++i) {
    std::string a = argv[i];
    if (i + 1 >= argc) { o.ok = false; break; }
    if (a == "--epsilon") o.epsilon = std::stof(argv[++i]);
    else if (a == "--weight") o.weight = argv[++i];
    else if (a == "--causal") o.causal = std::stoi(argv[++i]);
    else if (a == "--scale") o.scale = std::stof(argv[++i]);
    else if (a == "--s-cache") o.s_cache = std::stoi(argv[++i]);
    else { o.ok = false; break; }
  }
  return o;
}

int run_rmsnorm(int argc, char** argv) {
  if (argc < 4) return usage("rmsnorm IN OUT [--weight W.npy] [--epsilon E]");
  Opts o = parse_opts(argc, argv, 4);
  if (!o.ok) return usage("rmsnorm IN OUT [--weight W.npy] [--epsilon E]");
  Npy in = read_npy(argv[2], "<V2");
  int64_t rows = 0, cols = 0;
  if (!rows_cols(in, rows, cols)) return shape_error("rmsnorm", "input " + dims_str(in));
  Npy w;
  if (!o.weight.empty()) {
    w = read_npy(o.weight, "<V2");
    if (!is_vec(w, cols))
      return shape_error("rmsnorm", "weight " + dims_str(w) + " != cols " + std::to_string(cols));
  }
  Dev din(in), dout(in.bytes.size());
  const void* wp = nullptr;
  std::unique_ptr<Dev> dw;
  if (!o.weight.empty()) {
    dw.reset(new Dev(w));
    wp = dw->p;
  }
  int st = finish(pkb200_rmsnorm(din.p, wp, dout.p, static_cast<int>(rows), static_cast<int>(cols),
                                 o.epsilon, nullptr), "rmsnorm");
  if (!st) download(dout, in.shape, argv[3]);
  return st;
}

int run_gelu(int argc, char** argv) {
  if (argc != 4) return usage("gelu IN OUT");
  Npy in = read_npy(argv[2], "<V2");
  Dev din(in), dout(in.bytes.size());
  int st = finish(pkb200_gelu(din.p, dout.p, in.size(), nullptr), "gelu");
  if (!st) download(dout, in.shape, argv[3]);
  return st;
}

// softmax IN OUT [--axis A]: last axis only (the reference's cuda_run_main.cpp:210-234).
int run_softmax(int argc, char** argv) {
  const char* u = "softmax IN OUT [--axis A]";
  if (argc < 4) return usage(u);
  int axis = -1;
  for (int i = 4; i < argc; ++i) {
    const std::string a = argv[i];
    if (a == "--axis" && i + 1 < argc)
      axis = std::atoi(argv[++i]);
    else
      return usage(u);
  }
  Npy in = read_npy(argv[2], "<V2");
  if (in.shape.empty() || (axis != -1 && axis != static_cast<int>(in.shape.size()) - 1)) {
    std::fprintf(stderr, "softmax: only last-axis reduction supported (axis=-1)\n");
    return 1;
  }
  const int64_t cols = in.shape.back(), rows = cols ? in.size() / cols : 0;
  Dev din(in), dout(in.bytes.size());
  int st = finish(pkb200_softmax(din.p, dout.p, (int)rows, (int)cols, nullptr), "softmax");
  if (!st) download(dout, in.shape, argv[3]);
  return st;
}

int run_matmul(int argc, char** argv) {
  if (argc != 5) return usage("matmul A B C");
  Npy a = read_npy(argv[2], "<V2"), b = read_npy(argv[3], "<V2");
  int64_t M = 0, K = 0;
  if (!rows_cols(a, M, K)) return shape_error("matmul", "A " + dims_str(a));
  if (!is_kn(b, K)) return shape_error("matmul", "B " + dims_str(b) + " is not [" + std::to_string(K) + ", N]");
  const int64_t N = b.shape[1];
  Dev da(a), db(b), dc(static_cast<size_t>(M * N) * 2);
  int st = finish(pkb200_matmul(da.p, db.p, dc.p, (int)M, (int)N, (int)K, nullptr), "matmul");
  if (!st) download(dc, with_last(a.shape, N), argv[4]);
  return st;
}

int run_fused_rmsnorm_matmul(int argc, char** argv) {
  if (argc < 5) return usage("fused_rmsnorm_matmul X W OUT [--epsilon E] [--weight GAMMA.npy]");
  Opts o = parse_opts(argc, argv, 5);
  if (!o.ok) return usage("fused_rmsnorm_matmul X W OUT [--epsilon E] [--weight GAMMA.npy]");
  Npy x = read_npy(argv[2], "<V2"), w = read_npy(argv[3], "<V2");
  int64_t M = 0, K = 0;
  if (!rows_cols(x, M, K)) return shape_error("fused_rmsnorm_matmul", "X " + dims_str(x));
  if (!is_kn(w, K))
    return shape_error("fused_rmsnorm_matmul", "W " + dims_str(w) + " is not [" + std::to_string(K) + ", N]");
  const int64_t N = w.shape[1];
  Npy gm;
  if (!o.weight.empty()) {
    gm = read_npy(o.weight, "<V2");
    if (!is_vec(gm, K)) return shape_error("fused_rmsnorm_matmul", "gamma " + dims_str(gm) + " != K");
  }
  Dev dx(x), dw(w), dout(static_cast<size_t>(M * N) * 2);
  std::unique_ptr<Dev> dg;
  if (!o.weight.empty()) dg.reset(new Dev(gm));
  int st = finish(pkb200_fused_rmsnorm_matmul(dx.p, dw.p, dg ? dg->p : nullptr, dout.p, (int)M,
                                              (int)N, (int)K, o.epsilon, nullptr),
                  "fused_rmsnorm_matmul");
  if (!st) download(dout, with_last(x.shape, N), argv[4]);
  return st;
}

int run_fused_matmul_bias_gelu(int argc, char** argv) {
  if (argc != 6) return usage("fused_matmul_bias_gelu A B BIAS OUT");
  Npy a = read_npy(argv[2], "<V2"), b = read_npy(argv[3], "<V2"), bias = read_npy(argv[4], "<V2");
  int64_t M = 0, K = 0;
  if (!rows_cols(a, M, K)) return shape_error("fused_matmul_bias_gelu", "A " + dims_str(a));
  if (!is_kn(b, K)) return shape_error("fused_matmul_bias_gelu", "B " + dims_str(b) + " is not [K, N]");
  const int64_t N = b.shape[1];
  if (!is_vec(bias, N)) return shape_error("fused_matmul_bias_gelu", "bias " + dims_str(bias) + " != N");
  Dev da(a), db(b), dbias(bias), dout(static_cast<size_t>(M * N) * 2);
  int st = finish(pkb200_fused_matmul_bias_gelu(da.p, db.p, dbias.p, dout.p, (int)M, (int)N,
                                                (int)K, nullptr),
                  "fused_matmul_bias_gelu");
  if (!st) download(dout, with_last(a.shape, N), argv[5]);
  return st;
}

int run_matmul_int8(int argc, char** argv) {
  if (argc != 6) return usage("matmul_int8 A WQ SCALE OUT   (A bf16 [M,K], WQ int8 [K,N], SCALE fp32 [N])");
  Npy a = read_npy(argv[2], "<V2"), wq = read_npy(argv[3], "|i1"), sc = read_npy(argv[4], "<f4");
  int64_t M = 0, K = 0;
  if (!rows_cols(a, M, K)) return shape_error("matmul_int8", "A " + dims_str(a));
  if (!is_kn(wq, K)) return shape_error("matmul_int8", "WQ " + dims_str(wq) + " is not [K, N]");
  const int64_t N = wq.shape[1];
  if (!is_vec(sc, N)) return shape_error("matmul_int8", "SCALE " + dims_str(sc) + " != N");
  Dev da(a), dw(wq), ds(sc), dout(static_cast<size_t>(M * N) * 2);
  int st = finish(pkb200_matmul_int8(da.p, static_cast<const int8_t*>(dw.p),
                                     static_cast<const float*>(ds.p), dout.p, (int)M, (int)N,
                                     (int)K, nullptr),
                  "matmul_int8");
  if (!st) download(dout, with_last(a.shape, N), argv[5]);
  return st;
}

// fp8sim <e4m3|e5m2> A W OUT: the simulated fp8 weight path with the argument
// order of the reference's CPU driver (kernels/cpu/matmul_quant.cpp:168, `fp8sim`).
int run_fp8sim(int argc, char** argv) {
  if (argc != 6) return usage("fp8sim <e4m3|e5m2> A W OUT   (A bf16 [M,K], W bf16 [K,N])");
  const std::string fmt = argv[2];
  if (fmt != "e4m3" && fmt != "e5m2") return usage("fp8sim: format must be e4m3 or e5m2");
  Npy a = read_npy(argv[3], "<V2"), w = read_npy(argv[4], "<V2");
  int64_t M = 0, K = 0;
  if (!rows_cols(a, M, K)) return shape_error("fp8sim", "A " + dims_str(a));
  if (!is_kn(w, K)) return shape_error("fp8sim", "W " + dims_str(w) + " is not [K, N]");
  const int64_t N = w.shape[1];
  std::fprintf(stderr, "[pkb200-cuda_run] path=fp8_sim fmt=%s M=%lld N=%lld K=%lld\n",
               fmt.c_str(), (long long)M, (long long)N, (long long)K);
  Dev da(a), dw(w), dout(static_cast<size_t>(M * N) * 2);
  int st = finish(pkb200_matmul_fp8_sim(da.p, dw.p, dout.p, (int)M, (int)N, (int)K,
                                        fmt == "e4m3" ? 0 : 1, nullptr),
                  "fp8sim");
  if (!st) download(dout, with_last(a.shape, N), argv[5]);
  return st;
}

int run_mlp_block(int argc, char** argv) {
  const char* u = "mlp_block X GAMMA W1 B1 W2 B2 OUT [--epsilon E]";
  if (argc < 9) return usage(u);
  Opts o = parse_opts(argc, argv, 9);
  if (!o.ok) return usage(u);
  Npy x = read_npy(argv[2], "<V2"), g = read_npy(argv[3], "<V2"), w1 = read_npy(argv[4], "<V2"),
      b1 = read_npy(argv[5], "<V2"), w2 = read_npy(argv[6], "<V2"), b2 = read_npy(argv[7], "<V2");
  int64_t M = 0, d = 0;
  if (!rows_cols(x, M, d)) return shape_error("mlp_block", "X " + dims_str(x));
  if (!is_vec(g, d)) return shape_error("mlp_block", "GAMMA " + dims_str(g) + " != d");
  if (!is_kn(w1, d)) return shape_error("mlp_block", "W1 " + dims_str(w1) + " is not [d, ffn]");
  const int64_t ffn = w1.shape[1];
  if (!is_vec(b1, ffn)) return shape_error("mlp_block", "B1 " + dims_str(b1) + " != ffn");
  if (!is_kn(w2, ffn) || w2.shape[1] != d)
    return shape_error("mlp_block", "W2 " + dims_str(w2) + " is not [ffn, d]");
  if (!is_vec(b2, d)) return shape_error("mlp_block", "B2 " + dims_str(b2) + " != d");
  Dev dx(x), dg(g), dw1(w1), db1(b1), dw2(w2), db2(b2), dy(x.bytes.size());
  const size_t wsb = pkb200_mlp_block_workspace_size((int)M, (int)d, (int)ffn);
  Dev ws(wsb);
  int st = finish(pkb200_mlp_block(dx.p, dg.p, dw1.p, db1.p, dw2.p, db2.p, dy.p, (int)M, (int)d,
                                   (int)ffn, o.epsilon, ws.p, wsb, nullptr),
                  "mlp_block");
  if (!st) download(dy, x.shape, argv[8]);
  return st;
}

int run_attention_prefill(int argc, char** argv) {
  const char* u = "attention_prefill Q K V OUT [--causal N] [--scale S]";
  if (argc < 6) return usage(u);
  Opts o = parse_opts(argc, argv, 6);
  if (!o.ok) return usage(u);
  Npy q = read_npy(argv[2], "<V2"), k = read_npy(argv[3], "<V2"), v = read_npy(argv[4], "<V2");
  if (!is_4d(q) || !is_4d(k) || v.shape != k.shape)
    return shape_error("attention_prefill", "Q " + dims_str(q) + " K " + dims_str(k) + " V " + dims_str(v));
  if (k.shape[0] != q.shape[0] || k.shape[1] != q.shape[1] || k.shape[3] != q.shape[3])
    return shape_error("attention_prefill", "K " + dims_str(k) + " does not match Q " + dims_str(q) + " in B, H or D");
  const int B = (int)q.shape[0], H = (int)q.shape[1], Sq = (int)q.shape[2], D = (int)q.shape[3];
  const int Skv = (int)k.shape[2];
  const float scale = std::isnan(o.scale) ? 1.0f / std::sqrt(static_cast<float>(D)) : o.scale;
  Dev dq(q), dk(k), dv(v), dout(q.bytes.size());
  int st = finish(pkb200_attention_prefill(dq.p, dk.p, dv.p, dout.p, B, H, Sq, Skv, D, scale,
                                           o.causal, nullptr),
                  "attention_prefill");
  if (!st) download(dout, q.shape, argv[5]);
  return st;
}

int run_kv_cache_update(int argc, char** argv) {
  if (argc != 5) return usage("kv_cache_update CACHE NEW OUT");
  Npy c = read_npy(argv[2], "<V2"), n = read_npy(argv[3], "<V2");
  if (!is_4d(c) || !is_4d(n) || n.shape[0] != c.shape[0] || n.shape[1] != c.shape[1] ||
      n.shape[3] != c.shape[3])
    return shape_error("kv_cache_update", "CACHE " + dims_str(c) + " NEW " + dims_str(n));
  const int B = (int)c.shape[0], H = (int)c.shape[1], Sc = (int)c.shape[2], D = (int)c.shape[3];
  const int Sn = (int)n.shape[2];
  Dev dc(c), dn(n), dout(static_cast<size_t>(B) * H * (Sc + Sn) * D * 2);
  int st = finish(pkb200_kv_cache_update(dc.p, dn.p, dout.p, B, H, Sc, Sn, D, nullptr),
                  "kv_cache_update");
  if (!st) download(dout, {B, H, Sc + Sn, D}, argv[4]);
  return st;
}

// Fused append + attention on a preallocated cache: KCACHE/VCACHE [B,H,S_max,D]
// hold --s-cache valid rows; writes OUT and the updated caches.
int run_attention_append(int argc, char** argv) {
  const char* u =
      "attention_append Q KNEW VNEW KCACHE VCACHE OUT KOUT VOUT [--s-cache S] [--causal N]";
  if (argc < 10) return usage(u);
  Opts o = parse_opts(argc, argv, 10);
  if (!o.ok) return usage(u);
  Npy q = read_npy(argv[2], "<V2"), kn = read_npy(argv[3], "<V2"), vn = read_npy(argv[4], "<V2"),
      kc = read_npy(argv[5], "<V2"), vc = read_npy(argv[6], "<V2");
  if (!is_4d(q) || kn.shape != q.shape || vn.shape != q.shape)
    return shape_error("attention_append", "Q " + dims_str(q) + " KNEW " + dims_str(kn) + " VNEW " + dims_str(vn));
  if (!is_4d(kc) || vc.shape != kc.shape || kc.shape[0] != q.shape[0] || kc.shape[1] != q.shape[1] ||
      kc.shape[3] != q.shape[3])
    return shape_error("attention_append", "KCACHE " + dims_str(kc) + " VCACHE " + dims_str(vc));
  if (o.s_cache < 0 || o.s_cache + q.shape[2] > kc.shape[2])
    return shape_error("attention_append", "s_cache + S_new exceeds the cache rows");
  const int B = (int)q.shape[0], H = (int)q.shape[1], Sq = (int)q.shape[2], D = (int)q.shape[3];
  const int Smax = (int)kc.shape[2];
  Dev dq(q), dkn(kn), dvn(vn), dkc(kc), dvc(vc), dout(q.bytes.size());
  const float scale = std::isnan(o.scale) ? 1.0f / std::sqrt(static_cast<float>(D)) : o.scale;
  int st = finish(pkb200_attention_prefill_kv_append(dq.p, dkn.p, dvn.p, dkc.p, dvc.p, dout.p, B,
                                                     H, Sq, o.s_cache, Smax, D, scale, o.causal,
                                                     nullptr),
                  "attention_append");
  if (!st) {
    download(dout, q.shape, argv[7]);
    download(dkc, kc.shape, argv[8]);
    download(dvc, vc.shape, argv[9]);
  }
  return st;
}

int run_dev() {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    std::fprintf(stderr, "[pkb200-cuda_run] dev: no CUDA device (count=%d, %s)\n", n,
                 cudaGetErrorString(e != cudaSuccess ? e : cudaErrorNoDevice));
    return 1;
  }
  cudaDeviceProp p{};
  ck(cudaGetDeviceProperties(&p, 0), "cudaGetDeviceProperties");
  std::fprintf(stderr, "DEVICE %s COMPUTE_CAPABILITY %d.%d\n", p.name, p.major, p.minor);
  return 0;
}

// Negative probe: a shape the library must reject without launching anything.
int run_neg() {
  const int st = pkb200_matmul(nullptr, nullptr, nullptr, 4, 4, 4, nullptr);
  std::fprintf(stderr, "[pkb200-cuda_run] neg: null-operand matmul returned %s\n",
               cudaGetErrorString(static_cast<cudaError_t>(st)));
  if (st == 0) {
    std::fprintf(stderr, "[pkb200-cuda_run] neg: FAIL - invalid call accepted\n");
    return 2;
  }
  std::fprintf(stderr, "[pkb200-cuda_run] neg: PASS - invalid call rejected\n");
  return 1;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) return usage("<op> ...");
  const std::string op = argv[1];
  try {
    if (op == "rmsnorm") return run_rmsnorm(argc, argv);
    if (op == "gelu") return run_gelu(argc, argv);
    if (op == "matmul") return run_matmul(argc, argv);
    if (op == "softmax") return run_softmax(argc, argv);
    if (op == "fused_rmsnorm_matmul") return run_fused_rmsnorm_matmul(argc, argv);
    if (op == "fused_matmul_bias_gelu") return run_fused_matmul_bias_gelu(argc, argv);
    if (op == "matmul_int8") return run_matmul_int8(argc, argv);
    if (op == "fp8sim") return run_fp8sim(argc, argv);
    if (op == "mlp_block") return run_mlp_block(argc, argv);
    if (op == "attention_prefill") return run_attention_prefill(argc, argv);
    if (op == "kv_cache_update") return run_kv_cache_update(argc, argv);
    if (op == "attention_append") return run_attention_append(argc, argv);
    if (op == "dev") return run_dev();
    if (op == "neg") return run_neg();
  } catch (const std::exception& e) {
    std::fprintf(stderr, "[pkb200-cuda_run] error: %s\n", e.what());
    return 1;
  }
  return usage("unknown op");
}
