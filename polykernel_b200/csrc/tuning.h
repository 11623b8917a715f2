// tuning.h - the tuning cache of the runtime: parse a cache file in the
// reference's JSON format (tuning/schema.json, version 1: entries of
// {gpu, op, shape{M,N,K,dtype}, best{block_m, block_n, block_k, num_warps,
// vector_width, unroll, shared_memory_stages}, scored_by, time_ms, validated,
// correctness{cosine, max_rel_err, pcc}}), keep the validated entries, and
// answer (gpu, op, shape) lookups as the reference's KernelCache::Select does
// (lib/Runtime/KernelCache.cpp:83-100: only validated entries are served;
// a miss means "use the default").
//
// A malformed file is an error, never a silent default: unknown or missing
// fields, wrong types, version != 1, time_ms not null iff scored_by is
// "compile_time_model" (the rules of lib/Autotune/TuningCache.cpp:265).
#pragma once

#include <cctype>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

namespace pkb200 {
namespace tuning {

// ------------------------------------------------------------ JSON values --
struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0;
  bool is_int = false;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* get(const std::string& k) const {
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

class Parser {
 public:
  explicit Parser(const std::string& t) : s_(t) {}
  bool parse(Json& out, std::string& err) {
    if (!value(out, err)) return false;
    ws();
    if (i_ != s_.size()) return fail(err, "trailing characters");
    return true;
  }

 private:
  const std::string& s_;
  size_t i_ = 0;
  bool fail(std::string& err, const std::string& m) {
    err = m + " at offset " + std::to_string(i_);
    return false;
  }
  void ws() {
    while (i_ < s_.size() && std::isspace(static_cast<unsigned char>(s_[i_]))) ++i_;
  }
  bool lit(const char* w) {
    size_t n = std::char_traits<char>::length(w);
    if (s_.compare(i_, n, w) == 0) {
      i_ += n;
      return true;
    }
    return false;
  }
  bool string(std::string& out, std::string& err) {
    if (s_[i_] != '"') return fail(err, "expected string");
    ++i_;
    while (i_ < s_.size() && s_[i_] != '"') {
      char c = s_[i_++];
      if (c == '\\') {
        if (i_ >= s_.size()) return fail(err, "bad escape");
        char e = s_[i_++];
        switch (e) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (i_ + 4 > s_.size()) return fail(err, "bad \\u escape");
            const unsigned cp = std::stoul(s_.substr(i_, 4), nullptr, 16);
            i_ += 4;
            if (cp < 0x80) out += static_cast<char>(cp);
            else if (cp < 0x800) { out += static_cast<char>(0xC0 | (cp >> 6)); out += static_cast<char>(0x80 | (cp & 0x3F)); }
            else { out += static_cast<char>(0xE0 | (cp >> 12)); out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F)); out += static_cast<char>(0x80 | (cp & 0x3F)); }
            break;
          }
          default: out += e;
        }
      } else {
        out += c;
      }
    }
    if (i_ >= s_.size()) return fail(err, "unterminated string");
    ++i_;
    return true;
  }
  bool value(Json& v, std::string& err) {
    ws();
    if (i_ >= s_.size()) return fail(err, "unexpected end");
    const char c = s_[i_];
    if (c == '{') {
      v.kind = Json::Obj;
      ++i_;
      ws();
      if (i_ < s_.size() && s_[i_] == '}') { ++i_; return true; }
      while (true) {
        ws();
        std::string k;
        if (!string(k, err)) return false;
        ws();
        if (i_ >= s_.size() || s_[i_] != ':') return fail(err, "expected ':'");
        ++i_;
        Json child;
        if (!value(child, err)) return false;
        if (v.get(k)) return fail(err, "duplicate key '" + k + "'");
        v.obj.emplace_back(k, std::move(child));
        ws();
        if (i_ < s_.size() && s_[i_] == ',') { ++i_; continue; }
        if (i_ < s_.size() && s_[i_] == '}') { ++i_; return true; }
        return fail(err, "expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.kind = Json::Arr;
      ++i_;
      ws();
      if (i_ < s_.size() && s_[i_] == ']') { ++i_; return true; }
      while (true) {
        Json child;
        if (!value(child, err)) return false;
        v.arr.push_back(std::move(child));
        ws();
        if (i_ < s_.size() && s_[i_] == ',') { ++i_; continue; }
        if (i_ < s_.size() && s_[i_] == ']') { ++i_; return true; }
        return fail(err, "expected ',' or ']'");
      }
    }
    if (c == '"') { v.kind = Json::Str; return string(v.str, err); }
    if (lit("true")) { v.kind = Json::Bool; v.b = true; return true; }
    if (lit("false")) { v.kind = Json::Bool; v.b = false; return true; }
    if (lit("null")) { v.kind = Json::Null; return true; }
    const size_t start = i_;
    if (s_[i_] == '-') ++i_;
    bool frac = false;
    while (i_ < s_.size() && (std::isdigit(static_cast<unsigned char>(s_[i_])) || s_[i_] == '.' ||
                              s_[i_] == 'e' || s_[i_] == 'E' || s_[i_] == '+' || s_[i_] == '-')) {
      if (s_[i_] == '.' || s_[i_] == 'e' || s_[i_] == 'E') frac = true;
      ++i_;
    }
    if (i_ == start) return fail(err, "unexpected character");
    v.kind = Json::Num;
    v.num = std::strtod(s_.substr(start, i_ - start).c_str(), nullptr);
    v.is_int = !frac;
    return true;
  }
};

// ------------------------------------------------------------- the cache --
struct Config {
  int block_m = 128, block_n = 256, block_k = 64, num_warps = 10, vector_width = 8, unroll = 2,
      shared_memory_stages = 4;
};

struct Entry {
  std::string gpu, op, dtype;
  long long M = 0, N = 0, K = 0;
  Config best;
  bool validated = false;
  std::string scored_by = "measure";  // "measure" | "compile_time_model"
  bool has_time = true;               // time_ms is null iff scored by the model
  double time_ms = 0;
  double cosine = 0, max_rel_err = 0, pcc = 0;
};

inline bool expect_keys(const Json& o, const std::set<std::string>& keys, const std::string& where,
                        std::string& err) {
  if (o.kind != Json::Obj) {
    err = where + ": expected an object";
    return false;
  }
  for (auto& kv : o.obj)
    if (!keys.count(kv.first)) {
      err = where + ": unknown field '" + kv.first + "'";
      return false;
    }
  for (auto& k : keys)
    if (!o.get(k)) {
      err = where + ": missing field '" + k + "'";
      return false;
    }
  return true;
}

inline bool get_int(const Json& o, const char* k, long long& out, const std::string& where,
                    std::string& err) {
  const Json* v = o.get(k);
  if (!v || v->kind != Json::Num || !v->is_int) {
    err = where + "." + k + ": expected an integer";
    return false;
  }
  out = static_cast<long long>(v->num);
  return true;
}

inline bool get_num(const Json& o, const char* k, const std::string& where, std::string& err,
                    double* out = nullptr) {
  const Json* v = o.get(k);
  if (!v || v->kind != Json::Num) {
    err = where + "." + k + ": expected a number";
    return false;
  }
  if (out) *out = v->num;
  return true;
}

inline bool get_str(const Json& o, const char* k, std::string& out, const std::string& where,
                    std::string& err) {
  const Json* v = o.get(k);
  if (!v || v->kind != Json::Str) {
    err = where + "." + k + ": expected a string";
    return false;
  }
  out = v->str;
  return true;
}

// Parse a cache document into entries; false (with `err`) on any schema error.
inline bool parse_cache(const std::string& text, std::vector<Entry>& out, std::string& err) {
  Json root;
  if (!Parser(text).parse(root, err)) return false;
  if (!expect_keys(root, {"version", "entries"}, "cache", err)) return false;
  long long version = 0;
  if (!get_int(root, "version", version, "cache", err)) return false;
  if (version != 1) {
    err = "cache.version: unsupported version " + std::to_string(version) + " (expected 1)";
    return false;
  }
  const Json* entries = root.get("entries");
  if (entries->kind != Json::Arr) {
    err = "cache.entries: expected an array";
    return false;
  }
  for (size_t i = 0; i < entries->arr.size(); ++i) {
    const Json& e = entries->arr[i];
    const std::string w = "entries[" + std::to_string(i) + "]";
    if (!expect_keys(e, {"gpu", "op", "shape", "best", "scored_by", "time_ms", "validated",
                         "correctness"},
                     w, err))
      return false;
    Entry ent;
    if (!get_str(e, "gpu", ent.gpu, w, err) || !get_str(e, "op", ent.op, w, err)) return false;
    const Json& sh = *e.get("shape");
    if (!expect_keys(sh, {"M", "N", "K", "dtype"}, w + ".shape", err)) return false;
    if (!get_int(sh, "M", ent.M, w + ".shape", err) || !get_int(sh, "N", ent.N, w + ".shape", err) ||
        !get_int(sh, "K", ent.K, w + ".shape", err) ||
        !get_str(sh, "dtype", ent.dtype, w + ".shape", err))
      return false;
    const Json& b = *e.get("best");
    if (!expect_keys(b, {"block_m", "block_n", "block_k", "num_warps", "vector_width", "unroll",
                         "shared_memory_stages"},
                     w + ".best", err))
      return false;
    long long v[7];
    const char* names[7] = {"block_m", "block_n", "block_k", "num_warps", "vector_width", "unroll",
                            "shared_memory_stages"};
    for (int k = 0; k < 7; ++k)
      if (!get_int(b, names[k], v[k], w + ".best", err)) return false;
    ent.best = Config{static_cast<int>(v[0]), static_cast<int>(v[1]), static_cast<int>(v[2]),
                      static_cast<int>(v[3]), static_cast<int>(v[4]), static_cast<int>(v[5]),
                      static_cast<int>(v[6])};
    std::string scored;
    if (!get_str(e, "scored_by", scored, w, err)) return false;
    if (scored != "measure" && scored != "compile_time_model") {
      err = w + ".scored_by: must be \"measure\" or \"compile_time_model\"";
      return false;
    }
    const Json* tm = e.get("time_ms");
    if (tm->kind != Json::Null && tm->kind != Json::Num) {
      err = w + ".time_ms: expected a number or null";
      return false;
    }
    if ((tm->kind == Json::Null) != (scored == "compile_time_model")) {
      err = w + ".time_ms: null iff scored_by is \"compile_time_model\"";
      return false;
    }
    ent.scored_by = scored;
    ent.has_time = tm->kind == Json::Num;
    ent.time_ms = ent.has_time ? tm->num : 0;
    const Json* val = e.get("validated");
    if (val->kind != Json::Bool) {
      err = w + ".validated: expected a boolean";
      return false;
    }
    ent.validated = val->b;
    const Json& c = *e.get("correctness");
    if (!expect_keys(c, {"cosine", "max_rel_err", "pcc"}, w + ".correctness", err)) return false;
    if (!get_num(c, "cosine", w + ".correctness", err, &ent.cosine) ||
        !get_num(c, "max_rel_err", w + ".correctness", err, &ent.max_rel_err) ||
        !get_num(c, "pcc", w + ".correctness", err, &ent.pcc))
      return false;
    out.push_back(ent);
  }
  return true;
}

// ------------------------------------------------------------ serializer --
inline std::string json_string(const std::string& v) {
  std::string o = "\"";
  for (const char c : v) {
    switch (c) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\t': o += "\\t"; break;
      case '\r': o += "\\r"; break;
      default:
        if (static_cast<unsigned char>(c) < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof(buf), "\\u%04x", static_cast<unsigned char>(c));
          o += buf;
        } else {
          o += c;
        }
    }
  }
  return o + "\"";
}

inline std::string json_number(double v) {
  char buf[40];
  std::snprintf(buf, sizeof(buf), "%.17g", v);
  std::string s(buf);
  // keep it a JSON number that parses back as non-integer when it was one
  if (s.find_first_of(".eEn") == std::string::npos) s += ".0";
  return s;
}

inline std::string shape_json(const Entry& e) {
  return "{\"M\": " + std::to_string(e.M) + ", \"N\": " + std::to_string(e.N) +
         ", \"K\": " + std::to_string(e.K) + ", \"dtype\": " + json_string(e.dtype) + "}";
}

// A cache document in the schema parse_cache reads (version 1).
inline std::string serialize_cache(const std::vector<Entry>& entries) {
  std::string o = "{\n  \"version\": 1,\n  \"entries\": [";
  for (size_t i = 0; i < entries.size(); ++i) {
    const Entry& e = entries[i];
    const Config& b = e.best;
    o += i ? ",\n    {" : "\n    {";
    o += "\"gpu\": " + json_string(e.gpu) + ", \"op\": " + json_string(e.op) +
         ", \"shape\": " + shape_json(e) + ", \"best\": {\"block_m\": " +
         std::to_string(b.block_m) + ", \"block_n\": " + std::to_string(b.block_n) +
         ", \"block_k\": " + std::to_string(b.block_k) + ", \"num_warps\": " +
         std::to_string(b.num_warps) + ", \"vector_width\": " + std::to_string(b.vector_width) +
         ", \"unroll\": " + std::to_string(b.unroll) + ", \"shared_memory_stages\": " +
         std::to_string(b.shared_memory_stages) + "}, \"scored_by\": " +
         json_string(e.scored_by) + ", \"time_ms\": " +
         (e.has_time ? json_number(e.time_ms) : std::string("null")) +
         ", \"validated\": " + (e.validated ? "true" : "false") +
         ", \"correctness\": {\"cosine\": " + json_number(e.cosine) +
         ", \"max_rel_err\": " + json_number(e.max_rel_err) + ", \"pcc\": " +
         json_number(e.pcc) + "}}";
  }
  o += entries.empty() ? "]\n}\n" : "\n  ]\n}\n";
  return o;
}

}  // namespace tuning
}  // namespace pkb200
