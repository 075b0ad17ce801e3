// Checkpoint loading: safetensors files (single, or sharded with an index), the on-disk
// format the reference reads in src/weights.rs:27-210.
//
// Layout of a .safetensors file: an 8-byte little-endian header length N, N bytes of
// JSON mapping each tensor name to {"dtype", "shape", "data_offsets": [begin, end]}
// (offsets relative to the end of the header; "__metadata__" is not a tensor), then the
// raw little-endian data.  A sharded checkpoint adds model.safetensors.index.json whose
// "weight_map" maps tensor names to shard file names.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "context.h"
#include "model.h"

namespace wedlm {
namespace {

// ---- a small JSON reader (objects, arrays, strings, numbers, literals) -------------------
struct Json {
  enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
  double num = 0;
  bool b = false;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* get(const std::string& k) const {
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JsonReader {
  const char* p;
  const char* end;
  std::string err;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool fail(const char* what) {
    if (err.empty()) err = what;
    return false;
  }
  bool string(std::string* out) {
    if (p >= end || *p != '"') return fail("expected a string");
    ++p;
    out->clear();
    while (p < end && *p != '"') {
      char c = *p++;
      if (c == '\\') {
        if (p >= end) return fail("bad escape");
        const char e = *p++;
        switch (e) {
          case '"': case '\\': case '/': out->push_back(e); break;
          case 'b': out->push_back('\b'); break;
          case 'f': out->push_back('\f'); break;
          case 'n': out->push_back('\n'); break;
          case 'r': out->push_back('\r'); break;
          case 't': out->push_back('\t'); break;
          case 'u': {
            if (end - p < 4) return fail("bad \\u escape");
            unsigned v = 0;
            for (int i = 0; i < 4; ++i) {
              const char h = *p++;
              v <<= 4;
              if (h >= '0' && h <= '9') v |= (unsigned)(h - '0');
              else if (h >= 'a' && h <= 'f') v |= (unsigned)(h - 'a' + 10);
              else if (h >= 'A' && h <= 'F') v |= (unsigned)(h - 'A' + 10);
              else return fail("bad \\u escape");
            }
            // names are ASCII in practice; encode the code unit as UTF-8
            if (v < 0x80) out->push_back((char)v);
            else if (v < 0x800) {
              out->push_back((char)(0xC0 | (v >> 6)));
              out->push_back((char)(0x80 | (v & 0x3F)));
            } else {
              out->push_back((char)(0xE0 | (v >> 12)));
              out->push_back((char)(0x80 | ((v >> 6) & 0x3F)));
              out->push_back((char)(0x80 | (v & 0x3F)));
            }
            break;
          }
          default: return fail("bad escape");
        }
      } else {
        out->push_back(c);
      }
    }
    if (p >= end) return fail("unterminated string");
    ++p;
    return true;
  }
  bool value(Json* v, int depth) {
    if (depth > 64) return fail("JSON nested too deeply");
    ws();
    if (p >= end) return fail("unexpected end of JSON");
    const char c = *p;
    if (c == '{') {
      ++p;
      v->kind = Json::kObj;
      ws();
      if (p < end && *p == '}') {
        ++p;
        return true;
      }
      for (;;) {
        ws();
        std::string k;
        if (!string(&k)) return false;
        ws();
        if (p >= end || *p != ':') return fail("expected ':'");
        ++p;
        v->obj.emplace_back(k, Json());
        if (!value(&v->obj.back().second, depth + 1)) return false;
        ws();
        if (p < end && *p == ',') {
          ++p;
          continue;
        }
        if (p < end && *p == '}') {
          ++p;
          return true;
        }
        return fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      ++p;
      v->kind = Json::kArr;
      ws();
      if (p < end && *p == ']') {
        ++p;
        return true;
      }
      for (;;) {
        v->arr.emplace_back();
        if (!value(&v->arr.back(), depth + 1)) return false;
        ws();
        if (p < end && *p == ',') {
          ++p;
          continue;
        }
        if (p < end && *p == ']') {
          ++p;
          return true;
        }
        return fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v->kind = Json::kStr;
      return string(&v->str);
    }
    if (c == 't' && end - p >= 4 && !strncmp(p, "true", 4)) {
      p += 4;
      v->kind = Json::kBool;
      v->b = true;
      return true;
    }
    if (c == 'f' && end - p >= 5 && !strncmp(p, "false", 5)) {
      p += 5;
      v->kind = Json::kBool;
      return true;
    }
    if (c == 'n' && end - p >= 4 && !strncmp(p, "null", 4)) {
      p += 4;
      v->kind = Json::kNull;
      return true;
    }
    // number
    const char* q = p;
    while (q < end && *q != 0 && (std::strchr("+-.eE", *q) || (*q >= '0' && *q <= '9'))) ++q;
    if (q == p) return fail("unexpected character in JSON");
    v->kind = Json::kNum;
    try {
      v->num = std::stod(std::string(p, q));
    } catch (...) {
      return fail("bad number");
    }
    p = q;
    return true;
  }
};

Status parse_json(const char* text, size_t n, Json* out) {
  JsonReader r{text, text + n, {}};
  if (!r.value(out, 0))
    return Status::err(WEDLM_ERR_IO, "bad JSON: " + r.err + " at byte " +
                                         std::to_string(r.p - text));
  return Status::ok();
}

// ---- files ------------------------------------------------------------------------------
struct MappedFile {
  int fd = -1;
  void* base = MAP_FAILED;
  size_t size = 0;
  MappedFile() = default;
  MappedFile(const MappedFile&) = delete;
  MappedFile& operator=(const MappedFile&) = delete;
  ~MappedFile() {
    if (base != MAP_FAILED) munmap(base, size);
    if (fd >= 0) close(fd);
  }
  Status open_ro(const std::string& path) {
    fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) return Status::err(WEDLM_ERR_IO, "cannot open " + path);
    struct stat st;
    if (fstat(fd, &st) != 0) return Status::err(WEDLM_ERR_IO, "cannot stat " + path);
    size = (size_t)st.st_size;
    if (size == 0) return Status::err(WEDLM_ERR_IO, "empty file " + path);
    base = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (base == MAP_FAILED) return Status::err(WEDLM_ERR_IO, "cannot map " + path);
    return Status::ok();
  }
};

bool is_file(const std::string& path) {
  struct stat st;
  return stat(path.c_str(), &st) == 0 && S_ISREG(st.st_mode);
}

Status read_text(const std::string& path, std::string* out) {
  MappedFile f;
  WEDLM_TRY(f.open_ro(path));
  out->assign(static_cast<const char*>(f.base), f.size);
  return Status::ok();
}

// dtype name of a safetensors header -> ABI dtype code and element size (F64 is read
// as f64 and narrowed on the host; -1 = not a float type)
int st_dtype(const std::string& d, int* esz) {
  if (d == "BF16") { *esz = 2; return WEDLM_BF16; }
  if (d == "F16") { *esz = 2; return WEDLM_F16; }
  if (d == "F32") { *esz = 4; return WEDLM_F32; }
  if (d == "F64") { *esz = 8; return 100; }
  *esz = 0;
  return -1;
}

}  // namespace
}  // namespace wedlm

using wedlm::Status;

extern "C" int wedlm_load_weights(wedlm_ctx* ctx, const char* model_dir) {
  using namespace wedlm;
  if (!ctx) return WEDLM_ERR_INVALID_ARG;
  if (!ctx->has_model || !ctx->model)
    return ctx->fail(Status::err(WEDLM_ERR_STATE, "context has no model"));
  if (!model_dir) return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, "model_dir is NULL"));
  const std::string dir = model_dir;
  // the files to read: the index's shards (load_sharded_vb) or model.safetensors
  std::vector<std::string> files;
  const std::string index = dir + "/model.safetensors.index.json";
  if (is_file(index)) {
    std::string text;
    Status s = read_text(index, &text);
    Json j;
    if (s.good()) s = parse_json(text.data(), text.size(), &j);
    if (!s.good()) return ctx->fail(s);
    const Json* wm = j.kind == Json::kObj ? j.get("weight_map") : nullptr;
    if (!wm || wm->kind != Json::kObj)
      return ctx->fail(Status::err(WEDLM_ERR_IO, "index has no weight_map object"));
    std::set<std::string> seen;
    for (const auto& kv : wm->obj) {
      if (kv.second.kind != Json::kStr)
        return ctx->fail(Status::err(WEDLM_ERR_IO, "weight_map value is not a file name"));
      if (kv.second.str.find('/') != std::string::npos)
        return ctx->fail(Status::err(WEDLM_ERR_IO, "shard names must be plain file names"));
      if (seen.insert(kv.second.str).second) files.push_back(dir + "/" + kv.second.str);
    }
  } else if (is_file(dir + "/model.safetensors")) {
    files.push_back(dir + "/model.safetensors");
  } else {
    return ctx->fail(Status::err(WEDLM_ERR_NOT_FOUND,
                                 "No model.safetensors or model.safetensors.index.json found in " +
                                     dir));
  }

  const std::vector<std::string> names = model_weight_names(ctx->model);
  const std::set<std::string> needed(names.begin(), names.end());
  std::set<std::string> missing = needed;
  for (const std::string& path : files) {
    MappedFile f;
    Status s = f.open_ro(path);
    if (!s.good()) return ctx->fail(s);
    if (f.size < 8) return ctx->fail(Status::err(WEDLM_ERR_IO, path + ": too short"));
    const uint8_t* base = static_cast<const uint8_t*>(f.base);
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | base[i];
    if (hlen > f.size - 8) return ctx->fail(Status::err(WEDLM_ERR_IO, path + ": bad header length"));
    Json h;
    s = parse_json(reinterpret_cast<const char*>(base + 8), (size_t)hlen, &h);
    if (!s.good()) return ctx->fail(Status::err(s.code, path + ": " + s.msg));
    if (h.kind != Json::kObj) return ctx->fail(Status::err(WEDLM_ERR_IO, path + ": header is not an object"));
    const uint8_t* data = base + 8 + hlen;
    const uint64_t data_size = f.size - 8 - hlen;
    for (const auto& kv : h.obj) {
      const std::string& name = kv.first;
      if (name == "__metadata__" || !needed.count(name)) continue;  // extras are ignored
      const Json& t = kv.second;
      const Json* dt = t.get("dtype");
      const Json* sh = t.get("shape");
      const Json* off = t.get("data_offsets");
      if (!dt || dt->kind != Json::kStr || !sh || sh->kind != Json::kArr || !off ||
          off->kind != Json::kArr || off->arr.size() != 2)
        return ctx->fail(Status::err(WEDLM_ERR_IO, path + ": bad entry for " + name));
      int esz = 0;
      const int code = st_dtype(dt->str, &esz);
      if (code < 0)
        return ctx->fail(Status::err(WEDLM_ERR_UNSUPPORTED, name + ": unsupported dtype " + dt->str));
      std::vector<int64_t> shape;
      uint64_t numel = 1;
      for (const Json& d : sh->arr) {
        // dimensions are whole numbers below 2^62; their product must not wrap
        if (d.kind != Json::kNum || d.num < 0 || d.num >= 4.6e18 || d.num != (double)(uint64_t)d.num)
          return ctx->fail(Status::err(WEDLM_ERR_IO, path + ": bad shape of " + name));
        shape.push_back((int64_t)d.num);
        if (__builtin_mul_overflow(numel, (uint64_t)d.num, &numel))
          return ctx->fail(Status::err(WEDLM_ERR_IO, path + ": shape of " + name + " overflows"));
      }
      uint64_t nbytes = 0;
      if (__builtin_mul_overflow(numel, (uint64_t)esz, &nbytes))
        return ctx->fail(Status::err(WEDLM_ERR_IO, path + ": shape of " + name + " overflows"));
      // both offsets must be numbers before either value is read
      if (off->arr[0].kind != Json::kNum || off->arr[1].kind != Json::kNum ||
          off->arr[0].num < 0 || off->arr[1].num < 0 || off->arr[0].num >= 1.8e19 ||
          off->arr[1].num >= 1.8e19)
        return ctx->fail(Status::err(WEDLM_ERR_IO, path + ": bad data_offsets of " + name));
      const uint64_t b = (uint64_t)off->arr[0].num, e = (uint64_t)off->arr[1].num;
      if (b > e || e > data_size || e - b != nbytes)
        return ctx->fail(Status::err(WEDLM_ERR_IO, path + ": bad data_offsets of " + name));
      if (shape.empty() || shape.size() > 2)
        return ctx->fail(Status::err(WEDLM_ERR_INVALID_ARG, name + ": expected 1 or 2 dimensions"));
      const uint8_t* src = data + b;
      std::vector<float> conv;
      std::vector<uint64_t> aligned;
      int abi = code;
      if (code == 100) {  // f64: narrowed to f32 on the host
        conv.resize(numel);
        for (uint64_t i = 0; i < numel; ++i) {
          double v;
          memcpy(&v, src + i * 8, 8);
          conv[i] = (float)v;
        }
        src = reinterpret_cast<const uint8_t*>(conv.data());
        abi = WEDLM_F32;
      } else if (((uintptr_t)src % (uintptr_t)esz) != 0) {  // unaligned data: copy it out
        aligned.resize((numel * esz + 7) / 8);
        memcpy(aligned.data(), src, numel * esz);
        src = reinterpret_cast<const uint8_t*>(aligned.data());
      }
      const int rc = wedlm_set_weight(ctx, name.c_str(), src, abi, shape.data(), (int)shape.size());
      if (rc != WEDLM_OK) return rc;
      missing.erase(name);
    }
  }
  if (!missing.empty())
    return ctx->fail(Status::err(WEDLM_ERR_NOT_FOUND,
                                 "checkpoint lacks " + *missing.begin() +
                                     (missing.size() > 1 ? " (and " + std::to_string(missing.size() - 1) +
                                                               " more)"
                                                         : std::string())));
  return WEDLM_OK;
}

