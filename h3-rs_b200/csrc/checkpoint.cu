// checkpoint.cu -- ComfyUI safetensors checkpoints (weights.rs:23-139 SafeFile, :493-534 QLinear::load): the file
// header parsed natively, tensors read with pread and uploaded through pinned staging buffers on the caller's
// stream, and the per-layer quantization record (`<prefix>.comfy_quant`) decoded into a layer description.
//
// File format: 8-byte little-endian header length N, N bytes of JSON {name: {"dtype", "shape", "data_offsets"},
// "__metadata__": {...}}, then the data; offsets are relative to the end of the header.  Names lose the ComfyUI
// checkpoint prefix "model.diffusion_model." as the reference strips it.
#include <algorithm>
#include <cerrno>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <map>
#include <memory>
#include <string>
#include <sys/stat.h>
#include <unistd.h>
#include <utility>
#include <vector>
#include <cuda_runtime.h>
#include "../../include/h3q.h"

namespace h3q {
void set_last_error(const char* msg);
}

namespace {

h3q_status fail(h3q_status s, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  h3q::set_last_error(buf);
  return s;
}

// ------------------------------------------------------------------------------------------ a small JSON reader
struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0;
  bool is_uint = false;  // the number was written as a non-negative integer (exact in `u`)
  uint64_t u = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;

  const Json* get(const std::string& k) const {
    if (kind != Object) return nullptr;
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct Parser {
  const char* p;
  const char* end;
  std::string err;
  int depth = 0;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool fail_at(const char* what) {
    if (err.empty()) err = what;
    return false;
  }
  static void put_utf8(std::string& s, uint32_t c) {
    if (c < 0x80) s += (char)c;
    else if (c < 0x800) { s += (char)(0xC0 | (c >> 6)); s += (char)(0x80 | (c & 63)); }
    else if (c < 0x10000) { s += (char)(0xE0 | (c >> 12)); s += (char)(0x80 | ((c >> 6) & 63)); s += (char)(0x80 | (c & 63)); }
    else {
      s += (char)(0xF0 | (c >> 18)); s += (char)(0x80 | ((c >> 12) & 63));
      s += (char)(0x80 | ((c >> 6) & 63)); s += (char)(0x80 | (c & 63));
    }
  }
  bool hex4(uint32_t& v) {
    if (end - p < 4) return fail_at("truncated \\u escape");
    v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
      else return fail_at("bad \\u escape");
    }
    return true;
  }
  bool string(std::string& s) {
    if (p >= end || *p != '"') return fail_at("expected a string");
    ++p;
    while (p < end && *p != '"') {
      const char c = *p++;
      if ((unsigned char)c < 0x20) return fail_at("control character in a string");
      if (c != '\\') { s += c; continue; }
      if (p >= end) return fail_at("truncated escape");
      const char e = *p++;
      switch (e) {
        case '"': s += '"'; break;
        case '\\': s += '\\'; break;
        case '/': s += '/'; break;
        case 'b': s += '\b'; break;
        case 'f': s += '\f'; break;
        case 'n': s += '\n'; break;
        case 'r': s += '\r'; break;
        case 't': s += '\t'; break;
        case 'u': {
          uint32_t c1;
          if (!hex4(c1)) return false;
          if (c1 >= 0xD800 && c1 < 0xDC00 && end - p >= 6 && p[0] == '\\' && p[1] == 'u') {
            p += 2;
            uint32_t c2;
            if (!hex4(c2)) return false;
            if (c2 >= 0xDC00 && c2 < 0xE000) c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
            else return fail_at("bad surrogate pair");
          }
          put_utf8(s, c1);
          break;
        }
        default: return fail_at("bad escape");
      }
    }
    if (p >= end) return fail_at("unterminated string");
    ++p;
    return true;
  }
  bool number(Json& v) {
    const char* s = p;
    bool neg = false, integral = true;
    if (p < end && *p == '-') { neg = true; ++p; }
    if (p >= end || !((*p >= '0' && *p <= '9'))) return fail_at("bad number");
    uint64_t u = 0;
    bool overflow = false;
    while (p < end && *p >= '0' && *p <= '9') {
      const uint64_t d = (uint64_t)(*p - '0');
      if (u > (UINT64_MAX - d) / 10) overflow = true;
      else u = u * 10 + d;
      ++p;
    }
    if (p < end && *p == '.') {
      integral = false;
      ++p;
      while (p < end && *p >= '0' && *p <= '9') ++p;
    }
    if (p < end && (*p == 'e' || *p == 'E')) {
      integral = false;
      ++p;
      if (p < end && (*p == '+' || *p == '-')) ++p;
      while (p < end && *p >= '0' && *p <= '9') ++p;
    }
    v.kind = Json::Number;
    v.num = strtod(std::string(s, p).c_str(), nullptr);
    v.is_uint = integral && !neg && !overflow;
    v.u = v.is_uint ? u : 0;
    return true;
  }
  bool value(Json& v) {
    if (++depth > 64) return fail_at("nesting too deep");
    ws();
    if (p >= end) return fail_at("unexpected end of header");
    bool ok = true;
    if (*p == '{') {
      v.kind = Json::Object;
      ++p;
      ws();
      if (p < end && *p == '}') { ++p; --depth; return true; }
      for (;;) {
        ws();
        std::string k;
        if (!string(k)) return false;
        ws();
        if (p >= end || *p != ':') return fail_at("expected ':'");
        ++p;
        Json child;
        if (!value(child)) return false;
        v.obj.emplace_back(std::move(k), std::move(child));
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == '}') { ++p; break; }
        return fail_at("expected ',' or '}'");
      }
    } else if (*p == '[') {
      v.kind = Json::Array;
      ++p;
      ws();
      if (p < end && *p == ']') { ++p; --depth; return true; }
      for (;;) {
        Json child;
        if (!value(child)) return false;
        v.arr.push_back(std::move(child));
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == ']') { ++p; break; }
        return fail_at("expected ',' or ']'");
      }
    } else if (*p == '"') {
      v.kind = Json::String;
      ok = string(v.str);
    } else if (end - p >= 4 && !strncmp(p, "true", 4)) {
      v.kind = Json::Bool; v.b = true; p += 4;
    } else if (end - p >= 5 && !strncmp(p, "false", 5)) {
      v.kind = Json::Bool; v.b = false; p += 5;
    } else if (end - p >= 4 && !strncmp(p, "null", 4)) {
      v.kind = Json::Null; p += 4;
    } else {
      ok = number(v);
    }
    --depth;
    return ok;
  }
};

bool parse_json(const char* s, size_t n, Json& out, std::string& err) {
  Parser ps{s, s + n, {}};
  if (!ps.value(out)) { err = ps.err; return false; }
  ps.ws();
  // safetensors pads the header with spaces; anything else after the value is an error
  if (ps.p != ps.end) { err = "trailing characters after the header"; return false; }
  return true;
}

std::string to_text(const Json& v) {  // JSON text of a non-string metadata value (serde_json's to_string)
  switch (v.kind) {
    case Json::Null: return "null";
    case Json::Bool: return v.b ? "true" : "false";
    case Json::Number: {
      if (v.is_uint) return std::to_string(v.u);
      char b[64];
      snprintf(b, sizeof b, "%.17g", v.num);
      return b;
    }
    case Json::String: {
      std::string s = "\"";
      for (char c : v.str) {
        if (c == '"' || c == '\\') { s += '\\'; s += c; }
        else if ((unsigned char)c < 0x20) { char b[8]; snprintf(b, sizeof b, "\\u%04x", c); s += b; }
        else s += c;
      }
      return s + "\"";
    }
    case Json::Array: {
      std::string s = "[";
      for (size_t i = 0; i < v.arr.size(); ++i) s += (i ? "," : "") + to_text(v.arr[i]);
      return s + "]";
    }
    case Json::Object: {
      std::string s = "{";
      for (size_t i = 0; i < v.obj.size(); ++i) {
        Json k; k.kind = Json::String; k.str = v.obj[i].first;
        s += (i ? "," : "") + to_text(k) + ":" + to_text(v.obj[i].second);
      }
      return s + "}";
    }
  }
  return "";
}

// --------------------------------------------------------------------------------------------- the file itself
struct Dt { const char* name; int code; int size; };
const Dt kDtypes[] = {
    {"F32", H3Q_DT_F32, 4},   {"F16", H3Q_DT_F16, 2},         {"BF16", H3Q_DT_BF16, 2}, {"I8", H3Q_DT_I8, 1},
    {"U8", H3Q_DT_U8, 1},     {"F8_E4M3", H3Q_DT_F8_E4M3, 1}, {"BOOL", H3Q_DT_BOOL, 1}, {"I32", H3Q_DT_I32, 4},
    {"I64", H3Q_DT_I64, 8},   {"F64", H3Q_DT_F64, 8},
};

struct Tensor {
  int dtype = 0, esize = 1;
  std::vector<int64_t> shape;
  uint64_t start = 0, end = 0;  // relative to the data section
};

constexpr const char* kComfyPrefix = "model.diffusion_model.";
constexpr uint64_t kMaxHeader = 100ull << 20;  // the safetensors format's own header limit

}  // namespace

struct h3q_checkpoint {
  std::string path;
  int fd = -1;
  uint64_t file_size = 0, data_start = 0;
  std::map<std::string, Tensor> tensors;
  std::vector<std::string> names;  // sorted
  std::map<std::string, std::string> metadata;
  ~h3q_checkpoint() {
    if (fd >= 0) close(fd);
  }
};

namespace {

const Tensor* find(const h3q_checkpoint* f, const char* name) {
  if (!f || !name) return nullptr;
  auto it = f->tensors.find(name);
  return it == f->tensors.end() ? nullptr : &it->second;
}

h3q_status not_found(const h3q_checkpoint* f, const char* name) {
  return fail(H3Q_ERR_ARG, "tensor %s not found in %s", name ? name : "(null)", f ? f->path.c_str() : "(null)");
}

// pread the whole range or fail
bool read_all(int fd, void* dst, uint64_t n, uint64_t off) {
  uint8_t* d = static_cast<uint8_t*>(dst);
  while (n > 0) {
    const ssize_t r = pread(fd, d, n > (1u << 30) ? (1u << 30) : (size_t)n, (off_t)off);
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) return false;
    d += r;
    n -= (uint64_t)r;
    off += (uint64_t)r;
  }
  return true;
}

}  // namespace

extern "C" {

h3q_status h3q_checkpoint_open(const char* path, h3q_checkpoint** out) {
  if (!out) return fail(H3Q_ERR_ARG, "h3q_checkpoint_open: null output pointer");
  *out = nullptr;
  if (!path) return fail(H3Q_ERR_ARG, "h3q_checkpoint_open: null path");
  std::unique_ptr<h3q_checkpoint> f(new h3q_checkpoint);
  f->path = path;
  f->fd = open(path, O_RDONLY | O_CLOEXEC);
  if (f->fd < 0) return fail(H3Q_ERR_ARG, "opening %s: %s", path, strerror(errno));
  struct stat st;
  if (fstat(f->fd, &st) != 0) return fail(H3Q_ERR_ARG, "opening %s: %s", path, strerror(errno));
  f->file_size = (uint64_t)st.st_size;
  uint8_t lb[8];
  if (f->file_size < 8 || !read_all(f->fd, lb, 8, 0))
    return fail(H3Q_ERR_ARG, "%s: not a safetensors file (shorter than its 8-byte header length)", path);
  uint64_t n = 0;
  for (int i = 7; i >= 0; --i) n = (n << 8) | lb[i];
  if (n > kMaxHeader || n > f->file_size - 8)
    return fail(H3Q_ERR_ARG, "%s: header length %llu does not fit the file (%llu bytes)", path,
                (unsigned long long)n, (unsigned long long)f->file_size);
  std::string hdr(n, '\0');
  if (!read_all(f->fd, &hdr[0], n, 8)) return fail(H3Q_ERR_ARG, "%s: cannot read the header", path);
  f->data_start = 8 + n;
  Json root;
  std::string err;
  if (!parse_json(hdr.data(), hdr.size(), root, err)) return fail(H3Q_ERR_ARG, "%s: bad header JSON: %s", path, err.c_str());
  if (root.kind != Json::Object) return fail(H3Q_ERR_ARG, "%s: the header is not a JSON object", path);
  const uint64_t data_bytes = f->file_size - f->data_start;
  for (const auto& kv : root.obj) {
    if (kv.first == "__metadata__") {
      if (kv.second.kind == Json::Object)
        for (const auto& m : kv.second.obj)
          f->metadata[m.first] = m.second.kind == Json::String ? m.second.str : to_text(m.second);
      continue;
    }
    const Json& v = kv.second;
    const Json* dt = v.get("dtype");
    const Json* sh = v.get("shape");
    const Json* off = v.get("data_offsets");
    if (!dt || dt->kind != Json::String || !sh || sh->kind != Json::Array || !off || off->kind != Json::Array ||
        off->arr.size() != 2 || !off->arr[0].is_uint || !off->arr[1].is_uint)
      return fail(H3Q_ERR_ARG, "%s: tensor %s: malformed entry (dtype, shape, data_offsets)", path, kv.first.c_str());
    Tensor t;
    const Dt* d = nullptr;
    for (const auto& c : kDtypes)
      if (dt->str == c.name) d = &c;
    if (!d) return fail(H3Q_ERR_UNSUPPORTED, "unsupported safetensors dtype %s", dt->str.c_str());
    t.dtype = d->code;
    t.esize = d->size;
    if (sh->arr.size() > 8) return fail(H3Q_ERR_UNSUPPORTED, "%s: tensor %s has more than 8 dims", path, kv.first.c_str());
    uint64_t numel = 1;
    for (const auto& e : sh->arr) {
      if (!e.is_uint || e.u > (1ull << 48)) return fail(H3Q_ERR_ARG, "%s: tensor %s: bad shape", path, kv.first.c_str());
      t.shape.push_back((int64_t)e.u);
      numel = e.u == 0 ? 0 : (numel > UINT64_MAX / e.u ? UINT64_MAX : numel * e.u);
    }
    t.start = off->arr[0].u;
    t.end = off->arr[1].u;
    if (t.start > t.end || t.end > data_bytes)
      return fail(H3Q_ERR_ARG, "%s: tensor %s: data offsets [%llu, %llu) outside the %llu data bytes", path,
                  kv.first.c_str(), (unsigned long long)t.start, (unsigned long long)t.end,
                  (unsigned long long)data_bytes);
    if (numel == UINT64_MAX || numel * (uint64_t)t.esize != t.end - t.start)
      return fail(H3Q_ERR_ARG, "%s: tensor %s: %llu bytes for a %s tensor of %llu elements", path, kv.first.c_str(),
                  (unsigned long long)(t.end - t.start), dt->str.c_str(), (unsigned long long)numel);
    std::string name = kv.first;
    if (name.compare(0, strlen(kComfyPrefix), kComfyPrefix) == 0) name = name.substr(strlen(kComfyPrefix));
    f->tensors[name] = t;
  }
  for (const auto& kv : f->tensors) f->names.push_back(kv.first);
  *out = f.release();
  return H3Q_OK;
}

void h3q_checkpoint_close(h3q_checkpoint* f) { delete f; }

int64_t h3q_checkpoint_count(const h3q_checkpoint* f) { return f ? (int64_t)f->names.size() : 0; }

const char* h3q_checkpoint_name(const h3q_checkpoint* f, int64_t i) {
  if (!f || i < 0 || i >= (int64_t)f->names.size()) return nullptr;
  return f->names[(size_t)i].c_str();
}

const char* h3q_checkpoint_metadata(const h3q_checkpoint* f, const char* key) {
  if (!f || !key) return nullptr;
  auto it = f->metadata.find(key);
  return it == f->metadata.end() ? nullptr : it->second.c_str();
}

int h3q_checkpoint_has(const h3q_checkpoint* f, const char* name) { return find(f, name) ? 1 : 0; }

h3q_status h3q_checkpoint_info(const h3q_checkpoint* f, const char* name, int* dtype, int* ndim, int64_t* shape,
                               uint64_t* nbytes) {
  const Tensor* t = find(f, name);
  if (!t) return not_found(f, name);
  if (dtype) *dtype = t->dtype;
  if (ndim) *ndim = (int)t->shape.size();
  if (shape)
    for (size_t i = 0; i < t->shape.size(); ++i) shape[i] = t->shape[i];
  if (nbytes) *nbytes = t->end - t->start;
  return H3Q_OK;
}

h3q_status h3q_checkpoint_read(const h3q_checkpoint* f, const char* name, void* dst, uint64_t dst_bytes) {
  const Tensor* t = find(f, name);
  if (!t) return not_found(f, name);
  const uint64_t n = t->end - t->start;
  if (n == 0) return H3Q_OK;
  if (!dst || dst_bytes < n)
    return fail(H3Q_ERR_ARG, "h3q_checkpoint_read: %s needs %llu bytes, the buffer has %llu", name,
                (unsigned long long)n, (unsigned long long)dst_bytes);
  if (!read_all(f->fd, dst, n, f->data_start + t->start))
    return fail(H3Q_ERR_ARG, "%s: reading %s: %s", f->path.c_str(), name, strerror(errno));
  return H3Q_OK;
}

h3q_status h3q_checkpoint_upload(const h3q_checkpoint* f, const char* name, void* dst, uint64_t dst_bytes,
                                 int interleave_halves, void* stream) {
  const char* what = "h3q_checkpoint_upload";
  const Tensor* t = find(f, name);
  if (!t) return not_found(f, name);
  const uint64_t n = t->end - t->start;
  if (n == 0) return H3Q_OK;
  if (!dst || dst_bytes < n)
    return fail(H3Q_ERR_ARG, "%s: %s needs %llu bytes, the buffer has %llu", what, name, (unsigned long long)n,
                (unsigned long long)dst_bytes);
  uint64_t rows = 1, rb = n;
  if (interleave_halves) {
    if (t->shape.empty() || t->shape[0] < 2 || t->shape[0] % 2 != 0)
      return fail(H3Q_ERR_ARG, "%s: %s: interleaving (gate, up) rows needs an even first dimension", what, name);
    rows = (uint64_t)t->shape[0];
    rb = n / rows;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // two pinned staging buffers: the pread of one overlaps the host-to-device copy of the other
  const uint64_t kChunk = 16ull << 20;
  uint8_t* stage[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  h3q_status status = H3Q_OK;
  auto cuda_fail = [&](cudaError_t e, const char* op) {
    status = fail(H3Q_ERR_CUDA, "%s: %s: %s", what, op, cudaGetErrorString(e));
  };
  for (int b = 0; b < 2 && status == H3Q_OK; ++b) {
    cudaError_t e = cudaHostAlloc((void**)&stage[b], kChunk, cudaHostAllocDefault);
    if (e != cudaSuccess) { stage[b] = nullptr; cuda_fail(e, "pinned staging"); break; }
    e = cudaEventCreateWithFlags(&done[b], cudaEventDisableTiming);
    if (e != cudaSuccess) { done[b] = nullptr; cuda_fail(e, "event"); }
  }
  uint8_t* d = static_cast<uint8_t*>(dst);
  int k = 0;  // chunk counter
  // one piece: `len` file bytes from `foff` to the device at `doff`, or (rows_in_piece > 0) that many whole rows
  // placed every other row starting at device row `drow`
  auto piece = [&](uint64_t foff, uint64_t len, uint64_t doff, uint64_t nrows, uint64_t drow) {
    const int b = k++ & 1;
    cudaError_t e = cudaEventSynchronize(done[b]);
    if (e != cudaSuccess) { cuda_fail(e, "staging reuse"); return; }
    if (!read_all(f->fd, stage[b], len, f->data_start + t->start + foff)) {
      status = fail(H3Q_ERR_ARG, "%s: reading %s: %s", f->path.c_str(), name, strerror(errno));
      return;
    }
    if (nrows == 0) e = cudaMemcpyAsync(d + doff, stage[b], len, cudaMemcpyHostToDevice, st);
    else e = cudaMemcpy2DAsync(d + drow * rb, 2 * rb, stage[b], rb, rb, nrows, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) { cuda_fail(e, "host-to-device copy"); return; }
    e = cudaEventRecord(done[b], st);
    if (e != cudaSuccess) cuda_fail(e, "event record");
  };
  if (status == H3Q_OK) {
    if (!interleave_halves) {
      for (uint64_t o = 0; o < n && status == H3Q_OK; o += kChunk) piece(o, std::min(kChunk, n - o), o, 0, 0);
    } else {
      // interleave_swiglu (weights.rs:679-687, :765-800): gate row i -> row 2i, up row i -> row 2i + 1
      const uint64_t half = rows / 2;
      for (int hf = 0; hf < 2 && status == H3Q_OK; ++hf) {
        if (rb <= kChunk) {
          const uint64_t per = kChunk / rb;
          for (uint64_t r = 0; r < half && status == H3Q_OK; r += per) {
            const uint64_t nr = std::min(per, half - r);
            piece((hf * half + r) * rb, nr * rb, 0, nr, 2 * r + hf);
          }
        } else {
          for (uint64_t r = 0; r < half && status == H3Q_OK; ++r)
            for (uint64_t o = 0; o < rb && status == H3Q_OK; o += kChunk)
              piece((hf * half + r) * rb + o, std::min(kChunk, rb - o), (2 * r + hf) * rb + o, 0, 0);
        }
      }
    }
  }
  // the tensor is on the device (and the staging idle) when the call returns
  for (int b = 0; b < 2; ++b) {
    if (done[b]) {
      const cudaError_t e = cudaEventSynchronize(done[b]);
      if (e != cudaSuccess && status == H3Q_OK) cuda_fail(e, "completion");
      cudaEventDestroy(done[b]);
    }
    if (stage[b]) cudaFreeHost(stage[b]);
  }
  return status;
}

h3q_status h3q_checkpoint_qlinear(const h3q_checkpoint* f, const char* prefix, h3q_qlinear_spec* spec) {
  if (!f || !prefix || !spec) return fail(H3Q_ERR_ARG, "h3q_checkpoint_qlinear: null argument");
  memset(spec, 0, sizeof *spec);
  const std::string p = prefix;
  const Tensor* w = find(f, (p + ".weight").c_str());
  if (!w) return not_found(f, (p + ".weight").c_str());
  if (w->shape.size() != 2) return fail(H3Q_ERR_ARG, "%s.weight: expected a 2-D weight", prefix);
  spec->weight_dtype = w->dtype;
  spec->out_features = w->shape[0];
  spec->in_features = w->shape[1];
  spec->has_bias = find(f, (p + ".bias").c_str()) ? 1 : 0;
  const Tensor* cq = find(f, (p + ".comfy_quant").c_str());
  if (!cq) {
    spec->format = H3Q_FMT_DENSE;
    return H3Q_OK;
  }
  std::string text(cq->end - cq->start, '\0');
  if (!text.empty() && !read_all(f->fd, &text[0], text.size(), f->data_start + cq->start))
    return fail(H3Q_ERR_ARG, "%s: reading %s.comfy_quant", f->path.c_str(), prefix);
  Json conf;
  std::string err;
  if (!parse_json(text.data(), text.size(), conf, err) || conf.kind != Json::Object)
    return fail(H3Q_ERR_ARG, "%s.comfy_quant: bad JSON: %s", prefix, err.c_str());
  const Json* fmt = conf.get("format");
  if (!fmt || fmt->kind != Json::String) {  // the reference reads a missing format as a dense layer
    spec->format = H3Q_FMT_DENSE;
    return H3Q_OK;
  }
  auto scale_numel = [&](const char* suffix, int64_t& numel, int& dtype) -> h3q_status {
    const Tensor* s = find(f, (p + suffix).c_str());
    if (!s) return not_found(f, (p + suffix).c_str());
    numel = 1;
    for (int64_t e : s->shape) numel *= e;
    dtype = s->dtype;
    return H3Q_OK;
  };
  if (fmt->str == "int8_tensorwise") {
    spec->format = H3Q_FMT_INT8;
    const Json* cr = conf.get("convrot");
    if (cr && cr->kind == Json::Bool && cr->b) {
      const Json* g = conf.get("convrot_groupsize");
      spec->convrot = (g && g->is_uint) ? (int)g->u : 256;
    }
    return scale_numel(".weight_scale", spec->scale_numel, spec->scale_dtype);
  }
  if (fmt->str == "nvfp4") {
    spec->format = H3Q_FMT_NVFP4;
    spec->in_features = w->shape[1] * 2;
    int64_t gn;
    int gd;
    if (h3q_status s = scale_numel(".weight_scale_2", gn, gd)) return s;
    if (h3q_status s = scale_numel(".weight_scale", spec->scale_numel, spec->scale_dtype)) return s;
    spec->has_pre_quant_scale = find(f, (p + ".pre_quant_scale").c_str()) ? 1 : 0;
    return H3Q_OK;
  }
  return fail(H3Q_ERR_UNSUPPORTED, "%s: unsupported quantization format %s", prefix, fmt->str.c_str());
}

}  // extern "C"
