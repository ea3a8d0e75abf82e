// Safetensors checkpoints straight to the device (Weights::open, src/checkpoint.rs:315-396,
// and the tensor reads of Model::open, src/model.rs:418-451).
//
// A checkpoint directory holds model.safetensors, or model.safetensors.index.json whose
// weight_map names the shard files. Every shard is memory-mapped and its header validated
// as the reference does it (header size, dtypes F32/BF16/F16, shapes against byte extents,
// duplicate names, overlapping extents, shard paths of one component); then every tensor
// on the AR decode path is uploaded. BF16 matrices go through two pinned staging buffers:
// the host copies a chunk out of the mapping while the previous chunk's asynchronous copy
// to the device runs. Norm gains and F32/F16 matrices are converted on the host first,
// exactly as yue2_model_set_tensor converts them.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "../../include/yue2_cuda.h"
#include "detmath.h"
#include "engine.h"

namespace y2 {
namespace {

// ---------------------------------------------------------------- a small JSON reader
struct Json {
  enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
  double num = 0;
  bool b = false;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;  // in file order
  const Json* get(const std::string& k) const {
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct JsonReader {
  const char* p;
  const char* end;
  int depth = 0;
  bool ok = true;
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool lit(const char* s) {
    const size_t n = strlen(s);
    if ((size_t)(end - p) < n || memcmp(p, s, n)) return false;
    p += n;
    return true;
  }
  bool string(std::string& out) {
    if (p >= end || *p != '"') return false;
    ++p;
    while (p < end && *p != '"') {
      if (*p == '\\') {
        if (++p >= end) return false;
        switch (*p) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u': {  // code points below 0x80 only (tensor names and dtypes are ASCII)
            if (end - p < 5) return false;
            unsigned v = 0;
            for (int i = 1; i <= 4; ++i) {
              const char c = p[i];
              v = v * 16 + (c >= '0' && c <= '9' ? c - '0' : c >= 'a' && c <= 'f' ? c - 'a' + 10
                                                       : c >= 'A' && c <= 'F' ? c - 'A' + 10 : 99);
              if (v > 0xffff) return false;
            }
            if (v >= 0x80) return false;
            out += (char)v;
            p += 4;
            break;
          }
          default: return false;
        }
        ++p;
      } else {
        out += *p++;
      }
    }
    if (p >= end) return false;
    ++p;
    return true;
  }
  bool value(Json& v) {
    if (++depth > 64) return false;
    ws();
    if (p >= end) return false;
    bool r = true;
    if (*p == '{') {
      v.kind = Json::kObj;
      ++p;
      ws();
      if (p < end && *p == '}') {
        ++p;
      } else {
        for (;;) {
          ws();
          std::string k;
          if (!string(k)) { r = false; break; }
          ws();
          if (p >= end || *p != ':') { r = false; break; }
          ++p;
          Json child;
          if (!value(child)) { r = false; break; }
          v.obj.emplace_back(std::move(k), std::move(child));
          ws();
          if (p < end && *p == ',') { ++p; continue; }
          if (p < end && *p == '}') { ++p; break; }
          r = false;
          break;
        }
      }
    } else if (*p == '[') {
      v.kind = Json::kArr;
      ++p;
      ws();
      if (p < end && *p == ']') {
        ++p;
      } else {
        for (;;) {
          Json child;
          if (!value(child)) { r = false; break; }
          v.arr.push_back(std::move(child));
          ws();
          if (p < end && *p == ',') { ++p; continue; }
          if (p < end && *p == ']') { ++p; break; }
          r = false;
          break;
        }
      }
    } else if (*p == '"') {
      v.kind = Json::kStr;
      r = string(v.str);
    } else if (lit("true")) {
      v.kind = Json::kBool;
      v.b = true;
    } else if (lit("false")) {
      v.kind = Json::kBool;
    } else if (lit("null")) {
      v.kind = Json::kNull;
    } else {
      v.kind = Json::kNum;
      char* e = nullptr;
      std::string tok;
      while (p < end && (strchr("+-.eE", *p) || (*p >= '0' && *p <= '9'))) tok += *p++;
      if (tok.empty()) return false;
      v.num = strtod(tok.c_str(), &e);
      r = e && *e == '\0';
    }
    --depth;
    return r;
  }
};

bool parse_json(const char* data, size_t n, Json& out) {
  JsonReader rd{data, data + n};
  if (!rd.value(out)) return false;
  rd.ws();
  return rd.p == rd.end;
}

// a non-negative integer JSON number (shapes and offsets)
bool as_size(const Json& v, uint64_t& out) {
  if (v.kind != Json::kNum || !(v.num >= 0) || v.num > 9007199254740992.0 || v.num != (double)(uint64_t)v.num)
    return false;
  out = (uint64_t)v.num;
  return true;
}

// ---------------------------------------------------------------- shards
struct Mapping {
  void* addr = nullptr;
  size_t size = 0;
  ~Mapping() {
    if (addr && addr != MAP_FAILED) munmap(addr, size);
  }
};

struct Entry {
  std::shared_ptr<Mapping> map;
  size_t offset = 0;  // of the tensor's first byte in the mapping
  int dtype = 0;      // YUE2_DTYPE_*
  std::vector<uint64_t> shape;
  uint64_t count = 0;
};

int invalid(const std::string& msg) { return fail(YUE2_ERR_INVALID, msg); }

int open_shard(const std::string& path, std::map<std::string, Entry>& out) {
  const int fd = open(path.c_str(), O_RDONLY);
  if (fd < 0) return invalid("Cannot open checkpoint shard " + path);
  struct stat st;
  if (fstat(fd, &st) != 0) {
    close(fd);
    return invalid("Cannot stat checkpoint shard " + path);
  }
  auto map = std::make_shared<Mapping>();
  map->size = (size_t)st.st_size;
  if (map->size < 8) {
    close(fd);
    return invalid("Short safetensors file");
  }
  map->addr = mmap(nullptr, map->size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (map->addr == MAP_FAILED) return invalid("Cannot map checkpoint shard " + path);
  const unsigned char* bytes = (const unsigned char*)map->addr;
  uint64_t header = 0;
  for (int i = 7; i >= 0; --i) header = header << 8 | bytes[i];
  if (header > 100000000ull || header > map->size - 8) return invalid("Invalid safetensors header size");
  const size_t data = 8 + (size_t)header;
  Json root;
  if (!parse_json((const char*)bytes + 8, (size_t)header, root) || root.kind != Json::kObj)
    return invalid("Invalid safetensors header");
  std::vector<std::pair<uint64_t, uint64_t>> ranges;
  for (auto& kv : root.obj) {
    const std::string& name = kv.first;
    if (name == "__metadata__") continue;
    const Json& v = kv.second;
    const Json* dt = v.get("dtype");
    const Json* shape = v.get("shape");
    const Json* offs = v.get("data_offsets");
    if (v.kind != Json::kObj || !dt || dt->kind != Json::kStr || !shape || shape->kind != Json::kArr || !offs ||
        offs->kind != Json::kArr)
      return invalid("Invalid safetensors entry " + name);
    Entry e;
    if (dt->str == "F32") e.dtype = YUE2_DTYPE_F32;
    else if (dt->str == "BF16") e.dtype = YUE2_DTYPE_BF16;
    else if (dt->str == "F16") e.dtype = YUE2_DTYPE_F16;
    else return invalid("Unsupported dtype " + dt->str + " for " + name);
    uint64_t count = 1;
    for (auto& d : shape->arr) {
      uint64_t x;
      if (!as_size(d, x)) return invalid("Invalid shape for " + name);
      if (x && count > UINT64_MAX / x) return invalid("Tensor size overflow");
      count *= x;
      e.shape.push_back(x);
    }
    if (offs->arr.size() != 2) return invalid("Invalid tensor offsets");
    uint64_t a, b;
    if (!as_size(offs->arr[0], a) || !as_size(offs->arr[1], b)) return invalid("Invalid tensor offsets");
    const uint64_t width = e.dtype == YUE2_DTYPE_F32 ? 4 : 2;
    if (count > UINT64_MAX / width) return invalid("Tensor bytes overflow");
    if (b < a || b > map->size - data || b - a != count * width) return invalid("Invalid tensor extent " + name);
    ranges.push_back({a, b});
    e.map = map;
    e.offset = data + (size_t)a;
    e.count = count;
    if (!out.emplace(name, std::move(e)).second) return invalid("Duplicate tensor " + name);
  }
  std::sort(ranges.begin(), ranges.end());
  for (size_t i = 1; i < ranges.size(); ++i)
    if (ranges[i - 1].second > ranges[i].first) return invalid("Overlapping safetensors tensors");
  return 0;
}

int read_file(const std::string& path, std::string& out) {
  const int fd = open(path.c_str(), O_RDONLY);
  if (fd < 0) return invalid("Cannot open " + path);
  char buf[1 << 16];
  ssize_t n;
  while ((n = read(fd, buf, sizeof buf)) > 0) out.append(buf, (size_t)n);
  close(fd);
  return n < 0 ? invalid("Cannot read " + path) : 0;
}

// Weights::open: the shard files of a checkpoint directory, then every tensor entry.
int scan_checkpoint(const std::string& dir, std::map<std::string, Entry>& out) {
  std::vector<std::string> files;
  const std::string index = dir + "/model.safetensors.index.json";
  if (access(index.c_str(), F_OK) == 0) {
    std::string text;
    int rc = read_file(index, text);
    if (rc) return rc;
    Json root;
    if (!parse_json(text.data(), text.size(), root) || root.kind != Json::kObj)
      return invalid("Invalid checkpoint index");
    const Json* wm = root.get("weight_map");
    if (!wm || wm->kind != Json::kObj) return invalid("Invalid checkpoint index");
    std::set<std::string> names;
    for (auto& kv : wm->obj) {
      if (kv.second.kind != Json::kStr) return invalid("Invalid checkpoint index");
      names.insert(kv.second.str);
    }
    for (auto& f : names) {
      if (f.empty() || f.find('/') != std::string::npos || f == "." || f == "..") return invalid("Invalid shard path");
      files.push_back(f);
    }
  } else {
    files.push_back("model.safetensors");
  }
  for (auto& f : files) {
    const int rc = open_shard(dir + "/" + f, out);
    if (rc) return rc;
  }
  return 0;
}

float bf16_value(uint16_t b) { return det_u2f((uint32_t)b << 16); }
float half_value(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31, exp = (h >> 10) & 0x1f, man = h & 0x3ff;
  if (exp == 0) {
    if (man == 0) return det_u2f(sign);
    const float v = (float)man * (1.0f / 16777216.0f);
    return sign ? -v : v;
  }
  if (exp == 31) return det_u2f(sign | 0x7f800000u | (man << 13));
  return det_u2f(sign | ((exp + 112) << 23) | (man << 13));
}
float value_at(const Entry& e, size_t i) {
  const unsigned char* p = (const unsigned char*)e.map->addr + e.offset;
  if (e.dtype == YUE2_DTYPE_F32) {
    float f;
    memcpy(&f, p + 4 * i, 4);
    return f;
  }
  uint16_t h;
  memcpy(&h, p + 2 * i, 2);
  return e.dtype == YUE2_DTYPE_BF16 ? bf16_value(h) : half_value(h);
}

// Two pinned staging buffers and a copy stream: chunk k is copied out of the mapping into
// buffer k % 2 while chunk k - 1's device copy runs.
struct Stager {
  static constexpr size_t kChunk = 32u << 20;
  unsigned char* pin[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  cudaStream_t stream = nullptr;
  int next = 0;
  uint64_t bytes = 0;
  int init() {
    for (int i = 0; i < 2; ++i) {
      if (cudaMallocHost((void**)&pin[i], kChunk) != cudaSuccess ||
          cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming) != cudaSuccess)
        return cuda_fail(cudaGetLastError(), "checkpoint staging");
    }
    cudaError_t e = cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking);
    return e == cudaSuccess ? 0 : cuda_fail(e, "checkpoint stream");
  }
  int put(void* dst, const void* src, size_t n) {
    const unsigned char* s = (const unsigned char*)src;
    unsigned char* d = (unsigned char*)dst;
    for (size_t off = 0; off < n; off += kChunk) {
      const size_t len = std::min(kChunk, n - off);
      const int b = next;
      next ^= 1;
      cudaError_t e = cudaEventSynchronize(done[b]);  // the buffer's previous copy finished
      if (e != cudaSuccess) return cuda_fail(e, "checkpoint staging");
      memcpy(pin[b], s + off, len);
      if ((e = cudaMemcpyAsync(d + off, pin[b], len, cudaMemcpyHostToDevice, stream)) != cudaSuccess ||
          (e = cudaEventRecord(done[b], stream)) != cudaSuccess)
        return cuda_fail(e, "checkpoint upload");
      bytes += len;
    }
    return 0;
  }
  int finish() {
    const cudaError_t e = stream ? cudaStreamSynchronize(stream) : cudaSuccess;
    return e == cudaSuccess ? 0 : cuda_fail(e, "checkpoint upload");
  }
  ~Stager() {
    if (stream) {
      cudaStreamSynchronize(stream);
      cudaStreamDestroy(stream);
    }
    for (int i = 0; i < 2; ++i) {
      if (done[i]) cudaEventDestroy(done[i]);
      if (pin[i]) cudaFreeHost(pin[i]);
    }
  }
};

}  // namespace
}  // namespace y2

using namespace y2;

extern "C" {

int yue2_checkpoint_scan(const char* dir, uint64_t* tensors) {
  if (!dir) return fail(YUE2_ERR_INVALID, "null argument");
  std::map<std::string, Entry> entries;
  const int rc = scan_checkpoint(dir, entries);
  if (rc) return rc;
  if (tensors) *tensors = entries.size();
  return 0;
}

int yue2_model_load_checkpoint(Yue2Model* m, const char* dir, uint64_t* bytes_uploaded) {
  if (m && m->tp_world > 1)
    return fail(YUE2_ERR_INVALID, "a tensor-parallel model takes its shard through yue2_model_set_tensor");
  if (!m || !dir) return fail(YUE2_ERR_INVALID, "null argument");
  std::map<std::string, Entry> entries;
  int rc = scan_checkpoint(dir, entries);
  if (rc) return rc;
  if ((rc = y2_set_device(m))) return rc;
  Stager st;
  if ((rc = st.init())) return rc;
  std::vector<float> f32;
  std::vector<uint16_t> b16;
  for (auto& kv : entries) {
    auto it = m->slots.find(kv.first);
    if (it == m->slots.end()) continue;  // not on the AR decode path (NAR, latent, VAE bridges)
    const Entry& e = kv.second;
    const TensorSlot& t = it->second;
    const uint64_t rows = e.shape.size() > 1 ? e.shape[0] : 1;
    const uint64_t cols = e.shape.size() > 1 ? e.count / std::max<uint64_t>(1, e.shape[0]) : e.count;
    if (e.count != t.rows * t.cols || (!t.norm && (rows != t.rows || cols != t.cols)))
      return fail(YUE2_ERR_INVALID, "Tensor shape mismatch for " + kv.first);
    void* dst = m->slot_addr(t);
    // put() copies its source into pinned memory before it returns, so the host vectors
    // below may be refilled for the next tensor at once
    if (t.norm) {  // Norm::new: gains rounded to bf16 (src/tensor.rs:1126-1136), f32 on the device
      f32.resize(e.count);
      for (size_t i = 0; i < e.count; ++i) f32[i] = round_bf16(value_at(e, i));
      if ((rc = st.put(dst, f32.data(), e.count * 4))) return rc;
    } else if (e.dtype == YUE2_DTYPE_BF16) {
      if ((rc = st.put(dst, (const unsigned char*)e.map->addr + e.offset, e.count * 2))) return rc;
    } else {  // F32/F16 checkpoints are rounded to bf16 (src/tensor.rs:436-438)
      b16.resize(e.count);
      for (size_t i = 0; i < e.count; ++i) b16[i] = (uint16_t)(det_f2u(round_bf16(value_at(e, i))) >> 16);
      if ((rc = st.put(dst, b16.data(), e.count * 2))) return rc;
    }
    m->loaded.insert(kv.first);
    m->finalized = false;
  }
  if ((rc = st.finish())) return rc;
  if (bytes_uploaded) *bytes_uploaded = st.bytes;
  return 0;
}

}  // extern "C"
