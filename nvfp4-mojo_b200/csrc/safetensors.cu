// safetensors.cu -- the safetensors reader of include/nvfp4_loader.h: header
// parsing, host and device reads, shard discovery, NVFP4 linear / stacked
// expert / router loading (restating nvfp4/weight_loader.mojo:190-410,
// :614-760, :826-954), with tensor bytes streamed from the file into device
// memory through two pinned staging buffers.
#include <cuda_runtime.h>
#include <dirent.h>
#include <errno.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <thread>
#include <vector>

#include "../../include/nvfp4.h"
#include "../../include/nvfp4_loader.h"
#include "abi_util.h"

struct nvfp4_st_file {
  std::string path;
  int fd = -1;
  int64_t file_size = 0, header_size = 0, data_start = 0;
  std::vector<std::string> names;
  std::vector<nvfp4_st_tensor_info> infos;
  std::map<std::string, int64_t> first_index;
  // Pinned staging for device reads, allocated on first use.
  void *stage[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  bool pending[2] = {false, false};
};

struct nvfp4_st_model {
  std::vector<nvfp4_st_file *> shards;
};

namespace nvfp4 {
namespace {

constexpr size_t kStageBytes = 32u << 20;  // per staging buffer
constexpr int kReadThreads = 4;            // file reads per chunk run in parallel

// ---------------------------------------------------------------------------
// JSON: the subset a safetensors header uses (objects, arrays, strings,
// integers), plus skipping of any other value (numbers, true/false/null) so
// that __metadata__ and unknown fields parse.
// ---------------------------------------------------------------------------
struct Json {
  const char *p, *end;
  std::string err;

  bool fail_at(const char *what) {
    if (err.empty()) err = what;
    return false;
  }
  void ws() {
    while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool expect(char c) {
    ws();
    if (p >= end || *p != c) return fail_at("unexpected character");
    ++p;
    return true;
  }
  bool peek(char c) {
    ws();
    return p < end && *p == c;
  }
  static void put_utf8(std::string &s, uint32_t cp) {
    if (cp < 0x80) {
      s += (char)cp;
    } else if (cp < 0x800) {
      s += (char)(0xC0 | (cp >> 6));
      s += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      s += (char)(0xE0 | (cp >> 12));
      s += (char)(0x80 | ((cp >> 6) & 0x3F));
      s += (char)(0x80 | (cp & 0x3F));
    } else {
      s += (char)(0xF0 | (cp >> 18));
      s += (char)(0x80 | ((cp >> 12) & 0x3F));
      s += (char)(0x80 | ((cp >> 6) & 0x3F));
      s += (char)(0x80 | (cp & 0x3F));
    }
  }
  bool hex4(uint32_t &v) {
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
  bool string(std::string &out) {
    if (!expect('"')) return false;
    out.clear();
    while (p < end && *p != '"') {
      if ((unsigned char)*p < 0x20) return fail_at("control character in string");
      if (*p != '\\') {
        out += *p++;
        continue;
      }
      if (++p >= end) return fail_at("truncated escape");
      const char c = *p++;
      switch (c) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case '/': out += '/'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'n': out += '\n'; break;
        case 'r': out += '\r'; break;
        case 't': out += '\t'; break;
        case 'u': {
          uint32_t cp;
          if (!hex4(cp)) return false;
          if (cp >= 0xDC00 && cp < 0xE000) return fail_at("lone low surrogate");
          if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
            uint32_t lo;
            if (end - p < 6 || p[0] != '\\' || p[1] != 'u') return fail_at("lone surrogate");
            p += 2;
            if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return fail_at("bad surrogate");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          put_utf8(out, cp);
          break;
        }
        default: return fail_at("bad escape");
      }
    }
    if (p >= end) return fail_at("unterminated string");
    ++p;
    return true;
  }
  // A non-negative integer (shapes and offsets).
  bool uint(int64_t &v) {
    ws();
    if (p >= end || *p < '0' || *p > '9') return fail_at("expected an unsigned integer");
    v = 0;
    while (p < end && *p >= '0' && *p <= '9') {
      if (v > (INT64_MAX - 9) / 10) return fail_at("integer overflow");
      v = v * 10 + (*p++ - '0');
    }
    if (p < end && (*p == '.' || *p == 'e' || *p == 'E')) return fail_at("expected an integer");
    return true;
  }
  bool uint_array(std::vector<int64_t> &out) {
    out.clear();
    if (!expect('[')) return false;
    if (peek(']')) {
      ++p;
      return true;
    }
    for (;;) {
      int64_t v;
      if (!uint(v)) return false;
      out.push_back(v);
      if (peek(',')) {
        ++p;
        continue;
      }
      return expect(']');
    }
  }
  bool skip(int depth = 0) {
    if (depth > 64) return fail_at("nesting too deep");
    ws();
    if (p >= end) return fail_at("truncated value");
    if (*p == '"') {
      std::string t;
      return string(t);
    }
    if (*p == '{' || *p == '[') {
      const char close = *p == '{' ? '}' : ']';
      const bool obj = *p == '{';
      ++p;
      if (peek(close)) {
        ++p;
        return true;
      }
      for (;;) {
        if (obj) {
          std::string k;
          if (!string(k) || !expect(':')) return false;
        }
        if (!skip(depth + 1)) return false;
        if (peek(',')) {
          ++p;
          continue;
        }
        return expect(close);
      }
    }
    const char *s = p;
    while (p < end && (isalnum((unsigned char)*p) || *p == '-' || *p == '+' || *p == '.')) ++p;
    if (p == s) return fail_at("unexpected character");
    return true;
  }
};

// Well-formed UTF-8 (RFC 3629: no overlong forms, no surrogates, at most
// U+10FFFF), which the safetensors format requires of its header.
bool valid_utf8(const char *s, size_t n) {
  const unsigned char *p = reinterpret_cast<const unsigned char *>(s), *e = p + n;
  while (p < e) {
    const unsigned c = *p;
    int len;
    unsigned cp;
    if (c < 0x80) {
      ++p;
      continue;
    } else if ((c & 0xE0) == 0xC0) {
      len = 2;
      cp = c & 0x1F;
    } else if ((c & 0xF0) == 0xE0) {
      len = 3;
      cp = c & 0x0F;
    } else if ((c & 0xF8) == 0xF0) {
      len = 4;
      cp = c & 0x07;
    } else {
      return false;
    }
    if (e - p < len) return false;
    for (int i = 1; i < len; ++i) {
      if ((p[i] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (p[i] & 0x3F);
    }
    if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000) ||
        cp > 0x10FFFF || (cp >= 0xD800 && cp < 0xE000))
      return false;
    p += len;
  }
  return true;
}

// _parse_safetensors_header (nvfp4/weight_loader.mojo:292-363): a flat object
// of name -> {dtype, shape, data_offsets}, `__metadata__` skipped, header
// order kept.  Missing fields default as in the reference (dtype "", shape
// [], data offsets 0/0).
int parse_header(const char *json, size_t n, int64_t data_bytes, nvfp4_st_file *f) {
  if (!valid_utf8(json, n))
    return fail(NVFP4_ERR_INVALID_ARG, "safetensors header is not valid UTF-8");
  Json j{json, json + n, {}};
  if (!j.expect('{')) return fail(NVFP4_ERR_INVALID_ARG, "safetensors header: %s", j.err.c_str());
  if (j.peek('}')) return NVFP4_OK;
  for (;;) {
    std::string name;
    if (!j.string(name) || !j.expect(':'))
      return fail(NVFP4_ERR_INVALID_ARG, "safetensors header: %s", j.err.c_str());
    if (name.find('\0') != std::string::npos)
      return fail(NVFP4_ERR_INVALID_ARG, "safetensors header: NUL character in a tensor name");
    if (name == "__metadata__") {
      if (!j.skip()) return fail(NVFP4_ERR_INVALID_ARG, "safetensors header: %s", j.err.c_str());
    } else {
      nvfp4_st_tensor_info info;
      memset(&info, 0, sizeof(info));
      std::vector<int64_t> shape, offs;
      if (!j.expect('{')) return fail(NVFP4_ERR_INVALID_ARG, "tensor %s: %s", name.c_str(), j.err.c_str());
      if (!j.peek('}')) {
        for (;;) {
          std::string key;
          if (!j.string(key) || !j.expect(':'))
            return fail(NVFP4_ERR_INVALID_ARG, "tensor %s: %s", name.c_str(), j.err.c_str());
          bool ok;
          if (key == "dtype") {
            std::string dt;
            ok = j.string(dt);
            if (ok && dt.find('\0') != std::string::npos)
              return fail(NVFP4_ERR_INVALID_ARG, "tensor %s: NUL character in dtype", name.c_str());
            if (ok && dt.size() >= sizeof(info.dtype))
              return fail(NVFP4_ERR_INVALID_ARG, "tensor %s: dtype too long", name.c_str());
            if (ok) memcpy(info.dtype, dt.c_str(), dt.size() + 1);
          } else if (key == "shape") {
            ok = j.uint_array(shape);
          } else if (key == "data_offsets") {
            ok = j.uint_array(offs);
          } else {
            ok = j.skip();
          }
          if (!ok) return fail(NVFP4_ERR_INVALID_ARG, "tensor %s: %s", name.c_str(), j.err.c_str());
          if (j.peek(',')) {
            ++j.p;
            continue;
          }
          if (!j.expect('}'))
            return fail(NVFP4_ERR_INVALID_ARG, "tensor %s: %s", name.c_str(), j.err.c_str());
          break;
        }
      } else {
        ++j.p;
      }
      if (shape.size() > 8) return fail(NVFP4_ERR_INVALID_ARG, "tensor %s: more than 8 dims", name.c_str());
      info.ndim = (int32_t)shape.size();
      for (size_t d = 0; d < shape.size(); ++d) info.shape[d] = shape[d];
      if (offs.size() >= 2) {
        if (offs[1] < offs[0] || offs[1] > data_bytes)
          return fail(NVFP4_ERR_INVALID_ARG, "tensor %s: data offsets [%lld, %lld] outside the %lld data bytes",
                      name.c_str(), (long long)offs[0], (long long)offs[1], (long long)data_bytes);
        info.data_offset = offs[0];
        info.data_size = offs[1] - offs[0];
      }
      f->first_index.emplace(name, (int64_t)f->names.size());
      f->names.push_back(name);
      f->infos.push_back(info);
    }
    if (j.peek(',')) {
      ++j.p;
      continue;
    }
    if (!j.expect('}')) return fail(NVFP4_ERR_INVALID_ARG, "safetensors header: %s", j.err.c_str());
    return NVFP4_OK;
  }
}

// pread until `count` bytes or end of file; -1 on an I/O error.
int64_t pread_full(int fd, void *dst, int64_t count, int64_t offset) {
  int64_t total = 0;
  while (total < count) {
    const ssize_t r = pread(fd, static_cast<uint8_t *>(dst) + total, (size_t)(count - total),
                            (off_t)(offset + total));
    if (r < 0) {
      if (errno == EINTR) continue;
      return -1;
    }
    if (r == 0) break;
    total += r;
  }
  return total;
}

// pread of `count` bytes split over up to kReadThreads threads (reads from
// the page cache scale with threads); false on a short read or an error.
bool pread_parallel(int fd, uint8_t *dst, int64_t count, int64_t offset) {
  const int64_t min_part = 4 << 20;
  const int parts = (int)std::min<int64_t>(kReadThreads, std::max<int64_t>(1, count / min_part));
  if (parts == 1) return pread_full(fd, dst, count, offset) == count;
  const int64_t step = (count + parts - 1) / parts;
  bool ok[kReadThreads] = {};
  std::vector<std::thread> th;
  for (int q = 1; q < parts; ++q) {
    const int64_t o = q * step, n = std::min(step, count - o);
    th.emplace_back([=, &ok] { ok[q] = pread_full(fd, dst + o, n, offset + o) == n; });
  }
  ok[0] = pread_full(fd, dst, std::min(step, count), offset) == std::min(step, count);
  for (auto &t : th) t.join();
  bool all = true;
  for (int q = 0; q < parts; ++q) all = all && ok[q];
  return all;
}

void release_staging(nvfp4_st_file *f) {
  for (int b = 0; b < 2; ++b) {
    if (f->done[b]) {
      if (f->pending[b]) cudaEventSynchronize(f->done[b]);
      cudaEventDestroy(f->done[b]);
      f->done[b] = nullptr;
    }
    if (f->stage[b]) {
      cudaFreeHost(f->stage[b]);
      f->stage[b] = nullptr;
    }
    f->pending[b] = false;
  }
}

bool tensor_ok(const nvfp4_st_file *f, int64_t i) {
  return f && i >= 0 && i < (int64_t)f->infos.size();
}

// Reads a whole tensor into a host vector.
int read_vec(const nvfp4_st_file *f, int64_t i, std::vector<uint8_t> &out) {
  out.resize((size_t)f->infos[i].data_size);
  const int64_t n = nvfp4_st_read_host(f, i, out.data(), (int64_t)out.size());
  return n < 0 ? (int)n : NVFP4_OK;
}

std::string join(const char *prefix, const char *suffix) { return std::string(prefix) + suffix; }

// First shard holding `name` (tensor index through *index).
int find_in(const nvfp4_st_model *m, const std::string &name, int32_t *shard, int64_t *index) {
  for (size_t s = 0; s < m->shards.size(); ++s) {
    const int64_t i = nvfp4_st_find(m->shards[s], name.c_str());
    if (i >= 0) {
      *shard = (int32_t)s;
      *index = i;
      return NVFP4_OK;
    }
  }
  return -1;
}

// fp32 router [H, E] from a BF16 or F32 [E, H] gate weight (32 x 32 tiles).
template <typename T>
__global__ void router_transpose_kernel(const T *__restrict__ w, float *__restrict__ out, int E,
                                        int H) {
  __shared__ float tile[32][33];
  const int h0 = blockIdx.x * 32, e0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int e = e0 + r, h = h0 + threadIdx.x;
    float v = 0.0f;
    if (e < E && h < H) {
      if constexpr (sizeof(T) == 2)
        v = __uint_as_float((uint32_t)w[(int64_t)e * H + h] << 16);
      else
        v = w[(int64_t)e * H + h];
    }
    tile[r][threadIdx.x] = v;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int h = h0 + r, e = e0 + threadIdx.x;
    if (h < H && e < E) out[(int64_t)h * E + e] = tile[threadIdx.x][r];
  }
}

struct LinearLoc {
  nvfp4_st_linear_info info;
  int64_t w, sf, ws2, ins;  // tensor indices in the shard (-1 if absent)
};

int locate_linear(const nvfp4_st_model *m, const char *prefix, LinearLoc *loc) {
  if (!m || !prefix || !loc) return fail(NVFP4_ERR_INVALID_ARG, "null model, prefix or output");
  int32_t shard = -1;
  int64_t wi = -1;
  if (find_in(m, join(prefix, ".weight"), &shard, &wi) != NVFP4_OK)
    return fail(NVFP4_ERR_INVALID_ARG, "No shard contains %s.weight", prefix);
  const nvfp4_st_file *f = m->shards[shard];
  const int64_t si = nvfp4_st_find(f, join(prefix, ".weight_scale").c_str());
  if (si < 0) return fail(NVFP4_ERR_INVALID_ARG, "Tensor not found: %s.weight_scale", prefix);
  const nvfp4_st_tensor_info &w = f->infos[wi];
  if (w.ndim < 2) return fail(NVFP4_ERR_INVALID_ARG, "Weight tensor must be 2D: %s.weight", prefix);
  LinearLoc L;
  L.w = wi;
  L.sf = si;
  L.info.out_features = w.shape[0];
  L.info.in_features = w.shape[1] * 2;
  L.info.shard = shard;
  const int64_t packed = L.info.out_features * (L.info.in_features / 2);
  const int64_t scales = L.info.out_features * (L.info.in_features / 16);
  if (w.data_size != packed)
    return fail(NVFP4_ERR_INVALID_ARG, "Weight read size mismatch for %s.weight: expected %lld, got %lld",
                prefix, (long long)packed, (long long)w.data_size);
  if (f->infos[si].data_size != scales)
    return fail(NVFP4_ERR_INVALID_ARG, "Scale read size mismatch for %s.weight_scale", prefix);
  L.ws2 = nvfp4_st_find(f, join(prefix, ".weight_scale_2").c_str());
  L.ins = nvfp4_st_find(f, join(prefix, ".input_scale").c_str());
  L.info.weight_scale_2 = 1.0f;
  L.info.input_scale = 1.0f;
  L.info.weight_scale_2_rows = 0;
  std::vector<uint8_t> b;
  if (L.ws2 >= 0) {
    int rc = read_vec(f, L.ws2, b);
    if (rc) return rc;
    L.info.weight_scale_2 = nvfp4_st_f32_from_bytes(b.data(), (int64_t)b.size());
    L.info.weight_scale_2_rows =
        L.info.out_features > 1 && (int64_t)b.size() == 4 * L.info.out_features;
  }
  if (L.ins >= 0) {
    int rc = read_vec(f, L.ins, b);
    if (rc) return rc;
    L.info.input_scale = nvfp4_st_f32_from_bytes(b.data(), (int64_t)b.size());
  }
  *loc = L;
  return NVFP4_OK;
}

// Per-row fp32 weight_scale_2 (optionally times input_scale) into device memory.
int load_ws2_rows(nvfp4_st_model *m, const LinearLoc &L, float *dst, bool fold, cudaStream_t st) {
  const nvfp4_st_file *f = m->shards[L.info.shard];
  const int64_t n = L.info.out_features;
  std::vector<float> rows((size_t)n, L.info.weight_scale_2);
  if (L.info.weight_scale_2_rows) {
    std::vector<uint8_t> b;
    int rc = read_vec(f, L.ws2, b);
    if (rc) return rc;
    for (int64_t r = 0; r < n; ++r) rows[r] = nvfp4_st_f32_from_bytes(b.data() + 4 * r, 4);
  }
  if (fold)
    for (auto &v : rows) v = v * L.info.input_scale;
  cudaError_t e = cudaMemcpyAsync(dst, rows.data(), sizeof(float) * n, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return check_launch(e, "weight_scale_2 upload");
}

int load_linear_at(nvfp4_st_model *m, const LinearLoc &L, uint8_t *w, uint8_t *sf, float *ws2,
                   bool fold, cudaStream_t st) {
  nvfp4_st_file *f = m->shards[L.info.shard];
  int rc = nvfp4_st_read_device(f, L.w, w, st);
  if (rc) return rc;
  if ((rc = nvfp4_st_read_device(f, L.sf, sf, st))) return rc;
  return ws2 ? load_ws2_rows(m, L, ws2, fold, st) : NVFP4_OK;
}

}  // namespace
}  // namespace nvfp4

using namespace nvfp4;

extern "C" float nvfp4_st_f32_from_bytes(const uint8_t *buf, int64_t len) {
  if (!buf || len < 4) return 1.0f;
  const uint32_t bits = (uint32_t)buf[0] | ((uint32_t)buf[1] << 8) | ((uint32_t)buf[2] << 16) |
                        ((uint32_t)buf[3] << 24);
  const uint32_t exp = (bits >> 23) & 0xFFu;
  if (exp == 0) return (bits >> 31) ? -0.0f : 0.0f;
  if (exp == 255) return 1.0f;
  float v;
  memcpy(&v, &bits, 4);
  return v;
}

extern "C" int nvfp4_st_open(const char *path, nvfp4_st_file **out) {
  if (!path || !out) return fail(NVFP4_ERR_INVALID_ARG, "null path or output handle");
  *out = nullptr;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return fail(NVFP4_ERR_INVALID_ARG, "Failed to open: %s (%s)", path, strerror(errno));
  struct stat sb;
  if (fstat(fd, &sb) != 0) {
    close(fd);
    return fail(NVFP4_ERR_INVALID_ARG, "Failed to stat: %s", path);
  }
  auto *f = new nvfp4_st_file();
  f->path = path;
  f->fd = fd;
  f->file_size = (int64_t)sb.st_size;
  uint8_t hb[8];
  if (pread_full(fd, hb, 8, 0) != 8) {
    nvfp4_st_close(f);
    return fail(NVFP4_ERR_INVALID_ARG, "Failed to read safetensors header size: %s", path);
  }
  uint64_t hs = 0;
  for (int i = 0; i < 8; ++i) hs |= (uint64_t)hb[i] << (8 * i);
  if (hs == 0 || hs > (uint64_t)(f->file_size - 8)) {
    nvfp4_st_close(f);
    return fail(NVFP4_ERR_INVALID_ARG, "Invalid safetensors header size: %llu", (unsigned long long)hs);
  }
  f->header_size = (int64_t)hs;
  f->data_start = 8 + f->header_size;
  std::vector<char> json((size_t)hs);
  if (pread_full(fd, json.data(), (int64_t)hs, 8) != (int64_t)hs) {
    nvfp4_st_close(f);
    return fail(NVFP4_ERR_INVALID_ARG, "Failed to read safetensors JSON header: %s", path);
  }
  const int rc = parse_header(json.data(), json.size(), f->file_size - f->data_start, f);
  if (rc) {
    nvfp4_st_close(f);
    return rc;
  }
  *out = f;
  return NVFP4_OK;
}

extern "C" void nvfp4_st_close(nvfp4_st_file *f) {
  if (!f) return;
  release_staging(f);
  if (f->fd >= 0) close(f->fd);
  delete f;
}

extern "C" int64_t nvfp4_st_num_tensors(const nvfp4_st_file *f) {
  return f ? (int64_t)f->infos.size() : 0;
}

extern "C" const char *nvfp4_st_tensor_name(const nvfp4_st_file *f, int64_t i) {
  return tensor_ok(f, i) ? f->names[i].c_str() : nullptr;
}

extern "C" int64_t nvfp4_st_find(const nvfp4_st_file *f, const char *name) {
  if (!f || !name) return -1;
  auto it = f->first_index.find(name);
  return it == f->first_index.end() ? -1 : it->second;
}

extern "C" int nvfp4_st_get_tensor_info(const nvfp4_st_file *f, int64_t i,
                                        nvfp4_st_tensor_info *out) {
  if (!tensor_ok(f, i) || !out) return fail(NVFP4_ERR_INVALID_ARG, "bad file handle, index or output");
  *out = f->infos[i];
  return NVFP4_OK;
}

extern "C" int64_t nvfp4_st_read_host(const nvfp4_st_file *f, int64_t i, void *dst, int64_t cap) {
  if (!tensor_ok(f, i)) return fail(NVFP4_ERR_INVALID_ARG, "bad file handle or tensor index");
  const nvfp4_st_tensor_info &t = f->infos[i];
  if (t.data_size == 0) return 0;
  if (!dst || cap < t.data_size)
    return fail(NVFP4_ERR_INVALID_ARG, "destination of %lld bytes for a tensor of %lld",
                (long long)cap, (long long)t.data_size);
  const int64_t n = pread_full(f->fd, dst, t.data_size, f->data_start + t.data_offset);
  if (n != t.data_size)
    return fail(NVFP4_ERR_INVALID_ARG, "short read of %s: %lld of %lld bytes", f->names[i].c_str(),
                (long long)n, (long long)t.data_size);
  return n;
}

extern "C" int nvfp4_st_read_device(nvfp4_st_file *f, int64_t i, void *dst, void *stream) {
  NVFP4_ABI_RANGE();
  if (!tensor_ok(f, i)) return fail(NVFP4_ERR_INVALID_ARG, "bad file handle or tensor index");
  const nvfp4_st_tensor_info &t = f->infos[i];
  if (t.data_size == 0) return NVFP4_OK;
  if (!dst) return fail(NVFP4_ERR_INVALID_ARG, "null destination");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int b = 0; b < 2; ++b) {
    if (!f->stage[b]) {
      int rc = check_launch(cudaHostAlloc(&f->stage[b], kStageBytes, cudaHostAllocDefault),
                            "pinned staging buffer");
      if (rc) return rc;
    }
    if (!f->done[b]) {
      int rc = check_launch(cudaEventCreateWithFlags(&f->done[b], cudaEventDisableTiming),
                            "staging event");
      if (rc) return rc;
    }
  }
  // Read chunk c into buffer c % 2 while the copy of chunk c - 1 runs.
  int64_t off = 0;
  int b = 0, rc = NVFP4_OK;
  while (off < t.data_size) {
    const int64_t n = std::min<int64_t>((int64_t)kStageBytes, t.data_size - off);
    if (f->pending[b]) {
      rc = check_launch(cudaEventSynchronize(f->done[b]), "staging copy");
      f->pending[b] = false;
      if (rc) break;
    }
    if (!pread_parallel(f->fd, static_cast<uint8_t *>(f->stage[b]), n,
                        f->data_start + t.data_offset + off)) {
      rc = fail(NVFP4_ERR_INVALID_ARG, "short read of %s", f->names[i].c_str());
      break;
    }
    cudaError_t e = cudaMemcpyAsync(static_cast<uint8_t *>(dst) + off, f->stage[b], (size_t)n,
                                    cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaEventRecord(f->done[b], st);
    if ((rc = check_launch(e, "staging copy"))) break;
    f->pending[b] = true;
    off += n;
    b ^= 1;
  }
  // The staging buffers are free again (and the bytes in place) on return.
  for (int q = 0; q < 2; ++q) {
    if (f->pending[q]) {
      const int r2 = check_launch(cudaEventSynchronize(f->done[q]), "staging copy");
      if (!rc) rc = r2;
      f->pending[q] = false;
    }
  }
  return rc;
}

extern "C" int nvfp4_st_open_model(const char *dir, nvfp4_st_model **out) {
  if (!dir || !out) return fail(NVFP4_ERR_INVALID_ARG, "null directory or output handle");
  *out = nullptr;
  std::vector<std::string> paths;
  const std::string single = std::string(dir) + "/model.safetensors";
  if (access(single.c_str(), R_OK) == 0) {
    paths.push_back(single);
  } else {
    // model-NNNNN-of-TTTTT.safetensors: totals that have a shard 1, smallest first.
    std::map<int, std::map<int, std::string>> by_total;
    DIR *d = opendir(dir);
    if (!d) return fail(NVFP4_ERR_INVALID_ARG, "No safetensors files found in %s", dir);
    while (struct dirent *e = readdir(d)) {
      int i = 0, tot = 0;
      char check[64];
      if (sscanf(e->d_name, "model-%5d-of-%5d.safetensors", &i, &tot) == 2 && i >= 1 && tot >= i) {
        snprintf(check, sizeof(check), "model-%05d-of-%05d.safetensors", i, tot);
        if (strcmp(check, e->d_name) == 0) by_total[tot][i] = std::string(dir) + "/" + e->d_name;
      }
    }
    closedir(d);
    for (auto &kv : by_total) {
      if (!kv.second.count(1)) continue;
      for (int i = 1; i <= kv.first && kv.second.count(i); ++i) paths.push_back(kv.second[i]);
      break;
    }
    if (paths.empty()) return fail(NVFP4_ERR_INVALID_ARG, "No safetensors files found in %s", dir);
  }
  std::vector<const char *> ps;
  for (const auto &p : paths) ps.push_back(p.c_str());
  return nvfp4_st_open_files(ps.data(), (int32_t)ps.size(), out);
}

extern "C" int nvfp4_st_open_files(const char *const *paths, int32_t n, nvfp4_st_model **out) {
  if (!paths || n <= 0 || !out) return fail(NVFP4_ERR_INVALID_ARG, "no files or null output handle");
  *out = nullptr;
  auto *m = new nvfp4_st_model();
  for (int32_t i = 0; i < n; ++i) {
    nvfp4_st_file *f = nullptr;
    const int rc = nvfp4_st_open(paths[i], &f);
    if (rc) {
      nvfp4_st_close_model(m);
      return rc;
    }
    m->shards.push_back(f);
  }
  *out = m;
  return NVFP4_OK;
}

extern "C" void nvfp4_st_close_model(nvfp4_st_model *m) {
  if (!m) return;
  for (auto *f : m->shards) nvfp4_st_close(f);
  delete m;
}

extern "C" int32_t nvfp4_st_model_num_shards(const nvfp4_st_model *m) {
  return m ? (int32_t)m->shards.size() : 0;
}

extern "C" const char *nvfp4_st_model_shard_path(const nvfp4_st_model *m, int32_t s) {
  return m && s >= 0 && s < (int32_t)m->shards.size() ? m->shards[s]->path.c_str() : nullptr;
}

extern "C" nvfp4_st_file *nvfp4_st_model_shard(nvfp4_st_model *m, int32_t s) {
  return m && s >= 0 && s < (int32_t)m->shards.size() ? m->shards[s] : nullptr;
}

extern "C" int nvfp4_st_model_find(const nvfp4_st_model *m, const char *name, int32_t *shard,
                                   int64_t *index) {
  if (!m || !name || !shard || !index) return fail(NVFP4_ERR_INVALID_ARG, "null argument");
  if (find_in(m, name, shard, index) == NVFP4_OK) return NVFP4_OK;
  *shard = -1;
  *index = -1;
  return fail(NVFP4_ERR_INVALID_ARG, "No shard contains %s", name);
}

extern "C" int nvfp4_st_get_linear_info(const nvfp4_st_model *m, const char *prefix,
                                        nvfp4_st_linear_info *out) {
  LinearLoc L;
  const int rc = locate_linear(m, prefix, &L);
  if (rc) return rc;
  *out = L.info;
  return NVFP4_OK;
}

extern "C" int nvfp4_st_load_linear(nvfp4_st_model *m, const char *prefix, uint8_t *w,
                                    uint8_t *sf, float *ws2, uint32_t flags, void *stream) {
  NVFP4_ABI_RANGE();
  if (!w || !sf) return fail(NVFP4_ERR_INVALID_ARG, "null weight or blockscale destination");
  LinearLoc L;
  const int rc = locate_linear(m, prefix, &L);
  if (rc) return rc;
  return load_linear_at(m, L, w, sf, ws2, (flags & NVFP4_ST_FOLD_INPUT_SCALE) != 0,
                        static_cast<cudaStream_t>(stream));
}

extern "C" int nvfp4_st_load_experts(nvfp4_st_model *m, const char *layer, int32_t first,
                                     int32_t count, int32_t shared, uint8_t *gate_up,
                                     uint8_t *gate_up_scale, float *gate_up_scale_2,
                                     uint8_t *down, uint8_t *down_scale, float *down_scale_2,
                                     void *stream) {
  NVFP4_ABI_RANGE();
  if (!m || !layer) return fail(NVFP4_ERR_INVALID_ARG, "null model or layer prefix");
  if (count <= 0 || first < 0 || (shared && (count != 1 || first != 0)))
    return fail(NVFP4_ERR_INVALID_ARG, "bad expert range");
  if (!gate_up || !gate_up_scale || !gate_up_scale_2 || !down || !down_scale || !down_scale_2)
    return fail(NVFP4_ERR_INVALID_ARG, "null destination");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int64_t I = -1, H = -1;
  for (int32_t e = 0; e < count; ++e) {
    char p[512];
    if (shared)
      snprintf(p, sizeof(p), "%s.mlp.shared_expert", layer);
    else
      snprintf(p, sizeof(p), "%s.mlp.experts.%d", layer, first + e);
    const std::string base = p;
    LinearLoc g, u, d;
    int rc = locate_linear(m, (base + ".gate_proj").c_str(), &g);
    if (!rc) rc = locate_linear(m, (base + ".up_proj").c_str(), &u);
    if (!rc) rc = locate_linear(m, (base + ".down_proj").c_str(), &d);
    if (rc) return rc;
    if (e == 0) {
      I = g.info.out_features;
      H = g.info.in_features;
    }
    if (g.info.out_features != I || g.info.in_features != H || u.info.out_features != I ||
        u.info.in_features != H || d.info.out_features != H || d.info.in_features != I)
      return fail(NVFP4_ERR_INVALID_ARG, "%s: gate/up [%lld, %lld] and down [%lld, %lld] shapes differ "
                  "from the first expert's", p, (long long)g.info.out_features,
                  (long long)g.info.in_features, (long long)d.info.out_features,
                  (long long)d.info.in_features);
    const int64_t gu0 = (int64_t)e * 2 * I;  // first stacked gate_up row of this expert
    if ((rc = load_linear_at(m, g, gate_up + gu0 * (H / 2), gate_up_scale + gu0 * (H / 16),
                             gate_up_scale_2 + gu0, true, st)))
      return rc;
    if ((rc = load_linear_at(m, u, gate_up + (gu0 + I) * (H / 2),
                             gate_up_scale + (gu0 + I) * (H / 16), gate_up_scale_2 + gu0 + I,
                             true, st)))
      return rc;
    const int64_t d0 = (int64_t)e * H;
    if ((rc = load_linear_at(m, d, down + d0 * (I / 2), down_scale + d0 * (I / 16),
                             down_scale_2 + d0, true, st)))
      return rc;
  }
  return NVFP4_OK;
}

extern "C" int nvfp4_st_load_router(nvfp4_st_model *m, const char *layer, float *router_out,
                                    int32_t *num_experts, int32_t *hidden, void *stream) {
  if (!m || !layer) return fail(NVFP4_ERR_INVALID_ARG, "null model or layer prefix");
  int32_t s;
  int64_t i;
  const std::string name = join(layer, ".mlp.gate.weight");
  if (find_in(m, name, &s, &i) != NVFP4_OK)
    return fail(NVFP4_ERR_INVALID_ARG, "No shard contains %s", name.c_str());
  nvfp4_st_file *f = m->shards[s];
  const nvfp4_st_tensor_info &t = f->infos[i];
  const bool bf16 = strcmp(t.dtype, "BF16") == 0, f32 = strcmp(t.dtype, "F32") == 0;
  if (t.ndim != 2 || (!bf16 && !f32) || t.data_size != t.shape[0] * t.shape[1] * (bf16 ? 2 : 4))
    return fail(NVFP4_ERR_INVALID_ARG, "%s: expected a BF16 or F32 [E, H] matrix", name.c_str());
  const int64_t E = t.shape[0], H = t.shape[1];
  if (E <= 0 || H <= 0 || E > (1 << 20) || H > (1 << 20))
    return fail(NVFP4_ERR_INVALID_ARG, "%s: bad shape", name.c_str());
  if (num_experts) *num_experts = (int32_t)E;
  if (hidden) *hidden = (int32_t)H;
  if (!router_out) return NVFP4_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void *tmp = nullptr;
  int rc = check_launch(cudaMalloc(&tmp, (size_t)t.data_size), "router staging");
  if (rc) return rc;
  rc = nvfp4_st_read_device(f, i, tmp, stream);
  if (!rc) {
    dim3 grid((unsigned)((H + 31) / 32), (unsigned)((E + 31) / 32)), block(32, 8);
    if (bf16)
      router_transpose_kernel<uint16_t><<<grid, block, 0, st>>>(static_cast<const uint16_t *>(tmp),
                                                                 router_out, (int)E, (int)H);
    else
      router_transpose_kernel<float><<<grid, block, 0, st>>>(static_cast<const float *>(tmp),
                                                              router_out, (int)E, (int)H);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    rc = check_launch(e, "router transpose");
  }
  cudaFree(tmp);
  return rc;
}
