// checkpoint.cu -- safetensors checkpoints in the reference's on-disk layout
// and the loader of one MoE layer into a handle (include/gmoe.h,
// gm_checkpoint_* and gm_moe_load_layer).
//
// File format (safetensors/parser.mojo, safetensors/writer.mojo:39-75): an
// 8-byte little-endian header length N (at most 100 MiB,
// safetensors/parser.mojo:17), N bytes of JSON mapping each tensor name to
// {"dtype", "shape", "data_offsets": [begin, end]} with offsets relative to
// the first byte after the header ("__metadata__" holds strings), padding
// spaces, then the data.
//
// One MoE layer's tensors (modeling/gemma4_topology.mojo:143-158, prefix
// "model.language_model.layers.{i}." at :259).  In the butterquant file every
// quantized slot is its int8 weight plus a ".scale" member
// (quant/manifest.mojo:10-13, 93-120); the ".colsum" member is not written
// (quant/quantizer.mojo:503), the reference derives it while VNNI-packing at
// load (modeling/slot.mojo:263-300) and these kernels need none:
//   experts.gate_up_proj           I8 [128*1408][2816], .scale F32 [128*1408]
//   experts.down_proj              I8 [128*2816][704],  .scale F32 [128*2816]
//   router.proj.weight             BF16 [128][2816] (centered in the bq file)
//   router.scale                   BF16 [2816]  (baked at load)
//   router.per_expert_scale        BF16 [128]
//   pre_feedforward_layernorm_2.weight BF16 [2816] (split gain baked for bq)
//   post_feedforward_layernorm{_1,_2,}.weight BF16 [2816], layer_scalar BF16 [1]
// The original bf16 checkpoint holds experts.gate_up_proj BF16
// [128][1408][2816] and experts.down_proj BF16 [128][2816][704].
#include <dirent.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <thread>
#include <vector>

#include "../../include/gmoe.h"
#include "gm_kernels.h"

using namespace gm;

namespace {

constexpr uint64_t MAX_HEADER_BYTES = 100ull << 20;

struct DtypeTag {
  const char* tag;
  int code;
  int bytes;
};
constexpr DtypeTag DTYPES[] = {
    {"BOOL", GM_DTYPE_BOOL, 1}, {"U8", GM_DTYPE_U8, 1},       {"I8", GM_DTYPE_I8, 1},
    {"I16", GM_DTYPE_I16, 2},   {"U16", GM_DTYPE_U16, 2},     {"F16", GM_DTYPE_F16, 2},
    {"BF16", GM_DTYPE_BF16, 2}, {"I32", GM_DTYPE_I32, 4},     {"U32", GM_DTYPE_U32, 4},
    {"F32", GM_DTYPE_F32, 4},   {"I64", GM_DTYPE_I64, 8},     {"U64", GM_DTYPE_U64, 8},
    {"F64", GM_DTYPE_F64, 8},   {"F8_E4M3", GM_DTYPE_F8_E4M3, 1}, {"F8_E5M2", GM_DTYPE_F8_E5M2, 1},
};

const DtypeTag* dtype_by_tag(const std::string& s) {
  for (const auto& d : DTYPES)
    if (s == d.tag) return &d;
  return nullptr;
}
const char* dtype_name(int code) {
  for (const auto& d : DTYPES)
    if (d.code == code) return d.tag;
  return "?";
}
int dtype_bytes(int code) {
  for (const auto& d : DTYPES)
    if (d.code == code) return d.bytes;
  return 0;
}

// Minimal JSON reader for safetensors headers: strings (with escapes),
// integers, and skipping of any other value.
struct Json {
  const char* start;
  const char* p;
  const char* e;
  std::string err;

  bool fail(const char* what) {
    if (err.empty()) {
      char b[160];
      snprintf(b, sizeof b, "%s at header byte %ld", what, (long)(p - start));
      err = b;
    }
    return false;
  }
  void ws() {
    while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool lit(char c) {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  bool expect(char c) {
    if (lit(c)) return true;
    char b[32];
    snprintf(b, sizeof b, "expected '%c'", c);
    return fail(b);
  }
  static void put_utf8(std::string& o, uint32_t cp) {
    if (cp < 0x80) {
      o.push_back((char)cp);
    } else if (cp < 0x800) {
      o.push_back((char)(0xC0 | (cp >> 6)));
      o.push_back((char)(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
      o.push_back((char)(0xE0 | (cp >> 12)));
      o.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
      o.push_back((char)(0x80 | (cp & 0x3F)));
    } else {
      o.push_back((char)(0xF0 | (cp >> 18)));
      o.push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
      o.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
      o.push_back((char)(0x80 | (cp & 0x3F)));
    }
  }
  bool hex4(uint32_t& v) {
    if (e - p < 4) return fail("truncated \\u escape");
    v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
      else return fail("bad \\u escape");
    }
    return true;
  }
  bool str(std::string& out) {
    ws();
    if (p >= e || *p != '"') return fail("expected a string");
    ++p;
    out.clear();
    while (p < e && *p != '"') {
      const unsigned char c = (unsigned char)*p++;
      if (c < 0x20) return fail("control character in a string");
      if (c >= 0x80) {  // a UTF-8 sequence (RFC 3629): well formed, or the header is refused
        int n;
        uint32_t cp;
        if (c >= 0xC2 && c <= 0xDF) n = 1, cp = c & 0x1Fu;
        else if (c >= 0xE0 && c <= 0xEF) n = 2, cp = c & 0x0Fu;
        else if (c >= 0xF0 && c <= 0xF4) n = 3, cp = c & 0x07u;
        else return fail("invalid UTF-8 in a string");
        if (e - p < n) return fail("invalid UTF-8 in a string");
        out.push_back((char)c);
        for (int i = 0; i < n; ++i) {
          const unsigned char t = (unsigned char)*p++;
          if ((t & 0xC0) != 0x80) return fail("invalid UTF-8 in a string");
          cp = (cp << 6) | (t & 0x3Fu);
          out.push_back((char)t);
        }
        if ((n == 2 && cp < 0x800) || (n == 3 && (cp < 0x10000 || cp > 0x10FFFF)) ||
            (cp >= 0xD800 && cp <= 0xDFFF))
          return fail("invalid UTF-8 in a string");
        continue;
      }
      if (c != '\\') {
        out.push_back((char)c);
        continue;
      }
      if (p >= e) break;
      const char k = *p++;
      switch (k) {
        case '"': case '\\': case '/': out.push_back(k); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'n': out.push_back('\n'); break;
        case 'r': out.push_back('\r'); break;
        case 't': out.push_back('\t'); break;
        case 'u': {
          uint32_t cp;
          if (!hex4(cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
            uint32_t lo;
            if (e - p < 2 || p[0] != '\\' || p[1] != 'u') return fail("lone surrogate");
            p += 2;
            if (!hex4(lo)) return false;
            if (lo < 0xDC00 || lo > 0xDFFF) return fail("bad surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp <= 0xDFFF) {
            return fail("lone surrogate");
          }
          put_utf8(out, cp);
          break;
        }
        default: return fail("bad escape");
      }
    }
    if (p >= e) return fail("unterminated string");
    ++p;
    return true;
  }
  bool integer(int64_t& v) {
    ws();
    bool neg = false;
    if (p < e && *p == '-') {
      neg = true;
      ++p;
    }
    if (p >= e || *p < '0' || *p > '9') return fail("expected an integer");
    uint64_t acc = 0;
    while (p < e && *p >= '0' && *p <= '9') {
      const uint64_t d = (uint64_t)(*p++ - '0');
      if (acc > (UINT64_MAX - d) / 10) return fail("integer overflow");
      acc = acc * 10 + d;
    }
    if (p < e && (*p == '.' || *p == 'e' || *p == 'E')) return fail("expected an integer, got a fraction");
    if (acc > (uint64_t)INT64_MAX) return fail("integer overflow");
    v = neg ? -(int64_t)acc : (int64_t)acc;
    return true;
  }
  bool skip(int depth = 0) {
    if (depth > 64) return fail("nesting too deep");
    ws();
    if (p >= e) return fail("unexpected end of header");
    const char c = *p;
    if (c == '"') {
      std::string s;
      return str(s);
    }
    if (c == '{') {
      ++p;
      if (lit('}')) return true;
      do {
        std::string k;
        if (!str(k) || !expect(':') || !skip(depth + 1)) return false;
      } while (lit(','));
      return expect('}');
    }
    if (c == '[') {
      ++p;
      if (lit(']')) return true;
      do {
        if (!skip(depth + 1)) return false;
      } while (lit(','));
      return expect(']');
    }
    const char* s = p;
    while (p < e && (isalnum((unsigned char)*p) || *p == '-' || *p == '+' || *p == '.')) ++p;
    if (p == s) return fail("unexpected character");
    const std::string tok(s, p);
    if (tok == "true" || tok == "false" || tok == "null") return true;
    if (tok[0] == '-' || (tok[0] >= '0' && tok[0] <= '9')) return true;
    return fail("bad literal");
  }
};

struct Tensor {
  int file = 0;
  int dtype = 0;
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;
  int64_t rows = 1, cols = 1;  // 2-D fold
};

struct File {
  std::string path;
  int fd = -1;
  uint64_t data_start = 0;
};

int fail_thread(int code, const char* fmt, ...) {
  char buf[640];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  set_thread_error(buf);
  return code;
}

}  // namespace

struct gm_checkpoint {
  std::vector<File> files;
  std::map<std::string, Tensor> tensors;  // name order
  std::vector<const std::string*> order;
  ~gm_checkpoint() {
    for (auto& f : files)
      if (f.fd >= 0) close(f.fd);
  }
};

namespace {

int pread_all(int fd, void* dst, size_t n, uint64_t off, const std::string& path) {
  char* d = static_cast<char*>(dst);
  while (n > 0) {
    const ssize_t r = pread(fd, d, n, (off_t)off);
    if (r < 0) {
      if (errno == EINTR) continue;
      return fail_thread(GM_EINVAL, "%s: read at %llu: %s", path.c_str(), (unsigned long long)off,
                         strerror(errno));
    }
    if (r == 0)
      return fail_thread(GM_EINVAL, "%s: unexpected end of file at %llu", path.c_str(),
                         (unsigned long long)off);
    d += r;
    off += (uint64_t)r;
    n -= (size_t)r;
  }
  return GM_OK;
}

int parse_entry(Json& j, Tensor& t, uint64_t data_bytes) {
  if (!j.expect('{')) return GM_EINVAL;
  bool have_dtype = false, have_shape = false, have_off = false;
  if (!j.lit('}')) {
    do {
      std::string key;
      if (!j.str(key) || !j.expect(':')) return GM_EINVAL;
      if (key == "dtype") {
        std::string tag;
        if (!j.str(tag)) return GM_EINVAL;
        const DtypeTag* d = dtype_by_tag(tag);
        if (!d) {
          j.fail(("unknown dtype \"" + tag + "\"").c_str());
          return GM_EINVAL;
        }
        t.dtype = d->code;
        have_dtype = true;
      } else if (key == "shape") {
        if (!j.expect('[')) return GM_EINVAL;
        t.shape.clear();
        if (!j.lit(']')) {
          do {
            int64_t v;
            if (!j.integer(v)) return GM_EINVAL;
            if (v < 0) {
              j.fail("negative dimension");
              return GM_EINVAL;
            }
            t.shape.push_back(v);
          } while (j.lit(','));
          if (!j.expect(']')) return GM_EINVAL;
        }
        if (t.shape.size() > GM_CKPT_MAX_DIMS) {
          j.fail("too many dimensions");
          return GM_EINVAL;
        }
        have_shape = true;
      } else if (key == "data_offsets") {
        int64_t b, e;
        if (!j.expect('[') || !j.integer(b) || !j.expect(',') || !j.integer(e) || !j.expect(']'))
          return GM_EINVAL;
        if (b < 0 || e < b || (uint64_t)e > data_bytes) {
          j.fail("data_offsets outside the file's data");
          return GM_EINVAL;
        }
        t.begin = (uint64_t)b;
        t.end = (uint64_t)e;
        have_off = true;
      } else if (!j.skip()) {
        return GM_EINVAL;
      }
    } while (j.lit(','));
    if (!j.expect('}')) return GM_EINVAL;
  }
  if (!have_dtype || !have_shape || !have_off) {
    j.fail("entry lacks dtype, shape or data_offsets");
    return GM_EINVAL;
  }
  // byte count = numel * element size (overflow-checked)
  unsigned __int128 numel = 1;
  for (int64_t d : t.shape) {
    numel *= (unsigned __int128)d;
    if (numel > ((unsigned __int128)1 << 62)) {
      j.fail("tensor too large");
      return GM_EINVAL;
    }
  }
  if (numel * (unsigned __int128)dtype_bytes(t.dtype) != (unsigned __int128)(t.end - t.begin)) {
    j.fail("data_offsets span differs from shape x dtype size");
    return GM_EINVAL;
  }
  if (t.shape.empty()) {
    t.rows = t.cols = 1;
  } else if (t.shape.size() == 1) {
    t.rows = t.shape[0];
    t.cols = 1;
  } else {
    t.cols = t.shape.back();
    t.rows = 1;
    for (size_t i = 0; i + 1 < t.shape.size(); ++i) t.rows *= t.shape[i];
  }
  return GM_OK;
}

int open_file(gm_checkpoint* ck, const std::string& path) {
  File f;
  f.path = path;
  f.fd = open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (f.fd < 0) return fail_thread(GM_EINVAL, "%s: %s", path.c_str(), strerror(errno));
  const int idx = (int)ck->files.size();
  ck->files.push_back(f);  // closed by the checkpoint from here on
  struct stat st;
  if (fstat(f.fd, &st) != 0) return fail_thread(GM_EINVAL, "%s: %s", path.c_str(), strerror(errno));
  const uint64_t size = (uint64_t)st.st_size;
  if (size < 8) return fail_thread(GM_EINVAL, "%s: %llu bytes, shorter than the header length",
                                   path.c_str(), (unsigned long long)size);
  unsigned char lenb[8];
  int rc = pread_all(f.fd, lenb, 8, 0, path);
  if (rc) return rc;
  uint64_t n = 0;
  for (int i = 7; i >= 0; --i) n = (n << 8) | lenb[i];
  if (n > MAX_HEADER_BYTES)
    return fail_thread(GM_EINVAL, "%s: header length %llu exceeds %llu", path.c_str(),
                       (unsigned long long)n, (unsigned long long)MAX_HEADER_BYTES);
  if (n > size - 8)
    return fail_thread(GM_EINVAL, "%s: header length %llu exceeds the file (%llu bytes)",
                       path.c_str(), (unsigned long long)n, (unsigned long long)size);
  std::string hdr(n, '\0');
  if ((rc = pread_all(f.fd, &hdr[0], n, 8, path))) return rc;
  ck->files[idx].data_start = 8 + n;
  const uint64_t data_bytes = size - 8 - n;
  Json j{hdr.data(), hdr.data(), hdr.data() + hdr.size(), {}};
  auto bad = [&](void) { return fail_thread(GM_EINVAL, "%s: header: %s", path.c_str(), j.err.c_str()); };
  if (!j.expect('{')) return bad();
  if (!j.lit('}')) {
    do {
      std::string name;
      if (!j.str(name) || !j.expect(':')) return bad();
      if (name == "__metadata__") {
        if (!j.skip()) return bad();
        continue;
      }
      Tensor t;
      t.file = idx;
      if (parse_entry(j, t, data_bytes)) return bad();
      if (ck->tensors.count(name))
        return fail_thread(GM_EINVAL, "%s: tensor \"%s\" appears twice in the checkpoint",
                           path.c_str(), name.c_str());
      ck->tensors.emplace(name, t);
    } while (j.lit(','));
    if (!j.expect('}')) return bad();
  }
  j.ws();
  if (j.p != j.e) {
    j.fail("trailing bytes after the header object");
    return bad();
  }
  return GM_OK;
}

bool ends_with(const std::string& s, const char* suf) {
  const size_t n = strlen(suf);
  return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

const Tensor* find(const gm_checkpoint* ck, const std::string& name) {
  auto it = ck->tensors.find(name);
  return it == ck->tensors.end() ? nullptr : &it->second;
}

// Byte range [off, off+n) of a tensor's data into host memory; large reads are
// split over a few threads (page cache / NVMe queues).
int read_bytes(const gm_checkpoint* ck, const Tensor& t, uint64_t off, size_t n, void* dst) {
  const File& f = ck->files[t.file];
  const uint64_t base = f.data_start + t.begin + off;
  constexpr size_t PIECE = 8u << 20;
  const int nthreads = (int)std::min<size_t>(4, (n + PIECE - 1) / PIECE);
  if (nthreads <= 1) return pread_all(f.fd, dst, n, base, f.path);
  std::vector<int> rcs(nthreads, GM_OK);
  std::vector<std::string> errs(nthreads);
  std::vector<std::thread> th;
  const size_t per = (n + nthreads - 1) / nthreads;
  for (int i = 0; i < nthreads; ++i) {
    const size_t b = per * i, e = std::min(n, b + per);
    if (b >= e) break;
    th.emplace_back([&, i, b, e] {
      rcs[i] = pread_all(f.fd, static_cast<char*>(dst) + b, e - b, base + b, f.path);
      if (rcs[i]) errs[i] = gm_last_error(nullptr);
    });
  }
  for (auto& x : th) x.join();
  for (int i = 0; i < nthreads; ++i)
    if (rcs[i]) {
      set_thread_error(errs[i].c_str());
      return rcs[i];
    }
  return GM_OK;
}

}  // namespace

extern "C" {

int gm_checkpoint_open(gm_checkpoint_t** out, const char* path) {
  if (!out || !path) return fail_thread(GM_EINVAL, "gm_checkpoint_open: NULL argument");
  *out = nullptr;
  struct stat st;
  if (stat(path, &st) != 0) return fail_thread(GM_EINVAL, "%s: %s", path, strerror(errno));
  auto* ck = new gm_checkpoint();
  int rc = GM_OK;
  if (S_ISDIR(st.st_mode)) {
    std::vector<std::string> names;
    if (DIR* d = opendir(path)) {
      while (dirent* ent = readdir(d)) {
        const std::string n = ent->d_name;
        if (ends_with(n, ".safetensors")) names.push_back(n);
      }
      closedir(d);
    } else {
      rc = fail_thread(GM_EINVAL, "%s: %s", path, strerror(errno));
    }
    std::sort(names.begin(), names.end());
    if (!rc && names.empty()) rc = fail_thread(GM_EINVAL, "%s: no .safetensors files", path);
    for (size_t i = 0; !rc && i < names.size(); ++i)
      rc = open_file(ck, std::string(path) + "/" + names[i]);
  } else {
    rc = open_file(ck, path);
  }
  if (rc) {
    delete ck;
    return rc;
  }
  for (const auto& kv : ck->tensors) ck->order.push_back(&kv.first);
  *out = ck;
  return GM_OK;
}

int gm_checkpoint_close(gm_checkpoint_t* ck) {
  delete ck;
  return GM_OK;
}

int gm_checkpoint_tensor_count(const gm_checkpoint_t* ck) { return ck ? (int)ck->order.size() : 0; }

const char* gm_checkpoint_tensor_name(const gm_checkpoint_t* ck, int index) {
  if (!ck || index < 0 || index >= (int)ck->order.size()) return nullptr;
  return ck->order[index]->c_str();
}

int gm_checkpoint_tensor_info(const gm_checkpoint_t* ck, const char* name, int* dtype, int* ndim,
                              int64_t* shape) {
  if (!ck || !name) return fail_thread(GM_EINVAL, "gm_checkpoint_tensor_info: NULL argument");
  const Tensor* t = find(ck, name);
  if (!t) return fail_thread(GM_EINVAL, "tensor \"%s\" not in the checkpoint", name);
  if (dtype) *dtype = t->dtype;
  if (ndim) *ndim = (int)t->shape.size();
  if (shape)
    for (size_t i = 0; i < t->shape.size(); ++i) shape[i] = t->shape[i];
  return GM_OK;
}

int gm_checkpoint_read_rows(const gm_checkpoint_t* ck, const char* name, int64_t row0,
                            int64_t nrows, void* dst, size_t dst_bytes) {
  if (!ck || !name || (!dst && nrows > 0))
    return fail_thread(GM_EINVAL, "gm_checkpoint_read_rows: NULL argument");
  const Tensor* t = find(ck, name);
  if (!t) return fail_thread(GM_EINVAL, "tensor \"%s\" not in the checkpoint", name);
  if (row0 < 0 || nrows < 0 || row0 > t->rows || nrows > t->rows - row0)
    return fail_thread(GM_EINVAL, "%s: rows [%lld, %lld) outside [0, %lld)", name, (long long)row0,
                       (long long)(row0 + nrows), (long long)t->rows);
  const uint64_t row_bytes = (uint64_t)t->cols * dtype_bytes(t->dtype);
  const uint64_t n = row_bytes * (uint64_t)nrows;
  if (dst_bytes < n)
    return fail_thread(GM_EINVAL, "%s: destination holds %zu bytes, %llu needed", name, dst_bytes,
                       (unsigned long long)n);
  if (n == 0) return GM_OK;
  return read_bytes(ck, *t, row_bytes * (uint64_t)row0, (size_t)n, dst);
}

}  // extern "C"

// ------------------------------------------------------------- layer load --
namespace {

// Pinned double buffer: the file read of one chunk overlaps the copy of the
// previous one to the device.
struct Stager {
  static constexpr size_t CHUNK = 32u << 20;
  void* buf[2] = {nullptr, nullptr};
  cudaEvent_t ev[2] = {nullptr, nullptr};
  bool busy[2] = {false, false};
  ~Stager() {
    for (int i = 0; i < 2; ++i) {
      if (ev[i]) {
        if (busy[i]) cudaEventSynchronize(ev[i]);
        cudaEventDestroy(ev[i]);
      }
      if (buf[i]) cudaFreeHost(buf[i]);
    }
  }
  cudaError_t init() {
    for (int i = 0; i < 2; ++i) {
      cudaError_t e = cudaHostAlloc(&buf[i], CHUNK, cudaHostAllocDefault);
      if (e != cudaSuccess) return e;
      if ((e = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming)) != cudaSuccess) return e;
    }
    return cudaSuccess;
  }
};

// Device allocations of one load, freed on every exit path.
struct DevTemps {
  std::vector<void*> ptrs;
  ~DevTemps() { release(); }
  void release() {
    for (void* p : ptrs) cudaFree(p);
    ptrs.clear();
  }
  template <typename T>
  cudaError_t alloc(T** p, size_t count) {
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), std::max<size_t>(count, 1) * sizeof(T));
    if (e == cudaSuccess) ptrs.push_back(*p);
    return e;
  }
};

struct Loader {
  gm_moe* h;
  const gm_checkpoint* ck;
  std::string prefix;
  cudaStream_t s = nullptr;
  Stager st;
  DevTemps tmp;

  int fail(int code, const char* fmt, ...) {
    char buf[640];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return handle_fail(h, code, buf);
  }
  int cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return GM_OK;
    return fail(e == cudaErrorMemoryAllocation ? GM_ENOMEM : GM_ECUDA, "load %s: %s", what,
                cudaGetErrorString(e));
  }
  // The tensor prefix+name, checked against a dtype, a 2-D fold [rows][cols]
  // (cols 0 = any) and, for vectors, an element count.
  int lookup(const char* name, int dtype, int64_t rows, int64_t cols, const Tensor** out) {
    const std::string full = prefix + name;
    const Tensor* t = find(ck, full);
    if (!t) return fail(GM_EINVAL, "tensor \"%s\" not in the checkpoint", full.c_str());
    if (t->dtype != dtype)
      return fail(GM_EINVAL, "%s: dtype %s, expected %s", full.c_str(), dtype_name(t->dtype),
                  dtype_name(dtype));
    if (cols == 0) {  // vector: any shape of `rows` elements
      if (t->rows * t->cols != rows)
        return fail(GM_EINVAL, "%s: %lld elements, expected %lld", full.c_str(),
                    (long long)(t->rows * t->cols), (long long)rows);
    } else if (t->rows != rows || t->cols != cols) {
      return fail(GM_EINVAL, "%s: shape folds to [%lld][%lld], expected [%lld][%lld]", full.c_str(),
                  (long long)t->rows, (long long)t->cols, (long long)rows, (long long)cols);
    }
    *out = t;
    return GM_OK;
  }
  // Bytes [off, off+n) of a tensor to device memory through the pinned buffers.
  int upload(const Tensor& t, uint64_t off, size_t n, void* dev, const char* what) {
    int rc;
    for (size_t done = 0, i = 0; done < n; i ^= 1) {
      const size_t c = std::min(Stager::CHUNK, n - done);
      if (st.busy[i] && (rc = cuda(cudaEventSynchronize(st.ev[i]), what))) return rc;
      st.busy[i] = false;
      if ((rc = read_bytes(ck, t, off + done, c, st.buf[i])))
        return fail(rc, "%s", gm_last_error(nullptr));
      if ((rc = cuda(cudaMemcpyAsync(static_cast<char*>(dev) + done, st.buf[i], c,
                                     cudaMemcpyHostToDevice, s), what)))
        return rc;
      if ((rc = cuda(cudaEventRecord(st.ev[i], s), what))) return rc;
      st.busy[i] = true;
      done += c;
    }
    return GM_OK;
  }
  // Elements [elem0, elem0+count) of a tensor (flat, row-major order) to a
  // new device buffer; a row block of a 2-D fold is elem0 = row0*cols.
  template <typename T>
  int to_device(const Tensor& t, int64_t elem0, int64_t count, T** dev, const char* what) {
    const uint64_t eb = (uint64_t)dtype_bytes(t.dtype);
    const size_t n = (size_t)(eb * (uint64_t)count);
    int rc;
    if ((rc = cuda(tmp.alloc(dev, (n + sizeof(T) - 1) / sizeof(T)), what))) return rc;
    return upload(t, eb * (uint64_t)elem0, n, *dev, what);
  }
  template <typename T>
  int whole(const Tensor& t, T** dev, const char* what) {
    return to_device(t, 0, t.rows * t.cols, dev, what);
  }
  // row-major int8 [rows][cols] -> a new VNNI-packed copy (butterquant/vnni.mojo:31-83)
  int pack(const uint8_t* rm, int64_t rows, int cols, int8_t** packed, const char* what) {
    int rc;
    if ((rc = cuda(tmp.alloc(packed, (size_t)rows * cols), what))) return rc;
    return cuda(launch_vnni_permute(reinterpret_cast<const int8_t*>(rm), rows, cols, *packed, 0, s), what);
  }
};

}  // namespace

extern "C" int gm_moe_load_layer(gm_moe_t* h, int layer, const gm_checkpoint_t* ck,
                                 int ckpt_layer, const char* prefix, int flags) {
  int device = 0, base = 0, epr = 0, num_layers = 0;
  int rc = handle_shard(h, &device, &base, &epr, &num_layers);
  if (rc) return rc;
  if (layer < 0 || layer >= num_layers)
    return handle_fail(h, GM_EINVAL, "layer out of range");
  if (!ck) return handle_fail(h, GM_EINVAL, "NULL checkpoint");
  if (flags & ~(GM_LOAD_POST | GM_LOAD_DENSE | GM_LOAD_QUANTIZE))
    return handle_fail(h, GM_EINVAL, "unknown load flags");
  Loader ld{h, ck, {}};
  {
    char buf[512];
    const char* fmt = prefix ? prefix : "model.language_model.layers.%d.";
    if (strstr(fmt, "%d")) {
      // only one integer conversion is honoured; anything else is literal text
      const char* at = strstr(fmt, "%d");
      snprintf(buf, sizeof buf, "%.*s%d%s", (int)(at - fmt), fmt, ckpt_layer, at + 2);
    } else {
      snprintf(buf, sizeof buf, "%s", fmt);
    }
    ld.prefix = buf;
  }
  if ((rc = ld.cuda(cudaSetDevice(device), "set device"))) return rc;
  const Tensor* gu;
  {
    const std::string full = ld.prefix + "experts.gate_up_proj";
    gu = find(ck, full);
    if (!gu) return ld.fail(GM_EINVAL, "tensor \"%s\" not in the checkpoint", full.c_str());
  }
  const bool bq = gu->dtype == GM_DTYPE_I8;
  if (!bq && gu->dtype != GM_DTYPE_BF16)
    return ld.fail(GM_EINVAL, "%sexperts.gate_up_proj: dtype %s, expected I8 (butterquant) or BF16",
                   ld.prefix.c_str(), dtype_name(gu->dtype));
  const bool quantize = (flags & GM_LOAD_QUANTIZE) != 0;
  if (quantize && bq)
    return ld.fail(GM_EINVAL, "GM_LOAD_QUANTIZE needs a BF16 checkpoint; this one is butterquant");
  if ((flags & GM_LOAD_DENSE) && !bq && !quantize)
    return ld.fail(GM_EINVAL, "the dense MLP runs in butterquant only: load a BF16 checkpoint's "
                   "dense MLP with GM_LOAD_QUANTIZE");
  // ---- every tensor is looked up (dtype and shape checked) before any transfer
  const Tensor *t_gu, *t_dn, *t_gus = nullptr, *t_dns = nullptr, *t_r, *t_rs, *t_pes, *t_g2;
  const int wdt = bq ? GM_DTYPE_I8 : GM_DTYPE_BF16;
  if ((rc = ld.lookup("experts.gate_up_proj", wdt, (int64_t)E * GU, H, &t_gu)) ||
      (rc = ld.lookup("experts.down_proj", wdt, (int64_t)E * H, I, &t_dn)) ||
      (rc = ld.lookup("router.proj.weight", GM_DTYPE_BF16, E, H, &t_r)) ||
      (rc = ld.lookup("router.scale", GM_DTYPE_BF16, H, 0, &t_rs)) ||
      (rc = ld.lookup("router.per_expert_scale", GM_DTYPE_BF16, E, 0, &t_pes)) ||
      (rc = ld.lookup("pre_feedforward_layernorm_2.weight", GM_DTYPE_BF16, H, 0, &t_g2)))
    return rc;
  if (bq && ((rc = ld.lookup("experts.gate_up_proj.scale", GM_DTYPE_F32, (int64_t)E * GU, 0, &t_gus)) ||
             (rc = ld.lookup("experts.down_proj.scale", GM_DTYPE_F32, (int64_t)E * H, 0, &t_dns))))
    return rc;
  const Tensor *t_p1 = nullptr, *t_p2 = nullptr, *t_p = nullptr, *t_ls = nullptr;
  if ((flags & GM_LOAD_POST) &&
      ((rc = ld.lookup("post_feedforward_layernorm_1.weight", GM_DTYPE_BF16, H, 0, &t_p1)) ||
       (rc = ld.lookup("post_feedforward_layernorm_2.weight", GM_DTYPE_BF16, H, 0, &t_p2)) ||
       (rc = ld.lookup("post_feedforward_layernorm.weight", GM_DTYPE_BF16, H, 0, &t_p)) ||
       (rc = ld.lookup("layer_scalar", GM_DTYPE_BF16, 1, 0, &t_ls))))
    return rc;
  const Tensor *t_dg = nullptr, *t_du = nullptr, *t_dd = nullptr, *t_dgs = nullptr, *t_dus = nullptr,
               *t_dds = nullptr, *t_pf = nullptr;
  if (flags & GM_LOAD_DENSE) {
    if ((rc = ld.lookup("mlp.gate_proj.weight", wdt, DENSE_I, H, &t_dg)) ||
        (rc = ld.lookup("mlp.up_proj.weight", wdt, DENSE_I, H, &t_du)) ||
        (rc = ld.lookup("mlp.down_proj.weight", wdt, H, DENSE_I, &t_dd)) ||
        (rc = ld.lookup("pre_feedforward_layernorm.weight", GM_DTYPE_BF16, H, 0, &t_pf)))
      return rc;
    if (bq && ((rc = ld.lookup("mlp.gate_proj.weight.scale", GM_DTYPE_F32, DENSE_I, 0, &t_dgs)) ||
               (rc = ld.lookup("mlp.up_proj.weight.scale", GM_DTYPE_F32, DENSE_I, 0, &t_dus)) ||
               (rc = ld.lookup("mlp.down_proj.weight.scale", GM_DTYPE_F32, H, 0, &t_dds))))
      return rc;
  }

  if ((rc = ld.cuda(cudaStreamCreateWithFlags(&ld.s, cudaStreamNonBlocking), "stream"))) return rc;
  struct StreamGuard {
    cudaStream_t& s;
    ~StreamGuard() {
      if (s) {
        cudaStreamSynchronize(s);
        cudaStreamDestroy(s);
      }
    }
  } sg{ld.s};
  if ((rc = ld.cuda(ld.st.init(), "pinned staging"))) return rc;

  // ---- experts: this rank's row block (modeling/loader.mojo:113-125)
  const int64_t gu_rows = (int64_t)epr * GU, dn_rows = (int64_t)epr * H;
  uint8_t *gu_w, *dn_w;  // int8 (bq) or bf16 bytes
  float *gu_s = nullptr, *dn_s = nullptr;
  uint16_t *router, *rs_raw, *pes, *g2_raw, *rs_baked, *g2_use;
  if ((rc = ld.to_device(*t_gu, (int64_t)base * GU * H, gu_rows * H, &gu_w, "gate_up")) ||
      (rc = ld.to_device(*t_dn, (int64_t)base * H * I, dn_rows * I, &dn_w, "down")) ||
      (rc = ld.whole(*t_r, &router, "router.proj")) ||
      (rc = ld.whole(*t_rs, &rs_raw, "router.scale")) ||
      (rc = ld.whole(*t_pes, &pes, "per_expert_scale")) ||
      (rc = ld.whole(*t_g2, &g2_raw, "pre_ffn_norm_2")))
    return rc;
  if (bq && ((rc = ld.to_device(*t_gus, (int64_t)base * GU, gu_rows, &gu_s, "gate_up.scale")) ||
             (rc = ld.to_device(*t_dns, (int64_t)base * H, dn_rows, &dn_s, "down.scale"))))
    return rc;
  // load-time transforms (router scale bake for every format)
  if ((rc = ld.cuda(ld.tmp.alloc(&rs_baked, H), "router scale")) ||
      (rc = ld.cuda(launch_bake(rs_raw, rs_baked, H, 1, ld.s), "router scale bake")))
    return rc;
  g2_use = g2_raw;
  int8_t *gu_p = nullptr, *dn_p = nullptr;
  uint16_t* router_use = router;
  if (quantize) {
    // the reference quantizer on the device (quant/quantizer.mojo:963-1051):
    // MoeGateUp = PerRowQuant(128, SplitGamma(pre_feedforward_layernorm_2)),
    // MoeDown = PerRowQuant(64), Router = SoftmaxRouterCenter
    int8_t *gq, *dq;
    if ((rc = ld.cuda(ld.tmp.alloc(&gq, (size_t)gu_rows * H), "gate_up quantize")) ||
        (rc = ld.cuda(ld.tmp.alloc(&gu_s, (size_t)gu_rows), "gate_up quantize")) ||
        (rc = ld.cuda(launch_quantize_rows(reinterpret_cast<const uint16_t*>(gu_w), gu_rows, H, g2_raw,
                                           128, gq, gu_s, ld.s), "gate_up quantize")) ||
        (rc = ld.cuda(ld.tmp.alloc(&dq, (size_t)dn_rows * I), "down quantize")) ||
        (rc = ld.cuda(ld.tmp.alloc(&dn_s, (size_t)dn_rows), "down quantize")) ||
        (rc = ld.cuda(launch_quantize_rows(reinterpret_cast<const uint16_t*>(dn_w), dn_rows, I, nullptr,
                                           64, dq, dn_s, ld.s), "down quantize")) ||
        (rc = ld.cuda(ld.tmp.alloc(&router_use, (size_t)E * H), "router center")) ||
        (rc = ld.cuda(launch_router_center(router, E, H, router_use, ld.s), "router center")))
      return rc;
    gu_w = reinterpret_cast<uint8_t*>(gq);
    dn_w = reinterpret_cast<uint8_t*>(dq);
  }
  if (bq || quantize) {
    if ((rc = ld.cuda(ld.tmp.alloc(&g2_use, H), "split gain")) ||
        (rc = ld.cuda(launch_bake(g2_raw, g2_use, H, 0, ld.s), "split gain bake")) ||
        (rc = ld.pack(gu_w, gu_rows, H, &gu_p, "gate_up pack")) ||
        (rc = ld.pack(dn_w, dn_rows, I, &dn_p, "down pack")))
      return rc;
  }
  if ((rc = ld.cuda(cudaStreamSynchronize(ld.s), "load"))) return rc;
  rc = (bq || quantize)
           ? gm_moe_register_layer_bq(h, layer, gu_p, gu_s, dn_p, dn_s, router_use, rs_baked, pes, g2_use)
           : gm_moe_register_layer_bf16(h, layer, gu_w, dn_w, router, rs_baked, pes, g2_use);
  if (rc) return rc;
  ld.tmp.release();  // the expert temporaries are no longer needed

  // ---- post-MoE gains
  if (flags & GM_LOAD_POST) {
    uint16_t *p1, *p2, *p;
    uint16_t ls_bits = 0;
    if ((rc = ld.whole(*t_p1, &p1, "post_ffn_norm_1")) ||
        (rc = ld.whole(*t_p2, &p2, "post_ffn_norm_2")) || (rc = ld.whole(*t_p, &p, "post_ffn_norm")))
      return rc;
    if ((rc = read_bytes(ck, *t_ls, 0, 2, &ls_bits))) return ld.fail(rc, "%s", gm_last_error(nullptr));
    if ((rc = ld.cuda(cudaStreamSynchronize(ld.s), "load"))) return rc;
    const uint32_t fbits = (uint32_t)ls_bits << 16;
    float ls;
    memcpy(&ls, &fbits, sizeof ls);
    if ((rc = gm_moe_register_post(h, layer, p1, p2, p, ls))) return rc;
  }

  // ---- dense MLP (modeling/gemma_4_moe_bq.mojo:749-783; DenseGateUp =
  // PerRowQuant(128, SplitGamma(pre_feedforward_layernorm)), DenseDown =
  // PerRowQuant(64), :113-116), replicated on every rank
  if (flags & GM_LOAD_DENSE) {
    uint8_t *dg, *du, *dd;
    float *dgs = nullptr, *dus = nullptr, *dds = nullptr;
    uint16_t *pf_raw, *pf;
    if ((rc = ld.whole(*t_dg, &dg, "mlp.gate_proj")) || (rc = ld.whole(*t_du, &du, "mlp.up_proj")) ||
        (rc = ld.whole(*t_dd, &dd, "mlp.down_proj")) ||
        (rc = ld.whole(*t_pf, &pf_raw, "pre_feedforward_layernorm")))
      return rc;
    if (bq && ((rc = ld.whole(*t_dgs, &dgs, "mlp.gate_proj.scale")) ||
               (rc = ld.whole(*t_dus, &dus, "mlp.up_proj.scale")) ||
               (rc = ld.whole(*t_dds, &dds, "mlp.down_proj.scale"))))
      return rc;
    if (quantize) {
      int8_t *gq, *uq, *dq;
      if ((rc = ld.cuda(ld.tmp.alloc(&gq, (size_t)DENSE_I * H), "dense quantize")) ||
          (rc = ld.cuda(ld.tmp.alloc(&dgs, DENSE_I), "dense quantize")) ||
          (rc = ld.cuda(launch_quantize_rows(reinterpret_cast<const uint16_t*>(dg), DENSE_I, H, pf_raw,
                                             128, gq, dgs, ld.s), "dense quantize")) ||
          (rc = ld.cuda(ld.tmp.alloc(&uq, (size_t)DENSE_I * H), "dense quantize")) ||
          (rc = ld.cuda(ld.tmp.alloc(&dus, DENSE_I), "dense quantize")) ||
          (rc = ld.cuda(launch_quantize_rows(reinterpret_cast<const uint16_t*>(du), DENSE_I, H, pf_raw,
                                             128, uq, dus, ld.s), "dense quantize")) ||
          (rc = ld.cuda(ld.tmp.alloc(&dq, (size_t)H * DENSE_I), "dense quantize")) ||
          (rc = ld.cuda(ld.tmp.alloc(&dds, H), "dense quantize")) ||
          (rc = ld.cuda(launch_quantize_rows(reinterpret_cast<const uint16_t*>(dd), H, DENSE_I, nullptr,
                                             64, dq, dds, ld.s), "dense quantize")))
        return rc;
      dg = reinterpret_cast<uint8_t*>(gq);
      du = reinterpret_cast<uint8_t*>(uq);
      dd = reinterpret_cast<uint8_t*>(dq);
    }
    int8_t *dgp, *dup, *ddp;
    if ((rc = ld.cuda(ld.tmp.alloc(&pf, H), "split gain")) ||
        (rc = ld.cuda(launch_bake(pf_raw, pf, H, 0, ld.s), "split gain bake")) ||
        (rc = ld.pack(dg, DENSE_I, H, &dgp, "gate_proj pack")) ||
        (rc = ld.pack(du, DENSE_I, H, &dup, "up_proj pack")) ||
        (rc = ld.pack(dd, H, DENSE_I, &ddp, "down_proj pack")))
      return rc;
    if ((rc = ld.cuda(cudaStreamSynchronize(ld.s), "load"))) return rc;
    if ((rc = gm_moe_register_dense_bq(h, layer, dgp, dgs, dup, dus, ddp, dds, pf))) return rc;
  }
  return GM_OK;
}
