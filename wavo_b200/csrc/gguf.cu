// GGUF v3 reader (src/gguf.rs): the header with metadata values decoded when asked (a vocabulary
// nobody reads costs nothing, as in the reference), the tensor table, and tensor data read from the
// file in pieces. Host code; the device side of a GGUF load (the raw F32 / F16 / Q8_0 bytes turned
// into every device form a linear layer uses, pre-tiled for the TMA loads) is build_linear_kernel
// below, and wavo_linear_from_gguf (wavo_cuda.cu) streams a stacked layer from the file into it.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <functional>
#include <mutex>
#include <new>
#include <thread>

#include "../../include/wavo_cuda.h"
#include "gguf.cuh"
#include "kernels.cuh"

namespace {

// Bounds-checked little-endian reads over the header bytes (src/gguf.rs:306-393 `Reader`).
struct Reader {
  const uint8_t *b;
  size_t n, pos;
  bool take(size_t k, const uint8_t **out) {
    if (k > n - pos || pos > n) return false;
    *out = b + pos;
    pos += k;
    return true;
  }
  template <typename T>
  bool get(T *v) {
    const uint8_t *p;
    if (!take(sizeof(T), &p)) return false;
    std::memcpy(v, p, sizeof(T));
    return true;
  }
  bool bytes(const uint8_t **p, uint64_t *len) { return get(len) && take(size_t(*len), p); }
  // Moves past a value of GGUF type `ty` (0-12); false if truncated or of an unknown type.
  bool skip(uint32_t ty, int depth = 0) {
    const uint8_t *p;
    uint64_t len;
    switch (ty) {
      case 0: case 1: case 7: return take(1, &p);
      case 2: case 3: return take(2, &p);
      case 4: case 5: case 6: return take(4, &p);
      case 10: case 11: case 12: return take(8, &p);
      case 8: return bytes(&p, &len);
      case 9: {
        uint32_t item;
        uint64_t count;
        if (depth > 4 || !get(&item) || !get(&count)) return false;
        const int size = item <= 1 || item == 7 ? 1 : item <= 3 ? 2 : item <= 6 ? 4
                         : (item >= 10 && item <= 12) ? 8 : 0;
        if (size) return count <= (n - pos) / size && take(size_t(count) * size, &p);
        for (uint64_t i = 0; i < count; ++i)
          if (!skip(item, depth + 1)) return false;
        return true;
      }
      default: return false;
    }
  }
};

// A decoded scalar: the reference's `Value` (src/gguf.rs:40-56).
struct Value {
  enum Kind { Int, Float, Bool, Str, Array, Bad } kind = Bad;
  int64_t i = 0;
  double f = 0.0;
  const char *s = nullptr;
  uint64_t len = 0;     // string bytes, or array items
  uint32_t item = 0;    // array item type
};

bool read_value(Reader &r, uint32_t ty, Value &v) {
  uint8_t u8v; int8_t i8v; uint16_t u16v; int16_t i16v; uint32_t u32v; int32_t i32v;
  uint64_t u64v; int64_t i64v; float f32v; double f64v;
  switch (ty) {
    case 0: if (!r.get(&u8v)) return false; v.kind = Value::Int; v.i = u8v; return true;
    case 1: if (!r.get(&i8v)) return false; v.kind = Value::Int; v.i = i8v; return true;
    case 2: if (!r.get(&u16v)) return false; v.kind = Value::Int; v.i = u16v; return true;
    case 3: if (!r.get(&i16v)) return false; v.kind = Value::Int; v.i = i16v; return true;
    case 4: if (!r.get(&u32v)) return false; v.kind = Value::Int; v.i = u32v; return true;
    case 5: if (!r.get(&i32v)) return false; v.kind = Value::Int; v.i = i32v; return true;
    case 6: if (!r.get(&f32v)) return false; v.kind = Value::Float; v.f = f32v; return true;
    case 7: if (!r.get(&u8v)) return false; v.kind = Value::Bool; v.i = u8v != 0; return true;
    case 8: {
      const uint8_t *p;
      if (!r.bytes(&p, &v.len)) return false;
      v.kind = Value::Str;
      v.s = reinterpret_cast<const char *>(p);
      return true;
    }
    case 9:
      if (!r.get(&v.item) || !r.get(&v.len)) return false;
      v.kind = Value::Array;
      return true;
    case 10: if (!r.get(&u64v)) return false; v.kind = Value::Int; v.i = int64_t(u64v); return true;
    case 11: if (!r.get(&i64v)) return false; v.kind = Value::Int; v.i = i64v; return true;
    case 12: if (!r.get(&f64v)) return false; v.kind = Value::Float; v.f = f64v; return true;
    default: return false;
  }
}

// Strict UTF-8 (the reference's `std::str::from_utf8`: a string value that is not UTF-8 reads as
// no string).
bool utf8(const char *s, uint64_t n) {
  const unsigned char *p = reinterpret_cast<const unsigned char *>(s);
  for (uint64_t i = 0; i < n;) {
    const unsigned c = p[i];
    int extra = c < 0x80 ? 0 : (c >> 5) == 6 ? 1 : (c >> 4) == 14 ? 2 : (c >> 3) == 30 ? 3 : -1;
    if (extra < 0 || (extra > 0 && i + extra >= n)) return false;
    if (extra == 1 && c < 0xC2) return false;
    uint32_t cp = c & (0x7F >> extra);
    for (int k = 1; k <= extra; ++k) {
      if ((p[i + k] >> 6) != 2) return false;
      cp = (cp << 6) | (p[i + k] & 0x3F);
    }
    if ((extra == 2 && (cp < 0x800 || (cp >= 0xD800 && cp <= 0xDFFF))) ||
        (extra == 3 && (cp < 0x10000 || cp > 0x10FFFF)))
      return false;
    i += extra + 1;
  }
  return true;
}

uint64_t type_bytes(int ty, uint64_t n) {
  return ty == 0 ? n * 4 : ty == 1 ? n * 2 : n / 32 * 34;
}

// Parses the header in g->head (src/gguf.rs:130-188 `parse`). Returns 0, 1 if the header is cut
// off (read more of the file and try again), or 2 with the message in `err` on a bad file.
int parse(wavo_gguf *g, std::string &err) {
  Reader r{g->head.data(), g->head.size(), 0};
  const uint8_t *magic;
  if (!r.take(4, &magic)) return 1;
  if (std::memcmp(magic, "GGUF", 4) != 0) {
    err = "not a GGUF file";
    return 2;
  }
  uint32_t version;
  uint64_t n_tensors, n_meta;
  if (!r.get(&version)) return 1;
  if (version != 3) {
    err = "unsupported GGUF version " + std::to_string(version);
    return 2;
  }
  if (!r.get(&n_tensors) || !r.get(&n_meta)) return 1;
  g->meta.clear();
  g->tensors.clear();
  g->names.clear();
  for (uint64_t m = 0; m < n_meta; ++m) {
    const uint8_t *kp;
    uint64_t kl;
    uint32_t ty;
    if (!r.bytes(&kp, &kl) || !r.get(&ty)) return 1;
    std::string key(reinterpret_cast<const char *>(kp), size_t(kl));
    g->meta[key] = {ty, r.pos};
    const size_t before = r.pos;
    if (!r.skip(ty)) {
      if (ty > 12) {
        err = "unknown GGUF value type " + std::to_string(ty);
        return 2;
      }
      r.pos = before;
      return 1;
    }
  }
  for (uint64_t t = 0; t < n_tensors; ++t) {
    const uint8_t *np;
    uint64_t nl;
    uint32_t n_dims, id;
    if (!r.bytes(&np, &nl) || !r.get(&n_dims)) return 1;
    std::string name(reinterpret_cast<const char *>(np), size_t(nl));
    if (n_dims > 8) {
      err = "tensor " + name + ": " + std::to_string(n_dims) + " dimensions";
      return 2;
    }
    wavo_gguf::Info info;
    uint64_t count = 1;
    for (uint32_t d = 0; d < n_dims; ++d) {
      uint64_t dim;
      if (!r.get(&dim)) return 1;
      info.dims.push_back(dim);
      count *= dim;
    }
    if (!r.get(&id)) return 1;
    if (id != 0 && id != 1 && id != 8) {
      err = "tensor " + name + ": unsupported ggml type " + std::to_string(id);
      return 2;
    }
    if (!r.get(&info.offset)) return 1;
    info.ty = int(id);
    info.bytes = type_bytes(info.ty, count);
    if (!g->tensors.count(name)) g->names.push_back(name);
    g->tensors[name] = info;
  }
  uint64_t align = 32;
  auto it = g->meta.find("general.alignment");
  if (it != g->meta.end()) {
    Reader v{g->head.data(), g->head.size(), it->second.second};
    Value val;
    if (read_value(v, it->second.first, val) && val.kind == Value::Int && val.i > 0)
      align = uint64_t(val.i);
  }
  g->data = (uint64_t(r.pos) + align - 1) / align * align;
  for (auto &kv : g->tensors) {
    if (g->data + kv.second.offset + kv.second.bytes > g->file_len) {
      err = "tensor " + kv.first + " is out of file bounds";
      return 2;
    }
  }
  return 0;
}

bool lookup(const wavo_gguf *g, const char *key, Value &v, Reader *rest = nullptr) {
  if (!g || !key) return false;
  auto it = g->meta.find(key);
  if (it == g->meta.end()) {
    wv::fail_free(WAVO_EINVAL, "missing metadata %s", key);
    return false;
  }
  Reader r{g->head.data(), g->head.size(), it->second.second};
  if (!read_value(r, it->second.first, v)) {
    wv::fail_free(WAVO_EINVAL, "metadata %s: unreadable", key);
    return false;
  }
  if (rest) *rest = r;
  return true;
}

}  // namespace

namespace wv {

namespace {

bool pread_all(int fd, uint8_t *p, uint64_t bytes, uint64_t off) {
  while (bytes) {
    const ssize_t got = pread(fd, p, bytes > (1u << 30) ? (1u << 30) : size_t(bytes), off_t(off));
    if (got <= 0) return false;
    p += got;
    off += uint64_t(got);
    bytes -= uint64_t(got);
  }
  return true;
}

// A few reader threads shared by every load of the process: a large piece of a file is read as
// several ranges at once (one thread copies from the page cache at a fraction of what the host's
// memory and the PCIe link take).
class ReadPool {
 public:
  static constexpr int kHelpers = 3;
  // Never destroyed: its detached threads wait on its members until the process ends.
  static ReadPool &get() {
    static ReadPool *pool = new ReadPool();
    return *pool;
  }
  // Runs fn(0..parts-1), part 0 on the calling thread; true if every part returned true.
  bool run(int parts, const std::function<bool(int)> &fn) {
    std::unique_lock<std::mutex> lk(run_mu_);  // one multi-part read at a time
    int left = parts - 1;
    bool ok = true;
    std::mutex m;
    std::condition_variable cv;
    {
      std::lock_guard<std::mutex> q(mu_);
      for (int i = 1; i < parts; ++i)
        tasks_.push_back([&, i] {
          const bool r = fn(i);
          std::lock_guard<std::mutex> g(m);
          ok = ok && r;
          if (--left == 0) cv.notify_one();
        });
    }
    cv_.notify_all();
    const bool r0 = fn(0);
    std::unique_lock<std::mutex> g(m);
    cv.wait(g, [&] { return left == 0; });
    return ok && r0;
  }

 private:
  ReadPool() {
    for (int i = 0; i < kHelpers; ++i) std::thread([this] { loop(); }).detach();
  }
  void loop() {
    while (true) {
      std::function<void()> t;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [this] { return !tasks_.empty(); });
        t = std::move(tasks_.front());
        tasks_.pop_front();
      }
      t();
    }
  }
  std::mutex mu_, run_mu_;
  std::condition_variable cv_;
  std::deque<std::function<void()>> tasks_;
};

}  // namespace

bool gguf_pread(const wavo_gguf *g, void *dst, uint64_t bytes, uint64_t off) {
  uint8_t *p = static_cast<uint8_t *>(dst);
  const uint64_t min_part = 1u << 20;
  const int parts = int(std::min<uint64_t>(ReadPool::kHelpers + 1, (bytes + min_part - 1) / min_part));
  if (parts <= 1) return pread_all(g->fd, p, bytes, off);
  const uint64_t per = (bytes + parts - 1) / parts;
  return ReadPool::get().run(parts, [&](int i) {
    const uint64_t a = uint64_t(i) * per, n = std::min(per, bytes - std::min(bytes, a));
    return n == 0 || pread_all(g->fd, p + a, n, off + a);
  });
}

}  // namespace wv

// ---- C ABI: the file and its metadata (src/gguf.rs:100-240) -----------------------------------

extern "C" {

wavo_status wavo_gguf_open(const char *path, wavo_gguf **out) {
  if (!out || !path) return wavo_status(wv::fail_free(WAVO_EINVAL, "gguf: NULL argument"));
  *out = nullptr;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return wavo_status(wv::fail_free(WAVO_EINVAL, "gguf: cannot open %s", path));
  struct stat st;
  if (fstat(fd, &st) != 0) {
    close(fd);
    return wavo_status(wv::fail_free(WAVO_EINVAL, "gguf: cannot stat %s", path));
  }
  wavo_gguf *g = new (std::nothrow) wavo_gguf();
  if (!g) {
    close(fd);
    return wavo_status(wv::fail_free(WAVO_ENOMEM, "gguf: out of memory"));
  }
  g->path = path;
  g->fd = fd;
  g->file_len = uint64_t(st.st_size);
  // The header is usually far below 1 MiB; read more of the file while it does not fit.
  uint64_t n = g->file_len < (1u << 20) ? g->file_len : (1u << 20);
  std::string err;
  while (true) {
    g->head.resize(size_t(n));
    if (n && !wv::gguf_pread(g, g->head.data(), n, 0)) {
      err = "read failed";
      break;
    }
    const int r = parse(g, err);
    if (r == 0) {
      *out = g;
      return WAVO_OK;
    }
    if (r == 2) break;
    if (n >= g->file_len) {
      err = "truncated GGUF header";
      break;
    }
    n = n * 4 < g->file_len ? n * 4 : g->file_len;
  }
  close(fd);
  delete g;
  return wavo_status(wv::fail_free(WAVO_EINVAL, "gguf %s: %s", path, err.c_str()));
}

void wavo_gguf_close(wavo_gguf *g) {
  if (!g) return;
  if (g->fd >= 0) close(g->fd);
  delete g;
}

uint32_t wavo_gguf_tensor_count(const wavo_gguf *g) { return g ? uint32_t(g->names.size()) : 0; }

const char *wavo_gguf_tensor_name(const wavo_gguf *g, uint32_t i) {
  return g && i < g->names.size() ? g->names[i].c_str() : nullptr;
}

wavo_status wavo_gguf_tensor(const wavo_gguf *g, const char *name, const uint64_t *dims,
                             uint32_t n_dims, int *type, uint64_t *bytes) {
  if (!g || !name) return wavo_status(wv::fail_free(WAVO_EINVAL, "gguf: NULL argument"));
  auto it = g->tensors.find(name);
  if (it == g->tensors.end()) return wavo_status(wv::fail_free(WAVO_EINVAL, "missing tensor %s", name));
  const wavo_gguf::Info &t = it->second;
  if (dims && (n_dims != t.dims.size() || std::memcmp(dims, t.dims.data(), n_dims * 8) != 0)) {
    std::string got;
    for (uint64_t d : t.dims) got += (got.empty() ? "" : ", ") + std::to_string(d);
    return wavo_status(wv::fail_free(WAVO_EINVAL, "tensor %s: shape [%s] is not the expected one",
                                     name, got.c_str()));
  }
  if (type) *type = t.ty;
  if (bytes) *bytes = t.bytes;
  return WAVO_OK;
}

uint32_t wavo_gguf_tensor_dims(const wavo_gguf *g, const char *name, uint64_t *dims, uint32_t cap) {
  if (!g || !name) return 0;
  auto it = g->tensors.find(name);
  if (it == g->tensors.end()) return 0;
  const auto &d = it->second.dims;
  for (uint32_t i = 0; i < d.size() && i < cap; ++i) dims[i] = d[i];
  return uint32_t(d.size());
}

wavo_status wavo_gguf_read(const wavo_gguf *g, const char *name, uint64_t offset, void *dst,
                           uint64_t bytes) {
  if (!g || !name || (!dst && bytes))
    return wavo_status(wv::fail_free(WAVO_EINVAL, "gguf: NULL argument"));
  auto it = g->tensors.find(name);
  if (it == g->tensors.end()) return wavo_status(wv::fail_free(WAVO_EINVAL, "missing tensor %s", name));
  const wavo_gguf::Info &t = it->second;
  if (offset > t.bytes || bytes > t.bytes - offset)
    return wavo_status(wv::fail_free(WAVO_EINVAL, "tensor %s: read past its %llu bytes", name,
                                     (unsigned long long)t.bytes));
  const uint64_t at = g->data + t.offset + offset;
  // Tensors inside the header bytes already read come from memory (as the reference's `head`).
  if (at + bytes <= g->head.size()) {
    std::memcpy(dst, g->head.data() + at, size_t(bytes));
    return WAVO_OK;
  }
  if (!wv::gguf_pread(g, dst, bytes, at))
    return wavo_status(wv::fail_free(WAVO_EINVAL, "tensor %s: read failed", name));
  return WAVO_OK;
}

int wavo_gguf_has(const wavo_gguf *g, const char *key) {
  return g && key && g->meta.count(key) ? 1 : 0;
}

wavo_status wavo_gguf_get_int(const wavo_gguf *g, const char *key, int64_t *v) {
  Value x;
  if (!v || !lookup(g, key, x)) return WAVO_EINVAL;
  if (x.kind != Value::Int)
    return wavo_status(wv::fail_free(WAVO_EINVAL, "metadata %s: not an integer", key));
  *v = x.i;
  return WAVO_OK;
}

wavo_status wavo_gguf_get_float(const wavo_gguf *g, const char *key, double *v) {
  Value x;
  if (!v || !lookup(g, key, x)) return WAVO_EINVAL;
  if (x.kind != Value::Float)
    return wavo_status(wv::fail_free(WAVO_EINVAL, "metadata %s: not a float", key));
  *v = x.f;
  return WAVO_OK;
}

wavo_status wavo_gguf_get_bool(const wavo_gguf *g, const char *key, int *v) {
  Value x;
  if (!v || !lookup(g, key, x)) return WAVO_EINVAL;
  if (x.kind != Value::Bool)
    return wavo_status(wv::fail_free(WAVO_EINVAL, "metadata %s: not a bool", key));
  *v = int(x.i);
  return WAVO_OK;
}

wavo_status wavo_gguf_get_str(const wavo_gguf *g, const char *key, const char **s, uint64_t *len) {
  Value x;
  if (!s || !len || !lookup(g, key, x)) return WAVO_EINVAL;
  if (x.kind != Value::Str || !utf8(x.s, x.len))
    return wavo_status(wv::fail_free(WAVO_EINVAL, "metadata %s: not a UTF-8 string", key));
  *s = x.s;
  *len = x.len;
  return WAVO_OK;
}

wavo_status wavo_gguf_array(const wavo_gguf *g, const char *key, uint32_t *item, uint64_t *len) {
  Value x;
  if (!item || !len || !lookup(g, key, x)) return WAVO_EINVAL;
  if (x.kind != Value::Array)
    return wavo_status(wv::fail_free(WAVO_EINVAL, "metadata %s: not an array", key));
  *item = x.item;
  *len = x.len;
  return WAVO_OK;
}

// Every item of the array `key`: integers into ints, floats into floats, strings as pointers into
// the header with their lengths; a NULL output skips that kind. Fails if an item is not of a kind
// with an output, or a string item is not UTF-8 (src/gguf.rs:214-225 `array`).
wavo_status wavo_gguf_array_items(const wavo_gguf *g, const char *key, int64_t *ints,
                                  double *floats, const char **strs, uint64_t *lens,
                                  uint64_t cap) {
  Value x;
  Reader r{};
  if (!lookup(g, key, x, &r)) return WAVO_EINVAL;
  if (x.kind != Value::Array)
    return wavo_status(wv::fail_free(WAVO_EINVAL, "metadata %s: not an array", key));
  if (x.len > cap)
    return wavo_status(wv::fail_free(WAVO_EINVAL, "metadata %s: %llu items, room for %llu", key,
                                     (unsigned long long)x.len, (unsigned long long)cap));
  for (uint64_t i = 0; i < x.len; ++i) {
    Value v;
    if (!read_value(r, x.item, v))
      return wavo_status(wv::fail_free(WAVO_EINVAL, "metadata %s: unreadable item %llu", key,
                                       (unsigned long long)i));
    if (v.kind == Value::Int && ints) {
      ints[i] = v.i;
    } else if (v.kind == Value::Float && floats) {
      floats[i] = v.f;
    } else if (v.kind == Value::Str && strs && lens && utf8(v.s, v.len)) {
      strs[i] = v.s;
      lens[i] = v.len;
    } else {
      return wavo_status(wv::fail_free(WAVO_EINVAL, "metadata %s: item %llu is not of the asked kind",
                                       key, (unsigned long long)i));
    }
  }
  return WAVO_OK;
}

}  // extern "C"

// ---- device side of a load: the raw bytes into the kernels' forms, pre-tiled for TMA ------------

namespace wv {
namespace {

// One thread a Q8_0 block (src/gguf.rs:14-38: an f16 scale d, then 32 × i8; the weight is q·d):
// the int8 values into q8 [n][k] and q·d rounded to f16 into w16 [n][k] (the 2D row-major layouts
// the TMA maps tile), d into d8 [n][k/32] (the gemv) and the scale's f16 bits into s16t [k/32][n]
// (transposed: a K-step's scales for 128 rows are one contiguous box for the prologue GEMM). The
// block's bytes are read as 17 aligned 16-bit words (blocks start at even offsets).
__global__ void build_q8_kernel(const uint8_t *__restrict__ raw, long long blocks, int kq, int n,
                                int8_t *__restrict__ q8, float *__restrict__ d8,
                                __half *__restrict__ s16t, __half *__restrict__ w16) {
  const long long blk = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (blk >= blocks) return;
  const uint16_t *p = reinterpret_cast<const uint16_t *>(raw + blk * 34);
  uint16_t w[17];
#pragma unroll
  for (int i = 0; i < 17; ++i) w[i] = p[i];
  const __half hs = __ushort_as_half(w[0]);
  const float d = __half2float(hs);
  uint32_t words[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) words[m] = uint32_t(w[1 + 2 * m]) | (uint32_t(w[2 + 2 * m]) << 16);
  uint4 *q = reinterpret_cast<uint4 *>(q8 + blk * 32);
  q[0] = make_uint4(words[0], words[1], words[2], words[3]);
  q[1] = make_uint4(words[4], words[5], words[6], words[7]);
  uint32_t h[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int8_t a = int8_t((words[j >> 1] >> (16 * (j & 1))) & 0xFF);
    const int8_t b = int8_t((words[j >> 1] >> (16 * (j & 1) + 8)) & 0xFF);
    const __half ha = __float2half_rn(float(a) * d), hb = __float2half_rn(float(b) * d);
    h[j] = uint32_t(__half_as_ushort(ha)) | (uint32_t(__half_as_ushort(hb)) << 16);
  }
  uint4 *o = reinterpret_cast<uint4 *>(w16 + blk * 32);
#pragma unroll
  for (int v = 0; v < 4; ++v) o[v] = make_uint4(h[4 * v], h[4 * v + 1], h[4 * v + 2], h[4 * v + 3]);
  d8[blk] = d;
  const long long r = blk / kq, b = blk - r * kq;
  s16t[b * n + r] = hs;
}

// F32 weights: the GEMM's copy rounded to f16 (round to nearest even).
__global__ void build_f16_kernel(const float4 *__restrict__ w32, long long quads,
                                 uint2 *__restrict__ w16) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= quads) return;
  const float4 v = w32[i];
  const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
  w16[i] = make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
}

}  // namespace

cudaError_t launch_build_q8(const uint8_t *raw, int rows, int k, int n, int8_t *q8, float *d8,
                            __half *s16t, __half *w16, cudaStream_t s) {
  const long long blocks = (long long)rows * (k / 32);
  if (blocks <= 0) return cudaSuccess;
  build_q8_kernel<<<unsigned((blocks + 255) / 256), 256, 0, s>>>(raw, blocks, k / 32, n, q8, d8,
                                                                  s16t, w16);
  return cudaGetLastError();
}

cudaError_t launch_build_f16(const float *w32, long long count, __half *w16, cudaStream_t s) {
  const long long quads = count / 4;  // count is rows · k, k a multiple of 32
  if (quads <= 0) return cudaSuccess;
  build_f16_kernel<<<unsigned((quads + 255) / 256), 256, 0, s>>>(
      reinterpret_cast<const float4 *>(w32), quads, reinterpret_cast<uint2 *>(w16));
  return cudaGetLastError();
}

}  // namespace wv
