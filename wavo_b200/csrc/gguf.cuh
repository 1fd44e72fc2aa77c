// Internal: the parsed GGUF file shared by gguf.cu (reader, C ABI accessors) and wavo_cuda.cu
// (wavo_linear_from_gguf, which streams tensor data from it to the device).
#pragma once

#include <stdint.h>

#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

struct wavo_gguf {
  struct Info {
    std::vector<uint64_t> dims;  // ggml order: dims[0] contiguous
    int ty = 0;                  // 0 F32, 1 F16, 8 Q8_0
    uint64_t offset = 0;         // from the data section's start
    uint64_t bytes = 0;
  };
  std::string path;
  int fd = -1;
  uint64_t file_len = 0;
  std::vector<uint8_t> head;  // the start of the file, at least the header
  // Per key the value's GGUF type and its offset in `head`: values are decoded when read.
  std::unordered_map<std::string, std::pair<uint32_t, size_t>> meta;
  std::unordered_map<std::string, Info> tensors;
  std::vector<std::string> names;  // in file order
  uint64_t data = 0;               // the data section's offset in the file
};

namespace wv {
// Errors of the calls without a context go to the calling thread's last error (wavo_cuda.cu).
int fail_free(int status, const char *fmt, ...);
// Reads `bytes` at file offset `off` into `dst` (host); false on a short read.
bool gguf_pread(const wavo_gguf *g, void *dst, uint64_t bytes, uint64_t off);
}  // namespace wv
