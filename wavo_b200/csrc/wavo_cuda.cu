// C ABI of the wavo-b200 attention path (include/wavo_cuda.h): contexts, buffers, linear layers,
// argument checks, tensor maps and kernel dispatch. Each entry point cites the reference method it
// replaces in the header.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "../../include/wavo_cuda.h"
#include "gguf.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

struct wavo_ctx {
  int device = 0;
  int sms = 0;
  cudaStream_t own = nullptr;
  cudaStream_t stream = nullptr;
  int *dev_err = nullptr;    // the kernels' error word
  void *ws = nullptr;        // scratch for casts and repacks
  size_t ws_bytes = 0;
  bool capturing = false;
  int q8_mode = WAVO_Q8_AUTO;  // wavo_set_q8_gemm
  // wavo_linear_from_gguf: two pinned pieces of the file in flight to the device.
  void *stage[2] = {nullptr, nullptr};
  cudaEvent_t stage_ev[2] = {nullptr, nullptr};
  // The log-mel frontend's tables (made by the first frontend call).
  void *fe_dev = nullptr;
  wv::FrontendTables fe_tab{};
  std::mutex mu;
  std::string err;
};

struct wavo_linear {
  int device = 0;
  int ty = 0;
  uint32_t rows = 0, n = 0, cols = 0, k = 0, dual = 0;
  __half *w16 = nullptr;     // [n][k] f16, the GEMM's operand (W rounded to f16)
  float *w32 = nullptr;      // [n][k] f32 (F32 weights), the gemv operand
  int8_t *q8 = nullptr;      // [n][k] int8 (Q8_0 weights), the gemv operand
  float *d8 = nullptr;       // [n][k/32] scales (Q8_0)
  __half *s16t = nullptr;    // the same scales as f16, transposed: [k/32][n] (the prologue GEMM)
  float *bias = nullptr;     // max(n, cols + dual) floats
  CUtensorMap map_w128, map_w160, map_w256;  // W tiles of 128, 160 and 256 rows
  // The pair GEMM's half tiles (64, 80, 96 rows; 128 is map_w128), 2D and, when k is a multiple
  // of 64, 3D boxes of two 64-column chunks.
  CUtensorMap map_h64, map_h80, map_h96;
  CUtensorMap map3_h64, map3_h80, map3_h96;
  bool has3 = false;
  // Q8_0: int8 block values [n][k] as TMA boxes of {64, 128 / 160 / 256 rows}, and the transposed
  // scales as boxes of {128 / 160 / 256, 2} (the prologue GEMM).
  CUtensorMap map_q128, map_q160, map_q256;
  CUtensorMap map_s128, map_s160, map_s256;
  bool has_q8map = false;
  void *block = nullptr;     // wavo_linear_from_gguf: every buffer above in one allocation
};

struct wavo_graph {
  cudaGraphExec_t exec = nullptr;
  cudaGraph_t graph = nullptr;
};

namespace {

// The last error of the calls that have no context (a failed wavo_create, the context-free
// wavo_attend_batch_noalloc), one per thread: a failing call on one thread never replaces the
// message another thread is reading.
thread_local std::string t_last_err;

wavo_status fail(wavo_ctx *c, wavo_status s, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (c)
    c->err = buf;
  else
    t_last_err = buf;
  return s;
}

}  // namespace

namespace wv {
int fail_free(int status, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_last_err = buf;
  return status;
}
}  // namespace wv

namespace {

wavo_status cuda_fail(wavo_ctx *c, cudaError_t e, const char *what) {
  return fail(c, e == cudaErrorMemoryAllocation ? WAVO_ENOMEM : WAVO_ECUDA, "%s: %s", what,
              cudaGetErrorString(e));
}

#define CK(call, what)                                  \
  do {                                                  \
    cudaError_t e_ = (call);                            \
    if (e_ != cudaSuccess) return cuda_fail(ctx, e_, what); \
  } while (0)

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
typedef CUresult (*EncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

// A 3D f16 view {64, rows, cols / 64} of rows x cols (row stride ld elements; cols a multiple of
// 64; chunk c = columns 64c..): boxes {64, box_rows, 2}, two 64-column chunks per TMA load.
// f32 rows x cols (row stride ld elements) in boxes of 64 columns x 32 rows, no swizzle, zero fill
// outside: the gemv's rows of a, one box per 64-column chunk.
bool make_map_rows32(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows, uint64_t ld) {
  EncodeTiled enc = encoder();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15u) || ((ld * 4) & 15u) || cols == 0 ||
      rows == 0)
    return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 4};
  cuuint32_t box[2] = {64, 32};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map3(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows, uint64_t ld,
               uint32_t box_rows);

// An int8 tensor map over rows x cols bytes (row stride ld bytes), boxes of 64 x box_rows, no
// swizzle, zero fill outside: the Q8_0 GEMM's raw block values.
bool make_map_i8(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows, uint64_t ld,
                 uint32_t box_rows) {
  EncodeTiled enc = encoder();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15u) || (ld & 15u) || cols == 0 || rows == 0)
    return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The Q8_0 scales transposed, [rows][cols] f16 (cols = the layer's padded rows n, rows = k / 32),
// boxes of box_cols x 2: one K-step's two scale rows of a W tile.
bool make_map_s16(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows,
                  uint32_t box_cols) {
  EncodeTiled enc = encoder();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15u) || ((cols * 2) & 15u) || rows == 0)
    return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {box_cols, 2};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The pair GEMM's output map: rows x cols of f16 or f32 (row stride ld elements), boxes of 32 x 32,
// swizzle matching the epilogue's staging (64-byte rows for f16, 128-byte rows for f32).
bool make_map_c(CUtensorMap *m, void *base, bool f16, uint64_t cols, uint64_t rows, uint64_t ld);

// A 2D f16 tensor map over rows x cols (row stride ld elements), 64-column x box_rows boxes,
// 128-byte swizzle, zero fill outside.
bool make_map(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows, uint64_t ld,
              uint32_t box_rows) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || ((ld * 2) & 15u) || cols == 0 || rows == 0)
    return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map3(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows, uint64_t ld,
               uint32_t box_rows) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || ((ld * 2) & 15u) || cols % 64 || rows == 0)
    return false;
  cuuint64_t dims[3] = {64, rows, cols / 64};
  cuuint64_t strides[2] = {ld * 2, 128};
  cuuint32_t box[3] = {64, box_rows, 2};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The attention output as a TMA store target: f16 rows x cols (row stride ld elements), boxes of
// {box_cols, 16} rows, no swizzle (box_cols x 2 bytes a multiple of 16).
bool make_map_o(CUtensorMap *m, void *base, uint64_t cols, uint64_t rows, uint64_t ld,
                uint32_t box_cols) {
  EncodeTiled enc = encoder();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15u) || ((ld * 2) & 15u) ||
      ((box_cols * 2) & 15u) || box_cols > 256 || rows == 0)
    return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, 16};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_c(CUtensorMap *m, void *base, bool f16, uint64_t cols, uint64_t rows, uint64_t ld) {
  EncodeTiled enc = encoder();
  const uint64_t es = f16 ? 2 : 4;
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15u) || ((ld * es) & 15u) || rows == 0)
    return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * es};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base,
             dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             f16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Scratch of at least `bytes` (grows outside of a capture only).
wavo_status workspace(wavo_ctx *ctx, size_t bytes, void **out) {
  if (bytes > ctx->ws_bytes) {
    if (ctx->capturing)
      return fail(ctx, WAVO_EINVAL, "scratch of %zu bytes needed during a capture: call "
                  "wavo_reserve first", bytes);
    if (ctx->ws) {
      CK(cudaStreamSynchronize(ctx->stream), "scratch sync");
      CK(cudaFree(ctx->ws), "scratch free");
      ctx->ws = nullptr;
      ctx->ws_bytes = 0;
    }
    size_t sz = std::max(bytes, size_t(1) << 20);
    CK(cudaMalloc(&ctx->ws, sz), "scratch");
    ctx->ws_bytes = sz;
  }
  *out = ctx->ws;
  return WAVO_OK;
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// IEEE binary16 from f32, round to nearest even (the reference GPU GEMM's rounding of W).
uint16_t f16_bits(float x) {
  __half h = __float2half_rn(x);
  uint16_t b;
  std::memcpy(&b, &h, 2);
  return b;
}

float f16_value(uint16_t b) {
  __half h;
  std::memcpy(&h, &b, 2);
  return __half2float(h);
}

}  // namespace

extern "C" {

int wavo_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

const char *wavo_last_error(const wavo_ctx *ctx) {
  if (ctx) return ctx->err.c_str();
  return t_last_err.c_str();
}

wavo_status wavo_create(int device, wavo_ctx **out) {
  if (!out) return fail(nullptr, WAVO_EINVAL, "out is NULL");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0)
    return fail(nullptr, WAVO_EUNSUPPORTED, "no CUDA device: %s", cudaGetErrorString(e));
  if (device < 0 || device >= n)
    return fail(nullptr, WAVO_EINVAL, "device %d of %d", device, n);
  cudaDeviceProp prop;
  if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess)
    return fail(nullptr, WAVO_ECUDA, "device properties: %s", cudaGetErrorString(e));
  if (prop.major != 10 || prop.minor != 0)
    return fail(nullptr, WAVO_EUNSUPPORTED,
                "device %d (%s) is sm_%d%d: this library is built for sm_100a (B200)", device,
                prop.name, prop.major, prop.minor);
  if (!encoder()) return fail(nullptr, WAVO_EUNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  wavo_ctx *ctx = new (std::nothrow) wavo_ctx();
  if (!ctx) return fail(nullptr, WAVO_ENOMEM, "context");
  ctx->device = device;
  ctx->sms = prop.multiProcessorCount;
  if ((e = cudaSetDevice(device)) != cudaSuccess ||
      (e = cudaStreamCreateWithFlags(&ctx->own, cudaStreamNonBlocking)) != cudaSuccess ||
      (e = cudaMalloc(&ctx->dev_err, sizeof(int))) != cudaSuccess ||
      (e = cudaMemset(ctx->dev_err, 0, sizeof(int))) != cudaSuccess) {
    fail(nullptr, WAVO_ECUDA, "context setup: %s", cudaGetErrorString(e));
    if (ctx->own) cudaStreamDestroy(ctx->own);
    if (ctx->dev_err) cudaFree(ctx->dev_err);
    delete ctx;
    return WAVO_ECUDA;
  }
  ctx->stream = ctx->own;
  *out = ctx;
  return WAVO_OK;
}

void wavo_destroy(wavo_ctx *ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->ws) cudaFree(ctx->ws);
  for (int i = 0; i < 2; ++i) {
    if (ctx->stage[i]) cudaFreeHost(ctx->stage[i]);
    if (ctx->stage_ev[i]) cudaEventDestroy(ctx->stage_ev[i]);
  }
  if (ctx->dev_err) cudaFree(ctx->dev_err);
  if (ctx->fe_dev) cudaFree(ctx->fe_dev);
  if (ctx->own) cudaStreamDestroy(ctx->own);
  delete ctx;
}

wavo_status wavo_set_stream(wavo_ctx *ctx, void *stream) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (ctx->capturing) return fail(ctx, WAVO_EINVAL, "set_stream during a capture");
  ctx->stream = static_cast<cudaStream_t>(stream);  // NULL: the CUDA default stream
  return WAVO_OK;
}

void *wavo_get_stream(const wavo_ctx *ctx) { return ctx ? ctx->stream : nullptr; }
void *wavo_own_stream(const wavo_ctx *ctx) { return ctx ? ctx->own : nullptr; }
int wavo_sm_count(const wavo_ctx *ctx) { return ctx ? ctx->sms : 0; }

wavo_status wavo_malloc(wavo_ctx *ctx, size_t bytes, void **out) {
  if (!ctx || !out) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  cudaSetDevice(ctx->device);
  *out = nullptr;
  CK(cudaMalloc(out, bytes ? bytes : 1), "wavo_malloc");
  return WAVO_OK;
}

wavo_status wavo_free(wavo_ctx *ctx, void *p) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  cudaSetDevice(ctx->device);
  if (p) CK(cudaFree(p), "wavo_free");
  return WAVO_OK;
}

wavo_status wavo_upload(wavo_ctx *ctx, void *dst, const void *src, size_t bytes) {
  if (!ctx || (!dst && bytes) || (!src && bytes)) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  cudaSetDevice(ctx->device);
  CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream), "wavo_upload");
  return WAVO_OK;
}

wavo_status wavo_download(wavo_ctx *ctx, void *dst, const void *src, size_t bytes) {
  if (!ctx || (!dst && bytes) || (!src && bytes)) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  cudaSetDevice(ctx->device);
  CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream), "wavo_download");
  return WAVO_OK;
}

wavo_status wavo_memset(wavo_ctx *ctx, void *dst, int value, size_t bytes) {
  if (!ctx || (!dst && bytes)) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  cudaSetDevice(ctx->device);
  CK(cudaMemsetAsync(dst, value, bytes, ctx->stream), "wavo_memset");
  return WAVO_OK;
}

wavo_status wavo_reserve(wavo_ctx *ctx, size_t bytes) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  cudaSetDevice(ctx->device);
  void *p;
  return workspace(ctx, bytes, &p);
}

wavo_status wavo_sync(wavo_ctx *ctx, uint32_t timeout_ms) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  cudaSetDevice(ctx->device);
  auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t e = cudaStreamQuery(ctx->stream);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) return cuda_fail(ctx, e, "device");
    if (timeout_ms) {
      auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                    std::chrono::steady_clock::now() - t0)
                    .count();
      if (ms > timeout_ms)
        return fail(ctx, WAVO_ETIMEDOUT, "the stream did not finish within %u ms", timeout_ms);
    }
    std::this_thread::yield();
  }
  int code = 0;
  CK(cudaMemcpy(&code, ctx->dev_err, sizeof code, cudaMemcpyDeviceToHost), "error word");
  if (code) {
    CK(cudaMemset(ctx->dev_err, 0, sizeof(int)), "error word reset");
    static const char *what[] = {"", "TMA producer", "MMA issuer", "softmax/epilogue", "drain"};
    return fail(ctx, WAVO_EDEVICE, "a kernel's bounded wait gave up (%s, code %d)",
                code > 0 && code < 5 ? what[code] : "?", code);
  }
  return WAVO_OK;
}

// ---- linear layers ---------------------------------------------------------------------

namespace {

// The tensor maps of a linear layer whose device forms are in place (w16; q8 and s16t for Q8_0).
bool linear_maps(wavo_linear *l) {
  const uint32_t n = l->n, k = l->k;
  if (!make_map(&l->map_w128, l->w16, k, n, k, 128) || !make_map(&l->map_w160, l->w16, k, n, k, 160) ||
      !make_map(&l->map_w256, l->w16, k, n, k, 256) || !make_map(&l->map_h64, l->w16, k, n, k, 64) ||
      !make_map(&l->map_h80, l->w16, k, n, k, 80) || !make_map(&l->map_h96, l->w16, k, n, k, 96))
    return false;
  l->has_q8map = l->q8 && make_map_i8(&l->map_q128, l->q8, k, n, k, 128) &&
                 make_map_i8(&l->map_q160, l->q8, k, n, k, 160) &&
                 make_map_i8(&l->map_q256, l->q8, k, n, k, 256) &&
                 make_map_s16(&l->map_s128, l->s16t, n, k / 32, 128) &&
                 make_map_s16(&l->map_s160, l->s16t, n, k / 32, 160) &&
                 make_map_s16(&l->map_s256, l->s16t, n, k / 32, 256);
  l->has3 = k % 64 == 0 && make_map3(&l->map3_h64, l->w16, k, n, k, 64) &&
            make_map3(&l->map3_h80, l->w16, k, n, k, 80) &&
            make_map3(&l->map3_h96, l->w16, k, n, k, 96);
  return true;
}

}  // namespace

wavo_status wavo_linear_create(wavo_ctx *ctx, int ty, uint32_t rows, uint32_t k, const void *data,
                               const float *bias, size_t bias_len, wavo_linear **out) {
  if (!ctx || !out || !data) return WAVO_EINVAL;
  *out = nullptr;
  // Argument checks as Gpu::upload_linear (src/gpu/mod.rs:775-827).
  if (ty != WAVO_GGML_F32 && ty != WAVO_GGML_F16 && ty != WAVO_GGML_Q8_0 && ty != WAVO_GGML_BF16)
    return fail(ctx, WAVO_EINVAL, "linear layer: GGUF type %d is not F32, F16, Q8_0 or BF16", ty);
  if (rows == 0 || k == 0 || k % 32 != 0)
    return fail(ctx, WAVO_EINVAL, "linear layer %u->%u: needs k %% 32 == 0", k, rows);
  const uint32_t dual = bias_len > rows ? uint32_t(bias_len - rows) : 0;
  if ((bias_len != 0 && bias_len < rows) || dual > rows)
    return fail(ctx, WAVO_EINVAL, "linear layer %u->%u: bias has %zu values", k, rows, bias_len);
  const uint32_t n = (rows + 63) / 64 * 64;
  const uint32_t cols = rows % 32 == 0 ? rows : n;
  // W rounded to f16 for the GEMM, zero rows past `rows`.
  std::vector<uint16_t> w16(size_t(n) * k, 0);
  std::vector<float> w32;
  std::vector<int8_t> q8;
  std::vector<float> d8;
  const size_t nk = size_t(rows) * k;
  if (ty == WAVO_GGML_F32) {
    const float *f = static_cast<const float *>(data);
    w32.assign(f, f + nk);
    w32.resize(size_t(n) * k, 0.0f);
    for (size_t i = 0; i < nk; ++i) w16[i] = f16_bits(f[i]);
  } else if (ty == WAVO_GGML_F16) {
    std::memcpy(w16.data(), data, nk * 2);
  } else if (ty == WAVO_GGML_BF16) {
    // bf16 is the high half of an f32: exact in f32 (the gemv operand), rounded to f16 for the
    // GEMM as the reference rounds every W.
    const uint16_t *b = static_cast<const uint16_t *>(data);
    w32.assign(size_t(n) * k, 0.0f);
    for (size_t i = 0; i < nk; ++i) {
      const uint32_t bits = uint32_t(b[i]) << 16;
      std::memcpy(&w32[i], &bits, 4);
      w16[i] = f16_bits(w32[i]);
    }
  } else {
    const uint8_t *b = static_cast<const uint8_t *>(data);
    q8.assign(size_t(n) * k, 0);
    d8.assign(size_t(n) * k / 32, 0.0f);
    for (size_t blk = 0; blk < nk / 32; ++blk) {
      const uint8_t *p = b + 34 * blk;
      const float d = f16_value(uint16_t(p[0] | (p[1] << 8)));
      d8[blk] = d;
      for (int i = 0; i < 32; ++i) {
        const int8_t q = int8_t(p[2 + i]);
        q8[32 * blk + i] = q;
        w16[32 * blk + i] = f16_bits(float(q) * d);  // q·d exact in f32, then to f16
      }
    }
  }
  std::vector<float> bpad(std::max<size_t>(n, size_t(cols) + dual), 0.0f);
  if (bias && bias_len) {
    std::memcpy(bpad.data(), bias, size_t(rows) * 4);
    if (dual) std::memcpy(bpad.data() + cols, bias + rows, size_t(dual) * 4);
  }
  wavo_linear *l = new (std::nothrow) wavo_linear();
  if (!l) return fail(ctx, WAVO_ENOMEM, "linear");
  l->device = ctx->device;
  l->ty = ty;
  l->rows = rows;
  l->n = n;
  l->cols = cols;
  l->k = k;
  l->dual = dual;
  cudaError_t e = cudaSetDevice(ctx->device);
  auto up = [&](void **dst, const void *src, size_t bytes) {
    if (e != cudaSuccess) return;
    if ((e = cudaMalloc(dst, bytes)) != cudaSuccess) return;
    e = cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice);
  };
  up(reinterpret_cast<void **>(&l->w16), w16.data(), w16.size() * 2);
  up(reinterpret_cast<void **>(&l->bias), bpad.data(), bpad.size() * 4);
  if (!w32.empty()) up(reinterpret_cast<void **>(&l->w32), w32.data(), w32.size() * 4);
  if (!q8.empty()) {
    up(reinterpret_cast<void **>(&l->q8), q8.data(), q8.size());
    up(reinterpret_cast<void **>(&l->d8), d8.data(), d8.size() * 4);
    std::vector<uint16_t> s16t(d8.size());
    const size_t kq = k / 32;
    for (size_t r = 0; r < n; ++r)
      for (size_t b = 0; b < kq; ++b) s16t[b * n + r] = f16_bits(d8[r * kq + b]);  // exact
    up(reinterpret_cast<void **>(&l->s16t), s16t.data(), s16t.size() * 2);
  }
  if (e != cudaSuccess) {
    wavo_linear_destroy(l);
    std::lock_guard<std::mutex> g(ctx->mu);
    return cuda_fail(ctx, e, "linear upload");
  }
  if (!linear_maps(l)) {
    wavo_linear_destroy(l);
    return fail(ctx, WAVO_ECUDA, "linear: tensor map");
  }
  *out = l;
  return WAVO_OK;
}

// Gpu::linear over GGUF tensors (src/gpu/mod.rs:758-827 `upload_linear`): the named tensors,
// stacked by rows, streamed from the file in pieces through two pinned buffers (the read of one
// piece overlaps the copy of the other), raw as the file holds them; then one kernel turns them
// into every device form the kernels read (w16; w32 for F32; q8, d8 and the transposed f16 scales
// for Q8_0), and the tensor maps are made. F16 bytes land in w16 as they are, F32 in w32. The
// weights never pass through host code element by element.
wavo_status wavo_linear_from_gguf(wavo_ctx *ctx, const wavo_gguf *g, const char *const *names,
                                  uint32_t count, const float *bias, size_t bias_len,
                                  wavo_linear **out) {
  if (!ctx || !out) return WAVO_EINVAL;
  *out = nullptr;
  if (!g || !names || count == 0) return fail(ctx, WAVO_EINVAL, "linear from GGUF: no tensors");
  std::vector<const wavo_gguf::Info *> ts;
  uint64_t rows64 = 0, k = 0;
  int ty = -1;
  for (uint32_t i = 0; i < count; ++i) {
    auto it = names[i] ? g->tensors.find(names[i]) : g->tensors.end();
    if (it == g->tensors.end())
      return fail(ctx, WAVO_EINVAL, "missing tensor %s", names[i] ? names[i] : "(null)");
    const wavo_gguf::Info &t = it->second;
    uint64_t len = 1;
    for (uint64_t d : t.dims) len *= d;
    const uint64_t r = t.dims.empty() ? 1 : t.dims.back();
    if (r == 0) return fail(ctx, WAVO_EINVAL, "tensor %s is empty", names[i]);
    if (i == 0) {
      ty = t.ty;
      k = len / r;
    } else if (t.ty != ty || len / r != k) {
      return fail(ctx, WAVO_EINVAL, "stacked weights differ in type or shape");
    }
    rows64 += r;
    ts.push_back(&t);
  }
  if (k == 0 || k % 32 != 0 || rows64 > 0x7fffffffu || k > 0x7fffffffu)
    return fail(ctx, WAVO_EINVAL, "linear layer %llu->%llu: needs k %% 32 == 0",
                (unsigned long long)k, (unsigned long long)rows64);
  const uint32_t rows = uint32_t(rows64);
  const uint32_t dual = bias_len > rows ? uint32_t(bias_len - rows) : 0;
  if ((bias_len != 0 && bias_len < rows) || dual > rows)
    return fail(ctx, WAVO_EINVAL, "linear layer %llu->%u: bias has %zu values",
                (unsigned long long)k, rows, bias_len);
  std::lock_guard<std::mutex> lk(ctx->mu);
  cudaSetDevice(ctx->device);
  const uint32_t n = (rows + 63) / 64 * 64;
  const uint32_t cols = rows % 32 == 0 ? rows : n;
  wavo_linear *l = new (std::nothrow) wavo_linear();
  if (!l) return fail(ctx, WAVO_ENOMEM, "linear");
  l->device = ctx->device;
  l->ty = ty;
  l->rows = rows;
  l->n = n;
  l->cols = cols;
  l->k = uint32_t(k);
  l->dual = dual;
  const size_t nk = size_t(n) * k;
  const size_t nbias = std::max<size_t>(n, size_t(cols) + dual);
  // Every device form in one allocation (one cudaMalloc and one cudaFree a layer), zeroed so that
  // the rows past `rows` are zero; Q8_0's raw blocks land in the context's scratch.
  size_t sz[6] = {nk * 2, ty == WAVO_GGML_F32 ? nk * 4 : 0, ty == WAVO_GGML_Q8_0 ? nk : 0,
                  ty == WAVO_GGML_Q8_0 ? nk / 32 * 4 : 0, ty == WAVO_GGML_Q8_0 ? nk / 32 * 2 : 0,
                  nbias * 4};
  size_t offs[6], total = 0;
  for (int i = 0; i < 6; ++i) {
    offs[i] = total;
    total += align_up(sz[i], 256);
  }
  uint8_t *raw = nullptr;  // where the file's bytes land
  cudaError_t e = cudaMalloc(&l->block, total);
  if (e == cudaSuccess) e = cudaMemsetAsync(l->block, 0, total, ctx->stream);
  if (e == cudaSuccess) {
    uint8_t *b = static_cast<uint8_t *>(l->block);
    l->w16 = reinterpret_cast<__half *>(b + offs[0]);
    if (sz[1]) l->w32 = reinterpret_cast<float *>(b + offs[1]);
    if (sz[2]) {
      l->q8 = reinterpret_cast<int8_t *>(b + offs[2]);
      l->d8 = reinterpret_cast<float *>(b + offs[3]);
      l->s16t = reinterpret_cast<__half *>(b + offs[4]);
    }
    l->bias = reinterpret_cast<float *>(b + offs[5]);
  }
  if (ty == WAVO_GGML_F16) {
    raw = reinterpret_cast<uint8_t *>(l->w16);
  } else if (ty == WAVO_GGML_F32) {
    raw = reinterpret_cast<uint8_t *>(l->w32);
  } else if (e == cudaSuccess) {
    void *ws = nullptr;
    if (workspace(ctx, size_t(rows) * k / 32 * 34, &ws) != WAVO_OK) {
      wavo_linear_destroy(l);
      return WAVO_ENOMEM;
    }
    raw = static_cast<uint8_t *>(ws);
  }
  // Pinned pieces (allocated once per context); a piece is refilled once its copy has run.
  const size_t piece = size_t(34) << 17;  // 4.25 MB: whole Q8_0 blocks
  for (int i = 0; i < 2 && e == cudaSuccess; ++i) {
    if (!ctx->stage[i]) e = cudaHostAlloc(&ctx->stage[i], piece, cudaHostAllocDefault);
    if (e == cudaSuccess && !ctx->stage_ev[i])
      e = cudaEventCreateWithFlags(&ctx->stage_ev[i], cudaEventDisableTiming);
  }
  bool io_ok = true;
  uint64_t at = 0;
  int which = 0;
  bool used[2] = {false, false};
  for (size_t t = 0; t < ts.size() && e == cudaSuccess && io_ok; ++t) {
    const uint64_t base = g->data + ts[t]->offset, size = ts[t]->bytes;
    for (uint64_t off = 0; off < size && e == cudaSuccess; off += piece) {
      const uint64_t len = std::min<uint64_t>(piece, size - off);
      if (used[which] && (e = cudaEventSynchronize(ctx->stage_ev[which])) != cudaSuccess) break;
      if (base + off + len <= g->head.size()) {
        std::memcpy(ctx->stage[which], g->head.data() + base + off, size_t(len));
      } else if (!wv::gguf_pread(g, ctx->stage[which], len, base + off)) {
        io_ok = false;
        break;
      }
      if ((e = cudaMemcpyAsync(raw + at + off, ctx->stage[which], size_t(len),
                               cudaMemcpyHostToDevice, ctx->stream)) != cudaSuccess ||
          (e = cudaEventRecord(ctx->stage_ev[which], ctx->stream)) != cudaSuccess)
        break;
      used[which] = true;
      which ^= 1;
    }
    at += size;
  }
  if (e == cudaSuccess && io_ok) {
    if (ty == WAVO_GGML_Q8_0)
      e = wv::launch_build_q8(raw, int(rows), int(k), int(n), l->q8, l->d8, l->s16t, l->w16,
                              ctx->stream);
    else if (ty == WAVO_GGML_F32)
      e = wv::launch_build_f16(l->w32, (long long)rows * (long long)k, l->w16, ctx->stream);
  }
  std::vector<float> bpad(nbias, 0.0f);
  if (bias && bias_len) {
    std::memcpy(bpad.data(), bias, size_t(rows) * 4);
    if (dual) std::memcpy(bpad.data() + cols, bias + rows, size_t(dual) * 4);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(l->bias, bpad.data(), bpad.size() * 4, cudaMemcpyHostToDevice,
                          ctx->stream);
  }
  const cudaError_t es = cudaStreamSynchronize(ctx->stream);  // bpad and the pieces are host memory
  if (e == cudaSuccess) e = es;
  if (!io_ok) {
    wavo_linear_destroy(l);
    return fail(ctx, WAVO_EINVAL, "linear from GGUF: reading %s failed", g->path.c_str());
  }
  if (e != cudaSuccess) {
    wavo_linear_destroy(l);
    return cuda_fail(ctx, e, "linear from GGUF");
  }
  if (!linear_maps(l)) {
    wavo_linear_destroy(l);
    return fail(ctx, WAVO_ECUDA, "linear: tensor map");
  }
  *out = l;
  return WAVO_OK;
}

void wavo_linear_destroy(wavo_linear *l) {
  if (!l) return;
  cudaSetDevice(l->device);
  if (l->block) {
    cudaFree(l->block);
  } else {
    cudaFree(l->w16);
    cudaFree(l->w32);
    cudaFree(l->q8);
    cudaFree(l->d8);
    cudaFree(l->s16t);
    cudaFree(l->bias);
  }
  delete l;
}

uint32_t wavo_linear_width(const wavo_linear *l) { return l ? l->cols + l->dual : 0; }
uint32_t wavo_linear_k(const wavo_linear *l) { return l ? l->k : 0; }

// ---- projections -----------------------------------------------------------------------

wavo_status wavo_gemm(wavo_ctx *ctx, const void *a, int a_dtype, uint32_t lda, const wavo_linear *l,
                      void *c, int c_dtype, uint32_t ldc, uint32_t m, int epilogue, float alpha) {
  if (!ctx || !l) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (m == 0) return WAVO_OK;
  if (!a || !c) return fail(ctx, WAVO_EINVAL, "gemm: NULL buffer");
  if (l->device != ctx->device) return fail(ctx, WAVO_EINVAL, "gemm: layer of another device");
  if (epilogue < 0 || epilogue > WAVO_EPI_TANH) return fail(ctx, WAVO_EINVAL, "gemm: epilogue");
  if ((a_dtype != WAVO_F32 && a_dtype != WAVO_F16) || (c_dtype != WAVO_F32 && c_dtype != WAVO_F16))
    return fail(ctx, WAVO_EINVAL, "gemm: dtype");
  if (lda == 0) lda = l->k;
  if (ldc == 0) ldc = l->cols + l->dual;
  if (lda < l->k || ldc < l->cols + l->dual)
    return fail(ctx, WAVO_EINVAL, "gemm: lda %u < k %u or ldc %u < width %u", lda, l->k, ldc,
                l->cols + l->dual);
  cudaSetDevice(ctx->device);
  const __half *a16 = static_cast<const __half *>(a);
  uint32_t lda16 = lda;
  if (a_dtype == WAVO_F32 || (lda % 8) || (reinterpret_cast<uintptr_t>(a) & 15u)) {
    // The reference rounds a to f16 in the GEMM (src/cpu/gemm.rs:163): one cast pass.
    void *ws;
    wavo_status s = workspace(ctx, size_t(m) * l->k * 2, &ws);
    if (s) return s;
    if (a_dtype == WAVO_F32) {
      CK(wv::launch_cast_rows(static_cast<const float *>(a), lda, static_cast<__half *>(ws), l->k,
                              int(m), int(l->k), ctx->stream),
         "gemm cast");
    } else {
      CK(cudaMemcpy2DAsync(ws, size_t(l->k) * 2, a, size_t(lda) * 2, size_t(l->k) * 2, m,
                           cudaMemcpyDeviceToDevice, ctx->stream),
         "gemm repack");
    }
    a16 = static_cast<const __half *>(ws);
    lda16 = l->k;
  }
  wv::GemmArgs ga;
  ga.m = int(m);
  ga.cols = int(l->cols);
  ga.dual = int(l->dual);
  ga.k = int(l->k);
  ga.bias = l->bias;
  ga.c = c;
  ga.ldc = ldc;
  ga.c_f16 = c_dtype == WAVO_F16;
  ga.epilogue = epilogue;
  ga.alpha = alpha;
  ga.err = ctx->dev_err;
  ga.c_tma = 0;
  CUtensorMap map_a;
  const bool q8_prologue =
      l->ty == WAVO_GGML_Q8_0 && l->has_q8map && ctx->q8_mode == WAVO_Q8_PROLOGUE;
  if (q8_prologue) {
    // W dequantised as it is staged: int8 values by TMA, f16 tiles built in shared memory.
    if (!make_map(&map_a, a16, l->k, m, lda16, wv::kGemmBM))
      return fail(ctx, WAVO_ECUDA, "gemm: tensor map of a");
    const int bn = wv::gemm_pick_bn(int(m), int(l->cols), ctx->sms);
    const CUtensorMap &mq = bn == 256 ? l->map_q256 : bn == 160 ? l->map_q160 : l->map_q128;
    const CUtensorMap &ms = bn == 256 ? l->map_s256 : bn == 160 ? l->map_s160 : l->map_s128;
    CK(wv::launch_gemm_q8(map_a, mq, ms, ga, bn, ctx->sms, ctx->stream), "gemm launch");
    return WAVO_OK;
  }
  if (m > uint32_t(wv::kGemmBM)) {
    // Two or more row tiles: the pair GEMM (a CTA pair shares each UMMA of M=256).
    const int bn = wv::gemm2_pick_bn(int(m), int(l->cols), ctx->sms);
    const int kc = (l->has3 && bn <= 192) ? 2 : 1;
    const bool ok_a = kc == 2 ? make_map3(&map_a, a16, l->k, m, lda16, wv::kGemmBM)
                              : make_map(&map_a, a16, l->k, m, lda16, wv::kGemmBM);
    if (!ok_a) return fail(ctx, WAVO_ECUDA, "gemm: tensor map of a");
    const CUtensorMap &mw = kc == 2 ? (bn == 128 ? l->map3_h64 : bn == 160 ? l->map3_h80 : l->map3_h96)
                                    : (bn == 128 ? l->map_h64 : bn == 160 ? l->map_h80
                                       : bn == 192 ? l->map_h96 : l->map_w128);
    // c through TMA stores (reduce-adds for the residual epilogues, which need f32 c), when c is
    // 16-byte aligned and every 32-column box stays inside one output region.
    const bool resid = epilogue == WAVO_EPI_RESIDUAL || epilogue == WAVO_EPI_GELU_RESIDUAL;
    const bool f16 = c_dtype == WAVO_F16;
    CUtensorMap map_c = map_a;
    if ((!resid || !f16) && (!l->dual || (!resid && l->cols % 32 == 0 && l->dual % 32 == 0)) &&
        make_map_c(&map_c, c, f16, l->cols + l->dual, m, ldc))
      ga.c_tma = 1;
    CK(wv::launch_gemm2(map_a, mw, map_c, ga, bn, kc, ctx->sms, ctx->stream), "gemm launch");
    return WAVO_OK;
  }
  if (!make_map(&map_a, a16, l->k, m, lda16, wv::kGemmBM))
    return fail(ctx, WAVO_ECUDA, "gemm: tensor map of a");
  const int bn = wv::gemm_pick_bn(int(m), int(l->cols), ctx->sms);
  const CUtensorMap &mw = bn == 256 ? l->map_w256 : bn == 160 ? l->map_w160 : l->map_w128;
  CK(wv::launch_gemm(map_a, mw, ga, bn, 1, ctx->sms, ctx->stream),
     "gemm launch");
  return WAVO_OK;
}

int wavo_set_q8_gemm(wavo_ctx *ctx, int mode) {
  if (!ctx) return -1;
  std::lock_guard<std::mutex> g(ctx->mu);
  const int old = ctx->q8_mode;
  if (mode == WAVO_Q8_AUTO || mode == WAVO_Q8_DEQUANT || mode == WAVO_Q8_PROLOGUE)
    ctx->q8_mode = mode;
  return old;
}

wavo_status wavo_gemv_rows(wavo_ctx *ctx, const float *a, uint32_t lda, const wavo_linear *l,
                           float *c, uint32_t ldc, uint32_t rows, int epilogue, float alpha) {
  if (!ctx || !l) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (rows == 0) return WAVO_OK;
  if (!a || !c) return fail(ctx, WAVO_EINVAL, "gemv: NULL buffer");
  if (rows > 32) return fail(ctx, WAVO_EINVAL, "gemv: %u rows (at most 32)", rows);
  if (epilogue < 0 || epilogue > WAVO_EPI_TANH) return fail(ctx, WAVO_EINVAL, "gemv: epilogue");
  if (lda == 0) lda = l->k;
  if (ldc == 0) ldc = l->cols;
  if (lda < l->k || (lda % 4) || (reinterpret_cast<uintptr_t>(a) & 15u))
    return fail(ctx, WAVO_EINVAL, "gemv: a rows need k floats, 16-byte aligned");
  if (rows > 1 && ldc < l->cols) return fail(ctx, WAVO_EINVAL, "gemv: ldc");
  cudaSetDevice(ctx->device);
  const bool f32w = l->ty == WAVO_GGML_F32 || l->ty == WAVO_GGML_BF16;
  const void *w = f32w ? static_cast<const void *>(l->w32)
                  : l->ty == WAVO_GGML_Q8_0 ? static_cast<const void *>(l->q8)
                                            : static_cast<const void *>(l->w16);
  const int wt = f32w ? 0 : l->ty == WAVO_GGML_Q8_0 ? 8 : 1;
  // Pass::gemv writes l.cols outputs (src/gpu/mod.rs:1461-1467).
  CUtensorMap map_a;
  if (wt == 1 && make_map_rows32(&map_a, a, l->k, rows, lda)) {
    // F16 weights are exact in f16: the tensor-core form (split f16 rows, f32 accuracy).
    CK(wv::launch_gemv_tc(map_a, l->map_w128, l->bias, c, ldc, int(rows), int(l->cols),
                          int(l->k), epilogue, alpha, ctx->sms, ctx->dev_err, ctx->stream),
       "gemv launch");
    return WAVO_OK;
  }
  CK(wv::launch_gemv(a, lda, wt, w, l->d8, l->bias, c, ldc, int(rows), int(l->cols), int(l->k),
                     epilogue, alpha, ctx->stream),
     "gemv launch");
  return WAVO_OK;
}

wavo_status wavo_gemv(wavo_ctx *ctx, const float *a, const wavo_linear *l, float *c, int epilogue,
                      float alpha, uint32_t offset) {
  if (!c) return WAVO_EINVAL;
  return wavo_gemv_rows(ctx, a, 0, l, c + offset, 0, 1, epilogue, alpha);
}

// ---- encoder attention -------------------------------------------------------------------

uint32_t wavo_pos_rows(uint32_t t) { return 2 * t + 15; }

namespace {

// The layout of one attention call's operands.
struct AttnLayout {
  int sections;          // operand sections in qk: 2 ([q|k]), 3 ([q|k|v]) or 4 ([q+u|k|v|q+v])
  bool sep_v;            // v is its own buffer
  bool rel;
};

// Rotary positions applied inside the plain attention kernel (wavo_attention_rope_varlen).
struct RopeSpec {
  const float *table;
  uint32_t rot, pos;
  int neox;
};

wavo_status attention_impl(wavo_ctx *ctx, const void *qk, const void *v, const void *pos, void *o,
                           const int32_t *seg_start, const int32_t *seg_len, uint32_t nseg,
                           uint32_t max_len, uint32_t pos_t, uint32_t single_t, uint32_t heads,
                           uint32_t hd, int dtype, int o_dtype, const RopeSpec *rope = nullptr) {
  if (!qk || !o) return fail(ctx, WAVO_EINVAL, "attention: NULL buffer");
  if (dtype != WAVO_F32 && dtype != WAVO_F16) return fail(ctx, WAVO_EINVAL, "attention: dtype");
  if (o_dtype != WAVO_F32 && o_dtype != WAVO_F16) return fail(ctx, WAVO_EINVAL, "attention: o dtype");
  if (heads == 0 || hd == 0 || hd > 128 || hd % 2)
    return fail(ctx, WAVO_EINVAL, "attention: heads %u of %u dims (hd even, <= 128)", heads, hd);
  if (max_len == 0 || nseg == 0) return WAVO_OK;
  const bool rel = pos != nullptr;
  if (rel && v) return fail(ctx, WAVO_EINVAL, "attention: relative positions take no separate v");
  if (rel && pos_t < max_len)
    return fail(ctx, WAVO_EINVAL, "attention: position table for t=%u < segment length %u", pos_t,
                max_len);
  const AttnLayout L{rel ? 4 : (v ? 2 : 3), v != nullptr, rel};
  const uint32_t ch = heads * hd;
  const uint32_t ld = L.sections * ch;  // elements per qk row
  // Rows of every operand (the tensor maps' extent): the segment, or the caller's total.
  const uint64_t rows = single_t;
  // f16 operands in the reference layout go to the kernel as they are when every TMA box starts
  // on a 16-byte boundary; anything else is repacked into padded f16 heads first.
  const bool aligned16 = (reinterpret_cast<uintptr_t>(qk) & 15u) == 0 && ld % 8 == 0;
  const bool direct = dtype == WAVO_F16 && !v && aligned16 && hd % 16 == 0 &&
                      (rel ? (hd == 128 && (reinterpret_cast<uintptr_t>(pos) & 15u) == 0)
                           : (hd <= 64 || hd == 128));
  const int hd_pad = rel ? 128 : (hd <= 64 ? 64 : 128);
  cudaSetDevice(ctx->device);

  wv::AttnArgs a{};
  a.seg_start = seg_start;
  a.seg_len = seg_len;
  a.single_t = int(single_t);
  a.heads = int(heads);
  a.hd = int(hd);
  a.pos_t = int(pos_t);
  a.scale_log2 = float(1.4426950408889634 / std::sqrt(double(hd)));
  a.o = o;
  a.ldo = ch;
  a.o_f16 = o_dtype == WAVO_F16;
  a.err = ctx->dev_err;
  if (rope) {
    // The rotation happens on the f16 tiles the kernel stages from the operand rows, so the rows
    // must be the kernel's operands as they are (no repack).
    if (!direct || rel)
      return fail(ctx, WAVO_EUNSUPPORTED,
                  "attention with rotary positions: needs f16 [q | k | v] rows, 16-byte aligned, "
                  "heads of 16, 32, 48, 64 or 128");
    a.rope_table = rope->table;
    a.rope_rot = int(rope->rot);
    a.rope_neox = rope->neox;
    a.rope_pos = int(rope->pos);
  }

  CUtensorMap mq, mkv, mpos, mo;
  // f16 output whose head boxes start on 16-byte boundaries: stored with TMA (16 rows a warp).
  a.o_tma = a.o_f16 && (hd * 2) % 16 == 0 && make_map_o(&mo, o, ch, rows, ch, hd);
  const int bk = wv::attn_block_keys(rel, hd_pad);
  if (direct) {
    a.head_stride = int(hd);
    a.q_off = 0;
    a.k_off = int(ch);
    a.v_off = int(2 * ch);
    a.qv_off = int(3 * ch);
    a.pos_off = 0;
    const bool ok = rel ? make_map3(&mq, qk, ld, rows, ld, wv::kAttnBlockQ) &&
                              make_map3(&mkv, qk, ld, rows, ld, uint32_t(bk))
                        : make_map(&mq, qk, ld, rows, ld, wv::kAttnBlockQ) &&
                              make_map(&mkv, qk, ld, rows, ld, uint32_t(bk));
    if (!ok) return fail(ctx, WAVO_ECUDA, "attention: tensor map");
    mpos = mq;
    if (rel && !make_map3(&mpos, pos, ch, wavo_pos_rows(pos_t), ch,
                          uint32_t(wv::attn_pos_window_rows())))
      return fail(ctx, WAVO_ECUDA, "attention: tensor map of pos");
  } else {
    // Repack into f16 rows [sections][heads][hd_pad] (zeros past hd) in the scratch.
    const int sec = L.sections + (L.sep_v ? 1 : 0);
    const uint64_t ldp = uint64_t(sec) * heads * hd_pad;
    const uint64_t prow = rel ? wavo_pos_rows(pos_t) : 0;
    const size_t bytes = align_up(rows * ldp * 2, 256) + prow * heads * hd_pad * 2;
    void *ws;
    wavo_status st = workspace(ctx, bytes, &ws);
    if (st) return st;
    __half *pk = static_cast<__half *>(ws);
    __half *pp = reinterpret_cast<__half *>(static_cast<uint8_t *>(ws) + align_up(rows * ldp * 2, 256));
    const int in_f16 = dtype == WAVO_F16;
    if (L.sep_v) {
      const int off2[2] = {0, int(ch)};
      CK(wv::launch_pack_heads(qk, in_f16, 2 * ch, off2, 2, pk, ldp, int(rows), int(heads), int(hd),
                               hd_pad, ctx->stream),
         "attention repack");
      const int off1[1] = {0};
      CK(wv::launch_pack_heads(v, in_f16, ch, off1, 1, pk + 2 * heads * hd_pad, ldp, int(rows),
                               int(heads), int(hd), hd_pad, ctx->stream),
         "attention repack v");
    } else {
      const int offs[4] = {0, int(ch), int(2 * ch), int(3 * ch)};
      CK(wv::launch_pack_heads(qk, in_f16, ld, offs, L.sections, pk, ldp, int(rows), int(heads),
                               int(hd), hd_pad, ctx->stream),
         "attention repack");
    }
    a.head_stride = hd_pad;
    a.q_off = 0;
    a.k_off = int(heads * hd_pad);
    a.v_off = int(2 * heads * hd_pad);
    a.qv_off = int(3 * heads * hd_pad);
    const bool ok = rel ? make_map3(&mq, pk, ldp, rows, ldp, wv::kAttnBlockQ) &&
                              make_map3(&mkv, pk, ldp, rows, ldp, uint32_t(bk))
                        : make_map(&mq, pk, ldp, rows, ldp, wv::kAttnBlockQ) &&
                              make_map(&mkv, pk, ldp, rows, ldp, uint32_t(bk));
    if (!ok) return fail(ctx, WAVO_ECUDA, "attention: tensor map");
    mpos = mq;
    if (rel) {
      const int off1[1] = {0};
      CK(wv::launch_pack_heads(pos, in_f16, ch, off1, 1, pp, uint64_t(heads) * hd_pad, int(prow),
                               int(heads), int(hd), hd_pad, ctx->stream),
         "attention repack pos");
      a.pos_off = 0;
      if (!make_map3(&mpos, pp, uint64_t(heads) * hd_pad, prow, uint64_t(heads) * hd_pad,
                     uint32_t(wv::attn_pos_window_rows())))
        return fail(ctx, WAVO_ECUDA, "attention: tensor map of pos");
    }
  }
  if (!a.o_tma) mo = mq;  // not read
  CK(wv::launch_attention(mq, mkv, mpos, mo, a, hd_pad, rel, int(max_len), int(nseg),
                          ctx->stream),
     "attention launch");
  return WAVO_OK;
}

}  // namespace

wavo_status wavo_attention(wavo_ctx *ctx, const void *qk, const void *v, const void *pos, void *o,
                           uint32_t t, uint32_t heads, uint32_t hd, int dtype) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  return attention_impl(ctx, qk, v, pos, o, nullptr, nullptr, 1, t, t, t, heads, hd, dtype, dtype);
}

wavo_status wavo_attention_varlen(wavo_ctx *ctx, const void *qk, const void *v, const void *pos,
                                  void *o, uint32_t rows, const int32_t *seg_start,
                                  const int32_t *seg_len, uint32_t nseg, uint32_t max_len,
                                  uint32_t pos_t, uint32_t heads, uint32_t hd, int dtype,
                                  int o_dtype) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (!seg_start || !seg_len) return fail(ctx, WAVO_EINVAL, "attention: NULL segment arrays");
  if (max_len > rows) return fail(ctx, WAVO_EINVAL, "attention: max_len %u > rows %u", max_len, rows);
  if (nseg > 65535) return fail(ctx, WAVO_EINVAL, "attention: %u segments (at most 65535)", nseg);
  return attention_impl(ctx, qk, v, pos, o, seg_start, seg_len, nseg, max_len, pos ? pos_t : 0,
                        rows, heads, hd, dtype, o_dtype);
}

wavo_status wavo_attention_rope_varlen(wavo_ctx *ctx, const void *qkv, void *o, uint32_t rows,
                                       const int32_t *seg_start, const int32_t *seg_len,
                                       uint32_t nseg, uint32_t max_len, uint32_t heads,
                                       uint32_t hd, const float *table, uint32_t table_rows,
                                       uint32_t pos, uint32_t rot, int neox, int o_dtype) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (!seg_start || !seg_len || !table)
    return fail(ctx, WAVO_EINVAL, "attention with rotary positions: NULL segment arrays or table");
  if (max_len > rows) return fail(ctx, WAVO_EINVAL, "attention: max_len %u > rows %u", max_len, rows);
  if (nseg > 65535) return fail(ctx, WAVO_EINVAL, "attention: %u segments (at most 65535)", nseg);
  if (rot == 0 || rot > hd || rot % 2 || (neox ? (rot / 2) % 8 : rot % 8) ||
      (reinterpret_cast<uintptr_t>(table) & 15u))
    return fail(ctx, WAVO_EINVAL,
                "attention with rotary positions: rot %u of hd %u (rot / 2 a multiple of 8 with "
                "neox, rot a multiple of 8 without; table 16-byte aligned)", rot, hd);
  if (uint64_t(pos) + max_len > table_rows)
    return fail(ctx, WAVO_EINVAL, "attention with rotary positions: table of %u rows < %u + %u",
                table_rows, pos, max_len);
  const RopeSpec rs{table, rot, pos, neox};
  return attention_impl(ctx, qkv, nullptr, nullptr, o, seg_start, seg_len, nseg, max_len, 0, rows,
                        heads, hd, WAVO_F16, o_dtype, &rs);
}

// ---- encoder block: LayerNorm and the conv module ---------------------------------------------

wavo_status wavo_layer_norm(wavo_ctx *ctx, const float *x, const float *w, const float *b, void *y,
                            int y_dtype, uint32_t rows, uint32_t cols, const float *table,
                            const int32_t *positions, void *yr, uint32_t hd) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (rows == 0) return WAVO_OK;
  if (!x || !w || !b || !y) return fail(ctx, WAVO_EINVAL, "layer_norm: NULL buffer");
  if (y_dtype != WAVO_F32 && y_dtype != WAVO_F16) return fail(ctx, WAVO_EINVAL, "layer_norm: dtype");
  if (cols == 0 || cols > uint32_t(wv::layer_norm_max_cols()))
    return fail(ctx, WAVO_EINVAL, "layer_norm: %u columns (1..%d)", cols, wv::layer_norm_max_cols());
  if (table && (!yr || hd == 0 || hd % 2 || cols % hd))
    return fail(ctx, WAVO_EINVAL, "layer_norm: rotary copy needs yr and even hd dividing %u", cols);
  cudaSetDevice(ctx->device);
  CK(wv::launch_layer_norm(x, w, b, y, y_dtype == WAVO_F16, int(rows), int(cols), wv::kLnNorm,
                           table, positions, table ? yr : nullptr, int(hd), ctx->stream),
     "layer_norm launch");
  return WAVO_OK;
}

namespace {

wavo_status conv_glu_impl(wavo_ctx *ctx, const float *h, const float *dw_w, const float *dw_b,
                          uint32_t kernel, const float *n_w, const float *n_b, int norm, void *y,
                          int y_dtype, uint32_t rows, const int32_t *seg_start,
                          const int32_t *seg_len, uint32_t nseg, uint32_t max_len, uint32_t ch) {
  if (rows == 0 || nseg == 0 || max_len == 0) return WAVO_OK;
  if (!h || !dw_w || !dw_b || !n_w || !n_b || !y) return fail(ctx, WAVO_EINVAL, "conv_glu: NULL buffer");
  if (y_dtype != WAVO_F32 && y_dtype != WAVO_F16) return fail(ctx, WAVO_EINVAL, "conv_glu: dtype");
  if (norm != WAVO_CONV_LAYER_NORM && norm != WAVO_CONV_AFFINE)
    return fail(ctx, WAVO_EINVAL, "conv_glu: norm %d", norm);
  if (kernel == 0 || kernel % 2 == 0 || kernel > uint32_t(wv::dwconv_max_kernel()))
    return fail(ctx, WAVO_EINVAL, "conv_glu: kernel %u (odd, at most %d)", kernel,
                wv::dwconv_max_kernel());
  if (ch == 0 || ch > uint32_t(wv::layer_norm_max_cols()))
    return fail(ctx, WAVO_EINVAL, "conv_glu: %u channels (1..%d)", ch, wv::layer_norm_max_cols());
  if (max_len > rows) return fail(ctx, WAVO_EINVAL, "conv_glu: max_len %u > rows %u", max_len, rows);
  cudaSetDevice(ctx->device);
  if (norm == WAVO_CONV_AFFINE) {
    // One pass: the per-channel affine and SiLU need no other channel of the frame.
    CK(wv::launch_dwconv(h, dw_w, dw_b, y, int(ch), int(kernel), seg_start, seg_len, int(nseg),
                         int(max_len), n_w, n_b, y_dtype == WAVO_F16, ctx->stream),
       "conv_glu launch");
    return WAVO_OK;
  }
  // The depthwise output (before the norm) in the context's scratch, then the row pass.
  void *ws;
  wavo_status st = workspace(ctx, size_t(rows) * ch * 4, &ws);
  if (st) return st;
  float *z = static_cast<float *>(ws);
  CK(wv::launch_dwconv(h, dw_w, dw_b, z, int(ch), int(kernel), seg_start, seg_len, int(nseg),
                       int(max_len), nullptr, nullptr, 0, ctx->stream),
     "conv_glu depthwise launch");
  CK(wv::launch_layer_norm(z, n_w, n_b, y, y_dtype == WAVO_F16, int(rows), int(ch),
                           wv::kLnNormSilu, nullptr, nullptr, nullptr, 0, ctx->stream),
     "conv_glu norm launch");
  return WAVO_OK;
}

}  // namespace

wavo_status wavo_conv_glu(wavo_ctx *ctx, const float *h, const float *dw_w, const float *dw_b,
                          uint32_t kernel, const float *n_w, const float *n_b, int norm, void *y,
                          int y_dtype, uint32_t t, uint32_t ch) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  return conv_glu_impl(ctx, h, dw_w, dw_b, kernel, n_w, n_b, norm, y, y_dtype, t, nullptr, nullptr,
                       1, t, ch);
}

wavo_status wavo_conv_glu_varlen(wavo_ctx *ctx, const float *h, const float *dw_w,
                                 const float *dw_b, uint32_t kernel, const float *n_w,
                                 const float *n_b, int norm, void *y, int y_dtype, uint32_t rows,
                                 const int32_t *seg_start, const int32_t *seg_len, uint32_t nseg,
                                 uint32_t max_len, uint32_t ch) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (!seg_start || !seg_len) return fail(ctx, WAVO_EINVAL, "conv_glu: NULL segment arrays");
  if (nseg > 65535) return fail(ctx, WAVO_EINVAL, "conv_glu: %u segments (at most 65535)", nseg);
  return conv_glu_impl(ctx, h, dw_w, dw_b, kernel, n_w, n_b, norm, y, y_dtype, rows, seg_start,
                       seg_len, nseg, max_len, ch);
}

// ---- the decoder step's ends -----------------------------------------------------------------

wavo_status wavo_embed_rows(wavo_ctx *ctx, const wavo_linear *l, const float *positions,
                            const int32_t *tokens, uint32_t rows, uint32_t pos, float *x,
                            uint32_t ldx) {
  if (!ctx || !l) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (rows == 0) return WAVO_OK;
  if (!tokens || !x) return fail(ctx, WAVO_EINVAL, "embed: NULL buffer");
  if (l->device != ctx->device) return fail(ctx, WAVO_EINVAL, "embed: layer of another device");
  if (ldx == 0) ldx = l->k;
  if (ldx < l->k) return fail(ctx, WAVO_EINVAL, "embed: ldx %u < k %u", ldx, l->k);
  cudaSetDevice(ctx->device);
  const bool f32w = l->ty == WAVO_GGML_F32 || l->ty == WAVO_GGML_BF16;
  const void *w = f32w ? static_cast<const void *>(l->w32)
                  : l->ty == WAVO_GGML_Q8_0 ? static_cast<const void *>(l->q8)
                                            : static_cast<const void *>(l->w16);
  const int wt = f32w ? 0 : l->ty == WAVO_GGML_Q8_0 ? 8 : 1;
  // Token ids index the layer's rows; an id past them reads the zero padding rows (up to n) at
  // most: the kernel does not check ids, so callers pass ids below the layer's rows.
  CK(wv::launch_embed(w, wt, l->d8, l->bias, positions, tokens, int(rows), int(l->k), int(pos), x,
                      ldx, ctx->stream),
     "embed launch");
  return WAVO_OK;
}

wavo_status wavo_pick(wavo_ctx *ctx, float *logits, uint32_t ld, uint32_t rows, uint32_t vocab,
                      int32_t *history, int32_t *hist_len, uint32_t max_hist,
                      const int32_t *suppress, uint32_t n_suppress,
                      const int32_t *begin_suppress, uint32_t n_begin, uint32_t eot,
                      uint32_t no_timestamps, uint32_t begin, uint32_t max_initial,
                      int32_t *tokens, float *logprobs) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (rows == 0) return WAVO_OK;
  if (!logits || !history || !hist_len || !tokens || (n_suppress && !suppress) ||
      (n_begin && !begin_suppress))
    return fail(ctx, WAVO_EINVAL, "pick: NULL buffer");
  if (ld == 0) ld = vocab;
  if (vocab == 0 || ld < vocab || begin > vocab || eot >= vocab || max_hist == 0 ||
      vocab > 0x7fffffffu)
    return fail(ctx, WAVO_EINVAL, "pick: vocab %u, ld %u, begin %u, eot %u, history %u", vocab,
                ld, begin, eot, max_hist);
  cudaSetDevice(ctx->device);
  CK(wv::launch_pick(logits, ld, int(rows), int(vocab), history, hist_len, int(max_hist), suppress,
                     int(n_suppress), begin_suppress, int(n_begin), int(eot), int(no_timestamps),
                     int(begin), int(max_initial), tokens, logprobs, ctx->stream),
     "pick launch");
  return WAVO_OK;
}

// ---- the log-mel frontend ----------------------------------------------------------------

namespace {

wavo_status frontend_tables(wavo_ctx *ctx) {
  if (ctx->fe_dev) return WAVO_OK;
  if (ctx->capturing)
    return fail(ctx, WAVO_EINVAL, "log-mel: make the first frontend call before a capture");
  CK(cudaMalloc(&ctx->fe_dev, wv::frontend_table_bytes()), "log-mel tables");
  const cudaError_t e = wv::frontend_tables_upload(ctx->fe_dev, ctx->stream, &ctx->fe_tab);
  if (e != cudaSuccess) {
    cudaFree(ctx->fe_dev);
    ctx->fe_dev = nullptr;
    return cuda_fail(ctx, e, "log-mel tables");
  }
  return WAVO_OK;
}

}  // namespace

wavo_status wavo_log_mel(wavo_ctx *ctx, const float *pcm, uint64_t samples, uint64_t f0,
                         uint64_t f1, float *mel) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  const uint64_t frames = samples / 160 + 1;
  if (!pcm || !mel || samples == 0) return fail(ctx, WAVO_EINVAL, "log-mel: NULL buffer or no samples");
  if (f0 >= f1 || f1 > frames || f1 - f0 > 0x7fffffffu)
    return fail(ctx, WAVO_EINVAL, "log-mel: frames %llu..%llu of %llu", (unsigned long long)f0,
                (unsigned long long)f1, (unsigned long long)frames);
  cudaSetDevice(ctx->device);
  wavo_status st = frontend_tables(ctx);
  if (st != WAVO_OK) return st;
  CK(wv::launch_log_mel(pcm, (long long)samples, (long long)f0, int(f1 - f0), ctx->fe_tab, mel,
                        ctx->stream),
     "log-mel launch");
  return WAVO_OK;
}

wavo_status wavo_mel_features(wavo_ctx *ctx, const float *pcm, uint64_t samples, float *mel,
                              uint64_t *frames) {
  if (!ctx || !frames) return WAVO_EINVAL;
  *frames = 0;
  const uint64_t n = samples / 160 + 1;
  if (n < 3) return WAVO_OK;  // too few frames for the normalisation: no features
  if (n > 0x7fffffffu) return fail(ctx, WAVO_EINVAL, "mel features: %llu frames", (unsigned long long)n);
  if (!pcm || !mel) return fail(ctx, WAVO_EINVAL, "mel features: NULL buffer");
  std::lock_guard<std::mutex> g(ctx->mu);
  cudaSetDevice(ctx->device);
  wavo_status st = frontend_tables(ctx);
  if (st != WAVO_OK) return st;
  void *ws = nullptr;
  st = workspace(ctx, wv::mel_features_scratch_bytes(ctx->sms), &ws);
  if (st != WAVO_OK) return st;
  CK(wv::launch_mel_features(pcm, (long long)samples, int(n), ctx->fe_tab, mel, ws, ctx->sms,
                             ctx->stream),
     "mel features launch");
  *frames = n;
  return WAVO_OK;
}

// ---- Parakeet's conv subsampling ------------------------------------------------------------

namespace {
inline uint64_t half_up(uint64_t n) { return (n - 1) / 2 + 1; }
struct SubsampleLayout {
  uint64_t t2, t, a_bytes, h_bytes, total;
};
SubsampleLayout subsample_layout(uint64_t frames, uint64_t ch) {
  SubsampleLayout L{};
  L.t2 = half_up(half_up(frames));
  L.t = half_up(half_up(half_up(frames - 1)));
  L.a_bytes = align_up(L.t2 * 32 * ch * 4, 256);
  L.h_bytes = align_up(L.t * 16 * ch * 4, 256);
  L.total = 2 * L.a_bytes + 3 * L.h_bytes;
  return L;
}
}  // namespace

uint64_t wavo_subsample_scratch_bytes(uint32_t frames, uint32_t ch) {
  return frames >= 2 && ch ? subsample_layout(frames, ch).total : 0;
}

wavo_status wavo_subsample(wavo_ctx *ctx, const float *mel, uint32_t frames, uint32_t valid,
                           uint32_t ch, const float *w0, const float *b0, const float *w2,
                           const float *b2, const wavo_linear *conv3, const float *w5,
                           const float *b5, const wavo_linear *conv6, const wavo_linear *out,
                           float *x, void *scratch, uint32_t *t_out) {
  if (!ctx) return WAVO_EINVAL;
  if (!mel || !w0 || !b0 || !w2 || !b2 || !w5 || !b5 || !conv3 || !conv6 || !out || !x || !scratch)
    return fail(ctx, WAVO_EINVAL, "subsample: NULL argument");
  if (frames < 2 || valid == 0 || valid > frames || ch == 0 || ch % 32 != 0 || ch > 4096)
    return fail(ctx, WAVO_EINVAL, "subsample: %u frames (%u valid), %u channels", frames, valid, ch);
  if (conv3->k != ch || conv3->cols != ch || conv3->dual || conv6->k != ch || conv6->cols != ch ||
      conv6->dual || out->k != 16 * ch || out->dual)
    return fail(ctx, WAVO_EINVAL, "subsample: the pointwise layers must be %u -> %u and the output "
                "projection %u -> d", ch, ch, 16 * ch);
  if (reinterpret_cast<uintptr_t>(scratch) & 255u)
    return fail(ctx, WAVO_EINVAL, "subsample: scratch must be 256-byte aligned");
  const SubsampleLayout L = subsample_layout(frames, ch);
  uint8_t *sp = static_cast<uint8_t *>(scratch);
  // The GEMMs' operands (a, h, flat) are f16, their outputs (b, y) f32.
  __half *a = reinterpret_cast<__half *>(sp);
  float *b = reinterpret_cast<float *>(sp + L.a_bytes);
  __half *h = reinterpret_cast<__half *>(sp + 2 * L.a_bytes);
  float *y = reinterpret_cast<float *>(sp + 2 * L.a_bytes + L.h_bytes);
  __half *flat = reinterpret_cast<__half *>(sp + 2 * L.a_bytes + 2 * L.h_bytes);
  const int t2 = int(L.t2), t = int(L.t);
  {
    std::lock_guard<std::mutex> g(ctx->mu);
    cudaSetDevice(ctx->device);
    CK(wv::launch_conv02(mel, int(valid), t2, int(ch), w0, b0, w2, b2, a, ctx->stream),
       "subsample conv0/conv2 launch");
  }
  wavo_status st = wavo_gemm(ctx, a, WAVO_F16, ch, conv3, b, WAVO_F32, ch, uint32_t(t2) * 32,
                             WAVO_EPI_RELU, 1.0f);
  if (st != WAVO_OK) return st;
  {
    std::lock_guard<std::mutex> g(ctx->mu);
    CK(wv::launch_dw3s2(b, t2, 32, int(ch), t, w5, b5, h, ctx->stream), "subsample conv5 launch");
  }
  st = wavo_gemm(ctx, h, WAVO_F16, ch, conv6, y, WAVO_F32, ch, uint32_t(t) * 16, WAVO_EPI_RELU, 1.0f);
  if (st != WAVO_OK) return st;
  {
    std::lock_guard<std::mutex> g(ctx->mu);
    CK(wv::launch_flatten(y, t, 16, int(ch), flat, ctx->stream), "subsample flatten launch");
  }
  st = wavo_gemm(ctx, flat, WAVO_F16, 16 * ch, out, x, WAVO_F32, 0, uint32_t(t), WAVO_EPI_BIAS, 1.0f);
  if (st != WAVO_OK) return st;
  if (t_out) *t_out = uint32_t(t);
  return WAVO_OK;
}

namespace {
// The batch's scratch: conv0/conv2's image and conv3's output for the largest segment (reused
// segment after segment), then conv5's, conv6's and the flatten's images of every segment.
struct SubsampleBatchLayout {
  uint64_t a_bytes, h_bytes, total, rows;  // rows: the segments' output rows
};
bool subsample_batch_layout(const uint32_t *frames, uint32_t n, uint64_t ch,
                            SubsampleBatchLayout *L) {
  uint64_t t2_max = 0, rows = 0;
  for (uint32_t s = 0; s < n; ++s) {
    if (frames[s] < 2) return false;
    const SubsampleLayout one = subsample_layout(frames[s], ch);
    t2_max = one.t2 > t2_max ? one.t2 : t2_max;
    rows += one.t;
  }
  L->rows = rows;
  L->a_bytes = align_up(t2_max * 32 * ch * 4, 256);
  L->h_bytes = align_up(rows * 16 * ch * 4, 256);
  L->total = 2 * L->a_bytes + 3 * L->h_bytes;
  return true;
}
}  // namespace

uint64_t wavo_subsample_batch_scratch_bytes(const uint32_t *frames, uint32_t n, uint32_t ch) {
  SubsampleBatchLayout L{};
  return frames && n && ch && subsample_batch_layout(frames, n, ch, &L) ? L.total : 0;
}

wavo_status wavo_subsample_batch(wavo_ctx *ctx, const float *mel, const uint32_t *frames,
                                 const uint32_t *valid, uint32_t n, uint32_t ch, const float *w0,
                                 const float *b0, const float *w2, const float *b2,
                                 const wavo_linear *conv3, const float *w5, const float *b5,
                                 const wavo_linear *conv6, const wavo_linear *out, float *x,
                                 void *scratch, uint32_t *t_out) {
  if (!ctx) return WAVO_EINVAL;
  if (n == 0) return WAVO_OK;
  if (!mel || !frames || !valid || !w0 || !b0 || !w2 || !b2 || !w5 || !b5 || !conv3 || !conv6 ||
      !out || !x || !scratch)
    return fail(ctx, WAVO_EINVAL, "subsample batch: NULL argument");
  for (uint32_t s = 0; s < n; ++s)
    if (frames[s] < 2 || valid[s] == 0 || valid[s] > frames[s])
      return fail(ctx, WAVO_EINVAL, "subsample batch: segment %u has %u frames (%u valid)", s,
                  frames[s], valid[s]);
  if (ch == 0 || ch % 32 != 0 || ch > 4096)
    return fail(ctx, WAVO_EINVAL, "subsample batch: %u channels", ch);
  if (conv3->k != ch || conv3->cols != ch || conv3->dual || conv6->k != ch || conv6->cols != ch ||
      conv6->dual || out->k != 16 * ch || out->dual)
    return fail(ctx, WAVO_EINVAL, "subsample batch: the pointwise layers must be %u -> %u and the "
                "output projection %u -> d", ch, ch, 16 * ch);
  if (reinterpret_cast<uintptr_t>(scratch) & 255u)
    return fail(ctx, WAVO_EINVAL, "subsample batch: scratch must be 256-byte aligned");
  SubsampleBatchLayout L{};
  subsample_batch_layout(frames, n, ch, &L);
  if (L.rows * 16 > UINT32_MAX)
    return fail(ctx, WAVO_EINVAL, "subsample batch: %llu output rows", (unsigned long long)L.rows);
  uint8_t *sp = static_cast<uint8_t *>(scratch);
  __half *a = reinterpret_cast<__half *>(sp);
  float *b = reinterpret_cast<float *>(sp + L.a_bytes);
  __half *h = reinterpret_cast<__half *>(sp + 2 * L.a_bytes);
  float *y = reinterpret_cast<float *>(sp + 2 * L.a_bytes + L.h_bytes);
  __half *flat = reinterpret_cast<__half *>(sp + 2 * L.a_bytes + 2 * L.h_bytes);
  // Per segment (its conv3 output, 32 KB a conv2 row, stays in L2 for conv5): conv0/conv2, conv3,
  // conv5 into the segment's rows of h.
  uint64_t mel_row = 0, row = 0;
  for (uint32_t s = 0; s < n; ++s) {
    const SubsampleLayout one = subsample_layout(frames[s], ch);
    const int t2 = int(one.t2), t = int(one.t);
    {
      std::lock_guard<std::mutex> g(ctx->mu);
      cudaSetDevice(ctx->device);
      CK(wv::launch_conv02(mel + mel_row * 128, int(valid[s]), t2, int(ch), w0, b0, w2, b2, a,
                           ctx->stream),
         "subsample conv0/conv2 launch");
    }
    wavo_status st = wavo_gemm(ctx, a, WAVO_F16, ch, conv3, b, WAVO_F32, ch, uint32_t(t2) * 32,
                               WAVO_EPI_RELU, 1.0f);
    if (st != WAVO_OK) return st;
    {
      std::lock_guard<std::mutex> g(ctx->mu);
      CK(wv::launch_dw3s2(b, t2, 32, int(ch), t, w5, b5, h + row * 16 * ch, ctx->stream),
         "subsample conv5 launch");
    }
    if (t_out) t_out[s] = uint32_t(t);
    mel_row += frames[s];
    row += uint64_t(t);
  }
  // Every segment's rows at once: conv6, the flatten (row by row), the output projection.
  const uint32_t rows = uint32_t(L.rows);
  wavo_status st = wavo_gemm(ctx, h, WAVO_F16, ch, conv6, y, WAVO_F32, ch, rows * 16,
                             WAVO_EPI_RELU, 1.0f);
  if (st != WAVO_OK) return st;
  {
    std::lock_guard<std::mutex> g(ctx->mu);
    CK(wv::launch_flatten(y, int(rows), 16, int(ch), flat, ctx->stream), "subsample flatten launch");
  }
  return wavo_gemm(ctx, flat, WAVO_F16, 16 * ch, out, x, WAVO_F32, 0, rows, WAVO_EPI_BIAS, 1.0f);
}

// ---- rope --------------------------------------------------------------------------------

wavo_status wavo_rope_rows(wavo_ctx *ctx, const float *table, void *qkv, int dtype,
                           uint32_t stride, uint32_t rows, uint32_t pos, const int32_t *positions,
                           uint32_t heads, uint32_t hd, uint32_t rot, int neox) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (rows == 0) return WAVO_OK;
  if (!table || !qkv) return fail(ctx, WAVO_EINVAL, "rope: NULL buffer");
  if (rot > hd || rot % 2 || (dtype != WAVO_F32 && dtype != WAVO_F16))
    return fail(ctx, WAVO_EINVAL, "rope: rot %u of hd %u", rot, hd);
  if (stride == 0) stride = 3 * heads * hd;
  if (stride < 2 * heads * hd) return fail(ctx, WAVO_EINVAL, "rope: stride %u", stride);
  cudaSetDevice(ctx->device);
  CK(wv::launch_rope(table, qkv, dtype == WAVO_F16, stride, int(rows), int(pos), positions,
                     int(heads), int(hd), int(rot), neox ? 1 : 0, 2, ctx->stream),
     "rope launch");
  return WAVO_OK;
}

wavo_status wavo_rope(wavo_ctx *ctx, const float *table, void *qkv, int dtype, uint32_t stride,
                      uint32_t rows, uint32_t pos, uint32_t heads, uint32_t hd, uint32_t rot,
                      int neox) {
  return wavo_rope_rows(ctx, table, qkv, dtype, stride, rows, pos, nullptr, heads, hd, rot, neox);
}

// ---- decoder -----------------------------------------------------------------------------

wavo_status wavo_pack_batch(wavo_ctx *ctx, const float *x, uint32_t src, uint32_t stride,
                            uint64_t x_batch, void *cache, uint64_t cache_batch, uint32_t rows,
                            uint32_t d, uint32_t cols, uint32_t col, uint32_t batch) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (rows == 0 || batch == 0) return WAVO_OK;
  if (!x || !cache) return fail(ctx, WAVO_EINVAL, "pack: NULL buffer");
  if (d % 2 || col + rows > cols)
    return fail(ctx, WAVO_EINVAL, "pack: rows %u at %u of %u positions, d %u", rows, col, cols, d);
  if (batch > 65535) return fail(ctx, WAVO_EINVAL, "pack: batch %u (at most 65535)", batch);
  cudaSetDevice(ctx->device);
  CK(wv::launch_pack_cache(x, src, stride, static_cast<uint32_t *>(cache), int(rows), int(d),
                           int(cols), int(col), (long long)x_batch, (long long)cache_batch,
                           int(batch), ctx->stream),
     "pack launch");
  return WAVO_OK;
}

wavo_status wavo_pack(wavo_ctx *ctx, const float *x, uint32_t src, uint32_t stride, void *cache,
                      uint32_t rows, uint32_t d, uint32_t cols, uint32_t col) {
  return wavo_pack_batch(ctx, x, src, stride, 0, cache, 0, rows, d, cols, col, 1);
}

size_t wavo_attend_len(uint32_t n, uint32_t heads, uint32_t hd) {
  return wv::attend_part_floats(int(n), int(heads), int(hd), 1);
}

wavo_status wavo_attend_batch(wavo_ctx *ctx, const float *q, uint64_t q_stride, const void *kv,
                              uint64_t kv_stride, float *part, float *o, uint64_t o_stride,
                              uint32_t n, uint32_t cols, uint32_t heads, uint32_t hd,
                              uint32_t batch) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (n == 0 || batch == 0) return WAVO_OK;
  if (!q || !kv || !o) return fail(ctx, WAVO_EINVAL, "attend: NULL buffer");
  if (n > cols || hd > 128 || hd % 2 || heads == 0)
    return fail(ctx, WAVO_EINVAL, "attend: n %u of %u positions, heads %u of %u", n, cols, heads, hd);
  if (wv::attend_part_floats(int(n), int(heads), int(hd), 1) > size_t(heads) * (hd + 2) && !part)
    return fail(ctx, WAVO_EINVAL, "attend: part is NULL");
  cudaSetDevice(ctx->device);
  CK(wv::launch_attend(q, q_stride, static_cast<const uint32_t *>(kv), kv_stride, part, o, o_stride,
                       int(n), int(cols), int(heads), int(hd), int(batch), ctx->stream),
     "attend launch");
  return WAVO_OK;
}

wavo_status wavo_attend(wavo_ctx *ctx, const float *q, const void *kv, float *part, float *o,
                        uint32_t n, uint32_t cols, uint32_t heads, uint32_t hd) {
  return wavo_attend_batch(ctx, q, 0, kv, 0, part, o, 0, n, cols, heads, hd, 1);
}

// ---- graphs ------------------------------------------------------------------------------

wavo_status wavo_capture_begin(wavo_ctx *ctx) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (ctx->capturing) return fail(ctx, WAVO_EINVAL, "already capturing");
  cudaSetDevice(ctx->device);
  CK(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal), "capture begin");
  ctx->capturing = true;
  return WAVO_OK;
}

wavo_status wavo_capture_end(wavo_ctx *ctx, wavo_graph **out) {
  if (!ctx || !out) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (!ctx->capturing) return fail(ctx, WAVO_EINVAL, "not capturing");
  ctx->capturing = false;
  cudaSetDevice(ctx->device);
  wavo_graph *gr = new (std::nothrow) wavo_graph();
  if (!gr) return fail(ctx, WAVO_ENOMEM, "graph");
  cudaError_t e = cudaStreamEndCapture(ctx->stream, &gr->graph);
  if (e == cudaSuccess) e = cudaGraphInstantiate(&gr->exec, gr->graph, 0);
  if (e != cudaSuccess) {
    wavo_graph_destroy(gr);
    return cuda_fail(ctx, e, "capture end");
  }
  *out = gr;
  return WAVO_OK;
}

wavo_status wavo_graph_launch(wavo_ctx *ctx, const wavo_graph *gr) {
  if (!ctx || !gr) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  cudaSetDevice(ctx->device);
  CK(cudaGraphLaunch(gr->exec, ctx->stream), "graph launch");
  return WAVO_OK;
}

void wavo_graph_destroy(wavo_graph *gr) {
  if (!gr) return;
  if (gr->exec) cudaGraphExecDestroy(gr->exec);
  if (gr->graph) cudaGraphDestroy(gr->graph);
  delete gr;
}

// ---- self-checks ---------------------------------------------------------------------------

wavo_status wavo_selftest_wait_timeout(wavo_ctx *ctx, uint64_t limit_cycles) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (limit_cycles == 0 || limit_cycles > uint64_t(wv::kWaitCycles))
    return fail(ctx, WAVO_EINVAL, "selftest_wait_timeout: limit of %llu cycles (1 .. %lld)",
                (unsigned long long)limit_cycles, wv::kWaitCycles);
  cudaSetDevice(ctx->device);
  CK(wv::launch_wait_probe(ctx->dev_err, (long long)limit_cycles, ctx->stream), "wait probe");
  return WAVO_OK;
}

wavo_status wavo_selftest_exp2(wavo_ctx *ctx, const float *x, float *y, uint32_t n) {
  if (!ctx) return WAVO_EINVAL;
  std::lock_guard<std::mutex> g(ctx->mu);
  if (n == 0) return WAVO_OK;
  if (!x || !y) return fail(ctx, WAVO_EINVAL, "selftest_exp2: NULL buffer");
  if (n > 0x7fffffffu) return fail(ctx, WAVO_EINVAL, "selftest_exp2: n %u", n);
  cudaSetDevice(ctx->device);
  CK(wv::launch_exp2_probe(x, y, int(n), ctx->stream), "exp2 probe");
  return WAVO_OK;
}

// ---- sharding ----------------------------------------------------------------------------

wavo_status wavo_partition_lpt(const uint64_t *cost, uint32_t n, uint32_t parts, uint32_t *assign) {
  if ((!cost || !assign) && n) return WAVO_EINVAL;
  if (parts == 0) return WAVO_EINVAL;
  std::vector<uint32_t> order(n);
  for (uint32_t i = 0; i < n; ++i) order[i] = i;
  // Longest first; ties by index so the partition is deterministic.
  std::stable_sort(order.begin(), order.end(),
                   [&](uint32_t a, uint32_t b) { return cost[a] > cost[b]; });
  std::vector<uint64_t> load(parts, 0);
  for (uint32_t i : order) {
    uint32_t best = 0;
    for (uint32_t p = 1; p < parts; ++p)
      if (load[p] < load[best]) best = p;
    assign[i] = best;
    load[best] += cost[i];
  }
  return WAVO_OK;
}

}  // extern "C"

// ---- decoder attention without allocation ------------------------------------------------

namespace {

// The split partials of wavo_attend_batch_noalloc: one fixed array per device, in the module's
// own device memory (no cudaMalloc). Every element the combine step reads is written first by the
// same call, so it needs no initial value.
static __device__ __align__(256) float g_attend_noalloc_part[WAVO_ATTEND_NOALLOC_PART_FLOATS];

constexpr int kNoAllocDevices = 64;
std::mutex g_noalloc_mu;
float *g_noalloc_ptr[kNoAllocDevices] = {};

// The device address of the array on the current device, looked up once per device (with that
// device current) and cached.
wavo_status noalloc_part(int device, float **out) {
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (!g_noalloc_ptr[device]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_attend_noalloc_part);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "attend_noalloc: scratch address");
    if (!p) return fail(nullptr, WAVO_ECUDA, "attend_noalloc: scratch address is NULL");
    g_noalloc_ptr[device] = static_cast<float *>(p);
  }
  *out = g_noalloc_ptr[device];
  return WAVO_OK;
}

}  // namespace

extern "C" wavo_status wavo_attend_batch_noalloc(const float *q, uint64_t q_stride, const void *kv,
                                                 uint64_t kv_stride, float *o, uint64_t o_stride,
                                                 uint32_t n, uint32_t cols, uint32_t heads,
                                                 uint32_t hd, uint32_t batch, void *stream) {
  if (n == 0 || batch == 0) return WAVO_OK;
  if (!q || !kv || !o) return fail(nullptr, WAVO_EINVAL, "attend_noalloc: NULL buffer");
  if (n > cols || hd > 128 || hd % 2 || heads == 0)
    return fail(nullptr, WAVO_EINVAL, "attend_noalloc: n %u of %u positions, heads %u of %u", n,
                cols, heads, hd);
  const size_t split_floats = size_t(batch) * heads * (hd + 2);
  const size_t need = wv::attend_part_floats(int(n), int(heads), int(hd), int(batch));
  // One split writes the output directly and uses no partials.
  if (need > split_floats && need > WAVO_ATTEND_NOALLOC_PART_FLOATS)
    return fail(nullptr, WAVO_EINVAL,
                "attend_noalloc: %zu floats of partials needed (batch %u, heads %u of %u, %u "
                "keys), the fixed scratch holds %u: split the batch",
                need, batch, heads, hd, n, WAVO_ATTEND_NOALLOC_PART_FLOATS);
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "attend_noalloc: current device");
  if (device < 0 || device >= kNoAllocDevices)
    return fail(nullptr, WAVO_EUNSUPPORTED, "attend_noalloc: device %d", device);
  float *part = nullptr;
  wavo_status st = noalloc_part(device, &part);
  if (st != WAVO_OK) return st;
  e = wv::launch_attend(q, q_stride, static_cast<const uint32_t *>(kv), kv_stride, part, o,
                        o_stride, int(n), int(cols), int(heads), int(hd), int(batch),
                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "attend_noalloc launch");
  return WAVO_OK;
}
