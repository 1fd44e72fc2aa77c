// The rest of the Conformer encoder block around the attention path: LayerNorm (with the rotary
// copy GigaAM feeds its Q/K projection) and the conv module between the pointwise convs, the
// reference's `Pass::layer_norm` (src/gpu/mod.rs:1431-1449) and `Pass::conv_glu` (1538-1566),
// CPU forms src/cpu/ops.rs:65-110 and 133-182. Both are HBM-bound row passes:
//
//   layer_norm_kernel  one warp per row: the row in registers (lane l holds columns l, l + 32, ..),
//                      mean and variance by warp shuffles, y = (x - mean)·rstd·w + b; optional
//                      SiLU (the conv module's tail) or affine-only mode; optional rotary copy
//                      (NEOX pairs inside each head) through a per-warp shared-memory row.
//   dwconv_kernel      the GLU and depthwise conv over frames of packed segments: a CTA takes 64
//                      frames x 128 channels, stages the GLU of its window (64 + kernel - 1 frames,
//                      zero outside the segment) in shared memory, one column per thread, and sums
//                      the taps in the reference's order (bias first, taps k = 0..kernel-1,
//                      separately rounded products and sums).
#include "kernels.cuh"
#include "ptx.cuh"

namespace wv {
namespace {

constexpr int LN_WARPS = 4;       // rows per CTA
constexpr int LN_MAXV = 64;       // values a lane holds: cols <= 2048

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

template <typename OutT>
__device__ __forceinline__ void put(OutT *p, float v);
template <>
__device__ __forceinline__ void put<float>(float *p, float v) { *p = v; }
template <>
__device__ __forceinline__ void put<__half>(__half *p, float v) { *p = __float2half_rn(v); }

// mode: kLnNorm (LayerNorm), kLnNormSilu (LayerNorm then SiLU), kLnAffineSilu (w·x + b then SiLU).
template <typename OutT>
__global__ void __launch_bounds__(32 * LN_WARPS)
    layer_norm_kernel(const float *__restrict__ x, const float *__restrict__ w,
                      const float *__restrict__ b, OutT *__restrict__ y, int rows, int cols,
                      int mode, const float *__restrict__ table, const int *__restrict__ positions,
                      OutT *__restrict__ yr, int hd) {
  extern __shared__ float ln_rows[];  // rotary: one normalised row per warp
  const int warp = int(threadIdx.x >> 5), lane = int(threadIdx.x & 31u);
  const int r = int(blockIdx.x) * LN_WARPS + warp;
  if (r >= rows) return;
  const float *xr = x + (long long)r * cols;
  float v[LN_MAXV];
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i) {
    const int c = lane + 32 * i;
    v[i] = c < cols ? __ldg(xr + c) : 0.0f;
    s += v[i];
  }
  float mean = 0.0f, rstd = 1.0f;
  if (mode != kLnAffineSilu) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    mean = s / float(cols);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < LN_MAXV; ++i) {
      const int c = lane + 32 * i;
      if (c < cols) {
        const float d = v[i] - mean;
        q += d * d;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    rstd = 1.0f / sqrtf(q / float(cols) + 1e-5f);
  }
  OutT *yy = y + (long long)r * cols;
  float *row = ln_rows + warp * cols;
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i) {
    const int c = lane + 32 * i;
    if (c < cols) {
      float t = (v[i] - mean) * rstd * __ldg(w + c) + __ldg(b + c);
      if (mode != kLnNorm) t = silu_f(t);
      put(yy + c, t);
      if (table) row[c] = t;
    }
  }
  if (!table) return;
  __syncwarp();
  // The rotary copy: NEOX pairs (i, i + hd/2) of each head, table row positions[r] (or r).
  const int half = hd / 2;
  const float *cs = table + (long long)(positions ? positions[r] : r) * hd;
  OutT *yo = yr + (long long)r * cols;
  for (int p = lane; p < (cols / hd) * half; p += 32) {
    const int h0 = (p / half) * hd, i = p % half;
    const float y0 = row[h0 + i], y1 = row[h0 + i + half];
    const float c = __ldg(cs + i), sn = __ldg(cs + half + i);
    put(yo + h0 + i, y0 * c - y1 * sn);
    put(yo + h0 + i + half, y1 * c + y0 * sn);
  }
}

constexpr int DW_FRAMES = 64;    // output frames per CTA
constexpr int DW_CH = 128;       // channels per CTA (one per thread)
constexpr int DW_MAXK = 63;      // largest kernel

// z[f][c] = bias[c] + Σ_k taps[c][k] · glu(h[f + k - kernel/2][c]) over the frames of the segment,
// glu(h)[c] = h[c] / (1 + exp(-h[ch + c])).
__global__ void __launch_bounds__(DW_CH)
    dwconv_kernel(const float *__restrict__ h, const float *__restrict__ taps,
                  const float *__restrict__ bias, float *__restrict__ z, int ch, int kernel,
                  const int *__restrict__ seg_start, const int *__restrict__ seg_len, int single_t) {
  extern __shared__ float dw_win[];  // [DW_FRAMES + kernel - 1][DW_CH]
  const int seg = int(blockIdx.z);
  const int T = seg_len ? seg_len[seg] : single_t;
  const int row0 = seg_len ? seg_start[seg] : 0;
  const int f0 = int(blockIdx.x) * DW_FRAMES;
  if (f0 >= T) return;
  const int cl = int(threadIdx.x), c = int(blockIdx.y) * DW_CH + cl;
  const int pad = kernel / 2, win = DW_FRAMES + kernel - 1;
  const bool live = c < ch;
  for (int i = 0; i < win; ++i) {
    const int f = f0 - pad + i;
    float g = 0.0f;
    if (live && f >= 0 && f < T) {
      const float *hr = h + (long long)(row0 + f) * 2 * ch;
      g = __ldg(hr + c) / (1.0f + expf(-__ldg(hr + ch + c)));
    }
    dw_win[i * DW_CH + cl] = g;
  }
  if (!live) return;
  float tk[DW_MAXK];
#pragma unroll
  for (int k = 0; k < DW_MAXK; ++k) tk[k] = k < kernel ? __ldg(taps + (long long)c * kernel + k) : 0.0f;
  const float b = __ldg(bias + c);
  const int nf = min(DW_FRAMES, T - f0);
  for (int fo = 0; fo < nf; ++fo) {
    float acc = b;
#pragma unroll
    for (int k = 0; k < DW_MAXK; ++k)
      if (k < kernel) acc = __fadd_rn(acc, __fmul_rn(tk[k], dw_win[(fo + k) * DW_CH + cl]));
    z[(long long)(row0 + f0 + fo) * ch + c] = acc;
  }
}

}  // namespace

cudaError_t launch_layer_norm(const float *x, const float *w, const float *b, void *y, int y_f16,
                              int rows, int cols, int mode, const float *table,
                              const int *positions, void *yr, int hd, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  const dim3 grid((rows + LN_WARPS - 1) / LN_WARPS);
  const size_t smem = table ? size_t(LN_WARPS) * cols * 4 : 0;
  if (y_f16)
    layer_norm_kernel<__half><<<grid, 32 * LN_WARPS, smem, s>>>(
        x, w, b, static_cast<__half *>(y), rows, cols, mode, table, positions,
        static_cast<__half *>(yr), hd);
  else
    layer_norm_kernel<float><<<grid, 32 * LN_WARPS, smem, s>>>(
        x, w, b, static_cast<float *>(y), rows, cols, mode, table, positions,
        static_cast<float *>(yr), hd);
  return cudaGetLastError();
}

int layer_norm_max_cols() { return 32 * LN_MAXV; }
int dwconv_max_kernel() { return DW_MAXK; }

cudaError_t launch_dwconv(const float *h, const float *taps, const float *bias, float *z, int ch,
                          int kernel, const int *seg_start, const int *seg_len, int nseg,
                          int max_len, cudaStream_t s) {
  if (max_len <= 0 || nseg <= 0) return cudaSuccess;
  const size_t smem = size_t(DW_FRAMES + kernel - 1) * DW_CH * 4;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(dwconv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(size_t(DW_FRAMES + DW_MAXK - 1) * DW_CH * 4));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const dim3 grid((max_len + DW_FRAMES - 1) / DW_FRAMES, (ch + DW_CH - 1) / DW_CH, nseg);
  dwconv_kernel<<<grid, DW_CH, smem, s>>>(h, taps, bias, z, ch, kernel, seg_start, seg_len,
                                          seg_len ? 0 : max_len);
  return cudaGetLastError();
}

}  // namespace wv
