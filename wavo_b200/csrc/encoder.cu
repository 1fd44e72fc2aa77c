// The rest of the Conformer encoder block around the attention path: LayerNorm (with the rotary
// copy GigaAM feeds its Q/K projection) and the conv module between the pointwise convs, the
// reference's `Pass::layer_norm` (src/gpu/mod.rs:1431-1449) and `Pass::conv_glu` (1538-1566),
// CPU forms src/cpu/ops.rs:65-110 and 133-182. Both are HBM-bound row passes:
//
//   layer_norm_kernel  one warp per row: the row in registers (16-byte loads when the rows allow),
//                      mean and variance by warp shuffles, y = (x - mean)·rstd·w + b; optional
//                      SiLU (the conv module's tail) or affine-only mode; optional rotary copy
//                      (NEOX pairs inside each head) through a per-warp shared-memory row.
//   dwconv_kernel      the GLU and depthwise conv over frames of packed segments: a CTA takes 32
//                      frames x 128 channels, stages the GLU of its window (32 + kernel - 1 frames,
//                      zero outside the segment) in shared memory, one column per thread, and sums
//                      the taps in the reference's order (bias first, taps k = 0..kernel-1, one
//                      fused multiply-add each); kernels of 5, 9, 15 and 31 taps compiled with the
//                      taps in registers and eight outputs at a time from a register window. With the affine norm (a folded batch
//                      norm) the CTA also applies it and SiLU and writes y; the LayerNorm form
//                      writes the conv output for a row pass.
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

// Four consecutive outputs at p (16-byte aligned for f32, 8-byte for f16).
__device__ __forceinline__ void put4(float *p, float a, float b, float c, float d) {
  *reinterpret_cast<float4 *>(p) = make_float4(a, b, c, d);
}
__device__ __forceinline__ void put4(__half *p, float a, float b, float c, float d) {
  *reinterpret_cast<uint2 *>(p) = make_uint2(pack_half2(a, b), pack_half2(c, d));
}

// mode: kLnNorm (LayerNorm), kLnNormSilu (LayerNorm then SiLU), kLnAffineSilu (w·x + b then SiLU).
// VEC: cols a multiple of 128 and 16-byte aligned rows: lane l holds the float4 chunks l, l + 32,
// .. of the row (coalesced 512-byte warp loads); else lane l holds columns l, l + 32, ...
template <typename OutT, bool VEC>
__global__ void __launch_bounds__(32 * LN_WARPS)
    layer_norm_kernel(const float *__restrict__ x, const float *__restrict__ w,
                      const float *__restrict__ b, OutT *__restrict__ y, int rows, int cols,
                      int mode, const float *__restrict__ table, const int *__restrict__ positions,
                      OutT *__restrict__ yr, int hd) {
  griddep_launch_dependents();
  griddep_wait();  // the previous kernel of the stream has completed (programmatic launch)
  extern __shared__ float ln_rows[];  // rotary: one normalised row per warp
  const int warp = int(threadIdx.x >> 5), lane = int(threadIdx.x & 31u);
  const int r = int(blockIdx.x) * LN_WARPS + warp;
  if (r >= rows) return;
  const float *xr = x + (long long)r * cols;
  constexpr int NV = VEC ? LN_MAXV / 4 : LN_MAXV;  // loads a lane makes
  float v[LN_MAXV];
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (VEC) {
      const int c = 4 * (lane + 32 * i);
      const float4 t = c < cols ? __ldg(reinterpret_cast<const float4 *>(xr + c))
                                : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      v[4 * i] = t.x;
      v[4 * i + 1] = t.y;
      v[4 * i + 2] = t.z;
      v[4 * i + 3] = t.w;
      s += (t.x + t.y) + (t.z + t.w);
    } else {
      const int c = lane + 32 * i;
      v[i] = c < cols ? __ldg(xr + c) : 0.0f;
      s += v[i];
    }
  }
  // Column of value slot k of this lane.
  auto col = [&](int k) { return VEC ? 4 * (lane + 32 * (k >> 2)) + (k & 3) : lane + 32 * k; };
  float mean = 0.0f, rstd = 1.0f;
  if (mode != kLnAffineSilu) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    mean = s / float(cols);
    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < LN_MAXV; ++k) {
      if (col(k) < cols) {
        const float d = v[k] - mean;
        q += d * d;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    rstd = 1.0f / sqrtf(q / float(cols) + 1e-5f);
  }
  OutT *yy = y + (long long)r * cols;
  float *row = ln_rows + warp * cols;
  if (VEC) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = 4 * (lane + 32 * i);
      if (c < cols) {
        const float4 wv = __ldg(reinterpret_cast<const float4 *>(w + c));
        const float4 bv = __ldg(reinterpret_cast<const float4 *>(b + c));
        float t0 = (v[4 * i] - mean) * rstd * wv.x + bv.x;
        float t1 = (v[4 * i + 1] - mean) * rstd * wv.y + bv.y;
        float t2 = (v[4 * i + 2] - mean) * rstd * wv.z + bv.z;
        float t3 = (v[4 * i + 3] - mean) * rstd * wv.w + bv.w;
        if (mode != kLnNorm) {
          t0 = silu_f(t0);
          t1 = silu_f(t1);
          t2 = silu_f(t2);
          t3 = silu_f(t3);
        }
        put4(yy + c, t0, t1, t2, t3);
        if (table) *reinterpret_cast<float4 *>(row + c) = make_float4(t0, t1, t2, t3);
      }
    }
  } else {
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

constexpr int DW_FRAMES = 32;    // output frames per CTA
constexpr int DW_CH = 128;       // channels per CTA (one per thread)
constexpr int DW_MAXK = 63;      // largest kernel

// z[f][c] = bias[c] + Σ_k taps[c][k] · glu(h[f + k - kernel/2][c]) over the frames of the segment,
// glu(h)[c] = h[c] / (1 + exp(-h[ch + c])). K: the kernel size at compile time (the taps in
// registers, the tap loop unrolled), or 0: any odd size up to DW_MAXK (taps read from L1).
// With an affine norm (n_w non-NULL) the output is y = SiLU(n_w·z + n_b) directly, f16 when y_f16;
// else z itself (f32), for the LayerNorm pass that needs every channel of a frame.
template <int K>
__global__ void __launch_bounds__(DW_CH)
    dwconv_kernel(const float *__restrict__ h, const float *__restrict__ taps,
                  const float *__restrict__ bias, void *__restrict__ zout, int ch, int kernel,
                  const int *__restrict__ seg_start, const int *__restrict__ seg_len, int single_t,
                  const float *__restrict__ n_w, const float *__restrict__ n_b, int y_f16) {
  griddep_launch_dependents();
  griddep_wait();  // the previous kernel of the stream has completed (programmatic launch)
  extern __shared__ float dw_win[];  // [DW_FRAMES + kernel - 1][DW_CH]
  const int seg = int(blockIdx.z);
  const int T = seg_len ? seg_len[seg] : single_t;
  const int row0 = seg_len ? seg_start[seg] : 0;
  const int f0 = int(blockIdx.x) * DW_FRAMES;
  if (f0 >= T) return;
  const int cl = int(threadIdx.x), c = int(blockIdx.y) * DW_CH + cl;
  const int pad = kernel / 2, win = DW_FRAMES + kernel - 1;
  const bool live = c < ch;
  // The window, sixteen frames at a time with their loads in flight together.
  for (int i0 = 0; i0 < win; i0 += 16) {
    float hv[16], gv[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int f = f0 - pad + i0 + u;
      const bool in = live && i0 + u < win && f >= 0 && f < T;
      const float *hr = h + (long long)(row0 + (in ? f : 0)) * 2 * ch;
      hv[u] = in ? __ldg(hr + c) : 0.0f;
      gv[u] = in ? __ldg(hr + ch + c) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 16; ++u)
      if (i0 + u < win) dw_win[(i0 + u) * DW_CH + cl] = __fdividef(hv[u], 1.0f + __expf(-gv[u]));
  }
  if (!live) return;
  const float b = __ldg(bias + c);
  const int nf = min(DW_FRAMES, T - f0);
  const float *tc = taps + (long long)c * kernel;
  const float gw = n_w ? __ldg(n_w + c) : 1.0f, gb = n_w ? __ldg(n_b + c) : 0.0f;
  auto emit = [&](int fo, float acc) {
    const long long at = (long long)(row0 + f0 + fo) * ch + c;
    if (!n_w) {
      static_cast<float *>(zout)[at] = acc;
    } else {
      const float v = silu_f(acc * gw + gb);
      if (y_f16)
        static_cast<__half *>(zout)[at] = __float2half_rn(v);
      else
        static_cast<float *>(zout)[at] = v;
    }
  };
  if constexpr (K > 0) {
    float tk[K];
#pragma unroll
    for (int k = 0; k < K; ++k) tk[k] = __ldg(tc + k);
    // Eight outputs at a time from a register copy of the 8 + K - 1 window frames they read.
    for (int fo0 = 0; fo0 < nf; fo0 += 8) {
      float wv[8 + K - 1];
#pragma unroll
      for (int i = 0; i < 8 + K - 1; ++i) wv[i] = dw_win[(fo0 + i) * DW_CH + cl];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        float acc = b;
#pragma unroll
        for (int k = 0; k < K; ++k) acc = fmaf(tk[k], wv[u + k], acc);
        if (fo0 + u < nf) emit(fo0 + u, acc);
      }
    }
  } else {
    for (int fo = 0; fo < nf; ++fo) {
      float acc = b;
      for (int k = 0; k < kernel; ++k)
        acc = fmaf(__ldg(tc + k), dw_win[(fo + k) * DW_CH + cl], acc);
      emit(fo, acc);
    }
  }
}

}  // namespace

cudaError_t launch_layer_norm(const float *x, const float *w, const float *b, void *y, int y_f16,
                              int rows, int cols, int mode, const float *table,
                              const int *positions, void *yr, int hd, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  const dim3 grid((rows + LN_WARPS - 1) / LN_WARPS);
  const size_t smem = table ? size_t(LN_WARPS) * cols * 4 : 0;
  // The vector form: cols a multiple of 128 and every row, w, b, y and yr 16-byte aligned.
  const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
                       reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(y) |
                       reinterpret_cast<uintptr_t>(yr);
  const bool vec = cols % 128 == 0 && (al & 15u) == 0;
#define LN_LAUNCH(T, V)                                                                        \
  launch_pdl(layer_norm_kernel<T, V>, grid, dim3(32 * LN_WARPS), smem, s, x, w, b,               \
             static_cast<T *>(y), rows, cols, mode, table, positions, static_cast<T *>(yr), hd)
  cudaError_t e;
  if (y_f16)
    e = vec ? LN_LAUNCH(__half, true) : LN_LAUNCH(__half, false);
  else
    e = vec ? LN_LAUNCH(float, true) : LN_LAUNCH(float, false);
#undef LN_LAUNCH
  return e;
}

int layer_norm_max_cols() { return 32 * LN_MAXV; }
int dwconv_max_kernel() { return DW_MAXK; }

cudaError_t launch_dwconv(const float *h, const float *taps, const float *bias, void *z, int ch,
                          int kernel, const int *seg_start, const int *seg_len, int nseg,
                          int max_len, const float *n_w, const float *n_b, int y_f16,
                          cudaStream_t s) {
  if (max_len <= 0 || nseg <= 0) return cudaSuccess;
  const size_t smem = size_t(DW_FRAMES + kernel - 1) * DW_CH * 4;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    const int most = int(size_t(DW_FRAMES + DW_MAXK - 1) * DW_CH * 4);
    for (auto f : {dwconv_kernel<0>, dwconv_kernel<5>, dwconv_kernel<9>, dwconv_kernel<15>,
                   dwconv_kernel<31>}) {
      cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
      if (e != cudaSuccess) return e;
    }
    configured[dev] = true;
  }
  const dim3 grid((max_len + DW_FRAMES - 1) / DW_FRAMES, (ch + DW_CH - 1) / DW_CH, nseg);
  auto f = kernel == 5 ? dwconv_kernel<5> : kernel == 9 ? dwconv_kernel<9>
         : kernel == 15 ? dwconv_kernel<15> : kernel == 31 ? dwconv_kernel<31> : dwconv_kernel<0>;
  return launch_pdl(f, grid, dim3(DW_CH), smem, s, h, taps, bias, z, ch, kernel, seg_start,
                    seg_len, seg_len ? 0 : max_len, n_w, n_b, y_f16);
}

}  // namespace wv
