// The Parakeet log-mel frontend on the device (src/parakeet/frontend.rs, src/fft.rs): pre-emphasis
// in f64, a symmetric Hann(400) centred in an f64 FFT of 512, power cast to f32, the Slaney
// filterbank as f32 fused multiply-adds in bin order, ln(mel + 2^-24), then each mel bin normalised
// over all frames but the last, which is zero. The FFT performs the reference's operations in its
// order (radix-2 decimation in time, Stockham order, every multiply-add fused, the same cos/sin
// table), so the spectrum is the reference's bit for bit; the reductions of the normalisation are
// f64 sums in a fixed order (chunks of frames, then the chunks in order).
//
//   log_mel_kernel   a warp a frame at a time (13 warps, one CTA an SM, looping over frames): the
//                    tables copied once into shared memory, the frame's pcm staged from
//                    registers (the next frame's fetched during this one's FFT), the windowed
//                    frame in the first stage's order, nine butterfly stages between two
//                    shared-memory buffers (16-byte loads of each butterfly's input pair), the
//                    power spectrum, four mel bins a lane.
//   mel_sum_kernel   per chunk of 64 frames, a thread a mel bin: the f64 sum of the values (or of
//                    the squared deviations from the mean) in frame order (coalesced rows, eight
//                    loads in flight).
//   mel_stats_kernel the chunk sums in order: the mean, then 1 / (unbiased std + 1e-5).
//   mel_norm_kernel  (x - mean)·inv to f32; the last frame zero.
//   conv02_kernel / dw3s2_kernel / flatten_kernel
//                    Parakeet's 8x conv subsampling around the pointwise GEMMs
//                    (src/parakeet/cpu.rs:60-174).
#include <cuda_runtime.h>

#include <cmath>
#include <memory>
#include <vector>

#include "kernels.cuh"
#include "ptx.cuh"

namespace wv {
namespace {

constexpr int FE_MELS = 128, FE_NFFT = 512, FE_WINDOW = 400, FE_HOP = 160, FE_BINS = 257;
constexpr int FE_STAGES = 9, FE_HALF = FE_NFFT / 2;
constexpr int FE_WARPS = 13;  // one CTA an SM: 13 frames in flight (16 KB of buffers each)
constexpr int FE_CHUNK = 64;

constexpr int FE_SPAN_MAX = 16;  // FFT bins in a mel bin's nonzero span (12 for the Slaney bank)
constexpr int FE_STAGE_P = FE_NFFT + 1;               // pcm samples a frame reads
constexpr int FE_PF = (FE_STAGE_P + 31) / 32;         // of them a lane's (17)

// Shared tables of a CTA, built once on the host as one image in this layout: the 256 twiddles
// (every stage's twiddle is one of them: output i of the stage to blocks of `size` takes index
// i / (512 / size) · (512 / size)), the window in the first stage's order, that order, and the
// filterbank as each mel bin's nonzero span, weight k of bin m at fw[k][m] (a warp's lanes read
// consecutive words).
struct FeShared {
  double twc[256], tws[256], win[FE_NFFT];
  float fw[FE_SPAN_MAX][FE_MELS];
  int lo[FE_MELS], len[FE_MELS];
  uint16_t perm[FE_NFFT];
};
static_assert(sizeof(FeShared) % 16 == 0, "the image is copied in 16-byte words");
constexpr size_t FE_SMEM = sizeof(FeShared) + size_t(FE_WARPS) * 4 * FE_NFFT * 8;

// The frame's pcm is staged with a word of padding every 16: the first stage's order reads it at a
// stride of 16 words, which the padding spreads over all 32 banks.
__device__ __forceinline__ int fe_pad(int p) { return p + (p >> 4); }

// A lane's share of frame t's pcm (samples (f0 + t)·160 − 257 + p, p = lane + 32·q; 0 outside).
__device__ __forceinline__ void fe_fetch(const float *__restrict__ pcm, long long n_pcm,
                                         long long j0, int lane, float (&pf)[FE_PF]) {
#pragma unroll
  for (int q = 0; q < FE_PF; ++q) {
    const int p = lane + 32 * q;
    const long long idx = j0 - FE_NFFT / 2 - 1 + p;
    pf[q] = p < FE_STAGE_P && idx >= 0 && idx < n_pcm ? __ldg(pcm + idx) : 0.0f;
  }
}

__global__ void __launch_bounds__(32 * FE_WARPS, 1)
    log_mel_kernel(const float *__restrict__ pcm, long long n_pcm, long long f0, int frames,
                   const FrontendTables tab, float *__restrict__ mel) {
  extern __shared__ double fe_smem[];
  FeShared &sh = *reinterpret_cast<FeShared *>(fe_smem);
  {  // the constant tables, every load in flight at once, before the wait
    constexpr int WORDS = int(sizeof(FeShared) / 16);
    constexpr int PER = (WORDS + 32 * FE_WARPS - 1) / (32 * FE_WARPS);
    const uint4 *src = static_cast<const uint4 *>(tab.image);
    uint4 *dst = reinterpret_cast<uint4 *>(fe_smem);
    uint4 w[PER];
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int e = int(threadIdx.x) + 32 * FE_WARPS * q;
      if (e < WORDS) w[q] = __ldg(src + e);
    }
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int e = int(threadIdx.x) + 32 * FE_WARPS * q;
      if (e < WORDS) dst[e] = w[q];
    }
  }
  griddep_launch_dependents();
  griddep_wait();
  __syncthreads();
  const int warp = int(threadIdx.x >> 5), lane = int(threadIdx.x & 31);
  double *ar = fe_smem + sizeof(FeShared) / 8 + warp * 4 * FE_NFFT, *ai = ar + FE_NFFT;
  double *br = ai + FE_NFFT, *bi = br + FE_NFFT;
  float *stage = reinterpret_cast<float *>(br);  // the frame's pcm, before the first stage
  const int step = int(gridDim.x) * FE_WARPS;
  int t = int(blockIdx.x) * FE_WARPS + warp;
  float pf[FE_PF];
  if (t < frames) fe_fetch(pcm, n_pcm, (f0 + t) * FE_HOP, lane, pf);
#pragma unroll 1
  for (; t < frames; t += step) {
    const long long j0 = (f0 + t) * FE_HOP;  // the frame's first padded index + 256
    // Stage the frame's pcm (545 words with the padding, inside the second buffer), then fetch
    // the next frame's while this one is transformed.
#pragma unroll
    for (int q = 0; q < FE_PF; ++q) {
      const int p = lane + 32 * q;
      if (p < FE_STAGE_P) stage[fe_pad(p)] = pf[q];
    }
    if (t + step < frames) fe_fetch(pcm, n_pcm, (f0 + t + step) * FE_HOP, lane, pf);
    __syncwarp();
    // The windowed, pre-emphasised frame in the first stage's order (src/fft.rs:89-92).
    double xs[FE_NFFT / 32];
#pragma unroll
    for (int q = 0; q < FE_NFFT / 32; ++q) {
      const int v = lane + 32 * q;
      const int i = sh.perm[v];
      const long long j = j0 + i - FE_NFFT / 2;  // the pcm index of padded sample j0 + i
      double s = 0.0;
      if (j == 0)
        s = double(stage[fe_pad(i + 1)]);
      else if (j > 0 && j < n_pcm)
        s = __dsub_rn(double(stage[fe_pad(i + 1)]), __dmul_rn(double(0.97f), double(stage[fe_pad(i)])));
      xs[q] = __dmul_rn(s, sh.win[v]);
    }
    __syncwarp();  // the staged pcm is read before the buffer is reused
#pragma unroll
    for (int q = 0; q < FE_NFFT / 32; ++q) {
      ar[lane + 32 * q] = xs[q];
      ai[lane + 32 * q] = 0.0;
    }
    __syncwarp();
    // Nine radix-2 stages (src/fft.rs:131-143): output i reads inputs 2i and 2i + 1.
    double *sr = ar, *si = ai, *dr = br, *di = bi;
#pragma unroll 1
    for (int st = 0; st < FE_STAGES; ++st) {
      const int sh_bits = 8 - st;
#pragma unroll
      for (int q = 0; q < FE_HALF / 32; ++q) {
        const int i = lane + 32 * q;
        const int idx = (i >> sh_bits) << sh_bits;
        const double c = sh.twc[idx], s = sh.tws[idx];
        const double2 xr = reinterpret_cast<const double2 *>(sr)[i];
        const double2 xi = reinterpret_cast<const double2 *>(si)[i];
        const double a = xr.x, x = xr.y, b = xi.x, y = xi.y;
        dr[i] = fma(s, y, fma(c, x, a));
        di[i] = fma(-s, x, fma(c, y, b));
        dr[i + FE_HALF] = fma(-s, y, fma(-c, x, a));
        di[i + FE_HALF] = fma(s, x, fma(-c, y, b));
      }
      __syncwarp();
      double *tr = sr, *ti = si;
      sr = dr;
      si = di;
      dr = tr;
      di = ti;
    }
    // The power spectrum (f64 products and sum, cast to f32) over the freed buffer.
    float *power = reinterpret_cast<float *>(dr);
    for (int k = lane; k < FE_BINS; k += 32)
      power[k] = float(__dadd_rn(__dmul_rn(sr[k], sr[k]), __dmul_rn(si[k], si[k])));
    __syncwarp();
    float *out = mel + (long long)t * FE_MELS;
#pragma unroll
    for (int q = 0; q < FE_MELS / 32; ++q) {
      const int m = lane + 32 * q;
      const float *pw = power + sh.lo[m];
      float e = 0.0f;
      for (int k = 0; k < sh.len[m]; ++k) e = fmaf(sh.fw[k][m], pw[k], e);
      out[m] = logf(__fadd_rn(e, 1.0f / float(1 << 24)));
    }
    __syncwarp();  // power (in dr) is read before the next frame stages its pcm into br
  }
}

// Per chunk of FE_CHUNK frames of the first n, thread m: the f64 sum in frame order of mel values
// (mean == nullptr) or of their squared deviations from mean[m].
__global__ void mel_sum_kernel(const float *__restrict__ mel, long long n,
                               const double *__restrict__ mean, double *__restrict__ part) {
  griddep_launch_dependents();
  griddep_wait();
  const int m = int(threadIdx.x);
  const long long t0 = (long long)blockIdx.x * FE_CHUNK;
  const long long t1 = t0 + FE_CHUNK < n ? t0 + FE_CHUNK : n;
  double s = 0.0;
  const double mu = mean ? mean[m] : 0.0;
#pragma unroll 8
  for (long long t = t0; t < t1; ++t) {
    const double x = double(mel[t * FE_MELS + m]);
    if (mean) {
      const double d = __dsub_rn(x, mu);
      s = __dadd_rn(s, __dmul_rn(d, d));
    } else {
      s = __dadd_rn(s, x);
    }
  }
  part[(long long)blockIdx.x * FE_MELS + m] = s;
}

// The chunk sums in order: mean = Σ / n (var == nullptr), or inv = 1 / (sqrt(Σ / (n - 1)) + 1e-5).
__global__ void mel_stats_kernel(const double *__restrict__ part, int chunks, long long n,
                                 double *__restrict__ out, int is_var) {
  griddep_launch_dependents();
  griddep_wait();
  const int m = int(threadIdx.x);
  double s = 0.0;
  for (int c = 0; c < chunks; ++c) s = __dadd_rn(s, part[(long long)c * FE_MELS + m]);
  out[m] = is_var ? 1.0 / __dadd_rn(sqrt(s / double(n - 1)), double(1e-5f)) : s / double(n);
}

__global__ void mel_norm_kernel(float *__restrict__ mel, long long frames,
                                const double *__restrict__ mean, const double *__restrict__ inv) {
  griddep_launch_dependents();
  griddep_wait();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= frames * FE_MELS) return;
  const int m = int(i % FE_MELS);
  const long long t = i / FE_MELS;
  mel[i] = t == frames - 1 ? 0.0f : float(__dmul_rn(__dsub_rn(double(mel[i]), mean[m]), inv[m]));
}

// ---- Parakeet's 8x conv subsampling (src/parakeet/cpu.rs:100-174) -------------------------------
//
// Each output element by one thread (channels fastest: coalesced rows), in the reference's
// operation order: a bias, then each tap's product added (separate roundings, no fused
// multiply-add), taps in order.

// conv2 (depthwise 3x3, stride 2) over conv0 (3x3, stride 2, one input channel) + ReLU into
// a [t2][32][ch] as f16 (the pointwise GEMM's operand, which rounds its rows to f16 as the
// reference's GEMM does), rows from live on zero. A CTA takes conv2 row k, a thread a channel (its
// taps and biases in registers) over the row's 32 columns; the seven mel rows 4k - 3 .. 4k + 3
// the row reads are staged in shared memory with zeros past the valid frames and the band's
// edges. conv0 is evaluated where conv2 reads it (zero outside rows 0 .. t1 - 1, as the reference
// zero-fills), each value once along the row: a 3x3 window of it slides two columns a step, and
// the step's two conv0 columns read mel columns 4fo - 1 .. 4fo + 3 of each staged row (one 16-byte
// and one 4-byte load a row: the loads are the same for every thread of the CTA).
constexpr int C02_W = 132;  // a staged row: mel columns -1 .. 130 (16-byte aligned rows)

// conv0 at one pixel from its 3x3 mel patch p[dr][dc], in the reference's order.
__device__ __forceinline__ float conv0_px(float p00, float p01, float p02, float p10, float p11,
                                          float p12, float p20, float p21, float p22,
                                          const float (&w)[9], float bias) {
  const float v[9] = {p00, p01, p02, p10, p11, p12, p20, p21, p22};
  float p = bias;
#pragma unroll
  for (int t0 = 0; t0 < 9; ++t0) p = __fadd_rn(p, __fmul_rn(w[t0], v[t0]));
  return fmaxf(p, 0.0f);
}

__global__ void __launch_bounds__(256, 3) conv02_kernel(const float *__restrict__ mel, int valid, int t1, int t2, int live,
                              int ch, const float *__restrict__ w0, const float *__restrict__ b0,
                              const float *__restrict__ w2, const float *__restrict__ b2,
                              __half *__restrict__ a) {
  griddep_launch_dependents();
  griddep_wait();
  __shared__ __align__(16) float ms[7][C02_W];  // mel rows 4k - 3 + i, columns -1 .. 130
  const int k = int(blockIdx.x);
  for (int e = threadIdx.x; e < 7 * C02_W; e += blockDim.x) {
    const int i = e / C02_W, c = e % C02_W - 1;
    const int tm = 4 * k - 3 + i;
    ms[i][c + 1] = tm >= 0 && tm < valid && c >= 0 && c < 128 ? mel[(long long)tm * 128 + c] : 0.0f;
  }
  __syncthreads();
  for (int q = threadIdx.x; q < ch; q += blockDim.x) {
    __half *out = a + (long long)k * 32 * ch + q;
    if (k >= live) {
      for (int fo = 0; fo < 32; ++fo) out[fo * ch] = __float2half_rn(0.0f);
      continue;
    }
    float c0w[9], c2w[9];
#pragma unroll
    for (int tap = 0; tap < 9; ++tap) {
      c0w[tap] = w0[tap * ch + q];
      c2w[tap] = w2[tap * ch + q];
    }
    const float bias0 = b0[q], bias2 = b2[q];
    bool row_in[3];  // conv0 row 2k - 1 + rr exists (the reference zero-fills outside)
#pragma unroll
    for (int rr = 0; rr < 3; ++rr) row_in[rr] = 2 * k - 1 + rr >= 0 && 2 * k - 1 + rr < t1;
    // win[rr][cc]: conv0 at row 2k - 1 + rr (staged mel rows from 2rr on), column 2fo - 1 + cc.
    float win[3][3];
#pragma unroll
    for (int rr = 0; rr < 3; ++rr) win[rr][2] = 0.0f;  // column -1 (becomes cc = 0 below)
#pragma unroll 1
    for (int fo = 0; fo < 32; ++fo) {
      float m[7][5];  // mel columns 4fo - 1 .. 4fo + 3 of the seven staged rows
#pragma unroll
      for (int i = 0; i < 7; ++i) {
        const float4 v = *reinterpret_cast<const float4 *>(&ms[i][4 * fo]);
        m[i][0] = v.x;
        m[i][1] = v.y;
        m[i][2] = v.z;
        m[i][3] = v.w;
        m[i][4] = ms[i][4 * fo + 4];
      }
#pragma unroll
      for (int rr = 0; rr < 3; ++rr) {
        const int r = 2 * rr;
        win[rr][0] = win[rr][2];
        win[rr][1] = row_in[rr] ? conv0_px(m[r][0], m[r][1], m[r][2], m[r + 1][0], m[r + 1][1],
                                           m[r + 1][2], m[r + 2][0], m[r + 2][1], m[r + 2][2],
                                           c0w, bias0)
                                : 0.0f;
        win[rr][2] = row_in[rr] ? conv0_px(m[r][2], m[r][3], m[r][4], m[r + 1][2], m[r + 1][3],
                                           m[r + 1][4], m[r + 2][2], m[r + 2][3], m[r + 2][4],
                                           c0w, bias0)
                                : 0.0f;
      }
      float y = bias2;
#pragma unroll
      for (int tap = 0; tap < 9; ++tap) {
        if (fo == 0 && tap % 3 == 0) continue;  // column -1: outside conv0, no term
        y = __fadd_rn(y, __fmul_rn(c2w[tap], win[tap / 3][tap % 3]));
      }
      out[fo * ch] = __float2half_rn(y);
    }
  }
}

// Depthwise 3x3, stride 2, padding 1, + bias over x [t][f][ch] into y [rows][half(f)][ch].
__global__ void dw3s2_kernel(const float *__restrict__ x, int t, int f, int ch, int rows,
                             const float *__restrict__ w, const float *__restrict__ b,
                             __half *__restrict__ y) {
  griddep_launch_dependents();
  griddep_wait();
  const int fo_n = (f - 1) / 2 + 1;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)rows * fo_n * ch) return;
  const int q = int(i % ch);
  const int fo = int((i / ch) % fo_n);
  const int k = int(i / ((long long)fo_n * ch));
  float v = b[q];
#pragma unroll
  for (int tap = 0; tap < 9; ++tap) {
    const int ti = 2 * k + tap / 3, fi = 2 * fo + tap % 3;
    if (ti < 1 || ti > t || fi < 1 || fi > f) continue;
    v = __fadd_rn(v, __fmul_rn(w[tap * ch + q], x[((long long)(ti - 1) * f + fi - 1) * ch + q]));
  }
  y[i] = __float2half_rn(v);  // the pointwise GEMM's operand (rounded to f16 there as well)
}

// [t][f][ch] to [t][ch·f] (src/parakeet/cpu.rs:85-90).
__global__ void flatten_kernel(const float *__restrict__ y, int t, int f, int ch,
                               __half *__restrict__ h) {
  griddep_launch_dependents();
  griddep_wait();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long row = (long long)f * ch;
  if (i >= (long long)t * row) return;
  const long long r = i / row;
  const int e = int(i - r * row);
  h[i] = __float2half_rn(y[r * row + (e % f) * ch + e / f]);  // the output GEMM's f16 operand
}

}  // namespace

// ---- tables (host), as src/fft.rs:46-66 and src/parakeet/frontend.rs:30-47, 110-140 build them --

size_t frontend_table_bytes() { return sizeof(FeShared); }

cudaError_t frontend_tables_upload(void *dev, cudaStream_t s, FrontendTables *out) {
  const int n = FE_NFFT;
  std::vector<int> starts{0};
  while (int(starts.size()) < n) {  // leaf 1: all 512 points are radix-2 blocks
    std::vector<int> next;
    for (int v : starts) next.push_back(2 * v);
    for (int v : starts) next.push_back(2 * v + 1);
    starts = next;
  }
  std::unique_ptr<FeShared> owner(new FeShared());  // the image (18 KB), zero-filled
  FeShared &img = *owner;
  for (int i = 0; i < n; ++i) img.perm[i] = uint16_t(starts[i]);
  // The stages' twiddles: stage `size` takes cos/sin(tau·idx/512) at idx = i / (512 / size) ·
  // (512 / size), one of these 256.
  const double tau = 6.283185307179586;
  for (int idx = 0; idx < n / 2; ++idx) {
    const double phase = tau * double(idx) / double(n);
    img.twc[idx] = std::cos(phase);
    img.tws[idx] = std::sin(phase);
  }
  for (int v = 0; v < n; ++v) {  // the window, read in the first stage's order
    const int k = int(starts[v]) - (FE_NFFT - FE_WINDOW) / 2;
    img.win[v] = k >= 0 && k < FE_WINDOW
                     ? 0.5 - 0.5 * std::cos(2.0 * M_PI * double(k) / double(FE_WINDOW - 1))
                     : 0.0;
  }
  // Slaney filterbank (librosa mel(16000, 512, 128, 0, 8000, norm='slaney')) in f64, stored f32.
  const double fsp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / fsp;
  const double log_step = std::log(6.4) / 27.0;
  auto hz_to_mel = [&](double hz) {
    return hz < min_log_hz ? hz / fsp : min_log_mel + std::log(hz / min_log_hz) / log_step;
  };
  auto mel_to_hz = [&](double mel) {
    return mel < min_log_mel ? mel * fsp : min_log_hz * std::exp(log_step * (mel - min_log_mel));
  };
  const double mel_max = hz_to_mel(8000.0);
  std::vector<double> hz(FE_MELS + 2);
  for (int m = 0; m < FE_MELS + 2; ++m) hz[m] = mel_to_hz(mel_max * double(m) / double(FE_MELS + 1));
  std::vector<float> filters(FE_MELS * FE_BINS);
  std::vector<int> lo(FE_MELS), hi(FE_MELS);
  for (int m = 0; m < FE_MELS; ++m) {
    const double enorm = 2.0 / (hz[m + 2] - hz[m]);
    for (int k = 0; k < FE_BINS; ++k) {
      const double f = 16000.0 * double(k) / double(FE_NFFT);
      const double lower = (f - hz[m]) / (hz[m + 1] - hz[m]);
      const double upper = (hz[m + 2] - f) / (hz[m + 2] - hz[m + 1]);
      filters[m * FE_BINS + k] = float(std::fmax(std::fmin(lower, upper), 0.0) * enorm);
    }
    int a = 0;
    while (a < FE_BINS && filters[m * FE_BINS + a] == 0.0f) ++a;
    int b = FE_BINS;
    while (b > a && filters[m * FE_BINS + b - 1] == 0.0f) --b;
    lo[m] = a == FE_BINS ? 0 : a;
    hi[m] = a == FE_BINS ? 0 : b;
  }
  for (int m = 0; m < FE_MELS; ++m) {
    if (hi[m] - lo[m] > FE_SPAN_MAX) return cudaErrorInvalidValue;
    img.lo[m] = lo[m];
    img.len[m] = hi[m] - lo[m];
    for (int k = lo[m]; k < hi[m]; ++k) img.fw[k - lo[m]][m] = filters[m * FE_BINS + k];
  }
  cudaError_t e = cudaMemcpyAsync(dev, &img, sizeof(FeShared), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);  // before the host image is freed
  out->image = dev;
  return e;
}

cudaError_t launch_log_mel(const float *pcm, long long n_pcm, long long f0, int frames,
                           const FrontendTables &tab, float *mel, cudaStream_t s) {
  if (frames <= 0) return cudaSuccess;
  // The shared tables, then four 512-point complex f64 buffers a warp (16 KB).
  const size_t smem = FE_SMEM;
  static bool configured[64] = {};
  static int sms[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(log_mel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(smem));
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  // One CTA an SM at most, each warp looping over frames (the tables load once a CTA).
  int ctas = (frames + FE_WARPS - 1) / FE_WARPS;
  if (ctas > sms[dev]) ctas = sms[dev];
  return launch_pdl(log_mel_kernel, dim3(ctas), dim3(32 * FE_WARPS), smem, s, pcm, n_pcm, f0,
                    frames, tab, mel);
}

size_t mel_norm_scratch_bytes(long long frames) {
  const long long chunks = (frames + FE_CHUNK - 1) / FE_CHUNK;
  return size_t(chunks) * FE_MELS * 8 + 2 * FE_MELS * 8;
}

cudaError_t launch_mel_norm(float *mel, long long frames, void *scratch, cudaStream_t s) {
  const long long n = frames - 1;  // statistics over all frames but the last
  if (n < 2) return cudaErrorInvalidValue;
  const int chunks = int((n + FE_CHUNK - 1) / FE_CHUNK);
  double *part = static_cast<double *>(scratch);
  double *mean = part + (long long)chunks * FE_MELS, *inv = mean + FE_MELS;
  cudaError_t e;
  if ((e = launch_pdl(mel_sum_kernel, dim3(chunks), dim3(FE_MELS), 0, s, (const float *)mel, n,
                      (const double *)nullptr, part)) != cudaSuccess ||
      (e = launch_pdl(mel_stats_kernel, dim3(1), dim3(FE_MELS), 0, s, (const double *)part,
                      chunks, n, mean, 0)) != cudaSuccess ||
      (e = launch_pdl(mel_sum_kernel, dim3(chunks), dim3(FE_MELS), 0, s, (const float *)mel, n,
                      (const double *)mean, part)) != cudaSuccess ||
      (e = launch_pdl(mel_stats_kernel, dim3(1), dim3(FE_MELS), 0, s, (const double *)part,
                      chunks, n, inv, 1)) != cudaSuccess)
    return e;
  const long long total = frames * FE_MELS;
  return launch_pdl(mel_norm_kernel, dim3(unsigned((total + 255) / 256)), dim3(256), 0, s, mel,
                    frames, (const double *)mean, (const double *)inv);
}

}  // namespace wv

namespace wv {

cudaError_t launch_conv02(const float *mel, int valid, int t2, int ch, const float *w0,
                          const float *b0, const float *w2, const float *b2, __half *a,
                          cudaStream_t s) {
  const int t1 = (valid - 1) / 2 + 1, live = (t1 - 1) / 2 + 1;
  return launch_pdl(conv02_kernel, dim3(unsigned(t2)), dim3(ch < 256 ? ch : 256), 0, s, mel, valid,
                    t1, t2, live, ch, w0, b0, w2, b2, a);
}

cudaError_t launch_dw3s2(const float *x, int t, int f, int ch, int rows, const float *w,
                         const float *b, __half *y, cudaStream_t s) {
  const long long total = (long long)rows * ((f - 1) / 2 + 1) * ch;
  return launch_pdl(dw3s2_kernel, dim3(unsigned((total + 255) / 256)), dim3(256), 0, s, x, t, f, ch,
                    rows, w, b, y);
}

cudaError_t launch_flatten(const float *y, int t, int f, int ch, __half *h, cudaStream_t s) {
  const long long total = (long long)t * f * ch;
  return launch_pdl(flatten_kernel, dim3(unsigned((total + 255) / 256)), dim3(256), 0, s, y, t, f,
                    ch, h);
}

}  // namespace wv
