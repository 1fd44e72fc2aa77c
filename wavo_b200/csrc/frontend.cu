// The Parakeet log-mel frontend on the device (src/parakeet/frontend.rs, src/fft.rs): pre-emphasis
// in f64, a symmetric Hann(400) centred in an f64 FFT of 512, power cast to f32, the Slaney
// filterbank as f32 fused multiply-adds in bin order, ln(mel + 2^-24), then each mel bin normalised
// over all frames but the last, which is zero. The FFT performs the reference's operations in its
// order (radix-2 decimation in time, Stockham order, every multiply-add fused, the same cos/sin
// table), so the spectrum is the reference's bit for bit; the normalisation's statistics are f64
// sums of each bin's values and squares in a fixed order (a warp's frames in turn, a CTA's warps,
// the CTAs), its squared deviations Σx² − mean·Σx.
//
//   log_mel_kernel   a warp a frame at a time (16 warps, one CTA an SM, looping over frames): the
//                    tables copied once into shared memory, the frame's pcm staged from
//                    registers (the next frame's fetched during this one's FFT), the windowed
//                    frame in registers, 16 complex values a lane, the nine butterfly stages in
//                    three register phases with two exchanges through the warp's shared buffer,
//                    the power spectrum, four mel bins a lane.
//                    For the normalised features it also sums each bin's values and squares
//                    over the frames it takes (f64, in a fixed order: a warp's frames in turn,
//                    the CTA's warps in order).
//                    The last CTA to finish adds the CTAs' sums in order: the mean, then
//                    1 / (unbiased std + 1e-5).
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

constexpr int FE_WARPS = 12;  // one CTA an SM: 12 frames in flight (8 KB of buffer, 164 registers)

constexpr int FE_SPAN_MAX = 16;  // FFT bins in a mel bin's nonzero span (12 for the Slaney bank)
constexpr int FE_STAGE_P = FE_NFFT + 1;               // pcm samples a frame reads
constexpr int FE_PF = (FE_STAGE_P + 31) / 32;         // of them a lane's (17)
constexpr int FE_TWL = 23;                            // a lane's twiddles of stages 4..8

// The FFT in registers. Stage t of the reference's radix-2 Stockham FFT (output i from inputs 2i
// and 2i + 1, to positions i and i + 256) moves the element of label L from position rotr^t(L) to
// rotr^(t+1)(L) (9-bit rotations), pairing the labels that differ in bit t; label L starts at
// position L (the sample perm(L) = bitrev9(L)) and ends at frequency bin L. A lane holds 16 labels:
// stages 0-3 with label bits 0-3 in its registers (lane = bits 4-8), stages 4-7 with bits 4-7
// (lane = bits 0-3, 8), stage 8 with bits 0-2, 8 (lane = bits 3-7); the labels move between these
// layouts through the warp's shared buffer twice. Every butterfly has the reference's inputs,
// twiddle (idx = the label's low t bits · 2^(8-t)) and fused multiply-adds, so the spectrum is
// the same bit for bit.
//
// Shared tables of a CTA, built once on the host as one image in this layout: the 256 twiddles
// (cos, sin)(tau·idx/512); each lane's twiddles of stages 4-8 ([k][lane]: stage 4 one, 5 two, 6
// four, 7 eight, 8 eight); the window by sample index; the filterbank as each mel bin's nonzero
// span, weight k of bin m at fw[k][m] (a warp's lanes read consecutive words).
struct FeShared {
  double2 tw[256];
  double2 twl[FE_TWL][32];
  double win[FE_NFFT];
  float fw[FE_SPAN_MAX][FE_MELS];
  int lo[FE_MELS], len[FE_MELS];
};
static_assert(sizeof(FeShared) % 16 == 0, "the image is copied in 16-byte words");
constexpr size_t FE_BUF = FE_NFFT * sizeof(double2);  // a warp's buffer: the labels' exchange
// Then the warps' per-bin sums of the features and of their squares for the normalisation
// ([warp][2][128] f64).
constexpr size_t FE_ACC = size_t(FE_WARPS) * 2 * FE_MELS * 8;
constexpr size_t FE_SMEM = sizeof(FeShared) + size_t(FE_WARPS) * FE_BUF + FE_ACC;

// Where label L sits in the exchange buffer: its low three bits XOR a function of bits 3-7, so
// that every quarter-warp's eight 16-byte accesses of each layout fall in distinct bank groups.
__device__ __forceinline__ int fe_phys(int L) { return L ^ (((L >> 4) ^ (L >> 3)) & 7); }

// The butterfly of src/fft.rs:131-143: (a, b) at position 2i, (x, y) at 2i + 1, twiddle w; the
// results go to i (a, b) and i + 256 (x, y).
__device__ __forceinline__ void fe_bfly(double &a, double &b, double &x, double &y, double2 w) {
  const double c = w.x, s = w.y;
  const double r0 = fma(s, y, fma(c, x, a));
  const double i0 = fma(-s, x, fma(c, y, b));
  const double r1 = fma(-s, y, fma(-c, x, a));
  const double i1 = fma(s, x, fma(-c, y, b));
  a = r0;
  b = i0;
  x = r1;
  y = i1;
}

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
                   const FrontendTables tab, float *__restrict__ mel, int stat_frames,
                   double *__restrict__ part, double *__restrict__ stats) {
  // part != nullptr: also this CTA's per-bin f64 sums of the features of frames < stat_frames and
  // of their squares (part[blockIdx][0][m], part[blockIdx][1][m]), its warps added in order; the
  // last CTA to finish adds the CTAs' sums in order and writes each bin's mean (stats[m]) and
  // 1 / (sqrt(Σ(x − mean)² / (n − 1)) + 1e-5) (stats[128 + m]), Σ(x − mean)² = Σx² − mean·Σx.
  extern __shared__ __align__(16) double fe_smem[];
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
  double2 *xb = reinterpret_cast<double2 *>(reinterpret_cast<char *>(fe_smem) + sizeof(FeShared) +
                                            size_t(warp) * FE_BUF);
  float *stage = reinterpret_cast<float *>(xb);  // the frame's pcm, before the first exchange
  double *acc = reinterpret_cast<double *>(reinterpret_cast<char *>(fe_smem) + sizeof(FeShared) +
                                           size_t(FE_WARPS) * FE_BUF) +
                warp * 2 * FE_MELS;
#pragma unroll
  for (int q = 0; q < FE_MELS / 32; ++q) acc[lane + 32 * q] = acc[FE_MELS + lane + 32 * q] = 0.0;
  const int lrev = int(__brev(unsigned(lane)) >> 27);  // bitrev5(lane)
  const int step = int(gridDim.x) * FE_WARPS;
  int t = int(blockIdx.x) * FE_WARPS + warp;
  float pf[FE_PF];
  if (t < frames) fe_fetch(pcm, n_pcm, (f0 + t) * FE_HOP, lane, pf);
#pragma unroll 1
  for (; t < frames; t += step) {
    const long long j0 = (f0 + t) * FE_HOP;  // the frame's first padded index + 256
    // Stage the frame's pcm, then fetch the next frame's while this one is transformed.
#pragma unroll
    for (int q = 0; q < FE_PF; ++q) {
      const int p = lane + 32 * q;
      if (p < FE_STAGE_P) stage[p] = pf[q];
    }
    if (t + step < frames) fe_fetch(pcm, n_pcm, (f0 + t + step) * FE_HOP, lane, pf);
    __syncwarp();
    // Label lane·16 + r: position lane·16 + r holds sample bitrev4(r)·32 + bitrev5(lane),
    // pre-emphasised and windowed (src/fft.rs:89-92).
    double re[16], im[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const int rrev = ((r & 1) << 3) | ((r & 2) << 1) | ((r & 4) >> 1) | ((r & 8) >> 3);
      const int i = (rrev << 5) | lrev;
      const long long j = j0 + i - FE_NFFT / 2;  // the pcm index of padded sample j0 + i
      double s = 0.0;
      if (j == 0)
        s = double(stage[i + 1]);
      else if (j > 0 && j < n_pcm)
        s = __dsub_rn(double(stage[i + 1]), __dmul_rn(double(0.97f), double(stage[i])));
      re[r] = __dmul_rn(s, sh.win[i]);
      im[r] = 0.0;
    }
    // Stages 0-3: label bit t is register bit t; the twiddle is the same for every lane.
#pragma unroll
    for (int st = 0; st < 4; ++st)
#pragma unroll
      for (int r0 = 0; r0 < 16; ++r0) {
        if ((r0 >> st) & 1) continue;
        const int r1 = r0 | (1 << st);
        fe_bfly(re[r0], im[r0], re[r1], im[r1], sh.tw[(r0 & ((1 << st) - 1)) << (8 - st)]);
      }
    __syncwarp();  // the staged pcm is read before the buffer takes the labels
#pragma unroll
    for (int r = 0; r < 16; ++r) xb[fe_phys((lane << 4) | r)] = make_double2(re[r], im[r]);
    __syncwarp();
    // Stages 4-7: label bits 4-7 in the registers (each lane reads back the slots it writes).
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const double2 v = xb[fe_phys((lane & 15) | (r << 4) | ((lane >> 4) << 8))];
      re[r] = v.x;
      im[r] = v.y;
    }
#pragma unroll
    for (int st = 4; st < 8; ++st) {
      const int bit = st - 4, base = (1 << bit) - 1;  // stage st's first twl row
#pragma unroll
      for (int r0 = 0; r0 < 16; ++r0) {
        if ((r0 >> bit) & 1) continue;
        const int r1 = r0 | (1 << bit);
        fe_bfly(re[r0], im[r0], re[r1], im[r1], sh.twl[base + (r0 & ((1 << bit) - 1))][lane]);
      }
    }
#pragma unroll
    for (int r = 0; r < 16; ++r)
      xb[fe_phys((lane & 15) | (r << 4) | ((lane >> 4) << 8))] = make_double2(re[r], im[r]);
    __syncwarp();
    // Stage 8: label bits 0-2 and 8 in the registers.
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const double2 v = xb[fe_phys((r & 7) | (lane << 3) | ((r >> 3) << 8))];
      re[r] = v.x;
      im[r] = v.y;
    }
    __syncwarp();  // every label read before the power spectrum takes the buffer
#pragma unroll
    for (int r0 = 0; r0 < 8; ++r0) fe_bfly(re[r0], im[r0], re[r0 + 8], im[r0 + 8], sh.twl[15 + r0][lane]);
    // The power spectrum (f64 products and sum, cast to f32): bins lane·8 + r, and bin 256.
    float *power = reinterpret_cast<float *>(xb);
#pragma unroll
    for (int r = 0; r < 8; ++r)
      power[(lane << 3) | r] =
          float(__dadd_rn(__dmul_rn(re[r], re[r]), __dmul_rn(im[r], im[r])));
    if (lane == 0) power[256] = float(__dadd_rn(__dmul_rn(re[8], re[8]), __dmul_rn(im[8], im[8])));
    __syncwarp();
    float *out = mel + (long long)t * FE_MELS;
#pragma unroll
    for (int q = 0; q < FE_MELS / 32; ++q) {
      const int m = lane + 32 * q;
      const float *pw = power + sh.lo[m];
      float e = 0.0f;
      for (int k = 0; k < sh.len[m]; ++k) e = fmaf(sh.fw[k][m], pw[k], e);
      const float v = logf(__fadd_rn(e, 1.0f / float(1 << 24)));
      out[m] = v;
      if (t < stat_frames) {  // a lane's own bins: no other lane touches these words
        const double x = double(v);
        acc[m] = __dadd_rn(acc[m], x);
        acc[FE_MELS + m] = __dadd_rn(acc[FE_MELS + m], __dmul_rn(x, x));
      }
    }
    __syncwarp();  // power is read before the next frame stages its pcm
  }
  if (part == nullptr) return;  // uniform over the CTA
  __syncthreads();
  double *all = acc - warp * 2 * FE_MELS;
  for (int e = int(threadIdx.x); e < 2 * FE_MELS; e += blockDim.x) {
    double v = 0.0;
    for (int w = 0; w < FE_WARPS; ++w) v = __dadd_rn(v, all[w * 2 * FE_MELS + e]);
    part[(long long)blockIdx.x * 2 * FE_MELS + e] = v;
  }
  // The last CTA (no waiting: the others have published their sums before counting themselves).
  __threadfence();
  __syncthreads();
  __shared__ int is_last;
  if (threadIdx.x == 0) is_last = atomicAdd(tab.count, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // Thread (g, cp): columns 2cp, 2cp + 1 of the 256 (Σx of the bins, then Σx²) over CTAs
  // g·per .. (g + 1)·per − 1 in order, 16-byte loads sixteen CTAs at a time; then the G groups in
  // order.
  constexpr int G = 32 * FE_WARPS / FE_MELS;
  const int cp = int(threadIdx.x) % FE_MELS, g = int(threadIdx.x) / FE_MELS;
  const int ctas = int(gridDim.x), per = (ctas + G - 1) / G;
  const int c0 = g * per, c1 = min(c0 + per, ctas);
  double2 sum = make_double2(0.0, 0.0);
  constexpr int B = 16;
  for (int c = c0; c < c1; c += B) {
    double2 v[B];
#pragma unroll
    for (int j = 0; j < B; ++j)
      v[j] = __ldcg(reinterpret_cast<const double2 *>(part + (long long)min(c + j, c1 - 1) * 2 *
                                                                 FE_MELS) + cp);
#pragma unroll
    for (int j = 0; j < B; ++j)
      if (c + j < c1) sum = make_double2(__dadd_rn(sum.x, v[j].x), __dadd_rn(sum.y, v[j].y));
  }
  double2 *red = reinterpret_cast<double2 *>(all);  // [G][128] (the warps' sums are spent)
  red[g * FE_MELS + cp] = sum;
  __syncthreads();
  if (threadIdx.x < FE_MELS) {
    const int m = int(threadIdx.x);
    const double *r = reinterpret_cast<const double *>(red);  // [G][256]
    double sx = 0.0, sq = 0.0;
    for (int k = 0; k < G; ++k) {
      sx = __dadd_rn(sx, r[k * 2 * FE_MELS + m]);
      sq = __dadd_rn(sq, r[k * 2 * FE_MELS + FE_MELS + m]);
    }
    const long long n = stat_frames;
    const double mu = sx / double(n);
    const double ss = fmax(__dsub_rn(sq, __dmul_rn(mu, sx)), 0.0);
    stats[m] = mu;
    stats[FE_MELS + m] = 1.0 / __dadd_rn(sqrt(ss / double(n - 1)), double(1e-5f));
  }
  if (threadIdx.x == 0) atomicExch(tab.count, 0u);  // for the next launch
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

// Depthwise 3x3, stride 2, padding 1, + bias over x [t][f][ch] into y [rows][half(f)][ch]: a CTA
// an output row (blockIdx.x) and column (blockIdx.y), a thread a channel.
__global__ void dw3s2_kernel(const float *__restrict__ x, int t, int f, int ch,
                             const float *__restrict__ w, const float *__restrict__ b,
                             __half *__restrict__ y) {
  griddep_launch_dependents();
  griddep_wait();
  const int k = int(blockIdx.x), fo = int(blockIdx.y);
  __half *out = y + ((long long)k * gridDim.y + fo) * ch;
  for (int q = int(threadIdx.x); q < ch; q += blockDim.x) {
    // Every tap's operands loaded at once (a tap outside the image reads a clamped in-range
    // element and adds nothing), then the products added in tap order.
    float xv[9], wv[9];
#pragma unroll
    for (int tap = 0; tap < 9; ++tap) {
      const int ti = min(max(2 * k + tap / 3, 1), t), fi = min(max(2 * fo + tap % 3, 1), f);
      xv[tap] = x[((long long)(ti - 1) * f + fi - 1) * ch + q];
      wv[tap] = w[tap * ch + q];
    }
    float v = b[q];
#pragma unroll
    for (int tap = 0; tap < 9; ++tap) {
      const int ti = 2 * k + tap / 3, fi = 2 * fo + tap % 3;  // uniform over the CTA
      if (ti >= 1 && ti <= t && fi >= 1 && fi <= f) v = __fadd_rn(v, __fmul_rn(wv[tap], xv[tap]));
    }
    out[q] = __float2half_rn(v);  // the pointwise GEMM's operand (rounded to f16 there as well)
  }
}

// [t][16][ch] to [t][ch·16] (src/parakeet/cpu.rs:85-90): a CTA a row (blockIdx.x) and 256
// channels (blockIdx.y); thread c reads its 16 values (a warp's loads coalesced) and writes them as
// 32 contiguous bytes of the output GEMM's f16 operand.
constexpr int FL_F = 16;
__global__ void __launch_bounds__(256) flatten_kernel(const float *__restrict__ y, int ch,
                                                      __half *__restrict__ h) {
  griddep_launch_dependents();
  griddep_wait();
  const int c = int(blockIdx.y) * 256 + int(threadIdx.x);
  if (c >= ch) return;
  const long long row = (long long)blockIdx.x * FL_F * ch;
  __align__(16) __half o[FL_F];
#pragma unroll
  for (int j = 0; j < FL_F; ++j) o[j] = __float2half_rn(y[row + (long long)j * ch + c]);
  uint4 *d = reinterpret_cast<uint4 *>(h + row + (long long)c * FL_F);
  d[0] = reinterpret_cast<const uint4 *>(o)[0];
  d[1] = reinterpret_cast<const uint4 *>(o)[1];
}

}  // namespace

// ---- tables (host), as src/fft.rs:46-66 and src/parakeet/frontend.rs:30-47, 110-140 build them --

size_t frontend_table_bytes() { return sizeof(FeShared) + 256; }  // the image, then a counter

cudaError_t frontend_tables_upload(void *dev, cudaStream_t s, FrontendTables *out) {
  // The first stage's order (src/fft.rs: all 512 points radix-2 blocks, the even samples before
  // the odd ones at every level) is the 9-bit reversal, which the kernel computes.
  const int n = FE_NFFT;
  std::unique_ptr<FeShared> owner(new FeShared());  // the image (29 KB), zero-filled
  FeShared &img = *owner;
  // The twiddles: stage t's butterfly on label L0 (bit t clear) takes cos/sin(tau·idx/512) at
  // idx = (L0 mod 2^t)·2^(8-t), the reference's i / (512 / size) · (512 / size).
  const double tau = 6.283185307179586;
  for (int idx = 0; idx < n / 2; ++idx) {
    const double phase = tau * double(idx) / double(n);
    img.tw[idx] = make_double2(std::cos(phase), std::sin(phase));
  }
  auto tw_of = [&](int t, int L0) { return img.tw[(L0 & ((1 << t) - 1)) << (8 - t)]; };
  for (int l = 0; l < 32; ++l) {
    for (int t = 4; t < 8; ++t)  // labels (l mod 16) | r·16 | (l / 16)·256: r's low t-4 bits
      for (int rl = 0; rl < (1 << (t - 4)); ++rl)
        img.twl[(1 << (t - 4)) - 1 + rl][l] = tw_of(t, (l & 15) | (rl << 4));
    for (int r0 = 0; r0 < 8; ++r0)  // labels r0 | l·8 (| 256)
      img.twl[15 + r0][l] = tw_of(8, r0 | (l << 3));
  }
  for (int i = 0; i < n; ++i) {  // the window by sample index
    const int k = i - (FE_NFFT - FE_WINDOW) / 2;
    img.win[i] = k >= 0 && k < FE_WINDOW
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
  unsigned *count = reinterpret_cast<unsigned *>(static_cast<uint8_t *>(dev) + sizeof(FeShared));
  if (e == cudaSuccess) e = cudaMemsetAsync(count, 0, sizeof(unsigned), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);  // before the host image is freed
  out->image = dev;
  out->count = count;
  return e;
}

namespace {
int log_mel_ctas(int frames, cudaError_t *err) {
  // One CTA an SM at most, each warp looping over frames (the tables load once a CTA).
  static bool configured[64] = {};
  static int sms[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  *err = cudaSuccess;
  if (dev >= 64) {
    *err = cudaErrorInvalidDevice;
    return 0;
  }
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(log_mel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(FE_SMEM));
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) {
      *err = e;
      return 0;
    }
    configured[dev] = true;
  }
  const int ctas = (frames + FE_WARPS - 1) / FE_WARPS;
  return ctas < sms[dev] ? ctas : sms[dev];
}
}  // namespace

cudaError_t launch_log_mel(const float *pcm, long long n_pcm, long long f0, int frames,
                           const FrontendTables &tab, float *mel, cudaStream_t s) {
  if (frames <= 0) return cudaSuccess;
  cudaError_t e;
  const int ctas = log_mel_ctas(frames, &e);
  if (e != cudaSuccess) return e;
  return launch_pdl(log_mel_kernel, dim3(ctas), dim3(32 * FE_WARPS), FE_SMEM, s, pcm, n_pcm, f0,
                    frames, tab, mel, 0, (double *)nullptr, (double *)nullptr);
}

size_t mel_features_scratch_bytes(int sms) { return (size_t(sms) * 2 + 2) * FE_MELS * 8; }

cudaError_t launch_mel_features(const float *pcm, long long n_pcm, int frames,
                                const FrontendTables &tab, float *mel, void *scratch, int sms,
                                cudaStream_t s) {
  const long long n = frames - 1;  // statistics over all frames but the last
  if (n < 2) return cudaErrorInvalidValue;
  cudaError_t e;
  const int ctas = log_mel_ctas(frames, &e);
  if (e != cudaSuccess) return e;
  if (ctas > sms) return cudaErrorInvalidValue;  // the scratch holds sms CTAs' sums
  double *part = static_cast<double *>(scratch);
  double *mean = part + (long long)sms * 2 * FE_MELS, *inv = mean + FE_MELS;
  if ((e = launch_pdl(log_mel_kernel, dim3(ctas), dim3(32 * FE_WARPS), FE_SMEM, s, pcm, n_pcm,
                      0LL, frames, tab, mel, int(n), part, mean)) != cudaSuccess)
    return e;
  const long long total = (long long)frames * FE_MELS;
  return launch_pdl(mel_norm_kernel, dim3(unsigned((total + 255) / 256)), dim3(256), 0, s, mel,
                    (long long)frames, (const double *)mean, (const double *)inv);
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
  const int fo_n = (f - 1) / 2 + 1;
  if (rows <= 0) return cudaSuccess;
  if (fo_n > 65535) return cudaErrorInvalidValue;
  return launch_pdl(dw3s2_kernel, dim3(unsigned(rows), unsigned(fo_n)), dim3(ch < 256 ? ch : 256),
                    0, s, x, t, f, ch, w, b, y);
}

cudaError_t launch_flatten(const float *y, int t, int f, int ch, __half *h, cudaStream_t s) {
  if (t <= 0) return cudaSuccess;
  if (f != FL_F || ch % 32 != 0) return cudaErrorInvalidValue;
  return launch_pdl(flatten_kernel, dim3(unsigned(t), unsigned((ch + 255) / 256)), dim3(256), 0, s,
                    y, ch, h);
}

}  // namespace wv
