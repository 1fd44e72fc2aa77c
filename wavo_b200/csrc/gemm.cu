// Projection GEMM for sm_100a: c = epilogue(a · W^T + bias), the reference's `Pass::gemm`
// (src/gpu/mod.rs:1394-1425, gemm.wgsl:167-242) re-designed for the 5th-generation tensor cores.
//
// a [m][k] f16 and W [n][k] f16 are streamed by TMA into 128-byte-swizzled shared-memory stages;
// one thread issues tcgen05.mma (M=128, N=BN, K=16, f32 accumulators in TMEM); four epilogue warps
// read the accumulators back with tcgen05.ld (one row per thread), add the bias, apply the epilogue
// (a compile-time mode) and store the row. The kernel is persistent (one CTA per SM walks the output
// tiles) and keeps two accumulators in TMEM, so the epilogue of one tile overlaps the MMAs of the
// next. The tile width BN (128, 160 or 256) is chosen per shape to even out the last wave of tiles.
//
// Numerics match the reference GPU GEMM: a and W rounded to f16 (round to nearest even), products
// exact, sums in f32. Dual outputs (a bias longer than the rows) write the first `dual` outputs a
// second time at columns cols.. with their own bias and no epilogue, as src/gpu/mod.rs:758-834.
#include "kernels.cuh"
#include "ptx.cuh"

namespace wv {
namespace {

constexpr int BM = kGemmBM, BK = kGemmBK;

// KC: 64-column K chunks per pipeline stage. With KC = 2 each operand tile of a stage is one 3D
// TMA box of two chunks: a TMA instruction costs an SM a fixed ~250 cycles besides its bytes, so
// fewer, larger boxes keep the loads ahead of the UMMAs.
template <int BN, int KC = 1>
struct GemmCfg {
  static constexpr int A_BYTES = BM * BK * 2 * KC;
  static constexpr int B_BYTES = BN * BK * 2 * KC;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (216 * 1024) / STAGE_BYTES > 6 ? 6 : (216 * 1024) / STAGE_BYTES;
  // Two accumulators of BN columns; tcgen05.alloc takes a power of two.
  static constexpr int TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
  static_assert(BN % 32 == 0 && STAGE_BYTES % 1024 == 0, "tile shape");
  static constexpr uint32_t IDESC = idesc_f16(BM, BN, 0);
};

struct __align__(8) GemmBarriers {
  uint64_t full[6];
  uint64_t empty[6];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t abort;
};

__device__ __forceinline__ float gelu_f(float x) {
  // Abramowitz–Stegun 7.1.26 erf, as the reference's gelu (src/cpu/ops.rs:33-40).
  float z = fabsf(0.70710678118654752f * x);
  float t = 1.0f / (1.0f + 0.3275911f * z);
  float p = (((1.0614054f * t - 1.453152f) * t + 1.4214138f) * t - 0.28449674f) * t + 0.2548296f;
  float s = signbit(x) ? -1.0f : 1.0f;
  return 0.5f * x * (1.0f + s * (1.0f - p * t * __expf(-z * z)));
}

template <int E>
__device__ __forceinline__ float epi(float v, float c, float alpha) {
  if (E == kBias) return v;
  // SiLU with the hardware exponential and reciprocal: the epilogue of a wide GEMM (FFN, N = 4d)
  // runs one per output, and the accurate forms cost it more issue slots than the UMMAs take.
  if (E == kSilu) return __fdividef(v, 1.0f + __expf(-v));
  if (E == kRelu) return fmaxf(v, 0.0f);
  if (E == kResidual) return c + alpha * v;
  if (E == kGelu) return gelu_f(v);
  if (E == kGeluResidual) return c + gelu_f(v);
  return tanhf(fminf(fmaxf(v, -10.0f), 10.0f));
}

// Stores 32 consecutive outputs of one row (columns col0.. of `c`), reading c first for the
// residual epilogues. `lim` is the number of valid columns (<= 32); b holds the 32 biases.
template <int E>
__device__ __forceinline__ void store_row32(const GemmArgs &g, long long row, int col0, int lim,
                                            const float (&v)[32], const float (&b)[32]) {
  constexpr bool resid = (E == kResidual || E == kGeluResidual);
  if (g.c_f16) {
    __half *c = reinterpret_cast<__half *>(g.c) + row * g.ldc + col0;
    if (lim == 32 && ((reinterpret_cast<uintptr_t>(c) & 15u) == 0)) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 old = make_uint4(0, 0, 0, 0);
        if (resid) old = *reinterpret_cast<const uint4 *>(c + 8 * q);
        const __half *oh = reinterpret_cast<const __half *>(&old);
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int j = 8 * q + 2 * i;
          w[i] = pack_half2(epi<E>(v[j] + b[j], __half2float(oh[2 * i]), g.alpha),
                            epi<E>(v[j + 1] + b[j + 1], __half2float(oh[2 * i + 1]), g.alpha));
        }
        *reinterpret_cast<uint4 *>(c + 8 * q) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < lim) {
          const float old = resid ? __half2float(c[j]) : 0.0f;
          c[j] = __float2half_rn(epi<E>(v[j] + b[j], old, g.alpha));
        }
    }
  } else {
    float *c = reinterpret_cast<float *>(g.c) + row * g.ldc + col0;
    if (lim == 32 && ((reinterpret_cast<uintptr_t>(c) & 15u) == 0)) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 old = make_float4(0, 0, 0, 0);
        if (resid) old = *reinterpret_cast<const float4 *>(c + 4 * q);
        float4 o;
        o.x = epi<E>(v[4 * q + 0] + b[4 * q + 0], old.x, g.alpha);
        o.y = epi<E>(v[4 * q + 1] + b[4 * q + 1], old.y, g.alpha);
        o.z = epi<E>(v[4 * q + 2] + b[4 * q + 2], old.z, g.alpha);
        o.w = epi<E>(v[4 * q + 3] + b[4 * q + 3], old.w, g.alpha);
        *reinterpret_cast<float4 *>(c + 4 * q) = o;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < lim) {
          const float old = resid ? c[j] : 0.0f;
          c[j] = epi<E>(v[j] + b[j], old, g.alpha);
        }
    }
  }
}

// 32 biases from `bias` (16-byte aligned when `vec`), zeros past `lim`.
__device__ __forceinline__ void load_bias32(const float *bias, int lim, float (&b)[32]) {
  if (lim == 32 && ((reinterpret_cast<uintptr_t>(bias) & 15u) == 0)) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 t = __ldg(reinterpret_cast<const float4 *>(bias) + q);
      b[4 * q] = t.x;
      b[4 * q + 1] = t.y;
      b[4 * q + 2] = t.z;
      b[4 * q + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) b[j] = j < lim ? __ldg(bias + j) : 0.0f;
  }
}

template <int BN, int E, int KC>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_w,
                const GemmArgs g) {
  using C = GemmCfg<BN, KC>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  GemmBarriers *bar = reinterpret_cast<GemmBarriers *>(smem + STAGES * C::STAGE_BYTES);
  const uint32_t warp = warp_id(), lane = lane_id();

  const int num_m = (g.m + BM - 1) / BM;
  const int num_n = (g.cols + BN - 1) / BN;
  const int tiles = num_m * num_n;
  const int kblocks = (g.k + BK * KC - 1) / (BK * KC);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bar->full[s], 1);
      mbar_init(&bar->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar->acc_full[b], 1);
      mbar_init(&bar->acc_empty[b], 4);
    }
    mbar_init(&bar->drain, 1);
    bar->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tma_a);
    prefetch_tmap(&tma_w);
  }
  if (warp == 1) {
    tmem_alloc(&bar->tmem_base, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  const Abort ab{&bar->abort, g.err};
  griddep_launch_dependents();
  griddep_wait();  // the previous kernel of the stream has completed (programmatic launch)

  if (warp == 0) {
    // ---- TMA producer --------------------------------------------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0;  // stages armed at least once
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / num_n) * BM, n0 = (tile % num_n) * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&bar->empty[stage], phase ^ 1u, ab, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t *sa = smem + stage * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&bar->full[stage], C::STAGE_BYTES);
          if constexpr (KC == 1) {
            tma_load_2d(sa, &tma_a, &bar->full[stage], kb * BK, m0);
            tma_load_2d(sa + C::A_BYTES, &tma_w, &bar->full[stage], kb * BK, n0);
          } else {
            tma_load_3d(sa, &tma_a, &bar->full[stage], 0, m0, kb * KC);
            tma_load_3d(sa + C::A_BYTES, &tma_w, &bar->full[stage], 0, n0, kb * KC);
          }
          armed |= 1u << stage;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let every load this thread issued land before the CTA can exit: the last arm of each
        // stage is the one before `stage` in ring order.
        for (int s = 0; s < STAGES; ++s) {
          if (!(armed & (1u << s))) continue;
          const uint32_t par = (s < stage) ? phase : (phase ^ 1u);
          const long long t0 = clock64();
          while (!mbar_try_wait(&bar->full[s], par) && clock64() - t0 < kWaitCycles) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----------------------------------------------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued = false;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&bar->acc_empty[acc], acc_phase ^ 1u, ab, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&bar->full[stage], phase, ab, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sb = sa + C::A_BYTES;
          // Chunk c of a stage: BM (a) or BN (W) rows of 128 bytes.
#pragma unroll
          for (int ks = 0; ks < KC * BK / 16; ++ks) {
            const uint32_t oa = (ks >> 2) * BM * 128 + (ks & 3) * 32;
            const uint32_t ob = (ks >> 2) * BN * 128 + (ks & 3) * 32;
            umma_f16(d, sdesc_sw128(sa + oa, 16, 1024), sdesc_sw128(sb + ob, 16, 1024), C::IDESC,
                     (kb | ks) != 0);
          }
          issued = true;
          umma_commit(&bar->empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&bar->acc_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued) {
        umma_commit(&bar->drain);
        const long long t0 = clock64();
        while (!mbar_try_wait(&bar->drain, 0) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else {
    // ---- epilogue: warps 2..5, one accumulator row per thread -----------------------------
    const uint32_t quarter = warp & 3u;  // TMEM lanes this warp may access
    const int row_in_tile = int(quarter * 32 + lane);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      const int m0 = (tile / num_n) * BM, n0 = (tile % num_n) * BN;
      if (!mbar_wait_warp(&bar->acc_full[acc], acc_phase, ab, kErrTimeoutConsumer)) break;
      tc_fence_after();
      const long long row = m0 + row_in_tile;
      const bool row_ok = row < g.m;
#pragma unroll 1
      for (int chunk = 0; chunk < BN / 32; ++chunk) {
        const int col0 = n0 + chunk * 32;
        if (col0 >= g.cols) break;
        uint32_t r[32];
        tmem_ld32(tmem + ((quarter * 32u) << 16) + uint32_t(acc * BN + chunk * 32), r);
        const int lim = min(32, g.cols - col0);
        float b[32];
        load_bias32(g.bias + col0, lim, b);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (row_ok) store_row32<E>(g, row, col0, lim, v, b);
        if (col0 < g.dual) {
          const int lim2 = min(lim, g.dual - col0);
          load_bias32(g.bias + g.cols + col0, lim2, b);
          if (row_ok) store_row32<kBias>(g, row, g.cols + col0, lim2, v, b);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->acc_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ---- Q8_0 GEMM: W dequantised in the prologue -------------------------------------------------
//
// The reference's GPU GEMM reads Q8_0 blocks (int8 values, one f16 scale per 32) and dequantises
// them as it stages each K-step (src/gpu/gemm.wgsl:105-130, WTYPE = Q8_0). Here the int8 values of
// a 64-column K-step stream by TMA into a raw staging area of the stage (64 bytes a row, no
// swizzle); four converter warps turn them into the f16 W tile the UMMA reads (the canonical
// 128-byte-swizzled K-major layout), q·d rounded to f16 exactly as the load-time dequantisation
// (an f16 multiply of an exact integer and an exact scale is the correctly rounded product), so the
// results are bit-identical to the f16-weight GEMM. W moves through HBM and L2 at one byte per
// weight plus 2 bytes of scale per 32; the f16 tile never exists in global memory.
//   warp 0      TMA: a (f16, swizzled), the int8 block values of W and their two rows of scales
//               (a transposed f16 copy [k / 32][n] made at load, so that a K-step's scales are one
//               box)
//   warp 1      one thread issues the UMMAs of a stage once the converters finished its W tile
//   warps 2-5   epilogue (as gemm_kernel)
//   warps 6-13  converters: thread t converts 16-byte chunks (8 values) c = t % 8 of rows t / 8 +
//               32 i; a warp reads 256 contiguous staging bytes and writes four whole 128-byte rows
//               of the swizzled tile (no bank conflicts either way)
constexpr int kQ8ConvWarps = 8;
constexpr int kQ8Threads = 32 * (6 + kQ8ConvWarps);

template <int BN>
struct GemmQ8Cfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;  // the converted f16 tile
  static constexpr int Q_BYTES = BN * BK;      // int8 staging
  static constexpr int S_BYTES = 2 * BN * 2;   // the K-step's two scale rows (f16)
  static constexpr int STAGE_BYTES = (A_BYTES + B_BYTES + Q_BYTES + S_BYTES + 1023) / 1024 * 1024;
  static constexpr int STAGES = (208 * 1024) / STAGE_BYTES > 6 ? 6 : (208 * 1024) / STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
  static_assert(BN % 32 == 0 && STAGE_BYTES % 1024 == 0 && Q_BYTES % 1024 == 0, "tile shape");
  static constexpr uint32_t IDESC = idesc_f16(BM, BN, 0);
};

struct __align__(8) GemmQ8Barriers {
  uint64_t full[6];     // a and the int8 values landed (TMA)
  uint64_t conv[6];     // the f16 W tile is written (four converter warps)
  uint64_t empty[6];    // the stage's UMMAs completed
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t abort;
};

// Two f16 values of signed bytes b0, b1 of x: 0x6400 | (b ^ 0x80) is the f16 1024 + (b + 128),
// exact; subtracting 1152 leaves b.
__device__ __forceinline__ __half2 i8x2_to_h2(uint32_t x, uint32_t sel) {
  const uint32_t v = __byte_perm(x ^ 0x80808080u, 0x64646464u, sel);
  return __hsub2(*reinterpret_cast<const __half2 *>(&v), __float2half2_rn(1152.0f));
}

template <int BN, int E>
__global__ void __launch_bounds__(kQ8Threads, 1)
    gemm_q8_kernel(const __grid_constant__ CUtensorMap tma_a,
                   const __grid_constant__ CUtensorMap tma_q,
                   const __grid_constant__ CUtensorMap tma_s, const GemmArgs g) {
  using C = GemmQ8Cfg<BN>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  GemmQ8Barriers *bar = reinterpret_cast<GemmQ8Barriers *>(smem + STAGES * C::STAGE_BYTES);
  const uint32_t warp = warp_id(), lane = lane_id();

  const int num_m = (g.m + BM - 1) / BM;
  const int num_n = (g.cols + BN - 1) / BN;
  const int tiles = num_m * num_n;
  const int kblocks = (g.k + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bar->full[s], 1);
      mbar_init(&bar->conv[s], kQ8ConvWarps);
      mbar_init(&bar->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar->acc_full[b], 1);
      mbar_init(&bar->acc_empty[b], 4);
    }
    mbar_init(&bar->drain, 1);
    bar->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tma_a);
    prefetch_tmap(&tma_q);
    prefetch_tmap(&tma_s);
  }
  if (warp == 1) {
    tmem_alloc(&bar->tmem_base, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  const Abort ab{&bar->abort, g.err};
  griddep_launch_dependents();
  griddep_wait();  // the previous kernel of the stream has completed (programmatic launch)

  if (warp == 0) {
    // ---- TMA producer --------------------------------------------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / num_n) * BM, n0 = (tile % num_n) * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&bar->empty[stage], phase ^ 1u, ab, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t *sa = smem + stage * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&bar->full[stage], C::A_BYTES + C::Q_BYTES + C::S_BYTES);
          tma_load_2d(sa, &tma_a, &bar->full[stage], kb * BK, m0);
          tma_load_2d(sa + C::A_BYTES + C::B_BYTES, &tma_q, &bar->full[stage], kb * BK, n0);
          // Scale rows 2 kb, 2 kb + 1 (k % 64 == 32: the second is the TMA's zero fill).
          tma_load_2d(sa + C::A_BYTES + C::B_BYTES + C::Q_BYTES, &tma_s, &bar->full[stage], n0,
                      2 * kb);
          armed |= 1u << stage;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        for (int s = 0; s < STAGES; ++s) {
          if (!(armed & (1u << s))) continue;
          const uint32_t par = (s < stage) ? phase : (phase ^ 1u);
          const long long t0 = clock64();
          while (!mbar_try_wait(&bar->full[s], par) && clock64() - t0 < kWaitCycles) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----------------------------------------------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued = false;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&bar->acc_empty[acc], acc_phase ^ 1u, ab, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          // The converters waited for the stage's loads: their arrival covers a as well.
          if (!mbar_wait(&bar->conv[stage], phase, ab, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks)
            umma_f16(d, sdesc_sw128(sa + ks * 32, 16, 1024), sdesc_sw128(sb + ks * 32, 16, 1024),
                     C::IDESC, (kb | ks) != 0);
          issued = true;
          umma_commit(&bar->empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&bar->acc_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued) {
        umma_commit(&bar->drain);
        const long long t0 = clock64();
        while (!mbar_try_wait(&bar->drain, 0) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else if (warp < 6) {
    // ---- epilogue: warps 2..5, one accumulator row per thread -----------------------------
    const uint32_t quarter = warp & 3u;
    const int row_in_tile = int(quarter * 32 + lane);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      const int m0 = (tile / num_n) * BM, n0 = (tile % num_n) * BN;
      if (!mbar_wait_warp(&bar->acc_full[acc], acc_phase, ab, kErrTimeoutConsumer)) break;
      tc_fence_after();
      const long long row = m0 + row_in_tile;
      const bool row_ok = row < g.m;
#pragma unroll 1
      for (int chunk = 0; chunk < BN / 32; ++chunk) {
        const int col0 = n0 + chunk * 32;
        if (col0 >= g.cols) break;
        uint32_t r[32];
        tmem_ld32(tmem + ((quarter * 32u) << 16) + uint32_t(acc * BN + chunk * 32), r);
        const int lim = min(32, g.cols - col0);
        float b[32];
        load_bias32(g.bias + col0, lim, b);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (row_ok) store_row32<E>(g, row, col0, lim, v, b);
        if (col0 < g.dual) {
          const int lim2 = min(lim, g.dual - col0);
          load_bias32(g.bias + g.cols + col0, lim2, b);
          if (row_ok) store_row32<kBias>(g, row, g.cols + col0, lim2, v, b);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->acc_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  } else {
    // ---- converters: warps 6..13 -----------------------------------------------------------
    const int t = int(threadIdx.x) - 6 * 32;  // 0..255
    const int c = t & 7;                      // 16-byte chunk of a 128-byte row (8 values)
    int stage = 0;
    uint32_t phase = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      const int n0 = (tile % num_n) * BN;
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait_warp(&bar->full[stage], phase, ab, kErrTimeoutConsumer)) {
          ok = false;
          break;
        }
        uint8_t *sb = smem + stage * C::STAGE_BYTES + C::A_BYTES;
        const uint8_t *sq = sb + C::B_BYTES;
        // Chunk c's scale: Q8 block 2 kb + c / 4 of the row, scale row c / 4 of the stage.
        const __half *ss = reinterpret_cast<const __half *>(sq + C::Q_BYTES) + (c >> 2) * BN;
#pragma unroll
        for (int r = t >> 3; r < BN; r += 32) {
          const __half2 d2 = __half2half2(ss[r]);
          const uint2 q = *reinterpret_cast<const uint2 *>(sq + r * BK + c * 8);
          const __half2 h0 = __hmul2(i8x2_to_h2(q.x, 0x4140u), d2);
          const __half2 h1 = __hmul2(i8x2_to_h2(q.x, 0x4342u), d2);
          const __half2 h2 = __hmul2(i8x2_to_h2(q.y, 0x4140u), d2);
          const __half2 h3 = __hmul2(i8x2_to_h2(q.y, 0x4342u), d2);
          uint4 o;
          o.x = *reinterpret_cast<const uint32_t *>(&h0);
          o.y = *reinterpret_cast<const uint32_t *>(&h1);
          o.z = *reinterpret_cast<const uint32_t *>(&h2);
          o.w = *reinterpret_cast<const uint32_t *>(&h3);
          // 128-byte swizzle: chunk c of row r at chunk c ^ (r % 8) of its 128-byte line.
          *reinterpret_cast<uint4 *>(sb + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)) = o;
        }
        fence_proxy_async_smem();  // the generic-proxy writes are visible to the UMMA
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->conv[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ---- pair GEMM: one tile of 256 rows x BN columns on a cluster of two CTAs ---------------------
//
// A single SM streams its operand tiles at about 80 bytes per cycle through TMA, so a 128 x 128
// tile (32 KB per 64-deep k-block for 260 cycles of UMMAs) waits on its loads. A CTA pair shares
// one UMMA of M=256: each CTA loads its 128 rows of a and half of the tile's W rows, so a k-block
// costs each SM 16 KB + BN/2·128 bytes for 128·BN·64 multiply-adds, and the tensor core, not TMA,
// sets the pace. The leader CTA (rank 0) issues the UMMAs for both; each CTA's epilogue reads its
// own 128 accumulator rows from its own TMEM.

template <int BN, int KC = 1>
struct Gemm2Cfg {
  static constexpr int BNH = BN / 2;  // W rows per CTA
  static constexpr int A_BYTES = BM * BK * 2 * KC;
  static constexpr int B_BYTES = BNH * BK * 2 * KC;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STG_BYTES = 8 * 4096;  // epilogue staging: 2 buffers of 32 rows per warp
  static constexpr int STAGES = (200 * 1024 - STG_BYTES) / STAGE_BYTES > 8
                                    ? 8
                                    : (200 * 1024 - STG_BYTES) / STAGE_BYTES;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + STG_BYTES;  // + barriers
  static constexpr int TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
  static_assert(BN % 32 == 0 && BNH % 16 == 0 && STAGE_BYTES % 1024 == 0, "pair tile shape");
  static constexpr uint32_t IDESC = idesc_f16(2 * BM, BN, 0);
};

struct __align__(8) Gemm2Barriers {
  uint64_t full[8];       // leader: both CTAs' loads of a stage landed
  uint64_t empty[8];      // each CTA: the pair UMMAs reading its stage finished
  uint64_t acc_full[2];   // each CTA: an accumulator is complete
  uint64_t acc_empty[2];  // leader: both CTAs' epilogues have read an accumulator
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t abort;
};

template <int BN, int E, int KC>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tma_a,
                 const __grid_constant__ CUtensorMap tma_w,
                 const __grid_constant__ CUtensorMap tma_c, const GemmArgs g) {
  using C = Gemm2Cfg<BN, KC>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint8_t *stg = smem + STAGES * C::STAGE_BYTES;
  Gemm2Barriers *bar = reinterpret_cast<Gemm2Barriers *>(stg + C::STG_BYTES);
  const uint32_t warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  const int num_m = (g.m + 2 * BM - 1) / (2 * BM);
  const int num_n = (g.cols + BN - 1) / BN;
  const int tiles = num_m * num_n;
  const int kblocks = (g.k + BK * KC - 1) / (BK * KC);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bar->full[s], 1);
      mbar_init(&bar->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar->acc_full[b], 1);
      mbar_init(&bar->acc_empty[b], 8);  // 4 epilogue warps in each CTA
    }
    mbar_init(&bar->drain, 1);
    bar->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tma_a);
    prefetch_tmap(&tma_w);
    if (g.c_tma) prefetch_tmap(&tma_c);
  }
  // Both CTAs' barriers exist before either CTA signals one of the other's.
  cluster_sync();
  if (warp == 1) {
    tmem_alloc_pair(&bar->tmem_base, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  const Abort ab{&bar->abort, g.err};
  griddep_launch_dependents();
  griddep_wait();  // the previous kernel of the stream has completed (programmatic launch)

  if (warp == 0) {
    // ---- TMA producer (both CTAs): this CTA's rows of a and half of the W rows ---------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0;
      bool ok = true;
      for (int tile = pair; tile < tiles && ok; tile += npairs) {
        const int m0 = (tile / num_n) * (2 * BM) + int(rank) * BM;
        const int n0 = (tile % num_n) * BN + int(rank) * C::BNH;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&bar->empty[stage], phase ^ 1u, ab, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t *sa = smem + stage * C::STAGE_BYTES;
          const uint32_t full = mapa_shared(&bar->full[stage], 0);
          if (leader) mbar_arrive_expect_tx(&bar->full[stage], 2 * C::STAGE_BYTES);
          if constexpr (KC == 1) {
            tma_load_2d_pair(sa, &tma_a, full, kb * BK, m0);
            tma_load_2d_pair(sa + C::A_BYTES, &tma_w, full, kb * BK, n0);
          } else {
            tma_load_3d_pair(sa, &tma_a, full, 0, m0, kb * KC);
            tma_load_3d_pair(sa + C::A_BYTES, &tma_w, full, 0, n0, kb * KC);
          }
          armed |= 1u << stage;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && leader) {
        // Let the loads of every armed stage land (both CTAs' bytes count on these barriers).
        for (int s = 0; s < STAGES; ++s) {
          if (!(armed & (1u << s))) continue;
          const uint32_t par = (s < stage) ? phase : (phase ^ 1u);
          const long long t0 = clock64();
          while (!mbar_try_wait(&bar->full[s], par) && clock64() - t0 < kWaitCycles) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---- UMMA issuer (leader only) -------------------------------------------------------------
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued = false;
      const uint64_t d0 = sdesc_sw128(smem_u32(smem), 16, 1024);
      for (int tile = pair; tile < tiles && ok; tile += npairs) {
        if (!mbar_wait(&bar->acc_empty[acc], acc_phase ^ 1u, ab, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&bar->full[stage], phase, ab, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // Descriptors are linear in the start address (bits 0-13 hold address / 16).
          const uint64_t da = d0 + uint64_t((stage * C::STAGE_BYTES) >> 4);
          const uint64_t db = da + uint64_t(C::A_BYTES >> 4);
#pragma unroll
          for (int ks = 0; ks < KC * BK / 16; ++ks)
            umma_f16_pair(d, da + uint64_t(((ks >> 2) * BM * 128 + (ks & 3) * 32) >> 4),
                          db + uint64_t(((ks >> 2) * C::BNH * 128 + (ks & 3) * 32) >> 4),
                          C::IDESC, (kb | ks) != 0);
          issued = true;
          umma_commit_pair(&bar->empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&bar->acc_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued) {
        umma_commit_pair(&bar->drain);
        const long long t0 = clock64();
        while (!mbar_try_wait(&bar->drain, 0) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else {
    // ---- epilogue (both CTAs): warps 2..5, one accumulator row per thread ---------------------
    const uint32_t quarter = warp & 3u;
    const int row_in_tile = int(rank) * BM + int(quarter * 32 + lane);
    int acc = 0;
    uint32_t acc_phase = 0;
    if (g.c_tma) {
      // Each warp stages 32 rows x 32 columns in shared memory (one row per thread, in the tensor
      // map's swizzle, so the 32 threads' 16-byte writes spread over the banks) and one lane
      // stores the box with TMA, coalesced and asynchronous; an epilogue that adds into c
      // (residual) issues a TMA reduce-add instead, so c is never read into the SM.
      constexpr bool resid = (E == kResidual || E == kGeluResidual);
      uint8_t *sbuf = stg + (warp - 2) * 2 * 4096;
      const int row_box = int(rank) * BM + int(quarter * 32);
      int nbuf = 0;
      // 32 values of this thread's row into the next staging buffer, then one lane stores (or
      // reduce-adds) the warp's 32 x 32 box at column col, row row.
      auto stage_store = [&](const float (&v)[32], int col, int row, bool reduce) {
        uint8_t *buf = sbuf + nbuf * 4096;
        if (lane == 0) bulk_wait_read<1>();  // the store that used this buffer has read it
        __syncwarp();
        if (g.c_f16) {
          // 64-byte rows, 64-byte swizzle: 16-byte chunk c of row r at chunk c ^ ((r / 2) % 4).
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 q = make_uint4(pack_half2(v[8 * c], v[8 * c + 1]),
                                       pack_half2(v[8 * c + 2], v[8 * c + 3]),
                                       pack_half2(v[8 * c + 4], v[8 * c + 5]),
                                       pack_half2(v[8 * c + 6], v[8 * c + 7]));
            *reinterpret_cast<uint4 *>(buf + lane * 64 + ((c ^ ((lane >> 1) & 3)) * 16)) = q;
          }
        } else {
          // 128-byte rows, 128-byte swizzle: 16-byte chunk c of row r at chunk c ^ (r % 8).
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<float4 *>(buf + lane * 128 + ((c ^ (lane & 7)) * 16)) =
                make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (reduce) {
            tma_reduce_add_2d(&tma_c, buf, col, row);
          } else {
            tma_store_2d(&tma_c, buf, col, row);
          }
          bulk_commit();
        }
        nbuf ^= 1;
      };
      for (int tile = pair; tile < tiles; tile += npairs) {
        const int m0 = (tile / num_n) * (2 * BM), n0 = (tile % num_n) * BN;
        if (!mbar_wait_warp(&bar->acc_full[acc], acc_phase, ab, kErrTimeoutConsumer)) break;
        tc_fence_after();
#pragma unroll 1
        for (int chunk = 0; chunk < BN / 32; ++chunk) {
          const int col0 = n0 + chunk * 32;
          if (col0 >= g.cols) break;
          uint32_t r[32];
          tmem_ld32(tmem + ((quarter * 32u) << 16) + uint32_t(acc * BN + chunk * 32), r);
          float b[32];
          load_bias32(g.bias + col0, min(32, g.cols - col0), b);
          tmem_wait_ld();
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float x = __uint_as_float(r[j]) + b[j];
            v[j] = E == kResidual ? g.alpha * x : E == kGeluResidual ? gelu_f(x) : epi<E>(x, 0.0f, g.alpha);
          }
          stage_store(v, col0, m0 + row_box, resid);
          if (col0 < g.dual) {
            // The dual copy (a bias longer than the rows): plain bias, columns cols + col0...
            load_bias32(g.bias + g.cols + col0, min(32, g.dual - col0), b);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) + b[j];
            stage_store(v, g.cols + col0, m0 + row_box, false);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(mapa_shared(&bar->acc_empty[acc], 0));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (lane == 0) bulk_wait_all();
      __syncwarp();
    } else
    for (int tile = pair; tile < tiles; tile += npairs) {
      const int m0 = (tile / num_n) * (2 * BM), n0 = (tile % num_n) * BN;
      if (!mbar_wait_warp(&bar->acc_full[acc], acc_phase, ab, kErrTimeoutConsumer)) break;
      tc_fence_after();
      const long long row = m0 + row_in_tile;
      const bool row_ok = row < g.m;
#pragma unroll 1
      for (int chunk = 0; chunk < BN / 32; ++chunk) {
        const int col0 = n0 + chunk * 32;
        if (col0 >= g.cols) break;
        uint32_t r[32];
        tmem_ld32(tmem + ((quarter * 32u) << 16) + uint32_t(acc * BN + chunk * 32), r);
        const int lim = min(32, g.cols - col0);
        float b[32];
        load_bias32(g.bias + col0, lim, b);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (row_ok) store_row32<E>(g, row, col0, lim, v, b);
        if (col0 < g.dual) {
          const int lim2 = min(lim, g.dual - col0);
          load_bias32(g.bias + g.cols + col0, lim2, b);
          if (row_ok) store_row32<kBias>(g, row, g.cols + col0, lim2, v, b);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(&bar->acc_empty[acc], 0));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  // Both CTAs' epilogues have read their accumulators and every pair UMMA has completed before
  // the columns are released; neither CTA leaves while the other may still signal its barriers.
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, C::TMEM_COLS);
  cluster_sync();
}

// f32 rows to f16 rows, zero padded to ld_out columns.
__global__ void cast_rows_kernel(const float *__restrict__ in, long long ld_in,
                                 __half *__restrict__ out, long long ld_out, int rows, int cols) {
  griddep_launch_dependents();
  griddep_wait();  // the previous kernel of the stream has completed (programmatic launch)
  for (long long row = blockIdx.y; row < rows; row += gridDim.y) {
    const float *src = in + row * ld_in;
    __half *dst = out + row * ld_out;
    for (long long c = 2 * (blockIdx.x * (long long)blockDim.x + threadIdx.x); c < ld_out;
         c += 2LL * gridDim.x * blockDim.x) {
      float a = c < cols ? src[c] : 0.0f;
      float b = c + 1 < cols ? src[c + 1] : 0.0f;
      if (c + 1 < ld_out) {
        *reinterpret_cast<__half2 *>(dst + c) = __floats2half2_rn(a, b);
      } else {
        dst[c] = __float2half_rn(a);
      }
    }
  }
}

template <int BN, int E, int KC>
cudaError_t launch_bn_e(const CUtensorMap &a, const CUtensorMap &w, const GemmArgs &g, int grid,
                        cudaStream_t s) {
  using C = GemmCfg<BN, KC>;
  const size_t smem = 1024 + C::STAGES * C::STAGE_BYTES + sizeof(GemmBarriers);
  int dev = 0;
  cudaGetDevice(&dev);
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<BN, E, KC>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  return launch_pdl(gemm_kernel<BN, E, KC>, dim3(grid), dim3(kGemmThreads), smem, s, a, w, g);
}

template <int BN, int KC>
cudaError_t launch_bn(const CUtensorMap &a, const CUtensorMap &w, const GemmArgs &g, int grid,
                      cudaStream_t s) {
  switch (g.epilogue) {
    case kBias: return launch_bn_e<BN, kBias, KC>(a, w, g, grid, s);
    case kSilu: return launch_bn_e<BN, kSilu, KC>(a, w, g, grid, s);
    case kRelu: return launch_bn_e<BN, kRelu, KC>(a, w, g, grid, s);
    case kResidual: return launch_bn_e<BN, kResidual, KC>(a, w, g, grid, s);
    case kGelu: return launch_bn_e<BN, kGelu, KC>(a, w, g, grid, s);
    case kGeluResidual: return launch_bn_e<BN, kGeluResidual, KC>(a, w, g, grid, s);
    default: return launch_bn_e<BN, kTanh, KC>(a, w, g, grid, s);
  }
}

template <int BN, int E>
cudaError_t launch_q8_e(const CUtensorMap &a, const CUtensorMap &q, const CUtensorMap &sc,
                        const GemmArgs &g, int grid, cudaStream_t s) {
  using C = GemmQ8Cfg<BN>;
  const size_t smem = 1024 + C::STAGES * C::STAGE_BYTES + sizeof(GemmQ8Barriers);
  int dev = 0;
  cudaGetDevice(&dev);
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_q8_kernel<BN, E>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  return launch_pdl(gemm_q8_kernel<BN, E>, dim3(grid), dim3(kQ8Threads), smem, s, a, q, sc, g);
}

template <int BN>
cudaError_t launch_q8(const CUtensorMap &a, const CUtensorMap &q, const CUtensorMap &sc,
                      const GemmArgs &g, int grid, cudaStream_t s) {
  switch (g.epilogue) {
    case kBias: return launch_q8_e<BN, kBias>(a, q, sc, g, grid, s);
    case kSilu: return launch_q8_e<BN, kSilu>(a, q, sc, g, grid, s);
    case kRelu: return launch_q8_e<BN, kRelu>(a, q, sc, g, grid, s);
    case kResidual: return launch_q8_e<BN, kResidual>(a, q, sc, g, grid, s);
    case kGelu: return launch_q8_e<BN, kGelu>(a, q, sc, g, grid, s);
    case kGeluResidual: return launch_q8_e<BN, kGeluResidual>(a, q, sc, g, grid, s);
    default: return launch_q8_e<BN, kTanh>(a, q, sc, g, grid, s);
  }
}

template <int BN, int E, int KC>
cudaError_t launch2_bn_e(const CUtensorMap &a, const CUtensorMap &w, const CUtensorMap &c,
                         const GemmArgs &g, int pairs, cudaStream_t s) {
  using C = Gemm2Cfg<BN, KC>;
  const size_t smem = C::SMEM + sizeof(Gemm2Barriers);
  int dev = 0;
  cudaGetDevice(&dev);
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm2_kernel<BN, E, KC>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  return launch_pdl(gemm2_kernel<BN, E, KC>, dim3(2 * pairs), dim3(kGemmThreads), smem, s, a, w, c,
                    g);
}

template <int BN, int KC>
cudaError_t launch2_bn(const CUtensorMap &a, const CUtensorMap &w, const CUtensorMap &c,
                       const GemmArgs &g, int pairs, cudaStream_t s) {
  switch (g.epilogue) {
    case kBias: return launch2_bn_e<BN, kBias, KC>(a, w, c, g, pairs, s);
    case kSilu: return launch2_bn_e<BN, kSilu, KC>(a, w, c, g, pairs, s);
    case kRelu: return launch2_bn_e<BN, kRelu, KC>(a, w, c, g, pairs, s);
    case kResidual: return launch2_bn_e<BN, kResidual, KC>(a, w, c, g, pairs, s);
    case kGelu: return launch2_bn_e<BN, kGelu, KC>(a, w, c, g, pairs, s);
    case kGeluResidual: return launch2_bn_e<BN, kGeluResidual, KC>(a, w, c, g, pairs, s);
    default: return launch2_bn_e<BN, kTanh, KC>(a, w, c, g, pairs, s);
  }
}

}  // namespace

int gemm2_pick_bn(int m, int cols, int num_sms) {
  // Waves of pair tiles times the tile width, over the relative rate of a wave: a tile of 128
  // columns still waits on its loads (24 KB per k-block against 260 cycles of UMMAs).
  const int mt = (m + 2 * BM - 1) / (2 * BM);
  const int pairs = num_sms / 2;
  auto cost = [&](int bn, double eff) {
    const long long tiles = (long long)mt * ((cols + bn - 1) / bn);
    const long long waves = (tiles + pairs - 1) / pairs;
    return double(waves * bn) / eff;
  };
  int best = 256;
  double c = cost(256, 1.0);
  const int cand[3] = {192, 160, 128};
  const double eff[3] = {1.0, 1.0, 0.87};
  for (int i = 0; i < 3; ++i) {
    const double ci = cost(cand[i], eff[i]);
    if (ci < c) {
      c = ci;
      best = cand[i];
    }
  }
  return best;
}

cudaError_t launch_gemm2(const CUtensorMap &a, const CUtensorMap &w_half, const CUtensorMap &tma_c,
                         const GemmArgs &g, int bn, int kc, int num_sms, cudaStream_t s) {
  const int tiles = ((g.m + 2 * BM - 1) / (2 * BM)) * ((g.cols + bn - 1) / bn);
  const int pairs = tiles < num_sms / 2 ? tiles : num_sms / 2;
  if (pairs <= 0) return cudaSuccess;
  if (kc == 2) {
    switch (bn) {
      case 128: return launch2_bn<128, 2>(a, w_half, tma_c, g, pairs, s);
      case 160: return launch2_bn<160, 2>(a, w_half, tma_c, g, pairs, s);
      case 192: return launch2_bn<192, 2>(a, w_half, tma_c, g, pairs, s);
      default: return launch2_bn<256, 2>(a, w_half, tma_c, g, pairs, s);
    }
  }
  switch (bn) {
    case 128: return launch2_bn<128, 1>(a, w_half, tma_c, g, pairs, s);
    case 160: return launch2_bn<160, 1>(a, w_half, tma_c, g, pairs, s);
    case 192: return launch2_bn<192, 1>(a, w_half, tma_c, g, pairs, s);
    default: return launch2_bn<256, 1>(a, w_half, tma_c, g, pairs, s);
  }
}

int gemm_pick_bn(int m, int cols, int num_sms) {
  // Waves of tiles times the tile width: the cost of the last, partial wave included. The wider
  // tile moves a quarter fewer bytes per flop, so it wins ties.
  const int mt = (m + BM - 1) / BM;
  auto cost = [&](int bn) {
    const long long tiles = (long long)mt * ((cols + bn - 1) / bn);
    const long long waves = (tiles + num_sms - 1) / num_sms;
    return waves * bn;
  };
  // Relative throughput of a full wave by tile width (measured: wider tiles move fewer bytes per
  // flop through TMA and shared memory).
  const double c128 = cost(128) / 0.75, c160 = cost(160) / 0.85, c256 = double(cost(256));
  if (c256 <= c160 && c256 <= c128) return 256;
  return c160 <= c128 ? 160 : 128;
}

cudaError_t launch_gemm(const CUtensorMap &a, const CUtensorMap &w, const GemmArgs &g, int bn,
                        int kc, int num_sms, cudaStream_t s) {
  const int tiles = ((g.m + BM - 1) / BM) * ((g.cols + bn - 1) / bn);
  const int grid = tiles < num_sms ? tiles : num_sms;
  if (grid <= 0) return cudaSuccess;
  if (kc == 2) {
    if (bn == 160) return launch_bn<160, 2>(a, w, g, grid, s);
    return bn == 256 ? launch_bn<256, 2>(a, w, g, grid, s) : launch_bn<128, 2>(a, w, g, grid, s);
  }
  if (bn == 160) return launch_bn<160, 1>(a, w, g, grid, s);
  return bn == 256 ? launch_bn<256, 1>(a, w, g, grid, s) : launch_bn<128, 1>(a, w, g, grid, s);
}

cudaError_t launch_gemm_q8(const CUtensorMap &a, const CUtensorMap &q, const CUtensorMap &sc,
                           const GemmArgs &g, int bn, int num_sms, cudaStream_t s) {
  const int tiles = ((g.m + BM - 1) / BM) * ((g.cols + bn - 1) / bn);
  const int grid = tiles < num_sms ? tiles : num_sms;
  if (grid <= 0) return cudaSuccess;
  if (bn == 160) return launch_q8<160>(a, q, sc, g, grid, s);
  return bn == 256 ? launch_q8<256>(a, q, sc, g, grid, s) : launch_q8<128>(a, q, sc, g, grid, s);
}

cudaError_t launch_cast_rows(const float *in, long long ld_in, __half *out, long long ld_out,
                             int rows, int cols, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  int threads = 256;
  long long pairs = (ld_out + 1) / 2;
  int bx = int((pairs + threads - 1) / threads);
  if (bx > 64) bx = 64;
  dim3 grid(bx, rows < 65535 ? rows : 65535);
  return launch_pdl(cast_rows_kernel, grid, dim3(threads), 0, s, in, ld_in, out, ld_out, rows,
                    cols);
}

}  // namespace wv
