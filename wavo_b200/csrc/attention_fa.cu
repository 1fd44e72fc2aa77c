// Encoder self-attention without position terms (Whisper, GigaAM after RoPE): the reference's
// `Pass::attention` with qk [q | k | v] or [q | k] + v (src/gpu/mod.rs:1556-1605; attention.wgsl
// `flash`, flash_f16.wgsl), as a tcgen05 flash-attention kernel over segments of any length.
//
// A CTA takes two 128-query tiles of one head of one segment, so that the tensor core works on one
// tile while the other tile's softmax runs:
//   warp 0     TMA: both Q tiles once, then K and V blocks through three-slot rings;
//   warp 1     one thread issues the UMMAs: S_t = Q_t·K^T into TMEM, then O_t += P_t·V with P_t
//              read from TMEM;
//   warps 2-5  softmax of tile 0, warps 6-9 softmax of tile 1: one query row per thread, read from
//              TMEM with tcgen05.ld in two passes (row maximum, then probabilities); a lagging
//              maximum (the TMEM accumulator is rescaled only when a row maximum grows by more than
//              2^8); a quarter of the exponentials on the FMA pipe (a degree-4 polynomial for 2^f
//              on [-1/2, 1/2] fitted for this kernel, with the exponent added in the integer bits),
//              the rest on the MUFU; probabilities written back to TMEM as f16 pairs with
//              tcgen05.st (the UMMAs already use shared memory at its full read rate, so P stays
//              out of it); at the end the accumulator row is normalised and stored.
#include "kernels.cuh"
#include "ptx.cuh"

namespace wv {
namespace {

constexpr int BM = 128;
constexpr int NT = 2;  // query tiles per CTA
constexpr int THREADS = 64 + NT * 128;
constexpr int KVS = 3;  // K and V ring slots

template <int HD, int BN>
struct Fa {
  static constexpr int NBOX = HD / 64;
  static constexpr int ATOM_Q = BM * 128;
  static constexpr int ATOM_KV = BN * 128;
  static constexpr int Q_BYTES = BM * HD * 2;
  static constexpr int KV_BYTES = BN * HD * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + NT * Q_BYTES;
  static constexpr int OFF_V = OFF_K + KVS * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + KVS * KV_BYTES;
  // TMEM columns of tile t, from t·256: the scores S (BN f32 columns), the probabilities P (BN
  // f16, two per column: the A operand of P·V, read by the tensor core from TMEM, so that neither
  // the softmax's writes nor the UMMA's reads of P touch shared memory), the accumulator O.
  static constexpr int T_TILE = 256;
  static constexpr int T_S = 0;
  static constexpr int T_P = BN;
  static constexpr int T_O = (BN + BN / 2 + 31) / 32 * 32;
  static constexpr int TMEM_COLS = 512;
  static constexpr uint32_t IDESC_S = idesc_f16(BM, BN, 0);
  static constexpr uint32_t IDESC_PV = idesc_f16(BM, HD, 1);
  static_assert(T_O + HD <= T_TILE && NT * T_TILE <= TMEM_COLS, "TMEM");
};

struct __align__(8) FaBarriers {
  uint64_t q_full;
  uint64_t k_full[KVS], k_empty[KVS];
  uint64_t v_full[KVS], v_empty[KVS];
  uint64_t s_full[NT], s_free[NT];
  uint64_t p_full[NT], pv_done[NT];
  uint64_t o_full;
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t abort;
};

// 2^x for x in [-125, 8] on the FMA pipe: x = n + f with n = round(x), f in [-1/2, 1/2]; 2^f by a
// degree-4 polynomial (coefficients fitted here to the relative error of 2^f, max 7.7e-6 in f32),
// 2^n added to the exponent bits.
__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -125.0f);
  const float t = x + 12582912.0f;  // 1.5·2^23: rounds x to an integer in the low bits
  const float n = t - 12582912.0f;
  const float f = x - n;
  float p = 0.009251425974071026f;
  p = fmaf(p, f, 0.055853113532066345f);
  p = fmaf(p, f, 0.24031664431095123f);
  p = fmaf(p, f, 0.6931320428848267f);
  p = fmaf(p, f, 0.9999976754188538f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

template <int HD, int BN>
__global__ void __launch_bounds__(THREADS, 1)
    fa_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_kv,
              const AttnArgs a) {
  using C = Fa<HD, BN>;
  const int seg = blockIdx.z, h = blockIdx.y;
  const int T = a.seg_len ? a.seg_len[seg] : a.single_t;
  const int row0 = a.seg_len ? a.seg_start[seg] : 0;
  const int m0 = blockIdx.x * (NT * BM);
  if (m0 >= T) return;  // uniform: the whole CTA leaves before any setup
  const int nt = (m0 + BM < T) ? NT : 1;  // tiles with queries in the segment
  const int nb = (T + BN - 1) / BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  FaBarriers *bar = reinterpret_cast<FaBarriers *>(smem + C::OFF_BAR);
  const uint32_t warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    mbar_init(&bar->q_full, 1);
    for (int i = 0; i < KVS; ++i) {
      mbar_init(&bar->k_full[i], 1);
      mbar_init(&bar->k_empty[i], 1);
      mbar_init(&bar->v_full[i], 1);
      mbar_init(&bar->v_empty[i], 1);
    }
    for (int t = 0; t < NT; ++t) {
      mbar_init(&bar->s_full[t], 1);
      mbar_init(&bar->s_free[t], 4);
      mbar_init(&bar->p_full[t], 4);
      mbar_init(&bar->pv_done[t], 1);
    }
    mbar_init(&bar->o_full, 1);
    mbar_init(&bar->drain, 1);
    bar->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&map_q);
    prefetch_tmap(&map_kv);
  }
  if (warp == 1) {
    tmem_alloc(&bar->tmem_base, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;
  const Abort ab{&bar->abort, a.err};
  const int hoff = h * a.head_stride;

  if (warp == 0) {
    // ---- TMA producer ------------------------------------------------------------------------
    if (lane == 0) {
      bool ok = true;
      uint32_t k_last[KVS] = {}, v_last[KVS] = {};  // bit 1: armed; bit 0: parity
      mbar_arrive_expect_tx(&bar->q_full, NT * C::Q_BYTES);
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int b = 0; b < C::NBOX; ++b)
          tma_load_2d(smem + C::OFF_Q + t * C::Q_BYTES + b * C::ATOM_Q, &map_q, &bar->q_full,
                      a.q_off + hoff + 64 * b, row0 + m0 + t * BM);
      for (int j = 0; j < nb; ++j) {
        const int s = j % KVS;
        const uint32_t par = ((j / KVS) & 1) ^ 1u;
        if (!mbar_wait(&bar->k_empty[s], par, ab, kErrTimeoutProducer)) { ok = false; break; }
        mbar_arrive_expect_tx(&bar->k_full[s], C::KV_BYTES);
#pragma unroll
        for (int b = 0; b < C::NBOX; ++b)
          tma_load_2d(smem + C::OFF_K + s * C::KV_BYTES + b * C::ATOM_KV, &map_kv, &bar->k_full[s],
                      a.k_off + hoff + 64 * b, row0 + j * BN);
        k_last[s] = 2u | ((j / KVS) & 1u);
        if (!mbar_wait(&bar->v_empty[s], par, ab, kErrTimeoutProducer)) { ok = false; break; }
        mbar_arrive_expect_tx(&bar->v_full[s], C::KV_BYTES);
#pragma unroll
        for (int b = 0; b < C::NBOX; ++b)
          tma_load_2d(smem + C::OFF_V + s * C::KV_BYTES + b * C::ATOM_KV, &map_kv, &bar->v_full[s],
                      a.v_off + hoff + 64 * b, row0 + j * BN);
        v_last[s] = 2u | ((j / KVS) & 1u);
      }
      if (!ok) {
        const long long t0 = clock64();
        auto drain = [&](uint64_t *b, uint32_t last) {
          if (!(last & 2u)) return;
          while (!mbar_try_wait(b, last & 1u) && clock64() - t0 < kWaitCycles) {
          }
        };
        drain(&bar->q_full, 2u);
        for (int s = 0; s < KVS; ++s) {
          drain(&bar->k_full[s], k_last[s]);
          drain(&bar->v_full[s], v_last[s]);
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----------------------------------------------------------------------------
    if (lane == 0) {
      bool ok = mbar_wait(&bar->q_full, 0, ab, kErrTimeoutMma);
      bool issued = false;
      const int hsteps = (a.hd + 15) / 16;
      const uint32_t sq = smem_u32(smem + C::OFF_Q), sk = smem_u32(smem + C::OFF_K);
      const uint32_t sv = smem_u32(smem + C::OFF_V);
      tc_fence_after();
      // Per block j, tile by tile: S_t(j) as soon as tile t's softmax released S_t(j-1), then
      // P_t(j-1)·V(j-1). Tiles advance independently, so one tile's softmax overlaps the other
      // tile's UMMAs.
      for (int j = 0; j <= nb && ok; ++j) {
        const int sk_slot = j % KVS, sv_slot = (j + KVS - 1) % KVS;
        if (j < nb && !mbar_wait(&bar->k_full[sk_slot], (j / KVS) & 1, ab, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        if (j >= 1 &&
            !mbar_wait(&bar->v_full[sv_slot], ((j - 1) / KVS) & 1, ab, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        for (int t = 0; t < nt && ok; ++t) {
          if (j < nb) {
            if (j >= 1 && !mbar_wait(&bar->s_free[t], (j - 1) & 1, ab, kErrTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            for (int kk = 0; kk < hsteps; ++kk) {
              const uint64_t ad =
                  sdesc_sw128(sq + t * C::Q_BYTES + (kk >> 2) * C::ATOM_Q + (kk & 3) * 32, 16, 1024);
              const uint64_t bd = sdesc_sw128(
                  sk + sk_slot * C::KV_BYTES + (kk >> 2) * C::ATOM_KV + (kk & 3) * 32, 16, 1024);
              umma_f16(tmem + t * C::T_TILE + C::T_S, ad, bd, C::IDESC_S, kk > 0 ? 1u : 0u);
            }
            issued = true;
            umma_commit(&bar->s_full[t]);
          }
          if (j >= 1) {
            const int i = j - 1;
            if (!mbar_wait(&bar->p_full[t], i & 1, ab, kErrTimeoutMma)) { ok = false; break; }
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk) {
              // A = P from TMEM: keys 16kk.. are columns 8kk.. of the P region.
              const uint64_t bd =
                  sdesc_sw128(sv + sv_slot * C::KV_BYTES + kk * 16 * 128, C::ATOM_KV, 1024);
              umma_f16_ts(tmem + t * C::T_TILE + C::T_O, tmem + t * C::T_TILE + C::T_P + kk * 8,
                          bd, C::IDESC_PV, (i > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit(&bar->pv_done[t]);
          }
        }
        if (!ok) break;
        if (j < nb) umma_commit(&bar->k_empty[sk_slot]);
        if (j >= 1) umma_commit(&bar->v_empty[sv_slot]);
      }
      if (ok) {
        umma_commit(&bar->o_full);
      } else if (issued) {
        umma_commit(&bar->drain);
        const long long t0 = clock64();
        while (!mbar_try_wait(&bar->drain, 0) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else {
    // ---- softmax: warps 2..5 tile 0, warps 6..9 tile 1; one query row per thread ----------------
    const int t = int(warp - 2) >> 2;
    const uint32_t quarter = warp & 3u;
    const int ii = int(quarter * 32 + lane);
    const uint32_t tl = tmem + ((quarter * 32u) << 16);
    const uint32_t ts = tl + t * C::T_TILE + C::T_S, tp = tl + t * C::T_TILE + C::T_P;
    const uint32_t to = tl + t * C::T_TILE + C::T_O;
    const float c = a.scale_log2;
    float m_use = -INFINITY, l = 0.0f;
    bool ok = t < nt;
    for (int j = 0; j < nb && ok; ++j) {
      if (!mbar_wait(&bar->s_full[t], j & 1, ab, kErrTimeoutConsumer)) { ok = false; break; }
      tc_fence_after();
      // Keys past the segment (last block only) are masked to -inf in both passes.
      const int kvalid = T - j * BN;
      // Pass 1: the block's row maximum, 32 columns at a time, the next load in flight.
      float mx = -INFINITY;
      {
        uint32_t ra[32], rb[32];
        tmem_ld32(ts, ra);
#pragma unroll
        for (int q = 0; q < BN / 32; ++q) {
          uint32_t(&cur)[32] = (q & 1) ? rb : ra;
          uint32_t(&nxt)[32] = (q & 1) ? ra : rb;
          tmem_wait_ld();
          if (q + 1 < BN / 32) tmem_ld32(ts + (q + 1) * 32, nxt);
          if (kvalid < BN) {
#pragma unroll
            for (int x = 0; x < 32; ++x)
              if (q * 32 + x >= kvalid) cur[x] = __float_as_uint(-INFINITY);
          }
#pragma unroll
          for (int x = 0; x < 32; x += 2)
            mx = max3(mx, __uint_as_float(cur[x]), __uint_as_float(cur[x + 1]));
        }
      }
      const float m_blk = mx * c;
      // P_t is free and O_t stable once P·V of block j - 1 landed.
      if (j >= 1 && !mbar_wait(&bar->pv_done[t], (j - 1) & 1, ab, kErrTimeoutConsumer)) {
        ok = false;
        break;
      }
      const bool need = m_blk > m_use + 8.0f;
      if (__any_sync(0xffffffffu, need) && j > 0) {
        tc_fence_after();
        const float alpha = need ? ex2(m_use - m_blk) : 1.0f;
        uint32_t r[32];
#pragma unroll
        for (int q = 0; q < HD / 32; ++q) {
          tmem_ld32(to + q * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int x = 0; x < 32; ++x) r[x] = __float_as_uint(__uint_as_float(r[x]) * alpha);
          tmem_st32(to + q * 32, r);
        }
        tmem_wait_st();
        l *= alpha;
      }
      if (need) m_use = m_blk;
      const float nm = -m_use;
      // Pass 2: probabilities, 32 columns at a time, the next load in flight.
      {
        uint32_t ra[32], rb[32];
        tmem_ld32(ts, ra);
#pragma unroll
        for (int q = 0; q < BN / 32; ++q) {
          uint32_t(&cur)[32] = (q & 1) ? rb : ra;
          uint32_t(&nxt)[32] = (q & 1) ? ra : rb;
          tmem_wait_ld();
          if (q + 1 < BN / 32) tmem_ld32(ts + (q + 1) * 32, nxt);
          if (kvalid < BN) {
#pragma unroll
            for (int x = 0; x < 32; ++x)
              if (q * 32 + x >= kvalid) cur[x] = __float_as_uint(-INFINITY);
          }
          uint32_t pk[16];  // 32 probabilities as 16 f16 pairs: 16 columns of the P region
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            float p[8];
#pragma unroll
            for (int x = 0; x < 8; ++x) {
              const float e = fmaf(__uint_as_float(cur[8 * g + x]), c, nm);
              p[x] = ((x & 3) == 3) ? exp2_poly(e) : ex2(e);
            }
            l += ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
#pragma unroll
            for (int x = 0; x < 4; ++x) pk[4 * g + x] = pack_half2(p[2 * x], p[2 * x + 1]);
          }
          tmem_st16(tp + q * 16, pk);
        }
      }
      // The S columns are read and P is in TMEM: the next S of this tile may overwrite S, and the
      // P·V UMMA may read P.
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar->s_free[t]);
        mbar_arrive(&bar->p_full[t]);
      }
    }
    if (ok && mbar_wait(&bar->o_full, 0, ab, kErrTimeoutConsumer)) {
      tc_fence_after();
      const float inv = 1.0f / l;
      const int qrow = m0 + t * BM + ii;
      const bool store = qrow < T;
      const long long orow = (long long)(row0 + qrow) * a.ldo + (long long)h * a.hd;
#pragma unroll
      for (int q = 0; q < HD / 32; ++q) {
        uint32_t r[32];
        tmem_ld32(to + q * 32, r);
        tmem_wait_ld();
        if (store) {
          const int c0 = q * 32;
          if (a.o_f16) {
            __half *o = reinterpret_cast<__half *>(a.o) + orow;
            if (c0 + 32 <= a.hd && ((reinterpret_cast<uintptr_t>(o + c0) & 15u) == 0)) {
#pragma unroll
              for (int x = 0; x < 32; x += 8) {
                const uint4 v = make_uint4(
                    pack_half2(__uint_as_float(r[x]) * inv, __uint_as_float(r[x + 1]) * inv),
                    pack_half2(__uint_as_float(r[x + 2]) * inv, __uint_as_float(r[x + 3]) * inv),
                    pack_half2(__uint_as_float(r[x + 4]) * inv, __uint_as_float(r[x + 5]) * inv),
                    pack_half2(__uint_as_float(r[x + 6]) * inv, __uint_as_float(r[x + 7]) * inv));
                *reinterpret_cast<uint4 *>(o + c0 + x) = v;
              }
            } else {
#pragma unroll
              for (int x = 0; x < 32; ++x)
                if (c0 + x < a.hd) o[c0 + x] = __float2half_rn(__uint_as_float(r[x]) * inv);
            }
          } else {
            float *o = reinterpret_cast<float *>(a.o) + orow;
#pragma unroll
            for (int x = 0; x < 32; ++x)
              if (c0 + x < a.hd) o[c0 + x] = __uint_as_float(r[x]) * inv;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

template <int HD, int BN>
cudaError_t launch_fa(const CUtensorMap &q, const CUtensorMap &kv, const AttnArgs &a, int max_len,
                      int nseg, cudaStream_t s) {
  using C = Fa<HD, BN>;
  const size_t smem = 1024 + C::OFF_BAR + sizeof(FaBarriers);
  int dev = 0;
  cudaGetDevice(&dev);
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(fa_kernel<HD, BN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  dim3 grid((max_len + NT * BM - 1) / (NT * BM), a.heads, nseg);
  fa_kernel<HD, BN><<<grid, THREADS, smem, s>>>(q, kv, a);
  return cudaGetLastError();
}

}  // namespace

int fa_block_keys(int hd_pad) { return hd_pad == 64 ? 128 : 64; }

cudaError_t launch_fa_attention(const CUtensorMap &map_q, const CUtensorMap &map_kv,
                                const AttnArgs &a, int hd_pad, int max_len, int nseg,
                                cudaStream_t s) {
  if (max_len <= 0 || nseg <= 0) return cudaSuccess;
  if (hd_pad == 64) return launch_fa<64, 128>(map_q, map_kv, a, max_len, nseg, s);
  return launch_fa<128, 64>(map_q, map_kv, a, max_len, nseg, s);
}

}  // namespace wv
