// Encoder multi-head attention for sm_100a: the reference's `Pass::attention`
// (src/gpu/mod.rs:1556-1605; attention.wgsl `flash` / `relative`, flash_f16.wgsl) re-designed as a
// tcgen05 flash-attention kernel, over segments of any length in one launch.
//
// A CTA takes 128 queries of one head of one segment. Warp 0 streams tiles with TMA (Q once, then
// K/V blocks through two-deep rings), warp 1 issues the UMMAs (S = Q·K^T into a TMEM score buffer,
// O += P·V into a TMEM accumulator), warps 2..5 own one query row per thread: they read the row's
// scores with tcgen05.ld, run the online softmax in registers (exp2 on the MUFU, a lagging maximum
// that rescales the TMEM accumulator only when the row maximum grows by more than 2^8), write the
// probabilities as f16 into a 128-byte-swizzled shared tile (the A operand of P·V), and at the end
// normalise the accumulator and store the row.
//
// With relative positions (Transformer-XL, Parakeet): score (i, j) = ((q+u)_i·k_j +
// (q+v)_i·P[pos_t + 15 - (i - j)]) / sqrt(hd), the reference's score (src/cpu/ops.rs:223-273,
// attention.wgsl:305-492). For a 128-query x 64-key block the needed position rows form a window
// of 191 consecutive rows; BD' = (q+v)·window^T is one N=192 UMMA, and the rel-shift
// BD[i][j] = BD'[i][j - i + 127] is a per-lane shift of a 96-column slice of each row, done in
// registers by a 5-stage select network (no shared-memory round trip).
//
// Keys past a segment's length are masked; query rows past it are computed and not stored.
#include "kernels.cuh"
#include "ptx.cuh"

namespace wv {
namespace {

constexpr int BM = 128;

template <int HD, bool REL>
struct Cfg {
  static constexpr int BN = REL ? 64 : 128;          // keys per block
  static constexpr int NBOX = HD / 64;               // 64-column TMA boxes per tile row
  static constexpr int ATOM_Q = BM * 128;            // bytes of one 64-column block of a Q tile
  static constexpr int ATOM_KV = BN * 128;
  static constexpr int Q_BYTES = BM * HD * 2;
  static constexpr int KV_BYTES = BN * HD * 2;
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int PW_ROWS = REL ? BM + BN : 0;  // position window rows (191 used)
  static constexpr int PW_BYTES = PW_ROWS * HD * 2;
  static constexpr int ATOM_PW = PW_ROWS * 128;
  // Shared memory layout (every block 1024-aligned).
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_QV = OFF_Q + Q_BYTES;
  static constexpr int OFF_K = OFF_QV + (REL ? Q_BYTES : 0);
  static constexpr int OFF_V = OFF_K + 2 * KV_BYTES;
  static constexpr int OFF_P = OFF_V + 2 * KV_BYTES;
  static constexpr int OFF_PW = OFF_P + 2 * P_BYTES;
  static constexpr int OFF_BAR = OFF_PW + PW_BYTES;
  // TMEM columns: score buffers, then (rel) the BD' block, then the accumulator.
  static constexpr int T_S = 0;
  static constexpr int T_BD = REL ? BN : 0;
  static constexpr int T_O = 256;
  static constexpr int TMEM_COLS = 512;
  static constexpr uint32_t IDESC_S = idesc_f16(BM, BN, 0);
  static constexpr uint32_t IDESC_BD = idesc_f16(BM, REL ? PW_ROWS : 64, 0);
  static constexpr uint32_t IDESC_PV = idesc_f16(BM, HD, 1);
};

struct __align__(8) AttnBarriers {
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t pw_full, pw_empty;
  uint64_t s_full[2], s_free[2];
  uint64_t p_full[2], pv_done[2];
  uint64_t o_full;
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t abort;
};

// w[x] <- w[x + s] for x < 64, s in [0, 31]: a shift by a per-lane amount with static register
// indices (a select per element and stage; the unused upper outputs are dead code).
template <int SH, int OUT>
__device__ __forceinline__ void shift_stage(float (&w)[96], bool take) {
#pragma unroll
  for (int x = 0; x < OUT; ++x) w[x] = take ? w[x + SH] : w[x];
}

__device__ __forceinline__ void shift_left(float (&w)[96], uint32_t s) {
  // Each stage makes just the outputs the later stages read: 79, 71, 67, 65, 64.
  shift_stage<16, 79>(w, (s >> 4) & 1u);
  shift_stage<8, 71>(w, (s >> 3) & 1u);
  shift_stage<4, 67>(w, (s >> 2) & 1u);
  shift_stage<2, 65>(w, (s >> 1) & 1u);
  shift_stage<1, 64>(w, s & 1u);
}

template <int HD, bool REL>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_kv,
                const __grid_constant__ CUtensorMap map_pos, const AttnArgs a) {
  using C = Cfg<HD, REL>;
  constexpr int BN = C::BN;

  const int seg = blockIdx.z, h = blockIdx.y;
  const int T = a.seg_len ? a.seg_len[seg] : a.single_t;
  const int row0 = a.seg_len ? a.seg_start[seg] : 0;
  const int m0 = blockIdx.x * BM;
  if (m0 >= T) return;  // uniform: the whole CTA leaves before any setup
  const int nb = (T + BN - 1) / BN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  AttnBarriers *bar = reinterpret_cast<AttnBarriers *>(smem + C::OFF_BAR);
  const uint32_t warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    mbar_init(&bar->q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->k_full[i], 1);
      mbar_init(&bar->k_empty[i], 1);
      mbar_init(&bar->v_full[i], 1);
      mbar_init(&bar->v_empty[i], 1);
      mbar_init(&bar->s_full[i], 1);
      mbar_init(&bar->s_free[i], 128);
      mbar_init(&bar->p_full[i], 128);
      mbar_init(&bar->pv_done[i], 1);
    }
    mbar_init(&bar->pw_full, 1);
    mbar_init(&bar->pw_empty, 1);
    mbar_init(&bar->o_full, 1);
    mbar_init(&bar->drain, 1);
    bar->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&map_q);
    prefetch_tmap(&map_kv);
    if (REL) prefetch_tmap(&map_pos);
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
  griddep_launch_dependents();
  griddep_wait();  // the previous kernel of the stream has completed (programmatic launch)
  const int hoff = h * a.head_stride;

  if (warp == 0) {
    // ---- TMA producer ----------------------------------------------------------------------
    if (lane == 0) {
      bool ok = true;
      // Parity of the last arm of each ring slot (bit 1: armed at least once).
      uint32_t k_last[2] = {0, 0}, v_last[2] = {0, 0}, pw_last = 0;
      mbar_arrive_expect_tx(&bar->q_full, (REL ? 2 : 1) * C::Q_BYTES);
#pragma unroll
      for (int b = 0; b < C::NBOX; ++b) {
        tma_load_2d(smem + C::OFF_Q + b * C::ATOM_Q, &map_q, &bar->q_full, a.q_off + hoff + 64 * b,
                    row0 + m0);
        if (REL)
          tma_load_2d(smem + C::OFF_QV + b * C::ATOM_Q, &map_q, &bar->q_full,
                      a.qv_off + hoff + 64 * b, row0 + m0);
      }
      for (int j = 0; j < nb && ok; ++j) {
        const int s = j & 1;
        const uint32_t par = ((j >> 1) & 1) ^ 1u;
        if (!mbar_wait(&bar->k_empty[s], par, ab, kErrTimeoutProducer)) { ok = false; break; }
        mbar_arrive_expect_tx(&bar->k_full[s], C::KV_BYTES);
#pragma unroll
        for (int b = 0; b < C::NBOX; ++b)
          tma_load_2d(smem + C::OFF_K + s * C::KV_BYTES + b * C::ATOM_KV, &map_kv, &bar->k_full[s],
                      a.k_off + hoff + 64 * b, row0 + j * BN);
        k_last[s] = 2u | ((j >> 1) & 1u);
        if (REL) {
          if (!mbar_wait(&bar->pw_empty, (j & 1) ^ 1u, ab, kErrTimeoutProducer)) { ok = false; break; }
          mbar_arrive_expect_tx(&bar->pw_full, C::PW_BYTES);
          const int rho0 = a.pos_t + 15 + j * BN - m0 - (BM - 1);
#pragma unroll
          for (int b = 0; b < C::NBOX; ++b)
            tma_load_2d(smem + C::OFF_PW + b * C::ATOM_PW, &map_pos, &bar->pw_full,
                        a.pos_off + hoff + 64 * b, rho0);
          pw_last = 2u | (j & 1u);
        }
        if (!mbar_wait(&bar->v_empty[s], par, ab, kErrTimeoutProducer)) { ok = false; break; }
        mbar_arrive_expect_tx(&bar->v_full[s], C::KV_BYTES);
#pragma unroll
        for (int b = 0; b < C::NBOX; ++b)
          tma_load_2d(smem + C::OFF_V + s * C::KV_BYTES + b * C::ATOM_KV, &map_kv, &bar->v_full[s],
                      a.v_off + hoff + 64 * b, row0 + j * BN);
        v_last[s] = 2u | ((j >> 1) & 1u);
      }
      if (!ok) {
        // Wait (bounded) for the loads already issued to land before the CTA may exit.
        long long t0 = clock64();
        auto drain = [&](uint64_t *b, uint32_t last) {
          if (!(last & 2u)) return;
          while (!mbar_try_wait(b, last & 1u) && clock64() - t0 < kWaitCycles) {
          }
        };
        drain(&bar->q_full, 2u);
        for (int s = 0; s < 2; ++s) {
          drain(&bar->k_full[s], k_last[s]);
          drain(&bar->v_full[s], v_last[s]);
        }
        drain(&bar->pw_full, pw_last);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ------------------------------------------------------------------------
    if (lane == 0) {
      bool ok = mbar_wait(&bar->q_full, 0, ab, kErrTimeoutMma);
      bool issued = false;
      const int hsteps = (a.hd + 15) / 16;
      const uint32_t sq = smem_u32(smem + C::OFF_Q), sqv = smem_u32(smem + C::OFF_QV);
      const uint32_t sk = smem_u32(smem + C::OFF_K), sv = smem_u32(smem + C::OFF_V);
      const uint32_t sp = smem_u32(smem + C::OFF_P), spw = smem_u32(smem + C::OFF_PW);
      tc_fence_after();
      auto pv = [&](int i) -> bool {
        const int b = i & 1;
        if (!mbar_wait(&bar->p_full[b], (i >> 1) & 1, ab, kErrTimeoutMma)) return false;
        if (!mbar_wait(&bar->v_full[b], (i >> 1) & 1, ab, kErrTimeoutMma)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t ad = sdesc_sw128(sp + b * C::P_BYTES + (kk >> 2) * C::ATOM_Q + (kk & 3) * 32,
                                          16, 1024);
          const uint64_t bd = sdesc_sw128(sv + b * C::KV_BYTES + kk * 16 * 128, C::ATOM_KV, 1024);
          umma_f16(tmem + C::T_O, ad, bd, C::IDESC_PV, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bar->v_empty[b]);
        umma_commit(&bar->pv_done[b]);
        return true;
      };
      for (int j = 0; j <= nb && ok; ++j) {
        if (j < nb) {
          const int s = j & 1;
          if (!mbar_wait(&bar->k_full[s], (j >> 1) & 1, ab, kErrTimeoutMma)) { ok = false; break; }
          if (REL) {
            if (!mbar_wait(&bar->pw_full, j & 1, ab, kErrTimeoutMma)) { ok = false; break; }
            if (j >= 1 && !mbar_wait(&bar->s_free[0], (j - 1) & 1, ab, kErrTimeoutMma)) {
              ok = false;
              break;
            }
          } else if (j >= 2 && !mbar_wait(&bar->s_free[s], ((j - 2) >> 1) & 1, ab, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ts = tmem + C::T_S + (REL ? 0 : s * BN);
          if (REL) {
            for (int kk = 0; kk < hsteps; ++kk) {
              const uint64_t ad = sdesc_sw128(sqv + (kk >> 2) * C::ATOM_Q + (kk & 3) * 32, 16, 1024);
              const uint64_t bd = sdesc_sw128(spw + (kk >> 2) * C::ATOM_PW + (kk & 3) * 32, 16, 1024);
              umma_f16(tmem + C::T_BD, ad, bd, C::IDESC_BD, kk > 0 ? 1u : 0u);
            }
          }
          for (int kk = 0; kk < hsteps; ++kk) {
            const uint64_t ad = sdesc_sw128(sq + (kk >> 2) * C::ATOM_Q + (kk & 3) * 32, 16, 1024);
            const uint64_t bd =
                sdesc_sw128(sk + s * C::KV_BYTES + (kk >> 2) * C::ATOM_KV + (kk & 3) * 32, 16, 1024);
            umma_f16(ts, ad, bd, C::IDESC_S, kk > 0 ? 1u : 0u);
          }
          issued = true;
          umma_commit(&bar->s_full[REL ? 0 : s]);
          umma_commit(&bar->k_empty[s]);
          if (REL) umma_commit(&bar->pw_empty);
        }
        if (j >= 1) {
          if (!pv(j - 1)) { ok = false; break; }
        }
      }
      if (ok) {
        umma_commit(&bar->o_full);
      } else if (issued) {
        umma_commit(&bar->drain);
        long long t0 = clock64();
        while (!mbar_try_wait(&bar->drain, 0) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  } else {
    // ---- softmax / epilogue: warps 2..5, one query row per thread ---------------------------
    const uint32_t quarter = warp & 3u;
    const int ii = int(quarter * 32 + lane);
    const uint32_t tl = tmem + ((quarter * 32u) << 16);
    float m_use = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nb; ++j) {
      const int b = REL ? 0 : (j & 1);
      const uint32_t spar = REL ? (j & 1) : ((j >> 1) & 1);
      if (!mbar_wait(&bar->s_full[b], spar, ab, kErrTimeoutConsumer)) { ok = false; break; }
      tc_fence_after();
      float s[BN];
      if (REL) {
        float w[96];
        {
          uint32_t r[32];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tmem_ld32(tl + C::T_S + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int x = 0; x < 32; ++x) s[c * 32 + x] = __uint_as_float(r[x]);
          }
          const uint32_t cb = 96u - 32u * quarter;
#pragma unroll
          for (int c = 0; c < 3; ++c) {
            tmem_ld32(tl + C::T_BD + cb + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int x = 0; x < 32; ++x) w[c * 32 + x] = __uint_as_float(r[x]);
          }
        }
        tc_fence_before();
        mbar_arrive(&bar->s_free[0]);
        shift_left(w, 31u - lane);
#pragma unroll
        for (int x = 0; x < BN; ++x) s[x] = s[x] + w[x];
      } else {
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          tmem_ld32(tl + C::T_S + b * BN + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int x = 0; x < 32; ++x) s[c * 32 + x] = __uint_as_float(r[x]);
        }
        tc_fence_before();
        mbar_arrive(&bar->s_free[b]);
      }
      // Scale into log2 units, mask keys past the segment, block maximum.
      const int kvalid = T - j * BN;
      float mx = -INFINITY;
#pragma unroll
      for (int x = 0; x < BN; ++x) {
        s[x] = (x < kvalid) ? s[x] * a.scale_log2 : -INFINITY;
        mx = fmaxf(mx, s[x]);
      }
      // The probability buffer b is free once P·V of block j - 2 completed.
      const int pb = j & 1;
      if (j >= 2 && !mbar_wait(&bar->pv_done[pb], ((j - 2) >> 1) & 1, ab, kErrTimeoutConsumer)) {
        ok = false;
        break;
      }
      const float m_new = fmaxf(m_use, mx);
      const bool need = m_new > m_use + 8.0f;
      if (__any_sync(0xffffffffu, need) && j > 0) {
        // Rescale the accumulator row once P·V of block j - 1 has landed in it.
        if (!mbar_wait(&bar->pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, ab, kErrTimeoutConsumer)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float alpha = need ? ex2(m_use - m_new) : 1.0f;
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          tmem_ld32(tl + C::T_O + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int x = 0; x < 32; ++x) r[x] = __float_as_uint(__uint_as_float(r[x]) * alpha);
          tmem_st32(tl + C::T_O + c * 32, r);
        }
        tmem_wait_st();
        l *= alpha;
      }
      if (need) m_use = m_new;
      // Probabilities as f16 into the swizzled A tile of P·V.
      uint8_t *prow = smem + C::OFF_P + pb * C::P_BYTES;
#pragma unroll
      for (int c = 0; c < BN / 8; ++c) {
        float p[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) {
          p[x] = ex2(s[8 * c + x] - m_use);
          l += p[x];
        }
        uint4 v = make_uint4(pack_half2(p[0], p[1]), pack_half2(p[2], p[3]),
                             pack_half2(p[4], p[5]), pack_half2(p[6], p[7]));
        *reinterpret_cast<uint4 *>(prow + (c >> 3) * C::ATOM_Q + sw128_offset(ii, c & 7)) = v;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bar->p_full[pb]);
    }
    if (ok && mbar_wait(&bar->o_full, 0, ab, kErrTimeoutConsumer)) {
      tc_fence_after();
      const float inv = 1.0f / l;
      const int qrow = m0 + ii;
      const bool store = qrow < T;
      const long long orow = (long long)(row0 + qrow) * a.ldo + (long long)h * a.hd;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tl + C::T_O + c * 32, r);
        tmem_wait_ld();
        if (store) {
          const int c0 = c * 32;
          if (a.o_f16) {
            __half *o = reinterpret_cast<__half *>(a.o) + orow;
#pragma unroll
            for (int x = 0; x < 32; x += 2) {
              if (c0 + x + 1 < a.hd) {
                *reinterpret_cast<__half2 *>(o + c0 + x) = __floats2half2_rn(
                    __uint_as_float(r[x]) * inv, __uint_as_float(r[x + 1]) * inv);
              } else if (c0 + x < a.hd) {
                o[c0 + x] = __float2half_rn(__uint_as_float(r[x]) * inv);
              }
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

// f32 or f16 operand rows -> f16 rows with heads padded to hd_pad.
__global__ void pack_heads_kernel(const void *__restrict__ in, int in_f16, long long ld_in,
                                  const int4 offs, int sections, __half *__restrict__ out,
                                  long long ld_out, int rows, int heads, int hd, int hd_pad) {
  const long long width = (long long)sections * heads * hd_pad;
  for (long long row = blockIdx.y; row < rows; row += gridDim.y) {
    for (long long c = blockIdx.x * (long long)blockDim.x + threadIdx.x; c < width;
         c += (long long)gridDim.x * blockDim.x) {
      const int sec = int(c / (heads * hd_pad));
      const int rem = int(c % (heads * hd_pad));
      const int hh = rem / hd_pad, x = rem % hd_pad;
      const int off = sec == 0 ? offs.x : sec == 1 ? offs.y : sec == 2 ? offs.z : offs.w;
      float v = 0.0f;
      if (x < hd) {
        const long long at = row * ld_in + off + (long long)hh * hd + x;
        v = in_f16 ? __half2float(reinterpret_cast<const __half *>(in)[at])
                   : reinterpret_cast<const float *>(in)[at];
      }
      out[row * ld_out + c] = __float2half_rn(v);
    }
  }
}

template <int HD, bool REL>
cudaError_t launch_one(const CUtensorMap &q, const CUtensorMap &kv, const CUtensorMap &pos,
                       const AttnArgs &a, int max_len, int nseg, cudaStream_t s) {
  using C = Cfg<HD, REL>;
  const size_t smem = 1024 + C::OFF_BAR + sizeof(AttnBarriers);
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attn_kernel<HD, REL>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  dim3 grid((max_len + BM - 1) / BM, a.heads, nseg);
  return launch_pdl(attn_kernel<HD, REL>, grid, dim3(kAttnThreads), smem, s, q, kv, pos, a);
}

}  // namespace

cudaError_t launch_attention(const CUtensorMap &map_q, const CUtensorMap &map_kv,
                             const CUtensorMap &map_pos, const AttnArgs &a, int hd_pad, bool rel,
                             int max_len, int nseg, cudaStream_t s) {
  if (max_len <= 0 || nseg <= 0) return cudaSuccess;
  if (rel) return launch_one<128, true>(map_q, map_kv, map_pos, a, max_len, nseg, s);
  return launch_fa_attention(map_q, map_kv, a, hd_pad, max_len, nseg, s);
}

int attn_block_keys(bool rel, int hd_pad) {
  return rel ? Cfg<128, true>::BN : fa_block_keys(hd_pad);
}
int attn_pos_window_rows() { return Cfg<128, true>::PW_ROWS; }

cudaError_t launch_pack_heads(const void *in, int in_f16, long long ld_in, const int *in_off,
                              int sections, __half *out, long long ld_out, int rows, int heads,
                              int hd, int hd_pad, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  int4 offs = make_int4(in_off[0], sections > 1 ? in_off[1] : 0, sections > 2 ? in_off[2] : 0,
                        sections > 3 ? in_off[3] : 0);
  const long long width = (long long)sections * heads * hd_pad;
  int bx = int((width + 255) / 256);
  if (bx > 32) bx = 32;
  dim3 grid(bx, rows < 65535 ? rows : 65535);
  pack_heads_kernel<<<grid, 256, 0, s>>>(in, in_f16, ld_in, offs, sections, out, ld_out, rows,
                                         heads, hd, hd_pad);
  return cudaGetLastError();
}

}  // namespace wv
