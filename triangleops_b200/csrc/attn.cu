// attn.cu — biased, key-masked flash attention on tcgen05 for triangle attention
// (starting node, rows of the pair tensor) and attention-with-pair-bias (one row).
//
// Semantics per (row r, head h, query q)  [triangle_attn/kernel.py:194-253]:
//   S[q,k] = Q[r,h,q,:] . K[r,h,k,:] + bias[h,q,k]          (Q already scaled; log2 units)
//   O[r,q,h*D:(h+1)*D] = sum_k softmax_k(S over unmasked k) V[r,h,k,:]
// The bias is shared by every row r (triangle attention) — one CTA therefore
// processes TR rows x TQ query blocks for the same head, so each bias tile read
// from L2 serves TR rows and each K/V tile serves TQ query blocks.
//
// Key mask without per-element work: the projection stage zeroes V at masked keys
// and writes a 0/1 mask row; here that row is appended to V^T as row D of the PV
// B operand, so the PV MMA also produces l = sum_k p_k * mask_k in accumulator
// column D. Masked keys therefore contribute to neither O nor l (the reference's
// -1e9 additive mask gives the same result for any row with >= 1 unmasked key).
//
// Per CTA: w0 TMA producer, w1 MMA issuer, one softmax warpgroup per tile
// (one TMEM lane = one query row per thread). TMEM: per tile an S/P
// region of 64 fp32 columns (P is written back over S as packed 16-bit pairs and
// fed to the PV MMA straight from TMEM) and an O region of D+16 columns.
// Online softmax in the exp2 domain (Q carries scale*log2(e) and the bias log2(e),
// both folded in by the projection stage) with lazy rescaling (O is only rescaled
// when the running max grows by more than 2^8). The per-element work runs on f16
// pairs: S + bias is rounded to f16 (relative error 2^-11, well below the 2^-8
// rounding the 16-bit Q and K already put into S), the row max is a pairwise tree,
// and P = ex2.approx.f16x2(x - m) is written back to TMEM as the f16 A operand of
// the PV MMA; V^T and the mask row are f16 for that MMA.
//
// Cost model (measured on B200): one tcgen05.mma with M=128, K=16 occupies the
// tensor core for about 150 cycles whatever N is up to N=128, so at D=32 this
// kernel is bound by the number of MMA instructions (QK^T: D/16 per key block,
// PV: BK/16 per key block), not by FLOPs or by the exponentials.
#include "sm100.cuh"

namespace tops {

template <int D, int TR, int TQ, bool BF32 = false>
struct AttnCfg {
  static constexpr int NT = TR * TQ;            // tiles (128 queries x 1 row) per CTA
  static constexpr int NWG = NT;                // softmax warpgroups (one tile each)
  static constexpr int TPW = NT / NWG;          // tiles per warpgroup
  static constexpr int BK = 64;                 // keys per block
  static constexpr int NS = BF32 ? 2 : 3;       // pipeline stages
  static constexpr int NPV = D + 16;            // PV N: D value columns + mask row + zero pad
  static constexpr int Q_BYTES = 128 * D * 2;
  static constexpr int K_BYTES = BK * D * 2;
  static constexpr int V_BYTES = NPV * 128;     // NPV rows x 64 keys (128 B, SW128)
  static constexpr int B_BYTES = 128 * BK * (BF32 ? 4 : 2);  // bias tile (SW128; fp32: two 32-key boxes)
  static constexpr int STAGE = TR * (K_BYTES + V_BYTES) + TQ * B_BYTES;
  static constexpr int STAGE_TX = TR * (K_BYTES + D * 128 + 128) + TQ * B_BYTES;
  static constexpr uint32_t QK_SW = D == 32 ? kSw64 : kSw32;
  static constexpr uint32_t QK_SBO = 8 * D * 2;  // 8 rows x row bytes
  static constexpr int S_COL = 0;               // S/P of tile t at t*64
  static constexpr int O_COL = 256;             // O of tile t at 256 + t*NPV
  static_assert(NT <= 4 && NT * NPV <= 256, "TMEM budget");
  static_assert(NT % NWG == 0, "tiles per warpgroup");
};

struct AttnArgs {
  int R, Nq, Nk;
  void* out;  // [R][Nq][H*D]
  int H;
};

template <int D, int TR, int TQ, bool BF32>
struct AttnSmem {
  using Cfg = AttnCfg<D, TR, TQ, BF32>;
  alignas(1024) uint8_t q[Cfg::NT][Cfg::Q_BYTES];
  alignas(1024) uint8_t stage[Cfg::NS][Cfg::STAGE];
  uint64_t bar_q;
  uint64_t kv_full[Cfg::NS];
  uint64_t kv_empty[Cfg::NS];
  uint64_t s_full[Cfg::NT];
  uint64_t p_full[Cfg::NT];
  uint64_t o_full[Cfg::NT];
  uint32_t tmem_base;
  int abort;
};

template <typename T, int D, int TR, int TQ, bool BF32>
__global__ void __launch_bounds__(128 + 128 * AttnCfg<D, TR, TQ, BF32>::NWG, 1)
    attn_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_m,
                const __grid_constant__ CUtensorMap map_b, AttnArgs a) {
  using Cfg = AttnCfg<D, TR, TQ, BF32>;
  using E = Elem<T>;
  extern __shared__ uint8_t smem_raw[];
  auto& sm = *reinterpret_cast<AttnSmem<D, TR, TQ, BF32>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.z;
  const int row0 = blockIdx.y * TR;
  const int q0 = blockIdx.x * (128 * TQ);
  const int nkb = (a.Nk + Cfg::BK - 1) / Cfg::BK;
  const int H = a.H;

  // zero the padding rows (D+1 .. NPV-1) of every V^T operand tile once
  for (int idx = threadIdx.x; idx < Cfg::NS * TR * 15 * 32; idx += blockDim.x) {
    const int w4 = idx & 31, rowp = (idx >> 5) % 15, rs = idx / (15 * 32);
    const int s = rs / TR, r = rs % TR;
    uint32_t* v = reinterpret_cast<uint32_t*>(sm.stage[s] + r * (Cfg::K_BYTES + Cfg::V_BYTES) + Cfg::K_BYTES);
    v[(D + 1 + rowp) * 32 + w4] = 0u;
  }
  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_q, 1);
    for (int s = 0; s < Cfg::NS; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int t = 0; t < Cfg::NT; ++t) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.p_full[t], 4);
      mbar_init(&sm.o_full[t], 1);
    }
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&sm.tmem_base, 512);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;
  volatile int* abort = &sm.abort;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      tma_prefetch_desc(&map_q);
      tma_prefetch_desc(&map_k);
      tma_prefetch_desc(&map_v);
      tma_prefetch_desc(&map_m);
      tma_prefetch_desc(&map_b);
      mbar_expect_tx(&sm.bar_q, Cfg::NT * Cfg::Q_BYTES);
      for (int t = 0; t < Cfg::NT; ++t)
        tma_load_3d(sm.q[t], &map_q, &sm.bar_q, 0, q0 + (t % TQ) * 128, (row0 + t / TQ) * H + h);
      for (int j = 0; j < nkb; ++j) {
        const int s = j % Cfg::NS;
        if (!mbar_wait(&sm.kv_empty[s], ((j / Cfg::NS) & 1) ^ 1, abort, 201)) break;
        mbar_expect_tx(&sm.kv_full[s], Cfg::STAGE_TX);
        const int k0 = j * Cfg::BK;
        for (int r = 0; r < TR; ++r) {
          uint8_t* kt = sm.stage[s] + r * (Cfg::K_BYTES + Cfg::V_BYTES);
          const int rh = (row0 + r) * H + h;
          tma_load_3d(kt, &map_k, &sm.kv_full[s], 0, k0, rh);
          tma_load_3d(kt + Cfg::K_BYTES, &map_v, &sm.kv_full[s], k0, 0, rh);
          tma_load_2d(kt + Cfg::K_BYTES + D * 128, &map_m, &sm.kv_full[s], k0, row0 + r);
        }
        for (int qb = 0; qb < TQ; ++qb) {
          uint8_t* bt = sm.stage[s] + TR * (Cfg::K_BYTES + Cfg::V_BYTES) + qb * Cfg::B_BYTES;
          tma_load_3d(bt, &map_b, &sm.kv_full[s], k0, q0 + qb * 128, h);
          if (BF32) tma_load_3d(bt + 16384, &map_b, &sm.kv_full[s], k0 + 32, q0 + qb * 128, h);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc_qk = make_idesc_f16(128, Cfg::BK, E::kFmt, false, false);
      // P (ex2 output) and V^T are f16 whatever the IO dtype.
      const uint32_t idesc_pv = make_idesc_f16(128, Cfg::NPV, 0, false, false);
      bool ok = mbar_wait(&sm.bar_q, 0, abort, 202);
      auto issue_pv = [&](int t, int j) {
        const uint8_t* vt = sm.stage[j % Cfg::NS] + (t / TQ) * (Cfg::K_BYTES + Cfg::V_BYTES) + Cfg::K_BYTES;
        const uint32_t vb = smem_u32(vt);
        const uint32_t p_tmem = tbase + Cfg::S_COL + t * 64;
        const uint32_t o_tmem = tbase + Cfg::O_COL + t * Cfg::NPV;
#pragma unroll
        for (int kk = 0; kk < Cfg::BK / 16; ++kk)
          mma_ts(o_tmem, p_tmem + kk * 8, make_smem_desc(vb + kk * 32, 16, 1024, kSw128), idesc_pv, j > 0 || kk > 0);
      };
      for (int j = 0; ok && j < nkb; ++j) {
        const int s = j % Cfg::NS;
        if (!mbar_wait(&sm.kv_full[s], (j / Cfg::NS) & 1, abort, 203)) break;
        tc_fence_after();
        for (int t = 0; t < Cfg::NT; ++t) {
          if (j > 0) {
            if (!mbar_wait(&sm.p_full[t], (j - 1) & 1, abort, 204)) { ok = false; break; }
            tc_fence_after();
            issue_pv(t, j - 1);
          }
          const uint32_t qa = smem_u32(sm.q[t]);
          const uint32_t ka = smem_u32(sm.stage[s] + (t / TQ) * (Cfg::K_BYTES + Cfg::V_BYTES));
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_ss(tbase + Cfg::S_COL + t * 64, make_smem_desc(qa + kk * 32, 16, Cfg::QK_SBO, Cfg::QK_SW),
                   make_smem_desc(ka + kk * 32, 16, Cfg::QK_SBO, Cfg::QK_SW), idesc_qk, kk > 0);
          mma_commit(&sm.s_full[t]);
        }
        if (ok && j > 0) mma_commit(&sm.kv_empty[(j - 1) % Cfg::NS]);
      }
      if (ok) {
        for (int t = 0; t < Cfg::NT; ++t) {
          if (!mbar_wait(&sm.p_full[t], (nkb - 1) & 1, abort, 205)) break;
          tc_fence_after();
          issue_pv(t, nkb - 1);
          mma_commit(&sm.o_full[t]);
        }
        mma_commit(&sm.kv_empty[(nkb - 1) % Cfg::NS]);
      }
    }
  } else if (warp >= 4) {
    // ---------------- softmax warpgroups ----------------
    const int wg = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int qrow = wq * 32 + lane;  // TMEM lane == query row within the tile
    const uint32_t lane_addr = tbase + (static_cast<uint32_t>(wq * 32) << 16);
    float ms[Cfg::TPW];
#pragma unroll
    for (int u = 0; u < Cfg::TPW; ++u) ms[u] = 0.f;
    bool ok = true;
    for (int j = 0; ok && j < nkb; ++j) {
      const int s = j % Cfg::NS;
#pragma unroll
      for (int u = 0; u < Cfg::TPW; ++u) {
        const int t = wg * Cfg::TPW + u;
        const int qb = t % TQ;
        if (!mbar_wait(&sm.s_full[t], j & 1, abort, 206)) { ok = false; break; }
        tc_fence_after();
        const uint8_t* brow = sm.stage[s] + TR * (Cfg::K_BYTES + Cfg::V_BYTES) + qb * Cfg::B_BYTES;
        // x = S + bias (log2 units), packed to f16 pairs: the rest of the softmax runs
        // two lanes per instruction. S is read in two 32-column halves.
        __half2 xh[32];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t sv[32];
          tmem_ld32(lane_addr + Cfg::S_COL + t * 64 + half * 32, sv);
          if (BF32) {
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
              const float4 bf = *reinterpret_cast<const float4*>(brow + half * 16384 + sw128_off(qrow, ch));
              xh[half * 16 + ch * 2] = __floats2half2_rn(__uint_as_float(sv[ch * 4]) + bf.x,
                                                          __uint_as_float(sv[ch * 4 + 1]) + bf.y);
              xh[half * 16 + ch * 2 + 1] = __floats2half2_rn(__uint_as_float(sv[ch * 4 + 2]) + bf.z,
                                                              __uint_as_float(sv[ch * 4 + 3]) + bf.w);
            }
          } else {
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
              const int ch = half * 4 + cc;
              const uint4 bu = *reinterpret_cast<const uint4*>(brow + sw128_off(qrow, ch));
              const uint32_t b4[4] = {bu.x, bu.y, bu.z, bu.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int c = cc * 8 + 2 * e;
                xh[half * 16 + cc * 4 + e] =
                    __hadd2(__floats2half2_rn(__uint_as_float(sv[c]), __uint_as_float(sv[c + 1])),
                            *reinterpret_cast<const __half2*>(&b4[e]));
              }
            }
          }
        }
        __half2 mt[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) mt[c] = __hmax2(xh[2 * c], xh[2 * c + 1]);
#pragma unroll
        for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
          for (int c = 0; c < w; ++c) mt[c] = __hmax2(mt[c], mt[c + w]);
        const float mx = fmaxf(__low2float(mt[0]), __high2float(mt[0]));
        float m_use = ms[u];
        if (j == 0) {
          m_use = mx;
        } else {
          const bool need = mx > m_use + 8.0f;
          if (__any_sync(0xffffffffu, need)) {
            const float alpha = need ? ex2_approx(m_use - mx) : 1.0f;
            if (need) m_use = mx;
            uint32_t o[Cfg::NPV];
            const uint32_t oaddr = lane_addr + Cfg::O_COL + t * Cfg::NPV;
            if (D == 32) {
              tmem_ld32(oaddr, o);
              tmem_ld16(oaddr + 32, o + 32);
            } else {
              tmem_ld32(oaddr, o);
            }
#pragma unroll
            for (int c = 0; c < Cfg::NPV; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
            if (D == 32) {
              tmem_st32(oaddr, o);
              tmem_st16(oaddr + 32, o + 32);
            } else {
              tmem_st32(oaddr, o);
            }
          }
        }
        ms[u] = m_use;
        const __half2 mh = __float2half2_rn(m_use);  // exact: m_use is an f16 value
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const __half2 p = h2exp2(__hsub2(xh[c], mh));
          pk[c] = *reinterpret_cast<const uint32_t*>(&p);
        }
        tmem_st32(lane_addr + Cfg::S_COL + t * 64, pk);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full[t]);
      }
    }
    // ---------------- epilogue: O / l -> out ----------------
#pragma unroll
    for (int u = 0; u < Cfg::TPW; ++u) {
      const int t = wg * Cfg::TPW + u;
      const bool got = ok && mbar_wait(&sm.o_full[t], 0, abort, 207);
      tc_fence_after();
      uint32_t o[Cfg::NPV];
      const uint32_t oaddr = lane_addr + Cfg::O_COL + t * Cfg::NPV;
      if (D == 32) {
        tmem_ld32(oaddr, o);
        tmem_ld16(oaddr + 32, o + 32);
      } else {
        tmem_ld32(oaddr, o);
      }
      const int ri = row0 + t / TQ;
      const int q = q0 + (t % TQ) * 128 + qrow;
      if (got && ri < a.R && q < a.Nq) {
        const float inv = 1.0f / __uint_as_float(o[D]);
        uint32_t pk[D / 2];
#pragma unroll
        for (int c = 0; c < D / 2; ++c)
          pk[c] = E::pack2(__uint_as_float(o[2 * c]) * inv, __uint_as_float(o[2 * c + 1]) * inv);
        uint4* dst = reinterpret_cast<uint4*>(static_cast<T*>(a.out) +
                                              (static_cast<size_t>(ri) * a.Nq + q) * (H * D) + h * D);
#pragma unroll
        for (int c = 0; c < D / 8; ++c) dst[c] = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

}  // namespace tops
