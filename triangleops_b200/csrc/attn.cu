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
// Cost model (measured on B200): a tcgen05.mma with M=128, K=16 keeps its issuing
// thread busy for ~140 cycles whatever N is (up to N=128), while the tensor core
// itself can absorb a new small MMA every ~50 cycles when several warps issue. At
// D=32 the work per key block is many small MMAs (QK^T: D/16, PV: BK/16), so each
// tile has its OWN issuing warp: the tiles' MMA streams overlap in the tensor core.
//
// Per CTA: w0 TMA producer (K, V^T, mask row, bias tile per 64-key block into a ring
// of stages), w(1+t) MMA issuer of tile t, one softmax warpgroup per tile (one TMEM
// lane = one query row per thread). TMEM per tile: S (64 fp32 columns), P (32
// columns of packed f16 pairs, the A operand of PV) and O (D+16 columns). The
// softmax releases S as soon as it has loaded it, so QK^T(j+1) runs while the
// exponentials of block j are computed; P(j+1) is written once PV(j) has read P(j).
//
// Online softmax in the exp2 domain (Q carries scale*log2(e) and the bias log2(e),
// both folded in upstream) with lazy rescaling (O is only rescaled when the running
// max grows by more than 2^8). The per-element work runs on f16 pairs: S + bias is
// rounded to f16 (relative error 2^-11, well below the 2^-8 rounding the 16-bit Q
// and K already put into S), the row max is a pairwise tree, and
// P = ex2.approx.f16x2(x - m); V^T and the mask row are f16 for the PV MMA.
#include "sm100.cuh"

namespace tops {

// Optional phase timers (build with -DTOPS_TRACE): per-role cycle sums, read back
// with tops_attn_trace(). Compiled out of the library by default.
#ifdef TOPS_TRACE
__device__ unsigned long long g_attn_trace[16];
#define TOPS_TCLK(v) const long long v = clock64()
#define TOPS_TADD(i, a, b) tr_acc[i] += static_cast<unsigned long long>((b) - (a))
#define TOPS_TFLUSH()                                                              \
  for (int i_ = 0; i_ < 8; ++i_)                                                   \
    if (tr_acc[i_]) atomicAdd(&g_attn_trace[i_], tr_acc[i_])
#define TOPS_TDECL() unsigned long long tr_acc[8] = {0, 0, 0, 0, 0, 0, 0, 0}
#else
#define TOPS_TFLUSH()
#define TOPS_TDECL()
#define TOPS_TCLK(v)
#define TOPS_TADD(i, a, b)
#endif

template <int D, int TR, int TQ, bool BF32 = false>
struct AttnCfg {
  static constexpr int NT = TR * TQ;            // tiles (128 queries x 1 row) per CTA
  static constexpr int BK = 64;                 // keys per block
  static constexpr int NPV = D + 16;            // PV N: D value columns + mask row + zero pad
  static constexpr int Q_BYTES = 128 * D * 2;
  static constexpr int K_BYTES = BK * D * 2;
  static constexpr int V_BYTES = NPV * 128;     // NPV rows x 64 keys (128 B, SW128)
  static constexpr int B_BYTES = 128 * BK * (BF32 ? 4 : 2);  // bias tile (SW128; fp32: two 32-key boxes)
  static constexpr int STAGE = TQ * B_BYTES + TR * (K_BYTES + V_BYTES);
  static constexpr int STAGE_TX = TQ * B_BYTES + TR * (K_BYTES + D * 128 + 128);
  static constexpr int NS_FIT = (200 * 1024 - NT * Q_BYTES) / STAGE;
  static constexpr int NS = NS_FIT > 4 ? 4 : NS_FIT;  // pipeline stages
  static constexpr uint32_t QK_SW = D == 32 ? kSw64 : kSw32;
  static constexpr uint32_t QK_SBO = 8 * D * 2;  // 8 rows x row bytes
  static constexpr int S_COL = 0;               // S of tile t at t*64
  static constexpr int P_COL = 192;             // P of tile t at 192 + t*32
  static constexpr int O_COL = 288;             // O of tile t at 288 + t*NPV
  static_assert(NT <= 3 && O_COL + NT * NPV <= 512, "TMEM budget");
  static_assert(NS >= 2, "pipeline depth");
  static_assert(STAGE % 1024 == 0 && (K_BYTES + V_BYTES) % 1024 == 0, "alignment");
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
  uint64_t kv_empty[Cfg::NS];  // one commit per tile issuer
  uint64_t s_full[Cfg::NT];    // QK^T of the block landed in S
  uint64_t s_free[Cfg::NT];    // the softmax has loaded S (it may be overwritten)
  uint64_t p_full[Cfg::NT];    // P of the block written
  uint64_t pv_done[Cfg::NT];   // PV of the block finished (P reusable, O stable)
  uint64_t o_full[Cfg::NT];    // the last PV finished
  uint32_t tmem_base;
  int abort;
};

template <typename T, int D, int TR, int TQ, bool BF32>
__global__ void __launch_bounds__(128 + 128 * AttnCfg<D, TR, TQ, BF32>::NT, 1)
    attn_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_m,
                const __grid_constant__ CUtensorMap map_b, AttnArgs a) {
  using Cfg = AttnCfg<D, TR, TQ, BF32>;
  using E = Elem<T>;
  constexpr int NS = Cfg::NS, NT = Cfg::NT, BK = Cfg::BK;
  extern __shared__ uint8_t smem_raw[];
  auto& sm = *reinterpret_cast<AttnSmem<D, TR, TQ, BF32>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                            ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.z;
  const int row0 = blockIdx.y * TR;
  const int q0 = blockIdx.x * (128 * TQ);
  const int nkb = (a.Nk + BK - 1) / BK;
  const int H = a.H;
  TOPS_TDECL();
  auto kv_tile = [&](int s, int r) { return sm.stage[s] + TQ * Cfg::B_BYTES + r * (Cfg::K_BYTES + Cfg::V_BYTES); };

  // zero the padding rows (D+1 .. NPV-1) of every V^T operand tile once (32 words per 128 B row)
  for (int idx = threadIdx.x; idx < NS * TR * 15 * 32; idx += blockDim.x) {
    const int w = idx & 31, rowp = (idx >> 5) % 15, rs = idx / (15 * 32);
    uint32_t* v = reinterpret_cast<uint32_t*>(kv_tile(rs / TR, rs % TR) + Cfg::K_BYTES);
    v[(D + 1 + rowp) * 32 + w] = 0u;
  }
  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_q, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], NT);
    }
    for (int t = 0; t < NT; ++t) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.s_free[t], 4);
      mbar_init(&sm.p_full[t], 4);
      mbar_init(&sm.pv_done[t], 1);
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
      mbar_expect_tx(&sm.bar_q, NT * Cfg::Q_BYTES);
      for (int t = 0; t < NT; ++t)
        tma_load_3d(sm.q[t], &map_q, &sm.bar_q, 0, q0 + (t % TQ) * 128, (row0 + t / TQ) * H + h);
      for (int j = 0; j < nkb; ++j) {
        const int s = j % NS;
        TOPS_TCLK(te0);
        if (!mbar_wait(&sm.kv_empty[s], ((j / NS) & 1) ^ 1, abort, 201)) break;
        TOPS_TCLK(te1);
        TOPS_TADD(7, te0, te1);
        mbar_expect_tx(&sm.kv_full[s], Cfg::STAGE_TX);
        const int k0 = j * BK;
        for (int qb = 0; qb < TQ; ++qb) {
          uint8_t* bt = sm.stage[s] + qb * Cfg::B_BYTES;
          tma_load_3d(bt, &map_b, &sm.kv_full[s], k0, q0 + qb * 128, h);
          if (BF32) tma_load_3d(bt + 16384, &map_b, &sm.kv_full[s], k0 + 32, q0 + qb * 128, h);
        }
        for (int r = 0; r < TR; ++r) {
          uint8_t* kt = kv_tile(s, r);
          const int rh = (row0 + r) * H + h;
          tma_load_3d(kt, &map_k, &sm.kv_full[s], 0, k0, rh);
          tma_load_3d(kt + Cfg::K_BYTES, &map_v, &sm.kv_full[s], k0, 0, rh);
          tma_load_2d(kt + Cfg::K_BYTES + D * 128, &map_m, &sm.kv_full[s], k0, row0 + r);
        }
      }
    }
  } else if (warp <= NT) {
    if (lane == 0) {
      // ---------------- MMA issuer of tile t ----------------
      const int t = warp - 1;
      const uint32_t idesc_qk = make_idesc_f16(128, BK, 0, false, false);  // Q, K are f16
      // P (ex2 output) and V^T are f16 whatever the IO dtype.
      const uint32_t idesc_pv = make_idesc_f16(128, Cfg::NPV, 0, false, false);
      const uint32_t qa = smem_u32(sm.q[t]);
      const uint32_t s_tmem = tbase + Cfg::S_COL + t * 64;
      const uint32_t p_tmem = tbase + Cfg::P_COL + t * 32;
      const uint32_t o_tmem = tbase + Cfg::O_COL + t * Cfg::NPV;
      auto issue_pv = [&](int jp) {
        const uint32_t vb = smem_u32(kv_tile(jp % NS, t / TQ) + Cfg::K_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          mma_ts(o_tmem, p_tmem + kk * 8, make_smem_desc(vb + kk * 32, 16, 1024, kSw128), idesc_pv, jp > 0 || kk > 0);
        mma_commit(&sm.pv_done[t]);
        if (jp == nkb - 1) mma_commit(&sm.o_full[t]);
        mma_commit(&sm.kv_empty[jp % NS]);
      };
      bool ok = mbar_wait(&sm.bar_q, 0, abort, 202);
      for (int j = 0; ok && j < nkb; ++j) {
        const int s = j % NS;
        TOPS_TCLK(tk0);
        if (!mbar_wait(&sm.kv_full[s], (j / NS) & 1, abort, 203)) break;
        if (j > 0 && !mbar_wait(&sm.s_free[t], (j - 1) & 1, abort, 204)) break;
        TOPS_TCLK(tk1);
        TOPS_TADD(4, tk0, tk1);
        tc_fence_after();
        const uint32_t ka = smem_u32(kv_tile(s, t / TQ));
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_ss(s_tmem, make_smem_desc(qa + kk * 32, 16, Cfg::QK_SBO, Cfg::QK_SW),
                 make_smem_desc(ka + kk * 32, 16, Cfg::QK_SBO, Cfg::QK_SW), idesc_qk, kk > 0);
        mma_commit(&sm.s_full[t]);
        if (j > 0) {
          TOPS_TCLK(tp0);
          if (!mbar_wait(&sm.p_full[t], (j - 1) & 1, abort, 205)) break;
          TOPS_TCLK(tp1);
          TOPS_TADD(5, tp0, tp1);
          tc_fence_after();
          issue_pv(j - 1);
        }
        if (j == nkb - 1) {
          if (!mbar_wait(&sm.p_full[t], j & 1, abort, 205)) break;
          tc_fence_after();
          issue_pv(j);
        }
      }
    }
  } else if (warp >= 4) {
    // ---------------- softmax warpgroups (one tile each) ----------------
    const int t = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int qrow = wq * 32 + lane;  // TMEM lane == query row within the tile
    const int qb = t % TQ;
    const uint32_t lane_addr = tbase + (static_cast<uint32_t>(wq * 32) << 16);
    const uint32_t oaddr = lane_addr + Cfg::O_COL + t * Cfg::NPV;
    float m_use = 0.f;
    bool ok = true;
    for (int j = 0; ok && j < nkb; ++j) {
      const int s = j % NS;
      TOPS_TCLK(ts0);
      if (!mbar_wait(&sm.s_full[t], j & 1, abort, 206)) { ok = false; break; }
      if (!mbar_wait(&sm.kv_full[s], (j / NS) & 1, abort, 210)) { ok = false; break; }  // bias tile visible
      TOPS_TCLK(ts1);
      tc_fence_after();
      const uint8_t* brow = sm.stage[s] + qb * Cfg::B_BYTES;
      // x = S + bias (log2 units), packed to f16 pairs. S is read in two 32-column halves.
      __half2 xh[32];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t sv[32];
        tmem_ld32(lane_addr + Cfg::S_COL + t * 64 + half * 32, sv);
        if (BF32) {
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            const float4 bf = *reinterpret_cast<const float4*>(brow + half * 16384 + sw128_off(qrow, ch));
            xh[half * 16 + ch * 2] =
                __floats2half2_rn(__uint_as_float(sv[ch * 4]) + bf.x, __uint_as_float(sv[ch * 4 + 1]) + bf.y);
            xh[half * 16 + ch * 2 + 1] =
                __floats2half2_rn(__uint_as_float(sv[ch * 4 + 2]) + bf.z, __uint_as_float(sv[ch * 4 + 3]) + bf.w);
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
              xh[half * 16 + cc * 4 + e] = __hadd2(__floats2half2_rn(__uint_as_float(sv[c]), __uint_as_float(sv[c + 1])),
                                                   *reinterpret_cast<const __half2*>(&b4[e]));
            }
          }
        }
      }
      // S consumed: QK^T of the next block may overwrite it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.s_free[t]);
      TOPS_TCLK(ts2);
      __half2 mt[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) mt[c] = __hmax2(xh[2 * c], xh[2 * c + 1]);
#pragma unroll
      for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
        for (int c = 0; c < w; ++c) mt[c] = __hmax2(mt[c], mt[c + w]);
      const float mx = fmaxf(__low2float(mt[0]), __high2float(mt[0]));
      // P(j) overwrites P(j-1), and an O rescale needs O stable: both need PV(j-1) done.
      // The softmax of block j-1 already waited for PV(j-2), so pv_done is at most one
      // phase behind and the parity wait is exact.
      bool waited = false;
      if (j == 0) {
        m_use = mx;
      } else {
        const bool need = mx > m_use + 8.0f;
        if (__any_sync(0xffffffffu, need)) {
          if (!mbar_wait(&sm.pv_done[t], (j - 1) & 1, abort, 208)) { ok = false; break; }
          waited = true;
          tc_fence_after();
          const float alpha = need ? ex2_approx(m_use - mx) : 1.0f;
          if (need) m_use = mx;
          uint32_t o[Cfg::NPV];
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
      const __half2 mh = __float2half2_rn(m_use);  // exact: m_use is an f16 value
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const __half2 d = __hsub2(xh[c], mh);
        pk[c] = ex2_f16x2(*reinterpret_cast<const uint32_t*>(&d));
      }
      TOPS_TCLK(ts3);
      if (j > 0 && !waited) {
        if (!mbar_wait(&sm.pv_done[t], (j - 1) & 1, abort, 209)) { ok = false; break; }
        tc_fence_after();
      }
      tmem_st32(lane_addr + Cfg::P_COL + t * 32, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full[t]);
      TOPS_TCLK(ts4);
      if (lane == 0) {
        TOPS_TADD(0, ts0, ts1);
        TOPS_TADD(1, ts1, ts2);
        TOPS_TADD(2, ts2, ts3);
        TOPS_TADD(3, ts3, ts4);
      }
    }
    // ---------------- epilogue: O / l -> out ----------------
    const bool got = ok && mbar_wait(&sm.o_full[t], 0, abort, 207);
    tc_fence_after();
    uint32_t o[Cfg::NPV];
    if (D == 32) {
      tmem_ld32(oaddr, o);
      tmem_ld16(oaddr + 32, o + 32);
    } else {
      tmem_ld32(oaddr, o);
    }
    const int ri = row0 + t / TQ;
    const int q = q0 + qb * 128 + qrow;
    if (got && ri < a.R && q < a.Nq) {
      const float inv = 1.0f / __uint_as_float(o[D]);
      uint32_t pk[D / 2];
#pragma unroll
      for (int c = 0; c < D / 2; ++c)
        pk[c] = E::pack2(__uint_as_float(o[2 * c]) * inv, __uint_as_float(o[2 * c + 1]) * inv);
      uint4* dst =
          reinterpret_cast<uint4*>(static_cast<T*>(a.out) + (static_cast<size_t>(ri) * a.Nq + q) * (H * D) + h * D);
#pragma unroll
      for (int c = 0; c < D / 8; ++c) dst[c] = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
    }
  }
  TOPS_TFLUSH();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

}  // namespace tops
