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
// Bias without per-element work (f16 bias, triangle attention): the tensor core adds
// it — S = bias x I + Q K^T, with I the 64 x 64 identity in shared memory (products
// and sums exact in the fp32 accumulator) — so the softmax reads S ready-biased.
// The fp32 bias of the pair-bias attention is added by the softmax.
//
// Cost model (measured on B200): a tcgen05.mma with M=128, K=16 keeps its issuing
// thread busy for ~140 cycles whatever N is (up to N=128), while the tensor core
// itself can absorb a new small MMA every ~50 cycles when several warps issue. At
// D=32 the work per key block is many small MMAs (QK^T: D/16, PV: BK/16), so each
// tile has its OWN issuing threads (one for QK^T, one for PV): the MMA streams overlap
// in the tensor core.
//
// Per CTA: w0 TMA producer (per 64-key block: bias and K tiles into ring A, V^T and
// mask rows into ring B), w(1+t) QK^T and w(1+NT+t) PV issuer of tile t, one softmax
// warpgroup per tile (one TMEM
// lane = one query row per thread). TMEM per tile: S (64 fp32 columns), P (32
// columns of packed f16 pairs, the A operand of PV) and O (D+16 columns). The
// softmax releases S as soon as it has loaded it, so QK^T(j+1) runs while the
// exponentials of block j are computed; P(j+1) is written once PV(j) has read P(j).
//
// Online softmax in the exp2 domain (Q carries scale*log2(e) and the bias log2(e),
// both folded in upstream) with lazy rescaling (O is only rescaled when the running
// max grows by more than 2^8). The per-element work runs on f16 pairs: with the f16
// bias the tensor core accumulates S = bias x I + Q K^T in f16 (the bias terms are
// exact, each of the D/16 Q K^T steps rounds once, relative error 2^-11 each, below
// the 2^-8 rounding the 16-bit Q and K already put into S) and the softmax loads it
// as packed pairs (tcgen05.ld .pack::16b: no conversion); the fp32 bias path rounds
// S + bias to f16 pairs itself. The row max is a pairwise tree, and
// P = 2^(x - m), 2/3 of the pairs on the MUFU (ex2.approx.f16x2, which issues twice
// on the XU pipe) and 1/3 by a polynomial on the FMA pipe (ex2_poly_f16x2), so that
// neither pipe alone bounds the step; V^T and the mask row are f16 for the PV MMA.
#include "sm100.cuh"

namespace tops {

#ifndef TOPS_POLY_EXP
#define TOPS_POLY_EXP 1
#endif
constexpr bool kPolyExp = TOPS_POLY_EXP != 0;
#ifndef TOPS_POLY_PICK
#define TOPS_POLY_PICK(c) ((c) % 3 == 1)  // pairs whose 2^x takes the polynomial (11 of 32)
#endif
#ifndef TOPS_S_F16
#define TOPS_S_F16 1  // f16 bias path: S accumulated in f16 by the tensor core, loaded packed
#endif
#ifndef TOPS_ATTN_SMEM_KB
#define TOPS_ATTN_SMEM_KB 200  // operand budget (Q tiles + stages); the B200 allows 227 KB per CTA
#endif

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
  // warps: 0 TMA producer, 1..NT QK^T issuers, NT+1..2NT PV issuers, then one softmax
  // warpgroup per tile (any 4 consecutive warps cover the 4 TMEM lane quarters)
  static constexpr int SM_WARP0 = 1 + 2 * NT;
  static constexpr int THREADS = 32 * SM_WARP0 + 128 * NT;
  static constexpr int BK = 64;                 // keys per block
  static constexpr int NPV = D + 16;            // PV N: D value columns + mask row + zero pad
  static constexpr int Q_BYTES = 128 * D * 2;
  static constexpr int K_BYTES = BK * D * 2;
  static constexpr int V_BYTES = NPV * 128;     // NPV rows x 64 keys (128 B, SW128)
  static constexpr int B_BYTES = 128 * BK * (BF32 ? 4 : 2);  // bias tile (SW128; fp32: two 32-key boxes)
  // Two operand rings, released at different times: ring A (bias tiles + K tiles) is
  // free once QK^T has run and the softmax has read the bias, ring B (V^T with its
  // mask row) once PV has run — a block later. Separate rings let the next blocks'
  // K and bias stream in without waiting for the slower PV release.
  static constexpr int A_BYTES = TQ * B_BYTES + TR * K_BYTES;
  static constexpr int VB_BYTES = TR * V_BYTES;
  static constexpr int VB_TX = TR * (D * 128 + 128);
  static constexpr int BUDGET = TOPS_ATTN_SMEM_KB * 1024 - NT * Q_BYTES - (BF32 ? 1024 : BK * 128);
  static constexpr int NB = 4;
  static constexpr int NA_FIT = (BUDGET - NB * VB_BYTES) / A_BYTES;
  static constexpr int NA = NA_FIT > 4 ? 4 : NA_FIT;
  static constexpr uint32_t QK_SW = D == 32 ? kSw64 : kSw32;
  static constexpr uint32_t QK_SBO = 8 * D * 2;  // 8 rows x row bytes
  static constexpr int S_COL = 0;               // S of tile t at t*64
  static constexpr int P_COL = 192;             // P of tile t at 192 + t*32
  static constexpr int O_COL = 288;             // O of tile t at 288 + t*NPV
  static_assert(NT <= 3 && O_COL + NT * NPV <= 512, "TMEM budget");
  static_assert(NA >= 2, "pipeline depth");
  static_assert(A_BYTES % 1024 == 0 && V_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "alignment");
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
  alignas(1024) uint8_t ident[BF32 ? 1024 : Cfg::BK * 128];  // f16 identity (BK x BK, K-major SW128)
  alignas(1024) uint8_t ring_a[Cfg::NA][Cfg::A_BYTES];
  alignas(1024) uint8_t ring_b[Cfg::NB][Cfg::VB_BYTES];
  uint64_t bar_q;
  uint64_t q_empty;            // one commit per tile issuer (after the unit's last QK^T)
  uint64_t a_full[Cfg::NA];
  uint64_t a_empty[Cfg::NA];   // one commit per tile issuer (after QK^T and the softmax's bias read)
  uint64_t b_full[Cfg::NB];
  uint64_t b_empty[Cfg::NB];   // one commit per tile issuer (after PV)
  uint64_t s_full[Cfg::NT];    // QK^T of the block landed in S
  uint64_t s_free[Cfg::NT];    // the softmax has loaded S (it may be overwritten)
  uint64_t p_full[Cfg::NT];    // P of the block written
  uint64_t pv_done[Cfg::NT];   // PV of the block finished (P reusable, O stable)
  uint64_t o_full[Cfg::NT];    // the last PV of the unit finished
  uint64_t o_empty[Cfg::NT];   // the epilogue has read O (the next unit may overwrite it)
  uint32_t tmem_base;
  int abort;
#ifdef TOPS_TRACE
  long long t_qk[Cfg::NT];
#endif
};

template <typename T, int D, int TR, int TQ, bool BF32>
__global__ void __launch_bounds__(AttnCfg<D, TR, TQ, BF32>::THREADS, 1)
    attn_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_m,
                const __grid_constant__ CUtensorMap map_b, AttnArgs a) {
  using Cfg = AttnCfg<D, TR, TQ, BF32>;
  using E = Elem<T>;
  constexpr int NA = Cfg::NA, NB = Cfg::NB, NT = Cfg::NT, BK = Cfg::BK;
  extern __shared__ uint8_t smem_raw[];
  auto& sm = *reinterpret_cast<AttnSmem<D, TR, TQ, BF32>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                            ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = (a.Nk + BK - 1) / BK;
  const int H = a.H;
  TOPS_TDECL();
  auto k_tile = [&](int s, int r) { return sm.ring_a[s] + TQ * Cfg::B_BYTES + r * Cfg::K_BYTES; };
  auto v_tile = [&](int s, int r) { return sm.ring_b[s] + r * Cfg::V_BYTES; };
  constexpr int PAD_ROWS = Cfg::NPV - D - 1;

  // zero the padding rows (D+1 .. NPV-1) of every V^T operand tile once (32 words per 128 B row)
  for (int idx = threadIdx.x; idx < NB * TR * PAD_ROWS * 32; idx += blockDim.x) {
    const int w = idx & 31, rowp = (idx >> 5) % PAD_ROWS, rs = idx / (PAD_ROWS * 32);
    uint32_t* v = reinterpret_cast<uint32_t*>(v_tile(rs / TR, rs % TR));
    v[(D + 1 + rowp) * 32 + w] = 0u;
  }
  if (!BF32) {
    // identity: element (n, k) of the BK x BK K-major SW128 tile at n*128 + ((k/8 ^ n%8) * 16) + (k%8)*2
    for (int w = threadIdx.x; w < BK * 32; w += blockDim.x) {
      const int n = w >> 5, c = (w & 31) >> 2, k0 = ((c ^ (n & 7)) << 3) + ((w & 3) << 1);
      reinterpret_cast<uint32_t*>(sm.ident)[w] = (k0 == n ? 0x3C00u : 0u) | (k0 + 1 == n ? 0x3C000000u : 0u);
    }
  }
  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_q, 1);
    mbar_init(&sm.q_empty, NT);
    for (int s = 0; s < NA; ++s) {
      mbar_init(&sm.a_full[s], 1);
      mbar_init(&sm.a_empty[s], NT);
    }
    for (int s = 0; s < NB; ++s) {
      mbar_init(&sm.b_full[s], 1);
      mbar_init(&sm.b_empty[s], NT);
    }
    for (int t = 0; t < NT; ++t) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.s_free[t], 4);
      mbar_init(&sm.p_full[t], 4);
      mbar_init(&sm.pv_done[t], 1);
      mbar_init(&sm.o_full[t], 1);
      mbar_init(&sm.o_empty[t], 4);
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

  // Persistent: CTA b takes work units b, b + gridDim.x, ... A unit is TR rows x TQ
  // 128-query blocks of one head (x fastest: the CTAs running together share the bias
  // tiles of a head and the K/V of a row in L2). Ring slots and barrier phases run on
  // across units (g = blocks processed by this CTA so far, lu = units so far), so the
  // producer streams the next unit's tiles while the current one finishes.
  const int n_qb = (a.Nq + 128 * TQ - 1) / (128 * TQ);
  const int n_rg = (a.R + TR - 1) / TR;
  const int n_units = n_qb * n_rg * a.H;
  auto coords = [&](int u, int& q0, int& row0, int& h) {
    q0 = (u % n_qb) * (128 * TQ);
    const int rest = u / n_qb;
    row0 = (rest % n_rg) * TR;
    h = rest / n_rg;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      tma_prefetch_desc(&map_q);
      tma_prefetch_desc(&map_k);
      tma_prefetch_desc(&map_v);
      tma_prefetch_desc(&map_m);
      tma_prefetch_desc(&map_b);
      bool ok = true;
      int g = 0, lu = 0;
      for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++lu, g += nkb) {
        int q0, row0, h;
        coords(u, q0, row0, h);
        // ring A of block j, then ring B of block j-1 (V is consumed a block after K); the
        // unit's Q tiles after its first ring-A block, once the previous unit's QK^T is done
        for (int j = 0; j <= nkb; ++j) {
          if (j < nkb) {
            const int gg = g + j, s = gg % NA;
            TOPS_TCLK(te0);
            if (!mbar_wait(&sm.a_empty[s], ((gg / NA) & 1) ^ 1, abort, 201)) { ok = false; break; }
            TOPS_TCLK(te1);
            TOPS_TADD(7, te0, te1);
            mbar_expect_tx(&sm.a_full[s], Cfg::A_BYTES);
            const int k0 = j * BK;
            for (int qb = 0; qb < TQ; ++qb) {
              uint8_t* bt = sm.ring_a[s] + qb * Cfg::B_BYTES;
              tma_load_3d(bt, &map_b, &sm.a_full[s], k0, q0 + qb * 128, h);
              if (BF32) tma_load_3d(bt + 16384, &map_b, &sm.a_full[s], k0 + 32, q0 + qb * 128, h);
            }
            for (int r = 0; r < TR; ++r) tma_load_3d(k_tile(s, r), &map_k, &sm.a_full[s], 0, k0, (row0 + r) * H + h);
          }
          if (j == 0) {
            if (!mbar_wait(&sm.q_empty, (lu & 1) ^ 1, abort, 213)) { ok = false; break; }
            mbar_expect_tx(&sm.bar_q, NT * Cfg::Q_BYTES);
            for (int t = 0; t < NT; ++t)
              tma_load_3d(sm.q[t], &map_q, &sm.bar_q, 0, q0 + (t % TQ) * 128, (row0 + t / TQ) * H + h);
          }
          if (j >= 1) {
            const int gb = g + j - 1, s = gb % NB;
            if (!mbar_wait(&sm.b_empty[s], ((gb / NB) & 1) ^ 1, abort, 211)) { ok = false; break; }
            mbar_expect_tx(&sm.b_full[s], Cfg::VB_TX);
            const int k0 = (j - 1) * BK;
            for (int r = 0; r < TR; ++r) {
              uint8_t* vt = v_tile(s, r);
              tma_load_3d(vt, &map_v, &sm.b_full[s], k0, 0, (row0 + r) * H + h);
              tma_load_2d(vt + D * 128, &map_m, &sm.b_full[s], k0, row0 + r);
            }
          }
        }
      }
    }
  } else if (warp <= NT) {
    if (lane == 0) {
      // ---------------- QK^T issuer of tile t ----------------
      const int t = warp - 1;
      // Q, K are f16; S is fp32, or f16 (D format 0) for the f16-bias path with TOPS_S_F16
      const uint32_t idesc_qk =
          make_idesc_f16(128, BK, 0, false, false) & ((!BF32 && TOPS_S_F16) ? ~(3u << 4) : ~0u);
      const uint32_t qa = smem_u32(sm.q[t]);
      const uint32_t s_tmem = tbase + Cfg::S_COL + t * 64;
      bool ok = true;
      int g = 0, lu = 0;
      for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++lu, g += nkb) {
        if (!mbar_wait(&sm.bar_q, lu & 1, abort, 202)) break;
        for (int j = 0; j < nkb; ++j) {
          const int gg = g + j, s = gg % NA;
          TOPS_TCLK(tk0);
          if (gg > 0) {
            if (!mbar_wait(&sm.s_free[t], (gg - 1) & 1, abort, 204)) { ok = false; break; }
            // fp32 bias (read by the softmax): this tile is done with ring-A slot gg-1 once
            // its QK^T (the commit waits for it) and its softmax's bias read (s_free) are done
            if (BF32) mma_commit(&sm.a_empty[(gg - 1) % NA]);
          }
          if (!mbar_wait(&sm.a_full[s], (gg / NA) & 1, abort, 203)) { ok = false; break; }
          TOPS_TCLK(tk1);
          TOPS_TADD(4, tk0, tk1);
          tc_fence_after();
          const uint32_t ka = smem_u32(k_tile(s, t / TQ));
          if (!BF32) {
            // f16 bias: the tensor core adds it, S = bias x I + Q K^T (exact: I is the
            // identity, products and sums in fp32), so the softmax reads S ready-biased
            const uint32_t ba = smem_u32(sm.ring_a[s] + (t % TQ) * Cfg::B_BYTES), ia = smem_u32(sm.ident);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              mma_ss(s_tmem, make_smem_desc(ba + kk * 32, 16, 1024, kSw128),
                     make_smem_desc(ia + kk * 32, 16, 1024, kSw128), idesc_qk, kk > 0);
          }
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_ss(s_tmem, make_smem_desc(qa + kk * 32, 16, Cfg::QK_SBO, Cfg::QK_SW),
                   make_smem_desc(ka + kk * 32, 16, Cfg::QK_SBO, Cfg::QK_SW), idesc_qk, !BF32 || kk > 0);
          mma_commit(&sm.s_full[t]);
          if (!BF32) mma_commit(&sm.a_empty[s]);  // K and the bias tile consumed once these MMAs finish
          if (j == nkb - 1) mma_commit(&sm.q_empty);  // Q of this unit no longer needed
#ifdef TOPS_TRACE
          { TOPS_TCLK(tq); *reinterpret_cast<volatile long long*>(&sm.t_qk[t]) = tq; }
#endif
        }
      }
    }
  } else if (warp <= 2 * NT) {
    if (lane == 0) {
      // ---------------- PV issuer of tile t ----------------
      // (a thread of its own: one tcgen05.mma occupies the issuing thread ~140 cycles
      // whatever its N, so QK^T and PV of a tile go out from two threads in parallel)
      const int t = warp - 1 - NT;
      // P (ex2 output) and V^T are f16 whatever the IO dtype.
      const uint32_t idesc_pv = make_idesc_f16(128, Cfg::NPV, 0, false, false);
      const uint32_t p_tmem = tbase + Cfg::P_COL + t * 32;
      const uint32_t o_tmem = tbase + Cfg::O_COL + t * Cfg::NPV;
      bool ok = true;
      int g = 0, lu = 0;
      for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++lu, g += nkb) {
        for (int j = 0; j < nkb; ++j) {
          const int gg = g + j;
          TOPS_TCLK(tp0);
          if (!mbar_wait(&sm.p_full[t], gg & 1, abort, 205)) { ok = false; break; }
          TOPS_TCLK(tp1);
          TOPS_TADD(5, tp0, tp1);
          if (!mbar_wait(&sm.b_full[gg % NB], (gg / NB) & 1, abort, 212)) { ok = false; break; }
          // the first PV of a unit overwrites O: the previous unit's epilogue must have read it
          if (j == 0 && lu > 0 && !mbar_wait(&sm.o_empty[t], (lu - 1) & 1, abort, 214)) { ok = false; break; }
          tc_fence_after();
          const uint32_t vb = smem_u32(v_tile(gg % NB, t / TQ));
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_ts(o_tmem, p_tmem + kk * 8, make_smem_desc(vb + kk * 32, 16, 1024, kSw128), idesc_pv, j > 0 || kk > 0);
          mma_commit(&sm.pv_done[t]);
          if (j == nkb - 1) mma_commit(&sm.o_full[t]);
          mma_commit(&sm.b_empty[gg % NB]);
        }
      }
    }
  } else if (warp >= Cfg::SM_WARP0) {
    // ---------------- softmax warpgroups (one tile each) ----------------
    const int t = (warp - Cfg::SM_WARP0) >> 2;
    const int wq = warp & 3;
    const int qrow = wq * 32 + lane;  // TMEM lane == query row within the tile
    const int qb = t % TQ;
    const uint32_t lane_addr = tbase + (static_cast<uint32_t>(wq * 32) << 16);
    const uint32_t oaddr = lane_addr + Cfg::O_COL + t * Cfg::NPV;
    bool ok = true;
    int g = 0, lu = 0;
    for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++lu, g += nkb) {
      int q0, row0, h;
      coords(u, q0, row0, h);
      float m_use = 0.f;
      for (int j = 0; j < nkb; ++j) {
        const int gg = g + j, s = gg % NA;
        TOPS_TCLK(ts0);
        if (!mbar_wait(&sm.s_full[t], gg & 1, abort, 206)) { ok = false; break; }
        if (BF32 && !mbar_wait(&sm.a_full[s], (gg / NA) & 1, abort, 210)) { ok = false; break; }  // bias visible
        TOPS_TCLK(ts1);
#ifdef TOPS_TRACE
        if (lane == 0 && wq == 0) TOPS_TADD(6, *reinterpret_cast<volatile long long*>(&sm.t_qk[t]), ts1);
#endif
        tc_fence_after();
        // x = S + bias (log2 units) packed to f16 pairs. f16 bias: already in S (added by
        // the tensor core); fp32 bias: added here from the ring-A tile.
        __half2 xh[32];
        if (BF32) {
          const uint8_t* brow = sm.ring_a[s] + qb * Cfg::B_BYTES;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t sv[32];
            tmem_ld32(lane_addr + Cfg::S_COL + t * 64 + half * 32, sv);
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
              const float4 bf = *reinterpret_cast<const float4*>(brow + half * 16384 + sw128_off(qrow, ch));
              xh[half * 16 + ch * 2] =
                  __floats2half2_rn(__uint_as_float(sv[ch * 4]) + bf.x, __uint_as_float(sv[ch * 4 + 1]) + bf.y);
              xh[half * 16 + ch * 2 + 1] =
                  __floats2half2_rn(__uint_as_float(sv[ch * 4 + 2]) + bf.z, __uint_as_float(sv[ch * 4 + 3]) + bf.w);
            }
          }
        } else if (TOPS_S_F16) {
          tmem_ld64_pack16(lane_addr + Cfg::S_COL + t * 64, reinterpret_cast<uint32_t*>(xh));
        } else {
          uint32_t sv[64];
          tmem_ld64(lane_addr + Cfg::S_COL + t * 64, sv);
#pragma unroll
          for (int c = 0; c < 32; ++c) xh[c] = __floats2half2_rn(__uint_as_float(sv[2 * c]), __uint_as_float(sv[2 * c + 1]));
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
            if (!mbar_wait(&sm.pv_done[t], (gg - 1) & 1, abort, 208)) { ok = false; break; }
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
        // about 1/3 of the pairs take the polynomial 2^x on the FMA pipe, the rest the MUFU:
        // the XU pipe (2 issues per f16 pair) and the FMA pipe then finish together.
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const __half2 d = __hsub2(xh[c], mh);
          const uint32_t du = *reinterpret_cast<const uint32_t*>(&d);
          pk[c] = (kPolyExp && TOPS_POLY_PICK(c)) ? ex2_poly_f16x2(du) : ex2_f16x2(du);
        }
        TOPS_TCLK(ts3);
        if (j > 0 && !waited) {
          if (!mbar_wait(&sm.pv_done[t], (gg - 1) & 1, abort, 209)) { ok = false; break; }
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
      const bool got = ok && mbar_wait(&sm.o_full[t], lu & 1, abort, 207);
      if (!got) ok = false;
      tc_fence_after();
      uint32_t o[Cfg::NPV];
      if (D == 32) {
        tmem_ld32(oaddr, o);
        tmem_ld16(oaddr + 32, o + 32);
      } else {
        tmem_ld32(oaddr, o);
      }
      // O is in registers: the next unit's first PV may overwrite it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.o_empty[t]);
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
  }
  TOPS_TFLUSH();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

}  // namespace tops
