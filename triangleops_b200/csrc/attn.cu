// attn.cu — biased, key-masked flash attention on tcgen05 for triangle attention
// (starting node, rows of the pair tensor) and attention-with-pair-bias (one row).
//
// Semantics per (row r, head h, query q)  [triangle_attn/kernel.py:194-253]:
//   S[q,k] = Q[r,h,q,:] . K[r,h,k,:] + bias[h,q,k] + pen[r,k]   (Q already scaled; log2 units)
//   O[r,q,h*D:(h+1)*D] = sum_k softmax_k(S) V[r,h,k,:]
// pen[r,k] is 0 for an unmasked key and -inf for a masked one, and keys past Nk get
// -inf as well, so masked and out-of-range keys take part in neither the row max nor
// the sum (the reference's -1e9 / -inf additive masks, kernel.py:230-239). A row whose
// keys are all masked is left to attn_deadrow_kernel (the reference's uniform average).
//
// The bias is shared by every row r (triangle attention), so one CTA processes TR
// rows ("tiles", 128 queries each) of the same head and query block: each bias tile
// read from L2 serves TR rows.
//
// The tensor core builds S completely, running max included, so the softmax does per
// element only the block max and 2^x. Per 64-key block and tile, one thread issues into
// the f16 accumulator S:
//   S  = bias x I          4 MMAs (K = 64 keys in steps of 16; I = 64 x 64 identity)
//   S += Q K^T             D/16 MMAs
//   S += M x pen           1 MMA: M is the tile's 128 x 16 "row term" tile (column 0
//                          1.0, columns 1 and 2 the f16 pair hi + lo = -m of the query
//                          row), B an MN-major 16 x 64 tile whose row 0 is the pair
//                          row's penalty row and rows 1 and 2 ones, so every query gets
//                          pen[k] - m. m is the running max the softmax last settled on
//                          (0 at the start of a unit); the softmax rewrites its row of M
//                          only when m moves; the S issuer issues the other MMAs of
//                          the next block meanwhile and this one once m is settled.
// and one thread issues PV: O += P V^T (P from TMEM, 4 MMAs of 16 keys).
//
// Cost model (measured on B200): a warp pays ~82 cycles to issue one SS tcgen05.mma
// and ~164 cycles for a TS one (A from TMEM), whatever N is, and MMAs of different
// warps overlap. The f16 pair pipe (add/sub/fma on f16x2) and the MUFU are what the
// softmax spends its time on, so every per-element add that the tensor core can do
// instead is moved there.
//
// Per CTA: w0 TMA producer A (per 64-key block: bias, TR K tiles and TR penalty rows
// into ring A; the unit's Q tiles), w1 TMA producer B (TR V^T tiles into ring B),
// w(2+t) S issuer of tile t, w(2+TR+t) PV issuer of tile t, one softmax warpgroup per
// tile (one TMEM lane = one query row per thread). TMEM per tile: S (64 f16 columns),
// P (32 columns of packed f16 pairs per buffer, the A operand of PV; two buffers when
// TMEM has room), O (D+16 fp32 columns: D values, the row sum, zero padding).
//
// Row sum without per-element work: row D of every V^T operand tile is 1.0 (written
// once), so the PV MMA also produces l = sum_k p_k in accumulator column D.
//
// Online softmax in the exp2 domain (Q carries scale*log2(e) and the bias log2(e),
// both folded in upstream) with lazy rescaling (O is only rescaled when the running
// max grows by more than 2^8; the S the softmax loads is already x = s - m, so 2^x
// needs no subtraction unless m moves in this block). The per-element work runs on f16 pairs: the tensor
// core accumulates S in f16 (each step rounds once, relative error 2^-11, below the
// 2^-8 rounding the 16-bit operands already put into S), the softmax loads it as
// packed pairs (tcgen05.ld .pack::16b), takes the row max as a pairwise tree, and
// computes P = 2^(x - m) with part of the pairs on the MUFU (ex2.approx.f16x2) and
// the rest by a polynomial on the FMA pipe (ex2_poly_f16x2), so that neither pipe
// alone bounds the step.
#include "sm100.cuh"

namespace tops {

#ifndef TOPS_POLY_PICK
#define TOPS_POLY_PICK(c) ((c) % 3 == 1)  // pairs whose 2^x takes the polynomial (11 of 32)
#endif

// KS (key split): the NT tiles of a CTA share one row, query block and head and take
// NT consecutive ranges of the key blocks; their partial (O, l, max) are merged in the
// epilogue. Used where there are few work units (attention with pair bias: one row).
template <int D, int TR, bool KS = false>
struct AttnCfg {
  static constexpr int NT = TR;                 // tiles (128 queries x 1 row) per CTA
  // warps: 0 and 1 TMA producers (ring A, ring B), 2..NT+1 S issuers, NT+2..2NT+1 PV
  // issuers, then one softmax warpgroup per tile (any 4 consecutive warps cover the 4
  // TMEM lane quarters)
  static constexpr int SM_WARP0 = 2 + 2 * NT;
  static constexpr int THREADS = 32 * SM_WARP0 + 128 * NT;
  static constexpr int BK = 64;                 // keys per block
  static constexpr int NPV = D + 16;            // PV N: D value columns + ones row + zero pad
  static constexpr int Q_BYTES = 128 * D * 2;
  static constexpr int K_BYTES = BK * D * 2;
  static constexpr int V_BYTES = NPV * 128;     // NPV rows x 64 keys (128 B, SW128)
  static constexpr int BIAS_BYTES = 128 * BK * 2;  // f16 bias tile [128 q][64 k], SW128
  static constexpr int PEN_BYTES = 16 * 128;    // MN-major 16 x 64 tile, row 0 = penalty row
  // ring A: the bias tile, the TR K tiles and the TR penalty tiles (free once every S
  // MMA of the block has run); ring B: the TR V^T tiles (free once every PV has run)
  static constexpr int NBIAS = KS ? TR : 1;     // bias tiles per stage (KS: one per key range)
  static constexpr int K_OFF = NBIAS * BIAS_BYTES;
  static constexpr int PEN_OFF = K_OFF + TR * K_BYTES;
  static constexpr int A_BYTES = PEN_OFF + TR * PEN_BYTES;
  static constexpr int B_BYTES = TR * V_BYTES;
  static constexpr int NA = 3;
  static constexpr int NB = 3;
  static constexpr uint32_t QK_SW = D == 32 ? kSw64 : kSw32;
  static constexpr int QK_SBO = 8 * D * 2;       // 8 rows x row bytes
  // P buffers per tile: two when TMEM has room (the softmax then writes P(j+1) while
  // PV(j) still reads P(j)), else one
  static constexpr int NPB = (64 + 64 + NPV) * NT <= 512 ? 2 : 1;
  static constexpr int S_COL = 0;                      // S of tile t at t*64
  static constexpr int P_COL = 64 * NT;                // P buffer b of tile t at P_COL + (t*NPB + b)*32
  static constexpr int O_COL = P_COL + 32 * NPB * NT;  // O of tile t at O_COL + t*NPV
  static constexpr int TMEM_USED = O_COL + NPV * NT;
  static constexpr int TMEM_COLS = TMEM_USED <= 256 ? 256 : 512;
  static_assert(TMEM_USED <= 512, "TMEM budget");
  static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0 && Q_BYTES % 1024 == 0 && PEN_OFF % 1024 == 0,
                "alignment");
};

struct AttnArgs {
  int R, Nq, Nk;
  void* out;     // [R][Nq][H*D]
  int H;
  int has_mask;  // penalty rows present (else every key < Nk is valid)
};

template <int D, int TR, bool KS = false>
struct AttnSmem {
  using Cfg = AttnCfg<D, TR, KS>;
  alignas(1024) uint8_t q[Cfg::NT][Cfg::Q_BYTES];
  alignas(1024) uint8_t ring_a[Cfg::NA][Cfg::A_BYTES];
  alignas(1024) uint8_t ring_b[Cfg::NB][Cfg::B_BYTES];
  alignas(1024) uint8_t ident[64 * 128];   // f16 identity (64 x 64, K-major SW128)
  // per tile: the A operand of the penalty / running-max MMA (128 x 16 f16, K-major
  // SW32; row q = [1, -m_hi, -m_lo, 0, 0, 0, 0, 0] in both 16-byte halves, so the
  // 32-byte swizzle, which may swap the halves, leaves the logical columns 0..2 and
  // 8..10 equal; B rows 8..10 are zero)
  alignas(1024) uint8_t mtile[Cfg::NT][128 * 32];
  uint64_t bar_q;
  uint64_t q_empty;            // one commit per S issuer (after the unit's last QK^T)
  uint64_t a_full[Cfg::NA];
  uint64_t a_empty[Cfg::NA];   // one commit per S issuer
  uint64_t b_full[Cfg::NB];
  uint64_t b_empty[Cfg::NB];   // one commit per PV issuer
  uint64_t s_full[Cfg::NT];    // S of the block complete
  uint64_t s_free[Cfg::NT];    // the softmax has loaded S (it may be overwritten)
  uint64_t m_ready[Cfg::NT];   // the softmax has settled the block's max (row term tile written)
  uint64_t p_full[Cfg::NT];    // P of the block written
  uint64_t pv_done[Cfg::NT][2];  // PV of a block using P buffer b finished (P reusable, O stable)
  uint64_t o_full[Cfg::NT];    // the last PV of the unit finished
  uint64_t o_empty[Cfg::NT];   // the epilogue has read O (the next unit may overwrite it)
  // KS: tiles 1.. hand (O, l, max) of each query row to tile 0's epilogue
  float comb[KS ? TR - 1 : 1][KS ? 128 * (D + 2) : 1];
  uint64_t comb_full, comb_empty;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ float f16lo(uint32_t p) { return __half2float(__ushort_as_half(static_cast<unsigned short>(p & 0xFFFFu))); }
__device__ __forceinline__ float f16hi(uint32_t p) { return __half2float(__ushort_as_half(static_cast<unsigned short>(p >> 16))); }
__device__ __forceinline__ uint32_t hmax2_u(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

constexpr uint32_t kF16NegInf2 = 0xFC00FC00u;

template <typename T, int D, int TR, bool KS = false>
__global__ void __launch_bounds__(AttnCfg<D, TR, KS>::THREADS, 1)
    attn_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_pen,
                const __grid_constant__ CUtensorMap map_b, AttnArgs a) {
  using Cfg = AttnCfg<D, TR, KS>;
  using E = Elem<T>;
  constexpr int NA = Cfg::NA, NB = Cfg::NB, NT = Cfg::NT, BK = Cfg::BK, NPB = Cfg::NPB;
  extern __shared__ uint8_t smem_raw[];
  auto& sm = *reinterpret_cast<AttnSmem<D, TR, KS>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();  // the kernel after this one (the gate) may set itself up on SMs left free
  const int nkb = (a.Nk + BK - 1) / BK;
  // key blocks per unit and tile: all of them, or (KS) this tile's share of them; tile t's
  // key block at step j is kblk(t, j) (KS ranges past the last block are empty: TMA zero-fill,
  // every key out of range)
  const int nst = KS ? (nkb + NT - 1) / NT : nkb;
  auto kblk = [&](int t, int j) { return KS ? t * nst + j : j; };
  const int H = a.H;
  const bool has_mask = a.has_mask != 0;
  auto k_tile = [&](int s, int r) { return sm.ring_a[s] + Cfg::K_OFF + r * Cfg::K_BYTES; };
  auto pen_tile = [&](int s, int r) { return sm.ring_a[s] + Cfg::PEN_OFF + r * Cfg::PEN_BYTES; };
  auto v_tile = [&](int s, int r) { return sm.ring_b[s] + r * Cfg::V_BYTES; };

  // Constant operand parts, written once (TMA never touches them):
  //  * rows D .. NPV-1 of every V^T tile: row D all ones (the row-sum column of PV), the rest zero;
  //  * every penalty tile: row 0 zero (TMA overwrites it on masked calls), rows 1 and 2
  //    ones (they carry -m_hi and -m_lo of the row term tile), rows 3..15 zero;
  //  * the 64 x 64 identity (element (n, k) at n*128 + ((k/8 ^ n%8) * 16) + (k%8)*2) and
  //    the row term tiles (m = 0).
  constexpr int EXTRA_ROWS = Cfg::NPV - D;
  for (int idx = threadIdx.x; idx < NB * NT * EXTRA_ROWS * 32; idx += blockDim.x) {
    const int w = idx & 31, rowp = (idx >> 5) % EXTRA_ROWS, rs = idx / (EXTRA_ROWS * 32);
    uint32_t* v = reinterpret_cast<uint32_t*>(v_tile(rs / NT, rs % NT));
    v[(D + rowp) * 32 + w] = rowp == 0 ? 0x3C003C00u : 0u;
  }
  for (int idx = threadIdx.x; idx < NA * NT * 16 * 32; idx += blockDim.x) {
    const int w = idx & 31, row = (idx >> 5) & 15, rs = idx / (16 * 32);
    reinterpret_cast<uint32_t*>(pen_tile(rs / NT, rs % NT))[row * 32 + w] = (row == 1 || row == 2) ? 0x3C003C00u : 0u;
  }
  for (int w = threadIdx.x; w < 64 * 32; w += blockDim.x) {
    const int n = w >> 5, pc = w & 31;          // row n, 32-bit word pc of the 128-byte row
    const int k0 = ((pc >> 2) ^ (n & 7)) * 8 + (pc & 3) * 2;  // logical column of the word's low half
    reinterpret_cast<uint32_t*>(sm.ident)[w] = (k0 == n ? 0x3C00u : 0u) | (k0 + 1 == n ? 0x3C000000u : 0u);
  }
  for (int w = threadIdx.x; w < NT * 128 * 8; w += blockDim.x)
    reinterpret_cast<uint32_t*>(&sm.mtile[0][0])[w] = (w & 3) == 0 ? 0x00003C00u : 0u;
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
      mbar_init(&sm.m_ready[t], 4);
      mbar_init(&sm.p_full[t], 4);
      mbar_init(&sm.pv_done[t][0], 1);
      mbar_init(&sm.pv_done[t][1], 1);
      mbar_init(&sm.o_full[t], 1);
      mbar_init(&sm.o_empty[t], 4);
    }
    mbar_init(&sm.comb_full, 128 * (NT - 1 > 0 ? NT - 1 : 1));
    mbar_init(&sm.comb_empty, 128);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&sm.tmem_base, Cfg::TMEM_COLS);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;
  volatile int* abort = &sm.abort;

  // Persistent: CTA b takes work units b, b + gridDim.x, ... A unit is TR rows x one
  // 128-query block of one head (query block fastest: the CTAs running together share
  // the bias tiles of a head and the K/V of a row in L2). Ring slots and barrier
  // phases run on across units (g = blocks processed by this CTA so far, lu = units
  // so far), so the producers stream the next unit's tiles while the current one ends.
  const int n_qb = (a.Nq + 127) / 128;
  constexpr int UROWS = KS ? 1 : TR;  // pair rows per unit (KS: the tiles share one row)
  const int n_rg = (a.R + UROWS - 1) / UROWS;
  const int n_units = n_qb * n_rg * a.H;
  auto coords = [&](int u, int& q0, int& row0, int& h) {
    q0 = (u % n_qb) * 128;
    const int rest = u / n_qb;
    row0 = (rest % n_rg) * UROWS;
    h = rest / n_rg;
  };
  auto trow = [&](int row0, int t) { return KS ? row0 : row0 + t; };  // pair row of tile t

  if (warp == 0) {
    // ---------------- TMA producer A: bias, K and penalty tiles (ring A), Q tiles ----------------
    // The whole warp runs the loop; lane r issues the load of tile r, so the loads of a
    // block go out as few warp instructions.
    if (lane == 0) {
      tma_prefetch_desc(&map_q);
      tma_prefetch_desc(&map_k);
      tma_prefetch_desc(&map_b);
      if (has_mask) tma_prefetch_desc(&map_pen);
    }
    const uint32_t a_tx = Cfg::NBIAS * Cfg::BIAS_BYTES + NT * Cfg::K_BYTES + (has_mask ? NT * 128 : 0);
    bool ok = true;
    int g = 0, lu = 0;
    for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++lu, g += nst) {
      int q0, row0, h;
      coords(u, q0, row0, h);
      for (int j = 0; j < nst; ++j) {
        const int gg = g + j, s = gg % NA;
        if (!mbar_wait(&sm.a_empty[s], ((gg / NA) & 1) ^ 1, abort, 201)) { ok = false; break; }
        if (lane == 0) mbar_expect_tx(&sm.a_full[s], a_tx);
        __syncwarp();
        if (lane >= NT && lane < NT + Cfg::NBIAS)
          tma_load_3d(sm.ring_a[s] + (lane - NT) * Cfg::BIAS_BYTES, &map_b, &sm.a_full[s], kblk(lane - NT, j) * BK, q0, h);
        else if (lane < NT)
          tma_load_3d(k_tile(s, lane), &map_k, &sm.a_full[s], 0, kblk(lane, j) * BK, trow(row0, lane) * H + h);
        else if (has_mask && lane >= 16 && lane < 16 + NT)
          tma_load_2d(pen_tile(s, lane - 16), &map_pen, &sm.a_full[s], kblk(lane - 16, j) * BK, trow(row0, lane - 16));
        if (j == 0) {
          // the unit's Q tiles, once the previous unit's last QK^T has read them
          if (!mbar_wait(&sm.q_empty, (lu & 1) ^ 1, abort, 213)) { ok = false; break; }
          if (lane == 0) mbar_expect_tx(&sm.bar_q, NT * Cfg::Q_BYTES);
          __syncwarp();
          if (lane < NT) tma_load_3d(sm.q[lane], &map_q, &sm.bar_q, 0, q0, trow(row0, lane) * H + h);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- TMA producer B: V^T tiles (ring B) ----------------
    if (lane == 0) tma_prefetch_desc(&map_v);
    const uint32_t b_tx = NT * (D * 128);
    bool ok = true;
    int g = 0;
    for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, g += nst) {
      int q0, row0, h;
      coords(u, q0, row0, h);
      (void)q0;
      for (int j = 0; j < nst; ++j) {
        const int gg = g + j, sb = gg % NB;
        if (!mbar_wait(&sm.b_empty[sb], ((gg / NB) & 1) ^ 1, abort, 211)) { ok = false; break; }
        if (lane == 0) mbar_expect_tx(&sm.b_full[sb], b_tx);
        __syncwarp();
        if (lane < NT) tma_load_3d(v_tile(sb, lane), &map_v, &sm.b_full[sb], kblk(lane, j) * BK, 0, trow(row0, lane) * H + h);
      }
    }
  } else if (warp <= NT + 1) {
    if (lane == 0) {
      // ---------------- S issuer of tile t: bias x I, Q K^T, 1 x pen ----------------
      const int t = warp - 2;
      // every S operand is f16; S is accumulated in f16 (D format 0)
      const uint32_t idesc_s = make_idesc_f16(128, BK, 0, false, false) & ~(3u << 4);
      const uint32_t idesc_pen = make_idesc_f16(128, BK, 0, false, true) & ~(3u << 4);
      const uint32_t qa = smem_u32(sm.q[t]), ia = smem_u32(sm.ident);
      const uint64_t mt_desc = make_smem_desc(smem_u32(sm.mtile[t]), 16, 256, kSw32);
      const uint32_t s_tmem = tbase + Cfg::S_COL + t * 64;
      bool ok = true;
      int g = 0, lu = 0;
      for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++lu, g += nst) {
        if (!mbar_wait(&sm.bar_q, lu & 1, abort, 202)) break;
        for (int j = 0; j < nst; ++j) {
          const int gg = g + j, s = gg % NA;
          if (!mbar_wait(&sm.a_full[s], (gg / NA) & 1, abort, 203)) { ok = false; break; }
          if (gg > 0 && !mbar_wait(&sm.s_free[t], (gg - 1) & 1, abort, 204)) { ok = false; break; }
          tc_fence_after();
          const uint32_t ba = smem_u32(sm.ring_a[s] + (KS ? t : 0) * Cfg::BIAS_BYTES), ka = smem_u32(k_tile(s, t));
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_ss(s_tmem, make_smem_desc(ba + kk * 32, 16, 1024, kSw128), make_smem_desc(ia + kk * 32, 16, 1024, kSw128),
                   idesc_s, kk > 0);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_ss(s_tmem, make_smem_desc(qa + kk * 32, 16, Cfg::QK_SBO, Cfg::QK_SW),
                   make_smem_desc(ka + kk * 32, 16, Cfg::QK_SBO, Cfg::QK_SW), idesc_s, 1);
          // the row term of S(gg) carries the max the softmax settled on in block gg - 1: the
          // six MMAs above do not need it and run while the softmax takes that block's max
          if (gg > 0 && !mbar_wait(&sm.m_ready[t], (gg - 1) & 1, abort, 215)) { ok = false; break; }
          mma_ss(s_tmem, mt_desc, make_smem_desc(smem_u32(pen_tile(s, t)), 2048, 1024, kSw128), idesc_pen, 1);
          mma_commit(&sm.s_full[t]);
          mma_commit(&sm.a_empty[s]);  // bias, K and penalty tiles consumed once these finish
          if (j == nst - 1) mma_commit(&sm.q_empty);  // Q of this unit no longer needed
        }
      }
    }
  } else if (warp <= 2 * NT + 1) {
    if (lane == 0) {
      // ---------------- PV issuer of tile t ----------------
      const int t = warp - 2 - NT;
      // P (ex2 output) and V^T are f16 whatever the IO dtype.
      const uint32_t idesc_pv = make_idesc_f16(128, Cfg::NPV, 0, false, false);
      const uint32_t p_tmem0 = tbase + Cfg::P_COL + t * 32 * NPB;
      const uint32_t o_tmem = tbase + Cfg::O_COL + t * Cfg::NPV;
      bool ok = true;
      int g = 0, lu = 0;
      for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++lu, g += nst) {
        for (int j = 0; j < nst; ++j) {
          const int gg = g + j, sb = gg % NB;
          if (!mbar_wait(&sm.p_full[t], gg & 1, abort, 205)) { ok = false; break; }
          if (!mbar_wait(&sm.b_full[sb], (gg / NB) & 1, abort, 212)) { ok = false; break; }
          // the first PV of a unit overwrites O: the previous unit's epilogue must have read it
          if (j == 0 && lu > 0 && !mbar_wait(&sm.o_empty[t], (lu - 1) & 1, abort, 214)) { ok = false; break; }
          tc_fence_after();
          const uint32_t vb = smem_u32(v_tile(sb, t));
          const uint32_t p_tmem = p_tmem0 + (gg % NPB) * 32;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_ts(o_tmem, p_tmem + kk * 8, make_smem_desc(vb + kk * 32, 16, 1024, kSw128), idesc_pv, j > 0 || kk > 0);
          mma_commit(&sm.pv_done[t][gg % NPB]);
          if (j == nst - 1) mma_commit(&sm.o_full[t]);
          mma_commit(&sm.b_empty[sb]);
        }
      }
    }
  } else if (warp >= Cfg::SM_WARP0) {
    // ---------------- softmax warpgroups (one tile each) ----------------
    const int t = (warp - Cfg::SM_WARP0) >> 2;
    const int wq = warp & 3;
    const int qrow = wq * 32 + lane;  // TMEM lane == query row within the tile
    const uint32_t lane_addr = tbase + (static_cast<uint32_t>(wq * 32) << 16);
    const uint32_t oaddr = lane_addr + Cfg::O_COL + t * Cfg::NPV;
    bool ok = true;
    int g = 0, lu = 0;
    for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++lu, g += nst) {
      int q0, row0, h;
      coords(u, q0, row0, h);
      // m_use: the running max the P of this unit are relative to (-inf while every key seen
      // is masked); m_b: the value baked into S by the row term tile (m_use once finite,
      // 0 before: S then holds s itself)
      float m_use = -INFINITY, m_b = 0.f;
      for (int j = 0; j < nst; ++j) {
        const int gg = g + j;
        if (!mbar_wait(&sm.s_full[t], gg & 1, abort, 206)) { ok = false; break; }
        tc_fence_after();
        uint32_t x[32];
        tmem_ld64_pack16(lane_addr + Cfg::S_COL + t * 64, x);  // x = s - m_b
        // S consumed: the S MMAs of the next block may proceed (all but its row term)
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.s_free[t]);
        const int nvalid = a.Nk - kblk(t, j) * BK;
        if (nvalid < BK) {
          // keys past Nk (zero-filled K, bias and penalty) are out of range: -inf
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const uint32_t keep = (2 * c < nvalid ? 0x0000FFFFu : 0u) | (2 * c + 1 < nvalid ? 0xFFFF0000u : 0u);
            x[c] = (x[c] & keep) | (kF16NegInf2 & ~keep);
          }
        }
        uint32_t mt[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) mt[c] = hmax2_u(x[2 * c], x[2 * c + 1]);
#pragma unroll
        for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
          for (int c = 0; c < w; ++c) mt[c] = hmax2_u(mt[c], mt[c + w]);
        const float mxx = fmaxf(f16lo(mt[0]), f16hi(mt[0]));  // block max of s - m_b (f16 value)
        // the max moves on the first finite key of the row and when it grows past m_use + 8
        const bool need = m_use == -INFINITY ? mxx > -INFINITY : mxx > 8.0f;
        const float m_new = need ? m_b + mxx : m_use;
        // S of the next block (the next unit's first block after the last one) is built
        // against m_next: rewrite this row of the row term tile when it differs from m_b
        // (the row term MMA of this block has finished, the next one waits for m_ready)
        const float m_next = j == nst - 1 || m_new == -INFINITY ? 0.f : m_new;
        if (__any_sync(0xffffffffu, m_next != m_b)) {
          const __half hi = __float2half_rn(-m_next);
          const __half lo = __float2half_rn(-m_next - __half2float(hi));
          const uint2 w = make_uint2(0x3C00u | (static_cast<uint32_t>(__half_as_ushort(hi)) << 16),
                                     static_cast<uint32_t>(__half_as_ushort(lo)));
          uint2* mrow = reinterpret_cast<uint2*>(sm.mtile[t] + qrow * 32);
          mrow[0] = w;
          mrow[2] = w;
          fence_proxy_async_smem();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.m_ready[t]);
        // P(gg) reuses the buffer of PV(gg - NPB) and an O rescale needs O stable (PV(gg - 1)
        // done). The previous unit's PVs are all done (its epilogue waited for o_full).
        bool waited = false;
        if (__any_sync(0xffffffffu, need)) {
          if (j > 0) {
            if (!mbar_wait(&sm.pv_done[t][(gg - 1) % NPB], ((gg - 1) / NPB) & 1, abort, 208)) { ok = false; break; }
            waited = true;
            tc_fence_after();
            // m_use = -inf (every key so far masked): O holds only zero-weighted terms
            const float alpha = need ? ex2_approx(m_use - m_new) : 1.0f;
            // 16 columns at a time (few live registers on this rare path)
#pragma unroll
            for (int c0 = 0; c0 < Cfg::NPV; c0 += 16) {
              uint32_t o[16];
              tmem_ld16(oaddr + c0, o);
#pragma unroll
              for (int c = 0; c < 16; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
              tmem_st16(oaddr + c0, o);
            }
          }
          // this block against the new max: x - (m_new - m_b) = x - mxx (an f16 value)
          const __half2 d2 = __float2half2_rn(need ? mxx : 0.f);
          const uint32_t dh = *reinterpret_cast<const uint32_t*>(&d2);
#pragma unroll
          for (int c = 0; c < 32; ++c) x[c] = hsub2_u(x[c], dh);
        }
        m_use = m_new;
        m_b = m_next;
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) pk[c] = TOPS_POLY_PICK(c) ? ex2_poly_f16x2(x[c]) : ex2_f16x2(x[c]);
        if (j >= NPB && !waited) {
          if (!mbar_wait(&sm.pv_done[t][gg % NPB], ((gg - NPB) / NPB) & 1, abort, 209)) { ok = false; break; }
          tc_fence_after();
        }
        tmem_st32(lane_addr + Cfg::P_COL + (t * NPB + gg % NPB) * 32, pk);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_full[t]);
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
      if constexpr (KS) {
        // merge the key ranges: tiles 1.. hand (O, l, max) of their row to tile 0, which
        // rescales each part to the common max (an all-masked part has max -inf: weight 0)
        constexpr int W = D + 2;
        if (t > 0) {
          if (got && mbar_wait(&sm.comb_empty, (lu & 1) ^ 1, abort, 217)) {
            float* c = sm.comb[t - 1] + qrow * W;
#pragma unroll
            for (int d = 0; d <= D; ++d) c[d] = __uint_as_float(o[d]);
            c[D + 1] = m_use;
          } else {
            ok = false;
          }
          mbar_arrive(&sm.comb_full);
          continue;
        }
        if (!(got && mbar_wait(&sm.comb_full, lu & 1, abort, 218))) {
          ok = false;
          continue;
        }
        float m = m_use;
#pragma unroll
        for (int t2 = 1; t2 < NT; ++t2) m = fmaxf(m, sm.comb[t2 - 1][qrow * W + D + 1]);
        const float f0 = (m == -INFINITY || m_use == -INFINITY) ? 0.f : ex2_approx(m_use - m);
#pragma unroll
        for (int d = 0; d <= D; ++d) o[d] = __float_as_uint(__uint_as_float(o[d]) * f0);
#pragma unroll
        for (int t2 = 1; t2 < NT; ++t2) {
          const float* c = sm.comb[t2 - 1] + qrow * W;
          const float mt = c[D + 1];
          const float ft = (m == -INFINITY || mt == -INFINITY) ? 0.f : ex2_approx(mt - m);
#pragma unroll
          for (int d = 0; d <= D; ++d) o[d] = __float_as_uint(fmaf(c[d], ft, __uint_as_float(o[d])));
        }
        mbar_arrive(&sm.comb_empty);
      }
      const int ri = trow(row0, t);
      const int q = q0 + qrow;
      if (got && ri < a.R && q < a.Nq) {
        // l = 0: every key of the row is masked (attn_deadrow_kernel writes those rows)
        const float l = __uint_as_float(o[D]);
        const float inv = l > 0.f ? 1.0f / l : 0.f;
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
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, Cfg::TMEM_COLS);
}

// Rows whose keys are all masked. The reference adds -1e9 to every score of such a
// row, which makes them all equal in fp32: the softmax is uniform over the Nk keys
// and the output is the mean of V over all of them, masked keys included
// (triangle_attn/kernel.py:233-238). One CTA per row: a vote over the row's penalty
// entries, and for a dead row the H*D key means of V^T broadcast to every query.
template <typename T>
__global__ void __launch_bounds__(128) attn_deadrow_kernel(const __half* __restrict__ pen,
                                                           const __half* __restrict__ vt, T* __restrict__ out, int R,
                                                           int Nq, int Nk, int Nkp, int HD) {
  using E = Elem<T>;
  pdl_trigger();
  for (int r = blockIdx.x; r < R; r += gridDim.x) {
    const __half* prow = pen + static_cast<size_t>(r) * Nkp;
    bool alive = false;
    for (int k = threadIdx.x; k < Nk; k += blockDim.x) alive |= __half_as_ushort(prow[k]) == 0;
    // the vote reads only the projection's penalty row; a dead row's output overwrites
    // what the attention kernel (launched just before, still running) writes there
    pdl_wait();
    if (__syncthreads_or(alive)) continue;
    // dead row: thread c (< H*D) owns value column c = h*D + d, V^T row (r*H + h)*D + d
    float mean = 0.f;
    if (threadIdx.x < HD) {
      const __half* vrow = vt + (static_cast<size_t>(r) * HD + threadIdx.x) * Nkp;
      float s = 0.f;
      for (int k = 0; k < Nk; ++k) s += __half2float(vrow[k]);
      mean = s / static_cast<float>(Nk);
    }
    const T mv = E::from_f(mean);
    if (threadIdx.x < HD)
      for (int q = 0; q < Nq; ++q) out[(static_cast<size_t>(r) * Nq + q) * HD + threadIdx.x] = mv;
  }
}

}  // namespace tops
