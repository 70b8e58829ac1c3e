// trimul.cu — triangle multiplicative update on tcgen05 (replaces
// triangle_ops/triangle_mul/kernel.py and the cuBLAS einsum of module.py:70-76).
//
//   input phase   ab[k, m] = mask[m] * sigmoid(LN(x)[m] g_in[k]) * (LN(x)[m] p_in[k])   (k < 2C)
//                 with LN folded into the weights: LN(x) W^T = rstd (x Wc^T - mean sumW) + Bc
//                 [triangle_mul/kernel.py:35-162 with TRANS=True]
//   contraction   outgoing y[d,i,j] = sum_k a[d,i,k] b[d,j,k]      (both operands K-major)
//                 incoming y[d,i,j] = sum_k a[d,k,i] b[d,k,j]      (both operands MN-major)
//   output phase  out[m, c] = sigmoid(LN_in(x)[m] g_out[c]) * (LN_out(y)[m] p_out[c])
//                 [triangle_mul/kernel.py:282-326, y read D-major]
//
// Every phase is a persistent warp-specialised kernel: w0 TMA producer, w1 MMA
// issuer, w4-7 LayerNorm statistics (from the staged tile in shared memory),
// w8-11 epilogue (TMEM -> registers -> global).
#include "sm100.cuh"

namespace tops {

struct LnGateArgs {
  long long M;           // tokens
  float eps;
  const float* sum_w;    // [NOUT] folded column sums (fp32)
  const float* b_const;  // [NOUT] folded biases (fp32)
  const uint8_t* mask;   // [M] int8 multiplier (input phase only; nullptr = none)
  void* out;
  const void* residual;  // output phase: nullptr, or [M][C] added to the result (may alias out)
};

// LayerNorm statistics of a 128 x C row-major (K-major, SW128) staged tile row
// (two passes over shared memory, 16-byte chunks: no C-wide register array; four
// packed fp32-pair accumulators, so the adds form eight independent chains).
template <typename T, int C>
__device__ __forceinline__ void row_stats_kmajor(const uint8_t* tile, int row, float& mean, float& rstd, float eps) {
  using E = Elem<T>;
  auto chunk = [&](int i) {  // chunk i of the row: channels [8i, 8i + 8)
    return *reinterpret_cast<const uint4*>(tile + (i >> 3) * 16384 + sw128_off(row, i & 7));
  };
  unsigned long long acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll 4
  for (int i = 0; i < C / 8; ++i) {
    const uint4 u = chunk(i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[e] = f2_add(acc[e], f2_pack(E::lo(w[e]), E::hi(w[e])));
  }
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float lo, hi;
    f2_unpack(acc[e], lo, hi);
    s += lo + hi;
    acc[e] = 0ull;
  }
  mean = s * (1.0f / C);
  const unsigned long long nm = f2_pack(-mean, -mean);
#pragma unroll 4
  for (int i = 0; i < C / 8; ++i) {
    const uint4 u = chunk(i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const unsigned long long d = f2_add(f2_pack(E::lo(w[e]), E::hi(w[e])), nm);
      acc[e] = f2_fma(d, d, acc[e]);
    }
  }
  float v = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float lo, hi;
    f2_unpack(acc[e], lo, hi);
    v += lo + hi;
  }
  rstd = rsqrtf(v * (1.0f / C) + eps);
}

// LayerNorm statistics over the channel (K) axis of the 128 tokens of a C x 128
// MN-major SW128 staged tile (two 64-token halves, each C rows of 128 B), computed by
// one warpgroup together (wtid = thread index within it). Thread (warp w, lane) takes
// token group tg = 4w + lane/8 (tokens 8tg..8tg+7, one 16-byte chunk per channel) and
// channel subset cs = lane%8 (C/8 channels); the 8 lanes of a group combine their
// partial sums with a butterfly reduce-scatter, so lane cs ends with token 8tg + cs.
// Two passes (mean, then squared deviations). Returns the token (within the tile)
// whose statistics this thread holds; its 32 tokens are the warp's own 32 rows.
template <typename T, int C>
__device__ __forceinline__ int col_stats_coop(const uint8_t* tile, int wtid, float& mean, float& rstd, float eps) {
  using E = Elem<T>;
  constexpr int CS = C / 8;  // channels per subset
  static_assert((CS & (CS - 1)) == 0 && CS >= 8, "C / 8 must be a power of two >= 8");
  const int lane = wtid & 31, cs = lane & 7, tg = (wtid >> 5) * 4 + (lane >> 3);
  const uint8_t* base = tile + (tg >> 3) * (C * 128);
  const uint32_t chunk = tg & 7;
  auto ld = [&](int i) {
    // channel order rotated by cs: the 8 lanes of a group read 8 different 16-byte bank groups
    const int d = cs * CS + ((i + cs) & (CS - 1));
    return *reinterpret_cast<const uint4*>(base + d * 128 + ((chunk ^ (d & 7)) << 4));
  };
  auto reduce8 = [&](const unsigned long long (&acc)[4]) -> float {
    float v[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) f2_unpack(acc[e], v[2 * e], v[2 * e + 1]);
    const bool b2 = cs & 4, b1 = cs & 2, b0 = cs & 1;
    float t[4], u[2];
#pragma unroll
    for (int j = 0; j < 4; ++j) t[j] = (b2 ? v[4 + j] : v[j]) + __shfl_xor_sync(0xffffffffu, b2 ? v[j] : v[4 + j], 4);
#pragma unroll
    for (int j = 0; j < 2; ++j) u[j] = (b1 ? t[2 + j] : t[j]) + __shfl_xor_sync(0xffffffffu, b1 ? t[j] : t[2 + j], 2);
    return (b0 ? u[1] : u[0]) + __shfl_xor_sync(0xffffffffu, b0 ? u[0] : u[1], 1);
  };
  unsigned long long acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll 4
  for (int i = 0; i < CS; ++i) {
    const uint4 u = ld(i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[e] = f2_add(acc[e], f2_pack(E::lo(w[e]), E::hi(w[e])));
  }
  mean = reduce8(acc) * (1.0f / C);
  unsigned long long nm[4];
  const int g0 = lane & ~7;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    nm[e] = f2_pack(-__shfl_sync(0xffffffffu, mean, g0 + 2 * e), -__shfl_sync(0xffffffffu, mean, g0 + 2 * e + 1));
    acc[e] = 0ull;
  }
#pragma unroll 4
  for (int i = 0; i < CS; ++i) {
    const uint4 u = ld(i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const unsigned long long d = f2_add(f2_pack(E::lo(w[e]), E::hi(w[e])), nm[e]);
      acc[e] = f2_fma(d, d, acc[e]);
    }
  }
  rstd = rsqrtf(reduce8(acc) * (1.0f / C) + eps);
  return tg * 8 + cs;
}

// ===========================================================================
// input phase
// ===========================================================================
// epilogue warpgroups of the input phase (each takes C / kInEpiWG channels of a half)
#ifndef TOPS_IN_EPI_WG
#define TOPS_IN_EPI_WG 4
#endif
constexpr int kInEpiWG = TOPS_IN_EPI_WG;

template <int C>
struct TmInSmem {
  static constexpr int NOUT = 4 * C;
  static constexpr int TILE = (C / 64) * 16384;
  // weights per 64-channel K atom, rows reordered by halves: [P(0:C) G(0:C) P(C:2C) G(C:2C)]
  alignas(1024) uint8_t w[(C / 64) * NOUT * 128];
  alignas(1024) uint8_t x[2][TILE];
  // the LayerNorm terms as one more K step of 16 (K-major, 32-byte swizzle): per token
  // [-mean hi, -mean lo, -mean hi, 1/rstd hi, 1/rstd lo, 1/rstd hi, 0...] against, per
  // output channel, [sumW hi, sumW hi, sumW lo, Bc hi, Bc hi, Bc lo, 0...]
  alignas(1024) uint8_t aext[2][128 * 32];
  alignas(1024) uint8_t bext[2][2 * C * 32];
  // per epilogue warp: 8 channels x 32 tokens of the D-major output, stored by TMA
  alignas(128) uint8_t stage[4 * kInEpiWG][8 * 32 * 2];
  float rstd[2][128];
  uint64_t bar_w, x_full[2], x_empty[2], ext_full[2], st_ready[2], st_free[2], acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int abort;
};

// element k (< 8) of row r of a K-major 32-byte-swizzled tile of 16-bit values: byte offset
__device__ __forceinline__ uint32_t sw32_chunk_off(uint32_t r, uint32_t chunk) {
  return r * 32u + ((chunk ^ ((r >> 2) & 1u)) << 4);
}

// v = hi + lo in the 16-bit type (hi = v rounded, lo = the rounded remainder)
template <typename T>
__device__ __forceinline__ void split16(float v, uint16_t& hi, uint16_t& lo) {
  using E = Elem<T>;
  const T h = E::from_f(v);
  const T l = E::from_f(v - E::to_f(h));
  hi = *reinterpret_cast<const uint16_t*>(&h);
  lo = *reinterpret_cast<const uint16_t*>(&l);
}

// this token's row of a statistics K step: [-mean hi, -mean lo, -mean hi, 1/rstd hi, 1/rstd lo, 1/rstd hi, 0...]
template <typename T>
__device__ __forceinline__ void write_stats_row(uint8_t* tile, int row, float mean, float rstd) {
  uint16_t mh, ml, ih, il;
  split16<T>(-mean, mh, ml);
  split16<T>(1.0f / rstd, ih, il);
  *reinterpret_cast<uint4*>(tile + sw32_chunk_off(row, 0)) =
      make_uint4(mh | (static_cast<uint32_t>(ml) << 16), mh | (static_cast<uint32_t>(ih) << 16),
                 il | (static_cast<uint32_t>(ih) << 16), 0u);
  *reinterpret_cast<uint4*>(tile + sw32_chunk_off(row, 1)) = make_uint4(0u, 0u, 0u, 0u);
}

// an output channel's row of a statistics K step: [sumW hi, sumW hi, sumW lo, Bc hi, Bc hi, Bc lo, 0...]
template <typename T>
__device__ __forceinline__ void write_const_row(uint8_t* tile, int row, float sum_w, float b_const) {
  uint16_t sh, sl, bh, bl;
  split16<T>(sum_w, sh, sl);
  split16<T>(b_const, bh, bl);
  *reinterpret_cast<uint4*>(tile + sw32_chunk_off(row, 0)) =
      make_uint4(sh | (static_cast<uint32_t>(sh) << 16), sl | (static_cast<uint32_t>(bh) << 16),
                 bh | (static_cast<uint32_t>(bl) << 16), 0u);
  *reinterpret_cast<uint4*>(tile + sw32_chunk_off(row, 1)) = make_uint4(0u, 0u, 0u, 0u);
}

// Per 128-token tile the 2C outputs are produced in two halves of C channels: one
// MMA of N = 2C (P and G of the half) into one of two 2C-column TMEM accumulators,
// so the MMA of the next half overlaps the epilogue of the current one. The LayerNorm
// is folded into the GEMM: LN(x) W^T = rstd (x Wc^T - mean sumW + Bc / rstd), the
// bracket being the x MMAs plus one K step over the per-token statistics (split in
// 16-bit hi/lo pairs: fp32-exact products, fp32 accumulation), so the epilogue only
// scales by rstd.
template <typename T, int C>
__global__ void __launch_bounds__(128 + 128 + 128 * kInEpiWG, 1)
    trimul_in_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                     const __grid_constant__ CUtensorMap map_out, LnGateArgs a) {
  using E = Elem<T>;
  using S = TmInSmem<C>;
  constexpr int NOUT = S::NOUT;    // global weight rows: P [0, 2C), G [2C, 4C)
  constexpr int KATOMS = C / 64;
  constexpr int NH = 2 * C;        // accumulator columns per half: P(C) | G(C)
  static_assert(NH <= 256, "one MMA per half");
  extern __shared__ uint8_t smem_raw[];
  S& sm = *reinterpret_cast<S*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long n_tiles = (a.M + 127) / 128;
  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_w, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.x_full[s], 1);
      mbar_init(&sm.x_empty[s], 1 + 4);
      mbar_init(&sm.ext_full[s], 4);
      mbar_init(&sm.st_ready[s], 4);
      mbar_init(&sm.st_free[s], 4 * kInEpiWG);
      mbar_init(&sm.acc_full[s], 1);
      mbar_init(&sm.acc_empty[s], 4 * kInEpiWG);
    }
    sm.abort = 0;
    fence_mbar_init();
  }
  // the per-channel half of the LayerNorm K step (row n of half hh = output channel)
  for (int rr = threadIdx.x; rr < 2 * NH; rr += blockDim.x) {
    const int hh = rr / NH, n = rr % NH, is_g = n >= C;
    const int gidx = is_g * 2 * C + hh * C + (n - is_g * C);
    write_const_row<T>(sm.bext[hh], n, a.sum_w[gidx], a.b_const[gidx]);
  }
  fence_proxy_async_smem();
  if (warp == 1) tmem_alloc(&sm.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;
  volatile int* abort = &sm.abort;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&map_x);
      mbar_expect_tx(&sm.bar_w, KATOMS * NOUT * 128);
      // global row block r0 (C rows of P or G of one half) -> its place in the half-major order
      for (int ka = 0; ka < KATOMS; ++ka)
        for (int r0 = 0; r0 < NOUT; r0 += C) {
          const int is_g = r0 >= 2 * C, half = (r0 % (2 * C)) / C;
          const int dst_row = half * NH + is_g * C;
          tma_load_2d(sm.w + ka * NOUT * 128 + dst_row * 128, &map_w, &sm.bar_w, ka * 64, r0);
        }
      int it = 0;
      for (long long tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
        const int s = it & 1;
        if (!mbar_wait(&sm.x_empty[s], ((it >> 1) & 1) ^ 1, abort, 401)) break;
        mbar_expect_tx(&sm.x_full[s], S::TILE);
        for (int ka = 0; ka < KATOMS; ++ka)
          tma_load_2d(sm.x[s] + ka * 16384, &map_x, &sm.x_full[s], ka * 64, static_cast<int>(tile * 128));
        // the two-slot ring holds one tile in flight: keep a few more coming into L2
        const long long pf = tile + TOPS_L2_PREFETCH * static_cast<long long>(gridDim.x);
        if (TOPS_L2_PREFETCH > 0 && pf < n_tiles)
          for (int ka = 0; ka < KATOMS; ++ka) tma_prefetch_l2_2d(&map_x, ka * 64, static_cast<int>(pf * 128));
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(128, NH, E::kFmt, false, false);
      bool ok = mbar_wait(&sm.bar_w, 0, abort, 402);
      int it = 0;
      for (long long tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++it) {
        const int s = it & 1;
        if (!mbar_wait(&sm.x_full[s], (it >> 1) & 1, abort, 403)) break;
        const uint32_t xa = smem_u32(sm.x[s]), wa = smem_u32(sm.w);
        for (int hh = 0; hh < 2; ++hh) {
          const int u = 2 * it + hh, buf = u & 1;
          if (!mbar_wait(&sm.acc_empty[buf], ((u >> 1) & 1) ^ 1, abort, 404)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < C / 16; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            const uint32_t woff = (kk >> 2) * (NOUT * 128) + hh * NH * 128 + (kk & 3) * 32;
            mma_ss(tbase + buf * 256, make_smem_desc(xa + off, 16, 1024, kSw128),
                   make_smem_desc(wa + woff, 16, 1024, kSw128), idesc, kk > 0);
          }
          // the statistics K step, once the tile's statistics are in place
          if (hh == 0) {
            if (!mbar_wait(&sm.ext_full[s], (it >> 1) & 1, abort, 409)) { ok = false; break; }
            tc_fence_after();
          }
          mma_ss(tbase + buf * 256, make_smem_desc(smem_u32(sm.aext[s]), 16, 256, kSw32),
                 make_smem_desc(smem_u32(sm.bext[hh]), 16, 256, kSw32), idesc, 1u);
          mma_commit(&sm.acc_full[buf]);
        }
        if (!ok) break;
        mma_commit(&sm.x_empty[s]);
      }
    }
  } else if (warp >= 4 && warp < 8) {
    const int row = (warp - 4) * 32 + lane;
    int it = 0;
    for (long long tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
      const int s = it & 1;
      if (!mbar_wait(&sm.x_full[s], (it >> 1) & 1, abort, 405)) break;
      float mean, rstd;
      row_stats_kmajor<T, C>(sm.x[s], row, mean, rstd, a.eps);
      // this token's row of the statistics K step (the slot's previous MMAs are done:
      // x_full of this tile follows x_empty of the tile two back)
      write_stats_row<T>(sm.aext[s], row, mean, rstd);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.ext_full[s]);
        mbar_arrive(&sm.x_empty[s]);
      }
      if (!mbar_wait(&sm.st_free[s], ((it >> 1) & 1) ^ 1, abort, 406)) break;
      sm.rstd[s][row] = rstd;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.st_ready[s]);
    }
  } else if (warp >= 8) {
    // kInEpiWG epilogue warpgroups split the C channels of each half (a warp reaches only
    // its own 32 TMEM lanes, so the split is by columns). Each warp stages 8 channels x
    // its 32 tokens (the D-major layout of ab: one 64-byte row per channel) and stores
    // them with one TMA box; rows past M are clipped by the TMA unit.
    const int ew = (warp - 8) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_addr = tbase + (static_cast<uint32_t>(wq * 32) << 16);
    uint16_t* stage = reinterpret_cast<uint16_t*>(sm.stage[warp - 8]);
    bool ok = true;
    bool staged = false;  // a TMA store of this warp's stage buffer may still be reading it
    int it = 0;
    for (long long tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++it) {
      const int s = it & 1;
      if (!mbar_wait(&sm.st_ready[s], (it >> 1) & 1, abort, 407)) break;
      const float rstd = sm.rstd[s][row];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.st_free[s]);
      const long long m = tile * 128 + row;
      float mval = 1.0f;
      if (a.mask != nullptr && m < a.M) mval = static_cast<float>(static_cast<int8_t>(a.mask[m]));
      // per channel pair (k, k+1), in packed fp32 pairs (acc = x Wc^T - mean sumW + Bc/rstd):
      //   P' = rstd acc_p;  G/2 = rstd/2 acc_g;  out = (mval/2 + mval/2 tanh(G/2)) P' = mval sigmoid(G) P'
      const float hm = 0.5f * mval;
      const unsigned long long rs2 = f2_pack(rstd, rstd), rg2 = f2_pack(0.5f * rstd, 0.5f * rstd);
      const unsigned long long hm2 = f2_pack(hm, hm);
      for (int hh = 0; hh < 2; ++hh) {
        const int u = 2 * it + hh, buf = u & 1;
        if (!mbar_wait(&sm.acc_full[buf], (u >> 1) & 1, abort, 408)) { ok = false; break; }
        tc_fence_after();
        const uint32_t acc = lane_addr + buf * 256;
        // 8-channel steps, each step's TMEM loads issued before the previous step's math
        constexpr int NSTEP = C / kInEpiWG / 8;
        const int cbase = ew * (C / kInEpiWG);
        uint32_t pg[16], nxt[16];  // P then G of 8 channels
        tmem_ld8x2_async(acc + cbase, acc + C + cbase, pg);
        tmem_wait_ld16(pg);
#pragma unroll
        for (int j = 0; j < NSTEP; ++j) {
          const int c0 = cbase + 8 * j;
          const bool more = j + 1 < NSTEP;
          if (more) tmem_ld8x2_async(acc + c0 + 8, acc + C + c0 + 8, nxt);
          uint32_t pk[4];  // channel pairs (c0 + 2t, c0 + 2t + 1) of this token
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const unsigned long long pv = f2_mul(rs2, f2_pack(__uint_as_float(pg[2 * t]), __uint_as_float(pg[2 * t + 1])));
            const unsigned long long gh =
                f2_mul(rg2, f2_pack(__uint_as_float(pg[8 + 2 * t]), __uint_as_float(pg[8 + 2 * t + 1])));
            float g0, g1;
            f2_unpack(gh, g0, g1);
            const unsigned long long v = f2_mul(f2_fma(f2_pack(tanh_approx(g0), tanh_approx(g1)), hm2, hm2), pv);
            float v0, v1;
            f2_unpack(v, v0, v1);
            pk[t] = E::pack2(v0, v1);
          }
          // stage the 8 channels (once the previous box has left the buffer) and store them
          if (staged && lane == 0) bulk_wait_read0();
          __syncwarp();
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            stage[(2 * t) * 32 + lane] = static_cast<uint16_t>(pk[t] & 0xFFFFu);
            stage[(2 * t + 1) * 32 + lane] = static_cast<uint16_t>(pk[t] >> 16);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&map_out, stage, static_cast<int>(tile * 128 + wq * 32), hh * C + c0);
            bulk_commit();
          }
          staged = true;
          if (more) {
            tmem_wait_ld16(nxt);
#pragma unroll
            for (int t = 0; t < 16; ++t) pg[t] = nxt[t];
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
      }
    }
    if (lane == 0) bulk_wait0();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

// ===========================================================================
// contraction (per-channel batched GEMM, 256 x 256 tiles, BK = 64, 3 stages)
// ===========================================================================
// A 256 x 256 tile is two M=128 MMAs sharing each B tile: 2 x 256 TMEM columns
// (all of TMEM, one accumulator pair). The larger tile halves the operand bytes per
// FLOP against 128 x 256, which is what the stage ring can keep in flight from L2;
// the accumulator is not double-buffered. The epilogue (8 warps, one per TMEM lane
// quarter and row half) stages each 32 x 32 chunk of y in shared memory (64-byte
// swizzle) and writes it with one TMA store, so a warp's stores are 2 KB boxes rather
// than 32 scattered row segments, and it releases the accumulator after its last TMEM
// load, before the stores drain.
constexpr int kCtBM = 256, kCtBN = 256, kCtBK = 64, kCtStages = 3;
constexpr int kCtStageBytes = 32 * 32 * 2;  // one warp's 32 rows x 32 columns of y

struct CtSmem {
  alignas(1024) uint8_t a[kCtStages][kCtBM * kCtBK * 2];
  alignas(1024) uint8_t b[kCtStages][kCtBN * kCtBK * 2];
  alignas(1024) uint8_t ystage[8][2][kCtStageBytes];  // [epilogue warp][double buffer]
  uint64_t full[kCtStages], empty[kCtStages], acc_full, acc_empty;
  uint32_t tmem_base;
  int abort;
};

struct CtArgs {
  int L, nb;
  void* y;  // [nb][Mi][L]
  int Mi;   // rows of A / y (L unsharded; a row slab of size L/P when sharded)
  int nc;   // extent of one B chunk along j (B is P rank-major chunks of nc columns; nc = L unsharded)
  int j_base, j_end;  // the launch computes output columns [j_base, j_end) only (j_base % kCtBN == 0)
  int a_grouped;      // MN-major A: 1 = a 4-D map whose one box is the whole tile, 0 = one 3-D box per 64 rows
  int b_one;          // B: 1 = one box per stage (the tile never straddles a chunk), 0 = one per 128 / 64 rows
};

template <typename T, bool MN>
__global__ void __launch_bounds__(384, 1)
    trimul_contract_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                           const __grid_constant__ CUtensorMap map_y, CtArgs a) {
  using E = Elem<T>;
  extern __shared__ uint8_t smem_raw[];
  CtSmem& sm = *reinterpret_cast<CtSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nI = (a.Mi + kCtBM - 1) / kCtBM, nJ = (a.j_end - a.j_base + kCtBN - 1) / kCtBN;
  const long long n_tiles = static_cast<long long>(nI) * nJ * a.nb;
  const int nk = (a.L + kCtBK - 1) / kCtBK;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kCtStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.acc_full, 1);
    mbar_init(&sm.acc_empty, 8);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&sm.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;
  volatile int* abort = &sm.abort;
  auto decode = [&](long long tile, int& bb, int& i0, int& j0) {
    const int per_b = nI * nJ;
    bb = static_cast<int>(tile / per_b);
    const int r = static_cast<int>(tile - static_cast<long long>(bb) * per_b);
    i0 = (r / nJ) * kCtBM;
    j0 = a.j_base + (r % nJ) * kCtBN;
  };

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&map_a);
      tma_prefetch_desc(&map_b);
      int g = 0;  // global k-block counter (stage ring position)
      for (long long tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        int bb, i0, j0;
        decode(tile, bb, i0, j0);
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % kCtStages;
          if (!mbar_wait(&sm.empty[s], ((g / kCtStages) & 1) ^ 1, abort, 501)) { ok = false; break; }
          mbar_expect_tx(&sm.full[s], (kCtBM + kCtBN) * kCtBK * 2);
          const int k0 = kb * kCtBK;
          if (!MN) {
            tma_load_3d(sm.a[s], &map_a, &sm.full[s], k0, i0, bb);
            // B rows j live in rank-major chunks of nc rows: (j mod nc, chunk j / nc);
            // j >= L lands on chunk >= P, which the tensor map zero-fills.
            if (a.b_one) {
              const int ch = j0 / a.nc;
              tma_load_4d(sm.b[s], &map_b, &sm.full[s], k0, j0 - ch * a.nc, bb, ch);
            } else {
              for (int h = 0; h < kCtBN / 128; ++h) {
                const int j = j0 + h * 128, ch = j / a.nc;
                tma_load_4d(sm.b[s] + h * 16384, &map_b, &sm.full[s], k0, j - ch * a.nc, bb, ch);
              }
            }
          } else {
            if (a.a_grouped)
              tma_load_4d(sm.a[s], &map_a, &sm.full[s], 0, k0, i0 / 64, bb);
            else
              for (int h = 0; h < kCtBM / 64; ++h) tma_load_3d(sm.a[s] + h * 8192, &map_a, &sm.full[s], i0 + h * 64, k0, bb);
            if (a.b_one) {
              const int ch = j0 / a.nc;
              tma_load_5d(sm.b[s], &map_b, &sm.full[s], 0, k0, (j0 - ch * a.nc) / 64, bb, ch);
            } else {
              for (int h = 0; h < kCtBN / 64; ++h) {
                const int j = j0 + h * 64, ch = j / a.nc;
                tma_load_4d(sm.b[s] + h * 8192, &map_b, &sm.full[s], j - ch * a.nc, k0, bb, ch);
              }
            }
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(128, kCtBN, E::kFmt, MN, MN);
      int g = 0, it = 0;
      bool ok = true;
      for (long long tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++it) {
        if (!mbar_wait(&sm.acc_empty, (it & 1) ^ 1, abort, 502)) break;
        tc_fence_after();
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % kCtStages;
          if (!mbar_wait(&sm.full[s], (g / kCtStages) & 1, abort, 503)) { ok = false; break; }
          tc_fence_after();
          const uint32_t aa = smem_u32(sm.a[s]), ba = smem_u32(sm.b[s]);
#pragma unroll
          for (int kk = 0; kk < kCtBK / 16; ++kk) {
            const uint64_t bd = MN ? make_smem_desc(ba + kk * 2048, 8192, 1024, kSw128)
                                   : make_smem_desc(ba + kk * 32, 16, 1024, kSw128);
#pragma unroll
            for (int m = 0; m < 2; ++m) {  // rows [128m, 128m + 128): 16 KB into the A tile either way
              const uint64_t ad = MN ? make_smem_desc(aa + m * 16384 + kk * 2048, 8192, 1024, kSw128)
                                     : make_smem_desc(aa + m * 16384 + kk * 32, 16, 1024, kSw128);
              mma_ss(tbase + m * 256, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            }
          }
          mma_commit(&sm.empty[s]);
        }
        if (ok) mma_commit(&sm.acc_full);
      }
    }
  } else if (warp >= 4) {
    // 8 epilogue warps: row half m = (warp - 4) / 4 (its accumulator), lane quarter warp % 4
    const int m = (warp - 4) >> 2, wq = warp & 3;
    const int row = m * 128 + wq * 32 + lane;
    const uint32_t lane_addr = tbase + m * 256 + (static_cast<uint32_t>(wq * 32) << 16);
    uint8_t* stage0 = sm.ystage[warp - 4][0];
    // 64-byte swizzle: the 16-byte chunk q of row r sits at chunk q ^ ((r >> 1) & 3)
    const int sw = (lane >> 1) & 3;
    int it = 0, nst = 0;
    for (long long tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
      if (!mbar_wait(&sm.acc_full, it & 1, abort, 504)) break;
      tc_fence_after();
      int bb, i0, j0;
      decode(tile, bb, i0, j0);
      const int i = i0 + row, r0 = i0 + m * 128 + wq * 32;
      T* dst = static_cast<T*>(a.y) + (static_cast<size_t>(bb) * a.Mi + i) * a.L + j0;
#pragma unroll 1
      for (int c0 = 0; c0 < kCtBN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(lane_addr + c0, r);
        if (c0 + 32 == kCtBN) {  // the accumulator is free once its last columns are in registers
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.acc_empty);
        }
        if (r0 >= a.Mi) continue;
        uint32_t p[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) p[e] = E::pack2(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]));
        if (j0 + c0 + 32 <= a.j_end) {
          uint8_t* buf = stage0 + (nst & 1) * kCtStageBytes;
          if (lane == 0) bulk_wait_read1();  // the store that last read this buffer is done reading
          __syncwarp();
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(buf + lane * 64 + ((q ^ sw) << 4)) =
                make_uint4(p[4 * q], p[4 * q + 1], p[4 * q + 2], p[4 * q + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&map_y, buf, j0 + c0, r0, bb);  // rows >= Mi are clipped by the map
            bulk_commit();
          }
          ++nst;
        } else if (i < a.Mi) {
          for (int e = 0; e < 32; ++e)
            if (j0 + c0 + e < a.j_end) dst[c0 + e] = E::from_f(__uint_as_float(r[e]));
        }
      }
    }
    if (lane == 0) bulk_wait0();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

// ===========================================================================
// output phase
// ===========================================================================
// output phase warp roles after the producer / MMA warps (0-3): kOutStatWG statistics
// warpgroups, then kOutEpiWG epilogue warpgroups (kOutStatWG + kOutEpiWG = 3: 512 threads)
#ifndef TOPS_OUT_STAT_WG
#define TOPS_OUT_STAT_WG 2
#endif
constexpr int kOutStatWG = TOPS_OUT_STAT_WG;
constexpr int kOutEpiWG = 3 - kOutStatWG;

template <int C>
struct TmOutSmem {
  static constexpr int TILE = (C / 64) * 16384;
  alignas(1024) uint8_t w[2 * (C / 64) * C * 128];  // p_out rows [0,C), g_out rows [C,2C); per K atom
  alignas(1024) uint8_t y[2][TILE];                 // MN-major: two 64-token halves x C rows
  alignas(1024) uint8_t x[2][TILE];                 // K-major
  // the two LayerNorms as one more K step each (K-major, 32-byte swizzle), as in the
  // input phase: per token [-mean hi, -mean lo, -mean hi, 1/rstd hi, 1/rstd lo, 1/rstd hi]
  // of y (P) and of x (G), against per output channel [sumW hi, sumW hi, sumW lo, Bc hi, Bc hi, Bc lo]
  alignas(1024) uint8_t aext[2][2][128 * 32];        // [slot][y | x]
  alignas(1024) uint8_t bext[2][C * 32];             // [p_out | g_out]
  float st[2][2][128];                               // rstd_y, rstd_x
  uint64_t bar_w, in_full[2], in_empty[2], ext_full[2], st_ready[2], st_free[2], acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int abort;
};

template <typename T, int C>
__global__ void __launch_bounds__(512, 1)
    trimul_out_kernel(const __grid_constant__ CUtensorMap map_y, const __grid_constant__ CUtensorMap map_x,
                      const __grid_constant__ CUtensorMap map_w, LnGateArgs a) {
  using E = Elem<T>;
  using S = TmOutSmem<C>;
  constexpr int KATOMS = C / 64;
  extern __shared__ uint8_t smem_raw[];
  S& sm = *reinterpret_cast<S*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long n_tiles = (a.M + 127) / 128;
  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_w, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.in_full[s], 1);
      mbar_init(&sm.in_empty[s], 1 + 4 * kOutStatWG);
      mbar_init(&sm.ext_full[s], 4 * kOutStatWG);
      mbar_init(&sm.st_ready[s], 4 * kOutStatWG);
      mbar_init(&sm.st_free[s], 4 * kOutEpiWG);
      mbar_init(&sm.acc_full[s], 1);
      mbar_init(&sm.acc_empty[s], 4 * kOutEpiWG);
    }
    sm.abort = 0;
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < 2 * C; i += blockDim.x) write_const_row<T>(sm.bext[i / C], i % C, a.sum_w[i], a.b_const[i]);
  fence_proxy_async_smem();
  if (warp == 1) tmem_alloc(&sm.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;
  volatile int* abort = &sm.abort;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&map_y);
      tma_prefetch_desc(&map_x);
      mbar_expect_tx(&sm.bar_w, 2 * KATOMS * C * 128);
      for (int ka = 0; ka < KATOMS; ++ka) tma_load_2d(sm.w + ka * 2 * C * 128, &map_w, &sm.bar_w, ka * 64, 0);
      int it = 0;
      for (long long tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
        const int s = it & 1;
        if (!mbar_wait(&sm.in_empty[s], ((it >> 1) & 1) ^ 1, abort, 601)) break;
        mbar_expect_tx(&sm.in_full[s], 2 * S::TILE);
        const int m0 = static_cast<int>(tile * 128);
        for (int h = 0; h < 2; ++h) tma_load_2d(sm.y[s] + h * C * 128, &map_y, &sm.in_full[s], m0 + h * 64, 0);
        for (int ka = 0; ka < KATOMS; ++ka) tma_load_2d(sm.x[s] + ka * 16384, &map_x, &sm.in_full[s], ka * 64, m0);
        const long long pf = tile + TOPS_L2_PREFETCH * static_cast<long long>(gridDim.x);
        if (TOPS_L2_PREFETCH > 0 && pf < n_tiles) {
          const int p0 = static_cast<int>(pf * 128);
          for (int h = 0; h < 2; ++h) tma_prefetch_l2_2d(&map_y, p0 + h * 64, 0);
          for (int ka = 0; ka < KATOMS; ++ka) tma_prefetch_l2_2d(&map_x, ka * 64, p0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_y = make_idesc_f16(128, C, E::kFmt, true, false);
      const uint32_t id_x = make_idesc_f16(128, C, E::kFmt, false, false);
      bool ok = mbar_wait(&sm.bar_w, 0, abort, 602);
      int it = 0;
      for (long long tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++it) {
        const int s = it & 1;
        if (!mbar_wait(&sm.in_full[s], (it >> 1) & 1, abort, 603)) break;
        if (!mbar_wait(&sm.acc_empty[s], ((it >> 1) & 1) ^ 1, abort, 604)) break;
        tc_fence_after();
        const uint32_t ya = smem_u32(sm.y[s]), xa = smem_u32(sm.x[s]), wa = smem_u32(sm.w);
        const uint32_t acc = tbase + s * 256;
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk) {
          const uint32_t woff = (kk >> 2) * (2 * C * 128) + (kk & 3) * 32;
          // P = y (MN-major, K = channel d) x p_out^T
          mma_ss(acc, make_smem_desc(ya + kk * 2048, C * 128, 1024, kSw128),
                 make_smem_desc(wa + woff, 16, 1024, kSw128), id_y, kk > 0);
          // G = x (K-major) x g_out^T
          mma_ss(acc + C, make_smem_desc(xa + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024, kSw128),
                 make_smem_desc(wa + woff + C * 128, 16, 1024, kSw128), id_x, kk > 0);
        }
        // the LayerNorm K steps (K-major), once the tile's statistics are in place
        if (!mbar_wait(&sm.ext_full[s], (it >> 1) & 1, abort, 609)) break;
        tc_fence_after();
        mma_ss(acc, make_smem_desc(smem_u32(sm.aext[s][0]), 16, 256, kSw32),
               make_smem_desc(smem_u32(sm.bext[0]), 16, 256, kSw32), id_x, 1u);
        mma_ss(acc + C, make_smem_desc(smem_u32(sm.aext[s][1]), 16, 256, kSw32),
               make_smem_desc(smem_u32(sm.bext[1]), 16, 256, kSw32), id_x, 1u);
        mma_commit(&sm.in_empty[s]);
        mma_commit(&sm.acc_full[s]);
      }
    }
  } else if (warp >= 4 && warp < 4 + 4 * kOutStatWG) {
    // statistics: one warpgroup for both LayerNorms, or one for y and one for x
    const bool do_y = kOutStatWG == 1 || warp < 8, do_x = kOutStatWG == 1 || warp >= 8;
    const int row = (warp & 3) * 32 + lane;
    int it = 0;
    for (long long tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
      const int s = it & 1;
      if (!mbar_wait(&sm.in_full[s], (it >> 1) & 1, abort, 605)) break;
      float my = 0.f, ry = 1.f, mx = 0.f, rx = 1.f;
      int ytok = row;
      if (do_y) ytok = col_stats_coop<T, C>(sm.y[s], row, my, ry, a.eps);
      if (do_x) row_stats_kmajor<T, C>(sm.x[s], row, mx, rx, a.eps);
      // the slot's statistics rows (its previous MMAs are done: in_full of this tile
      // follows in_empty of the tile two back)
      if (do_y) write_stats_row<T>(sm.aext[s][0], ytok, my, ry);
      if (do_x) write_stats_row<T>(sm.aext[s][1], row, mx, rx);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.ext_full[s]);
        mbar_arrive(&sm.in_empty[s]);
      }
      if (!mbar_wait(&sm.st_free[s], ((it >> 1) & 1) ^ 1, abort, 606)) break;
      if (do_y) sm.st[s][0][ytok] = ry;
      if (do_x) sm.st[s][1][row] = rx;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.st_ready[s]);
    }
  } else if (warp >= 4 + 4 * kOutStatWG) {
    // kOutEpiWG epilogue warpgroups split the C output columns of every tile
    constexpr int CW = C / kOutEpiWG;
    const int ew = (warp - 4 - 4 * kOutStatWG) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_addr = tbase + (static_cast<uint32_t>(wq * 32) << 16);
    int it = 0;
    for (long long tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
      const int s = it & 1;
      if (!mbar_wait(&sm.st_ready[s], (it >> 1) & 1, abort, 607)) break;
      const float ry = sm.st[s][0][row], rx = sm.st[s][1][row];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.st_free[s]);
      if (!mbar_wait(&sm.acc_full[s], (it >> 1) & 1, abort, 608)) break;
      tc_fence_after();
      const long long m = tile * 128 + row;
      T* dst = static_cast<T*>(a.out) + m * C;
      const T* res = a.residual != nullptr ? static_cast<const T*>(a.residual) + m * C : nullptr;
      // acc = z Wc^T - mean sumW + Bc / rstd for z = y (P) and x (G):
      //   P' = rstd_y acc_p;  G/2 = rstd_x/2 acc_g;  out = (1/2 + 1/2 tanh(G/2)) P' (+ residual)
      const unsigned long long ry2 = f2_pack(ry, ry), rx2 = f2_pack(0.5f * rx, 0.5f * rx);
      const unsigned long long half2 = f2_pack(0.5f, 0.5f);
      const uint32_t acc = lane_addr + s * 256;
      // chunk loads (P then G of 16 columns) one chunk ahead of the math
      uint32_t pg[32], nxt[32];
      tmem_ld16x2_async(acc + ew * CW, acc + C + ew * CW, pg);
      tmem_wait_ld32(pg);
      for (int c0 = ew * CW; c0 < (ew + 1) * CW; c0 += 16) {
        const bool more = c0 + 16 < (ew + 1) * CW;
        if (more) tmem_ld16x2_async(acc + c0 + 16, acc + C + c0 + 16, nxt);
        if (m < a.M) {
#pragma unroll
          for (int sub = 0; sub < 16; sub += 8) {
            const int cc = c0 + sub;
            uint32_t rs[4];
            if (res != nullptr) {
              const uint4 u = *reinterpret_cast<const uint4*>(res + cc);
              rs[0] = u.x;
              rs[1] = u.y;
              rs[2] = u.z;
              rs[3] = u.w;
            }
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = sub + 2 * e;
              const unsigned long long pv = f2_mul(ry2, f2_pack(__uint_as_float(pg[i]), __uint_as_float(pg[i + 1])));
              const unsigned long long gh =
                  f2_mul(rx2, f2_pack(__uint_as_float(pg[16 + i]), __uint_as_float(pg[16 + i + 1])));
              float g0, g1;
              f2_unpack(gh, g0, g1);
              unsigned long long v = f2_mul(f2_fma(f2_pack(tanh_approx(g0), tanh_approx(g1)), half2, half2), pv);
              if (res != nullptr) v = f2_add(v, f2_pack(E::lo(rs[e]), E::hi(rs[e])));
              float v0, v1;
              f2_unpack(v, v0, v1);
              o[e] = E::pack2(v0, v1);
            }
            *reinterpret_cast<uint4*>(dst + cc) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
        if (more) {
          tmem_wait_ld32(nxt);
#pragma unroll
          for (int i = 0; i < 32; ++i) pg[i] = nxt[i];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[s]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

}  // namespace tops
