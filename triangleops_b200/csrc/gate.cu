// gate.cu — fused gate + output projection (tcgen05, persistent):
//
//   out[t,:] = ( O[t,:] * sigmoid(gin[t,:] Wg^T + bg) ) Wo^T + bo
//
// triangle attention: gin = LN(x), no biases  [triangle_attn/kernel.py:387-470]
// attention_pair_bias: gin = X (raw), biases   [attn_pair_bias/module.py:65-66]
//
// Per 128-token tile: MMA1 acc1 = gin Wg^T (TMEM); a warpgroup turns acc1 into the
// gate, multiplies the attention output O (read from the same shared-memory stage),
// rounds to the IO dtype — the rounding point of the reference — and writes the
// product over the gin tile (gin is dead once MMA1 completes); MMA2 acc2 = that
// product times Wo^T; the warpgroup adds bo (and optionally a residual: the
// Pairformer update x += op(x), in place) and stores, optionally transposed. Two pairs of warpgroups
// alternate tiles, each pair with its own TMEM accumulator pair and each warpgroup of
// a pair taking half of the C channels, and MMA1 of the next tile is
// issued before MMA2 of the current one so the tensor core never waits on a gate.
#include "sm100.cuh"

namespace tops {

template <int C>
struct GateCfg {
  static constexpr int KATOMS = C / 64;
  static constexpr int TILE = KATOMS * 16384;  // one 128 x C operand tile
  static constexpr int W = KATOMS * C * 128;   // one C x C weight
};

template <int C>
struct GateSmem {
  using Cfg = GateCfg<C>;
  alignas(1024) uint8_t wg[Cfg::W];
  alignas(1024) uint8_t wo[Cfg::W];
  alignas(1024) uint8_t gin[2][Cfg::TILE];
  alignas(1024) uint8_t o[2][Cfg::TILE];
  uint64_t bar_w;
  uint64_t in_full[2], in_empty[2], acc1_full[2], a2_ready[2], acc2_full[2], acc_free[2];
  uint32_t tmem_base;
  int abort;
};

struct GateArgs {
  int T;
  const float* bg;  // [C] or nullptr
  const float* bo;  // [C] or nullptr
  void* out;        // [T][C]
  const void* residual;  // nullptr, or added to the result; same indexing as out (may alias out)
  int trans_n;      // 0: token t -> out row t. n > 0: token t = i*n + k -> out row k*n + i
                    // (the ending-node result written back in the untransposed pair layout)
};

template <typename T, int C>
__global__ void __launch_bounds__(640, 1)
    gate_kernel(const __grid_constant__ CUtensorMap map_gin, const __grid_constant__ CUtensorMap map_o,
                const __grid_constant__ CUtensorMap map_wg, const __grid_constant__ CUtensorMap map_wo, GateArgs a) {
  using Cfg = GateCfg<C>;
  using E = Elem<T>;
  extern __shared__ uint8_t smem_raw[];
  auto& sm = *reinterpret_cast<GateSmem<C>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (a.T + 127) / 128;

  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_w, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.in_full[s], 1);
      mbar_init(&sm.in_empty[s], 1);
      mbar_init(&sm.acc1_full[s], 1);
      mbar_init(&sm.a2_ready[s], 8);
      mbar_init(&sm.acc2_full[s], 1);
      mbar_init(&sm.acc_free[s], 8);
    }
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&sm.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;
  volatile int* abort = &sm.abort;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&map_gin);
      tma_prefetch_desc(&map_o);
      mbar_expect_tx(&sm.bar_w, 2 * Cfg::W);
      for (int ka = 0; ka < Cfg::KATOMS; ++ka) {
        tma_load_2d(sm.wg + ka * C * 128, &map_wg, &sm.bar_w, ka * 64, 0);
        tma_load_2d(sm.wo + ka * C * 128, &map_wo, &sm.bar_w, ka * 64, 0);
      }
      pdl_wait();  // O and x~ come from the kernels before this one
      int it = 0;
      for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
        const int s = it & 1;
        if (!mbar_wait(&sm.in_empty[s], ((it >> 1) & 1) ^ 1, abort, 301)) break;
        mbar_expect_tx(&sm.in_full[s], 2 * Cfg::TILE);
        for (int ka = 0; ka < Cfg::KATOMS; ++ka) {
          tma_load_2d(sm.gin[s] + ka * 16384, &map_gin, &sm.in_full[s], ka * 64, tile * 128);
          tma_load_2d(sm.o[s] + ka * 16384, &map_o, &sm.in_full[s], ka * 64, tile * 128);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(128, C, E::kFmt, false, false);
      bool ok = mbar_wait(&sm.bar_w, 0, abort, 302);
      auto gemm = [&](uint32_t d_tmem, const uint8_t* a_tile, const uint8_t* w) {
        const uint32_t aa = smem_u32(a_tile), wa = smem_u32(w);
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          const uint32_t woff = (kk >> 2) * (C * 128) + (kk & 3) * 32;
          mma_ss(d_tmem, make_smem_desc(aa + off, 16, 1024, kSw128), make_smem_desc(wa + woff, 16, 1024, kSw128),
                 idesc, kk > 0);
        }
      };
      auto issue1 = [&](int it) -> bool {
        const int s = it & 1;
        if (!mbar_wait(&sm.in_full[s], (it >> 1) & 1, abort, 303)) return false;
        if (!mbar_wait(&sm.acc_free[s], ((it >> 1) & 1) ^ 1, abort, 304)) return false;
        tc_fence_after();
        gemm(tbase + s * 256, sm.gin[s], sm.wg);
        mma_commit(&sm.acc1_full[s]);
        return true;
      };
      const int my_tiles = blockIdx.x < n_tiles ? (n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
      if (ok && my_tiles > 0) ok = issue1(0);
      for (int it = 0; ok && it < my_tiles; ++it) {
        const int s = it & 1;
        if (it + 1 < my_tiles && !issue1(it + 1)) break;
        if (!mbar_wait(&sm.a2_ready[s], (it >> 1) & 1, abort, 305)) break;
        tc_fence_after();
        gemm(tbase + s * 256 + 128, sm.gin[s], sm.wo);
        mma_commit(&sm.acc2_full[s]);
        mma_commit(&sm.in_empty[s]);
      }
    }
  } else if (warp >= 4) {
    pdl_wait();  // the residual may be the previous kernel's output
    const int wg = (warp - 4) >> 3;           // tile slot (alternate tiles)
    const int wq = warp & 3;
    const int half = ((warp - 4) >> 2) & 1;  // column half of the slot's tile
    const int row = wq * 32 + lane;
    const uint32_t lane_addr = tbase + (static_cast<uint32_t>(wq * 32) << 16);
    int it = wg;
    for (int tile = blockIdx.x + wg * gridDim.x; tile < n_tiles; tile += 2 * gridDim.x, it += 2) {
      const int s = it & 1;  // == wg
      const uint32_t acc1 = lane_addr + s * 256, acc2 = acc1 + 128;
      if (!mbar_wait(&sm.acc1_full[s], (it >> 1) & 1, abort, 306)) break;
      tc_fence_after();
      uint8_t* gtile = sm.gin[s];
      const uint8_t* otile = sm.o[s];
#pragma unroll 1
      for (int c0 = half * (C / 2); c0 < (half + 1) * (C / 2); c0 += 32) {
        uint32_t r[32];
        tmem_ld32(acc1 + c0, r);
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          const int c = c0 + ch * 8;
          const uint32_t off = (c >> 6) * 16384 + sw128_off(row, (c & 63) >> 3);
          const uint4 ou = *reinterpret_cast<const uint4*>(otile + off);
          const uint32_t o4[4] = {ou.x, ou.y, ou.z, ou.w};
          uint32_t w4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int cc = c + 2 * e;
            float g0 = __uint_as_float(r[ch * 8 + 2 * e]), g1 = __uint_as_float(r[ch * 8 + 2 * e + 1]);
            if (a.bg != nullptr) {
              g0 += __ldg(a.bg + cc);
              g1 += __ldg(a.bg + cc + 1);
            }
            w4[e] = E::pack2(E::lo(o4[e]) * sigmoid_fast(g0), E::hi(o4[e]) * sigmoid_fast(g1));
          }
          *reinterpret_cast<uint4*>(gtile + off) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.a2_ready[s]);
      if (!mbar_wait(&sm.acc2_full[s], (it >> 1) & 1, abort, 307)) break;
      tc_fence_after();
      const long long tok = static_cast<long long>(tile) * 128 + row;
      long long orow = tok;
      if (a.trans_n > 0) {
        const long long i = tok / a.trans_n;
        orow = (tok - i * a.trans_n) * a.trans_n + i;
      }
      T* dst = static_cast<T*>(a.out) + orow * C;
      const T* res = a.residual != nullptr ? static_cast<const T*>(a.residual) + orow * C : nullptr;
#pragma unroll 1
      for (int c0 = half * (C / 2); c0 < (half + 1) * (C / 2); c0 += 32) {
        uint32_t r[32];
        tmem_ld32(acc2 + c0, r);
        if (tok < a.T) {
          uint32_t rs[16];
          if (res != nullptr) {
            const uint4* r4 = reinterpret_cast<const uint4*>(res + c0);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 u = r4[q];
              rs[4 * q] = u.x;
              rs[4 * q + 1] = u.y;
              rs[4 * q + 2] = u.z;
              rs[4 * q + 3] = u.w;
            }
          }
          uint32_t p[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float v0 = __uint_as_float(r[2 * e]), v1 = __uint_as_float(r[2 * e + 1]);
            if (a.bo != nullptr) {
              v0 += __ldg(a.bo + c0 + 2 * e);
              v1 += __ldg(a.bo + c0 + 2 * e + 1);
            }
            if (res != nullptr) {
              v0 += E::lo(rs[e]);
              v1 += E::hi(rs[e]);
            }
            p[e] = E::pack2(v0, v1);
          }
          uint4* d4 = reinterpret_cast<uint4*>(dst + c0);
#pragma unroll
          for (int q = 0; q < 4; ++q) d4[q] = make_uint4(p[4 * q], p[4 * q + 1], p[4 * q + 2], p[4 * q + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_free[s]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

}  // namespace tops
