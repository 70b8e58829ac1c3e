// proj.cu — token projection for the attention ops (tcgen05, persistent).
//
// For a stream of T tokens x[t, 0:C) (token t = (row i, position k), t = i*Nk + k)
// one kernel produces everything the attention kernel consumes:
//
//   x~  = LN(x) (optional; eps, affine w/b; rounded to the IO dtype and also
//         written out for the gate stage)                [triangle_attn/module.py:73-79]
//   Q   = (x~ WQ) * scale   -> Q [R][H][Nk][D]  f16      [triangle_attn/kernel.py:194-195]
//                              (callers pass scale * log2(e): the attention works in log2 units)
//   K   =  x~ WK            -> K [R][H][Nk][D]  f16
//                              (Q, K, V^T are f16 whatever the IO dtype: they are LN-scale
//                              projections, and f16 keeps three more mantissa bits than bf16)
//   V   =  x~ WV            -> Vt[R][H][D][Nkp]  f16 (transposed)
//   pen = mask[i,k] ? 0 : -inf -> pen[R][Nkp]     f16 key penalty (only when a mask is given)
//   Bp  = (x~ WZ^T + BZ) * log2(e) -> Bp[H][R][Nkp] f16 (optional) [triangle_attn/kernel.py:36-98]
//
// One GEMM per 128-token tile: x~ (128 x C, K-major, SW128) times the resident
// concatenated weight Wcat (NOUT x C, K-major, SW128) into a TMEM accumulator of
// NOUT fp32 columns. Warp roles: w0 TMA producer, w1 MMA issuer, w4-7 LayerNorm
// (in place in shared memory), w8-15 epilogue (TMEM -> global; two warpgroups, half the heads each).
#include "sm100.cuh"

namespace tops {

template <int C, bool HAS_BP>
struct ProjCfg {
  static constexpr int KATOMS = C / 64;                 // 64-element (128 B) swizzle atoms along K
  static constexpr int NOUT = 3 * C + (HAS_BP ? 16 : 0);
  static constexpr int N0 = NOUT > 256 ? 256 : NOUT;    // first MMA chunk
  static constexpr int N1 = NOUT - N0;                  // second MMA chunk (0 if none)
  static constexpr int WBOX = NOUT > 256 ? NOUT / 2 : NOUT;  // rows per weight TMA box
  static constexpr int XSTAGE = KATOMS * 128 * 128;     // bytes of one x tile
  static constexpr int WBYTES = KATOMS * NOUT * 128;
  static constexpr int TMEM_COLS = NOUT <= 256 ? 256 : 512;
  static_assert(NOUT % 16 == 0 && N1 % 16 == 0, "MMA N must be a multiple of 16");
  static_assert(WBOX % 8 == 0 && WBOX <= 256, "weight box");
};

struct ProjArgs {
  int T;        // tokens
  int Nk;       // positions per row
  int R;        // rows (T = R * Nk)
  int Nkp;      // padded position stride of Vt / pen / Bp (multiple of 8)
  float scale;  // applied to Q
  float eps;
  const float* ln_w;   // [C] fp32 (HAS_LN)
  const float* ln_b;   // [C] fp32 (HAS_LN)
  const float* bz;     // [H] fp32 (HAS_BP)
  const uint8_t* mask; // [R][Nk] (nullptr = all ones)
  void* xln_out;       // [T][C] (nullptr = do not write)
  void* q;
  void* k;
  void* vt;
  void* pen;           // [R][Nkp] f16 (nullptr = not written)
  void* bp;
  int trans;           // 1: token (i, k) is x[k][i] of a square [Nk][Nk] pair array (ending node)
  int pdl;             // 1: launched to run beside the previous kernel (it reads none of that
                       // kernel's results); the CTAs exit only once that kernel has completed
};

// Token tiles. Row-major input: 128 consecutive tokens of the flattened stream.
// Transposed input: tiles never straddle a row i, so that one 3-D TMA box (128
// positions k of column i, stride Nk*C) fills the tile; the last tile of a row is ragged.
__device__ __forceinline__ int proj_tiles(const ProjArgs& a) {
  return a.trans ? a.R * ((a.Nk + 127) / 128) : (a.T + 127) / 128;
}
__device__ __forceinline__ long long proj_token(const ProjArgs& a, int tile, int row, bool& valid) {
  if (a.trans) {
    const int tpr = (a.Nk + 127) / 128;
    const int i = tile / tpr;
    const int k = (tile - i * tpr) * 128 + row;
    valid = k < a.Nk;
    return static_cast<long long>(i) * a.Nk + k;
  }
  const long long tok = static_cast<long long>(tile) * 128 + row;
  valid = tok < a.T;
  return tok;
}

template <int C, bool HAS_BP>
struct ProjSmem {
  using Cfg = ProjCfg<C, HAS_BP>;
  alignas(1024) uint8_t w[Cfg::WBYTES];
  alignas(1024) uint8_t x[2][Cfg::XSTAGE];
  alignas(16) float ln_w[C];
  alignas(16) float ln_b[C];
  uint64_t bar_w;
  uint64_t bar_x_full[2];
  uint64_t bar_x_ready[2];
  uint64_t bar_x_empty[2];
  uint64_t bar_acc_full;
  uint64_t bar_acc_empty;
  uint32_t tmem_base;
  int abort;
};

template <typename T, int C, int D, bool HAS_LN, bool HAS_BP>
__global__ void __launch_bounds__(512, 1)
    proj_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w, ProjArgs a) {
  using Cfg = ProjCfg<C, HAS_BP>;
  using E = Elem<T>;
  constexpr int H = C / D;
  extern __shared__ uint8_t smem_raw[];
  auto& sm = *reinterpret_cast<ProjSmem<C, HAS_BP>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = proj_tiles(a);

  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_w, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.bar_x_full[s], 1);
      mbar_init(&sm.bar_x_ready[s], HAS_LN ? 4 : 1);
      mbar_init(&sm.bar_x_empty[s], 1);
    }
    mbar_init(&sm.bar_acc_full, 1);
    mbar_init(&sm.bar_acc_empty, 8);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (HAS_LN)
    for (int i = threadIdx.x; i < C; i += blockDim.x) {
      sm.ln_w[i] = a.ln_w[i];
      sm.ln_b[i] = a.ln_b[i];
    }
  if (warp == 1) tmem_alloc(&sm.tmem_base, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;
  volatile int* abort = &sm.abort;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&map_x);
      tma_prefetch_desc(&map_w);
      mbar_expect_tx(&sm.bar_w, Cfg::WBYTES);
      for (int ka = 0; ka < Cfg::KATOMS; ++ka)
        for (int r0 = 0; r0 < Cfg::NOUT; r0 += Cfg::WBOX)
          tma_load_2d(sm.w + ka * Cfg::NOUT * 128 + r0 * 128, &map_w, &sm.bar_w, ka * 64, r0);
      int it = 0;
      for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
        const int s = it & 1;
        if (!mbar_wait(&sm.bar_x_empty[s], ((it >> 1) & 1) ^ 1, abort, 101)) break;
        mbar_expect_tx(&sm.bar_x_full[s], Cfg::XSTAGE);
        if (a.trans) {
          const int tpr = (a.Nk + 127) / 128;
          const int i = tile / tpr, k0 = (tile - i * tpr) * 128;
          for (int ka = 0; ka < Cfg::KATOMS; ++ka)
            tma_load_3d(sm.x[s] + ka * 16384, &map_x, &sm.bar_x_full[s], ka * 64, i, k0);
        } else {
          for (int ka = 0; ka < Cfg::KATOMS; ++ka)
            tma_load_2d(sm.x[s] + ka * 16384, &map_x, &sm.bar_x_full[s], ka * 64, tile * 128);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc0 = make_idesc_f16(128, Cfg::N0, E::kFmt, false, false);
      const uint32_t idesc1 = make_idesc_f16(128, Cfg::N1 > 0 ? Cfg::N1 : 16, E::kFmt, false, false);
      bool ok = mbar_wait(&sm.bar_w, 0, abort, 102);
      int it = 0;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++it) {
        const int s = it & 1;
        if (HAS_LN) {
          if (!mbar_wait(&sm.bar_x_ready[s], (it >> 1) & 1, abort, 103)) break;
        } else {
          if (!mbar_wait(&sm.bar_x_full[s], (it >> 1) & 1, abort, 103)) break;
        }
        if (!mbar_wait(&sm.bar_acc_empty, (it & 1) ^ 1, abort, 104)) break;
        tc_fence_after();
        const uint32_t xa = smem_u32(sm.x[s]);
        const uint32_t wa = smem_u32(sm.w);
        for (int kk = 0; kk < C / 16; ++kk) {
          const uint32_t koff = (kk >> 2) * 16384 + (kk & 3) * 32;
          const uint32_t woff = (kk >> 2) * (Cfg::NOUT * 128) + (kk & 3) * 32;
          const uint64_t adesc = make_smem_desc(xa + koff, 16, 1024, kSw128);
          mma_ss(tbase, adesc, make_smem_desc(wa + woff, 16, 1024, kSw128), idesc0, kk > 0);
          if (Cfg::N1 > 0)
            mma_ss(tbase + Cfg::N0, adesc, make_smem_desc(wa + woff + Cfg::N0 * 128, 16, 1024, kSw128), idesc1,
                   kk > 0);
        }
        mma_commit(&sm.bar_x_empty[s]);
        mma_commit(&sm.bar_acc_full);
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ---------------- LayerNorm in place (w4-7), or forwarding of x_full ----------------
    if (HAS_LN) {
      const int row = (warp - 4) * 32 + lane;
      int it = 0;
      for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
        const int s = it & 1;
        if (!mbar_wait(&sm.bar_x_full[s], (it >> 1) & 1, abort, 105)) break;
        uint8_t* xs = sm.x[s];
        // two statistics passes and one normalising pass over the row's 16-byte chunks
        // (no C-wide register array)
        auto chunk_ptr = [&](int i) { return xs + (i >> 3) * 16384 + sw128_off(row, i & 7); };
        float sum = 0.f;
#pragma unroll 4
        for (int i = 0; i < C / 8; ++i) {
          const uint4 u = *reinterpret_cast<const uint4*>(chunk_ptr(i));
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) sum += E::lo(w[e]) + E::hi(w[e]);
        }
        const float mean = sum * (1.0f / C);
        float var = 0.f;
#pragma unroll 4
        for (int i = 0; i < C / 8; ++i) {
          const uint4 u = *reinterpret_cast<const uint4*>(chunk_ptr(i));
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float d0 = E::lo(w[e]) - mean, d1 = E::hi(w[e]) - mean;
            var = fmaf(d0, d0, fmaf(d1, d1, var));
          }
        }
        const float rstd = rsqrtf(var * (1.0f / C) + a.eps);
        bool tvalid;
        const long long tok = proj_token(a, tile, row, tvalid);
        T* xo = a.xln_out != nullptr && tvalid ? static_cast<T*>(a.xln_out) + tok * C : nullptr;
#pragma unroll 2
        for (int i = 0; i < C / 8; ++i) {
          uint8_t* cp = chunk_ptr(i);
          const uint4 u = *reinterpret_cast<const uint4*>(cp);
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
          const float4 g0 = reinterpret_cast<const float4*>(sm.ln_w)[2 * i], g1 = reinterpret_cast<const float4*>(sm.ln_w)[2 * i + 1];
          const float4 b0 = reinterpret_cast<const float4*>(sm.ln_b)[2 * i], b1 = reinterpret_cast<const float4*>(sm.ln_b)[2 * i + 1];
          const float gw[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
          const float bw[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
          uint32_t w4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w4[e] = E::pack2(fmaf((E::lo(w[e]) - mean) * rstd, gw[2 * e], bw[2 * e]),
                             fmaf((E::hi(w[e]) - mean) * rstd, gw[2 * e + 1], bw[2 * e + 1]));
          const uint4 o = make_uint4(w4[0], w4[1], w4[2], w4[3]);
          *reinterpret_cast<uint4*>(cp) = o;
          if (xo != nullptr) *reinterpret_cast<uint4*>(xo + i * 8) = o;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.bar_x_ready[s]);
      }
    }
  } else if (warp >= 8) {
    // ---------------- epilogue (w8-11) ----------------
    // two epilogue warpgroups: heads [0, H/2) and [H/2, H); the first also writes the
    // bias and mask rows
    const int ew = (warp - 8) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_addr = tbase + (static_cast<uint32_t>(wq * 32) << 16);
    float bz[H];
    if (HAS_BP)
#pragma unroll
      for (int h = 0; h < H; ++h) bz[h] = a.bz[h];
    int it = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
      if (!mbar_wait(&sm.bar_acc_full, it & 1, abort, 106)) break;
      tc_fence_after();
      bool valid;
      const long long tok = proj_token(a, tile, row, valid);
      const int ri = valid ? static_cast<int>(tok / a.Nk) : 0;
      const int kpos = valid ? static_cast<int>(tok - static_cast<long long>(ri) * a.Nk) : 0;
      const bool masked = a.mask != nullptr && valid && a.mask[static_cast<long long>(ri) * a.Nk + kpos] == 0;
      uint32_t r[32];
#pragma unroll
      for (int h = ew * (H / 2); h < (ew + 1) * (H / 2); ++h) {
        const size_t qk_off = ((static_cast<size_t>(ri) * H + h) * a.Nk + kpos) * D;
        // Q
        if (D == 32) tmem_ld32(lane_addr + h * D, r); else tmem_ld16(lane_addr + h * D, r);
        if (valid) {
          uint32_t p[D / 2];
#pragma unroll
          for (int d = 0; d < D / 2; ++d)
            p[d] = Elem<__half>::pack2(__uint_as_float(r[2 * d]) * a.scale, __uint_as_float(r[2 * d + 1]) * a.scale);
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(a.q) + qk_off);
#pragma unroll
          for (int c = 0; c < D / 8; ++c) dst[c] = make_uint4(p[4 * c], p[4 * c + 1], p[4 * c + 2], p[4 * c + 3]);
        }
        // K
        if (D == 32) tmem_ld32(lane_addr + C + h * D, r); else tmem_ld16(lane_addr + C + h * D, r);
        if (valid) {
          uint32_t p[D / 2];
#pragma unroll
          for (int d = 0; d < D / 2; ++d)
            p[d] = Elem<__half>::pack2(__uint_as_float(r[2 * d]), __uint_as_float(r[2 * d + 1]));
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(a.k) + qk_off);
#pragma unroll
          for (int c = 0; c < D / 8; ++c) dst[c] = make_uint4(p[4 * c], p[4 * c + 1], p[4 * c + 2], p[4 * c + 3]);
        }
        // V (transposed; masked keys keep their values: their softmax weight is exactly 0)
        if (D == 32) tmem_ld32(lane_addr + 2 * C + h * D, r); else tmem_ld16(lane_addr + 2 * C + h * D, r);
        if (valid) {
          __half* dst = static_cast<__half*>(a.vt) + (static_cast<size_t>(ri) * H + h) * D * a.Nkp + kpos;
#pragma unroll
          for (int d = 0; d < D; ++d) dst[static_cast<size_t>(d) * a.Nkp] = __float2half_rn(__uint_as_float(r[d]));
        }
      }
      if (HAS_BP && ew == 0) {
        tmem_ld16(lane_addr + 3 * C, r);
        if (valid)
#pragma unroll
          for (int h = 0; h < H; ++h)
            static_cast<__half*>(a.bp)[(static_cast<size_t>(h) * a.R + ri) * a.Nkp + kpos] =
                __float2half_rn((__uint_as_float(r[h]) + bz[h]) * 1.4426950408889634f);
      }
      if (valid && ew == 0 && a.pen != nullptr)
        static_cast<unsigned short*>(a.pen)[static_cast<size_t>(ri) * a.Nkp + kpos] = masked ? 0xFC00u : 0u;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.bar_acc_empty);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, Cfg::TMEM_COLS);
  // a kernel that follows this one in the stream then also follows the kernel this one
  // ran beside (no-op without programmatic launch)
  pdl_wait();
}

}  // namespace tops
