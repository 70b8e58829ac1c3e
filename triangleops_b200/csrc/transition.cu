// transition.cu — the Pairformer pair transition, fused on tcgen05:
//
//   out[t,:] = x[t,:] + ( silu(xhat W1'^T + b1) * (xhat W2'^T + b2) ) W3^T
//
// xhat = (x - mean) / sqrt(var + eps) per token; the LayerNorm affine is folded into the
// weights on the host (W1' = W1 * gamma, b1 = W1 beta; the same for W2), hidden width
// NH = 4C. This is the AlphaFold-3 transition layer (supplementary Algorithm 11); the
// reference ships no transition, so there is no reference kernel it replaces.
//
// Persistent kernel, one 128-token tile at a time per CTA, the hidden dimension in
// chunks of 64:
//   w0       TMA producer: per chunk h the weight stage [W1'_h ; W2'_h] (128 x C) and
//            W3_h (C x 64) into a 2-deep ring
//   w3       TMA producer of the x tiles (the next tile's x lands during this tile's chunks)
//   w1       MMA1 issuer: U_h = xhat [W1'_h ; W2'_h]^T (N = 128: u | v) into one of two
//            TMEM buffers
//   w2       MMA2 issuer: ACC += H_h W3_h^T (N = C)
//   w4..     kTrWG warpgroups, one token row (TMEM lane) per thread, each owning a slice
//            of the columns: LayerNorm of the row into its slice of the xhat tile, per
//            chunk its slice of H_h = silu(u + b1) * (v + b2) into a shared-memory tile
//            (double-buffered), then its slice of the epilogue x + ACC
// TMEM: U buffers at columns 0 and 128 (128 fp32 each), ACC at 256 (C columns).
#include "sm100.cuh"

namespace tops {

constexpr int kTrC = 128;            // channels
constexpr int kTrNH = 4 * kTrC;      // hidden width
constexpr int kTrCH = 64;            // hidden chunk
constexpr int kTrNCH = kTrNH / kTrCH;  // chunks per tile
constexpr int kTrStages = 2;
constexpr int kTrWG = 2;              // LayerNorm / SwiGLU / epilogue warpgroups (column halves)
constexpr int kTrThreads = 128 + 128 * kTrWG;

struct TrSmem {
  alignas(1024) uint8_t xraw[2][16384];          // x tile as loaded: 128 rows x 128 ch, two SW128 atoms
  alignas(1024) uint8_t xh[2][16384];            // xhat tile: 128 rows x 128 ch, two 64-ch SW128 atoms
  alignas(1024) uint8_t hbuf[2][16384];          // H_h: 128 rows x 64 hidden, one SW128 atom, two buffers
  alignas(1024) uint8_t w12[kTrStages][2][16384];  // [W1'_h ; W2'_h]: 128 rows x 128 K (two K atoms)
  alignas(1024) uint8_t w3[kTrStages][16384];    // W3_h: 128 rows (C) x 64 K (hidden)
  float b12[kTrNCH * 128];                       // the folded biases of every chunk
  uint64_t x_full, x_empty;                      // x tile landed / every warpgroup has read it
  uint64_t w_full[kTrStages], w_empty[kTrStages];
  uint64_t xh_full, xh_empty;                    // xhat written / every MMA1 of the tile done
  uint64_t u_full[2], u_empty[2];                // U buffer b holds chunk h / was read
  uint64_t h_full[2], h_empty[2];                // H buffer b written / MMA2 read it
  uint64_t acc_full, acc_empty;
  uint32_t tmem_base;
  int abort;
};

struct TrArgs {
  int M;              // tokens
  float eps;
  const void* x;      // [M][C]
  void* out;          // [M][C] (may alias x)
  const float* b12;   // [NCH][128]: chunk h -> b1[h*64..] | b2[h*64..]
};

// byte offset of element (row r, column c) in a 128-byte-row SW128 atom (c < 64)
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return r * 128 + ((((c >> 3) ^ (r & 7)) & 7) << 4) + (c & 7) * 2;
}

template <typename T>
__global__ void __launch_bounds__(kTrThreads, 1)
    transition_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w12,
                      const __grid_constant__ CUtensorMap map_w3, TrArgs a) {
  using E = Elem<T>;
  extern __shared__ uint8_t smem_raw[];
  TrSmem& sm = *reinterpret_cast<TrSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (a.M + 127) / 128;
  for (int i = threadIdx.x; i < kTrNCH * 128; i += blockDim.x) sm.b12[i] = a.b12[i];
  if (threadIdx.x == 0) {
    mbar_init(&sm.x_full, 1);
    mbar_init(&sm.x_empty, 4 * kTrWG);
    for (int s = 0; s < kTrStages; ++s) {
      mbar_init(&sm.w_full[s], 1);
      mbar_init(&sm.w_empty[s], 2);  // MMA1 (W12) and MMA2 (W3) both release the stage
    }
    mbar_init(&sm.xh_full, 128 * kTrWG);
    mbar_init(&sm.xh_empty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.u_full[b], 1);
      mbar_init(&sm.u_empty[b], 128 * kTrWG);
      mbar_init(&sm.h_full[b], 128 * kTrWG);
      mbar_init(&sm.h_empty[b], 1);
    }
    mbar_init(&sm.acc_full, 1);
    mbar_init(&sm.acc_empty, 128 * kTrWG);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&sm.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;
  volatile int* abort = &sm.abort;
  constexpr uint32_t kFmt = E::kFmt;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- weight producer ----------------
      tma_prefetch_desc(&map_w12);
      tma_prefetch_desc(&map_w3);
      int g = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
        for (int h = 0; h < kTrNCH; ++h, ++g) {
          const int s = g % kTrStages;
          if (!mbar_wait(&sm.w_empty[s], ((g / kTrStages) & 1) ^ 1, abort, 801)) { ok = false; break; }
          mbar_expect_tx(&sm.w_full[s], 3 * 16384);
          tma_load_2d(sm.w12[s][0], &map_w12, &sm.w_full[s], 0, h * 128);
          tma_load_2d(sm.w12[s][1], &map_w12, &sm.w_full[s], 64, h * 128);
          tma_load_2d(sm.w3[s], &map_w3, &sm.w_full[s], h * kTrCH, 0);
        }
      }
    }
  } else if (warp == 3) {
    if (lane == 0) {
      // ---------------- x tiles: the next tile's x lands while this tile computes ----------------
      tma_prefetch_desc(&map_x);
      int it = 0;
      for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
        if (!mbar_wait(&sm.x_empty, (it & 1) ^ 1, abort, 812)) break;
        mbar_expect_tx(&sm.x_full, 2 * 16384);
        tma_load_2d(sm.xraw[0], &map_x, &sm.x_full, 0, tile * 128);
        tma_load_2d(sm.xraw[1], &map_x, &sm.x_full, 64, tile * 128);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA1: U_h = xhat [W1'_h ; W2'_h]^T ----------------
      const uint32_t idesc = make_idesc_f16(128, 128, kFmt, false, false);
      int g = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++it) {
        if (!mbar_wait(&sm.xh_full, it & 1, abort, 802)) break;
        for (int h = 0; h < kTrNCH; ++h, ++g) {
          const int s = g % kTrStages, ub = g & 1;
          if (!mbar_wait(&sm.w_full[s], (g / kTrStages) & 1, abort, 803)) { ok = false; break; }
          if (g >= 2 && !mbar_wait(&sm.u_empty[ub], ((g >> 1) - 1) & 1, abort, 804)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kTrC / 16; ++kk) {
            const uint32_t ao = smem_u32(sm.xh[kk >> 2]) + (kk & 3) * 32;
            const uint32_t bo = smem_u32(sm.w12[s][kk >> 2]) + (kk & 3) * 32;
            mma_ss(tbase + ub * 128, make_smem_desc(ao, 16, 1024, kSw128), make_smem_desc(bo, 16, 1024, kSw128),
                   idesc, kk > 0);
          }
          mma_commit(&sm.u_full[ub]);
          mma_commit(&sm.w_empty[s]);
        }
        if (ok) mma_commit(&sm.xh_empty);
      }
    }
  } else if (warp == 2) {
    if (lane == 0) {
      // ---------------- MMA2: ACC += H_h W3_h^T ----------------
      const uint32_t idesc = make_idesc_f16(128, kTrC, kFmt, false, false);
      int g = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++it) {
        for (int h = 0; h < kTrNCH; ++h, ++g) {
          const int s = g % kTrStages, hb = g & 1;
          if (!mbar_wait(&sm.h_full[hb], (g >> 1) & 1, abort, 805)) { ok = false; break; }
          if (!mbar_wait(&sm.w_full[s], (g / kTrStages) & 1, abort, 806)) { ok = false; break; }
          // the first chunk of a tile overwrites ACC: the previous tile's epilogue must have read it
          if (h == 0 && it > 0 && !mbar_wait(&sm.acc_empty, (it - 1) & 1, abort, 807)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kTrCH / 16; ++kk) {
            const uint32_t ao = smem_u32(sm.hbuf[hb]) + kk * 32;
            const uint32_t bo = smem_u32(sm.w3[s]) + kk * 32;
            mma_ss(tbase + 256, make_smem_desc(ao, 16, 1024, kSw128), make_smem_desc(bo, 16, 1024, kSw128), idesc,
                   (h > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&sm.h_empty[hb]);
          mma_commit(&sm.w_empty[s]);
        }
        if (ok) mma_commit(&sm.acc_full);
      }
    }
  } else if (warp >= 4) {
    // ---------------- LayerNorm, SwiGLU and epilogue warpgroups ----------------
    constexpr int QX = kTrC / kTrWG;    // xhat / output columns of this warpgroup
    constexpr int QH = kTrCH / kTrWG;   // hidden columns of this warpgroup per chunk
    const int wq = warp & 3, k = (warp - 4) >> 2;
    const int row = wq * 32 + lane;  // token row of the tile == TMEM lane
    const uint32_t lane_addr = tbase + (static_cast<uint32_t>(wq * 32) << 16);
    int g = 0, it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++it) {
      const int tok = tile * 128 + row;
      const bool valid = tok < a.M;
      // LayerNorm statistics of the whole row (fp32) from the staged x tile; this warpgroup
      // writes its QX columns of xhat and keeps them of x for the residual
      if (!mbar_wait(&sm.x_full, it & 1, abort, 813)) { ok = false; break; }
      // two streaming passes over the row in shared memory (few live registers)
      auto xchunk = [&](int c) { return *reinterpret_cast<const uint4*>(sm.xraw[c >> 3] + sw128_off(row, (c & 7) * 8)); };
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint4 v4 = xchunk(c);
        const uint32_t w4[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) sum += E::lo(w4[e]) + E::hi(w4[e]);
      }
      const float mean = sum * (1.0f / kTrC);
      float var = 0.f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint4 v4 = xchunk(c);
        const uint32_t w4[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float d0 = E::lo(w4[e]) - mean, d1 = E::hi(w4[e]) - mean;
          var += d0 * d0 + d1 * d1;
        }
      }
      const float rstd = valid ? rsqrtf(var * (1.0f / kTrC) + a.eps) : 0.f;
      // this warpgroup's columns of x: the residual and the xhat it writes
      uint4 xres[QX / 8];
#pragma unroll
      for (int c = 0; c < QX / 8; ++c) xres[c] = xchunk(k * (QX / 8) + c);
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.x_empty);
      // the previous tile's MMA1s must be done with the xhat tile
      if (it > 0 && !mbar_wait(&sm.xh_empty, (it - 1) & 1, abort, 808)) { ok = false; break; }
#pragma unroll
      for (int c = 0; c < QX / 8; ++c) {
        const uint32_t w4[4] = {xres[c].x, xres[c].y, xres[c].z, xres[c].w};
        uint32_t o4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) o4[e] = E::pack2((E::lo(w4[e]) - mean) * rstd, (E::hi(w4[e]) - mean) * rstd);
        const int cg = k * (QX / 8) + c;  // 8-column chunk of the row
        *reinterpret_cast<uint4*>(sm.xh[cg >> 3] + sw128_off(row, (cg & 7) * 8)) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&sm.xh_full);
      for (int h = 0; h < kTrNCH; ++h, ++g) {
        const int ub = g & 1, hb = g & 1;
        if (!mbar_wait(&sm.u_full[ub], (g >> 1) & 1, abort, 809)) { ok = false; break; }
        tc_fence_after();
        uint32_t uv[2 * QH];  // u = uv[0..QH), v = uv[QH..2QH)
        if constexpr (QH == 16) {
          tmem_ld16x2_async(lane_addr + ub * 128 + k * QH, lane_addr + ub * 128 + 64 + k * QH, uv);
          tmem_wait_ld32(uv);
        } else {
          static_assert(QH == 32 || QH == 16, "u and v loads of 16 or 32 columns");
          tmem_ld32(lane_addr + ub * 128 + k * QH, uv);
          tmem_ld32(lane_addr + ub * 128 + 64 + k * QH, uv + QH);
        }
        const uint32_t* u = uv;
        const uint32_t* v = uv + QH;
        tc_fence_before();
        mbar_arrive(&sm.u_empty[ub]);
        const float4* bb = reinterpret_cast<const float4*>(sm.b12 + h * 128 + k * QH);
        uint32_t hp[QH / 2];
#pragma unroll
        for (int c = 0; c < QH / 4; ++c) {
          const float4 b1 = bb[c], b2 = bb[16 + c];
          const float u0 = __uint_as_float(u[4 * c]) + b1.x, u1 = __uint_as_float(u[4 * c + 1]) + b1.y;
          const float u2 = __uint_as_float(u[4 * c + 2]) + b1.z, u3 = __uint_as_float(u[4 * c + 3]) + b1.w;
          const float v0 = __uint_as_float(v[4 * c]) + b2.x, v1 = __uint_as_float(v[4 * c + 1]) + b2.y;
          const float v2 = __uint_as_float(v[4 * c + 2]) + b2.z, v3 = __uint_as_float(v[4 * c + 3]) + b2.w;
          hp[2 * c] = E::pack2(u0 * sigmoid_fast(u0) * v0, u1 * sigmoid_fast(u1) * v1);
          hp[2 * c + 1] = E::pack2(u2 * sigmoid_fast(u2) * v2, u3 * sigmoid_fast(u3) * v3);
        }
        // H buffer hb held chunk g-2: MMA2 must have read it
        if (g >= 2 && !mbar_wait(&sm.h_empty[hb], ((g >> 1) - 1) & 1, abort, 810)) { ok = false; break; }
#pragma unroll
        for (int c = 0; c < QH / 8; ++c)
          *reinterpret_cast<uint4*>(sm.hbuf[hb] + sw128_off(row, k * QH + c * 8)) =
              make_uint4(hp[4 * c], hp[4 * c + 1], hp[4 * c + 2], hp[4 * c + 3]);
        fence_proxy_async_smem();
        mbar_arrive(&sm.h_full[hb]);
      }
      if (!ok) break;
      // epilogue: out = x + ACC over this warpgroup's QX columns
      if (!mbar_wait(&sm.acc_full, it & 1, abort, 811)) { ok = false; break; }
      tc_fence_after();
      uint32_t r[QX];
#pragma unroll
      for (int c0 = 0; c0 < QX; c0 += 32) tmem_ld32(lane_addr + 256 + k * QX + c0, r + c0);
      tc_fence_before();
      mbar_arrive(&sm.acc_empty);
      if (valid) {
        uint4* dst = static_cast<uint4*>(a.out) + static_cast<size_t>(tok) * 16 + k * QX / 8;
        static_assert(QX % 32 == 0, "epilogue in 32-column loads");
#pragma unroll
        for (int q = 0; q < QX / 8; ++q) {
          const uint4 xq = xres[q];
          const uint32_t w4[4] = {xq.x, xq.y, xq.z, xq.w};
          uint32_t o4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            o4[e] = E::pack2(E::lo(w4[e]) + __uint_as_float(r[8 * q + 2 * e]),
                             E::hi(w4[e]) + __uint_as_float(r[8 * q + 2 * e + 1]));
          dst[q] = make_uint4(o4[0], o4[1], o4[2], o4[3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, 512);
}

}  // namespace tops

using namespace tops;

namespace tops {
template <typename T>
int launch_transition(int dtype, int64_t M, const void* x, const void* w12, const void* w3, const float* b12,
                      float eps, void* out, cudaStream_t st) {
  CUtensorMap mx, m12, m3;
  if (!map_rows(&mx, dtype, x, M, kTrC, 128)) return TOPS_ERR_TMAP;
  if (!map_rows(&m12, dtype, w12, kTrNH * 2, kTrC, 128)) return TOPS_ERR_TMAP;
  if (!map_rows(&m3, dtype, w3, kTrC, kTrNH, 128)) return TOPS_ERR_TMAP;
  TrArgs args{static_cast<int>(M), eps, x, out, b12};
  const size_t smem = sizeof(TrSmem) + 1024;
  auto kern = transition_kernel<T>;
  set_smem(kern, smem);
  const long long tiles = (M + 127) / 128;
  const int grid = tiles < sm_count() ? static_cast<int>(tiles) : sm_count();
  kern<<<grid, kTrThreads, smem, st>>>(mx, m12, m3, args);
  return launch_status();
}
}  // namespace tops

// Pairformer pair transition over M tokens (see the header): out = x + transition(x).
extern "C" int tops_transition_forward(int dtype, int64_t M, int64_t C, const void* x, const void* w12,
                                       const void* w3, const float* b12, float eps, void* out, void* stream) {
  if (dtype != TOPS_BF16 && dtype != TOPS_F16) return TOPS_ERR_DTYPE;
  if (M <= 0 || M >= (int64_t(1) << 31) || C != kTrC) return TOPS_ERR_SHAPE;
  const void* ptrs[] = {x, w12, w3, b12, out};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return TOPS_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == TOPS_BF16 ? launch_transition<__nv_bfloat16>(dtype, M, x, w12, w3, b12, eps, out, st)
                            : launch_transition<__half>(dtype, M, x, w12, w3, b12, eps, out, st);
}
