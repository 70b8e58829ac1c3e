// zbias.cu — attention-pair-bias logits from the raw pair tensor, z read once for
// all heads (HBM-bound streaming kernel).
//
//   bias[h, q, k] = rstd(z[q,k,:]) * (sum_c z[q,k,c] Wc[h,c] - mean(z[q,k,:]) sumW[h]) + Bc[h]
//
// i.e. LN(z) W_proj_z + B_proj_z with the LN affine folded into (Wc, sumW, Bc)
// [attn_pair_bias/module.py:29-35, attn_pair_bias/kernel.py:149-185]. The reference
// recomputes this inside the attention loop once per head (z read H times); here
// z streams through shared memory by TMA, the tensor core takes the head dots and one
// thread per token the statistics (16-byte vector loads from the staged tile, two passes
// over its row in registers with eight independent accumulation chains). The logits are stored as f16 in log2 units, the operand format of the
// attention kernel (the reference adds them in fp32; f16 keeps 11 bits, |error| below
// 2^-11 of the logit).
#include "sm100.cuh"

namespace tops {

struct ZBiasArgs {
  long long n_tok;      // Mq * M
  int M, Mkp;           // key count, padded key stride of the output rows
  int Mq;               // query rows in this call (rows of z and of each bias head)
  float eps;
  const float* wc;      // [H][Cz] fp32
  const float* sum_w;   // [H]
  const float* b_const; // [H]
  __half* bias;         // [H][Mq][Mkp] f16, in log2 units (times log2(e))
};

constexpr int kZbTile = 128;        // tokens per tile (one TMEM lane each)
constexpr int kZbStages = 5;        // tiles in flight per SM (32 KB each)
constexpr int kZbThreads = 384;     // w0 TMA, w1 MMA, w4..w7 and w8..w11 statistics / epilogue (even / odd tiles)

struct ZbSmem {
  alignas(1024) uint8_t tile[kZbStages][2][16384];  // z tile: 128 tokens x 128 ch, two SW128 atoms
  alignas(1024) uint8_t wt[2][2048];                // B: 16 rows (W_hi | W_lo | 0) x 128 ch, two atoms
  uint64_t full[kZbStages], empty[kZbStages];
  uint64_t acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int abort;
};

// Persistent, one CTA per SM. The per-head dot products z . Wc[h] run on the tensor core:
// D[token, n] = sum_c z[token, c] B[n, c] with B rows 0..3 = Wc rounded to the IO dtype
// and rows 4..7 = the rounding residue (so D[h] + D[4+h] carries the fp32 weights), one
// M=128, N=16, K=128 MMA chain per 128-token tile. The LayerNorm statistics need the
// second moment, which is not linear in z: one thread per token computes mean and
// variance (two passes over its row in registers) from the same shared-memory tile,
// then combines them with the dots and stores the four heads' logits (consecutive
// threads write consecutive keys).
template <typename T, int CZ, int H>
__global__ void __launch_bounds__(kZbThreads, 1)
    zbias_kernel(const __grid_constant__ CUtensorMap map_z, ZBiasArgs a) {
  using E = Elem<T>;
  static_assert(CZ == 128 && H == 4, "Cz = 128, four heads");
  extern __shared__ uint8_t smem_raw[];
  ZbSmem& sm = *reinterpret_cast<ZbSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();  // the token projection (launched next, programmatically) runs beside this kernel
  const long long n_tiles = (a.n_tok + kZbTile - 1) / kZbTile;
  // B tile: element (n, c) of the K-major SW128 layout at atom c/64, n*128 + ((c%64/8 ^ n%8)*16) + (c%8)*2
  for (int idx = threadIdx.x; idx < 16 * CZ; idx += blockDim.x) {
    const int n = idx / CZ, c = idx % CZ;
    float v = 0.f;
    if (n < H) {
      v = a.wc[n * CZ + c];
    } else if (n < 2 * H) {
      const float w = a.wc[(n - H) * CZ + c];
      v = w - E::to_f(E::from_f(w));
    }
    const T tv = E::from_f(v);
    *reinterpret_cast<T*>(sm.wt[c >> 6] + n * 128 + ((((c & 63) >> 3) ^ (n & 7)) << 4) + (c & 7) * 2) = tv;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kZbStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1 + 4);  // the MMA commit and the four statistics warps
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 4);
    }
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&sm.tmem_base, 32);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;
  volatile int* abort = &sm.abort;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&map_z);
      int it = 0;
      for (long long t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
        const int s = it % kZbStages;
        if (!mbar_wait(&sm.empty[s], ((it / kZbStages) & 1) ^ 1, abort, 601)) break;
        mbar_expect_tx(&sm.full[s], 2 * 16384);
        tma_load_2d(sm.tile[s][0], &map_z, &sm.full[s], 0, static_cast<int>(t * kZbTile));
        tma_load_2d(sm.tile[s][1], &map_z, &sm.full[s], 64, static_cast<int>(t * kZbTile));
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(128, 16, E::kFmt, false, false);
      int it = 0;
      for (long long t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
        const int s = it % kZbStages, b = it & 1;
        if (!mbar_wait(&sm.full[s], (it / kZbStages) & 1, abort, 602)) break;
        if (it >= 2 && !mbar_wait(&sm.acc_empty[b], ((it >> 1) - 1) & 1, abort, 603)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < CZ / 16; ++kk)
          mma_ss(tbase + b * 16, make_smem_desc(smem_u32(sm.tile[s][kk >> 2]) + (kk & 3) * 32, 16, 1024, kSw128),
                 make_smem_desc(smem_u32(sm.wt[kk >> 2]) + (kk & 3) * 32, 16, 1024, kSw128), idesc, kk > 0);
        mma_commit(&sm.acc_full[b]);
        mma_commit(&sm.empty[s]);
      }
    }
  } else if (warp >= 4) {
    // two warpgroups take the tiles in turn (tile it uses accumulator it & 1)
    const int wg = (warp - 4) >> 2;
    const int wq = warp & 3, r = wq * 32 + lane;
    const uint32_t lane_addr = tbase + (static_cast<uint32_t>(wq * 32) << 16);
    float sw[H], bc[H];
#pragma unroll
    for (int h = 0; h < H; ++h) {
      sw[h] = a.sum_w[h];
      bc[h] = a.b_const[h];
    }
    int it = 0;
    for (long long t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
      const int s = it % kZbStages, b = it & 1;
      if (b != wg) continue;
      if (!mbar_wait(&sm.full[s], (it / kZbStages) & 1, abort, 604)) break;
      uint32_t p[64];
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint4 u = *reinterpret_cast<const uint4*>(sm.tile[s][c >> 3] + r * 128 + ((((c & 7) ^ (r & 7))) << 4));
        p[4 * c] = u.x;
        p[4 * c + 1] = u.y;
        p[4 * c + 2] = u.z;
        p[4 * c + 3] = u.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[s]);
      // eight independent add chains (four packed fp32 pairs) per moment, not one 128-long
      // dependent chain: the statistics keep pace with the TMA stream
      unsigned long long acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
      for (int e = 0; e < 64; ++e) acc[e & 3] = f2_add(acc[e & 3], f2_pack(E::lo(p[e]), E::hi(p[e])));
      float sum = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float lo, hi;
        f2_unpack(acc[e], lo, hi);
        sum += lo + hi;
        acc[e] = 0ull;
      }
      const float mean = sum * (1.0f / CZ);
      const unsigned long long nm = f2_pack(-mean, -mean);
#pragma unroll
      for (int e = 0; e < 64; ++e) {
        const unsigned long long dd = f2_add(f2_pack(E::lo(p[e]), E::hi(p[e])), nm);
        acc[e & 3] = f2_fma(dd, dd, acc[e & 3]);
      }
      float m2 = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float lo, hi;
        f2_unpack(acc[e], lo, hi);
        m2 += lo + hi;
      }
      const float rstd = rsqrtf(m2 * (1.0f / CZ) + a.eps);
      if (!mbar_wait(&sm.acc_full[b], (it >> 1) & 1, abort, 605)) break;
      tc_fence_after();
      uint32_t d[8];
      asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n\t"
                   "tcgen05.wait::ld.sync.aligned;"
                   : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]), "=r"(d[7])
                   : "r"(lane_addr + b * 16)
                   : "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[b]);
      const long long tok = t * kZbTile + r;
      if (tok < a.n_tok) {
        const long long q = tok / a.M, k = tok - q * a.M;
#pragma unroll
        for (int h = 0; h < H; ++h) {
          const float dot = __uint_as_float(d[h]) + __uint_as_float(d[H + h]);
          const float bv = fmaf(rstd, dot - mean * sw[h], bc[h]);
          a.bias[(static_cast<long long>(h) * a.Mq + q) * a.Mkp + k] = __float2half_rn(bv * 1.4426950408889634f);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tbase, 32);
}

}  // namespace tops
