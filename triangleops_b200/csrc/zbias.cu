// zbias.cu — attention-pair-bias logits from the raw pair tensor, z read once for
// all heads (HBM-bound streaming kernel).
//
//   bias[h, q, k] = rstd(z[q,k,:]) * (sum_c z[q,k,c] Wc[h,c] - mean(z[q,k,:]) sumW[h]) + Bc[h]
//
// i.e. LN(z) W_proj_z + B_proj_z with the LN affine folded into (Wc, sumW, Bc)
// [attn_pair_bias/module.py:29-35, attn_pair_bias/kernel.py:149-185]. The reference
// recomputes this inside the attention loop once per head (z read H times); here
// z streams through shared memory by bulk copies, eight lanes share one token (16-byte vector loads, 256 contiguous bytes per
// token), merge their partial statistics with warp-shuffle Welford (Chan's
// pairwise update for equal counts) and reduce the H dot products in the same
// shuffle tree. The logits are stored as f16 in log2 units, the operand format of the
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

constexpr int kZbTile = 128;        // tokens per bulk copy (32 KB at Cz = 128, bf16)
constexpr int kZbStages = 6;        // tiles in flight per SM
constexpr int kZbWarps = 12;        // consumer warps
constexpr int kZbThreads = 32 * (kZbWarps + 1);

struct ZbSmem {
  alignas(128) uint8_t tile[kZbStages][kZbTile * 256];
  uint64_t full[kZbStages], empty[kZbStages];
  int abort;
};

// Persistent, one CTA per SM: warp kZbWarps streams contiguous 128-token tiles of z into
// a kZbStages-deep shared-memory ring with bulk copies (so the bytes in flight per SM do
// not depend on how many threads the math leaves room for), and kZbWarps warps reduce
// them: eight lanes per token, each lane two 16-byte chunks (channels [8s, 8s+8) and
// [64+8s, 64+8s+8)), read conflict-free from shared memory.
template <typename T, int CZ, int H>
__global__ void __launch_bounds__(kZbThreads, 1) zbias_kernel(const T* __restrict__ z, ZBiasArgs a) {
  using E = Elem<T>;
  static_assert(CZ == 128, "one token = 8 lanes x 16 channels = 256 bytes");
  extern __shared__ uint8_t smem_raw[];
  ZbSmem& sm = *reinterpret_cast<ZbSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = lane & 7, grp = lane >> 3;
  const long long n_tiles = (a.n_tok + kZbTile - 1) / kZbTile;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kZbStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kZbWarps);
    }
    sm.abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  volatile int* abort = &sm.abort;
  if (warp == kZbWarps) {
    if (lane == 0) {
      int it = 0;
      for (long long t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
        const int s = it % kZbStages;
        if (!mbar_wait(&sm.empty[s], ((it / kZbStages) & 1) ^ 1, abort, 601)) break;
        const long long t0 = t * kZbTile;
        const long long n = a.n_tok - t0 < kZbTile ? a.n_tok - t0 : kZbTile;
        const uint32_t bytes = static_cast<uint32_t>(n) * CZ * 2;
        mbar_expect_tx(&sm.full[s], bytes);
        bulk_load(sm.tile[s], z + t0 * CZ, bytes, &sm.full[s]);
      }
    }
    return;
  }
  // this lane's channels: [sub*8, sub*8+8) and [64+sub*8, 64+sub*8+8)
  float w[H][16];
#pragma unroll
  for (int h = 0; h < H; ++h)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      w[h][e] = a.wc[h * CZ + sub * 8 + e];
      w[h][8 + e] = a.wc[h * CZ + 64 + sub * 8 + e];
    }
  float sw[H], bc[H];
#pragma unroll
  for (int h = 0; h < H; ++h) {
    sw[h] = a.sum_w[h];
    bc[h] = a.b_const[h];
  }
  int it = 0;
  for (long long t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
    const int s = it % kZbStages;
    if (!mbar_wait(&sm.full[s], (it / kZbStages) & 1, abort, 602)) break;
    for (int gi = warp; gi < kZbTile / 4; gi += kZbWarps) {
      const int local = gi * 4 + grp;
      const long long tok = t * kZbTile + local;
      const bool valid = tok < a.n_tok;
      const uint4* src = reinterpret_cast<const uint4*>(sm.tile[s] + local * 256);
      const uint4 u0 = src[sub], u1 = src[8 + sub];
      float v[16];
      {
        const uint32_t p[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          v[2 * e] = E::lo(p[e]);
          v[2 * e + 1] = E::hi(p[e]);
        }
      }
      float mean = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) mean += v[e];
      mean *= (1.0f / 16);
      float m2 = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float d = v[e] - mean;
        m2 = fmaf(d, d, m2);
      }
      float dot[H];
#pragma unroll
      for (int h = 0; h < H; ++h) {
        float acc = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) acc = fmaf(v[e], w[h][e], acc);
        dot[h] = acc;
      }
      // merge the 8 lanes of a token: Welford/Chan for equal counts, and the dots
      float n = 16.f;
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, mean, off);
        const float o2 = __shfl_xor_sync(0xffffffffu, m2, off);
        const float d = om - mean;
        mean += 0.5f * d;
        m2 += o2 + d * d * (0.5f * n);
        n *= 2.f;
#pragma unroll
        for (int h = 0; h < H; ++h) dot[h] += __shfl_xor_sync(0xffffffffu, dot[h], off);
      }
      const float rstd = rsqrtf(m2 * (1.0f / CZ) + a.eps);
      if (valid && sub < H) {
        float bv = 0.f;
#pragma unroll
        for (int h = 0; h < H; ++h)
          if (h == sub) bv = fmaf(rstd, dot[h] - mean * sw[h], bc[h]);
        const long long q = tok / a.M, k = tok - q * a.M;
        a.bias[(static_cast<long long>(sub) * a.Mq + q) * a.Mkp + k] = __float2half_rn(bv * 1.4426950408889634f);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[s]);
  }
}

}  // namespace tops
