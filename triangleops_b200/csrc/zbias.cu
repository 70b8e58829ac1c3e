// zbias.cu — attention-pair-bias logits from the raw pair tensor, z read once for
// all heads (HBM-bound streaming kernel).
//
//   bias[h, q, k] = rstd(z[q,k,:]) * (sum_c z[q,k,c] Wc[h,c] - mean(z[q,k,:]) sumW[h]) + Bc[h]
//
// i.e. LN(z) W_proj_z + B_proj_z with the LN affine folded into (Wc, sumW, Bc)
// [attn_pair_bias/module.py:29-35, attn_pair_bias/kernel.py:149-185]. The reference
// recomputes this inside the attention loop once per head (z read H times); here
// eight lanes share one token (16-byte vector loads, 256 contiguous bytes per
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

template <typename T, int CZ, int H>
__global__ void __launch_bounds__(256) zbias_kernel(const T* __restrict__ z, ZBiasArgs a) {
  using E = Elem<T>;
  static_assert(CZ == 128, "one token = 8 lanes x 16 channels");
  const int lane = threadIdx.x & 31, sub = lane & 7, grp = lane >> 3;
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
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const long long wid = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  // the next group's 32 bytes per lane are loaded before this group is reduced, so two
  // groups' loads are in flight per warp (the kernel is bound by loads in flight; a
  // third group measured no faster)
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  auto load = [&](long long t, uint4& u0, uint4& u1) {
    if (t < a.n_tok) {
      const uint4* src = reinterpret_cast<const uint4*>(z + t * CZ);
      u0 = __ldcs(src + sub);
      u1 = __ldcs(src + 8 + sub);
    } else {
      u0 = zero;
      u1 = zero;
    }
  };
  uint4 nx0, nx1;
  load(wid * 4 + grp, nx0, nx1);
  for (long long base = wid * 4; base < a.n_tok; base += warps * 4) {
    const long long tok = base + grp;
    const bool valid = tok < a.n_tok;
    const uint4 u0 = nx0, u1 = nx1;
    load(base + warps * 4 + grp, nx0, nx1);
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
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) s = fmaf(v[e], w[h][e], s);
      dot[h] = s;
    }
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
      a.bias[(static_cast<long long>(sub) * a.Mq + q) * a.Mkp + k] = __float2half_rn(bv * 1.4426950408889634f);  // log2 units
    }
  }
}

}  // namespace tops
