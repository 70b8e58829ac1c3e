// f32.cu — fp32 IO path of the three ops (the reference's dtype contract admits
// fp32, _common/dtype.py:7-19). The tensor-core kernels are 16-bit; fp32 runs on
// CUDA cores with four small generic kernels that the Python layer composes:
//
//   tops_f32_layernorm   y = LN(x) rows of width C (two-pass mean / variance)
//   tops_f32_gemm        batched, fully strided C = A B^T (+ bias[n]) — the
//                        projections and the triangular contraction
//   tops_f32_attention   online-softmax attention, one query row per thread
//   tops_f32_gated_mul   y = a * sigmoid(g + bg[col]) (* mask[row])
//
// Accuracy, not speed, is the goal here: everything accumulates in fp32.
#include <cuda_runtime.h>
#include "status.h"

namespace tops {

__global__ void f32_layernorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                     const float* __restrict__ b, float eps, float* __restrict__ y, long long T,
                                     int C) {
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const float* xr = x + row * C;
  float s = 0.f;
  for (int c = lane; c < C; c += 32) s += xr[c];
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / C;
  float v = 0.f;
  for (int c = lane; c < C; c += 32) {
    const float d = xr[c] - mean;
    v += d * d;
  }
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const float rstd = rsqrtf(v / C + eps);
  for (int c = lane; c < C; c += 32) {
    const float t = (xr[c] - mean) * rstd;
    y[row * C + c] = (w ? w[c] : 1.f) * t + (b ? b[c] : 0.f);
  }
}

struct GemmStrides {
  long long ab, am, ak;  // A element (b, m, k)
  long long bb, bn, bk;  // B element (b, n, k)
  long long cb, cm, cn;  // C element (b, m, n)
};

// 64 x 64 output tile per block, 16 x 16 threads, 4 x 4 outputs per thread, K in steps of 16
__global__ void __launch_bounds__(256) f32_gemm_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                       const float* __restrict__ bias, float* __restrict__ Cm, int M,
                                                       int N, int K, GemmStrides s) {
  __shared__ float As[16][65];
  __shared__ float Bs[16][65];
  const int bz = blockIdx.z;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const float* Ab = A + bz * s.ab;
  const float* Bb = B + bz * s.bb;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = threadIdx.x; i < 64 * 16; i += 256) {
      const int r = i >> 4, kk = i & 15;
      const int m = m0 + r, n = n0 + r, k = k0 + kk;
      As[kk][r] = (m < M && k < K) ? Ab[m * s.am + k * s.ak] : 0.f;
      Bs[kk][r] = (n < N && k < K) ? Bb[n * s.bn + k * s.bk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = As[kk][ty * 4 + i];
        b[i] = Bs[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
      if (m < M && n < N) Cm[bz * s.cb + m * s.cm + n * s.cn] = acc[i][j] + (bias ? bias[n] : 0.f);
    }
}

// One thread per query. Q, K, V fp32, element (r, h, n, d) at r*sr + h*sh + n*sn + d (token-major
// [R][N][H*D] is sr = N*H*D, sh = D, sn = H*D); bias [H][Nq][Nk] fp32 (natural units);
// mask [R][Nk] uint8 or null. mask_mode 0: masked keys get -1e9 added (triangle attention,
// triangle_attn/kernel.py:233-238); mask_mode 1: masked keys are dropped (-inf,
// benchmarks/references.py:273-274). S = scale * (q . k) + bias. O: [R][Nq][H*D].
// Head size D <= DMAX at run time (registers and shared tiles sized by DMAX; KB keys per
// shared-memory block).
template <int DMAX, int KB>
__global__ void __launch_bounds__(128) f32_attn_kernel(const float* __restrict__ Q, const float* __restrict__ K,
                                                       const float* __restrict__ V, const float* __restrict__ bias,
                                                       const unsigned char* __restrict__ mask, float* __restrict__ O,
                                                       int R, int H, int Nq, int Nk, float scale, int mask_mode,
                                                       long long sr, long long sh, long long sn, int D) {
  __shared__ float Ks[KB][DMAX + 1];
  __shared__ float Vs[KB][DMAX + 1];
  const int r = blockIdx.z, h = blockIdx.y;
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  const bool qv = q < Nq;
  float qr[DMAX], o[DMAX];
  const float* qp = Q + r * sr + h * sh + static_cast<long long>(qv ? q : 0) * sn;
#pragma unroll
  for (int d = 0; d < DMAX; ++d) {
    qr[d] = d < D ? qp[d] : 0.f;
    o[d] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const float* kb = K + r * sr + h * sh;
  const float* vb = V + r * sr + h * sh;
  for (int k0 = 0; k0 < Nk; k0 += KB) {
    for (int i = threadIdx.x; i < KB * D; i += blockDim.x) {
      const int kk = i / D, d = i % D;
      Ks[kk][d] = k0 + kk < Nk ? kb[static_cast<long long>(k0 + kk) * sn + d] : 0.f;
      Vs[kk][d] = k0 + kk < Nk ? vb[static_cast<long long>(k0 + kk) * sn + d] : 0.f;
    }
    __syncthreads();
    const int kn = Nk - k0 < KB ? Nk - k0 : KB;
    for (int kk = 0; kk < kn; ++kk) {
      const int k = k0 + kk;
      float sdot = 0.f;
#pragma unroll
      for (int d = 0; d < DMAX; ++d)
        if (d < D) sdot = fmaf(qr[d], Ks[kk][d], sdot);
      float sv = scale * sdot + (qv ? bias[(static_cast<long long>(h) * Nq + q) * Nk + k] : 0.f);
      if (mask != nullptr && !mask[static_cast<long long>(r) * Nk + k]) {
        if (mask_mode == 1) continue;
        sv += -1e9f;
      }
      const float mn = fmaxf(m, sv);
      const float alpha = expf(m - mn), p = expf(sv - mn);
      l = l * alpha + p;
#pragma unroll
      for (int d = 0; d < DMAX; ++d)
        if (d < D) o[d] = fmaf(o[d], alpha, p * Vs[kk][d]);
      m = mn;
    }
    __syncthreads();
  }
  if (qv) {
    float* op = O + (static_cast<long long>(r) * Nq + q) * (H * D) + h * D;
    const float inv = 1.f / l;
#pragma unroll
    for (int d = 0; d < DMAX; ++d)
      if (d < D) op[d] = o[d] * inv;
  }
}

__global__ void f32_gated_mul_kernel(const float* __restrict__ a, const float* __restrict__ g,
                                     const float* __restrict__ bg, const unsigned char* __restrict__ mask,
                                     float* __restrict__ y, long long rows, int cols, long long lda, long long ldg,
                                     long long ldy) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const long long r = i / cols;
  const int c = static_cast<int>(i - r * cols);
  const float gv = g[r * ldg + c] + (bg ? bg[c] : 0.f);
  float v = a[r * lda + c] * (1.f / (1.f + expf(-gv)));
  if (mask != nullptr) v *= static_cast<float>(static_cast<signed char>(mask[r]));
  y[r * ldy + c] = v;
}

}  // namespace tops

using namespace tops;

extern "C" int tops_f32_layernorm(int64_t T, int64_t C, const float* x, const float* w, const float* b, float eps,
                                  float* y, void* stream) {
  if (T <= 0 || C <= 0 || x == nullptr || y == nullptr) return TOPS_ERR_SHAPE;
  const int rows_per_block = 8;
  f32_layernorm_kernel<<<static_cast<unsigned>((T + rows_per_block - 1) / rows_per_block), 32 * rows_per_block, 0,
                         static_cast<cudaStream_t>(stream)>>>(x, w, b, eps, y, T, static_cast<int>(C));
  return cudaGetLastError() == cudaSuccess ? TOPS_OK : TOPS_ERR_CUDA;
}

// strides: 9 int64 element strides {A: b, m, k; B: b, n, k; C: b, m, n}
extern "C" int tops_f32_gemm(int64_t batch, int64_t M, int64_t N, int64_t K, const float* A, const float* B,
                             const float* bias, float* Cm, const int64_t* strides, void* stream) {
  if (batch <= 0 || M <= 0 || N <= 0 || K <= 0 || batch > 65535 || strides == nullptr) return TOPS_ERR_SHAPE;
  if (A == nullptr || B == nullptr || Cm == nullptr) return TOPS_ERR_ALIGN;
  GemmStrides s{strides[0], strides[1], strides[2], strides[3], strides[4], strides[5], strides[6], strides[7],
                strides[8]};
  dim3 grid(static_cast<unsigned>((N + 63) / 64), static_cast<unsigned>((M + 63) / 64), static_cast<unsigned>(batch));
  f32_gemm_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(A, B, bias, Cm, static_cast<int>(M),
                                                                      static_cast<int>(N), static_cast<int>(K), s);
  return cudaGetLastError() == cudaSuccess ? TOPS_OK : TOPS_ERR_CUDA;
}

extern "C" int tops_f32_attention(int64_t R, int64_t H, int64_t Nq, int64_t Nk, int64_t D, const float* q,
                                  const float* k, const float* v, int64_t sr, int64_t sh, int64_t sn,
                                  const float* bias, const uint8_t* mask, float scale, int mask_mode, float* out,
                                  void* stream) {
  if (R <= 0 || H <= 0 || Nq <= 0 || Nk <= 0 || H > 65535 || R > 65535) return TOPS_ERR_SHAPE;
  if (mask_mode != 0 && mask_mode != 1) return TOPS_ERR_ARG;
  dim3 grid(static_cast<unsigned>((Nq + 127) / 128), static_cast<unsigned>(H), static_cast<unsigned>(R));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int d = static_cast<int>(D);
#define TOPS_F32_ATTN(DM, KB)                                                                                     \
  f32_attn_kernel<DM, KB><<<grid, 128, 0, st>>>(q, k, v, bias, mask, out, static_cast<int>(R), static_cast<int>(H), \
                                                static_cast<int>(Nq), static_cast<int>(Nk), scale, mask_mode, sr, sh, \
                                                sn, d)
  if (D <= 0 || D > 128)
    return TOPS_ERR_SHAPE;
  else if (D <= 16)
    TOPS_F32_ATTN(16, 64);
  else if (D <= 32)
    TOPS_F32_ATTN(32, 64);
  else if (D <= 64)
    TOPS_F32_ATTN(64, 64);
  else
    TOPS_F32_ATTN(128, 32);
#undef TOPS_F32_ATTN
  return cudaGetLastError() == cudaSuccess ? TOPS_OK : TOPS_ERR_CUDA;
}

extern "C" int tops_f32_gated_mul(int64_t rows, int64_t cols, const float* a, int64_t lda, const float* g, int64_t ldg,
                                  const float* bg, const uint8_t* mask, float* y, int64_t ldy, void* stream) {
  if (rows <= 0 || cols <= 0) return TOPS_ERR_SHAPE;
  const long long n = rows * cols;
  f32_gated_mul_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      a, g, bg, mask, y, rows, static_cast<int>(cols), lda, ldg, ldy);
  return cudaGetLastError() == cudaSuccess ? TOPS_OK : TOPS_ERR_CUDA;
}
