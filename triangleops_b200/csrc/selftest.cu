// selftest.cu — single-tile checks of every UMMA operand mode the TriangleOps
// kernels rely on. Each mode runs one TMA load + one tcgen05 MMA chain on one
// CTA and writes the fp32 accumulator back, so the host can compare it with a
// plain matmul. This isolates descriptor / swizzle / TMEM-layout errors from
// the logic of the real kernels.
//
//   mode 0: A,B K-major, 128B swizzle   (M=128, N=128, K=64)   D = A B^T
//   mode 1: A,B K-major,  64B swizzle   (M=128, N=64,  K=32)   D = A B^T
//   mode 2: A,B MN-major, 128B swizzle  (M=128, N=128, K=64)   D = A^T B   (A,B stored [K][M], [K][N])
//   mode 3: A from TMEM (packed pairs), B K-major 128B swizzle (M=128, N=48, K=64)
#include "sm100.cuh"
#include "tmap.h"
#include "status.h"

namespace tops {

struct SelftestSmem {
  alignas(1024) uint8_t a[16384];
  alignas(1024) uint8_t b[16384];
  uint64_t bar_load;
  uint64_t bar_mma;
  uint32_t tmem_base;
  int abort;
};

template <int MODE>
__global__ void __launch_bounds__(128) selftest_kernel(const __grid_constant__ CUtensorMap map_a,
                                                       const __grid_constant__ CUtensorMap map_b,
                                                       const __nv_bfloat16* __restrict__ a_rows, float* __restrict__ d,
                                                       int n_out) {
  extern __shared__ uint8_t smem_raw[];
  SelftestSmem& sm = *reinterpret_cast<SelftestSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    mbar_init(&sm.bar_load, 1);
    mbar_init(&sm.bar_mma, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&sm.tmem_base, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;

  if (MODE == 3) {
    // stage A (row r = thread) into TMEM columns [128, 160) as packed bf16 pairs
    uint32_t r[32];
    const uint32_t* src = reinterpret_cast<const uint32_t*>(a_rows + tid * 64);
    for (int i = 0; i < 32; ++i) r[i] = src[i];
    tmem_st32(tbase + (static_cast<uint32_t>(warp * 32) << 16) + 128, r);
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (tid == 0) {
    uint32_t bytes = 0;
    if (MODE == 0) {
      bytes = 16384 + 16384;
      mbar_expect_tx(&sm.bar_load, bytes);
      tma_load_2d(sm.a, &map_a, &sm.bar_load, 0, 0);
      tma_load_2d(sm.b, &map_b, &sm.bar_load, 0, 0);
    } else if (MODE == 1) {
      bytes = 8192 + 4096;
      mbar_expect_tx(&sm.bar_load, bytes);
      tma_load_2d(sm.a, &map_a, &sm.bar_load, 0, 0);
      tma_load_2d(sm.b, &map_b, &sm.bar_load, 0, 0);
    } else if (MODE == 2) {
      bytes = 16384 + 16384;
      mbar_expect_tx(&sm.bar_load, bytes);
      tma_load_2d(sm.a, &map_a, &sm.bar_load, 0, 0);
      tma_load_2d(sm.a + 8192, &map_a, &sm.bar_load, 64, 0);
      tma_load_2d(sm.b, &map_b, &sm.bar_load, 0, 0);
      tma_load_2d(sm.b + 8192, &map_b, &sm.bar_load, 64, 0);
    } else {
      bytes = 48 * 128;
      mbar_expect_tx(&sm.bar_load, bytes);
      tma_load_2d(sm.b, &map_b, &sm.bar_load, 0, 0);
    }
    if (mbar_wait(&sm.bar_load, 0, &sm.abort, 9001)) {
      tc_fence_after();
      const uint32_t sa = smem_u32(sm.a), sb = smem_u32(sm.b);
      if (MODE == 0) {
        const uint32_t idesc = make_idesc_f16(128, 128, 1, false, false);
        for (int kk = 0; kk < 4; ++kk)
          mma_ss(tbase, make_smem_desc(sa + kk * 32, 16, 1024, kSw128), make_smem_desc(sb + kk * 32, 16, 1024, kSw128),
                 idesc, kk > 0);
      } else if (MODE == 1) {
        const uint32_t idesc = make_idesc_f16(128, 64, 1, false, false);
        for (int kk = 0; kk < 2; ++kk)
          mma_ss(tbase, make_smem_desc(sa + kk * 32, 16, 512, kSw64), make_smem_desc(sb + kk * 32, 16, 512, kSw64),
                 idesc, kk > 0);
      } else if (MODE == 2) {
        const uint32_t idesc = make_idesc_f16(128, 128, 1, true, true);
        for (int kk = 0; kk < 4; ++kk)
          mma_ss(tbase, make_smem_desc(sa + kk * 2048, 8192, 1024, kSw128),
                 make_smem_desc(sb + kk * 2048, 8192, 1024, kSw128), idesc, kk > 0);
      } else {
        const uint32_t idesc = make_idesc_f16(128, 48, 1, false, false);
        for (int kk = 0; kk < 4; ++kk)
          mma_ts(tbase, tbase + 128 + kk * 8, make_smem_desc(sb + kk * 32, 16, 1024, kSw128), idesc, kk > 0);
      }
      mma_commit(&sm.bar_mma);
    }
  }
  __syncwarp();
  const bool ok = mbar_wait(&sm.bar_mma, 0, &sm.abort, 9002);
  tc_fence_after();
  uint32_t r[32];
  for (int c0 = 0; c0 < n_out; c0 += 16) {
    tmem_ld16(tbase + (static_cast<uint32_t>(warp * 32) << 16) + c0, r);
    if (ok)
      for (int i = 0; i < 16; ++i) d[tid * n_out + c0 + i] = __uint_as_float(r[i]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 256);
}

}  // namespace tops

using namespace tops;

extern "C" int tops_selftest_umma(int mode, const void* a, const void* b, float* d, void* stream) {
  CUtensorMap ma{}, mb{};
  const uint64_t sA0[1] = {64 * 2};
  bool ok = true;
  int n_out = 128;
  switch (mode) {
    case 0: {
      uint64_t dims[2] = {64, 128};
      uint32_t box[2] = {64, 128};
      ok &= make_tmap(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, dims, sA0, box, CU_TENSOR_MAP_SWIZZLE_128B);
      ok &= make_tmap(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b, dims, sA0, box, CU_TENSOR_MAP_SWIZZLE_128B);
      break;
    }
    case 1: {
      uint64_t da[2] = {32, 128}, db[2] = {32, 64}, st[1] = {64};
      uint32_t ba[2] = {32, 128}, bb[2] = {32, 64};
      ok &= make_tmap(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, da, st, ba, CU_TENSOR_MAP_SWIZZLE_64B);
      ok &= make_tmap(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b, db, st, bb, CU_TENSOR_MAP_SWIZZLE_64B);
      n_out = 64;
      break;
    }
    case 2: {
      uint64_t dims[2] = {128, 64}, st[1] = {256};
      uint32_t box[2] = {64, 64};
      ok &= make_tmap(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B);
      ok &= make_tmap(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B);
      break;
    }
    case 3: {
      uint64_t dims[2] = {64, 48};
      uint32_t box[2] = {64, 48};
      ok &= make_tmap(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b, dims, sA0, box, CU_TENSOR_MAP_SWIZZLE_128B);
      ok &= make_tmap(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b, dims, sA0, box, CU_TENSOR_MAP_SWIZZLE_128B);
      n_out = 48;
      break;
    }
    default:
      return TOPS_ERR_ARG;
  }
  if (!ok) return TOPS_ERR_TMAP;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t smem = sizeof(SelftestSmem) + 1024;
  const __nv_bfloat16* arows = static_cast<const __nv_bfloat16*>(a);
  switch (mode) {
#define TOPS_LAUNCH_SELFTEST(M)                                                                        \
  case M:                                                                                            \
    cudaFuncSetAttribute(selftest_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    selftest_kernel<M><<<1, 128, smem, s>>>(ma, mb, arows, d, n_out);                                \
    break;
    TOPS_LAUNCH_SELFTEST(0)
    TOPS_LAUNCH_SELFTEST(1)
    TOPS_LAUNCH_SELFTEST(2)
    TOPS_LAUNCH_SELFTEST(3)
#undef TOPS_LAUNCH_SELFTEST
  }
  return cudaGetLastError() == cudaSuccess ? TOPS_OK : TOPS_ERR_CUDA;
}

namespace tops {
// 2^x of n f16 values by the two paths the attention softmax uses: the polynomial on
// the FMA pipe (ex2_poly_f16x2) and the MUFU (ex2.approx.f16x2).
__global__ void selftest_ex2_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ poly,
                                    uint16_t* __restrict__ mufu, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (2 * i >= n) return;
  const uint32_t lo = x[2 * i], hi = 2 * i + 1 < n ? x[2 * i + 1] : 0u;
  const uint32_t v = lo | (hi << 16);
  const uint32_t p = ex2_poly_f16x2(v), m = ex2_f16x2(v);
  poly[2 * i] = static_cast<uint16_t>(p & 0xFFFFu);
  mufu[2 * i] = static_cast<uint16_t>(m & 0xFFFFu);
  if (2 * i + 1 < n) {
    poly[2 * i + 1] = static_cast<uint16_t>(p >> 16);
    mufu[2 * i + 1] = static_cast<uint16_t>(m >> 16);
  }
}
}  // namespace tops

extern "C" int tops_selftest_ex2(const void* x_f16, void* poly_f16, void* mufu_f16, int64_t n, void* stream) {
  if (n <= 0 || n >= (int64_t(1) << 30)) return TOPS_ERR_SHAPE;
  if (x_f16 == nullptr || poly_f16 == nullptr || mufu_f16 == nullptr) return TOPS_ERR_ARG;
  const int pairs = static_cast<int>((n + 1) / 2);
  tops::selftest_ex2_kernel<<<(pairs + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(x_f16), static_cast<uint16_t*>(poly_f16), static_cast<uint16_t*>(mufu_f16),
      static_cast<int>(n));
  return cudaGetLastError() == cudaSuccess ? TOPS_OK : TOPS_ERR_CUDA;
}
