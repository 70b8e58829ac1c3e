// capi_trimul.cu — C-ABI entry points of the triangle multiplicative update.
// Declared in include/triangleops_b200.h.
#include <cuda_runtime.h>
#include "sm100.cuh"
#include "status.h"
#include "tmap.h"

namespace tops {

template <typename T, int C>
int launch_trimul_in(int dtype, const void* x, const void* w, const LnGateArgs& args, cudaStream_t st) {
  CUtensorMap mx, mw, mo;
  if (!map_rows(&mx, dtype, x, args.M, C, 128)) return TOPS_ERR_TMAP;
  if (!map_rows(&mw, dtype, w, 4 * C, C, C)) return TOPS_ERR_TMAP;  // C-row boxes, placed by half
  {
    // ab, D-major [2C][M]: boxes of 32 tokens x 8 channels, one per epilogue warp and step
    const uint64_t dims[2] = {static_cast<uint64_t>(args.M), static_cast<uint64_t>(2 * C)};
    const uint64_t str[1] = {static_cast<uint64_t>(args.M) * 2};
    const uint32_t box[2] = {32, 8};
    if (!make_tmap(&mo, tmap_dtype(dtype), 2, args.out, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE))
      return TOPS_ERR_TMAP;
  }
  const size_t smem = sizeof(TmInSmem<C>) + 1024;
  static_assert(sizeof(TmInSmem<C>) + 1024 <= 227 * 1024, "input phase shared memory");
  auto kern = trimul_in_kernel<T, C>;
  set_smem(kern, smem);
  const long long tiles = (args.M + 127) / 128;
  const int grid = tiles < sm_count() ? static_cast<int>(tiles) : sm_count();
  kern<<<grid, 256 + 128 * kInEpiWG, smem, st>>>(mx, mw, mo, args);
  return launch_status();
}

template <typename T, int C>
int launch_trimul_out(int dtype, const void* y, const void* x, const void* w, const LnGateArgs& args, cudaStream_t st) {
  CUtensorMap my, mx, mw;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(args.M), static_cast<uint64_t>(C)};
    const uint64_t str[1] = {static_cast<uint64_t>(args.M) * 2};
    const uint32_t box[2] = {64, C};
    if (!make_tmap(&my, tmap_dtype(dtype), 2, y, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B)) return TOPS_ERR_TMAP;
  }
  if (!map_rows(&mx, dtype, x, args.M, C, 128)) return TOPS_ERR_TMAP;
  if (!map_rows(&mw, dtype, w, 2 * C, C, 2 * C)) return TOPS_ERR_TMAP;
  const size_t smem = sizeof(TmOutSmem<C>) + 1024;
  auto kern = trimul_out_kernel<T, C>;
  set_smem(kern, smem);
  const long long tiles = (args.M + 127) / 128;
  const int grid = tiles < sm_count() ? static_cast<int>(tiles) : sm_count();
  kern<<<grid, 512, smem, st>>>(my, mx, mw, args);
  return launch_status();
}

template <typename T, bool MN>
int launch_contract(int dtype, int nb, int Mi, int L, int P, const void* a, const void* b, void* y, cudaStream_t st,
                    int j_begin, int j_end) {
  CUtensorMap ma, mb;
  int a_groups = 0;
  const int nc = L / P;
  const uint64_t e = 2;
  // a 256-column tile of B stays inside one rank-major chunk: one box per stage
  int b_one = (P == 1 || nc % kCtBN == 0) && nc % 64 == 0 ? 1 : 0;
  // MN-major B: one grouped 5-D box measured slower than four 64-column boxes (1.63 vs
  // 1.56 ms at L = 2048), so that path keeps the four loads
  constexpr int b_one_mn = 0;
  if (!MN) {
    // A [nb][Mi][L] (K = L contiguous); B: P chunks of [nb][nc][L]
    const uint64_t da[3] = {static_cast<uint64_t>(L), static_cast<uint64_t>(Mi), static_cast<uint64_t>(nb)};
    const uint64_t sa[2] = {L * e, static_cast<uint64_t>(Mi) * L * e};
    const uint32_t ba[3] = {kCtBK, kCtBM, 1};
    const uint64_t db[4] = {static_cast<uint64_t>(L), static_cast<uint64_t>(nc), static_cast<uint64_t>(nb),
                            static_cast<uint64_t>(P)};
    const uint64_t sb[3] = {L * e, static_cast<uint64_t>(nc) * L * e, static_cast<uint64_t>(nb) * nc * L * e};
    const uint32_t bbx[4] = {kCtBK, b_one ? static_cast<uint32_t>(kCtBN) : 128u, 1, 1};
    if (!make_tmap(&ma, tmap_dtype(dtype), 3, a, da, sa, ba, CU_TENSOR_MAP_SWIZZLE_128B)) return TOPS_ERR_TMAP;
    if (!make_tmap(&mb, tmap_dtype(dtype), 4, b, db, sb, bbx, CU_TENSOR_MAP_SWIZZLE_128B)) return TOPS_ERR_TMAP;
  } else {
    // A [nb][L][Mi] (M = i contiguous) viewed as {i mod 64, k, i / 64, nb}: one box of
    // {64, BK, BM / 64, 1} is the whole MN-major tile, its four 64-row groups 8 KB apart
    // (Mi % 64 == 0 on this path; else four 3-D boxes, one per group)
    const bool a4 = Mi % 64 == 0;
    const uint64_t da[4] = {64, static_cast<uint64_t>(L), static_cast<uint64_t>(Mi) / 64, static_cast<uint64_t>(nb)};
    const uint64_t sa[3] = {static_cast<uint64_t>(Mi) * e, 128, static_cast<uint64_t>(Mi) * L * e};
    const uint32_t bx[4] = {64, kCtBK, kCtBM / 64, 1};
    const uint64_t da3[3] = {static_cast<uint64_t>(Mi), static_cast<uint64_t>(L), static_cast<uint64_t>(nb)};
    const uint64_t sa3[2] = {static_cast<uint64_t>(Mi) * e, static_cast<uint64_t>(Mi) * L * e};
    const uint32_t bx3[3] = {64, kCtBK, 1};
    const uint64_t db[4] = {static_cast<uint64_t>(nc), static_cast<uint64_t>(L), static_cast<uint64_t>(nb),
                            static_cast<uint64_t>(P)};
    const uint64_t sb[3] = {static_cast<uint64_t>(nc) * e, static_cast<uint64_t>(nc) * L * e,
                            static_cast<uint64_t>(nb) * nc * L * e};
    const uint32_t bbx[4] = {64, kCtBK, 1, 1};
    // grouped view of B as for A: {j mod 64, k, j / 64 within the chunk, nb, chunk}
    const uint64_t db5[5] = {64, static_cast<uint64_t>(L), static_cast<uint64_t>(nc) / 64, static_cast<uint64_t>(nb),
                             static_cast<uint64_t>(P)};
    const uint64_t sb5[4] = {static_cast<uint64_t>(nc) * e, 128, static_cast<uint64_t>(nc) * L * e,
                             static_cast<uint64_t>(nb) * nc * L * e};
    const uint32_t bbx5[5] = {64, kCtBK, kCtBN / 64, 1, 1};
    if (a4 ? !make_tmap(&ma, tmap_dtype(dtype), 4, a, da, sa, bx, CU_TENSOR_MAP_SWIZZLE_128B)
           : !make_tmap(&ma, tmap_dtype(dtype), 3, a, da3, sa3, bx3, CU_TENSOR_MAP_SWIZZLE_128B))
      return TOPS_ERR_TMAP;
    if (b_one_mn ? !make_tmap(&mb, tmap_dtype(dtype), 5, b, db5, sb5, bbx5, CU_TENSOR_MAP_SWIZZLE_128B)
                 : !make_tmap(&mb, tmap_dtype(dtype), 4, b, db, sb, bbx, CU_TENSOR_MAP_SWIZZLE_128B))
      return TOPS_ERR_TMAP;
    a_groups = a4 ? 1 : 0;
    b_one = b_one_mn;
  }
  // y [nb][Mi][L], written in 32 x 32 boxes (64-byte swizzle) by the epilogue warps
  CUtensorMap my;
  {
    const uint64_t dy[3] = {static_cast<uint64_t>(L), static_cast<uint64_t>(Mi), static_cast<uint64_t>(nb)};
    const uint64_t sy[2] = {L * e, static_cast<uint64_t>(Mi) * L * e};
    const uint32_t by[3] = {32, 32, 1};
    if (!make_tmap(&my, tmap_dtype(dtype), 3, y, dy, sy, by, CU_TENSOR_MAP_SWIZZLE_64B)) return TOPS_ERR_TMAP;
  }
  CtArgs args{L, nb, y, Mi, nc, j_begin, j_end, a_groups, b_one};
  static_assert(sizeof(CtSmem) + 1024 <= 227 * 1024, "contraction shared memory");
  const size_t smem = sizeof(CtSmem) + 1024;
  auto kern = trimul_contract_kernel<T, MN>;
  set_smem(kern, smem);
  const long long tiles = static_cast<long long>((Mi + kCtBM - 1) / kCtBM) * ((j_end - j_begin + kCtBN - 1) / kCtBN) * nb;
  const int grid = tiles < sm_count() ? static_cast<int>(tiles) : sm_count();
  kern<<<grid, 384, smem, st>>>(ma, mb, my, args);
  return launch_status();
}

int run_trimul_in(int dtype, int C, const void* x, const void* w, const LnGateArgs& args, cudaStream_t st) {
  if (dtype == TOPS_BF16) {
    if (C == 128) return launch_trimul_in<__nv_bfloat16, 128>(dtype, x, w, args, st);
    if (C == 64) return launch_trimul_in<__nv_bfloat16, 64>(dtype, x, w, args, st);
  } else if (dtype == TOPS_F16) {
    if (C == 128) return launch_trimul_in<__half, 128>(dtype, x, w, args, st);
    if (C == 64) return launch_trimul_in<__half, 64>(dtype, x, w, args, st);
  }
  return TOPS_ERR_SHAPE;
}

int run_trimul_out(int dtype, int C, const void* y, const void* x, const void* w, const LnGateArgs& args,
                   cudaStream_t st) {
  if (dtype == TOPS_BF16) {
    if (C == 128) return launch_trimul_out<__nv_bfloat16, 128>(dtype, y, x, w, args, st);
    if (C == 64) return launch_trimul_out<__nv_bfloat16, 64>(dtype, y, x, w, args, st);
  } else if (dtype == TOPS_F16) {
    if (C == 128) return launch_trimul_out<__half, 128>(dtype, y, x, w, args, st);
    if (C == 64) return launch_trimul_out<__half, 64>(dtype, y, x, w, args, st);
  }
  return TOPS_ERR_SHAPE;
}

int run_contract(int dtype, int direction, int nb, int Mi, int L, int P, const void* a, const void* b, void* y,
                 cudaStream_t st, int j_begin = 0, int j_end = -1) {
  if (j_end < 0) j_end = L;
  if (dtype == TOPS_BF16)
    return direction == 0 ? launch_contract<__nv_bfloat16, false>(dtype, nb, Mi, L, P, a, b, y, st, j_begin, j_end)
                          : launch_contract<__nv_bfloat16, true>(dtype, nb, Mi, L, P, a, b, y, st, j_begin, j_end);
  return direction == 0 ? launch_contract<__half, false>(dtype, nb, Mi, L, P, a, b, y, st, j_begin, j_end)
                        : launch_contract<__half, true>(dtype, nb, Mi, L, P, a, b, y, st, j_begin, j_end);
}

}  // namespace tops

using namespace tops;

extern "C" int tops_trimul_input_phase(int dtype, int64_t M, int64_t C, const void* x, const uint8_t* mask,
                                       const void* w_in, const float* sum_in, const float* b_in, float eps,
                                       void* ab_out, void* stream) {
  if (dtype != TOPS_BF16 && dtype != TOPS_F16) return TOPS_ERR_DTYPE;
  if (M <= 0 || (C != 128 && C != 64)) return TOPS_ERR_SHAPE;
  if (M % 8 != 0) return TOPS_ERR_ALIGN;  // D-major rows of ab start 16-byte aligned; token pairs whole
  const void* ptrs[] = {x, w_in, sum_in, b_in, ab_out};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return TOPS_ERR_ALIGN;
  LnGateArgs args{M, eps, sum_in, b_in, mask, ab_out};
  return run_trimul_in(dtype, static_cast<int>(C), x, w_in, args, static_cast<cudaStream_t>(stream));
}

extern "C" int tops_trimul_contract(int dtype, int direction, int64_t nb, int64_t L, const void* a, const void* b,
                                    void* y, void* stream) {
  if (dtype != TOPS_BF16 && dtype != TOPS_F16) return TOPS_ERR_DTYPE;
  if (direction != 0 && direction != 1) return TOPS_ERR_ARG;
  if (nb <= 0 || L <= 0 || nb >= (1 << 30) || L >= (1 << 20)) return TOPS_ERR_SHAPE;
  if (L % 8 != 0) return TOPS_ERR_ALIGN;
  const void* ptrs[] = {a, b, y};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return TOPS_ERR_ALIGN;
  return run_contract(dtype, direction, static_cast<int>(nb), static_cast<int>(L), static_cast<int>(L), 1, a, b, y,
                      static_cast<cudaStream_t>(stream));
}

// Row-slab contraction for sharded runs: this rank's Mi output rows against the
// all-gathered B, which is laid out as P rank-major chunks of L/P columns
// (exactly what all_gather_into_tensor produces). See the header for layouts.
extern "C" int tops_trimul_contract_slab(int dtype, int direction, int64_t nb, int64_t Mi, int64_t L, int64_t P,
                                         const void* a, const void* b, void* y, void* stream) {
  if (dtype != TOPS_BF16 && dtype != TOPS_F16) return TOPS_ERR_DTYPE;
  if (direction != 0 && direction != 1) return TOPS_ERR_ARG;
  if (nb <= 0 || L <= 0 || Mi <= 0 || P <= 0 || Mi > L || nb >= (1 << 30) || L >= (1 << 20)) return TOPS_ERR_SHAPE;
  if (L % P != 0) return TOPS_ERR_SHAPE;
  if (L % 8 != 0 || Mi % 8 != 0) return TOPS_ERR_ALIGN;
  if (P > 1 && (L / P) % 128 != 0) return TOPS_ERR_SHAPE;  // a 128-row B box stays inside one chunk
  const void* ptrs[] = {a, b, y};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return TOPS_ERR_ALIGN;
  return run_contract(dtype, direction, static_cast<int>(nb), static_cast<int>(Mi), static_cast<int>(L),
                      static_cast<int>(P), a, b, y, static_cast<cudaStream_t>(stream));
}

// The same contraction restricted to output columns [j_begin, j_begin + j_count): lets a
// sharded caller contract each chunk of B as soon as the collective has delivered it.
// j_begin must be a multiple of 256 (the tile width), and so must j_count unless the
// range ends at L; B is still the full rank-major chunk buffer (only the chunks holding
// the range are read).
extern "C" int tops_trimul_contract_slab_cols(int dtype, int direction, int64_t nb, int64_t Mi, int64_t L, int64_t P,
                                              int64_t j_begin, int64_t j_count, const void* a, const void* b, void* y,
                                              void* stream) {
  if (dtype != TOPS_BF16 && dtype != TOPS_F16) return TOPS_ERR_DTYPE;
  if (direction != 0 && direction != 1) return TOPS_ERR_ARG;
  if (nb <= 0 || L <= 0 || Mi <= 0 || P <= 0 || Mi > L || nb >= (1 << 30) || L >= (1 << 20)) return TOPS_ERR_SHAPE;
  if (L % P != 0) return TOPS_ERR_SHAPE;
  if (L % 8 != 0 || Mi % 8 != 0) return TOPS_ERR_ALIGN;
  if (P > 1 && (L / P) % 128 != 0) return TOPS_ERR_SHAPE;
  if (j_begin < 0 || j_count <= 0 || j_begin + j_count > L || j_begin % 256 != 0) return TOPS_ERR_SHAPE;
  if (j_count % 256 != 0 && j_begin + j_count != L) return TOPS_ERR_SHAPE;
  const void* ptrs[] = {a, b, y};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return TOPS_ERR_ALIGN;
  return run_contract(dtype, direction, static_cast<int>(nb), static_cast<int>(Mi), static_cast<int>(L),
                      static_cast<int>(P), a, b, y, static_cast<cudaStream_t>(stream), static_cast<int>(j_begin),
                      static_cast<int>(j_begin + j_count));
}

extern "C" int tops_trimul_output_phase(int dtype, int64_t M, int64_t C, const void* y, const void* x,
                                        const void* w_out, const float* sum_out, const float* b_out, float eps,
                                        void* out, void* stream) {
  if (dtype != TOPS_BF16 && dtype != TOPS_F16) return TOPS_ERR_DTYPE;
  if (M <= 0 || (C != 128 && C != 64)) return TOPS_ERR_SHAPE;
  if (M % 8 != 0) return TOPS_ERR_ALIGN;
  const void* ptrs[] = {y, x, w_out, sum_out, b_out, out};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return TOPS_ERR_ALIGN;
  LnGateArgs args{M, eps, sum_out, b_out, nullptr, out};
  return run_trimul_out(dtype, static_cast<int>(C), y, x, w_out, args, static_cast<cudaStream_t>(stream));
}

extern "C" int tops_trimul_output_phase_residual(int dtype, int64_t M, int64_t C, const void* y, const void* x,
                                                 const void* w_out, const float* sum_out, const float* b_out,
                                                 float eps, const void* residual, void* out, void* stream) {
  if (dtype != TOPS_BF16 && dtype != TOPS_F16) return TOPS_ERR_DTYPE;
  if (M <= 0 || (C != 128 && C != 64)) return TOPS_ERR_SHAPE;
  if (M % 8 != 0) return TOPS_ERR_ALIGN;
  const void* ptrs[] = {y, x, w_out, sum_out, b_out, residual, out};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return TOPS_ERR_ALIGN;
  LnGateArgs args{M, eps, sum_out, b_out, nullptr, out, residual};
  return run_trimul_out(dtype, static_cast<int>(C), y, x, w_out, args, static_cast<cudaStream_t>(stream));
}

// The whole op: input phase -> contraction -> output phase on one stream.
// ab_ws: [2C][B*L*L] workspace, y_ws: [C][B*L*L] workspace.
extern "C" int tops_trimul_forward(int dtype, int direction, int64_t B, int64_t L, int64_t C, const void* x,
                                   const uint8_t* mask, const void* w_in, const float* sum_in, const float* b_in,
                                   const void* w_out, const float* sum_out, const float* b_out, float eps,
                                   void* ab_ws, void* y_ws, void* out, void* stream) {
  if (direction != 0 && direction != 1) return TOPS_ERR_ARG;
  const int64_t M = B * L * L;
  int rc = tops_trimul_input_phase(dtype, M, C, x, mask, w_in, sum_in, b_in, eps, ab_ws, stream);
  if (rc != TOPS_OK) return rc;
  const size_t half = static_cast<size_t>(C) * M * 2;
  rc = tops_trimul_contract(dtype, direction, C * B, L, ab_ws, static_cast<const uint8_t*>(ab_ws) + half, y_ws,
                            stream);
  if (rc != TOPS_OK) return rc;
  return tops_trimul_output_phase(dtype, M, C, y_ws, x, w_out, sum_out, b_out, eps, out, stream);
}
