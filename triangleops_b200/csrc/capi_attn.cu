// capi_attn.cu — C-ABI entry points of the attention ops (triangle attention,
// fused gate, attention with pair bias). Declared in include/triangleops_b200.h.
#include <cuda_runtime.h>
#include <utility>
#include "sm100.cuh"
#include "status.h"
#include "tmap.h"

namespace tops {

inline int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

constexpr float kLog2e = 1.4426950408889634f;

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline CUtensorMapDataType tmap_dtype(int dtype) {
  return dtype == TOPS_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

inline int launch_status() { return cudaGetLastError() == cudaSuccess ? TOPS_OK : TOPS_ERR_CUDA; }

template <typename K>
inline void set_smem(K kernel, size_t bytes) {
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
}

// Launch with programmatic stream serialization: the kernel may be scheduled while the
// previous kernel in the stream still runs (from that kernel's pdl_trigger, or its exit
// when it has none); the kernel orders its reads of that kernel's results with pdl_wait.
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), int grid, int block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// 2-D row-major [rows][C] operand, 128-row x 64-column boxes, 128B swizzle
inline bool map_rows(CUtensorMap* m, int dtype, const void* p, int64_t rows, int64_t C, uint32_t box_rows) {
  const uint64_t dims[2] = {static_cast<uint64_t>(C), static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {static_cast<uint64_t>(C) * 2};
  const uint32_t box[2] = {64, box_rows};
  return make_tmap(m, tmap_dtype(dtype), 2, p, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// ---------------------------------------------------------------------------
// projection
// ---------------------------------------------------------------------------
template <typename T, int C, int D, bool LN, bool BP>
int launch_proj(int dtype, const void* x, const void* w, const ProjArgs& args, cudaStream_t st) {
  using Cfg = ProjCfg<C, BP>;
  CUtensorMap mx, mw;
  if (args.trans) {
    // token (i, k) at x[k * Nk + i]: dims {C, i, k}, one box = 128 positions k of one column i
    const uint64_t dims[3] = {static_cast<uint64_t>(C), static_cast<uint64_t>(args.R), static_cast<uint64_t>(args.Nk)};
    const uint64_t str[2] = {static_cast<uint64_t>(C) * 2, static_cast<uint64_t>(args.Nk) * C * 2};
    const uint32_t box[3] = {64, 1, 128};
    if (!make_tmap(&mx, tmap_dtype(dtype), 3, x, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B)) return TOPS_ERR_TMAP;
  } else if (!map_rows(&mx, dtype, x, args.T, C, 128)) {
    return TOPS_ERR_TMAP;
  }
  if (!map_rows(&mw, dtype, w, Cfg::NOUT, C, Cfg::WBOX)) return TOPS_ERR_TMAP;
  const size_t smem = sizeof(ProjSmem<C, BP>) + 1024;
  auto kern = proj_kernel<T, C, D, LN, BP>;
  set_smem(kern, smem);
  const int tiles = args.trans ? args.R * ((args.Nk + 127) / 128) : (args.T + 127) / 128;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  if (args.pdl)
    launch_pdl(kern, grid, 512, smem, st, mx, mw, args);
  else
    kern<<<grid, 512, smem, st>>>(mx, mw, args);
  return launch_status();
}

template <typename T, int C, int D>
int dispatch_proj(int dtype, bool ln, bool bp, const void* x, const void* w, const ProjArgs& args, cudaStream_t st) {
  if (ln && bp) return launch_proj<T, C, D, true, true>(dtype, x, w, args, st);
  if (!ln && bp) return launch_proj<T, C, D, false, true>(dtype, x, w, args, st);
  if (!ln && !bp) return launch_proj<T, C, D, false, false>(dtype, x, w, args, st);
  return launch_proj<T, C, D, true, false>(dtype, x, w, args, st);
}

int run_proj(int dtype, int C, int D, bool ln, bool bp, const void* x, const void* w, const ProjArgs& args,
             cudaStream_t st) {
  if (dtype == TOPS_BF16) {
    if (C == 128 && D == 32) return dispatch_proj<__nv_bfloat16, 128, 32>(dtype, ln, bp, x, w, args, st);
    if (C == 64 && D == 16) return dispatch_proj<__nv_bfloat16, 64, 16>(dtype, ln, bp, x, w, args, st);
  } else if (dtype == TOPS_F16) {
    if (C == 128 && D == 32) return dispatch_proj<__half, 128, 32>(dtype, ln, bp, x, w, args, st);
    if (C == 64 && D == 16) return dispatch_proj<__half, 64, 16>(dtype, ln, bp, x, w, args, st);
  }
  return TOPS_ERR_SHAPE;
}

// ---------------------------------------------------------------------------
// attention
// ---------------------------------------------------------------------------
template <typename T, int D, int TR, bool KS = false>
int launch_attn(int R, int H, int Nq, int Nk, int Nkp, const void* q, const void* k, const void* vt, const void* pen,
                const void* bias, void* out, cudaStream_t st, int q_head_rows) {
  using Cfg = AttnCfg<D, TR, KS>;
  const CUtensorMapSwizzle qk_sw = D == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
  const CUtensorMapDataType f16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap mq, mk, mv, mp, mb;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(Nq), static_cast<uint64_t>(R) * H};
    const uint64_t str[2] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(q_head_rows) * D * 2};
    const uint32_t box[3] = {D, 128, 1};
    if (!make_tmap(&mq, f16, 3, q, dims, str, box, qk_sw)) return TOPS_ERR_TMAP;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(Nk), static_cast<uint64_t>(R) * H};
    const uint64_t str[2] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(Nk) * D * 2};
    const uint32_t box[3] = {D, Cfg::BK, 1};
    if (!make_tmap(&mk, f16, 3, k, dims, str, box, qk_sw)) return TOPS_ERR_TMAP;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(Nk), static_cast<uint64_t>(D), static_cast<uint64_t>(R) * H};
    const uint64_t str[2] = {static_cast<uint64_t>(Nkp) * 2, static_cast<uint64_t>(Nkp) * D * 2};
    const uint32_t box[3] = {Cfg::BK, D, 1};
    if (!make_tmap(&mv, f16, 3, vt, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B)) return TOPS_ERR_TMAP;
  }
  if (pen != nullptr) {
    const uint64_t dims[2] = {static_cast<uint64_t>(Nk), static_cast<uint64_t>(R)};
    const uint64_t str[1] = {static_cast<uint64_t>(Nkp) * 2};
    const uint32_t box[2] = {Cfg::BK, 1};
    if (!make_tmap(&mp, f16, 2, pen, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE)) return TOPS_ERR_TMAP;
  } else {
    mp = mv;  // unused (has_mask = 0)
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(Nk), static_cast<uint64_t>(Nq), static_cast<uint64_t>(H)};
    const uint64_t str[2] = {static_cast<uint64_t>(Nkp) * 2, static_cast<uint64_t>(Nkp) * Nq * 2};
    const uint32_t box[3] = {static_cast<uint32_t>(Cfg::BK), 128, 1};
    if (!make_tmap(&mb, f16, 3, bias, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B)) return TOPS_ERR_TMAP;
  }
  AttnArgs args{R, Nq, Nk, out, H, pen != nullptr ? 1 : 0};
  static_assert(sizeof(AttnSmem<D, TR, KS>) + 1024 <= 227 * 1024, "attention shared memory");
  const size_t smem = sizeof(AttnSmem<D, TR, KS>) + 1024;
  auto kern = attn_kernel<T, D, TR, KS>;
  set_smem(kern, smem);
  // persistent: one CTA per SM (shared memory and TMEM allow no second), looping over units
  constexpr int urows = KS ? 1 : TR;
  const long long units = static_cast<long long>((Nq + 127) / 128) * ((R + urows - 1) / urows) * H;
  const int grid = units < sm_count() ? static_cast<int>(units) : sm_count();
  kern<<<grid, Cfg::THREADS, smem, st>>>(mq, mk, mv, mp, mb, args);
  if (cudaGetLastError() != cudaSuccess) return TOPS_ERR_CUDA;
  if (pen != nullptr) {
    // rows whose keys are all masked (rare: one vote per row, work only for dead rows)
    const int grid_d = R < 4 * sm_count() ? R : 4 * sm_count();
    // launched programmatically: the vote runs beside the attention where SMs are free
    launch_pdl(attn_deadrow_kernel<T>, grid_d, 128, 0, st, static_cast<const __half*>(pen),
               static_cast<const __half*>(vt), static_cast<T*>(out), R, Nq, Nk, Nkp, H * D);
  }
  return launch_status();
}

// TR rows share one bias tile (TR > 1 only pays off when many rows share the bias).
// pen: the [R][Nkp] f16 key-penalty rows (0 / -inf), or NULL when no key is masked.
#ifndef TOPS_ATTN_TR
#define TOPS_ATTN_TR 3
#endif
template <int TR, bool KS = false>
int run_attn(int dtype, int D, int R, int H, int Nq, int Nk, int Nkp, const void* q, const void* k, const void* vt,
             const void* pen, const void* bias, void* out, cudaStream_t st, int q_head_rows = 0) {
  // q_head_rows: rows per head of the Q buffer (Q may be a row window of a longer
  // [R][H][q_head_rows][D] array, q pointing at its first row); 0 means Nq.
  if (q_head_rows == 0) q_head_rows = Nq;
  if (q_head_rows < Nq) return TOPS_ERR_SHAPE;
  if (dtype == TOPS_BF16) {
    if (D == 32) return launch_attn<__nv_bfloat16, 32, TR, KS>(R, H, Nq, Nk, Nkp, q, k, vt, pen, bias, out, st, q_head_rows);
    if (D == 16) return launch_attn<__nv_bfloat16, 16, TR, KS>(R, H, Nq, Nk, Nkp, q, k, vt, pen, bias, out, st, q_head_rows);
  } else if (dtype == TOPS_F16) {
    if (D == 32) return launch_attn<__half, 32, TR, KS>(R, H, Nq, Nk, Nkp, q, k, vt, pen, bias, out, st, q_head_rows);
    if (D == 16) return launch_attn<__half, 16, TR, KS>(R, H, Nq, Nk, Nkp, q, k, vt, pen, bias, out, st, q_head_rows);
  }
  return TOPS_ERR_SHAPE;
}

// ---------------------------------------------------------------------------
// gate
// ---------------------------------------------------------------------------
template <typename T, int C>
int launch_gate(int dtype, int64_t T_, const void* o, const void* gin, const void* wg, const void* wo, const float* bg,
                const float* bo, void* out, cudaStream_t st, const void* residual, int trans_n) {
  CUtensorMap mg, mo, mwg, mwo;
  if (!map_rows(&mg, dtype, gin, T_, C, 128)) return TOPS_ERR_TMAP;
  if (!map_rows(&mo, dtype, o, T_, C, 128)) return TOPS_ERR_TMAP;
  if (!map_rows(&mwg, dtype, wg, C, C, C)) return TOPS_ERR_TMAP;
  if (!map_rows(&mwo, dtype, wo, C, C, C)) return TOPS_ERR_TMAP;
  GateArgs args{static_cast<int>(T_), bg, bo, out, residual, trans_n};
  const size_t smem = sizeof(GateSmem<C>) + 1024;
  auto kern = gate_kernel<T, C>;
  set_smem(kern, smem);
  const int tiles = static_cast<int>((T_ + 127) / 128);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  // scheduled early (its prologue and weight loads overlap the end of the attention);
  // the kernel waits for the previous kernel's results before it reads O or the residual
  launch_pdl(kern, grid, 640, smem, st, mg, mo, mwg, mwo, args);
  return launch_status();
}

int run_gate(int dtype, int64_t T_, int64_t C, const void* o, const void* gin, const void* wg, const void* wo,
             const float* bg, const float* bo, void* out, cudaStream_t st, const void* residual = nullptr,
             int trans_n = 0) {
  if (dtype == TOPS_BF16) {
    if (C == 128) return launch_gate<__nv_bfloat16, 128>(dtype, T_, o, gin, wg, wo, bg, bo, out, st, residual, trans_n);
    if (C == 64) return launch_gate<__nv_bfloat16, 64>(dtype, T_, o, gin, wg, wo, bg, bo, out, st, residual, trans_n);
  } else if (dtype == TOPS_F16) {
    if (C == 128) return launch_gate<__half, 128>(dtype, T_, o, gin, wg, wo, bg, bo, out, st, residual, trans_n);
    if (C == 64) return launch_gate<__half, 64>(dtype, T_, o, gin, wg, wo, bg, bo, out, st, residual, trans_n);
  }
  return TOPS_ERR_SHAPE;
}

inline bool attn_shape_ok(int64_t C, int64_t H, int64_t D) {
  return (C == 128 && H == 4 && D == 32) || (C == 64 && H == 4 && D == 16);
}

}  // namespace tops

using namespace tops;

static int project_impl(int dtype, int64_t R, int64_t N, int64_t C, int64_t H, int64_t D, const void* x, int apply_ln,
                        const float* ln_w, const float* ln_b, const void* w_qkvz, const float* bz, const uint8_t* mask,
                        float scale, float eps, void* xln_ws, void* q_ws, void* k_ws, void* vt_ws, void* pen_ws,
                        void* bias_ws, void* stream, int trans) {
  if (dtype != TOPS_BF16 && dtype != TOPS_F16) return TOPS_ERR_DTYPE;
  if (N <= 0 || R <= 0 || R > N || !attn_shape_ok(C, H, D)) return TOPS_ERR_SHAPE;
  if (R * N >= (int64_t(1) << 31)) return TOPS_ERR_SHAPE;
  if (apply_ln && (ln_w == nullptr || ln_b == nullptr)) return TOPS_ERR_ARG;
  const void* ptrs[] = {x, w_qkvz, bz, q_ws, k_ws, vt_ws, bias_ws};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return TOPS_ERR_ALIGN;
  if (xln_ws != nullptr && !aligned16(xln_ws)) return TOPS_ERR_ALIGN;
  // the penalty rows are written only for a masked call (and then required)
  if (mask != nullptr && (pen_ws == nullptr || !aligned16(pen_ws))) return TOPS_ERR_ALIGN;
  if (mask == nullptr) pen_ws = nullptr;
  const int n = static_cast<int>(N), r = static_cast<int>(R);
  const int nkp = (n + 7) & ~7;
  ProjArgs pa{r * n, n, r, nkp, scale * kLog2e, eps, ln_w, ln_b, bz, mask, apply_ln ? xln_ws : nullptr,
              q_ws, k_ws, vt_ws, pen_ws, bias_ws, trans};
  return run_proj(dtype, static_cast<int>(C), static_cast<int>(D), apply_ln != 0, true, x, w_qkvz, pa,
                  static_cast<cudaStream_t>(stream));
}

extern "C" int tops_triangle_attn_project(int dtype, int64_t R, int64_t N, int64_t C, int64_t H, int64_t D,
                                          const void* x, int apply_ln, const float* ln_w, const float* ln_b,
                                          const void* w_qkvz, const float* bz, const uint8_t* mask, float scale,
                                          float eps, void* xln_ws, void* q_ws, void* k_ws, void* vt_ws,
                                          void* pen_ws, void* bias_ws, void* stream) {
  return project_impl(dtype, R, N, C, H, D, x, apply_ln, ln_w, ln_b, w_qkvz, bz, mask, scale, eps, xln_ws, q_ws, k_ws,
                      vt_ws, pen_ws, bias_ws, stream, 0);
}

extern "C" int tops_triangle_attn_project_transposed(int dtype, int64_t R, int64_t N, int64_t C, int64_t H,
                                                     int64_t D, const void* x, int apply_ln, const float* ln_w,
                                                     const float* ln_b, const void* w_qkvz, const float* bz,
                                                     const uint8_t* mask, float scale, float eps, void* xln_ws,
                                                     void* q_ws, void* k_ws, void* vt_ws, void* pen_ws,
                                                     void* bias_ws, void* stream) {
  if (N % 8 != 0) return TOPS_ERR_ALIGN;  // the column stride N*C*2 bytes must be a multiple of 16
  return project_impl(dtype, R, N, C, H, D, x, apply_ln, ln_w, ln_b, w_qkvz, bz, mask, scale, eps, xln_ws, q_ws, k_ws,
                      vt_ws, pen_ws, bias_ws, stream, 1);
}

extern "C" int tops_triangle_attn_attend(int dtype, int64_t R, int64_t N, int64_t H, int64_t D, const void* q_ws,
                                         const void* k_ws, const void* vt_ws, const void* pen_ws,
                                         const void* bias_ws, void* o_out, void* stream) {
  if (dtype != TOPS_BF16 && dtype != TOPS_F16) return TOPS_ERR_DTYPE;
  if (N <= 0 || R <= 0 || R * N >= (int64_t(1) << 31) || H != 4 || (D != 32 && D != 16)) return TOPS_ERR_SHAPE;
  const void* ptrs[] = {q_ws, k_ws, vt_ws, bias_ws, o_out};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return TOPS_ERR_ALIGN;
  if (pen_ws != nullptr && !aligned16(pen_ws)) return TOPS_ERR_ALIGN;
  const int n = static_cast<int>(N);
  return run_attn<TOPS_ATTN_TR>(dtype, static_cast<int>(D), static_cast<int>(R), static_cast<int>(H), n, n, (n + 7) & ~7,
                        q_ws, k_ws, vt_ws, pen_ws, bias_ws, o_out, static_cast<cudaStream_t>(stream));
}

extern "C" int tops_triangle_attn_forward(int dtype, int64_t N, int64_t C, int64_t H, int64_t D, const void* x,
                                          int apply_ln, const float* ln_w, const float* ln_b, const void* w_qkvz,
                                          const float* bz, const uint8_t* mask, float scale, float eps, void* xln_ws,
                                          void* q_ws, void* k_ws, void* vt_ws, void* pen_ws, void* bias_ws,
                                          void* o_out, void* stream) {
  int rc = tops_triangle_attn_project(dtype, N, N, C, H, D, x, apply_ln, ln_w, ln_b, w_qkvz, bz, mask, scale, eps,
                                      xln_ws, q_ws, k_ws, vt_ws, pen_ws, bias_ws, stream);
  if (rc != TOPS_OK) return rc;
  return tops_triangle_attn_attend(dtype, N, N, H, D, q_ws, k_ws, vt_ws, mask != nullptr ? pen_ws : nullptr, bias_ws,
                                   o_out, stream);
}

extern "C" int tops_fused_gate_forward(int dtype, int64_t T_, int64_t C, const void* o, const void* gin,
                                       const void* wg, const void* wo, const float* bg, const float* bo, void* out,
                                       void* stream) {
  if (dtype != TOPS_BF16 && dtype != TOPS_F16) return TOPS_ERR_DTYPE;
  if (T_ <= 0 || T_ >= (int64_t(1) << 31) || (C != 128 && C != 64)) return TOPS_ERR_SHAPE;
  const void* ptrs[] = {o, gin, wg, wo, out};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return TOPS_ERR_ALIGN;
  return run_gate(dtype, T_, C, o, gin, wg, wo, bg, bo, out, static_cast<cudaStream_t>(stream));
}

extern "C" int tops_fused_gate_residual(int dtype, int64_t T_, int64_t C, const void* o, const void* gin,
                                        const void* wg, const void* wo, const float* bg, const float* bo,
                                        const void* residual, void* out, int64_t trans_n, void* stream) {
  if (dtype != TOPS_BF16 && dtype != TOPS_F16) return TOPS_ERR_DTYPE;
  if (T_ <= 0 || T_ >= (int64_t(1) << 31) || (C != 128 && C != 64)) return TOPS_ERR_SHAPE;
  if (trans_n < 0 || (trans_n > 0 && T_ % trans_n != 0)) return TOPS_ERR_SHAPE;
  const void* ptrs[] = {o, gin, wg, wo, out};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return TOPS_ERR_ALIGN;
  if (residual != nullptr && !aligned16(residual)) return TOPS_ERR_ALIGN;
  return run_gate(dtype, T_, C, o, gin, wg, wo, bg, bo, out, static_cast<cudaStream_t>(stream), residual,
                  static_cast<int>(trans_n));
}

