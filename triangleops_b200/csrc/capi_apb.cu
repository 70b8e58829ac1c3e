// capi_apb.cu — C-ABI entry point of attention with pair bias.
// Declared in include/triangleops_b200.h.
#include <cuda_runtime.h>
#include "sm100.cuh"
#include "status.h"

namespace tops {

template <typename T>
int launch_zbias(int dtype, const void* z, const ZBiasArgs& args, cudaStream_t st, int reserve_sms) {
  CUtensorMap mz;
  if (!map_rows(&mz, dtype, z, args.n_tok, 128, kZbTile)) return TOPS_ERR_TMAP;
  const long long tiles = (args.n_tok + kZbTile - 1) / kZbTile;
  // persistent, leaving reserve_sms SMs to the token projection that runs beside it
  int sms = sm_count() - reserve_sms;
  if (sms < sm_count() / 2) sms = sm_count() / 2;
  const int grid = tiles < sms ? static_cast<int>(tiles) : sms;
  const size_t smem = sizeof(ZbSmem) + 1024;
  auto kern = zbias_kernel<T, 128, 4>;
  set_smem(kern, smem);
  kern<<<grid, kZbThreads, smem, st>>>(mz, args);
  return launch_status();
}

}  // namespace tops

using namespace tops;

extern "C" int tops_apb_forward_rows(int dtype, int64_t M, int64_t q0, int64_t Mq, int64_t C, int64_t Cz, int64_t H,
                                     int64_t D, const void* x, const void* w_qkv, const void* z_rows, const float* wc,
                                     const float* sum_w, const float* b_const, const uint8_t* key_mask, float scale,
                                     float eps, void* q_ws, void* k_ws, void* vt_ws, void* pen_ws, void* bias_ws,
                                     void* og_rows, void* stream) {
  if (dtype != TOPS_BF16 && dtype != TOPS_F16) return TOPS_ERR_DTYPE;
  if (M <= 0 || M >= (1 << 20) || Cz != 128 || H != 4 || !attn_shape_ok(C, H, D)) return TOPS_ERR_SHAPE;
  if (q0 < 0 || Mq <= 0 || q0 + Mq > M) return TOPS_ERR_SHAPE;
  const void* ptrs[] = {x, w_qkv, z_rows, wc, sum_w, b_const, q_ws, k_ws, vt_ws, bias_ws, og_rows};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return TOPS_ERR_ALIGN;
  if (key_mask != nullptr && (pen_ws == nullptr || !aligned16(pen_ws))) return TOPS_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int m = static_cast<int>(M), mq = static_cast<int>(Mq);
  const int mkp = (m + 7) & ~7;
  ZBiasArgs za{static_cast<long long>(Mq) * M, m, mkp, mq, eps, wc, sum_w, b_const, static_cast<__half*>(bias_ws)};
  // the projection's CTAs (one per 128 tokens) run on SMs the z-bias kernel leaves free
  const int proj_ctas = (m + 127) / 128;
  int rc = dtype == TOPS_BF16 ? launch_zbias<__nv_bfloat16>(dtype, z_rows, za, st, proj_ctas)
                              : launch_zbias<__half>(dtype, z_rows, za, st, proj_ctas);
  if (rc != TOPS_OK) return rc;
  // Q/K/V projection of the whole (replicated, M x C) sequence: K/V are needed for
  // every key, and Q for all M rows costs less than a gather of the window; the
  // key mask becomes the penalty row (0 / -inf) the attention adds to every score.
  // Launched programmatically beside the z-bias kernel (it reads none of its output).
  void* pen = key_mask != nullptr ? pen_ws : nullptr;
  ProjArgs pa{m, m, 1, mkp, scale * kLog2e, eps, nullptr, nullptr, nullptr, key_mask, nullptr, q_ws, k_ws, vt_ws, pen,
              nullptr};
  pa.pdl = 1;
  rc = run_proj(dtype, static_cast<int>(C), static_cast<int>(D), false, false, x, w_qkv, pa, st);
  if (rc != TOPS_OK) return rc;
  // attention of query rows [q0, q0 + Mq): a row window of Q ([H][M][D], f16)
  const void* q_win = static_cast<const char*>(q_ws) + q0 * D * 2;
  // one row: few work units, so each CTA's two tiles split the keys of one query block
  return run_attn<2, true>(dtype, static_cast<int>(D), 1, static_cast<int>(H), mq, m, mkp, q_win, k_ws, vt_ws, pen, bias_ws,
                     og_rows, st, m);
}

extern "C" int tops_apb_forward(int dtype, int64_t M, int64_t C, int64_t Cz, int64_t H, int64_t D, const void* x,
                                const void* w_qkv, const void* z, const float* wc, const float* sum_w,
                                const float* b_const, const uint8_t* key_mask, float scale, float eps, void* q_ws,
                                void* k_ws, void* vt_ws, void* pen_ws, void* bias_ws, void* og_out, void* stream) {
  return tops_apb_forward_rows(dtype, M, 0, M, C, Cz, H, D, x, w_qkv, z, wc, sum_w, b_const, key_mask, scale, eps,
                               q_ws, k_ws, vt_ws, pen_ws, bias_ws, og_out, stream);
}
