// workspace.cu — byte sizes of the caller-owned workspaces of each entry point
// (host-only; no device work). A C caller sizes its allocations with these
// instead of restating the layouts; each also validates the shape it is given.
#include <cstdint>
#include "status.h"

namespace {
inline int64_t pad8(int64_t n) { return (n + 7) & ~int64_t(7); }
inline int64_t io_bytes(int dtype) { return dtype == TOPS_F32 ? 4 : 2; }
}  // namespace

// triangle attention over R pair rows of an N x N pair tensor (R = N unsharded):
// bytes[0..5] = xln, q, k, vt, pen, bias (the bias for the R rows projected here;
// tops_triangle_attn_attend takes the full [H][N][Np] bias, i.e. R = N)
extern "C" int tops_triangle_attn_workspace_bytes(int dtype, int64_t R, int64_t N, int64_t C, int64_t H, int64_t D,
                                                  int64_t* bytes) {
  if (bytes == nullptr) return TOPS_ERR_ARG;
  if (dtype != TOPS_BF16 && dtype != TOPS_F16) return TOPS_ERR_DTYPE;
  if (R <= 0 || N <= 0 || R > N || C <= 0 || H <= 0 || D <= 0) return TOPS_ERR_SHAPE;
  const int64_t np = pad8(N);
  bytes[0] = R * N * C * io_bytes(dtype);  // x~ [R][N][C]
  bytes[1] = R * H * N * D * 2;            // Q  [R][H][N][D] f16
  bytes[2] = R * H * N * D * 2;            // K
  bytes[3] = R * H * D * np * 2;           // V^T [R][H][D][Np] f16
  bytes[4] = R * np * 2;                   // key-penalty rows [R][Np] f16 (masked calls only)
  bytes[5] = H * R * np * 2;               // bias [H][R][Np] f16
  return TOPS_OK;
}

// triangle multiplicative update: bytes[0] = ab [2C][B*L*L], bytes[1] = y [C][B*L*L]
extern "C" int tops_trimul_workspace_bytes(int dtype, int64_t B, int64_t L, int64_t C, int64_t* bytes) {
  if (bytes == nullptr) return TOPS_ERR_ARG;
  if (dtype != TOPS_BF16 && dtype != TOPS_F16) return TOPS_ERR_DTYPE;
  if (B <= 0 || L <= 0 || C <= 0) return TOPS_ERR_SHAPE;
  const int64_t m = B * L * L;
  bytes[0] = 2 * C * m * io_bytes(dtype);
  bytes[1] = C * m * io_bytes(dtype);
  return TOPS_OK;
}

// attention with pair bias over query rows [q0, q0 + Mq) of M tokens (Mq = M unsharded):
// bytes[0..4] = q, k, vt, pen, bias
extern "C" int tops_apb_workspace_bytes(int64_t M, int64_t Mq, int64_t H, int64_t D, int64_t* bytes) {
  if (bytes == nullptr) return TOPS_ERR_ARG;
  if (M <= 0 || Mq <= 0 || Mq > M || H <= 0 || D <= 0) return TOPS_ERR_SHAPE;
  const int64_t mp = pad8(M);
  bytes[0] = H * M * D * 2;   // Q [H][M][D] f16 (all M rows: the row window is read from it)
  bytes[1] = H * M * D * 2;   // K
  bytes[2] = H * D * mp * 2;  // V^T [H][D][Mp]
  bytes[3] = mp * 2;          // key-penalty row [Mp] f16 (masked calls only)
  bytes[4] = H * Mq * mp * 2; // bias [H][Mq][Mp] f16 (log2 units)
  return TOPS_OK;
}
