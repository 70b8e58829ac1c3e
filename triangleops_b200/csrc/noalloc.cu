// noalloc.cu — attention with pair bias for callers that cannot allocate device
// memory.
//
// tops_apb_forward needs five caller-provided workspaces (q, k, v^T, key-penalty row,
// f16 bias logits). Some hosts of this library cannot provide them: a serving
// runtime that owns a fixed device-memory budget and forbids any allocation after
// start-up, or an embedding framework that hands out only its own input and output
// buffers (cudaMalloc there would break its accounting, and cudaMalloc/cudaFree
// can synchronise the device in the middle of its schedule). For them,
// tops_apb_forward_noalloc runs the same three kernels with the workspaces carved
// out of one fixed array in device global memory that the library itself owns.
//
// Limits and rules:
//   * M <= kNoAllocMaxM (512) tokens; larger M returns TOPS_ERR_CAPACITY and launches
//     nothing. The array is kNoAllocBytes (about 2.5 MB) and every GPU that loads the
//     library holds it until the process exits.
//   * The array is shared by every call on a device and keeps the last call's
//     contents. Each call writes every workspace byte it later reads, so nothing has
//     to start at zero — but two calls whose kernels overlap on the GPU (e.g. on two
//     streams) race on the array and corrupt each other's results.
//   * The first call on a device looks up the array's device address with that
//     device current (cudaGetSymbolAddress). Make that first call before any CUDA
//     stream capture. The address is cached per device for the life of the process:
//     after cudaDeviceReset (or anything else that destroys and recreates the
//     device's primary context) the cached address is stale, so do not call this
//     entry point again in such a process.
#include <cuda_runtime.h>
#include <mutex>
#include "sm100.cuh"
#include "status.h"

namespace tops {

constexpr int kNoAllocMaxM = 512;
constexpr int kNoAllocH = 4, kNoAllocD = 32;

constexpr size_t na_align(size_t b) { return (b + 255) & ~size_t(255); }
constexpr size_t na_bytes(int m) {
  return 2 * na_align(size_t(kNoAllocH) * m * kNoAllocD * 2)           // q, k
         + na_align(size_t(kNoAllocH) * kNoAllocD * ((m + 7) & ~7) * 2)  // v^T
         + na_align(size_t((m + 7) & ~7) * 2)                            // key-penalty row
         + na_align(size_t(kNoAllocH) * m * ((m + 7) & ~7) * 2);         // f16 bias logits
}
constexpr size_t kNoAllocBytes = na_bytes(kNoAllocMaxM);

// The scratch itself. In host code this name is only a stand-in for the symbol,
// never a usable address: the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_apb_noalloc_scratch[kNoAllocBytes];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_na_mu;
void* g_na_ptr[kMaxDevices] = {};

// Device address of the scratch on the current device (looked up once per device).
int noalloc_scratch(uint8_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TOPS_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_na_mu);
  if (g_na_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_apb_noalloc_scratch) != cudaSuccess || p == nullptr) return TOPS_ERR_CUDA;
    g_na_ptr[dev] = p;
  }
  *out = static_cast<uint8_t*>(g_na_ptr[dev]);
  return TOPS_OK;
}
}  // namespace

}  // namespace tops

using namespace tops;

// Same contract as tops_apb_forward without the five workspace arguments; the
// workspaces live in the library-owned scratch array described above.
extern "C" int tops_apb_forward_noalloc(int dtype, int64_t M, int64_t C, int64_t Cz, int64_t H, int64_t D,
                                        const void* x, const void* w_qkv, const void* z, const float* wc,
                                        const float* sum_w, const float* b_const, const uint8_t* key_mask,
                                        float scale, float eps, void* og_out, void* stream) {
  if (dtype != TOPS_BF16 && dtype != TOPS_F16) return TOPS_ERR_DTYPE;
  if (C != 128 || H != kNoAllocH || D != kNoAllocD || Cz != 128 || M <= 0) return TOPS_ERR_SHAPE;
  if (M > kNoAllocMaxM) return TOPS_ERR_CAPACITY;
  uint8_t* base = nullptr;
  const int rc = noalloc_scratch(&base);
  if (rc != TOPS_OK) return rc;
  const int m = static_cast<int>(M), mkp = (m + 7) & ~7;
  uint8_t* q = base;
  uint8_t* k = q + na_align(size_t(kNoAllocH) * m * kNoAllocD * 2);
  uint8_t* vt = k + na_align(size_t(kNoAllocH) * m * kNoAllocD * 2);
  uint8_t* maskf = vt + na_align(size_t(kNoAllocH) * kNoAllocD * mkp * 2);
  uint8_t* bias = maskf + na_align(size_t(mkp) * 2);
  return tops_apb_forward(dtype, M, C, Cz, H, D, x, w_qkv, z, wc, sum_w, b_const, key_mask, scale, eps, q, k, vt,
                          maskf, bias, og_out, stream);
}
