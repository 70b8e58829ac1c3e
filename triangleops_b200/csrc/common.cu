// common.cu — library-wide state: the device error word and its C-ABI accessors.
#include <cuda_runtime.h>
#include "sm100.cuh"
#include "status.h"

extern "C" int tops_version(void) { return 100; /* 0.1.0 */ }

extern "C" const char* tops_status_string(int code) {
  switch (code) {
    case TOPS_OK: return "ok";
    case TOPS_ERR_SHAPE: return "shape mismatch";
    case TOPS_ERR_DTYPE: return "unsupported IO dtype";
    case TOPS_ERR_ARG: return "invalid argument";
    case TOPS_ERR_ALIGN: return "misaligned pointer or stride";
    case TOPS_ERR_TMAP: return "TMA tensor-map encode failed";
    case TOPS_ERR_CUDA: return "CUDA error";
    case TOPS_ERR_TIMEOUT: return "device-side wait timed out";
    case TOPS_ERR_CAPACITY: return "size exceeds the fixed scratch capacity of this entry point";
    default: return "unknown status";
  }
}

// Copies the device error word (and the site id of the first wait that gave up)
// to the host and clears it. Synchronises the given stream. Returns TOPS_OK when
// no device-side wait has timed out since the last call, TOPS_ERR_TIMEOUT otherwise.
extern "C" int tops_device_error(void* stream, int* site) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int err = 0, where = 0;
  if (cudaStreamSynchronize(s) != cudaSuccess) return TOPS_ERR_CUDA;
  if (cudaMemcpyFromSymbol(&err, tops::g_device_error, sizeof(int)) != cudaSuccess) return TOPS_ERR_CUDA;
  if (cudaMemcpyFromSymbol(&where, tops::g_device_error_site, sizeof(int)) != cudaSuccess) return TOPS_ERR_CUDA;
  int zero = 0;
  cudaMemcpyToSymbol(tops::g_device_error, &zero, sizeof(int));
  cudaMemcpyToSymbol(tops::g_device_error_site, &zero, sizeof(int));
  if (site) *site = where;
  return err == 0 ? TOPS_OK : TOPS_ERR_TIMEOUT;
}
