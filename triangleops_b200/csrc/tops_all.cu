// tops_all.cu — unity build of the TriangleOps B200 library: every kernel and
// C-ABI entry point lives in one translation unit (no relocatable device code).
#include "common.cu"
#include "selftest.cu"
#include "proj.cu"
#include "attn.cu"
#include "gate.cu"
#include "capi_attn.cu"
#include "trimul.cu"
#include "capi_trimul.cu"
#include "zbias.cu"
#include "capi_apb.cu"
#include "noalloc.cu"
#include "f32.cu"
