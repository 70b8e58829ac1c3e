// status.h — status codes returned by every C-ABI entry point.
#pragma once

#define TOPS_OK 0
#define TOPS_ERR_SHAPE (-1)    /* shape / size mismatch      -> AssertionError on the Python side */
#define TOPS_ERR_DTYPE (-2)    /* unsupported IO dtype       -> ValueError                        */
#define TOPS_ERR_ARG (-3)      /* bad enum argument (e.g. direction) -> ValueError                */
#define TOPS_ERR_ALIGN (-4)    /* pointer / stride alignment not met -> AssertionError            */
#define TOPS_ERR_TMAP (-5)     /* tensor-map encode failed   -> RuntimeError                      */
#define TOPS_ERR_CUDA (-6)     /* CUDA launch / runtime error -> RuntimeError                     */
#define TOPS_ERR_TIMEOUT (-7)  /* a device-side bounded wait gave up -> RuntimeError              */
#define TOPS_ERR_CAPACITY (-8) /* problem larger than a fixed-capacity entry point accepts         */

/* IO dtype enum shared with the Python layer */
#define TOPS_F16 0
#define TOPS_BF16 1
#define TOPS_F32 2
