// q35b.cu -- libq35b: the whole library as one translation unit (the device
// error word and the shared device helpers then need no relocatable device
// code).  Build: qwen35_b200/build.py (nvcc -gencode arch=compute_100a,
// code=sm_100a -fmad=false -shared).
#include <cstdint>
#include <cstring>

#include "q35.h"
#include "common.cuh"
#include "quant.cuh"
#include "gemv.cuh"
#include "gemv_lpr.cuh"
#include "mmq.cuh"
#include "ew.cuh"
#include "gdn.cuh"
#include "wy_tc.cuh"
#include "attn.cuh"
#include "sample.cuh"
#include "api.cuh"
#include "engine_api.cuh"
#include "noalloc.cuh"
