// The library is built as one translation unit (no relocatable device code):
// nvcc -gencode arch=compute_100a,code=sm_100a -O3 -shared praxis_b200_moe.cu
#include "common.cuh"
#include "kernels.h"

#include "router.cu"
#include "dispatch.cu"
#include "quantize.cu"
#include "gemm_nvfp4.cu"
#include "combine.cu"
#include "tail.cu"
#include "swiglu.cu"
#include "capi.cu"
