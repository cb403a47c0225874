// nvfp4_lib.cu -- the whole library as one translation unit (one definition of the device
// status word and of every kernel; no relocatable device code needed).
#include "capi_util.cu"
#include "capi.cu"
#include "quantize.cu"
#include "quantize_noalloc.cu"
#include "gemm.cu"
#include "gemm_2sm.cu"
#include "gemm_small.cu"
#include "gemm_api.cu"
#include "allreduce.cu"
