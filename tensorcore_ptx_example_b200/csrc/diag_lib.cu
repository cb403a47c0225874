// diag_lib.cu -- the diagnostics library (libnvfp4_diag.so) as one translation unit: hardware
// arithmetic probes for the parity tests and the FP4 MMA issue-rate microbenchmark.  It is built
// beside the product library and shares its sources' helpers, but nothing of the data path
// (quantizer, GEMM, all-reduce) links against it.
#include "capi_util.cu"
#include "diag_codec.cu"
#include "diag_mma.cu"
#include "diag_tile.cu"
