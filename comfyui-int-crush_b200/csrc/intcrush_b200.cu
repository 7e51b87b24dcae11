// Single translation unit of libintcrush_b200.so: the kernels share one
// device error word and are linked without relocatable device code.
#include "ic_common.cuh"
#include "prep.cu"
#include "gemm_tc.cu"
#include "skinny.cu"
#include "weights.cu"
#include "abi.cu"
