// ct_b200.cu -- libct_b200.so is built from this single translation unit.
#include "ct_common.cuh"
#include "gemm.cu"
#include "kernels.cu"
#include "backend_abi.cu"
#include "engine.cu"
#include "noalloc.cu"
