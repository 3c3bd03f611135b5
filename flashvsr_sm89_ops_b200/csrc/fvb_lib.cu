// Unity translation unit of libflashvsr_b200.so: the kernels share one device
// error word, so they are compiled together (no relocatable device code).
#include "status.cu"
#include "quant.cu"
#include "norm.cu"
#include "layout.cu"
#include "gemm_fp8.cu"
#include "bsa.cu"
#include "noalloc.cu"
#include "crop_copy.cu"
