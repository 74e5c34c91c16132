// Single translation unit of libscmp_b200.so: the kernels share one device
// error record, so they are compiled together instead of with -rdc.
#include "tables.cu"
#include "quant.cu"
#include "gemm_simt.cu"
#include "gemm_tc.cu"
#include "api.cu"
#include "levels.cu"
#include "quant_ref.cu"
#include "noalloc.cu"
