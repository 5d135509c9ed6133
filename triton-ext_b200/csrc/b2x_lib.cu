// Single translation unit for libb2x.so: the device status word and the
// kernels share one module without relocatable device code.
#include "b2x_api.cu"
#include "fp8_cast.cu"
#include "fp8_gemm.cu"
#include "fp8_gemm_pair.cu"
#include "fp8_gemm_smallm.cu"
#include "fp8_gemm_blockscaled.cu"
#include "fp8_gemm_blockscaled_pair.cu"
#include "fp8_gemm_mx.cu"
#include "fp8_gemm_grouped.cu"
#include "splitk_reduce.cu"
#include "stoch_round.cu"
#include "fp8_gemm_noalloc.cu"
