// Single translation unit of libtalm_b200.so: the device status word and every kernel live in
// one module, so no relocatable device code is needed.
#include "abi.cu"
#include "nf4.cu"
#include "nf4_gemm.cu"
#include "peer.cu"
#include "head.cu"
#include "head_noalloc.cu"
