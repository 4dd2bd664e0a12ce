// libb200q8.cu -- the whole library as one translation unit, so the per-device
// status word and the kernels share one module without relocatable device code.
#include "quantize.cu"
#include "gemv.cu"
#include "gemm.cu"
#include "gemm_tc.cu"
#include "decode_step.cu"
#include "attention.cu"
#include "abi.cu"
#include "chain.cu"
#include "pack_host.cu"
#include "noalloc.cu"
#include "gguf.cu"
#include "frame.cu"
