// Single translation unit for libb2attn.so: the device error record is one
// __device__ symbol shared by every kernel, without relocatable device code.
#include "api.cu"
#include "decode.cu"
#include "rope_append.cu"
#include "prefill.cu"
#include "prefill_pair.cu"
#include "prefill_head.cu"
#include "prefill_f32.cu"
#include "gemm.cu"
#include "kvconvert.cu"
#include "qwen35_layer.cu"
#include "q8gemv.cu"
#include "rowops.cu"
