// Unity translation unit of libs2s.so: the kernels share the device error word
// g_s2s_err, so they are compiled together instead of with relocatable device code.
#include "gemm_tc.cu"
#include "attention.cu"
#include "qkv_attention.cu"
#include "mlp.cu"
#include "misc.cu"
#include "halo_push.cu"
#include "engine.cu"
#include "image.cu"
#include "noalloc.cu"
