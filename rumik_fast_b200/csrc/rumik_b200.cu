// rumik_b200.cu - single translation unit of librumik_b200.so, so that the kernels and the C ABI share
// the device-side error word without relocatable device code.
#include "capi.cu"
#include "gemv_int4.cu"
#include "gemv_int8.cu"
#include "gemv_int4_multi.cu"
#include "gemv_int4_tc.cu"
#include "gemv_int8_tc.cu"
#include "mm_int4_tc.cu"
#include "allreduce.cu"
#include "attn_decode.cu"
#include "sample.cu"
#include "decode_step.cu"
