// lib.cu -- single translation unit of libwohper_b200.so (keeps the one
// __constant__ act-quant table and every kernel in one module, no -rdc).
#include "fp8_gemv.cu"
#include "moe.cu"
#include "decode.cu"
#include "libm_exact.cu"
#include "mla.cu"
#include "mhc.cu"
#include "grouped.cu"
#include "ep.cu"
#include "lmhead.cu"
#include "capi.cu"
#include "zcblk.cu"
#include "noalloc.cu"
