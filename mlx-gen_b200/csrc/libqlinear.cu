// libqlinear.cu -- single translation unit of libqlinear.so.
//
// The kernels share one device-side error word (ql::g_dev_error); building them
// as one translation unit keeps that a plain __device__ variable without
// relocatable device code.
#include "api.cu"
#include "qgemm_sm100.cu"
#include "qgemv.cu"
#include "qgemv_tma.cu"
#include "qgemv_tc.cu"
#include "qmm_generic.cu"
#include "quantize.cu"
#include "noalloc.cu"
#include "modulate.cu"
