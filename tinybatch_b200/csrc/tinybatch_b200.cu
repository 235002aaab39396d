// Single translation unit of the library: the kernels share the device
// status word and inline helpers, so they are compiled together.
#include "host.cu"
#include "gemm.cu"
#include "attention.cu"
#include "misc.cu"
#include "capi.cu"
#include "comm.cu"
#include "static_scratch.cu"
