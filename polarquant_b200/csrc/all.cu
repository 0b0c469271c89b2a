// Single translation unit for the library (device globals are shared across
// the kernels without relocatable device code).
#include "capi.cu"
#include "scan.cu"
#include "rotate.cu"
#include "sort.cu"
#include "encode.cu"
#include "batched.cu"
#include "ivf.cu"
#include "noalloc.cu"
