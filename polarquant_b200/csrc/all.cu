// Single translation unit for the library (device globals are shared across
// the kernels without relocatable device code).
#include "capi.cu"
#include "scan.cu"
#include "rotate.cu"
#include "sort.cu"
#include "encode.cu"
#include "scan2.cu"
#include "batched.cu"
#include "batched_i8.cu"
#include "batched2.cu"
#include "ivf.cu"
#include "noalloc.cu"
#include "selftest.cu"
