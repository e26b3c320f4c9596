// Single translation unit of liblcpp_b200.so: the per-device error word and
// spin cap are shared by every kernel without relocatable device code.
#include "runtime.cu"
#include "reduce.cu"
#include "scan.cu"
#include "scan_pipe.cu"
#include "radix_sort.cu"
#include "segment_reduce.cu"
#include "arg_reduce.cu"
#include "scan_noalloc.cu"
#include "by_key.cu"
