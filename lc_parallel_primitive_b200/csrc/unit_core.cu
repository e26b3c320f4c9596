// Compilation unit of liblcpp_b200.so: Reduce, ArgMin/ArgMax, segment reduce and the library-wide state.
#include "runtime.cu"
#include "reduce.cu"
#include "segment_reduce.cu"
#include "arg_reduce.cu"
