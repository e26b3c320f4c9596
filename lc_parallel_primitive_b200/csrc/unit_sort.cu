// Compilation unit of liblcpp_b200.so: Radix sort and the multi-GPU primitives built on it.
#include "radix_sort.cu"
#include "mg.cu"
