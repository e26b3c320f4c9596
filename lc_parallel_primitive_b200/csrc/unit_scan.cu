// Compilation unit of liblcpp_b200.so: Scans: tile kernel, pipelined persistent kernel, temp-free variant.
#include "scan.cu"
#include "scan_pipe.cu"
#include "scan_noalloc.cu"
