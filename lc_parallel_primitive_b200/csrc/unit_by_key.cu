// Compilation unit of liblcpp_b200.so: ScanByKey / ReduceByKey.
#include "by_key.cu"
