// Compilation unit of liblcpp_b200.so (relocatable device code): ScanByKey / ReduceByKey.
#include "by_key.cu"
