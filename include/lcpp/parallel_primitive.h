/*
 * Umbrella include of the B200 build, same path as the reference's
 * src/lcpp/parallel_primitive.h:8-33 (which also pulls in the block/warp/
 * thread layers; those are internal to the sm_100a kernels here).
 */
#pragma once
#include "lcpp/runtime/core.h"
#include "lcpp/device/device_reduce.h"
#include "lcpp/device/device_scan.h"
#include "lcpp/device/device_radix_sort.h"
#include "lcpp/device/device_segment_reduce.h"
#include "lcpp/device/device_multi_gpu.h"
