/*
 * DeviceSegmentReduce — same class template, methods and argument meaning as
 * the reference (src/lcpp/device/device_segment_reduce.h:26-194): begin/end
 * offset overloads and fixed-size overloads of Sum/Min/Max, through
 * lcpp_segment_reduce() / lcpp_segment_reduce_fixed().
 */
#pragma once
#include "lcpp/runtime/core.h"

namespace luisa::parallel_primitive {

template <size_t BLOCK_SIZE = details::BLOCK_SIZE, size_t WARP_NUMS = details::WARP_SIZE,
          size_t ITEMS_PER_THREAD = details::ITEMS_PER_THREAD>
class DeviceSegmentReduce : public LuisaModule {
  public:
    void create(Device& device, Stream* debug_stream = nullptr) {  // device_segment_reduce.h:52-62
        m_device = device;
        m_debug_stream = debug_stream;
    }

    // The reference returns 0 (device_segment_reduce.h:71-75).  Here the size
    // enables the long-segment work list for up to num_item + 1 segments;
    // with less temp (or none) every segment is reduced by one warp.
    template <typename Type4Byte>
    static size_t GetTempStorageBytes(size_t num_item) {
        return lcpp_segment_reduce_temp_bytes(lcpp_dtype_of<Type4Byte>(), num_item, num_item + 1);
    }
    template <typename Type4Byte>
    static size_t GetTempStorageBytes(size_t num_item, size_t num_segments) {
        return lcpp_segment_reduce_temp_bytes(lcpp_dtype_of<Type4Byte>(), num_item, num_segments);
    }

#define LCPP_SEGMENT_OP(NAME, OP)                                                                               \
    template <NumericT Type4Byte>                                                                               \
    void NAME(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<Type4Byte> d_in,                  \
              BufferView<Type4Byte> d_out, uint num_segments, BufferView<uint> d_begin_offsets,                 \
              BufferView<uint> d_end_offsets) {                                                                 \
        cmdlist << [=](cudaStream_t s) {                                                                        \
            return lcpp_segment_reduce(OP, lcpp_dtype_of<Type4Byte>(), d_in.data(), d_out.data(), num_segments, \
                                       d_begin_offsets.data(), d_end_offsets.data(), temp_storage.data(),       \
                                       temp_storage.size_bytes(), s);                                           \
        };                                                                                                      \
        lcpp_check(cmdlist, m_debug_stream);                                                                    \
    }                                                                                                           \
    template <NumericT Type4Byte>                                                                               \
    void NAME(CommandList& cmdlist, BufferView<uint> /*temp_storage*/, BufferView<Type4Byte> d_in,              \
              BufferView<Type4Byte> d_out, uint num_segments, uint segment_size) {                              \
        cmdlist << [=](cudaStream_t s) {                                                                        \
            return lcpp_segment_reduce_fixed(OP, lcpp_dtype_of<Type4Byte>(), d_in.data(), d_out.data(),         \
                                             num_segments, segment_size, s);                                    \
        };                                                                                                      \
        lcpp_check(cmdlist, m_debug_stream);                                                                    \
    }

    LCPP_SEGMENT_OP(Sum, LCPP_OP_SUM)
    LCPP_SEGMENT_OP(Min, LCPP_OP_MIN)
    LCPP_SEGMENT_OP(Max, LCPP_OP_MAX)  // empty segment -> lowest() (device_segment_reduce.h:186-194)
#undef LCPP_SEGMENT_OP

    // ArgMin / ArgMax per segment, index relative to the segment begin
    // (device_segment_reduce.h:197-349).  No temp needed; the size function
    // is kept for the reference's call sequence.
    template <typename Type4Byte>
    static size_t GetArgTempStorageBytes(size_t /*num_item*/, size_t /*num_segments*/) { return 0; }

#define LCPP_SEGMENT_ARG(NAME, OP)                                                                             \
    template <NumericT ValueType>                                                                              \
    void NAME(CommandList& cmdlist, BufferView<uint> /*temp_storage*/, BufferView<ValueType> d_in,             \
              BufferView<ValueType> d_out, BufferView<uint> d_index_out, uint num_segments,                    \
              BufferView<uint> d_begin_offsets, BufferView<uint> d_end_offsets) {                              \
        cmdlist << [=](cudaStream_t s) {                                                                       \
            return lcpp_segment_arg_reduce(OP, lcpp_dtype_of<ValueType>(), d_in.data(), d_out.data(),          \
                                           d_index_out.data(), num_segments, d_begin_offsets.data(),           \
                                           d_end_offsets.data(), s);                                           \
        };                                                                                                     \
        lcpp_check(cmdlist, m_debug_stream);                                                                   \
    }                                                                                                          \
    template <NumericT ValueType>                                                                              \
    void NAME(CommandList& cmdlist, BufferView<uint> /*temp_storage*/, BufferView<ValueType> d_in,             \
              BufferView<ValueType> d_out, BufferView<uint> d_index_out, uint num_segments,                    \
              uint segment_size) {                                                                             \
        cmdlist << [=](cudaStream_t s) {                                                                       \
            return lcpp_segment_arg_reduce_fixed(OP, lcpp_dtype_of<ValueType>(), d_in.data(), d_out.data(),    \
                                                 d_index_out.data(), num_segments, segment_size, s);           \
        };                                                                                                     \
        lcpp_check(cmdlist, m_debug_stream);                                                                   \
    }

    LCPP_SEGMENT_ARG(ArgMin, LCPP_OP_MIN)
    LCPP_SEGMENT_ARG(ArgMax, LCPP_OP_MAX)
#undef LCPP_SEGMENT_ARG

  private:
    Device m_device;
    Stream* m_debug_stream = nullptr;
};

}  // namespace luisa::parallel_primitive
