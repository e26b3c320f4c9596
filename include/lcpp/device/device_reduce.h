/*
 * DeviceReduce — same class template, methods and argument meaning as the
 * reference (src/lcpp/device/device_reduce.h:41-325); the work runs in the
 * sm_100a kernels of liblcpp_b200.so through lcpp_reduce(), lcpp_transform_reduce(),
 * lcpp_arg_reduce() and lcpp_reduce_by_key().
 */
#pragma once
#include "lcpp/runtime/core.h"

namespace luisa::parallel_primitive {

template <size_t BLOCK_SIZE = details::BLOCK_SIZE, size_t WARP_NUMS = details::WARP_SIZE,
          size_t ITEMS_PER_THREAD = details::ITEMS_PER_THREAD>
class DeviceReduce : public LuisaModule {
  public:
    // Reference: device_reduce.h:68-78.  The debug stream, when given, makes
    // every call commit and synchronize at once and assert success (debug
    // builds), as lcpp_check does.
    void create(Device& device, Stream* debug_stream = nullptr) {
        m_device = device;
        m_debug_stream = debug_stream;
        m_created = true;
    }

    // Reference: device_reduce.h:84-91.
    template <typename Type4Byte>
    static size_t GetTempStorageBytes(size_t num_item) {
        return lcpp_reduce_temp_bytes(lcpp_dtype_of<Type4Byte>(), num_item);
    }

    template <NumericT Type4Byte>
    void Sum(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<Type4Byte> d_in,
             BufferView<Type4Byte> d_out, size_t num_item) {
        record(cmdlist, LCPP_OP_SUM, temp_storage, d_in, d_out, num_item);
    }
    template <NumericT Type4Byte>
    void Min(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<Type4Byte> d_in,
             BufferView<Type4Byte> d_out, size_t num_item) {
        record(cmdlist, LCPP_OP_MIN, temp_storage, d_in, d_out, num_item);
    }
    // Starts from numeric_limits<T>::lowest() (the reference's min() at
    // device_reduce.h:184 differs only for floating point).
    template <NumericT Type4Byte>
    void Max(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<Type4Byte> d_in,
             BufferView<Type4Byte> d_out, size_t num_item) {
        record(cmdlist, LCPP_OP_MAX, temp_storage, d_in, d_out, num_item);
    }

    // Reference: device_reduce.h:93-108, 187-275.  Ties: ArgMin the first
    // minimum, ArgMax the last maximum (ArgMinOp / ArgMaxOp).
    template <typename Type4Byte>
    static size_t GetArgTempStorageBytes(size_t num_item) {
        return lcpp_arg_reduce_temp_bytes(lcpp_dtype_of<Type4Byte>(), num_item);
    }
    template <NumericT Type4Byte>
    void ArgMin(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<Type4Byte> d_in,
                BufferView<Type4Byte> d_out, BufferView<uint> d_index_out, size_t num_item) {
        record_arg(cmdlist, LCPP_OP_MIN, temp_storage, d_in, d_out, d_index_out, num_item);
    }
    template <NumericT Type4Byte>
    void ArgMax(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<Type4Byte> d_in,
                BufferView<Type4Byte> d_out, BufferView<uint> d_index_out, size_t num_item) {
        record_arg(cmdlist, LCPP_OP_MAX, temp_storage, d_in, d_out, d_index_out, num_item);
    }

    // Reference: device_reduce.h:331-348.  ReduceOp: SumOp / MinOp / MaxOp;
    // TransformOp: IdentityOp / SquareOp / AbsOp / NegateOp.  Temp: GetTempStorageBytes.
    template <NumericT Type4Byte, typename ReduceOp, typename TransformOp>
    void TransformReduce(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<Type4Byte> d_in,
                         BufferView<Type4Byte> d_out, size_t num_item, ReduceOp, TransformOp, Type4Byte init) {
        const int op = ReduceOp::lcpp_op, xf = TransformOp::lcpp_xf;
        cmdlist << [=](cudaStream_t s) {
            return lcpp_transform_reduce(op, xf, lcpp_dtype_of<Type4Byte>(), d_in.data(), d_out.data(), num_item,
                                         &init, temp_storage.data(), temp_storage.size_bytes(), s);
        };
        lcpp_check(cmdlist, m_debug_stream);
    }

    // Reference: device_reduce.h:110-125 (temp size), 277-325.  ReduceOp must
    // be SumOp, MinOp or MaxOp; g_num_runs_out receives the number of runs.
    template <NumericT KeyType, NumericT ValueType>
    static size_t GetReduceByKeyTempStorageBytes(size_t num_elements) {
        return lcpp_reduce_by_key_temp_bytes(lcpp_dtype_of<KeyType>(), lcpp_dtype_of<ValueType>(), num_elements);
    }
    template <NumericT KeyType, NumericT ValueType, typename ReduceOp>
    void ReduceByKey(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<KeyType> d_keys_in,
                     BufferView<ValueType> d_values_in, BufferView<KeyType> d_unique_out,
                     BufferView<ValueType> g_aggregates_out, BufferView<uint> g_num_runs_out, ReduceOp,
                     size_t num_elements) {
        const int op = ReduceOp::lcpp_op;
        cmdlist << [=](cudaStream_t s) {
            return lcpp_reduce_by_key(op, lcpp_dtype_of<KeyType>(), lcpp_dtype_of<ValueType>(), d_keys_in.data(),
                                      d_values_in.data(), d_unique_out.data(), g_aggregates_out.data(),
                                      g_num_runs_out.data(), num_elements, temp_storage.data(),
                                      temp_storage.size_bytes(), s);
        };
        lcpp_check(cmdlist, m_debug_stream);
    }

  private:
    template <typename T>
    void record_arg(CommandList& cmdlist, int op, BufferView<uint> temp, BufferView<T> in, BufferView<T> out,
                    BufferView<uint> idx, size_t n) {
        cmdlist << [=](cudaStream_t s) {
            return lcpp_arg_reduce(op, lcpp_dtype_of<T>(), in.data(), out.data(), idx.data(), n, temp.data(),
                                   temp.size_bytes(), s);
        };
        lcpp_check(cmdlist, m_debug_stream);
    }
    template <typename T>
    void record(CommandList& cmdlist, int op, BufferView<uint> temp, BufferView<T> in, BufferView<T> out,
                size_t n) {
        static_assert(lcpp_dtype_of<T>() >= 0, "unsupported element type");
        cmdlist << [=](cudaStream_t s) {
            return lcpp_reduce(op, lcpp_dtype_of<T>(), in.data(), out.data(), n, temp.data(), temp.size_bytes(), s);
        };
        lcpp_check(cmdlist, m_debug_stream);
    }
    Device m_device;
    Stream* m_debug_stream = nullptr;
    bool m_created = false;
};

}  // namespace luisa::parallel_primitive
