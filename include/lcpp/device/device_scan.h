/*
 * DeviceScan — same class template, methods and argument meaning as the
 * reference (src/lcpp/device/device_scan.h:33-345); single-pass decoupled
 * look-back scans in liblcpp_b200.so through lcpp_scan*() and
 * lcpp_scan_by_key().  Element types: any of the six numeric types (int32,
 * uint32, float, int64, uint64, double), as the reference's NumericT.
 */
#pragma once
#include "lcpp/runtime/core.h"

namespace luisa::parallel_primitive {

template <size_t BLOCK_SIZE = details::BLOCK_SIZE, size_t WARP_NUMS = details::WARP_SIZE,
          size_t ITEMS_PER_THREAD = details::ITEMS_PER_THREAD>
class DeviceScan : public LuisaModule {
  public:
    void create(Device& device, Stream* debug_stream = nullptr) {  // device_scan.h:59-69
        m_device = device;
        m_debug_stream = debug_stream;
    }

    template <typename Type4Byte>
    static size_t GetTempStorageBytes(size_t num_items) {  // device_scan.h:75-89
        return lcpp_scan_temp_bytes(lcpp_dtype_of<Type4Byte>(), num_items);
    }

    template <NumericT Type4Byte>
    void ExclusiveSum(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<Type4Byte> d_in,
                      BufferView<Type4Byte> d_out, size_t num_items) {
        record(cmdlist, LCPP_SCAN_EXCLUSIVE, temp_storage, d_in, d_out, num_items);
    }
    template <NumericT Type4Byte>
    void InclusiveSum(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<Type4Byte> d_in,
                      BufferView<Type4Byte> d_out, size_t num_items) {
        record(cmdlist, LCPP_SCAN_INCLUSIVE, temp_storage, d_in, d_out, num_items);
    }

    // Reference: device_scan.h:114-178.  ScanOp must be SumOp, MinOp or MaxOp
    // (DSL lambdas cannot be passed to precompiled kernels).
    template <NumericT Type4Byte, typename ScanOp>
    void ExclusiveScan(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<Type4Byte> d_in,
                       BufferView<Type4Byte> d_out, size_t num_items, ScanOp, Type4Byte initial_value) {
        record_op(cmdlist, LCPP_SCAN_EXCLUSIVE, ScanOp::lcpp_op, temp_storage, d_in, d_out, num_items, initial_value);
    }
    template <NumericT Type4Byte, typename ScanOp>
    void InclusiveScan(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<Type4Byte> d_in,
                       BufferView<Type4Byte> d_out, size_t num_items, ScanOp, Type4Byte initial_value) {
        record_op(cmdlist, LCPP_SCAN_INCLUSIVE, ScanOp::lcpp_op, temp_storage, d_in, d_out, num_items, initial_value);
    }

    // Reference: device_scan.h:93-107 (temp size), 206-345.  Segments are runs
    // of equal consecutive keys; ScanOp must be SumOp, MinOp or MaxOp.
    template <NumericT KeyType, NumericT ValueType>
    static size_t GetScanByKeyTempStorageBytes(size_t num_items) {
        return lcpp_scan_by_key_temp_bytes(lcpp_dtype_of<KeyType>(), lcpp_dtype_of<ValueType>(), num_items);
    }
    template <NumericT KeyType, NumericT ValueType, typename ScanOp>
    void ExclusiveScanByKey(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<KeyType> d_keys_in,
                            BufferView<ValueType> d_values_in, BufferView<ValueType> d_values_out, ScanOp,
                            size_t num_items, ValueType initial_value) {
        record_by_key(cmdlist, LCPP_SCAN_EXCLUSIVE, ScanOp::lcpp_op, temp_storage, d_keys_in, d_values_in,
                      d_values_out, num_items, initial_value);
    }
    template <NumericT KeyType, NumericT ValueType, typename ScanOp>
    void InclusiveScanByKey(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<KeyType> d_keys_in,
                            BufferView<ValueType> d_values_in, BufferView<ValueType> d_values_out, ScanOp,
                            size_t num_items, ValueType initial_value) {
        record_by_key(cmdlist, LCPP_SCAN_INCLUSIVE, ScanOp::lcpp_op, temp_storage, d_keys_in, d_values_in,
                      d_values_out, num_items, initial_value);
    }
    template <NumericT Type4Byte>
    void ExclusiveSumByKey(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<Type4Byte> d_keys_in,
                           BufferView<Type4Byte> d_values_in, BufferView<Type4Byte> d_values_out, size_t num_items) {
        record_by_key(cmdlist, LCPP_SCAN_EXCLUSIVE, LCPP_OP_SUM, temp_storage, d_keys_in, d_values_in, d_values_out,
                      num_items, Type4Byte(0));
    }
    template <NumericT Type4Byte>
    void InclusiveSumByKey(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<Type4Byte> d_keys_in,
                           BufferView<Type4Byte> d_values_in, BufferView<Type4Byte> d_values_out, size_t num_items) {
        record_by_key(cmdlist, LCPP_SCAN_INCLUSIVE, LCPP_OP_SUM, temp_storage, d_keys_in, d_values_in, d_values_out,
                      num_items, Type4Byte(0));
    }

  private:
    template <typename K, typename T>
    void record_by_key(CommandList& cmdlist, int kind, int op, BufferView<uint> temp, BufferView<K> keys,
                       BufferView<T> in, BufferView<T> out, size_t n, T init) {
        cmdlist << [=](cudaStream_t s) {
            return lcpp_scan_by_key(kind, op, lcpp_dtype_of<K>(), lcpp_dtype_of<T>(), keys.data(), in.data(),
                                    out.data(), n, &init, temp.data(), temp.size_bytes(), s);
        };
        lcpp_check(cmdlist, m_debug_stream);
    }
    template <typename T>
    void record_op(CommandList& cmdlist, int kind, int op, BufferView<uint> temp, BufferView<T> in,
                   BufferView<T> out, size_t n, T init) {
        cmdlist << [=](cudaStream_t s) {
            return lcpp_scan_op(kind, op, lcpp_dtype_of<T>(), in.data(), out.data(), n, &init, temp.data(),
                                temp.size_bytes(), s);
        };
        lcpp_check(cmdlist, m_debug_stream);
    }
    template <typename T>
    void record(CommandList& cmdlist, int kind, BufferView<uint> temp, BufferView<T> in, BufferView<T> out,
                size_t n) {
        cmdlist << [=](cudaStream_t s) {
            return lcpp_scan(kind, lcpp_dtype_of<T>(), in.data(), out.data(), n, temp.data(), temp.size_bytes(), s);
        };
        lcpp_check(cmdlist, m_debug_stream);
    }
    Device m_device;
    Stream* m_debug_stream = nullptr;
};

}  // namespace luisa::parallel_primitive
