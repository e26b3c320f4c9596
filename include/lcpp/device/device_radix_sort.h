/*
 * DeviceRadixSort — same class template, methods and argument meaning as the
 * reference (src/lcpp/device/device_radix_sort.h:37-184): stable onesweep LSD
 * radix sort in liblcpp_b200.so through lcpp_radix_sort().  Inputs are not
 * modified; the sorted data lands in d_keys_out / d_values_out.
 */
#pragma once
#include "lcpp/runtime/core.h"

namespace luisa::parallel_primitive {

template <size_t BLOCK_SIZE = details::BLOCK_SIZE, size_t WARP_NUMS = details::WARP_SIZE,
          size_t ITEMS_PER_THREAD = details::ITEMS_PER_THREAD>
class DeviceRadixSort : public LuisaModule {
  public:
    void create(Device& device, Stream* debug_stream = nullptr) {  // device_radix_sort.h:67-76
        m_device = device;
        m_debug_stream = debug_stream;
    }

    template <typename KeyType, typename ValueType>
    static size_t GetSortPairsTempStorageBytes(uint num_items) {  // device_radix_sort.h:83-115
        return lcpp_radix_sort_temp_bytes(lcpp_dtype_of<KeyType>(), value_dtype<ValueType>(), num_items);
    }
    template <typename KeyType>
    static size_t GetSortKeysTempStorageBytes(uint num_items) {  // device_radix_sort.h:118-122
        return lcpp_radix_sort_temp_bytes(lcpp_dtype_of<KeyType>(), LCPP_NONE, num_items);
    }

    template <NumericT KeyType, NumericT ValueType>
    void SortPairs(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<KeyType> d_keys_in,
                   BufferView<KeyType> d_keys_out, BufferView<ValueType> d_values_in,
                   BufferView<ValueType> d_values_out, uint num_items) {
        record(cmdlist, false, temp_storage, d_keys_in, d_keys_out, d_values_in.data(), d_values_out.data(),
               value_dtype<ValueType>(), num_items);
    }
    template <NumericT KeyType>
    void SortKeys(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<KeyType> d_keys_in,
                  BufferView<KeyType> d_keys_out, uint num_items) {
        record(cmdlist, false, temp_storage, d_keys_in, d_keys_out, nullptr, nullptr, LCPP_NONE, num_items);
    }
    template <NumericT KeyType, NumericT ValueType>
    void SortPairsDescending(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<KeyType> d_keys_in,
                             BufferView<KeyType> d_keys_out, BufferView<ValueType> d_values_in,
                             BufferView<ValueType> d_values_out, uint num_items) {
        record(cmdlist, true, temp_storage, d_keys_in, d_keys_out, d_values_in.data(), d_values_out.data(),
               value_dtype<ValueType>(), num_items);
    }
    template <NumericT KeyType>
    void SortKeysDescending(CommandList& cmdlist, BufferView<uint> temp_storage, BufferView<KeyType> d_keys_in,
                            BufferView<KeyType> d_keys_out, uint num_items) {
        record(cmdlist, true, temp_storage, d_keys_in, d_keys_out, nullptr, nullptr, LCPP_NONE, num_items);
    }

  private:
    // Values move as raw bits: any 4- or 8-byte type.
    template <typename V>
    static constexpr int value_dtype() {
        static_assert(sizeof(V) == 4 || sizeof(V) == 8, "4- or 8-byte values");
        return sizeof(V) == 4 ? LCPP_U32 : LCPP_U64;
    }
    template <typename K>
    void record(CommandList& cmdlist, bool desc, BufferView<uint> temp, BufferView<K> kin, BufferView<K> kout,
                const void* vin, void* vout, int vdt, uint n) {
        static_assert(lcpp_dtype_of<K>() >= 0, "unsupported key type");
        cmdlist << [=](cudaStream_t s) {
            return lcpp_radix_sort(lcpp_dtype_of<K>(), vdt, desc ? 1 : 0, kin.data(), kout.data(), vin, vout, n, 0,
                                   0, temp.data(), temp.size_bytes(), s);
        };
        lcpp_check(cmdlist, m_debug_stream);
    }
    Device m_device;
    Stream* m_debug_stream = nullptr;
};

}  // namespace luisa::parallel_primitive
