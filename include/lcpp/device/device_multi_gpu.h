/*
 * MultiDevice — multi-GPU extensions of DeviceReduce::Sum/Min/Max
 * (src/lcpp/device/device_reduce.h:169-185), DeviceScan::ExclusiveSum/
 * InclusiveSum (device_scan.h:180-204) and DeviceRadixSort::SortPairs/SortKeys
 * (device_radix_sort.h:129-153).  The reference is single-GPU; these calls
 * take a shard per rank of an NCCL communicator (one process per GPU) and
 * work on the concatenation of the shards in rank order, through
 * lcpp_mg_reduce / lcpp_mg_scan / lcpp_mg_sort of liblcpp_b200.so.
 *
 * The communicator is the caller's ncclComm_t, passed as void* (this header
 * does not need nccl.h); every rank records the same calls.  Commands are
 * recorded in a CommandList and run when it is committed, like the
 * single-GPU classes.  SortPairs/SortKeys write this rank's slice length to
 * *n_out (host memory) when the command runs.
 */
#pragma once
#include "lcpp/runtime/core.h"

namespace luisa::parallel_primitive {

class MultiDevice : public LuisaModule {
  public:
    void create(Device& device, void* nccl_comm, Stream* debug_stream = nullptr) {
        m_device = device;
        m_comm = nccl_comm;
        m_debug_stream = debug_stream;
    }

    // ---- reduce (result on every rank) -------------------------------------
    template <NumericT T>
    static size_t GetReduceTempStorageBytes(size_t num_local) {
        return lcpp_mg_reduce_temp_bytes(lcpp_dtype_of<T>(), num_local);
    }
    template <NumericT T>
    void Sum(CommandList& cmdlist, BufferView<uint> temp, BufferView<T> d_in, BufferView<T> d_out, size_t num_local) {
        record_reduce(cmdlist, LCPP_OP_SUM, temp, d_in, d_out, num_local);
    }
    template <NumericT T>
    void Min(CommandList& cmdlist, BufferView<uint> temp, BufferView<T> d_in, BufferView<T> d_out, size_t num_local) {
        record_reduce(cmdlist, LCPP_OP_MIN, temp, d_in, d_out, num_local);
    }
    template <NumericT T>
    void Max(CommandList& cmdlist, BufferView<uint> temp, BufferView<T> d_in, BufferView<T> d_out, size_t num_local) {
        record_reduce(cmdlist, LCPP_OP_MAX, temp, d_in, d_out, num_local);
    }

    // ---- prefix sums with cross-GPU carries ---------------------------------
    template <NumericT T>
    static size_t GetScanTempStorageBytes(size_t num_local, int num_ranks) {
        return lcpp_mg_scan_temp_bytes(lcpp_dtype_of<T>(), num_local, num_ranks);
    }
    template <NumericT T>
    void ExclusiveSum(CommandList& cmdlist, BufferView<uint> temp, BufferView<T> d_in, BufferView<T> d_out,
                      size_t num_local) {
        record_scan(cmdlist, LCPP_SCAN_EXCLUSIVE, temp, d_in, d_out, num_local);
    }
    template <NumericT T>
    void InclusiveSum(CommandList& cmdlist, BufferView<uint> temp, BufferView<T> d_in, BufferView<T> d_out,
                      size_t num_local) {
        record_scan(cmdlist, LCPP_SCAN_INCLUSIVE, temp, d_in, d_out, num_local);
    }

    // ---- global stable sort --------------------------------------------------
    // capacity: room for this rank's slice in the output buffers (>= num_local).
    template <NumericT K, NumericT V>
    static size_t GetSortPairsTempStorageBytes(uint num_local, uint capacity, int num_ranks) {
        return lcpp_mg_sort_temp_bytes(lcpp_dtype_of<K>(), lcpp_dtype_of<V>(), num_local, capacity, num_ranks);
    }
    template <NumericT K>
    static size_t GetSortKeysTempStorageBytes(uint num_local, uint capacity, int num_ranks) {
        return lcpp_mg_sort_temp_bytes(lcpp_dtype_of<K>(), LCPP_NONE, num_local, capacity, num_ranks);
    }
    template <NumericT K, NumericT V>
    void SortPairs(CommandList& cmdlist, BufferView<uint> temp, BufferView<K> d_keys_in, BufferView<K> d_keys_out,
                   BufferView<V> d_values_in, BufferView<V> d_values_out, uint num_local, uint capacity,
                   uint64_t* n_out) {
        void* comm = m_comm;
        cmdlist << [=](cudaStream_t s) {
            return lcpp_mg_sort(lcpp_dtype_of<K>(), lcpp_dtype_of<V>(), d_keys_in.data(), d_values_in.data(),
                                num_local, d_keys_out.data(), d_values_out.data(), capacity, n_out, temp.data(),
                                temp.size_bytes(), comm, s);
        };
        lcpp_check(cmdlist, m_debug_stream);
    }
    template <NumericT K>
    void SortKeys(CommandList& cmdlist, BufferView<uint> temp, BufferView<K> d_keys_in, BufferView<K> d_keys_out,
                  uint num_local, uint capacity, uint64_t* n_out) {
        void* comm = m_comm;
        cmdlist << [=](cudaStream_t s) {
            return lcpp_mg_sort(lcpp_dtype_of<K>(), LCPP_NONE, d_keys_in.data(), nullptr, num_local,
                                d_keys_out.data(), nullptr, capacity, n_out, temp.data(), temp.size_bytes(), comm, s);
        };
        lcpp_check(cmdlist, m_debug_stream);
    }

  private:
    template <typename T>
    void record_reduce(CommandList& cmdlist, int op, BufferView<uint> temp, BufferView<T> in, BufferView<T> out,
                       size_t n) {
        void* comm = m_comm;
        cmdlist << [=](cudaStream_t s) {
            return lcpp_mg_reduce(op, lcpp_dtype_of<T>(), in.data(), out.data(), n, temp.data(), temp.size_bytes(),
                                  comm, s);
        };
        lcpp_check(cmdlist, m_debug_stream);
    }
    template <typename T>
    void record_scan(CommandList& cmdlist, int kind, BufferView<uint> temp, BufferView<T> in, BufferView<T> out,
                     size_t n) {
        void* comm = m_comm;
        cmdlist << [=](cudaStream_t s) {
            return lcpp_mg_scan(kind, lcpp_dtype_of<T>(), in.data(), out.data(), n, temp.data(), temp.size_bytes(),
                                comm, s);
        };
        lcpp_check(cmdlist, m_debug_stream);
    }
    Device m_device;
    void* m_comm = nullptr;
    Stream* m_debug_stream = nullptr;
};

}  // namespace luisa::parallel_primitive
