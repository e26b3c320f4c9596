/*
 * lcpp_b200.h — C ABI of liblcpp_b200.so, the B200 (sm_100a) implementation of
 * LCPP's device-level primitives (DeviceReduce, DeviceScan, DeviceRadixSort,
 * DeviceSegmentReduce).
 *
 * Conventions shared by every entry point:
 *   - All pointers are device pointers unless the name says host.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - Every call is asynchronous on `stream`, allocates no device memory and
 *     takes its scratch space from the caller's `temp` buffer, whose size is
 *     given by the matching *_temp_bytes() function (CUB-style two-phase use,
 *     as in the reference's GetTempStorageBytes).  `temp` must be 256-byte
 *     aligned (cudaMalloc memory always is).
 *   - Return value: LCPP_OK or a negative lcpp_status.  Launch-time errors are
 *     returned directly; device-side errors (a look-back wait that gave up)
 *     are latched in a per-device error word read by lcpp_last_device_error().
 *   - Calls are reentrant: distinct calls on distinct streams with distinct
 *     temp buffers are independent.
 *
 * Reference interfaces replaced (paths inside Ligo04/lc_parallel_primitive):
 *   DeviceReduce        src/lcpp/device/device_reduce.h:84-91,131-185
 *   DeviceScan          src/lcpp/device/device_scan.h:75-89,114-204
 *   DeviceRadixSort     src/lcpp/device/device_radix_sort.h:83-184
 *   DeviceSegmentReduce src/lcpp/device/device_segment_reduce.h:71-194
 * The C++ class templates of those files are kept, with the same names and
 * signatures, in include/lcpp/ and forward to the functions below.
 */
#ifndef LCPP_B200_H
#define LCPP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int lcpp_status;

enum {
    LCPP_OK                   = 0,
    LCPP_ERR_INVALID_ARG      = -1, /* bad dtype/op, null pointer, n too large  */
    LCPP_ERR_TEMP_TOO_SMALL   = -2, /* temp_bytes < *_temp_bytes()               */
    LCPP_ERR_CUDA             = -3, /* a CUDA runtime call or launch failed      */
    LCPP_ERR_LOOKBACK_TIMEOUT = -4, /* a look-back wait hit its iteration cap    */
    LCPP_ERR_NCCL             = -5, /* an NCCL call failed (multi-GPU entries)   */
    LCPP_ERR_UNSUPPORTED      = -6, /* valid request this build does not serve   */
    LCPP_ERR_CAPACITY         = -7  /* multi-GPU sort: rank's slice > capacity   */
};

/* Element types.  The reference's NumericT (common/type_trait.h:11-14) admits
 * every integral and floating type; this ABI serves the 4- and 8-byte ones. */
typedef enum {
    LCPP_I32 = 0,
    LCPP_U32 = 1,
    LCPP_F32 = 2,
    LCPP_I64 = 3,
    LCPP_U64 = 4,
    LCPP_F64 = 5,
    LCPP_NONE = 15 /* "no values" for SortKeys */
} lcpp_dtype;

/* Reduction operators: SumOp / MinOp / MaxOp of common/thread_operators.h. */
typedef enum { LCPP_OP_SUM = 0, LCPP_OP_MIN = 1, LCPP_OP_MAX = 2 } lcpp_op;

typedef enum { LCPP_SCAN_EXCLUSIVE = 0, LCPP_SCAN_INCLUSIVE = 1 } lcpp_scan_kind;

const char* lcpp_status_string(lcpp_status s);
size_t      lcpp_dtype_size(int dtype);

/* ---- DeviceReduce ------------------------------------------------------
 * out[0] = init (+) reduce(in[0..n)), init = 0 / +max / lowest for
 * Sum / Min / Max.  Replaces DeviceReduce::Sum/Min/Max
 * (device_reduce.h:169-185) and GetTempStorageBytes (device_reduce.h:84-91).
 * Max starts from numeric_limits<T>::lowest() (the reference's min() at
 * device_reduce.h:184 is wrong for negative floats; ints are identical).
 * dtype: any of I32 U32 F32 I64 U64 F64.  Integer sums wrap (mod 2^bits). */
size_t      lcpp_reduce_temp_bytes(int dtype, uint64_t n);
lcpp_status lcpp_reduce(int op, int dtype, const void* in, void* out, uint64_t n,
                        void* temp, size_t temp_bytes, void* stream);

/* ---- DeviceScan ---------------------------------------------------------
 * Exclusive: out[i] = sum(in[0..i)), out[0] = 0.  Inclusive: sum(in[0..i]).
 * Replaces DeviceScan::ExclusiveSum/InclusiveSum (device_scan.h:180-204) and
 * GetTempStorageBytes (device_scan.h:75-89).  Single-pass decoupled
 * look-back.  dtype: any of I32 U32 F32 I64 U64 F64 (the reference's
 * NumericT, common/type_trait.h:11-14); integer sums wrap.  In-place
 * (in == out) is allowed. */
size_t      lcpp_scan_temp_bytes(int dtype, uint64_t n);
lcpp_status lcpp_scan(int kind, int dtype, const void* in, void* out, uint64_t n,
                      void* temp, size_t temp_bytes, void* stream);
/* Same, with every output offset by the device scalar *carry_in (same dtype);
 * carry_in == NULL means 0.  Used by the sharded multi-GPU scan. */
lcpp_status lcpp_scan_carry(int kind, int dtype, const void* in, void* out, uint64_t n,
                            const void* carry_in, void* temp, size_t temp_bytes,
                            void* stream);

/* Exclusive / inclusive scan with op in {LCPP_OP_SUM, LCPP_OP_MIN, LCPP_OP_MAX}
 * and an initial value: out[i] = init (+) in[0] (+) ... (+) in[i-1]
 * (exclusive; out[0] = init) or ... (+) in[i] (inclusive).  init is a HOST
 * pointer to one element of dtype (NULL = the op's identity).  Replaces
 * DeviceScan::ExclusiveScan / InclusiveScan with SumOp / MinOp / MaxOp
 * (device_scan.h:114-178); arbitrary DSL lambdas cannot cross a C ABI. */
lcpp_status lcpp_scan_op(int kind, int op, int dtype, const void* in, void* out, uint64_t n,
                         const void* init, void* temp, size_t temp_bytes, void* stream);

/* ---- DeviceRadixSort ----------------------------------------------------
 * Stable LSD radix sort (8-bit digits, onesweep) of keys[begin_bit,end_bit),
 * values travelling with their keys.  keys_in/values_in are not modified.
 * Replaces DeviceRadixSort::SortKeys/SortPairs(+Descending)
 * (device_radix_sort.h:129-184) and Get*TempStorageBytes
 * (device_radix_sort.h:83-122).
 * key_dtype: I32 U32 F32 I64 U64 F64.  value_dtype: LCPP_NONE (keys only) or
 * any 4- or 8-byte dtype (values are moved as raw bits).  Floats order by
 * value with -0.0 == +0.0 (radix_rank_sort_operations.h:30-43); NaNs order by
 * bit pattern.  n < 2^32.  begin_bit/end_bit as in CUB (0 / 8*sizeof(K) for
 * a full sort); pass end_bit <= 0 for "all bits". */
size_t      lcpp_radix_sort_temp_bytes(int key_dtype, int value_dtype, uint64_t n);
lcpp_status lcpp_radix_sort(int key_dtype, int value_dtype, int descending,
                            const void* keys_in, void* keys_out,
                            const void* values_in, void* values_out, uint64_t n,
                            int begin_bit, int end_bit,
                            void* temp, size_t temp_bytes, void* stream);

/* Boundaries of the 256 digit runs of keys that are already ordered by the
 * 8-bit digit at bit_start (e.g. after lcpp_radix_sort with
 * begin_bit = bit_start, end_bit = bit_start + 8): starts[d] = first index
 * whose digit is >= d, starts[256] = n (257 uint64 outputs, device memory).
 * Digits use the same order-preserving key image as the sort (ascending).
 * No counterpart in the reference; the multi-GPU sort uses it to cut a
 * partitioned shard into per-rank bucket ranges. */
lcpp_status lcpp_radix_bucket_starts(int key_dtype, const void* keys, uint64_t n, int bit_start,
                                     uint64_t* starts, void* stream);

/* ---- DeviceSegmentReduce ------------------------------------------------
 * out[s] = init (+) reduce(in[begin[s]..end[s])); empty segment -> init.
 * Replaces DeviceSegmentReduce::Sum/Min/Max with begin/end offset views
 * (device_segment_reduce.h:125-194; Max's init is lowest(), :186-194).
 * dtype: any of I32 U32 F32 I64 U64 F64.  Offsets are uint32 (the
 * reference's BufferView<uint>); a CSR offsets[S+1] array is passed as
 * begin = offsets, end = offsets + 1.  With the temp of
 * lcpp_segment_reduce_temp_bytes(dtype, num_items, S) (num_items = the last
 * end offset) and monotone offsets (begin[s] <= end[s] <= begin[s+1], e.g.
 * CSR), the work is split by items into 32 KiB tiles, whatever the segment
 * lengths; other offsets are reduced one warp per segment (checked on the
 * device).  temp may be NULL or smaller (the reference's GetTempStorageBytes
 * returns 0 here, device_segment_reduce.h:71-75): the call then reduces one
 * warp per segment. */
size_t      lcpp_segment_reduce_temp_bytes(int dtype, uint64_t num_items,
                                           uint64_t num_segments);
lcpp_status lcpp_segment_reduce(int op, int dtype, const void* in, void* out,
                                uint64_t num_segments, const uint32_t* begin_offsets,
                                const uint32_t* end_offsets,
                                void* temp, size_t temp_bytes, void* stream);
/* Fixed-size segments: segment s is in[s*segment_size .. (s+1)*segment_size).
 * Replaces the segment_size overloads (device_segment_reduce.h:109-123,
 * 137-170).  Needs no temp. */
lcpp_status lcpp_segment_reduce_fixed(int op, int dtype, const void* in, void* out,
                                      uint64_t num_segments, uint64_t segment_size,
                                      void* stream);

/* ---- DeviceScan without temp storage ----------------------------------
 * No counterpart in the reference.  For callers that cannot allocate device
 * memory when they scan (allocator or memory-pool callbacks, plug-ins that
 * only receive their input/output buffers, real-time paths that forbid
 * allocation after start-up): same result as lcpp_scan, with the scratch
 * taken from a fixed ~128 KiB device array inside the library instead of a
 * caller temp buffer.  n <= lcpp_scan_noalloc_max_items() (2^29), larger n
 * returns LCPP_ERR_INVALID_ARG.  The array is shared by all calls on a device:
 * calls that overlap on the GPU race and must be serialized.  The first call
 * on a device looks up the array's address (cudaGetSymbolAddress); make it
 * before any stream capture (made during capture it returns
 * LCPP_ERR_UNSUPPORTED).  The address is kept per device ordinal, so
 * cudaDeviceReset while the library is loaded is not supported.  Allocates
 * nothing. */
uint64_t    lcpp_scan_noalloc_max_items(void);
lcpp_status lcpp_scan_noalloc(int kind, int dtype, const void* in, void* out, uint64_t n,
                              void* stream);

/* ---- ArgMin / ArgMax ---------------------------------------------------
 * Value and index of the minimum / maximum.  Replaces DeviceReduce::ArgMin/
 * ArgMax and GetArgTempStorageBytes (device_reduce.h:93-108,187-275) and
 * DeviceSegmentReduce::ArgMin/ArgMax (device_segment_reduce.h:197-349).
 * Ties follow the reference's ArgMinOp / ArgMaxOp (thread_operators.h:19-47):
 * ArgMin returns the smallest index, ArgMax the largest.  Segment indices are
 * relative to the segment begin.  Empty input / segment: index 1 and
 * value max() (ArgMin) or lowest() (ArgMax).  op: LCPP_OP_MIN or LCPP_OP_MAX;
 * dtype: any of I32 U32 F32 I64 U64 F64; n < 2^32. */
size_t      lcpp_arg_reduce_temp_bytes(int dtype, uint64_t n);
lcpp_status lcpp_arg_reduce(int op, int dtype, const void* in, void* out_value, uint32_t* out_index,
                            uint64_t n, void* temp, size_t temp_bytes, void* stream);
lcpp_status lcpp_segment_arg_reduce(int op, int dtype, const void* in, void* out_value,
                                    uint32_t* out_index, uint64_t num_segments,
                                    const uint32_t* begin_offsets, const uint32_t* end_offsets,
                                    void* stream);
lcpp_status lcpp_segment_arg_reduce_fixed(int op, int dtype, const void* in, void* out_value,
                                          uint32_t* out_index, uint64_t num_segments,
                                          uint64_t segment_size, void* stream);

/* ---- TransformReduce ----------------------------------------------------
 * out = op(init, reduce_op over transform(in[i])).  Replaces DeviceReduce::
 * TransformReduce (device_reduce.h:331-348), whose reduce and transform
 * operators are DSL lambdas: here op is LCPP_OP_SUM/MIN/MAX and transform one
 * of the LCPP_XF_* element maps below (integer square / negate wrap).  init is
 * a HOST pointer to one element of dtype (NULL = the op's identity).  Temp:
 * lcpp_reduce_temp_bytes. */
enum { LCPP_XF_IDENTITY = 0, LCPP_XF_SQUARE = 1, LCPP_XF_ABS = 2, LCPP_XF_NEGATE = 3 };
lcpp_status lcpp_transform_reduce(int op, int transform, int dtype, const void* in, void* out, uint64_t n,
                                  const void* init, void* temp, size_t temp_bytes, void* stream);

/* ---- ScanByKey / ReduceByKey ------------------------------------------
 * Segments are runs of equal consecutive keys (a new one starts where
 * keys[i] != keys[i-1]; float keys compare by value).  op in {SUM, MIN, MAX};
 * key_dtype and value_dtype: any of I32 U32 F32 I64 U64 F64; n < 2^32.
 *
 * lcpp_scan_by_key: per-segment scan of values_in, seeded by the HOST value
 * *init (NULL = the op's identity): exclusive out[i] = init at a segment head,
 * op(v[head] .. v[i-1], init) elsewhere; inclusive out[i] =
 * op(v[head] .. v[i], init).  values_out may equal values_in.  Replaces
 * DeviceScan::ExclusiveScanByKey / InclusiveScanByKey / ExclusiveSumByKey /
 * InclusiveSumByKey and GetScanByKeyTempStorageBytes (device_scan.h:93-107,
 * 206-345).
 *
 * lcpp_reduce_by_key: one output per run: unique_out[r] = key of the run's
 * last item, aggregates_out[r] = op over the run's values, *num_runs_out
 * (device) = number of runs (0 for n == 0).  Replaces DeviceReduce::
 * ReduceByKey and GetReduceByKeyTempStorageBytes (device_reduce.h:110-125,
 * 277-325). */
size_t      lcpp_scan_by_key_temp_bytes(int key_dtype, int value_dtype, uint64_t n);
lcpp_status lcpp_scan_by_key(int kind, int op, int key_dtype, int value_dtype, const void* keys,
                             const void* values_in, void* values_out, uint64_t n, const void* init,
                             void* temp, size_t temp_bytes, void* stream);
size_t      lcpp_reduce_by_key_temp_bytes(int key_dtype, int value_dtype, uint64_t n);
lcpp_status lcpp_reduce_by_key(int op, int key_dtype, int value_dtype, const void* keys_in,
                               const void* values_in, void* unique_out, void* aggregates_out,
                               uint32_t* num_runs_out, uint64_t n, void* temp, size_t temp_bytes,
                               void* stream);


/* ---- Multi-GPU (one process per GPU, NCCL) -----------------------------
 * No counterpart in the reference, which is single-GPU and limits item
 * counts to 32 bits (device_radix_sort.h:136, details/scan.h:72).  These
 * extend DeviceReduce::Sum/Min/Max (device_reduce.h:169-185),
 * DeviceScan::ExclusiveSum/InclusiveSum (device_scan.h:180-204) and
 * DeviceRadixSort::SortPairs/SortKeys (device_radix_sort.h:129-153) to data
 * sharded over the ranks of an NCCL communicator: the global sequence is
 * the concatenation of the ranks' shards in rank order.  `comm` is an
 * ncclComm_t passed as void*; every rank of it must make the same call.
 * NCCL is loaded at run time (libnccl.so.2); without it these return
 * LCPP_ERR_NCCL.  Scratch comes from `temp`; nothing is allocated. */
size_t      lcpp_mg_unique_id_bytes(void);                 /* sizeof(ncclUniqueId) */
lcpp_status lcpp_mg_get_unique_id(void* id_out);           /* ncclGetUniqueId */
lcpp_status lcpp_mg_comm_init_rank(void** comm_out, int nranks, const void* id, int rank);
lcpp_status lcpp_mg_comm_destroy(void* comm);
lcpp_status lcpp_mg_comm_shape(void* comm, int* rank, int* nranks);

/* *out (device, every rank) = op over all ranks' shards.  Asynchronous. */
size_t      lcpp_mg_reduce_temp_bytes(int dtype, uint64_t n_local);
lcpp_status lcpp_mg_reduce(int op, int dtype, const void* in, void* out, uint64_t n_local,
                           void* temp, size_t temp_bytes, void* comm, void* stream);

/* Prefix sum of the global sequence; each rank writes its shard's part.
 * Local reduce -> all-gather of the G shard totals -> carry = sum of the
 * lower ranks' totals (rank order) -> local scan seeded with the carry.
 * Integer results are bit-exact (mod 2^bits).  dtype: any of the six.
 * Asynchronous. */
size_t      lcpp_mg_scan_temp_bytes(int dtype, uint64_t n_local, int nranks);
lcpp_status lcpp_mg_scan(int kind, int dtype, const void* in, void* out, uint64_t n_local,
                         void* temp, size_t temp_bytes, void* comm, void* stream);

/* Global stable ascending sort of (key, value) pairs (value_dtype LCPP_NONE:
 * keys only).  Rank r receives the r-th contiguous slice of the sorted global
 * sequence in keys_out/values_out (room for `capacity` items, capacity >=
 * n_local) and its length in *n_out (host).  Ranks are cut at splitters
 * sampled from every shard (4096 samples per rank) on the extended key
 * (key, rank, index), so slices are near n_total / nranks whatever the key
 * distribution, duplicates included; a slice longer than capacity returns
 * LCPP_ERR_CAPACITY.  At most 256 ranks.  Slices move by CUDA IPC pulls (copy
 * engines, LCPP_MG_PULL_STREAMS streams per source, default 4) when every
 * rank's temp can be exported, else by NCCL send/recv (environment
 * LCPP_MG_EXCHANGE=nccl forces it).  Equal keys keep
 * their global input order.  Waits on `stream` for the exchange sizes (and
 * once more for the ranks' agreement on the IPC path); the rest is
 * asynchronous.  n_local, capacity < 2^32. */
size_t      lcpp_mg_sort_temp_bytes(int key_dtype, int value_dtype, uint64_t n_local,
                                    uint64_t capacity, int nranks);
lcpp_status lcpp_mg_sort(int key_dtype, int value_dtype, const void* keys_in, const void* values_in,
                         uint64_t n_local, void* keys_out, void* values_out, uint64_t capacity,
                         uint64_t* n_out, void* temp, size_t temp_bytes, void* comm, void* stream);
/* The sort's splitter choice on the host (the device computes the same):
 * given the gathered samples in ascending extended-key order (key image,
 * position = rank << 32 | index) with their weights, splitter r-1 (r = 1 ..
 * nranks-1) is the sample where the running weight crosses r/nranks of the
 * total.  Host pointers; no GPU needed. */
lcpp_status lcpp_mg_pick_splitters(const uint64_t* keys, const uint64_t* pos, const uint64_t* weights,
                                   uint64_t count, int nranks, uint64_t* split_keys, uint64_t* split_pos);

/* ---- Device error word --------------------------------------------------
 * Synchronizes `stream`, returns the first device-side error latched since
 * the last call on the current device (LCPP_OK if none) and clears it.  The
 * reference has no device-side error reporting (runtime/core.h:57-66). */
lcpp_status lcpp_last_device_error(void* stream);

/* ---- Look-back unit hooks ----------------------------------------------
 * Run the scan's decoupled look-back alone, one tile per CTA, with tile t
 * contributing aggregates[t]: exclusive_out[t] = sum(aggregates[0..t)),
 * inclusive_out[t] = exclusive_out[t] + aggregates[t].  Mirrors the
 * reference's stand-alone TilePrefixCallbackOp test
 * (tests/decoupled_look_back.cpp:57-180).  temp: lcpp_lookback_temp_bytes. */
size_t      lcpp_lookback_temp_bytes(uint64_t num_tiles);
lcpp_status lcpp_lookback_tiles(const uint32_t* aggregates, uint32_t* exclusive_out,
                                uint32_t* inclusive_out, uint64_t num_tiles,
                                void* temp, size_t temp_bytes, void* stream);
/* Caps every look-back wait at `iterations` polls (0 restores the default,
 * about one second) on the current device. */
lcpp_status lcpp_set_spin_limit(uint32_t iterations);
/* One warp runs the look-back of tile `tile` against the caller's descriptor
 * array (num_tiles 64-bit words, status in the high half: 0 = not yet
 * published, 1 = partial, 2 = inclusive) and writes the exclusive prefix to
 * *exclusive_out.  A descriptor that is never published makes the wait run
 * out: the kernel returns, *exclusive_out is unspecified and
 * lcpp_last_device_error() reports LCPP_ERR_LOOKBACK_TIMEOUT. */
lcpp_status lcpp_lookback_probe(const uint64_t* descriptors, uint64_t tile,
                                uint32_t* exclusive_out, void* stream);

/* ---- Per-kernel timing ---------------------------------------------------
 * lcpp_profile_enable(1) makes every launch site of this library bracket its
 * kernel with CUDA events on the launching stream (0 turns it off); both
 * calls reset the totals.  lcpp_profile_read() waits for the recorded events
 * and returns, for one kernel kind ("reduce", "scan", "rs_memset",
 * "rs_histogram", "rs_bins_scan", "rs_onesweep", "seg_warp", "seg_block"),
 * the number of timed launches and their summed duration in ms. */
lcpp_status lcpp_profile_enable(int on);
lcpp_status lcpp_profile_read(const char* kernel, uint64_t* launches, double* total_ms);

/* ---- Library info ------------------------------------------------------ */
/* Number of kernels this library launched from the calling process (all
 * devices, all streams) since load; for launch accounting in benchmarks. */
uint64_t    lcpp_kernel_launch_count(void);
/* Binary version (major*10+minor, e.g. 100 for sm_100a) of the library's
 * kernels on the current device (cudaFuncGetAttributes), or a negative
 * lcpp_status. */
int         lcpp_kernel_binary_version(void);
const char* lcpp_build_info(void);

#ifdef __cplusplus
}
#endif
#endif /* LCPP_B200_H */
