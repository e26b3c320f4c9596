// Multi-GPU primitives on one node over NCCL (one process per GPU): reduce,
// scan with cross-GPU carries, and a global stable sort.  The reference has
// no multi-GPU code; these extend its single-GPU entry points
// (src/lcpp/device/device_reduce.h:169-185, device_scan.h:180-204,
// device_radix_sort.h:129-153) to data sharded in rank order, and lift the
// reference's 32-bit item count (device_radix_sort.h:136, details/scan.h:72).
//
// NCCL is resolved at run time (dlopen of libnccl.so.2; in a process that
// already loaded NCCL, e.g. through PyTorch, that copy is reused), so the
// library loads and its single-GPU entry points work on hosts without NCCL.
// The communicator is the caller's ncclComm_t, passed as void*.
//
// Every entry point is asynchronous on the caller's stream except
// lcpp_mg_sort, which waits for the exchange sizes (they must be known on the
// host) and, on the IPC path, once more for the ranks' agreement on it.  Scratch comes from
// the caller's temp buffer; nothing is allocated.
//
// Global sort, G ranks (ascending, stable over the concatenation of the
// shards in rank order):
//   1. each rank takes 4096 evenly spaced samples of its shard, as extended
//      keys (order-preserving key image, rank << 32 | index) weighted by the
//      shard size; NCCL all-gathers them.  The gathered samples are sorted on the device
//      by this library's radix sort, and G-1 splitters are picked where the
//      running weight crosses r/G.  Splitting on extended keys cuts runs of
//      equal keys between ranks in input order, so every rank gets about
//      n_total/G items whatever the key distribution.
//   2. a bucket kernel gives every item its destination rank (number of
//      splitters <= its extended key, one byte) and reduces the shard's key
//      min/max; one stable onesweep pass over those bytes groups the shard
//      by destination.
//   3. one NCCL group all-gathers the G bucket starts and all-reduces the
//      global key min/max (bits above the highest differing bit are equal in
//      every key and need no sorting); this rank's send offsets and receive
//      counts are copied to the host (the one synchronisation).
//   4. exchange of keys and values, runs landing in source rank order: each
//      rank pulls its slices from the peers' shards by cudaMemcpyAsync over
//      CUDA IPC mappings (copy engines, one stream per source; a one-word NCCL
//      all-reduce then fences the shards), or, where a shard cannot be
//      exported, grouped ncclSend/ncclRecv.
//   5. local onesweep sort of the bits that differ, from the received runs
//      into the caller's output.  Stable passes + rank-ordered runs keep
//      equal keys in global input order.
// Rank r ends with the r-th contiguous slice of the global order and its
// length is returned.
#include "common.cuh"
#include <algorithm>
#include <dlfcn.h>
#include <nccl.h>
#include <mutex>
#include <string>
#include <vector>

namespace lcpp {

// ---------------------------------------------------------------------------
// NCCL entry points, resolved once.
// ---------------------------------------------------------------------------
struct NcclApi {
    bool ok = false;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommCount)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*CommUserRank)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
};

static const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        bool ok = true;
        auto get = [&](auto& fp, const char* name) {
            fp = reinterpret_cast<std::remove_reference_t<decltype(fp)>>(dlsym(h, name));
            ok = ok && fp != nullptr;
        };
        get(api.GetUniqueId, "ncclGetUniqueId");
        get(api.CommInitRank, "ncclCommInitRank");
        get(api.CommDestroy, "ncclCommDestroy");
        get(api.CommCount, "ncclCommCount");
        get(api.CommUserRank, "ncclCommUserRank");
        get(api.AllReduce, "ncclAllReduce");
        get(api.AllGather, "ncclAllGather");
        get(api.Send, "ncclSend");
        get(api.Recv, "ncclRecv");
        get(api.GroupStart, "ncclGroupStart");
        get(api.GroupEnd, "ncclGroupEnd");
        api.ok = ok;
    });
    return api;
}

#define MG_NCCL(call)                                         \
    do {                                                      \
        if ((call) != ncclSuccess) return LCPP_ERR_NCCL;      \
    } while (0)
#define MG_CUDA(call)                                         \
    do {                                                      \
        if ((call) != cudaSuccess) return LCPP_ERR_CUDA;      \
    } while (0)

// Non-blocking side streams per device (created on first use): stream 0
// copies this rank's own slice, streams 1 + p K .. p K + K pull from peer p.
struct SideStreams {
    std::mutex mu;
    std::vector<std::vector<cudaStream_t>> per_dev;
};
static SideStreams& side_streams() {
    static SideStreams s;
    return s;
}
static cudaStream_t side_stream(int i = 0) {
    SideStreams& ss = side_streams();
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || i < 0) return nullptr;
    std::lock_guard<std::mutex> g(ss.mu);
    if ((size_t)dev >= ss.per_dev.size()) ss.per_dev.resize((size_t)dev + 1);
    auto& v = ss.per_dev[dev];
    if ((size_t)i >= v.size()) v.resize((size_t)i + 1, nullptr);
    if (!v[i] && cudaStreamCreateWithFlags(&v[i], cudaStreamNonBlocking) != cudaSuccess) v[i] = nullptr;
    return v[i];
}
// Wait for every side stream of the current device.
static void sync_side_streams() {
    SideStreams& ss = side_streams();
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return;
    std::lock_guard<std::mutex> g(ss.mu);
    if ((size_t)dev < ss.per_dev.size())
        for (cudaStream_t st : ss.per_dev[dev])
            if (st) cudaStreamSynchronize(st);
}

// ---------------------------------------------------------------------------
// Exchange by CUDA IPC: every rank exports the allocation that holds its
// partitioned shard (cudaIpcGetMemHandle on the allocation's base, found with
// cuMemGetAddressRange), the handles travel with the bucket-start all-gather,
// and each rank pulls its slices from the peers with cudaMemcpyAsync (copy
// engines; no kernel reads peer memory).  Peer mappings are kept per device
// and handle for the life of the process, so that repeated sorts from the
// same buffers open each peer allocation once.
// ---------------------------------------------------------------------------
struct MgIpcRec {           // one per rank, all-gathered (12 x uint64)
    cudaIpcMemHandle_t h;   // 64 bytes
    uint64_t off_k, off_v;  // offsets of the partitioned keys / values from the allocation base
    uint64_t ok;            // 1: exported
};
static_assert(sizeof(MgIpcRec) == 88, "MgIpcRec layout");
constexpr size_t MG_IPC_REC_U64 = 12;  // 96 bytes on the wire

using GetAddressRangeFn = int (*)(unsigned long long*, size_t*, unsigned long long);

static bool alloc_base(const void* p, char** base) {
    static GetAddressRangeFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (GetAddressRangeFn) nullptr;
        return (GetAddressRangeFn)f;
    }();
    if (!fn) return false;
    unsigned long long b = 0;
    size_t sz = 0;
    if (fn(&b, &sz, (unsigned long long)(uintptr_t)p) != 0) return false;
    *base = (char*)(uintptr_t)b;
    return true;
}

// Copy streams per source rank of the IPC exchange (LCPP_MG_PULL_STREAMS, 1..16).
static int mg_pull_streams() {
    static const int k = [] {
        const char* e = getenv("LCPP_MG_PULL_STREAMS");
        const int v = e ? atoi(e) : 4;
        return v < 1 ? 1 : (v > 16 ? 16 : v);
    }();
    return k;
}

static bool mg_ipc_enabled() {
    static const bool on = [] {
        const char* e = getenv("LCPP_MG_EXCHANGE");
        return !(e && e[0] == 'n');  // LCPP_MG_EXCHANGE=nccl: NCCL send/recv only
    }();
    return on;
}

// Mapping of peer p's exported allocation in this process, kept per (device,
// communicator, peer): a sort from the same buffers reuses it; when the peer
// exports a different allocation, the old mapping is closed (after this
// device's side streams, the only users of mappings, have drained), so that a
// mapping never keeps a peer allocation alive after the peer has moved on.
static char* open_peer(void* comm, int p, const cudaIpcMemHandle_t& h) {
    struct Entry { int dev; void* comm; int peer; cudaIpcMemHandle_t h; char* ptr; };
    static std::mutex mu;
    static std::vector<Entry> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> g(mu);
    for (auto it = cache.begin(); it != cache.end(); ++it) {
        if (it->dev != dev || it->comm != comm || it->peer != p) continue;
        if (memcmp(&it->h, &h, sizeof(h)) == 0) return it->ptr;
        sync_side_streams();  // no copy from the old mapping is still in flight
        cudaIpcCloseMemHandle(it->ptr);
        cache.erase(it);
        break;
    }
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    cache.push_back(Entry{dev, comm, p, h, (char*)ptr});
    return (char*)ptr;
}

static bool nccl_type(int dtype, ncclDataType_t& t) {
    switch (dtype) {
        case LCPP_I32: t = ncclInt32; return true;
        case LCPP_U32: t = ncclUint32; return true;
        case LCPP_F32: t = ncclFloat32; return true;
        case LCPP_I64: t = ncclInt64; return true;
        case LCPP_U64: t = ncclUint64; return true;
        case LCPP_F64: t = ncclFloat64; return true;
        default: return false;
    }
}

static bool comm_shape(void* comm, int& rank, int& nranks) {
    const NcclApi& A = nccl();
    if (!A.ok || !comm) return false;
    return A.CommCount((ncclComm_t)comm, &nranks) == ncclSuccess &&
           A.CommUserRank((ncclComm_t)comm, &rank) == ncclSuccess && nranks > 0;
}

// ---------------------------------------------------------------------------
// Small kernels
// ---------------------------------------------------------------------------
// carry = totals[0] (+) ... (+) totals[rank-1], in rank order (one thread:
// G <= a few hundred), so every rank folds the same floats in the same order.
template <typename T>
__global__ void mg_carry_kernel(const T* totals, int rank, T* carry) {
    T c = T(0);
    for (int h = 0; h < rank; ++h) c = OpSum::apply<T>(c, totals[h]);
    *carry = c;
}

// Bits that still differ from the global {min, ~max}: info[1] = hb + 1,
// hb = highest bit where min and max differ (0: all keys equal).
__global__ void mg_range_bits_kernel(const unsigned long long* gmm, uint32_t* info) {
    const unsigned long long x = gmm[0] ^ ~gmm[1];
    const int hb = x ? 63 - __clzll((long long)x) : -1;
    info[0] = 0;
    info[1] = (uint32_t)(hb + 1);
}

// Splitters are samples of the extended key (key image, position), position
// = rank << 32 | local index: the global stable order is the lexicographic
// order of extended keys, so equal keys are split between ranks in input
// order and every rank gets an even share whatever the key distribution.
constexpr int MG_SAMPLES = 4096;  // per rank

// Sample i of this rank: the item at i * n / MG_SAMPLES, weighted by n (each
// sample stands for n / MG_SAMPLES items).  Empty shards give weight-0
// samples that sort last.
template <typename KB, int KIND>
__global__ void mg_sample_kernel(const KB* keys, uint64_t n, int me, uint64_t* skey, uint64_t* spos,
                                 uint64_t* sw, uint32_t* sidx, int G) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < MG_SAMPLES) {
        if (n) {
            const uint64_t p = (uint64_t)i * n / MG_SAMPLES;
            skey[i] = (uint64_t)ordered_bits<KB, KIND, false>(keys[p]);
            spos[i] = ((uint64_t)me << 32) | p;
            sw[i] = n;
        } else {
            skey[i] = ~0ull;
            spos[i] = ~0ull;
            sw[i] = 0;
        }
    }
    // indices 0..G*MG_SAMPLES-1 for the sort of the gathered samples
    for (int j = i; j < G * MG_SAMPLES; j += gridDim.x * blockDim.x) sidx[j] = (uint32_t)j;
}

// Splitter r (1..G-1) is the sample at which the running weight of the
// sorted samples crosses r/G of the total: cum_excl <= target < cum_incl.
__host__ __device__ inline uint64_t mg_target(uint64_t total, int r, int G) {
    return (total / G) * r + (total % G) * r / G;
}

// One CTA of 1024 threads: sorted sample order `order`, weights sw; writes
// G-1 splitter records {key, pos} to split (unused slots: {~0, ~0}).
__global__ void __launch_bounds__(1024) mg_pick_splitters_kernel(const uint64_t* skey_sorted, const uint32_t* order,
                                                                 const uint64_t* spos, const uint64_t* sw, int S,
                                                                 int G, ulonglong2* split) {
    __shared__ uint64_t s_part[1024];
    const int t = threadIdx.x;
    const int per = (S + 1023) / 1024;
    const int lo = min(S, t * per), hi = min(S, lo + per);
    uint64_t mine = 0;
    for (int j = lo; j < hi; ++j) mine += sw[order[j]];
    s_part[t] = mine;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {  // inclusive scan of the chunk sums
        const uint64_t v = t >= o ? s_part[t - o] : 0;
        __syncthreads();
        s_part[t] += v;
        __syncthreads();
    }
    const uint64_t total = s_part[1023];
    for (int r = t; r < G - 1; r += 1024) split[r] = make_ulonglong2(~0ull, ~0ull);
    __syncthreads();
    uint64_t cum = t ? s_part[t - 1] : 0;
    for (int j = lo; j < hi; ++j) {
        const uint64_t w = sw[order[j]];
        for (int r = 1; r < G; ++r) {
            const uint64_t target = mg_target(total, r, G);
            if (cum <= target && target < cum + w) split[r - 1] = make_ulonglong2(skey_sorted[j], spos[order[j]]);
        }
        cum += w;
    }
}

// Bucket (destination rank) of every item: the number of splitters <= its
// extended key, written as one byte per item.
template <typename KB, int KIND>
__global__ void mg_bucket_kernel(const KB* keys, uint64_t n, int me, const ulonglong2* split, int nsplit,
                                 uint8_t* digits, unsigned long long* mm) {
    __shared__ ulonglong2 s_split[256];
    // {min, ~max} of the order-preserving key image (a min-reduction of both
    // words gives the global min and max); empty shards leave the identity
    unsigned long long kmin = ~0ull, nkmax = ~0ull;
    for (int i = threadIdx.x; i < nsplit; i += blockDim.x) s_split[i] = split[i];
    __syncthreads();
    const uint64_t rank_hi = (uint64_t)me << 32;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t o = (uint64_t)ordered_bits<KB, KIND, false>(ldcs(keys + i));
        const uint64_t pos = rank_hi | i;
        int lo = 0, hi = nsplit;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            const ulonglong2 sp = s_split[mid];
            const bool le = sp.x < o || (sp.x == o && sp.y <= pos);
            if (le) lo = mid + 1; else hi = mid;
        }
        digits[i] = (uint8_t)lo;
        kmin = o < kmin ? o : kmin;
        nkmax = ~o < nkmax ? ~o : nkmax;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const unsigned long long x = __shfl_xor_sync(0xffffffffu, kmin, off);
        const unsigned long long y = __shfl_xor_sync(0xffffffffu, nkmax, off);
        kmin = x < kmin ? x : kmin;
        nkmax = y < nkmax ? y : nkmax;
    }
    if ((threadIdx.x & 31) == 0) {
        atomicMin(mm, kmin);
        atomicMin(mm + 1, nkmax);
    }
}

// Plan of this rank from the all-gathered digit starts (G rows of 257:
// starts[0..255] of the rank's partition pass, then its n).  Bucket p goes
// to rank p.  out (uint64): [0..G] send offsets into this rank's partitioned
// shard, [G+1..2G] receive counts per source rank, [2G+1] = info[1],
// [2G+2..3G+1] where this rank's slice starts in each source's shard.
__global__ void mg_plan_kernel(const uint64_t* rows, int G, int me, const uint32_t* info, uint64_t* out) {
    const uint64_t* mine = rows + (size_t)me * 257;
    for (int p = threadIdx.x; p <= G; p += blockDim.x) out[p] = p < 256 ? mine[p] : mine[256];
    for (int p = threadIdx.x; p < G; p += blockDim.x) {
        const uint64_t* row = rows + (size_t)p * 257;
        const uint64_t hi = me + 1 < 256 ? row[me + 1] : row[256];
        out[G + 1 + p] = hi - row[me];
    }
    for (int p = threadIdx.x; p < G; p += blockDim.x) out[2 * G + 2 + p] = rows[(size_t)p * 257 + me];
    if (threadIdx.x == 0) out[2 * G + 1] = info[1];
}

// Row of this rank for the all-gather: the partition pass's digit starts
// (uint32, in the sort's temp) widened, plus n.
__global__ void mg_pack_starts_kernel(const uint32_t* starts, uint64_t n, uint64_t* row) {
    const int t = threadIdx.x;
    if (t < 256) row[t] = starts[t];
    if (t == 0) row[256] = n;
}

// ---------------------------------------------------------------------------
// Sort temp layout
// ---------------------------------------------------------------------------
struct MgSortLayout {
    size_t mm, info, rows, plan, ipc, skey, spos, sw, sidx, skey_sorted, order, split, digits;
    size_t part_k, part_v, recv_k, recv_v, sort, total;
};

static MgSortLayout mg_sort_layout(int kdt, int vdt, uint64_t n_local, uint64_t capacity, int G) {
    MgSortLayout L{};
    const size_t ks = lcpp_dtype_size(kdt);
    const size_t vs = vdt == LCPP_NONE ? 0 : lcpp_dtype_size(vdt);
    const size_t S = (size_t)G * MG_SAMPLES;
    size_t o = 0;
    auto take = [&](size_t bytes) { const size_t at = o; o = align_up(o + bytes, 256); return at; };
    L.mm = take(6 * sizeof(unsigned long long));  // local {min,~max}, global {min,~max}, agreement word
    L.info = take(2 * sizeof(uint32_t));
    L.rows = take((size_t)G * 257 * sizeof(uint64_t));
    L.plan = take((size_t)(3 * G + 2) * sizeof(uint64_t));
    L.ipc = take((size_t)G * MG_IPC_REC_U64 * sizeof(uint64_t));
    uint64_t m = n_local;
    if (G > 1) {
        L.skey = take(S * 8);
        L.spos = take(S * 8);
        L.sw = take(S * 8);
        L.sidx = take(S * 4);
        L.skey_sorted = take(S * 8);
        L.order = take(S * 4);
        L.split = take(256 * sizeof(ulonglong2));
        L.digits = take(n_local);
        L.part_k = take(n_local * ks);
        L.part_v = take(n_local * vs);
        L.recv_k = take(capacity * ks);
        L.recv_v = take(capacity * vs);
        m = std::max<uint64_t>(std::max<uint64_t>(capacity, n_local), S);
    }
    // one region serves, in turn, the sample sort, the partition pass and the final sort
    const size_t big = lcpp_radix_sort_temp_bytes(kdt, vdt, m ? m : 1);
    const size_t smp = G > 1 ? lcpp_radix_sort_temp_bytes(LCPP_U64, LCPP_U32, S) : 0;
    L.sort = take(std::max(big, smp));
    L.total = o;
    return L;
}

static lcpp_status rs_sort_impl(int key_dtype, int value_dtype, int descending, const void* keys_in, void* keys_out,
                                const void* values_in, void* values_out, uint64_t n, int begin_bit, int end_bit,
                                void* temp, size_t temp_bytes, void* stream, const uint8_t* digits);

}  // namespace lcpp

using namespace lcpp;

// ---------------------------------------------------------------------------
// Communicator helpers (so that callers without their own NCCL binding, e.g.
// Python over ctypes, can build a communicator).
// ---------------------------------------------------------------------------
extern "C" size_t lcpp_mg_unique_id_bytes(void) { return sizeof(ncclUniqueId); }

extern "C" lcpp_status lcpp_mg_get_unique_id(void* id_out) {
    const NcclApi& A = nccl();
    if (!A.ok) return LCPP_ERR_NCCL;
    if (!id_out) return LCPP_ERR_INVALID_ARG;
    ncclUniqueId id;
    MG_NCCL(A.GetUniqueId(&id));
    memcpy(id_out, &id, sizeof(id));
    return LCPP_OK;
}

extern "C" lcpp_status lcpp_mg_comm_init_rank(void** comm_out, int nranks, const void* id, int rank) {
    const NcclApi& A = nccl();
    if (!A.ok) return LCPP_ERR_NCCL;
    if (!comm_out || !id || nranks <= 0 || rank < 0 || rank >= nranks) return LCPP_ERR_INVALID_ARG;
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclComm_t c = nullptr;
    MG_NCCL(A.CommInitRank(&c, nranks, uid, rank));
    *comm_out = (void*)c;
    return LCPP_OK;
}

extern "C" lcpp_status lcpp_mg_comm_destroy(void* comm) {
    const NcclApi& A = nccl();
    if (!A.ok) return LCPP_ERR_NCCL;
    if (!comm) return LCPP_ERR_INVALID_ARG;
    MG_NCCL(A.CommDestroy((ncclComm_t)comm));
    return LCPP_OK;
}

extern "C" lcpp_status lcpp_mg_comm_shape(void* comm, int* rank, int* nranks) {
    if (!rank || !nranks) return LCPP_ERR_INVALID_ARG;
    return comm_shape(comm, *rank, *nranks) ? LCPP_OK : LCPP_ERR_NCCL;
}

// ---------------------------------------------------------------------------
// Reduce
// ---------------------------------------------------------------------------
extern "C" size_t lcpp_mg_reduce_temp_bytes(int dtype, uint64_t n_local) {
    const size_t r = lcpp_reduce_temp_bytes(dtype, n_local);
    return r ? 256 + r : 0;
}

extern "C" lcpp_status lcpp_mg_reduce(int op, int dtype, const void* in, void* out, uint64_t n_local,
                                      void* temp, size_t temp_bytes, void* comm, void* stream) {
    ncclDataType_t t;
    if (!nccl_type(dtype, t) || op < 0 || op > 2 || !out || (n_local && !in)) return LCPP_ERR_INVALID_ARG;
    const size_t need = lcpp_mg_reduce_temp_bytes(dtype, n_local);
    if (!temp || temp_bytes < need) return LCPP_ERR_TEMP_TOO_SMALL;
    int rank, G;
    if (!comm_shape(comm, rank, G)) return LCPP_ERR_NCCL;
    cudaStream_t s = (cudaStream_t)stream;
    char* part = (char*)temp;  // this rank's partial (one element)
    const lcpp_status st = lcpp_reduce(op, dtype, in, part, n_local, (char*)temp + 256, need - 256, stream);
    if (st != LCPP_OK) return st;
    const ncclRedOp_t rop = op == LCPP_OP_SUM ? ncclSum : op == LCPP_OP_MIN ? ncclMin : ncclMax;
    ProfScope ps("mg_allreduce", s);
    MG_NCCL(nccl().AllReduce(part, out, 1, t, rop, (ncclComm_t)comm, s));
    return LCPP_OK;
}

// ---------------------------------------------------------------------------
// Scan
// ---------------------------------------------------------------------------
extern "C" size_t lcpp_mg_scan_temp_bytes(int dtype, uint64_t n_local, int nranks) {
    const size_t es = lcpp_dtype_size(dtype);
    const size_t sc = lcpp_scan_temp_bytes(dtype, n_local);
    if (!es || !sc || nranks <= 0) return 0;
    const size_t r = lcpp_reduce_temp_bytes(dtype, n_local);
    // [total | carry | G totals][reduce temp][scan temp]
    const size_t head = align_up(2 * 8 + (size_t)nranks * es, 256);
    return head + align_up(r, 256) + sc;
}

extern "C" lcpp_status lcpp_mg_scan(int kind, int dtype, const void* in, void* out, uint64_t n_local,
                                    void* temp, size_t temp_bytes, void* comm, void* stream) {
    ncclDataType_t t;
    if (!nccl_type(dtype, t) || (kind != LCPP_SCAN_EXCLUSIVE && kind != LCPP_SCAN_INCLUSIVE) ||
        (n_local && (!in || !out)))
        return LCPP_ERR_INVALID_ARG;
    int rank, G;
    if (!comm_shape(comm, rank, G)) return LCPP_ERR_NCCL;
    const size_t need = lcpp_mg_scan_temp_bytes(dtype, n_local, G);
    if (!need) return LCPP_ERR_INVALID_ARG;
    if (!temp || temp_bytes < need) return LCPP_ERR_TEMP_TOO_SMALL;
    cudaStream_t s = (cudaStream_t)stream;
    const size_t es = lcpp_dtype_size(dtype);
    char* base = (char*)temp;
    char* total = base;
    char* carry = base + 8;
    char* totals = base + 16;
    const size_t head = align_up(2 * 8 + (size_t)G * es, 256);
    const size_t rt = align_up(lcpp_reduce_temp_bytes(dtype, n_local), 256);
    char* rtemp = base + head;
    char* stemp = rtemp + rt;
    lcpp_status st;
    if (G == 1) {  // no carry to exchange: the local scan is the global scan
        ProfScope ps("mg_carry_scan", s);
        return n_local ? lcpp_scan_carry(kind, dtype, in, out, n_local, nullptr, stemp, temp_bytes - head - rt, stream)
                       : LCPP_OK;
    }
    {
        ProfScope ps("mg_local_reduce", s);
        st = lcpp_reduce(LCPP_OP_SUM, dtype, in, total, n_local, rtemp, rt, stream);
    }
    if (st != LCPP_OK) return st;
    {
        ProfScope ps("mg_allgather", s);
        MG_NCCL(nccl().AllGather(total, totals, 1, t, (ncclComm_t)comm, s));
        st = dispatch_dtype(dtype, [&](auto zero) -> lcpp_status {
            using T = decltype(zero);
            mg_carry_kernel<T><<<1, 1, 0, s>>>((const T*)totals, rank, (T*)carry);
            count_launch();
            return check_launch();
        });
    }
    if (st != LCPP_OK) return st;
    if (n_local == 0) return LCPP_OK;
    ProfScope ps("mg_carry_scan", s);
    return lcpp_scan_carry(kind, dtype, in, out, n_local, carry, stemp, temp_bytes - head - rt, stream);
}

// ---------------------------------------------------------------------------
// Global sort
// ---------------------------------------------------------------------------
extern "C" size_t lcpp_mg_sort_temp_bytes(int key_dtype, int value_dtype, uint64_t n_local, uint64_t capacity,
                                          int nranks) {
    if (nranks <= 0 || lcpp_radix_sort_temp_bytes(key_dtype, value_dtype, 1) == 0) return 0;
    return mg_sort_layout(key_dtype, value_dtype, n_local, capacity, nranks).total;
}

extern "C" lcpp_status lcpp_mg_pick_splitters(const uint64_t* keys, const uint64_t* pos, const uint64_t* weights,
                                               uint64_t count, int nranks, uint64_t* split_keys,
                                               uint64_t* split_pos) {
    if (!keys || !pos || !weights || !split_keys || !split_pos || nranks <= 0 || nranks > 256)
        return LCPP_ERR_INVALID_ARG;
    uint64_t total = 0;
    for (uint64_t j = 0; j < count; ++j) total += weights[j];
    for (int r = 0; r + 1 < nranks; ++r) split_keys[r] = split_pos[r] = ~0ull;
    uint64_t cum = 0;
    for (uint64_t j = 0; j < count; ++j) {
        for (int r = 1; r < nranks; ++r) {
            const uint64_t target = mg_target(total, r, nranks);
            if (cum <= target && target < cum + weights[j]) {
                split_keys[r - 1] = keys[j];
                split_pos[r - 1] = pos[j];
            }
        }
        cum += weights[j];
    }
    return LCPP_OK;
}

static int unsigned_view(size_t ks) { return ks == 4 ? LCPP_U32 : LCPP_U64; }

extern "C" lcpp_status lcpp_mg_sort(int key_dtype, int value_dtype, const void* keys_in, const void* values_in,
                                    uint64_t n_local, void* keys_out, void* values_out, uint64_t capacity,
                                    uint64_t* n_out, void* temp, size_t temp_bytes, void* comm, void* stream) {
    const int kind = key_kind(key_dtype);
    const size_t ks = lcpp_dtype_size(key_dtype);
    const size_t vs = value_dtype == LCPP_NONE ? 0 : lcpp_dtype_size(value_dtype);
    if (kind < 0 || (value_dtype != LCPP_NONE && vs == 0) || !n_out) return LCPP_ERR_INVALID_ARG;
    if ((n_local && !keys_in) || (vs && n_local && !values_in) || !keys_out || (vs && !values_out))
        return LCPP_ERR_INVALID_ARG;
    if (n_local >= (1ull << 32) || capacity >= (1ull << 32) || capacity < n_local) return LCPP_ERR_INVALID_ARG;
    int me, G;
    if (!comm_shape(comm, me, G)) return LCPP_ERR_NCCL;
    if (G > 256) return LCPP_ERR_UNSUPPORTED;  // bucket ids are bytes
    const MgSortLayout L = mg_sort_layout(key_dtype, value_dtype, n_local, capacity, G);
    if (!temp || temp_bytes < L.total) return LCPP_ERR_TEMP_TOO_SMALL;
    const NcclApi& A = nccl();
    ncclComm_t c = (ncclComm_t)comm;
    cudaStream_t s = (cudaStream_t)stream;
    char* T = (char*)temp;
    const size_t sort_bytes = L.total - L.sort;
    *n_out = 0;

    if (G == 1) {  // the local sort is the global sort
        *n_out = n_local;
        ProfScope ps("mg_local_sort", s);
        return rs_sort_impl(key_dtype, value_dtype, 0, keys_in, keys_out, values_in, values_out, n_local, 0, 0,
                            T + L.sort, sort_bytes, stream, nullptr);
    }

    unsigned long long* mm = (unsigned long long*)(T + L.mm);
    uint32_t* info = (uint32_t*)(T + L.info);
    const int S = G * MG_SAMPLES;
    uint64_t* skey = (uint64_t*)(T + L.skey);
    uint64_t* spos = (uint64_t*)(T + L.spos);
    uint64_t* sw = (uint64_t*)(T + L.sw);
    uint32_t* sidx = (uint32_t*)(T + L.sidx);
    ulonglong2* split = (ulonglong2*)(T + L.split);
    uint8_t* digits = (uint8_t*)(T + L.digits);
    const DeviceInfo di = device_info();
    const unsigned grid = (unsigned)std::min<uint64_t>(ceil_div(n_local ? n_local : 1, 1024), (uint64_t)di.sms * 4);
    lcpp_status st;
    // 1. splitters from all ranks' samples
    {
        ProfScope ps("mg_splitters", s);
        MG_CUDA(cudaMemsetAsync(mm, 0xFF, 2 * sizeof(unsigned long long), s));
        auto go = [&](auto kb) -> lcpp_status {
            using KB = decltype(kb);
            const KB* k = (const KB*)keys_in;
            const unsigned sg = (unsigned)ceil_div((uint64_t)MG_SAMPLES, 256);
            switch (kind) {
                case 0: mg_sample_kernel<KB, 0><<<sg, 256, 0, s>>>(k, n_local, me, skey + (size_t)me * MG_SAMPLES,
                                                                   spos + (size_t)me * MG_SAMPLES, sw + (size_t)me * MG_SAMPLES, sidx, G);
                        break;
                case 1: mg_sample_kernel<KB, 1><<<sg, 256, 0, s>>>(k, n_local, me, skey + (size_t)me * MG_SAMPLES,
                                                                   spos + (size_t)me * MG_SAMPLES, sw + (size_t)me * MG_SAMPLES, sidx, G);
                        break;
                default: mg_sample_kernel<KB, 2><<<sg, 256, 0, s>>>(k, n_local, me, skey + (size_t)me * MG_SAMPLES,
                                                                    spos + (size_t)me * MG_SAMPLES, sw + (size_t)me * MG_SAMPLES, sidx, G);
                         break;
            }
            count_launch();
            return check_launch();
        };
        st = ks == 4 ? go((uint32_t)0) : go((uint64_t)0);
        if (st != LCPP_OK) return st;
        MG_NCCL(A.GroupStart());
        MG_NCCL(A.AllGather(skey + (size_t)me * MG_SAMPLES, skey, MG_SAMPLES, ncclUint64, c, s));
        MG_NCCL(A.AllGather(spos + (size_t)me * MG_SAMPLES, spos, MG_SAMPLES, ncclUint64, c, s));
        MG_NCCL(A.AllGather(sw + (size_t)me * MG_SAMPLES, sw, MG_SAMPLES, ncclUint64, c, s));
        MG_NCCL(A.GroupEnd());
        // samples are gathered rank-major, positions ascending: a stable sort by
        // key leaves them in extended-key order
        st = rs_sort_impl(LCPP_U64, LCPP_U32, 0, skey, T + L.skey_sorted, sidx, T + L.order, (uint64_t)S, 0, 0,
                          T + L.sort, sort_bytes, stream, nullptr);
        if (st != LCPP_OK) return st;
        mg_pick_splitters_kernel<<<1, 1024, 0, s>>>((const uint64_t*)(T + L.skey_sorted), (const uint32_t*)(T + L.order),
                                                    spos, sw, S, G, split);
        count_launch();
        if ((st = check_launch()) != LCPP_OK) return st;
    }
    // 2. bucket of every item, then one stable pass that groups the shard by bucket
    char* pk = T + L.part_k;
    char* pv = vs ? T + L.part_v : nullptr;
    {
        ProfScope ps("mg_partition", s);
        if (n_local) {
            auto go = [&](auto kb) -> lcpp_status {
                using KB = decltype(kb);
                const KB* k = (const KB*)keys_in;
                switch (kind) {
                    case 0: mg_bucket_kernel<KB, 0><<<grid, 1024, 0, s>>>(k, n_local, me, split, G - 1, digits, mm); break;
                    case 1: mg_bucket_kernel<KB, 1><<<grid, 1024, 0, s>>>(k, n_local, me, split, G - 1, digits, mm); break;
                    default: mg_bucket_kernel<KB, 2><<<grid, 1024, 0, s>>>(k, n_local, me, split, G - 1, digits, mm); break;
                }
                count_launch();
                return check_launch();
            };
            st = ks == 4 ? go((uint32_t)0) : go((uint64_t)0);
            if (st != LCPP_OK) return st;
            st = rs_sort_impl(unsigned_view(ks), value_dtype, 0, keys_in, pk, values_in, pv, n_local, 0, 8,
                              T + L.sort, sort_bytes, stream, digits);
            if (st != LCPP_OK) return st;
        } else {
            MG_CUDA(cudaMemsetAsync(T + L.sort, 0, 256 * sizeof(uint32_t), s));
        }
    }
    // 3. all-gathered bucket starts -> exchange sizes -> host
    std::vector<uint64_t> plan((size_t)3 * G + 2);
    std::vector<MgIpcRec> recs((size_t)G);
    uint64_t* rows = (uint64_t*)(T + L.rows);
    uint64_t* ipc = (uint64_t*)(T + L.ipc);
    {
        MgIpcRec mine{};
        char* base = nullptr;
        if (mg_ipc_enabled() && alloc_base(pk, &base) && cudaIpcGetMemHandle(&mine.h, base) == cudaSuccess) {
            mine.off_k = (uint64_t)(pk - base);
            mine.off_v = pv ? (uint64_t)(pv - base) : 0;
            mine.ok = 1;
        }
        cudaGetLastError();  // an allocation that cannot be exported only selects the NCCL path
        uint64_t wire[MG_IPC_REC_U64] = {};
        memcpy(wire, &mine, sizeof(mine));
        MG_CUDA(cudaMemcpyAsync(ipc + (size_t)me * MG_IPC_REC_U64, wire, sizeof(wire), cudaMemcpyHostToDevice, s));
        ProfScope ps("mg_plan", s);
        // the partition pass leaves its 256 digit starts at the start of its temp (bins of pass 0)
        mg_pack_starts_kernel<<<1, 256, 0, s>>>((const uint32_t*)(T + L.sort), n_local, rows + (size_t)me * 257);
        count_launch();
        if ((st = check_launch()) != LCPP_OK) return st;
        MG_NCCL(A.GroupStart());
        MG_NCCL(A.AllGather(rows + (size_t)me * 257, rows, 257, ncclUint64, c, s));
        MG_NCCL(A.AllReduce(mm, mm + 2, 2, ncclUint64, ncclMin, c, s));
        MG_NCCL(A.AllGather(ipc + (size_t)me * MG_IPC_REC_U64, ipc, MG_IPC_REC_U64, ncclUint64, c, s));
        MG_NCCL(A.GroupEnd());
        mg_range_bits_kernel<<<1, 1, 0, s>>>(mm + 2, info);
        count_launch();
        mg_plan_kernel<<<1, 256, 0, s>>>(rows, G, me, info, (uint64_t*)(T + L.plan));
        count_launch();
        if ((st = check_launch()) != LCPP_OK) return st;
        MG_CUDA(cudaMemcpyAsync(plan.data(), T + L.plan, plan.size() * sizeof(uint64_t), cudaMemcpyDeviceToHost, s));
        std::vector<uint64_t> wires((size_t)G * MG_IPC_REC_U64);
        MG_CUDA(cudaMemcpyAsync(wires.data(), ipc, wires.size() * sizeof(uint64_t), cudaMemcpyDeviceToHost, s));
        MG_CUDA(cudaStreamSynchronize(s));
        for (int p = 0; p < G; ++p) memcpy(&recs[p], wires.data() + (size_t)p * MG_IPC_REC_U64, sizeof(MgIpcRec));
    }
    const uint64_t* so = plan.data();
    const uint64_t* rc = plan.data() + G + 1;
    const int end_bit = (int)plan[2 * G + 1];
    std::vector<uint64_t> ro(G + 1, 0);
    for (int p = 0; p < G; ++p) ro[p + 1] = ro[p] + rc[p];
    const uint64_t n_recv = ro[G];
    if (n_recv > capacity) return LCPP_ERR_CAPACITY;
    // 4. exchange (runs land in source-rank order)
    char* rk = T + L.recv_k;
    char* rv = vs ? T + L.recv_v : nullptr;
    unsigned long long* agree = mm + 4;  // the path choice and the closing barrier
    {
        ProfScope ps("mg_exchange", s);
        // IPC pull when every rank exported its shard and mapped the peers it
        // pulls from (decided together, so that no rank waits on a transfer its
        // peer does not issue); NCCL send/recv otherwise.
        bool use_ipc = true;
        for (int p = 0; p < G; ++p) use_ipc = use_ipc && recs[p].ok == 1;
        std::vector<char*> peer((size_t)G, nullptr);
        if (use_ipc) {
            unsigned long long mapped = 1;
            for (int p = 0; p < G; ++p)
                if (p != me && rc[p] && !(peer[p] = open_peer(comm, p, recs[p].h))) mapped = 0;
            MG_CUDA(cudaMemcpyAsync(agree, &mapped, sizeof(mapped), cudaMemcpyHostToDevice, s));
            MG_NCCL(A.AllReduce(agree, agree, 1, ncclUint64, ncclMin, c, s));
            MG_CUDA(cudaMemcpyAsync(&mapped, agree, sizeof(mapped), cudaMemcpyDeviceToHost, s));
            MG_CUDA(cudaStreamSynchronize(s));
            use_ipc = mapped == 1;
        }
        if (use_ipc) {
            // K side streams per source (this rank included), forked from and
            // joined to s: each carries 1/K of the slice, so that several copy
            // engines pull from every source at once.
            const int K = mg_pull_streams();
            std::vector<cudaEvent_t> ev((size_t)G * K + 1, nullptr);
            for (auto& e : ev) MG_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
            MG_CUDA(cudaEventRecord(ev[(size_t)G * K], s));
            for (int p = 0; p < G; ++p) {
                if (!rc[p]) continue;
                const char* src_k = p == me ? pk + so[me] * ks : peer[p] + recs[p].off_k + plan[2 * G + 2 + p] * ks;
                const char* src_v = !vs ? nullptr
                                  : p == me ? pv + so[me] * vs
                                            : peer[p] + recs[p].off_v + plan[2 * G + 2 + p] * vs;
                const uint64_t per = ceil_div(rc[p], (uint64_t)K);
                for (int j = 0; j < K; ++j) {
                    const uint64_t b0 = (uint64_t)j * per;
                    if (b0 >= rc[p]) break;
                    const uint64_t cnt = std::min<uint64_t>(per, rc[p] - b0);
                    cudaStream_t sp = side_stream(1 + p * K + j);
                    if (!sp) return LCPP_ERR_CUDA;
                    MG_CUDA(cudaStreamWaitEvent(sp, ev[(size_t)G * K], 0));
                    MG_CUDA(cudaMemcpyAsync(rk + (ro[p] + b0) * ks, src_k + b0 * ks, cnt * ks, cudaMemcpyDeviceToDevice, sp));
                    if (vs)
                        MG_CUDA(cudaMemcpyAsync(rv + (ro[p] + b0) * vs, src_v + b0 * vs, cnt * vs,
                                                cudaMemcpyDeviceToDevice, sp));
                    MG_CUDA(cudaEventRecord(ev[(size_t)p * K + j], sp));
                    MG_CUDA(cudaStreamWaitEvent(s, ev[(size_t)p * K + j], 0));
                }
            }
            for (auto& e : ev) cudaEventDestroy(e);
            // every peer has finished reading this rank's shard before it is reused
            MG_NCCL(A.AllReduce(agree, agree, 1, ncclUint64, ncclMin, c, s));
        } else {
            // this rank's own slice moves on a side stream, alongside the NCCL transfers
            const uint64_t self = so[me + 1] - so[me];
            cudaStream_t side = self ? side_stream() : nullptr;
            cudaEvent_t ev_in = nullptr, ev_out = nullptr;
            if (side) {
                MG_CUDA(cudaEventCreateWithFlags(&ev_in, cudaEventDisableTiming));
                MG_CUDA(cudaEventCreateWithFlags(&ev_out, cudaEventDisableTiming));
                MG_CUDA(cudaEventRecord(ev_in, s));
                MG_CUDA(cudaStreamWaitEvent(side, ev_in, 0));
            }
            if (self) {
                cudaStream_t cs = side ? side : s;
                MG_CUDA(cudaMemcpyAsync(rk + ro[me] * ks, pk + so[me] * ks, self * ks, cudaMemcpyDeviceToDevice, cs));
                if (vs) MG_CUDA(cudaMemcpyAsync(rv + ro[me] * vs, pv + so[me] * vs, self * vs, cudaMemcpyDeviceToDevice, cs));
            }
            if (side) MG_CUDA(cudaEventRecord(ev_out, side));
            MG_NCCL(A.GroupStart());
            for (int p = 0; p < G; ++p) {
                if (p == me) continue;
                const uint64_t sc = so[p + 1] - so[p];
                if (sc) {
                    MG_NCCL(A.Send(pk + so[p] * ks, sc * ks, ncclUint8, p, c, s));
                    if (vs) MG_NCCL(A.Send(pv + so[p] * vs, sc * vs, ncclUint8, p, c, s));
                }
                if (rc[p]) {
                    MG_NCCL(A.Recv(rk + ro[p] * ks, rc[p] * ks, ncclUint8, p, c, s));
                    if (vs) MG_NCCL(A.Recv(rv + ro[p] * vs, rc[p] * vs, ncclUint8, p, c, s));
                }
            }
            MG_NCCL(A.GroupEnd());
            if (side) {
                MG_CUDA(cudaStreamWaitEvent(s, ev_out, 0));
                cudaEventDestroy(ev_in);
                cudaEventDestroy(ev_out);
            }
        }
    }
    // 5. local sort of the bits that still differ
    *n_out = n_recv;
    if (n_recv == 0) return LCPP_OK;
    ProfScope ps("mg_local_sort", s);
    if (end_bit <= 0) {  // every key equal: arrival order is the stable order
        MG_CUDA(cudaMemcpyAsync(keys_out, rk, n_recv * ks, cudaMemcpyDeviceToDevice, s));
        if (vs) MG_CUDA(cudaMemcpyAsync(values_out, rv, n_recv * vs, cudaMemcpyDeviceToDevice, s));
        return LCPP_OK;
    }
    return rs_sort_impl(key_dtype, value_dtype, 0, rk, keys_out, rv, values_out, n_recv, 0, end_bit, T + L.sort,
                        sort_bytes, stream, nullptr);
}
