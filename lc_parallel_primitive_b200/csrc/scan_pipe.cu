// Pipelined persistent DeviceScan kernel for 16-byte-aligned inputs.
//
// Same single-pass decoupled look-back as scan_kernel, reorganised so that
// HBM never waits on the look-back:
//  * persistent CTAs (2 per SM, 512 threads) stream 8192-item tiles through
//    three 32 KiB shared-memory stages filled by TMA bulk copies
//    (cp.async.bulk, this GPU's memory only, no multicast);
//  * a CTA publishes the aggregate of its NEXT tile as soon as that tile's
//    bulk load lands, before it resolves the look-back of its current tile;
//    the next tile's warp sums and the current tile's warp totals cross one
//    CTA barrier together (three barriers per tile in all).
//    Partial descriptors therefore appear one tile ahead of the scan
//    frontier, so a look-back never waits for another CTA's data to arrive
//    (with one tile per CTA and no early publish, every look-back waits for
//    the loads of all tiles in flight, which locks the CTAs into step);
//  * results are written back into the stage and leave by bulk store.
//
// Forward progress: each CTA takes tile tickets in ascending order and
// publishes a tile's aggregate depending only on that tile's own load; a
// look-back waits only for aggregates of smaller tiles, which their CTAs
// publish without waiting on anything else.  All waits are bounded.
#include "bulk.cuh"
#include "common.cuh"

namespace lcpp {

constexpr int SP_THREADS = 512;
constexpr int SP_WARPS = SP_THREADS / 32;
constexpr int SP_VECS = 4;
constexpr int SP_STAGE_BYTES = SP_THREADS * SP_VECS * 16;  // 32 KiB: 8192 4-byte or 4096 8-byte items
constexpr int SP_CTAS_PER_SM = 2;
constexpr int SP_STAGES = 3;
constexpr size_t SP_SMEM = SP_STAGES * (size_t)SP_STAGE_BYTES;
static_assert(SP_STAGE_BYTES == SCAN_DESC_TILE_BYTES, "descriptor arrays are sized for SCAN_DESC_TILE_BYTES tiles");

template <typename Op, typename T, bool INCLUSIVE>
__global__ void __launch_bounds__(SP_THREADS, SP_CTAS_PER_SM)
scan_pipe_kernel(const T* in, T* out, uint64_t n, uint64_t num_tiles, const T* carry_in, T init,
                 unsigned int* ticket, ScanDesc<T> desc) {
    constexpr int V = scan_vec_items<T>();
    constexpr int SP_WARP_ITEMS = 32 * SP_VECS * V;
    constexpr int SP_TILE = SP_THREADS * SP_VECS * V;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t s_bar[SP_STAGES];
    __shared__ unsigned int s_tile[SP_STAGES];
    __shared__ T s_agg[SP_STAGES];      // aggregate of the tile held by each stage
    __shared__ T s_wnext[SP_WARPS];     // warp sums of the next tile
    __shared__ T s_wcur[SP_WARPS];      // warp totals of the current tile
    __shared__ T s_wex[SP_WARPS];       // prefix of each warp's slice of the current tile

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint64_t full_tiles = n / SP_TILE;
    const uint32_t limit = g_spin_limit;
    const T c0 = carry_in ? *carry_in : init;
    const uint32_t woff = (uint32_t)warp * SP_WARP_ITEMS + lane * V;
    uint32_t phase_bits = 0;  // bit st: parity of stage st's next phase

    auto issue = [&](unsigned int t, int st) {  // thread 0
        if (t < full_tiles) {
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&s_bar[st], SP_STAGE_BYTES);
            bulk_load(smem + st * SP_STAGE_BYTES, in + (uint64_t)t * SP_TILE, SP_STAGE_BYTES, &s_bar[st]);
        }
    };
    // Make stage st hold tile t for this thread's slice (the ragged last tile
    // is copied slice by slice with identity fill, so no CTA barrier is needed).
    auto wait_stage = [&](uint64_t t, int st) -> T* {
        T* buf = reinterpret_cast<T*>(smem + st * SP_STAGE_BYTES);
        if (t < full_tiles) {
            if (!mbar_wait(&s_bar[st], (phase_bits >> st) & 1u, limit)) set_error(LCPP_ERR_LOOKBACK_TIMEOUT);
            phase_bits ^= 1u << st;
        } else {
#pragma unroll
            for (int j = 0; j < SP_VECS; ++j)
#pragma unroll
                for (int k = 0; k < V; ++k) {
                    const uint32_t i = woff + j * 32 * V + k;
                    const uint64_t g = t * SP_TILE + i;
                    buf[i] = g < n ? in[g] : Op::template identity<T>();
                }
        }
        return buf;
    };
    auto slice_sum = [&](const T* buf) -> T {  // warp-reduced sum of the warp's slice
        T r = Op::template identity<T>();
#pragma unroll
        for (int j = 0; j < SP_VECS; ++j) {
            const uint4 q = *reinterpret_cast<const uint4*>(buf + woff + j * 32 * V);
            const T* e = reinterpret_cast<const T*>(&q);
#pragma unroll
            for (int k = 0; k < V; ++k) r = Op::template apply<T>(r, e[k]);
        }
        return warp_reduce<Op>(r);
    };
    auto tile_sum = [&](const T* ws) -> T {  // warp 0: sum of the SP_WARPS warp values
        T a = lane < SP_WARPS ? ws[lane] : Op::template identity<T>();
        return warp_reduce<Op>(a);
    };

    if (tid == 0) {
        for (int i = 0; i < SP_STAGES; ++i) mbar_init(&s_bar[i], 1);
        fence_mbar_init();
        for (int i = 0; i < SP_STAGES; ++i) {
            const unsigned int t = atomicAdd(ticket, 1u);
            s_tile[i] = t;
            issue(t, i);
        }
    }
    __syncthreads();

    uint64_t c = s_tile[0];
    int st = 0;
    if (c < num_tiles) {  // aggregate of the first tile
        const T r = slice_sum(wait_stage(c, 0));
        if (lane == 0) s_wnext[warp] = r;
        __syncthreads();
        if (warp == 0) {
            const T a = tile_sum(s_wnext);
            if (lane == 0) {
                s_agg[0] = a;
                if (c == 0) desc.inclusive(0, Op::template apply<T>(c0, a));
                else desc.partial((int64_t)c, a);
            }
        }
        __syncthreads();
    }
    while (c < num_tiles) {
        const int nst = st + 1 == SP_STAGES ? 0 : st + 1;
        const uint64_t nt = s_tile[nst];
        T* buf = reinterpret_cast<T*>(smem + st * SP_STAGE_BYTES);
        // ---- local scan of the current tile; warp sums of the next one ---------
        T x[SP_VECS][V];
#pragma unroll
        for (int j = 0; j < SP_VECS; ++j) {
            const uint4 q = *reinterpret_cast<const uint4*>(buf + woff + j * 32 * V);
            const T* e = reinterpret_cast<const T*>(&q);
#pragma unroll
            for (int k = 0; k < V; ++k) x[j][k] = e[k];
        }
        T pre[SP_VECS];
        T carry = Op::template identity<T>();
#pragma unroll
        for (int j = 0; j < SP_VECS; ++j) {
#pragma unroll
            for (int k = 1; k < V; ++k) x[j][k] = Op::template apply<T>(x[j][k - 1], x[j][k]);
            T incl = x[j][V - 1];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const T y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl = Op::template apply<T>(y, incl);
            }
            T excl = __shfl_up_sync(0xffffffffu, incl, 1);
            if (lane == 0) excl = Op::template identity<T>();
            pre[j] = Op::template apply<T>(carry, excl);
            carry = Op::template apply<T>(carry, __shfl_sync(0xffffffffu, incl, 31));
        }
        if (lane == 0) s_wcur[warp] = carry;
        if (nt < num_tiles) {
            const T r = slice_sum(wait_stage(nt, nst));
            if (lane == 0) s_wnext[warp] = r;
        }
        __syncthreads();
        // ---- warp 0: publish the next tile's aggregate, then resolve this one ---
        if (warp == 0) {
            if (nt < num_tiles) {
                const T a = tile_sum(s_wnext);
                if (lane == 0) {
                    s_agg[nst] = a;
                    desc.partial((int64_t)nt, a);  // nt > c >= 0
                }
            }
            T incl = lane < SP_WARPS ? s_wcur[lane] : Op::template identity<T>();
#pragma unroll
            for (int o = 1; o < SP_WARPS; o <<= 1) {
                const T y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl = Op::template apply<T>(y, incl);
            }
            T wex = __shfl_up_sync(0xffffffffu, incl, 1);
            if (lane == 0) wex = Op::template identity<T>();
            T excl = c0;
            if (c != 0) {
                excl = lookback_warp<Op, T>(desc, (int64_t)c);
                if (lane == 0) desc.inclusive((int64_t)c, Op::template apply<T>(excl, s_agg[st]));
            }
            if (lane < SP_WARPS) s_wex[lane] = Op::template apply<T>(excl, wex);
        }
        __syncthreads();
        // ---- results into the stage (bulk store) or, for the ragged tile, out ---
        const T wbase = s_wex[warp];
        const bool full = c < full_tiles;
#pragma unroll
        for (int j = 0; j < SP_VECS; ++j) {
            const T b = Op::template apply<T>(wbase, pre[j]);
            T r[V];
            if (INCLUSIVE) {
#pragma unroll
                for (int k = 0; k < V; ++k) r[k] = Op::template apply<T>(b, x[j][k]);
            } else {
                r[0] = b;
#pragma unroll
                for (int k = 1; k < V; ++k) r[k] = Op::template apply<T>(b, x[j][k - 1]);
            }
            if (full) {
                *reinterpret_cast<uint4*>(buf + woff + j * 32 * V) = *reinterpret_cast<const uint4*>(r);
            } else {
#pragma unroll
                for (int k = 0; k < V; ++k) {
                    const uint64_t g = c * SP_TILE + woff + j * 32 * V + k;
                    if (g < n) out[g] = r[k];
                }
            }
        }
        if (full) fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            if (full) {
                bulk_store(out + c * SP_TILE, buf, SP_STAGE_BYTES);
                bulk_commit();
            }
            const unsigned int nnt = atomicAdd(ticket, 1u);
            s_tile[st] = nnt;
            bulk_wait_read_all();  // this stage's bulk store has read it
            issue(nnt, st);
        }
        c = nt;
        st = nst;
    }
    if (tid == 0) bulk_wait_all();
}

template <typename Op, typename T>
static lcpp_status scan_pipe_launch(bool inclusive, const T* in, T* out, uint64_t n, const T* carry_in, T init,
                                    unsigned int* ticket, void* desc, cudaStream_t s) {
    constexpr uint64_t SP_TILE = SP_STAGE_BYTES / sizeof(T);
    const uint64_t tiles = ceil_div(n, SP_TILE);
    const DeviceInfo di = device_info();
    uint64_t grid = (uint64_t)di.sms * SP_CTAS_PER_SM;
    if (grid > ceil_div(tiles, 2)) grid = ceil_div(tiles, 2);
    auto k = inclusive ? scan_pipe_kernel<Op, T, true> : scan_pipe_kernel<Op, T, false>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SP_SMEM) != cudaSuccess)
        return LCPP_ERR_CUDA;
    k<<<(unsigned)grid, SP_THREADS, SP_SMEM, s>>>(in, out, n, tiles, carry_in, init, ticket,
                                                   ScanDesc<T>::carve(desc, tiles));
    count_launch();
    return check_launch();
}

}  // namespace lcpp
