// Single-pass prefix sum (decoupled look-back): onHost::inclusiveScan / exclusiveScan / *InPlace.
//
// Replaces the three-level Scan_ScanBlocksKernel + recursion + Scan_AddIncrementsKernel scheme of
// include/alpaka/onHost/algo/internal/scan.hpp:114-472 (about 4N-5N elements of traffic and 2*levels launches) with
// one launch that reads every element once and writes it once (2N).
//
// Tile = 256 threads x 4 rounds x one 16-byte pack per thread (4096 x 4-byte or 2048 x 8-byte elements). Warp w of a
// tile owns a contiguous segment; in round r lane l holds the pack at segment offset (r*32 + l), so each load and
// store instruction of a warp covers 512 contiguous bytes. Scans run in registers: within the pack, across lanes
// (shfl_up), across rounds (running segment total), across the 8 warps (shared memory), then across tiles.
//
// Cross-tile protocol: a tile takes its index from an atomic ticket (so every tile it waits on belongs to a block that
// is already running), publishes its aggregate (flag A), looks back over windows of 32 predecessors with one lane per
// predecessor until it meets an inclusive prefix (flag P), then publishes its own inclusive prefix. Status words
// carry the call's epoch, so the scratch needs no clearing between calls on a stream: the block that takes the last
// ticket resets the ticket and advances the epoch. 4-byte types pack flag, epoch and value in one 64-bit word
// (relaxed 64-bit loads/stores are single-copy atomic); 8-byte types keep values in separate aggregate/prefix slots
// published with a release store of the flag word and read after an acquire load of it.
// Every spin is bounded by %globaltimer; on timeout the tile raises the device error word and an abort mark that
// stops the other tiles' waits of the same call.
#include <type_traits>

#include "common.cuh"

namespace a3b
{
    namespace
    {
        constexpr int kBlock = 256;
        constexpr int kWarps = kBlock / 32;
        constexpr int kRounds = 4;
        constexpr unsigned kEpochMask = 0x3FFFFFFFu;
        constexpr unsigned kFlagA = 1u, kFlagP = 2u;

        struct ScanHeader
        {
            unsigned ticket;
            unsigned epoch;
            unsigned abortEpoch;
            unsigned pad[13];
        };
        static_assert(sizeof(ScanHeader) == 64, "header size");

        template<typename T>
        struct Traits
        {
            static constexpr int W = 16 / static_cast<int>(sizeof(T));
            static constexpr int ITEMS = W * kRounds;
            static constexpr int TILE = kBlock * ITEMS;
            using Bits = std::conditional_t<sizeof(T) == 4, uint32_t, uint64_t>;
        };

        template<typename T>
        __device__ __forceinline__ T add(T a, T b)
        {
            if constexpr(std::is_same_v<T, float>)
                return __fadd_rn(a, b);
            else if constexpr(std::is_same_v<T, double>)
                return __dadd_rn(a, b);
            else
                return static_cast<T>(static_cast<std::make_unsigned_t<T>>(a) + static_cast<std::make_unsigned_t<T>>(b));
        }

        template<typename T>
        __device__ __forceinline__ typename Traits<T>::Bits toBits(T v)
        {
            typename Traits<T>::Bits b;
            memcpy(&b, &v, sizeof(T));
            return b;
        }

        template<typename T>
        __device__ __forceinline__ T fromBits(typename Traits<T>::Bits b)
        {
            T v;
            memcpy(&v, &b, sizeof(T));
            return v;
        }

        __host__ __device__ inline size_t align256(size_t x)
        {
            return (x + 255u) & ~size_t{255u};
        }

        // scratch layout: header | 4-byte T: u64 status[tiles] | 8-byte T: u32 flags[tiles], u64 agg[tiles], u64 pre[tiles]
        template<typename T>
        __host__ __device__ inline size_t scratchBytes(uint64_t tiles)
        {
            if constexpr(sizeof(T) == 4)
                return sizeof(ScanHeader) + align256(tiles * 8u);
            else
                return sizeof(ScanHeader) + align256(tiles * 4u) + 2u * align256(tiles * 8u);
        }

        template<typename T>
        struct StatusView
        {
            uint64_t* word;   // 4-byte T
            unsigned* flags;  // 8-byte T
            uint64_t* agg;
            uint64_t* pre;

            __device__ static StatusView make(ScanHeader* hdr, uint64_t tiles)
            {
                StatusView v{};
                char* base = reinterpret_cast<char*>(hdr + 1);
                if constexpr(sizeof(T) == 4)
                    v.word = reinterpret_cast<uint64_t*>(base);
                else
                {
                    v.flags = reinterpret_cast<unsigned*>(base);
                    v.agg = reinterpret_cast<uint64_t*>(base + align256(tiles * 4u));
                    v.pre = reinterpret_cast<uint64_t*>(base + align256(tiles * 4u) + align256(tiles * 8u));
                }
                return v;
            }

            __device__ void publish(uint64_t tile, unsigned flag, unsigned epoch, T value) const
            {
                if constexpr(sizeof(T) == 4)
                {
                    uint64_t const w = (static_cast<uint64_t>(flag) << 62) | (static_cast<uint64_t>(epoch) << 32)
                                       | static_cast<uint64_t>(toBits(value));
                    stRelaxedU64(word + tile, w);
                }
                else
                {
                    stRelaxedU64((flag == kFlagA ? agg : pre) + tile, toBits(value));
                    stReleaseU32(flags + tile, (flag << 30) | epoch);
                }
            }

            // returns the flag seen for `tile` in this epoch (0 = not yet) and its value
            __device__ unsigned peek(uint64_t tile, unsigned epoch, T& value) const
            {
                if constexpr(sizeof(T) == 4)
                {
                    uint64_t const w = ldRelaxedU64(word + tile);
                    unsigned const e = static_cast<unsigned>(w >> 32) & kEpochMask;
                    if(e != epoch)
                        return 0u;
                    value = fromBits<T>(static_cast<uint32_t>(w));
                    return static_cast<unsigned>(w >> 62);
                }
                else
                {
                    unsigned const f = ldAcquireU32(flags + tile);
                    if((f & kEpochMask) != epoch)
                        return 0u;
                    unsigned const flag = f >> 30;
                    value = fromBits<T>(ldRelaxedU64((flag == kFlagA ? agg : pre) + tile));
                    return flag;
                }
            }
        };

        template<typename T>
        __device__ __forceinline__ T warpSum(T v)
        {
            // butterfly; every lane ends with the same total
#pragma unroll
            for(int m = 1; m < 32; m <<= 1)
                v = add(v, __shfl_xor_sync(0xffffffffu, v, m));
            return v;
        }

        template<typename T, bool INCL, bool VEC>
        __global__ void __launch_bounds__(kBlock) scanKernel(
            T const* in,
            T* out,
            uint64_t n,
            uint64_t tiles,
            T const* carryIn,
            ScanHeader* hdr,
            unsigned* errWord,
            uint64_t timeoutNs,
            uint64_t stallTile)
        {
            using Tr = Traits<T>;
            constexpr int W = Tr::W;
            __shared__ uint64_t sTile;
            __shared__ unsigned sEpoch;
            __shared__ T sWarpTotal[kWarps];
            __shared__ T sWarpPrefix[kWarps];
            __shared__ T sTilePrefix;

            int const warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

            if(threadIdx.x == 0)
            {
                unsigned const e = ldRelaxedU32(&hdr->epoch);
                __threadfence(); // the epoch read precedes the ticket claim
                unsigned const t = atomicAdd(&hdr->ticket, 1u);
                unsigned cur = (e + 1u) & kEpochMask;
                if(cur == 0u)
                    cur = 1u;
                if(t == tiles - 1u)
                {
                    // every other block has claimed (and so has read the epoch): reset for the next call
                    __threadfence();
                    stRelaxedU32(&hdr->ticket, 0u);
                    stRelaxedU32(&hdr->epoch, cur);
                }
                sTile = t;
                sEpoch = cur;
            }
            __syncthreads();
            uint64_t const tile = sTile;
            unsigned const epoch = sEpoch;
            StatusView<T> const st = StatusView<T>::make(hdr, tiles);

            // ---- load: warp segment of 32*ITEMS elements, round r / lane l -> pack (r*32 + l)
            uint64_t const segBase = tile * Tr::TILE + static_cast<uint64_t>(warp) * (32 * Tr::ITEMS);
            bool const full = (tile + 1u) * Tr::TILE <= n;
            T v[kRounds][W];
            if(VEC && full)
            {
#pragma unroll
                for(int r = 0; r < kRounds; ++r)
                {
                    uint4 raw = __ldcs(reinterpret_cast<uint4 const*>(in + segBase) + (r * 32 + lane));
                    memcpy(&v[r][0], &raw, 16);
                }
            }
            else
            {
#pragma unroll
                for(int r = 0; r < kRounds; ++r)
#pragma unroll
                    for(int k = 0; k < W; ++k)
                    {
                        uint64_t const idx = segBase + static_cast<uint64_t>(r * 32 + lane) * W + k;
                        v[r][k] = idx < n ? in[idx] : T(0);
                    }
            }

            // ---- scan inside the warp segment (values become segment-relative exclusive/inclusive prefixes)
            T run = T(0);
#pragma unroll
            for(int r = 0; r < kRounds; ++r)
            {
                T incl[W];
                incl[0] = v[r][0];
#pragma unroll
                for(int k = 1; k < W; ++k)
                    incl[k] = add(incl[k - 1], v[r][k]);
                T x = incl[W - 1];
#pragma unroll
                for(int d = 1; d < 32; d <<= 1)
                {
                    T const y = __shfl_up_sync(0xffffffffu, x, d);
                    if(lane >= d)
                        x = add(y, x);
                }
                T laneExcl = __shfl_up_sync(0xffffffffu, x, 1);
                if(lane == 0)
                    laneExcl = T(0);
                T const roundTotal = __shfl_sync(0xffffffffu, x, 31);
                T const pre = add(run, laneExcl);
                if constexpr(INCL)
                {
#pragma unroll
                    for(int k = 0; k < W; ++k)
                        v[r][k] = add(pre, incl[k]);
                }
                else
                {
                    v[r][0] = pre;
#pragma unroll
                    for(int k = 1; k < W; ++k)
                        v[r][k] = add(pre, incl[k - 1]);
                }
                run = add(run, roundTotal);
            }
            if(lane == 0)
                sWarpTotal[warp] = run;
            __syncthreads();

            // ---- tile aggregate, warp prefixes, look-back (warp 0)
            if(warp == 0)
            {
                T x = lane < kWarps ? sWarpTotal[lane] : T(0);
#pragma unroll
                for(int d = 1; d < kWarps; d <<= 1)
                {
                    T const y = __shfl_up_sync(0xffffffffu, x, d);
                    if(lane >= d)
                        x = add(y, x);
                }
                T wEx = __shfl_up_sync(0xffffffffu, x, 1);
                if(lane == 0)
                    wEx = T(0);
                if(lane < kWarps)
                    sWarpPrefix[lane] = wEx;
                T const tileAgg = __shfl_sync(0xffffffffu, x, kWarps - 1);
                bool const stalled = (tile == stallTile);

                T prefix = T(0);
                if(tile == 0)
                {
                    if(carryIn)
                        prefix = *carryIn;
                }
                else
                {
                    if(lane == 0 && !stalled)
                        st.publish(tile, kFlagA, epoch, tileAgg);
                    uint64_t const t0 = globalTimerNs();
                    bool gaveUp = false;
                    int64_t pred = static_cast<int64_t>(tile) - 1;
                    T acc = T(0);
                    while(true)
                    {
                        int64_t const j = pred - lane;
                        T val = T(0);
                        unsigned flag = kFlagP; // lanes before tile 0 count as an (empty) inclusive prefix
                        int spins = 0;
                        while(true)
                        {
                            if(j >= 0)
                                flag = st.peek(static_cast<uint64_t>(j), epoch, val);
                            if(__all_sync(0xffffffffu, flag != 0u))
                                break;
                            ++spins;
                            if(spins > 8)
                                __nanosleep(spins > 64 ? 256 : 32);
                            bool timedOut = false;
                            if(lane == 0)
                                timedOut = (globalTimerNs() - t0 > timeoutNs)
                                           || (ldRelaxedU32(&hdr->abortEpoch) == epoch);
                            if(__shfl_sync(0xffffffffu, timedOut, 0))
                            {
                                gaveUp = true;
                                break;
                            }
                        }
                        if(gaveUp)
                            break;
                        unsigned const pmask = __ballot_sync(0xffffffffu, flag == kFlagP);
                        int const stop = __ffs(pmask) - 1; // nearest predecessor holding an inclusive prefix
                        T const mine = (pmask == 0u || lane <= stop) && j >= 0 ? val : T(0);
                        acc = add(warpSum(mine), acc);
                        if(pmask != 0u)
                            break;
                        pred -= 32;
                    }
                    if(gaveUp && lane == 0)
                    {
                        atomicOr(errWord, kErrTimeout);
                        stRelaxedU32(&hdr->abortEpoch, epoch);
                    }
                    prefix = acc;
                }
                if(lane == 0)
                {
                    if(!stalled)
                        st.publish(tile, kFlagP, epoch, add(prefix, tileAgg));
                    sTilePrefix = prefix;
                }
            }
            __syncthreads();

            // ---- add tile and warp offsets, store
            T const off = add(sTilePrefix, sWarpPrefix[warp]);
            if(VEC && full)
            {
#pragma unroll
                for(int r = 0; r < kRounds; ++r)
                {
#pragma unroll
                    for(int k = 0; k < W; ++k)
                        v[r][k] = add(off, v[r][k]);
                    uint4 raw;
                    memcpy(&raw, &v[r][0], 16);
                    __stcs(reinterpret_cast<uint4*>(out + segBase) + (r * 32 + lane), raw);
                }
            }
            else
            {
#pragma unroll
                for(int r = 0; r < kRounds; ++r)
#pragma unroll
                    for(int k = 0; k < W; ++k)
                    {
                        uint64_t const idx = segBase + static_cast<uint64_t>(r * 32 + lane) * W + k;
                        if(idx < n)
                            out[idx] = add(off, v[r][k]);
                    }
            }
        }

        template<typename T>
        uint64_t tilesFor(uint64_t n)
        {
            return (n + Traits<T>::TILE - 1) / Traits<T>::TILE;
        }

        template<typename T>
        int scanT(
            cudaStream_t s,
            int inclusive,
            T const* in,
            T* out,
            uint64_t n,
            T const* carry,
            void* buffer,
            size_t bufBytes,
            uint64_t stallTile)
        {
            if(n == 0)
                return A3B_OK;
            A3B_REQUIRE(in && out, "null input/output");
            DeviceProps const* props = nullptr;
            int rc = currentDevice(&props);
            if(rc)
                return rc;
            uint64_t const tiles = tilesFor<T>(n);
            if(tiles >= 0xFFFFFFFFull)
            {
                setError("scan of %llu elements exceeds the tile index range", static_cast<unsigned long long>(n));
                return A3B_ERR_TOO_LARGE;
            }
            size_t const need = scratchBytes<T>(tiles);
            void* scr = nullptr;
            if(buffer)
            {
                if(bufBytes < need)
                {
                    setError("scan buffer too small: %zu bytes given, %zu needed", bufBytes, need);
                    return A3B_ERR_INVALID;
                }
                A3B_CUDA(cudaMemsetAsync(buffer, 0, need, s));
                scr = buffer;
            }
            else
            {
                rc = streamScratch(s, kScratchScan, need, &scr);
                if(rc)
                    return rc;
            }
            auto* hdr = static_cast<ScanHeader*>(scr);
            bool const vec = aligned16(in) && aligned16(out);
            uint64_t const to = waitTimeoutNs();
            dim3 const grid(static_cast<unsigned>(tiles));
#define A3B_SCAN_LAUNCH(INCL, VEC)                                                                                    \
    scanKernel<T, INCL, VEC><<<grid, kBlock, 0, s>>>(in, out, n, tiles, carry, hdr, props->errWord, to, stallTile)
            if(inclusive)
            {
                if(vec)
                    A3B_SCAN_LAUNCH(true, true);
                else
                    A3B_SCAN_LAUNCH(true, false);
            }
            else
            {
                if(vec)
                    A3B_SCAN_LAUNCH(false, true);
                else
                    A3B_SCAN_LAUNCH(false, false);
            }
#undef A3B_SCAN_LAUNCH
            A3B_CHECK_LAUNCH("scan launch");
            return A3B_OK;
        }

        int scanEntry(
            a3b_stream_t stream,
            int dtype,
            int inclusive,
            void const* in,
            void* out,
            uint64_t n,
            void const* carry,
            void* buffer,
            size_t bufBytes,
            uint64_t stallTile)
        {
            auto s = static_cast<cudaStream_t>(stream);
            switch(dtype)
            {
            case A3B_I32:
                return scanT<int32_t>(s, inclusive, (int32_t const*) in, (int32_t*) out, n, (int32_t const*) carry, buffer, bufBytes, stallTile);
            case A3B_U32:
                return scanT<uint32_t>(s, inclusive, (uint32_t const*) in, (uint32_t*) out, n, (uint32_t const*) carry, buffer, bufBytes, stallTile);
            case A3B_I64:
                return scanT<int64_t>(s, inclusive, (int64_t const*) in, (int64_t*) out, n, (int64_t const*) carry, buffer, bufBytes, stallTile);
            case A3B_U64:
                return scanT<uint64_t>(s, inclusive, (uint64_t const*) in, (uint64_t*) out, n, (uint64_t const*) carry, buffer, bufBytes, stallTile);
            case A3B_F32:
                return scanT<float>(s, inclusive, (float const*) in, (float*) out, n, (float const*) carry, buffer, bufBytes, stallTile);
            case A3B_F64:
                return scanT<double>(s, inclusive, (double const*) in, (double*) out, n, (double const*) carry, buffer, bufBytes, stallTile);
            default:
                setError("unknown dtype %d", dtype);
                return A3B_ERR_INVALID;
            }
        }
    } // namespace
} // namespace a3b

using namespace a3b;

extern "C"
{
    size_t a3b_scan_buffer_size(int dtype, uint64_t n)
    {
        int const es = dtypeSize(dtype);
        if(es == 0)
            return 0;
        uint64_t const tile = static_cast<uint64_t>(kBlock) * kRounds * (16 / es);
        uint64_t const tiles = (n + tile - 1) / tile;
        return es == 4 ? scratchBytes<uint32_t>(tiles) : scratchBytes<uint64_t>(tiles);
    }

    int a3b_scan(a3b_stream_t stream, int dtype, int inclusive, void const* in, void* out, uint64_t n,
                 void const* carry_in, void* buffer, size_t buffer_bytes)
    {
        return scanEntry(stream, dtype, inclusive, in, out, n, carry_in, buffer, buffer_bytes, ~0ull);
    }

    int a3b_scan_debug_stall(a3b_stream_t stream, int dtype, void const* in, void* out, uint64_t n, uint64_t stall_tile)
    {
        return scanEntry(stream, dtype, 0, in, out, n, nullptr, nullptr, 0, stall_tile);
    }
}
