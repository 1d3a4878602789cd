// Single-pass prefix sum on a persistent, software-pipelined grid: onHost::inclusiveScan / exclusiveScan / *InPlace.
//
// Replaces the three-level Scan_ScanBlocksKernel + recursion + Scan_AddIncrementsKernel scheme of
// include/alpaka/onHost/algo/internal/scan.hpp:114-472 (about 4N-5N elements of traffic and 2*levels launches) with
// one launch that reads every element from HBM once and writes it once (2N).
//
// The array is cut into 36 KB tiles. The grid has G blocks (one per SM), all resident at once (cooperative launch),
// and block b walks the tiles b, b + G, b + 2G, ... in rounds. In round i block b
//   * reduces tile (i + L) * G + b, which a TMA bulk copy issued two rounds earlier has brought from HBM into one of
//     three "ahead" shared-memory slots, and publishes the tile's aggregate (one tagged status word per 32 value bits);
//   * scans its own tile i * G + b, which a TMA bulk copy issued one round earlier has brought into one of three "own"
//     slots. The tile was read from HBM L rounds ago by the reduction above, so this second read is served from L2
//     (L * G tiles, ~11 MB, stay well inside the 126 MB L2). The scanned tile goes back into its slot and leaves with
//     one TMA bulk store, so HBM sees one read and one write per element;
//   * takes its tile's exclusive prefix as its previous tile's prefix plus the aggregates of the G tiles from its
//     previous tile up to this one (round 0: the carry plus the aggregates of tiles 0 .. b-1). Those aggregates were
//     published L rounds earlier, so the status words loaded at the top of the round are valid when they are used;
//     no block waits for another block's scan. The sums run in a fixed order, so floating-point results do not
//     depend on timing.
// Round i of block b only waits for aggregates that the other blocks publish in rounds i - L and earlier, so with all
// blocks resident every wait ends. The reduction of a tile and its scan happen in the same block, L rounds apart, and
// its store after both: an in-place scan overwrites a tile only after its own block has read it twice.
//
// Inside a tile each thread owns 9 consecutive 16-byte packs (an odd count, so the threads of a quarter-warp read and
// write 16-byte words in 8 different bank groups): a serial scan over its elements, a warp scan of the thread
// totals, a block scan of the warp totals. Measured on B200 (exclusive int32 2^30 / inclusive uint64 2^28): 256
// threads x 9 packs with 3 + 3 slots and L = 2 reach 6.86 / 6.60 TB/s; 7 packs 5.85 / 5.44, 11 packs (2 ahead slots)
// 6.46 / 6.34, a striped layout (one warp scan per 16-byte pack) 5.68 / 4.48, L = 1 4.17 / 3.70.
//
// Status words carry an epoch handed out by the host per call on the stream's cached scratch (a caller buffer is
// cleared and uses epoch 1), so the scratch needs no clearing between calls: a word is flag (2 bits) | epoch (30 bits)
// | 32 value bits, and an 8-byte aggregate's two words are accepted only when both carry the same epoch. Every wait is
// bounded by %globaltimer; on timeout the block raises the device error word and an abort mark that ends the other
// blocks' waits of the same call. Tiles that are not whole, or arrays not 16-byte aligned, move through the slots with
// coalesced per-element copies instead of TMA.
#include <type_traits>

#include "common.cuh"

namespace a3b
{
    namespace
    {
        constexpr int kThreads = 256;
        constexpr int kWarps = kThreads / 32;
        constexpr int kPacks = 9;                            // consecutive 16-byte packs per thread (odd)
        constexpr int kTileBytes = kThreads * kPacks * 16;   // 36 KB
        constexpr int kAheadSlots = 3;                       // tiles coming from HBM for their aggregate
        constexpr int kOwnSlots = 3;                         // tiles coming from L2, scanned, stored to HBM
        constexpr int kOwnAhead = kOwnSlots - 2;             // rounds between an own copy's issue and its use
        constexpr int kSmemBytes = (kAheadSlots + kOwnSlots) * kTileBytes;
        constexpr int kLagRounds = 2;                        // rounds between a tile's reduction and its scan
        static_assert(kPacks % 2 == 1, "odd pack count");
        constexpr int kMaxRange = 4; // aggregates per thread and round: G <= 4 * threads
        constexpr unsigned kEpochMask = 0x3FFFFFFFu;
        constexpr unsigned kFlagA = 1u;

        struct ScanHeader
        {
            unsigned abortEpoch; // epoch of a call whose waits gave up
            unsigned pad[15];
        };
        static_assert(sizeof(ScanHeader) == 64, "header size");

        template<typename T>
        struct Traits
        {
            static constexpr int W = 16 / static_cast<int>(sizeof(T));    // elements per pack
            static constexpr int TILE = kTileBytes / static_cast<int>(sizeof(T)); // elements per tile
            static constexpr int WORDS = static_cast<int>(sizeof(T)) / 4; // 64-bit status words per tile
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

        __host__ __device__ inline size_t align256(size_t x)
        {
            return (x + 255u) & ~size_t{255u};
        }

        // scratch layout: header | u64 aggregate[tiles * WORDS]
        __host__ __device__ inline size_t scratchBytes(uint64_t tiles, int words)
        {
            return sizeof(ScanHeader) + align256(tiles * 8u * static_cast<uint64_t>(words));
        }

        template<typename T>
        struct Aggregates
        {
            uint64_t* word; // aggregate of each tile, written once per call

            __device__ void publish(uint64_t tile, unsigned epoch, T value) const
            {
                constexpr int WD = Traits<T>::WORDS;
                uint32_t parts[WD];
                memcpy(parts, &value, sizeof(T));
                uint64_t const tag = (static_cast<uint64_t>(kFlagA) << 62) | (static_cast<uint64_t>(epoch) << 32);
#pragma unroll
                for(int k = 0; k < WD; ++k)
                    stRelaxedU64(word + tile * WD + k, tag | parts[k]);
            }

            __device__ void load(uint64_t tile, uint64_t (&w)[Traits<T>::WORDS]) const
            {
#pragma unroll
                for(int k = 0; k < Traits<T>::WORDS; ++k)
                    w[k] = ldRelaxedU64(word + tile * Traits<T>::WORDS + k);
            }

            // true when all words carry this epoch's tag; value decoded
            __device__ static bool decode(uint64_t const (&w)[Traits<T>::WORDS], unsigned epoch, T& value)
            {
                constexpr int WD = Traits<T>::WORDS;
                unsigned const tag = static_cast<unsigned>(w[0] >> 32);
                if((tag & kEpochMask) != epoch)
                    return false;
                uint32_t parts[WD];
#pragma unroll
                for(int k = 0; k < WD; ++k)
                {
                    if(static_cast<unsigned>(w[k] >> 32) != tag)
                        return false;
                    parts[k] = static_cast<uint32_t>(w[k]);
                }
                memcpy(&value, parts, sizeof(T));
                return true;
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

        template<typename T>
        struct Shared
        {
            T warpTotal[kWarps];
            T aheadTotal[kWarps];
            T rangeTotal[kWarps];
            alignas(8) unsigned long long bar[kAheadSlots + kOwnSlots];
        };

        __device__ __forceinline__ void raiseAbort(ScanHeader* hdr, unsigned epoch, unsigned* errWord)
        {
            atomicOr(errWord, kErrTimeout);
            stRelaxedU32(&hdr->abortEpoch, epoch);
        }

        // Scan of one warp-segment round in place: p holds one 16-byte pack per lane; `run` is the segment total so
        // far (uniform in the warp) and is advanced by the round total.
        template<typename T, bool INCL>
        __device__ __forceinline__ void scanRound(T (&p)[Traits<T>::W], T& run)
        {
            constexpr int W = Traits<T>::W;
            int const lane = threadIdx.x & 31;
            T incl[W];
            incl[0] = p[0];
#pragma unroll
            for(int k = 1; k < W; ++k)
                incl[k] = add(incl[k - 1], p[k]);
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
                    p[k] = add(pre, incl[k]);
            }
            else
            {
                p[0] = pre;
#pragma unroll
                for(int k = 1; k < W; ++k)
                    p[k] = add(pre, incl[k - 1]);
            }
            run = add(run, roundTotal);
        }

        // ------------------------------------------------------------------------------------------- the kernel
        template<typename T, bool INCL, bool VEC>
        __global__ void __launch_bounds__(kThreads, 1) scanKernel(
            T const* in,
            T* out,
            uint64_t n,
            uint64_t tiles,
            T const* carryIn,
            ScanHeader* hdr,
            unsigned epoch,
            unsigned* errWord,
            uint64_t timeoutNs,
            uint64_t stallTile)
        {
            using Tr = Traits<T>;
            constexpr int W = Tr::W;
            constexpr int WD = Tr::WORDS;
            constexpr int E = kPacks * W; // consecutive elements per thread
            extern __shared__ __align__(128) uint4 smem[]; // kAheadSlots + kOwnSlots tiles
            __shared__ Shared<T> sh;
            int const warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
            int64_t const G = gridDim.x, b = blockIdx.x, L = kLagRounds;
            int64_t const lastRound = (static_cast<int64_t>(tiles) - 1 - b) / G; // grid <= tiles, so b < tiles
            Aggregates<T> const agg{reinterpret_cast<uint64_t*>(hdr + 1)};

            auto full = [&](int64_t tile) { return VEC && static_cast<uint64_t>(tile + 1) * Tr::TILE <= n; };
            auto aheadTile = [&](int64_t i) { return (i + L) * G + b; };
            auto ownTile = [&](int64_t i) { return i * G + b; };
            auto aheadSlot = [&](int64_t i) { return static_cast<int>((i + L) % kAheadSlots); };
            auto aheadParity = [&](int64_t i) { return static_cast<unsigned>(((i + L) / kAheadSlots) & 1); };
            auto ownSlot = [&](int64_t i) { return kAheadSlots + static_cast<int>(i % kOwnSlots); };
            auto ownParity = [&](int64_t i) { return static_cast<unsigned>((i / kOwnSlots) & 1); };
            auto slotPtr = [&](int s) { return smem + static_cast<size_t>(s) * (kTileBytes / 16); };

            // thread 0 issues the copies; only whole, aligned tiles go through TMA
            auto issueAhead = [&](int64_t i) {
                int64_t const a = aheadTile(i);
                if(i >= -L && i <= lastRound - L && full(a))
                {
                    int const s = aheadSlot(i);
                    bulkLoad(smemAddr(slotPtr(s)), in + a * Tr::TILE, kTileBytes, smemAddr(&sh.bar[s]));
                }
            };
            auto issueOwn = [&](int64_t i) {
                int64_t const t = ownTile(i);
                if(i >= 0 && i <= lastRound && full(t))
                {
                    int const s = ownSlot(i);
                    bulkLoad(smemAddr(slotPtr(s)), in + t * Tr::TILE, kTileBytes, smemAddr(&sh.bar[s]));
                }
            };

            if(threadIdx.x == 0 && VEC)
            {
                for(int s = 0; s < kAheadSlots + kOwnSlots; ++s)
                    mbarInit(smemAddr(&sh.bar[s]), 1u);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                for(int k = 0; k < kAheadSlots - 1; ++k)
                    issueAhead(-L + k);
                for(int64_t j = 0; j < kOwnAhead - L; ++j) // own copies due before the first round
                    issueOwn(j);
            }
            __syncthreads();

            T prefix = carryIn ? *carryIn : T(0); // exclusive prefix of the tile before this round's range
            bool abort = false;
            for(int64_t i = -L; i <= lastRound; ++i)
            {
                if(VEC && threadIdx.x == 0)
                {
                    bulkWaitRead<1>(); // the slot refilled now was stored two rounds ago
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    issueAhead(i + kAheadSlots - 1);
                    issueOwn(i + kOwnAhead);
                }
                bool const own = i >= 0;
                int64_t const t = ownTile(i);

                // status words of the aggregates between the previous own tile and this one (round 0: tiles 0..b-1)
                int64_t const lo = i == 0 ? 0 : t - G;
                int const count = own ? static_cast<int>(t - lo) : 0;
                uint64_t raw[kMaxRange][WD];
#pragma unroll
                for(int q = 0; q < kMaxRange; ++q)
                {
                    int const k = q * kThreads + static_cast<int>(threadIdx.x);
                    if(k < count)
                        agg.load(static_cast<uint64_t>(lo + k), raw[q]);
                }

                // (a) aggregate of the ahead tile
                int64_t const a = aheadTile(i);
                bool const doAhead = i <= lastRound - L;
                if(doAhead)
                {
                    T part = T(0);
                    if(full(a))
                    {
                        int const s = aheadSlot(i);
                        mbarWait(smemAddr(&sh.bar[s]), aheadParity(i), timeoutNs, errWord);
                        uint4 const* src = slotPtr(s);
#pragma unroll
                        for(int k = 0; k < kPacks; ++k)
                        {
                            T e[W];
                            uint4 const q = src[k * kThreads + threadIdx.x];
                            memcpy(e, &q, 16);
#pragma unroll
                            for(int c = 0; c < W; ++c)
                                part = add(part, e[c]);
                        }
                    }
                    else
                    {
                        uint64_t const base = static_cast<uint64_t>(a) * Tr::TILE;
                        for(int k = threadIdx.x; k < Tr::TILE; k += kThreads)
                            if(base + k < n)
                                part = add(part, in[base + k]);
                    }
                    part = warpSum(part);
                    if(lane == 0)
                        sh.aheadTotal[warp] = part;
                }

                // (b) own tile: each thread scans its E consecutive elements, then the warp scans the thread totals
                T x[E];
                T laneExcl = T(0);
                T* const slotT = reinterpret_cast<T*>(own ? slotPtr(ownSlot(i)) : smem);
                bool const tma = own && full(t);
                if(own)
                {
                    if(tma)
                        mbarWait(smemAddr(&sh.bar[ownSlot(i)]), ownParity(i), timeoutNs, errWord);
                    else
                    {
                        // coalesced per-element copy into the slot, zero beyond the end
                        uint64_t const base = static_cast<uint64_t>(t) * Tr::TILE;
                        for(int k = threadIdx.x; k < Tr::TILE; k += kThreads)
                            slotT[k] = base + k < n ? in[base + k] : T(0);
                        __syncthreads();
                    }
                    uint4 const* mine = slotPtr(ownSlot(i)) + threadIdx.x * kPacks;
#pragma unroll
                    for(int k = 0; k < kPacks; ++k)
                    {
                        uint4 const q = mine[k];
                        memcpy(&x[k * W], &q, 16);
                    }
#pragma unroll
                    for(int e = 1; e < E; ++e)
                        x[e] = add(x[e - 1], x[e]);
                    T inc = x[E - 1];
#pragma unroll
                    for(int d = 1; d < 32; d <<= 1)
                    {
                        T const y = __shfl_up_sync(0xffffffffu, inc, d);
                        if(lane >= d)
                            inc = add(y, inc);
                    }
                    laneExcl = __shfl_up_sync(0xffffffffu, inc, 1);
                    if(lane == 0)
                        laneExcl = T(0);
                    if(lane == 31)
                        sh.warpTotal[warp] = inc;

                    // the range of aggregates: bounded waits for any that are not published yet
                    T part = T(0);
#pragma unroll
                    for(int q = 0; q < kMaxRange; ++q)
                    {
                        int const k = q * kThreads + static_cast<int>(threadIdx.x);
                        if(k < count)
                        {
                            T val = T(0);
                            if(!Aggregates<T>::decode(raw[q], epoch, val) && !abort)
                            {
                                uint64_t const t0 = globalTimerNs();
                                int polls = 0;
                                while(true)
                                {
                                    __nanosleep(64);
                                    agg.load(static_cast<uint64_t>(lo + k), raw[q]);
                                    if(Aggregates<T>::decode(raw[q], epoch, val))
                                        break;
                                    if((++polls & 15) == 0
                                       && (globalTimerNs() - t0 > timeoutNs || ldRelaxedU32(&hdr->abortEpoch) == epoch))
                                    {
                                        raiseAbort(hdr, epoch, errWord);
                                        abort = true;
                                        val = T(0);
                                        break;
                                    }
                                }
                            }
                            part = add(part, val);
                        }
                    }
                    part = warpSum(part);
                    if(lane == 0)
                        sh.rangeTotal[warp] = part;
                }
                __syncthreads();

                if(doAhead && threadIdx.x == 0 && a != static_cast<int64_t>(stallTile))
                {
                    T total = T(0);
#pragma unroll
                    for(int w = 0; w < kWarps; ++w)
                        total = add(total, sh.aheadTotal[w]);
                    agg.publish(static_cast<uint64_t>(a), epoch, total);
                }
                if(own)
                {
                    T range = T(0), warpPrefix = T(0);
#pragma unroll
                    for(int w = 0; w < kWarps; ++w)
                    {
                        range = add(range, sh.rangeTotal[w]);
                        if(w < warp)
                            warpPrefix = add(warpPrefix, sh.warpTotal[w]);
                    }
                    prefix = add(prefix, range);
                    T const off = add(add(prefix, warpPrefix), laneExcl);
                    T y[E];
                    if constexpr(INCL)
                    {
#pragma unroll
                        for(int e = 0; e < E; ++e)
                            y[e] = add(off, x[e]);
                    }
                    else
                    {
                        y[0] = off;
#pragma unroll
                        for(int e = 1; e < E; ++e)
                            y[e] = add(off, x[e - 1]);
                    }
                    uint4* mineOut = slotPtr(ownSlot(i)) + threadIdx.x * kPacks;
#pragma unroll
                    for(int k = 0; k < kPacks; ++k)
                    {
                        uint4 q;
                        memcpy(&q, &y[k * W], 16);
                        mineOut[k] = q;
                    }
                    if(tma)
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); // the bulk store reads it
                }
                __syncthreads(); // slot written; totals are reused by the next round
                if(own)
                {
                    if(tma)
                    {
                        if(threadIdx.x == 0)
                            bulkStore(out + t * Tr::TILE, smemAddr(slotPtr(ownSlot(i))), kTileBytes);
                    }
                    else
                    {
                        uint64_t const base = static_cast<uint64_t>(t) * Tr::TILE;
                        for(int k = threadIdx.x; k < Tr::TILE; k += kThreads)
                            if(base + k < n)
                                out[base + k] = slotT[k];
                    }
                }
            }
            if(VEC && threadIdx.x == 0)
                bulkWaitAll();
        }

        template<typename T>
        uint64_t tilesFor(uint64_t n)
        {
            return (n + Traits<T>::TILE - 1) / Traits<T>::TILE;
        }

        // Launch data of one kernel instantiation per device: resident blocks per SM (0 = not set up yet).
        template<typename T, bool INCL, bool VEC>
        int kernelResident(DeviceProps const* props, int* resident)
        {
            static std::atomic<int> cache[kMaxDevices];
            int r = cache[props->ordinal].load(std::memory_order_relaxed);
            if(r == 0)
            {
                auto kernel = scanKernel<T, INCL, VEC>;
                int const dyn = kSmemBytes;
                A3B_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn));
                int bps = 0;
                A3B_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bps, kernel, kThreads, dyn));
                if(bps < 1)
                {
                    setError("scan kernel does not fit on an SM");
                    return A3B_ERR_UNSUPPORTED;
                }
                r = bps;
                cache[props->ordinal].store(r, std::memory_order_relaxed);
            }
            *resident = r;
            return A3B_OK;
        }

        template<typename T, bool INCL, bool VEC>
        int launchScan(
            cudaStream_t s,
            DeviceProps const* props,
            T const* in,
            T* out,
            uint64_t n,
            uint64_t tiles,
            T const* carry,
            ScanHeader* hdr,
            unsigned epoch,
            uint64_t stallTile)
        {
            int resident = 0;
            int rc = kernelResident<T, INCL, VEC>(props, &resident);
            if(rc)
                return rc;
            uint64_t grid = static_cast<uint64_t>(props->smCount) * static_cast<uint64_t>(resident);
            if(grid > static_cast<uint64_t>(kMaxRange) * kThreads)
                grid = static_cast<uint64_t>(kMaxRange) * kThreads;
            if(grid > tiles)
                grid = tiles;
            unsigned* errWord = props->errWord;
            uint64_t timeout = waitTimeoutNs();
            void* args[] = {(void*) &in, (void*) &out, (void*) &n, (void*) &tiles, (void*) &carry,
                            (void*) &hdr, (void*) &epoch, (void*) &errWord, (void*) &timeout, (void*) &stallTile};
            size_t const dyn = kSmemBytes;
            A3B_CUDA(cudaLaunchCooperativeKernel(
                reinterpret_cast<void const*>(scanKernel<T, INCL, VEC>),
                dim3(static_cast<unsigned>(grid)),
                dim3(kThreads),
                args,
                dyn,
                s));
            return A3B_OK;
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
            size_t const need = scratchBytes(tiles, Traits<T>::WORDS);
            void* scr = nullptr;
            unsigned epoch = 1u;
            if(buffer)
            {
                if(bufBytes < need)
                {
                    setError("scan buffer too small: %zu bytes given, %zu needed", bufBytes, need);
                    return A3B_ERR_INVALID;
                }
                A3B_CUDA(cudaMemsetAsync(buffer, 0, need, s)); // caller memory: cleared, then epoch 1
                scr = buffer;
            }
            else
            {
                rc = streamScratch(s, kScratchScan, need, &scr, &epoch);
                if(rc)
                    return rc;
            }
            auto* hdr = static_cast<ScanHeader*>(scr);
            bool const vec = aligned16(in) && aligned16(out);
            if(inclusive)
                return vec ? launchScan<T, true, true>(s, props, in, out, n, tiles, carry, hdr, epoch, stallTile)
                           : launchScan<T, true, false>(s, props, in, out, n, tiles, carry, hdr, epoch, stallTile);
            return vec ? launchScan<T, false, true>(s, props, in, out, n, tiles, carry, hdr, epoch, stallTile)
                       : launchScan<T, false, false>(s, props, in, out, n, tiles, carry, hdr, epoch, stallTile);
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
        uint64_t const tile = static_cast<uint64_t>(kTileBytes / es);
        uint64_t const tiles = (n + tile - 1) / tile;
        return scratchBytes(tiles, es / 4);
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
