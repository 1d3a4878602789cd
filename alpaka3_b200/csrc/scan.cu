// Single-pass prefix sum with aggregates published ahead: onHost::inclusiveScan / exclusiveScan / *InPlace.
//
// Replaces the three-level Scan_ScanBlocksKernel + recursion + Scan_AddIncrementsKernel scheme of
// include/alpaka/onHost/algo/internal/scan.hpp:114-472 (about 4N-5N elements of traffic and 2*levels launches) with
// one launch that reads every element from HBM once and writes it once (2N).
//
// One block per tile (tile = blockIdx.x; blocks are dispatched in index order, so every block a tile waits for is
// resident or finished). A tile is 256 threads x 16 packs of 16 bytes (64 KB), two blocks per SM. Warp w owns a
// contiguous segment; in round r lane l holds the pack at segment offset (r*32 + l), so every load and store
// instruction of a warp covers 512 contiguous bytes. Scans run in registers: within the pack, across lanes
// (shfl_up), across rounds (running segment total), across the 8 warps (shared memory), then across tiles.
//
// Aggregates ahead of prefixes. In a plain decoupled look-back a tile's prefix waits until every predecessor up to
// the nearest inclusive prefix has loaded its tile from HBM, and the waiting blocks hold their tiles on chip; at full
// HBM load that wait (several L2 round trips behind loads still in flight) limits the scan to ~60% of the copy rate.
// Here block b also reduces tile b + lag: at its start one thread issues a TMA bulk copy of that tile into shared
// memory, and after block b has written its own tile it sums the staged tile and publishes it as the aggregate of
// tile b + lag. By the time block b + lag runs, the aggregates of all its recent predecessors are long published, so
// its look-back resolves in its first poll (whose status words it loads before its own tile), and its own tile (read
// by the TMA copy a few microseconds earlier) is served from L2: HBM still sees one read and one write per element.
// lag = 2 x the resident blocks of the launch keeps the in-between window (lag tiles, ~40 MB) well inside the 126 MB
// L2. Tiles below lag publish their own aggregate. Aggregates and inclusive prefixes live in separate status arrays,
// so every status word has one writer. When input and output overlap (in-place scan), block b waits until the
// aggregate of its tile is published, i.e. until the ahead copy has read the tile, before it overwrites it.
//
// Status words carry an epoch handed out by the host per call on the stream's cached scratch (a caller buffer is
// cleared and uses epoch 1), so the scratch needs no clearing between calls. A status is one 64-bit word per 32 bits
// of value: flag (2 bits) | epoch (30 bits) | 32 value bits; relaxed 64-bit accesses are single-copy atomic, and an
// 8-byte value's two words are accepted only when both carry the same flag and epoch. Every spin is bounded by
// %globaltimer; on timeout the block raises the device error word and an abort mark that ends the other blocks'
// waits of the same call. Input or output not aligned to 16 bytes uses the same kernel with per-element loads and
// no TMA.
#include <type_traits>

#include "common.cuh"

namespace a3b
{
    namespace
    {
        constexpr int kBlock = 256;
        constexpr int kWarps = kBlock / 32;
        constexpr int kLookSpan = 512; // predecessors polled per look-back window (multiple of 256)
        constexpr unsigned kEpochMask = 0x3FFFFFFFu;
        constexpr unsigned kFlagA = 1u, kFlagP = 2u;

        struct ScanHeader
        {
            unsigned abortEpoch; // epoch of a call whose waits gave up
            unsigned pad[15];
        };
        static_assert(sizeof(ScanHeader) == 64, "header size");

#ifndef A3B_SCAN_ROUNDS
#define A3B_SCAN_ROUNDS 16
#endif
#ifndef A3B_SCAN_MINB
#define A3B_SCAN_MINB 2
#endif
#ifndef A3B_SCAN_PACK
#define A3B_SCAN_PACK 16
#endif
        template<typename T>
        struct Traits
        {
            static constexpr int PB = A3B_SCAN_PACK;                      // bytes per pack (one 256-bit access)
            static constexpr int W = PB / static_cast<int>(sizeof(T));    // elements per pack
            static constexpr int ROUNDS = A3B_SCAN_ROUNDS;                // packs per thread
            static constexpr int TILE = kBlock * ROUNDS * W;              // elements per tile
            static constexpr int STAGE = kBlock * ROUNDS * PB;            // bytes per tile
            static constexpr int WORDS = static_cast<int>(sizeof(T)) / 4; // 64-bit status words per tile
            static constexpr int MIN_BLOCKS = A3B_SCAN_MINB;
        };

        // one pack of global memory <-> registers, evict-first (each element is read once and written once here)
        template<int PB>
        __device__ __forceinline__ void loadPack(void const* p, uint32_t (&w)[PB / 4])
        {
            if constexpr(PB == 32)
            {
                unsigned long long r0, r1, r2, r3;
                asm volatile("ld.global.cs.v4.u64 {%0, %1, %2, %3}, [%4];"
                             : "=l"(r0), "=l"(r1), "=l"(r2), "=l"(r3)
                             : "l"(p));
                unsigned long long const raw[4] = {r0, r1, r2, r3};
                memcpy(w, raw, 32);
            }
            else
            {
                uint4 const v = __ldcs(static_cast<uint4 const*>(p));
                memcpy(w, &v, 16);
            }
        }

        template<int PB>
        __device__ __forceinline__ void storePack(void* p, uint32_t const (&w)[PB / 4])
        {
            if constexpr(PB == 32)
            {
                unsigned long long raw[4];
                memcpy(raw, w, 32);
                asm volatile("st.global.cs.v4.u64 [%0], {%1, %2, %3, %4};" ::"l"(p), "l"(raw[0]), "l"(raw[1]),
                             "l"(raw[2]), "l"(raw[3])
                             : "memory");
            }
            else
            {
                uint4 v;
                memcpy(&v, w, 16);
                __stcs(static_cast<uint4*>(p), v);
            }
        }

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

        // scratch layout: header | u64 aggregate[tiles * WORDS] | u64 inclusive[tiles * WORDS]
        __host__ __device__ inline size_t statusBytes(uint64_t tiles, int words)
        {
            return align256(tiles * 8u * static_cast<uint64_t>(words));
        }

        __host__ __device__ inline size_t scratchBytes(uint64_t tiles, int words)
        {
            return sizeof(ScanHeader) + 2u * statusBytes(tiles, words);
        }

        template<typename T>
        struct Status
        {
            uint64_t* agg; // aggregate of each tile (flag A), written once per call
            uint64_t* inc; // inclusive prefix of each tile (flag P), written once per call

            __device__ static void put(uint64_t* base, uint64_t tile, unsigned flag, unsigned epoch, T value)
            {
                constexpr int WD = Traits<T>::WORDS;
                uint32_t parts[WD];
                memcpy(parts, &value, sizeof(T));
                uint64_t const tag = (static_cast<uint64_t>(flag) << 62) | (static_cast<uint64_t>(epoch) << 32);
#pragma unroll
                for(int k = 0; k < WD; ++k)
                    stRelaxedU64(base + tile * WD + k, tag | parts[k]);
            }

            // true when all words of w carry this epoch's tag; value decoded
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

            __device__ void publishA(uint64_t tile, unsigned epoch, T value) const
            {
                put(agg, tile, kFlagA, epoch, value);
            }

            __device__ void publishP(uint64_t tile, unsigned epoch, T value) const
            {
                put(inc, tile, kFlagP, epoch, value);
            }

            // raw status words of one tile, as loaded
            struct Raw
            {
                uint64_t i[Traits<T>::WORDS];
                uint64_t a[Traits<T>::WORDS];
            };

            __device__ void load(uint64_t tile, Raw& r) const
            {
                constexpr int WD = Traits<T>::WORDS;
#pragma unroll
                for(int k = 0; k < WD; ++k)
                {
                    r.i[k] = ldRelaxedU64(inc + tile * WD + k);
                    r.a[k] = ldRelaxedU64(agg + tile * WD + k);
                }
            }

            // kFlagP with the inclusive prefix, else kFlagA with the aggregate, else 0 (not yet published)
            __device__ static unsigned classify(Raw const& r, unsigned epoch, T& value)
            {
                if(decode(r.i, epoch, value))
                    return kFlagP;
                if(decode(r.a, epoch, value))
                    return kFlagA;
                return 0u;
            }

            __device__ unsigned peek(uint64_t tile, unsigned epoch, T& value) const
            {
                Raw r;
                load(tile, r);
                return classify(r, epoch, value);
            }

            __device__ bool aggPublished(uint64_t tile, unsigned epoch) const
            {
                constexpr int WD = Traits<T>::WORDS;
                uint64_t wa[WD];
#pragma unroll
                for(int k = 0; k < WD; ++k)
                    wa[k] = ldRelaxedU64(agg + tile * WD + k);
                T v;
                return decode(wa, epoch, v);
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
            T red[kWarps];
            int firstP[kLookSpan / 32];
            int firstInv[kLookSpan / 32];
            int abort;
            alignas(8) unsigned long long mbar;
        };

        __device__ __forceinline__ bool abortRequested(ScanHeader* hdr, unsigned epoch, uint64_t t0, uint64_t timeoutNs)
        {
            return (globalTimerNs() - t0 > timeoutNs) || (ldRelaxedU32(&hdr->abortEpoch) == epoch);
        }

        __device__ __forceinline__ void raiseAbort(ScanHeader* hdr, unsigned epoch, unsigned* errWord)
        {
            atomicOr(errWord, kErrTimeout);
            stRelaxedU32(&hdr->abortEpoch, epoch);
        }

        // Block-wide look-back for `tile` (> 0); returns the exclusive prefix. One window covers kLookSpan
        // predecessors: thread i polls predecessors at distance i, i + 256, ... so a single L2 round trip spans more
        // tiles than a launch keeps in flight. A window is complete as soon as every predecessor up to the nearest
        // inclusive prefix is valid (stragglers farther back do not matter); without a prefix in the window all of
        // it must be valid and the window moves back. Sets sh.abort (and the error word) when a wait gives up.
        constexpr int kLookQ = kLookSpan / kBlock; // predecessors per thread and window

        // the first window's status words, loaded before the block's own tile so that they are not queued behind it
        template<typename T>
        __device__ __forceinline__ void prefetchWindow(
            Status<T> const& st,
            uint64_t tile,
            typename Status<T>::Raw (&pre)[kLookQ])
        {
#pragma unroll
            for(int q = 0; q < kLookQ; ++q)
            {
                int64_t const j = static_cast<int64_t>(tile) - 1 - static_cast<int64_t>(threadIdx.x) - q * kBlock;
                if(j >= 0)
                    st.load(static_cast<uint64_t>(j), pre[q]);
            }
        }

        template<typename T, bool PRE>
        __device__ T lookBack(
            Status<T> const& st,
            uint64_t tile,
            unsigned epoch,
            Shared<T>& sh,
            ScanHeader* hdr,
            unsigned* errWord,
            uint64_t timeoutNs,
            typename Status<T>::Raw const (&pre)[kLookQ])
        {
            constexpr int Q = kLookQ;
            int const warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
            uint64_t const t0 = globalTimerNs();
            int64_t pred = static_cast<int64_t>(tile) - 1;
            T acc = T(0);
            int polls = 0;
            while(true)
            {
                T val[Q];
                unsigned flag[Q];
                int64_t j[Q];
#pragma unroll
                for(int q = 0; q < Q; ++q)
                {
                    j[q] = pred - static_cast<int64_t>(threadIdx.x) - q * kBlock;
                    val[q] = T(0);
                    flag[q] = j[q] >= 0 ? 0u : kFlagP; // before tile 0: an empty inclusive prefix
                }
                int stop;
                bool firstPoll = PRE && pred == static_cast<int64_t>(tile) - 1;
                while(true)
                {
#pragma unroll
                    for(int q = 0; q < Q; ++q)
                        if(flag[q] != kFlagP)
                            flag[q] = firstPoll ? Status<T>::classify(pre[q], epoch, val[q])
                                                : st.peek(static_cast<uint64_t>(j[q]), epoch, val[q]);
                    firstPoll = false;
#pragma unroll
                    for(int q = 0; q < Q; ++q)
                    {
                        unsigned const pm = __ballot_sync(0xffffffffu, flag[q] == kFlagP);
                        unsigned const im = __ballot_sync(0xffffffffu, flag[q] == 0u);
                        if(lane == 0)
                        {
                            sh.firstP[q * kWarps + warp] = pm ? __ffs(pm) - 1 : 32;
                            sh.firstInv[q * kWarps + warp] = im ? __ffs(im) - 1 : 32;
                        }
                    }
                    __syncthreads();
                    // distance d = q*256 + w*32 + lane: scan (q, w) from the far end so the last hit is the nearest
                    stop = kLookSpan;
                    int inv = kLookSpan;
#pragma unroll
                    for(int k = Q * kWarps - 1; k >= 0; --k)
                    {
                        if(sh.firstP[k] < 32)
                            stop = k * 32 + sh.firstP[k];
                        if(sh.firstInv[k] < 32)
                            inv = k * 32 + sh.firstInv[k];
                    }
                    if(stop < kLookSpan ? inv > stop : inv == kLookSpan)
                        break;
                    if(threadIdx.x == 0 && (++polls & 7) == 0)
                        sh.abort = abortRequested(hdr, epoch, t0, timeoutNs);
                    __syncthreads(); // firstP / firstInv are rewritten by the next poll
                    if(sh.abort)
                        break;
                    if(polls > 4)
                        __nanosleep(32);
                }
                if(sh.abort)
                    break;
                T mine = T(0);
#pragma unroll
                for(int q = 0; q < Q; ++q)
                    if(q * kBlock + static_cast<int>(threadIdx.x) <= stop && j[q] >= 0)
                        mine = add(mine, val[q]);
                T const ws = warpSum(mine);
                if(lane == 0)
                    sh.red[warp] = ws;
                __syncthreads();
                T window = T(0);
#pragma unroll
                for(int w = 0; w < kWarps; ++w)
                    window = add(window, sh.red[w]);
                acc = add(window, acc);
                __syncthreads(); // firstP / red are rewritten by the next window
                if(stop < kLookSpan)
                    break;
                pred -= kLookSpan;
            }
            if(sh.abort && threadIdx.x == 0)
                raiseAbort(hdr, epoch, errWord);
            return acc;
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

        // Total of one warp-segment round, combined in exactly the order scanRound combines it (so a tile's
        // aggregate has the same bits whether the ahead reduction or the tile's own scan computes it).
        template<typename T>
        __device__ __forceinline__ T roundTotal(T const (&p)[Traits<T>::W])
        {
            constexpr int W = Traits<T>::W;
            int const lane = threadIdx.x & 31;
            T x = p[0];
#pragma unroll
            for(int k = 1; k < W; ++k)
                x = add(x, p[k]);
#pragma unroll
            for(int d = 1; d < 32; d <<= 1)
            {
                T const y = __shfl_up_sync(0xffffffffu, x, d);
                if(lane >= d)
                    x = add(y, x);
            }
            return __shfl_sync(0xffffffffu, x, 31);
        }

        // ------------------------------------------------------------------------------ TMA bulk copy + mbarrier
        __device__ __forceinline__ uint32_t smemAddr(void const* p)
        {
            return static_cast<uint32_t>(__cvta_generic_to_shared(p));
        }

        __device__ __forceinline__ void mbarInit(uint32_t bar, unsigned count)
        {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }

        __device__ __forceinline__ void mbarExpectTx(uint32_t bar, unsigned bytes)
        {
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
        }

        // global -> shared bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned), completing on `bar`
        __device__ __forceinline__ void bulkLoad(uint32_t dst, void const* src, unsigned bytes, uint32_t bar)
        {
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                         ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                         : "memory");
        }

        __device__ __forceinline__ bool mbarTryWait(uint32_t bar, unsigned parity)
        {
            unsigned done;
            asm volatile(
                "{\n\t.reg .pred p;\n\t"
                "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                "selp.u32 %0, 1, 0, p;\n\t}"
                : "=r"(done)
                : "r"(bar), "r"(parity)
                : "memory");
            return done != 0u;
        }

        // bounded wait for phase 0 of `bar`; false when `timeoutNs` passed first
        __device__ bool mbarWaitBounded(uint32_t bar, uint64_t timeoutNs)
        {
            uint64_t const t0 = globalTimerNs();
            while(!mbarTryWait(bar, 0u))
                if(globalTimerNs() - t0 > timeoutNs)
                    return false;
            return true;
        }

        // Sum of a staged tile (Traits<T>::STAGE bytes in shared memory) in the order the tile's own scan combines
        // it, so that the aggregate has the same bits either way; integer sums wrap and need no particular order.
        template<typename T>
        __device__ __forceinline__ T stagedTotal(uint4 const* stage, Shared<T>& sh)
        {
            using Tr = Traits<T>;
            constexpr int W = Tr::W, R = Tr::ROUNDS;
            int const warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
            T run = T(0);
            if constexpr(std::is_integral_v<T>)
            {
                // conflict-free: thread i reads the 16-byte words i, i + 256, ...
                constexpr int N16 = Tr::STAGE / 16 / kBlock;
                uint64_t acc = 0u;
#pragma unroll
                for(int k = 0; k < N16; ++k)
                {
                    uint4 const q = stage[k * kBlock + threadIdx.x];
                    if constexpr(sizeof(T) == 4)
                        acc += static_cast<uint64_t>(q.x) + q.y + q.z + q.w;
                    else
                        acc += (static_cast<uint64_t>(q.y) << 32 | q.x) + (static_cast<uint64_t>(q.w) << 32 | q.z);
                }
                run = static_cast<T>(acc);
                run = warpSum(run);
            }
            else
            {
                uint4 const* seg = stage + warp * (32 * R * Tr::PB / 16);
#pragma unroll
                for(int r = 0; r < R; ++r)
                {
                    T p[W];
                    memcpy(&p[0], seg + (r * 32 + lane) * (Tr::PB / 16), Tr::PB);
                    run = add(run, roundTotal<T>(p));
                }
            }
            if(lane == 0)
                sh.aheadTotal[warp] = run;
            __syncthreads();
            T total = T(0);
#pragma unroll
            for(int w = 0; w < kWarps; ++w)
                total = add(total, sh.aheadTotal[w]);
            return total;
        }

        // ------------------------------------------------------------------------------------------- the kernel
        // Tile = blockIdx.x. Block b: (1) issues the TMA copy of tile b + lag into shared memory, (2) loads its own
        // tile into registers, (3) looks back (b >= lag: while its loads are in flight; b < lag: after publishing its
        // own aggregate), scans and publishes its inclusive prefix, (4) writes its tile, (5) sums the staged tile
        // b + lag and publishes that aggregate. VEC: input and output aligned to the pack size (TMA and 32-byte
        // packs); otherwise per-element accesses and no TMA.
        template<typename T, bool INCL, bool VEC>
        __global__ void __launch_bounds__(kBlock, Traits<T>::MIN_BLOCKS) scanTileKernel(
            T const* in,
            T* out,
            uint64_t n,
            uint64_t tiles,
            uint64_t lag,
            int overlap,
            T const* carryIn,
            ScanHeader* hdr,
            unsigned epoch,
            unsigned* errWord,
            uint64_t timeoutNs,
            uint64_t stallTile)
        {
            using Tr = Traits<T>;
            constexpr int W = Tr::W;
            constexpr int R = Tr::ROUNDS;
            constexpr int PW = Tr::PB / 4; // 32-bit words per pack
            extern __shared__ __align__(128) uint4 stage[]; // the ahead tile (VEC only): Tr::STAGE bytes
            __shared__ Shared<T> sh;
            int const warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
            uint64_t const tile = blockIdx.x;
            Status<T> const st{
                reinterpret_cast<uint64_t*>(hdr + 1),
                reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(hdr + 1) + statusBytes(tiles, Tr::WORDS))};

            // (1) ahead copy
            uint64_t const ahead = tile + lag;
            bool const doAhead = lag != 0 && ahead < tiles;
            bool const aheadTma = VEC && doAhead && (ahead + 1u) * Tr::TILE <= n;
            uint32_t const bar = smemAddr(&sh.mbar);
            if(threadIdx.x == 0)
            {
                sh.abort = 0;
                if(aheadTma)
                {
                    mbarInit(bar, 1u);
                    mbarExpectTx(bar, Tr::STAGE);
                    bulkLoad(smemAddr(stage), in + ahead * Tr::TILE, Tr::STAGE, bar);
                }
            }

            // (2) own tile. A tile whose aggregate an earlier block publishes (tile >= lag) finds its predecessors'
            // aggregates published already: its first look-back window is loaded before the tile and evaluated while
            // the tile's loads are in flight.
            bool const stalled = (tile == stallTile);
            bool const ownAgg = lag == 0 || tile < lag; // else block tile - lag publishes it
            typename Status<T>::Raw pre[kLookQ];
            if(tile != 0 && !ownAgg)
                prefetchWindow<T>(st, tile, pre);
            uint64_t const segBase = tile * Tr::TILE + static_cast<uint64_t>(warp) * (32 * R * W);
            bool const full = (tile + 1u) * Tr::TILE <= n;
            T v[R][W];
            if(VEC && full)
            {
#pragma unroll
                for(int r = 0; r < R; ++r)
                {
                    uint32_t w[PW];
                    loadPack<Tr::PB>(in + segBase + static_cast<uint64_t>(r * 32 + lane) * W, w);
                    memcpy(&v[r][0], w, Tr::PB);
                }
            }
            else
            {
#pragma unroll
                for(int r = 0; r < R; ++r)
#pragma unroll
                    for(int k = 0; k < W; ++k)
                    {
                        uint64_t const idx = segBase + static_cast<uint64_t>(r * 32 + lane) * W + k;
                        v[r][k] = idx < n ? in[idx] : T(0);
                    }
            }

            // (3) prefix and scan
            T prefix = T(0);
            if(tile != 0 && !ownAgg)
                prefix = lookBack<T, true>(st, tile, epoch, sh, hdr, errWord, timeoutNs, pre);
            T run = T(0);
#pragma unroll
            for(int r = 0; r < R; ++r)
                scanRound<T, INCL>(v[r], run);
            if(lane == 0)
                sh.warpTotal[warp] = run;
            __syncthreads();
            T warpPrefix = T(0), agg = T(0);
#pragma unroll
            for(int w = 0; w < kWarps; ++w)
            {
                T const t = sh.warpTotal[w];
                if(w < warp)
                    warpPrefix = add(warpPrefix, t);
                agg = add(agg, t);
            }
            if(tile == 0)
            {
                if(carryIn)
                    prefix = *carryIn;
            }
            else if(ownAgg)
            {
                if(threadIdx.x == 0 && !stalled)
                    st.publishA(tile, epoch, agg);
                prefix = lookBack<T, false>(st, tile, epoch, sh, hdr, errWord, timeoutNs, pre);
            }
            if(threadIdx.x == 0 && !stalled)
                st.publishP(tile, epoch, add(prefix, agg));
            if(overlap && !ownAgg)
            {
                // in place: the ahead copy of block tile - lag must have read this tile before it is overwritten
                if(threadIdx.x == 0)
                {
                    uint64_t const t0 = globalTimerNs();
                    int polls = 0;
                    while(!sh.abort && !st.aggPublished(tile, epoch))
                    {
                        if((++polls & 7) == 0 && abortRequested(hdr, epoch, t0, timeoutNs))
                        {
                            sh.abort = 1;
                            raiseAbort(hdr, epoch, errWord);
                        }
                        __nanosleep(64);
                    }
                }
                __syncthreads();
            }

            // (4) own output
            T const off = add(prefix, warpPrefix);
            if(VEC && full)
            {
#pragma unroll
                for(int r = 0; r < R; ++r)
                {
#pragma unroll
                    for(int k = 0; k < W; ++k)
                        v[r][k] = add(off, v[r][k]);
                    uint32_t w[PW];
                    memcpy(w, &v[r][0], Tr::PB);
                    storePack<Tr::PB>(out + segBase + static_cast<uint64_t>(r * 32 + lane) * W, w);
                }
            }
            else
            {
#pragma unroll
                for(int r = 0; r < R; ++r)
#pragma unroll
                    for(int k = 0; k < W; ++k)
                    {
                        uint64_t const idx = segBase + static_cast<uint64_t>(r * 32 + lane) * W + k;
                        if(idx < n)
                            out[idx] = add(off, v[r][k]);
                    }
            }

            // (5) aggregate of tile + lag
            if(!doAhead)
                return;
            T aa = T(0);
            bool ok = true;
            if(aheadTma)
            {
                ok = mbarWaitBounded(bar, timeoutNs);
                if(!ok)
                {
                    // the copy still owns the staging buffer: give it one more bounded wait before the block exits
                    if(threadIdx.x == 0)
                        atomicOr(errWord, kErrTimeout);
                    mbarWaitBounded(bar, timeoutNs);
                }
                ok = __syncthreads_and(ok) != 0; // publish only when every thread saw the staged tile
                if(ok)
                    aa = stagedTotal<T>(stage, sh);
            }
            else
            {
                uint64_t const aBase = ahead * Tr::TILE + static_cast<uint64_t>(warp) * (32 * R * W);
                T aheadRun = T(0);
#pragma unroll
                for(int r = 0; r < R; ++r)
                {
                    T p[W];
#pragma unroll
                    for(int k = 0; k < W; ++k)
                    {
                        uint64_t const idx = aBase + static_cast<uint64_t>(r * 32 + lane) * W + k;
                        p[k] = idx < n ? in[idx] : T(0);
                    }
                    aheadRun = add(aheadRun, roundTotal<T>(p));
                }
                if(lane == 0)
                    sh.aheadTotal[warp] = aheadRun;
                __syncthreads();
#pragma unroll
                for(int w = 0; w < kWarps; ++w)
                    aa = add(aa, sh.aheadTotal[w]);
            }
            if(threadIdx.x == 0 && ok && ahead != stallTile)
                st.publishA(ahead, epoch, aa);
        }

        template<typename T>
        uint64_t tilesFor(uint64_t n)
        {
            return (n + Traits<T>::TILE - 1) / Traits<T>::TILE;
        }

        // per-device launch data of one kernel instantiation: resident blocks per SM (0 = not set up yet)
        template<typename T, bool INCL, bool VEC>
        int kernelResident(DeviceProps const* props, int* resident)
        {
            static std::atomic<int> cache[kMaxDevices];
            int r = cache[props->ordinal].load(std::memory_order_relaxed);
            if(r == 0)
            {
                auto kernel = scanTileKernel<T, INCL, VEC>;
                int const dyn = VEC ? Traits<T>::STAGE : 0;
                if(dyn > 0)
                    A3B_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn));
                int b = 0;
                A3B_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, kBlock, dyn));
                r = b > 0 ? b : 1;
                cache[props->ordinal].store(r, std::memory_order_relaxed);
            }
            *resident = r;
            return A3B_OK;
        }

        // Tiles between a tile and the block that reduces it ahead: 2 x the blocks the launch keeps resident
        // (A3B_SCAN_LAG overrides it for tuning; 0 turns the ahead reduction off).
        uint64_t lagFor(DeviceProps const* props, int residentPerSm)
        {
            static long long const env = [] {
                char const* e = getenv("A3B_SCAN_LAG");
                return e ? atoll(e) : -1ll;
            }();
            if(env >= 0)
                return static_cast<uint64_t>(env);
            return 2ull * static_cast<uint64_t>(props->smCount) * static_cast<uint64_t>(residentPerSm);
        }

        template<typename T, bool INCL, bool VEC>
        int launchScan(
            cudaStream_t s,
            DeviceProps const* props,
            T const* in,
            T* out,
            uint64_t n,
            uint64_t tiles,
            int overlap,
            T const* carry,
            ScanHeader* hdr,
            unsigned epoch,
            uint64_t stallTile)
        {
            int resident = 0;
            int rc = kernelResident<T, INCL, VEC>(props, &resident);
            if(rc)
                return rc;
            uint64_t const lag = lagFor(props, resident);
            int const dyn = VEC ? Traits<T>::STAGE : 0;
            scanTileKernel<T, INCL, VEC><<<dim3(static_cast<unsigned>(tiles)), kBlock, dyn, s>>>(
                in, out, n, tiles, lag, overlap, carry, hdr, epoch, props->errWord, waitTimeoutNs(), stallTile);
            A3B_CHECK_LAUNCH("scan launch");
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
            if(tiles >= 0x7FFFFFFFull)
            {
                setError("scan of %llu elements exceeds the tile index range", static_cast<unsigned long long>(n));
                return A3B_ERR_TOO_LARGE;
            }
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
            auto const packAligned = [](void const* p) {
                return (reinterpret_cast<uintptr_t>(p) % static_cast<uintptr_t>(Traits<T>::PB)) == 0u;
            };
            bool const vec = packAligned(in) && packAligned(out);
            auto const ib = reinterpret_cast<uintptr_t>(in), ob = reinterpret_cast<uintptr_t>(out);
            int const overlap = (ib < ob + n * sizeof(T) && ob < ib + n * sizeof(T)) ? 1 : 0;
            if(inclusive)
                return vec ? launchScan<T, true, true>(s, props, in, out, n, tiles, overlap, carry, hdr, epoch, stallTile)
                           : launchScan<T, true, false>(s, props, in, out, n, tiles, overlap, carry, hdr, epoch, stallTile);
            return vec ? launchScan<T, false, true>(s, props, in, out, n, tiles, overlap, carry, hdr, epoch, stallTile)
                       : launchScan<T, false, false>(s, props, in, out, n, tiles, overlap, carry, hdr, epoch, stallTile);
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
        uint64_t const tile = es == 4 ? Traits<uint32_t>::TILE : Traits<uint64_t>::TILE;
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
