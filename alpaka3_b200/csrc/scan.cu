// Single-pass prefix sum (decoupled look-back): onHost::inclusiveScan / exclusiveScan / *InPlace.
//
// Replaces the three-level Scan_ScanBlocksKernel + recursion + Scan_AddIncrementsKernel scheme of
// include/alpaka/onHost/algo/internal/scan.hpp:114-472 (about 4N-5N elements of traffic and 2*levels launches) with
// one launch that reads every element once and writes it once (2N).
//
// One block per tile (tile = blockIdx.x; blocks are dispatched in index order, so every predecessor a tile waits for
// is resident or finished). A tile is 256 threads x ROUNDS 16-byte packs held in registers: 48 KB (12 rounds) for
// 4-byte and 64 KB (16 rounds) for 8-byte types, the largest tiles that keep 3 / 2 blocks resident per SM; larger
// tiles mean fewer look-backs per byte. Warp w owns a contiguous segment; in round r lane l holds the pack at segment
// offset (r*32 + l), so every load and store instruction of a warp covers 512 contiguous bytes. Scans run in
// registers: within the pack, across lanes (shfl_up), across rounds (running segment total), across the 8 warps
// (shared memory), then across tiles. Unaligned input or output uses the same kernel with per-element loads.
//
// Cross-tile protocol: a tile publishes its aggregate (flag A), then the WHOLE block looks back: thread i polls the
// predecessors at distance i, i + 256, ... so one L2 round trip covers a window of kLookSpan tiles, more than a
// launch keeps in flight. The window is complete as soon as every predecessor up to the nearest inclusive prefix
// (flag P) is valid; the tile then publishes its own inclusive prefix. Status words carry an epoch handed out by the
// host per call on the stream's cached scratch (a caller buffer is cleared and uses epoch 1), so the scratch needs no
// clearing between calls. A status is one 64-bit word per 32 bits of value: flag (2 bits) | epoch (30 bits) | 32
// value bits; relaxed 64-bit accesses are single-copy atomic, and an 8-byte value's two words are accepted only when
// both carry the same flag and epoch. Every spin is bounded by %globaltimer; on timeout the block raises the device
// error word and an abort mark that ends the other blocks' waits of the same call.
#include <type_traits>

#include "common.cuh"

namespace a3b
{
    namespace
    {
        constexpr int kBlock = 256;
        constexpr int kWarps = kBlock / 32;
#ifndef A3B_SCAN_LOOKSPAN
#define A3B_SCAN_LOOKSPAN 512
#endif
        constexpr int kLookSpan = A3B_SCAN_LOOKSPAN; // predecessors polled per look-back window (multiple of 256)
        constexpr unsigned kEpochMask = 0x3FFFFFFFu;
        constexpr unsigned kFlagA = 1u, kFlagP = 2u;

        struct ScanHeader
        {
            unsigned abortEpoch; // epoch of a call whose waits gave up
            unsigned pad[15];
        };
        static_assert(sizeof(ScanHeader) == 64, "header size");

        // Tile shape per element size (measured on B200): 48 KB tiles for 4-byte and 64 KB tiles for 8-byte types
        // (12 / 16 rounds of one 16-byte pack per thread), the largest that keep 3 / 2 blocks resident per SM.
        template<int ES>
        constexpr int roundsFor()
        {
            return ES == 4 ? 12 : 16;
        }

        template<typename T>
        struct Traits
        {
            static constexpr int W = 16 / static_cast<int>(sizeof(T));    // elements per 16-byte pack
            static constexpr int ROUNDS = roundsFor<sizeof(T)>();         // packs per thread
            static constexpr int TILE = kBlock * ROUNDS * W;              // elements per tile
            static constexpr int WORDS = static_cast<int>(sizeof(T)) / 4; // 64-bit status words per tile
            static constexpr int MIN_BLOCKS = ROUNDS <= 8 ? 4 : (ROUNDS <= 12 ? 3 : 2);
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

        // scratch layout: header | u64 status[tiles * WORDS]
        __host__ __device__ inline size_t scratchBytes(uint64_t tiles, int words)
        {
            return sizeof(ScanHeader) + align256(tiles * 8u * static_cast<uint64_t>(words));
        }

        template<typename T>
        struct Status
        {
            uint64_t* word;

            __device__ void publish(uint64_t tile, unsigned flag, unsigned epoch, T value) const
            {
                constexpr int WD = Traits<T>::WORDS;
                uint32_t parts[WD];
                memcpy(parts, &value, sizeof(T));
                uint64_t const tag = (static_cast<uint64_t>(flag) << 62) | (static_cast<uint64_t>(epoch) << 32);
#pragma unroll
                for(int k = 0; k < WD; ++k)
                    stRelaxedU64(word + tile * WD + k, tag | parts[k]);
            }

            // flag seen for `tile` in this epoch (0 = not yet, or the words of an 8-byte value disagree) and its value
            __device__ unsigned peek(uint64_t tile, unsigned epoch, T& value) const
            {
                constexpr int WD = Traits<T>::WORDS;
                uint64_t w[WD];
#pragma unroll
                for(int k = 0; k < WD; ++k)
                    w[k] = ldRelaxedU64(word + tile * WD + k);
                unsigned const tag = static_cast<unsigned>(w[0] >> 32);
                if((tag & kEpochMask) != epoch)
                    return 0u;
                uint32_t parts[WD];
#pragma unroll
                for(int k = 0; k < WD; ++k)
                {
                    if(static_cast<unsigned>(w[k] >> 32) != tag)
                        return 0u;
                    parts[k] = static_cast<uint32_t>(w[k]);
                }
                memcpy(&value, parts, sizeof(T));
                return tag >> 30;
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
            T red[kWarps];
            int firstP[kLookSpan / 32];
            int firstInv[kLookSpan / 32];
            int abort;
        };

        // Block-wide look-back for `tile` (> 0) whose aggregate is already published; returns the exclusive prefix.
        // One window covers kLookSpan predecessors: thread i polls predecessors at distance i, i + 256, ... so a
        // single L2 round trip spans more tiles than a launch keeps in flight (the distance to the nearest published
        // inclusive prefix stays inside one window). A window is complete as soon as every predecessor up to the
        // nearest inclusive prefix is valid (stragglers farther back do not matter); without a prefix in the window
        // all of it must be valid and the window moves back. Sets sh.abort (and the error word) when a wait gives up.
        template<typename T>
        __device__ T lookBack(
            Status<T> const& st,
            uint64_t tile,
            unsigned epoch,
            Shared<T>& sh,
            ScanHeader* hdr,
            unsigned* errWord,
            uint64_t timeoutNs)
        {
            constexpr int Q = kLookSpan / kBlock;
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
                while(true)
                {
#pragma unroll
                    for(int q = 0; q < Q; ++q)
                        if(flag[q] == 0u)
                            flag[q] = st.peek(static_cast<uint64_t>(j[q]), epoch, val[q]);
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
                        sh.abort = (globalTimerNs() - t0 > timeoutNs) || (ldRelaxedU32(&hdr->abortEpoch) == epoch);
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
            {
                atomicOr(errWord, kErrTimeout);
                stRelaxedU32(&hdr->abortEpoch, epoch);
            }
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

        // ---------------------------------------------------------------- one tile per block, data in registers
        // Tile = blockIdx.x: blocks are dispatched in index order, so every predecessor a block waits for is already
        // resident (the bounded waits turn any violation into a reported timeout, never a hang).
        template<typename T, bool INCL, bool VEC>
        __global__ void __launch_bounds__(kBlock, Traits<T>::MIN_BLOCKS) scanTileKernel(
            T const* in,
            T* out,
            uint64_t n,
            T const* carryIn,
            ScanHeader* hdr,
            unsigned epoch,
            unsigned* errWord,
            uint64_t timeoutNs,
            uint64_t stallTile)
        {
            using Tr = Traits<T>;
            constexpr int W = Tr::W;
            __shared__ Shared<T> sh;
            int const warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
            uint64_t const tile = blockIdx.x;
            if(threadIdx.x == 0)
                sh.abort = 0;
            Status<T> const st{reinterpret_cast<uint64_t*>(hdr + 1)};

            constexpr int kRounds = Tr::ROUNDS;
            uint64_t const segBase = tile * Tr::TILE + static_cast<uint64_t>(warp) * (32 * kRounds * W);
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
            T run = T(0);
#pragma unroll
            for(int r = 0; r < kRounds; ++r)
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
            bool const stalled = (tile == stallTile);
            T prefix = T(0);
            if(tile == 0)
            {
                if(carryIn)
                    prefix = *carryIn;
            }
            else
            {
                if(threadIdx.x == 0 && !stalled)
                    st.publish(tile, kFlagA, epoch, agg);
                prefix = lookBack<T>(st, tile, epoch, sh, hdr, errWord, timeoutNs);
            }
            if(threadIdx.x == 0 && !stalled)
                st.publish(tile, kFlagP, epoch, add(prefix, agg));
            T const off = add(prefix, warpPrefix);
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
            uint64_t const to = waitTimeoutNs();
            bool const vec = aligned16(in) && aligned16(out);
            dim3 const grid(static_cast<unsigned>(tiles));
#define A3B_SCAN_LAUNCH(INCL, VEC)                                                                                    \
    scanTileKernel<T, INCL, VEC><<<grid, kBlock, 0, s>>>(in, out, n, carry, hdr, epoch, props->errWord, to, stallTile)
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
