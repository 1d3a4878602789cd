// One-pass transform-reduce: onHost::transformReduce / onHost::reduce and the BabelStream dot.
//
// Replaces SimdTransformReduceKernel + its host driver (include/alpaka/onHost/algo/internal/transformReduce.hpp:23-202)
// and SimdTransformReduce::reduceSimdPackExecution (include/alpaka/onAcc/internal/SimdTransformReduce.hpp:359-499).
//
// Design (one launch, no pre-fill of `out`):
//   * the input is cut into chunks of 256 threads x ppt packs (ppt = 8 packs of 32 bytes, i.e. 64 KB, for large
//     inputs; fewer for small ones so that there are still ~2048 chunks) and block b reduces chunk b: a full grid of
//     short-lived blocks that the scheduler hands out in index order, so the GPU sweeps the input front to back. On
//     B200 this read 7.48 TB/s against 7.17-7.20 TB/s for a resident grid walking the input grid-stride;
//   * each thread keeps ppt independent accumulators (all its loads of a chunk are in flight together);
//   * fp32 inputs: the transformed elements of one pack are summed in fp32, the pack sum is added to an fp64
//     accumulator; fp64 inputs accumulate in fp64; integer + accumulates in 64-bit unsigned (wraps like the
//     reference's atomicAdd on the narrow type once truncated);
//   * warp butterfly (shfl_xor), then a block step through shared memory, gives one partial per block;
//   * two-level last-block-done: the last block of each group of 256 blocks (threadfence + atomic ticket) combines
//     the group's partials, one per thread, into a group partial; the last group combines the group partials and
//     writes out[0]. Every ticket is reset by the block that drew the last number, so the scratch is left ready for
//     the next call on the stream.
// The combination order depends only on n: repeated runs, and runs on GPUs with other SM counts, give identical bits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cfloat>
#include <climits>
#include <mutex>
#include <type_traits>

#include <map>
#include <set>
#include <utility>
#include <vector>

#include "common.cuh"

namespace a3b
{
    namespace
    {
        constexpr int kBlock = 256;
        constexpr int kWarps = kBlock / 32;
        constexpr int kMaxPpt = 8;                 // packs per thread per chunk, at most (16-byte packs)
        constexpr unsigned kGroup = kBlock;        // blocks per first-level group: one partial per thread
        constexpr uint64_t kMaxGrid = 1ull << 20;  // blocks; larger inputs (and capped grids) loop over chunks
        constexpr uint64_t kTargetChunks = 2048;   // smaller inputs get smaller chunks, down to ppt = 1
        constexpr unsigned kMaxGroups = static_cast<unsigned>(kMaxGrid / kGroup);

        // Packs per thread per chunk, at most: 128 bytes in flight per thread over all inputs (Σx²: 4 packs of 32
        // bytes; dot: 2 of each input), at most kMaxPpt; this keeps the kernels at 64 registers or fewer, 4 resident
        // blocks per SM.
        template<typename T, int W, int XOp>
        __host__ __device__ constexpr int maxPpt()
        {
            constexpr int bytes = W * static_cast<int>(sizeof(T)) * (XOp == A3B_XFORM_PRODUCT ? 2 : 1);
            return bytes >= 128 ? 1 : (128 / bytes < kMaxPpt ? 128 / bytes : kMaxPpt);
        }

        // Packs per thread per chunk for nPacks packs: the largest of maxPpt, ..., 2, 1 that still leaves
        // kTargetChunks chunks (a function of n alone, so the combination order does not depend on the device).
        inline int pptFor(uint64_t nPacks, int maxPpt)
        {
            int ppt = maxPpt;
            while(ppt > 1 && nPacks < kTargetChunks * kBlock * static_cast<uint64_t>(ppt))
                ppt /= 2;
            return ppt;
        }

        inline uint64_t chunksFor(uint64_t nPacks, int ppt)
        {
            uint64_t const chunk = static_cast<uint64_t>(kBlock) * static_cast<uint64_t>(ppt);
            return (nPacks + chunk - 1) / chunk;
        }

        // accumulator type
        template<typename T, int ROp>
        struct AccOf
        {
            using type = std::conditional_t<
                std::is_floating_point_v<T>,
                std::conditional_t<ROp == A3B_REDUCE_PLUS, double, T>,
                std::conditional_t<ROp == A3B_REDUCE_PLUS, uint64_t, T>>;
        };

        template<typename A, int ROp>
        __device__ __forceinline__ A combine(A x, A y)
        {
            if constexpr(ROp == A3B_REDUCE_PLUS)
            {
                if constexpr(std::is_same_v<A, double>)
                    return __dadd_rn(x, y);
                else
                    return x + y;
            }
            else if constexpr(ROp == A3B_REDUCE_MIN)
                return y < x ? y : x;
            else
                return y > x ? y : x;
        }

        template<int XOp, typename T>
        __device__ __forceinline__ T xform(T x, T y)
        {
            if constexpr(XOp == A3B_XFORM_IDENTITY)
                return x;
            else if constexpr(XOp == A3B_XFORM_SQUARE)
            {
                if constexpr(std::is_same_v<T, float>)
                    return __fmul_rn(x, x);
                else if constexpr(std::is_same_v<T, double>)
                    return __dmul_rn(x, x);
                else
                    return static_cast<T>(static_cast<std::make_unsigned_t<T>>(x) * static_cast<std::make_unsigned_t<T>>(x));
            }
            else
            {
                if constexpr(std::is_same_v<T, float>)
                    return __fmul_rn(x, y);
                else if constexpr(std::is_same_v<T, double>)
                    return __dmul_rn(x, y);
                else
                    return static_cast<T>(static_cast<std::make_unsigned_t<T>>(x) * static_cast<std::make_unsigned_t<T>>(y));
            }
        }

        // widen one transformed element into the accumulator type
        template<typename A, typename T>
        __device__ __forceinline__ A widen(T v)
        {
            if constexpr(std::is_same_v<A, uint64_t> && std::is_signed_v<T>)
                return static_cast<uint64_t>(static_cast<int64_t>(v));
            else
                return static_cast<A>(v);
        }

        template<typename T, int W>
        struct alignas(W * sizeof(T) >= 32 ? 32 : 16) Pack
        {
            T v[W];
        };

        // KEEP = false: evict-first (the data is read once). KEEP = true: normal L2 eviction, for a pass whose last
        // reads are read again right after it (the carry pass of a scan split across ranks).
        template<typename T, int W, bool KEEP = false>
        __device__ __forceinline__ Pack<T, W> loadPack(T const* base, uint64_t packIdx)
        {
            if constexpr(W * sizeof(T) == 32)
            {
                // 256-bit load (sm_100)
                unsigned long long r0, r1, r2, r3;
                if constexpr(KEEP)
                    asm volatile("ld.global.cg.v4.u64 {%0, %1, %2, %3}, [%4];"
                                 : "=l"(r0), "=l"(r1), "=l"(r2), "=l"(r3)
                                 : "l"(base + packIdx * W));
                else
                    asm volatile("ld.global.cs.v4.u64 {%0, %1, %2, %3}, [%4];"
                                 : "=l"(r0), "=l"(r1), "=l"(r2), "=l"(r3)
                                 : "l"(base + packIdx * W));
                unsigned long long raw[4] = {r0, r1, r2, r3};
                Pack<T, W> p;
                memcpy(&p, raw, 32);
                return p;
            }
            else if constexpr(W * sizeof(T) == 16)
            {
                uint4 raw = KEEP ? __ldcg(reinterpret_cast<uint4 const*>(base) + packIdx)
                                 : __ldcs(reinterpret_cast<uint4 const*>(base) + packIdx);
                return *reinterpret_cast<Pack<T, W>*>(&raw);
            }
            else
            {
                Pack<T, W> p;
#pragma unroll
                for(int k = 0; k < W; ++k)
                    p.v[k] = KEEP ? __ldcg(base + packIdx * W + k) : __ldcs(base + packIdx * W + k);
                return p;
            }
        }

        // fold one pack (already transformed element-wise) into an accumulator
        template<typename T, int W, int ROp, int XOp, typename A>
        __device__ __forceinline__ A foldPack(A acc, Pack<T, W> const& x, Pack<T, W> const& y)
        {
            if constexpr(std::is_same_v<T, float> && ROp == A3B_REDUCE_PLUS)
            {
                // fp32 pack sum (pairwise), then one fp64 add
                float t[W];
#pragma unroll
                for(int k = 0; k < W; ++k)
                    t[k] = xform<XOp>(x.v[k], y.v[k]);
#pragma unroll
                for(int w = 1; w < W; w *= 2)
#pragma unroll
                    for(int k = 0; k + w < W; k += 2 * w)
                        t[k] = __fadd_rn(t[k], t[k + w]);
                return __dadd_rn(acc, static_cast<double>(t[0]));
            }
            else
            {
#pragma unroll
                for(int k = 0; k < W; ++k)
                    acc = combine<A, ROp>(acc, widen<A>(xform<XOp>(x.v[k], y.v[k])));
                return acc;
            }
        }

        template<typename A>
        __device__ __forceinline__ A shflXor(A v, int m)
        {
            return __shfl_xor_sync(0xffffffffu, v, m);
        }

        template<typename A, int ROp>
        __device__ __forceinline__ A warpReduce(A v)
        {
#pragma unroll
            for(int m = 16; m > 0; m >>= 1)
                v = combine<A, ROp>(v, shflXor(v, m));
            return v;
        }

        template<typename A, int ROp>
        __device__ __forceinline__ A blockReduce(A v, A* smem)
        {
            v = warpReduce<A, ROp>(v);
            int const warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
            __syncthreads(); // smem may still be read by a previous blockReduce
            if(lane == 0)
                smem[warp] = v;
            __syncthreads();
            A r = smem[0];
#pragma unroll
            for(int w = 1; w < kWarps; ++w)
                r = combine<A, ROp>(r, smem[w]);
            return r;
        }

        // Scratch of one reduction: the final ticket, one ticket and one partial per group, one partial per block.
        // Tickets start at zero (fresh scratch is zero-filled) and are reset by the block that drew the last number.
        template<typename A>
        struct ReduceWork
        {
            unsigned* ticket;
            unsigned* groupTickets;
            A* groupPartials;
            A* partials;
        };

        inline size_t roundUp64(size_t b)
        {
            return (b + 63u) & ~size_t{63u};
        }

        // bytes of scratch for `grid` blocks with room for `maxGroups` groups
        template<typename A>
        size_t workBytes(unsigned maxGroups, uint64_t grid)
        {
            return 64u + roundUp64(sizeof(unsigned) * maxGroups) + roundUp64(sizeof(A) * maxGroups)
                   + sizeof(A) * static_cast<size_t>(grid);
        }

        // the layout at `base`: the tickets first (a caller that must clear them clears the first
        // 64 + roundUp64(4 * maxGroups) bytes), the partials after them
        template<typename A>
        ReduceWork<A> workAt(void* base, unsigned maxGroups)
        {
            auto* b = static_cast<unsigned char*>(base);
            ReduceWork<A> w;
            w.ticket = reinterpret_cast<unsigned*>(b);
            w.groupTickets = reinterpret_cast<unsigned*>(b + 64);
            size_t const off = 64u + roundUp64(sizeof(unsigned) * maxGroups);
            w.groupPartials = reinterpret_cast<A*>(b + off);
            w.partials = reinterpret_cast<A*>(b + off + roundUp64(sizeof(A) * maxGroups));
            return w;
        }

        // Hand-over of a stream's two scratch sets between early-started calls. Call e (numbered per stream by the
        // host) uses set e & 1. Its blocks write their partials only after the call that used the set before it
        // (e - 2) has published done[e & 1] >= e - 2, and its final block publishes done[e & 1] = e as soon as it no
        // longer touches the set -- before it waits for the previous call, so a waiting block never holds up the
        // call it waits for. Every earlier call's blocks have all started when a call's blocks run (each block lets
        // the next call launch from its first instruction), so the wait ends; it is bounded all the same.
        struct SetTurn
        {
            unsigned long long* done; // done word of this call's set
            unsigned long long epoch; // this call's number on the stream (from 1)
            unsigned* errWord;
            uint64_t timeoutNs;
        };

        // Thread 0 reads the done word with acquire semantics at the start of its block, before the block's pass over
        // the input (the read's latency hides under the other resident blocks' loads; every later access of the
        // thread, the scratch writes included, is ordered after it); after the pass it spins only when that early
        // value was too old. Measured on B200 against waiting for the previous call in every block: Σx² 2^30 fp32
        // unchanged (7.45 vs 7.43 TB/s), BabelStream dot 2^25 fp64 6.3 -> 7.4 TB/s (a short call no longer stalls
        // behind the previous call's combination); a fence after a relaxed early read instead cost Σx² 3-7%.
        __device__ __forceinline__ unsigned long long peekTurn(SetTurn const& t)
        {
            return ldAcquireU64(t.done);
        }

        __device__ __forceinline__ void waitTurn(SetTurn const& t, unsigned long long early)
        {
            if(t.epoch <= 2u || early >= t.epoch - 2u)
                return;
            uint64_t const t0 = globalTimerNs();
            while(ldAcquireU64(t.done) < t.epoch - 2u)
            {
                if(globalTimerNs() - t0 > t.timeoutNs)
                {
                    atomicOr(t.errWord, kErrTimeout);
                    return;
                }
                __nanosleep(32);
            }
        }

        // Finish: convert accumulator to the output element (or store the raw partial).
        template<typename T, typename A>
        __device__ __forceinline__ void writeResult(void* out, A r, bool rawPartial)
        {
            if(rawPartial)
            {
                // 8-byte partial: double for float types, 64-bit integer for integer types
                if constexpr(std::is_floating_point_v<T>)
                    *static_cast<double*>(out) = static_cast<double>(r);
                else if constexpr(std::is_signed_v<T>)
                    *static_cast<int64_t*>(out) = static_cast<int64_t>(r);
                else
                    *static_cast<uint64_t*>(out) = static_cast<uint64_t>(r);
            }
            else
            {
                if constexpr(std::is_same_v<A, uint64_t> && !std::is_same_v<T, uint64_t>)
                    *static_cast<T*>(out) = static_cast<T>(static_cast<std::make_unsigned_t<T>>(r));
                else
                    *static_cast<T*>(out) = static_cast<T>(r);
            }
        }

        // This block's partial (identical in every thread on return). Without LOOP the grid has one block per chunk
        // and block b reduces chunk b; with LOOP (grids capped below the chunk count) block b takes chunks b,
        // b + gridDim.x, ... A full chunk at ppt == U loads all its packs at once (compile-time count, no
        // predicates: the fewest registers); other chunks go pack by pack. PITCHED: rows of rowLen elements,
        // rowPitch bytes apart; packs never straddle rows (rowLen % W == 0).
        // REV: chunks in reverse order with normally cached loads, so the start of the input is read last and stays
        // in L2 for a pass that follows.
        template<typename T, int W, int ROp, int XOp, bool PITCHED, bool LOOP, bool REV = false>
        __device__ __forceinline__ typename AccOf<T, ROp>::type blockPartial(
            T const* __restrict__ in0,
            T const* __restrict__ in1,
            uint64_t n,
            uint64_t rowLen,
            uint64_t rowPitch,
            T neutral,
            int ppt,
            typename AccOf<T, ROp>::type* smem)
        {
            using A = typename AccOf<T, ROp>::type;
            constexpr int U = maxPpt<T, W, XOp>();
            A const neutralA = widen<A>(neutral);
            A acc[U];
#pragma unroll
            for(int u = 0; u < U; ++u)
                acc[u] = neutralA;

            uint64_t const nPacks = n / W;
            uint64_t const packsPerRow = rowLen / W;
            auto addr = [&](T const* base, uint64_t p) -> T const*
            {
                if constexpr(PITCHED)
                {
                    uint64_t const r = p / packsPerRow;
                    uint64_t const c = p - r * packsPerRow;
                    return reinterpret_cast<T const*>(reinterpret_cast<char const*>(base) + r * rowPitch) + c * W;
                }
                else
                    return base + p * W;
            };

            uint64_t const chunk = static_cast<uint64_t>(kBlock) * static_cast<uint64_t>(ppt);
            uint64_t const nChunks = (nPacks + chunk - 1) / chunk;
            auto reduceChunk = [&](uint64_t c)
            {
                uint64_t const first = c * chunk + threadIdx.x;
                if(ppt == U && c * chunk + chunk <= nPacks)
                {
                    Pack<T, W> x[U], y[U];
#pragma unroll
                    for(int u = 0; u < U; ++u)
                    {
                        uint64_t const p = first + static_cast<uint64_t>(u) * kBlock;
                        x[u] = loadPack<T, W, REV>(addr(in0, p), 0);
                        if constexpr(XOp == A3B_XFORM_PRODUCT)
                            y[u] = loadPack<T, W, REV>(addr(in1, p), 0);
                        else
                            y[u] = x[u];
                    }
#pragma unroll
                    for(int u = 0; u < U; ++u)
                        acc[u] = foldPack<T, W, ROp, XOp>(acc[u], x[u], y[u]);
                }
                else
                {
#pragma unroll
                    for(int u = 0; u < U; ++u)
                    {
                        uint64_t const p = first + static_cast<uint64_t>(u) * kBlock;
                        if(u < ppt && p < nPacks)
                        {
                            Pack<T, W> x = loadPack<T, W, REV>(addr(in0, p), 0);
                            Pack<T, W> y = x;
                            if constexpr(XOp == A3B_XFORM_PRODUCT)
                                y = loadPack<T, W, REV>(addr(in1, p), 0);
                            acc[u] = foldPack<T, W, ROp, XOp>(acc[u], x, y);
                        }
                    }
                }
            };
            if constexpr(LOOP)
            {
                for(uint64_t c = blockIdx.x; c < nChunks; c += gridDim.x)
                    reduceChunk(REV ? nChunks - 1 - c : c);
            }
            else if(blockIdx.x < nChunks)
                reduceChunk(REV ? nChunks - 1 - blockIdx.x : blockIdx.x);
            if constexpr(W > 1 && !PITCHED)
            {
                uint64_t const e = nPacks * W + static_cast<uint64_t>(blockIdx.x) * kBlock + threadIdx.x;
                if(e < n)
                {
                    T const x = in0[e];
                    T y = x;
                    if constexpr(XOp == A3B_XFORM_PRODUCT)
                        y = in1[e];
                    acc[0] = combine<A, ROp>(acc[0], widen<A>(xform<XOp>(x, y)));
                }
            }

            A v = acc[0];
#pragma unroll
            for(int u = 1; u < U; ++u)
                v = combine<A, ROp>(v, acc[u]);
            v = blockReduce<A, ROp>(v, smem);
            return v;
        }

        // Two-level last-block-done combination of the block partials `v` (identical in every thread). Returns true
        // in every thread of the one block that finishes last, with the grid's total in *total; false elsewhere.
        template<typename A, int ROp>
        __device__ __forceinline__ bool combineGrid(A v, A neutralA, ReduceWork<A> const& w, A* smem, bool* flag, A* total)
        {
            unsigned const g = blockIdx.x / kGroup;
            unsigned const nGroups = (gridDim.x + kGroup - 1) / kGroup;
            unsigned const inGroup = min(kGroup, gridDim.x - g * kGroup);
            if(threadIdx.x == 0)
            {
                w.partials[blockIdx.x] = v;
                __threadfence();
                *flag = atomicAdd(w.groupTickets + g, 1u) == inGroup - 1u;
            }
            __syncthreads();
            if(!*flag)
                return false;
            __threadfence();
            // the group's partials, one per thread, in block order
            A r = threadIdx.x < inGroup ? __ldcg(w.partials + g * kGroup + threadIdx.x) : neutralA;
            r = blockReduce<A, ROp>(r, smem); // its barriers order every thread's read of *flag before the next write
            if(nGroups == 1u)
            {
                if(threadIdx.x == 0)
                    w.groupTickets[g] = 0u;
                *total = r;
                return true;
            }
            if(threadIdx.x == 0)
            {
                w.groupTickets[g] = 0u;
                w.groupPartials[g] = r;
                __threadfence();
                *flag = atomicAdd(w.ticket, 1u) == nGroups - 1u;
            }
            __syncthreads();
            if(!*flag)
                return false;
            __threadfence();
            A t = neutralA;
            for(unsigned k = threadIdx.x; k < nGroups; k += kBlock)
                t = combine<A, ROp>(t, __ldcg(w.groupPartials + k));
            t = blockReduce<A, ROp>(t, smem);
            if(threadIdx.x == 0)
                *w.ticket = 0u;
            *total = t;
            return true;
        }

        // PDL: the kernel overlaps the previous kernel of its stream (launched with programmatic stream
        // serialisation): every block lets the next call launch from its first instruction; the blocks write their
        // partials into this call's scratch set once the call two before has released it (SetTurn), and only the
        // final block waits for the previous call to complete (griddepcontrol.wait) before it writes `out`. So the
        // blocks of consecutive calls stream their inputs back to back; the inputs themselves are guarded on the host
        // (earlyStartAllowed).
        template<typename T, int W, int ROp, int XOp, bool PITCHED, bool LOOP, bool PDL>
        __global__ void __launch_bounds__(kBlock) reduceKernel(
            T const* __restrict__ in0,
            T const* __restrict__ in1,
            uint64_t n,
            uint64_t rowLen,
            uint64_t rowPitch,
            T neutral,
            int ppt,
            void* out,
            bool rawPartial,
            ReduceWork<typename AccOf<T, ROp>::type> work,
            SetTurn turn)
        {
            using A = typename AccOf<T, ROp>::type;
            __shared__ A smem[kWarps];
            __shared__ bool flag;
            unsigned long long early = 0;
            if constexpr(PDL)
            {
                if(threadIdx.x == 0)
                {
                    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
                    early = peekTurn(turn);
                }
            }
            A const v = blockPartial<T, W, ROp, XOp, PITCHED, LOOP>(in0, in1, n, rowLen, rowPitch, neutral, ppt, smem);
            if constexpr(PDL)
            {
                if(threadIdx.x == 0)
                    waitTurn(turn, early); // the call two before this one is done with this call's scratch set
            }
            A total;
            if(!combineGrid<A, ROp>(v, widen<A>(neutral), work, smem, &flag, &total))
                return;
            if constexpr(PDL)
            {
                __syncthreads();
                if(threadIdx.x == 0)
                    stReleaseU64(turn.done, turn.epoch); // the set is free for the call after next
                asm volatile("griddepcontrol.wait;" ::: "memory"); // the previous call has completed: write `out`
            }
            if(threadIdx.x == 0)
                writeResult<T, A>(out, total, rawPartial);
        }

        // The early start is opt-in per (device, stream) (a3b_set_early_start): a reduction launched with it reads its
        // input before griddepcontrol.wait, so a kernel just before it on the stream that signals its dependents early
        // (griddepcontrol.launch_dependents) could still be writing that input. The caller who enables it asserts that
        // no kernel on the stream does so; everything else is launched fully ordered.
        //
        // Outputs of the reductions launched with the early start on each (device, stream) since the last one launched
        // fully ordered. Such a call may still be running while a later call of the stream reads its input (that read
        // comes before the later call's griddepcontrol.wait). A call whose input overlaps one of these outputs, or a
        // history grown past kMaxEarly entries, is launched fully ordered, which also clears the history: a plain
        // launch starts only after all earlier work of the stream has completed.
        constexpr size_t kMaxEarly = 64;
        std::mutex gEarlyMutex;
        std::set<std::pair<int, cudaStream_t>> gEarlyEnabled;
        std::map<std::pair<int, cudaStream_t>, std::vector<std::pair<uintptr_t, uintptr_t>>> gEarlyOutputs;

        void setEarlyStart(int dev, cudaStream_t s, bool enable)
        {
            std::lock_guard<std::mutex> lock(gEarlyMutex);
            auto const key = std::make_pair(dev, s);
            if(enable)
                gEarlyEnabled.insert(key);
            else
            {
                gEarlyEnabled.erase(key);
                gEarlyOutputs.erase(key);
            }
        }

        // true: launch with the early start; in both cases `out` (8 bytes) joins the stream's history
        bool earlyStartAllowed(int dev, cudaStream_t s, void const* in0, void const* in1, uint64_t inBytes, void* out)
        {
            std::lock_guard<std::mutex> lock(gEarlyMutex);
            auto const key = std::make_pair(dev, s);
            if(!gEarlyEnabled.count(key))
            {
                gEarlyOutputs.erase(key); // fully ordered launches only: nothing can still run when the next call starts
                return false;
            }
            auto& h = gEarlyOutputs[key];
            auto hit = [&](void const* p)
            {
                if(!p)
                    return false;
                auto const a = reinterpret_cast<uintptr_t>(p);
                for(auto const& r : h)
                    if(a < r.second && r.first < a + inBytes)
                        return true;
                return false;
            };
            bool const early = !(hit(in0) || hit(in1)) && h.size() < kMaxEarly;
            if(!early)
                h.clear();
            auto const o = reinterpret_cast<uintptr_t>(out);
            bool known = false;
            for(auto const& r : h)
                known = known || (r.first == o && r.second == o + 8u);
            if(!known)
                h.emplace_back(o, o + 8u);
            return early;
        }

        // The reduction scratch of a (device, stream): a 256-byte header holding the two sets' done words, then two
        // sets of `stride` bytes (SetTurn). The stride grows to the largest set any call on the stream has needed;
        // a new stride or a new buffer clears the whole scratch in stream order (an early start never crosses a
        // memset) and restarts the call numbering.
        struct StreamTurns
        {
            void* base = nullptr;
            size_t stride = 0;
            unsigned long long epoch = 0;
        };
        std::mutex gTurnMutex;
        std::map<std::pair<int, cudaStream_t>, StreamTurns> gTurns;

        template<typename A>
        int reduceScratch(cudaStream_t s, DeviceProps const* props, uint64_t grid, ReduceWork<A>* work, SetTurn* turn)
        {
            size_t const need = (workBytes<A>(kMaxGroups, grid) + 255u) & ~size_t{255u};
            std::lock_guard<std::mutex> lock(gTurnMutex);
            StreamTurns& t = gTurns[std::make_pair(props->ordinal, s)];
            bool reset = false;
            if(need > t.stride)
            {
                t.stride = need;
                reset = true;
            }
            void* scr = nullptr;
            int const rc = streamScratch(s, kScratchReduce, 256u + 2u * t.stride, &scr);
            if(rc)
                return rc;
            if(scr != t.base)
            {
                t.base = scr;
                reset = true;
            }
            if(reset)
            {
                A3B_CUDA(cudaMemsetAsync(scr, 0, 256u + 2u * t.stride, s));
                t.epoch = 0;
            }
            unsigned long long const e = ++t.epoch;
            auto* base = static_cast<unsigned char*>(scr);
            *work = workAt<A>(base + 256u + static_cast<size_t>(e & 1u) * t.stride, kMaxGroups);
            turn->done = reinterpret_cast<unsigned long long*>(base) + (e & 1u);
            turn->epoch = e;
            turn->errWord = props->errWord;
            turn->timeoutNs = waitTimeoutNs();
            return A3B_OK;
        }

        // ---------------------------------------------------------------- fused with the all-reduce over peers
        __device__ __forceinline__ void stRelaxedSys(unsigned long long* p, unsigned long long v)
        {
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
        }

        __device__ __forceinline__ unsigned long long ldAcquireSys(unsigned long long const* p)
        {
            unsigned long long v;
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
            return v;
        }

        __device__ __forceinline__ unsigned long long ldRelaxedSys(unsigned long long const* p)
        {
            unsigned long long v;
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
            return v;
        }

        // peers.slots[q] for a run-time q without indexing the parameter array (a dynamic index would copy the
        // whole struct to a per-thread stack frame in every block)
        __device__ __forceinline__ unsigned long long* slotOf(PeerSlots const& peers, int q)
        {
            unsigned long long* r = peers.slots[0];
#pragma unroll
            for(int k = 1; k < kMaxPeers; ++k)
                if(q == k)
                    r = peers.slots[k];
            return r;
        }

        // Local reduction as reduceKernel; the last block then stores the unrounded local total into slot
        // [epoch parity][rank] of every rank's slot buffer (value, then the epoch with release semantics), waits for
        // the world's values in its own buffer and combines them in rank order: every rank computes the same bits.
        // With lowerRanksOnly the combination covers ranks 0 .. rank-1 (the carry of a scan split across ranks); the
        // wait still covers every rank, so one call's slots are never overwritten by the next call too early.
        //
        // Consecutive calls on a stream overlap (programmatic dependent launch, a3b_set_early_start): every block lets
        // the next call's kernel launch as soon as it has started, writes its partial into this call's scratch set
        // once the call two before has released it (SetTurn), and only the final block waits for the previous call's
        // kernel to complete before it touches the slots or `out` (a call whose input may have been written by a call
        // still in flight is launched fully ordered: earlyStartAllowed). The next call's HBM pass thus runs while this
        // call combines and waits for the other ranks. A call reaches its exchange only after the previous call has
        // completed, so the exchanges of two calls never overlap and two slot parities suffice.
        template<typename T, int W, int ROp, int XOp, bool LOOP, bool REV>
        __global__ void __launch_bounds__(kBlock) reduceAllRanksKernel(
            T const* __restrict__ in0,
            T const* __restrict__ in1,
            uint64_t n,
            T neutral,
            int ppt,
            void* out,
            ReduceWork<typename AccOf<T, ROp>::type> work,
            PeerSlots peers,
            bool lowerRanksOnly,
            unsigned* errWord,
            uint64_t timeoutNs,
            SetTurn turn)
        {
            using A = typename AccOf<T, ROp>::type;
            __shared__ A smem[kWarps];
            __shared__ bool flag;
            unsigned long long early = 0;
            if(threadIdx.x == 0)
            {
                asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
                early = peekTurn(turn);
            }
            A const neutralA = widen<A>(neutral);
            A const v = blockPartial<T, W, ROp, XOp, false, LOOP, REV>(in0, in1, n, n, 0, neutral, ppt, smem);
            if(threadIdx.x == 0)
                waitTurn(turn, early); // the call two before this one is done with this call's scratch set
            A r;
            if(!combineGrid<A, ROp>(v, neutralA, work, smem, &flag, &r))
                return;
            __syncthreads();
            if(threadIdx.x == 0)
                stReleaseU64(turn.done, turn.epoch); // the set is free for the call after next
            // the previous call on this stream has completed: its exchange is over, the slots and `out` may be used
            asm volatile("griddepcontrol.wait;" ::: "memory");
            if(threadIdx.x >= 32)
                return;
            // warp 0: lane q exchanges with rank q (all ranks in parallel, one system-scope fence per lane)
            int const lane = threadIdx.x;
            static_assert(sizeof(A) <= 8, "partials are exchanged as 8-byte words");
            unsigned long long bits = 0;
            memcpy(&bits, &r, sizeof(A));
            unsigned const par = peers.epoch & 1u;
            bool const active = lane < peers.world;
            if(active)
            {
                unsigned long long* slot = slotOf(peers, lane) + 2 * (par * kMaxPeers + peers.rank);
                stRelaxedSys(slot, bits);
                __threadfence_system(); // the value is visible to rank `lane` before the epoch that announces it
                stRelaxedSys(slot + 1, peers.epoch);
            }
            bool ok = true;
            unsigned long long vb = 0;
            if(active)
            {
                unsigned long long const* slot = slotOf(peers, peers.rank) + 2 * (par * kMaxPeers + lane);
                uint64_t const t0 = globalTimerNs();
                while(ldAcquireSys(slot + 1) != peers.epoch)
                {
                    if(globalTimerNs() - t0 > timeoutNs)
                    {
                        ok = false;
                        break;
                    }
                    __nanosleep(20);
                }
                if(ok)
                    vb = ldRelaxedSys(slot);
            }
            bool const allOk = __all_sync(0xffffffffu, ok);
            // combine in rank order on lane 0: every rank gets the same bits
            A total = neutralA;
            for(int q = 0; q < peers.world; ++q)
            {
                unsigned long long const w = __shfl_sync(0xffffffffu, vb, q);
                if(!lowerRanksOnly || q < peers.rank)
                {
                    A val;
                    memcpy(&val, &w, sizeof(A));
                    total = combine<A, ROp>(total, val);
                }
            }
            if(lane != 0)
                return;
            if(!allOk)
                atomicOr(errWord, kErrTimeout);
            writeResult<T, A>(out, total, false);
        }

        template<typename T, int W, int ROp, int XOp>
        int launchAllRanks(cudaStream_t s, a3b_peer_group* g, T const* in0, T const* in1, uint64_t n, T neutral, void* out,
                           bool lower)
        {
            using A = typename AccOf<T, ROp>::type;
            DeviceProps const* props = nullptr;
            int rc = currentDevice(&props);
            if(rc)
                return rc;
            int const ppt = pptFor(n / W, maxPpt<T, W, XOp>());
            uint64_t const chunks = chunksFor(n / W, ppt);
            bool const loop = chunks > kMaxGrid;
            uint64_t const grid = loop ? kMaxGrid : (chunks > 0 ? chunks : 1);
            ReduceWork<A> w;
            SetTurn turn;
            rc = reduceScratch<A>(s, props, grid, &w, &turn);
            if(rc)
                return rc;
            PeerSlots peers;
            rc = peerSlots(g, &peers);
            if(rc)
                return rc;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(static_cast<unsigned>(grid));
            cfg.blockDim = dim3(kBlock);
            cfg.dynamicSmemBytes = 0;
            cfg.stream = s;
            cfg.attrs = attr;
            cfg.numAttrs = earlyStartAllowed(props->ordinal, s, in0, in1, n * sizeof(T), out) ? 1 : 0;
            uint64_t const to = waitTimeoutNs();
            // the carry of a scan split across ranks (plain sums, lower ranks only) walks its shard back to front with
            // normally cached loads, so the shard's first tiles are still in L2 when the carried scan starts reading
            // them (carry + scan measured 1-2% faster at 2^27 int32 and 2^25 uint64 per rank)
            if constexpr(ROp == A3B_REDUCE_PLUS && XOp == A3B_XFORM_IDENTITY)
            {
                if(lower)
                {
                    if(loop)
                        A3B_CUDA(cudaLaunchKernelEx(&cfg, reduceAllRanksKernel<T, W, ROp, XOp, true, true>, in0, in1, n,
                                                    neutral, ppt, out, w, peers, lower, props->errWord, to, turn));
                    else
                        A3B_CUDA(cudaLaunchKernelEx(&cfg, reduceAllRanksKernel<T, W, ROp, XOp, false, true>, in0, in1, n,
                                                    neutral, ppt, out, w, peers, lower, props->errWord, to, turn));
                    return A3B_OK;
                }
            }
            if(loop)
                A3B_CUDA(cudaLaunchKernelEx(&cfg, reduceAllRanksKernel<T, W, ROp, XOp, true, false>, in0, in1, n, neutral,
                                            ppt, out, w, peers, lower, props->errWord, to, turn));
            else
                A3B_CUDA(cudaLaunchKernelEx(&cfg, reduceAllRanksKernel<T, W, ROp, XOp, false, false>, in0, in1, n,
                                            neutral, ppt, out, w, peers, lower, props->errWord, to, turn));
            return A3B_OK;
        }

        template<typename T, int ROp, int XOp>
        int allRanksLayout(cudaStream_t s, a3b_peer_group* g, T const* in0, T const* in1, uint64_t n, T neutral, void* out,
                           bool lower)
        {
            auto al = [&](uintptr_t a)
            {
                auto ok = [&](void const* p) { return (reinterpret_cast<uintptr_t>(p) & (a - 1u)) == 0u; };
                return ok(in0) && (XOp != A3B_XFORM_PRODUCT || ok(in1));
            };
            constexpr int W = 16 / sizeof(T);
            if(al(32))
                return launchAllRanks<T, 2 * W, ROp, XOp>(s, g, in0, in1, n, neutral, out, lower);
            if(al(16))
                return launchAllRanks<T, W, ROp, XOp>(s, g, in0, in1, n, neutral, out, lower);
            return launchAllRanks<T, 1, ROp, XOp>(s, g, in0, in1, n, neutral, out, lower);
        }

        template<typename T, int ROp>
        int allRanksXform(cudaStream_t s, a3b_peer_group* g, int xop, T const* in0, T const* in1, uint64_t n, T neutral, void* out,
                          bool lower)
        {
            switch(xop)
            {
            case A3B_XFORM_IDENTITY:
                return allRanksLayout<T, ROp, A3B_XFORM_IDENTITY>(s, g, in0, in1, n, neutral, out, lower);
            case A3B_XFORM_SQUARE:
                return allRanksLayout<T, ROp, A3B_XFORM_SQUARE>(s, g, in0, in1, n, neutral, out, lower);
            case A3B_XFORM_PRODUCT:
                A3B_REQUIRE(in1, "product transform needs two inputs");
                return allRanksLayout<T, ROp, A3B_XFORM_PRODUCT>(s, g, in0, in1, n, neutral, out, lower);
            default:
                setError("unknown transform op %d", xop);
                return A3B_ERR_INVALID;
            }
        }

        template<typename T>
        int allRanksReduce(cudaStream_t s, a3b_peer_group* g, int rop, int xop, void const* in0, void const* in1, uint64_t n,
                           void const* neutral, void* out, bool lower = false)
        {
            T const nv = *static_cast<T const*>(neutral);
            auto i0 = static_cast<T const*>(in0);
            auto i1 = static_cast<T const*>(in1);
            switch(rop)
            {
            case A3B_REDUCE_PLUS:
                return allRanksXform<T, A3B_REDUCE_PLUS>(s, g, xop, i0, i1, n, nv, out, lower);
            case A3B_REDUCE_MIN:
                return allRanksXform<T, A3B_REDUCE_MIN>(s, g, xop, i0, i1, n, nv, out, lower);
            case A3B_REDUCE_MAX:
                return allRanksXform<T, A3B_REDUCE_MAX>(s, g, xop, i0, i1, n, nv, out, lower);
            default:
                setError("unknown reduce op %d", rop);
                return A3B_ERR_INVALID;
            }
        }


        template<typename T, int W, int ROp, int XOp, bool PITCHED>
        int launchReduce(
            cudaStream_t s,
            T const* in0,
            T const* in1,
            uint64_t n,
            uint64_t rowLen,
            uint64_t rowPitch,
            T neutral,
            void* out,
            bool raw)
        {
            using A = typename AccOf<T, ROp>::type;
            DeviceProps const* props = nullptr;
            int rc = currentDevice(&props);
            if(rc)
                return rc;
            int const ppt = pptFor(n / W, maxPpt<T, W, XOp>());
            uint64_t const chunks = chunksFor(n / W, ppt);
            bool const loop = chunks > kMaxGrid;
            uint64_t const grid = loop ? kMaxGrid : (chunks > 0 ? chunks : 1);
            ReduceWork<A> w;
            SetTurn turn;
            rc = reduceScratch<A>(s, props, grid, &w, &turn);
            if(rc)
                return rc;
            uint64_t const rows = PITCHED ? (n + rowLen - 1) / rowLen : 1u;
            uint64_t const inBytes = PITCHED ? rows * rowPitch : n * sizeof(T);
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(static_cast<unsigned>(grid));
            cfg.blockDim = dim3(kBlock);
            cfg.stream = s;
            cfg.attrs = attr;
            cfg.numAttrs = earlyStartAllowed(props->ordinal, s, in0, in1, inBytes, out) ? 1 : 0;
            if(loop)
                A3B_CUDA(cudaLaunchKernelEx(&cfg, reduceKernel<T, W, ROp, XOp, PITCHED, true, true>, in0, in1, n, rowLen,
                                            rowPitch, neutral, ppt, out, raw, w, turn));
            else
                A3B_CUDA(cudaLaunchKernelEx(&cfg, reduceKernel<T, W, ROp, XOp, PITCHED, false, true>, in0, in1, n, rowLen,
                                            rowPitch, neutral, ppt, out, raw, w, turn));
            return A3B_OK;
        }

        template<typename T, int ROp, int XOp>
        int dispatchLayout(
            cudaStream_t s,
            T const* in0,
            T const* in1,
            uint64_t rows,
            uint64_t rowLen,
            uint64_t rowPitch,
            T neutral,
            void* out,
            bool raw)
        {
            constexpr int W = 16 / sizeof(T);
            bool const dense = rows <= 1 || rowPitch == rowLen * sizeof(T);
            bool const al = aligned16(in0) && (XOp != A3B_XFORM_PRODUCT || aligned16(in1));
            auto a32 = [](void const* p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0u; };
            bool const al32 = a32(in0) && (XOp != A3B_XFORM_PRODUCT || a32(in1));
            uint64_t const n = rows * rowLen;
            if(dense)
            {
                if(al32)
                    return launchReduce<T, 2 * W, ROp, XOp, false>(s, in0, in1, n, n, 0, neutral, out, raw);
                if(al)
                    return launchReduce<T, W, ROp, XOp, false>(s, in0, in1, n, n, 0, neutral, out, raw);
                return launchReduce<T, 1, ROp, XOp, false>(s, in0, in1, n, n, 0, neutral, out, raw);
            }
            if constexpr(XOp != A3B_XFORM_PRODUCT)
            {
                if(al && rowLen % W == 0 && rowPitch % 16 == 0)
                    return launchReduce<T, W, ROp, XOp, true>(s, in0, in1, n, rowLen, rowPitch, neutral, out, raw);
                return launchReduce<T, 1, ROp, XOp, true>(s, in0, in1, n, rowLen, rowPitch, neutral, out, raw);
            }
            setError("pitched layout is supported for single-input reductions only");
            return A3B_ERR_INVALID;
        }

        template<typename T, int ROp>
        int dispatchXform(
            cudaStream_t s,
            int xop,
            T const* in0,
            T const* in1,
            uint64_t rows,
            uint64_t rowLen,
            uint64_t pitch,
            T neutral,
            void* out,
            bool raw)
        {
            switch(xop)
            {
            case A3B_XFORM_IDENTITY:
                return dispatchLayout<T, ROp, A3B_XFORM_IDENTITY>(s, in0, in1, rows, rowLen, pitch, neutral, out, raw);
            case A3B_XFORM_SQUARE:
                return dispatchLayout<T, ROp, A3B_XFORM_SQUARE>(s, in0, in1, rows, rowLen, pitch, neutral, out, raw);
            case A3B_XFORM_PRODUCT:
                A3B_REQUIRE(in1, "product transform needs two inputs");
                return dispatchLayout<T, ROp, A3B_XFORM_PRODUCT>(s, in0, in1, rows, rowLen, pitch, neutral, out, raw);
            default:
                setError("unknown transform op %d", xop);
                return A3B_ERR_INVALID;
            }
        }

        template<typename T>
        int dispatchReduce(
            cudaStream_t s,
            int rop,
            int xop,
            void const* in0,
            void const* in1,
            uint64_t rows,
            uint64_t rowLen,
            uint64_t pitch,
            void const* neutral,
            void* out,
            bool raw)
        {
            T const nv = *static_cast<T const*>(neutral);
            auto i0 = static_cast<T const*>(in0);
            auto i1 = static_cast<T const*>(in1);
            switch(rop)
            {
            case A3B_REDUCE_PLUS:
                return dispatchXform<T, A3B_REDUCE_PLUS>(s, xop, i0, i1, rows, rowLen, pitch, nv, out, raw);
            case A3B_REDUCE_MIN:
                return dispatchXform<T, A3B_REDUCE_MIN>(s, xop, i0, i1, rows, rowLen, pitch, nv, out, raw);
            case A3B_REDUCE_MAX:
                return dispatchXform<T, A3B_REDUCE_MAX>(s, xop, i0, i1, rows, rowLen, pitch, nv, out, raw);
            default:
                setError("unknown reduce op %d", rop);
                return A3B_ERR_INVALID;
            }
        }

        int reduceEntry(
            a3b_stream_t stream,
            int dtype,
            int rop,
            int xop,
            void const* in0,
            void const* in1,
            uint64_t rows,
            uint64_t rowLen,
            uint64_t pitch,
            void const* neutral,
            void* out,
            bool raw)
        {
            A3B_REQUIRE(out && neutral, "null out/neutral");
            A3B_REQUIRE(in0 || rows * rowLen == 0, "null input");
            auto s = static_cast<cudaStream_t>(stream);
            switch(dtype)
            {
            case A3B_I32:
                return dispatchReduce<int32_t>(s, rop, xop, in0, in1, rows, rowLen, pitch, neutral, out, raw);
            case A3B_U32:
                return dispatchReduce<uint32_t>(s, rop, xop, in0, in1, rows, rowLen, pitch, neutral, out, raw);
            case A3B_I64:
                return dispatchReduce<int64_t>(s, rop, xop, in0, in1, rows, rowLen, pitch, neutral, out, raw);
            case A3B_U64:
                return dispatchReduce<uint64_t>(s, rop, xop, in0, in1, rows, rowLen, pitch, neutral, out, raw);
            case A3B_F32:
                return dispatchReduce<float>(s, rop, xop, in0, in1, rows, rowLen, pitch, neutral, out, raw);
            case A3B_F64:
                return dispatchReduce<double>(s, rop, xop, in0, in1, rows, rowLen, pitch, neutral, out, raw);
            default:
                setError("unknown dtype %d", dtype);
                return A3B_ERR_INVALID;
            }
        }
    } // namespace
} // namespace a3b

namespace a3b
{
    namespace
    {
        // ------------------------------------------------------------------------------------------------------
        // Variant for callers that cannot allocate device memory: processes whose device memory is owned by another
        // allocator's pool (a framework that reserves the GPU's memory up front), services that must keep a fixed,
        // accounted memory footprint, and latency-critical loops that cannot afford an allocation's implicit
        // synchronisation. Its scratch (ticket header + one 8-byte partial per block) lives in this fixed static
        // array, which every device that loads the library holds until the process exits.
        constexpr size_t kNoAllocScratchBytes = 16384; // tickets for 8 groups + 8 group partials + 2024 partials
        constexpr unsigned kNoAllocGroups = 8;
        __device__ __align__(256) unsigned char g_noAllocScratch[kNoAllocScratchBytes];

        std::mutex gNoAllocMutex;
        struct NoAllocSlot
        {
            void* address;            // device address of g_noAllocScratch in the context below
            unsigned long long ctxId; // driver id of the context that address belongs to (0: unknown)
        };
        NoAllocSlot gNoAllocSlots[64] = {};

        // Driver id of the context current on this thread, 0 if there is none or it cannot be read. Context ids are
        // unique for the life of the process, so a context re-created after cudaDeviceReset gets a new one.
        unsigned long long currentContextId()
        {
            static PFN_cuCtxGetCurrent getCurrent = nullptr;
            static PFN_cuCtxGetId getId = nullptr;
            static std::once_flag once;
            std::call_once(
                once,
                []
                {
                    cudaDriverEntryPointQueryResult q{};
                    if(cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", reinterpret_cast<void**>(&getCurrent), 4000,
                                                        cudaEnableDefault, &q)
                           != cudaSuccess
                       || q != cudaDriverEntryPointSuccess)
                        getCurrent = nullptr;
                    if(cudaGetDriverEntryPointByVersion("cuCtxGetId", reinterpret_cast<void**>(&getId), 12000,
                                                        cudaEnableDefault, &q)
                           != cudaSuccess
                       || q != cudaDriverEntryPointSuccess)
                        getId = nullptr;
                });
            CUcontext ctx = nullptr;
            unsigned long long id = 0;
            if(!getCurrent || !getId || getCurrent(&ctx) != CUDA_SUCCESS || !ctx || getId(ctx, &id) != CUDA_SUCCESS)
                return 0;
            return id;
        }

        // Device address of the static scratch for the current device. The array's name is a host-side stand-in,
        // not a device address, so it is resolved with cudaGetSymbolAddress once per device and context: on the
        // first call on a device, and again when the device's context has been re-created (cudaDeviceReset unloads
        // the module, so the array may sit at another address afterwards). Those calls must not happen inside a
        // stream capture.
        int noAllocScratch(void** ptr)
        {
            int dev = 0;
            A3B_CUDA(cudaGetDevice(&dev));
            A3B_REQUIRE(dev >= 0 && dev < 64, "device ordinal out of range");
            std::lock_guard<std::mutex> lock(gNoAllocMutex);
            NoAllocSlot& slot = gNoAllocSlots[dev];
            unsigned long long const ctx = currentContextId();
            if(!slot.address || ctx == 0 || ctx != slot.ctxId)
            {
                void* a = nullptr;
                cudaError_t const e = cudaGetSymbolAddress(&a, g_noAllocScratch);
                if(e != cudaSuccess)
                    return cudaFail(e, "cudaGetSymbolAddress(no-allocation scratch)");
                slot.address = a;
                slot.ctxId = currentContextId(); // the lookup has made the device's context current
            }
            *ptr = slot.address;
            return A3B_OK;
        }

        template<typename T, int W, int ROp, int XOp>
        int launchReduceNoAlloc(cudaStream_t s, T const* in0, T const* in1, uint64_t n, T neutral, void* out)
        {
            using A = typename AccOf<T, ROp>::type;
            DeviceProps const* props = nullptr;
            int rc = currentDevice(&props);
            if(rc)
                return rc;
            // as many blocks as the array has room for partials; larger inputs give each block several chunks
            size_t const fixed = workBytes<A>(kNoAllocGroups, 0);
            uint64_t const room = (kNoAllocScratchBytes - fixed) / sizeof(A);
            uint64_t const cap = room < uint64_t{kNoAllocGroups} * kGroup ? room : uint64_t{kNoAllocGroups} * kGroup;
            int const ppt = pptFor(n / W, maxPpt<T, W, XOp>());
            uint64_t const chunks = chunksFor(n / W, ppt);
            uint64_t const grid = chunks < cap ? (chunks > 0 ? chunks : 1) : cap;
            size_t const need = workBytes<A>(kNoAllocGroups, grid);
            if(need > kNoAllocScratchBytes)
            {
                setError("a3b_transform_reduce_noalloc needs %zu bytes of scratch for %llu blocks, more than its fixed "
                         "%zu-byte static array",
                         need, static_cast<unsigned long long>(grid), kNoAllocScratchBytes);
                return A3B_ERR_TOO_LARGE;
            }
            void* scr = nullptr;
            rc = noAllocScratch(&scr);
            if(rc)
                return rc;
            // the array keeps the previous call's contents: the tickets must start at zero
            A3B_CUDA(cudaMemsetAsync(scr, 0, 64u + roundUp64(sizeof(unsigned) * kNoAllocGroups), s));
            reduceKernel<T, W, ROp, XOp, false, true, false><<<static_cast<unsigned>(grid), kBlock, 0, s>>>(
                in0, in1, n, n, 0, neutral, ppt, out, false, workAt<A>(scr, kNoAllocGroups), SetTurn{});
            A3B_CHECK_LAUNCH("transform_reduce_noalloc launch");
            return A3B_OK;
        }

        template<typename T, int ROp, int XOp>
        int noAllocLayout(cudaStream_t s, T const* in0, T const* in1, uint64_t n, T neutral, void* out)
        {
            auto al = [&](uintptr_t a)
            {
                auto ok = [&](void const* p) { return (reinterpret_cast<uintptr_t>(p) & (a - 1u)) == 0u; };
                return ok(in0) && (XOp != A3B_XFORM_PRODUCT || ok(in1));
            };
            constexpr int W = 16 / sizeof(T);
            if(al(32))
                return launchReduceNoAlloc<T, 2 * W, ROp, XOp>(s, in0, in1, n, neutral, out);
            if(al(16))
                return launchReduceNoAlloc<T, W, ROp, XOp>(s, in0, in1, n, neutral, out);
            return launchReduceNoAlloc<T, 1, ROp, XOp>(s, in0, in1, n, neutral, out);
        }

        template<typename T, int ROp>
        int noAllocXform(cudaStream_t s, int xop, T const* in0, T const* in1, uint64_t n, T neutral, void* out)
        {
            switch(xop)
            {
            case A3B_XFORM_IDENTITY:
                return noAllocLayout<T, ROp, A3B_XFORM_IDENTITY>(s, in0, in1, n, neutral, out);
            case A3B_XFORM_SQUARE:
                return noAllocLayout<T, ROp, A3B_XFORM_SQUARE>(s, in0, in1, n, neutral, out);
            case A3B_XFORM_PRODUCT:
                A3B_REQUIRE(in1, "product transform needs two inputs");
                return noAllocLayout<T, ROp, A3B_XFORM_PRODUCT>(s, in0, in1, n, neutral, out);
            default:
                setError("unknown transform op %d", xop);
                return A3B_ERR_INVALID;
            }
        }

        template<typename T>
        int noAllocReduce(cudaStream_t s, int rop, int xop, void const* in0, void const* in1, uint64_t n,
                          void const* neutral, void* out)
        {
            T const nv = *static_cast<T const*>(neutral);
            auto i0 = static_cast<T const*>(in0);
            auto i1 = static_cast<T const*>(in1);
            switch(rop)
            {
            case A3B_REDUCE_PLUS:
                return noAllocXform<T, A3B_REDUCE_PLUS>(s, xop, i0, i1, n, nv, out);
            case A3B_REDUCE_MIN:
                return noAllocXform<T, A3B_REDUCE_MIN>(s, xop, i0, i1, n, nv, out);
            case A3B_REDUCE_MAX:
                return noAllocXform<T, A3B_REDUCE_MAX>(s, xop, i0, i1, n, nv, out);
            default:
                setError("unknown reduce op %d", rop);
                return A3B_ERR_INVALID;
            }
        }
    } // namespace
} // namespace a3b

using namespace a3b;

extern "C"
{
    int a3b_transform_reduce(a3b_stream_t stream, int dtype, int reduce_op, int transform_op, void const* in0,
                             void const* in1, uint64_t n, void const* neutral, void* out)
    {
        return reduceEntry(stream, dtype, reduce_op, transform_op, in0, in1, 1, n, 0, neutral, out, false);
    }

    int a3b_transform_reduce_partial(a3b_stream_t stream, int dtype, int reduce_op, int transform_op,
                                     void const* in0, void const* in1, uint64_t n, void const* neutral,
                                     void* partial_out)
    {
        return reduceEntry(stream, dtype, reduce_op, transform_op, in0, in1, 1, n, 0, neutral, partial_out, true);
    }

    int a3b_reduce_2d(a3b_stream_t stream, int dtype, int reduce_op, void const* in, uint64_t rows, uint64_t row_len,
                      uint64_t row_pitch_bytes, void const* neutral, void* out)
    {
        int const es = dtypeSize(dtype);
        A3B_REQUIRE(es > 0, "unknown dtype");
        A3B_REQUIRE(rows <= 1 || row_pitch_bytes >= row_len * static_cast<uint64_t>(es), "row pitch smaller than a row");
        return reduceEntry(stream, dtype, reduce_op, A3B_XFORM_IDENTITY, in, nullptr, rows, row_len, row_pitch_bytes,
                           neutral, out, false);
    }

    int a3b_set_early_start(a3b_stream_t stream, int enable)
    {
        int dev = 0;
        A3B_CUDA(cudaGetDevice(&dev));
        setEarlyStart(dev, static_cast<cudaStream_t>(stream), enable != 0);
        return A3B_OK;
    }

    int a3b_debug_early_start_enable(int device, a3b_stream_t stream, int enable)
    {
        setEarlyStart(device, static_cast<cudaStream_t>(stream), enable != 0);
        return A3B_OK;
    }

    int a3b_debug_early_start_probe(int device, a3b_stream_t stream, void const* in0, void const* in1,
                                    uint64_t in_bytes, void* out, int* early)
    {
        A3B_REQUIRE(early, "null result pointer");
        *early = earlyStartAllowed(device, static_cast<cudaStream_t>(stream), in0, in1, in_bytes, out) ? 1 : 0;
        return A3B_OK;
    }

    int a3b_transform_reduce_noalloc(a3b_stream_t stream, int dtype, int reduce_op, int transform_op, void const* in0,
                                     void const* in1, uint64_t n, void const* neutral, void* out)
    {
        A3B_REQUIRE(out && neutral, "null out/neutral");
        A3B_REQUIRE(in0 || n == 0, "null input");
        auto s = static_cast<cudaStream_t>(stream);
        switch(dtype)
        {
        case A3B_I32:
            return noAllocReduce<int32_t>(s, reduce_op, transform_op, in0, in1, n, neutral, out);
        case A3B_U32:
            return noAllocReduce<uint32_t>(s, reduce_op, transform_op, in0, in1, n, neutral, out);
        case A3B_I64:
            return noAllocReduce<int64_t>(s, reduce_op, transform_op, in0, in1, n, neutral, out);
        case A3B_U64:
            return noAllocReduce<uint64_t>(s, reduce_op, transform_op, in0, in1, n, neutral, out);
        case A3B_F32:
            return noAllocReduce<float>(s, reduce_op, transform_op, in0, in1, n, neutral, out);
        case A3B_F64:
            return noAllocReduce<double>(s, reduce_op, transform_op, in0, in1, n, neutral, out);
        default:
            setError("unknown dtype %d", dtype);
            return A3B_ERR_INVALID;
        }
    }

    int a3b_transform_reduce_allranks(a3b_stream_t stream, a3b_peer_group* group, int dtype, int reduce_op,
                                      int transform_op, void const* in0, void const* in1, uint64_t n,
                                      void const* neutral, void* out)
    {
        A3B_REQUIRE(group && out && neutral, "null group/out/neutral");
        A3B_REQUIRE(in0 || n == 0, "null input");
        auto s = static_cast<cudaStream_t>(stream);
        switch(dtype)
        {
        case A3B_I32:
            return allRanksReduce<int32_t>(s, group, reduce_op, transform_op, in0, in1, n, neutral, out);
        case A3B_U32:
            return allRanksReduce<uint32_t>(s, group, reduce_op, transform_op, in0, in1, n, neutral, out);
        case A3B_I64:
            return allRanksReduce<int64_t>(s, group, reduce_op, transform_op, in0, in1, n, neutral, out);
        case A3B_U64:
            return allRanksReduce<uint64_t>(s, group, reduce_op, transform_op, in0, in1, n, neutral, out);
        case A3B_F32:
            return allRanksReduce<float>(s, group, reduce_op, transform_op, in0, in1, n, neutral, out);
        case A3B_F64:
            return allRanksReduce<double>(s, group, reduce_op, transform_op, in0, in1, n, neutral, out);
        default:
            setError("unknown dtype %d", dtype);
            return A3B_ERR_INVALID;
        }
    }

    int a3b_reduce_lower_ranks(a3b_stream_t stream, a3b_peer_group* group, int dtype, void const* in, uint64_t n,
                               void* carry_out)
    {
        A3B_REQUIRE(group && carry_out, "null group/out");
        A3B_REQUIRE(in || n == 0, "null input");
        auto s = static_cast<cudaStream_t>(stream);
        int64_t const zero = 0;
        double const zf = 0.0;
        float const zf32 = 0.f;
        switch(dtype)
        {
        case A3B_I32:
            return allRanksReduce<int32_t>(s, group, A3B_REDUCE_PLUS, A3B_XFORM_IDENTITY, in, nullptr, n, &zero, carry_out, true);
        case A3B_U32:
            return allRanksReduce<uint32_t>(s, group, A3B_REDUCE_PLUS, A3B_XFORM_IDENTITY, in, nullptr, n, &zero, carry_out, true);
        case A3B_I64:
            return allRanksReduce<int64_t>(s, group, A3B_REDUCE_PLUS, A3B_XFORM_IDENTITY, in, nullptr, n, &zero, carry_out, true);
        case A3B_U64:
            return allRanksReduce<uint64_t>(s, group, A3B_REDUCE_PLUS, A3B_XFORM_IDENTITY, in, nullptr, n, &zero, carry_out, true);
        case A3B_F32:
            return allRanksReduce<float>(s, group, A3B_REDUCE_PLUS, A3B_XFORM_IDENTITY, in, nullptr, n, &zf32, carry_out, true);
        case A3B_F64:
            return allRanksReduce<double>(s, group, A3B_REDUCE_PLUS, A3B_XFORM_IDENTITY, in, nullptr, n, &zf, carry_out, true);
        default:
            setError("unknown dtype %d", dtype);
            return A3B_ERR_INVALID;
        }
    }
}
