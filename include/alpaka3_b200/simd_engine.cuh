/* B200 engine for alpaka3's device functors (header-only CUDA, sm_100a; nvcc translation units that include
 * <alpaka/alpaka.hpp>).
 *
 * alpaka3 calls every user functor of its primitive layer through one device primitive: for each SIMD pack of an
 * N-D index domain, func(acc, SimdPtr{data, idx}...) with one SimdPtr per data source (include/alpaka/onAcc/internal/
 * SimdConcurrent.hpp:86-93, 122-234), and SimdTransformReduce folds the transformed packs with the reduce functor
 * (include/alpaka/onAcc/internal/SimdTransformReduce.hpp:359-499). A functor cannot cross a C ABI, so this engine is
 * a set of kernel templates that nvcc compiles in the caller's translation unit with the caller's functors. What it
 * replaces is the grid and the reduction scheme, not the calling convention:
 *
 *   - the index domain is cut into rows (all but the fastest dimension) and every row into chunks of
 *     kThreads x P packs x W elements, W = 16 bytes / the widest element type of the call; block b handles chunk b
 *     (one chunk per block while the grid fits, so the block scheduler sweeps memory front to back, as the library's
 *     own element-wise and reduction kernels do); the ragged end of a row is handled element by element (W = 1);
 *   - each pack is handed to the functor as alpaka::SimdPtr objects of width W (AutoAligned: the load width follows
 *     the data source's own alignment, as in alpaka3), together with an accelerator object that describes this
 *     engine's 1-D launch (functors that take `acc` see this grid and block);
 *   - reductions fold the transformed lanes into one value per thread with the reduce functor, combine the block in
 *     shared memory in a fixed tree order and finish in the last block to arrive (ticket), which combines the
 *     per-block values in block order: one launch, no pre-fill of `out`, and the same bits for the same input and
 *     grid. The grid is capped at 8 blocks per SM (each block folds several chunks), so the per-block values fit a
 *     small scratch array that the library caches per stream (a3b_engine_scratch); the ticket is reset by the last
 *     block.
 */
#pragma once

#include <alpaka/alpaka.hpp>

#include "../alpaka3_b200.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>
#include <utility>

namespace alpaka3_b200::simd
{
    constexpr int kThreads = 256;
    constexpr std::uint64_t kMaxGrid = (std::uint64_t{1} << 31) - 1u;
    constexpr unsigned kReduceBlocksPerSm = 8u;

    //! Launch description of this engine for alpaka3's CUDA index layers: a 1-D grid of 1-D blocks.
    using LaunchSpec = alpaka::onHost::unifiedCudaHip::CallKernel::
        OptimizedThreadSpec<alpaka::Vec<std::uint32_t, 1u>, alpaka::Vec<std::uint32_t, 1u>>;

    /** The accelerator object alpaka3's device functors take as their optional first argument, for this engine's
     * launch: the CUDA block/thread index layers over `spec`, block synchronisation, the API, device kind and
     * executor of the queue, and the warp size (the entries alpaka3's own CUDA kernel entry provides,
     * include/alpaka/api/unifiedCudaHip/Queue.hpp:187-209). */
    template<typename TApi, typename TDeviceKind, typename TExec>
    __device__ __forceinline__ auto makeAcc(LaunchSpec const& spec)
    {
        constexpr auto warp = alpaka::onAcc::unifiedCudaHip::internal::WarpSize::Get<TDeviceKind>{}();
        return alpaka::onAcc::Acc{alpaka::Dict{
            alpaka::DictEntry(alpaka::layer::block, alpaka::onAcc::unifiedCudaHip::BlockLayer{spec}),
            alpaka::DictEntry(alpaka::layer::thread, alpaka::onAcc::unifiedCudaHip::ThreadLayer{spec}),
            alpaka::DictEntry(alpaka::object::launchedWidthFrameSpec, std::bool_constant<false>{}),
            alpaka::DictEntry(alpaka::action::threadBlockSync, alpaka::onAcc::unifiedCudaHip::Sync{}),
            alpaka::DictEntry(alpaka::object::api, TApi{}),
            alpaka::DictEntry(alpaka::object::deviceKind, TDeviceKind{}),
            alpaka::DictEntry(alpaka::object::exec, TExec{}),
            alpaka::DictEntry(alpaka::object::warpSize, warp)}};
    }

    //! Index of element `col` of row `row` of an N-D domain (rows enumerate all but the fastest dimension, row-major).
    template<typename TExt>
    __device__ __forceinline__ TExt indexOf(TExt const& ext, std::uint64_t row, std::uint64_t col)
    {
        using I = typename TExt::type;
        constexpr std::uint32_t dim = TExt::dim();
        TExt idx = ext;
        idx[dim - 1u] = static_cast<I>(col);
        if constexpr(dim > 1u)
        {
            std::uint64_t r = row;
            for(int d = static_cast<int>(dim) - 2; d >= 0; --d)
            {
                std::uint64_t const e = static_cast<std::uint64_t>(ext[static_cast<std::uint32_t>(d)]);
                idx[static_cast<std::uint32_t>(d)] = static_cast<I>(r % e);
                r /= e;
            }
        }
        return idx;
    }

    template<typename TSrc>
    using ValueOf = std::remove_cv_t<alpaka::trait::GetValueType_t<std::decay_t<TSrc>>>;

    //! Pack width of a call: 16 bytes of its widest element type (1 for elements of 16 bytes or more).
    template<typename... TSrc>
    constexpr std::uint32_t packWidth()
    {
        std::size_t m = 1;
        ((m = sizeof(ValueOf<TSrc>) > m ? sizeof(ValueOf<TSrc>) : m), ...);
        return m >= 16 ? 1u : static_cast<std::uint32_t>(16 / m);
    }

    //! Chunking of an N-D domain: rows x rowLen elements, chunks of kThreads * P * W elements along each row.
    struct Domain
    {
        std::uint64_t rows = 0;
        std::uint64_t rowLen = 0;
        std::uint64_t chunksPerRow = 0;
        std::uint64_t chunks = 0;
    };

    template<typename TExt>
    Domain domainOf(TExt const& ext, std::uint64_t chunk)
    {
        constexpr std::uint32_t dim = TExt::dim();
        Domain d;
        d.rows = 1u;
        for(std::uint32_t k = 0; k + 1u < dim; ++k)
            d.rows *= static_cast<std::uint64_t>(ext[k]);
        d.rowLen = static_cast<std::uint64_t>(ext[dim - 1u]);
        d.chunksPerRow = (d.rowLen + chunk - 1u) / chunk;
        d.chunks = d.rows * d.chunksPerRow;
        return d;
    }

    /** Calls body(acc, SimdPtr...) for every pack of chunk `chunk` of this thread (P packs of W elements; elements of
     * a row's ragged end one by one). */
    template<std::uint32_t W, int P, typename TAcc, typename TExt, typename Body, typename... Src>
    __device__ __forceinline__ void eachInChunk(
        TAcc const& acc,
        TExt const& ext,
        Domain const& dom,
        std::uint64_t chunk,
        Body const& body,
        Src&... src)
    {
        constexpr std::uint64_t kChunk = std::uint64_t{kThreads} * P * W;
        std::uint64_t const row = chunk / dom.chunksPerRow;
        std::uint64_t const col0 = (chunk - row * dom.chunksPerRow) * kChunk;
#pragma unroll
        for(int p = 0; p < P; ++p)
        {
            std::uint64_t const c = col0 + (static_cast<std::uint64_t>(p) * kThreads + threadIdx.x) * W;
            if(c + W <= dom.rowLen)
            {
                auto const idx = indexOf(ext, row, c);
                body(acc, alpaka::SimdPtr{src, idx, alpaka::AutoAligned{}, alpaka::CVec<std::uint32_t, W>{}}...);
            }
            else
            {
                for(std::uint64_t e = c; e < dom.rowLen && e < c + W; ++e)
                {
                    auto const idx = indexOf(ext, row, e);
                    body(acc, alpaka::SimdPtr{src, idx, alpaka::AutoAligned{}, alpaka::CVec<std::uint32_t, 1u>{}}...);
                }
            }
        }
    }

    template<
        std::uint32_t W,
        int P,
        typename TApi,
        typename TDeviceKind,
        typename TExec,
        typename TExt,
        typename Body,
        typename... Src>
    __global__ void __launch_bounds__(kThreads) eachKernel(TExt ext, Domain dom, Body body, Src... src)
    {
        LaunchSpec const spec{alpaka::Vec<std::uint32_t, 1u>{gridDim.x}, alpaka::Vec<std::uint32_t, 1u>{blockDim.x}};
        auto const acc = makeAcc<TApi, TDeviceKind, TExec>(spec);
        for(std::uint64_t chunk = blockIdx.x; chunk < dom.chunks; chunk += gridDim.x)
            eachInChunk<W, P>(acc, ext, dom, chunk, body, src...);
    }

    /** body(acc, SimdPtr...) over every pack of the domain `extents` (asynchronous on `stream`). The data sources are
     * alpaka3 objects accessible in kernels (MdSpans, views, generators). */
    template<typename TApi, typename TDeviceKind, typename TExec, typename TExt, typename Body, typename... Src>
    cudaError_t each(cudaStream_t stream, TExt const& extents, Body const& body, Src const&... src)
    {
        using Ext = typename std::decay_t<TExt>::UniVec;
        Ext const ext{extents};
        constexpr std::uint32_t W = packWidth<Src...>();
        constexpr int P = sizeof...(Src) <= 2 ? 2 : 1;
        Domain const dom = domainOf(ext, std::uint64_t{kThreads} * P * W);
        if(dom.chunks == 0u)
            return cudaSuccess;
        std::uint64_t const grid = dom.chunks < kMaxGrid ? dom.chunks : kMaxGrid;
        eachKernel<W, P, TApi, TDeviceKind, TExec, Ext, Body, Src...>
            <<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(ext, dom, body, src...);
        return cudaGetLastError();
    }

    // ------------------------------------------------------------------------------------ functor adapters

    template<typename F>
    constexpr bool isStencil = alpaka::isSpecializationOf_v<std::decay_t<F>, alpaka::StencilFunc>;
    template<typename F>
    constexpr bool isScalar = alpaka::isSpecializationOf_v<std::decay_t<F>, alpaka::ScalarFunc>;

    //! fn(acc?, a[K], b[K], ...): lane K of a pack computed on scalars
    template<std::uint32_t K, typename TAcc, typename Fn, typename... S>
    __device__ __forceinline__ auto laneOf(TAcc const& acc, Fn const& fn, S const&... packs)
    {
        return alpaka::callFunctor(acc, fn, packs[K]...);
    }

    //! The lanes of a pack computed one by one: Simd{fn(acc?, a[k], b[k], ...)...} (alpaka3's ScalarFunc semantics).
    template<std::uint32_t... K, typename TAcc, typename Fn, typename... S>
    __device__ __forceinline__ auto scalarLanes(
        std::integer_sequence<std::uint32_t, K...>,
        TAcc const& acc,
        Fn const& fn,
        S const&... packs)
    {
        return alpaka::Simd{laneOf<K>(acc, fn, packs...)...};
    }

    //! onHost::concurrent: fn(acc?, SimdPtr...) (include/alpaka/onHost/algo/internal/concurrent.hpp:18-41).
    template<typename Fn>
    struct ConcurrentBody
    {
        Fn fn;

        template<typename TAcc, typename... Ptr>
        __device__ __forceinline__ void operator()(TAcc const& acc, Ptr... p) const
        {
            alpaka::callFunctor(acc, fn, p...);
        }
    };

    //! SimdAlgo::concurrent inside a user kernel: op(acc, SimdPtr...) (include/alpaka/onAcc/SimdAlgo.hpp:73-112).
    template<typename Op>
    struct AccFirstBody
    {
        Op op;

        template<typename TAcc, typename... Ptr>
        __device__ __forceinline__ void operator()(TAcc const& acc, Ptr... p) const
        {
            op(acc, p...);
        }
    };

    //! onHost::transform: out = fn(...) with SimdPtrs (StencilFunc), lane by lane (ScalarFunc) or loaded packs
    //! (include/alpaka/onHost/algo/internal/transform.hpp:21-81).
    template<typename Fn>
    struct TransformBody
    {
        Fn fn;

        template<typename TAcc, typename Out, typename... In>
        __device__ __forceinline__ void operator()(TAcc const& acc, Out out, In const&... in) const
        {
            if constexpr(isStencil<Fn>)
                out = alpaka::callFunctor(acc, fn, in...);
            else if constexpr(isScalar<Fn>)
                out = scalarLanes(std::make_integer_sequence<std::uint32_t, Out::width()>{}, acc, fn, in.load()...);
            else
                out = alpaka::callFunctor(acc, fn, in.load()...);
        }
    };

    //! onHost::iota: every output gets init + the linear index of each element, computed per pack as alpaka3 does
    //! (base = linear index of the pack's first element + init, lane k adds k; include/alpaka/onHost/algo/internal/
    //! iota.hpp:19-50), so floating-point outputs round the same way.
    template<typename T, typename TExt>
    struct IotaBody
    {
        TExt ext;
        T init;

        template<typename TAcc, typename P0, typename... Ptr>
        __device__ __forceinline__ void operator()(TAcc const&, P0 out0, Ptr... outs) const
        {
            using SimdType = decltype(out0.load());
            T const base = static_cast<T>(alpaka::linearize(ext, out0.getIdx())) + init;
            auto const result = SimdType([&](auto const& lane) constexpr { return base + static_cast<T>(lane); });
            out0 = alpaka::pCast<alpaka::trait::GetValueType_t<P0>>(result);
            ((outs = alpaka::pCast<alpaka::trait::GetValueType_t<Ptr>>(result)), ...);
        }
    };

    //! onHost::fill of a buffer that is not one dense block (pitched rows, sub-views)
    template<typename T>
    struct FillBody
    {
        T value;

        template<typename TAcc, typename P0>
        __device__ __forceinline__ void operator()(TAcc const&, P0 out) const
        {
            out = decltype(out.load())::fill(value);
        }
    };

    //! The transform of onHost::transformReduce, as SimdTransformReduce wraps it
    //! (include/alpaka/onAcc/internal/SimdTransformReduce.hpp:108-144).
    template<typename Fn>
    struct ReduceTransform
    {
        Fn fn;

        template<typename TAcc, typename P0, typename... Ptr>
        __device__ __forceinline__ auto operator()(TAcc const& acc, P0 const& p0, Ptr const&... p) const
        {
            if constexpr(isStencil<Fn>)
                return alpaka::callFunctor(acc, fn, p0, p...);
            else if constexpr(isScalar<Fn>)
                return scalarLanes(
                    std::make_integer_sequence<std::uint32_t, P0::width()>{},
                    acc,
                    fn,
                    p0.load(),
                    p.load()...);
            else
                return alpaka::callFunctor(acc, fn, p0.load(), p.load()...);
        }
    };

    //! a = rop(a, lane) for every lane of a transformed pack (or the scalar itself)
    template<typename T, typename ROp, typename R>
    __device__ __forceinline__ void foldLanes(T& a, ROp const& rop, R const& r)
    {
        if constexpr(alpaka::concepts::Simd<std::decay_t<R>>)
        {
#pragma unroll
            for(std::uint32_t k = 0; k < std::decay_t<R>::width(); ++k)
                a = static_cast<T>(rop(a, static_cast<T>(+r[k])));
        }
        else
            a = static_cast<T>(rop(a, static_cast<T>(r)));
    }

    template<typename T, typename ROp, typename XOp>
    struct FoldBody
    {
        ROp rop;
        XOp xop;
        T* acc;

        template<typename TAcc, typename... Ptr>
        __device__ __forceinline__ void operator()(TAcc const& a, Ptr... p) const
        {
            foldLanes(*acc, rop, xop(a, p...));
        }
    };

    //! Scratch of one reduction: the ticket of the last-block-done step, then one value per block.
    template<typename T>
    struct ReduceWork
    {
        unsigned* ticket;
        T* partials;
    };

    template<typename T>
    constexpr std::size_t partialsOffset()
    {
        return alignof(T) > 256 ? alignof(T) : 256;
    }

    //! Combines kThreads values of a block in shared memory, in a fixed tree order; the result is in s[0].
    template<typename T, typename ROp>
    __device__ __forceinline__ void blockTree(T* s, ROp const& rop)
    {
        for(int w = kThreads / 2; w > 0; w /= 2)
        {
            __syncthreads();
            if(static_cast<int>(threadIdx.x) < w)
                s[threadIdx.x] = static_cast<T>(rop(s[threadIdx.x], s[threadIdx.x + w]));
        }
        __syncthreads();
    }

    template<
        std::uint32_t W,
        int P,
        typename TApi,
        typename TDeviceKind,
        typename TExec,
        typename TExt,
        typename T,
        typename ROp,
        typename XOp,
        typename... Src>
    __global__ void __launch_bounds__(kThreads) reduceKernel(
        TExt ext,
        Domain dom,
        T neutral,
        ROp rop,
        XOp xop,
        T* out,
        ReduceWork<T> work,
        Src... src)
    {
        __shared__ alignas(T) unsigned char raw[kThreads * sizeof(T)];
        __shared__ bool last;
        T* const s = reinterpret_cast<T*>(raw);
        LaunchSpec const spec{alpaka::Vec<std::uint32_t, 1u>{gridDim.x}, alpaka::Vec<std::uint32_t, 1u>{blockDim.x}};
        auto const acc = makeAcc<TApi, TDeviceKind, TExec>(spec);

        T a = neutral;
        FoldBody<T, ROp, XOp> const fold{rop, xop, &a};
        for(std::uint64_t chunk = blockIdx.x; chunk < dom.chunks; chunk += gridDim.x)
            eachInChunk<W, P>(acc, ext, dom, chunk, fold, src...);
        s[threadIdx.x] = a;
        blockTree(s, rop);
        if(threadIdx.x == 0)
        {
            work.partials[blockIdx.x] = s[0];
            __threadfence();
            last = atomicAdd(work.ticket, 1u) == gridDim.x - 1u;
        }
        __syncthreads();
        if(!last)
            return;
        __threadfence();
        T b = neutral;
        for(unsigned k = threadIdx.x; k < gridDim.x; k += kThreads)
            b = static_cast<T>(rop(b, work.partials[k]));
        s[threadIdx.x] = b;
        blockTree(s, rop);
        if(threadIdx.x == 0)
        {
            *out = s[0];
            *work.ticket = 0u; // ready for the next call on the stream
        }
    }

    /** out[0] = fold of rop over xop's lanes of every pack of `extents`, starting from `neutral` (asynchronous on
     * `stream`; `out` is a device pointer). */
    template<
        typename TApi,
        typename TDeviceKind,
        typename TExec,
        typename TExt,
        typename T,
        typename ROp,
        typename XOp,
        typename... Src>
    cudaError_t reduce(
        cudaStream_t stream,
        TExt const& extents,
        T const& neutral,
        ROp const& rop,
        XOp const& xop,
        T* out,
        Src const&... src)
    {
        static_assert(std::is_trivially_copyable_v<T>, "the reduced type must be trivially copyable");
        using Ext = typename std::decay_t<TExt>::UniVec;
        Ext const ext{extents};
        constexpr std::uint32_t W = packWidth<Src...>();
        constexpr int P = sizeof...(Src) <= 2 ? 2 : 1;
        Domain const dom = domainOf(ext, std::uint64_t{kThreads} * P * W);
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if(e != cudaSuccess)
            return e;
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if(e != cudaSuccess)
            return e;
        std::uint64_t const cap = static_cast<std::uint64_t>(sms) * kReduceBlocksPerSm;
        std::uint64_t const grid = dom.chunks == 0u ? 1u : (dom.chunks < cap ? dom.chunks : cap);
        void* scr = nullptr;
        if(a3b_engine_scratch(stream, partialsOffset<T>() + grid * sizeof(T), &scr) != A3B_OK)
            return cudaErrorMemoryAllocation;
        ReduceWork<T> const work{
            static_cast<unsigned*>(scr),
            reinterpret_cast<T*>(static_cast<unsigned char*>(scr) + partialsOffset<T>())};
        reduceKernel<W, P, TApi, TDeviceKind, TExec, Ext, T, ROp, XOp, Src...>
            <<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(ext, dom, neutral, rop, xop, out, work, src...);
        return cudaGetLastError();
    }
} // namespace alpaka3_b200::simd
