/* alpaka3 binding of the B200 primitive library (header-only, C++20).
 *
 * Include after (or instead of) <alpaka/alpaka.hpp> and link libalpaka3_b200.so. The header adds overloads of
 *   alpaka::onHost::transformReduce   (alpaka3: include/alpaka/onHost/algo/transformReduce.hpp:59-114)
 *   alpaka::onHost::reduce            (include/alpaka/onHost/algo/reduce.hpp:28-79)
 *   alpaka::onHost::exclusiveScan / inclusiveScan / *InPlace   (include/alpaka/onHost/algo/scan.hpp:45-218)
 *   alpaka::onHost::transform         (include/alpaka/onHost/algo/transform.hpp:50-88)
 *   alpaka::onHost::concurrent        (include/alpaka/onHost/algo/concurrent.hpp:44-82)
 *   alpaka::onHost::iota              (include/alpaka/onHost/algo/iota.hpp:29-85)
 *   alpaka::onHost::fill              (include/alpaka/onHost/Queue.hpp:346)
 * for queues of CUDA devices (Queue<Device<api::Cuda, K>, Q>). Partial ordering picks them over alpaka3's generic
 * templates because their queue parameter is more specialised. A call runs on one of three paths:
 *
 *   1. the library's tuned kernels through the C ABI, when the functors are known by their TYPE: std::plus (or a
 *      ScalarFunc around a type declared below) as the reduce functor, std::identity (one input) or std::multiplies
 *      (two inputs) as the transform; int32/uint32/int64/uint64/float/double device buffers laid out densely or as
 *      rows with one constant pitch. A caller declares its own functor types with the traits
 *      alpaka3_b200::ReduceKind<F> / TransformKind<F> (e.g. BabelStream's DotMultiplication as A3B_XFORM_PRODUCT).
 *      Scans with + of those types, fill of dense buffers and integer iota into one dense buffer also go here.
 *      Classifying unknown functor types by evaluating them on a few values is available behind
 *      ALPAKA3_B200_PROBE_FUNCTORS (off by default: a functor that agrees with x*x on small positive values but not
 *      on negative ones would be misrouted);
 *   2. in translation units compiled by nvcc, every other transformReduce / reduce / transform / concurrent call runs
 *      on the B200 engines compiled here with the caller's functors: include/alpaka3_b200/elementwise.cuh for
 *      transforms of SIMD or scalar functors over plain device buffers, include/alpaka3_b200/simd_engine.cuh for the
 *      rest (StencilFunc and ScalarFunc functors, functors that take an accelerator, generator sources such as
 *      LinearizedIdxGenerator, up-casting outputs, any reduce functor); they call the functors exactly as alpaka3
 *      does (SimdPtr / Simd packs, optional accelerator first argument);
 *   3. anything else (host translation units without nvcc, unsupported data sources) is forwarded unchanged to
 *      alpaka3's own implementation (onHost::internal::*).
 * alpaka3_b200::routingStats() counts the calls per path. Backend errors throw std::runtime_error, as alpaka3's
 * ALPAKA_UNIFORM_CUDA_HIP_RT_CHECK does (include/alpaka/core/UniformCudaHip.hpp:42). Blocking queues wait for the
 * call to finish.
 */
#pragma once

#include <alpaka/alpaka.hpp>

#include "../alpaka3_b200.h"
#if defined(__CUDACC__)
#    include "elementwise.cuh"
#    include "simd_engine.cuh"
#endif

#include <atomic>
#include <cstdint>
#include <functional>
#include <optional>
#include <stdexcept>
#include <string>
#include <string_view>
#include <type_traits>
#include <utility>

namespace alpaka3_b200
{
    //! How many calls this process sent to the library (C ABI or a B200 engine compiled here: `routed`, of which
    //! `engine` ran on an engine) / forwarded to alpaka3's own implementation.
    struct RoutingStats
    {
        std::atomic<std::uint64_t> routed{0};
        std::atomic<std::uint64_t> engine{0};
        std::atomic<std::uint64_t> forwarded{0};
    };

    /** What a reduce functor type computes, for the C ABI path: A3B_REDUCE_PLUS / _MIN / _MAX, or -1 (unknown: the
     * call runs on the engine with the functor itself). Specialise for your own functor types. */
    template<typename F>
    struct ReduceKind : std::integral_constant<int, -1>
    {
    };

    template<>
    struct ReduceKind<std::plus<>> : std::integral_constant<int, A3B_REDUCE_PLUS>
    {
    };

    template<typename T>
    struct ReduceKind<std::plus<T>> : std::integral_constant<int, A3B_REDUCE_PLUS>
    {
    };

    template<typename F>
    struct ReduceKind<alpaka::ScalarFunc<F>> : ReduceKind<F>
    {
    };

    /** What a transform functor type computes: A3B_XFORM_IDENTITY (one input), A3B_XFORM_SQUARE (one input, x*x),
     * A3B_XFORM_PRODUCT (two inputs, a*b), or -1. Specialise for your own functor types. */
    template<typename F>
    struct TransformKind : std::integral_constant<int, -1>
    {
    };

    template<>
    struct TransformKind<std::identity> : std::integral_constant<int, A3B_XFORM_IDENTITY>
    {
    };

    template<>
    struct TransformKind<std::multiplies<>> : std::integral_constant<int, A3B_XFORM_PRODUCT>
    {
    };

    template<typename T>
    struct TransformKind<std::multiplies<T>> : std::integral_constant<int, A3B_XFORM_PRODUCT>
    {
    };

    template<typename F>
    struct TransformKind<alpaka::ScalarFunc<F>> : TransformKind<F>
    {
    };

    namespace detail
    {
        template<typename T>
        constexpr std::string_view prettyName()
        {
            return __PRETTY_FUNCTION__;
        }

        constexpr bool identChar(char c)
        {
            return (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || (c >= '0' && c <= '9') || c == '_';
        }

        //! true when `name` occurs as a whole identifier in the compiler's spelling of T
        template<typename T>
        constexpr bool typeNamed(std::string_view name)
        {
            std::string_view const p = prettyName<T>();
            for(auto pos = p.find(name); pos != std::string_view::npos; pos = p.find(name, pos + 1))
            {
                bool const before = pos == 0 || !identChar(p[pos - 1]);
                bool const after = pos + name.size() >= p.size() || !identChar(p[pos + name.size()]);
                if(before && after)
                    return true;
            }
            return false;
        }

        template<typename K>
        constexpr bool listedSimdForEachKernel()
        {
#if defined(ALPAKA3_B200_SIMD_FOR_EACH_KERNELS)
            std::string_view list = ALPAKA3_B200_SIMD_FOR_EACH_KERNELS;
            while(!list.empty())
            {
                auto const sp = list.find(' ');
                std::string_view const tok = list.substr(0, sp);
                if(!tok.empty() && typeNamed<K>(tok))
                    return true;
                if(sp == std::string_view::npos)
                    break;
                list.remove_prefix(sp + 1);
            }
#endif
            return false;
        }
    } // namespace detail

    /** Kernel types K whose body is exactly
     *      onAcc::SimdAlgo{onAcc::worker::threadsInGrid}.concurrent(acc, arg0.getExtents(), op, arg0, args...)
     * for a bundle KernelBundle{K{}, op, arg0, args...} -- BabelStream's SimdForEachKernel
     * (benchmark/babelstream/src/babelStreamMainTest.cpp:61-75). queue.enqueue(FrameSpec, bundle) of such a kernel
     * on a CUDA queue runs the bundle's op on the B200 SIMD engine instead of the kernel body (same op calls, the
     * engine's grid). The binding cannot see a kernel's body, so this is opt-in: specialise the trait, or list the
     * kernel type names (space separated) in the compile definition ALPAKA3_B200_SIMD_FOR_EACH_KERNELS, e.g.
     * -DALPAKA3_B200_SIMD_FOR_EACH_KERNELS='"SimdForEachKernel"', which leaves the caller's source unchanged. */
    template<typename K>
    struct IsSimdForEachKernel : std::bool_constant<detail::listedSimdForEachKernel<K>()>
    {
    };

    inline RoutingStats& routingStats()
    {
        static RoutingStats s;
        return s;
    }

    namespace detail
    {
        inline void check(int rc, char const* what)
        {
            if(rc != A3B_OK)
                throw std::runtime_error(std::string(what) + ": " + a3b_last_error());
        }

        template<typename T>
        constexpr int dtypeOf()
        {
            if constexpr(std::is_same_v<T, std::int32_t>)
                return A3B_I32;
            else if constexpr(std::is_same_v<T, std::uint32_t>)
                return A3B_U32;
            else if constexpr(std::is_same_v<T, std::int64_t> || (std::is_same_v<T, long long> && sizeof(T) == 8))
                return A3B_I64;
            else if constexpr(std::is_same_v<T, std::uint64_t> || (std::is_same_v<T, unsigned long long> && sizeof(T) == 8))
                return A3B_U64;
            else if constexpr(std::is_same_v<T, float>)
                return A3B_F32;
            else if constexpr(std::is_same_v<T, double>)
                return A3B_F64;
            else
                return -1;
        }

        template<typename T, typename R>
        std::optional<T> scalarOf(R const& r)
        {
            if constexpr(std::is_arithmetic_v<std::decay_t<R>>)
                return static_cast<T>(r);
            else if constexpr(requires { r[0]; })
                return static_cast<T>(r[0]);
            else
                return std::nullopt;
        }

        template<typename T, typename>
        using Pack1 = alpaka::Simd<T, 1u>;

        //! Evaluate a functor on the host with scalar arguments, or with one-lane SIMD packs when it takes packs.
        template<typename T, typename F, typename... A>
        std::optional<T> probe(F const& f, A... a)
        {
            if constexpr(std::is_invocable_v<F const&, A...>)
                return scalarOf<T>(f(a...));
            else if constexpr(std::is_invocable_v<F const&, Pack1<T, A>...>)
                return scalarOf<T>(f(Pack1<T, A>{static_cast<T>(a)}...));
            else
                return std::nullopt;
        }

        template<typename T, typename F>
        int reduceOpOf([[maybe_unused]] F const& f)
        {
            using D = std::decay_t<F>;
            if constexpr(ReduceKind<D>::value >= 0)
                return ReduceKind<D>::value;
#if defined(ALPAKA3_B200_PROBE_FUNCTORS)
            else
            {
                auto const a = probe<T>(f, T(3), T(5)), b = probe<T>(f, T(5), T(3)), c = probe<T>(f, T(7), T(2));
                if(!a || !b || !c)
                    return -1;
                if(*a == T(8) && *b == T(8) && *c == T(9))
                    return A3B_REDUCE_PLUS;
                if(*a == T(3) && *b == T(3) && *c == T(2))
                    return A3B_REDUCE_MIN;
                if(*a == T(5) && *b == T(5) && *c == T(7))
                    return A3B_REDUCE_MAX;
                return -1;
            }
#else
            else
                return -1;
#endif
        }

        template<typename T, int NIN, typename F>
        int transformOpOf([[maybe_unused]] F const& f)
        {
            using D = std::decay_t<F>;
            constexpr int kind = TransformKind<D>::value;
            if constexpr(kind >= 0)
                return (kind == A3B_XFORM_PRODUCT) == (NIN == 2) ? kind : -1;
#if defined(ALPAKA3_B200_PROBE_FUNCTORS)
            else if constexpr(NIN == 1)
            {
                auto const a = probe<T>(f, T(3)), b = probe<T>(f, T(5));
                if(!a || !b)
                    return -1;
                if(*a == T(3) && *b == T(5))
                    return A3B_XFORM_IDENTITY;
                if(*a == T(9) && *b == T(25))
                    return A3B_XFORM_SQUARE;
                return -1;
            }
            else if constexpr(NIN == 2)
            {
                auto const a = probe<T>(f, T(3), T(5)), b = probe<T>(f, T(7), T(2));
                if(a && b && *a == T(15) && *b == T(14))
                    return A3B_XFORM_PRODUCT;
                return -1;
            }
#endif
            else
                return -1;
        }

        //! Device buffer view as (pointer, rows, row length, row pitch in bytes); false when the layout does not fit.
        struct Layout
        {
            void const* ptr = nullptr;
            std::uint64_t rows = 0, rowLen = 0, rowPitch = 0;

            bool dense() const
            {
                return rows <= 1u || rowPitch == 0u;
            }
        };

        template<typename T>
        bool layoutOf(auto const& view, Layout& out)
        {
            auto const ext = alpaka::onHost::getExtents(view);
            auto const pitch = alpaka::onHost::getPitches(view);
            constexpr auto dim = std::decay_t<decltype(ext)>::dim();
            out.ptr = static_cast<void const*>(alpaka::onHost::data(view));
            if(static_cast<std::uint64_t>(pitch[dim - 1u]) != sizeof(T))
                return false;
            std::uint64_t rows = 1u;
            for(std::uint32_t d = 0; d + 1u < dim; ++d)
                rows *= static_cast<std::uint64_t>(ext[d]);
            out.rowLen = static_cast<std::uint64_t>(ext[dim - 1u]);
            out.rows = rows;
            if constexpr(dim >= 2u)
            {
                // slower dimensions must be dense over rows: pitch[d] == ext[d+1] * pitch[d+1] for d < dim - 2
                for(std::uint32_t d = 0; d + 2u < dim; ++d)
                    if(static_cast<std::uint64_t>(pitch[d]) != static_cast<std::uint64_t>(ext[d + 1u]) * pitch[d + 1u])
                        return false;
                std::uint64_t const rp = static_cast<std::uint64_t>(pitch[dim - 2u]);
                out.rowPitch = (rp == out.rowLen * sizeof(T)) ? 0u : rp;
            }
            return true;
        }

        template<typename Q>
        void* streamOf(Q const& queue)
        {
            return reinterpret_cast<void*>(queue.getNativeHandle());
        }

        template<typename Q>
        void finish(Q const& queue)
        {
            if constexpr(std::is_same_v<ALPAKA_TYPEOF(queue.getQueueKind()), alpaka::queueKind::Blocking>)
                check(a3b_stream_synchronize(streamOf(queue)), "alpaka3_b200 blocking queue");
        }

        // Route transformReduce to the C ABI; false when the call is not covered.
        template<typename T, typename Q>
        bool tryTransformReduce(
            Q const& queue,
            T const& neutral,
            auto& out,
            auto const& reduceFn,
            auto const& transformFn,
            auto const&... in)
        {
            constexpr int NIN = sizeof...(in);
            constexpr int dt = dtypeOf<T>();
            if constexpr(dt < 0 || NIN < 1 || NIN > 2)
                return false;
            else if constexpr(!(alpaka::concepts::IMdSpan<std::decay_t<decltype(in)>> && ...))
                return false;
            else if constexpr(!(std::is_same_v<alpaka::trait::GetValueType_t<std::decay_t<decltype(in)>>, T> && ...))
                return false;
            else
            {
                int const rop = reduceOpOf<T>(reduceFn);
                int const xop = transformOpOf<T, NIN>(transformFn);
                if(rop < 0 || xop < 0)
                    return false;
                Layout l[NIN];
                int k = 0;
                bool ok = true;
                ((ok = ok && layoutOf<T>(in, l[k++])), ...);
                if(!ok)
                    return false;
                Layout o;
                if(!layoutOf<T>(out, o))
                    return false;
                void* const s = streamOf(queue);
                void* const outPtr = const_cast<void*>(o.ptr);
                if constexpr(NIN == 1)
                {
                    if(l[0].dense())
                        check(a3b_transform_reduce(s, dt, rop, xop, l[0].ptr, nullptr, l[0].rows * l[0].rowLen,
                                                   &neutral, outPtr),
                              "alpaka3_b200 transformReduce");
                    else if(xop == A3B_XFORM_IDENTITY)
                        check(a3b_reduce_2d(s, dt, rop, l[0].ptr, l[0].rows, l[0].rowLen, l[0].rowPitch, &neutral,
                                            outPtr),
                              "alpaka3_b200 reduce");
                    else
                        return false;
                }
                else
                {
                    if(!l[0].dense() || !l[1].dense() || l[0].rows * l[0].rowLen != l[1].rows * l[1].rowLen)
                        return false;
                    check(a3b_transform_reduce(s, dt, rop, xop, l[0].ptr, l[1].ptr, l[0].rows * l[0].rowLen,
                                               &neutral, outPtr),
                          "alpaka3_b200 transformReduce");
                }
                finish(queue);
                ++routingStats().routed;
                return true;
            }
        }

        // Route a scan to the C ABI; false when the call is not covered.
        // `buffer` is a pointer to the caller's scan buffer, or nullptr (std::nullptr_t) when the call has none.
        template<typename Q, typename B>
        bool tryScan(Q const& queue, bool inclusive, B buffer, auto& out, auto const& in)
        {
            using T = alpaka::trait::GetValueType_t<std::decay_t<decltype(in)>>;
            using TO = alpaka::trait::GetValueType_t<std::decay_t<decltype(out)>>;
            constexpr int dt = dtypeOf<std::remove_const_t<T>>();
            if constexpr(dt < 0 || !std::is_same_v<std::remove_const_t<T>, std::remove_const_t<TO>>)
                return false;
            else if constexpr(!alpaka::concepts::IMdSpan<std::decay_t<decltype(in)>>)
                return false;
            else
            {
                Layout li, lo;
                if(!layoutOf<std::remove_const_t<T>>(in, li) || !layoutOf<std::remove_const_t<T>>(out, lo))
                    return false;
                if(!li.dense() || !lo.dense() || li.rows * li.rowLen != lo.rows * lo.rowLen)
                    return false;
                void* bp = nullptr;
                std::size_t bb = 0;
                if constexpr(!std::is_null_pointer_v<B>)
                {
                    bp = const_cast<void*>(static_cast<void const*>(alpaka::onHost::data(*buffer)));
                    auto const ext = alpaka::onHost::getExtents(*buffer);
                    bb = static_cast<std::size_t>(ext.product())
                         * sizeof(alpaka::trait::GetValueType_t<std::decay_t<decltype(*buffer)>>);
                    if(bb < a3b_scan_buffer_size(dt, li.rows * li.rowLen))
                    {
                        // a buffer sized for alpaka3's own multi-level scan may be smaller: use the cached scratch
                        bp = nullptr;
                        bb = 0;
                    }
                }
                check(a3b_scan(streamOf(queue), dt, inclusive ? 1 : 0, li.ptr, const_cast<void*>(lo.ptr),
                               li.rows * li.rowLen, nullptr, bp, bb),
                      "alpaka3_b200 scan");
                finish(queue);
                ++routingStats().routed;
                return true;
            }
        }

#if defined(__CUDACC__)
        template<typename T, int V>
        __device__ __forceinline__ auto toSimd(elementwise::Vec<T, V> const& x)
        {
            return alpaka::Simd<T, static_cast<std::uint32_t>(V)>([&](auto i) { return x.v[i]; });
        }

        //! Calls an alpaka3 functor with alpaka::Simd packs, as alpaka3's SimdTransformKernel does.
        template<typename Fn, typename TOut, typename... TIn>
        struct SimdOp
        {
            Fn fn;

            template<int V>
            __device__ __forceinline__ void apply(
                elementwise::Vec<TOut, V>& out,
                elementwise::Vec<TIn, V> const&... in) const
            {
                auto const r = fn(toSimd(in)...);
#    pragma unroll
                for(int k = 0; k < V; ++k)
                    out.v[k] = static_cast<TOut>(r[k]);
            }
        };

        template<typename F, typename TOut, std::uint32_t V, typename... TIn>
        concept SimdCallable = requires(F const& f, alpaka::Simd<TIn, V> const&... s) {
            { f(s...)[0u] } -> std::convertible_to<TOut>;
        };

        template<typename F, typename TOut, typename... TIn>
        concept ScalarCallable = requires(F const& f, TIn const&... a) {
            { f(a...) } -> std::convertible_to<TOut>;
        };

        //! 1: call with SIMD packs, 2: call with scalars (ScalarFunc), 0: not covered (stencil or accelerator functors)
        template<typename F, typename TOut, typename... TIn>
        constexpr int transformKind()
        {
            constexpr std::uint32_t W = static_cast<std::uint32_t>(elementwise::packWidth<TOut, TIn...>());
            if constexpr(!std::is_arithmetic_v<TOut> || !(std::is_arithmetic_v<TIn> && ...))
                return 0;
            else if constexpr(alpaka::isSpecializationOf_v<F, alpaka::StencilFunc>)
                return 0;
            else if constexpr(alpaka::isSpecializationOf_v<F, alpaka::ScalarFunc>)
                return ScalarCallable<F, TOut, TIn...> ? 2 : 0;
            else if constexpr(SimdCallable<F, TOut, W, TIn...> && SimdCallable<F, TOut, 1u, TIn...>)
                return 1;
            else
                return 0;
        }

        template<typename T>
        elementwise::Rows<T> rowsOf(Layout const& l, bool dense)
        {
            auto* p = static_cast<T*>(const_cast<void*>(l.ptr));
            return {p, dense ? 0u : (l.rowPitch != 0u ? l.rowPitch : l.rowLen * sizeof(std::remove_const_t<T>))};
        }

        template<typename A>
        using ElemOf = std::remove_const_t<alpaka::trait::GetValueType_t<std::decay_t<A>>>;

        // Run transform on the element-wise engine; false when the call is not covered.
        template<typename Q, typename Out, typename Fn, typename... In>
        bool tryTransform(Q const& queue, Out& out, Fn const& fn, In const&... in)
        {
            using TOut = ElemOf<Out>;
            using F = std::decay_t<Fn>;
            constexpr int NIN = sizeof...(In);
            if constexpr(NIN < 1 || !(alpaka::concepts::IMdSpan<std::decay_t<In>> && ...))
                return false;
            else
            {
                constexpr int kind = transformKind<F, TOut, ElemOf<In>...>();
                if constexpr(kind == 0)
                    return false;
                else
                {
                    auto const ext = alpaka::onHost::getExtents(out);
                    if(((alpaka::onHost::getExtents(in) != ext) || ...))
                        return false;
                    Layout lo;
                    Layout li[NIN];
                    if(!layoutOf<TOut>(out, lo))
                        return false;
                    int k = 0;
                    bool ok = true;
                    ((ok = ok && layoutOf<ElemOf<In>>(in, li[k++])), ...); // a fold over "," runs left to right
                    if(!ok)
                        return false;
                    bool dense = lo.dense();
                    for(int j = 0; j < NIN; ++j)
                        dense = dense && li[j].dense();
                    std::uint64_t const rows = dense ? 1u : lo.rows;
                    std::uint64_t const rowLen = dense ? lo.rows * lo.rowLen : lo.rowLen;
                    auto const s = static_cast<cudaStream_t>(streamOf(queue));
                    using Op = std::conditional_t<
                        kind == 1,
                        SimdOp<F, TOut, ElemOf<In>...>,
                        elementwise::ScalarOp<F, TOut, ElemOf<In>...>>;
                    cudaError_t const e = [&]<std::size_t... I>(std::index_sequence<I...>)
                    {
                        return elementwise::launch(
                            s,
                            rowsOf<TOut>(lo, dense),
                            rows,
                            rowLen,
                            Op{fn},
                            rowsOf<ElemOf<In> const>(li[I], dense)...);
                    }(std::index_sequence_for<In...>{});
                    if(e == cudaErrorInvalidValue)
                        return false; // more chunks than one launch takes
                    if(e != cudaSuccess)
                        throw std::runtime_error(std::string("alpaka3_b200 transform: ") + cudaGetErrorString(e));
                    finish(queue);
                    ++routingStats().routed;
                    return true;
                }
            }
        }
#endif

        // Route fill to the C ABI; false when the call is not covered.
        template<typename Q, typename T>
        bool tryFill(Q const& queue, auto& dest, T const& value)
        {
            constexpr int dt = dtypeOf<std::remove_const_t<T>>();
            if constexpr(dt < 0 || !alpaka::concepts::IMdSpan<std::decay_t<decltype(dest)>>)
                return false;
            else
            {
                Layout l;
                if(!layoutOf<std::remove_const_t<T>>(dest, l) || !l.dense())
                    return false;
                check(a3b_fill(streamOf(queue), dt, const_cast<void*>(l.ptr), l.rows * l.rowLen, &value),
                      "alpaka3_b200 fill");
                finish(queue);
                ++routingStats().routed;
                return true;
            }
        }

        // Route iota to the C ABI: one dense output of an integer type equal to the iota's type (the values are then
        // exact whatever the order of the additions); false when the call is not covered.
        template<typename T, typename Q>
        bool tryIota(Q const& queue, T const& init, auto& out, auto const&... others)
        {
            using V = std::remove_const_t<alpaka::trait::GetValueType_t<std::decay_t<decltype(out)>>>;
            constexpr int dt = dtypeOf<V>();
            if constexpr(sizeof...(others) != 0 || dt < 0 || !std::is_integral_v<V> || !std::is_same_v<V, T>)
                return false;
            else
            {
                Layout l;
                if(!layoutOf<V>(out, l) || !l.dense())
                    return false;
                check(a3b_iota(streamOf(queue), dt, const_cast<void*>(l.ptr), l.rows * l.rowLen, &init),
                      "alpaka3_b200 iota");
                finish(queue);
                ++routingStats().routed;
                return true;
            }
        }

        template<typename Q>
        auto resolveExec(Q const& queue, auto exec)
        {
            if constexpr(std::is_same_v<std::decay_t<decltype(exec)>, alpaka::exec::AnyExecutor>)
                return alpaka::onHost::defaultExecutor(queue.getDevice());
            else
                return exec;
        }

#if defined(__CUDACC__)
        template<typename A, typename... R>
        A const& firstOf(A const& a, R const&...)
        {
            return a;
        }

        inline void engineCheck(cudaError_t e, char const* what)
        {
            if(e != cudaSuccess)
                throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
        }

        template<typename Q>
        void engineDone(Q const& queue)
        {
            finish(queue);
            ++routingStats().routed;
            ++routingStats().engine;
        }

        //! transformReduce / reduce with any functors on the B200 engine (simd_engine.cuh): fold over the lanes of
        //! the transformed packs, one launch, out[0] written by the last block.
        template<typename TApi, typename TDeviceKind, typename T, typename Q>
        void engineTransformReduce(
            Q const& queue,
            auto exec,
            T const& neutral,
            auto& out,
            auto const& reduceFn,
            auto const& transformFn,
            auto const&... in)
        {
            using TExec = std::decay_t<decltype(resolveExec(queue, exec))>;
            auto* const outPtr = const_cast<T*>(static_cast<T const*>(alpaka::onHost::data(out)));
            engineCheck(
                simd::reduce<TApi, TDeviceKind, TExec>(
                    static_cast<cudaStream_t>(streamOf(queue)),
                    alpaka::onHost::getExtents(firstOf(in...)),
                    neutral,
                    reduceFn,
                    simd::ReduceTransform<std::decay_t<decltype(transformFn)>>{transformFn},
                    outPtr,
                    alpaka::onHost::makeAccessibleOnAcc(in)...),
                "alpaka3_b200 transformReduce engine");
            engineDone(queue);
        }

        //! transform with any functor on the B200 engine: out = fn(in...) over out's extents.
        template<typename TApi, typename TDeviceKind, typename Q>
        void engineTransform(Q const& queue, auto exec, auto& out, auto const& fn, auto const&... in)
        {
            using TExec = std::decay_t<decltype(resolveExec(queue, exec))>;
            engineCheck(
                simd::each<TApi, TDeviceKind, TExec>(
                    static_cast<cudaStream_t>(streamOf(queue)),
                    alpaka::onHost::getExtents(out),
                    simd::TransformBody<std::decay_t<decltype(fn)>>{fn},
                    alpaka::onHost::makeAccessibleOnAcc(out),
                    alpaka::onHost::makeAccessibleOnAcc(in)...),
                "alpaka3_b200 transform engine");
            engineDone(queue);
        }

        //! iota into any number of outputs on the B200 engine
        template<typename TApi, typename TDeviceKind, typename T, typename Q>
        void engineIota(Q const& queue, auto exec, T const& init, auto&& out0, auto&&... outs)
        {
            using TExec = std::decay_t<decltype(resolveExec(queue, exec))>;
            auto const ext = alpaka::onHost::getExtents(out0);
            using Ext = typename std::decay_t<decltype(ext)>::UniVec;
            engineCheck(
                simd::each<TApi, TDeviceKind, TExec>(
                    static_cast<cudaStream_t>(streamOf(queue)),
                    ext,
                    simd::IotaBody<T, Ext>{Ext{ext}, init},
                    alpaka::onHost::makeAccessibleOnAcc(out0),
                    alpaka::onHost::makeAccessibleOnAcc(outs)...),
                "alpaka3_b200 iota engine");
            engineDone(queue);
        }

        //! fill of any device buffer layout on the B200 engine
        template<typename TApi, typename TDeviceKind, typename T, typename Q>
        void engineFill(Q const& queue, auto&& dest, T const& value)
        {
            using TExec = std::decay_t<decltype(alpaka::onHost::defaultExecutor(queue.getDevice()))>;
            engineCheck(
                simd::each<TApi, TDeviceKind, TExec>(
                    static_cast<cudaStream_t>(streamOf(queue)),
                    alpaka::onHost::getExtents(dest),
                    simd::FillBody<T>{value},
                    alpaka::onHost::makeAccessibleOnAcc(dest)),
                "alpaka3_b200 fill engine");
            engineDone(queue);
        }

        //! concurrent on the B200 engine: fn(acc?, SimdPtr...) over `extents`.
        template<typename TApi, typename TDeviceKind, typename Q>
        void engineConcurrent(Q const& queue, auto exec, auto const& extents, auto const& fn, auto&&... inOut)
        {
            using TExec = std::decay_t<decltype(resolveExec(queue, exec))>;
            alpaka::Vec const ext = extents;
            engineCheck(
                simd::each<TApi, TDeviceKind, TExec>(
                    static_cast<cudaStream_t>(streamOf(queue)),
                    ext,
                    simd::ConcurrentBody<std::decay_t<decltype(fn)>>{fn},
                    alpaka::onHost::makeAccessibleOnAcc(inOut)...),
                "alpaka3_b200 concurrent engine");
            engineDone(queue);
        }
#endif
    } // namespace detail
} // namespace alpaka3_b200

namespace alpaka::onHost
{
    // ------------------------------------------------------------------------------------------ transformReduce
    template<typename DataType, alpaka::concepts::DeviceKind T_DeviceKind, alpaka::concepts::QueueKind T_QueueKind>
    inline void transformReduce(
        Queue<Device<api::Cuda, T_DeviceKind>, T_QueueKind> const& queue,
        alpaka::concepts::Executor auto const exec,
        DataType const& neutralElement,
        alpaka::concepts::IMdSpan auto out,
        auto&& binaryReduceFn,
        auto&& transformFn,
        alpaka::concepts::IDataSource auto&&... in)
        requires(std::same_as<DataType, alpaka::trait::GetValueType_t<ALPAKA_TYPEOF(out)>>)
    {
        if(alpaka3_b200::detail::tryTransformReduce<DataType>(queue, neutralElement, out, binaryReduceFn, transformFn, in...))
            return;
#if defined(__CUDACC__)
        if constexpr(std::is_trivially_copyable_v<DataType>)
        {
            alpaka3_b200::detail::engineTransformReduce<api::Cuda, T_DeviceKind>(
                queue,
                exec,
                neutralElement,
                out,
                binaryReduceFn,
                transformFn,
                in...);
            return;
        }
#endif
        ++alpaka3_b200::routingStats().forwarded;
        internal::transformReduce(
            queue,
            alpaka3_b200::detail::resolveExec(queue, exec),
            neutralElement,
            out,
            ALPAKA_FORWARD(binaryReduceFn),
            ALPAKA_FORWARD(transformFn),
            ALPAKA_FORWARD(in)...);
    }

    template<typename DataType, alpaka::concepts::DeviceKind T_DeviceKind, alpaka::concepts::QueueKind T_QueueKind>
    inline void transformReduce(
        Queue<Device<api::Cuda, T_DeviceKind>, T_QueueKind> const& queue,
        DataType const& neutralElement,
        alpaka::concepts::IMdSpan auto out,
        auto&& binaryReduceFn,
        auto&& transformFn,
        alpaka::concepts::IDataSource auto&&... in)
        requires(std::same_as<DataType, alpaka::trait::GetValueType_t<ALPAKA_TYPEOF(out)>>)
    {
        transformReduce(
            queue,
            defaultExecutor(queue.getDevice()),
            neutralElement,
            out,
            ALPAKA_FORWARD(binaryReduceFn),
            ALPAKA_FORWARD(transformFn),
            ALPAKA_FORWARD(in)...);
    }

    // --------------------------------------------------------------------------------------------------- reduce
    template<typename DataType, alpaka::concepts::DeviceKind T_DeviceKind, alpaka::concepts::QueueKind T_QueueKind>
    inline void reduce(
        Queue<Device<api::Cuda, T_DeviceKind>, T_QueueKind> const& queue,
        alpaka::concepts::Executor auto const exec,
        DataType const& neutralElement,
        alpaka::concepts::IMdSpan auto out,
        auto&& binaryReduceFn,
        auto&& in) requires(std::same_as<DataType, alpaka::trait::GetValueType_t<ALPAKA_TYPEOF(out)>>)
    {
        if(alpaka3_b200::detail::tryTransformReduce<DataType>(queue, neutralElement, out, binaryReduceFn, std::identity{}, in))
            return;
#if defined(__CUDACC__)
        if constexpr(std::is_trivially_copyable_v<DataType>)
        {
            alpaka3_b200::detail::engineTransformReduce<api::Cuda, T_DeviceKind>(
                queue,
                exec,
                neutralElement,
                out,
                binaryReduceFn,
                std::identity{},
                in);
            return;
        }
#endif
        ++alpaka3_b200::routingStats().forwarded;
        internal::transformReduce(
            queue,
            alpaka3_b200::detail::resolveExec(queue, exec),
            neutralElement,
            out,
            ALPAKA_FORWARD(binaryReduceFn),
            std::identity{},
            ALPAKA_FORWARD(in));
    }

    template<typename DataType, alpaka::concepts::DeviceKind T_DeviceKind, alpaka::concepts::QueueKind T_QueueKind>
    inline void reduce(
        Queue<Device<api::Cuda, T_DeviceKind>, T_QueueKind> const& queue,
        DataType const& neutralElement,
        alpaka::concepts::IMdSpan auto out,
        auto&& binaryReduceFn,
        alpaka::concepts::IDataSource auto&& in)
        requires(std::same_as<DataType, alpaka::trait::GetValueType_t<ALPAKA_TYPEOF(out)>>)
    {
        reduce(
            queue,
            defaultExecutor(queue.getDevice()),
            neutralElement,
            out,
            ALPAKA_FORWARD(binaryReduceFn),
            ALPAKA_FORWARD(in));
    }

    // ----------------------------------------------------------------------------------------------------- scans
#define ALPAKA3_B200_SCAN_OVERLOADS(NAME, INCL, KIND)                                                                 \
    template<alpaka::concepts::DeviceKind T_DeviceKind, alpaka::concepts::QueueKind T_QueueKind>                      \
    void NAME(                                                                                                        \
        Queue<Device<api::Cuda, T_DeviceKind>, T_QueueKind> const& queue,                                             \
        alpaka::concepts::Executor auto exec,                                                                         \
        alpaka::concepts::IMdSpan auto& buffer,                                                                       \
        alpaka::concepts::IMdSpan auto& outputVec,                                                                    \
        alpaka::concepts::IDataSource auto const& inputVec)                                                           \
    {                                                                                                                 \
        if(alpaka3_b200::detail::tryScan(queue, INCL, &buffer, outputVec, inputVec))                                  \
            return;                                                                                                   \
        ++alpaka3_b200::routingStats().forwarded;                                                                     \
        auto devAcc = queue.getDevice();                                                                              \
        auto ex = alpaka3_b200::detail::resolveExec(queue, exec);                                                     \
        auto q = queue;                                                                                               \
        internal::scan<internal::KIND>(q, devAcc, ex, buffer, outputVec, inputVec);                                   \
    }                                                                                                                 \
    template<alpaka::concepts::DeviceKind T_DeviceKind, alpaka::concepts::QueueKind T_QueueKind>                      \
    void NAME(                                                                                                        \
        Queue<Device<api::Cuda, T_DeviceKind>, T_QueueKind> const& queue,                                             \
        alpaka::concepts::Executor auto exec,                                                                         \
        alpaka::concepts::IMdSpan auto& outputVec,                                                                    \
        alpaka::concepts::IDataSource auto const& inputVec)                                                           \
    {                                                                                                                 \
        if(alpaka3_b200::detail::tryScan(queue, INCL, nullptr, outputVec, inputVec))                                  \
            return;                                                                                                   \
        ++alpaka3_b200::routingStats().forwarded;                                                                     \
        auto devAcc = queue.getDevice();                                                                              \
        auto ex = alpaka3_b200::detail::resolveExec(queue, exec);                                                     \
        auto q = queue;                                                                                               \
        internal::scan<internal::KIND>(q, devAcc, ex, outputVec, inputVec);                                           \
    }                                                                                                                 \
    template<alpaka::concepts::DeviceKind T_DeviceKind, alpaka::concepts::QueueKind T_QueueKind>                      \
    void NAME##InPlace(                                                                                               \
        Queue<Device<api::Cuda, T_DeviceKind>, T_QueueKind> const& queue,                                             \
        alpaka::concepts::Executor auto exec,                                                                         \
        alpaka::concepts::IMdSpan auto& buffer,                                                                       \
        alpaka::concepts::IMdSpan auto& dataVec)                                                                      \
    {                                                                                                                 \
        if(alpaka3_b200::detail::tryScan(queue, INCL, &buffer, dataVec, dataVec))                                     \
            return;                                                                                                   \
        ++alpaka3_b200::routingStats().forwarded;                                                                     \
        auto devAcc = queue.getDevice();                                                                              \
        auto ex = alpaka3_b200::detail::resolveExec(queue, exec);                                                     \
        auto q = queue;                                                                                               \
        internal::scan<internal::KIND>(q, devAcc, ex, buffer, dataVec, dataVec);                                      \
    }                                                                                                                 \
    template<alpaka::concepts::DeviceKind T_DeviceKind, alpaka::concepts::QueueKind T_QueueKind>                      \
    void NAME##InPlace(                                                                                               \
        Queue<Device<api::Cuda, T_DeviceKind>, T_QueueKind> const& queue,                                             \
        alpaka::concepts::Executor auto exec,                                                                         \
        alpaka::concepts::IMdSpan auto& dataVec)                                                                      \
    {                                                                                                                 \
        if(alpaka3_b200::detail::tryScan(queue, INCL, nullptr, dataVec, dataVec))                                     \
            return;                                                                                                   \
        ++alpaka3_b200::routingStats().forwarded;                                                                     \
        auto devAcc = queue.getDevice();                                                                              \
        auto ex = alpaka3_b200::detail::resolveExec(queue, exec);                                                     \
        auto q = queue;                                                                                               \
        internal::scan<internal::KIND>(q, devAcc, ex, dataVec, dataVec);                                              \
    }

    ALPAKA3_B200_SCAN_OVERLOADS(exclusiveScan, false, EXCLUSIVE_SCAN)
    ALPAKA3_B200_SCAN_OVERLOADS(inclusiveScan, true, INCLUSIVE_SCAN)
#undef ALPAKA3_B200_SCAN_OVERLOADS
    // ----------------------------------------------------------------------------------------------------- iota
    template<typename T_DataType, alpaka::concepts::DeviceKind T_DeviceKind, alpaka::concepts::QueueKind T_QueueKind>
    requires(std::is_fundamental_v<T_DataType>)
    inline void iota(
        Queue<Device<api::Cuda, T_DeviceKind>, T_QueueKind> const& queue,
        alpaka::concepts::Executor auto const exec,
        T_DataType const& initValue,
        alpaka::concepts::IMdSpan auto&& out0,
        alpaka::concepts::IMdSpan auto&&... outOther)
        requires(
            std::is_convertible_v<T_DataType, alpaka::trait::GetValueType_t<ALPAKA_TYPEOF(out0)>>
            && std::conjunction_v<
                std::is_convertible<T_DataType, typename alpaka::trait::GetValueType_t<ALPAKA_TYPEOF(outOther)>>...>)
    {
        if(alpaka3_b200::detail::tryIota(queue, initValue, out0, outOther...))
            return;
#if defined(__CUDACC__)
        alpaka3_b200::detail::engineIota<api::Cuda, T_DeviceKind>(queue, exec, initValue, out0, outOther...);
        return;
#endif
        ++alpaka3_b200::routingStats().forwarded;
        internal::iota<T_DataType>(
            queue,
            alpaka3_b200::detail::resolveExec(queue, exec),
            onHost::getExtents(out0),
            initValue,
            ALPAKA_FORWARD(out0),
            ALPAKA_FORWARD(outOther)...);
    }

    template<typename T_DataType, alpaka::concepts::DeviceKind T_DeviceKind, alpaka::concepts::QueueKind T_QueueKind>
    requires(std::is_fundamental_v<T_DataType>)
    inline void iota(
        Queue<Device<api::Cuda, T_DeviceKind>, T_QueueKind> const& queue,
        T_DataType const& initValue,
        alpaka::concepts::IMdSpan auto&& out0,
        alpaka::concepts::IMdSpan auto&&... outOther)
        requires(
            std::is_convertible_v<T_DataType, alpaka::trait::GetValueType_t<ALPAKA_TYPEOF(out0)>>
            && std::conjunction_v<
                std::is_convertible<T_DataType, typename alpaka::trait::GetValueType_t<ALPAKA_TYPEOF(outOther)>>...>)
    {
        iota<T_DataType>(
            queue,
            defaultExecutor(queue.getDevice()),
            initValue,
            ALPAKA_FORWARD(out0),
            ALPAKA_FORWARD(outOther)...);
    }

    // ----------------------------------------------------------------------------------------------------- fill
    template<typename T_Value, alpaka::concepts::DeviceKind T_DeviceKind, alpaka::concepts::QueueKind T_QueueKind>
    inline void fill(Queue<Device<api::Cuda, T_DeviceKind>, T_QueueKind> const& queue, auto&& dest, T_Value elementValue)
        requires(
            std::same_as<alpaka::trait::GetValueType_t<ALPAKA_TYPEOF(dest)>, T_Value>
            && std::same_as<ALPAKA_TYPEOF(alpaka::internal::getApi(queue)), ALPAKA_TYPEOF(alpaka::internal::getApi(dest))>)
    {
        if(alpaka3_b200::detail::tryFill(queue, dest, elementValue))
            return;
#if defined(__CUDACC__)
        alpaka3_b200::detail::engineFill<api::Cuda, T_DeviceKind>(queue, dest, elementValue);
        return;
#endif
        ++alpaka3_b200::routingStats().forwarded;
        fill(queue, ALPAKA_FORWARD(dest), elementValue, internal::getExtents(dest));
    }

    // ------------------------------------------------------------------------------------------------ transform
    template<alpaka::concepts::DeviceKind T_DeviceKind, alpaka::concepts::QueueKind T_QueueKind>
    inline void transform(
        Queue<Device<api::Cuda, T_DeviceKind>, T_QueueKind> const& queue,
        alpaka::concepts::Executor auto const exec,
        alpaka::concepts::IMdSpan auto&& out,
        auto&& fn,
        alpaka::concepts::IDataSource auto&&... in)
    {
#if defined(__CUDACC__)
        if(alpaka3_b200::detail::tryTransform(queue, out, fn, in...))
            return;
        alpaka3_b200::detail::engineTransform<api::Cuda, T_DeviceKind>(queue, exec, out, fn, in...);
        return;
#endif
        ++alpaka3_b200::routingStats().forwarded;
        internal::transform(
            queue,
            alpaka3_b200::detail::resolveExec(queue, exec),
            ALPAKA_FORWARD(out),
            ALPAKA_FORWARD(fn),
            ALPAKA_FORWARD(in)...);
    }

    template<alpaka::concepts::DeviceKind T_DeviceKind, alpaka::concepts::QueueKind T_QueueKind>
    inline void transform(
        Queue<Device<api::Cuda, T_DeviceKind>, T_QueueKind> const& queue,
        alpaka::concepts::IMdSpan auto&& out,
        auto&& fn,
        alpaka::concepts::IDataSource auto&&... in)
    {
        transform(
            queue,
            defaultExecutor(queue.getDevice()),
            ALPAKA_FORWARD(out),
            ALPAKA_FORWARD(fn),
            ALPAKA_FORWARD(in)...);
    }

    // ----------------------------------------------------------------------------------------------- concurrent
    template<typename T_DataType, alpaka::concepts::DeviceKind T_DeviceKind, alpaka::concepts::QueueKind T_QueueKind>
    inline void concurrent(
        Queue<Device<api::Cuda, T_DeviceKind>, T_QueueKind> const& queue,
        alpaka::concepts::Executor auto const exec,
        alpaka::concepts::VectorOrScalar auto const& extents,
        auto&& fn,
        alpaka::concepts::IDataSource auto&&... inOut)
    {
#if defined(__CUDACC__)
        alpaka3_b200::detail::engineConcurrent<api::Cuda, T_DeviceKind>(queue, exec, extents, fn, inOut...);
#else
        ++alpaka3_b200::routingStats().forwarded;
        internal::concurrent<T_DataType>(
            queue,
            alpaka3_b200::detail::resolveExec(queue, exec),
            extents,
            ALPAKA_FORWARD(fn),
            ALPAKA_FORWARD(inOut)...);
#endif
    }

    template<typename T_DataType, alpaka::concepts::DeviceKind T_DeviceKind, alpaka::concepts::QueueKind T_QueueKind>
    inline void concurrent(
        Queue<Device<api::Cuda, T_DeviceKind>, T_QueueKind> const& queue,
        alpaka::concepts::VectorOrScalar auto const& extents,
        auto&& fn,
        alpaka::concepts::IDataSource auto&&... inOut)
    {
        concurrent<T_DataType>(
            queue,
            defaultExecutor(queue.getDevice()),
            extents,
            ALPAKA_FORWARD(fn),
            ALPAKA_FORWARD(inOut)...);
    }
} // namespace alpaka::onHost

#if defined(__CUDACC__)
namespace alpaka::onHost::internal
{
    // queue.enqueue(FrameSpec, KernelBundle{K{}, op, arg0, args...}) of a SIMD for-each kernel (see
    // alpaka3_b200::IsSimdForEachKernel) on a CUDA queue: the op runs on the B200 SIMD engine over arg0's extents, in
    // place of alpaka3's own launch (include/alpaka/api/unifiedCudaHip/Queue.hpp:441-460).
    template<
        typename T_Device,
        alpaka::concepts::UnifiedCudaHipExecutor T_Executor,
        typename T_NumFrames,
        typename T_FrameExtents,
        typename K,
        typename Op,
        typename A0,
        typename... A>
    requires(alpaka3_b200::IsSimdForEachKernel<std::decay_t<K>>::value)
    struct Enqueue::Kernel<
        unifiedCudaHip::Queue<T_Device>,
        FrameSpec<T_NumFrames, T_FrameExtents, T_Executor>,
        KernelBundle<K, Op, A0, A...>>
    {
        void operator()(
            unifiedCudaHip::Queue<T_Device>& queue,
            FrameSpec<T_NumFrames, T_FrameExtents, T_Executor> const&,
            KernelBundle<K, Op, A0, A...> const& bundle) const
        {
            using TApi = ALPAKA_TYPEOF(alpaka::internal::getApi(queue));
            using TDeviceKind = ALPAKA_TYPEOF(queue.getDeviceKind());
            auto const stream = static_cast<cudaStream_t>(queue.getNativeHandle());
            alpaka::apply(
                [&](auto const& op, auto const& arg0, auto const&... args)
                {
                    alpaka3_b200::detail::engineCheck(
                        alpaka3_b200::simd::each<TApi, TDeviceKind, T_Executor>(
                            stream,
                            arg0.getExtents(),
                            alpaka3_b200::simd::AccFirstBody<std::decay_t<decltype(op)>>{op},
                            arg0,
                            args...),
                        "alpaka3_b200 SIMD for-each kernel");
                },
                bundle.m_args);
            queue.conditionalWait();
            ++alpaka3_b200::routingStats().routed;
            ++alpaka3_b200::routingStats().engine;
        }
    };
} // namespace alpaka::onHost::internal
#endif
