/* alpaka3 functors shared by the reference harnesses (oracle/ref_harness.cpp on the host backend,
 * oracle/ref_cuda_bench.cpp on the CUDA backend). Test and measurement infrastructure only.
 *
 * The BabelStream operation functors live in the reference's benchmark TU
 * (benchmark/babelstream/src/babelStreamMainTest.cpp:61-141) and cannot be included; each one here states the same
 * element-wise assignment as the reference op it mirrors, driven through SimdAlgo::concurrent like the reference's
 * SimdForEachKernel.
 */
#pragma once

#include <alpaka/alpaka.hpp>

namespace a3b_ref
{
    using namespace alpaka;

    // ---- BabelStream element-wise operations (babelStreamMainTest.cpp:61-141) ----
    constexpr double kInitA = 0.1, kInitB = 0.2, kInitC = 0.0, kScalar = 0.4; // babelStreamCommon.hpp:31,45-48

    struct ForEach
    {
        ALPAKA_FN_ACC void operator()(
            auto const& acc,
            auto const& func,
            alpaka::concepts::IDataSource auto arg0,
            alpaka::concepts::IDataSource auto... args) const
        {
            onAcc::SimdAlgo{onAcc::worker::threadsInGrid}.concurrent(acc, arg0.getExtents(), func, arg0, args...);
        }
    };

    struct InitOp
    {
        constexpr void operator()(auto const&, auto a, auto b, auto c) const
        {
            using S = ALPAKA_TYPEOF(a.load());
            a = S::fill(kInitA);
            b = S::fill(kInitB);
            c = S::fill(kInitC);
        }
    };

    struct CopyOp
    {
        constexpr void operator()(auto const&, auto const a, auto c) const
        {
            c = a.load();
        }
    };

    struct MulOp
    {
        constexpr void operator()(auto const&, auto b, auto const c) const
        {
            using T = trait::GetValueType_t<ALPAKA_TYPEOF(b)>;
            b = static_cast<T>(kScalar) * c.load();
        }
    };

    struct AddOp
    {
        constexpr void operator()(auto const&, auto const a, auto b, auto c) const
        {
            c = a.load() + b.load();
        }
    };

    struct TriadOp
    {
        constexpr void operator()(auto const&, auto a, auto const b, auto const c) const
        {
            using T = trait::GetValueType_t<ALPAKA_TYPEOF(a)>;
            a = b.load() + static_cast<T>(kScalar) * c.load();
        }
    };

    struct NStreamOp
    {
        constexpr void operator()(auto const&, auto a, auto const b, auto const c) const
        {
            using T = trait::GetValueType_t<ALPAKA_TYPEOF(a)>;
            a = a.load() + b.load() + static_cast<T>(kScalar) * c.load();
        }
    };

    struct Product
    {
        constexpr auto operator()(auto&& x, auto&& y) const
        {
            return x * y;
        }
    };

    struct Square
    {
        constexpr auto operator()(auto&& x) const
        {
            return x * x;
        }
    };

} // namespace a3b_ref
