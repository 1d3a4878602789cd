/* alpaka3's own algorithm tests, re-expressed without Catch2, run through alpaka3's public onHost API on a CUDA queue
 * with the alpaka3_b200 binding included: every call goes to libalpaka3_b200.so (C ABI) or to a B200 engine compiled
 * here with the test's functors; none is forwarded to alpaka3's own CUDA backend. Mirrors
 *   test/unit/algorithm/scan.cpp:74-197 (int iota, 4 sizes, exclusive/inclusive x out-of-place / in-place x
 *     with/without buffer, std::exclusive_scan / std::inclusive_scan as ground truth),
 *   test/unit/algorithm/reduce.cpp:135-232 (int iota over N-D extents, plus / ScalarFunc min / max, and the
 *     LinearizedIdxGenerator source),
 *   test/unit/algorithm/transformReduce.cpp:173-260 (six reduce / transform pairs over the same extents: std::plus,
 *     StencilFunc with and without an accelerator, an up-casting transform, a ScalarFunc lambda, a ScalarFunc min),
 *   test/unit/algorithm/transform.cpp:147-180 (std::minus, std::plus, StencilFunc, ScalarFunc with and without an
 *     accelerator argument, up-casting functors) and :399-405 (the SimdPtr cross stencil over 1-D..4-D extents),
 *   test/unit/algorithm/concurrent.cpp (StencilAddWithAcc, StencilAddMin over the same extents),
 *   test/unit/algorithm/iota.cpp:13-118 and element-wise fill,
 * plus BabelStream's dot (benchmark/babelstream/src/babelStreamMainTest.cpp:135-141, 337-345), a large in-place
 * transform with a ragged end, and a ScalarFunc x * |x| on negative inputs (a functor that agrees with x * x on
 * positive values). Prints "PASS routed=<n> engine=<e> forwarded=<m>" and exits 0, or lists the failures and exits 1. */
#include <alpaka3_b200/alpaka_backend.hpp>

#include <cstdio>
#include <cstdlib>
#include <numeric>
#include <vector>

using namespace alpaka;

namespace
{
    int failures = 0;

    void expect(bool ok, char const* what, long long a = 0, long long b = 0)
    {
        if(!ok)
        {
            ++failures;
            std::printf("FAIL %s (%lld vs %lld)\n", what, a, b);
        }
    }

    struct MinValue
    {
        constexpr auto operator()(auto const& a, auto const& b) const
        {
            return math::min(a, b);
        }
    };

    ALPAKA_FN_ACC void alpakaAtomicInvoke(MinValue const&, onAcc::concepts::Acc auto const& acc, auto* d, auto s)
    {
        onAcc::atomicMin(acc, d, s);
    }

    struct MaxValue
    {
        constexpr auto operator()(auto const& a, auto const& b) const
        {
            return math::max(a, b);
        }
    };

    ALPAKA_FN_ACC void alpakaAtomicInvoke(MaxValue const&, onAcc::concepts::Acc auto const& acc, auto* d, auto s)
    {
        onAcc::atomicMax(acc, d, s);
    }

    struct DotMultiplication
    {
        constexpr auto operator()(concepts::Simd auto&& simdA, concepts::Simd auto&& simdB) const
        {
            return simdA * simdB;
        }
    };

    struct Cube // no known type: runs on the engine with the functor itself
    {
        constexpr auto operator()(auto const& x) const
        {
            return x * x * x;
        }
    };

    struct SignedSquare
    {
        ALPAKA_FN_ACC float operator()(float x) const
        {
            return x * (x < 0.f ? -x : x);
        }
    };

    template<typename T>
    void checkScan(auto& queue, auto& host, auto& dev, std::size_t n, bool inclusive, char const* what)
    {
        auto back = onHost::allocHost<T>(Vec{n});
        onHost::memcpy(queue, back, dev);
        onHost::wait(queue);
        std::vector<T> want(n);
        if(inclusive)
            std::inclusive_scan(host.data(), host.data() + n, want.data());
        else
            std::exclusive_scan(host.data(), host.data() + n, want.data(), T{0});
        std::size_t bad = 0;
        for(std::size_t i = 0; i < n; ++i)
            bad += back.data()[i] != want[i];
        expect(bad == 0, what, static_cast<long long>(bad), static_cast<long long>(n));
    }

    void scanTests(auto& dev, auto& queue, auto exec)
    {
        using T = int;
        for(std::size_t n : {std::size_t{12}, std::size_t{1024}, std::size_t{654321}, std::size_t{20971520}})
        {
            auto ext = Vec{n};
            auto in = onHost::alloc<T>(dev, ext);
            auto out = onHost::alloc<T>(dev, ext);
            auto host = onHost::allocHostLike(in);
            T c = 0;
            for(auto& v : host)
                v = c++;
            auto buffer = onHost::alloc<std::byte>(dev, onHost::getScanBufferSize<T>(in.getExtents()));
            for(int incl = 0; incl < 2; ++incl)
            {
                onHost::memcpy(queue, in, host);
                if(incl)
                    onHost::inclusiveScan(queue, exec, out, in);
                else
                    onHost::exclusiveScan(queue, exec, out, in);
                checkScan<T>(queue, host, out, n, incl, "scan, no buffer");
                if(incl)
                    onHost::inclusiveScanInPlace(queue, exec, in);
                else
                    onHost::exclusiveScanInPlace(queue, exec, in);
                checkScan<T>(queue, host, in, n, incl, "scan, no buffer, in-place");
                onHost::memcpy(queue, in, host);
                if(incl)
                    onHost::inclusiveScan(queue, exec, buffer, out, in);
                else
                    onHost::exclusiveScan(queue, exec, buffer, out, in);
                checkScan<T>(queue, host, out, n, incl, "scan, with buffer");
                if(incl)
                    onHost::inclusiveScanInPlace(queue, exec, buffer, in);
                else
                    onHost::exclusiveScanInPlace(queue, exec, buffer, in);
                checkScan<T>(queue, host, in, n, incl, "scan, with buffer, in-place");
            }
        }
    }

    // functors of test/unit/algorithm/transform.cpp
    struct StencilAdd
    {
        constexpr auto operator()(concepts::SimdPtr auto const& a, concepts::SimdPtr auto const& b) const
        {
            return a.load() + b.load();
        }
    };

    struct ScalarMinPlusOne
    {
        constexpr auto operator()(int const& a, int const& b) const
        {
            return math::min(a + 1, b);
        }
    };

    struct ScalarOpWithAcc
    {
        constexpr auto operator()(onAcc::concepts::Acc auto const&, auto const& a, auto const& b) const
        {
            using ValueType = trait::GetValueType_t<ALPAKA_TYPEOF(a)>;
            return math::min(a + ValueType{1}, +b);
        }
    };

    struct AddUpCast
    {
        constexpr auto operator()(concepts::Simd auto const& a, concepts::Simd auto const& b) const
        {
            return pCast<std::size_t>(a + b);
        }
    };

    struct AddUpCastWithAcc
    {
        constexpr auto operator()(
            onAcc::concepts::Acc auto const&,
            concepts::Simd auto const& a,
            concepts::Simd auto const& b) const
        {
            return pCast<std::size_t>(a + b);
        }
    };

    //! out = fn(a, b) with a[i] = i, b[i] = 3 - 2 i over `extents`; checks every element against `want` and whether
    //! the call ran on the element-wise engine (routed) or on alpaka3's own backend (forwarded).
    template<typename TOut>
    void transformOne(auto& dev, auto& queue, auto exec, auto extents, auto fn, auto want, bool routed, char const* what)
    {
        using T = int;
        auto a = onHost::alloc<T>(dev, extents);
        auto b = onHost::allocLike(dev, a);
        auto ha = onHost::allocHostLike(a);
        auto hb = onHost::allocHostLike(b);
        T c = 0;
        for(auto& v : ha)
            v = c++;
        c = 0;
        for(auto& v : hb)
            v = 3 - 2 * c++;
        onHost::memcpy(queue, a, ha);
        onHost::memcpy(queue, b, hb);
        auto out = onHost::alloc<TOut>(dev, extents);
        auto ho = onHost::allocHostLike(out);
        auto const before = alpaka3_b200::routingStats().routed.load();
        onHost::transform(queue, exec, out, fn, a, b);
        onHost::memcpy(queue, ho, out);
        onHost::wait(queue);
        expect((alpaka3_b200::routingStats().routed.load() != before) == routed, what, routed ? 1 : 0, 0);
        long long i = 0;
        int bad = 0;
        for(auto const& v : ho)
        {
            T const x = static_cast<T>(i), y = static_cast<T>(3 - 2 * i);
            if(v != static_cast<TOut>(want(x, y)) && bad++ < 3)
                expect(false, what, static_cast<long long>(v), static_cast<long long>(want(x, y)));
            ++i;
        }
    }

    void transformTests(auto& dev, auto& queue, auto exec, auto extents)
    {
        auto minus = [](int x, int y) { return x - y; };
        auto plus = [](int x, int y) { return x + y; };
        auto minPlusOne = [](int x, int y) { return std::min(x + 1, y); };
        transformOne<int>(dev, queue, exec, extents, std::minus{}, minus, true, "transform minus");
        transformOne<int>(dev, queue, exec, extents, std::plus{}, plus, true, "transform plus");
        transformOne<int>(dev, queue, exec, extents, StencilFunc{StencilAdd{}}, plus, true, "transform stencil");
        transformOne<int>(dev, queue, exec, extents, ScalarFunc{ScalarMinPlusOne{}}, minPlusOne, true, "transform scalar");
        transformOne<int>(dev, queue, exec, extents, ScalarFunc{ScalarOpWithAcc{}}, minPlusOne, true, "transform scalar acc");
        transformOne<std::size_t>(dev, queue, exec, extents, AddUpCast{}, plus, true, "transform up-cast");
        transformOne<std::size_t>(dev, queue, exec, extents, AddUpCastWithAcc{}, plus, true, "transform up-cast acc");
    }

    struct TwiceAndOne
    {
        constexpr auto operator()(auto const& x) const
        {
            return x * 2.f + 1.f;
        }
    };

    //! the element-wise engine on a large 1-D array with a ragged end, in place
    void transformLarge(auto& dev, auto& queue, auto exec)
    {
        std::size_t const n = (std::size_t{1} << 22) + 5;
        auto a = onHost::alloc<float>(dev, Vec{n});
        auto ha = onHost::allocHostLike(a);
        float c = 0.f;
        for(auto& v : ha)
            v = c++ * 0.25f;
        onHost::memcpy(queue, a, ha);
        auto const before = alpaka3_b200::routingStats().routed.load();
        onHost::transform(queue, exec, a, TwiceAndOne{}, a);
        auto h2 = onHost::allocHostLike(a);
        onHost::memcpy(queue, h2, a);
        onHost::wait(queue);
        expect(alpaka3_b200::routingStats().routed.load() == before + 1, "transform large routed");
        std::size_t i = 0, bad = 0;
        for(auto const& v : h2)
        {
            float const want = (static_cast<float>(i) * 0.25f) * 2.f + 1.f;
            if(v != want && bad++ < 3)
                expect(false, "transform large", static_cast<long long>(v), static_cast<long long>(want));
            ++i;
        }
    }

    //! iota<size_t> with init 42 into one buffer, then init 43 into two (test/unit/algorithm/iota.cpp:13-85); element
    //! by element in the extents' row-major order. One dense output goes to the C ABI, two outputs to alpaka3.
    void iotaOne(auto& dev, auto& queue, auto exec, auto extents)
    {
        using T = std::size_t;
        auto b0 = onHost::alloc<T>(dev, extents);
        auto b1 = onHost::allocLike(dev, b0);
        auto h0 = onHost::allocHostLike(b0);
        auto h1 = onHost::allocHostLike(b1);
        for(int outputs = 1; outputs <= 2; ++outputs)
        {
            T const init = outputs == 1 ? T{42} : T{43};
            onHost::memset(queue, b0, 0u);
            onHost::memset(queue, b1, 0u);
            if(outputs == 1)
                onHost::iota<T>(queue, exec, init, b0);
            else
                onHost::iota<T>(queue, exec, init, b0, b1);
            onHost::memcpy(queue, h0, b0);
            onHost::memcpy(queue, h1, b1);
            onHost::wait(queue);
            T want = init;
            int bad = 0;
            auto it1 = h1.begin();
            for(auto const& v : h0)
            {
                T const w1 = *it1;
                ++it1;
                if((v != want || (outputs == 2 && w1 != want)) && bad++ < 3)
                    expect(false, outputs == 1 ? "iota" : "iota two outputs", static_cast<long long>(v),
                           static_cast<long long>(want));
                ++want;
            }
        }
        // fill: element-wise value into the same buffer
        onHost::fill(queue, b0, T{7});
        onHost::memcpy(queue, h0, b0);
        onHost::wait(queue);
        for(auto const& v : h0)
            if(v != T{7})
            {
                expect(false, "fill", static_cast<long long>(v), 7);
                break;
            }
    }

    template<typename T>
    T hostReduce(int op, std::size_t n, T init)
    {
        T r = init;
        for(std::size_t i = 0; i < n; ++i)
        {
            T const v = static_cast<T>(i);
            r = op == 0 ? static_cast<T>(static_cast<unsigned>(r) + static_cast<unsigned>(v)) : (op == 1 ? std::min(r, v) : std::max(r, v));
        }
        return r;
    }

    void reduceOne(auto& dev, auto& queue, auto exec, auto extents)
    {
        using T = int;
        auto in = onHost::alloc<T>(dev, extents);
        auto host = onHost::allocHostLike(in);
        T c = 0;
        for(auto& v : host)
            v = c++;
        onHost::memcpy(queue, in, host);
        auto out = onHost::alloc<T>(dev, extents.fill(1));
        auto outHost = onHost::allocHostLike(out);
        std::size_t const n = static_cast<std::size_t>(extents.product());
        for(int op = 0; op < 3; ++op)
        {
            if(op == 0)
                onHost::reduce(queue, exec, T{0}, out, std::plus{}, in);
            else if(op == 1)
                onHost::reduce(queue, exec, std::numeric_limits<T>::max(), out, ScalarFunc{MinValue{}}, in);
            else
                onHost::reduce(queue, exec, std::numeric_limits<T>::min(), out, ScalarFunc{MaxValue{}}, in);
            onHost::memcpy(queue, outHost, out);
            onHost::wait(queue);
            T const want = hostReduce<T>(op, n, op == 0 ? 0 : (op == 1 ? std::numeric_limits<T>::max() : std::numeric_limits<T>::min()));
            expect(*outHost.data() == want, "reduce", *outHost.data(), want);
        }
        // generator source (not device memory): the engine reads it through SimdPtr like alpaka3 does
        auto generator = LinearizedIdxGenerator{extents};
        onHost::reduce(queue, exec, T{0}, out, std::plus{}, generator);
        onHost::memcpy(queue, outHost, out);
        onHost::wait(queue);
        expect(*outHost.data() == hostReduce<T>(0, n, 0), "reduce generator", *outHost.data(), hostReduce<T>(0, n, 0));
    }

    void transformReduceTests(auto& dev, auto& queue, auto exec)
    {
        // BabelStream dot: a = 0.1, b = 0.2 over 2^20 doubles -> N * a * b
        std::size_t const n = std::size_t{1} << 20;
        auto a = onHost::alloc<double>(dev, Vec{n});
        auto b = onHost::allocLike(dev, a);
        onHost::fill(queue, a, 0.1);
        onHost::fill(queue, b, 0.2);
        auto out = onHost::alloc<double>(dev, Vec{std::size_t{1}});
        auto outHost = onHost::allocHostLike(out);
        onHost::transformReduce(queue, exec, 0.0, out, std::plus{}, DotMultiplication{}, a, b);
        onHost::memcpy(queue, outHost, out);
        onHost::wait(queue);
        double const want = static_cast<double>(n) * 0.1 * 0.2;
        expect(std::abs(*outHost.data() - want) <= 1e-12 * want, "dot", static_cast<long long>(*outHost.data()), static_cast<long long>(want));
        // a transform of no known type: the engine calls it with SIMD packs
        onHost::transformReduce(queue, exec, 0.0, out, std::plus{}, Cube{}, a);
        onHost::memcpy(queue, outHost, out);
        onHost::wait(queue);
        double const want2 = static_cast<double>(n) * (0.1 * 0.1 * 0.1);
        expect(std::abs(*outHost.data() - want2) <= 1e-9 * want2, "transformReduce cube", 0, 0);
        // x * |x| agrees with x * x on small positive values (value probing would take it for a square) but not on
        // negative ones: sum over x_i = -(i % 7) * 0.5 must be -sum x_i^2
        std::size_t const m = 100003;
        auto neg = onHost::alloc<float>(dev, Vec{m});
        auto hneg = onHost::allocHostLike(neg);
        double wantNeg = 0.0;
        for(std::size_t i = 0; i < m; ++i)
        {
            float const x = -static_cast<float>(i % 7u) * 0.5f;
            hneg.data()[i] = x;
            wantNeg -= static_cast<double>(x) * x;
        }
        onHost::memcpy(queue, neg, hneg);
        auto fout = onHost::alloc<float>(dev, Vec{std::size_t{1}});
        auto fhost = onHost::allocHostLike(fout);
        onHost::transformReduce(queue, exec, 0.f, fout, std::plus{}, ScalarFunc{SignedSquare{}}, neg);
        onHost::memcpy(queue, fhost, fout);
        onHost::wait(queue);
        expect(std::abs(*fhost.data() - wantNeg) <= 1e-5 * std::abs(wantNeg), "x*|x| on negative inputs",
               static_cast<long long>(*fhost.data()), static_cast<long long>(wantNeg));
    }

    // functors of test/unit/algorithm/transformReduce.cpp:20-82
    struct StencilAddWithAcc
    {
        constexpr auto operator()(
            onAcc::concepts::Acc auto const&,
            concepts::SimdPtr auto const& a,
            concepts::SimdPtr auto const& b) const
        {
            return a.load() + b.load();
        }
    };

    struct MinPlusOne
    {
        ALPAKA_FN_ACC int operator()(int const& a, int const& b) const
        {
            auto lhs = a + 1;
            return math::min(lhs, b);
        }
    };

    //! transformReduce(neutral, out, reduceFn, transformFn, iota, iota) against a host fold
    template<typename TOut>
    void transformReduceOne(
        auto& dev,
        auto& queue,
        auto exec,
        auto extents,
        TOut neutral,
        auto reduceFn,
        auto transformFn,
        auto reduceRef,
        auto transformRef,
        char const* what)
    {
        using T = int;
        auto in0 = onHost::alloc<T>(dev, extents);
        auto in1 = onHost::allocLike(dev, in0);
        auto host = onHost::allocHostLike(in0);
        T c = 0;
        for(auto& v : host)
            v = c++;
        onHost::memcpy(queue, in0, host);
        onHost::memcpy(queue, in1, host);
        auto out = onHost::alloc<TOut>(dev, extents.fill(1));
        auto outHost = onHost::allocHostLike(out);
        onHost::transformReduce(queue, exec, neutral, out, reduceFn, transformFn, in0, in1);
        onHost::memcpy(queue, outHost, out);
        onHost::wait(queue);
        TOut want = neutral;
        std::size_t const n = static_cast<std::size_t>(extents.product());
        for(std::size_t i = 0; i < n; ++i)
            want = reduceRef(want, transformRef(static_cast<T>(i), static_cast<T>(i)));
        expect(*outHost.data() == want, what, static_cast<long long>(*outHost.data()), static_cast<long long>(want));
    }

    void transformReducePins(auto& dev, auto& queue, auto exec, auto extents)
    {
        // int + wraps as two's complement on the device; the host fold does the same in unsigned arithmetic
        auto wrapPlus = [](int a, int b) { return static_cast<int>(static_cast<unsigned>(a) + static_cast<unsigned>(b)); };
        auto minPlusOne = [](int a, int b) { return std::min(a + 1, b); };
        auto upCast = [](int a, int b) { return static_cast<std::size_t>(a + b); };
        auto minRef = [](int a, int b) { return std::min(a, b); };
        transformReduceOne<int>(dev, queue, exec, extents, 0, std::plus{}, std::plus{}, wrapPlus, wrapPlus,
                                "transformReduce plus(plus)");
        transformReduceOne<int>(dev, queue, exec, extents, 0, std::plus{}, StencilFunc{StencilAdd{}}, wrapPlus,
                                wrapPlus, "transformReduce plus(stencil)");
        transformReduceOne<int>(dev, queue, exec, extents, 0, std::plus{}, StencilFunc{StencilAddWithAcc{}},
                                wrapPlus, wrapPlus, "transformReduce plus(stencil acc)");
        transformReduceOne<std::size_t>(dev, queue, exec, extents, std::size_t{0}, std::plus{}, AddUpCastWithAcc{},
                                        std::plus<std::size_t>{}, upCast, "transformReduce plus(up-cast acc)");
        transformReduceOne<int>(dev, queue, exec, extents, 0, std::plus{}, ScalarFunc{MinPlusOne{}}, wrapPlus,
                                minPlusOne, "transformReduce plus(scalar)");
        transformReduceOne<int>(dev, queue, exec, extents, std::numeric_limits<int>::max(), ScalarFunc{MinValue{}},
                                std::plus{}, minRef, wrapPlus, "transformReduce min(plus)");
    }

    // functors of test/unit/algorithm/concurrent.cpp
    struct ConcurrentAddWithAcc
    {
        constexpr void operator()(
            onAcc::concepts::Acc auto const&,
            concepts::SimdPtr auto a,
            concepts::SimdPtr auto const& b) const
        {
            a = a.load() + b.load();
        }
    };

    struct ConcurrentAddMin
    {
        constexpr void operator()(concepts::SimdPtr auto a, concepts::SimdPtr auto const& b) const
        {
            constexpr uint32_t simdWidth = a.width();
            alpaka::concepts::Simd auto aSimd = a.load();
            alpaka::concepts::Simd auto bSimd = b.load();
            for(uint32_t idx = 0u; idx < simdWidth; ++idx)
                aSimd[idx] += math::min(+aSimd[idx], +bSimd[idx]);
            a = aSimd;
        }
    };

    // BabelStream's kernel and ops in the benchmark's form (benchmark/babelstream/src/babelStreamMainTest.cpp:61-141):
    // enqueued with queue.enqueue(FrameSpec, KernelBundle{SimdForEachKernel{}, op, a, b, c}). The build lists
    // SimdForEachKernel in ALPAKA3_B200_SIMD_FOR_EACH_KERNELS, so these launches run on the SIMD engine.
    constexpr double kInitA = 0.1, kInitB = 0.2, kInitC = 0.0, kScalar = 0.4;

    struct CopyOpLike
    {
    };

    struct SimdForEachKernel
    {
        ALPAKA_FN_ACC void operator()(
            auto const& acc,
            auto const& func,
            alpaka::concepts::IDataSource auto arg0,
            alpaka::concepts::IDataSource auto... args) const
        {
            auto simdGrid = onAcc::SimdAlgo{onAcc::worker::threadsInGrid};
            simdGrid.concurrent(acc, arg0.getExtents(), func, arg0, args...);
        }
    };

    static_assert(alpaka3_b200::IsSimdForEachKernel<SimdForEachKernel>::value, "listed at compile time");
    static_assert(!alpaka3_b200::IsSimdForEachKernel<CopyOpLike>::value, "not listed");

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

    //! the benchmark's run sequence (init; runs x copy, mul, add, triad, dot; then nstream) against the uniform
    //! values the host computes; counts the launches that ran on the engine
    template<typename T>
    void babelStreamKernels(auto& dev, auto& queue, auto exec, std::uint32_t n, int runs, double tol)
    {
        auto a = onHost::alloc<T>(dev, n);
        auto b = onHost::allocLike(dev, a);
        auto c = onHost::allocLike(dev, a);
        auto frames = onHost::FrameSpec{(n + 512u * 8u - 1u) / (512u * 8u), 512u, exec};
        auto const before = alpaka3_b200::routingStats().engine.load();
        queue.enqueue(frames, KernelBundle{SimdForEachKernel{}, InitOp{}, a, b, c});
        T ha = static_cast<T>(kInitA), hb = static_cast<T>(kInitB), hc = static_cast<T>(kInitC);
        T const s = static_cast<T>(kScalar);
        auto out = onHost::alloc<T>(dev, std::uint32_t{1});
        auto hout = onHost::allocHostLike(out);
        for(int r = 0; r < runs; ++r)
        {
            queue.enqueue(frames, KernelBundle{SimdForEachKernel{}, CopyOp{}, a, c});
            queue.enqueue(frames, KernelBundle{SimdForEachKernel{}, MulOp{}, b, c});
            queue.enqueue(frames, KernelBundle{SimdForEachKernel{}, AddOp{}, a, b, c});
            queue.enqueue(frames, KernelBundle{SimdForEachKernel{}, TriadOp{}, a, b, c});
            hc = ha;
            hb = s * hc;
            hc = ha + hb;
            ha = hb + s * hc;
        }
        onHost::transformReduce(queue, exec, T{0}, out, std::plus{}, DotMultiplication{}, a, b);
        queue.enqueue(frames, KernelBundle{SimdForEachKernel{}, NStreamOp{}, a, b, c});
        T const dotWant = static_cast<T>(n) * ha * hb;
        ha = ha + hb + s * hc;
        auto h = onHost::allocHostLike(a);
        onHost::memcpy(queue, hout, out);
        onHost::memcpy(queue, h, a);
        onHost::wait(queue);
        expect(
            alpaka3_b200::routingStats().engine.load() - before == static_cast<std::uint64_t>(2 + 4 * runs + 1),
            "babelstream kernels on the engine",
            static_cast<long long>(alpaka3_b200::routingStats().engine.load() - before),
            2 + 4 * runs + 1);
        std::size_t bad = 0;
        for(auto const& v : h)
            bad += std::abs(static_cast<double>(v) - static_cast<double>(ha)) > tol * std::abs(static_cast<double>(ha));
        expect(bad == 0, "babelstream a after nstream", static_cast<long long>(bad), 0);
        expect(std::abs(static_cast<double>(*hout.data()) - static_cast<double>(dotWant)) <= tol * std::abs(static_cast<double>(dotWant)),
               "babelstream dot", 0, 0);
    }

    //! concurrent<int>(extents, fn, a, b) with a = b = iota; a must become want(i, i)
    void concurrentOne(auto& dev, auto& queue, auto exec, auto extents, auto fn, auto want, char const* what)
    {
        using T = int;
        auto a = onHost::alloc<T>(dev, extents);
        auto b = onHost::allocLike(dev, a);
        auto host = onHost::allocHostLike(a);
        T c = 0;
        for(auto& v : host)
            v = c++;
        onHost::memcpy(queue, a, host);
        onHost::memcpy(queue, b, host);
        onHost::concurrent<T>(queue, exec, extents, fn, a, b);
        auto back = onHost::allocHostLike(a);
        onHost::memcpy(queue, back, a);
        onHost::wait(queue);
        T i = 0;
        int bad = 0;
        for(auto const& v : back)
        {
            if(v != want(i, i) && bad++ < 3)
                expect(false, what, v, want(i, i));
            ++i;
        }
    }

    void concurrentPins(auto& dev, auto& queue, auto exec, auto extents)
    {
        concurrentOne(dev, queue, exec, extents, ConcurrentAddWithAcc{}, [](int x, int y) { return x + y; },
                      "concurrent add acc");
        concurrentOne(dev, queue, exec, extents, ConcurrentAddMin{}, [](int x, int y) { return x + std::min(x, y); },
                      "concurrent add min");
    }

    // test/unit/algorithm/transform.cpp: the cross stencil over the inner volume of a halo-padded buffer
    struct CrossStencil
    {
        constexpr auto operator()(concepts::SimdPtr auto const& in) const
        {
            using VecIdxType = typename ALPAKA_TYPEOF(in)::IdxType;
            concepts::Simd auto result = in.load();
            using SimdType = ALPAKA_TYPEOF(result);
            result += SimdType::fill(42);
            for(uint32_t d = 0u; d < VecIdxType::dim(); ++d)
            {
                concepts::Vector auto negative = VecIdxType::fill(0);
                concepts::Vector auto positive = VecIdxType::fill(0);
                negative[d] = -1;
                positive[d] = 1;
                result += in[negative].load() * 3;
                result += in[positive].load() * 5;
            }
            return result;
        }
    };

    void crossStencilOne(auto& dev, auto& queue, auto exec, auto extentMd)
    {
        using T = int32_t;
        using Extent = std::decay_t<decltype(extentMd)>;
        auto const halo = Extent::fill(1);
        auto const inner = extentMd - Extent::fill(2);
        auto in = onHost::alloc<T>(dev, extentMd);
        auto out = onHost::alloc<T>(dev, inner);
        auto hin = onHost::allocHostLike(in);
        auto hout = onHost::allocHostLike(out);
        meta::ndLoopIncIdx(extentMd, [&](auto idx) { hin[idx] = alpaka::linearize(Extent::fill(1000), idx); });
        onHost::memcpy(queue, in, hin);
        auto shifted = in.getView().getSubView(halo, inner);
        onHost::transform(queue, exec, out, StencilFunc{CrossStencil{}}, shifted);
        onHost::memcpy(queue, hout, out);
        onHost::wait(queue);
        int bad = 0;
        meta::ndLoopIncIdx(
            inner,
            [&](auto outIdx)
            {
                auto const inIdx = outIdx + halo;
                T want = hin[inIdx] + 42;
                for(uint32_t d = 0u; d < extentMd.dim(); ++d)
                {
                    auto neg = inIdx;
                    auto pos = inIdx;
                    --neg[d];
                    ++pos[d];
                    want += hin[neg] * 3;
                    want += hin[pos] * 5;
                }
                if(hout[outIdx] != want && bad++ < 3)
                    expect(false, "cross stencil", hout[outIdx], want);
            });
    }
} // namespace

int main()
{
    auto selector = onHost::makeDeviceSelector(onHost::DeviceSpec{api::cuda, deviceKind::nvidiaGpu});
    if(!selector.isAvailable())
    {
        std::printf("SKIP no CUDA device\n");
        return 77;
    }
    auto dev = selector.makeDevice(0);
    auto queue = dev.makeQueue();
    auto exec = exec::gpuCuda;
    scanTests(dev, queue, exec);
    // extents of test/unit/algorithm/reduce.cpp:150-151
    reduceOne(dev, queue, exec, Vec{5, 7, 3, 11});
    reduceOne(dev, queue, exec, Vec{93, 7, 123});
    reduceOne(dev, queue, exec, Vec{5, 7, 4111});
    reduceOne(dev, queue, exec, Vec{5, 7, 3});
    reduceOne(dev, queue, exec, Vec{7, 3});
    reduceOne(dev, queue, exec, Vec{3});
    transformReduceTests(dev, queue, exec);
    // extents of test/unit/algorithm/transform.cpp:177-178
    transformTests(dev, queue, exec, Vec{5, 7, 3, 11});
    transformTests(dev, queue, exec, Vec{93, 7, 123});
    transformTests(dev, queue, exec, Vec{5, 7, 4111});
    transformTests(dev, queue, exec, Vec{5, 7, 3});
    transformTests(dev, queue, exec, Vec{7, 3});
    transformTests(dev, queue, exec, Vec{3});
    transformLarge(dev, queue, exec);
    // extents of test/unit/algorithm/transformReduce.cpp:254-255 and concurrent.cpp
    transformReducePins(dev, queue, exec, Vec{5, 7, 3, 11});
    transformReducePins(dev, queue, exec, Vec{93, 7, 123});
    transformReducePins(dev, queue, exec, Vec{5, 7, 4111});
    transformReducePins(dev, queue, exec, Vec{5, 7, 3});
    transformReducePins(dev, queue, exec, Vec{7, 3});
    transformReducePins(dev, queue, exec, Vec{3});
    concurrentPins(dev, queue, exec, Vec{5, 7, 3, 11});
    concurrentPins(dev, queue, exec, Vec{93, 7, 123});
    concurrentPins(dev, queue, exec, Vec{5, 7, 4111});
    concurrentPins(dev, queue, exec, Vec{5, 7, 3});
    concurrentPins(dev, queue, exec, Vec{7, 3});
    concurrentPins(dev, queue, exec, Vec{3});
    // BabelStream through queue.enqueue: 2^18 elements (the benchmark's minimum array size), 10 runs
    babelStreamKernels<double>(dev, queue, exec, 1u << 18, 10, 1e-12);
    babelStreamKernels<float>(dev, queue, exec, (1u << 18) + 3u, 10, 1e-5);
    // test/unit/algorithm/transform.cpp:399-405
    crossStencilOne(dev, queue, exec, Vec{17});
    crossStencilOne(dev, queue, exec, Vec{17, 19});
    crossStencilOne(dev, queue, exec, Vec{13, 17, 19});
    crossStencilOne(dev, queue, exec, Vec{7, 11, 13, 17});
    // extents of test/unit/algorithm/iota.cpp:112-113
    auto const routedBeforeIota = alpaka3_b200::routingStats().routed.load();
    iotaOne(dev, queue, exec, Vec{5, 7, 3, 11});
    iotaOne(dev, queue, exec, Vec{93, 7, 123});
    iotaOne(dev, queue, exec, Vec{5, 7, 4111});
    iotaOne(dev, queue, exec, Vec{5, 7, 3});
    iotaOne(dev, queue, exec, Vec{7, 3});
    iotaOne(dev, queue, exec, Vec{3});
    std::printf("iota/fill routed=%llu\n",
                static_cast<unsigned long long>(alpaka3_b200::routingStats().routed.load() - routedBeforeIota));
    auto& st = alpaka3_b200::routingStats();
    if(failures == 0)
        std::printf("PASS routed=%llu engine=%llu forwarded=%llu\n", static_cast<unsigned long long>(st.routed.load()),
                    static_cast<unsigned long long>(st.engine.load()), static_cast<unsigned long long>(st.forwarded.load()));
    return failures == 0 ? 0 : 1;
}
