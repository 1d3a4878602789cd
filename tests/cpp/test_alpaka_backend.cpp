/* alpaka3's own algorithm tests, re-expressed without Catch2, run through alpaka3's public onHost API on a CUDA queue
 * with the alpaka3_b200 binding included: the covered calls go to libalpaka3_b200.so, the rest to alpaka3's own CUDA
 * backend. Mirrors test/unit/algorithm/scan.cpp:74-197 (int iota, 4 sizes, exclusive/inclusive x out-of-place /
 * in-place x with/without buffer, std::exclusive_scan / std::inclusive_scan as ground truth) and
 * test/unit/algorithm/reduce.cpp:135-232 (int iota over N-D extents, plus / min / max, plus the generator source),
 * plus BabelStream's dot (benchmark/babelstream/src/babelStreamMainTest.cpp:135-141, 337-345), and
 * test/unit/algorithm/transform.cpp:147-180 (int inputs over the same N-D extents with std::minus, std::plus, a
 * StencilFunc, ScalarFunc with and without an accelerator argument, and an up-casting functor), plus an in-place
 * transform of a large 1-D float array with a ragged end, test/unit/algorithm/iota.cpp:13-118 (size_t iota over the
 * same extents, into one buffer and into two) and element-wise fill.
 * Prints one line "PASS routed=<n> forwarded=<m>" and exits 0, or lists the failures and exits 1. */
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

    struct Cube // not recognised: must be forwarded to alpaka3's own implementation
    {
        constexpr auto operator()(auto const& x) const
        {
            return x * x * x;
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
        transformOne<int>(dev, queue, exec, extents, StencilFunc{StencilAdd{}}, plus, false, "transform stencil");
        transformOne<int>(dev, queue, exec, extents, ScalarFunc{ScalarMinPlusOne{}}, minPlusOne, true, "transform scalar");
        transformOne<int>(dev, queue, exec, extents, ScalarFunc{ScalarOpWithAcc{}}, minPlusOne, false, "transform scalar acc");
        transformOne<std::size_t>(dev, queue, exec, extents, AddUpCast{}, plus, true, "transform up-cast");
        transformOne<std::size_t>(dev, queue, exec, extents, AddUpCastWithAcc{}, plus, false, "transform up-cast acc");
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
        // generator source (not device memory): forwarded to alpaka3's own implementation
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
        // a transform the binding does not recognise: alpaka3's own kernel computes it
        onHost::transformReduce(queue, exec, 0.0, out, std::plus{}, Cube{}, a);
        onHost::memcpy(queue, outHost, out);
        onHost::wait(queue);
        double const want2 = static_cast<double>(n) * (0.1 * 0.1 * 0.1);
        expect(std::abs(*outHost.data() - want2) <= 1e-9 * want2, "transformReduce forwarded", 0, 0);
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
        std::printf("PASS routed=%llu forwarded=%llu\n", static_cast<unsigned long long>(st.routed.load()),
                    static_cast<unsigned long long>(st.forwarded.load()));
    return failures == 0 ? 0 : 1;
}
