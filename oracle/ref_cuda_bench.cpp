/* Reference GPU comparator: alpaka3's OWN CUDA backend (api::cuda + exec::gpuCuda), compiled by nvcc for sm_100a
 * from the reference's unmodified headers, run on the same workloads, sizes and seeded inputs as bench.py.
 *
 * This file is MEASUREMENT AND TEST INFRASTRUCTURE, never the product path: it does not include or link the
 * alpaka3_b200 library, so every call below runs the reference's generic kernels. Built by oracle/build_ref.sh into
 * oracle/_ref/ref_cuda_bench (out of git; travels with the snapshot next to liboracle.so, which supplies the
 * Philox4x32-10 inputs).
 *
 * Each workload calls the reference the way its own benchmark or example does:
 *   sumsq      onHost::transformReduce(q, gpuCuda, 0.f, out, std::plus, square, in)   (onHost/algo/transformReduce.hpp:59-114)
 *   babelstream SimdAlgo::concurrent kernels enqueued with the benchmark's FrameSpec     (babelStreamMainTest.cpp:224-227),
 *              each operation timed on its own; dot through onHost::transformReduce    (:337-345)
 *   scan_i32 / scan_u64  onHost::exclusiveScan / inclusiveScan with a caller buffer of getScanBufferSize bytes
 *                                                                                      (onHost/algo/scan.hpp:26-218)
 *   heat       StencilKernel, 16x16 chunks, 18x18 shared tile                           (heatEquation2D.cpp:134-176)
 *   nbody      UpdateVelocitiesKernel + onHost::concurrent(UpdatePositions), 256-body chunks (nBody.cpp:166-205);
 *              the kernel's softening is its built-in EPS (common.hpp:41), which leaves the flop count unchanged
 *
 * Timing: W untimed steps, then K steps back to back on the queue's stream between two CUDA events (the same bracket
 * bench.py puts around its own K steps). Every workload checks its own result and reports "check": "ok" or why not.
 *
 * usage: ref_cuda_bench [--small] [--steps K] [--warmup W] [--only NAME]
 * prints one JSON line per workload.
 */
#include <alpaka/alpaka.hpp>

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <string>
#include <type_traits>
#include <vector>

#include "Kernels.hpp"       // example/nBody/src
#include "StencilKernel.hpp" // example/heatEquation2D/src
#include "ref_ops.hpp"

extern "C"
{
    // oracle/oracle.c
    void orc_gen_u32(uint64_t seed, uint64_t start, uint64_t n, int shift, uint32_t* out);
    void orc_gen_u64(uint64_t seed, uint64_t start, uint64_t n, uint64_t* out);
    void orc_gen_f32(uint64_t seed, uint64_t start, uint64_t n, float lo, float hi, float* out);
}

using namespace alpaka;
using namespace a3b_ref;

namespace
{
    constexpr uint64_t kSeed = 0x5EED0001ull;

    struct Options
    {
        bool small = false;
        int steps = 10;
        int warmup = 3;
        std::string only;
    };

    void die(char const* what, cudaError_t e)
    {
        std::fprintf(stderr, "%s: %s\n", what, cudaGetErrorString(e));
        std::exit(2);
    }

#define RCB_CUDA(call)                                                                                                \
    do                                                                                                                \
    {                                                                                                                 \
        cudaError_t e_ = (call);                                                                                      \
        if(e_ != cudaSuccess)                                                                                         \
            die(#call, e_);                                                                                           \
    } while(0)

    // device time of `steps` back-to-back calls of `step` on `stream`, after `warmup` untimed calls (ms per step)
    template<typename F>
    double timeSteps(cudaStream_t stream, int warmup, int steps, F&& step)
    {
        for(int i = 0; i < warmup; ++i)
            step(i);
        RCB_CUDA(cudaStreamSynchronize(stream));
        cudaEvent_t a, b;
        RCB_CUDA(cudaEventCreate(&a));
        RCB_CUDA(cudaEventCreate(&b));
        RCB_CUDA(cudaEventRecord(a, stream));
        for(int i = 0; i < steps; ++i)
            step(warmup + i);
        RCB_CUDA(cudaEventRecord(b, stream));
        RCB_CUDA(cudaEventSynchronize(b));
        float ms = 0.f;
        RCB_CUDA(cudaEventElapsedTime(&ms, a, b));
        RCB_CUDA(cudaEventDestroy(a));
        RCB_CUDA(cudaEventDestroy(b));
        RCB_CUDA(cudaGetLastError());
        return static_cast<double>(ms) / steps;
    }

    void emit(
        char const* workload,
        uint64_t n,
        double msPerStep,
        double unitsPerStep,
        char const* unit,
        int steps,
        std::string const& check,
        std::string const& extra = "")
    {
        double const value = unitsPerStep / (msPerStep * 1e-3) / (std::strcmp(unit, "TFLOP/s") == 0 ? 1e12 : 1e9);
        std::printf(
            "{\"impl\": \"alpaka3-cuda\", \"workload\": \"%s\", \"n\": %llu, \"value\": %.2f, \"unit\": \"%s\", "
            "\"ms_per_step\": %.5f, \"steps\": %d, \"check\": \"%s\"%s}\n",
            workload,
            static_cast<unsigned long long>(n),
            value,
            unit,
            msPerStep,
            steps,
            check.c_str(),
            extra.c_str());
        std::fflush(stdout);
    }

    std::string relCheck(double got, double want, double tol)
    {
        double const rel = std::fabs(got - want) / std::fabs(want);
        char buf[128];
        if(rel <= tol)
            return "ok";
        std::snprintf(buf, sizeof(buf), "relative error %.3e above %.1e", rel, tol);
        return buf;
    }

    template<typename Q>
    cudaStream_t streamOf(Q& q)
    {
        return reinterpret_cast<cudaStream_t>(q.getNativeHandle());
    }

    // ---------------------------------------------------------------- transformReduce: sum of squares, fp32
    template<typename D, typename Q>
    void runSumsq(D& dev, Q& q, Options const& o)
    {
        uint32_t const n = o.small ? (1u << 22) : (1u << 30);
        auto host = onHost::allocHost<float>(Vec{n});
        orc_gen_f32(kSeed, 0, n, -1.0f, 1.0f, host.data());
        double want = 0.0;
        for(uint32_t i = 0; i < n; ++i)
            want += static_cast<double>(host.data()[i]) * static_cast<double>(host.data()[i]);
        auto in = onHost::alloc<float>(dev, Vec{n});
        onHost::memcpy(q, in, host);
        auto out = onHost::alloc<float>(dev, Vec{1u});
        auto outHost = onHost::allocHostLike(out);
        double const ms = timeSteps(
            streamOf(q),
            o.warmup,
            o.steps,
            [&](int) { onHost::transformReduce(q, exec::gpuCuda, 0.f, out, std::plus{}, Square{}, in); });
        onHost::memcpy(q, outHost, out);
        onHost::wait(q);
        emit("sumsq", n, ms, 4.0 * n, "GB/s", o.steps, relCheck(outHost.data()[0], want, 1e-5));
    }

    // ---------------------------------------------------------------- BabelStream fp64
    template<typename D, typename Q>
    void runBabelstream(D& dev, Q& q, Options const& o)
    {
        uint32_t const n = o.small ? (1u << 20) : (1u << 25);
        auto a = onHost::alloc<double>(dev, Vec{n});
        auto b = onHost::allocLike(dev, a);
        auto c = onHost::allocLike(dev, a);
        auto out = onHost::alloc<double>(dev, Vec{1u});
        auto outHost = onHost::allocHostLike(out);
        uint32_t const elemsPerItem = getNumElemPerThread<double>(q);
        auto const numFrames = divExZero(n, uint32_t{512} * elemsPerItem);
        auto const spec = onHost::FrameSpec{numFrames, uint32_t{512}, exec::gpuCuda};
        q.enqueue(spec, KernelBundle{ForEach{}, InitOp{}, a, b, c});
        cudaStream_t const s = streamOf(q);
        // each operation W + K times back to back, the K timed between two events (the same bracket as the other
        // workloads); the arrays then hold a = b + s*c, b = s*c, c = a0 + b with a0 the initial a
        double ms[5];
        ms[0] = timeSteps(s, o.warmup, o.steps, [&](int) { q.enqueue(spec, KernelBundle{ForEach{}, CopyOp{}, a, c}); });
        ms[1] = timeSteps(s, o.warmup, o.steps, [&](int) { q.enqueue(spec, KernelBundle{ForEach{}, MulOp{}, b, c}); });
        ms[2] = timeSteps(s, o.warmup, o.steps, [&](int) { q.enqueue(spec, KernelBundle{ForEach{}, AddOp{}, a, b, c}); });
        ms[3] = timeSteps(s, o.warmup, o.steps, [&](int) { q.enqueue(spec, KernelBundle{ForEach{}, TriadOp{}, a, b, c}); });
        ms[4] = timeSteps(
            s,
            o.warmup,
            o.steps,
            [&](int) { onHost::transformReduce(q, exec::gpuCuda, 0.0, out, std::plus{}, Product{}, a, b); });
        double const gc0 = kInitA;
        double const gb = kScalar * gc0;
        double const gc = kInitA + gb;
        double const ga = gb + kScalar * gc;
        onHost::memcpy(q, outHost, out);
        onHost::wait(q);
        auto ha = onHost::allocHostLike(a);
        auto hb = onHost::allocHostLike(b);
        auto hc = onHost::allocHostLike(c);
        onHost::memcpy(q, ha, a);
        onHost::memcpy(q, hb, b);
        onHost::memcpy(q, hc, c);
        onHost::wait(q);
        // the benchmark's own tolerance style (babelStreamMainTest.cpp:399-431): relative error of each array's mean
        auto meanErr = [&](double const* p, double gold)
        {
            double m = 0.0;
            for(uint32_t i = 0; i < n; ++i)
                m += std::fabs(p[i] - gold);
            return m / n / std::fabs(gold);
        };
        double const err = std::max({meanErr(ha.data(), ga), meanErr(hb.data(), gb), meanErr(hc.data(), gc)});
        std::string const arrays = err <= 1e-8 ? "ok" : "array error above 1e-8";
        std::string const dot = relCheck(outHost.data()[0], ga * gb * n, 1e-8);
        char const* names[5] = {"copy", "mul", "add", "triad", "dot"};
        double const bytes[5] = {16.0 * n, 16.0 * n, 24.0 * n, 24.0 * n, 16.0 * n};
        for(int k = 0; k < 5; ++k)
        {
            std::string const wl = std::string("babelstream_") + names[k];
            emit(wl.c_str(), n, ms[k], bytes[k], "GB/s", o.steps, k == 4 ? dot : arrays);
        }
    }

    // ---------------------------------------------------------------- scans
    template<typename T, bool T_inclusive, typename D, typename Q>
    void runScan(D& dev, Q& q, Options const& o, char const* name, uint32_t n)
    {
        auto host = onHost::allocHost<T>(Vec{n});
        if constexpr(sizeof(T) == 4)
            orc_gen_u32(kSeed, 0, n, 28, reinterpret_cast<uint32_t*>(host.data()));
        else
            orc_gen_u64(kSeed, 0, n, reinterpret_cast<uint64_t*>(host.data()));
        auto in = onHost::alloc<T>(dev, Vec{n});
        auto out = onHost::allocLike(dev, in);
        auto buffer = onHost::alloc<std::byte>(dev, onHost::getScanBufferSize<T>(in.getExtents()));
        onHost::memcpy(q, in, host);
        double const ms = timeSteps(
            streamOf(q),
            o.warmup,
            o.steps,
            [&](int)
            {
                if constexpr(T_inclusive)
                    onHost::inclusiveScan(q, exec::gpuCuda, buffer, out, in);
                else
                    onHost::exclusiveScan(q, exec::gpuCuda, buffer, out, in);
            });
        auto back = onHost::allocHostLike(out);
        onHost::memcpy(q, back, out);
        onHost::wait(q);
        // wrapping unsigned prefix sum, element by element
        using U = std::make_unsigned_t<T>;
        U run = 0;
        uint64_t bad = 0;
        for(uint32_t i = 0; i < n; ++i)
        {
            U const x = static_cast<U>(host.data()[i]);
            U const want = T_inclusive ? static_cast<U>(run + x) : run;
            bad += static_cast<U>(back.data()[i]) != want;
            run = static_cast<U>(run + x);
        }
        std::string const check = bad == 0 ? "ok" : std::to_string(bad) + " elements differ from the prefix sum";
        emit(name, n, ms, 2.0 * sizeof(T) * n, "GB/s", o.steps, check);
    }

    // ---------------------------------------------------------------- heat stencil, fp64
    template<typename D, typename Q>
    void runHeat(D& dev, Q& q, Options const& o)
    {
        using IdxVec = Vec<uint32_t, 2u>;
        uint32_t const n = o.small ? 512u : 32768u;
        IdxVec const numNodes{n, n};
        // The buffers get 64-bit extents: MdSpan computes byte offsets in its index type (mem/MdSpan.hpp:267-282),
        // and the example's uint32 extents (heatEquation2D.cpp:27) wrap past 4 GiB, which a 32768^2 fp64 field
        // exceeds (with uint32 extents the field came out wrong on the B200 at this size).
        using BufVec = Vec<uint64_t, 2u>;
        BufVec const extent{n + 2ull, n + 2ull};
        double const dx = 1.0 / static_cast<double>(n + 1u);
        double const r = 0.2;
        double const dt = r * dx * dx;
        constexpr double pi = 3.14159265358979323846;
        auto host = onHost::allocHost<double>(extent);
        {
            std::vector<double> sx(n + 2u);
            for(uint32_t i = 0; i < n + 2u; ++i)
                sx[i] = (i == 0u || i == n + 1u) ? 0.0 : std::sin(pi * i * dx);
            auto md = host.getMdSpan();
            for(uint32_t j = 0; j < n + 2u; ++j)
                for(uint32_t i = 0; i < n + 2u; ++i)
                    md[BufVec{j, i}] = sx[j] * sx[i];
        }
        auto cur = onHost::alloc<double>(dev, extent);
        auto nxt = onHost::allocLike(dev, cur);
        onHost::memcpy(q, cur, host);
        onHost::memcpy(q, nxt, host);
        constexpr auto chunk = CVec<uint32_t, 16u, 16u>{};
        auto const smemExt = CVec<uint32_t, 18u, 18u>{};
        IdxVec const numChunks{n / 16u, n / 16u};
        auto const spec = onHost::FrameSpec{numChunks, chunk, exec::gpuCuda};
        StencilKernel k;
        double const ms = timeSteps(
            streamOf(q),
            o.warmup,
            o.steps,
            [&](int)
            {
                q.enqueue(spec, KernelBundle{k, cur, nxt, chunk, smemExt, numNodes, dx, dx, dt});
                std::swap(cur, nxt);
            });
        // sin(pi x) sin(pi y) is a discrete eigenmode: every step scales it by lambda
        int const total = o.warmup + o.steps;
        double const lambda = 1.0 - 4.0 * r * (1.0 - std::cos(pi * dx));
        auto back = onHost::allocHostLike(cur);
        onHost::memcpy(q, back, cur);
        onHost::wait(q);
        auto md = back.getMdSpan();
        auto h0 = host.getMdSpan();
        double err = 0.0, scale = 0.0;
        for(uint32_t j : {1u, n / 3u, n / 2u, n})
            for(uint32_t i = 0; i < n + 2u; ++i)
            {
                double const want = h0[BufVec{j, i}] * std::pow(lambda, total);
                err = std::max(err, std::fabs(md[BufVec{j, i}] - want));
                scale = std::max(scale, std::fabs(h0[BufVec{j, i}]));
            }
        char buf[96];
        std::snprintf(buf, sizeof(buf), "normwise error %.3e above 1e-12", err / scale);
        emit("heat", uint64_t{n} * n, ms, 16.0 * n * n, "GB/s", o.steps, err / scale <= 1e-12 ? "ok" : buf);
    }

    // ---------------------------------------------------------------- nBody all-pairs, fp32
    template<typename D, typename Q>
    void runNbody(D& dev, Q& q, Options const& o)
    {
        using namespace alpaka::example::nBody;
        uint32_t const n = o.small ? 4096u : 262144u;
        float const dt = 1e-3f;
        auto ext = Vec{n};
        auto hm = onHost::allocHost<float>(ext);
        auto hx = onHost::allocHost<float>(ext);
        auto hy = onHost::allocHost<float>(ext);
        auto hz = onHost::allocHost<float>(ext);
        auto hv = onHost::allocHost<float>(ext);
        orc_gen_f32(kSeed + 1, 0, n, 0.5f, 1.0f, hm.data());
        orc_gen_f32(kSeed + 2, 0, n, 0.0f, 1.0f, hx.data());
        orc_gen_f32(kSeed + 3, 0, n, 0.0f, 1.0f, hy.data());
        orc_gen_f32(kSeed + 4, 0, n, 0.0f, 1.0f, hz.data());
        std::fill(hv.data(), hv.data() + n, 0.0f);
        auto m = onHost::alloc<float>(dev, ext);
        auto x = onHost::allocLike(dev, m);
        auto y = onHost::allocLike(dev, m);
        auto z = onHost::allocLike(dev, m);
        auto vx = onHost::allocLike(dev, m);
        auto vy = onHost::allocLike(dev, m);
        auto vz = onHost::allocLike(dev, m);
        onHost::memcpy(q, m, hm);
        onHost::memcpy(q, x, hx);
        onHost::memcpy(q, y, hy);
        onHost::memcpy(q, z, hz);
        onHost::memcpy(q, vx, hv);
        onHost::memcpy(q, vy, hv);
        onHost::memcpy(q, vz, hv);
        auto pd = ParticleData{
            m.getView(),
            x.getView(),
            y.getView(),
            z.getView(),
            vx.getView(),
            vy.getView(),
            vz.getView()};
        constexpr auto chunk = CVec<uint32_t, 256u>{};
        auto const spec = onHost::FrameSpec{divCeil(ext, chunk), chunk, exec::gpuCuda};
        UpdateVelocitiesKernel vk;
        UpdatePositions pk{dt};
        double const ms = timeSteps(
            streamOf(q),
            o.warmup,
            o.steps,
            [&](int)
            {
                q.enqueue(spec, KernelBundle{vk, pd, chunk, dt});
                onHost::concurrent<float>(
                    q,
                    pd.xPositions.getExtents(),
                    pk,
                    pd.xPositions,
                    pd.yPositions,
                    pd.zPositions,
                    pd.xVelocities,
                    pd.yVelocities,
                    pd.zVelocities);
            });
        // the all-pairs forces are antisymmetric: total momentum stays ~0 from rest
        auto back = onHost::allocHostLike(vx);
        std::string check = "ok";
        for(auto* v : {&vx, &vy, &vz})
        {
            onHost::memcpy(q, back, *v);
            onHost::wait(q);
            double p = 0.0, sc = 0.0;
            for(uint32_t i = 0; i < n; ++i)
            {
                p += static_cast<double>(hm.data()[i]) * back.data()[i];
                sc += static_cast<double>(hm.data()[i]) * std::fabs(back.data()[i]);
                if(!std::isfinite(back.data()[i]))
                    sc = NAN;
            }
            if(!(std::fabs(p) <= 1e-4 * sc))
                check = "momentum not conserved or non-finite velocities";
        }
        emit("nbody", n, ms, 20.0 * double(n) * double(n), "TFLOP/s", o.steps, check);
    }
} // namespace

int main(int argc, char** argv)
{
    Options o;
    for(int i = 1; i < argc; ++i)
    {
        std::string const a = argv[i];
        if(a == "--small")
            o.small = true;
        else if(a == "--steps" && i + 1 < argc)
            o.steps = std::atoi(argv[++i]);
        else if(a == "--warmup" && i + 1 < argc)
            o.warmup = std::atoi(argv[++i]);
        else if(a == "--only" && i + 1 < argc)
            o.only = argv[++i];
        else
        {
            std::fprintf(stderr, "usage: %s [--small] [--steps K] [--warmup W] [--only NAME]\n", argv[0]);
            return 2;
        }
    }
    if(o.steps < 1 || o.warmup < 0)
        return 2;
    auto selector = onHost::makeDeviceSelector(onHost::DeviceSpec{api::cuda, deviceKind::nvidiaGpu});
    if(!selector.isAvailable())
    {
        std::fprintf(stderr, "no CUDA device\n");
        return 3;
    }
    auto dev = selector.makeDevice(0);
    auto q = dev.makeQueue();
    auto want = [&](char const* name) { return o.only.empty() || o.only == name; };
    if(want("sumsq"))
        runSumsq(dev, q, o);
    if(want("babelstream"))
        runBabelstream(dev, q, o);
    if(want("scan_i32"))
        runScan<int32_t, false>(dev, q, o, "scan_i32", o.small ? (1u << 22) : (1u << 30));
    if(want("scan_u64"))
        runScan<uint64_t, true>(dev, q, o, "scan_u64", o.small ? (1u << 20) : (1u << 28));
    if(want("heat"))
        runHeat(dev, q, o);
    if(want("nbody"))
        runNbody(dev, q, o);
    return 0;
}
