/* Reference harness: drives alpaka3's OWN host backend (api::host + exec::cpuOmpBlocks / exec::cpuSerial)
 * through its public onHost API, compiled from the reference's unmodified headers.
 *
 * This file is TEST INFRASTRUCTURE (the checker and the timed CPU baseline), never the product path.
 * It is built by oracle/build_ref.sh into oracle/_ref/libalpaka_ref.so, which stays out of git.
 *
 * Each entry point names the reference code it runs:
 *   ref_babelstream      benchmark/babelstream/src/babelStreamMainTest.cpp:61-141 (ops), :285-366 (run loop)
 *   ref_transform_reduce include/alpaka/onHost/algo/transformReduce.hpp:59-90
 *   ref_reduce           include/alpaka/onHost/algo/reduce.hpp:28-79, test/unit/algorithm/reduce.cpp:135-152
 *   ref_scan             include/alpaka/onHost/algo/scan.hpp:45-218
 *   ref_heat_steps       example/heatEquation2D/src/StencilKernel.hpp:26-86 driven as heatEquation2D.cpp:134-196
 *   ref_heat_problem     the example's own problem end to end: initalizeBuffer, StencilKernel + BoundaryKernel per
 *                        step (heatEquation2D.cpp:97-196, BoundaryKernel.hpp:23-57, analyticalSolution.hpp:17-78)
 *   ref_nbody_steps      example/nBody/src/Kernels.hpp:24-142 driven as nBody.cpp:171-205 (EPS fixed at 4 there)
 * The BabelStream operation functors below are written here (they live in the reference's benchmark TU and cannot
 * be included); each states the same element-wise assignment as the reference op it mirrors.
 */
#include <alpaka/alpaka.hpp>

#include <chrono>
#include <cstdint>
#include <cstring>
#include <functional>
#include <limits>
#include <vector>

// reference example kernels, included from their own location in the reference tree
#include "BoundaryKernel.hpp"  // example/heatEquation2D/src
#include "StencilKernel.hpp"   // example/heatEquation2D/src
#include "analyticalSolution.hpp"
#include "Kernels.hpp"         // example/nBody/src
#include "ref_ops.hpp"

using namespace alpaka;
using namespace a3b_ref;

namespace
{
    auto& hostDevice()
    {
        static auto dev = onHost::makeDeviceSelector(onHost::DeviceSpec{api::host, deviceKind::cpu}).makeDevice(0);
        return dev;
    }

    auto& hostQueue()
    {
        static auto q = hostDevice().makeQueue();
        return q;
    }

    template<typename F>
    int withExec(int execKind, F&& f)
    {
        if(execKind == 0)
            f(exec::cpuSerial);
        else
            f(exec::cpuOmpBlocks);
        return 0;
    }

    double secondsSince(std::chrono::high_resolution_clock::time_point t0)
    {
        return std::chrono::duration<double>(std::chrono::high_resolution_clock::now() - t0).count();
    }

    // min/max reduce functors as the reference test declares them (test/unit/algorithm/reduce.cpp:22-56)
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

    template<typename T>
    int babelstream(int execKind, T* a, T* b, T* c, uint32_t n, int runs, int kernels, T* dotOut, double* times)
    {
        auto& q = hostQueue();
        auto va = makeView(api::host, a, Vec{n});
        auto vb = makeView(api::host, b, Vec{n});
        auto vc = makeView(api::host, c, Vec{n});
        return withExec(
            execKind,
            [&](auto ex)
            {
                // frame shape as babelStreamMainTest.cpp:224-227
                uint32_t elemsPerItem = getNumElemPerThread<T>(q);
                auto numFrames = divExZero(n, uint32_t{512} * elemsPerItem);
                auto spec = onHost::FrameSpec{numFrames, uint32_t{512}, ex};
                q.enqueue(spec, KernelBundle{ForEach{}, InitOp{}, va, vb, vc});
                onHost::wait(q);
                auto out = onHost::alloc<T>(hostDevice(), 1u);
                for(int r = 0; r < runs; ++r)
                {
                    auto t0 = std::chrono::high_resolution_clock::now();
                    if(kernels & 1)
                    {
                        q.enqueue(spec, KernelBundle{ForEach{}, CopyOp{}, va, vc});
                        onHost::wait(q);
                    }
                    if(times)
                        times[5 * r + 0] = secondsSince(t0);
                    t0 = std::chrono::high_resolution_clock::now();
                    if(kernels & 2)
                    {
                        q.enqueue(spec, KernelBundle{ForEach{}, MulOp{}, vb, vc});
                        onHost::wait(q);
                    }
                    if(times)
                        times[5 * r + 1] = secondsSince(t0);
                    t0 = std::chrono::high_resolution_clock::now();
                    if(kernels & 4)
                    {
                        q.enqueue(spec, KernelBundle{ForEach{}, AddOp{}, va, vb, vc});
                        onHost::wait(q);
                    }
                    if(times)
                        times[5 * r + 2] = secondsSince(t0);
                    t0 = std::chrono::high_resolution_clock::now();
                    if(kernels & 8)
                    {
                        q.enqueue(spec, KernelBundle{ForEach{}, TriadOp{}, va, vb, vc});
                        onHost::wait(q);
                    }
                    if(kernels & 32)
                    {
                        q.enqueue(spec, KernelBundle{ForEach{}, NStreamOp{}, va, vb, vc});
                        onHost::wait(q);
                    }
                    if(times)
                        times[5 * r + 3] = secondsSince(t0);
                    t0 = std::chrono::high_resolution_clock::now();
                    if(kernels & 16)
                    {
                        onHost::transformReduce(q, ex, T{0}, out, std::plus{}, Product{}, va, vb);
                        onHost::wait(q);
                        *dotOut = out.data()[0];
                    }
                    if(times)
                        times[5 * r + 4] = secondsSince(t0);
                }
            });
    }

    template<typename T>
    int scan(int execKind, int inclusive, T const* in, T* out, uint64_t n)
    {
        auto& q = hostQueue();
        auto vin = makeView(api::host, const_cast<T*>(in), Vec{n});
        auto vout = makeView(api::host, out, Vec{n});
        return withExec(
            execKind,
            [&](auto ex)
            {
                if(inclusive)
                    onHost::inclusiveScan(q, ex, vout, vin);
                else
                    onHost::exclusiveScan(q, ex, vout, vin);
                onHost::wait(q);
            });
    }

    template<typename T>
    int reduceT(int execKind, int op, T const* in, uint64_t const* ext, int dim, T* result)
    {
        auto& q = hostQueue();
        auto run = [&](auto extents)
        {
            auto vin = makeView(api::host, const_cast<T*>(in), extents);
            auto out = onHost::alloc<T>(hostDevice(), extents.fill(1));
            withExec(
                execKind,
                [&](auto ex)
                {
                    if(op == 0)
                        onHost::reduce(q, ex, T{0}, out, std::plus{}, vin);
                    else if(op == 1)
                        onHost::reduce(q, ex, std::numeric_limits<T>::max(), out, ScalarFunc{MinValue{}}, vin);
                    else
                        onHost::reduce(q, ex, std::numeric_limits<T>::lowest(), out, ScalarFunc{MaxValue{}}, vin);
                    onHost::wait(q);
                });
            *result = out.data()[0];
        };
        switch(dim)
        {
        case 1:
            run(Vec{ext[0]});
            break;
        case 2:
            run(Vec{ext[0], ext[1]});
            break;
        case 3:
            run(Vec{ext[0], ext[1], ext[2]});
            break;
        case 4:
            run(Vec{ext[0], ext[1], ext[2], ext[3]});
            break;
        default:
            return 1;
        }
        return 0;
    }
} // namespace

#include "helper.hpp" // benchmark/HACCmk/src: the reference's CPU gold of the short-range force

extern "C"
{
    /** kernels bitmask: 1 copy, 2 mul, 4 add, 8 triad, 16 dot, 32 nstream. times: 5 doubles per run (or null). */
    int ref_babelstream_f64(int e, double* a, double* b, double* c, uint32_t n, int runs, int k, double* dot, double* t)
    {
        return babelstream<double>(e, a, b, c, n, runs, k, dot, t);
    }

    int ref_babelstream_f32(int e, float* a, float* b, float* c, uint32_t n, int runs, int k, float* dot, double* t)
    {
        return babelstream<float>(e, a, b, c, n, runs, k, dot, t);
    }

    /** transformReduce(q, exec, 0, out, std::plus{}, x*x, in) over fp32 */
    int ref_sumsq_f32(int execKind, float const* in, uint64_t n, float* result)
    {
        auto& q = hostQueue();
        auto vin = makeView(api::host, const_cast<float*>(in), Vec{n});
        auto out = onHost::alloc<float>(hostDevice(), Vec{uint64_t{1}});
        withExec(
            execKind,
            [&](auto ex)
            {
                onHost::transformReduce(q, ex, 0.f, out, std::plus{}, Square{}, vin);
                onHost::wait(q);
            });
        *result = out.data()[0];
        return 0;
    }

    int ref_sumsq_f64(int execKind, double const* in, uint64_t n, double* result)
    {
        auto& q = hostQueue();
        auto vin = makeView(api::host, const_cast<double*>(in), Vec{n});
        auto out = onHost::alloc<double>(hostDevice(), Vec{uint64_t{1}});
        withExec(
            execKind,
            [&](auto ex)
            {
                onHost::transformReduce(q, ex, 0.0, out, std::plus{}, Square{}, vin);
                onHost::wait(q);
            });
        *result = out.data()[0];
        return 0;
    }

    int ref_dot_f64(int execKind, double const* a, double const* b, uint64_t n, double* result)
    {
        auto& q = hostQueue();
        auto va = makeView(api::host, const_cast<double*>(a), Vec{n});
        auto vb = makeView(api::host, const_cast<double*>(b), Vec{n});
        auto out = onHost::alloc<double>(hostDevice(), Vec{uint64_t{1}});
        withExec(
            execKind,
            [&](auto ex)
            {
                onHost::transformReduce(q, ex, 0.0, out, std::plus{}, Product{}, va, vb);
                onHost::wait(q);
            });
        *result = out.data()[0];
        return 0;
    }

    /** op: 0 plus, 1 min, 2 max. ext: extents, slowest first (alpaka Vec order), dim 1..4 */
    int ref_reduce_i32(int e, int op, int32_t const* in, uint64_t const* ext, int dim, int32_t* r)
    {
        return reduceT<int32_t>(e, op, in, ext, dim, r);
    }

    int ref_reduce_f64(int e, int op, double const* in, uint64_t const* ext, int dim, double* r)
    {
        return reduceT<double>(e, op, in, ext, dim, r);
    }

    int ref_scan_i32(int e, int incl, int32_t const* in, int32_t* out, uint64_t n)
    {
        return scan<int32_t>(e, incl, in, out, n);
    }

    int ref_scan_u32(int e, int incl, uint32_t const* in, uint32_t* out, uint64_t n)
    {
        return scan<uint32_t>(e, incl, in, out, n);
    }

    int ref_scan_u64(int e, int incl, uint64_t const* in, uint64_t* out, uint64_t n)
    {
        return scan<uint64_t>(e, incl, in, out, n);
    }

    int ref_scan_i64(int e, int incl, int64_t const* in, int64_t* out, uint64_t n)
    {
        return scan<int64_t>(e, incl, in, out, n);
    }

    int ref_scan_f64(int e, int incl, double const* in, double* out, uint64_t n)
    {
        return scan<double>(e, incl, in, out, n);
    }

    /** Runs `steps` Jacobi steps of the reference StencilKernel on a (n+2)x(n+2) row-major grid with halo ring
     * (heatEquation2D.cpp:97-99); n must be a multiple of 16. cur/next are both read and written (ping-pong); after the
     * call the newest field is in `cur` (the buffers are swapped back when steps is odd). */
    int ref_heat_steps(int execKind, double* cur, double* next, uint32_t n, uint32_t steps, double dx, double dy, double dt)
    {
        if(n % 16u != 0u)
            return 1;
        auto& q = hostQueue();
        using IdxVec = Vec<uint32_t, 2u>;
        IdxVec const numNodes{n, n};
        IdxVec const extent{n + 2u, n + 2u};
        auto vcur = makeView(api::host, cur, extent);
        auto vnext = makeView(api::host, next, extent);
        constexpr auto chunk = CVec<uint32_t, 16u, 16u>{};
        auto const smemExt = CVec<uint32_t, 18u, 18u>{};
        IdxVec const numChunks{n / 16u, n / 16u};
        withExec(
            execKind,
            [&](auto ex)
            {
                auto spec = onHost::FrameSpec{numChunks, chunk, ex};
                StencilKernel k;
                for(uint32_t s = 0; s < steps; ++s)
                {
                    q.enqueue(spec, KernelBundle{k, vcur, vnext, chunk, smemExt, numNodes, dx, dy, dt});
                    onHost::wait(q);
                    std::swap(vcur, vnext);
                }
            });
        if(steps % 2u == 1u)
            std::memcpy(cur, next, sizeof(double) * (n + 2u) * (n + 2u));
        return 0;
    }

    /** The heatEquation2D example's own problem: n x n interior (n a multiple of 16), `steps` steps up to tMax, exact
     * solution e^{-pi^2 t}(sin pi x + sin pi y) as initial field and time-dependent Dirichlet ring. Writes the final
     * (n+2)^2 field to `out` and returns the example's own validation error (max |u - exact| over the interior). */
    double ref_heat_problem(int execKind, uint32_t n, uint32_t steps, double tMax, double* out)
    {
        using namespace alpaka::onHost;
        if(n % 16u != 0u)
            return -1.0;
        auto& q = hostQueue();
        using IdxVec = Vec<uint32_t, 2u>;
        IdxVec const numNodes{n, n};
        IdxVec const extent{n + 2u, n + 2u};
        double const dx = 1.0 / static_cast<double>(extent[1] - 1);
        double const dy = 1.0 / static_cast<double>(extent[0] - 1);
        double const dt = tMax / static_cast<double>(steps);
        std::vector<double> a((n + 2u) * (n + 2u)), b((n + 2u) * (n + 2u));
        auto va = makeView(api::host, a.data(), extent);
        auto vb = makeView(api::host, b.data(), extent);
        initalizeBuffer(va, dx, dy);
        constexpr auto chunk = CVec<uint32_t, 16u, 16u>{};
        auto const smemExt = CVec<uint32_t, 18u, 18u>{};
        IdxVec const numChunks{n / 16u, n / 16u};
        auto const withHalo = numNodes + IdxVec{2u, 2u};
        withExec(
            execKind,
            [&](auto ex)
            {
                auto spec = FrameSpec{numChunks, chunk, ex};
                auto const longest = std::max(withHalo.y(), withHalo.x());
                auto border = FrameSpec{Vec{longest / chunk.x()}, Vec{std::max(chunk.y(), chunk.x())}, ex};
                StencilKernel sk;
                BoundaryKernel bk;
                auto cur = va;
                auto nxt = vb;
                for(uint32_t step = 1; step <= steps; ++step)
                {
                    q.enqueue(spec, KernelBundle{sk, cur, nxt, chunk, smemExt, numNodes, dx, dy, dt});
                    q.enqueue(border, KernelBundle{bk, nxt, withHalo, step, dx, dy, dt});
                    onHost::wait(q);
                    std::swap(cur, nxt);
                }
                std::memcpy(out, cur.data(), sizeof(double) * (n + 2u) * (n + 2u));
            });
        auto check = makeView(api::host, out, extent);
        return validateSolution(check, extent, dx, dy, tMax).second;
    }

    /** Runs `steps` of the reference nBody step (UpdateVelocitiesKernel with its built-in EPS, then UpdatePositions
     * through onHost::concurrent). n must be a multiple of 256 (nBody.cpp:27 chunk). Arrays are SoA float32. */
    int ref_nbody_steps(
        int execKind,
        float* m,
        float* x,
        float* y,
        float* z,
        float* vx,
        float* vy,
        float* vz,
        uint32_t n,
        uint32_t steps,
        float dt)
    {
        using namespace alpaka::example::nBody;
        if(n % 256u != 0u)
            return 1;
        auto& q = hostQueue();
        auto ext = Vec{n};
        auto pd = ParticleData{
            makeView(api::host, m, ext),
            makeView(api::host, x, ext),
            makeView(api::host, y, ext),
            makeView(api::host, z, ext),
            makeView(api::host, vx, ext),
            makeView(api::host, vy, ext),
            makeView(api::host, vz, ext)};
        constexpr auto chunk = CVec<uint32_t, 256u>{};
        withExec(
            execKind,
            [&](auto ex)
            {
                auto spec = onHost::FrameSpec{divCeil(ext, chunk), chunk, ex};
                UpdateVelocitiesKernel vk;
                UpdatePositions pk{dt};
                for(uint32_t s = 0; s < steps; ++s)
                {
                    q.enqueue(spec, KernelBundle{vk, pd, chunk, dt});
                    onHost::concurrent<float>(
                        q,
                        ex,
                        pd.xPositions.getExtents(),
                        pk,
                        pd.xPositions,
                        pd.yPositions,
                        pd.zPositions,
                        pd.xVelocities,
                        pd.yVelocities,
                        pd.zVelocities);
                    onHost::wait(q);
                }
            });
        return 0;
    }

    // HACCmk's CPU gold (benchmark/HACCmk/src/helper.hpp:19-66) for the first n1 particles, as the benchmark applies it
    // (main_alpaka.cpp:288-293, velocities starting at 0)
    int ref_haccmk_gold(int n1, int n2, float const* xx, float const* yy, float const* zz, float const* mass,
                        float fsrrmax2, float mp_rsm2, float fcoeff, float* vx, float* vy, float* vz)
    {
        for(int i = 0; i < n1; ++i)
        {
            float dx2 = 0.f, dy2 = 0.f, dz2 = 0.f;
            hacc::haccmk_gold(n2, xx[i], yy[i], zz[i], fsrrmax2, mp_rsm2, xx, yy, zz, mass, &dx2, &dy2, &dz2);
            vx[i] = 0.f + dx2 * fcoeff;
            vy[i] = 0.f + dy2 * fcoeff;
            vz[i] = 0.f + dz2 * fcoeff;
        }
        return 0;
    }

    // OpenMP thread count for every later call (the process may have inherited OMP_NUM_THREADS=1 from a launcher)
    void ref_set_num_threads(int n)
    {
        if(n > 0)
            omp_set_num_threads(n);
    }

    int ref_num_threads()
    {
        int t = 1;
#pragma omp parallel
        {
#pragma omp single
            t = omp_get_num_threads();
        }
        return t;
    }
}
