// heatEquation2D: explicit 5-point Jacobi step on an fp64 grid with a 1-cell halo ring.
//
// Replaces StencilKernel (example/heatEquation2D/src/StencilKernel.hpp:26-86), which stages 18x18 tiles in shared
// memory (~1.27x read amplification from the halos). Here each thread owns two adjacent columns (one 16-byte pack) of
// a band of rows and marches down the band with a three-row register window (north, centre, south), so every interior
// cell of `cur` is read from HBM once per band and `next` is written once: 16 bytes of traffic per cell plus two halo
// rows per band. West/east neighbours come from the adjacent lanes by warp shuffles; only the two edge lanes of a warp
// load one extra value per row (an L1/L2 hit). The update is evaluated in the reference's source order with each
// operation rounded on its own:
//   next = c*(1 - 2rX - 2rY) + w*rX + e*rX + n*rY + s*rY
#include <math_constants.h>

#include "common.cuh"

namespace a3b
{
    namespace
    {
        constexpr int kThreads = 256;
        constexpr int kBand = 64; // rows per block
        constexpr int kAhead = 4; // rows loaded per step of the march

        __device__ __forceinline__ double cell(double c, double w, double e, double n, double s, double k, double rX,
                                               double rY)
        {
            double v = __dmul_rn(c, k);
            v = __dadd_rn(v, __dmul_rn(w, rX));
            v = __dadd_rn(v, __dmul_rn(e, rX));
            v = __dadd_rn(v, __dmul_rn(n, rY));
            v = __dadd_rn(v, __dmul_rn(s, rY));
            return v;
        }

        // storage columns (c0, c0 + 1) with c0 = 2 * (global thread x); rows [rb, re) of the interior band
        __global__ void __launch_bounds__(kThreads) heatKernelVec(
            double const* __restrict__ cur,
            double* __restrict__ next,
            uint64_t cols,
            uint64_t pitch,
            uint64_t rowBegin,
            uint64_t rowEnd,
            double rX,
            double rY)
        {
            int const lane = threadIdx.x & 31;
            uint64_t const width = cols + 2u; // storage columns
            uint64_t const c0 = 2u * (static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x);
            uint64_t const rb = rowBegin + static_cast<uint64_t>(blockIdx.y) * kBand;
            if(rb >= rowEnd)
                return;
            uint64_t const re = rb + kBand < rowEnd ? rb + kBand : rowEnd;
            bool const live = c0 < width;       // this thread's pack starts inside the row
            bool const hasHi = c0 + 1u < width; // and its second column exists
            uint64_t const cl = live ? c0 : 0u; // clamped load column (always a valid pack start)
            double const k = __dsub_rn(__dsub_rn(1.0, __dmul_rn(2.0, rX)), __dmul_rn(2.0, rY));

            auto ldPack = [&](uint64_t r) -> double2
            {
                double const* p = cur + r * pitch + cl;
                if(hasHi)
                    return __ldcs(reinterpret_cast<double2 const*>(p));
                return make_double2(live ? __ldcs(p) : 0.0, 0.0);
            };
            auto ldOne = [&](uint64_t r, uint64_t c) -> double { return __ldg(cur + r * pitch + c); };

            double2 up = ldPack(rb - 1u);
            double2 mid = ldPack(rb);
            for(uint64_t r = rb; r < re; r += kAhead)
            {
                double2 dn[kAhead];
#pragma unroll
                for(int a = 0; a < kAhead; ++a)
                    dn[a] = (r + a < re) ? ldPack(r + a + 1u) : make_double2(0.0, 0.0);
                // edge values of the warp for each of the kAhead centre rows
                double wEdge[kAhead], eEdge[kAhead];
#pragma unroll
                for(int a = 0; a < kAhead; ++a)
                {
                    wEdge[a] = 0.0;
                    eEdge[a] = 0.0;
                    if(r + a < re)
                    {
                        if(lane == 0 && live && c0 > 0u)
                            wEdge[a] = ldOne(r + a, c0 - 1u);
                        if(lane == 31 && live && c0 + 2u < width)
                            eEdge[a] = ldOne(r + a, c0 + 2u);
                    }
                }
#pragma unroll
                for(int a = 0; a < kAhead; ++a)
                {
                    double2 const south = dn[a];
                    double westOfLo = __shfl_up_sync(0xffffffffu, mid.y, 1);
                    double eastOfHi = __shfl_down_sync(0xffffffffu, mid.x, 1);
                    if(lane == 0)
                        westOfLo = wEdge[a];
                    if(lane == 31)
                        eastOfHi = eEdge[a];
                    uint64_t const row = r + a;
                    if(row < re && live)
                    {
                        double* const q = next + row * pitch + c0;
                        bool const loIn = c0 >= 1u && c0 <= cols;
                        bool const hiIn = hasHi && c0 + 1u <= cols;
                        double const lo = cell(mid.x, westOfLo, mid.y, up.x, south.x, k, rX, rY);
                        double const hi = cell(mid.y, mid.x, eastOfHi, up.y, south.y, k, rX, rY);
                        if(loIn && hiIn)
                            __stcs(reinterpret_cast<double2*>(q), make_double2(lo, hi));
                        else
                        {
                            if(loIn)
                                q[0] = lo;
                            if(hiIn)
                                q[1] = hi;
                        }
                    }
                    up = mid;
                    mid = south;
                }
            }
        }

        // fallback for unaligned grids: one column per thread, plain loads
        __global__ void __launch_bounds__(kThreads) heatKernelScalar(
            double const* __restrict__ cur,
            double* __restrict__ next,
            uint64_t cols,
            uint64_t pitch,
            uint64_t rowBegin,
            uint64_t rowEnd,
            double rX,
            double rY)
        {
            uint64_t const c = 1u + static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
            if(c > cols)
                return;
            uint64_t const rb = rowBegin + static_cast<uint64_t>(blockIdx.y) * kBand;
            uint64_t const re = rb + kBand < rowEnd ? rb + kBand : rowEnd;
            double const k = __dsub_rn(__dsub_rn(1.0, __dmul_rn(2.0, rX)), __dmul_rn(2.0, rY));
            for(uint64_t r = rb; r < re; ++r)
            {
                double const* p = cur + r * pitch + c;
                next[r * pitch + c] = cell(p[0], p[-1], p[1], p[-static_cast<int64_t>(pitch)], p[pitch], k, rX, rY);
            }
        }

        __global__ void __launch_bounds__(kThreads) heatInitKernel(
            double* u,
            uint64_t rows,
            uint64_t cols,
            uint64_t pitch,
            uint64_t rowOffset,
            uint64_t globalRows,
            double dx,
            double dy)
        {
            uint64_t const c = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
            uint64_t const r = blockIdx.y;
            if(c >= cols + 2u || r >= rows + 2u)
                return;
            uint64_t const gr = r + rowOffset; // global storage row (0 = top ring)
            double v = 0.0;
            if(gr >= 1u && gr <= globalRows && c >= 1u && c <= cols)
                v = sin(CUDART_PI * (static_cast<double>(c) * dx)) * sin(CUDART_PI * (static_cast<double>(gr) * dy));
            u[r * pitch + c] = v;
        }
        // Exact solution of the heatEquation2D example, e^{-pi^2 t} (sin pi x + sin pi y) (analyticalSolution.hpp:17-21),
        // at x = col*dx, y = global_row*dy: on every cell (initial field) or on the global ring only (the example's
        // time-dependent Dirichlet boundary, BoundaryKernel.hpp:23-57).
        __global__ void __launch_bounds__(kThreads) heatExactKernel(
            double* u,
            uint64_t rows,
            uint64_t cols,
            uint64_t pitch,
            uint64_t rowOffset,
            uint64_t globalRows,
            double t,
            double dx,
            double dy,
            bool ringOnly)
        {
            uint64_t const c = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x;
            double const decay = exp(-CUDART_PI * CUDART_PI * t);
            for(uint64_t r = blockIdx.y; r < rows + 2u; r += gridDim.y)
            {
                if(c >= cols + 2u)
                    return;
                uint64_t const gr = r + rowOffset;
                bool const ring = gr == 0u || gr == globalRows + 1u || c == 0u || c == cols + 1u;
                if(ringOnly && !ring)
                    continue;
                double const x = static_cast<double>(c) * dx;
                double const y = static_cast<double>(gr) * dy;
                u[r * pitch + c] = decay * (sin(CUDART_PI * x) + sin(CUDART_PI * y));
            }
        }
    } // namespace
} // namespace a3b

using namespace a3b;

extern "C"
{
    int a3b_heat_step(a3b_stream_t stream, double const* cur, double* next, uint64_t rows, uint64_t cols,
                      uint64_t pitch_elems, uint64_t row_begin, uint64_t row_end, double rX, double rY)
    {
        A3B_REQUIRE(cur && next, "null grid pointer");
        A3B_REQUIRE(cur != next, "cur and next must be different buffers");
        A3B_REQUIRE(pitch_elems >= cols + 2u, "pitch smaller than a row with its halo");
        A3B_REQUIRE(row_begin >= 1u && row_begin <= row_end && row_end <= rows + 1u, "row range outside the interior");
        if(row_begin == row_end || cols == 0)
            return A3B_OK;
        DeviceProps const* props = nullptr;
        int rc = currentDevice(&props);
        if(rc)
            return rc;
        auto s = static_cast<cudaStream_t>(stream);
        uint64_t const bands = (row_end - row_begin + kBand - 1) / kBand;
        A3B_REQUIRE(bands < 65536u, "too many row bands");
        bool const vec = aligned16(cur) && aligned16(next) && pitch_elems % 2u == 0u;
        if(vec)
        {
            uint64_t const packs = (cols + 2u + 1u) / 2u;
            dim3 const grid(static_cast<unsigned>((packs + kThreads - 1) / kThreads), static_cast<unsigned>(bands));
            heatKernelVec<<<grid, kThreads, 0, s>>>(cur, next, cols, pitch_elems, row_begin, row_end, rX, rY);
        }
        else
        {
            dim3 const grid(static_cast<unsigned>((cols + kThreads - 1) / kThreads), static_cast<unsigned>(bands));
            heatKernelScalar<<<grid, kThreads, 0, s>>>(cur, next, cols, pitch_elems, row_begin, row_end, rX, rY);
        }
        A3B_CHECK_LAUNCH("heat step launch");
        return A3B_OK;
    }

    int a3b_heat_init(a3b_stream_t stream, double* u, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                      uint64_t row_offset, uint64_t global_rows, double dx, double dy)
    {
        A3B_REQUIRE(u, "null grid pointer");
        A3B_REQUIRE(pitch_elems >= cols + 2u, "pitch smaller than a row with its halo");
        A3B_REQUIRE(rows + 2u < 2147483647u, "too many rows");
        dim3 const grid(static_cast<unsigned>((cols + 2u + kThreads - 1) / kThreads), static_cast<unsigned>(rows + 2u));
        heatInitKernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(u, rows, cols, pitch_elems,
                                                                                  row_offset, global_rows, dx, dy);
        A3B_CHECK_LAUNCH("heat init launch");
        return A3B_OK;
    }

    int a3b_heat_exact(a3b_stream_t stream, double* u, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                       uint64_t row_offset, uint64_t global_rows, double t, double dx, double dy, int ring_only)
    {
        A3B_REQUIRE(u, "null grid pointer");
        A3B_REQUIRE(pitch_elems >= cols + 2u, "pitch smaller than a row with its halo");
        uint64_t const gy = rows + 2u < 65535u ? rows + 2u : 65535u;
        dim3 const grid(static_cast<unsigned>((cols + 2u + kThreads - 1) / kThreads), static_cast<unsigned>(gy));
        heatExactKernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
            u, rows, cols, pitch_elems, row_offset, global_rows, t, dx, dy, ring_only != 0);
        A3B_CHECK_LAUNCH("heat exact launch");
        return A3B_OK;
    }
}
