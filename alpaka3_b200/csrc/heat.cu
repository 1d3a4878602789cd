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

#include <cstring>

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

        // One band of rows [rb, re) for the thread's storage columns (c0, c0 + 1), c0 = 2 * (global thread x). Ghost
        // rows 0 and rows + 1 come from `north` / `south` when those are set (a neighbour's boundary row in this rank's
        // halo mailbox, read past L1), otherwise from `cur` like every other row.
        __device__ __forceinline__ void heatBand(
            double const* __restrict__ cur,
            double* __restrict__ next,
            uint64_t cols,
            uint64_t pitch,
            uint64_t rb,
            uint64_t re,
            double rX,
            double rY,
            uint64_t rows,
            double const* north,
            double const* south)
        {
            int const lane = threadIdx.x & 31;
            uint64_t const width = cols + 2u; // storage columns
            uint64_t const c0 = 2u * (static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x);
            bool const live = c0 < width;       // this thread's pack starts inside the row
            bool const hasHi = c0 + 1u < width; // and its second column exists
            uint64_t const cl = live ? c0 : 0u; // clamped load column (always a valid pack start)
            double const k = __dsub_rn(__dsub_rn(1.0, __dmul_rn(2.0, rX)), __dmul_rn(2.0, rY));

            auto ldPack = [&](uint64_t r) -> double2
            {
                double const* ghost = (r == 0u) ? north : (r == rows + 1u ? south : nullptr);
                if(ghost)
                {
                    if(hasHi)
                        return __ldcg(reinterpret_cast<double2 const*>(ghost + cl));
                    return make_double2(live ? __ldcg(ghost + cl) : 0.0, 0.0);
                }
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
                    double2 const south2 = dn[a];
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
                        double const lo = cell(mid.x, westOfLo, mid.y, up.x, south2.x, k, rX, rY);
                        double const hi = cell(mid.y, mid.x, eastOfHi, up.y, south2.y, k, rX, rY);
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
                    mid = south2;
                }
            }
        }

        // ------------------------------------------------------------------ rows streamed through a shared ring
        // The same march with the loads taken off the threads: each block owns a strip of kStrip storage columns of a
        // band of kRingBand rows; thread 0 copies every row segment the band needs (the strip plus two columns on
        // each side, 16-byte aligned) from HBM into a ring of kStages shared-memory slots with cp.async.bulk, a few
        // rows ahead of the threads (own-GPU memory only, no multicast), and refills a slot as soon as every thread
        // has read it. The threads keep north / centre in registers, take the south row and the warp-edge
        // neighbours from shared memory and the other neighbours by shuffles, and store straight to HBM. The loads in
        // flight no longer occupy registers, so the copy depth is set by the ring (kStages - 2 rows of 4 KB per block)
        // rather than by the registers that limited the register-window march.
        constexpr int kRingThreads = 256;
        constexpr int kStrip = 2 * kRingThreads; // storage columns computed per block
        constexpr int kSlot = kStrip + 4;        // doubles per ring slot: the strip and two columns each side
        // Measured at 32768^2 (5 interleaved rounds, medians, GB/s of 16 B per cell): 10 stages x 32-row bands 6551
        // (kept), 8 x 64 6425, 12 x 64 6438, 8 x 128 6331, 128-thread strips with 12 x 32 6315; the register-window
        // march (heatKernelVec) ran 6114-6161.
        constexpr int kStages = 10;
        constexpr int kRingBand = 32;
        constexpr size_t kRingSmem = static_cast<size_t>(kStages) * kSlot * sizeof(double);

        // Rows [rb, re) of the strip of block x, streamed through the ring (`ring`: kStages slots of kSlot doubles,
        // `bar`: kStages mbarriers, both in shared memory). Rows rb - 1 .. re of `cur` are read.
        __device__ __forceinline__ void ringBand(
            double const* __restrict__ cur,
            double* __restrict__ next,
            uint64_t cols,
            uint64_t pitch,
            uint64_t rb,
            uint64_t re,
            double rX,
            double rY,
            uint64_t timeoutNs,
            unsigned* errWord,
            double* ring,
            unsigned long long* bar)
        {
            uint64_t const width = cols + 2u;                             // storage columns (even here)
            uint64_t const s0 = static_cast<uint64_t>(blockIdx.x) * kStrip; // first storage column of the strip
            uint64_t const lo = s0 >= 2u ? s0 - 2u : 0u;                  // first column copied (even)
            uint64_t const hi = s0 + kStrip + 2u < width ? s0 + kStrip + 2u : width; // one past the last (even)
            unsigned const bytes = static_cast<unsigned>((hi - lo) * sizeof(double));
            unsigned const dstOff = static_cast<unsigned>(lo + 2u - s0);   // slot index of column lo (0 or 2)
            uint64_t const first = rb - 1u;                                // first row copied (north of rb)

            auto slot = [&](uint64_t q) { return ring + ((q - first) % kStages) * kSlot; };
            auto barOf = [&](uint64_t q) { return smemAddr(&bar[(q - first) % kStages]); };
            auto parity = [&](uint64_t q) { return static_cast<unsigned>(((q - first) / kStages) & 1u); };
            auto issue = [&](uint64_t q) { bulkLoad(smemAddr(slot(q) + dstOff), cur + q * pitch + lo, bytes, barOf(q)); };

            if(threadIdx.x == 0)
            {
                for(int k = 0; k < kStages; ++k)
                    mbarInit(smemAddr(&bar[k]), 1u);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                for(uint64_t q = first; q < first + kStages && q <= re; ++q)
                    issue(q);
            }
            __syncthreads();

            int const lane = threadIdx.x & 31;
            uint64_t const c0 = s0 + 2u * threadIdx.x; // storage columns c0, c0 + 1 of this thread
            bool const live = c0 < width;
            int const i0 = 2 + 2 * static_cast<int>(threadIdx.x); // slot index of c0
            double const k = __dsub_rn(__dsub_rn(1.0, __dmul_rn(2.0, rX)), __dmul_rn(2.0, rY));
            auto pairAt = [&](uint64_t q) { return *reinterpret_cast<double2 const*>(slot(q) + i0); };

            mbarWait(barOf(first), parity(first), timeoutNs, errWord);
            double2 up = pairAt(first);
            mbarWait(barOf(rb), parity(rb), timeoutNs, errWord);
            double2 mid = pairAt(rb);
            __syncthreads(); // the slot of row rb - 1 is free
            if(threadIdx.x == 0 && first + kStages <= re)
            {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue(first + kStages);
            }
            for(uint64_t r = rb; r < re; ++r)
            {
                mbarWait(barOf(r + 1u), parity(r + 1u), timeoutNs, errWord);
                double2 const dn = pairAt(r + 1u);
                double const* const cs = slot(r);
                double westOfLo = __shfl_up_sync(0xffffffffu, mid.y, 1);
                double eastOfHi = __shfl_down_sync(0xffffffffu, mid.x, 1);
                if(lane == 0)
                    westOfLo = cs[i0 - 1];
                if(lane == 31)
                    eastOfHi = cs[i0 + 2];
                if(live)
                {
                    double* const q = next + r * pitch + c0;
                    bool const loIn = c0 >= 1u && c0 <= cols;
                    bool const hiIn = c0 + 1u <= cols;
                    double const vlo = cell(mid.x, westOfLo, mid.y, up.x, dn.x, k, rX, rY);
                    double const vhi = cell(mid.y, mid.x, eastOfHi, up.y, dn.y, k, rX, rY);
                    if(loIn && hiIn)
                        __stcs(reinterpret_cast<double2*>(q), make_double2(vlo, vhi));
                    else
                    {
                        if(loIn)
                            q[0] = vlo;
                        if(hiIn)
                            q[1] = vhi;
                    }
                }
                up = mid;
                mid = dn;
                __syncthreads(); // every thread is done with the slot of row r
                if(threadIdx.x == 0 && r + kStages <= re)
                {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    issue(r + kStages);
                }
            }
        }

        __global__ void __launch_bounds__(kRingThreads) heatKernelRing(
            double const* __restrict__ cur,
            double* __restrict__ next,
            uint64_t cols,
            uint64_t pitch,
            uint64_t rowBegin,
            uint64_t rowEnd,
            double rX,
            double rY,
            uint64_t timeoutNs,
            unsigned* errWord)
        {
            extern __shared__ __align__(128) double ring[]; // kStages slots of kSlot doubles
            __shared__ __align__(8) unsigned long long bar[kStages];
            uint64_t const rb = rowBegin + static_cast<uint64_t>(blockIdx.y) * kRingBand;
            if(rb >= rowEnd)
                return;
            uint64_t const re = rb + kRingBand < rowEnd ? rb + kRingBand : rowEnd;
            ringBand(cur, next, cols, pitch, rb, re, rX, rY, timeoutNs, errWord, ring, bar);
        }

        // rows [rowBegin, rowEnd) of the interior, one band of kBand rows per blockIdx.y
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
            uint64_t const rb = rowBegin + static_cast<uint64_t>(blockIdx.y) * kBand;
            if(rb >= rowEnd)
                return;
            uint64_t const re = rb + kBand < rowEnd ? rb + kBand : rowEnd;
            heatBand(cur, next, cols, pitch, rb, re, rX, rY, ~uint64_t{0} - 1u, nullptr, nullptr);
        }

        // ------------------------------------------------------------------------ step fused with the halo exchange
        // Halo mailbox of one rank (cudaMalloc, mapped by its neighbours through CUDA IPC):
        //   u32  flag[2 sides][2 parities][kMaxColBlocks]   step number (+1) whose row slice column block x has written
        //   f64  row[2 sides][2 parities][cols + 2]         a neighbour's boundary row (storage columns)
        // side 0 holds the upper neighbour's last interior row (this rank's north ghost), side 1 the lower neighbour's
        // first interior row (south ghost). Step s reads parity (s - 1) & 1 and writes parity s & 1 of its neighbours.
        constexpr unsigned kMaxColBlocks = 1024; // columns up to 2 * 256 * 1024 - 2
        constexpr uint64_t kFlagBytes = 2u * 2u * kMaxColBlocks * sizeof(unsigned);

        __host__ __device__ inline uint64_t mailRowStride(uint64_t cols)
        {
            return ((cols + 2u) + 31u) & ~uint64_t{31u}; // doubles, 256-byte multiple
        }

        __host__ __device__ inline uint64_t mailBytes(uint64_t cols)
        {
            return kFlagBytes + 4u * mailRowStride(cols) * sizeof(double);
        }

        struct Mail
        {
            unsigned* flags;
            double* rows;
            uint64_t stride;

            __device__ unsigned* flag(int side, unsigned parity, unsigned x) const
            {
                return flags + (static_cast<unsigned>(side) * 2u + parity) * kMaxColBlocks + x;
            }

            __device__ double* row(int side, unsigned parity) const
            {
                return rows + (static_cast<uint64_t>(side) * 2u + parity) * stride;
            }
        };

        __device__ __forceinline__ unsigned ldAcquireSys32(unsigned const* p)
        {
            unsigned v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
            return v;
        }

        __device__ __forceinline__ void stReleaseSys32(unsigned* p, unsigned v)
        {
            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
        }

        // Thread 0 waits until flag >= want (bounded by %globaltimer); false (and the error word raised) on timeout.
        __device__ bool waitFlag(unsigned const* flag, unsigned want, uint64_t timeoutNs, unsigned* errWord)
        {
            __shared__ int ok;
            if(threadIdx.x == 0)
            {
                ok = 1;
                uint64_t const t0 = globalTimerNs();
                while(static_cast<int>(ldAcquireSys32(flag) - want) < 0)
                {
                    if(globalTimerNs() - t0 > timeoutNs)
                    {
                        atomicOr(errWord, kErrTimeout);
                        ok = 0;
                        break;
                    }
                    __nanosleep(128);
                }
            }
            __syncthreads();
            bool const r = ok != 0;
            __syncthreads(); // every thread has read `ok` before a second wait of the block rewrites it
            return r;
        }

        // This block's columns of `row` (storage row of `next`) into a neighbour's mailbox row, then the block's flag.
        __device__ void sendRow(double const* row, uint64_t cols, double* dst, unsigned* flag, unsigned value)
        {
            uint64_t const width = cols + 2u;
            uint64_t const c0 = 2u * (static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x);
            if(c0 + 1u < width)
                *reinterpret_cast<double2*>(dst + c0) = *reinterpret_cast<double2 const*>(row + c0);
            else if(c0 < width)
                dst[c0] = row[c0];
            __threadfence_system(); // the row reaches the neighbour before the flag that announces it
            __syncthreads();
            if(threadIdx.x == 0)
                stReleaseSys32(flag, value);
        }

        // One step of the slab: blockIdx.y = 0 is the first band, 1 the last band, the others the bands in between, so
        // that both boundary rows are computed and sent first. The boundary bands wait for the neighbours' rows of the
        // previous step; the interior bands never wait.
        __global__ void __launch_bounds__(kThreads) heatExchangeKernel(
            double const* __restrict__ cur,
            double* __restrict__ next,
            uint64_t rows,
            uint64_t cols,
            uint64_t pitch,
            double rX,
            double rY,
            Mail mine,
            Mail up,   // upper neighbour's mailbox (rows == nullptr: none, global boundary)
            Mail down, // lower neighbour's mailbox
            unsigned step,
            uint64_t timeoutNs,
            unsigned* errWord)
        {
            uint64_t const bands = (rows + kBand - 1u) / kBand;
            uint64_t band = blockIdx.y;
            if(bands > 1u)
                band = blockIdx.y == 0u ? 0u : (blockIdx.y == 1u ? bands - 1u : blockIdx.y - 1u);
            else if(blockIdx.y > 0u)
                return;
            uint64_t const rb = 1u + band * kBand;
            uint64_t const re = rb + kBand < rows + 1u ? rb + kBand : rows + 1u;
            bool const top = rb == 1u, bottom = re == rows + 1u;
            unsigned const rd = (step - 1u) & 1u, wr = step & 1u;
            double const* north = nullptr;
            double const* south = nullptr;
            if(top && up.rows)
            {
                if(!waitFlag(mine.flag(0, rd, blockIdx.x), step, timeoutNs, errWord))
                    return;
                north = mine.row(0, rd);
            }
            if(bottom && down.rows)
            {
                if(!waitFlag(mine.flag(1, rd, blockIdx.x), step, timeoutNs, errWord))
                    return;
                south = mine.row(1, rd);
            }
            heatBand(cur, next, cols, pitch, rb, re, rX, rY, rows, north, south);
            if(top && up.rows)
            {
                __syncthreads(); // the block's row 1 is in `next`
                sendRow(next + pitch, cols, up.row(1, wr), up.flag(1, wr, blockIdx.x), step + 1u);
            }
            if(bottom && down.rows)
            {
                __syncthreads();
                sendRow(next + rows * pitch, cols, down.row(0, wr), down.flag(0, wr, blockIdx.x), step + 1u);
            }
        }

        // The same step with the interior on the shared-memory ring (even storage widths): blockIdx.y = 0 is the first
        // band of kBand rows, 1 the last band (both on the register march, which takes its ghost rows from the
        // mailbox), the others the interior rows between them in bands of kRingBand rows streamed through the ring.
        __global__ void __launch_bounds__(kThreads) heatExchangeRingKernel(
            double const* __restrict__ cur,
            double* __restrict__ next,
            uint64_t rows,
            uint64_t cols,
            uint64_t pitch,
            double rX,
            double rY,
            Mail mine,
            Mail up,
            Mail down,
            unsigned step,
            uint64_t timeoutNs,
            unsigned* errWord)
        {
            extern __shared__ __align__(128) double ring[];
            __shared__ __align__(8) unsigned long long bar[kStages];
            uint64_t const topEnd = 1u + kBand < rows + 1u ? 1u + kBand : rows + 1u;
            uint64_t const lastBegin = rows + 1u > kBand ? rows + 1u - kBand : 1u;
            uint64_t const botBegin = lastBegin > topEnd ? lastBegin : topEnd;
            if(blockIdx.y >= 2u)
            {
                uint64_t const rb = topEnd + static_cast<uint64_t>(blockIdx.y - 2u) * kRingBand;
                if(rb >= botBegin)
                    return;
                uint64_t const re = rb + kRingBand < botBegin ? rb + kRingBand : botBegin;
                ringBand(cur, next, cols, pitch, rb, re, rX, rY, timeoutNs, errWord, ring, bar);
                return;
            }
            uint64_t rb = 1u, re = topEnd;
            if(blockIdx.y == 1u)
            {
                if(botBegin >= rows + 1u)
                    return; // one band holds every row: block y = 0 does it
                rb = botBegin;
                re = rows + 1u;
            }
            bool const top = rb == 1u, bottom = re == rows + 1u;
            unsigned const rd = (step - 1u) & 1u, wr = step & 1u;
            double const* north = nullptr;
            double const* south = nullptr;
            if(top && up.rows)
            {
                if(!waitFlag(mine.flag(0, rd, blockIdx.x), step, timeoutNs, errWord))
                    return;
                north = mine.row(0, rd);
            }
            if(bottom && down.rows)
            {
                if(!waitFlag(mine.flag(1, rd, blockIdx.x), step, timeoutNs, errWord))
                    return;
                south = mine.row(1, rd);
            }
            heatBand(cur, next, cols, pitch, rb, re, rX, rY, rows, north, south);
            if(top && up.rows)
            {
                __syncthreads(); // the block's row 1 is in `next`
                sendRow(next + pitch, cols, up.row(1, wr), up.flag(1, wr, blockIdx.x), step + 1u);
            }
            if(bottom && down.rows)
            {
                __syncthreads();
                sendRow(next + rows * pitch, cols, down.row(0, wr), down.flag(0, wr, blockIdx.x), step + 1u);
            }
        }

        // Step-0 rows: this rank's first and last interior rows of the initial field into the neighbours' mailboxes.
        __global__ void __launch_bounds__(kThreads) heatPublishKernel(
            double const* __restrict__ u,
            uint64_t rows,
            uint64_t cols,
            uint64_t pitch,
            Mail up,
            Mail down,
            unsigned step)
        {
            unsigned const wr = step & 1u;
            if(blockIdx.y == 0u && up.rows)
                sendRow(u + pitch, cols, up.row(1, wr), up.flag(1, wr, blockIdx.x), step + 1u);
            if(blockIdx.y == 1u && down.rows)
                sendRow(u + rows * pitch, cols, down.row(0, wr), down.flag(0, wr, blockIdx.x), step + 1u);
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

// Halo mailbox of one rank and the mappings of its neighbours' mailboxes (CUDA IPC over NVLink).
struct a3b_halo
{
    int device = -1;
    int world = 0;
    int rank = 0;
    uint64_t cols = 0;
    void* local = nullptr;
    void* up = nullptr;   // mailbox of rank - 1
    void* down = nullptr; // mailbox of rank + 1
    unsigned step = 0;    // steps (and publications) issued so far, the same sequence on every rank
    bool connected = false;
};

using namespace a3b;

namespace
{
    Mail mailOf(void* base, uint64_t cols)
    {
        if(!base)
            return Mail{nullptr, nullptr, 0u};
        auto* b = static_cast<unsigned char*>(base);
        return Mail{reinterpret_cast<unsigned*>(b), reinterpret_cast<double*>(b + kFlagBytes), mailRowStride(cols)};
    }

    int haloCheck(a3b_halo* h, double const* u, uint64_t rows, uint64_t cols, uint64_t pitch, unsigned* colBlocks)
    {
        A3B_REQUIRE(h && h->connected, "halo mailbox not connected");
        A3B_REQUIRE(u, "null grid pointer");
        A3B_REQUIRE(cols == h->cols, "grid columns differ from the mailbox's");
        A3B_REQUIRE(rows >= 1u && pitch >= cols + 2u, "bad slab shape");
        A3B_REQUIRE(aligned16(u) && pitch % 2u == 0u, "halo steps need 16-byte aligned rows (even pitch)");
        int dev = -1;
        A3B_CUDA(cudaGetDevice(&dev));
        A3B_REQUIRE(dev == h->device, "halo mailbox used on a different device than the one it was created on");
        uint64_t const packs = (cols + 2u + 1u) / 2u;
        *colBlocks = static_cast<unsigned>((packs + kThreads - 1) / kThreads);
        return A3B_OK;
    }
} // namespace

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
        if(vec && cols % 2u == 0u)
        {
            // even storage width: every copied row segment is a whole number of 16-byte units
            static std::atomic<int> attrSet[kMaxDevices] = {};
            if(!attrSet[props->ordinal].load(std::memory_order_relaxed))
            {
                A3B_CUDA(cudaFuncSetAttribute(heatKernelRing, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              static_cast<int>(kRingSmem)));
                attrSet[props->ordinal].store(1, std::memory_order_relaxed);
            }
            uint64_t const ringBands = (row_end - row_begin + kRingBand - 1) / kRingBand;
            uint64_t const strips = (cols + 2u + kStrip - 1) / kStrip;
            A3B_REQUIRE(ringBands < 65536u, "too many row bands");
            dim3 const grid(static_cast<unsigned>(strips), static_cast<unsigned>(ringBands));
            heatKernelRing<<<grid, kRingThreads, kRingSmem, s>>>(cur, next, cols, pitch_elems, row_begin, row_end, rX,
                                                                 rY, waitTimeoutNs(), props->errWord);
        }
        else if(vec)
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

    size_t a3b_halo_bytes(uint64_t cols)
    {
        return static_cast<size_t>(mailBytes(cols));
    }

    int a3b_halo_create(int world, int rank, uint64_t cols, a3b_halo** halo, void* local_handle)
    {
        A3B_REQUIRE(halo && local_handle, "null argument");
        A3B_REQUIRE(world >= 1 && rank >= 0 && rank < world, "world/rank out of range");
        A3B_REQUIRE(cols >= 1u && (cols + 2u + 1u) / 2u <= static_cast<uint64_t>(kThreads) * kMaxColBlocks,
                    "too many columns for the halo mailbox");
        auto* h = new a3b_halo{};
        h->world = world;
        h->rank = rank;
        h->cols = cols;
        cudaError_t e = cudaGetDevice(&h->device);
        if(e == cudaSuccess)
            e = cudaMalloc(&h->local, mailBytes(cols));
        if(e == cudaSuccess)
            e = cudaMemset(h->local, 0, mailBytes(cols));
        if(e == cudaSuccess)
            e = cudaDeviceSynchronize(); // zeroed before a neighbour can write into it
        cudaIpcMemHandle_t ih{};
        if(e == cudaSuccess)
            e = cudaIpcGetMemHandle(&ih, h->local);
        if(e != cudaSuccess)
        {
            if(h->local)
                cudaFree(h->local);
            delete h;
            return cudaFail(e, "a3b_halo_create");
        }
        std::memcpy(local_handle, &ih, sizeof(ih));
        *halo = h;
        return A3B_OK;
    }

    int a3b_halo_connect(a3b_halo* h, void const* handles)
    {
        A3B_REQUIRE(h && handles, "null argument");
        A3B_REQUIRE(!h->connected, "halo mailbox already connected");
        auto const* hs = static_cast<cudaIpcMemHandle_t const*>(handles);
        cudaError_t e = cudaSuccess;
        if(h->rank > 0)
            e = cudaIpcOpenMemHandle(&h->up, hs[h->rank - 1], cudaIpcMemLazyEnablePeerAccess);
        if(e == cudaSuccess && h->rank + 1 < h->world)
            e = cudaIpcOpenMemHandle(&h->down, hs[h->rank + 1], cudaIpcMemLazyEnablePeerAccess);
        if(e != cudaSuccess)
        {
            if(h->up)
                cudaIpcCloseMemHandle(h->up);
            h->up = nullptr;
            return cudaFail(e, "cudaIpcOpenMemHandle (halo mailbox)");
        }
        h->connected = true;
        return A3B_OK;
    }

    int a3b_halo_destroy(a3b_halo* h)
    {
        if(!h)
            return A3B_OK;
        int rc = A3B_OK;
        if(h->up && cudaIpcCloseMemHandle(h->up) != cudaSuccess)
            rc = A3B_ERR_CUDA;
        if(h->down && cudaIpcCloseMemHandle(h->down) != cudaSuccess)
            rc = A3B_ERR_CUDA;
        if(h->local && cudaFree(h->local) != cudaSuccess)
            rc = A3B_ERR_CUDA;
        delete h;
        if(rc)
            setError("a3b_halo_destroy: releasing a mapping or the mailbox failed");
        return rc;
    }

    int a3b_heat_halo_publish(a3b_stream_t stream, a3b_halo* h, double const* u, uint64_t rows, uint64_t cols,
                              uint64_t pitch_elems)
    {
        unsigned colBlocks = 0;
        int rc = haloCheck(h, u, rows, cols, pitch_elems, &colBlocks);
        if(rc)
            return rc;
        unsigned const step = ++h->step;
        dim3 const grid(colBlocks, 2u);
        heatPublishKernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
            u, rows, cols, pitch_elems, mailOf(h->up, cols), mailOf(h->down, cols), step);
        A3B_CHECK_LAUNCH("heat halo publish launch");
        return A3B_OK;
    }

    int a3b_heat_step_halo(a3b_stream_t stream, a3b_halo* h, double const* cur, double* next, uint64_t rows,
                           uint64_t cols, uint64_t pitch_elems, double rX, double rY)
    {
        unsigned colBlocks = 0;
        int rc = haloCheck(h, cur, rows, cols, pitch_elems, &colBlocks);
        if(rc)
            return rc;
        A3B_REQUIRE(next && aligned16(next) && cur != next, "bad output grid");
        DeviceProps const* props = nullptr;
        rc = currentDevice(&props);
        if(rc)
            return rc;
        uint64_t const bands = (rows + kBand - 1) / kBand;
        A3B_REQUIRE(bands < 65536u, "too many row bands");
        unsigned const step = ++h->step;
        if(cols % 2u == 0u)
        {
            // boundary bands of kBand rows, the interior in ring bands of kRingBand rows
            static std::atomic<int> attrSet[kMaxDevices] = {};
            if(!attrSet[props->ordinal].load(std::memory_order_relaxed))
            {
                A3B_CUDA(cudaFuncSetAttribute(heatExchangeRingKernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              static_cast<int>(kRingSmem)));
                attrSet[props->ordinal].store(1, std::memory_order_relaxed);
            }
            uint64_t const topEnd = 1u + kBand < rows + 1u ? 1u + kBand : rows + 1u;
            uint64_t const lastBegin = rows + 1u > kBand ? rows + 1u - kBand : 1u;
            uint64_t const botBegin = lastBegin > topEnd ? lastBegin : topEnd;
            uint64_t const inner = (botBegin - topEnd + kRingBand - 1) / kRingBand;
            A3B_REQUIRE(inner + 2u < 65536u, "too many row bands");
            dim3 const grid(colBlocks, static_cast<unsigned>(2u + inner));
            heatExchangeRingKernel<<<grid, kThreads, kRingSmem, static_cast<cudaStream_t>(stream)>>>(
                cur, next, rows, cols, pitch_elems, rX, rY, mailOf(h->local, cols), mailOf(h->up, cols),
                mailOf(h->down, cols), step, waitTimeoutNs(), props->errWord);
        }
        else
        {
            dim3 const grid(colBlocks, static_cast<unsigned>(bands));
            heatExchangeKernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
                cur, next, rows, cols, pitch_elems, rX, rY, mailOf(h->local, cols), mailOf(h->up, cols),
                mailOf(h->down, cols), step, waitTimeoutNs(), props->errWord);
        }
        A3B_CHECK_LAUNCH("heat halo step launch");
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
