// All-pairs nBody velocity kick (+ optional fused drift) on the FP32 pipe.
//
// Replaces UpdateVelocitiesKernel (example/nBody/src/Kernels.hpp:24-124) and, in the fused step, the UpdatePositions
// functor run through onHost::concurrent (Kernels.hpp:126-142, nBody.cpp:196-205).
//
// Per pair (i, j): d = p_j - p_i; r2 = |d|^2 + eps; inv = rsqrt(r2^3); a_i += m_j * inv * d. Not a dense contraction,
// so no tensor cores: the pair math is 12 FP32 lane operations plus one MUFU rsqrt. Each thread keeps 6 i-bodies in
// registers as three packed pairs and evaluates them with the sm_100 packed FP32x2 instructions (__fadd2_rn,
// __fmul2_rn, __ffma2_rn), which halves the issue slots of the FP32 work and leaves room for the MUFU and the shared
// memory broadcast of each j-body (one 16-byte LDS per j for 6 pairs).
//
// Work split: items = (block of 768 i-bodies) x (slice of the j range). A resident grid pulls items from an atomic
// counter (dynamic balance across the 148 SMs) and writes per-slice partial accelerations; a second kernel sums the
// slices in fixed order, applies v += a*dt and optionally x += v*dt, so results do not depend on scheduling.
#include "common.cuh"

namespace a3b
{
    namespace
    {
#ifndef A3B_NBODY_PAIRS
#define A3B_NBODY_PAIRS 3
#endif
#ifndef A3B_NBODY_THREADS
#define A3B_NBODY_THREADS 128
#endif
        constexpr int kThreads = A3B_NBODY_THREADS;
        constexpr int kPairs = A3B_NBODY_PAIRS;         // packed i-body pairs per thread
        constexpr int kPerThread = 2 * kPairs;
        constexpr int kIBlock = kThreads * kPerThread; // i-bodies per work item
        constexpr int kJTile = 512;                    // j-bodies staged in shared memory per step
        constexpr float kFar = 1.0e15f;                // padding body: far away and massless => contributes 0

        // Reciprocal square root as the single PTX instruction rsqrt.approx.ftz.f32 (one MUFU operation; the
        // library rsqrtf adds denormal handling around it, which cost 20% of the pair throughput here). Arguments are
        // r^6 with r^2 >= eps > 0, far above the denormal range; the parity tests bound the effect on positions.
        __device__ __forceinline__ float rsqrtApprox(float x)
        {
            float r;
            asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
            return r;
        }

        struct NbHeader
        {
            unsigned counter;
            unsigned pad[15];
        };

        __global__ void __launch_bounds__(kThreads) forceKernel(
            float const* __restrict__ m,
            float const* __restrict__ x,
            float const* __restrict__ y,
            float const* __restrict__ z,
            uint64_t nAll,
            uint64_t iBegin,
            uint64_t iCount,
            float eps,
            unsigned slices,
            uint64_t jPerSlice,
            unsigned nItems,
            NbHeader* hdr,
            float* __restrict__ partial, // [slices][3][iCount]
            uint64_t partialStride)      // = iCount
        {
            __shared__ float4 sj[kJTile];
            __shared__ unsigned sItem;
            float2 const eps2 = make_float2(eps, eps);

            while(true)
            {
                __syncthreads(); // previous item's readers of sj / sItem are done
                if(threadIdx.x == 0)
                {
                    unsigned const it = atomicAdd(&hdr->counter, 1u);
                    if(it == nItems + gridDim.x - 1u)
                        hdr->counter = 0u; // last claim of the launch: ready for the next call
                    sItem = it;
                }
                __syncthreads();
                unsigned const item = sItem;
                if(item >= nItems)
                    break;
                unsigned const iblk = item / slices;
                unsigned const slice = item - iblk * slices;

                // i-bodies of this thread: local index li = iblk*kIBlock + threadIdx.x + k*kThreads
                float2 nxi[kPairs], nyi[kPairs], nzi[kPairs]; // negated positions, packed pairs (2p, 2p+1)
                float2 ax[kPairs], ay[kPairs], az[kPairs];
#pragma unroll
                for(int p = 0; p < kPairs; ++p)
                {
                    float px[2], py[2], pz[2];
#pragma unroll
                    for(int h = 0; h < 2; ++h)
                    {
                        uint64_t const li = static_cast<uint64_t>(iblk) * kIBlock + threadIdx.x + (2 * p + h) * kThreads;
                        bool const ok = li < iCount;
                        uint64_t const gi = iBegin + (ok ? li : 0u);
                        px[h] = ok ? -x[gi] : 0.f;
                        py[h] = ok ? -y[gi] : 0.f;
                        pz[h] = ok ? -z[gi] : 0.f;
                    }
                    nxi[p] = make_float2(px[0], px[1]);
                    nyi[p] = make_float2(py[0], py[1]);
                    nzi[p] = make_float2(pz[0], pz[1]);
                    ax[p] = ay[p] = az[p] = make_float2(0.f, 0.f);
                }

                uint64_t const jBegin = static_cast<uint64_t>(slice) * jPerSlice;
                uint64_t jEnd = jBegin + jPerSlice;
                if(jEnd > nAll)
                    jEnd = nAll;
                for(uint64_t jt = jBegin; jt < jEnd; jt += kJTile)
                {
                    __syncthreads();
                    for(int t = threadIdx.x; t < kJTile; t += kThreads)
                    {
                        uint64_t const j = jt + t;
                        sj[t] = j < jEnd ? make_float4(x[j], y[j], z[j], m[j]) : make_float4(kFar, kFar, kFar, 0.f);
                    }
                    __syncthreads();
#pragma unroll 4
                    for(int t = 0; t < kJTile; ++t)
                    {
                        float4 const b = sj[t];
                        float2 const bx = make_float2(b.x, b.x);
                        float2 const by = make_float2(b.y, b.y);
                        float2 const bz = make_float2(b.z, b.z);
                        float2 const bm = make_float2(b.w, b.w);
#pragma unroll
                        for(int p = 0; p < kPairs; ++p)
                        {
                            float2 const dx = __fadd2_rn(bx, nxi[p]);
                            float2 const dy = __fadd2_rn(by, nyi[p]);
                            float2 const dz = __fadd2_rn(bz, nzi[p]);
                            float2 r2 = __ffma2_rn(dz, dz, eps2);
                            r2 = __ffma2_rn(dy, dy, r2);
                            r2 = __ffma2_rn(dx, dx, r2);
                            float2 const r6 = __fmul2_rn(__fmul2_rn(r2, r2), r2);
                            float2 const inv = make_float2(rsqrtApprox(r6.x), rsqrtApprox(r6.y));
                            float2 const s = __fmul2_rn(bm, inv);
                            ax[p] = __ffma2_rn(s, dx, ax[p]);
                            ay[p] = __ffma2_rn(s, dy, ay[p]);
                            az[p] = __ffma2_rn(s, dz, az[p]);
                        }
                    }
                }

                float* const px = partial + static_cast<uint64_t>(slice) * 3u * partialStride;
#pragma unroll
                for(int p = 0; p < kPairs; ++p)
#pragma unroll
                    for(int h = 0; h < 2; ++h)
                    {
                        uint64_t const li = static_cast<uint64_t>(iblk) * kIBlock + threadIdx.x + (2 * p + h) * kThreads;
                        if(li < iCount)
                        {
                            px[li] = h ? ax[p].y : ax[p].x;
                            px[partialStride + li] = h ? ay[p].y : ay[p].x;
                            px[2 * partialStride + li] = h ? az[p].y : az[p].x;
                        }
                    }
            }
        }

        // v += (sum over slices of a) * dt; optionally x += v * dt (positions of the local bodies at pos + iBegin)
        __global__ void __launch_bounds__(256) kickKernel(
            float const* __restrict__ partial,
            uint64_t stride,
            unsigned slices,
            uint64_t iCount,
            float* __restrict__ vx,
            float* __restrict__ vy,
            float* __restrict__ vz,
            float dt,
            float* __restrict__ x,
            float* __restrict__ y,
            float* __restrict__ z)
        {
            uint64_t const S = static_cast<uint64_t>(gridDim.x) * blockDim.x;
            for(uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < iCount; i += S)
            {
                float a[3] = {0.f, 0.f, 0.f};
                for(unsigned s = 0; s < slices; ++s)
                {
                    float const* p = partial + static_cast<uint64_t>(s) * 3u * stride;
                    a[0] = __fadd_rn(a[0], p[i]);
                    a[1] = __fadd_rn(a[1], p[stride + i]);
                    a[2] = __fadd_rn(a[2], p[2 * stride + i]);
                }
                float const nvx = __fadd_rn(vx[i], __fmul_rn(a[0], dt));
                float const nvy = __fadd_rn(vy[i], __fmul_rn(a[1], dt));
                float const nvz = __fadd_rn(vz[i], __fmul_rn(a[2], dt));
                vx[i] = nvx;
                vy[i] = nvy;
                vz[i] = nvz;
                if(x)
                {
                    x[i] = __fadd_rn(x[i], __fmul_rn(nvx, dt));
                    y[i] = __fadd_rn(y[i], __fmul_rn(nvy, dt));
                    z[i] = __fadd_rn(z[i], __fmul_rn(nvz, dt));
                }
            }
        }

        int nbodyRun(
            cudaStream_t s,
            float const* m,
            float const* x,
            float const* y,
            float const* z,
            uint64_t nAll,
            uint64_t iBegin,
            uint64_t iCount,
            float* vx,
            float* vy,
            float* vz,
            float dt,
            float eps,
            float* px,
            float* py,
            float* pz)
        {
            A3B_REQUIRE(m && x && y && z && vx && vy && vz, "null pointer");
            A3B_REQUIRE(iBegin + iCount <= nAll, "i range outside the body arrays");
            A3B_REQUIRE(eps >= 0.f, "softening must be non-negative");
            if(iCount == 0)
                return A3B_OK;
            DeviceProps const* props = nullptr;
            int rc = currentDevice(&props);
            if(rc)
                return rc;
            static std::atomic<int> resident[kMaxDevices] = {};
            int r = 0;
            rc = residentPerSm(props, resident, forceKernel, kThreads, &r);
            if(rc)
                return rc;
            unsigned const grid = static_cast<unsigned>(props->smCount) * static_cast<unsigned>(r);
            uint64_t const iBlocks = (iCount + kIBlock - 1) / kIBlock;
            // enough items for ~8 per resident block, slices of at least 2 j-tiles
            uint64_t slices = 1;
            while(iBlocks * slices < 8ull * grid && nAll / (slices * 2) >= 2ull * kJTile)
                slices *= 2;
            uint64_t const jPer = ((nAll + slices - 1) / slices + kJTile - 1) / kJTile * kJTile;
            slices = (nAll + jPer - 1) / jPer;
            uint64_t const nItems = iBlocks * slices;
            A3B_REQUIRE(nItems + grid < 0xFFFFFFFFull, "problem too large");

            void* scr = nullptr;
            size_t const need = sizeof(NbHeader) + sizeof(float) * 3u * slices * iCount;
            rc = streamScratch(s, kScratchNbody, need, &scr);
            if(rc)
                return rc;
            auto* hdr = static_cast<NbHeader*>(scr);
            auto* partial = reinterpret_cast<float*>(hdr + 1);
            forceKernel<<<grid, kThreads, 0, s>>>(m, x, y, z, nAll, iBegin, iCount, eps, static_cast<unsigned>(slices),
                                                  jPer, static_cast<unsigned>(nItems), hdr, partial, iCount);
            A3B_CHECK_LAUNCH("nbody force launch");
            uint64_t const kb = (iCount + 255) / 256;
            unsigned const kgrid = static_cast<unsigned>(kb < 4096 ? kb : 4096);
            kickKernel<<<kgrid, 256, 0, s>>>(partial, iCount, static_cast<unsigned>(slices), iCount, vx, vy, vz, dt, px,
                                             py, pz);
            A3B_CHECK_LAUNCH("nbody kick launch");
            return A3B_OK;
        }
    } // namespace
} // namespace a3b

using namespace a3b;

extern "C"
{
    int a3b_nbody_update_velocities(a3b_stream_t stream, float const* m, float const* x, float const* y,
                                    float const* z, uint64_t n_all, uint64_t i_begin, uint64_t i_count, float* vx,
                                    float* vy, float* vz, float dt, float eps)
    {
        return nbodyRun(static_cast<cudaStream_t>(stream), m, x, y, z, n_all, i_begin, i_count, vx, vy, vz, dt, eps,
                        nullptr, nullptr, nullptr);
    }

    int a3b_nbody_step(a3b_stream_t stream, float const* m, float* x, float* y, float* z, uint64_t n_all,
                       uint64_t i_begin, uint64_t i_count, float* vx, float* vy, float* vz, float dt, float eps)
    {
        A3B_REQUIRE(x && y && z, "null pointer");
        return nbodyRun(static_cast<cudaStream_t>(stream), m, x, y, z, n_all, i_begin, i_count, vx, vy, vz, dt, eps,
                        x + i_begin, y + i_begin, z + i_begin);
    }
}
