// All-pairs nBody velocity kick (+ optional drift) on the FP32 pipe.
//
// Replaces UpdateVelocitiesKernel (example/nBody/src/Kernels.hpp:24-124) and, in the full step, the UpdatePositions
// functor run through onHost::concurrent (Kernels.hpp:126-142, nBody.cpp:196-205).
//
// Per pair (i, j): d = p_j - p_i; r2 = |d|^2 + eps; inv = rsqrt(r2^3); a_i += m_j * inv * d. Not a dense contraction,
// so no tensor cores: the pair math is 12 FP32 lane operations plus one MUFU rsqrt. Each thread keeps PAIRS packed
// pairs of i-bodies in registers and evaluates them with the sm_100 packed FP32x2 instructions (__fadd2_rn,
// __fmul2_rn, __ffma2_rn), which halves the issue slots of the FP32 work and leaves room for the MUFU and the shared
// memory broadcast of each j-body (one 16-byte LDS per j).
//
// Summation order: every i-body accumulates its pairs one j after the other in index order, as the reference kernel
// does (its per-thread loop over the j chunks, Kernels.hpp:67-111). fp32 sums of 2^18 terms carry rounding errors
// large enough that a different order (e.g. partial sums over j-slices combined afterwards) moves the bodies of the
// 262144-body, 10-step workload by up to 2.3e-4 of the position range away from the reference's trajectory, above
// the 1e-4 tolerance; with the reference's order the kernel stays within 4e-6 (FMA contraction and the MUFU rsqrt
// are the only differences). So the work is split over i only: a block owns 2 * PAIRS * THREADS i-bodies, walks
// all j-bodies through shared memory tiles, and applies the kick v += a * dt to its own bodies at the end. The block
// size is picked per launch so that the blocks spread evenly over the SMs; grids that would leave 3-4 warps per SM
// sub-partition run a variant with one i-body per thread and the j-bodies packed in pairs instead (same bits).
#include "common.cuh"

namespace a3b
{
    namespace
    {
        constexpr int kJTile = 512;             // j-bodies staged in shared memory per step
        constexpr float kFar = 1.0e15f;         // padding body: far away and massless => contributes exactly 0

        // Reciprocal square root as the single PTX instruction rsqrt.approx.ftz.f32 (one MUFU operation; the
        // library rsqrtf adds denormal handling around it, which cost 20% of the pair throughput here). Arguments are
        // r^6 with r^2 >= eps > 0, far above the denormal range; the parity tests bound the effect on positions.
        __device__ __forceinline__ float rsqrtApprox(float x)
        {
            float r;
            asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
            return r;
        }

        // At least MINB resident blocks: with 8, 50.2 TFLOP/s (64 threads) against 45.9 without the bound at 262144
        // bodies; the compiler keeps more j-steps in flight.
        template<int PAIRS, int THREADS, int JILP, int MINB>
        __global__ void __launch_bounds__(THREADS, MINB) forceKickKernel(
            float const* __restrict__ m,
            float const* __restrict__ x,
            float const* __restrict__ y,
            float const* __restrict__ z,
            uint64_t nAll,
            uint64_t iBegin,
            uint64_t iCount,
            float eps,
            float dt,
            float* __restrict__ vx,
            float* __restrict__ vy,
            float* __restrict__ vz)
        {
            constexpr int kIBlock = 2 * PAIRS * THREADS;
            constexpr int kUnroll = PAIRS == 1 ? 8 : 4;
            static_assert(kJTile % JILP == 0 && kUnroll % JILP == 0, "j-steps must divide the tile and the unroll");
            __shared__ float4 sj[kJTile]; // {x, y, z, m} per j-body; one broadcast 16-byte load per j
            float2 const eps2 = make_float2(eps, eps);

            // i-bodies of this thread: local index li = blockIdx.x * kIBlock + threadIdx.x + k * THREADS
            float2 nxi[PAIRS], nyi[PAIRS], nzi[PAIRS]; // negated positions, packed pairs (2p, 2p+1)
            float2 ax[PAIRS], ay[PAIRS], az[PAIRS];
#pragma unroll
            for(int p = 0; p < PAIRS; ++p)
            {
                float px[2], py[2], pz[2];
#pragma unroll
                for(int h = 0; h < 2; ++h)
                {
                    uint64_t const li = static_cast<uint64_t>(blockIdx.x) * kIBlock + threadIdx.x + (2 * p + h) * THREADS;
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

            for(uint64_t jt = 0; jt < nAll; jt += kJTile)
            {
                __syncthreads(); // the previous tile's readers are done
                for(int t = threadIdx.x; t < kJTile; t += THREADS)
                {
                    uint64_t const j = jt + t;
                    sj[t] = j < nAll ? make_float4(x[j], y[j], z[j], m[j]) : make_float4(kFar, kFar, kFar, 0.f);
                }
                __syncthreads();
#pragma unroll(kUnroll / JILP)
                for(int t = 0; t < kJTile; t += JILP)
                {
                    // the distance terms of JILP consecutive j-bodies are independent of each other and of the
                    // sums; the sums then take them in index order
                    float2 dx[JILP][PAIRS], dy[JILP][PAIRS], dz[JILP][PAIRS], sc[JILP][PAIRS];
#pragma unroll
                    for(int q = 0; q < JILP; ++q)
                    {
                        float4 const b = sj[t + q];
                        float2 const bx = make_float2(b.x, b.x);
                        float2 const by = make_float2(b.y, b.y);
                        float2 const bz = make_float2(b.z, b.z);
                        float2 const bm = make_float2(b.w, b.w);
#pragma unroll
                        for(int p = 0; p < PAIRS; ++p)
                        {
                            dx[q][p] = __fadd2_rn(bx, nxi[p]);
                            dy[q][p] = __fadd2_rn(by, nyi[p]);
                            dz[q][p] = __fadd2_rn(bz, nzi[p]);
                            float2 r2 = __ffma2_rn(dz[q][p], dz[q][p], eps2);
                            r2 = __ffma2_rn(dy[q][p], dy[q][p], r2);
                            r2 = __ffma2_rn(dx[q][p], dx[q][p], r2);
                            float2 const r6 = __fmul2_rn(__fmul2_rn(r2, r2), r2);
                            float2 const inv = make_float2(rsqrtApprox(r6.x), rsqrtApprox(r6.y));
                            sc[q][p] = __fmul2_rn(bm, inv);
                        }
                    }
#pragma unroll
                    for(int q = 0; q < JILP; ++q)
#pragma unroll
                        for(int p = 0; p < PAIRS; ++p)
                        {
                            ax[p] = __ffma2_rn(sc[q][p], dx[q][p], ax[p]);
                            ay[p] = __ffma2_rn(sc[q][p], dy[q][p], ay[p]);
                            az[p] = __ffma2_rn(sc[q][p], dz[q][p], az[p]);
                        }
                }
            }

            // kick: v += a * dt (two roundings, as Kernels.hpp:116-120)
#pragma unroll
            for(int p = 0; p < PAIRS; ++p)
#pragma unroll
                for(int h = 0; h < 2; ++h)
                {
                    uint64_t const li = static_cast<uint64_t>(blockIdx.x) * kIBlock + threadIdx.x + (2 * p + h) * THREADS;
                    if(li < iCount)
                    {
                        vx[li] = __fadd_rn(vx[li], __fmul_rn(h ? ax[p].y : ax[p].x, dt));
                        vy[li] = __fadd_rn(vy[li], __fmul_rn(h ? ay[p].y : ay[p].x, dt));
                        vz[li] = __fadd_rn(vz[li], __fmul_rn(h ? az[p].y : az[p].x, dt));
                    }
                }
        }

        // The same kick with one i-body per thread and the j-bodies taken in pairs: the distance terms of j and j+1
        // are one packed FP32x2 operation each (the i-position broadcast into both halves once, before the loop), and
        // the two contributions are accumulated one after the other, so every body still sums its j-bodies in index
        // order with the same operations: the bits equal forceKickKernel's. Twice the threads of the packed-i kernel
        // for the same bodies, at three more instructions per two pairs (scalar accumulation, a second 16-byte LDS):
        // it wins where the packed-i grid leaves 3-4 warps per SM sub-partition (131072 local bodies: 45.9 against
        // 43.0 TFLOP/s) and loses with more warps (262144: 47.7 against 50.2) or fewer (65536: 38.3 against 40.4).
        template<int THREADS, int MINB>
        __global__ void __launch_bounds__(THREADS, MINB) forceKickJPairKernel(
            float const* __restrict__ m,
            float const* __restrict__ x,
            float const* __restrict__ y,
            float const* __restrict__ z,
            uint64_t nAll,
            uint64_t iBegin,
            uint64_t iCount,
            float eps,
            float dt,
            float* __restrict__ vx,
            float* __restrict__ vy,
            float* __restrict__ vz)
        {
            constexpr int kJPairs = kJTile / 2;
            __shared__ float4 sxy[kJPairs]; // {x_j, x_j+1, y_j, y_j+1}
            __shared__ float4 szm[kJPairs]; // {z_j, z_j+1, m_j, m_j+1}
            uint64_t const li = static_cast<uint64_t>(blockIdx.x) * THREADS + threadIdx.x;
            bool const ok = li < iCount;
            uint64_t const gi = iBegin + (ok ? li : 0u);
            float const nx = ok ? -x[gi] : 0.f;
            float const ny = ok ? -y[gi] : 0.f;
            float const nz = ok ? -z[gi] : 0.f;
            float2 const nx2 = make_float2(nx, nx);
            float2 const ny2 = make_float2(ny, ny);
            float2 const nz2 = make_float2(nz, nz);
            float2 const eps2 = make_float2(eps, eps);
            float ax = 0.f, ay = 0.f, az = 0.f;
            for(uint64_t jt = 0; jt < nAll; jt += kJTile)
            {
                __syncthreads(); // the previous tile's readers are done
                for(int p = threadIdx.x; p < kJPairs; p += THREADS)
                {
                    uint64_t const j0 = jt + 2 * p;
                    uint64_t const j1 = j0 + 1;
                    float4 a, b;
                    if(j0 < nAll)
                    {
                        a.x = x[j0];
                        a.z = y[j0];
                        b.x = z[j0];
                        b.z = m[j0];
                    }
                    else
                    {
                        a.x = a.z = b.x = kFar;
                        b.z = 0.f;
                    }
                    if(j1 < nAll)
                    {
                        a.y = x[j1];
                        a.w = y[j1];
                        b.y = z[j1];
                        b.w = m[j1];
                    }
                    else
                    {
                        a.y = a.w = b.y = kFar;
                        b.w = 0.f;
                    }
                    sxy[p] = a;
                    szm[p] = b;
                }
                __syncthreads();
#pragma unroll 4
                for(int p = 0; p < kJPairs; ++p)
                {
                    float4 const a = sxy[p];
                    float4 const b = szm[p];
                    float2 const dx = __fadd2_rn(make_float2(a.x, a.y), nx2);
                    float2 const dy = __fadd2_rn(make_float2(a.z, a.w), ny2);
                    float2 const dz = __fadd2_rn(make_float2(b.x, b.y), nz2);
                    float2 r2 = __ffma2_rn(dz, dz, eps2);
                    r2 = __ffma2_rn(dy, dy, r2);
                    r2 = __ffma2_rn(dx, dx, r2);
                    float2 const r6 = __fmul2_rn(__fmul2_rn(r2, r2), r2);
                    float2 const inv = make_float2(rsqrtApprox(r6.x), rsqrtApprox(r6.y));
                    float2 const sc = __fmul2_rn(make_float2(b.z, b.w), inv);
                    ax = __fmaf_rn(sc.x, dx.x, ax);
                    ay = __fmaf_rn(sc.x, dy.x, ay);
                    az = __fmaf_rn(sc.x, dz.x, az);
                    ax = __fmaf_rn(sc.y, dx.y, ax);
                    ay = __fmaf_rn(sc.y, dy.y, ay);
                    az = __fmaf_rn(sc.y, dz.y, az);
                }
            }
            if(ok)
            {
                vx[li] = __fadd_rn(vx[li], __fmul_rn(ax, dt));
                vy[li] = __fadd_rn(vy[li], __fmul_rn(ay, dt));
                vz[li] = __fadd_rn(vz[li], __fmul_rn(az, dt));
            }
        }

        // drift x += v * dt of the local bodies (UpdatePositions, Kernels.hpp:126-142), after every kick of the step
        __global__ void __launch_bounds__(256) driftLocalKernel(
            float* __restrict__ x,
            float* __restrict__ y,
            float* __restrict__ z,
            float const* __restrict__ vx,
            float const* __restrict__ vy,
            float const* __restrict__ vz,
            uint64_t n,
            float dt)
        {
            uint64_t const S = static_cast<uint64_t>(gridDim.x) * blockDim.x;
            for(uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += S)
            {
                x[i] = __fadd_rn(x[i], __fmul_rn(vx[i], dt));
                y[i] = __fadd_rn(y[i], __fmul_rn(vy[i], dt));
                z[i] = __fadd_rn(z[i], __fmul_rn(vz[i], dt));
            }
        }

        // One block shape of the force kernel: i-bodies per thread (2 per packed pair, or 1 for the j-pair kernel),
        // threads per block and its launch function.
        struct Shape
        {
            int pairs;
            int threads;
            void (*kernel)(float const*, float const*, float const*, float const*, uint64_t, uint64_t, uint64_t, float,
                           float, float*, float*, float*);
            int bodiesPerThread() const
            {
                return pairs > 0 ? 2 * pairs : 1;
            }
        };

        // Measured at 262144 bodies (B200, TFLOP/s by the 20-flop convention): 1 pair x 64 threads 50.2, 1 x 128
        // 49.6, 2 x 128 40.2 (86% of the SMs' share filled), 3 x 128 36.0 (77%). The 64-thread shape is also the best
        // at the 32768 local bodies of 8 ranks (33.0 against 31.3). Its entry evaluates the distance terms of two
        // j-bodies side by side under a register cap for 10 resident blocks (5 warps per SM sub-partition): 50.6
        // against 50.1 for the plain loop at 8 blocks, measured in the same process.
        constexpr Shape kShapes[] = {
            {1, 64, forceKickKernel<1, 64, 2, 10>},
            {1, 128, forceKickKernel<1, 128, 1, 8>},
            {2, 128, forceKickKernel<2, 128, 1, 8>},
            {3, 128, forceKickKernel<3, 128, 1, 8>},
        };
        // The 1 x 64 shape with the distance terms of two j-bodies evaluated side by side, for grids that leave at
        // most 2 warps per SM sub-partition (local counts <= 65536): 32768 bodies 34.8 against 32.7 TFLOP/s, 65536
        // 40.3 against 39.7 (a four-j variant measured the same as two).
        constexpr Shape kFewWarpsShape = {1, 64, forceKickKernel<1, 64, 2, 8>};
        // One i-body per thread with j-bodies in pairs (forceKickJPairKernel), for grids of the 1 x 64 shape that
        // leave 3-4 warps per SM sub-partition.
        constexpr Shape kJPairShape = {0, 128, forceKickJPairKernel<128, 8>};
        constexpr int kNumShapes = sizeof(kShapes) / sizeof(kShapes[0]);

        // Picks the shape whose blocks spread most evenly over the SMs: the busiest SM runs ceil(blocks / SMs)
        // blocks, so the useful fraction is iCount / (SMs * ceil(blocks / SMs) * bodies per block), scaled down when
        // an SM would hold fewer than 8 warps (too few to keep the FP32 pipe busy). Ties go to more pairs per
        // thread (more independent work per thread).
        int pickShape(DeviceProps const* props, uint64_t iCount, Shape const** shape)
        {
            static std::atomic<int> resident[kNumShapes][kMaxDevices] = {};
            double best = -1.0;
            int pick = 0;
            for(int k = 0; k < kNumShapes; ++k)
            {
                int r = 0;
                int rc = residentPerSm(props, resident[k], kShapes[k].kernel, kShapes[k].threads, &r);
                if(rc)
                    return rc;
                uint64_t const perBlock = static_cast<uint64_t>(kShapes[k].bodiesPerThread()) * kShapes[k].threads;
                uint64_t const blocks = (iCount + perBlock - 1) / perBlock;
                uint64_t const sms = static_cast<uint64_t>(props->smCount);
                uint64_t const perSm = (blocks + sms - 1) / sms;
                double score = static_cast<double>(iCount) / static_cast<double>(sms * perSm * perBlock);
                double const warps = static_cast<double>(perSm < static_cast<uint64_t>(r) ? perSm : r)
                                     * (kShapes[k].threads / 32);
                if(warps < 8.0)
                    score *= warps / 8.0;
                if(score > best * (1.0 + 1e-9)
                   || (score >= best * (1.0 - 1e-9) && kShapes[k].pairs > kShapes[pick].pairs))
                {
                    best = score;
                    pick = k;
                }
            }
#ifdef A3B_NBODY_FORCE_SHAPE
            pick = A3B_NBODY_FORCE_SHAPE; // tuning builds: one fixed entry of kShapes
#endif
            *shape = &kShapes[pick];
            uint64_t const perBlock0 = static_cast<uint64_t>(kShapes[0].bodiesPerThread()) * kShapes[0].threads;
            uint64_t const perSm0 = ((iCount + perBlock0 - 1) / perBlock0 + props->smCount - 1) / props->smCount;
            uint64_t const warps0 = perSm0 * (kShapes[0].threads / 32);
            if(pick == 0 && warps0 <= 8)
                *shape = &kFewWarpsShape; // <= 2 warps per sub-partition
            else if(pick == 0 && warps0 <= 16)
                *shape = &kJPairShape; // 3-4 warps per sub-partition
            return A3B_OK;
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
            Shape const* sh = nullptr;
            rc = pickShape(props, iCount, &sh);
            if(rc)
                return rc;
            uint64_t const perBlock = static_cast<uint64_t>(sh->bodiesPerThread()) * sh->threads;
            uint64_t const blocks = (iCount + perBlock - 1) / perBlock;
            A3B_REQUIRE(blocks < 0x7FFFFFFFull, "problem too large");
            sh->kernel<<<static_cast<unsigned>(blocks), sh->threads, 0, s>>>(m, x, y, z, nAll, iBegin, iCount, eps, dt,
                                                                             vx, vy, vz);
            A3B_CHECK_LAUNCH("nbody force launch");
            if(px)
            {
                uint64_t const kb = (iCount + 255) / 256;
                unsigned const grid = static_cast<unsigned>(kb < 4096 ? kb : 4096);
                driftLocalKernel<<<grid, 256, 0, s>>>(px, py, pz, vx, vy, vz, iCount, dt);
                A3B_CHECK_LAUNCH("nbody drift launch");
            }
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
