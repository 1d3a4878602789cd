// Element-wise streaming kernels: BabelStream copy/mul/add/triad/nstream/init, onHost::transform with recognised
// functors, fill, iota, the nBody drift and the seeded Philox input generators.
//
// Replaces SimdForEachKernel + SimdAlgo::concurrent (benchmark/babelstream/src/babelStreamMainTest.cpp:61-75,
// include/alpaka/onAcc/internal/SimdConcurrent.hpp:122-234) and SimdTransformKernel / SimdConcurrentKernel /
// SimdIotaKernel / generic fill (include/alpaka/onHost/algo/internal/transform.hpp:21-107, concurrent.hpp:18-67,
// iota.hpp:19-75, include/alpaka/api/generic.hpp:45-88).
//
// Design: the arrays are cut into chunks of 512 threads x (1 or 2) 16-byte packs per array and block b handles
// chunk b: a full grid of short-lived blocks, which the block scheduler hands out in index order, so the whole GPU
// sweeps memory front to back. Operations that touch two arrays (copy, mul, map) move two packs per thread (16 KB
// per array per block), those that touch three or four (add, triad, nstream) one (8 KB per array per block); these
// shapes measured best on B200 among 16/32-byte packs, 128/256/512-thread blocks and 1-4 packs per thread (2^25
// fp64: copy 6.70, add 6.98, triad 7.00 TB/s, against 6.24 / 6.50 TB/s for a resident grid walking the arrays
// grid-stride). Pointers that are not 16-byte aligned are walked element by element in the same chunk shape.
// Floating-point operations use explicitly rounded intrinsics, so results are bit-identical to an IEEE CPU
// evaluation of the same expression without contraction.
#include <type_traits>

#include "common.cuh"

namespace a3b
{
    namespace
    {
        constexpr int kBlock = 256;               // iota, generators, drift
        constexpr int kStreamBlock = 512;         // element-wise chunk kernel
        constexpr uint64_t kMaxGrid = 1ull << 31; // gridDim.x limit

        // packs per thread per chunk: 32 bytes of each array for operations on two arrays, 16 bytes for three or four
        template<typename T, int W, typename Op>
        __host__ __device__ constexpr int packsPerThread()
        {
            constexpr int mask = Op::R | Op::Wr;
            constexpr int arrays = (mask & 1) + ((mask >> 1) & 1) + ((mask >> 2) & 1);
            constexpr int bytes = arrays <= 2 ? 32 : 16;
            constexpr int pack = W * static_cast<int>(sizeof(T));
            return bytes / pack > 0 ? bytes / pack : 1;
        }

        template<typename T, int W>
        struct alignas(16) Pack
        {
            T v[W];
        };

        template<typename T>
        constexpr int packWidth()
        {
            return 16 / static_cast<int>(sizeof(T));
        }

        // explicitly rounded arithmetic (no FMA contraction); integers wrap
        __device__ __forceinline__ float addRn(float a, float b)
        {
            return __fadd_rn(a, b);
        }

        __device__ __forceinline__ double addRn(double a, double b)
        {
            return __dadd_rn(a, b);
        }

        __device__ __forceinline__ float mulRn(float a, float b)
        {
            return __fmul_rn(a, b);
        }

        __device__ __forceinline__ double mulRn(double a, double b)
        {
            return __dmul_rn(a, b);
        }

        template<typename T>
        __device__ __forceinline__ T addRn(T a, T b)
        {
            using U = std::make_unsigned_t<T>;
            return static_cast<T>(static_cast<U>(a) + static_cast<U>(b));
        }

        template<typename T>
        __device__ __forceinline__ T mulRn(T a, T b)
        {
            using U = std::make_unsigned_t<T>;
            return static_cast<T>(static_cast<U>(a) * static_cast<U>(b));
        }

        template<typename T, int W>
        __device__ __forceinline__ Pack<T, W> loadPack(T const* base, uint64_t packIdx)
        {
            if constexpr(W * sizeof(T) == 16)
            {
                uint4 raw = reinterpret_cast<uint4 const*>(base)[packIdx];
                return *reinterpret_cast<Pack<T, W>*>(&raw);
            }
            else
            {
                Pack<T, W> p;
#pragma unroll
                for(int k = 0; k < W; ++k)
                    p.v[k] = __ldcs(base + packIdx * W + k);
                return p;
            }
        }

        template<typename T, int W>
        __device__ __forceinline__ void storePack(T* base, uint64_t packIdx, Pack<T, W> const& p)
        {
            if constexpr(W * sizeof(T) == 16)
            {
                reinterpret_cast<uint4*>(base)[packIdx] = *reinterpret_cast<uint4 const*>(&p);
            }
            else
            {
#pragma unroll
                for(int k = 0; k < W; ++k)
                    __stcs(base + packIdx * W + k, p.v[k]);
            }
        }

        // ---------------------------------------------------------------- element-wise operations
        // Each op declares which of the three arrays it reads (R) and writes (Wr) as bit masks (1 = p0, 2 = p1,
        // 4 = p2) and maps one element triple.
        template<typename T>
        struct OpInit
        {
            static constexpr int R = 0, Wr = 7;
            T ia, ib, ic;
            __device__ void operator()(T& a, T& b, T& c) const
            {
                a = ia;
                b = ib;
                c = ic;
            }
        };

        template<typename T>
        struct OpCopy // c = a
        {
            static constexpr int R = 1, Wr = 4;
            __device__ void operator()(T& a, T&, T& c) const
            {
                c = a;
            }
        };

        template<typename T>
        struct OpMul // b = s * c
        {
            static constexpr int R = 4, Wr = 2;
            T s;
            __device__ void operator()(T&, T& b, T& c) const
            {
                b = mulRn(s, c);
            }
        };

        template<typename T>
        struct OpAdd // c = a + b
        {
            static constexpr int R = 3, Wr = 4;
            __device__ void operator()(T& a, T& b, T& c) const
            {
                c = addRn(a, b);
            }
        };

        template<typename T>
        struct OpTriad // a = b + s * c
        {
            static constexpr int R = 6, Wr = 1;
            T s;
            __device__ void operator()(T& a, T& b, T& c) const
            {
                a = addRn(b, mulRn(s, c));
            }
        };

        template<typename T>
        struct OpNStream // a = a + b + s * c  ==  (a + b) + (s * c)
        {
            static constexpr int R = 7, Wr = 1;
            T s;
            __device__ void operator()(T& a, T& b, T& c) const
            {
                a = addRn(addRn(a, b), mulRn(s, c));
            }
        };

        // onHost::transform with recognised functors: p0 = out, p1 = in0, p2 = in1
        template<typename T>
        struct MapCopy
        {
            static constexpr int R = 2, Wr = 1;
            __device__ void operator()(T& o, T& x, T&) const
            {
                o = x;
            }
        };

        template<typename T>
        struct MapScale
        {
            static constexpr int R = 2, Wr = 1;
            T alpha;
            __device__ void operator()(T& o, T& x, T&) const
            {
                o = mulRn(alpha, x);
            }
        };

        template<typename T>
        struct MapAdd
        {
            static constexpr int R = 6, Wr = 1;
            __device__ void operator()(T& o, T& x, T& y) const
            {
                o = addRn(x, y);
            }
        };

        template<typename T>
        struct MapMul
        {
            static constexpr int R = 6, Wr = 1;
            __device__ void operator()(T& o, T& x, T& y) const
            {
                o = mulRn(x, y);
            }
        };

        template<typename T>
        struct MapAxpy
        {
            static constexpr int R = 6, Wr = 1;
            T alpha;
            __device__ void operator()(T& o, T& x, T& y) const
            {
                o = addRn(x, mulRn(alpha, y));
            }
        };

        template<typename T>
        struct MapSquare
        {
            static constexpr int R = 2, Wr = 1;
            __device__ void operator()(T& o, T& x, T&) const
            {
                o = mulRn(x, x);
            }
        };

        template<typename T>
        struct MapFill
        {
            static constexpr int R = 0, Wr = 1;
            T value;
            __device__ void operator()(T& o, T&, T&) const
            {
                o = value;
            }
        };

        template<typename T, int W, int U, typename Op>
        __device__ __forceinline__ void applyPacks(
            Op const& op,
            T* p0,
            T* p1,
            T* p2,
            uint64_t const (&idx)[U],
            int count)
        {
            Pack<T, W> a[U], b[U], c[U];
#pragma unroll
            for(int u = 0; u < U; ++u)
            {
                if(u < count)
                {
                    if constexpr(Op::R & 1)
                        a[u] = loadPack<T, W>(p0, idx[u]);
                    if constexpr(Op::R & 2)
                        b[u] = loadPack<T, W>(p1, idx[u]);
                    if constexpr(Op::R & 4)
                        c[u] = loadPack<T, W>(p2, idx[u]);
                }
            }
#pragma unroll
            for(int u = 0; u < U; ++u)
            {
                if(u < count)
                {
#pragma unroll
                    for(int k = 0; k < W; ++k)
                        op(a[u].v[k], b[u].v[k], c[u].v[k]);
                    if constexpr(Op::Wr & 1)
                        storePack<T, W>(p0, idx[u], a[u]);
                    if constexpr(Op::Wr & 2)
                        storePack<T, W>(p1, idx[u], b[u]);
                    if constexpr(Op::Wr & 4)
                        storePack<T, W>(p2, idx[u], c[u]);
                }
            }
        }

        // W elements per pack; block c covers packs [c * kStreamBlock * U, (c + 1) * kStreamBlock * U), thread t
        // takes packs c * kStreamBlock * U + u * kStreamBlock + t (each warp instruction covers 32 consecutive
        // packs). The grid has one block per chunk (at least one): a full chunk moves all its packs at once with no
        // predicates, the last chunk checks each pack.
        template<typename T, int W, typename Op>
        __global__ void __launch_bounds__(kStreamBlock) streamKernel(Op op, T* p0, T* p1, T* p2, uint64_t n)
        {
            constexpr int U = packsPerThread<T, W, Op>();
            uint64_t const nPacks = n / W;
            uint64_t const chunk = static_cast<uint64_t>(kStreamBlock) * U;
            uint64_t const c = blockIdx.x;
            uint64_t idx[U];
#pragma unroll
            for(int u = 0; u < U; ++u)
                idx[u] = c * chunk + static_cast<uint64_t>(u) * kStreamBlock + threadIdx.x;
            if(c * chunk + chunk <= nPacks)
                applyPacks<T, W, U>(op, p0, p1, p2, idx, U);
            else
            {
                int count = 0;
#pragma unroll
                for(int u = 0; u < U; ++u)
                    if(idx[u] < nPacks)
                        count = u + 1;
                if(count > 0)
                    applyPacks<T, W, U>(op, p0, p1, p2, idx, count);
            }
            if constexpr(W > 1)
            {
                // tail elements after the last whole pack
                uint64_t const t = static_cast<uint64_t>(blockIdx.x) * kStreamBlock + threadIdx.x;
                uint64_t const e = nPacks * W + t;
                if(e < n)
                {
                    T a{}, b{}, c{};
                    if constexpr(Op::R & 1)
                        a = p0[e];
                    if constexpr(Op::R & 2)
                        b = p1[e];
                    if constexpr(Op::R & 4)
                        c = p2[e];
                    op(a, b, c);
                    if constexpr(Op::Wr & 1)
                        p0[e] = a;
                    if constexpr(Op::Wr & 2)
                        p1[e] = b;
                    if constexpr(Op::Wr & 4)
                        p2[e] = c;
                }
            }
        }

        // one block per chunk (at least one, so the tail elements of a pack-less array are handled); 0 when the
        // array needs more blocks than a grid holds (more than 2^39 packs)
        template<typename T, int W, typename Op>
        unsigned gridFor(uint64_t n)
        {
            uint64_t const chunk = static_cast<uint64_t>(kStreamBlock) * packsPerThread<T, W, Op>();
            uint64_t const chunks = (n / W + chunk - 1) / chunk;
            if(chunks >= kMaxGrid)
                return 0u;
            return static_cast<unsigned>(chunks > 0 ? chunks : 1);
        }

        template<typename T, typename Op>
        int launchStream(cudaStream_t s, Op op, T* p0, T* p1, T* p2, uint64_t n)
        {
            if(n == 0)
                return A3B_OK;
            DeviceProps const* props = nullptr;
            int rc = currentDevice(&props);
            if(rc)
                return rc;
            auto alignedTo = [&](uintptr_t a)
            {
                auto ok = [&](void const* p) { return (reinterpret_cast<uintptr_t>(p) & (a - 1u)) == 0u; };
                return (!(Op::R & 1 || Op::Wr & 1) || ok(p0)) && (!(Op::R & 2 || Op::Wr & 2) || ok(p1))
                       && (!(Op::R & 4 || Op::Wr & 4) || ok(p2));
            };
            constexpr int W16 = packWidth<T>();
            bool const a16 = alignedTo(16);
            unsigned const grid = a16 ? gridFor<T, W16, Op>(n) : gridFor<T, 1, Op>(n);
            if(grid == 0u)
            {
                setError("array of %llu elements needs more blocks than a grid holds", static_cast<unsigned long long>(n));
                return A3B_ERR_TOO_LARGE;
            }
            if(a16)
                streamKernel<T, W16, Op><<<grid, kStreamBlock, 0, s>>>(op, p0, p1, p2, n);
            else
                streamKernel<T, 1, Op><<<grid, kStreamBlock, 0, s>>>(op, p0, p1, p2, n);
            A3B_CHECK_LAUNCH("stream kernel launch");
            return A3B_OK;
        }

        template<typename T>
        int babel(cudaStream_t s, int kind, T* a, T* b, T* c, uint64_t n, double scalar, double const* init)
        {
            T const sc = static_cast<T>(scalar);
            switch(kind)
            {
            case A3B_STREAM_INIT:
                A3B_REQUIRE(init, "init values required for A3B_STREAM_INIT");
                return launchStream<T>(
                    s, OpInit<T>{static_cast<T>(init[0]), static_cast<T>(init[1]), static_cast<T>(init[2])}, a, b, c, n);
            case A3B_STREAM_COPY:
                return launchStream<T>(s, OpCopy<T>{}, a, b, c, n);
            case A3B_STREAM_MUL:
                return launchStream<T>(s, OpMul<T>{sc}, a, b, c, n);
            case A3B_STREAM_ADD:
                return launchStream<T>(s, OpAdd<T>{}, a, b, c, n);
            case A3B_STREAM_TRIAD:
                return launchStream<T>(s, OpTriad<T>{sc}, a, b, c, n);
            case A3B_STREAM_NSTREAM:
                return launchStream<T>(s, OpNStream<T>{sc}, a, b, c, n);
            default:
                setError("unknown BabelStream kind %d", kind);
                return A3B_ERR_INVALID;
            }
        }

        template<typename T>
        int mapT(cudaStream_t s, int kind, T* out, T* in0, T* in1, uint64_t n, double alpha)
        {
            T const al = static_cast<T>(alpha);
            switch(kind)
            {
            case A3B_MAP_COPY:
                return launchStream<T>(s, MapCopy<T>{}, out, in0, in1, n);
            case A3B_MAP_SCALE:
                return launchStream<T>(s, MapScale<T>{al}, out, in0, in1, n);
            case A3B_MAP_ADD:
                A3B_REQUIRE(in1, "in1 required");
                return launchStream<T>(s, MapAdd<T>{}, out, in0, in1, n);
            case A3B_MAP_MUL:
                A3B_REQUIRE(in1, "in1 required");
                return launchStream<T>(s, MapMul<T>{}, out, in0, in1, n);
            case A3B_MAP_AXPY:
                A3B_REQUIRE(in1, "in1 required");
                return launchStream<T>(s, MapAxpy<T>{al}, out, in0, in1, n);
            case A3B_MAP_SQUARE:
                return launchStream<T>(s, MapSquare<T>{}, out, in0, in1, n);
            default:
                setError("unknown transform kind %d", kind);
                return A3B_ERR_INVALID;
            }
        }

        template<typename T>
        __global__ void __launch_bounds__(kBlock) iotaKernel(T* out, uint64_t n, T start)
        {
            uint64_t const S = static_cast<uint64_t>(gridDim.x) * kBlock;
            for(uint64_t i = static_cast<uint64_t>(blockIdx.x) * kBlock + threadIdx.x; i < n; i += S)
                out[i] = addRn(start, static_cast<T>(i));
        }

        __global__ void __launch_bounds__(kBlock) randU32Kernel(uint32_t* out, uint64_t n, uint64_t seed, uint64_t start, int shift)
        {
            uint64_t const S = static_cast<uint64_t>(gridDim.x) * kBlock;
            for(uint64_t i = static_cast<uint64_t>(blockIdx.x) * kBlock + threadIdx.x; i < n; i += S)
                out[i] = philox4x32_10(seed, start + i).x >> shift;
        }

        __global__ void __launch_bounds__(kBlock) randU64Kernel(uint64_t* out, uint64_t n, uint64_t seed, uint64_t start)
        {
            uint64_t const S = static_cast<uint64_t>(gridDim.x) * kBlock;
            for(uint64_t i = static_cast<uint64_t>(blockIdx.x) * kBlock + threadIdx.x; i < n; i += S)
            {
                uint4 const r = philox4x32_10(seed, start + i);
                out[i] = (static_cast<uint64_t>(r.y) << 32) | r.x;
            }
        }

        __global__ void __launch_bounds__(kBlock) randF32Kernel(float* out, uint64_t n, uint64_t seed, uint64_t start, float lo, float hi)
        {
            uint64_t const S = static_cast<uint64_t>(gridDim.x) * kBlock;
            float const w = __fsub_rn(hi, lo);
            for(uint64_t i = static_cast<uint64_t>(blockIdx.x) * kBlock + threadIdx.x; i < n; i += S)
            {
                uint32_t const r = philox4x32_10(seed, start + i).x;
                float const u = __fmul_rn(static_cast<float>(r >> 8), 0x1p-24f);
                out[i] = __fadd_rn(lo, __fmul_rn(w, u));
            }
        }

        __global__ void __launch_bounds__(kBlock) driftKernel(
            float* __restrict__ x,
            float* __restrict__ y,
            float* __restrict__ z,
            float const* __restrict__ vx,
            float const* __restrict__ vy,
            float const* __restrict__ vz,
            uint64_t n,
            float dt)
        {
            uint64_t const S = static_cast<uint64_t>(gridDim.x) * kBlock;
            for(uint64_t i = static_cast<uint64_t>(blockIdx.x) * kBlock + threadIdx.x; i < n; i += S)
            {
                x[i] = __fadd_rn(x[i], __fmul_rn(vx[i], dt));
                y[i] = __fadd_rn(y[i], __fmul_rn(vy[i], dt));
                z[i] = __fadd_rn(z[i], __fmul_rn(vz[i], dt));
            }
        }

        int simpleGrid(uint64_t n, int* grid)
        {
            DeviceProps const* props = nullptr;
            int rc = currentDevice(&props);
            if(rc)
                return rc;
            uint64_t const want = (n + kBlock - 1) / kBlock;
            uint64_t const cap = static_cast<uint64_t>(props->smCount) * 8u;
            *grid = static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
            return A3B_OK;
        }
    } // namespace
} // namespace a3b

using namespace a3b;

extern "C"
{
    int a3b_babelstream(a3b_stream_t stream, int kind, int dtype, void* a, void* b, void* c, uint64_t n,
                        double scalar, double const* init)
    {
        A3B_REQUIRE(a && b && c, "null array pointer");
        auto s = static_cast<cudaStream_t>(stream);
        if(dtype == A3B_F64)
            return babel<double>(s, kind, static_cast<double*>(a), static_cast<double*>(b), static_cast<double*>(c), n,
                                 scalar, init);
        if(dtype == A3B_F32)
            return babel<float>(s, kind, static_cast<float*>(a), static_cast<float*>(b), static_cast<float*>(c), n,
                                scalar, init);
        setError("BabelStream supports A3B_F32 and A3B_F64 only (dtype %d)", dtype);
        return A3B_ERR_INVALID;
    }

    int a3b_transform(a3b_stream_t stream, int kind, int dtype, void* out, void const* in0, void const* in1,
                      uint64_t n, double alpha)
    {
        A3B_REQUIRE(out && in0, "null pointer");
        auto s = static_cast<cudaStream_t>(stream);
        void* i0 = const_cast<void*>(in0);
        void* i1 = const_cast<void*>(in1 ? in1 : in0);
        switch(dtype)
        {
        case A3B_I32:
            return mapT<int32_t>(s, kind, (int32_t*) out, (int32_t*) i0, (int32_t*) i1, n, alpha);
        case A3B_U32:
            return mapT<uint32_t>(s, kind, (uint32_t*) out, (uint32_t*) i0, (uint32_t*) i1, n, alpha);
        case A3B_I64:
            return mapT<int64_t>(s, kind, (int64_t*) out, (int64_t*) i0, (int64_t*) i1, n, alpha);
        case A3B_U64:
            return mapT<uint64_t>(s, kind, (uint64_t*) out, (uint64_t*) i0, (uint64_t*) i1, n, alpha);
        case A3B_F32:
            return mapT<float>(s, kind, (float*) out, (float*) i0, (float*) i1, n, alpha);
        case A3B_F64:
            return mapT<double>(s, kind, (double*) out, (double*) i0, (double*) i1, n, alpha);
        default:
            setError("unknown dtype %d", dtype);
            return A3B_ERR_INVALID;
        }
    }

    int a3b_fill(a3b_stream_t stream, int dtype, void* out, uint64_t n, void const* value)
    {
        A3B_REQUIRE(out && value, "null pointer");
        auto s = static_cast<cudaStream_t>(stream);
        switch(dtype)
        {
        case A3B_I32:
            return launchStream<int32_t>(s, MapFill<int32_t>{*(int32_t const*) value}, (int32_t*) out, nullptr, nullptr, n);
        case A3B_U32:
            return launchStream<uint32_t>(s, MapFill<uint32_t>{*(uint32_t const*) value}, (uint32_t*) out, nullptr, nullptr, n);
        case A3B_I64:
            return launchStream<int64_t>(s, MapFill<int64_t>{*(int64_t const*) value}, (int64_t*) out, nullptr, nullptr, n);
        case A3B_U64:
            return launchStream<uint64_t>(s, MapFill<uint64_t>{*(uint64_t const*) value}, (uint64_t*) out, nullptr, nullptr, n);
        case A3B_F32:
            return launchStream<float>(s, MapFill<float>{*(float const*) value}, (float*) out, nullptr, nullptr, n);
        case A3B_F64:
            return launchStream<double>(s, MapFill<double>{*(double const*) value}, (double*) out, nullptr, nullptr, n);
        default:
            setError("unknown dtype %d", dtype);
            return A3B_ERR_INVALID;
        }
    }

    int a3b_iota(a3b_stream_t stream, int dtype, void* out, uint64_t n, void const* start)
    {
        A3B_REQUIRE(out && start, "null pointer");
        if(n == 0)
            return A3B_OK;
        auto s = static_cast<cudaStream_t>(stream);
        int grid = 1;
        int rc = simpleGrid(n, &grid);
        if(rc)
            return rc;
        switch(dtype)
        {
        case A3B_I32:
            iotaKernel<int32_t><<<grid, kBlock, 0, s>>>((int32_t*) out, n, *(int32_t const*) start);
            break;
        case A3B_U32:
            iotaKernel<uint32_t><<<grid, kBlock, 0, s>>>((uint32_t*) out, n, *(uint32_t const*) start);
            break;
        case A3B_I64:
            iotaKernel<int64_t><<<grid, kBlock, 0, s>>>((int64_t*) out, n, *(int64_t const*) start);
            break;
        case A3B_U64:
            iotaKernel<uint64_t><<<grid, kBlock, 0, s>>>((uint64_t*) out, n, *(uint64_t const*) start);
            break;
        case A3B_F32:
            iotaKernel<float><<<grid, kBlock, 0, s>>>((float*) out, n, *(float const*) start);
            break;
        case A3B_F64:
            iotaKernel<double><<<grid, kBlock, 0, s>>>((double*) out, n, *(double const*) start);
            break;
        default:
            setError("unknown dtype %d", dtype);
            return A3B_ERR_INVALID;
        }
        A3B_CHECK_LAUNCH("iota launch");
        return A3B_OK;
    }

    int a3b_nbody_update_positions(a3b_stream_t stream, float* x, float* y, float* z, float const* vx,
                                   float const* vy, float const* vz, uint64_t n, float dt)
    {
        A3B_REQUIRE(x && y && z && vx && vy && vz, "null pointer");
        if(n == 0)
            return A3B_OK;
        int grid = 1;
        int rc = simpleGrid(n, &grid);
        if(rc)
            return rc;
        driftKernel<<<grid, kBlock, 0, static_cast<cudaStream_t>(stream)>>>(x, y, z, vx, vy, vz, n, dt);
        A3B_CHECK_LAUNCH("drift launch");
        return A3B_OK;
    }

    int a3b_random_u32(a3b_stream_t stream, uint32_t* out, uint64_t n, uint64_t seed, uint64_t start, int shift)
    {
        A3B_REQUIRE(out, "null pointer");
        A3B_REQUIRE(shift >= 0 && shift < 32, "shift out of range");
        if(n == 0)
            return A3B_OK;
        int grid = 1;
        int rc = simpleGrid(n, &grid);
        if(rc)
            return rc;
        randU32Kernel<<<grid, kBlock, 0, static_cast<cudaStream_t>(stream)>>>(out, n, seed, start, shift);
        A3B_CHECK_LAUNCH("random_u32 launch");
        return A3B_OK;
    }

    int a3b_random_u64(a3b_stream_t stream, uint64_t* out, uint64_t n, uint64_t seed, uint64_t start)
    {
        A3B_REQUIRE(out, "null pointer");
        if(n == 0)
            return A3B_OK;
        int grid = 1;
        int rc = simpleGrid(n, &grid);
        if(rc)
            return rc;
        randU64Kernel<<<grid, kBlock, 0, static_cast<cudaStream_t>(stream)>>>(out, n, seed, start);
        A3B_CHECK_LAUNCH("random_u64 launch");
        return A3B_OK;
    }

    int a3b_random_f32(a3b_stream_t stream, float* out, uint64_t n, uint64_t seed, uint64_t start, float lo, float hi)
    {
        A3B_REQUIRE(out, "null pointer");
        if(n == 0)
            return A3B_OK;
        int grid = 1;
        int rc = simpleGrid(n, &grid);
        if(rc)
            return rc;
        randF32Kernel<<<grid, kBlock, 0, static_cast<cudaStream_t>(stream)>>>(out, n, seed, start, lo, hi);
        A3B_CHECK_LAUNCH("random_f32 launch");
        return A3B_OK;
    }
}
