/* Element-wise engine for arbitrary device functors on B200 (header-only CUDA, sm_100a).
 *
 * A user functor cannot cross a C ABI, so this part of the library is a kernel template that nvcc compiles in the
 * caller's translation unit. It replaces alpaka3's SimdTransformKernel (include/alpaka/onHost/algo/internal/
 * transform.hpp:21-107) on top of SimdAlgo::concurrent (include/alpaka/onAcc/internal/SimdConcurrent.hpp:122-234)
 * for out[i] = fn(in0[i], in1[i], ...) over arrays laid out as rows of `rowLen` elements, each array with its own row
 * pitch (rows == 1: a dense 1-D array of any original dimensionality).
 *
 * Design (the one measured for the library's own element-wise kernels, alpaka3_b200/csrc/stream.cu): the rows are cut
 * into chunks of 512 threads x P packs x W elements and block b handles chunk b, so the block scheduler sweeps memory
 * front to back with a full grid of short-lived blocks. W = 16 bytes / the largest element size of the operation, so
 * the widest array moves one 16-byte access per pack; P = 2 for operations on two arrays, 1 for more. The functor is
 * called once per pack through an `Op` adapter:
 *
 *     struct Op {
 *         template<int V> __device__ void apply(Vec<TOut, V>& out, Vec<TIn, V> const&... in) const;
 *     };
 *
 * V is W for whole packs and 1 for the elements of a row's ragged end. ScalarOp (below) calls a scalar functor lane by
 * lane; the alpaka3 binding adds an adapter that passes alpaka::Simd packs, as alpaka3 does.
 */
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

namespace alpaka3_b200::elementwise
{
    constexpr int kThreads = 512;
    constexpr std::uint64_t kMaxGrid = (std::uint64_t{1} << 31) - 1u;

    //! V consecutive elements, aligned for one vector access (V * sizeof(T) is a power of two up to 16 bytes).
    template<typename T, int V>
    struct alignas(V * sizeof(T) <= 16 ? V * sizeof(T) : 16) Vec
    {
        T v[V];
    };

    //! One array of the operation: its first row and the distance between rows in bytes.
    template<typename T>
    struct Rows
    {
        T* ptr;
        std::uint64_t pitch;
    };

    template<typename T>
    __device__ __forceinline__ T* rowOf(Rows<T> const& a, std::uint64_t row)
    {
        using B = std::conditional_t<std::is_const_v<T>, unsigned char const, unsigned char>;
        return reinterpret_cast<T*>(reinterpret_cast<B*>(a.ptr) + row * a.pitch);
    }

    //! Calls a scalar functor lane by lane and converts its result to the output type.
    template<typename Fn, typename TOut, typename... TIn>
    struct ScalarOp
    {
        Fn fn;

        template<int V>
        __device__ __forceinline__ void apply(Vec<TOut, V>& out, Vec<TIn, V> const&... in) const
        {
#pragma unroll
            for(int k = 0; k < V; ++k)
                out.v[k] = static_cast<TOut>(fn(in.v[k]...));
        }
    };

    template<int W, int P, typename Op, typename TOut, typename... TIn>
    __global__ void __launch_bounds__(kThreads) elementwiseKernel(
        Rows<TOut> out,
        std::uint64_t rowLen,
        std::uint64_t chunksPerRow,
        Op op,
        Rows<TIn const>... in)
    {
        constexpr std::uint64_t kChunk = std::uint64_t{kThreads} * P * W;
        std::uint64_t const chunk = blockIdx.x;
        std::uint64_t const row = chunk / chunksPerRow;
        std::uint64_t const col0 = (chunk - row * chunksPerRow) * kChunk;
        TOut* const o = rowOf(out, row);
#pragma unroll
        for(int p = 0; p < P; ++p)
        {
            std::uint64_t const c = col0 + (static_cast<std::uint64_t>(p) * kThreads + threadIdx.x) * W;
            if(c + W <= rowLen)
            {
                Vec<TOut, W> r;
                op.template apply<W>(r, *reinterpret_cast<Vec<TIn, W> const*>(rowOf(in, row) + c)...);
                *reinterpret_cast<Vec<TOut, W>*>(o + c) = r;
            }
            else
            {
                for(std::uint64_t e = c; e < rowLen && e < c + W; ++e)
                {
                    Vec<TOut, 1> r;
                    op.template apply<1>(r, *reinterpret_cast<Vec<TIn, 1> const*>(rowOf(in, row) + e)...);
                    o[e] = r.v[0];
                }
            }
        }
    }

    //! Widest pack width the operation's element types allow: 16 bytes of its largest type.
    template<typename TOut, typename... TIn>
    constexpr int packWidth()
    {
        std::size_t m = sizeof(TOut);
        ((m = sizeof(TIn) > m ? sizeof(TIn) : m), ...);
        return m >= 16 ? 1 : static_cast<int>(16 / m);
    }

    //! true when a row start of `a` is aligned for packs of `w` elements
    template<typename T>
    bool packAligned(Rows<T> const& a, std::uint64_t rows, int w)
    {
        std::uint64_t const bytes = static_cast<std::uint64_t>(w) * sizeof(T);
        return reinterpret_cast<std::uintptr_t>(a.ptr) % bytes == 0u && (rows <= 1u || a.pitch % bytes == 0u);
    }

    template<int W, typename Op, typename TOut, typename... TIn>
    cudaError_t launchWidth(
        cudaStream_t stream,
        Rows<TOut> out,
        std::uint64_t rows,
        std::uint64_t rowLen,
        Op const& op,
        Rows<TIn const>... in)
    {
        constexpr int P = sizeof...(TIn) <= 1 ? 2 : 1;
        constexpr std::uint64_t kChunk = std::uint64_t{kThreads} * P * W;
        std::uint64_t const chunksPerRow = (rowLen + kChunk - 1u) / kChunk;
        std::uint64_t const grid = rows * chunksPerRow;
        if(grid == 0u)
            return cudaSuccess;
        if(grid > kMaxGrid)
            return cudaErrorInvalidValue;
        elementwiseKernel<W, P, Op, TOut, TIn...>
            <<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(out, rowLen, chunksPerRow, op, in...);
        return cudaGetLastError();
    }

    /** out[r][c] = op(in...[r][c]) for rows x rowLen elements; asynchronous on `stream`.
     *
     * Uses packs of packWidth<TOut, TIn...>() elements when every row start is aligned for them, single elements
     * otherwise. Returns cudaErrorInvalidValue when the grid would exceed 2^31 - 1 chunks. */
    template<typename Op, typename TOut, typename... TIn>
    cudaError_t launch(
        cudaStream_t stream,
        Rows<TOut> out,
        std::uint64_t rows,
        std::uint64_t rowLen,
        Op const& op,
        Rows<TIn const>... in)
    {
        constexpr int W = packWidth<TOut, TIn...>();
        if constexpr(W > 1)
        {
            if(packAligned(out, rows, W) && (packAligned(in, rows, W) && ...))
                return launchWidth<W>(stream, out, rows, rowLen, op, in...);
        }
        return launchWidth<1>(stream, out, rows, rowLen, op, in...);
    }

    //! out[i] = fn(in0[i], ...) for i < n over dense arrays, with a functor taking scalars.
    template<typename Fn, typename TOut, typename... TIn>
    cudaError_t transform(cudaStream_t stream, TOut* out, std::uint64_t n, Fn const& fn, TIn const*... in)
    {
        return launch(
            stream,
            Rows<TOut>{out, 0u},
            std::uint64_t{1},
            n,
            ScalarOp<Fn, TOut, TIn...>{fn},
            Rows<TIn const>{in, 0u}...);
    }
} // namespace alpaka3_b200::elementwise
