/* alpaka3_b200 -- C ABI of the B200 (sm_100a) data-parallel primitive library.
 *
 * Plain pointers and sizes only: every device pointer is a CUDA device (or managed) address on the device that is
 * current on the calling thread, every stream is a cudaStream_t passed as void*, and every entry point returns an
 * int status (A3B_OK == 0). On failure a3b_last_error() returns a message for the calling thread. All entry points
 * are asynchronous with respect to the host unless stated otherwise; results are visible after the stream is
 * synchronised.
 *
 * Each entry point names the alpaka3 interface whose backend dispatch it replaces (paths inside the alpaka3 project).
 */
#ifndef ALPAKA3_B200_H
#define ALPAKA3_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define A3B_VERSION 100

#if defined(__GNUC__)
#define A3B_API __attribute__((visibility("default")))
#else
#define A3B_API
#endif

typedef void* a3b_stream_t; /* cudaStream_t */

enum a3b_status
{
    A3B_OK = 0,
    A3B_ERR_INVALID = 1,     /* bad argument (null pointer, unsupported dtype/op combination, bad size) */
    A3B_ERR_CUDA = 2,        /* a CUDA runtime call failed; message has the CUDA error string */
    A3B_ERR_UNSUPPORTED = 3, /* no device / wrong architecture */
    A3B_ERR_TIMEOUT = 4,     /* a bounded device-side wait gave up (reported by a3b_get_device_error) */
    A3B_ERR_NOMEM = 5,
    A3B_ERR_TOO_LARGE = 6
};

enum a3b_dtype
{
    A3B_I32 = 0,
    A3B_U32 = 1,
    A3B_I64 = 2,
    A3B_U64 = 3,
    A3B_F32 = 4,
    A3B_F64 = 5
};

/* binary reduce functors: std::plus, ScalarFunc{min}, ScalarFunc{max} (test/unit/algorithm/reduce.cpp:22-56) */
enum a3b_reduce_op
{
    A3B_REDUCE_PLUS = 0,
    A3B_REDUCE_MIN = 1,
    A3B_REDUCE_MAX = 2
};

/* transform functors recognised on the C path: identity (onHost::reduce), x*x, a*b (BabelStream DotMultiplication) */
enum a3b_transform_op
{
    A3B_XFORM_IDENTITY = 0,
    A3B_XFORM_SQUARE = 1,
    A3B_XFORM_PRODUCT = 2
};

/* BabelStream element-wise kernels (benchmark/babelstream/src/babelStreamMainTest.cpp:78-133) */
enum a3b_stream_kind
{
    A3B_STREAM_INIT = 0,   /* a = init[0], b = init[1], c = init[2] */
    A3B_STREAM_COPY = 1,   /* c = a */
    A3B_STREAM_MUL = 2,    /* b = scalar * c */
    A3B_STREAM_ADD = 3,    /* c = a + b */
    A3B_STREAM_TRIAD = 4,  /* a = b + scalar * c */
    A3B_STREAM_NSTREAM = 5 /* a = a + b + scalar * c */
};

/* element-wise transforms for onHost::transform / onHost::concurrent with recognised functors */
enum a3b_map_kind
{
    A3B_MAP_COPY = 0,  /* out = in0 */
    A3B_MAP_SCALE = 1, /* out = alpha * in0 */
    A3B_MAP_ADD = 2,   /* out = in0 + in1 */
    A3B_MAP_MUL = 3,   /* out = in0 * in1 */
    A3B_MAP_AXPY = 4,  /* out = in0 + alpha * in1 (each operation rounded on its own) */
    A3B_MAP_SQUARE = 5 /* out = in0 * in0 */
};

typedef struct a3b_device_info
{
    int ordinal;
    int sm_count;
    int cc_major;
    int cc_minor;
    uint64_t global_mem_bytes;
    uint64_t l2_bytes;
    int max_threads_per_block;
    int warp_size;
    char name[128];
} a3b_device_info;

/* ------------------------------------------------------------------------------------------------- runtime */

A3B_API int a3b_version(void);
A3B_API const char* a3b_last_error(void);
/* onHost::DeviceSelector::getDeviceCount / getDeviceProperties (include/alpaka/onHost/DeviceProperties.hpp:28-56) */
A3B_API int a3b_device_count(int* count);
A3B_API int a3b_device_info_get(int ordinal, a3b_device_info* info);
/* onHost::alloc / allocDeferred: stream-ordered device allocation (include/alpaka/onHost/Queue.hpp:410) */
A3B_API int a3b_malloc_async(void** ptr, size_t bytes, a3b_stream_t stream);
A3B_API int a3b_free_async(void* ptr, a3b_stream_t stream);
/* onHost::memcpy (include/alpaka/onHost/Queue.hpp:237): any direction, one cudaMemcpyAsync */
A3B_API int a3b_memcpy_async(void* dst, void const* src, size_t bytes, a3b_stream_t stream);
/* onHost::wait(queue) (include/alpaka/onHost/interface.hpp:142) */
A3B_API int a3b_stream_synchronize(a3b_stream_t stream);
/* Device scratch for the kernels that the header-only engines (include/alpaka3_b200/simd_engine.cuh) instantiate in
 * the caller's translation unit: at least `bytes`, cached per (device, stream), zero-filled when first allocated or
 * grown. Work ordered on `stream` may use it; the engines leave it as they found it (their tickets are reset by the
 * kernel that drew the last number). No counterpart in alpaka3, whose reductions pre-fill the output instead. */
A3B_API int a3b_engine_scratch(a3b_stream_t stream, size_t bytes, void** ptr);
/* Reads (and with clear != 0 resets) the device-side error word of the current device: bit 0 = a bounded wait timed
 * out (A3B_ERR_TIMEOUT). Synchronises `stream`. */
A3B_API int a3b_get_device_error(a3b_stream_t stream, uint32_t* error_bits, int clear);
/* Limit in nanoseconds for every device-side spin-wait issued afterwards by this process (default 1 s). */
A3B_API int a3b_set_wait_timeout_ns(uint64_t ns);

/* ------------------------------------------------------------------------------- element-wise (transform) */

/* BabelStream kernels: queue.enqueue(FrameSpec, KernelBundle{SimdForEachKernel{}, Simd<Op>{}, a, b, c})
 * (benchmark/babelstream/src/babelStreamMainTest.cpp:285-364). dtype A3B_F32 or A3B_F64. init may be null unless
 * kind == A3B_STREAM_INIT. Every floating-point operation is rounded on its own (no contraction). */
A3B_API int a3b_babelstream(a3b_stream_t stream, int kind, int dtype, void* a, void* b, void* c, uint64_t n, double scalar,
                    double const* init);

/* onHost::transform(queue, out, fn, in0[, in1]) with a recognised fn (include/alpaka/onHost/algo/transform.hpp:50-88).
 * in1 is ignored for unary kinds. Integer dtypes wrap; alpha is converted to dtype first. */
A3B_API int a3b_transform(a3b_stream_t stream, int kind, int dtype, void* out, void const* in0, void const* in1, uint64_t n,
                  double alpha);

/* onHost::fill (include/alpaka/onHost/Queue.hpp:346): value points to one host element of dtype */
A3B_API int a3b_fill(a3b_stream_t stream, int dtype, void* out, uint64_t n, void const* value);

/* onHost::iota (include/alpaka/onHost/algo/iota.hpp:29-85): out[i] = start + i (host start value of dtype) */
A3B_API int a3b_iota(a3b_stream_t stream, int dtype, void* out, uint64_t n, void const* start);

/* nBody drift, onHost::concurrent(..., UpdatePositions{dt}, x, y, z, vx, vy, vz) (example/nBody/src/Kernels.hpp:126-142):
 * x = x + vx*dt per component, fp32 */
A3B_API int a3b_nbody_update_positions(a3b_stream_t stream, float* x, float* y, float* z, float const* vx, float const* vy,
                               float const* vz, uint64_t n, float dt);

/* Seeded Philox4x32-10 streams (counter = start + element index, key = seed), identical to the CPU oracle:
 *   u32: word0 >> shift;   u64: (word1 << 32) | word0;   f32: lo + (hi - lo) * ((word0 >> 8) * 2^-24). */
A3B_API int a3b_random_u32(a3b_stream_t stream, uint32_t* out, uint64_t n, uint64_t seed, uint64_t start, int shift);
A3B_API int a3b_random_u64(a3b_stream_t stream, uint64_t* out, uint64_t n, uint64_t seed, uint64_t start);
A3B_API int a3b_random_f32(a3b_stream_t stream, float* out, uint64_t n, uint64_t seed, uint64_t start, float lo, float hi);

/* ---------------------------------------------------------------------------------------------- reductions */

/* onHost::transformReduce(queue, neutral, out, reduceFn, transformFn, in0[, in1])
 * (include/alpaka/onHost/algo/transformReduce.hpp:59-90; kernel internal/transformReduce.hpp:23-202).
 * out: device pointer to ONE element of dtype, written with the final value (no pre-fill launch needed).
 * neutral: host pointer to one element of dtype. One launch; the final combination runs in the last block in a fixed
 * order, so a given (device, n) always gives the same bits. fp32 inputs are accumulated in fp64 inside the kernel;
 * integer + wraps (two's complement).
 * Ordering: by default the launch is fully ordered after all earlier work of the stream. With a3b_set_early_start
 * enabled on the stream it may start while the previous kernel of the stream still runs (see there). */
A3B_API int a3b_transform_reduce(a3b_stream_t stream, int dtype, int reduce_op, int transform_op, void const* in0,
                         void const* in1, uint64_t n, void const* neutral, void* out);

/* Same, but the per-block partials are left as fp64 (float dtypes) / 64-bit integers in partial_out[0] instead of
 * being rounded to dtype: used to combine shards across GPUs before the final rounding. Ordering as
 * a3b_transform_reduce. */
A3B_API int a3b_transform_reduce_partial(a3b_stream_t stream, int dtype, int reduce_op, int transform_op, void const* in0,
                                 void const* in1, uint64_t n, void const* neutral, void* partial_out);

/* No counterpart in the reference: a3b_transform_reduce for callers that cannot allocate device memory -- a process
 * whose device memory is owned by another allocator's pool, a service that must keep a fixed, accounted memory
 * footprint, a latency-critical loop that cannot afford an allocation's implicit synchronisation. Same arguments as
 * a3b_transform_reduce over a dense 1-D input; it allocates nothing. The result is the same for integer data; for
 * floating-point data it agrees within rounding (its grid is capped at 2024 blocks, so above that size the partials
 * are combined in another order) and is deterministic for a given n. Its scratch is one fixed 16 KB static device
 * array per GPU that loads the library (held until the process exits): the tickets and partials of at most 2024
 * blocks, each of which takes several chunks of a large input (A3B_ERR_TOO_LARGE is kept for a layout that would not
 * fit). The first call on a device (and the first after the device's context was re-created, e.g. by
 * cudaDeviceReset) looks up that array's device address, so make that call before any stream capture. All calls
 * share the array: calls that overlap on the GPU (different streams, devices' own streams in parallel) race and must
 * be serialised by the caller. Always launched fully ordered. */
A3B_API int a3b_transform_reduce_noalloc(a3b_stream_t stream, int dtype, int reduce_op, int transform_op,
                                         void const* in0, void const* in1, uint64_t n, void const* neutral, void* out);

/* Early start of the reductions on `stream` of the current device (a3b_transform_reduce, _partial, a3b_reduce_2d,
 * a3b_transform_reduce_allranks, a3b_reduce_lower_ranks); off by default. No counterpart in alpaka3, whose kernels
 * are plain launches. When enabled, a reduction is launched with programmatic dependent launch: it starts as soon as
 * the previous kernel of the stream lets its dependents launch, reads its input, and waits for that kernel to
 * complete only before it touches its scratch or `out`. The next call thus streams its input while this one combines
 * (and, across ranks, waits for its peers). The library launches fully ordered any call whose input overlaps the
 * output of one of its own reductions that may still run (every reduction started early since the last fully ordered
 * launch). ENABLE IT ONLY IF no other kernel on the stream executes griddepcontrol.launch_dependents
 * (cudaTriggerProgrammaticLaunchCompletion) before its output is written -- e.g. kernels built with programmatic
 * dependent launch by CUTLASS or some cuBLASLt kernels: the reduction could read that output before it is written.
 * Copies, memsets and kernels without that instruction are always complete before the reduction reads its input. */
A3B_API int a3b_set_early_start(a3b_stream_t stream, int enable);

/* onHost::reduce(queue, neutral, out, reduceFn, in) (include/alpaka/onHost/algo/reduce.hpp:28-79) over a pitched
 * 2-D view: `rows` rows of `row_len` elements, consecutive rows `row_pitch_bytes` apart (rows = 1 for 1-D data).
 * N-D alpaka buffers whose slower dimensions are dense multiples of the row pitch map onto this form. Ordering as
 * a3b_transform_reduce. */
A3B_API int a3b_reduce_2d(a3b_stream_t stream, int dtype, int reduce_op, void const* in, uint64_t rows, uint64_t row_len,
                  uint64_t row_pitch_bytes, void const* neutral, void* out);

/* --------------------------------------------------------------------------------------- multi-GPU (one node) */

/* A peer group connects the ranks of one node (one process per GPU) through a small slot buffer per rank that every
 * other rank maps over NVLink (CUDA IPC). Protocol: each rank calls a3b_peer_group_create on its device, exchanges
 * the a3b_ipc_handle_size() bytes written to `local_handle` with all ranks (any host channel), then calls
 * a3b_peer_group_connect with the world handles in rank order. No counterpart in alpaka3, which has no multi-device
 * layer. */
typedef struct a3b_peer_group a3b_peer_group;
A3B_API size_t a3b_ipc_handle_size(void);
A3B_API int a3b_peer_group_create(int world, int rank, a3b_peer_group** group, void* local_handle);
A3B_API int a3b_peer_group_connect(a3b_peer_group* group, void const* handles);
A3B_API int a3b_peer_group_destroy(a3b_peer_group* group);

/* onHost::transformReduce over data sharded across the ranks of a peer group, fused with the all-reduce: one launch
 * per rank reduces the local shard, its last block stores the unrounded partial into every rank's slot (peer stores
 * over NVLink), waits (bounded) for all ranks' partials and combines them in rank order, so every rank writes the
 * same bits to its `out`. All ranks must make the same sequence of calls. A wait that runs out sets bit 0 of the
 * device error word (a3b_get_device_error). Ordering as a3b_transform_reduce: with a3b_set_early_start enabled on the
 * stream, consecutive calls overlap, so a call reads its input while the previous call still waits for the other
 * ranks. */
A3B_API int a3b_transform_reduce_allranks(a3b_stream_t stream, a3b_peer_group* group, int dtype, int reduce_op,
                                          int transform_op, void const* in0, void const* in1, uint64_t n,
                                          void const* neutral, void* out);

/* Carry of a scan split across the ranks of a peer group: sums this rank's shard in one launch, exchanges the shard
 * totals through the peer slots and writes sum(totals of ranks 0 .. rank-1) to carry_out (device pointer, one
 * element of dtype; integers wrap). Feed it to a3b_scan as carry_in. */
A3B_API int a3b_reduce_lower_ranks(a3b_stream_t stream, a3b_peer_group* group, int dtype, void const* in, uint64_t n,
                                   void* carry_out);

/* ------------------------------------------------------------------------------------------------------ scan */

/* onHost::getScanBufferSize<T>(extents) (include/alpaka/onHost/algo/scan.hpp:26-30): bytes of the caller buffer that
 * a3b_scan accepts for n elements of dtype. */
A3B_API size_t a3b_scan_buffer_size(int dtype, uint64_t n);

/* onHost::inclusiveScan / exclusiveScan / *InPlace (include/alpaka/onHost/algo/scan.hpp:45-218), operator +,
 * exclusive identity 0. One cooperative launch of one block per SM that reads every element from HBM once and writes
 * it once (tile aggregates published two rounds ahead of the tiles' scans). in == out is allowed (in-place).
 * buffer: optional caller scratch of at least a3b_scan_buffer_size bytes (any contents; it is cleared on the
 *         stream); null uses a scratch cached by the library per (device, stream).
 * carry_in: optional DEVICE pointer to one element added to every output (the sum of all preceding shards when a
 *         scan is split across GPUs); null means 0. Integer arithmetic wraps (two's complement). */
A3B_API int a3b_scan(a3b_stream_t stream, int dtype, int inclusive, void const* in, void* out, uint64_t n,
             void const* carry_in, void* buffer, size_t buffer_bytes);

/* ----------------------------------------------------------------------------------------------------- nBody */

/* UpdateVelocitiesKernel (example/nBody/src/Kernels.hpp:24-124) for the i-bodies [i_begin, i_begin + i_count) against
 * all n_all j-bodies: v_i += dt * sum_j m_j d_ij / ((|d_ij|^2 + eps)^3)^(1/2), d_ij = p_j - p_i.
 * m, x, y, z hold all n_all bodies; vx, vy, vz hold the i_count local velocities. fp32, SoA. */
A3B_API int a3b_nbody_update_velocities(a3b_stream_t stream, float const* m, float const* x, float const* y, float const* z,
                                uint64_t n_all, uint64_t i_begin, uint64_t i_count, float* vx, float* vy, float* vz,
                                float dt, float eps);

/* One full nBody time step for the local bodies (nBody.cpp:188-205): the velocity kick above for [i_begin,
 * i_begin + i_count), then the drift x += v*dt of those bodies' positions (x + i_begin ...), in one call. The positions
 * of all n_all bodies are read before any is moved (the drift runs after every force is known). */
A3B_API int a3b_nbody_step(a3b_stream_t stream, float const* m, float* x, float* y, float* z, uint64_t n_all,
                   uint64_t i_begin, uint64_t i_count, float* vx, float* vy, float* vz, float dt, float eps);

/* --------------------------------------------------------------------------------------------------- HACCmk */

/* HACCmk's short-range force step (benchmark/HACCmk/src/main_alpaka.cpp:47-123 Step10Kernel, CPU gold
 * helper.hpp:19-66): for the first n1 particles (targets) against all n2 particles (sources),
 *   d = p_j - p_i, r2 = |d|^2, m = (r2 < fsrrmax2) ? mass_j : 0, f = r2 + mp_rsm2,
 *   f = m * (1 / (f * sqrt f) - poly(r2)),  v_i = fcoeff * sum_j f * d   (written to vx2/vy2/vz2[i], i < n1).
 * fp32, SoA; 0 <= n1 <= n2. */
A3B_API int a3b_haccmk_step10(a3b_stream_t stream, float const* xx, float const* yy, float const* zz, float const* mass,
                              int n1, int n2, float fsrrmax2, float mp_rsm2, float fcoeff, float* vx2, float* vy2,
                              float* vz2);

/* ------------------------------------------------------------------------------------------------------ heat */

/* StencilKernel (example/heatEquation2D/src/StencilKernel.hpp:26-86): one explicit 5-point Jacobi step on a row-major
 * fp64 grid of (rows + 2) x (cols + 2) cells (1-cell halo ring), consecutive rows `pitch_elems` apart. Updates interior
 * rows [row_begin, row_end) (1 <= row_begin <= row_end <= rows + 1) and all interior columns:
 *   next = cur*(1 - 2rX - 2rY) + west*rX + east*rX + north*rY + south*rY   (left to right, each op rounded).
 * The halo ring of `next` is not written. */
A3B_API int a3b_heat_step(a3b_stream_t stream, double const* cur, double* next, uint64_t rows, uint64_t cols,
                  uint64_t pitch_elems, uint64_t row_begin, uint64_t row_end, double rX, double rY);

/* Initial field of the heat workload: interior sin(pi*j*dx)*sin(pi*(i + row_offset)*dy), ring set to 0 only at the
 * global boundary (row i of this slab is global row i + row_offset). grid as in a3b_heat_step, rows = local rows. */
A3B_API int a3b_heat_init(a3b_stream_t stream, double* u, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                  uint64_t row_offset, uint64_t global_rows, double dx, double dy);

/* The heatEquation2D example's own problem (example/heatEquation2D/src/analyticalSolution.hpp:17-78,
 * BoundaryKernel.hpp:23-57): writes the exact solution e^{-pi^2 t}(sin pi x + sin pi y), x = col*dx, y = row*dy, to
 * every cell (ring_only == 0, the initial field initalizeBuffer writes) or only to the cells on the global ring
 * (ring_only != 0, the time-dependent Dirichlet boundary applied after each step). Grid as in a3b_heat_step. */
A3B_API int a3b_heat_exact(a3b_stream_t stream, double* u, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                           uint64_t row_offset, uint64_t global_rows, double t, double dx, double dy, int ring_only);

/* Row slabs of the heat grid across the ranks of one node, halo exchange fused into the stencil step. alpaka3's
 * heatEquation2D example runs on one device (example/heatEquation2D/src/heatEquation2D.cpp:97-214); the row
 * decomposition with one ghost row per side is new here.
 *
 * Each rank owns a halo mailbox (a small cudaMalloc'd buffer: two ghost rows per side, double-buffered by step
 * parity, and one step flag per column block) that its upper and lower neighbours map through CUDA IPC. Create it
 * on every rank, exchange the a3b_ipc_handle_size()-byte handles (rank order), connect. */
typedef struct a3b_halo a3b_halo;
A3B_API size_t a3b_halo_bytes(uint64_t cols);
A3B_API int a3b_halo_create(int world, int rank, uint64_t cols, a3b_halo** halo, void* local_handle);
A3B_API int a3b_halo_connect(a3b_halo* halo, void const* handles);
/* Call only when no neighbour is still writing into this mailbox (after a barrier that follows the last step). */
A3B_API int a3b_halo_destroy(a3b_halo* halo);

/* Sends this rank's first and last interior rows of u (the initial field) to the neighbours' mailboxes; call once on
 * every rank after a3b_heat_init and before the first a3b_heat_step_halo. u: (rows + 2) x pitch_elems fp64, rows
 * 16-byte aligned (even pitch). */
A3B_API int a3b_heat_halo_publish(a3b_stream_t stream, a3b_halo* halo, double const* u, uint64_t rows, uint64_t cols,
                                  uint64_t pitch_elems);

/* One a3b_heat_step over the whole slab (rows 1..rows) in one launch, with the ghost rows taken from this rank's
 * mailbox (the neighbours' boundary rows of the previous step; a rank without an upper / lower neighbour uses its
 * own ghost row, the global Dirichlet ring) and its own boundary rows stored into the neighbours' mailboxes over
 * NVLink. The bands holding rows 1 and `rows` run first and wait, bounded by a3b_set_wait_timeout_ns, for the
 * neighbours' flags (a timeout raises bit 0 of the device error word); the other bands never wait. Every rank makes
 * the same sequence of publish / step calls. */
A3B_API int a3b_heat_step_halo(a3b_stream_t stream, a3b_halo* halo, double const* cur, double* next, uint64_t rows,
                               uint64_t cols, uint64_t pitch_elems, double rX, double rY);

#ifdef __cplusplus
}
#endif

#endif /* ALPAKA3_B200_H */
