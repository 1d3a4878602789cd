/* CPU oracle: a plain-C restatement of the reference algorithms on the primitive path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product (alpaka3_b200/, include/) links, loads or calls this file; it
 * exists so that tests/, the smoke check and bench.py's CPU-baseline leg can check the CUDA kernels against the
 * reference's semantics on identical inputs. The restatement is pinned against the reference itself: the same
 * functions are cross-checked against oracle/_ref/libalpaka_ref.so (alpaka3's own host backend compiled from the
 * reference headers, see ref_harness.cpp) and against the committed golden vectors under tests/golden/.
 *
 * Built with -ffp-contract=off: every floating-point operation is rounded on its own, in source order, exactly
 * like the explicitly rounded (_rn) device code and the reference harness built with the same flag.
 *
 * Reference algorithms restated here (paths inside the alpaka3 project):
 *   babelstream ops      benchmark/babelstream/src/babelStreamMainTest.cpp:78-141, constants babelStreamCommon.hpp:31,45-48
 *   reduce/transformReduce  include/alpaka/onHost/algo/internal/transformReduce.hpp:23-130 (result semantics only:
 *                        out[0] = reduce(neutral, transform(in...)) over all elements; integer + wraps like the
 *                        reference's device atomicAdd)
 *   scan                 include/alpaka/onHost/algo/internal/scan.hpp:114-354 (exclusive identity T{0}; the unit test
 *                        ground truth is std::exclusive_scan / std::inclusive_scan, test/unit/algorithm/scan.cpp:40-48)
 *   heat stencil         example/heatEquation2D/src/StencilKernel.hpp:71-83, grid convention heatEquation2D.cpp:97-104
 *   nBody                example/nBody/src/Kernels.hpp:90-121 (velocity kick), :126-142 (drift)
 *   Philox4x32-10        Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC'11
 *                        (the same published generator as include/alpaka/rand/engine/philox/)
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------------------------------ Philox4x32-10 */

static inline void philox_round(uint32_t c[4], uint32_t const k[2])
{
    uint64_t const p0 = (uint64_t)0xD2511F53u * c[0];
    uint64_t const p1 = (uint64_t)0xCD9E8D57u * c[2];
    uint32_t const hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    uint32_t const hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    uint32_t const n0 = hi1 ^ c[1] ^ k[0];
    uint32_t const n2 = hi0 ^ c[3] ^ k[1];
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
}

/* counter = (i_lo, i_hi, 0, 0), key = (seed_lo, seed_hi); ten rounds with the Weyl key schedule */
void orc_philox(uint64_t seed, uint64_t i, uint32_t out[4])
{
    uint32_t c[4] = {(uint32_t)i, (uint32_t)(i >> 32), 0u, 0u};
    uint32_t k[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    for(int r = 0; r < 10; ++r)
    {
        philox_round(c, k);
        k[0] += 0x9E3779B9u;
        k[1] += 0xBB67AE85u;
    }
    memcpy(out, c, sizeof(c));
}

/* u32 stream: word 0 of the block for counter i, shifted right by `shift` (shift 28 gives [0,16)) */
void orc_gen_u32(uint64_t seed, uint64_t start, uint64_t n, int shift, uint32_t* out)
{
#pragma omp parallel for schedule(static)
    for(int64_t j = 0; j < (int64_t)n; ++j)
    {
        uint32_t r[4];
        orc_philox(seed, start + (uint64_t)j, r);
        out[j] = r[0] >> shift;
    }
}

/* u64 stream: (word1 << 32) | word0 */
void orc_gen_u64(uint64_t seed, uint64_t start, uint64_t n, uint64_t* out)
{
#pragma omp parallel for schedule(static)
    for(int64_t j = 0; j < (int64_t)n; ++j)
    {
        uint32_t r[4];
        orc_philox(seed, start + (uint64_t)j, r);
        out[j] = ((uint64_t)r[1] << 32) | r[0];
    }
}

/* fp32 uniform [lo, hi): lo + (hi - lo) * ((word0 >> 8) * 2^-24), each operation rounded on its own */
void orc_gen_f32(uint64_t seed, uint64_t start, uint64_t n, float lo, float hi, float* out)
{
    float const w = hi - lo;
#pragma omp parallel for schedule(static)
    for(int64_t j = 0; j < (int64_t)n; ++j)
    {
        uint32_t r[4];
        orc_philox(seed, start + (uint64_t)j, r);
        float const u = (float)(r[0] >> 8) * 0x1p-24f;
        float const t = w * u;
        out[j] = lo + t;
    }
}

/* ------------------------------------------------------------------------------------------------ BabelStream */

enum
{
    ORC_INIT = 0,
    ORC_COPY = 1,
    ORC_MUL = 2,
    ORC_ADD = 3,
    ORC_TRIAD = 4,
    ORC_NSTREAM = 5
};

#define ORC_STREAM(T, NAME)                                                                                           \
    void NAME(int kind, T* a, T* b, T* c, uint64_t n, T scalar, T ia, T ib, T ic)                                     \
    {                                                                                                                 \
        _Pragma("omp parallel for schedule(static)") for(int64_t i = 0; i < (int64_t)n; ++i)                          \
        {                                                                                                             \
            switch(kind)                                                                                              \
            {                                                                                                         \
            case ORC_INIT:                                                                                            \
                a[i] = ia;                                                                                            \
                b[i] = ib;                                                                                            \
                c[i] = ic;                                                                                            \
                break;                                                                                                \
            case ORC_COPY:                                                                                            \
                c[i] = a[i];                                                                                          \
                break;                                                                                                \
            case ORC_MUL:                                                                                             \
                b[i] = scalar * c[i];                                                                                 \
                break;                                                                                                \
            case ORC_ADD:                                                                                             \
                c[i] = a[i] + b[i];                                                                                   \
                break;                                                                                                \
            case ORC_TRIAD:                                                                                           \
                a[i] = b[i] + scalar * c[i];                                                                          \
                break;                                                                                                \
            case ORC_NSTREAM:                                                                                         \
                a[i] = a[i] + b[i] + scalar * c[i];                                                                   \
                break;                                                                                                \
            }                                                                                                         \
        }                                                                                                             \
    }

ORC_STREAM(double, orc_stream_f64)
ORC_STREAM(float, orc_stream_f32)

/* --------------------------------------------------------------------------------------- reductions (checkers) */

/* Neumaier-compensated fp64 sum, split over threads in fixed static chunks and combined in chunk order. */
#define ORC_COMP_SUM(NAME, ARGS, TERM)                                                                                \
    double NAME ARGS                                                                                                  \
    {                                                                                                                 \
        int nt = 1;                                                                                                   \
        double part[256];                                                                                             \
        double comp[256];                                                                                             \
        _Pragma("omp parallel") {                                                                                     \
            int t = 0;                                                                                                \
            int T = 1;                                                                                                \
            ORC_OMP_IDS(t, T);                                                                                        \
            if(T > 256)                                                                                               \
                T = 256;                                                                                              \
            if(t < T)                                                                                                 \
            {                                                                                                         \
                if(t == 0)                                                                                            \
                    nt = T;                                                                                           \
                uint64_t const b = n * (uint64_t)t / (uint64_t)T;                                                     \
                uint64_t const e = n * (uint64_t)(t + 1) / (uint64_t)T;                                               \
                double s = 0.0, cc = 0.0;                                                                             \
                for(uint64_t i = b; i < e; ++i)                                                                       \
                {                                                                                                     \
                    double const v = (TERM);                                                                          \
                    double const u = s + v;                                                                           \
                    if(fabs(s) >= fabs(v))                                                                            \
                        cc += (s - u) + v;                                                                            \
                    else                                                                                              \
                        cc += (v - u) + s;                                                                            \
                    s = u;                                                                                            \
                }                                                                                                     \
                part[t] = s;                                                                                          \
                comp[t] = cc;                                                                                         \
            }                                                                                                         \
        }                                                                                                             \
        double s = 0.0, cc = 0.0;                                                                                     \
        for(int t = 0; t < nt; ++t)                                                                                   \
        {                                                                                                             \
            double const v = part[t];                                                                                 \
            double const u = s + v;                                                                                   \
            if(fabs(s) >= fabs(v))                                                                                    \
                cc += (s - u) + v;                                                                                    \
            else                                                                                                      \
                cc += (v - u) + s;                                                                                    \
            s = u;                                                                                                    \
            cc += comp[t];                                                                                            \
        }                                                                                                             \
        return s + cc;                                                                                                \
    }

#ifdef _OPENMP
#define ORC_OMP_IDS(t, T)                                                                                             \
    do                                                                                                                \
    {                                                                                                                 \
        t = omp_get_thread_num();                                                                                     \
        T = omp_get_num_threads();                                                                                    \
    } while(0)
#else
#define ORC_OMP_IDS(t, T)                                                                                             \
    do                                                                                                                \
    {                                                                                                                 \
    } while(0)
#endif

ORC_COMP_SUM(orc_sumsq_f32, (float const* x, uint64_t n), (double)x[i] * (double)x[i])
ORC_COMP_SUM(orc_sumsq_f64, (double const* x, uint64_t n), x[i] * x[i])
ORC_COMP_SUM(orc_sum_f32, (float const* x, uint64_t n), (double)x[i])
ORC_COMP_SUM(orc_sum_f64, (double const* x, uint64_t n), x[i])
ORC_COMP_SUM(orc_dot_f64, (double const* x, double const* y, uint64_t n), x[i] * y[i])
ORC_COMP_SUM(orc_dot_f32, (float const* x, float const* y, uint64_t n), (double)x[i] * (double)y[i])

/* integer reductions: op 0 plus (two's-complement wrap), 1 min, 2 max */
#define ORC_IREDUCE(T, U, NAME)                                                                                       \
    T NAME(int op, T const* x, uint64_t n, T neutral)                                                                 \
    {                                                                                                                 \
        U acc = (U)neutral;                                                                                           \
        T best = neutral;                                                                                             \
        for(uint64_t i = 0; i < n; ++i)                                                                               \
        {                                                                                                             \
            if(op == 0)                                                                                               \
                acc = (U)(acc + (U)x[i]);                                                                             \
            else if(op == 1)                                                                                          \
                best = x[i] < best ? x[i] : best;                                                                     \
            else                                                                                                      \
                best = x[i] > best ? x[i] : best;                                                                     \
        }                                                                                                             \
        return op == 0 ? (T)acc : best;                                                                               \
    }

ORC_IREDUCE(int32_t, uint32_t, orc_reduce_i32)
ORC_IREDUCE(uint32_t, uint32_t, orc_reduce_u32)
ORC_IREDUCE(int64_t, uint64_t, orc_reduce_i64)
ORC_IREDUCE(uint64_t, uint64_t, orc_reduce_u64)

/* ------------------------------------------------------------------------------------------------------- scans */

/* exclusive: out[0] = 0, out[i] = out[i-1] + in[i-1]; inclusive: out[i] = out[i-1] + in[i]; unsigned wrap.
 * In-place (out == in) is supported, as the reference's *ScanInPlace entry points require. */
#define ORC_SCAN(T, NAME)                                                                                             \
    void NAME(int inclusive, T const* in, T* out, uint64_t n)                                                         \
    {                                                                                                                 \
        T run = (T)0;                                                                                                 \
        for(uint64_t i = 0; i < n; ++i)                                                                               \
        {                                                                                                             \
            T const v = in[i];                                                                                        \
            if(inclusive)                                                                                             \
            {                                                                                                         \
                run = (T)(run + v);                                                                                   \
                out[i] = run;                                                                                         \
            }                                                                                                         \
            else                                                                                                      \
            {                                                                                                         \
                out[i] = run;                                                                                         \
                run = (T)(run + v);                                                                                   \
            }                                                                                                         \
        }                                                                                                             \
    }

ORC_SCAN(uint32_t, orc_scan_u32)
ORC_SCAN(uint64_t, orc_scan_u64)
ORC_SCAN(float, orc_scan_f32)
ORC_SCAN(double, orc_scan_f64)

/* ------------------------------------------------------------------------------------------------ heat stencil */

/* u0 on the (n+2)x(n+2) grid, row-major, x fastest: x = j*dx, y = i*dy; interior sin(pi x) sin(pi y); ring = 0 */
void orc_heat_init(double* u, uint32_t n, double dx, double dy)
{
    uint64_t const w = (uint64_t)n + 2u;
    double const pi = 3.14159265358979323846;
#pragma omp parallel for schedule(static)
    for(int64_t i = 0; i < (int64_t)w; ++i)
        for(uint64_t j = 0; j < w; ++j)
        {
            double v = 0.0;
            if(i > 0 && (uint64_t)i < w - 1u && j > 0 && j < w - 1u)
                v = sin(pi * ((double)j * dx)) * sin(pi * ((double)i * dy));
            u[(uint64_t)i * w + j] = v;
        }
}

/* One Jacobi step over interior cells, evaluated in the reference's source order (StencilKernel.hpp:81-82):
 * c*(1 - 2rX - 2rY) + w*rX + e*rX + n*rY + s*rY, left to right, with the ring left untouched. */
void orc_heat_step(double const* cur, double* next, uint32_t n, double rX, double rY)
{
    uint64_t const w = (uint64_t)n + 2u;
    double const k = 1.0 - 2.0 * rX - 2.0 * rY;
#pragma omp parallel for schedule(static)
    for(int64_t i = 1; i <= (int64_t)n; ++i)
        for(uint64_t j = 1; j <= n; ++j)
        {
            uint64_t const p = (uint64_t)i * w + j;
            next[p] = cur[p] * k + cur[p - 1] * rX + cur[p + 1] * rX + cur[p - w] * rY + cur[p + w] * rY;
        }
}

/* ------------------------------------------------------------------------------------------------------ nBody */

/* One step: velocity kick over all j in index order (Kernels.hpp:90-121), then the drift (Kernels.hpp:126-142).
 * Per pair: d = p_j - p_i; r2 = (dx*dx + (dy*dy + dz*dz)) + eps (the Simd<3> tree sum); r6 = r2*r2*r2;
 * inv = 1/sqrt(r6); s = m_j*inv; a += s*d. Then v += a*dt, x += v*dt.
 * The i-bodies are taken 16 at a time so the compiler can vectorise across them; every body still accumulates its
 * pairs one j after the other in index order, so each result is the same as a scalar loop over j. */
#define ORC_NB_IB 16
void orc_nbody_step(
    float const* m,
    float* x,
    float* y,
    float* z,
    float* vx,
    float* vy,
    float* vz,
    uint64_t n,
    float dt,
    float eps)
{
#pragma omp parallel for schedule(dynamic, 4)
    for(int64_t i0 = 0; i0 < (int64_t)n; i0 += ORC_NB_IB)
    {
        int const cnt = (int64_t)n - i0 < ORC_NB_IB ? (int)((int64_t)n - i0) : ORC_NB_IB;
        float xi[ORC_NB_IB], yi[ORC_NB_IB], zi[ORC_NB_IB], ax[ORC_NB_IB], ay[ORC_NB_IB], az[ORC_NB_IB];
        for(int k = 0; k < ORC_NB_IB; ++k)
        {
            int64_t const i = i0 + (k < cnt ? k : 0);
            xi[k] = x[i];
            yi[k] = y[i];
            zi[k] = z[i];
            ax[k] = ay[k] = az[k] = 0.f;
        }
        for(uint64_t j = 0; j < n; ++j)
        {
            float const xj = x[j], yj = y[j], zj = z[j], mj = m[j];
            for(int k = 0; k < ORC_NB_IB; ++k)
            {
                float const dx = xj - xi[k];
                float const dy = yj - yi[k];
                float const dz = zj - zi[k];
                float const r2 = (dx * dx + (dy * dy + dz * dz)) + eps;
                float const r6 = r2 * r2 * r2;
                float const inv = 1.0f / sqrtf(r6);
                float const s = mj * inv;
                ax[k] += s * dx;
                ay[k] += s * dy;
                az[k] += s * dz;
            }
        }
        for(int k = 0; k < cnt; ++k)
        {
            vx[i0 + k] += ax[k] * dt;
            vy[i0 + k] += ay[k] * dt;
            vz[i0 + k] += az[k] * dt;
        }
    }
#pragma omp parallel for schedule(static)
    for(int64_t i = 0; i < (int64_t)n; ++i)
    {
        x[i] = x[i] + vx[i] * dt;
        y[i] = y[i] + vy[i] * dt;
        z[i] = z[i] + vz[i] * dt;
    }
}

/* fp64 accelerations of the sampled bodies idx[0..k) (all-pairs sum in double; a size-independent check) */
void orc_nbody_accel_sample(
    float const* m,
    float const* x,
    float const* y,
    float const* z,
    uint64_t n,
    float eps,
    int64_t const* idx,
    uint64_t k,
    double* acc3)
{
#pragma omp parallel for schedule(dynamic, 4)
    for(int64_t q = 0; q < (int64_t)k; ++q)
    {
        int64_t const i = idx[q];
        double ax = 0.0, ay = 0.0, az = 0.0;
        for(uint64_t j = 0; j < n; ++j)
        {
            double const dx = (double)x[j] - (double)x[i];
            double const dy = (double)y[j] - (double)y[i];
            double const dz = (double)z[j] - (double)z[i];
            double const r2 = dx * dx + dy * dy + dz * dz + (double)eps;
            double const inv = 1.0 / sqrt(r2 * r2 * r2);
            ax += (double)m[j] * inv * dx;
            ay += (double)m[j] * inv * dy;
            az += (double)m[j] * inv * dz;
        }
        acc3[3 * q + 0] = ax;
        acc3[3 * q + 1] = ay;
        acc3[3 * q + 2] = az;
    }
}

/* ----------------------------------------------------------------------------------------------------- HACCmk */

/* The benchmark's input (benchmark/HACCmk/src/main_alpaka.cpp:254-272): positions advanced by fixed steps in fp32
 * one particle after the other, masses i * 0.01 + x_i. */
void orc_haccmk_init(int n2, float* xx, float* yy, float* zz, float* mass)
{
    float const dx1 = 1.0f / (float)n2, dy1 = 2.0f / (float)n2, dz1 = 3.0f / (float)n2;
    xx[0] = 0.f;
    yy[0] = 0.f;
    zz[0] = 0.f;
    mass[0] = 2.f;
    for(int i = 1; i < n2; ++i)
    {
        xx[i] = xx[i - 1] + dx1;
        yy[i] = yy[i - 1] + dy1;
        zz[i] = zz[i - 1] + dz1;
        mass[i] = (float)i * 0.01f + xx[i];
    }
}

/* Short-range force of the first n1 particles against all n2, each target's pairs summed in source order, as the
 * reference's CPU gold (helper.hpp:19-66) computes it; v = fcoeff * sum (main_alpaka.cpp:288-293). */
void orc_haccmk_step10(int n1, int n2, float const* xx, float const* yy, float const* zz, float const* mass,
                       float fsrrmax2, float mp_rsm2, float fcoeff, float* vx, float* vy, float* vz)
{
    float const ma0 = 0.269327f, ma1 = -0.0750978f, ma2 = 0.0114808f, ma3 = -0.00109313f, ma4 = 0.0000605491f,
                ma5 = -0.00000147177f;
#pragma omp parallel for schedule(static)
    for(int i = 0; i < n1; ++i)
    {
        float sx = 0.f, sy = 0.f, sz = 0.f;
        for(int j = 0; j < n2; ++j)
        {
            float const dxc = xx[j] - xx[i];
            float const dyc = yy[j] - yy[i];
            float const dzc = zz[j] - zz[i];
            float const r2 = dxc * dxc + dyc * dyc + dzc * dzc;
            float const m = r2 < fsrrmax2 ? mass[j] : 0.f;
            float f = r2 + mp_rsm2;
            f = m * (1.f / (f * sqrtf(f)) - (ma0 + r2 * (ma1 + r2 * (ma2 + r2 * (ma3 + r2 * (ma4 + r2 * ma5))))));
            sx = sx + f * dxc;
            sy = sy + f * dyc;
            sz = sz + f * dzc;
        }
        vx[i] = 0.f + sx * fcoeff;
        vy[i] = 0.f + sy * fcoeff;
        vz[i] = 0.f + sz * fcoeff;
    }
}

int orc_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
