/*
 * ORACLE — test infrastructure only. Never linked into, imported by, or called from the product path
 * (torchsoftdtw_b200). Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
 * may load it, and only as the checker or the timed CPU baseline.
 *
 * A plain-C restatement of the reference's CPU Soft-DTW operator (angelo-ortiz/torchsoftdtw):
 *   - band predicate ............ src/torchsoftdtw/csrc/band.h:23-38
 *   - forward (R wavefront) ..... src/torchsoftdtw/csrc/softdtw.cpp:97-173
 *   - backward (log-space E) .... src/torchsoftdtw/csrc/softdtw.cpp:176-285
 *   - logsumexp3 ................ src/torchsoftdtw/csrc/softdtw.cpp:87-92
 * The arithmetic follows the reference operation by operation (same divisions by gamma, same max shift,
 * same left-to-right sums, libm exp/log), so that on x86-64 without FMA contraction it reproduces the
 * reference's outputs bit for bit. Pinned against the compiled reference by tests/golden/.
 *
 * Layouts (all contiguous, row-major): D (B,N,M); R (B,N+2,M+2); E (B,N,M); lengths int64 (B,).
 * The batch loop is split over `nthreads` POSIX threads (the reference uses an intra-op parallel_for
 * over the batch, softdtw.cpp:134 and :215).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* band.h:23-38 — integer Sakoe-Chiba test on the scaled diagonal. */
int oracle_in_band(int64_t i, int64_t j, int64_t nx, int64_t ny, int64_t bandwidth)
{
    if (bandwidth < 0) return 1;
    const int x_short = nx <= ny;
    const int64_t K = x_short ? nx : ny;
    const int64_t L = x_short ? ny : nx;
    if (K <= 1) return 1;
    const int64_t k = x_short ? i : j;
    const int64_t l = x_short ? j : i;
    int64_t diff = l * (K - 1) - k * (L - 1);
    if (diff < 0) diff = -diff;
    const int64_t band = 2 * bandwidth * (K - 1);
    const int64_t width = band > L - 1 ? band : L - 1;
    return 2 * diff <= width;
}

/* Exact number of in-band cells with i < nx and j < ny (the DP cells the operator evaluates). */
int64_t oracle_count_cells(const int64_t* lx, const int64_t* ly, int64_t B, int64_t bandwidth)
{
    int64_t total = 0;
    for (int64_t b = 0; b < B; b++)
        for (int64_t i = 0; i < lx[b]; i++)
            for (int64_t j = 0; j < ly[b]; j++) total += oracle_in_band(i, j, lx[b], ly[b], bandwidth);
    return total;
}

typedef struct {
    const void* D;
    const void* R;
    void* out0;
    void* out1;
    int64_t B, N, M;
    const int64_t* lx;
    const int64_t* ly;
    double gamma;
    int64_t bandwidth;
    int64_t b_begin, b_end;
} job_t;

/* ---------------------------------------------------------------------------------------------------
 * The two kernels are written once as macros over the scalar type, so float and double follow the
 * same statement sequence (the reference instantiates one template for both, softdtw.cpp:124, :203).
 * ------------------------------------------------------------------------------------------------- */

#define DEFINE_FORWARD(T, SUF, EXPF, LOGF)                                                           \
    static void fwd_range_##SUF(const job_t* jb)                                                     \
    {                                                                                                 \
        const T* D = (const T*)jb->D;                                                                \
        T* R = (T*)jb->out0;                                                                         \
        T* costs = (T*)jb->out1;                                                                     \
        const int64_t N = jb->N, M = jb->M, RM = M + 2;                                              \
        const T gamma_val = (T)jb->gamma;                                                            \
        const T INF = (T)INFINITY;                                                                   \
        for (int64_t b = jb->b_begin; b < jb->b_end; b++) {                                          \
            const int64_t nx = jb->lx[b], ny = jb->ly[b];                                            \
            const T* Db = D + b * N * M;                                                             \
            T* Rb = R + b * (N + 2) * RM;                                                            \
            for (int64_t q = 0; q < (N + 2) * RM; q++) Rb[q] = INF;                                  \
            Rb[0] = (T)0;                                                                            \
            for (int64_t i = 0; i < nx; i++) {                                                       \
                for (int64_t j = 0; j < ny; j++) {                                                   \
                    if (!oracle_in_band(i, j, nx, ny, jb->bandwidth)) continue;                      \
                    const int64_t ri = i + 1, rj = j + 1;                                            \
                    T r0 = -Rb[(ri - 1) * RM + (rj - 1)] / gamma_val;                                \
                    T r1 = -Rb[(ri - 1) * RM + rj] / gamma_val;                                      \
                    T r2 = -Rb[ri * RM + (rj - 1)] / gamma_val;                                      \
                    T rmax = r0 > r1 ? r0 : r1;                                                      \
                    rmax = rmax > r2 ? rmax : r2;                                                    \
                    T softmin;                                                                       \
                    if (isinf(rmax) && rmax < 0) {                                                   \
                        softmin = INF;                                                               \
                    } else {                                                                         \
                        softmin = -gamma_val *                                                       \
                                  (LOGF(EXPF(r0 - rmax) + EXPF(r1 - rmax) + EXPF(r2 - rmax)) + rmax); \
                    }                                                                                \
                    Rb[ri * RM + rj] = Db[i * M + j] + softmin;                                      \
                }                                                                                    \
            }                                                                                        \
            costs[b] = Rb[nx * RM + ny];                                                             \
        }                                                                                             \
    }

#define DEFINE_BACKWARD(T, SUF, EXPF, LOGF)                                                          \
    static T logsumexp3_##SUF(T a, T b, T c)                                                         \
    {                                                                                                 \
        T m = a > b ? a : b;                                                                         \
        m = m > c ? m : c;                                                                           \
        if (isinf(m) && m < 0) return m;                                                             \
        return m + LOGF(EXPF(a - m) + EXPF(b - m) + EXPF(c - m));                                    \
    }                                                                                                 \
    static void bwd_range_##SUF(const job_t* jb)                                                     \
    {                                                                                                 \
        const T* D = (const T*)jb->D;                                                                \
        const T* R = (const T*)jb->R;                                                                \
        T* Eout = (T*)jb->out0;                                                                      \
        const int64_t N = jb->N, M = jb->M, RM = M + 2, RS = (N + 2) * (M + 2);                      \
        const T gamma_val = (T)jb->gamma;                                                            \
        const T INF = (T)INFINITY, NINF = -(T)INFINITY;                                              \
        T* Rbw = (T*)malloc(sizeof(T) * RS);                                                         \
        T* E = (T*)malloc(sizeof(T) * RS);                                                           \
        for (int64_t b = jb->b_begin; b < jb->b_end; b++) {                                          \
            const int64_t nx = jb->lx[b], ny = jb->ly[b];                                            \
            const T* Db = D + b * N * M;                                                             \
            const T* Rb = R + b * RS;                                                                \
            memcpy(Rbw, Rb, sizeof(T) * RS);                                                         \
            for (int64_t q = 0; q < RS; q++) E[q] = NINF;                                            \
            Rbw[(nx + 1) * RM + (ny + 1)] = Rb[nx * RM + ny];                                        \
            E[(nx + 1) * RM + (ny + 1)] = (T)0;                                                      \
            for (int64_t i = nx - 1; i >= 0; i--) {                                                  \
                for (int64_t j = ny - 1; j >= 0; j--) {                                              \
                    if (!oracle_in_band(i, j, nx, ny, jb->bandwidth)) continue;                      \
                    const int64_t ri = i + 1, rj = j + 1;                                            \
                    /* safe_R maps +inf to -inf; D_pad is 0 outside [1,nx]x[1,ny] (:229-238) */      \
                    T v;                                                                             \
                    v = Rbw[ri * RM + rj];                                                           \
                    const T R_ij = (v == INF) ? NINF : v;                                            \
                    v = Rbw[(ri + 1) * RM + rj];                                                     \
                    const T Ra = (v == INF) ? NINF : v;                                              \
                    v = Rbw[ri * RM + rj + 1];                                                       \
                    const T Rb_ = (v == INF) ? NINF : v;                                             \
                    v = Rbw[(ri + 1) * RM + rj + 1];                                                 \
                    const T Rc = (v == INF) ? NINF : v;                                              \
                    const T Da = (ri + 1 <= nx) ? Db[ri * M + (rj - 1)] : (T)0;                      \
                    const T Dbv = (rj + 1 <= ny) ? Db[(ri - 1) * M + rj] : (T)0;                     \
                    const T Dc = (ri + 1 <= nx && rj + 1 <= ny) ? Db[ri * M + rj] : (T)0;            \
                    const T la = (Ra - R_ij - Da) / gamma_val;                                       \
                    const T lb = (Rb_ - R_ij - Dbv) / gamma_val;                                     \
                    const T lc = (Rc - R_ij - Dc) / gamma_val;                                       \
                    const T t1 = E[(ri + 1) * RM + rj] + la;                                         \
                    const T t2 = E[ri * RM + rj + 1] + lb;                                           \
                    const T t3 = E[(ri + 1) * RM + rj + 1] + lc;                                     \
                    E[ri * RM + rj] = logsumexp3_##SUF(t1, t2, t3);                                  \
                }                                                                                    \
            }                                                                                        \
            /* E = exp(logE) on the valid box, 0 elsewhere; return E[1:N+1, 1:M+1] (:261-283) */     \
            T* Eb = Eout + b * N * M;                                                                \
            for (int64_t i = 1; i <= N; i++) {                                                       \
                for (int64_t j = 1; j <= M; j++) {                                                   \
                    Eb[(i - 1) * M + (j - 1)] = (i <= nx && j <= ny) ? EXPF(E[i * RM + j]) : (T)0;   \
                }                                                                                    \
            }                                                                                        \
        }                                                                                             \
        free(Rbw);                                                                                   \
        free(E);                                                                                     \
    }

DEFINE_FORWARD(double, f64, exp, log)
DEFINE_FORWARD(float, f32, expf, logf)
DEFINE_BACKWARD(double, f64, exp, log)
DEFINE_BACKWARD(float, f32, expf, logf)

typedef void (*range_fn)(const job_t*);

typedef struct {
    job_t job;
    range_fn fn;
} task_t;

static void* run_job(void* p)
{
    const task_t* t = (const task_t*)p;
    t->fn(&t->job);
    return NULL;
}

static void run_parallel(range_fn fn, const job_t* proto, int nthreads)
{
    const int64_t B = proto->B;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > B) nthreads = (int)(B > 0 ? B : 1);
    task_t* tasks = (task_t*)calloc((size_t)nthreads, sizeof(task_t));
    pthread_t* th = (pthread_t*)calloc((size_t)nthreads, sizeof(pthread_t));
    for (int t = 0; t < nthreads; t++) {
        tasks[t].job = *proto;
        tasks[t].job.b_begin = B * t / nthreads;
        tasks[t].job.b_end = B * (t + 1) / nthreads;
        tasks[t].fn = fn;
    }
    for (int t = 1; t < nthreads; t++) pthread_create(&th[t], NULL, run_job, &tasks[t]);
    run_job(&tasks[0]);
    for (int t = 1; t < nthreads; t++) pthread_join(th[t], NULL);
    free(th);
    free(tasks);
}

#define DEFINE_ENTRY(T, SUF)                                                                         \
    void oracle_forward_##SUF(const T* D, int64_t B, int64_t N, int64_t M, const int64_t* lx,        \
                              const int64_t* ly, double gamma, int64_t bandwidth, T* R, T* costs,    \
                              int nthreads)                                                          \
    {                                                                                                 \
        job_t jb = {D, NULL, R, costs, B, N, M, lx, ly, gamma, bandwidth, 0, B};                     \
        run_parallel(fwd_range_##SUF, &jb, nthreads);                                                \
    }                                                                                                 \
    void oracle_backward_##SUF(const T* D, const T* R, int64_t B, int64_t N, int64_t M,              \
                               const int64_t* lx, const int64_t* ly, double gamma, int64_t bandwidth, \
                               T* E, int nthreads)                                                   \
    {                                                                                                 \
        job_t jb = {D, R, E, NULL, B, N, M, lx, ly, gamma, bandwidth, 0, B};                         \
        run_parallel(bwd_range_##SUF, &jb, nthreads);                                                \
    }

DEFINE_ENTRY(double, f64)
DEFINE_ENTRY(float, f32)
