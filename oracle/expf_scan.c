/* expf_scan.c -- test infrastructure, not product code.
 *
 * Compares the host libm's expf, which the reference's softmax calls
 * (std::exp on a float, src/router/CpuRouterBackend.cpp:54), with the
 * correctly rounded exponential on every float in [-104, 0] (the range of
 * score - max; below -104 both give 0).  The correctly rounded value is expl
 * rounded to float; inputs whose extended-precision result lies within 1e-17
 * (relative) of a float midpoint are reported as ambiguous instead of judged.
 *
 *   make -C oracle expf_scan && oracle/_build/expf_scan [-v]
 *
 * Prints the number of misrounded and ambiguous inputs and a histogram by
 * binade of |x|; -v also lists every misrounded input. */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include <unistd.h>

static float f_of(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t u_of(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

enum { kMaxThreads = 256, kBins = 300 };
static uint32_t g_lo, g_hi;
static int g_threads, g_verbose;
static pthread_mutex_t g_print = PTHREAD_MUTEX_INITIALIZER;

typedef struct {
    int id;
    long mism, amb;
    long hist[kBins];
} Part;

static void* scan(void* arg) {
    Part* p = (Part*)arg;
    for (uint64_t i = (uint64_t)g_lo + (uint64_t)p->id; i <= g_hi; i += (uint64_t)g_threads) {
        const float x = f_of((uint32_t)i);
        const float g = expf(x);
        const long double e = expl((long double)x);
        const float r = (float)e;
        const float other = nextafterf(r, e > (long double)r ? INFINITY : 0.0f);
        const long double mid = ((long double)r + (long double)other) / 2;
        if (e != 0 && fabsl(e - mid) / e < 1e-17L) {
            p->amb++;
            continue;
        }
        if (u_of(g) != u_of(r)) {
            int ex;
            frexpf(x, &ex);
            p->hist[ex + 150]++;
            p->mism++;
            if (g_verbose) {
                pthread_mutex_lock(&g_print);
                printf("%a %a %a\n", x, g, r);
                pthread_mutex_unlock(&g_print);
            }
        }
    }
    return NULL;
}

int main(int argc, char** argv) {
    g_verbose = argc > 1 && strcmp(argv[1], "-v") == 0;
    g_lo = 0x80000000u;
    g_hi = u_of(-104.0f);
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    g_threads = n < 1 ? 1 : n > kMaxThreads ? kMaxThreads : (int)n;
    static Part parts[kMaxThreads];
    pthread_t th[kMaxThreads];
    for (int t = 0; t < g_threads; ++t) {
        parts[t].id = t;
        pthread_create(&th[t], NULL, scan, &parts[t]);
    }
    long mism = 0, amb = 0, hist[kBins] = {0};
    for (int t = 0; t < g_threads; ++t) {
        pthread_join(th[t], NULL);
        mism += parts[t].mism;
        amb += parts[t].amb;
        for (int b = 0; b < kBins; ++b) hist[b] += parts[t].hist[b];
    }
    for (int b = 0; b < kBins; ++b)
        if (hist[b]) printf("|x| in [2^%d, 2^%d): %ld misrounded\n", b - 151, b - 150, hist[b]);
    printf("scanned %u floats in [-104, 0] on %d threads: expf misrounded %ld, ambiguous %ld\n",
           g_hi - g_lo + 1, g_threads, mism, amb);
    return 0;
}
