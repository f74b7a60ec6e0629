/* Oracle thread pool: a persistent pool that runs parallel-for loops over [0, n) with dynamic chunking, the role
 * Parallel.For plays in the reference (Transformer.cs:496-501, 357). Results never depend on the thread count:
 * every index is computed by one thread with the same arithmetic. Test infrastructure only (see oracle.h). */
#include "oracle.h"
#include <pthread.h>
#include <stdatomic.h>
#include <unistd.h>
#include <stdlib.h>

#define MAX_THREADS 256

static pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;      /* serialises whole parallel-for calls */
static pthread_mutex_t g_job_mu = PTHREAD_MUTEX_INITIALIZER;
static pthread_cond_t g_job_cv = PTHREAD_COND_INITIALIZER;
static pthread_cond_t g_done_cv = PTHREAD_COND_INITIALIZER;
static int g_started = 0, g_nthreads = 0;
static uint64_t g_generation = 0;
static int g_active_workers = 0, g_pending = 0;
static or_task_fn g_fn; static void* g_ctx; static int64_t g_n, g_chunk;
static atomic_llong g_next;

int or_default_threads(void)
{
    const char* env = getenv("WINDLASS_ORACLE_THREADS");
    if (env && atoi(env) > 0) return atoi(env);
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

static void run_chunks(void)
{
    for (;;) {
        int64_t b = atomic_fetch_add(&g_next, g_chunk);
        if (b >= g_n) break;
        int64_t e = b + g_chunk < g_n ? b + g_chunk : g_n;
        g_fn(g_ctx, b, e);
    }
}

static void* worker(void* arg)
{
    int id = (int)(intptr_t)arg;
    uint64_t seen = 0;
    for (;;) {
        pthread_mutex_lock(&g_job_mu);
        while (g_generation == seen || id >= g_active_workers) {
            if (g_generation != seen) seen = g_generation;   /* a job this worker sits out */
            pthread_cond_wait(&g_job_cv, &g_job_mu);
        }
        seen = g_generation;
        pthread_mutex_unlock(&g_job_mu);
        run_chunks();
        pthread_mutex_lock(&g_job_mu);
        if (--g_pending == 0) pthread_cond_signal(&g_done_cv);
        pthread_mutex_unlock(&g_job_mu);
    }
    return NULL;
}

static void start_pool(void)
{
    g_nthreads = or_default_threads();
    if (g_nthreads > MAX_THREADS) g_nthreads = MAX_THREADS;
    for (int i = 1; i < g_nthreads; i++) {          /* the caller is worker 0 */
        pthread_t t;
        pthread_create(&t, NULL, worker, (void*)(intptr_t)i);
        pthread_detach(t);
    }
    g_started = 1;
}

void or_parallel_for(int64_t n, int threads, or_task_fn fn, void* ctx)
{
    if (n <= 0) return;
    pthread_mutex_lock(&g_mu);
    if (!g_started) start_pool();
    int want = threads > 0 ? threads : g_nthreads;
    if (want > g_nthreads) want = g_nthreads;
    if (want > n) want = (int)n;
    if (want <= 1) { fn(ctx, 0, n); pthread_mutex_unlock(&g_mu); return; }
    g_fn = fn; g_ctx = ctx; g_n = n;
    g_chunk = n / (want * 4); if (g_chunk < 1) g_chunk = 1;
    atomic_store(&g_next, 0);
    pthread_mutex_lock(&g_job_mu);
    g_active_workers = want;          /* workers 1..want-1 join; ids >= want sit this job out */
    g_pending = want - 1;
    g_generation++;
    pthread_cond_broadcast(&g_job_cv);
    pthread_mutex_unlock(&g_job_mu);
    run_chunks();
    pthread_mutex_lock(&g_job_mu);
    while (g_pending > 0) pthread_cond_wait(&g_done_cv, &g_job_mu);
    pthread_mutex_unlock(&g_job_mu);
    pthread_mutex_unlock(&g_mu);
}
