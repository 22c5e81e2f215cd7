/*
 * Native multi-threaded driver for the reference's OpenSSL backend
 * (lmcache_aes128gcm_seal / lmcache_aes128gcm_open from _ref/libcpu_seal.so).
 * Test and CPU-reference-timing infrastructure only: bench.py's reference leg calls it to
 * time the CPU path on all host cores without a Python interpreter between
 * calls (small objects take microseconds, so a Python loop would time the
 * interpreter, not OpenSSL).
 *
 *   int cpu_threads_sweep(key, P, threads, per, &seal_s, &open_s)
 *
 * Each of `threads` pthreads seals `per` objects of P bytes from its own
 * buffer, then opens its frame `per` times; both legs start behind a
 * barrier and are timed on the calling thread. Returns 0, or -1 on an
 * allocation failure or a nonzero rc from the backend.
 *
 *   int cpu_threads_objects(key, srcs, frames, outs, P, count, threads, &seal_s, &open_s)
 *
 * The caller's `count` distinct objects of P bytes (srcs[k]) are dealt to
 * `threads` pthreads (object k to thread k mod threads); each thread seals
 * its objects into frames[k] (P + 29 bytes), then, in the second timed leg,
 * opens every frame into outs[k]. Returns 0 when every call succeeded and
 * every outs[k] equals srcs[k], else -1.
 */
#define _GNU_SOURCE
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

/* the reference backend's C interface (experiments/gpu_kv_seal/native/cpu_seal_openssl.cpp) */
int lmcache_aes128gcm_seal(const uint8_t* key, const uint8_t* src, size_t len, uint8_t* dst, size_t cap);
int lmcache_aes128gcm_open(const uint8_t* key, const uint8_t* src, size_t len, uint8_t* dst, size_t cap);

struct job {
    const uint8_t* key;
    size_t P;
    long per;
    uint8_t* src;
    uint8_t* frame;
    uint8_t* out;
    pthread_barrier_t* start;
    pthread_barrier_t* done;
    int failed;
};

static void* worker(void* arg)
{
    struct job* j = (struct job*)arg;
    /* seal leg */
    pthread_barrier_wait(j->start);
    for (long k = 0; k < j->per; ++k) {
        if (lmcache_aes128gcm_seal(j->key, j->src, j->P, j->frame, j->P + 29) != 0) {
            j->failed = 1;
        }
    }
    pthread_barrier_wait(j->done);
    /* open leg */
    pthread_barrier_wait(j->start);
    for (long k = 0; k < j->per; ++k) {
        if (lmcache_aes128gcm_open(j->key, j->frame, j->P + 29, j->out, j->P) != 0) {
            j->failed = 1;
        }
    }
    pthread_barrier_wait(j->done);
    return NULL;
}

static double now_s(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

int cpu_threads_sweep(const uint8_t* key, size_t P, int threads, long per, double* seal_s, double* open_s)
{
    if (threads < 1 || per < 1) {
        return -1;
    }
    struct job* jobs = calloc((size_t)threads, sizeof(struct job));
    pthread_t* tids = calloc((size_t)threads, sizeof(pthread_t));
    pthread_barrier_t start, done;
    int rc = 0;
    if (jobs == NULL || tids == NULL) {
        free(jobs);
        free(tids);
        return -1;
    }
    pthread_barrier_init(&start, NULL, (unsigned)threads + 1);
    pthread_barrier_init(&done, NULL, (unsigned)threads + 1);
    for (int t = 0; t < threads; ++t) {
        struct job* j = &jobs[t];
        j->key = key;
        j->P = P;
        j->per = per;
        j->src = malloc(P ? P : 1);
        j->frame = malloc(P + 29);
        j->out = malloc(P ? P : 1);
        j->start = &start;
        j->done = &done;
        if (j->src == NULL || j->frame == NULL || j->out == NULL) {
            rc = -1;
            break;
        }
        uint64_t x = 0x9e3779b97f4a7c15ull * (uint64_t)(t + 1);
        for (size_t b = 0; b < P; ++b) {
            x ^= x << 13;
            x ^= x >> 7;
            x ^= x << 17;
            j->src[b] = (uint8_t)x;
        }
        /* frames for the open leg */
        if (lmcache_aes128gcm_seal(key, j->src, P, j->frame, P + 29) != 0) {
            rc = -1;
            break;
        }
    }
    if (rc == 0) {
        for (int t = 0; t < threads; ++t) {
            pthread_create(&tids[t], NULL, worker, &jobs[t]);
        }
        pthread_barrier_wait(&start);
        double t0 = now_s();
        pthread_barrier_wait(&done);
        *seal_s = now_s() - t0;
        pthread_barrier_wait(&start);
        t0 = now_s();
        pthread_barrier_wait(&done);
        *open_s = now_s() - t0;
        for (int t = 0; t < threads; ++t) {
            pthread_join(tids[t], NULL);
            if (jobs[t].failed || memcmp(jobs[t].out, jobs[t].src, P) != 0) {
                rc = -1;
            }
        }
    }
    for (int t = 0; t < threads; ++t) {
        free(jobs[t].src);
        free(jobs[t].frame);
        free(jobs[t].out);
    }
    pthread_barrier_destroy(&start);
    pthread_barrier_destroy(&done);
    free(jobs);
    free(tids);
    return rc;
}

struct obj_job {
    const uint8_t* key;
    size_t P;
    int count;
    int threads;
    int t;
    uint8_t* const* srcs;
    uint8_t* const* frames;
    uint8_t* const* outs;
    pthread_barrier_t* start;
    pthread_barrier_t* done;
    int failed;
};

static void* obj_worker(void* arg)
{
    struct obj_job* j = (struct obj_job*)arg;
    pthread_barrier_wait(j->start);
    for (int k = j->t; k < j->count; k += j->threads) {
        if (lmcache_aes128gcm_seal(j->key, j->srcs[k], j->P, j->frames[k], j->P + 29) != 0) {
            j->failed = 1;
        }
    }
    pthread_barrier_wait(j->done);
    pthread_barrier_wait(j->start);
    for (int k = j->t; k < j->count; k += j->threads) {
        if (lmcache_aes128gcm_open(j->key, j->frames[k], j->P + 29, j->outs[k], j->P) != 0) {
            j->failed = 1;
        }
    }
    pthread_barrier_wait(j->done);
    return NULL;
}

int cpu_threads_objects(const uint8_t* key, uint8_t* const* srcs, uint8_t* const* frames, uint8_t* const* outs,
                        size_t P, int count, int threads, double* seal_s, double* open_s)
{
    if (threads < 1 || count < 1) {
        return -1;
    }
    if (threads > count) {
        threads = count;
    }
    struct obj_job* jobs = calloc((size_t)threads, sizeof(struct obj_job));
    pthread_t* tids = calloc((size_t)threads, sizeof(pthread_t));
    if (jobs == NULL || tids == NULL) {
        free(jobs);
        free(tids);
        return -1;
    }
    pthread_barrier_t start, done;
    pthread_barrier_init(&start, NULL, (unsigned)threads + 1);
    pthread_barrier_init(&done, NULL, (unsigned)threads + 1);
    for (int t = 0; t < threads; ++t) {
        jobs[t] = (struct obj_job){key, P, count, threads, t, srcs, frames, outs, &start, &done, 0};
        pthread_create(&tids[t], NULL, obj_worker, &jobs[t]);
    }
    pthread_barrier_wait(&start);
    double t0 = now_s();
    pthread_barrier_wait(&done);
    *seal_s = now_s() - t0;
    pthread_barrier_wait(&start);
    t0 = now_s();
    pthread_barrier_wait(&done);
    *open_s = now_s() - t0;
    int rc = 0;
    for (int t = 0; t < threads; ++t) {
        pthread_join(tids[t], NULL);
        rc |= jobs[t].failed ? -1 : 0;
    }
    for (int k = 0; k < count && rc == 0; ++k) {
        if (memcmp(outs[k], srcs[k], P) != 0) {
            rc = -1;
        }
    }
    pthread_barrier_destroy(&start);
    pthread_barrier_destroy(&done);
    free(jobs);
    free(tids);
    return rc;
}
