/*
 * scheduler.c -- single-decoder-thread micro-batcher over the batch engine,
 * with the contract of the reference's src/server/scheduler.c:45-168:
 * callers block in slate_llama_scheduler_decode() while one decoder thread
 * drains up to max_batch pending (slot, token) requests into one
 * slate_llama_batch_step() and wakes each caller with its result.
 *
 * Differences that follow from the device engine: requests carry a slot id
 * instead of a session pointer, the step returns the greedy token, and the
 * [n, vocab] logits are copied back only when some request in the batch asked
 * for them.  A batch never holds one slot twice; a second request for a slot
 * waits for the next batch.
 */
#define _GNU_SOURCE
#include "slate_cuda.h"

#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

#define POOL_CAP 256   /* pending-queue capacity, scheduler.c:17 */

typedef struct req {
    int slot;
    int32_t token;
    int32_t* out_token;
    float* out_logits;
    int done, rc;
    pthread_mutex_t lock;
    pthread_cond_t cond;
} req_t;

struct slate_llama_scheduler {
    slate_llama_batch_t* batch;
    int max_batch, vocab;
    pthread_mutex_t pool_lock;
    pthread_cond_t pool_cond;
    req_t* pending[POOL_CAP];
    int n_pending;
    pthread_t decoder;
    _Atomic int running;
    _Atomic uint64_t total_batches, total_requests;
};

static void* decoder_main(void* arg) {
    slate_llama_scheduler_t* s = (slate_llama_scheduler_t*)arg;
    req_t* drain[POOL_CAP];
    int32_t slots[POOL_CAP], toks[POOL_CAP], outs[POOL_CAP];
    float* logits = (float*)malloc((size_t)s->vocab * s->max_batch * sizeof(float));
    while (1) {
        pthread_mutex_lock(&s->pool_lock);
        while (atomic_load(&s->running) && s->n_pending == 0)
            pthread_cond_wait(&s->pool_cond, &s->pool_lock);
        if (!atomic_load(&s->running) && s->n_pending == 0) {
            pthread_mutex_unlock(&s->pool_lock);
            break;
        }
        int n = 0, keep = 0;
        for (int i = 0; i < s->n_pending; ++i) {
            req_t* r = s->pending[i];
            int dup = 0;
            for (int j = 0; j < n; ++j) dup |= (slots[j] == r->slot);
            if (n < s->max_batch && !dup) {
                drain[n] = r;
                slots[n] = r->slot;
                toks[n] = r->token;
                ++n;
            } else {
                s->pending[keep++] = r;
            }
        }
        s->n_pending = keep;
        pthread_mutex_unlock(&s->pool_lock);

        int want_logits = 0;
        for (int i = 0; i < n; ++i) want_logits |= drain[i]->out_logits != NULL;
        int rc = slate_llama_batch_step(s->batch, slots, n, toks, outs,
                                        want_logits && logits ? logits : NULL);
        atomic_fetch_add(&s->total_batches, 1);
        atomic_fetch_add(&s->total_requests, (uint64_t)n);
        for (int i = 0; i < n; ++i) {
            req_t* r = drain[i];
            if (rc == 0) {
                if (r->out_token) *r->out_token = outs[i];
                if (r->out_logits)
                    memcpy(r->out_logits, logits + (size_t)i * s->vocab, (size_t)s->vocab * 4);
            }
            pthread_mutex_lock(&r->lock);
            r->rc = rc;
            r->done = 1;
            pthread_cond_signal(&r->cond);
            pthread_mutex_unlock(&r->lock);
        }
    }
    free(logits);
    return NULL;
}

slate_llama_scheduler_t* slate_llama_scheduler_new(slate_llama_batch_t* b, int max_batch) {
    if (!b || max_batch <= 0) return NULL;
    if (max_batch > POOL_CAP) max_batch = POOL_CAP;
    if (max_batch > slate_llama_batch_max_batch(b)) max_batch = slate_llama_batch_max_batch(b);
    slate_llama_scheduler_t* s = (slate_llama_scheduler_t*)calloc(1, sizeof(*s));
    if (!s) return NULL;
    s->batch = b;
    s->max_batch = max_batch;
    s->vocab = slate_llama_batch_vocab(b);
    pthread_mutex_init(&s->pool_lock, NULL);
    pthread_cond_init(&s->pool_cond, NULL);
    atomic_store(&s->running, 1);
    if (pthread_create(&s->decoder, NULL, decoder_main, s) != 0) {
        pthread_mutex_destroy(&s->pool_lock);
        pthread_cond_destroy(&s->pool_cond);
        free(s);
        return NULL;
    }
    return s;
}

void slate_llama_scheduler_free(slate_llama_scheduler_t* s) {
    if (!s) return;
    atomic_store(&s->running, 0);
    pthread_mutex_lock(&s->pool_lock);
    pthread_cond_broadcast(&s->pool_cond);
    pthread_mutex_unlock(&s->pool_lock);
    pthread_join(s->decoder, NULL);
    pthread_mutex_destroy(&s->pool_lock);
    pthread_cond_destroy(&s->pool_cond);
    free(s);
}

int slate_llama_scheduler_decode(slate_llama_scheduler_t* s, int slot, int32_t token,
                                 int32_t* out_token, float* out_logits) {
    if (!s || slot < 0) return -1;
    req_t r;
    memset(&r, 0, sizeof r);
    r.slot = slot;
    r.token = token;
    r.out_token = out_token;
    r.out_logits = out_logits;
    pthread_mutex_init(&r.lock, NULL);
    pthread_cond_init(&r.cond, NULL);
    pthread_mutex_lock(&s->pool_lock);
    if (s->n_pending >= POOL_CAP || !atomic_load(&s->running)) {
        pthread_mutex_unlock(&s->pool_lock);
        pthread_mutex_destroy(&r.lock);
        pthread_cond_destroy(&r.cond);
        return -2;
    }
    s->pending[s->n_pending++] = &r;
    pthread_cond_signal(&s->pool_cond);
    pthread_mutex_unlock(&s->pool_lock);
    pthread_mutex_lock(&r.lock);
    while (!r.done) pthread_cond_wait(&r.cond, &r.lock);
    int rc = r.rc;
    pthread_mutex_unlock(&r.lock);
    pthread_mutex_destroy(&r.lock);
    pthread_cond_destroy(&r.cond);
    return rc;
}

int slate_llama_scheduler_pending(const slate_llama_scheduler_t* s) {
    if (!s) return 0;
    pthread_mutex_lock((pthread_mutex_t*)&s->pool_lock);
    int n = s->n_pending;
    pthread_mutex_unlock((pthread_mutex_t*)&s->pool_lock);
    return n;
}
uint64_t slate_llama_scheduler_total_batches(const slate_llama_scheduler_t* s) {
    return s ? atomic_load(&s->total_batches) : 0;
}
double slate_llama_scheduler_avg_batch_size(const slate_llama_scheduler_t* s) {
    if (!s) return 0.0;
    uint64_t b = atomic_load(&s->total_batches), r = atomic_load(&s->total_requests);
    return b ? (double)r / (double)b : 0.0;
}
