/*
 * CPU ORACLE — test infrastructure only (see g4a_oracle.h).
 *
 * Restates gemma4-rs's f32 attention arithmetic step for step, in the same
 * operation order, so that its results are the reference's on the same libm.
 * Compiled with -O2 -ffp-contract=off and no fast-math: Rust never fuses a
 * multiply and an add, and neither may this file.
 */
#define _GNU_SOURCE
#include "g4a_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

/* ------------------------------------------------------------------------ */
/* Rust float helpers                                                         */
/* ------------------------------------------------------------------------ */

/* f32::total_cmp key (core::f32::total_cmp): flip the magnitude bits of
 * negative values so that a signed integer compare gives IEEE totalOrder. */
static int32_t total_key(float x) {
    int32_t i;
    memcpy(&i, &x, sizeof i);
    i ^= (int32_t)(((uint32_t)(i >> 31)) >> 1);
    return i;
}

float orc_round_f16(float x) { return (float)(_Float16)x; }

float orc_round_bf16(float x) {
    uint32_t u;
    memcpy(&u, &x, sizeof u);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) { /* NaN stays NaN */
        u |= 0x00400000u;
    } else {
        u += 0x7fffu + ((u >> 16) & 1u); /* round to nearest, ties to even */
    }
    u &= 0xffff0000u;
    memcpy(&x, &u, sizeof x);
    return x;
}

/* ------------------------------------------------------------------------ */
/* ops.rs                                                                     */
/* ------------------------------------------------------------------------ */

/* ops.rs:45-56 rms_norm: mean of squares accumulated in f64 (each square is
 * an f32 product widened to f64, summed left to right), mean cast to f32,
 * scale = 1 / sqrt(mean + eps) in f32, y = x * scale [* weight]. */
int orc_rms_norm(const float *x, size_t n, const float *weight, float eps, float *out) {
    if (n == 0 || eps < 0.0f) return ORC_COMPUTE;
    double sum = -0.0;
    for (size_t i = 0; i < n; i++) {
        float sq = x[i] * x[i];
        sum += (double)sq;
    }
    float mean = (float)(sum / (double)n);
    float scale = 1.0f / sqrtf(mean + eps);
    if (weight) {
        for (size_t i = 0; i < n; i++) out[i] = (x[i] * scale) * weight[i];
    } else {
        for (size_t i = 0; i < n; i++) out[i] = x[i] * scale;
    }
    return ORC_OK;
}

/* ops.rs:65-76 dot_f32: 16 strided accumulators (element i goes to lane
 * i % 16 for the full chunks), lanes summed in order from -0.0 (Rust's f32
 * Sum identity), then the tail (its own in-order sum) added last. */
float orc_dot_f32(const float *a, const float *b, size_t n) {
    enum { LANES = 16 };
    float lanes[LANES] = {0};
    size_t full = n - n % LANES;
    float tail = -0.0f;
    for (size_t i = full; i < n; i++) tail += a[i] * b[i];
    for (size_t c = 0; c < full; c += LANES)
        for (int l = 0; l < LANES; l++) lanes[l] += a[c + l] * b[c + l];
    float s = -0.0f;
    for (int l = 0; l < LANES; l++) s += lanes[l];
    return s + tail;
}

/* ops.rs:105-127 softmax_f32: max by total_cmp, e = exp(x - max), in-order
 * f32 sum, error if the sum is not finite or zero, p = e / sum. */
int orc_softmax_f32(const float *x, size_t n, float *out) {
    if (n == 0) return ORC_COMPUTE;
    float mx = x[0];
    int32_t mk = total_key(mx);
    for (size_t i = 1; i < n; i++) { /* max_by keeps the last of equal maxima */
        int32_t k = total_key(x[i]);
        if (k >= mk) { mk = k; mx = x[i]; }
    }
    float sum = -0.0f;
    for (size_t i = 0; i < n; i++) {
        out[i] = expf(x[i] - mx);
        sum += out[i];
    }
    if (!isfinite(sum) || sum == 0.0f) return ORC_NONFINITE;
    for (size_t i = 0; i < n; i++) out[i] = out[i] / sum;
    return ORC_OK;
}

/* ops.rs:134-162 rope_neox: pairs (x[i], x[i + n_rot/2]); the angle of pair
 * i is theta_i / factor_i with theta_0 = position and theta_{i+1} =
 * theta_i * base^(-2/n_rot), built by repeated f32 multiplication. */
int orc_rope_neox(float *x, size_t len, size_t position, float base, size_t n_rot,
                  const float *freq_factors, size_t n_factors) {
    size_t half = n_rot / 2;
    if (n_rot == 0 || n_rot % 2 != 0 || n_rot > len || base <= 0.0f ||
        (freq_factors && n_factors < half))
        return ORC_COMPUTE;
    float theta_scale = powf(base, -2.0f / (float)n_rot);
    float theta = (float)position;
    for (size_t i = 0; i < half; i++) {
        float factor = freq_factors ? freq_factors[i] : 1.0f;
        float angle = theta / factor;
        float s = sinf(angle), c = cosf(angle);
        float a = x[i], b = x[i + half];
        float ac = a * c, bs = b * s, as_ = a * s, bc = b * c;
        x[i] = ac - bs;
        x[i + half] = as_ + bc;
        theta *= theta_scale;
    }
    return ORC_OK;
}

void orc_rope_sincos(size_t position, float base, size_t n_rot, const float *freq_factors,
                     float *sin_out, float *cos_out) {
    size_t half = n_rot / 2;
    float theta_scale = powf(base, -2.0f / (float)n_rot);
    float theta = (float)position;
    for (size_t i = 0; i < half; i++) {
        float factor = freq_factors ? freq_factors[i] : 1.0f;
        float angle = theta / factor;
        sin_out[i] = sinf(angle);
        cos_out[i] = cosf(angle);
        theta *= theta_scale;
    }
}

/* ------------------------------------------------------------------------ */
/* idea/mod.rs, eng/mod.rs                                                    */
/* ------------------------------------------------------------------------ */

/* idea/mod.rs:48-68 Gemma4HyperParams::e2b (attention fields). */
void orc_hparams_e2b(orc_hparams *hp) {
    hp->n_layers = 35;
    hp->n_heads = 8;
    hp->n_kv_heads = 1;
    hp->head_dim_local = 256;
    hp->head_dim_global = 512;
    hp->sliding_window = 512;
    hp->shared_kv_layers = 20;
    hp->local_rope_base = 10000.0f;
    hp->global_rope_base = 1000000.0f;
    hp->global_p = 0.25f;
    hp->rms_norm_eps = 1e-6f;
}

/* idea/mod.rs:148-156 layer_attention_kind: global iff last layer or l%5==4. */
int orc_layer_is_global(const orc_hparams *hp, int32_t layer) {
    return (layer + 1 == hp->n_layers) || (layer % 5 == 4);
}

/* idea/mod.rs:140-145 head_dim. */
int32_t orc_head_dim(const orc_hparams *hp, int32_t layer) {
    return orc_layer_is_global(hp, layer) ? hp->head_dim_global : hp->head_dim_local;
}

/* eng/mod.rs:71-90 kv_source_layer. err_detail receives the KvShareError
 * variant on failure: 1 LayerOutOfRange, 2 TooManySharedLayers,
 * 3 NoEarlierLayerOfSameKind. */
int orc_kv_source_layer(const orc_hparams *hp, int32_t layer, int32_t *source, int32_t *err_detail) {
    int32_t n = hp->n_layers;
    if (layer < 0 || layer >= n) { if (err_detail) *err_detail = 1; return ORC_BAD_LAYER; }
    int32_t first_shared = n - hp->shared_kv_layers;
    if (hp->shared_kv_layers > n || first_shared <= 0) { if (err_detail) *err_detail = 2; return ORC_BAD_LAYER; }
    if (layer < first_shared) { *source = layer; return ORC_OK; }
    int kind = orc_layer_is_global(hp, layer);
    for (int32_t e = first_shared - 1; e >= 0; e--) {
        if (orc_layer_is_global(hp, e) == kind) { *source = e; return ORC_OK; }
    }
    if (err_detail) *err_detail = 3;
    return ORC_BAD_LAYER;
}

/* eng/mod.rs:10-12 windowed_len: seq_len.saturating_sub(window)..seq_len. */
void orc_windowed_len(size_t seq_len, size_t window, size_t *lo, size_t *hi) {
    *lo = seq_len > window ? seq_len - window : 0;
    *hi = seq_len;
}

/* idea/mod.rs:162-165 proportional_rope_freq_factors. */
void orc_proportional_rope_freq_factors(size_t head_dim, float p, float *out) {
    size_t rotated = (size_t)((float)head_dim * p / 2.0f);
    for (size_t pair = 0; pair < head_dim / 2; pair++) out[pair] = pair < rotated ? 1.0f : 1e30f;
}

/* ------------------------------------------------------------------------ */
/* pool.rs: persistent workers, atomic chunk claims, spin then sleep          */
/* ------------------------------------------------------------------------ */

#define SPIN_FOR_NS 200000L   /* pool.rs:28 SPIN_FOR = 200 us */
#define CHUNKS_PER_THREAD 4   /* pool.rs:36 */

typedef struct orc_task {
    size_t chunks;
    atomic_size_t next;
    atomic_size_t remaining;
    atomic_int refs;
    void (*run_chunk)(void *ctx, size_t chunk);
    void *ctx;
    pthread_mutex_t mu;
    pthread_cond_t cv;
    int finished;
} orc_task;

typedef struct qnode { orc_task *task; struct qnode *next; } qnode;

typedef struct worker {
    pthread_t th;
    pthread_mutex_t mu;
    pthread_cond_t cv;
    qnode *head, *tail;
    atomic_int pending;
} worker;

static struct {
    pthread_mutex_t init_mu;
    int inited;
    int n_workers;
    worker *workers;
} g_pool = {PTHREAD_MUTEX_INITIALIZER, 0, 0, NULL};

static long now_ns(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1000000000L + ts.tv_nsec;
}

static void task_release(orc_task *t) {
    if (atomic_fetch_sub(&t->refs, 1) == 1) {
        pthread_mutex_destroy(&t->mu);
        pthread_cond_destroy(&t->cv);
        free(t);
    }
}

/* pool.rs:49-63 Task::work: claim chunks until none are left. */
static void task_work(orc_task *t) {
    for (;;) {
        size_t chunk = atomic_fetch_add_explicit(&t->next, 1, memory_order_relaxed);
        if (chunk >= t->chunks) return;
        t->run_chunk(t->ctx, chunk);
        if (atomic_fetch_sub_explicit(&t->remaining, 1, memory_order_acq_rel) == 1) {
            pthread_mutex_lock(&t->mu);
            t->finished = 1;
            pthread_cond_broadcast(&t->cv);
            pthread_mutex_unlock(&t->mu);
        }
    }
}

/* pool.rs:65-77 Task::wait: spin for SPIN_FOR, then sleep on the signal. */
static void task_wait(orc_task *t) {
    long deadline = now_ns() + SPIN_FOR_NS;
    while (now_ns() < deadline) {
        if (atomic_load_explicit(&t->remaining, memory_order_acquire) == 0) return;
    }
    pthread_mutex_lock(&t->mu);
    while (!t->finished) pthread_cond_wait(&t->cv, &t->mu);
    pthread_mutex_unlock(&t->mu);
}

/* pool.rs:114-124 next_task: spin for SPIN_FOR before sleeping. */
static orc_task *next_task(worker *w) {
    long deadline = now_ns() + SPIN_FOR_NS;
    for (;;) {
        if (atomic_load_explicit(&w->pending, memory_order_acquire) > 0 || now_ns() >= deadline) {
            pthread_mutex_lock(&w->mu);
            while (!w->head) pthread_cond_wait(&w->cv, &w->mu);
            qnode *n = w->head;
            w->head = n->next;
            if (!w->head) w->tail = NULL;
            atomic_fetch_sub(&w->pending, 1);
            pthread_mutex_unlock(&w->mu);
            orc_task *t = n->task;
            free(n);
            return t;
        }
    }
}

static void *worker_main(void *arg) {
    worker *w = (worker *)arg;
    for (;;) {
        orc_task *t = next_task(w);
        task_work(t);
        task_release(t);
    }
    return NULL;
}

/* pool.rs:86-110 pool(): LLM_THREADS if set, else every core. `threads`
 * > 0 overrides (used to time the baseline at a stated thread count); the
 * pool can be sized once per process. */
int orc_pool_init(int threads) {
    pthread_mutex_lock(&g_pool.init_mu);
    if (!g_pool.inited) {
        if (threads <= 0) {
            const char *env = getenv("LLM_THREADS");
            threads = env ? atoi(env) : 0;
            if (threads <= 0) threads = (int)sysconf(_SC_NPROCESSORS_ONLN);
            if (threads <= 0) threads = 1;
        }
        g_pool.n_workers = threads - 1;
        g_pool.workers = calloc((size_t)(g_pool.n_workers > 0 ? g_pool.n_workers : 1), sizeof(worker));
        for (int i = 0; i < g_pool.n_workers; i++) {
            worker *w = &g_pool.workers[i];
            pthread_mutex_init(&w->mu, NULL);
            pthread_cond_init(&w->cv, NULL);
            atomic_init(&w->pending, 0);
            pthread_create(&w->th, NULL, worker_main, w);
            pthread_detach(w->th);
        }
        g_pool.inited = 1;
    }
    int n = g_pool.n_workers + 1;
    pthread_mutex_unlock(&g_pool.init_mu);
    return n;
}

/* pool.rs:82-84 threads(). */
int orc_pool_threads(void) { return orc_pool_init(0); }

/* pool.rs:160-197 run_chunks: inline below the work threshold, otherwise
 * ceil(count / (threads * 4)) items per chunk, claimed by the caller and the
 * workers. Each chunk writes its own output slots, so no concatenation step
 * is needed here. */
static void run_chunks(size_t count, size_t work_per_item, size_t parallel_min_work,
                       void (*run_range)(void *ctx, size_t lo, size_t hi), void *ctx);

typedef struct { void (*run_range)(void *, size_t, size_t); void *ctx; size_t chunk_len, count; } range_ctx;
static void run_chunk_range(void *c, size_t chunk) {
    range_ctx *rc = (range_ctx *)c;
    size_t lo = chunk * rc->chunk_len;
    size_t hi = lo + rc->chunk_len < rc->count ? lo + rc->chunk_len : rc->count;
    rc->run_range(rc->ctx, lo, hi);
}

static void run_chunks(size_t count, size_t work_per_item, size_t parallel_min_work,
                       void (*run_range)(void *ctx, size_t lo, size_t hi), void *ctx) {
    int threads = orc_pool_init(0);
    size_t work = count * work_per_item;
    if (threads <= 1 || work < parallel_min_work) { run_range(ctx, 0, count); return; }
    size_t per = (size_t)threads * CHUNKS_PER_THREAD;
    size_t chunk_len = (count + per - 1) / per;
    if (chunk_len == 0) chunk_len = 1;
    size_t chunks = (count + chunk_len - 1) / chunk_len;
    range_ctx rc = {run_range, ctx, chunk_len, count};
    orc_task *t = calloc(1, sizeof *t);
    t->chunks = chunks;
    atomic_init(&t->next, 0);
    atomic_init(&t->remaining, chunks);
    atomic_init(&t->refs, g_pool.n_workers + 1);
    t->run_chunk = run_chunk_range;
    t->ctx = &rc;
    pthread_mutex_init(&t->mu, NULL);
    pthread_cond_init(&t->cv, NULL);
    for (int i = 0; i < g_pool.n_workers; i++) { /* pool.rs:188-190 send to every worker */
        worker *w = &g_pool.workers[i];
        qnode *n = malloc(sizeof *n);
        n->task = t;
        n->next = NULL;
        pthread_mutex_lock(&w->mu);
        if (w->tail) w->tail->next = n; else w->head = n;
        w->tail = n;
        atomic_fetch_add(&w->pending, 1);
        pthread_cond_signal(&w->cv);
        pthread_mutex_unlock(&w->mu);
    }
    task_work(t);
    task_wait(t);
    /* Workers that arrive after the last chunk only see next >= chunks and
     * never touch rc; the task itself lives until every worker let go. */
    task_release(t);
}

/* ------------------------------------------------------------------------ */
/* model.rs:307-366 attention                                                 */
/* ------------------------------------------------------------------------ */

#define ATTENTION_PARALLEL_MIN_WORK ((size_t)1 << 18) /* model.rs:308 */

typedef struct {
    const float *q, *keys, *values;
    size_t len, kv_width, head_dim, n_heads, n_kv_heads;
    float scale;
    float *out;
    int *head_failed;
} attn_job;

/* model.rs:326-343 attend_head: scores = dot_f32(q_h, k_j[kv]) * scale for
 * every key in order, softmax, out = sum_j p_j * v_j[kv] accumulated in key
 * order. A failed softmax marks the head (the reference returns an empty
 * vector, which attend then reports as non-finite). */
static void attend_head(const attn_job *job, size_t head) {
    size_t hd = job->head_dim;
    const float *qh = job->q + head * hd;
    size_t kv_head = head * job->n_kv_heads / job->n_heads;
    size_t off = kv_head * hd;
    float *scores = malloc((job->len ? job->len : 1) * sizeof(float));
    float *probs = malloc((job->len ? job->len : 1) * sizeof(float));
    for (size_t j = 0; j < job->len; j++)
        scores[j] = orc_dot_f32(qh, job->keys + j * job->kv_width + off, hd) * job->scale;
    float *o = job->out + head * hd;
    if (job->len == 0 || orc_softmax_f32(scores, job->len, probs) != ORC_OK) {
        job->head_failed[head] = 1;
    } else {
        for (size_t i = 0; i < hd; i++) o[i] = 0.0f;
        for (size_t j = 0; j < job->len; j++) {
            const float *vj = job->values + j * job->kv_width + off;
            float p = probs[j];
            for (size_t i = 0; i < hd; i++) {
                float pv = p * vj[i];
                o[i] += pv;
            }
        }
    }
    free(scores);
    free(probs);
}

static void attend_range(void *ctx, size_t lo, size_t hi) {
    for (size_t h = lo; h < hi; h++) attend_head((const attn_job *)ctx, h);
}

/* model.rs:348-366 attend: keys/values are already one contiguous row per
 * position (the reference's `concat`), heads run on the pool once
 * n_heads * 2 * len * head_dim reaches ATTENTION_PARALLEL_MIN_WORK. */
int orc_attend(const float *q, const float *keys, const float *values, size_t len,
               size_t n_heads, size_t n_kv_heads, size_t head_dim, float scale, float *out) {
    if (n_heads == 0 || n_kv_heads == 0 || head_dim == 0) return ORC_COMPUTE;
    int failed[1024];
    if (n_heads > 1024) return ORC_COMPUTE;
    memset(failed, 0, n_heads * sizeof(int));
    attn_job job = {q, keys, values, len, n_kv_heads * head_dim, head_dim, n_heads, n_kv_heads,
                    scale, out, failed};
    size_t work_per_head = 2 * len * head_dim;
    run_chunks(n_heads, work_per_head, ATTENTION_PARALLEL_MIN_WORK, attend_range, &job);
    for (size_t h = 0; h < n_heads; h++)
        if (failed[h]) return ORC_NONFINITE; /* model.rs:362-364 */
    return ORC_OK;
}

/* ------------------------------------------------------------------------ */
/* context_memory.rs                                                          */
/* ------------------------------------------------------------------------ */

typedef struct { float *keys, *values; size_t len, cap, width; } kv_layer;
struct orc_kv { kv_layer *layers; size_t n_layers; };

orc_kv *orc_kv_create(void) { return calloc(1, sizeof(orc_kv)); }

void orc_kv_clear(orc_kv *kv) { /* context_memory.rs:83-85 */
    for (size_t i = 0; i < kv->n_layers; i++) { free(kv->layers[i].keys); free(kv->layers[i].values); }
    free(kv->layers);
    kv->layers = NULL;
    kv->n_layers = 0;
}

void orc_kv_destroy(orc_kv *kv) { if (kv) { orc_kv_clear(kv); free(kv); } }

/* context_memory.rs:44-51 append: grow the layer list, push one row. */
int orc_kv_append(orc_kv *kv, size_t layer, const float *k, const float *v, size_t width) {
    if (kv->n_layers <= layer) {
        kv->layers = realloc(kv->layers, (layer + 1) * sizeof(kv_layer));
        memset(kv->layers + kv->n_layers, 0, (layer + 1 - kv->n_layers) * sizeof(kv_layer));
        kv->n_layers = layer + 1;
    }
    kv_layer *L = &kv->layers[layer];
    if (L->len > 0 && L->width != width) return ORC_COMPUTE;
    L->width = width;
    if (L->len == L->cap) {
        L->cap = L->cap ? 2 * L->cap : 64;
        L->keys = realloc(L->keys, L->cap * width * sizeof(float));
        L->values = realloc(L->values, L->cap * width * sizeof(float));
    }
    memcpy(L->keys + L->len * width, k, width * sizeof(float));
    memcpy(L->values + L->len * width, v, width * sizeof(float));
    L->len++;
    return ORC_OK;
}

/* n appends of consecutive rows (k, v each [n][width]). */
int orc_kv_append_rows(orc_kv *kv, size_t layer, const float *k, const float *v, size_t width, size_t n) {
    for (size_t i = 0; i < n; i++) {
        int rc = orc_kv_append(kv, layer, k + i * width, v + i * width, width);
        if (rc) return rc;
    }
    return ORC_OK;
}

/* context_memory.rs:53-69 view: a missing layer is fine only for len 0;
 * asking for more rows than stored is ContextTooLong. A layer that exists
 * only because a later one was appended (resize_with) has zero rows. */
int orc_kv_view(const orc_kv *kv, size_t layer, size_t len, const float **keys,
                const float **values, size_t *width, size_t *max_len) {
    if (layer >= kv->n_layers) {
        if (len == 0) { *keys = NULL; *values = NULL; *width = 0; return ORC_OK; }
        return ORC_MISSING_LAYER;
    }
    const kv_layer *L = &kv->layers[layer];
    if (max_len) *max_len = L->len;
    if (len > L->len) return ORC_CONTEXT_TOO_LONG;
    *keys = L->keys;
    *values = L->values;
    *width = L->width;
    return ORC_OK;
}

/* ------------------------------------------------------------------------ */
/* model.rs:393-410: one layer's attention block without the projections      */
/* ------------------------------------------------------------------------ */

/* norm_heads (model.rs:283-290) over n_heads heads of width hd, in place. */
static int norm_heads(float *x, size_t n_heads, size_t hd, const float *w, float eps) {
    float *tmp = malloc(hd * sizeof(float));
    for (size_t h = 0; h < n_heads; h++) {
        int rc = orc_rms_norm(x + h * hd, hd, w, eps, tmp);
        if (rc) { free(tmp); return rc; }
        memcpy(x + h * hd, tmp, hd * sizeof(float));
    }
    free(tmp);
    return ORC_OK;
}

/* rope_heads (model.rs:295-304): local layers use the local base and no
 * factors; global layers use the global base and rope_freqs. */
static int rope_heads(float *x, size_t n_heads, size_t hd, size_t pos, int global,
                      const orc_hparams *hp, const float *rope_freqs) {
    float base = global ? hp->global_rope_base : hp->local_rope_base;
    const float *ff = global ? rope_freqs : NULL;
    for (size_t h = 0; h < n_heads; h++) {
        int rc = orc_rope_neox(x + h * hd, hd, pos, base, hd, ff, ff ? hd / 2 : 0);
        if (rc) return rc;
    }
    return ORC_OK;
}

int orc_attention_block(orc_kv *kv, const orc_hparams *hp, int32_t layer, size_t position,
                        const float *q_raw, const float *k_raw, const float *v_raw,
                        const float *q_norm_w, const float *k_norm_w,
                        const float *rope_freqs, int kv_store, float *out) {
    size_t nh = (size_t)hp->n_heads, nkv = (size_t)hp->n_kv_heads;
    size_t hd = (size_t)orc_head_dim(hp, layer);
    int global = orc_layer_is_global(hp, layer);
    float *q = malloc(nh * hd * sizeof(float));
    memcpy(q, q_raw, nh * hd * sizeof(float));
    int rc = norm_heads(q, nh, hd, q_norm_w, hp->rms_norm_eps);           /* :395 */
    if (!rc) rc = rope_heads(q, nh, hd, position, global, hp, rope_freqs); /* :396 */
    int32_t source = -1;
    if (!rc) rc = orc_kv_source_layer(hp, layer, &source, NULL);            /* :398 */
    if (!rc && source == layer) {                                           /* :399-406 */
        size_t w = nkv * hd;
        float *k = malloc(w * sizeof(float)), *v = malloc(w * sizeof(float));
        memcpy(k, k_raw, w * sizeof(float));
        memcpy(v, v_raw, w * sizeof(float));
        rc = norm_heads(k, nkv, hd, k_norm_w, hp->rms_norm_eps);
        if (!rc) rc = norm_heads(v, nkv, hd, NULL, hp->rms_norm_eps);
        if (!rc) rc = rope_heads(k, nkv, hd, position, global, hp, rope_freqs);
        if (!rc && kv_store == 1)
            for (size_t i = 0; i < w; i++) { k[i] = orc_round_f16(k[i]); v[i] = orc_round_f16(v[i]); }
        if (!rc) rc = orc_kv_append(kv, (size_t)layer, k, v, w);
        free(k);
        free(v);
    }
    const float *keys = NULL, *values = NULL;
    size_t width = 0;
    if (!rc) rc = orc_kv_view(kv, (size_t)source, position + 1, &keys, &values, &width, NULL); /* :407 */
    if (!rc) {
        size_t lo, hi;                                                       /* :408 */
        if (global) { lo = 0; hi = position + 1; }
        else orc_windowed_len(position + 1, (size_t)hp->sliding_window, &lo, &hi);
        /* model.rs:352-353: attend concatenates the windowed rows into fresh
         * buffers on every call; the copy is part of the reference's cost. */
        size_t n = (hi - lo) * width;
        float *kc = malloc((n ? n : 1) * sizeof(float)), *vc = malloc((n ? n : 1) * sizeof(float));
        memcpy(kc, keys + lo * width, n * sizeof(float));
        memcpy(vc, values + lo * width, n * sizeof(float));
        rc = orc_attend(q, kc, vc, hi - lo, nh, nkv, hd, 1.0f, out);         /* :410 */
        free(kc);
        free(vc);
    }
    free(q);
    return rc;
}

/* Token-at-a-time prefill attention over T positions of one KV head:
 * position t attends keys [max(0, t+1-window), t] (window 0 = global),
 * each position one call of the reference's attend. */
int orc_prefill_attend(const float *q, const float *k, const float *v, size_t T, size_t n_heads,
                       size_t head_dim, size_t window, float *out) {
    for (size_t t = 0; t < T; t++) {
        size_t lo = 0, hi = t + 1;
        if (window) orc_windowed_len(t + 1, window, &lo, &hi);
        int rc = orc_attend(q + t * n_heads * head_dim, k + lo * head_dim, v + lo * head_dim,
                            hi - lo, n_heads, 1, head_dim, 1.0f, out + t * n_heads * head_dim);
        if (rc) return rc;
    }
    return ORC_OK;
}

/* ------------------------------------------------------------------------ */
/* Q8_0 mat-vec: crates/llm-backend-cpu/src/matvec.rs                         */
/* ------------------------------------------------------------------------ */

#define Q8_BLOCK 32       /* matvec.rs:15 Q8_0_BLOCK_VALUES */
#define Q8_BLOCK_BYTES 34 /* matvec.rs:16 Q8_0_BLOCK_BYTES */
#define MATVEC_PARALLEL_MIN_WORK ((size_t)1 << 20) /* matvec.rs:223 */

/* f32 -> i8 as Rust's `as i8` does: saturating, NaN -> 0. */
static int8_t sat_i8(float v) {
    if (v != v) return 0;
    if (v >= 127.0f) return 127;
    if (v <= -128.0f) return -128;
    return (int8_t)v;
}

static float f16_le(const uint8_t *b) {
    uint16_t bits = (uint16_t)(b[0] | (b[1] << 8));
    _Float16 h;
    memcpy(&h, &bits, 2);
    return (float)h;
}

/* matvec.rs:36-54 quantize_q8_0: per 32 values, scale = max|x| / 127 (f32),
 * inverse = 1 / scale (0 for a zero scale), stored scale rounded to f16,
 * quants = round_ties_even(x * inverse) cast to i8. */
int orc_quantize_q8_0(const float *x, size_t n, float *scales, int8_t *quants) {
    if (n % Q8_BLOCK) return ORC_COMPUTE;
    for (size_t b = 0; b < n / Q8_BLOCK; b++) {
        const float *blk = x + b * Q8_BLOCK;
        float max = 0.0f;
        for (int i = 0; i < Q8_BLOCK; i++) max = fmaxf(max, fabsf(blk[i]));
        float scale = max / 127.0f;
        float inverse = scale == 0.0f ? 0.0f : 1.0f / scale;
        scales[b] = (float)(_Float16)scale;
        for (int i = 0; i < Q8_BLOCK; i++) quants[b * Q8_BLOCK + i] = sat_i8(rintf(blk[i] * inverse));
    }
    return ORC_OK;
}

/* matvec.rs:137-150 dot_q8_0: integer dot per block, times (w_scale *
 * x_scale), summed over blocks in order. Rust's f32 `Sum` starts from -0.0. */
static float dot_q8_0(const uint8_t *row, size_t nb, const float *scales, const int8_t *quants) {
    float sum = -0.0f;
    for (size_t b = 0; b < nb; b++) {
        const uint8_t *blk = row + b * Q8_BLOCK_BYTES;
        float ws = f16_le(blk);
        int32_t dot = 0;
        for (int i = 0; i < Q8_BLOCK; i++) dot += (int32_t)(int8_t)blk[2 + i] * (int32_t)quants[b * Q8_BLOCK + i];
        sum = sum + (float)dot * (ws * scales[b]);
    }
    return sum;
}

/* ops.rs:85-89 gelu_tanh, evaluated left to right without fused multiply-adds. */
float orc_gelu_tanh(float x) {
    const float sqrt_2_over_pi = 0.7978846f, coef_a = 0.044715f;
    return 0.5f * x * (1.0f + tanhf(sqrt_2_over_pi * x * (1.0f + coef_a * x * x)));
}

/* ops.rs:79-81 softcap: tanh(value / cap) * cap, with the division as a
 * multiplication by the reciprocal. */
float orc_softcap(float v, float cap) { return tanhf(v * (1.0f / cap)) * cap; }

typedef struct {
    const uint8_t *w, *w2;
    size_t cols;
    const float *scales;
    const int8_t *quants;
    float cap;
    int kind; /* 0 matvec, 1 geglu, 2 softcap */
    float *out;
} q8_job;

static void q8_rows(void *c, size_t lo, size_t hi) {
    const q8_job *j = (const q8_job *)c;
    const size_t nb = j->cols / Q8_BLOCK, row_len = nb * Q8_BLOCK_BYTES;
    for (size_t r = lo; r < hi; r++) {
        float v = dot_q8_0(j->w + r * row_len, nb, j->scales, j->quants);
        if (j->kind == 1) v = orc_gelu_tanh(v) * dot_q8_0(j->w2 + r * row_len, nb, j->scales, j->quants);
        else if (j->kind == 2) v = orc_softcap(v, j->cap);
        j->out[r] = v;
    }
}

/* matvec.rs:58-63 / :88-103 / :67-80, rows split over the pool.rs workers
 * above 2^20 multiply-adds (matvec.rs:223), as map_rows / map_indices do. */
static int q8_run(const uint8_t *w, const uint8_t *w2, size_t rows, size_t cols, const float *scales,
                  const int8_t *quants, float cap, int kind, float *out) {
    if (cols % Q8_BLOCK || !w || (kind == 1 && !w2)) return ORC_COMPUTE;
    q8_job j = {w, w2, cols, scales, quants, cap, kind, out};
    run_chunks(rows, kind == 1 ? 2 * cols : cols, MATVEC_PARALLEL_MIN_WORK, q8_rows, &j);
    return ORC_OK;
}

int orc_matvec_q8_0(const uint8_t *w, size_t rows, size_t cols, const float *scales, const int8_t *quants,
                    float *out) {
    return q8_run(w, NULL, rows, cols, scales, quants, 0.0f, 0, out);
}
int orc_geglu_q8_0(const uint8_t *gate, const uint8_t *up, size_t rows, size_t cols, const float *scales,
                   const int8_t *quants, float *out) {
    return q8_run(gate, up, rows, cols, scales, quants, 0.0f, 1, out);
}
int orc_matvec_q8_0_softcap(const uint8_t *w, size_t rows, size_t cols, const float *scales,
                            const int8_t *quants, float cap, float *out) {
    return q8_run(w, NULL, rows, cols, scales, quants, cap, 2, out);
}

/* dequant.rs:13-24 */
int orc_dequant_q8_0(const uint8_t *bytes, size_t n_bytes, float *out) {
    if (n_bytes % Q8_BLOCK_BYTES) return ORC_COMPUTE;
    for (size_t b = 0; b < n_bytes / Q8_BLOCK_BYTES; b++) {
        const uint8_t *blk = bytes + b * Q8_BLOCK_BYTES;
        float scale = f16_le(blk);
        for (int i = 0; i < Q8_BLOCK; i++) out[b * Q8_BLOCK + i] = (float)(int8_t)blk[2 + i] * scale;
    }
    return ORC_OK;
}

/* tests/matvec.rs:10-18 values(): an LCG, top 24 bits mapped to [-1, 1). */
void orc_test_values(uint64_t seed, size_t len, float *out) {
    uint64_t state = seed;
    for (size_t i = 0; i < len; i++) {
        state = state * 6364136223846793005ull + 1ull;
        out[i] = (float)(state >> 40) / (float)(1u << 23) - 1.0f;
    }
}

/* tests/matvec.rs:21-31 q8_0_bytes(): scale = max|w| / 127, bytes of its f16,
 * then round-half-away(w / scale) cast to i8. */
void orc_test_q8_0_bytes(const float *w, size_t n, uint8_t *out) {
    for (size_t b = 0; b < n / Q8_BLOCK; b++) {
        const float *blk = w + b * Q8_BLOCK;
        float max = 0.0f;
        for (int i = 0; i < Q8_BLOCK; i++) max = fmaxf(max, fabsf(blk[i]));
        float scale = max / 127.0f;
        _Float16 h = (_Float16)scale;
        uint16_t bits;
        memcpy(&bits, &h, 2);
        uint8_t *o = out + b * Q8_BLOCK_BYTES;
        o[0] = (uint8_t)(bits & 0xff);
        o[1] = (uint8_t)(bits >> 8);
        for (int i = 0; i < Q8_BLOCK; i++) o[2 + i] = (uint8_t)sat_i8(roundf(blk[i] / scale));
    }
}

/* ------------------------------------------------------------------------ */
/* E2B decoder, one token: crates/llm-gemma4/src/impl_/model.rs:252-449       */
/* ------------------------------------------------------------------------ */

/* model.rs:208-216 project() with the default numerics: W @ quantize_q8_0(x). */
static int dec_project(const uint8_t *w, size_t rows, const float *x, size_t cols, float *out) {
    float *s = malloc((cols / Q8_BLOCK) * sizeof(float));
    int8_t *q = malloc(cols);
    int rc = orc_quantize_q8_0(x, cols, s, q);
    if (!rc) rc = orc_matvec_q8_0(w, rows, cols, s, q, out);
    free(s);
    free(q);
    return rc;
}

/* dequant of row `index` of a [rows][cols] Q8_0 matrix (model.rs:196-200) */
static void dec_row(const uint8_t *w, size_t index, size_t cols, float *out) {
    size_t row_bytes = cols / Q8_BLOCK * Q8_BLOCK_BYTES;
    orc_dequant_q8_0(w + index * row_bytes, row_bytes, out);
}

int32_t orc_argmax_total(const float *x, size_t n) {
    size_t best = 0;
    for (size_t i = 1; i < n; i++)
        if (total_key(x[i]) >= total_key(x[best])) best = i; /* max_by keeps the last maximum */
    return (int32_t)best;
}

int orc_dec_forward(orc_kv *kv, const orc_hparams *hp, const orc_dec_w *w, int32_t token, size_t position,
                    float *logits) {
    const size_t d = (size_t)w->d_model, ple = (size_t)w->ple_dim, L = (size_t)hp->n_layers;
    const float eps = hp->rms_norm_eps;
    if (token < 0 || token >= w->vocab) return ORC_COMPUTE;
    int rc = ORC_OK;
    /* embed (model.rs:376-384): the token's row times sqrt(d_model) */
    float *x = malloc(d * sizeof(float));
    dec_row(w->token_embd, (size_t)token, d, x);
    const float scale = sqrtf((float)d);
    for (size_t i = 0; i < d; i++) x[i] = x[i] * scale;
    /* per_layer_inputs (model.rs:252-270) */
    const size_t width = L * ple;
    float *pli = malloc((width ? width : 1) * sizeof(float));
    if (ple) {
        float *projected = malloc(width * sizeof(float)), *table = malloc(width * sizeof(float));
        float *scaled = malloc(ple * sizeof(float)), *normed = malloc(ple * sizeof(float));
        rc = dec_project(w->ple_model_proj, width, x, d, projected);
        dec_row(w->ple_token_embd, (size_t)token, width, table);
        const float projection_scale = 1.0f / sqrtf((float)d);
        const float table_scale = sqrtf((float)ple);
        const float input_scale = 1.0f / sqrtf(2.0f);
        for (size_t l = 0; l < L && !rc; l++) {
            for (size_t i = 0; i < ple; i++) scaled[i] = projected[l * ple + i] * projection_scale;
            rc = orc_rms_norm(scaled, ple, w->ple_proj_norm, eps, normed);
            for (size_t i = 0; i < ple; i++) pli[l * ple + i] = (normed[i] + table[l * ple + i] * table_scale) * input_scale;
        }
        free(projected); free(table); free(scaled); free(normed);
    }
    const size_t qmax = (size_t)hp->n_heads * (size_t)hp->head_dim_global;
    float *normalized = malloc(d * sizeof(float)), *q = malloc(qmax * sizeof(float));
    float *k = malloc((size_t)hp->head_dim_global * sizeof(float)), *v = malloc((size_t)hp->head_dim_global * sizeof(float));
    float *att = malloc(qmax * sizeof(float)), *proj = malloc(d * sizeof(float)), *tmp = malloc(d * sizeof(float));
    float *gated = malloc((size_t)w->d_ff * sizeof(float)), *gate = malloc((ple ? ple : 1) * sizeof(float));
    for (size_t l = 0; l < L && !rc; l++) {
        const orc_dec_layer_w *lw = &w->layers[l];
        const size_t hd = (size_t)orc_head_dim(hp, (int32_t)l), qd = (size_t)hp->n_heads * hd;
        int32_t source = -1;
        rc = orc_kv_source_layer(hp, (int32_t)l, &source, NULL);
        if (rc) break;
        rc = orc_rms_norm(x, d, lw->attn_norm, eps, normalized);                       /* :392 */
        if (!rc) rc = dec_project(lw->attn_q, qd, normalized, d, q);                    /* :393 */
        if (!rc && source == (int32_t)l) {                                              /* :399-401 */
            rc = dec_project(lw->attn_k, hd, normalized, d, k);
            if (!rc) rc = dec_project(lw->attn_v, hd, normalized, d, v);
        }
        /* :394-396, :402-410: norms, RoPE, append, view, window, attend */
        if (!rc) rc = orc_attention_block(kv, hp, (int32_t)l, position, q, k, v, lw->attn_q_norm, lw->attn_k_norm,
                                          w->rope_freqs, 0, att);
        if (!rc) rc = dec_project(lw->attn_output, d, att, qd, proj);                  /* :411 */
        if (!rc) rc = orc_rms_norm(proj, d, lw->post_attention_norm, eps, tmp);        /* :412 */
        for (size_t i = 0; i < d; i++) x[i] = x[i] + tmp[i];                            /* :413 residual */
        if (!rc) rc = orc_rms_norm(x, d, lw->ffn_norm, eps, normalized);               /* :415 */
        if (!rc) {                                                                      /* :416-417 */
            float *s = malloc((d / Q8_BLOCK) * sizeof(float));
            int8_t *qq = malloc(d);
            rc = orc_quantize_q8_0(normalized, d, s, qq);
            if (!rc) rc = orc_geglu_q8_0(lw->ffn_gate, lw->ffn_up, (size_t)w->d_ff, d, s, qq, gated);
            free(s);
            free(qq);
        }
        if (!rc) rc = dec_project(lw->ffn_down, d, gated, (size_t)w->d_ff, proj);     /* :418 */
        if (!rc) rc = orc_rms_norm(proj, d, lw->post_ffw_norm, eps, tmp);              /* :419 */
        for (size_t i = 0; i < d; i++) x[i] = x[i] + tmp[i];                            /* :420 */
        if (!rc && ple) {                                                               /* :422-432 */
            rc = dec_project(lw->inp_gate, ple, x, d, gate);
            for (size_t i = 0; i < ple; i++) gate[i] = orc_gelu_tanh(gate[i]) * pli[l * ple + i];
            if (!rc) rc = dec_project(lw->proj, d, gate, ple, proj);
            if (!rc) rc = orc_rms_norm(proj, d, lw->post_norm, eps, tmp);
            for (size_t i = 0; i < d; i++) x[i] = x[i] + tmp[i];
        }
        if (lw->layer_output_scale != 1.0f)                                            /* :433-435 */
            for (size_t i = 0; i < d; i++) x[i] = x[i] * lw->layer_output_scale;
    }
    /* logits (model.rs:438-449): output norm, tied head, soft-cap */
    if (!rc) rc = orc_rms_norm(x, d, w->output_norm, eps, normalized);
    if (!rc) {
        float *s = malloc((d / Q8_BLOCK) * sizeof(float));
        int8_t *qq = malloc(d);
        rc = orc_quantize_q8_0(normalized, d, s, qq);
        if (!rc) rc = orc_matvec_q8_0_softcap(w->token_embd, (size_t)w->vocab, d, s, qq, w->final_logit_softcap, logits);
        free(s);
        free(qq);
    }
    free(x); free(pli); free(normalized); free(q); free(k); free(v); free(att); free(proj); free(tmp); free(gated);
    free(gate);
    return rc;
}
