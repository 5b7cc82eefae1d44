/* CPU oracle (test infrastructure only): see azoracle.h for what it restates
 * and why. Compile with -ffp-contract=off and no -march flag, as the
 * reference's Release build has no FMA either (CMakeLists.txt:8-10), so that
 * a * b + c stays two roundings exactly as in src/backend.cpp:135. */
#include "azoracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ rng */

static uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

/* src/rng.cpp:19-25 */
uint64_t az_splitmix64(uint64_t* x) {
    uint64_t z = (*x += 0x9E3779B97F4A7C15ULL);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* src/rng.cpp:27-37: fold a, b, c, d in order, mixing after each. */
uint64_t az_derive_seed(uint64_t a, uint64_t b, uint64_t c, uint64_t d) {
    const uint64_t in[4] = {a, b, c, d};
    uint64_t h = 0x243F6A8885A308D3ULL;
    for (int i = 0; i < 4; ++i) {
        uint64_t x = h ^ in[i];
        h = az_splitmix64(&x);
    }
    return h;
}

/* src/rng.cpp:39-44 */
void az_rng_seed(az_rng* r, uint64_t seed) {
    uint64_t x = seed;
    for (int i = 0; i < 4; ++i) r->s[i] = az_splitmix64(&x);
}

/* xoshiro256** (Blackman & Vigna 2018), src/rng.cpp:46-57 */
uint64_t az_rng_next(az_rng* r) {
    uint64_t* s = r->s;
    const uint64_t result = rotl64(s[1] * 5, 7) * 9;
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl64(s[3], 45);
    return result;
}

/* src/rng.cpp:59-62: top 53 bits over 2^53 */
double az_rng_uniform(az_rng* r) { return (double)(az_rng_next(r) >> 11) * 0x1.0p-53; }

/* Lemire multiply-shift with rejection, src/rng.cpp:64-80 */
int az_rng_below(az_rng* r, int n) {
    const uint32_t range = (uint32_t)n;
    uint64_t m = (az_rng_next(r) >> 32) * range;
    uint32_t low = (uint32_t)m;
    if (low < range) {
        const uint32_t threshold = (0u - range) % range;
        while (low < threshold) {
            m = (az_rng_next(r) >> 32) * range;
            low = (uint32_t)m;
        }
    }
    return (int)(m >> 32);
}

/* Box-Muller without a cached second value, src/rng.cpp:82-86 */
double az_rng_normal(az_rng* r) {
    const double two_pi = 6.283185307179586476925286766559;
    const double u1 = 1.0 - az_rng_uniform(r);
    const double u2 = az_rng_uniform(r);
    return sqrt(-2.0 * log(u1)) * cos(two_pi * u2);
}

/* --------------------------------------------------------------- layout */

enum { KIND_CONV_W, KIND_BN_GAMMA, KIND_BN_BETA, KIND_FC_W, KIND_FC_B, KIND_BN_MEAN, KIND_BN_VAR };

typedef struct entry {
    char name[48];
    size_t size, offset;
    int kind, decay;
    int fan_in; /* He-normal fan-in for weights */
} entry;

typedef struct layout {
    entry* params;
    entry* buffers;
    int nparams, nbuffers;
    size_t param_floats, buffer_floats;
} layout;

static size_t align64(size_t f) { return (f + 63) / 64 * 64; }

static void push(entry* list, int* n, size_t* floats, const char* name, size_t size, int kind,
                 int decay, int fan_in) {
    entry* e = &list[(*n)++];
    snprintf(e->name, sizeof e->name, "%s", name);
    e->size = size;
    e->offset = *floats;
    e->kind = kind;
    e->decay = decay;
    e->fan_in = fan_in;
    *floats = align64(*floats + size);
}

/* Network::params() / buffers() order (src/network.cpp:113-165) with
 * ParamLayout's 64-float offsets (src/param_layout.cpp:18-29). */
static layout make_layout(const az_netcfg* c) {
    layout L;
    const int cap = 32 + 8 * c->blocks;
    L.params = (entry*)calloc((size_t)cap, sizeof(entry));
    L.buffers = (entry*)calloc((size_t)cap, sizeof(entry));
    L.nparams = L.nbuffers = 0;
    L.param_floats = L.buffer_floats = 0;
    const int F = c->filters, P = 2 * c->history + 2, A = c->board * c->board, V = c->value_hidden;
    char name[48];
#define PARAM(nm, sz, kind, decay, fan) push(L.params, &L.nparams, &L.param_floats, nm, sz, kind, decay, fan)
#define BUF(nm, sz, kind) push(L.buffers, &L.nbuffers, &L.buffer_floats, nm, sz, kind, 0, 0)
#define BN_PARAMS(prefix, ch)                                                    \
    do {                                                                         \
        snprintf(name, sizeof name, "%s.gamma", prefix);                         \
        PARAM(name, (size_t)(ch), KIND_BN_GAMMA, 0, 0);                          \
        snprintf(name, sizeof name, "%s.beta", prefix);                          \
        PARAM(name, (size_t)(ch), KIND_BN_BETA, 0, 0);                           \
    } while (0)
#define BN_BUFS(prefix, ch)                                                      \
    do {                                                                         \
        snprintf(name, sizeof name, "%s.runMean", prefix);                       \
        BUF(name, (size_t)(ch), KIND_BN_MEAN);                                   \
        snprintf(name, sizeof name, "%s.runVar", prefix);                        \
        BUF(name, (size_t)(ch), KIND_BN_VAR);                                    \
    } while (0)
    PARAM("stem.conv.w", (size_t)F * P * 9, KIND_CONV_W, 1, P * 9);
    BN_PARAMS("stem.bn", F);
    for (int i = 0; i < c->blocks; ++i) {
        char pre[40];
        snprintf(pre, sizeof pre, "block%d.conv1.w", i);
        PARAM(pre, (size_t)F * F * 9, KIND_CONV_W, 1, F * 9);
        snprintf(pre, sizeof pre, "block%d.bn1", i);
        BN_PARAMS(pre, F);
        snprintf(pre, sizeof pre, "block%d.conv2.w", i);
        PARAM(pre, (size_t)F * F * 9, KIND_CONV_W, 1, F * 9);
        snprintf(pre, sizeof pre, "block%d.bn2", i);
        BN_PARAMS(pre, F);
    }
    PARAM("policy.conv.w", (size_t)2 * F, KIND_CONV_W, 1, F);
    BN_PARAMS("policy.bn", 2);
    PARAM("policy.fc.w", (size_t)(A + 1) * 2 * A, KIND_FC_W, 1, 2 * A);
    PARAM("policy.fc.b", (size_t)(A + 1), KIND_FC_B, 0, 0);
    PARAM("value.conv.w", (size_t)F, KIND_CONV_W, 1, F);
    BN_PARAMS("value.bn", 1);
    PARAM("value.fc1.w", (size_t)V * A, KIND_FC_W, 1, A);
    PARAM("value.fc1.b", (size_t)V, KIND_FC_B, 0, 0);
    PARAM("value.fc2.w", (size_t)V, KIND_FC_W, 1, V);
    PARAM("value.fc2.b", 1, KIND_FC_B, 0, 0);
    if (c->ownership) {
        PARAM("ownership.conv.w", (size_t)F, KIND_CONV_W, 1, F);
        BN_PARAMS("ownership.bn", 1);
    }
    BN_BUFS("stem.bn", F);
    for (int i = 0; i < c->blocks; ++i) {
        char pre[40];
        snprintf(pre, sizeof pre, "block%d.bn1", i);
        BN_BUFS(pre, F);
        snprintf(pre, sizeof pre, "block%d.bn2", i);
        BN_BUFS(pre, F);
    }
    BN_BUFS("policy.bn", 2);
    BN_BUFS("value.bn", 1);
    if (c->ownership) BN_BUFS("ownership.bn", 1);
#undef PARAM
#undef BUF
#undef BN_PARAMS
#undef BN_BUFS
    return L;
}

static void free_layout(layout* L) {
    free(L->params);
    free(L->buffers);
}

static const entry* find(const layout* L, const char* name) {
    for (int i = 0; i < L->nparams; ++i)
        if (!strcmp(L->params[i].name, name)) return &L->params[i];
    for (int i = 0; i < L->nbuffers; ++i)
        if (!strcmp(L->buffers[i].name, name)) return &L->buffers[i];
    return NULL;
}

int az_layout_count(const az_netcfg* cfg, int which) {
    layout L = make_layout(cfg);
    const int n = which == 0 ? L.nparams : L.nbuffers;
    free_layout(&L);
    return n;
}

int az_layout_entry(const az_netcfg* cfg, int which, int index, char* name, size_t name_cap,
                    size_t* size, size_t* offset, int* decay) {
    layout L = make_layout(cfg);
    const int n = which == 0 ? L.nparams : L.nbuffers;
    int ok = index >= 0 && index < n;
    if (ok) {
        const entry* e = which == 0 ? &L.params[index] : &L.buffers[index];
        if (name && name_cap) snprintf(name, name_cap, "%s", e->name);
        if (size) *size = e->size;
        if (offset) *offset = e->offset;
        if (decay) *decay = e->decay;
    }
    free_layout(&L);
    return ok ? 0 : -1;
}

size_t az_layout_floats(const az_netcfg* cfg, int which) {
    layout L = make_layout(cfg);
    const size_t n = which == 0 ? L.param_floats : L.buffer_floats;
    free_layout(&L);
    return n;
}

/* ------------------------------------------------------------- networks */

/* Network(cfg, seed): src/network.cpp:77-111. One generator; He-normal
 * weights (stddev sqrt(2/fanIn) in double, src/layers.cpp:14-17) drawn in
 * init order: stem conv, each block's conv1 then conv2, policy conv, policy
 * fc, value conv, value fc1, value fc2, then the ownership conv. That is
 * params() order restricted to weights, which make_layout lists in. Linear
 * biases are zero (src/layers.cpp:164-167); BN gamma 1, beta 0
 * (src/layers.cpp:79-81), running mean 0 and variance 1. */
void az_network_init(const az_netcfg* cfg, uint64_t seed, float* params, float* buffers) {
    layout L = make_layout(cfg);
    memset(params, 0, L.param_floats * sizeof(float));
    memset(buffers, 0, L.buffer_floats * sizeof(float));
    az_rng rng;
    az_rng_seed(&rng, seed);
    /* The ownership conv is drawn last (src/network.cpp:108-110), after the
     * value head, although params() lists it after value.fc2 as well. */
    for (int i = 0; i < L.nparams; ++i) {
        const entry* e = &L.params[i];
        float* v = params + e->offset;
        if (e->kind == KIND_CONV_W || e->kind == KIND_FC_W) {
            const double stddev = sqrt(2.0 / e->fan_in);
            for (size_t j = 0; j < e->size; ++j) v[j] = (float)(az_rng_normal(&rng) * stddev);
        } else if (e->kind == KIND_BN_GAMMA) {
            for (size_t j = 0; j < e->size; ++j) v[j] = 1.0f;
        }
    }
    for (int i = 0; i < L.nbuffers; ++i) {
        const entry* e = &L.buffers[i];
        if (e->kind == KIND_BN_VAR)
            for (size_t j = 0; j < e->size; ++j) buffers[e->offset + j] = 1.0f;
    }
    free_layout(&L);
}

void az_randomize(const az_netcfg* cfg, int kind, uint64_t seed, float* params, float* buffers) {
    layout L = make_layout(cfg);
    az_rng rng;
    az_rng_seed(&rng, kind == 0 ? az_derive_seed(seed, 1, 0, 0) : seed + 17);
    for (int i = 0; i < L.nparams; ++i) {
        const entry* e = &L.params[i];
        float* v = params + e->offset;
        if (e->kind == KIND_BN_GAMMA) {
            for (size_t j = 0; j < e->size; ++j) v[j] = (float)(0.5 + az_rng_uniform(&rng));
        } else if (!e->decay) { /* beta, and linear biases */
            if (kind == 0) {
                if (e->kind == KIND_BN_BETA)
                    for (size_t j = 0; j < e->size; ++j) v[j] = (float)(0.1 * az_rng_normal(&rng));
            } else {
                for (size_t j = 0; j < e->size; ++j) v[j] = (float)(0.4 * az_rng_uniform(&rng) - 0.2);
            }
        }
    }
    for (int i = 0; i < L.nbuffers; ++i) {
        const entry* e = &L.buffers[i];
        float* v = buffers + e->offset;
        const int var = e->kind == KIND_BN_VAR;
        for (size_t j = 0; j < e->size; ++j) {
            if (var) v[j] = (float)(0.5 + az_rng_uniform(&rng));
            else v[j] = kind == 0 ? (float)(0.1 * az_rng_normal(&rng)) : (float)(0.4 * az_rng_uniform(&rng) - 0.2);
        }
    }
    free_layout(&L);
}

/* ---------------------------------------------------------------- inputs */

/* Planes as encodePlanes writes them for one history position and no
 * symmetry (src/encode.cpp:14-43): plane 0 own stones, plane 1 the
 * opponent's, planes 2..2H-1 zero, plane 2H all ones when Black moves,
 * plane 2H+1 all ones when White moves. */
void az_inputs_positions(const az_netcfg* cfg, uint64_t seed, long first, int B, float* out) {
    const int A = cfg->board * cfg->board, H = cfg->history, P = 2 * H + 2;
    for (int b = 0; b < B; ++b) {
        az_rng rng;
        az_rng_seed(&rng, az_derive_seed(seed, 2, (uint64_t)(first + b), 0));
        float* x = out + (size_t)b * P * A;
        memset(x, 0, (size_t)P * A * sizeof(float));
        const int to_move = az_rng_below(&rng, 2); /* 0 black, 1 white */
        for (int p = 0; p < A; ++p) {
            if (az_rng_uniform(&rng) < 0.4) {
                const int colour = az_rng_below(&rng, 2);
                x[(size_t)(colour == to_move ? 0 : 1) * A + p] = 1.0f;
            }
        }
        float* plane = x + (size_t)(2 * H + to_move) * A;
        for (int p = 0; p < A; ++p) plane[p] = 1.0f;
    }
}

void az_inputs_planes(uint64_t seed, size_t count, float* out) {
    az_rng rng;
    az_rng_seed(&rng, seed);
    for (size_t i = 0; i < count; ++i) out[i] = (float)az_rng_below(&rng, 2);
}

/* --------------------------------------------------------- float forward */

static const float* P_(const layout* L, const float* params, const float* buffers, const char* name) {
    const entry* e = find(L, name);
    if (!e) {
        fprintf(stderr, "azoracle: no tensor %s\n", name);
        abort();
    }
    const int is_param = e >= L->params && e < L->params + L->nparams;
    return (is_param ? params : buffers) + e->offset;
}

/* Conv2d::forward with k = 3 (src/layers.cpp:35-46): y [cout][M] = w
 * [cout][cin*9] . im2col(x) with x [cin][B][n][n]; each output is the float
 * sum over k = (ci*3 + dy)*3 + dx ascending of w*col, col 0 off the board
 * (src/backend.cpp:21-55), accumulated from +0 as gemmRows does
 * (src/backend.cpp:115-140). */
static void conv3_f32(const float* x, int cin, int cout, int B, int n, const float* w, float* y, int threads) {
    const int A = n * n;
    const size_t M = (size_t)B * A;
    (void)threads;
#pragma omp parallel for num_threads(threads) schedule(static)
    for (int co = 0; co < cout; ++co) {
        const float* wr = w + (size_t)co * cin * 9;
        float* yr = y + (size_t)co * M;
        for (int b = 0; b < B; ++b)
            for (int py = 0; py < n; ++py)
                for (int px = 0; px < n; ++px) {
                    float acc = 0.0f;
                    for (int ci = 0; ci < cin; ++ci) {
                        const float* xc = x + ((size_t)ci * B + b) * A;
                        for (int dy = 0; dy < 3; ++dy)
                            for (int dx = 0; dx < 3; ++dx) {
                                const int sy = py + dy - 1, sx = px + dx - 1;
                                const float v = (sy < 0 || sy >= n || sx < 0 || sx >= n) ? 0.0f : xc[sy * n + sx];
                                const float prod = wr[(ci * 3 + dy) * 3 + dx] * v;
                                acc = acc + prod;
                            }
                    }
                    yr[(size_t)b * A + py * n + px] = acc;
                }
    }
}

/* A 1x1 conv: y [cout][M] = w [cout][cin] . x [cin][M], k ascending. */
static void conv1_f32(const float* x, int cin, int cout, size_t M, const float* w, float* y) {
    for (int co = 0; co < cout; ++co)
        for (size_t m = 0; m < M; ++m) {
            float acc = 0.0f;
            for (int ci = 0; ci < cin; ++ci) {
                const float prod = w[(size_t)co * cin + ci] * x[(size_t)ci * M + m];
                acc = acc + prod;
            }
            y[(size_t)co * M + m] = acc;
        }
}

/* BatchNorm2d::forwardInfer (src/layers.cpp:88-97): scale = gamma/sqrt(var+eps),
 * shift = beta - scale*mean, y = scale*x + shift, all in float. */
static void bn_f32(float* x, int C, size_t M, const float* gamma, const float* beta, const float* mean,
                   const float* var) {
    for (int c = 0; c < C; ++c) {
        const float scale = gamma[c] / sqrtf(var[c] + 1e-5f);
        const float prod = scale * mean[c];
        const float shift = beta[c] - prod;
        float* xc = x + (size_t)c * M;
        for (size_t i = 0; i < M; ++i) {
            const float s = scale * xc[i];
            xc[i] = s + shift;
        }
    }
}

/* reluForward (src/layers.cpp:191-195): x > 0 ? x : 0 (-0 and NaN to +0). */
static void relu_f32(float* x, size_t count) {
    for (size_t i = 0; i < count; ++i) x[i] = x[i] > 0.0f ? x[i] : 0.0f;
}

/* Linear::forward (src/layers.cpp:169-176): y [B][out] = x [B][in] . w^T,
 * the sum over in ascending, then + b. */
static void linear_f32(const float* x, int B, int in, int out, const float* w, const float* bias, float* y) {
    for (int s = 0; s < B; ++s)
        for (int o = 0; o < out; ++o) {
            float acc = 0.0f;
            for (int i = 0; i < in; ++i) {
                const float prod = x[(size_t)s * in + i] * w[(size_t)o * in + i];
                acc = acc + prod;
            }
            y[(size_t)s * out + o] = acc + bias[o];
        }
}

#define T(name) P_(&L, params, buffers, name)

/* Network::forward in Mode::Infer (src/network.cpp:228-309). */
void az_forward_f32(const az_netcfg* cfg, const float* params, const float* buffers, const float* input, int B,
                    float* logits, float* values, float* ownership, int threads) {
    layout L = make_layout(cfg);
    const int n = cfg->board, A = n * n, P = 2 * cfg->history + 2, F = cfg->filters, V = cfg->value_hidden;
    const size_t M = (size_t)B * A;
    if (threads < 1) threads = 1;
    float* in = (float*)malloc((size_t)P * M * sizeof(float));
    float* x = (float*)malloc((size_t)F * M * sizeof(float));
    float* mid = (float*)malloc((size_t)F * M * sizeof(float));
    float* out = (float*)malloc((size_t)F * M * sizeof(float));
    float* head = (float*)malloc(2 * M * sizeof(float));
    float* flat = (float*)malloc(2 * M * sizeof(float));
    float* hidden = (float*)malloc((size_t)B * V * sizeof(float));
    /* [B][P][A] -> [P][B][A] (src/network.cpp:239-246) */
    for (int b = 0; b < B; ++b)
        for (int p = 0; p < P; ++p)
            memcpy(in + ((size_t)p * B + b) * A, input + ((size_t)b * P + p) * A, (size_t)A * sizeof(float));
    char nm[64], bn[64];
    conv3_f32(in, P, F, B, n, T("stem.conv.w"), x, threads);
    bn_f32(x, F, M, T("stem.bn.gamma"), T("stem.bn.beta"), T("stem.bn.runMean"), T("stem.bn.runVar"));
    relu_f32(x, (size_t)F * M);
    for (int i = 0; i < cfg->blocks; ++i) {
char pre[40];
        snprintf(nm, sizeof nm, "block%d.conv1.w", i);
        conv3_f32(x, F, F, B, n, T(nm), mid, threads);
        snprintf(pre, sizeof pre, "block%d.bn1", i);
        {
            const float *g, *be, *mu, *va;
            snprintf(bn, sizeof bn, "%s.gamma", pre); g = T(bn);
            snprintf(bn, sizeof bn, "%s.beta", pre); be = T(bn);
            snprintf(bn, sizeof bn, "%s.runMean", pre); mu = T(bn);
            snprintf(bn, sizeof bn, "%s.runVar", pre); va = T(bn);
            bn_f32(mid, F, M, g, be, mu, va);
        }
        relu_f32(mid, (size_t)F * M);
        snprintf(nm, sizeof nm, "block%d.conv2.w", i);
        conv3_f32(mid, F, F, B, n, T(nm), out, threads);
        snprintf(pre, sizeof pre, "block%d.bn2", i);
        {
            const float *g, *be, *mu, *va;
            snprintf(bn, sizeof bn, "%s.gamma", pre); g = T(bn);
            snprintf(bn, sizeof bn, "%s.beta", pre); be = T(bn);
            snprintf(bn, sizeof bn, "%s.runMean", pre); mu = T(bn);
            snprintf(bn, sizeof bn, "%s.runVar", pre); va = T(bn);
            bn_f32(out, F, M, g, be, mu, va);
        }
        /* the skip, then ReLU (src/network.cpp:269-270) */
        for (size_t j = 0; j < (size_t)F * M; ++j) out[j] = out[j] + x[j];
        relu_f32(out, (size_t)F * M);
        float* t = x;
        x = out;
        out = t;
    }
    /* policy head (src/network.cpp:274-286) */
    conv1_f32(x, F, 2, M, T("policy.conv.w"), head);
    bn_f32(head, 2, M, T("policy.bn.gamma"), T("policy.bn.beta"), T("policy.bn.runMean"), T("policy.bn.runVar"));
    relu_f32(head, 2 * M);
    for (int b = 0; b < B; ++b)
        for (int c = 0; c < 2; ++c)
            memcpy(flat + (size_t)b * 2 * A + (size_t)c * A, head + ((size_t)c * B + b) * A, (size_t)A * sizeof(float));
    linear_f32(flat, B, 2 * A, A + 1, T("policy.fc.w"), T("policy.fc.b"), logits);
    /* value head (src/network.cpp:288-296) */
    conv1_f32(x, F, 1, M, T("value.conv.w"), head);
    bn_f32(head, 1, M, T("value.bn.gamma"), T("value.bn.beta"), T("value.bn.runMean"), T("value.bn.runVar"));
    relu_f32(head, M);
    linear_f32(head, B, A, V, T("value.fc1.w"), T("value.fc1.b"), hidden);
    relu_f32(hidden, (size_t)B * V);
    linear_f32(hidden, B, V, 1, T("value.fc2.w"), T("value.fc2.b"), values);
    for (int b = 0; b < B; ++b) values[b] = tanhf(values[b]);
    /* ownership head (src/network.cpp:301-308) */
    if (cfg->ownership && ownership) {
        conv1_f32(x, F, 1, M, T("ownership.conv.w"), head);
        bn_f32(head, 1, M, T("ownership.bn.gamma"), T("ownership.bn.beta"), T("ownership.bn.runMean"),
               T("ownership.bn.runVar"));
        for (size_t j = 0; j < M; ++j) ownership[j] = tanhf(head[j]);
    }
    free(in);
    free(x);
    free(mid);
    free(out);
    free(head);
    free(flat);
    free(hidden);
    free_layout(&L);
}

/* -------------------------------------------------------- double forward */

static void conv_f64(const double* x, int cin, int cout, int k, int B, int n, const float* w, double* y,
                     int threads) {
    const int A = n * n, r = k / 2;
    (void)threads;
#pragma omp parallel for num_threads(threads) schedule(static)
    for (int co = 0; co < cout; ++co)
        for (int b = 0; b < B; ++b)
            for (int p = 0; p < A; ++p) {
                double sum = 0.0;
                for (int ci = 0; ci < cin; ++ci)
                    for (int dy = 0; dy < k; ++dy)
                        for (int dx = 0; dx < k; ++dx) {
                            const int yy = p / n + dy - r, xx = p % n + dx - r;
                            if (yy < 0 || yy >= n || xx < 0 || xx >= n) continue;
                            sum += (double)w[(((size_t)co * cin + ci) * k + dy) * k + dx] *
                                   x[((size_t)ci * B + b) * A + yy * n + xx];
                        }
                y[((size_t)co * B + b) * A + p] = sum;
            }
}

static void bn_f64(double* x, int C, size_t M, const float* g, const float* be, const float* mu, const float* va) {
    for (int c = 0; c < C; ++c) {
        const double scale = (double)g[c] / sqrt((double)va[c] + (double)1e-5f);
        for (size_t i = 0; i < M; ++i) {
            double* v = &x[(size_t)c * M + i];
            *v = (*v - mu[c]) * scale + be[c];
        }
    }
}

static void relu_f64(double* x, size_t count) {
    for (size_t i = 0; i < count; ++i) x[i] = x[i] > 0.0 ? x[i] : 0.0;
}

static void linear_f64(const double* x, int B, int in, int out, const float* w, const float* bias, double* y) {
    for (int s = 0; s < B; ++s)
        for (int o = 0; o < out; ++o) {
            double sum = bias[o];
            for (int i = 0; i < in; ++i) sum += x[(size_t)s * in + i] * w[(size_t)o * in + i];
            y[(size_t)s * out + o] = sum;
        }
}

/* doubleInfer (tests/test_cuda.cpp:659-752): the network from its
 * definition, every operation in double. */
void az_forward_f64(const az_netcfg* cfg, const float* params, const float* buffers, const float* input, int B,
                    float* logits, float* values, float* ownership, int threads) {
    layout L = make_layout(cfg);
    const int n = cfg->board, A = n * n, P = 2 * cfg->history + 2, F = cfg->filters, V = cfg->value_hidden;
    const size_t M = (size_t)B * A;
    if (threads < 1) threads = 1;
    double* in = (double*)malloc((size_t)P * M * sizeof(double));
    double* h = (double*)malloc((size_t)F * M * sizeof(double));
    double* mid = (double*)malloc((size_t)F * M * sizeof(double));
    double* out = (double*)malloc((size_t)F * M * sizeof(double));
    double* head = (double*)malloc(2 * M * sizeof(double));
    double* flat = (double*)malloc(2 * M * sizeof(double));
    double* hidden = (double*)malloc((size_t)B * V * sizeof(double));
    double* res = (double*)malloc((size_t)B * (A + 1) * sizeof(double));
    for (int b = 0; b < B; ++b)
        for (int p = 0; p < P; ++p)
            for (int a = 0; a < A; ++a) in[((size_t)p * B + b) * A + a] = input[((size_t)b * P + p) * A + a];
    char bn[64];
#define BN4(pre)                                                                                           \
    do {                                                                                                   \
        snprintf(bn, sizeof bn, "%s.gamma", pre); g = T(bn);                                               \
        snprintf(bn, sizeof bn, "%s.beta", pre); be = T(bn);                                               \
        snprintf(bn, sizeof bn, "%s.runMean", pre); mu = T(bn);                                            \
        snprintf(bn, sizeof bn, "%s.runVar", pre); va = T(bn);                                             \
    } while (0)
    const float *g, *be, *mu, *va;
    conv_f64(in, P, F, 3, B, n, T("stem.conv.w"), h, threads);
    BN4("stem.bn");
    bn_f64(h, F, M, g, be, mu, va);
    relu_f64(h, (size_t)F * M);
    for (int i = 0; i < cfg->blocks; ++i) {
        char nm[48], pre[40];
        snprintf(nm, sizeof nm, "block%d.conv1.w", i);
        conv_f64(h, F, F, 3, B, n, T(nm), mid, threads);
        snprintf(pre, sizeof pre, "block%d.bn1", i);
        BN4(pre);
        bn_f64(mid, F, M, g, be, mu, va);
        relu_f64(mid, (size_t)F * M);
        snprintf(nm, sizeof nm, "block%d.conv2.w", i);
        conv_f64(mid, F, F, 3, B, n, T(nm), out, threads);
        snprintf(pre, sizeof pre, "block%d.bn2", i);
        BN4(pre);
        bn_f64(out, F, M, g, be, mu, va);
        for (size_t j = 0; j < (size_t)F * M; ++j) out[j] += h[j];
        relu_f64(out, (size_t)F * M);
        double* t = h;
        h = out;
        out = t;
    }
    conv_f64(h, F, 2, 1, B, n, T("policy.conv.w"), head, 1);
    BN4("policy.bn");
    bn_f64(head, 2, M, g, be, mu, va);
    relu_f64(head, 2 * M);
    for (int c = 0; c < 2; ++c)
        for (int b = 0; b < B; ++b)
            for (int a = 0; a < A; ++a) flat[(size_t)b * 2 * A + (size_t)c * A + a] = head[((size_t)c * B + b) * A + a];
    linear_f64(flat, B, 2 * A, A + 1, T("policy.fc.w"), T("policy.fc.b"), res);
    for (size_t j = 0; j < (size_t)B * (A + 1); ++j) logits[j] = (float)res[j];
    conv_f64(h, F, 1, 1, B, n, T("value.conv.w"), head, 1);
    BN4("value.bn");
    bn_f64(head, 1, M, g, be, mu, va);
    relu_f64(head, M);
    linear_f64(head, B, A, V, T("value.fc1.w"), T("value.fc1.b"), hidden);
    relu_f64(hidden, (size_t)B * V);
    linear_f64(hidden, B, V, 1, T("value.fc2.w"), T("value.fc2.b"), res);
    for (int b = 0; b < B; ++b) values[b] = (float)tanh(res[b]);
    if (cfg->ownership && ownership) {
        conv_f64(h, F, 1, 1, B, n, T("ownership.conv.w"), head, 1);
        BN4("ownership.bn");
        bn_f64(head, 1, M, g, be, mu, va);
        for (size_t j = 0; j < M; ++j) ownership[j] = (float)tanh(head[j]);
    }
#undef BN4
    free(in);
    free(h);
    free(mid);
    free(out);
    free(head);
    free(flat);
    free(hidden);
    free(res);
    free_layout(&L);
}
#undef T
