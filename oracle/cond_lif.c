/*
 * ORACLE — test infrastructure, not product code. Only the test suite, the smoke
 * check and bench.py's CPU-baseline arm load this library, and only as the checker
 * (or the timed CPU baseline); the engine never calls it.
 *
 * A plain-C restatement of wiretorch's conductance-based LIF time loop,
 * ``wiretorch.network_simulators.conductance.dynamics.simulate``
 * (src/wiretorch/network_simulators/conductance/dynamics.py:146-237), for networks
 * whose weights are given as CSR rows per pathway. Every floating-point step follows the
 * reference's PyTorch expressions in the same order and in float32 (built with
 * -ffp-contract=off, so nothing is fused); the one deliberate difference is the
 * recurrent and feedforward activation ``pre @ W`` (network.py:260-271, 142-157), which
 * the reference leaves to a BLAS matmul: here each target's sum is accumulated in
 * double over the fired rows and rounded once.
 *
 * Per step, for every trial (trials and neurons run in parallel with OpenMP):
 *   held = counter > 0                                   network.py:294-302
 *   s    = H(v - theta) (1 - held)  [or noise < sigmoid]  dynamics.py:103-107
 *   v'   = membrane(v, max(s, held), g, g_a)             dynamics.py:116-143
 *   counter, g_a updated                                  network.py:313-318, dynamics.py:201-202
 *   a_k  = (pre_k * f_k) @ W_k  per pathway               network.py:260-271
 *   g    = g * decay + sum_k a_k (jump * scale_k * made_k) dynamics.py:206-208
 * with the presynaptic gating (short-term plasticity, saturation) of network.py:186-223.
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    int n_rows;             /* source rows of the pathway */
    const int64_t *rows;    /* (n_rows): neuron (recurrent) or input column (feedforward) */
    const int64_t *row_ptr; /* (n_rows + 1) CSR over targets */
    const int32_t *cols;    /* (E) */
    const float *w;         /* (E) weights W[row, col] */
    const float *scale;     /* (N) this pathway's kernel scale per target */
    const uint8_t *made;    /* (S) which synapse types it makes */
    int recurrent;          /* 1: rows are the network's own neurons */
    int gate;               /* 0: no presynaptic dynamics */
    int stp, saturates, start, n;
    float c, d, U, d_D, d_F; /* Gate.params */
} WtoPathway;

typedef struct {
    int B, N, S, n_in, K;
    const WtoPathway *pathways; /* recurrent first, as the reference orders them */
    /* per neuron (N) */
    const float *theta, *U_reset, *E_L, *C_m, *beta;
    const int32_t *n_ref;                       /* NULL: no refractory period */
    const float *adapt, *adapt_decay, *E_adapt; /* NULL: no adaptation */
    /* per synapse type (S); decay and jump are (2, S) */
    const float *E_syn, *g_clip, *decay, *jump;
    const float *mg_c, *mg_a; /* NULL: no Mg block */
    float dt, surr_scale;
    int sample; /* escape noise: spike where noise < sigmoid(k (v - theta)) */
    int R;      /* columns of the gating state */
    /* 1: current-based neurons (network_simulators/current/dynamics.py:116-205): E_L
     * holds U_rest, C_m the resistance R, E_syn the types' signs; decay and jump (2, S)
     * with no rise component. The step's input enters the currents before the membrane
     * update, which uses them. */
    int current;
} WtoNet;

typedef struct {
    float *v;         /* (B, N) */
    float *g;         /* (B, N, 2, S) */
    int32_t *counter; /* (B, N) or NULL */
    float *g_a;       /* (B, N) or NULL */
    float *gating;    /* (B, R) or NULL */
} WtoState;

typedef struct {
    uint8_t *spikes;  /* (B, T, N) */
    float *v_track;   /* (B, T, N) voltage after each step, or NULL */
    float *prob;      /* (B, T, N) or NULL */
} WtoOut;

static float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

/* gate_step (network.py:186-223) for one trial: the factors f (n) of spikes s (n),
 * stepping the pathway's columns of the gating state in place. */
static void gate_step(const WtoPathway *p, float *state, const float *s, float *f) {
    int n = p->n;
    for (int i = 0; i < n; i++) {
        float fi = 1.0f;
        int have = 0;
        if (p->stp) {
            float u = state[p->start + i], x = state[p->start + n + i];
            x = 1.0f - (1.0f - x) * p->d_D;
            u = p->U + (u - p->U) * p->d_F;
            float r = u * x;
            fi = r / p->U;
            have = 1;
            x = x - s[i] * r;
            u = u + s[i] * p->U * (1.0f - u);
            state[p->start + i] = u;
            state[p->start + n + i] = x;
        }
        if (p->saturates) {
            int col = p->start + 2 * n * p->stp + i;
            float g = state[col] * p->d;
            float closed = 1.0f - g;
            if (!have)
                fi = p->c * closed;
            else {
                float a = p->c * fi * closed;
                fi = a < closed ? a : closed;
            }
            float gn = g + s[i] * fi;
            state[col] = gn < 1.0f ? gn : 1.0f;
        }
        f[i] = fi;
    }
}

/* The spike of neuron n of trial b entering step t (and its refractory mask, its
 * escape-noise probability). */
static void spike_of(const WtoNet *net, const float *v, const int32_t *counter, const float *noise, int b,
                     int T, int t, int n, float *s, float *held, float *prob) {
    const int N = net->N;
    held[n] = (net->n_ref && counter[n] > 0) ? 1.0f : 0.0f;
    float sn;
    if (net->sample) {
        float p = sigmoidf_(net->surr_scale * (v[n] - net->theta[n]));
        sn = noise[((size_t)b * T + t) * N + n] < p ? 1.0f : 0.0f;
    } else {
        sn = (v[n] - net->theta[n]) > 0.0f ? 1.0f : 0.0f;
    }
    if (net->n_ref) sn = sn * (1.0f - held[n]);
    s[n] = sn;
    if (prob) {
        float p = sigmoidf_(net->surr_scale * (v[n] - net->theta[n]));
        prob[((size_t)b * T + t) * N + n] = net->n_ref ? p * (1.0f - held[n]) : p;
    }
}

/* Membrane, counter and adaptation of neuron n: exponential Euler with the
 * conductances entering the step. */
static void membrane_of(const WtoNet *net, const float *v, const float *g, int32_t *counter, float *g_a,
                        const float *s, const float *held, float *v_next, int n) {
    const int S = net->S;
    const float *gn = g + (size_t)n * 2 * S;
    float gt[64];
    float vn = v[n];
    float G = 0.0f, Isum = 0.0f;
    for (int j = 0; j < S; j++) {
        float gs = gn[j] + gn[S + j];
        gs = gs > 0.0f ? gs : 0.0f; /* clamp(min=0) */
        gs = gs < net->g_clip[j] ? gs : net->g_clip[j];
        if (net->mg_c) gs = gs * sigmoidf_(net->mg_a[j] * vn - logf(net->mg_c[j]));
        gt[j] = gs;
    }
    for (int j = 0; j < S; j++) G = G + gt[j];
    for (int j = 0; j < S; j++) Isum = Isum + gt[j] * (vn - net->E_syn[j]);
    float rate = -log1pf(net->beta[n] - 1.0f) / net->dt;
    float g_L = net->C_m[n] * rate;
    float I_leak = g_L * (vn - net->E_L[n]);
    float J = Isum + I_leak;
    if (g_a) {
        G = G + g_a[n];
        J = J + g_a[n] * (vn - net->E_adapt[n]);
    }
    float xx = net->dt * rate + net->dt * G / net->C_m[n];
    float step = -expm1f(-xx) / (g_L + G);
    float r = s[n] > held[n] ? s[n] : held[n];
    v_next[n] = (vn - step * J) * (1.0f - r) + net->U_reset[n] * r;
    /* refractory counters and adaptation */
    if (net->n_ref) {
        int32_t c = counter[n] - 1;
        counter[n] = s[n] > 0.0f ? net->n_ref[n] : (c > 0 ? c : 0);
    }
    if (g_a) g_a[n] = g_a[n] * net->adapt_decay[n] + net->adapt[n] * s[n];
}

/* The current-based membrane of neuron n (current/dynamics.py:116-125, 180-183), with
 * the currents after this step's input: the adaptation current rises by the spike, then
 * v' = (beta v + (1 - beta)(U_rest + R (sum_j sign_j I_j - I_a)))(1 - r) + U_reset r. */
static void membrane_current(const WtoNet *net, const float *v, const float *g, int32_t *counter, float *g_a,
                             const float *s, const float *held, float *v_next, int n) {
    const int S = net->S;
    const float *gn = g + (size_t)n * 2 * S;
    if (g_a) g_a[n] = g_a[n] * net->adapt_decay[n] + net->adapt[n] * s[n];
    float Isyn = 0.0f;
    for (int j = 0; j < S; j++) Isyn = Isyn + gn[S + j] * net->E_syn[j];
    if (g_a) Isyn = Isyn - g_a[n];
    const float b = net->beta[n];
    const float r = s[n] > held[n] ? s[n] : held[n];
    v_next[n] = (b * v[n] + (1.0f - b) * (net->E_L[n] + net->C_m[n] * Isyn)) * (1.0f - r) + net->U_reset[n] * r;
    if (net->n_ref) {
        int32_t c = counter[n] - 1;
        counter[n] = s[n] > 0.0f ? net->n_ref[n] : (c > 0 ? c : 0);
    }
}

/* Pathway k's activation a_k = (pre_k * f_k) @ W_k of one trial, event-driven over the
 * rows that carry input, each target's sum in double. */
static void activation_of(const WtoNet *net, int k, const float *s, const float *xt, float *gating, float *pre,
                          float *fac, double *a) {
    const WtoPathway *p = &net->pathways[k];
    memset(a, 0, sizeof(double) * (size_t)net->N);
    for (int r = 0; r < p->n_rows; r++) pre[r] = p->recurrent ? s[p->rows[r]] : xt[p->rows[r]];
    if (p->gate) {
        gate_step(p, gating, pre, fac);
        for (int r = 0; r < p->n_rows; r++) pre[r] = pre[r] * fac[r];
    }
    for (int r = 0; r < p->n_rows; r++) {
        float q = pre[r];
        if (q == 0.0f) continue;
        for (int64_t e = p->row_ptr[r]; e < p->row_ptr[r + 1]; e++) a[p->cols[e]] += (double)q * (double)p->w[e];
    }
}

/* g = g * decay + sum_k a_k * kernel_k for neuron n, then the step's outputs. */
static void conductances_of(const WtoNet *net, float *g, const double *acc, int n) {
    const int S = net->S, K = net->K, N = net->N;
    float *gn = g + (size_t)n * 2 * S;
    for (int c = 0; c < 2; c++)
        for (int j = 0; j < S; j++) gn[c * S + j] = gn[c * S + j] * net->decay[c * S + j];
    for (int k = 0; k < K; k++) {
        const WtoPathway *p = &net->pathways[k];
        float a = (float)acc[(size_t)k * N + n];
        for (int c = 0; c < 2; c++)
            for (int j = 0; j < S; j++) {
                float kern = net->jump[c * S + j] * p->scale[n] * (p->made[j] ? 1.0f : 0.0f);
                gn[c * S + j] = gn[c * S + j] + a * kern;
            }
    }
}

/* Simulate T steps of every trial from state st with input x (B, T, n_in). With at
 * least as many trials as threads, each thread runs whole trials; otherwise each step's
 * per-neuron work runs in parallel over (trial, neuron) and the activations over
 * (trial, pathway), so that all the host's threads take part. The arithmetic of every
 * neuron and every sum is the same either way. */
int wto_simulate(const WtoNet *net, WtoState *st, const float *x, int T, WtoOut *out,
                 const float *noise /* (B, T, N) if sample */) {
    const int B = net->B, N = net->N, S = net->S, K = net->K, n_in = net->n_in;
    if (S > 64) return 2;
    if (B >= omp_get_max_threads()) {
        int status = 0;
        const int rows_max = N > n_in ? N : n_in;
#pragma omp parallel for schedule(dynamic, 1)
        for (int b = 0; b < B; b++) {
            float *v = st->v + (size_t)b * N, *g = st->g + (size_t)b * N * 2 * S;
            int32_t *counter = st->counter ? st->counter + (size_t)b * N : NULL;
            float *g_a = st->g_a ? st->g_a + (size_t)b * N : NULL;
            float *gating = st->gating ? st->gating + (size_t)b * net->R : NULL;
            float *sb = malloc(sizeof(float) * N), *hb = malloc(sizeof(float) * N);
            float *vn = malloc(sizeof(float) * N);
            double *ab = malloc(sizeof(double) * (size_t)K * N);
            float *pr = malloc(sizeof(float) * rows_max), *fc = malloc(sizeof(float) * rows_max);
            if (!sb || !hb || !vn || !ab || !pr || !fc) {
#pragma omp atomic write
                status = 1;
            } else {
                for (int t = 0; t < T; t++) {
                    const float *xt = x + ((size_t)b * T + t) * n_in;
                    for (int n = 0; n < N; n++) spike_of(net, v, counter, noise, b, T, t, n, sb, hb, out->prob);
                    if (!net->current)
                        for (int n = 0; n < N; n++) membrane_of(net, v, g, counter, g_a, sb, hb, vn, n);
                    for (int k = 0; k < K; k++) activation_of(net, k, sb, xt, gating, pr, fc, ab + (size_t)k * N);
                    for (int n = 0; n < N; n++) {
                        conductances_of(net, g, ab, n);
                        if (net->current) membrane_current(net, v, g, counter, g_a, sb, hb, vn, n);
                        v[n] = vn[n];
                        size_t o = ((size_t)b * T + t) * N + n;
                        out->spikes[o] = sb[n] > 0.0f;
                        if (out->v_track) out->v_track[o] = v[n];
                    }
                }
            }
            free(sb); free(hb); free(vn); free(ab); free(pr); free(fc);
        }
        return status;
    }
    const size_t BN = (size_t)B * N;
    const int rows_max = N > n_in ? N : n_in;
    float *s = malloc(sizeof(float) * BN);
    float *held = malloc(sizeof(float) * BN);
    float *v_next = malloc(sizeof(float) * BN);
    double *acc = malloc(sizeof(double) * (size_t)K * BN);
    float *pre = malloc(sizeof(float) * (size_t)B * K * rows_max);
    float *fac = malloc(sizeof(float) * (size_t)B * K * rows_max);
    if (!s || !held || !v_next || !acc || !pre || !fac) {
        free(s); free(held); free(v_next); free(acc); free(pre); free(fac);
        return 1;
    }
    for (int t = 0; t < T; t++) {
#pragma omp parallel for schedule(static)
        for (long long i = 0; i < (long long)BN; i++) {
            const int b = (int)(i / N), n = (int)(i % N);
            const float *v = st->v + (size_t)b * N;
            const int32_t *counter = st->counter ? st->counter + (size_t)b * N : NULL;
            spike_of(net, v, counter, noise, b, T, t, n, s + (size_t)b * N, held + (size_t)b * N, out->prob);
        }
#pragma omp parallel for schedule(static)
        for (long long i = 0; i < (long long)BN; i++) {
            const int b = (int)(i / N), n = (int)(i % N);
            if (net->current) continue;  /* after the currents take the step's input */
            membrane_of(net, st->v + (size_t)b * N, st->g + (size_t)b * N * 2 * S,
                        st->counter ? st->counter + (size_t)b * N : NULL, st->g_a ? st->g_a + (size_t)b * N : NULL,
                        s + (size_t)b * N, held + (size_t)b * N, v_next + (size_t)b * N, n);
        }
#pragma omp parallel for schedule(dynamic, 1)
        for (int i = 0; i < B * K; i++) {
            const int b = i / K, k = i % K;
            const float *xt = x + ((size_t)b * T + t) * n_in;
            float *gating = st->gating ? st->gating + (size_t)b * net->R : NULL;
            activation_of(net, k, s + (size_t)b * N, xt, gating, pre + (size_t)i * rows_max,
                          fac + (size_t)i * rows_max, acc + (size_t)i * N);
        }
#pragma omp parallel for schedule(static)
        for (long long i = 0; i < (long long)BN; i++) {
            const int b = (int)(i / N), n = (int)(i % N);
            conductances_of(net, st->g + (size_t)b * N * 2 * S, acc + (size_t)b * K * N, n);
            if (net->current)
                membrane_current(net, st->v + (size_t)b * N, st->g + (size_t)b * N * 2 * S,
                                 st->counter ? st->counter + (size_t)b * N : NULL,
                                 st->g_a ? st->g_a + (size_t)b * N : NULL, s + (size_t)b * N, held + (size_t)b * N,
                                 v_next + (size_t)b * N, n);
            st->v[i] = v_next[i];
            size_t o = ((size_t)b * T + t) * N + n;
            out->spikes[o] = s[i] > 0.0f;
            if (out->v_track) out->v_track[o] = st->v[i];
        }
    }
    free(s); free(held); free(v_next); free(acc); free(pre); free(fac);
    return 0;
}

int wto_version(void) { return 2; }
