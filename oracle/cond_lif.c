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
 * Per step, for every trial (trials are independent, so OpenMP runs them in
 * parallel):
 *   held = counter > 0                                   network.py:294-302
 *   s    = H(v - theta) (1 - held)  [or noise < sigmoid]  dynamics.py:103-107
 *   v'   = membrane(v, max(s, held), g, g_a)             dynamics.py:116-143
 *   counter, g_a updated                                  network.py:313-318, dynamics.py:201-202
 *   a_k  = (pre_k * f_k) @ W_k  per pathway               network.py:260-271
 *   g    = g * decay + sum_k a_k (jump * scale_k * made_k) dynamics.py:206-208
 * with the presynaptic gating (short-term plasticity, saturation) of network.py:186-223.
 */
#include <math.h>
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

/* Simulate T steps of every trial from state st with input x (B, T, n_in). */
int wto_simulate(const WtoNet *net, WtoState *st, const float *x, int T, WtoOut *out,
                 const float *noise /* (B, T, N) if sample */) {
    const int B = net->B, N = net->N, S = net->S, K = net->K, n_in = net->n_in;
    int status = 0;
#pragma omp parallel for schedule(dynamic, 1)
    for (int b = 0; b < B; b++) {
        float *v = st->v + (size_t)b * N;
        float *g = st->g + (size_t)b * N * 2 * S;
        int32_t *counter = st->counter ? st->counter + (size_t)b * N : NULL;
        float *g_a = st->g_a ? st->g_a + (size_t)b * N : NULL;
        float *gating = st->gating ? st->gating + (size_t)b * net->R : NULL;
        float *s = malloc(sizeof(float) * N);
        float *held = malloc(sizeof(float) * N);
        float *v_next = malloc(sizeof(float) * N);
        float *gt = malloc(sizeof(float) * S);
        double *acc = malloc(sizeof(double) * (size_t)K * N);
        float *pre = malloc(sizeof(float) * (N > n_in ? N : n_in));
        float *fac = malloc(sizeof(float) * (N > n_in ? N : n_in));
        if (!s || !held || !v_next || !gt || !acc || !pre || !fac) {
            status = 1;
            free(s); free(held); free(v_next); free(gt); free(acc); free(pre); free(fac);
            continue;
        }
        for (int t = 0; t < T; t++) {
            const float *xt = x + ((size_t)b * T + t) * n_in;
            /* spike and refractory mask */
            for (int n = 0; n < N; n++) {
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
                if (out->prob) {
                    float p = sigmoidf_(net->surr_scale * (v[n] - net->theta[n]));
                    out->prob[((size_t)b * T + t) * N + n] = net->n_ref ? p * (1.0f - held[n]) : p;
                }
            }
            /* membrane: exponential Euler with the conductances entering the step */
            for (int n = 0; n < N; n++) {
                const float *gn = g + (size_t)n * 2 * S;
                float vn = v[n];
                float G = 0.0f, Isum = 0.0f;
                for (int j = 0; j < S; j++) {
                    float gs = gn[j] + gn[S + j];
                    gs = gs > 0.0f ? gs : 0.0f; /* clamp(min=0) */
                    gs = gs < net->g_clip[j] ? gs : net->g_clip[j];
                    if (net->mg_c)
                        gs = gs * sigmoidf_(net->mg_a[j] * vn - logf(net->mg_c[j]));
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
            }
            /* refractory counters and adaptation */
            for (int n = 0; n < N; n++) {
                if (net->n_ref) {
                    int32_t c = counter[n] - 1;
                    counter[n] = s[n] > 0.0f ? net->n_ref[n] : (c > 0 ? c : 0);
                }
                if (g_a) g_a[n] = g_a[n] * net->adapt_decay[n] + net->adapt[n] * s[n];
            }
            /* activations per pathway, event-driven over the rows that carry input */
            memset(acc, 0, sizeof(double) * (size_t)K * N);
            for (int k = 0; k < K; k++) {
                const WtoPathway *p = &net->pathways[k];
                for (int r = 0; r < p->n_rows; r++)
                    pre[r] = p->recurrent ? s[p->rows[r]] : xt[p->rows[r]];
                if (p->gate) {
                    gate_step(p, gating, pre, fac);
                    for (int r = 0; r < p->n_rows; r++) pre[r] = pre[r] * fac[r];
                }
                double *a = acc + (size_t)k * N;
                for (int r = 0; r < p->n_rows; r++) {
                    float q = pre[r];
                    if (q == 0.0f) continue;
                    for (int64_t e = p->row_ptr[r]; e < p->row_ptr[r + 1]; e++)
                        a[p->cols[e]] += (double)q * (double)p->w[e];
                }
            }
            /* g = g * decay + sum_k a_k * kernel_k */
            for (int n = 0; n < N; n++) {
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
            for (int n = 0; n < N; n++) {
                v[n] = v_next[n];
                size_t o = ((size_t)b * T + t) * N + n;
                out->spikes[o] = s[n] > 0.0f;
                if (out->v_track) out->v_track[o] = v[n];
            }
        }
        free(s); free(held); free(v_next); free(gt); free(acc); free(pre); free(fac);
    }
    return status;
}

int wto_version(void) { return 1; }
