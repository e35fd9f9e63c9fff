/*
 * wiretorch_b200 — the C ABI of the B200 engine for wiretorch's conductance-based LIF
 * simulation step.
 *
 * Every entry point takes plain device pointers and sizes (in the structures below) and
 * a CUDA stream, enqueues its kernels on that stream and returns at once: 0 on success,
 * a nonzero WT_ERR_* code if the arguments are inconsistent or a launch failed. None
 * allocates memory (the caller passes every buffer, sized with wt_workspace_bytes) and
 * none synchronises. Errors met by the kernels themselves — a grid barrier that timed
 * out, an event list or fixed-point accumulator that overflowed — are written to the
 * device word `err` of the workspace, which the caller reads after the stream has
 * synchronised. wt_last_error() describes the last host-side failure of this thread.
 *
 * Layouts (row-major, contiguous): state v (B, N); conductances g (B, 2, S, N), i.e.
 * per trial, component (rise, decay) and synapse channel, contiguous over neurons;
 * refractory counters (B, N) int32; adaptation (B, N); presynaptic gating (B, R);
 * input x (B, T, n_in); spikes (B, T, N) float32.
 *
 * The reference (rory-bedford/wiretorch) is pure Python with Triton kernels and binds
 * no foreign functions; each entry point names the Python/Triton function of the
 * reference whose work it replaces.
 */
#ifndef WIRETORCH_B200_H
#define WIRETORCH_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WT_MAX_CHANNELS 8 /* synapse channels a neuron carries in the fast kernels */
#define WT_CHUNK_EDGES 128 /* edges of one scatter work item */

enum {
    WT_OK = 0,
    WT_ERR_ARGS = 1,        /* inconsistent sizes or missing buffers */
    WT_ERR_LAUNCH = 2,      /* a kernel launch failed (see wt_last_error) */
    WT_ERR_BARRIER = 3,     /* device: a grid barrier gave up waiting */
    WT_ERR_EVENTS = 4,      /* device: an event list overflowed its capacity */
    WT_ERR_FIXED_POINT = 5, /* device: a synaptic input exceeded the fixed-point range */
    WT_ERR_UNSUPPORTED = 6, /* a combination the kernels do not implement */
    WT_ERR_RANGE = 7,       /* device: an index outside its table (partitioned runs check; the
                             * bits above 8 name the check), the access skipped */
};

/* Feature flags of a forward run (WtForward.flags). */
enum {
    WT_F_REFRACTORY = 1 << 0, /* n_ref / counter are used */
    WT_F_MG_BLOCK = 1 << 1,   /* some channel has a voltage-dependent Mg block */
    WT_F_ADAPT = 1 << 2,      /* adaptation conductance */
    WT_F_SAMPLE = 1 << 3,     /* escape-noise spikes: noise < sigmoid(k (v - theta)) */
    WT_F_GATED = 1 << 4,      /* presynaptic gating (short-term plasticity, saturation) */
    WT_F_SAVE = 1 << 5,       /* save what the backward pass needs */
    WT_F_TRACK = 1 << 6,      /* per-step v, currents, conductances */
    WT_F_PROB = 1 << 7,       /* escape-noise probabilities output */
    WT_F_SAVE_INPUT = 1 << 8, /* save each step's synaptic input X (learnt decay/jump) */
    WT_F_PARTITION = 1 << 9,  /* one rank of a neuron-partitioned run (WtForward.words...) */
    WT_F_STREAM = 1 << 10,    /* keep the state in HBM even where it fits on chip (tests) */
    WT_F_CURRENT = 1 << 11,   /* current-based neurons (see WtNet): the step's own input enters
                               * the currents before the membrane update */
};

/* The network as the kernels see it (built once per network and per call from the
 * reference's Drive and Physiology; see wiretorch_b200/plan.py). */
typedef struct {
    int32_t B, N, n_in;  /* trials, neurons, input columns */
    int32_t S, C;        /* synapse channels carried per neuron, input channels */
    /* per neuron (N) */
    const float *theta, *U_reset, *E_L, *C_m, *beta;
    /* (WT_F_CURRENT, network_simulators/current/dynamics.py:116-205: E_L holds U_rest,
     * C_m the resistance R, E_syn the synapse types' signs, adapt and adapt_decay the
     * adaptation current's rise and decay; each channel a single exponential, decay_d
     * and jump_d 1) */
    const int32_t *n_ref;                       /* WT_F_REFRACTORY */
    const float *adapt, *adapt_decay, *E_adapt; /* WT_F_ADAPT */
    /* per channel (S): decays and jumps of the rise (r) and decay (d) components */
    float decay_r[WT_MAX_CHANNELS], decay_d[WT_MAX_CHANNELS];
    float jump_r[WT_MAX_CHANNELS], jump_d[WT_MAX_CHANNELS];
    float E_syn[WT_MAX_CHANNELS], g_clip[WT_MAX_CHANNELS];
    float mg_a[WT_MAX_CHANNELS], mg_lc[WT_MAX_CHANNELS]; /* block: sigmoid(mg_a v - mg_lc) */
    int32_t input_of[WT_MAX_CHANNELS]; /* input channel feeding each channel, -1: none */
    float fx_inv[WT_MAX_CHANNELS];     /* per input channel: 2^-s of its fixed point */
    float dt, surr_scale;
    /* connectivity: sources are the N neurons then the n_in input columns; each source
     * owns slots (one per pathway it belongs to), each slot chunks of at most
     * WT_CHUNK_EDGES edges of its CSR row (a chunk is one work item) */
    const int32_t *src_slot;    /* (N + n_in + 1) */
    const int32_t *slot_chunk;  /* (n_slots + 1) */
    const int32_t *src_chunk;   /* (N + n_in + 1): each source's first chunk (a source's
                                   chunks are contiguous: its slots' chunks in order) */
    const int64_t *chunk_desc;  /* (n_chunks): first edge | edge count << 56 */
    const uint32_t *edge_col;   /* (E): target | input channel << 27 */
    const uint64_t *edge_cw;    /* (E): edge_col | folded weight bits << 32, the weight
                                   times 2^s of its channel (written by wt_fold_weights) */
    int32_t n_slots, n_chunks;
    int64_t n_rec_edges;        /* edges of the neurons' pathways (they come first) */
    /* presynaptic gating (WT_F_GATED): per slot its gate (-1: none) and row */
    const int32_t *slot_gate, *slot_row;
    const float *gate_params;   /* (n_gates, 5): c, d, U, d_D, d_F */
    const int32_t *gate_cols;   /* (n_gates, 4): u column (-1: no STP), n rows,
                                   saturation column (-1: none), saved-factor column */
    int32_t R, R_f;             /* gating columns, saved-factor columns */
    /* sources that are neurons: N, or in a neuron-partitioned run every rank's neurons
     * (the N targets here are this rank's; input column i is source N_src + i) */
    int32_t N_src;
    /* optional, gated runs (N_src + n_in, 2): per source its gate and row when it owns at
     * most one slot (gate -1: that slot is ungated or there is none), gate -2 when it
     * owns several. With it the forward kernel steps a source's gating state without
     * walking its slots; NULL: every gated source walks its slots. */
    const int32_t *src_gate;
} WtNet;

/* One scatter work item: a chunk of a source's edges, for one trial. */
typedef struct {
    int64_t edge;               /* first edge */
    uint32_t trial_len;         /* trial << 8 | edge count */
    float amp;                  /* the spike's (or input's) value times its gating factor */
} WtEvent;

/* Buffers of one forward run of T steps (outputs indexed by step t0 + t of a chunk of
 * T_total steps, so a chunk may be run in several launches). */
typedef struct {
    int32_t T, T_total, t0, flags;
    float *v, *g;               /* state, updated in place */
    int32_t *counter;           /* WT_F_REFRACTORY */
    float *g_a;                 /* WT_F_ADAPT */
    float *gating;              /* WT_F_GATED: (B, R) */
    const float *x;             /* (B, T_total, n_in) */
    const float *noise;         /* WT_F_SAMPLE: (B, T_total, N) uniform */
    float *spikes;              /* (B, T_total, N) */
    float *prob;                /* WT_F_PROB */
    /* WT_F_SAVE: v entering each step (B, T, N); summed conductances (B, T, S, N);
     * spike and refractory bits (B, T, ceil(N / 32)); adaptation (B, T, N); gating
     * factors (B, T, R_f); WT_F_SAVE_INPUT: input (B, T, C, N) */
    float *v_saved, *G_saved;
    uint32_t *spike_bits, *held_bits;
    float *a_saved, *f_saved, *X_saved;
    /* WT_F_TRACK: trial track_b (-1: all) — v (Bt, T_total, N), currents
     * (Bt, T_total, N, S + 1), conductances (Bt, T_total, N, 2, S), adaptation */
    float *track_v, *track_I, *track_g, *track_a;
    int32_t track_b;
    /* WT_F_PARTITION: this rank holds neurons word0 * 32 .. of the N_src; each step's
     * spike words of all ranks' neurons are replicated on every rank — words
     * (2, B, ceil(N_src / 32)) here and the same buffers on the n_ranks ranks (peer
     * pointers, this rank's own among them), written by their owners — and each rank's
     * progress through the run is a slot, (epoch << 32) | (step + 1), in every rank's
     * progress (n_ranks uint64). epoch: the same on all ranks, larger on every call. */
    uint32_t *words;
    uint32_t *peer_words[8];
    unsigned long long *progress;
    unsigned long long *peer_progress[8];
    int32_t n_ranks, rank, word0;
    uint32_t epoch;
    /* optional, WT_F_PARTITION with WT_F_GATED when every neuron owns at most one slot
     * (WtNet.src_gate never -2): the factors of each step's spikes, (2, B,
     * ceil(N_src / 32) * 32) floats here and on the n_ranks ranks, written by the rank
     * that owns the neuron (it alone steps that neuron's gating state; the other ranks'
     * copies of those columns are left as they were). NULL: every rank steps every
     * source's gates from the spike words. */
    float *amps;
    float *peer_amps[8];
    /* optional, a partitioned run whose ranks push their events (networks without gating,
     * or whose gates their owners step): instead of publishing spike words for every rank
     * to walk, a rank writes the events of its own neurons' spikes onto each rank r's
     * targets straight into r's inbound event area over the interconnect, so that a step
     * takes one grid barrier (fused with the progress exchange). Per rank r: r's chunk
     * range of every neuron (push_src_chunk[r], N_src + 1 entries) and r's chunk
     * descriptors (push_chunk_desc[r]), local copies; this rank's region of r's area
     * (push_ev[r], push_cap[r] events, the two step parities push_half[r] events apart)
     * and r's inbound counts (push_count[r]: [2][8], this rank's at [parity][rank]).
     * push_reserve ([2][8], zeroed): this rank's reservations per parity and rank. This
     * rank's own area: pull_ev (regions pull_off[q] of source rank q, parities pull_half
     * apart) and pull_count ([2][8], written by the ranks). NULL push_reserve: words. */
    const int32_t *push_src_chunk[8];
    const long long *push_chunk_desc[8];
    WtEvent *push_ev[8];
    long long push_cap[8], push_half[8];
    uint32_t *push_count[8];
    uint32_t *push_reserve;
    const WtEvent *pull_ev;
    long long pull_off[8];
    long long pull_half;
    const uint32_t *pull_count;
    /* optional, instrumented runs: per step and warp of the grid, the global timer (ns)
     * at the ends of the step's phases, (T, phase_warps, WT_PHASES); warps of the grid
     * beyond phase_warps record nothing. NULL: no record. */
    unsigned long long *phases;
    int32_t phase_warps;
} WtForward;

/* The phases of a forward step that WtForward.phases records, in order: the step's
 * start; the next step's input columns emitted; the early scatter done (the even warps
 * of a block scatter before their items); the warp's items done (membrane update and
 * spike emission); the late scatter done (the odd warps); the grid barrier passed; the
 * spike exchange of a partitioned run done (its progress wait, barrier and emission). */
#define WT_PHASES 7

/* Scratch memory of a forward run; all of it device memory the caller allocated. */
typedef struct {
    unsigned long long *X;      /* (2, C, B, Np) fixed-point input accumulators, Np = N rounded
                                 * up to a multiple of 32; 16-byte aligned */
    WtEvent *ev;                /* (2, ev_cap) events of two consecutive steps */
    uint32_t *ev_count;         /* (T + 1) */
    uint32_t *barrier;          /* (64) */
    int32_t *err;               /* (1): a device error code, 0 if none */
    int64_t ev_cap;
    unsigned long long *edges;  /* (2) or NULL: edges traversed (recurrent, input) */
} WtWorkspace;

/* Bytes of each workspace buffer for a run of T steps (X, ev, ev_count, barrier, err,
 * edges), written to bytes[0..5]. */
int wt_workspace_bytes(const WtNet *net, int32_t T, int64_t bytes[6]);

/* Fold the per-edge weights: the weight of edge_cw[e] = w[e] * scale[k(e), col(e)] *
 * jf[k(e), c(e)] * 2^s(c(e)) for every edge of every chunk, from the raw weights w and the
 * pathway of each chunk. Replaces the per-call kernel scale of the reference's Drive
 * (network_simulators/network.py:816-854 `_drive`, conductance/dynamics.py:95-100
 * `jumps`). */
int wt_fold_weights(const WtNet *net, const float *w_raw, const int32_t *chunk_path,
                    const float *scale /* (K, N) */, const float *jf /* (K, C) */,
                    const float *fx_scale /* (C) */, uint64_t *edge_cw_out, void *stream);

/* Simulate T steps: one persistent kernel. Replaces the reference's per-step launches
 * of `compact_spikes` + `recurrent_step` (network_simulators/kernels.py:132-204,
 * conductance/kernels.py:571-700, driven by conductance/engine.py:306-355 `_recurrent`)
 * and its feedforward scan `scan_forward` (conductance/kernels.py:158-289, driven by
 * conductance/engine.py:285-303 `_scan`). */
int wt_forward(const WtNet *net, const WtForward *run, const WtWorkspace *ws, void *stream);

/* wt_forward with no caller-allocated workspace: the scratch is a static device array of
 * 32 MiB per device; runs whose workspace (wt_workspace_bytes) does not fit are rejected
 * with WT_ERR_ARGS. No counterpart in the reference (its engine allocates its buffers
 * with PyTorch on every call). For callers that cannot allocate device memory on this
 * path. The first call on a device looks up the array (do it before any stream capture);
 * calls overlapping in time share the array and race, so a caller serialises them. The
 * address looked up belongs to the device's context: after cudaDeviceReset this entry
 * point must not be called again in the process. A call rejected by the argument checks
 * launches nothing and keeps the previous run's device error code. The run's device
 * error code is read with wt_noalloc_error. Allocates nothing. */
int wt_forward_noalloc(const WtNet *net, const WtForward *run, void *stream);

/* The device error code (0: none) of the last wt_forward_noalloc on the current device,
 * after waiting for `stream`, which must be the stream that run was enqueued on (a read
 * on another stream may come before the run ends). No counterpart in the reference. */
int wt_noalloc_error(void *stream, int32_t *code);

/* Gradients wanted by a backward pass (WtBackward.wants): the physiology, in the order
 * of the reference's PHYSIOLOGY (conductance/engine.py:190-193). */
enum {
    WT_W_THETA = 1 << 0, WT_W_RESET = 1 << 1, WT_W_E_L = 1 << 2, WT_W_C_M = 1 << 3,
    WT_W_BETA = 1 << 4, WT_W_E_SYN = 1 << 5, WT_W_DECAY = 1 << 6, WT_W_JUMP = 1 << 7,
    WT_W_ADAPT = 1 << 8, WT_W_ADAPT_DECAY = 1 << 9, WT_W_E_ADAPT = 1 << 10,
};

/* One reverse scan over the T steps of a forward run saved with WT_F_SAVE (flags as
 * that run's). Per (trial, neuron): the adjoint of each input channel at every step,
 * Q (B, T, C, N) — dL/dX, what a unit of input of that channel at that step is worth —
 * and per-(trial, neuron) partial sums of the physiology gradients wanted: theta,
 * U_reset, E_L, C_m, beta, adapt, adapt_decay, E_adapt (B, N) each; E_syn (B, S, N);
 * decay and jump (B, 2, S, N). grad_spikes (B, T, N) is dL/d(spike), grad_prob
 * dL/d(probability) with WT_F_PROB. g_init (B, 2, S, N), the conductances entering the
 * run, and the saved input X (WT_F_SAVE_INPUT) are read for decay and jump. */
typedef struct {
    int32_t T, flags, wants;
    const float *grad_spikes, *grad_prob;
    const float *v_saved, *G_saved, *a_saved, *X_saved, *g_init;
    const uint32_t *spike_bits, *held_bits;
    float *Q;
    float *g_theta, *g_reset, *g_E_L, *g_C_m, *g_beta, *g_E_syn, *g_decay, *g_jump;
    float *g_adapt, *g_adapt_decay, *g_E_adapt;
    /* Steps t_hi - 1 down to t_lo (t_hi 0: T). With `adj` (B, 2 + 4 S, N) — dL/dv, the
     * adaptation's adjoint, dL/dg rise and decay per channel, the decays' H — the scan
     * starts from that state, leaves its end state there and adds to the physiology
     * outputs instead of writing them (one chunk of a scan taken step by step); without,
     * it starts from zero. R (B, N), when given, is added to dL/d(spike) of the steps
     * (the recurrent pathways' carry of a single step, wt_recurrent_carry). */
    int32_t t_lo, t_hi;
    float *adj;
    const float *R;
    /* optional, a whole scan (no adj, t_lo 0, t_hi T): the same adjoints target-major,
     * QT (C, N, B, Tp) with Tp = T rounded up to a multiple of 8 (entries past T are
     * zero), for the edge gradients' target-by-target pass; with QT, Q may be NULL. */
    float *QT;
} WtBackward;

/* Gradients carried along the connectome's edges, from the adjoints Q of a reverse scan:
 * for every event of the run (a recurrent spike, from the saved spike bits, or a
 * non-zero input x) and every edge e of its slot (pathway k, target n, input channel c),
 * with a = the event's value times its gating factor (summed per edge over the source's
 * events first, then added once per edge):
 *   g_scale[k, n] += a * w[e] * jf[k, c] * Q[b, t, c, n]      (B-summed, float64)
 *   g_w[e]        += a * scale[k, n] * jf[k, c] * Q[b, t, c, n] (float64)
 * and, for every input column i, trial and step, whether or not it fired,
 *   g_x[b, t, i] = sum over i's slots of f * sum_e w[e] scale[k, n] jf[k, c] Q[b, t, c, n]. */
typedef struct {
    int32_t T;
    const uint32_t *spike_bits;  /* (B, T, ceil(N / 32)) */
    const float *x, *f_saved, *Q;
    const float *w_raw, *scale, *jf;
    const int32_t *chunk_path;
    double *g_scale;             /* (K, N) or NULL */
    double *g_w;                 /* (E) or NULL; accumulated into (the caller zeroes it) */
    float *g_x;                  /* (B, T, n_in) or NULL */
    /* scratch for g_scale / g_w: each source's firing bits over (trial, step),
     * wt_edge_grads_scratch_words(net, T) words, and a work counter (1 word) */
    uint32_t *fired;
    uint32_t *work;
    /* optional: g_scale and g_w target by target from QT (WtBackward.QT, Tp = T rounded
     * up to 8) instead of source by source from Q: a block per target stages the
     * target's adjoints of a slice of trials in shared memory (wt_edge_grads_slice_trials
     * trials at a time) and sums every in-edge's events from there, so each adjoint is
     * read from HBM once. The in-edges of each target, by pathway then edge (in_ptr
     * (N + 1), and per in-edge its edge, its source and its pathway and input channel as
     * 8 k + c, (E_in) each; in_fcol
     * its gating factor's column of f_saved, -1 ungated, or NULL when nothing is gated);
     * scratch: ev_start ((N + n_in) (slices + 1)) and ev (ev_cap) for each source's events
     * (b Tp + t) and where each slice of trials starts among them, in_acc (E_in) floats,
     * and err: WT_ERR_EVENTS when the run's events exceed ev_cap (below 2^31). */
    const float *QT;
    const int32_t *in_ptr, *in_edge, *in_src, *in_path, *in_fcol;
    int32_t *ev_start, *ev;
    long long ev_cap;
    float *in_acc;
    int32_t *err;
} WtEdgeGrads;

/* 32-bit words of WtEdgeGrads.fired for a run of T steps. */
int64_t wt_edge_grads_scratch_words(const WtNet *net, int32_t T);

/* Trials per slice of the target-by-target edge gradients (WtEdgeGrads.QT) for a run of
 * T steps; 0 when even one trial's adjoints of a target do not fit in shared memory (use
 * Q, source by source). */
int32_t wt_edge_grads_slice_trials(const WtNet *net, int32_t T);

/* The reverse scan. Replaces `scan_backward` (conductance/kernels.py:382-568, driven by
 * conductance/engine.py:358-383 `_backward`). */
int wt_backward(const WtNet *net, const WtBackward *bwd, void *stream);

/* Gradients through the recurrent spikes (Drive.recurrent_gradients): what step t's
 * input adjoints pass back to the spikes of that step's recurrent sources,
 * R[b, j] = sum over j's edges e (pathway k, target n, channel c) of
 * w_e scale[k, n] jf[k, c] Q[b, t, c, n] (a gated pathway's edges times that step's
 * factors), Q of step t formed from the adjoint state `adj` entering the step (the
 * layout of WtBackward.adj). Qt (C, N, B) is scratch. Replaces `carry_to_sources` with
 * `presynaptic` (network_simulators/engine.py:257-306), driven per step by
 * `_recurrent_backward` (conductance/engine.py:386-436). */
typedef struct {
    int32_t T, t;
    const float *adj;
    const float *f_saved;  /* (B, T, R_f) when the net is gated */
    float *Qt;
    float *R;
} WtRecurrentCarry;

int wt_recurrent_carry(const WtNet *net, const WtRecurrentCarry *rc, void *stream);

/* The edge gradients. Replaces the scale partials of `scan_backward`, the weight
 * gradient `weight_gradient` (network_simulators/engine.py:327-350) and the input
 * gradient of `_SparseActivations.backward` (network_simulators/engine.py:96-116). */
int wt_edge_grads(const WtNet *net, const WtEdgeGrads *eg, void *stream);

/* The double-exponential filter of the spike-train losses, over (B, T, N) trains:
 * rise_t = a_rise rise_{t-1} + x_t, smooth_t = a_decay smooth_{t-1} + rise_t, the carried
 * state entering undecayed at t = 0. x is read with element strides (a t-stride of 0
 * filters a train constant in time). */
typedef struct {
    int32_t B, T, N;
    const float *x;
    int64_t x_bstride, x_tstride;
    const float *carry_rise, *carry_smooth;  /* (B, N), or NULL for zero */
    float a_rise, a_decay;
    float *rise, *smooth;                    /* (B, T, N), either may be NULL */
    float *last_rise, *last_smooth;          /* (B, N), either may be NULL */
} WtFilterArgs;

/* The filter's adjoint: dL/dx from dL/dsmooth times grad_scale (no gradient flows into
 * the carried state or through rise). */
typedef struct {
    int32_t B, T, N;
    const float *grad_smooth;
    float grad_scale;
    float a_rise, a_decay;
    float *grad_x;
} WtFilterGradArgs;

/* Replaces `_filter_forward` (training_utils/filtering.py:103-120) and the CPU Toeplitz
 * path of `double_exponential` (filtering.py:28-73). */
int wt_filter_forward(const WtFilterArgs *f, void *stream);

/* Replaces `_filter_backward` (training_utils/filtering.py:123-135). */
int wt_filter_backward(const WtFilterGradArgs *f, void *stream);

/* The van Rossum rate loss of one chunk in one pass: the double-exponential filter of the
 * output x and of the target rate y (each from its carried state), the difference of the
 * smoothed trains err = smooth(x) - smooth(y), saved for the backward pass, and per block
 * of 256 (trial, neuron) columns the sum of err^2 (partial[ceil(B N / 256)]). x and y have
 * unit neuron stride; y's strides may be 0 (a rate constant in time or across trials). */
typedef struct {
    int32_t B, T, N;
    const float *x;
    int64_t x_bstride, x_tstride;
    const float *y;
    int64_t y_bstride, y_tstride;
    const float *carry; /* (4, B, N) or NULL: output rise, output smooth, target rise, smooth */
    float a_rise, a_decay;
    float *err;         /* (B, T, N) */
    float *last;        /* (4, B, N): the states after the last step, as carry */
    double *partial;    /* (ceil(B N / 256)) */
} WtVanRossumArgs;

/* dL/dx of the loss mean(err^2): the filter's adjoint applied to scale * grad_loss * err,
 * scale = 2 / (B T N), grad_loss a device scalar (no host read). */
typedef struct {
    int32_t B, T, N;
    const float *err;
    const float *grad_loss;
    float scale;
    float a_rise, a_decay;
    float *grad_x;
} WtVanRossumGradArgs;

/* Replaces `VanRossumRateLoss.forward` (training_utils/losses.py:140-194): its two
 * `double_exponential` calls (training_utils/filtering.py:28-48) and the mean of the
 * squared difference, which the reference computes as separate passes. */
int wt_van_rossum_forward(const WtVanRossumArgs *a, void *stream);

/* The backward pass of that loss down to the output train (filtering.py:123-135 applied
 * to the loss's gradient). */
int wt_van_rossum_backward(const WtVanRossumGradArgs *a, void *stream);

/* The factorised recurrent drive of one step on the tensor cores: for pathways k < KP
 * (1..4) with weights W_k = U_k V^T, D[k, b, n] = sum_r V[n, r] P[b, k, r], P_k = S_k U_k
 * the spikes' sum of U rows (fp32), V bf16 with 64 rank slots (a lower rank zero-padded).
 * tcgen05.mma with the accumulator in tensor memory; P enters as three bf16 parts, so the
 * product keeps fp32 accuracy. Replaces the dense per-step gather of the assembled
 * factorised weights (network_simulators/network.py:731-752 `_assemble`, then
 * conductance/kernels.py:657-689). */
typedef struct {
    int32_t B, N, KP;
    const uint16_t *V;  /* (N, 64) bf16 */
    const float *P;     /* (B, KP, 64) */
    float *D;           /* (KP, B, N) */
    int32_t *err;       /* device error word (WT_ERR_BARRIER if an MMA never completed) */
} WtLowRankProduct;

int wt_lowrank_product(const WtLowRankProduct *a, void *stream);

/* A network whose recurrent pathways are all factorised, W_k = U_k V^T (k < KP <= 2, one
 * shared V of rank <= 64), driven by one input column per neuron (n_in == N, input weight
 * w_in[n]); conductance LIF with refractoriness, S <= 4 synapse channels (exact, one per
 * synapse type). */
typedef struct {
    int32_t B, N, S, KP;
    const float *theta, *U_reset, *E_L, *C_m, *beta;
    /* (WT_F_CURRENT, network_simulators/current/dynamics.py:116-205: E_L holds U_rest,
     * C_m the resistance R, E_syn the synapse types' signs, adapt and adapt_decay the
     * adaptation current's rise and decay; each channel a single exponential, decay_d
     * and jump_d 1) */ /* (N) */
    const int32_t *n_ref;                            /* (N) or NULL */
    float decay_r[WT_MAX_CHANNELS], decay_d[WT_MAX_CHANNELS];
    float jump_r[WT_MAX_CHANNELS], jump_d[WT_MAX_CHANNELS];
    float E_syn[WT_MAX_CHANNELS], g_clip[WT_MAX_CHANNELS];
    float dt;
    const uint16_t *U;      /* (N, 64) bf16: each neuron's U row as a source (zero if none) */
    const int8_t *path_of;  /* (N): the pathway a neuron is a source of, -1: none */
    const uint16_t *V;      /* (N, 64) bf16 */
    const float *scale;     /* (KP + 1, N): each pathway's target scale, then the input's */
    const float *w_in;      /* (N) */
    uint32_t made;          /* bit 8 k + s: pathway k (k == KP: the input) drives channel s */
} WtLowRankNet;

/* One forward run of T steps of a WtLowRankNet (same state and output layout as
 * WtForward: v (B, N), g (B, 2, S, N), counter (B, N), x and spikes (B, T_total, N)). */
typedef struct {
    int32_t T, T_total, t0;
    float *v, *g;
    int32_t *counter;       /* when n_ref */
    const float *x;
    float *spikes;
    float *P;               /* scratch (3, B, KP, 64) */
    uint32_t *barrier;      /* (64), zeroed by the call */
    int32_t *err;           /* device error word */
} WtLowRankRun;

/* Simulate T steps of a factorised network: one persistent kernel, the recurrent input
 * of every step a tcgen05.mma product with its accumulator in tensor memory, read by the
 * same kernel's membrane update (network_simulators/network.py:731-752 and
 * conductance/engine.py:306-355 in the reference: a dense W assembled, then gathered). */
int wt_lowrank_forward(const WtLowRankNet *net, const WtLowRankRun *run, void *stream);

/* Spikes as bits, the form in which the runners move spikes between host and device: a
 * spike tensor of `rows` rows (the product of all but its last dimension) of n spikes,
 * each row packed into ceil(n / 8) bytes, spike i of a row in bit i % 8 (least
 * significant first) of byte i / 8 (numpy's packbits(x, axis=-1, bitorder="little")).
 * An eighth of the bytes of the bool spike tensors that the reference's data path copies
 * whole (snn_runners/chunks.py:19-25 `to_device`, used by `Prefetcher` at
 * chunks.py:28-70; snn_runners/inference_runner.py:111-150 `_Stager`), a thirty-second of
 * a float tensor's. */
#define WT_SPIKES_F32 0 /* float, 0 or 1 */
#define WT_SPIKES_U8 1  /* bool or uint8, 0 or 1 */
typedef struct {
    int64_t rows;
    int32_t n;
    int32_t kind;           /* WT_SPIKES_F32 or WT_SPIKES_U8 */
    uint8_t *bits;          /* (rows, ceil(n / 8)) */
    void *spikes;           /* (rows, n) of `kind` */
    int32_t *err;           /* wt_pack_spikes: device error word, or null */
} WtSpikeBits;

/* bits -> spikes (0 or 1 of `kind`), on the device. */
int wt_unpack_spikes(const WtSpikeBits *a, void *stream);

/* spikes -> bits, on the device: a spike is any value other than 0; a value other than
 * 0 or 1 (a count the bits cannot hold) records WT_ERR_ARGS in `err`. */
int wt_pack_spikes(const WtSpikeBits *a, void *stream);

/* Reading back: a static description of the last host-side error on this thread. */
const char *wt_last_error(void);

/* The version of this ABI. */
int wt_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif
