// The extern "C" entry points of include/wiretorch_b200.h: argument checks, workspace
// sizes, and the launches. Nothing here allocates or synchronises.
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace wt {
long long forward_x_row(int N);
cudaError_t launch_forward_s(const WtNet &net, const WtForward &run, const WtWorkspace &ws,
                             cudaStream_t st, int grid_cap);
cudaError_t launch_backward(const WtNet &net, const WtBackward &bw, cudaStream_t st);
cudaError_t launch_edge_grads(const WtNet &net, const WtEdgeGrads &eg, cudaStream_t st);
long long edge_grads_fired_words(const WtNet &net, int T);
int edge_grads_slice_trials(const WtNet &net, int T);
cudaError_t launch_lowrank_product(const WtLowRankProduct &a, cudaStream_t st);
cudaError_t launch_lowrank_forward(const WtLowRankNet &net, const WtLowRankRun &run, cudaStream_t st);
cudaError_t launch_recurrent_carry(const WtNet &net, const WtRecurrentCarry &rc, cudaStream_t st);
cudaError_t launch_filter(const WtFilterArgs &f, cudaStream_t st);
cudaError_t launch_filter_grad(const WtFilterGradArgs &f, cudaStream_t st);
cudaError_t launch_van_rossum(const WtVanRossumArgs &a, cudaStream_t st);
cudaError_t launch_van_rossum_grad(const WtVanRossumGradArgs &a, cudaStream_t st);
cudaError_t launch_unpack_spikes(const WtSpikeBits &a, cudaStream_t st);
cudaError_t launch_pack_spikes(const WtSpikeBits &a, cudaStream_t st);
cudaError_t launch_fold(const WtNet &net, const float *w_raw, const int32_t *chunk_path, const float *scale,
                        const float *jf, const float *fx_scale, uint64_t *out, cudaStream_t st);
}

namespace {
thread_local char g_error[512] = "";

int fail(int code, const char *fmt, const char *detail = "") {
    std::snprintf(g_error, sizeof g_error, fmt, detail);
    return code;
}

int launch_status(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return WT_OK;
    std::snprintf(g_error, sizeof g_error, "%s: %s", what, cudaGetErrorString(e));
    return WT_ERR_LAUNCH;
}

int check_net(const WtNet *n) {
    if (!n) return fail(WT_ERR_ARGS, "net is null%s");
    if (n->B <= 0 || n->N <= 0 || n->n_in < 0) return fail(WT_ERR_ARGS, "bad sizes%s");
    if (n->S < 1 || n->S > WT_MAX_CHANNELS) return fail(WT_ERR_UNSUPPORTED, "S must be in 1..8%s");
    if (n->C < 1 || n->C > WT_MAX_CHANNELS) return fail(WT_ERR_UNSUPPORTED, "C must be in 1..8%s");
    if (n->N >= (1 << 27)) return fail(WT_ERR_UNSUPPORTED, "N must be below 2^27%s");
    if ((unsigned long long)n->B * (((unsigned long long)n->n_in + 31) & ~31ull) + 32 >= (1ull << 32))
        return fail(WT_ERR_UNSUPPORTED, "trials x input columns must be below 2^32%s");
    if ((unsigned long long)n->B * (unsigned long long)(n->n_chunks > 0 ? n->n_chunks : 1) >= (1ull << 32))
        return fail(WT_ERR_UNSUPPORTED, "trials x chunks must be below 2^32%s");
    if (!n->theta || !n->U_reset || !n->E_L || !n->C_m || !n->beta)
        return fail(WT_ERR_ARGS, "missing neuron tables%s");
    if (!n->src_slot || !n->slot_chunk || !n->src_chunk || (n->n_chunks && (!n->chunk_desc || !n->edge_col)))
        return fail(WT_ERR_ARGS, "missing connectivity%s");
    if (n->N_src != 0 && (n->N_src < n->N || n->N_src >= (1 << 27))) return fail(WT_ERR_ARGS, "bad N_src%s");
    return WT_OK;
}
}  // namespace

namespace wt {
// Records `message` as the last error (wt_last_error) and returns `code`; for the entry
// points defined in other files.
int set_last_error(int code, const char *message) { return fail(code, "%s", message); }
}  // namespace wt

extern "C" {

const char *wt_last_error(void) { return g_error; }

int wt_abi_version(void) { return 1; }

int wt_workspace_bytes(const WtNet *net, int32_t T, int64_t bytes[6]) {
    int rc = check_net(net);
    if (rc) return rc;
    const long long cap = (long long)net->B * (net->n_chunks > 0 ? net->n_chunks : 1);
    bytes[0] = 2LL * net->C * net->B * wt::forward_x_row(net->N) * 8;  // X (rows padded to 32)
    bytes[1] = 2LL * cap * (long long)sizeof(WtEvent);  // ev
    bytes[2] = ((long long)T + 1) * 4;                // ev_count
    bytes[3] = 64 * 4;                                // barrier
    bytes[4] = 4;                                     // err
    bytes[5] = 2 * 8;                                 // edges
    return WT_OK;
}

int wt_fold_weights(const WtNet *net, const float *w_raw, const int32_t *chunk_path, const float *scale,
                    const float *jf, const float *fx_scale, uint64_t *edge_cw_out, void *stream) {
    int rc = check_net(net);
    if (rc) return rc;
    if (net->n_chunks && (!w_raw || !chunk_path || !scale || !jf || !fx_scale || !edge_cw_out || !net->edge_col))
        return fail(WT_ERR_ARGS, "missing fold buffers%s");
    return launch_status(wt::launch_fold(*net, w_raw, chunk_path, scale, jf, fx_scale, edge_cw_out,
                                         (cudaStream_t)stream),
                         "fold");
}

}  // extern "C"

namespace wt {
// Every argument check of wt_forward, with no device work: WT_OK if wt_forward would
// launch (or return at once for T = 0), else its error code with wt_last_error set.
int check_forward(const WtNet *net, const WtForward *run, const WtWorkspace *ws) {
    int rc = check_net(net);
    if (rc) return rc;
    if (!run || !ws) return fail(WT_ERR_ARGS, "run or workspace is null%s");
    if (run->T < 0 || run->t0 < 0 || run->t0 + run->T > run->T_total)
        return fail(WT_ERR_ARGS, "steps out of range%s");
    if (run->T > (1 << 24)) return fail(WT_ERR_UNSUPPORTED, "at most 2^24 steps a call%s");  // the barrier's count
    if (!run->v || !run->g || !run->spikes || (net->n_in && !run->x))
        return fail(WT_ERR_ARGS, "missing state or output%s");
    const int f = run->flags;
    if ((f & WT_F_REFRACTORY) && (!run->counter || !net->n_ref)) return fail(WT_ERR_ARGS, "refractory buffers%s");
    if ((f & WT_F_ADAPT) && (!run->g_a || !net->adapt || !net->adapt_decay || (!net->E_adapt && !(f & WT_F_CURRENT))))
        return fail(WT_ERR_ARGS, "adaptation buffers%s");
    if ((f & WT_F_CURRENT) && (f & (WT_F_PARTITION | WT_F_MG_BLOCK)))
        return fail(WT_ERR_UNSUPPORTED, "current-based neurons: no neuron partition or Mg block%s");
    if ((f & WT_F_SAMPLE) && !run->noise) return fail(WT_ERR_ARGS, "noise buffer%s");
    if ((f & WT_F_GATED) && (!run->gating || !net->slot_gate || !net->slot_row || !net->gate_params ||
                             !net->gate_cols))
        return fail(WT_ERR_ARGS, "gating buffers%s");
    if ((f & WT_F_SAVE) && (!run->v_saved || !run->G_saved || !run->spike_bits ||
                            ((f & WT_F_REFRACTORY) && !run->held_bits) ||
                            ((f & WT_F_ADAPT) && !run->a_saved) || ((f & WT_F_GATED) && !run->f_saved)))
        return fail(WT_ERR_ARGS, "saved-tensor buffers%s");
    if ((f & WT_F_SAVE_INPUT) && !run->X_saved) return fail(WT_ERR_ARGS, "saved-input buffer%s");
    if ((f & WT_F_PROB) && !run->prob) return fail(WT_ERR_ARGS, "probability buffer%s");
    if ((f & WT_F_TRACK) && (!run->track_v || !run->track_I || !run->track_g ||
                             ((f & WT_F_ADAPT) && !run->track_a)))
        return fail(WT_ERR_ARGS, "tracking buffers%s");
    if (net->n_chunks && !net->edge_cw) return fail(WT_ERR_ARGS, "missing folded edges%s");
    if (!ws->X || !ws->ev || !ws->ev_count || !ws->barrier || !ws->err)
        return fail(WT_ERR_ARGS, "workspace buffers%s");
    if (ws->ev_cap < (long long)net->B * net->n_chunks) return fail(WT_ERR_ARGS, "event capacity too small%s");
    if (((uintptr_t)ws->X & 15) || ((uintptr_t)ws->ev & 15))
        return fail(WT_ERR_ARGS, "workspace X and ev must be 16-byte aligned%s");
    if (f & WT_F_PARTITION) {
        if (f & (WT_F_SAVE | WT_F_SAVE_INPUT)) return fail(WT_ERR_UNSUPPORTED, "a partitioned run is forward only%s");
        if (run->n_ranks < 1 || run->n_ranks > 8 || run->rank < 0 || run->rank >= run->n_ranks || !run->words ||
            !run->progress)
            return fail(WT_ERR_ARGS, "bad partition%s");
        for (int r = 0; r < run->n_ranks; r++)
            if (!run->peer_words[r] || !run->peer_progress[r]) return fail(WT_ERR_ARGS, "missing peer buffers%s");
        if (run->push_reserve) {  // pushed events
            if ((f & WT_F_GATED) && !run->amps) return fail(WT_ERR_ARGS, "a gated run pushes its events only with owner-stepped gates%s");
            if (!run->pull_ev || !run->pull_count) return fail(WT_ERR_ARGS, "missing inbound event area%s");
            for (int r = 0; r < run->n_ranks; r++)
                if (!run->push_src_chunk[r] || !run->push_chunk_desc[r] || !run->push_ev[r] || !run->push_count[r])
                    return fail(WT_ERR_ARGS, "missing push tables%s");
        }
        if (run->amps) {  // owner-stepped gates
            if (!(f & WT_F_GATED) || !net->src_gate) return fail(WT_ERR_ARGS, "amplitudes need a gated net with src_gate%s");
            for (int r = 0; r < run->n_ranks; r++)
                if (!run->peer_amps[r]) return fail(WT_ERR_ARGS, "missing peer amplitude buffers%s");
        }
        const int n_src = net->N_src ? net->N_src : net->N;
        if (run->word0 < 0 || (long long)run->word0 * 32 + net->N > ((long long)n_src + 31) / 32 * 32)
            return fail(WT_ERR_ARGS, "this rank's neurons lie outside the sources%s");
    } else if (net->N_src && net->N_src != net->N) {
        return fail(WT_ERR_ARGS, "a net with other neurons' sources needs WT_F_PARTITION%s");
    }
    return WT_OK;
}
}  // namespace wt

extern "C" {

int wt_forward(const WtNet *net, const WtForward *run, const WtWorkspace *ws, void *stream) {
    const int rc = wt::check_forward(net, run, ws);
    if (rc) return rc;
    if (run->T == 0) return WT_OK;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = cudaMemsetAsync(ws->barrier, 0, 64 * 4, st);
    if (e != cudaSuccess) return launch_status(e, "barrier reset");
    return launch_status(wt::launch_forward_s(*net, *run, *ws, st, 0), "forward");
}

int wt_backward(const WtNet *net, const WtBackward *bw, void *stream) {
    int rc = check_net(net);
    if (rc) return rc;
    if (net->N_src && net->N_src != net->N) return fail(WT_ERR_UNSUPPORTED, "no backward pass for a partitioned net%s");
    if (!bw || bw->T < 0) return fail(WT_ERR_ARGS, "bad backward arguments%s");
    if (!bw->grad_spikes || !bw->v_saved || !bw->G_saved || !bw->spike_bits || !(bw->Q || bw->QT))
        return fail(WT_ERR_ARGS, "missing saved tensors%s");
    if (bw->QT && (bw->adj || bw->t_lo != 0 || (bw->t_hi != 0 && bw->t_hi != bw->T) ||
                   ((uintptr_t)bw->QT & 15)))
        return fail(WT_ERR_ARGS, "target-major adjoints need a whole scan and a 16-byte aligned buffer%s");
    const int f = bw->flags, w = bw->wants;
    if ((f & WT_F_REFRACTORY) && !bw->held_bits) return fail(WT_ERR_ARGS, "missing refractory bits%s");
    if ((f & WT_F_ADAPT) && (!bw->a_saved || !net->adapt_decay || (!net->E_adapt && !(f & WT_F_CURRENT))))
        return fail(WT_ERR_ARGS, "missing adaptation%s");
    if ((f & WT_F_CURRENT) && ((bw->wants & (WT_W_E_SYN | WT_W_JUMP | WT_W_E_ADAPT)) || (f & WT_F_MG_BLOCK)))
        return fail(WT_ERR_UNSUPPORTED, "current-based neurons: no sign, jump or E_adapt gradients%s");
    if ((f & WT_F_CURRENT) && (f & WT_F_ADAPT) && !net->adapt) return fail(WT_ERR_ARGS, "missing adaptation%s");
    if ((f & WT_F_CURRENT) && (bw->wants & WT_W_DECAY) && !bw->g_init)
        return fail(WT_ERR_ARGS, "decay gradients need the currents entering the run%s");
    if ((w & (WT_W_DECAY | WT_W_JUMP)) && !bw->X_saved) return fail(WT_ERR_ARGS, "missing saved input%s");
    if ((w & WT_W_DECAY) && !bw->g_init) return fail(WT_ERR_ARGS, "missing initial conductances%s");
    float *const outs[11] = {bw->g_theta, bw->g_reset, bw->g_E_L, bw->g_C_m, bw->g_beta, bw->g_E_syn,
                             bw->g_decay, bw->g_jump, bw->g_adapt, bw->g_adapt_decay, bw->g_E_adapt};
    for (int i = 0; i < 11; i++)
        if ((w >> i & 1) && !outs[i]) return fail(WT_ERR_ARGS, "missing gradient output%s");
    if (bw->T == 0) return WT_OK;
    return launch_status(wt::launch_backward(*net, *bw, (cudaStream_t)stream), "backward");
}

int wt_edge_grads(const WtNet *net, const WtEdgeGrads *eg, void *stream) {
    int rc = check_net(net);
    if (rc) return rc;
    if (net->N_src && net->N_src != net->N) return fail(WT_ERR_UNSUPPORTED, "no backward pass for a partitioned net%s");
    if (!eg || eg->T < 0 || !eg->chunk_path || !eg->jf) return fail(WT_ERR_ARGS, "bad edge arguments%s");
    if (!eg->Q && (eg->g_x || !eg->QT)) return fail(WT_ERR_ARGS, "missing adjoints%s");
    if (eg->QT && (eg->g_scale || eg->g_w) &&
        (!eg->in_ptr || !eg->in_edge || !eg->in_src || !eg->in_path || (net->slot_gate && !eg->in_fcol) ||
         !eg->ev_start || !eg->ev || eg->ev_cap < 1 || eg->ev_cap >= (1LL << 31) || !eg->in_acc || !eg->err ||
         wt::edge_grads_slice_trials(*net, eg->T) < 1 || ((uintptr_t)eg->QT & 15)))
        return fail(WT_ERR_ARGS, "missing in-edge tables or event scratch%s");
    if ((eg->g_scale || eg->g_w) && (!eg->spike_bits || (net->n_in && !eg->x)))
        return fail(WT_ERR_ARGS, "missing events%s");
    if (eg->g_scale && !eg->w_raw) return fail(WT_ERR_ARGS, "missing raw weights%s");
    if ((eg->g_w || eg->g_x) && !eg->scale) return fail(WT_ERR_ARGS, "missing scale%s");
    if (eg->g_x && !eg->w_raw) return fail(WT_ERR_ARGS, "missing raw weights%s");
    if (net->slot_gate && !eg->f_saved) return fail(WT_ERR_ARGS, "missing gating factors%s");
    if ((eg->g_scale || eg->g_w) && (!eg->fired || !eg->work)) return fail(WT_ERR_ARGS, "missing edge scratch%s");
    if ((long long)net->B * eg->T >= (1LL << 31)) return fail(WT_ERR_UNSUPPORTED, "trials x steps must be below 2^31%s");
    if (eg->T == 0) return WT_OK;
    return launch_status(wt::launch_edge_grads(*net, *eg, (cudaStream_t)stream), "edge gradients");
}

int64_t wt_edge_grads_scratch_words(const WtNet *net, int32_t T) {
    if (check_net(net) || T < 0) return -1;
    return wt::edge_grads_fired_words(*net, T);
}

int32_t wt_edge_grads_slice_trials(const WtNet *net, int32_t T) {
    if (check_net(net) || T < 0) return 0;
    return wt::edge_grads_slice_trials(*net, T);
}

static int check_spike_bits(const WtSpikeBits *a) {
    if (!a || a->rows < 0 || a->n < 0 || (a->kind != WT_SPIKES_F32 && a->kind != WT_SPIKES_U8))
        return fail(WT_ERR_ARGS, "bad spike-bit arguments%s");
    if (a->rows && a->n && (!a->bits || !a->spikes)) return fail(WT_ERR_ARGS, "missing spike or bit buffer%s");
    return WT_OK;
}

int wt_unpack_spikes(const WtSpikeBits *a, void *stream) {
    const int rc = check_spike_bits(a);
    if (rc) return rc;
    return launch_status(wt::launch_unpack_spikes(*a, (cudaStream_t)stream), "unpack spikes");
}

int wt_pack_spikes(const WtSpikeBits *a, void *stream) {
    const int rc = check_spike_bits(a);
    if (rc) return rc;
    return launch_status(wt::launch_pack_spikes(*a, (cudaStream_t)stream), "pack spikes");
}

int wt_filter_forward(const WtFilterArgs *f, void *stream) {
    if (!f || f->B < 0 || f->T < 0 || f->N < 0 || (f->B && f->T && f->N && !f->x))
        return fail(WT_ERR_ARGS, "bad filter arguments%s");
    return launch_status(wt::launch_filter(*f, (cudaStream_t)stream), "filter");
}

int wt_filter_backward(const WtFilterGradArgs *f, void *stream) {
    if (!f || f->B < 0 || f->T < 0 || f->N < 0 || (f->B && f->T && f->N && (!f->grad_smooth || !f->grad_x)))
        return fail(WT_ERR_ARGS, "bad filter-gradient arguments%s");
    return launch_status(wt::launch_filter_grad(*f, (cudaStream_t)stream), "filter gradient");
}

int wt_van_rossum_forward(const WtVanRossumArgs *a, void *stream) {
    if (!a || a->B < 0 || a->T < 0 || a->N < 0) return fail(WT_ERR_ARGS, "bad loss arguments%s");
    if (a->B && a->N && (!a->last || !a->partial || (a->T && (!a->x || !a->y || !a->err))))
        return fail(WT_ERR_ARGS, "missing loss buffers%s");
    return launch_status(wt::launch_van_rossum(*a, (cudaStream_t)stream), "van Rossum loss");
}

int wt_van_rossum_backward(const WtVanRossumGradArgs *a, void *stream) {
    if (!a || a->B < 0 || a->T < 0 || a->N < 0) return fail(WT_ERR_ARGS, "bad loss-gradient arguments%s");
    if (a->B && a->N && a->T && (!a->err || !a->grad_loss || !a->grad_x))
        return fail(WT_ERR_ARGS, "missing loss-gradient buffers%s");
    return launch_status(wt::launch_van_rossum_grad(*a, (cudaStream_t)stream), "van Rossum loss gradient");
}

int wt_lowrank_product(const WtLowRankProduct *a, void *stream) {
    if (!a || a->B < 0 || a->N < 0 || a->KP < 1 || a->KP > 4) return fail(WT_ERR_ARGS, "bad low-rank product arguments%s");
    if (!a->B || !a->N) return WT_OK;
    if (!a->V || !a->P || !a->D || !a->err) return fail(WT_ERR_ARGS, "missing low-rank product buffers%s");
    if (((uintptr_t)a->V & 15) || ((uintptr_t)a->P & 15)) return fail(WT_ERR_ARGS, "V and P must be 16-byte aligned%s");
    return launch_status(wt::launch_lowrank_product(*a, (cudaStream_t)stream), "low-rank product");
}

int wt_lowrank_forward(const WtLowRankNet *net, const WtLowRankRun *run, void *stream) {
    if (!net || !run) return fail(WT_ERR_ARGS, "net or run is null%s");
    if (net->B <= 0 || net->N <= 0 || net->N >= (1 << 27)) return fail(WT_ERR_ARGS, "bad sizes%s");
    if (net->S < 1 || net->S > 4) return fail(WT_ERR_UNSUPPORTED, "the factorised kernel carries 1..4 channels%s");
    if (net->KP < 1 || net->KP > 2) return fail(WT_ERR_UNSUPPORTED, "the factorised kernel takes 1 or 2 pathways%s");
    if (!net->theta || !net->U_reset || !net->E_L || !net->C_m || !net->beta || !net->U || !net->path_of ||
        !net->V || !net->scale || !net->w_in)
        return fail(WT_ERR_ARGS, "missing network tables%s");
    if (((uintptr_t)net->U & 15) || ((uintptr_t)net->V & 15)) return fail(WT_ERR_ARGS, "U and V must be 16-byte aligned%s");
    if (run->T < 0 || run->t0 < 0 || run->t0 + run->T > run->T_total) return fail(WT_ERR_ARGS, "steps out of range%s");
    if (run->T > (1 << 24)) return fail(WT_ERR_UNSUPPORTED, "at most 2^24 steps a call%s");  // the barrier's count
    if (!run->v || !run->g || !run->spikes || !run->P || !run->barrier || !run->err || (run->T && !run->x) ||
        (net->n_ref && !run->counter))
        return fail(WT_ERR_ARGS, "missing run buffers%s");
    if ((uintptr_t)run->P & 15) return fail(WT_ERR_ARGS, "P must be 16-byte aligned%s");
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = cudaMemsetAsync(run->barrier, 0, 64 * 4, st);
    if (e != cudaSuccess) return launch_status(e, "barrier reset");
    return launch_status(wt::launch_lowrank_forward(*net, *run, st), "factorised forward");
}

int wt_recurrent_carry(const WtNet *net, const WtRecurrentCarry *rc, void *stream) {
    int r = check_net(net);
    if (r) return r;
    if (!rc || rc->t < 0 || rc->t >= rc->T || !rc->adj || !rc->Qt || !rc->R)
        return fail(WT_ERR_ARGS, "bad recurrent-carry arguments%s");
    if (net->n_chunks && !net->edge_cw) return fail(WT_ERR_ARGS, "missing folded edges%s");
    if (net->slot_gate && !rc->f_saved) return fail(WT_ERR_ARGS, "missing gating factors%s");
    return launch_status(wt::launch_recurrent_carry(*net, *rc, (cudaStream_t)stream), "recurrent carry");
}

}  // extern "C"
