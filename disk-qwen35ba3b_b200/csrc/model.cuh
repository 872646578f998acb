// model.cuh -- the HBM-resident expert pool and per-layer trunk weights
// (the device-side replacement of the reference's disk pool + LRU cache,
// src/cache.c:140-214 / src/st.c:127-180), and the MoE-step workspace.
#pragma once

#include "common.cuh"
#include "../../include/ds4f/gpu_cuda.h"

namespace ds4f {

struct SlotCache;                // stream.cu: the expert-cache policy

struct ModelDesc {
    int fmt;              // DS4F_FMT_FP8 or DS4F_FMT_MXFP4 (routed experts)
    int n_layers;
    int hidden;           // H
    int moe_inter;        // M
    int n_experts;        // E
    int topk;             // K
    int renorm;           // norm_topk_prob
    int expert_first;     // expert shard [first, first + count) held here
    int expert_count;
    int router_exact;     // 1: every router logit in the reference's exact
                          //    sequential fp32 order (slow, bit-exact weights)
};

// Expert slot layout: gate, up, down, each values then scales -- the order
// in which the engine reads an expert's tensor entries (src/moe.c:598-605).
// The converter writes sorted-name order (down, gate, up) into its pool file;
// poolfile.cu places those by name.
struct SlotLayout {
    int64_t rel_v[3], rel_s[3], nbytes;
};

// Per-layer trunk (bf16) offsets, in elements from the layer base.
struct TrunkLayout {
    int64_t norm, router, sh_gate, sh_up, sh_down, sh_gw, n;
};

// Device workspace for one token's layer step.
struct Work {
    float *xin;           // [H] normed input
    double *S;            // [E] router logits (exact-sum in double)
    double *Bnd;          // [E] bound |reference fp32 logit - S|
    int *idx;             // [K] selected experts, selection order
    float *w;             // [K] routing weights (after renorm)
    float *chain;         // [(K+1) M] silu(g)*u per selection, shared last
    float *sgate;         // [1] shared_expert_gate logit
    float *acc;           // [H] moe output before the residual
    unsigned *diag;       // [4] 0: layers routed, 1: exact fallbacks, 2: error
                          //     code of the persistent kernel, 3: its CTA
    uint64_t *st_ll;      // [H] persistent kernel: tagged state words
    uint64_t *sb_ll;      // [E][4] tagged router logits and interval ends (fp32)
    uint64_t *ch_ll;      // [(K+1) M + 1] tagged chains + shared-gate logit
};

struct Model {
    ModelDesc d;
    SlotLayout slot;
    TrunkLayout tr;
    int device;
    uint8_t *pool;        // [L][count] slots
    uint16_t *trunk;      // [L] trunk blocks
    Work w;
    void *ws_base;
    float *state_dev;     // [Bmax H] staging for the host-buffer API
    int *idx_dev;
    float *w_dev;
    int bmax;
    cudaStream_t stream;
    cudaGraphExec_t graph;       // captured stack step (B = 1)
    float *graph_state;
    int graph_ok;
    int path;                    // 0 auto, 1 per-layer kernels, 2 persistent
    unsigned long long *trace;   // optional phase stamps of the persistent kernel
    int64_t trace_n;
    int epoch;                   // last persistent launch's tag epoch
    int64_t wait_limit;          // persistent kernel: polls before a wait gives up (0: default)
    int stall_cta, stall_t;      // test hook of the persistent kernel (-1: off)
    int stall_peer_t;            // test hook of the fused multi-GPU step (-1: off)
    int *log_idx;                // route log of the persistent kernel (log_n layer-steps
    float *log_w, *log_state;    //   of the next launch): selections, weights, output state
    int log_n;
    void *log_base;
    void *pf_ws;                 // batched-prefill workspace (prefill.cu), grown on demand
    size_t pf_bytes;
    unsigned *pf_err_h;          // pinned copy of the prefill pipeline error word,
                                 //   written after each asynchronous step
    // streaming pool (ds4f_gpu_model_create_streaming): the experts live in
    // a pinned host copy of the packed pool; `pool` is an arena of
    // stream_slots slots managed by `cache`
    const uint8_t *host_pool;
    int stream_slots;
    SlotCache *cache;
    int *slot_dev;               // [K] arena slots of the current selections
    int *idx_h, *slot_h;         // [K] pinned host copies
    cudaGraphExec_t bgraph;      // captured batched decode step (prefill.cu), valid for
    float *bgraph_state;         //   these states, batch and workspace
    int bgraph_B;
    void *bgraph_ws;
    void *ep;                    // expert-parallel state (ep.cu), when attached
};

int slot_layout(int fmt, int H, int M, SlotLayout *s);
int trunk_layout(int H, int M, int E, TrunkLayout *t);

// One token through layer L: state (device, [H]) updated in place; idx / w
// (device, [K]) optional copies of the routing.
int moe_layer_launch(Model *m, int L, float *state, int *idx_out,
                     float *w_out, cudaStream_t st);
// The same with the expert-parallel options: partial = this model's shard
// only, acc_out gets the partial sum and the state is not updated;
// add_shared includes the shared expert.
int moe_layer_launch_ex(Model *m, int L, float *state, int *idx_out, float *w_out, float *acc_out,
                        bool partial, bool add_shared, cudaStream_t st);
// The certified router and top-K of layer L for B tokens at once (moe.cu):
// states [B][H] -> xin [B][H], S / Bnd [B][E], idx / w [B][K] (device).
int route_batch_launch(Model *m, int L, const float *states, int B, float *xin, double *S, double *Bnd,
                       int *idx, float *w, cudaStream_t st);

// Whole decode steps in one persistent cooperative launch (decode.cu).
// Several GPUs, one persistent launch each (decode.cu): every rank's
// [2][K][H] tagged down-output words (out[rank] its own, the others peer
// mappings) and the launch-epoch counter every rank advances in step.
struct DecodePeers {
    uint64_t *out[8];
    int rank, world;
    int *epoch;
    int64_t *lsteps;             // layer-steps of every fused launch so far (buffer parity)
    int split_sel;               // 1: whole pool on every GPU, selections split by index
};
bool decode_eligible(const Model *m);                         // the whole pool on this GPU
bool decode_eligible_ep(const Model *m, int rank, int world, int split_sel);  // shard or whole pool
int decode_launch(Model *m, float *state, int n_steps, cudaStream_t st, const DecodePeers *peers = nullptr);

// GPU copy of the seeded fixture generator (oracle/fixture.c): fills the
// model's trunk and expert shard.
int synth_model(Model *m, uint64_t seed, double sigma, cudaStream_t st);
int synth_f32(float *dst, int64_t n, uint64_t key, double sigma, cudaStream_t st);

// Streaming models (stream.cu): the current layer's selections (m->w.idx)
// looked up in the slot cache, misses copied in from the host pool, their
// slots uploaded to m->slot_dev; ordered on st.
int stream_fetch(Model *m, int L, cudaStream_t st);
SlotCache *slot_cache_new(int n);
void slot_cache_delete(SlotCache *c);
void slot_cache_stats(const SlotCache *c, int64_t *req, int64_t *hit, int64_t *drop, int64_t *fetched);

// Batched prefill of one layer (prefill.cu): states [T][H] in/out, routing
// sel / w [T][K] (global expert ids; ids outside this shard are skipped).
// first_layer resets the pipeline error word; last_layer synchronises and
// reports it. acc_out: expert-parallel partial -- the combine goes to
// acc_out [T][H] and the states are left alone; add_shared: include the
// shared expert (one rank of a partition).
int prefill_layer(Model *m, int L, float *states, int T, const int *sel, const float *w,
                  cudaStream_t st, bool first_layer, bool last_layer, float *acc_out, bool add_shared);

// Batched decode of one layer (prefill.cu): the certified router and top-K
// of B tokens, then the grouped tensor-core chain; acc_out / add_shared as
// prefill_layer; async: errors reported by a later call.
int decode_batch_layer(Model *m, int L, float *states, int B, int *idx, float *w, cudaStream_t st,
                       bool first_layer, bool last_layer, float *acc_out, bool add_shared, bool async);
// Size the batched-prefill workspace for T tokens now (it is otherwise grown
// on demand), and report (synchronising st) a pipeline wait that gave up
// since the last check.
int prefill_pre_size(Model *m, int T);
int prefill_check(Model *m, cudaStream_t st);
// Expert parallelism (ep.cu): release the model's communicator and buffers.
void ep_free(Model *m);

// Enqueue `fn` on the model stream ordered after the caller's stream, and
// make the caller's stream wait for it (timing on the caller's stream then
// brackets the work).
template <typename F>
int on_model_stream(Model &m, void *stream, F fn) {
    cudaStream_t cs = (cudaStream_t)stream;
    cudaEvent_t e0, e1;
    DS4F_CUDA(cudaEventCreateWithFlags(&e0, cudaEventDisableTiming));
    DS4F_CUDA(cudaEventCreateWithFlags(&e1, cudaEventDisableTiming));
    int rc = 0;
    if (cudaEventRecord(e0, cs) != cudaSuccess || cudaStreamWaitEvent(m.stream, e0, 0) != cudaSuccess) rc = -1;
    if (!rc) rc = fn(m.stream);
    if (cudaEventRecord(e1, m.stream) != cudaSuccess || cudaStreamWaitEvent(cs, e1, 0) != cudaSuccess) rc = -1;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (rc && !ds4f_gpu_last_error()[0]) set_error("stream ordering failed");
    return rc;
}

inline const uint8_t *expert_ptr(const Model *m, int L, int e) {
    return m->pool + ((int64_t)L * m->d.expert_count + (e - m->d.expert_first)) *
                         m->slot.nbytes;
}

}  // namespace ds4f

// The C ABI's opaque model handle.
struct Ds4fGpuModel {
    ds4f::Model m;
};
