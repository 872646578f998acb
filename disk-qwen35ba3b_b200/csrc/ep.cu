// ep.cu -- expert parallelism across the GPUs of one node, inside the
// library: one process (or host thread) per GPU, a NCCL communicator per
// model, and the data plane behind the C ABI (no torch on it).
//
// Partition (as the pool invites it: experts are independent slots,
// src/st.c:127-180): rank r of N holds experts [r E/N, (r+1) E/N) of every
// layer and the whole bf16 trunk (router, norm, shared expert).
//
// Decode (ds4f_gpu_ep_stack_dev): the B token states are the same on every
// rank. Per layer every rank routes them on the full router (the certified
// top-K gives the same bits everywhere), runs the selections its experts
// received, rank 0 also the shared expert, and the partial combines are
// summed by one all-reduce of acc [B][H]; then state += acc (the residual,
// src/moe.c:1424). A whole step (every layer's kernels and all-reduces) is
// one CUDA graph, replayed.
//
// Prefill (ds4f_gpu_ep_prefill): the chunk's tokens are partitioned, each
// rank holds its own T_r states and their routing. Per layer:
//   1. dispatch: each token's state row, with its selections and weights,
//      goes to every rank that owns one of its selected experts (grouped
//      send/recv, one message per peer);
//   2. each rank runs the batched tensor-core step on the rows it received
//      (its own experts only, the reference's grouping by expert,
//      src/moe.c:1516-1530), giving each row its partial combine;
//   3. combine: the partials go back to the token's owner, which sums them
//      in rank order, adds the shared expert it ran on its own tokens and
//      the residual (selection-order combine per rank, src/moe.c:1614-1630).
// Which rows go where depends on the routing only, so all layers' plans
// are made once on the host at the start (ds4f_ep_plan_dispatch) and the
// layers then run without a host synchronisation.
//
// NCCL is loaded when a model attaches (dlopen of libnccl.so.2, the library
// the process already uses if one is loaded): single-GPU users need none.
// A collective waits for every peer; a peer that is lost leaves it waiting
// until ds4f_gpu_ep_abort (from another host thread) aborts the
// communicator.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "model.cuh"

namespace ds4f {

int prefill_pre_size(Model *m, int T);

namespace {

struct NcclApi {
    bool ok = false;
    std::string why;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) { api.why = std::string("cannot load libnccl.so.2: ") + dlerror(); return; }
        bool all = true;
        auto get = [&](auto &fn, const char *name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            if (!fn) all = false;
        };
        get(api.GetUniqueId, "ncclGetUniqueId");
        get(api.CommInitRank, "ncclCommInitRank");
        get(api.CommDestroy, "ncclCommDestroy");
        get(api.CommAbort, "ncclCommAbort");
        get(api.AllReduce, "ncclAllReduce");
        get(api.AllGather, "ncclAllGather");
        get(api.Send, "ncclSend");
        get(api.Recv, "ncclRecv");
        get(api.GroupStart, "ncclGroupStart");
        get(api.GroupEnd, "ncclGroupEnd");
        get(api.GetErrorString, "ncclGetErrorString");
        if (!all) { api.why = "libnccl.so.2 lacks a symbol this library needs"; return; }
        api.ok = true;
    });
    return api;
}

#define DS4F_NCCL(call)                                                                       \
    do {                                                                                      \
        ncclResult_t r_ = (call);                                                             \
        if (r_ != ncclSuccess) {                                                              \
            ::ds4f::set_error("%s:%d: %s: %s", __FILE__, __LINE__, #call,                      \
                              ::ds4f::nccl().GetErrorString(r_));                               \
            return -1;                                                                        \
        }                                                                                     \
    } while (0)

// ---- kernels ----------------------------------------------------------------------------
__global__ void k_add(float *__restrict__ a, const float *__restrict__ b, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        a[i] = __fadd_rn(a[i], b[i]);
}

// sendbuf row i = [state of token rows[i] (H floats) | its K selections (as
// int bits) | its K weights]
__global__ void k_pack(const float *__restrict__ states, const int *__restrict__ sel, const float *__restrict__ w,
                       const int *__restrict__ rows, int H, int K, float *__restrict__ buf) {
    const int i = blockIdx.x, t = rows[i];
    float *dst = buf + (int64_t)i * (H + 2 * K);
    const float4 *src = (const float4 *)(states + (int64_t)t * H);
    for (int c = threadIdx.x; c < H / 4; c += blockDim.x) ((float4 *)dst)[c] = src[c];
    if (threadIdx.x < K) {
        dst[H + threadIdx.x] = __int_as_float(sel[(int64_t)t * K + threadIdx.x]);
        dst[H + K + threadIdx.x] = w[(int64_t)t * K + threadIdx.x];
    }
}

__global__ void k_unpack(const float *__restrict__ buf, int H, int K, float *__restrict__ states,
                         int *__restrict__ sel, float *__restrict__ w) {
    const int i = blockIdx.x;
    const float *src = buf + (int64_t)i * (H + 2 * K);
    for (int c = threadIdx.x; c < H / 4; c += blockDim.x)
        ((float4 *)(states + (int64_t)i * H))[c] = ((const float4 *)src)[c];
    if (threadIdx.x < K) {
        sel[(int64_t)i * K + threadIdx.x] = __float_as_int(src[H + threadIdx.x]);
        w[(int64_t)i * K + threadIdx.x] = src[H + K + threadIdx.x];
    }
}

// Token t: acc = sum over ranks d (ascending) of its partial from d, then
// + its shared expert's term (acc_sh), state += acc.
__global__ void k_final(float *__restrict__ states, const float *__restrict__ back, const float *__restrict__ acc_sh,
                        const int *__restrict__ tok_rows, int N, int H) {
    const int t = blockIdx.x;
    const int *tr = tok_rows + (int64_t)t * N;
    for (int c = threadIdx.x; c < H; c += blockDim.x) {
        float acc = 0.0f;
        for (int d = 0; d < N; d++) {
            const int i = tr[d];
            if (i >= 0) acc = __fadd_rn(acc, back[(int64_t)i * H + c]);
        }
        acc = __fadd_rn(acc, acc_sh[(int64_t)t * H + c]);
        states[(int64_t)t * H + c] = __fadd_rn(states[(int64_t)t * H + c], acc);
    }
}

}  // namespace

// ---- the dispatch plan (host) -------------------------------------------------------------
// For T tokens with K selections each (global expert ids, < 0 skipped) over
// N ranks of E / N experts: counts[d] = tokens with a selection on rank d;
// send_rows = those tokens, rank by rank, ascending within a rank;
// tok_rows[t][d] = the position of token t in send_rows for rank d, or -1.
int ep_plan(const int *sel, int T, int K, int E, int N, int *counts, int *send_rows, int *tok_rows) {
    DS4F_REQUIRE(T >= 0 && K > 0 && E > 0 && N > 0 && E % N == 0 && (T == 0 || sel),
                 "ep plan: bad arguments (T %d, K %d, E %d, N %d)", T, K, E, N);
    const int per = E / N;
    std::vector<uint8_t> need((size_t)T * N, 0);
    for (int t = 0; t < T; t++)
        for (int j = 0; j < K; j++) {
            const int e = sel[(int64_t)t * K + j];
            if (e < 0) continue;
            DS4F_REQUIRE(e < E, "ep plan: token %d selection %d is expert %d of %d", t, j, e, E);
            need[(size_t)t * N + e / per] = 1;
        }
    int pos = 0;
    for (int d = 0; d < N; d++) {
        int c = 0;
        for (int t = 0; t < T; t++) {
            int v = -1;
            if (need[(size_t)t * N + d]) {
                if (send_rows) send_rows[pos] = t;
                v = pos++;
                c++;
            }
            if (tok_rows) tok_rows[(int64_t)t * N + d] = v;
        }
        counts[d] = c;
    }
    return 0;
}

struct EpState {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    float *acc = nullptr;             // decode: [bmax][H] partial combine
    cudaGraphExec_t graph = nullptr;  // decode: one captured step
    float *g_states = nullptr;
    int g_B = 0;
    void *g_ws = nullptr;
    bool g_eager_done = false;
    // prefill buffers, grown on demand
    void *pf = nullptr;
    size_t pf_bytes = 0;
    // the fused one-token decode (the persistent kernel on every rank, the
    // down outputs stored straight into the other GPUs' memory): this GPU's
    // [2][K][H] words, every rank's mapping of them, the shared launch epoch
    bool fused = true;                // use it where eligible (ds4f_gpu_ep_set_fused)
    bool fused_ok = false;            // buffers mapped on every rank
    uint64_t *pout_own = nullptr;
    uint64_t *pout[8] = {};
    bool opened[8] = {};
    int epoch = 0;
    int64_t lsteps = 0;
    // every rank holds the whole pool: the fused step splits the K
    // selections by index instead (no per-layer imbalance; one-token fused
    // steps only)
    bool split_sel = false;
};

void ep_free(Model *m) {
    EpState *ep = (EpState *)m->ep;
    if (!ep) return;
    if (ep->graph) cudaGraphExecDestroy(ep->graph);
    for (int p = 0; p < 8; p++)
        if (ep->opened[p]) cudaIpcCloseMemHandle(ep->pout[p]);
    if (ep->pout_own) cudaFree(ep->pout_own);
    if (ep->acc) cudaFree(ep->acc);
    if (ep->pf) cudaFree(ep->pf);
    if (ep->comm && nccl().ok) nccl().CommDestroy(ep->comm);
    delete ep;
    m->ep = nullptr;
}

// The fused decode's exchange buffers: each rank allocates its [2][K][H]
// words, the ranks all-gather (NCCL) the CUDA IPC handle and device UUID of
// each, and every rank maps the others'. Ranks sharing a device (kernels
// that wait on one another must not share a GPU) or a mapping that fails
// leave the fused path off; the per-layer path with its all-reduce stays.
void ep_map_peers(Model &m, EpState *ep) {
    const int N = ep->world, me = ep->rank;
    const size_t ob = (size_t)2 * m.d.topk * m.d.hidden * 8;
    if (N > 8) return;
    if (cudaMalloc(&ep->pout_own, ob) != cudaSuccess) { cudaGetLastError(); ep->pout_own = nullptr; return; }
    cudaMemset(ep->pout_own, 0, ob);
    ep->pout[me] = ep->pout_own;
    if (N == 1) { ep->fused_ok = true; return; }
    struct Rec { cudaIpcMemHandle_t h; char uuid[16]; };
    Rec mine = {};
    cudaDeviceProp prop;
    if (cudaIpcGetMemHandle(&mine.h, ep->pout_own) != cudaSuccess ||
        cudaGetDeviceProperties(&prop, m.device) != cudaSuccess) { cudaGetLastError(); return; }
    memcpy(mine.uuid, &prop.uuid, 16);
    std::vector<Rec> all(N);
    Rec *dev = nullptr;
    if (cudaMalloc(&dev, sizeof(Rec) * N) != cudaSuccess) { cudaGetLastError(); return; }
    cudaMemcpy(dev + me, &mine, sizeof(Rec), cudaMemcpyHostToDevice);
    const ncclResult_t r = nccl().AllGather(dev + me, dev, sizeof(Rec), ncclUint8, ep->comm, m.stream);
    cudaStreamSynchronize(m.stream);
    cudaMemcpy(all.data(), dev, sizeof(Rec) * N, cudaMemcpyDeviceToHost);
    cudaFree(dev);
    if (r != ncclSuccess) return;
    for (int p = 0; p < N; p++)
        for (int q = 0; q < p; q++)
            if (!memcmp(all[p].uuid, all[q].uuid, 16)) return;      // two ranks on one GPU
    for (int p = 0; p < N; p++) {
        if (p == me) continue;
        void *ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, all[p].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            return;
        }
        ep->pout[p] = (uint64_t *)ptr;
        ep->opened[p] = true;
    }
    // every rank mapped every peer before any fused launch (a rank whose
    // mapping failed stays on the other path, so all of them must agree)
    int *flag = nullptr;
    if (cudaMalloc(&flag, 4) != cudaSuccess) { cudaGetLastError(); return; }
    const int one = 1;
    cudaMemcpy(flag, &one, 4, cudaMemcpyHostToDevice);
    const ncclResult_t r2 = nccl().AllReduce(flag, flag, 1, ncclInt32, ncclMin, ep->comm, m.stream);
    cudaStreamSynchronize(m.stream);
    int all_ok = 0;
    cudaMemcpy(&all_ok, flag, 4, cudaMemcpyDeviceToHost);
    cudaFree(flag);
    ep->fused_ok = r2 == ncclSuccess && all_ok == 1;
}

namespace {

int launch_add(float *a, const float *b, int64_t n, cudaStream_t st) {
    const int blocks = (int)std::min<int64_t>(592, (n + 255) / 256);
    k_add<<<blocks, 256, 0, st>>>(a, b, n);
    DS4F_CUDA(cudaGetLastError());
    return 0;
}

// One decode step of B tokens through every layer, expert-parallel.
int ep_step(Model *m, EpState *ep, float *states, int B, cudaStream_t st) {
    const int H = m->d.hidden;
    for (int L = 0; L < m->d.n_layers; L++) {
        const bool sh = ep->rank == 0;
        if (B == 1) {
            if (moe_layer_launch_ex(m, L, states, nullptr, nullptr, ep->acc, true, sh, st)) return -1;
        } else {
            if (decode_batch_layer(m, L, states, B, nullptr, nullptr, st, false, false, ep->acc, sh, true))
                return -1;
        }
        if (ep->world > 1) DS4F_NCCL(nccl().AllReduce(ep->acc, ep->acc, (size_t)B * H, ncclFloat, ncclSum, ep->comm, st));
        if (launch_add(states, ep->acc, (int64_t)B * H, st)) return -1;
    }
    return 0;
}

template <typename T>
T *carve(uint8_t *&p, size_t n) {
    T *r = (T *)p;
    p += (n * sizeof(T) + 255) / 256 * 256;
    return r;
}

}  // namespace
}  // namespace ds4f

using ds4f::EpState;
using ds4f::set_error;

extern "C" {

int ds4f_gpu_ep_unique_id(uint8_t id[128]) {
    DS4F_REQUIRE(id, "ep_unique_id: null argument");
    const ds4f::NcclApi &n = ds4f::nccl();
    DS4F_REQUIRE(n.ok, "ep: %s", n.why.c_str());
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
    ncclUniqueId u;
    DS4F_NCCL(n.GetUniqueId(&u));
    memcpy(id, &u, 128);
    return 0;
}

int ds4f_gpu_ep_attach(Ds4fGpuModel *h, const uint8_t id[128], int rank, int world) {
    DS4F_REQUIRE(h && id && world >= 1 && rank >= 0 && rank < world, "ep_attach: bad arguments");
    ds4f::Model &m = h->m;
    const ds4f::NcclApi &n = ds4f::nccl();
    DS4F_REQUIRE(n.ok, "ep: %s", n.why.c_str());
    DS4F_REQUIRE(!m.ep, "ep_attach: the model is attached already");
    DS4F_REQUIRE(!m.cache, "ep_attach: a streaming model cannot be sharded");
    const int E = m.d.n_experts;
    const bool whole = world > 1 && m.d.expert_first == 0 && m.d.expert_count == E;
    DS4F_REQUIRE(whole || (E % world == 0 && m.d.expert_first == rank * (E / world) && m.d.expert_count == E / world),
                 "ep_attach: rank %d of %d must hold experts [%d, %d) (or every expert); the model holds [%d, %d)",
                 rank, world, rank * (E / world), (rank + 1) * (E / world), m.d.expert_first,
                 m.d.expert_first + m.d.expert_count);
    EpState *ep = new EpState();
    ep->rank = rank;
    ep->world = world;
    ep->split_sel = whole;
    ncclUniqueId u;
    memcpy(&u, id, 128);
    DS4F_CUDA(cudaSetDevice(m.device));
    ncclResult_t r = n.CommInitRank(&ep->comm, world, u, rank);
    if (r != ncclSuccess) {
        delete ep;
        set_error("ep_attach: ncclCommInitRank: %s", n.GetErrorString(r));
        return -1;
    }
    m.ep = ep;
    if (cudaMalloc(&ep->acc, (size_t)m.bmax * m.d.hidden * 4) != cudaSuccess) {
        ds4f::ep_free(&m);
        set_error("ep_attach: workspace allocation failed");
        return -1;
    }
    // connect every peer now (NCCL sets connections up on first use, which
    // cannot happen inside a graph capture)
    int rc = 0;
    if (world > 1) {
        rc = [&]() -> int {
            DS4F_NCCL(n.AllReduce(ep->acc, ep->acc, 1, ncclFloat, ncclSum, ep->comm, m.stream));
            DS4F_NCCL(n.GroupStart());
            for (int d = 0; d < world; d++) {
                DS4F_NCCL(n.Send(ep->acc, 1, ncclFloat, d, ep->comm, m.stream));
                DS4F_NCCL(n.Recv(ep->acc + 1 + d, 1, ncclFloat, d, ep->comm, m.stream));
            }
            DS4F_NCCL(n.GroupEnd());
            DS4F_CUDA(cudaStreamSynchronize(m.stream));
            return 0;
        }();
    }
    if (rc) {
        ds4f::ep_free(&m);
        return rc;
    }
    ds4f::ep_map_peers(m, ep);
    return 0;
}

int ds4f_gpu_ep_set_fused(Ds4fGpuModel *h, int on) {
    DS4F_REQUIRE(h && h->m.ep, "ep_set_fused: model not attached");
    ((EpState *)h->m.ep)->fused = on != 0;
    return 0;
}

int ds4f_gpu_ep_fused_ready(const Ds4fGpuModel *h) {
    DS4F_REQUIRE(h && h->m.ep, "ep_fused_ready: model not attached");
    const EpState *ep = (const EpState *)h->m.ep;
    return ep->fused_ok && ds4f::decode_eligible_ep(&h->m, ep->rank, ep->world, ep->split_sel) ? 1 : 0;
}

int ds4f_gpu_ep_detach(Ds4fGpuModel *h) {
    DS4F_REQUIRE(h, "ep_detach: null model");
    if (h->m.stream) cudaStreamSynchronize(h->m.stream);
    ds4f::ep_free(&h->m);
    return 0;
}

int ds4f_gpu_ep_abort(Ds4fGpuModel *h) {
    DS4F_REQUIRE(h && h->m.ep, "ep_abort: model not attached");
    EpState *ep = (EpState *)h->m.ep;
    if (ep->comm) DS4F_NCCL(ds4f::nccl().CommAbort(ep->comm));
    ep->comm = nullptr;
    return 0;
}

int ds4f_ep_plan_dispatch(const int *sel, int T, int K, int n_experts, int world, int *counts, int *send_rows,
                          int *tok_rows) {
    DS4F_REQUIRE(counts, "ep_plan_dispatch: null counts");
    return ds4f::ep_plan(sel, T, K, n_experts, world, counts, send_rows, tok_rows);
}

int ds4f_gpu_ep_stack_dev(Ds4fGpuModel *h, float *states, int B, int n_steps, void *stream) {
    DS4F_REQUIRE(h && states && B > 0 && n_steps >= 0, "ep_stack: bad arguments");
    ds4f::Model &m = h->m;
    EpState *ep = (EpState *)m.ep;
    DS4F_REQUIRE(ep && ep->comm, "ep_stack: model not attached to a communicator (ds4f_gpu_ep_attach)");
    DS4F_REQUIRE(B <= m.bmax, "ep_stack: batch %d above %d", B, m.bmax);
    if (B == 1 && ep->fused && ep->fused_ok && ds4f::decode_eligible_ep(&m, ep->rank, ep->world, ep->split_sel)) {
        // one persistent launch per rank for all n_steps x layers
        return ds4f::on_model_stream(m, stream, [&](cudaStream_t st) -> int {
            ds4f::DecodePeers pe;
            for (int p = 0; p < 8; p++) pe.out[p] = ep->pout[p];
            pe.rank = ep->rank;
            pe.world = ep->world;
            pe.epoch = &ep->epoch;
            pe.lsteps = &ep->lsteps;
            pe.split_sel = ep->split_sel;
            return n_steps > 0 ? ds4f::decode_launch(&m, states, n_steps, st, &pe) : 0;
        });
    }
    DS4F_REQUIRE(!ep->split_sel, "ep_stack: with every expert on every rank only fused one-token steps run "
                                 "(B = 1, ds4f_gpu_ep_fused_ready)");
    return ds4f::on_model_stream(m, stream, [&](cudaStream_t st) -> int {
        int s = 0;
        const bool fresh = !ep->graph || ep->g_states != states || ep->g_B != B ||
                           (B > 1 && ep->g_ws != m.pf_ws);
        if (fresh && n_steps > 0) {
            // the first step runs eagerly: it sizes the workspaces and sets the
            // kernels up; the later ones replay one captured step
            if (ds4f::ep_step(&m, ep, states, B, st)) return -1;
            s = 1;
            if (ep->graph) { cudaGraphExecDestroy(ep->graph); ep->graph = nullptr; }
            cudaGraph_t g;
            DS4F_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            int rc = ds4f::ep_step(&m, ep, states, B, st);
            cudaError_t e = cudaStreamEndCapture(st, &g);
            if (rc) { if (e == cudaSuccess) cudaGraphDestroy(g); return -1; }
            DS4F_CUDA(e);
            e = cudaGraphInstantiate(&ep->graph, g, 0);
            cudaGraphDestroy(g);
            DS4F_CUDA(e);
            ep->g_states = states;
            ep->g_B = B;
            ep->g_ws = m.pf_ws;
        }
        for (; s < n_steps; s++) DS4F_CUDA(cudaGraphLaunch(ep->graph, st));
        return 0;
    });
}

int ds4f_gpu_ep_prefill(Ds4fGpuModel *h, float *states, int T, const int *sel, const float *w, void *stream) {
    DS4F_REQUIRE(h && T >= 0 && (T == 0 || (states && sel && w)), "ep_prefill: bad arguments");
    ds4f::Model &m = h->m;
    EpState *ep = (EpState *)m.ep;
    DS4F_REQUIRE(ep && ep->comm, "ep_prefill: model not attached to a communicator (ds4f_gpu_ep_attach)");
    DS4F_REQUIRE(!ep->split_sel, "ep_prefill: needs each rank's shard of E / N experts");
    const ds4f::NcclApi &n = ds4f::nccl();
    const int NL = m.d.n_layers, H = m.d.hidden, K = m.d.topk, E = m.d.n_experts, N = ep->world, me = ep->rank;
    const int RW = H + 2 * K;                       // floats per dispatched row
    cudaStream_t st = (cudaStream_t)stream;
    // 1. every layer's plan from the routing (one read-back)
    std::vector<int> sel_h((size_t)NL * T * K);
    if (T) DS4F_CUDA(cudaMemcpyAsync(sel_h.data(), sel, sel_h.size() * 4, cudaMemcpyDeviceToHost, st));
    DS4F_CUDA(cudaStreamSynchronize(st));
    std::vector<int> counts((size_t)NL * N), rows((size_t)NL * T * N), tok((size_t)NL * T * N);
    std::vector<int> row_off(NL + 1, 0);
    for (int L = 0; L < NL; L++) {
        if (ds4f::ep_plan(sel_h.data() + (size_t)L * T * K, T, K, E, N, &counts[(size_t)L * N],
                          rows.data() + (size_t)L * T * N, tok.data() + (size_t)L * T * N))
            return -1;
        int tot = 0;
        for (int d = 0; d < N; d++) tot += counts[(size_t)L * N + d];
        row_off[L + 1] = row_off[L] + tot;
    }
    // 2. every rank's counts (all-gather), so each knows what it receives
    std::vector<int> all((size_t)N * NL * N);
    {
        int *dcnt = nullptr;
        DS4F_CUDA(cudaMallocAsync((void **)&dcnt, all.size() * 4, st));
        DS4F_CUDA(cudaMemcpyAsync(dcnt + (size_t)me * NL * N, counts.data(), counts.size() * 4,
                                  cudaMemcpyHostToDevice, st));
        ncclResult_t r = N > 1 ? n.AllGather(dcnt + (size_t)me * NL * N, dcnt, (size_t)NL * N, ncclInt32, ep->comm, st)
                               : ncclSuccess;
        cudaMemcpyAsync(all.data(), dcnt, all.size() * 4, cudaMemcpyDeviceToHost, st);
        cudaFreeAsync(dcnt, st);
        DS4F_CUDA(cudaStreamSynchronize(st));
        if (r != ncclSuccess) { set_error("ep_prefill: ncclAllGather: %s", n.GetErrorString(r)); return -1; }
    }
    auto rcount = [&](int L, int s) { return all[((size_t)s * NL + L) * N + me]; };   // rows s sends me
    int send_max = 0, recv_max = 0;
    for (int L = 0; L < NL; L++) {
        send_max = std::max(send_max, row_off[L + 1] - row_off[L]);
        int r = 0;
        for (int s = 0; s < N; s++) r += rcount(L, s);
        recv_max = std::max(recv_max, r);
    }
    // 3. device buffers and plans
    const size_t need = 256 * 16 + (size_t)row_off[NL] * 4 + (size_t)NL * T * N * 4 + (size_t)send_max * RW * 4 +
                        (size_t)recv_max * RW * 4 + (size_t)recv_max * (H + 2 * K) * 4 + (size_t)recv_max * H * 4 +
                        (size_t)send_max * H * 4 + (size_t)T * H * 4;
    if (need > ep->pf_bytes) {
        if (ep->pf) { cudaStreamSynchronize(st); cudaFree(ep->pf); ep->pf = nullptr; ep->pf_bytes = 0; }
        DS4F_CUDA(cudaMalloc(&ep->pf, need));
        ep->pf_bytes = need;
    }
    uint8_t *p = (uint8_t *)ep->pf;
    int *d_rows = ds4f::carve<int>(p, std::max(1, row_off[NL]));
    int *d_tok = ds4f::carve<int>(p, std::max<size_t>(1, (size_t)NL * T * N));
    float *sendb = ds4f::carve<float>(p, (size_t)std::max(1, send_max) * RW);
    float *recvb = ds4f::carve<float>(p, (size_t)std::max(1, recv_max) * RW);
    float *rst = ds4f::carve<float>(p, (size_t)std::max(1, recv_max) * H);
    int *rsel = ds4f::carve<int>(p, (size_t)std::max(1, recv_max) * K);
    float *rw = ds4f::carve<float>(p, (size_t)std::max(1, recv_max) * K);
    float *racc = ds4f::carve<float>(p, (size_t)std::max(1, recv_max) * H);
    float *back = ds4f::carve<float>(p, (size_t)std::max(1, send_max) * H);
    float *acc_sh = ds4f::carve<float>(p, (size_t)std::max(1, T) * H);
    {   // compact the per-layer rows
        std::vector<int> flat(std::max(1, row_off[NL]));
        for (int L = 0; L < NL; L++)
            std::copy(rows.begin() + (size_t)L * T * N, rows.begin() + (size_t)L * T * N + (row_off[L + 1] - row_off[L]),
                      flat.begin() + row_off[L]);
        DS4F_CUDA(cudaMemcpyAsync(d_rows, flat.data(), flat.size() * 4, cudaMemcpyHostToDevice, st));
        if (T) DS4F_CUDA(cudaMemcpyAsync(d_tok, tok.data(), tok.size() * 4, cudaMemcpyHostToDevice, st));
    }
    // the batched step's workspace, sized once for the largest call
    if (ds4f::prefill_pre_size(&m, std::max(1, std::max(recv_max, T)))) return -1;
    // 4. the layers
    for (int L = 0; L < NL; L++) {
        const int ns = row_off[L + 1] - row_off[L];
        int nr = 0;
        std::vector<int> roff(N + 1, 0), soff(N + 1, 0);
        for (int d = 0; d < N; d++) {
            soff[d + 1] = soff[d] + counts[(size_t)L * N + d];
            roff[d + 1] = roff[d] + rcount(L, d);
        }
        nr = roff[N];
        const int *selL = sel + (size_t)L * T * K;
        const float *wL = w + (size_t)L * T * K;
        if (ns) {
            ds4f::k_pack<<<ns, 256, 0, st>>>(states, selL, wL, d_rows + row_off[L], H, K, sendb);
            DS4F_CUDA(cudaGetLastError());
        }
        DS4F_NCCL(n.GroupStart());
        for (int d = 0; d < N; d++) {
            const int c_s = soff[d + 1] - soff[d], c_r = roff[d + 1] - roff[d];
            if (c_s) DS4F_NCCL(n.Send(sendb + (size_t)soff[d] * RW, (size_t)c_s * RW, ncclFloat, d, ep->comm, st));
            if (c_r) DS4F_NCCL(n.Recv(recvb + (size_t)roff[d] * RW, (size_t)c_r * RW, ncclFloat, d, ep->comm, st));
        }
        DS4F_NCCL(n.GroupEnd());
        if (nr) {
            ds4f::k_unpack<<<nr, 256, 0, st>>>(recvb, H, K, rst, rsel, rw);
            DS4F_CUDA(cudaGetLastError());
            if (ds4f::prefill_layer(&m, L, rst, nr, rsel, rw, st, false, false, racc, false)) return -1;
        }
        if (T && ds4f::prefill_layer(&m, L, states, T, nullptr, nullptr, st, false, false, acc_sh, true)) return -1;
        DS4F_NCCL(n.GroupStart());
        for (int d = 0; d < N; d++) {
            const int c_s = soff[d + 1] - soff[d], c_r = roff[d + 1] - roff[d];
            if (c_r) DS4F_NCCL(n.Send(racc + (size_t)roff[d] * H, (size_t)c_r * H, ncclFloat, d, ep->comm, st));
            if (c_s) DS4F_NCCL(n.Recv(back + (size_t)soff[d] * H, (size_t)c_s * H, ncclFloat, d, ep->comm, st));
        }
        DS4F_NCCL(n.GroupEnd());
        if (T) {
            ds4f::k_final<<<T, 256, 0, st>>>(states, back, acc_sh, d_tok + (size_t)L * T * N, N, H);
            DS4F_CUDA(cudaGetLastError());
        }
    }
    return ds4f::prefill_check(&m, st);
}

}  // extern "C"
