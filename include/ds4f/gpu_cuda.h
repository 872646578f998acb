/*
 * gpu_cuda.h -- libds4f_cuda: the B200 (sm_100a) implementation of the
 * engine's GPU shim and of its routed-expert hot path.
 *
 * Drop-in boundary. The reference engine (C99) calls its GPU shim through
 * include/ds4f/gpu.h, implemented by src/gpu_stub.c (always -1) or
 * src/gpu_metal.mm (Apple Metal). libds4f_cuda links in their place: it
 * exports the four gpu.h symbols unchanged and adds the entry points below
 * for the FP8 / MXFP4 expert path. Plain C types only; no CUDA or torch
 * types appear in any signature (streams are `void *`, a cudaStream_t).
 *
 * Conventions (as gpu.h:20-21): every int-returning call returns 0 on
 * success and -1 on failure; ds4f_gpu_last_error() then holds a message
 * (per host thread). Unlike the reference there is NO CPU fallback behind
 * these calls: a caller that gets -1 reports the message and stops.
 * Host-buffer calls are synchronous on return. `_dev` calls take device
 * pointers and enqueue on the given stream; NULL is the default stream,
 * except for ds4f_gpu_mv_run and ds4f_gpu_synth_f32, which take NULL as the
 * library's own stream. One host thread per model, head or cache; calls are
 * not re-entrant.
 */
#ifndef DS4F_GPU_CUDA_H
#define DS4F_GPU_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- the reference shim, unchanged (include/ds4f/gpu.h:22-52) ------- */

/* gpu.h:22 -- 0 when a CUDA device is usable. */
int ds4f_gpu_init(void);
/* gpu.h:23 */
void ds4f_gpu_free(void);
/* gpu.h:30 -- MLX-4bit matvec. Implemented (y = sum_c (q*s+b) x_c, the
 * layout of ds4f_mlx4_matvec, src/kernels.c:154-222). */
int ds4f_gpu_mlx4_matvec(const uint32_t *vals, const uint16_t *scales,
                         const uint16_t *biases, int R, int C,
                         const float *x, float *y);
/* gpu.h:47-52 -- batched MLX-4bit jobs with weights cached per stable id
 * (the reference arena, src/gpu_metal.mm:186-254). */
int ds4f_gpu_mlx4_batch(const uint32_t *const *vals,
                        const uint16_t *const *scales,
                        const uint16_t *const *biases,
                        const float *const *xs, float *const *ys,
                        const void *const *ids, int R, int C, int njobs);

/* Last error message of this host thread ("" if none). New. */
const char *ds4f_gpu_last_error(void);

/* ---- formats ------------------------------------------------------- */
#define DS4F_FMT_MXFP4 0        /* e2m1 + E8M0 per bsize (moe.h:28 fmt 0) */
#define DS4F_FMT_FP8   2        /* E4M3 + block scales                   */
#define DS4F_FMT_BF16  3        /* bf16 (router, shared expert)          */
#define DS4F_SCALE_E8M0 0       /* FP8 block scales as E8M0 bytes        */
#define DS4F_SCALE_F32  1       /* FP8 block scales as fp32              */

/* ---- dequant-matvec, host buffers ---------------------------------- */

/* Replaces ds4f_f8_matvec (src/kernels.c:243-270, kernels.h:48-56):
 * y[r] = sum_c e4m3(W[r,c]) * s[r*SR/R][c*SC/C] * x[c]. scale_kind picks
 * E8M0 bytes (the reference) or fp32 (BASELINE's 128x128 scales). E4M3
 * bytes with exponent 15 decode to +-448 as in the reference table. */
int ds4f_gpu_f8_matvec(const uint8_t *W, int scale_kind, const void *scales,
                       int R, int C, int SR, int SC, const float *x, float *y);
/* Replaces ds4f_mxfp4_matvec (src/kernels.c:48-62, kernels.h:31-35);
 * bsize 16 or 32. No scratch: decode is fused. */
int ds4f_gpu_mxfp4_matvec(const uint8_t *vals, const uint8_t *scales, int R,
                          int C, int bsize, const float *x, float *y);
/* Replaces ds4f_bf16_matvec (src/kernels.c:91-103, kernels.h:45-46). */
int ds4f_gpu_bf16_matvec(const uint16_t *W, int R, int C, const float *x,
                         const float *bias, float *y);
/* Dequantised values, bit-exact: replaces ds4f_f8_decode_row
 * (src/kernels.c:294-306) for rows [r0, r1) -> out[(r1-r0) x C]. */
int ds4f_gpu_f8_decode_rows(const uint8_t *W, int scale_kind,
                            const void *scales, int R, int C, int SR, int SC,
                            int r0, int r1, float *out);
/* Replaces ds4f_mxfp4_decode (src/kernels.c:34-46). */
int ds4f_gpu_mxfp4_decode(const uint8_t *vals, const uint8_t *scales,
                          int64_t n, int bsize, float *out);

/* ---- dequant-matvec, device job lists ------------------------------ */

/* One y = W x on device pointers. fmt DS4F_FMT_*; scales: FP8 block
 * scales (scale_kind), MXFP4 E8M0 bytes per bsize, BF16 optional fp32
 * bias. canon: apply the e=15 -> 448 rule in-kernel (needed unless the
 * bytes came from a canonicalised pool). */
typedef struct Ds4fMvJob {
    const void *w;
    const void *scales;
    const float *x;
    float *y;
    int R, C, SR, SC;
    int fmt, scale_kind, bsize, canon;
} Ds4fMvJob;

typedef struct Ds4fMvPlan Ds4fMvPlan;
/* Plan a job list (copied to the device once). The batched form of the
 * reference's per-expert matvecs (src/moe.c:619-640, :728-740) and of its
 * Metal batch dispatch (gpu_metal.mm:256-367): all jobs in one launch. */
int  ds4f_gpu_mv_plan(const Ds4fMvJob *jobs, int njobs, Ds4fMvPlan **plan);
int  ds4f_gpu_mv_run(const Ds4fMvPlan *plan, void *stream);
void ds4f_gpu_mv_plan_free(Ds4fMvPlan *plan);

/* ---- resident expert pool + MoE step ------------------------------- */

typedef struct Ds4fGpuModelDesc {
    int fmt;              /* DS4F_FMT_FP8 or DS4F_FMT_MXFP4              */
    int n_layers;         /* Ds4fCfg.n_layers (ds4f.h:57)                */
    int hidden;           /* H  (Ds4fCfg.hidden)                         */
    int moe_inter;        /* M  (Ds4fCfg.moe_inter)                      */
    int n_experts;        /* E  (Ds4fCfg.n_experts)                      */
    int topk;             /* K  (Ds4fCfg.topk)                           */
    int renorm;           /* norm_topk_prob: 1 divides the top-k weights by
                             their sum (the reference keeps them raw,
                             src/moe.c:547-560)                          */
    int expert_first;     /* this device's expert shard [first, first+count) */
    int expert_count;     /* (count = n_experts: the whole pool)          */
    int router_exact;     /* 1: all router logits in the reference's exact
                             sequential order (bit-exact weights, slower) */
} Ds4fGpuModelDesc;

typedef struct Ds4fGpuModel Ds4fGpuModel;

/* Allocate the HBM-resident pool for the shard (the device-side
 * replacement of the expert cache, src/cache.c:140-214, with the memory
 * plan refusing past 95% of free HBM like ds4f_mem_refuses, mem.c). */
int  ds4f_gpu_model_create(const Ds4fGpuModelDesc *desc, Ds4fGpuModel **out);
void ds4f_gpu_model_destroy(Ds4fGpuModel *m);
/* Bytes of one expert slot (gate, up, down; values then scales each, the
 * order in which the engine reads an expert's tensors, src/moe.c:598-605)
 * and its offsets. */
int  ds4f_gpu_model_slot(const Ds4fGpuModel *m, int64_t rel_v[3],
                         int64_t rel_s[3], int64_t *nbytes);
/* Fill the whole shard with the seeded synthetic weights (sigma 0.02). */
int  ds4f_gpu_model_synth(Ds4fGpuModel *m, uint64_t seed);
/* Upload one layer's resident bf16 weights (the trunk tensors the
 * reference reads at src/main.c:1014-1083 and src/moe.c:1235-1293):
 * norm [H], router [E x H], shared gate/up [M x H], down [H x M],
 * shared_expert_gate [H]. */
int  ds4f_gpu_model_set_trunk(Ds4fGpuModel *m, int layer, const uint16_t *norm,
                              const uint16_t *router, const uint16_t *sh_gate,
                              const uint16_t *sh_up, const uint16_t *sh_down,
                              const uint16_t *sh_gw);
int  ds4f_gpu_model_get_trunk(const Ds4fGpuModel *m, int layer, uint16_t *norm,
                              uint16_t *router, uint16_t *sh_gate,
                              uint16_t *sh_up, uint16_t *sh_down,
                              uint16_t *sh_gw);
/* Upload / download one expert slot (host bytes, slot layout above). FP8
 * bytes are canonicalised on upload (e=15 -> +-448, value-preserving under
 * the reference table). */
int  ds4f_gpu_model_set_expert(Ds4fGpuModel *m, int layer, int expert,
                               const uint8_t *slot);
int  ds4f_gpu_model_get_expert(const Ds4fGpuModel *m, int layer, int expert,
                               uint8_t *slot);
/* Load this shard from a packed pool file: [u64 expert_nbytes][u64
 * n_layers][u64 n_experts] then slots layer-major, expert N of layer L at
 * 24 + (L*E + N)*nbytes (ds4f_pool_open_packed, src/st.c:127-180), each slot
 * already in this library's slot layout. A pool written by the converter
 * (tensors in sorted-name order) loads with ds4f_gpu_pool_load_json. */
int  ds4f_gpu_pool_load(Ds4fGpuModel *m, const char *path);

/* The converter's layout file beside a packed pool (pool-mxfp4.json,
 * tools/convert-ds4f.py:1321-1393; read by ds4f_pool_layout_load,
 * src/moe.c:51-160): per tensor its name, layer, expert, shape and absolute
 * v_off / s_off / v_nbytes / s_nbytes. The converter writes each expert's
 * tensors in sorted-name order (down, gate, up for Qwen names); these calls
 * place each by its name (".gate_proj.weight", ".up_proj.weight",
 * ".down_proj.weight"), or by entry order gate, up, down where entries carry
 * no name, as the engine reads them (src/moe.c:598-605). Format
 * "mxfp4-pool-v1" (e2m1 + E8M0 per 32) for MXFP4 models, "fp8-pool-v1"
 * (E4M3 bytes + fp32 scale per 128x128 block, row-major) for FP8 ones.
 * Refused as in the engine: missing keys, other layer/expert counts, a tensor
 * outside its slot; and here also: a shape or byte count other than the
 * model's, a role given twice or missing. */
/* Host only: offsets[(L * n_experts + X) * 6 + 2 * role (+1 for scales)] =
 * absolute file offsets, roles gate, up, down; may be NULL to validate. */
int  ds4f_pool_layout_plan(const char *json_path, int fmt, int hidden, int moe_inter,
                           int n_layers, int n_experts, int64_t *offsets,
                           int64_t *expert_nbytes);
/* Load this shard from the packed pool and its layout file (header and size
 * checked against the layout). */
int  ds4f_gpu_pool_load_json(Ds4fGpuModel *m, const char *pool_path, const char *json_path);

/* ---- the output head (the step after the MoE path) ----------------- */

/* Logits over the vocabulary and the greedy pick: ds4f_head_logits
 * (src/head.c:243-299) with the weights resident in HBM, and ds4f_argmax
 * (src/head.c:303-309: the first index whose logit is strictly greater than
 * every earlier one, starting from logits[0] -- so ties go to the lower
 * index, NaN logits are never picked, and a NaN logits[0] gives 0). dtype is
 * the reference head's w_dtype: 2 = F8_E4M3 with E8M0 block scales
 * [SR x SC] (scales may be NULL: 1.0), 4 (or 3) = BF16, 6 = MLX 4-bit (U32
 * words of 8 nibbles, BF16 scale and optional bias per 64; H is the decoded
 * width, 8 x the packed columns). F32 (0), I8 (1) and F16 (5) heads are
 * refused. The weights are copied at create. */
typedef struct Ds4fGpuHead Ds4fGpuHead;
int  ds4f_gpu_head_create(int dtype, const void *w, const void *scales, const void *biases,
                          int V, int H, int SR, int SC, Ds4fGpuHead **out);
void ds4f_gpu_head_free(Ds4fGpuHead *h);
/* Host buffers: state[H] in; logits[V] and *argmax out (either may be NULL). */
int  ds4f_gpu_head_logits(Ds4fGpuHead *h, const float *state, float *logits, int *argmax);
/* Device pointers on `stream` (NULL: the default stream); no sync. */
int  ds4f_gpu_head_logits_dev(Ds4fGpuHead *h, const float *state_dev, float *logits_dev,
                              int *argmax_dev, void *stream);
/* The pick alone over n device logits -> *out_dev. */
int  ds4f_gpu_argmax_dev(const float *logits_dev, int n, int *out_dev, void *stream);

/* ---- pools larger than HBM: the expert cache ------------------------ */

/* The reference's routed-expert cache policy (ds4f_cache_init /
 * ds4f_cache_getmany / ds4f_cache_pin, include/ds4f/ds4f.h:221-232,
 * src/cache.c:140-223), host only: a slot holds nothing, an expert being
 * fetched, or (layer, expert). A request for n experts reserves serially (a
 * resident expert is a hit; else the first empty slot, else the non-pinned
 * slot fetched longest ago -- hits do not refresh it; none left: slot -1, a
 * drop), then marks the reserved slots fetched in pool-offset order, each
 * taking the next clock value. getmany fills out_slot[n] and returns the
 * number of slots to fill (the caller copies them in); a request above 64
 * experts is cut to its first 64, as the reference's DS4F_MAX_TOPK cuts it.
 * No device needed. */
typedef struct Ds4fSlotCache Ds4fSlotCache;
/* flags: 0 = the reference's policy exactly. DS4F_SLOTCACHE_GUARD = a
 * request's own hits are not evicted by its later misses and an expert named
 * twice shares one slot (in the reference a hit slot can be re-reserved in
 * the same request, src/cache.c:150-170, leaving an earlier selection on
 * another expert's bytes); the streaming model runs guarded. */
#define DS4F_SLOTCACHE_GUARD 1
int  ds4f_slotcache_create(int n_slots, int flags, Ds4fSlotCache **out);
void ds4f_slotcache_free(Ds4fSlotCache *c);
int  ds4f_slotcache_getmany(Ds4fSlotCache *c, int layer, const int *experts, int n,
                            int *out_slot);
int  ds4f_slotcache_pin(Ds4fSlotCache *c, int slot, int pin);
int  ds4f_slotcache_stats(const Ds4fSlotCache *c, int64_t *requests, int64_t *hits,
                          int64_t *drops, int64_t *fetched);

/* A model whose experts stay in host memory (the reference's disk-backed
 * pool + cache, src/cache.c:140-214, for pools that do not fit in HBM):
 * host_pool holds every expert in the packed layout, expert (L, X) at
 * (L * n_experts + X) * slot bytes (ds4f_gpu_model_slot), and stays owned by
 * the caller (the library pins it for the model's lifetime). The HBM holds
 * the trunk and an arena of n_slots (>= top-k) expert slots run by the
 * policy above, guarded; per layer the routing is read back, the misses are copied in
 * (host to device) and the layer runs on the arena. Layer and stack calls
 * work as for a resident model (each layer waits on the host for its
 * routing, so none of them can be captured in a CUDA graph); synth,
 * set/get_expert, pool_load, prefill and the batched calls refuse it. */
int  ds4f_gpu_model_create_streaming(const Ds4fGpuModelDesc *desc, const uint8_t *host_pool,
                                     int n_slots, Ds4fGpuModel **out);
/* The streaming model's cache counters: experts requested, hits, slots
 * copied in. */
int  ds4f_gpu_stream_stats(const Ds4fGpuModel *m, int64_t *requests, int64_t *hits,
                           int64_t *fetched);

/* One token through one layer (host buffers): state[H] in/out; idx[K],
 * w[K] receive the routing (may be NULL). Replaces the reference's
 * per-layer route (src/main.c:1014-1088) + ds4f_moe_step
 * (src/moe.c:948-1456) for Qwen3.5 layers. */
int  ds4f_gpu_moe_layer(Ds4fGpuModel *m, int layer, float *state, int *idx,
                        float *w);
int  ds4f_gpu_moe_layer_dev(Ds4fGpuModel *m, int layer, float *state,
                            int *idx, float *w, void *stream);
/* n_steps decode steps of the whole layer stack: each step runs layers
 * 0..n_layers-1 on state[H], carried through the residual (the per-token
 * loop of src/main.c:848-1138, MoE part). */
int  ds4f_gpu_moe_stack(Ds4fGpuModel *m, float *state, int n_steps);
int  ds4f_gpu_moe_stack_dev(Ds4fGpuModel *m, float *state, int n_steps,
                            void *stream);
/* Expert-parallel layer step (no reference counterpart: the reference runs
 * on one host): the model holds the expert shard [expert_first,
 * expert_first + expert_count) of every layer and the whole trunk. For each
 * of B tokens (state [B][H], device, read only) the router and top-K run
 * on the full state, as on every rank; acc [B][H] (device) receives the
 * shard's part of the selection-order combine (ds4f_moe_step's
 * acc, src/moe.c:1224-1225) plus, when add_shared, the shared expert
 * (:1279-1282). Summing acc over the ranks of a full partition (NCCL
 * all-reduce) and adding it to the state completes the step (src/moe.c:1424).
 * Enqueued on `stream`. */
int  ds4f_gpu_moe_layer_partial_dev(Ds4fGpuModel *m, int layer, const float *state, int B,
                                    float *acc, int add_shared, void *stream);

/* Decode-step implementation: DS4F_PATH_AUTO (persistent kernel where it
 * covers the model: top-8, (H, M) = (2048, 512) or (1024, 256), 64 or 256
 * experts, whole pool on this device), DS4F_PATH_LAYERED (four kernels per
 * layer in a CUDA graph), DS4F_PATH_PERSISTENT (fail if not covered). */
#define DS4F_PATH_AUTO 0
#define DS4F_PATH_LAYERED 1
#define DS4F_PATH_PERSISTENT 2
int  ds4f_gpu_model_set_path(Ds4fGpuModel *m, int path);
/* Phase trace of the persistent decode kernel (the counterpart of the
 * reference's per-phase timers, src/main.c:253-258, 1522-1546): with
 * n_stamps > 0 every launch whose layers x steps x SMs x 32 stamps fit
 * records %globaltimer (ns) per (layer-step, CTA) in 32 slots, of which
 * 0..13 are used: start, state ready, normed, router rows done, routes
 * visible, top-k done, copies issued, softmax done, first gate/up group
 * landed, chains done, down rows landed, state written (11), chains
 * gathered (12), row-dots done (13); 14..16 hold the copy rounds of the
 * state, router-logit and chain gathers, 17 a bitmask of the gate/up copy
 * groups that had landed before their compute, 18 the time every router
 * word was visible (before the top-k), 21..23 gate/up copy groups 1..3
 * landed, 24 the gate/up dots of warp 0 done, 25 every warp's done, 26 the
 * first down row-dot of warp 0 done; with expert parallelism 19 this GPU's
 * down rows stored to the other GPUs, 20 theirs arrived; 27..31 inside the
 * top-k (keys read, network done, certificate, byte counts, group 0's
 * copies issued).
 * n_stamps = 0 turns it off. */
int  ds4f_gpu_model_trace(Ds4fGpuModel *m, int64_t n_stamps);
int  ds4f_gpu_model_trace_read(const Ds4fGpuModel *m, uint64_t *out, int64_t n_stamps);
/* Route log of the persistent decode kernel: the counterpart of the
 * reference's routing and state probes (src/main.c:1089-1094 prints each
 * layer's selections and weights, :1095-1110 checksums the state). With
 * n_layer_steps > 0 every later persistent call records, for its layer-steps
 * t < n_layer_steps (t = step * n_layers + layer, counted from the call's
 * first layer), the K selections, their weights and the layer's output
 * state; entries not written read as -1 / NaN. 0 turns it off. */
int  ds4f_gpu_model_route_log(Ds4fGpuModel *m, int n_layer_steps);
/* idx [n][K], w [n][K], states [n][H] (host; any may be NULL). */
int  ds4f_gpu_model_route_log_read(const Ds4fGpuModel *m, int *idx, float *w, float *states,
                                   int n_layer_steps);
/* Counters: [0] layers routed, [1] router exact-fallbacks taken. Also
 * reports (-1) a persistent-kernel wait that gave up. */
int  ds4f_gpu_model_stats(const Ds4fGpuModel *m, uint64_t out[2]);
/* Bounded waits of the persistent decode kernel (no reference counterpart:
 * the reference's waits are pthread joins, src/moe.c:1185-1192, and its
 * failures are exit codes, src/main.c:1-7). A wait on a weight copy gives up
 * after `polls` polls, a gather of another CTA's words after polls / 16 copy
 * rounds; the CTA then records an error code and its index, drains its own
 * copies and returns, every other CTA follows, and the call reports -1
 * ("decode kernel gave up waiting (code C at CTA N)"); the model stays
 * usable. 0 restores the default, 2^24 polls (about a second). */
int  ds4f_gpu_model_set_wait_limit(Ds4fGpuModel *m, int64_t polls);
/* Failure injection for tests (no reference counterpart): in the following
 * persistent launches CTA `cta` does not publish its rows of the state at
 * layer-step `layer_step` of a launch (0 = the first layer of its first
 * step), as a CTA that stalled would not; the other CTAs' bounded waits for
 * those rows run out and the call returns -1 with code 1 (the state gather).
 * cta < 0 turns it off. Nothing faults: the missing words are never
 * written, and every wait for them is bounded. */
int  ds4f_gpu_model_inject_stall(Ds4fGpuModel *m, int cta, int layer_step);
/* The same for the fused multi-GPU step (ds4f_gpu_ep_stack_dev): in the
 * following launches this rank stores none of its down rows to the other
 * GPUs at layer-step `layer_step`, as a stalled GPU would not; the others'
 * bounded waits for them run out and their calls return -1 with code 11,
 * then this rank's own waits for the next layer's rows of the GPUs that gave
 * up do too. layer_step < 0 turns it off. */
int  ds4f_gpu_model_inject_peer_stall(Ds4fGpuModel *m, int layer_step);

/* ---- allocation-free layer step ------------------------------------- */

/* One MoE layer's weights as caller-owned device pointers (16-byte
 * aligned): the E expert slots back to back, slot_bytes apart, in the slot
 * layout of ds4f_gpu_model_slot; the bf16 trunk tensors as in
 * ds4f_gpu_model_set_trunk. */
typedef struct Ds4fLayerDev {
    int fmt, hidden, moe_inter, n_experts, topk, renorm;
    const void *experts;
    int64_t slot_bytes;
    const uint16_t *norm, *router, *sh_gate, *sh_up, *sh_down, *sh_gw;
} Ds4fLayerDev;

/* No counterpart in the reference: an extra entry point for hosts that
 * cannot let this library allocate device memory (an engine that owns all
 * of it through its own pre-sized arena and budget). Same computation as
 * ds4f_gpu_moe_layer_dev; the per-call workspace lives in a static device
 * array of ~56 KB held by every GPU that loads the library, so the call
 * makes no cudaMalloc / cudaFree. Limits: hidden <= 2048, moe_inter <=
 * 512, n_experts <= 256, topk <= 16 (larger sizes return -1 with a
 * message). The first call on a device looks up the array's address with
 * that device current; make it before any stream capture. Calls share the
 * array: calls that overlap on the GPU race. state [H] in/out, idx [K] and
 * w [K] optional outputs, all device pointers; enqueued on `stream`. */
int  ds4f_gpu_moe_layer_static(const Ds4fLayerDev *layer, float *state, int *idx,
                               float *w, void *stream);

/* Seeded N(0, sigma) fp32 vector on the device (the synthetic activations
 * of the BASELINE configs): element i of tensor (seed, layer, kind, x, t). */
int  ds4f_gpu_synth_f32(float *dst_dev, int64_t n, uint64_t seed,
                        uint32_t layer, uint32_t kind, uint32_t x, uint32_t t,
                        double sigma, void *stream);

/* ---- batched prefill building blocks (tensor cores) ------------------- */

/* Activation quantiser of the batched prefill (no reference counterpart:
 * the reference's ds4f_moe_step_batch, src/moe.c:1480-1707, multiplies fp32
 * activations; this build feeds the FP8 tensor cores). Per row and
 * 128-column block: a = max |x|, r = 240 / a, s = a / 240 (fp32; a = 0:
 * r = 0, s = 1), y = x r, then ND in 1..3 E4M3 digits (round to nearest
 * even): d0 = E4M3(y), d1 = E4M3((y - d0) 16), d2 = E4M3(((y - d0) 16 - d1)
 * 16), so x = s (d0 + d1 / 16 + d2 / 256) within 2^-13 relative at ND 3.
 * x [N][C] fp32; q [ND][N][C] digit planes; s [N][C/128]; device pointers,
 * C a multiple of 128. Synchronous on `stream`. */
int  ds4f_gpu_quant_f8_digits(const float *x, int N, int C, int ND, uint8_t *q, float *s,
                              void *stream);

/* Block-scaled FP8 GEMM on the tensor cores (tcgen05.mma kind::f8f6f4,
 * TMEM accumulators, TMA tiles):
 *   Y[n][r] = sum_kb sW[r/128][kb] sX[n][kb] sum_{c in kb} W[r][c] x~[n][c]
 * with kb the 128-column blocks and x~ = d0 + d1/16 + d2/256 the digits of
 * ds4f_gpu_quant_f8_digits (planes X [ND][N][C], scales sX [N][C/128]).
 * W [R][C] canonical E4M3 with fp32 block scales sW [R/128][C/128] (the FP8
 * expert tensors, ds4f_f8_matvec's W / scales, src/kernels.c:243-270);
 * Y [N][R] fp32. Device pointers, 16-byte aligned; R and C multiples of
 * 128. Synchronous on `stream`. */
int  ds4f_gpu_f8_gemm(const uint8_t *W, const float *sW, const uint8_t *X, const float *sX,
                      float *Y, int R, int C, int N, int ND, void *stream);

/* Batched prefill of one MoE layer on the tensor cores: the GPU
 * counterpart of ds4f_moe_step_batch (include/ds4f/moe.h:171,
 * src/moe.c:1480-1707) for T tokens with their routing given. Per token
 * RMSNorm of the state, the routed experts' gate/up/SiLU/down as grouped
 * GEMMs over the tokens each expert received (FP8 weights x 3-digit E4M3
 * activations, ds4f_gpu_f8_gemm), the bf16 shared expert and its sigmoid
 * gate, the selection-order combine and the residual add. states_dev
 * [T][H] fp32 in/out; sel_dev [T][K] global expert ids (ids outside this
 * model's shard are skipped: the shard's partial sum); w_dev [T][K]
 * routing weights. FP8 pools. Synchronous on `stream`. */
int  ds4f_gpu_moe_prefill(Ds4fGpuModel *m, int layer, float *states_dev, int T,
                          const int *sel_dev, const float *w_dev, void *stream);
/* Expert-parallel partial of ds4f_gpu_moe_prefill (no reference
 * counterpart): the model's shard of the routed combine, plus the shared
 * expert when add_shared, into acc_dev [T][H]; states_dev is read only.
 * Summing acc over a partition of the experts and adding it to the states
 * completes the layer. Asynchronous on `stream` (it is called once per layer
 * between collectives): a tensor-core pipeline wait that gave up is reported
 * (-1) by a later partial call of this model. */
int  ds4f_gpu_moe_prefill_partial(Ds4fGpuModel *m, int layer, const float *states_dev, int T,
                                  const int *sel_dev, const float *w_dev, float *acc_dev,
                                  int add_shared, void *stream);
/* Every layer in order: sel_dev / w_dev [n_layers][T][K]. */
int  ds4f_gpu_prefill(Ds4fGpuModel *m, float *states_dev, int T, const int *sel_dev,
                      const float *w_dev, void *stream);

/* Batched decode of B tokens through one layer: the per-token router and
 * top-K (src/main.c:1014-1088, ds4f_topk src/moe.c:531-561, certified as
 * in ds4f_gpu_moe_layer: bit-exact indices) for all B tokens on the device,
 * then the grouped expert chain of the batched step (ds4f_moe_step_batch,
 * src/moe.c:1480-1707) on the tensor cores with that routing, as
 * ds4f_gpu_moe_prefill computes it (3-digit E4M3 activations). states_dev
 * [B][H] in/out; idx_dev / w_dev [B][K] receive the routing (may be NULL).
 * Synchronous on `stream`. */
int  ds4f_gpu_moe_layer_batch_dev(Ds4fGpuModel *m, int layer, float *states_dev, int B,
                                  int *idx_dev, float *w_dev, void *stream);
/* Expert-parallel form (no reference counterpart): routing on the full
 * states as on every rank, this shard's part of the combine (plus the
 * shared expert when add_shared) into acc_dev [B][H]; states unchanged.
 * Asynchronous on `stream`, errors reported by a later partial call, as
 * ds4f_gpu_moe_prefill_partial. */
int  ds4f_gpu_moe_layer_batch_partial_dev(Ds4fGpuModel *m, int layer, const float *states_dev,
                                          int B, float *acc_dev, int add_shared, void *stream);
/* n_steps decode steps of B tokens through every layer (the batched
 * counterpart of ds4f_gpu_moe_stack_dev); one pipeline check at the end. */
int  ds4f_gpu_moe_stack_batch_dev(Ds4fGpuModel *m, float *states_dev, int B, int n_steps,
                                  void *stream);

/* ---- expert parallelism across the GPUs of one node ------------------ */

/* No reference counterpart (the reference runs on one host, its experts
 * streamed from one disk): the pool's experts partitioned over N GPUs, one
 * process (or host thread) and one model per GPU, NCCL over NVLink inside
 * this library (loaded at the first call: libnccl.so.2). Rank r's model is
 * created with expert_first = r E / N, expert_count = E / N and holds the
 * whole trunk. The caller moves the 128-byte id from rank 0 to the other
 * ranks (any channel), then every rank attaches. A model holding every
 * expert on every rank (N > 1) attaches too: its fused one-token step
 * splits the K selections by index, rank r taking [r K / N, (r + 1) K / N)
 * (the same work on every rank each layer, at N times the memory); only
 * that step runs on it. */
#define DS4F_EP_ID_BYTES 128
int  ds4f_gpu_ep_unique_id(uint8_t id[DS4F_EP_ID_BYTES]);
/* Collective over the N ranks: builds the communicator on the model's
 * device and connects every peer; with one rank per GPU it also maps every
 * rank's down-output words of the fused decode (CUDA IPC handles exchanged
 * over the communicator). */
int  ds4f_gpu_ep_attach(Ds4fGpuModel *m, const uint8_t id[DS4F_EP_ID_BYTES], int rank, int world);
/* 1 when one-token steps run fused (below): attached, every rank's words
 * mapped (each rank on its own GPU) and the shape one the persistent
 * kernel covers. */
int  ds4f_gpu_ep_fused_ready(const Ds4fGpuModel *m);
/* Choose the fused one-token step where ready (1, the default) or the
 * per-layer kernels with an all-reduce per layer (0), e.g. to compare. */
int  ds4f_gpu_ep_set_fused(Ds4fGpuModel *m, int on);
int  ds4f_gpu_ep_detach(Ds4fGpuModel *m);
/* A collective waits for every peer. If a peer is lost, another host
 * thread calls this to abort the communicator: the waiting calls then
 * return -1 and the model must be detached (no further expert-parallel
 * calls). */
int  ds4f_gpu_ep_abort(Ds4fGpuModel *m);
/* n_steps decode steps of B (<= 64) tokens through every layer, the
 * expert-parallel form of ds4f_gpu_moe_stack_dev (src/main.c:848-1138, MoE
 * part): states [B][H] (device), the same on every rank before and after.
 * Per layer: the router and certified top-K on every rank, this rank's
 * selections (and on rank 0 the shared expert), one all-reduce of the
 * partial combine acc [B][H], state += acc (src/moe.c:1224-1225, 1424).
 * The first step of a (states, B) pair runs eagerly, the later ones replay
 * one captured CUDA graph of a whole step. Enqueued on `stream`.
 * B = 1 with ds4f_gpu_ep_fused_ready: instead, one persistent launch per
 * rank runs every step and layer (the kernel of DS4F_PATH_PERSISTENT on the
 * rank's shard): each rank routes the whole state, runs the chains of the
 * selections it holds, stores their output rows straight into every other
 * GPU's memory (tagged words, plain stores over NVLink) and combines every
 * selection's rows in selection order itself -- the same bits as one GPU
 * holding every expert, with no collective call. Ranks wait for each other
 * inside the kernel, bounded: a lost peer makes the call return -1 ("gave
 * up waiting (code 11 ...)") after about a second. */
int  ds4f_gpu_ep_stack_dev(Ds4fGpuModel *m, float *states, int B, int n_steps, void *stream);
/* Batched prefill of every layer with the chunk's tokens partitioned over
 * the ranks (the expert-parallel ds4f_moe_step_batch, src/moe.c:1480-1707):
 * this rank's T states [T][H] (device, in/out) and their routing sel / w
 * [n_layers][T][K] (device; global expert ids). Per layer each token's row
 * goes to every rank owning one of its selected experts (NCCL send/recv),
 * each rank runs the grouped tensor-core step on the rows it received (its
 * experts only), the partial combines come back to the owner, which adds
 * them in rank order, its shared expert and the residual. T may differ
 * between ranks, and be 0. Synchronous on `stream`. */
int  ds4f_gpu_ep_prefill(Ds4fGpuModel *m, float *states, int T, const int *sel, const float *w,
                         void *stream);
/* The dispatch plan of one layer (host only): for T tokens' K selections
 * (global ids, < 0 skipped) over `world` ranks of n_experts / world experts,
 * counts[world] = tokens with a selection on each rank; send_rows = those
 * tokens rank by rank, ascending (may be NULL); tok_rows [T][world] = each
 * token's position in send_rows for each rank, or -1 (may be NULL). */
int  ds4f_ep_plan_dispatch(const int *sel, int T, int K, int n_experts, int world, int *counts,
                           int *send_rows, int *tok_rows);

#ifdef __cplusplus
}
#endif

#endif /* DS4F_GPU_CUDA_H */
