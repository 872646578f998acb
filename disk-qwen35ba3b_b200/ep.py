"""ep.py -- expert-parallel decode across the GPUs of one node.

Rank r of N holds experts [r E/N, (r + 1) E/N) of every layer (the model's
expert shard) and the whole bf16 trunk. One decode step of B tokens, per
layer:

  1. ds4f_gpu_moe_layer_partial_dev (one token) or
     ds4f_gpu_moe_layer_batch_partial_dev (B > 1: the grouped tensor-core
     chain) on every rank: RMSNorm, router and certified top-K on the full
     state (the same result on every rank, the state being identical),
     gate/up/SiLU/down of the selections this rank holds, their part of the
     selection-order combine; the shared expert on rank 0 only;
  2. one all-reduce (sum) of acc [B][H] fp32 over the ranks (NCCL over
     NVLink on GPUs);
  3. state += acc on every rank (the residual, src/moe.c:1424).

The reference runs on one host and has no counterpart; this is the
partitioning the expert pool's layout invites (experts are independent
slots, src/st.c:127-180).

Batched prefill (ExpertParallelPrefill) follows the same pattern with
the tensor-core grouped GEMMs of the selections each rank's experts
received and one all-reduce of acc [T][H] per layer.

The per-rank layer step is a backend: `GpuShard` wraps the library; tests
drive the same drivers on CPU ranks (gloo) with an oracle backend.
"""
import torch
import torch.distributed as dist


def shard_of(rank, world, n_experts):
    """[first, first + count) of the experts rank `rank` holds."""
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not split over {world} ranks")
    count = n_experts // world
    return rank * count, count


class GpuShard:
    """One rank's expert shard on its GPU (the library's model with
    expert_first / expert_count set)."""

    def __init__(self, dc, fmt, n_layers, hidden, moe_inter, n_experts, topk, rank, world, seed=0):
        first, count = shard_of(rank, world, n_experts)
        self.model = dc.Model(fmt, n_layers, hidden, moe_inter, n_experts, topk,
                              expert_first=first, expert_count=count)
        self.model.synth(seed)
        self.n_layers, self.hidden = n_layers, hidden

    def layer_partial(self, L, states, acc, add_shared, stream=None):
        # one token: the per-token kernels (fp32 chains); a batch: the
        # routing of every token at once and the grouped tensor-core chain,
        # each expert's weights streamed once for all its tokens
        if states.dim() == 2 and states.shape[0] > 1:
            self.model.layer_batch_partial_dev(L, states, acc, add_shared, stream)
        else:
            self.model.layer_partial_dev(L, states, acc, add_shared, stream)

    def prefill_partial(self, L, states, sel, w, acc, add_shared, stream=None):
        self.model.prefill_partial_dev(L, states, sel, w, acc, add_shared, stream)

    def close(self):
        self.model.close()


class ExpertParallelDecoder:
    """Decode steps of a token batch over an expert-sharded process group."""

    def __init__(self, backend, group=None):
        self.b = backend
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.acc = None

    def step(self, states, stream=None):
        """states [B][H] (this rank's device), updated in place; identical on
        every rank before and after."""
        if self.acc is None or self.acc.shape != states.shape:
            self.acc = torch.empty_like(states)
        for L in range(self.b.n_layers):
            self.b.layer_partial(L, states, self.acc, self.rank == 0, stream)
            if self.world > 1:
                dist.all_reduce(self.acc, op=dist.ReduceOp.SUM, group=self.group)
            states.add_(self.acc)
        return states


class ExpertParallelPrefill:
    """Batched prefill of a token chunk over an expert-sharded process
    group: every rank holds the chunk's states and routing, runs the grouped
    tensor-core GEMMs of the selections its experts received (the shared
    expert on rank 0), and one all-reduce of acc [T][H] per layer completes
    the combine before the residual."""

    def __init__(self, backend, group=None):
        self.b = backend
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.acc = None

    def step(self, states, sel, w, stream=None):
        """states [T][H]; sel / w [n_layers][T][K] (global expert ids)."""
        if self.acc is None or self.acc.shape != states.shape:
            self.acc = torch.empty_like(states)
        for L in range(self.b.n_layers):
            self.b.prefill_partial(L, states, sel[L], w[L], self.acc, self.rank == 0, stream)
            if self.world > 1:
                dist.all_reduce(self.acc, op=dist.ReduceOp.SUM, group=self.group)
            states.add_(self.acc)
        return states
