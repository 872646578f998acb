"""ep.py -- expert parallelism across the GPUs of one node.

Rank r of N holds experts [r E/N, (r + 1) E/N) of every layer (the model's
expert shard) and the whole bf16 trunk. The reference runs on one host and
has no counterpart; this is the partitioning the expert pool's layout
invites (experts are independent slots, src/st.c:127-180).

On GPUs the data plane is the library's (libds4f_cuda, NCCL inside it, no
torch on it): `attach` moves the communicator id from rank 0 to the others
over the caller's process group and every rank attaches its model; then
`GpuShard.decode` (ds4f_gpu_ep_stack_dev) and `GpuShard.prefill`
(ds4f_gpu_ep_prefill) run whole steps.

The same two algorithms are written out below over torch.distributed with a
pluggable per-rank backend, so that their host-side logic (the partition,
the dispatch plan of ds4f_ep_plan_dispatch, the exchange and combine order)
runs on CPU ranks (gloo) against the oracle:

  ExpertParallelDecoder: per layer every rank routes the full state (the
    same certified top-K everywhere), runs the selections its experts
    received plus, on rank 0, the shared expert; one all-reduce of the
    partial combine acc [B][H]; state += acc (src/moe.c:1424).
  TokenParallelPrefill: the chunk's tokens partitioned over the ranks; per
    layer each token's row (state, selections, weights) goes to every rank
    owning one of its experts (all-to-all), each rank runs its experts on
    the rows it received, the partial combines come back (all-to-all) and
    the owner adds them in rank order, then its own tokens' shared expert
    and the residual (grouping src/moe.c:1516-1530, combine :1614-1630).
"""
import numpy as np
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

    def __init__(self, dc, fmt, n_layers, hidden, moe_inter, n_experts, topk, rank, world, seed=0, whole=False):
        """whole: every expert on this rank too (the fused one-token step then
        splits the K selections by index; N times the memory)."""
        first, count = (0, n_experts) if whole else shard_of(rank, world, n_experts)
        self.model = dc.Model(fmt, n_layers, hidden, moe_inter, n_experts, topk,
                              expert_first=first, expert_count=count)
        self.model.synth(seed)
        self.dc, self.rank, self.world = dc, rank, world
        self.n_layers, self.hidden = n_layers, hidden

    def attach(self, group=None):
        """Every rank: the library's communicator, its id made on rank 0
        and sent to the others over `group` (the only use of the caller's
        process group)."""
        box = [self.dc.ep_unique_id() if self.rank == 0 else None]
        dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group else 0, group=group)
        self.model.ep_attach(box[0], self.rank, self.world)

    def decode(self, states, n_steps, stream=None):
        """n_steps decode steps of states [B][H] (device, the same on every rank)."""
        self.model.ep_stack_dev(states, n_steps, stream)

    def prefill(self, states, sel, w, stream=None):
        """This rank's tokens: states [T][H], sel / w [n_layers][T][K] (device)."""
        self.model.ep_prefill_dev(states, sel, w, stream)

    def close(self):
        self.model.close()


def selection_owner(j, idx, n_experts, world, by_index):
    """The rank that runs selection j of a token routed to experts idx: the
    owner of its expert (E / N experts per rank), or, with every expert on
    every rank, rank r for j in [r K / N, (r + 1) K / N) -- the split of the
    library's fused one-token step (ds4f_gpu_ep_stack_dev)."""
    K = len(idx)
    if by_index:
        for r in range(world):
            if r * K // world <= j < (r + 1) * K // world:
                return r
        raise ValueError("selection index out of range")
    return int(idx[j]) // (n_experts // world)


class SelectionExchangeDecoder:
    """The algorithm of the library's fused one-token step over a process
    group: every rank routes the full state and runs the expert chains of
    the selections it owns (selection_owner); the ranks exchange those
    output rows (the kernel stores them into each other's memory; here an
    all-gather); every rank then combines all K rows in selection order and
    adds the shared expert and the residual itself -- so every rank holds
    exactly the single-host result (src/moe.c:1224-1225, 1279-1282, 1424).
    backend: route(L, state) -> (idx, w, xin), chain(L, e, xin) -> [H]
    float32, shared_add(L, xin, acc) (acc in place), n_layers, hidden,
    n_experts."""

    def __init__(self, backend, by_index=False, group=None):
        self.b = backend
        self.by_index = by_index
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def step(self, states):
        """states [B][H] float32 (CPU), updated in place; identical on every
        rank before and after."""
        H = self.b.hidden
        for L in range(self.b.n_layers):
            for t in range(states.shape[0]):
                x = states[t].numpy()
                idx, w, xin = self.b.route(L, x)
                K = len(idx)
                mine = torch.zeros((K, H), dtype=torch.float32)
                for j in range(K):
                    if selection_owner(j, idx, self.b.n_experts, self.world, self.by_index) == self.rank:
                        mine[j] = torch.from_numpy(self.b.chain(L, int(idx[j]), xin))
                rows = [torch.empty_like(mine) for _ in range(self.world)]
                dist.all_gather(rows, mine, group=self.group)
                acc = np.zeros(H, np.float32)
                for j in range(K):
                    r = selection_owner(j, idx, self.b.n_experts, self.world, self.by_index)
                    acc = (acc + np.float32(w[j]) * rows[r][j].numpy()).astype(np.float32)
                self.b.shared_add(L, xin, acc)
                states[t] = torch.from_numpy((x + acc).astype(np.float32))
        return states


class ExpertParallelDecoder:
    """Decode steps of a token batch over an expert-sharded process group;
    backend.layer_partial(L, states, acc, add_shared) fills acc [B][H]."""

    def __init__(self, backend, group=None):
        self.b = backend
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.acc = None

    def step(self, states, stream=None):
        """states [B][H], updated in place; identical on every rank before
        and after."""
        if self.acc is None or self.acc.shape != states.shape:
            self.acc = torch.empty_like(states)
        for L in range(self.b.n_layers):
            self.b.layer_partial(L, states, self.acc, self.rank == 0, stream)
            if self.world > 1:
                dist.all_reduce(self.acc, op=dist.ReduceOp.SUM, group=self.group)
            states.add_(self.acc)
        return states


class TokenParallelPrefill:
    """Batched prefill with the tokens partitioned over an expert-sharded
    process group (the algorithm of ds4f_gpu_ep_prefill). plan(sel, E, N)
    is ds4f_ep_plan_dispatch; backend.rows_partial(L, states, sel, w) returns
    each received row's partial combine over this rank's experts, and
    backend.shared(L, states) each own token's shared-expert term."""

    def __init__(self, backend, plan, n_experts, group=None):
        self.b, self.plan, self.E = backend, plan, n_experts
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def _a2a(self, send, send_counts, recv_counts, width):
        out = torch.empty((int(sum(recv_counts)), width), dtype=send.dtype)
        if self.world == 1:
            out.copy_(send)
        else:
            dist.all_to_all_single(out, send, output_split_sizes=[int(c) for c in recv_counts],
                                   input_split_sizes=[int(c) for c in send_counts], group=self.group)
        return out

    def step(self, states, sel, w):
        """states [T][H] (this rank's tokens, updated in place); sel / w
        [n_layers][T][K]."""
        T, H = states.shape
        K = sel.shape[-1]
        N = self.world
        for L in range(self.b.n_layers):
            counts, rows, tok = self.plan(sel[L].numpy(), self.E, N)
            send_counts = torch.from_numpy(counts.astype(np.int64))
            recv_counts = torch.empty_like(send_counts)
            if N > 1:
                dist.all_to_all_single(recv_counts, send_counts, group=self.group)
            else:
                recv_counts.copy_(send_counts)
            rws = torch.from_numpy(rows.astype(np.int64))
            send = torch.cat([states[rws], sel[L][rws].view(torch.float32), w[L][rws]], 1)
            recv = self._a2a(send, counts, recv_counts.tolist(), H + 2 * K)
            racc = self.b.rows_partial(L, recv[:, :H].contiguous(), recv[:, H:H + K].contiguous().view(torch.int32),
                                       recv[:, H + K:].contiguous())
            acc_sh = self.b.shared(L, states)
            back = self._a2a(racc, recv_counts.tolist(), counts, H)
            for t in range(T):
                acc = torch.zeros(H, dtype=torch.float32)
                for d in range(N):
                    if tok[t, d] >= 0:
                        acc = acc + back[int(tok[t, d])]
                states[t] += acc + acc_sh[t]
        return states
