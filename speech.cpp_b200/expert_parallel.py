"""Expert parallelism for the routed-expert FFN stack (TextModel::experts, src/families/drama3/text-model.cpp:198-221).

The reference runs a Drama 3 layer's routed experts on one device (or splits whole layers GPU/CPU through
ggml_backend_sched, src/engines/drama3-engine.cpp:51-88). Here the experts of every layer are split across the GPUs of
one node: rank r holds experts [r E/N, (r+1) E/N). The router runs on every rank and the token activations are
replicated (they come out of the replicated attention / mixer part of the layer), so dispatch moves no bytes: each
rank's b200_moe_ffn skips the (token, slot) pairs routed to other ranks and leaves its experts' partial weighted sum,
and one all-reduce per layer adds the partial sums into the layer output every rank needs next: an NCCL all-reduce,
or (PeerCombine) the combine kernel itself, over NVLink peer memory.

With 256 tokens x top-8 of 128 experts, an all-to-all dispatch + combine would move each token-slot's activation row
(2176 B as q8_0) out and its 8 KB f32 output row back for 7/8 of the 2048 slots, about 16.8 MB per layer over the
node; the all-reduce of the [256, 2048] f32 output moves 2 MB per rank.
"""

from __future__ import annotations

import ctypes


def expert_shard(n_expert: int, world: int, rank: int) -> tuple[int, int]:
    """(first expert, number of experts) of `rank`'s shard; experts split evenly, contiguous, in rank order."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if n_expert % world:
        raise ValueError(f"{n_expert} experts do not split evenly over {world} ranks")
    n = n_expert // world
    return rank * n, n


def place_experts(expert_bytes, n_expert: int, rest_bytes: int, free_bytes=None):
    """How many of this node's GPUs the routed experts need: the counterpart of the reference's place_experts
    (src/engines/drama3-engine.cpp:51-88 with expert_layers_on_device, src/families/drama3/placement.cpp:58-74), which
    keeps the layers whose experts fit on its one GPU and computes the rest on the CPU. Here every layer's experts stay
    on GPUs: b200_ep_place returns the fewest ranks (a power of two dividing n_expert) whose expert shard fits each
    GPU's free memory beside `rest_bytes` (the replicated weights, caches and working memory). `expert_bytes` holds
    each layer's routed-expert bytes; `free_bytes` defaults to every visible device's free memory (b200_device_info).
    Raises B200Error (ALLOC) when the experts fit no count of the GPUs, as the reference raises OutOfMemory when the
    rest of the model does not fit."""
    from . import device_count, device_info, ep_place

    if free_bytes is None:
        free_bytes = [device_info(d)[1] for d in range(device_count())]
    return ep_place(list(free_bytes), list(expert_bytes), n_expert, rest_bytes)


class PeerCombine:
    """The mailboxes of an expert-parallel group (b200_ep_*): each rank allocates one, the 64-byte CUDA IPC handles
    are exchanged over the torch.distributed group, each rank maps the others' and creates the group. Then
    b200_moe_ffn_ep combines the ranks' partial sums in one kernel over NVLink peer memory (a two-shot all-reduce:
    partial rows pushed to each token's owner, owners' sums pushed to every rank) instead of an NCCL all-reduce."""

    def __init__(self, ctx, group, max_tokens: int, hidden: int, timeout_us: int = 0):
        import torch.distributed as dist

        self.ctx, self.group = ctx, group
        L = ctx.L
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        ctx.check(L.b200_ep_mailbox_alloc(ctx.h, self.world, max_tokens, hidden, ctypes.byref(self.own), handle))
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self.peers, ptrs = [], []
        for g in range(self.world):
            if g == self.rank:
                ptrs.append(self.own.value)
                continue
            p = ctypes.c_void_p()
            ctx.check(L.b200_ep_mailbox_open(ctx.h, ctypes.create_string_buffer(handles[g], 64), ctypes.byref(p)))
            self.peers.append(p)
            ptrs.append(p.value)
        arr = (ctypes.c_void_p * self.world)(*ptrs)
        self.handle = ctypes.c_void_p()
        ctx.check(L.b200_ep_create(ctx.h, self.rank, self.world, max_tokens, hidden, arr, ctypes.byref(self.handle)))
        if timeout_us:
            ctx.check(L.b200_ep_set_timeout(self.handle, timeout_us))
        dist.barrier(group=group)  # every rank has mapped every mailbox before any rank writes into one

    def close(self):
        """Collective: every rank's kernels are done before any mailbox is unmapped or freed."""
        import torch.distributed as dist

        if self.handle is None:
            return
        self.ctx.synchronize()
        dist.barrier(group=self.group)
        L = self.ctx.L
        L.b200_ep_destroy(self.handle)
        for p in self.peers:
            L.b200_ep_mailbox_close(self.ctx.h, p)
        dist.barrier(group=self.group)
        L.b200_ep_mailbox_free(self.ctx.h, self.own)
        self.handle = None


class ExpertParallelMoe:
    """One rank's share of an MoE FFN stack: per layer (gate_up, down) expert weights of experts
    [expert0, expert0 + n_local) of n_expert. `ffn` is any object with moe_ffn(gate_up, down, x, ids, w, expert0=,
    n_expert_total=, out=) and prefetch_l2(weight, stream) (a speech.cpp_b200 Context); `group` a torch.distributed
    process group or None.

    prefetch: ask L2 for layer l + 1's experts on a side stream once layer l's kernels are queued, so they could arrive
    while layer l's partial sums cross NVLink. Off unless asked for: on one GPU running one rank's share of config 5
    (no NVLink wait to hide it in) it slowed a layer from 57 to 148 us, and it has not been measured on eight GPUs."""

    def __init__(self, ffn, layers, expert0: int, n_expert: int, group=None, peer: PeerCombine | None = None, prefetch=False):
        self.ffn = ffn
        self.layers = list(layers)
        self.expert0 = expert0
        self.n_expert = n_expert
        self.group = group
        self.peer = peer  # when set: the combine and the all-reduce are one kernel over peer memory
        self.prefetch = bool(prefetch) and hasattr(ffn, "prefetch_l2")
        self._side = None

    def _all_reduce(self, t):
        if self.group is None:
            return
        import torch.distributed as dist

        if dist.get_world_size(self.group) > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def _prefetch(self, l: int):
        """Layer l's experts into L2 on the side stream, after the work queued so far on the current stream."""
        import torch

        if self._side is None:
            self._side = torch.cuda.Stream()
        self._side.wait_stream(torch.cuda.current_stream())
        gu, dn = self.layers[l]
        self.ffn.prefetch_l2(gu, self._side)
        self.ffn.prefetch_l2(dn, self._side)

    def layer(self, l: int, x, ids, w, out):
        """out = the full weighted sum of layer l's routed experts for tokens x (every rank gets the same out)."""
        gu, dn = self.layers[l]
        if self.peer is not None:
            self.ffn.moe_ffn_ep(gu, dn, x, ids, w, self.expert0, self.n_expert, self.peer.handle, out=out)
            if self.prefetch and l + 1 < len(self.layers):
                self._prefetch(l + 1)
            return out
        self.ffn.moe_ffn(gu, dn, x, ids, w, expert0=self.expert0, n_expert_total=self.n_expert, out=out)
        if self.prefetch and l + 1 < len(self.layers):
            self._prefetch(l + 1)
        self._all_reduce(out)
        return out

    def step(self, xs, ids, w):
        """Runs every layer, layer l reading xs[l] and writing xs[l + 1]; ids [L, T, k], w [L, T, k]."""
        import torch

        for l in range(len(self.layers)):
            self.layer(l, xs[l], ids[l], w[l], xs[l + 1])
        if self._side is not None:
            torch.cuda.current_stream().wait_stream(self._side)  # the side stream joins back (graph capture needs it)
        return xs[len(self.layers)]
