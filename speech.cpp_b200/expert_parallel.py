"""Expert parallelism for the routed-expert FFN stack (TextModel::experts, src/families/drama3/text-model.cpp:198-221).

The reference runs a Drama 3 layer's routed experts on one device (or splits whole layers GPU/CPU through
ggml_backend_sched, src/engines/drama3-engine.cpp:51-88). Here the experts of every layer are split across the GPUs of
one node: rank r holds experts [r E/N, (r+1) E/N). The router runs on every rank and the token activations are
replicated (they come out of the replicated attention / mixer part of the layer), so dispatch moves no bytes: each
rank's b200_moe_ffn skips the (token, slot) pairs routed to other ranks and leaves its experts' partial weighted sum,
and one all-reduce per layer adds the partial sums into the layer output every rank needs next.

With 256 tokens x top-8 of 128 experts, an all-to-all dispatch + combine would move each token-slot's activation row
(2176 B as q8_0) out and its 8 KB f32 output row back for 7/8 of the 2048 slots, about 16.8 MB per layer over the
node; the all-reduce of the [256, 2048] f32 output moves 2 MB per rank.
"""

from __future__ import annotations


def expert_shard(n_expert: int, world: int, rank: int) -> tuple[int, int]:
    """(first expert, number of experts) of `rank`'s shard; experts split evenly, contiguous, in rank order."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if n_expert % world:
        raise ValueError(f"{n_expert} experts do not split evenly over {world} ranks")
    n = n_expert // world
    return rank * n, n


class ExpertParallelMoe:
    """One rank's share of an MoE FFN stack: per layer (gate_up, down) expert weights of experts
    [expert0, expert0 + n_local) of n_expert. `ffn(ctx-like)` is any object with moe_ffn(gate_up, down, x, ids, w,
    expert0=, n_expert_total=, out=) (a speech.cpp_b200 Context); `group` a torch.distributed process group or None."""

    def __init__(self, ffn, layers, expert0: int, n_expert: int, group=None):
        self.ffn = ffn
        self.layers = list(layers)
        self.expert0 = expert0
        self.n_expert = n_expert
        self.group = group

    def _all_reduce(self, t):
        if self.group is None:
            return
        import torch.distributed as dist

        if dist.get_world_size(self.group) > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def layer(self, l: int, x, ids, w, out):
        """out = the full weighted sum of layer l's routed experts for tokens x (every rank gets the same out)."""
        gu, dn = self.layers[l]
        self.ffn.moe_ffn(gu, dn, x, ids, w, expert0=self.expert0, n_expert_total=self.n_expert, out=out)
        self._all_reduce(out)
        return out

    def step(self, xs, ids, w):
        """Runs every layer, layer l reading xs[l] and writing xs[l + 1]; ids [L, T, k], w [L, T, k]."""
        for l in range(len(self.layers)):
            self.layer(l, xs[l], ids[l], w[l], xs[l + 1])
        return xs[len(self.layers)]
