"""Column-split (output-row-split) products for many activation rows: the partitioning of batched MUL_MAT nodes
(multi-stream decode, prefill; the products of src/common/qwen3-decoder.cpp:362-426 with M > 1) across the GPUs of
one node.

Rank r of G holds rows [r N/G, (r+1) N/G) of a weight W [N][K] (the whole K), computes y_r = x W_r^T for the
replicated activations x [M][K] with b200_mul_mat_rows semantics, and an all-gather assembles y [M][N] on every rank:
gathered [G][M][N/G] -> y[m][r N/G + j] = gathered[r][m][j]. The one exchange is the all-gather; the assembly is a
permuting copy. (The reference runs every product on one device; this is the multi-GPU extension of the same node.)
"""

from __future__ import annotations


def row_shard(n_rows: int, world: int, rank: int, align: int = 128) -> tuple[int, int]:
    """(first row, rows) of `rank`'s shard: equal shards, each a multiple of `align` rows (whole 128-row tensor-core
    tiles)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if n_rows % (world * align):
        raise ValueError(f"{n_rows} rows do not split into {world} shards of whole {align}-row tiles")
    n = n_rows // world
    return rank * n, n


class ColumnParallelProduct:
    """One rank's shard of a product. `mm(w, x, out)` computes out [M][rows] = x [M][K] times the shard's rows (a
    speech.cpp_b200 Context's mul_mat, or any stand-in with the same semantics); `group` a torch.distributed process
    group or None."""

    def __init__(self, mm, shard_weight, n_rows: int, group=None):
        self.mm = mm
        self.w = shard_weight
        self.n_rows = n_rows
        self.group = group

    def __call__(self, x, local_out, gathered, out):
        """x [M][K] -> out [M][n_rows] on every rank; local_out [M][n_rows / G] and gathered [G][M][n_rows / G] are
        the caller's buffers (kept across calls: a CUDA graph can hold them)."""
        import torch.distributed as dist

        if self.group is None or dist.get_world_size(self.group) == 1:
            self.mm(self.w, x, out)
            return out
        self.mm(self.w, x, local_out)

        G, M, n = gathered.shape
        dist.all_gather_into_tensor(gathered.view(G * M, n), local_out, group=self.group)
        out.view(M, G, n).copy_(gathered.permute(1, 0, 2))
        return out
