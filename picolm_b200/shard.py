"""KV-axis split of one long sequence over several GPUs (one process per GPU).

picolm decodes one sequence at a time (model.c:820-892): every new token
attends all cached positions [0, pos].  When the cache of a single sequence
is too long for one device's bandwidth, it is split along the sequence axis:

* rank r of `world` holds the contiguous positions [row0, row0 + n_rows) of
  the first `n_cached` positions, in its local cache rows [0, n_rows);
* the LAST rank also holds every position appended after n_cached (its
  local row pos - row0), so a decode step appends on exactly one rank;
* per layer and step every rank computes the partial triple (m, l, o) of
  its rows with pl_attn_decode_partial_dev (8,704 bytes for 32 heads of
  64) and
  the partials are merged in rank order on every rank, either after an
  NCCL all-gather with pl_attn_combine_dev (AttnShardOps) or by one kernel
  that pushes them over NVLink peer memory (P2PShardOps):
      M = max_g m_g,  L = sum_g l_g 2^(m_g - M),  O = sum_g 2^(m_g - M) o_g / L.

The arithmetic of the merge is the log-sum-exp form of the online softmax
of model.c:848-892 applied to whole shards instead of single rows.

A long sequence can instead be split by KV head (`head_shard`): every rank
holds all positions of its heads and runs the unchanged decode on them, and
the per-head outputs need no merge.

`KVSplitDecoder` holds the per-rank bookkeeping and is independent of the
backend: `ops` supplies `partial(...)` and `combine(...)`; `AttnShardOps`
and `P2PShardOps` are the CUDA implementations on top of the C ABI.
"""
from __future__ import annotations

from dataclasses import dataclass

# Floats per head in a partial block at head_dim 64: m, l, 2 pad, o[64].  A
# caller sizes `part` as n_heads * attn.part_stride floats (head_dim + 4 per
# head, so 132 at head_dim 128) and `parts_all` as world times that.
PART_STRIDE = 68


def head_shard(n_heads: int, n_kv_heads: int, world: int, rank: int) -> tuple[int, int, int, int]:
    """(head0, n_heads_r, kv_head0, n_kv_heads_r): the query and KV heads of
    `rank` when attention is split by KV head instead of by position.

    Each rank holds every position of n_kv_heads / world KV heads and runs
    their kv_mul query heads (model.c:848's kv_h = h / kv_mul keeps them
    together), so its output is a disjoint slice of heads and no merge is
    needed.  The slices of q, k, v and out are contiguous: head h occupies
    [h * head_dim, (h + 1) * head_dim) of its row."""
    if world < 1 or not 0 <= rank < world or n_kv_heads % world or n_heads % n_kv_heads:
        raise ValueError(f"cannot split {n_heads}/{n_kv_heads} heads over {world} ranks")
    hk = n_kv_heads // world
    hq = hk * (n_heads // n_kv_heads)
    return rank * hq, hq, rank * hk, hk


def shard_range(n_cached: int, world: int, rank: int) -> tuple[int, int]:
    """(row0, n_rows): the positions of [0, n_cached) that `rank` holds.

    Contiguous blocks of ceil(n_cached / world) positions in rank order; the
    last blocks may be shorter or empty when n_cached is small."""
    if world < 1 or not 0 <= rank < world or n_cached < 0:
        raise ValueError(f"bad shard request n_cached={n_cached} world={world} rank={rank}")
    per = -(-n_cached // world)
    row0 = min(rank * per, n_cached)
    return row0, min(n_cached, row0 + per) - row0


@dataclass
class KVSplitDecoder:
    """Rank-local state of a KV-split decode.

    rank, world: this process's place; n_cached: positions already in the
    cache before the first decode step; ops: backend with
      ops.partial(layer, pos, row0, n_rows, append, q, k, v, part)
      ops.gather(part, parts_all)     # rank-ordered all-gather
      ops.combine(world, parts_all, out)
    """
    rank: int
    world: int
    n_cached: int
    ops: object

    def __post_init__(self):
        self.row0, self.n_rows = shard_range(self.n_cached, self.world, self.rank)
        self.appends = self.rank == self.world - 1

    def local_capacity(self, n_new: int) -> int:
        """Local cache rows this rank needs for n_new decode steps."""
        per = -(-self.n_cached // self.world)
        return per + (n_new if self.appends else 0)

    def rows_at(self, pos: int) -> int:
        """Local rows attended when decoding global position `pos`."""
        if pos < self.n_cached:
            raise ValueError(f"decode position {pos} is inside the cached prefix")
        return pos - self.row0 + 1 if self.appends else self.n_rows

    def step(self, layer: int, pos: int, q, k, v, part, parts_all, out) -> None:
        """One layer of one decode step: partial, all-gather, combine."""
        self.ops.partial(layer, pos, self.row0, self.rows_at(pos), self.appends, q, k, v, part)
        self.ops.gather(part, parts_all)
        self.ops.combine(self.world, parts_all, out)


class AttnShardOps:
    """CUDA backend: the module's partial and combine kernels, NCCL gather.

    All tensors are torch CUDA tensors on this rank's device; every call is
    enqueued on `stream` (torch's current stream), which NCCL orders against."""

    def __init__(self, attn, stream_handle: int, group=None, seq: int = 0):
        self.attn = attn
        self.stream = stream_handle
        self.group = group
        self.seq = seq  # cache slot holding this rank's rows

    def partial(self, layer, pos, row0, n_rows, append, q, k, v, part):
        self.attn.decode_partial_dev(self.seq, layer, pos, row0, n_rows, append, q.data_ptr(),
                                     k.data_ptr(), v.data_ptr(), part.data_ptr(), self.stream)

    def gather(self, part, parts_all):
        import torch.distributed as dist
        dist.all_gather_into_tensor(parts_all, part, group=self.group)

    def combine(self, world, parts_all, out):
        self.attn.combine_dev(world, parts_all.data_ptr(), out.data_ptr(), self.stream)


class P2PShardOps(AttnShardOps):
    """CUDA backend whose merge pushes the partials over NVLink peer memory.

    At construction every rank allocates its receive buffer, the IPC handles
    are exchanged once over `group` (any backend; they are 64-byte objects),
    and each rank maps the others.  With `fused` (the default) one call per
    layer, pl_attn_decode_p2p_dev, computes this rank's partial, and each
    block of the grid that merges its segments stores its head into every
    rank's buffer, waits for that head from every rank and merges it.
    Without `fused`, pl_attn_decode_partial_dev writes the partial and
    pl_attn_combine_p2p_dev (one kernel) pushes, waits and merges.  Every
    value travels with the merge's epoch in the same 16-byte store, so no
    fence or flag is needed.  Either way `gather` has nothing left to do,
    and the merges are numbered on the device, so the calls can be captured
    in a CUDA graph and replayed."""

    def __init__(self, attn, stream_handle: int, rank: int, world: int, group=None,
                 seq: int = 0, fused: bool = True):
        super().__init__(attn, stream_handle, group, seq)
        import torch.distributed as dist
        handle = attn.xfer_setup(world, rank)
        handles = [None] * world
        dist.all_gather_object(handles, handle, group=group)
        attn.xfer_connect(handles)
        self.fused = fused
        self._part = None
        self._args = None

    def partial(self, layer, pos, row0, n_rows, append, q, k, v, part):
        self._part = part
        if self.fused:
            self._args = (layer, pos, row0, n_rows, append, q, k, v)
        else:
            super().partial(layer, pos, row0, n_rows, append, q, k, v, part)

    def gather(self, part, parts_all):
        pass

    def combine(self, world, parts_all, out):
        if self.fused:
            layer, pos, row0, n_rows, append, q, k, v = self._args
            self.attn.decode_p2p_dev(self.seq, layer, pos, row0, n_rows, append, q.data_ptr(),
                                     k.data_ptr(), v.data_ptr(), out.data_ptr(), self.stream)
        else:
            self.attn.combine_p2p_dev(self._part.data_ptr(), out.data_ptr(), self.stream)
